// thff_paper_fft — the device-API timing CLI.  Its command line, CSV columns
// and two stderr header lines follow the reference's paper benchmark
// (sample/bench/paper_fft.cu:159-185, Table 3 "differential compute time"),
// so that the two programs' outputs line up row for row:
//
//   thff_paper_fft N fp16|tf32 register|shared [repeats=1000] [trials=3] [batch=65536]
//
// What runs: one block per batch_per_block<N> signals calls the composable
// device API (ThunderFFT_kernel_reg on a 32-element-per-thread fragment)
// `repeats` times inside one kernel.  "register" keeps the fragment in
// registers between calls; "shared" moves it through the block's shared tile
// every call (smem2reg / kernel_reg / reg2smem).
//   compute_us          = (t(2R) - t(R)) / R, which cancels launch and
//                         global-memory time;
//   e2e_out_of_place_us = one load -> FFT -> store launch.
// Every time is the median of kRuns event-timed launches on a private stream
// after one untimed launch of the same shape.
// Accuracy gate (before any timing): 64 signals of the benchmark's LCG input,
// rounded to T, through one forward FFT; relative L2 against an FP64 radix-2
// FFT computed on the host from the same rounded values must be <= 5e-3.
#include <thunderfft/thunderfft.cuh>
#include <thunderfft/thunderfft_layout_tuned.h>
#include <cufft.h>

#include <algorithm>
#include <cmath>
#include <complex>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

namespace {

constexpr int kRuns = 5;               // event-timed launches per figure (median)
constexpr int kGateSignals = 64;
constexpr double kGateLimit = 5e-3;

struct CudaCall {
  const char* what;
  void operator<<(cudaError_t e) const {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
};

struct Options {
  int n = 0;
  bool half = false;
  bool shared = false;
  int repeats = 1000;
  int trials = 3;
  int batch = 65536;
};

int to_int(const char* s, const char* name) {
  char* end = nullptr;
  const long v = std::strtol(s, &end, 10);
  if (!end || *end || v <= 0 || v > (1L << 30)) throw std::runtime_error(std::string("invalid ") + name + ": " + s);
  return int(v);
}

// ---------------------------------------------------------------- inputs
// The accuracy input: linear-congruential values in [-1, 1) / sqrt(N) per
// element index (re from z, im from the next step); the timed input: a real
// sinusoid over each signal, / sqrt(N).  Both as the reference benchmark's.
__device__ float lcg_unit(unsigned z) { return (float(int(z & 65535u)) - 32768.0f) / 32768.0f; }

template <class T>
__global__ void fill_accuracy(vec2_t<T>* x, size_t count, int n) {
  const float s = 1.0f / sqrtf(float(n));
  const size_t step = size_t(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < count; i += step) {
    const unsigned z0 = unsigned(i) * 1664525u + 1013904223u;
    const unsigned z1 = z0 * 1664525u + 1013904223u;
    const float re = lcg_unit(z0) * s, im = lcg_unit(z1) * s;
    if constexpr (std::is_same_v<T, half>) x[i] = __floats2half2_rn(re, im);
    else x[i] = make_float2(re, im);
  }
}

template <class T>
__global__ void fill_timing(vec2_t<T>* x, size_t count, int n) {
  const float s = 1.0f / sqrtf(float(n));
  const size_t step = size_t(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < count; i += step) {
    const float re = sinf(float(6.283185307179586 * double(i % n) / n)) * s;
    if constexpr (std::is_same_v<T, half>) x[i] = __floats2half2_rn(re, 0.0f);
    else x[i] = make_float2(re, 0.0f);
  }
}

template <class T>
std::complex<double> widen(const vec2_t<T>& v) {
  if constexpr (std::is_same_v<T, half>) return {double(__half2float(v.x)), double(__half2float(v.y))};
  else return {double(v.x), double(v.y)};
}

// In-place FP64 radix-2 forward FFT (decimation in time, bit-reversed input
// order), the accuracy reference.
void fft_fp64(std::complex<double>* a, int n) {
  for (int i = 1, j = 0; i < n; ++i) {
    int bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) std::swap(a[i], a[j]);
  }
  for (int len = 2; len <= n; len <<= 1) {
    const double ang = -2.0 * M_PI / len;
    for (int k = 0; k < len / 2; ++k) {
      const std::complex<double> w(std::cos(ang * k), std::sin(ang * k));
      for (int i = k; i < n; i += len) {
        const std::complex<double> u = a[i], v = a[i + len / 2] * w;
        a[i] = u + v;
        a[i + len / 2] = u - v;
      }
    }
  }
}

// ---------------------------------------------------------------- kernel
template <class T, int N, bool kShared, bool kOnce>
__global__ void bench(const vec2_t<T>* in, vec2_t<T>* out, unsigned repeats) {
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  constexpr int EPT = N * BPB / (32 * WPB);
  using L_in = typename thunderfft::bench_layout<T, N, BPB>::L_in;
  using L_out = typename thunderfft::bench_layout<T, N, BPB>::L_out;
  extern __shared__ __align__(16) unsigned char raw[];
  auto* ws = reinterpret_cast<vec2_t<T>*>(raw);
  vec2_t<T> reg[EPT], coef[36];
  if constexpr (std::is_same_v<T, half>) thunderfft::unit_fp16::make_reg_b_precompute<N, true>(coef);
  thunderfft::ThunderFFT_gmem2smem<T, L_in>(ws, in + blockIdx.x * BPB * N);
  __syncthreads();
  const unsigned r = kOnce ? 1u : repeats;
  if constexpr (kShared) {
#pragma unroll 1
    for (unsigned i = 0; i < r; ++i) {
      thunderfft::ThunderFFT_smem2reg<T, L_in>(reg, ws);
      __syncthreads();
      thunderfft::ThunderFFT_kernel_reg<T, N, BPB, true>(reg, coef, ws);
      __syncthreads();
      thunderfft::ThunderFFT_reg2smem<T, L_out>(ws, reg);
      __syncthreads();
    }
  } else {
    thunderfft::ThunderFFT_smem2reg<T, L_in>(reg, ws);
    __syncthreads();
#pragma unroll 1
    for (unsigned i = 0; i < r; ++i) {
      thunderfft::ThunderFFT_kernel_reg<T, N, BPB, true>(reg, coef, ws);
      __syncthreads();
    }
    thunderfft::ThunderFFT_reg2smem<T, L_out>(ws, reg);
    __syncthreads();
  }
  thunderfft::ThunderFFT_smem2gmem<T, L_out>(out + blockIdx.x * BPB * N, ws);
}

// ---------------------------------------------------------------- runner
// Owns the device buffers, the stream and the events of one (T, N,
// placement) measurement; everything is released by the destructor.
template <class T, int N, bool kShared>
class Runner {
 public:
  using V = vec2_t<T>;
  static constexpr int BPB = thunderfft::batch_per_block<N>;
  static constexpr int WPB = thunderfft::warp_per_block<N>;
  static constexpr size_t kSmem = sizeof(V) * size_t(N + pad_h(N)) * BPB;

  explicit Runner(const Options& o) : opt_(o) {
    if (o.batch % BPB) throw std::runtime_error("batch must be a positive multiple of batch_per_block");
    CudaCall{"cudaStreamCreate"} << cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
    CudaCall{"cudaEventCreate"} << cudaEventCreate(&start_);
    CudaCall{"cudaEventCreate"} << cudaEventCreate(&stop_);
    CudaCall{"cudaFuncSetAttribute"} << cudaFuncSetAttribute(bench<T, N, kShared, false>,
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
    CudaCall{"cudaFuncSetAttribute"} << cudaFuncSetAttribute(bench<T, N, kShared, true>,
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
    thunderfft::ThunderFFTInitialize<T>(N);
    initialized_ = true;
    const size_t elems = size_t(N) * std::max(o.batch, kGateSignals);
    CudaCall{"cudaMalloc(input)"} << cudaMalloc(&in_, elems * sizeof(V));
    CudaCall{"cudaMalloc(output)"} << cudaMalloc(&out_, elems * sizeof(V));
  }
  ~Runner() {
    if (in_) cudaFree(in_);
    if (out_) cudaFree(out_);
    if (start_) cudaEventDestroy(start_);
    if (stop_) cudaEventDestroy(stop_);
    if (stream_) cudaStreamDestroy(stream_);
    if (initialized_) {
      try { thunderfft::ThunderFFTFinalize<T>(); } catch (...) {}
    }
  }
  Runner(const Runner&) = delete;
  Runner& operator=(const Runner&) = delete;

  // Relative L2 of one forward FFT of the accuracy input against FP64.
  double accuracy() {
    const size_t count = size_t(N) * kGateSignals;
    fill_accuracy<T><<<64, 256, 0, stream_>>>(in_, count, N);
    CudaCall{"fill"} << cudaGetLastError();
    launch(kGateSignals, 1, true);
    std::vector<V> x(count), y(count);
    CudaCall{"copy input"} << cudaMemcpyAsync(x.data(), in_, count * sizeof(V), cudaMemcpyDeviceToHost, stream_);
    CudaCall{"copy output"} << cudaMemcpyAsync(y.data(), out_, count * sizeof(V), cudaMemcpyDeviceToHost, stream_);
    CudaCall{"synchronize"} << cudaStreamSynchronize(stream_);
    std::vector<std::complex<double>> want(N);
    double err = 0, ref = 0;
    for (int s = 0; s < kGateSignals; ++s) {
      for (int i = 0; i < N; ++i) want[i] = widen<T>(x[size_t(s) * N + i]);
      fft_fp64(want.data(), N);
      for (int i = 0; i < N; ++i) {
        const std::complex<double> got = widen<T>(y[size_t(s) * N + i]);
        if (!std::isfinite(got.real()) || !std::isfinite(got.imag())) return NAN;
        err += std::norm(got - want[i]);
        ref += std::norm(want[i]);
      }
    }
    return std::sqrt(err / ref);
  }

  // Median event time (us) of one launch of `repeats` calls over the batch.
  double time_us(unsigned repeats, bool once) {
    launch(opt_.batch, repeats, once);   // untimed: same shape, warm caches
    std::vector<double> t;
    for (int i = 0; i < kRuns; ++i) {
      CudaCall{"cudaEventRecord"} << cudaEventRecord(start_, stream_);
      launch(opt_.batch, repeats, once);
      CudaCall{"cudaEventRecord"} << cudaEventRecord(stop_, stream_);
      CudaCall{"cudaEventSynchronize"} << cudaEventSynchronize(stop_);
      float ms = 0.f;
      CudaCall{"cudaEventElapsedTime"} << cudaEventElapsedTime(&ms, start_, stop_);
      t.push_back(double(ms) * 1e3);
    }
    std::nth_element(t.begin(), t.begin() + kRuns / 2, t.end());
    return t[kRuns / 2];
  }

  void prepare_timing_input() {
    fill_timing<T><<<1024, 256, 0, stream_>>>(in_, size_t(N) * opt_.batch, N);
    CudaCall{"fill"} << cudaGetLastError();
    for (int w = 0; w < 3; ++w) launch(opt_.batch, unsigned(opt_.repeats), false);
    CudaCall{"warm-up"} << cudaStreamSynchronize(stream_);
  }

 private:
  void launch(int count, unsigned repeats, bool once) {
    const dim3 grid(count / BPB), block(32, WPB);
    if (once) bench<T, N, kShared, true><<<grid, block, kSmem, stream_>>>(in_, out_, repeats);
    else bench<T, N, kShared, false><<<grid, block, kSmem, stream_>>>(in_, out_, repeats);
    CudaCall{"bench launch"} << cudaGetLastError();
  }

  Options opt_;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t start_ = nullptr, stop_ = nullptr;
  V* in_ = nullptr;
  V* out_ = nullptr;
  bool initialized_ = false;
};

template <class T, int N, bool kShared>
void measure(const Options& o) {
  Runner<T, N, kShared> run(o);
  const double rel = run.accuracy();
  if (!(rel <= kGateLimit)) throw std::runtime_error("accuracy gate failed: relative L2 " + std::to_string(rel));
  run.prepare_timing_input();
  const unsigned r = unsigned(o.repeats);
  for (int trial = 0; trial < o.trials; ++trial) {
    const double t_r = run.time_us(r, false);
    const double t_2r = run.time_us(2 * r, false);
    if (!(std::isfinite(t_r) && std::isfinite(t_2r) && t_2r > t_r))
      throw std::runtime_error("differential timing is not positive");
    const double e2e = run.time_us(1, true);
    std::printf("%d,%s,%s,%d,%d,%d,%.9g,%.9g,%.9g,%.9g,%.12g,%zu\n", N, o.half ? "fp16" : "tf32",
                o.shared ? "shared" : "register", o.batch, o.repeats, trial, t_r, t_2r, (t_2r - t_r) / r, e2e, rel,
                Runner<T, N, kShared>::kSmem);
    std::fflush(stdout);
  }
}

// Every (N, type, placement) the CLI accepts, as one table.
struct Entry {
  int n;
  bool half, shared;
  void (*fn)(const Options&);
};
template <int N>
constexpr Entry entries_for(int which) {
  return which == 0   ? Entry{N, false, false, &measure<float, N, false>}
         : which == 1 ? Entry{N, false, true, &measure<float, N, true>}
         : which == 2 ? Entry{N, true, false, &measure<half, N, false>}
                      : Entry{N, true, true, &measure<half, N, true>};
}
template <int... Ns>
struct Table {
  static constexpr int kCount = 4 * int(sizeof...(Ns));
  Entry e[kCount];
  constexpr Table() : e{} {
    int i = 0;
    ((e[i++] = entries_for<Ns>(0), e[i++] = entries_for<Ns>(1), e[i++] = entries_for<Ns>(2),
      e[i++] = entries_for<Ns>(3)), ...);
  }
};
constexpr Table<64, 128, 256, 512, 1024, 2048, 4096> kTable;

Options parse(int argc, char** argv) {
  Options o;
  o.n = to_int(argv[1], "N");
  const std::string prec = argv[2], place = argv[3];
  if (prec != "fp16" && prec != "tf32") throw std::runtime_error("precision must be fp16 or tf32");
  if (place != "register" && place != "shared") throw std::runtime_error("placement must be register or shared");
  o.half = prec == "fp16";
  o.shared = place == "shared";
  if (argc > 4) o.repeats = to_int(argv[4], "repeats");
  if (argc > 5) o.trials = to_int(argv[5], "trials");
  if (argc > 6) o.batch = to_int(argv[6], "batch");
  return o;
}

void print_headers(const Options& o) {
  cudaDeviceProp prop;
  CudaCall{"cudaGetDeviceProperties"} << cudaGetDeviceProperties(&prop, 0);
  int driver = 0, runtime = 0, cufft = 0;
  CudaCall{"cudaDriverGetVersion"} << cudaDriverGetVersion(&driver);
  CudaCall{"cudaRuntimeGetVersion"} << cudaRuntimeGetVersion(&runtime);
  if (cufftGetVersion(&cufft) != CUFFT_SUCCESS) cufft = 0;
  std::fprintf(stderr, "compiled_CUDART=%d runtime=%d driver=%d cuFFT=%d extra_R_warmups=3\n", CUDART_VERSION, runtime,
               driver, cufft);
  std::fprintf(stderr, "GPU=%s compute=%d.%d batch=%d R=%d trials=%d single_fft_relL2_limit=0.005\n", prop.name,
               prop.major, prop.minor, o.batch, o.repeats, o.trials);
  std::puts("N,precision,placement,batch,inside_repeats,trial,t_R_us,t_2R_us,compute_us,e2e_out_of_place_us,"
            "single_fft_relL2,shared_bytes");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 4 || argc > 7) {
    std::fprintf(stderr, "usage: %s N fp16|tf32 register|shared [repeats=1000] [trials=3] [batch=65536]\n", argv[0]);
    return 2;
  }
  try {
    const Options o = parse(argc, argv);
    const Entry* hit = nullptr;
    for (const Entry& e : kTable.e)
      if (e.n == o.n && e.half == o.half && e.shared == o.shared) hit = &e;
    if (!hit) throw std::runtime_error("unsupported N: " + std::to_string(o.n));
    print_headers(o);
    hit->fn(o);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ERROR: %s\n", e.what());
    return 1;
  }
}
