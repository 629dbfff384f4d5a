// thff_paper_fft — the device-API timing CLI, CSV-compatible with the
// reference's paper benchmark (sample/bench/paper_fft.cu:159-185, Table 3:
// "differential compute time").
//
//   thff_paper_fft N fp16|tf32 register|shared [repeats=1000] [trials=3] [batch=65536]
//
// One block per batch_per_block<N> signals runs the composable device API
// (ThunderFFT_kernel_reg on a 32-element-per-thread fragment) `repeats`
// times in a loop inside one kernel; "register" keeps the fragment in
// registers between calls, "shared" reloads it from the block's shared tile
// each call (smem2reg / kernel_reg / reg2smem).  compute_us =
// (t_2R - t_R) / R cancels launch and global-memory time.  e2e_out_of_place_us
// is one load -> FFT -> store launch.  Before timing, a 64-signal forward FFT
// is checked against cuFFT Z2Z in FP64 on the same (rounded) input, gate
// relative L2 <= 5e-3.  CSV columns and stderr header lines follow the
// reference's.
#include <thunderfft/thunderfft.cuh>
#include <thunderfft/thunderfft_layout_tuned.h>
#include <cufft.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void ckf(cufftResult e, const char* what) {
  if (e != CUFFT_SUCCESS) throw std::runtime_error(std::string(what) + ": cuFFT " + std::to_string(int(e)));
}

template <class T>
__device__ vec2_t<T> enc(float x, float y) {
  if constexpr (std::is_same_v<T, half>) return __floats2half2_rn(x, y);
  else return make_float2(x, y);
}
template <class T>
__device__ double2 widen(vec2_t<T> v) {
  if constexpr (std::is_same_v<T, half>) return make_double2(__half2float(v.x), __half2float(v.y));
  else return make_double2(v.x, v.y);
}

// Timed inputs: a real sinusoid over each signal / sqrt(N); the accuracy
// input: linear-congruential values in [-1, 1) / sqrt(N) (both as in the
// reference benchmark), with the FP64 copy taken after rounding to T.
template <class T>
__global__ void fill(vec2_t<T>* x, double2* ref, size_t count, int n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const float s = 1.0f / sqrtf((float)n);
    float re, im;
    if (ref) {
      unsigned z = (unsigned)i * 1664525u + 1013904223u;
      re = (float((int)(z & 65535u)) - 32768.0f) / 32768.0f * s;
      z = z * 1664525u + 1013904223u;
      im = (float((int)(z & 65535u)) - 32768.0f) / 32768.0f * s;
    } else {
      re = sinf(float(6.283185307179586 * double(i % n) / n)) * s;
      im = 0.0f;
    }
    x[i] = enc<T>(re, im);
    if (ref) ref[i] = widen<T>(x[i]);
  }
}

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

template <class F>
double elapsed_us(F&& launch, int runs) {
  cudaEvent_t a, b;
  ck(cudaEventCreate(&a), "event");
  ck(cudaEventCreate(&b), "event");
  ck(cudaEventRecord(a), "record");
  for (int i = 0; i < runs; ++i) launch();
  ck(cudaEventRecord(b), "record");
  ck(cudaEventSynchronize(b), "sync");
  float ms = 0.f;
  ck(cudaEventElapsedTime(&ms, a, b), "elapsed");
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return double(ms) * 1000.0 / runs;
}

template <class T, int N, bool kShared>
void run(int batch, int repeats, int trials) {
  using V = vec2_t<T>;
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  constexpr size_t smem = sizeof(V) * size_t(N + pad_h(N)) * BPB;
  if (batch <= 0 || batch % BPB) throw std::runtime_error("batch must be a positive multiple of batch_per_block");
  ck(cudaFuncSetAttribute(bench<T, N, kShared, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "attr");
  ck(cudaFuncSetAttribute(bench<T, N, kShared, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "attr");
  thunderfft::ThunderFFTInitialize<T>(N);
  auto launch = [&](const V* in, V* out, int count, unsigned r, bool once) {
    const dim3 grid(count / BPB), block(32, WPB);
    if (once) bench<T, N, kShared, true><<<grid, block, smem>>>(in, out, r);
    else bench<T, N, kShared, false><<<grid, block, smem>>>(in, out, r);
    ck(cudaGetLastError(), "launch");
  };
  // accuracy gate
  constexpr int vb = 64;
  const size_t vc = size_t(N) * vb;
  V *vi = nullptr, *vo = nullptr;
  double2* vr = nullptr;
  ck(cudaMalloc(&vi, vc * sizeof(V)), "malloc");
  ck(cudaMalloc(&vo, vc * sizeof(V)), "malloc");
  ck(cudaMalloc(&vr, vc * sizeof(double2)), "malloc");
  fill<T><<<128, 256>>>(vi, vr, vc, N);
  ck(cudaGetLastError(), "fill");
  cufftHandle plan;
  ckf(cufftPlan1d(&plan, N, CUFFT_Z2Z, vb), "plan");
  ckf(cufftExecZ2Z(plan, reinterpret_cast<cufftDoubleComplex*>(vr), reinterpret_cast<cufftDoubleComplex*>(vr),
                   CUFFT_FORWARD), "exec");
  launch(vi, vo, vb, 1, true);
  ck(cudaDeviceSynchronize(), "sync");
  std::vector<V> got(vc);
  std::vector<double2> want(vc);
  ck(cudaMemcpy(got.data(), vo, vc * sizeof(V), cudaMemcpyDeviceToHost), "copy");
  ck(cudaMemcpy(want.data(), vr, vc * sizeof(double2), cudaMemcpyDeviceToHost), "copy");
  double se = 0, sr = 0;
  bool finite = true;
  for (size_t i = 0; i < vc; ++i) {
    double x, y;
    if constexpr (std::is_same_v<T, half>) { x = __half2float(got[i].x); y = __half2float(got[i].y); }
    else { x = got[i].x; y = got[i].y; }
    finite = finite && std::isfinite(x) && std::isfinite(y);
    se += (x - want[i].x) * (x - want[i].x) + (y - want[i].y) * (y - want[i].y);
    sr += want[i].x * want[i].x + want[i].y * want[i].y;
  }
  const double rel = std::sqrt(se / sr);
  cufftDestroy(plan);
  cudaFree(vi); cudaFree(vo); cudaFree(vr);
  if (!finite || !(rel <= 5e-3)) throw std::runtime_error("single-FFT correctness gate failed relL2=" + std::to_string(rel));
  // timing
  V *in = nullptr, *out = nullptr;
  const size_t bytes = size_t(N) * batch * sizeof(V);
  ck(cudaMalloc(&in, bytes), "malloc");
  ck(cudaMalloc(&out, bytes), "malloc");
  fill<T><<<1024, 256>>>(in, nullptr, size_t(N) * batch, N);
  ck(cudaDeviceSynchronize(), "fill");
  for (int w = 0; w < 3; ++w) { launch(in, out, batch, unsigned(repeats), false); ck(cudaDeviceSynchronize(), "warmup"); }
  for (int t = 0; t < trials; ++t) {
    launch(in, out, batch, unsigned(repeats), false);
    ck(cudaDeviceSynchronize(), "sync");
    const double t_r = elapsed_us([&] { launch(in, out, batch, unsigned(repeats), false); }, 1);
    launch(in, out, batch, unsigned(2 * repeats), false);
    ck(cudaDeviceSynchronize(), "sync");
    const double t_2r = elapsed_us([&] { launch(in, out, batch, unsigned(2 * repeats), false); }, 1);
    if (!(std::isfinite(t_r) && std::isfinite(t_2r) && t_2r > t_r))
      throw std::runtime_error("nonpositive/nonfinite differential timing");
    launch(in, out, batch, 1, true);
    ck(cudaDeviceSynchronize(), "sync");
    const double e2e = elapsed_us([&] { launch(in, out, batch, 1, true); }, 10);
    std::printf("%d,%s,%s,%d,%d,%d,%.9g,%.9g,%.9g,%.9g,%.12g,%zu\n", N, std::is_same_v<T, half> ? "fp16" : "tf32",
                kShared ? "shared" : "register", batch, repeats, t, t_r, t_2r, (t_2r - t_r) / repeats, e2e, rel, smem);
    std::fflush(stdout);
  }
  cudaFree(in);
  cudaFree(out);
  thunderfft::ThunderFFTFinalize<T>();
}

template <int N>
void choose(const std::string& prec, const std::string& place, int b, int r, int t) {
  if (prec == "fp16") {
    if (place == "shared") run<half, N, true>(b, r, t); else run<half, N, false>(b, r, t);
  } else {
    if (place == "shared") run<float, N, true>(b, r, t); else run<float, N, false>(b, r, t);
  }
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc < 4 || argc > 7) {
      std::fprintf(stderr, "usage: %s N fp16|tf32 register|shared [repeats=1000] [trials=3] [batch=65536]\n", argv[0]);
      return 2;
    }
    const int n = std::stoi(argv[1]);
    const int r = argc > 4 ? std::stoi(argv[4]) : 1000, t = argc > 5 ? std::stoi(argv[5]) : 3;
    const int b = argc > 6 ? std::stoi(argv[6]) : 65536;
    const std::string prec = argv[2], place = argv[3];
    if ((prec != "fp16" && prec != "tf32") || (place != "register" && place != "shared") || r <= 0 || t <= 0)
      throw std::runtime_error("invalid arguments");
    cudaDeviceProp prop;
    ck(cudaGetDeviceProperties(&prop, 0), "properties");
    int drv = 0, rt = 0, cufft_v = 0;
    cudaDriverGetVersion(&drv);
    cudaRuntimeGetVersion(&rt);
    cufftGetVersion(&cufft_v);
    std::fprintf(stderr, "compiled_CUDART=%d runtime=%d driver=%d cuFFT=%d extra_R_warmups=3\n", CUDART_VERSION, rt,
                 drv, cufft_v);
    std::fprintf(stderr, "GPU=%s compute=%d.%d batch=%d R=%d trials=%d single_fft_relL2_limit=0.005\n", prop.name,
                 prop.major, prop.minor, b, r, t);
    std::puts("N,precision,placement,batch,inside_repeats,trial,t_R_us,t_2R_us,compute_us,e2e_out_of_place_us,"
              "single_fft_relL2,shared_bytes");
    switch (n) {
      case 64: choose<64>(prec, place, b, r, t); break;
      case 128: choose<128>(prec, place, b, r, t); break;
      case 256: choose<256>(prec, place, b, r, t); break;
      case 512: choose<512>(prec, place, b, r, t); break;
      case 1024: choose<1024>(prec, place, b, r, t); break;
      case 2048: choose<2048>(prec, place, b, r, t); break;
      case 4096: choose<4096>(prec, place, b, r, t); break;
      default: throw std::runtime_error("unsupported N");
    }
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ERROR: %s\n", e.what());
    return 1;
  }
}
