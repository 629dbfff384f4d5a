// Device-API composition test, written as the reference's validate_core
// (sample/validation/fft_validation.cu:83-123): a user kernel stages a tile
// with ThunderFFT_gmem2smem<bench_layout::L_in>, loads the fragment with
// smem2reg, runs ThunderFFT_kernel_reg, stores with reg2smem<L_out> and
// smem2gmem, while 64 sentinel elements after the (N + pad_h(N)) * BPB
// workspace must survive.  For every (T, N, direction) the program writes
// input and output as raw float32 pairs to <outdir>/devapi_<T>_<N>_<dir>.bin
// for the oracle comparison in tests/test_header_api.py.
#include <thunderfft/thunderfft.cuh>
#include <thunderfft/thunderfft_layout_tuned.h>

#include <cmath>
#include <cstdio>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace {
constexpr int kGuard = 64;
template <int N>
inline constexpr int kWorkspace = (N + pad_h(N)) * thunderfft::batch_per_block<N>;

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
__host__ __device__ vec2_t<T> enc(float2 v) {
  if constexpr (std::is_same_v<T, half>) return __floats2half2_rn(v.x, v.y);
  else return v;
}
template <class T>
float2 dec(vec2_t<T> v) {
  if constexpr (std::is_same_v<T, half>) return __half22float2(v);
  else return v;
}

template <class T, int N, bool Forward>
__global__ void validate_core(const vec2_t<T>* in, vec2_t<T>* out, int* guard_changes) {
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  constexpr int EPT = N * BPB / (32 * WPB);
  extern __shared__ __align__(16) unsigned char raw[];
  auto* ws = reinterpret_cast<vec2_t<T>*>(raw);
  vec2_t<T> reg[EPT], coef[36];
  const int tid = threadIdx.x + 32 * threadIdx.y;
  for (int j = tid; j < kGuard; j += 32 * WPB) ws[kWorkspace<N> + j] = enc<T>(make_float2(299.f, -299.f));
  __syncthreads();
  if constexpr (std::is_same_v<T, half>) thunderfft::unit_fp16::make_reg_b_precompute<N, Forward>(coef);
  using L_in = typename thunderfft::bench_layout<T, N, BPB>::L_in;
  using L_out = typename thunderfft::bench_layout<T, N, BPB>::L_out;
  thunderfft::ThunderFFT_gmem2smem<T, L_in>(ws, in + blockIdx.x * BPB * N);
  __syncthreads();
  thunderfft::ThunderFFT_smem2reg<T, L_in>(reg, ws);
  __syncthreads();
  thunderfft::ThunderFFT_kernel_reg<T, N, BPB, Forward>(reg, coef, ws);
  __syncthreads();
  thunderfft::ThunderFFT_reg2smem<T, L_out>(ws, reg);
  __syncthreads();
  thunderfft::ThunderFFT_smem2gmem<T, L_out>(out + blockIdx.x * BPB * N, ws);
  __syncthreads();
  if (tid == 0) {
    int changed = 0;
    for (int j = 0; j < kGuard; ++j) {
      float2 v;
      if constexpr (std::is_same_v<T, half>) v = __half22float2(ws[kWorkspace<N> + j]);
      else v = ws[kWorkspace<N> + j];
      changed += (v.x != 299.f || v.y != -299.f);
    }
    guard_changes[blockIdx.x] = changed;
  }
}

// Also exercises gmem2reg/reg2gmem (register fragment straight from global).
template <class T, int N, bool Forward>
__global__ void direct_core(const vec2_t<T>* in, vec2_t<T>* out) {
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  constexpr int EPT = N * BPB / (32 * WPB);
  extern __shared__ __align__(16) unsigned char raw[];
  vec2_t<T> reg[EPT];
  thunderfft::ThunderFFT_gmem2reg<T, N, BPB>(reg, in + blockIdx.x * BPB * N);
  thunderfft::ThunderFFT_kernel_reg<T, N, BPB, Forward>(reg, nullptr, raw);
  thunderfft::ThunderFFT_reg2gmem<T, N, BPB>(out + blockIdx.x * BPB * N, reg);
}

template <class T, int N, bool Forward>
int run(const std::string& outdir, int blocks) {
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  const int batch = blocks * BPB;
  const size_t total = size_t(batch) * N;
  std::vector<float2> x(total);
  std::mt19937 rng(17 + N);
  std::uniform_real_distribution<float> U(-1.f, 1.f);
  for (auto& v : x) v = make_float2(U(rng), U(rng));
  std::vector<vec2_t<T>> hin(total), hout(total), hout2(total);
  for (size_t i = 0; i < total; ++i) hin[i] = enc<T>(x[i]);
  vec2_t<T> *din, *dout, *dout2;
  int* dguard;
  ck(cudaMalloc(&din, total * sizeof(vec2_t<T>)), "malloc");
  ck(cudaMalloc(&dout, total * sizeof(vec2_t<T>)), "malloc");
  ck(cudaMalloc(&dout2, total * sizeof(vec2_t<T>)), "malloc");
  ck(cudaMalloc(&dguard, blocks * sizeof(int)), "malloc");
  ck(cudaMemcpy(din, hin.data(), total * sizeof(vec2_t<T>), cudaMemcpyHostToDevice), "h2d");
  const int smem = int(sizeof(vec2_t<T>)) * (kWorkspace<N> + kGuard);
  ck(cudaFuncSetAttribute(validate_core<T, N, Forward>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "attr");
  validate_core<T, N, Forward><<<blocks, dim3(32, WPB), smem>>>(din, dout, dguard);
  ck(cudaGetLastError(), "launch");
  const int smem2 = int(sizeof(vec2_t<T>)) * kWorkspace<N>;
  ck(cudaFuncSetAttribute(direct_core<T, N, Forward>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2), "attr");
  direct_core<T, N, Forward><<<blocks, dim3(32, WPB), smem2>>>(din, dout2);
  ck(cudaGetLastError(), "launch");
  ck(cudaDeviceSynchronize(), "sync");
  std::vector<int> guard(blocks);
  ck(cudaMemcpy(hout.data(), dout, total * sizeof(vec2_t<T>), cudaMemcpyDeviceToHost), "d2h");
  ck(cudaMemcpy(hout2.data(), dout2, total * sizeof(vec2_t<T>), cudaMemcpyDeviceToHost), "d2h");
  ck(cudaMemcpy(guard.data(), dguard, blocks * sizeof(int), cudaMemcpyDeviceToHost), "d2h");
  int guard_bad = 0;
  for (int g : guard) guard_bad += g;
  const std::string name = outdir + "/devapi_" + (std::is_same_v<T, half> ? "half" : "float") + "_" +
                           std::to_string(N) + "_" + (Forward ? "fwd" : "inv") + ".bin";
  FILE* f = std::fopen(name.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot write " + name);
  const int hdr[4] = {N, batch, guard_bad, 0};
  std::fwrite(hdr, sizeof(int), 4, f);
  for (size_t i = 0; i < total; ++i) { float2 v = dec<T>(hin[i]); std::fwrite(&v, 8, 1, f); }
  for (size_t i = 0; i < total; ++i) { float2 v = dec<T>(hout[i]); std::fwrite(&v, 8, 1, f); }
  for (size_t i = 0; i < total; ++i) { float2 v = dec<T>(hout2[i]); std::fwrite(&v, 8, 1, f); }
  std::fclose(f);
  cudaFree(din); cudaFree(dout); cudaFree(dout2); cudaFree(dguard);
  return guard_bad;
}

template <class T>
int run_type(const std::string& outdir) {
  thunderfft::ThunderFFTInitialize<T>(64);  // FP16 unit table for make_reg_b_precompute
  int bad = 0;
  bad += run<T, 64, true>(outdir, 3) + run<T, 64, false>(outdir, 3);
  bad += run<T, 128, true>(outdir, 3) + run<T, 128, false>(outdir, 3);
  bad += run<T, 256, true>(outdir, 3) + run<T, 256, false>(outdir, 3);
  bad += run<T, 512, true>(outdir, 3) + run<T, 512, false>(outdir, 3);
  bad += run<T, 1024, true>(outdir, 3) + run<T, 1024, false>(outdir, 3);
  bad += run<T, 2048, true>(outdir, 3) + run<T, 2048, false>(outdir, 3);
  bad += run<T, 4096, true>(outdir, 3) + run<T, 4096, false>(outdir, 3);
  thunderfft::ThunderFFTFinalize<T>();
  return bad;
}
}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) { std::fprintf(stderr, "usage: %s OUTDIR\n", argv[0]); return 2; }
  try {
    const int bad = run_type<float>(argv[1]) + run_type<half>(argv[1]);
    std::printf("device api: 28 configurations written, guard changes %d\n", bad);
    return bad == 0 ? 0 : 1;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "device api error: %s\n", e.what());
    return 2;
  }
}
