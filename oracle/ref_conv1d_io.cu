// ref_conv1d_io.cu — TEST INFRASTRUCTURE ONLY: runs the REFERENCE's fused
// FFT convolution kernel, thunder_convN_block_kernel_realin_realout
// (sample/conv1d/conv1d_fullfft_l4096_thunder.cu:280-331), on inputs given
// in a file, so that this library's conv1d can be compared with it on
// identical signals and taps.
//
// oracle/build_ref.py compiles this file with THFF_REF_CONV1D_SOURCE set to
// the path of that sample (read where it lies, never copied) and the
// reference's include/ directory on the include path; the sample's main is
// renamed and not called.  The filter spectrum is prepared the way the
// sample prepares it for one channel (D = 1, :449-472): N = 4096 through
// cuFFT, f32_to_h2 and permute_filter_layout4096; N = 1024 through the
// sample's own FFT kernel and permute_filter_layout1024.
//
//   ref_conv1d_io <N> <taps> <batch> <in.bin> <out.bin>
//     in.bin : float32 x[batch][N] (each value converted to half, as the
//              sample stores its signals), then float32 h[taps]
//     out.bin: float32 y[batch][N], the kernel's half outputs widened; the
//              sample's own check (:499-545) reads them as N times the
//              circular convolution of x with h.
// Output: oracle/_ref/ref_conv1d_io, run only by tests.
#define main thff_ref_conv1d_sample_main
#include THFF_REF_CONV1D_SOURCE
#undef main

#include <cstdio>

namespace {

bool read_floats(std::FILE* f, std::vector<float>& v) { return std::fread(v.data(), sizeof(float), v.size(), f) == v.size(); }

template <int N>
int run_io(int taps, int batch, const char* in_path, const char* out_path) {
  constexpr int BPB = thunderfft::batch_per_block<N>;
  constexpr int WPB = thunderfft::warp_per_block<N>;
  static_assert(BPB == 1, "one signal per block at N = 1024 and 4096");
  const int D = 1;
  const size_t elems = size_t(batch) * N;

  std::vector<float> x(elems), h(taps);
  std::FILE* fin = std::fopen(in_path, "rb");
  if (!fin) return std::fprintf(stderr, "cannot open %s\n", in_path), 2;
  const bool ok = read_floats(fin, x) && read_floats(fin, h);
  std::fclose(fin);
  if (!ok) return std::fprintf(stderr, "short input file %s\n", in_path), 2;

  std::vector<half> x_half(elems);
  for (size_t i = 0; i < elems; ++i) x_half[i] = __float2half(x[i]);
  std::vector<float2> taps_c(N, make_float2(0.f, 0.f));
  for (int k = 0; k < taps; ++k) taps_c[k].x = h[k];

  half *d_x = nullptr, *d_y = nullptr;
  cpx_h *d_H = nullptr, *d_H_perm = nullptr, *d_taps_h = nullptr;
  float2 *d_taps = nullptr, *d_taps_f = nullptr;
  CHECK_CUDA(cudaMalloc(&d_x, sizeof(half) * elems));
  CHECK_CUDA(cudaMalloc(&d_y, sizeof(half) * elems));
  CHECK_CUDA(cudaMalloc(&d_H, sizeof(cpx_h) * N));
  CHECK_CUDA(cudaMalloc(&d_H_perm, sizeof(cpx_h) * N));
  CHECK_CUDA(cudaMemcpy(d_x, x_half.data(), sizeof(half) * elems, cudaMemcpyHostToDevice));

  thunderfft::ThunderFFTInitialize<half>(N);
  const dim3 block(thunderfft::threads_per_warp, WPB);
  const size_t smem = sizeof(cpx_h) * (N + pad_h(N)) * BPB;
  CHECK_CUDA(cudaFuncSetAttribute(thunder_convN_block_kernel_realin_realout<N>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));

  cufftHandle plan = 0;
  if constexpr (N == 4096) {
    CHECK_CUDA(cudaMalloc(&d_taps, sizeof(float2) * N));
    CHECK_CUDA(cudaMalloc(&d_taps_f, sizeof(float2) * N));
    CHECK_CUDA(cudaMemcpy(d_taps, taps_c.data(), sizeof(float2) * N, cudaMemcpyHostToDevice));
    CHECK_CUFFT(cufftPlan1d(&plan, N, CUFFT_C2C, D));
    CHECK_CUFFT(cufftExecC2C(plan, reinterpret_cast<cufftComplex*>(d_taps), reinterpret_cast<cufftComplex*>(d_taps_f),
                             CUFFT_FORWARD));
    f32_to_h2<<<(N + 255) / 256, 256>>>(d_taps_f, d_H, N);
    CHECK_CUDA(cudaGetLastError());
    permute_filter_layout4096<N><<<D, block>>>(d_H, d_H_perm, D);
  } else {
    std::vector<cpx_h> taps_h(N);
    for (int n = 0; n < N; ++n) taps_h[n] = __floats2half2_rn(taps_c[n].x, taps_c[n].y);
    CHECK_CUDA(cudaMalloc(&d_taps_h, sizeof(cpx_h) * N));
    CHECK_CUDA(cudaMemcpy(d_taps_h, taps_h.data(), sizeof(cpx_h) * N, cudaMemcpyHostToDevice));
    thunder_fftN_block_kernel<N, true><<<1, block, smem>>>(d_taps_h, d_H);
    CHECK_CUDA(cudaGetLastError());
    permute_filter_layout1024<N><<<D, block>>>(d_H, d_H_perm, D);
  }
  CHECK_CUDA(cudaGetLastError());
  thunder_convN_block_kernel_realin_realout<N><<<batch / BPB, block, smem>>>(d_x, d_H, d_H_perm, d_y, D);
  CHECK_CUDA(cudaGetLastError());
  CHECK_CUDA(cudaDeviceSynchronize());

  std::vector<half> y_half(elems);
  CHECK_CUDA(cudaMemcpy(y_half.data(), d_y, sizeof(half) * elems, cudaMemcpyDeviceToHost));
  std::vector<float> y(elems);
  for (size_t i = 0; i < elems; ++i) y[i] = __half2float(y_half[i]);
  std::FILE* fout = std::fopen(out_path, "wb");
  if (!fout || std::fwrite(y.data(), sizeof(float), elems, fout) != elems)
    return std::fprintf(stderr, "cannot write %s\n", out_path), 2;
  std::fclose(fout);

  if (plan) CHECK_CUFFT(cufftDestroy(plan));
  thunderfft::ThunderFFTFinalize<half>();
  for (void* p : {(void*)d_x, (void*)d_y, (void*)d_H, (void*)d_H_perm, (void*)d_taps_h, (void*)d_taps, (void*)d_taps_f})
    if (p) CHECK_CUDA(cudaFree(p));
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 6) {
    std::fprintf(stderr, "usage: %s <N: 1024|4096> <taps> <batch> <in.bin> <out.bin>\n", argv[0]);
    return 2;
  }
  const int n = std::atoi(argv[1]), taps = std::atoi(argv[2]), batch = std::atoi(argv[3]);
  if ((n != 1024 && n != 4096) || taps < 1 || taps > n || batch < 1) {
    std::fprintf(stderr, "need N in {1024, 4096}, 1 <= taps <= N, batch >= 1\n");
    return 2;
  }
  return n == 4096 ? run_io<4096>(taps, batch, argv[4], argv[5]) : run_io<1024>(taps, batch, argv[4], argv[5]);
}
