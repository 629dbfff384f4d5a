// conv2d_kernels.cuh — filter-spectrum kernels of the 2-D FFT convolution.
//
// Counterpart of the reference's 2-D FFT convolution sample
// (sample/conv2d/thunder.cu:70-207,410-592: row FFT, column FFT x H x column
// IFFT, row IFFT).  Here for BASELINE config 5: real fp32 images [B][C][H][W]
// with one real F x F filter per channel, circular convolution
//     y[b][c] = x[b][c] (*) h[c]   (filter zero-padded to H x W).
// Two images of the same channel (batch b and b+1) share one complex 2-D
// transform (z = x_b + i x_{b+1}; the filter is real, so Re/Im of the result
// are the two outputs).  The four transform passes are fft2_kernel
// instances with the conv2d input/output modes (fft_kernels.cuh); this file
// holds the one-time filter-spectrum preparation and the range exponents of
// the half2 (mixed-arithmetic) pipeline.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "fft_kernels.cuh"

namespace thff {

// 2-D filter spectra, stored transposed (the column-transform layout):
// spec[ch][k2][k1] = (1/(H W)) sum_{u,v < F} h[ch][u][v] exp(-2 pi i (u k1 / H + v k2 / W)).
// Separable: first g[ch][u][k2] = sum_v h[ch][u][v] w_W^(v k2) (FP64 accumulation).
__global__ void conv2d_filter_rows_kernel(const float* __restrict__ h, int C, int F, int W, double2* __restrict__ g) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)C * F * W) return;
  const int k2 = (int)(i % W);
  const long long cu = i / W;  // ch*F + u
  double sr = 0.0, si = 0.0;
  for (int v = 0; v < F; ++v) {
    double s, c;
    sincospi(-2.0 * (double)(((long long)v * k2) % W) / (double)W, &s, &c);
    const double hv = h[cu * F + v];
    sr += hv * c;
    si += hv * s;
  }
  g[i] = make_double2(sr, si);
}

__global__ void conv2d_filter_cols_kernel(const double2* __restrict__ g, int C, int F, int H, int W,
                                          float2* __restrict__ spec) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (ch, k2, k1)
  if (i >= (long long)C * H * W) return;
  const int k1 = (int)(i % H);
  const int k2 = (int)((i / H) % W);
  const long long ch = i / ((long long)H * W);
  double sr = 0.0, si = 0.0;
  for (int u = 0; u < F; ++u) {
    double s, c;
    sincospi(-2.0 * (double)(((long long)u * k1) % H) / (double)H, &s, &c);
    const double2 gv = g[(ch * F + u) * W + k2];
    sr += gv.x * c - gv.y * s;
    si += gv.x * s + gv.y * c;
  }
  const double scale = 1.0 / ((double)H * (double)W);
  spec[i] = make_float2((float)(sr * scale), (float)(si * scale));
}

// ---- range exponents of the half2 pipeline ------------------------------
// Every half2 intermediate is kept at or below 2^9 per real or imaginary part,
// so that inside a pass the stage-1 partial sums (at most NS * sqrt2 times
// larger, NS <= 64) stay below the FP16 maximum 65504.  The bounds are exact
// consequences of |DFT_n(v)| <= n max|v|, so no input overflows:
//   P1 stores Y 2^e1,        e1 = 9 - ceil_log2(w sqrt2 max|x|)   per image pair
//   P2 stores X H 2^e2,      e2 = -ceil_log2(2 h max|H|)           per call
//   P3 stores Z 2^e3,        e3 = -ceil_log2(h sqrt2)              per call
//   P4 multiplies by 2^-(e1 + e2 + e3).
// The products get a 1e-4 relative margin against float rounding.

// e1 of image pairs pair0 .. pair0 + gridDim.x - 1 into e1_out[blockIdx.x].
__global__ void conv2d_pair_exp_kernel(const float* __restrict__ x, long long nimg_b, int chans, long long ppc,
                                       long long pair0, int h, int w, int* __restrict__ e1_out) {
  const long long pg = pair0 + blockIdx.x;
  const long long ch = pg / ppc, b = 2 * (pg - ch * ppc);
  const long long hw4 = (long long)h * w / 4;
  float m = 0.f;
  for (int img = 0; img < 2; ++img) {
    if (b + img >= nimg_b) break;
    const float4* src = reinterpret_cast<const float4*>(x + ((b + img) * chans + ch) * hw4 * 4);
    for (long long i = threadIdx.x; i < hw4; i += blockDim.x) {
      const float4 v = __ldg(src + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) {
      const float bound = m * (float)w * 1.41421356f * 1.0001f;
      // clamped to pow2f's exact range: P1 scales by 2^e1 alone
      const int e1 = m > 0.f ? 9 - detail::ceil_log2f(bound) : 0;
      e1_out[blockIdx.x] = e1 < -120 ? -120 : (e1 > 120 ? 120 : e1);
    }
  }
}

// Largest real or imaginary part of the spectra, as float bits (nonnegative
// floats order like their bit patterns) into *amax (zeroed by the caller).
__global__ void conv2d_spectra_absmax_kernel(const float* __restrict__ spec, long long count, unsigned* amax) {
  float m = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__ldg(spec + i)));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(m));
}

// e2, e3 of one call into e[0], e[1] from the spectra's largest part.
__global__ void conv2d_call_exp_kernel(const unsigned* amax, int h, int* e) {
  const float mh = __uint_as_float(*amax);
  // clamped to pow2f's exact range: P2 scales by 2^e2 alone
  const int e2 = mh > 0.f ? -detail::ceil_log2f(2.0f * (float)h * mh * 1.0001f) : 0;
  e[0] = e2 < -120 ? -120 : (e2 > 120 ? 120 : e2);
  e[1] = -detail::ceil_log2f((float)h * 1.41421356f * 1.0001f);
}

}  // namespace thff
