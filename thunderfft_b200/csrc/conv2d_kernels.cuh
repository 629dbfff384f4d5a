// conv2d_kernels.cuh — helper kernels of the 2-D FFT convolution.
//
// Counterpart of the reference's 2-D FFT convolution sample
// (sample/conv2d/thunder.cu:70-207,410-592: row FFT, column FFT x H x column
// IFFT, row IFFT).  Here for BASELINE config 5: real fp32 images [B][C][H][W]
// with one real F x F filter per channel, circular convolution
//     y[b][c] = x[b][c] (*) h[c]   (filter zero-padded to H x W).
// Two images of the same channel (batch b and b+1) share one complex 2-D
// transform (z = x_b + i x_{b+1}; the filter is real, so Re/Im of the result
// are the two outputs).  The transforms themselves are the tcgen05 C2C
// kernels; the kernels here are the HBM-bound glue between them.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace thff {

// z[p][r][c] = (x[b][ch][r][c], x[b+1][ch][r][c]), pair p = (b/2)*C + ch,
// missing partner image (odd B) -> 0.  One thread per 4 columns.
__global__ void conv2d_pack_kernel(const float* __restrict__ x, float2* __restrict__ z, int B, int C, int HW,
                                   long long pair0, long long npairs) {
  const long long i4 = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // index of 4 pixels
  const long long hw4 = HW / 4;
  if (i4 >= npairs * hw4) return;
  const long long pl = i4 / hw4, q = i4 % hw4;
  const long long p = pair0 + pl;
  const long long b = 2 * (p / C), ch = p % C;
  const float4 a = reinterpret_cast<const float4*>(x + (b * C + ch) * (long long)HW)[q];
  float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
  if (b + 1 < B) bb = reinterpret_cast<const float4*>(x + ((b + 1) * C + ch) * (long long)HW)[q];
  float4* dst = reinterpret_cast<float4*>(z + pl * (long long)HW + 4 * q);
  dst[0] = make_float4(a.x, bb.x, a.y, bb.y);
  dst[1] = make_float4(a.z, bb.z, a.w, bb.w);
}

// y[b][ch] = Re z[p], y[b+1][ch] = Im z[p].
__global__ void conv2d_unpack_kernel(const float2* __restrict__ z, float* __restrict__ y, int B, int C, int HW,
                                     long long pair0, long long npairs) {
  const long long i4 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long hw4 = HW / 4;
  if (i4 >= npairs * hw4) return;
  const long long pl = i4 / hw4, q = i4 % hw4;
  const long long p = pair0 + pl;
  const long long b = 2 * (p / C), ch = p % C;
  const float4* src = reinterpret_cast<const float4*>(z + pl * (long long)HW + 4 * q);
  const float4 s0 = src[0], s1 = src[1];
  reinterpret_cast<float4*>(y + (b * C + ch) * (long long)HW)[q] = make_float4(s0.x, s0.z, s1.x, s1.z);
  if (b + 1 < B)
    reinterpret_cast<float4*>(y + ((b + 1) * C + ch) * (long long)HW)[q] = make_float4(s0.y, s0.w, s1.y, s1.w);
}

// Per-image complex transpose [n][rows][cols] -> [n][cols][rows] through
// 32x32 shared tiles; optionally multiplies by a per-channel spectrum that is
// already in the destination layout (spec[ch][cols][rows]).
template <bool kMul>
__global__ void conv2d_transpose_kernel(const float2* __restrict__ src, float2* __restrict__ dst, int rows, int cols,
                                        const float2* __restrict__ spec, int C, long long pair0) {
  __shared__ float2 tile[32][33];
  const long long img = blockIdx.z;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const float2* s = src + img * (long long)rows * cols;
  float2* d = dst + img * (long long)rows * cols;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) tile[i][threadIdx.x] = s[(long long)(r0 + i) * cols + c0 + threadIdx.x];
  __syncthreads();
  const float2* h = kMul ? spec + ((pair0 + img) % C) * (long long)rows * cols : nullptr;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    float2 v = tile[threadIdx.x][i];
    const long long o = (long long)(c0 + i) * rows + r0 + threadIdx.x;
    if constexpr (kMul) {
      const float2 w = h[o];
      v = make_float2(v.x * w.x - v.y * w.y, v.x * w.y + v.y * w.x);
    }
    d[o] = v;
  }
}

// In-place z[p] *= spec[ch(p)] (same layout).
__global__ void conv2d_mul_kernel(float2* __restrict__ z, const float2* __restrict__ spec, int C, long long HW,
                                  long long pair0, long long npairs) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= npairs * HW) return;
  const long long pl = i / HW, o = i % HW;
  const float2 w = spec[((pair0 + pl) % C) * HW + o];
  const float2 v = z[i];
  z[i] = make_float2(v.x * w.x - v.y * w.y, v.x * w.y + v.y * w.x);
}

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

}  // namespace thff
