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
// holds the one-time filter-spectrum preparation.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

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

}  // namespace thff
