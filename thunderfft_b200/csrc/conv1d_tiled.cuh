// conv1d_tiled.cuh — operator of the tiled (overlap-save) 1-D convolution.
//
// Counterpart of the reference's tiled conv1d sample
// (sample/conv1d/main.cu:38-129, 146-153, 214-276): a long complex sequence
// is cut into 64-point windows that advance by V = 64 - f + 1; each window
// goes through a 64-point FFT, a multiply by the spectrum of the filter
// placed at (64 - k) mod 64 and scaled by 1/64, and an inverse FFT, and its
// first V outputs are kept.  The result is the valid correlation
//     y[i] = sum_{k<f} x[i + k] g[k],   i < L - f + 1
// (main.cu:157-172).
//
// For a fixed filter that FFT -> multiply -> inverse FFT chain is one 64 x 64
// complex linear map of the window, the circulant C[j][m] = g[(m - j) mod 64]
// (zero where (m - j) mod 64 >= f); on the first V outputs it never wraps.
// Here it is formed once, exactly, from the taps and stored as the real
// 128 x 128 B operand of the N = 64 kernel (dft1_kernel in window mode),
// which applies it to 128 windows per tcgen05 MMA pass:
//     row n = 2 j + c_out (output j, re|im), column K = 2 m + c_in,
//     [re, im]_j = sum_m [[g.re, -g.im], [g.im, g.re]] [re, im]_m,
// laid out K-major with 128-B swizzle like the DFT matrix it replaces.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"

namespace thff {

template <bool kHalf>
__global__ void conv1d_tiled_operator_kernel(const float2* __restrict__ filter, int f, uint8_t* __restrict__ img) {
  constexpr int R = 128, ESZ = kHalf ? 2 : 4, E = 128 / ESZ;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * R) return;
  const int n = i / R, K = i % R;             // output row, input column
  const int j = n >> 1, co = n & 1, m = K >> 1, ci = K & 1;
  const int d = m - j;
  float v = 0.f;
  if (d >= 0 && d < f) {
    const float2 g = filter[d];
    v = co == 0 ? (ci == 0 ? g.x : -g.y) : (ci == 0 ? g.y : g.x);
  }
  const uint32_t off = (uint32_t)(K / E) * (R * 128u) + sm100::sw128((uint32_t)n * 128u + (uint32_t)(K % E) * ESZ);
  if constexpr (kHalf) {
    *reinterpret_cast<__half*>(img + off) = __float2half_rn(v);
  } else {
    *reinterpret_cast<float*>(img + off) = sm100::round_tf32(v);
  }
}

}  // namespace thff
