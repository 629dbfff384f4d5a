// thunderfft_impl_device_fft.cuh — ThunderFFT_kernel_reg: the composable
// in-kernel FFT of the device API.
//
// The reference's device routine (ThunderFFT_kernel_reg, shared_kernel_n*.cuh)
// is a warp-MMA register FFT with size-specific fragment maps.  This library
// keeps its calling contract (block shape, 32-element fragments, caller
// workspace and barriers) but computes it as a self-sorting (Stockham)
// radix-4 FFT over the caller's shared-memory workspace, FP32 arithmetic
// with exactly reduced twiddles (sincospif), FP16 storage rounding between
// passes for half.  Fused kernels keep their data on chip; the large batched
// transforms use the tcgen05 kernels behind ThunderFFT_global.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "util_arith.h"
#include "util_cuda.h"

namespace thunderfft {
namespace detail {

template <typename T>
__device__ __forceinline__ float2 to_f2(vec2_t<T> v) {
  if constexpr (std::is_same_v<T, half>) return __half22float2(v);
  else return v;
}
template <typename T>
__device__ __forceinline__ vec2_t<T> from_f2(float2 v) {
  if constexpr (std::is_same_v<T, half>) return __floats2half2_rn(v.x, v.y);
  else return v;
}

// exp(sign * 2*pi*i * num / den) with exact argument reduction.
__device__ __forceinline__ float2 unit_root(int num, int den, bool forward) {
  float s, c;
  sincospif(2.0f * float(num % den) / float(den), &s, &c);
  return make_float2(c, forward ? -s : s);
}

// One Stockham pass of radix R over `count` signals of length N held in
// `ws`: butterfly j (< N/R) of each signal reads x[j + r*N/R], applies
// w_{Ns*R}^{r*(j mod Ns)}, transforms, and writes y[(j/Ns)*Ns*R + j%Ns + r*Ns].
template <typename T, int N, int R, int P, int COUNT, bool forward>
__device__ __forceinline__ void stockham_pass(vec2_t<T>* ws, int Ns, int t) {
  constexpr int BF = N * COUNT / R;  // butterflies in the tile
  constexpr int PER = (BF + P - 1) / P;
  float2 v[PER][R];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int b = t + P * q;
    if (b < BF) {
      const int sig = b / (N / R), j = b % (N / R);
#pragma unroll
      for (int r = 0; r < R; ++r) v[q][r] = to_f2<T>(ws[sig * N + j + r * (N / R)]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int b = t + P * q;
    if (b < BF) {
      const int sig = b / (N / R), j = b % (N / R);
      const int k = j % Ns;
#pragma unroll
      for (int r = 1; r < R; ++r) v[q][r] = cmul(v[q][r], unit_root(r * k, Ns * R, forward));
      float2 o[R];
      if constexpr (R == 2) {
        o[0] = make_float2(v[q][0].x + v[q][1].x, v[q][0].y + v[q][1].y);
        o[1] = make_float2(v[q][0].x - v[q][1].x, v[q][0].y - v[q][1].y);
      } else {
        const float2 t0 = make_float2(v[q][0].x + v[q][2].x, v[q][0].y + v[q][2].y);
        const float2 t1 = make_float2(v[q][0].x - v[q][2].x, v[q][0].y - v[q][2].y);
        const float2 t2 = make_float2(v[q][1].x + v[q][3].x, v[q][1].y + v[q][3].y);
        const float2 d = make_float2(v[q][1].x - v[q][3].x, v[q][1].y - v[q][3].y);
        // w4 * d with w4 = -i (forward) or +i (inverse)
        const float2 t3 = forward ? make_float2(d.y, -d.x) : make_float2(-d.y, d.x);
        o[0] = make_float2(t0.x + t2.x, t0.y + t2.y);
        o[2] = make_float2(t0.x - t2.x, t0.y - t2.y);
        o[1] = make_float2(t1.x + t3.x, t1.y + t3.y);
        o[3] = make_float2(t1.x - t3.x, t1.y - t3.y);
      }
      const int dst = (j / Ns) * Ns * R + k;
#pragma unroll
      for (int r = 0; r < R; ++r) ws[sig * N + dst + r * Ns] = from_f2<T>(o[r]);
    }
  }
  __syncthreads();
}

template <typename T, int N, int COUNT, bool forward, int P>
__device__ __forceinline__ void stockham_fft(vec2_t<T>* ws, int t) {
  int Ns = 1;
  constexpr int L = LOG2P_builtin<N>;
#pragma unroll
  for (int p = 0; p < L / 2; ++p) {
    stockham_pass<T, N, 4, P, COUNT, forward>(ws, Ns, t);
    Ns *= 4;
  }
  if constexpr (L % 2 == 1) stockham_pass<T, N, 2, P, COUNT, forward>(ws, Ns, t);
}

}  // namespace detail

template <typename T, int N, int batch, bool forward>
__device__ __forceinline__ void ThunderFFT_kernel_reg(vec2_t<T>* __restrict__ reg, vec2_t<T>* __restrict__ W,
                                                      void* workspace) {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>, "float and half only");
  static_assert(N == 64 || N == 128 || N == 256 || N == 512 || N == 1024 || N == 2048 || N == 4096,
                "Unsupported ThunderFFT length");
  (void)W;
  using F = detail::frag<N, batch>;
  vec2_t<T>* ws = static_cast<vec2_t<T>*>(workspace);
  const int t = detail::block_thread();
#pragma unroll
  for (int i = 0; i < F::EPT; ++i) ws[t + F::P * i] = reg[i];
  __syncthreads();
  detail::stockham_fft<T, N, batch, forward, F::P>(ws, t);
#pragma unroll
  for (int i = 0; i < F::EPT; ++i) reg[i] = ws[t + F::P * i];
}

}  // namespace thunderfft
