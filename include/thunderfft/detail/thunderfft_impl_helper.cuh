// thunderfft_impl_helper.cuh — layout-aware data movement of the device API.
//
// Fragment convention of this library: with P = 32 * warp_per_block<N>
// threads and t = threadIdx.x + 32 * threadIdx.y, thread t holds element
// e = t + P * i (i < 32) of the block's tile in signal order (e = j*N + n);
// half2 N = 64 (16 signals) and N = 128 (8 signals) and float2 N = 64, 128
// and 256 use their MMA operand orders instead (frag_elem); the float2
// output orders differ from their input orders (frag_elem_out).
// The input fragment holds input elements, the output fragment output
// elements, both in natural order; the helpers translate to and from any
// layout_t (strides, periodic padding, digit-reversed shared tiles).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "thunderfft_impl_device_mma.cuh"
#include "util_arith.h"
#include "util_cuda.h"

namespace thunderfft {
namespace detail {

template <typename sL>
__device__ __forceinline__ int layout_index(int j, int n) {
  int idx = n * sL::elem_stride + j * sL::batch_stride;
  return idx + (idx / sL::pad_period) * sL::pad;
}

// Position in a layout's tile that holds natural element n of a signal.
template <typename sL>
__device__ __forceinline__ int stored_position(int n) {
  if constexpr (sL::reversed) return unreverse_bit_groups<2, LOG2P_builtin<sL::N>>(n);
  else return n;
}

template <int N, int batch>
struct frag {
  static constexpr int P = 32 * warp_per_block<N>;
  static constexpr int EPT = N * batch / P;
  static_assert(EPT * P == N * batch, "tile must split evenly over the block");
};

__device__ __forceinline__ int block_thread() { return threadIdx.x + threadIdx.y * blockDim.x; }

// Fragment slot i of block thread t holds element n of signal j of the
// block's tile: t + P i in signal order, except for half2 N = 64 with 16
// signals and N = 128 with 8, whose warp-MMA routines keep the MMA operand
// order (mfft::frag64, mfft::frag128), the float2 TF32 routines, and half2
// N = 256 with 16 signals (mfft::frag256_h: 16 elements of two signals).
template <typename T, int N, int batch>
__device__ __forceinline__ void frag_elem(int t, int i, int& j, int& n) {
  if constexpr (mfft::enabled<T, N, batch> || mfft::tf32_enabled<T, N, batch>) {
    if constexpr (N == 64) mfft::frag64(t, i, j, n);
    else if constexpr (N == 128) mfft::frag128(t, i, j, n);
    else mfft::frag256_tf32_in(t, i, j, n);
  } else if constexpr (mfft::h256_enabled<T, N, batch>) {
    mfft::frag256_h(t, i, j, n);
  } else {
    const int e = t + frag<N, batch>::P * i;
    j = e / N;
    n = e % N;
  }
}

// Fragment slot i of block thread t in an OUTPUT fragment: the input order
// (frag_elem), except for the TF32 warp-MMA routines (float2 N = 64, 128,
// 256 and half2 N = 128), which end with an in-lane DFT and leave its
// outputs in the lane that computed them (mfft::frag64_tf32_out,
// frag128_tf32_out, frag256_tf32_out).
template <typename T, int N, int batch>
__device__ __forceinline__ void frag_elem_out(int t, int i, int& j, int& k) {
  if constexpr (mfft::split_order<T, N, batch>) {
    if constexpr (N == 64) mfft::frag64_tf32_out(t, i, j, k);
    else if constexpr (N == 128) mfft::frag128_tf32_out(t, i, j, k);
    else mfft::frag256_tf32_out(t, i, j, k);
  } else {
    frag_elem<T, N, batch>(t, i, j, k);
  }
}

}  // namespace detail

// Contiguous natural-order global tile -> shared memory described by sL
// (sL::reversed stores the digit-reversed permutation).
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_gmem2smem(vec2_t<T>* __restrict__ smem, const vec2_t<T>* __restrict__ gmem) {
  constexpr int N = sL::N, B = sL::batch, P = 32 * warp_per_block<N>;
  const int t = detail::block_thread();
  for (int e = t; e < N * B; e += P) {
    const int j = e / N, p = e % N;
    const int n = sL::reversed ? reverse_bit_groups<2, LOG2P_builtin<N>>(p) : p;
    smem[detail::layout_index<sL>(j, p)] = gmem[j * N + n];
  }
}

// Shared memory described by sL -> contiguous natural-order global tile.
// Requires sL::reversed == false (a reversed layout writes nothing).
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_smem2gmem(vec2_t<T>* __restrict__ gmem, const vec2_t<T>* __restrict__ smem) {
  constexpr int N = sL::N, B = sL::batch, P = 32 * warp_per_block<N>;
  if constexpr (!sL::reversed) {
    const int t = detail::block_thread();
    for (int e = t; e < N * B; e += P) gmem[e] = smem[detail::layout_index<sL>(e / N, e % N)];
  }
}

// Shared memory described by sL -> input fragment.
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_smem2reg(vec2_t<T>* __restrict__ reg, const vec2_t<T>* __restrict__ smem) {
  using F = detail::frag<sL::N, sL::batch>;
  const int t = detail::block_thread();
#pragma unroll
  for (int i = 0; i < F::EPT; ++i) {
    int j, n;
    detail::frag_elem<T, sL::N, sL::batch>(t, i, j, n);
    reg[i] = smem[detail::layout_index<sL>(j, detail::stored_position<sL>(n))];
  }
}

// Output fragment -> shared memory described by sL (natural order, or the
// digit-reversed order when sL::reversed).
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_reg2smem(vec2_t<T>* __restrict__ smem, const vec2_t<T>* __restrict__ reg) {
  using F = detail::frag<sL::N, sL::batch>;
  const int t = detail::block_thread();
#pragma unroll
  for (int i = 0; i < F::EPT; ++i) {
    int j, k;
    detail::frag_elem_out<T, sL::N, sL::batch>(t, i, j, k);
    smem[detail::layout_index<sL>(j, detail::stored_position<sL>(k))] = reg[i];
  }
}

// Global memory -> input fragment (gmem = block-local base of `batch`
// contiguous natural-order signals).
template <typename T, int N, int batch>
__device__ __forceinline__ void ThunderFFT_gmem2reg(vec2_t<T>* __restrict__ reg, const vec2_t<T>* __restrict__ gmem) {
  ThunderFFT_smem2reg<T, layout_t<N, batch, 1, N, 1, 0, false>>(reg, gmem);
}

// Output fragment -> natural-order contiguous global tile.
template <typename T, int N, int batch>
__device__ __forceinline__ void ThunderFFT_reg2gmem(vec2_t<T>* __restrict__ gmem, const vec2_t<T>* __restrict__ reg) {
  ThunderFFT_reg2smem<T, layout_t<N, batch, 1, N, 1, 0, false>>(gmem, reg);
}

}  // namespace thunderfft
