// thunderfft.cuh — ThunderFFT public API, B200 (sm_100a) backend.
//
// Drop-in for the reference header (include/thunderfft/thunderfft.cuh of
// mcrl/thunderfft): same namespace, templates, layout descriptor, argument,
// exception and synchronization contracts.  Host entry points forward to the
// C ABI of libthunderfft_b200.so (include/thff.h), whose tcgen05/TMA kernels
// compute the transform; link with -lthunderfft_b200 (CMake target
// `thunderfft`).  The device-side routines below are header-inline so that
// they can be fused into a caller's kernel.
//
// T names the component type: float uses float2 (real, imaginary) storage
// and TF32 tensor-core arithmetic; half uses half2 (low = real, high =
// imaginary) storage and FP16 tensor-core arithmetic (FP32 accumulation).
#pragma once
#include <cuComplex.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "detail/util_cuda.h"

namespace thunderfft {

// Block-local layout descriptor used by the device data-movement helpers.
// N_ and Batch_ describe one block's tile, not the global batch.
//   i : element index within a signal, j : batch index
//   idx        = i * elem_stride + j * batch_stride
//   padded_idx = idx + (idx / pad_period) * pad
// PadPeriod_ must be positive even when Pad_ is zero.  Reversed_ means the
// shared-memory tile holds the signal in base-4 digit-reversed order
// (position p holds element reverse_bit_groups<2, log2 N>(p)).
template <int N_, int Batch_, int ElemStride_, int BatchStride_, int PadPeriod_, int Pad_, bool Reversed_>
struct layout_t {
  static constexpr int N = N_;
  static constexpr int batch = Batch_;
  static constexpr int elem_stride = ElemStride_;
  static constexpr int batch_stride = BatchStride_;
  static constexpr int pad_period = PadPeriod_;
  static constexpr int pad = Pad_;
  static constexpr int reversed = Reversed_;
};

// Initialize internal twiddle tables and FFT constants for T = float or half
// and N in {64, ..., 4096} on the current CUDA device.  Unsupported N throws
// std::invalid_argument before touching CUDA.  One cached N per T per
// device; another N replaces that device's cache.  CUDA failures throw
// std::runtime_error.
template <typename T>
void ThunderFFTInitialize(int N);

// Release the current device's cached table for T; repeated calls are fine.
template <typename T>
void ThunderFFTFinalize();

// Reserved declaration without a definition (as in the reference).
template <typename T>
static T* preprocess_W(int N);

// ---- device data movement (collective over the block; see detail/) ------
template <typename T, int N, int batch>
__device__ __forceinline__ void ThunderFFT_gmem2reg(vec2_t<T>* __restrict__ reg, const vec2_t<T>* __restrict__ gmem);
template <typename T, int N, int batch>
__device__ __forceinline__ void ThunderFFT_reg2gmem(vec2_t<T>* __restrict__ gmem, const vec2_t<T>* __restrict__ reg);
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_smem2reg(vec2_t<T>* __restrict__ reg, const vec2_t<T>* __restrict__ smem);
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_reg2smem(vec2_t<T>* __restrict__ smem, const vec2_t<T>* __restrict__ reg);
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_gmem2smem(vec2_t<T>* __restrict__ smem, const vec2_t<T>* __restrict__ gmem);
template <typename T, typename sL>
__device__ __forceinline__ void ThunderFFT_smem2gmem(vec2_t<T>* __restrict__ gmem, const vec2_t<T>* __restrict__ smem);

// Host launch wrapper for batched complex-to-complex FFTs.  Input and output
// are separate device buffers of batch*N complex elements (signal j at
// offset j*N, natural order).  forward=true uses exp(-2*pi*i*k/N); false is
// the unnormalized inverse.  A zero batch is a no-op before CUDA or pointer
// access; a negative batch, a null pointer for a positive batch, or
// identical/overlapping input and output throws std::invalid_argument.
// The wrapper synchronizes `stream` before returning (including prior work);
// CUDA launch/completion failures and device-side pipeline timeouts throw
// std::runtime_error.  This is not an asynchronous interface.
template <typename T, int N, bool forward = true>
inline void ThunderFFT_global(vec2_t<T>* d_input, vec2_t<T>* d_output, int batch, cudaStream_t stream = 0);

// Reserved declarations without definitions (as in the reference).
template <typename T>
__device__ __forceinline__ void ThunderFFT_kernel_smem(vec2_t<T>* __restrict__ s_input, vec2_t<T>* __restrict__ s_output,
                                                       const T* __restrict__ W_N, int N, int batch);
template <typename T, typename input_L, typename output_L>
__device__ __forceinline__ void ThunderFFT_kernel_smem_pad(vec2_t<T>* __restrict__ s_input,
                                                           vec2_t<T>* __restrict__ s_output,
                                                           const T* __restrict__ W_N, int N, int batch);

// Device FFT for fusion into a caller-owned kernel.  Launch a complete block
// of dim3(32, warp_per_block<N>) and call collectively (it contains block
// barriers).  reg is the per-thread fragment of N*batch/(32*warp_per_block<N>)
// = 32 complex values produced by ThunderFFT_smem2reg/gmem2reg; it is
// overwritten with the output fragment, which ThunderFFT_reg2smem/reg2gmem
// write back in natural order.  workspace is caller-owned shared memory of
// at least (N + pad_h(N)) * batch elements; its contents are clobbered.
// W is accepted for source compatibility (FP16 callers fill it with
// unit_fp16::make_reg_b_precompute) and may be null.
template <typename T, int N, int batch, bool forward>
__device__ __forceinline__ void ThunderFFT_kernel_reg(vec2_t<T>* __restrict__ reg, vec2_t<T>* __restrict__ W,
                                                      void* workspace);

}  // namespace thunderfft

#include "thunderfft/detail/thunderfft_impl.cuh"
