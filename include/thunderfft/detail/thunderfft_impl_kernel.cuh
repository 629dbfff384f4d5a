// thunderfft_impl_kernel.cuh — ThunderFFT_global, the host launch wrapper.
// Same contract as the reference wrapper
// (detail/thunderfft_impl_kernel.cuh:6-41); the launch itself is the C ABI
// entry thff_global (tcgen05/TMA kernels of libthunderfft_b200.so).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <type_traits>

#include "../../thff.h"
#include "util_cuda.h"

namespace thunderfft {

template <typename T, int N, bool forward>
inline void ThunderFFT_global(vec2_t<T>* d_input, vec2_t<T>* d_output, int batch, cudaStream_t stream) {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>, "ThunderFFT_global supports float and half only");
  static_assert(N == 64 || N == 128 || N == 256 || N == 512 || N == 1024 || N == 2048 || N == 4096,
                "Unsupported ThunderFFT length");
  if (batch < 0) throw std::invalid_argument("ThunderFFT batch must be nonnegative");
  if (batch == 0) return;
  if (!d_input || !d_output || d_input == d_output)
    throw std::invalid_argument("ThunderFFT requires separate non-null input/output buffers");
  detail::throw_status(thff_global(detail::dtype_code<T>(), N, forward ? 1 : 0, d_input, d_output, batch,
                                   static_cast<void*>(stream)));
}

}  // namespace thunderfft
