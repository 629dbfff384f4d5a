// thunderfft_impl.cuh — launch tuples and the implementation includes.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "util_arith.h"

namespace thunderfft {

// Launch tuples of the device API (FFTs per block, warps per block).  They
// are part of the fusion contract (callers size blocks, fragments and
// workspaces with them), so they keep the reference's values
// (detail/thunderfft_impl.cuh:14-32): every thread holds 32 complex values.
template <int N>
inline constexpr int batch_per_block = (N == 64)    ? 16
                                       : (N == 128) ? 8
                                       : (N == 256) ? 16
                                       : (N == 512) ? 2
                                       : (N == 1024 || N == 2048 || N == 4096) ? 1
                                                                                : 0;

template <int N>
inline constexpr int warp_per_block = (N == 64 || N == 128 || N == 512 || N == 1024) ? 1
                                      : (N == 256 || N == 4096)                     ? 4
                                      : (N == 2048)                                 ? 2
                                                                                    : 0;

constexpr int threads_per_warp = 32;

}  // namespace thunderfft

#include "thunderfft_impl_twiddle.cuh"
#include "thunderfft_impl_helper.cuh"
#include "thunderfft_impl_device_fft.cuh"
#include "thunderfft_impl_kernel.cuh"
