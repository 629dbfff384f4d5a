// thunderfft_impl_twiddle.cuh — twiddle cache API (host) and the device
// symbols that mirror it.
//
// The cache itself lives in libthunderfft_b200.so (thff_initialize /
// thff_finalize / thff_twiddle_table); this header keeps, per translation
// unit, the device symbols the reference exposes for inspection
// (reference: detail/thunderfft_impl_twiddle.cuh:44-52) and updates them on
// every Initialize/Finalize, so the same observable contract holds:
//   d_twiddle_f / d_twiddle_N_f  (float),  d_twiddle_h / d_twiddle_N_h (half):
//   pointer to W[k] = (cos 2 pi k/N, sin 2 pi k/N), k < N, and N; null/0
//   after Finalize.
//   d_unit_twiddle_half2: the FP16 per-lane coefficient table that
//   unit_fp16::make_reg_b_precompute reads, equal to build_unit_twiddle_host().
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "../../thff.h"
#include "util_cuda.h"

namespace thunderfft {

constexpr int WARP_SIZE = 32;
constexpr int UNIT_ENTRIES = 36;
constexpr int UNIT_W_SIZE = UNIT_ENTRIES * WARP_SIZE * 2;

template <typename T>
struct TwiddleCache {
  using TwiddleT = std::conditional_t<std::is_same_v<T, float>, float2, half2>;
  // Devices whose FP16 unit table has been uploaded in this translation unit.
  inline static std::map<int, bool> unit_ready;
  inline static std::mutex mutex;
};

namespace detail {

__device__ __constant__ const float2* d_twiddle_f = nullptr;
__device__ __constant__ int d_twiddle_N_f = 0;
__device__ __constant__ const half2* d_twiddle_h = nullptr;
__device__ __constant__ int d_twiddle_N_h = 0;

__device__ half2 d_unit_twiddle_half2[UNIT_W_SIZE];
__device__ float2 d_unit_twiddle_float2[UNIT_W_SIZE];

inline void throw_status(thff_status st) {
  if (st == THFF_OK) return;
  const char* msg = thff_last_error();
  if (st == THFF_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

template <typename T>
constexpr int dtype_code() {
  return std::is_same_v<T, half> ? THFF_F16 : THFF_F32;
}

template <typename T>
inline void set_twiddle_symbols(const void* pointer, int n) {
  if constexpr (std::is_same_v<T, float>) {
    const float2* p = static_cast<const float2*>(pointer);
    tf_check_cuda(cudaMemcpyToSymbol(d_twiddle_f, &p, sizeof(p)), "MemcpyToSymbol(d_twiddle_f)");
    tf_check_cuda(cudaMemcpyToSymbol(d_twiddle_N_f, &n, sizeof(n)), "MemcpyToSymbol(d_twiddle_N_f)");
  } else {
    const half2* p = static_cast<const half2*>(pointer);
    tf_check_cuda(cudaMemcpyToSymbol(d_twiddle_h, &p, sizeof(p)), "MemcpyToSymbol(d_twiddle_h)");
    tf_check_cuda(cudaMemcpyToSymbol(d_twiddle_N_h, &n, sizeof(n)), "MemcpyToSymbol(d_twiddle_N_h)");
  }
}

}  // namespace detail

template <typename PairT>
inline PairT make_pair(float a, float b);
template <>
inline half2 make_pair<half2>(float a, float b) {
  return __halves2half2(__float2half_rn(a), __float2half_rn(b));
}
template <>
inline float2 make_pair<float2>(float a, float b) {
  return make_float2(a, b);
}

// Per-lane unit coefficients of this library's FP16 device path:
//   W[(dir * 36 + e) * 32 + lane] = exp(s * 2*pi*i * ((lane * e) mod 1152) / 1152),
//   s = -1 for dir 0 (forward), +1 for dir 1 (inverse).
template <typename PairT>
void build_unit_twiddle_host(std::vector<PairT>& W) {
  W.resize(UNIT_W_SIZE);
  constexpr double tau = 6.283185307179586476925286766559;
  for (int dir = 0; dir < 2; ++dir)
    for (int e = 0; e < UNIT_ENTRIES; ++e)
      for (int lane = 0; lane < WARP_SIZE; ++lane) {
        const double th = (dir == 0 ? -1.0 : 1.0) * tau * double((lane * e) % 1152) / 1152.0;
        W[(dir * UNIT_ENTRIES + e) * WARP_SIZE + lane] = make_pair<PairT>(float(std::cos(th)), float(std::sin(th)));
      }
}

template <typename T>
inline void ThunderFFTInitialize(int N) {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>,
                "ThunderFFTInitialize<T>: supported T are float and half only");
  if (N != 64 && N != 128 && N != 256 && N != 512 && N != 1024 && N != 2048 && N != 4096)
    throw std::invalid_argument("ThunderFFTInitialize<T>: unsupported FFT size");
  std::lock_guard<std::mutex> lock(TwiddleCache<T>::mutex);
  detail::throw_status(thff_initialize(detail::dtype_code<T>(), N));
  const void* table = nullptr;
  int n = 0;
  detail::throw_status(thff_twiddle_table(detail::dtype_code<T>(), &table, &n));
  detail::set_twiddle_symbols<T>(table, n);
  if constexpr (std::is_same_v<T, half>) {
    int device = 0;
    tf_check_cuda(cudaGetDevice(&device), "cudaGetDevice (initialize)");
    if (!TwiddleCache<T>::unit_ready[device]) {
      std::vector<half2> unit;
      build_unit_twiddle_host(unit);
      tf_check_cuda(cudaMemcpyToSymbol(detail::d_unit_twiddle_half2, unit.data(), sizeof(half2) * UNIT_W_SIZE),
                    "MemcpyToSymbol(d_unit_twiddle_half2)");
      TwiddleCache<T>::unit_ready[device] = true;
    }
  }
}

template <typename T>
inline void ThunderFFTFinalize() {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>,
                "ThunderFFTFinalize<T>: supported T are float and half only");
  std::lock_guard<std::mutex> lock(TwiddleCache<T>::mutex);
  detail::throw_status(thff_finalize(detail::dtype_code<T>()));
  detail::set_twiddle_symbols<T>(nullptr, 0);
}

template <typename T>
__device__ __forceinline__ const typename TwiddleCache<T>::TwiddleT* ThunderFFT_get_twiddle();
template <>
__device__ __forceinline__ const float2* ThunderFFT_get_twiddle<float>() {
  return detail::d_twiddle_f;
}
template <>
__device__ __forceinline__ const half2* ThunderFFT_get_twiddle<half>() {
  return detail::d_twiddle_h;
}
__device__ __forceinline__ half2* ThunderFFT_get_unit_twiddle_half2() { return detail::d_unit_twiddle_half2; }
__device__ __forceinline__ float2* ThunderFFT_get_unit_twiddle_float2() { return detail::d_unit_twiddle_float2; }

namespace unit_fp16 {
// Fill the per-thread coefficient array (36 entries) for this lane.
template <int N, bool forward>
__device__ __forceinline__ void make_reg_b_precompute(vec2_t<half>* W) {
  const int lane = threadIdx.x & 31;
  const int dir = forward ? 0 : 1;
#pragma unroll
  for (int e = 0; e < UNIT_ENTRIES; ++e) W[e] = detail::d_unit_twiddle_half2[(dir * UNIT_ENTRIES + e) * WARP_SIZE + lane];
}
}  // namespace unit_fp16

}  // namespace thunderfft
