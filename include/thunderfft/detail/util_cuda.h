// util_cuda.h — basic types and error helpers of the ThunderFFT header API.
// Same names and meaning as the reference's detail/util_cuda.h (vec2_t at
// :46-49, tf_check_cuda at :20-24): the public signatures depend on them.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <type_traits>

// Complex storage type: float -> float2 (x = re, y = im); half -> half2
// (low = re, high = im).
template <class T>
using vec2_t = typename std::conditional_t<std::is_same_v<std::remove_cv_t<T>, float>, float2, half2>;

// CUDA failures surface as std::runtime_error("[ThunderFFT] <what>: <cuda message>").
static inline void tf_check_cuda(cudaError_t e, const char* msg) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("[ThunderFFT] ") + msg + ": " + cudaGetErrorString(e));
}

template <typename T>
constexpr const char* type_cstr() {
  using U = std::remove_cv_t<T>;
  if constexpr (std::is_same_v<U, float>) return "float";
  else if constexpr (std::is_same_v<U, double>) return "double";
  else if constexpr (std::is_same_v<U, int>) return "int";
  else if constexpr (std::is_same_v<U, float2>) return "float2";
  else if constexpr (std::is_same_v<U, half>) return "half";
  else if constexpr (std::is_same_v<U, half2>) return "half2";
  else return "unknown";
}
