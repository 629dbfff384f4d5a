// util_arith.h — small arithmetic helpers used by the device-side API.
//
// pad_h(N) and reverse_bit_groups keep the reference's names and meaning
// because caller code sizes workspaces with pad_h and layout_t's Reversed_
// flag is defined through reverse_bit_groups (reference
// detail/util_arith.h:17-30, :123-136).  The values of pad_h are this
// library's own: the device FFT uses only the first N*batch elements of a
// workspace, and the tuned layouts stay inside (N + pad_h(N)) * batch.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

template <unsigned int N>
inline constexpr unsigned LOG2P_builtin = [] {
  static_assert(N && (N & (N - 1)) == 0, "N must be a power of two");
  unsigned l = 0;
  while ((1u << l) < N) ++l;
  return l;
}();

// Base-2^r digit reversal of the low (Bits / r) * r bits of x, with the
// Bits % r leftover high bits appended at the bottom.
template <int r, int Bits>
__host__ __device__ __forceinline__ int reverse_bit_groups(int x) {
  constexpr int groups = Bits / r;
  int result = 0;
  for (int i = 0; i < groups; ++i) result |= ((x >> (r * i)) & ((1 << r) - 1)) << (r * (groups - 1 - i));
  for (int i = 0; i < Bits % r; ++i) result = (result << 1) | ((x >> (r * groups + i)) & 1);
  return result;
}

// Inverse permutation of reverse_bit_groups<r, Bits>.
template <int r, int Bits>
__host__ __device__ __forceinline__ int unreverse_bit_groups(int y) {
  constexpr int groups = Bits / r, extra = Bits % r;
  const int low = y >> extra;  // digit-reversed groups
  int x = 0;
  for (int i = 0; i < groups; ++i) x |= ((low >> (r * i)) & ((1 << r) - 1)) << (r * (groups - 1 - i));
  for (int i = 0; i < extra; ++i) x |= ((y >> (extra - 1 - i)) & 1) << (r * groups + i);
  return x;
}

// Workspace padding rule (elements per signal) for the standard launch:
// a workspace of (N + pad_h(N)) * batch elements is always sufficient.
constexpr int pad_h(int N) { return N / 16; }

__host__ __device__ __forceinline__ float2 cmul(float2 a, float2 w) {
  return make_float2(a.x * w.x - a.y * w.y, a.y * w.x + a.x * w.y);
}
