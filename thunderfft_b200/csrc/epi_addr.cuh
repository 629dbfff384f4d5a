// epi_addr.cuh — per-thread address bases for the unrolled epilogue loops.
//
// An epilogue thread writes one value per (row block bi, 64-column chunk c,
// 8-column group o) of the accumulator it drains.  The write address is a
// function F(warp, lane, bi, c, o) of the thread and of those compile-time loop
// indices.  Written out per value, F costs several integer instructions
// (divisions by the tile shape, the K-row rotation, the swizzle XOR), which
// made integer work the largest instruction class of the 2-D convolution's
// passes.  Most of F is the same for every (c, o) of a thread: when
//     F(w, l, bi, c, o) - F(w, l, bi, 0, 0)
// is the same number for every thread (checked below, at compile time, over
// every warp and lane of the epilogue), a thread computes F(w, l, bi, 0, 0)
// once per kernel and each write adds a compile-time constant, which the
// store instruction takes as its immediate offset.  When only
//     F(w, l, bi, c, o) - F(w, l, bi, 0, o)
// is thread-independent (the swizzle XOR depends on o and on the lane), a
// thread keeps one base per o instead.  Otherwise the caller evaluates F per
// value as before.
#pragma once
#include <cstdint>

namespace thff {
namespace epi {

// kind 2: one base per bi; kind 1: one base per (bi, o); kind 0: none.
// Off::f(warp, lane, bi, c, o) is evaluated for warps [kWarp0, kWarp0 + kWarps),
// lanes 0..31, bi < kBPW, c < kCH and o = 0, kOStep, ... < kO.
template <class Off, int kWarp0, int kWarps, int kBPW, int kCH, int kO, int kOStep = 1>
__host__ __device__ constexpr int addr_kind() {
  bool full = true, per_o = true;
  for (int w = kWarp0; w < kWarp0 + kWarps; ++w)
    for (int l = 0; l < 32; ++l)
      for (int bi = 0; bi < kBPW; ++bi)
        for (int c = 0; c < kCH; ++c)
          for (int o = 0; o < kO; o += kOStep) {
            const uint32_t v = Off::f(w, l, bi, c, o);
            const uint32_t r = Off::f(kWarp0, 0, bi, c, o);
            if (v - Off::f(w, l, bi, 0, 0) != r - Off::f(kWarp0, 0, bi, 0, 0)) full = false;
            if (v - Off::f(w, l, bi, 0, o) != r - Off::f(kWarp0, 0, bi, 0, o)) per_o = false;
          }
  return full ? 2 : (per_o ? 1 : 0);
}

// The compile-time part of F for (bi, c, o) relative to the base the thread
// keeps for that kind.
template <class Off, int kWarp0, int kKind>
__host__ __device__ constexpr uint32_t addr_delta(int bi, int c, int o) {
  return Off::f(kWarp0, 0, bi, c, o) - Off::f(kWarp0, 0, bi, 0, kKind == 2 ? 0 : o);
}

}  // namespace epi
}  // namespace thff
