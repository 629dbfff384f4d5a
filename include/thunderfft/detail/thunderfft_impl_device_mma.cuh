// thunderfft_impl_device_mma.cuh — ThunderFFT_kernel_reg for half2 N = 64 (16
// signals, one warp; and N = 128 on top of it, run128) as two warp-MMA DFT
// stages, the form of the reference's
// routine (detail/kernel/shared_kernel_n64_b16.cuh), written for this
// library's own operand maps.  (The float2 branches below are kept
// compilable and correct; see `enabled` for why float2 does not use them.)
//
// Fragment (input and output): lane (gid, tig) = (lane / 4, lane % 4) holds
// signals gid and gid + 8, elements 16 tig ... 16 tig + 15 of each:
//   reg[i]: signal gid + 8 (i / 16), element 16 tig + i % 16.
//
// With n = n_lo + 8 n_hi and k = k1 + 8 k2:
//
//   stage A  Y[n_lo][k1]   = sum_{n_hi} x[n_lo + 8 n_hi] w_8^(n_hi k1)
//   stage B  X[k1 + 8 k2]  = sum_{n_lo} Y[n_lo][k1] w_64^(n_lo (k1 + 8 k2))
//
// (the twiddle w_64^(n_lo k1) is folded into stage B's matrix, one per k1).
// Each stage is D = A B with the data as A (rows = the 16 signals) and the
// constant DFT matrix as B:
//   * stage A, per n_lo: K = n_hi.  The lane's n_hi are 2 tig and 2 tig + 1,
//     so the matrix's K index tig stands for n_hi = 2 tig and tig + 4 for
//     2 tig + 1: the A operand is the fragment itself.  Outputs k1 = 4 nt +
//     tig land in the lane (nt = n tile).
//   * between the stages the four lanes of a quad exchange through shared
//     memory, from (all n_lo, k1 in {tig, tig + 4}) to (n_lo in {2 tig,
//     2 tig + 1}, all k1);
//   * stage B, per k1: K = n_lo, K index tig = n_lo 2 tig, tig + 4 = 2 tig + 1;
//     the N columns are ordered so that n tile nt gives k2 = 2 tig + nt, i.e.
//     outputs 16 tig + 8 nt + k1: the fragment order again.
// float2 uses mma.m16n8k8 .tf32 (one K step for the real parts, one for the
// imaginary parts); half2 uses mma.m16n8k16 .f16 with FP32 accumulation (K =
// 8 inputs with (re, im) interleaved, so an A register is one half2
// element).  Columns of a B tile are (output, re|im) interleaved.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>
#include <utility>

#include "util_arith.h"
#include "util_cuda.h"

namespace thunderfft {
namespace detail {
namespace mfft {

// The warp-MMA routine serves half2 N = 64 with the API's 16 signals per
// block: 0.49 us per paper-benchmark call (16384 signals) against 1.02 us for
// the packed-FP16 register FFT.  Its float2 form (mma.m16n8k8 .tf32, 64 MMAs
// per call) computes correctly (rel-L2 7.5e-4) at 1.24 us, no faster than
// the FP32 register FFT, which is also exact to 1e-7, so float2 keeps that.
// half2 N = 128 (8 signals) reuses it on 16 rows after a radix-2 step
// (run128).
template <typename T, int N, int batch>
inline constexpr bool enabled =
    std::is_same_v<T, half> && ((N == 64 && batch == 16) || (N == 128 && batch == 8));

// Fragment slot i of block thread t: signal j, element n (the order above).
__device__ __forceinline__ void frag64(int t, int i, int& j, int& n) {
  const int lane = t & 31;
  j = (lane >> 2) + 8 * (i >> 4);
  n = 16 * (lane & 3) + (i & 15);
}

// N = 128 with 8 signals: lane (gid, tig) holds signal gid, elements
// 16 tig + i and 64 + 16 tig + i (i < 16) in slots i and 16 + i.
__device__ __forceinline__ void frag128(int t, int i, int& j, int& n) {
  const int lane = t & 31;
  j = lane >> 2;
  n = 16 * (lane & 3) + (i & 15) + 64 * (i >> 4);
}

__device__ __forceinline__ uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ uint32_t half2_bits(float lo, float hi) {
  const half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// (cos, sin)(2 pi m / L), m reduced exactly to (-L/2, L/2] first.  The fast
// hardware sine and cosine are accurate to about 1e-6 on [-pi, pi], far
// below the TF32 / FP16 rounding the values go through.
__device__ __forceinline__ float2 unit_root(int m, int L) {
  m &= L - 1;
  if (2 * m > L) m -= L;
  float s, c;
  __sincosf(6.283185307179586f * float(m) / float(L), &s, &c);
  return make_float2(c, s);
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// B tile of a stage matrix for this lane: rows K = tig (input in0) and
// tig + 4 (input in1), column gid = (output q, re|im = c).  The entry for
// input m and output q is w^(m q) with w = exp(-+ 2 pi i / L), as the real
// 2 x 2 block [[cos, -+sin], [+-sin, cos]] acting on (re, im); ang0/ang1 =
// m q for the two rows.  float2: b[0..1] = rows for the real parts, b[2..3]
// = rows for the imaginary parts; half2: b[0..1] = (re, im) pairs.
template <bool kHalf, bool fwd>
__device__ __forceinline__ void matrix_tile(uint32_t (&b)[4], int ang0, int ang1, int L, int c) {
  const float2 w0 = unit_root(ang0, L), w1 = unit_root(ang1, L);
  // forward: Re_out += cos xr + sin xi, Im_out += -sin xr + cos xi
  const float s0 = fwd ? w0.y : -w0.y, s1 = fwd ? w1.y : -w1.y;
  const float re0 = c ? -s0 : w0.x, im0 = c ? w0.x : s0;   // coefficients of xr, xi (row tig)
  const float re1 = c ? -s1 : w1.x, im1 = c ? w1.x : s1;   // (row tig + 4)
  if constexpr (kHalf) {
    b[0] = half2_bits(re0, im0);
    b[1] = half2_bits(re1, im1);
    b[2] = b[3] = 0u;
  } else {
    b[0] = tf32_bits(re0);
    b[1] = tf32_bits(re1);
    b[2] = tf32_bits(im0);
    b[3] = tf32_bits(im1);
  }
}

// D (+)= [xr | xi] B for data registers a0..a3 (the A fragment positions
// (gid, tig), (gid + 8, tig), (gid, tig + 4), (gid + 8, tig + 4)).
template <typename T>
__device__ __forceinline__ void stage_mma(float (&d)[4], const vec2_t<T>& a0, const vec2_t<T>& a1,
                                          const vec2_t<T>& a2, const vec2_t<T>& a3, const uint32_t (&b)[4]) {
  if constexpr (std::is_same_v<T, half>) {
    mma_f16(d, *reinterpret_cast<const uint32_t*>(&a0), *reinterpret_cast<const uint32_t*>(&a1),
            *reinterpret_cast<const uint32_t*>(&a2), *reinterpret_cast<const uint32_t*>(&a3), b[0], b[1]);
  } else {
    mma_tf32(d, __float_as_uint(a0.x), __float_as_uint(a1.x), __float_as_uint(a2.x), __float_as_uint(a3.x), b[0],
             b[1]);
    mma_tf32(d, __float_as_uint(a0.y), __float_as_uint(a1.y), __float_as_uint(a2.y), __float_as_uint(a3.y), b[2],
             b[3]);
  }
}

template <typename T>
__device__ __forceinline__ vec2_t<T> to_vec2(float re, float im) {
  if constexpr (std::is_same_v<T, half>) return __floats2half2_rn(re, im);
  else return make_float2(re, im);
}

// Exchange area: Y[signal][k1][n_lo] at signal * 68 + k1 * 8 + n_lo (16 * 68
// = (64 + pad_h(64)) * 16, the workspace the API guarantees).
constexpr int kExSig = 68, kExRow = 8;

template <typename T, bool fwd>
__device__ __forceinline__ void run64(vec2_t<T>* reg, vec2_t<T>* ws, int t) {
  constexpr bool kHalf = std::is_same_v<T, half>;
  using V = vec2_t<T>;
  const int lane = t & 31, gid = lane >> 2, tig = lane & 3;

  // stage matrices (per lane; independent of the data, so a caller that
  // repeats the routine keeps them in registers)
  uint32_t bA[2][4], bB[8][2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int k1 = 4 * nt + (gid >> 1);
    matrix_tile<kHalf, fwd>(bA[nt], (2 * tig) * k1, (2 * tig + 1) * k1, 8, gid & 1);
  }
#pragma unroll
  for (int k1 = 0; k1 < 8; ++k1)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int k = k1 + 8 * (2 * (gid >> 1) + nt);
      matrix_tile<kHalf, fwd>(bB[k1][nt], (2 * tig) * k, (2 * tig + 1) * k, 64, gid & 1);
    }

  // stage A: per n_lo, rows = signals gid / gid + 8, K = n_hi 2 tig (reg
  // n_lo) and 2 tig + 1 (reg 8 + n_lo)
  float y[8][2][4];
#pragma unroll
  for (int nl = 0; nl < 8; ++nl)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int q = 0; q < 4; ++q) y[nl][nt][q] = 0.f;
      stage_mma<T>(y[nl][nt], reg[nl], reg[16 + nl], reg[8 + nl], reg[24 + nl], bA[nt]);
    }

  // y[nl][nt] = (re, im) of Y[n_lo = nl][k1 = 4 nt + tig] for signal gid
  // ([0], [1]) and gid + 8 ([2], [3]) -> exchange rows (signal, k1).  The
  // barrier first: the caller may still be reading its workspace.
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      V* row = ws + (gid + 8 * h) * kExSig + (4 * nt + tig) * kExRow;
      if constexpr (kHalf) {
        // 16-byte stores of four n_lo: with rows 68 elements apart the eight
        // lanes of a quarter warp hit eight distinct 16-byte bank groups
        // (8-byte stores collided up to 4-way)
#pragma unroll
        for (int nl = 0; nl < 8; nl += 4) {
          uint32_t u[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) u[e] = half2_bits(y[nl + e][nt][2 * h], y[nl + e][nt][2 * h + 1]);
          *reinterpret_cast<uint4*>(row + nl) = make_uint4(u[0], u[1], u[2], u[3]);
        }
      } else {
#pragma unroll
        for (int nl = 0; nl < 8; nl += 2) {
          const V v0 = to_vec2<T>(y[nl][nt][2 * h], y[nl][nt][2 * h + 1]);
          const V v1 = to_vec2<T>(y[nl + 1][nt][2 * h], y[nl + 1][nt][2 * h + 1]);
          *reinterpret_cast<float4*>(row + nl) = make_float4(v0.x, v0.y, v1.x, v1.y);
        }
      }
    }
  __syncwarp();

  // stage B: per k1, rows = signals, K = n_lo 2 tig / 2 tig + 1
#pragma unroll
  for (int k1 = 0; k1 < 8; ++k1) {
    const V* r0 = ws + gid * kExSig + k1 * kExRow + 2 * tig;
    const V* r1 = r0 + 8 * kExSig;
    V a0, a1, a2, a3;
    if constexpr (kHalf) {
      const uint2 u0 = *reinterpret_cast<const uint2*>(r0), u1 = *reinterpret_cast<const uint2*>(r1);
      a0 = *reinterpret_cast<const half2*>(&u0.x);
      a2 = *reinterpret_cast<const half2*>(&u0.y);
      a1 = *reinterpret_cast<const half2*>(&u1.x);
      a3 = *reinterpret_cast<const half2*>(&u1.y);
    } else {
      const float4 f0 = *reinterpret_cast<const float4*>(r0), f1 = *reinterpret_cast<const float4*>(r1);
      a0 = make_float2(f0.x, f0.y);
      a2 = make_float2(f0.z, f0.w);
      a1 = make_float2(f1.x, f1.y);
      a3 = make_float2(f1.z, f1.w);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      stage_mma<T>(d, a0, a1, a2, a3, bB[k1][nt]);
      reg[8 * nt + k1] = to_vec2<T>(d[0], d[1]);        // element 16 tig + 8 nt + k1, signal gid
      reg[16 + 8 * nt + k1] = to_vec2<T>(d[2], d[3]);   // signal gid + 8
    }
  }
}

// half2 N = 128, 8 signals per warp (frag128).  A radix-2 decimation-in-
// frequency step in registers,
//   a[n] = x[n] + x[n + 64],  b[n] = (x[n] - x[n + 64]) w_128^n   (n < 64),
// turns the lane's two chunks of signal gid into rows gid (a) and gid + 8 (b)
// of the 64-point routine, whose outputs are A[k] = X[2k] and B[k] =
// X[2k + 1].  One shared-memory pass then puts X back in frag128 order, so
// the output order equals the input order.
constexpr int kEx128Sig = 136;   // 8 * 136 = (128 + pad_h(128)) * 8
__host__ __device__ constexpr int ex128_pos(int k) { return k ^ (((k >> 5) & 1) << 2); }

// (cos, sin)(2 pi i / 128) for i < 16, as compile-time constants
// (sin(x) = cos(pi/2 - x) with a short Taylor series in double).
__host__ __device__ constexpr double taylor_cos(double x) {
  double term = 1.0, sum = 1.0;
  for (int k = 1; k < 12; ++k) {
    term *= -x * x / double((2 * k - 1) * (2 * k));
    sum += term;
  }
  return sum;
}
template <int I>
struct Root128 {
  static constexpr double x = 6.283185307179586476925 * I / 128.0;
  static constexpr float c = float(taylor_cos(x)), s = float(taylor_cos(1.5707963267948966192 - x));
};

template <bool fwd, int... I>
__device__ __forceinline__ void radix2_dif128(half2* reg, float2 wt, std::integer_sequence<int, I...>) {
  // twiddle w_128^(16 tig + i) = w_8^tig * w_128^i: one per-lane root times a
  // compile-time constant; applied as a packed complex multiply,
  // (dr, di) * (wr, wi) = (dr, di) * (wr, wr) + (di, dr) * (-wi, wi)
  (
      [&] {
        constexpr float ci = Root128<I>::c, si = fwd ? -Root128<I>::s : Root128<I>::s;
        const float wr = wt.x * ci - wt.y * si, wi = wt.x * si + wt.y * ci;
        const half2 wrr = __floats2half2_rn(wr, wr), wii = __floats2half2_rn(-wi, wi);
        const half2 x0 = reg[I], x1 = reg[16 + I];
        const half2 d = __hsub2(x0, x1);
        reg[I] = __hadd2(x0, x1);
        reg[16 + I] = __hfma2(__lowhigh2highlow(d), wii, __hmul2(d, wrr));
      }(),
      ...);
}

template <bool fwd>
__device__ __forceinline__ void run128(half2* reg, half2* ws, int t) {
  const int lane = t & 31, gid = lane >> 2, tig = lane & 3;
  {
    const float2 w8 = unit_root(16 * tig, 128);
    radix2_dif128<fwd>(reg, make_float2(w8.x, fwd ? -w8.y : w8.y), std::make_integer_sequence<int, 16>{});
  }
  run64<half, fwd>(reg, ws, t);
  // reg[i] = X[2k'], reg[16 + i] = X[2k' + 1], k' = 16 tig + i -> frag128
  __syncwarp();
  half2* row = ws + gid * kEx128Sig;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int k = 2 * (16 * tig + i);
    *reinterpret_cast<uint2*>(row + ex128_pos(k)) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&reg[i]), *reinterpret_cast<const uint32_t*>(&reg[16 + i]));
  }
  __syncwarp();
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 q = *reinterpret_cast<const uint4*>(row + ex128_pos(64 * h + 16 * tig + 4 * v));
      reg[16 * h + 4 * v + 0] = *reinterpret_cast<const half2*>(&q.x);
      reg[16 * h + 4 * v + 1] = *reinterpret_cast<const half2*>(&q.y);
      reg[16 * h + 4 * v + 2] = *reinterpret_cast<const half2*>(&q.z);
      reg[16 * h + 4 * v + 3] = *reinterpret_cast<const half2*>(&q.w);
    }
}

}  // namespace mfft
}  // namespace detail
}  // namespace thunderfft
