// thunderfft_impl_device_mma.cuh — the warp-MMA forms of ThunderFFT_kernel_reg
// (the reference computes its device routine with warp MMAs too:
// detail/kernel/unit_kernel_fp32.cuh, unit_kernel_fp16.cuh), each written for
// this library's own operand maps:
//   * half2 N = 64 (16 signals, one warp) as two FP16 MMA DFT stages (run64);
//   * float2 N = 64, 128, 256 with one TF32 MMA stage (radix 4, 8, 4) and
//     in-lane FP32 DFTs (run64_tf32, run128_tf32, run256_tf32, at the end);
//     half2 N = 128 runs run128_tf32 on FP32 copies of its registers (half2
//     values are exact in TF32): 1.56 us per paper-benchmark call against
//     1.97 us for a radix-2 step on top of run64, at rel-L2 2.4e-4.
// The run64 template's float2 branches are not used (run64_tf32 serves
// float2 N = 64).
//
// half2 N = 64:
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

// The two-stage warp-MMA routine serves half2 N = 64 with the API's 16
// signals per block: 0.49 us per paper-benchmark call (16384 signals) against
// 1.02 us for the packed-FP16 register FFT.  Its float2 form (mma.m16n8k8
// .tf32, 64 MMAs and a shared-memory exchange per call) measured 1.24 us;
// run64_tf32 (16 MMAs, no exchange) takes 0.48 us.
template <typename T, int N, int batch>
inline constexpr bool enabled = std::is_same_v<T, half> && N == 64 && batch == 16;

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

// ---------------------------------------------------------------------------
// float2 N = 64, 16 signals per warp, TF32 warp MMAs (the reference's float
// contract: TF32 MMA arithmetic, shared_kernel_n64_b16.cuh).
//
// With n = n1 + 16 n2 and k = 4 k1 + k2 (n1, k1 < 16; n2, k2 < 4):
//   X[4 k1 + k2] = sum_{n1} w_16^(n1 k1) Y[n1][k2],
//   Y[n1][k2]    = sum_{n2} x[n1 + 16 n2] w_64^((n1 + 16 n2) k2).
// Input fragment: frag64 (lane (gid, tig) holds n2 = tig, register i holds
// n1 = i % 16, signals gid and gid + 8).
//   * Y: one mma.m16n8k8 .tf32 per n1: rows = the 16 signals, K = (re | im of
//     input n2 = tig), columns = (k2, re | im); the twiddle is in the B
//     matrix, so lane tig receives Y[n1][k2 = tig] for every n1.  No data
//     moves between lanes.
//   * X: the lane's 16-point DFT over n1 (its own k2), radix 4 x 4 in FP32
//     registers with compile-time roots.
// Output fragment (frag64_tf32_out): lane (gid, tig), register i holds
// X[4 (i % 16) + tig] of signal gid + 8 (i / 16).  The inverse runs the same
// way with conjugate roots, unnormalized.
template <typename T, int N, int batch>
inline constexpr bool tf32_enabled =
    (std::is_same_v<T, float> && ((N == 64 && batch == 16) || (N == 128 && batch == 8) || (N == 256 && batch == 16))) ||
    (std::is_same_v<T, half> && N == 128 && batch == 8);
// routines whose output fragment order differs from the input order
template <typename T, int N, int batch>
inline constexpr bool split_order = tf32_enabled<T, N, batch>;

// half2 N = 256 (16 signals, 4 warps): two radix-16 passes in packed FP16
// (dfft::run256_h).  Thread t = 16 p + q holds elements q + 16 i' of
// signals 2p (registers 0-15) and 2p + 1 (registers 16-31), input and
// output alike.
template <typename T, int N, int batch>
inline constexpr bool h256_enabled = std::is_same_v<T, half> && N == 256 && batch == 16;
__device__ __forceinline__ void frag256_h(int t, int i, int& j, int& n) {
  j = 2 * (t >> 4) + (i >> 4);
  n = (t & 15) + 16 * (i & 15);
}

__device__ __forceinline__ void frag64_tf32_out(int t, int i, int& j, int& k) {
  const int lane = t & 31;
  j = (lane >> 2) + 8 * (i >> 4);
  k = (lane & 3) + 4 * (i & 15);
}
// N = 128 (8 signals): input frag128; output: lane (gid, tig), register i
// holds X[8 (i % 16) + 4 (i / 16) + tig] of signal gid.
__device__ __forceinline__ void frag128_tf32_out(int t, int i, int& j, int& k) {
  const int lane = t & 31;
  j = lane >> 2;
  k = 8 * (i & 15) + 4 * (i >> 4) + (lane & 3);
}
// N = 256 (16 signals, 4 warps): warp w, lane (gid, tig), register i holds
// signal gid + 8 (i / 16): input element 16 w + i % 16 + 64 tig, output
// element 16 (i % 16) + 4 tig + w.
__device__ __forceinline__ void frag256_tf32_in(int t, int i, int& j, int& n) {
  const int lane = t & 31, w = t >> 5;
  j = (lane >> 2) + 8 * (i >> 4);
  n = 16 * w + (i & 15) + 64 * (lane & 3);
}
__device__ __forceinline__ void frag256_tf32_out(int t, int i, int& j, int& k) {
  const int lane = t & 31, w = t >> 5;
  j = (lane >> 2) + 8 * (i >> 4);
  k = 16 * (i & 15) + 4 * (lane & 3) + w;
}

// x * w_16^M (forward; conjugate root for the inverse), M a compile-time
// exponent: 0, 4, 8, 12 need no multiply.
template <int M, bool fwd>
__device__ __forceinline__ float2 rot16(float2 x) {
  constexpr int m = M & 15;
  if constexpr (m == 0) {
    return x;
  } else if constexpr (m == 8) {
    return make_float2(-x.x, -x.y);
  } else if constexpr (m == 4 || m == 12) {
    // w_16^4 = -i (forward), +i (inverse); w_16^12 the opposite
    constexpr bool minus_i = (m == 4) == fwd;
    return minus_i ? make_float2(x.y, -x.x) : make_float2(-x.y, x.x);
  } else {
    constexpr float c = Root128<8 * m>::c, s = fwd ? -Root128<8 * m>::s : Root128<8 * m>::s;
    return make_float2(x.x * c - x.y * s, x.x * s + x.y * c);
  }
}

// 4-point DFT in place: (u0, u1, u2, u3) -> (U0, U1, U2, U3).
template <bool fwd>
__device__ __forceinline__ void dft4(float2& u0, float2& u1, float2& u2, float2& u3) {
  const float2 s0 = make_float2(u0.x + u2.x, u0.y + u2.y), d0 = make_float2(u0.x - u2.x, u0.y - u2.y);
  const float2 s1 = make_float2(u1.x + u3.x, u1.y + u3.y), d1 = make_float2(u1.x - u3.x, u1.y - u3.y);
  u0 = make_float2(s0.x + s1.x, s0.y + s1.y);
  u2 = make_float2(s0.x - s1.x, s0.y - s1.y);
  // U1 = d0 + w_4 d1, U3 = d0 - w_4 d1 with w_4 = -i (forward) or +i
  const float2 wd = fwd ? make_float2(d1.y, -d1.x) : make_float2(-d1.y, d1.x);
  u1 = make_float2(d0.x + wd.x, d0.y + wd.y);
  u3 = make_float2(d0.x - wd.x, d0.y - wd.y);
}

// 16-point DFT of v[0..15] (natural order in and out), radix 4 x 4:
// n = a + 4 b, k = c + 4 d:  X[c + 4d] = sum_a w_4^(a d) w_16^(a c) sum_b v[a + 4b] w_4^(b c).
template <bool fwd, int... A>
__device__ __forceinline__ void twiddle16(float2 (&v)[16], std::integer_sequence<int, A...>) {
  // v[a + 4c] *= w_16^(a c)
  ((v[(A & 3) + 4 * (A >> 2)] = rot16<(A & 3) * (A >> 2), fwd>(v[(A & 3) + 4 * (A >> 2)])), ...);
}
template <bool fwd>
__device__ __forceinline__ void dft16(float2 (&v)[16]) {
#pragma unroll
  for (int a = 0; a < 4; ++a) dft4<fwd>(v[a], v[a + 4], v[a + 8], v[a + 12]);   // v[a + 4c] = T[a][c]
  twiddle16<fwd>(v, std::make_integer_sequence<int, 16>{});
#pragma unroll
  for (int c = 0; c < 4; ++c) dft4<fwd>(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);   // v[4c + d] = X[c + 4d]
  float2 o[16];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int d = 0; d < 4; ++d) o[c + 4 * d] = v[4 * c + d];
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = o[k];
}

__device__ __forceinline__ float2 cmulf(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
// B fragment (rows tig: re, tig + 4: im of the lane's input; column: the
// lane's output, re | im = plane) of the coefficient c.
__device__ __forceinline__ void b_frag(uint32_t& b0, uint32_t& b1, float2 c, int plane) {
  b0 = tf32_bits(plane ? c.y : c.x);
  b1 = tf32_bits(plane ? c.x : -c.y);
}
// exp(-+ 2 pi i m / L) (forward: minus)
template <bool fwd>
__device__ __forceinline__ float2 root(int m, int L) {
  const float2 w = unit_root(m, L);
  return make_float2(w.x, fwd ? -w.y : w.y);
}

template <bool fwd>
__device__ __forceinline__ void run64_tf32(float2* reg, int t) {
  const int lane = t & 31, gid = lane >> 2, tig = lane & 3;
  const int k2 = gid >> 1, plane = gid & 1;   // this lane's B column: output k2, re | im
  // B rows tig (re of input n2 = tig) and tig + 4 (im), column gid: the
  // coefficient c(n1) = w_64^((n1 + 16 tig) k2) = w_4^(tig k2) w_64^(k2)^n1,
  // stepped by one complex multiply per n1
  const float2 q = root<fwd>(k2, 64);
  float2 c = root<fwd>(16 * tig * k2, 64);
#pragma unroll
  for (int n1 = 0; n1 < 16; ++n1) {
    uint32_t b0, b1;
    b_frag(b0, b1, c, plane);
    c = cmulf(c, q);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    // A: (signal gid | gid + 8) x (re | im of input n2 = tig); the tensor
    // core reads the TF32 part of each fp32 value
    mma_tf32(d, __float_as_uint(reg[n1].x), __float_as_uint(reg[16 + n1].x), __float_as_uint(reg[n1].y),
             __float_as_uint(reg[16 + n1].y), b0, b1);
    reg[n1] = make_float2(d[0], d[1]);        // Y[n1][k2 = tig], signal gid (in place)
    reg[16 + n1] = make_float2(d[2], d[3]);   // signal gid + 8
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float2 y[16];
#pragma unroll
    for (int n1 = 0; n1 < 16; ++n1) y[n1] = reg[16 * h + n1];
    dft16<fwd>(y);
#pragma unroll
    for (int k1 = 0; k1 < 16; ++k1) reg[16 * h + k1] = y[k1];   // X[4 k1 + tig]
  }
}

// float2 N = 128, 8 signals per warp, one radix-8 MMA stage.  With
// n = n1 + 16 n2 and k = 8 k1 + k2 (n1, k1 < 16; n2, k2 < 8):
//   Y[n1][k2]    = sum_{n2} x[n1 + 16 n2] w_128^((n1 + 16 n2) k2),
//   X[8 k1 + k2] = sum_{n1} w_16^(n1 k1) Y[n1][k2].
// frag128 gives the lane n2 = tig (register i) and n2 = tig + 4 (register
// 16 + i), n1 = i % 16, of signal gid.  Per m < 8, four mma.m16n8k8 (two K
// steps: n2 < 4, n2 >= 4; two N tiles: k2 < 4, k2 >= 4) with rows (signal
// gid, n1 = m) and (signal gid, n1 = m + 8); the B matrix holds the
// twiddle of n1 = m, so the second row half is multiplied by w_128^(8 k2) =
// w_16^k2 afterwards (k2 = 4 tile + tig, a per-lane root).  The lane then
// holds all 16 n1 of k2 = tig and tig + 4 and runs two 16-point DFTs.
// Output (frag128_tf32_out): register i holds X[8 (i % 16) + 4 (i / 16) + tig].
template <bool fwd>
__device__ __forceinline__ void run128_tf32(float2* reg, int t) {
  const int lane = t & 31, gid = lane >> 2, tig = lane & 3;
  const int kb = gid >> 1, plane = gid & 1;   // this lane's B column within an N tile
  // second row half's factor w_16^(4 tile + tig), one per N tile
  const float2 post0 = root<fwd>(tig, 16), post1 = root<fwd>(4 + tig, 16);
  // coefficients c(ks, nt, m) = w_128^((m + 16 (4 ks + tig)) (4 nt + kb)),
  // stepped in m by q(nt) = w_128^(4 nt + kb)
  const float2 q0 = root<fwd>(kb, 128), q1 = root<fwd>(4 + kb, 128);
  float2 c00 = root<fwd>(16 * tig * kb, 128), c01 = root<fwd>(16 * tig * (4 + kb), 128);
  float2 c10 = root<fwd>(16 * (4 + tig) * kb, 128), c11 = root<fwd>(16 * (4 + tig) * (4 + kb), 128);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    // inputs n1 = m, m + 8 for n2 = tig (ks 0) and tig + 4 (ks 1)
    const float2 x0 = reg[m], x0h = reg[m + 8], x1 = reg[16 + m], x1h = reg[24 + m];
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t b0, b1;
    b_frag(b0, b1, c00, plane);
    mma_tf32(d0, __float_as_uint(x0.x), __float_as_uint(x0h.x), __float_as_uint(x0.y), __float_as_uint(x0h.y), b0, b1);
    b_frag(b0, b1, c10, plane);
    mma_tf32(d0, __float_as_uint(x1.x), __float_as_uint(x1h.x), __float_as_uint(x1.y), __float_as_uint(x1h.y), b0, b1);
    b_frag(b0, b1, c01, plane);
    mma_tf32(d1, __float_as_uint(x0.x), __float_as_uint(x0h.x), __float_as_uint(x0.y), __float_as_uint(x0h.y), b0, b1);
    b_frag(b0, b1, c11, plane);
    mma_tf32(d1, __float_as_uint(x1.x), __float_as_uint(x1h.x), __float_as_uint(x1.y), __float_as_uint(x1h.y), b0, b1);
    c00 = cmulf(c00, q0); c10 = cmulf(c10, q0); c01 = cmulf(c01, q1); c11 = cmulf(c11, q1);
    // in place: N tile 0 (k2 = tig) -> registers 0..15, tile 1 (k2 = 4 + tig) -> 16..31
    reg[m] = make_float2(d0[0], d0[1]);
    reg[m + 8] = cmulf(make_float2(d0[2], d0[3]), post0);
    reg[16 + m] = make_float2(d1[0], d1[1]);
    reg[24 + m] = cmulf(make_float2(d1[2], d1[3]), post1);
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    float2 y[16];
#pragma unroll
    for (int n1 = 0; n1 < 16; ++n1) y[n1] = reg[16 * nt + n1];
    dft16<fwd>(y);
#pragma unroll
    for (int k1 = 0; k1 < 16; ++k1) reg[16 * nt + k1] = y[k1];   // X[8 k1 + 4 nt + tig]
  }
}

// float2 N = 256, 16 signals, 4 warps.  With n = n1 + 64 n2, k = 4 k1 + k2:
//   Y[n1][k2] = sum_{n2} x[n1 + 64 n2] w_256^((n1 + 64 n2) k2)   (one TF32 MMA per n1)
//   X[4 k1 + k2] = sum_{n1} w_64^(n1 k1) Y[n1][k2]                 (64-point routine)
// Warp w holds n1 = 16 w + i % 16 for n2 = tig (frag256_tf32_in), computes
// its Y, and one exchange through the workspace gives warp w all n1 of
// k2 = w in the 64-point routine's input order.  Exchange position of
// (signal j, k2, n1): ((64 k2 + n1) 16 + j) with its low bit 3 flipped by
// bit 0 of (k2 ^ n1 / 16): the stores (k2 = tig) and the loads (n1 / 16 =
// tig) of one instruction then fill 16 distinct 8-byte bank pairs twice,
// the minimum of two wavefronts.
__device__ __forceinline__ int ex256_pos(int j, int k2, int n1) {
  return (((64 * k2 + n1) << 4) + j) ^ ((((k2 ^ (n1 >> 4)) & 1)) << 3);
}

template <bool fwd>
__device__ __forceinline__ void run256_tf32(float2* reg, float2* ws, int t) {
  const int lane = t & 31, gid = lane >> 2, tig = lane & 3, w = t >> 5;
  const int k2 = gid >> 1, plane = gid & 1;   // this lane's B column
  // c(m) = w_256^((16 w + m + 64 tig) k2), stepped in m by w_256^k2
  const float2 q = root<fwd>(k2, 256);
  float2 c = root<fwd>((16 * w + 64 * tig) * k2, 256);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    uint32_t b0, b1;
    b_frag(b0, b1, c, plane);
    c = cmulf(c, q);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_tf32(d, __float_as_uint(reg[m].x), __float_as_uint(reg[16 + m].x), __float_as_uint(reg[m].y),
             __float_as_uint(reg[16 + m].y), b0, b1);
    reg[m] = make_float2(d[0], d[1]);        // Y[n1 = 16 w + m][k2 = tig], signal gid
    reg[16 + m] = make_float2(d[2], d[3]);   // signal gid + 8
  }
  __syncthreads();   // the caller may still be reading its workspace
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int m = 0; m < 16; ++m) ws[ex256_pos(gid + 8 * h, tig, 16 * w + m)] = reg[16 * h + m];
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int i = 0; i < 16; ++i) reg[16 * h + i] = ws[ex256_pos(gid + 8 * h, w, 16 * tig + i)];
  run64_tf32<fwd>(reg, t);
}

}  // namespace mfft
}  // namespace detail
}  // namespace thunderfft
