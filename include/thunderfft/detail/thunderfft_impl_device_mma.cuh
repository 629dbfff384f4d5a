// thunderfft_impl_device_mma.cuh — warp-MMA form of ThunderFFT_kernel_reg for
// half2 N = 64, where the register FFT's packed-FP16 passes lag the
// reference's warp-MMA routine (detail/kernel/shared_kernel_n64_b16.cuh).
//
// N = NH * NL, n = n_lo + NL * n_hi, k = k1 + NH * k2:
//
//   stage A (mma.sync)  Y[n_lo][k1]       = sum_{n_hi} x[n_lo + NL n_hi] w_NH^(n_hi k1)
//   twiddle (FP32)      Y'[n_lo][k1]      = Y[n_lo][k1] * w_N^(n_lo k1)
//   stage B (mma.sync)  X[k1 + NH k2]     = sum_{n_lo} Y'[n_lo][k1] w_NL^(n_lo k2)
//
// Each stage is a real matrix product D = A * B per signal: A is the stage's
// DFT matrix with rows (output, re|im) in 16-row tiles [8 re | 8 im], B the
// data with K = the contracted index and columns = the other index.
//   * float2: mma.m16n8k8 .tf32, one K step for the real parts of 8 inputs
//     and one for the imaginary parts;
//   * half2:  mma.m16n8k16 .f16 (FP32 accumulation), K = 8 inputs with
//     (re, im) interleaved, so a B register is one half2 element.
// Stage A's accumulator leaves lane (gid, tig) with n_lo = 8nt + 2tig and
// 8nt + 2tig + 1 of output k1 = 8mt + gid.  Stage B takes those registers as
// its B operand unchanged: its K index kappa = tig stands for n_lo = 2tig and
// kappa = tig + 4 for 2tig + 1 (stage_b_input), which only reorders the
// columns of the constant stage-B matrix.  Data therefore crosses shared
// memory twice per call: fragment -> natural-order staging (read by stage A)
// and stage-B outputs -> staging -> fragment.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "util_arith.h"

namespace thunderfft {
namespace detail {
namespace mfft {

template <int N>
struct shape;
template <>
struct shape<64> {
  static constexpr int NH = 8, NL = 8;
};

// Used for half2 N = 64: 0.86 us per call of the paper benchmark (16384
// signals) against 1.02 us for the packed-FP16 register FFT.  The float2 form
// (mma.m16n8k8 .tf32) computes correctly (rel-L2 7.7e-4) but took 1.51 us
// against 1.24 us for the FP32 register FFT, which is also exact to 1e-7, so
// float2 keeps that.
template <typename T, int N>
inline constexpr bool enabled = std::is_same_v<T, half> && N == 64;

// Staging position of element n of a signal.  Bit 4 of n flips bit 2: the
// stage-A operand loads of a half warp (n = gid + 8 tig, gid < 4) and the
// stage-B pair stores (n = 2 tig + 8 gid) then touch 16 distinct 8-byte bank
// pairs; consecutive n stay a permutation of one 16-element run.
__host__ __device__ constexpr int stage_pos(int n) { return n ^ (((n >> 4) & 1) << 2); }

// Stage-B K index -> the n_lo it stands for (see the file comment).
__host__ __device__ constexpr int stage_b_input(int kappa) {
  return 8 * (kappa / 8) + 2 * (kappa % 4) + (kappa % 8) / 4;
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
// below the TF32 / FP16 rounding the values go through; the accurate library
// routines cost several times the MMA work of a whole call here.
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

// One 16 x (8 complex inputs) tile of a stage DFT matrix of length L, for
// outputs o = 8 mt + gid and inputs in(kappa), kappa = 8 kb + tig, + 4.
// Forward (w = exp(-i theta)): Re += c xr + s xi, Im += -s xr + c xi.
// float2: r[0..3] multiplies the real parts, r[4..7] the imaginary parts
// (a0..a3 order: (gid, tig), (gid+8, tig), (gid, tig+4), (gid+8, tig+4)).
// half2: r[0..3] = a0..a3 of the interleaved K = (kappa, re|im).
template <bool kHalf, int L, bool fwd, bool kStageB>
__device__ __forceinline__ void matrix_tile(uint32_t (&r)[8], int mt, int kb, int gid, int tig) {
  const int o = 8 * mt + gid;
  const int k0 = 8 * kb + tig, k1 = k0 + 4;
  const int i0 = kStageB ? stage_b_input(k0) : k0, i1 = kStageB ? stage_b_input(k1) : k1;
  const float2 w0 = unit_root(o * i0, L), w1 = unit_root(o * i1, L);
  const float s0 = fwd ? w0.y : -w0.y, s1 = fwd ? w1.y : -w1.y;
  if constexpr (kHalf) {
    r[0] = half2_bits(w0.x, s0);
    r[1] = half2_bits(-s0, w0.x);
    r[2] = half2_bits(w1.x, s1);
    r[3] = half2_bits(-s1, w1.x);
  } else {
    r[0] = tf32_bits(w0.x);
    r[1] = tf32_bits(-s0);
    r[2] = tf32_bits(w1.x);
    r[3] = tf32_bits(-s1);
    r[4] = tf32_bits(s0);
    r[5] = tf32_bits(w0.x);
    r[6] = tf32_bits(s1);
    r[7] = tf32_bits(w1.x);
  }
}

template <bool kHalf>
__device__ __forceinline__ void mma_tile(float (&d)[4], const uint32_t (&a)[8], uint32_t b0re, uint32_t b1re,
                                         uint32_t b0im, uint32_t b1im) {
  if constexpr (kHalf) {
    mma_f16(d, a[0], a[1], a[2], a[3], b0re, b1re);   // b0re/b1re hold whole half2 elements
  } else {
    mma_tf32(d, a[0], a[1], a[2], a[3], b0re, b1re);
    mma_tf32(d, a[4], a[5], a[6], a[7], b0im, b1im);
  }
}

// The FFT of the block's tile.  reg: the fragment (element t + P i of the
// tile), ws: at least N * B elements of shared memory.
template <typename T, int N, int B, int EPT, int P, bool fwd>
__device__ __forceinline__ void run(vec2_t<T>* reg, vec2_t<T>* ws, int t) {
  constexpr bool kHalf = std::is_same_v<T, half>;
  using S = shape<N>;
  constexpr int NH = S::NH, NL = S::NL;
  constexpr int MTA = NH / 8, NTA = NL / 8, KBA = NH / 8;   // stage A tiles: k1, n_lo, n_hi
  constexpr int MTB = NL / 8, NTB = NH / 8, KBB = NL / 8;   // stage B tiles: k2, k1, n_lo
  constexpr int W = P / 32, SPW = B / W;                    // warps, signals per warp
  static_assert(SPW * W == B, "signals must split evenly over the warps");
  const int lane = t & 31, warp = t >> 5;
  const int gid = lane >> 2, tig = lane & 3;

  // fragment -> natural-order staging.  Element t + P i of the tile is
  // element t + P (i % (N/P)) of signal i / (N/P) (t < P, N % P == 0), and
  // stage_pos only permutes bits 2 and 4, so its position is a per-thread base
  // plus a compile-time offset.
  static_assert(N % P == 0, "a block's threads cover whole signals");
  constexpr int SPS = N / P;   // fragment slots per signal
  vec2_t<T>* const frag_base = ws + stage_pos(t);
#pragma unroll
  for (int i = 0; i < EPT; ++i) frag_base[(i / SPS) * N + P * (i % SPS)] = reg[i];

  // per-lane constants: stage matrices and twiddles
  uint32_t aA[MTA][KBA][8], aB[MTB][KBB][8];
#pragma unroll
  for (int mt = 0; mt < MTA; ++mt)
#pragma unroll
    for (int kb = 0; kb < KBA; ++kb) matrix_tile<kHalf, NH, fwd, false>(aA[mt][kb], mt, kb, gid, tig);
#pragma unroll
  for (int mt = 0; mt < MTB; ++mt)
#pragma unroll
    for (int kb = 0; kb < KBB; ++kb) matrix_tile<kHalf, NL, fwd, true>(aB[mt][kb], mt, kb, gid, tig);
  float2 tw[MTA][NTA][2];
#pragma unroll
  for (int mt = 0; mt < MTA; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 w = unit_root((8 * nt + 2 * tig + h) * (8 * mt + gid), N);
        tw[mt][nt][h] = make_float2(w.x, fwd ? -w.y : w.y);
      }
  __syncthreads();

  // Signals go through in groups of G, each phase interleaved over the
  // group: one signal's chain (loads, 2 dependent MMA stages, stores) is
  // latency-bound, and a block has few warps.
  constexpr int G = SPW < 4 ? SPW : 4;
  static_assert(SPW % G == 0, "signal groups");
#pragma unroll 1
  for (int j0 = 0; j0 < SPW; j0 += G) {
    vec2_t<T>* x0 = ws + (warp * SPW + j0) * N;
    // stage A operands of the group
    uint32_t bre[G][NTA][KBA][2], bim[G][NTA][KBA][2];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
        for (int kb = 0; kb < KBA; ++kb) {
          const int n0 = (8 * nt + gid) + NL * (8 * kb + tig), n1 = n0 + 4 * NL;
          const vec2_t<T> e0 = x0[g * N + stage_pos(n0)], e1 = x0[g * N + stage_pos(n1)];
          if constexpr (kHalf) {
            bre[g][nt][kb][0] = *reinterpret_cast<const uint32_t*>(&e0);
            bre[g][nt][kb][1] = *reinterpret_cast<const uint32_t*>(&e1);
            bim[g][nt][kb][0] = bim[g][nt][kb][1] = 0u;
          } else {
            bre[g][nt][kb][0] = __float_as_uint(e0.x);
            bre[g][nt][kb][1] = __float_as_uint(e1.x);
            bim[g][nt][kb][0] = __float_as_uint(e0.y);
            bim[g][nt][kb][1] = __float_as_uint(e1.y);
          }
        }
    // stage A
    float acc[G][MTA][NTA][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int mt = 0; mt < MTA; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTA; ++nt) {
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[g][mt][nt][q] = 0.f;
#pragma unroll
          for (int kb = 0; kb < KBA; ++kb)
            mma_tile<kHalf>(acc[g][mt][nt], aA[mt][kb], bre[g][nt][kb][0], bre[g][nt][kb][1], bim[g][nt][kb][0],
                            bim[g][nt][kb][1]);
        }
    // twiddle, then stage B with the accumulator registers as its operand
    float out[G][MTB][NTB][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int mb = 0; mb < MTB; ++mb)
#pragma unroll
        for (int nb = 0; nb < NTB; ++nb)
#pragma unroll
          for (int q = 0; q < 4; ++q) out[g][mb][nb][q] = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int nb = 0; nb < NTB; ++nb)      // k1 tile = stage-A m tile
#pragma unroll
        for (int kb = 0; kb < KBB; ++kb) {  // n_lo tile = stage-A n tile
          const float* c = acc[g][nb][kb];
          const float2 w0 = tw[nb][kb][0], w1 = tw[nb][kb][1];
          const float y0r = fmaf(c[0], w0.x, -c[2] * w0.y), y0i = fmaf(c[0], w0.y, c[2] * w0.x);
          const float y1r = fmaf(c[1], w1.x, -c[3] * w1.y), y1i = fmaf(c[1], w1.y, c[3] * w1.x);
          uint32_t b0re, b1re, b0im = 0, b1im = 0;
          if constexpr (kHalf) {
            b0re = half2_bits(y0r, y0i);
            b1re = half2_bits(y1r, y1i);
          } else {
            b0re = __float_as_uint(y0r);
            b1re = __float_as_uint(y1r);
            b0im = __float_as_uint(y0i);
            b1im = __float_as_uint(y1i);
          }
#pragma unroll
          for (int mb = 0; mb < MTB; ++mb) mma_tile<kHalf>(out[g][mb][nb], aB[mb][kb], b0re, b1re, b0im, b1im);
        }
    // out[g][mb][nb]: X[k1 = 8nb + 2tig + {0,1}][k2 = 8mb + gid]; k = k1 + NH k2
    // (in place: the group's stage-A operands were all read above, and
    // every lane's reads precede the MMAs that consume them)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int mb = 0; mb < MTB; ++mb)
#pragma unroll
        for (int nb = 0; nb < NTB; ++nb) {
          const int k = (8 * nb + 2 * tig) + NH * (8 * mb + gid);
          const float* o = out[g][mb][nb];
          if constexpr (kHalf) {
            const uint2 v = make_uint2(half2_bits(o[0], o[2]), half2_bits(o[1], o[3]));
            *reinterpret_cast<uint2*>(x0 + g * N + stage_pos(k)) = v;
          } else {
            *reinterpret_cast<float4*>(x0 + g * N + stage_pos(k)) = make_float4(o[0], o[2], o[1], o[3]);
          }
        }
  }
  __syncthreads();

  // staging -> fragment
#pragma unroll
  for (int i = 0; i < EPT; ++i) reg[i] = frag_base[(i / SPS) * N + P * (i % SPS)];
}

}  // namespace mfft
}  // namespace detail
}  // namespace thunderfft
