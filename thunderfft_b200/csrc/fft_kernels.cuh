// fft_kernels.cuh — batched C2C FFT kernels for sm_100a (tcgen05 + TMA).
//
// Two kernel families compute the same transform as the reference's
// ThunderFFT_global_kernel (include/thunderfft/detail/kernel/global_kernel.cuh:21-100):
//
//  * fft2_kernel  — N = Ns * Na in two tensor-core stages.
//      x[n], n = a + Na*s  (a: contiguous index, s: strided index).
//      stage 1 (DFT over s, length Ns):  Y[a][ks] = sum_s x[a + Na s] w_Ns^(s ks)
//      twiddle:                         Y'[a][ks] = Y[a][ks] * w_N^(a ks)
//      stage 2 (DFT over a, length Na):  X[Ns ka + ks] = sum_a Y'[a][ks] w_Na^(a ka)
//    Each stage is one UMMA D = A x B with
//      A = the real-valued stage DFT matrix, rows (ks, re|im) in 16-row blocks
//          [8 rows cos | 8 rows sin], columns = the stage's input index,
//          K-major, no swizzle, resident in shared memory for the whole kernel;
//          G independent signal groups share one MMA through a block-diagonal
//          A (K = G*L rows of B, M = 2*G*L rows of A);
//      B = the data, MN-major: K rows = stage input index, N columns =
//          (signal, other index, re|im).  Stage-1 B is the natural input
//          layout brought in by one TMA box per tile; stage-2 B is written by
//          the stage-1 epilogue.
//    A 16x256b TMEM load then hands each thread, for one (ks, a) pair, the
//    four partial sums cos*re, cos*im, sin*re, sin*im of the same output, so
//    the complex combine, the twiddle and the re/im interleave stay in
//    registers (no shuffles).
//
//  * dft1_kernel  — N = 64: one stage with the data as the K-major A operand
//    (rows = signals, K = 2N interleaved re/im) and the real 2N x 2N DFT
//    matrix as B; TMEM rows are then whole output signals, staged to shared
//    memory and written back by TMA.
//
// Roles (persistent CTA, one per SM): warp 0 loads tiles (TMA, or masked
// thread loads for a partial/unaligned tile), warp 1 allocates TMEM and
// issues MMAs from one thread, the remaining warps are epilogues.  All
// hand-offs are mbarriers; every wait is bounded (sm100.cuh) so a stall turns
// into an error code instead of a hung GPU.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"
#include "epi_addr.cuh"

namespace thff {

// Every kernel here is persistent (one CTA per SM) and allocates all 512 TMEM
// columns.  A second CTA resident on the same SM would block in tcgen05.alloc
// until the first exits, leaving other SMs idle, so each launch requests at
// least this much dynamic shared memory: more than half of an SM's 228 KB
// makes a second resident CTA impossible regardless of register use.
constexpr uint32_t kExclusiveSmemBytes = 120u * 1024u;
__host__ __device__ constexpr uint32_t exclusive_smem(uint32_t bytes) {
  return bytes > kExclusiveSmemBytes ? bytes : kExclusiveSmemBytes;
}

// ---------------------------------------------------------------------------
// Storage/arithmetic traits: float2 storage -> kind::tf32; half2 -> kind::f16.
// ---------------------------------------------------------------------------
template <bool kHalf>
struct DType;

template <>
struct DType<false> {
  static constexpr int kEsz = 4;                 // bytes per real
  static constexpr int kElemsPer128B = 32;
  static constexpr int kMmaK = 8;                // K per tcgen05.mma
  static constexpr uint32_t kFmt = sm100::kFmtTF32;
  // MN-major tf32 operands: 128-B rows, 32-B swizzle atoms, 4 rows per group.
  static constexpr uint32_t kBSwizzle = 1;       // SWIZZLE_128B_BASE32B
  static constexpr uint32_t kBSbo = 512;
  __host__ __device__ static constexpr uint32_t swz(uint32_t o) { return o ^ (((o >> 7) & 3u) << 5); }
};

template <>
struct DType<true> {
  static constexpr int kEsz = 2;
  static constexpr int kElemsPer128B = 64;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kFmt = sm100::kFmtF16;
  static constexpr uint32_t kBSwizzle = sm100::kSw128;
  static constexpr uint32_t kBSbo = 1024;
  __host__ __device__ static constexpr uint32_t swz(uint32_t o) { return o ^ (((o >> 7) & 7u) << 4); }
};

// ---------------------------------------------------------------------------
// Two-stage configuration per (dtype, N).
// ---------------------------------------------------------------------------
template <bool kHalf, int kN, int kVar = 0>
struct Fft2Shape;
// float2 / tf32.  Two input slots (SIN) for every size: measured against
// three and four on the same box, two took N = 128 ... 2048 from 0.85-0.86
// to 0.97-0.997 of the measured copy peak (N = 4096 already used two, at
// 0.97).  half2 keeps eight: two lost 5-12 %, four measured the same.
template <> struct Fft2Shape<false, 128>  { static constexpr int NS = 8,  NA = 16, G1 = 4, G2 = 2, T = 32, SIN = 2, EPW = 1; };
template <> struct Fft2Shape<false, 256>  { static constexpr int NS = 16, NA = 16, G1 = 2, G2 = 2, T = 16, SIN = 2, EPW = 1; };
template <> struct Fft2Shape<false, 512>  { static constexpr int NS = 32, NA = 16, G1 = 1, G2 = 2, T = 8,  SIN = 2, EPW = 2; };
template <> struct Fft2Shape<false, 1024> { static constexpr int NS = 32, NA = 32, G1 = 1, G2 = 1, T = 4,  SIN = 2, EPW = 2; };
template <> struct Fft2Shape<false, 2048> { static constexpr int NS = 64, NA = 32, G1 = 1, G2 = 1, T = 2,  SIN = 2, EPW = 2; };
template <> struct Fft2Shape<false, 4096> { static constexpr int NS = 64, NA = 64, G1 = 1, G2 = 1, T = 1,  SIN = 2, EPW = 1; };
// half2 / f16
template <> struct Fft2Shape<true, 128>   { static constexpr int NS = 4,  NA = 32, G1 = 8, G2 = 1, T = 32, SIN = 8, EPW = 1; };
template <> struct Fft2Shape<true, 256>   { static constexpr int NS = 8,  NA = 32, G1 = 4, G2 = 1, T = 16, SIN = 8, EPW = 1; };
template <> struct Fft2Shape<true, 512>   { static constexpr int NS = 16, NA = 32, G1 = 2, G2 = 1, T = 8,  SIN = 8, EPW = 1; };
template <> struct Fft2Shape<true, 1024>  { static constexpr int NS = 32, NA = 32, G1 = 1, G2 = 1, T = 4,  SIN = 8, EPW = 1; };
template <> struct Fft2Shape<true, 2048>  { static constexpr int NS = 64, NA = 32, G1 = 1, G2 = 1, T = 2,  SIN = 8, EPW = 1; };
template <> struct Fft2Shape<true, 4096>  { static constexpr int NS = 64, NA = 64, G1 = 1, G2 = 1, T = 1,  SIN = 8, EPW = 1; };
// float2 / tf32, variant 1: NA = 32 so that one 128-B shared-memory line
// holds 32 consecutive reals of one input row.  Used by the 2-D convolution's
// first pass, whose pair-planar tiles keep the two real images in separate
// 128-B column atoms.
template <> struct Fft2Shape<false, 128, 1> { static constexpr int NS = 4,  NA = 32, G1 = 8, G2 = 1, T = 32, SIN = 2, EPW = 2; };
template <> struct Fft2Shape<false, 256, 1> { static constexpr int NS = 8,  NA = 32, G1 = 4, G2 = 1, T = 16, SIN = 2, EPW = 2; };
template <> struct Fft2Shape<false, 512, 1> { static constexpr int NS = 16, NA = 32, G1 = 2, G2 = 1, T = 8,  SIN = 2, EPW = 2; };

template <bool kHalf, int kN, int kVar = 0, int kHSlots = 0>
struct Fft2Cfg {
  using D = DType<kHalf>;
  using S = Fft2Shape<kHalf, kN, kVar>;
  static constexpr bool kIsHalf = kHalf;
  static constexpr int kVariant = kVar;
  // kHSlots > 0 (kEpiMulNatural): the producer stages each tile's spectrum
  // rows in shared memory (kHSlots slots); the input ring shrinks to 2 tiles.
  static constexpr int HS = kHSlots;
  static constexpr int N = kN, NS = S::NS, NA = S::NA, G1 = S::G1, G2 = S::G2, T = S::T;
  static constexpr int SIN = (kHSlots > 0 && S::SIN > 2) ? 2 : S::SIN;
  static_assert(NS * NA == N, "factorization");
  static constexpr int ESZ = D::kEsz, E = D::kElemsPer128B;
  static constexpr int C1 = T / G1, C2 = T / G2;          // signals along MMA N per stage
  static constexpr int M1 = 2 * NS * G1, M2 = 2 * NA * G2; // MMA M per stage
  static constexpr int K1 = NS * G1, K2 = NA * G2;         // MMA K per stage
  static constexpr int N1 = C1 * 2 * NA, N2 = C2 * 2 * NS; // MMA N per stage (TMEM columns)
  static constexpr int H = (2 * NA * ESZ) / 128;           // 128-B atoms per signal row
  static constexpr int TILE_BYTES = T * N * 2 * ESZ;
  static constexpr int A1_BYTES = M1 * K1 * ESZ, A2_BYTES = M2 * K2 * ESZ;
  static constexpr uint32_t LBO1 = K1 * 128, LBO2 = K2 * 128;  // B: stride between N-atoms
  static constexpr int KSTEPS1 = K1 / D::kMmaK, KSTEPS2 = K2 / D::kMmaK;
  static constexpr uint32_t KSTEP_BYTES = D::kMmaK * 128;  // B rows per MMA * 128 B
  static_assert(M1 == 64 || M1 == 128, "M1");
  static_assert(M2 == 64 || M2 == 128, "M2");
  static_assert(N1 <= 256 && N2 <= 256 && N1 % 16 == 0 && N2 % 16 == 0, "N per MMA");
  static_assert(M1 == 64 || N1 <= 128, "TMEM budget stage 1");
  static_assert(M2 == 64 || N2 <= 128, "TMEM budget stage 2");
  static_assert(H >= 1, "128-B rows");
  static constexpr bool kNaturalTma = (H == 1 || G1 == 1);  // natural-layout TMA box exists
  static_assert(K1 % D::kMmaK == 0 && K2 % D::kMmaK == 0, "K");
  // shared-memory map (offsets from a 1024-B aligned base)
  static constexpr uint32_t OFF_A1 = 0;
  static constexpr uint32_t OFF_A2 = (A1_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t OFF_IN = OFF_A2 + (A2_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t OFF_Y = OFF_IN + SIN * TILE_BYTES;
  static constexpr uint32_t OFF_H = OFF_Y + 2 * TILE_BYTES;   // spectrum tiles (kHSlots)
  // a tile's spectrum rows: T * N complex fp32 values (the tile itself for
  // float2 storage, twice its size for half2)
  static constexpr int SPEC_BYTES = T * N * 8;
  static constexpr uint32_t SMEM_DATA = OFF_H + HS * SPEC_BYTES;
  static constexpr uint32_t SMEM_BYTES = exclusive_smem(SMEM_DATA + 1024 /*align slack*/);
  static_assert(SMEM_BYTES + 512 <= 232448, "shared memory budget");
  static constexpr int EPW = S::EPW;                       // epilogue warps per TMEM lane quadrant
  static constexpr int kEpiWarps = 4 * EPW;                // per epilogue stage
  // Warps: producer, MMA issuer, the two epilogue groups, and (kSplitMma) a
  // second MMA issuer for stage 2.  One thread issuing both stages' MMAs
  // waits on each stage's barriers in turn while its tcgen05.mma issue stalls
  // for most of the previous stage's execution (a clock64 timeline of half2
  // N = 4096 showed the issuing thread busy ~1400 of ~1750 cycles per tile).
  // Measured per storage type: half2 C2C gained 1-10 % (N = 4096: 0.74 ->
  // 0.81 of the copy peak), float2 lost 1-2 %, so float2 keeps one issuer.
  static constexpr bool kSplitMma = kHalf;
  static constexpr int kMma2Warp = kSplitMma ? 2 + 2 * kEpiWarps : -1;
  static constexpr int kThreads = 32 * (2 + 2 * kEpiWarps + (kSplitMma ? 1 : 0));
};

// Host-visible kernel parameters (besides tensor maps).
struct FftParams {
  const void* in;
  void* out;
  const void* a1;        // stage-1 A image (global), built by the host
  const void* a2;        // stage-2 A image
  const float2* tw;      // N-entry twiddle table exp(sign*2*pi*i*k/N) (fp32)
  long long batch;
  int use_tma;           // input tiles via TMA (aligned input) or thread loads
  uint32_t* err;         // device error word (0 = ok)
  // Input/output modes used by the 2-D convolution (the C2C API uses the
  // natural layouts).  Signals come in images of R signals; image pair
  // pg = pair0 + sig / R belongs to channel pg / ppc and batch images
  // b = 2 (pg % ppc), b + 1 (channel-major pair order, so consecutive pairs
  // share one filter spectrum).
  const float2* spec;    // kEpiMulNatural: out *= spec[ch][sig % R][k]
  long long rows;        // R: signals per image
  long long pair0;       // first image pair of this launch
  int chans;             // C
  long long nimg_b;      // B (images per channel)
  long long ppc;         // image pairs per channel = ceil(B / 2)
  int blk_log2;          // kEpiBlocked: log2 of the block width Cb
  // Power-of-two range scaling of the half2 2-D convolution (null for every
  // other use): conv_exp[0], [1] = call exponents e2, e3; conv_exp[2 + i] =
  // exponent e1 of image pair pair0 + i.  The stage-2 epilogue multiplies its
  // outputs by 2^e, e = conv_pass 1: e1, 2: e2, 3: e3, 4: -(e1 + e2 + e3).
  const int* conv_exp;
  int conv_pass;
  // Fused conv2d column pass (conv2d_cols_kernel): A image of the inverse's
  // second stage (A1 with stage 2's K-row rotation).
  const void* a4;
  // Overlapping windows (dft1_kernel<C, true>, the tiled convolution): signal
  // w is window t = w % win_per_sig of sequence b = w / win_per_sig, i.e.
  // in[b][t*win_stride + n] (zero past in_len); only its first win_stride
  // outputs are stored, at out[b][t*win_stride + n] (n < out_len - t*win_stride).
  int win_stride;
  long long win_per_sig;
  long long in_len;
  long long out_len;
  long long win_tmax;    // last window index lying wholly inside its sequence (-1: none)
};

// Stage-2 epilogue output modes.
enum EpiMode : int {
  kEpiNatural = 0,        // out[sig][k]
  kEpiBlocked = 2,        // out[img][k / Cb][r][k % Cb] (sig = img*R + r): column-blocked
  kEpiMulNatural = 3,     // out[sig][k] * spec[ch][r][k]
  kEpiUnpackPair = 4,     // real fp32 images: Re -> y[b][ch][r][k], Im -> y[b+1][ch][r][k]
};

// Stage-1 input modes.  All three land in the same MN-major B layout
// ([128-B column atom][K row][128 B]); they differ in the column order
// inside a tile, which the stage-1 epilogue undoes:
//   natural     column = (c * NA + a) * 2 + plane      (interleaved complex rows)
//   pair planar column = c * 2 NA + plane * NA + a     (two real images, plane = image)
//   blocked     column = (a * C1 + c) * 2 + plane      (signals are matrix columns)
// Every TMA box row is one whole 128-B line (a narrower box row would be
// padded to the swizzle span in shared memory), which is why the pair-planar
// mode needs NA >= 32 and the column mode reads the column-blocked layout
// written by kEpiBlocked with Cb = C1: 16 / C1 consecutive rows of a block
// form one contiguous 128-B line.
enum InMode : int {
  kInNatural = 0,         // in[sig][n] complex, by TMA or masked thread loads
  kInPairPlanar = 1,      // real fp32 x[b][ch][r][n]: signal = row r of images (b, b+1), by TMA
  kInBlocked = 2,         // in[img][r / C1][n][r % C1] complex: signal r of image img, by TMA
};

namespace detail {

// 2^e as a float, e clamped to [-120, 120] (exact).
__device__ __forceinline__ float pow2f(int e) {
  e = e < -120 ? -120 : (e > 120 ? 120 : e);
  return __int_as_float((127 + e) << 23);
}

// ceil(log2(x)) for finite x > 0 (exact, from the bits; subnormals -> -126).
__device__ __forceinline__ int ceil_log2f(float x) {
  const uint32_t b = __float_as_uint(x);
  const int e = (int)((b >> 23) & 0xffu);
  if (e == 0) return -126;
  return e - 127 + ((b & 0x7fffffu) ? 1 : 0);
}

// Stage-2 K row of stage-2 input index r (= g2 * NA + a): a permutation of
// r's low three bits, chosen per configuration so that the four rows one
// stage-1 epilogue store covers (one per lane of a quad) fall on distinct
// shared-memory banks under the operand swizzle.  The host permutes the
// stage-2 DFT matrix's K columns the same way.
//   1 (half2): a store covers consecutive a; row bits [2:1] = r bits [1:0],
//     row bit 0 = r bit 2.  Under the 128-B swizzle (16-B chunk ^= row % 8)
//     rows differing only in bit 0 shared a 32-B chunk pair, two wavefronts
//     per store (half2 N = 4096: 1,190,106 -> 80,228 conflicts).
//   2 (float2, pair-planar input of the 2-D convolution's first pass): a
//     store covers a = 8j + 2l + e, every other row; row bits [1:0] = r bits
//     [2:1], row bit 2 = r bit 0.  The float swizzle keys its 32-B granules
//     on row % 4, which took only two values over those rows.
//   0: identity (float2 natural input: consecutive rows, already minimal).
__host__ __device__ constexpr int stage2_rotation(bool half, int variant) {
  return half ? 1 : (variant == 1 ? 2 : 0);
}

// Stage-2 column pair of stage-1 output ks (C2C kernels, NS % 8 == 0):
// ks = 8m + 2l + h -> pair 8m + 4h + l.
__host__ __device__ constexpr int stage2_col_pair(int ks) {
  return (ks & ~7) | ((ks & 1) << 2) | ((ks >> 1) & 3);
}
__host__ __device__ constexpr int stage2_krow(int rotation, int r) {
  return rotation == 1   ? ((r & ~7) | ((r & 3) << 1) | ((r >> 2) & 1))
         : rotation == 2 ? ((r & ~7) | ((r >> 1) & 3) | ((r & 1) << 2))
                         : r;
}

template <bool kHalf>
__device__ __forceinline__ void store_complex(uint32_t saddr, float re, float im);
template <>
__device__ __forceinline__ void store_complex<false>(uint32_t saddr, float re, float im) {
  sm100::st_shared_v2(saddr, sm100::round_tf32(re), sm100::round_tf32(im));
}
template <>
__device__ __forceinline__ void store_complex<true>(uint32_t saddr, float re, float im) {
  __half2 h = __floats2half2_rn(re, im);
  sm100::st_shared_b32(saddr, *reinterpret_cast<uint32_t*>(&h));
}

template <bool kHalf>
__device__ __forceinline__ void store_out(void* out, long long idx, float re, float im);
template <>
__device__ __forceinline__ void store_out<false>(void* out, long long idx, float re, float im) {
  reinterpret_cast<float2*>(out)[idx] = make_float2(re, im);
}
template <>
__device__ __forceinline__ void store_out<true>(void* out, long long idx, float re, float im) {
  reinterpret_cast<__half2*>(out)[idx] = __floats2half2_rn(re, im);
}

// Byte offset of complex element (sig, s, a) of a stage-1 tile in shared
// memory (MN-major B: N-atom = column/E, K row = g*NS + s, 128-B rows).
template <class C>
__device__ __forceinline__ uint32_t in_tile_offset(int sig, int s, int a) {
  const int g = sig / C::C1, c = sig % C::C1;
  const int col = c * 2 * C::NA + 2 * a;
  const int atom = col / C::E, e = col % C::E;
  const uint32_t krow = g * C::NS + s;
  return atom * C::LBO1 + C::D::swz(krow * 128u + e * C::ESZ);
}

// Stage-1 epilogue geometry of fft2_kernel (one accumulator per stage): M=64
// -> one 16-row block per TMEM lane quadrant, its 64-column chunks split over
// the EPW warps of the quadrant; M=128 -> two row blocks per quadrant, split
// over the EPW warps.
template <int kM, int kNcols, int kEPW>
struct EpiGeo {
  static constexpr int kNC = kNcols / 64;
  static constexpr int BPW = (kM == 64) ? 1 : 2 / kEPW;
  static constexpr int CH = (kM == 64) ? kNC / kEPW : kNC;
  __host__ __device__ static constexpr int ch0(int h) { return (kM == 64 && kEPW > 1) ? h * CH : 0; }
  __host__ __device__ static constexpr int block(int q, int h, int bi) { return (kM == 64) ? q : 2 * q + h * BPW + bi; }
};

// Byte offset in the stage-2 operand buffer of the value that stage-1
// epilogue warp `warp` (absolute index), lane `lane` writes for row block bi,
// chunk c and output o (input modes with one chunk per signal group).
template <class C, int kIn, bool kColPairs>
struct Fft2E1Off {
  __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int o) {
    using G = EpiGeo<C::M1, C::N1, C::EPW>;
    const int q = warp & 3, h = (warp - 2) >> 2, l = lane & 3;
    const int ch0 = G::ch0(h);
    const int rp = G::block(q, h, bi) * 8 + (lane >> 2);
    const int g1 = rp / C::NS, ks = rp % C::NS;
    int c1 = 0, a = 0;
    if (kIn == kInPairPlanar) {
      const int jr = (C::NA == 16) ? ((o >> 1) >> 1) * 4 + ((o >> 1) & 1) : (o >> 1);
      const int col = 64 * (ch0 + c) + 8 * jr + 2 * l + (o & 1);
      c1 = col / (2 * C::NA);
      a = col % (2 * C::NA);
    } else {
      const int pidx = 4 * ((ch0 + c) * 8 + o) + l;
      if (kIn == kInNatural) { c1 = pidx / C::NA; a = pidx % C::NA; }
      else { a = pidx / C::C1; c1 = pidx % C::C1; }
    }
    const int sig = g1 * C::C1 + c1;
    const int g2 = sig / C::C2, c2 = sig % C::C2;
    const uint32_t krow = (uint32_t)stage2_krow(stage2_rotation(C::kIsHalf, C::kVariant), g2 * C::NA + a);
    const int col = c2 * 2 * C::NS + 2 * (kColPairs ? stage2_col_pair(ks) : ks);
    return (uint32_t)(col / C::E) * C::LBO2 + C::D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
  }
};

// Stage-2 epilogue with column pairs: the outputs k0, k0 + 1 of tile signal
// sl that warp `warp`, lane `lane` holds for row block bi, chunk c and
// iteration pair j (even).  kWhat 0: sl * N + k0 (element offset in the
// tile's natural output rows); 1: sl; 2: the 128-B-swizzled byte offset of
// that element in a staged complex fp32 tile.
template <class C, int kWhat>
struct Fft2E2Pos {
  __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int j) {
    using G = EpiGeo<C::M2, C::N2, C::EPW>;
    const int q = warp & 3, h = (warp - 2 - C::kEpiWarps) >> 2, l4 = lane & 3;
    const int rp = G::block(q, h, bi) * 8 + (lane >> 2);
    const int g2 = rp / C::NA, ka = rp % C::NA;
    const int pidx = 4 * ((G::ch0(h) + c) * 8 + j) + l4;
    const int c2 = pidx / C::NS, pp = pidx % C::NS;
    const int k0 = C::NS * ka + (pp & ~7) + 2 * l4;
    const int sl = g2 * C::C2 + c2;
    if (kWhat == 1) return (uint32_t)sl;
    const uint32_t e = (uint32_t)(sl * C::N + k0);
    if (kWhat == 0) return e;
    const uint32_t byte = e * 8u;
    return byte ^ (((byte >> 7) & 7u) << 4);
  }
};

// Stage-2 epilogue, half2 column-blocked output with block width 4 and
// paired signal rows: for the jv-th stored iteration j of chunk c (the j with
// (j / PJ) even, PJ = NS / 4), kWhat 0: k >> 2 (the output's block row),
// 1: the element offset inside the block rows, (sl + row) * 4 + 2 (l4 & 1),
// where row 0/1 is the signal row this lane stores.  The element offset of
// the store is then (k >> 2) * rows * 4 + kWhat-1 value + the tile's base.
template <class C, int kWhat>
struct Fft2E2PairRows {
  __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int jv) {
    using G = EpiGeo<C::M2, C::N2, C::EPW>;
    constexpr int PJ = C::NS / 4;
    const int j = (jv / PJ) * 2 * PJ + (jv % PJ);
    const int q = warp & 3, h = (warp - 2 - C::kEpiWarps) >> 2, l4 = lane & 3;
    const int rp = G::block(q, h, bi) * 8 + (lane >> 2);
    const int g2 = rp / C::NA, ka = rp % C::NA;
    const int pidx = 4 * ((G::ch0(h) + c) * 8 + j) + l4;
    const int c2 = pidx / C::NS, ks = pidx % C::NS;
    const int sl = g2 * C::C2 + c2;
    const int k = C::NS * ka + ks;
    if (kWhat == 0) return (uint32_t)(k >> 2);
    return (uint32_t)((sl + (l4 < 2 ? 0 : 1)) * 4 + 2 * (l4 & 1));
  }
};

}  // namespace detail

// ---------------------------------------------------------------------------
// Two-stage kernel
// ---------------------------------------------------------------------------
// kOutHalf: storage of the complex outputs (half2 or float2); it differs from
// the configuration's storage only in the first pass of the half2 2-D
// convolution (float2 input tile, half2 output).
template <class C, int kEpi = kEpiNatural, int kIn = kInNatural, bool kOutHalf = C::kIsHalf>
__global__ void __launch_bounds__(C::kThreads, 1)
fft2_kernel(const __grid_constant__ CUtensorMap tmap_in, const __grid_constant__ CUtensorMap tmap_spec,
            const FftParams p) {
  using namespace sm100;
  using D = typename C::D;
  // Column pairs: the stage-1 epilogue puts output ks of stage 1 at stage-2
  // column pair stage2_col_pair(ks) (a permutation inside each group of 8),
  // so that the 16x256b TMEM loads of stage 2 hand a thread outputs k and
  // k + 1 in consecutive iterations.  Each lane then stores two outputs (8 or
  // 16 B) and a quad of lanes whole 32-B sectors, without shuffles; the
  // stage-1 epilogue's stores keep their footprint (one aligned group of 8
  // column pairs per row).  Used by the outputs along k: C2C, fp32 spectrum
  // products, fp32 image rows.  Measured against plain 4/8-B stores (C2C):
  // half2 +2 % (N = 512) to +12 % (N = 256), float2 +1-2 % (N = 2048 within
  // +-1 %); the fp32 image rows of the 2-D convolution's last pass: -24 %
  // time (float2), -3 % (half2).
  constexpr bool kColPairs = C::NS % 8 == 0 &&
                             ((kEpi == kEpiNatural && kIn == kInNatural) ||
                              (kEpi == kEpiMulNatural && !(kOutHalf && C::HS > 0)) || kEpi == kEpiUnpackPair);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in_full[C::SIN], bar_in_empty[C::SIN];
  __shared__ uint64_t bar_acc1_full[2], bar_acc1_empty[2], bar_y_full[2], bar_y_empty[2];
  __shared__ uint64_t bar_acc2_full[2], bar_acc2_empty[2], bar_const, bar_done, bar_done2;
  __shared__ uint64_t bar_h_full[C::HS > 0 ? C::HS : 1], bar_h_empty[C::HS > 0 ? C::HS : 1];
  __shared__ uint32_t tmem_slot;
  constexpr bool kStageH = kEpi == kEpiMulNatural && C::HS > 0;   // spectrum tiles via TMA

  const uint32_t warp = warp_id(), lane = lane_id();
  const long long batch = p.batch;
  const long long num_tiles = (batch + C::T - 1) / C::T;
  const long long full_tiles = batch / C::T;
  // tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = (int)((num_tiles > blockIdx.x) ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::SIN; ++i) { mbar_init(&bar_in_full[i], 1); mbar_init(&bar_in_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_acc1_full[i], 1); mbar_init(&bar_acc1_empty[i], C::kEpiWarps);
      mbar_init(&bar_y_full[i], C::kEpiWarps); mbar_init(&bar_y_empty[i], 1);
      mbar_init(&bar_acc2_full[i], 1); mbar_init(&bar_acc2_empty[i], C::kEpiWarps);
    }
    mbar_init(&bar_const, 1);
    mbar_init(&bar_done, 1);
    mbar_init(&bar_done2, 1);
    if constexpr (kStageH)
      for (int i = 0; i < C::HS; ++i) { mbar_init(&bar_h_full[i], 1); mbar_init(&bar_h_empty[i], C::kEpiWarps); }
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  // Stage-2 MMAs of tile j, issued by one thread (the MMA issuer, or the
  // second issuer with kSplitMma); false when a wait gave up.
  auto issue_stage2 = [&](int j) -> bool {
    using namespace sm100;
    const int buf = j & 1;
    const uint32_t ph = (uint32_t)(j >> 1) & 1u;
    if (!mbar_wait(&bar_y_full[buf], ph, p.err, kDevTimeoutMma)) return false;
    if (!mbar_wait(&bar_acc2_empty[buf], ph ^ 1u, p.err, kDevTimeoutMma)) return false;
    tc_fence_after();
    const uint32_t idesc2 = instr_desc(D::kFmt, C::M2, C::N2, 0, 1);
    const uint32_t lboA2 = (C::M2 / 8) * 128;   // A image: K-major, no swizzle
    const uint64_t adA2 = smem_desc(smem_u32(smem + C::OFF_A2), lboA2, 128, kSwNone);
    const uint64_t bd0 = smem_desc(smem_u32(smem + C::OFF_Y), C::LBO2, D::kBSbo, D::kBSwizzle) +
                         (uint64_t)(buf * (C::TILE_BYTES >> 4));
    const uint32_t d = (C::M2 == 64) ? tmem + 256u + ((uint32_t)(16 * buf) << 16)
                                     : tmem + 256u + (uint32_t)(buf * C::N2);
#pragma unroll
    for (int k = 0; k < C::KSTEPS2; ++k) {
      const uint64_t ad = adA2 + (uint64_t)((k * 2 * lboA2) >> 4);
      const uint64_t bd = bd0 + (uint64_t)((k * C::KSTEP_BYTES) >> 4);
      if constexpr (C::kIsHalf) umma_f16(d, ad, bd, idesc2, k > 0);
      else umma_tf32(d, ad, bd, idesc2, k > 0);
    }
    umma_commit(&bar_y_empty[buf]);
    umma_commit(&bar_acc2_full[buf]);
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (p.use_tma) tma_prefetch_desc(&tmap_in);
      if constexpr (kStageH) tma_prefetch_desc(&tmap_spec);
      // constant stage matrices (bulk copies of host-built images)
      mbar_arrive_expect_tx(&bar_const, C::A1_BYTES + C::A2_BYTES);
      bulk_load(smem + C::OFF_A1, p.a1, C::A1_BYTES, &bar_const);
      bulk_load(smem + C::OFF_A2, p.a2, C::A2_BYTES, &bar_const);
    }
    for (int i = 0; i < my_tiles; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int slot = i % C::SIN;
      const uint32_t ph = (uint32_t)(i / C::SIN) & 1u;
      if (!mbar_wait_warp(&bar_in_empty[slot], ph ^ 1u, p.err, kDevTimeoutProducer)) break;
      uint8_t* dst = smem + C::OFF_IN + slot * C::TILE_BYTES;
      if constexpr (kIn != kInNatural) {
        // conv2d modes: whole tiles inside one image (R % T == 0, checked by the host)
        if (lane == 0) {
          const long long sig0 = tile * C::T;
          const long long img = sig0 / p.rows, r0 = sig0 - img * p.rows;
          int c0 = 0, c1 = 0, c2 = 0, c3 = 0, c4 = 0;
          if constexpr (kIn == kInPairPlanar) {
            static_assert(C::NA >= 32, "pair-planar rows must fill 128-B lines");
            const long long pg = p.pair0 + img, ch = pg / p.ppc;
            c3 = (int)(2 * (pg - ch * p.ppc));                     // {a, s, g | a_hi, plane, row}
            c4 = (int)(ch * p.rows + r0);
          } else {
            c4 = (int)tile;                                        // {line, s, g, a_hi, tile}
          }
          mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
          tma_load_5d(dst, &tmap_in, &bar_in_full[slot], c0, c1, c2, c3, c4);
        }
        __syncwarp();
      } else if (p.use_tma && tile < full_tiles) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
          tma_load_5d(dst, &tmap_in, &bar_in_full[slot], 0, 0, 0, 0, (int)tile);
        }
        __syncwarp();
      } else {
        // masked thread loads (partial last tile or unaligned input)
        const long long sig0 = tile * C::T;
        const uint32_t base = smem_u32(dst);
        if (p.use_tma) {
          // aligned input (the partial last tile): 16-byte vectors, 4 half2 or
          // 2 float2 consecutive elements of one stage-1 row, which stay
          // contiguous in the tile under either operand swizzle.  One warp
          // loading the tile element by element kept the CTA that owns the
          // last tile busy for microseconds after all others had finished.
          constexpr int V = 16 / (2 * C::ESZ);
          static_assert(C::NA % V == 0, "vectors stay inside one stage-1 row");
#pragma unroll 4
          for (int idx = lane; idx < C::T * C::N / V; idx += 32) {
            const int e0 = idx * V;
            const int sig = e0 / C::N, n = e0 % C::N;
            const uint32_t off = detail::in_tile_offset<C>(sig, n / C::NA, n % C::NA);
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (sig0 + sig < batch) v = __ldg(reinterpret_cast<const uint4*>(p.in) + ((sig0 + sig) * C::N + n) / V);
            st_shared_v4(base + off, v.x, v.y, v.z, v.w);
          }
        } else
        for (int idx = lane; idx < C::T * C::N; idx += 32) {
          const int sig = idx / C::N, n = idx % C::N;
          const int s = n / C::NA, a = n % C::NA;
          const uint32_t off = detail::in_tile_offset<C>(sig, s, a);
          if (sig0 + sig < batch) {
            if constexpr (C::kIsHalf) {
              const uint32_t v = __ldg(reinterpret_cast<const unsigned int*>(p.in) + (sig0 + sig) * C::N + n);
              st_shared_b32(base + off, v);
            } else {
              const float2 v = __ldg(reinterpret_cast<const float2*>(p.in) + (sig0 + sig) * C::N + n);
              st_shared_v2(base + off, v.x, v.y);
            }
          } else {
            if constexpr (C::kIsHalf) st_shared_b32(base + off, 0u);
            else st_shared_v2(base + off, 0.f, 0.f);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_in_full[slot]);
      }
      if constexpr (kStageH) {
        // spectrum rows of this tile: spec[ch][r0 .. r0+T)[0 .. N) = T*N complex,
        // one 2-D box of 128-B lines (128-B swizzle against bank conflicts).
        // Issued after the tile's input: the slot frees when the previous
        // tile's stage-2 epilogue ends, which needs this tile's stage 1.
        const int hs = i % C::HS;
        if (!mbar_wait_warp(&bar_h_empty[hs], ((uint32_t)(i / C::HS) & 1u) ^ 1u, p.err, kDevTimeoutProducer)) break;
        if (lane == 0) {
          const long long sig0 = tile * C::T;
          const long long img = sig0 / p.rows, r0 = sig0 - img * p.rows;
          const long long pg = p.pair0 + img, ch = pg / p.ppc;
          mbar_arrive_expect_tx(&bar_h_full[hs], C::SPEC_BYTES);
          tma_load_3d(smem + C::OFF_H + hs * C::SPEC_BYTES, &tmap_spec, &bar_h_full[hs], 0,
                      (int)(((ch * p.rows + r0) * C::N) / 16), 0);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&bar_const, 0, p.err, kDevTimeoutMma);
      const uint32_t a1 = smem_u32(smem + C::OFF_A1);
      const uint32_t idesc1 = instr_desc(D::kFmt, C::M1, C::N1, 0, 1);
      // A images: K-major, no swizzle, core matrix (8 rows x 16 B) contiguous;
      // LBO = K-direction core stride = M/8 * 128 B, SBO = 128 B.
      const uint32_t lboA1 = (C::M1 / 8) * 128;
      // Descriptors are built once; a K step, an input slot or a Y buffer adds
      // its byte offset >> 4 to the start-address field (shared addresses
      // < 256 KB never carry out of it).  The issuing thread then spends a
      // few integer adds per MMA.
      const uint64_t adA1 = smem_desc(a1, lboA1, 128, kSwNone);
      const uint64_t bdIn0 = smem_desc(smem_u32(smem + C::OFF_IN), C::LBO1, D::kBSbo, D::kBSwizzle);
      // stage 1 of tile i, then (one issuer) stage 2 of tile i - 1
      for (int i = 0; ok && i <= my_tiles; ++i) {
        if (i < my_tiles) {
          const int slot = i % C::SIN, buf = i & 1;
          if (!mbar_wait(&bar_in_full[slot], (uint32_t)(i / C::SIN) & 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          if (!mbar_wait(&bar_acc1_empty[buf], ((uint32_t)(i >> 1) & 1u) ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bd0 = bdIn0 + (uint64_t)(slot * (C::TILE_BYTES >> 4));
          const uint32_t d = (C::M1 == 64) ? tmem + ((uint32_t)(16 * buf) << 16) : tmem + (uint32_t)(buf * C::N1);
#pragma unroll
          for (int k = 0; k < C::KSTEPS1; ++k) {
            const uint64_t ad = adA1 + (uint64_t)((k * 2 * lboA1) >> 4);
            const uint64_t bd = bd0 + (uint64_t)((k * C::KSTEP_BYTES) >> 4);
            if constexpr (C::kIsHalf) umma_f16(d, ad, bd, idesc1, k > 0);
            else umma_tf32(d, ad, bd, idesc1, k > 0);
          }
          umma_commit(&bar_in_empty[slot]);
          umma_commit(&bar_acc1_full[buf]);
        }
        if constexpr (!C::kSplitMma) {
          if (i > 0 && !issue_stage2(i - 1)) { ok = false; break; }
        }
      }
      // drain: all issued MMAs complete before TMEM is released
      umma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.err, kDevTimeoutMma);
    }
    __syncwarp();
  } else if (C::kSplitMma && warp == (uint32_t)C::kMma2Warp) {
    // ------------------------------------------------------------ stage-2 MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&bar_const, 0, p.err, kDevTimeoutMma);
      for (int j = 0; ok && j < my_tiles; ++j)
        if (!issue_stage2(j)) ok = false;
      umma_commit(&bar_done2);
      mbar_wait(&bar_done2, 0, p.err, kDevTimeoutMma);
    }
    __syncwarp();
  } else if (warp < 2 + C::kEpiWarps) {
    // ------------------------------------------------------------ epilogue 1
    // Two warps per TMEM lane quadrant q (warp % 4).  M=64: row block q
    // (lanes 32q + 16*buf), the two warps split its 64-column chunks;
    // M=128: row blocks 2q, 2q+1 (lanes 32q, 32q+16), one per warp.
    // Each thread's twiddles are the same for every tile and are loaded once.
    static_assert(kIn != kInPairPlanar || !C::kIsHalf, "the pair-planar input mode reads fp32 images");
    const uint32_t q = warp & 3u;
    const int h = (int)(warp - 2) >> 2;                 // warp index within its quadrant
    const int l = (int)(lane & 3u);
    constexpr int kNC = C::N1 / 64;
    // M=64: one row block per quadrant, chunks split over EPW warps;
    // M=128: two row blocks per quadrant, split over EPW warps.
    constexpr int BPW = (C::M1 == 64) ? 1 : 2 / C::EPW;
    constexpr int CH = (C::M1 == 64) ? kNC / C::EPW : kNC;
    const int ch0 = (C::M1 == 64 && C::EPW > 1) ? h * CH : 0;
    // A pair-planar signal with NA = 64 spans two chunks (re plane, im plane).
    constexpr int GC = (kIn == kInPairPlanar && C::NA == 64) ? 2 : 1;
    static_assert(CH % GC == 0 && (GC == 1 || C::EPW == 1), "chunk groups");
    // Twiddles w_N^(a ks), one slot per distinct a of this thread:
    //   natural     a = l + 4 slot                   (slot < NA/4)
    //   pair planar a = 8 (slot/2) + 2 l + slot%2    (slot < NA/4)
    //   transposed  a = (4 m + l) / C1, m = ch0*8 + slot*kTq (the warp's chunks only)
    constexpr int kTq = (kIn == kInBlocked && C::C1 >= 4) ? C::C1 / 4 : 1;
    constexpr int kTw = (kIn == kInBlocked) ? CH * 8 / kTq : C::NA / 4;
    static_assert(kIn != kInNatural || (CH * 8) % kTw == 0, "twiddle slot must not depend on the warp's chunk offset");
    float2 tw[BPW][kTw];
#pragma unroll
    for (int bi = 0; bi < BPW; ++bi) {
      const int block = (C::M1 == 64) ? (int)q : (int)(2 * q) + h * BPW + bi;
      const int ks = (block * 8 + (int)(lane >> 2)) % C::NS;
#pragma unroll
      for (int i = 0; i < kTw; ++i) {
        int a;
        if constexpr (kIn == kInNatural) a = l + 4 * i;
        else if constexpr (kIn == kInPairPlanar) a = 8 * (i >> 1) + 2 * l + (i & 1);
        else a = (4 * (ch0 * 8 + i * kTq) + l) / C::C1;
        tw[bi][i] = p.tw[(a * ks) % C::N];
      }
    }
    const uint32_t ybase = smem_u32(smem + C::OFF_Y);
    // store addresses: per-thread bases plus compile-time offsets (epi_addr.cuh)
    using E1Off = detail::Fft2E1Off<C, kIn, kColPairs>;
    constexpr int kAK = (GC == 1) ? epi::addr_kind<E1Off, 2, C::kEpiWarps, BPW, CH, 8>() : 0;
    uint32_t abase[BPW][kAK == 1 ? 8 : 1];
#pragma unroll
    for (int bi = 0; bi < BPW; ++bi) {
#pragma unroll
      for (int o = 0; o < (kAK == 1 ? 8 : 1); ++o) abase[bi][o] = E1Off::f((int)warp, (int)lane, bi, 0, o);
    }
    for (int i = 0; i < my_tiles; ++i) {
      const int buf = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!mbar_wait_warp(&bar_acc1_full[buf], ph, p.err, kDevTimeoutEpilogue)) break;
      if (!mbar_wait_warp(&bar_y_empty[buf], ph ^ 1u, p.err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t yb = ybase + buf * C::TILE_BYTES;
      // One output: the four partial sums cos*re, cos*im, sin*re, sin*im of
      // stage-1 output (ks, a) -> twiddled complex value into the stage-2 operand.
      auto emit1 = [&](int bi, int c, int o, float rr, float ri, float ir, float ii) {
        const int block = (C::M1 == 64) ? (int)q : (int)(2 * q) + h * BPW + bi;
        const int rp = block * 8 + (int)(lane >> 2);
        const int g1 = rp / C::NS, ks = rp % C::NS;
        int c1, a, slot;
        if constexpr (kIn == kInPairPlanar) {
          constexpr int d = C::NA / 8;  // sub-chunks between the re and im planes
          const int jr = (C::NA == 16) ? ((o >> 1) >> 1) * 4 + ((o >> 1) & 1) : (o >> 1);
          const int e = o & 1;
          const int col = 64 * (ch0 + c) + 8 * jr + 2 * l + e;
          c1 = col / (2 * C::NA); a = col % (2 * C::NA);
          slot = 2 * (jr % d) + e;
        } else {
          const int pidx = 4 * ((ch0 + c) * 8 + o) + l;
          if constexpr (kIn == kInNatural) {
            c1 = pidx / C::NA; a = pidx % C::NA;
            // a = l + 4*((ch0+c)*8 + o) mod NA -> slot ((ch0+c)*8 + o) mod NA/4
            // = (c*8 + o) mod NA/4 because ch0*8 is a multiple of NA/4
            slot = (c * 8 + o) % kTw;
          } else {
            a = pidx / C::C1; c1 = pidx % C::C1;
            slot = (c * 8 + o) / kTq;
          }
        }
        const float yr = rr - ii, yi = ir + ri;
        const float2 w = tw[bi][slot];
        const float zr = yr * w.x - yi * w.y, zi = yr * w.y + yi * w.x;
        uint32_t off;
        if constexpr (kAK != 0) {
          off = abase[bi][kAK == 1 ? o : 0] + epi::addr_delta<E1Off, 2, kAK>(bi, c, o);
        } else {
          const int sig = g1 * C::C1 + c1;
          const int g2 = sig / C::C2, c2 = sig % C::C2;
          const uint32_t krow = (uint32_t)detail::stage2_krow(detail::stage2_rotation(C::kIsHalf, C::kVariant), g2 * C::NA + a);
          const int col = c2 * 2 * C::NS + 2 * (kColPairs ? detail::stage2_col_pair(ks) : ks);
          off = (col / C::E) * C::LBO2 + D::swz(krow * 128u + (col % C::E) * C::ESZ);
        }
        detail::store_complex<C::kIsHalf>(yb + off, zr, zi);
      };
      // TMEM address of (row block bi, chunk c) of this tile's accumulator
      auto acc1 = [&](int bi, int c) -> uint32_t {
        const uint32_t lanes = (C::M1 == 64) ? 32u * q + 16u * buf : 32u * q + 16u * (uint32_t)(h * BPW + bi);
        const uint32_t cols = (C::M1 == 64) ? 0u : (uint32_t)(buf * C::N1);
        return tmem + (lanes << 16) + cols + (uint32_t)(ch0 + c) * 64u;
      };
      // Overlapped TMEM loads (the next 32-column piece loads while this one is
      // processed) measured faster for the 2-D convolution's passes and
      // slower for the C2C transform (half2 N = 256, 512: 4-9 %), which keeps
      // whole-chunk loads written out in place.
      if constexpr (kIn == kInNatural) {
#pragma unroll
        for (int bi = 0; bi < BPW; ++bi) {
          const int block = (C::M1 == 64) ? (int)q : (int)(2 * q) + h * BPW + bi;
          const int rp = block * 8 + (int)(lane >> 2);
          const int g1 = rp / C::NS, ks = rp % C::NS;
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            uint32_t r[32];
            tmem_ld_16x256b_x8(acc1(bi, c), r);
            tmem_wait_ld();
#pragma unroll
            for (int o = 0; o < 8; ++o) {
              const int pidx = 4 * ((ch0 + c) * 8 + o) + l;
              const int c1 = pidx / C::NA, a = pidx % C::NA;
              // a = l + 4*((ch0+c)*8 + o) mod NA -> slot ((ch0+c)*8 + o) mod NA/4
              // = (c*8 + o) mod NA/4 because ch0*8 is a multiple of NA/4
              const int slot = (c * 8 + o) % kTw;
              const float rr = __uint_as_float(r[4 * o]), ri = __uint_as_float(r[4 * o + 1]);
              const float ir = __uint_as_float(r[4 * o + 2]), ii = __uint_as_float(r[4 * o + 3]);
              const float yr = rr - ii, yi = ir + ri;
              const float2 w = tw[bi][slot];
              const float zr = yr * w.x - yi * w.y, zi = yr * w.y + yi * w.x;
              uint32_t off;
              if constexpr (kAK != 0) {
                off = abase[bi][kAK == 1 ? o : 0] + epi::addr_delta<E1Off, 2, kAK>(bi, c, o);
              } else {
                const int sig = g1 * C::C1 + c1;
                const int g2 = sig / C::C2, c2 = sig % C::C2;
                const uint32_t krow = (uint32_t)detail::stage2_krow(detail::stage2_rotation(C::kIsHalf, C::kVariant), g2 * C::NA + a);
                const int col = c2 * 2 * C::NS + 2 * (kColPairs ? detail::stage2_col_pair(ks) : ks);
                off = (col / C::E) * C::LBO2 + D::swz(krow * 128u + (col % C::E) * C::ESZ);
              }
              detail::store_complex<C::kIsHalf>(yb + off, zr, zi);
            }
          }
        }
      } else if constexpr (kIn != kInPairPlanar) {
        // 32-column pieces, the next one loading while this one is processed
        constexpr int NIT = BPW * CH * 2;
        uint32_t rb[2][16];
        tmem_ld_16x256b_x4(acc1(0, 0), rb[0]);
#pragma unroll
        for (int it = 0; it < NIT; ++it) {
          tmem_wait_ld();
          tmem_regs_ready(rb[it & 1]);
          if (it + 1 < NIT)
            tmem_ld_16x256b_x4(acc1((it + 1) / (2 * CH), ((it + 1) / 2) % CH) + 32u * (uint32_t)((it + 1) & 1),
                               rb[(it + 1) & 1]);
          const int bi = it / (2 * CH), c = (it / 2) % CH, hh = it & 1;
#pragma unroll
          for (int oo = 0; oo < 4; ++oo)
            emit1(bi, c, 4 * hh + oo, __uint_as_float(rb[it & 1][4 * oo]), __uint_as_float(rb[it & 1][4 * oo + 1]),
                  __uint_as_float(rb[it & 1][4 * oo + 2]), __uint_as_float(rb[it & 1][4 * oo + 3]));
        }
      } else if constexpr (kIn == kInPairPlanar && GC == 1 && C::NA == 32) {
        // pair-planar, NA = 32: output o of a chunk needs column groups jr and
        // jr + 4 (re and im planes, jr = o / 2).  Pieces of 16 registers hold
        // groups {2p, 2p+1, 2p+4, 2p+5} (two 16-column loads); the next piece
        // loads while this one is processed.
        constexpr int NIT = BPW * CH * 2;
        uint32_t rb[2][16];
        auto piece = [&](int it, uint32_t (&v)[16]) {
          const uint32_t a = acc1(it / (2 * CH), (it / 2) % CH) + 16u * (uint32_t)(it & 1);
          tmem_ld_16x256b_x2(a, *reinterpret_cast<uint32_t(*)[8]>(&v[0]));
          tmem_ld_16x256b_x2(a + 32u, *reinterpret_cast<uint32_t(*)[8]>(&v[8]));
        };
        piece(0, rb[0]);
#pragma unroll
        for (int it = 0; it < NIT; ++it) {
          tmem_wait_ld();
          tmem_regs_ready(rb[it & 1]);
          if (it + 1 < NIT) piece(it + 1, rb[(it + 1) & 1]);
          const int bi = it / (2 * CH), c = (it / 2) % CH, pc = it & 1;
#pragma unroll
          for (int jq = 0; jq < 2; ++jq) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int o = 2 * (2 * pc + jq) + e;
              emit1(bi, c, o, __uint_as_float(rb[it & 1][4 * jq + e]), __uint_as_float(rb[it & 1][8 + 4 * jq + e]),
                    __uint_as_float(rb[it & 1][4 * jq + 2 + e]), __uint_as_float(rb[it & 1][8 + 4 * jq + 2 + e]));
            }
          }
        }
      } else {
#pragma unroll
        for (int bi = 0; bi < BPW; ++bi) {
#pragma unroll
          for (int c = 0; c < CH; c += GC) {
            uint32_t r[GC][32];
#pragma unroll
            for (int g = 0; g < GC; ++g) tmem_ld_16x256b_x8(acc1(bi, c + g), r[g]);
            tmem_wait_ld();
#pragma unroll
            for (int o = 0; o < 8 * GC; ++o) {
              // registers of cos*re, cos*im, sin*re, sin*im of this output
              int iRR = 4 * o, iRI = 4 * o + 1, iIR = 4 * o + 2, iII = 4 * o + 3;
              if constexpr (kIn == kInPairPlanar) {
                constexpr int d = C::NA / 8;  // sub-chunks between the re and im planes
                const int jr = (C::NA == 16) ? ((o >> 1) >> 1) * 4 + ((o >> 1) & 1) : (o >> 1);
                const int e = o & 1;
                iRR = 4 * jr + e; iIR = 4 * jr + 2 + e; iRI = 4 * (jr + d) + e; iII = 4 * (jr + d) + 2 + e;
              }
              emit1(bi, c, o, __uint_as_float(r[iRR >> 5][iRR & 31]), __uint_as_float(r[iRI >> 5][iRI & 31]),
                    __uint_as_float(r[iIR >> 5][iIR & 31]), __uint_as_float(r[iII >> 5][iII & 31]));
            }
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&bar_acc1_empty[buf]); mbar_arrive(&bar_y_full[buf]); }
    }
  } else {
    // ------------------------------------------------------------ epilogue 2
    const uint32_t q = warp & 3u;
    const int h = (int)(warp - 2 - C::kEpiWarps) >> 2;
    constexpr int kNC = C::N2 / 64;
    constexpr int BPW = (C::M2 == 64) ? 1 : 2 / C::EPW;
    constexpr int CH = (C::M2 == 64) ? kNC / C::EPW : kNC;
    const int ch0 = (C::M2 == 64 && C::EPW > 1) ? h * CH : 0;
    // column-pair outputs: per-thread bases of the element offset, the signal
    // and the staged-spectrum byte offset (epi_addr.cuh)
    constexpr int kE2W0 = 2 + C::kEpiWarps;
    using PosOff = detail::Fft2E2Pos<C, 0>;
    using SigOff = detail::Fft2E2Pos<C, 1>;
    using SpecOff = detail::Fft2E2Pos<C, 2>;
    constexpr int kPosK = kColPairs ? epi::addr_kind<PosOff, kE2W0, C::kEpiWarps, BPW, CH, 8, 2>() : 0;
    constexpr int kSigK = kColPairs ? epi::addr_kind<SigOff, kE2W0, C::kEpiWarps, BPW, CH, 8, 2>() : 0;
    constexpr int kSpecK = (kColPairs && kStageH) ? epi::addr_kind<SpecOff, kE2W0, C::kEpiWarps, BPW, CH, 8, 2>() : 0;
    uint32_t pos_base[BPW][kPosK == 1 ? 4 : 1], sig_base[BPW][kSigK == 1 ? 4 : 1], spec_base[BPW][kSpecK == 1 ? 4 : 1];
    // half2 column-blocked output with paired signal rows (block width 4)
    constexpr bool kPairRows = kEpi == kEpiBlocked && kOutHalf && C::NS <= 16 && C::C2 % 2 == 0;
    using KqOff = detail::Fft2E2PairRows<C, 0>;
    using ErOff = detail::Fft2E2PairRows<C, 1>;
    constexpr int kKqK = kPairRows ? epi::addr_kind<KqOff, kE2W0, C::kEpiWarps, BPW, CH, 4>() : 0;
    constexpr int kErK = kPairRows ? epi::addr_kind<ErOff, kE2W0, C::kEpiWarps, BPW, CH, 4>() : 0;
    uint32_t kq_base[BPW][kKqK == 1 ? 4 : 1], er_base[BPW][kErK == 1 ? 4 : 1];
    const uint32_t rows4 = (uint32_t)p.rows * 4u;
#pragma unroll
    for (int bi = 0; bi < BPW; ++bi) {
#pragma unroll
      for (int jh = 0; jh < 4; ++jh) {
        if (jh < (kPosK == 1 ? 4 : 1)) pos_base[bi][kPosK == 1 ? jh : 0] = PosOff::f((int)warp, (int)lane, bi, 0, 2 * jh);
        if (jh < (kSigK == 1 ? 4 : 1)) sig_base[bi][kSigK == 1 ? jh : 0] = SigOff::f((int)warp, (int)lane, bi, 0, 2 * jh);
        if (jh < (kSpecK == 1 ? 4 : 1)) spec_base[bi][kSpecK == 1 ? jh : 0] = SpecOff::f((int)warp, (int)lane, bi, 0, 2 * jh);
        if (jh < (kKqK == 1 ? 4 : 1)) kq_base[bi][kKqK == 1 ? jh : 0] = KqOff::f((int)warp, (int)lane, bi, 0, jh);
        if (jh < (kErK == 1 ? 4 : 1)) er_base[bi][kErK == 1 ? jh : 0] = ErOff::f((int)warp, (int)lane, bi, 0, jh);
      }
    }
    for (int i = 0; i < my_tiles; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int buf = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      const bool full_tile = (tile + 1) * C::T <= batch;   // no per-output bounds test
      if (!mbar_wait_warp(&bar_acc2_full[buf], ph, p.err, kDevTimeoutEpilogue)) break;
      const int hs = kStageH ? i % (C::HS > 0 ? C::HS : 1) : 0;
      if constexpr (kStageH)
        if (!mbar_wait_warp(&bar_h_full[hs], (uint32_t)(i / C::HS) & 1u, p.err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t hbase = smem_u32(smem + C::OFF_H + hs * C::SPEC_BYTES);
      const long long sig0 = tile * C::T;
      // conv2d modes: all T signals of a tile lie in one image (R % T == 0,
      // checked by the host), so the image bookkeeping is per tile.
      long long img = 0, r0 = 0;
      float osc = 1.f, osc2 = 1.f;      // range scale osc * osc2 of the half2 2-D convolution (1 otherwise)
      const float2* spec_t = nullptr;   // kEpiMulNatural: spectrum rows of this tile
      float* y0 = nullptr;              // kEpiUnpackPair: output rows of images b, b+1
      float* y1 = nullptr;
      if constexpr (kEpi != kEpiNatural) {
        img = sig0 / p.rows;
        r0 = sig0 - img * p.rows;
        const long long pg = p.pair0 + img, ch = pg / p.ppc, b = 2 * (pg - ch * p.ppc);
        if constexpr (kEpi == kEpiMulNatural) spec_t = p.spec + (ch * p.rows + r0) * C::N;
        if (p.conv_exp) {
          const int* e = p.conv_exp;
          const int e1 = e[2 + (pg - p.pair0)];
          const int se = p.conv_pass == 1 ? e1 : p.conv_pass == 2 ? e[0] : p.conv_pass == 3 ? e[1] : -(e1 + e[0] + e[1]);
          // e1, e2, e3 each lie within pow2f's exact range (+-120); the
          // unscale -(e1 + e2 + e3) of the last pass can leave it for a
          // representable output (inputs and spectra both large) and is
          // applied as two exact factors there
          if (kEpi == kEpiUnpackPair) {
            osc = detail::pow2f(se >> 1);
            osc2 = detail::pow2f(se - (se >> 1));
          } else {
            osc = detail::pow2f(se);
          }
        }
        if constexpr (kEpi == kEpiUnpackPair) {
          y0 = reinterpret_cast<float*>(p.out) + ((b * p.chans + ch) * p.rows + r0) * C::N;
          if (b + 1 < p.nimg_b) y1 = y0 + (long long)p.chans * p.rows * C::N;
        }
      }
#pragma unroll
      for (int bi = 0; bi < BPW; ++bi) {
        const int block = (C::M2 == 64) ? (int)q : (int)(2 * q) + h * BPW + bi;
        const uint32_t lanes = (C::M2 == 64) ? 32u * q + 16u * buf : 32u * q + 16u * (uint32_t)(h * BPW + bi);
        const uint32_t cols = 256u + ((C::M2 == 64) ? 0u : (uint32_t)(buf * C::N2));
        const int rp = block * 8 + (int)(lane >> 2);
        const int g2 = rp / C::NA, ka = rp % C::NA;
        if constexpr (kColPairs) {
          // iterations j (even) and j + 1 hold outputs k0 = NS ka + 8m + 2l
          // and k0 + 1 of one signal (stage2_col_pair)
          constexpr int kVec = kOutHalf ? 8 : 16;   // bytes of two complex outputs
          const bool vec_ok = kEpi != kEpiNatural || (reinterpret_cast<uintptr_t>(p.out) & (kVec - 1)) == 0;
          // 32-column pieces.  The 2-D convolution's passes load the next piece
          // while this one is processed (faster there); the C2C transform loads
          // whole 64-column chunks (the overlapped form measured 4-9 % slower
          // for half2 N = 256 and 512).
          constexpr bool kOverlap2 = !(kEpi == kEpiNatural && kIn == kInNatural);
          constexpr int NIT2 = kOverlap2 ? CH * 2 : CH;
          uint32_t rb[2][16];
          if constexpr (kOverlap2) tmem_ld_16x256b_x4(tmem + (lanes << 16) + cols + (uint32_t)ch0 * 64u, rb[0]);
#pragma unroll
          for (int it = 0; it < NIT2; ++it) {
            uint32_t rw[32];
            const uint32_t* r;
            int c, jlo;
            if constexpr (kOverlap2) {
              tmem_wait_ld();
              tmem_regs_ready(rb[it & 1]);
              if (it + 1 < NIT2)
                tmem_ld_16x256b_x4(tmem + (lanes << 16) + cols + (uint32_t)(ch0 + (it + 1) / 2) * 64u + 32u * (uint32_t)((it + 1) & 1),
                                   rb[(it + 1) & 1]);
              r = rb[it & 1];
              c = it / 2;
              jlo = 4 * (it & 1);
            } else {
              tmem_ld_16x256b_x8(tmem + (lanes << 16) + cols + (uint32_t)(ch0 + it) * 64u, rw);
              tmem_wait_ld();
              r = rw;
              c = it;
              jlo = 0;
            }
#pragma unroll
            for (int j = jlo; j < jlo + (kOverlap2 ? 4 : 8); j += 2) {
              // element offset sl * N + k0 and signal sl from per-thread bases
              // (epi_addr.cuh; the generic forms otherwise)
              uint32_t pos, sl_u, sbyte = 0u;
              if constexpr (kPosK != 0) pos = pos_base[bi][kPosK == 1 ? j / 2 : 0] + epi::addr_delta<PosOff, kE2W0, kPosK>(bi, c, j);
              else pos = PosOff::f((int)warp, (int)lane, bi, c, j);
              if constexpr (kSigK != 0) sl_u = sig_base[bi][kSigK == 1 ? j / 2 : 0] + epi::addr_delta<SigOff, kE2W0, kSigK>(bi, c, j);
              else sl_u = SigOff::f((int)warp, (int)lane, bi, c, j);
              if constexpr (kStageH) {
                if constexpr (kSpecK != 0) sbyte = spec_base[bi][kSpecK == 1 ? j / 2 : 0] + epi::addr_delta<SpecOff, kE2W0, kSpecK>(bi, c, j);
                else sbyte = SpecOff::f((int)warp, (int)lane, bi, c, j);
              }
              const int sl = (int)sl_u;
              float xr[2], xi[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int jj = kOverlap2 ? (j + e) & 3 : j + e;   // register group in r
                const float rr = __uint_as_float(r[4 * jj + 0]), ri = __uint_as_float(r[4 * jj + 1]);
                const float ir = __uint_as_float(r[4 * jj + 2]), ii = __uint_as_float(r[4 * jj + 3]);
                xr[e] = rr - ii;
                xi[e] = ir + ri;
              }
              if (full_tile || sig0 + sl < batch) {
                if constexpr (kEpi == kEpiUnpackPair) {
                  // fp32 real outputs: Re -> image b, Im -> image b + 1
                  *reinterpret_cast<float2*>(y0 + pos) = make_float2(xr[0] * osc * osc2, xr[1] * osc * osc2);
                  if (y1) *reinterpret_cast<float2*>(y1 + pos) = make_float2(xi[0] * osc * osc2, xi[1] * osc * osc2);
                } else {
                  if constexpr (kEpi == kEpiMulNatural) {
                    // spectrum values at k0 (x, y) and k0 + 1 (z, w): one 16-B piece
                    float4 w;
                    if constexpr (kStageH) {
                      w = ld_shared_v4f(hbase + sbyte);
                    } else {
                      w = __ldg(reinterpret_cast<const float4*>(spec_t + pos));
                    }
                    w.x *= osc; w.y *= osc; w.z *= osc; w.w *= osc;
                    const float a0 = xr[0] * w.x - xi[0] * w.y, b0 = xr[0] * w.y + xi[0] * w.x;
                    const float a1 = xr[1] * w.z - xi[1] * w.w, b1 = xr[1] * w.w + xi[1] * w.z;
                    xr[0] = a0; xi[0] = b0; xr[1] = a1; xi[1] = b1;
                  }
                  if constexpr (kOutHalf) {
                    __half2 h0 = __floats2half2_rn(xr[0], xi[0]), h1 = __floats2half2_rn(xr[1], xi[1]);
                    uint32_t* dst = reinterpret_cast<uint32_t*>(p.out) + sig0 * C::N + pos;
                    const uint32_t v0 = *reinterpret_cast<uint32_t*>(&h0), v1 = *reinterpret_cast<uint32_t*>(&h1);
                    if (vec_ok) *reinterpret_cast<uint2*>(dst) = make_uint2(v0, v1);
                    else { dst[0] = v0; dst[1] = v1; }   // output only 4-byte aligned
                  } else {
                    float2* dst = reinterpret_cast<float2*>(p.out) + sig0 * C::N + pos;
                    if (vec_ok) *reinterpret_cast<float4*>(dst) = make_float4(xr[0], xi[0], xr[1], xi[1]);
                    else { dst[0] = make_float2(xr[0], xi[0]); dst[1] = make_float2(xr[1], xi[1]); }
                  }
                }
              }
            }
          }
        } else {
        // half2 column-blocked output with Cb = 4 (one block row = 16 bytes):
        // signal rows sl, sl+1 of one output k are neighbours in the layout,
        // and a thread holds both (iterations j and j + NS/4).  Two quad
        // shuffles per value let each lane store 8 bytes, so one store
        // instruction writes whole 32-byte sectors.
        const bool pair_rows = kPairRows && p.blk_log2 == 2;
        // tile base of the paired-row blocked output: img N rows + r0 * 4 elements
        uint32_t* const blk_out = reinterpret_cast<uint32_t*>(p.out) + (img * C::N * p.rows + r0 * 4);
        if constexpr (kPairRows && (C::NS == 16 || C::NS == 8)) {
          if (pair_rows) {
            // Stored iteration j pairs with j + PJ (PJ = NS / 4).  Pieces of 16
            // registers hold column groups {j0, j0 + 1, j0 + PJ, j0 + PJ + 1}
            // (two 16-column loads), the next piece loading while this one is
            // processed.
            constexpr int PJ = C::NS / 4;
            const uint32_t l4 = lane & 3u, qbase = lane & ~3u;
            const uint32_t s0 = qbase + ((2u * l4) & 3u), s1 = qbase + ((2u * l4 + 1u) & 3u);
            const bool first_row = l4 < 2u;
            constexpr int NIT = CH * 2;
            // first stored iteration of piece it: PJ = 4 -> 2 (it & 1); PJ = 2 -> 4 (it & 1)
            auto j0_of = [](int it) { return (PJ == 4 ? 2 : 4) * (it & 1); };
            auto piece = [&](int it, uint32_t (&v)[16]) {
              const uint32_t a = tmem + (lanes << 16) + cols + (uint32_t)(ch0 + it / 2) * 64u + 8u * (uint32_t)j0_of(it);
              tmem_ld_16x256b_x2(a, *reinterpret_cast<uint32_t(*)[8]>(&v[0]));
              tmem_ld_16x256b_x2(a + 8u * PJ, *reinterpret_cast<uint32_t(*)[8]>(&v[8]));
            };
            uint32_t rb[2][16];
            piece(0, rb[0]);
#pragma unroll
            for (int it = 0; it < NIT; ++it) {
              tmem_wait_ld();
              tmem_regs_ready(rb[it & 1]);
              if (it + 1 < NIT) piece(it + 1, rb[(it + 1) & 1]);
              const int c = it / 2;
#pragma unroll
              for (int jq = 0; jq < 2; ++jq) {
                const int j = j0_of(it) + jq;
                const int jv = (j / (2 * PJ)) * PJ + j % PJ;
                uint32_t kq, er;
                if constexpr (kKqK != 0) kq = kq_base[bi][kKqK == 1 ? jv : 0] + epi::addr_delta<KqOff, kE2W0, kKqK>(bi, c, jv);
                else kq = KqOff::f((int)warp, (int)lane, bi, c, jv);
                if constexpr (kErK != 0) er = er_base[bi][kErK == 1 ? jv : 0] + epi::addr_delta<ErOff, kE2W0, kErK>(bi, c, jv);
                else er = ErOff::f((int)warp, (int)lane, bi, c, jv);
                uint32_t v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const uint32_t* g = &rb[it & 1][8 * e + 4 * jq];   // group j (e = 0) or j + PJ (e = 1)
                  const float rr = __uint_as_float(g[0]), ri = __uint_as_float(g[1]);
                  const float ir = __uint_as_float(g[2]), ii = __uint_as_float(g[3]);
                  __half2 hh = __floats2half2_rn((rr - ii) * osc, (ir + ri) * osc);
                  v[e] = *reinterpret_cast<uint32_t*>(&hh);
                }
                const uint32_t a0 = __shfl_sync(0xffffffffu, v[0], s0), b0 = __shfl_sync(0xffffffffu, v[1], s0);
                const uint32_t a1 = __shfl_sync(0xffffffffu, v[0], s1), b1 = __shfl_sync(0xffffffffu, v[1], s1);
                *reinterpret_cast<uint2*>(blk_out + (kq * rows4 + er)) =
                    make_uint2(first_row ? a0 : b0, first_row ? a1 : b1);
              }
            }
            continue;
          }
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          uint32_t r[32];
          tmem_ld_16x256b_x8(tmem + (lanes << 16) + cols + (ch0 + c) * 64, r);
          tmem_wait_ld();
          if constexpr (kPairRows) {
            if (pair_rows) {
              constexpr int PJ = C::NS / 4;
              const uint32_t l4 = lane & 3u, qbase = lane & ~3u;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if ((j / PJ) % 2 != 0) continue;
                const int jv = (j / (2 * PJ)) * PJ + j % PJ;
                // block row k >> 2 and in-row element offset from per-thread
                // bases (epi_addr.cuh), or the generic forms
                uint32_t kq, er;
                if constexpr (kKqK != 0) kq = kq_base[bi][kKqK == 1 ? jv : 0] + epi::addr_delta<KqOff, kE2W0, kKqK>(bi, c, jv);
                else kq = KqOff::f((int)warp, (int)lane, bi, c, jv);
                if constexpr (kErK != 0) er = er_base[bi][kErK == 1 ? jv : 0] + epi::addr_delta<ErOff, kE2W0, kErK>(bi, c, jv);
                else er = ErOff::f((int)warp, (int)lane, bi, c, jv);
                uint32_t v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int jj = j + e * PJ;
                  const float rr = __uint_as_float(r[4 * jj + 0]), ri = __uint_as_float(r[4 * jj + 1]);
                  const float ir = __uint_as_float(r[4 * jj + 2]), ii = __uint_as_float(r[4 * jj + 3]);
                  __half2 hh = __floats2half2_rn((rr - ii) * osc, (ir + ri) * osc);
                  v[e] = *reinterpret_cast<uint32_t*>(&hh);
                }
                // lane l of the quad stores row sl + l/2, complex pair 2 (l%2), 2 (l%2) + 1
                const uint32_t s0 = qbase + ((2u * l4) & 3u), s1 = qbase + ((2u * l4 + 1u) & 3u);
                const uint32_t a0 = __shfl_sync(0xffffffffu, v[0], s0), b0 = __shfl_sync(0xffffffffu, v[1], s0);
                const uint32_t a1 = __shfl_sync(0xffffffffu, v[0], s1), b1 = __shfl_sync(0xffffffffu, v[1], s1);
                const bool first_row = l4 < 2u;
                // ((img N + k) >> 2) rows 4 + (r0 + sl + row) 4 + 2 (l4 & 1), N a multiple of 4
                *reinterpret_cast<uint2*>(blk_out + (kq * rows4 + er)) =
                    make_uint2(first_row ? a0 : b0, first_row ? a1 : b1);
              }
              continue;
            }
          }
          // half2 spectrum products (staged spectrum): iterations j and j + 1
          // hold outputs k and k + 4 of one signal, so a quad shuffle gives
          // each lane 8 contiguous bytes and the quad a whole 32-byte sector.
          // Conv-mode tiles are never partial.  (Column pairs, which need no
          // shuffles, measured 20 % slower here: their 16-B spectrum loads
          // from the staged tile.)
          constexpr bool kPairK = kEpi == kEpiMulNatural && kOutHalf && kStageH && C::NS % 8 == 0;
          if constexpr (kPairK) {
            const uint32_t l4 = lane & 3u, qbase = lane & ~3u;
            const uint32_t s0 = qbase + ((2u * l4) & 3u), s1 = qbase + ((2u * l4 + 1u) & 3u);
            const bool first = l4 < 2u;
            auto pair_store = [&](uint32_t* dst, uint32_t va, uint32_t vb) {
              const uint32_t a0 = __shfl_sync(0xffffffffu, va, s0), b0 = __shfl_sync(0xffffffffu, vb, s0);
              const uint32_t a1 = __shfl_sync(0xffffffffu, va, s1), b1 = __shfl_sync(0xffffffffu, vb, s1);
              *reinterpret_cast<uint2*>(dst + 2 * l4) = make_uint2(first ? a0 : b0, first ? a1 : b1);
            };
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const int pidx = 4 * ((ch0 + c) * 8 + j) + (int)l4;
              const int c2 = pidx / C::NS, ks = pidx % C::NS;    // ks % 8 < 4: k + 4 is this signal's too
              const int sl = g2 * C::C2 + c2;
              const int kq = C::NS * ka + ks - (int)l4;           // the quad's first output
              float xr[2], xi[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int jj = j + e;
                const float rr = __uint_as_float(r[4 * jj + 0]), ri = __uint_as_float(r[4 * jj + 1]);
                const float ir = __uint_as_float(r[4 * jj + 2]), ii = __uint_as_float(r[4 * jj + 3]);
                xr[e] = rr - ii;
                xi[e] = ir + ri;
              }
              if constexpr (kEpi == kEpiMulNatural) {
                uint32_t v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const uint32_t byte = (uint32_t)(sl * C::N + kq + (int)l4 + 4 * e) * 8u;
                  float2 w = ld_shared_v2f(hbase + (byte ^ (((byte >> 7) & 7u) << 4)));
                  w.x *= osc;
                  w.y *= osc;
                  __half2 hh = __floats2half2_rn(xr[e] * w.x - xi[e] * w.y, xr[e] * w.y + xi[e] * w.x);
                  v[e] = *reinterpret_cast<uint32_t*>(&hh);
                }
                pair_store(reinterpret_cast<uint32_t*>(p.out) + (sig0 + sl) * C::N + kq, v[0], v[1]);
              } else {
                pair_store(reinterpret_cast<uint32_t*>(y0 + sl * C::N + kq), __float_as_uint(xr[0] * osc * osc2),
                           __float_as_uint(xr[1] * osc * osc2));
                if (y1)
                  pair_store(reinterpret_cast<uint32_t*>(y1 + sl * C::N + kq), __float_as_uint(xi[0] * osc * osc2),
                             __float_as_uint(xi[1] * osc * osc2));
              }
            }
            continue;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int pidx = 4 * ((ch0 + c) * 8 + j) + (int)(lane & 3u);
            const int c2 = pidx / C::NS, ks = pidx % C::NS;
            const float rr = __uint_as_float(r[4 * j + 0]), ri = __uint_as_float(r[4 * j + 1]);
            const float ir = __uint_as_float(r[4 * j + 2]), ii = __uint_as_float(r[4 * j + 3]);
            const int sl = g2 * C::C2 + c2;   // signal within the tile
            if (sig0 + sl < batch) {
              const int k = C::NS * ka + ks;
              float xr = rr - ii, xi = ir + ri;
              if constexpr (kEpi == kEpiUnpackPair) {
                xr = xr * osc * osc2;
                xi = xi * osc * osc2;
              } else if constexpr (kEpi != kEpiNatural && kEpi != kEpiMulNatural) {
                xr *= osc;
                xi *= osc;
              }
              if constexpr (kEpi == kEpiNatural) {
                detail::store_out<kOutHalf>(p.out, (sig0 + sl) * C::N + k, xr, xi);
              } else if constexpr (kEpi == kEpiMulNatural) {
                float2 w;
                if constexpr (kStageH) {
                  // 128-B-swizzled staging: 16-B chunk XOR (128-B line % 8)
                  const uint32_t byte = (uint32_t)(sl * C::N + k) * 8u;
                  w = ld_shared_v2f(hbase + (byte ^ (((byte >> 7) & 7u) << 4)));
                } else {
                  w = __ldg(spec_t + sl * C::N + k);
                }
                w.x *= osc;
                w.y *= osc;
                detail::store_out<kOutHalf>(p.out, (sig0 + sl) * C::N + k, xr * w.x - xi * w.y, xr * w.y + xi * w.x);
              } else if constexpr (kEpi == kEpiBlocked) {
                const int lb = p.blk_log2;
                const long long o = (((img * C::N + k) >> lb) * p.rows + r0 + sl) * (1LL << lb) + (k & ((1 << lb) - 1));
                detail::store_out<kOutHalf>(p.out, o, xr, xi);
              } else {
                // fp32 real outputs: Re -> image b, Im -> image b + 1
                y0[sl * C::N + k] = xr;
                if (y1) y1[sl * C::N + k] = xi;
              }
            }
          }
        }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar_acc2_empty[buf]);
        if constexpr (kStageH) mbar_arrive(&bar_h_empty[hs]);
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// One-stage kernel for N = 64: data tile (128 signals) is the K-major A
// operand, the real 128 x 128 DFT matrix (rows (k, re|im), K = (j, re|im))
// is B.  TMEM row = one signal's full interleaved output.
// ---------------------------------------------------------------------------
template <bool kHalf>
struct Dft1Cfg {
  using D = DType<kHalf>;
  static constexpr bool kIsHalf = kHalf;
  static constexpr int N = 64, T = 128;                 // signals per tile = MMA M
  static constexpr int ESZ = D::kEsz, E = D::kElemsPer128B;
  static constexpr int KATOMS = (2 * N * ESZ) / 128;     // 128-B K atoms per row
  static constexpr int TILE_BYTES = T * 2 * N * ESZ;      // also the B size
  static constexpr int B_BYTES = 2 * N * 2 * N * ESZ;
  static constexpr int KSTEPS = 2 * N / D::kMmaK;
  static constexpr int SIN = kHalf ? 4 : 2;
  // float2 C2C: outputs leave through two dedicated 16 KB staging slabs (one
  // 32-column chunk each) so an input slot is free as soon as its MMAs end;
  // half2 and window mode stage into the input slot they came from.
  static constexpr int STG_BYTES = T * 128;
  static constexpr int NSTG = kHalf ? 0 : 2;
  static constexpr uint32_t OFF_B = 0;
  static constexpr uint32_t OFF_IN = B_BYTES;
  static constexpr uint32_t OFF_STG = OFF_IN + SIN * TILE_BYTES;
  static constexpr uint32_t SMEM_BYTES = exclusive_smem(OFF_STG + NSTG * STG_BYTES + 1024);
  static_assert(SMEM_BYTES + 512 <= 232448, "shared memory budget");
  static constexpr int kThreads = 192;                   // producer, MMA, 4 epilogue warps
};

template <class C, bool kWin = false>
__global__ void __launch_bounds__(C::kThreads, 1)
dft1_kernel(const __grid_constant__ CUtensorMap tmap_in, const __grid_constant__ CUtensorMap tmap_out,
            const FftParams p, int use_tma_store) {
  using namespace sm100;
  using D = typename C::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in_full[C::SIN], bar_in_empty[C::SIN];
  __shared__ uint64_t bar_acc_full[2], bar_acc_empty[2], bar_staged[2], bar_const, bar_done;
  __shared__ uint64_t bar_stg_full[2], bar_stg_free[2];
  __shared__ uint32_t tmem_slot;
  // separate output staging (float2 C2C, TMA store available): the MMA thread
  // releases each input slot by tcgen05.commit when the slot's MMAs are done
  const bool sep = !C::kIsHalf && !kWin && use_tma_store;

  const uint32_t warp = warp_id(), lane = lane_id();
  const long long batch = p.batch;
  const long long num_tiles = (batch + C::T - 1) / C::T;
  const int my_tiles = (int)((num_tiles > blockIdx.x) ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::SIN; ++i) { mbar_init(&bar_in_full[i], 1); mbar_init(&bar_in_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_acc_full[i], 1); mbar_init(&bar_acc_empty[i], 4); mbar_init(&bar_staged[i], 4);
      mbar_init(&bar_stg_full[i], 4); mbar_init(&bar_stg_free[i], 1);
    }
    mbar_init(&bar_const, 1);
    mbar_init(&bar_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&tmem_slot, 256); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  // element (sig, col) of a tile: K-major SW128, [katom][sig][128 B]
  auto tile_off = [](int sig, int col) -> uint32_t {
    return (uint32_t)(col / C::E) * (C::T * 128u) + sw128((uint32_t)sig * 128u + (col % C::E) * C::ESZ);
  };
  // Window mode: a tile whose 128 windows lie in one sequence and wholly
  // inside it moves by one TMA box in and one bulk copy out (when the host
  // found the strides 16-byte aligned); other tiles take thread loads/stores.
  auto interior = [&](long long tile, long long& b0, long long& t0) -> bool {
    const long long w0 = tile * C::T;
    b0 = w0 / p.win_per_sig;
    t0 = w0 - b0 * p.win_per_sig;
    return t0 + C::T <= p.win_per_sig && t0 + C::T - 1 <= p.win_tmax;
  };

  if (warp == 0) {
    if (lane == 0) {
      if (p.use_tma) tma_prefetch_desc(&tmap_in);
      mbar_arrive_expect_tx(&bar_const, C::B_BYTES);
      bulk_load(smem + C::OFF_B, p.a1, C::B_BYTES, &bar_const);
    }
    for (int i = 0; i < my_tiles; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int slot = i % C::SIN;
      if (!mbar_wait_warp(&bar_in_empty[slot], ((uint32_t)(i / C::SIN) & 1u) ^ 1u, p.err, kDevTimeoutProducer)) break;
      uint8_t* dst = smem + C::OFF_IN + slot * C::TILE_BYTES;
      long long wb0 = 0, wt0 = 0;
      if (!kWin && p.use_tma) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
          tma_load_3d(dst, &tmap_in, &bar_in_full[slot], 0, (int)(tile * C::T), 0);
        }
        __syncwarp();
      } else if (kWin && p.use_tma && interior(tile, wb0, wt0)) {
        // 128 windows = rows of a 4-D map {element, window (stride V), atom, sequence}
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
          tma_load_4d(dst, &tmap_in, &bar_in_full[slot], 0, (int)wt0, 0, (int)wb0);
        }
        __syncwarp();
      } else if constexpr (kWin) {
        // overlapping windows by thread loads, zero past each sequence's end;
        // each window's 64 elements are contiguous (two per lane)
        const long long w0 = tile * C::T;
        const uint32_t base = smem_u32(dst);
        long long b = w0 / p.win_per_sig, t = w0 - b * p.win_per_sig;
        for (int sig = 0; sig < C::T; ++sig) {
          const bool live = w0 + sig < batch;
#pragma unroll
          for (int h = 0; h < C::N / 32; ++h) {
            const int n = (int)lane + 32 * h;
            const long long e = t * p.win_stride + n;
            const bool ok = live && e < p.in_len;
            const long long gi = b * p.in_len + e;
            const uint32_t off = tile_off(sig, 2 * n);
            if constexpr (C::kIsHalf) {
              st_shared_b32(base + off, ok ? __ldg(reinterpret_cast<const unsigned int*>(p.in) + gi) : 0u);
            } else {
              const float2 v = ok ? __ldg(reinterpret_cast<const float2*>(p.in) + gi) : make_float2(0.f, 0.f);
              st_shared_v2(base + off, v.x, v.y);
            }
          }
          if (++t == p.win_per_sig) { t = 0; ++b; }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_in_full[slot]);
      } else {
        const long long sig0 = tile * C::T;
        const uint32_t base = smem_u32(dst);
        for (int idx = lane; idx < C::T * C::N; idx += 32) {
          const int sig = idx / C::N, n = idx % C::N;
          const uint32_t off = tile_off(sig, 2 * n);
          if (sig0 + sig < batch) {
            if constexpr (C::kIsHalf) {
              st_shared_b32(base + off, __ldg(reinterpret_cast<const unsigned int*>(p.in) + (sig0 + sig) * C::N + n));
            } else {
              const float2 v = __ldg(reinterpret_cast<const float2*>(p.in) + (sig0 + sig) * C::N + n);
              st_shared_v2(base + off, v.x, v.y);
            }
          } else {
            if constexpr (C::kIsHalf) st_shared_b32(base + off, 0u);
            else st_shared_v2(base + off, 0.f, 0.f);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_in_full[slot]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&bar_const, 0, p.err, kDevTimeoutMma);
      const uint32_t bsm = smem_u32(smem + C::OFF_B);
      const uint32_t idesc = instr_desc(D::kFmt, 128, 2 * C::N, 0, 0);
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int slot = i % C::SIN, buf = i & 1;
        if (!mbar_wait(&bar_in_full[slot], (uint32_t)(i / C::SIN) & 1u, p.err, kDevTimeoutMma)) break;
        if (!mbar_wait(&bar_acc_empty[buf], ((uint32_t)(i >> 1) & 1u) ^ 1u, p.err, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + C::OFF_IN + slot * C::TILE_BYTES);
        const uint32_t d = tmem + (uint32_t)(buf * 128);
        constexpr int kStepsPerAtom = 128 / (D::kMmaK * C::ESZ);
#pragma unroll
        for (int k = 0; k < C::KSTEPS; ++k) {
          const int ka = k / kStepsPerAtom, kin = k % kStepsPerAtom;
          const uint32_t koff = ka * (C::T * 128u) + kin * 32u;
          const uint64_t ad = smem_desc(a + koff, 16, 1024, kSw128);
          const uint64_t bd = smem_desc(bsm + koff, 16, 1024, kSw128);
          if constexpr (C::kIsHalf) umma_f16(d, ad, bd, idesc, k > 0);
          else umma_tf32(d, ad, bd, idesc, k > 0);
        }
        umma_commit(&bar_acc_full[buf]);
        if (sep) umma_commit(&bar_in_empty[slot]);
      }
      umma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.err, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // epilogue: warp -> quadrant q = warp & 3, thread = signal 32q + lane
    const uint32_t q = warp & 3u;
    int pending_slot = -1;
    if (sep) {
      // Chunk g = 4 i + c (32 accumulator columns = 16 outputs of each of the
      // tile's signals) goes through staging slab g & 1: every warp waits for
      // the slab to be free, writes its 32 rows and arrives on stg_full; warp
      // 2 lane 0 stores the slab (box {32, T, 1}) and, once the store of chunk
      // g - 1 has read its slab, frees that one.
      const int sig = (int)(32 * q + lane);
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const long long tile = blockIdx.x + (long long)i * gridDim.x;
        const int buf = i & 1;
        if (!mbar_wait_warp(&bar_acc_full[buf], (uint32_t)(i >> 1) & 1u, p.err, kDevTimeoutEpilogue)) break;
        tc_fence_after();
#pragma unroll 1
        for (int chunk = 0; chunk < 4; ++chunk) {
          const int g = 4 * i + chunk, sb = g & 1;
          const uint32_t use = (uint32_t)(g >> 1);
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + ((32u * q) << 16) + (uint32_t)(buf * 128 + chunk * 32), r);
          tmem_wait_ld();
          if (chunk == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_acc_empty[buf]);
          }
          if (!mbar_wait_warp(&bar_stg_free[sb], (use & 1u) ^ 1u, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
          const uint32_t sbase = smem_u32(smem + C::OFF_STG + sb * C::STG_BYTES);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            st_shared_v4(sbase + sw128((uint32_t)sig * 128u + 16u * v), r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_stg_full[sb]);
          if (warp == 2 && lane == 0) {
            if (mbar_wait(&bar_stg_full[sb], use & 1u, p.err, kDevTimeoutEpilogue)) {
              tma_store_3d(&tmap_out, smem + C::OFF_STG + sb * C::STG_BYTES, 0, (int)(tile * C::T), chunk);
              bulk_commit_group();
              bulk_wait_group_read<1>();   // chunk g - 1's store has read its slab
              if (g >= 1) mbar_arrive(&bar_stg_free[sb ^ 1]);
            } else {
              ok = false;
            }
          }
          ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
          if (!ok) break;
        }
      }
      if (warp == 2 && lane == 0) bulk_wait_group<0>();
    }
    for (int i = 0; !sep && i < my_tiles; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int slot = i % C::SIN, buf = i & 1;
      if (!mbar_wait_warp(&bar_acc_full[buf], (uint32_t)(i >> 1) & 1u, p.err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      // the MMA that filled acc[buf] has finished reading in[slot]; reuse it
      // as the output staging tile.
      uint8_t* stage = smem + C::OFF_IN + slot * C::TILE_BYTES;
      const uint32_t sbase = smem_u32(stage);
      const int sig = (int)(32 * q + lane);
      const long long gsig = tile * C::T + sig;
      long long wb0 = 0, wt0 = 0;
      const bool win_bulk = kWin && use_tma_store && interior(tile, wb0, wt0);
#pragma unroll 1
      for (int chunk = 0; chunk < 4; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((32u * q) << 16) + (uint32_t)(buf * 128 + chunk * 32), r);
        tmem_wait_ld();
        if (win_bulk) {
          // window sig's first V outputs, contiguous after window sig-1's.
          // The bulk path has V * (bytes per complex) % 16 == 0 (host), so
          // they go out as 16-byte vectors: 4 half2 or 2 float2 outputs per
          // store.  One output per store put neighbouring lanes V * 4 bytes
          // apart, an 8-way bank conflict for V = 56 (ncu: 3.98 M conflicts
          // in 4.50 M store wavefronts).
          constexpr int kPer = 16 / (2 * C::ESZ);   // outputs per 16-byte store
#pragma unroll
          for (int v = 0; v < 16 / kPer; ++v) {
            const int j = chunk * 16 + kPer * v;
            if (j < p.win_stride) {
              const uint32_t o = (uint32_t)(sig * p.win_stride + j) * (uint32_t)(2 * C::ESZ);
              if constexpr (C::kIsHalf) {
                uint32_t h[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  __half2 t2 = __floats2half2_rn(__uint_as_float(r[2 * (4 * v + u)]),
                                                 __uint_as_float(r[2 * (4 * v + u) + 1]));
                  h[u] = *reinterpret_cast<uint32_t*>(&t2);
                }
                st_shared_v4(sbase + o, h[0], h[1], h[2], h[3]);
              } else {
                st_shared_v4(sbase + o, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
              }
            }
          }
        } else if (!kWin && use_tma_store) {
          if constexpr (C::kIsHalf) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t h[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                __half2 t2 = __floats2half2_rn(__uint_as_float(r[8 * v + 2 * u]), __uint_as_float(r[8 * v + 2 * u + 1]));
                h[u] = *reinterpret_cast<uint32_t*>(&t2);
              }
              st_shared_v4(sbase + tile_off(sig, chunk * 32 + 8 * v), h[0], h[1], h[2], h[3]);
            }
          } else {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              st_shared_v4(sbase + tile_off(sig, chunk * 32 + 4 * v), r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          }
        } else if (gsig < batch) {
          if constexpr (kWin) {
            // the window's first win_stride outputs that lie inside its sequence
            const long long b = gsig / p.win_per_sig, t = gsig - b * p.win_per_sig;
            const long long o0 = t * p.win_stride, rem = p.out_len - o0;
            const int lim = (int)(rem < p.win_stride ? rem : p.win_stride);
#pragma unroll
            for (int u = 0; u < 16; ++u)
              if (chunk * 16 + u < lim)
                detail::store_out<C::kIsHalf>(p.out, b * p.out_len + o0 + chunk * 16 + u, __uint_as_float(r[2 * u]),
                                              __uint_as_float(r[2 * u + 1]));
          } else {
#pragma unroll
            for (int u = 0; u < 16; ++u)
              detail::store_out<C::kIsHalf>(p.out, gsig * C::N + chunk * 16 + u, __uint_as_float(r[2 * u]),
                                            __uint_as_float(r[2 * u + 1]));
          }
        }
      }
      // Hand-off: each epilogue warp arrives on staged[buf] after its part of
      // the tile is in shared memory (and visible to the async proxy); one
      // thread then stores the tile and, one tile later, releases the
      // staging slot back to the producer.
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&bar_acc_empty[buf]); mbar_arrive(&bar_staged[buf]); }
      if (warp == 2) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&bar_staged[buf], (uint32_t)(i >> 1) & 1u, p.err, kDevTimeoutEpilogue);
        if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
        if (lane == 0) {
          if (win_bulk) {
            // the tile's outputs: one contiguous span of 128 V elements
            uint8_t* g = reinterpret_cast<uint8_t*>(p.out) +
                         (wb0 * p.out_len + wt0 * p.win_stride) * (long long)(2 * C::ESZ);
            bulk_store(g, stage, (uint32_t)(C::T * p.win_stride * 2 * C::ESZ));
            bulk_commit_group();
            bulk_wait_group_read<1>();
          } else if (!kWin && use_tma_store) {
            tma_store_3d(&tmap_out, stage, 0, (int)(tile * C::T), 0);
            bulk_commit_group();
            bulk_wait_group_read<1>();   // the previous tile's store has read its slot
          }
          if (pending_slot >= 0) mbar_arrive(&bar_in_empty[pending_slot]);
        }
        pending_slot = slot;
      }
      __syncwarp();
    }
    if (!sep && warp == 2 && lane == 0) {
      if (use_tma_store) bulk_wait_group<0>();   // (window mode: bulk stores)
      if (pending_slot >= 0) mbar_arrive(&bar_in_empty[pending_slot]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Failure-detection self-test: one thread waits on an mbarrier that nothing
// will ever arrive on; the bounded wait must give up after `limit_ns`,
// record kDevTimeoutOther in *err and let the kernel exit normally.
__global__ void wait_timeout_selftest_kernel(uint32_t* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
    sm100::mbar_wait_limit(&bar, 0, err, sm100::kDevTimeoutOther, limit_ns);
  }
}

}  // namespace thff
