// conv2d_fused.cuh — the column pass of the 2-D FFT convolution as ONE
// kernel: column FFT -> x filter spectrum -> column inverse FFT.
//
// Counterpart of the reference's fused column kernel conv1024_y_fwd_mul_inv
// (sample/conv2d/thunder.cu:111-163), which keeps the column spectrum on chip
// between the forward transform, the multiply and the inverse transform.
// Here each tile holds T column signals (length h) of one image pair, read in
// the column-blocked layout the row pass writes, and goes through four
// tcgen05 stages with the same factorization h = NS * NA as fft2_kernel:
//
//   S1 forward over s  (length NS, G1 groups, A1)   B1 = input tile (TMA)
//   E1 combine, twiddle w_h^(a ks)                   -> B2  [K row a ][c, ks]
//   S2 forward over a  (length NA, G2 groups, A2)   X[NS ka + ks]
//   E2 combine, x H[k2][NS ka + ks]                  -> B3  [K row ka][c, ks]
//   S3 inverse over ka (length NA, G2 groups, A2)   sine terms flipped in E3
//   E3 combine, twiddle w_h^-(ks ks')                -> B4  [K row ks][c, ks']
//   S4 inverse over ks (length NS, G1 groups, A4)   Z[NA ka' + ks']
//   E4 combine                                       -> column-blocked output
//
// The inverse uses the mirrored factorization (input index k = NS ka + ks
// read as a' + NS s' with a' = ks, s' = ka), so the forward output of S2 is
// already in the inverse's input order: E2 only writes each value to K row ka
// instead of ks, and no transpose is needed.  All four stages use forward DFT
// matrices; the inverse stages flip the sine terms in the epilogue combine.
// A4 is A1 with its K columns in the rotated order E3 writes (the same
// bank-conflict rotation as stage 2's, detail::stage2_rotation).
//
// The MMA thread runs S1(r), S2(r-1), S3(r-2), S4(r-3) in round r, one TMEM
// accumulator per stage; epilogue group A (E1, E3) and group B (E2, E4) each
// own half the epilogue warps.  The spectrum rows of a tile are staged by TMA
// like fft2_kernel's multiply mode.  Every wait is bounded (sm100.cuh).
#pragma once
#include "fft_kernels.cuh"

namespace thff {

template <bool kHalf, int kN>
struct Conv2dColCfg {
  using D = DType<kHalf>;
  using S = Fft2Shape<kHalf, kN>;
  static constexpr bool kIsHalf = kHalf;
  static constexpr int N = kN, NS = S::NS, NA = S::NA, G1 = S::G1, G2 = S::G2, T = S::T;
  static constexpr int ESZ = D::kEsz, E = D::kElemsPer128B;
  static constexpr int C1 = T / G1, C2 = T / G2;           // signals per column group, stages over s / a
  static constexpr int M1 = 2 * NS * G1, M2 = 2 * NA * G2; // MMA M: S1, S4 / S2, S3
  static constexpr int K1 = NS * G1, K2 = NA * G2;         // MMA K
  static constexpr int N1 = C1 * 2 * NA, N2 = C2 * 2 * NS; // MMA N (TMEM columns)
  static constexpr int TILE_BYTES = T * N * 2 * ESZ;
  static constexpr int A1_BYTES = M1 * K1 * ESZ, A2_BYTES = M2 * K2 * ESZ;
  static constexpr uint32_t LBO1 = K1 * 128, LBO2 = K2 * 128;  // B operands: stride between column atoms
  static constexpr int KSTEPS1 = K1 / D::kMmaK, KSTEPS2 = K2 / D::kMmaK;
  static constexpr uint32_t KSTEP_BYTES = D::kMmaK * 128;
  static constexpr int R2 = detail::stage2_rotation(kHalf, 0);  // K-row rotation of B2, B3, B4
  static constexpr bool kColPairs2 = NS % 8 == 0;  // E1 orders B2's columns for paired E2 outputs
  static constexpr bool kColPairs4 = NA % 8 == 0;  // E3 orders B4's columns for paired E4 outputs
  static_assert(kColPairs4, "NA is 16, 32 or 64");
  // Distinct stage matrices: A2 is A1 when both stages are the same DFT with
  // the same K order; A4 (NS, G1, rotation R2) is A1 without rotation, or A2
  // when the two stage lengths and groups agree.
  static constexpr bool kA2isA1 = R2 == 0 && NS == NA && G1 == G2;
  static constexpr bool kA4isA1 = R2 == 0;
  static constexpr bool kA4isA2 = !kA4isA1 && NS == NA && G1 == G2;
  __host__ __device__ static constexpr uint32_t al(uint32_t b) { return (b + 1023u) / 1024u * 1024u; }
  static constexpr uint32_t OFF_A1 = 0;
  static constexpr uint32_t OFF_A2 = kA2isA1 ? OFF_A1 : OFF_A1 + al(A1_BYTES);
  static constexpr uint32_t END_A2 = kA2isA1 ? al(A1_BYTES) : OFF_A2 + al(A2_BYTES);
  static constexpr uint32_t OFF_A4 = kA4isA1 ? OFF_A1 : (kA4isA2 ? OFF_A2 : END_A2);
  static constexpr uint32_t END_A = (kA4isA1 || kA4isA2) ? END_A2 : END_A2 + al(A1_BYTES);
  static constexpr uint32_t A_LOAD_BYTES =
      A1_BYTES + (kA2isA1 ? 0 : A2_BYTES) + ((kA4isA1 || kA4isA2) ? 0 : A1_BYTES);
  static constexpr int SPEC_BYTES = T * N * 8;             // a tile's spectrum rows (complex fp32)
  // input slots and spectrum slots: as many as fit (input first)
  static constexpr uint32_t kBudget = 232448u - 1024u /*align*/ - 1024u /*static*/;
  __host__ __device__ static constexpr uint32_t fixed_bytes() { return END_A + 3u * TILE_BYTES; }
  __host__ __device__ static constexpr int pick(int which) {
    const int sin0 = kHalf ? 4 : 2;
    for (int s = sin0; s >= 1; --s)
      for (int h = 2; h >= 1; --h)
        if (fixed_bytes() + (uint32_t)s * TILE_BYTES + (uint32_t)h * SPEC_BYTES <= kBudget) return which ? h : s;
    return 0;
  }
  static constexpr int SIN = pick(0), HS = pick(1);
  static_assert(SIN >= 1 && HS >= 1, "shared memory budget");
  static constexpr uint32_t OFF_IN = END_A;
  static constexpr uint32_t OFF_B = OFF_IN + SIN * TILE_BYTES;   // B2, B3, B4
  static constexpr uint32_t OFF_H = OFF_B + 3 * TILE_BYTES;
  static constexpr uint32_t SMEM_BYTES = exclusive_smem(OFF_H + HS * SPEC_BYTES + 1024);
  static_assert(SMEM_BYTES + 1024 <= 232448, "shared memory budget");
  static_assert(M1 == 64 || M1 == 128, "M1");
  static_assert(M2 == 64 || M2 == 128, "M2");
  static_assert(M1 == 64 ? N1 <= 256 : N1 <= 128, "TMEM: D1 and D4 share 256 columns");
  static_assert(M2 == 64 ? N2 <= 256 : N2 <= 128, "TMEM: D2 and D3 share 256 columns");
  // Epilogue warps per TMEM lane quadrant and group: two (18 warps, four
  // epilogue warps per scheduler to hide the TMEM, shared-memory and FMA
  // latencies of the epilogues; config 5 measured 1.47 ms for the pass with
  // one, 1.08 with two), except for float2 N >= 1024, whose per-thread
  // twiddles spill under the 96-register cap of 576 threads.
  static constexpr int EPW = (kHalf || kN <= 512) ? 2 : 1;
  static constexpr int kEpiWarps = 4 * EPW;                   // per epilogue group
  // Two MMA issuers: warp 1 issues stages 1 and 3, warp kMma2Warp (after the
  // epilogue warps) stages 2 and 4, so a wait or a stalled issue of one
  // stage does not hold up the others.
  static constexpr int kMma2Warp = 2 + 2 * kEpiWarps;
  static constexpr int kThreads = 32 * (kMma2Warp + 1);
  // TMEM accumulators: D1/D4 in columns [0, 256), D2/D3 in [256, 512); an
  // M = 64 pair shares its columns through lanes 0-15 / 16-31 of each
  // quadrant, an M = 128 pair splits the columns.
  __host__ __device__ static constexpr uint32_t lane_off(int m, int second) { return (m == 64 && second) ? 16u : 0u; }
  __host__ __device__ static constexpr uint32_t col_off(int m, int region, int second) {
    return 256u * (uint32_t)region + ((m == 128 && second) ? 128u : 0u);
  }
  // the input layout for encode_conv_input (column-blocked, as fft2's kInBlocked)
  static constexpr int kVariant = 0;
};

// Accumulator geometry of one stage for its epilogue warps (fft2_kernel's
// mapping): M = 64 -> one 16-row block per quadrant, its 64-column chunks
// split over the EPW warps of the quadrant; M = 128 -> two blocks per
// quadrant, split over the EPW warps.
template <int kM, int kNcols, int kEPW>
struct AccGeo {
  static constexpr int kNC = kNcols / 64;
  static constexpr int BPW = (kM == 64) ? 1 : 2 / kEPW;
  static constexpr int CH = (kM == 64) ? kNC / kEPW : kNC;
  static_assert(kM == 64 ? kNC % kEPW == 0 : 2 % kEPW == 0, "epilogue split");
  __host__ __device__ static constexpr int ch0(int h) { return (kM == 64 && kEPW > 1) ? h * CH : 0; }
  __host__ __device__ static constexpr int block(uint32_t q, int h, int bi) {
    return (kM == 64) ? (int)q : (int)(2 * q) + h * BPW + bi;
  }
  __device__ static uint32_t lanes(uint32_t q, int h, int bi, uint32_t loff) {
    return (kM == 64) ? 32u * q + loff : 32u * q + 16u * (uint32_t)(h * BPW + bi);
  }
};

// Write addresses of the four epilogues as functions of (warp, lane, row
// block bi, chunk c, 8-column group o) for epi::addr_kind (epi_addr.cuh).
// Group A is warps [2, 2 + kEpiWarps), group B the next kEpiWarps.
template <class C>
struct Conv2dColAddr {
  using D = typename C::D;
  // E1: byte offset in B2 of the twiddled stage-1 output
  struct E1 {
    __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int o) {
      using G = AccGeo<C::M1, C::N1, C::EPW>;
      const int q = warp & 3, h = (warp - 2) >> 2, l4 = lane & 3;
      const int rp = G::block((uint32_t)q, h, bi) * 8 + (lane >> 2);
      const int g1 = rp / C::NS, ks = rp % C::NS;
      const int pidx = 4 * ((G::ch0(h) + c) * 8 + o) + l4;
      const int a = pidx / C::C1, c1 = pidx % C::C1;
      const int sig = g1 * C::C1 + c1;
      const int g2 = sig / C::C2, c2 = sig % C::C2;
      const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + a);
      const int col = c2 * 2 * C::NS + 2 * (C::kColPairs2 ? detail::stage2_col_pair(ks) : ks);
      return (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
    }
  };
  // E3: byte offset in B4 of the twiddled inverse stage-1 output
  struct E3 {
    __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int o) {
      using G = AccGeo<C::M2, C::N2, C::EPW>;
      const int q = warp & 3, h = (warp - 2) >> 2, l4 = lane & 3;
      const int rp = G::block((uint32_t)q, h, bi) * 8 + (lane >> 2);
      const int g3 = rp / C::NA, ksp = rp % C::NA;
      const int pidx = 4 * ((G::ch0(h) + c) * 8 + o) + l4;
      const int c3 = pidx / C::NS, ap = pidx % C::NS;
      const int sig = g3 * C::C2 + c3;
      const int g4 = sig / C::C1, c4 = sig % C::C1;
      const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g4 * C::NS + ap);
      const int col = c4 * 2 * C::NA + 2 * detail::stage2_col_pair(ksp);
      return (uint32_t)(col / C::E) * C::LBO1 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
    }
  };
  // E2 (column pairs, o even): kWhat 0: byte offset in B3 of outputs k0,
  // k0 + 1; 1: their 128-B-swizzled byte offset in the staged spectrum tile
  template <int kWhat>
  struct E2 {
    __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int o) {
      using G = AccGeo<C::M2, C::N2, C::EPW>;
      const int q = warp & 3, h = (warp - 2 - C::kEpiWarps) >> 2, l4 = lane & 3;
      const int rp = G::block((uint32_t)q, h, bi) * 8 + (lane >> 2);
      const int g2 = rp / C::NA, ka = rp % C::NA;
      const int pidx = 4 * ((G::ch0(h) + c) * 8 + o) + l4;
      const int c2 = pidx / C::NS, pp = pidx % C::NS;
      const int ks0 = (pp & ~7) + 2 * l4;
      if (kWhat == 1) {
        const uint32_t byte = (uint32_t)((g2 * C::C2 + c2) * C::N + C::NS * ka + ks0) * 8u;
        return byte ^ (((byte >> 7) & 7u) << 4);
      }
      const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + ka);
      const int col = c2 * 2 * C::NS + 2 * ks0;
      return (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
    }
  };
  // E4 (o even), column-blocked output with block width 4: kWhat 0: m0 >> 2
  // (the block row of output row m0); 1: sl * 4 + (m0 & 3).  The element
  // offset is then (m0 >> 2) * rows * 4 + the kWhat-1 value + the tile base.
  template <int kWhat>
  struct E4 {
    __host__ __device__ static constexpr uint32_t f(int warp, int lane, int bi, int c, int o) {
      using G = AccGeo<C::M1, C::N1, C::EPW>;
      const int q = warp & 3, h = (warp - 2 - C::kEpiWarps) >> 2, l4 = lane & 3;
      const int rp = G::block((uint32_t)q, h, bi) * 8 + (lane >> 2);
      const int g4 = rp / C::NS, kap = rp % C::NS;
      const int pidx = 4 * ((G::ch0(h) + c) * 8 + o) + l4;
      const int c4 = pidx / C::NA, pp = pidx % C::NA;
      const int m0 = C::NA * kap + (pp & ~7) + 2 * l4;
      const int sl = g4 * C::C1 + c4;
      return kWhat == 0 ? (uint32_t)(m0 >> 2) : (uint32_t)(sl * 4 + (m0 & 3));
    }
  };
};

struct Conv2dColShared {
  uint64_t* d_full;
  uint64_t* d_empty;
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* h_full;
  uint64_t* h_empty;
  uint8_t* smem;
};

// Epilogue group A: E1 (D1 -> B2) for tile j1 and E3 (D3 -> B4) for tile j3
// of each round.  Per-thread twiddles are loaded once.
template <class C>
__device__ __forceinline__ void conv2d_cols_group_a(const FftParams& p, int ntiles, uint32_t tmem,
                                                    const Conv2dColShared& sh, uint32_t warp, uint32_t lane) {
  using namespace sm100;
  using D = typename C::D;
  using G1g = AccGeo<C::M1, C::N1, C::EPW>;
  using G3g = AccGeo<C::M2, C::N2, C::EPW>;
  const uint32_t q = warp & 3u;
  const int h = (int)(warp - 2) >> 2;
  const int l4 = (int)(lane & 3u);
  // E1: blocked input columns (a, c1): a = pidx / C1.  Twiddle slot per
  // distinct a of this thread (fft2_kernel's blocked-input rule).
  constexpr int kTq1 = (C::C1 >= 4) ? C::C1 / 4 : 1;
  constexpr int kTw1 = G1g::CH * 8 / kTq1;
  // E3: B3 columns (c3, a'), a' = pidx % NS = l4 + 4 slot; inverse twiddles.
  constexpr int kTw3 = C::NS / 4;
  static_assert(C::NS >= 4 && (G3g::CH * 8) % kTw3 == 0, "E3 twiddle slots");
  float2 tw1[G1g::BPW][kTw1];
  float2 tw3[G3g::BPW][kTw3];
  const int ch01 = G1g::ch0(h), ch03 = G3g::ch0(h);
#pragma unroll
  for (int bi = 0; bi < G1g::BPW; ++bi) {
    const int ks = (G1g::block(q, h, bi) * 8 + (int)(lane >> 2)) % C::NS;
#pragma unroll
    for (int i = 0; i < kTw1; ++i) {
      const int a = (4 * (ch01 * 8 + i * kTq1) + l4) / C::C1;
      tw1[bi][i] = p.tw[(a * ks) % C::N];
    }
  }
#pragma unroll
  for (int bi = 0; bi < G3g::BPW; ++bi) {
    const int ksp = (G3g::block(q, h, bi) * 8 + (int)(lane >> 2)) % C::NA;
#pragma unroll
    for (int i = 0; i < kTw3; ++i) {
      const float2 w = p.tw[((l4 + 4 * i) * ksp) % C::N];
      tw3[bi][i] = make_float2(w.x, -w.y);
    }
  }
  const uint32_t b2 = smem_u32(sh.smem + C::OFF_B);
  const uint32_t b4 = b2 + 2u * C::TILE_BYTES;
  // store addresses: per-thread bases plus compile-time offsets (epi_addr.cuh)
  using A1 = typename Conv2dColAddr<C>::E1;
  using A3 = typename Conv2dColAddr<C>::E3;
  constexpr int kK1 = epi::addr_kind<A1, 2, C::kEpiWarps, G1g::BPW, G1g::CH, 8>();
  constexpr int kK3 = epi::addr_kind<A3, 2, C::kEpiWarps, G3g::BPW, G3g::CH, 8>();
  uint32_t base1[G1g::BPW][kK1 == 1 ? 8 : 1], base3[G3g::BPW][kK3 == 1 ? 8 : 1];
#pragma unroll
  for (int bi = 0; bi < G1g::BPW; ++bi)
#pragma unroll
    for (int o = 0; o < (kK1 == 1 ? 8 : 1); ++o) base1[bi][o] = b2 + A1::f((int)warp, (int)lane, bi, 0, o);
#pragma unroll
  for (int bi = 0; bi < G3g::BPW; ++bi)
#pragma unroll
    for (int o = 0; o < (kK3 == 1 ? 8 : 1); ++o) base3[bi][o] = b4 + A3::f((int)warp, (int)lane, bi, 0, o);

  for (int r = 0; r < ntiles + 2; ++r) {
    // ---------------------------------------------------------------- E1(r)
    if (r < ntiles) {
      const uint32_t ph = (uint32_t)r & 1u;
      if (!mbar_wait_warp(&sh.d_full[0], ph, p.err, kDevTimeoutEpilogue)) return;
      if (!mbar_wait_warp(&sh.b_empty[0], ph ^ 1u, p.err, kDevTimeoutEpilogue)) return;
      tc_fence_after();
      // 32-column TMEM pieces, the next one loading while this one is processed
      constexpr int kNIT1 = G1g::BPW * G1g::CH * 2;
      auto taddr1 = [&](int it) -> uint32_t {
        const int bi = it / (2 * G1g::CH), c = (it / 2) % G1g::CH, hh = it & 1;
        return tmem + (G1g::lanes(q, h, bi, C::lane_off(C::M1, 0)) << 16) + C::col_off(C::M1, 0, 0) + (uint32_t)(ch01 + c) * 64u + 32u * (uint32_t)hh;
      };
      uint32_t vb[2][16];
      tmem_ld_16x256b_x4(taddr1(0), vb[0]);
#pragma unroll
      for (int bi = 0; bi < G1g::BPW; ++bi) {
        const int rp = G1g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g1 = rp / C::NS, ks = rp % C::NS;
#pragma unroll
        for (int c = 0; c < G1g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          const int it = (bi * G1g::CH + c) * 2 + hh;
          tmem_wait_ld();
          tmem_regs_ready(vb[it & 1]);
          if (it + 1 < kNIT1) tmem_ld_16x256b_x4(taddr1(it + 1), vb[(it + 1) & 1]);
          const uint32_t (&v)[16] = vb[it & 1];
#pragma unroll
          for (int oo = 0; oo < 4; ++oo) {
            const int o = 4 * hh + oo;
            const int pidx = 4 * ((ch01 + c) * 8 + o) + l4;
            const int a = pidx / C::C1, c1 = pidx % C::C1;
            const float RR = __uint_as_float(v[4 * oo]), RI = __uint_as_float(v[4 * oo + 1]);
            const float IR = __uint_as_float(v[4 * oo + 2]), II = __uint_as_float(v[4 * oo + 3]);
            const float yr = RR - II, yi = IR + RI;
            const float2 w = tw1[bi][(c * 8 + o) / kTq1];
            const float zr = yr * w.x - yi * w.y, zi = yr * w.y + yi * w.x;
            uint32_t addr;
            if constexpr (kK1 != 0) {
              addr = base1[bi][kK1 == 1 ? o : 0] + epi::addr_delta<A1, 2, kK1>(bi, c, o);
            } else {
              const int sig = g1 * C::C1 + c1;
              const int g2 = sig / C::C2, c2 = sig % C::C2;
              const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + a);
              const int col = c2 * 2 * C::NS + 2 * (C::kColPairs2 ? detail::stage2_col_pair(ks) : ks);
              addr = b2 + (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
            }
            detail::store_complex<C::kIsHalf>(addr, zr, zi);
          }
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&sh.d_empty[0]); mbar_arrive(&sh.b_full[0]); }
    }
    // ---------------------------------------------------------------- E3(r-2)
    const int j = r - 2;
    if (j >= 0 && j < ntiles) {
      const uint32_t ph = (uint32_t)j & 1u;
      if (!mbar_wait_warp(&sh.d_full[2], ph, p.err, kDevTimeoutEpilogue)) return;
      if (!mbar_wait_warp(&sh.b_empty[2], ph ^ 1u, p.err, kDevTimeoutEpilogue)) return;
      tc_fence_after();
      // 32-column TMEM pieces, the next one loading while this one is processed
      constexpr int kNIT3 = G3g::BPW * G3g::CH * 2;
      auto taddr3 = [&](int it) -> uint32_t {
        const int bi = it / (2 * G3g::CH), c = (it / 2) % G3g::CH, hh = it & 1;
        return tmem + (G3g::lanes(q, h, bi, C::lane_off(C::M2, 1)) << 16) + C::col_off(C::M2, 1, 1) + (uint32_t)(ch03 + c) * 64u + 32u * (uint32_t)hh;
      };
      uint32_t vb[2][16];
      tmem_ld_16x256b_x4(taddr3(0), vb[0]);
#pragma unroll
      for (int bi = 0; bi < G3g::BPW; ++bi) {
        const int rp = G3g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g3 = rp / C::NA, ksp = rp % C::NA;
#pragma unroll
        for (int c = 0; c < G3g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          const int it = (bi * G3g::CH + c) * 2 + hh;
          tmem_wait_ld();
          tmem_regs_ready(vb[it & 1]);
          if (it + 1 < kNIT3) tmem_ld_16x256b_x4(taddr3(it + 1), vb[(it + 1) & 1]);
          const uint32_t (&v)[16] = vb[it & 1];
#pragma unroll
          for (int oo = 0; oo < 4; ++oo) {
            const int o = 4 * hh + oo;
            const int pidx = 4 * ((ch03 + c) * 8 + o) + l4;
            const int c3 = pidx / C::NS, ap = pidx % C::NS;
            const float RR = __uint_as_float(v[4 * oo]), RI = __uint_as_float(v[4 * oo + 1]);
            const float IR = __uint_as_float(v[4 * oo + 2]), II = __uint_as_float(v[4 * oo + 3]);
            const float yr = RR + II, yi = RI - IR;     // inverse: sine terms flipped
            const float2 w = tw3[bi][(c * 8 + o) % kTw3];
            const float zr = yr * w.x - yi * w.y, zi = yr * w.y + yi * w.x;
            uint32_t addr;
            if constexpr (kK3 != 0) {
              addr = base3[bi][kK3 == 1 ? o : 0] + epi::addr_delta<A3, 2, kK3>(bi, c, o);
            } else {
              const int sig = g3 * C::C2 + c3;
              const int g4 = sig / C::C1, c4 = sig % C::C1;
              const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g4 * C::NS + ap);
              const int col = c4 * 2 * C::NA + 2 * detail::stage2_col_pair(ksp);
              addr = b4 + (uint32_t)(col / C::E) * C::LBO1 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
            }
            detail::store_complex<C::kIsHalf>(addr, zr, zi);
          }
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&sh.d_empty[2]); mbar_arrive(&sh.b_full[2]); }
    }
  }
}

// Epilogue group B: E2 (D2 x H -> B3) for tile r-1 and E4 (D4 -> global) for
// tile r-3 of each round.
template <class C>
__device__ __forceinline__ void conv2d_cols_group_b(const FftParams& p, int ntiles, uint32_t tmem,
                                                    const Conv2dColShared& sh, uint32_t warp, uint32_t lane) {
  using namespace sm100;
  using D = typename C::D;
  using G2g = AccGeo<C::M2, C::N2, C::EPW>;
  using G4g = AccGeo<C::M1, C::N1, C::EPW>;
  const uint32_t q = warp & 3u;
  const int h = (int)(warp - 2 - C::kEpiWarps) >> 2;
  const int l4 = (int)(lane & 3u);
  const int ch02 = G2g::ch0(h), ch04 = G4g::ch0(h);
  // range scales of the half2 pipeline (exact powers of two): the spectrum
  // product is stored x 2^e2, the output x 2^e3
  const float sc2 = p.conv_exp ? detail::pow2f(p.conv_exp[0]) : 1.f;
  const float sc3 = p.conv_exp ? detail::pow2f(p.conv_exp[1]) : 1.f;
  const uint32_t b3 = smem_u32(sh.smem + C::OFF_B) + (uint32_t)C::TILE_BYTES;
  const int lb = p.blk_log2;
  const long long cbm = (1LL << lb) - 1;
  // addresses: per-thread bases plus compile-time offsets (epi_addr.cuh)
  using A2s = typename Conv2dColAddr<C>::template E2<0>;
  using A2h = typename Conv2dColAddr<C>::template E2<1>;
  using A4q = typename Conv2dColAddr<C>::template E4<0>;
  using A4r = typename Conv2dColAddr<C>::template E4<1>;
  constexpr int kW0 = 2 + C::kEpiWarps;
  constexpr int kK2s = C::kColPairs2 ? epi::addr_kind<A2s, kW0, C::kEpiWarps, G2g::BPW, G2g::CH, 8, 2>() : 0;
  constexpr int kK2h = C::kColPairs2 ? epi::addr_kind<A2h, kW0, C::kEpiWarps, G2g::BPW, G2g::CH, 8, 2>() : 0;
  constexpr int kK4q = epi::addr_kind<A4q, kW0, C::kEpiWarps, G4g::BPW, G4g::CH, 8, 2>();
  constexpr int kK4r = epi::addr_kind<A4r, kW0, C::kEpiWarps, G4g::BPW, G4g::CH, 8, 2>();
  uint32_t base2s[G2g::BPW][kK2s == 1 ? 4 : 1], base2h[G2g::BPW][kK2h == 1 ? 4 : 1];
  uint32_t base4q[G4g::BPW][kK4q == 1 ? 4 : 1], base4r[G4g::BPW][kK4r == 1 ? 4 : 1];
#pragma unroll
  for (int bi = 0; bi < G2g::BPW; ++bi)
#pragma unroll
    for (int jh = 0; jh < 4; ++jh) {
      if (jh < (kK2s == 1 ? 4 : 1)) base2s[bi][kK2s == 1 ? jh : 0] = b3 + A2s::f((int)warp, (int)lane, bi, 0, 2 * jh);
      if (jh < (kK2h == 1 ? 4 : 1)) base2h[bi][kK2h == 1 ? jh : 0] = A2h::f((int)warp, (int)lane, bi, 0, 2 * jh);
    }
#pragma unroll
  for (int bi = 0; bi < G4g::BPW; ++bi)
#pragma unroll
    for (int jh = 0; jh < 4; ++jh) {
      if (jh < (kK4q == 1 ? 4 : 1)) base4q[bi][kK4q == 1 ? jh : 0] = A4q::f((int)warp, (int)lane, bi, 0, 2 * jh);
      if (jh < (kK4r == 1 ? 4 : 1)) base4r[bi][kK4r == 1 ? jh : 0] = A4r::f((int)warp, (int)lane, bi, 0, 2 * jh);
    }
  const uint32_t rows4 = (uint32_t)p.rows * 4u;

  for (int r = 1; r < ntiles + 3; ++r) {
    // ---------------------------------------------------------------- E2(r-1)
    const int j2 = r - 1;
    if (j2 < ntiles) {
      const uint32_t ph = (uint32_t)j2 & 1u;
      const int hs = j2 % C::HS;
      if (!mbar_wait_warp(&sh.d_full[1], ph, p.err, kDevTimeoutEpilogue)) return;
      if (!mbar_wait_warp(&sh.b_empty[1], ph ^ 1u, p.err, kDevTimeoutEpilogue)) return;
      if (!mbar_wait_warp(&sh.h_full[hs], (uint32_t)(j2 / C::HS) & 1u, p.err, kDevTimeoutEpilogue)) return;
      tc_fence_after();
      const uint32_t hbase = smem_u32(sh.smem + C::OFF_H + hs * C::SPEC_BYTES);
      // 32-column TMEM pieces, the next one loading while this one is processed
      constexpr int kNIT2 = G2g::BPW * G2g::CH * 2;
      auto taddr2 = [&](int it) -> uint32_t {
        const int bi = it / (2 * G2g::CH), c = (it / 2) % G2g::CH, hh = it & 1;
        return tmem + (G2g::lanes(q, h, bi, C::lane_off(C::M2, 0)) << 16) + C::col_off(C::M2, 1, 0) + (uint32_t)(ch02 + c) * 64u + 32u * (uint32_t)hh;
      };
      uint32_t vb[2][16];
      tmem_ld_16x256b_x4(taddr2(0), vb[0]);
#pragma unroll
      for (int bi = 0; bi < G2g::BPW; ++bi) {
        const int rp = G2g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g2 = rp / C::NA, ka = rp % C::NA;
        const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + ka);
#pragma unroll
        for (int c = 0; c < G2g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          const int it = (bi * G2g::CH + c) * 2 + hh;
          tmem_wait_ld();
          tmem_regs_ready(vb[it & 1]);
          if (it + 1 < kNIT2) tmem_ld_16x256b_x4(taddr2(it + 1), vb[(it + 1) & 1]);
          const uint32_t (&v)[16] = vb[it & 1];
          if constexpr (C::kColPairs2) {
            // iterations j, j + 1 hold ks0 = 8m + 2 l4 and ks0 + 1 of one signal
#pragma unroll
            for (int j2 = 0; j2 < 4; j2 += 2) {
              const int jj = 4 * hh + j2;
              const int pidx = 4 * ((ch02 + c) * 8 + jj) + l4;
              const int c2 = pidx / C::NS, pp = pidx % C::NS;
              const int ks0 = (pp & ~7) + 2 * l4;
              const int sl = g2 * C::C2 + c2;
              const int k0 = C::NS * ka + ks0;
              float xr[2], xi[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float RR = __uint_as_float(v[4 * (j2 + e)]), RI = __uint_as_float(v[4 * (j2 + e) + 1]);
                const float IR = __uint_as_float(v[4 * (j2 + e) + 2]), II = __uint_as_float(v[4 * (j2 + e) + 3]);
                xr[e] = RR - II;
                xi[e] = IR + RI;
              }
              uint32_t sbyte;
              if constexpr (kK2h != 0) {
                sbyte = base2h[bi][kK2h == 1 ? jj / 2 : 0] + epi::addr_delta<A2h, kW0, kK2h>(bi, c, jj);
              } else {
                const uint32_t byte = (uint32_t)(sl * C::N + k0) * 8u;
                sbyte = byte ^ (((byte >> 7) & 7u) << 4);
              }
              float4 w = ld_shared_v4f(hbase + sbyte);
              w.x *= sc2; w.y *= sc2; w.z *= sc2; w.w *= sc2;
              const float z0r = xr[0] * w.x - xi[0] * w.y, z0i = xr[0] * w.y + xi[0] * w.x;
              const float z1r = xr[1] * w.z - xi[1] * w.w, z1i = xr[1] * w.w + xi[1] * w.z;
              uint32_t addr;
              if constexpr (kK2s != 0) {
                addr = base2s[bi][kK2s == 1 ? jj / 2 : 0] + epi::addr_delta<A2s, kW0, kK2s>(bi, c, jj);
              } else {
                const int col = c2 * 2 * C::NS + 2 * ks0;
                addr = b3 + (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
              }
              if constexpr (C::kIsHalf) {
                __half2 h0 = __floats2half2_rn(z0r, z0i), h1 = __floats2half2_rn(z1r, z1i);
                asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(*reinterpret_cast<uint32_t*>(&h0)),
                             "r"(*reinterpret_cast<uint32_t*>(&h1))
                             : "memory");
              } else {
                st_shared_v4(addr, __float_as_uint(round_tf32(z0r)), __float_as_uint(round_tf32(z0i)),
                             __float_as_uint(round_tf32(z1r)), __float_as_uint(round_tf32(z1i)));
              }
            }
          } else {
#pragma unroll
            for (int oo = 0; oo < 4; ++oo) {
              const int o = 4 * hh + oo;
              const int pidx = 4 * ((ch02 + c) * 8 + o) + l4;
              const int c2 = pidx / C::NS, ks = pidx % C::NS;
              const int sl = g2 * C::C2 + c2;
              const int k = C::NS * ka + ks;
              const float RR = __uint_as_float(v[4 * oo]), RI = __uint_as_float(v[4 * oo + 1]);
              const float IR = __uint_as_float(v[4 * oo + 2]), II = __uint_as_float(v[4 * oo + 3]);
              const float xr = RR - II, xi = IR + RI;
              const uint32_t byte = (uint32_t)(sl * C::N + k) * 8u;
              float2 w = ld_shared_v2f(hbase + (byte ^ (((byte >> 7) & 7u) << 4)));
              w.x *= sc2; w.y *= sc2;
              const int col = c2 * 2 * C::NS + 2 * ks;
              const uint32_t off = (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
              detail::store_complex<C::kIsHalf>(b3 + off, xr * w.x - xi * w.y, xr * w.y + xi * w.x);
            }
          }
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&sh.d_empty[1]); mbar_arrive(&sh.b_full[1]); mbar_arrive(&sh.h_empty[hs]); }
    }
    // ---------------------------------------------------------------- E4(r-3)
    const int j4 = r - 3;
    if (j4 >= 0) {
      const uint32_t ph = (uint32_t)j4 & 1u;
      if (!mbar_wait_warp(&sh.d_full[3], ph, p.err, kDevTimeoutEpilogue)) return;
      tc_fence_after();
      const long long tile = blockIdx.x + (long long)j4 * gridDim.x;
      const long long sig0 = tile * C::T;
      const long long img = sig0 / p.rows, r0 = sig0 - img * p.rows;
      // element base of this tile in the block-width-4 layout: img N rows + r0 * 4
      uint8_t* const tile_out = reinterpret_cast<uint8_t*>(p.out) + (img * C::N * p.rows + r0 * 4) * (C::kIsHalf ? 4 : 8);
      // 32-column TMEM pieces, the next one loading while this one is processed
      constexpr int kNIT4 = G4g::BPW * G4g::CH * 2;
      auto taddr4 = [&](int it) -> uint32_t {
        const int bi = it / (2 * G4g::CH), c = (it / 2) % G4g::CH, hh = it & 1;
        return tmem + (G4g::lanes(q, h, bi, C::lane_off(C::M1, 1)) << 16) + C::col_off(C::M1, 0, 1) + (uint32_t)(ch04 + c) * 64u + 32u * (uint32_t)hh;
      };
      uint32_t vb[2][16];
      tmem_ld_16x256b_x4(taddr4(0), vb[0]);
#pragma unroll
      for (int bi = 0; bi < G4g::BPW; ++bi) {
        const int rp = G4g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g4 = rp / C::NS, kap = rp % C::NS;
#pragma unroll
        for (int c = 0; c < G4g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          const int it = (bi * G4g::CH + c) * 2 + hh;
          tmem_wait_ld();
          tmem_regs_ready(vb[it & 1]);
          if (it + 1 < kNIT4) tmem_ld_16x256b_x4(taddr4(it + 1), vb[(it + 1) & 1]);
          const uint32_t (&v)[16] = vb[it & 1];
#pragma unroll
          for (int j2 = 0; j2 < 4; j2 += 2) {
            const int jj = 4 * hh + j2;
            // iterations jj, jj + 1 hold ks0' = 8m + 2 l4 and ks0' + 1 of one signal
            const int pidx = 4 * ((ch04 + c) * 8 + jj) + l4;
            const int c4 = pidx / C::NA, pp = pidx % C::NA;
            const int ks0 = (pp & ~7) + 2 * l4;
            const int sl = g4 * C::C1 + c4;
            const long long m0 = (long long)C::NA * kap + ks0;    // image row of the first output
            float xr[2], xi[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float RR = __uint_as_float(v[4 * (j2 + e)]), RI = __uint_as_float(v[4 * (j2 + e) + 1]);
              const float IR = __uint_as_float(v[4 * (j2 + e) + 2]), II = __uint_as_float(v[4 * (j2 + e) + 3]);
              xr[e] = (RR + II) * sc3;
              xi[e] = (RI - IR) * sc3;
            }
            // column-blocked [img][m / Cb][column][m % Cb]; m0 even, so with
            // Cb >= 2 outputs m0 and m0 + 1 are neighbours
            if (lb == 2) {
              // Cb = 4: ((img N + m0) >> 2) rows 4 + (r0 + sl) 4 + (m0 & 3), N a multiple of 4
              uint32_t mq, er;
              if constexpr (kK4q != 0) mq = base4q[bi][kK4q == 1 ? jj / 2 : 0] + epi::addr_delta<A4q, kW0, kK4q>(bi, c, jj);
              else mq = A4q::f((int)warp, (int)lane, bi, c, jj);
              if constexpr (kK4r != 0) er = base4r[bi][kK4r == 1 ? jj / 2 : 0] + epi::addr_delta<A4r, kW0, kK4r>(bi, c, jj);
              else er = A4r::f((int)warp, (int)lane, bi, c, jj);
              const uint32_t e = mq * rows4 + er;
              if constexpr (C::kIsHalf) {
                __half2 h0 = __floats2half2_rn(xr[0], xi[0]), h1 = __floats2half2_rn(xr[1], xi[1]);
                *reinterpret_cast<uint2*>(reinterpret_cast<uint32_t*>(tile_out) + e) =
                    make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
              } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float2*>(tile_out) + e) = make_float4(xr[0], xi[0], xr[1], xi[1]);
              }
              continue;
            }
            const long long o0 = (((img * C::N + m0) >> lb) * p.rows + r0 + sl) * (cbm + 1) + (m0 & cbm);
            if (lb >= 1) {
              if constexpr (C::kIsHalf) {
                __half2 h0 = __floats2half2_rn(xr[0], xi[0]), h1 = __floats2half2_rn(xr[1], xi[1]);
                *reinterpret_cast<uint2*>(reinterpret_cast<uint32_t*>(p.out) + o0) =
                    make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
              } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float2*>(p.out) + o0) = make_float4(xr[0], xi[0], xr[1], xi[1]);
              }
            } else {
              const long long o1 = (((img * C::N + m0 + 1) >> lb) * p.rows + r0 + sl) * (cbm + 1) + ((m0 + 1) & cbm);
              detail::store_out<C::kIsHalf>(p.out, o0, xr[0], xi[0]);
              detail::store_out<C::kIsHalf>(p.out, o1, xr[1], xi[1]);
            }
          }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.d_empty[3]);
    }
  }
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
conv2d_cols_kernel(const __grid_constant__ CUtensorMap tmap_in, const __grid_constant__ CUtensorMap tmap_spec,
                   const FftParams p) {
  using namespace sm100;
  using D = typename C::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in_full[C::SIN], bar_in_empty[C::SIN], bar_h_full[C::HS], bar_h_empty[C::HS];
  __shared__ uint64_t bar_d_full[4], bar_d_empty[4], bar_b_full[3], bar_b_empty[3], bar_const, bar_done[2];
  __shared__ uint32_t tmem_slot;

  const uint32_t warp = warp_id(), lane = lane_id();
  // conv2d tiles never straddle images and the batch is whole tiles (host)
  const long long num_tiles = p.batch / C::T;
  const int ntiles = (int)((num_tiles > blockIdx.x) ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::SIN; ++i) { mbar_init(&bar_in_full[i], 1); mbar_init(&bar_in_empty[i], 1); }
    for (int i = 0; i < C::HS; ++i) { mbar_init(&bar_h_full[i], 1); mbar_init(&bar_h_empty[i], C::kEpiWarps); }
    for (int i = 0; i < 4; ++i) { mbar_init(&bar_d_full[i], 1); mbar_init(&bar_d_empty[i], C::kEpiWarps); }
    for (int i = 0; i < 3; ++i) { mbar_init(&bar_b_full[i], C::kEpiWarps); mbar_init(&bar_b_empty[i], 1); }
    mbar_init(&bar_const, 1);
    mbar_init(&bar_done[0], 1);
    mbar_init(&bar_done[1], 1);
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_in);
      tma_prefetch_desc(&tmap_spec);
      mbar_arrive_expect_tx(&bar_const, C::A_LOAD_BYTES);
      bulk_load(smem + C::OFF_A1, p.a1, C::A1_BYTES, &bar_const);
      if constexpr (!C::kA2isA1) bulk_load(smem + C::OFF_A2, p.a2, C::A2_BYTES, &bar_const);
      if constexpr (!C::kA4isA1 && !C::kA4isA2) bulk_load(smem + C::OFF_A4, p.a4, C::A1_BYTES, &bar_const);
    }
    for (int i = 0; i < ntiles; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int slot = i % C::SIN;
      if (!mbar_wait_warp(&bar_in_empty[slot], ((uint32_t)(i / C::SIN) & 1u) ^ 1u, p.err, kDevTimeoutProducer)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
        tma_load_5d(smem + C::OFF_IN + slot * C::TILE_BYTES, &tmap_in, &bar_in_full[slot], 0, 0, 0, 0, (int)tile);
      }
      __syncwarp();
      // the tile's spectrum rows spec[ch][r0 .. r0 + T)[0 .. N): one 2-D box of 128-B lines
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
  } else if (warp == 1 || warp == (uint32_t)C::kMma2Warp) {
    // ------------------------------------------------------------ MMA issuers
    // warp 1: stages 1 and 3; warp kMma2Warp: stages 2 and 4
    const int par = (warp == 1) ? 0 : 1;
    if (lane == 0) {
      bool ok = mbar_wait(&bar_const, 0, p.err, kDevTimeoutMma);
      const uint32_t idesc1 = instr_desc(D::kFmt, C::M1, C::N1, 0, 1);
      const uint32_t idesc2 = instr_desc(D::kFmt, C::M2, C::N2, 0, 1);
      // A images: K-major, no swizzle; LBO = K-direction core stride = M/8 * 128 B
      const uint32_t lboA1 = (C::M1 / 8) * 128, lboA2 = (C::M2 / 8) * 128;
      const uint64_t adA1 = smem_desc(smem_u32(smem + C::OFF_A1), lboA1, 128, kSwNone);
      const uint64_t adA2 = smem_desc(smem_u32(smem + C::OFF_A2), lboA2, 128, kSwNone);
      const uint64_t adA4 = smem_desc(smem_u32(smem + C::OFF_A4), lboA1, 128, kSwNone);
      const uint64_t bdIn0 = smem_desc(smem_u32(smem + C::OFF_IN), C::LBO1, D::kBSbo, D::kBSwizzle);
      const uint64_t bdB2 = smem_desc(smem_u32(smem + C::OFF_B), C::LBO2, D::kBSbo, D::kBSwizzle);
      const uint64_t bdB3 = smem_desc(smem_u32(smem + C::OFF_B + C::TILE_BYTES), C::LBO2, D::kBSbo, D::kBSwizzle);
      const uint64_t bdB4 = smem_desc(smem_u32(smem + C::OFF_B + 2 * C::TILE_BYTES), C::LBO1, D::kBSbo, D::kBSwizzle);
      const uint32_t dD1 = tmem + (C::lane_off(C::M1, 0) << 16) + C::col_off(C::M1, 0, 0);
      const uint32_t dD4 = tmem + (C::lane_off(C::M1, 1) << 16) + C::col_off(C::M1, 0, 1);
      const uint32_t dD2 = tmem + (C::lane_off(C::M2, 0) << 16) + C::col_off(C::M2, 1, 0);
      const uint32_t dD3 = tmem + (C::lane_off(C::M2, 1) << 16) + C::col_off(C::M2, 1, 1);
      auto stage = [&](uint32_t d, uint64_t ad, uint32_t lboA, uint64_t bd, uint32_t idesc, int ksteps) {
#pragma unroll 4
        for (int k = 0; k < ksteps; ++k) {
          const uint64_t a = ad + (uint64_t)((k * 2 * lboA) >> 4);
          const uint64_t b = bd + (uint64_t)((k * C::KSTEP_BYTES) >> 4);
          if constexpr (C::kIsHalf) umma_f16(d, a, b, idesc, k > 0);
          else umma_tf32(d, a, b, idesc, k > 0);
        }
      };
      for (int r = 0; ok && r < ntiles + 3; ++r) {
        if (par == 0 && r < ntiles) {   // S1(r): input slot -> D1
          const int slot = r % C::SIN;
          if (!mbar_wait(&bar_in_full[slot], (uint32_t)(r / C::SIN) & 1u, p.err, kDevTimeoutMma) ||
              !mbar_wait(&bar_d_empty[0], ((uint32_t)r & 1u) ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          stage(dD1, adA1, lboA1, bdIn0 + (uint64_t)(slot * (C::TILE_BYTES >> 4)), idesc1, C::KSTEPS1);
          umma_commit(&bar_in_empty[slot]);
          umma_commit(&bar_d_full[0]);
        }
#pragma unroll 1
        for (int s = 1; s < 4; ++s) {   // S2(r-1), S3(r-2), S4(r-3): B(s+1) -> D(s+1)
          const int j = r - s;
          if ((s & 1) != (par ^ 1) || j < 0 || j >= ntiles) continue;
          if (!mbar_wait(&bar_b_full[s - 1], (uint32_t)j & 1u, p.err, kDevTimeoutMma) ||
              !mbar_wait(&bar_d_empty[s], ((uint32_t)j & 1u) ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          if (s == 1) stage(dD2, adA2, lboA2, bdB2, idesc2, C::KSTEPS2);
          else if (s == 2) stage(dD3, adA2, lboA2, bdB3, idesc2, C::KSTEPS2);
          else stage(dD4, adA4, lboA1, bdB4, idesc1, C::KSTEPS1);
          umma_commit(&bar_b_empty[s - 1]);
          umma_commit(&bar_d_full[s]);
        }
      }
      // drain: all issued MMAs complete before TMEM is released
      umma_commit(&bar_done[par]);
      mbar_wait(&bar_done[par], 0, p.err, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    Conv2dColShared sh;
    sh.d_full = bar_d_full; sh.d_empty = bar_d_empty; sh.b_full = bar_b_full; sh.b_empty = bar_b_empty;
    sh.h_full = bar_h_full; sh.h_empty = bar_h_empty; sh.smem = smem;
    if (warp < 2 + C::kEpiWarps) conv2d_cols_group_a<C>(p, ntiles, tmem, sh, warp, lane);
    else conv2d_cols_group_b<C>(p, ntiles, tmem, sh, warp, lane);
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace thff
