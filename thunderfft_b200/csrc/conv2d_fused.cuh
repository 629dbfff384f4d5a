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
  static constexpr int kThreads = 32 * (2 + 2 * kEpiWarps);
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
  __device__ static int ch0(int h) { return (kM == 64 && kEPW > 1) ? h * CH : 0; }
  __device__ static int block(uint32_t q, int h, int bi) { return (kM == 64) ? (int)q : (int)(2 * q) + h * BPW + bi; }
  __device__ static uint32_t lanes(uint32_t q, int h, int bi, uint32_t loff) {
    return (kM == 64) ? 32u * q + loff : 32u * q + 16u * (uint32_t)(h * BPW + bi);
  }
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

  for (int r = 0; r < ntiles + 2; ++r) {
    // ---------------------------------------------------------------- E1(r)
    if (r < ntiles) {
      const uint32_t ph = (uint32_t)r & 1u;
      if (!mbar_wait_warp(&sh.d_full[0], ph, p.err, kDevTimeoutEpilogue)) return;
      if (!mbar_wait_warp(&sh.b_empty[0], ph ^ 1u, p.err, kDevTimeoutEpilogue)) return;
      tc_fence_after();
#pragma unroll
      for (int bi = 0; bi < G1g::BPW; ++bi) {
        const int rp = G1g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g1 = rp / C::NS, ks = rp % C::NS;
        const uint32_t base = tmem + (G1g::lanes(q, h, bi, C::lane_off(C::M1, 0)) << 16) + C::col_off(C::M1, 0, 0);
#pragma unroll
        for (int c = 0; c < G1g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          uint32_t v[16];
          tmem_ld_16x256b_x4(base + (uint32_t)(ch01 + c) * 64u + 32u * (uint32_t)hh, v);
          tmem_wait_ld();
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
            const int sig = g1 * C::C1 + c1;
            const int g2 = sig / C::C2, c2 = sig % C::C2;
            const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + a);
            const int col = c2 * 2 * C::NS + 2 * (C::kColPairs2 ? detail::stage2_col_pair(ks) : ks);
            const uint32_t off = (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
            detail::store_complex<C::kIsHalf>(b2 + off, zr, zi);
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
#pragma unroll
      for (int bi = 0; bi < G3g::BPW; ++bi) {
        const int rp = G3g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g3 = rp / C::NA, ksp = rp % C::NA;
        const uint32_t base = tmem + (G3g::lanes(q, h, bi, C::lane_off(C::M2, 1)) << 16) + C::col_off(C::M2, 1, 1);
#pragma unroll
        for (int c = 0; c < G3g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          uint32_t v[16];
          tmem_ld_16x256b_x4(base + (uint32_t)(ch03 + c) * 64u + 32u * (uint32_t)hh, v);
          tmem_wait_ld();
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
            const int sig = g3 * C::C2 + c3;
            const int g4 = sig / C::C1, c4 = sig % C::C1;
            const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g4 * C::NS + ap);
            const int col = c4 * 2 * C::NA + 2 * detail::stage2_col_pair(ksp);
            const uint32_t off = (uint32_t)(col / C::E) * C::LBO1 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
            detail::store_complex<C::kIsHalf>(b4 + off, zr, zi);
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
#pragma unroll
      for (int bi = 0; bi < G2g::BPW; ++bi) {
        const int rp = G2g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g2 = rp / C::NA, ka = rp % C::NA;
        const uint32_t krow = (uint32_t)detail::stage2_krow(C::R2, g2 * C::NA + ka);
        const uint32_t base = tmem + (G2g::lanes(q, h, bi, C::lane_off(C::M2, 0)) << 16) + C::col_off(C::M2, 1, 0);
#pragma unroll
        for (int c = 0; c < G2g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          uint32_t v[16];
          tmem_ld_16x256b_x4(base + (uint32_t)(ch02 + c) * 64u + 32u * (uint32_t)hh, v);
          tmem_wait_ld();
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
              const uint32_t byte = (uint32_t)(sl * C::N + k0) * 8u;
              float4 w = ld_shared_v4f(hbase + (byte ^ (((byte >> 7) & 7u) << 4)));
              w.x *= sc2; w.y *= sc2; w.z *= sc2; w.w *= sc2;
              const float z0r = xr[0] * w.x - xi[0] * w.y, z0i = xr[0] * w.y + xi[0] * w.x;
              const float z1r = xr[1] * w.z - xi[1] * w.w, z1i = xr[1] * w.w + xi[1] * w.z;
              const int col = c2 * 2 * C::NS + 2 * ks0;
              const uint32_t off = (uint32_t)(col / C::E) * C::LBO2 + D::swz(krow * 128u + (uint32_t)(col % C::E) * C::ESZ);
              if constexpr (C::kIsHalf) {
                __half2 h0 = __floats2half2_rn(z0r, z0i), h1 = __floats2half2_rn(z1r, z1i);
                asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(b3 + off), "r"(*reinterpret_cast<uint32_t*>(&h0)),
                             "r"(*reinterpret_cast<uint32_t*>(&h1))
                             : "memory");
              } else {
                st_shared_v4(b3 + off, __float_as_uint(round_tf32(z0r)), __float_as_uint(round_tf32(z0i)),
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
#pragma unroll
      for (int bi = 0; bi < G4g::BPW; ++bi) {
        const int rp = G4g::block(q, h, bi) * 8 + (int)(lane >> 2);
        const int g4 = rp / C::NS, kap = rp % C::NS;
        const uint32_t base = tmem + (G4g::lanes(q, h, bi, C::lane_off(C::M1, 1)) << 16) + C::col_off(C::M1, 0, 1);
#pragma unroll
        for (int c = 0; c < G4g::CH; ++c) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {   // two 32-column loads: 16 registers in flight
          uint32_t v[16];
          tmem_ld_16x256b_x4(base + (uint32_t)(ch04 + c) * 64u + 32u * (uint32_t)hh, v);
          tmem_wait_ld();
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
  __shared__ uint64_t bar_d_full[4], bar_d_empty[4], bar_b_full[3], bar_b_empty[3], bar_const, bar_done;
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
    mbar_init(&bar_done, 1);
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
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
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
        if (r < ntiles) {   // S1(r): input slot -> D1
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
          if (j < 0 || j >= ntiles) continue;
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
      umma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.err, kDevTimeoutMma);
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
