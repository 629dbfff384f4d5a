// conv1d_kernel.cuh — fused real 1-D FFT convolution on sm_100a.
//
// Counterpart of the reference's fused conv1d sample kernel
// (sample/conv1d/conv1d_fullfft_l4096_thunder.cu:280-331: real input ->
// FFT -> x filter spectrum -> inverse FFT -> real output in one kernel).
// For each real signal x (length Lin <= N, zero-padded to N) and one real
// filter with spectrum H (1/N folded in):
//     y = IFFT( FFT(x) * H ),   i.e.  y[m] = (1/N) sum_k x[(m-k) mod N] h[k].
//
// Two real signals share one complex transform: z = x0 + i*x1 gives
// IFFT(FFT(z) * H) = (x0 (*) h) + i (x1 (*) h) because h is real, so the real
// and imaginary parts of the result are the two outputs.
//
// N = L * L runs as four tcgen05 stages on one tile (TC complex signals):
//   S1 forward DFT over s     (B1: input rows, TMA, zero rows for padding)
//   E1 combine + twiddle w_N^-(a ks)           -> B2
//   S2 forward DFT over a, E2 combine, * H      -> B3 (transposed = inverse input order)
//   S3 inverse DFT over s', E3 combine + w_N^+(a ks) -> B4
//   S4 inverse DFT over a', E4 combine          -> y (global)
// Every B operand is planar: columns (signal c, plane re|im, index) so that
// one TMEM 16x256b load gives a thread, for two neighbouring indices, all
// four partial sums (cos|sin) x (re|im) of its outputs.  All stages use the
// same forward DFT matrix; the inverse stages flip the sine terms in the
// epilogue.  The MMA thread runs the four stages of four different tiles in
// each round (S1(r), S2(r-1), S3(r-2), S4(r-3)) so all stages overlap.
#pragma once
#include "fft_kernels.cuh"

namespace thff {

template <int kN, bool kMixed = false>
struct Conv1dCfg {
  using D = DType<false>;  // float storage / TF32 tensor cores
  // kMixed: stage 1 reads the fp32 input as TF32; stages 2-4 take FP16
  // operands (same 11-bit significand as TF32, half the shared-memory bytes
  // and twice the MMA rate), with FP32 accumulation in TMEM.  The epilogues
  // scale each FP16 operand by a power of two chosen from a bound on its
  // magnitude (see Conv1dParams::scale*), so any finite fp32 input stays in
  // FP16 range.
  static constexpr bool kF16 = kMixed;
  static constexpr int N = kN;
  static constexpr int L = (kN == 4096) ? 64 : 32;     // N = L * L
  static_assert(L * L == N, "conv1d supports N = 1024 and 4096");
  static constexpr int M = 2 * L;                        // MMA M (rows: ks x {cos, sin})
  static constexpr int TC = (kN == 4096) ? 1 : 4;        // complex signals (= 2*TC real) per tile
  static constexpr int NCOL = TC * 2 * L;                // MMA N (columns: c x plane x index)
  static constexpr int E = 32;                           // floats per 128-B atom row
  static constexpr int H = L * 4 / 128;                  // 128-B atoms per input row
  static constexpr int TILE_BYTES = TC * N * 8;          // planar complex tile (B1..B4)
  static constexpr int A_BYTES = M * L * 4;
  static constexpr uint32_t LBO = L * 128;
  static constexpr int KSTEPS = L / 8;
  static constexpr int SIN = (kN == 4096) ? 2 : 3;
  // FP16 operands of stages 2-4 (kMixed): 64 columns per 128-B atom
  static constexpr int E16 = 64;
  static constexpr int A16_BYTES = kMixed ? M * L * 2 : 0;
  static constexpr int BT_BYTES = kMixed ? TC * N * 4 : TILE_BYTES;   // one B2/B3/B4 tile
  static constexpr int KSTEPS16 = L / 16;
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_A16 = (A_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t OFF_IN = OFF_A16 + (A16_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t OFF_B = OFF_IN + SIN * TILE_BYTES;   // B2, B3, B4
  static constexpr uint32_t SMEM_BYTES = exclusive_smem(OFF_B + 3 * BT_BYTES + 1024);
  static_assert(SMEM_BYTES + 1024 <= 232448, "shared memory budget");
  static_assert(M == 128 ? NCOL <= 128 : NCOL <= 256, "TMEM budget (4 accumulators)");
  // Two epilogue warps per TMEM lane quadrant and group: each takes two of a
  // stage's four accumulator pieces (N = 4096: one of the quadrant's two
  // 16-row blocks), so four warps per scheduler hide the epilogues' TMEM,
  // shared-memory and FMA latencies.
  static constexpr int EPW = 2;
  static constexpr int kGroupWarps = 4 * EPW;            // per epilogue group
  static constexpr int kThreads = 32 * (2 + 2 * kGroupWarps + (kMixed ? 1 : 0));   // + range-scale warp
  static constexpr int kBlocks = M / 64;                 // 16-row blocks per TMEM lane quadrant
  static constexpr int kWarpBlocks = (L == 64) ? kBlocks / EPW : kBlocks;   // blocks one epilogue warp owns
};

struct Conv1dParams {
  const float* x;        // [batch][lin] real input
  float* y;              // [batch][N] real output
  const void* a;         // forward DFT matrix image (K-major, no swizzle)
  const float2* tw;      // forward twiddles exp(-2 pi i k / N)
  const float2* spec;    // filter spectrum H[k] / N (complex fp32)
  long long batch;       // real signals
  int lin;               // input length (<= N, multiple of L)
  int rows_valid;        // lin / L: non-zero K rows of stage 1
  uint32_t* err;
  const void* a16;       // kMixed: forward DFT matrix image in FP16
};

namespace detail {

template <class C>
__device__ __forceinline__ uint32_t planar_off(int krow, int col) {
  return (uint32_t)(col / C::E) * C::LBO + C::D::swz((uint32_t)krow * 128u + (uint32_t)(col % C::E) * 4u);
}

// TMEM address of accumulator s (0..3) for 16-row block `block` of this warp.
template <class C>
__device__ __forceinline__ uint32_t acc_addr(uint32_t tmem, int s, uint32_t q, int bi) {
  if constexpr (C::M == 64) {
    return tmem + ((32u * q + 16u * (uint32_t)(s & 1)) << 16) + 256u * (uint32_t)(s >> 1);
  } else {
    return tmem + ((32u * q + 16u * (uint32_t)bi) << 16) + 128u * (uint32_t)s;
  }
}

}  // namespace detail

// Shared state the epilogue warps use (pointers into the kernel's shared memory).
struct Conv1dShared {
  uint64_t* d_full;
  uint64_t* d_empty;
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* scale_full;   // kMixed: per input slot, the tile's stage-2 input scale is ready
  int* e1_ring;           // kMixed: exponent of that scale, per tile j at j % 8
  uint8_t* bbuf;          // B2, B3, B4
  int e2, e3;             // kMixed: exponents of the stage-3 / stage-4 input scales (per call)
};

// One epilogue pass of stage S (0..3) on tile j of the conv1d kernel (see
// the kernel for the thread <-> data mapping and the per-thread constants).
//
// Range scaling (kMixed).  Stages 2-4 read FP16 operands, so each epilogue
// that writes one scales it by a power of two (exact) chosen from a bound on
// its magnitude, aiming every real or imaginary part at <= 2^13 (FP16 stops
// at 65504 ~ 2^16):
//   B2 = Y1 w s1,  |Y1| <= R sqrt2 max|x|       s1 per tile (range-scale warp)
//   B3 = X H s2,   |X| <= L |B2|, |B2| <= 2^13.5  s2 per call from max|H|
//   B4 = Z w s3,   |Z| <= L |B3|                  s3 = 2^-ceil(log2(L sqrt2))
// and the last epilogue multiplies by 1/(s1 s2 s3).
template <class C, int S>
__device__ __forceinline__ bool conv1d_epilogue(const Conv1dParams& p, int j, uint32_t tmem, const Conv1dShared& sh,
                                                uint32_t q, uint32_t lane, int l4, int hw,
                                                const int (&ksv)[C::kWarpBlocks],
                                                const float4 (&cst)[C::kWarpBlocks][C::L / 8],
                                                const uint32_t (&ba)[C::kWarpBlocks][4],
                                                const uint32_t (&bb)[C::kWarpBlocks][8]) {
  using namespace sm100;
  constexpr int kB = C::kBlocks;
  constexpr bool kInverse = S >= 2;
  constexpr bool kF16 = C::kF16;
  const long long batch = p.batch;
  const uint32_t ph = (uint32_t)j & 1u;
  if (!mbar_wait_warp(&sh.d_full[S], ph, p.err, kDevTimeoutEpilogue)) return false;
  if (S < 3 && !mbar_wait_warp(&sh.b_empty[S], ph ^ 1u, p.err, kDevTimeoutEpilogue)) return false;
  float scale = 1.f;
  if constexpr (kF16) {
    if constexpr (S == 0) {
      if (!mbar_wait_warp(&sh.scale_full[j % C::SIN], (uint32_t)(j / C::SIN) & 1u, p.err, kDevTimeoutEpilogue))
        return false;
      scale = detail::pow2f(sh.e1_ring[j & 7]);
    } else if constexpr (S == 2) {
      scale = detail::pow2f(sh.e3);
    } else if constexpr (S == 3) {
      scale = detail::pow2f(-(sh.e1_ring[j & 7] + sh.e2 + sh.e3));
    }
  }
  tc_fence_after();
  const long long tile = blockIdx.x + (long long)j * gridDim.x;
  const uint32_t bdst = smem_u32(sh.bbuf + (S < 3 ? S : 0) * C::BT_BYTES);
  // The accumulator is read in four pieces of 32 registers (re and im planes
  // of four index pairs u): L = 64 -> (block, half of the u range), L = 32 ->
  // (signal c).  Epilogue warp hw of its quadrant takes pieces 2 hw and
  // 2 hw + 1 (L = 64: block hw, whose constants are its block 0).  The load
  // of each piece completes before it is processed; with four epilogue
  // warps per scheduler the other warps cover that latency (a second buffer
  // in flight measured the same and spilled under the 96-register cap).
  static_assert(kB * C::TC * (C::L / 32) == 4, "four accumulator pieces per stage");
  static_assert(C::EPW == 2, "two pieces per epilogue warp");
  auto load_piece = [&](int pc, uint32_t (&v)[32]) {
    if constexpr (C::L == 64) {
      const uint32_t a = detail::acc_addr<C>(tmem, S, q, pc >> 1) + 32u * (uint32_t)(pc & 1);
      tmem_ld_16x256b_x4(a, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
      tmem_ld_16x256b_x4(a + C::L, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
    } else {
      tmem_ld_16x256b_x8(detail::acc_addr<C>(tmem, S, q, 0) + (uint32_t)(pc * 2 * C::L), v);
    }
  };
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const int pc = 2 * hw + pp;
    uint32_t v[32];   // v[0..15]: re plane, v[16..31]: im plane
    load_piece(pc, v);
    tmem_wait_ld();
    tmem_regs_ready(v);
    const int bi = 0;                       // the warp's own block (L = 64) or the only one
    const int c = (C::L == 64) ? 0 : pc;
    const int u0 = (C::L == 64) ? 4 * (pc & 1) : 0;
    // column-atom offsets of signal c (f32: its re / im planes)
    const uint32_t atom_re = kF16 ? (uint32_t)((c * 2 * C::L) / C::E16) * C::LBO
                                  : (uint32_t)((c * 2 * C::L) / C::E) * C::LBO;
    const uint32_t atom_im = kF16 ? atom_re : (uint32_t)((c * 2 * C::L + C::L) / C::E) * C::LBO;
    float* yre = nullptr;
    float* yim = nullptr;
    if constexpr (S == 3) {
      const long long sig0 = tile * (2LL * C::TC) + 2 * c;
      float* row = p.y + sig0 * C::N + C::L * ksv[bi] + 2 * l4;
      if (sig0 < batch) yre = row;
      if (sig0 + 1 < batch) yim = row + C::N;
    }
#pragma unroll
    for (int uu = 0; uu < 4; ++uu) {
      const int u = u0 + uu;
      float yr[2], yi[2];
#pragma unroll
      for (int o = 0; o < 2; ++o) {
        const float RR = __uint_as_float(v[4 * uu + o]), IR = __uint_as_float(v[4 * uu + 2 + o]);
        const float RI = __uint_as_float(v[16 + 4 * uu + o]), II = __uint_as_float(v[16 + 4 * uu + 2 + o]);
        yr[o] = kInverse ? RR + II : RR - II;
        yi[o] = kInverse ? RI - IR : IR + RI;
      }
      const float4 k4 = cst[bi][u];
      if constexpr (S == 0 || S == 2) {
        // twiddle, then B(S+2)[K row = i0 + o][c, plane, ks]
#pragma unroll
        for (int o = 0; o < 2; ++o) {
          const float wx = o ? k4.z : k4.x;
          const float wy = kInverse ? -(o ? k4.w : k4.y) : (o ? k4.w : k4.y);
          const float zr = yr[o] * wx - yi[o] * wy, zi = yr[o] * wy + yi[o] * wx;
          if constexpr (kF16) {
            const uint32_t off = atom_re + 1024u * (uint32_t)u;
            st_shared_b16(bdst + off + ba[bi][o], __half_as_ushort(__float2half_rn(zr * scale)));
            st_shared_b16(bdst + off + ba[bi][2 + o], __half_as_ushort(__float2half_rn(zi * scale)));
          } else {
            const uint32_t off = 1024u * (uint32_t)u + ba[bi][o];
            st_shared_b32(bdst + atom_re + off, __float_as_uint(round_tf32(zr)));
            st_shared_b32(bdst + atom_im + off, __float_as_uint(round_tf32(zi)));
          }
        }
      } else if constexpr (S == 1) {
        // X[L ka + i0 + o] * H, written as the inverse's input B3[K row = ka][c, plane, i0 + o]
        const float z0r = yr[0] * k4.x - yi[0] * k4.y, z0i = yr[0] * k4.y + yi[0] * k4.x;
        const float z1r = yr[1] * k4.z - yi[1] * k4.w, z1i = yr[1] * k4.w + yi[1] * k4.z;
        if constexpr (kF16) {
          // half2 of (i0, i0+1); 16-B chunk v = (plane L mod 64)/8 + u of the plane's atom
          constexpr int vim = (C::L % 64) / 8;
          const uint32_t pim = (uint32_t)(C::L / 64) * C::LBO;   // im plane in the next atom (L = 64)
          __half2 hr = __floats2half2_rn(z0r, z1r), hi = __floats2half2_rn(z0i, z1i);
          st_shared_b32(bdst + atom_re + bb[bi][u], *reinterpret_cast<uint32_t*>(&hr));
          st_shared_b32(bdst + atom_re + pim + bb[bi][vim + u], *reinterpret_cast<uint32_t*>(&hi));
        } else {
          const uint32_t off = (uint32_t)(u / 4) * C::LBO + bb[bi][u % 4];
          st_shared_v2(bdst + atom_re + off, round_tf32(z0r), round_tf32(z1r));
          st_shared_v2(bdst + atom_im + off, round_tf32(z0i), round_tf32(z1i));
        }
      } else {
        // outputs m = L ks + i0 + o: re -> signal 2c, im -> signal 2c+1
        if (yre) *reinterpret_cast<float2*>(yre + 8 * u) = make_float2(yr[0] * scale, yr[1] * scale);
        if (yim) *reinterpret_cast<float2*>(yim + 8 * u) = make_float2(yi[0] * scale, yi[1] * scale);
      }
    }
  }
  tc_fence_before();
  if (S < 3) fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    mbar_arrive(&sh.d_empty[S]);
    if (S < 3) mbar_arrive(&sh.b_full[S]);
  }
  return true;
}

// Epilogue warps of the conv1d kernel: group A (kGroupA, warps 2-5) runs E1
// and E3, group B (warps 6-9) runs E2 and E4, each over all rounds.  The two
// groups keep different per-thread constants, so they are separate
// instantiations (the registers of one never hold the other's).
template <class C, bool kGroupA>
__device__ __forceinline__ void conv1d_epilogue_group(const Conv1dParams& p, int T, uint32_t tmem,
                                                      const Conv1dShared& sh, uint32_t warp, uint32_t lane,
                                                      int hw, float spec_scale) {
  const uint32_t q = warp & 3u;
  const int l4 = (int)(lane & 3u);
  constexpr int kU = C::L / 8;
  constexpr int kB = C::kWarpBlocks;
  int ksv[kB];
  // the warp's 16-row blocks: M = 128 (L = 64) -> block hw of the quadrant's
  // two; M = 64 -> the quadrant's only block
#pragma unroll
  for (int bi = 0; bi < kB; ++bi) ksv[bi] = ((C::M == 64) ? (int)q : (int)(2 * q) + hw) * 8 + (int)(lane >> 2);
  // group A: forward twiddles w_N^-(a ks) of its pairs (inverse = conjugate);
  // group B: spectrum values H[L ka + i0 + o] (ka = ks) as float4 pairs.
  float4 cst[kB][kU];
  // Shared-memory store bases with the swizzle XOR folded in.
  //  f32 operands (128-B rows, 32-B swizzle atoms, 32 columns per atom):
  //   E1/E3: B[K row 8u + 2 l4 + o][col base + ks] = atom + 1024 u + ba[bi][o]
  //   E2:    B3[K row ks][col base + 8u + 2 l4] (v2)  = atom + LBO (u / 4) + bb[bi][u % 4]
  //  f16 operands (128-B rows, 16-B swizzle chunks, 64 columns per atom):
  //   E1/E3: + 1024 u + ba[bi][2 plane + o]   (one half per store)
  //   E2:    + bb[bi][chunk]                   (a half2 of i0, i0+1)
  uint32_t ba[kB][4], bb[kB][8];
#pragma unroll
  for (int bi = 0; bi < kB; ++bi) {
    const int ks = ksv[bi];
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const uint32_t kr = (uint32_t)(2 * l4 + o);
      if constexpr (C::kF16) {
#pragma unroll
        for (int pl = 0; pl < 2; ++pl) {
          const int col = pl * C::L + ks;   // within the signal's 2L columns
          ba[bi][2 * pl + o] = (uint32_t)(col / C::E16) * C::LBO + kr * 128u +
                               ((uint32_t)((col % C::E16) * 2) ^ ((kr & 7u) << 4));
        }
      } else {
        ba[bi][o] = (uint32_t)(ks / C::E) * C::LBO + kr * 128u + ((uint32_t)((ks % C::E) * 4) ^ ((kr & 3u) << 5));
        ba[bi][2 + o] = 0;
      }
    }
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      if constexpr (C::kF16)
        bb[bi][v] = (uint32_t)ks * 128u + 4u * (uint32_t)l4 + ((uint32_t)(v ^ (ks & 7)) << 4);
      else
        bb[bi][v] = (uint32_t)ks * 128u + 8u * (uint32_t)l4 + ((uint32_t)((v & 3) ^ (ks & 3)) << 5);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int i0 = 8 * u + 2 * l4;
      if constexpr (kGroupA) {
        const float2 w0 = p.tw[(i0 * ks) % C::N], w1 = p.tw[((i0 + 1) * ks) % C::N];
        cst[bi][u] = make_float4(w0.x, w0.y, w1.x, w1.y);
      } else {
        const float4 h = __ldg(reinterpret_cast<const float4*>(p.spec + C::L * ks + i0));
        cst[bi][u] = make_float4(h.x * spec_scale, h.y * spec_scale, h.z * spec_scale, h.w * spec_scale);
      }
    }
  }

  for (int r = 0; r < T + 3; ++r) {
    bool ok = true;
    if constexpr (kGroupA) {
      if (r < T) ok = conv1d_epilogue<C, 0>(p, r, tmem, sh, q, lane, l4, hw, ksv, cst, ba, bb);
      if (ok && r >= 2 && r - 2 < T)
        ok = conv1d_epilogue<C, 2>(p, r - 2, tmem, sh, q, lane, l4, hw, ksv, cst, ba, bb);
    } else {
      if (r >= 1 && r - 1 < T) ok = conv1d_epilogue<C, 1>(p, r - 1, tmem, sh, q, lane, l4, hw, ksv, cst, ba, bb);
      if (ok && r >= 3) ok = conv1d_epilogue<C, 3>(p, r - 3, tmem, sh, q, lane, l4, hw, ksv, cst, ba, bb);
    }
    if (!ok) break;
  }
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
conv1d_kernel(const __grid_constant__ CUtensorMap tmap_x, const Conv1dParams p) {
  using namespace sm100;
  using D = typename C::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_in_full[C::SIN], bar_in_empty[C::SIN], bar_scale[C::SIN];
  __shared__ uint64_t bar_d_full[4], bar_d_empty[4], bar_b_full[3], bar_b_empty[3], bar_const, bar_done;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t spec_max_bits;
  __shared__ int e1_ring[8];

  const uint32_t warp = warp_id(), lane = lane_id();
  const long long batch = p.batch;
  const long long per_tile = 2LL * C::TC;
  const long long num_tiles = (batch + per_tile - 1) / per_tile;
  const int T = (int)((num_tiles > blockIdx.x) ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0);

  if (threadIdx.x == 0) {
    // kMixed: an input slot is free once stage 1 read it and the range-scale warp scanned it
    for (int i = 0; i < C::SIN; ++i) {
      mbar_init(&bar_in_full[i], 1); mbar_init(&bar_in_empty[i], C::kF16 ? 2 : 1); mbar_init(&bar_scale[i], 1);
    }
    for (int i = 0; i < 4; ++i) { mbar_init(&bar_d_full[i], 1); mbar_init(&bar_d_empty[i], C::kGroupWarps); }
    for (int i = 0; i < 3; ++i) { mbar_init(&bar_b_full[i], C::kGroupWarps); mbar_init(&bar_b_empty[i], 1); }
    mbar_init(&bar_const, 1);
    mbar_init(&bar_done, 1);
    spec_max_bits = 0u;
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (C::kF16) {
    // CTA-wide max |H| (for the stage-3 input scale); non-negative floats
    // order like their bit patterns
    float m = 0.f;
    for (int k = threadIdx.x; k < C::N; k += blockDim.x) {
      const float2 h = __ldg(p.spec + k);
      m = fmaxf(m, fmaxf(fabsf(h.x), fabsf(h.y)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) atomicMax(&spec_max_bits, __float_as_uint(m));
    __syncthreads();
  }
  const uint32_t tmem = tmem_slot;
  uint8_t* const bbuf = smem + C::OFF_B;  // B2, B3, B4

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      mbar_arrive_expect_tx(&bar_const, C::A_BYTES + C::A16_BYTES);
      bulk_load(smem + C::OFF_A, p.a, C::A_BYTES, &bar_const);
      if constexpr (C::kF16) bulk_load(smem + C::OFF_A16, p.a16, C::A16_BYTES, &bar_const);
    }
    for (int i = 0; i < T; ++i) {
      const long long tile = blockIdx.x + (long long)i * gridDim.x;
      const int slot = i % C::SIN;
      if (!mbar_wait_warp(&bar_in_empty[slot], ((uint32_t)(i / C::SIN) & 1u) ^ 1u, p.err, kDevTimeoutProducer)) break;
      if (lane == 0) {
        // 2*TC real signals, rows s < L (rows >= lin/L and signals >= batch
        // are zero-filled by the tensor map bounds)
        mbar_arrive_expect_tx(&bar_in_full[slot], C::TILE_BYTES);
        tma_load_4d(smem + C::OFF_IN + slot * C::TILE_BYTES, &tmap_x, &bar_in_full[slot], 0, 0, 0,
                    (int)(tile * per_tile));
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&bar_const, 0, p.err, kDevTimeoutMma);
      const uint32_t idesc = instr_desc(D::kFmt, C::M, C::NCOL, 0, 1);
      const uint32_t idesc16 = instr_desc(kFmtF16, C::M, C::NCOL, 0, 1);
      const uint32_t lboA = (C::M / 8) * 128;
      const int ks1 = (p.rows_valid + 7) / 8;  // stage 1 skips all-zero K rows
      // All descriptors are built once; a K step adds its byte offset >> 4 to
      // the start-address field (addresses < 256 KB never carry out of it).
      // The K loops are fully unrolled: a single issuing thread that rebuilds
      // descriptors per MMA cannot keep the tensor core fed.
      const uint64_t adA = smem_desc(smem_u32(smem + C::OFF_A), lboA, 128, kSwNone);
      const uint64_t adA16 = smem_desc(smem_u32(smem + C::OFF_A16), lboA, 128, kSwNone);
      // input slot i / B tile i: the descriptor of slot 0 / B2 plus i tiles
      const uint64_t bdIn0 = smem_desc(smem_u32(smem + C::OFF_IN), C::LBO, D::kBSbo, D::kBSwizzle);
      const uint64_t bdB0 = C::kF16 ? smem_desc(smem_u32(bbuf), C::LBO, 1024, kSw128)
                                    : smem_desc(smem_u32(bbuf), C::LBO, D::kBSbo, D::kBSwizzle);
      // TF32: K step of 8 = 2 A core columns, 8 B rows (1024 B)
      auto stage_tf32 = [&](uint32_t d, uint64_t bd, int ksteps) {
#pragma unroll
        for (int k = 0; k < C::KSTEPS; ++k)
          if (k < ksteps)
            umma_tf32(d, adA + (uint64_t)((k * 2 * lboA) >> 4), bd + (uint64_t)((k * 1024) >> 4), idesc, k > 0);
      };
      // FP16: K step of 16 = 2 A core columns, 16 B rows (2048 B)
      auto stage_f16 = [&](uint32_t d, uint64_t bd) {
#pragma unroll
        for (int k = 0; k < C::KSTEPS16; ++k)
          umma_f16(d, adA16 + (uint64_t)((k * 2 * lboA) >> 4), bd + (uint64_t)((k * 2048) >> 4), idesc16, k > 0);
      };
      for (int r = 0; ok && r < T + 3; ++r) {
        // S1(r): input slot -> D0
        if (r < T) {
          const int slot = r % C::SIN;
          if (!mbar_wait(&bar_in_full[slot], (uint32_t)(r / C::SIN) & 1u, p.err, kDevTimeoutMma) ||
              !mbar_wait(&bar_d_empty[0], ((uint32_t)r & 1u) ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          stage_tf32(detail::acc_addr<C>(tmem, 0, 0, 0), bdIn0 + (uint64_t)(slot * (C::TILE_BYTES >> 4)), ks1);
          umma_commit(&bar_in_empty[slot]);
          umma_commit(&bar_d_full[0]);
        }
        // S2(r-1), S3(r-2), S4(r-3): B(s-2) -> D(s-1)
#pragma unroll 1
        for (int s = 1; s < 4; ++s) {
          const int j = r - s;
          if (j < 0 || j >= T) continue;
          if (!mbar_wait(&bar_b_full[s - 1], (uint32_t)j & 1u, p.err, kDevTimeoutMma) ||
              !mbar_wait(&bar_d_empty[s], ((uint32_t)j & 1u) ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bd = bdB0 + (uint64_t)((s - 1) * (C::BT_BYTES >> 4));
          if constexpr (C::kF16) stage_f16(detail::acc_addr<C>(tmem, s, 0, 0), bd);
          else stage_tf32(detail::acc_addr<C>(tmem, s, 0, 0), bd, C::KSTEPS);
          umma_commit(&bar_b_empty[s - 1]);
          umma_commit(&bar_d_full[s]);
        }
      }
      umma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.err, kDevTimeoutMma);
    }
    __syncwarp();
  } else if (warp < 2 + 2 * C::kGroupWarps) {
    // ------------------------------------------------------------ epilogues
    // group A (warps 2-9): E1 (D0 -> B2) and E3 (D2 -> B4)
    // group B (warps 10-17): E2 (D1 -> *H -> B3) and E4 (D3 -> y)
    // (two warps per TMEM lane quadrant in each group, hw = 0, 1)
    // Thread (q = warp % 4, lane) owns, per 16-row block bi, the row pair
    // ks = block*8 + lane/4 and the index pairs (i0, i0+1), i0 = 8u + 2*l4,
    // u < L/8.  Everything that depends only on (ks, l4) — twiddles or
    // spectrum values, shared-memory bases with the swizzle folded in — is
    // computed once; per element only compile-time offsets remain.
    Conv1dShared sh;
    sh.d_full = bar_d_full; sh.d_empty = bar_d_empty; sh.b_full = bar_b_full; sh.b_empty = bar_b_empty;
    sh.scale_full = bar_scale; sh.e1_ring = e1_ring; sh.bbuf = bbuf;
    sh.e2 = 0; sh.e3 = 0;
    float spec_scale = 1.f;
    if constexpr (C::kF16) {
      const float mh = __uint_as_float(spec_max_bits);
      // |B3| <= L 2^13.5 |H|  ->  s2 = 2^-ceil(log2(L sqrt2 max|H|))
      sh.e2 = (mh > 0.f) ? -detail::ceil_log2f((float)C::L * 1.41421357f * mh) : 0;
      sh.e3 = -detail::ceil_log2f((float)C::L * 1.41421357f);
      spec_scale = detail::pow2f(sh.e2);
    }
    const bool group_a = warp < 2 + C::kGroupWarps;
    const int hw = (int)((warp - 2 - (group_a ? 0 : C::kGroupWarps)) >> 2);
    if (group_a) conv1d_epilogue_group<C, true>(p, T, tmem, sh, warp, lane, hw, spec_scale);
    else conv1d_epilogue_group<C, false>(p, T, tmem, sh, warp, lane, hw, spec_scale);
  } else if constexpr (C::kF16) {
    // ------------------------------------------------------------ range scale
    // Per input tile: max |x| over its real signals -> exponent of the
    // stage-2 input scale, s1 = 2^(13 - ceil(log2(R sqrt2 max|x|))).
    const float rb = (float)p.rows_valid * 1.41421357f;
    for (int i = 0; i < T; ++i) {
      const int slot = i % C::SIN;
      if (!mbar_wait_warp(&bar_in_full[slot], (uint32_t)(i / C::SIN) & 1u, p.err, kDevTimeoutEpilogue)) break;
      const float4* t = reinterpret_cast<const float4*>(smem + C::OFF_IN + slot * C::TILE_BYTES);
      float m = 0.f;
#pragma unroll 8
      for (int k = (int)lane; k < C::TILE_BYTES / 16; k += 32) {
        const float4 v = t[k];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) {
        // clamped to pow2f's exact range (+-120) here, where every later use
        // reads it, so the stage scales stay consistent.  (The final unscale
        // -(e1 + e2 + e3) <= log2(max|x| max|H|) + 10 stays in that range
        // while max|x| max|H| <= 2^110.)
        const int e1 = (m > 0.f) ? 13 - detail::ceil_log2f(rb * m) : 0;
        e1_ring[i & 7] = e1 < -120 ? -120 : (e1 > 120 ? 120 : e1);
        mbar_arrive(&bar_scale[slot]);
        mbar_arrive(&bar_in_empty[slot]);
      }
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Filter spectrum H[k] = (1/N) sum_{j<taps} h[j] exp(-2 pi i j k / N) by
// direct summation with exact angle reduction (one thread per bin).
__global__ void conv1d_spectrum_kernel(const float* __restrict__ h, int taps, int n, float2* __restrict__ spec) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  double sr = 0.0, si = 0.0;
  for (int j = 0; j < taps; ++j) {
    const long long idx = ((long long)j * k) % n;
    double s, c;
    sincospi(-2.0 * (double)idx / (double)n, &s, &c);
    sr += h[j] * c;
    si += h[j] * s;
  }
  spec[k] = make_float2((float)(sr / n), (float)(si / n));
}

}  // namespace thff
