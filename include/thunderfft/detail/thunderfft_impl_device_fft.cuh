// thunderfft_impl_device_fft.cuh — ThunderFFT_kernel_reg: the composable
// in-kernel FFT of the device API.
//
// The reference's device routine (ThunderFFT_kernel_reg, shared_kernel_n*.cuh)
// is a warp-MMA register FFT with size-specific fragment maps.  This library
// keeps its calling contract (block shape, 32-element fragments, caller
// workspace and barriers) and computes it as a mixed-radix self-sorting
// (Stockham) FFT in FP32 registers:
//
//   * thread t of the P = 32 * warp_per_block<N> threads holds elements
//     n = t + P*m (m < M = N/P) of each of its signals, so the first pass is
//     an M-point DFT over the thread's own fragment and needs no exchange;
//   * the middle passes (radix 2..16) run butterflies q = t + P*h, read and
//     written through the caller's workspace with a per-exchange padding
//     that keeps the shared-memory accesses free of bank conflicts;
//   * the last pass is again M-point with butterfly j = t, so its outputs
//     k = t + P*r land in the fragment convention with no exchange.
//
// Radix plans (first | middle | last): 64: 2|16|2, 128: 4|8|4,
// 256: 2|8|8|2, 512: 16|2|16, 1024: 32|32, 2048: 32|2|32, 4096: 32|4|32.
// Register DFTs are radix-2 decimation in frequency with compile-time roots;
// inter-pass twiddles come from a few exact sincospif anchors (every 8th
// power) and depth-3 product trees, or from compile-time roots where a
// thread's twiddle base takes only two values.  Workspace accesses are a
// per-thread base plus compile-time offsets.
//
// half2 storage computes in packed FP16 (the half2/FP16 storage-arithmetic
// pair): a thread's butterflies are processed two at a time, the real parts
// of both in one half2 and the imaginary parts in another, so each half2
// instruction advances two butterflies with the same twiddles.  A pass with
// a single butterfly per thread (the radix-32 passes of N >= 1024) runs in
// FP32 between half2 loads and stores.  half2 N = 64 (16 signals) instead
// runs two warp-MMA DFT stages, and N = 128 (8 signals) the float2 TF32
// warp-MMA routine on FP32 copies of its registers, each on its own fragment
// orders (thunderfft_impl_device_mma.cuh).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <utility>

#include "thunderfft_impl_device_mma.cuh"
#include "util_arith.h"
#include "util_cuda.h"

namespace thunderfft {
namespace detail {

template <typename T>
__device__ __forceinline__ float2 to_f2(vec2_t<T> v) {
  if constexpr (std::is_same_v<T, half>) return __half22float2(v);
  else return v;
}
template <typename T>
__device__ __forceinline__ vec2_t<T> from_f2(float2 v) {
  if constexpr (std::is_same_v<T, half>) return __floats2half2_rn(v.x, v.y);
  else return v;
}

namespace dfft {

// ---- compile-time roots of unity ------------------------------------------
struct CRoot {
  double c, s;
};

// (cos, sin)(2*pi*k/n): exact quadrant reduction in integers, then a Taylor
// series on [0, pi/2) in double.
__host__ __device__ constexpr CRoot croot(int k, int n) {
  k %= n;
  if (k < 0) k += n;
  const int q = (4 * k) / n;
  const int rem = 4 * k - q * n;  // angle inside the quadrant = (pi/2) * rem / n
  const double x = 1.5707963267948966192 * double(rem) / double(n);
  double s = x, c = 1.0, ts = x, tc = 1.0;
  for (int i = 1; i < 16; ++i) {
    ts *= -x * x / double((2 * i) * (2 * i + 1));
    tc *= -x * x / double((2 * i - 1) * (2 * i));
    s += ts;
    c += tc;
  }
  if (rem == 0) {
    s = 0.0;
    c = 1.0;
  }
  switch (q) {
    case 1: return CRoot{-s, c};
    case 2: return CRoot{-c, -s};
    case 3: return CRoot{s, -c};
    default: return CRoot{c, s};
  }
}

// v * exp(sign * 2*pi*i * K / D), sign = -1 forward; trivial and 45-degree
// roots take the short forms.
template <int K, int D, bool fwd>
__device__ __forceinline__ float2 rot(float2 v) {
  constexpr int k = ((K % D) + D) % D;
  if constexpr (k == 0) {
    return v;
  } else if constexpr (2 * k == D) {
    return make_float2(-v.x, -v.y);
  } else if constexpr (4 * k == D || 4 * k == 3 * D) {
    // exp(-i pi/2) = -i forward; the inverse and the 3/4 turn flip it
    constexpr bool minus_i = (4 * k == D) == fwd;
    return minus_i ? make_float2(v.y, -v.x) : make_float2(-v.y, v.x);
  } else {
    constexpr CRoot w = croot(k, D);
    constexpr float c = float(w.c), s = fwd ? float(-w.s) : float(w.s);
    if constexpr ((8 * k) % D == 0) {
      // |c| = |s| = sqrt(1/2)
      constexpr float a = c > 0 ? 0.70710678118654752f : -0.70710678118654752f;
      constexpr bool same = (c > 0) == (s > 0);
      return same ? make_float2(a * (v.x - v.y), a * (v.x + v.y)) : make_float2(a * (v.x + v.y), a * (v.y - v.x));
    } else {
      return make_float2(fmaf(v.x, c, -v.y * s), fmaf(v.x, s, v.y * c));
    }
  }
}

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmulf(float2 a, float2 w) {
  return make_float2(fmaf(a.x, w.x, -a.y * w.y), fmaf(a.x, w.y, a.y * w.x));
}

// ---- packed FP16: two complex values per (re, im) pair of half2 ----------
// Lane 0 of both halves is one butterfly's value, lane 1 another's; every
// half2 instruction advances both butterflies.
struct HP {
  half2 re, im;
};

// IEEE binary16 bits of x (round to nearest even); x is 0 or normal-range
// (the roots of unity used here are >= sin(2*pi/4096) in magnitude).
__host__ __device__ constexpr unsigned short half_bits(double x) {
  if (x == 0.0) return 0;
  const unsigned short sign = x < 0 ? 0x8000 : 0;
  if (x < 0) x = -x;
  int e = 0;
  while (x >= 2.0) { x *= 0.5; ++e; }
  while (x < 1.0) { x *= 2.0; --e; }
  const double m = (x - 1.0) * 1024.0;
  long long mi = (long long)m;
  const double frac = m - double(mi);
  if (frac > 0.5 || (frac == 0.5 && (mi & 1))) ++mi;
  if (mi == 1024) { mi = 0; ++e; }
  return (unsigned short)(sign | (unsigned short)((e + 15) << 10) | (unsigned short)mi);
}
template <unsigned short B>
__device__ __forceinline__ half2 hconst2() {
  return __halves2half2(__ushort_as_half(B), __ushort_as_half(B));
}

__device__ __forceinline__ HP cadd(HP a, HP b) { return HP{__hadd2(a.re, b.re), __hadd2(a.im, b.im)}; }
__device__ __forceinline__ HP csub(HP a, HP b) { return HP{__hsub2(a.re, b.re), __hsub2(a.im, b.im)}; }
// v * w, w the same root in both lanes
__device__ __forceinline__ HP cmulh(HP v, HP w) {
  return HP{__hfma2(v.re, w.re, __hneg2(__hmul2(v.im, w.im))), __hfma2(v.re, w.im, __hmul2(v.im, w.re))};
}
__device__ __forceinline__ HP hpack(half2 a, half2 b) { return HP{__lows2half2(a, b), __highs2half2(a, b)}; }
__device__ __forceinline__ half2 hlo(HP v) { return __lows2half2(v.re, v.im); }
__device__ __forceinline__ half2 hhi(HP v) { return __highs2half2(v.re, v.im); }
__device__ __forceinline__ HP hbroadcast(float2 w) { return HP{__float2half2_rn(w.x), __float2half2_rn(w.y)}; }

template <int K, int D, bool fwd>
__device__ __forceinline__ HP rot(HP v) {
  constexpr int k = ((K % D) + D) % D;
  if constexpr (k == 0) {
    return v;
  } else if constexpr (2 * k == D) {
    return HP{__hneg2(v.re), __hneg2(v.im)};
  } else if constexpr (4 * k == D || 4 * k == 3 * D) {
    constexpr bool minus_i = (4 * k == D) == fwd;
    return minus_i ? HP{v.im, __hneg2(v.re)} : HP{__hneg2(v.im), v.re};
  } else {
    constexpr CRoot w = croot(k, D);
    constexpr double c = w.c, s = fwd ? -w.s : w.s;
    if constexpr ((8 * k) % D == 0) {
      const half2 a = hconst2<half_bits(c > 0 ? 0.70710678118654752 : -0.70710678118654752)>();
      constexpr bool same = (c > 0) == (s > 0);
      return same ? HP{__hmul2(a, __hsub2(v.re, v.im)), __hmul2(a, __hadd2(v.re, v.im))}
                  : HP{__hmul2(a, __hadd2(v.re, v.im)), __hmul2(a, __hsub2(v.im, v.re))};
    } else {
      const half2 hc = hconst2<half_bits(c)>(), hs = hconst2<half_bits(s)>();
      return HP{__hfma2(v.re, hc, __hneg2(__hmul2(v.im, hs))), __hfma2(v.re, hs, __hmul2(v.im, hc))};
    }
  }
}

// ---- R-point DFT in registers (radix-2 DIF; X[k] ends in v[brev<R>(k)]) ---
// V is float2 (FP32) or HP (two complex values in packed FP16).
template <int L, bool fwd, int I, typename V>
__device__ __forceinline__ void dif_bfly(V* v) {
  constexpr int k = I % L, p = (I / L) * 2 * L + k;
  const V a = v[p], b = v[p + L];
  v[p] = cadd(a, b);
  v[p + L] = rot<k, 2 * L, fwd>(csub(a, b));
}
template <int L, bool fwd, typename V, int... I>
__device__ __forceinline__ void dif_stage(V* v, std::integer_sequence<int, I...>) {
  (dif_bfly<L, fwd, I>(v), ...);
}
template <int R, int L, bool fwd, typename V>
__device__ __forceinline__ void dif_stages(V* v) {
  dif_stage<L, fwd>(v, std::make_integer_sequence<int, R / 2>{});
  if constexpr (L > 1) dif_stages<R, L / 2, fwd>(v);
}
template <int R, bool fwd, typename V>
__device__ __forceinline__ void dft(V* v) {
  if constexpr (R > 1) dif_stages<R, R / 2, fwd>(v);
}

template <int R>
__host__ __device__ constexpr int brev(int k) {
  int r = 0;
  for (int m = R; m > 1; m >>= 1) {
    r = (r << 1) | (k & 1);
    k >>= 1;
  }
  return r;
}

// v[0..R) from bit-reversed to natural order (register renaming only).
template <int R, typename V>
__device__ __forceinline__ void unscramble(V* v) {
  V tmp[R];
#pragma unroll
  for (int r = 0; r < R; ++r) tmp[r] = v[brev<R>(r)];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = tmp[r];
}

// exp(sign * 2*pi*i * num / den), den a power of two, exact argument.
template <bool fwd>
__device__ __forceinline__ float2 root(int num, int den) {
  float s, c;
  sincospif(float(num & (den - 1)) * (2.0f / float(den)), &s, &c);
  return make_float2(c, fwd ? -s : s);
}

template <int K, int D, bool fwd>
__device__ __forceinline__ float2 croot_f2() {
  constexpr CRoot w = croot(K, D);
  return make_float2(float(w.c), fwd ? float(-w.s) : float(w.s));
}
template <int D, bool fwd, int... I>
__device__ __forceinline__ void select_powers(float2* w, bool odd, std::integer_sequence<int, I...>) {
  ((w[I] = odd ? croot_f2<I, D, fwd>() : make_float2(1.0f, 0.0f)), ...);
}

// w[r] = exp(sign * 2*pi*i * r*km / den) for r < R.  km < 2: compile-time
// roots selected per thread.  Otherwise one exact sincospif root, powers
// 2..7 by a depth-3 product tree, and another sincospif anchor every 8
// powers.
template <int R, int Ns, bool fwd>
__device__ __forceinline__ void root_powers(float2* w, int km) {
  constexpr int den = Ns * R;
  if constexpr (Ns == 2) {
    select_powers<den, fwd>(w, km != 0, std::make_integer_sequence<int, R>{});
  } else {
    w[0] = make_float2(1.0f, 0.0f);
    if constexpr (R > 1) w[1] = root<fwd>(km, den);
    if constexpr (R > 2) w[2] = cmulf(w[1], w[1]);
    if constexpr (R > 3) w[3] = cmulf(w[2], w[1]);
    if constexpr (R > 4) w[4] = cmulf(w[2], w[2]);
    if constexpr (R > 5) w[5] = cmulf(w[4], w[1]);
    if constexpr (R > 6) w[6] = cmulf(w[4], w[2]);
    if constexpr (R > 7) w[7] = cmulf(w[4], w[3]);
#pragma unroll
    for (int a = 1; a < R / 8; ++a) {
      const float2 anchor = root<fwd>(8 * a * km, den);
      w[8 * a] = anchor;
#pragma unroll
      for (int b = 1; b < 8; ++b) w[8 * a + b] = cmulf(anchor, w[b]);
    }
  }
}

// Workspace layout of one exchange: element p at p + (p >> kPad) (kPad = 0:
// no padding).  kPad >= 4 stays inside (N + pad_h(N)) * batch elements.
template <int kPad>
__host__ __device__ constexpr int xidx(int p) {
  if constexpr (kPad == 0) return p;
  else return p + (p >> kPad);
}

// Radix plan and exchange layouts per N (register-file bound: M = N/P
// elements of each signal per thread in the first and last pass).
template <int N>
struct plan;
template <> struct plan<64>   { static constexpr int n = 3, R[4] = {2, 16, 2, 0},  pad8[3] = {4, 4, 0}, pad4[3] = {4, 4, 0}; };
template <> struct plan<128>  { static constexpr int n = 3, R[4] = {4, 8, 4, 0},   pad8[3] = {4, 4, 0}, pad4[3] = {5, 4, 0}; };
template <> struct plan<256>  { static constexpr int n = 4, R[4] = {2, 8, 8, 2},   pad8[3] = {4, 4, 0}, pad4[3] = {5, 5, 0}; };
template <> struct plan<512>  { static constexpr int n = 3, R[4] = {16, 2, 16, 0}, pad8[3] = {4, 0, 0}, pad4[3] = {5, 0, 0}; };
template <> struct plan<1024> { static constexpr int n = 2, R[4] = {32, 32, 0, 0}, pad8[3] = {5, 0, 0}, pad4[3] = {5, 0, 0}; };
template <> struct plan<2048> { static constexpr int n = 3, R[4] = {32, 2, 32, 0}, pad8[3] = {5, 0, 0}, pad4[3] = {5, 0, 0}; };
template <> struct plan<4096> { static constexpr int n = 3, R[4] = {32, 4, 32, 0}, pad8[3] = {5, 0, 0}, pad4[3] = {5, 0, 0}; };

template <typename T, int N>
__host__ __device__ constexpr int exchange_pad(int x) {
  return sizeof(vec2_t<T>) == 8 ? plan<N>::pad8[x] : plan<N>::pad4[x];
}

// Workspace positions of pass (R, Ns): butterfly q = t + P*h is (signal
// b = q / NB, j = q % NB), NB = N/R; it reads x[b][j + r*NB] and writes
// X[b][(j/Ns)*Ns*R + j%Ns + r*Ns].  With t < P and every factor a power of
// two, both positions are bit-field concatenations of t's bits and (h, r)'s
// bits, so index(t, h, r) = index(t, 0, 0) | index(0, h, r) and xidx splits
// the same way: each access is a per-thread base plus a compile-time offset.
template <int N, int P, int R>
__host__ __device__ constexpr int rd_index(int t, int h, int r) {
  return ((t + P * h) / (N / R)) * N + (t + P * h) % (N / R) + r * (N / R);
}
template <int N, int P, int R, int Ns>
__host__ __device__ constexpr int wr_index(int t, int h, int r) {
  const int q = t + P * h, j = q % (N / R);
  return (q / (N / R)) * N + (j / Ns) * Ns * R + j % Ns + r * Ns;
}

// Pass s of the plan over the thread's EPT registers.  Input r of a
// butterfly is multiplied by w^r, w = W_{Ns*R}^{j mod Ns} (j mod Ns =
// t mod Ns because Ns divides P).  The first pass (Ns = 1) reads the
// fragment; the last (Ns*R = N, NB = P, j = t) leaves its outputs in the
// fragment.
template <typename T, int N, int EPT, int P, bool fwd, int s, int Ns>
__device__ __forceinline__ void run_passes(float2* v, vec2_t<T>* ws, int t) {
  using Pl = plan<N>;
  constexpr int R = Pl::R[s], C = EPT / R;
  constexpr bool first = s == 0, last = s == Pl::n - 1;
  if constexpr (!first) {
    constexpr int padin = exchange_pad<T, N>(s - 1);
    const vec2_t<T>* src = ws + xidx<padin>(rd_index<N, P, R>(t, 0, 0));
#pragma unroll
    for (int h = 0; h < C; ++h) {
#pragma unroll
      for (int r = 0; r < R; ++r) v[h * R + r] = to_f2<T>(src[xidx<padin>(rd_index<N, P, R>(0, h, r))]);
    }
    float2 w[R];
    root_powers<R, Ns, fwd>(w, t & (Ns - 1));
#pragma unroll
    for (int h = 0; h < C; ++h) {
#pragma unroll
      for (int r = 1; r < R; ++r) v[h * R + r] = cmulf(v[h * R + r], w[r]);
    }
  }
#pragma unroll
  for (int h = 0; h < C; ++h) dft<R, fwd>(v + h * R);
  if constexpr (last) {
#pragma unroll
    for (int h = 0; h < C; ++h) unscramble<R>(v + h * R);
  } else {
    constexpr int padout = exchange_pad<T, N>(s);
    vec2_t<T>* dst = ws + xidx<padout>(wr_index<N, P, R, Ns>(t, 0, 0));
    __syncthreads();  // every thread's reads of the workspace are done
#pragma unroll
    for (int h = 0; h < C; ++h) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        dst[xidx<padout>(wr_index<N, P, R, Ns>(0, h, r))] = from_f2<T>(v[h * R + brev<R>(r)]);
    }
    __syncthreads();
    run_passes<T, N, EPT, P, fwd, s + 1, Ns * R>(v, ws, t);
  }
}

// half2 storage.  Passes whose thread owns C >= 2 butterflies run them in
// pairs (m, m + C/2) in packed FP16; a pass with one butterfly per thread
// (the radix-32 passes of N >= 1024) runs in FP32.  Same plan, positions and
// barriers as run_passes.
//
// For N <= 512 (batch_per_block >= 2) the pair (m, m + C/2) is, in every
// pass, the same position of signals b and b + B/2, so the workspace keeps
// the pairs packed: a plane of (re_b, re_b+B/2) half2 values followed by a
// plane of the imaginary parts, indexed by the lower signal's position.  Only
// entry and exit then move between the fragment's (re, im) half2 and the
// packed pairs.  Larger N exchange (re, im) half2 elements.
template <int N, int B>
__host__ __device__ constexpr bool packed_exchange() {
  return B >= 2 && N <= 512;
}

template <int N, int B, int EPT, int P, bool fwd, int s, int Ns>
__device__ __forceinline__ void run_passes_h(half2* reg, half2* ws, int t) {
  using Pl = plan<N>;
  constexpr int R = Pl::R[s], C = EPT / R;
  constexpr bool first = s == 0, last = s == Pl::n - 1;
  constexpr bool soa = packed_exchange<N, B>();
  constexpr int padin = first ? 0 : exchange_pad<half, N>(s - 1);
  constexpr int padout = last ? 0 : exchange_pad<half, N>(s);
  // packed planes: imaginary plane after the padded real plane of B/2 signals
  constexpr int PLin = soa ? xidx<padin>(B / 2 * N) : 0, PLout = soa ? xidx<padout>(B / 2 * N) : 0;
  const half2* src = ws + xidx<padin>(rd_index<N, P, R>(t, 0, 0));
  half2* dst = ws + xidx<padout>(wr_index<N, P, R, Ns>(t, 0, 0));
  if constexpr (C >= 2) {
    constexpr int CP = C / 2;
    HP v[CP * R];
#pragma unroll
    for (int m = 0; m < CP; ++m) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if constexpr (first) {
          v[m * R + r] = hpack(reg[m * R + r], reg[(m + CP) * R + r]);
        } else if constexpr (soa) {
          const int o = xidx<padin>(rd_index<N, P, R>(0, m, r));
          v[m * R + r] = HP{src[o], src[PLin + o]};
        } else {
          v[m * R + r] = hpack(src[xidx<padin>(rd_index<N, P, R>(0, m, r))],
                               src[xidx<padin>(rd_index<N, P, R>(0, m + CP, r))]);
        }
      }
    }
    if constexpr (!first) {
      float2 w[R];
      root_powers<R, Ns, fwd>(w, t & (Ns - 1));
#pragma unroll
      for (int r = 1; r < R; ++r) {
        const HP wh = hbroadcast(w[r]);
#pragma unroll
        for (int m = 0; m < CP; ++m) v[m * R + r] = cmulh(v[m * R + r], wh);
      }
    }
#pragma unroll
    for (int m = 0; m < CP; ++m) dft<R, fwd>(v + m * R);
    if constexpr (last) {
#pragma unroll
      for (int m = 0; m < CP; ++m) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          reg[m * R + r] = hlo(v[m * R + brev<R>(r)]);
          reg[(m + CP) * R + r] = hhi(v[m * R + brev<R>(r)]);
        }
      }
    } else {
      __syncthreads();  // every thread's reads of the workspace are done
#pragma unroll
      for (int m = 0; m < CP; ++m) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const HP x = v[m * R + brev<R>(r)];
          if constexpr (soa) {
            const int o = xidx<padout>(wr_index<N, P, R, Ns>(0, m, r));
            dst[o] = x.re;
            dst[PLout + o] = x.im;
          } else {
            dst[xidx<padout>(wr_index<N, P, R, Ns>(0, m, r))] = hlo(x);
            dst[xidx<padout>(wr_index<N, P, R, Ns>(0, m + CP, r))] = hhi(x);
          }
        }
      }
      __syncthreads();
    }
  } else {
    static_assert(!soa, "packed exchanges need two butterflies per thread in every pass");
    float2 v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if constexpr (first) v[r] = __half22float2(reg[r]);
      else v[r] = __half22float2(src[xidx<padin>(rd_index<N, P, R>(0, 0, r))]);
    }
    if constexpr (!first) {
      float2 w[R];
      root_powers<R, Ns, fwd>(w, t & (Ns - 1));
#pragma unroll
      for (int r = 1; r < R; ++r) v[r] = cmulf(v[r], w[r]);
    }
    dft<R, fwd>(v);
    if constexpr (last) {
#pragma unroll
      for (int r = 0; r < R; ++r) reg[r] = __floats2half2_rn(v[brev<R>(r)].x, v[brev<R>(r)].y);
    } else {
      __syncthreads();
#pragma unroll
      for (int r = 0; r < R; ++r)
        dst[xidx<padout>(wr_index<N, P, R, Ns>(0, 0, r))] = __floats2half2_rn(v[brev<R>(r)].x, v[brev<R>(r)].y);
      __syncthreads();
    }
  }
  if constexpr (!last) run_passes_h<N, B, EPT, P, fwd, s + 1, Ns * R>(reg, ws, t);
}

// half2 N = 256, 16 signals, 128 threads (fragment mfft::frag256_h): thread
// t = 16 p + q runs signals 2p and 2p + 1 as packed pairs.  256 = 16 x 16:
//   pass 1  Y[q][k1] = sum_r x[q + 16 r] W16^(r k1), times W256^(q k1)
//   pass 2  X[k1 + 16 k2] = sum_q Y[q][k1] W16^(q k2), thread q' taking k1 = q'
// One exchange through the workspace: planes of packed real and imaginary
// parts, pair p's plane row k1 at p (N + pad_h(N)) + 17 k1 (the odd row
// stride keeps both the row writes and the column reads free of bank
// conflicts); the two planes use 2 x 8 x 272 = (N + pad_h(N)) x 16 elements.
template <bool fwd>
__device__ __forceinline__ void run256_h(half2* reg, half2* ws, int t) {
  constexpr int kPair = 256 + 256 / 16, kPlane = 8 * kPair;   // N + pad_h(N) per pair
  const int p = t >> 4, q = t & 15;
  HP v[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) v[r] = hpack(reg[r], reg[16 + r]);
  dft<16, fwd>(v);   // v[brev(k1)] = Y[q][k1] before the twiddle
  float2 w[16];
  root_powers<16, 16, fwd>(w, q);   // w[k1] = W256^(q k1)
  half2* const row = ws + p * kPair + q;
  __syncthreads();  // every thread's reads of the workspace are done
#pragma unroll
  for (int k1 = 0; k1 < 16; ++k1) {
    const HP y = (k1 == 0) ? v[0] : cmulh(v[brev<16>(k1)], hbroadcast(w[k1]));
    row[17 * k1] = y.re;
    row[kPlane + 17 * k1] = y.im;
  }
  __syncthreads();
  const half2* const col = ws + p * kPair + 17 * q;
#pragma unroll
  for (int qq = 0; qq < 16; ++qq) v[qq] = HP{col[qq], col[kPlane + qq]};
  dft<16, fwd>(v);   // v[brev(k2)] = X[q + 16 k2]
#pragma unroll
  for (int k2 = 0; k2 < 16; ++k2) {
    reg[k2] = hlo(v[brev<16>(k2)]);
    reg[16 + k2] = hhi(v[brev<16>(k2)]);
  }
}

}  // namespace dfft
}  // namespace detail

template <typename T, int N, int batch, bool forward>
__device__ __forceinline__ void ThunderFFT_kernel_reg(vec2_t<T>* __restrict__ reg, vec2_t<T>* __restrict__ W,
                                                      void* workspace) {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>, "float and half only");
  static_assert(N == 64 || N == 128 || N == 256 || N == 512 || N == 1024 || N == 2048 || N == 4096,
                "Unsupported ThunderFFT length");
  (void)W;
  using F = detail::frag<N, batch>;
  static_assert(F::EPT % (N / F::P) == 0, "fragment must hold whole first-pass butterflies");
  vec2_t<T>* ws = static_cast<vec2_t<T>*>(workspace);
  const int t = detail::block_thread();
  if constexpr (detail::mfft::enabled<T, N, batch>) {
    detail::mfft::run64<T, forward>(reg, ws, t);
  } else if constexpr (detail::mfft::tf32_enabled<T, N, batch> && std::is_same_v<T, half>) {
    // half2 N = 128: the TF32 routine on FP32 copies of the registers (the
    // half2 values are exact in TF32; FP32 accumulation), rounded back
    float2 r[detail::frag<N, batch>::EPT];
#pragma unroll
    for (int i = 0; i < detail::frag<N, batch>::EPT; ++i) r[i] = __half22float2(reg[i]);
    detail::mfft::run128_tf32<forward>(r, t);
#pragma unroll
    for (int i = 0; i < detail::frag<N, batch>::EPT; ++i) reg[i] = __float22half2_rn(r[i]);
  } else if constexpr (detail::mfft::tf32_enabled<T, N, batch>) {
    float2* r = reinterpret_cast<float2*>(reg);
    if constexpr (N == 64) detail::mfft::run64_tf32<forward>(r, t);
    else if constexpr (N == 128) detail::mfft::run128_tf32<forward>(r, t);
    else detail::mfft::run256_tf32<forward>(r, reinterpret_cast<float2*>(ws), t);
  } else if constexpr (detail::mfft::h256_enabled<T, N, batch>) {
    detail::dfft::run256_h<forward>(reg, ws, t);
  } else if constexpr (std::is_same_v<T, half>) {
    detail::dfft::run_passes_h<N, batch, F::EPT, F::P, forward, 0, 1>(reg, ws, t);
  } else {
    float2 v[F::EPT];
#pragma unroll
    for (int i = 0; i < F::EPT; ++i) v[i] = reg[i];
    detail::dfft::run_passes<T, N, F::EPT, F::P, forward, 0, 1>(v, ws, t);
#pragma unroll
    for (int i = 0; i < F::EPT; ++i) reg[i] = v[i];
  }
  __syncthreads();  // the workspace is the caller's again
}

}  // namespace thunderfft
