// thff_capi.cu — C ABI of libthunderfft_b200.so (declared in include/thff.h).
//
// Host side of the batched C2C FFT: argument contract of the reference's
// ThunderFFT_global wrapper (include/thunderfft/detail/thunderfft_impl_kernel.cuh:6-41),
// the reference-compatible twiddle cache (thunderfft_impl_twiddle.cuh:26-378),
// per-device FFT constants (stage DFT matrices in the UMMA operand layouts the
// kernels read, twiddle tables), TMA tensor maps and kernel launches.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/thff.h"
#include "fft_kernels.cuh"
#include "conv1d_kernel.cuh"
#include "conv2d_kernels.cuh"
#include "conv2d_fused.cuh"
#include "conv1d_tiled.cuh"

namespace {

constexpr double kTau = 6.283185307179586476925286766559;

thread_local std::string g_last_error;

thff_status fail(thff_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

thff_status cuda_fail(cudaError_t e, const char* what) {
  return fail(THFF_CUDA_ERROR, std::string("[ThunderFFT] ") + what + ": " + cudaGetErrorString(e));
}

// Host-side fault injection (thff_test_inject_cuda_error): per calling
// thread, the (skip+1)-th CUDA status checked through THFF_CUDA reads as the
// armed error.  The CUDA call itself has run; only its reported status
// changes, so the error paths above the C ABI can be exercised without
// making a GPU fail.
thread_local int g_inject_error = 0;
thread_local int g_inject_skip = 0;

cudaError_t injected(cudaError_t real) {
  if (g_inject_error == 0) return real;
  if (g_inject_skip > 0) {
    --g_inject_skip;
    return real;
  }
  const cudaError_t e = static_cast<cudaError_t>(g_inject_error);
  g_inject_error = 0;
  return e;
}

// Kernels this library has launched in this process (all devices); every
// launch site checks its launch through launched().
std::atomic<unsigned long long> g_launches{0};

cudaError_t launched() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

#define THFF_CUDA(expr, what)                      \
  do {                                             \
    cudaError_t e_ = injected(expr);               \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

bool valid_n(int n) {
  return n == 64 || n == 128 || n == 256 || n == 512 || n == 1024 || n == 2048 || n == 4096;
}
bool valid_dtype(int dt) { return dt == THFF_F32 || dt == THFF_F16; }

// ---------------------------------------------------------------------------
// Host-side value encodings
// ---------------------------------------------------------------------------
uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// Round to the nearest TF32 value (10 explicit mantissa bits), ties away —
// the tensor core would otherwise truncate the low 13 bits.
float tf32_rn(float x) {
  uint32_t u = f32_bits(x);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u = (u + 0x1000u) & 0xffffe000u;
  return bits_f32(u);
}

void put_value(std::vector<uint8_t>& img, size_t off, double v, bool half) {
  if (half) {
    const __half h = __float2half_rn(float(v));
    std::memcpy(img.data() + off, &h, 2);
  } else {
    const float f = tf32_rn(float(v));
    std::memcpy(img.data() + off, &f, 4);
  }
}

// Byte offset of element (m, k) of an M x K K-major operand without swizzle:
// 8x16-byte core matrices stored contiguously, core (m/8, kbyte/16) at
// ((kbyte/16) * (M/8) + m/8) * 128.
size_t kmajor_noswz_off(int m, int k, int M, int esz) {
  const int kb = k * esz;
  return size_t((kb / 16) * (M / 8) + m / 8) * 128 + (m % 8) * 16 + (kb % 16);
}

// Stage DFT matrix of length L for G signal groups (block diagonal):
// rows (g, ks, re|im) laid out in 16-row blocks [8 cos rows | 8 sin rows],
// rp = g*L + ks, row = 16*(rp/8) + 8*c + rp%8; columns k = g*L + s.
//   row (rp, 0): cos(theta), row (rp, 1): sin(theta), theta = sign*2*pi*s*ks/L
// rotation (fft2_kernel stage 2, thff::detail::stage2_rotation): column
// g*L + s sits at K index stage2_krow(rotation, g*L + s), the row where the
// stage-1 epilogue puts input s of group g.
std::vector<uint8_t> build_stage_matrix(int L, int G, int sign, bool half, int rotation = 0) {
  const int esz = half ? 2 : 4;
  const int M = 2 * L * G, K = L * G;
  std::vector<uint8_t> img(size_t(M) * K * esz, 0);
  for (int g = 0; g < G; ++g)
    for (int ks = 0; ks < L; ++ks) {
      const int rp = g * L + ks;
      for (int c = 0; c < 2; ++c) {
        const int m = 16 * (rp / 8) + 8 * c + rp % 8;
        for (int s = 0; s < L; ++s) {
          const double th = sign * kTau * double((s * ks) % L) / double(L);
          const int k = thff::detail::stage2_krow(rotation, g * L + s);
          put_value(img, kmajor_noswz_off(m, k, M, esz), c == 0 ? std::cos(th) : std::sin(th), half);
        }
      }
    }
  return img;
}

// Real 2N x 2N DFT matrix for the one-stage kernel, K-major with 128-B
// swizzle: row n = 2k + c_out, column K = 2j + c_in, stored
// [K/E][row][128 B] with the 16-B chunk index XORed by (row % 8).
std::vector<uint8_t> build_dft1_matrix(int N, int sign, bool half) {
  const int esz = half ? 2 : 4, E = 128 / esz, R = 2 * N;
  std::vector<uint8_t> img(size_t(R) * R * esz, 0);
  for (int n = 0; n < R; ++n)
    for (int K = 0; K < R; ++K) {
      const int k = n / 2, co = n % 2, j = K / 2, ci = K % 2;
      const double th = sign * kTau * double((j * k) % N) / double(N);
      const double c = std::cos(th), s = std::sin(th);
      const double v = (co == 0) ? (ci == 0 ? c : -s) : (ci == 0 ? s : c);
      const uint32_t within = uint32_t(n) * 128u + uint32_t(K % E) * esz;
      const size_t off = size_t(K / E) * (size_t(R) * 128) + thff::sm100::sw128(within);
      put_value(img, off, v, half);
    }
  return img;
}

// ---------------------------------------------------------------------------
// Per-device state
// ---------------------------------------------------------------------------
struct Consts {            // per (dtype, N, direction)
  void* a1 = nullptr;      // stage-1 A image (or the one-stage DFT matrix)
  void* a2 = nullptr;      // stage-2 A image
  void* tw = nullptr;      // float2 twiddles exp(sign 2 pi i k / N)
  void* a4 = nullptr;      // fused conv2d column pass: the inverse stage-2 A image
};

struct RefCache {          // reference-compatible twiddle cache entry
  void* dW = nullptr;
  int n = 0;
};

// Device error words, one per stream.  A kernel's bounded wait that runs
// out records its code in the word of the stream it was launched on, and
// every wait of that launch gives up once the word is non-zero, so a stalled
// CTA drains instead of waiting for work that will not come.  Launches on
// other streams have their own words: a timeout on one stream neither aborts
// another stream's kernels nor is reported to that stream's caller.  A word
// stays set until thff_sync_check on its stream reads it; the read clears it
// in stream order.  The words live in this fixed device array (no
// allocation); a device's first kErrSlots distinct streams get words of
// their own, later streams share them round robin.
constexpr int kErrSlots = 256;
static __device__ uint32_t g_err_words[kErrSlots];

struct DeviceState {
  bool ready = false;
  int sms = 0;
  uint32_t* d_err_words = nullptr;           // device address of g_err_words
  std::map<cudaStream_t, int> err_slot;      // stream -> index into g_err_words
  int err_next = 0;
  std::map<int, Consts> consts;  // key = (dtype*2 + fwd)*8192 + N
  RefCache ref[2];
  std::map<const void*, bool> attr_done;
};

std::mutex g_mutex;
std::mutex g_err_mutex;                      // guards DeviceState::err_slot / err_next
std::map<int, DeviceState> g_dev;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// The error word of `stream` on this device.
uint32_t* stream_err(DeviceState& st, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_err_mutex);
  auto it = st.err_slot.find(stream);
  if (it == st.err_slot.end()) {
    it = st.err_slot.emplace(stream, st.err_next).first;
    st.err_next = (st.err_next + 1) % kErrSlots;
  }
  return st.d_err_words + it->second;
}

thread_local uint32_t* t_err_host = nullptr;  // pinned readback word per thread

thff_status current_device(int* dev) {
  THFF_CUDA(cudaGetDevice(dev), "cudaGetDevice");
  return THFF_OK;
}

thff_status ensure_device(int dev, DeviceState** out) {
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    cudaDeviceProp prop;
    THFF_CUDA(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
    if (prop.major != 10)
      return fail(THFF_UNSUPPORTED, std::string("[ThunderFFT] this build targets sm_100a (B200); device is ") +
                                        prop.name + " sm_" + std::to_string(prop.major) + std::to_string(prop.minor));
    st.sms = prop.multiProcessorCount;
    THFF_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&st.d_err_words), g_err_words),
              "cudaGetSymbolAddress(error words)");
    THFF_CUDA(cudaMemset(st.d_err_words, 0, sizeof(uint32_t) * kErrSlots), "cudaMemset(error words)");
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      THFF_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
      if (!fn || q != cudaDriverEntryPointSuccess)
        return fail(THFF_CUDA_ERROR, "[ThunderFFT] cuTensorMapEncodeTiled unavailable");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    st.ready = true;
  }
  *out = &st;
  return THFF_OK;
}

thff_status upload(const std::vector<uint8_t>& img, void** dst) {
  THFF_CUDA(cudaMalloc(dst, img.size()), "cudaMalloc(FFT constants)");
  THFF_CUDA(cudaMemcpy(*dst, img.data(), img.size(), cudaMemcpyHostToDevice), "cudaMemcpy(FFT constants)");
  return THFF_OK;
}

template <bool kHalf, int kN, int kVar = 0>
struct ShapeOf {
  using S = thff::Fft2Shape<kHalf, kN, kVar>;
  static constexpr int NS = S::NS, NA = S::NA, G1 = S::G1, G2 = S::G2;
};

// Shape variant 1 (NA = 32, float storage, N <= 512) exists for the 2-D
// convolution's pair-planar first pass.
bool has_variant1(int dtype, int n) { return dtype == THFF_F32 && (n == 128 || n == 256 || n == 512); }

thff_status build_consts(int dtype, int n, bool fwd, int var, Consts* c) {
  const bool half = dtype == THFF_F16;
  const int sign = fwd ? -1 : 1;
  thff_status st;
  if (n == 64) {
    if ((st = upload(build_dft1_matrix(64, sign, half), &c->a1)) != THFF_OK) return st;
  } else {
    int NS = 0, NA = 0, G1 = 0, G2 = 0;
#define THFF_SHAPE(H, NN, V)                                                                   \
  if (half == H && n == NN && var == V) {                                                      \
    NS = ShapeOf<H, NN, V>::NS; NA = ShapeOf<H, NN, V>::NA; G1 = ShapeOf<H, NN, V>::G1;        \
    G2 = ShapeOf<H, NN, V>::G2;                                                                 \
  }
    THFF_SHAPE(false, 128, 0) THFF_SHAPE(false, 256, 0) THFF_SHAPE(false, 512, 0) THFF_SHAPE(false, 1024, 0)
    THFF_SHAPE(false, 2048, 0) THFF_SHAPE(false, 4096, 0) THFF_SHAPE(true, 128, 0) THFF_SHAPE(true, 256, 0)
    THFF_SHAPE(true, 512, 0) THFF_SHAPE(true, 1024, 0) THFF_SHAPE(true, 2048, 0) THFF_SHAPE(true, 4096, 0)
    THFF_SHAPE(false, 128, 1) THFF_SHAPE(false, 256, 1) THFF_SHAPE(false, 512, 1)
#undef THFF_SHAPE
    if (NS == 0) return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] no such FFT shape");
    if ((st = upload(build_stage_matrix(NS, G1, sign, half), &c->a1)) != THFF_OK) return st;
    if ((st = upload(build_stage_matrix(NA, G2, sign, half, thff::detail::stage2_rotation(half, var)), &c->a2)) !=
        THFF_OK)
      return st;
  }
  std::vector<uint8_t> tw(size_t(n) * 8);
  for (int k = 0; k < n; ++k) {
    const double th = sign * kTau * double(k) / double(n);
    const float v[2] = {float(std::cos(th)), float(std::sin(th))};
    std::memcpy(tw.data() + size_t(k) * 8, v, 8);
  }
  return upload(tw, &c->tw);
}

int consts_key(int dtype, int n, bool fwd, int var) { return ((var * 2 + dtype) * 2 + (fwd ? 1 : 0)) * 8192 + n; }

thff_status get_consts(DeviceState& st, int dtype, int n, bool fwd, const Consts** out, int var = 0) {
  const int key = consts_key(dtype, n, fwd, var);
  auto it = st.consts.find(key);
  if (it == st.consts.end()) {
    Consts c;
    thff_status s = build_consts(dtype, n, fwd, var, &c);
    if (s != THFF_OK) return s;
    it = st.consts.emplace(key, c).first;
  }
  *out = &it->second;
  return THFF_OK;
}

// ---------------------------------------------------------------------------
// Launch helpers
// ---------------------------------------------------------------------------
thff_status encode(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                   const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                   CUtensorMapSwizzle swz) {
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) { gd[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = g_encode(map, dt, rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(THFF_CUDA_ERROR, "[ThunderFFT] cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return THFF_OK;
}

template <class K>
thff_status set_smem_attr(DeviceState& st, K kernel, int bytes) {
  const void* key = reinterpret_cast<const void*>(kernel);
  if (!st.attr_done[key]) {
    THFF_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
              "cudaFuncSetAttribute(max dynamic shared memory)");
    st.attr_done[key] = true;
  }
  return THFF_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tensor map of a conv2d input mode.  Both modes deliver the stage-1 tile in
// the MN-major [128-B column atom][K row][128 B] layout with every box row one
// whole 128-B line; see thff::InMode for the column order.  The pair-planar
// mode reads fp32 images; the column-blocked mode reads float2 or half2.
template <class C, int kIn>
thff_status encode_conv_input(CUtensorMap* map, const void* in, const thff::FftParams& ex, long long batch) {
  static_assert(kIn != thff::kInPairPlanar || !C::kIsHalf, "the pair-planar mode reads fp32 images");
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  if constexpr (kIn == thff::kInPairPlanar) {
    // x[b][ch][r][n] real; signal c of group g = row r0 + g*C1 + c of images
    // (b, b+1); n = a + NA s.  Shared memory [c][plane][g | a_hi][s][a].
    static_assert(C::NA == 32 || (C::NA == 64 && C::G1 == 1), "pair-planar rows must fill 128-B lines");
    const uint64_t W = C::N, rows = uint64_t(ex.chans) * uint64_t(ex.rows);
    const uint64_t plane = rows * W * 4;  // image b -> b + 1 of the same channel
    if constexpr (C::NA == 32) {        // {a, s, g, plane, row}
      const uint64_t d[5] = {32, uint64_t(C::NS), uint64_t(C::G1), uint64_t(ex.nimg_b), rows};
      const uint64_t st[4] = {128, uint64_t(C::C1) * W * 4, plane, W * 4};
      const uint32_t b[5] = {32, uint32_t(C::NS), uint32_t(C::G1), 2, uint32_t(C::C1)};
      std::memcpy(dims, d, sizeof d); std::memcpy(strides, st, sizeof st); std::memcpy(box, b, sizeof b);
    } else {                            // {a_lo, s, a_hi, plane, row}
      const uint64_t d[5] = {32, uint64_t(C::NS), 2, uint64_t(ex.nimg_b), rows};
      const uint64_t st[4] = {256, 128, plane, W * 4};
      const uint32_t b[5] = {32, uint32_t(C::NS), 2, 2, uint32_t(C::C1)};
      std::memcpy(dims, d, sizeof d); std::memcpy(strides, st, sizeof st); std::memcpy(box, b, sizeof b);
    }
  } else {
    // Column-blocked in[blk][n][c] complex, blk = sig / C1 (C1 signals per
    // block, ex.rows signals per image, blocks consecutive across images);
    // n = a + NA s, a = a_lo + (16 / C1) a_hi: one 128-B line = 16 / C1
    // consecutive n of a block.  Shared memory [a_hi][g][s][line].
    // CPL complex values per 128-B line; elements of E = 2 CPL reals
    constexpr uint64_t CSZ = 2 * C::ESZ, CPL = 128 / CSZ;
    static_assert(CPL % C::C1 == 0, "C1 divides a 128-B line");
    constexpr uint64_t ALO = CPL / C::C1, AHI = C::NA / ALO;
    const uint64_t blk = uint64_t(C::N) * C::C1 * CSZ, tiles = uint64_t(batch) / C::T;
    const uint64_t d[5] = {2 * CPL, uint64_t(C::NS), uint64_t(C::G1), AHI, tiles};
    const uint64_t st[4] = {uint64_t(C::NA) * C::C1 * CSZ, blk, 128, uint64_t(C::G1) * blk};
    const uint32_t b[5] = {uint32_t(2 * CPL), uint32_t(C::NS), uint32_t(C::G1), uint32_t(AHI), 1};
    std::memcpy(dims, d, sizeof d); std::memcpy(strides, st, sizeof st); std::memcpy(box, b, sizeof b);
  }
  return encode(map, C::kIsHalf ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, in, dims,
                strides, box, C::kIsHalf ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

template <bool kHalf, int kN, int kEpi = thff::kEpiNatural, int kIn = thff::kInNatural, int kVar = 0,
          int kHS = 0, bool kOutHalf = kHalf>
thff_status launch_fft2(DeviceState& st, const Consts& c, const void* in, void* out, long long batch,
                        cudaStream_t stream, const thff::FftParams* extra = nullptr) {
  using C = thff::Fft2Cfg<kHalf, kN, kVar, kHS>;
  const long long num_tiles = (batch + C::T - 1) / C::T;
  const long long full_tiles = batch / C::T;
  const bool use_tma = kIn != thff::kInNatural || aligned16(in);
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if constexpr (kIn != thff::kInNatural) {
    if (!extra || extra->rows % C::T != 0 || batch % extra->rows != 0 || !aligned16(in))
      return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] conv2d pass: tiles must not straddle images");
    thff_status s = encode_conv_input<C, kIn>(&map, in, *extra, batch);
    if (s != THFF_OK) return s;
  } else if (use_tma) {
    static_assert(C::kNaturalTma, "natural-layout TMA box needs H or G1 trivial");
    const uint64_t sig_bytes = uint64_t(C::N) * 2 * C::ESZ;
    uint64_t dims[5], strides[4];
    uint32_t box[5];
    dims[0] = C::E;            box[0] = C::E;
    dims[1] = C::NS;           box[1] = C::NS;     strides[0] = uint64_t(2 * C::NA * C::ESZ);
    if (C::H > 1) { dims[2] = C::H;  box[2] = C::H;  strides[1] = 128; }
    else if (C::G1 > 1) { dims[2] = C::G1; box[2] = C::G1; strides[1] = uint64_t(C::C1) * sig_bytes; }
    else { dims[2] = 1; box[2] = 1; strides[1] = 128; }
    dims[3] = C::C1;           box[3] = C::C1;     strides[2] = sig_bytes;
    dims[4] = uint64_t(full_tiles > 0 ? full_tiles : 1); box[4] = 1;
    strides[3] = uint64_t(C::T) * sig_bytes;
    thff_status s = encode(&map, kHalf ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5,
                           in, dims, strides, box,
                           kHalf ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (s != THFF_OK) return s;
  }
  if constexpr (kEpi != thff::kEpiNatural) {
    if (!extra || extra->rows % C::T != 0 || extra->ppc < 1)
      return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] conv2d pass: tiles must not straddle images");
  }
  thff::FftParams p;
  std::memset(&p, 0, sizeof(p));
  if (extra) p = *extra;
  p.in = in; p.out = out; p.a1 = c.a1; p.a2 = c.a2; p.tw = reinterpret_cast<const float2*>(c.tw);
  p.batch = batch; p.use_tma = use_tma ? 1 : 0; p.err = stream_err(st, stream);
  if (!extra) { p.rows = 1; p.chans = 1; p.ppc = 1; }
  // spectrum staging (kEpiMulNatural with slots): the spectra as 128-B lines,
  // one box = the T*N complex values of one tile
  CUtensorMap map_spec;
  std::memset(&map_spec, 0, sizeof(map_spec));
  if constexpr (kEpi == thff::kEpiMulNatural && kHS > 0) {
    static_assert((C::T * C::N) % 16 == 0 && C::T * C::N / 16 <= 256, "spectrum box");
    const uint64_t lines = uint64_t(p.chans) * uint64_t(p.rows) * C::N / 16;
    const uint64_t dims[3] = {32, lines, 1};
    const uint64_t strides[2] = {128, lines * 128};
    const uint32_t box[3] = {32, uint32_t(C::T * C::N / 16), 1};
    if (!p.spec || !aligned16(p.spec)) return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] conv2d pass: spectrum");
    thff_status s = encode(&map_spec, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.spec, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != THFF_OK) return s;
  }
  auto kernel = thff::fft2_kernel<C, kEpi, kIn, kOutHalf>;
  thff_status s = set_smem_attr(st, kernel, int(C::SMEM_BYTES));
  if (s != THFF_OK) return s;
  const long long grid = num_tiles < st.sms ? num_tiles : st.sms;
  kernel<<<unsigned(grid), C::kThreads, C::SMEM_BYTES, stream>>>(map, map_spec, p);
  THFF_CUDA(launched(), "ThunderFFT_global launch");
  return THFF_OK;
}

template <bool kHalf>
thff_status launch_dft1(DeviceState& st, const Consts& c, const void* in, void* out, long long batch,
                        cudaStream_t stream) {
  using C = thff::Dft1Cfg<kHalf>;
  const long long num_tiles = (batch + C::T - 1) / C::T;
  const bool use_tma = aligned16(in);
  const bool tma_store = aligned16(out);
  CUtensorMap map_in, map_out;
  std::memset(&map_in, 0, sizeof(map_in));
  std::memset(&map_out, 0, sizeof(map_out));
  const uint64_t dims[3] = {uint64_t(C::E), uint64_t(batch), uint64_t(C::KATOMS)};
  const uint64_t strides[2] = {uint64_t(2 * C::N * C::ESZ), 128};
  const uint32_t box[3] = {uint32_t(C::E), uint32_t(C::T), uint32_t(C::KATOMS)};
  // float2 stores one 32-column chunk (one K atom) per TMA store, half2 the tile
  const uint32_t box_out[3] = {uint32_t(C::E), uint32_t(C::T), kHalf ? uint32_t(C::KATOMS) : 1u};
  const CUtensorMapDataType dt = kHalf ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  thff_status s;
  if (use_tma && (s = encode(&map_in, dt, 3, in, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) != THFF_OK) return s;
  if (tma_store && (s = encode(&map_out, dt, 3, out, dims, strides, box_out, CU_TENSOR_MAP_SWIZZLE_128B)) != THFF_OK)
    return s;
  thff::FftParams p;
  p.in = in; p.out = out; p.a1 = c.a1; p.a2 = nullptr; p.tw = nullptr;
  p.batch = batch; p.use_tma = use_tma ? 1 : 0; p.err = stream_err(st, stream);
  auto kernel = thff::dft1_kernel<C>;
  if ((s = set_smem_attr(st, kernel, int(C::SMEM_BYTES))) != THFF_OK) return s;
  const long long grid = num_tiles < st.sms ? num_tiles : st.sms;
  kernel<<<unsigned(grid), C::kThreads, C::SMEM_BYTES, stream>>>(map_in, map_out, p, tma_store ? 1 : 0);
  THFF_CUDA(launched(), "ThunderFFT_global launch");
  return THFF_OK;
}

// Tiled (overlap-save) convolution: the N = 64 kernel in window mode with
// the filter's circulant operator as its B matrix.
template <bool kHalf>
thff_status launch_conv1d_tiled(DeviceState& st, const void* op, const void* in, void* out, long long nseq,
                                long long in_len, int f, cudaStream_t stream) {
  using C = thff::Dft1Cfg<kHalf>;
  const long long out_len = in_len - f + 1, stride = C::N - f + 1;
  const long long wps = (out_len + stride - 1) / stride;   // windows per sequence
  const long long windows = wps * nseq;
  const long long num_tiles = (windows + C::T - 1) / C::T;
  CUtensorMap map_in, map_out;
  std::memset(&map_in, 0, sizeof(map_in));
  std::memset(&map_out, 0, sizeof(map_out));
  thff::FftParams p;
  std::memset(&p, 0, sizeof(p));
  const uint64_t csz = 2 * C::ESZ;   // bytes per complex element
  // Fast tiles (128 windows inside one sequence): a TMA box in when the
  // window stride and the sequence stride are 16-byte multiples, one bulk copy
  // of the contiguous outputs out when the output side is aligned as well.
  const bool tma_in = aligned16(in) && (stride * csz) % 16 == 0 && (in_len * csz) % 16 == 0;
  const bool bulk_out = aligned16(out) && (stride * csz) % 16 == 0 && (nseq == 1 || (out_len * csz) % 16 == 0);
  thff_status s;
  if (tma_in) {
    const uint64_t dims[4] = {uint64_t(C::E), uint64_t(wps), uint64_t(C::KATOMS), uint64_t(nseq)};
    const uint64_t strides[3] = {uint64_t(stride) * csz, 128, uint64_t(in_len) * csz};
    const uint32_t box[4] = {uint32_t(C::E), uint32_t(C::T), uint32_t(C::KATOMS), 1};
    if ((s = encode(&map_in, kHalf ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, in, dims,
                    strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) != THFF_OK)
      return s;
  }
  p.in = in; p.out = out; p.a1 = op; p.batch = windows; p.use_tma = tma_in ? 1 : 0; p.err = stream_err(st, stream);
  p.win_stride = int(stride); p.win_per_sig = wps; p.in_len = in_len; p.out_len = out_len;
  p.win_tmax = in_len >= C::N ? (in_len - C::N) / stride : -1;
  auto kernel = thff::dft1_kernel<C, true>;
  if ((s = set_smem_attr(st, kernel, int(C::SMEM_BYTES))) != THFF_OK) return s;
  const long long grid = num_tiles < st.sms ? num_tiles : st.sms;
  kernel<<<unsigned(grid), C::kThreads, C::SMEM_BYTES, stream>>>(map_in, map_out, p, bulk_out ? 1 : 0);
  THFF_CUDA(launched(), "tiled conv1d launch");
  return THFF_OK;
}

thff_status dispatch_c2c(DeviceState& st, const Consts& c, int dtype, int n, const void* in, void* out,
                         long long batch, cudaStream_t stream) {
  const bool half = dtype == THFF_F16;
  switch (n) {
    case 64: return half ? launch_dft1<true>(st, c, in, out, batch, stream) : launch_dft1<false>(st, c, in, out, batch, stream);
    case 128: return half ? launch_fft2<true, 128>(st, c, in, out, batch, stream) : launch_fft2<false, 128>(st, c, in, out, batch, stream);
    case 256: return half ? launch_fft2<true, 256>(st, c, in, out, batch, stream) : launch_fft2<false, 256>(st, c, in, out, batch, stream);
    case 512: return half ? launch_fft2<true, 512>(st, c, in, out, batch, stream) : launch_fft2<false, 512>(st, c, in, out, batch, stream);
    case 1024: return half ? launch_fft2<true, 1024>(st, c, in, out, batch, stream) : launch_fft2<false, 1024>(st, c, in, out, batch, stream);
    case 2048: return half ? launch_fft2<true, 2048>(st, c, in, out, batch, stream) : launch_fft2<false, 2048>(st, c, in, out, batch, stream);
    case 4096: return half ? launch_fft2<true, 4096>(st, c, in, out, batch, stream) : launch_fft2<false, 4096>(st, c, in, out, batch, stream);
  }
  return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] unsupported FFT length");
}

template <int kN, bool kMixed>
thff_status launch_conv1d(DeviceState& st, const Consts& c, int lin, const void* x, const void* spec, void* y,
                          long long batch, cudaStream_t stream) {
  using C = thff::Conv1dCfg<kN, kMixed>;
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  const uint64_t dims[4] = {uint64_t(C::E), uint64_t(lin / C::L), uint64_t(C::H), uint64_t(batch)};
  const uint64_t strides[3] = {uint64_t(C::L) * 4, 128, uint64_t(lin) * 4};
  const uint32_t box[4] = {uint32_t(C::E), uint32_t(C::L), uint32_t(C::H), uint32_t(2 * C::TC)};
  thff_status s = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  if (s != THFF_OK) return s;
  thff::Conv1dParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = static_cast<const float*>(x);
  p.y = static_cast<float*>(y);
  p.a = c.a1;
  p.a16 = c.a2;
  p.tw = reinterpret_cast<const float2*>(c.tw);
  p.spec = static_cast<const float2*>(spec);
  p.batch = batch;
  p.lin = lin;
  p.rows_valid = lin / C::L;
  p.err = stream_err(st, stream);
  auto kernel = thff::conv1d_kernel<C>;
  if ((s = set_smem_attr(st, kernel, int(C::SMEM_BYTES))) != THFF_OK) return s;
  const long long tiles = (batch + 2 * C::TC - 1) / (2 * C::TC);
  const long long grid = tiles < st.sms ? tiles : st.sms;
  kernel<<<unsigned(grid), C::kThreads, C::SMEM_BYTES, stream>>>(map, p);
  THFF_CUDA(launched(), "conv1d launch");
  return THFF_OK;
}

// Arithmetic of the conv1d stages 2-4: THFF_CONV_MIXED (FP16 operands with
// per-tile power-of-two range scaling) or THFF_CONV_TF32.
std::atomic<int> g_conv1d_arith{THFF_CONV_MIXED};
std::atomic<int> g_conv2d_arith{THFF_CONV_MIXED};

// Stage matrix + twiddles of the conv kernel: the forward DFT matrix of
// length L = sqrt(n) (one group) and the forward twiddles of length n.
thff_status get_conv_consts(DeviceState& st, int n, const Consts** out) {
  const int key = 15 * 8192 + n;  // outside the range of consts_key
  auto it = st.consts.find(key);
  if (it == st.consts.end()) {
    Consts c;
    const int L = n == 4096 ? 64 : 32;
    thff_status s = upload(build_stage_matrix(L, 1, -1, false), &c.a1);
    if (s != THFF_OK) return s;
    if ((s = upload(build_stage_matrix(L, 1, -1, true), &c.a2)) != THFF_OK) return s;   // FP16 image
    std::vector<uint8_t> tw(size_t(n) * 8);
    for (int k = 0; k < n; ++k) {
      const double th = -kTau * double(k) / double(n);
      const float v[2] = {float(std::cos(th)), float(std::sin(th))};
      std::memcpy(tw.data() + size_t(k) * 8, v, 8);
    }
    if ((s = upload(tw, &c.tw)) != THFF_OK) return s;
    it = st.consts.emplace(key, c).first;
  }
  *out = &it->second;
  return THFF_OK;
}

// Signals per stage-1 column group (C1) of the length-n FFT (float2 or half2
// storage): the block width of the column-blocked layout that pass reads.
int conv2d_c1(int n, bool half = false) {
  switch (n) {
    case 128: return half ? thff::Fft2Cfg<true, 128>::C1 : thff::Fft2Cfg<false, 128>::C1;
    case 256: return half ? thff::Fft2Cfg<true, 256>::C1 : thff::Fft2Cfg<false, 256>::C1;
    case 512: return half ? thff::Fft2Cfg<true, 512>::C1 : thff::Fft2Cfg<false, 512>::C1;
    case 1024: return half ? thff::Fft2Cfg<true, 1024>::C1 : thff::Fft2Cfg<false, 1024>::C1;
    case 2048: return half ? thff::Fft2Cfg<true, 2048>::C1 : thff::Fft2Cfg<false, 2048>::C1;
    default: return half ? thff::Fft2Cfg<true, 4096>::C1 : thff::Fft2Cfg<false, 4096>::C1;
  }
}

// One pass of the 2-D convolution pipeline: length-n C2C transform of
// `batch` signals with input mode kIn and stage-2 epilogue mode kEpi, in
// float2 (kHalf false) or half2 storage; kOutHalf: half2 outputs.
// Spectrum staging slots of the length-n multiply pass: two when they fit
// beside a 2-tile input ring, else one (computed without instantiating the
// configuration that would not fit).
template <bool kHalf, int kN>
constexpr int conv2d_hslots() {
  using B = thff::Fft2Cfg<kHalf, kN>;
  // the producer loads a tile's spectrum right after its input, so the
  // spectrum slots bound how far it runs ahead: as many as fit, up to 4
  for (int hs = 4; hs > 1; --hs)
    if (B::OFF_IN + (2 + 2) * B::TILE_BYTES + hs * (B::T * B::N * 8) + 1024 + 512 <= 232448u) return hs;
  return 1;
}

template <int kEpi, int kIn, bool kHalf = false, bool kOutHalf = kHalf>
thff_status conv2d_pass(DeviceState& st, const Consts& c, int n, const void* in, void* out, long long batch,
                        const thff::FftParams& extra, cudaStream_t cs) {
  // the pair-planar pass uses the float NA = 32 shape variant where one
  // exists; the spectrum-multiply pass stages the spectrum tiles in shared
  // memory
  constexpr int kV = (kIn == thff::kInPairPlanar) ? 1 : 0;
  constexpr bool kMul = kEpi == thff::kEpiMulNatural;
  switch (n) {
    case 128: return launch_fft2<kHalf, 128, kEpi, kIn, kV, kMul ? conv2d_hslots<kHalf, 128>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
    case 256: return launch_fft2<kHalf, 256, kEpi, kIn, kV, kMul ? conv2d_hslots<kHalf, 256>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
    case 512: return launch_fft2<kHalf, 512, kEpi, kIn, kV, kMul ? conv2d_hslots<kHalf, 512>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
    case 1024: return launch_fft2<kHalf, 1024, kEpi, kIn, 0, kMul ? conv2d_hslots<kHalf, 1024>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
    case 2048: return launch_fft2<kHalf, 2048, kEpi, kIn, 0, kMul ? conv2d_hslots<kHalf, 2048>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
    case 4096: return launch_fft2<kHalf, 4096, kEpi, kIn, 0, kMul ? conv2d_hslots<kHalf, 4096>() : 0, kOutHalf>(st, c, in, out, batch, cs, &extra);
  }
  return fail(THFF_INVALID_ARGUMENT, "conv2d: image sides must be in {128, ..., 4096}");
}

int ilog2(int v) { int l = 0; while ((1 << l) < v) ++l; return l; }

// Constants of the fused column pass (conv2d_cols_kernel, half2 storage: the
// mixed-arithmetic pipeline) for column length n: the forward stage matrices A1
// (NS, G1 groups) and A2 (NA, G2 groups, K rows rotated as stage 2 writes
// them), A4 = A1 with that rotation (the inverse's second stage), and the
// forward twiddles.  A4 aliases A1 or A2 where they are the same matrix.
int conv2d_cols_key(bool half, int n) { return (half ? 13 : 14) * 8192 + n; }

template <bool kHalf, int kN>
thff_status build_conv2d_cols_consts(Consts* c) {
  using C = thff::Conv2dColCfg<kHalf, kN>;
  thff_status s;
  if ((s = upload(build_stage_matrix(C::NS, C::G1, -1, kHalf), &c->a1)) != THFF_OK) return s;
  if ((s = upload(build_stage_matrix(C::NA, C::G2, -1, kHalf, C::R2), &c->a2)) != THFF_OK) return s;
  if (C::kA4isA1) c->a4 = c->a1;
  else if (C::kA4isA2) c->a4 = c->a2;
  else if ((s = upload(build_stage_matrix(C::NS, C::G1, -1, kHalf, C::R2), &c->a4)) != THFF_OK) return s;
  std::vector<uint8_t> tw(size_t(kN) * 8);
  for (int k = 0; k < kN; ++k) {
    const double th = -kTau * double(k) / double(kN);
    const float v[2] = {float(std::cos(th)), float(std::sin(th))};
    std::memcpy(tw.data() + size_t(k) * 8, v, 8);
  }
  return upload(tw, &c->tw);
}

thff_status get_conv2d_cols_consts(DeviceState& st, bool half, int n, const Consts** out) {
  const int key = conv2d_cols_key(half, n);
  auto it = st.consts.find(key);
  if (it == st.consts.end()) {
    Consts c;
    thff_status s = THFF_INVALID_ARGUMENT;
    switch (n) {
#define THFF_COLS(NN)                                                                                   \
  case NN: s = half ? build_conv2d_cols_consts<true, NN>(&c) : THFF_INVALID_ARGUMENT; break;
      THFF_COLS(128) THFF_COLS(256) THFF_COLS(512) THFF_COLS(1024) THFF_COLS(2048) THFF_COLS(4096)
#undef THFF_COLS
    }
    if (s != THFF_OK) return s;
    it = st.consts.emplace(key, c).first;
  }
  *out = &it->second;
  return THFF_OK;
}

// The fused column pass over `batch` column signals (whole tiles, never
// straddling image pairs): reads the column-blocked layout the row pass
// writes (extra.rows = w column signals per pair), writes the column-blocked
// layout of the last row pass (block width 2^extra.blk_log2).
template <bool kHalf, int kN>
thff_status launch_conv2d_cols(DeviceState& st, const Consts& c, const void* in, void* out, long long batch,
                               cudaStream_t stream, const thff::FftParams& extra) {
  using C = thff::Conv2dColCfg<kHalf, kN>;
  if (extra.rows % C::T != 0 || batch % extra.rows != 0 || !aligned16(in) || !aligned16(out))
    return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] conv2d column pass: tiles must not straddle images");
  CUtensorMap map, map_spec;
  std::memset(&map, 0, sizeof(map));
  std::memset(&map_spec, 0, sizeof(map_spec));
  thff_status s = encode_conv_input<C, thff::kInBlocked>(&map, in, extra, batch);
  if (s != THFF_OK) return s;
  static_assert((C::T * C::N) % 16 == 0 && C::T * C::N / 16 <= 256, "spectrum box");
  const uint64_t lines = uint64_t(extra.chans) * uint64_t(extra.rows) * C::N / 16;
  const uint64_t dims[3] = {32, lines, 1};
  const uint64_t strides[2] = {128, lines * 128};
  const uint32_t box[3] = {32, uint32_t(C::T * C::N / 16), 1};
  if (!extra.spec || !aligned16(extra.spec)) return fail(THFF_INVALID_ARGUMENT, "[ThunderFFT] conv2d pass: spectrum");
  if ((s = encode(&map_spec, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, extra.spec, dims, strides, box,
                  CU_TENSOR_MAP_SWIZZLE_128B)) != THFF_OK)
    return s;
  thff::FftParams p = extra;
  p.in = in; p.out = out; p.a1 = c.a1; p.a2 = c.a2; p.a4 = c.a4;
  p.tw = reinterpret_cast<const float2*>(c.tw);
  p.batch = batch; p.use_tma = 1; p.err = stream_err(st, stream);
  auto kernel = thff::conv2d_cols_kernel<C>;
  if ((s = set_smem_attr(st, kernel, int(C::SMEM_BYTES))) != THFF_OK) return s;
  const long long tiles = batch / C::T;
  const long long grid = tiles < st.sms ? tiles : st.sms;
  kernel<<<unsigned(grid), C::kThreads, C::SMEM_BYTES, stream>>>(map, map_spec, p);
  THFF_CUDA(launched(), "conv2d column pass launch");
  return THFF_OK;
}

template <bool kHalf>
thff_status conv2d_cols(DeviceState& st, const Consts& c, int n, const void* in, void* out, long long batch,
                        const thff::FftParams& extra, cudaStream_t cs) {
  switch (n) {
    case 128: return launch_conv2d_cols<kHalf, 128>(st, c, in, out, batch, cs, extra);
    case 256: return launch_conv2d_cols<kHalf, 256>(st, c, in, out, batch, cs, extra);
    case 512: return launch_conv2d_cols<kHalf, 512>(st, c, in, out, batch, cs, extra);
    case 1024: return launch_conv2d_cols<kHalf, 1024>(st, c, in, out, batch, cs, extra);
    case 2048: return launch_conv2d_cols<kHalf, 2048>(st, c, in, out, batch, cs, extra);
    case 4096: return launch_conv2d_cols<kHalf, 4096>(st, c, in, out, batch, cs, extra);
  }
  return fail(THFF_INVALID_ARGUMENT, "conv2d: image sides must be in {128, ..., 4096}");
}

// The whole 2-D convolution in TF32 (THFF_CONV_TF32, and the
// allocation-free entry point) over image pairs [0, pairs) in chunks of
// `chunk` pairs through the scratch buffers z0, z1 (chunk * h * w complex
// each).  The column FFT, the spectrum product and the column IFFT stay two
// passes here: fused into one kernel (conv2d_cols_kernel) with float2 tiles,
// only one spectrum slot fits beside the operand buffers, and config 5
// measured 2.29 ms for the fused pass against 1.08 + 0.88 ms for the two.
//   P1 rows    (length w): real image pair -> complex, FFT     -> z0 [pair][k2 / Ch][r][k2 % Ch]
//   P2 columns (length h): FFT, x spectrum                      -> z1 [pair][k2][k1]
//   P3 columns (length h): inverse FFT                          -> z0 [pair][r / Cw][k2][r % Cw]
//   P4 rows    (length w): inverse FFT, Re/Im -> the two images -> y
// Ch, Cw = signals per stage-1 column group of the length-h, length-w
// transforms: P2 and P4 read their signals (columns of the previous pass's
// output) as whole 128-B lines of the column-blocked layout, and every pass
// stores rows of at least Cb consecutive complex values.  consts(n, fwd,
// var, &c) finds the FFT constants of each pass.
template <class Lookup>
thff_status conv2d_run(DeviceState& st, Lookup&& consts, long long nimg_b, int chans, int h, int w,
                       const void* d_x, const void* d_spectra, void* d_y, float2* z0, float2* z1, long long chunk,
                       cudaStream_t cs) {
  const Consts *row_f, *col_f, *col_i, *row_i;
  thff_status s;
  if ((s = consts(w, true, has_variant1(THFF_F32, w) ? 1 : 0, &row_f)) != THFF_OK ||
      (s = consts(h, true, 0, &col_f)) != THFF_OK || (s = consts(h, false, 0, &col_i)) != THFF_OK ||
      (s = consts(w, false, 0, &row_i)) != THFF_OK)
    return s;
  const long long ppc = (nimg_b + 1) / 2, pairs = ppc * chans;
  thff::FftParams ex;
  std::memset(&ex, 0, sizeof(ex));
  ex.chans = chans; ex.nimg_b = nimg_b; ex.ppc = ppc; ex.spec = static_cast<const float2*>(d_spectra);
  for (long long p0 = 0; p0 < pairs; p0 += chunk) {
    const long long np = (pairs - p0 < chunk) ? pairs - p0 : chunk;
    ex.pair0 = p0;
    ex.rows = h;                     // P1: h row signals per image
    ex.blk_log2 = ilog2(conv2d_c1(h));
    if ((s = conv2d_pass<thff::kEpiBlocked, thff::kInPairPlanar>(st, *row_f, w, d_x, z0, np * h, ex, cs)) != THFF_OK)
      return s;
    ex.rows = w;                     // P2, P3: w column signals per image
    if ((s = conv2d_pass<thff::kEpiMulNatural, thff::kInBlocked>(st, *col_f, h, z0, z1, np * w, ex, cs)) != THFF_OK)
      return s;
    ex.blk_log2 = ilog2(conv2d_c1(w));
    if ((s = conv2d_pass<thff::kEpiBlocked, thff::kInNatural>(st, *col_i, h, z1, z0, np * w, ex, cs)) != THFF_OK)
      return s;
    ex.rows = h;                     // P4: h row signals per image
    if ((s = conv2d_pass<thff::kEpiUnpackPair, thff::kInBlocked>(st, *row_i, w, z0, d_y, np * h, ex, cs)) != THFF_OK)
      return s;
  }
  return THFF_OK;
}

// Mixed-arithmetic form of conv2d_run (THFF_CONV_MIXED): the intermediates
// are half2.  P1 reads the fp32 images in TF32 and stores half2; P2 and P3
// are FP16 passes with FP32 accumulation.  Power-of-two exponents
// (conv2d_kernels.cuh) keep every half2 intermediate at or below 2^9 for any
// finite input, and P3 undoes them.  Scratch: z0, z1 (chunk * h * w half2
// each), e (2 + chunk ints), amax (one word).  consts_f finds the float
// constants of P1, consts_h the half ones of P3, cols_h those of P2.
template <class LookupF, class LookupH, class LookupCols>
thff_status conv2d_run_h(DeviceState& st, LookupF&& consts_f, LookupH&& consts_h, LookupCols&& cols_h,
                         long long nimg_b, int chans, int h, int w, const void* d_x, const void* d_spectra, void* d_y,
                         void* z0, void* z1, int* e, unsigned* amax, long long chunk, cudaStream_t cs) {
  const Consts *row_f, *col, *row_i;
  thff_status s;
  if ((s = consts_f(w, true, has_variant1(THFF_F32, w) ? 1 : 0, &row_f)) != THFF_OK ||
      (s = cols_h(h, &col)) != THFF_OK || (s = consts_h(w, false, &row_i)) != THFF_OK)
    return s;
  const long long ppc = (nimg_b + 1) / 2, pairs = ppc * chans;
  // call exponents e2, e3 from the spectra's largest part
  THFF_CUDA(cudaMemsetAsync(amax, 0, sizeof(unsigned), cs), "conv2d range word");
  thff::conv2d_spectra_absmax_kernel<<<unsigned(4 * st.sms), 256, 0, cs>>>(static_cast<const float*>(d_spectra),
                                                                          2LL * chans * h * w, amax);
  THFF_CUDA(launched(), "conv2d range launch");
  thff::conv2d_call_exp_kernel<<<1, 1, 0, cs>>>(amax, h, e);
  THFF_CUDA(launched(), "conv2d range launch");
  thff::FftParams ex;
  std::memset(&ex, 0, sizeof(ex));
  ex.chans = chans; ex.nimg_b = nimg_b; ex.ppc = ppc; ex.spec = static_cast<const float2*>(d_spectra);
  ex.conv_exp = e;
  for (long long p0 = 0; p0 < pairs; p0 += chunk) {
    const long long np = (pairs - p0 < chunk) ? pairs - p0 : chunk;
    ex.pair0 = p0;
    thff::conv2d_pair_exp_kernel<<<unsigned(np), 256, 0, cs>>>(static_cast<const float*>(d_x), nimg_b, chans, ppc,
                                                                p0, h, w, e + 2);
    THFF_CUDA(launched(), "conv2d range launch");
    ex.rows = h;                     // P1: h row signals per image
    ex.blk_log2 = ilog2(conv2d_c1(h, true));
    ex.conv_pass = 1;
    if ((s = conv2d_pass<thff::kEpiBlocked, thff::kInPairPlanar, false, true>(st, *row_f, w, d_x, z0, np * h, ex,
                                                                               cs)) != THFF_OK)
      return s;
    ex.rows = w;                     // P2: w column signals per image
    ex.blk_log2 = ilog2(conv2d_c1(w, true));
    ex.conv_pass = 2;
    if ((s = conv2d_cols<true>(st, *col, h, z0, z1, np * w, ex, cs)) != THFF_OK) return s;
    ex.rows = h;                     // P3: h row signals per image
    ex.conv_pass = 4;
    if ((s = conv2d_pass<thff::kEpiUnpackPair, thff::kInBlocked, true>(st, *row_i, w, z1, d_y, np * h, ex, cs)) !=
        THFF_OK)
      return s;
  }
  return THFF_OK;
}

bool conv2d_side_ok(int v) { return v == 128 || v == 256 || v == 512 || v == 1024 || v == 2048 || v == 4096; }

// ---------------------------------------------------------------------------
// Allocation-free 2-D convolution (thff_conv2d_noalloc)
//
// Some callers cannot call cudaMalloc at the point where they run the
// convolution: plugins and real-time pipelines whose host application owns
// all device memory and forbids allocation on the hot path,
// and frameworks whose pooling allocator must account for every byte.  For
// them the scratch of the 2-D convolution lives in this fixed device array
// instead of a caller workspace.  Every GPU that loads the library holds it
// (kNoAllocScratchBytes) until the process exits.
// ---------------------------------------------------------------------------
// 16 MiB: one pass holds scratch / per_pair image pairs, per_pair = 2*h*w*8
// bytes (the two float2 scratch images z0, z1 of one pair).
constexpr long long kNoAllocScratchBytes = 16LL << 20;
static __device__ __align__(256) unsigned char g_conv2d_scratch[kNoAllocScratchBytes];

// Look up FFT constants without building them (building would allocate).
const Consts* find_consts(DeviceState& st, int dtype, int n, bool fwd, int var = 0) {
  auto it = st.consts.find(consts_key(dtype, n, fwd, var));
  return it == st.consts.end() ? nullptr : &it->second;
}

// Synchronizes `stream` and reads (and clears) its error word.  Another
// stream's word is never touched.
thff_status read_device_error(DeviceState& st, cudaStream_t stream) {
  if (!t_err_host) THFF_CUDA(cudaMallocHost(&t_err_host, sizeof(uint32_t)), "cudaMallocHost(error word)");
  *t_err_host = 0;
  uint32_t* word = stream_err(st, stream);
  THFF_CUDA(cudaMemcpyAsync(t_err_host, word, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream),
            "cudaMemcpyAsync(error word)");
  THFF_CUDA(cudaStreamSynchronize(stream), "ThunderFFT_global synchronize");
  if (*t_err_host != 0) {
    const uint32_t code = *t_err_host;
    cudaMemsetAsync(word, 0, sizeof(uint32_t), stream);
    cudaStreamSynchronize(stream);
    return fail(THFF_DEVICE_TIMEOUT, "[ThunderFFT] device pipeline wait timed out (code " + std::to_string(code) + ")");
  }
  return THFF_OK;
}

}  // namespace

extern "C" {

const char* thff_version(void) { return "thunderfft_b200 0.1 (sm_100a tcgen05/TMA)"; }

const char* thff_last_error(void) { return g_last_error.c_str(); }

unsigned long long thff_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

thff_status thff_initialize(int dtype, int n) {
  if (!valid_dtype(dtype)) return fail(THFF_INVALID_ARGUMENT, "ThunderFFTInitialize<T>: supported T are float and half only");
  if (!valid_n(n)) return fail(THFF_INVALID_ARGUMENT, "ThunderFFTInitialize<T>: unsupported FFT size");
  std::lock_guard<std::mutex> lock(g_mutex);
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  RefCache& rc = st->ref[dtype];
  if (!(rc.dW && rc.n == n)) {
    if (rc.dW) {
      rc.n = 0;
      THFF_CUDA(cudaFree(rc.dW), "cudaFree cached twiddle (initialize)");
      rc.dW = nullptr;
    }
    // W[k] = (cos 2 pi k / N, sin 2 pi k / N) (positive angle, as the
    // reference's preprocess_W_*: thunderfft_impl_twiddle.cuh:76-114).
    const bool half = dtype == THFF_F16;
    std::vector<uint8_t> h(size_t(n) * (half ? 4 : 8));
    for (int k = 0; k < n; ++k) {
      const double th = kTau * double(k) / double(n);
      if (half) {
        const __half2 v = __halves2half2(__float2half_rn(float(std::cos(th))), __float2half_rn(float(std::sin(th))));
        std::memcpy(h.data() + size_t(k) * 4, &v, 4);
      } else {
        const float v[2] = {float(std::cos(th)), float(std::sin(th))};
        std::memcpy(h.data() + size_t(k) * 8, v, 8);
      }
    }
    void* d = nullptr;
    if ((s = upload(h, &d)) != THFF_OK) return s;
    rc.dW = d;
    rc.n = n;
  }
  // FFT constants for both directions of this length.
  const Consts* c;
  if ((s = get_consts(*st, dtype, n, true, &c)) != THFF_OK) return s;
  if ((s = get_consts(*st, dtype, n, false, &c)) != THFF_OK) return s;
  if (has_variant1(dtype, n) && (s = get_consts(*st, dtype, n, true, &c, 1)) != THFF_OK) return s;
  return THFF_OK;
}

thff_status thff_finalize(int dtype) {
  if (!valid_dtype(dtype)) return fail(THFF_INVALID_ARGUMENT, "ThunderFFTFinalize<T>: supported T are float and half only");
  std::lock_guard<std::mutex> lock(g_mutex);
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  auto it = g_dev.find(dev);
  if (it == g_dev.end()) return THFF_OK;
  RefCache& rc = it->second.ref[dtype];
  rc.n = 0;
  if (rc.dW) {
    void* d = rc.dW;
    rc.dW = nullptr;
    THFF_CUDA(cudaFree(d), "cudaFree cached twiddle (finalize)");
  }
  return THFF_OK;
}

thff_status thff_twiddle_table(int dtype, const void** table, int* n) {
  if (!valid_dtype(dtype) || !table || !n) return fail(THFF_INVALID_ARGUMENT, "thff_twiddle_table: bad arguments");
  std::lock_guard<std::mutex> lock(g_mutex);
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  auto it = g_dev.find(dev);
  *table = (it == g_dev.end()) ? nullptr : it->second.ref[dtype].dW;
  *n = (it == g_dev.end()) ? 0 : it->second.ref[dtype].n;
  return THFF_OK;
}

thff_status thff_c2c_async(int dtype, int n, int forward, const void* d_input, void* d_output,
                           long long batch, void* stream) {
  if (!valid_dtype(dtype)) return fail(THFF_INVALID_ARGUMENT, "ThunderFFT_global supports float and half only");
  if (!valid_n(n)) return fail(THFF_INVALID_ARGUMENT, "Unsupported ThunderFFT length");
  if (batch < 0) return fail(THFF_INVALID_ARGUMENT, "ThunderFFT batch must be nonnegative");
  if (batch == 0) return THFF_OK;
  if (!d_input || !d_output || d_input == d_output)
    return fail(THFF_INVALID_ARGUMENT, "ThunderFFT requires separate non-null input/output buffers");
  const size_t esz = dtype == THFF_F16 ? 4 : 8;
  const uintptr_t a = reinterpret_cast<uintptr_t>(d_input), b = reinterpret_cast<uintptr_t>(d_output);
  const uintptr_t bytes = uintptr_t(batch) * uintptr_t(n) * esz;
  if (a < b + bytes && b < a + bytes)
    return fail(THFF_INVALID_ARGUMENT, "ThunderFFT requires separate non-null input/output buffers");
  if ((a % esz) || (b % esz)) return fail(THFF_INVALID_ARGUMENT, "ThunderFFT buffers must be aligned to the complex element size");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  const Consts* c;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
    if ((s = get_consts(*st, dtype, n, forward != 0, &c)) != THFF_OK) return s;
  }
  return dispatch_c2c(*st, *c, dtype, n, d_input, d_output, batch, reinterpret_cast<cudaStream_t>(stream));
}

thff_status thff_sync_check(void* stream) {
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  }
  return read_device_error(*st, reinterpret_cast<cudaStream_t>(stream));
}

thff_status thff_global(int dtype, int n, int forward, const void* d_input, void* d_output, int batch,
                        void* stream) {
  if (batch < 0) return fail(THFF_INVALID_ARGUMENT, "ThunderFFT batch must be nonnegative");
  if (batch == 0) return THFF_OK;
  thff_status s = thff_c2c_async(dtype, n, forward, d_input, d_output, batch, stream);
  if (s != THFF_OK) return s;
  return thff_sync_check(stream);
}

thff_status thff_selftest_wait_timeout(int limit_us, void* stream) {
  if (limit_us <= 0 || limit_us > 1000000) return fail(THFF_INVALID_ARGUMENT, "selftest: limit must be in (0, 1e6] us");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  thff::wait_timeout_selftest_kernel<<<1, 32, 0, cs>>>(stream_err(*st, cs), 1000ull * (unsigned long long)limit_us);
  THFF_CUDA(launched(), "selftest launch");
  return read_device_error(*st, cs);
}

thff_status thff_test_inject_cuda_error(int cuda_error, int skip) {
  if (cuda_error < 0 || skip < 0) return fail(THFF_INVALID_ARGUMENT, "inject: error code and skip must be >= 0");
  g_inject_error = cuda_error;
  g_inject_skip = cuda_error == 0 ? 0 : skip;
  return THFF_OK;
}

long long thff_conv1d_spectrum_bytes(int dtype, int n) {
  if (dtype != THFF_F32 || (n != 1024 && n != 4096)) return -1;
  return (long long)n * 8;
}

thff_status thff_conv1d_filter_spectrum(int dtype, int n, const float* d_filter, int taps, void* d_spectrum,
                                        void* stream) {
  if (dtype != THFF_F32) return fail(THFF_INVALID_ARGUMENT, "conv1d: float storage only");
  if (n != 1024 && n != 4096) return fail(THFF_INVALID_ARGUMENT, "conv1d: n must be 1024 or 4096");
  if (taps < 1 || taps > n) return fail(THFF_INVALID_ARGUMENT, "conv1d: taps must be in [1, n]");
  if (!d_filter || !d_spectrum) return fail(THFF_INVALID_ARGUMENT, "conv1d: null filter or spectrum");
  thff::conv1d_spectrum_kernel<<<(n + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_filter, taps, n, static_cast<float2*>(d_spectrum));
  THFF_CUDA(launched(), "conv1d spectrum launch");
  return THFF_OK;
}

thff_status thff_conv1d_async(int dtype, int n, int lin, const void* d_x, const void* d_spectrum, void* d_y,
                              long long batch, void* stream) {
  if (dtype != THFF_F32) return fail(THFF_INVALID_ARGUMENT, "conv1d: float storage only");
  if (n != 1024 && n != 4096) return fail(THFF_INVALID_ARGUMENT, "conv1d: n must be 1024 or 4096");
  const int L = n == 4096 ? 64 : 32;
  if (lin <= 0 || lin > n || lin % L != 0)
    return fail(THFF_INVALID_ARGUMENT, "conv1d: input length must be a positive multiple of sqrt(n), <= n");
  if (batch < 0) return fail(THFF_INVALID_ARGUMENT, "conv1d: batch must be nonnegative");
  if (batch == 0) return THFF_OK;
  if (!d_x || !d_spectrum || !d_y) return fail(THFF_INVALID_ARGUMENT, "conv1d: null pointer");
  if (!aligned16(d_x) || !aligned16(d_spectrum) || (reinterpret_cast<uintptr_t>(d_y) & 7u))
    return fail(THFF_INVALID_ARGUMENT, "conv1d: x and spectrum must be 16-byte aligned, y 8-byte aligned");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  const Consts* c;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
    if ((s = get_conv_consts(*st, n, &c)) != THFF_OK) return s;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (g_conv1d_arith.load() == THFF_CONV_MIXED)
    return n == 4096 ? launch_conv1d<4096, true>(*st, *c, lin, d_x, d_spectrum, d_y, batch, cs)
                     : launch_conv1d<1024, true>(*st, *c, lin, d_x, d_spectrum, d_y, batch, cs);
  return n == 4096 ? launch_conv1d<4096, false>(*st, *c, lin, d_x, d_spectrum, d_y, batch, cs)
                   : launch_conv1d<1024, false>(*st, *c, lin, d_x, d_spectrum, d_y, batch, cs);
}

long long thff_conv1d_tiled_operator_bytes(int dtype) {
  if (!valid_dtype(dtype)) return -1;
  return 128LL * 128LL * (dtype == THFF_F16 ? 2 : 4);
}

thff_status thff_conv1d_tiled_operator(int dtype, const void* d_filter, int f, void* d_operator, void* stream) {
  if (!valid_dtype(dtype)) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: dtype must be THFF_F32 or THFF_F16");
  if (f < 1 || f > 64) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: filter length must be in [1, 64]");
  if (!d_filter || !d_operator) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: null pointer");
  if (!aligned16(d_operator) || (reinterpret_cast<uintptr_t>(d_filter) & 7u))
    return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: operator must be 16-byte aligned, filter 8-byte aligned");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceState* st;
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const int total = 128 * 128;
  if (dtype == THFF_F16)
    thff::conv1d_tiled_operator_kernel<true><<<(total + 255) / 256, 256, 0, cs>>>(
        static_cast<const float2*>(d_filter), f, static_cast<uint8_t*>(d_operator));
  else
    thff::conv1d_tiled_operator_kernel<false><<<(total + 255) / 256, 256, 0, cs>>>(
        static_cast<const float2*>(d_filter), f, static_cast<uint8_t*>(d_operator));
  THFF_CUDA(launched(), "tiled conv1d operator launch");
  return THFF_OK;
}

thff_status thff_conv1d_tiled_async(int dtype, long long input_len, int f, const void* d_x, const void* d_operator,
                                    void* d_y, long long batch, void* stream) {
  if (!valid_dtype(dtype)) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: dtype must be THFF_F32 or THFF_F16");
  if (f < 1 || f > 64) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: filter length must be in [1, 64]");
  if (input_len < f) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: input length must be >= filter length");
  if (batch < 0) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: batch must be nonnegative");
  if (batch == 0) return THFF_OK;
  if (!d_x || !d_operator || !d_y) return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: null pointer");
  const uintptr_t esz = dtype == THFF_F16 ? 4 : 8;
  if ((reinterpret_cast<uintptr_t>(d_x) % esz) || (reinterpret_cast<uintptr_t>(d_y) % esz) || !aligned16(d_operator))
    return fail(THFF_INVALID_ARGUMENT, "tiled conv1d: x/y must be element aligned, the operator 16-byte aligned");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  return dtype == THFF_F16 ? launch_conv1d_tiled<true>(*st, d_operator, d_x, d_y, batch, input_len, f, cs)
                           : launch_conv1d_tiled<false>(*st, d_operator, d_x, d_y, batch, input_len, f, cs);
}

thff_status thff_conv1d_tiled(int dtype, long long input_len, int f, const void* d_x, const void* d_operator,
                              void* d_y, long long batch, void* stream) {
  thff_status s = thff_conv1d_tiled_async(dtype, input_len, f, d_x, d_operator, d_y, batch, stream);
  if (s != THFF_OK || batch == 0) return s;
  return thff_sync_check(stream);
}

thff_status thff_conv2d_set_arithmetic(int mode) {
  if (mode != THFF_CONV_MIXED && mode != THFF_CONV_TF32)
    return fail(THFF_INVALID_ARGUMENT, "conv2d: arithmetic must be THFF_CONV_MIXED or THFF_CONV_TF32");
  g_conv2d_arith.store(mode);
  return THFF_OK;
}

thff_status thff_conv1d_set_arithmetic(int mode) {
  if (mode != THFF_CONV_MIXED && mode != THFF_CONV_TF32)
    return fail(THFF_INVALID_ARGUMENT, "conv1d: arithmetic must be THFF_CONV_MIXED or THFF_CONV_TF32");
  g_conv1d_arith.store(mode);
  return THFF_OK;
}

thff_status thff_conv1d(int dtype, int n, int lin, const void* d_x, const void* d_spectrum, void* d_y,
                        long long batch, void* stream) {
  thff_status s = thff_conv1d_async(dtype, n, lin, d_x, d_spectrum, d_y, batch, stream);
  if (s != THFF_OK || batch == 0) return s;
  return thff_sync_check(stream);
}

long long thff_conv2d_workspace_bytes(int dtype, int h, int w, long long pairs) {
  if (dtype != THFF_F32 || !conv2d_side_ok(h) || !conv2d_side_ok(w) || pairs <= 0) return -1;
  return 2LL * pairs * h * w * 8;
}

thff_status thff_conv2d_filter_spectra(int dtype, int h, int w, int chans, int f, const float* d_filters,
                                       void* d_spectra, void* d_workspace, long long workspace_bytes,
                                       void* stream) {
  if (dtype != THFF_F32) return fail(THFF_INVALID_ARGUMENT, "conv2d: float storage only");
  if (!conv2d_side_ok(h) || !conv2d_side_ok(w)) return fail(THFF_INVALID_ARGUMENT, "conv2d: image sides must be in {128, ..., 4096}");
  if (chans <= 0 || f <= 0 || f > h || f > w) return fail(THFF_INVALID_ARGUMENT, "conv2d: need channels > 0 and 0 < filter size <= image side");
  if (!d_filters || !d_spectra || !d_workspace) return fail(THFF_INVALID_ARGUMENT, "conv2d: null pointer");
  const long long need = (long long)chans * f * w * 16;
  if (workspace_bytes < need) return fail(THFF_INVALID_ARGUMENT, "conv2d: filter workspace too small (need channels*f*w*16 bytes)");
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  double2* g = static_cast<double2*>(d_workspace);
  const long long n1 = (long long)chans * f * w, n2 = (long long)chans * h * w;
  thff::conv2d_filter_rows_kernel<<<unsigned((n1 + 255) / 256), 256, 0, cs>>>(d_filters, chans, f, w, g);
  THFF_CUDA(launched(), "conv2d filter spectrum launch");
  thff::conv2d_filter_cols_kernel<<<unsigned((n2 + 255) / 256), 256, 0, cs>>>(g, chans, f, h, w, static_cast<float2*>(d_spectra));
  THFF_CUDA(launched(), "conv2d filter spectrum launch");
  return THFF_OK;
}

thff_status thff_conv2d_async(int dtype, long long nimg_b, int chans, int h, int w, const void* d_x,
                              const void* d_spectra, void* d_y, void* d_workspace, long long workspace_bytes,
                              void* stream) {
  if (dtype != THFF_F32) return fail(THFF_INVALID_ARGUMENT, "conv2d: float storage only");
  if (!conv2d_side_ok(h) || !conv2d_side_ok(w)) return fail(THFF_INVALID_ARGUMENT, "conv2d: image sides must be in {128, ..., 4096}");
  if (nimg_b < 0 || chans <= 0) return fail(THFF_INVALID_ARGUMENT, "conv2d: need batch >= 0 and channels > 0");
  if (nimg_b == 0) return THFF_OK;
  if (!d_x || !d_spectra || !d_y || !d_workspace) return fail(THFF_INVALID_ARGUMENT, "conv2d: null pointer");
  if (!aligned16(d_x) || !aligned16(d_y) || !aligned16(d_workspace) || !aligned16(d_spectra))
    return fail(THFF_INVALID_ARGUMENT, "conv2d: buffers must be 16-byte aligned");
  const long long per_pair = 2LL * h * w * 8;
  if (workspace_bytes / per_pair < 1)
    return fail(THFF_INVALID_ARGUMENT, "conv2d: workspace smaller than one image pair (2*h*w*8 bytes)");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if ((s = ensure_device(dev, &st)) != THFF_OK) return s;
  }
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  auto consts = [st](int n, bool fwd, int var, const Consts** c) -> thff_status {
    std::lock_guard<std::mutex> lock(g_mutex);
    return get_consts(*st, THFF_F32, n, fwd, c, var);
  };
  const bool mixed = g_conv2d_arith.load() == THFF_CONV_MIXED;
  auto cols = [st](int n, const Consts** c) -> thff_status {
    std::lock_guard<std::mutex> lock(g_mutex);
    return get_conv2d_cols_consts(*st, true, n, c);
  };
  if (mixed) {
    // half2 scratch: z0, z1 of chunk * h * w half2, then 2 + chunk pair
    // exponents, the range word and chunk * h row exponents (the float
    // workspace size always covers them)
    const long long chunk = (workspace_bytes - 16) / (2LL * h * w * 4 + 4);
    uint8_t* base = static_cast<uint8_t*>(d_workspace);
    void* z0 = base;
    void* z1 = base + chunk * h * w * 4;
    int* e = reinterpret_cast<int*>(base + 2 * chunk * h * w * 4);
    unsigned* amax = reinterpret_cast<unsigned*>(e + 2 + chunk);
    auto consts_h = [st](int n, bool fwd, const Consts** c) -> thff_status {
      std::lock_guard<std::mutex> lock(g_mutex);
      return get_consts(*st, THFF_F16, n, fwd, c, 0);
    };
    return conv2d_run_h(*st, consts, consts_h, cols, nimg_b, chans, h, w, d_x, d_spectra, d_y, z0, z1, e, amax,
                        chunk, cs);
  }
  const long long chunk = workspace_bytes / per_pair;
  float2* z0 = static_cast<float2*>(d_workspace);
  float2* z1 = z0 + (size_t)chunk * h * w;
  return conv2d_run(*st, consts, nimg_b, chans, h, w, d_x, d_spectra, d_y, z0, z1, chunk, cs);
}

thff_status thff_conv2d(int dtype, long long nimg_b, int chans, int h, int w, const void* d_x, const void* d_spectra,
                        void* d_y, void* d_workspace, long long workspace_bytes, void* stream) {
  thff_status s = thff_conv2d_async(dtype, nimg_b, chans, h, w, d_x, d_spectra, d_y, d_workspace, workspace_bytes,
                                    stream);
  if (s != THFF_OK || nimg_b == 0) return s;
  return thff_sync_check(stream);
}

thff_status thff_conv2d_noalloc(int dtype, long long nimg_b, int chans, int h, int w, const void* d_x,
                                const void* d_spectra, void* d_y, void* stream) {
  if (dtype != THFF_F32) return fail(THFF_INVALID_ARGUMENT, "conv2d: float storage only");
  if (!conv2d_side_ok(h) || !conv2d_side_ok(w)) return fail(THFF_INVALID_ARGUMENT, "conv2d: image sides must be in {128, ..., 4096}");
  if (nimg_b < 0 || chans <= 0) return fail(THFF_INVALID_ARGUMENT, "conv2d: need batch >= 0 and channels > 0");
  const long long per_pair = 2LL * h * w * 8;
  if (per_pair > kNoAllocScratchBytes)
    return fail(THFF_INVALID_ARGUMENT, "thff_conv2d_noalloc: an image pair needs " + std::to_string(per_pair) +
                                           " bytes of scratch but the fixed scratch holds " +
                                           std::to_string(kNoAllocScratchBytes) + " (h*w must be <= 1048576)");
  if (nimg_b == 0) return THFF_OK;
  if (!d_x || !d_spectra || !d_y) return fail(THFF_INVALID_ARGUMENT, "conv2d: null pointer");
  if (!aligned16(d_x) || !aligned16(d_y) || !aligned16(d_spectra))
    return fail(THFF_INVALID_ARGUMENT, "conv2d: buffers must be 16-byte aligned");
  int dev;
  thff_status s = current_device(&dev);
  if (s != THFF_OK) return s;
  DeviceState* st = nullptr;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_dev.find(dev);
    if (it == g_dev.end() || !it->second.ready)
      return fail(THFF_INVALID_ARGUMENT, "thff_conv2d_noalloc: call thff_initialize on this device first "
                                         "(this entry point allocates nothing)");
    st = &it->second;
  }
  // The device address of the array in the current device's context.  It is
  // looked up on every call (the lookup allocates nothing), so an address
  // never outlives the context it belongs to.  In host code the array's name
  // is only a host-side stand-in and must not be passed to a kernel.
  THFF_CUDA(cudaGetSymbolAddress(&scratch, g_conv2d_scratch), "cudaGetSymbolAddress(conv2d scratch)");
  const long long chunk = kNoAllocScratchBytes / per_pair;
  float2* z0 = static_cast<float2*>(scratch);
  float2* z1 = z0 + (size_t)chunk * h * w;
  // Constants are looked up, never built (building allocates).  Every pass
  // writes its whole output region before the next pass reads it, so nothing
  // left in the scratch by an earlier call is read.
  auto consts = [st](int n, bool fwd, int var, const Consts** c) -> thff_status {
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      *c = find_consts(*st, THFF_F32, n, fwd, var);
    }
    if (*c) return THFF_OK;
    return fail(THFF_INVALID_ARGUMENT, "thff_conv2d_noalloc: call thff_initialize(THFF_F32, " + std::to_string(n) +
                                           ") on this device first (this entry point allocates nothing)");
  };
  return conv2d_run(*st, consts, nimg_b, chans, h, w, d_x, d_spectra, d_y, z0, z1, chunk,
                    reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
