/* thff.h — C ABI of libthunderfft_b200.so, the B200 (sm_100a) backend behind
 * the ThunderFFT header API (include/thunderfft/thunderfft.cuh).
 *
 * Plain C: pointers, sizes and int status codes only.  Every entry point
 * operates on the CUDA device that is current on the calling thread.  Device
 * buffers are caller-owned; the library owns only its per-device constants
 * (stage DFT matrices, twiddle tables) and the reference-compatible twiddle
 * cache.  On failure a status is returned and thff_last_error() describes it
 * (thread-local).  No entry point falls back to the CPU.
 *
 * Data layout (same as the reference): `batch` contiguous signals of N complex
 * values, element n of signal b at b*N + n, complex = float2 (x = re, y = im)
 * for THFF_F32 or half2 (low = re, high = im) for THFF_F16.  Forward uses
 * exp(-2*pi*i*k*n/N); inverse uses exp(+...) without 1/N normalization.
 */
#ifndef THFF_H_
#define THFF_H_

#ifdef __cplusplus
extern "C" {
#endif

typedef int thff_status;

enum {
  THFF_OK = 0,
  THFF_INVALID_ARGUMENT = 1, /* maps to std::invalid_argument in the C++ header */
  THFF_CUDA_ERROR = 2,       /* maps to std::runtime_error                    */
  THFF_DEVICE_TIMEOUT = 3,   /* a kernel's bounded wait ran out (runtime_error) */
  THFF_UNSUPPORTED = 4       /* e.g. not an sm_100 device                      */
};

enum { THFF_F32 = 0, THFF_F16 = 1 };

/* Library version string. */
const char* thff_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* thff_last_error(void);

/* Number of kernels this library has launched in this process, on all
 * devices (no reference counterpart).  Benchmarks and tests take the
 * difference across a region to count the library's launches in it. */
unsigned long long thff_launch_count(void);

/* Replaces ThunderFFTInitialize<T>(N)
 * (reference: include/thunderfft/detail/thunderfft_impl_twiddle.cuh:279-327).
 * Validates N in {64,...,4096} before any CUDA call; builds/keeps one cached
 * twiddle table W[k] = (cos 2*pi*k/N, sin 2*pi*k/N) per (dtype, device) —
 * another N replaces it — and prepares the device's FFT constants for N. */
thff_status thff_initialize(int dtype, int n);

/* Replaces ThunderFFTFinalize<T>()
 * (reference: include/thunderfft/detail/thunderfft_impl_twiddle.cuh:358-378).
 * Releases the current device's cached table for dtype; repeated calls are
 * no-ops. */
thff_status thff_finalize(int dtype);

/* The current device's cached table for dtype (NULL/0 when released), the
 * values the reference keeps in d_twiddle_f/_N_f (float) or d_twiddle_h/_N_h
 * (half) (reference: thunderfft_impl_twiddle.cuh:44-48). */
thff_status thff_twiddle_table(int dtype, const void** table, int* n);

/* Replaces ThunderFFT_global<T,N,forward>(in, out, batch, stream)
 * (reference: include/thunderfft/detail/thunderfft_impl_kernel.cuh:6-41):
 * batch < 0 -> INVALID_ARGUMENT; batch == 0 -> OK with no CUDA or pointer
 * access; null or identical pointers -> INVALID_ARGUMENT; unsupported N ->
 * INVALID_ARGUMENT; then launches and synchronizes `stream` (a cudaStream_t,
 * NULL = legacy default stream) before returning, including prior work. */
thff_status thff_global(int dtype, int n, int forward, const void* d_input, void* d_output,
                        int batch, void* stream);

/* Same transform, asynchronous: enqueues on `stream` and returns; 64-bit
 * batch.  Device-side timeouts are reported by the next thff_sync_check. */
thff_status thff_c2c_async(int dtype, int n, int forward, const void* d_input, void* d_output,
                           long long batch, void* stream);

/* Synchronizes `stream` and reports any device-side error of earlier
 * launches on that stream.  Each stream has its own device error word: a
 * bounded wait that runs out in a kernel on one stream is reported only to
 * that stream's next thff_sync_check (which clears it) and never aborts or
 * fails work on another stream.  A device's first 256 distinct streams get
 * words of their own; later streams share them round robin. */
thff_status thff_sync_check(void* stream);


/* Failure-detection self-test (no reference counterpart): launches a kernel
 * whose bounded mbarrier wait can never be satisfied and must give up after
 * limit_us microseconds.  Returns THFF_DEVICE_TIMEOUT when the device-side
 * timeout path works (the CUDA context stays usable), THFF_OK if it did not
 * trigger, or a CUDA error. */
thff_status thff_selftest_wait_timeout(int limit_us, void* stream);

/* Test hook for host-side fault injection (no counterpart in the reference,
 * whose error path is tf_check_cuda, detail/util_cuda.h:20-24).  On the
 * calling thread, the (skip+1)-th CUDA status this library checks after the
 * call reads as `cuda_error` (a cudaError_t value).  The CUDA call itself has
 * still run; only its reported status changes.  The entry point that meets it
 * returns THFF_CUDA_ERROR with the message
 * "[ThunderFFT] <what>: <cudaGetErrorString(cuda_error)>", which the C++
 * header throws as std::runtime_error.  cuda_error = 0 disarms it.  Lets
 * callers and tests exercise their CUDA-failure handling without making a
 * GPU fail. */
thff_status thff_test_inject_cuda_error(int cuda_error, int skip);

/* ---- fused real 1-D FFT convolution --------------------------------------
 * Counterpart of the reference's fused conv1d sample
 * (sample/conv1d/conv1d_fullfft_l4096_thunder.cu:280-331), here for float
 * storage.  For each of `batch` real
 * signals x[b] of length `lin` (zero-padded to n) and one real filter h:
 *     y[b][m] = sum_k x[b][(m-k) mod n] * h[k],   m < n,
 * computed as FFT -> multiply by the filter spectrum -> inverse FFT in ONE
 * kernel.  n in {1024, 4096}; lin <= n and a multiple of sqrt(n); x must be
 * 16-byte aligned; y holds batch*n floats.  With lin + taps - 1 <= n the
 * result equals the linear convolution. */

/* Bytes of the filter spectrum buffer (complex fp32, n entries). */
long long thff_conv1d_spectrum_bytes(int dtype, int n);

/* spectrum[k] = (1/n) * sum_{j<taps} h[j] exp(-2 pi i j k / n), computed on
 * the device (the reference prepares it with cuFFT). */
thff_status thff_conv1d_filter_spectrum(int dtype, int n, const float* d_filter, int taps, void* d_spectrum,
                                        void* stream);

/* Asynchronous fused convolution (see above). */
thff_status thff_conv1d_async(int dtype, int n, int lin, const void* d_x, const void* d_spectrum, void* d_y,
                              long long batch, void* stream);

/* Same, then synchronizes `stream` and reports device-side errors. */
thff_status thff_conv1d(int dtype, int n, int lin, const void* d_x, const void* d_spectrum, void* d_y,
                        long long batch, void* stream);

/* Tensor-core arithmetic of the conv1d kernels (process-wide; default
 * THFF_CONV_MIXED).  Stage 1 always reads the fp32 input as TF32.
 *   THFF_CONV_MIXED: stages 2-4 take FP16 operands (the same 11-bit
 *     significand as TF32) with FP32 accumulation; every FP16 operand is
 *     scaled by an exact power of two chosen from a bound on its magnitude
 *     (per tile for the stage-2 input, per call from max|H| for stage 3), so
 *     any finite fp32 input stays in FP16 range.  The output unscale is one
 *     exact power of two while max|x| * max|H| <= 2^110 (outputs below
 *     about 2^110); past that, near the top of fp32 range, use
 *     THFF_CONV_TF32.
 *   THFF_CONV_TF32: all four stages TF32.
 * No reference counterpart (the reference's conv1d is FP16 only). */
enum { THFF_CONV_MIXED = 0, THFF_CONV_TF32 = 1 };
thff_status thff_conv1d_set_arithmetic(int mode);

/* ---- tiled (overlap-save) 1-D convolution ---------------------------------
 * Counterpart of the reference's tiled conv1d sample (sample/conv1d/main.cu:
 * 38-129, 214-276): each of `batch` complex sequences x[b] (input_len
 * elements, float2 for THFF_F32 or half2 for THFF_F16) is cut into 64-point
 * windows advancing by V = 65 - f; every window goes through FFT -> x filter
 * spectrum -> inverse FFT and keeps its first V outputs.  Result: the valid
 * correlation with the complex filter g (f <= 64 taps),
 *     y[b][i] = sum_{k<f} x[b][i + k] g[k],   i < input_len - f + 1,
 * stored as y[b][input_len - f + 1] in the input's storage type.  The
 * window chain is applied as one precomputed operator (see
 * thff_conv1d_tiled_operator) by the N = 64 tensor-core kernel. */

/* Bytes of the operator buffer for `dtype`. */
long long thff_conv1d_tiled_operator_bytes(int dtype);

/* Builds the operator of filter g (f complex fp32 taps on the device, f in
 * [1, 64]) for `dtype` in d_operator (16-byte aligned, size above).  The
 * reference prepares the filter spectrum with cuFFT (main.cu:145-153,
 * 253-265). */
thff_status thff_conv1d_tiled_operator(int dtype, const void* d_filter, int f, void* d_operator, void* stream);

/* Asynchronous tiled convolution; thff_conv1d_tiled also synchronizes
 * `stream` and reports device-side errors. */
thff_status thff_conv1d_tiled_async(int dtype, long long input_len, int f, const void* d_x, const void* d_operator,
                                    void* d_y, long long batch, void* stream);
thff_status thff_conv1d_tiled(int dtype, long long input_len, int f, const void* d_x, const void* d_operator,
                              void* d_y, long long batch, void* stream);

/* ---- 2-D FFT convolution --------------------------------------------------
 * Counterpart of the reference's 2-D FFT convolution sample
 * (sample/conv2d/thunder.cu:70-207,410-592: row FFT, column FFT x H x
 * column IFFT, row IFFT), here for real fp32 images x[B][C][h][w] with one
 * real f x f filter per channel and circular convolution:
 *     y[b][c][i][j] = sum_{u,v<f} filt[c][u][v] * x[b][c][(i-u) mod h][(j-v) mod w].
 * Images b and b+1 of a channel share one complex 2-D transform.  h, w in
 * {128, ..., 4096}.  The caller provides scratch: a workspace of
 * thff_conv2d_workspace_bytes(..., pairs) bytes processes `pairs` image
 * pairs per pass (any size >= one pair works; larger is faster). */

/* Workspace bytes for processing `pairs` image pairs at a time. */
long long thff_conv2d_workspace_bytes(int dtype, int h, int w, long long pairs);

/* spectra[c][k2][k1] = (1/(h*w)) * sum_{u,v} filt[c][u][v] exp(-2 pi i (u k1/h + v k2/w)),
 * complex fp32 (c*h*w entries); needs channels*f*w*16 bytes of workspace. */
thff_status thff_conv2d_filter_spectra(int dtype, int h, int w, int channels, int f, const float* d_filters,
                                       void* d_spectra, void* d_workspace, long long workspace_bytes,
                                       void* stream);

/* Asynchronous 2-D convolution of all B*C images (see above). */
thff_status thff_conv2d_async(int dtype, long long batch, int channels, int h, int w, const void* d_x,
                              const void* d_spectra, void* d_y, void* d_workspace, long long workspace_bytes,
                              void* stream);

/* Same, then synchronizes `stream` and reports device-side errors. */
thff_status thff_conv2d(int dtype, long long batch, int channels, int h, int w, const void* d_x,
                        const void* d_spectra, void* d_y, void* d_workspace, long long workspace_bytes,
                        void* stream);

/* Arithmetic of thff_conv2d[_async] (process-wide, default THFF_CONV_MIXED;
 * no reference counterpart, the reference's conv2d sample is FP16
 * throughout).
 *   THFF_CONV_TF32: float2 intermediates, TF32 tensor-core passes.
 *   THFF_CONV_MIXED: half2 intermediates; the row pass reads the fp32 images
 *     in TF32, the other three are FP16 passes with FP32 accumulation.  Exact
 *     power-of-two scales chosen from bounds (per image pair from max|x|, per
 *     call from max|H|) keep every half2 value at or below 2^9, so any finite
 *     input stays in FP16 range; the last pass removes them.  It moves 10
 *     instead of 16 bytes per pixel and image pair through HBM.
 * The same workspace size serves both.  thff_conv2d_noalloc always uses
 * THFF_CONV_TF32. */
thff_status thff_conv2d_set_arithmetic(int mode);

/* Allocation-free variant of thff_conv2d_async (no counterpart in the
 * reference).  For callers that cannot allocate device memory where they
 * convolve: plugins and real-time pipelines whose host owns all device
 * memory, pooling allocators that must account for every byte.  The scratch
 * is a fixed 16 MiB device array inside the library (every GPU that loads
 * the library holds it until exit), so one image pair must fit in it:
 * h*w <= 1048576; larger images are rejected with THFF_INVALID_ARGUMENT.
 * Any batch works (pairs are processed in passes).  The call allocates
 * nothing: call thff_initialize(THFF_F32, h) and thff_initialize(THFF_F32, w)
 * on the device beforehand.  The first call on a device resolves the array's
 * device address (cudaGetSymbolAddress).  Asynchronous: synchronize the
 * stream (thff_sync_check) before reading y.  All calls share the one
 * array, so calls whose work overlaps on the GPU (e.g. on two streams)
 * race; serialize them. */
thff_status thff_conv2d_noalloc(int dtype, long long batch, int channels, int h, int w, const void* d_x,
                                const void* d_spectra, void* d_y, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* THFF_H_ */
