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
 * launches on this device. */
thff_status thff_sync_check(void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* THFF_H_ */
