// ref_harness.cu — TEST INFRASTRUCTURE ONLY: a C-callable wrapper around the
// REFERENCE's own ThunderFFT_global (mcrl/thunderfft, header-only; its
// include/ directory is put on the include path by oracle/build_ref.py).
// Built for sm_100a into oracle/_ref/libthff_ref.so so that tests can
// compare this library's output with the reference's output on the same
// GPU and inputs, and bench.py can time the reference beside it.  Nothing of
// the product links or loads this file.
#include <thunderfft/thunderfft.cuh>

#include <cstring>
#include <stdexcept>
#include <string>

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_err;

template <class T, int N>
int call(int fwd, void* in, void* out, int batch, cudaStream_t s) {
  using V = vec2_t<T>;
  if (fwd) thunderfft::ThunderFFT_global<T, N, true>(static_cast<V*>(in), static_cast<V*>(out), batch, s);
  else thunderfft::ThunderFFT_global<T, N, false>(static_cast<V*>(in), static_cast<V*>(out), batch, s);
  return 0;
}

template <class T>
int dispatch(int n, int fwd, void* in, void* out, int batch, cudaStream_t s) {
  switch (n) {
    case 64: return call<T, 64>(fwd, in, out, batch, s);
    case 128: return call<T, 128>(fwd, in, out, batch, s);
    case 256: return call<T, 256>(fwd, in, out, batch, s);
    case 512: return call<T, 512>(fwd, in, out, batch, s);
    case 1024: return call<T, 1024>(fwd, in, out, batch, s);
    case 2048: return call<T, 2048>(fwd, in, out, batch, s);
    case 4096: return call<T, 4096>(fwd, in, out, batch, s);
  }
  throw std::invalid_argument("unsupported N");
}
}  // namespace

REF_API const char* thff_ref_last_error() { return g_err.c_str(); }

// dtype 0 = float (float2/TF32), 1 = half (half2/FP16)
REF_API int thff_ref_initialize(int dtype, int n) {
  try {
    if (dtype == 0) thunderfft::ThunderFFTInitialize<float>(n);
    else thunderfft::ThunderFFTInitialize<half>(n);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

REF_API int thff_ref_finalize(int dtype) {
  try {
    if (dtype == 0) thunderfft::ThunderFFTFinalize<float>();
    else thunderfft::ThunderFFTFinalize<half>();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

REF_API int thff_ref_global(int dtype, int n, int fwd, void* in, void* out, int batch, void* stream) {
  try {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dtype == 0 ? dispatch<float>(n, fwd, in, out, batch, s) : dispatch<half>(n, fwd, in, out, batch, s);
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}
