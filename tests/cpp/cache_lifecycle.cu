// Twiddle-cache lifecycle through the header API, mirroring the reference's
// sample/validation/cache_validation.cu (check_live / check_lifecycle /
// cross-device check_type): device symbols hold the live table pointer and
// N; W[0] = 1+0i, W[1] = (cos 2pi/N, sin 2pi/N); same-N initialization keeps
// the allocation, another N replaces it, Finalize clears pointer and length,
// repeated Finalize is fine, per-device ownership; the FP16 unit table
// equals build_unit_twiddle_host bit for bit.  No FFT kernels are launched.
#include <thunderfft/thunderfft.cuh>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace {
int checks = 0;
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void require(bool c, const std::string& what) {
  if (!c) throw std::runtime_error("cache check failed: " + what);
  ++checks;
}
template <class T>
using Pair = typename thunderfft::TwiddleCache<T>::TwiddleT;
template <class T>
struct Snap {
  const Pair<T>* p = nullptr;
  int n = 0;
};
template <class T>
Snap<T> snapshot() {
  Snap<T> s;
  if constexpr (std::is_same_v<T, float>) {
    ck(cudaMemcpyFromSymbol(&s.p, thunderfft::detail::d_twiddle_f, sizeof(s.p)), "sym");
    ck(cudaMemcpyFromSymbol(&s.n, thunderfft::detail::d_twiddle_N_f, sizeof(s.n)), "sym");
  } else {
    ck(cudaMemcpyFromSymbol(&s.p, thunderfft::detail::d_twiddle_h, sizeof(s.p)), "sym");
    ck(cudaMemcpyFromSymbol(&s.n, thunderfft::detail::d_twiddle_N_h, sizeof(s.n)), "sym");
  }
  return s;
}
template <class T>
Snap<T> check_live(int device, int n) {
  const auto s = snapshot<T>();
  require(s.p != nullptr, "live pointer");
  require(s.n == n, "live length");
  cudaPointerAttributes a{};
  ck(cudaPointerGetAttributes(&a, s.p), "attrs");
  require(a.type == cudaMemoryTypeDevice && a.device == device, "device ownership");
  Pair<T> w[2];
  ck(cudaMemcpy(w, s.p, sizeof(w), cudaMemcpyDeviceToHost), "d2h");
  float2 z, o;
  if constexpr (std::is_same_v<T, half>) { z = __half22float2(w[0]); o = __half22float2(w[1]); }
  else { z = w[0]; o = w[1]; }
  const double tol = std::is_same_v<T, half> ? 1e-3 : 1e-6, tau = 6.283185307179586;
  require(z.x == 1.f && z.y == 0.f, "W[0] == 1+0i");
  require(std::abs(o.x - std::cos(tau / n)) <= tol && std::abs(o.y - std::sin(tau / n)) <= tol, "W[1]");
  if constexpr (std::is_same_v<T, half>) {
    std::vector<half2> expect, got(thunderfft::UNIT_W_SIZE);
    thunderfft::build_unit_twiddle_host(expect);
    ck(cudaMemcpyFromSymbol(got.data(), thunderfft::detail::d_unit_twiddle_half2, got.size() * sizeof(half2)), "sym");
    require(std::memcmp(got.data(), expect.data(), got.size() * sizeof(half2)) == 0, "unit table");
  }
  return s;
}
template <class T>
void check_released() {
  const auto s = snapshot<T>();
  require(s.p == nullptr && s.n == 0, "released");
}
template <class T>
void lifecycle(int device) {
  ck(cudaSetDevice(device), "set device");
  thunderfft::ThunderFFTInitialize<T>(64);
  const auto first = check_live<T>(device, 64);
  thunderfft::ThunderFFTInitialize<T>(64);
  require(check_live<T>(device, 64).p == first.p, "cache hit keeps allocation");
  thunderfft::ThunderFFTInitialize<T>(128);
  check_live<T>(device, 128);
  thunderfft::ThunderFFTFinalize<T>();
  check_released<T>();
  thunderfft::ThunderFFTFinalize<T>();
  check_released<T>();
  thunderfft::ThunderFFTInitialize<T>(64);
  check_live<T>(device, 64);
  thunderfft::ThunderFFTFinalize<T>();
  check_released<T>();
}
template <class T>
void cross_device(int count) {
  std::vector<Snap<T>> live;
  for (int d = 0; d < count; ++d) {
    ck(cudaSetDevice(d), "set device");
    thunderfft::ThunderFFTInitialize<T>(d % 2 ? 128 : 64);
    live.push_back(check_live<T>(d, d % 2 ? 128 : 64));
  }
  for (int d = 0; d < count; ++d) {
    ck(cudaSetDevice(d), "set device");
    require(check_live<T>(d, live[d].n).p == live[d].p, "other devices keep their allocation");
    thunderfft::ThunderFFTFinalize<T>();
    check_released<T>();
  }
}
}  // namespace

int main() {
  try {
    int count = 0;
    ck(cudaGetDeviceCount(&count), "device count");
    for (int d = 0; d < count; ++d) { lifecycle<float>(d); lifecycle<half>(d); }
    cross_device<float>(count);
    cross_device<half>(count);
    std::printf("cache lifecycle: %d checks passed on %d device(s)\n", checks, count);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "cache lifecycle error: %s\n", e.what());
    return 2;
  }
}
