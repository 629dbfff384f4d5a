// Host-only argument contract of the header API, written as a user of the
// reference would (sample/validation/fft_validation.cu:331-352): every check
// must throw std::invalid_argument (or return for batch 0) before any CUDA
// call, so this program runs without a GPU.  Exit 0 = all 18 checks passed.
#include <thunderfft/thunderfft.cuh>

#include <cstdio>
#include <stdexcept>
#include <string>

static int checks = 0;

template <class Op>
static void expect_invalid(Op op, const char* what) {
  try {
    op();
  } catch (const std::invalid_argument&) {
    ++checks;
    return;
  }
  throw std::runtime_error(std::string("did not reject ") + what);
}

template <class T>
static void check_host_arguments() {
  vec2_t<T> value{};
  expect_invalid([] { thunderfft::ThunderFFT_global<T, 64>(nullptr, nullptr, -1); }, "negative batch");
  expect_invalid([&] { thunderfft::ThunderFFT_global<T, 64>(nullptr, &value, 1); }, "null input");
  expect_invalid([&] { thunderfft::ThunderFFT_global<T, 64>(&value, nullptr, 1); }, "null output");
  expect_invalid([&] { thunderfft::ThunderFFT_global<T, 64>(&value, &value, 1); }, "aliased input/output");
  thunderfft::ThunderFFT_global<T, 64>(nullptr, nullptr, 0);
  ++checks;
  for (int n : {-1, 0, 32, 8192})
    expect_invalid([n] { thunderfft::ThunderFFTInitialize<T>(n); }, "unsupported initialization length");
}

int main() {
  try {
    check_host_arguments<float>();
    check_host_arguments<half>();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "host contract FAILED: %s\n", e.what());
    return 1;
  }
  std::printf("host contract: %d checks passed before any CUDA call\n", checks);
  return checks == 18 ? 0 : 1;
}
