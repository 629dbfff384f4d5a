// CUDA-failure contract of the header API (the reference's tf_check_cuda,
// detail/util_cuda.h:20-24): a failing CUDA call inside ThunderFFT_global or
// ThunderFFTInitialize surfaces as std::runtime_error whose message reads
// "[ThunderFFT] <what>: <cudaGetErrorString(e)>", and the library keeps
// working afterwards.  The failure is injected on the host through
// thff_test_inject_cuda_error (the CUDA call still runs; only its reported
// status changes), so no GPU is made to fail.
#include <thunderfft/thunderfft.cuh>

#include <cstdio>
#include <stdexcept>
#include <string>

namespace {
int checks = 0;
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void require(bool c, const std::string& what) {
  if (!c) throw std::runtime_error("contract check failed: " + what);
  ++checks;
}
bool ends_with(const std::string& s, const std::string& tail) {
  return s.size() >= tail.size() && s.compare(s.size() - tail.size(), tail.size(), tail) == 0;
}

// Runs f with `code` injected into the (skip+1)-th checked CUDA status; it
// must throw std::runtime_error with the reference's message shape.
template <class F>
void expect_cuda_failure(F&& f, cudaError_t code, int skip, const char* what) {
  if (thff_test_inject_cuda_error(int(code), skip) != THFF_OK) throw std::runtime_error("inject refused");
  bool thrown = false;
  try {
    f();
  } catch (const std::invalid_argument&) {
    require(false, std::string(what) + ": invalid_argument instead of runtime_error");
  } catch (const std::runtime_error& e) {
    thrown = true;
    const std::string m = e.what();
    require(m.rfind("[ThunderFFT] ", 0) == 0, std::string(what) + ": message prefix, got '" + m + "'");
    require(ends_with(m, std::string(": ") + cudaGetErrorString(code)),
            std::string(what) + ": message suffix, got '" + m + "'");
  }
  thff_test_inject_cuda_error(0, 0);  // disarm in case the path checked fewer statuses
  require(thrown, std::string(what) + ": no exception");
}
}  // namespace

int main() {
  try {
    constexpr int N = 1024, B = 8;
    float2 *in = nullptr, *out = nullptr;
    ck(cudaMalloc(&in, sizeof(float2) * N * B), "malloc");
    ck(cudaMalloc(&out, sizeof(float2) * N * B), "malloc");
    ck(cudaMemset(in, 0, sizeof(float2) * N * B), "memset");
    thunderfft::ThunderFFTInitialize<float>(N);
    auto run = [&] { thunderfft::ThunderFFT_global<float, N, true>(in, out, B, 0); };
    run();  // works before
    for (int skip = 0; skip < 3; ++skip) {
      expect_cuda_failure(run, cudaErrorMemoryAllocation, skip, "ThunderFFT_global");
      expect_cuda_failure(run, cudaErrorLaunchFailure, skip, "ThunderFFT_global");
      run();  // and after: nothing sticky was left behind
    }
    expect_cuda_failure([] { thunderfft::ThunderFFTInitialize<half>(256); }, cudaErrorMemoryAllocation, 0,
                        "ThunderFFTInitialize");
    thunderfft::ThunderFFTInitialize<half>(256);
    thunderfft::ThunderFFTFinalize<half>();
    thunderfft::ThunderFFTFinalize<float>();
    // invalid arguments stay invalid_argument even when a failure is armed
    thff_test_inject_cuda_error(int(cudaErrorMemoryAllocation), 0);
    bool inv = false;
    try {
      thunderfft::ThunderFFT_global<float, N, true>(in, in, B, 0);
    } catch (const std::invalid_argument&) {
      inv = true;
    }
    thff_test_inject_cuda_error(0, 0);
    require(inv, "aliased buffers are invalid_argument");
    ck(cudaFree(in), "free");
    ck(cudaFree(out), "free");
    std::printf("cuda error contract: %d checks passed\n", checks);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "cuda error contract error: %s\n", e.what());
    return 2;
  }
}
