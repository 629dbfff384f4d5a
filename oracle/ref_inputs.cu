// ref_inputs.cu — TEST INFRASTRUCTURE ONLY: exposes the REFERENCE's own
// seeded input generator, make_input (sample/validation/fft_validation.cu:
// 130-163), through a C entry point, so that the oracle's restatement of it
// can be checked bit for bit against the compiled original.
//
// oracle/build_ref.py compiles this file with THFF_REF_VALIDATION_SOURCE set
// to the path of the reference's fft_validation.cu (read where it lies, never
// copied) and the reference's include/ directory on the include path.  The
// program's main is renamed so that this translation unit can be a shared
// library; no kernel of it is ever launched.  Output: oracle/_ref/
// libthff_ref_inputs.so, used only by tests/golden/make_ref_inputs.py.
#define main thff_ref_validation_main
#include THFF_REF_VALIDATION_SOURCE
#undef main

#include <cstring>

extern "C" __attribute__((visibility("default"))) void thff_ref_make_input(int n, int batch, int kind, float* out) {
  const std::vector<float2> v = make_input(n, batch, kind);
  std::memcpy(out, v.data(), v.size() * sizeof(float2));
}
