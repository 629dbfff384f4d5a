// thff_oracle.cpp — TEST INFRASTRUCTURE ONLY.
//
// FP64 CPU restatement of the ThunderFFT hot path, used as the checker for the
// CUDA library (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline leg)
// and never as a product code path.
//
// What it restates (reference paths are inside mcrl/thunderfft):
//  * the transform definition of ThunderFFT_global:
//      forward  X[k] = sum_n x[n] exp(-2*pi*i*k*n/N)
//      inverse  x[n] = sum_k X[k] exp(+2*pi*i*k*n/N)   (unnormalized)
//    include/thunderfft/thunderfft.cuh:129-132 (the wrapper contract); the
//    reference itself checks its kernels against cuFFT Z2Z in FP64 on the
//    represented input (sample/validation/fft_validation.cu:202-222).
//    Here that reference transform is an FP64 iterative radix-2 FFT
//    (Cooley & Tukey 1965) plus a naive FP64 DFT for spot checks.
//  * the circular convolution the fused conv1d sample validates against
//    (sample/conv1d/conv1d_fullfft_l4096_thunder.cu:499-545):
//      y[n] = sum_k x[(n-k) mod N] * h[k]
//  * 2-D circular convolution of a zero-padded filter (the conv2d config).
//  * the reference's seeded input generators, so golden inputs match
//    bit-for-bit: sample/validation/fft_validation.cu:130-163 (make_input),
//    sample/fft1d/main.cu:63-77 (tones), sample/bench/paper_fft.cu:27-43 (LCG).
//  * the FP16 "unit" coefficient table the reference's cache test compares
//    bit-for-bit (include/thunderfft/detail/thunderfft_impl_twiddle.cuh:133-274)
//    is NOT restated here: the new library has no such table (its FP16 path
//    has its own operand layout).
//
// Parity status: pinned.  The FFT is checked against numpy.fft (an
// independent FP64 implementation) and against the analytic answers of the
// reference's own validation inputs (impulse -> phase ramp, tone -> single
// bin, constant -> N*c in bin 0); see tests/test_oracle.py.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>
#include <algorithm>

namespace {

constexpr double kTau = 6.283185307179586476925286766559;

int log2_exact(int64_t n) {
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return (int64_t(1) << l) == n ? l : -1;
}

struct Plan {
  int64_t n;
  int logn;
  std::vector<double> wr, wi;      // exp(-2 pi i k / n), k < n/2
  std::vector<uint32_t> rev;
  explicit Plan(int64_t n_) : n(n_), logn(log2_exact(n_)), wr(n_ / 2 + 1), wi(n_ / 2 + 1), rev(n_) {
    for (int64_t k = 0; k < n / 2 + 1; ++k) {
      // exact angle reduction keeps the table at ~1 ulp
      const double a = -kTau * double(k) / double(n);
      wr[k] = std::cos(a);
      wi[k] = std::sin(a);
    }
    for (int64_t i = 0; i < n; ++i) {
      uint32_t r = 0;
      for (int b = 0; b < logn; ++b) r |= ((uint32_t(i) >> b) & 1u) << (logn - 1 - b);
      rev[i] = r;
    }
  }
  // in-place on interleaved complex
  void run(double* x, int forward) const {
    for (int64_t i = 0; i < n; ++i) {
      const int64_t j = rev[i];
      if (j > i) {
        std::swap(x[2 * i], x[2 * j]);
        std::swap(x[2 * i + 1], x[2 * j + 1]);
      }
    }
    const double sgn = forward ? 1.0 : -1.0;
    for (int64_t len = 2; len <= n; len <<= 1) {
      const int64_t half = len >> 1, step = n / len;
      for (int64_t i = 0; i < n; i += len) {
        for (int64_t k = 0; k < half; ++k) {
          const double cr = wr[k * step], ci = sgn * wi[k * step];
          double* a = x + 2 * (i + k);
          double* b = x + 2 * (i + k + half);
          const double tr = b[0] * cr - b[1] * ci;
          const double ti = b[0] * ci + b[1] * cr;
          b[0] = a[0] - tr;
          b[1] = a[1] - ti;
          a[0] += tr;
          a[1] += ti;
        }
      }
    }
  }
};

template <class F>
void parallel_for(int64_t count, int threads, F&& body) {
  if (threads <= 0) threads = int(std::max(1u, std::thread::hardware_concurrency()));
  threads = int(std::min<int64_t>(threads, std::max<int64_t>(count, 1)));
  if (threads <= 1) {
    body(int64_t(0), count);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t chunk = (count + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int64_t b = t * chunk, e = std::min(count, b + chunk);
    if (b >= e) break;
    pool.emplace_back([&body, b, e] { body(b, e); });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int thff_oracle_hardware_threads() { return int(std::max(1u, std::thread::hardware_concurrency())); }

// Batched FP64 C2C FFT, interleaved complex, signal b at [2*b*n, 2*(b+1)*n).
// Returns 0, or -1 for a length that is not a power of two.
int thff_oracle_fft_f64(const double* in, double* out, int64_t n, int64_t batch, int forward,
                        int threads) {
  if (n <= 0 || log2_exact(n) < 0 || batch < 0) return -1;
  Plan plan(n);
  parallel_for(batch, threads, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      if (out + 2 * b * n != in + 2 * b * n) std::memcpy(out + 2 * b * n, in + 2 * b * n, sizeof(double) * 2 * n);
      plan.run(out + 2 * b * n, forward);
    }
  });
  return 0;
}

// Same transform with float32 input/output storage (FP64 arithmetic inside).
int thff_oracle_fft_f32io(const float* in, float* out, int64_t n, int64_t batch, int forward,
                          int threads) {
  if (n <= 0 || log2_exact(n) < 0 || batch < 0) return -1;
  Plan plan(n);
  parallel_for(batch, threads, [&](int64_t b0, int64_t b1) {
    std::vector<double> buf(2 * n);
    for (int64_t b = b0; b < b1; ++b) {
      for (int64_t i = 0; i < 2 * n; ++i) buf[i] = in[2 * b * n + i];
      plan.run(buf.data(), forward);
      for (int64_t i = 0; i < 2 * n; ++i) out[2 * b * n + i] = float(buf[i]);
    }
  });
  return 0;
}

// Naive FP64 DFT (definition), exact angle reduction (k*j mod n).
int thff_oracle_dft_f64(const double* in, double* out, int64_t n, int64_t batch, int forward,
                        int threads) {
  if (n <= 0 || batch < 0) return -1;
  std::vector<double> cr(n), ci(n);
  const double sgn = forward ? -1.0 : 1.0;
  for (int64_t k = 0; k < n; ++k) {
    cr[k] = std::cos(sgn * kTau * double(k) / double(n));
    ci[k] = std::sin(sgn * kTau * double(k) / double(n));
  }
  parallel_for(batch, threads, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const double* x = in + 2 * b * n;
      double* y = out + 2 * b * n;
      for (int64_t k = 0; k < n; ++k) {
        double sr = 0, si = 0;
        for (int64_t j = 0; j < n; ++j) {
          const int64_t idx = (k * j) % n;
          sr += x[2 * j] * cr[idx] - x[2 * j + 1] * ci[idx];
          si += x[2 * j] * ci[idx] + x[2 * j + 1] * cr[idx];
        }
        y[2 * k] = sr;
        y[2 * k + 1] = si;
      }
    }
  });
  return 0;
}

// Direct FP64 circular convolution of real signals with one real filter:
//   y[b][n] = sum_{k<taps} x[b][(n-k) mod N] * h[k]
// (sample/conv1d/conv1d_fullfft_l4096_thunder.cu:499-545 restated for real data).
int thff_oracle_circconv1d_f64(const double* x, const double* h, double* y, int64_t n,
                               int64_t taps, int64_t batch, int threads) {
  if (n <= 0 || taps <= 0 || taps > n || batch < 0) return -1;
  parallel_for(batch, threads, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const double* xs = x + b * n;
      double* ys = y + b * n;
      for (int64_t i = 0; i < n; ++i) {
        double acc = 0;
        for (int64_t k = 0; k < taps; ++k) {
          int64_t j = i - k;
          if (j < 0) j += n;
          acc += xs[j] * h[k];
        }
        ys[i] = acc;
      }
    }
  });
  return 0;
}

// Direct FP64 2-D circular convolution of real images (H x W) with a real
// F x F filter zero-padded to H x W:
//   y[i][j] = sum_{u<F} sum_{v<F} h[u][v] * x[(i-u) mod H][(j-v) mod W]
// filt_index[b] selects the filter of image b (filters are F*F each).
int thff_oracle_circconv2d_f64(const double* x, const double* filters, const int32_t* filt_index,
                               double* y, int64_t H, int64_t W, int64_t F, int64_t batch,
                               int threads) {
  if (H <= 0 || W <= 0 || F <= 0 || F > H || F > W || batch < 0) return -1;
  parallel_for(batch, threads, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const double* xs = x + b * H * W;
      const double* h = filters + int64_t(filt_index[b]) * F * F;
      double* ys = y + b * H * W;
      for (int64_t i = 0; i < H; ++i)
        for (int64_t j = 0; j < W; ++j) {
          double acc = 0;
          for (int64_t u = 0; u < F; ++u) {
            int64_t ii = i - u;
            if (ii < 0) ii += H;
            const double* row = xs + ii * W;
            const double* hr = h + u * F;
            for (int64_t v = 0; v < F; ++v) {
              int64_t jj = j - v;
              if (jj < 0) jj += W;
              acc += hr[v] * row[jj];
            }
          }
          ys[i * W + j] = acc;
        }
    }
  });
  return 0;
}

// The reference validation's seeded inputs, float2 interleaved
// (sample/validation/fft_validation.cu:130-163):
//  kind 0: gaussian (mt19937(1234+n), normal(0,1) floats), scaled per signal to RMS 1
//  kind 1: offset impulse (.75,.25) at (13b+7)%n
//  kind 2: complex tone f = 1 + (7b)%(n-1), amplitude .5, phase .13b
//  kind 3: constant (.25,-.125)
// Kind 0 builds each element as make_float2(normal(random), normal(random))
// (fft_validation.cu:139).  The order in which C++ evaluates two function
// arguments is unspecified; g++ (nvcc's host compiler) evaluates them right
// to left, so the imaginary part is drawn first.  The bit-equality of these
// inputs with the reference's compiled generator is checked by
// tests/test_oracle.py against tests/golden/ref_inputs.npz.
void thff_oracle_make_validation_input(int n, int batch, int kind, float* out) {
  std::fill(out, out + size_t(2) * n * batch, 0.f);
  std::mt19937 random(1234 + n);
  std::normal_distribution<float> normal(0.f, 1.f);
  for (int b = 0; b < batch; ++b) {
    float* s = out + size_t(2) * b * n;
    if (kind == 0) {
      double sq = 0;
      for (int i = 0; i < n; ++i) {
        const float im = normal(random);
        const float re = normal(random);
        s[2 * i] = re;
        s[2 * i + 1] = im;
        sq += double(re) * re + double(im) * im;
      }
      const double scale = std::sqrt(n / sq);
      for (int i = 0; i < n; ++i) {
        s[2 * i] *= scale;
        s[2 * i + 1] *= scale;
      }
    } else if (kind == 1) {
      const int at = (13 * b + 7) % n;
      s[2 * at] = .75f;
      s[2 * at + 1] = .25f;
    } else if (kind == 2) {
      const int f = 1 + (7 * b) % (n - 1);
      for (int i = 0; i < n; ++i) {
        const double ph = kTau * f * i / n + .13 * b;
        s[2 * i] = float(.5 * std::cos(ph));
        s[2 * i + 1] = float(.5 * std::sin(ph));
      }
    } else {
      for (int i = 0; i < n; ++i) {
        s[2 * i] = .25f;
        s[2 * i + 1] = -.125f;
      }
    }
  }
}

// Quick-start tones (sample/fft1d/main.cu:63-77), N = 64.
void thff_oracle_make_fft1d_input(int batch, float* out) {
  const int n = 64;
  for (int b = 0; b < batch; ++b) {
    const double f = 1 + b % 13, amp = 0.5 + 0.1 * (b % 8);
    for (int i = 0; i < n; ++i) {
      const double ph = kTau * i / n;
      out[2 * (size_t(b) * n + i)] = float(amp * std::cos(f * ph) + 0.1 * std::cos(7.0 * ph));
      out[2 * (size_t(b) * n + i) + 1] = float(amp * std::sin(f * ph) + 0.1 * std::sin(7.0 * ph));
    }
  }
}

// Paper-benchmark accuracy input (sample/bench/paper_fft.cu:27-43, the
// `reference != nullptr` branch): LCG complex values scaled by 1/sqrt(n).
void thff_oracle_make_paper_input(int n, int64_t count, float* out) {
  const float inv = 1.0f / std::sqrt(float(n));
  for (int64_t i = 0; i < count; ++i) {
    unsigned z = unsigned(i) * 1664525u + 1013904223u;
    float x = (float(int(z & 65535u)) - 32768.0f) / 32768.0f * inv;
    z = z * 1664525u + 1013904223u;
    float y = (float(int(z & 65535u)) - 32768.0f) / 32768.0f * inv;
    out[2 * i] = x;
    out[2 * i + 1] = y;
  }
}

}  // extern "C"
