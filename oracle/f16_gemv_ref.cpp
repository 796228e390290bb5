// TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's f16 GEMV
// (crates/ffai-mercury/src/asr/f16_gemv.rs), the checker of the CUDA f16
// GEMV in the tests and the bench's CPU leg.  Never the product.
//
// Step for step as the reference:
//   - F16Gemv::new (f16_gemv.rs:89-119): weights to f16, nearest-even
//     (half::f16::from_f32 through candle's to_dtype);
//   - dot_f16 (:170-194): acc0 / acc1, 8 lanes each; per 16 columns
//     acc0[i] = fma(w[k + i], x[k + i], acc0[i]) and acc1[i] likewise for
//     columns k + 8 + i; an 8-column tail into acc0; then
//     a = acc0 + acc1, s = a[0:4] + a[4:8], t = (s0 + s2, s1 + s3), t0 + t1.
// Compiled with -ffp-contract=off so the adds stay adds; the fmas are fmaf.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

float f16_to_f32(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return static_cast<float>(v);
}

float dot_f16(const uint16_t* w, const float* x, int d) {
  float acc0[8] = {}, acc1[8] = {};
  int k = 0;
  for (; k + 16 <= d; k += 16) {
    for (int i = 0; i < 8; ++i) acc0[i] = std::fmaf(f16_to_f32(w[k + i]), x[k + i], acc0[i]);
    for (int i = 0; i < 8; ++i) acc1[i] = std::fmaf(f16_to_f32(w[k + 8 + i]), x[k + 8 + i], acc1[i]);
  }
  for (; k + 8 <= d; k += 8)
    for (int i = 0; i < 8; ++i) acc0[i] = std::fmaf(f16_to_f32(w[k + i]), x[k + i], acc0[i]);
  float a[8];
  for (int i = 0; i < 8; ++i) a[i] = acc0[i] + acc1[i];
  float s[4];
  for (int i = 0; i < 4; ++i) s[i] = a[i] + a[i + 4];
  const float t0 = s[0] + s[2], t1 = s[1] + s[3];
  return t0 + t1;
}

}  // namespace

extern "C" {

// w (rows, cols) f32 -> f16 bits, nearest-even.
void ora_f16_round(const float* w, long long n, uint16_t* out) {
  for (long long i = 0; i < n; ++i) {
    const _Float16 v = static_cast<_Float16>(w[i]);
    std::memcpy(&out[i], &v, 2);
  }
}

// Returns 1 when the shape is not served (cols % 8 != 0), as F16Gemv::new's None.
int ora_f16_serves(int cols) { return cols > 0 && cols % 8 == 0 ? 0 : 1; }

// x (batch, cols) -> out (batch, rows), each activation row on its own (the
// reference's per-row loop), plus bias when given (added after, QLinear).
void ora_f16_gemv(const float* x, int batch, const uint16_t* w16, const float* bias, int rows,
                  int cols, float* out, int threads) {
  auto work = [&](int r0, int r1) {
    for (int b = 0; b < batch; ++b)
      for (int r = r0; r < r1; ++r) {
        float y = dot_f16(w16 + static_cast<size_t>(r) * cols, x + static_cast<size_t>(b) * cols, cols);
        if (bias) y = y + bias[r];
        out[static_cast<size_t>(b) * rows + r] = y;
      }
  };
  const int nt = threads > 0 ? threads : 1;
  std::vector<std::thread> ts;
  const int per = (rows + nt - 1) / nt;
  for (int t = 0; t < nt; ++t) {
    const int r0 = t * per, r1 = r0 + per < rows ? r0 + per : rows;
    if (r0 < r1) ts.emplace_back(work, r0, r1);
  }
  for (auto& t : ts) t.join();
}

}  // extern "C"
