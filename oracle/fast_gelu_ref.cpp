// TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's FastGelu
// (crates/ffai-mercury/src/asr/text_decoder.rs:341-350, gelu_scalar), the
// checker of the GEMM epilogue's activation.  Never the product.
//
//   u   = 0.7978846 * mul_add(0.044715 * t * t, t, t)
//   u2  = min(u * u, 64)
//   num = u * (135135 + u2 * (17325 + u2 * (378 + u2)))
//   den = 135135 + u2 * (62370 + u2 * (3150 + u2 * 28))
//   out = 0.5 * t * (1 + clamp(num / den, -1, 1))
// f32 throughout; mul_add is a fused multiply-add (std::fmaf), every other
// operation rounded on its own (-ffp-contract=off), left to right as written.
#include <algorithm>
#include <cmath>

extern "C" {

void ora_fast_gelu(const float* x, float* y, long long n) {
  for (long long i = 0; i < n; ++i) {
    const float t = x[i];
    const float u = 0.7978846f * std::fmaf(0.044715f * t * t, t, t);
    const float u2 = std::fmin(u * u, 64.0f);  // Rust f32::min: a NaN yields the other operand
    const float num = u * (135135.0f + u2 * (17325.0f + u2 * (378.0f + u2)));
    const float den = 135135.0f + u2 * (62370.0f + u2 * (3150.0f + u2 * 28.0f));
    const float r = std::min(std::max(num / den, -1.0f), 1.0f);  // NaN stays NaN, as Rust clamp
    y[i] = 0.5f * t * (1.0f + r);
  }
}

}  // extern "C"
