// TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's int8 GEMV
// (crates/ffai-mercury/src/asr/vocab_int8.rs), used by the tests and the
// bench's CPU leg as the checker of the CUDA int8 GEMV.  Never the product.
//
// The arithmetic is the reference's, step for step, so results can be
// compared bit for bit:
//   - Int8Vocab::new (vocab_int8.rs:97-166): per row, per block of `blk`
//     weights: amax, scale = amax / 127 (1 when amax == 0), q = round(w /
//     scale) clamped to [-127, 127] (round half away from zero, Rust's
//     f32::round), block sum of q; c += scale * blocksum in block order;
//     corr = 64 * c.
//   - Int8VocabOp::cpu_fwd (:226-266): activation amax, sx = amax / 63 (1
//     when 0), xu = round(x / sx) clamped to [-64, 63] plus 64 (a u8 in
//     [0, 127]); per row the blocked dot, then (acc - corr) * sx.
//   - dot_i8_blocked (:280-305): per block the exact integer sum of
//     xu * q (the reference's maddubs pair sums cannot saturate: 7-bit
//     activations), converted to f32, times the block scale, added to a f32
//     accumulator in block order.
// Compiled with -ffp-contract=off so `acc += s * b` stays a multiply then an
// add, as in the Rust source.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

float rust_round(float x) { return std::round(x); }  // half away from zero, like f32::round

// f32::clamp then `as` to an integer: NaN (which clamp passes through)
// becomes 0 under Rust's saturating cast.
int rust_clamp_cast(float r, float lo, float hi) {
  if (std::isnan(r)) return 0;
  return static_cast<int>(std::fmin(std::fmax(r, lo), hi));
}

}  // namespace

extern "C" {

// w (vocab, d) f32 row-major -> qw (vocab, d) int8, bscale (vocab, d / blk),
// corr (vocab).  Returns 1 when the shape is not served (the reference's
// `Ok(None)`): blk == 0, blk % 32 != 0 or d % blk != 0.
int ora_int8_quantize(const float* w, int vocab, int d, int blk, int8_t* qw, float* bscale,
                      float* corr) {
  if (blk <= 0 || blk % 32 != 0 || d % blk != 0) return 1;
  const int nb = d / blk;
  for (int v = 0; v < vocab; ++v) {
    const float* row = w + static_cast<size_t>(v) * d;
    float c = 0.f;
    for (int b = 0; b < nb; ++b) {
      const float* bw = row + b * blk;
      float amax = 0.f;
      for (int k = 0; k < blk; ++k) amax = std::fmax(amax, std::fabs(bw[k]));
      const float sc = amax > 0.f ? amax / 127.0f : 1.0f;
      bscale[static_cast<size_t>(v) * nb + b] = sc;
      int32_t bsum = 0;
      for (int k = 0; k < blk; ++k) {
        const int8_t qi = static_cast<int8_t>(rust_clamp_cast(rust_round(bw[k] / sc), -127.0f, 127.0f));
        qw[static_cast<size_t>(v) * d + b * blk + k] = qi;
        bsum += qi;
      }
      c += sc * static_cast<float>(bsum);
    }
    corr[v] = 64.0f * c;
  }
  return 0;
}

// x (batch, d) f32 -> out (batch, vocab) f32, each activation row quantized
// on its own (the reference is called once per row).
void ora_int8_gemv(const float* x, int batch, const int8_t* qw, const float* bscale,
                   const float* corr, int vocab, int d, int blk, float* out, int threads) {
  const int nb = d / blk;
  for (int bi = 0; bi < batch; ++bi) {
    const float* xr = x + static_cast<size_t>(bi) * d;
    float amax = 0.f;
    for (int k = 0; k < d; ++k) amax = std::fmax(amax, std::fabs(xr[k]));
    const float sx = amax > 0.f ? amax / 63.0f : 1.0f;
    std::vector<uint8_t> xu(d);
    for (int k = 0; k < d; ++k) {
      xu[k] = static_cast<uint8_t>(rust_clamp_cast(rust_round(xr[k] / sx), -64.0f, 63.0f) + 64);
    }
    float* o = out + static_cast<size_t>(bi) * vocab;
    auto rows = [&](int v0, int v1) {
      for (int v = v0; v < v1; ++v) {
        const int8_t* wr = qw + static_cast<size_t>(v) * d;
        float acc = 0.f;
        for (int b = 0; b < nb; ++b) {
          int32_t s = 0;
          for (int k = 0; k < blk; ++k) s += static_cast<int32_t>(xu[b * blk + k]) * wr[b * blk + k];
          acc += static_cast<float>(s) * bscale[static_cast<size_t>(v) * nb + b];
        }
        o[v] = (acc - corr[v]) * sx;
      }
    };
    const int nt = threads > 0 ? threads : 1;
    std::vector<std::thread> ts;
    const int per = (vocab + nt - 1) / nt;
    for (int t = 0; t < nt; ++t) {
      const int v0 = t * per, v1 = std::min(vocab, v0 + per);
      if (v0 < v1) ts.emplace_back(rows, v0, v1);
    }
    for (auto& t : ts) t.join();
  }
}

}  // extern "C"
