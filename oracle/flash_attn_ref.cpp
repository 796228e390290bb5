// TEST INFRASTRUCTURE ONLY -- the CPU oracle for the Whisper attention path.
//
// This file is a C++ restatement of the reference's AVX2 flash attention,
// `crates/ffai-mercury/src/asr/flash_attn.rs` (Remade-With-Rust/FFAI 0.6.2).
// The reference is Rust; no Rust toolchain exists on the build or GPU hosts,
// so the reference itself cannot be compiled or run.  This restatement keeps
// the reference's tiling (BQ=64 query rows x BK=256 key columns, 4x16 AVX2
// register blocks), its loop and reduction orders, its vectorised `exp`
// polynomial and its scalar tails, so that it reproduces the reference's
// arithmetic, not merely the mathematical function.  Compile with
// -ffp-contract=off: Rust never contracts `a += x * y` into an FMA, and the
// scalar tails must round the same way.
//
// Parity pin: the reference ships no golden vectors for attention.  Its only
// known-answer tests are `matches_three_op_path` (flash_attn.rs:1005-1021,
// max |delta| < 1e-4 against softmax(q@k)@v at H=4, N=512) and
// `declines_unsupported_shapes` (flash_attn.rs:1024-1039); the test suite
// replays both against this file.  Parity with the reference is therefore
// pinned to the reference's own tests, not to outputs of the reference.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
// load this library.  The product path (ffai_b200/) never calls it.

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int BQ = 64;   // flash_attn.rs:48
constexpr int BK = 256;  // flash_attn.rs:49
constexpr int HD = 64;   // flash_attn.rs:50
constexpr int MIN_SEQ = 256;  // flash_attn.rs:55

// FFAI_DECODE_MIN_KEYS knob, default 8 (knobs.rs:163-168).  The oracle reads
// the same environment variable once, as the reference's knob does.
int min_decode_keys() {
  static int v = [] {
    const char* s = std::getenv("FFAI_DECODE_MIN_KEYS");
    if (s && *s) {
      char* end = nullptr;
      long x = std::strtol(s, &end, 10);
      if (end && *end == 0 && x >= 0) return static_cast<int>(x);
    }
    return 8;
  }();
  return v;
}

bool have_avx2() {  // flash_attn.rs:84-91
  static bool ok = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  return ok;
}

bool have_f16c() {  // flash_attn.rs:75-80
  static bool ok = __builtin_cpu_supports("f16c");
  return ok;
}

// --- vector helpers (flash_attn.rs:545-593) --------------------------------

// exp(x) = 2^(x log2 e): integer part into the exponent field, fractional
// part f in [-0.5, 0.5] by the reference's degree-5 polynomial
// (flash_attn.rs:553-572, coefficients :559-564).
__attribute__((target("avx2,fma"))) inline __m256 exp256(__m256 x) {
  x = _mm256_max_ps(x, _mm256_set1_ps(-87.0f));
  const __m256 t = _mm256_mul_ps(x, _mm256_set1_ps(1.44269504088896340736f));
  const __m256 k = _mm256_round_ps(t, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  const __m256 f = _mm256_sub_ps(t, k);
  __m256 p = _mm256_set1_ps(0.0013333558f);
  p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.009618129f));
  p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.05550411f));
  p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.2402265f));
  p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(0.6931472f));
  p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(1.0f));
  const __m256i ki = _mm256_cvtps_epi32(k);
  const __m256 pow2k = _mm256_castsi256_ps(
      _mm256_slli_epi32(_mm256_add_epi32(ki, _mm256_set1_epi32(127)), 23));
  return _mm256_mul_ps(p, pow2k);
}

__attribute__((target("avx2,fma"))) inline float hmax256(__m256 v) {
  __m128 m = _mm_max_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  m = _mm_max_ps(m, _mm_movehl_ps(m, m));
  m = _mm_max_ss(m, _mm_shuffle_ps(m, m, 1));
  return _mm_cvtss_f32(m);
}

__attribute__((target("avx2,fma"))) inline float hsum256(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
  return _mm_cvtss_f32(s);
}

inline float rust_max(float a, float b) {
  // f32::max ignores a NaN operand; inputs here are finite or -inf.
  if (std::isnan(a)) return b;
  if (std::isnan(b)) return a;
  return a > b ? a : b;
}

inline float f16_to_f32(uint16_t h) {  // half::f16 -> f32, exact widening
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// --- encoder kernel pieces (flash_attn.rs:797-998) ---------------------------

// S = Q_block @ K_block with a 4x16 register block over the 64-step
// contraction; scalar remainders for ragged columns and rows
// (flash_attn.rs:797-873).
__attribute__((target("avx2,fma"))) void scores_tile(const float* qs, const float* kt,
                                                     float* scores, int rows, int k0, int cols,
                                                     int seq) {
  int i0 = 0;
  for (; i0 + 4 <= rows; i0 += 4) {
    int j0 = 0;
    for (; j0 + 16 <= cols; j0 += 16) {
      __m256 a00 = _mm256_setzero_ps(), a01 = _mm256_setzero_ps();
      __m256 a10 = _mm256_setzero_ps(), a11 = _mm256_setzero_ps();
      __m256 a20 = _mm256_setzero_ps(), a21 = _mm256_setzero_ps();
      __m256 a30 = _mm256_setzero_ps(), a31 = _mm256_setzero_ps();
      for (int t = 0; t < HD; ++t) {
        const float* kp = kt + static_cast<size_t>(t) * seq + k0 + j0;
        const __m256 kv0 = _mm256_loadu_ps(kp);
        const __m256 kv1 = _mm256_loadu_ps(kp + 8);
        const __m256 q0 = _mm256_set1_ps(qs[i0 * HD + t]);
        const __m256 q1 = _mm256_set1_ps(qs[(i0 + 1) * HD + t]);
        const __m256 q2 = _mm256_set1_ps(qs[(i0 + 2) * HD + t]);
        const __m256 q3 = _mm256_set1_ps(qs[(i0 + 3) * HD + t]);
        a00 = _mm256_fmadd_ps(q0, kv0, a00);
        a01 = _mm256_fmadd_ps(q0, kv1, a01);
        a10 = _mm256_fmadd_ps(q1, kv0, a10);
        a11 = _mm256_fmadd_ps(q1, kv1, a11);
        a20 = _mm256_fmadd_ps(q2, kv0, a20);
        a21 = _mm256_fmadd_ps(q2, kv1, a21);
        a30 = _mm256_fmadd_ps(q3, kv0, a30);
        a31 = _mm256_fmadd_ps(q3, kv1, a31);
      }
      _mm256_storeu_ps(scores + i0 * BK + j0, a00);
      _mm256_storeu_ps(scores + i0 * BK + j0 + 8, a01);
      _mm256_storeu_ps(scores + (i0 + 1) * BK + j0, a10);
      _mm256_storeu_ps(scores + (i0 + 1) * BK + j0 + 8, a11);
      _mm256_storeu_ps(scores + (i0 + 2) * BK + j0, a20);
      _mm256_storeu_ps(scores + (i0 + 2) * BK + j0 + 8, a21);
      _mm256_storeu_ps(scores + (i0 + 3) * BK + j0, a30);
      _mm256_storeu_ps(scores + (i0 + 3) * BK + j0 + 8, a31);
    }
    for (int j = j0; j < cols; ++j) {
      for (int m = 0; m < 4; ++m) {
        float a = 0.0f;
        for (int t = 0; t < HD; ++t) {
          a += qs[(i0 + m) * HD + t] * kt[static_cast<size_t>(t) * seq + k0 + j];
        }
        scores[(i0 + m) * BK + j] = a;
      }
    }
  }
  for (int i = i0; i < rows; ++i) {
    for (int j = 0; j < cols; ++j) {
      float a = 0.0f;
      for (int t = 0; t < HD; ++t) {
        a += qs[i * HD + t] * kt[static_cast<size_t>(t) * seq + k0 + j];
      }
      scores[i * BK + j] = a;
    }
  }
}

// acc += P_block @ V_block, 4 rows x 16 head dims in registers
// (flash_attn.rs:880-948).
__attribute__((target("avx2,fma"))) void accum_pv(const float* scores, const float* v,
                                                  float* acc, int rows, int k0, int cols) {
  int i0 = 0;
  for (; i0 + 4 <= rows; i0 += 4) {
    for (int d0 = 0; d0 < HD; d0 += 16) {
      float* ap = acc;
      __m256 a00 = _mm256_loadu_ps(ap + i0 * HD + d0);
      __m256 a01 = _mm256_loadu_ps(ap + i0 * HD + d0 + 8);
      __m256 a10 = _mm256_loadu_ps(ap + (i0 + 1) * HD + d0);
      __m256 a11 = _mm256_loadu_ps(ap + (i0 + 1) * HD + d0 + 8);
      __m256 a20 = _mm256_loadu_ps(ap + (i0 + 2) * HD + d0);
      __m256 a21 = _mm256_loadu_ps(ap + (i0 + 2) * HD + d0 + 8);
      __m256 a30 = _mm256_loadu_ps(ap + (i0 + 3) * HD + d0);
      __m256 a31 = _mm256_loadu_ps(ap + (i0 + 3) * HD + d0 + 8);
      for (int j = 0; j < cols; ++j) {
        const float* vp = v + static_cast<size_t>(k0 + j) * HD + d0;
        const __m256 vv0 = _mm256_loadu_ps(vp);
        const __m256 vv1 = _mm256_loadu_ps(vp + 8);
        const __m256 p0 = _mm256_set1_ps(scores[i0 * BK + j]);
        const __m256 p1 = _mm256_set1_ps(scores[(i0 + 1) * BK + j]);
        const __m256 p2 = _mm256_set1_ps(scores[(i0 + 2) * BK + j]);
        const __m256 p3 = _mm256_set1_ps(scores[(i0 + 3) * BK + j]);
        a00 = _mm256_fmadd_ps(p0, vv0, a00);
        a01 = _mm256_fmadd_ps(p0, vv1, a01);
        a10 = _mm256_fmadd_ps(p1, vv0, a10);
        a11 = _mm256_fmadd_ps(p1, vv1, a11);
        a20 = _mm256_fmadd_ps(p2, vv0, a20);
        a21 = _mm256_fmadd_ps(p2, vv1, a21);
        a30 = _mm256_fmadd_ps(p3, vv0, a30);
        a31 = _mm256_fmadd_ps(p3, vv1, a31);
      }
      _mm256_storeu_ps(ap + i0 * HD + d0, a00);
      _mm256_storeu_ps(ap + i0 * HD + d0 + 8, a01);
      _mm256_storeu_ps(ap + (i0 + 1) * HD + d0, a10);
      _mm256_storeu_ps(ap + (i0 + 1) * HD + d0 + 8, a11);
      _mm256_storeu_ps(ap + (i0 + 2) * HD + d0, a20);
      _mm256_storeu_ps(ap + (i0 + 2) * HD + d0 + 8, a21);
      _mm256_storeu_ps(ap + (i0 + 3) * HD + d0, a30);
      _mm256_storeu_ps(ap + (i0 + 3) * HD + d0 + 8, a31);
    }
  }
  for (int i = i0; i < rows; ++i) {
    for (int j = 0; j < cols; ++j) {
      const float p = scores[i * BK + j];
      for (int d = 0; d < HD; ++d) {
        acc[i * HD + d] += p * v[static_cast<size_t>(k0 + j) * HD + d];
      }
    }
  }
}

struct SoftmaxStep {
  float new_max, correction, block_sum;
};

// Online softmax over one score row (flash_attn.rs:955-998).  The correction
// is 0 while the running max is still -inf (:976-980); tails use scalar exp.
__attribute__((target("avx2,fma"))) SoftmaxStep softmax_row(float* row, int cols, float run_max) {
  __m256 vmax = _mm256_set1_ps(-INFINITY);
  int j = 0;
  for (; j + 8 <= cols; j += 8) vmax = _mm256_max_ps(vmax, _mm256_loadu_ps(row + j));
  float block_max = cols >= 8 ? hmax256(vmax) : -INFINITY;
  for (int jj = j; jj < cols; ++jj) block_max = rust_max(block_max, row[jj]);

  const float new_max = rust_max(run_max, block_max);
  const float correction = std::isfinite(run_max) ? std::exp(run_max - new_max) : 0.0f;

  const __m256 vnm = _mm256_set1_ps(new_max);
  __m256 vsum = _mm256_setzero_ps();
  j = 0;
  for (; j + 8 <= cols; j += 8) {
    const __m256 p = exp256(_mm256_sub_ps(_mm256_loadu_ps(row + j), vnm));
    _mm256_storeu_ps(row + j, p);
    vsum = _mm256_add_ps(vsum, p);
  }
  float block_sum = cols >= 8 ? hsum256(vsum) : 0.0f;
  for (int jj = j; jj < cols; ++jj) {
    row[jj] = std::exp(row[jj] - new_max);
    block_sum += row[jj];
  }
  return {new_max, correction, block_sum};
}

// One head of encoder attention: 64-row query blocks x 256-key blocks,
// online softmax, rescale only when the correction is not exactly 1.0, and a
// final 1/run_sum (flash_attn.rs:429-487).  `out_stride` is the distance
// between consecutive query rows of `out`: HD for the head-split layout,
// heads*HD for the merged layout.
__attribute__((target("avx2,fma"))) void flash_head_strided(const float* q, const float* kt,
                                                            const float* v, float* out, int seq,
                                                            int out_stride) {
  std::vector<float> scores(BQ * BK, 0.0f), acc(BQ * HD, 0.0f);
  std::vector<float> run_max(BQ, 0.0f), run_sum(BQ, 0.0f);
  for (int q0 = 0; q0 < seq; q0 += BQ) {
    const int rows = std::min(BQ, seq - q0);
    std::fill(acc.begin(), acc.begin() + rows * HD, 0.0f);
    std::fill(run_max.begin(), run_max.begin() + rows, -INFINITY);
    std::fill(run_sum.begin(), run_sum.begin() + rows, 0.0f);
    const float* qblock = q + static_cast<size_t>(q0) * HD;
    for (int k0 = 0; k0 < seq; k0 += BK) {
      const int cols = std::min(BK, seq - k0);
      scores_tile(qblock, kt, scores.data(), rows, k0, cols, seq);
      for (int i = 0; i < rows; ++i) {
        const SoftmaxStep st = softmax_row(scores.data() + i * BK, cols, run_max[i]);
        run_sum[i] = std::fma(run_sum[i], st.correction, st.block_sum);  // mul_add, :460
        run_max[i] = st.new_max;
        if (st.correction != 1.0f) {  // exact compare on purpose, :462-470
          for (int d = 0; d < HD; ++d) acc[i * HD + d] *= st.correction;
        }
      }
      accum_pv(scores.data(), v, acc.data(), rows, k0, cols);
    }
    for (int i = 0; i < rows; ++i) {
      const float inv = 1.0f / run_sum[i];
      float* o = out + static_cast<size_t>(q0 + i) * out_stride;
      for (int d = 0; d < HD; ++d) o[d] = acc[i * HD + d] * inv;
    }
  }
}

// --- decode kernels (flash_attn.rs:602-789) ---------------------------------

// Shared softmax + PV tail of both decode heads (flash_attn.rs:645-695 and
// :750-788): full-row max, vectorised exp with scalar tail, then o = sum_j
// (s_j * inv) V_j with eight 8-wide accumulators.
template <typename LoadV8>
__attribute__((target("avx2,fma"))) void xattn_softmax_pv(float* s, int keys, float* out,
                                                          LoadV8 load_v8) {
  __m256 vmax = _mm256_set1_ps(-INFINITY);
  int j = 0;
  for (; j + 8 <= keys; j += 8) vmax = _mm256_max_ps(vmax, _mm256_loadu_ps(s + j));
  float mx = keys >= 8 ? hmax256(vmax) : -INFINITY;
  for (int jj = j; jj < keys; ++jj) mx = rust_max(mx, s[jj]);
  const __m256 vmx = _mm256_set1_ps(mx);
  __m256 vsum = _mm256_setzero_ps();
  j = 0;
  for (; j + 8 <= keys; j += 8) {
    const __m256 p = exp256(_mm256_sub_ps(_mm256_loadu_ps(s + j), vmx));
    _mm256_storeu_ps(s + j, p);
    vsum = _mm256_add_ps(vsum, p);
  }
  float sum = keys >= 8 ? hsum256(vsum) : 0.0f;
  for (int jj = j; jj < keys; ++jj) {
    s[jj] = std::exp(s[jj] - mx);
    sum += s[jj];
  }
  const float inv = 1.0f / sum;
  __m256 a[8];
  for (auto& x : a) x = _mm256_setzero_ps();
  for (int jj = 0; jj < keys; ++jj) {
    const __m256 w = _mm256_set1_ps(s[jj] * inv);
    for (int c = 0; c < 8; ++c) a[c] = _mm256_fmadd_ps(w, load_v8(jj, c), a[c]);
  }
  for (int c = 0; c < 8; ++c) _mm256_storeu_ps(out + c * 8, a[c]);
}

// Decode head, f32 cache: scores by AXPY over the head-dim-major K^T
// (flash_attn.rs:602-696).
__attribute__((target("avx2,fma"))) void xattn_head(const float* q, const float* kt,
                                                    const float* v, float* out, int keys,
                                                    float* s) {
  std::fill(s, s + keys, 0.0f);
  for (int t = 0; t < HD; ++t) {
    const __m256 qv = _mm256_set1_ps(q[t]);
    const float* krow = kt + static_cast<size_t>(t) * keys;
    int j = 0;
    for (; j + 8 <= keys; j += 8) {
      _mm256_storeu_ps(s + j, _mm256_fmadd_ps(qv, _mm256_loadu_ps(krow + j), _mm256_loadu_ps(s + j)));
    }
    const float qs = q[t];
    for (int jj = j; jj < keys; ++jj) s[jj] += qs * krow[jj];
  }
  xattn_softmax_pv(s, keys, out, [&](int jj, int c) {
    return _mm256_loadu_ps(v + static_cast<size_t>(jj) * HD + c * 8);
  });
}

// Decode head, f16 cache widened with F16C (flash_attn.rs:714-789).
__attribute__((target("avx2,fma,f16c"))) void xattn_head_f16(const float* q, const uint16_t* kt,
                                                             const uint16_t* v, float* out,
                                                             int keys, float* s) {
  std::fill(s, s + keys, 0.0f);
  for (int t = 0; t < HD; ++t) {
    const __m256 qv = _mm256_set1_ps(q[t]);
    const uint16_t* krow = kt + static_cast<size_t>(t) * keys;
    int j = 0;
    for (; j + 8 <= keys; j += 8) {
      const __m256 kf =
          _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(krow + j)));
      _mm256_storeu_ps(s + j, _mm256_fmadd_ps(qv, kf, _mm256_loadu_ps(s + j)));
    }
    const float qs = q[t];
    for (int jj = j; jj < keys; ++jj) s[jj] += qs * f16_to_f32(krow[jj]);
  }
  xattn_softmax_pv(s, keys, out, [&](int jj, int c) {
    return _mm256_cvtph_ps(
        _mm_loadu_si128(reinterpret_cast<const __m128i*>(v + static_cast<size_t>(jj) * HD + c * 8)));
  });
}

// rayon stand-in: run fn(i) for i in [0, n) on up to `threads` std::threads.
template <typename Fn>
void parallel_for(int n, int threads, Fn fn) {
  if (threads <= 1 || n <= 1) {
    for (int i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int> next{0};
  const int nt = std::min(threads, n);
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (int t = 0; t < nt; ++t) {
    pool.emplace_back([&] {
      for (int i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// Status codes mirror the product ABI: 0 served, 1 declined (the reference's
// Ok(None)), negative = error.
enum { ORA_OK = 0, ORA_DECLINED = 1, ORA_ERR = -1 };

int ora_have_avx2(void) { return have_avx2() ? 1 : 0; }
int ora_have_f16c(void) { return have_f16c() ? 1 : 0; }
int ora_min_decode_keys(void) { return min_decode_keys(); }

// Vectorised exp over n floats (flash_attn.rs:553-572); n must be a multiple of 8.
__attribute__((target("avx2,fma"))) void ora_exp256(const float* x, float* y, int n) {
  for (int i = 0; i + 8 <= n; i += 8) _mm256_storeu_ps(y + i, exp256(_mm256_loadu_ps(x + i)));
}

// One head, any seq >= 1 (the dispatcher's MIN_SEQ floor is a performance
// floor, not a correctness one).  q (seq,64) pre-scaled, kt (64,seq), v
// (seq,64); out rows `out_stride` apart.
void ora_flash_head_strided(const float* q, const float* kt, const float* v, float* out, int seq,
                            int out_stride) {
  flash_head_strided(q, kt, v, out, seq, out_stride);
}

// Many independent heads at once: unit u reads q/kt/v at u*seq*64 and writes
// out at u*seq*64 (head-split).  The units run on `threads` host threads, as
// rayon runs heads in the reference; this is the timed CPU baseline.
void ora_flash_units(const float* q, const float* kt, const float* v, float* out, int units,
                     int seq, int threads) {
  const size_t per = static_cast<size_t>(seq) * HD;
  parallel_for(units, threads, [&](int u) {
    flash_head_strided(q + u * per, kt + u * per, v + u * per, out + u * per, seq, HD);
  });
}

void ora_xattn_head(const float* q, const float* kt, const float* v, float* out, int keys) {
  std::vector<float> s(keys);
  xattn_head(q, kt, v, out, keys, s.data());
}

void ora_xattn_head_f16(const float* q, const uint16_t* kt, const uint16_t* v, float* out,
                        int keys) {
  std::vector<float> s(keys);
  xattn_head_f16(q, kt, v, out, keys, s.data());
}

// Decode rows: `rows` independent (q, K^T, V) triples of one key length each,
// f32 cache.  Row r reads q at r*64, kt at r*64*keys, v at r*keys*64.
void ora_xattn_rows(const float* q, const float* kt, const float* v, float* out, int rows,
                    int keys, int threads) {
  const size_t per = static_cast<size_t>(keys) * HD;
  parallel_for(rows, threads, [&](int r) {
    std::vector<float> s(keys);
    xattn_head(q + r * HD, kt + r * per, v + r * per, out + r * HD, keys, s.data());
  });
}

void ora_xattn_rows_f16(const float* q, const uint16_t* kt, const uint16_t* v, float* out,
                        int rows, int keys, int threads) {
  const size_t per = static_cast<size_t>(keys) * HD;
  parallel_for(rows, threads, [&](int r) {
    std::vector<float> s(keys);
    xattn_head_f16(q + r * HD, kt + r * per, v + r * per, out + r * HD, keys, s.data());
  });
}

// flash_attn::attend + FlashAttnOp::cpu_fwd, f32 operands
// (flash_attn.rs:218-264, :266-413).  Shapes are the reference's: q
// (1,heads,qlen,64), kt (1,heads,64,keys), v (1,heads,keys,64); out
// (1,heads,qlen,64).  Returns ORA_DECLINED where the reference returns
// Ok(None).
int ora_attend(const float* q, const float* kt, const float* v, float* out, int heads, int qlen,
               int keys, int head_dim, int masked, int threads) {
  if (masked || !have_avx2()) return ORA_DECLINED;
  if (head_dim != HD || heads <= 0 || qlen <= 0 || keys < 0) return ORA_DECLINED;
  const int floor = qlen == 1 ? min_decode_keys() : MIN_SEQ;
  if (keys < floor) return ORA_DECLINED;
  if (qlen != 1 && qlen != keys) return ORA_DECLINED;
  if (qlen == 1) {
    // Decode step: heads serial by default (flash_attn.rs:370-399); the
    // FFAI_PAR_HEADS knob fans them out, which `threads` stands in for.
    ora_xattn_rows(q, kt, v, out, heads, keys, threads);
  } else {
    ora_flash_units(q, kt, v, out, heads, keys, threads);
  }
  return ORA_OK;
}

// The f16 K/V decode branch of FlashAttnOp::cpu_fwd (flash_attn.rs:289-356).
int ora_attend_f16kv(const float* q, const uint16_t* kt, const uint16_t* v, float* out, int heads,
                     int qlen, int keys, int head_dim, int masked, int threads) {
  if (masked || !have_avx2() || !have_f16c()) return ORA_DECLINED;
  if (head_dim != HD || heads <= 0 || qlen != 1) return ORA_DECLINED;
  if (keys < min_decode_keys()) return ORA_DECLINED;
  ora_xattn_rows_f16(q, kt, v, out, heads, keys, threads);
  return ORA_OK;
}

// flash_attn::attend_merged + MergedAttnOp::cpu_fwd (flash_attn.rs:135-210):
// output (1, seq, heads*64), each head writing its own column band.
int ora_attend_merged(const float* q, const float* kt, const float* v, float* out, int heads,
                      int qlen, int keys, int head_dim, int threads) {
  if (head_dim != HD || !have_avx2() || heads <= 0) return ORA_DECLINED;
  if (qlen != keys || keys < MIN_SEQ) return ORA_DECLINED;
  const int seq = keys;
  const size_t per = static_cast<size_t>(seq) * HD;
  const int width = heads * HD;
  parallel_for(heads, threads, [&](int h) {
    flash_head_strided(q + h * per, kt + h * per, v + h * per, out + h * HD, seq, width);
  });
  return ORA_OK;
}

// flash_attn::serves (flash_attn.rs:104-129): kt (1,h1,64,keys), v (1,h2,k2,64).
int ora_serves(int kt_b, int kt_h, int kt_d, int kt_keys, int v_b, int v_h, int v_keys, int v_d) {
  if (!have_avx2()) return 0;
  if (kt_b != 1 || kt_d != HD || v_b != 1 || v_d != HD) return 0;
  return (kt_h == v_h && kt_keys == v_keys && kt_keys >= std::max(MIN_SEQ, min_decode_keys())) ? 1
                                                                                               : 0;
}

// The three-op path the reference's test compares against
// (flash_attn.rs:1016): softmax_last_dim(q @ kt) @ v, all f32, per head.
// Plain loops: this is the comparator, not a restatement of candle's GEMM.
void ora_three_op(const float* q, const float* kt, const float* v, float* out, int heads, int qlen,
                  int keys) {
  std::vector<float> row(keys);
  for (int h = 0; h < heads; ++h) {
    const float* qh = q + static_cast<size_t>(h) * qlen * HD;
    const float* kh = kt + static_cast<size_t>(h) * HD * keys;
    const float* vh = v + static_cast<size_t>(h) * keys * HD;
    float* oh = out + static_cast<size_t>(h) * qlen * HD;
    for (int i = 0; i < qlen; ++i) {
      float mx = -INFINITY;
      for (int j = 0; j < keys; ++j) {
        float a = 0.0f;
        for (int t = 0; t < HD; ++t) a += qh[i * HD + t] * kh[static_cast<size_t>(t) * keys + j];
        row[j] = a;
        mx = std::max(mx, a);
      }
      float sum = 0.0f;
      for (int j = 0; j < keys; ++j) {
        row[j] = std::exp(row[j] - mx);
        sum += row[j];
      }
      for (int j = 0; j < keys; ++j) row[j] /= sum;
      for (int d = 0; d < HD; ++d) {
        float a = 0.0f;
        for (int j = 0; j < keys; ++j) a += row[j] * vh[static_cast<size_t>(j) * HD + d];
        oh[i * HD + d] = a;
      }
    }
  }
}

}  // extern "C"
