// C ABI of libffai_attn.so: argument checking (the reference's "decline"
// contract), per-device context and workspace, tensor-map encoding, work
// lists, kernel dispatch, the host-buffer pipeline, and the mirror of the
// reference's candle custom-op surface (crates/ffai-mercury/src/asr/
// flash_attn.rs).
#include <cudaTypedefs.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/ffai_attn.h"
#include "kernels.h"

using namespace ffai;

namespace {

constexpr int kHD = 64;
constexpr int kMinSeq = 256;  // flash_attn.rs:55, performance floor of the encoder shape

thread_local std::string g_tls_error;
thread_local int g_tls_status = FFAI_ATTN_OK;

// FFAI_DECODE_MIN_KEYS (knobs.rs:163-168, default 8): the decode floor the
// reference's `serves` and `attend` share (flash_attn.rs:65-67, :112-128).
int min_decode_keys() {
  const char* s = std::getenv("FFAI_DECODE_MIN_KEYS");
  if (s && *s) {
    char* end = nullptr;
    const long v = std::strtol(s, &end, 10);
    if (end && *end == 0 && v >= 0) return static_cast<int>(v);
  }
  return 8;
}

bool env_on(const char* name) {
  const char* s = std::getenv(name);
  return s && (!std::strcmp(s, "1") || !std::strcmp(s, "on") || !std::strcmp(s, "true"));
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

size_t dtype_size(int dt) { return dt == FFAI_DT_F32 ? 4 : 2; }

}  // namespace

struct ffai_attn_ctx {
  int device = 0;
  int num_sms = 148;
  unsigned* d_err = nullptr;
  // decode workspace
  float* d_part = nullptr;
  size_t part_cap = 0;  // floats
  unsigned* d_counters = nullptr;
  size_t counters_cap = 0;
  // prefill work list and per-sequence arrays
  int4* d_units = nullptr;
  size_t units_cap = 0;
  int* d_seq = nullptr;  // q_start | q_len | k_start | k_len, each seq_cap long
  size_t seq_cap = 0;
  std::vector<long long> wl_key;
  int wl_units = 0;
  int wl_seqs = 0;
  // bf16 staging for f32 or K^T operands
  void* d_stage = nullptr;
  size_t stage_cap = 0;
  // host pipeline
  cudaStream_t s_h2d = nullptr, s_comp = nullptr, s_d2h = nullptr;
  cudaEvent_t ev_h2d[2] = {}, ev_comp[2] = {}, ev_d2h[2] = {};
  void* d_pipe = nullptr;
  size_t pipe_cap = 0;
  // int8 GEMV: quantised activations and their scales, between its two kernels
  uint8_t* d_gemv_x = nullptr;
  size_t gemv_x_cap = 0;
  ffai_attn_ctx* pipe_ctx = nullptr;  // inner context used for the pipeline's kernels
  std::string last_error;
  int last_status = FFAI_ATTN_OK;
  // opt-in launch timing (FFAI_ATTN_PROFILE=1 or ffai_attn_profile): CUDA
  // events around each prefill / decode / varlen call, and NVTX ranges
  struct ProfRec {
    int op;
    cudaEvent_t a, b;
  };
  bool prof = false;
  std::vector<ProfRec> prof_pending;
  double prof_ms[3] = {0, 0, 0};
  long long prof_n[3] = {0, 0, 0};
};

namespace {

int set_error(const ffai_attn_ctx* ctx, int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx) {
    auto* c = const_cast<ffai_attn_ctx*>(ctx);
    c->last_error = buf;
    c->last_status = status;
  }
  g_tls_error = buf;
  g_tls_status = status;
  return status;
}

int cuda_fail(const ffai_attn_ctx* ctx, cudaError_t e, const char* what) {
  return set_error(ctx, FFAI_ATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define FFAI_CUDA(ctx, call)                                \
  do {                                                      \
    cudaError_t e_ = (call);                                \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
  } while (0)

// Makes ctx->device current for the duration of a call and restores the
// caller's device afterwards.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

template <typename T>
int ensure(ffai_attn_ctx* ctx, T** ptr, size_t* cap, size_t need_elems, bool zero = false) {
  if (*cap >= need_elems && *ptr) return FFAI_ATTN_OK;
  if (*ptr) {
    cudaDeviceSynchronize();  // the old buffer may still be read by queued work
    cudaFree(*ptr);
    *ptr = nullptr;
    *cap = 0;
  }
  size_t n = std::max<size_t>(need_elems, 1);
  n = n + n / 4;  // growth slack
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(ptr), n * sizeof(T));
  if (e != cudaSuccess) {
    *ptr = nullptr;
    return set_error(ctx, FFAI_ATTN_ERR_NOMEM, "workspace allocation of %zu bytes failed: %s",
                     n * sizeof(T), cudaGetErrorString(e));
  }
  if (zero) {
    e = cudaMemset(*ptr, 0, n * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemset(workspace)");
  }
  *cap = n;
  return FFAI_ATTN_OK;
}

bool valid_dtype(int dt) { return dt == FFAI_DT_F32 || dt == FFAI_DT_BF16 || dt == FFAI_DT_F16; }

// Shape/dtype gate shared by every entry point.  Returns OK, DECLINED (a
// well-formed request this library does not serve) or ERR_INVALID, with a
// message.
int check_desc(const ffai_attn_ctx* ctx, const ffai_attn_desc* d, int op) {
  if (!d) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null descriptor");
  if (d->head_dim != kHD)
    return set_error(ctx, FFAI_ATTN_DECLINED, "head_dim %d: only 64 is served", d->head_dim);
  if (d->heads <= 0) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "heads %d <= 0", d->heads);
  if (!valid_dtype(d->q_dtype) || !valid_dtype(d->kv_dtype))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "unknown dtype (q %d, kv %d)", d->q_dtype,
                     d->kv_dtype);
  if (d->out_dtype != FFAI_DT_F32 && d->out_dtype != FFAI_DT_BF16)
    return set_error(ctx, FFAI_ATTN_DECLINED, "out_dtype %d: f32 or bf16 only", d->out_dtype);
  if (!(d->scale > 0.f) || !std::isfinite(d->scale))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "scale must be finite and > 0");
  if (d->token_stride != 0 &&
      (d->token_stride < d->heads * kHD || d->token_stride % 8 != 0))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID,
                     "token_stride %d: 0, or a multiple of 8 of at least heads * 64",
                     d->token_stride);
  if (op == FFAI_OP_VARLEN) {
    if (d->q_layout != FFAI_LAYOUT_TOKEN_MAJOR || d->k_layout != FFAI_LAYOUT_TOKEN_MAJOR ||
        d->v_layout != FFAI_LAYOUT_TOKEN_MAJOR || d->out_layout != FFAI_LAYOUT_TOKEN_MAJOR)
      return set_error(ctx, FFAI_ATTN_DECLINED, "varlen: token-major (T,H,64) layouts only");
    if (d->q_dtype != d->kv_dtype || d->q_dtype == FFAI_DT_F32)
      return set_error(ctx, FFAI_ATTN_DECLINED, "varlen: bf16 or f16 q/k/v of one type only");
    if (d->causal) return set_error(ctx, FFAI_ATTN_DECLINED, "varlen: causal not served");
    return FFAI_ATTN_OK;
  }
  if (d->batch <= 0 || d->q_len <= 0 || d->kv_len <= 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "batch %d, q_len %d, kv_len %d must be >= 1",
                     d->batch, d->q_len, d->kv_len);
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : d->kv_len;
  if (cap < d->kv_len)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "kv_capacity %d < kv_len %d", cap, d->kv_len);
  if (d->q_layout == FFAI_LAYOUT_KT || d->v_layout == FFAI_LAYOUT_KT ||
      d->out_layout == FFAI_LAYOUT_KT)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "only k may use the KT layout");
  auto layout_ok = [](int l) { return l >= 0 && l <= 2; };
  if (!layout_ok(d->q_layout) || !layout_ok(d->k_layout) || !layout_ok(d->v_layout) ||
      !layout_ok(d->out_layout))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "unknown layout");
  if (d->causal && (d->q_offset < 0))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "causal q_offset %d < 0", d->q_offset);

  if (op == FFAI_OP_DECODE) {
    if (d->q_len != 1) return set_error(ctx, FFAI_ATTN_DECLINED, "decode: q_len must be 1");
    if (d->q_dtype != FFAI_DT_F32 && d->q_dtype != d->kv_dtype)
      return set_error(ctx, FFAI_ATTN_DECLINED, "decode: q must be f32 or the cache dtype");
    if (d->k_layout == FFAI_LAYOUT_TOKEN_MAJOR || d->v_layout != FFAI_LAYOUT_HEADS_SPLIT)
      return set_error(ctx, FFAI_ATTN_DECLINED,
                       "decode: k must be KT or heads-split, v heads-split");
    // The decode kernels address q and out as dense (row, 64) rows.
    if (d->token_stride != 0)
      return set_error(ctx, FFAI_ATTN_DECLINED, "decode: dense q and out only (token_stride 0)");
    return FFAI_ATTN_OK;
  }
  // prefill
  if (d->q_dtype != d->kv_dtype)
    return set_error(ctx, FFAI_ATTN_DECLINED, "prefill: q and k/v must share a dtype");
  const bool checked = (d->flags & FFAI_ATTN_FLAG_CHECKED_F32) != 0;
  if (checked && d->q_dtype != FFAI_DT_F32)
    return set_error(ctx, FFAI_ATTN_DECLINED, "checked-f32 mode needs f32 operands");
  if (d->causal && d->q_offset < 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "causal q_offset %d < 0", d->q_offset);
  return FFAI_ATTN_OK;
}

// Element strides (b, h, row, d) of an operand of `rows` rows per head.
// token_stride: elements between tokens of a TOKEN_MAJOR operand (0: dense).
Strides strides_of(int layout, int H, long long rows, long long token_stride = 0) {
  Strides s{};
  const long long ts = token_stride > 0 ? token_stride : static_cast<long long>(H) * kHD;
  switch (layout) {
    case FFAI_LAYOUT_HEADS_SPLIT:
      s = {H * rows * kHD, rows * kHD, kHD, 1};
      break;
    case FFAI_LAYOUT_TOKEN_MAJOR:
      s = {rows * ts, kHD, ts, 1};
      break;
    case FFAI_LAYOUT_KT:
      s = {H * rows * kHD, rows * kHD, 1, rows};
      break;
  }
  return s;
}

void init_encoder() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

// 3-d bf16/f16 tensor map over 64-element (128-byte) rows with a box of 128
// rows and 128-byte swizzle.  token_major: dims {64, H, T}; else {64, rows, B*H}.
int make_map(ffai_attn_ctx* ctx, CUtensorMap* map, const void* base, bool token_major, int H,
             long long rows_or_tokens, long long groups, long long token_stride = 0,
             int box_rows = kTcRows) {
  if (!g_encode) return set_error(ctx, FFAI_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "operand base address not 16-byte aligned");
  cuuint64_t dims[3];
  cuuint64_t strides[2];
  cuuint32_t box[3];
  const cuuint32_t estr[3] = {1, 1, 1};
  if (token_major) {
    dims[0] = kHD;
    dims[1] = static_cast<cuuint64_t>(H);
    dims[2] = static_cast<cuuint64_t>(rows_or_tokens);
    strides[0] = kHD * 2;
    strides[1] = static_cast<cuuint64_t>(token_stride > 0 ? token_stride : H * kHD) * 2;
    box[0] = kHD;
    box[1] = 1;
    box[2] = static_cast<cuuint32_t>(box_rows);
  } else {
    dims[0] = kHD;
    dims[1] = static_cast<cuuint64_t>(rows_or_tokens);
    dims[2] = static_cast<cuuint64_t>(groups);
    strides[0] = kHD * 2;
    strides[1] = static_cast<cuuint64_t>(rows_or_tokens) * kHD * 2;
    box[0] = kHD;
    box[1] = static_cast<cuuint32_t>(box_rows);
    box[2] = 1;
  }
  // The data type only sets the element size here (both are 2 bytes).
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, FFAI_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled: %d", r);
  return FFAI_ATTN_OK;
}

// Build (or reuse) the device work list: per-sequence offsets/lengths and
// units of up to 256 query rows, longest sequences first.
// keep_tail: leave a short last wave of two-tile units as it is (the caller
// launches back to back with stable inputs, so the next launch fills it).
int prepare_work(ffai_attn_ctx* ctx, const std::vector<int>& q_start, const std::vector<int>& q_len,
                 const std::vector<int>& k_start, const std::vector<int>& k_len, int H,
                 cudaStream_t s, int causal = 0, int q_offset = 0, bool keep_tail = false) {
  const int nseq = static_cast<int>(q_len.size());
  std::vector<long long> key;
  key.reserve(4 * nseq + 5);
  key.push_back(H);
  key.push_back(nseq);
  key.push_back(causal);
  key.push_back(causal ? q_offset : 0);
  key.push_back(keep_tail);
  for (int i = 0; i < nseq; ++i) {
    key.push_back(q_start[i]);
    key.push_back(q_len[i]);
    key.push_back(k_start[i]);
    key.push_back(k_len[i]);
  }
  if (key == ctx->wl_key && ctx->d_units) return FFAI_ATTN_OK;

  std::vector<int> order(nseq);
  for (int i = 0; i < nseq; ++i) order[i] = i;
  // Longest-processing-time first: cost ~ q_len * k_len.  Stable, so equal
  // sequences keep their natural order (adjacent units share K/V in L2).
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return static_cast<long long>(q_len[a]) * k_len[a] > static_cast<long long>(q_len[b]) * k_len[b];
  });
  std::vector<int4> units;
  for (int si : order) {
    for (int h = 0; h < H; ++h) {
      for (int r0 = 0; r0 < q_len[si]; r0 += 2 * kTcRows) {
        const int left = q_len[si] - r0;
        units.push_back(make_int4(si, h, r0, left > kTcRows ? 2 : 1));
      }
    }
  }
  if (causal) {
    // Causal units differ in cost (key blocks of their tiles): longest first.
    auto cost = [&](const int4& u) {
      return tc_tile_blocks(1, q_offset, q_len[u.x], k_len[u.x], u.z, u.w, 0) +
             tc_tile_blocks(1, q_offset, q_len[u.x], k_len[u.x], u.z, u.w, 1);
    };
    std::stable_sort(units.begin(), units.end(),
                     [&](const int4& a, const int4& b) { return cost(a) > cost(b); });
  }
  // Persistent CTAs take units u, u + G, u + 2G, ...: a last wave of r < G / 2
  // units leaves most SMs idle while r finish.  Splitting those r two-tile
  // units into 2r one-tile units (at the end of the list, so the full waves
  // keep their CTAs) lets the last wave finish in about the time of one tile.
  const long long G = std::min<long long>(static_cast<long long>(units.size()), ctx->num_sms);
  if (2 * static_cast<long long>(units.size()) <= ctx->num_sms) {
    // A batch too small for one wave (the single 6-head window of a small
    // Whisper): one-tile units put twice as many SMs to work.
    std::vector<int4> all;
    all.swap(units);
    for (const int4& t : all) {
      units.push_back(make_int4(t.x, t.y, t.z, 1));
      if (t.w == 2) units.push_back(make_int4(t.x, t.y, t.z + kTcRows, 1));
    }
  } else if (!keep_tail && G > 0 && static_cast<long long>(units.size()) > G) {
    const long long r = static_cast<long long>(units.size()) % G;
    if (r > 0 && 2 * r <= G) {
      std::vector<int4> tail(units.end() - r, units.end());
      units.resize(units.size() - r);
      for (const int4& t : tail) {
        if (t.w == 2) {
          units.push_back(make_int4(t.x, t.y, t.z, 1));
          units.push_back(make_int4(t.x, t.y, t.z + kTcRows, 1));
        } else {
          units.push_back(t);
        }
      }
    }
  }
  int st = ensure(ctx, &ctx->d_units, &ctx->units_cap, units.size());
  if (st) return st;
  st = ensure(ctx, &ctx->d_seq, &ctx->seq_cap, 4 * static_cast<size_t>(nseq));
  if (st) return st;
  std::vector<int> seq(4 * static_cast<size_t>(nseq));
  for (int i = 0; i < nseq; ++i) {
    seq[i] = q_start[i];
    seq[nseq + i] = q_len[i];
    seq[2 * nseq + i] = k_start[i];
    seq[3 * nseq + i] = k_len[i];
  }
  FFAI_CUDA(ctx, cudaMemcpyAsync(ctx->d_units, units.data(), units.size() * sizeof(int4),
                                 cudaMemcpyHostToDevice, s));
  FFAI_CUDA(ctx, cudaMemcpyAsync(ctx->d_seq, seq.data(), seq.size() * sizeof(int),
                                 cudaMemcpyHostToDevice, s));
  // Pageable sources: the copies are staged before these calls return.
  ctx->wl_key.swap(key);
  ctx->wl_units = static_cast<int>(units.size());
  ctx->wl_seqs = nseq;
  return FFAI_ATTN_OK;
}

// One TMA operand: base pointer, layout, and the map geometry (rows per
// (sequence, head) and head groups for heads-split; tokens for token-major).
struct Operand {
  const void* ptr;
  bool token_major;
  long long rows;
  long long groups;
  long long token_stride = 0;  // token-major: elements between tokens (0: dense)
};

int run_tc(ffai_attn_ctx* ctx, const Operand& q, const Operand& k, const Operand& v, int H,
           int ab_f16, void* o, int out_bf16, bool out_tm, long long out_rows, float* lse,
           long long lse_tokens, float scale, cudaStream_t s, int causal = 0, int q_offset = 0,
           bool inputs_stable = false) {
  if (reinterpret_cast<uintptr_t>(o) % 8 != 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "prefill output must be 8-byte aligned");
  CUtensorMap tq, tk, tv;
  int st = make_map(ctx, &tq, q.ptr, q.token_major, H, q.rows, q.groups, q.token_stride);
  if (st) return st;
  st = make_map(ctx, &tk, k.ptr, k.token_major, H, k.rows, k.groups, k.token_stride);
  if (st) return st;
  st = make_map(ctx, &tv, v.ptr, v.token_major, H, v.rows, v.groups, v.token_stride);
  if (st) return st;
  // bf16 output: a map of 16-row boxes for the kernel's TMA-store epilogue.
  CUtensorMap to = tq;
  const bool o_tma = out_bf16 && reinterpret_cast<uintptr_t>(o) % 16 == 0;
  if (o_tma) {
    st = out_tm ? make_map(ctx, &to, o, true, H, lse_tokens, 1, 0, 16)
                : make_map(ctx, &to, o, false, H, out_rows, q.groups, 0, 16);
    if (st) return st;
  }
  TcParams p{};
  p.units = ctx->d_units;
  p.num_units = ctx->wl_units;
  p.q_start = ctx->d_seq;
  p.q_len = ctx->d_seq + ctx->wl_seqs;
  p.k_start = ctx->d_seq + 2 * ctx->wl_seqs;
  p.k_len = ctx->d_seq + 3 * ctx->wl_seqs;
  p.heads = H;
  p.q_token_major = q.token_major;
  p.k_token_major = k.token_major;
  p.v_token_major = v.token_major;
  p.out = o;
  p.out_bf16 = out_bf16;
  p.out_token_major = out_tm;
  p.out_rows = out_rows;
  p.lse = lse;
  p.lse_tokens = lse_tokens;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = ctx->d_err;
  p.causal = causal;
  p.q_offset = q_offset;
  p.o_tma = o_tma ? 1 : 0;
  p.inputs_stable = inputs_stable ? 1 : 0;
  const int grid = std::min(ctx->wl_units, ctx->num_sms);
  if (grid <= 0) return FFAI_ATTN_OK;
  FFAI_CUDA(ctx, launch_prefill_tc(tq, tk, tv, to, p, grid, ab_f16, s));
  return FFAI_ATTN_OK;
}

int prefill_impl(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                 const void* v, void* o, float* lse, cudaStream_t s) {
  const int B = d->batch, H = d->heads, Nq = d->q_len, Nk = d->kv_len;
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : Nk;
  const bool out_tm = d->out_layout == FFAI_LAYOUT_TOKEN_MAJOR;

  if (d->flags & FFAI_ATTN_FLAG_CHECKED_F32) {
    SimtParams p{};
    p.q = static_cast<const float*>(q);
    p.k = static_cast<const float*>(k);
    p.v = static_cast<const float*>(v);
    p.out = o;
    p.lse = lse;
    p.qs = strides_of(d->q_layout, H, Nq, d->token_stride);
    p.ks = strides_of(d->k_layout, H, cap, d->token_stride);
    p.vs = strides_of(d->v_layout, H, cap, d->token_stride);
    p.os = strides_of(d->out_layout, H, Nq);
    if (out_tm) {
      p.lse_sb = Nq;
      p.lse_sh = static_cast<long long>(B) * Nq;
    } else {
      p.lse_sb = static_cast<long long>(H) * Nq;
      p.lse_sh = Nq;
    }
    p.B = B;
    p.H = H;
    p.Nq = Nq;
    p.Nk = Nk;
    p.out_dtype = d->out_dtype;
    p.causal = d->causal;
    p.q_offset = d->q_offset;
    p.scale = d->scale;
    FFAI_CUDA(ctx, launch_prefill_simt(p, s));
    return FFAI_ATTN_OK;
  }

  // Tensor-core path: operands must be 16-bit in heads-split or token-major
  // layout.  f32 operands are gathered into bf16 staging; K^T (whose row
  // pitch TMA cannot describe in general) is gathered into heads-split rows
  // of its own 16-bit type.
  const bool f32 = d->q_dtype == FFAI_DT_F32;
  const int dt16 = f32 ? FFAI_DT_BF16 : d->q_dtype;
  const bool stage_q = f32;
  const bool stage_k = f32 || d->k_layout == FFAI_LAYOUT_KT;
  const bool stage_v = f32;
  const size_t q_elems = static_cast<size_t>(B) * H * Nq * kHD;
  const size_t kv_elems = static_cast<size_t>(B) * H * Nk * kHD;
  const size_t stage = (stage_q ? q_elems : 0) + (stage_k ? kv_elems : 0) + (stage_v ? kv_elems : 0);
  const void *qq = q, *kk = k, *vv = v;
  bool q_tm = d->q_layout == FFAI_LAYOUT_TOKEN_MAJOR;
  bool k_tm = d->k_layout == FFAI_LAYOUT_TOKEN_MAJOR;
  bool v_tm = d->v_layout == FFAI_LAYOUT_TOKEN_MAJOR;
  int kcap = cap, vcap = cap;
  if (stage) {
    int st = ensure(ctx, reinterpret_cast<uint16_t**>(&ctx->d_stage), &ctx->stage_cap, stage);
    if (st) return st;
    uint16_t* base = static_cast<uint16_t*>(ctx->d_stage);
    // One launch converts every staged operand.
    StageBatch sb{};
    sb.B = B;
    sb.H = H;
    if (stage_q) {
      sb.op[sb.n++] = StageOp{q, d->q_dtype, strides_of(d->q_layout, H, Nq, d->token_stride), Nq,
                              base, 0, 0};
      qq = base;
      q_tm = false;
      base += q_elems;
    }
    if (stage_k) {
      sb.op[sb.n++] = StageOp{k, d->kv_dtype, strides_of(d->k_layout, H, cap, d->token_stride), Nk,
                              base, 0, 0};
      kk = base;
      k_tm = false;
      kcap = Nk;
      base += kv_elems;
    }
    if (stage_v) {
      sb.op[sb.n++] = StageOp{v, d->kv_dtype, strides_of(d->v_layout, H, cap, d->token_stride), Nk,
                              base, 0, 0};
      vv = base;
      v_tm = false;
      vcap = Nk;
    }
    FFAI_CUDA(ctx, launch_stage_batch(sb, dt16 == FFAI_DT_F16, s));
  }
  const int ab_f16 = dt16 == FFAI_DT_F16;

  std::vector<int> qs(B), ql(B, Nq), ks(B), kl(B, Nk);
  for (int b = 0; b < B; ++b) {
    qs[b] = b * Nq;
    ks[b] = b * cap;  // token-major K/V are never staged, so they keep `cap`
  }
  // Staged operands are written by the staging kernels just before.
  const bool stable = (d->flags & FFAI_ATTN_FLAG_INPUTS_STABLE) && !stage;
  int st = prepare_work(ctx, qs, ql, ks, kl, H, s, d->causal, d->q_offset, stable);
  if (st) return st;
  const long long BH = static_cast<long long>(B) * H;
  Operand oq{qq, q_tm, q_tm ? static_cast<long long>(B) * Nq : Nq, BH, d->token_stride};
  Operand ok{kk, k_tm, k_tm ? static_cast<long long>(B) * kcap : kcap, BH, d->token_stride};
  Operand ov{vv, v_tm, v_tm ? static_cast<long long>(B) * vcap : vcap, BH, d->token_stride};
  return run_tc(ctx, oq, ok, ov, H, ab_f16, o, d->out_dtype == FFAI_DT_BF16,
                d->out_layout == FFAI_LAYOUT_TOKEN_MAJOR, Nq, lse, static_cast<long long>(B) * Nq,
                d->scale, s, d->causal, d->q_offset, stable);
}

int decode_impl(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                const void* v, void* o, float* lse, int num_splits, cudaStream_t s,
                const void* pf_k = nullptr, const void* pf_v = nullptr) {
  const int rows = d->batch * d->heads;
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : d->kv_len;
  int kv = d->kv_len;
  if (d->causal) kv = std::min(kv, d->q_offset + 1);
  if (kv <= 0) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "no visible keys");
  for (const void* ptr : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "decode operands must be 16-byte aligned");
  if (num_splits == 0 && d->k_layout != FFAI_LAYOUT_KT &&
      static_cast<long long>(rows) * kDecodeMaxCluster >= ctx->num_sms) {
    // Row-major cache with enough rows to fill the GPU: the cluster kernel.
    // Two CTAs per SM; each row split over S <= 8 CTAs of one cluster, with
    // at least 16 keys per CTA.
    int S = static_cast<int>(std::min<long long>(kDecodeMaxCluster, 2LL * ctx->num_sms / rows));
    S = std::max(1, std::min(S, (kv + 15) / 16));
    const int kpc = (kv + S - 1) / S;
    DecodeParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.out = o;
    p.lse = lse;
    p.rows = rows;
    p.kv_len = kv;
    p.cap = cap;
    p.q_dtype = d->q_dtype;
    p.kv_dtype = d->kv_dtype;
    p.out_dtype = d->out_dtype;
    p.scale_log2 = d->scale * 1.4426950408889634f;
    p.err = ctx->d_err;
    p.kv_stable = (d->flags & FFAI_ATTN_FLAG_KV_STABLE) != 0;
    p.kv_append_only = !p.kv_stable && (d->flags & FFAI_ATTN_FLAG_KV_APPEND_ONLY) != 0;
    p.pf_k = pf_k;
    p.pf_v = pf_v;
    FFAI_CUDA(ctx, launch_decode_cluster(p, S, kpc, s));
    return FFAI_ATTN_OK;
  }
  int chunk;
  if (num_splits > 0) {
    chunk = (kv + num_splits - 1) / num_splits;
    chunk = std::min(std::max(chunk, 1), 128);
  } else {
    chunk = d->kv_dtype == FFAI_DT_F32 ? 64 : 128;
    const int splits128 = (kv + chunk - 1) / chunk;
    if (chunk == 128 && static_cast<long long>(rows) * splits128 < 2LL * ctx->num_sms && kv > 64)
      chunk = 64;
  }
  const int splits = (kv + chunk - 1) / chunk;
  DecodeParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = o;
  p.lse = lse;
  p.rows = rows;
  p.kv_len = kv;
  p.cap = cap;
  p.chunk = chunk;
  p.splits = splits;
  p.q_dtype = d->q_dtype;
  p.kv_dtype = d->kv_dtype;
  p.out_dtype = d->out_dtype;
  p.k_kt = d->k_layout == FFAI_LAYOUT_KT;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.err = ctx->d_err;
  if (splits > 1) {
    int st = ensure(ctx, &ctx->d_part, &ctx->part_cap,
                    static_cast<size_t>(rows) * splits * kPartStride);
    if (st) return st;
    st = ensure(ctx, &ctx->d_counters, &ctx->counters_cap, static_cast<size_t>(rows), true);
    if (st) return st;
    p.part = ctx->d_part;
    p.counters = ctx->d_counters;
  }
  FFAI_CUDA(ctx, launch_decode(p, s));
  return FFAI_ATTN_OK;
}

}  // namespace

extern "C" {

const char* ffai_attn_version(void) { return "ffai-attn-b200 1 sm_100a"; }

void ffai_attn_desc_init(ffai_attn_desc* d) {
  if (!d) return;
  std::memset(d, 0, sizeof *d);
  d->batch = 1;
  d->heads = 1;
  d->q_len = 1;
  d->kv_len = 1;
  d->head_dim = kHD;
  d->q_dtype = d->kv_dtype = d->out_dtype = FFAI_DT_F32;
  d->q_layout = d->k_layout = d->v_layout = d->out_layout = FFAI_LAYOUT_HEADS_SPLIT;
  d->scale = 1.0f;
}

int ffai_attn_check(const ffai_attn_desc* d, int op) {
  if (op < FFAI_OP_PREFILL || op > FFAI_OP_VARLEN)
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "unknown op %d", op);
  return check_desc(nullptr, d, op);
}

ffai_attn_ctx* ffai_attn_create(int device, int* status) {
  auto fail = [&](int st) -> ffai_attn_ctx* {
    if (status) *status = st;
    return nullptr;
  };
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    set_error(nullptr, FFAI_ATTN_ERR_NO_DEVICE, "no CUDA device");
    return fail(FFAI_ATTN_ERR_NO_DEVICE);
  }
  if (device < 0 || device >= n) {
    set_error(nullptr, FFAI_ATTN_ERR_INVALID, "device %d out of range [0,%d)", device, n);
    return fail(FFAI_ATTN_ERR_INVALID);
  }
  DeviceGuard g(device);
  if (!g.ok) {
    set_error(nullptr, FFAI_ATTN_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    return fail(FFAI_ATTN_ERR_CUDA);
  }
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
    set_error(nullptr, FFAI_ATTN_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is sm_100a",
              device, prop.major, prop.minor);
    return fail(FFAI_ATTN_ERR_NO_DEVICE);
  }
  std::call_once(g_encode_once, init_encoder);
  auto* ctx = new ffai_attn_ctx();
  ctx->device = device;
  ctx->prof = env_on("FFAI_ATTN_PROFILE");
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaMalloc(&ctx->d_err, sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(ctx->d_err, 0, sizeof(unsigned)) != cudaSuccess) {
    delete ctx;
    set_error(nullptr, FFAI_ATTN_ERR_NOMEM, "error word allocation failed");
    return fail(FFAI_ATTN_ERR_NOMEM);
  }
  if (status) *status = FFAI_ATTN_OK;
  return ctx;
}

void ffai_attn_destroy(ffai_attn_ctx* ctx) {
  if (!ctx) return;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->pipe_ctx) ffai_attn_destroy(ctx->pipe_ctx);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_part);
  cudaFree(ctx->d_counters);
  cudaFree(ctx->d_units);
  cudaFree(ctx->d_seq);
  cudaFree(ctx->d_stage);
  cudaFree(ctx->d_pipe);
  cudaFree(ctx->d_gemv_x);
  for (int i = 0; i < 2; ++i) {
    if (ctx->ev_h2d[i]) cudaEventDestroy(ctx->ev_h2d[i]);
    if (ctx->ev_comp[i]) cudaEventDestroy(ctx->ev_comp[i]);
    if (ctx->ev_d2h[i]) cudaEventDestroy(ctx->ev_d2h[i]);
  }
  if (ctx->s_h2d) cudaStreamDestroy(ctx->s_h2d);
  if (ctx->s_comp) cudaStreamDestroy(ctx->s_comp);
  if (ctx->s_d2h) cudaStreamDestroy(ctx->s_d2h);
  for (auto& r : ctx->prof_pending) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  delete ctx;
}

}  // extern "C"

namespace {

// Brackets one entry-point call with CUDA events (on its stream) and an NVTX
// range when the context's profiling is on; otherwise does nothing.
struct ProfScope {
  ffai_attn_ctx* ctx;
  int op;
  cudaStream_t s;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(ffai_attn_ctx* c, int o, cudaStream_t st, const char* name) : ctx(c), op(o), s(st) {
    if (!ctx->prof) return;
    nvtxRangePushA(name);
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess ||
        cudaEventRecord(a, s) != cudaSuccess) {
      if (a) cudaEventDestroy(a);
      if (b) cudaEventDestroy(b);
      a = b = nullptr;
    }
  }
  ~ProfScope() {
    if (!ctx->prof) return;
    if (a && cudaEventRecord(b, s) == cudaSuccess) {
      ctx->prof_pending.push_back({op, a, b});
    } else {
      if (a) cudaEventDestroy(a);
      if (b) cudaEventDestroy(b);
    }
    nvtxRangePop();
  }
};

}  // namespace

extern "C" {

int ffai_attn_profile(ffai_attn_ctx* ctx, int32_t enable, double* ms, int64_t* launches) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  DeviceGuard g(ctx->device);
  if (ms || launches) {
    for (auto& r : ctx->prof_pending) {
      float t = 0.f;
      if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess) {
        ctx->prof_ms[r.op] += t;
        ctx->prof_n[r.op] += 1;
      }
      cudaEventDestroy(r.a);
      cudaEventDestroy(r.b);
    }
    ctx->prof_pending.clear();
    for (int i = 0; i < 3; ++i) {
      if (ms) ms[i] = ctx->prof_ms[i];
      if (launches) launches[i] = ctx->prof_n[i];
      ctx->prof_ms[i] = 0;
      ctx->prof_n[i] = 0;
    }
  }
  if (enable >= 0) ctx->prof = enable != 0;
  return FFAI_ATTN_OK;
}

int ffai_attn_prefill(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                      const void* v, void* o, float* lse, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  const int st = check_desc(ctx, d, FFAI_OP_PREFILL);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null operand");
  DeviceGuard g(ctx->device);
  ProfScope ps(ctx, FFAI_OP_PREFILL, static_cast<cudaStream_t>(stream), "ffai_attn_prefill");
  return prefill_impl(ctx, d, q, k, v, o, lse, static_cast<cudaStream_t>(stream));
}

int ffai_attn_decode(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                     const void* v, void* o, float* lse, int32_t num_splits, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  const int st = check_desc(ctx, d, FFAI_OP_DECODE);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null operand");
  DeviceGuard g(ctx->device);
  ProfScope ps(ctx, FFAI_OP_DECODE, static_cast<cudaStream_t>(stream), "ffai_attn_decode");
  return decode_impl(ctx, d, q, k, v, o, lse, num_splits, static_cast<cudaStream_t>(stream));
}

int ffai_attn_decode_prefetch(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                              const void* k, const void* v, const void* next_k,
                              const void* next_v, void* o, float* lse, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  const int st = check_desc(ctx, d, FFAI_OP_DECODE);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null operand");
  if ((next_k == nullptr) != (next_v == nullptr))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "decode_prefetch: next_k and next_v go together");
  if (reinterpret_cast<uintptr_t>(next_k) % 16 != 0 || reinterpret_cast<uintptr_t>(next_v) % 16 != 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "decode_prefetch: next cache not 16-byte aligned");
  DeviceGuard g(ctx->device);
  ProfScope ps(ctx, FFAI_OP_DECODE, static_cast<cudaStream_t>(stream), "ffai_attn_decode_prefetch");
  return decode_impl(ctx, d, q, k, v, o, lse, 0, static_cast<cudaStream_t>(stream), next_k, next_v);
}

int ffai_attn_varlen(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const int32_t* cu_q,
                     const int32_t* cu_k, int32_t n_seg, const void* q, const void* k,
                     const void* v, void* o, float* lse, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  int st = check_desc(ctx, d, FFAI_OP_VARLEN);
  if (st) return st;
  if (!cu_q || !cu_k || n_seg <= 0 || !q || !k || !v || !o)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "varlen: null argument or n_seg <= 0");
  std::vector<int> qs(n_seg), ql(n_seg), ks(n_seg), kl(n_seg);
  for (int i = 0; i < n_seg; ++i) {
    qs[i] = cu_q[i];
    ql[i] = cu_q[i + 1] - cu_q[i];
    ks[i] = cu_k[i];
    kl[i] = cu_k[i + 1] - cu_k[i];
    if (ql[i] < 0 || kl[i] < 0 || cu_q[i] < 0 || cu_k[i] < 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "varlen: cu_seqlens must be non-decreasing");
    if (ql[i] > 0 && kl[i] == 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "varlen: segment %d has queries but no keys", i);
  }
  const long long Tq = cu_q[n_seg], Tk = cu_k[n_seg];
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps(ctx, FFAI_OP_VARLEN, s, "ffai_attn_varlen");
  const bool stable = (d->flags & FFAI_ATTN_FLAG_INPUTS_STABLE) != 0;
  st = prepare_work(ctx, qs, ql, ks, kl, d->heads, s, 0, 0, stable);
  if (st) return st;
  if (Tq == 0) return FFAI_ATTN_OK;
  const Operand oq{q, true, Tq, 1, d->token_stride}, ok{k, true, Tk, 1, d->token_stride},
      ov{v, true, Tk, 1, d->token_stride};
  return run_tc(ctx, oq, ok, ov, d->heads, d->q_dtype == FFAI_DT_F16, o,
                d->out_dtype == FFAI_DT_BF16, true, 0, lse, Tq, d->scale, s, 0, 0, stable);
}

int ffai_attn_prefill_host(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                           const void* k, const void* v, void* o, float* lse) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  int st = check_desc(ctx, d, FFAI_OP_PREFILL);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null operand");
  if (d->token_stride != 0)
    return set_error(ctx, FFAI_ATTN_DECLINED, "host prefill: dense operands only (token_stride 0)");
  DeviceGuard g(ctx->device);
  if (!ctx->s_h2d) {
    FFAI_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->s_h2d, cudaStreamNonBlocking));
    FFAI_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->s_comp, cudaStreamNonBlocking));
    FFAI_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->s_d2h, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
      FFAI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_h2d[i], cudaEventDisableTiming));
      FFAI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_comp[i], cudaEventDisableTiming));
      FFAI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_d2h[i], cudaEventDisableTiming));
    }
  }
  if (!ctx->pipe_ctx) {
    int cst = 0;
    ctx->pipe_ctx = ffai_attn_create(ctx->device, &cst);
    if (!ctx->pipe_ctx) return set_error(ctx, cst, "pipeline context: %s", g_tls_error.c_str());
  }
  const int B = d->batch, H = d->heads, Nq = d->q_len;
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : d->kv_len;
  // Per-sequence byte sizes: every layout keeps one sequence contiguous.
  const size_t qb = static_cast<size_t>(H) * Nq * kHD * dtype_size(d->q_dtype);
  const size_t kb = static_cast<size_t>(H) * cap * kHD * dtype_size(d->kv_dtype);
  const size_t ob = static_cast<size_t>(H) * Nq * kHD * dtype_size(d->out_dtype);
  const size_t lb = lse ? static_cast<size_t>(H) * Nq * sizeof(float) : 0;
  if (lse && d->out_layout == FFAI_LAYOUT_TOKEN_MAJOR)
    return set_error(ctx, FFAI_ATTN_DECLINED, "host prefill: lse needs heads-split output");
  // Chunks of sequences (about an eighth of the batch: the first chunk's
  // copy-in and the last chunk's kernel and copy-out are the part that does
  // not overlap), two slots in flight.
  const int chunk = std::max(1, std::min(B, (B + 7) / 8));
  const size_t slot = chunk * (qb + 2 * kb + ob + lb);
  const size_t slot_al = (slot + 255) / 256 * 256;
  st = ensure(ctx, reinterpret_cast<uint8_t**>(&ctx->d_pipe), &ctx->pipe_cap, 2 * slot_al);
  if (st) return st;
  uint8_t* dev = static_cast<uint8_t*>(ctx->d_pipe);
  const uint8_t* hq = static_cast<const uint8_t*>(q);
  const uint8_t* hk = static_cast<const uint8_t*>(k);
  const uint8_t* hv = static_cast<const uint8_t*>(v);
  uint8_t* ho = static_cast<uint8_t*>(o);
  uint8_t* hl = reinterpret_cast<uint8_t*>(lse);
  const int nchunks = (B + chunk - 1) / chunk;
  // Fresh state for every call: the previous call's last D2H completed before it returned.
  for (int c = 0; c < nchunks; ++c) {
    const int b0 = c * chunk;
    const int nb = std::min(chunk, B - b0);
    const int sl = c % 2;
    uint8_t* base = dev + sl * slot_al;
    uint8_t* dq = base;
    uint8_t* dk = dq + chunk * qb;
    uint8_t* dv = dk + chunk * kb;
    uint8_t* do_ = dv + chunk * kb;
    uint8_t* dl = do_ + chunk * ob;
    if (c >= 2) FFAI_CUDA(ctx, cudaStreamWaitEvent(ctx->s_h2d, ctx->ev_d2h[sl], 0));
    FFAI_CUDA(ctx, cudaMemcpyAsync(dq, hq + b0 * qb, nb * qb, cudaMemcpyHostToDevice, ctx->s_h2d));
    FFAI_CUDA(ctx, cudaMemcpyAsync(dk, hk + b0 * kb, nb * kb, cudaMemcpyHostToDevice, ctx->s_h2d));
    FFAI_CUDA(ctx, cudaMemcpyAsync(dv, hv + b0 * kb, nb * kb, cudaMemcpyHostToDevice, ctx->s_h2d));
    FFAI_CUDA(ctx, cudaEventRecord(ctx->ev_h2d[sl], ctx->s_h2d));
    FFAI_CUDA(ctx, cudaStreamWaitEvent(ctx->s_comp, ctx->ev_h2d[sl], 0));
    ffai_attn_desc dc = *d;
    dc.batch = nb;
    st = prefill_impl(ctx->pipe_ctx, &dc, dq, dk, dv, do_, lse ? reinterpret_cast<float*>(dl) : nullptr,
                      ctx->s_comp);
    if (st) return set_error(ctx, st, "%s", ctx->pipe_ctx->last_error.c_str());
    FFAI_CUDA(ctx, cudaEventRecord(ctx->ev_comp[sl], ctx->s_comp));
    FFAI_CUDA(ctx, cudaStreamWaitEvent(ctx->s_d2h, ctx->ev_comp[sl], 0));
    FFAI_CUDA(ctx, cudaMemcpyAsync(ho + b0 * ob, do_, nb * ob, cudaMemcpyDeviceToHost, ctx->s_d2h));
    if (lse)
      FFAI_CUDA(ctx, cudaMemcpyAsync(hl + b0 * lb, dl, nb * lb, cudaMemcpyDeviceToHost, ctx->s_d2h));
    FFAI_CUDA(ctx, cudaEventRecord(ctx->ev_d2h[sl], ctx->s_d2h));
  }
  FFAI_CUDA(ctx, cudaStreamSynchronize(ctx->s_d2h));
  unsigned err = 0;
  FFAI_CUDA(ctx, cudaMemcpy(&err, ctx->pipe_ctx->d_err, sizeof err, cudaMemcpyDeviceToHost));
  if (err) {
    cudaMemset(ctx->pipe_ctx->d_err, 0, sizeof(unsigned));
    return set_error(ctx, FFAI_ATTN_ERR_TIMEOUT, "in-kernel wait timed out (error bits 0x%x)", err);
  }
  return FFAI_ATTN_OK;
}

}  // extern "C"

namespace {

// Chunks [0, n_chunks) run on n_workers host threads: worker w starts with
// chunk w, then takes chunks from one queue.  A worker whose `work` fails
// puts the chunk back at the front,
// records the status and retires; the surviving workers drain the queue
// (a worker waits while the queue is empty but others are still busy, since
// a failing one may hand its chunk back).  Returns FFAI_ATTN_OK when every
// chunk completed, else the first failure.  owner[c] (optional) receives the
// worker that completed chunk c; *failed (optional) the number of workers
// that failed.
int run_chunk_queue(int n_workers, int n_chunks, const std::function<int(int, int)>& work,
                    int32_t* owner, int32_t* failed) {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<int> queue;
  for (int c = n_workers; c < n_chunks; ++c) queue.push_back(c);
  int done = 0, first_err = FFAI_ATTN_OK, n_failed = 0;
  int busy = std::min(n_workers, n_chunks);  // the workers' first chunks
  std::vector<std::thread> threads;
  threads.reserve(n_workers);
  for (int w = 0; w < n_workers; ++w) {
    threads.emplace_back([&, w] {
      int c = w < n_chunks ? w : -1;
      while (true) {
        if (c < 0) {
          std::unique_lock<std::mutex> lock(mu);
          cv.wait(lock, [&] { return !queue.empty() || busy == 0; });
          if (queue.empty()) return;
          c = queue.front();
          queue.pop_front();
          ++busy;
        }
        const int st = work(w, c);
        std::lock_guard<std::mutex> lock(mu);
        --busy;
        if (st == FFAI_ATTN_OK) {
          ++done;
          if (owner) owner[c] = w;
          c = -1;
          cv.notify_all();
        } else {
          queue.push_front(c);
          if (first_err == FFAI_ATTN_OK) first_err = st;
          ++n_failed;
          cv.notify_all();
          return;
        }
      }
    });
  }
  for (auto& t : threads) t.join();
  if (failed) *failed = n_failed;
  if (done == n_chunks) return FFAI_ATTN_OK;
  return first_err != FFAI_ATTN_OK ? first_err : FFAI_ATTN_ERR_INVALID;
}

// FFAI_ATTN_FAULT_WORKER=i makes worker i of the multi-device entry fail its
// first chunk on the host, before any copy or launch (fault injection for
// the re-queue path; no GPU is faulted).
int fault_worker() {
  const char* s = std::getenv("FFAI_ATTN_FAULT_WORKER");
  if (!s || !*s) return -1;
  char* end = nullptr;
  const long v = std::strtol(s, &end, 10);
  return (end && *end == 0 && v >= 0) ? static_cast<int>(v) : -1;
}

}  // namespace

extern "C" {

int ffai_attn_multi_prefill_host(ffai_attn_ctx* const* ctxs, int32_t n_ctx,
                                 const ffai_attn_desc* d, const void* q, const void* k,
                                 const void* v, void* o, float* lse, int32_t chunk_segments,
                                 int32_t* failed_workers) {
  if (!ctxs || n_ctx <= 0) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "no contexts");
  for (int i = 0; i < n_ctx; ++i)
    if (!ctxs[i]) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "context %d is null", i);
  int st = check_desc(nullptr, d, FFAI_OP_PREFILL);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null operand");
  if (d->token_stride != 0)
    return set_error(nullptr, FFAI_ATTN_DECLINED, "host prefill: dense operands only");
  if (lse && d->out_layout == FFAI_LAYOUT_TOKEN_MAJOR)
    return set_error(nullptr, FFAI_ATTN_DECLINED, "host prefill: lse needs heads-split output");
  const int B = d->batch, H = d->heads, Nq = d->q_len;
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : d->kv_len;
  const int chunk = chunk_segments > 0 ? std::min(chunk_segments, B) : (B + n_ctx - 1) / n_ctx;
  const int n_chunks = (B + chunk - 1) / chunk;
  // Every layout keeps one sequence contiguous: chunk c is a byte range.
  const size_t qb = static_cast<size_t>(H) * Nq * kHD * dtype_size(d->q_dtype);
  const size_t kb = static_cast<size_t>(H) * cap * kHD * dtype_size(d->kv_dtype);
  const size_t ob = static_cast<size_t>(H) * Nq * kHD * dtype_size(d->out_dtype);
  const size_t lb = static_cast<size_t>(H) * Nq;
  const int faulty = fault_worker();
  std::vector<char> faulted(n_ctx, 0);
  std::vector<std::string> errors(n_ctx);
  auto work = [&](int w, int c) -> int {
    if (w == faulty && !faulted[w]) {
      faulted[w] = 1;
      errors[w] = "injected host-side fault";
      return set_error(ctxs[w], FFAI_ATTN_ERR_CUDA, "worker %d: injected host-side fault", w);
    }
    const int b0 = c * chunk, nb = std::min(chunk, B - b0);
    ffai_attn_desc dc = *d;
    dc.batch = nb;
    const int r = ffai_attn_prefill_host(
        ctxs[w], &dc, static_cast<const uint8_t*>(q) + b0 * qb,
        static_cast<const uint8_t*>(k) + b0 * kb, static_cast<const uint8_t*>(v) + b0 * kb,
        static_cast<uint8_t*>(o) + b0 * ob, lse ? lse + b0 * lb : nullptr);
    if (r != FFAI_ATTN_OK) errors[w] = ctxs[w]->last_error;
    return r;
  };
  int32_t n_failed = 0;
  st = run_chunk_queue(n_ctx, n_chunks, work, nullptr, &n_failed);
  if (failed_workers) *failed_workers = n_failed;
  if (st != FFAI_ATTN_OK) {
    std::string all;
    for (int i = 0; i < n_ctx; ++i)
      if (!errors[i].empty()) all += " [worker " + std::to_string(i) + ": " + errors[i] + "]";
    return set_error(nullptr, st, "multi-device prefill: no worker left for the remaining "
                     "segments;%s", all.c_str());
  }
  return FFAI_ATTN_OK;
}

int ffai_attn_chunk_queue_selftest(int32_t n_workers, int32_t n_chunks, uint32_t fail_mask,
                                   int32_t* owner, int32_t* failed_workers) {
  if (n_workers <= 0 || n_workers > 32 || n_chunks < 0)
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "selftest: 1..32 workers");
  std::vector<char> faulted(n_workers, 0);
  auto work = [&](int w, int) -> int {
    if (((fail_mask >> w) & 1u) && !faulted[w]) {
      faulted[w] = 1;
      return FFAI_ATTN_ERR_CUDA;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
    return FFAI_ATTN_OK;
  };
  return run_chunk_queue(n_workers, n_chunks, work, owner, failed_workers);
}

int ffai_attn_sync(ffai_attn_ctx* ctx, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  DeviceGuard g(ctx->device);
  FFAI_CUDA(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  unsigned err = 0;
  FFAI_CUDA(ctx, cudaMemcpy(&err, ctx->d_err, sizeof err, cudaMemcpyDeviceToHost));
  if (err) {
    FFAI_CUDA(ctx, cudaMemset(ctx->d_err, 0, sizeof(unsigned)));
    if (err & kErrBadArgs)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID,
                       "a paged-cache call met a page id outside the pool or a length past its "
                       "block table (error bits 0x%x)", err);
    return set_error(ctx, FFAI_ATTN_ERR_TIMEOUT, "in-kernel wait timed out (error bits 0x%x)", err);
  }
  return FFAI_ATTN_OK;
}

namespace {

int paged_params(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* k_pool,
                 const void* v_pool, int32_t num_pages, const int32_t* block_table,
                 const int32_t* seq_lens, int32_t max_pages, DecodeParams& p) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (!d) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null descriptor");
  if (d->head_dim != kHD)
    return set_error(ctx, FFAI_ATTN_DECLINED, "head_dim %d: only 64 is served", d->head_dim);
  if (d->batch <= 0 || d->heads <= 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "batch %d, heads %d must be >= 1", d->batch,
                     d->heads);
  if (!valid_dtype(d->kv_dtype)) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "unknown kv dtype");
  if (!k_pool || !v_pool || !block_table || !seq_lens || num_pages <= 0 || max_pages <= 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "paged cache: null pointer or empty pool/table");
  for (const void* ptr : {k_pool, v_pool})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "page pools must be 16-byte aligned");
  p = DecodeParams{};
  p.k = k_pool;
  p.v = v_pool;
  p.rows = d->batch * d->heads;
  p.q_dtype = d->q_dtype;
  p.kv_dtype = d->kv_dtype;
  p.out_dtype = d->out_dtype;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.err = ctx->d_err;
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.max_pages = max_pages;
  p.num_pages = num_pages;
  p.heads = d->heads;
  return FFAI_ATTN_OK;
}

}  // namespace

int ffai_attn_decode_paged(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                           const void* k_pool, const void* v_pool, int32_t num_pages,
                           const int32_t* block_table, const int32_t* seq_lens, int32_t max_pages,
                           void* o, float* lse, void* stream) {
  DecodeParams p{};
  int st = paged_params(ctx, d, k_pool, v_pool, num_pages, block_table, seq_lens, max_pages, p);
  if (st) return st;
  if (d->q_len != 1) return set_error(ctx, FFAI_ATTN_DECLINED, "decode: q_len must be 1");
  if (d->q_dtype != FFAI_DT_F32 && d->q_dtype != d->kv_dtype)
    return set_error(ctx, FFAI_ATTN_DECLINED, "decode: q must be f32 or the cache dtype");
  if (d->out_dtype != FFAI_DT_F32 && d->out_dtype != FFAI_DT_BF16)
    return set_error(ctx, FFAI_ATTN_DECLINED, "out_dtype %d: f32 or bf16 only", d->out_dtype);
  if (!(d->scale > 0.f) || !std::isfinite(d->scale))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "scale must be finite and > 0");
  if (!q || !o) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null operand");
  for (const void* ptr : {q, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "decode operands must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  ProfScope ps(ctx, FFAI_OP_DECODE, static_cast<cudaStream_t>(stream), "ffai_attn_decode_paged");
  // Keys bound for the split: d->kv_len when given, else the table's reach.
  const long long bound = d->kv_len > 0 ? d->kv_len : static_cast<long long>(max_pages) * kPageKeys;
  int S = static_cast<int>(std::min<long long>(kDecodeMaxCluster, 2LL * ctx->num_sms / p.rows));
  S = std::max(1, std::min<int>(S, static_cast<int>((bound + kPageKeys - 1) / kPageKeys)));
  p.q = q;
  p.out = o;
  p.lse = lse;
  p.kv_len = static_cast<int>(std::min<long long>(bound, 1LL << 30));
  FFAI_CUDA(ctx, launch_decode_paged(p, S, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

int ffai_kv_append(ffai_attn_ctx* ctx, const ffai_attn_desc* d, void* k_pool, void* v_pool,
                   int32_t num_pages, const int32_t* block_table, int32_t* seq_lens,
                   int32_t max_pages, const void* k_new, const void* v_new, void* stream) {
  DecodeParams p{};
  int st = paged_params(ctx, d, k_pool, v_pool, num_pages, block_table, seq_lens, max_pages, p);
  if (st) return st;
  if (!k_new || !v_new) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null key or value");
  DeviceGuard g(ctx->device);
  FFAI_CUDA(ctx, launch_kv_append(p, d->batch, k_new, v_new, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

int ffai_kv_copy_pages(ffai_attn_ctx* ctx, const ffai_attn_desc* d, void* k_pool, void* v_pool,
                       int32_t num_pages, const int32_t* src_pages, const int32_t* dst_pages,
                       int32_t n, void* stream) {
  DecodeParams p{};
  static const int32_t kOne = 0;
  int st = paged_params(ctx, d, k_pool, v_pool, num_pages, &kOne, &kOne, 1, p);
  if (st) return st;
  if (n < 0 || (n > 0 && (!src_pages || !dst_pages)))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "page copy: bad page lists");
  DeviceGuard g(ctx->device);
  FFAI_CUDA(ctx, launch_kv_copy_pages(p, src_pages, dst_pages, n, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

int ffai_attn_last_error(const ffai_attn_ctx* ctx, char* buf, size_t n) {
  const std::string& msg = ctx ? ctx->last_error : g_tls_error;
  const int st = ctx ? ctx->last_status : g_tls_status;
  if (buf && n) {
    std::strncpy(buf, msg.c_str(), n - 1);
    buf[n - 1] = 0;
  }
  return st;
}

// ---------------------------------------------------------------------------
// The reference's custom-op surface (flash_attn.rs:104-264), mirrored.
// ---------------------------------------------------------------------------

int ffai_flash_serves(const ffai_tensor4* kt, const ffai_tensor4* v) {
  if (!kt || !v || kt->device < 0 || v->device < 0) return 0;
  // (1, h1, 64, keys) and (1, h2, keys, 64), same heads and keys, and keys at
  // or above the floor the consumer applies (flash_attn.rs:112-128).
  if (kt->dims[0] != 1 || kt->dims[2] != kHD || v->dims[0] != 1 || v->dims[3] != kHD) return 0;
  const int64_t keys = kt->dims[3];
  return (kt->dims[1] == v->dims[1] && keys == v->dims[2] &&
          keys >= std::max(kMinSeq, min_decode_keys()))
             ? 1
             : 0;
}

namespace {

// The decline rules of attend / attend_merged (flash_attn.rs:135-158,
// :218-264) on the operands alone: FFAI_ATTN_OK with `d` filled in for the
// call, or FFAI_ATTN_DECLINED where the reference returns Ok(None).  Errors
// and declines are recorded on `ctx` (null: the calling thread).
int flash_gate(const ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
               const ffai_tensor4* v, int masked, bool merged, ffai_attn_desc* d) {
  if (!q || !kt || !v) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null tensor");
  if (masked) return set_error(ctx, FFAI_ATTN_DECLINED, "masked attention is not served");
  if (q->device < 0 || kt->device != q->device || v->device != q->device)
    return set_error(ctx, FFAI_ATTN_DECLINED, "operands are not on one CUDA device");
  if (q->dtype != FFAI_DT_F32) return set_error(ctx, FFAI_ATTN_DECLINED, "q must be f32");
  const int64_t b = q->dims[0], heads = q->dims[1], qlen = q->dims[2], hd = q->dims[3];
  if (b != 1 || hd != kHD) return set_error(ctx, FFAI_ATTN_DECLINED, "batch 1, head_dim 64 only");
  if (kt->dims[0] != 1 || kt->dims[1] != heads || kt->dims[2] != kHD)
    return set_error(ctx, FFAI_ATTN_DECLINED, "kt must be (1,H,64,keys)");
  const int64_t keys = kt->dims[3];
  if (v->dims[0] != 1 || v->dims[1] != heads || v->dims[2] != keys || v->dims[3] != kHD)
    return set_error(ctx, FFAI_ATTN_DECLINED, "v must be (1,H,keys,64)");
  if (kt->dtype != v->dtype) return set_error(ctx, FFAI_ATTN_DECLINED, "k/v dtypes differ");
  const bool half_kv = kt->dtype != FFAI_DT_F32;
  if (half_kv && (qlen != 1 || merged))
    return set_error(ctx, FFAI_ATTN_DECLINED, "f16/bf16 K/V is served at the decode shape only");
  const int64_t floor = qlen == 1 && !merged ? min_decode_keys() : kMinSeq;
  if (keys < floor)
    return set_error(ctx, FFAI_ATTN_DECLINED, "%lld keys below the floor %lld",
                     static_cast<long long>(keys), static_cast<long long>(floor));
  if (merged ? qlen != keys : (qlen != 1 && qlen != keys))
    return set_error(ctx, FFAI_ATTN_DECLINED, "q_len %lld not served against %lld keys",
                     static_cast<long long>(qlen), static_cast<long long>(keys));
  ffai_attn_desc_init(d);
  d->heads = static_cast<int32_t>(heads);
  d->q_len = static_cast<int32_t>(qlen);
  d->kv_len = static_cast<int32_t>(keys);
  d->q_dtype = FFAI_DT_F32;
  d->kv_dtype = kt->dtype;
  d->k_layout = FFAI_LAYOUT_KT;
  d->out_layout = merged ? FFAI_LAYOUT_TOKEN_MAJOR : FFAI_LAYOUT_HEADS_SPLIT;
  d->scale = 1.0f;  // q arrives pre-scaled (flash_attn.rs:214-217)
  if (env_on("FFAI_ATTN_CHECKED_F32")) d->flags |= FFAI_ATTN_FLAG_CHECKED_F32;
  return FFAI_ATTN_OK;
}

int attend_common(ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
                  const ffai_tensor4* v, int masked, ffai_tensor4* out, bool merged, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (!q || !kt || !v || !out) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "null tensor");
  if (q->device != ctx->device || kt->device != ctx->device || v->device != ctx->device ||
      out->device != ctx->device)
    return set_error(ctx, FFAI_ATTN_DECLINED, "operands are not on this context's CUDA device");
  ffai_attn_desc d;
  const int st = flash_gate(ctx, q, kt, v, masked, merged, &d);
  if (st) return st;
  if (out->dtype != FFAI_DT_F32) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "out must be f32");
  const int64_t qlen = d.q_len;
  if (qlen == 1 && !merged)
    return ffai_attn_decode(ctx, &d, q->data, kt->data, v->data, out->data, nullptr, 0, stream);
  return ffai_attn_prefill(ctx, &d, q->data, kt->data, v->data, out->data, nullptr, stream);
}

}  // namespace

int ffai_flash_attend(ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
                      const ffai_tensor4* v, int32_t masked, ffai_tensor4* out, void* stream) {
  return attend_common(ctx, q, kt, v, masked, out, false, stream);
}

int ffai_flash_attend_merged(ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
                             const ffai_tensor4* v, ffai_tensor4* out, void* stream) {
  return attend_common(ctx, q, kt, v, 0, out, true, stream);
}

int ffai_flash_check(const ffai_tensor4* q, const ffai_tensor4* kt, const ffai_tensor4* v,
                     int32_t masked, int32_t merged) {
  ffai_attn_desc d;
  return flash_gate(nullptr, q, kt, v, masked, merged != 0, &d);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without a context and without allocating: the split kernel's
// tickets and partials live in this statically allocated device array.
//
//   words [0, kStaticRows)                      per-row tickets; must be zero
//                                               before a launch: zero when the
//                                               module loads, and the last CTA
//                                               of each row re-zeroes its
//                                               ticket, so they stay zero
//                                               between launches
//   words [kStaticRows, + kStaticPartFloats)    (row, split) partials (m, l,
//                                               o[64]); no initial value needed
//
// One copy per device: two launches in flight at once on one device (two
// streams, two host threads) share it and race.
namespace {
constexpr int kStaticRows = 4096;                         // max batch x heads
constexpr int kStaticSlots = 4096;                        // max rows x splits
constexpr int kStaticPartFloats = kStaticSlots * kPartStride;
constexpr int kStaticWords = kStaticRows + kStaticPartFloats;  // 1.07 MiB
constexpr int kStaticMaxDevices = 64;
}  // namespace

static __device__ __align__(256) uint32_t g_decode_scratch[kStaticWords];

extern "C" int ffai_attn_decode_static(const ffai_attn_desc* d, const void* q, const void* k,
                                       const void* v, void* o, float* lse, int32_t num_splits,
                                       void* stream) {
  const int st = check_desc(nullptr, d, FFAI_OP_DECODE);
  if (st) return st;
  if (!q || !k || !v || !o) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null operand");
  if (num_splits < 0)
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "num_splits %d < 0", num_splits);
  for (const void* ptr : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "decode operands must be 16-byte aligned");
  const long long rows = static_cast<long long>(d->batch) * d->heads;
  if (rows > 65535)
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "decode_static: %lld rows > 65535", rows);
  const int cap = d->kv_capacity > 0 ? d->kv_capacity : d->kv_len;
  int kv = d->kv_len;
  if (d->causal) kv = std::min(kv, d->q_offset + 1);
  if (kv <= 0) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "no visible keys");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
  if (dev < 0 || dev >= kStaticMaxDevices)
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "device %d out of range", dev);
  // Same chunking as ffai_attn_decode's split kernel.
  int chunk;
  if (num_splits > 0) {
    chunk = (kv + num_splits - 1) / num_splits;
    chunk = std::min(std::max(chunk, 1), 128);
  } else {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaDeviceGetAttribute");
    chunk = d->kv_dtype == FFAI_DT_F32 ? 64 : 128;
    const int splits128 = (kv + chunk - 1) / chunk;
    if (chunk == 128 && rows * splits128 < 2LL * sms && kv > 64) chunk = 64;
  }
  const int splits = (kv + chunk - 1) / chunk;
  if (splits > 1 && (rows > kStaticRows || rows * splits > kStaticSlots))
    return set_error(nullptr, FFAI_ATTN_ERR_INVALID,
                     "decode_static: %lld rows x %d splits exceeds the static scratch "
                     "(at most %d rows and %d rows x splits)",
                     rows, splits, kStaticRows, kStaticSlots);
  // Device address of the scratch, fetched once per device with it current.
  static std::mutex mu;
  static void* addr[kStaticMaxDevices] = {};
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
      e = cudaGetSymbolAddress(&addr[dev], g_decode_scratch);
      if (e != cudaSuccess) {
        addr[dev] = nullptr;
        return cuda_fail(nullptr, e, "cudaGetSymbolAddress(g_decode_scratch)");
      }
    }
    base = addr[dev];
  }
  DecodeParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = o;
  p.lse = lse;
  p.rows = static_cast<int>(rows);
  p.kv_len = kv;
  p.cap = cap;
  p.chunk = chunk;
  p.splits = splits;
  p.q_dtype = d->q_dtype;
  p.kv_dtype = d->kv_dtype;
  p.out_dtype = d->out_dtype;
  p.k_kt = d->k_layout == FFAI_LAYOUT_KT;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.counters = static_cast<unsigned*>(base);
  p.part = reinterpret_cast<float*>(static_cast<uint32_t*>(base) + kStaticRows);
  // The launch reports its status through the runtime's last-error slot, so
  // an error that earlier, unrelated work left there would be read as this
  // launch's.  Report it as what it is, without launching and without
  // clearing it: it belongs to the caller.
  e = cudaPeekAtLastError();
  if (e != cudaSuccess)
    return set_error(nullptr, FFAI_ATTN_ERR_CUDA,
                     "decode_static: a CUDA error was pending before the launch (left by "
                     "earlier work on this thread): %s",
                     cudaGetErrorString(e));
  e = launch_decode(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "launch_decode");
  return FFAI_ATTN_OK;
}

// ---------------------------------------------------------------------------
// int8 GEMV (the reference's Int8Vocab, vocab_int8.rs)

extern "C" {

int ffai_int8_gemv_layout(int32_t rows, int32_t cols, int32_t blk, int64_t* packed_bytes,
                          int64_t* corr_count) {
  if (rows <= 0 || !int8_gemv_served(cols, blk))
    return set_error(nullptr, FFAI_ATTN_DECLINED,
                     "int8 GEMV: blk %d must be a multiple of 32 up to %d dividing cols %d "
                     "(at most %d)", blk, kGvMaxBlk, cols, kGvMaxCols);
  const long long groups = int8_gemv_groups(rows);
  if (packed_bytes) *packed_bytes = groups * (cols / blk) * int8_gemv_record(blk);
  if (corr_count) *corr_count = groups * kGvRows;
  return FFAI_ATTN_OK;
}

int ffai_int8_gemv_quantize(ffai_attn_ctx* ctx, const void* w, int32_t w_dtype, int32_t rows,
                            int32_t cols, int32_t blk, void* packed, float* corr, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (rows <= 0 || !int8_gemv_served(cols, blk))
    return set_error(ctx, FFAI_ATTN_DECLINED,
                     "int8 GEMV: blk %d must be a multiple of 32 up to %d dividing cols %d "
                     "(at most %d)", blk, kGvMaxBlk, cols, kGvMaxCols);
  if (!valid_dtype(w_dtype)) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "unknown weight dtype");
  if (!w || !packed || !corr)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "int8 GEMV quantize: null pointer");
  DeviceGuard g(ctx->device);
  FFAI_CUDA(ctx, launch_int8_quantize(w, w_dtype, rows, cols, blk, static_cast<uint8_t*>(packed),
                                      corr, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

int ffai_int8_gemv(ffai_attn_ctx* ctx, const float* x, int32_t batch, const void* packed,
                   const float* corr, int32_t rows, int32_t cols, int32_t blk, float* out,
                   uint32_t flags, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (flags & ~FFAI_INT8_FLAG_WEIGHTS_STABLE)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "int8 GEMV: unknown flags 0x%x", flags);
  if (rows <= 0 || !int8_gemv_served(cols, blk))
    return set_error(ctx, FFAI_ATTN_DECLINED,
                     "int8 GEMV: blk %d must be a multiple of 32 up to %d dividing cols %d "
                     "(at most %d)", blk, kGvMaxBlk, cols, kGvMaxCols);
  if (batch < 1 || batch > kGvMaxBatch)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "int8 GEMV: batch %d not in [1, %d]", batch,
                     kGvMaxBatch);
  if (!x || !packed || !corr || !out)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "int8 GEMV: null pointer");
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID,
                     "int8 GEMV: packed weights and activations 16-byte aligned");
  Int8GemvParams p{};
  if (!int8_gemv_plan(rows, cols, blk, batch, ctx->num_sms, &p.plan))
    return set_error(ctx, FFAI_ATTN_DECLINED, "int8 GEMV: no shared-memory plan for %d x %d",
                     rows, cols);
  DeviceGuard g(ctx->device);
  constexpr size_t kXqBytes = static_cast<size_t>(kGvMaxCols) / 16 * 128;
  int st = ensure(ctx, &ctx->d_gemv_x, &ctx->gemv_x_cap, kXqBytes + kGvMaxBatch * sizeof(float));
  if (st) return st;
  p.xq = ctx->d_gemv_x;
  p.sx = reinterpret_cast<float*>(ctx->d_gemv_x + kXqBytes);
  p.x = x;
  p.batch = batch;
  p.packed = static_cast<const uint8_t*>(packed);
  p.corr = corr;
  p.rows = rows;
  p.cols = cols;
  p.blk = blk;
  p.out = out;
  p.err = ctx->d_err;
  p.weights_stable = (flags & FFAI_INT8_FLAG_WEIGHTS_STABLE) != 0;
  FFAI_CUDA(ctx, launch_int8_gemv(p, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}


// ---------------------------------------------------------------------------
// f16 GEMV (the reference's F16Gemv, f16_gemv.rs)

int ffai_f16_gemv_layout(int32_t rows, int32_t cols, int64_t* packed_bytes) {
  if (rows <= 0 || !f16_gemv_served(cols))
    return set_error(nullptr, FFAI_ATTN_DECLINED,
                     "f16 GEMV: cols %d must be a positive multiple of 8 (at most %d)", cols,
                     kHgMaxCols);
  if (packed_bytes)
    *packed_bytes = f16_gemv_groups(rows) * f16_gemv_steps(cols) * kHgRows * 16 * 2;
  return FFAI_ATTN_OK;
}

int ffai_f16_gemv_pack(ffai_attn_ctx* ctx, const void* w, int32_t w_dtype, int32_t rows,
                       int32_t cols, void* packed, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (rows <= 0 || !f16_gemv_served(cols))
    return set_error(ctx, FFAI_ATTN_DECLINED,
                     "f16 GEMV: cols %d must be a positive multiple of 8 (at most %d)", cols,
                     kHgMaxCols);
  if (!valid_dtype(w_dtype)) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "unknown weight dtype");
  if (!w || !packed) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "f16 GEMV pack: null pointer");
  DeviceGuard g(ctx->device);
  FFAI_CUDA(ctx, launch_f16_pack(w, w_dtype, rows, cols, static_cast<uint16_t*>(packed),
                                 static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

int ffai_f16_gemv(ffai_attn_ctx* ctx, const float* x, int32_t batch, const void* packed,
                  const float* bias, int32_t rows, int32_t cols, float* out, uint32_t flags,
                  void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (flags & ~FFAI_GEMV_FLAG_WEIGHTS_STABLE)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "f16 GEMV: unknown flags 0x%x", flags);
  if (rows <= 0 || !f16_gemv_served(cols))
    return set_error(ctx, FFAI_ATTN_DECLINED,
                     "f16 GEMV: cols %d must be a positive multiple of 8 (at most %d)", cols,
                     kHgMaxCols);
  if (batch < 1 || batch > kHgMaxBatch)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "f16 GEMV: batch %d not in [1, %d]", batch,
                     kHgMaxBatch);
  if (!x || !packed || !out) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "f16 GEMV: null pointer");
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "f16 GEMV: packed weights 16-byte aligned");
  F16GemvParams p{};
  if (!f16_gemv_plan(rows, cols, batch, ctx->num_sms, &p.plan))
    return set_error(ctx, FFAI_ATTN_DECLINED, "f16 GEMV: no shared-memory plan for %d x %d", rows,
                     cols);
  DeviceGuard g(ctx->device);
  p.x = x;
  p.batch = batch;
  p.packed = static_cast<const uint16_t*>(packed);
  p.bias = bias;
  p.rows = rows;
  p.cols = cols;
  p.out = out;
  p.err = ctx->d_err;
  p.weights_stable = (flags & FFAI_GEMV_FLAG_WEIGHTS_STABLE) != 0;
  FFAI_CUDA(ctx, launch_f16_gemv(p, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// bf16 GEMM with a fused epilogue (the projections around the attention)

namespace {

// 2-d tensor map over a row-major (rows, cols) matrix with row stride ld
// elements: box box_cols x box_rows; the box's rows (box_cols x element
// size bytes) swizzled at that width (128 or 64 bytes).
int make_map_2d(ffai_attn_ctx* ctx, CUtensorMap* map, const void* base, long long cols,
                long long rows, long long ld, int box_rows, bool f32 = false, int box_cols = 64) {
  if (!g_encode) return set_error(ctx, FFAI_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int esize = f32 ? 4 : 2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw =
      box_cols * esize == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                              2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, FFAI_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled: %d", r);
  return FFAI_ATTN_OK;
}

}  // namespace

extern "C" {

int ffai_gemm_bf16(ffai_attn_ctx* ctx, const void* a, int64_t lda, const void* b, int64_t ldb,
                   const float* bias, const void* residual, int64_t ldr, void* out, int64_t ldo,
                   int32_t M, int32_t N, int32_t K, int32_t out_dtype, int32_t act, void* stream) {
  if (!ctx) return set_error(nullptr, FFAI_ATTN_ERR_INVALID, "null context");
  if (M <= 0 || N <= 0 || K <= 0)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: empty shape %d x %d x %d", M, N, K);
  if (N % 32 != 0 || K % 8 != 0)
    return set_error(ctx, FFAI_ATTN_DECLINED, "GEMM: N (%d) a multiple of 32, K (%d) of 8", N, K);
  if (out_dtype != FFAI_DT_F32 && out_dtype != FFAI_DT_BF16)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: output f32 or bf16");
  if (act != FFAI_GEMM_ACT_NONE && act != FFAI_GEMM_ACT_FAST_GELU)
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: unknown activation %d", act);
  if (!a || !b || !out) return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: null pointer");
  const int vec = out_dtype == FFAI_DT_F32 ? 4 : 8;  // elements per 16-byte access
  if (lda < K || ldb < K || lda % 8 != 0 || ldb % 8 != 0 || ldo < N || ldo % vec != 0 ||
      (residual && (ldr < N || ldr % vec != 0)))
    return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: leading dimensions (16-byte rows)");
  for (const void* q : {a, b, static_cast<const void*>(out), residual, static_cast<const void*>(bias)})
    if (q && reinterpret_cast<uintptr_t>(q) % 16 != 0)
      return set_error(ctx, FFAI_ATTN_ERR_INVALID, "GEMM: operands 16-byte aligned");
  DeviceGuard g(ctx->device);
  CUtensorMap tma, tmb;
  int st = make_map_2d(ctx, &tma, a, K, M, lda, 128);
  if (st) return st;
  st = make_map_2d(ctx, &tmb, b, K, N, ldb, 128);  // B tiles as two 128-row boxes
  if (st) return st;
  CUtensorMap tmo, tmr;  // 32 x 32 output / residual blocks of the epilogue's TMA copies
  st = make_map_2d(ctx, &tmo, out, N, M, ldo, 32, out_dtype == FFAI_DT_F32, 32);
  if (st) return st;
  tmr = tmo;
  if (residual) {
    st = make_map_2d(ctx, &tmr, residual, N, M, ldr, 32, out_dtype == FFAI_DT_F32, 32);
    if (st) return st;
  }
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = (M + 127) / 128;
  p.n_tiles = (N + 255) / 256;
  {
    // The last wave's tiles (fewer than the SMs) run as 128-column halves
    // when that still fits one wave: the wave takes half as long.  Not when
    // the right-most column of tiles is at most 128 columns wide: its second
    // halves would lie wholly past N and take a CTA for no output.
    const long long tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
    const long long sms = ctx->num_sms;
    const long long tail = tiles - (tiles - 1) / sms * sms;  // tiles of the last wave
    const int last_cols = N - (p.n_tiles - 1) * 256;
    const bool split = 2 * tail <= sms && last_cols > 128;
    p.split_from = static_cast<int>(split ? tiles - tail : tiles);
    p.items = static_cast<int>(split ? tiles + tail : tiles);
  }
  p.bias = bias;
  p.residual = residual;
  p.ldr = ldr;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_dtype == FFAI_DT_F32;
  p.act = act;
  p.err = ctx->d_err;
  p.f2_one = 0x3F8000003F800000ull;
  p.f2_neg_zero = 0x8000000080000000ull;
  FFAI_CUDA(ctx, launch_gemm(tma, tmb, tmo, tmr, p, ctx->num_sms, static_cast<cudaStream_t>(stream)));
  return FFAI_ATTN_OK;
}

}  // extern "C"
