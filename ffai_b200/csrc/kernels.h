// Internal interface between the C ABI (api.cu) and the kernels.  Plain
// structs of device pointers and sizes; no torch or candle types.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ffai {

// Error bits written to the context's device error word.
enum : unsigned {
  kErrTimeoutProducer = 1u << 0,
  kErrTimeoutMma = 1u << 1,
  kErrTimeoutSoftmax = 1u << 2,
  kErrTimeoutDrain = 1u << 3,
  kErrTimeoutConsumer = 1u << 4,
  kErrBadArgs = 1u << 8,
};

// ---- decode (decode.cu) ----------------------------------------------------

constexpr int kPartStride = 66;  // per (row, split): m, l, o[64]

struct DecodeParams {
  const void* q;  // (rows, 64) of q_dtype
  const void* k;  // rows x cap x 64 (row-major) or rows x 64 x cap (KT)
  const void* v;  // rows x cap x 64
  void* out;      // (rows, 64) f32 or bf16
  float* lse;     // (rows) or null
  float* part;    // rows x splits x kPartStride   (splits > 1)
  unsigned* counters;  // rows tickets, zero between launches (splits > 1)
  int rows;
  int kv_len;
  int cap;
  int chunk;   // keys per CTA, <= 128
  int splits;  // ceil(kv_len / chunk)
  int q_dtype, kv_dtype, out_dtype;
  int k_kt;
  float scale_log2;
  unsigned* err;  // device error word (bounded waits of the cluster kernel)
  int kv_stable;  // cluster kernel: copy K/V before the programmatic-dependency wait
  int kv_append_only;  // cluster kernel: only key kv_len - 1 may be written by the
                       // preceding kernel; copy the others before the wait
  // cluster kernel, row-major caches: another cache of the same shape (the next
  // decode call's) whose keys [k0, k1) of each CTA's row are prefetched into L2
  // once the CTA's own copies are issued; null for none
  const void* pf_k;
  const void* pf_v;
  // paged caches (launch_decode_paged): k, v are pools of pages of kPageKeys
  // keys, (num_pages, heads, kPageKeys, 64); row = b * heads + h
  const int* block_table;  // (batch, max_pages) page ids
  const int* seq_lens;     // (batch) live keys per sequence
  int max_pages;
  int num_pages;
  int heads;
};

constexpr int kPageKeys = 64;

cudaError_t launch_decode(const DecodeParams& p, cudaStream_t s);

// Cluster variant for row-major K (heads-split caches): p.rows x `splits`
// CTAs, each row's keys split into ranges of `keys_per_cta` over one cluster
// of `splits` CTAs (1..kDecodeMaxCluster) that merge through distributed
// shared memory.  Uses no workspace (p.part, p.counters, p.chunk ignored).
constexpr int kDecodeMaxCluster = 8;
cudaError_t launch_decode_cluster(const DecodeParams& p, int splits, int keys_per_cta,
                                  cudaStream_t s);
// The cluster kernel over a paged cache: each sequence's live length comes
// from p.seq_lens (read on the device, after the preceding kernel), split
// into page-aligned ranges over `splits` CTAs.  Rows with no keys get zeros.
cudaError_t launch_decode_paged(const DecodeParams& p, int splits, cudaStream_t s);
// Append one key and value per (sequence, head) at position seq_lens[b]
// (page block_table[b][pos / kPageKeys]) and advance seq_lens[b].
// k_new, v_new: (batch, heads, 64) of the cache type.
cudaError_t launch_kv_append(const DecodeParams& p, int batch, const void* k_new,
                             const void* v_new, cudaStream_t s);
// Copy whole pages src[i] -> dst[i] of both pools (a beam taking over a
// partly filled page before appending to it).
cudaError_t launch_kv_copy_pages(const DecodeParams& p, const int* src, const int* dst, int n,
                                 cudaStream_t s);

// ---- int8 GEMV (gemv_int8.cu) ----------------------------------------------

// Device layout of the quantised weights: rows padded to G = ceil(rows / 16)
// groups of 16 (padding zero); group g is nb = cols / blk block records in
// column order, each int8_gemv_record(blk) = blk * 16 + 64 bytes:
//   bytes [0, blk * 16): chunk c (16 columns) of the block for row l at
//     (c * 16 + l) * 16 -- 16 rows x 16 bytes per chunk, so 8 rows of a chunk
//     are one 128-byte matrix for ldmatrix;
//   bytes [blk * 16, blk * 16 + 64): the 16 rows' f32 block scales, row l at
//     float (l % 8) * 2 + l / 8 (rows l and l + 8 side by side, as the mma's
//     accumulator fragment holds them).
// A group's records are contiguous (group g at g * nb * record bytes), so
// any run of a group's blocks is one bulk copy.  corr: (G * 16) f32.
constexpr int kGvMaxBatch = 8;
constexpr int kGvMaxCols = 8192;
constexpr int kGvMaxBlk = 1024;
constexpr int kGvRows = 16;  // rows per group

__host__ __device__ inline int int8_gemv_record(int blk) { return blk * kGvRows + 64; }
inline bool int8_gemv_served(int cols, int blk) {
  return blk > 0 && blk % 32 == 0 && blk <= kGvMaxBlk && cols > 0 && cols % blk == 0 &&
         cols <= kGvMaxCols;
}
__host__ __device__ inline long long int8_gemv_groups(long long rows) {
  return (rows + kGvRows - 1) / kGvRows;
}

// Launch geometry, computed on the host.  CTA c takes the contiguous groups
// [c * groups / grid, (c + 1) * groups / grid) in rounds of one group per
// consumer warp, each group cut into units of S block records streamed
// through a ring of `ring` shared-memory slots, unit-major within a round.
struct Int8GemvPlan {
  int groups, grid, ring, S;
  int slot_bytes;  // S * record bytes
  int x_off, bar_off, smem;
};
bool int8_gemv_plan(int rows, int cols, int blk, int batch, int sms, Int8GemvPlan* plan);

struct Int8GemvParams {
  const float* x;          // (batch, cols) f32 activations, 16-byte aligned
  int batch;               // 1..8
  uint8_t* xq;             // (cols / 16) * 128 bytes: quantised activations
  float* sx;               // (8) activation scales
  const uint8_t* packed;   // block records (layout above)
  const float* corr;       // (G * 32) activation-offset corrections
  int rows, cols, blk;     // int8_gemv_served(cols, blk)
  float* out;              // (batch, rows)
  unsigned* err;
  int weights_stable;      // weights not written by the preceding kernel
  Int8GemvPlan plan;
};

cudaError_t launch_int8_quantize(const void* w, int w_dtype, int rows, int cols, int blk,
                                 uint8_t* packed, float* corr, cudaStream_t s);
cudaError_t launch_int8_gemv(const Int8GemvParams& p, cudaStream_t s);

// ---- f16 GEMV (gemv_f16.cu) ------------------------------------------------

// Device layout of the f16 weights: rows padded to groups of kHgRows = 8
// (padding zero); group g is steps j = 0 .. ceil(cols / 16) - 1 of 256 bytes:
// for each of the 16 columns 16 j + c, the group's rows 4 s + i (s = 0, 1;
// i = 0 .. 3) at halfword ((g * steps + j) * 16 + c) * 8 + 4 s + i -- so lane
// (s, c) of a warp reads its 4 rows' weights of a column as one 8-byte load
// and the warp's step is 256 contiguous bytes.  Columns past `cols` (cols %
// 16 == 8) are zero and never read.  A group's steps are contiguous, so a
// run of them is one bulk copy.
constexpr int kHgRows = 8;
constexpr int kHgLaneRows = 4;  // rows per lane
constexpr int kHgMaxBatch = 8;
constexpr int kHgMaxCols = 65536;

__host__ __device__ inline long long f16_gemv_groups(long long rows) {
  return (rows + kHgRows - 1) / kHgRows;
}
__host__ __device__ inline int f16_gemv_steps(int cols) { return (cols + 15) / 16; }
inline bool f16_gemv_served(int cols) { return cols > 0 && cols % 8 == 0 && cols <= kHgMaxCols; }

// Launch geometry (host): as for the int8 GEMV -- CTA c takes a contiguous
// range of groups in rounds, each group cut into units of S steps streamed
// unit-major through `ring` slots.  q warps (1, 2 or 4) share a group, each
// taking 4 / q of every lane's 4 rows; a round is consumer warps / q groups.
struct F16GemvPlan {
  int groups, grid, ring, S;
  int q;           // warps per group
  int slot_bytes;  // S * 64
  int bar_off, x_off, x_pitch, smem;  // x_pitch 0: activations read through L1
};
bool f16_gemv_plan(int rows, int cols, int batch, int sms, F16GemvPlan* plan);

struct F16GemvParams {
  const float* x;           // (batch, cols) f32 activations
  int batch;                // 1..8
  const uint16_t* packed;   // f16 weights (layout above)
  const float* bias;        // (rows) or null
  int rows, cols;           // f16_gemv_served(cols)
  float* out;               // (batch, rows)
  unsigned* err;
  int weights_stable;       // weights not written by the preceding kernel
  F16GemvPlan plan;
};

cudaError_t launch_f16_pack(const void* w, int w_dtype, int rows, int cols, uint16_t* packed,
                            cudaStream_t s);
cudaError_t launch_f16_gemv(const F16GemvParams& p, cudaStream_t s);

// ---- bf16 GEMM with a fused epilogue (gemm_tc.cu) ---------------------------

// out[m][n] = act(sum_k A[m][k] B[n][k] + bias[n]) (+ residual[m][n]);
// A, B bf16 row-major (B as weights are stored, (N, K)); act 0 none, 1 the
// reference's FastGelu; out / residual bf16 or f32 (out_f32).
struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles;
  const float* bias;       // (N) or null
  const void* residual;    // (M, ldr) of the output type, or null
  long long ldr;
  void* out;               // (M, ldo)
  long long ldo;
  int out_f32;
  int act;
  unsigned* err;
  // f32x2 pairs (1, 1) and (-0, -0), read by the epilogue's activation as
  // runtime operands: written as constants, ptxas folds them and fuses the
  // activation's separately rounded multiplies and adds.
  unsigned long long f2_one, f2_neg_zero;
  // Work items: tiles [0, split_from) whole, then each tile of [split_from,
  // m_tiles * n_tiles) as two 128-column halves (the last, partial wave split
  // so that it runs on twice as many SMs); items = their count.
  int split_from, items;
};
size_t gemm_smem_bytes();
cudaError_t launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                        const CUtensorMap& tmR, const GemmParams& p, int sms, cudaStream_t s);

// ---- checked f32 prefill (prefill_simt.cu) ---------------------------------

// Element offset of (b, h, row, d) is b*sb + h*sh + row*sr + d*sd.
struct Strides {
  long long sb, sh, sr, sd;
};

struct SimtParams {
  const float* q;
  const float* k;
  const float* v;
  void* out;
  float* lse;  // indexed by b*lse_sb + h*lse_sh + row, or null
  Strides qs, ks, vs, os;
  long long lse_sb, lse_sh;
  int B, H, Nq, Nk;
  int out_dtype;
  int causal, q_offset;
  float scale;
};

cudaError_t launch_prefill_simt(const SimtParams& p, cudaStream_t s);

// ---- tensor-core prefill (prefill_tc.cu) -----------------------------------

constexpr int kTcRows = 128;    // query rows per tile (MMA M)
constexpr int kTcKeys = 128;    // keys per block (MMA N of Q.K^T)
constexpr int kTcStages = 4;    // K/V ring depth (3: 797 against 804 TFLOP/s in five alternating runs)
constexpr int kTcThreads = 608; // 4 softmax warpgroups + TMA warp + 2 MMA warps

// One work unit: query rows [row0, row0 + 128*ntiles) of (seq, head).
struct TcUnit {
  int seq, head, row0, ntiles;
};

struct TcParams {
  const int4* units;  // TcUnit as int4
  int num_units;
  const int* q_start;  // per sequence: first packed token (token-major) or 0
  const int* q_len;
  const int* k_start;
  const int* k_len;
  int heads;
  int q_token_major;   // 0: map coords {0,row,seq*H+head}; 1: {0,head,q_start+row}
  int k_token_major;
  int v_token_major;
  void* out;
  int out_bf16;
  int out_token_major;
  long long out_rows;  // heads-split output: rows per (seq, head)
  float* lse;
  long long lse_tokens;  // token-major lse is (H, lse_tokens)
  float scale_log2;
  unsigned* err;
  int causal;    // key j visible to query row i (within its sequence) iff j <= q_offset + i
  int q_offset;  // >= 0
  int o_tma;     // 1: bf16 output through the tmO tensor map (16-row boxes)
  int inputs_stable;  // 1: q/k/v not written by the preceding kernel; read them
                      // before the programmatic-dependency wait
};

// Key blocks (of kTcKeys) that tile t (0, 1) of a unit needs: all of the
// sequence's blocks, or with `causal` those up to the last row's horizon;
// 0 for an absent tile.  Shared by the kernel and the host's work ordering.
__host__ __device__ inline int tc_tile_blocks(int causal, int q_offset, int q_len, int k_len,
                                              int row0, int ntiles, int t) {
  if (t >= ntiles) return 0;
  const int nblk = (k_len + kTcKeys - 1) / kTcKeys;
  if (!causal) return nblk;
  const int last = row0 + t * kTcRows + kTcRows - 1 < q_len - 1 ? row0 + t * kTcRows + kTcRows - 1
                                                                : q_len - 1;
  const int horizon = (q_offset + last + 1 + kTcKeys - 1) / kTcKeys;  // blocks holding keys <= q_offset+last
  return horizon < nblk ? horizon : nblk;
}

// tm*: 3-d tensor maps built by the host for 128-row x 64-col boxes with
// 128-byte swizzle.  ab_f16: 1 for f16 operands, 0 for bf16.
cudaError_t launch_prefill_tc(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                              const CUtensorMap& tmV, const CUtensorMap& tmO, const TcParams& p,
                              int grid, int ab_f16, cudaStream_t s);
size_t prefill_tc_smem_bytes();

// ---- conversions (convert.cu) -----------------------------------------------

// dst (B,H,N,64) heads-split contiguous 16-bit (bf16, or f16 when dst_f16)
// <- src element (b,h,row,d) at b*sb + h*sh + row*sr + d*sd of f32 / bf16 /
// f16 (src_dtype 0/1/2).
// Several operands of one call (B, H shared) converted in one launch, each
// into its own contiguous heads-split 16-bit buffer of B*H*N rows; the launch
// is a programmatic dependent of the preceding kernel.
struct StageOp {
  const void* src;
  int src_dtype;
  Strides st;
  int N;
  uint16_t* dst;
  int kt;          // set by the launcher: head-dim-major source
  long long rows;  // set by the launcher
};
struct StageBatch {
  StageOp op[3];
  int n;
  int B, H;
  long long end[3];  // set by the launcher: cumulative block counts
};
cudaError_t launch_stage_batch(StageBatch sb, int dst_f16, cudaStream_t s);

}  // namespace ffai
