/*
 * ffai_attn.h -- C ABI of the B200 Whisper attention library (libffai_attn.so).
 *
 * This library replaces the fused CPU attention of the reference,
 * crates/ffai-mercury/src/asr/flash_attn.rs (Remade-With-Rust/FFAI 0.6.2):
 * encoder self-attention, decoder self-attention over the KV cache, and
 * decoder cross-attention.  A Rust crate binds these functions with
 * `extern "C"` declarations; nothing here names a Rust, candle or torch type.
 *
 * Conventions shared by every entry point:
 *   - Status: FFAI_ATTN_OK (0) served; FFAI_ATTN_DECLINED (1) the shape is not
 *     one this library serves and the caller should take its fallback path
 *     (the reference's `Ok(None)`, flash_attn.rs:135-158, :218-264); negative
 *     values are errors (the reference's `Err`, e.g. the `bail!`s at
 *     flash_attn.rs:181-185, :359-363).  ffai_attn_last_error() describes the
 *     last error or decline of a context.
 *   - Buffers are caller-owned device pointers unless a function says host.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - One context per device.  Calls on one context must not overlap on the
 *     GPU (the context owns one workspace): serialise them, as the reference's
 *     engine does behind its Mutex (whisper_candle.rs:50-51, :222).
 *   - head_dim is 64 (every Whisper size; flash_attn.rs:50).
 */
#ifndef FFAI_ATTN_H
#define FFAI_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFAI_ATTN_ABI_VERSION 1

/* ---- status codes ---- */
#define FFAI_ATTN_OK 0
#define FFAI_ATTN_DECLINED 1
#define FFAI_ATTN_ERR_INVALID (-1)  /* malformed descriptor or pointer */
#define FFAI_ATTN_ERR_CUDA (-2)     /* a CUDA runtime/driver call failed */
#define FFAI_ATTN_ERR_TIMEOUT (-3)  /* a bounded in-kernel wait gave up */
#define FFAI_ATTN_ERR_NOMEM (-4)    /* workspace allocation failed */
#define FFAI_ATTN_ERR_NO_DEVICE (-5)

/* ---- element types ---- */
#define FFAI_DT_F32 0
#define FFAI_DT_BF16 1
#define FFAI_DT_F16 2

/* ---- layouts (B = batch of independent sequences, H = heads, N = rows) ----
 * HEADS_SPLIT  (B, H, N, 64): the reference's q and v layout (flash_attn.rs:212-217).
 * TOKEN_MAJOR  (B, N, H, 64), i.e. the merged (B, N, H*64) layout that
 *              attend_merged returns (flash_attn.rs:131-134); also the packed
 *              layout of the variable-length entry point, (T, H, 64).
 * KT           (B, H, 64, N): K transposed, head-dim major, as the reference's
 *              callers hand it over (text_decoder.rs:1107-1114).  K only.     */
#define FFAI_LAYOUT_HEADS_SPLIT 0
#define FFAI_LAYOUT_TOKEN_MAJOR 1
#define FFAI_LAYOUT_KT 2

/* ---- flags ---- */
/* Run the f32 SIMT kernel (f32 operands only) instead of the bf16 tensor-core
 * kernel: max relative error 1e-5 instead of the bf16 path's 1e-2 abs. */
#define FFAI_ATTN_FLAG_CHECKED_F32 0x1u
/* Decode only: the K/V cache is not written by work queued earlier on the
 * same stream.  The decode kernel is always launched as a programmatic
 * dependent (it waits for the preceding kernel before reading q); with this
 * flag it also starts copying the cache before that wait, overlapping the
 * preceding kernel's tail.  True for cross-attention caches (written once per
 * utterance); false for a self-attention cache whose newest key the
 * preceding kernel appends.  No reference counterpart. */
#define FFAI_ATTN_FLAG_KV_STABLE 0x2u
/* Decode only: work queued earlier on the same stream writes at most the
 * cache's newest key (position kv_len - 1 of every row), as the decoder's
 * self-attention append does just before its decode.  The kernel copies the
 * other keys before waiting for that work and the newest after, so the copy
 * of the cache overlaps the preceding kernels.  Implied by KV_STABLE.  No
 * reference counterpart. */
#define FFAI_ATTN_FLAG_KV_APPEND_ONLY 0x4u
/* Prefill and varlen (tensor-core path): no work still pending on the stream
 * when the call is made writes q, k or v (they were written before a
 * synchronisation, or are earlier launches' untouched inputs).  The prefill
 * kernel is always launched as a programmatic dependent: it waits for the
 * preceding kernel before its first read of q/k/v and again before its first
 * write of out/lse.  With this flag it reads and computes before the first
 * of those waits, so a launch over one batch fills the SMs that the preceding
 * launch's last wave leaves idle; the work list then keeps two-tile units in
 * a short last wave (the next launch fills the tail) instead of splitting
 * them.  Ignored where the library stages the operands itself (f32 operands,
 * the K^T layout): the staging kernel writes what the prefill kernel reads.
 * No reference counterpart. */
#define FFAI_ATTN_FLAG_INPUTS_STABLE 0x8u

/* ---- operations, for ffai_attn_check ---- */
#define FFAI_OP_PREFILL 0
#define FFAI_OP_DECODE 1
#define FFAI_OP_VARLEN 2

typedef struct ffai_attn_desc {
  int32_t batch;       /* independent sequences: segments or beams          */
  int32_t heads;       /* heads per sequence                                */
  int32_t q_len;       /* query rows per (sequence, head)                   */
  int32_t kv_len;      /* keys per (sequence, head) that are attended       */
  int32_t head_dim;    /* must be 64                                        */
  int32_t kv_capacity; /* allocated keys per (sequence, head) in k and v;
                          0 means kv_len.  A KV cache of capacity 448 can be
                          attended at its current length kv_len <= 448.     */
  int32_t q_dtype;     /* FFAI_DT_*                                         */
  int32_t kv_dtype;    /* FFAI_DT_*                                         */
  int32_t out_dtype;   /* FFAI_DT_F32 or FFAI_DT_BF16                       */
  int32_t q_layout;    /* FFAI_LAYOUT_*                                     */
  int32_t k_layout;
  int32_t v_layout;
  int32_t out_layout;  /* HEADS_SPLIT or TOKEN_MAJOR                        */
  int32_t causal;      /* 1: key j visible to row i iff j <= q_offset + i   */
  int32_t q_offset;
  float scale;         /* logits = scale * q.k; the reference folds it into
                          q before the kernel, so its callers pass 1.0      */
  uint32_t flags;      /* FFAI_ATTN_FLAG_*                                  */
  int32_t token_stride; /* TOKEN_MAJOR q/k/v inputs: elements from one token's
                          row to the next; 0 means heads * 64 (dense).  With
                          3 * heads * 64, q, k and v can be the three views of
                          one fused QKV projection output (T, 3, heads, 64),
                          read in place with no head split (the reference's
                          prep glue, text_decoder.rs:1083-1124).  A multiple
                          of 8.  Not for the host-buffer entries.          */
} ffai_attn_desc;

typedef struct ffai_attn_ctx ffai_attn_ctx;

/* Library version string, e.g. "ffai-attn-b200 1 sm_100a". */
const char* ffai_attn_version(void);

/* Fill `d` with defaults: batch 1, head_dim 64, f32 everywhere, heads-split
 * layouts, scale 1.0, no flags. */
void ffai_attn_desc_init(ffai_attn_desc* d);

/* Host-only shape/dtype gate: FFAI_ATTN_OK if `op` serves `d`, else
 * FFAI_ATTN_DECLINED or FFAI_ATTN_ERR_INVALID.  Needs no GPU. */
int ffai_attn_check(const ffai_attn_desc* d, int op);

/* Create a context on CUDA device `device` (workspace, device error word,
 * TMA descriptor encoder).  Replaces the reference's lazy CPU feature
 * detection (flash_attn.rs:75-97).  Returns NULL and sets *status on error. */
ffai_attn_ctx* ffai_attn_create(int device, int* status);
void ffai_attn_destroy(ffai_attn_ctx* ctx);

/* Encoder/prefill attention over `batch` equal-length sequences:
 *   o = softmax(scale * q k^T) v per (sequence, head).
 * Replaces MergedAttnOp::cpu_fwd / FlashAttnOp::cpu_fwd's encoder branch
 * (flash_attn.rs:170-209, :400-405) and flash_head_strided (:429-487).
 * bf16/f16 operands run the tcgen05 tensor-core kernel; f32 operands are
 * converted to bf16 on the device first, unless FFAI_ATTN_FLAG_CHECKED_F32
 * selects the f32 SIMT kernel.  `causal` (q_offset >= 0) masks key j from
 * query row i unless j <= q_offset + i: the decoder's prompt prefill over its
 * KV cache (the reference builds this mask in causal_mask,
 * text_decoder.rs:904-923, and declines the fused kernel for it,
 * flash_attn.rs:219); both kernels serve it.  `lse` (optional, f32) receives
 * the natural log-sum-exp of each row's scaled logits: (B,H,N) for
 * heads-split output, (H, B*N) for token-major output. */
int ffai_attn_prefill(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                      const void* v, void* o, float* lse, void* stream);

/* Decode attention, q_len = 1, over batch*heads rows (beams x heads), with
 * split-KV partial softmax and an in-kernel combine.  Replaces the decode
 * branch of FlashAttnOp::cpu_fwd (flash_attn.rs:289-399), xattn_head (:602-696)
 * and xattn_head_f16 (:714-789).  q is f32 or the cache type; the cache (k, v)
 * is f32, bf16 or f16; k is KT or HEADS_SPLIT (row-major keys); v is
 * HEADS_SPLIT.  `num_splits` 0 = automatic.  Output (B,H,1,64). */
int ffai_attn_decode(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q, const void* k,
                     const void* v, void* o, float* lse, int32_t num_splits, void* stream);

/* ffai_attn_decode (automatic split) that also brings another cache of the
 * same shape, dtype and layout -- the next decode call's, e.g. the next
 * layer's cross-attention keys and values, which a decoder step knows in
 * advance -- into L2 while this call streams its own: each CTA of the cluster
 * kernel prefetches (cp.async.bulk.prefetch.L2) the same key range of the
 * same row of next_k / next_v once its own copies are issued, so the next
 * call reads them from L2 and HBM keeps streaming through this call's tail.
 * A prefetch only fills the cache, it reads nothing into this call's results,
 * so next_k / next_v may still be written by other work.  Results are those
 * of ffai_attn_decode with num_splits 0.  Both null: no prefetch.  Only the
 * cluster kernel (row-major caches with batch x heads x 8 >= the GPU's SMs)
 * prefetches; other shapes ignore the hint.  No reference counterpart (the
 * reference's decode heads read host memory, flash_attn.rs:602-789). */
int ffai_attn_decode_prefetch(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                              const void* k, const void* v, const void* next_k,
                              const void* next_v, void* o, float* lse, void* stream);

/* Decode as ffai_attn_decode's split kernel does (same chunking for the same
 * num_splits, same results), but with no context and no memory allocation:
 * it calls no cudaMalloc / cudaFree or allocating library function.  For
 * callers that cannot allocate device memory during a decode step: a runtime
 * whose device memory is all owned by its own caching pool, or a
 * latency-bound streaming thread that must not block in the driver
 * (cudaFree synchronises the device).  No reference counterpart.
 *
 * Runs on the calling thread's current CUDA device, which must own the
 * buffers and `stream`.  The split partials and per-row tickets live in a
 * static device array of the library (1.07 MiB per device): at most 4096
 * rows (batch x heads) and 4096 rows x splits when a row is split; larger
 * shapes return FFAI_ATTN_ERR_INVALID.  The tickets start at zero when the
 * library's module loads and every launch leaves them at zero.  The scratch
 * address is looked up once per device on the first call with that device
 * current; make that first call before any stream capture.  Calls that can
 * be in flight at the same time on one device (different streams or host
 * threads) share the scratch and race: serialise them.  Errors and declines
 * are reported through ffai_attn_last_error(NULL, ...).  A CUDA error that
 * earlier work left pending on the calling thread is reported as such
 * (FFAI_ATTN_ERR_CUDA, nothing launched) and left in place for its owner. */
int ffai_attn_decode_static(const ffai_attn_desc* d, const void* q, const void* k, const void* v,
                            void* o, float* lse, int32_t num_splits, void* stream);

/* ---- paged KV cache ------------------------------------------------------
 * A device-resident cache that grows in place, replacing the reference's
 * per-step Tensor::cat of the decoder self-attention cache and its per-step
 * split / transpose / contiguous copies (DecoderState, text_decoder.rs:
 * 1226-1243; growth at :657-664; re-layout at :841), and letting beams share
 * pages instead of cloning caches (TextDecoder::save/restore, :1363-1381).
 * Pools k_pool, v_pool hold num_pages pages of FFAI_PAGE_KEYS keys for every
 * head: (num_pages, heads, FFAI_PAGE_KEYS, 64) of d->kv_dtype.  Sequence b
 * (a beam) owns pages block_table[b * max_pages + i] for its keys
 * [i * FFAI_PAGE_KEYS, (i + 1) * FFAI_PAGE_KEYS) and has seq_lens[b] live
 * keys; block_table and seq_lens are DEVICE int32 arrays.  The host owns the
 * page allocation (a page must be in the table before a key lands in it). */
#define FFAI_PAGE_KEYS 64

/* Decode over a paged cache: q (batch, heads, 1, 64) against each
 * sequence's seq_lens[b] keys (read on the device, so an append queued just
 * before on the stream is seen).  d->kv_len, when > 0, is an upper bound of
 * the lengths that sets the work split (0: the table's reach, max_pages * 64);
 * the block table must not be written by the kernel queued just before (the
 * host writes it), since it is read ahead of that kernel's completion.  Rows
 * with no keys give zeros.  Page ids outside [0, num_pages), or a length
 * above the bound, are not read: ffai_attn_sync then reports
 * FFAI_ATTN_ERR_INVALID. */
int ffai_attn_decode_paged(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                           const void* k_pool, const void* v_pool, int32_t num_pages,
                           const int32_t* block_table, const int32_t* seq_lens, int32_t max_pages,
                           void* o, float* lse, void* stream);

/* Append one key and value per (sequence, head): k_new, v_new (batch, heads,
 * 64) of d->kv_dtype land at position seq_lens[b], which then advances by 1
 * (in place; the reference concatenates a new tensor each step). */
int ffai_kv_append(ffai_attn_ctx* ctx, const ffai_attn_desc* d, void* k_pool, void* v_pool,
                   int32_t num_pages, const int32_t* block_table, int32_t* seq_lens,
                   int32_t max_pages, const void* k_new, const void* v_new, void* stream);

/* Copy whole pages src_pages[i] -> dst_pages[i] (device int32 lists) in both
 * pools: a beam that forks from another takes its own copy of the shared,
 * partly filled last page before appending to it. */
int ffai_kv_copy_pages(ffai_attn_ctx* ctx, const ffai_attn_desc* d, void* k_pool, void* v_pool,
                       int32_t num_pages, const int32_t* src_pages, const int32_t* dst_pages,
                       int32_t n, void* stream);

/* ---- int8 GEMV ---------------------------------------------------------
 * The reference's block-scaled int8 GEMV (Int8Vocab, vocab_int8.rs), which
 * it runs for the vocabulary projection (text_decoder.rs:945-969) and the
 * decoder MLP's single-row layers (:94-104, :210-226).  Same quantisation and
 * arithmetic, so outputs equal the reference's bit for bit.  Weights W are
 * (rows, cols) row-major; blk (the reference's FFAI_VOCAB_BLK, default 32) is
 * a multiple of 32, at most 1024, dividing cols (at most 8192) -- other
 * shapes are FFAI_ATTN_DECLINED, as Int8Vocab::new (:102-131) returns None.
 *
 * The quantised weights are kept in a device layout of their own, rows padded
 * to G = ceil(rows / 32) groups of 32 (padding zero).  Group g is cols / blk
 * block records in column order (group g at byte g * (cols / blk) * R, R =
 * blk * 32 + 128), record b holding, for the group's 32 rows l:
 *   bytes [0, blk * 32): weight (int8) of column 16c + j of the block at
 *          (c * 32 + l) * 16 + j;
 *   bytes [blk * 32, R): the f32 scale of block b of row l at blk * 32 + 4 l.
 * corr: f32 (G * 32).  Device buffers throughout. */

/* Sizes of the two buffers for a (rows, cols) matrix: packed bytes and corr
 * element count.  FFAI_ATTN_DECLINED for shapes not served. */
int ffai_int8_gemv_layout(int32_t rows, int32_t cols, int32_t blk, int64_t* packed_bytes,
                          int64_t* corr_count);

/* Int8Vocab::new (vocab_int8.rs:97-166) on the device: W of w_dtype (f32,
 * bf16 or f16; widened to f32 exactly) into the layout above. */
int ffai_int8_gemv_quantize(ffai_attn_ctx* ctx, const void* w, int32_t w_dtype, int32_t rows,
                            int32_t cols, int32_t blk, void* packed, float* corr, void* stream);

/* Int8VocabOp::cpu_fwd (vocab_int8.rs:218-305) for `batch` (1..8) activation
 * rows at once: x (batch, cols) f32 -> out (batch, rows) f32, each row
 * quantised on its own as the reference does per call; the weights are read
 * once for all rows (a small kernel quantises x into the context's scratch,
 * then the GEMV kernel streams the weights: calls on one context must not
 * run concurrently on different streams).  packed and x 16-byte aligned.
 * flags: 0 or
 * FFAI_INT8_FLAG_WEIGHTS_STABLE -- the weights were not written by the kernel
 * launched just before on the stream, so the GEMV may start streaming them
 * before that kernel ends (x is always read after it). */
#define FFAI_INT8_FLAG_WEIGHTS_STABLE 0x2u
#define FFAI_GEMV_FLAG_WEIGHTS_STABLE 0x2u /* the same flag, for ffai_f16_gemv */
int ffai_int8_gemv(ffai_attn_ctx* ctx, const float* x, int32_t batch, const void* packed,
                   const float* corr, int32_t rows, int32_t cols, int32_t blk, float* out,
                   uint32_t flags, void* stream);

/* ---- f16 GEMV ----------------------------------------------------------
 * The reference's F16Gemv (f16_gemv.rs), the default path of the decoder's
 * single-row projections (QLinear::Half, text_decoder.rs:106-118, :231-252):
 * weights rounded to f16 once, f32 fused multiply-adds in 16 chains of
 * columns (chain c: columns 16 j + c in order of j; an 8-column tail feeds
 * chains 0-7), reduced as ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7))
 * with a_i = c_i + c_{i+8}; outputs equal the reference's bit for bit (NaN
 * payloads aside).  cols a positive multiple of 8 (f16_gemv.rs:99-103),
 * at most 65536.  Device layout of the f16 weights: rows in groups of 8;
 * group g is ceil(cols / 16) steps of 16 columns x 8 rows (256 bytes):
 * column 16 j + c of row 8 g + i at halfword ((g * steps + j) * 16 + c) * 8
 * + i, padding zero. */

/* Bytes of the packed f16 weights; FFAI_ATTN_DECLINED when not served. */
int ffai_f16_gemv_layout(int32_t rows, int32_t cols, int64_t* packed_bytes);

/* F16Gemv::new (f16_gemv.rs:89-119) on the device: W (rows, cols) row-major
 * of w_dtype, rounded to f16 (nearest-even) into the layout above. */
int ffai_f16_gemv_pack(ffai_attn_ctx* ctx, const void* w, int32_t w_dtype, int32_t rows,
                       int32_t cols, void* packed, void* stream);

/* F16GemvOp::cpu_fwd (f16_gemv.rs:145-164) for `batch` (1..8) activation
 * rows at once (the reference loops rows, text_decoder.rs:158-170): x
 * (batch, cols) f32 -> out (batch, rows) f32, plus bias (rows) when not
 * null, added after the dot product as QLinear::forward does (:281-289).
 * packed 16-byte aligned; flags 0 or FFAI_GEMV_FLAG_WEIGHTS_STABLE (the
 * weights were not written by the kernel launched just before). */
int ffai_f16_gemv(ffai_attn_ctx* ctx, const float* x, int32_t batch, const void* packed,
                  const float* bias, int32_t rows, int32_t cols, float* out, uint32_t flags,
                  void* stream);

/* ---- bf16 GEMM with a fused epilogue ------------------------------------
 * The projections around the attention, which the reference runs on candle's
 * CPU GEMM: the encoder MLP (fc1 -> FastGelu -> fc2 + residual,
 * audio_encoder.rs:147-165), the q/k/v projection that feeds the attention in
 * its layout (text_decoder.rs:1083-1124) and the out-projection:
 *   out[m][n] = act(sum_k a[m][k] b[n][k] + bias[n]) (+ residual[m][n])
 * a (M, K) and b (N, K) bf16 row-major (b as weights are stored), leading
 * dimensions in elements (multiples of 8); bias f32 (N) or null; out and
 * residual of out_dtype (FFAI_DT_F32 or FFAI_DT_BF16), residual null for
 * none; act FFAI_GEMM_ACT_FAST_GELU applies the reference's FastGelu
 * (text_decoder.rs:341-350) in f32 before the residual.  N a multiple of 32,
 * K of 8 (else FFAI_ATTN_DECLINED); f32 accumulation on the tensor cores.
 * The q/k/v projection's output (T, 3 * H * 64) is the attention's three
 * TOKEN_MAJOR operands with token_stride = 3 * H * 64, as it stands. */
#define FFAI_GEMM_ACT_NONE 0
#define FFAI_GEMM_ACT_FAST_GELU 1
int ffai_gemm_bf16(ffai_attn_ctx* ctx, const void* a, int64_t lda, const void* b, int64_t ldb,
                   const float* bias, const void* residual, int64_t ldr, void* out, int64_t ldo,
                   int32_t M, int32_t N, int32_t K, int32_t out_dtype, int32_t act, void* stream);

/* Variable-length (ragged) prefill over packed segments, TOKEN_MAJOR
 * (T, H, 64) operands and output.  Segment s owns query rows
 * [cu_seqlens_q[s], cu_seqlens_q[s+1]) and keys [cu_seqlens_k[s],
 * cu_seqlens_k[s+1]); each attends only within itself.  The cu_seqlens arrays
 * are HOST arrays of n_seg+1 int32 (lengths are known to the host that packed
 * the buffer); the context schedules the (segment, head, row-tile) work items
 * longest first.  No reference counterpart: the reference loops windows one
 * at a time (text_decoder.rs:1069-1076).  d->batch, q_len and kv_len are
 * ignored; d->heads, dtypes, scale and flags apply.  `lse` is (H, T). */
int ffai_attn_varlen(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const int32_t* cu_seqlens_q,
                     const int32_t* cu_seqlens_k, int32_t n_seg, const void* q, const void* k,
                     const void* v, void* o, float* lse, void* stream);

/* Host-buffer prefill: q, k, v, o (and lse) are HOST pointers (pinned memory
 * recommended).  The context streams the batch through the device in
 * sequence chunks, overlapping host-to-device copies, kernels and
 * device-to-host copies on its own streams, and returns when `o` holds the
 * result.  This is the end-to-end entry a CPU caller (the reference's
 * candle CPU tensors) uses.  Same layouts and semantics as
 * ffai_attn_prefill. */
int ffai_attn_prefill_host(ffai_attn_ctx* ctx, const ffai_attn_desc* d, const void* q,
                           const void* k, const void* v, void* o, float* lse);

/* Multi-device host-buffer prefill (the host side of segment sharding).
 * The batch's sequences are cut into chunks of `chunk_segments` (0: one
 * chunk per context); n_ctx worker threads, one per context (a context per
 * GPU, or several on one GPU), take chunks from a shared queue and run each
 * through ffai_attn_prefill_host, which writes the chunk's rows straight into
 * the host output (the host gather; no collective, no peer traffic).  A
 * worker whose chunk fails hands the chunk back and retires; the surviving
 * workers finish the batch, and the call still returns FFAI_ATTN_OK.
 * *failed_workers (optional) receives the number of workers that failed.
 * The environment variable FFAI_ATTN_FAULT_WORKER=i makes worker i fail its
 * first chunk on the host, before any copy or launch (fault injection).
 * No reference counterpart: the reference runs one window at a time
 * (text_decoder.rs:1069-1076). */
int ffai_attn_multi_prefill_host(ffai_attn_ctx* const* ctxs, int32_t n_ctx,
                                 const ffai_attn_desc* d, const void* q, const void* k,
                                 const void* v, void* o, float* lse, int32_t chunk_segments,
                                 int32_t* failed_workers);

/* Self-test of ffai_attn_multi_prefill_host's chunk queue without a GPU:
 * n_workers (1..32) threads take n_chunks chunks; worker w fails its first
 * chunk when bit w of fail_mask is set.  owner[c] (optional) receives the
 * worker that completed chunk c.  Returns FFAI_ATTN_OK when every chunk
 * completed.  Test infrastructure; no reference counterpart. */
int ffai_attn_chunk_queue_selftest(int32_t n_workers, int32_t n_chunks, uint32_t fail_mask,
                                   int32_t* owner, int32_t* failed_workers);

/* Opt-in launch timing: with profiling on (this call with enable = 1, or
 * FFAI_ATTN_PROFILE=1 when the context is created) every prefill, decode and
 * varlen call on `ctx` is bracketed by CUDA events on its stream and an NVTX
 * range.  With ms / launches non-null, the call waits for the recorded
 * events, writes the total milliseconds and call counts per operation
 * (index FFAI_OP_PREFILL, FFAI_OP_DECODE, FFAI_OP_VARLEN) and resets them.
 * enable: 1 on, 0 off, -1 unchanged.  The reference's counterpart is its
 * FFAI_PROFILE stage counters (profile.rs:1-32). */
int ffai_attn_profile(ffai_attn_ctx* ctx, int32_t enable, double* ms, int64_t* launches);

/* Synchronise `stream` and report the device error word: FFAI_ATTN_OK, or
 * FFAI_ATTN_ERR_TIMEOUT if an in-kernel bounded wait gave up since the last
 * call (the word is then cleared), or FFAI_ATTN_ERR_CUDA. */
int ffai_attn_sync(ffai_attn_ctx* ctx, void* stream);

/* Copy the last error or decline message of `ctx` (or of the calling thread
 * when ctx is NULL) into buf; returns the status it belongs to. */
int ffai_attn_last_error(const ffai_attn_ctx* ctx, char* buf, size_t n);

/* ---- the reference's custom-op surface, mirrored ------------------------
 * A contiguous 4-d tensor as the reference's candle Tensor presents it to
 * flash_attn.rs.  device = CUDA ordinal, or -1 for host memory. */
typedef struct ffai_tensor4 {
  void* data;
  int64_t dims[4];
  int32_t dtype;  /* FFAI_DT_* */
  int32_t device;
} ffai_tensor4;

/* flash_attn::serves (flash_attn.rs:104-129): 1 if the decode kernel will
 * serve this K^T (1,H,64,keys) / V (1,H,keys,64) pair, else 0.  Callers use
 * it to choose the cross-attention cache dtype before building the cache. */
int ffai_flash_serves(const ffai_tensor4* kt, const ffai_tensor4* v);

/* flash_attn::attend (flash_attn.rs:218-264): q (1,H,qlen,64) pre-scaled f32,
 * kt (1,H,64,keys), v (1,H,keys,64) f32 (or f16/bf16 at qlen = 1).  Writes
 * out (1,H,qlen,64) f32.  FFAI_ATTN_DECLINED where the reference returns
 * Ok(None): masked, head_dim != 64, keys below the floor
 * (FFAI_DECODE_MIN_KEYS for qlen = 1, 256 otherwise), qlen not in {1, keys},
 * or host memory.
 *
 * Numerics differ from the reference's f32 kernel at the encoder shape
 * (qlen = keys): the f32 operands are rounded to bf16 on the device and run
 * on the tensor cores with f32 accumulation, so the output differs from the
 * reference's by about 5e-4 (max abs, Whisper-scaled inputs; the reference's
 * own kernel matches its three-op path to 6.9e-7, flash_attn.rs:7).  With
 * the environment variable FFAI_ATTN_CHECKED_F32=1 (read on every call) the
 * encoder shape runs the f32 kernel instead, within 1e-5 relative of the
 * reference, at a fraction of the throughput.  The decode shape (qlen = 1)
 * always computes in f32 over the cache's own type. */
int ffai_flash_attend(ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
                      const ffai_tensor4* v, int32_t masked, ffai_tensor4* out, void* stream);

/* flash_attn::attend_merged (flash_attn.rs:135-158): as attend for the
 * encoder shape, writing out (1, seq, H*64) f32 directly. */
int ffai_flash_attend_merged(ffai_attn_ctx* ctx, const ffai_tensor4* q, const ffai_tensor4* kt,
                             const ffai_tensor4* v, ffai_tensor4* out, void* stream);

/* The decline decision of ffai_flash_attend (merged = 0) or
 * ffai_flash_attend_merged (merged = 1) on the operands alone, without a
 * context or a GPU: FFAI_ATTN_OK if the call would be served, else
 * FFAI_ATTN_DECLINED (the reference's Ok(None)) or an error; the message is
 * in ffai_attn_last_error(NULL, ...).  A candle op cannot return "declined"
 * from its cuda_fwd, so the CUDA branch of attend / attend_merged asks here
 * first, as the reference's functions check before apply_op3
 * (flash_attn.rs:135-158, :218-264). */
int ffai_flash_check(const ffai_tensor4* q, const ffai_tensor4* kt, const ffai_tensor4* v,
                     int32_t masked, int32_t merged);

#ifdef __cplusplus
}
#endif

#endif /* FFAI_ATTN_H */
