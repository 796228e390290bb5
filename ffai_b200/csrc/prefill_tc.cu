// Tensor-core prefill attention for sm_100a: TMA -> shared memory ->
// tcgen05.mma with accumulators in tensor memory, f32 online softmax.
//
// Replaces the reference's encoder kernel (crates/ffai-mercury/src/asr/
// flash_attn.rs:429-487 flash_head_strided, with scores_tile :797-873,
// softmax_row :955-998, accum_pv :880-948): same mathematics -- blocks of
// keys, running max and sum, rescale of the accumulator, final 1/sum -- laid
// out for Blackwell instead of AVX2.
//
// One persistent CTA per SM walks a list of work units.  A unit is up to 256
// query rows (two 128-row tiles, t = 0, 1) of one (sequence, head); both
// tiles share every K/V block, so each block is fetched once for 256 rows.
//
//   warp 16     TMA producer: Q tiles, then a 4-stage ring of K/V blocks of
//               128 keys (16 KB each, 128-byte swizzle).  Also owns TMEM.
//   warps 17,18 MMA issuers, one warp per tile:   S_t = Q_t K^T   (M=128, N=128, K=64)
//                                         O_t += P_t V    (M=128, N=64,  K=128)
//               with P_t read straight from tensor memory (the "A in TMEM"
//               form), so probabilities never touch shared memory.  S_t(j+1)
//               is issued as soon as the softmax has *read* S_t(j), before
//               P_t(j).V, so the tensor core computes the next scores while
//               the softmax of the current ones runs.
//   warps 0-15  softmax, 8 warps per tile.  A warp owns 16 query rows, four
//               lanes per row, each lane a quarter of the row's 128 keys (the
//               16x256b TMEM access shape), so a row's max and sum reduce with
//               two warp shuffles.  Each lane loads its scores, releases S,
//               exponentiates in the log2 domain (packed f32x2 scaling, MUFU
//               ex2; a polynomial exp2 on the FMA pipe can take a share of
//               the pairs), sums the rounded probabilities it writes (so
//               the applied weights P/l sum to 1) and stores bf16 P into its
//               own TMEM buffer (16x128b shape, which lines up with the
//               scores' layout).  The running max is only moved (and O
//               rescaled in TMEM) when it grows by more than 2^8, so most
//               blocks never touch O.  After the last block: O / l to global
//               memory.
//
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), P0 [256,320),
// P1 [320,384), O0 [384,448), O1 [448,512).
//
// Every wait is bounded (common.cuh); on a timeout the CTA raises an error
// bit, drains its MMAs and TMA loads, frees TMEM and exits.
//
// The kernel is a programmatic dependent of the preceding kernel on its
// stream and lets its own dependents launch once all its CTAs are resident.
// It waits for the preceding kernel before the producer's first load (unless
// the caller marks q/k/v stable) and before the first store of its output,
// so with stable inputs back-to-back launches over independent batches run
// the next batch's units on the SMs the previous launch's last wave frees.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr uint32_t kTileBytes = kTcRows * 64 * 2;  // 16 KB: 128 rows x 128 B
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;  // + 128 t, + 64 t, + 64 t
// Warps 0-15 softmax (warp w: tile w/8, TMEM lanes 32(w%4) + 16((w/4)%2) + [0,16)),
// 16 the TMA producer, 17 and 18 the per-tile MMA issuers.
constexpr int kWarpProducer = 16, kWarpMma0 = 17;

struct __align__(8) TcBars {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kTcStages], v_full[kTcStages], kv_empty[kTcStages];
  uint64_t s_full[2], sc_done[2], p_full[2], o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// Q0, Q1, and the K and V rings, then the barriers.
// Output staging for the TMA-store epilogue: per softmax warp, 16 rows of
// 64 bf16 (2 KB) in the 128-byte-swizzled layout of the output tensor map.
constexpr uint32_t kStageBytes = 16 * 128;
constexpr size_t kSmemTiles = (2 + 2 * kTcStages) * kTileBytes + 16 * kStageBytes;
constexpr size_t kSmemBytes = kSmemTiles + sizeof(TcBars) + 1024;  // +1024: alignment slack

__device__ __forceinline__ void unit_at(const TcParams& p, int u, TcUnit& out) {
  const int4 w = __ldg(p.units + u);
  out.seq = w.x;
  out.head = w.y;
  out.row0 = w.z;
  out.ntiles = w.w;
}

// Key blocks tile t of unit w attends (0 when the tile is absent).
__device__ __forceinline__ int tile_blocks(const TcParams& p, const TcUnit& w, int t) {
  return tc_tile_blocks(p.causal, p.q_offset, __ldg(p.q_len + w.seq), __ldg(p.k_len + w.seq),
                        w.row0, w.ntiles, t);
}

// Key blocks the unit loads: those of its last tile, which sees the most.
__device__ __forceinline__ int unit_blocks(const TcParams& p, const TcUnit& w) {
  return tile_blocks(p, w, w.ntiles - 1);
}

// TMA coordinates of a 128-row box of (seq, head) starting at `row`.
__device__ __forceinline__ void box_coords(int token_major, int start, int heads, int seq, int head,
                                           int row, int& c1, int& c2) {
  if (token_major) {
    c1 = head;
    c2 = start + row;
  } else {
    c1 = row;
    c2 = seq * heads + head;
  }
}

// A wait whose outcome is the same for all 32 lanes, so that the warp-wide
// tcgen05.ld/st that follow are never reached by part of a warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned* err, unsigned code) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, code);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- producer
// After an abort: wait (bounded, ignoring the abort flag) for the most
// recently armed phase of every load barrier, so that no TMA write lands in
// shared memory after the CTA has exited.  The producer is the only thread
// that arms these barriers, so the last armed phase is the newest one and
// waiting for it returns at once if it has already completed.
__device__ void drain_loads(TcBars* bars, const uint32_t (&q_arms)[2], uint32_t kv_arms,
                            unsigned* err) {
  int none = 0;
  for (int t = 0; t < 2; ++t)
    if (q_arms[t] > 0) mbar_wait(&bars->q_full[t], (q_arms[t] - 1) & 1, &none, err, kErrTimeoutDrain);
  for (uint32_t s = 0; s < static_cast<uint32_t>(kTcStages); ++s) {
    if (kv_arms <= s) continue;
    const uint32_t arms = (kv_arms - 1 - s) / kTcStages + 1;  // times stage s was armed
    mbar_wait(&bars->k_full[s], (arms - 1) & 1, &none, err, kErrTimeoutDrain);
    mbar_wait(&bars->v_full[s], (arms - 1) & 1, &none, err, kErrTimeoutDrain);
  }
}

__device__ __forceinline__ void run_producer(const CUtensorMap* tmQ, const CUtensorMap* tmK,
                             const CUtensorMap* tmV, const TcParams& p, uint8_t* sQ, uint8_t* sK,
                             uint8_t* sV, TcBars* bars) {
  volatile int* abort_flag = &bars->abort_flag;
  uint32_t q_use[2] = {0, 0};
  uint32_t kv_cnt = 0;
  bool ok = true;
  // The operands may come from the preceding kernel (programmatic dependent
  // launch) unless the caller says they do not.
  if (!p.inputs_stable) griddep_wait();
  for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
    TcUnit w;
    unit_at(p, u, w);
    const int qs = __ldg(p.q_start + w.seq);
    const int ks = __ldg(p.k_start + w.seq);
    for (int t = 0; ok && t < w.ntiles; ++t) {
      if (q_use[t] > 0 &&
          !warp_wait(&bars->q_empty[t], (q_use[t] - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      int c1, c2;
      box_coords(p.q_token_major, qs, p.heads, w.seq, w.head, w.row0 + t * kTcRows, c1, c2);
      mbar_arrive_expect_tx_w(&bars->q_full[t], kTileBytes);
      tma_load_3d_w(sQ + t * kTileBytes, tmQ, &bars->q_full[t], 0, c1, c2);
      ++q_use[t];
    }
    const int nblk = unit_blocks(p, w);
    for (int j = 0; ok && j < nblk; ++j) {
      const uint32_t s = kv_cnt % kTcStages;
      if (kv_cnt >= static_cast<uint32_t>(kTcStages) &&
          !warp_wait(&bars->kv_empty[s], ((kv_cnt / kTcStages) - 1) & 1, abort_flag, p.err,
                     kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      int c1, c2;
      box_coords(p.k_token_major, ks, p.heads, w.seq, w.head, j * kTcKeys, c1, c2);
      mbar_arrive_expect_tx_w(&bars->k_full[s], kTileBytes);
      tma_load_3d_w(sK + s * kTileBytes, tmK, &bars->k_full[s], 0, c1, c2);
      box_coords(p.v_token_major, ks, p.heads, w.seq, w.head, j * kTcKeys, c1, c2);
      mbar_arrive_expect_tx_w(&bars->v_full[s], kTileBytes);
      tma_load_3d_w(sV + s * kTileBytes, tmV, &bars->v_full[s], 0, c1, c2);
      ++kv_cnt;
    }
  }
  if (!ok || *abort_flag) drain_loads(bars, q_use, kv_cnt, p.err);
}

// ---------------------------------------------------------------- MMA issuer
struct MmaState {
  uint32_t q_use[2];   // Q tiles consumed per tile slot
  uint32_t s_cnt[2];   // S MMAs issued per tile slot
  uint32_t pv_cnt[2];  // P.V groups issued per tile slot
  uint32_t k_ready;    // (block index whose K stage has been waited for) + 1
};

template <int AB_F16>
__device__ __forceinline__ bool issue_s(int t, bool first_of_unit, bool last_of_unit, uint32_t g,
                                        MmaState& st, uint8_t* sQ, uint8_t* sK, uint32_t tmem,
                                        TcBars* bars, unsigned* err) {
  volatile int* abort_flag = &bars->abort_flag;
  const uint32_t s = g % kTcStages;
  if (st.k_ready != g + 1) {
    if (!warp_wait(&bars->k_full[s], (g / kTcStages) & 1, abort_flag, err, kErrTimeoutMma))
      return false;
    st.k_ready = g + 1;
  }
  if (first_of_unit) {
    if (!warp_wait(&bars->q_full[t], st.q_use[t] & 1, abort_flag, err, kErrTimeoutMma)) return false;
    ++st.q_use[t];
  }
  // S_t is about to be overwritten: the softmax must have read the last one.
  if (st.s_cnt[t] > 0 &&
      !warp_wait(&bars->sc_done[t], (st.s_cnt[t] - 1) & 1, abort_flag, err, kErrTimeoutMma))
    return false;
  tc_fence_after();
  constexpr uint32_t idesc = idesc_f16(AB_F16 ? 0u : 1u, kTcRows, kTcKeys, 0, 0);
  const uint64_t dq = smem_desc_sw128(smem_u32(sQ + t * kTileBytes), 16, 1024);
  const uint64_t dk = smem_desc_sw128(smem_u32(sK + s * kTileBytes), 16, 1024);
#pragma unroll
  for (int k = 0; k < 4; ++k)  // K = 64 = 4 x 16; +32 bytes per step inside the swizzle atom
    mma_ss_w(tmem + kColS + t * 128, dq + 2 * k, dk + 2 * k, idesc, k > 0 ? 1u : 0u);
  mma_commit_w(&bars->s_full[t]);
  ++st.s_cnt[t];
  if (last_of_unit) mma_commit_w(&bars->q_empty[t]);
  return true;
}

// One MMA thread per Q tile, so the two tiles' chains (S -> softmax -> P.V)
// advance independently; they meet only in the K/V ring, whose stages are
// released when both threads have finished with them (kv_empty counts 2).
// A thread whose tile is absent from a unit still walks that unit's blocks
// and arrives on kv_empty for each, after waiting for the block's V, so its
// arrivals can never run ahead into a later phase of the same stage.
template <int AB_F16>
__device__ __forceinline__ void run_mma(const TcParams& p, int t, uint8_t* sQ, uint8_t* sK,
                                        uint8_t* sV, uint32_t tmem, TcBars* bars) {
  volatile int* abort_flag = &bars->abort_flag;
  MmaState st{};
  int u = blockIdx.x;
  if (u >= p.num_units) return;
  TcUnit cur;
  unit_at(p, u, cur);
  int cur_nblk = unit_blocks(p, cur);
  int cur_tb = tile_blocks(p, cur, t);  // blocks this tile computes (a prefix of the unit's)
  int j = 0;
  uint32_t g = 0;
  if (cur_tb > 0 && !issue_s<AB_F16>(t, true, cur_tb == 1, g, st, sQ, sK, tmem, bars, p.err))
    return;

  // P.V: M=128, N=64, A = P from TMEM, B = V MN-major (head dim contiguous).
  constexpr uint32_t idesc_pv = idesc_f16(AB_F16 ? 0u : 1u, kTcRows, 64, 0, 1);
  while (true) {
    // Next block in this CTA's flat sequence of (unit, key block).
    TcUnit nxt = cur;
    int nxt_j = j + 1, nxt_nblk = cur_nblk, nxt_tb = cur_tb;
    bool has_next = true;
    if (nxt_j >= cur_nblk) {
      const int nu = u + gridDim.x;
      if (nu < p.num_units) {
        unit_at(p, nu, nxt);
        nxt_j = 0;
        nxt_nblk = unit_blocks(p, nxt);
        nxt_tb = tile_blocks(p, nxt, t);
      } else {
        has_next = false;
      }
    }
    // Across a unit boundary the order flips: the unit's last P.V goes
    // first, since the softmax waits for it before its epilogue, which
    // leaves the next unit's first scores plenty of time.
    const bool next_first = has_next && nxt_j < nxt_tb;
    const bool boundary = nxt_j == 0;
    if (next_first && !boundary &&
        !issue_s<AB_F16>(t, nxt_j == 0, nxt_j == nxt_tb - 1, g + 1, st, sQ, sK, tmem, bars,
                         p.err))
      return;
    const uint32_t s = g % kTcStages;
    if (!warp_wait(&bars->v_full[s], (g / kTcStages) & 1, abort_flag, p.err, kErrTimeoutMma)) return;
    if (j < cur_tb) {
      if (!warp_wait(&bars->p_full[t], st.pv_cnt[t] & 1, abort_flag, p.err, kErrTimeoutMma))
        return;
      tc_fence_after();
      const uint64_t dv = smem_desc_sw128(smem_u32(sV + s * kTileBytes), 8192, 1024);
      const uint32_t tp = tmem + kColP + t * 64;  // P_t: bf16 pairs
#pragma unroll
      for (int k = 0; k < 8; ++k)  // 128 keys = 8 x 16; V advances 16 rows = 2048 B per step
        mma_ts_w(tmem + kColO + t * 64, tp + k * 8, dv + k * (2048 >> 4), idesc_pv,
               (j > 0 || k > 0) ? 1u : 0u);
      mma_commit_w(&bars->o_done[t]);
      ++st.pv_cnt[t];
      mma_commit_w(&bars->kv_empty[s]);
    } else {
      mbar_arrive_w(&bars->kv_empty[s]);
    }
    if (next_first && boundary &&
        !issue_s<AB_F16>(t, true, nxt_tb == 1, g + 1, st, sQ, sK, tmem, bars, p.err))
      return;
    if (!has_next) break;
    if (nxt_j == 0) u += gridDim.x;
    cur = nxt;
    cur_nblk = nxt_nblk;
    cur_tb = nxt_tb;
    j = nxt_j;
    ++g;
  }
}

// ---------------------------------------------------------------- softmax + epilogue
// Store this thread's quarter of one output row, scaled by `inv`: head dims
// 8k + 2 t0 and 8k + 2 t0 + 1 (k = 0..7) of row v of the 16x256b layout.
__device__ __forceinline__ void store_row_quarter(const TcParams& p, const TcUnit& w, int row,
                                                  int t0, const uint32_t (&o)[32], int v,
                                                  float inv) {
  long long base;
  if (p.out_token_major)
    base = (static_cast<long long>(__ldg(p.q_start + w.seq) + row) * p.heads + w.head) * 64;
  else
    base = ((static_cast<long long>(w.seq) * p.heads + w.head) * p.out_rows + row) * 64;
  base += 2 * t0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float a = __uint_as_float(o[4 * k + 2 * v]) * inv;
    const float b = __uint_as_float(o[4 * k + 2 * v + 1]) * inv;
    if (p.out_bf16)
      *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(p.out) + base + 8 * k) =
          pack_bf16x2(a, b);
    else
      *reinterpret_cast<float2*>(static_cast<float*>(p.out) + base + 8 * k) = make_float2(a, b);
  }
}

// Which pairs take the polynomial exp2 (FMA pipe) instead of MUFU ex2:
// kPolyOf8 of every 8 (full blocks only; a block with masked keys uses MUFU
// throughout).  MUFU sustains 16 ex2 per clock per SM and the exponentials
// of a block pair need 2048 of its cycles; the polynomial costs about ten
// issue slots per pair on the FMA pipe.  Measured on the long-form encoder
// workload, 64 / 8 segments (TFLOP/s): 0 -> 794 / 762, 1 -> 798 / 766,
// 2 -> 786 / 751, and 1 at k % 8 == 4 instead of 0 -> 778 / 754.
constexpr int kPolyOf8 = 1;

// f32 += one 16-bit half of a packed pair, in one instruction.
template <int AB_F16>
__device__ __forceinline__ float add_half_lo(float acc, uint32_t pk) {
  if (AB_F16)
    asm("{ .reg .b16 l, h;\n mov.b32 {l, h}, %1;\n add.rn.f32.f16 %0, l, %0;\n}"
        : "+f"(acc) : "r"(pk));
  else
    asm("{ .reg .b16 l, h;\n mov.b32 {l, h}, %1;\n add.rn.f32.bf16 %0, l, %0;\n}"
        : "+f"(acc) : "r"(pk));
  return acc;
}

template <int AB_F16>
__device__ __forceinline__ float add_half_hi(float acc, uint32_t pk) {
  if (AB_F16)
    asm("{ .reg .b16 l, h;\n mov.b32 {l, h}, %1;\n add.rn.f32.f16 %0, h, %0;\n}"
        : "+f"(acc) : "r"(pk));
  else
    asm("{ .reg .b16 l, h;\n mov.b32 {l, h}, %1;\n add.rn.f32.bf16 %0, h, %0;\n}"
        : "+f"(acc) : "r"(pk));
  return acc;
}

// Exponentiate this thread's 64 raw scores of its two rows (v = 0, 1),
// p = 2^(s * sl2 - m_v), and pack them into the 16-bit pairs the 16x128b
// store writes: pk[2k + v] holds the keys 8k + 2 t0 and 8k + 2 t0 + 1 of row
// v, i.e. P word 4k + t0.  Adds the rounded (packed) values to sum[v].
//
// The polynomial path (FMA pipe) takes x = s * sl2 - m clamped at -125 and
// splits it by the 1.5 * 2^23 trick: t = x + 1.5*2^23 holds round(x) in its
// low mantissa bits (exact), f = x - round(x) in [-0.5, 0.5] (exact); 2^f by
// a degree-3 polynomial (this project's own minimax fit of 2^f on
// [-0.5, 0.5], max relative error 7.5e-5) and round(x) spliced into the
// exponent field.  The clamp keeps the splice in range and f bounded: a score
// more than 125 below the row's reference gives 2^-125 or so, negligible
// beside the reference's 1 (an unclamped f there made the cubic, and with it
// the spliced value, large).
template <int AB_F16, bool kTail>
__device__ __forceinline__ void exp_pack_rows(const float* sf, float sl2, const float (&m)[2],
                                              uint32_t (&pk)[32], float (&sum)[2]) {
  const float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t magic2 = f2_pack(kMagic, kMagic);
  uint64_t n2[2];
#pragma unroll
  for (int v = 0; v < 2; ++v) {
    const float neg = (m[v] == -INFINITY) ? 0.f : -m[v];
    n2[v] = f2_pack(neg, neg);
  }
  const uint64_t kC3 = f2_pack(0.055171434f, 0.055171434f);
  const uint64_t kC2 = f2_pack(0.24261081f, 0.24261081f);
  const uint64_t kC1 = f2_pack(0.69326097f, 0.69326097f);
  const uint64_t kC0 = f2_pack(0.99992812f, 0.99992812f);
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
  for (int k = 0; k < 16; ++k) {
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      float p0, p1;
      const uint64_t sv = f2_pack(sf[4 * k + 2 * v], sf[4 * k + 2 * v + 1]);
      if (!kTail && (k % 8) < kPolyOf8) {
        float x0, x1;
        f2_unpack(f2_fma(sv, c2, n2[v]), x0, x1);
        const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
        const uint64_t t = f2_add(x, magic2);               // 1.5*2^23 + round(x)
        const uint64_t f = f2_sub(x, f2_sub(t, magic2));    // x - round(x)
        float t0, t1;
        f2_unpack(t, t0, t1);
        uint64_t q = f2_fma(kC3, f, kC2);
        q = f2_fma(q, f, kC1);
        q = f2_fma(q, f, kC0);
        float q0, q1;
        f2_unpack(q, q0, q1);
        // (bits(t) << 23) == round(x) << 23 modulo 2^32
        p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
        p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
      } else {  // MUFU; masked columns are -inf and give exactly 0
        float x0, x1;
        f2_unpack(f2_fma(sv, c2, n2[v]), x0, x1);
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      const uint32_t w = AB_F16 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
      pk[2 * k + v] = w;
      acc[v][k & 1] = add_half_hi<AB_F16>(add_half_lo<AB_F16>(acc[v][k & 1], w), w);
    }
  }
  sum[0] = acc[0][0] + acc[0][1];
  sum[1] = acc[1][0] + acc[1][1];
}

// Softmax warp w (0..15) serves tile t = w / 8, TMEM lanes [lb, lb + 16) with
// lb = 32 (w % 4) + 16 ((w / 4) % 2): each lane quarter is reachable only from
// warps with the same w % 4.  Thread (t0, t1) = (lane % 4, lane / 4) handles
// rows lb + t1 and lb + t1 + 8, a quarter of each row's columns; the four
// threads of a row reduce its max and sum with two shuffles.
template <int AB_F16, bool CAUSAL>
__device__ __forceinline__ void run_softmax(const TcParams& p, uint32_t tmem, TcBars* bars,
                                            const CUtensorMap* tmO, uint8_t* sO) {
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int t = warp / 8;
  const int lb = 32 * (warp % 4) + 16 * ((warp / 4) % 2);
  const int t0 = lane & 3, t1 = lane >> 2;
  const uint32_t lane_addr = static_cast<uint32_t>(lb) << 16;
  const uint32_t tS = tmem + lane_addr + kColS + t * 128;
  const uint32_t tP = tmem + lane_addr + kColP + t * 64;
  const uint32_t tO = tmem + lane_addr + kColO + t * 64;
  const float sl2 = p.scale_log2;
  uint32_t s_cnt = 0, pv_cnt = 0;

  bool dependency_done = false;
  for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
    TcUnit w;
    unit_at(p, u, w);
    if (t >= w.ntiles) continue;
    const int kv_len = __ldg(p.k_len + w.seq);
    const int nblk = CAUSAL ? tile_blocks(p, w, t) : (kv_len + kTcKeys - 1) / kTcKeys;
    // Keys visible to this thread's two rows: all kv_len, or with `causal`
    // those up to q_offset + row.
    int lim[2] = {kv_len, kv_len};
    if constexpr (CAUSAL) {
#pragma unroll
      for (int v = 0; v < 2; ++v)
        lim[v] = min(kv_len, p.q_offset + w.row0 + t * kTcRows + lb + t1 + 8 * v + 1);
    }
    float m_run[2] = {-INFINITY, -INFINITY};  // per row: log2 domain, integer-valued
    float l_run[2] = {0.f, 0.f};              // per row: this thread's share of the sum

    for (int j = 0; j < nblk; ++j) {
      if (!warp_wait(&bars->s_full[t], s_cnt & 1, abort_flag, p.err, kErrTimeoutSoftmax)) return;
      ++s_cnt;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld_16x256b_x16(tS, sr);
      tmem_wait_ld();
      // S_t is in registers: the next block's scores may overwrite it.
      tc_fence_before();
      mbar_arrive(&bars->sc_done[t]);
      float* sf = reinterpret_cast<float*>(sr);

      // Valid keys of this block per row (the sequence's tail, or the causal
      // diagonal); columns past them are -inf and exponentiate to exactly 0.
      const int rem0 = lim[0] - j * kTcKeys, rem1 = lim[1] - j * kTcKeys;
      const bool tail = (CAUSAL ? min(rem0, rem1) : rem0) < kTcKeys;
      if (tail) {
#pragma unroll
        for (int k = 0; k < 16; ++k)
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int col = 8 * k + 2 * t0 + x;
            if constexpr (CAUSAL) {
              if (col >= rem0) sf[4 * k + x] = -INFINITY;
              if (col >= rem1) sf[4 * k + 2 + x] = -INFINITY;
            } else if (col >= rem0) {
              sf[4 * k + x] = sf[4 * k + 2 + x] = -INFINITY;
            }
          }
      }
      float mx[2];
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        float a = fmaxf(sf[2 * v], sf[2 * v + 1]), b = fmaxf(sf[4 + 2 * v], sf[4 + 2 * v + 1]);
#pragma unroll
        for (int k = 2; k < 16; k += 2) {
          a = max3f(a, sf[4 * k + 2 * v], sf[4 * k + 2 * v + 1]);
          b = max3f(b, sf[4 * k + 4 + 2 * v], sf[4 * k + 4 + 2 * v + 1]);
        }
        mx[v] = fmaxf(a, b);  // this thread's quarter of the row
      }
      // Move a row's running max only when it grows by more than 8 (a factor
      // of 256): P stays <= 256, exact in f32 sums and in bf16's exponent
      // range.  It is kept integer-valued, so corrections are exact powers of
      // two and the polynomial exp2 can fold its range reduction into the
      // scaling FMA.  A row can only grow if one of its quarters does, so
      // the quarters' maxima are combined (shuffles) only when some thread of
      // the warp sees growth: on a unit's first block, and rarely after.
      float corr[2] = {1.f, 1.f};
      bool grow_any = false;
      if (__any_sync(0xffffffffu,
                     mx[0] * sl2 > m_run[0] + 8.0f || mx[1] * sl2 > m_run[1] + 8.0f)) {
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          mx[v] = fmaxf(mx[v], __shfl_xor_sync(0xffffffffu, mx[v], 1));
          mx[v] = fmaxf(mx[v], __shfl_xor_sync(0xffffffffu, mx[v], 2));
          const float m_blk = mx[v] * sl2;
          if (m_blk > m_run[v] + 8.0f) {
            const float m_new = ceilf(m_blk);
            corr[v] = ex2_approx(m_run[v] - m_new);  // 0 when m_run is -inf
            m_run[v] = m_new;
            grow_any = true;
          }
        }
      }
      uint32_t pk[32];
      float bsum[2];
      if (tail)
        exp_pack_rows<AB_F16, true>(sf, sl2, m_run, pk, bsum);
      else
        exp_pack_rows<AB_F16, false>(sf, sl2, m_run, pk, bsum);
      l_run[0] = fmaf(l_run[0], corr[0], bsum[0]);
      l_run[1] = fmaf(l_run[1], corr[1], bsum[1]);
      // P_t and O_t are free once the previous P_t.V has completed.
      if (pv_cnt > 0 &&
          !warp_wait(&bars->o_done[t], (pv_cnt - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax))
        return;
      tc_fence_after();
      if (__any_sync(0xffffffffu, grow_any && j > 0)) {
        if constexpr (!CAUSAL) {
          // In 16-column chunks: eight registers at a time instead of 32
          // keeps this rare path from raising the loop's register pressure
          // (measured: 766 -> 788 TFLOP/s on the long-form encoder workload;
          // the causal instance compiles without spills only as one load).
#pragma unroll 1
          for (int h = 0; h < 4; ++h) {
            uint32_t orr[8];
            tmem_ld_16x256b_x2(tO + 16 * h, orr);
            tmem_wait_ld_regs8(orr);
#pragma unroll
            for (int c = 0; c < 8; ++c)
              orr[c] = __float_as_uint(__uint_as_float(orr[c]) * corr[(c >> 1) & 1]);
            tmem_st_16x256b_x2(tO + 16 * h, orr);
          }
        } else {
          uint32_t orr[32];
          tmem_ld_16x256b_x8(tO, orr);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c)
            orr[c] = __float_as_uint(__uint_as_float(orr[c]) * corr[(c >> 1) & 1]);
          tmem_st_16x256b_x8(tO, orr);
        }
      }
      tmem_st_16x128b_x16(tP, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
      ++pv_cnt;
    }

    // Epilogue: O_t / l to global memory.
    if (!warp_wait(&bars->o_done[t], (pv_cnt - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) return;
    tc_fence_after();
    // out and lse may still be read or written by the preceding kernel.
    if (!dependency_done) {
      griddep_wait();
      dependency_done = true;
    }
    uint32_t orr[32];
    tmem_ld_16x256b_x8(tO, orr);
    tmem_wait_ld();
    const int q_len = __ldg(p.q_len + w.seq);
    const int row_base = w.row0 + t * kTcRows + lb;  // the warp's 16 rows
    // bf16 output with all 16 rows inside the sequence: one TMA store per
    // warp from its staging buffer (the TMEM layout's 4-byte pieces are
    // scattered over 8 rows; the tensor store writes whole rows).
    const bool tma = p.o_tma && row_base + 16 <= q_len;
    uint8_t* stg = sO + warp * kStageBytes;
    if (tma) {
      if (lane == 0) bulk_wait_read_all();  // the previous store has read the buffer
      __syncwarp();
    }
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      float l = l_run[v];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      l_run[v] = l;
      const int row = row_base + t1 + 8 * v;
      if (tma) {
        // row r = t1 + 8 v of the box, 16-byte chunk k at k ^ (r % 8) = k ^ t1
        const float inv = 1.f / l;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<uint32_t*>(stg + (t1 + 8 * v) * 128 + ((k ^ t1) << 4) + 4 * t0) =
              pack_bf16x2(__uint_as_float(orr[4 * k + 2 * v]) * inv,
                          __uint_as_float(orr[4 * k + 2 * v + 1]) * inv);
      } else if (row < q_len) {
        store_row_quarter(p, w, row, t0, orr, v, 1.f / l);
      }
    }
    if (tma) {
      fence_proxy_async_smem();  // the generic-proxy writes, seen by the tensor store
      __syncwarp();
      if (lane == 0) {
        if (p.out_token_major)
          tma_store_3d(tmO, stg, 0, w.head, __ldg(p.q_start + w.seq) + row_base);
        else
          tma_store_3d(tmO, stg, 0, row_base, w.seq * p.heads + w.head);
        bulk_commit();
      }
    }
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const float l = l_run[v];
      const int row = row_base + t1 + 8 * v;
      if (row < q_len) {
        if (p.lse && t0 == 0) {
          const float lse = (m_run[v] + __log2f(l)) * 0.69314718055994530942f;
          if (p.out_token_major)
            p.lse[static_cast<long long>(w.head) * p.lse_tokens + __ldg(p.q_start + w.seq) + row] = lse;
          else
            p.lse[(static_cast<long long>(w.seq) * p.heads + w.head) * p.out_rows + row] = lse;
        }
      }
    }
    // The next unit's first P.V overwrites O_t only after this thread's next
    // P arrive, which follows these TMEM reads in program order.
    tc_fence_before();
  }
}

template <int AB_F16, bool CAUSAL>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmO, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kTileBytes;
  uint8_t* sV = sK + kTcStages * kTileBytes;
  uint8_t* sO = sV + kTcStages * kTileBytes;  // 16 x kStageBytes, 1024-byte aligned
  TcBars* bars = reinterpret_cast<TcBars*>(sO + 16 * kStageBytes);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->q_full[t], 1);
      mbar_init(&bars->q_empty[t], 1);
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->sc_done[t], 256);  // the tile's 8 softmax warps
      mbar_init(&bars->p_full[t], 256);
      mbar_init(&bars->o_done[t], 1);
    }
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 2);  // one arrival per tile's MMA thread
    }
    mbar_init(&bars->drain, 2);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpProducer) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpMma0 && lane == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    if (p.o_tma) prefetch_tensormap(&tmO);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Every CTA is resident: the next kernel on the stream may start its CTAs
  // on the SMs this grid leaves (it waits for this grid before it reads what
  // this grid writes).
  griddep_launch_dependents();

  if (warp == kWarpProducer) {
    run_producer(&tmQ, &tmK, &tmV, p, sQ, sK, sV, bars);
  } else if (warp == kWarpMma0 || warp == kWarpMma0 + 1) {
    run_mma<AB_F16>(p, warp - kWarpMma0, sQ, sK, sV, tmem, bars);
    // Wait for every MMA either warp issued before TMEM is released.
    int none = 0;
    mma_commit_w(&bars->drain);
    mbar_wait(&bars->drain, 0, &none, p.err, kErrTimeoutDrain);
  } else {
    run_softmax<AB_F16, CAUSAL>(p, tmem, bars, &tmO, sO);
    if (lane == 0 && p.o_tma) bulk_wait_all();  // output stores complete before exit
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpProducer) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

size_t prefill_tc_smem_bytes() { return kSmemBytes; }

cudaError_t launch_prefill_tc(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                              const CUtensorMap& tmV, const CUtensorMap& tmO, const TcParams& p,
                              int grid, int ab_f16, cudaStream_t s) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[4][64];  // racing first calls both set it
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const int which = ab_f16 * 2 + (p.causal ? 1 : 0);
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
               const TcParams) =
      which == 0   ? prefill_tc_kernel<0, false>
      : which == 1 ? prefill_tc_kernel<0, true>
      : which == 2 ? prefill_tc_kernel<1, false>
                   : prefill_tc_kernel<1, true>;
  if (!configured[which][dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured[which][dev].store(true, std::memory_order_release);
  }
  // A programmatic dependent of the preceding kernel: see run_producer and
  // the epilogue for the two waits.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tmQ, tmK, tmV, tmO, p);
}

}  // namespace ffai
