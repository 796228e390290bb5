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
//   warp 8      TMA producer: Q tiles, then a 3-stage ring of K/V blocks of
//               128 keys (16 KB each, 128-byte swizzle).  Also owns TMEM.
//   warp 9      MMA issuer (one thread):  S_t = Q_t K^T   (M=128, N=128, K=64)
//                                         O_t += P_t V    (M=128, N=64,  K=128)
//               with P_t read straight from tensor memory (the "A in TMEM"
//               form), so probabilities never touch shared memory.
//   warps 0-3   softmax for tile 0, warps 4-7 for tile 1: one thread per
//               query row.  Each thread loads its row of S from TMEM, takes
//               the block max, exponentiates in the log2 domain, keeps the
//               row sum in f32 and writes bf16 P back over S.  The running
//               max is only moved (and O rescaled in TMEM) when it grows by
//               more than 2^8, so most blocks never touch O.  The last block
//               is followed by the epilogue: O / sum to global memory.
//
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,320),
// O1 [320,384).  P_t aliases the first 64 columns of S_t.
//
// Every wait is bounded (common.cuh); on a timeout the CTA raises an error
// bit, drains its MMAs and TMA loads, frees TMEM and exits.
#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr uint32_t kTileBytes = kTcRows * 64 * 2;  // 16 KB: 128 rows x 128 B
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;

struct __align__(8) TcBars {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kTcStages], v_full[kTcStages], kv_empty[kTcStages];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kSmemTiles = (2 + 2 * kTcStages) * kTileBytes;
constexpr size_t kSmemBytes = kSmemTiles + sizeof(TcBars) + 1024;  // +1024: alignment slack

__device__ __forceinline__ void unit_at(const TcParams& p, int u, TcUnit& out) {
  const int4 w = __ldg(p.units + u);
  out.seq = w.x;
  out.head = w.y;
  out.row0 = w.z;
  out.ntiles = w.w;
}

__device__ __forceinline__ int num_blocks(const TcParams& p, int seq) {
  return (__ldg(p.k_len + seq) + kTcKeys - 1) / kTcKeys;
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
  for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
    TcUnit w;
    unit_at(p, u, w);
    const int qs = __ldg(p.q_start + w.seq);
    const int ks = __ldg(p.k_start + w.seq);
    for (int t = 0; ok && t < w.ntiles; ++t) {
      if (q_use[t] > 0 &&
          !mbar_wait(&bars->q_empty[t], (q_use[t] - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      int c1, c2;
      box_coords(p.q_token_major, qs, p.heads, w.seq, w.head, w.row0 + t * kTcRows, c1, c2);
      mbar_arrive_expect_tx(&bars->q_full[t], kTileBytes);
      tma_load_3d(sQ + t * kTileBytes, tmQ, &bars->q_full[t], 0, c1, c2);
      ++q_use[t];
    }
    const int nblk = num_blocks(p, w.seq);
    for (int j = 0; ok && j < nblk; ++j) {
      const uint32_t s = kv_cnt % kTcStages;
      if (kv_cnt >= static_cast<uint32_t>(kTcStages) &&
          !mbar_wait(&bars->kv_empty[s], ((kv_cnt / kTcStages) - 1) & 1, abort_flag, p.err,
                     kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      int c1, c2;
      box_coords(p.k_token_major, ks, p.heads, w.seq, w.head, j * kTcKeys, c1, c2);
      mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
      tma_load_3d(sK + s * kTileBytes, tmK, &bars->k_full[s], 0, c1, c2);
      box_coords(p.v_token_major, ks, p.heads, w.seq, w.head, j * kTcKeys, c1, c2);
      mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
      tma_load_3d(sV + s * kTileBytes, tmV, &bars->v_full[s], 0, c1, c2);
      ++kv_cnt;
    }
  }
  if (!ok || *abort_flag) drain_loads(bars, q_use, kv_cnt, p.err);
}

// ---------------------------------------------------------------- MMA issuer
struct MmaState {
  uint32_t kv_cnt;     // K/V blocks consumed (global over units)
  uint32_t q_use[2];   // Q tiles consumed per tile slot
  uint32_t pv_cnt[2];  // PV groups issued per tile slot
  uint32_t k_ready;    // kv_cnt value whose K stage has been waited for, +1
};

template <int AB_F16>
__device__ __forceinline__ bool issue_s(int t, bool first_of_unit, bool last_of_unit, uint32_t g, MmaState& st,
                        uint8_t* sQ, uint8_t* sK, uint32_t tmem, TcBars* bars, unsigned* err) {
  volatile int* abort_flag = &bars->abort_flag;
  const uint32_t s = g % kTcStages;
  if (st.k_ready != g + 1) {
    if (!mbar_wait(&bars->k_full[s], (g / kTcStages) & 1, abort_flag, err, kErrTimeoutMma))
      return false;
    st.k_ready = g + 1;
  }
  if (first_of_unit) {
    if (!mbar_wait(&bars->q_full[t], st.q_use[t] & 1, abort_flag, err, kErrTimeoutMma)) return false;
    ++st.q_use[t];
  }
  // S_t / P_t are about to be overwritten: the previous P_t.V must have read P_t.
  if (st.pv_cnt[t] > 0 &&
      !mbar_wait(&bars->o_done[t], (st.pv_cnt[t] - 1) & 1, abort_flag, err, kErrTimeoutMma))
    return false;
  tc_fence_after();
  constexpr uint32_t idesc = idesc_f16(AB_F16 ? 0u : 1u, kTcRows, kTcKeys, 0, 0);
  const uint64_t dq = smem_desc_sw128(smem_u32(sQ + t * kTileBytes), 16, 1024);
  const uint64_t dk = smem_desc_sw128(smem_u32(sK + s * kTileBytes), 16, 1024);
#pragma unroll
  for (int k = 0; k < 4; ++k)  // K = 64 = 4 x 16; +32 bytes per step inside the swizzle atom
    mma_ss(tmem + kColS + t * 128, dq + 2 * k, dk + 2 * k, idesc, k > 0 ? 1u : 0u);
  mma_commit(&bars->s_full[t]);
  if (last_of_unit) mma_commit(&bars->q_empty[t]);
  return true;
}

template <int AB_F16>
__device__ __forceinline__ void run_mma(const TcParams& p, uint8_t* sQ, uint8_t* sK, uint8_t* sV, uint32_t tmem,
                        TcBars* bars) {
  volatile int* abort_flag = &bars->abort_flag;
  MmaState st{};
  int u = blockIdx.x;
  if (u >= p.num_units) return;
  TcUnit cur;
  unit_at(p, u, cur);
  int cur_nblk = num_blocks(p, cur.seq);
  int j = 0;
  uint32_t g = 0;
  for (int t = 0; t < cur.ntiles; ++t)
    if (!issue_s<AB_F16>(t, true, cur_nblk == 1, g, st, sQ, sK, tmem, bars, p.err)) return;

  constexpr uint32_t idesc_pv = idesc_f16(AB_F16 ? 0u : 1u, kTcRows, 64, 0, 1);
  while (true) {
    // Next block in this CTA's flat sequence of (unit, key block).
    TcUnit nxt = cur;
    int nxt_j = j + 1, nxt_nblk = cur_nblk;
    bool has_next = true;
    if (nxt_j >= cur_nblk) {
      const int nu = u + gridDim.x;
      if (nu < p.num_units) {
        unit_at(p, nu, nxt);
        nxt_j = 0;
        nxt_nblk = num_blocks(p, nxt.seq);
      } else {
        has_next = false;
      }
    }
    const uint32_t s = g % kTcStages;
    if (!mbar_wait(&bars->v_full[s], (g / kTcStages) & 1, abort_flag, p.err, kErrTimeoutMma)) return;
    const uint64_t dv = smem_desc_sw128(smem_u32(sV + s * kTileBytes), 8192, 1024);
    for (int t = 0; t < 2; ++t) {
      if (t < cur.ntiles) {
        if (!mbar_wait(&bars->p_full[t], st.pv_cnt[t] & 1, abort_flag, p.err, kErrTimeoutMma))
          return;
        tc_fence_after();
        const uint32_t tp = tmem + kColS + t * 128;  // P_t: bf16 pairs in the first 64 columns
#pragma unroll
        for (int k = 0; k < 8; ++k)  // 128 keys = 8 x 16; V advances 16 rows = 2048 B per step
          mma_ts(tmem + kColO + t * 64, tp + k * 8, dv + k * (2048 >> 4), idesc_pv,
                 (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&bars->o_done[t]);
        ++st.pv_cnt[t];
      }
      if (has_next && t < nxt.ntiles) {
        if (!issue_s<AB_F16>(t, nxt_j == 0, nxt_j == nxt_nblk - 1, g + 1, st, sQ, sK, tmem, bars,
                             p.err))
          return;
      }
    }
    mma_commit(&bars->kv_empty[s]);
    if (!has_next) break;
    if (nxt_j == 0) u += gridDim.x;
    cur = nxt;
    cur_nblk = nxt_nblk;
    j = nxt_j;
    ++g;
  }
}

// ---------------------------------------------------------------- softmax + epilogue
__device__ __forceinline__ void store_row(const TcParams& p, const TcUnit& w, int row,
                                          const float* o, float inv) {
  if (p.out_bf16) {
    __nv_bfloat16* dst;
    if (p.out_token_major)
      dst = static_cast<__nv_bfloat16*>(p.out) +
            (static_cast<long long>(__ldg(p.q_start + w.seq) + row) * p.heads + w.head) * 64;
    else
      dst = static_cast<__nv_bfloat16*>(p.out) +
            ((static_cast<long long>(w.seq) * p.heads + w.head) * p.out_rows + row) * 64;
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 v;
      v.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
      v.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
      v.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
      v.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
      d4[c] = v;
    }
  } else {
    float* dst;
    if (p.out_token_major)
      dst = static_cast<float*>(p.out) +
            (static_cast<long long>(__ldg(p.q_start + w.seq) + row) * p.heads + w.head) * 64;
    else
      dst = static_cast<float*>(p.out) +
            ((static_cast<long long>(w.seq) * p.heads + w.head) * p.out_rows + row) * 64;
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int c = 0; c < 16; ++c)
      d4[c] = make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv,
                          o[4 * c + 3] * inv);
  }
}

template <int AB_F16>
__device__ __forceinline__ void run_softmax(const TcParams& p, int t, uint32_t tmem, TcBars* bars) {
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int quarter = warp % 4;  // TMEM lanes [32*quarter, 32*quarter+32)
  const int r_in_tile = quarter * 32 + lane;
  const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t tS = tmem + lane_addr + kColS + t * 128;
  const uint32_t tO = tmem + lane_addr + kColO + t * 64;
  const float sl2 = p.scale_log2;
  uint32_t s_cnt = 0, pv_cnt = 0;

  for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
    TcUnit w;
    unit_at(p, u, w);
    if (t >= w.ntiles) continue;
    const int kv_len = __ldg(p.k_len + w.seq);
    const int nblk = (kv_len + kTcKeys - 1) / kTcKeys;
    float m_run = -INFINITY;  // running max, log2 domain, scaled
    float l_run = 0.f;

    for (int j = 0; j < nblk; ++j) {
      if (!warp_wait(&bars->s_full[t], s_cnt & 1, abort_flag, p.err, kErrTimeoutSoftmax)) return;
      ++s_cnt;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
      tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
      tmem_wait_ld();
      float* sf = reinterpret_cast<float*>(sr);

      const int rem = kv_len - j * kTcKeys;
      if (rem < kTcKeys) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= rem) sf[c] = -INFINITY;
      }
      float mx0 = sf[0], mx1 = sf[1], mx2 = sf[2], mx3 = sf[3];
#pragma unroll
      for (int c = 4; c < 128; c += 4) {
        mx0 = fmaxf(mx0, sf[c]);
        mx1 = fmaxf(mx1, sf[c + 1]);
        mx2 = fmaxf(mx2, sf[c + 2]);
        mx3 = fmaxf(mx3, sf[c + 3]);
      }
      const float m_blk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
      // Move the running max only when it grows by more than 8 (a factor of
      // 256): P stays <= 256, exact in f32 sums and in bf16's exponent range.
      const bool grow = m_blk > m_run + 8.0f;
      float corr = 1.f;
      if (grow) {
        corr = ex2_approx(m_run - m_blk);  // 0 when m_run is -inf
        m_run = m_blk;
      }
      const float neg = (m_run == -INFINITY) ? 0.f : -m_run;
      float sum0 = 0.f, sum1 = 0.f, sum2 = 0.f, sum3 = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = ex2_approx(fmaf(sf[2 * c + 0], sl2, neg));
        const float p1 = ex2_approx(fmaf(sf[2 * c + 1], sl2, neg));
        const float p2 = ex2_approx(fmaf(sf[2 * c + 2], sl2, neg));
        const float p3 = ex2_approx(fmaf(sf[2 * c + 3], sl2, neg));
        sum0 += p0;
        sum1 += p1;
        sum2 += p2;
        sum3 += p3;
        if (AB_F16) {
          pk[c] = pack_f16x2(p0, p1);
          pk[c + 1] = pack_f16x2(p2, p3);
        } else {
          pk[c] = pack_bf16x2(p0, p1);
          pk[c + 1] = pack_bf16x2(p2, p3);
        }
      }
      l_run = fmaf(l_run, corr, (sum0 + sum1) + (sum2 + sum3));
      tmem_st32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(pk + 0));
      tmem_st32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(pk + 32));
      tmem_wait_st();
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        // Rescale this warp's rows of O_t once the previous P.V has landed.
        // Done after P is written, when the S registers are dead; the P
        // arrive below still orders it before this block's P.V.
        if (!warp_wait(&bars->o_done[t], (pv_cnt - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax))
          return;
        tc_fence_after();
        uint32_t orr[64];
        tmem_ld32(tO + 0, *reinterpret_cast<uint32_t(*)[32]>(orr + 0));
        tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(orr + 32));
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * corr);
        tmem_st32(tO + 0, *reinterpret_cast<uint32_t(*)[32]>(orr + 0));
        tmem_st32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(orr + 32));
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
      ++pv_cnt;
    }

    // Epilogue: O_t / l to global memory.
    if (!warp_wait(&bars->o_done[t], (pv_cnt - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) return;
    tc_fence_after();
    uint32_t orr[64];
    tmem_ld32(tO + 0, *reinterpret_cast<uint32_t(*)[32]>(orr + 0));
    tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(orr + 32));
    tmem_wait_ld();
    const int row = w.row0 + t * kTcRows + r_in_tile;
    const int q_len = __ldg(p.q_len + w.seq);
    if (row < q_len) {
      const float inv = 1.f / l_run;
      store_row(p, w, row, reinterpret_cast<const float*>(orr), inv);
      if (p.lse) {
        const float lse = (m_run + __log2f(l_run)) * 0.69314718055994530942f;
        if (p.out_token_major)
          p.lse[static_cast<long long>(w.head) * p.lse_tokens + __ldg(p.q_start + w.seq) + row] = lse;
        else
          p.lse[(static_cast<long long>(w.seq) * p.heads + w.head) * p.out_rows + row] = lse;
      }
    }
    // The next unit's first P.V overwrites O_t only after this thread's next
    // P arrive, which follows these TMEM reads in program order.
    tc_fence_before();
  }
}

template <int AB_F16>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kTileBytes;
  uint8_t* sV = sK + kTcStages * kTileBytes;
  TcBars* bars = reinterpret_cast<TcBars*>(sV + kTcStages * kTileBytes);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->q_full[t], 1);
      mbar_init(&bars->q_empty[t], 1);
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 128);
      mbar_init(&bars->o_done[t], 1);
    }
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 9 && lane == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    if (lane == 0) run_producer(&tmQ, &tmK, &tmV, p, sQ, sK, sV, bars);
  } else if (warp == 9) {
    if (lane == 0) {
      run_mma<AB_F16>(p, sQ, sK, sV, tmem, bars);
      // Wait for every MMA this thread issued before TMEM is released.
      int none = 0;
      mma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, &none, p.err, kErrTimeoutDrain);
    }
  } else {
    run_softmax<AB_F16>(p, warp / 4, tmem, bars);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

size_t prefill_tc_smem_bytes() { return kSmemBytes; }

cudaError_t launch_prefill_tc(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                              const CUtensorMap& tmV, const TcParams& p, int grid, int ab_f16,
                              cudaStream_t s) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static bool configured[2][64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[ab_f16][dev]) {
    e = ab_f16 ? cudaFuncSetAttribute(prefill_tc_kernel<1>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kSmemBytes))
               : cudaFuncSetAttribute(prefill_tc_kernel<0>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured[ab_f16][dev] = true;
  }
  if (ab_f16)
    prefill_tc_kernel<1><<<grid, kTcThreads, kSmemBytes, s>>>(tmQ, tmK, tmV, p);
  else
    prefill_tc_kernel<0><<<grid, kTcThreads, kSmemBytes, s>>>(tmQ, tmK, tmV, p);
  return cudaGetLastError();
}

}  // namespace ffai
