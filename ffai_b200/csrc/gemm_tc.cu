// bf16 GEMM on the tensor cores with a fused epilogue, for the projections
// around the attention: out = act(A . B^T + bias) (+ residual).
//
// The reference runs these on candle's CPU GEMM (f32): the encoder's fc1 ->
// GELU -> fc2 with the residual add (audio_encoder.rs:147-165), the q/k/v
// projection whose head split feeds the attention (text_decoder.rs:1083-1124)
// and the out-projection.  Here A (M x K, activations) and B (N x K, weights
// as stored: (out, in)) are bf16, accumulation f32 in tensor memory, and the
// epilogue adds the bias, applies the reference's FastGelu (gelu_scalar,
// text_decoder.rs:341-350, same f32 operations in the same order) and the
// residual, and stores bf16 or f32.
//
// B200 structure: persistent CTAs, one per SM, over 128 x 256 output tiles
// (all n-tiles of an m-tile adjacent, so the activation tile stays in L2; a
// short last wave's tiles split into 128-column halves, see gm_item).
// Warps 0..E-1 are the epilogue (E = 8, or 12 for a bf16 output with the
// activation; warp w reads TMEM lanes 32 (w % 4) .. and every (E / 4)-th
// 32-column chunk from 32 (w / 4)), warp E is the TMA producer (4-stage ring
// of 128 x 64 A and 256 x 64 B tiles, 128-byte swizzle), warp E + 1 issues
// tcgen05.mma (M = 128, N = 256, K = 16 steps) into one of two TMEM
// accumulators, so the epilogue of a tile overlaps the main loop of the
// next.  Every wait is
// bounded; on a time-out the CTA drains its copies and MMAs, frees TMEM and
// leaves an error bit.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr int kGmBM = 128, kGmBN = 256, kGmBK = 64;
constexpr int kGmStages = 4;
constexpr int kGmABytes = kGmBM * kGmBK * 2;   // 16 KB
constexpr int kGmBBytes = kGmBN * kGmBK * 2;   // 32 KB
constexpr int kGmStageBytes = kGmABytes + kGmBBytes;
// Epilogue warps: 8 (two per scheduler), or 12 for a bf16 output with the
// activation, whose dependent f32 chains need a third warp per scheduler to
// keep the tensor core busy.  Warp w reads TMEM lanes 32 (w % 4) .. and the
// 32-column chunks j, j + E / 4, j + 2 E / 4, ... of the tile (j = w / 4).
constexpr int kGmMaxEpiWarps = 12;
// Per epilogue warp, the staging of its 32 x 32 output blocks for the TMA
// store: with 8 epilogue warps one f32 block or two bf16 blocks
// (double-buffered), with 12 one bf16 block (shared memory is full).
template <int E>
struct GmCfg {
  static constexpr int kStageOut = E == 8 ? 4096 : 2048;
  static constexpr int kProducer = E, kMma = E + 1;
  static constexpr int kThreads = (E + 2) * 32;
};
constexpr int kGmTmemCols = 2 * kGmBN;  // two accumulators

// Work item i: tile (tm, tn), and which columns -- half 0: all 256, half 1 /
// 2: the first / second 128.
struct GmItem {
  int tm, tn, half;
};
__device__ __forceinline__ GmItem gm_item(const GemmParams& p, int i) {
  int t = i, h = 0;
  if (i >= p.split_from) {
    const int j = i - p.split_from;
    t = p.split_from + (j >> 1);
    h = 1 + (j & 1);
  }
  GmItem w;
  w.tm = t / p.n_tiles;
  w.tn = t - w.tm * p.n_tiles;
  w.half = h;
  return w;
}

struct GmBars {
  uint64_t full[kGmStages], empty[kGmStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t done;
  uint64_t res[kGmMaxEpiWarps];  // per epilogue warp: its residual block has landed
  uint32_t tmem_base;
  int abort_flag;
};
template <int E>
constexpr size_t gm_smem() {
  return 1024 + kGmStages * kGmStageBytes + E * GmCfg<E>::kStageOut + sizeof(GmBars) + 64;
}
static_assert(gm_smem<8>() <= 227 * 1024 && gm_smem<12>() <= 227 * 1024, "shared memory");

// One element of the division num / den in fast_gelu2, rounded to nearest
// even without a division instruction.  q1n is the negated quotient, within
// one ulp of it, r1 = num + q1n den its exact remainder; cn is q1n moved one
// ulp towards the true quotient (the sign of r1 says which side it lies on),
// rc its exact remainder, and the closer of the two (smaller |remainder|)
// is the rounded quotient.  A quotient of two f32 is never exactly halfway
// between two f32 (the midpoint has 25 significant bits, num only 24), so
// there is no tie.  A NaN (num infinite or NaN) falls back to num * (-1/den).
__device__ __forceinline__ float div_pick(float q1n, float r1, float rc_of_cn, float cn, float q0n) {
  float x = fabsf(rc_of_cn) < fabsf(r1) ? cn : q1n;
  return x != x ? q0n : x;
}
__device__ __forceinline__ float div_neighbour(float q1n, float r1) {
  const uint32_t grow = (__float_as_uint(r1) ^ __float_as_uint(q1n)) >> 31;
  return __uint_as_float(__float_as_uint(q1n) + 2u * grow - 1u);
}

// Whisper's GELU as the reference computes it (gelu_scalar,
// text_decoder.rs:341-350), two elements at a time with f32x2 arithmetic:
//   u = 0.7978846 * mul_add(0.044715 t t, t, t),  u2 = min(u u, 64)
//   num = u (135135 + u2 (17325 + u2 (378 + u2)))
//   den = 135135 + u2 (62370 + u2 (3150 + u2 28))
//   out = 0.5 t (1 + clamp(num / den, -1, 1))
// Every operation is the same separately rounded f32 operation as the
// reference's, in the same order.  The division is the correctly rounded
// quotient, reached without a division instruction (den >= 135135 is
// normal): a MUFU reciprocal y of -den, the negated quotient q0n = num y,
// one residual correction q1n = q0n + (num + q0n den) y, which lands within
// one ulp of the quotient (y's error of about 2^-23 enters squared), then
// div_pick.  The remainders num + q den are exact f32 values whenever q is
// within one ulp of the quotient, so the fused multiply-adds compute them
// without error.  Quotients below 2^-25 in magnitude (where the remainders
// may underflow) leave 1 + clamp(..) = 1 whatever their last bits.
__device__ __forceinline__ void fast_gelu2(float& t0, float& t1, uint64_t k1, uint64_t kz) {
  const uint64_t t = f2_pack(t0, t1);
  const uint64_t c = f2_fma(f2_mul_rn(f2_mul_rn(f2_pack(0.044715f, 0.044715f), t, kz), t, kz), t, t);
  const uint64_t u = f2_mul_rn(f2_pack(0.7978846f, 0.7978846f), c, kz);
  float a0, a1;
  f2_unpack(f2_mul_rn(u, u, kz), a0, a1);
  const uint64_t u2 = f2_pack(fminf(a0, 64.0f), fminf(a1, 64.0f));
  uint64_t n = f2_add_rn(f2_pack(378.0f, 378.0f), u2, k1);
  n = f2_add_rn(f2_pack(17325.0f, 17325.0f), f2_mul_rn(u2, n, kz), k1);
  n = f2_add_rn(f2_pack(135135.0f, 135135.0f), f2_mul_rn(u2, n, kz), k1);
  n = f2_mul_rn(u, n, kz);
  uint64_t d = f2_mul_rn(u2, f2_pack(28.0f, 28.0f), kz);
  d = f2_add_rn(f2_pack(3150.0f, 3150.0f), d, k1);
  d = f2_add_rn(f2_pack(62370.0f, 62370.0f), f2_mul_rn(u2, d, kz), k1);
  d = f2_add_rn(f2_pack(135135.0f, 135135.0f), f2_mul_rn(u2, d, kz), k1);
  float d0, d1;
  f2_unpack(d, d0, d1);
  const uint64_t ny = f2_pack(rcp_approx(-d0), rcp_approx(-d1));
  const uint64_t q0n = f2_mul_rn(n, ny, kz);
  const uint64_t q1n = f2_fma(f2_fma(q0n, d, n), ny, q0n);
  const uint64_t r1 = f2_fma(q1n, d, n);
  float qa, qb, ra, rb, pa, pb;
  f2_unpack(q1n, qa, qb);
  f2_unpack(r1, ra, rb);
  f2_unpack(q0n, pa, pb);
  const float ca = div_neighbour(qa, ra), cb = div_neighbour(qb, rb);
  float sa, sb;
  f2_unpack(f2_fma(f2_pack(ca, cb), d, n), sa, sb);
  const float xa = -div_pick(qa, ra, sa, ca, pa), xb = -div_pick(qb, rb, sb, cb, pb);
  const uint64_t r = f2_pack(fminf(fmaxf(xa, -1.0f), 1.0f), fminf(fmaxf(xb, -1.0f), 1.0f));
  f2_unpack(f2_mul_rn(f2_mul_rn(f2_pack(0.5f, 0.5f), t, kz), f2_add_rn(f2_pack(1.0f, 1.0f), r, k1), kz), t0, t1);
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

template <int E>
__global__ void __launch_bounds__(GmCfg<E>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                   GemmParams p) {
  extern __shared__ uint8_t dsm_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_out = dsm + kGmStages * kGmStageBytes;
  constexpr int kStageOut = GmCfg<E>::kStageOut;
  constexpr int kGmProducer = GmCfg<E>::kProducer, kGmMma = GmCfg<E>::kMma;
  GmBars* bars = reinterpret_cast<GmBars*>(stage_out + E * kStageOut);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int items = p.items;
  const int kblocks = (p.K + kGmBK - 1) / kGmBK;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGmStages; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], E);
    }
    mbar_init(&bars->done, 1);
    for (int i = 0; i < E; ++i) mbar_init(&bars->res[i], 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kGmMma) {
    tmem_alloc(&bars->tmem_base, kGmTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  griddep_launch_dependents();

  if (warp == kGmProducer) {
    if (lane == 0) {
      griddep_wait();  // A may come from the preceding kernel
      prefetch_tensormap(&tmA);
      prefetch_tensormap(&tmB);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x) {
        const GmItem w = gm_item(p, t);
        const int tm = w.tm, tn = w.tn;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kGmStages;
          if (it >= kGmStages &&
              !mbar_wait(&bars->empty[s], ((it / kGmStages) - 1) & 1, abort_flag, p.err,
                         kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = dsm + s * kGmStageBytes;
          // B in two 128-row boxes; a half item loads only its own half
          // (to the same place as in a whole tile)
          mbar_arrive_expect_tx(&bars->full[s], w.half ? kGmABytes + kGmBBytes / 2 : kGmStageBytes);
          tma_load_2d(sa, &tmA, &bars->full[s], kb * kGmBK, tm * kGmBM);
          if (w.half != 2)
            tma_load_2d(sa + kGmABytes, &tmB, &bars->full[s], kb * kGmBK, tn * kGmBN);
          if (w.half != 1)
            tma_load_2d(sa + kGmABytes + kGmBBytes / 2, &tmB, &bars->full[s], kb * kGmBK,
                        tn * kGmBN + kGmBN / 2);
        }
      }
      if (!ok || *abort_flag) {
        // let the copies in flight land before the CTA exits
        int none = 0;
        for (uint32_t i = 0; i < kGmStages && i < it; ++i) {
          const uint32_t arms = (it - 1 - i) / kGmStages + 1;
          mbar_wait(&bars->full[i], (arms - 1) & 1, &none, p.err, kErrTimeoutDrain);
        }
      }
    }
  } else if (warp == kGmMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(1u, kGmBM, kGmBN, 0, 0);
      constexpr uint32_t idesc_half = idesc_f16(1u, kGmBM, kGmBN / 2, 0, 0);
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++ti) {
        const uint32_t acc = ti & 1;
        // a half item: N = 128 from B's rows 0-127 or 128-255 (16 KB on, a
        // whole number of 1 KB swizzle atoms)
        const int half = gm_item(p, t).half;
        const uint32_t id = half ? idesc_half : idesc;
        const uint32_t b_off = half == 2 ? kGmBBytes / 2 : 0;
        if (ti >= 2 && !mbar_wait(&bars->acc_empty[acc], ((ti >> 1) - 1) & 1, abort_flag, p.err,
                                  kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % kGmStages;
          if (!mbar_wait(&bars->full[s], (it / kGmStages) & 1, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(dsm + s * kGmStageBytes), 16, 1024);
          const uint64_t db =
              smem_desc_sw128(smem_u32(dsm + s * kGmStageBytes + kGmABytes + b_off), 16, 1024);
#pragma unroll
          for (int k = 0; k < kGmBK / 16; ++k)  // +32 bytes per K step inside the swizzle atom
            mma_ss(tmem + acc * kGmBN, da + 2 * k, db + 2 * k, id, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&bars->empty[s]);
        }
        if (!ok) break;
        mma_commit(&bars->acc_full[acc]);
      }
      // every MMA issued has finished before TMEM is freed
      mma_commit(&bars->done);
      int none = 0;
      mbar_wait(&bars->done, 0, &none, p.err, kErrTimeoutDrain);
    }
  } else {
    // Epilogue: warp w, TMEM lanes 32 (w % 4) + i = tile row, the 32-column
    // chunks w / 4 + (E / 4) k of the tile.  Each 32 x 32 block goes through
    // a swizzled shared-memory staging buffer to one TMA store (rows past M
    // are clipped by the store).  The residual and the output may belong to
    // the preceding kernel.
    griddep_wait();
    const int lg = warp & 3, ch = warp >> 2;
    uint8_t* stg = stage_out + warp * kStageOut;
    // two bf16 blocks in flight per warp where the staging holds them
    const bool dbuf = kStageOut == 4096 && !p.out_f32;
    uint32_t stores = 0, res_loads = 0, res_issued = 0;
    const bool has_res = p.residual != nullptr;
    const uint32_t blk_bytes = p.out_f32 ? 4096u : 2048u;
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < items; t += gridDim.x, ++ti) {
      const uint32_t acc = ti & 1;
      if (!mbar_wait(&bars->acc_full[acc], (ti >> 1) & 1, abort_flag, p.err, kErrTimeoutConsumer))
        break;
      tc_fence_after();
      const GmItem w = gm_item(p, t);
      const int row0 = w.tm * kGmBM + 32 * lg;
      const int width = w.half ? kGmBN / 2 : kGmBN;  // accumulator columns of the item
      const int col0 = w.tn * kGmBN + (w.half == 2 ? kGmBN / 2 : 0);
      for (int c0 = 32 * ch; c0 < width; c0 += 32 * (E / 4)) {
        const int n0 = col0 + c0;
        // this block's staging buffer; its previous TMA store must have read it
        uint8_t* buf = dbuf ? stg + (stores & 1) * 2048 : stg;
        if (n0 < p.N) {
          if (lane == 0) {
            if (dbuf)
              bulk_wait_read_1();
            else
              bulk_wait_read_all();
            if (has_res) {  // the residual block lands in the buffer the output leaves from
              mbar_arrive_expect_tx(&bars->res[warp], blk_bytes);
              tma_load_2d(buf, &tmR, &bars->res[warp], n0, row0);
            }
          }
          if (has_res) ++res_issued;
          __syncwarp();
        }
        uint32_t r[32];
        tmem_ld32(tmem + acc * kGmBN + (static_cast<uint32_t>(32 * lg) << 16) + c0, r);
        tmem_wait_ld();
        if (n0 >= p.N) continue;  // warp-uniform; N % 32 == 0
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (p.bias != nullptr) {
          // the same 32 values for every lane: 8 broadcast 16-byte loads
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(b4 + i);
            v[4 * i] = __fadd_rn(v[4 * i], bb.x);
            v[4 * i + 1] = __fadd_rn(v[4 * i + 1], bb.y);
            v[4 * i + 2] = __fadd_rn(v[4 * i + 2], bb.z);
            v[4 * i + 3] = __fadd_rn(v[4 * i + 3], bb.w);
          }
        }
        if (p.act == 1) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) fast_gelu2(v[i], v[i + 1], p.f2_one, p.f2_neg_zero);
        }
        if (has_res) {
          if (!mbar_wait(&bars->res[warp], res_loads & 1, abort_flag, p.err, kErrTimeoutConsumer))
            break;
          ++res_loads;
        }
        if (p.out_f32) {
          // 128-byte rows, 128-byte swizzle: 16-byte unit k of row r at k ^ (r % 8)
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float4* q = reinterpret_cast<float4*>(buf + lane * 128 + ((k ^ (lane & 7)) << 4));
            float4 w = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            if (has_res) {
              const float4 rr = *q;
              w.x = __fadd_rn(w.x, rr.x);
              w.y = __fadd_rn(w.y, rr.y);
              w.z = __fadd_rn(w.z, rr.z);
              w.w = __fadd_rn(w.w, rr.w);
            }
            *q = w;
          }
        } else {
          // 64-byte rows, 64-byte swizzle: unit k of row r at k ^ ((r / 2) % 4)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4* q = reinterpret_cast<uint4*>(buf + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4));
            float w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w[e] = v[8 * k + e];
            if (has_res) {
              const uint4 rr = *q;
              const uint32_t qq[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                w[2 * e] = __fadd_rn(w[2 * e], lo_half(qq[e], 0));
                w[2 * e + 1] = __fadd_rn(w[2 * e + 1], hi_half(qq[e], 0));
              }
            }
            uint4 pk;
            pk.x = pack_bf16x2(w[0], w[1]);
            pk.y = pack_bf16x2(w[2], w[3]);
            pk.z = pack_bf16x2(w[4], w[5]);
            pk.w = pack_bf16x2(w[6], w[7]);
            *q = pk;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmO, buf, n0, row0);
          bulk_commit();
        }
        ++stores;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[acc]);
    }
    if (res_loads < res_issued) {  // an abort: the residual block in flight lands first
      int none = 0;
      mbar_wait(&bars->res[warp], res_loads & 1, &none, p.err, kErrTimeoutDrain);
    }
    if (lane == 0) bulk_wait_all();  // the output is written before the CTA ends
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kGmMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kGmTmemCols);
  }
}

}  // namespace

size_t gemm_smem_bytes() { return gm_smem<8>() > gm_smem<12>() ? gm_smem<8>() : gm_smem<12>(); }

namespace {

template <int E>
cudaError_t launch_gemm_e(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                          const CUtensorMap& tmR, const GemmParams& p, int sms, cudaStream_t s) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[64];
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(gemm_tc_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(gm_smem<E>()));
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const int items = p.items;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(items < sms ? items : sms));
  cfg.blockDim = dim3(GmCfg<E>::kThreads);
  cfg.dynamicSmemBytes = gm_smem<E>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<E>, tmA, tmB, tmO, tmR, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                        const CUtensorMap& tmR, const GemmParams& p, int sms, cudaStream_t s) {
  if (p.act == 1 && !p.out_f32) return launch_gemm_e<12>(tmA, tmB, tmO, tmR, p, sms, s);
  return launch_gemm_e<8>(tmA, tmB, tmO, tmR, p, sms, s);
}

}  // namespace ffai
