// Block-scaled int8 GEMV for the decoder's single-row projections.
//
// Replaces the reference's AVX2 Int8Vocab (crates/ffai-mercury/src/asr/
// vocab_int8.rs): the vocabulary projection (51865 x d per generated token)
// and the decoder MLP layers that reuse it (text_decoder.rs:94-104, :210-226).
// Same quantisation and the same arithmetic, so results match the reference
// bit for bit:
//   weights: per row, per block of `blk` (a multiple of 32) weights, scale =
//     amax / 127 (1 when the block is zero), q = round(w / scale) in
//     [-127, 127], corr[row] = 64 * sum_b scale_b * blocksum_b (f32, block
//     order) -- Int8Vocab::new, vocab_int8.rs:97-166;
//   activations: per row, sx = amax / 63 (1 when zero), xu = round(x / sx)
//     in [-64, 63] + 64, a 7-bit unsigned value -- cpu_fwd, :218-258;
//   out = (sum_b f32(blocksum_b(xu * q)) * scale_b  -  corr) * sx, the sum
//     taken in block order in f32 with separate multiply and add --
//     dot_i8_blocked, :280-305.
//
// B200 layout: the projection streams the whole weight matrix once per token
// (75 MB for 51865 x 1280), so it is HBM-bound, and shared memory is the
// next limit: every byte is written by the bulk copy and read once more.
// The integer block sums are exact on the tensor cores (mma.sync m16n8k32,
// s8 weights x u8 activations -> s32; the activation rows of a step -- beams,
// up to 8 -- are the 8 columns), leaving the SIMT pipes the reference's f32
// epilogue: per block, convert, multiply by the row's scale, add in block
// order.  One warp owns a 16-row group (an m16 tile) for all its blocks, so
// the ordered sum stays in its registers and nothing else touches shared
// memory.
//
// Streaming: persistent CTAs, one per SM, each take a contiguous range of
// groups in rounds of one group per consumer warp.  A group is cut into units
// of S block records (weights and their scales are contiguous in the packed
// layout, so a unit is ONE bulk copy); a round's units go through a ring of
// shared-memory slots unit-major (unit k of every group of the round, then
// unit k + 1), each slot refilled by its own producer lane: bulk copies
// issued by one thread complete one after another, so a ring only turns
// into bytes in flight when every slot has its own issuing thread.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

#ifndef FFAI_GV_WARPS
#define FFAI_GV_WARPS 24
#endif
constexpr int kGvConsWarps = FFAI_GV_WARPS;  // consumer warps: groups of a round
constexpr int kGvThreads = (kGvConsWarps + 1) * 32;  // + the producer warp
constexpr int kGvCons = kGvConsWarps * 32;
#ifndef FFAI_GV_SLOT_TARGET
#define FFAI_GV_SLOT_TARGET 6144
#endif
#ifndef FFAI_GV_RING_MAX
#define FFAI_GV_RING_MAX 32
#endif
constexpr int kGvSlotTarget = FFAI_GV_SLOT_TARGET;  // bytes per slot to aim for
constexpr int kGvMaxRing = FFAI_GV_RING_MAX;        // slots, one producer lane each
// Dynamic shared memory the kernel may use (227 KB per block, less a little
// for its static arrays).
constexpr int kGvSmemMax = 227 * 1024 - 1024;
constexpr int kGvBarX = 1;  // named barrier of the activation quantisation
#ifndef FFAI_GV_BATCH
#define FFAI_GV_BATCH 3
#endif
constexpr int kGvBatch = FFAI_GV_BATCH;  // blocks whose mmas are in flight together

// One warp per row: block scales, int8 weights and the row's correction term
// in the reference's order of operations, written as block records.  Warps
// past `rows` (up to the group boundary) write the zero padding.
template <typename T>
__global__ void __launch_bounds__(256) int8_quantize_kernel(const T* w, int rows, int cols, int blk,
                                                            uint8_t* packed, float* corr) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int padded = static_cast<int>(int8_gemv_groups(rows)) * kGvRows;
  if (row >= padded) return;
  const int g = row / kGvRows, l = row % kGvRows, nb = cols / blk, rec = int8_gemv_record(blk);
  auto record = [&](int b) { return packed + (static_cast<size_t>(g) * nb + b) * rec; };
  // column k (within block b) of this row
  auto qbyte = [&](int b, int k) { return record(b) + ((k / 16) * kGvRows + l) * 16 + k % 16; };
  auto scale = [&](int b) {
    return reinterpret_cast<float*>(record(b) + blk * kGvRows) + (l % 8) * 2 + l / 8;
  };
  if (row >= rows) {
    for (int b = 0; b < nb; ++b) {
      for (int k = lane; k < blk; k += 32) *qbyte(b, k) = 0;
      if (lane == 0) *scale(b) = 0.f;
    }
    if (lane == 0) corr[row] = 0.f;
    return;
  }
  const T* src = w + static_cast<size_t>(row) * cols;
  float c = 0.f;
  for (int b = 0; b < nb; ++b) {
    float amax = 0.f;
    for (int k = lane; k < blk; k += 32) amax = fmaxf(amax, fabsf(to_f32(src[b * blk + k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    int bsum = 0;
    for (int k = lane; k < blk; k += 32) {
      const float r = roundf(__fdiv_rn(to_f32(src[b * blk + k]), sc));  // half away from zero
      // NaN -> 0, as Rust's saturating `as` cast after clamp
      const int qi = r == r ? static_cast<int>(fminf(fmaxf(r, -127.0f), 127.0f)) : 0;
      *qbyte(b, k) = static_cast<uint8_t>(static_cast<int8_t>(qi));
      bsum += qi;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
    c = __fadd_rn(c, __fmul_rn(sc, static_cast<float>(bsum)));
    if (lane == 0) *scale(b) = sc;
  }
  if (lane == 0) corr[row] = __fmul_rn(64.0f, c);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
// d += a (16 x 32, s8, row-major) * b (32 x 8, u8, column-major), exact s32.
__device__ __forceinline__ void mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// f32 of an integer block sum, exact: through the float 1.5 * 2^23 + s when
// |s| < 2^22 (blocks of up to 256 columns: |s| <= 256 * 127 * 127), else by
// conversion.
template <bool SMALL>
__device__ __forceinline__ float sum_to_f32(int s) {
  if (SMALL) return __fsub_rn(__int_as_float(0x4B400000 + s), 12582912.0f);
  return __int2float_rn(s);
}

// round(x / sx) as the reference computes it -- the IEEE quotient, rounded
// half away from zero -- clamped to [-64, 63].  With fast_ok the approximate
// quotient q is within 2 ulp of x / sx, so within 3 ulp of the IEEE
// quotient; |q| <= 64 (|x| <= 63 sx), where 3 ulp < 3e-5.  A q more than
// 6.4e-5 from every rounding boundary k + 1/2 therefore rounds like the IEEE
// quotient; closer (or not finite), the IEEE division decides.  A NaN
// quotient gives 0, as Rust's saturating `as` cast does.
__device__ __forceinline__ int quant_act(float x, float sx, bool fast_ok) {
  float q = __fdividef(x, sx);
  const float a = fabsf(q);
  const float dist = fabsf((a - floorf(a)) - 0.5f);
  if (!(fast_ok && dist > 6.4e-5f)) q = __fdiv_rn(x, sx);
  if (q != q) return 0;
  return static_cast<int>(fminf(fmaxf(roundf(q), -64.0f), 63.0f));
}

// Activations, once per GEMV: CTA b quantises row b of x -- amax over the
// row, sx = amax / 63 (1 when zero), xu = round(x / sx) + 64 -- into the
// layout the GEMV's ldmatrix reads: xq[(c * 8 + b) * 16 + j] = xu of column
// 16 c + j; CTA 0 also zeroes the rows past the batch.
constexpr int kActThreads = 256;
__global__ void __launch_bounds__(kActThreads) int8_act_kernel(const float* x, int B, int cols,
                                                               uint8_t* xq, float* sx_out) {
  __shared__ float s_red[kActThreads / 32];
  __shared__ float s_sx;
  griddep_launch_dependents();
  griddep_wait();  // x comes from the preceding kernel
  const int b = blockIdx.x, tid = threadIdx.x, c4 = cols / 4;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * cols);
  constexpr int kRegs = kGvMaxCols / 4 / kActThreads;
  float4 v[kRegs];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kRegs; ++j) {
    const int i = tid + j * kActThreads;
    if (i < c4) {
      v[j] = __ldg(xr + i);
      m = fmaxf(fmaxf(fmaxf(m, fabsf(v[j].x)), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (tid % 32 == 0) s_red[tid / 32] = m;
  __syncthreads();
  if (tid == 0) {
    float a = 0.f;
    for (int w = 0; w < kActThreads / 32; ++w) a = fmaxf(a, s_red[w]);
    s_sx = a > 0.f ? __fdiv_rn(a, 63.0f) : 1.0f;
    sx_out[b] = s_sx;
  }
  __syncthreads();
  const float sx = s_sx;
  // sx well inside the normal range: the approximate quotient is good to 2 ulp
  const bool fast_ok = sx >= 0x1p-120f && sx <= 0x1p120f;
  uint32_t* xw = reinterpret_cast<uint32_t*>(xq);
#pragma unroll
  for (int j = 0; j < kRegs; ++j) {
    const int i = tid + j * kActThreads;
    if (i < c4) {
      const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      uint32_t word = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t)
        word |= static_cast<uint32_t>(quant_act(e[t], sx, fast_ok) + 64) << (8 * t);
      const int col = 4 * i;
      xw[((col >> 4) * 8 + b) * 4 + ((col >> 2) & 3)] = word;
    }
  }
  if (b == 0) {
    const int nc = cols / 16;
    for (int w = tid; w < nc * 32; w += kActThreads)
      if (((w >> 2) & 7) >= B) xw[w] = 0u;
  }
}

template <bool SMALL>
__global__ void __launch_bounds__(kGvThreads, 1) int8_gemv_kernel(Int8GemvParams p) {
  const Int8GemvPlan& P = p.plan;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* xq = dsm + P.x_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + P.bar_off);
  uint64_t* empty = full + kGvMaxRing;
  __shared__ float s_sx[kGvMaxBatch];
  // s_use[r]: the use of slot r the producer has armed last.  Warps consume
  // different units and may run ahead of one another, so a warp can come to
  // wait for use m of a slot while use m - 1 is still in flight; a parity
  // wait cannot tell those apart, the counter can.
  __shared__ int s_use[kGvMaxRing];
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int cols = p.cols, blk = p.blk, B = p.batch;
  const int nb = cols / blk, gc = blk / 16, nc = cols / 16, rec = int8_gemv_record(blk);
  const int S = P.S, ring = P.ring;
  const int upg = (nb + S - 1) / S;  // units (slot loads) per group
  const int g_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * P.groups / P.grid);
  const int g_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * P.groups / P.grid);

  if (tid == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // the warp that owns the unit's group
      s_use[i] = -1;
    }
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  // Producer: units in stream order j (round by round: unit k of each of
  // the round's groups, k = 0 .. upg - 1); lane r refills slot r with units
  // r, r + ring, ...  Stable weights stream while the preceding kernel
  // finishes; the activations come from it, so the consumers always wait.
  if (warp == kGvConsWarps) {
    if (!p.weights_stable) griddep_wait();
    if (lane >= ring) return;
    uint64_t* fb = &full[lane];
    const int units = (g_end - g_begin) * upg;
    const int full_round = kGvConsWarps * upg;  // units of a full round
    int issued = 0;
    bool ok = true;
    for (int j = lane; j < units; j += ring, ++issued) {
      if (issued > 0 &&
          !mbar_wait(&empty[lane], (issued - 1) & 1, &s_abort, p.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      const int ro = j / full_round, g0 = g_begin + ro * kGvConsWarps;
      const int n = min(kGvConsWarps, g_end - g0), rem = j - ro * full_round;
      const int k = rem / n, i = rem - k * n;
      const uint32_t bytes = static_cast<uint32_t>(min(S, nb - k * S)) * rec;
      // The uses before this one have landed and been consumed (empty above).
      // A plain store: shared memory has one copy, and a fence here would
      // wait for this warp's earlier bulk copies.
      *reinterpret_cast<volatile int*>(&s_use[lane]) = issued;
      mbar_arrive_expect_tx(fb, bytes);
      bulk_load(dsm + static_cast<size_t>(lane) * P.slot_bytes,
                p.packed + (static_cast<size_t>(g0 + i) * nb + static_cast<size_t>(k) * S) * rec,
                bytes, fb);
    }
    if (issued > 0 && (!ok || s_abort)) {
      // Let this slot's last copy land before the CTA exits.
      int none = 0;
      mbar_wait(fb, (issued - 1) & 1, &none, p.err, kErrTimeoutDrain);
    }
    return;
  }

  // Activations, quantised by int8_act_kernel just before (the preceding
  // kernel): xq [chunk of 16 columns][8 rows][16 bytes] -- the mma's B
  // operand, 8 x 16 bytes per ldmatrix -- and sx per row.
  griddep_wait();
  {
    const uint4* src = reinterpret_cast<const uint4*>(p.xq);
    uint4* dst = reinterpret_cast<uint4*>(xq);
    for (int i = tid; i < nc * 8; i += kGvCons) dst[i] = src[i];
    if (tid < B) s_sx[tid] = p.sx[tid];
  }
  named_bar_sync(kGvBarX, kGvCons);

  // Consumers: warp w takes group w of each round, all its blocks in order;
  // thread (gq, tig) accumulates rows gq, gq + 8 x beams 2 tig, 2 tig + 1.
  const int gq = lane >> 2, tig = lane & 3;
  // ldmatrix row addresses: A -- lanes 8m .. 8m + 7 give the rows of matrix m
  // (m = 0, 1: chunk 2s, rows 0-7 / 8-15; m = 2, 3: chunk 2s + 1);
  // B -- lanes 0-7 / 8-15 give the 8 activation rows of chunk 2s / 2s + 1.
  const uint32_t a_lane = ((lane >> 4) * kGvRows + (lane & 7) + ((lane >> 3) & 1) * 8) * 16;
  const uint32_t b_lane = ((((lane >> 3) & 1) * 8) + (lane & 7)) * 16;
  const uint32_t xq_s = smem_u32(xq), dsm_s = smem_u32(dsm);
  int j0 = 0;  // stream index of the round's first unit
  for (int g0 = g_begin; g0 < g_end; g0 += kGvConsWarps) {
    const int n = min(kGvConsWarps, g_end - g0);
    if (warp >= n) {
      j0 += n * upg;
      continue;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int k = 0; k < upg; ++k) {
      const int j = j0 + k * n + warp, r = j % ring, use = j / ring;
      if (!wait_slot_use(&s_use[r], use, &s_abort, p.err) ||
          !mbar_wait(&full[r], use & 1, &s_abort, p.err, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      const int sk = min(S, nb - k * S);
      const uint32_t slot_s = dsm_s + r * P.slot_bytes;
      // kGvBatch blocks at a time: their loads and mmas all in flight before
      // the products are added in block order
      for (int kb0 = 0; kb0 < sk; kb0 += kGvBatch) {
        int d[kGvBatch][4];
        uint32_t rec_s[kGvBatch], x_s[kGvBatch];
#pragma unroll
        for (int i = 0; i < kGvBatch; ++i) {
          const int kb = min(kb0 + i, sk - 1);  // past the end: a valid block, result unused
          rec_s[i] = slot_s + kb * rec;
          x_s[i] = xq_s + static_cast<uint32_t>((k * S + kb) * gc) * 128;
#pragma unroll
          for (int t = 0; t < 4; ++t) d[i][t] = 0;
        }
        for (int sl = 0; sl < gc / 2; ++sl) {
          uint32_t a[kGvBatch][4], bx[kGvBatch][2];
#pragma unroll
          for (int i = 0; i < kGvBatch; ++i) {
            ldsm_x4(rec_s[i] + sl * 512 + a_lane, a[i][0], a[i][1], a[i][2], a[i][3]);
            ldsm_x2(x_s[i] + sl * 256 + b_lane, bx[i][0], bx[i][1]);
          }
#pragma unroll
          for (int i = 0; i < kGvBatch; ++i)
            mma_s8u8(d[i], a[i][0], a[i][1], a[i][2], a[i][3], bx[i][0], bx[i][1]);
        }
        float2 sc[kGvBatch];
#pragma unroll
        for (int i = 0; i < kGvBatch; ++i)
          sc[i] = *reinterpret_cast<const float2*>(dsm + (rec_s[i] - dsm_s) + blk * kGvRows + gq * 8);
#pragma unroll
        for (int i = 0; i < kGvBatch; ++i) {
          if (kb0 + i < sk) {
            acc[0] = __fadd_rn(acc[0], __fmul_rn(sum_to_f32<SMALL>(d[i][0]), sc[i].x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(sum_to_f32<SMALL>(d[i][1]), sc[i].x));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(sum_to_f32<SMALL>(d[i][2]), sc[i].y));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(sum_to_f32<SMALL>(d[i][3]), sc[i].y));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[r]);
    }
    j0 += n * upg;
    if (!ok) break;
    const int r0 = (g0 + warp) * kGvRows + gq, r1 = r0 + 8;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int b = 2 * tig + e;
      if (b >= B) continue;
      const float sx = s_sx[b];
      if (r0 < p.rows)
        p.out[static_cast<size_t>(b) * p.rows + r0] =
            __fmul_rn(__fsub_rn(acc[e], __ldg(p.corr + r0)), sx);
      if (r1 < p.rows)
        p.out[static_cast<size_t>(b) * p.rows + r1] =
            __fmul_rn(__fsub_rn(acc[2 + e], __ldg(p.corr + r1)), sx);
    }
  }
}

}  // namespace

bool int8_gemv_plan(int rows, int cols, int blk, int batch, int sms, Int8GemvPlan* plan) {
  if (!int8_gemv_served(cols, blk) || rows <= 0 || batch < 1 || batch > kGvMaxBatch || sms <= 0)
    return false;
  Int8GemvPlan P{};
  const long long groups = int8_gemv_groups(rows);
  P.groups = static_cast<int>(groups);
  P.grid = static_cast<int>(std::min<long long>(sms, groups));
  const int rec = int8_gemv_record(blk), nb = cols / blk;
  const int upg = std::max(1, (nb * rec + kGvSlotTarget - 1) / kGvSlotTarget);
  P.S = (nb + upg - 1) / upg;
  P.slot_bytes = P.S * rec;
  const int x_bytes = (cols / 16) * 128;
  const int bar_bytes = 2 * kGvMaxRing * 8;
  const int avail = kGvSmemMax - x_bytes - bar_bytes;
  P.ring = std::min(kGvMaxRing, avail / P.slot_bytes);
  if (P.ring < 2) return false;
  P.x_off = P.ring * P.slot_bytes;
  P.bar_off = P.x_off + x_bytes;
  P.smem = P.bar_off + bar_bytes;
  *plan = P;
  return true;
}

cudaError_t launch_int8_quantize(const void* w, int w_dtype, int rows, int cols, int blk,
                                 uint8_t* packed, float* corr, cudaStream_t s) {
  const long long padded = int8_gemv_groups(rows) * 32;
  const int blocks = static_cast<int>((padded + 7) / 8);  // 8 warps of 32
  switch (w_dtype) {
    case 0:
      int8_quantize_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), rows, cols,
                                                         blk, packed, corr);
      break;
    case 1:
      int8_quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(w), rows, cols, blk, packed, corr);
      break;
    case 2:
      int8_quantize_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w), rows,
                                                          cols, blk, packed, corr);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_int8_gemv(const Int8GemvParams& p, cudaStream_t s) {
  const Int8GemvPlan& P = p.plan;
  if (p.batch < 1 || p.batch > kGvMaxBatch || !int8_gemv_served(p.cols, p.blk) ||
      P.smem > kGvSmemMax || P.ring < 2 || P.ring > kGvMaxRing)
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // The attribute is per device; set it to the largest layout once.
  static std::atomic<bool> configured[64];
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    for (auto fn : {int8_gemv_kernel<true>, int8_gemv_kernel<false>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kGvSmemMax);
      if (e != cudaSuccess) return e;
    }
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t acfg{};
  acfg.gridDim = dim3(static_cast<unsigned>(p.batch));
  acfg.blockDim = dim3(kActThreads);
  acfg.stream = s;
  acfg.attrs = attr;
  acfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&acfg, int8_act_kernel, p.x, p.batch, p.cols, p.xq, p.sx);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(P.grid));
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(P.smem);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.blk <= 256)
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<true>, p);
  else
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<false>, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ffai
