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
//     dot_i8_blocked, :280-305.  The integer block sums are exact (dp4a).
//
// B200 layout: the projection streams the whole weight matrix once per token
// (75 MB for 51865 x 1280), so it is HBM-bound.  Because the f32 sum over a
// row's blocks must run in block order, one lane owns one weight row and walks
// its blocks in order; the weights are stored packed (kernels.h) so that the
// 32 lanes of a warp read their 32 rows' next 16 bytes as one conflict-free
// 512-byte shared-memory access.  Persistent CTAs, one per SM, each take a
// contiguous range of 32-row groups; a producer warp streams the groups'
// columns through a ring of shared-memory slots with 1-d bulk copies (weights
// and block scales of a step are contiguous in the packed layout), and all
// activation rows of the step (beams, up to 8) share that one pass.  Where a
// CTA has few groups (the MLP's 1280-row fc2), the 16 consumer warps split
// each group's blocks; their block products go through shared memory to the
// warp that adds them in order.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr int kGvWarps = 16;
constexpr int kGvThreads = (kGvWarps + 1) * 32;  // + the producer warp
constexpr int kGvCons = kGvWarps * 32;
constexpr int kGvMaxStages = 6;
constexpr int kGvStageBudget = 40960;  // target bytes per ring slot
// Dynamic shared memory the kernel may use (227 KB per block, less a little
// for its static arrays).
constexpr int kGvSmemMax = 227 * 1024 - 1024;
constexpr int kGvBarX = 1;  // named barrier of the activation quantisation

// One warp per row: block scales, int8 weights and the row's correction term
// in the reference's order of operations, written in the packed layout.
// Warps past `rows` (up to the group boundary) write the zero padding.
template <typename T>
__global__ void __launch_bounds__(256) int8_quantize_kernel(const T* w, int rows, int cols, int blk,
                                                            int8_t* qw, float* bscale,
                                                            float* corr) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int padded = static_cast<int>(int8_gemv_groups(rows)) * 32;
  if (row >= padded) return;
  const int g = row / 32, l = row % 32, nb = cols / blk, nc = cols / 16;
  // byte column k of this row in the packed layout
  auto qidx = [&](int k) {
    return ((static_cast<size_t>(g) * nc + k / 16) * 32 + l) * 16 + k % 16;
  };
  auto sidx = [&](int b) { return (static_cast<size_t>(g) * nb + b) * 32 + l; };
  if (row >= rows) {
    for (int k = lane; k < cols; k += 32) qw[qidx(k)] = 0;
    for (int b = lane; b < nb; b += 32) bscale[sidx(b)] = 0.f;
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
      float r = roundf(__fdiv_rn(to_f32(src[b * blk + k]), sc));  // half away from zero
      r = fminf(fmaxf(r, -127.0f), 127.0f);
      const int qi = static_cast<int>(r);
      qw[qidx(b * blk + k)] = static_cast<int8_t>(qi);
      bsum += qi;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
    c = __fadd_rn(c, __fmul_rn(sc, static_cast<float>(bsum)));
    if (lane == 0) bscale[sidx(b)] = sc;
  }
  if (lane == 0) corr[row] = __fmul_rn(64.0f, c);
}

// NB: activation rows handled (a power of two >= p.batch, <= 8).
template <int NB>
__global__ void __launch_bounds__(kGvThreads, 1) int8_gemv_kernel(Int8GemvParams p) {
  const Int8GemvPlan& P = p.plan;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* xq = dsm + P.x_off;
  float* prod = reinterpret_cast<float*>(dsm + P.p_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + P.bar_off);
  uint64_t* empty = full + kGvMaxStages;
  uint64_t* gbar = empty + kGvMaxStages;  // per group of a round: products ready
  __shared__ float s_sx[kGvMaxBatch];
  __shared__ float s_red[kGvMaxBatch][kGvWarps];
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int cols = p.cols, blk = p.blk, B = p.batch;
  const int nb = cols / blk, gc = blk / 16, nc = cols / 16;
  const int S = P.S, nmax = P.nmax, wpg = P.wpg, stages = P.stages;
  const int steps = (nb + S - 1) / S;
  const int g_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * P.groups / P.grid);
  const int g_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * P.groups / P.grid);
  const int w_slot = nmax * S * blk * 32;  // weight bytes of a slot; scales follow

  if (tid == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGvWarps);
    }
    for (int i = 0; i < nmax; ++i) mbar_init(&gbar[i], wpg);
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  // Producer: per round and step, the S-block column range of each group
  // (weights, then scales), one pair of bulk copies per group.  Stable
  // weights stream while the preceding kernel finishes; the activations come
  // from it, so the consumers always wait for it.
  if (warp == kGvWarps) {
    if (!p.weights_stable) griddep_wait();
    int seq = 0;
    bool ok = true;
    for (int g0 = g_begin; g0 < g_end && ok; g0 += nmax) {
      const int n = min(nmax, g_end - g0);
      for (int k = 0; k < steps; ++k, ++seq) {
        const int st = seq % stages;
        if (seq >= stages) {
          int got = 1;
          if (lane == 0)
            got = mbar_wait(&empty[st], ((seq / stages) - 1) & 1, &s_abort, p.err,
                            kErrTimeoutProducer);
          if (!__shfl_sync(0xffffffffu, got, 0)) {
            ok = false;
            break;
          }
        }
        const int sk = min(S, nb - k * S);
        if (lane == 0)
          mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(n) * sk * (blk * 32 + 128));
        __syncwarp();
        if (lane < n) {
          const size_t g = static_cast<size_t>(g0 + lane);
          uint8_t* slot = dsm + static_cast<size_t>(st) * P.slot_bytes;
          bulk_load(slot + static_cast<size_t>(lane) * S * blk * 32,
                    p.qw + (g * nc + static_cast<size_t>(k) * S * gc) * 512,
                    static_cast<uint32_t>(sk) * blk * 32, &full[st]);
          bulk_load(slot + w_slot + static_cast<size_t>(lane) * S * 128,
                    p.bscale + (g * nb + static_cast<size_t>(k) * S) * 32,
                    static_cast<uint32_t>(sk) * 128, &full[st]);
        }
      }
    }
    if (!ok && lane == 0) {
      // Let the copies in flight land before the CTA exits.
      int none = 0;
      for (int i = 0; i < stages && i < seq; ++i) {
        const int arms = (seq - 1 - i) / stages + 1;
        mbar_wait(&full[i], (arms - 1) & 1, &none, p.err, kErrTimeoutDrain);
      }
    }
    return;  // the producer takes no part in the barriers below
  }

  // Activations: per row b, sx = amax / 63 and xu = round(x / sx) + 64, once
  // per CTA into shared memory.
  griddep_wait();
  for (int b = 0; b < B; ++b) {
    const float* xr = p.x + static_cast<size_t>(b) * cols;
    float amax = 0.f;
    for (int k = tid; k < cols; k += kGvCons) amax = fmaxf(amax, fabsf(xr[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) s_red[b][warp] = amax;
  }
  named_bar_sync(kGvBarX, kGvCons);
  if (tid < B) {
    float m = 0.f;
    for (int w = 0; w < kGvWarps; ++w) m = fmaxf(m, s_red[tid][w]);
    s_sx[tid] = m > 0.f ? __fdiv_rn(m, 63.0f) : 1.0f;
  }
  named_bar_sync(kGvBarX, kGvCons);
  for (int i = tid; i < B * cols; i += kGvCons) {
    const int b = i / cols;
    float r = roundf(__fdiv_rn(p.x[i], s_sx[b]));
    r = fminf(fmaxf(r, -64.0f), 63.0f);
    xq[i] = static_cast<uint8_t>(static_cast<int>(r) + 64);
  }
  named_bar_sync(kGvBarX, kGvCons);

  // Consumers: warp w works on group gi = w / wpg of each round, on the
  // blocks j, j + wpg, ... (j = w % wpg) of each step; lane l is row 32g + l.
  const int gi = warp / wpg, j = warp % wpg;
  int seq = 0, buf = 0, gphase = 0;
  bool ok = true;
  for (int g0 = g_begin; g0 < g_end && ok; g0 += nmax) {
    const int n = min(nmax, g_end - g0);
    const bool active = gi < n;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    for (int k = 0; k < steps; ++k, ++seq) {
      const int st = seq % stages;
      if (!mbar_wait(&full[st], (seq / stages) & 1, &s_abort, p.err, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      const int sk = min(S, nb - k * S);
      if (active) {
        const uint8_t* ws = dsm + static_cast<size_t>(st) * P.slot_bytes +
                            static_cast<size_t>(gi) * S * blk * 32;
        const float* ss = reinterpret_cast<const float*>(dsm + static_cast<size_t>(st) * P.slot_bytes +
                                                         w_slot) + gi * S * 32;
        for (int kb = j; kb < sk; kb += wpg) {
          int is[NB];
#pragma unroll
          for (int b = 0; b < NB; ++b) is[b] = 0;
          const int c0 = (k * S + kb) * gc;  // first column chunk of the block
#pragma unroll 2
          for (int ch = 0; ch < gc; ++ch) {
            const uint4 wv = *reinterpret_cast<const uint4*>(ws + ((kb * gc + ch) * 32 + lane) * 16);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              if (b < B) {
                const uint4 xv = *reinterpret_cast<const uint4*>(xq + b * cols + (c0 + ch) * 16);
                int s = __dp4a(static_cast<int>(wv.x), static_cast<int>(xv.x), is[b]);
                s = __dp4a(static_cast<int>(wv.y), static_cast<int>(xv.y), s);
                s = __dp4a(static_cast<int>(wv.z), static_cast<int>(xv.z), s);
                is[b] = __dp4a(static_cast<int>(wv.w), static_cast<int>(xv.w), s);
              }
            }
          }
          const float sc = ss[kb * 32 + lane];
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            if (b < B) {
              const float pr = __fmul_rn(__int2float_rn(is[b]), sc);
              if (wpg == 1)
                acc[b] = __fadd_rn(acc[b], pr);
              else
                prod[((((buf * nmax + gi) * S + kb) * B + b) * 32) + lane] = pr;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (wpg > 1 && active) {
        // Every warp of the group has written its products of this step:
        // warp j adds, in block order, those of the beams b = j (mod wpg).
        if (lane == 0) mbar_arrive(&gbar[gi]);
        if (!mbar_wait(&gbar[gi], gphase & 1, &s_abort, p.err, kErrTimeoutConsumer)) {
          ok = false;
          break;
        }
        ++gphase;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < B && b % wpg == j) {
            const float* src = prod + (((buf * nmax + gi) * S) * B + b) * 32 + lane;
            for (int kb = 0; kb < sk; ++kb) acc[b] = __fadd_rn(acc[b], src[kb * B * 32]);
          }
        }
        buf ^= 1;
      }
    }
    if (ok && active) {
      const int row = (g0 + gi) * 32 + lane;
      if (row < p.rows) {
        const float cr = __ldg(p.corr + row);
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b < B && b % wpg == j)
            p.out[static_cast<size_t>(b) * p.rows + row] = __fmul_rn(__fsub_rn(acc[b], cr), s_sx[b]);
      }
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
  const int per_gb = blk * 32 + 128;  // one block of one group: weights and scales
  const int per_cta = static_cast<int>((groups + P.grid - 1) / P.grid);
  P.nmax = std::min(kGvWarps, per_cta);
  P.nmax = std::min(P.nmax, std::max(1, kGvStageBudget / per_gb));
  P.wpg = std::max(1, kGvWarps / P.nmax);
  const int nb = cols / blk;
  P.S = std::min(nb, std::max(1, kGvStageBudget / (P.nmax * per_gb)));
  if (P.wpg > 1 && P.S >= P.wpg) P.S = P.S / P.wpg * P.wpg;
  P.slot_bytes = P.nmax * P.S * per_gb;
  const int x_bytes = (batch * cols + 127) / 128 * 128;
  const int p_bytes = P.wpg > 1 ? 2 * P.nmax * P.S * batch * 128 : 0;
  const int bar_bytes = (2 * kGvMaxStages + kGvWarps) * 8;
  const int avail = kGvSmemMax - x_bytes - p_bytes - bar_bytes;
  P.stages = std::min(kGvMaxStages, avail / P.slot_bytes);
  if (P.stages < 2) return false;
  P.x_off = P.stages * P.slot_bytes;
  P.p_off = P.x_off + x_bytes;
  P.bar_off = P.p_off + p_bytes;
  P.smem = P.bar_off + bar_bytes;
  *plan = P;
  return true;
}

cudaError_t launch_int8_quantize(const void* w, int w_dtype, int rows, int cols, int blk,
                                 int8_t* qw, float* bscale, float* corr, cudaStream_t s) {
  const long long padded = int8_gemv_groups(rows) * 32;
  const int blocks = static_cast<int>((padded + 7) / 8);  // 8 warps of 32
  switch (w_dtype) {
    case 0:
      int8_quantize_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), rows, cols,
                                                         blk, qw, bscale, corr);
      break;
    case 1:
      int8_quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(w), rows, cols, blk, qw, bscale, corr);
      break;
    case 2:
      int8_quantize_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w), rows,
                                                          cols, blk, qw, bscale, corr);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_int8_gemv(const Int8GemvParams& p, cudaStream_t s) {
  const Int8GemvPlan& P = p.plan;
  if (p.batch < 1 || p.batch > kGvMaxBatch || !int8_gemv_served(p.cols, p.blk) ||
      P.smem > kGvSmemMax || P.stages < 2 || P.stages > kGvMaxStages || P.nmax > kGvWarps)
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // The attribute is per device; set it to the largest layout once.
  static std::atomic<bool> configured[64];
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    for (auto fn : {int8_gemv_kernel<1>, int8_gemv_kernel<2>, int8_gemv_kernel<4>,
                    int8_gemv_kernel<8>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kGvSmemMax);
      if (e != cudaSuccess) return e;
    }
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(P.grid));
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(P.smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.batch <= 1)
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<1>, p);
  else if (p.batch <= 2)
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<2>, p);
  else if (p.batch <= 4)
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<4>, p);
  else
    e = cudaLaunchKernelEx(&cfg, int8_gemv_kernel<8>, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ffai
