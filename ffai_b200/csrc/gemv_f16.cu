// f16-weight GEMV for the decoder's single-row projections.
//
// Replaces the reference's AVX2 + F16C F16Gemv (crates/ffai-mercury/src/asr/
// f16_gemv.rs), the default path of the decoder's q/k/v/out projections and
// MLP (QLinear::Half, text_decoder.rs:106-118, loaded by from_vb_gemv_f16,
// :231-252).  Same arithmetic, so the outputs equal the reference's bit for
// bit: weights rounded to f16 once (nearest-even), widened back to f32; per
// output row, 16 f32 accumulators -- chain c takes the columns 16 j + c in
// order of j with a fused multiply-add (dot_f16, :170-194: two 8-lane
// accumulators stepping 16 columns, an 8-column tail into the first) -- then
// the fixed reduction ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)) with
// a_i = c_i + c_{i+8}; the bias, when the layer has one, is added after
// (QLinear::forward, :281-289).
//
// B200 layout: HBM-bound (2 bytes per weight per token).  The sixteen chains
// of a row are sixteen lanes of a warp, each chain a sequential FMA over the
// row; the reduction is four shuffles.  A lane keeps its chain for 4 rows and
// a warp takes 8 rows, so an activation value loaded from shared memory
// feeds 4 rows (shared-memory traffic, not HBM, is what limits several
// activation rows).  Where a matrix has few groups for its width (the
// tall, narrow fc2 and out-projection), 2 or 4 warps share a group, each
// taking 2 or 1 of a lane's 4 rows: more chains in flight, same layout.  Weights are stored [8-row group][16-column step][column]
// [8 rows], so a lane's 4 rows are one 8-byte load, a warp's step 256
// contiguous bytes and a run of a group's steps one bulk copy.  Streaming
// as in the int8 GEMV (gemv_int8.cu): persistent CTAs over contiguous group
// ranges, rounds of one group per consumer warp, units of S steps through a
// ring of shared-memory slots, one producer lane per slot.  The activation
// rows of a call (beams, up to 8) share the weight stream; they are read
// through L1.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

#ifndef FFAI_HG_WARPS
#define FFAI_HG_WARPS 24
#endif
#ifndef FFAI_HG_SLOT_TARGET
#define FFAI_HG_SLOT_TARGET 8192
#endif
constexpr int kHgConsWarps = FFAI_HG_WARPS;
constexpr int kHgThreads = (kHgConsWarps + 1) * 32;  // + the producer warp
constexpr int kHgSlotTarget = FFAI_HG_SLOT_TARGET;
constexpr int kHgMaxRing = 32;  // one producer lane per slot
constexpr int kHgStepBytes = kHgRows * 16 * 2;
constexpr int kHgStepHalves = kHgRows * 16;
// Dynamic shared memory per block (227 KB less a little for static arrays);
// without staged activations the ring leaves kHgL1Room of it to L1.
constexpr int kHgSmemMax = 227 * 1024 - 1024;
constexpr int kHgL1Room = 64 * 1024;

// Row-major weights of w_dtype -> f16 (nearest-even) in the packed layout;
// one thread per output half.
template <typename T>
__global__ void f16_pack_kernel(const T* w, int rows, int cols, uint16_t* packed) {
  const int steps = f16_gemv_steps(cols);
  const long long groups = f16_gemv_groups(rows);
  const long long n = groups * steps * kHgStepHalves;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int ri = static_cast<int>(i % kHgRows);         // 4 s + i
    const int c = static_cast<int>((i / kHgRows) % 16);
    const long long gj = i / kHgStepHalves;
    const int j = static_cast<int>(gj % steps);
    const long long g = gj / steps;
    const long long row = g * kHgRows + ri;
    const int col = 16 * j + c;
    uint16_t h = 0;
    if (row < rows && col < cols)
      h = __half_as_ushort(__float2half_rn(to_f32(w[row * cols + col])));
    packed[i] = h;
  }
}

// XS: the activations staged in shared memory, chain-major ([row b][chain c]
// [step j], a lane's next 4 steps one 16-byte load); else read through L1.
// LR: rows per lane (4 or 2), i.e. 4 / LR warps per group.
template <int NB, bool XS, int LR>
__global__ void __launch_bounds__(kHgThreads, 1) f16_gemv_kernel(F16GemvParams p) {
  constexpr int Q = kHgLaneRows / LR;          // warps per group
  constexpr int kGpr = kHgConsWarps / Q;       // groups per round
  const F16GemvPlan& P = p.plan;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + P.bar_off);
  uint64_t* empty = full + kHgMaxRing;
  __shared__ int s_use[kHgMaxRing];  // see wait_slot_use
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int cols = p.cols, steps = f16_gemv_steps(cols);
  const int S = P.S, ring = P.ring;
  const int upg = (steps + S - 1) / S;  // units per group
  const int g_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * P.groups / P.grid);
  const int g_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * P.groups / P.grid);

  if (tid == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Q);  // the warps that own the unit's group
      s_use[i] = -1;
    }
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  // Producer: lane r refills slot r with units r, r + ring, ... of the
  // stream (round by round: unit k of each of the round's groups).
  if (warp == kHgConsWarps) {
    if (!p.weights_stable) griddep_wait();
    if (lane >= ring) return;
    uint64_t* fb = &full[lane];
    const int units = (g_end - g_begin) * upg;
    const int full_round = kGpr * upg;
    int issued = 0;
    bool ok = true;
    for (int j = lane; j < units; j += ring, ++issued) {
      if (issued > 0 &&
          !mbar_wait(&empty[lane], (issued - 1) & 1, &s_abort, p.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      const int ro = j / full_round, g0 = g_begin + ro * kGpr;
      const int n = min(kGpr, g_end - g0), rem = j - ro * full_round;
      const int k = rem / n, i = rem - k * n;
      const uint32_t bytes = static_cast<uint32_t>(min(S, steps - k * S)) * kHgStepBytes;
      *reinterpret_cast<volatile int*>(&s_use[lane]) = issued;
      mbar_arrive_expect_tx(fb, bytes);
      bulk_load(dsm + static_cast<size_t>(lane) * P.slot_bytes,
                reinterpret_cast<const uint8_t*>(p.packed) +
                    (static_cast<size_t>(g0 + i) * steps + static_cast<size_t>(k) * S) * kHgStepBytes,
                bytes, fb);
    }
    if (issued > 0 && (!ok || s_abort)) {
      int none = 0;  // let this slot's last copy land before the CTA exits
      mbar_wait(fb, (issued - 1) & 1, &none, p.err, kErrTimeoutDrain);
    }
    return;
  }

  griddep_wait();  // the activations come from the preceding kernel
  // Lane (r, c): chain c of row r of the warp's group.  A step past `cols`
  // (the 8-column tail) is taken by chains 0-7 only, as the reference's
  // tail loop feeds only its first accumulator.
  // rows 4 r + LR q .. + LR - 1 of the warp's group gi
  const int r = lane >> 4, c = lane & 15, gi = warp / Q, q = warp - gi * Q;
  const bool tail8 = (cols & 15) != 0;
  const float* xb = p.x + c;
  float* xt = reinterpret_cast<float*>(dsm + P.x_off);
  const int pitch = P.x_pitch;  // floats per (row, chain); a multiple of 4, odd / 4
  if constexpr (XS) {
    // Item (b, quad, c): chain c's steps 4 quad .. 4 quad + 3 of activation
    // row b, gathered (a half-warp reads 64 contiguous bytes per step) into
    // one 16-byte store.  Items are walked without division; two items'
    // loads are in flight before their stores.
    constexpr int kStride = kHgConsWarps * 32;
    const int per_b = 16 * ((steps + 3) / 4), total = NB * per_b;
    auto gather = [&](int b, int rem, float (&v)[4]) {
      const float* xr = p.x + static_cast<size_t>(b) * cols + (rem & 15) + 64 * (rem >> 4);
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = 64 * (rem >> 4) + 16 * u + (rem & 15) < cols ? xr[16 * u] : 0.f;
    };
    auto put = [&](int b, int rem, const float (&v)[4]) {
      *reinterpret_cast<float4*>(xt + (b * 16 + (rem & 15)) * pitch + 4 * (rem >> 4)) =
          make_float4(v[0], v[1], v[2], v[3]);
    };
    auto advance = [&](int& b, int& rem) {
      rem += kStride;
      while (rem >= per_b) {
        rem -= per_b;
        ++b;
      }
    };
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) {
      // 16-byte loads of 4 consecutive columns (4 chains of one step), all
      // activation rows' loads in flight before the scattered 4-byte stores
      for (int j = tid; j < cols / 4; j += kStride) {
        float4 v[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b)
          v[b] = *reinterpret_cast<const float4*>(p.x + static_cast<size_t>(b) * cols + 4 * j);
        const int step = j >> 2, c0 = (4 * j) & 15;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          float* d = xt + (b * 16 + c0) * pitch + step;
          d[0] = v[b].x;
          d[pitch] = v[b].y;
          d[2 * pitch] = v[b].z;
          d[3 * pitch] = v[b].w;
        }
      }
    } else {
      int b0 = 0, r0 = tid;
      while (r0 >= per_b) {
        r0 -= per_b;
        ++b0;
      }
      for (int i = tid; i < total; i += 2 * kStride) {
        int b1 = b0, r1 = r0;
        advance(b1, r1);
        float v0[4], v1[4];
        gather(b0, r0, v0);
        const bool two = i + kStride < total;
        if (two) gather(b1, r1, v1);
        put(b0, r0, v0);
        if (two) put(b1, r1, v1);
        b0 = b1;
        r0 = r1;
        advance(b0, r0);
      }
    }
    named_bar_sync(1, kHgConsWarps * 32);
  }
  const float* xl = xt + c * pitch;  // this lane's chain, row 0
  auto x1 = [&](int b, int step) -> float {
    if constexpr (XS)
      return xl[b * 16 * pitch + step];
    else
      return __ldg(xb + static_cast<size_t>(b) * cols + 16 * step);
  };
  int j0 = 0;  // stream index of the round's first unit
  for (int g0 = g_begin; g0 < g_end; g0 += kGpr) {
    const int n = min(kGpr, g_end - g0);
    if (gi >= n) {
      j0 += n * upg;
      continue;
    }
    float acc[NB][LR];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int i = 0; i < LR; ++i) acc[b][i] = 0.f;
    bool ok = true;
    for (int k = 0; k < upg; ++k) {
      const int j = j0 + k * n + gi, slot = j % ring, use = j / ring;
      if (!wait_slot_use(&s_use[slot], use, &s_abort, p.err) ||
          !mbar_wait(&full[slot], use & 1, &s_abort, p.err, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      const int s0 = k * S, sk = min(S, steps - s0);
      // the last step of the row, when it is the 8-column tail: chains 0-7
      const int full_steps = (tail8 && s0 + sk == steps) ? sk - 1 : sk;
      // this lane's LR rows of column 16 j + c: 2 LR bytes at step j
      const __half* wsl = reinterpret_cast<const __half*>(dsm + static_cast<size_t>(slot) * P.slot_bytes) +
                          c * kHgRows + kHgLaneRows * r + LR * q;
      auto wrow = [&](int step, float (&wv)[LR]) {
        const __half* h = wsl + step * kHgStepHalves;
        if constexpr (LR == 4) {
          const uint2 u = *reinterpret_cast<const uint2*>(h);
          const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
          const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
          wv[0] = lo.x;
          wv[1] = lo.y;
          wv[2] = hi.x;
          wv[3] = hi.y;
        } else {
          static_assert(LR == 2, "rows per lane");
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(h));
          wv[0] = f.x;
          wv[1] = f.y;
        }
      };
      int t = 0;
      if constexpr (XS) {
        // s0 and t are multiples of 4: the activations of 4 steps are one
        // float4.  kXU steps' loads are issued before their FMAs (one or two
        // warps per scheduler here: the shared-memory latency needs ILP).
        constexpr int kXU = LR == 2 ? 8 : 4;
        auto batch = [&](auto xu) {
          constexpr int U = decltype(xu)::value;
          float wv[U][LR];
#pragma unroll
          for (int u = 0; u < U; ++u) wrow(t + u, wv[u]);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int h = 0; h < U / 4; ++h) {
              const float4 xv = *reinterpret_cast<const float4*>(xl + b * 16 * pitch + s0 + t + 4 * h);
              const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int i = 0; i < LR; ++i)
                  acc[b][i] = __fmaf_rn(wv[4 * h + u][i], xs[u], acc[b][i]);
            }
          }
        };
        for (; t + kXU <= full_steps; t += kXU) batch(std::integral_constant<int, kXU>{});
        for (; t + 4 <= full_steps; t += 4) batch(std::integral_constant<int, 4>{});
      } else {
        for (; t + 2 <= full_steps; t += 2) {
          float wv[2][LR], xv[2][NB];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            wrow(t + u, wv[u]);
#pragma unroll
            for (int b = 0; b < NB; ++b) xv[u][b] = x1(b, s0 + t + u);
          }
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int b = 0; b < NB; ++b)
#pragma unroll
              for (int i = 0; i < LR; ++i) acc[b][i] = __fmaf_rn(wv[u][i], xv[u][b], acc[b][i]);
        }
      }
      for (; t < full_steps; ++t) {
        float wv[LR];
        wrow(t, wv);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float xv = x1(b, s0 + t);
#pragma unroll
          for (int i = 0; i < LR; ++i) acc[b][i] = __fmaf_rn(wv[i], xv, acc[b][i]);
        }
      }
      if (full_steps < sk && c < 8) {
        float wv[LR];
        wrow(full_steps, wv);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float xv = x1(b, s0 + full_steps);
#pragma unroll
          for (int i = 0; i < LR; ++i) acc[b][i] = __fmaf_rn(wv[i], xv, acc[b][i]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    j0 += n * upg;
    if (!ok) break;
    // ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)), a_i = c_i + c_{i+8}:
    // each add is of a pair of lanes, and IEEE addition is commutative
#pragma unroll
    for (int i = 0; i < LR; ++i) {
      const int row = (g0 + gi) * kHgRows + kHgLaneRows * r + LR * q + i;
      const float bias = (p.bias != nullptr && row < p.rows) ? __ldg(p.bias + row) : 0.f;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float v = acc[b][i];
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        if (c == 0 && row < p.rows)
          p.out[static_cast<size_t>(b) * p.rows + row] = p.bias != nullptr ? __fadd_rn(v, bias) : v;
      }
    }
  }
}

template <int NB, int LR>
cudaError_t launch_nb_lr(const F16GemvParams& p, cudaLaunchConfig_t& cfg) {
  return p.plan.x_pitch > 0 ? cudaLaunchKernelEx(&cfg, f16_gemv_kernel<NB, true, LR>, p)
                            : cudaLaunchKernelEx(&cfg, f16_gemv_kernel<NB, false, LR>, p);
}

template <int NB>
cudaError_t launch_nb(const F16GemvParams& p, cudaLaunchConfig_t& cfg) {
  return p.plan.q == 2 ? launch_nb_lr<NB, 2>(p, cfg) : launch_nb_lr<NB, 4>(p, cfg);
}

template <int NB>
cudaError_t configure_nb() {
  for (auto fn : {f16_gemv_kernel<NB, true, 4>, f16_gemv_kernel<NB, false, 4>,
                  f16_gemv_kernel<NB, true, 2>, f16_gemv_kernel<NB, false, 2>}) {
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kHgSmemMax);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool f16_gemv_plan(int rows, int cols, int batch, int sms, F16GemvPlan* plan) {
  if (!f16_gemv_served(cols) || rows <= 0 || batch < 1 || batch > kHgMaxBatch || sms <= 0)
    return false;
  F16GemvPlan P{};
  const long long groups = f16_gemv_groups(rows);
  P.groups = static_cast<int>(groups);
  P.grid = static_cast<int>(std::min<long long>(sms, groups));
  // Two warps per group where that leaves the number of rounds of the
  // busiest CTA unchanged (the extra warps would otherwise idle).  Measured
  // on the decoder's shapes: 2 beats 1 by 4-22 %; 4 loses to 2 everywhere
  // (each warp's 2-byte loads and conversions outweigh the extra chains).
  const int gpc = static_cast<int>((groups + P.grid - 1) / P.grid);
  auto rounds = [&](int q) { return (gpc + kHgConsWarps / q - 1) / (kHgConsWarps / q); };
  P.q = rounds(2) == rounds(1) ? 2 : 1;
  const int steps = f16_gemv_steps(cols);
  const int upg = std::max(1, (steps * kHgStepBytes + kHgSlotTarget - 1) / kHgSlotTarget);
  P.S = ((steps + upg - 1) / upg + 3) / 4 * 4;  // a multiple of 4 steps
  P.slot_bytes = P.S * kHgStepBytes;
  const int bar_bytes = 2 * kHgMaxRing * 8;
  // Activations in shared memory when they leave room for a ring of 4
  // slots.  The pitch (floats per activation row and chain) is 4 x an odd
  // number, so the 16-byte loads of 8 consecutive chains fall in 8 different
  // bank groups: a row's 16 chains are two wavefronts.
  int q4 = (steps + 3) / 4;
  if (q4 % 2 == 0) ++q4;
  const long long x_bytes = static_cast<long long>(batch) * 16 * 4 * q4 * 4;
  const bool xs = x_bytes + 4LL * P.slot_bytes + bar_bytes <= kHgSmemMax;
  P.x_pitch = xs ? 4 * q4 : 0;
  const int ring_bytes = kHgSmemMax - bar_bytes - (xs ? static_cast<int>(x_bytes) : kHgL1Room);
  P.ring = std::min(kHgMaxRing, ring_bytes / P.slot_bytes);
  if (P.ring < 2) return false;
  P.bar_off = P.ring * P.slot_bytes;
  P.x_off = P.bar_off + bar_bytes;
  P.smem = P.x_off + (xs ? static_cast<int>(x_bytes) : 0);
  *plan = P;
  return true;
}

cudaError_t launch_f16_pack(const void* w, int w_dtype, int rows, int cols, uint16_t* packed,
                            cudaStream_t s) {
  const long long n = f16_gemv_groups(rows) * f16_gemv_steps(cols) * kHgStepHalves;
  const int blocks = static_cast<int>(std::min<long long>((n + 255) / 256, 65535));
  switch (w_dtype) {
    case 0:
      f16_pack_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), rows, cols, packed);
      break;
    case 1:
      f16_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w),
                                                            rows, cols, packed);
      break;
    case 2:
      f16_pack_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w), rows, cols,
                                                     packed);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_f16_gemv(const F16GemvParams& p, cudaStream_t s) {
  const F16GemvPlan& P = p.plan;
  if (p.batch < 1 || p.batch > kHgMaxBatch || !f16_gemv_served(p.cols) || P.smem > kHgSmemMax ||
      P.ring < 2 || P.ring > kHgMaxRing || (P.q != 1 && P.q != 2))
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[64];
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    for (auto cfg_fn : {configure_nb<1>, configure_nb<2>, configure_nb<3>, configure_nb<4>,
                        configure_nb<5>, configure_nb<6>, configure_nb<7>, configure_nb<8>}) {
      e = cfg_fn();
      if (e != cudaSuccess) return e;
    }
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(P.grid));
  cfg.blockDim = dim3(kHgThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(P.smem);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (p.batch) {
    case 1: e = launch_nb<1>(p, cfg); break;
    case 2: e = launch_nb<2>(p, cfg); break;
    case 3: e = launch_nb<3>(p, cfg); break;
    case 4: e = launch_nb<4>(p, cfg); break;
    case 5: e = launch_nb<5>(p, cfg); break;
    case 6: e = launch_nb<6>(p, cfg); break;
    case 7: e = launch_nb<7>(p, cfg); break;
    default: e = launch_nb<8>(p, cfg); break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ffai
