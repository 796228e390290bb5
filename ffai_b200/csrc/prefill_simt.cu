// Checked f32 prefill attention on the CUDA cores.
//
// The f32 counterpart of the reference's encoder kernel, flash_head_strided
// (crates/ffai-mercury/src/asr/flash_attn.rs:429-487): 64 query rows per CTA
// stream over 64-key blocks with an online softmax in f32 and an exact
// `expf`.  It exists for callers that need f32 accuracy (relative error
// <= 1e-5 against the f32 reference) rather than the bf16 tensor-core path.
//
// Thread (ty, tx) of the 16x16 CTA owns query rows 4ty..4ty+3 and, for the
// scores, keys tx+16c (c < 4); for the output, head dims tx+16c.  Each thread
// also keeps the row sums of its four rows, accumulated in the P.V loop.  Shared
// tiles are padded to 65 floats per row so every access is bank-conflict free.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr int kBM = 64, kBN = 64, kPad = 65;

__global__ void __launch_bounds__(256) prefill_simt_kernel(SimtParams p) {
  extern __shared__ float sm[];
  float* sQ = sm;                 // [64][65]
  float* sK = sQ + kBM * kPad;    // [64][65]  key-major
  float* sV = sK + kBN * kPad;    // [64][65]  key-major
  float* sP = sV + kBN * kPad;    // [64][65]  row-major probabilities

  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * kBM;

  const float* qb = p.q + b * p.qs.sb + h * p.qs.sh;
  const float* kb = p.k + b * p.ks.sb + h * p.ks.sh;
  const float* vb = p.v + b * p.vs.sb + h * p.vs.sh;

  for (int idx = tid; idx < kBM * 64; idx += 256) {
    const int r = idx / 64, d = idx % 64;
    const int row = q0 + r;
    sQ[r * kPad + d] = row < p.Nq ? qb[row * p.qs.sr + d * p.qs.sd] * p.scale : 0.f;
  }

  float o[4][4], m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[i][c] = 0.f;
  }

  int kv_end = p.Nk;
  if (p.causal) kv_end = min(kv_end, p.q_offset + min(q0 + kBM, p.Nq));
  for (int k0 = 0; k0 < kv_end; k0 += kBN) {
    __syncthreads();  // previous block's sK/sV/sP reads are done
    for (int idx = tid; idx < kBN * 64; idx += 256) {
      int j, d;
      if (p.ks.sd == 1) {
        j = idx / 64;
        d = idx % 64;
      } else {  // head-dim-major K^T: walk keys fastest for coalescing
        d = idx / kBN;
        j = idx % kBN;
      }
      const int key = k0 + j;
      sK[j * kPad + d] = key < p.Nk ? kb[key * p.ks.sr + d * p.ks.sd] : 0.f;
    }
    for (int idx = tid; idx < kBN * 64; idx += 256) {
      const int j = idx / 64, d = idx % 64;
      const int key = k0 + j;
      sV[j * kPad + d] = key < p.Nk ? vb[key * p.vs.sr + d * p.vs.sd] : 0.f;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 8
    for (int d = 0; d < 64; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = sQ[(ty * 4 + i) * kPad + d];
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = sK[(tx + 16 * c) * kPad + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[i][c] = fmaf(qv[i], kv[c], s[i][c]);
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + ty * 4 + i;
      float bmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = k0 + tx + 16 * c;
        const bool ok = key < p.Nk && (!p.causal || key <= p.q_offset + row);
        if (!ok) s[i][c] = -INFINITY;
        bmax = fmaxf(bmax, s[i][c]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1)
        bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, off));
      const float m_new = fmaxf(m[i], bmax);
      const float corr = (m[i] == -INFINITY) ? 0.f : expf(m[i] - m_new);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
#pragma unroll
      for (int c = 0; c < 4; ++c) sP[(ty * 4 + i) * kPad + tx + 16 * c] = expf(s[i][c] - m_use);
      m[i] = m_new;
      l[i] *= corr;
#pragma unroll
      for (int c = 0; c < 4; ++c) o[i][c] *= corr;
    }
    __syncthreads();

#pragma unroll 4
    for (int j = 0; j < kBN; ++j) {
      float pv[4], vv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = sP[(ty * 4 + i) * kPad + j];
#pragma unroll
      for (int c = 0; c < 4; ++c) vv[c] = sV[j * kPad + tx + 16 * c];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int c = 0; c < 4; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
        // The normaliser accumulates the same products in the same order as
        // the outputs (a column of ones), so the applied weights P/l sum to 1
        // in this kernel's own f32 arithmetic.
        l[i] = fmaf(pv[i], 1.0f, l[i]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + ty * 4 + i;
    if (row >= p.Nq) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    const long long base = b * p.os.sb + h * p.os.sh + row * p.os.sr;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const long long off = base + (tx + 16 * c) * p.os.sd;
      const float r = o[i][c] * inv;
      if (p.out_dtype == 0)
        static_cast<float*>(p.out)[off] = r;
      else
        static_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16(r);
    }
    if (p.lse && tx == 0) p.lse[b * p.lse_sb + h * p.lse_sh + row] = m[i] + logf(l[i]);
  }
}

}  // namespace

cudaError_t launch_prefill_simt(const SimtParams& p, cudaStream_t s) {
  const size_t smem = 4 * 64 * kPad * sizeof(float);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[64];  // the attribute is per device
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(prefill_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  dim3 grid((p.Nq + kBM - 1) / kBM, p.B * p.H);
  prefill_simt_kernel<<<grid, 256, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ffai
