// Split-KV decode attention (q_len = 1) for Whisper decoder self- and
// cross-attention.
//
// Replaces the reference's streaming decode heads xattn_head /
// xattn_head_f16 (crates/ffai-mercury/src/asr/flash_attn.rs:602-696,
// :714-789): one query row per (beam, head) against `kv_len` cached keys.
// The reference runs one head at a time on one core; here every (row, key
// chunk) pair is a CTA, so a 60-row x 1500-key cross-attention step becomes
// 720 CTAs that stream the whole cache from HBM at once.
//
// Memory-bound: each CTA issues all of its 16-byte K and V loads up front
// (coalesced: a key's 64 values are one 128-byte line for bf16), computes its
// chunk's scores with lane-group shuffles, a chunk-local softmax (m, l) and
// the chunk's P.V, and writes a partial (m, l, o[64]) to the workspace.  The
// last CTA of a row to finish (an atomic ticket) combines the partials, so a
// decode step is a single launch.
#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

constexpr int kDecThreads = 128;

template <typename T>
struct Vec16 {  // 16 bytes of T
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
__device__ __forceinline__ void load16(Vec16<T>& dst, const T* src) {
  *reinterpret_cast<uint4*>(&dst) = __ldg(reinterpret_cast<const uint4*>(src));
}

__device__ __forceinline__ float load_q(const void* q, int dtype, size_t i) {
  if (dtype == 0) return static_cast<const float*>(q)[i];
  if (dtype == 1) return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
  return __half2float(static_cast<const __half*>(q)[i]);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// T: cache element type.  CH: max keys per CTA.  KT: K is head-dim major
// (B,H,64,cap) as the reference lays it out; otherwise row-major (B,H,cap,64).
template <typename T, int CH, bool KT>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(DecodeParams p) {
  constexpr int EPV = Vec16<T>::N;        // elements per 16-byte vector
  constexpr int TPK = 64 / EPV;           // threads per key
  constexpr int KPI = kDecThreads / TPK;  // keys per iteration
  constexpr int NI = CH / KPI;            // iterations to cover CH keys

  __shared__ float sq[64];
  __shared__ float ss[CH];
  __shared__ float red[kDecThreads / 32][64];
  __shared__ float sred[2][kDecThreads / 32];
  __shared__ int s_last;
  // K^T chunk staged as [64][CH] for the head-dim-major layout.
  __shared__ __align__(16) T skt[KT ? 64 * CH : 1];

  const int row = blockIdx.y;
  const int split = blockIdx.x;
  const int tid = threadIdx.x;
  const int k0 = split * p.chunk;
  const int n = min(p.chunk, p.kv_len - k0);
  const size_t cap = static_cast<size_t>(p.cap);

  const T* vrow = static_cast<const T*>(p.v) + static_cast<size_t>(row) * cap * 64;
  const int sub = tid % TPK;
  const int slot = tid / TPK;

  // Issue the V loads first: they do not depend on the scores, and keeping
  // them in flight while the scores are computed is what saturates HBM.
  Vec16<T> vreg[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int kk = slot + i * KPI;
    if (kk < n) load16(vreg[i], vrow + static_cast<size_t>(k0 + kk) * 64 + sub * EPV);
  }

  if (tid < 64) sq[tid] = load_q(p.q, p.q_dtype, static_cast<size_t>(row) * 64 + tid) * p.scale_log2;

  if constexpr (!KT) {
    const T* krow = static_cast<const T*>(p.k) + static_cast<size_t>(row) * cap * 64;
    Vec16<T> kreg[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int kk = slot + i * KPI;
      if (kk < n) load16(kreg[i], krow + static_cast<size_t>(k0 + kk) * 64 + sub * EPV);
    }
    __syncthreads();
    float qv[EPV];
#pragma unroll
    for (int e = 0; e < EPV; ++e) qv[e] = sq[sub * EPV + e];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int kk = slot + i * KPI;
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < EPV; ++e) a = fmaf(qv[e], to_f32(kreg[i].v[e]), a);
#pragma unroll
      for (int o = TPK / 2; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (sub == 0 && kk < n) ss[kk] = a;
    }
  } else {
    // Stage K^T[:, k0:k0+n] into shared memory, vectorised when the rows are
    // 16-byte aligned (cap and k0 multiples of EPV), element-wise otherwise.
    // A vector that starts below k0+n ends at or before cap, because cap and
    // its start are both multiples of EPV.
    const T* kbase = static_cast<const T*>(p.k) + static_cast<size_t>(row) * 64 * cap;
    if ((p.cap % EPV) == 0 && (k0 % EPV) == 0) {
      constexpr int VPR = CH / EPV;  // vectors per staged row
      for (int idx = tid; idx < 64 * VPR; idx += kDecThreads) {
        const int d = idx / VPR, c = idx % VPR;
        if (c * EPV < n) {
          Vec16<T> t;
          load16(t, kbase + static_cast<size_t>(d) * cap + k0 + c * EPV);
          *reinterpret_cast<Vec16<T>*>(&skt[d * CH + c * EPV]) = t;
        }
      }
    } else {
      for (int idx = tid; idx < 64 * CH; idx += kDecThreads) {
        const int d = idx / CH, c = idx % CH;
        if (c < n) skt[d * CH + c] = kbase[static_cast<size_t>(d) * cap + k0 + c];
      }
    }
    __syncthreads();
    for (int c = tid; c < n; c += kDecThreads) {
      float a = 0.f;
#pragma unroll 16
      for (int d = 0; d < 64; ++d) a = fmaf(sq[d], to_f32(skt[d * CH + c]), a);
      ss[c] = a;
    }
  }
  __syncthreads();

  // Chunk softmax in the log2 domain (q carries scale * log2 e).
  const int warp = tid / 32, lane = tid % 32;
  float mx = -INFINITY;
  for (int c = tid; c < n; c += kDecThreads) mx = fmaxf(mx, ss[c]);
  mx = warp_max(mx);
  if (lane == 0) sred[0][warp] = mx;
  __syncthreads();
  mx = sred[0][0];
#pragma unroll
  for (int w = 1; w < kDecThreads / 32; ++w) mx = fmaxf(mx, sred[0][w]);
  float l = 0.f;
  for (int c = tid; c < n; c += kDecThreads) {
    const float e = exp2f(ss[c] - mx);
    ss[c] = e;
    l += e;
  }
  l = warp_sum(l);
  if (lane == 0) sred[1][warp] = l;
  __syncthreads();
  l = 0.f;
#pragma unroll
  for (int w = 0; w < kDecThreads / 32; ++w) l += sred[1][w];

  // P.V: this thread owns head dims [sub*EPV, sub*EPV+EPV) for keys slot+i*KPI.
  float acc[EPV];
#pragma unroll
  for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int kk = slot + i * KPI;
    if (kk < n) {
      const float pk = ss[kk];
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[e] = fmaf(pk, to_f32(vreg[i].v[e]), acc[e]);
    }
  }
  // Reduce over the key slots of this warp (lanes sharing `sub`), then across warps.
#pragma unroll
  for (int e = 0; e < EPV; ++e) {
#pragma unroll
    for (int o = TPK; o < 32; o <<= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
  }
  if (lane < TPK) {
#pragma unroll
    for (int e = 0; e < EPV; ++e) red[warp][lane * EPV + e] = acc[e];
  }
  __syncthreads();

  float o_d = 0.f;
  if (tid < 64) {
#pragma unroll
    for (int w = 0; w < kDecThreads / 32; ++w) o_d += red[w][tid];
  }

  const float kLn2 = 0.69314718055994530942f;
  if (p.splits == 1) {
    if (tid < 64) {
      const float r = o_d / l;
      if (p.out_dtype == 0)
        static_cast<float*>(p.out)[static_cast<size_t>(row) * 64 + tid] = r;
      else
        static_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(row) * 64 + tid] = __float2bfloat16(r);
    }
    if (tid == 0 && p.lse) p.lse[row] = (mx + log2f(l)) * kLn2;
    return;
  }

  float* part = p.part + (static_cast<size_t>(row) * p.splits + split) * kPartStride;
  if (tid < 64) part[2 + tid] = o_d;
  if (tid == 0) {
    part[0] = mx;
    part[1] = l;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned ticket = atomicAdd(&p.counters[row], 1u);
    s_last = (ticket == static_cast<unsigned>(p.splits - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA of this row: merge the partials.
  const float* rp = p.part + static_cast<size_t>(row) * p.splits * kPartStride;
  if (tid < 64) {
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(rp + s * kPartStride));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float w = exp2f(__ldcg(rp + s * kPartStride) - M);
      L = fmaf(__ldcg(rp + s * kPartStride + 1), w, L);
      O = fmaf(__ldcg(rp + s * kPartStride + 2 + tid), w, O);
    }
    const float r = O / L;
    if (p.out_dtype == 0)
      static_cast<float*>(p.out)[static_cast<size_t>(row) * 64 + tid] = r;
    else
      static_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(row) * 64 + tid] = __float2bfloat16(r);
    if (tid == 0) {
      if (p.lse) p.lse[row] = (M + log2f(L)) * kLn2;
      p.counters[row] = 0u;  // re-arm the ticket for the next launch
    }
  }
}

template <typename T, int CH>
cudaError_t launch_t(const DecodeParams& p, cudaStream_t s) {
  dim3 grid(p.splits, p.rows);
  if (p.k_kt)
    decode_split_kernel<T, CH, true><<<grid, kDecThreads, 0, s>>>(p);
  else
    decode_split_kernel<T, CH, false><<<grid, kDecThreads, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_ch(const DecodeParams& p, cudaStream_t s) {
  if (p.chunk <= 64) return launch_t<T, 64>(p, s);
  return launch_t<T, 128>(p, s);
}

}  // namespace

cudaError_t launch_decode(const DecodeParams& p, cudaStream_t s) {
  switch (p.kv_dtype) {
    case 0:
      return launch_ch<float>(p, s);
    case 1:
      return launch_ch<__nv_bfloat16>(p, s);
    case 2:
      return launch_ch<__half>(p, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ffai
