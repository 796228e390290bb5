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
#include <atomic>

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

// ---------------------------------------------------------------------------
// Cluster decode for row-major caches (keys of 64 contiguous values).
//
// Row r is split into S contiguous key ranges, one per CTA of a thread-block
// cluster of S CTAs (S <= 8), and the grid is rows x S CTAs with two CTAs
// resident per SM, so a Whisper decode step (60-100 rows) fills every SM in a
// single wave.  A producer lane copies the CTA's whole range into a ring of
// shared-memory stages with 1-d bulk copies at kernel start (refilling the
// ring only when a range is longer than the ring), so each SM has its share
// of the cache in flight at once.  The eight consumer warps take disjoint
// key slices of every stage and each keeps its own running (max, sum,
// output): no block-wide barrier inside the key loop.  The warps' partials
// merge once in shared memory, and the S CTAs' partials merge in the leader
// CTA's shared memory over the cluster (distributed shared memory), so the
// step needs no global workspace and no atomics.
//
// The kernel is launched as a programmatic dependent of the preceding kernel
// on the stream: its CTAs are scheduled while that kernel drains and wait for
// it (griddepcontrol.wait) before reading q; with kv_stable the producer
// copies the cache before that wait.
constexpr int kClWarps = 8;                        // consumer warps
constexpr int kClThreads = (kClWarps + 1) * 32;    // + one producer warp
constexpr int kClStages = 6;
constexpr int kClSlot = 66;                        // m, l, o[64]

template <typename T>
struct ClCfg {
  static constexpr int kKeys = 8192 / (64 * sizeof(T));  // keys per stage: 8 KB of K, 8 KB of V
  static constexpr int kWarpKeys = kKeys / kClWarps;     // keys per warp per stage
  static constexpr int kSteps = kWarpKeys / 4;           // 4 keys per warp-step
  static constexpr size_t kSmem = 2ull * kClStages * kKeys * 64 * sizeof(T) +
                                  2ull * kClStages * sizeof(uint64_t) +
                                  2ull * kClWarps * kClSlot * sizeof(float) + 16;
};

// Eight consecutive cache values as f32 (16-bit caches: one 16-byte load).
template <typename T>
__device__ __forceinline__ void load8_f32(const T* src, float (&x)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(src);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        x[2 * i] = __uint_as_float(u[i] << 16);
        x[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
      }
    }
  }
}

template <typename T, bool PAGED>
__global__ void __launch_bounds__(kClThreads, 2) decode_cluster_kernel(DecodeParams p, int S,
                                                                        int kpc) {
  using Cfg = ClCfg<T>;
  constexpr int KS = Cfg::kKeys;
  extern __shared__ __align__(128) uint8_t dsm[];
  T* kbuf = reinterpret_cast<T*>(dsm);
  T* vbuf = kbuf + kClStages * KS * 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(vbuf + kClStages * KS * 64);
  uint64_t* empty = full + kClStages;
  float* wslot = reinterpret_cast<float*>(empty + kClStages);  // [8][66] per-warp partials
  float* cslot = wslot + kClWarps * kClSlot;                   // [8][66] per-CTA partials (leader)
  __shared__ int s_abort;
  __shared__ int s_page[32];  // paged: the first 32 stages' pages, loaded in parallel

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int rank = S > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int row = blockIdx.x / S;
  if (S > 1) cluster_arrive_relaxed();  // paired with the wait before the merge
  griddep_launch_dependents();
  int len = p.kv_len;
  if constexpr (PAGED) {
    // kpc is page-aligned and comes from the host's length bound, so this
    // CTA's range start, and the pages of its first 32 stages, are known
    // before the dependency wait; the block table is written by the host,
    // not by the preceding kernel.  The lengths may come from the preceding
    // kernel (an append), so they are read after the wait.
    if (warp == kClWarps) {
      const int slot = (rank * kpc + lane * KS) / kPageKeys;
      if (lane * KS < kpc && slot < p.max_pages)
        s_page[lane] = __ldcg(p.block_table + static_cast<size_t>(row / p.heads) * p.max_pages + slot);
    }
    griddep_wait();
    len = min(max(__ldcg(p.seq_lens + row / p.heads), 0), p.max_pages * kPageKeys);
    if (len > S * kpc) {  // longer than the caller's bound: not covered, reported
      if (tid == 0 && rank == S - 1 && p.err) atomicOr(p.err, kErrBadArgs);
      len = S * kpc;
    }
  }
  const int k0 = min(len, rank * kpc);
  const int k1 = min(len, k0 + kpc);
  const int nch = (k1 - k0 + KS - 1) / KS;

  if (tid == 0) {
    for (int i = 0; i < kClStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kClWarps);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const size_t base = PAGED ? 0 : (static_cast<size_t>(row) * p.cap + k0) * 64;
  if (warp == kClWarps) {
    // Producer: all of the range's stages at once, then refills as warps free them.
    // With kv_append_only, only the row's newest key may still be written by
    // the preceding kernel: the stages before the one that holds it are
    // copied first, and the wait comes before that stage.
    const bool early = p.kv_stable || (!PAGED && p.kv_append_only);
    if (!early) griddep_wait();
    if constexpr (PAGED) __syncwarp();  // s_page written by the warp's lanes
    if (lane == 0) {
      int issued = 0;
      bool waited = !early || p.kv_stable;
      for (int c = 0; c < nch; ++c) {
        const int st = c % kClStages;
        if (!waited && k0 + (c + 1) * KS >= len) {  // this stage holds key len - 1
          griddep_wait();
          waited = true;
        }
        if (c >= kClStages &&
            !mbar_wait(&empty[st], ((c / kClStages) - 1) & 1, &s_abort, p.err, kErrTimeoutProducer))
          break;
        const int n = min(KS, k1 - k0 - c * KS);
        const uint32_t bytes = static_cast<uint32_t>(n) * 64 * sizeof(T);
        size_t off = base + static_cast<size_t>(c) * KS * 64;
        bool ok_src = true;
        if constexpr (PAGED) {
          // A stage never crosses a page: ranges start on page boundaries and
          // KS divides kPageKeys.
          const int j0 = k0 + c * KS;
          const int page = (c < 32 && k0 == rank * kpc)
                               ? s_page[c]
                               : __ldcg(p.block_table +
                                        static_cast<size_t>(row / p.heads) * p.max_pages +
                                        j0 / kPageKeys);
          ok_src = page >= 0 && page < p.num_pages;
          off = ((static_cast<size_t>(page) * p.heads + row % p.heads) * kPageKeys +
                 j0 % kPageKeys) * 64;
        }
        if (ok_src) {
          mbar_arrive_expect_tx(&full[st], 2 * bytes);
          bulk_load(kbuf + st * KS * 64, static_cast<const T*>(p.k) + off, bytes, &full[st]);
          bulk_load(vbuf + st * KS * 64, static_cast<const T*>(p.v) + off, bytes, &full[st]);
        } else {  // bad page id: flag it, copy nothing, let the stage complete
          if (p.err) atomicOr(p.err, kErrBadArgs);
          mbar_arrive(&full[st]);
        }
        ++issued;
        // The ring is filled (or the range issued): bring the same keys of
        // the next call's cache into L2 behind this CTA's own copies.
        if (!PAGED && p.pf_k && c == min(nch, kClStages) - 1) {
          const uint32_t pf = static_cast<uint32_t>(k1 - k0) * 64 * sizeof(T);
          bulk_prefetch_l2(static_cast<const T*>(p.pf_k) + base, pf);
          bulk_prefetch_l2(static_cast<const T*>(p.pf_v) + base, pf);
        }
      }
      if (s_abort) {
        // Wait (bounded, ignoring the abort flag) for the last armed phase of
        // every stage so no copy lands after the CTA has exited.
        int none = 0;
        for (int i = 0; i < kClStages && i < issued; ++i) {
          const int arms = (issued - 1 - i) / kClStages + 1;
          mbar_wait(&full[i], (arms - 1) & 1, &none, p.err, kErrTimeoutDrain);
        }
      }
    }
    __syncwarp();
  } else {
    // Consumer warp: lanes 8g..8g+7 hold key g of each 4-key step, 8 head
    // dims each (part); the running max m is warp-uniform.
    const int kin = lane / 8, part = lane % 8;
    griddep_wait();  // q (and the output buffers) belong to the preceding kernels
    float qv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      qv[e] = load_q(p.q, p.q_dtype, static_cast<size_t>(row) * 64 + part * 8 + e) * p.scale_log2;
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    for (int c = 0; c < nch; ++c) {
      const int st = c % kClStages;
      if (!mbar_wait(&full[st], (c / kClStages) & 1, &s_abort, p.err, kErrTimeoutConsumer)) break;
      const int n = min(KS, k1 - k0 - c * KS);
      const T* ks = kbuf + st * KS * 64;
      const T* vs = vbuf + st * KS * 64;
      float sc[Cfg::kSteps];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < Cfg::kSteps; ++i) {
        const int key = warp * Cfg::kWarpKeys + i * 4 + kin;
        float a = 0.f;
        if (key < n) {
          float x[8];
          load8_f32(ks + key * 64 + part * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) a = fmaf(qv[e], x[e], a);
        }
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        a += __shfl_xor_sync(0xffffffffu, a, 4);
        sc[i] = key < n ? a : -INFINITY;
        mx = fmaxf(mx, sc[i]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      if (mx > m) {  // warp-uniform
        const float corr = m == -INFINITY ? 0.f : exp2f(m - mx);
        m = mx;
        l *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= corr;
      }
#pragma unroll
      for (int i = 0; i < Cfg::kSteps; ++i) {
        const int key = warp * Cfg::kWarpKeys + i * 4 + kin;
        if (key < n) {
          const float pj = exp2f(sc[i] - m);
          l += pj;
          float x[8];
          load8_f32(vs + key * 64 + part * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = fmaf(pj, x[e], o[e]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // Sum the four key groups; lanes 0-7 then hold the warp's o[64].
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o[e] += __shfl_xor_sync(0xffffffffu, o[e], 8);
      o[e] += __shfl_xor_sync(0xffffffffu, o[e], 16);
    }
    float* ws = wslot + warp * kClSlot;
    if (lane < 8) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ws[2 + lane * 8 + e] = o[e];
    }
    if (lane == 0) {
      ws[0] = m;
      ws[1] = l;
    }
  }
  __syncthreads();

  // CTA partial over the eight warps (threads 0-63: one head dim each).
  float M = -INFINITY, L = 0.f, O = 0.f;
  if (tid < 64) {
#pragma unroll
    for (int w = 0; w < kClWarps; ++w) M = fmaxf(M, wslot[w * kClSlot]);
#pragma unroll
    for (int w = 0; w < kClWarps; ++w) {
      const float mw = wslot[w * kClSlot];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L = fmaf(wslot[w * kClSlot + 1], f, L);
      O = fmaf(wslot[w * kClSlot + 2 + tid], f, O);
    }
  }
  if (S > 1) {
    __syncwarp();
    cluster_wait();  // every CTA of the cluster has started: its shared memory is mapped
    if (tid < 64) {
      const uint32_t dst = mapa_shared(smem_u32(cslot + rank * kClSlot), 0);
      st_cluster_f32(dst + 4u * (2 + tid), O);
      if (tid == 0) {
        st_cluster_f32(dst, M);
        st_cluster_f32(dst + 4u, L);
      }
    }
    __syncwarp();
    cluster_arrive();
    cluster_wait();
    if (rank != 0) return;
    if (tid < 64) {
      M = -INFINITY;
      for (int c = 0; c < S; ++c) M = fmaxf(M, cslot[c * kClSlot]);
      L = 0.f;
      O = 0.f;
      for (int c = 0; c < S; ++c) {
        const float mc = cslot[c * kClSlot];
        const float f = mc == -INFINITY ? 0.f : exp2f(mc - M);
        L = fmaf(cslot[c * kClSlot + 1], f, L);
        O = fmaf(cslot[c * kClSlot + 2 + tid], f, O);
      }
    }
  }
  if (tid < 64) {
    const float val = L > 0.f ? O / L : 0.f;  // a paged row with no keys gives zeros
    if (p.out_dtype == 0)
      static_cast<float*>(p.out)[static_cast<size_t>(row) * 64 + tid] = val;
    else
      static_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(row) * 64 + tid] =
          __float2bfloat16(val);
    if (tid == 0 && p.lse) p.lse[row] = (M + log2f(L)) * 0.69314718055994530942f;
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

template <typename T, bool PAGED>
cudaError_t launch_cluster_t(const DecodeParams& p, int S, int kpc, cudaStream_t s) {
  const size_t smem = ClCfg<T>::kSmem;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[64];  // per device; racing first calls both set it
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(decode_cluster_kernel<T, PAGED>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows) * S);
  cfg.blockDim = dim3(kClThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, decode_cluster_kernel<T, PAGED>, p, S, kpc);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_cluster(const DecodeParams& p, int splits, int keys_per_cta,
                                  cudaStream_t s) {
  if (splits < 1 || splits > kDecodeMaxCluster) return cudaErrorInvalidValue;
  switch (p.kv_dtype) {
    case 0:
      return launch_cluster_t<float, false>(p, splits, keys_per_cta, s);
    case 1:
      return launch_cluster_t<__nv_bfloat16, false>(p, splits, keys_per_cta, s);
    case 2:
      return launch_cluster_t<__half, false>(p, splits, keys_per_cta, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode_paged(const DecodeParams& p, int splits, cudaStream_t s) {
  if (splits < 1 || splits > kDecodeMaxCluster) return cudaErrorInvalidValue;
  // Page-aligned ranges over the length bound p.kv_len.
  const int kpc = ((p.kv_len + splits - 1) / splits + kPageKeys - 1) / kPageKeys * kPageKeys;
  switch (p.kv_dtype) {
    case 0:
      return launch_cluster_t<float, true>(p, splits, kpc, s);
    case 1:
      return launch_cluster_t<__nv_bfloat16, true>(p, splits, kpc, s);
    case 2:
      return launch_cluster_t<__half, true>(p, splits, kpc, s);
  }
  return cudaErrorInvalidValue;
}

namespace {

// One CTA per sequence: writes its heads' new key and value rows at the
// sequence's current length, then advances the length.
template <typename T>
__global__ void kv_append_kernel(DecodeParams p, const T* k_new, const T* v_new) {
  const int b = blockIdx.x;
  __shared__ int s_pos, s_page;
  if (threadIdx.x == 0) {
    s_pos = p.seq_lens[b];
    const int slot = s_pos / kPageKeys;
    s_page = (s_pos >= 0 && slot < p.max_pages)
                 ? p.block_table[static_cast<size_t>(b) * p.max_pages + slot]
                 : -1;
    if (s_page < 0 || s_page >= p.num_pages) {
      if (p.err) atomicOr(p.err, kErrBadArgs);
      s_page = -1;
    }
  }
  __syncthreads();
  if (s_page < 0) return;
  const int pos = s_pos;
  T* kd = static_cast<T*>(const_cast<void*>(p.k));
  T* vd = static_cast<T*>(const_cast<void*>(p.v));
  for (int i = threadIdx.x; i < p.heads * 64; i += blockDim.x) {
    const int h = i / 64, d = i % 64;
    const size_t dst =
        ((static_cast<size_t>(s_page) * p.heads + h) * kPageKeys + pos % kPageKeys) * 64 + d;
    const size_t src = (static_cast<size_t>(b) * p.heads + h) * 64 + d;
    kd[dst] = k_new[src];
    vd[dst] = v_new[src];
  }
  __syncthreads();
  if (threadIdx.x == 0) const_cast<int*>(p.seq_lens)[b] = pos + 1;
}

// Block i copies page src[i] to page dst[i] in both pools, 16 bytes a thread.
__global__ void kv_copy_pages_kernel(DecodeParams p, const int* src, const int* dst,
                                     size_t page_bytes) {
  const int a = src[blockIdx.x], b = dst[blockIdx.x];
  if (a < 0 || a >= p.num_pages || b < 0 || b >= p.num_pages) {
    if (threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadArgs);
    return;
  }
  const uint4* ks = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.k) + a * page_bytes);
  const uint4* vs = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.v) + a * page_bytes);
  uint4* kd = reinterpret_cast<uint4*>(static_cast<uint8_t*>(const_cast<void*>(p.k)) + b * page_bytes);
  uint4* vd = reinterpret_cast<uint4*>(static_cast<uint8_t*>(const_cast<void*>(p.v)) + b * page_bytes);
  for (size_t i = threadIdx.x; i < page_bytes / 16; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

}  // namespace

cudaError_t launch_kv_append(const DecodeParams& p, int batch, const void* k_new,
                             const void* v_new, cudaStream_t s) {
  switch (p.kv_dtype) {
    case 0:
      kv_append_kernel<float><<<batch, 256, 0, s>>>(p, static_cast<const float*>(k_new),
                                                    static_cast<const float*>(v_new));
      break;
    case 1:
      kv_append_kernel<__nv_bfloat16><<<batch, 256, 0, s>>>(
          p, static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new));
      break;
    case 2:
      kv_append_kernel<__half><<<batch, 256, 0, s>>>(p, static_cast<const __half*>(k_new),
                                                     static_cast<const __half*>(v_new));
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_kv_copy_pages(const DecodeParams& p, const int* src, const int* dst, int n,
                                 cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const size_t elem = p.kv_dtype == 0 ? 4 : 2;
  const size_t page_bytes = static_cast<size_t>(p.heads) * kPageKeys * 64 * elem;
  kv_copy_pages_kernel<<<n, 256, 0, s>>>(p, src, dst, page_bytes);
  return cudaGetLastError();
}

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
