// Operand preparation for the tensor-core prefill: gather f32/bf16/f16
// operands of any supported layout into contiguous heads-split (B,H,N,64)
// 16-bit (bf16 or f16) buffers, all of a call's operands in one launch.
// Used for the reference's f32 operands (its callers hold f32 candle tensors,
// flash_attn.rs:212-217) and for K^T (B,H,64,N) whose row pitch is not a
// multiple of 16 bytes and so cannot be described to TMA.
#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

template <bool F16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  return F16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

// Row-major source: one warp per destination row (64 elements, two per lane).
template <typename T, bool F16>
__device__ __forceinline__ void stage_rows(const StageOp& op, int H, long long blk) {
  const long long rows = op.rows;
  const long long row = (blk * 256 + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const Strides st = op.st;
  const int n = static_cast<int>(row % op.N);
  const long long bh = row / op.N;
  const int h = static_cast<int>(bh % H);
  const long long b = bh / H;
  const T* s = static_cast<const T*>(op.src) + b * st.sb + h * st.sh + n * st.sr;
  const float x0 = to_f32(s[(2 * lane) * st.sd]);
  const float x1 = to_f32(s[(2 * lane + 1) * st.sd]);
  reinterpret_cast<uint32_t*>(op.dst + row * 64)[lane] = pack16<F16>(x0, x1);
}

// Head-dim-major source (sd != 1, sr == 1): a 64x64 tile transposed through
// shared memory so both the reads (along keys) and writes (along dims) coalesce.
template <typename T, bool F16>
__device__ __forceinline__ void stage_kt(const StageOp& op, int H, long long blk,
                                         float (&tile)[64][65]) {
  const int ntiles = (op.N + 63) / 64;
  const long long bh = blk / ntiles;
  const int n0 = static_cast<int>(blk % ntiles) * 64;
  const int h = static_cast<int>(bh % H);
  const long long b = bh / H;
  const Strides st = op.st;
  const T* s = static_cast<const T*>(op.src) + b * st.sb + h * st.sh;
  for (int idx = threadIdx.x; idx < 64 * 64; idx += blockDim.x) {
    const int d = idx / 64, j = idx % 64;
    const int n = n0 + j;
    tile[d][j] = n < op.N ? to_f32(s[static_cast<long long>(n) * st.sr + d * st.sd]) : 0.f;
  }
  __syncthreads();
  uint16_t* o = op.dst + (bh * op.N) * 64;
  for (int idx = threadIdx.x; idx < 64 * 32; idx += blockDim.x) {
    const int j = idx / 32, dp = idx % 32;
    const int n = n0 + j;
    if (n < op.N)
      reinterpret_cast<uint32_t*>(o + static_cast<long long>(n) * 64)[dp] =
          pack16<F16>(tile[2 * dp][j], tile[2 * dp + 1][j]);
  }
}

// Up to three operands in one launch (q, k, v of one prefill call): block
// ranges [end[i-1], end[i]) convert operand i, with the row-major or the
// K^T body above.  A programmatic dependent of the preceding kernel (its
// sources may come from there), letting the prefill that reads its output
// launch at once.
template <bool F16>
__global__ void __launch_bounds__(256) stage_kernel(StageBatch sb) {
  __shared__ float tile[64][65];
  griddep_wait();
  griddep_launch_dependents();
  int i = 0;
  while (i + 1 < sb.n && blockIdx.x >= sb.end[i]) ++i;
  const StageOp& op = sb.op[i];
  const long long blk = static_cast<long long>(blockIdx.x) - (i ? sb.end[i - 1] : 0);
  if (op.kt) {
    switch (op.src_dtype) {
      case 0: stage_kt<float, F16>(op, sb.H, blk, tile); break;
      case 1: stage_kt<__nv_bfloat16, F16>(op, sb.H, blk, tile); break;
      default: stage_kt<__half, F16>(op, sb.H, blk, tile); break;
    }
  } else {
    switch (op.src_dtype) {
      case 0: stage_rows<float, F16>(op, sb.H, blk); break;
      case 1: stage_rows<__nv_bfloat16, F16>(op, sb.H, blk); break;
      default: stage_rows<__half, F16>(op, sb.H, blk); break;
    }
  }
}

}  // namespace

cudaError_t launch_stage_batch(StageBatch sb, int dst_f16, cudaStream_t s) {
  long long blocks = 0;
  for (int i = 0; i < sb.n; ++i) {
    StageOp& op = sb.op[i];
    if (op.src_dtype < 0 || op.src_dtype > 2) return cudaErrorInvalidValue;
    op.kt = op.st.sd != 1 && op.st.sr == 1;
    op.rows = static_cast<long long>(sb.B) * sb.H * op.N;
    blocks += op.kt ? static_cast<long long>((op.N + 63) / 64) * sb.B * sb.H : (op.rows * 32 + 255) / 256;
    sb.end[i] = blocks;
  }
  if (sb.n <= 0 || blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return dst_f16 ? cudaLaunchKernelEx(&cfg, stage_kernel<true>, sb)
                 : cudaLaunchKernelEx(&cfg, stage_kernel<false>, sb);
}

}  // namespace ffai
