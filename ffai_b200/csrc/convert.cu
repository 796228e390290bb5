// Operand preparation for the tensor-core prefill: gather an f32/bf16/f16
// operand of any supported layout into a contiguous heads-split (B,H,N,64)
// 16-bit (bf16 or f16) buffer.  Used for the reference's f32 operands (its callers hold f32
// candle tensors, flash_attn.rs:212-217) and for K^T (B,H,64,N) whose row
// pitch is not a multiple of 16 bytes and so cannot be described to TMA.
#include "common.cuh"
#include "kernels.h"

namespace ffai {

namespace {

template <bool F16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  return F16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

template <typename T, bool F16>
__global__ void to_16bit_rows_kernel(const T* __restrict__ src, Strides st, int H, int N,
                                     uint16_t* __restrict__ dst, long long total_rows) {
  // One warp per destination row (64 elements, two per lane).
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= total_rows) return;
  const int n = static_cast<int>(row % N);
  const long long bh = row / N;
  const int h = static_cast<int>(bh % H);
  const long long b = bh / H;
  const T* s = src + b * st.sb + h * st.sh + n * st.sr;
  const float x0 = to_f32(s[(2 * lane) * st.sd]);
  const float x1 = to_f32(s[(2 * lane + 1) * st.sd]);
  reinterpret_cast<uint32_t*>(dst + row * 64)[lane] = pack16<F16>(x0, x1);
}

// Head-dim-major source (sd != 1, sr == 1): transpose 64x64 tiles through
// shared memory so both the reads (along keys) and writes (along dims) coalesce.
template <typename T, bool F16>
__global__ void kt_to_16bit_rows_kernel(const T* __restrict__ src, Strides st, int H, int N,
                                        uint16_t* __restrict__ dst) {
  __shared__ float tile[64][65];
  const int bh = blockIdx.y;
  const int h = bh % H;
  const long long b = bh / H;
  const int n0 = blockIdx.x * 64;
  const T* s = src + b * st.sb + h * st.sh;
  for (int idx = threadIdx.x; idx < 64 * 64; idx += blockDim.x) {
    const int d = idx / 64, j = idx % 64;
    const int n = n0 + j;
    tile[d][j] = n < N ? to_f32(s[static_cast<long long>(n) * st.sr + d * st.sd]) : 0.f;
  }
  __syncthreads();
  uint16_t* o = dst + (static_cast<long long>(bh) * N) * 64;
  for (int idx = threadIdx.x; idx < 64 * 32; idx += blockDim.x) {
    const int j = idx / 32, dp = idx % 32;
    const int n = n0 + j;
    if (n < N)
      reinterpret_cast<uint32_t*>(o + static_cast<long long>(n) * 64)[dp] =
          pack16<F16>(tile[2 * dp][j], tile[2 * dp + 1][j]);
  }
}

template <typename T, bool F16>
cudaError_t launch_typed(const void* src, Strides st, int B, int H, int N, void* dst,
                         cudaStream_t s) {
  const T* sp = static_cast<const T*>(src);
  uint16_t* dp = static_cast<uint16_t*>(dst);
  if (st.sd != 1 && st.sr == 1) {
    dim3 grid((N + 63) / 64, B * H);
    kt_to_16bit_rows_kernel<T, F16><<<grid, 256, 0, s>>>(sp, st, H, N, dp);
  } else {
    const long long rows = static_cast<long long>(B) * H * N;
    const long long blocks = (rows * 32 + 255) / 256;
    to_16bit_rows_kernel<T, F16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(sp, st, H, N, dp,
                                                                              rows);
  }
  return cudaGetLastError();
}

template <bool F16>
cudaError_t launch_dst(const void* src, int src_dtype, Strides st, int B, int H, int N, void* dst,
                       cudaStream_t s) {
  switch (src_dtype) {
    case 0:
      return launch_typed<float, F16>(src, st, B, H, N, dst, s);
    case 1:
      return launch_typed<__nv_bfloat16, F16>(src, st, B, H, N, dst, s);
    case 2:
      return launch_typed<__half, F16>(src, st, B, H, N, dst, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_to_16bit_heads_split(const void* src, int src_dtype, Strides st, int B, int H,
                                        int N, void* dst, int dst_f16, cudaStream_t s) {
  if (B <= 0 || H <= 0 || N <= 0) return cudaSuccess;
  return dst_f16 ? launch_dst<true>(src, src_dtype, st, B, H, N, dst, s)
                 : launch_dst<false>(src, src_dtype, st, B, H, N, dst, s);
}

}  // namespace ffai
