// RMSNorm and residual-add + RMSNorm, bf16 in/out, fp32 accumulation.
// One warp per row, 16-byte vector loads; the row is kept in registers between
// the sum-of-squares pass and the scaling pass, so each element is read once.
// Replaces rms_norm / fused_add_rms_norm of the reference
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:205-241,
//  pio/plugins/cpu/c_src/tensor_ops.c:369-383) which used one thread per row.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "launch.cuh"

namespace mb {

// H is a compile-time multiple of 256 (8 bf16 per lane per chunk).
template <int H, bool ADD>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int rows,
                               float eps) {
  pdl_wait();
  pdl_trigger();
  constexpr int kChunks = H / 256;
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[kChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 256 + lane * 8;
    uint4 raw = *reinterpret_cast<const uint4*>(x + (size_t)row * H + col);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[c][q] = __bfloat162float(h[q]);
    if (ADD) {
      uint4 rr = *reinterpret_cast<const uint4*>(residual + (size_t)row * H + col);
      const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(&rr);
      __align__(16) __nv_bfloat16 s[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[c][q] += __bfloat162float(r[q]);
        s[q] = __float2bfloat16(v[c][q]);
        v[c][q] = __bfloat162float(s[q]);  // the stored residual is what later layers see
      }
      *reinterpret_cast<uint4*>(residual + (size_t)row * H + col) = *reinterpret_cast<uint4*>(s);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += v[c][q] * v[c][q];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / H + eps);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 256 + lane * 8;
    uint4 wr = *reinterpret_cast<const uint4*>(w + col);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wr);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16(v[c][q] * inv * __bfloat162float(wh[q]));
    *reinterpret_cast<uint4*>(out + (size_t)row * H + col) = *reinterpret_cast<uint4*>(o);
  }
}

// Generic fallback for hidden sizes that are not a multiple of 256.
template <bool ADD>
__global__ void rmsnorm_generic_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                                       const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H,
                                       float eps) {
  pdl_wait();
  pdl_trigger();
  const size_t row = blockIdx.x;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = __bfloat162float(x[row * H + i]);
    if (ADD) {
      v += __bfloat162float(residual[row * H + i]);
      __nv_bfloat16 s = __float2bfloat16(v);
      residual[row * H + i] = s;
      v = __bfloat162float(s);
    }
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = ADD ? __bfloat162float(residual[row * H + i]) : __bfloat162float(x[row * H + i]);
    out[row * H + i] = __float2bfloat16(v * inv * __bfloat162float(w[i]));
  }
}

// out = rmsnorm(x) * w ; if residual is given: residual += x first and the
// norm is taken of the updated residual (x is left untouched).
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& out,
             double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous());
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(w.numel() == H && out.numel() == x.numel());
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const bool add = residual && residual->defined();
  __nv_bfloat16* r = nullptr;
  if (add) {
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == x.numel());
    r = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
  }
  auto px = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto pw = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto po = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const int wpb = 8;
  dim3 grid((rows + wpb - 1) / wpb), block(32 * wpb);
#define MB_RMS(HH)                                                                       \
  case HH:                                                                               \
    if (add) launch_k(rmsnorm_kernel<HH, true>, grid, block, 0, st, px, r, pw, po, rows, eps); \
    else launch_k(rmsnorm_kernel<HH, false>, grid, block, 0, st, px, r, pw, po, rows, eps);    \
    break;
  switch (H) {
    MB_RMS(256) MB_RMS(512) MB_RMS(768) MB_RMS(1024) MB_RMS(1536) MB_RMS(2048) MB_RMS(3072) MB_RMS(4096)
   
    default:
      if (add) launch_k(rmsnorm_generic_kernel<true>, rows, 256, 0, st, px, r, pw, po, H, eps);
      else launch_k(rmsnorm_generic_kernel<false>, rows, 256, 0, st, px, r, pw, po, H, eps);
  }
#undef MB_RMS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
