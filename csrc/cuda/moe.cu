// Mixture-of-experts routing on the device, with no host synchronisation:
//   1. moe_topk      : softmax over expert logits, top-k, optional renormalise;
//                      histogram of expert loads (atomic counts).
//   2. moe_scan      : exclusive scan of the counts -> group offsets [E+1].
//   3. moe_permute   : each (token, k) pair claims a row of its expert's
//                      segment and copies the token's hidden row there.
//   4. grouped GEMMs (gemm.cu) over the permuted rows.
//   5. moe_combine   : out[t] = residual[t] + sum_k w[t,k] * y[pos[t,k]], in a
//                      fixed k order (deterministic, no float atomics).
// The reference runs this as a Python loop over top-k slots with a
// device->host copy per slot (pio/models/qwen3_coder_30b/model.py:308-353)
// and count_value / gather_by_value / scatter_add_by_index kernels
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:384-418).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "status.h"
#include "launch.cuh"

namespace mb {

// One warp per token.  E <= 1024, K <= 16.
template <int EPL>  // experts per lane
__global__ void moe_topk_kernel(const __nv_bfloat16* __restrict__ logits, int T, int E, int K, bool renorm,
                                int* __restrict__ ids, float* __restrict__ wts, int* __restrict__ counts,
                                int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? __bfloat162float(logits[(size_t)t * E + e]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? __expf(v[i] - mx) : -1.f;  // probabilities; -1 marks padding
    sum += e < E ? v[i] : 0.f;
  }
  sum = warp_sum(sum);
  float picked_sum = 0.f;
  float my_w = 0.f;
  int my_id = -1;
  for (int k = 0; k < K; ++k) {
    // arg-max over (value, lowest index on ties)
    float bv = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (v[i] > bv) { bv = v[i]; bi = i * 32 + lane; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == k) { my_w = bv / sum; my_id = bi; }
    picked_sum += bv / sum;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i * 32 + lane == bi) v[i] = -2.f;
  }
  if (lane < K) {
    // non-finite logits select nothing: never index with an invalid id
    if (my_id < 0 || my_id >= E) {
      set_status(status, kErrBounds);
      my_id = 0;
      my_w = 0.f;
    }
    ids[(size_t)t * K + lane] = my_id;
    wts[(size_t)t * K + lane] = renorm ? my_w / picked_sum : my_w;
    atomicAdd(&counts[my_id], 1);
  }
}

// Single CTA: offs[0]=0, offs[e+1]=offs[e]+counts[e]; resets cursors.
__global__ void moe_scan_kernel(const int* __restrict__ counts, int E, int* __restrict__ offs,
                                int* __restrict__ cursor) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s[1024];
  const int i = threadIdx.x;
  s[i] = i < E ? counts[i] : 0;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    int x = i >= o ? s[i - o] : 0;
    __syncthreads();
    s[i] += x;
    __syncthreads();
  }
  if (i < E) {
    offs[i + 1] = s[i];
    cursor[i] = 0;
  }
  if (i == 0) offs[0] = 0;
}

// One warp per (token, k) pair: claim a row and copy the hidden vector.
__global__ void moe_permute_kernel(const __nv_bfloat16* __restrict__ x, int T, int K, int H,
                                   const int* __restrict__ ids, const int* __restrict__ offs,
                                   int* __restrict__ cursor, int* __restrict__ pos, __nv_bfloat16* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int pair = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (pair >= T * K) return;
  int p = 0;
  if (lane == 0) {
    const int e = ids[pair];  // always in [0, E): moe_topk clamps invalid selections
    p = offs[e] + atomicAdd(&cursor[e], 1);
    pos[pair] = p;
  }
  p = __shfl_sync(0xffffffffu, p, 0);
  const int t = pair / K;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)p * H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

// One CTA per token.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos,
                                   const float* __restrict__ wts, int K, int H,
                                   const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int k = 0; k < K; ++k) {
      const int p = pos[(size_t)t * K + k];
      const float w = wts[(size_t)t * K + k];
      uint4 raw = *reinterpret_cast<const uint4*>(y + (size_t)p * H + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += w * __bfloat162float(h[q]);
    }
    if (residual) {
      uint4 raw = *reinterpret_cast<const uint4*>(residual + (size_t)t * H + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(h[q]);
    }
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16(acc[q]);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = *reinterpret_cast<uint4*>(o);
  }
}

// Routing: logits [T, E] bf16 -> ids [T,K] int32, wts [T,K] f32,
// counts [E] int32 (zeroed here), offs [E+1] int32, cursor [E] int32.
void moe_route(const at::Tensor& logits, int64_t K, bool renorm, at::Tensor& ids, at::Tensor& wts,
               at::Tensor& counts, at::Tensor& offs, at::Tensor& cursor) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous());
  const int T = (int)logits.size(0), E = (int)logits.size(1);
  TORCH_CHECK(E <= 1024 && K <= 32 && K <= E);
  c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(counts.data_ptr(), 0, E * sizeof(int), st));
  if (T > 0) {
    const int wpb = 8;
    dim3 grid((T + wpb - 1) / wpb), block(wpb * 32);
    auto pl = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
    const int epl = (E + 31) / 32;
#define MB_TOPK(N) \
  launch_k(moe_topk_kernel<N>, grid, block, 0, st, pl, T, E, (int)K, renorm, ids.data_ptr<int>(), wts.data_ptr<float>(), \
                                             counts.data_ptr<int>(), status_ptr(logits.device().index()))
    if (epl <= 1) MB_TOPK(1);
    else if (epl <= 2) MB_TOPK(2);
    else if (epl <= 4) MB_TOPK(4);
    else if (epl <= 8) MB_TOPK(8);
    else if (epl <= 16) MB_TOPK(16);
    else MB_TOPK(32);
#undef MB_TOPK
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  launch_k(moe_scan_kernel, 1, 1024, 0, st, counts.data_ptr<int>(), E, offs.data_ptr<int>(), cursor.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_permute(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& offs, at::Tensor& cursor,
                 at::Tensor& pos, at::Tensor& xs) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && xs.is_contiguous());
  const int T = (int)x.size(0), H = (int)x.size(1), K = (int)ids.size(1);
  TORCH_CHECK(H % 8 == 0 && xs.size(0) >= (int64_t)T * K);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int wpb = 8;
  launch_k(moe_permute_kernel, (T * K + wpb - 1) / wpb, wpb * 32, 0, st, 
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), T, K, H, ids.data_ptr<int>(), offs.data_ptr<int>(),
      cursor.data_ptr<int>(), pos.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(xs.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(const at::Tensor& y, const at::Tensor& pos, const at::Tensor& wts,
                 const c10::optional<at::Tensor>& residual, at::Tensor& out) {
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && out.is_contiguous());
  const int T = (int)out.size(0), H = (int)out.size(1), K = (int)pos.size(1);
  TORCH_CHECK(H % 8 == 0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(y.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* r = (residual && residual->defined())
                               ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr())
                               : nullptr;
  const int threads = std::min(256, std::max(32, H / 8));
  launch_k(moe_combine_kernel, T, threads, 0, st, reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
                                            pos.data_ptr<int>(), wts.data_ptr<float>(), K, H, r,
                                            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
