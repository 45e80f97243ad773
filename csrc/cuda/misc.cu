// Small memory-bound kernels: embedding gather, standalone SwiGLU, greedy
// argmax over the vocabulary and speculative-decoding prefix verification.
// Reference counterparts: embed_kernel, swiglu_kernel, argmax (undefined in
// the reference build) and verify_tokens_kernel
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:182-203, 496-513, 782-788).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "launch.cuh"

namespace mb {

// out[t] = table[ids[t] - vocab_start] if the id falls in this shard, else 0
// (vocab-parallel embedding: the shards are then summed/gathered).
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int H, int64_t vocab_start, int64_t vocab_rows) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int64_t id = ids[t] - vocab_start;
  const bool in = id >= 0 && id < vocab_rows;
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  const uint4* src = reinterpret_cast<const uint4*>(table + (in ? id : 0) * (size_t)H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = in ? src[i] : make_uint4(0, 0, 0, 0);
}

void embed(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t vocab_start) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && table.scalar_type() == at::kBFloat16 && table.is_contiguous());
  const int T = (int)ids.numel(), H = (int)table.size(1);
  TORCH_CHECK(H % 8 == 0 && out.is_contiguous() && out.numel() == (int64_t)T * H);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(table.device());
  launch_k(embed_kernel, T, 128, 0, at::cuda::getCurrentCUDAStream(), 
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H, vocab_start, table.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// gu [T, 2I] = [gate | up] -> out [T, I] = silu(gate) * up
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int I,
                              int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t t = i / I, c = i % I;
  const float g = __bfloat162float(gu[t * 2 * I + c]);
  const float u = __bfloat162float(gu[t * 2 * I + I + c]);
  out[i] = __float2bfloat16(silu(g) * u);
}

void swiglu(const at::Tensor& gu, at::Tensor& out) {
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.is_contiguous() && out.is_contiguous());
  const int I = (int)(gu.size(-1) / 2);
  const int64_t n = out.numel();
  TORCH_CHECK(n * 2 == gu.numel());
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(gu.device());
  launch_k(swiglu_kernel, (unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), I, n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Row argmax with the lowest index on ties; also writes the max value so a
// vocab-parallel caller can reduce (value, index) pairs across ranks.
__global__ void argmax_kernel(const __nv_bfloat16* __restrict__ logits, int V, int64_t* __restrict__ out_idx,
                              float* __restrict__ out_val, int64_t index_offset) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const __nv_bfloat16* row = logits + (size_t)r * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if ((V & 7) == 0) {
    for (int i = threadIdx.x * 8; i < V; i += blockDim.x * 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + i);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __bfloat162float(h[q]);
        if (v > bv) { bv = v; bi = i + q; }
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = __bfloat162float(row[i]);
      if (v > bv) { bv = v; bi = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      out_idx[r] = (int64_t)bi + index_offset;
      if (out_val) out_val[r] = bv;
    }
  }
}

void argmax(const at::Tensor& logits, at::Tensor& out_idx, const c10::optional<at::Tensor>& out_val,
            int64_t index_offset) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous() && out_idx.scalar_type() == at::kLong);
  const int R = (int)logits.size(0), V = (int)logits.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  float* pv = (out_val && out_val->defined()) ? out_val->data_ptr<float>() : nullptr;
  launch_k(argmax_kernel, R, 1024, 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), V, out_idx.data_ptr<int64_t>(), pv, index_offset);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Speculative decoding: number of leading draft tokens that match the target
// model's tokens, per row.  draft/target [R, L] int64 -> out [R] int32.
__global__ void verify_tokens_kernel(const int64_t* __restrict__ draft, const int64_t* __restrict__ target, int L,
                                     int* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  int first_bad = L;
  for (int i = threadIdx.x; i < L; i += blockDim.x)
    if (draft[(size_t)r * L + i] != target[(size_t)r * L + i]) first_bad = min(first_bad, i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first_bad = min(first_bad, __shfl_xor_sync(0xffffffffu, first_bad, o));
  if (threadIdx.x == 0) out[r] = first_bad;
}

void verify_tokens(const at::Tensor& draft, const at::Tensor& target, at::Tensor& out) {
  TORCH_CHECK(draft.scalar_type() == at::kLong && target.scalar_type() == at::kLong && draft.sizes() == target.sizes());
  TORCH_CHECK(draft.is_contiguous() && target.is_contiguous() && out.scalar_type() == at::kInt);
  const int R = (int)draft.size(0), L = (int)draft.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(draft.device());
  launch_k(verify_tokens_kernel, R, 32, 0, at::cuda::getCurrentCUDAStream(), draft.data_ptr<int64_t>(),
                                                                        target.data_ptr<int64_t>(), L,
                                                                        out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb

namespace mb {

// Advances n live decode rows by one token on the device, so consecutive
// replays of a captured decode step run at a growing context without host
// work: ids[b] = sampled[b]; pos[b] += 1; ctx[b] += 1; slots[b] = the KV slot
// of the new position in row b of the block table (-1 past the row's end).
__global__ void decode_advance_kernel(const int64_t* __restrict__ sampled, int64_t* __restrict__ ids,
                                      int* __restrict__ pos, int* __restrict__ ctx, int* __restrict__ slots,
                                      const int* __restrict__ bt, int n, int max_blocks, int block_size) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  ids[b] = sampled[b];
  const int p = pos[b] + 1;
  pos[b] = p;
  ctx[b] = ctx[b] + 1;
  const int blk = p / block_size;
  slots[b] = blk < max_blocks ? bt[(size_t)b * max_blocks + blk] * block_size + p % block_size : -1;
}

void decode_advance(const at::Tensor& sampled, at::Tensor& ids, at::Tensor& pos, at::Tensor& ctx, at::Tensor& slots,
                    const at::Tensor& bt, int64_t n, int64_t block_size) {
  TORCH_CHECK(sampled.scalar_type() == at::kLong && ids.scalar_type() == at::kLong);
  TORCH_CHECK(pos.scalar_type() == at::kInt && ctx.scalar_type() == at::kInt && slots.scalar_type() == at::kInt &&
              bt.scalar_type() == at::kInt && bt.dim() == 2 && bt.is_contiguous());
  TORCH_CHECK(n <= sampled.numel() && n <= ids.numel() && n <= pos.numel() && n <= ctx.numel() &&
              n <= slots.numel() && n <= bt.size(0));
  if (n <= 0) return;
  c10::cuda::CUDAGuard guard(ids.device());
  launch_k(decode_advance_kernel, (unsigned)((n + 127) / 128), 128, 0, at::cuda::getCurrentCUDAStream(),
           (const int64_t*)sampled.data_ptr<int64_t>(), ids.data_ptr<int64_t>(), pos.data_ptr<int>(),
           ctx.data_ptr<int>(), slots.data_ptr<int>(), (const int*)bt.data_ptr<int>(), (int)n, (int)bt.size(1),
           (int)block_size);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
