// Fused per-head QK-RMSNorm + rotary embedding + paged KV-cache write.
//
// Input is the packed QKV projection [T, (Hq + 2*Hkv) * D].  For every token:
//   q_h  <- rope(rmsnorm(q_h) * q_w)      -> q_out [T, Hq, D]
//   k_h  <- rope(rmsnorm(k_h) * k_w)      -> k_cache[block, h, off, :]
//   v_h                                   -> v_cache[block, h, :, off]
// with (block, off) = divmod(slot_mapping[t], block_size).  RoPE is the
// rotate-half (NeoX) form on the first `rot_dim` dimensions (rot_dim < D gives
// the partial rotary of Qwen3-Next attention).  Angles are computed on the fly
// from an fp32 inverse-frequency table, so no [max_pos, D] table is kept.
//
// Replaces rope / fused_split_rope / set_slice of the reference
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:331-349, 620-652, 688-710) and
// fixes its GQA overrun (pio/plugins/cpu/c_src/tensor_ops.c:384-415): K heads
// are iterated with their own count.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "launch.cuh"

namespace mb {

template <int D>
__global__ void rope_qknorm_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
                                   const __nv_bfloat16* __restrict__ kw, const int* __restrict__ pos,
                                   const float* __restrict__ inv_freq, const int* __restrict__ slots,
                                   __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                   __nv_bfloat16* __restrict__ v_cache, int Hq, int Hkv, int rot_dim, int block_size,
                                   float eps, int q_stride) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = D / 32;  // elements per lane
  __shared__ float buf[8][D];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = Hq + 2 * Hkv;
  const int p = pos[t];
  const int slot = slots ? slots[t] : -1;
  const __nv_bfloat16* row = qkv + (size_t)t * q_stride;
  for (int h = warp; h < nheads; h += blockDim.x / 32) {
    float v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = __bfloat162float(row[h * D + lane * E + e]);
    const bool is_q = h < Hq;
    const bool is_k = !is_q && h < Hq + Hkv;
    __nv_bfloat16* dst;
    int dstride = 1;  // element stride of the destination along D
    if (is_q) {
      dst = q_out + ((size_t)t * Hq + h) * D;
    } else {
      if (slot < 0) continue;
      const int hk = is_k ? h - Hq : h - Hq - Hkv;
      const size_t blk = slot / block_size, off = slot % block_size;
      if (is_k) {
        dst = k_cache + ((blk * Hkv + hk) * block_size + off) * D;
      } else {  // V is stored [blk, Hkv, D, block_size]
        dst = v_cache + ((blk * Hkv + hk) * D) * block_size + off;
        dstride = block_size;
      }
    }
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? qw : kw;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += v[e] * v[e];
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / D + eps);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          // round to bf16 like the unfused module chain (norm output is bf16)
          v[e] = __bfloat162float(__float2bfloat16(v[e] * inv * __bfloat162float(nw[lane * E + e])));
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) buf[warp][lane * E + e] = v[e];
      __syncwarp();
      const int half = rot_dim / 2;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int d = lane * E + e;
        if (d < rot_dim) {
          const int i = d < half ? d : d - half;
          float s, c;
          sincosf((float)p * inv_freq[i], &s, &c);
          const float other = d < half ? -buf[warp][d + half] : buf[warp][d - half];
          v[e] = v[e] * c + other * s;
        }
      }
      __syncwarp();
    }
#pragma unroll
    for (int e = 0; e < E; ++e) dst[(size_t)(lane * E + e) * dstride] = __float2bfloat16(v[e]);
  }
}

void rope_qknorm(const at::Tensor& qkv, const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                 const at::Tensor& positions, const at::Tensor& inv_freq, const c10::optional<at::Tensor>& slots,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                 int64_t rot_dim, double eps) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1);
  TORCH_CHECK(positions.scalar_type() == at::kInt && inv_freq.scalar_type() == at::kFloat);
  TORCH_CHECK(inv_freq.numel() >= rot_dim / 2 && rot_dim <= D && rot_dim % 2 == 0);
  const int T = (int)qkv.size(0);
  TORCH_CHECK(qkv.size(1) >= (Hq + 2 * Hkv) * D && positions.numel() == T);
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == T * Hq * D);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(1) == Hkv && k_cache.size(3) == D);
  TORCH_CHECK(v_cache.size(1) == Hkv && v_cache.size(2) == D && v_cache.size(3) == k_cache.size(2), "V cache must be [blocks, Hkv, D, block_size]");
  if (slots && slots->defined()) TORCH_CHECK(slots->scalar_type() == at::kInt && slots->numel() == T);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto bf = [](const c10::optional<at::Tensor>& o) -> const __nv_bfloat16* {
    return (o && o->defined()) ? reinterpret_cast<const __nv_bfloat16*>(o->data_ptr()) : nullptr;
  };
  const int* ps = (slots && slots->defined()) ? slots->data_ptr<int>() : nullptr;
  const int bs = (int)k_cache.size(2);
#define MB_ROPE(DD)                                                                                            \
  launch_k(rope_qknorm_kernel<DD>, T, 256, 0, st,                                                                    \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), bf(q_w), bf(k_w), positions.data_ptr<int>(),     \
      inv_freq.data_ptr<float>(), ps, reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),                      \
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), \
      (int)Hq, (int)Hkv, (int)rot_dim, bs, (float)eps, (int)qkv.stride(0))
  if (D == 128) MB_ROPE(128);
  else if (D == 256) MB_ROPE(256);
  else if (D == 64) MB_ROPE(64);
  else TORCH_CHECK(false, "rope_qknorm: unsupported head_dim ", D);
#undef MB_ROPE
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
