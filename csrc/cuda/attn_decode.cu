// Paged decode attention with GQA packing and split-KV.
//
// q        [B, Hq, D]           one query token per sequence
// k cache  [num_blocks, Hkv, BS, D], v cache [num_blocks, Hkv, D, BS], BS = 16
// block_tables [B, max_blocks] int32, context_lens [B] int32
// out      [B, Hq, D]
//
// One CTA per (sequence, KV head, split).  All G = Hq/Hkv query heads that
// share a KV head are processed together, so every K/V byte is read from HBM
// once per sequence.  Each warp takes one 16-token KV block per iteration:
// for Q.K lane l owns token l%16 and half (l/16) of the head dimension; for
// P.V lane l owns D/32 output dimensions.  Online softmax (base-2) per head.
// With more than one split, each split writes an fp32 partial + log-sum-exp
// and a second kernel merges them.
//
// Replaces fused_attention / paged_attention of the reference
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:529-618,
//  pio/plugins/common/c_src/tensor_ops_opencl.c:526-565).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "attn_decode.cuh"
#include "launch.cuh"

namespace mb {

// workspace: fp32, at least B*Hq*splits*(D+1) elements when splits > 1.
void attn_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                 const at::Tensor& block_tables, const at::Tensor& ctx_lens, at::Tensor& out, int64_t splits,
                 const c10::optional<at::Tensor>& workspace, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(2) == 16);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt);
  TORCH_CHECK(block_tables.is_contiguous());
  const int B = (int)q.size(0), Hq = (int)q.size(1), D = (int)q.size(2);
  const int Hkv = (int)k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0 && k_cache.size(3) == D);
  const int G = Hq / Hkv;
  if (B == 0) return;
  splits = std::max<int64_t>(1, splits);
  float* po = nullptr;
  float* pl = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace && workspace->defined() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)B * Hq * splits * (D + 1),
                "attn_decode: split-KV needs an fp32 workspace of B*Hq*splits*(D+1)");
    po = workspace->data_ptr<float>();
    pl = po + (size_t)B * Hq * splits * D;
  }
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);
  dim3 grid(B, Hkv, (unsigned)splits);
  auto pq = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  auto pk = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  auto pv = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  auto pout = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const int mbk = (int)block_tables.size(1);
#define MB_ATT(DD, GG)                                                                                         \
  if (D == DD && G == GG) {                                                                                    \
    launch_k(attn_decode_kernel<DD, GG>, grid, kWarps * 32, 0, st, pq, pk, pv, block_tables.data_ptr<int>(),         \
                                                            ctx_lens.data_ptr<int>(), pout, po, pl, Hkv, mbk,  \
                                                            (int)splits, sl2);                                 \
    launched = true;                                                                                           \
  }
  bool launched = false;
  MB_ATT(128, 1) MB_ATT(128, 2) MB_ATT(128, 4) MB_ATT(128, 8) MB_ATT(128, 16)
  MB_ATT(256, 1) MB_ATT(256, 2) MB_ATT(256, 4) MB_ATT(256, 8)
  MB_ATT(64, 1) MB_ATT(64, 2) MB_ATT(64, 4) MB_ATT(64, 8)
#undef MB_ATT
  TORCH_CHECK(launched, "attn_decode: unsupported head_dim/group ", D, "/", G);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (splits > 1) {
    if (D == 128) launch_k(attn_combine_kernel<128>, B * Hq, 128, 0, st, po, pl, pout, (int)splits);
    else if (D == 256) launch_k(attn_combine_kernel<256>, B * Hq, 128, 0, st, po, pl, pout, (int)splits);
    else launch_k(attn_combine_kernel<64>, B * Hq, 64, 0, st, po, pl, pout, (int)splits);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace mb
