// C++17 + OpenMP CPU backend (fp32).  Same operator set as the GPU path, used
// as the plumbing / host reference path and for the CPU benchmark config.
// Replaces the reference's C CPU library (pio/plugins/cpu/c_src/tensor_ops.c)
// with correct GQA, causal attention, QK-norm and gated DeltaNet.
#pragma once
#include <torch/extension.h>

namespace mbcpu {
void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y);
void linear_w8(const at::Tensor& x, const at::Tensor& q, const at::Tensor& scale, at::Tensor& y);
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& out,
             double eps);
void rope_qknorm(const at::Tensor& qkv, const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                 const at::Tensor& positions, const at::Tensor& inv_freq, const c10::optional<at::Tensor>& slots,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                 int64_t rot_dim, double eps);
void attn_paged(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                const at::Tensor& block_tables, const at::Tensor& ctx_lens, const at::Tensor& q_lens,
                at::Tensor& out, double scale);
void swiglu(const at::Tensor& gu, at::Tensor& out);
void gelu_tanh(const at::Tensor& x, at::Tensor& out);
void embed(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out);
at::Tensor argmax(const at::Tensor& logits);
void moe_route(const at::Tensor& logits, int64_t k, bool renorm, at::Tensor& ids, at::Tensor& wts);
void moe_experts(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& wts, const at::Tensor& w13,
                 const at::Tensor& w2, int64_t e_lo, int64_t num_local, at::Tensor& out);
void deltanet_recurrence(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                         const at::Tensor& beta, at::Tensor& state, at::Tensor& out);
void conv1d_causal(const at::Tensor& x, const at::Tensor& w, at::Tensor& state, at::Tensor& out);
void resize_bilinear(const at::Tensor& img, at::Tensor& out);
}  // namespace mbcpu
