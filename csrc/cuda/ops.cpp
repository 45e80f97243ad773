// Python bindings of the sm_100a kernels (module mod_b200._C).
#include <torch/extension.h>
#include "status.h"

namespace mb {
void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& residual,
            const c10::optional<at::Tensor>& workspace, int64_t splits, int64_t orient);
void swiglu_linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& workspace,
                   int64_t wait_flags, const c10::optional<at::Tensor>& state, int64_t nranks);
void grouped_linear(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y, int64_t groups,
                    bool swiglu, int64_t max_rows_per_group);
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& out,
             double eps);
void rope_qknorm(const at::Tensor& qkv, const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                 const at::Tensor& positions, const at::Tensor& inv_freq, const c10::optional<at::Tensor>& slots,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                 int64_t rot_dim, double eps);
void attn_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                 const at::Tensor& block_tables, const at::Tensor& ctx_lens, at::Tensor& out, int64_t splits,
                 const c10::optional<at::Tensor>& workspace, double scale);
void deltanet_decode(const at::Tensor& mixed, const at::Tensor& z, const at::Tensor& ba, const at::Tensor& conv_w,
                     at::Tensor& conv_state, at::Tensor& ssm, const at::Tensor& slots, const at::Tensor& A_log,
                     const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor& out, int64_t Hk, int64_t Hv,
                     int64_t dk, int64_t dv, double eps);
void deltanet_prefill(const at::Tensor& mixed, const at::Tensor& z, const at::Tensor& ba, const at::Tensor& conv_w,
                      at::Tensor& conv_state, at::Tensor& ssm, const at::Tensor& slots, const at::Tensor& cu,
                      const at::Tensor& seq_of, const at::Tensor& A_log, const at::Tensor& dt_bias,
                      const at::Tensor& norm_w, at::Tensor& out, at::Tensor& xc, int64_t Hk, int64_t Hv, int64_t dk,
                      int64_t dv, double eps);
void linear_w8(const at::Tensor& x, const at::Tensor& wq, const at::Tensor& scale, at::Tensor& y,
               const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& workspace,
               const c10::optional<at::Tensor>& offs, int64_t groups, bool swiglu, int64_t max_rows_per_group);
void sample_tokens(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                   const at::Tensor& top_p, const at::Tensor& seeds, const at::Tensor& steps, at::Tensor& out);
void patchify(const at::Tensor& images, int64_t size, int64_t patch, int64_t merge, std::vector<double> mean,
              std::vector<double> stdv, at::Tensor& out);
void bias_act(at::Tensor& y, const c10::optional<at::Tensor>& bias, bool gelu);
void ep_dispatch2(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                  const at::Tensor& x, const at::Tensor& ids, const at::Tensor& counts, const at::Tensor& offs_g,
                  at::Tensor& cursor, at::Tensor& map, at::Tensor& offs);
int64_t ep_flag_addr(const at::Tensor& peers, int64_t rank, int64_t C, int64_t H);
int64_t ep_recv_addr(const at::Tensor& peers, int64_t rank, int64_t C, int64_t H);
void ep_combine2(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                 const at::Tensor& offs, const at::Tensor& y, const at::Tensor& map, const at::Tensor& wts,
                 const c10::optional<at::Tensor>& residual, at::Tensor& out);
void grouped_linear_wait(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y,
                         int64_t groups, bool swiglu, int64_t max_rows_per_group, int64_t flags, at::Tensor& state,
                         int64_t nranks, int64_t epoch_add);
void vis_scatter_gemm(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                      const at::Tensor& row_map, const at::Tensor& peers, int64_t rank, int64_t peer_rows,
                      int64_t off, int64_t flag_off, at::Tensor& state);
void vis_release(const at::Tensor& peers, int64_t rank, int64_t flag_off, at::Tensor& state);
void vis_wait_merge(const at::Tensor& peers, int64_t rank, int64_t off, int64_t flag_off, at::Tensor& state,
                    const at::Tensor& rows, at::Tensor& h);
void attn_decode_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                    const at::Tensor& block_tables, const at::Tensor& ctx_lens, at::Tensor& out, int64_t splits,
                    const c10::optional<at::Tensor>& workspace, double scale, at::Tensor& work);
bool attn_decode_tc_supported(int64_t D, int64_t G);
void attn_prefill_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                     const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens,
                     at::Tensor& out, int64_t max_q_len, double scale, bool causal);
void moe_route(const at::Tensor& logits, int64_t K, bool renorm, at::Tensor& ids, at::Tensor& wts,
               at::Tensor& counts, at::Tensor& offs, at::Tensor& cursor);
void moe_permute(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& offs, at::Tensor& cursor,
                 at::Tensor& pos, at::Tensor& xs);
void moe_combine(const at::Tensor& y, const at::Tensor& pos, const at::Tensor& wts,
                 const c10::optional<at::Tensor>& residual, at::Tensor& out);
int64_t ep_buffer_bytes(int64_t N, int64_t C, int64_t H);
void ep_dispatch(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                 const at::Tensor& x, const at::Tensor& ids, at::Tensor& map, at::Tensor& row_pos, at::Tensor& offs,
                 at::Tensor& xs, at::Tensor& abort);
void ep_combine(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                const at::Tensor& row_pos, const at::Tensor& y, const at::Tensor& map, const at::Tensor& wts,
                const c10::optional<at::Tensor>& residual, at::Tensor& out);
void ep_recv_only(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El, int64_t H,
                  at::Tensor& row_pos, at::Tensor& offs, at::Tensor& abort);
void tp_gemm(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, bool wait, bool scatter, bool swiglu,
             int64_t ag_flags, at::Tensor& state, int64_t rank, int64_t nranks, int64_t peer_rows,
             const at::Tensor& rs_peers, int64_t rs_off, int64_t rs_flag_off, const c10::optional<at::Tensor>& workspace);
at::Tensor wrap_bf16(int64_t addr, int64_t rows, int64_t cols);
void tp_reduce(const at::Tensor& peers, int64_t rank, bool with_partials, int64_t rows, int64_t H, int64_t ag_off,
               int64_t rs_off, int64_t ag_flag_off, int64_t rs_flag_off, at::Tensor& state,
               const c10::optional<at::Tensor>& x_add, at::Tensor& residual, const at::Tensor& w, double eps,
               const c10::optional<at::Tensor>& local_out);
void tp_argmax_exchange(const at::Tensor& peers, int64_t rank, int64_t cap, int64_t slot_off, int64_t flag_off,
                        at::Tensor& state, const at::Tensor& vals, const at::Tensor& idxs, at::Tensor& out);
void tp_nvls_reduce(int64_t self, int64_t mc, int64_t rank, int64_t nranks, bool with_partials, int64_t rows,
                    int64_t row_stride, bool publish, int64_t H, int64_t ag_off, int64_t part_off, int64_t ag_flag_off, int64_t rs_flag_off,
                    at::Tensor& state, const c10::optional<at::Tensor>& x_add, at::Tensor& residual,
                    const at::Tensor& w, double eps, const c10::optional<at::Tensor>& local_out);
bool multicast_supported(int64_t device);
void ep_agrs_publish(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                     const at::Tensor& offsets, at::Tensor& state, const at::Tensor& x, const at::Tensor& logits,
                     bool renorm);
void ep_agrs_place(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                   int64_t H, const at::Tensor& offsets, at::Tensor& state, at::Tensor& xs, at::Tensor& slot_of,
                   at::Tensor& offs, int64_t grid);
void ep_agrs_combine(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                     int64_t H, const at::Tensor& offsets, at::Tensor& state, const at::Tensor& slot_of,
                     const at::Tensor& y);
void tp_gather_rows(const at::Tensor& peers, int64_t rank, int64_t peer_rows, int64_t ag_off, int64_t ag_flag_off,
                    at::Tensor& state, const at::Tensor& idx, at::Tensor& out);
std::tuple<int64_t, std::string> ipc_alloc(int64_t bytes);
int64_t ipc_open(const std::string& handle);
void ipc_close(int64_t ptr);
void ipc_free(int64_t ptr);
void ep_route_dispatch(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                       const at::Tensor& x, const at::Tensor& wr, int64_t K, bool renorm, at::Tensor& ids,
                       at::Tensor& wts, at::Tensor& map, at::Tensor& offs, at::Tensor& scratch, at::Tensor& logits,
                       const c10::optional<at::Tensor>& pos_map, const c10::optional<at::Tensor>& trace);
void ep_combine_send(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                     const at::Tensor& offs, const at::Tensor& y, int64_t H);
void ep_combine_norm(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                     const at::Tensor& map, const at::Tensor& wts, at::Tensor& residual, const at::Tensor& w,
                     at::Tensor& out, double eps, const c10::optional<at::Tensor>& rows);
void linear_cluster(const at::Tensor& x, const at::Tensor& w, at::Tensor& y,
                    const c10::optional<at::Tensor>& residual, int64_t cs, int64_t ag_flags,
                    const c10::optional<at::Tensor>& state, int64_t nranks);
void swiglu_cluster(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, int64_t cs, int64_t ag_flags,
                    const c10::optional<at::Tensor>& state, int64_t nranks);
void linear_cluster_w8(const at::Tensor& x, const at::Tensor& wq, const at::Tensor& scale, at::Tensor& y,
                       const c10::optional<at::Tensor>& residual, int64_t cs);
void qkv_rope_cluster(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& q_w,
                      const c10::optional<at::Tensor>& k_w, const at::Tensor& positions, const at::Tensor& inv_freq,
                      const c10::optional<at::Tensor>& slots, at::Tensor& q_out, at::Tensor& k_cache,
                      at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t rot_dim, double eps, int64_t cs,
                      int64_t ag_flags, const c10::optional<at::Tensor>& state, int64_t nranks);
void vit_rope_kv(const at::Tensor& qkv, const at::Tensor& pos, int64_t N, int64_t heads, int64_t D, double theta,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache);
void decode_advance(const at::Tensor& sampled, at::Tensor& ids, at::Tensor& pos, at::Tensor& ctx, at::Tensor& slots,
                    const at::Tensor& bt, int64_t n, int64_t block_size);
void embed(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t vocab_start);
void swiglu(const at::Tensor& gu, at::Tensor& out);
void argmax(const at::Tensor& logits, at::Tensor& out_idx, const c10::optional<at::Tensor>& out_val,
            int64_t index_offset);
void verify_tokens(const at::Tensor& draft, const at::Tensor& target, at::Tensor& out);
}  // namespace mb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mod_b200 sm_100a kernels";
  m.def("linear", &mb::linear);
  m.def("linear_cluster", &mb::linear_cluster);
  m.def("swiglu_cluster", &mb::swiglu_cluster);
  m.def("qkv_rope_cluster", &mb::qkv_rope_cluster);
  m.def("linear_cluster_w8", &mb::linear_cluster_w8);
  m.def("grouped_linear", &mb::grouped_linear);
  m.def("swiglu_linear", &mb::swiglu_linear);
  m.def("rmsnorm", &mb::rmsnorm);
  m.def("rope_qknorm", &mb::rope_qknorm);
  m.def("attn_decode", &mb::attn_decode);
  m.def("attn_decode_tc", &mb::attn_decode_tc);
  m.def("deltanet_decode", &mb::deltanet_decode);
  m.def("linear_w8", &mb::linear_w8);
  m.def("sample_tokens", &mb::sample_tokens);
  m.def("patchify", &mb::patchify);
  m.def("vit_rope_kv", &mb::vit_rope_kv);
  m.def("bias_act", &mb::bias_act);
  m.def("deltanet_prefill", &mb::deltanet_prefill);
  m.def("attn_decode_tc_supported", &mb::attn_decode_tc_supported);
  m.def("attn_prefill_tc", &mb::attn_prefill_tc);
  m.def("moe_route", &mb::moe_route);
  m.def("moe_permute", &mb::moe_permute);
  m.def("moe_combine", &mb::moe_combine);
  m.def("ep_buffer_bytes", &mb::ep_buffer_bytes);
  m.def("ep_dispatch", &mb::ep_dispatch);
  m.def("ep_dispatch2", &mb::ep_dispatch2);
  m.def("ep_route_dispatch", &mb::ep_route_dispatch);
  m.def("ep_combine_send", &mb::ep_combine_send);
  m.def("ep_combine_norm", &mb::ep_combine_norm);
  m.def("vis_scatter_gemm", &mb::vis_scatter_gemm);
  m.def("vis_release", &mb::vis_release);
  m.def("vis_wait_merge", &mb::vis_wait_merge);
  m.def("grouped_linear_wait", &mb::grouped_linear_wait);
  m.def("ep_combine2", &mb::ep_combine2);
  m.def("ep_flag_addr", &mb::ep_flag_addr);
  m.def("ep_recv_addr", &mb::ep_recv_addr);
  m.def("ep_combine", &mb::ep_combine);
  m.def("ep_recv_only", &mb::ep_recv_only);
  m.def("tp_gemm", &mb::tp_gemm);
  m.def("wrap_bf16", &mb::wrap_bf16);
  m.def("tp_reduce", &mb::tp_reduce);
  m.def("tp_gather_rows", &mb::tp_gather_rows);
  m.def("tp_argmax_exchange", &mb::tp_argmax_exchange);
  m.def("tp_nvls_reduce", &mb::tp_nvls_reduce);
  m.def("multicast_supported", &mb::multicast_supported);
  m.def("ep_agrs_publish", &mb::ep_agrs_publish);
  m.def("ep_agrs_place", &mb::ep_agrs_place);
  m.def("ep_agrs_combine", &mb::ep_agrs_combine);
  m.def("ipc_alloc", [](int64_t b) {
    auto r = mb::ipc_alloc(b);
    return pybind11::make_tuple(std::get<0>(r), pybind11::bytes(std::get<1>(r)));
  });
  m.def("ipc_open", [](pybind11::bytes h) { return mb::ipc_open(std::string(h)); });
  m.def("ipc_close", &mb::ipc_close);
  m.def("ipc_free", &mb::ipc_free);
  m.def("embed", &mb::embed);
  m.def("decode_advance", &mb::decode_advance);
  m.def("swiglu", &mb::swiglu);
  m.def("argmax", &mb::argmax);
  m.def("verify_tokens", &mb::verify_tokens);
  m.def("read_and_clear_status", &mb::read_and_clear_status);
}
