// Python bindings of the sm_100a kernel library (module prism_cp_b200._C).
#include <torch/extension.h>

namespace prism {
void gemm_sm100(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, bool a_mn, bool b_mn, bool accumulate,
                const c10::optional<at::Tensor>& row_scale, at::Tensor& status);
void gemm_allreduce_sm100(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, bool a_mn, bool b_mn,
                          const at::Tensor& regions, int64_t me, int64_t max_tiles, int64_t ld, int64_t seq,
                          at::Tensor& status);
void rownorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& z,
                 at::Tensor& y, at::Tensor& rstd, int64_t heads, int64_t n, double inv_n, double eps);
c10::optional<at::Tensor> rownorm_bwd(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                                      const c10::optional<at::Tensor>& z, const at::Tensor& rstd, at::Tensor& dx,
                                      const c10::optional<at::Tensor>& dz, int64_t heads, int64_t n, double inv_n);
void rope_inplace(at::Tensor& x, const at::Tensor& pos, int64_t heads, int64_t d, double base, bool inverse);
at::Tensor conv1d_silu_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& halo,
                           const at::Tensor& cu);
std::vector<at::Tensor> conv1d_silu_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                        const c10::optional<at::Tensor>& halo, const at::Tensor& cu, at::Tensor& dx);
void swiglu_fwd(const at::Tensor& x, at::Tensor& y);
void swiglu_bwd(const at::Tensor& dy, const at::Tensor& x, at::Tensor& dx);
void ce_fused(at::Tensor& logits, const at::Tensor& labels, const at::Tensor& weight, at::Tensor& loss,
              const c10::optional<at::Tensor>& lse);
void sumsq_accumulate(const at::Tensor& g, at::Tensor& out);
void adamw_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& p_bf16, const at::Tensor& sumsq, double max_norm, double lr,
                double b1, double b2, double eps, double wd, double bc1, double bc2);
void attention_fwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu_q,
                         const at::Tensor& cu_k, const at::Tensor& tiles, at::Tensor& out, at::Tensor& lse,
                         bool causal, double softmax_scale, at::Tensor& status);
void attention_bwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& out,
                         const at::Tensor& lse, const at::Tensor& dout, const at::Tensor& cu_q, const at::Tensor& cu_k,
                         const at::Tensor& tiles_q, const at::Tensor& tiles_k, at::Tensor& dq, at::Tensor& dk,
                         at::Tensor& dv, bool causal, double softmax_scale, at::Tensor& status);
void gdn_state_fwd(const at::Tensor& W, const at::Tensor& U, const at::Tensor& Kd, const at::Tensor& gamma,
                   const c10::optional<at::Tensor>& S0, const at::Tensor& seq_chunks, at::Tensor& Delta,
                   at::Tensor& S_all, at::Tensor& S_final);
void gdn_state_bwd(const at::Tensor& W, const at::Tensor& dDelta_ext, const at::Tensor& Kd, const at::Tensor& gamma,
                   const at::Tensor& dS_ext, const c10::optional<at::Tensor>& dS_final, const at::Tensor& seq_chunks,
                   at::Tensor& dDelta, at::Tensor& G_next, at::Tensor& dS0);
std::vector<at::Tensor> gdn_chunk_prep(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const at::Tensor& g, const at::Tensor& beta, const at::Tensor& tok0,
                                       const at::Tensor& len, double scale, bool with_aux, at::Tensor& status);
void gdn_chunk_fwd(const at::Tensor& Wn, const at::Tensor& U, const at::Tensor& Kd, const at::Tensor& Qg,
                   const at::Tensor& Aqk, const at::Tensor& gam, const at::Tensor& tok0, const at::Tensor& len,
                   const at::Tensor& seq_chunks, const c10::optional<at::Tensor>& S0,
                   const c10::optional<at::Tensor>& out, const c10::optional<at::Tensor>& S_final,
                   const c10::optional<at::Tensor>& states, const c10::optional<at::Tensor>& rows,
                   at::Tensor& status);
void gdn_chunk_bwd_state(const at::Tensor& Wn, const at::Tensor& Kd, const at::Tensor& Qg, const at::Tensor& Aqk,
                         const at::Tensor& gam, const at::Tensor& dout, const at::Tensor& tok0, const at::Tensor& len,
                         const at::Tensor& seq_chunks, const c10::optional<at::Tensor>& dS_final,
                         const c10::optional<at::Tensor>& dS0, at::Tensor& states, at::Tensor& rows,
                         at::Tensor& status);
bool gdn_local_tc_enabled(int64_t set);
std::vector<at::Tensor> gdn_chunk_bwd_local(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& g, const at::Tensor& beta, const at::Tensor& tok0,
                                            const at::Tensor& len, const at::Tensor& Gc, const at::Tensor& aux,
                                            const at::Tensor& states,
                                            const at::Tensor& dstates, const at::Tensor& rows,
                                            const at::Tensor& drows, const at::Tensor& dout, double scale,
                                            at::Tensor& status, const std::vector<at::Tensor>& second);
void attention_fwd_peer(const at::Tensor& q, const std::vector<at::Tensor>& k_peers,
                        const std::vector<at::Tensor>& v_peers, const at::Tensor& tiles, const at::Tensor& seq_n,
                        const at::Tensor& seq_row0, at::Tensor& out, at::Tensor& lse, double softmax_scale,
                        at::Tensor& status);
void attention_bwd_peer(const std::vector<at::Tensor>& q_peers, const std::vector<at::Tensor>& k_peers,
                        const std::vector<at::Tensor>& v_peers, const std::vector<at::Tensor>& do_peers,
                        const std::vector<at::Tensor>& lse_peers, const std::vector<at::Tensor>& dsum_peers,
                        int64_t rank, const at::Tensor& tiles, const at::Tensor& seq_n, const at::Tensor& seq_row0,
                        at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, double softmax_scale, at::Tensor& status);
void attention_bwd_dsum(const at::Tensor& out, const at::Tensor& dout, at::Tensor& dsum);
int64_t symm_alloc(int64_t bytes);
void symm_free(int64_t ptr);
at::Tensor symm_handle(int64_t ptr);
int64_t symm_open(const at::Tensor& handle);
void symm_close(int64_t ptr);
void symm_signal(const at::Tensor& peer_signal_bases, int64_t slot, int64_t value);
void symm_wait(int64_t my_signal_base, int64_t first, int64_t count, int64_t value, at::Tensor& status,
               int64_t limit_ns);
void symm_gather_rows(const at::Tensor& peer_bases, const at::Tensor& routes, const at::Tensor& block_route,
                      const at::Tensor& block_row0, int64_t rows_per_block, int64_t row_bytes, at::Tensor& dst,
                      at::Tensor& status);
at::Tensor symm_tensor(int64_t ptr, std::vector<int64_t> sizes, int64_t dtype_code, int64_t device);
}  // namespace prism

// Every op releases the GIL while it runs: launches never call back into Python, and a
// host call that blocks (an allocation that synchronises) must not stall other Python threads.
PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "prism_cp_b200 sm_100a kernels";
  m.def("gemm", &prism::gemm_sm100, py::call_guard<py::gil_scoped_release>(), "tcgen05 GEMM C (+)= rowscale * A B^T");
  m.def("gemm_allreduce", &prism::gemm_allreduce_sm100, py::call_guard<py::gil_scoped_release>(), "tcgen05 GEMM fused with an all-reduce over peer memory");
  m.def("rownorm_fwd", &prism::rownorm_fwd, py::call_guard<py::gil_scoped_release>());
  m.def("rownorm_bwd", &prism::rownorm_bwd, py::call_guard<py::gil_scoped_release>());
  m.def("rope_inplace", &prism::rope_inplace, py::call_guard<py::gil_scoped_release>());
  m.def("conv1d_silu_fwd", &prism::conv1d_silu_fwd, py::call_guard<py::gil_scoped_release>());
  m.def("conv1d_silu_bwd", &prism::conv1d_silu_bwd, py::call_guard<py::gil_scoped_release>());
  m.def("swiglu_fwd", &prism::swiglu_fwd, py::call_guard<py::gil_scoped_release>());
  m.def("swiglu_bwd", &prism::swiglu_bwd, py::call_guard<py::gil_scoped_release>());
  m.def("ce_fused", &prism::ce_fused, py::call_guard<py::gil_scoped_release>());
  m.def("sumsq_accumulate", &prism::sumsq_accumulate, py::call_guard<py::gil_scoped_release>());
  m.def("adamw_step", &prism::adamw_step, py::call_guard<py::gil_scoped_release>());
  m.def("attention_fwd", &prism::attention_fwd_sm100, py::call_guard<py::gil_scoped_release>(), "tcgen05 varlen GQA flash attention forward");
  m.def("attention_bwd", &prism::attention_bwd_sm100, py::call_guard<py::gil_scoped_release>(), "tcgen05 varlen GQA flash attention backward");
  m.def("gdn_state_fwd", &prism::gdn_state_fwd, py::call_guard<py::gil_scoped_release>());
  m.def("gdn_state_bwd", &prism::gdn_state_bwd, py::call_guard<py::gil_scoped_release>());
  m.def("gdn_chunk_prep", &prism::gdn_chunk_prep, py::call_guard<py::gil_scoped_release>(), "GDN chunk prep: WY form, decays, Aqk (CUDA cores)");
  m.def("gdn_chunk_fwd", &prism::gdn_chunk_fwd, py::call_guard<py::gil_scoped_release>(), "GDN tcgen05 state pass with the output fused");
  m.def("gdn_chunk_bwd_state", &prism::gdn_chunk_bwd_state, py::call_guard<py::gil_scoped_release>(), "GDN tcgen05 reverse state pass");
  m.def("gdn_local_tc_enabled", &prism::gdn_local_tc_enabled, "select (1) or query (-1) the tcgen05 GDN local backward");
  m.def("gdn_chunk_bwd_local", &prism::gdn_chunk_bwd_local, py::call_guard<py::gil_scoped_release>(), "GDN chunk-local backward (tcgen05 + CUDA cores)");
  m.def("attention_fwd_peer", &prism::attention_fwd_peer, py::call_guard<py::gil_scoped_release>(),
        "context-parallel attention forward reading every KV tile from its owner's symmetric buffer");
  m.def("attention_bwd_peer", &prism::attention_bwd_peer, py::call_guard<py::gil_scoped_release>(),
        "context-parallel attention backward reading peer Q/dO/K/V tiles and LSE/D rows");
  m.def("attention_bwd_dsum", &prism::attention_bwd_dsum, py::call_guard<py::gil_scoped_release>());
  m.def("symm_alloc", &prism::symm_alloc, py::call_guard<py::gil_scoped_release>());
  m.def("symm_free", &prism::symm_free, py::call_guard<py::gil_scoped_release>());
  m.def("symm_handle", &prism::symm_handle, py::call_guard<py::gil_scoped_release>());
  m.def("symm_open", &prism::symm_open, py::call_guard<py::gil_scoped_release>());
  m.def("symm_close", &prism::symm_close, py::call_guard<py::gil_scoped_release>());
  m.def("symm_signal", &prism::symm_signal, py::call_guard<py::gil_scoped_release>());
  m.def("symm_wait", &prism::symm_wait, py::call_guard<py::gil_scoped_release>());
  m.def("symm_gather_rows", &prism::symm_gather_rows, py::call_guard<py::gil_scoped_release>(), "P2P row gather over NVLink (CP-transition reshard)");
  m.def("symm_tensor", &prism::symm_tensor, py::call_guard<py::gil_scoped_release>());
}
