// Python bindings of the sm_100a kernels (module trainium_frontier_b200._C).
#include <torch/extension.h>

namespace tfb {
void gemm_bf16(torch::Tensor A, bool a_mn, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
               torch::Tensor D, int64_t epi, double alpha, double beta, c10::optional<torch::Tensor> R,
               c10::optional<torch::Tensor> D2, double tau, int64_t split_k, int64_t bn, torch::Tensor err,
               c10::optional<torch::Tensor> alpha_t, double rcoef);
void gemm_tp(int64_t mode, torch::Tensor A, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
             torch::Tensor D, int64_t epi, c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> D2,
             double tau, double rcoef, int64_t rank, int64_t world, int64_t rows_per_rank, int64_t epoch,
             std::vector<int64_t> ag_src, std::vector<int64_t> ag_ready, c10::optional<torch::Tensor> claim,
             c10::optional<torch::Tensor> done, std::vector<int64_t> rs_recv, std::vector<int64_t> rs_flag,
             torch::Tensor sched, int64_t bn, torch::Tensor err);
void gemm_rope(torch::Tensor A, torch::Tensor B, torch::Tensor D, torch::Tensor cos, torch::Tensor sin, int64_t T,
               int64_t rope_cols, c10::optional<torch::Tensor> rstd, torch::Tensor err);
void gemm_ce(torch::Tensor A, torch::Tensor B, torch::Tensor D, torch::Tensor tgt, int64_t T,
             c10::optional<torch::Tensor> roww, int64_t V, double S, torch::Tensor part, torch::Tensor yc,
             torch::Tensor loss, bool write_dz, torch::Tensor err);
void gemm_splitk_fin(torch::Tensor A, torch::Tensor B, torch::Tensor ws, torch::Tensor cnt, torch::Tensor out,
                     c10::optional<torch::Tensor> R, bool relu2, double tau, int64_t split, torch::Tensor err);
void rmsnorm_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> rstd);
void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor rstd, c10::optional<torch::Tensor> dadd,
                 torch::Tensor dx);
void mix_norm_fwd(torch::Tensor x, torch::Tensor x0, torch::Tensor lr, torch::Tensor l0, torch::Tensor xm,
                  torch::Tensor h, torch::Tensor rstd);
void mix_norm_bwd(torch::Tensor dxm, torch::Tensor dh, torch::Tensor x, torch::Tensor x0, torch::Tensor xm,
                  torch::Tensor rstd, torch::Tensor lr, torch::Tensor l0, torch::Tensor dx, torch::Tensor dx0_acc,
                  bool dx0_init, torch::Tensor dlr, torch::Tensor dl0);
void embed_norm_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor out, torch::Tensor rstd);
void embed_norm_bwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor rstd, c10::optional<torch::Tensor> gacc,
                    c10::optional<torch::Tensor> gb, torch::Tensor dwte);
void causal_conv_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y);
void causal_conv_bwd(torch::Tensor x, torch::Tensor w, torch::Tensor dy, torch::Tensor dx, torch::Tensor dw,
                     torch::Tensor part, bool accumulate);
void ngram_gather(torch::Tensor idx, int64_t order, int64_t p1, int64_t p2, int64_t p3, int64_t mod, int64_t pad,
                  torch::Tensor table, torch::Tensor out, torch::Tensor rows);
void ngram_scatter(torch::Tensor rows, torch::Tensor dout, torch::Tensor grad);
void muon_fro_scale(torch::Tensor x, torch::Tensor fro);
void normuon_tail(torch::Tensor gq, torch::Tensor second, torch::Tensor one_b2, c10::optional<torch::Tensor> out,
                  c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> lr, c10::optional<torch::Tensor> lrwd);
void fa_trace_set(c10::optional<torch::Tensor> buf);
void embed_grad_det(torch::Tensor idx, torch::Tensor wte, torch::Tensor rstd, c10::optional<torch::Tensor> gacc,
                    c10::optional<torch::Tensor> gb, torch::Tensor dwte);
void rope_norm_fwd(torch::Tensor buf, int64_t head0, int64_t nheads, int64_t D, torch::Tensor cos,
                   torch::Tensor sin, int64_t T, int64_t pos_offset, c10::optional<torch::Tensor> rstd,
                   c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> pos_t);
void decode_attn(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor len, int64_t H,
                 int64_t D, double scale, torch::Tensor out);
void decode_attn_split(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor len, int64_t H,
                       int64_t D, double scale, torch::Tensor out, torch::Tensor ws, torch::Tensor cnt, int64_t splits,
                       bool pdl);
void decode_gemm(torch::Tensor X, torch::Tensor W, torch::Tensor out, int64_t epi, bool row_norm,
                 c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> X0, c10::optional<torch::Tensor> lam_r,
                 c10::optional<torch::Tensor> lam_0, double tau, c10::optional<torch::Tensor> cos,
                 c10::optional<torch::Tensor> sin, c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> kc,
                 c10::optional<torch::Tensor> vc, int64_t H, int64_t split, bool pdl, torch::Tensor err);
void decode_gemm_trace_set(c10::optional<torch::Tensor> buf);
void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor pos);
void step_advance(torch::Tensor counters);
void argmax_rows(torch::Tensor logits, int64_t V, torch::Tensor idx_out, c10::optional<torch::Tensor> tokens,
                 torch::Tensor counters, int64_t start);
void rope_norm_bwd(torch::Tensor gbuf, torch::Tensor zbuf, int64_t head0, int64_t nheads, int64_t D,
                   torch::Tensor cos, torch::Tensor sin, int64_t T, torch::Tensor rstd);
void softcap_ce(torch::Tensor logits, torch::Tensor targets, int64_t T, c10::optional<torch::Tensor> row_w,
                int64_t V, double S, double scale, torch::Tensor loss, bool write_grad);
void adamw_multi(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> m,
                 std::vector<torch::Tensor> v, torch::Tensor lr, double beta1, double beta2, double eps, double wd,
                 std::vector<double> bc1, std::vector<double> bc2, bool cautious);
void fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t B, int64_t T, int64_t H, int64_t D,
            double scale, bool causal, torch::Tensor out, torch::Tensor lse, torch::Tensor err);
void fa_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout, torch::Tensor lse,
            int64_t B, int64_t T, int64_t H, int64_t D, double scale, bool causal, torch::Tensor dq_acc,
            torch::Tensor dq_out, torch::Tensor dk, torch::Tensor dv, torch::Tensor dvec, torch::Tensor err);
void muon_apply(torch::Tensor w, torch::Tensor g, torch::Tensor lr, torch::Tensor lrwd);
void symm_barrier(std::vector<int64_t> pad_ptrs, int64_t rank, int64_t epoch, torch::Tensor err);
void symm_rs(std::vector<int64_t> peer_ptrs, int64_t src_off, int64_t n, torch::Tensor out, double inv,
             c10::optional<torch::Tensor> sumsq, int64_t mc_ptr);
void muon_pre(torch::Tensor g, torch::Tensor mb, torch::Tensor x, c10::optional<torch::Tensor> coef, torch::Tensor mom,
              torch::Tensor one_mom, torch::Tensor fro);
void symm_ag_apply(std::vector<int64_t> upd_ptrs, torch::Tensor runs_i64);
}  // namespace tfb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.doc() = "trainium_frontier_b200 sm_100a kernels";
  m.def("gemm_bf16", &tfb::gemm_bf16, "tcgen05 bf16 GEMM with fused epilogues", py::arg("A"), py::arg("a_mn"),
        py::arg("B"), py::arg("b_mn"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("D"), py::arg("epi"),
        py::arg("alpha"), py::arg("beta"), py::arg("R"), py::arg("D2"), py::arg("tau"), py::arg("split_k"),
        py::arg("bn"), py::arg("err"), py::arg("alpha_t") = py::none(), py::arg("rcoef") = 1.0);
  m.def("gemm_tp", &tfb::gemm_tp);
  m.def("gemm_splitk_fin", &tfb::gemm_splitk_fin);
  m.def("gemm_ce", &tfb::gemm_ce, "lm_head GEMM with softcap + cross-entropy (+ dlogits) in the epilogue");
  m.def("gemm_rope", &tfb::gemm_rope, "tcgen05 bf16 GEMM with RoPE + per-head RMSNorm on the leading columns");
  m.def("rmsnorm_fwd", &tfb::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &tfb::rmsnorm_bwd);
  m.def("mix_norm_fwd", &tfb::mix_norm_fwd);
  m.def("mix_norm_bwd", &tfb::mix_norm_bwd);
  m.def("embed_norm_fwd", &tfb::embed_norm_fwd);
  m.def("embed_norm_bwd", &tfb::embed_norm_bwd);
  m.def("embed_grad_det", &tfb::embed_grad_det, "deterministic embedding gradient (sorted segmented sums)");
  m.def("rope_norm_fwd", &tfb::rope_norm_fwd, py::arg("buf"), py::arg("head0"), py::arg("nheads"), py::arg("D"),
        py::arg("cos"), py::arg("sin"), py::arg("T"), py::arg("pos_offset"), py::arg("rstd"), py::arg("out"),
        py::arg("pos_t") = py::none());
  m.def("decode_attn", &tfb::decode_attn);
  m.def("decode_attn_split", &tfb::decode_attn_split);
  m.def("decode_gemm", &tfb::decode_gemm);
  m.def("decode_gemm_trace_set", &tfb::decode_gemm_trace_set);
  m.def("kv_append", &tfb::kv_append);
  m.def("step_advance", &tfb::step_advance);
  m.def("argmax_rows", &tfb::argmax_rows);
  m.def("rope_norm_bwd", &tfb::rope_norm_bwd);
  m.def("softcap_ce", &tfb::softcap_ce);
  m.def("adamw_multi", &tfb::adamw_multi);
  m.def("muon_apply", &tfb::muon_apply);
  m.def("symm_barrier", &tfb::symm_barrier);
  m.def("symm_rs", &tfb::symm_rs);
  m.def("muon_pre", &tfb::muon_pre);
  m.def("symm_ag_apply", &tfb::symm_ag_apply);
  m.def("causal_conv_fwd", &tfb::causal_conv_fwd, "causal depthwise conv1d forward (bf16)");
  m.def("causal_conv_bwd", &tfb::causal_conv_bwd, "causal depthwise conv1d backward (dx, deterministic dw)");
  m.def("ngram_gather", &tfb::ngram_gather, "hashed n-gram row ids + gather (bf16 out)");
  m.def("ngram_scatter", &tfb::ngram_scatter, "n-gram table gradient scatter-add (fp32)");
  m.def("muon_fro_scale", &tfb::muon_fro_scale, "Muon Frobenius normalisation (reference bf16 op order)");
  m.def("normuon_tail", &tfb::normuon_tail, "NorMuon second moment + scaled update (or its apply)");
  m.def("fa_trace_set", &tfb::fa_trace_set, "install / remove the flash-attention phase timeline buffer");
  m.def("fa_fwd", &tfb::fa_fwd, "tcgen05 causal flash attention forward");
  m.def("fa_bwd", &tfb::fa_bwd, "tcgen05 causal flash attention backward");
}
