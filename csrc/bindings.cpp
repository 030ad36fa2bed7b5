// Python bindings of the nano_gpic_b200 CUDA extension (module nano_gpic_b200._C).
#include <torch/extension.h>

#include "status.h"

namespace ng {
void gemm_torch(const at::Tensor& A, bool a_mn, int64_t lda, int64_t a_bs, const at::Tensor& B, bool b_mn, int64_t ldb,
                int64_t b_bs, int64_t b_rows, const at::Tensor& out, int64_t ldo, int64_t out_bs, int64_t epi, int64_t M,
                int64_t N, int64_t K, int64_t batch, const c10::optional<at::Tensor>& out2, int64_t ldo2,
                const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res, int64_t ldr,
                int64_t res_bs, const c10::optional<at::Tensor>& gate, int64_t ldg, int64_t rows_per_group,
                const c10::optional<at::Tensor>& aux, int64_t ld_aux, int64_t half_n, double alpha, double beta,
                bool accumulate, const c10::optional<at::Tensor>& seg);
void rms_mod_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& shift,
                 const c10::optional<at::Tensor>& scale, const at::Tensor& h, const at::Tensor& rstd, int64_t rpg,
                 double eps, const c10::optional<at::Tensor>& seg);
void rms_mod_bwd(const at::Tensor& dh, const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& w,
                 const c10::optional<at::Tensor>& scale, const c10::optional<at::Tensor>& dres, const at::Tensor& dx,
                 const c10::optional<at::Tensor>& dw, const c10::optional<at::Tensor>& dshift,
                 const c10::optional<at::Tensor>& dscale, int64_t rpg, const c10::optional<at::Tensor>& cu,
                 int64_t max_rows);
void rms_mod_fwd_mx(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& shift,
                    const c10::optional<at::Tensor>& scale, const at::Tensor& h, const at::Tensor& rstd,
                    const at::Tensor& q, const at::Tensor& sf, int64_t rpg, double eps);
void layernorm_fwd(const at::Tensor& x, const at::Tensor& h, const at::Tensor& mu, const at::Tensor& rstd, double eps);
void layernorm_bwd(const at::Tensor& dh, const at::Tensor& x, const at::Tensor& mu, const at::Tensor& rstd,
                   const at::Tensor& dx);
void qk_norm_fwd(const at::Tensor& src, const at::Tensor& w, const c10::optional<at::Tensor>& cosT,
                 const c10::optional<at::Tensor>& sinT, const at::Tensor& out, const at::Tensor& rstd, int64_t L,
                 double eps);
void qk_norm_bwd(const at::Tensor& dout, const at::Tensor& src, const at::Tensor& rstd, const at::Tensor& w,
                 const c10::optional<at::Tensor>& cosT, const c10::optional<at::Tensor>& sinT, const at::Tensor& dsrc,
                 const c10::optional<at::Tensor>& dw, int64_t L);
void attn_fwd(const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0, const c10::optional<at::Tensor>& k1,
              const c10::optional<at::Tensor>& v1, const at::Tensor& n0, const at::Tensor& n1, const at::Tensor& o,
              const at::Tensor& lse, int64_t Lq, int64_t L0, int64_t L1, double scale);
void attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0,
              const c10::optional<at::Tensor>& k1, const c10::optional<at::Tensor>& v1, const at::Tensor& n0,
              const at::Tensor& n1, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dq,
              const at::Tensor& dk0, const at::Tensor& dv0, const c10::optional<at::Tensor>& dk1,
              const c10::optional<at::Tensor>& dv1, int64_t Lq, int64_t L0, int64_t L1, double scale);
void gate_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& gate, const at::Tensor& dy,
              const c10::optional<at::Tensor>& dgate, const c10::optional<at::Tensor>& dbias, int64_t rpg,
              const c10::optional<at::Tensor>& cu, int64_t max_rows);
void gather_rows(const at::Tensor& src, const at::Tensor& idx, const at::Tensor& out);
void u8_to_unit(const at::Tensor& img, const at::Tensor& out);
void fm_prep(const at::Tensor& x, const at::Tensor& noise, const at::Tensor& t, const at::Tensor& xt_tok, int64_t p);
void fm_loss(const at::Tensor& pred, const at::Tensor& x, const at::Tensor& noise, const at::Tensor& t,
             const c10::optional<at::Tensor>& dpred, const at::Tensor& per_sample, int64_t p, double t_eps,
             double grad_scale);
void patchify(const at::Tensor& img, const at::Tensor& tok, int64_t p);
void unpatchify(const at::Tensor& tok, const at::Tensor& img, int64_t p);
void attn_fwd_tc(const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0, const c10::optional<at::Tensor>& k1,
                 const c10::optional<at::Tensor>& v1, const at::Tensor& n0, const at::Tensor& n1, const at::Tensor& o,
                 const at::Tensor& lse, int64_t Lq, int64_t L0, int64_t L1, double scale, int64_t version);
void gemm_set_pair(int64_t on);
std::vector<at::Tensor> mx_quant(const at::Tensor& x);
void muon_gather(const at::Tensor& tab, double beta, bool nesterov, int64_t max_numel, double mom, bool out_bf16);
void scale_by(const at::Tensor& buf, const at::Tensor& coef);
void ns_normalize(const at::Tensor& x, bool transpose, const at::Tensor& out);
void transpose_bf16(const at::Tensor& x, const at::Tensor& out);
void muon_apply(const at::Tensor& tab, double decay, int64_t max_numel, double ema_w);
void adamw_apply(const at::Tensor& tab, std::vector<double> scalars, int64_t max_numel);
void resize_passes(const at::Tensor& src, const at::Tensor& tab, const at::Tensor& desc, const at::Tensor& tmp,
                   const at::Tensor& out, int64_t max_h, int64_t max_w);
void gemm_mx_torch(const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B, const at::Tensor& sfb,
                   const at::Tensor& out, int64_t epi, int64_t N, const c10::optional<at::Tensor>& out2,
                   const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res,
                   const c10::optional<at::Tensor>& gate, int64_t rows_per_group, int64_t half_n,
                   const c10::optional<at::Tensor>& act_q, const c10::optional<at::Tensor>& act_sf,
                   const c10::optional<at::Tensor>& aux);
at::Tensor p2p_alloc(int64_t nbytes, int64_t device);
at::Tensor p2p_export(const at::Tensor& t);
int64_t p2p_import(const at::Tensor& handle, int64_t device);
void p2p_close(int64_t ptr);
void p2p_reduce_scatter(const at::Tensor& grad, const at::Tensor& recv, const std::vector<int64_t>& peer_recv,
                        const at::Tensor& flags, const std::vector<int64_t>& peer_flags, const at::Tensor& acks,
                        const std::vector<int64_t>& peer_acks, const at::Tensor& counters, const at::Tensor& sumsq,
                        int64_t rank, int64_t nb, int64_t b, int64_t start, int64_t seg, int64_t epoch);
void p2p_bcast_bf16(const at::Tensor& master, const std::vector<int64_t>& peer_w16, const std::vector<int64_t>& peer_flags,
                    const at::Tensor& counters, int64_t rank, int64_t nb, int64_t b, int64_t off, int64_t n,
                    int64_t epoch);
void p2p_wait(const at::Tensor& flags, int64_t world, int64_t rank, int64_t nb, int64_t b0, int64_t b1, int64_t epoch,
              int64_t budget_ns);
void p2p_fused_apply(const at::Tensor& table_t, int64_t nent, const at::Tensor& p, const at::Tensor& g,
                     const at::Tensor& m1, const at::Tensor& m2, const at::Tensor& upd,
                     const c10::optional<at::Tensor>& ema, const std::vector<int64_t>& peer_w16,
                     const std::vector<int64_t>& peer_wflags, const at::Tensor& counters, std::vector<double> scalars,
                     int64_t rank, int64_t nb, int64_t b, int64_t epoch);
void attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0,
                 const c10::optional<at::Tensor>& k1, const c10::optional<at::Tensor>& v1, const at::Tensor& n0,
                 const at::Tensor& n1, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dq,
                 const at::Tensor& dk0, const at::Tensor& dv0, const c10::optional<at::Tensor>& dk1,
                 const c10::optional<at::Tensor>& dv1, int64_t Lq, int64_t L0, int64_t L1, double scale, int64_t version);
void attn_prof_set(const c10::optional<at::Tensor>& counters);
void colsum(const at::Tensor& src, const at::Tensor& out, bool accumulate);
void add_rows(const at::Tensor& a, const at::Tensor& table, const at::Tensor& out, int64_t period);
}  // namespace ng

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_gpic_b200 sm_100a kernels";
  m.def("gemm", &ng::gemm_torch, "tcgen05 GEMM with fused epilogues");
  m.def("rms_mod_fwd", &ng::rms_mod_fwd);
  m.def("rms_mod_bwd", &ng::rms_mod_bwd);
  m.def("layernorm_fwd", &ng::layernorm_fwd);
  m.def("layernorm_bwd", &ng::layernorm_bwd);
  m.def("qk_norm_fwd", &ng::qk_norm_fwd);
  m.def("qk_norm_bwd", &ng::qk_norm_bwd);
  m.def("attn_fwd", &ng::attn_fwd);
  m.def("attn_bwd", &ng::attn_bwd);
  m.def("p2p_alloc", &ng::p2p_alloc, "cudaMalloc'd, zero-filled, IPC-shareable bytes");
  m.def("p2p_export", &ng::p2p_export, "CUDA IPC handle of a p2p_alloc tensor");
  m.def("p2p_import", &ng::p2p_import, "open a peer's CUDA IPC handle; returns its device address here");
  m.def("p2p_close", &ng::p2p_close);
  m.def("p2p_reduce_scatter", &ng::p2p_reduce_scatter, "peer-memory reduce-scatter of one gradient bucket");
  m.def("p2p_bcast_bf16", &ng::p2p_bcast_bf16, "owner's fp32 segment -> bf16 in every rank's weights, with flags");
  m.def("p2p_fused_apply", &ng::p2p_fused_apply,
        "sharded AdamW / Muon apply + EMA of one bucket's owned parameters, bf16 weights into every rank, flags");
  m.def("p2p_wait", &ng::p2p_wait, "wait (bounded) for every peer's weight flags of a bucket range", py::arg("flags"),
        py::arg("world"), py::arg("rank"), py::arg("nb"), py::arg("b0"), py::arg("b1"), py::arg("epoch"),
        py::arg("budget_ns") = 0);
  m.def("resize_passes", &ng::resize_passes, "Pillow-exact bicubic crop passes for a packed batch");
  m.def("muon_gather", &ng::muon_gather, "stacked Nesterov inputs of every Muon unit from a pointer table");
  m.def("muon_apply", &ng::muon_apply, "param = param * decay + coef * update for every Muon unit from a pointer table");
  m.def("adamw_apply", &ng::adamw_apply, "AdamW (+ EMA) of every row of a pointer table in one launch");
  m.def("scale_by", &ng::scale_by, "buf *= coef (fp32, coef read on the device)");
  m.def("ns_normalize", &ng::ns_normalize, "per matrix X / (||X|| + 1e-7) in bf16, optionally transposed");
  m.def("transpose_bf16", &ng::transpose_bf16, "batched bf16 transpose [n, a, b] -> [n, b, a]");
  m.def("rms_mod_fwd_mx", &ng::rms_mod_fwd_mx, "RMSNorm + adaLN modulate forward that also writes h in MXFP8");
  m.def("mx_quant", &ng::mx_quant, "bf16 [rows, K] -> MXFP8 (e4m3 values, E8M0 scale blocks)");
  m.def("gemm_mx", &ng::gemm_mx_torch, "MXFP8 block-scaled tcgen05 GEMM with the bf16 / gated / SwiGLU epilogues");
  m.def("gemm_set_pair", &ng::gemm_set_pair, "use CTA-pair (cta_group::2) GEMM tiles when M >= 256 (default on)");
  m.def("attn_fwd_tc", &ng::attn_fwd_tc, "masked attention forward on tcgen05/TMEM (version 2: persistent, two query "
        "tiles per CTA; version 1: one query tile per CTA)", py::arg("q"), py::arg("k0"), py::arg("v0"), py::arg("k1"),
        py::arg("v1"), py::arg("n0"), py::arg("n1"), py::arg("o"), py::arg("lse"), py::arg("Lq"), py::arg("L0"),
        py::arg("L1"), py::arg("scale"), py::arg("version") = 2);
  m.def("attn_prof_set", &ng::attn_prof_set, "cycle counters for the profiled attention kernels (None: off)");
  m.def("attn_bwd_tc", &ng::attn_bwd_tc, "masked attention backward on tcgen05/TMEM (version 2: persistent, 8 compute "
        "warps; version 1: CTA per key tile)", py::arg("dout"), py::arg("q"), py::arg("k0"), py::arg("v0"),
        py::arg("k1"), py::arg("v1"), py::arg("n0"), py::arg("n1"), py::arg("o"), py::arg("lse"), py::arg("dq"),
        py::arg("dk0"), py::arg("dv0"), py::arg("dk1"), py::arg("dv1"), py::arg("Lq"), py::arg("L0"), py::arg("L1"),
        py::arg("scale"), py::arg("version") = 2);
  m.def("gate_bwd", &ng::gate_bwd);
  m.def("gather_rows", &ng::gather_rows, "out[r] = src[idx[r]] (bf16 rows), zeros where idx[r] < 0");
  m.def("u8_to_unit", &ng::u8_to_unit, "uint8 [B, H, W, 3] -> fp32 [B, 3, H, W] in [-1, 1] (ToTensor + Normalize 0.5)");
  m.def("fm_prep", &ng::fm_prep);
  m.def("fm_loss", &ng::fm_loss);
  m.def("patchify", &ng::patchify);
  m.def("unpatchify", &ng::unpatchify);
  m.def("add_rows", &ng::add_rows);
  m.def("colsum", &ng::colsum, "deterministic column sums (fp32/bf16 source) into an fp32 vector");
  m.def("status_read", &ng::status_read, "read the device error word (synchronizes the current stream)");
  m.def("launch_count", &ng::launch_count, "kernel launches issued by this extension so far (host count)");
  m.def("status_clear", &ng::status_clear, "clear the device error word");
  m.def("status_copy_async", &ng::status_copy_async, "copy the device error word into a pinned host int32, no wait");
}
