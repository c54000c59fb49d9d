// Python bindings of the sm_100a kernels (one extension module, dllm_qwen38_b200._C).
#include <torch/extension.h>

namespace bdllm {
void gemm(const at::Tensor& a, bool a_mn, int64_t lda, const at::Tensor& b, bool b_mn, int64_t ldb, int64_t M,
          int64_t N, int64_t K, at::Tensor& c, int64_t ldc, int64_t epi, const c10::optional<at::Tensor>& r,
          int64_t ldr, const c10::optional<at::Tensor>& gu, int64_t bn, double alpha,
          const c10::optional<at::Tensor>& alpha_t);
at::Tensor dswiglu(const at::Tensor& dact, const at::Tensor& gu);
at::Tensor group_sum(const at::Tensor& x, int64_t groups);
std::vector<at::Tensor> mask_sample(const at::Tensor& x0, const at::Tensor& prompt_len,
                                    const c10::optional<at::Tensor>& valid_len, int64_t block, int64_t mask_id,
                                    int64_t seed);
at::Tensor conv_fwd(const at::Tensor& raw, const at::Tensor& w, int64_t L, int64_t block, int64_t mode);
std::vector<at::Tensor> conv_bwd(const at::Tensor& dy, const at::Tensor& raw, const at::Tensor& w, int64_t L,
                                 int64_t block, int64_t mode);
at::Tensor ce_rows_(at::Tensor& logits, const at::Tensor& tgt);
void sumsq_(const at::Tensor& x, at::Tensor& sq, const c10::optional<at::Tensor>& dst);
void adamw_step(at::Tensor& w, at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1,
                double b2, double eps, double wd, double coef, const c10::optional<at::Tensor>& coef_dev, double bc1,
                double bc2);
int64_t read_error_word(bool reset);
std::vector<std::tuple<std::string, int64_t, int64_t, int64_t, int64_t>> bounds_report(bool reset);
bool debug_bounds_build();
at::Tensor rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w1, double eps);
std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w1, double eps);
at::Tensor gated_rmsnorm_fwd(const at::Tensor& x, const at::Tensor& z, const at::Tensor& w, double eps);
std::vector<at::Tensor> gated_rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& z,
                                          const at::Tensor& w, double eps);
at::Tensor qk_norm_rope_fwd(const at::Tensor& src, const at::Tensor& w1, const at::Tensor& cs, const at::Tensor& sn,
                            double eps);
std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dout, const at::Tensor& src, const at::Tensor& w1,
                                         const at::Tensor& cs, const at::Tensor& sn, double eps);
std::vector<at::Tensor> gdn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                const at::Tensor& beta, int64_t L, int64_t C, bool concat);
bool gdn_tc_eligible(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L, int64_t C,
                     bool concat);
std::vector<at::Tensor> gdn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                   const at::Tensor& beta, int64_t L);
std::vector<at::Tensor> gdn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S_in, int64_t L,
                                int64_t C, bool concat);
std::vector<at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L,
                                 int64_t block, double scale, bool leak);
std::vector<at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                 const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, int64_t L,
                                 int64_t block, double scale, bool leak);
at::Tensor attn_prefix(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t tk_host,
                       const c10::optional<at::Tensor>& tk, double scale);
std::vector<at::Tensor> gdn_rows(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                 const at::Tensor& beta, const at::Tensor& S0, const c10::optional<at::Tensor>& S_final,
                                 int64_t C);
std::vector<at::Tensor> gdn_fwd_rows(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                     const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S0, int64_t C);
std::vector<at::Tensor> gdn_bwd_rows(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                     const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                     const at::Tensor& S_in, int64_t C, const c10::optional<at::Tensor>& inj,
                                     bool want_dS0);
at::Tensor conv_tail(const at::Tensor& raw, at::Tensor& tail, const at::Tensor& w, bool update_tail);
void confidence(const at::Tensor& logits, at::Tensor& conf, at::Tensor& pick);
void commit(const at::Tensor& conf, const at::Tensor& pick, at::Tensor& masked, at::Tensor& ids, double threshold,
            int64_t sub_block, at::Tensor& forwards, at::Tensor& remaining);
int64_t gemm_tp(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, int64_t epi,
                const c10::optional<at::Tensor>& gu, const std::vector<int64_t>& peers, int64_t rank,
                int64_t rows_per_rank, int64_t part_off, int64_t flag_off, const at::Tensor& ctr, bool wait_ag,
                double timeout_s, int64_t bn, int64_t ksplit);
void gemm_ag(const at::Tensor& a, const at::Tensor& w, at::Tensor& c, int64_t epi, const c10::optional<at::Tensor>& gu,
             const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes,
             at::Tensor& gathered, at::Tensor& ready, at::Tensor& claim, int64_t seq, int64_t epoch, int64_t flag_off,
             double timeout_s, int64_t lo, int64_t hi);
void splitk_reduce(const at::Tensor& ws, int64_t S, at::Tensor& out, const c10::optional<at::Tensor>& residual,
                   bool swiglu);
void tp_reduce_norm_push(const std::vector<int64_t>& peers, int64_t rank, int64_t R, int64_t D, int64_t part_off,
                         at::Tensor& h, bool has_partials, const at::Tensor& w1, double eps, int64_t gather_off,
                         int64_t flag_off, at::Tensor& ctr, double timeout_s, bool do_push, int64_t nslots);
void tp_confidence(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& logits, int64_t v0,
                   int64_t conf_off, int64_t flag_off, at::Tensor& ctr, at::Tensor& conf, at::Tensor& pick,
                   double timeout_s);
at::Tensor embed_fwd(const at::Tensor& ids, const at::Tensor& table);
void embed_bwd_(at::Tensor& grad, const at::Tensor& ids, const at::Tensor& dh);
void embed_bwd_sorted(at::Tensor& grad, const at::Tensor& sid, const at::Tensor& perm, const at::Tensor& dh);
at::Tensor swiglu_act(const at::Tensor& gu);
at::Tensor out_gate_fwd(const at::Tensor& o, const at::Tensor& g);
std::vector<at::Tensor> out_gate_bwd(const at::Tensor& dy, const at::Tensor& o, const at::Tensor& g);
std::vector<at::Tensor> gdn_gates_fwd(const at::Tensor& a, const at::Tensor& b, const at::Tensor& A_log,
                                      const at::Tensor& dt_bias);
std::vector<at::Tensor> gdn_gates_bwd(const at::Tensor& dg, const at::Tensor& dbeta, const at::Tensor& a,
                                      const at::Tensor& b, const at::Tensor& A_log, const at::Tensor& dt_bias);
void gemm_splitk(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, at::Tensor& ws, int64_t S,
                 const c10::optional<at::Tensor>& residual);
namespace peer {
int64_t alloc(int64_t bytes);
at::Tensor handle(int64_t ptr);
int64_t open(const at::Tensor& h);
void close(int64_t ptr);
void release(int64_t ptr);
at::Tensor view(int64_t ptr, int64_t numel, const at::Tensor& like);
void signal(const std::vector<int64_t>& peers, int64_t rank, int64_t slot, int64_t value);
void all_gather(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes, at::Tensor& out,
                int64_t epoch, int64_t max_blocks, double timeout_s);
void gather_range(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes, at::Tensor& out,
                  int64_t lo, int64_t hi, int64_t epoch, double timeout_s);
void reduce_scatter(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard, bool in_f32,
                    at::Tensor& out, double scale, const c10::optional<at::Tensor>& sq, int64_t seq,
                    int64_t max_blocks, double timeout_s, const std::vector<at::Tensor>& adam_state,
                    const std::vector<double>& adam_hp);
void allreduce_f32(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& vals, at::Tensor& out,
                   int64_t seq, double timeout_s);
}  // namespace peer
}  // namespace bdllm

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dllm_qwen38_b200 sm_100a kernels";
  m.def("gemm", &bdllm::gemm, "tcgen05 bf16 GEMM with fused epilogues", py::arg("a"), py::arg("a_mn"),
        py::arg("lda"), py::arg("b"), py::arg("b_mn"), py::arg("ldb"), py::arg("M"), py::arg("N"), py::arg("K"),
        py::arg("c"), py::arg("ldc"), py::arg("epi"), py::arg("r") = c10::nullopt, py::arg("ldr") = 0,
        py::arg("gu") = c10::nullopt, py::arg("bn") = 256, py::arg("alpha") = 1.0,
        py::arg("alpha_t") = c10::nullopt);
  m.def("dswiglu", &bdllm::dswiglu);
  m.def("conv_fwd", &bdllm::conv_fwd);
  m.def("conv_bwd", &bdllm::conv_bwd);
  m.def("ce_rows_", &bdllm::ce_rows_);
  m.def("adamw_step", &bdllm::adamw_step);
  m.def("sumsq_", &bdllm::sumsq_, "sq += ||x||^2 (optionally writing x as fp32)", py::arg("x"), py::arg("sq"),
        py::arg("dst") = c10::nullopt);
  m.def("mask_sample", &bdllm::mask_sample, "complementary masks and both noised views of a step, one launch");
  m.def("group_sum", &bdllm::group_sum, "GQA: bf16 [..., H, D] summed over each of `groups` head groups");
  m.def("gdn_fwd", &bdllm::gdn_fwd, "state-fork chunked gated delta rule forward");
  m.def("gdn_tc_eligible", &bdllm::gdn_tc_eligible, "whether the tcgen05 GDN forward takes this problem");
  m.def("gdn_fwd_tc", &bdllm::gdn_fwd_tc, "state-fork GDN forward on tcgen05 / TMEM / TMA (head dim 128, chunk 32)");
  m.def("gdn_bwd", &bdllm::gdn_bwd, "state-fork chunked gated delta rule backward");
  m.def("attn_fwd", &bdllm::attn_fwd, "complementary-mask flash attention forward");
  m.def("attn_bwd", &bdllm::attn_bwd, "complementary-mask flash attention backward");
  m.def("rmsnorm_fwd", &bdllm::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &bdllm::rmsnorm_bwd);
  m.def("gated_rmsnorm_fwd", &bdllm::gated_rmsnorm_fwd);
  m.def("gated_rmsnorm_bwd", &bdllm::gated_rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &bdllm::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &bdllm::qk_norm_rope_bwd);
  m.def("attn_prefix", &bdllm::attn_prefix, "attention of a query block over a KV cache (every key visible)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("tk_host"), py::arg("tk") = c10::nullopt, py::arg("scale"));
  m.def("gdn_fwd_rows", &bdllm::gdn_fwd_rows, "gated delta rule rows from initial states, with chunk states");
  m.def("gdn_bwd_rows", &bdllm::gdn_bwd_rows, "backward of gated delta rule rows (injected state grads, dS0)",
        py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("beta"), py::arg("S_in"),
        py::arg("C"), py::arg("inj") = c10::nullopt, py::arg("want_dS0") = false);
  m.def("gdn_rows", &bdllm::gdn_rows, "gated delta rule over decode rows from a cached state", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("g"), py::arg("beta"), py::arg("S0"), py::arg("S_final") = c10::nullopt,
        py::arg("C"));
  m.def("conv_tail", &bdllm::conv_tail, "short causal conv + SiLU of a block over a cached conv tail");
  m.def("confidence", &bdllm::confidence, "softmax max probability and argmax per logits row");
  m.def("commit", &bdllm::commit, "confidence-threshold commit rule per batch row, on the device");
  m.def("gemm_tp", &bdllm::gemm_tp,
        "tensor-parallel tcgen05 GEMM: fused all-gather wait in the producer, peer-store partial epilogue",
        py::arg("a"), py::arg("b"), py::arg("c"), py::arg("epi"), py::arg("gu"), py::arg("peers"), py::arg("rank"),
        py::arg("rows_per_rank"), py::arg("part_off"), py::arg("flag_off"), py::arg("ctr"), py::arg("wait_ag"),
        py::arg("timeout_s"), py::arg("bn") = 256, py::arg("ksplit") = 1);
  m.def("gemm_ag", &bdllm::gemm_ag,
        "fused FSDP all-gather -> GEMM: copy warps pull the unit's shards from the peers while the tiles wait per chunk",
        py::arg("a"), py::arg("w"), py::arg("c"), py::arg("epi"), py::arg("gu"), py::arg("peers"), py::arg("rank"),
        py::arg("src_off"), py::arg("shard_bytes"), py::arg("gathered"), py::arg("ready"), py::arg("claim"),
        py::arg("seq"), py::arg("epoch"), py::arg("flag_off"), py::arg("timeout_s"), py::arg("lo") = 0,
        py::arg("hi") = 0);
  m.def("splitk_reduce", &bdllm::splitk_reduce, "sum of k-split partials (+ residual, or SwiGLU of gate|up)",
        py::arg("ws"), py::arg("S"), py::arg("out"), py::arg("residual") = c10::nullopt, py::arg("swiglu") = false);
  m.def("tp_reduce_norm_push", &bdllm::tp_reduce_norm_push,
        "owner rows: sum peers' partials + residual, RMSNorm, push to every rank's gathered buffer");
  m.def("tp_confidence", &bdllm::tp_confidence, "vocab-parallel confidence: per-slice push + rank-order merge");
  m.def("embed_fwd", &bdllm::embed_fwd, "embedding row gather");
  m.def("embed_bwd_", &bdllm::embed_bwd_, "embedding gradient scatter-add into an fp32 table");
  m.def("embed_bwd_sorted", &bdllm::embed_bwd_sorted,
        "embedding gradient as per-id sums of the sorted rows, written as bf16 rows (others untouched)");
  m.def("swiglu_act", &bdllm::swiglu_act, "act = silu(gate) * up from the stored bf16 (gate | up)");
  m.def("out_gate_fwd", &bdllm::out_gate_fwd, "attention output gate y = o * sigmoid(gate)");
  m.def("out_gate_bwd", &bdllm::out_gate_bwd, "output gate backward: (d o, d gate)");
  m.def("gdn_gates_fwd", &bdllm::gdn_gates_fwd, "beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias)");
  m.def("gdn_gates_bwd", &bdllm::gdn_gates_bwd);
  m.def("gemm_splitk", &bdllm::gemm_splitk, "split-K tcgen05 GEMM for skinny problems (+ residual)",
        py::arg("a"), py::arg("b"), py::arg("out"), py::arg("ws"), py::arg("S"), py::arg("residual") = c10::nullopt);
  m.def("peer_alloc", &bdllm::peer::alloc, "symmetric heap: zeroed device region");
  m.def("peer_handle", &bdllm::peer::handle, "CUDA IPC handle of a heap (64-byte CPU tensor)");
  m.def("peer_open", &bdllm::peer::open, "map a peer's heap from its IPC handle");
  m.def("peer_close", &bdllm::peer::close);
  m.def("peer_release", &bdllm::peer::release);
  m.def("peer_view", &bdllm::peer::view, "non-owning tensor over heap memory");
  m.def("peer_signal", &bdllm::peer::signal);
  m.def("peer_all_gather", &bdllm::peer::all_gather, "all-gather of heap shards by peer loads");
  m.def("peer_gather_range", &bdllm::peer::gather_range, "bytes [lo, hi) of a gathered buffer from the owning shards");
  m.def("peer_reduce_scatter", &bdllm::peer::reduce_scatter,
        "reduce-scatter by peer loads, fused fp32 cast, scale and sum of squares", py::arg("peers"),
        py::arg("rank"), py::arg("src_off"), py::arg("shard"), py::arg("in_f32"), py::arg("out"), py::arg("scale"),
        py::arg("sq"), py::arg("seq"), py::arg("max_blocks"), py::arg("timeout_s"),
        py::arg("adam_state") = std::vector<at::Tensor>{}, py::arg("adam_hp") = std::vector<double>{});
  m.def("peer_allreduce_f32", &bdllm::peer::allreduce_f32);
  m.def("bounds_report", &bdllm::bounds_report,
        "debug-bounds build: (file, line, index, limit, failures) per translation unit with a failed check",
        py::arg("reset") = true);
  m.def("debug_bounds_build", &bdllm::debug_bounds_build, "true in the -DBDLLM_DEBUG_BOUNDS extension (_C_dbg)");
  m.def("read_error_word", &bdllm::read_error_word, "device error word (bounded-wait expiries)",
        py::arg("reset") = false);
}
