// Python bindings of the lumenrl_b200._C extension.
#include <torch/extension.h>

#include "comm/comm_api.h"

#include <execinfo.h>
#include <fcntl.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <vector>

// Opt-in diagnostics (LRL_SEGV_BACKTRACE=1 in the tests): on SIGSEGV print the
// native call stack of this process's host code, then hand the signal to the
// handler that was installed before (Python's faulthandler).
namespace {
struct sigaction g_prev_segv;
int g_segv_fd = 2;
void lrl_segv_handler(int sig, siginfo_t* info, void* uctx) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  char head[160];
  const int len = snprintf(head, sizeof(head), "lumenrl_b200: signal %d, fault address %p; native stack:\n", sig,
                           info ? info->si_addr : nullptr);
  if (len > 0) (void)!write(g_segv_fd, head, (size_t)len);
  backtrace_symbols_fd(frames, n, g_segv_fd);
  sigaction(SIGSEGV, &g_prev_segv, nullptr);
  raise(sig);
}
// `path`: file the stack is appended to (test runners capture fd 2), "" = stderr
void install_segv_backtrace(const std::string& path) {
  if (!path.empty()) {
    const int fd = open(path.c_str(), O_WRONLY | O_CREAT | O_APPEND, 0644);
    if (fd >= 0) g_segv_fd = fd;
  }
  struct sigaction sa = {};
  sa.sa_sigaction = lrl_segv_handler;
  sa.sa_flags = SA_SIGINFO;
  sigemptyset(&sa.sa_mask);
  sigaction(SIGSEGV, &sa, &g_prev_segv);
}
}  // namespace

namespace lrl {
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                          c10::optional<torch::Tensor> dres);
std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                                            torch::Tensor inv_freq, int64_t nh, int64_t nkv, int64_t hd, double eps,
                                            c10::optional<torch::Tensor> kc, c10::optional<torch::Tensor> vc,
                                            c10::optional<torch::Tensor> slots, double inv_ks, double inv_vs);
torch::Tensor qk_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                               torch::Tensor qw, torch::Tensor kw, torch::Tensor pos, torch::Tensor inv_freq,
                               torch::Tensor rq, torch::Tensor rk, torch::Tensor dqw, torch::Tensor dkw, int64_t nh,
                               int64_t nkv, int64_t hd, double eps);
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor dh, torch::Tensor gu);
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor w16, double lr,
                double b1, double b2, double eps, double wd, int64_t step, double clip);
torch::Tensor sumsq(torch::Tensor x);
torch::Tensor group_adv(torch::Tensor r, int64_t G, bool unbiased, double eps);
std::vector<torch::Tensor> ppo_clip_fwd_bwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv,
                                            torch::Tensor mask, c10::optional<torch::Tensor> isw, double lo, double hi,
                                            double cc, double denom);
void logprob_fwd(torch::Tensor logits, torch::Tensor targets, double inv_t, torch::Tensor logp, torch::Tensor ent,
                 torch::Tensor lse);
void logprob_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor lse, torch::Tensor dlogp,
                 c10::optional<torch::Tensor> dent, double inv_t, c10::optional<torch::Tensor> ent);
std::vector<torch::Tensor> sample(torch::Tensor logits, double inv_t, double top_p, torch::Tensor row_seed,
                                  torch::Tensor step);
torch::Tensor paged_decode_attn(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                                torch::Tensor seq_lens, double scale, double k_scale, double v_scale,
                                int64_t max_len_hint);
torch::Tensor paged_decode_attn_shared(torch::Tensor q, torch::Tensor kc, torch::Tensor vc,
                                       torch::Tensor block_table, torch::Tensor seq_lens, torch::Tensor prefix_len,
                                       int64_t group, double scale, double k_scale, double v_scale,
                                       int64_t max_prefix_hint, int64_t max_suffix_hint);
torch::Tensor paged_decode_attn_tma(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                                    torch::Tensor seq_lens, double scale, double v_scale, int64_t max_len_hint);
torch::Tensor paged_decode_attn_shared_tma(torch::Tensor q, torch::Tensor kc, torch::Tensor vc,
                                           torch::Tensor block_table, torch::Tensor seq_lens,
                                           torch::Tensor prefix_len, int64_t group, double scale, double v_scale,
                                           int64_t max_prefix_hint, int64_t max_suffix_hint);
int64_t decode_tma_status();
std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu,
                                  int64_t max_seqlen, double scale, int64_t variant, bool causal);
int64_t fa_fwd_status();
std::vector<torch::Tensor> fa_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                  torch::Tensor out, torch::Tensor lse, torch::Tensor cu, int64_t max_seqlen,
                                  double scale, int64_t streams, int64_t variant, bool causal);
int64_t fa_bwd_status();
void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor kc, torch::Tensor vc, torch::Tensor slots,
               double inv_ks, double inv_vs);
torch::Tensor tc_gemm(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> c, int64_t epi, int64_t bn);
int64_t tc_gemm_status();
torch::Tensor tc_gemm_splitk(torch::Tensor a, torch::Tensor b, int64_t splits);
torch::Tensor gemm2sm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, c10::optional<torch::Tensor> c,
                      int64_t epi, int64_t bn);
int64_t gemm2sm_status();
std::vector<torch::Tensor> gemm2sm_logprob(torch::Tensor h, torch::Tensor w, torch::Tensor targets, double inv_t);
std::vector<torch::Tensor> ttt_diag_fwd(torch::Tensor q, torch::Tensor o0, torch::Tensor lse0,
                                        std::vector<torch::Tensor> kd, std::vector<torch::Tensor> vd, double scale);
std::vector<torch::Tensor> ttt_diag_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor out, torch::Tensor lse,
                                        std::vector<torch::Tensor> kd, std::vector<torch::Tensor> vd,
                                        torch::Tensor dq, double scale);
std::vector<torch::Tensor> fkl_fwd(torch::Tensor zt, torch::Tensor zd);
torch::Tensor skinny_sk(torch::Tensor x, torch::Tensor w, int64_t grid);
std::vector<torch::Tensor> moe_route(torch::Tensor logits, int64_t k, bool norm, c10::optional<torch::Tensor> replay);
torch::Tensor moe_route_bwd(torch::Tensor probs, torch::Tensor ids, torch::Tensor w, torch::Tensor dw,
                            c10::optional<torch::Tensor> dprobs, bool norm);
int64_t skinny_sk_status();
torch::Tensor skinny_fp8(torch::Tensor x, torch::Tensor qw, torch::Tensor sw, int64_t grid);
int64_t skinny_fp8_status();
void row_scale_(torch::Tensor x, torch::Tensor g);
torch::Tensor skinny_gemm(torch::Tensor x, torch::Tensor w, int64_t ksplit);
int64_t skinny_gemm_status();
torch::Tensor grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets);
int64_t grouped_gemm_status();
void tp_publish(std::vector<int64_t> sig_ptrs, int64_t rank, int64_t slot, int64_t epoch);
torch::Tensor ag_gemm(std::vector<int64_t> shard_ptrs, int64_t Ml, torch::Tensor b, std::vector<int64_t> sig_ptrs,
                      int64_t rank, int64_t slot, int64_t epoch, torch::Tensor status, int64_t wait_cycles);
torch::Tensor gemm_rs(torch::Tensor a, torch::Tensor b, std::vector<int64_t> recv_ptrs,
                      std::vector<int64_t> sig_ptrs, torch::Tensor counter, int64_t rank, int64_t slot, int64_t epoch,
                      torch::Tensor status, int64_t wait_cycles);
std::vector<torch::Tensor> quant_act_1x128(torch::Tensor x, bool e5m2);
std::vector<torch::Tensor> quant_weight_128x128(torch::Tensor w, bool e5m2);
std::vector<torch::Tensor> quant_t_1x128(torch::Tensor x, bool e5m2, bool kb_major);
torch::Tensor fp8_gemm_ex(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb,
                          c10::optional<torch::Tensor> c, bool b_row, torch::Tensor err);
torch::Tensor fp8_gemm(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, torch::Tensor err);
}  // namespace lrl

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  lrl::def_comm_ops(m);
  m.doc() = "lumenrl_b200 sm_100a kernels";
  m.def("install_segv_backtrace", &install_segv_backtrace, py::arg("path") = "");
  m.def("rmsnorm_fwd", &lrl::rmsnorm_fwd);
  m.def("add_rmsnorm_fwd", &lrl::add_rmsnorm_fwd);
  m.def("rmsnorm_bwd", &lrl::rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dw"),
        py::arg("dres") = py::none());
  m.def("qk_norm_rope_fwd", &lrl::qk_norm_rope_fwd, py::arg("qkv"), py::arg("qw"), py::arg("kw"), py::arg("pos"),
        py::arg("inv_freq"), py::arg("nh"), py::arg("nkv"), py::arg("hd"), py::arg("eps"), py::arg("kc") = py::none(),
        py::arg("vc") = py::none(), py::arg("slots") = py::none(), py::arg("inv_ks") = 1.0, py::arg("inv_vs") = 1.0);
  m.def("qk_norm_rope_bwd", &lrl::qk_norm_rope_bwd);
  m.def("swiglu_fwd", &lrl::swiglu_fwd);
  m.def("swiglu_bwd", &lrl::swiglu_bwd);
  m.def("adamw_step", &lrl::adamw_step);
  m.def("sumsq", &lrl::sumsq);
  m.def("group_adv", &lrl::group_adv);
  m.def("ppo_clip_fwd_bwd", &lrl::ppo_clip_fwd_bwd, py::arg("logp"), py::arg("old"), py::arg("adv"), py::arg("mask"),
        py::arg("isw"), py::arg("lo"), py::arg("hi"), py::arg("cc"), py::arg("denom"));
  m.def("logprob_fwd", &lrl::logprob_fwd);
  m.def("logprob_bwd", &lrl::logprob_bwd, py::arg("logits"), py::arg("targets"), py::arg("lse"), py::arg("dlogp"),
        py::arg("dent"), py::arg("inv_t"), py::arg("ent") = py::none());
  m.def("sample", &lrl::sample);
  m.def("paged_decode_attn", &lrl::paged_decode_attn, py::arg("q"), py::arg("kc"), py::arg("vc"),
        py::arg("block_table"), py::arg("seq_lens"), py::arg("scale"), py::arg("k_scale") = 1.0,
        py::arg("v_scale") = 1.0, py::arg("max_len_hint") = 0);
  m.def("paged_decode_attn_shared", &lrl::paged_decode_attn_shared, py::arg("q"), py::arg("kc"), py::arg("vc"),
        py::arg("block_table"), py::arg("seq_lens"), py::arg("prefix_len"), py::arg("group"), py::arg("scale"),
        py::arg("k_scale") = 1.0, py::arg("v_scale") = 1.0, py::arg("max_prefix_hint") = 0,
        py::arg("max_suffix_hint") = 0);
  m.def("paged_decode_attn_tma", &lrl::paged_decode_attn_tma);
  m.def("paged_decode_attn_shared_tma", &lrl::paged_decode_attn_shared_tma);
  m.def("decode_tma_status", &lrl::decode_tma_status);
  m.def("fa_fwd", &lrl::fa_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu"), py::arg("max_seqlen"),
        py::arg("scale"), py::arg("variant") = -1, py::arg("causal") = true);
  m.def("fa_fwd_status", &lrl::fa_fwd_status);
  m.def("fa_bwd", &lrl::fa_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"),
        py::arg("lse"), py::arg("cu"), py::arg("max_seqlen"), py::arg("scale"), py::arg("streams") = 1, py::arg("variant") = -1,
        py::arg("causal") = true);
  m.def("fa_bwd_status", &lrl::fa_bwd_status);
  m.def("kv_append", &lrl::kv_append);
  m.def("tc_gemm", &lrl::tc_gemm, py::arg("a"), py::arg("b"), py::arg("c") = py::none(), py::arg("epi") = 0,
        py::arg("bn") = 0);
  m.def("tc_gemm_status", &lrl::tc_gemm_status);
  m.def("tc_gemm_splitk", &lrl::tc_gemm_splitk, py::arg("a"), py::arg("b"), py::arg("splits") = 0);
  m.def("gemm2sm", &lrl::gemm2sm, py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"),
        py::arg("c") = py::none(), py::arg("epi") = 0, py::arg("bn") = 0);
  m.def("gemm2sm_status", &lrl::gemm2sm_status);
  m.def("gemm2sm_logprob", &lrl::gemm2sm_logprob);
  m.def("ttt_diag_fwd", &lrl::ttt_diag_fwd);
  m.def("ttt_diag_bwd", &lrl::ttt_diag_bwd);
  m.def("fkl_fwd", &lrl::fkl_fwd);
  m.def("skinny_sk", &lrl::skinny_sk, py::arg("x"), py::arg("w"), py::arg("grid") = 0);
  m.def("skinny_sk_status", &lrl::skinny_sk_status);
  m.def("skinny_fp8", &lrl::skinny_fp8, py::arg("x"), py::arg("qw"), py::arg("sw"), py::arg("grid") = 0);
  m.def("skinny_fp8_status", &lrl::skinny_fp8_status);
  m.def("moe_route", &lrl::moe_route, py::arg("logits"), py::arg("k"), py::arg("norm"), py::arg("replay") = py::none());
  m.def("moe_route_bwd", &lrl::moe_route_bwd, py::arg("probs"), py::arg("ids"), py::arg("w"), py::arg("dw"),
        py::arg("dprobs") = py::none(), py::arg("norm") = true);
  m.def("row_scale_", &lrl::row_scale_);
  m.def("skinny_gemm", &lrl::skinny_gemm, py::arg("x"), py::arg("w"), py::arg("ksplit") = 0);
  m.def("skinny_gemm_status", &lrl::skinny_gemm_status);
  m.def("grouped_gemm", &lrl::grouped_gemm);
  m.def("grouped_gemm_status", &lrl::grouped_gemm_status);
  m.def("tp_publish", &lrl::tp_publish);
  m.def("ag_gemm", &lrl::ag_gemm);
  m.def("gemm_rs", &lrl::gemm_rs);
  m.def("quant_act_1x128", &lrl::quant_act_1x128);
  m.def("quant_weight_128x128", &lrl::quant_weight_128x128);
  m.def("quant_t_1x128", &lrl::quant_t_1x128, py::arg("x"), py::arg("e5m2") = false, py::arg("kb_major") = false);
  m.def(
      "fp8_gemm_ex",
      [](torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, torch::Tensor err,
         c10::optional<torch::Tensor> c, bool b_row) { return lrl::fp8_gemm_ex(a, sa, b, sb, c, b_row, err); },
      py::arg("a"), py::arg("sa"), py::arg("b"), py::arg("sb"), py::arg("err"), py::arg("c") = py::none(),
      py::arg("b_row") = false);
  m.def("fp8_gemm", &lrl::fp8_gemm);
}
