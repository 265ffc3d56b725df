// Host entry points of the NVLink communication kernels (csrc/comm/*.cu) and
// their Python bindings.  Both extension modules bind them with def_comm_ops:
// lumenrl_b200._C (ordinary build) and lumenrl_b200._C_bounds (the same
// sources compiled with -DLRL_DEBUG_BOUNDS, every peer access checked).
#pragma once

#include <torch/extension.h>

#include <vector>

namespace lrl {

// symmetric buffers over CUDA IPC
std::vector<int64_t> symm_malloc(int64_t nbytes);
int64_t symm_open(std::vector<int64_t> handle_words);
void symm_close(int64_t ptr);
void symm_free(int64_t ptr);
torch::Tensor symm_tensor(int64_t ptr, int64_t numel, torch::ScalarType dtype);
int64_t symm_signal_words();

// fused optimizer collectives and the replicated-DP all-reduce
void rs_norm(std::vector<int64_t> grad_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
             torch::Tensor out, int64_t epoch, torch::Tensor status, int64_t wait_cycles);
void adamw_ag(std::vector<int64_t> weight_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
              torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1, double b2,
              double eps, double wd, int64_t step, double max_norm, int64_t epoch, torch::Tensor status,
              torch::Tensor norm_out, int64_t wait_cycles);
void rs_norm_mc(int64_t mc_grads, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
                torch::Tensor out, int64_t epoch, torch::Tensor status, int64_t wait_cycles);
void adamw_ag_mc(int64_t mc_weights, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t lo, int64_t n,
                 torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1, double b2,
                 double eps, double wd, int64_t step, double max_norm, int64_t epoch, torch::Tensor status,
                 torch::Tensor norm_out, int64_t wait_cycles);
void nvlink_allreduce(std::vector<int64_t> buf_ptrs, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t n,
                      double scale, int64_t epoch, torch::Tensor status, int64_t wait_cycles);
void nvlink_allreduce_mc(int64_t mc_buf, std::vector<int64_t> sig_ptrs, int64_t rank, int64_t n, double scale,
                         int64_t epoch, torch::Tensor status, int64_t wait_cycles);

// point-to-point pushes
void p2p_push(torch::Tensor src, int64_t dst_ptr, int64_t ready_flag_ptr, int64_t epoch, torch::Tensor counter);
void p2p_wait(int64_t flag_ptr, int64_t epoch, torch::Tensor status, int64_t tag, int64_t wait_cycles);
void p2p_signal(int64_t flag_ptr, int64_t epoch);

// expert-parallel token exchange
int64_t ep_flag_slots();
void ep_exchange_counts(torch::Tensor counts, std::vector<int64_t> table_ptrs, std::vector<int64_t> sig_ptrs,
                        int64_t rank, int64_t slot, int64_t epoch, torch::Tensor status, int64_t wait_cycles);
void ep_scatter_rows(torch::Tensor src, c10::optional<torch::Tensor> src_row, torch::Tensor dst_rank,
                     torch::Tensor dst_row, std::vector<int64_t> buf_ptrs, int64_t cap,
                     std::vector<int64_t> sig_ptrs, int64_t rank, int64_t slot, int64_t epoch, torch::Tensor counter,
                     torch::Tensor status);
void ep_wait_all(int64_t my_sig_ptr, int64_t W, int64_t slot, int64_t epoch, torch::Tensor status,
                 int64_t wait_cycles);

// bounds registry and status (bounds.cuh)
void bounds_register(int64_t ptr, int64_t bytes);
void bounds_unregister(int64_t ptr);
std::vector<int64_t> bounds_lookup(int64_t ptr);
int64_t bounds_status();
void bounds_reset();
bool debug_bounds_build();

inline void def_comm_ops(pybind11::module_& m) {
  m.def("symm_malloc", &symm_malloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("symm_tensor", &symm_tensor);
  m.def("symm_signal_words", &symm_signal_words);
  m.def("rs_norm", &rs_norm);
  m.def("adamw_ag", &adamw_ag);
  m.def("rs_norm_mc", &rs_norm_mc);
  m.def("adamw_ag_mc", &adamw_ag_mc);
  m.def("nvlink_allreduce", &nvlink_allreduce);
  m.def("nvlink_allreduce_mc", &nvlink_allreduce_mc);
  m.def("p2p_push", &p2p_push);
  m.def("p2p_wait", &p2p_wait);
  m.def("p2p_signal", &p2p_signal);
  m.def("ep_flag_slots", &ep_flag_slots);
  m.def("ep_exchange_counts", &ep_exchange_counts);
  m.def("ep_scatter_rows", &ep_scatter_rows);
  m.def("ep_wait_all", &ep_wait_all);
  m.def("bounds_register", &bounds_register);
  m.def("bounds_unregister", &bounds_unregister);
  m.def("bounds_lookup", &bounds_lookup);
  m.def("bounds_status", &bounds_status);
  m.def("bounds_reset", &bounds_reset);
  m.def("debug_bounds_build", &debug_bounds_build);
}

}  // namespace lrl
