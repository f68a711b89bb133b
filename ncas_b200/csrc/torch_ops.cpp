// torch_ops.cpp -- the C ABI of libnca_b200 (include/nca_b200.h) registered as torch operators
// (torch.ops.nca_b200.*), so that the rollout's kernels are dispatched by torch on its current
// CUDA stream and raise Python exceptions on failure.
//
// The descriptors of the C ABI (NcaModelDesc, NcaBatchDesc, NcaState, NcaFireDesc) travel as CPU
// uint8 tensors that hold the structs' bytes (ncas_b200.engine builds them with ctypes and views
// them with torch.frombuffer, so an operator that updates a state updates the caller's struct).
// Device buffers are CUDA tensors.  Every operator checks the NcaStatus of its call and raises a
// RuntimeError naming the status.
#include <ATen/cuda/CUDAContext.h>
#include <torch/library.h>

#include <optional>
#include <string>

#include "../../include/nca_b200.h"

namespace {

template <class T>
T* desc(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == at::kByte && t.is_contiguous(), name,
              " must be a contiguous CPU uint8 tensor holding the struct");
  TORCH_CHECK((size_t)t.numel() == sizeof(T), name, " has ", t.numel(), " bytes, the struct ",
              sizeof(T));
  return reinterpret_cast<T*>(t.data_ptr());
}

void* dptr(const at::Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "device buffers must be contiguous CUDA tensors");
  return t.data_ptr();
}
void* dptr(const std::optional<at::Tensor>& t) { return t.has_value() ? dptr(*t) : nullptr; }

void* stream() { return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

void check(int32_t status, const char* what) {
  TORCH_CHECK(status == NCA_OK, what, ": ", nca_b200_status_string(status), " (status ", status, ")");
}

void op_state_init(const at::Tensor& state, const at::Tensor& model, const at::Tensor& batch) {
  check(nca_b200_state_init(desc<NcaState>(state, "state"), desc<NcaModelDesc>(model, "model"),
                            desc<NcaBatchDesc>(batch, "batch"), stream()),
        "nca_b200_state_init");
}

void op_load_nchw(const at::Tensor& state, const at::Tensor& x) {
  check(nca_b200_state_load_nchw(desc<NcaState>(state, "state"), static_cast<const float*>(dptr(x)),
                                 stream()),
        "nca_b200_state_load_nchw");
}

void op_store_nchw(const at::Tensor& state, const at::Tensor& out) {
  check(nca_b200_state_store_nchw(desc<NcaState>(state, "state"), static_cast<float*>(dptr(out)),
                                  stream()),
        "nca_b200_state_store_nchw");
}

void op_run_steps(const at::Tensor& model, const at::Tensor& batch, const at::Tensor& state,
               int64_t n_steps, const at::Tensor& fire, const at::Tensor& ctrl, int64_t timeout_ms) {
  check(nca_b200_run_steps(desc<NcaModelDesc>(model, "model"), desc<NcaBatchDesc>(batch, "batch"),
                           desc<NcaState>(state, "state"), (int32_t)n_steps,
                           desc<NcaFireDesc>(fire, "fire"), static_cast<int32_t*>(dptr(ctrl)),
                           (int32_t)timeout_ms, stream()),
        "nca_b200_run_steps");
}

void op_readout(const at::Tensor& model, const at::Tensor& batch, const at::Tensor& state,
             const std::optional<at::Tensor>& pred, const std::optional<at::Tensor>& cell_conf,
             const at::Tensor& board_conf, const std::optional<at::Tensor>& targets,
             const std::optional<at::Tensor>& cell_acc, const std::optional<at::Tensor>& exact) {
  check(nca_b200_readout(desc<NcaModelDesc>(model, "model"), desc<NcaBatchDesc>(batch, "batch"),
                         desc<NcaState>(state, "state"), static_cast<uint8_t*>(dptr(pred)),
                         static_cast<float*>(dptr(cell_conf)), static_cast<float*>(dptr(board_conf)),
                         static_cast<const uint8_t*>(dptr(targets)), static_cast<float*>(dptr(cell_acc)),
                         static_cast<uint8_t*>(dptr(exact)), stream()),
        "nca_b200_readout");
}

void op_select(const at::Tensor& board_conf, const std::optional<at::Tensor>& alive, int64_t n_boards,
            int64_t trials, int64_t k_limit, const at::Tensor& best_idx, const at::Tensor& best_conf,
            const std::optional<at::Tensor>& pred, int64_t hw, const std::optional<at::Tensor>& best_pred) {
  check(nca_b200_select(static_cast<const float*>(dptr(board_conf)), static_cast<const uint8_t*>(dptr(alive)),
                        (int32_t)n_boards, (int32_t)trials, (int32_t)k_limit,
                        static_cast<int32_t*>(dptr(best_idx)), static_cast<float*>(dptr(best_conf)),
                        static_cast<const uint8_t*>(dptr(pred)), (int32_t)hw,
                        static_cast<uint8_t*>(dptr(best_pred)), stream()),
        "nca_b200_select");
}

void op_prune_refill(const at::Tensor& pred, const at::Tensor& board_conf, int64_t n_boards, int64_t trials,
                  int64_t hw, int64_t n_cap, const at::Tensor& src, const at::Tensor& kept) {
  check(nca_b200_prune_refill(static_cast<const uint8_t*>(dptr(pred)), static_cast<const float*>(dptr(board_conf)),
                              (int32_t)n_boards, (int32_t)trials, (int32_t)hw, (int32_t)n_cap,
                              static_cast<int32_t*>(dptr(src)), static_cast<uint8_t*>(dptr(kept)), stream()),
        "nca_b200_prune_refill");
}

void op_clone(const at::Tensor& state, const at::Tensor& src) {
  check(nca_b200_clone(desc<NcaState>(state, "state"), static_cast<const int32_t*>(dptr(src)), stream()),
        "nca_b200_clone");
}

void op_damage(const at::Tensor& model, const at::Tensor& batch, const at::Tensor& state,
            const at::Tensor& masks) {
  check(nca_b200_damage(desc<NcaModelDesc>(model, "model"), desc<NcaBatchDesc>(batch, "batch"),
                        desc<NcaState>(state, "state"), static_cast<const uint8_t*>(dptr(masks)), stream()),
        "nca_b200_damage");
}

void op_niches(const at::Tensor& pred, const at::Tensor& board_conf, const at::Tensor& row_start,
            int64_t n_boards, int64_t max_rows, int64_t hw, const at::Tensor& niche, const at::Tensor& rank,
            const at::Tensor& n_niches) {
  check(nca_b200_niches(static_cast<const uint8_t*>(dptr(pred)), static_cast<const float*>(dptr(board_conf)),
                        static_cast<const int32_t*>(dptr(row_start)), (int32_t)n_boards, (int32_t)max_rows,
                        (int32_t)hw, static_cast<int32_t*>(dptr(niche)), static_cast<int32_t*>(dptr(rank)),
                        static_cast<int32_t*>(dptr(n_niches)), stream()),
        "nca_b200_niches");
}

void op_halving(const at::Tensor& niche, const at::Tensor& rank, const at::Tensor& n_niches,
             const at::Tensor& row_start, const at::Tensor& order, const at::Tensor& order_start,
             int64_t n_boards, int64_t max_rows, int64_t n_cap, const at::Tensor& keep) {
  check(nca_b200_halving(static_cast<const int32_t*>(dptr(niche)), static_cast<const int32_t*>(dptr(rank)),
                         static_cast<const int32_t*>(dptr(n_niches)), static_cast<const int32_t*>(dptr(row_start)),
                         static_cast<const int32_t*>(dptr(order)), static_cast<const int32_t*>(dptr(order_start)),
                         (int32_t)n_boards, (int32_t)max_rows, (int32_t)n_cap,
                         static_cast<uint8_t*>(dptr(keep)), stream()),
        "nca_b200_halving");
}

void op_gather(const at::Tensor& src_state, const at::Tensor& dst_state, const at::Tensor& sel) {
  check(nca_b200_gather(desc<NcaState>(src_state, "src"), desc<NcaState>(dst_state, "dst"),
                        static_cast<const int32_t*>(dptr(sel)), stream()),
        "nca_b200_gather");
}

// Synchronises the current stream and returns the first kernel-side failure as
// [status, site] (0, 0 when none); the control words are cleared when a failure is returned.
std::vector<int64_t> op_ctrl_status(const at::Tensor& ctrl) {
  int32_t detail = 0;
  const int32_t s = nca_b200_ctrl_status(static_cast<int32_t*>(dptr(ctrl)), &detail, stream());
  return {s, detail};
}

}  // namespace

TORCH_LIBRARY(nca_b200, m) {
  m.def("state_init(Tensor state, Tensor model, Tensor batch) -> ()", &op_state_init);
  m.def("load_nchw(Tensor state, Tensor x) -> ()", &op_load_nchw);
  m.def("store_nchw(Tensor state, Tensor(a!) out) -> ()", &op_store_nchw);
  m.def("run_steps(Tensor model, Tensor batch, Tensor state, int n_steps, Tensor fire, Tensor(a!) ctrl, "
        "int timeout_ms) -> ()",
        &op_run_steps);
  m.def("readout(Tensor model, Tensor batch, Tensor state, Tensor(a!)? pred, Tensor(b!)? cell_conf, "
        "Tensor(c!) board_conf, Tensor? targets, Tensor(d!)? cell_acc, Tensor(e!)? exact) -> ()",
        &op_readout);
  m.def("select(Tensor board_conf, Tensor? alive, int n_boards, int trials, int k_limit, "
        "Tensor(a!) best_idx, Tensor(b!) best_conf, Tensor? pred, int hw, Tensor(c!)? best_pred) -> ()",
        &op_select);
  m.def("prune_refill(Tensor pred, Tensor board_conf, int n_boards, int trials, int hw, int n_cap, "
        "Tensor(a!) src, Tensor(b!) kept) -> ()",
        &op_prune_refill);
  m.def("clone(Tensor state, Tensor src) -> ()", &op_clone);
  m.def("damage(Tensor model, Tensor batch, Tensor state, Tensor masks) -> ()", &op_damage);
  m.def("niches(Tensor pred, Tensor board_conf, Tensor row_start, int n_boards, int max_rows, int hw, "
        "Tensor(a!) niche, Tensor(b!) rank, Tensor(c!) n_niches) -> ()",
        &op_niches);
  m.def("halving(Tensor niche, Tensor rank, Tensor n_niches, Tensor row_start, Tensor order, "
        "Tensor order_start, int n_boards, int max_rows, int n_cap, Tensor(a!) keep) -> ()",
        &op_halving);
  m.def("gather(Tensor src_state, Tensor dst_state, Tensor sel) -> ()", &op_gather);
  m.def("ctrl_status(Tensor(a!) ctrl) -> int[]", &op_ctrl_status);
}
