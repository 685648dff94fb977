// Python bindings for the sm_100a kernels (one extension module, `_C`).
#include <torch/extension.h>
#include <atomic>

#include "comm_engine.h"

namespace dtb {

static std::atomic<long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

// gemm.cu
void gemm(torch::Tensor a, bool a_trans, torch::Tensor b, bool b_trans, torch::Tensor out, int64_t epi,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> aux,
          double alpha, bool accumulate, int64_t force_bn, int64_t force_splits,
          c10::optional<torch::Tensor> workspace);
torch::Tensor gemm_gather(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi,
                          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> resid,
                          c10::optional<torch::Tensor> aux, std::vector<int64_t> peers, int64_t rank, int64_t woff,
                          int64_t nflat, torch::Tensor state, int64_t site);
torch::Tensor gemm_lse(torch::Tensor a, torch::Tensor b, torch::Tensor out);
std::vector<int64_t> gemm_tiling(int64_t M, int64_t N, int64_t K);
// layernorm.cu
std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps);
torch::Tensor layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                            torch::Tensor rstd, c10::optional<torch::Tensor> dresid, torch::Tensor dw,
                            torch::Tensor db, bool accumulate, c10::optional<torch::Tensor> dres_sum);
void bias_grad(torch::Tensor g, torch::Tensor db, bool accumulate);
// embed_xent.cu
torch::Tensor embed_fwd(torch::Tensor idx, torch::Tensor tok, torch::Tensor pos, torch::Tensor bad_flag);
void embed_bwd(torch::Tensor idx, torch::Tensor dx, torch::Tensor dtok, torch::Tensor dpos, int64_t B, int64_t T,
               bool accumulate);
std::vector<torch::Tensor> sort_ids(torch::Tensor idx, int64_t V);
std::vector<torch::Tensor> xent_fwd(torch::Tensor logits, torch::Tensor tgt);
std::vector<torch::Tensor> xent_from_parts(torch::Tensor part, torch::Tensor logits, torch::Tensor tgt);
void xent_bwd(torch::Tensor logits, torch::Tensor tgt, torch::Tensor lse, torch::Tensor gscale);
// optim.cu
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double b1, double b2, double eps, double wd, int64_t t, c10::optional<torch::Tensor> sq,
                double max_norm);
void grad_sqnorm(torch::Tensor g, torch::Tensor out, double scale);
void cast_f32_bf16(torch::Tensor x, torch::Tensor y);
void scale_f32(torch::Tensor x, double s);
// attention.cu
std::vector<torch::Tensor> attn_fwd(torch::Tensor qkv, int64_t B, int64_t T, int64_t H, int64_t D, bool legacy);
torch::Tensor attn_bwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, int64_t B,
                       int64_t T, int64_t H, int64_t D, bool legacy);
// comm.cu
std::tuple<int64_t, torch::Tensor> symm_alloc(int64_t nbytes);
int64_t symm_open(torch::Tensor handle);
void symm_close(int64_t peer_ptr);
void symm_free(int64_t ptr);
torch::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> sizes, c10::ScalarType dtype, int64_t device);
// vmm.cpp
std::tuple<int64_t, int64_t, int64_t> vmm_alloc(int64_t nbytes);
int64_t vmm_import(int64_t fd, int64_t size);
void vmm_free(int64_t va);
void comm_abort_prepare();
void comm_abort(int64_t own_sig_ptr);
bool mc_supported();
int64_t mc_granularity(int64_t ndev);
std::tuple<int64_t, int64_t> mc_create(int64_t size, int64_t ndev);
int64_t mc_import(int64_t fd);
void mc_add_device(int64_t mc);
void mc_release(int64_t mc);
int64_t mc_bind_map(int64_t mc, int64_t local_va, int64_t size, int64_t ndev);
void mc_free(int64_t mc_va);
int64_t comm_status();
void comm_status_clear();
int64_t allreduce(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset, int64_t n,
                  int64_t in_dtype, int64_t out_ptr, int64_t out_dtype, int64_t algo, int64_t order, double scale,
                  double timeout_s, int64_t blocks, bool lean, std::vector<int64_t> sq_pads, int64_t sq_base,
                  int64_t sq_stride);
int64_t collective_blocks(int64_t nbytes, int64_t want, bool lean);
void stamp(torch::Tensor buf, int64_t slot);
void sq_total(torch::Tensor pad, torch::Tensor out, int64_t world, int64_t stride, int64_t lo, int64_t hi);
int64_t reduce_scatter(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset,
                       int64_t n, int64_t dtype, int64_t out_ptr, int64_t order, double scale, int64_t sq_part_ptr,
                       double timeout_s, int64_t blocks);
int64_t all_gather(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset, int64_t n,
                   int64_t dtype, double timeout_s, int64_t blocks);
int64_t broadcast(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset,
                  int64_t nbytes, int64_t root, int64_t cast_src, int64_t out16, int64_t n16, double timeout_s,
                  int64_t blocks);
int64_t device_barrier(std::vector<int64_t> sigs, int64_t rank, double timeout_s);
int64_t zero_rs_adamw(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> grads,
                      std::vector<int64_t> sq_parts, torch::Tensor master, torch::Tensor m, torch::Tensor v,
                      std::vector<int64_t> work16, std::vector<int64_t> master32, int64_t n, double lr, double b1,
                      double b2, double eps, double wd, int64_t t, double scale, double max_norm,
                      c10::optional<torch::Tensor> sq_out, bool gather_master, double timeout_s, int64_t blocks,
                      c10::optional<torch::Tensor> keep, c10::optional<torch::Tensor> gen_word);
int64_t zero_adamw_allgather(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> sq_parts, int64_t nparts,
                             torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v,
                             std::vector<int64_t> work16, std::vector<int64_t> master32, int64_t n, double lr,
                             double b1, double b2, double eps, double wd, int64_t t, double max_norm,
                             c10::optional<torch::Tensor> sq_out, bool gather_master, double timeout_s,
                             int64_t blocks, c10::optional<torch::Tensor> keep, c10::optional<torch::Tensor> gen_word);
int64_t comm_max_blocks();
int64_t comm_max_ranks();

int status_gemm();
int status_layernorm();
int status_embed_xent();
int status_optim();
int status_attention();
int status_comm();
int status_attention_tc();

// First non-zero device status word over all kernel files (and clears them).
int64_t device_status() {
  int codes[] = {status_gemm(), status_layernorm(), status_embed_xent(), status_optim(), status_attention(),
                 status_comm(), status_attention_tc()};
  for (int c : codes)
    if (c) return c;
  return 0;
}

}  // namespace dtb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace dtb;
  namespace py = pybind11;
  m.def("launch_count", &launch_count);
  m.def("device_status", &device_status);
  m.def("gemm", &gemm, py::arg("a"), py::arg("a_trans"), py::arg("b"), py::arg("b_trans"), py::arg("out"),
        py::arg("epi"), py::arg("bias") = py::none(), py::arg("resid") = py::none(), py::arg("aux") = py::none(),
        py::arg("alpha") = 1.0, py::arg("accumulate") = false, py::arg("force_bn") = 0, py::arg("force_splits") = 0,
        py::arg("workspace") = py::none());
  m.def("gemm_gather", &gemm_gather, py::arg("a"), py::arg("b"), py::arg("out"), py::arg("epi"),
        py::arg("bias") = py::none(), py::arg("resid") = py::none(), py::arg("aux") = py::none(), py::arg("peers"),
        py::arg("rank"), py::arg("woff"), py::arg("nflat"), py::arg("state"), py::arg("site"));
  m.def("gemm_lse", &gemm_lse);
  m.def("xent_from_parts", &xent_from_parts);
  m.def("gemm_tiling", &gemm_tiling);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("mean"),
        py::arg("rstd"), py::arg("dresid"), py::arg("dw"), py::arg("db"), py::arg("accumulate") = false,
        py::arg("dres_sum") = py::none());
  m.def("bias_grad", &bias_grad);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("sort_ids", &sort_ids);
  m.def("xent_fwd", &xent_fwd);
  m.def("xent_bwd", &xent_bwd);
  m.def("adamw_step", &adamw_step);
  m.def("grad_sqnorm", &grad_sqnorm);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("scale_f32", &scale_f32);
  m.def("attn_fwd", &attn_fwd, py::arg("qkv"), py::arg("B"), py::arg("T"), py::arg("H"), py::arg("D"),
        py::arg("legacy") = false);
  m.def("attn_bwd", &attn_bwd, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"), py::arg("B"),
        py::arg("T"), py::arg("H"), py::arg("D"), py::arg("legacy") = false);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("vmm_alloc", &vmm_alloc);
  m.def("vmm_import", &vmm_import);
  m.def("vmm_free", &vmm_free);
  m.def("mc_supported", &mc_supported);
  m.def("mc_granularity", &mc_granularity);
  m.def("mc_create", &mc_create);
  m.def("mc_import", &mc_import);
  m.def("mc_add_device", &mc_add_device);
  m.def("mc_release", &mc_release);
  m.def("mc_bind_map", &mc_bind_map);
  m.def("mc_free", &mc_free);
  m.def("comm_status", &comm_status);
  m.def("comm_status_clear", &comm_status_clear);
  m.def("comm_abort_prepare", &comm_abort_prepare);
  m.def("comm_abort", &comm_abort);
  m.def("allreduce", &allreduce);
  m.def("collective_blocks", &collective_blocks);
  m.def("sq_total", &sq_total);
  m.def("stamp", &stamp);
  m.def("reduce_scatter", &reduce_scatter);
  m.def("all_gather", &all_gather);
  m.def("broadcast", &broadcast);
  m.def("device_barrier", &device_barrier);
  m.def("zero_adamw_allgather", &zero_adamw_allgather);
  m.def("zero_rs_adamw", &zero_rs_adamw);
  m.def("comm_max_blocks", &comm_max_blocks);
  py::class_<CommEngine>(m, "CommEngine")
      .def(py::init<int64_t, int64_t, std::vector<int64_t>, double, int64_t>())
      .def("register_buffer", &CommEngine::register_buffer, py::arg("ptrs"), py::arg("nbytes"), py::arg("mc_ptr") = 0)
      .def("has_multicast", &CommEngine::has_multicast)
      .def("allreduce_nvls", &CommEngine::allreduce_nvls, py::arg("t"), py::arg("scale"), py::arg("blocks"),
           py::arg("lean"), py::arg("sq_pad"), py::arg("sq_base"), py::arg("sq_stride"))
      .def("reduce_scatter_nvls", &CommEngine::reduce_scatter_nvls)
      .def("forget_buffers", &CommEngine::forget_buffers)
      .def("contains", &CommEngine::contains)
      .def("peer_ptrs", &CommEngine::peer_ptrs)
      .def("allreduce_inplace", &CommEngine::allreduce_inplace, py::arg("t"), py::arg("order"), py::arg("scale"),
           py::arg("blocks") = 0, py::arg("lean") = false, py::arg("sq_pad") = py::none(), py::arg("sq_base") = 0,
           py::arg("sq_stride") = 0)
      .def("reduce_scatter", &CommEngine::reduce_scatter)
      .def("all_gather", &CommEngine::all_gather)
      .def("barrier", &CommEngine::barrier)
      .def("note_issued", &CommEngine::note_issued)
      .def_property_readonly("issued", &CommEngine::issued)
      .def("device_epoch", &CommEngine::device_epoch)
      .def_property("timeout", &CommEngine::timeout, &CommEngine::set_timeout)
      .def_property_readonly("blocks", &CommEngine::blocks);
  m.def("comm_max_ranks", &comm_max_ranks);
}
