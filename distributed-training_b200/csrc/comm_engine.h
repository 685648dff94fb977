// Host-side state of one NVLink process group (see comm.cu).
#pragma once

#include <torch/extension.h>

#include <cstdint>
#include <vector>

namespace dtb {

class CommEngine {
 public:
  CommEngine(int64_t rank, int64_t world, std::vector<int64_t> sigs, double timeout_s, int64_t blocks);

  // Every rank registers the same buffers in the same order (collective).  `mc_ptr`
  // is the buffer's NVSwitch multicast address (0: not multicast-mapped).
  int64_t register_buffer(std::vector<int64_t> ptrs, int64_t nbytes, int64_t mc_ptr = 0);
  void forget_buffers();
  bool has_multicast(torch::Tensor t) const;
  bool contains(torch::Tensor t) const;
  std::vector<int64_t> peer_ptrs(torch::Tensor t) const;

  // In-place two-shot all-reduce of a tensor inside a registered buffer; returns the
  // CTA count.  `blocks` 0 sizes the grid by the message; `lean` selects the
  // 128-thread CTAs that run beside a GEMM; with `sq_pad` (an fp64 registered
  // buffer of world * sq_stride slots) CTA b also publishes the sum of squares of
  // its reduced slice into slot [rank * sq_stride + sq_base + b] of every rank's pad.
  int64_t allreduce_inplace(torch::Tensor t, int64_t order, double scale, int64_t blocks, bool lean,
                            c10::optional<torch::Tensor> sq_pad, int64_t sq_base, int64_t sq_stride);
  // In-place all-reduce through the switch (multimem.ld_reduce + multimem.st) of a
  // tensor in a multicast-mapped buffer; same lean and sum-of-squares options as above.
  int64_t allreduce_nvls(torch::Tensor t, double scale, int64_t blocks, bool lean,
                         c10::optional<torch::Tensor> sq_pad, int64_t sq_base, int64_t sq_stride);
  // Reduce-scatter through the switch (fp32); returns this rank's partition.
  torch::Tensor reduce_scatter_nvls(torch::Tensor flat, double scale, int64_t sq_part_ptr, int64_t blocks);
  // Returns this rank's partition of `flat` (holding the reduced values).
  torch::Tensor reduce_scatter(torch::Tensor flat, int64_t order, double scale, int64_t sq_part_ptr, int64_t blocks);
  void all_gather(torch::Tensor flat);
  void barrier();

  // Collectives issued through this engine (host count; graph replays not included).
  int64_t issued() const { return issued_; }
  void note_issued() { ++issued_; }
  // The rank's device epoch counter (synchronous read: for tests and diagnostics).
  int64_t device_epoch() const;
  double timeout() const { return timeout_; }
  void set_timeout(double t) { timeout_ = t; }
  int64_t blocks() const { return blocks_; }

 private:
  bool locate(const torch::Tensor& t, int64_t& id, int64_t& off) const;

  int64_t rank_, world_;
  std::vector<int64_t> sigs_;
  double timeout_;
  int64_t blocks_;
  int64_t issued_ = 0;
  std::vector<std::vector<int64_t>> bufs_;
  std::vector<int64_t> sizes_;
  std::vector<int64_t> mcs_;
};

}  // namespace dtb
