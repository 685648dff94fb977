// Host-side state of one NVLink process group (see comm.cu).
#pragma once

#include <torch/extension.h>

#include <cstdint>
#include <vector>

namespace dtb {

class CommEngine {
 public:
  CommEngine(int64_t rank, int64_t world, std::vector<int64_t> sigs, double timeout_s, int64_t blocks);

  // Every rank registers the same buffers in the same order (collective).
  int64_t register_buffer(std::vector<int64_t> ptrs, int64_t nbytes);
  void forget_buffers();
  bool contains(torch::Tensor t) const;
  std::vector<int64_t> peer_ptrs(torch::Tensor t) const;

  // In-place two-shot all-reduce of a tensor inside a registered buffer.
  void allreduce_inplace(torch::Tensor t, int64_t order, double scale);
  // Returns this rank's partition of `flat` (holding the reduced values).
  torch::Tensor reduce_scatter(torch::Tensor flat, int64_t order, double scale, int64_t sq_part_ptr, int64_t blocks);
  void all_gather(torch::Tensor flat);
  void barrier();

  int64_t epoch() const { return epoch_; }
  void advance(int64_t n) { epoch_ += n; }
  double timeout() const { return timeout_; }
  void set_timeout(double t) { timeout_ = t; }
  int64_t blocks() const { return blocks_; }

 private:
  bool locate(const torch::Tensor& t, int64_t& id, int64_t& off) const;

  int64_t rank_, world_;
  std::vector<int64_t> sigs_;
  double timeout_;
  int64_t blocks_;
  int64_t epoch_ = 1;
  std::vector<std::vector<int64_t>> bufs_;
  std::vector<int64_t> sizes_;
};

}  // namespace dtb
