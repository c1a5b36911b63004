// Tensor-parallel context: one process per GPU, an NCCL communicator over NVLink for the
// collectives the plan inserts at row-parallel projection outputs (all-reduce) and after the
// vocabulary-split lm_head (all-gather).
#pragma once

#include <cuda_runtime.h>

#include <vector>

namespace b200ep {

struct Slot;
struct Step;

struct TpContext {
  int rank = 0;
  int world = 1;
  void* comm = nullptr;  // ncclComm_t
  bool owns_comm = false;
  ~TpContext();
};

int tp_collective(const TpContext& tp, const Step& s, const std::vector<Slot>& slots, cudaStream_t st);

}  // namespace b200ep
