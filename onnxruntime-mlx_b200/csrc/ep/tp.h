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
  // peer-memory all-reduce mailboxes (see MnbAr in kernels/mnb_mma.h); ar_ok = false -> NCCL only
  bool ar_ok = false;
  void* ar_local = nullptr;     // this rank's mailbox
  void* ar_ctrs = nullptr;      // local epoch / CTA counters
  void* ar_peer[8] = {};        // every rank's mailbox mapped into this process
  size_t ar_slot_bytes = 0;     // one source rank's partial: rows x hidden of the I/O dtype
  ~TpContext();
};

// Allocates this rank's mailbox and maps every peer's (CUDA IPC handles exchanged over the NCCL
// communicator).  Collective: every rank calls it.  Leaves ar_ok = false (NCCL fallback) when the
// ranks cannot map each other's memory.
int tp_mailbox_init(TpContext& tp, size_t slot_bytes);

int tp_collective(const TpContext& tp, const Step& s, const std::vector<Slot>& slots, cudaStream_t st);

}  // namespace b200ep
