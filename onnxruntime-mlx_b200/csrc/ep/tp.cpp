// Tensor parallelism over NCCL (one process per GPU).  The plan shards column-parallel projections
// (q/k/v, gate/up: output rows split), row-parallel projections (o, down: K split at block
// boundaries, followed by an all-reduce of the partial sums) and attention by KV head; the
// vocabulary-split lm_head is followed by an all-gather.  Collectives are issued on the plan's
// stream and are captured into its CUDA graph like the kernels.
#include "tp.h"

#include <cstring>
#include <string>

#include "../common.cuh"
#include "plan.h"
#include "../kernels/mnb_mma.h"

#ifdef B200EP_HAVE_NCCL
#include <nccl.h>
#endif

namespace b200ep {

TpContext::~TpContext() {
  for (int r = 0; r < world && r < 8; ++r)
    if (r != rank && ar_peer[r]) cudaIpcCloseMemHandle(ar_peer[r]);
  if (ar_local) cudaFree(ar_local);
  if (ar_ctrs) cudaFree(ar_ctrs);
#ifdef B200EP_HAVE_NCCL
  if (owns_comm && comm) ncclCommDestroy(static_cast<ncclComm_t>(comm));
#endif
}

int tp_mailbox_init(TpContext& tp, size_t slot_bytes) {
#ifdef B200EP_HAVE_NCCL
  if (tp.world < 2 || tp.world > kArMaxRanks) return B200EP_OK;
  const size_t bytes = kArFlagsBytes + 2 * (size_t)tp.world * slot_bytes;
  // every rank takes the same steps (allocation, the exchange, the mapping) so that the exchange
  // below never waits on a rank that bailed out; failures only turn the fused path off
  bool ok = cudaMalloc(&tp.ar_local, bytes) == cudaSuccess && cudaMemset(tp.ar_local, 0, bytes) == cudaSuccess &&
            cudaMalloc(&tp.ar_ctrs, 256) == cudaSuccess && cudaMemset(tp.ar_ctrs, 0, 256) == cudaSuccess;
  cudaIpcMemHandle_t mine{};
  if (ok) ok = cudaIpcGetMemHandle(&mine, tp.ar_local) == cudaSuccess;
  cudaGetLastError();
  // exchange handles (and the ok bits) over NCCL
  const size_t rec = sizeof(cudaIpcMemHandle_t) + 8;
  void* dbuf = nullptr;
  if (cudaMalloc(&dbuf, rec * tp.world) != cudaSuccess) return set_error(B200EP_ECUDA, "mailbox exchange buffer");
  std::vector<unsigned char> host(rec * tp.world, 0);
  memcpy(host.data() + rec * tp.rank, &mine, sizeof(mine));
  host[rec * tp.rank + sizeof(mine)] = ok ? 1 : 0;
  cudaMemcpy(static_cast<char*>(dbuf) + rec * tp.rank, host.data() + rec * tp.rank, rec, cudaMemcpyHostToDevice);
  ncclResult_t r = ncclAllGather(static_cast<char*>(dbuf) + rec * tp.rank, dbuf, rec, ncclUint8,
                                 static_cast<ncclComm_t>(tp.comm), nullptr);
  cudaStreamSynchronize(nullptr);
  cudaMemcpy(host.data(), dbuf, rec * tp.world, cudaMemcpyDeviceToHost);
  cudaFree(dbuf);
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("mailbox exchange: ") + ncclGetErrorString(r));
  bool all = true;
  for (int k = 0; k < tp.world; ++k) all &= host[rec * k + sizeof(mine)] == 1;
  if (!all) return B200EP_OK;
  for (int k = 0; k < tp.world && all; ++k) {
    if (k == tp.rank) {
      tp.ar_peer[k] = tp.ar_local;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, host.data() + rec * k, sizeof(h));
    all &= cudaIpcOpenMemHandle(&tp.ar_peer[k], h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
  }
  cudaGetLastError();
  // agree on the outcome (a rank that could not map a peer turns the path off everywhere)
  int flag = all ? 1 : 0, *dflag = nullptr;
  cudaMalloc(&dflag, sizeof(int));
  cudaMemcpy(dflag, &flag, sizeof(int), cudaMemcpyHostToDevice);
  r = ncclAllReduce(dflag, dflag, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(tp.comm), nullptr);
  cudaStreamSynchronize(nullptr);
  cudaMemcpy(&flag, dflag, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dflag);
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("mailbox agreement: ") + ncclGetErrorString(r));
  tp.ar_slot_bytes = slot_bytes;
  tp.ar_ok = flag == 1;
  return B200EP_OK;
#else
  (void)tp;
  (void)slot_bytes;
  return B200EP_OK;
#endif
}

int tp_collective(const TpContext& tp, const Step& s, const std::vector<Slot>& S, cudaStream_t st) {
#ifdef B200EP_HAVE_NCCL
  const Slot& x = S[s.in[0]];
  const Slot& y = S[s.out[0]];
  ncclDataType_t dt = x.dtype == kF16 ? ncclFloat16 : x.dtype == kBF16 ? ncclBfloat16 : ncclFloat32;
  ncclResult_t r;
  if (s.kind == StepKind::kAllReduce) {
    r = ncclAllReduce(x.ptr, y.ptr, (size_t)x.numel(), dt, ncclSum, static_cast<ncclComm_t>(tp.comm), st);
  } else {
    // every rank holds [rows, shard] columns of [rows, shard * world]: gather rank-major, then
    // place each rank's block at its column offset (one 2-D copy per rank; none for one row)
    const int64_t shard = s.shard_cols, rows = x.numel() / std::max<int64_t>(shard, 1);
    if (rows == 1) {
      r = ncclAllGather(x.ptr, y.ptr, (size_t)x.numel(), dt, static_cast<ncclComm_t>(tp.comm), st);
    } else {
      const Slot& stage = S[s.ws_slot];
      r = ncclAllGather(x.ptr, stage.ptr, (size_t)x.numel(), dt, static_cast<ncclComm_t>(tp.comm), st);
      const size_t esz = (size_t)dtype_size(x.dtype);
      for (int k = 0; r == ncclSuccess && k < tp.world; ++k) {
        cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(y.ptr) + k * shard * esz, (size_t)s.N * esz,
                                          static_cast<const char*>(stage.ptr) + (size_t)k * rows * shard * esz,
                                          shard * esz, shard * esz, rows, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_status(e, "tensor-parallel gather placement");
      }
    }
  }
  if (r != ncclSuccess) return set_error(B200EP_ENCCL, std::string("NCCL: ") + ncclGetErrorString(r));
  return B200EP_OK;
#else
  (void)tp;
  (void)s;
  (void)S;
  (void)st;
  return set_error(B200EP_EUNSUPPORTED, "library built without NCCL");
#endif
}

}  // namespace b200ep
