// Prepacked int4 MatMulNBits on the tensor cores (mnb_mma.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200ep {

// Geometry and device buffer of one prepacked weight: ntiles x ksteps4 group records of
// record_bytes each (16 rows x 64 k of int4 weights plus their block scales / zero points).
struct MnbPacked {
  int64_t N = 0, K = 0;
  int block = 32;
  int64_t nblocks_src = 0;  // blocks per row in the ORT layout
  int64_t ntiles = 0;       // 16-row tiles
  int64_t ksteps4 = 0;      // 64-k groups after padding K to a multiple of max(64, block)
  int record_bytes = 0;
  size_t bytes = 0;
  void* w = nullptr;
};

// Producer of the GEMV's activations fused into its shared-memory staging (decode sizes only, see
// mnb_prologue_fits).  kProRms / kProSkipRms: A = rms_norm(x [+ skip]) * gamma, the skip form also
// writing the rounded sum x + skip to `residual` (may be null); kProSiluMul: A = silu(g) * u with
// x = [M, 2K] holding g in columns [0, K) and u in [K, 2K).
enum MnbProKind : int { kProNone = 0, kProRms = 1, kProSkipRms = 2, kProSiluMul = 3 };
// Peer-memory all-reduce between tensor-parallel ranks (one process per GPU, NVLink P2P).  Every
// rank owns a mailbox mapped into all ranks: [flags: uint32 per source rank][2 regions][source
// rank slots].  A producer GEMV stores its partial output, rounded to the I/O dtype, into slot
// `rank` of region (epoch & 1) of every rank's mailbox, fences, and its last CTA publishes
// `epoch` in every rank's flag word for `rank` (release, system scope).  A consumer prologue reads
// the local epoch counter, waits (bounded) until every source's flag reaches it, and sums the
// slots in rank order — the same order on every rank, so replicated activations stay identical.
constexpr int kArMaxRanks = 8;
constexpr size_t kArFlagsBytes = 256;
struct MnbAr {
  int world = 0;                        // 0 = off
  int rank = 0;
  unsigned* ctrs = nullptr;             // local: [0] epoch of the last producer, [1] its finished CTAs
  char* mbox[kArMaxRanks] = {};         // every rank's mailbox (mapped); mbox[rank] = local
  size_t region_bytes = 0;              // world * slot_bytes
  size_t slot_bytes = 0;
};

struct MnbPro {
  int kind = kProNone;
  const void* x = nullptr;
  const void* skip = nullptr;
  const void* gamma = nullptr;
  void* residual = nullptr;
  float eps = 0.f;
  MnbAr ar;  // world > 0: x is the sum of the mailbox slots (kProSkipRms only)
  // epilogue: the weight rows are interleaved 8 gate / 8 up per 16-row tile (N = 2 F); the GEMV
  // writes h = SiLU(gate) * up, F outputs per row, instead of the 2 F projections
  int swiglu = 0;
};

int mnb_record_bytes(int block);
MnbPacked mnb_packed_geometry(int64_t N, int64_t K, int block);
bool mnb_mma_supported(int dtype, int bits, int block, int64_t K);
cudaError_t launch_mnb_prepack(const uint8_t* B, const void* scales, const uint8_t* zp, int scale_dtype,
                               const MnbPacked& p, cudaStream_t st);
cudaError_t launch_mnb_packed(const void* A, const MnbPacked& p, void* Y, int dtype, int64_t M, cudaStream_t st,
                              const MnbPro* pro = nullptr, const MnbAr* out_ar = nullptr);
// Whether a prologue can run fused for M rows of K activations (they must fit the staging area).
bool mnb_prologue_fits(int64_t M, int64_t K, int block);

// Many rows (prefill): tcgen05 / TMEM GEMM over the same prepacked records (mnb_gemm.cu).
bool mnb_gemm_supported(int64_t M, int64_t K, const void* A);
cudaError_t launch_mnb_gemm(const void* A, const MnbPacked& p, void* Y, int dtype, int64_t M, cudaStream_t st);

}  // namespace b200ep
