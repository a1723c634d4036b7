// Host-side interface of the sm_100a transfer kernel (wb_transfer.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "wb_common.h"

namespace wb {

// Completion signal of one launch.
struct Signal {
  uint32_t* counter;           // scratch word, zero between launches (the last CTA resets it)
  const uint64_t* flag_addrs;  // device array: addresses of the flag words to publish to (bit 0
                               // set: an NVLink multicast address, written with multimem.st)
  uint32_t n_flags;
  const uint64_t* epoch;       // device word holding this sync's epoch
  uint32_t* status;            // ST_* bits, or null
};

struct TransferArgs {
  const Item* items;           // generic items (all threads, vector loads/stores)
  uint32_t n_items;
  const Item* bulk_items;      // 16-byte aligned copies for the TMA pipeline
  uint32_t n_bulk;
  const QuantDesc* qdescs;
  const QuantWork* qwork;
  uint32_t n_qwork;
  uint32_t piece_bytes;        // TMA stage size (multiple of 16)
  uint32_t mbar_spin_limit;    // polls before an mbarrier wait gives up
  Signal sig;
  // TMA-fed quantisation (TMA modes only; null: every block takes the register path):
  // one 128-byte CUtensorMap per quant descriptor (64-byte aligned) and a byte per
  // descriptor, 1 where that map is valid (encode_quant_maps)
  const uint8_t* qmaps;
  const uint8_t* qtma;
};

// Bytes of one 128 x 128 block of 16-bit source elements: a quant stage in shared memory.
constexpr uint32_t kQBlockBytes = 128u * 128u * 2u;

// Encode the tensor maps of the quant descriptors the TMA path can load (host): bf16 / fp16
// sources, 128 x 128 blocks, 16-byte aligned source rows, 8-byte aligned destination rows,
// columns a multiple of 8.  Writes maps[i] (128 bytes each) and valid[i]; returns how many
// descriptors qualified.  Throws if the driver's encoder is unavailable.
uint32_t encode_quant_maps(const QuantDesc* descs, uint32_t n, uint8_t* maps, uint8_t* valid);

// mode 0: no TMA pipeline (bulk items must be empty); 1: 8 stages; 2: 12 stages; 3: 4 stages
int bulk_stages(int mode);
cudaError_t launch_transfer(const TransferArgs& a, int mode, int grid, cudaStream_t stream);
cudaError_t launch_wait_flags(const uint64_t* flags, uint32_t n, const uint64_t* epoch, uint64_t timeout_ns,
                              uint32_t* status, uint32_t* where, cudaStream_t stream);

}  // namespace wb
