// Host interface of the synthetic-weight fill kernel (wb_synth.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace wb {

constexpr int kSynthMaxDims = 8;

// One strided view to fill: element (c_0, ..., c_{n-1}) of the view lives at
// dst + sum(c_k * vstride[k]) elements and holds the synthetic value of logical element
// sum((lo[k] + c_k) * lstride[k]) of the full tensor.
struct SynthDesc {
  uint64_t dst;
  int32_t ndim;
  uint32_t dtype;                  // DT_F32 / DT_BF16 / DT_F16 / DT_F64 (wb_common.h)
  uint64_t key;                    // per-tensor key (name hash xor seed), below 2^32
  double std;
  int64_t ext[kSynthMaxDims];      // view extents
  int64_t vstride[kSynthMaxDims];  // view strides, elements
  int64_t lo[kSynthMaxDims];       // first logical coordinate per dimension
  int64_t lstride[kSynthMaxDims];  // logical row-major strides of the full tensor
};

bool synth_dtype_supported(uint32_t code);
cudaError_t launch_synth_fill(const SynthDesc& d, cudaStream_t stream);

}  // namespace wb
