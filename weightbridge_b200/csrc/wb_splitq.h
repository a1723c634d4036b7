// Host-side interface of the split-block quantisation kernels (wb_splitq.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "wb_common.h"

namespace wb {

// partial[i] = max |x| over piece i (one CTA per piece, grid-stride).
cudaError_t launch_split_amax(const SplitPiece* pieces, uint32_t n, float* partial, cudaStream_t stream);
// Quantise piece i with the block amax amax[i]: scale = amax / 448, q = satfinite_e4m3(x * RN(1 / scale));
// writes the scale to the piece's scale cell.
cudaError_t launch_split_quant(const SplitPiece* pieces, uint32_t n, const float* amax, cudaStream_t stream);

}  // namespace wb
