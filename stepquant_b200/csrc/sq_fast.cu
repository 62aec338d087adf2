// Register-resident decode kernels for K = V = 128 GDN heads (placeholder:
// not eligible until the fast path is built; everything runs on sq_tile.cu).
#include "sq_tile.cuh"

namespace sq {

bool fast_eligible(const sq_plan &) { return false; }

cudaError_t launch_fast(int, const TileParams &, int, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace sq
