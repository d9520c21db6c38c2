// Momentum scan backward and backward-summary kernels for fp32 activations (one
// compilation unit per element type and side, so they build in parallel).
#include "mmscan_kernels.cuh"

namespace mmb {
template int mmscan_launch<ElemF32, false>(const MMParams&, int64_t, int, int, cudaStream_t);
}  // namespace mmb
