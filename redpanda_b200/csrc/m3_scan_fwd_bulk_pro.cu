// Bulk-staged forward scan kernels with the layer's prologue fused into their
// staging (bf16 dt and x_proj rows; softplus, BCNorm and MIMO fold per landed
// chunk), one per tile of m3_tiles.h and stored-y element type.
#include "m3_scan_fwd.cuh"

namespace m3 {

cudaError_t launch_fwd_bulk_pro(const Tile& t, const FwdParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb, gs)                                                     \
  if (t.R == r && t.T == tt && t.ND == nd)                                               \
    return p.y_bf16 ? fwd::launch_fwd_impl<r, tt, nd, true, false, 1, 1, true>(p, s)       \
                    : fwd::launch_fwd_impl<r, tt, nd, true, false, 1, 0, true>(p, s);
  M3_TILE_LIST(M3_X)
  M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
