// Bulk-staged forward scan kernels with delta/u in bf16 that also write the final (h, dBu) state, one per
// tile of m3_tiles.h (element type fixed at compile time).
#include "m3_scan_fwd.cuh"

namespace m3 {

cudaError_t launch_fwd_bulk_bf16_state(const Tile& t, const FwdParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb, gs)                                              \
  if (t.R == r && t.T == tt && t.ND == nd)                                        \
    return p.y_bf16 ? fwd::launch_fwd_impl<r, tt, nd, true, true, 1, 1>(p, s)     \
                    : fwd::launch_fwd_impl<r, tt, nd, true, true, 1, 0>(p, s);
  M3_TILE_LIST(M3_X)
  M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
