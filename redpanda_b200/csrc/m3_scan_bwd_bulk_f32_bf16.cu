// Bulk-staged analytic backward kernels with delta/u in f32 and dy in
// bf16 (element types fixed at compile time), one per tile of m3_tiles.h
// whose bulk layout fits in shared memory.
#include "m3_scan_bwd.cuh"

namespace m3 {

cudaError_t launch_bwd_bulk_f32_bf16(const Tile& t, const BwdParams& p, cudaStream_t s, bool* handled) {
  *handled = false;
#define M3_X(r, tt, nd, ndb, nthb, gs)                                                  \
  if constexpr (ndb > 0 &&                                                              \
                bwd::BwdCfg<r, tt, (ndb > 0 ? ndb : 2), nthb, (gs != 0), true>::smem_bytes <= \
                    bwd::kMaxSmemPerCta)                                                \
    if (t.R == r && t.T == tt && t.ND == nd) {                                          \
      const cudaError_t e = bwd::launch_bwd_impl<r, tt, ndb, nthb, (gs != 0), true, 0, 1>(p, s);  \
      *handled = e != cudaErrorNotSupported;                                      \
      return e;                                                                     \
    }
  M3_TILE_LIST(M3_X)
  M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
  return cudaSuccess;
}

}  // namespace m3
