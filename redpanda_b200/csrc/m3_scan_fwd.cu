// K1/K3 dispatch: tile, element-type and variant selection of the forward scan.
// The element-wise-staging variants (run-time element type) are compiled here;
// the bulk-staged variants, one translation unit per (delta/u element type,
// return_state) pair, in m3_scan_fwd_bulk_*.cu from the kernel template in
// m3_scan_fwd.cuh, so that the build compiles them in parallel.
#include "m3_scan_fwd.cuh"

namespace m3 {

// defined in m3_scan_fwd_bulk_<dtype>_<state>.cu: launch the bulk-staged kernel of tile t
cudaError_t launch_fwd_bulk_bf16_state(const Tile& t, const FwdParams& p, cudaStream_t s);
cudaError_t launch_fwd_bulk_bf16_nostate(const Tile& t, const FwdParams& p, cudaStream_t s);
cudaError_t launch_fwd_bulk_f32_state(const Tile& t, const FwdParams& p, cudaStream_t s);
cudaError_t launch_fwd_bulk_f32_nostate(const Tile& t, const FwdParams& p, cudaStream_t s);

cudaError_t launch_fwd_bulk_pro(const Tile& t, const FwdParams& p, cudaStream_t s);

cudaError_t launch_scan_fwd(const Tile& t, const FwdParams& p, cudaStream_t s) {
  // the fused prologue exists only as a bf16 bulk-staged kernel (the C ABI
  // checks eligibility first; no fallback)
  if (p.pro) return launch_fwd_bulk_pro(t, p, s);
  if (p.bulk) {
    const bool bf = p.dt_du == M3_BF16, st = p.h_last != nullptr;
    const cudaError_t e =
        bf ? (st ? launch_fwd_bulk_bf16_state(t, p, s) : launch_fwd_bulk_bf16_nostate(t, p, s))
           : (st ? launch_fwd_bulk_f32_state(t, p, s) : launch_fwd_bulk_f32_nostate(t, p, s));
    if (e != cudaErrorNotSupported) return e;   // else: no tensor maps, element-wise staging
  }
#define M3_X(r, tt, nd, ndb, nthb, gs)                                              \
  if (t.R == r && t.T == tt && t.ND == nd)                                        \
    return p.h_last ? fwd::launch_fwd_impl<r, tt, nd, false, true, -1, -1>(p, s)    \
                    : fwd::launch_fwd_impl<r, tt, nd, false, false, -1, -1>(p, s);
  M3_TILE_LIST(M3_X)
  M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
