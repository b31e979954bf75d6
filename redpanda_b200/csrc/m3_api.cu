// C ABI of the scan library: argument validation, tile selection, workspace
// layout and kernel dispatch.  No allocation, no exceptions, no host sync.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_tiles.h"
#include "m3scan.h"

namespace m3 {

__device__ int g_err_word = 0;

int* device_err_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_err_word) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

bool select_tile(int n_rot, int n_track, Tile* out) {
  const int rr = (n_rot + 3) / 4, tt = (n_track + 3) / 4;
  static const Tile kTiles[] = {
#define M3_X(r, t, nd, ndb, nthb, gs) {r, t, nd, ndb, nthb, gs},
      M3_TILE_LIST(M3_X)
#undef M3_X
  };
  const Tile* best = nullptr;
  for (const Tile& t : kTiles) {
    if (t.R == rr && t.T == tt) { *out = t; return true; }
  }
  for (const Tile& t : kTiles) {
    if (t.R >= rr && t.T >= tt && (!best || t.R + t.T < best->R + best->T)) best = &t;
  }
  if (!best) return false;
  *out = *best;
  return true;
}

namespace {

constexpr int kMaxState = 128;

int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return -1; }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return sms;
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return M3_ERR_NO_DEVICE; }
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return M3_ERR_NO_DEVICE;
  }
  return major == 10 ? M3_OK : M3_ERR_NO_DEVICE;
}

bool dtype_ok(int dt) { return dt == M3_F32 || dt == M3_BF16; }
int dsize(int dt) { return dt == M3_BF16 ? 2 : 4; }
bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_scan_desc(const m3_scan_desc* d, Tile* tile) {
  if (!d) return M3_ERR_NULL;
  if (d->batch < 1 || d->seqlen < 1 || d->d_inner < 1 || d->d_state < 1 ||
      d->d_state > kMaxState || d->n_rot < 0 || d->n_rot > d->d_state)
    return M3_ERR_SHAPE;
  if (!dtype_ok(d->dtype_du) || !dtype_ok(d->dtype_bc)) return M3_ERR_DTYPE;
  if (d->direction < M3_DIR_FWD || d->direction > M3_DIR_BIDIR) return M3_ERR_SHAPE;
  if (!select_tile(d->n_rot, d->d_state - d->n_rot, tile)) return M3_ERR_UNSUPPORTED;
  // fewer forward CTAs than SMs: the small-batch tiling of the same lane split
  // (same bits, 4x the CTAs of the config-0 tile)
  const int sms = device_sms();
  if (sms > 0 && (long long)d->batch * ((d->d_inner + tile->dt() - 1) / tile->dt()) < sms) {
    static const Tile kSmall[] = {
#define M3_X(r, t, nd, ndb, nthb, gs) {r, t, nd, ndb, nthb, gs},
        M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
    };
    for (const Tile& s : kSmall)
      if (s.R == tile->R && s.T == tile->T) { *tile = s; break; }
  }
  const long long g = (d->d_inner + tile->dt() - 1) / tile->dt();
  if (g > 65535) return M3_ERR_SHAPE;
  return M3_OK;
}

int nchunks(int L, int len = kCK) { return (L + len - 1) / len; }

size_t ckpt_floats(const m3_scan_desc* d, const Tile& t) {
  const int nch = nchunks(d->seqlen, t.cki());
  if (nch <= 1) return 0;
  const size_t ndirs = d->direction == M3_DIR_BIDIR ? 2 : 1;
  return (size_t)d->batch * ndirs * (nch - 1) * d->d_inner * t.np();
}

struct BwdLayout {
  int G, Bg;
  size_t off_a, off_bc, off_du, total;
};

size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

bool bwd_layout(const m3_scan_desc* d, const Tile& t, BwdLayout* lay) {
  if (t.NDB == 0) return false;
  const int sms = device_sms();
  if (sms <= 0) return false;
  lay->G = (d->d_inner + t.dt_bwd() - 1) / t.dt_bwd();
  const int slots = sms * t.bwd_ctas_per_sm();   // one resident wave
  int bg = lay->G >= slots ? 1 : slots / lay->G;
  if (bg > d->batch) bg = d->batch;
  if (bg < 1) bg = 1;
  lay->Bg = bg;
  const size_t np = t.np();
  const size_t a_bytes = (size_t)lay->Bg * 3 * d->d_inner * np * 4;
  const size_t ndirs = d->direction == M3_DIR_BIDIR ? 2 : 1;
  const size_t bc_bytes = (size_t)lay->G * ndirs * d->batch * d->seqlen * 2 * np * 4;
  const size_t du_bytes = d->direction == M3_DIR_BIDIR
                              ? (size_t)lay->G * lay->Bg * d->seqlen * t.dt_bwd() * 2 * 4
                              : 0;
  lay->off_a = 0;
  lay->off_bc = round256(a_bytes);
  lay->off_du = lay->off_bc + round256(bc_bytes);
  lay->total = lay->off_du + round256(du_bytes);
  return true;
}

}  // namespace
}  // namespace m3

using namespace m3;

extern "C" {

const char* m3_strerror(int code) {
  switch (code) {
    case M3_OK: return "ok";
    case M3_ERR_NULL: return "m3: a required pointer is NULL";
    case M3_ERR_SHAPE: return "m3: a size argument is out of range";
    case M3_ERR_DTYPE: return "m3: unsupported element type (float32 or bfloat16 only)";
    case M3_ERR_UNSUPPORTED: return "m3: no compiled kernel serves this shape";
    case M3_ERR_ALIGN: return "m3: a pointer is not aligned to its element size";
    case M3_ERR_WORKSPACE: return "m3: workspace missing or too small";
    case M3_ERR_LAUNCH: return "m3: CUDA kernel launch failed";
    case M3_ERR_DEVICE: return "m3: a kernel recorded a device-side error";
    case M3_ERR_NO_DEVICE: return "m3: no sm_100 CUDA device is current";
    case M3_ERR_ALIAS: return "m3: two buffers that must be distinct overlap";
    case M3_ERR_SCRATCH_LIMIT:
      return "m3: problem needs more backward scratch than the built-in no-allocation buffer "
             "(M3_NOALLOC_SCRATCH_BYTES); use m3_scan_bwd with a workspace";
    default: return "m3: unknown status code";
  }
}

int m3_version(void) { return (1 << 16) | 1; }

size_t m3_scan_ckpt_floats(const m3_scan_desc* desc) {
  Tile t;
  if (check_scan_desc(desc, &t) != M3_OK) return 0;
  return ckpt_floats(desc, t);
}

int m3_scan_fwd(const m3_scan_desc* desc, const void* delta, const void* u, const void* Bc,
                const void* Cc, const float* A_real_p, const float* A_imag_p,
                const float* track_p, float* y, float* ckpt, float* h_last, float* dbu_last,
                void* stream) {
  return m3_scan_fwd_typed(desc, delta, u, Bc, Cc, A_real_p, A_imag_p, track_p, y, M3_F32, ckpt,
                           h_last, dbu_last, stream);
}

static int fwd_common(const m3_scan_desc* desc, const void* delta, const void* u,
                      const void* Bc, const void* Cc, const float* A_real_p,
                      const float* A_imag_p, const float* track_p, void* y, int32_t dtype_y,
                      float* ckpt, float* h_last, float* dbu_last, const void* pro_args,
                      void* stream);

namespace {
// the fused prologue's inputs (m3_scan_fwd_fused / m3_scan_bwd_fused)
struct ProArgs {
  int32_t mimo_p; const void* xbc; int64_t ld_x; int32_t off_b, off_c;
  const float* wb; const float* wc; float eps;
};

// Shapes the fused-prologue kernels take: bf16 delta/u rows and x_proj rows
// that TMA can stage (16-byte aligned bases, strides and box rows; column
// offsets on 8-element boundaries), whole channel tiles of at most 128
// channels, and raw B/C rows that fit the staging buffer of the padded lanes.
int check_pro(const m3_scan_desc* d, const Tile& t, const ProArgs& a, const void* dt,
              const void* u, int dt_tile) {
  const int64_t np = (int64_t)d->d_state * a.mimo_p;
  if (a.mimo_p < 1 || a.off_b < 0 || a.off_c < 0 || a.off_b + np > a.ld_x ||
      a.off_c + np > a.ld_x || !(a.eps >= 0.f))
    return M3_ERR_SHAPE;
  if (!a.xbc || ((a.wb == nullptr) != (a.wc == nullptr))) return M3_ERR_NULL;
  if (d->dtype_du != M3_BF16) return M3_ERR_DTYPE;
  if (!aligned(dt, 16) || !aligned(u, 16) || !aligned(a.xbc, 16) ||
      (a.wb && (!aligned(a.wb, 4) || !aligned(a.wc, 4))))
    return M3_ERR_ALIGN;
  if ((d->d_inner % dt_tile) != 0 || dt_tile > 128 || (d->d_inner % 8) != 0 ||
      ((a.ld_x * 2) % 16) != 0 || (a.off_b % 8) != 0 || (a.off_c % 8) != 0 ||
      (np % 8) != 0 || np > 256 || np > 4 * t.np() || getenv("M3_NO_BULK") != nullptr)
    return M3_ERR_UNSUPPORTED;
  return M3_OK;
}
}  // namespace

int m3_scan_fwd_typed(const m3_scan_desc* desc, const void* delta, const void* u,
                      const void* Bc, const void* Cc, const float* A_real_p,
                      const float* A_imag_p, const float* track_p, void* y, int32_t dtype_y,
                      float* ckpt, float* h_last, float* dbu_last, void* stream) {
  return fwd_common(desc, delta, u, Bc, Cc, A_real_p, A_imag_p, track_p, y, dtype_y, ckpt,
                    h_last, dbu_last, nullptr, stream);
}

int m3_scan_fwd_fused(const m3_scan_desc* desc, int32_t mimo_p, const void* dt,
                      const void* xbc, int64_t ld_x, int32_t off_b, int32_t off_c,
                      const float* wb, const float* wc, float eps, const void* u,
                      const float* A_real_p, const float* A_imag_p, const float* track_p,
                      void* y, int32_t dtype_y, float* ckpt, void* stream) {
  const ProArgs a{mimo_p, xbc, ld_x, off_b, off_c, wb, wc, eps};
  // Bc/Cc are not read: pass xbc so that the shared checks see valid pointers
  return fwd_common(desc, dt, u, xbc, xbc, A_real_p, A_imag_p, track_p, y, dtype_y, ckpt,
                    nullptr, nullptr, &a, stream);
}

static int fwd_common(const m3_scan_desc* desc, const void* delta, const void* u,
                      const void* Bc, const void* Cc, const float* A_real_p,
                      const float* A_imag_p, const float* track_p, void* y, int32_t dtype_y,
                      float* ckpt, float* h_last, float* dbu_last, const void* pro_args,
                      void* stream) {
  const ProArgs* pro = static_cast<const ProArgs*>(pro_args);
  if (dtype_y != M3_F32 && dtype_y != M3_BF16) return M3_ERR_DTYPE;
  const int esy = dtype_y == M3_BF16 ? 2 : 4;
  Tile t;
  int rc = check_scan_desc(desc, &t);
  if (rc != M3_OK) return rc;
  if (!delta || !u || !Bc || !Cc || !A_real_p || !A_imag_p || !track_p || !y) return M3_ERR_NULL;
  if ((h_last == nullptr) != (dbu_last == nullptr)) return M3_ERR_NULL;
  if (h_last && desc->direction == M3_DIR_BIDIR) return M3_ERR_SHAPE;
  const int esd = dsize(desc->dtype_du), esb = dsize(desc->dtype_bc);
  if (!aligned(delta, esd) || !aligned(u, esd) || !aligned(Bc, esb) || !aligned(Cc, esb) ||
      !aligned(A_real_p, 4) || !aligned(A_imag_p, 4) || !aligned(track_p, 4) ||
      !aligned(y, esy) || (ckpt && !aligned(ckpt, 16)) ||
      (h_last && (!aligned(h_last, 4) || !aligned(dbu_last, 4))))
    return M3_ERR_ALIGN;
  if (pro && (rc = check_pro(desc, t, *pro, delta, u, t.dt())) != M3_OK) return rc;
  if ((rc = check_device()) != M3_OK) return rc;

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.delta = delta; p.u = u; p.Bc = Bc; p.Cc = Cc;
  p.Ar = A_real_p; p.Ai = A_imag_p; p.Tk = track_p;
  p.y = y; p.y_bf16 = dtype_y == M3_BF16; p.ckpt = ckpt_floats(desc, t) ? ckpt : nullptr;
  p.h_last = h_last; p.dbu_last = dbu_last;
  p.B = desc->batch; p.L = desc->seqlen; p.D = desc->d_inner; p.N = desc->d_state;
  p.NR = desc->n_rot; p.NT = desc->d_state - desc->n_rot;
  p.dt_du = desc->dtype_du; p.dt_bc = desc->dtype_bc;
  p.direction = desc->direction;
  p.nch = nchunks(desc->seqlen);
  p.cki = t.cki();
  p.nck = nchunks(desc->seqlen, p.cki) - 1;
  p.async_ok = aligned(delta, 4) && aligned(u, 4) &&
               (desc->dtype_du == M3_F32 || (desc->d_inner % 2) == 0);
  // bulk staging: whole channel tiles and 16-byte aligned rows of every input
  p.bulk = (desc->d_inner % t.dt()) == 0 && ((desc->d_inner * esd) % 16) == 0 &&
           ((desc->d_state * esb) % 16) == 0 && aligned(delta, 16) && aligned(u, 16) &&
           aligned(Bc, 16) && aligned(Cc, 16) && aligned(y, 16) &&
           ((desc->d_inner * esy) % 16) == 0 && getenv("M3_NO_BULK") == nullptr;
  if (pro) {
    if (!p.bulk) return M3_ERR_UNSUPPORTED;
    p.pro = 1; p.xbc = pro->xbc; p.ld_x = pro->ld_x; p.off_b = pro->off_b;
    p.off_c = pro->off_c; p.P = pro->mimo_p; p.wb = pro->wb; p.wc = pro->wc; p.eps = pro->eps;
  }
  p.err = device_err_ptr();
  cudaError_t e = launch_scan_fwd(t, p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

size_t m3_scan_bwd_workspace_bytes(const m3_scan_desc* desc) {
  Tile t;
  if (check_scan_desc(desc, &t) != M3_OK) return 0;
  BwdLayout lay;
  if (!bwd_layout(desc, t, &lay)) return 0;
  return lay.total;
}

int m3_scan_bwd(const m3_scan_desc* desc, const void* delta, const void* u, const void* Bc,
                const void* Cc, const float* A_real_p, const float* A_imag_p,
                const float* track_p, const void* dy, int32_t dtype_dy, const float* ckpt,
                void* d_delta, void* d_u, void* d_Bc, void* d_Cc, float* d_A_real_p,
                float* d_A_imag_p, float* d_track_p, void* workspace, size_t workspace_bytes,
                void* stream) {
  Tile t;
  int rc = check_scan_desc(desc, &t);
  if (rc != M3_OK) return rc;
  if (t.NDB == 0) return M3_ERR_UNSUPPORTED;
  if (!dtype_ok(dtype_dy)) return M3_ERR_DTYPE;
  if (!delta || !u || !Bc || !Cc || !A_real_p || !A_imag_p || !track_p || !dy || !d_delta ||
      !d_u || !d_Bc || !d_Cc || !d_A_real_p || !d_A_imag_p || !d_track_p)
    return M3_ERR_NULL;
  if (ckpt_floats(desc, t) > 0 && !ckpt) return M3_ERR_NULL;
  const int esd = dsize(desc->dtype_du), esb = dsize(desc->dtype_bc), esy = dsize(dtype_dy);
  if (!aligned(delta, esd) || !aligned(u, esd) || !aligned(d_delta, esd) || !aligned(d_u, esd) ||
      !aligned(Bc, esb) || !aligned(Cc, esb) || !aligned(d_Bc, esb) || !aligned(d_Cc, esb) ||
      !aligned(dy, esy) || !aligned(A_real_p, 4) || !aligned(A_imag_p, 4) ||
      !aligned(track_p, 4) || !aligned(d_A_real_p, 4) || !aligned(d_A_imag_p, 4) ||
      !aligned(d_track_p, 4) || (ckpt && !aligned(ckpt, 16)) || !aligned(workspace, 256))
    return M3_ERR_ALIGN;
  if ((rc = check_device()) != M3_OK) return rc;
  BwdLayout lay;
  if (!bwd_layout(desc, t, &lay)) return M3_ERR_NO_DEVICE;
  if (!workspace || workspace_bytes < lay.total) return M3_ERR_WORKSPACE;

  char* ws = static_cast<char*>(workspace);
  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.delta = delta; p.u = u; p.Bc = Bc; p.Cc = Cc;
  p.Ar = A_real_p; p.Ai = A_imag_p; p.Tk = track_p;
  p.dy = dy; p.ckpt = ckpt;
  p.d_delta = d_delta; p.d_u = d_u;
  p.part_a = reinterpret_cast<float*>(ws + lay.off_a);
  p.part_bc = reinterpret_cast<float*>(ws + lay.off_bc);
  p.scratch_du =
      desc->direction == M3_DIR_BIDIR ? reinterpret_cast<float*>(ws + lay.off_du) : nullptr;
  p.B = desc->batch; p.L = desc->seqlen; p.D = desc->d_inner; p.N = desc->d_state;
  p.NR = desc->n_rot; p.NT = desc->d_state - desc->n_rot;
  p.dt_du = desc->dtype_du; p.dt_bc = desc->dtype_bc; p.dt_dy = dtype_dy;
  p.direction = desc->direction;
  p.nch = nchunks(desc->seqlen, t.cki());
  p.G = lay.G; p.Bg = lay.Bg;
  p.async_du = aligned(delta, 4) && aligned(u, 4) &&
               (desc->dtype_du == M3_F32 || (desc->d_inner % 2) == 0);
  p.async_dy = aligned(dy, 4) && (dtype_dy == M3_F32 || (desc->d_inner % 2) == 0);
  // bulk staging: whole channel tiles and 16-byte aligned rows of every input
  // and of d_delta/d_u (the flush writes 4 channels per vector store)
  p.bulk = (desc->d_inner % t.dt_bwd()) == 0 && ((desc->d_inner * esd) % 16) == 0 &&
           ((desc->d_inner * esy) % 16) == 0 && ((desc->d_state * esb) % 16) == 0 &&
           aligned(delta, 16) && aligned(u, 16) && aligned(dy, 16) && aligned(Bc, 16) &&
           aligned(Cc, 16) && aligned(d_delta, 16) && aligned(d_u, 16) &&
           (!ckpt || aligned(ckpt, 16)) && getenv("M3_NO_BULK") == nullptr;
  p.err = device_err_ptr();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_scan_bwd(t, p, s);
  if (e != cudaSuccess) return M3_ERR_LAUNCH;

  ReduceParams r;
  memset(&r, 0, sizeof(r));
  r.part_bc = p.part_bc; r.part_a = p.part_a;
  r.d_Bc = d_Bc; r.d_Cc = d_Cc;
  r.dAr = d_A_real_p; r.dAi = d_A_imag_p; r.dTk = d_track_p;
  r.B = p.B; r.L = p.L; r.D = p.D; r.N = p.N; r.NR = p.NR; r.NT = p.NT;
  r.dt_bc = p.dt_bc; r.G = p.G; r.Bg = p.Bg;
  r.ndirs = desc->direction == M3_DIR_BIDIR ? 2 : 1;
  e = launch_bwd_reduce(t, r, s);
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

// Arguments of the fused prologue (m3_step_gated_fused).
struct StepPro {
  const float* dt; int64_t ld_dt;
  const float* dt_bias;
  const float* xbc; int64_t ld_x;
  int32_t off_b, off_c, P;
  const float* wb; const float* wc;
  float eps;
  const float* wdt = nullptr; int32_t dt_rank = 0;   // dt formed in the kernel
  int pdl = 0;                                        // programmatic dependent launch
};

static int step_common(const m3_step_desc* desc, float* h, float* dbu, const float* fac_prev,
                       float* fac_next, const void* delta, const void* u, const void* Bc,
                       const void* Cc, const float* A_real_p, const float* A_imag_p,
                       const float* track_p, float* y, void* stream,
                       const float* z = nullptr, int64_t ld_z = 0,
                       const float* d_skip = nullptr, const StepPro* pro = nullptr) {
  if (!desc) return M3_ERR_NULL;
  if (desc->batch < 1 || desc->d_inner < 1 || desc->d_state < 1 || desc->d_state > kMaxState ||
      desc->n_rot < 0 || desc->n_rot > desc->d_state)
    return M3_ERR_SHAPE;
  if (!dtype_ok(desc->dtype_du) || !dtype_ok(desc->dtype_bc)) return M3_ERR_DTYPE;
  const bool factored = fac_next != nullptr;
  if (!h || !delta || !u || !Bc || !Cc || !A_real_p || !A_imag_p || !track_p || !y)
    return M3_ERR_NULL;
  if (factored ? !fac_prev : !dbu) return M3_ERR_NULL;
  Tile t;
  if (!select_tile(desc->n_rot, desc->d_state - desc->n_rot, &t)) return M3_ERR_UNSUPPORTED;
  if ((desc->d_inner + 31) / 32 > 65535) return M3_ERR_SHAPE;
  const int esd = dsize(desc->dtype_du), esb = dsize(desc->dtype_bc);
  if (!aligned(h, 16) || (dbu && !aligned(dbu, 16)) || (fac_prev && !aligned(fac_prev, 4)) ||
      (fac_next && !aligned(fac_next, 4)) || !aligned(delta, esd) || !aligned(u, esd) ||
      !aligned(Bc, esb) || !aligned(Cc, esb) || !aligned(A_real_p, 4) || !aligned(A_imag_p, 4) ||
      !aligned(track_p, 4) || !aligned(y, 4))
    return M3_ERR_ALIGN;
  if (factored) {
    const size_t bytes = (size_t)desc->batch * (desc->d_inner + desc->d_state) * 4;
    const char* a = reinterpret_cast<const char*>(fac_prev);
    const char* b = reinterpret_cast<const char*>(fac_next);
    if (a < b + bytes && b < a + bytes) return M3_ERR_ALIAS;
  }
  int rc = check_device();
  if (rc != M3_OK) return rc;
  StepParams p;
  memset(&p, 0, sizeof(p));
  p.h = h; p.dbu = dbu; p.fac_in = fac_prev; p.fac_out = fac_next; p.factored = factored;
  p.delta = delta; p.u = u; p.Bc = Bc; p.Cc = Cc;
  p.Ar = A_real_p; p.Ai = A_imag_p; p.Tk = track_p; p.y = y;
  p.B = desc->batch; p.D = desc->d_inner; p.N = desc->d_state;
  p.NR = desc->n_rot; p.NT = desc->d_state - desc->n_rot;
  p.dt_du = desc->dtype_du; p.dt_bc = desc->dtype_bc;
  p.vec_bc = aligned(Bc, 16) && aligned(Cc, 16);
  p.vec_fac = factored && aligned(fac_prev, 16) && aligned(fac_next, 16) &&
              (desc->d_inner % 4) == 0;
  // Pipelined kernel: dense lane tile (no virtual lanes), whole 32-channel tiles,
  // and every staged row a 16-byte multiple at a 16-byte aligned address.
  p.bulk = desc->n_rot == 4 * t.R && desc->d_state - desc->n_rot == 4 * t.T &&
           (desc->d_inner % 32) == 0 && ((desc->d_state * esb) % 16) == 0 &&
           aligned(delta, 16) && aligned(u, 16) && aligned(Bc, 16) && aligned(Cc, 16) &&
           (!factored || (aligned(fac_prev, 16) && aligned(fac_next, 16))) &&
           getenv("M3_NO_BULK") == nullptr;
  p.gated = z != nullptr;
  p.z = z; p.ld_z = ld_z; p.d_skip = d_skip;
  p.err = device_err_ptr();
  if (pro) {   // the fused prologue needs the pipelined kernel on a 32-lane tile
    if (!p.bulk || desc->d_state != 32) return M3_ERR_UNSUPPORTED;
    p.pro = 1;
    p.dt = pro->dt; p.ld_dt = pro->ld_dt; p.dt_bias = pro->dt_bias;
    p.xbc = pro->xbc; p.ld_x = pro->ld_x;
    p.off_b = pro->off_b; p.off_c = pro->off_c; p.P = pro->P;
    p.wb = pro->wb; p.wc = pro->wc; p.eps = pro->eps;
    p.wdt = pro->wdt; p.dt_rank = pro->dt_rank; p.pdl = pro->pdl;
  }
  cudaError_t e = launch_step(t, p, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported) return M3_ERR_UNSUPPORTED;
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_step(const m3_step_desc* desc, float* h, float* dbu, const void* delta, const void* u,
            const void* Bc, const void* Cc, const float* A_real_p, const float* A_imag_p,
            const float* track_p, float* y, void* stream) {
  return step_common(desc, h, dbu, nullptr, nullptr, delta, u, Bc, Cc, A_real_p, A_imag_p,
                     track_p, y, stream);
}

// workspace of the fused backward: the regular backward's, then the fp32 B/C
// gradients (rows, N) x 2 and the BCNorm weight-gradient partials
static bool fused_bwd_layout(const m3_scan_desc* d, const Tile& t, int32_t mimo_p,
                             BwdLayout* lay, size_t* off_g, size_t* off_w, size_t* total) {
  if (!bwd_layout(d, t, lay)) return false;
  const long long rows = (long long)d->batch * d->seqlen;
  *off_g = lay->total;
  *off_w = *off_g + round256((size_t)rows * d->d_state * 4 * 2);
  *total = *off_w + round256((size_t)step_inputs_bwd_ctas(rows) * 2 * d->d_state * mimo_p * 4);
  return true;
}

size_t m3_scan_bwd_fused_workspace_bytes(const m3_scan_desc* desc, int32_t mimo_p) {
  Tile t;
  if (check_scan_desc(desc, &t) != M3_OK || mimo_p < 1) return 0;
  BwdLayout lay;
  size_t og, ow, total;
  if (!fused_bwd_layout(desc, t, mimo_p, &lay, &og, &ow, &total)) return 0;
  return total;
}

int m3_scan_bwd_fused(const m3_scan_desc* desc, int32_t mimo_p, const void* dt,
                      const void* xbc, int64_t ld_x, int32_t off_b, int32_t off_c,
                      const float* wb, const float* wc, float eps, const void* u,
                      const float* A_real_p, const float* A_imag_p, const float* track_p,
                      const void* dy, int32_t dtype_dy, const float* ckpt, void* d_dt,
                      void* d_u, void* d_xbc, float* d_wb, float* d_wc, float* d_A_real_p,
                      float* d_A_imag_p, float* d_track_p, void* workspace,
                      size_t workspace_bytes, void* stream) {
  Tile t;
  int rc = check_scan_desc(desc, &t);
  if (rc != M3_OK) return rc;
  if (t.NDB == 0) return M3_ERR_UNSUPPORTED;
  if (!dtype_ok(dtype_dy)) return M3_ERR_DTYPE;
  if (!dt || !u || !A_real_p || !A_imag_p || !track_p || !dy || !d_dt || !d_u || !d_xbc ||
      !d_A_real_p || !d_A_imag_p || !d_track_p || (wb && (!d_wb || !d_wc)))
    return M3_ERR_NULL;
  if (ckpt_floats(desc, t) > 0 && !ckpt) return M3_ERR_NULL;
  const ProArgs a{mimo_p, xbc, ld_x, off_b, off_c, wb, wc, eps};
  if ((rc = check_pro(desc, t, a, dt, u, t.dt_bwd())) != M3_OK) return rc;
  const int esy = dsize(dtype_dy);
  if (!aligned(dy, 16) || ((desc->d_inner * esy) % 16) != 0 || !aligned(d_dt, 16) ||
      !aligned(d_u, 16) || !aligned(d_xbc, 2) || !aligned(A_real_p, 4) ||
      !aligned(A_imag_p, 4) || !aligned(track_p, 4) || !aligned(d_A_real_p, 4) ||
      !aligned(d_A_imag_p, 4) || !aligned(d_track_p, 4) || (ckpt && !aligned(ckpt, 16)) ||
      !aligned(workspace, 256) || (d_wb && (!aligned(d_wb, 4) || !aligned(d_wc, 4))))
    return M3_ERR_ALIGN;
  if ((rc = check_device()) != M3_OK) return rc;
  BwdLayout lay;
  size_t off_g, off_w, total;
  if (!fused_bwd_layout(desc, t, mimo_p, &lay, &off_g, &off_w, &total)) return M3_ERR_NO_DEVICE;
  if (!workspace || workspace_bytes < total) return M3_ERR_WORKSPACE;

  char* ws = static_cast<char*>(workspace);
  const long long rows = (long long)desc->batch * desc->seqlen;
  float* gB = reinterpret_cast<float*>(ws + off_g);
  float* gC = gB + (size_t)rows * desc->d_state;
  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.delta = dt; p.u = u; p.Bc = xbc; p.Cc = xbc;
  p.Ar = A_real_p; p.Ai = A_imag_p; p.Tk = track_p;
  p.dy = dy; p.ckpt = ckpt;
  p.d_delta = d_dt; p.d_u = d_u;
  p.part_a = reinterpret_cast<float*>(ws + lay.off_a);
  p.part_bc = reinterpret_cast<float*>(ws + lay.off_bc);
  p.scratch_du =
      desc->direction == M3_DIR_BIDIR ? reinterpret_cast<float*>(ws + lay.off_du) : nullptr;
  p.B = desc->batch; p.L = desc->seqlen; p.D = desc->d_inner; p.N = desc->d_state;
  p.NR = desc->n_rot; p.NT = desc->d_state - desc->n_rot;
  p.dt_du = M3_BF16; p.dt_bc = M3_BF16; p.dt_dy = dtype_dy;
  p.direction = desc->direction;
  p.nch = nchunks(desc->seqlen, t.cki());
  p.G = lay.G; p.Bg = lay.Bg;
  p.async_du = 1; p.async_dy = 1; p.bulk = 1;
  p.pro = 1; p.xbc = xbc; p.ld_x = ld_x; p.off_b = off_b; p.off_c = off_c; p.P = mimo_p;
  p.wb = wb; p.wc = wc; p.eps = eps;
  p.err = device_err_ptr();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_scan_bwd(t, p, s);
  if (e == cudaErrorNotSupported) return M3_ERR_UNSUPPORTED;
  if (e != cudaSuccess) return M3_ERR_LAUNCH;

  ReduceParams r;
  memset(&r, 0, sizeof(r));
  r.part_bc = p.part_bc; r.part_a = p.part_a;
  r.d_Bc = gB; r.d_Cc = gC; r.bc_f32_of_bf16 = 1;
  r.dAr = d_A_real_p; r.dAi = d_A_imag_p; r.dTk = d_track_p;
  r.B = p.B; r.L = p.L; r.D = p.D; r.N = p.N; r.NR = p.NR; r.NT = p.NT;
  r.dt_bc = M3_F32; r.G = p.G; r.Bg = p.Bg;
  r.ndirs = desc->direction == M3_DIR_BIDIR ? 2 : 1;
  e = launch_bwd_reduce(t, r, s);
  if (e != cudaSuccess) return M3_ERR_LAUNCH;

  // BCNorm + MIMO-fold backward over the bf16 rows (the dt part was applied in
  // the scan's flush)
  InputsBwdParams q;
  memset(&q, 0, sizeof(q));
  q.dt = nullptr; q.xbc = xbc; q.x_bf16 = 1; q.ld_x = ld_x; q.off_b = off_b; q.off_c = off_c;
  q.wb = wb; q.wc = wc; q.eps = eps; q.g_Bc = gB; q.g_Cc = gC;
  q.d_xbc = d_xbc; q.d_wb = d_wb; q.d_wc = d_wc;
  q.part_w = reinterpret_cast<float*>(ws + off_w);
  q.rows = rows; q.D = desc->d_inner; q.N = desc->d_state; q.P = mimo_p;
  e = launch_step_inputs_bwd(q, s);
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_step_factored(const m3_step_desc* desc, float* h, const float* fac_prev, float* fac_next,
                     const void* delta, const void* u, const void* Bc, const void* Cc,
                     const float* A_real_p, const float* A_imag_p, const float* track_p,
                     float* y, void* stream) {
  if (!fac_next) return M3_ERR_NULL;
  return step_common(desc, h, nullptr, fac_prev, fac_next, delta, u, Bc, Cc, A_real_p, A_imag_p,
                     track_p, y, stream);
}

int m3_step_gated(const m3_step_desc* desc, float* h, float* dbu, const float* fac_prev,
                  float* fac_next, const void* delta, const void* u, const void* Bc,
                  const void* Cc, const float* A_real_p, const float* A_imag_p,
                  const float* track_p, const float* z, int64_t ld_z, const float* d_skip,
                  float* out, void* stream) {
  if (!desc || !z || !d_skip) return M3_ERR_NULL;
  if ((dbu != nullptr) == (fac_next != nullptr)) return M3_ERR_NULL;   // exactly one state form
  if (ld_z < desc->d_inner) return M3_ERR_SHAPE;
  if (!aligned(z, 4) || !aligned(d_skip, 4)) return M3_ERR_ALIGN;
  return step_common(desc, h, dbu, fac_prev, fac_next, delta, u, Bc, Cc, A_real_p, A_imag_p,
                     track_p, out, stream, z, ld_z, d_skip);
}

int m3_step_gated_fused(const m3_step_desc* desc, int32_t mimo_p, float* h, float* dbu,
                        const float* fac_prev, float* fac_next, const float* dt, int64_t ld_dt,
                        const float* dt_bias, const float* xbc, int64_t ld_x, int32_t off_b,
                        int32_t off_c,
                        const float* wb, const float* wc, float eps, const void* u,
                        const float* A_real_p, const float* A_imag_p, const float* track_p,
                        const float* z, int64_t ld_z, const float* d_skip, float* out,
                        void* stream) {
  if (!desc || !z || !d_skip || !dt || !xbc) return M3_ERR_NULL;
  if ((dbu != nullptr) == (fac_next != nullptr)) return M3_ERR_NULL;   // exactly one state form
  if ((wb == nullptr) != (wc == nullptr)) return M3_ERR_NULL;
  if (desc->dtype_bc != M3_F32) return M3_ERR_DTYPE;
  const int64_t np = (int64_t)desc->d_state * mimo_p;
  if (ld_z < desc->d_inner || ld_dt < desc->d_inner || mimo_p < 1 || off_b < 0 || off_c < 0 ||
      off_b + np > ld_x || off_c + np > ld_x || !(eps >= 0.f))
    return M3_ERR_SHAPE;
  if (!aligned(z, 4) || !aligned(d_skip, 4) || !aligned(dt, 4) || !aligned(xbc, 4) ||
      (wb && (!aligned(wb, 4) || !aligned(wc, 4))) || (dt_bias && !aligned(dt_bias, 4)))
    return M3_ERR_ALIGN;
  // every staged row a 16-byte multiple at a 16-byte aligned address
  if (mimo_p > 2 || np % 4 != 0 || !aligned(dt, 16) || ld_dt % 4 != 0 || !aligned(xbc, 16) ||
      ld_x % 4 != 0 || off_b % 4 != 0 || off_c % 4 != 0)
    return M3_ERR_UNSUPPORTED;
  const StepPro pro{dt, ld_dt, dt_bias, xbc, ld_x, off_b, off_c, mimo_p, wb, wc, eps};
  // delta/Bc/Cc are not read under the fused prologue; dt and xbc stand in
  // for the pointer checks (both 16-byte aligned)
  return step_common(desc, h, dbu, fac_prev, fac_next, dt, u, xbc, xbc, A_real_p, A_imag_p,
                     track_p, out, stream, z, ld_z, d_skip, &pro);
}

int m3_step_gated_fused_proj(const m3_step_desc* desc, int32_t mimo_p, float* h, float* dbu,
                             const float* fac_prev, float* fac_next, const float* W_dt,
                             int32_t dt_rank, const float* dt_bias, const float* xbc,
                             int64_t ld_x, int32_t off_b, int32_t off_c, const float* wb,
                             const float* wc, float eps, const void* u, const float* A_real_p,
                             const float* A_imag_p, const float* track_p, const float* z,
                             int64_t ld_z, const float* d_skip, float* out, int32_t overlap,
                             void* stream) {
  if (!desc || !z || !d_skip || !W_dt || !xbc) return M3_ERR_NULL;
  if ((dbu != nullptr) == (fac_next != nullptr)) return M3_ERR_NULL;   // exactly one state form
  if ((wb == nullptr) != (wc == nullptr)) return M3_ERR_NULL;
  if (desc->dtype_bc != M3_F32) return M3_ERR_DTYPE;
  const int64_t np = (int64_t)desc->d_state * mimo_p;
  if (ld_z < desc->d_inner || mimo_p < 1 || dt_rank < 1 || dt_rank > ld_x || off_b < 0 ||
      off_c < 0 || off_b + np > ld_x || off_c + np > ld_x || !(eps >= 0.f))
    return M3_ERR_SHAPE;
  if (!aligned(z, 4) || !aligned(d_skip, 4) || !aligned(W_dt, 4) || !aligned(xbc, 4) ||
      (wb && (!aligned(wb, 4) || !aligned(wc, 4))) || (dt_bias && !aligned(dt_bias, 4)))
    return M3_ERR_ALIGN;
  if (dt_rank > kMaxDtRank || mimo_p > 2 || np % 4 != 0 || !aligned(xbc, 16) || ld_x % 4 != 0 ||
      off_b % 4 != 0 || off_c % 4 != 0)
    return M3_ERR_UNSUPPORTED;
  StepPro pro{nullptr, 0, dt_bias, xbc, ld_x, off_b, off_c, mimo_p, wb, wc, eps};
  pro.wdt = W_dt;
  pro.dt_rank = dt_rank;
  pro.pdl = overlap != 0;
  // delta/Bc/Cc are not read under the fused prologue; xbc stands in for the
  // pointer checks (16-byte aligned)
  return step_common(desc, h, dbu, fac_prev, fac_next, xbc, u, xbc, xbc, A_real_p, A_imag_p,
                     track_p, out, stream, z, ld_z, d_skip, &pro);
}

int m3_step_inputs(const m3_step_desc* desc, int32_t mimo_p, const void* dt, int64_t ld_dt,
                   const float* dt_bias, const void* xbc, int64_t ld_x, int32_t off_b,
                   int32_t off_c, const float* wb, const float* wc, float eps, void* delta,
                   void* Bc, void* Cc, void* stream) {
  if (!desc) return M3_ERR_NULL;
  const int64_t np = (int64_t)desc->d_state * mimo_p;
  if (desc->batch < 1 || desc->d_inner < 1 || desc->d_state < 1 || mimo_p < 1 ||
      ld_dt < desc->d_inner || off_b < 0 || off_c < 0 || off_b + np > ld_x ||
      off_c + np > ld_x || !(eps >= 0.f))
    return M3_ERR_SHAPE;
  if (!dtype_ok(desc->dtype_du) || !dtype_ok(desc->dtype_bc)) return M3_ERR_DTYPE;
  if (!dt || !xbc || !delta || !Bc || !Cc || ((wb == nullptr) != (wc == nullptr)))
    return M3_ERR_NULL;
  const int esd = dsize(desc->dtype_du), esb = dsize(desc->dtype_bc);
  if (!aligned(dt, esd) || !aligned(xbc, esb) || !aligned(delta, esd) || !aligned(Bc, esb) ||
      !aligned(Cc, esb) || (wb && (!aligned(wb, 4) || !aligned(wc, 4))) ||
      (dt_bias && !aligned(dt_bias, 4)))
    return M3_ERR_ALIGN;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  InputsParams p;
  memset(&p, 0, sizeof(p));
  p.dt = dt; p.ld_dt = ld_dt; p.dt_bias = dt_bias;
  p.xbc = xbc; p.ld_x = ld_x; p.off_b = off_b; p.off_c = off_c;
  p.wb = wb; p.wc = wc; p.eps = eps; p.delta = delta; p.Bc = Bc; p.Cc = Cc;
  p.B = desc->batch; p.D = desc->d_inner; p.N = desc->d_state; p.P = mimo_p;
  p.du_bf16 = desc->dtype_du == M3_BF16;
  p.bc_bf16 = desc->dtype_bc == M3_BF16;
  p.vec4 = !p.du_bf16 && (desc->d_inner % 4) == 0 && ld_dt % 4 == 0 && aligned(dt, 16) &&
           aligned(delta, 16) && (!dt_bias || aligned(dt_bias, 16));
  cudaError_t e = launch_step_inputs(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

namespace {
// [a, a + an) and [b, b + bn) bytes intersect
bool spans_overlap(const void* a, size_t an, const void* b, size_t bn) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return a && b && x < y + bn && y < x + an;
}
size_t rows_span(int64_t rows, int64_t ld, int64_t width) {
  return (size_t)((rows - 1) * ld + width) * sizeof(float);
}
}  // namespace

int m3_rows_linear(int32_t rows, int32_t d_in, int32_t d_out, const float* x, int64_t ld_x,
                   const float* norm_w, float eps, const float* W, const float* bias,
                   const float* residual, int64_t ld_r, int32_t split, int32_t silu,
                   float* out0, int64_t ld0, float* out1, int64_t ld1, int32_t overlap,
                   void* stream) {
  if (rows < 1 || d_in < 4 || d_out < 1 || split < 0 || split > d_out) return M3_ERR_SHAPE;
  if (rows > kSmallRows || d_in % 4 != 0 ||
      (int64_t)small_rows_pad(rows) * d_in > kSmallStage)
    return M3_ERR_UNSUPPORTED;
  if (!x || !W || (split > 0 && !out0) || (split < d_out && !out1)) return M3_ERR_NULL;
  if (ld_x < d_in || (residual && ld_r < d_out) || (split > 0 && ld0 < split) ||
      (split < d_out && ld1 < d_out - split))
    return M3_ERR_SHAPE;
  if (!aligned(W, 16) || !aligned(x, 4) || (norm_w && !aligned(norm_w, 4)) ||
      (bias && !aligned(bias, 4)) || (residual && !aligned(residual, 4)) ||
      (out0 && !aligned(out0, 4)) || (out1 && !aligned(out1, 4)))
    return M3_ERR_ALIGN;
  // every CTA stages all of x before writing, but CTAs run in any order: the
  // outputs must not overlap the input (the residual may be out0 itself)
  const size_t xs = rows_span(rows, ld_x, d_in);
  if ((split > 0 && spans_overlap(x, xs, out0, rows_span(rows, ld0, split))) ||
      (split < d_out && spans_overlap(x, xs, out1, rows_span(rows, ld1, d_out - split))))
    return M3_ERR_ALIAS;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  RowsLinearParams p;
  memset(&p, 0, sizeof(p));
  p.x = x; p.ld_x = ld_x; p.norm_w = norm_w; p.eps = eps; p.W = W; p.bias = bias;
  p.residual = residual; p.ld_r = ld_r; p.out0 = out0; p.ld0 = ld0; p.out1 = out1; p.ld1 = ld1;
  p.rows = rows; p.d_in = d_in; p.d_out = d_out; p.split = split; p.silu = silu != 0;
  p.pdl = overlap != 0;
  p.vec = aligned(x, 16) && ld_x % 4 == 0 && (!norm_w || aligned(norm_w, 16));
  cudaError_t e = launch_rows_linear(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_xdt_proj(int32_t rows, int32_t d_inner, int32_t n_x, int32_t dt_rank, const float* u,
                const float* W_x, const float* b_x, const float* W_dt, float* x_dbl, float* dt,
                int32_t overlap, void* stream) {
  if (rows < 1 || d_inner < 4 || dt_rank < 1 || n_x < dt_rank) return M3_ERR_SHAPE;
  if (rows > kSmallRows || d_inner % 4 != 0 || dt_rank > kMaxDtRank ||
      (int64_t)small_rows_pad(rows) * (d_inner + dt_rank) > kSmallStage)
    return M3_ERR_UNSUPPORTED;
  if (!u || !W_x || !W_dt || !x_dbl || !dt) return M3_ERR_NULL;
  if (!aligned(W_x, 16) || !aligned(u, 4) || !aligned(W_dt, 4) || (b_x && !aligned(b_x, 4)) ||
      !aligned(x_dbl, 4) || !aligned(dt, 4))
    return M3_ERR_ALIGN;
  const size_t us = (size_t)rows * d_inner * sizeof(float);
  const size_t xs = (size_t)rows * n_x * sizeof(float);
  if (spans_overlap(u, us, x_dbl, xs) || spans_overlap(u, us, dt, us) ||
      spans_overlap(x_dbl, xs, dt, us))
    return M3_ERR_ALIAS;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  XdtParams p;
  memset(&p, 0, sizeof(p));
  p.u = u; p.Wx = W_x; p.bx = b_x; p.Wdt = W_dt; p.x_dbl = x_dbl; p.dt = dt;
  p.rows = rows; p.D = d_inner; p.n_x = n_x; p.r = dt_rank;
  p.pdl = overlap != 0;
  p.vec = aligned(u, 16);
  cudaError_t e = launch_xdt_proj(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_silu(int64_t rows, int32_t d, const float* x, int64_t ld_x, float* out, void* stream) {
  if (rows < 1 || d < 1 || ld_x < d) return M3_ERR_SHAPE;
  if (!x || !out) return M3_ERR_NULL;
  if (!aligned(x, 4) || !aligned(out, 4)) return M3_ERR_ALIGN;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  SiluParams p;
  memset(&p, 0, sizeof(p));
  p.x = x; p.ld_x = ld_x; p.out = out; p.rows = rows; p.D = d;
  p.vec4 = d % 4 == 0 && ld_x % 4 == 0 && aligned(x, 16) && aligned(out, 16);
  cudaError_t e = launch_silu(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

size_t m3_step_inputs_bwd_workspace_bytes(const m3_step_desc* desc, int32_t mimo_p) {
  if (!desc || desc->batch < 1 || desc->d_state < 1 || mimo_p < 1) return 0;
  const size_t np = (size_t)desc->d_state * mimo_p;
  return (size_t)step_inputs_bwd_ctas(desc->batch) * 2 * np * sizeof(float);
}

int m3_step_inputs_bwd(const m3_step_desc* desc, int32_t mimo_p, const void* dt,
                       int64_t ld_dt, const void* xbc, int64_t ld_x, int32_t off_b,
                       int32_t off_c, const float* wb, const float* wc, float eps,
                       const void* g_delta, const void* g_Bc, const void* g_Cc,
                       void* d_dt, void* d_xbc, float* d_wb, float* d_wc, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (!desc) return M3_ERR_NULL;
  const int64_t np = (int64_t)desc->d_state * mimo_p;
  if (desc->batch < 1 || desc->d_inner < 1 || desc->d_state < 1 || mimo_p < 1 ||
      ld_dt < desc->d_inner || off_b < 0 || off_c < 0 || off_b + np > ld_x ||
      off_c + np > ld_x || !(eps >= 0.f) || np * 2 * 8 * 4 > 200 * 1024)
    return M3_ERR_SHAPE;
  if (!dt || !xbc || !g_delta || !g_Bc || !g_Cc || !d_dt || !d_xbc ||
      ((wb == nullptr) != (wc == nullptr)) || (wb && (!d_wb || !d_wc)))
    return M3_ERR_NULL;
  if (!dtype_ok(desc->dtype_du) || !dtype_ok(desc->dtype_bc)) return M3_ERR_DTYPE;
  const int esd = dsize(desc->dtype_du), esb = dsize(desc->dtype_bc);
  if (!aligned(dt, esd) || !aligned(xbc, esb) || !aligned(g_delta, esd) || !aligned(g_Bc, esb) ||
      !aligned(g_Cc, esb) || !aligned(d_dt, esd) || !aligned(d_xbc, esb) ||
      (wb && (!aligned(wb, 4) || !aligned(wc, 4) || !aligned(d_wb, 4) || !aligned(d_wc, 4))))
    return M3_ERR_ALIGN;
  if (wb && (!workspace || workspace_bytes < m3_step_inputs_bwd_workspace_bytes(desc, mimo_p)))
    return M3_ERR_WORKSPACE;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  InputsBwdParams p;
  memset(&p, 0, sizeof(p));
  p.dt = dt; p.ld_dt = ld_dt; p.xbc = xbc; p.ld_x = ld_x; p.off_b = off_b; p.off_c = off_c;
  p.wb = wb; p.wc = wc; p.eps = eps; p.g_delta = g_delta; p.g_Bc = g_Bc; p.g_Cc = g_Cc;
  p.d_dt = d_dt; p.d_xbc = d_xbc; p.d_wb = d_wb; p.d_wc = d_wc;
  p.part_w = static_cast<float*>(workspace);
  p.rows = desc->batch; p.D = desc->d_inner; p.N = desc->d_state; p.P = mimo_p;
  p.du_bf16 = desc->dtype_du == M3_BF16;
  p.x_bf16 = p.gbc_bf16 = desc->dtype_bc == M3_BF16;
  cudaError_t e = launch_step_inputs_bwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_gate(int64_t rows, int32_t d_inner, const float* y, const void* u, int32_t dtype_u,
            const float* z, int64_t ld_z, const float* d_skip, float coef, float* out,
            void* stream) {
  return m3_gate_typed(rows, d_inner, y, M3_F32, u, dtype_u, z, M3_F32, ld_z, d_skip, coef, 0,
                       out, M3_F32, stream);
}

int m3_gate_typed(int64_t rows, int32_t d_inner, const void* y, int32_t dtype_y, const void* u,
                  int32_t dtype_u, const void* z, int32_t dtype_z, int64_t ld_z,
                  const float* d_skip, float coef, int32_t round_silu, void* out,
                  int32_t dtype_out, void* stream) {
  if (rows < 1 || d_inner < 1 || ld_z < d_inner) return M3_ERR_SHAPE;
  if (!dtype_ok(dtype_y) || !dtype_ok(dtype_u) || !dtype_ok(dtype_z) || !dtype_ok(dtype_out))
    return M3_ERR_DTYPE;
  if (!y || !u || !z || !d_skip || !out) return M3_ERR_NULL;
  if (!aligned(y, dsize(dtype_y)) || !aligned(u, dsize(dtype_u)) || !aligned(z, dsize(dtype_z)) ||
      !aligned(d_skip, 4) || !aligned(out, dsize(dtype_out)))
    return M3_ERR_ALIGN;
  // out may alias y only when both have the same element type (in place)
  if (out == y && dtype_out != dtype_y) return M3_ERR_ALIAS;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  GateParams p;
  memset(&p, 0, sizeof(p));
  p.y = y; p.y_bf16 = dtype_y == M3_BF16;
  p.u = u; p.u_bf16 = dtype_u == M3_BF16;
  p.z = z; p.z_bf16 = dtype_z == M3_BF16; p.ld_z = ld_z;
  p.d_skip = d_skip; p.coef = coef;
  p.out = out; p.out_bf16 = dtype_out == M3_BF16;
  p.rows = rows; p.D = d_inner;
  p.round_silu = round_silu != 0;
  cudaError_t e = launch_gate(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

size_t m3_gate_bwd_workspace_bytes(int64_t rows, int32_t d_inner) {
  if (rows < 1 || d_inner < 1) return 0;
  return (size_t)gate_bwd_row_ctas(rows, d_inner) * d_inner * sizeof(float);
}

int m3_gate_bwd(int64_t rows, int32_t d_inner, const void* y, int32_t dtype_y, const void* u,
                int32_t dtype_u, const void* z, int32_t dtype_z, int64_t ld_z,
                const float* d_skip, float coef, int32_t round_silu, const void* g,
                int32_t dtype_g, void* d_y, void* d_u, void* d_z, float* d_dskip,
                void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 1 || d_inner < 1 || ld_z < d_inner) return M3_ERR_SHAPE;
  if (!dtype_ok(dtype_y) || !dtype_ok(dtype_u) || !dtype_ok(dtype_z) || !dtype_ok(dtype_g))
    return M3_ERR_DTYPE;
  if (!y || !u || !z || !d_skip || !g || !d_y || !d_u || !d_z || !d_dskip) return M3_ERR_NULL;
  if (!workspace || workspace_bytes < m3_gate_bwd_workspace_bytes(rows, d_inner))
    return M3_ERR_WORKSPACE;
  if (!aligned(y, dsize(dtype_y)) || !aligned(u, dsize(dtype_u)) || !aligned(z, dsize(dtype_z)) ||
      !aligned(g, dsize(dtype_g)) || !aligned(d_y, dsize(dtype_y)) ||
      !aligned(d_u, dsize(dtype_u)) || !aligned(d_z, dsize(dtype_z)) || !aligned(d_skip, 4) ||
      !aligned(d_dskip, 4) || !aligned(workspace, 4))
    return M3_ERR_ALIGN;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  GateBwdParams p;
  memset(&p, 0, sizeof(p));
  p.y = y; p.y_bf16 = dtype_y == M3_BF16;
  p.u = u; p.u_bf16 = dtype_u == M3_BF16;
  p.z = z; p.z_bf16 = dtype_z == M3_BF16; p.ld_z = ld_z;
  p.d_skip = d_skip; p.coef = coef; p.round_silu = round_silu != 0;
  p.g = g; p.g_bf16 = dtype_g == M3_BF16;
  p.dy = d_y; p.du = d_u; p.dz = d_z;
  p.part = static_cast<float*>(workspace); p.d_dskip = d_dskip;
  p.rows = rows; p.D = d_inner;
  p.gx = gate_bwd_row_ctas(rows, d_inner);
  cudaError_t e = launch_gate_bwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH;
}

int m3_device_error(int32_t* code, int32_t clear) {
  if (!code) return M3_ERR_NULL;
  int rc = check_device();
  if (rc != M3_OK) return rc;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_err_word, sizeof(int)) != cudaSuccess) return M3_ERR_LAUNCH;
  *code = v;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_err_word, &z, sizeof(int)) != cudaSuccess) return M3_ERR_LAUNCH;
  }
  return M3_OK;
}

}  // extern "C"
