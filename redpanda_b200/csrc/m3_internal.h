// Internal launch interface shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// M3_GS_CHUNK: steps per backward chunk (= forward checkpoint interval) of the
// tilings that keep the gates in Tensor Memory; M3_BWD_MIN_BLOCKS caps the
// backward's CTAs per SM the compiler budgets registers for (0: as many as
// Tensor Memory allows).  Tuning knobs; the defaults are the measured best.
#ifndef M3_GS_CHUNK
#define M3_GS_CHUNK 8
#endif
#ifndef M3_BWD_MIN_BLOCKS
#define M3_BWD_MIN_BLOCKS 0
#endif

namespace m3 {

// Per-thread lane tiling: R rotational + T tracking lanes per channel, ND
// channels per thread, 4 threads per channel group, 128 threads per CTA.
struct Tile {
  int R, T, ND;      // ND: channels per thread in the forward and step kernels
  int NDB, NTHB;     // backward: channels per thread, threads per CTA
  int GS;            // backward keeps the gates in Tensor Memory (8-step chunks)
  int cki() const { return GS ? M3_GS_CHUNK : 16; }   // checkpoint interval = backward chunk
  // Tensor Memory columns of one backward CTA (the kernel's BwdCfg::NCOLS) and
  // the backward CTAs that fit on one SM by Tensor Memory (512 columns)
  int bwd_cols() const {
    const int c = NDB * (R + T) + (GS ? NDB * R * 2 : 0);
    int cs = 1;
    while (cs < c) cs <<= 1;
    const int cols = (NTHB / 128) * cki() * cs;
    return cols < 32 ? 32 : cols;
  }
  int bwd_ctas_per_sm() const { const int n = 512 / bwd_cols(); return n < 1 ? 1 : n; }
  int nl() const { return R + T; }
  int np() const { return 4 * (R + T); }       // padded state lanes per channel
  int dt() const { return 32 * ND; }           // forward channels per CTA
  int dt_bwd() const { return NTHB / 4 * NDB; }  // backward channels per CTA
};

// Tile chosen for a (n_rot, n_track) split; identical for scan, backward and
// step so that their arithmetic (and the y reduction order) agrees.
bool select_tile(int n_rot, int n_track, Tile* out);

struct FwdParams {
  const void* delta; const void* u; const void* Bc; const void* Cc;
  const float* Ar; const float* Ai; const float* Tk;
  void* y; float* ckpt; float* h_last; float* dbu_last;
  int y_bf16;      // y is bf16 (else fp32); fp32 state and accumulation either way
  int B, L, D, N, NR, NT;
  int dt_du, dt_bc;
  int direction;   // 0 fwd, 1 rev, 2 bidir
  int nch;         // chunks of kCK steps
  int cki, nck;    // checkpoint interval (8 or 16 steps) and checkpoints per direction
  int async_ok;    // cp.async staging allowed (alignment checked on the host)
  int bulk;        // every staged row is a 16-byte aligned bulk copy
  // fused prologue (pro != 0, bf16 bulk path only): delta points at dt, the
  // dt_proj output before softplus, and Bc/Cc are unused; B_raw and C_raw are
  // columns [off_b, off_b + N*P) and [off_c, off_c + N*P) of the bf16 rows xbc
  // (B*L, ld_x); delta = bf16(softplus(dt)), Bc/Cc = bf16(MIMO fold of BCNorm)
  int pro;
  const void* xbc; long long ld_x; int off_b, off_c, P;
  const float* wb; const float* wc; float eps;
  int* err;
};

struct BwdParams {
  const void* delta; const void* u; const void* Bc; const void* Cc;
  const float* Ar; const float* Ai; const float* Tk;
  const void* dy; const float* ckpt;
  void* d_delta; void* d_u;
  float* part_bc;     // [G][ndirs][B][L][2][NL][4 quarters]
  float* part_a;      // [Bg][3][D][NP]
  float* scratch_du;  // [G*Bg][L][DT][2]  (bidirectional only)
  int B, L, D, N, NR, NT;
  int dt_du, dt_bc, dt_dy;
  int direction;
  int nch;            // chunks of the tile's checkpoint interval
  int G, Bg;
  int async_du, async_dy;   // cp.async staging allowed for delta/u and dy
  int bulk;                 // every staged row is a 16-byte aligned bulk copy
  // fused prologue (pro != 0; bf16 bulk path only): delta points at dt and
  // d_delta receives d dt; Bc/Cc are unused (see FwdParams)
  int pro;
  const void* xbc; long long ld_x; int off_b, off_c, P;
  const float* wb; const float* wc; float eps;
  int* err;
};

struct StepParams {
  float* h; float* dbu;                       // full state (dbu unused when factored)
  const float* fac_in; float* fac_out;        // factored state: [delta*u | B], (B, D + N)
  int factored;
  int vec_bc;                                 // Bc/Cc 16-byte aligned: vector row loads
  int vec_fac;                                // factors 16-byte aligned, D % 4 == 0
  int bulk;                                   // pipelined bulk-copy kernel eligible
  int gated;                                  // y -> (y + u*d_skip) * silu(z)
  const float* z; long long ld_z;             // (B, ld_z) pre-activation gate
  const float* d_skip;                        // (D,) skip weight
  const void* delta; const void* u; const void* Bc; const void* Cc;
  const float* Ar; const float* Ai; const float* Tk;
  float* y;
  int B, D, N, NR, NT;
  int dt_du, dt_bc;
  int* err;
  // pro: the step's prologue fused into the pipelined kernel -- delta =
  // softplus(dt) and Bc/Cc = BCNorm + MIMO fold of the raw x_proj rows, with
  // the device functions of step_inputs_kernel (m3_prologue.cuh); fp32 dt and
  // rows; `delta`, `Bc`, `Cc` are unused then
  int pro;
  const float* dt; long long ld_dt;
  const float* dt_bias;                       // (D,) or nullptr: delta = softplus(dt + bias)
  const float* xbc; long long ld_x;
  int off_b, off_c, P;
  const float* wb; const float* wc;
  float eps;
  // pro with the dt product: dt = xbc[:, :dt_rank] wdt^T computed in the
  // kernel (dt_proj, wdt (D, dt_rank) row-major); `dt` is unused then
  const float* wdt; int dt_rank;
  int pdl;                                    // programmatic dependent launch (bulk kernel)
};

struct ReduceParams {
  const float* part_bc; const float* part_a;
  void* d_Bc; void* d_Cc;
  float* dAr; float* dAi; float* dTk;
  int B, L, D, N, NR, NT;
  int dt_bc;
  int G, Bg;
  int ndirs;          // direction slots of part_bc
  int bc_f32_of_bf16; // d_Bc/d_Cc are fp32 buffers receiving the bf16-rounded sums
};

cudaError_t launch_scan_fwd(const Tile& t, const FwdParams& p, cudaStream_t s);
cudaError_t launch_scan_bwd(const Tile& t, const BwdParams& p, cudaStream_t s);
cudaError_t launch_bwd_reduce(const Tile& t, const ReduceParams& p, cudaStream_t s);
cudaError_t launch_step(const Tile& t, const StepParams& p, cudaStream_t s);

struct InputsParams {
  const void* dt; long long ld_dt;        // (B, ld_dt): dt_proj output before softplus
  const float* dt_bias;                   // (D,) dt_proj bias added first, or nullptr
  int vec4;                               // fp32 dt rows, bias and delta as float4
  const void* xbc; long long ld_x;        // (B, ld_x): row of x_proj output
  int off_b, off_c;                       // column offsets of B_raw and C_raw (N*p each)
  const float* wb; const float* wc;       // (N*p,) BCNorm weights
  float eps;
  void* delta; void* Bc; void* Cc;        // (B, D), (B, N), (B, N)
  int du_bf16;                            // dt and delta are bf16 (else fp32)
  int bc_bf16;                            // xbc, Bc and Cc are bf16 (else fp32)
  int B, D, N, P;
};
cudaError_t launch_step_inputs(const InputsParams& p, cudaStream_t s);

struct SiluParams {
  const float* x; long long ld_x;         // (rows, ld_x)
  float* out;                             // (rows, D) contiguous
  long long rows; int D;
  int vec4;                               // x rows and out as float4
};
cudaError_t launch_silu(const SiluParams& p, cudaStream_t s);

struct InputsBwdParams {
  const void* dt; long long ld_dt;        // nullptr: skip the softplus part
  const void* xbc; long long ld_x;        // float, or bf16 when x_bf16
  int x_bf16;                             // xbc and d_xbc are bf16
  int gbc_bf16;                           // g_Bc and g_Cc are bf16
  int du_bf16;                            // dt, g_delta and d_dt are bf16
  int off_b, off_c;
  const float* wb; const float* wc;
  float eps;
  const void* g_delta; const void* g_Bc; const void* g_Cc;      // (rows, D), (rows, N) x2
  void* d_dt; void* d_xbc;                                      // (rows, D), (rows, ld_x)
  float* d_wb; float* d_wc;                                     // (N*P,) each
  float* part_w;                                                // [ctas][2][N*P]
  long long rows; int D, N, P;
};
int step_inputs_bwd_ctas(long long rows);
cudaError_t launch_step_inputs_bwd(const InputsBwdParams& p, cudaStream_t s);

struct GateParams {
  const void* y; int y_bf16;
  const void* u; int u_bf16;
  const void* z; int z_bf16; long long ld_z;
  const float* d_skip; float coef;
  void* out; int out_bf16;
  long long rows; int D;
  int round_silu;                             // silu(z) rounded to bf16 when z is bf16
};
cudaError_t launch_gate(const GateParams& p, cudaStream_t s);

// Backward of out = (y + coef*u*d_skip) * silu(z) over (rows, D).
struct GateBwdParams {
  const void* y; int y_bf16;
  const void* u; int u_bf16;
  const void* z; int z_bf16; long long ld_z;
  const float* d_skip; float coef; int round_silu;
  const void* g; int g_bf16;                  // (rows, D) gradient of out
  void* dy; void* du; void* dz;               // (rows, D), element types of y, u, z
  float* part;                                // (gx, D) partial sums of d d_skip
  float* d_dskip;                             // (D,)
  long long rows; int D;
  int gx;                                     // CTAs along the rows
};
int gate_bwd_row_ctas(long long rows, int d);
cudaError_t launch_gate_bwd(const GateBwdParams& p, cudaStream_t s);

// Small-batch projections of the step layer (m3_gemv.cu): rows <= kSmallRows.
constexpr int kSmallRows = 8;
constexpr int kSmallStage = 12288;            // staged input floats per CTA (48 KB)
int small_rows_pad(int rows);                 // rows rounded up to the compiled 1, 2, 4, 8
constexpr int kMaxDtRank = 64;                // dt_rank limit of the small-batch dt product

// out = act(residual + bias + norm(x) W^T), columns [0, split) to out0 (silu
// when silu), [split, d_out) to out1.
struct RowsLinearParams {
  const float* x; long long ld_x;             // (rows, d_in)
  const float* norm_w; float eps;             // RMSNorm weight or nullptr
  const float* W;                             // (d_out, d_in) row-major
  const float* bias;                          // (d_out,) or nullptr
  const float* residual; long long ld_r;      // (rows, d_out) or nullptr
  float* out0; long long ld0;
  float* out1; long long ld1;
  int rows, d_in, d_out, split, silu;
  int pdl;                                    // programmatic dependent launch
  int vec;                                    // x rows and norm_w 16-byte aligned
};
cudaError_t launch_rows_linear(const RowsLinearParams& p, cudaStream_t s);

// x_dbl = u W_x^T + b_x and dt = x_dbl[:, :r] W_dt^T in one launch.
struct XdtParams {
  const float* u;                             // (rows, D) contiguous
  const float* Wx; const float* bx;           // (n_x, D), (n_x,) or nullptr
  const float* Wdt;                           // (D, r)
  float* x_dbl;                               // (rows, n_x)
  float* dt;                                  // (rows, D)
  int rows, D, n_x, r;
  int pdl;                                    // programmatic dependent launch
  int vec;                                    // u 16-byte aligned
};
cudaError_t launch_xdt_proj(const XdtParams& p, cudaStream_t s);

// device error word of the current device
int* device_err_ptr();

}  // namespace m3
