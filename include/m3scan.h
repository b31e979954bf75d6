/*
 * m3scan.h - C ABI of the B200 (sm_100a) Mamba-3 trapezoidal selective scan.
 *
 * Drop-in kernels for the hot path of PranavPrasannaV/RedPanda's Mamba-3
 * backbone.  Every entry point takes plain device pointers, sizes and a CUDA
 * stream (passed as void*), returns 0 or an M3_ERR_* code, never throws,
 * never allocates and never frees: the caller owns every input, output and
 * workspace buffer.  All pointers are device pointers to dense, row-major
 * (contiguous) tensors.
 *
 * Interface map (reference file:line -> entry point):
 *   redpanda/engine/triton_scan.py:248-281  _TrapezoidalScanFn.forward  -> m3_scan_fwd
 *   redpanda/engine/triton_scan.py:283-315  _TrapezoidalScanFn.backward -> m3_scan_bwd
 *   redpanda/engine/mamba.py:254-260        bidirectional scan pair     -> m3_scan_fwd/bwd with
 *                                                                          M3_DIR_BIDIR
 *   redpanda/engine/mamba.py:343,377-379    return_state (h_last, dBu_last) -> m3_scan_fwd h_last/dbu_last
 *   redpanda/engine/mamba.py:466-493        Mamba3Block.step recurrence -> m3_step
 *   redpanda/engine/mamba.py:455-469        step inputs (softplus, BCNorm, MIMO fold) -> m3_step_inputs
 *   redpanda/engine/mamba.py:490-497        step + gated output (y + u*D) * silu(z) -> m3_step_gated
 *   redpanda/engine/mamba.py:455-497        step inputs + step + gated output in one launch
 *                                           -> m3_step_gated_fused (+ dt_proj: _proj)
 *   redpanda/engine/mamba.py:262-265        (y + u*D) * silu(z) after a scan -> m3_gate
 *                                           and its autograd backward -> m3_gate_bwd
 *   redpanda/engine/mamba.py:243, 452       u = silu(x half of in_proj) -> m3_silu
 *   redpanda/engine/mamba.py:82-89, 450-452 RMSNorm + in_proj + silu, small batch -> m3_rows_linear
 *   redpanda/engine/mamba.py:454, 463       x_proj + dt_proj product, small batch -> m3_xdt_proj
 *   redpanda/engine/mamba.py:497, 591-595   out_proj + residual add, small batch -> m3_rows_linear
 *
 * Shapes (B batch, L length, D = d_inner, N = d_state, n_rot rotational lanes,
 * N - n_rot tracking lanes):
 *   delta, u            (B, L, D)  dtype_du  (post-softplus delta, SSM input)
 *   Bc, Cc              (B, L, N)  dtype_bc  (MIMO-contracted, BCNorm'ed B and C)
 *   A_real_p, A_imag_p  (D, N)     float32   rotational eigenvalues in columns
 *                                            [0, n_rot), zero elsewhere
 *   track_p             (D, N)     float32   tanh(theta) in columns [n_rot, N)
 *   (the padded parameter layout of triton_scan.py:325-335)
 *   y                   (B, L, D)  float32   scan output WITHOUT the u*D skip
 */
#ifndef M3SCAN_H
#define M3SCAN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define M3_API __attribute__((visibility("default")))
#else
#define M3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum { M3_F32 = 0, M3_BF16 = 1 };

/* scan directions.  M3_DIR_REV scans the sequence back to front, which equals
 * flip(scan(flip(x))) of the reference (mamba.py:258-260); M3_DIR_BIDIR writes
 * y_fwd + y_rev in one launch. */
enum { M3_DIR_FWD = 0, M3_DIR_REV = 1, M3_DIR_BIDIR = 2 };

/* status codes */
enum {
  M3_OK = 0,
  M3_ERR_NULL = 1,         /* a required pointer is NULL */
  M3_ERR_SHAPE = 2,        /* a size is out of range */
  M3_ERR_DTYPE = 3,        /* unsupported element type */
  M3_ERR_UNSUPPORTED = 4,  /* no compiled kernel serves this shape (a (d_state, n_rot)
                              split, or a size past a kernel's stated limit) */
  M3_ERR_ALIGN = 5,        /* a pointer is not aligned to its element size */
  M3_ERR_WORKSPACE = 6,    /* workspace missing or too small */
  M3_ERR_LAUNCH = 7,       /* the CUDA launch failed (see cudaGetLastError) */
  M3_ERR_DEVICE = 8,       /* a kernel recorded a device-side error */
  M3_ERR_NO_DEVICE = 9,    /* no CUDA device / the current device is not sm_100 */
  M3_ERR_SCRATCH_LIMIT = 10, /* m3_scan_bwd_noalloc: the problem needs more scratch than
                                M3_NOALLOC_SCRATCH_BYTES */
  M3_ERR_ALIAS = 11          /* two buffers that must be distinct overlap */
};

typedef struct m3_scan_desc {
  int32_t batch;      /* B >= 1 */
  int32_t seqlen;     /* L >= 1 */
  int32_t d_inner;    /* D >= 1 */
  int32_t d_state;    /* N, 1..128 */
  int32_t n_rot;      /* 0..N rotational lanes; N - n_rot tracking lanes */
  int32_t dtype_du;   /* element type of delta and u (M3_F32 or M3_BF16) */
  int32_t dtype_bc;   /* element type of Bc and Cc */
  int32_t direction;  /* M3_DIR_FWD, M3_DIR_REV or M3_DIR_BIDIR */
} m3_scan_desc;

typedef struct m3_step_desc {
  int32_t batch;      /* rows advanced in lockstep */
  int32_t d_inner;
  int32_t d_state;
  int32_t n_rot;
  int32_t dtype_du;
  int32_t dtype_bc;
} m3_step_desc;

/* Human-readable text of a status code (static storage). */
M3_API const char* m3_strerror(int code);

/* ABI version: (major << 16) | minor. */
M3_API int m3_version(void);

/* Number of float32 elements of the forward checkpoint buffer the backward
 * consumes: the state every 8 steps for the (16 rotational + 16 tracking)
 * lane layout, every 16 steps otherwise; 0 when L fits one interval.  The
 * buffer must be 16-byte aligned.  Replaces the hck/dck chunk checkpoints that
 * triton_scan.py:261-262 allocates. */
M3_API size_t m3_scan_ckpt_floats(const m3_scan_desc* desc);

/* Forward scan.  Replaces _TrapezoidalScanFn.forward (triton_scan.py:248-281)
 * and the return_state branch of _selective_scan_trapezoidal (mamba.py:377-379).
 *   y         required, (B, L, D) float32
 *   ckpt      optional (NULL = inference only); m3_scan_ckpt_floats() floats,
 *             16-byte aligned, to be handed to m3_scan_bwd
 *   h_last,   optional, (B, D, N) float32: state after the last token of the
 *   dbu_last  scan direction (M3_DIR_FWD or M3_DIR_REV only) */
M3_API int m3_scan_fwd(const m3_scan_desc* desc,
                const void* delta, const void* u, const void* Bc, const void* Cc,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                float* y, float* ckpt, float* h_last, float* dbu_last,
                void* stream);

/* m3_scan_fwd with the element type of y chosen by dtype_y (M3_F32 or
 * M3_BF16); the state and every accumulation stay fp32 and only the stored y
 * is rounded.  Replaces the same _TrapezoidalScanFn.forward
 * (triton_scan.py:248-281) for a bf16 layer (the reference's autocast
 * training, train.py:268, and the bf16 Eval-Mamba forward of model.py:110-132).
 * With M3_DIR_BIDIR and a bf16 y the first direction's partial is stored in
 * bf16 and the second adds to it in fp32 before rounding again (at most one
 * bf16 ulp more than a single rounding). */
M3_API int m3_scan_fwd_typed(const m3_scan_desc* desc,
                const void* delta, const void* u, const void* Bc, const void* Cc,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                void* y, int32_t dtype_y, float* ckpt, float* h_last, float* dbu_last,
                void* stream);

/* Forward scan with the layer's prologue fused into its staging
 * (mamba.py:284-301 and 336-337, the projections' softplus, BCNorm and MIMO
 * fold that otherwise run before the scan).  bf16 inputs only (the
 * config-1/2 element types; desc->dtype_du must be M3_BF16, dtype_bc is
 * ignored):
 *   dt      (B, L, D) bf16: dt_proj output including its bias, before softplus
 *   xbc     (B*L, ld_x) bf16: x_proj output rows; B_raw = columns
 *           [off_b, off_b + N*mimo_p), C_raw = [off_c, off_c + N*mimo_p)
 *   wb, wc  (N*mimo_p,) float32 BCNorm weights, or both NULL (use_bcnorm=False)
 *   u       (B, L, D) bf16
 * The scan sees delta = bf16(softplus(dt)) and Bc, Cc = bf16 of the fold of
 * BCNorm(B_raw), BCNorm(C_raw) (computed in fp32 as m3_step_inputs does), so
 * y and ckpt equal those of m3_step_inputs + casts to bf16 + m3_scan_fwd_typed
 * bit for bit.  Shapes the staging cannot take (column offsets off 8-element
 * boundaries, N*mimo_p above 256, channel counts off the tile) return
 * M3_ERR_UNSUPPORTED: run the unfused pair then. */
M3_API int m3_scan_fwd_fused(const m3_scan_desc* desc, int32_t mimo_p, const void* dt,
                const void* xbc, int64_t ld_x, int32_t off_b, int32_t off_c,
                const float* wb, const float* wc, float eps, const void* u,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                void* y, int32_t dtype_y, float* ckpt, void* stream);

/* Workspace bytes m3_scan_bwd needs on the current device. */
M3_API size_t m3_scan_bwd_workspace_bytes(const m3_scan_desc* desc);

/* Analytic backward.  Replaces _TrapezoidalScanFn.backward
 * (triton_scan.py:283-315) with deterministic reductions (no atomics).
 *   dy        (B, L, D) of dtype_dy, the gradient of y
 *   ckpt      the forward's checkpoint buffer (NULL allowed when
 *             m3_scan_ckpt_floats() is 0)
 *   d_delta, d_u   (B, L, D) of dtype_du
 *   d_Bc, d_Cc     (B, L, N) of dtype_bc
 *   d_A_real_p, d_A_imag_p, d_track_p   (D, N) float32 in the padded layout
 *   workspace      >= m3_scan_bwd_workspace_bytes(desc) bytes */
M3_API int m3_scan_bwd(const m3_scan_desc* desc,
                const void* delta, const void* u, const void* Bc, const void* Cc,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                const void* dy, int32_t dtype_dy, const float* ckpt,
                void* d_delta, void* d_u, void* d_Bc, void* d_Cc,
                float* d_A_real_p, float* d_A_imag_p, float* d_track_p,
                void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of m3_scan_bwd_fused on the current device. */
M3_API size_t m3_scan_bwd_fused_workspace_bytes(const m3_scan_desc* desc, int32_t mimo_p);

/* Analytic backward of m3_scan_fwd_fused: the scan's backward with the
 * prologue's backward fused in (the gradients torch's softplus, RMSNorm and
 * sum give for mamba.py:284-301 and 336-337).  Inputs as m3_scan_fwd_fused,
 * plus dy (B, L, D) of dtype_dy and the forward's ckpt.  Outputs:
 *   d_dt    (B, L, D) bf16: softplus'(dt) times the bf16-rounded d delta
 *   d_u     (B, L, D) bf16
 *   d_xbc   (B*L, ld_x) bf16: the B_raw and C_raw columns are written; the
 *           caller zero-fills the rest (the dt_raw columns get their gradient
 *           through dt_proj)
 *   d_wb, d_wc (N*mimo_p,) float32 BCNorm weight gradients (fixed-order sums)
 *   d_A_real_p, d_A_imag_p, d_track_p  as m3_scan_bwd
 * Every output equals, bit for bit, what the unfused bf16 layer's backward
 * (m3_scan_bwd on the bf16 delta/Bc/Cc, then m3_step_inputs_bwd on the fp32
 * values of their bf16 gradients) produces. */
M3_API int m3_scan_bwd_fused(const m3_scan_desc* desc, int32_t mimo_p, const void* dt,
                const void* xbc, int64_t ld_x, int32_t off_b, int32_t off_c,
                const float* wb, const float* wc, float eps, const void* u,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                const void* dy, int32_t dtype_dy, const float* ckpt, void* d_dt, void* d_u,
                void* d_xbc, float* d_wb, float* d_wc, float* d_A_real_p, float* d_A_imag_p,
                float* d_track_p, void* workspace, size_t workspace_bytes, void* stream);

/* O(1) recurrent step of B rows, in place.  Replaces the recurrence of
 * Mamba3Block.step (mamba.py:466-493):
 *   h, dbu    (B, D, N) float32, read and overwritten with the new state
 *   delta, u  (B, D) of dtype_du;  Bc, Cc  (B, N) of dtype_bc
 *   y         (B, D) float32, sum_n h*C without the u*D skip
 * Bit-identical to m3_scan_fwd (M3_DIR_FWD) at every position when fed the
 * same per-token inputs and the scan's state. */
M3_API int m3_step(const m3_step_desc* desc, float* h, float* dbu,
            const void* delta, const void* u, const void* Bc, const void* Cc,
            const float* A_real_p, const float* A_imag_p, const float* track_p,
            float* y, void* stream);

/* O(1) step with the factored state: the same recurrence as m3_step with half
 * its HBM traffic.  The state is h (B, D, N) fp32, updated in place, and the
 * factors of the last token's input contribution, fac (B, D + N) fp32 =
 * [delta*u (D) | B (N)], read from fac_prev and written to fac_next (distinct
 * buffers; swap them between steps).  dBu = (delta*u)*B is rebuilt with the
 * scan's own rounding, so the outputs equal m3_step's bit for bit.  The
 * factors after a scan are [delta[L-1]*u[L-1] | Bc[L-1]] of its inputs.
 * Extends the cache contract of Mamba3Block.step (mamba.py:487-498), whose
 * dBu tensor it replaces by its two factors. */
M3_API int m3_step_factored(const m3_step_desc* desc, float* h, const float* fac_prev,
            float* fac_next, const void* delta, const void* u, const void* Bc, const void* Cc,
            const float* A_real_p, const float* A_imag_p, const float* track_p,
            float* y, void* stream);

/* The per-token step inputs from the layer's projection outputs, in one launch.
 * Replaces the elementwise part of Mamba3Block.step (mamba.py:455-469):
 *   delta (B, D)  = softplus(dt), torch's threshold 20
 *   Bc, Cc (B, N) = sum over the p MIMO columns of BCNorm(B_raw), BCNorm(C_raw)
 * with BCNorm(x) = x * rsqrt(mean(x^2) + eps) * w over the N*p vector
 * (mamba.py:82-89, 297-299, 336-337).
 *   dt      (B, ld_dt) desc->dtype_du: dt_proj(dt_raw), with its bias or without it
 *   dt_bias (D,) float32 dt_proj bias, added to dt first (one fp32 rounding, as
 *           torch's matmul-then-add), or NULL when dt includes it
 *   xbc     (B, ld_x) desc->dtype_bc: rows of x_proj's output; B_raw starts at
 *           column off_b and C_raw at off_c, N*p columns each
 *   wb, wc  (N*p,) float32 BCNorm weights, or both NULL (use_bcnorm=False: plain sum)
 *   delta   (B, D) desc->dtype_du; Bc, Cc (B, N) desc->dtype_bc
 * Arithmetic is fp32; a bf16 output is rounded once (the bits of the fp32
 * result cast to bf16, as a bf16 layer's casts give).  desc->n_rot is ignored. */
M3_API int m3_step_inputs(const m3_step_desc* desc, int32_t mimo_p,
            const void* dt, int64_t ld_dt, const float* dt_bias, const void* xbc,
            int64_t ld_x, int32_t off_b, int32_t off_c, const float* wb, const float* wc,
            float eps, void* delta, void* Bc, void* Cc, void* stream);

/* u = silu(x) = x / (1 + exp(-x)) over (rows, d) of a row-strided x: the x half
 * of in_proj's output (mamba.py:243, 452), read in place; out (rows, d) float32
 * contiguous. */
M3_API int m3_silu(int64_t rows, int32_t d, const float* x, int64_t ld_x, float* out,
            void* stream);

/* Small-batch projections of the step layer (at most 8 rows; a search node or
 * a few lines), fp32, for the launch-latency-bound regime where each
 * projection is a matrix-vector product.  One warp per output column; sums in
 * a fixed order (deterministic); weights (nn.Linear layout, (d_out, d_in)
 * row-major) 16-byte aligned with d_in % 4 == 0.  rows > 8, or inputs past 48 KB
 * of staged floats (8 rows x 1536, 4 x 3072, ...), return M3_ERR_UNSUPPORTED.
 *
 * m3_rows_linear: out = act(residual + (bias + xn W^T)) with
 *   xn = x * rsqrt(mean(x^2) + eps) * norm_w    (RMSNorm, mamba.py:82-89) when
 *        norm_w != NULL, else x;
 *   columns [0, split) -> out0 (row stride ld0), silu applied when silu != 0
 *        (the x half of in_proj, mamba.py:450-452); columns [split, d_out) ->
 *        out1 (row stride ld1; the z half);
 *   residual (rows, ld_r) or NULL, added last (mamba.py:595); it may be out0
 *        itself (out_proj + residual in place), but no output may overlap x
 *        (M3_ERR_ALIAS).
 * Rounding differs from a cuBLAS GEMM only by the summation order.
 *
 * overlap != 0 (here, in m3_xdt_proj and in m3_step_gated_fused_proj): launch
 * as a programmatic dependent launch, so that the kernel starts while the one
 * ahead of it on the stream finishes (a chain of these calls, as one step
 * layer makes, then pays one launch latency instead of one per call).
 * m3_rows_linear reads the first part of its weight rows W before that kernel
 * has completed: set overlap only when no kernel queued before the call
 * writes W.  Everything else is read after it has completed. */
M3_API int m3_rows_linear(int32_t rows, int32_t d_in, int32_t d_out, const float* x,
            int64_t ld_x, const float* norm_w, float eps, const float* W,
            const float* bias, const float* residual, int64_t ld_r, int32_t split,
            int32_t silu, float* out0, int64_t ld0, float* out1, int64_t ld1,
            int32_t overlap, void* stream);

/* m3_xdt_proj: x_dbl = u W_x^T + b_x  (rows, n_x; mamba.py:454) and
 * dt = x_dbl[:, :dt_rank] W_dt^T  (rows, d_inner; dt_proj without its bias,
 * mamba.py:463 -- m3_step_gated_fused / m3_step_inputs add it) in one launch.
 * u (rows, d_inner) contiguous; W_x (n_x, d_inner); b_x (n_x,) or NULL; W_dt
 * (d_inner, dt_rank), dt_rank <= 64 (else M3_ERR_UNSUPPORTED).  u, x_dbl and dt
 * must not overlap. */
M3_API int m3_xdt_proj(int32_t rows, int32_t d_inner, int32_t n_x, int32_t dt_rank,
            const float* u, const float* W_x, const float* b_x, const float* W_dt,
            float* x_dbl, float* dt, int32_t overlap, void* stream);

/* Workspace bytes of m3_step_inputs_bwd (the BCNorm weight-gradient partials). */
M3_API size_t m3_step_inputs_bwd_workspace_bytes(const m3_step_desc* desc, int32_t mimo_p);

/* Backward of m3_step_inputs over desc->batch rows (the training-path prologue:
 * the gradients that torch's softplus, RMSNorm and sum backward give for
 * mamba.py:284-301 and 336-337):
 *   dt, g_delta, d_dt       (rows, D) of desc->dtype_du; d_dt = g_delta * softplus'(dt)
 *   xbc, d_xbc              (rows, ld_x) of desc->dtype_bc: columns [off_b, off_b + N*p)
 *                           and [off_c, off_c + N*p) of d_xbc are written (the gradients
 *                           of B_raw, C_raw); other columns are left untouched
 *   g_Bc, g_Cc              (rows, N) of desc->dtype_bc: upstream gradients
 *   d_wb, d_wc (N*p,) float32 BCNorm weight gradients, reduced over the rows in a
 *           fixed order (bitwise reproducible); unused when wb == wc == NULL
 *   workspace >= m3_step_inputs_bwd_workspace_bytes(desc, mimo_p) bytes
 * Arithmetic is fp32; bf16 gradients are rounded once. */
M3_API int m3_step_inputs_bwd(const m3_step_desc* desc, int32_t mimo_p,
            const void* dt, int64_t ld_dt, const void* xbc, int64_t ld_x,
            int32_t off_b, int32_t off_c, const float* wb, const float* wc, float eps,
            const void* g_delta, const void* g_Bc, const void* g_Cc,
            void* d_dt, void* d_xbc, float* d_wb, float* d_wc,
            void* workspace, size_t workspace_bytes, void* stream);

/* m3_step (dbu != NULL) or m3_step_factored (fac_prev, fac_next != NULL, dbu
 * NULL) whose output is the layer's gated activation instead of y
 * (mamba.py:493-497):
 *   out (B, D) float32 = (y + u * d_skip) * silu(z),   silu(z) = z / (1 + exp(-z))
 *   z       (B, ld_z) float32: the z half of in_proj's output (before silu)
 *   d_skip  (D,) float32: the layer's skip weight D
 * The state update is identical to m3_step / m3_step_factored. */
M3_API int m3_step_gated(const m3_step_desc* desc, float* h, float* dbu,
            const float* fac_prev, float* fac_next, const void* delta, const void* u,
            const void* Bc, const void* Cc, const float* A_real_p, const float* A_imag_p,
            const float* track_p, const float* z, int64_t ld_z, const float* d_skip,
            float* out, void* stream);

/* m3_step_gated with the step's prologue in the same launch (mamba.py:455-497:
 * softplus(dt_proj), BCNorm of B_raw / C_raw, the MIMO fold, the recurrence and
 * the gated output): the kernel stages each row's dt and raw x_proj rows and
 * computes delta, Bc and Cc itself with the arithmetic of m3_step_inputs, so
 * the state and out are bit-identical to m3_step_inputs followed by
 * m3_step_gated.
 *   dt      (B, ld_dt) float32: dt_proj output, before softplus; dt_bias (D,) or
 *           NULL as for m3_step_inputs
 *   xbc     (B, ld_x) float32: x_proj output; B_raw at column off_b, C_raw at
 *           off_c, N * mimo_p values each
 *   wb, wc  (N * mimo_p,) float32 BCNorm weights, or both NULL (plain fold)
 *   u       (B, D) of desc->dtype_du; desc->dtype_bc must be M3_F32
 * Served by the pipelined step kernel for dense 32-lane states (N = 32, no
 * virtual lanes) with D % 32 == 0, mimo_p <= 2, and 16-byte aligned rows of dt,
 * xbc (ld_x, off_b, off_c multiples of 4), u and the state; any other shape
 * returns M3_ERR_UNSUPPORTED with nothing launched (run m3_step_inputs and
 * m3_step_gated instead). */
M3_API int m3_step_gated_fused(const m3_step_desc* desc, int32_t mimo_p, float* h, float* dbu,
            const float* fac_prev, float* fac_next, const float* dt, int64_t ld_dt,
            const float* dt_bias, const float* xbc, int64_t ld_x, int32_t off_b, int32_t off_c,
            const float* wb, const float* wc, float eps, const void* u,
            const float* A_real_p, const float* A_imag_p, const float* track_p,
            const float* z, int64_t ld_z, const float* d_skip, float* out, void* stream);

/* m3_step_gated_fused with dt_proj's product formed in the kernel too:
 * dt = xbc[:, :dt_rank] W_dt^T (mamba.py:463, the dt_raw columns of x_proj's
 * output times dt_proj's weight, W_dt (D, dt_rank) row-major float32,
 * dt_rank <= 64), then delta = softplus(dt + dt_bias) and the rest as
 * m3_step_gated_fused.  One launch for the whole step after x_proj; the dt sum
 * runs in a fixed order (4 strided partials, then pairs), so results are
 * deterministic but not the bits of a cuBLAS dt_proj. */
M3_API int m3_step_gated_fused_proj(const m3_step_desc* desc, int32_t mimo_p, float* h,
            float* dbu, const float* fac_prev, float* fac_next, const float* W_dt,
            int32_t dt_rank, const float* dt_bias, const float* xbc, int64_t ld_x,
            int32_t off_b, int32_t off_c, const float* wb, const float* wc, float eps,
            const void* u, const float* A_real_p, const float* A_imag_p,
            const float* track_p, const float* z, int64_t ld_z, const float* d_skip,
            float* out, int32_t overlap, void* stream);

/* The layer's gated activation after a scan (mamba.py:262-265), elementwise
 * over (rows, D) = (B*L, D):
 *   out = (y + coef * (u * d_skip)) * silu(z),   silu(z) = z / (1 + exp(-z))
 *   y (rows, D) float32 scan output; u (rows, D) of dtype_u (the SSM input);
 *   z (rows, ld_z) float32, the z half of in_proj's output; d_skip (D,) float32;
 *   coef 1 for one direction, 2 for the bidirectional pair (which adds u*D once
 *   per direction, mamba.py:256-260).  out may equal y (in place). */
M3_API int m3_gate(int64_t rows, int32_t d_inner, const float* y, const void* u,
            int32_t dtype_u, const float* z, int64_t ld_z, const float* d_skip, float coef,
            float* out, void* stream);

/* m3_gate with an element type per operand (M3_F32 or M3_BF16): y, u, z and
 * out of a bf16 layer (mamba.py:262-265 under the reference's autocast,
 * train.py:268; the bf16 Eval-Mamba forward, model.py:110-132).  Arithmetic is
 * fp32; out is rounded once.  out may equal y only when dtype_out == dtype_y.
 * round_silu != 0 rounds silu(z) to bf16 when z is bf16, as torch's F.silu on a
 * bf16 tensor does before the product (the training path's autograd formula,
 * mamba.py:265). */
M3_API int m3_gate_typed(int64_t rows, int32_t d_inner, const void* y, int32_t dtype_y,
            const void* u, int32_t dtype_u, const void* z, int32_t dtype_z, int64_t ld_z,
            const float* d_skip, float coef, int32_t round_silu, void* out, int32_t dtype_out,
            void* stream);

/* Workspace bytes of m3_gate_bwd (the per-row-chunk partial sums of d d_skip). */
M3_API size_t m3_gate_bwd_workspace_bytes(int64_t rows, int32_t d_inner);

/* Backward of m3_gate_typed (the autograd of mamba.py:262-265 / 496-497 in one
 * launch plus a fixed-order reduction): with a = y + coef*u*d_skip,
 * s = silu(z) (rounded as in the forward), sig = 1/(1+exp(-z)) and g the
 * gradient of out (rows, D) of dtype_g:
 *   d_y = g*s,  d_u = (g*s*d_skip)*coef,  d_z = (g*a)*sig*(1 + z*(1 - sig)),
 *   d_dskip = sum over rows of g*s*coef*u (deterministic)
 * in fp32, each rounded once to its input's element type; d_y, d_u, d_z are
 * (rows, D) contiguous, d_dskip (D,) float32.
 *   workspace >= m3_gate_bwd_workspace_bytes(rows, d_inner) bytes */
M3_API int m3_gate_bwd(int64_t rows, int32_t d_inner, const void* y, int32_t dtype_y,
            const void* u, int32_t dtype_u, const void* z, int32_t dtype_z, int64_t ld_z,
            const float* d_skip, float coef, int32_t round_silu, const void* g, int32_t dtype_g,
            void* d_y, void* d_u, void* d_z, float* d_dskip, void* workspace,
            size_t workspace_bytes, void* stream);

/* Size of the scratch buffer built into the library for m3_scan_bwd_noalloc. */
#define M3_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)

/* The analytic backward without a caller-supplied workspace.  No counterpart in
 * the reference: it exists for callers that cannot allocate device memory when
 * they run the backward (memory carved up at start-up by an allocator they have
 * no handle to, or loops that must not call cudaMalloc).  Inputs and outputs
 * are exactly those of m3_scan_bwd; the workspace comes from a device buffer of
 * M3_NOALLOC_SCRATCH_BYTES that the library holds on every GPU that loads it,
 * until the process exits.  This entry point never allocates or frees.
 *   - Problems whose m3_scan_bwd_workspace_bytes() exceeds the buffer are
 *     rejected with M3_ERR_SCRATCH_LIMIT.
 *   - The first call on each device looks up the buffer's device address (with
 *     that device current) and caches it; make that first call before any
 *     stream capture.  The cached address belongs to the device's current
 *     context: after cudaDeviceReset (or any other reset of the primary
 *     context) in the same process, this entry point must not be called
 *     again, since it would hand the kernels the stale address.
 *   - All calls on a device share the one buffer, which keeps the last call's
 *     contents.  Calls whose executions overlap on the GPU (other streams, or
 *     other host threads) race on it and corrupt each other's results. */
M3_API int m3_scan_bwd_noalloc(const m3_scan_desc* desc,
                const void* delta, const void* u, const void* Bc, const void* Cc,
                const float* A_real_p, const float* A_imag_p, const float* track_p,
                const void* dy, int32_t dtype_dy, const float* ckpt,
                void* d_delta, void* d_u, void* d_Bc, void* d_Cc,
                float* d_A_real_p, float* d_A_imag_p, float* d_track_p, void* stream);

/* Reads (and clears when clear != 0) the device-side error word of the
 * current device; *code receives 0 or an M3_ERR_* value. */
M3_API int m3_device_error(int32_t* code, int32_t clear);

#ifdef __cplusplus
}
#endif

#endif /* M3SCAN_H */
