/*
 * ews_b200.h — C ABI of the B200 (sm_100a) EWS hot-path library, libews_b200.so.
 *
 * The exponentially weighted signature (EWS) of a path x with clock theta and generator A is the
 * modified-Chen prefix scan of per-interval local terms: with M_t = exp(-dtheta_t A),
 *
 *     S_k,t = M_t^{(x)k} S_k,t-1 + sum_{i=1}^{k-1} (M_t^{(x)i} S_i,t-1) (x) s_{k-i},t + s_k,t,
 *
 * and the local terms s_k,t come from the series leaf (letters b_p = (-dtheta/p) A b_{p-1}, b_0 = dx).
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, never allocates, and
 * returns EWS_OK or an error code. Buffers are stream-ordered; the caller owns all memory,
 * including the workspaces whose sizes the *_workspace_size queries return.
 *
 * The reference interface these replace is the combine engine boundary
 *     combine_packed(kind, local_signatures, A, interval_times, N, chen_expm, cached, basepoint,
 *                    *, terminal, block_sizes, chunk_target, tile, jordan_chain)
 * (ews/core/kernels/combine.py:193-224 of alexandre-bloch/exponentially-weighted-signature) together
 * with the leaf it is fed by (ews/core/leaf.py:50-198) and the custom VJPs of its kernels
 * (ews/core/kernels/pallas_combine.py:1673-1801 block, :2628-2711 dense). Unlike the reference, the
 * local terms and the lift B (ews/params.py:1181-1192) are fused into the kernels, so the VJP returns
 * gradients for the increments, the clock steps and the generator tables directly.
 */
#ifndef EWS_B200_H
#define EWS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ews_stream_t; /* = cudaStream_t */

/* ---- status codes ---------------------------------------------------------------------------- */
#define EWS_OK 0
#define EWS_ERR_INVALID_ARGUMENT 1   /* bad shape, null pointer, unsupported combination */
#define EWS_ERR_UNSUPPORTED 2        /* valid but not built: e.g. dim above the engine's limit */
#define EWS_ERR_WORKSPACE 3          /* workspace missing or smaller than the query returned */
#define EWS_ERR_LAUNCH 4             /* a CUDA launch failed (cudaGetLastError after the launch) */
#define EWS_ERR_LOOKBACK_TIMEOUT 5   /* a device-side wait for a neighbouring chunk ran out (read
                                        with ews_read_device_status; the outputs are then invalid) */

/* ---- flags ----------------------------------------------------------------------------------- */
#define EWS_F_UNIFORM 1u        /* uniform clock: per-sample constant flow/local tables (cached flows,
                                   ews/core/chen_scan.py:155-168 cached=True) */
#define EWS_F_INCREMENTS 2u     /* `path` holds increments (B, T, d_in) instead of knots (B, T+1, d_in) */
#define EWS_F_BF16 4u           /* `path` is bfloat16 (accumulation stays float32) */
#define EWS_F_BASEPOINT 8u      /* uniform with basepoint: step 0 has the identity flow
                                   (ews/core/chen_scan.py:160-166) */
#define EWS_F_DETERMINISTIC 16u /* bit-reproducible results: every chunk waits for its neighbour's inclusive
                                   value instead of folding in whatever aggregates are ready (the grouping of
                                   a decoupled look-back depends on timing, hence so does its rounding) */
#define EWS_F_TEST_WITHHOLD 32u /* failure-detection test: the chunk every other chunk depends on never
                                   publishes, so their bounded waits run out and the call reports
                                   EWS_ERR_LOOKBACK_TIMEOUT through ews_read_device_status */
#define EWS_F_TERMINAL_SCAN 64u /* diagonal engine, uniform clock, terminal readout: evaluate the terminal
                                   value with the chunked scan instead of its closed form (see below) */

#define EWS_F_LOGSIG 128u      /* diagonal engine, closed-form terminal path (uniform clock, terminal readout,
                                   depth 2): `out` receives the compressed log-signature (B, N + N (N - 1) / 2),
                                   the letters then the Lyndon words (i, j), i < j, in lexicographic order, of
                                   log(1 + X) = (X1, X2 - X1 X1^T / 2) (the LogEWS epilogue, ews/layer.py:488-498),
                                   and the backward's `grad_out` is its cotangent; other paths return
                                   EWS_ERR_UNSUPPORTED */

#define EWS_READOUT_PREFIX 0    /* out: (B, T, 1 + D), row t = [1, S_1,t, ..., S_n,t] */
#define EWS_READOUT_TERMINAL 1  /* out: (B, 1 + D), the last row only */

/* ---- diagonal engine: A = diag(lambda) --------------------------------------------------------
 * Replaces combine_packed(kind="block_kernel", block_sizes=(1,)*N) fed by leaf="series" /
 * "block_series" (ews/core/kernels/combine.py:233-258, ews/core/kernels/blockdiag_engine.py:88-163,
 * ews/core/series_leaf.py:72-127). Depth 2, dim <= 32.
 *
 * Uniform clock (EWS_F_UNIFORM): with x_b = -h_b lambda (h_b the shared clock step of sample b),
 *   tab_x  (B, dim)       log-flows x, flow rho = exp(x)
 *   tab_q1 (B, dim)       Q1_i  = sum_{p<=q} c1_p x_i^p / p!             (s1_i = Q1_i dy_i)
 *   tab_q2 (B, dim, dim)  Q2_ij = sum_{a+b<=q} c2_ab x_i^a x_j^b / a!b!  (s2_ij = Q2_ij dy_i dy_j)
 * where dy = lift @ dx. The backward returns dL/dx (grad_x), dL/dQ1, dL/dQ2 per sample, so the caller
 * chains them to lambda and the clock with the (tiny) table maps.
 *
 * Per-interval clock (flags without EWS_F_UNIFORM; the reference's default reweighting mode
 * "displacement", ews/layer.py:154-169 with ews/core/chen_scan.py:155-168 cached=False): interval t of
 * sample b has its own step dtheta_t = clock[b, t+1] - clock[b, t] and log-flow x_t = dtheta_t r_b with
 *   clock  (B, T+1)       clock knots
 *   tab_x  (B, dim)       rates r = -lambda (per sample)
 * and the series tables Q1(x_t), Q2(x_t) of order series_q (<= 8) are evaluated in the kernel for every
 * interval (tab_q1 / tab_q2 unused). The backward returns dL/dr in grad_x and dL/d(dtheta) in
 * grad_dtheta (B, T); grad_q1 / grad_q2 are unused. EWS_F_BASEPOINT does not apply: a basepoint interval
 * is an interval with dtheta = 0.
 *
 * Uniform clock with the terminal readout (no basepoint, d_in <= 32, dim * d_in <= 1024): the terminal
 * value is evaluated in closed form, as a reweighted depth-2 signature. With r_t = exp(x (T-1-t)) dy_t,
 *   S1_T = Q1 sum_t r_t,   S2_T = diag(Q1) M diag(Q1) + Q2 G,   M = sum_t (sum_{tau<t} r_tau) r_t^T,
 *   G = sum_t r_t r_t^T
 * (the reference reduces the Chen products in a tree, ews/core/chen_scan.py:218-298: the same value in
 * another order). EWS_F_TERMINAL_SCAN selects the chunked scan instead. */
typedef struct ews_diag_args {
    int batch;         /* B */
    int steps;         /* T: intervals per path */
    int d_in;          /* input channels (before the lift) */
    int dim;           /* N: state dimension (after the lift) */
    int depth;         /* truncation depth (2) */
    int chunk;         /* chunk length (0: the library's choice) */
    int readout;       /* EWS_READOUT_* */
    unsigned flags;    /* EWS_F_* */
    int series_q;      /* series order (non-uniform tables) */
    int spin_limit;    /* polls before a look-back wait gives up (0: default) */
    /* inputs */
    const void* path;        /* (B, T+1, d_in) knots or (B, T, d_in) increments; f32 or bf16 */
    const float* clock;      /* (B, T+1) clock knots (non-uniform) or NULL */
    const float* lift;       /* (dim, d_in) lift B, or NULL for the identity (d_in == dim) */
    const float* tab_x;      /* see above */
    const float* tab_q1;
    const float* tab_q2;
    /* forward output */
    float* out;
    /* backward */
    const float* grad_out;   /* same shape as out */
    float* grad_dx;          /* (B, T, d_in): dL/d(increments) */
    float* grad_lift;        /* (dim, d_in) or NULL */
    float* grad_x;           /* (B, dim): dL/dx (uniform) or dL/dr (per-interval clock) */
    float* grad_q1;          /* (B, dim), uniform only */
    float* grad_q2;          /* (B, dim, dim), uniform only */
    /* workspaces: fwd_ws is written by the forward and read by the backward (chunk aggregates and
       carries); bwd_ws is private to the backward */
    void* fwd_ws;
    size_t fwd_ws_bytes;
    void* bwd_ws;
    size_t bwd_ws_bytes;
    /* backward, per-interval clock only */
    float* grad_dtheta;      /* (B, T): dL/d(dtheta_t) */
    /* per-interval clock only, optional (NULL: the series leaf of order series_q): HOST pointer to 9 + 81
       floats, the polynomial coefficients of the local tables in the log-flow x,
       Q1(x) = sum_a k1[a] x^a and Q2(x_i, x_j) = sum_{a,b} k2[9 a + b] x_i^a x_j^b (k1 then k2). Another
       leaf whose diagonal tables are such power series runs through the same kernels: the Van Loan leaf
       (ews/core/van_loan.py:30-88 with ews/core/signature.py:19-36, the reference's default) truncated
       at degree 8 in each variable. Read during the call; not kept. */
    const float* leaf_coef;
} ews_diag_args;

int ews_diag_workspace_size(const ews_diag_args* a, size_t* fwd_bytes, size_t* bwd_bytes);
int ews_diag_fwd(const ews_diag_args* a, ews_stream_t stream);
int ews_diag_bwd(const ews_diag_args* a, ews_stream_t stream);

/* Forward that allocates nothing and needs no workspace from the caller. This entry point has no
 * counterpart in the reference. It is for callers that cannot allocate device memory for the library:
 * a plugin host that passes a kernel only its inputs and outputs, or a serving loop that forbids
 * cudaMalloc because an allocation can synchronise the device. Same arguments and results as
 * ews_diag_fwd, except that fwd_ws / fwd_ws_bytes are ignored: the look-back workspace is a file-scope
 * device array of EWS_NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU loading the library holds until the
 * process exits. Problems whose forward workspace (ews_diag_workspace_size) exceeds that return
 * EWS_ERR_WORKSPACE before anything runs. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current); make that first call before any stream
 * capture. Every call shares the one array and it keeps the last call's contents (the call clears what
 * must start at zero), so calls whose executions overlap on the GPU race on it: serialise them, e.g. on
 * one stream. Because the array is reused, a backward (ews_diag_bwd) cannot consume this forward's
 * workspace; use ews_diag_fwd when gradients are needed. */
#define EWS_NOALLOC_SCRATCH_BYTES (16u << 20)
int ews_diag_fwd_noalloc(const ews_diag_args* a, ews_stream_t stream);

/* Status of the last no-alloc forward on the current device: copies the error word at the start of the
 * library's array (EWS_OK or EWS_ERR_LOOKBACK_TIMEOUT) to *status; synchronises the stream. Like the array,
 * it has no counterpart in the reference: the no-alloc caller holds no workspace pointer to pass to
 * ews_read_device_status. */
int ews_diag_fwd_noalloc_status(ews_stream_t stream, int* status);

/* ---- dense engine: any generator A (uniform clock) --------------------------------------------
 * Replaces combine_packed(kind="dense_kernel" / "lean") fed by leaf="series" (ews/core/kernels/combine.py:
 * 260-269, ews/core/kernels/pallas_combine.py:803-858 forward, :2628-2711 custom VJP) with the series
 * local terms fused. Depth 2, dim <= 32, d_in <= 32, series_q <= 11. With the sample's shared clock step h,
 * P_a = (-hA)^a / a!, K1 = sum_p c_p P_p and K2_a = sum_b c_ab P_b (ews/core/series_leaf.py:45-113), and the
 * lift W, the per-sample tables are
 *   tab_d (B, N, N)          the flow complement D = I - expm(-h A) (evaluate it in float64: the engine
 *                            applies M X as X - D X, so the rounding stays relative to D)
 *   tab_f (B, N, d_in)       F = K1 W            (s1 = F dx)
 *   tab_g (B, q+1, N, d_in)  G_a = P_a W         (s2 = sum_a (G_a dx)(H_a dx)^T)
 *   tab_h (B, q+1, N, d_in)  H_a = K2_a W
 * The backward returns dL/d(tables) per sample and dL/d(increments); prefix readout only (the terminal
 * value is the prefix's last row, as in the reference's dense kernel). */
typedef struct ews_dense_args {
    int batch, steps, d_in, dim, depth, chunk, readout;
    unsigned flags;
    int series_q;
    int spin_limit;
    const void* path;        /* (B, T+1, d_in) knots or (B, T, d_in) increments */
    const float* tab_d;
    const float* tab_f;
    const float* tab_g;
    const float* tab_h;
    float* out;              /* (B, T, 1 + D) prefix or (B, 1 + D) terminal (forward only) */
    const float* grad_out;
    float* grad_dx;          /* (B, T, d_in) */
    float* grad_d;           /* (B, N, N) */
    float* grad_f;           /* (B, N, d_in) */
    float* grad_g;           /* (B, q+1, N, d_in) */
    float* grad_h;           /* (B, q+1, N, d_in) */
    void* fwd_ws;
    size_t fwd_ws_bytes;
    void* bwd_ws;
    size_t bwd_ws_bytes;
} ews_dense_args;

int ews_dense_workspace_size(const ews_dense_args* a, size_t* fwd_bytes, size_t* bwd_bytes);
/* Kernel launches of one ews_dense_fwd / ews_dense_bwd call with these arguments (the carry scans take
 * log2(chunk groups) rounds). A query of this library with no counterpart in the reference. */
int ews_dense_launches(const ews_dense_args* a, int* fwd_launches, int* bwd_launches);
int ews_dense_fwd(const ews_dense_args* a, ews_stream_t stream);
int ews_dense_bwd(const ews_dense_args* a, ews_stream_t stream);

/* ---- block engine: A block-diagonal with 2x2 blocks, depth 3, per-interval clock ----------------
 * Replaces combine_packed(kind="block_kernel", block_sizes=(2,)*K) fed by leaf="series"
 * (ews/core/kernels/combine.py:233-258; forward ews/core/kernels/pallas_combine.py:1342-1422 and
 * :1221-1289, custom VJP :1698-1801; series leaf ews/core/series_leaf.py:72-127). dim = 2K <= 8, depth 3.
 * Interval t of sample b has clock step dtheta_t = clock[b, t+1] - clock[b, t], flow expm(-dtheta_t A)
 * and series local terms of order series_q (<= 8) built in the kernel from the letters
 * b_p = (-dtheta_t A / p) b_{p-1}, b_0 = lift @ dx_t. A uniform clock is passed as evenly spaced knots.
 *   blocks (K, 2, 2)  the diagonal blocks A_k of the generator, shared by the batch
 * The backward returns dL/d(increments), dL/d(dtheta) (B, T), dL/dA_k (K, 2, 2) and dL/dlift. */
typedef struct ews_block_args {
    int batch;         /* B */
    int steps;         /* T */
    int d_in;          /* input channels (before the lift) */
    int dim;           /* N = 2K <= 8 */
    int depth;         /* 3 */
    int chunk;         /* chunk length (0: the library's choice) */
    int readout;       /* EWS_READOUT_* */
    unsigned flags;    /* EWS_F_INCREMENTS, EWS_F_BF16, EWS_F_DETERMINISTIC, EWS_F_TEST_WITHHOLD */
    int series_q;      /* series order, 0..8 */
    int spin_limit;    /* polls before a look-back wait gives up (0: default) */
    const void* path;        /* (B, T+1, d_in) knots or (B, T, d_in) increments; f32 or bf16 */
    const float* clock;      /* (B, T+1) clock knots */
    const float* blocks;     /* (K, 2, 2) */
    const float* lift;       /* (dim, d_in), or NULL for the identity (d_in == dim) */
    float* out;              /* (B, T, 1 + N + N^2 + N^3) prefix or (B, 1 + ...) terminal */
    const float* grad_out;   /* same shape as out */
    float* grad_dx;          /* (B, T, d_in) */
    float* grad_dtheta;      /* (B, T) */
    float* grad_blocks;      /* (K, 2, 2) */
    float* grad_lift;        /* (dim, d_in) or NULL */
    void* fwd_ws;
    size_t fwd_ws_bytes;
    void* bwd_ws;
    size_t bwd_ws_bytes;
} ews_block_args;

int ews_block_workspace_size(const ews_block_args* a, size_t* fwd_bytes, size_t* bwd_bytes);
int ews_block_fwd(const ews_block_args* a, ews_stream_t stream);
/* Terminal readout: grad_out is the (B, 1 + ...) terminal row's cotangent; the states are recomputed
 * from the forward workspace's chunk carries (ews/core/kernels/pallas_combine.py:1911-2027,
 * block_terminal_vjp), into rows of the backward workspace sized by ews_block_workspace_size for the
 * same readout. The same holds for ews_dense_bwd. */
int ews_block_bwd(const ews_block_args* a, ews_stream_t stream);

/* ---- flow tables of the dense engine ---------------------------------------------------------------
 * Replaces expm_matrix(-h A, "exact") (ews/core/chen_scan.py:155-168, ews/core/expm_approx.py:34-41),
 * the dense flow the reference builds per clock step, and its VJP. Row-major float64 matrices on the
 * device; one CTA per matrix, scaling and squaring with a degree-14 Taylor polynomial (the scaling is
 * chosen in the kernel, nothing is read back to the host).
 *   ews_expm_batched:          out_b = expm(x_b),            x, out (batch, n, n), n <= 64
 *   ews_expm_adjoint_batched:  out_b = d<g_b, expm(x_b)>/dx_b = L(x_b^T, g_b), n <= 32 */
int ews_expm_batched(const double* x, double* out, int batch, int n, ews_stream_t stream);
int ews_expm_adjoint_batched(const double* x, const double* g, double* out, int batch, int n, ews_stream_t stream);

/* ---- series-leaf tables of the dense engine ----------------------------------------------------------
 * Replaces the letters and level assembly of series_local_signatures (ews/core/series_leaf.py:72-113) for a
 * uniform clock, as per-sample tables: with x_b = -h_b A (batch, n, n) float64 and the lift W (n, d_in)
 * float64 (NULL: the identity, d_in == n), P_a = x^a / a!, G_a = P_a W, F = sum_p c1_p G_p and
 * H_a = sum_b c2_ab G_b for a, b = 0..order (c1 (order+1), c2 (order+1, order+1) float64 on the device).
 * Outputs float32: F (batch, n, d_in), G and H (batch, order+1, n, d_in). n, d_in <= 32, order <= 11.
 *   ews_series_tables_adjoint: from dF, dG, dH (float32, same shapes) the per-sample gradients
 *   dX (batch, n, n) and dW (batch, n, d_in; may be NULL) in float64, summed over samples by the caller. */
int ews_series_tables(const double* x, const double* lift, const double* c1, const double* c2, int batch, int n,
                      int d_in, int order, float* F, float* G, float* H, ews_stream_t stream);
int ews_series_tables_adjoint(const double* x, const double* lift, const double* c1, const double* c2, int batch,
                              int n, int d_in, int order, const float* dF, const float* dG, const float* dH,
                              double* dX, double* dW, ews_stream_t stream);

/* ---- the dense leaf, fused ------------------------------------------------------------------------------
 * Both per-sample tables of the dense engine for a uniform clock in one launch, from the generator itself:
 * the flow complement D_b = I - expm(x_b), x_b = -h_b A (ews/core/chen_scan.py:155-168), and the series
 * tables F, G, H of x^l_b = -h_b A_leaf (A_leaf NULL: A) as ews_series_tables defines them. A, A_leaf (n, n),
 * h (batch,), lift (n, d_in; NULL: the identity, d_in == n) float32; c1, c2 float64 on the device; outputs
 * float32 D (batch, n, n), F (batch, n, d_in), G, H (batch, order+1, n, d_in). Evaluated in float64 (the
 * exponential as ews_expm_batched). n, d_in <= 32, order <= 11.
 *   ews_dense_leaf_adjoint: from the cotangents dD, dF, dG, dH (float32; any may be NULL: zeros) the
 *   gradients dA (n, n), dA_leaf (n, n; required iff A_leaf), dh (batch,; may be NULL) and dW (n, d_in;
 *   required iff lift), float32, each summed over samples in sample order (bit-reproducible). `work` is
 *   caller-owned device memory of at least ews_dense_leaf_work_size(batch, n, d_in) bytes. Two launches. */
size_t ews_dense_leaf_work_size(int batch, int n, int d_in);
int ews_dense_leaf(const float* A, const float* A_leaf, const float* h, const float* lift, const double* c1,
                   const double* c2, int batch, int n, int d_in, int order, float* D, float* F, float* G, float* H,
                   ews_stream_t stream);
int ews_dense_leaf_adjoint(const float* A, const float* A_leaf, const float* h, const float* lift, const double* c1,
                           const double* c2, int batch, int n, int d_in, int order, const float* dD, const float* dF,
                           const float* dG, const float* dH, void* work, size_t work_bytes, float* dA, float* dA_leaf,
                           float* dh, float* dW, ews_stream_t stream);

/* ---- the block's stream consumer: graded RMS norm of the prefix stream --------------------------------
 * Replaces the block's level-0 drop, zero-row prepend and GradedRMSNorm "live_rms" (ews/block.py:282-306 and
 * :406, ews/norms.py:47-135) in one pass over the EWS prefix output: flat (batch, steps, 1 + D) float32 with
 * D = d + d^2 (+ d^3) for `levels` = 2 (3) -> y (batch, steps + 1, D): y[:, 0] = 0 and row t + 1 level k =
 * gains[k] x_k / (RMS(x_k) + eps[k]), x = flat[:, t, 1:], RMS 0 for an all-zero level. gains on the device
 * (levels floats), eps a host array of `levels` positive floats.
 *   ews_graded_norm_bwd: from dy (batch, steps + 1, D) the input gradient dflat (batch, steps, 1 + D; level-0
 *   column zero) and dgains (levels), the latter summed in a fixed order; `work` is caller-owned device memory
 *   of ews_graded_norm_work_size bytes. */
size_t ews_graded_norm_work_size(int batch, int steps, int d, int levels);
int ews_graded_norm_fwd(const float* flat, const float* gains, const float* eps, int batch, int steps, int d,
                        int levels, float* y, ews_stream_t stream);
int ews_graded_norm_bwd(const float* flat, const float* gains, const float* eps, const float* dy, int batch,
                        int steps, int d, int levels, float* dflat, float* dgains, void* work, size_t work_bytes,
                        ews_stream_t stream);

/* ---- the block's clock prologue: the token-gated clock ---------------------------------------------
 * Replaces GatedClock "token_gated" without a mask (ews/clocks.py:409-466) on the block input: x (batch,
 * steps, dim) float32, w (dim) and b (one float) on the device -> theta (batch, steps), theta_0 = 0 and
 * theta_{t+1} = (1/norm_constant) sum_{tau <= t} relu(<in_scale x_{tau+1} - in_scale x_tau, w> - b).
 *   ews_gated_clock_bwd: from dtheta the gradients dx (batch, steps, dim), dw (dim) and db (one float), the
 *   latter two summed over samples in a fixed order; `work` is caller-owned device memory of
 *   ews_gated_clock_work_size bytes. dim <= 8192. */
size_t ews_gated_clock_work_size(int batch, int steps, int dim);
int ews_gated_clock_fwd(const float* x, const float* w, const float* b, float in_scale, float norm_constant, int batch,
                        int steps, int dim, float* theta, ews_stream_t stream);
int ews_gated_clock_bwd(const float* x, const float* w, const float* b, float in_scale, float norm_constant,
                        const float* dtheta, int batch, int steps, int dim, float* dx, float* dw, float* db, void* work,
                        size_t work_bytes, ews_stream_t stream);

/* ---- utilities --------------------------------------------------------------------------------- */
/* Every forward and backward workspace begins with a status block whose error word the call clears and
 * a timed-out device wait sets. */
/* Copies the device-side status word of a workspace (EWS_OK or EWS_ERR_LOOKBACK_TIMEOUT) to the host;
 * synchronises the stream. */
int ews_read_device_status(const void* workspace, ews_stream_t stream, int* status);
/* Stream-ordered, no synchronisation: after the workspace's call, folds its error word into *sticky, a
 * caller-owned device int (the first non-zero code is kept; the caller clears it). A host that copies
 * *sticky to pinned memory asynchronously learns of a timeout without waiting on the GPU, and can raise
 * it as the reference raises its errors (ews/layer.py:112-152). */
int ews_status_fold(const void* workspace, int* sticky, ews_stream_t stream);
const char* ews_error_string(int code);
int ews_version(void);

#ifdef __cplusplus
}
#endif
#endif /* EWS_B200_H */
