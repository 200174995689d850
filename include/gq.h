/*
 * libgq -- B200 (sm_100a) kernels for the jax_gptq quantization hot path.
 *
 * C ABI: plain pointers, sizes and a CUDA stream passed as void*.  Every
 * function returns a gq_status; on failure gq_last_error() describes it.
 * All array pointers are DEVICE pointers unless stated otherwise.  Matrices
 * are row-major with an explicit leading dimension (elements).  Calls are
 * stream-ordered and return before the work finishes unless documented as
 * blocking.  No function allocates device memory: scratch space is passed in
 * by the caller (query it with the matching *_workspace_size function).
 *
 * The reference (davidtweedle/jax_gptq) is pure Python/JAX and has no FFI of
 * its own; each entry point names the reference function whose array
 * contract it implements (paths relative to the reference's src/jax_gptq/).
 */
#ifndef GQ_H_
#define GQ_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GQ_OK = 0,
  GQ_EINVAL = 1,        /* bad argument (shape, size, mode); nothing launched */
  GQ_ENOTPD = 2,        /* damped Hessian not positive definite after all retries */
  GQ_ETIMEOUT = 3,      /* a bounded device-side wait expired */
  GQ_ECUDA = 4,         /* CUDA runtime error */
  GQ_EUNSUPPORTED = 5,  /* valid input outside what this build supports */
  GQ_ENCCL = 6          /* NCCL missing or an NCCL call failed */
} gq_status;

/* Grid cap for the persistent tensor-core kernels (fp32 GEMM, H
 * accumulation) launched afterwards by the calling host thread: at most n
 * CTAs, one per SM (0 = every SM, the default).  For hosts that run several
 * independent chains on different streams and want SMs left free for a
 * latency-bound one; results do not depend on it.  No counterpart in the
 * reference (single stream). */
int gq_set_cta_budget(int n);

/* Form of the bf16 statistics kernels (gq_syrk_bf16, gq_gemm_tn_bf16)
 * launched afterwards by the calling host thread: 1 (default) = clusters of
 * two CTAs sharing 256 x 256 tiles (tcgen05 cta_group::2), 0 = one CTA per
 * 128 x 256 tile.  Both give the same bits; the pair form moves a third less
 * data from L2 per flop.  Without a cluster of two available the one-CTA
 * form runs regardless. */
int gq_set_pair_kernels(int enable);

/* Rows per CTA of the GPTQ sweep's block step, for sweeps launched
 * afterwards (process-wide): r groups of 32 rows share one CTA and one staged
 * copy of the block's U band (r = 1, 2 or 4); 0 (default) picks by row count
 * (one group while such CTAs fit in one wave on the device, four while those
 * do, else the one-warp form); -1 forces the one-warp form.  Every form gives
 * the same bits; more groups per CTA leave more SMs to work on other
 * streams.  GQ_EINVAL for any other value. */
int gq_set_sweep_row_groups(int r);

/* Library version (major*10000 + minor*100 + patch). */
int gq_version(void);

/* Message for the most recent failing call on this host thread. */
const char* gq_last_error(void);

/* Number of kernels this library has launched since it was loaded
 * (instrumentation; no reference counterpart). */
long long gq_launch_count(void);

/* ------------------------------------------------------------------------
 * quant.py:6-37 quantize_dequantize, and the RTN core of
 * gptq_ref.py:152-155 gptq_forward_step (permute -> RTN -> un-permute).
 *
 * w       [m, n] float32 (ldw).  n % group_size == 0, group_size > 0.
 * perm    [n] int32 column order, or NULL for the identity.  Groups are
 *         group_size consecutive columns of w[:, perm].
 * dequant [m, n] float32, original column order (NULL to skip).
 * codes   [m, n] uint8 = q - qmin, original column order (NULL to skip).
 * scales, zeros  [m, n / group_size] float32, groups in permuted order
 *         (NULL to skip).
 * Bit-exact with the reference's float32 arithmetic: IEEE division,
 * round-half-to-even, scale floor 1e-8.
 */
int gq_rtn(const float* w, int64_t m, int64_t n, int64_t ldw, const int32_t* perm,
           int w_bits, int group_size, int sym,
           float* dequant, uint8_t* codes, float* scales, float* zeros, void* stream);

/* ------------------------------------------------------------------------
 * Float32-accurate GEMM: C = alpha * op(A) op(B) + beta * C with op(A) M x K,
 * op(B) K x N, row-major storage (trans_* = 1 means the stored matrix is the
 * transpose).  uplo = 0 computes all of C, 1 only tiles that touch the lower
 * triangle, 2 only tiles that touch the upper triangle (tiles on the diagonal
 * are computed whole).  Used for the GPTQ lazy trailing update, Cholesky /
 * inverse updates, Qronos and the QR compact-WY update.
 * gq_sgemm runs the tcgen05 3xTF32 kernel (gq_gemm_f32_tc) when trans_a = 0,
 * trans_b = 1, N >= 128, K >= 32, A and B are 16-byte aligned and lda, ldb
 * are multiples of 4 (any M >= 1, so a row's result does not depend on how
 * many rows share the call), and the CUDA-core kernel (gq_sgemm_simt)
 * otherwise.
 */
int gq_sgemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
             const float* a, int64_t lda, const float* b, int64_t ldb, float beta,
             float* c, int64_t ldc, int uplo, void* stream);
int gq_sgemm_simt(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                  const float* a, int64_t lda, const float* b, int64_t ldb, float beta,
                  float* c, int64_t ldc, int uplo, void* stream);
/* tcgen05 kind::tf32 with a 3-pass hi/lo operand split (error near 2^-21 per
 * product); A [M, K] and B [N, K] row-major (trans_b must be 1: both operands
 * K-major); GQ_EINVAL for any other layout or for N < 128 or K < 32. */
int gq_gemm_f32_tc(int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                   const float* a, int64_t lda, const float* b, int64_t ldb, float beta,
                   float* c, int64_t ldc, int uplo, void* stream);

/* ------------------------------------------------------------------------
 * stats.py:4-18 h_g_from_activations, bf16 activations, fp32 accumulation
 * on the tcgen05 tensor cores (TMEM accumulators, TMA-fed shared memory).
 *
 * x [tokens, d] bf16 (raw uint16 bits), row-major with ldx (elements, multiple
 *   of 8), base 16-byte aligned.
 * gq_syrk_bf16:    h[d, d] (+)= x^T x   (stats.py:16; full symmetric result)
 * gq_gemm_tn_bf16: g[da, db] (+)= xa^T xb   (stats.py:17 with xa = x_float,
 *                  xb = x_quant)
 * accumulate = 0 overwrites, 1 adds to the existing contents (streamed
 * calibration batches).  ldh/ldg are in elements.
 * Products are summed in chunks of 1024 tokens (each chunk in tensor memory),
 * and the chunk results are added in token order to a float32 running sum
 * that starts from the existing contents when accumulating; so splitting the
 * tokens into calls at multiples of 1024 gives the same bits as one call.
 */
int gq_syrk_bf16(const uint16_t* x, int64_t tokens, int64_t d, int64_t ldx,
                 float* h, int64_t ldh, int accumulate, void* stream);
int gq_gemm_tn_bf16(const uint16_t* xa, int64_t lda, const uint16_t* xb, int64_t ldb,
                    int64_t tokens, int64_t da, int64_t db,
                    float* g, int64_t ldg, int accumulate, void* stream);

/* Device status word written by kernels with bounded waits (0 = fine,
 * 1 = a wait timed out, 2 = not positive definite).  BLOCKING: synchronizes
 * the stream; reset = 1 clears the word afterwards. */
int gq_device_status(int* status_out, int reset, void* stream);

/* gq_device_status as a status code: BLOCKING (synchronizes the stream),
 * clears the word, and returns GQ_ETIMEOUT when a kernel's bounded wait
 * expired since the last check (that kernel returned early and its outputs
 * are incomplete), GQ_OK otherwise.  The reference has no device-side waits;
 * this is the device half of its failure handling (gptq_ref.py:79-92 catches
 * numeric failures on the host). */
int gq_check_device(void* stream);

/* Bound, in nanoseconds, on every device-side wait of the tensor-core
 * kernels launched afterwards on the current device (default 2 s; accepted
 * range 1 ms .. 60 s).  For tests that make a wait expire on purpose. */
int gq_set_wait_limit_ns(uint64_t ns);

/* Test entry: launches one thread that waits on an mbarrier nothing arrives
 * on, through the same bounded-wait code as the statistics kernels (unit 0)
 * or the fp32 tensor-core GEMM (unit 1).  The wait expires after the limit
 * above, *observed (device int) becomes 1, and the unit's status word reads
 * GQ_DEVERR_TIMEOUT; nothing traps or faults.  No reference counterpart. */
int gq_test_expire_wait(int unit, int* observed, void* stream);

/* stats.py:4-18 for float32 activations (CUDA-core fp32 GEMM). */
int gq_syrk_f32(const float* x, int64_t tokens, int64_t d, int64_t ldx,
                float* h, int64_t ldh, int accumulate, void* stream);
int gq_gemm_tn_f32(const float* xa, int64_t lda, const float* xb, int64_t ldb,
                   int64_t tokens, int64_t da, int64_t db,
                   float* g, int64_t ldg, int accumulate, void* stream);

/* Mirror the upper triangle of h[d, d] into the lower triangle. */
int gq_symmetrize_upper(float* h, int64_t d, int64_t ldh, void* stream);

/* ------------------------------------------------------------------------
 * gptq_ref.py:67-70: ordering = 0 ("none") writes arange(d); ordering = 1
 * ("diag_h") writes argsort(diag(h))[::-1] with a stable sort, i.e.
 * descending diagonal, equal values highest-index-first.
 */
int gq_act_order_perm(const float* h, int64_t d, int64_t ldh, int ordering,
                      int32_t* perm, void* stream);

/* ------------------------------------------------------------------------
 * gptq_ref.py:72-92 (the damped-Cholesky branch, working): for attempt
 * e = 0..4 with damp = 10^e * damp_percent * mean(diag(h)) (mean 0 -> 1),
 * factor Hd = h[perm][:, perm] + damp I and return the upper factor
 * u = chol(Hd^-1, upper) (u^T u = Hd^-1), computed as the inverse of the
 * upper factor R of Hd = R R^T.  BLOCKING: synchronizes the stream once per
 * attempt to read the positive-definiteness flag.  Returns GQ_ENOTPD (u
 * untouched) when all five attempts fail; *attempt_out receives the
 * exponent used.  hd_out (nullable) receives the damped, permuted Hessian
 * of the successful attempt.
 *
 * Part of the factor's work runs on a library-owned side stream (one per
 * device and caller stream, created on the first call with the caller
 * stream's priority) that forks from and joins back into `stream` through
 * events, so everything is complete in `stream` order when the call's work
 * is.  Make that first call outside stream capture; later calls may be
 * captured.
 */
int64_t gq_hessian_factor_workspace_size(int64_t d);
int gq_hessian_factor(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                      double damp_percent, float* u, int64_t ldu, float* hd_out,
                      void* workspace, int64_t workspace_bytes, int* attempt_out,
                      void* stream);

/* One damping attempt of gq_hessian_factor -- iteration `attempt` (0..4) of
 * gptq_ref.py:80-83, damp = damp_percent * 10^attempt -- enqueued on `stream`
 * with no host synchronization.  `status` is an int in DEVICE memory: 0 when
 * the damped Hessian factored (u then holds the factor), non-zero when a
 * pivot was not positive (u is then meaningless).  Lets a caller run the
 * factors of several Hessians concurrently on different streams and read all
 * statuses after one synchronization; gq_hessian_factor is this call in a
 * loop with a synchronization per attempt.  Same workspace as
 * gq_hessian_factor (the status word may live anywhere else). */
int gq_hessian_factor_attempt(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                              double damp_percent, int attempt, float* u, int64_t ldu,
                              float* hd_out, void* workspace, int64_t workspace_bytes,
                              int* status, void* stream);

/* The factor's building blocks, for hosts that split the factorization's
 * products across GPUs (jax_gptq_b200.distributed.factor_hessian_sharded):
 *
 * gq_hessian_prepare  b [d, d] (ld d) = J (h[perm][:, perm] + damp I) J in
 *                     its lower triangle, zeros above (J reverses the order;
 *                     damp = damp_percent * 10^attempt * mean(diag h), mean 0
 *                     -> 1, as gptq_ref.py:72-83); hd_out (nullable, ld d) the
 *                     damped permuted Hessian itself; mean: one device float.
 * gq_inv_chol         in place: the lower triangle of a [n, n] (lda, strict
 *                     upper zero) becomes L^-1 where a = L L^T (the recursion
 *                     and leaves of gq_hessian_factor); a non-positive pivot
 *                     sets *status (device int, not cleared here) non-zero.
 * gq_reverse_lower    u = J x J for the lower triangle x: u is the upper factor
 *                     u = chol(Hd^-1, upper) when x = L^-1 of the prepared b.
 * gq_sgemm_tri        gq_sgemm (uplo 0) with a triangular operand whose zero
 *                     triangle starts on 128 boundaries skipped per tile:
 *                     tri 1 A upper (k >= row), 2 A lower (k <= row), 3 B lower
 *                     (k <= col), 4 B upper (k >= col); 0 none.  Rows and
 *                     columns are the call's own, so a row slice of a
 *                     triangular A needs tri 0.
 */
int gq_hessian_prepare(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                       double damp_percent, int attempt, float* b, float* hd_out, float* mean,
                       void* stream);
int64_t gq_inv_chol_workspace_size(int64_t n);
int gq_inv_chol(float* a, int64_t n, int64_t lda, void* workspace, int64_t workspace_bytes,
                int* status, void* stream);
int gq_reverse_lower(const float* x, int64_t d, int64_t ldx, float* u, int64_t ldu, void* stream);
int gq_sgemm_tri(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                 const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
                 int64_t ldc, int tri, void* stream);

/* No counterpart in the reference: attempt 0 of the factor, formed straight
 * from the bf16 activations x[tokens, d] (ld ldx), with the same u and perm,
 * bit for bit, as gq_syrk_bf16 -> gq_act_order_perm(ordering) ->
 * gq_hessian_factor_attempt(attempt 0).  The Hessian is accumulated on
 * stats_stream in the factor's (act-order, reversed) feature order, leading
 * block first, and the factor runs on chain_stream: its first half starts as
 * soon as the leading block is formed, while the rest of H accumulates with
 * reserve_sms SMs left free.  The full H is never materialised (redo a
 * failed attempt, status != 0, from gq_syrk_bf16 and gq_hessian_factor).
 * x may be reused once stats_stream passes this call's work; u, perm and
 * status are complete in chain_stream order.  Requires d and ldx multiples
 * of 8, x 16-byte aligned, a 256-byte aligned workspace of
 * gq_factor_from_x_workspace_size(tokens, d) bytes, and d * 6 bytes of
 * shared memory for the column gather (d <= 37000 or so). */
int64_t gq_factor_from_x_workspace_size(int64_t tokens, int64_t d);
int gq_factor_from_x_attempt(const uint16_t* x, int64_t tokens, int64_t d, int64_t ldx,
                             int ordering, double damp_percent, int reserve_sms,
                             float* u, int64_t ldu, int32_t* perm,
                             void* workspace, int64_t workspace_bytes, int* status,
                             void* stats_stream, void* chain_stream);

/* ------------------------------------------------------------------------
 * GPTQ column sweep (the computation gptq_ref.py:136-155 stands in for).
 * With u = I it reproduces gptq_forward_step bit-exactly.
 *
 * w        [m, n] float32 original weights (ldw).
 * start    NULL, or [m, n] float32 (ld n) initial estimate already in permuted
 *          column order (replaces w[:, perm]).
 * u        [n, n] float32 upper factor in permuted coordinates (ldu).
 * perm     [n] int32 (NULL = identity).
 * block    lazy-batch width; 128 is supported.
 * group_size must divide n and either divide 128 (>= 4) or be a multiple of 128.
 * group0_scale/group0_zero  NULL, or [m] presets for group 0's parameters.
 * noprop_cols  leading (permuted) columns whose error is not propagated.
 * Outputs (each nullable): dequant/codes [m, n] original column order;
 * scales/zeros [m, n / group_size] permuted group order; g_idx [n] =
 * group of each original column.
 */
int64_t gq_gptq_sweep_workspace_size(int64_t m, int64_t n);
int gq_gptq_sweep(const float* w, int64_t m, int64_t n, int64_t ldw, const float* start,
                  const float* u, int64_t ldu, const int32_t* perm,
                  int w_bits, int group_size, int sym, int block,
                  const float* group0_scale, const float* group0_zero, int noprop_cols,
                  float* dequant, uint8_t* codes, float* scales, float* zeros,
                  int32_t* g_idx, void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * No counterpart in the reference.  gq_gptq_sweep for callers that cannot
 * allocate device memory -- e.g. a host framework that has reserved nearly
 * all GPU memory for its own pool, so that a cudaMalloc from a plugin fails,
 * with no way for the plugin to borrow from that pool.  Same arguments and
 * results as gq_gptq_sweep minus the workspace: the scratch comes from one
 * static device buffer of GQ_SWEEP_STATIC_SCRATCH_BYTES per GPU, held until
 * the process exits.  Sweeps needing more scratch than that
 * (gq_gptq_sweep_workspace_size(m, n) > GQ_SWEEP_STATIC_SCRATCH_BYTES,
 * roughly 6 million weights) return GQ_EINVAL.  All calls on a device share the
 * buffer: calls that may overlap on the GPU race and must be ordered.  The
 * first call on each device looks up the buffer's address; make it before any
 * stream capture begins.  The address is cached per (device, CUDA context);
 * a call made from another context (after cudaDeviceReset, or a context the
 * caller created) looks it up again, so that first call after the change
 * must also come before any capture.
 */
#define GQ_SWEEP_STATIC_SCRATCH_BYTES (32ll * 1024 * 1024)
int gq_gptq_sweep_static(const float* w, int64_t m, int64_t n, int64_t ldw, const float* start,
                         const float* u, int64_t ldu, const int32_t* perm,
                         int w_bits, int group_size, int sym, int block,
                         const float* group0_scale, const float* group0_zero, int noprop_cols,
                         float* dequant, uint8_t* codes, float* scales, float* zeros,
                         int32_t* g_idx, void* stream);

/* ------------------------------------------------------------------------
 * Qronos update (the computation qronos_ref.py:7-25 stands in for), with
 * h = Xt^T Xt from the quantized-model activations Xt and g = X^T Xt
 * (h_g_from_activations(x_quant=Xt, x_float=X)).
 *
 * w, w_orig [m, n] float32 (ld n): starting estimate and target weights.
 * hd  [n, n] damped Hessian in permuted coordinates (gq_hessian_factor's
 *     hd_out); u [n, n] its inverse-Cholesky factor; g [n, n] unpermuted.
 * perm [n] int32 (NULL = identity).  Outputs as for gq_gptq_sweep.
 */
int64_t gq_qronos_workspace_size(int64_t m, int64_t n);
int gq_qronos(const float* w, const float* w_orig, int64_t m, int64_t n, const float* hd,
              const float* u, const float* g, const int32_t* perm, int w_bits, int group_size,
              int sym, int block, float* dequant, uint8_t* codes, float* scales, float* zeros,
              int32_t* g_idx, void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * pallas/blocked_pivoted_qr.py:1627-1722 blocked_pivoted_qr: column-pivoted
 * Householder QR of a [m, n] float32 (lda), in place: on return a holds R in
 * its upper triangle and explicit zeros below (like the reference's `work`),
 * perm [n] int32 the column order.  pivot_mode 0 = "largest", 1 = "smallest",
 * 2 = no pivoting (plain Householder QR; perm is the identity; used with
 * semantics 1 for the unpivoted reduced QR of gptq_ref.py:112-122).
 * semantics 0 reproduces the reference's compiled panel path exactly (index
 * quirks and stale mid-panel pivots included); 1 is a correct blocked QRCP
 * (A[:, perm] = Q R, run in 64-wide panels).  panel_size <= 256 or >= min(m, n);
 * m <= 25600.  Optional outputs: v_out [m, min(m, n)] (ldv) the Householder
 * vectors (unit diagonal, zeros above), tau_out [min(m, n)], panel_ends and
 * n_panels the realized panel boundaries.  BLOCKING: synchronizes the stream
 * once per panel.
 */
int64_t gq_qrcp_workspace_size(int64_t m, int64_t n, int panel_size);
int gq_qrcp(float* a, int64_t m, int64_t n, int64_t lda, int panel_size, int pivot_mode,
            int semantics, int32_t* perm, float* v_out, int64_t ldv, float* tau_out,
            int32_t* panel_ends, int* n_panels, void* workspace, int64_t workspace_bytes,
            void* stream);

/* pallas/blocked_pivoted_qr.py:1412-1476 factor_panel_pallas: one panel from
 * column k, updating a, perm and norms in place; y_out [m - k, P] (ld P),
 * tau_out [P], t_out [P, P] with P = min(panel_size, min(m, n) - k);
 * *panel_end_out = k + accepted reflectors.  BLOCKING (one sync). */
int gq_qr_factor_panel(float* a, int64_t m, int64_t n, int64_t lda, int32_t* perm, float* norms,
                       int64_t k, int panel_size, int pivot_mode, int semantics, float* y_out,
                       float* tau_out, float* t_out, int* panel_end_out, void* workspace,
                       int64_t workspace_bytes, void* stream);

/* pallas/blocked_pivoted_qr.py:818-862 apply_compact_panel_to_block (and
 * :1592-1624 apply_panel_to_trailing_pallas on the block a[k:, panel_end:]):
 * b [rows, cols] <- b - Y (T^T (Y^T b)) with y [rows, width] (ldy),
 * t [width, width] (ldt).  scratch: 2 * width * cols floats. */
int gq_qr_apply_panel(float* b, int64_t rows, int64_t cols, int64_t ldb, const float* y,
                      int64_t ldy, const float* t, int64_t ldt, int width, float* scratch,
                      void* stream);

/* ------------------------------------------------------------------------
 * Packed quantized weights (the reference returns only the dequantized
 * floats of quant.py:37; this is the checkpoint form of a sweep's output).
 * packed [m, ldp] uint32: row r's codes (original column order, as
 * gq_gptq_sweep / gq_rtn write them) as one little-endian bit stream -- code c
 * in bits [c*bits, (c+1)*bits), word w = stream bits [32w, 32w+32).
 * gq_packed_words(n, bits) = ceil(n * bits / 32) words per row (-1 on bad
 * arguments).  gq_unpack_dequant returns the codes and/or the dequantized
 * weights (code + qmin - zero[g_idx[c]]) * scale[g_idx[c]], bit-identical to
 * the sweep's dequant output; scales/zeros [m, n_groups], g_idx [n]. */
int64_t gq_packed_words(int64_t n, int bits);
int gq_pack_codes(const uint8_t* codes, int64_t m, int64_t n, int64_t ldc, int bits,
                  uint32_t* packed, int64_t ldp, void* stream);
int gq_unpack_dequant(const uint32_t* packed, int64_t m, int64_t n, int64_t ldp, int bits, int sym,
                      const float* scales, const float* zeros, int64_t n_groups,
                      const int32_t* g_idx, float* dequant, uint8_t* codes, void* stream);

/* ------------------------------------------------------------------------
 * gptq_ref.py:95-99 (jnp.linalg.eigh of the Hessian in process_hessian's
 * eigh branch): symmetric eigendecomposition by parallel cyclic Jacobi.
 *
 * a [n, n] float32 symmetric (lda; read only).  w [n] eigenvalues in
 * ascending order (ties by index), v [n, n] (ldv) the matching eigenvectors
 * as columns, a = v diag(w) v^T.  Sweeps stop when a sweep rotates no pair
 * (|a_pq| <= 4 eps sqrt(|a_pp a_qq|) for all p < q) or after max_sweeps
 * (1..100); *sweeps_done (host, nullable) reports the count.  n <= 51200.
 * BLOCKING: synchronizes the stream once per sweep.  Workspace from
 * gq_syevj_workspace_size(n) (two n x n float32 buffers), 256-byte aligned.
 */
int64_t gq_syevj_workspace_size(int64_t n);
int gq_syevj(const float* a, int64_t n, int64_t lda, float* w, float* v, int64_t ldv,
             int max_sweeps, int* sweeps_done, void* workspace, int64_t workspace_bytes,
             void* stream);

/* ------------------------------------------------------------------------
 * eval.py:9-22 _masked_nll_from_logits: the next-token negative
 * log-likelihood summed over scored positions, for perplexity evaluation.
 *
 * logits  [batch, tokens, vocab] contiguous, dtype 0 = float32, 1 = bf16.
 * labels  [batch, tokens] int64; position t of entry b is scored against
 *         labels[b, t + 1] unless that label is -100 (then skipped); labels
 *         outside [0, vocab) are clamped to the range.
 * nll_sum (device double) = sum of logsumexp(logits[b, t]) - logits[b, t,
 *         label]; count (device int64) = number of scored positions.
 * Deterministic (fixed-order reduction).  Workspace from
 * gq_masked_nll_workspace_size(batch, tokens), 256-byte aligned.
 */
int64_t gq_masked_nll_workspace_size(int64_t batch, int64_t tokens);
int gq_masked_nll(const void* logits, int dtype, int64_t batch, int64_t tokens, int64_t vocab,
                  const int64_t* labels, double* nll_sum, int64_t* count, void* workspace,
                  int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Packed upper triangle of a symmetric d x d float32 matrix (row-major, ld
 * ldh), for summing token-sharded Hessians across GPUs with about half the
 * bytes.  128-row blocks b hold rows [128 b, 128 b + 128) from column 128 b
 * on, row-major, back to back (block b starts at 128 (b d - 64 b (b - 1))).
 * gq_sym_packed_size   floats of the packed form (about d^2 / 2 + 64 d).
 * gq_sym_pack_upper    packed <- h (h must be symmetric; the diagonal tiles
 *                      are copied whole).
 * gq_sym_unpack_upper  h <- the packed entries on or above the diagonal,
 *                      mirrored below it: exactly symmetric.
 * GQ_EINVAL for d < 0, NULL pointers with d > 0, or ldh < d. */
int64_t gq_sym_packed_size(int64_t d);
int gq_sym_pack_upper(const float* h, int64_t d, int64_t ldh, float* packed, void* stream);
int gq_sym_unpack_upper(const float* packed, int64_t d, float* h, int64_t ldh, void* stream);

/* ------------------------------------------------------------------------
 * Multi-GPU: a per-device handle with an optional NCCL communicator and the
 * in-place fp32 sum all-reduce used for token-sharded Hessians (H = sum over
 * ranks of X_r^T X_r).  The reference is single-device and has no
 * counterpart; these are the C-ABI form of jax_gptq_b200/distributed.py.
 * NCCL is loaded with dlopen on first use (a copy already loaded in the
 * process is reused); without it these calls return GQ_ENCCL.
 *
 * gq_nccl_unique_id     writes a 128-byte NCCL id (rank 0; share it with the
 *                       other ranks out of band).
 * gq_handle_create      wraps a caller-owned ncclComm_t (or NULL: a handle
 *                       without collectives); the comm is not destroyed.
 * gq_handle_create_nccl creates and owns a communicator: collective over
 *                       the nranks callers, one per GPU, same id.
 * gq_allreduce_sum_f32  buf[0:count] summed over the ranks, in place,
 *                       stream-ordered on `stream` (device of the handle).
 *                       A rank that never joins leaves the others waiting
 *                       inside NCCL until a host-side watchdog (a heartbeat
 *                       or a timeout on another thread) calls
 *                       gq_handle_abort, which ends the wait with an error.
 * gq_allreduce_sym_f32  the symmetric d x d x (ld ldx) summed over the ranks
 *                       in place through its packed upper triangle (half
 *                       the bytes): gq_sym_pack_upper into `packed`
 *                       (gq_sym_packed_size(d) floats, device memory), the
 *                       all-reduce, gq_sym_unpack_upper back into x.
 * gq_comm_check         polls NCCL's asynchronous error state (a failed or
 *                       lost peer); GQ_ENCCL when set, after aborting the
 *                       communicator if abort_on_error and the handle owns it.
 *                       Later collectives on an aborted handle return
 *                       GQ_ENCCL without launching.
 * gq_handle_abort       aborts an owned communicator (safe from another host
 *                       thread while a collective is stuck). */
typedef struct gq_handle gq_handle;
int gq_nccl_unique_id(void* id_out, int64_t id_bytes);
int gq_handle_create(int device, void* nccl_comm, gq_handle** out);
int gq_handle_create_nccl(int device, const void* unique_id, int nranks, int rank,
                          gq_handle** out);
int gq_handle_destroy(gq_handle* h);
int gq_handle_ranks(const gq_handle* h, int* nranks, int* rank);
int gq_allreduce_sum_f32(gq_handle* h, float* buf, int64_t count, void* stream);
int gq_allreduce_sym_f32(gq_handle* h, float* x, int64_t d, int64_t ldx, float* packed,
                         void* stream);
int gq_comm_check(gq_handle* h, int abort_on_error);
int gq_handle_abort(gq_handle* h);

#ifdef __cplusplus
}
#endif

#endif /* GQ_H_ */
