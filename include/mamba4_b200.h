/*
 * mamba4_b200 - C ABI of the B200 (sm_100a) FlashMamba hot path.
 *
 * Two operators of tasmaikeni13/mamba4's `lm/kernels` surface, each a
 * forward/backward pair:
 *
 *   - the selective conjugate memory read
 *       (reference: selective_memory_fused, lm/kernels/mamba4_fused.py:372-454,
 *        contract of selective_gaussian_memory, lm/kernels/mamba4.py:228-338)
 *   - the Mamba-3 SISO chunked scan in the projection layout
 *       (reference: mamba3_fused, lm/kernels/flashmamba.py:1114-1162,
 *        fused_scan custom_vjp, :859-1102)
 *
 * Conventions
 *   - All pointers are device pointers (cudaMalloc'd or framework-owned).
 *     The library never allocates: the caller sizes residual and workspace
 *     buffers with the *_bytes queries and passes them in.
 *   - `stream` is a cudaStream_t passed as void*; every call is asynchronous
 *     on it and reentrant (no global mutable state; the one exception,
 *     m4_scan_bwd_noalloc, documents its shared scratch below).
 *   - Tensors are dense, row-major, in the layouts stated per argument.
 *   - Every entry point returns an M4Status; nonzero means nothing was
 *     launched (argument errors) or a launch failed (M4_ERR_LAUNCH).
 *     m4_status_string() names a code. No entry point traps or asserts.
 *   - Results are deterministic: fixed reduction orders, no float atomics.
 */
#ifndef MAMBA4_B200_H
#define MAMBA4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  M4_OK = 0,
  M4_ERR_DIMS = 1,        /* a dimension is non-positive or inconsistent */
  M4_ERR_UNSUPPORTED = 2, /* a dimension this build does not implement */
  M4_ERR_NULL = 3,        /* a required pointer is NULL */
  M4_ERR_ALIGN = 4,       /* a pointer is not 16-byte aligned */
  M4_ERR_LAUNCH = 5,      /* a CUDA launch reported an error */
  M4_ERR_WORKSPACE = 6,   /* residual/workspace buffer too small */
  M4_ERR_TIMEOUT = 7      /* a bounded device wait on the tensor cores gave up */
} M4Status;

/* Memory-read problem size. key_dim must be 64 and value_dim 64 or 128
 * (the host adapter pads smaller dimensions with an identity block, as the
 * reference's batched_solve pads to 8, lm/kernels/mamba4_fused.py:289-297). */
typedef struct {
  int batch;      /* B */
  int time;       /* T, any length >= 1 (padded internally) */
  int heads;      /* H */
  int key_dim;    /* D = 64 */
  int value_dim;  /* P = 64 or 128 */
} M4MemDims;

/* Bytes of the forward residual (stored LDL^T factors, solutions and
 * chunk-start statistics) that m4_memread_bwd consumes. The reference keeps
 * the same residuals under the remat name "memory_solve"
 * (lm/kernels/mamba4_fused.py:329-337). */
size_t m4_memread_residual_bytes(const M4MemDims* dims);

/* Bytes of scratch the backward needs. */
size_t m4_memread_workspace_bytes(const M4MemDims* dims);

/* Forward read. Replaces selective_memory_fused's forward
 * (lm/kernels/mamba4_fused.py:372-454; custom-VJP forward :329-337).
 *   keys, queries [B,T,H,D]; values [B,T,H,P]; beta, log_decay [B,T,H];
 *   floor [H,D]; init_evidence [B,H,D,D] and init_cross [B,H,P,D] or NULL
 *   (zero state, lm/kernels/mamba4.py:221-225).
 * Outputs: output [B,T,H,P], variance [B,T,H], final_evidence [B,H,D,D],
 *   final_cross [B,H,P,D]; residual as sized above. */
int m4_memread_fwd(const M4MemDims* dims, const float* keys, const float* values,
                   const float* queries, const float* beta, const float* log_decay,
                   const float* floor, const float* init_evidence,
                   const float* init_cross, float* output, float* variance,
                   float* final_evidence, float* final_cross, void* residual,
                   size_t residual_bytes, void* stream);

/* Backward of the read. Replaces _chunk_solve_backward
 * (lm/kernels/mamba4_fused.py:340-366) together with the JAX autodiff of the
 * surrounding chunk algebra (:402-447). Inputs as m4_memread_fwd plus the
 * residual it wrote and the cotangents d_output [B,T,H,P],
 * d_variance [B,T,H], d_final_evidence [B,H,D,D] / d_final_cross [B,H,P,D]
 * (either may be NULL = zero). Writes every input gradient; d_init_evidence
 * and d_init_cross may be NULL when no initial state is differentiated. */
int m4_memread_bwd(const M4MemDims* dims, const float* keys, const float* values,
                   const float* queries, const float* beta, const float* log_decay,
                   const float* floor, const float* init_evidence,
                   const float* init_cross, const void* residual,
                   size_t residual_bytes, const float* d_output,
                   const float* d_variance, const float* d_final_evidence,
                   const float* d_final_cross, float* d_keys, float* d_values,
                   float* d_queries, float* d_beta, float* d_log_decay,
                   float* d_floor, float* d_init_evidence, float* d_init_cross,
                   void* workspace, size_t workspace_bytes, void* stream);

/* One-token read against a carried state. Replaces selective_decode
 * (lm/kernels/mamba4.py:341-355): evidence' = lam evidence + beta k k^T,
 * cross' = lam cross + beta v k^T, y = (evidence' + diag(floor))^-1 query,
 * output = cross' y, variance = query . y, lam = exp(log_decay).
 * dims: batch, heads, key_dim 64, value_dim 64 or 128 (time is ignored).
 *   evidence [B,H,D,D], cross [B,H,P,D]; key, query [B,H,D] (16-byte aligned);
 *   value [B,H,P]; beta, log_decay [B,H]; floor [H,D].
 * Outputs: output [B,H,P], variance [B,H], evidence_out [B,H,D,D],
 *   cross_out [B,H,P,D]; evidence_out / cross_out may be evidence / cross
 *   (updated in place). */
int m4_memread_decode(const M4MemDims* dims, const float* evidence, const float* cross,
                      const float* key, const float* value, const float* query,
                      const float* beta, const float* log_decay, const float* floor,
                      float* output, float* variance, float* evidence_out, float* cross_out,
                      void* stream);

/* Standalone SPD solve. Replaces spd_solve (lm/kernels/mamba4.py:187-218)
 * with its factorization backends (_cholesky_loop / _cholesky_blocked /
 * _cholesky_unrolled, :31-125, and _triangular_solves, :138-158): for each of
 * `count` matrices, solve precision y = rhs with a block LDL^T factorization
 * (8x8 pivot blocks; the same exact solve as the reference's Cholesky to
 * float32 rounding).
 *   precision [count, dim, dim] row-major, SPD, only the lower triangle read;
 *   rhs, solution [count, dim]; dim 1..64 (orders below 64 are padded with an
 *   identity block inside the kernel). No alignment needed for these.
 *   factor: the stored LDL^T factor for the backward, sized by
 *   m4_spd_solve_factor_bytes (9,216 bytes per matrix, 16-byte aligned).
 * count 0 launches nothing and returns M4_OK. */
size_t m4_spd_solve_factor_bytes(int count, int dim);
int m4_spd_solve_fwd(int count, int dim, const float* precision, const float* rhs,
                     float* solution, void* factor, size_t factor_bytes, void* stream);

/* Backward of m4_spd_solve_fwd (_spd_solve_backward, lm/kernels/mamba4.py:208-215):
 * z = precision^-1 d_solution from the stored factor, d_rhs = z [count, dim],
 * d_precision = -(z y^T + y z^T) / 2 [count, dim, dim] (every entry, the
 * reference's symmetric cotangent), y = the forward's solution. */
int m4_spd_solve_bwd(int count, int dim, const void* factor, size_t factor_bytes,
                     const float* solution, const float* d_solution, float* d_precision,
                     float* d_rhs, void* stream);

/* Scan problem size (projection layout of mamba3_fused). */
typedef struct {
  int batch;        /* B */
  int time;         /* T, any length >= 1 */
  int heads;        /* H */
  int head_dim;     /* P = 64 */
  int state_dim;    /* N = 64 */
  int angle_count;  /* A <= N/2 rotation pairs */
  int chunk;        /* chunk length: 64 */
  int bf16;         /* 1: c, b, x, y, d_y, dc, db, dx are bfloat16; 0: float32 */
  int per_head;     /* 1: q/k [B,T,H,N] and angles [B,T,H,A] per head
                       (mamba3_flash_heads, lm/kernels/flashmamba.py:467-502);
                       0: shared c/b [B,T,N] and angles [B,T,A] (mamba3_fused) */
} M4ScanDims;

size_t m4_scan_residual_bytes(const M4ScanDims* dims);
size_t m4_scan_workspace_bytes(const M4ScanDims* dims);

/* Forward scan. Replaces mamba3_fused's forward
 * (lm/kernels/flashmamba.py:1114-1162 -> _fused_forward_pass :901-959).
 *   c (queries C), b (keys B): [B,T,N] (per_head: [B,T,H,N]); x [B,T,H*P];
 *   adt, dt, trap_logits [B,T,H] float32; angles [B,T,A] (per_head [B,T,H,A])
 *   float32 rates; q_bias, k_bias [H,N] float32 (may be NULL = zero).
 * Outputs: y [B,T,H*P] (dtype of x), final_state [B,H,N,P] float32;
 *   residual: chunk-start states and phases (remat name "ssd_scan").
 * bfloat16 operands: c, b and x must be 16-byte aligned (M4_ERR_ALIGN). */
int m4_scan_fwd(const M4ScanDims* dims, const void* c, const void* b, const void* x,
                const float* adt, const float* dt, const float* trap_logits,
                const float* angles, const float* q_bias, const float* k_bias,
                void* y, float* final_state, void* residual, size_t residual_bytes,
                void* stream);

/* Backward scan. Replaces _fused_backward (lm/kernels/flashmamba.py:996-1099)
 * and the JAX autodiff of mamba3_fused's preprocessing (:1142-1147,
 * angle_rates :1105-1111). d_final may be NULL (zero). Writes dc, db
 * (dtype of c/b; shared layouts sum over heads in a fixed order), dx,
 * d_adt, d_dt, d_trap_logits [B,T,H], d_angles (shape of angles),
 * d_q_bias, d_k_bias [H,N] (may be NULL). bfloat16 operands: c, b, x and
 * d_y must be 16-byte aligned (M4_ERR_ALIGN). */
int m4_scan_bwd(const M4ScanDims* dims, const void* c, const void* b, const void* x,
                const float* adt, const float* dt, const float* trap_logits,
                const float* angles, const float* q_bias, const float* k_bias,
                const void* residual, size_t residual_bytes, const void* d_y,
                const float* d_final, void* dc, void* db, void* dx, float* d_adt,
                float* d_dt, float* d_trap_logits, float* d_angles,
                float* d_q_bias, float* d_k_bias, void* workspace,
                size_t workspace_bytes, void* stream);

/* One-token scan step against a carried cache. Replaces the scan core of
 * _Mamba3StepMixer (lm/models/mamba4.py:412-481): phase' = phase + rate dt;
 * Q, K = rotate(c + q_bias, phase'), rotate(b + k_bias, phase') (rounded to
 * the model dtype after the bias and after the rotation, as the reference);
 * state' = e^(adt) (state + dt (1 - sigmoid(trap)) k_prev v_prev^T)
 *          + dt sigmoid(trap) K x^T;  y = Q^T state'.
 * dims: batch, heads, head_dim 64, state_dim 64, angle_count, bf16, per_head
 * (time and chunk are ignored).
 *   cache: state [B,H,N,P] (16-byte aligned), prev_keys [B,H,N],
 *   prev_values [B,H,P], phase [B,H,A], all float32;
 *   c, b [B,N] (per_head: [B,H,N]) and x [B,H*P] in the model dtype;
 *   adt, dt, trap_logits [B,H]; angles [B,A] (per_head [B,H,A]) rates;
 *   q_bias, k_bias [H,N] or NULL.
 * Outputs: y [B,H*P] (model dtype) and the new cache (K, x and phase'); the
 * output cache pointers may equal the input ones (updated in place).
 * Stepping a zero cache through a sequence reproduces m4_scan_fwd's y and
 * final state. */
int m4_scan_step(const M4ScanDims* dims, const float* state, const float* prev_keys,
                 const float* prev_values, const float* phase, const void* c, const void* b,
                 const void* x, const float* adt, const float* dt, const float* trap_logits,
                 const float* angles, const float* q_bias, const float* k_bias, void* y,
                 float* state_out, float* prev_keys_out, float* prev_values_out,
                 float* phase_out, void* stream);

/* Backward scan that allocates nothing (no counterpart in the reference).
 * For callers that may not allocate device memory while the operator runs:
 * an XLA FFI custom call or other framework plugin that must not use the
 * device allocator, work recorded into a CUDA graph, or a server that
 * reserves all device memory up front. Same arguments and results as
 * m4_scan_bwd, without the workspace: its scratch is a fixed 32 MiB array
 * inside the library, held on every GPU that loads the library until exit.
 * Limit: m4_scan_workspace_bytes(dims) must not exceed 32 MiB (batch x time
 * x heads up to about 36,000); larger problems return M4_ERR_WORKSPACE and
 * launch nothing. The first call on a device looks up the array's device
 * address (with the current device) - make that first call before any
 * stream capture. The address is kept for the life of the process, so the
 * device's context must not be reset (cudaDeviceReset) between calls. All
 * calls share the one array: calls that overlap on the GPU (on different
 * streams) race and must not be issued. Nothing in the array needs clearing
 * between calls: every scratch byte a call reads, it writes first. */
int m4_scan_bwd_noalloc(const M4ScanDims* dims, const void* c, const void* b, const void* x,
                        const float* adt, const float* dt, const float* trap_logits,
                        const float* angles, const float* q_bias, const float* k_bias,
                        const void* residual, size_t residual_bytes, const void* d_y,
                        const float* d_final, void* dc, void* db, void* dx, float* d_adt,
                        float* d_dt, float* d_trap_logits, float* d_angles,
                        float* d_q_bias, float* d_k_bias, void* stream);

/* ------------------------------------------------------------------------
 * Model glue (PyTorch Mamba 4 LM in this repository). Fused forms of the
 * reference's XLA elementwise code around the scan; all bf16 tensors are
 * row-major, one row per token.
 * ---------------------------------------------------------------------- */

/* Mamba-3 mixer in-projection layout (lm/models/mamba3.py:60-73): each row of
 * `proj` holds z [inner], x [inner], b [N], c [N], raw_dt [heads],
 * raw_a [heads], trap [heads], angles [angles] (bfloat16), N = state_dim. */
typedef struct {
  int rows;       /* B*T */
  int inner;      /* d_model * expand, a multiple of 256, = 64 * heads */
  int heads;      /* <= 32 */
  int angles;     /* rotation pairs, <= state_dim / 2 */
  float eps;      /* RMSNorm epsilon of B_norm / C_norm */
  int stride;     /* elements between rows of proj and d_proj: a multiple of 8 that
                     is at least 2 inner + 2 state_dim + 3 heads + angles */
  int state_dim;  /* N: 64, 96 or 128 (the width of the b and c slices) */
} M4MixerDims;

/* Rows of the per-warp partial-sum buffers the backward calls need
 * (post: rows x heads floats; prep: rows x (2 state_dim + heads) floats). */
size_t m4_mixer_partial_rows(const M4MixerDims* dims);

/* Before the scan (lm/models/mamba3.py:76-103): c = C_norm(c), b = B_norm(b)
 * [rows,N] bf16; x copied to [rows,inner]; dt = softplus(raw_dt + dt_bias),
 * adt = -max(heavy_tail(raw_a), 1e-4) * dt, trap, angles as float32. */
int m4_mixer_prep_fwd(const M4MixerDims* dims, const void* proj, const float* b_scale,
                      const float* c_scale, const float* dt_bias, void* c_out, void* b_out,
                      void* x_out, float* adt, float* dt, float* trap, float* angles,
                      void* stream);

/* After the scan (lm/models/mamba3.py:115-117):
 * out = bf16((y + x * D[head]) * silu(z)), [rows, inner]. */
int m4_mixer_post_fwd(const M4MixerDims* dims, const void* proj, const void* y, const float* D,
                      void* out, void* stream);

/* Backward of m4_mixer_post_fwd: d_y (scan cotangent, bf16 [rows,inner]), the z
 * columns of d_proj, and dD [heads] (via dD_part). */
int m4_mixer_post_bwd(const M4MixerDims* dims, const void* proj, const void* y, const float* D,
                      const void* g_out, void* d_y, void* d_proj, float* dD_part, float* dD,
                      void* stream);

/* Backward of m4_mixer_prep_fwd and of the x term of the D skip: every
 * d_proj column except z, and the B/C norm scale and dt_bias gradients. */
int m4_mixer_prep_bwd(const M4MixerDims* dims, const void* proj, const float* b_scale,
                      const float* c_scale, const float* dt_bias, const float* D, const void* g_out,
                      const void* dc, const void* db, const void* dx, const float* d_adt,
                      const float* d_dt, const float* d_trap, const float* d_angles, void* d_proj,
                      float* part, float* d_b_scale, float* d_c_scale, float* d_dt_bias,
                      void* stream);

/* bfloat16 RMSNorm with float32 statistics (lm/models/common.py:25-45) over
 * `features` in {256, 512, 768, 1024}; rstd [rows] is saved for backward. */
/* Residual add fused with the next block's RMSNorm (decode, no backward):
 * x_out = bf16(x + delta), y = bf16(rmsnorm(x_out) * scale) over bf16 rows of
 * `features` in {256, 512, 768, 1024}; x_out may alias x (the decode blocks'
 * residual, lm/models/mamba4.py:358 and :404, followed by the next block's
 * norm or the final norm, :514-522). */
int m4_add_rmsnorm_fwd(int rows, int features, float eps, const void* x, const void* delta,
                       const float* scale, void* x_out, void* y, void* stream);
size_t m4_rmsnorm_partial_rows(int rows);
int m4_rmsnorm_fwd(int rows, int features, float eps, const void* x, const float* scale, void* y,
                   float* rstd, void* stream);
int m4_rmsnorm_bwd(int rows, int features, const void* x, const float* scale, const float* rstd,
                   const void* gy, void* gx, float* part, float* d_scale, void* stream);

/* Selective-memory mixer glue (lm/models/mamba4.py:155-260): key dim 64,
 * value dim 128, 1 to 16 heads. `rest` is the projection
 * after the gate columns: value [128h], key [64h], query [64h],
 * beta_raw [h], dt_raw [h], order_raw [h] per row (bf16, row stride
 * `stride`, a multiple of 8); d_rest has the same row stride. The gate view
 * has row stride `gate_stride`, and so has d_gate [rows,128h]: the two
 * gradients can be column slices of one projection-gradient buffer. */
typedef struct {
  int batch, time, heads;
  int stride;       /* row stride of rest, elements */
  int gate_stride;  /* row stride of the gate view, elements */
  float beta_max;   /* memory_beta_max */
} M4MemMixDims;

/* Floats needed by the `part` scratch of the backward calls. */
size_t m4_memmix_partial_floats(const M4MemMixDims* dims);

/* Causal depthwise conv (weights minus `bound`, bias) + SiLU of the value/key/
 * query channels (:98-108, :170-182); keys shifted one token (:183-194) and
 * unit-normalised with queries (:37-39); beta = beta_max sigmoid(raw + bias),
 * log_decay = -exp(a_log) softplus(raw + dt_bias), order logit = raw + 2. */
int m4_memmix_prep_fwd(const M4MemMixDims* dims, const void* rest, const float* conv_w,
                       const float* conv_b, float bound, const float* beta_bias, const float* dt_bias,
                       const float* a_log, float* values, float* keys, float* queries, float* beta,
                       float* log_decay, float* order_logit, void* stream);
int m4_memmix_prep_bwd(const M4MemMixDims* dims, const void* rest, const float* conv_w,
                       const float* conv_b, float bound, const float* beta_bias, const float* dt_bias,
                       const float* a_log, const float* d_values, const float* d_keys,
                       const float* d_queries, const float* d_beta, const float* d_log_decay,
                       const float* d_order_logit, float* d_conv, void* d_rest, float* part,
                       float* d_conv_w, float* d_conv_b, float* d_beta_bias, float* d_dt_bias,
                       float* d_a_log, void* stream);

/* Order head h_t = lam_t h_(t-1) + (1 - lam_t) v_t, lam = sigmoid(logit)
 * (:59-95), [B,T,h,128], segment-parallel over 64-token segments; backward
 * writes d_values and four per-warp partials of d_logit per (b, t, head).
 * `scratch` holds m4_memmix_order_scratch_floats(dims) floats. */
size_t m4_memmix_order_scratch_floats(const M4MemMixDims* dims);
int m4_memmix_order_fwd(const M4MemMixDims* dims, const float* values, const float* logit,
                        float* ordered, float* scratch, void* stream);
int m4_memmix_order_bwd(const M4MemMixDims* dims, const float* values, const float* logit,
                        const float* ordered, const float* g_ordered, float* d_values,
                        float* d_logit4, float* scratch, void* stream);

/* Confidence gate, D skip, order mix, read RMSNorm (eps) and SiLU gate
 * (:238-260): y [rows, 128h] bf16, rstd [rows*h] saved for backward. */
int m4_memmix_post_fwd(const M4MemMixDims* dims, float eps, const float* out, const float* var,
                       const float* values, const float* ordered, const void* gate,
                       const float* conf_scale, const float* D, const float* order_mix,
                       const float* scale, void* y, float* rstd, void* stream);
int m4_memmix_post_bwd(const M4MemMixDims* dims, const float* out, const float* var,
                       const float* values, const float* ordered, const void* gate,
                       const float* conf_scale, const float* D, const float* order_mix,
                       const float* scale, const float* rstd, const void* g_y, float* d_out,
                       float* d_var, float* d_values, float* d_ordered, void* d_gate, float* part,
                       float* d_conf_scale, float* d_D, float* d_order_mix, float* d_scale,
                       void* stream);

/* One cached decode token of the mixer glue (the cache branch of
 * lm/models/mamba4.py:127-337). prep_step: `rest` holds, per sequence,
 * `time` rows (the conv history, oldest first, then the current token; row
 * stride `stride`); only the current token is written ([batch, h, ...]),
 * with its own unit key, not shifted - the caller reads with the key it
 * carried from the previous token. post_step (time = 1): as post_fwd, with
 * the order head advanced in place of a precomputed order output:
 * o = s o_prev + (1 - s) v, s = sigmoid(order_logit) (order_prev and
 * order_out [batch, h, 128] both NULL: no order head, o = 0); no rstd. */
int m4_memmix_prep_step(const M4MemMixDims* dims, const void* rest, const float* conv_w,
                        const float* conv_b, float bound, const float* beta_bias, const float* dt_bias,
                        const float* a_log, float* values, float* keys, float* queries, float* beta,
                        float* log_decay, float* order_logit, void* stream);
int m4_memmix_post_step(const M4MemMixDims* dims, float eps, const float* out, const float* var,
                        const float* values, const float* order_logit, const float* order_prev,
                        float* order_out, const void* gate, const float* conf_scale, const float* D,
                        const float* order_mix, const float* scale, void* y, void* stream);

/* Softmax cross-entropy over bf16 logits [rows, vocab], rows `ld` elements
 * apart (ld >= vocab, a multiple of 8; columns past vocab are ignored), with
 * int64 targets (lm/train.py:81-87): loss and log-sum-exp [rows]; targets
 * outside [0, vocab) give loss 0. The backward overwrites `logits` with
 * g[r] * (softmax - onehot) in bf16 (0 past vocab). */
int m4_cross_entropy_fwd(int rows, int vocab, int ld, const void* logits, const int64_t* targets,
                         float* loss, float* lse, void* stream);
int m4_cross_entropy_bwd(int rows, int vocab, int ld, void* logits, const int64_t* targets,
                         const float* lse, const float* g, void* stream);

/* Device-side status of the tensor-core (tcgen05) kernels on the current
 * device: M4_ERR_TIMEOUT if a bounded wait for tensor-core completion gave
 * up since the last call (the flag is then cleared), else M4_OK.
 * Synchronous; call after the stream work of interest has finished. */
int m4_device_status(void);

/* Name of a status code (static string). */
const char* m4_status_string(int status);

/* Library version string, e.g. "mamba4_b200 0.1 sm_100a". */
const char* m4_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA4_B200_H */
