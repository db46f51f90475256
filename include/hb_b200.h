/* hummingbird-b200: C ABI of the B200 (sm_100a) kernels for hummingbird's three hot paths.
 *
 * Conventions for every entry point:
 *   - plain device pointers and sizes; bf16 tensors are passed as `const void*` holding IEEE bfloat16;
 *   - buffers are owned by the caller; nothing here allocates device memory; work that needs scratch
 *     space takes a caller-provided workspace whose size the matching *_workspace_bytes query returns;
 *   - every call is asynchronous on the given stream and returns an HbStatus (0 = HB_OK); an
 *     unsupported shape returns HB_ERR_SHAPE before anything is launched (the reference raises
 *     ValueError at trace time for the same cases);
 *   - there is no CPU fallback: a non-sm_100 device returns HB_ERR_ARCH.
 * The reference is kelechi-c/hummingbird (Python package `sa3jax`); citations are file:line in it.
 */
#ifndef HB_B200_H_
#define HB_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status --------------------------------------------------------------------------------------- */
/* Values of HbStatus: see hummingbird_b200/csrc/hb_status.h (0 ok, 1 shape, 2 align, 3 arch, 4 launch,
 * 5 device, 6 timeout, 7 workspace, 8 nccl, 9 null). */

/* Library version, major * 10000 + minor * 100 + patch. */
int hb_version(void);

/* Read and clear the device status word of the current device that the kernels set when a bounded
 * device-side wait expires (HB_ERR_TIMEOUT) or a device check fails. Synchronises `stream` first.
 * No reference counterpart: the reference surfaces errors only as Python exceptions at trace time. */
int hb_device_status(unsigned int* status_out, cudaStream_t stream);

/* ---- dense differential self-attention (DiT) ------------------------------------------------------- */
/* Bytes of workspace hb_dense_diff_attn needs for `pair_count` head pairs. */
int hb_dense_workspace_bytes(int batch, int length, int pair_count, size_t* bytes);

/* Replaces `sa3jax.dense_attention.dense_attention(qkv, q_weight, k_weight, cos, sin, mask, num_heads,
 * head_dim, half, eps)` (dense_attention.py:104-153), the kernel `dit._self_attention` calls under
 * `DiTConfig.attention == "fused"` (dit.py:185-195, config.py:57).
 *   qkv       bf16 [batch, length, qkv_row_stride]; columns [q | k | v | q_diff | k_diff], each
 *             num_heads * 64 wide (dense_attention.py:9-10); qkv_row_stride >= 5 * num_heads * 64.
 *   q_weight, k_weight  fp32 [64] RMSNorm scales.
 *   cos, sin  fp32 [length, table_stride] lane tables (`dense_attention.tables`, dense_attention.py:97-101):
 *             column d < 64 is the cos / signed sin for head dim d; table_stride >= 64 (128 for the
 *             reference's lane tables).
 *   vmask     bf16 value mask, element (b, l) at vmask[b * mask_batch_stride + l * mask_row_stride].
 *   lam       fp32 [num_heads / 2] per-pair lambda of `A - lambda * B`, or NULL for lambda = 1 (the reference).
 *   out       bf16; row (b, l) at out + (b * length + l) * out_row_stride, pointing at the output column of
 *             head 2 * pair_begin; 2 * pair_count * 64 columns are written.
 *   half      rotate-half width (16 for the reference's 32-dim rotary, 32 for a full-head rotary); a
 *             multiple of 8 in [8, 32].
 *   pair_begin, pair_count  head-pair range computed (head-pair sharding; the full call is 0, num_heads/2).
 * head_dim must be 64 and num_heads even (dense_attention.py:119-120). */
int hb_dense_diff_attn(const void* qkv, int64_t qkv_row_stride, const float* q_weight, const float* k_weight,
                       const float* cos, const float* sin, int64_t table_stride, const void* vmask,
                       int64_t mask_batch_stride, int64_t mask_row_stride, const float* lam, void* out,
                       int64_t out_row_stride, int batch, int length, int num_heads, int head_dim, int half,
                       float eps, int pair_begin, int pair_count, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* Allocation-free form of hb_dense_diff_attn, for callers that cannot allocate device memory or pass a
 * workspace (e.g. a handler inside a runtime that has reserved most of the GPU's memory for its own
 * allocator, or code that must not let cudaMalloc / cudaFree synchronise the device mid-stream). No
 * counterpart exists in the reference. Same arguments and results as hb_dense_diff_attn without the
 * workspace: the prepared tiles go to one scratch array of hb_dense_noalloc_max_bytes (64 MiB) built into
 * the library, which every device that loads the library holds until the process exits.
 *   - Problems whose workspace (hb_dense_workspace_bytes) exceeds that size return HB_ERR_WORKSPACE before
 *     anything is launched (e.g. B=1, L=1,422, 24 heads needs 22.5 MiB; B=2, L=2,648, 16 heads 53.8 MiB).
 *   - The first call on a device looks up the scratch's device address (once per device, with that device
 *     current); make that first call before capturing a stream.
 *   - All calls on a device share the one scratch array and it keeps the previous call's contents (each call
 *     rewrites every byte it reads, so nothing needs clearing): calls that may overlap on the GPU (other
 *     streams, other host threads) race on it and must be serialised by the caller. */
int hb_dense_noalloc_max_bytes(size_t* bytes);
int hb_dense_diff_attn_noalloc(const void* qkv, int64_t qkv_row_stride, const float* q_weight, const float* k_weight,
                               const float* cos, const float* sin, int64_t table_stride, const void* vmask,
                               int64_t mask_batch_stride, int64_t mask_row_stride, const float* lam, void* out,
                               int64_t out_row_stride, int batch, int length, int num_heads, int head_dim, int half,
                               float eps, int pair_begin, int pair_count, cudaStream_t stream);

/* ---- differential cross-attention (DiT) ------------------------------------------------------------- */
/* Replaces the attention of `sa3jax.dit._cross_attention` (dit.py:203-215): `_attend` with no RoPE and no
 * mask (dit.py:150-176) and `_attend_out`'s `SDPA(q, k, v) - SDPA(q_diff, k_diff, v)` (dit.py:131-147), up to
 * (not including) `to_out`. The reference runs it as XLA ops; this is one kernel:
 *   q         bf16 [batch, q_len, q_row_stride]: the `to_q` output, columns [q | q_diff], each num_heads * 64.
 *   kv        bf16 [batch, kv_len, kv_row_stride]: the hoisted `to_kv` output (dit.py:274-284), columns
 *             [k | k_diff | v], each num_heads * 64; kv_len <= 384.
 *   q_weight  fp32 [64] q RMSNorm scale (applied to q and q_diff, dit.py:167-169).
 *   k_weight  fp32 [64] k RMSNorm scale applied to k and k_diff here, or NULL when kv already holds the
 *             k-normed keys (the reference hoists the norm, dit.py:122-128, 283).
 *   lam       fp32 [num_heads / 2] per-pair lambda of `A - lambda * B`, or NULL for lambda = 1 (the reference).
 *   out       bf16; row (b, l) at out + (b * q_len + l) * out_row_stride, head h at column h * 64.
 * Scores are q k^T / 8 in fp32; softmax in fp32 with bf16 weights into P V, normalised after P V; each branch
 * normalised, then one fp32 subtraction and one bf16 cast. head_dim must be 64; rows 16-byte aligned. */
int hb_cross_diff_attn(const void* q, int64_t q_row_stride, const void* kv, int64_t kv_row_stride,
                       const float* q_weight, const float* k_weight, const float* lam, void* out,
                       int64_t out_row_stride, int batch, int q_len, int kv_len, int num_heads, int head_dim,
                       float eps, cudaStream_t stream);

/* ---- band (sliding-window) differential attention (SAME-L decoder) --------------------------------- */
/* Bytes of workspace hb_band_diff_attn needs for `rows` buffer rows, `pair_count` head pairs, `window` and
 * rotate-half width `half`: a rows x half (cos, sin) table for window <= 128 (the fused kernel), prepared
 * operand tiles otherwise. */
int hb_band_workspace_bytes(int batch, int rows, int pair_count, int window, int half, size_t* bytes);

/* Stage selector of hb_band_diff_attn: the call is a prologue kernel that prepares DyT/RoPE'd operand
 * tiles in the workspace, then the attention kernel that consumes them. HB_STAGE_ALL runs both; the two
 * halves can be issued separately (same arguments, same workspace) to overlap other work between them. */
#define HB_STAGE_PREPARE 1
#define HB_STAGE_ATTEND 2
#define HB_STAGE_ALL 3

/* Replaces `sa3jax.band_attention.band_attention(qkv, q_norm, k_norm, inv_freq, num_heads, head_dim,
 * window)` (band_attention.py:123-180), the kernel `same_l._attention` calls under
 * `SameConfig.attention == "pallas"` (same_l.py:151-161, config.py:115).
 *   qkv       bf16 [batch, rows, qkv_row_stride], columns as for the dense path. `rows` counts every row
 *             in the buffer, including halo rows received from neighbouring sequence shards.
 *   q_norm, k_norm  fp32 [129] DyT parameters {alpha, gamma[64], beta[64]} shared by both branches.
 *   inv_freq  fp32 [half] RoPE frequencies; angles are fp32(pos0 + row) * inv_freq (band_attention.py:43-58).
 *   lam       fp32 [num_heads / 2] or NULL (lambda = 1).
 *   out       bf16; query row i (0 <= i < q_count, buffer row q_begin + i) of batch b at
 *             out + (b * q_count + i) * out_row_stride, pointing at the column of head 2 * pair_begin.
 *   window    band half-width: query at buffer row r sees keys k with |k - r| <= window, 0 <= k < rows.
 *   pos0      global sequence position of buffer row 0 (0 unless sequence-sharded).
 * head_dim must be 64 (band_attention.py:138-140). */
int hb_band_diff_attn(const void* qkv, int64_t qkv_row_stride, const float* q_norm, const float* k_norm,
                      const float* inv_freq, int half, const float* lam, void* out, int64_t out_row_stride,
                      int batch, int rows, int q_begin, int q_count, int64_t pos0, int num_heads, int head_dim,
                      int window, int pair_begin, int pair_count, void* workspace, size_t workspace_bytes,
                      int stages, cudaStream_t stream);

/* The SAME-L attention front end in one GEMM (same_l.py:157-160, 191): qkv = bf16(x' to_qkv^T) with
 * x' = bf16(DyT(x, pre_norm)) when pre_norm is given (`_block`'s `_dyt(x, pre_norm).astype(compute)`), x otherwise.
 *   x         bf16 [batch, rows, d_model] (row stride ldx elements); 64 <= d_model <= 512, a multiple of 64.
 *   pre_norm  fp32 [1 + 2 d_model] {alpha, gamma[d_model], beta[d_model]} or NULL.
 *   w         bf16 [5 * num_heads * 64, d_model] (row stride ldw): the checkpoint's `to_qkv` weight [out, in].
 *   out       bf16 [batch, rows, ldo], columns [q | k | v | q_diff | k_diff] as hb_band_diff_attn reads them.
 *   prepare   0: out is the projection. 1: the q, k, q_diff, k_diff columns are DyT'd (q_norm / k_norm, fp32
 *             [129]) and rotated (RoPE, inv_freq fp32 [half], angles fp32(pos0 + row) * inv_freq) in fp32 and
 *             rounded to bf16 once, with the fused band kernel's arithmetic: hb_band_diff_attn_prepared on this
 *             output equals hb_band_diff_attn on the prepare = 0 output bit for bit (window <= 128).
 * No reference counterpart as one entry point: the reference runs the projection as an XLA matmul and the
 * DyT / RoPE inside its Pallas kernel. */
int hb_band_qkv_project(const void* x, int64_t ldx, const float* pre_norm, const void* w, int64_t ldw,
                        const float* q_norm, const float* k_norm, const float* inv_freq, int half, void* out,
                        int64_t ldo, int batch, int rows, int64_t pos0, int d_model, int num_heads, int head_dim,
                        int prepare, cudaStream_t stream);

/* hb_band_diff_attn on qkv that hb_band_qkv_project prepared (prepare = 1; halo rows from neighbouring shards
 * prepared at their own positions): the fused kernel without its preparation stage. Arguments as for
 * hb_band_diff_attn; window <= 128. */
int hb_band_diff_attn_prepared(const void* qkv, int64_t qkv_row_stride, const float* lam, void* out,
                               int64_t out_row_stride, int batch, int rows, int q_begin, int q_count, int num_heads,
                               int head_dim, int window, int pair_begin, int pair_count, cudaStream_t stream);

/* ---- W8A8 int8 GEMM (DiT MLP) ------------------------------------------------------------------------ */
/* Per-row symmetric int8 quantisation of a bf16 matrix x [rows, K] (leading dim ldx elements):
 * scale[r] = absmax / 127 (1 for an all-zero row), q = clamp(rint(x / scale), -127, 127).
 * Used per token on activations and per output channel on weights [N, K]. No reference counterpart:
 * the reference's MLP is a bf16 `_linear` (dit.py:33-36, 218-221); the scheme is the benchmark's. */
int hb_quant_rows_int8(const void* x, int64_t ldx, int rows, int K, void* q, int64_t ldq, float* scale,
                       cudaStream_t stream);

/* y[m, n] = bf16(((float)acc[m, n] * sx[m]) * sw[n] + bias[n]), acc = sum_k qx[m, k] * qw[n, k] in int32.
 * Replaces `dit._linear(x, W, b)` (dit.py:33-36) at its `_feed_forward` call sites (dit.py:220-221).
 *   qx  int8 [M, K] (ld ldqx bytes, multiple of 16), sx fp32 [M]; qw int8 [N, K], sw fp32 [N];
 *   bias bf16 [N] or NULL; out bf16 [M, N] (ld ldo elements);
 *   acc_out  optional int32 [M, N] copy of the accumulators (ld ldacc), NULL to skip.
 * N must be a multiple of 32, K a multiple of 16. */
int hb_w8a8_gemm(const void* qx, int64_t ldqx, const float* sx, const void* qw, int64_t ldqw, const float* sw,
                 const void* bias, void* out, int64_t ldo, int32_t* acc_out, int64_t ldacc, int M, int N, int K,
                 cudaStream_t stream);

/* The MLP's first GEMM with its GLU in the epilogue (`dit._feed_forward`, dit.py:218-221:
 * z = value * silu(gate) of `_linear(x, glu_proj)`), writing only z bf16 [M, F] (ld ldz elements).
 *   qw   int8 [2F, K] weight rows interleaved in blocks of 128: rows [256 t, 256 t + 128) are value rows
 *        [128 t, 128 t + 128) of the checkpoint's `glu_proj` weight [2F, K] (value = its first F rows) and rows
 *        [256 t + 128, 256 t + 256) the matching gate rows [F + 128 t, F + 128 t + 128); sw fp32 [2F] and bias
 *        bf16 [2F] (or NULL) in the same order. `hummingbird_b200.w8a8.glu_interleave` builds the order.
 * z equals, bit for bit, hb_glu_rows (bf16 mode) applied to hb_w8a8_gemm's output with the plain row order:
 * value and gate rounded to bf16 as that GEMM stores them, silu rounded to bf16, z rounded to bf16. Quantise z
 * with hb_quant_rows_int8 for the MLP's second GEMM (bit-identical to hb_glu_rows' int8 mode).
 * F a multiple of 128, K a multiple of 16. No reference counterpart as an entry point (the reference's MLP is a
 * bf16 matmul, then separate XLA ops for the GLU). */
int hb_w8a8_gemm_glu(const void* qx, int64_t ldqx, const float* sx, const void* qw, int64_t ldqw, const float* sw,
                     const void* bias, void* z, int64_t ldz, int M, int F, int K, cudaStream_t stream);

/* ---- DiT block glue (the elementwise steps around the kernels above) ------------------------------------ */
/* No reference counterpart as entry points: the reference runs these steps as separate XLA ops inside
 * `dit._block` (dit.py:224-250); here each fuses several of them into one pass over the activation rows.
 * All tensors bf16, row-major; rows = B * rows_per_batch; batch b = row / rows_per_batch.
 *
 * In place on h [rows, d] (ld ldh), then an optional normalised copy x [rows, d] (ld ldx):
 *   h <- h + y * sigmoid(1 - gate[b])        if y (gate [B, d] with row stride ldc, NULL = no gate)
 *   h <- h + local                           on rows with (row % rows_per_batch) >= local_row0, if local
 *   x <- RMSNorm(h, eps) * weight            if x (weight [d])
 *   x <- x * (1 + scale[b]) + shift[b]       if scale and shift ([B, d], row stride ldc)
 * The adaLN pre-norms (dit.py:234-235, 247-248), the gated residuals (dit.py:237, 250), the cross-attention
 * residual with `to_local_embed` (dit.py:240, 244) and the norm before it (dit.py:239).
 * d a multiple of 256, <= 2048. */
int hb_dit_residual_norm(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate, const void* scale,
                         const void* shift, int64_t ldc, const void* local, int local_row0, const void* weight,
                         void* x, int64_t ldx, int rows, int rows_per_batch, int d, float eps, cudaStream_t stream);

/* hb_dit_residual_norm with the normalised, modulated x written quantised per row instead of as bf16: q int8
 * [rows, d] (ld ldq bytes, 8-byte aligned rows) and qscale fp32 [rows], by hb_quant_rows_int8's rules applied to
 * the bf16 x (bit-identical to running that quantiser on hb_dit_residual_norm's x). Feeds a W8A8 GEMM (the MLP,
 * dit.py:246-249) without a separate quantiser pass. Same arguments otherwise (weight required). */
int hb_dit_residual_norm_int8(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate, const void* scale,
                              const void* shift, int64_t ldc, const void* local, int local_row0, const void* weight,
                              void* q, int64_t ldq, float* qscale, int rows, int rows_per_batch, int d, float eps,
                              cudaStream_t stream);

/* GLU of `dit._feed_forward` (dit.py:218-221): per row of glu [rows, 2F] (value = columns [0, F), gate =
 * [F, 2F)), z = value * silu(gate) rounded to bf16; written to z [rows, F] (ld ldz) OR quantised per row
 * with hb_quant_rows_int8's rules into q int8 [rows, F] (ld ldq bytes) and scale fp32 [rows] (exactly one
 * of z, q). F a multiple of 8, <= 8192. */
int hb_glu_rows(const void* glu, int64_t ldg, int rows, int F, void* z, int64_t ldz, void* q, int64_t ldq,
                float* scale, cudaStream_t stream);

/* `dit._rms` over every 64-dim head of x [rows, heads * 64] (ld ldx) with weight [64] (bf16), to out
 * (ld ldo; may equal x): the q / q_diff norm that `_attend` applies to the cross-attention queries
 * (dit.py:150-176, 203-215). */
int hb_head_rms_norm(const void* x, int64_t ldx, int rows, int heads, const void* weight, float eps, void* out,
                     int64_t ldo, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HB_B200_H_ */
