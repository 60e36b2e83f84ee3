/*
 * techjam_b200.h - C ABI of the B200 (sm_100a) encoder-layer library
 * (libtechjam_b200.so).
 *
 * The library replaces the device work of
 * `UserOptimizedTransformer.forward(x, valid_token_mask)` in v16_1_clean.py
 * (v16_1_clean.py:728-735 -> _forward_impl :599-628).  Every entry point takes
 * plain device pointers, sizes and a CUDA stream (as `void*`, NULL = legacy
 * default stream), enqueues its kernels on that stream and returns without
 * synchronising.  No entry point allocates device memory: the caller passes
 * every buffer, including the workspace sized by tj_encoder_workspace_bytes().
 *
 * Return codes: TJ_OK (0) on success, otherwise one of the TJ_ERR_* values;
 * tj_last_error() then describes the failure (thread-local).  No C++
 * exception crosses this boundary.
 *
 * Device-side failures (a pipeline wait inside a kernel that exceeded its time
 * limit, code 1; a row table in device memory that points outside its
 * buffer, code 2) are recorded in a per-device status word instead of
 * hanging, trapping or faulting the GPU; tj_device_status() reads and clears
 * it.  With
 * tj_set_sync_check(1) every entry point synchronises its stream and reports a
 * recorded device error as TJ_ERR_DEVICE (debugging and tests only).
 *
 * Tensor layouts (row-major, innermost last):
 *   x, out          float32 [B, S, D]
 *   mask            uint8/bool [B, S], nonzero = valid token (may be NULL)
 *   weights         float16 [N, K] (nn.Linear layout), biases float32 [N]
 *   LayerNorm       gamma/beta float32 [D], eps as given (nn.LayerNorm: 1e-5)
 *   qkv (head-major) float16 [3][H][rows][P] with P = 64, 128 or 256, the
 *                   smallest that holds the head dim (1..256); each head's
 *                   row is its head_dim values then zeros up to P
 *   ctx             float16 [rows][D]
 *   "compact rows"  the valid tokens of the batch packed densely in
 *                   (sample, position) order, as the token plan defines.
 */
#ifndef TECHJAM_B200_H_
#define TECHJAM_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TJ_API __attribute__((visibility("default")))
#else
#define TJ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TJ_ABI_VERSION 1

#define TJ_OK 0
#define TJ_ERR_INVALID_ARGUMENT 1
#define TJ_ERR_UNSUPPORTED 2
#define TJ_ERR_CUDA 3
#define TJ_ERR_DEVICE 4
#define TJ_ERR_WORKSPACE 5

/* ---- library ---------------------------------------------------------- */

/* ABI version (TJ_ABI_VERSION).  No reference counterpart. */
TJ_API int tj_abi_version(void);

/* Message for the last failed call on this thread ("" if none). */
TJ_API const char* tj_last_error(void);

/* Copies the message into buf (always NUL-terminated); returns its length. */
TJ_API int tj_get_last_error(char* buf, size_t len);

/* Enables (1) or disables (0) a stream synchronise + device-status check at
 * the end of every entry point.  Returns the previous setting. */
TJ_API int tj_set_sync_check(int enabled);

/* Synchronises `stream`, then copies the current device's status word into
 * out4 ([0] code, [1] wait site, [2..3] block index; all zero when healthy)
 * and clears it.  Returns TJ_OK, or TJ_ERR_DEVICE if a device error was
 * recorded, or TJ_ERR_CUDA if the synchronise itself failed. */
TJ_API int tj_device_status(int* out4, void* stream);

/* ---- debugging and tests (no reference counterpart) ---------------------
 * Device-side failure detection is tested without a GPU fault: a test
 * shortens the wait limit and withholds one barrier arrive, the wait runs
 * out, the kernel records the site and returns, and tj_device_status reports
 * it.  Both settings are per device (the current one) and stay until reset. */

/* Time limit of every pipeline wait inside the kernels, in nanoseconds
 * (0 restores the default, 2 s). */
TJ_API int tj_debug_set_wait_limit_ns(uint64_t ns);

#define TJ_WITHHOLD_NONE 0
#define TJ_WITHHOLD_ATTN_P_READY 1 /* attention: the first "P ready" arrive of each CTA (wait site 213) */

/* Makes every following kernel launch on the current device withhold the
 * selected barrier arrive (TJ_WITHHOLD_NONE to stop).  Tests only. */
TJ_API int tj_debug_withhold_arrive(int which);

/* ---- token plan --------------------------------------------------------- */

/* Number of int32 entries tj_token_plan writes for a [B, S] batch. */
TJ_API int64_t tj_token_plan_ints(int batch, int seq_len);

/* Builds the valid-token plan from `mask` (NULL = every token valid):
 *   plan[0]                      nv, number of valid tokens
 *   plan[1 .. B+1]               cu, compact offset of each sample (cu[B] = nv)
 *   plan[B+2 .. 2B+1]            per-sample valid counts
 *   plan[2B+2 .. 2B+2+BS)        compact row -> original row b*S+s
 *   plan[2B+2+BS .. 2B+2+2BS)    original row -> compact row, or -1 if padded
 *   plan[2B+2+2BS .. 3B+2+2BS)   samples by decreasing valid count (stable;
 *                                identity when batch > 256)
 * Replaces the mask plumbing of v16_1_clean.py:607-611 (key mask [B,1,1,S] and
 * query mask [B,S,1]); padded tokens then never enter a GEMM or attention. */
TJ_API int tj_token_plan(const uint8_t* mask, int batch, int seq_len, int32_t* plan, void* stream);

/* ---- single kernels ------------------------------------------------------ */

/* y16[r] = fp16(LayerNorm(x[row_map ? row_map[r] : r])) for r < min(rows,
 * *row_count) (row_count may be NULL).  Replaces layer.norm1(x) / norm2(x)
 * followed by .to(float16): v16_1_clean.py:615-616 + :476, and :527. */
TJ_API int tj_ln_cast_f16(const float* x, const int32_t* row_map, const int32_t* row_count, int rows,
                   int d_model, const float* gamma, const float* beta, float eps, void* y16,
                   void* stream);

/* out[m] = LayerNorm(x[inv_map[m]]) for inv_map[m] >= 0, else exact zeros, for
 * m < rows (inv_map NULL = identity).  Replaces final_norm + masked_fill:
 * v16_1_clean.py:625-627. */
TJ_API int tj_ln_final_mask(const float* x, const int32_t* inv_map, int rows, int d_model,
                     const float* gamma, const float* beta, float eps, float* out, void* stream);

/* Residual add fused into the LayerNorm that follows it.  For r < min(rows,
 * *row_count):
 *   s = x[row_map ? row_map[r] : r] + float(add16[r])          (fp32)
 *   sum_out[r] = s   (if sum_out is not NULL)
 *   y16[r] = fp16(LayerNorm(s))
 * Replaces `x = x + attention_output` / `x = x + ffn_output` (the branch output
 * being the fp16 F.linear result .float()) and the norm2 / next layer's norm1
 * that reads it: v16_1_clean.py:620-621 + :527, :615-616. */
TJ_API int tj_add_ln_cast_f16(const float* x, const int32_t* row_map, const void* add16,
                       const int32_t* row_count, int rows, int d_model, const float* gamma,
                       const float* beta, float eps, float* sum_out, void* y16, void* stream);

/* out[m] = LayerNorm(x[c] + float(add16[c])) with c = inv_map[m] >= 0, else
 * exact zeros, for m < rows.  Replaces the last layer's `x = x + ffn_output`
 * with final_norm + masked_fill: v16_1_clean.py:621-627. */
TJ_API int tj_add_ln_final_mask(const float* x, const void* add16, const int32_t* inv_map, int rows,
                         int d_model, const float* gamma, const float* beta, float eps, float* out,
                         void* stream);

/* out[m] = LayerNorm((x[r] + float(attn16[c])) + float(ffn16[c])) with
 * c = inv_map[m] >= 0 and r = m if x_at_original else c; exact zeros where
 * inv_map[m] < 0.  The last layer's two residual adds (:620-621) fused with
 * final_norm + masked_fill (:625-627), so x + attention is never stored; with
 * one layer x is the encoder input itself, read at the original row. */
TJ_API int tj_add2_ln_final_mask(const float* x, int x_at_original, const void* attn16,
                          const void* ffn16, const int32_t* inv_map, int rows, int d_model,
                          const float* gamma, const float* beta, float eps, float* out,
                          void* stream);

/* qkv16 (head-major [3][H][rows_max][P], see above) = fp16(a16 @ w_qkv^T + b_qkv) for the
 * first min(rows_max, *row_count) rows; w_qkv is the packed [3D, D] q/k/v
 * weight.  Replaces the packed F.linear + reshape/permute/unbind of
 * v16_1_clean.py:474-489. */
TJ_API int tj_gemm_qkv_headmajor(const void* a16, const void* w_qkv16, const float* b_qkv,
                          const int32_t* row_count, int rows_max, int d_model, int num_heads,
                          void* qkv16, void* stream);

/* out[r] = a16[r] @ w^T + bias + resid[resid_map ? resid_map[r] : r]  (fp32)
 * Replaces the fp16 out-projection + .float() + residual add of
 * v16_1_clean.py:519-523,620 and the FFN-out F.linear + residual of
 * v16_1_clean.py:533-537,621. */
TJ_API int tj_gemm_bias_residual_f32(const void* a16, const void* w16, const float* bias,
                              const float* resid, const int32_t* resid_map,
                              const int32_t* row_count, int rows_max, int n, int k, float* out,
                              void* stream);

/* out16[r] = fp16(a16[r] @ w^T + bias).  Replaces the fp16 F.linear of the
 * output projection (v16_1_clean.py:519-523) and of FFN-out (:533-537); the
 * .float() + residual add is tj_add_ln_cast_f16 / tj_add_ln_final_mask. */
TJ_API int tj_gemm_bias_f16(const void* a16, const void* w16, const float* bias,
                     const int32_t* row_count, int rows_max, int n, int k, void* out16,
                     void* stream);

/* out16[r] = fp16(gelu_erf(a16[r] @ w^T + bias)), GELU evaluated on the fp32
 * accumulator.  Replaces torch.ops.techjam.v16_1_clean_fused_ffn_gelu_no_preround
 * (v16_1_clean.py:304-365, Triton kernel :221-301). */
TJ_API int tj_gemm_bias_gelu_f16(const void* a16, const void* w16, const float* bias,
                          const int32_t* row_count, int rows_max, int n, int k, void* out16,
                          void* stream);

/* Masked multi-head attention over compact rows, head_dim 1..256.
 *   q16       [H][q_rows][P] (head_dim values then zeros up to P = 64, 128
 *             or 256, the smallest that holds head_dim)
 *   k16, v16  addressed as [G][H][kv_rows][P] with element strides
 *             kv_stride_h (between heads) and kv_stride_g (between segments)
 *   q_cu      [batch+1]: queries of sample b are q rows [q_cu[b], q_cu[b+1])
 *   kv_off, kv_len [batch*G]: keys of sample b are, for g = 0..G-1 in order,
 *             rows [kv_off[b*G+g], +kv_len[b*G+g]) of segment g
 *   ctx16     [q_rows][H*head_dim]: softmax(q k^T * scale) v per head
 *   causal    mask keys whose position (order within the sample's keys) is
 *             after the query position q_pos0[b] + (row - q_cu[b]);
 *             q_pos0 may be NULL (= 0) when G == 1.
 * Replaces F.scaled_dot_product_attention with the [B,1,1,S] key mask
 * (v16_1_clean.py:505-514) and the causal branch (:491-504). */
TJ_API int tj_flash_attn_fwd(const void* q16, const void* k16, const void* v16, int num_heads,
                      int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                      int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                      const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                      float scale, int causal, const int32_t* q_pos0, void* ctx16, void* stream);

/* tj_flash_attn_fwd with the context row stride given: ctx16 row r, head h
 * starts at element r*ld_ctx + h*head_dim (ld_ctx >= num_heads*head_dim, a
 * multiple of 8 when head_dim is; 0 = num_heads*head_dim).  Lets a caller run
 * attention for a group of heads straight into its columns of a wider
 * context, e.g. per head group as each group's K/V arrive (the context-
 * parallel path overlaps the all-gather with attention this way). */
TJ_API int tj_flash_attn_fwd_strided(const void* q16, const void* k16, const void* v16, int num_heads,
                              int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                              int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                              const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                              float scale, int causal, const int32_t* q_pos0, void* ctx16,
                              int64_t ld_ctx, void* stream);

/* tj_flash_attn_fwd_strided over part of each sample's keys, for attention
 * split into two launches (context parallelism: a rank's own keys while the
 * other ranks' keys are still arriving, then those).  part_mode:
 *   1  writes the partial result of these keys instead of ctx16 (which may be
 *      NULL): part_o [q_rows][num_heads*head_dim] fp32, the normalised context
 *      of these keys, and part_lse [q_rows][num_heads], log2 of their softmax
 *      denominator in base-2 units (log2 of the sum of 2^(s*scale*log2 e) over
 *      the keys; -inf for a row without keys);
 *   2  merges these keys' result with that partial and writes ctx16, equal to
 *      attention over both key sets in one launch up to rounding;
 *   0  plain tj_flash_attn_fwd_strided.
 * part_o must be 16-byte aligned.  A query row's two launches must use the
 * same q rows, scale and head layout.  Replaces, with the key set split, the
 * SDPA call of v16_1_clean.py:505-514. */
TJ_API int tj_flash_attn_fwd_partial(const void* q16, const void* k16, const void* v16, int num_heads,
                              int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                              int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                              const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                              float scale, int causal, const int32_t* q_pos0, void* ctx16,
                              int64_t ld_ctx, float* part_o, float* part_lse, int part_mode,
                              void* stream);

/* ---- whole encoder ----------------------------------------------------- */

typedef struct tj_encoder_desc {
  int batch, seq_len, d_model, num_heads, ffn_dim, num_layers, causal;
  float ln_eps;
} tj_encoder_desc;

/* fp16 weights are [N, K] row-major with rows padded to K8 = K rounded up
 * to a multiple of 8 columns (K8 = K when K is a multiple of 8); the padding
 * columns are never read. */
typedef struct tj_layer_weights {
  const float* ln1_gamma;   /* norm1.weight [D] */
  const float* ln1_beta;    /* norm1.bias [D] */
  const void* w_qkv16;      /* cat(q,k,v)_proj.weight as fp16 [3D, D8] */
  const float* b_qkv;       /* cat(q,k,v)_proj.bias [3D] */
  const void* w_out16;      /* attention.out_proj.weight fp16 [D, D8] */
  const float* b_out;       /* [D] */
  const float* ln2_gamma;   /* norm2.weight */
  const float* ln2_beta;
  const void* w_ffn_in16;   /* ffn_in.weight fp16 [F, D8] */
  const float* b_ffn_in;    /* [F] */
  const void* w_ffn_out16;  /* ffn_out.weight fp16 [D, F8] */
  const float* b_ffn_out;   /* [D] */
} tj_layer_weights;

/* Workspace bytes tj_encoder_forward needs for this shape (0 on bad shape). */
TJ_API int64_t tj_encoder_workspace_bytes(const tj_encoder_desc* desc);

/* out = encoder(x, mask): num_layers blocks of
 *   x = x + out_proj(attn(LN1(x))); x = x + ffn_out(gelu(ffn_in(LN2(x))))
 * then final LayerNorm, with padded rows exactly zero.  Same arithmetic
 * contract as UserOptimizedTransformer._forward_impl (v16_1_clean.py:599-628):
 * fp32 LayerNorm/residual/output, fp16 GEMM operands, fp32 accumulation,
 * erf-GELU from the fp32 accumulator.  x and out may not alias. */
TJ_API int tj_encoder_forward(const tj_encoder_desc* desc, const tj_layer_weights* layers,
                       const float* final_gamma, const float* final_beta, const float* x,
                       const uint8_t* mask, float* out, void* workspace, int64_t workspace_bytes,
                       void* stream);

/* ---- peer exchange (the batch-sharded output gather) --------------------
 *
 * The reference runs on one GPU and has no multi-GPU code; its single-GPU
 * batch split (balanced sample ranges, candidates/v19/parallel_batch_common.py:31-51)
 * is what these entry points scale out.  A batch split over the GPUs of one
 * node ends with the output gather: each rank pushes the valid rows of its
 * finished samples into every rank's [B, S, D] output over NVLink
 * (tj_push_segments), while its next micro-batch computes.  The library does not
 * allocate: the caller exports its own buffers and maps the peers'. */

#define TJ_IPC_HANDLE_BYTES 64

/* Exports the device allocation that contains `ptr` for the other processes
 * of this node: handle_out receives TJ_IPC_HANDLE_BYTES bytes and offset_out
 * the byte offset of ptr inside that allocation (the caller adds it to the
 * base tj_ipc_open returns in the other process).  The allocation must come
 * from cudaMalloc (e.g. torch's default caching allocator). */
TJ_API int tj_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);

/* Maps a peer's exported allocation into this process, with peer access over
 * NVLink, and returns its base address; undo with tj_ipc_close. */
TJ_API int tj_ipc_open(const void* handle, void** base_out);

/* Unmaps an allocation mapped by tj_ipc_open (NULL is a no-op). */
TJ_API int tj_ipc_close(void* base);

typedef struct tj_copy_segment {
  void* dst;        /* device address, may be a peer mapping from tj_ipc_open */
  const void* src;  /* device address; NULL = fill dst with zero bytes */
  int64_t bytes;
} tj_copy_segment;

/* Enqueues, in order on `stream`, one asynchronous device-to-device copy (or
 * zero fill, src == NULL) per segment.  Copies to a peer mapping run on the
 * copy engines over NVLink; no kernel is launched. */
TJ_API int tj_copy_segments(const tj_copy_segment* segs, int n, void* stream);

#define TJ_PUSH_MAX_DST 8
#define TJ_PUSH_MAX_SEGS 64

typedef struct tj_push_segment {
  int64_t dst_offset;  /* byte offset inside every destination buffer */
  const void* src;     /* device address of the bytes to send */
  int64_t bytes;
} tj_push_segment;

/* One kernel on `stream` that copies every segment to dst_offset of each of
 * the num_dst destination buffers (this GPU's own or peers' mappings from
 * tj_ipc_open): one 16-byte load per unit, one store per destination, the
 * stores fenced at system scope before the kernel ends.  Sources, offsets and
 * sizes must be 16-byte aligned; `blocks` is the total CTA count to spread
 * over the segments (0 = 4 per segment). */
TJ_API int tj_push_segments(void* const* dst_bases, int num_dst, const tj_push_segment* segs, int num_segs,
                            int blocks, void* stream);

/* Enables (1) or disables (0, the default) the fused path of
 * tj_encoder_forward for small models: sequences of at most 128 tokens,
 * d_model and ffn_dim at most 128, at most 8 layers, where one CTA runs every
 * layer of one sample (the reference's official 128-token shapes are this
 * size).  Results agree with the layer-by-layer path within fp16 rounding
 * (different accumulation order).  Returns the previous setting; process-wide.
 * No reference counterpart (the reference fuses these with torch.compile). */
TJ_API int tj_set_small_encoder(int enabled);

/* ---- encoder without a caller workspace --------------------------------- */

/* Size of the library's static device workspace used by
 * tj_encoder_forward_noalloc (64 MiB, held on every GPU that loads the
 * library until the process exits). */
#define TJ_NOALLOC_WORKSPACE_BYTES (64ull << 20)

/* Same computation and arguments as tj_encoder_forward, minus the workspace:
 * scratch space comes from a fixed library-owned device array, so this call
 * allocates no device memory.  No counterpart in the reference; it exists for
 * callers that cannot allocate device memory where they run the encoder (a
 * host binding the library through a thin FFI without a device allocator,
 * serving code whose device memory is planned up front, or code that must
 * not let cudaMalloc/cudaFree synchronise the device).
 *   - Shapes whose tj_encoder_workspace_bytes() exceeds
 *     TJ_NOALLOC_WORKSPACE_BYTES are rejected with TJ_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is cached per device and CUDA
 *     context: after a device reset, or from another context on the device,
 *     the next call looks it up again (make that call outside capture too).
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams or threads) race.  Nothing in it needs to start at zero. */
TJ_API int tj_encoder_forward_noalloc(const tj_encoder_desc* desc, const tj_layer_weights* layers,
                                      const float* final_gamma, const float* final_beta,
                                      const float* x, const uint8_t* mask, float* out,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TECHJAM_B200_H_ */
