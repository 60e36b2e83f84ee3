// C-ABI entry points of libtechjam_b200.so and the whole-encoder executor.
//
// The library is built as one translation unit (this file includes the kernel
// files) so that every kernel shares the single per-device status word.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "plan_layernorm.cu"
#include "gemm_tcgen05.cu"
#include "attention_tcgen05.cu"
#include "small_encoder.cu"

namespace tj {

static_assert(kWithholdAttnPFull == TJ_WITHHOLD_ATTN_P_READY, "withhold switch numbering");

static thread_local std::string g_last_error;
static std::atomic<int> g_sync_check{0};

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ensure_device_props(int* num_sms) {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(TJ_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10 || minor != 0)
      return set_error(TJ_ERR_UNSUPPORTED,
                       "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                       major, minor);
    cached[dev] = sms;
  }
  *num_sms = cached[dev];
  return TJ_OK;
}

static int finish(int rc, cudaStream_t stream) {
  if (rc != TJ_OK || g_sync_check.load(std::memory_order_relaxed) == 0) return rc;
  int st[4];
  return tj_device_status(st, stream);
}

static int check_device() {
  int sms = 0;
  return ensure_device_props(&sms);
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct EncoderWorkspace {
  size_t plan, a16, qkv16, x1, x2, h16, y16, y16b, total;
};

static bool workspace_layout(const tj_encoder_desc* d, EncoderWorkspace* w) {
  if (!d || d->batch <= 0 || d->seq_len <= 0 || d->d_model <= 0 || d->num_heads <= 0 ||
      d->ffn_dim <= 0 || d->num_layers <= 0 || d->d_model % d->num_heads != 0)
    return false;
  const size_t rows = (size_t)d->batch * d->seq_len;
  // fp16 rows padded to a multiple of 8 columns (16-byte TMA rows).
  const size_t D = d->d_model, F = d->ffn_dim, D8 = align_up(D, 8), F8 = align_up(F, 8);
  size_t off = 0;
  w->plan = off;
  off = align_up(off + (size_t)plan_ints(d->batch, d->seq_len) * 4, 256);
  w->a16 = off;
  off = align_up(off + rows * D8 * 2, 256);
  w->qkv16 = off;  // head-major [3][H][rows][P], heads zero-padded to P = 64, 128 or 256
  off = align_up(off + 3 * rows * (size_t)d->num_heads * attn_head_pad(d->d_model / d->num_heads) * 2, 256);
  w->x1 = off;
  off = align_up(off + rows * D * 4, 256);
  w->x2 = off;
  off = align_up(off + rows * D * 4, 256);
  w->h16 = off;
  off = align_up(off + rows * F8 * 2, 256);
  w->y16 = off;  // fp16 output of the out-projection / FFN-out before its residual add
  off = align_up(off + rows * D8 * 2, 256);
  w->y16b = off;  // the last layer's FFN-out (its out-projection output stays in y16)
  off = align_up(off + rows * D8 * 2, 256);
  w->total = off;
  return true;
}

}  // namespace tj

using namespace tj;

extern "C" {

int tj_abi_version(void) { return TJ_ABI_VERSION; }

const char* tj_last_error(void) { return g_last_error.c_str(); }

int tj_get_last_error(char* buf, size_t len) {
  if (buf && len) {
    strncpy(buf, g_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return (int)g_last_error.size();
}

int tj_set_sync_check(int enabled) { return g_sync_check.exchange(enabled ? 1 : 0); }

int tj_device_status(int* out4, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "stream synchronize: %s", cudaGetErrorString(e));
  int host[4] = {0, 0, 0, 0};
  e = cudaMemcpyFromSymbol(host, g_status, sizeof(host));
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  if (out4) memcpy(out4, host, sizeof(host));
  if (host[0] != 0) {
    const int zero[4] = {0, 0, 0, 0};
    cudaMemcpyToSymbol(g_status, zero, sizeof(zero));
    return set_error(TJ_ERR_DEVICE, "device error %d recorded by a kernel (site %d, block %d,%d): %s", host[0],
                     host[1], host[2], host[3],
                     host[0] == kDevWaitTimeout   ? "a pipeline wait exceeded its time limit"
                     : host[0] == kDevBadArgument ? "a row table in device memory points outside its buffer"
                                                  : "unknown code");
  }
  return TJ_OK;
}

int tj_set_small_encoder(int enabled) { return set_small_encoder(enabled); }

int tj_debug_set_wait_limit_ns(uint64_t ns) {
  int rc = check_device();
  if (rc) return rc;
  const unsigned long long v = ns ? (unsigned long long)ns : kWaitLimitNs;
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v));
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "debug_set_wait_limit_ns: %s", cudaGetErrorString(e));
  return TJ_OK;
}

int tj_debug_withhold_arrive(int which) {
  int rc = check_device();
  if (rc) return rc;
  if (which != 0 && which != kWithholdAttnPFull)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "debug_withhold_arrive: unknown switch %d", which);
  cudaError_t e = cudaMemcpyToSymbol(g_debug_withhold, &which, sizeof(which));
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "debug_withhold_arrive: %s", cudaGetErrorString(e));
  return TJ_OK;
}

int64_t tj_token_plan_ints(int batch, int seq_len) {
  if (batch <= 0 || seq_len <= 0) return 0;
  return plan_ints(batch, seq_len);
}

int tj_token_plan(const uint8_t* mask, int batch, int seq_len, int32_t* plan, void* stream) {
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_token_plan(mask, batch, seq_len, plan, s), s);
}

int tj_ln_cast_f16(const float* x, const int32_t* row_map, const int32_t* row_count, int rows,
                   int d_model, const float* gamma, const float* beta, float eps, void* y16,
                   void* stream) {
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_ln_cast_f16(x, row_map, row_count, rows, d_model, gamma, beta, eps, y16, s), s);
}

int tj_ln_final_mask(const float* x, const int32_t* inv_map, int rows, int d_model,
                     const float* gamma, const float* beta, float eps, float* out, void* stream) {
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_ln_final(x, inv_map, rows, d_model, gamma, beta, eps, out, s), s);
}

int tj_add_ln_cast_f16(const float* x, const int32_t* row_map, const void* add16,
                       const int32_t* row_count, int rows, int d_model, const float* gamma,
                       const float* beta, float eps, float* sum_out, void* y16, void* stream) {
  int rc = check_device();
  if (rc) return rc;
  if (!add16) return set_error(TJ_ERR_INVALID_ARGUMENT, "add_ln_cast_f16: null addend");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_ln_cast_f16(x, row_map, row_count, rows, d_model, gamma, beta, eps, y16, s,
                                   add16, sum_out),
                s);
}

int tj_add2_ln_final_mask(const float* x, int x_at_original, const void* attn16,
                          const void* ffn16, const int32_t* inv_map, int rows, int d_model,
                          const float* gamma, const float* beta, float eps, float* out,
                          void* stream) {
  int rc = check_device();
  if (rc) return rc;
  if (!attn16 || !ffn16) return set_error(TJ_ERR_INVALID_ARGUMENT, "add2_ln_final_mask: null addend");
  if (x_at_original && !inv_map)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "add2_ln_final_mask: x_at_original needs inv_map");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_ln_final(x, inv_map, rows, d_model, gamma, beta, eps, out, s, attn16, ffn16,
                                x_at_original != 0),
                s);
}

int tj_add_ln_final_mask(const float* x, const void* add16, const int32_t* inv_map, int rows,
                         int d_model, const float* gamma, const float* beta, float eps, float* out,
                         void* stream) {
  int rc = check_device();
  if (rc) return rc;
  if (!add16) return set_error(TJ_ERR_INVALID_ARGUMENT, "add_ln_final_mask: null addend");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_ln_final(x, inv_map, rows, d_model, gamma, beta, eps, out, s, add16), s);
}

int tj_gemm_qkv_headmajor(const void* a16, const void* w_qkv16, const float* b_qkv,
                          const int32_t* row_count, int rows_max, int d_model, int num_heads,
                          void* qkv16, void* stream) {
  int rc = check_device();
  if (rc) return rc;
  if (num_heads <= 0 || d_model <= 0 || d_model % num_heads != 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm_qkv_headmajor: d_model %d not divisible by heads %d", d_model, num_heads);
  GemmArgs a{};
  a.a16 = a16;
  a.w16 = w_qkv16;
  a.bias = b_qkv;
  a.row_count = row_count;
  a.rows_max = rows_max;
  a.N = 3 * d_model;
  a.K = d_model;
  a.out = qkv16;
  a.heads = num_heads;
  a.head_dim = d_model / num_heads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_gemm(kEpiQkvHeadMajor, a, s), s);
}

int tj_gemm_bias_residual_f32(const void* a16, const void* w16, const float* bias,
                              const float* resid, const int32_t* resid_map,
                              const int32_t* row_count, int rows_max, int n, int k, float* out,
                              void* stream) {
  int rc = check_device();
  if (rc) return rc;
  GemmArgs a{};
  a.a16 = a16;
  a.w16 = w16;
  a.bias = bias;
  a.row_count = row_count;
  a.rows_max = rows_max;
  a.N = n;
  a.K = k;
  a.out = out;
  a.ld_out = n;
  a.resid = resid;
  a.resid_map = resid_map;
  a.ld_resid = n;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_gemm(kEpiResidualF32, a, s), s);
}

int tj_gemm_bias_f16(const void* a16, const void* w16, const float* bias,
                     const int32_t* row_count, int rows_max, int n, int k, void* out16,
                     void* stream) {
  int rc = check_device();
  if (rc) return rc;
  GemmArgs a{};
  a.a16 = a16;
  a.w16 = w16;
  a.bias = bias;
  a.row_count = row_count;
  a.rows_max = rows_max;
  a.N = n;
  a.K = k;
  a.out = out16;
  a.ld_out = n;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_gemm(kEpiBiasF16, a, s), s);
}

int tj_gemm_bias_gelu_f16(const void* a16, const void* w16, const float* bias,
                          const int32_t* row_count, int rows_max, int n, int k, void* out16,
                          void* stream) {
  int rc = check_device();
  if (rc) return rc;
  GemmArgs a{};
  a.a16 = a16;
  a.w16 = w16;
  a.bias = bias;
  a.row_count = row_count;
  a.rows_max = rows_max;
  a.N = n;
  a.K = k;
  a.out = out16;
  a.ld_out = n;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_gemm(kEpiGeluF16, a, s), s);
}

int tj_flash_attn_fwd_partial(const void* q16, const void* k16, const void* v16, int num_heads,
                              int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                              int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                              const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                              float scale, int causal, const int32_t* q_pos0, void* ctx16,
                              int64_t ld_ctx, float* part_o, float* part_lse, int part_mode,
                              void* stream) {
  int rc = check_device();
  if (rc) return rc;
  AttnArgs a{};
  a.q = q16;
  a.k = k16;
  a.v = v16;
  a.H = num_heads;
  a.head_dim = head_dim;
  a.q_rows = q_rows;
  a.kv_rows = kv_rows;
  a.kv_stride_h = kv_stride_h;
  a.kv_stride_g = kv_stride_g;
  a.G = num_segments;
  a.B = batch;
  a.max_q_per_sample = max_q_per_sample;
  a.q_cu = q_cu;
  a.kv_off = kv_off;
  a.kv_len = kv_len;
  a.kv_len_stride = num_segments;
  a.scale = scale;
  a.causal = causal;
  a.q_pos0 = q_pos0;
  a.ctx = ctx16;
  a.ld_ctx = ld_ctx;
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.part_mode = part_mode;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return finish(launch_attention(a, s), s);
}

int tj_flash_attn_fwd_strided(const void* q16, const void* k16, const void* v16, int num_heads,
                              int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                              int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                              const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                              float scale, int causal, const int32_t* q_pos0, void* ctx16,
                              int64_t ld_ctx, void* stream) {
  return tj_flash_attn_fwd_partial(q16, k16, v16, num_heads, head_dim, q_rows, kv_rows, kv_stride_h,
                                   kv_stride_g, num_segments, batch, max_q_per_sample, q_cu, kv_off,
                                   kv_len, scale, causal, q_pos0, ctx16, ld_ctx, nullptr, nullptr, 0,
                                   stream);
}

int tj_flash_attn_fwd(const void* q16, const void* k16, const void* v16, int num_heads,
                      int head_dim, int q_rows, int kv_rows, int64_t kv_stride_h,
                      int64_t kv_stride_g, int num_segments, int batch, int max_q_per_sample,
                      const int32_t* q_cu, const int32_t* kv_off, const int32_t* kv_len,
                      float scale, int causal, const int32_t* q_pos0, void* ctx16, void* stream) {
  return tj_flash_attn_fwd_strided(q16, k16, v16, num_heads, head_dim, q_rows, kv_rows, kv_stride_h,
                                   kv_stride_g, num_segments, batch, max_q_per_sample, q_cu, kv_off,
                                   kv_len, scale, causal, q_pos0, ctx16, 0, stream);
}

int64_t tj_encoder_workspace_bytes(const tj_encoder_desc* desc) {
  EncoderWorkspace w;
  if (!workspace_layout(desc, &w)) return 0;
  return (int64_t)w.total;
}

int tj_encoder_forward(const tj_encoder_desc* d, const tj_layer_weights* layers,
                       const float* final_gamma, const float* final_beta, const float* x,
                       const uint8_t* mask, float* out, void* workspace, int64_t workspace_bytes,
                       void* stream) {
  int rc = check_device();
  if (rc) return rc;
  EncoderWorkspace w;
  if (!workspace_layout(d, &w))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "encoder_forward: invalid descriptor");
  if (!layers || !final_gamma || !final_beta || !x || !out)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "encoder_forward: null pointer");
  if (workspace == nullptr || workspace_bytes < (int64_t)w.total)
    return set_error(TJ_ERR_WORKSPACE, "encoder_forward: workspace of %lld bytes, %lld needed",
                     (long long)workspace_bytes, (long long)w.total);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(TJ_ERR_WORKSPACE, "encoder_forward: workspace must be 256-byte aligned");
  if (x == out) return set_error(TJ_ERR_INVALID_ARGUMENT, "encoder_forward: x and out alias");
  const int D = d->d_model, H = d->num_heads, F = d->ffn_dim, B = d->batch, S = d->seq_len;
  const int dh = D / H;
  if (dh > 256)
    return set_error(TJ_ERR_UNSUPPORTED, "encoder_forward: head_dim %d (1..256 supported)", dh);
  if (D > (D % 4 == 0 ? 32768 : 8192))
    return set_error(TJ_ERR_UNSUPPORTED, "encoder_forward: d_model %d above %d", D, D % 4 == 0 ? 32768 : 8192);
  // fp16 activations and weights have rows padded to a multiple of 8 columns,
  // whole 16-byte units for the GEMMs' TMA loads (which stop at the true K).
  const int D8 = (D + 7) / 8 * 8, F8 = (F + 7) / 8 * 8;
  const int kPad = attn_head_pad(dh);  // head-major row length of the QKV buffer
  if ((int64_t)B * S > INT32_MAX / 4)
    return set_error(TJ_ERR_UNSUPPORTED, "encoder_forward: B*S too large");
  const int rows = B * S;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Small models (S <= 128, d_model and ffn_dim <= 128): one fused kernel,
  // one CTA per sample through every layer (small_encoder.cu).
  if (small_encoder_fits(d))
    return finish(launch_small_encoder(d, layers, final_gamma, final_beta, x, mask, out, s), s);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  PlanView plan{reinterpret_cast<int32_t*>(ws + w.plan), B, S};
  __half* a16 = reinterpret_cast<__half*>(ws + w.a16);
  __half* qkv16 = reinterpret_cast<__half*>(ws + w.qkv16);
  float* x1 = reinterpret_cast<float*>(ws + w.x1);
  float* x2 = reinterpret_cast<float*>(ws + w.x2);
  __half* h16 = reinterpret_cast<__half*>(ws + w.h16);
  __half* y16 = reinterpret_cast<__half*>(ws + w.y16);
  __half* y16b = reinterpret_cast<__half*>(ws + w.y16b);
  const int32_t* nv = plan.nv();

  rc = launch_token_plan(mask, B, S, plan.base, s);
  if (rc) return rc;
  // Residual stream (fp32, compact rows): layer 0 reads the input through the
  // plan's row map; afterwards x1 holds x after attention and x2 the input of
  // the next layer.  The out-projection and FFN-out leave their fp16 result in
  // y16 and the next LayerNorm kernel adds it to the stream.  In the last
  // layer the sum x + attention is not stored: the final LayerNorm adds both
  // fp16 branch outputs (y16, y16b) to the layer input itself, which saves
  // the fp32 write and read of x1.
  for (int l = 0; l < d->num_layers; ++l) {
    const tj_layer_weights& L = layers[l];
    const bool last = l + 1 == d->num_layers;
    const float* xin = (l == 0) ? x : x2;
    const int32_t* in_map = (l == 0) ? plan.orig() : nullptr;
    if (l == 0)
      rc = launch_ln_cast_f16(x, in_map, nv, rows, D, L.ln1_gamma, L.ln1_beta, d->ln_eps, a16, s, nullptr,
                              nullptr, D8, D8);
    else  // x2 = x1 + FFN-out of the previous layer
      rc = launch_ln_cast_f16(x1, nullptr, nv, rows, D, L.ln1_gamma, L.ln1_beta, d->ln_eps, a16, s,
                              y16, x2, D8, D8);
    if (rc) return rc;
    GemmArgs g{};
    g.a16 = a16;
    g.w16 = L.w_qkv16;
    g.bias = L.b_qkv;
    g.row_count = nv;
    g.rows_max = rows;
    g.N = 3 * D;
    g.K = D;
    g.lda = g.ldw = D8;
    g.out = qkv16;
    g.heads = H;
    g.head_dim = dh;
    rc = launch_gemm(kEpiQkvHeadMajor, g, s);
    if (rc) return rc;
    AttnArgs a{};
    a.q = qkv16;
    a.k = qkv16 + (size_t)H * rows * kPad;
    a.v = qkv16 + 2 * (size_t)H * rows * kPad;
    a.H = H;
    a.head_dim = dh;
    a.q_rows = rows;
    a.kv_rows = rows;
    a.kv_stride_h = (int64_t)rows * kPad;
    a.kv_stride_g = 3 * (int64_t)H * rows * kPad;
    a.G = 1;
    a.B = B;
    a.max_q_per_sample = S;
    a.q_cu = plan.cu();
    a.kv_off = plan.cu();
    a.kv_len = plan.n();
    a.kv_len_stride = 1;
    a.scale = 1.0f / sqrtf((float)dh);
    a.causal = d->causal;
    a.q_pos0 = nullptr;
    a.order = plan.order();
    a.ctx = a16;  // LN1 output is dead once the QKV GEMM has run
    a.ld_ctx = D8;
    rc = launch_attention(a, s);
    if (rc) return rc;
    GemmArgs o{};
    o.a16 = a16;
    o.w16 = L.w_out16;
    o.bias = L.b_out;
    o.row_count = nv;
    o.rows_max = rows;
    o.N = D;
    o.K = D;
    o.lda = o.ldw = D8;
    o.out = y16;
    o.ld_out = D8;
    rc = launch_gemm(kEpiBiasF16, o, s);
    if (rc) return rc;
    // x1 = x + attention output; a16 = LN2(x1)
    rc = launch_ln_cast_f16(xin, in_map, nv, rows, D, L.ln2_gamma, L.ln2_beta, d->ln_eps, a16, s, y16,
                            last ? nullptr : x1, D8, D8);
    if (rc) return rc;
    GemmArgs f1{};
    f1.a16 = a16;
    f1.w16 = L.w_ffn_in16;
    f1.bias = L.b_ffn_in;
    f1.row_count = nv;
    f1.rows_max = rows;
    f1.N = F;
    f1.K = D;
    f1.lda = f1.ldw = D8;
    f1.out = h16;
    f1.ld_out = F8;
    rc = launch_gemm(kEpiGeluF16, f1, s);
    if (rc) return rc;
    GemmArgs f2{};
    f2.a16 = h16;
    f2.w16 = L.w_ffn_out16;
    f2.bias = L.b_ffn_out;
    f2.row_count = nv;
    f2.rows_max = rows;
    f2.N = D;
    f2.K = F;
    f2.lda = f2.ldw = F8;
    f2.out = last ? y16b : y16;
    f2.ld_out = D8;
    rc = launch_gemm(kEpiBiasF16, f2, s);
    if (rc) return rc;
  }
  // out = final LN((x + attention output) + FFN-out) of the last layer,
  // scattered to the original rows; x is the input itself (one layer, read
  // at the output row) or the last layer's compact input x2.
  const bool one_layer = d->num_layers == 1;
  rc = launch_ln_final(one_layer ? x : x2, plan.inv(), rows, D, final_gamma, final_beta, d->ln_eps, out,
                       s, y16, y16b, one_layer, D8);
  return finish(rc, s);
}

}  // extern "C"

// Workspace-free variant of tj_encoder_forward (its own file: static device
// workspace and the per-device address lookup).
#include "noalloc.cu"
// Peer-memory plumbing of the batch-sharded output gather.
#include "exchange.cu"
