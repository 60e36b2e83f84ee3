// Host-side launchers shared between the kernel files and the C-ABI layer.
// Every launcher checks its own arguments and returns a tj status code
// (TJ_OK on success); none of them synchronises or allocates.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/techjam_b200.h"

namespace tj {

// Launches `kernel` on `stream` with programmatic stream serialization (see
// pdl_wait/pdl_trigger in common.cuh).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Records a printf-style message for tj_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

int ensure_device_props(int* num_sms);

// Index of the current device for per-device caches of launch attributes
// (call after ensure_device_props, which rejects indices >= 64).
inline int device_index() {
  int d = 0;
  cudaGetDevice(&d);
  return d & 63;
}

// Number of int32 entries of the token plan for a [B, S] batch.
int64_t plan_ints(int B, int S);

// Token plan layout (int32):
//   [0]                 nv  (number of valid tokens)
//   [1, 1+B+1)          cu  (compact offset of each sample; cu[B] = nv)
//   [B+2, B+2+B)        n   (valid tokens per sample)
//   [2B+2, 2B+2+BS)     orig (compact row -> original row b*S+s)
//   [2B+2+BS, ...+BS)   inv  (original row -> compact row, or -1)
//   [2B+2+2BS, ...+B)   order (samples by decreasing valid count; identity
//                        for batches above 256)
struct PlanView {
  int32_t* base;
  int B, S;
  int32_t* nv() const { return base; }
  int32_t* cu() const { return base + 1; }
  int32_t* n() const { return base + 2 + B; }
  int32_t* orig() const { return base + 2 + 2 * B; }
  int32_t* inv() const { return base + 2 + 2 * B + (int64_t)B * S; }
  int32_t* order() const { return base + 2 + 2 * B + 2 * (int64_t)B * S; }
};

int launch_token_plan(const uint8_t* mask, int B, int S, int32_t* plan, cudaStream_t stream);

// add16 (optional, fp16, compact rows) is added to the x row before the
// LayerNorm; sum_out (optional) receives that fp32 sum.  fp32 rows have
// stride D; ld_y / ld_add are the fp16 row strides (0 = D).
int launch_ln_cast_f16(const float* x, const int32_t* row_map, const int32_t* row_count, int rows,
                       int D, const float* gamma, const float* beta, float eps, void* y16,
                       cudaStream_t stream, const void* add16 = nullptr, float* sum_out = nullptr,
                       int ld_y = 0, int ld_add = 0);

// add16b (optional) is a second fp16 addend; with x_at_original, x is read
// at the output row m instead of the compact row inv_map[m].  ld_add is the
// fp16 addends' row stride (0 = D).
int launch_ln_final(const float* x, const int32_t* inv_map, int rows, int D, const float* gamma,
                    const float* beta, float eps, float* out, cudaStream_t stream,
                    const void* add16 = nullptr, const void* add16b = nullptr,
                    bool x_at_original = false, int ld_add = 0);

enum GemmEpilogue : int {
  kEpiQkvHeadMajor = 0,   // fp16 out, head-major [3][H][rows_max][attn_head_pad(dh)]
  kEpiResidualF32 = 1,    // fp32 out = acc + bias + residual[row_map(row)]
  kEpiGeluF16 = 2,        // fp16 out = gelu_erf(acc + bias)
  kEpiBiasF16 = 3,        // fp16 out = acc + bias
};

struct GemmArgs {
  const void* a16;          // [rows_max, K] fp16, row stride lda
  const void* w16;          // [N, K] fp16, row stride ldw (nn.Linear layout)
  const float* bias;        // [N]
  const int32_t* row_count; // device int (rows actually present), or null = rows_max
  int rows_max, N, K;
  int lda, ldw;             // row strides in elements, multiples of 8 (0 = K)
  void* out;                // epilogue-dependent
  int ld_out;               // elements
  const float* resid;       // kEpiResidualF32
  const int32_t* resid_map; // optional gather map for residual rows
  int ld_resid;
  int heads, head_dim;      // kEpiQkvHeadMajor
};

int launch_gemm(int epilogue, const GemmArgs& args, cudaStream_t stream);

struct AttnArgs {
  const void* q;            // fp16 [H][q_rows][P], P = attn_head_pad(head_dim)
  const void* k;            // fp16, addressed as [G][H][kv_rows][P] with strides below
  const void* v;
  int H, head_dim;
  int q_rows;               // rows of the Q slab per head
  int kv_rows;              // rows of one K/V slab per head and segment
  int64_t kv_stride_h;      // elements between heads
  int64_t kv_stride_g;      // elements between segments
  int G;                    // key segments per sample
  int B;                    // samples
  int max_q_per_sample;     // upper bound on valid queries per sample
  const int32_t* q_cu;      // [B+1] compact query offsets
  const int32_t* kv_off;    // [B*G] row offset of each key segment
  const int32_t* kv_len;    // [B*G] keys in each segment
  int64_t kv_len_stride;    // stride between samples in kv_off/kv_len (usually G)
  float scale;              // softmax scale (head_dim^-0.5)
  int causal;               // 1: key position > query position masked
  const int32_t* q_pos0;    // causal only: position of the first query of each sample
  const int32_t* order;     // optional [B]: sample of each grid row (longest first)
  void* ctx;                // fp16 [q_rows][ld_ctx]: head h in columns [h*dh, h*dh + dh)
  int64_t ld_ctx;           // elements between context rows; 0 = H*dh
  float* part_o;            // partial context fp32 [q_rows][H*dh] (part_mode 1 writes, 2 reads)
  float* part_lse;          // partial log2-sum-exp [q_rows][H]
  int part_mode;            // 0 ctx, 1 write the partial, 2 merge with the partial into ctx
};

int launch_attention(const AttnArgs& args, cudaStream_t stream);

// Row length (halves) of the head-major q/k/v buffers for a head dim: 64,
// 128 or 256 (heads are zero-padded up to it).
int attn_head_pad(int head_dim);

}  // namespace tj
