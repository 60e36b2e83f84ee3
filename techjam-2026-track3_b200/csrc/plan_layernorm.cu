// Token plan (valid-token compaction) and the two LayerNorm kernels.
//
// The reference masks padded keys inside attention and zeroes padded rows
// after the block and after the final LayerNorm
// (torch_transformer_benchmark.py:105-108,143-144,169-171).  Rows are
// independent everywhere except in attention, where a padded key only ever
// contributes exp(-inf) = 0.  So the whole layer can run on the valid tokens
// alone, packed densely: the token plan maps each valid token to a compact row
// (and back), the GEMMs and attention see only compact rows, and the final
// LayerNorm scatters back to [B, S, D] writing exact zeros for padded rows.
//
// LayerNorm follows nn.LayerNorm (biased variance, eps inside the rsqrt) as
// used at torch_transformer_benchmark.py:128-130,160 and
// v16_1_clean.py:615,527,625.  HBM-bound: one warp per row, the row kept in
// registers between the mean and the variance pass.
#include <stdarg.h>

#include "common.cuh"
#include "internal.h"

namespace tj {

// ---------------------------------------------------------------------------
// Token plan: one CTA of 1024 threads = 32 warps.  Warp w owns a contiguous
// segment of the B*S mask bytes and reads it 32 bytes at a time (coalesced),
// 16 groups per batch with every load issued before the first is used; a
// ballot gives the valid lanes, popc their rank.  Pass 1 counts each segment,
// a scan of the 32 counts gives each warp its first compact row, and pass 2
// re-reads the segment and writes orig/inv/cu coalesced.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanOrderMaxB = 256;  // batches up to this size get a longest-first order
constexpr int kPlanBatch = 16;  // 32-byte groups loaded per batch

// Valid flags of groups g0 .. g0+15 of the warp's segment, bit k for group k.
__device__ __forceinline__ uint32_t plan_load_batch(const uint8_t* __restrict__ mask, int g0, int end,
                                                     int lane) {
  uint8_t v[kPlanBatch];
#pragma unroll
  for (int k = 0; k < kPlanBatch; ++k) {
    const int i = g0 + 32 * k + lane;
    v[k] = (i < end) ? (mask ? __ldg(mask + i) : (uint8_t)1) : (uint8_t)0;
  }
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < kPlanBatch; ++k) bits |= (v[k] != 0 ? 1u : 0u) << k;
  return bits;
}

__global__ void __launch_bounds__(kPlanThreads) token_plan_kernel(const uint8_t* __restrict__ mask,
                                                                  int B, int S,
                                                                  int32_t* __restrict__ plan) {
  pdl_wait();
  const int total = B * S;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = ((total + 31) / 32 + 31) / 32 * 32;  // multiple of 32 elements
  const int begin = min(total, warp * seg);
  const int end = min(total, begin + seg);

  int32_t* cu = plan + 1;
  int32_t* cnt = plan + 2 + B;
  int32_t* orig = plan + 2 + 2 * B;
  int32_t* inv = orig + total;

  int count = 0;
  for (int g0 = begin; g0 < end; g0 += 32 * kPlanBatch) {
    const uint32_t bits = plan_load_batch(mask, g0, end, lane);
#pragma unroll
    for (int k = 0; k < kPlanBatch; ++k) count += __popc(__ballot_sync(0xffffffffu, (bits >> k) & 1u));
  }
  __shared__ int warp_base[32];
  if (lane == 0) warp_base[warp] = count;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_base[lane];
    int incl = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    warp_base[lane] = incl - w;
    if (lane == 31) {
      plan[0] = incl;
      cu[B] = incl;
    }
  }
  __syncthreads();
  int run = warp_base[warp];
  int next_start = (begin + S - 1) / S * S;  // first sample start at or after `begin`
  for (int g0 = begin; g0 < end; g0 += 32 * kPlanBatch) {
    const uint32_t bits = plan_load_batch(mask, g0, end, lane);
#pragma unroll
    for (int k = 0; k < kPlanBatch; ++k) {
      const int group0 = g0 + 32 * k;
      if (group0 >= end) break;  // uniform for the warp
      const int i = group0 + lane;
      const bool in = i < end;
      const bool valid = ((bits >> k) & 1u) != 0;
      const unsigned bal = __ballot_sync(0xffffffffu, valid);
      const int rank = __popc(bal & ((1u << lane) - 1u));
      // Samples starting inside this 32-element group (several when S < 32).
      while (next_start < group0 + 32 && next_start < end) {
        const int kk = next_start - group0;  // lane holding the sample start
        if (lane == kk) cu[next_start / S] = run + rank;
        next_start += S;
      }
      if (in) {
        if (valid) {
          orig[run + rank] = i;
          inv[i] = run + rank;
        } else {
          inv[i] = -1;
        }
      }
      run += __popc(bal);
    }
  }
  __syncthreads();
  __threadfence_block();
  int32_t* order = inv + total;
  __shared__ int cnt_s[kPlanOrderMaxB];
  for (int b = threadIdx.x; b < B; b += kPlanThreads) {
    const int c = ((volatile int32_t*)cu)[b + 1] - ((volatile int32_t*)cu)[b];
    cnt[b] = c;
    if (B <= kPlanOrderMaxB) cnt_s[b] = c;
  }
  // Samples by decreasing valid-token count (stable): attention launches its
  // CTAs for the longest samples first, so the last wave holds short ones.
  if (B <= kPlanOrderMaxB) {
    __syncthreads();
    for (int b = threadIdx.x; b < B; b += kPlanThreads) {
      const int c = cnt_s[b];
      int rank = 0;
      for (int o = 0; o < B; ++o) {
        const int co = cnt_s[o];
        rank += (co > c || (co == c && o < b)) ? 1 : 0;
      }
      order[rank] = b;
    }
  } else {
    for (int b = threadIdx.x; b < B; b += kPlanThreads) order[b] = b;
  }
  pdl_trigger();
}

int64_t plan_ints(int B, int S) { return 2 + 3 * (int64_t)B + 2 * (int64_t)B * S; }

int launch_token_plan(const uint8_t* mask, int B, int S, int32_t* plan, cudaStream_t stream) {
  if (B <= 0 || S <= 0) return set_error(TJ_ERR_INVALID_ARGUMENT, "token_plan: B=%d S=%d", B, S);
  if ((int64_t)B * S > (int64_t)INT32_MAX - 1)
    return set_error(TJ_ERR_UNSUPPORTED, "token_plan: B*S=%lld exceeds int32", (long long)B * S);
  if (plan == nullptr) return set_error(TJ_ERR_INVALID_ARGUMENT, "token_plan: null plan buffer");
  cudaError_t e = launch_pdl(token_plan_kernel, dim3(1), dim3(kPlanThreads), 0, stream, mask, B, S, plan);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "token_plan launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

// ---------------------------------------------------------------------------
// LayerNorm.  RT threads per row: one warp (RT = 32) or a whole CTA of 256
// threads (RT = 256) for wide rows.  A row is cut into groups of VW columns
// (4: float4 loads; 1 when D is not a multiple of 4); thread k of a row holds
// groups k, k+RT, ... (VPL of them, so D <= VW * RT * VPL), and the row stays
// in registers between the mean and the variance pass.  fp32 rows have stride
// D; fp16 rows (outputs and addends) their own stride, which the encoder pads
// to a multiple of 8 for the GEMMs' 16-byte TMA rows.
// ---------------------------------------------------------------------------
constexpr int kLnThreads = 256;
constexpr int kLnWideMaxD = 4 * kLnThreads * 32;

// Sum over the RT threads of a row (all of them get it).  RT = 256 goes
// through `red` (kLnThreads / 32 floats of shared memory), and every thread
// of the CTA must call it.
template <int RT>
__device__ __forceinline__ float ln_row_sum(float s, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if constexpr (RT > 32) {
    constexpr int kWarps = RT / 32;
    __syncthreads();  // an earlier sum may still be reading red
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w];
  }
  return s;
}

template <int VW>
__device__ __forceinline__ void ln_load(const float* row, int g, float (&v)[VW]) {
  if constexpr (VW == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row) + g);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else {
    v[0] = __ldg(row + g);
  }
}

template <int VW>
__device__ __forceinline__ void ln_store(float* row, int g, const float (&v)[VW]) {
  if constexpr (VW == 4)
    reinterpret_cast<float4*>(row)[g] = make_float4(v[0], v[1], v[2], v[3]);
  else
    row[g] = v[0];
}

// v += the VW fp16 values of group g of an addend row (fp32 sum).
template <int VW>
__device__ __forceinline__ void ln_add_f16(const __half* row, int g, float (&v)[VW]) {
  if constexpr (VW == 4) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(row) + g);
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] += lo.x;
    v[1] += lo.y;
    v[2] += hi.x;
    v[3] += hi.y;
  } else {
    v[0] += __half2float(row[g]);
  }
}

template <int VPL, int RT, int VW>
__device__ __forceinline__ void ln_row_stats(const float (&v)[VPL][VW], int D, int k, float& mean,
                                             float& rstd, float eps, float* red) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if ((i * RT + k) * VW < D)
#pragma unroll
      for (int e = 0; e < VW; ++e) s += v[i][e];
  mean = ln_row_sum<RT>(s, red) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if ((i * RT + k) * VW < D)
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const float c = v[i][e] - mean;
        q += c * c;
      }
  rstd = 1.0f / sqrtf(ln_row_sum<RT>(q, red) / (float)D + eps);
}

// y[r] = fp16(LayerNorm(x[row_map[r]] (+ add16[r]))), and with sum_out the
// fp32 row x[row_map[r]] + add16[r] is stored to sum_out[r] (the residual
// stream after a branch whose output the GEMM left in fp16).
template <int VPL, int RT, int VW>
__global__ void __launch_bounds__(kLnThreads) ln_cast_f16_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ row_map,
    const __half* __restrict__ add16, int ld_add, const int32_t* __restrict__ row_count, int rows,
    int D, const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
    float* __restrict__ sum_out, __half* __restrict__ y, int ld_y) {
  __shared__ float red[kLnThreads / 32];
  const int k = (int)threadIdx.x % RT;
  const int row = blockIdx.x * (kLnThreads / RT) + (int)threadIdx.x / RT;
  pdl_wait();
  pdl_trigger();
  const int limit = row_count ? min(rows, *row_count) : rows;
  if (row >= limit) return;  // uniform for the RT threads of a row
  const int64_t src = row_map ? (int64_t)row_map[row] : (int64_t)row;
  const float* xr = x + src * D;
  float v[VPL][VW];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      ln_load<VW>(xr, g, v[i]);
      if (add16) ln_add_f16<VW>(add16 + (int64_t)row * ld_add, g, v[i]);
      if (sum_out) ln_store<VW>(sum_out + (int64_t)row * D, g, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) v[i][e] = 0.f;
    }
  }
  float mean, rstd;
  ln_row_stats<VPL, RT, VW>(v, D, k, mean, rstd, eps, red);
  __half* yr = y + (int64_t)row * ld_y;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      float ga[VW], be[VW];
      ln_load<VW>(gamma, g, ga);
      ln_load<VW>(beta, g, be);
      if constexpr (VW == 4) {
        uint2 o;
        o.x = pack_half2((v[i][0] - mean) * rstd * ga[0] + be[0], (v[i][1] - mean) * rstd * ga[1] + be[1]);
        o.y = pack_half2((v[i][2] - mean) * rstd * ga[2] + be[2], (v[i][3] - mean) * rstd * ga[3] + be[3]);
        reinterpret_cast<uint2*>(yr)[g] = o;
      } else {
        yr[g] = __float2half_rn((v[i][0] - mean) * rstd * ga[0] + be[0]);
      }
    }
  }
}

// out[m] = LayerNorm(x + add16[c] (+ add16b[c])) for c = inv_map[m] >= 0 (x
// read at row c, or at row m with x_at_original), exact zeros otherwise.
template <int VPL, int RT, int VW>
__global__ void __launch_bounds__(kLnThreads) ln_final_kernel(const float* __restrict__ x,
                                                              const __half* __restrict__ add16,
                                                              const __half* __restrict__ add16b,
                                                              int ld_add, int x_at_original,
                                                              const int32_t* __restrict__ inv_map,
                                                              int rows, int D,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float eps,
                                                              float* __restrict__ out) {
  __shared__ float red[kLnThreads / 32];
  const int k = (int)threadIdx.x % RT;
  const int row = blockIdx.x * (kLnThreads / RT) + (int)threadIdx.x / RT;
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;  // uniform for the RT threads of a row
  const int64_t src = inv_map ? (int64_t)inv_map[row] : (int64_t)row;
  float* orow = out + (int64_t)row * D;
  if (src < 0) {  // padded token: exact zero, as masked_fill(~mask, 0) gives
    const float z[VW] = {};
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * VW < D) ln_store<VW>(orow, g, z);
    }
    return;
  }
  const float* xr = x + (x_at_original ? (int64_t)row : src) * D;
  float v[VPL][VW];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      ln_load<VW>(xr, g, v[i]);
      if (add16) ln_add_f16<VW>(add16 + src * ld_add, g, v[i]);
      if (add16b) ln_add_f16<VW>(add16b + src * ld_add, g, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) v[i][e] = 0.f;
    }
  }
  float mean, rstd;
  ln_row_stats<VPL, RT, VW>(v, D, k, mean, rstd, eps, red);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      float ga[VW], be[VW], o[VW];
      ln_load<VW>(gamma, g, ga);
      ln_load<VW>(beta, g, be);
#pragma unroll
      for (int e = 0; e < VW; ++e) o[e] = (v[i][e] - mean) * rstd * ga[e] + be[e];
      ln_store<VW>(orow, g, o);
    }
  }
}

// Groups per thread for a row of D columns in groups of VW: a warp per row up
// to 32 * 32 groups (VPL 1..32), then a CTA per row (VPL 8, 16, 32 of 256
// threads).  Returns 0 when the row is wider than that.
static int ln_vpl(int D, int VW, bool* wide) {
  const int groups = D / VW;
  *wide = groups > 32 * 32;
  const int per = *wide ? (groups + kLnThreads - 1) / kLnThreads : (groups + 31) / 32;
  for (int v = 1; v <= 32; v *= 2)
    if (per <= v) return *wide && v < 8 ? 8 : v;
  return 0;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_ln_cast_f16(const float* x, const int32_t* row_map, const int32_t* row_count, int rows,
                       int D, const float* gamma, const float* beta, float eps, void* y16,
                       cudaStream_t stream, const void* add16, float* sum_out, int ld_y, int ld_add) {
  if (ld_y <= 0) ld_y = D;
  if (ld_add <= 0) ld_add = D;
  if (rows < 0 || D <= 0 || ld_y < D || ld_add < D)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_cast_f16: rows=%d D=%d ld_y=%d ld_add=%d", rows, D, ld_y, ld_add);
  // float4 groups need 16-byte fp32 rows and 8-byte fp16 rows.
  const int VW = (D % 4 == 0 && ld_y % 4 == 0 && ld_add % 4 == 0 && aligned16(x) && aligned16(gamma) &&
                  aligned16(beta) && aligned16(sum_out) && (reinterpret_cast<uintptr_t>(y16) & 7u) == 0 &&
                  (reinterpret_cast<uintptr_t>(add16) & 7u) == 0)
                     ? 4 : 1;
  bool wide = false;
  const int vpl = ln_vpl(D, VW, &wide);
  if (vpl == 0)
    return set_error(TJ_ERR_UNSUPPORTED, "ln_cast_f16: D=%d above %d", D, VW == 4 ? kLnWideMaxD : kLnWideMaxD / 4);
  if (!x || !gamma || !beta || !y16 || (reinterpret_cast<uintptr_t>(x) & 3u) ||
      (reinterpret_cast<uintptr_t>(gamma) & 3u) || (reinterpret_cast<uintptr_t>(beta) & 3u) ||
      (reinterpret_cast<uintptr_t>(sum_out) & 3u) || (reinterpret_cast<uintptr_t>(y16) & 1u) ||
      (reinterpret_cast<uintptr_t>(add16) & 1u))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_cast_f16: null or misaligned pointer");
  if (rows == 0) return TJ_OK;
  const int per_cta = wide ? 1 : kLnThreads / 32;
  dim3 grid((rows + per_cta - 1) / per_cta);
  __half* y = static_cast<__half*>(y16);
  const __half* add = static_cast<const __half*>(add16);
  cudaError_t e = cudaSuccess;
#define TJ_LN_CASE(V, R, W) \
  e = launch_pdl(ln_cast_f16_kernel<V, R, W>, grid, dim3(kLnThreads), 0, stream, x, row_map, add, ld_add, row_count, rows, D, gamma, beta, eps, sum_out, y, ld_y)
#define TJ_LN_SWITCH(W)                                   \
  if (!wide) {                                            \
    switch (vpl) {                                        \
      case 1: TJ_LN_CASE(1, 32, W); break;                \
      case 2: TJ_LN_CASE(2, 32, W); break;                \
      case 4: TJ_LN_CASE(4, 32, W); break;                \
      case 8: TJ_LN_CASE(8, 32, W); break;                \
      case 16: TJ_LN_CASE(16, 32, W); break;              \
      default: TJ_LN_CASE(32, 32, W); break;              \
    }                                                     \
  } else {                                                \
    switch (vpl) {                                        \
      case 8: TJ_LN_CASE(8, kLnThreads, W); break;        \
      case 16: TJ_LN_CASE(16, kLnThreads, W); break;      \
      default: TJ_LN_CASE(32, kLnThreads, W); break;      \
    }                                                     \
  }
  if (VW == 4) {
    TJ_LN_SWITCH(4)
  } else {
    TJ_LN_SWITCH(1)
  }
#undef TJ_LN_SWITCH
#undef TJ_LN_CASE
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "ln_cast_f16 launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

int launch_ln_final(const float* x, const int32_t* inv_map, int rows, int D, const float* gamma,
                    const float* beta, float eps, float* out, cudaStream_t stream,
                    const void* add16, const void* add16b, bool x_at_original, int ld_add) {
  if (ld_add <= 0) ld_add = D;
  if (rows < 0 || D <= 0 || ld_add < D)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_final_mask: rows=%d D=%d ld_add=%d", rows, D, ld_add);
  const int VW = (D % 4 == 0 && ld_add % 4 == 0 && aligned16(x) && aligned16(gamma) && aligned16(beta) &&
                  aligned16(out) && (reinterpret_cast<uintptr_t>(add16) & 7u) == 0 &&
                  (reinterpret_cast<uintptr_t>(add16b) & 7u) == 0)
                     ? 4 : 1;
  bool wide = false;
  const int vpl = ln_vpl(D, VW, &wide);
  if (vpl == 0)
    return set_error(TJ_ERR_UNSUPPORTED, "ln_final_mask: D=%d above %d", D, VW == 4 ? kLnWideMaxD : kLnWideMaxD / 4);
  if (!x || !gamma || !beta || !out || (reinterpret_cast<uintptr_t>(x) & 3u) ||
      (reinterpret_cast<uintptr_t>(gamma) & 3u) || (reinterpret_cast<uintptr_t>(beta) & 3u) ||
      (reinterpret_cast<uintptr_t>(out) & 3u) || (reinterpret_cast<uintptr_t>(add16) & 1u) ||
      (reinterpret_cast<uintptr_t>(add16b) & 1u) || (add16b && !add16))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_final_mask: null or misaligned pointer");
  if (rows == 0) return TJ_OK;
  const int per_cta = wide ? 1 : kLnThreads / 32;
  dim3 grid((rows + per_cta - 1) / per_cta);
  const __half* add = static_cast<const __half*>(add16);
  const __half* addb = static_cast<const __half*>(add16b);
  const int xo = x_at_original ? 1 : 0;
  cudaError_t e = cudaSuccess;
#define TJ_LN_CASE(V, R, W) \
  e = launch_pdl(ln_final_kernel<V, R, W>, grid, dim3(kLnThreads), 0, stream, x, add, addb, ld_add, xo, inv_map, rows, D, gamma, beta, eps, out)
#define TJ_LN_SWITCH(W)                                   \
  if (!wide) {                                            \
    switch (vpl) {                                        \
      case 1: TJ_LN_CASE(1, 32, W); break;                \
      case 2: TJ_LN_CASE(2, 32, W); break;                \
      case 4: TJ_LN_CASE(4, 32, W); break;                \
      case 8: TJ_LN_CASE(8, 32, W); break;                \
      case 16: TJ_LN_CASE(16, 32, W); break;              \
      default: TJ_LN_CASE(32, 32, W); break;              \
    }                                                     \
  } else {                                                \
    switch (vpl) {                                        \
      case 8: TJ_LN_CASE(8, kLnThreads, W); break;        \
      case 16: TJ_LN_CASE(16, kLnThreads, W); break;      \
      default: TJ_LN_CASE(32, kLnThreads, W); break;      \
    }                                                     \
  }
  if (VW == 4) {
    TJ_LN_SWITCH(4)
  } else {
    TJ_LN_SWITCH(1)
  }
#undef TJ_LN_SWITCH
#undef TJ_LN_CASE
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "ln_final_mask launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

}  // namespace tj
