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
// LayerNorm.  RT threads per row: one warp (RT = 32, D <= 4096) or a whole
// CTA of 256 threads (RT = 256, wider rows up to 32768).  Thread k of a row
// holds float4 groups k, k+RT, ... (VPL groups, so D <= 4 * RT * VPL), and
// the row stays in registers between the mean and the variance pass.
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

template <int VPL, int RT>
__device__ __forceinline__ void ln_row_stats(const float4 (&v)[VPL], int D, int k, float& mean,
                                             float& rstd, float eps, float* red) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if ((i * RT + k) * 4 < D) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  mean = ln_row_sum<RT>(s, red) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if ((i * RT + k) * 4 < D) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  rstd = 1.0f / sqrtf(ln_row_sum<RT>(q, red) / (float)D + eps);
}

// v[i] += the four fp16 values of group g of an addend row (fp32 sum).
template <int VPL, int RT>
__device__ __forceinline__ void add_f16_row(float4 (&v)[VPL], const __half* add_row, int D, int k) {
  const uint2* ar = reinterpret_cast<const uint2*>(add_row);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * 4 < D) {
      const uint2 u = __ldg(ar + g);
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[i].x += lo.x;
      v[i].y += lo.y;
      v[i].z += hi.x;
      v[i].w += hi.y;
    }
  }
}

// y[r] = fp16(LayerNorm(x[row_map[r]] (+ add16[r]))), and with sum_out the
// fp32 row x[row_map[r]] + add16[r] is stored to sum_out[r] (the residual
// stream after a branch whose output the GEMM left in fp16).
template <int VPL, int RT>
__global__ void __launch_bounds__(kLnThreads) ln_cast_f16_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ row_map,
    const __half* __restrict__ add16, const int32_t* __restrict__ row_count, int rows, int D,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
    float* __restrict__ sum_out, __half* __restrict__ y) {
  __shared__ float red[kLnThreads / 32];
  const int k = (int)threadIdx.x % RT;
  const int row = blockIdx.x * (kLnThreads / RT) + (int)threadIdx.x / RT;
  pdl_wait();
  pdl_trigger();
  const int limit = row_count ? min(rows, *row_count) : rows;
  if (row >= limit) return;  // uniform for the RT threads of a row
  const int64_t src = row_map ? (int64_t)row_map[row] : (int64_t)row;
  const float4* xr = reinterpret_cast<const float4*>(x + src * D);
  float4 v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    v[i] = (g * 4 < D) ? __ldg(xr + g) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (add16) add_f16_row<VPL, RT>(v, add16 + (int64_t)row * D, D, k);
  if (sum_out) {
    float4* sr = reinterpret_cast<float4*>(sum_out + (int64_t)row * D);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * 4 < D) sr[g] = v[i];
    }
  }
  float mean, rstd;
  ln_row_stats<VPL, RT>(v, D, k, mean, rstd, eps, red);
  uint2* yr = reinterpret_cast<uint2*>(y + (int64_t)row * D);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * 4 < D) {
      const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma) + g);
      const float4 be = __ldg(reinterpret_cast<const float4*>(beta) + g);
      uint2 o;
      o.x = pack_half2((v[i].x - mean) * rstd * ga.x + be.x, (v[i].y - mean) * rstd * ga.y + be.y);
      o.y = pack_half2((v[i].z - mean) * rstd * ga.z + be.z, (v[i].w - mean) * rstd * ga.w + be.w);
      yr[g] = o;
    }
  }
}

// out[m] = LayerNorm(x + add16[c] (+ add16b[c])) for c = inv_map[m] >= 0 (x
// read at row c, or at row m with x_at_original), exact zeros otherwise.
template <int VPL, int RT>
__global__ void __launch_bounds__(kLnThreads) ln_final_kernel(const float* __restrict__ x,
                                                              const __half* __restrict__ add16,
                                                              const __half* __restrict__ add16b,
                                                              int x_at_original,
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
  float4* orow = reinterpret_cast<float4*>(out + (int64_t)row * D);
  if (src < 0) {  // padded token: exact zero, as masked_fill(~mask, 0) gives
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * 4 < D) orow[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  const float4* xr = reinterpret_cast<const float4*>(x + (x_at_original ? (int64_t)row : src) * D);
  float4 v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    v[i] = (g * 4 < D) ? __ldg(xr + g) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (add16) add_f16_row<VPL, RT>(v, add16 + src * D, D, k);
  if (add16b) add_f16_row<VPL, RT>(v, add16b + src * D, D, k);
  float mean, rstd;
  ln_row_stats<VPL, RT>(v, D, k, mean, rstd, eps, red);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * 4 < D) {
      const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma) + g);
      const float4 be = __ldg(reinterpret_cast<const float4*>(beta) + g);
      float4 o;
      o.x = (v[i].x - mean) * rstd * ga.x + be.x;
      o.y = (v[i].y - mean) * rstd * ga.y + be.y;
      o.z = (v[i].z - mean) * rstd * ga.z + be.z;
      o.w = (v[i].w - mean) * rstd * ga.w + be.w;
      orow[g] = o;
    }
  }
}

// Groups of 4 columns per thread for a row of D columns: a warp per row up to
// D = 4096 (VPL 1..32), then a CTA per row (VPL 8, 16, 32 of 256 threads).
// Returns 0 when D is above kLnWideMaxD.
static int ln_vpl(int D, bool* wide) {
  const int groups = D / 4;
  *wide = groups > 32 * 32;
  const int per = *wide ? (groups + kLnThreads - 1) / kLnThreads : (groups + 31) / 32;
  for (int v = 1; v <= 32; v *= 2)
    if (per <= v) return *wide && v < 8 ? 8 : v;
  return 0;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_ln_cast_f16(const float* x, const int32_t* row_map, const int32_t* row_count, int rows,
                       int D, const float* gamma, const float* beta, float eps, void* y16,
                       cudaStream_t stream, const void* add16, float* sum_out) {
  if (rows < 0 || D <= 0 || D % 4 != 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_cast_f16: rows=%d D=%d (D must be a positive multiple of 4)", rows, D);
  bool wide = false;
  const int vpl = ln_vpl(D, &wide);
  if (vpl == 0) return set_error(TJ_ERR_UNSUPPORTED, "ln_cast_f16: D=%d above %d", D, kLnWideMaxD);
  if (!x || !gamma || !beta || !y16 || !aligned16(x) || !aligned16(gamma) || !aligned16(beta) ||
      (reinterpret_cast<uintptr_t>(y16) & 7u) || (reinterpret_cast<uintptr_t>(add16) & 7u) ||
      !aligned16(sum_out))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_cast_f16: null or misaligned pointer");
  if (rows == 0) return TJ_OK;
  const int per_cta = wide ? 1 : kLnThreads / 32;
  dim3 grid((rows + per_cta - 1) / per_cta);
  __half* y = static_cast<__half*>(y16);
  const __half* add = static_cast<const __half*>(add16);
  cudaError_t e = cudaSuccess;
#define TJ_LN_CASE(V, R) \
  e = launch_pdl(ln_cast_f16_kernel<V, R>, grid, dim3(kLnThreads), 0, stream, x, row_map, add, row_count, rows, D, gamma, beta, eps, sum_out, y)
  if (!wide) {
    switch (vpl) {
      case 1: TJ_LN_CASE(1, 32); break;
      case 2: TJ_LN_CASE(2, 32); break;
      case 4: TJ_LN_CASE(4, 32); break;
      case 8: TJ_LN_CASE(8, 32); break;
      case 16: TJ_LN_CASE(16, 32); break;
      default: TJ_LN_CASE(32, 32); break;
    }
  } else {
    switch (vpl) {
      case 8: TJ_LN_CASE(8, kLnThreads); break;
      case 16: TJ_LN_CASE(16, kLnThreads); break;
      default: TJ_LN_CASE(32, kLnThreads); break;
    }
  }
#undef TJ_LN_CASE
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "ln_cast_f16 launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

int launch_ln_final(const float* x, const int32_t* inv_map, int rows, int D, const float* gamma,
                    const float* beta, float eps, float* out, cudaStream_t stream,
                    const void* add16, const void* add16b, bool x_at_original) {
  if (rows < 0 || D <= 0 || D % 4 != 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_final_mask: rows=%d D=%d (D must be a positive multiple of 4)", rows, D);
  bool wide = false;
  const int vpl = ln_vpl(D, &wide);
  if (vpl == 0) return set_error(TJ_ERR_UNSUPPORTED, "ln_final_mask: D=%d above %d", D, kLnWideMaxD);
  if (!x || !gamma || !beta || !out || !aligned16(x) || !aligned16(gamma) || !aligned16(beta) ||
      !aligned16(out) || (reinterpret_cast<uintptr_t>(add16) & 7u) ||
      (reinterpret_cast<uintptr_t>(add16b) & 7u) || (add16b && !add16))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ln_final_mask: null or misaligned pointer");
  if (rows == 0) return TJ_OK;
  const int per_cta = wide ? 1 : kLnThreads / 32;
  dim3 grid((rows + per_cta - 1) / per_cta);
  const __half* add = static_cast<const __half*>(add16);
  const __half* addb = static_cast<const __half*>(add16b);
  const int xo = x_at_original ? 1 : 0;
  cudaError_t e = cudaSuccess;
#define TJ_LN_CASE(V, R) \
  e = launch_pdl(ln_final_kernel<V, R>, grid, dim3(kLnThreads), 0, stream, x, add, addb, xo, inv_map, rows, D, gamma, beta, eps, out)
  if (!wide) {
    switch (vpl) {
      case 1: TJ_LN_CASE(1, 32); break;
      case 2: TJ_LN_CASE(2, 32); break;
      case 4: TJ_LN_CASE(4, 32); break;
      case 8: TJ_LN_CASE(8, 32); break;
      case 16: TJ_LN_CASE(16, 32); break;
      default: TJ_LN_CASE(32, 32); break;
    }
  } else {
    switch (vpl) {
      case 8: TJ_LN_CASE(8, kLnThreads); break;
      case 16: TJ_LN_CASE(16, kLnThreads); break;
      default: TJ_LN_CASE(32, kLnThreads); break;
    }
  }
#undef TJ_LN_CASE
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "ln_final_mask launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

}  // namespace tj
