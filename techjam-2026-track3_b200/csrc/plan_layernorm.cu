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
// Token plan: CTAs of 1024 threads = 32 warps, CTA k owning the mask bytes
// [k*seg, (k+1)*seg) (seg >= kPlanMinSeg, so at most kPlanMaxCtas CTAs).  No
// CTA waits for another: each first counts the valid tokens before its
// segment itself (16-byte loads over the mask ahead of it; cheap next to the
// writes), then warp w owns a 32-byte-aligned part of the segment and reads it
// 32 bytes at a time (coalesced), 16 groups per batch with every load issued
// before the first is used; a ballot gives the valid lanes, popc their rank.
// Pass 1 counts each part, a scan of the 32 counts (after the CTA's prefix)
// gives each warp its first compact row, and pass 2 re-reads the part and
// writes orig/inv/cu coalesced.  The CTA holding a sample's first token
// position also writes that sample's count (reading the sample's tail past
// its segment if needed), the last CTA the total, and CTA 0 the longest-first
// sample order, for which it counts every sample's tokens on its own.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanMinSeg = 4096;
constexpr int kPlanMaxCtas = 256;
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

// Sum over the CTA (every thread gets it; all must call).
__device__ __forceinline__ int plan_block_sum(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red may still be read by an earlier sum
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int w = 0; w < kPlanThreads / 32; ++w) s += red[w];
  return s;
}

// Nonzero bytes of a 32-bit word.
__device__ __forceinline__ int plan_nz4(uint32_t w) { return __popc(__vcmpne4(w, 0u)) >> 3; }

// Valid tokens among mask bytes [lo, hi), counted by the whole CTA.
__device__ int plan_count(const uint8_t* __restrict__ mask, int lo, int hi, int* red) {
  int c = 0;
  if (hi > lo) {
    if (mask == nullptr) {
      c = threadIdx.x == 0 ? hi - lo : 0;
    } else {
      const uintptr_t p_lo = reinterpret_cast<uintptr_t>(mask + lo);
      const int a16 = min(hi, lo + (int)(((p_lo + 15) & ~(uintptr_t)15) - p_lo));
      const int n16 = (hi - a16) >> 4;
      const int b16 = a16 + 16 * n16;
      for (int i = lo + (int)threadIdx.x; i < a16; i += kPlanThreads) c += mask[i] != 0;
      const uint4* v = reinterpret_cast<const uint4*>(mask + a16);
      for (int i = threadIdx.x; i < n16; i += kPlanThreads) {
        const uint4 w = __ldg(v + i);
        c += plan_nz4(w.x) + plan_nz4(w.y) + plan_nz4(w.z) + plan_nz4(w.w);
      }
      for (int i = b16 + (int)threadIdx.x; i < hi; i += kPlanThreads) c += mask[i] != 0;
    }
  }
  return plan_block_sum(c, red);
}

static int plan_segment(int64_t total) {
  int64_t seg = (total + kPlanMaxCtas - 1) / kPlanMaxCtas;
  if (seg < kPlanMinSeg) seg = kPlanMinSeg;
  return (int)((seg + 1023) / 1024 * 1024);  // whole 32-byte groups for each of the 32 warps
}

__global__ void __launch_bounds__(kPlanThreads) token_plan_kernel(const uint8_t* __restrict__ mask,
                                                                  int B, int S, int seg,
                                                                  int32_t* __restrict__ plan) {
  __shared__ int red[32];
  __shared__ int warp_base[32];
  __shared__ int cnt_s[kPlanOrderMaxB];
  pdl_wait();
  const int total = B * S;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cb = (int)blockIdx.x * seg;
  const int ce = min(total, cb + seg);
  const int wseg = seg / 32;  // a multiple of 32
  const int begin = min(ce, cb + warp * wseg);
  const int end = min(ce, begin + wseg);

  int32_t* cu = plan + 1;
  int32_t* cnt = plan + 2 + B;
  int32_t* orig = plan + 2 + 2 * B;
  int32_t* inv = orig + total;
  int32_t* order = inv + total;

  const int prefix = cb > 0 ? plan_count(mask, 0, cb, red) : 0;  // uniform for the CTA

  int count = 0;
  for (int g0 = begin; g0 < end; g0 += 32 * kPlanBatch) {
    const uint32_t bits = plan_load_batch(mask, g0, end, lane);
#pragma unroll
    for (int k = 0; k < kPlanBatch; ++k) count += __popc(__ballot_sync(0xffffffffu, (bits >> k) & 1u));
  }
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
    red[lane] = incl;  // lane 31: the segment's count (red is free until the next sum)
  }
  __syncthreads();
  const int seg_end_row = prefix + red[31];  // compact row of the first token after the segment
  int run = prefix + warp_base[warp];
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
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
    plan[0] = seg_end_row;
    cu[B] = seg_end_row;
  }
  __syncthreads();
  __threadfence_block();
  // Counts of the samples starting in this segment: up to the next start
  // inside it, or to the segment end plus the sample's tokens past it.
  const int b_first = (cb + S - 1) / S;
  const int b_end = min(B, (ce + S - 1) / S);  // samples b_first .. b_end-1 start here
  if (b_first < b_end) {
    const volatile int32_t* vcu = cu;
    for (int bb = b_first + (int)threadIdx.x; bb < b_end; bb += kPlanThreads)
      if ((bb + 1) * S <= ce) cnt[bb] = ((bb + 1) * S < ce ? vcu[bb + 1] : seg_end_row) - vcu[bb];
    const int bl = b_end - 1;  // the last one may run past the segment
    if ((bl + 1) * S > ce) {
      const int tail = plan_count(mask, ce, (bl + 1) * S, red);
      if (threadIdx.x == 0) cnt[bl] = seg_end_row - vcu[bl] + tail;
    }
  }
  // Samples by decreasing valid-token count (stable): attention launches its
  // CTAs for the longest samples first, so the last wave holds short ones.
  if (blockIdx.x == 0) {
    if (B <= kPlanOrderMaxB && gridDim.x == 1) {
      // One CTA holds the whole mask: this CTA wrote every count above.
      __syncthreads();
      __threadfence_block();
      for (int bb = threadIdx.x; bb < B; bb += kPlanThreads) cnt_s[bb] = ((volatile int32_t*)cnt)[bb];
    } else if (B <= kPlanOrderMaxB) {
      for (int bb = threadIdx.x; bb < B; bb += kPlanThreads) cnt_s[bb] = mask ? 0 : S;
      __syncthreads();
      if (mask) {
        // Each thread counts a contiguous stretch of the mask, one
        // shared-memory add per sample it touches: 16 bytes per load where
        // the address is 16-byte aligned and the 16 bytes lie in one sample
        // and the stretch, single bytes elsewhere (after a sample boundary
        // until the next aligned address).
        const uintptr_t base = reinterpret_cast<uintptr_t>(mask);
        const int per = ((total + kPlanThreads - 1) / kPlanThreads + 15) & ~15;
        const int lo = min(total, (int)threadIdx.x * per), hi = min(total, lo + per);
        int cur = lo / S, acc = 0;
        int64_t next_b = (int64_t)(cur + 1) * S;
        for (int i = lo; i < hi;) {
          if (((base + (uintptr_t)i) & 15u) == 0 && i + 16 <= hi && i + 16 <= next_b) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(mask + i));
            acc += plan_nz4(w.x) + plan_nz4(w.y) + plan_nz4(w.z) + plan_nz4(w.w);
            i += 16;
          } else {
            acc += mask[i] != 0;
            ++i;
          }
          if (i == next_b) {
            if (acc) atomicAdd(&cnt_s[cur], acc);
            acc = 0;
            ++cur;
            next_b += S;
          }
        }
        if (acc) atomicAdd(&cnt_s[cur], acc);
      }
    }
    if (B <= kPlanOrderMaxB) {
      __syncthreads();
      for (int bb = threadIdx.x; bb < B; bb += kPlanThreads) {
        const int c = cnt_s[bb];
        int rank = 0;
        for (int o = 0; o < B; ++o) {
          const int co = cnt_s[o];
          rank += (co > c || (co == c && o < bb)) ? 1 : 0;
        }
        order[rank] = bb;
      }
    } else {
      for (int bb = threadIdx.x; bb < B; bb += kPlanThreads) order[bb] = bb;
    }
  }
  pdl_trigger();
}

int64_t plan_ints(int B, int S) { return 2 + 3 * (int64_t)B + 2 * (int64_t)B * S; }

int launch_token_plan(const uint8_t* mask, int B, int S, int32_t* plan, cudaStream_t stream) {
  if (B <= 0 || S <= 0) return set_error(TJ_ERR_INVALID_ARGUMENT, "token_plan: B=%d S=%d", B, S);
  if ((int64_t)B * S > (int64_t)INT32_MAX - 1)
    return set_error(TJ_ERR_UNSUPPORTED, "token_plan: B*S=%lld exceeds int32", (long long)B * S);
  if (plan == nullptr) return set_error(TJ_ERR_INVALID_ARGUMENT, "token_plan: null plan buffer");
  const int seg = plan_segment((int64_t)B * S);
  const int ctas = (int)(((int64_t)B * S + seg - 1) / seg);
  cudaError_t e = launch_pdl(token_plan_kernel, dim3(ctas), dim3(kPlanThreads), 0, stream, mask, B, S, seg, plan);
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
  // Every load of the row is issued before the first use.
  float v[VPL][VW];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      ln_load<VW>(xr, g, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) v[i][e] = 0.f;
    }
  }
  if (add16) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * VW < D) ln_add_f16<VW>(add16 + (int64_t)row * ld_add, g, v[i]);
    }
  }
  if (sum_out) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * VW < D) ln_store<VW>(sum_out + (int64_t)row * D, g, v[i]);
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
  // Every load of the row is issued before the first use.
  float v[VPL][VW];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int g = i * RT + k;
    if (g * VW < D) {
      ln_load<VW>(xr, g, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) v[i][e] = 0.f;
    }
  }
  if (add16) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * VW < D) ln_add_f16<VW>(add16 + src * ld_add, g, v[i]);
    }
  }
  if (add16b) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int g = i * RT + k;
      if (g * VW < D) ln_add_f16<VW>(add16b + src * ld_add, g, v[i]);
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
