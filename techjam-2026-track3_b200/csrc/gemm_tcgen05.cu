// Persistent tcgen05 GEMM, C[M,N] = A[M,K] * W[N,K]^T with fp16 operands and an
// fp32 TMEM accumulator, and the epilogues of the encoder layer's projections:
//
//   kEpiQkvHeadMajor  QKV projection (v16_1_clean.py:474-489): +bias, fp16,
//                     stored straight into the head-major [3][H][rows][P]
//                     layout attention reads (heads zero-padded to P = 64, 128
//                     or 256 columns), so no permute/contiguous pass.
//   kEpiResidualF32   output projection (v16_1_clean.py:516-523 + :620) and
//                     FFN-out (v16_1_clean.py:533-537 + :621): +bias, +fp32
//                     residual, fp32 store.
//   kEpiGeluF16       FFN-in (v16_1_clean.py:221-301, the Triton fused op):
//                     +bias, erf-GELU on the fp32 accumulator, fp16.
//   kEpiBiasF16       output projection (v16_1_clean.py:519-523) and FFN-out
//                     (v16_1_clean.py:533-537): +bias, fp16, as the reference's
//                     F.linear in fp16; the residual add happens in the
//                     LayerNorm kernel that reads the result.
//
// Structure (one CTA per SM, 64 + 32 * epilogue-warps threads):
//   warp 0      TMA producer: A and W tiles (128-byte swizzle) into a ring of
//               shared-memory stages, completion on mbarriers.
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) into one of two TMEM accumulators.
//   warps 2..    epilogue (8 or 16 warps): tcgen05.ld of the accumulator (warp
//               w reads TMEM lanes 32*(w%4)..+31 = tile rows; the warps of a
//               lane quarter split the tile's columns), fused math, stores.
// Two accumulators let the epilogue of tile i overlap the main loop of tile
// i+1.  Tiles are walked n-fastest so CTAs running at the same time share the
// A tile through L2.  The number of rows comes from device memory (the token
// plan), so the host never synchronises to learn it.  Large problems run the
// CTA-pair variant (gemm_tcgen05_pair_kernel: two SMs per 256x256 tile with
// tcgen05.mma.cta_group::2, each loading half of A and half of W).  Row
// strides may exceed K (rows padded to whole 16-byte units); the tile loads
// stop at K and zero-fill the rest of the last k-block.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"

namespace tj {

// Epilogue warps per CTA: 8 for the residual epilogue (each thread keeps the
// prefetched residual of its row in registers), 16 for the fp16 epilogues
// (GELU is ALU-heavy; more warps hide its latency).
__host__ __device__ constexpr int epi_warps_for(int bn, int epi) {
  return bn < 256 ? 8 : (epi == 1 ? 8 : 16);
}
__host__ __device__ constexpr int gemm_threads_for(int bn, int epi) {
  return 64 + 32 * epi_warps_for(bn, epi);
}
constexpr int kBM = 128;
constexpr int kBK = 64;

struct GemmKernelParams {
  const float* bias;
  const int32_t* row_count;
  int rows_max, N, K;
  void* out;
  int ld_out;
  const float* resid;
  const int32_t* resid_map;
  int ld_resid;
  int heads, head_dim, d_model;
  int head_pad;  // head-major row length (halves) of the QKV output: 64, 128 or 256
  // 1: the fp16 epilogue stores whole 32-row blocks with TMA (tensor map tmC
  // of the pair kernel; 64-byte swizzle, 32 x 32 boxes); 0: st.global only.
  int tma_store;
};

// Shared-memory scratch of the epilogue warps (one 32-row block each), used to
// turn the TMEM layout (thread = row) into row-contiguous global accesses.
constexpr uint32_t kEpiScratchBytes = 32768;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  static constexpr size_t kSmemBytes = 1024 /*align slack*/ + (size_t)kStages * kStageBytes +
                                       256 /*barriers etc*/ + kEpiScratchBytes;
};

// GELU(x) = x * Phi(x) with Phi(x) = (1 + erf(x / sqrt(2))) / 2 and erf from
// Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7,
// so Phi(x) = 1 - c/2 for x >= 0 and c/2 for x < 0, c = erfc(|x| / sqrt(2)).
// Branch-free, on pairs (packed FMA); the absolute error on GELU stays below
// 5e-7, far under the fp16 rounding of the output.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 gelu2(float2 x) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f,
                  kA4 = -1.453152027f, kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  constexpr float kNegLog2e = -1.4426950408889634f;
  const float2 z = make_float2(fabsf(x.x) * kInvSqrt2, fabsf(x.y) * kInvSqrt2);
  const float2 den = ffma2(z, make_float2(kP, kP), make_float2(1.f, 1.f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  float2 q = ffma2(make_float2(kA5, kA5), t, make_float2(kA4, kA4));
  q = ffma2(q, t, make_float2(kA3, kA3));
  q = ffma2(q, t, make_float2(kA2, kA2));
  q = ffma2(q, t, make_float2(kA1, kA1));
  q = fmul2(q, t);
  const float2 arg = fmul2(fmul2(z, z), make_float2(kNegLog2e, kNegLog2e));
  const float2 e = make_float2(exp2_approx(arg.x), exp2_approx(arg.y));
  const float2 hc = fmul2(fmul2(q, e), make_float2(0.5f, 0.5f));  // erfc(|x|/sqrt2) / 2
  const float2 phi = make_float2(x.x >= 0.f ? 1.f - hc.x : hc.x, x.y >= 0.f ? 1.f - hc.y : hc.y);
  return fmul2(x, phi);
}

// Wait without the CTA abort flag: used on the exit path to let TMA loads or
// MMAs already in flight land before the CTA releases its shared memory/TMEM.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Bulk tensor stores (shared -> global, completion tracked per thread in bulk
// groups).  The innermost coordinate is a multiple of 32 fp16 elements.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The bulk stores of this thread have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// The bulk stores of this thread are complete (written to global memory).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Epilogue of one accumulator tile for one epilogue warp: its 32 rows (TMEM
// lane quarter) and its column slice, in 32-column chunks.  Each chunk is
// read from TMEM with one row per thread, passed through the warp's scratch
// (16-byte granules XOR-swizzled by row, so neither the row-wise writes nor
// the column-wise reads conflict) and written with consecutive lanes on
// consecutive addresses of a row:
//   fp32 (residual): lane = (row l/8 + 4i, 4 columns), 128 B per row segment;
//   fp16 (QKV, GELU): lane = (row l/4 + 8i, 8 columns), 64 B per row segment.
// The residual is prefetched in the store layout before the accumulator is
// waited for, so its DRAM latency hides behind the tile's main loop.
// With tmC (the pair kernel, p.tma_store), a full 32-row block of an fp16
// output leaves the scratch as one bulk tensor store instead: the scratch
// rows are 64 bytes with the granules XOR-swizzled by (row >> 1) & 3, which is
// the 64-byte TMA swizzle, and the scratch is 512-byte aligned.  Before the
// scratch is rewritten, lane 0 waits until its last store has read it.
// Returns false if the CTA aborts.
template <int BN, int EPI, int kEpiWarps>
__device__ __forceinline__ bool epilogue_tile(const GemmKernelParams& p, uint32_t tmem_acc, int m0,
                                              int n0, int rows, int quarter, int slice, uint32_t lane,
                                              uint32_t tfull_bar, uint32_t tfull_parity,
                                              volatile int* abort_flag, uint32_t scratch,
                                              const CUtensorMap* tmC = nullptr) {
  constexpr int kSlices = kEpiWarps / 4;
  constexpr int kChunks = BN / 32 / kSlices;
  const int row_base = m0 + quarter * 32;
  const uint32_t t_row = tmem_acc + ((uint32_t)(quarter * 32) << 16);

  if constexpr (EPI == kEpiResidualF32) {
    const int sub = (int)(lane >> 3);
    const int c4 = (int)(lane & 7) * 4;
    int rrow[8];  // residual row of each output row, -1 past the row count
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = row_base + sub + 4 * i;
      rrow[i] = row < rows ? (p.resid_map ? p.resid_map[row] : row) : -1;
    }
    float4 res[kChunks][8];
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int col = n0 + (slice * kChunks + cc) * 32 + c4;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        res[cc][i] = (rrow[i] >= 0 && col < p.N)
                         ? __ldg(reinterpret_cast<const float4*>(p.resid + (int64_t)rrow[i] * p.ld_resid + col))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (!mbar_wait(tfull_bar, tfull_parity, abort_flag, 131)) return false;
    tc_fence_after();
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int c = slice * kChunks + cc;
      const int col = n0 + c * 32 + c4;
      uint32_t r[32];
      tmem_ld32(t_row + (uint32_t)(c * 32), r);
      tmem_ld_wait();
#pragma unroll
      for (int k = 0; k < 8; ++k)
        st_shared_v4(scratch + lane * 128 + ((k ^ (lane & 7)) << 4),
                     make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]));
      __syncwarp();
      const float4 b4 = col < p.N ? __ldg(reinterpret_cast<const float4*>(p.bias + col))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t rr = (uint32_t)(sub + 4 * i);
        const uint4 a = ld_shared_v4(scratch + rr * 128 + (((lane & 7) ^ (rr & 7)) << 4));
        if (rrow[i] >= 0 && col < p.N) {
          const float4 rs = res[cc][i];
          *reinterpret_cast<float4*>(static_cast<float*>(p.out) + (int64_t)(row_base + (int)rr) * p.ld_out + col) =
              make_float4(__uint_as_float(a.x) + b4.x + rs.x, __uint_as_float(a.y) + b4.y + rs.y,
                          __uint_as_float(a.z) + b4.z + rs.z, __uint_as_float(a.w) + b4.w + rs.w);
        }
      }
      __syncwarp();  // the next chunk reuses the scratch
    }
    return true;
  } else {
    if (!mbar_wait(tfull_bar, tfull_parity, abort_flag, 130 + EPI)) return false;
    tc_fence_after();
    // Two TMEM chunks per wait when the slice has them.
    constexpr int kPerWait = kChunks < 2 ? 1 : 2;
    const bool hm_fast = EPI == kEpiQkvHeadMajor && (p.head_dim & 31) == 0;
    uint32_t rbuf[kPerWait][32];
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int c = slice * kChunks + cc;
      if (cc % kPerWait == 0) {
#pragma unroll
        for (int u = 0; u < kPerWait; ++u) tmem_ld32(t_row + (uint32_t)((c + u) * 32), rbuf[u]);
        tmem_ld_wait();
      }
      const uint32_t (&r)[32] = rbuf[cc % kPerWait];
      const int nc = n0 + c * 32;
      if (nc >= p.N) continue;  // uniform for the warp
      // Bias + op in the TMEM layout (thread = row), packed to fp16.
      uint32_t pk[16];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int n = nc + 8 * g;
        float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
        if (n + 8 <= p.N) {
          b0 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
          b1 = __ldg(reinterpret_cast<const float4*>(p.bias + n) + 1);
        } else if (n < p.N) {  // last, partial group of an N that is not a multiple of 8
          float bb[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) bb[e] = n + e < p.N ? __ldg(p.bias + n + e) : 0.f;
          b0 = make_float4(bb[0], bb[1], bb[2], bb[3]);
          b1 = make_float4(bb[4], bb[5], bb[6], bb[7]);
        }
        float2 w[4] = {make_float2(__uint_as_float(r[8 * g + 0]) + b0.x, __uint_as_float(r[8 * g + 1]) + b0.y),
                       make_float2(__uint_as_float(r[8 * g + 2]) + b0.z, __uint_as_float(r[8 * g + 3]) + b0.w),
                       make_float2(__uint_as_float(r[8 * g + 4]) + b1.x, __uint_as_float(r[8 * g + 5]) + b1.y),
                       make_float2(__uint_as_float(r[8 * g + 6]) + b1.z, __uint_as_float(r[8 * g + 7]) + b1.w)};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (EPI == kEpiGeluF16) w[u] = gelu2(w[u]);
          pk[4 * g + u] = pack_half2(w[u].x, w[u].y);
        }
      }
      const int row = row_base + (int)lane;
      if (EPI == kEpiQkvHeadMajor && !hm_fast) {
        // Head dims that are not a multiple of 32: head-major addressing per
        // 8-column group (or per element), one row per thread; padding
        // columns up to 64 are zeroed by the writer of a head's last column.
        if (row < rows) {
          __half* qkv = static_cast<__half*>(p.out);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int n = nc + 8 * g;
            if (n >= p.N) break;
            if ((p.head_dim & 7) == 0) {
              const int which = n / p.d_model;
              const int rem = n - which * p.d_model;
              const int h = rem / p.head_dim;
              const int d = rem - h * p.head_dim;
              __half* rowp = qkv + ((int64_t)(which * p.heads + h) * p.rows_max + row) * p.head_pad;
              *reinterpret_cast<uint4*>(rowp + d) = make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
              if (d + 8 == p.head_dim)
                for (int z = p.head_dim; z < p.head_pad; z += 8)
                  *reinterpret_cast<uint4*>(rowp + z) = make_uint4(0u, 0u, 0u, 0u);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int ne = n + e;
                if (ne >= p.N) break;
                const int which = ne / p.d_model;
                const int rem = ne - which * p.d_model;
                const int h = rem / p.head_dim;
                const int d = rem - h * p.head_dim;
                __half* rowp = qkv + ((int64_t)(which * p.heads + h) * p.rows_max + row) * p.head_pad;
                const uint32_t bits = pk[4 * g + (e >> 1)] >> ((e & 1) * 16);
                rowp[d] = __ushort_as_half((unsigned short)(bits & 0xFFFFu));
                if (d + 1 == p.head_dim)
                  for (int z = p.head_dim; z < p.head_pad; ++z) rowp[z] = __float2half_rn(0.f);
              }
            }
          }
        }
        continue;
      }
      // Row-contiguous stores through the scratch: 32 rows x 64 bytes.
      const bool tma = tmC != nullptr && p.tma_store && row_base + 32 <= rows;  // uniform for the warp
      if (tmC != nullptr && p.tma_store) {
        if (lane == 0) bulk_wait_read();  // an earlier bulk store has read the scratch
        __syncwarp();
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        st_shared_v4(scratch + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4),
                     make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]));
      if (tma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (EPI == kEpiQkvHeadMajor) {
            // a 32-column chunk lies inside one head (head_dim == head_pad here)
            const int which = nc / p.d_model;
            const int rem = nc - which * p.d_model;
            const int h = rem / p.head_dim;
            tma_store_3d(tmC, scratch, rem - h * p.head_dim, row_base, which * p.heads + h);
          } else {
            tma_store_2d(tmC, scratch, nc, row_base);
          }
          bulk_commit();
        }
        continue;
      }
      __syncwarp();
      const uint32_t k = lane & 3;
      const int col = nc + 8 * (int)k;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t rr = (lane >> 2) + 8 * i;
        const uint4 v = ld_shared_v4(scratch + rr * 64 + ((k ^ ((rr >> 1) & 3)) << 4));
        const int orow = row_base + (int)rr;
        if (orow >= rows || col >= p.N) continue;
        if (EPI != kEpiQkvHeadMajor) {
          *reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + (int64_t)orow * p.ld_out + col) = v;
        } else {
          // A 32-column chunk lies inside one head (head_dim is a multiple of 32);
          // the writer of a head's last chunk zeroes its padding up to head_pad.
          const int which = nc / p.d_model;
          const int rem = nc - which * p.d_model;
          const int h = rem / p.head_dim;
          const int d0 = rem - h * p.head_dim;
          __half* rowp = static_cast<__half*>(p.out) +
                         ((int64_t)(which * p.heads + h) * p.rows_max + orow) * p.head_pad;
          *reinterpret_cast<uint4*>(rowp + d0 + 8 * (int)k) = v;
          if (d0 + 32 == p.head_dim)
            for (int z = p.head_dim + 8 * (int)k; z < p.head_pad; z += 32)
              *reinterpret_cast<uint4*>(rowp + z) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      __syncwarp();  // the next chunk reuses the scratch
    }
    return true;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(gemm_threads_for(BN, EPI), 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmKernelParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr int kEpiWarps = epi_warps_for(BN, EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  // bars: full[S], empty[S], tfull[2], tempty[2], final
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t scratch_base = smem_u32(reinterpret_cast<uint8_t*>(bars) + 256);

  const int warp = warp_idx();
  const uint32_t lane = lane_id();

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + S + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * S + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * S + 2 + a); };
  const uint32_t final_bar = smem_u32(bars + 2 * S + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kEpiWarps);
    }
    mbar_init(final_bar, 1);
    *abort_flag = device_failed() ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the row count, A and the residual come from earlier kernels

  const int rows = p.row_count ? min(p.rows_max, *p.row_count) : p.rows_max;
  const int m_tiles = (rows + kBM - 1) / kBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int total_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_parity[S];
      for (int s = 0; s < S; ++s) last_parity[s] = -1;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t / n_tiles) * kBM;
        const int n0 = (t % n_tiles) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, 100 + EPI)) break;
          mbar_arrive_expect_tx(full_bar(stage), Cfg::kStageBytes);
          tma_load_2d(smem_u32(sA + stage * Cfg::kABytes), &tmA, full_bar(stage), kb * kBK, m0);
          tma_load_2d(smem_u32(sB + stage * Cfg::kBBytes), &tmB, full_bar(stage), kb * kBK, n0);
          last_parity[stage] = (int)phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Let every issued load land before the CTA can exit.
      for (int s = 0; s < S; ++s)
        if (last_parity[s] >= 0) drain_wait(full_bar(s), (uint32_t)last_parity[s]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1, abort_flag, 110 + EPI)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, 120 + EPI)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = sw128_desc(smem_u32(sA + stage * Cfg::kABytes), 16, 1024);
          const uint64_t b_desc = sw128_desc(smem_u32(sB + stage * Cfg::kBBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per K=16 step inside the 128-byte swizzled row.
            mma_f16_ss(d_tmem, a_desc + (uint64_t)(2 * k), b_desc + (uint64_t)(2 * k), idesc,
                       (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          mma_commit(empty_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (issued) {
        mma_commit(final_bar);
        drain_wait(final_bar, 0);
      }
    }
  } else {
    // Epilogue warps: TMEM lane quarter = warp % 4; the kEpiWarps/4 warps of a
    // quarter split the tile's columns into slices.
    const int quarter = warp & 3;
    const int slice = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
      const int m0 = (t / n_tiles) * kBM;
      const int n0 = (t % n_tiles) * BN;
      if (!epilogue_tile<BN, EPI, kEpiWarps>(p, tmem_base + (uint32_t)(acc * BN), m0, n0, rows, quarter,
                                             slice, lane, tfull_bar(acc), acc_phase, abort_flag,
                                             scratch_base + (uint32_t)(warp - 2) * (kEpiScratchBytes / kEpiWarps)))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(tempty_bar(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant for large problems: a cluster of two CTAs (on two SMs)
// computes one 256 x 256 tile with tcgen05.mma.cta_group::2 (M=256, N=256).
// CTA r loads rows m0+128r.. of A and rows n0+128r.. of W (32 KB per K block
// instead of 48 KB for a 128 x 256 tile on one SM), which leaves room for six
// pipeline stages; its TMEM holds rows m0+128r.. of the accumulator for all
// 256 columns, so the epilogue is the one-CTA epilogue at BN=256.
//   - Both CTAs' TMA loads complete on the leader's (rank 0) full barrier;
//     the leader's producer expects the bytes of both.
//   - The leader's MMA lane issues the pair MMAs and commits, once to its own
//     barrier and once to the peer's, for the stage-empty and
//     accumulator-full events (no multicast).
//   - Each CTA's epilogue warps arrive on the leader's accumulator-empty
//     barrier (count 2 x epilogue warps).
// Every wait is bounded as in the one-CTA kernel; both CTAs meet at a cluster
// barrier before TMEM is freed, so neither leaves while the other can still
// touch its shared memory.
// ---------------------------------------------------------------------------
struct PairCfg {
  static constexpr int kBN = 256;
  static constexpr int kStages = 6;
  static constexpr uint32_t kABytes = kBM * kBK * 2;            // this CTA's 128 rows of A
  static constexpr uint32_t kBBytes = (kBN / 2) * kBK * 2;      // this CTA's 128 rows of W
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * kBN;
  static constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 256 + kEpiScratchBytes;
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm_threads_for(256, EPI), 1)
    gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, const GemmKernelParams p) {
  using Cfg = PairCfg;
  constexpr int S = Cfg::kStages;
  constexpr int BN = Cfg::kBN;
  constexpr int kEpiWarps = epi_warps_for(BN, EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  // epilogue scratch (1024-byte aligned: the bulk stores read it in the
  // 64-byte swizzle), then the barriers
  const uint32_t scratch_base = smem_u32(sB + S * Cfg::kBBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes + kEpiScratchBytes);
  // bars: full[S] (leader's used), empty[S], tfull[2], tempty[2] (leader's used), final
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_idx();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + S + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * S + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * S + 2 + a); };
  const uint32_t final_bar = smem_u32(bars + 2 * S + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * kEpiWarps);
    }
    mbar_init(final_bar, 1);
    *abort_flag = device_failed() ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  const int rows = p.row_count ? min(p.rows_max, *p.row_count) : p.rows_max;
  const int m_tiles = (rows + 2 * kBM - 1) / (2 * kBM);
  const int n_tiles = (p.N + BN - 1) / BN;
  const int total_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + kBK - 1) / kBK;
  const int cluster_id = (int)(blockIdx.x >> 1);
  const int num_clusters = (int)(gridDim.x >> 1);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_parity[S];
      for (int s = 0; s < S; ++s) last_parity[s] = -1;
      for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters) {
        const int m0 = (t / n_tiles) * (2 * kBM) + (int)rank * kBM;
        const int n0 = (t % n_tiles) * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, 140 + EPI)) break;
          if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * Cfg::kStageBytes);
          const uint32_t leader_full = mapa_shared(full_bar(stage), 0);
          tma_load_2d_pair(smem_u32(sA + stage * Cfg::kABytes), &tmA, leader_full, kb * kBK, m0);
          tma_load_2d_pair(smem_u32(sB + stage * Cfg::kBBytes), &tmB, leader_full, kb * kBK, n0);
          last_parity[stage] = (int)phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // The leader's full barriers count both CTAs' loads: once they have
      // completed, nothing either CTA issued is still landing.
      if (leader)
        for (int s = 0; s < S; ++s)
          if (last_parity[s] >= 0) drain_wait(full_bar(s), (uint32_t)last_parity[s]);
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * kBM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters) {
        if (!mbar_wait<true>(tempty_bar(acc), acc_phase ^ 1, abort_flag, 150 + EPI)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, 160 + EPI)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = sw128_desc(smem_u32(sA + stage * Cfg::kABytes), 16, 1024);
          const uint64_t b_desc = sw128_desc(smem_u32(sB + stage * Cfg::kBBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_ss_pair(d_tmem, a_desc + (uint64_t)(2 * k), b_desc + (uint64_t)(2 * k), idesc,
                            (kb | k) != 0 ? 1u : 0u);
          issued = true;
          mma_commit_pair(empty_bar(stage));
          mma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(tfull_bar(acc));
        mma_commit_pair(mapa_shared(tfull_bar(acc), 1));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (issued) {
        mma_commit_pair(final_bar);
        drain_wait(final_bar, 0);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int slice = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters) {
      const int m0 = (t / n_tiles) * (2 * kBM) + (int)rank * kBM;
      const int n0 = (t % n_tiles) * BN;
      if (!epilogue_tile<BN, EPI, kEpiWarps>(p, tmem_base + (uint32_t)(acc * BN), m0, n0, rows, quarter,
                                             slice, lane, tfull_bar(acc), acc_phase, abort_flag,
                                             scratch_base + (uint32_t)(warp - 2) * (kEpiScratchBytes / kEpiWarps),
                                             &tmC))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(tempty_bar(acc), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's bulk stores have landed
  }

  __syncwarp();
  pdl_trigger();
  tc_fence_before();
  cluster_sync();  // the peer no longer reads this CTA's shared memory or barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// fp16 tensor map of rank 2..5 with the given swizzle.  dims/strides are in
// elements, innermost first; strides has rank-1 entries (dims 1..rank-1).
static int make_tmap_f16_sw(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                            const uint64_t* strides_elems, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return set_error(TJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_elems[i] * 2;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void*>(base),
                  gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d) rank=%d", (int)r,
                     rank);
  return TJ_OK;
}

// fp16 tensor map of rank 2..5 with a 128-byte swizzle (the operand tiles).
int make_tmap_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_elems, const uint32_t* box) {
  return make_tmap_f16_sw(map, base, rank, dims, strides_elems, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN, int EPI>
static int launch_gemm_t(const GemmArgs& a, const GemmKernelParams& kp, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  uint64_t da[2] = {(uint64_t)a.K, (uint64_t)a.rows_max};
  uint64_t sa[1] = {(uint64_t)a.lda};
  uint32_t ba[2] = {kBK, kBM};
  int rc = make_tmap_f16(&ta, a.a16, 2, da, sa, ba);
  if (rc) return rc;
  uint64_t db[2] = {(uint64_t)a.K, (uint64_t)a.N};
  uint64_t sb[1] = {(uint64_t)a.ldw};
  uint32_t bb[2] = {kBK, (uint32_t)BN};
  rc = make_tmap_f16(&tb, a.w16, 2, db, sb, bb);
  if (rc) return rc;

  int num_sms = 0;
  rc = ensure_device_props(&num_sms);
  if (rc) return rc;
  static bool attr_set[64] = {};
  const int dev = device_index();
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tcgen05_kernel<BN, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::kSmemBytes);
    if (e != cudaSuccess)
      return set_error(TJ_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const int max_tiles = ((a.rows_max + kBM - 1) / kBM) * ((a.N + BN - 1) / BN);
  const int grid = max_tiles < num_sms ? max_tiles : num_sms;
  if (grid <= 0) return TJ_OK;
  cudaError_t e = launch_pdl(gemm_tcgen05_kernel<BN, EPI>, dim3(grid), dim3(gemm_threads_for(BN, EPI)),
                             Cfg::kSmemBytes, stream, ta, tb, kp);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

// Co-resident CTA-pair clusters of the pair kernel (0 if it cannot launch).
template <int EPI>
static int pair_clusters() {
  int num_sms = 0;
  if (ensure_device_props(&num_sms)) return 0;
  static int cache[64];
  static bool known[64] = {};
  const int dev = device_index();
  int& cached = cache[dev];
  if (known[dev]) return cached;
  known[dev] = true;
  cached = 0;
  if (cudaFuncSetAttribute(gemm_tcgen05_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)PairCfg::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return cached;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms & ~1);
  cfg.blockDim = dim3(gemm_threads_for(256, EPI));
  cfg.dynamicSmemBytes = PairCfg::kSmemBytes;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tcgen05_pair_kernel<EPI>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cached = n;
  return cached;
}

// TJ_GEMM_TMA_STORE=0 keeps the fp16 epilogues on st.global (for A/B timing).
static bool gemm_tma_store_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("TJ_GEMM_TMA_STORE");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

static bool pair_gemm_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("TJ_GEMM_PAIR");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

template <int EPI>
static int launch_gemm_pair(const GemmArgs& a, const GemmKernelParams& kp, int clusters,
                            cudaStream_t stream) {
  CUtensorMap ta, tb;
  uint64_t da[2] = {(uint64_t)a.K, (uint64_t)a.rows_max};
  uint64_t sa[1] = {(uint64_t)a.lda};
  uint32_t ba[2] = {kBK, kBM};
  int rc = make_tmap_f16(&ta, a.a16, 2, da, sa, ba);
  if (rc) return rc;
  uint64_t db[2] = {(uint64_t)a.K, (uint64_t)a.N};
  uint64_t sb[1] = {(uint64_t)a.ldw};
  uint32_t bb[2] = {kBK, (uint32_t)(PairCfg::kBN / 2)};
  rc = make_tmap_f16(&tb, a.w16, 2, db, sb, bb);
  if (rc) return rc;
  // fp16 outputs in whole 32 x 32 blocks leave through bulk tensor stores: the
  // QKV head-major layout when heads are not padded (head_dim = 64/128/256),
  // the plain [rows][ld_out] layout when N is a multiple of 32.
  GemmKernelParams kq = kp;
  CUtensorMap tc = ta;  // unused unless kq.tma_store
  kq.tma_store = 0;
  if (EPI == kEpiQkvHeadMajor && kp.head_dim == kp.head_pad) {
    uint64_t dc[3] = {(uint64_t)kp.head_pad, (uint64_t)a.rows_max, (uint64_t)(3 * kp.heads)};
    uint64_t sc[2] = {(uint64_t)kp.head_pad, (uint64_t)kp.head_pad * (uint64_t)a.rows_max};
    uint32_t bc[3] = {32, 32, 1};
    rc = make_tmap_f16_sw(&tc, a.out, 3, dc, sc, bc, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    kq.tma_store = 1;
  } else if ((EPI == kEpiBiasF16 || EPI == kEpiGeluF16) && a.N % 32 == 0) {
    uint64_t dc[2] = {(uint64_t)a.N, (uint64_t)a.rows_max};
    uint64_t sc[1] = {(uint64_t)a.ld_out};
    uint32_t bc[2] = {32, 32};
    rc = make_tmap_f16_sw(&tc, a.out, 2, dc, sc, bc, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    kq.tma_store = 1;
  }
  if (!gemm_tma_store_enabled()) kq.tma_store = 0;
  cudaError_t e = launch_pdl(gemm_tcgen05_pair_kernel<EPI>, dim3(2 * clusters),
                             dim3(gemm_threads_for(256, EPI)), PairCfg::kSmemBytes, stream, ta, tb, tc, kq);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "gemm pair launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

// 256-column tiles keep the operand traffic per FLOP low; when they would give
// fewer tiles than SMs (small batches), 64-column tiles spread the work (and
// the per-tile epilogue) over four times as many SMs.
template <int EPI>
static int launch_gemm_bn(const GemmArgs& a, const GemmKernelParams& kp, cudaStream_t stream) {
  int num_sms = 0;
  int rc = ensure_device_props(&num_sms);
  if (rc) return rc;
  const long long tiles256 = (long long)((a.rows_max + kBM - 1) / kBM) * ((a.N + 255) / 256);
  if (tiles256 < num_sms) return launch_gemm_t<64, EPI>(a, kp, stream);
  // 256 x 256 tiles on CTA pairs once there is at least a full wave of them.
  const long long pair_tiles = (long long)((a.rows_max + 2 * kBM - 1) / (2 * kBM)) * ((a.N + 255) / 256);
  const int clusters = pair_gemm_enabled() ? pair_clusters<EPI>() : 0;
  if (clusters > 0 && pair_tiles >= clusters)
    return launch_gemm_pair<EPI>(a, kp, clusters, stream);
  return launch_gemm_t<256, EPI>(a, kp, stream);
}

int launch_gemm(int epilogue, const GemmArgs& args, cudaStream_t stream) {
  GemmArgs a = args;
  if (a.lda <= 0) a.lda = a.K;
  if (a.ldw <= 0) a.ldw = a.K;
  if (a.rows_max < 0 || a.N <= 0 || a.K <= 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm: rows=%d N=%d K=%d", a.rows_max, a.N, a.K);
  // TMA rows are whole 16-byte units; a K that is not a multiple of 8 is read
  // through padded row strides (the tile loads zero-fill past K).
  if (a.lda < a.K || a.ldw < a.K || a.lda % 8 != 0 || a.ldw % 8 != 0)
    return set_error(TJ_ERR_UNSUPPORTED,
                     "gemm: K=%d needs row strides that are multiples of 8 and >= K (lda=%d ldw=%d)", a.K,
                     a.lda, a.ldw);
  if (!a.a16 || !a.w16 || !a.bias || !a.out)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm: null pointer");
  if ((reinterpret_cast<uintptr_t>(a.a16) | reinterpret_cast<uintptr_t>(a.w16) |
       reinterpret_cast<uintptr_t>(a.bias) | reinterpret_cast<uintptr_t>(a.out)) & 15u)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm: operands must be 16-byte aligned");
  if (a.rows_max == 0) return TJ_OK;
  GemmKernelParams kp{};
  kp.bias = a.bias;
  kp.row_count = a.row_count;
  kp.rows_max = a.rows_max;
  kp.N = a.N;
  kp.K = a.K;
  kp.out = a.out;
  kp.ld_out = a.ld_out;
  kp.resid = a.resid;
  kp.resid_map = a.resid_map;
  kp.ld_resid = a.ld_resid;
  kp.heads = a.heads;
  kp.head_dim = a.head_dim;
  switch (epilogue) {
    case kEpiQkvHeadMajor:
      if (a.heads <= 0 || a.head_dim <= 0 || a.head_dim > 256 || a.N != 3 * a.heads * a.head_dim)
        return set_error(TJ_ERR_UNSUPPORTED,
                         "gemm_qkv_headmajor: N=%d must be 3*H*dh with dh <= 256 (H=%d dh=%d)",
                         a.N, a.heads, a.head_dim);
      kp.d_model = a.heads * a.head_dim;
      kp.head_pad = attn_head_pad(a.head_dim);
      return launch_gemm_bn<kEpiQkvHeadMajor>(a, kp, stream);
    case kEpiResidualF32:
      if (a.N % 8 != 0)
        return set_error(TJ_ERR_UNSUPPORTED, "gemm_bias_residual_f32: N=%d must be a multiple of 8", a.N);
      if (!a.resid || (reinterpret_cast<uintptr_t>(a.resid) & 15u) || a.ld_resid % 4 != 0 ||
          a.ld_out % 4 != 0)
        return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm_bias_residual_f32: residual must be 16-byte aligned");
      return launch_gemm_bn<kEpiResidualF32>(a, kp, stream);
    // The fp16 epilogues store 8 columns at a time: a last partial group
    // writes zeros into the row padding, so the row stride must cover it.
    case kEpiGeluF16:
      if (a.ld_out % 8 != 0 || a.ld_out < (a.N + 7) / 8 * 8)
        return set_error(TJ_ERR_INVALID_ARGUMENT,
                         "gemm_bias_gelu_f16: ld_out=%d must be a multiple of 8 covering N=%d", a.ld_out, a.N);
      return launch_gemm_bn<kEpiGeluF16>(a, kp, stream);
    case kEpiBiasF16:
      if (a.ld_out % 8 != 0 || a.ld_out < (a.N + 7) / 8 * 8)
        return set_error(TJ_ERR_INVALID_ARGUMENT,
                         "gemm_bias_f16: ld_out=%d must be a multiple of 8 covering N=%d", a.ld_out, a.N);
      return launch_gemm_bn<kEpiBiasF16>(a, kp, stream);
    default:
      return set_error(TJ_ERR_INVALID_ARGUMENT, "gemm: unknown epilogue %d", epilogue);
  }
}

}  // namespace tj
