// Fused encoder for small models: one CTA runs every layer of one sample.
//
// The reference's official benchmark shapes are mostly 128-token sequences of
// a d_model-128 model over 4 layers (STATEMENT.md 3.7; tools/matrix_runner.py:49-64).
// There each of the ~30 kernels of the layer-by-layer path lasts a few
// microseconds and the forward is bound by their latency.  Here one CTA holds
// one sample (S <= 128 tokens = one 128-row MMA tile) through all layers:
// the fp32 residual stream stays in registers, every GEMM is a tcgen05 MMA
// from shared memory into TMEM, attention runs head by head on the same
// tile, and only the input, the weights and the output touch global memory.
// It computes exactly what tj_encoder_forward computes (same roundings: fp16
// GEMM operands, fp32 accumulation, fp16 projection outputs added to the fp32
// stream, erf-GELU on the fp32 accumulator, fp32 LayerNorm and softmax), for
// v16_1_clean.py:599-628 with S <= 128, d_model <= 128, ffn_dim <= 128.
//
// Threads: 256 = 8 warps.  Thread (warp w, lane) owns token row
// r = 32*(w%4) + lane (= its TMEM lane) and column half w/4 of every row-wise
// result; the two halves of a row meet through shared memory for row
// statistics (LayerNorm mean/variance, softmax max/sum).
//
// TMEM (512 columns): [0, 384) the QKV accumulator of a head group (q | k | v,
// each head padded to dhp = round_up(head_dim, 16) columns), later the
// projection/FFN accumulators and each head's P.V output (written over the
// head's q columns, already copied out); [384, 512) the head's scores S, then
// P (fp16 pairs) over S's first 64 columns.
//
// Shared memory (all MMA operands K-major, 128-byte swizzle, 64-column
// chunks of 128 rows = 16 KB): A (LayerNorm output / FFN hidden), ctx
// (attention output, the out-projection's A), Q_h and K_h of the current
// head, V_h^T ([dhp][128 keys], the P.V B operand), and two weight buffers.
// Weights stream from global (L2-resident: every CTA reads the same ones) in
// units of at most 128 rows x 128 columns with cp.async into the swizzled
// layout, the next unit in flight while the current one multiplies.
//
// Every phase is synchronous inside the CTA (MMA issue by one thread, commit
// to an mbarrier, all threads wait); the waits are bounded like every other
// wait of the library.
#include "common.cuh"
#include "internal.h"

namespace tj {

constexpr int kSmallThreads = 256;
constexpr int kSmallMaxLayers = 8;
constexpr uint32_t kSmallChunk = 128 * 128;  // one 64-column chunk of 128 rows, bytes
constexpr uint32_t kSmallWBuf = 2 * kSmallChunk;  // <= 128 weight rows x 128 columns
constexpr uint32_t kSmallSCol = 384;  // TMEM column of S / P

struct SmallEncParams {
  const float* x;
  const uint8_t* mask;
  float* out;
  int S, D, H, F, L, causal;
  float eps;
  int dh, dhp, G;        // head dim, padded to 16, heads per QKV group
  int qkv_units;         // weight units of the QKV GEMMs of one layer (all groups)
  int units_per_layer;   // qkv_units + 3 (out-proj, FFN-in, FFN-out)
  float scale_log2;
  const float* final_gamma;
  const float* final_beta;
  tj_layer_weights layers[kSmallMaxLayers];
};

__host__ __device__ inline int small_round16(int v) { return (v + 15) / 16 * 16; }

// Byte offset of (row, column) in a K-major, 128-byte-swizzled operand whose
// 64-column chunks of `rows` rows are `rows * 128` bytes apart.
__device__ __forceinline__ uint32_t sw_off(int row, int col, int rows) {
  return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// 32 lanes x 8 consecutive 32-bit columns (thread i: lane 32*(warp%4) + i).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// What one weight unit multiplies: rows [n0, n0 + nrows) of a virtual weight
// matrix, K columns, written to TMEM column acc_col.
struct SmallUnit {
  const __half* w;   // fp16 [*, ldw] (nn.Linear layout, rows padded to 8 columns)
  int ldw, K, nrows, kind;  // kind 0: QKV piece, 1: out-proj, 2: FFN-in, 3: FFN-out
  int n0, group, acc_col;
};

__device__ __forceinline__ SmallUnit small_unit(const SmallEncParams& p, int u) {
  SmallUnit su;
  const int layer = u / p.units_per_layer;
  int k = u - layer * p.units_per_layer;
  const tj_layer_weights& L = p.layers[layer < p.L ? layer : p.L - 1];
  const int D8 = (p.D + 7) & ~7, F8 = (p.F + 7) & ~7;
  su.n0 = 0;
  su.group = 0;
  su.acc_col = 0;
  if (k < p.qkv_units) {
    // QKV pieces, group by group: 128 rows of the group's [q | k | v] matrix each
    int g = 0;
    for (;; ++g) {
      const int gh = min(p.G, p.H - g * p.G);
      const int pieces = (3 * gh * p.dhp + 127) / 128;
      if (k < pieces) {
        su.kind = 0;
        su.group = g;
        su.n0 = 128 * k;
        su.nrows = min(128, 3 * gh * p.dhp - 128 * k);
        su.acc_col = 128 * k;
        break;
      }
      k -= pieces;
    }
    su.w = static_cast<const __half*>(L.w_qkv16);
    su.ldw = D8;
    su.K = p.D;
  } else {
    k -= p.qkv_units;
    su.kind = 1 + k;
    if (k == 0) {
      su.w = static_cast<const __half*>(L.w_out16), su.ldw = D8, su.K = p.D, su.nrows = small_round16(p.D);
    } else if (k == 1) {
      su.w = static_cast<const __half*>(L.w_ffn_in16), su.ldw = D8, su.K = p.D, su.nrows = small_round16(p.F);
    } else {
      su.w = static_cast<const __half*>(L.w_ffn_out16), su.ldw = F8, su.K = p.F, su.nrows = small_round16(p.D);
    }
  }
  return su;
}

// Source row of local row n of a unit (-1 = a zero row).
__device__ __forceinline__ int small_src_row(const SmallEncParams& p, const SmallUnit& su, int n) {
  if (su.kind == 0) {
    const int gh = min(p.G, p.H - su.group * p.G);
    const int m = su.n0 + n;
    const int part = m / (gh * p.dhp);
    const int within = m - part * gh * p.dhp;
    const int hh = within / p.dhp, d = within - hh * p.dhp;
    return d < p.dh ? part * p.D + (su.group * p.G + hh) * p.dh + d : -1;
  }
  const int N = su.kind == 2 ? p.F : p.D;
  return n < N ? n : -1;
}

// All threads: cp.async of unit u into weight buffer u % 2 (an empty group
// past the last unit, so every thread always has exactly two groups to track).
__device__ __forceinline__ void small_load_unit(const SmallEncParams& p, int u, int total, uint8_t* sW) {
  if (u < total) {
    const SmallUnit su = small_unit(p, u);
    uint8_t* buf = sW + (u & 1) * kSmallWBuf;
    const int kchunks = (su.K + 63) / 64;
    const int granules = su.nrows * 8 * kchunks;
    for (int i = threadIdx.x; i < granules; i += kSmallThreads) {
      const int n = i / (8 * kchunks), j = i - n * 8 * kchunks;  // j: 8-column granule of the row
      const int col = 8 * j;
      const int src_row = small_src_row(p, su, n);
      const bool ok = src_row >= 0 && col < ((su.K + 7) & ~7);
      const __half* src = ok ? su.w + (size_t)src_row * su.ldw + col : su.w;
      cp_async16(smem_u32(buf + sw_off(n, col, su.nrows)), src, ok ? 16 : 0);
    }
  }
  cp_async_commit();
}

// One thread: D[tmem] = A[128 x K] * W[nrows x K]^T, both from shared memory.
__device__ __forceinline__ void small_mma_ss(uint32_t d_tmem, uint32_t a_base, uint32_t b_base, int nrows,
                                             int K) {
  const uint32_t idesc = idesc_f16_f32(128, nrows, 0, 0);
  const int ksteps = (K + 15) / 16;
  for (int s = 0; s < ksteps; ++s) {
    const int c = s >> 2, k = s & 3;
    const uint64_t a = sw128_desc(a_base + c * kSmallChunk, 16, 1024) + (uint64_t)(2 * k);
    const uint64_t b = sw128_desc(b_base + c * nrows * 128, 16, 1024) + (uint64_t)(2 * k);
    mma_f16_ss(d_tmem, a, b, idesc, s > 0 ? 1u : 0u);
  }
}

// Sum of v over the two threads of a row (column halves), through xchg.
__device__ __forceinline__ float small_row_sum(float v, float* xchg, int row, int half) {
  xchg[half * 128 + row] = v;
  __syncthreads();
  const float s = xchg[row] + xchg[128 + row];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float small_row_max(float v, float* xchg, int row, int half) {
  xchg[half * 128 + row] = v;
  __syncthreads();
  const float s = fmaxf(xchg[row], xchg[128 + row]);
  __syncthreads();
  return s;
}

// LayerNorm of the thread's half row xr (columns half*64 + [0, 64), real
// below D) -> fp16 into the K-major operand `dst` (zeros past D).
__device__ __forceinline__ void small_layernorm_f16(const float (&xr)[64], const float* gamma, const float* beta,
                                                    int D, float eps, int row, int half, float* xchg,
                                                    uint8_t* dst) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < 64; ++c)
    if (half * 64 + c < D) s += xr[c];
  const float mean = small_row_sum(s, xchg, row, half) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < 64; ++c)
    if (half * 64 + c < D) {
      const float d = xr[c] - mean;
      q += d * d;
    }
  const float rstd = 1.0f / sqrtf(small_row_sum(q, xchg, row, half) / (float)D + eps);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int c0 = half * 64 + 8 * g;
    if (c0 >= ((D + 15) & ~15)) break;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + 2 * e;
      const float a = c < D ? (xr[8 * g + 2 * e] - mean) * rstd * gamma[c] + beta[c] : 0.f;
      const float b = c + 1 < D ? (xr[8 * g + 2 * e + 1] - mean) * rstd * gamma[c + 1] + beta[c + 1] : 0.f;
      w[e] = pack_half2(a, b);
    }
    *reinterpret_cast<uint4*>(dst + sw_off(row, c0, 128)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void __launch_bounds__(kSmallThreads, 1) small_encoder_kernel(const __grid_constant__ SmallEncParams p) {
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int qch = p.dhp > 64 ? 2 : 1;  // 64-column chunks of Q_h / K_h
  uint8_t* sA = smem;                            // 2 chunks
  uint8_t* sCtx = sA + 2 * kSmallChunk;          // 2 chunks
  uint8_t* sQ = sCtx + 2 * kSmallChunk;          // qch chunks
  uint8_t* sK = sQ + qch * kSmallChunk;          // qch chunks
  uint8_t* sVt = sK + qch * kSmallChunk;         // 2 chunks of dhp rows (128 keys)
  uint8_t* sW = sVt + 2 * p.dhp * 128;           // 2 weight buffers
  float* xchg = reinterpret_cast<float*>(sW + 2 * kSmallWBuf);  // [2][128]
  uint8_t* sMask = reinterpret_cast<uint8_t*>(xchg + 256);      // [128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sMask + 128);
  const uint32_t mma_bar = smem_u32(bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int b = blockIdx.x;
  const int warp = warp_idx();
  const int lane = (int)lane_id();
  const int row = 32 * (warp & 3) + lane;
  const int half = warp >> 2;
  const int S = p.S, D = p.D;
  const int total_units = p.units_per_layer * p.L;

  if (threadIdx.x == 0) {
    mbar_init(mma_bar, 1);
    *abort_flag = device_failed() ? 1 : 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 128)
    sMask[threadIdx.x] = (threadIdx.x < S && (p.mask == nullptr || p.mask[(size_t)b * S + threadIdx.x] != 0)) ? 1 : 0;
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  small_load_unit(p, 0, total_units, sW);
  small_load_unit(p, 1, total_units, sW);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
  const bool row_valid = sMask[row] != 0;
  uint32_t mma_phase = 0;
  bool ok = *abort_flag == 0;

  // The residual stream: this thread's half row, fp32 (columns past D stay 0).
  float xr[64];
  {
    const float* xrow = p.x + ((size_t)b * S + row) * D;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const int col = half * 64 + c;
      xr[c] = (row < S && col < D) ? xrow[col] : 0.f;
    }
  }

  // MMA by one thread, then everyone waits for it.
  // `ok` stays CTA-uniform, so an abort leaves every thread on the same path.
  // Thread 0 counts the phases it committed and the ones it saw complete.
  int n_commit = 0, n_done = 0;
  auto mma_wait = [&](int site) {
    bool mine = ok && mbar_wait(mma_bar, mma_phase, abort_flag, site);
    if (threadIdx.x == 0 && mine) ++n_done;
    mma_phase ^= 1u;
    tc_fence_after();
    ok = __syncthreads_and(mine ? 1 : 0) != 0;
  };
  // Weight unit u is in buffer u % 2 once every thread's copies have landed.
  auto unit_ready = [&]() {
    cp_async_wait1();
    fence_proxy_async_smem();
    __syncthreads();
  };

  int u = 0;
  for (int layer = 0; layer < p.L && ok; ++layer) {
    const tj_layer_weights& Lw = p.layers[layer];
    // ---- LN1 -> A
    small_layernorm_f16(xr, Lw.ln1_gamma, Lw.ln1_beta, D, p.eps, row, half, xchg, sA);
    fence_proxy_async_smem();
    // ---- attention, head group by head group
    for (int g = 0; g * p.G < p.H && ok; ++g) {
      const int gh = min(p.G, p.H - g * p.G);
      const int pieces = (3 * gh * p.dhp + 127) / 128;
      for (int pc = 0; pc < pieces; ++pc, ++u) {
        unit_ready();
        if (threadIdx.x == 0 && ok) {
          tc_fence_after();
          const SmallUnit su = small_unit(p, u);
          small_mma_ss(tmem + (uint32_t)su.acc_col, smem_u32(sA), smem_u32(sW + (u & 1) * kSmallWBuf), su.nrows,
                       su.K);
          mma_commit(mma_bar);
          ++n_commit;
        }
        mma_wait(300);
        small_load_unit(p, u + 2, total_units, sW);
      }
      for (int hh = 0; hh < gh && ok; ++hh) {
        const int head = g * p.G + hh;
        // ---- Q_h, K_h, V_h^T (+bias, fp16) from the accumulator into shared memory
        const int hw = p.dhp / 2;  // columns of the head per thread
        for (int part = 0; part < 3; ++part) {
          const int col0 = part * gh * p.dhp + hh * p.dhp + half * hw;
          const float* bias = Lw.b_qkv + part * D + head * p.dh;
          for (int c0 = 0; c0 < hw; c0 += 8) {
            uint32_t v[8];
            tmem_ld8(t_lane + (uint32_t)(col0 + c0), v);
            tmem_ld_wait();
            const int d0 = half * hw + c0;  // column inside the padded head
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int d = d0 + i;
              f[i] = (row_valid && d < p.dh) ? __uint_as_float(v[i]) + bias[d] : 0.f;
            }
            if (part < 2) {
              uint8_t* dst = part == 0 ? sQ : sK;
              *reinterpret_cast<uint4*>(dst + sw_off(row, d0, 128)) =
                  make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                             pack_half2(f[6], f[7]));
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                *reinterpret_cast<__half*>(sVt + sw_off(d0 + i, row, p.dhp)) = __float2half_rn(f[i]);
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- S = Q_h K_h^T
        if (threadIdx.x == 0 && ok) {
          tc_fence_after();
          small_mma_ss(tmem + kSmallSCol, smem_u32(sQ), smem_u32(sK), 128, p.dhp);
          mma_commit(mma_bar);
          ++n_commit;
        }
        mma_wait(301);
        if (!ok) break;
        // ---- softmax over the row's keys (this thread: keys half*64 + [0, 64))
        float pf[64];
        {
          uint32_t sv[32];
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 32) {
            tmem_ld32(t_lane + kSmallSCol + (uint32_t)(half * 64 + c0), sv);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int key = half * 64 + c0 + i;
              const bool valid = key < S && sMask[key] && (!p.causal || key <= row);
              pf[c0 + i] = valid ? __uint_as_float(sv[i]) * p.scale_log2 : -INFINITY;
            }
          }
        }
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) m = fmaxf(m, pf[i]);
        m = small_row_max(m, xchg, row, half);  // also: every S load of the CTA is done
        const float mu = m == -INFINITY ? 0.f : m;
        float l = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e0 = exp2_approx(pf[2 * i] - mu), e1 = exp2_approx(pf[2 * i + 1] - mu);
          l += e0 + e1;
          pk[i] = pack_half2(e0, e1);
        }
        tmem_st32(t_lane + kSmallSCol + (uint32_t)(half * 32), pk);
        tmem_st_wait();
        xchg[half * 128 + row] = l;
        tc_fence_before();
        __syncthreads();
        const float lsum = xchg[row] + xchg[128 + row];
        // ---- O_h = P V_h, over the head's q columns of the accumulator
        const uint32_t o_col = (uint32_t)(hh * p.dhp);
        if (threadIdx.x == 0 && ok) {
          tc_fence_after();
          const uint32_t idesc = idesc_f16_f32(128, p.dhp, 0, 0);
#pragma unroll 1
          for (int k = 0; k < 8; ++k) {  // 128 keys, K = 16 per MMA
            const uint64_t bdesc = sw128_desc(smem_u32(sVt) + (k >> 2) * p.dhp * 128, 16, 1024) + (uint64_t)(2 * (k & 3));
            mma_f16_ts(tmem + o_col, tmem + kSmallSCol + (uint32_t)(8 * k), bdesc, idesc, k > 0 ? 1u : 0u);
          }
          mma_commit(mma_bar);
          ++n_commit;
        }
        mma_wait(302);
        if (!ok) break;
        // ---- ctx columns head*dh + [0, dh): O / l, fp16
        {
          const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
          for (int c0 = 0; c0 < hw; c0 += 8) {
            uint32_t v[8];
            tmem_ld8(t_lane + o_col + (uint32_t)(half * hw + c0), v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int d = half * hw + c0 + i;
              if (d < p.dh)
                *reinterpret_cast<__half*>(sCtx + sw_off(row, head * p.dh + d, 128)) =
                    __float2half_rn(__uint_as_float(v[i]) * inv);
            }
          }
        }
        tc_fence_before();
        __syncthreads();  // Q_h/K_h/V_h and S are free for the next head
      }
    }
    if (!ok) break;
    // zero ctx columns past D up to the MMA's K (a multiple of 16)
    for (int c = D + half; c < ((D + 15) & ~15); c += 2)
      *reinterpret_cast<__half*>(sCtx + sw_off(row, c, 128)) = __float2half_rn(0.f);
    fence_proxy_async_smem();
    // ---- out-projection: x += fp16(ctx Wo^T + bo)
    unit_ready();
    if (threadIdx.x == 0 && ok) {
      tc_fence_after();
      const SmallUnit su = small_unit(p, u);
      small_mma_ss(tmem, smem_u32(sCtx), smem_u32(sW + (u & 1) * kSmallWBuf), su.nrows, su.K);
      mma_commit(mma_bar);
      ++n_commit;
    }
    mma_wait(303);
    small_load_unit(p, u + 2, total_units, sW);
    ++u;
    if (!ok) break;
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      uint32_t v[32];
      tmem_ld32(t_lane + (uint32_t)(half * 64 + c0), v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = half * 64 + c0 + i;
        if (col < D) xr[c0 + i] += __half2float(__float2half_rn(__uint_as_float(v[i]) + Lw.b_out[col]));
      }
    }
    tc_fence_before();
    // ---- LN2 -> A
    small_layernorm_f16(xr, Lw.ln2_gamma, Lw.ln2_beta, D, p.eps, row, half, xchg, sA);
    fence_proxy_async_smem();
    // ---- FFN-in + erf-GELU -> A (the hidden layer, F columns)
    unit_ready();
    if (threadIdx.x == 0 && ok) {
      tc_fence_after();
      const SmallUnit su = small_unit(p, u);
      small_mma_ss(tmem, smem_u32(sA), smem_u32(sW + (u & 1) * kSmallWBuf), su.nrows, su.K);
      mma_commit(mma_bar);
      ++n_commit;
    }
    mma_wait(304);
    small_load_unit(p, u + 2, total_units, sW);
    ++u;
    if (!ok) break;
    {
      const int Fp = small_round16(p.F);
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(t_lane + (uint32_t)(half * 64 + c0), v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          const int col = half * 64 + c0 + e;
          if (col >= Fp) break;
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int ca = col + 2 * i;
            float2 a = make_float2(ca < p.F ? __uint_as_float(v[e + 2 * i]) + Lw.b_ffn_in[ca] : 0.f,
                                   ca + 1 < p.F ? __uint_as_float(v[e + 2 * i + 1]) + Lw.b_ffn_in[ca + 1] : 0.f);
            a = gelu2(a);
            w[i] = pack_half2(a.x, a.y);
          }
          *reinterpret_cast<uint4*>(sA + sw_off(row, col, 128)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    // ---- FFN-out: x += fp16(h W2^T + b2); padded rows of x become 0
    unit_ready();
    if (threadIdx.x == 0 && ok) {
      tc_fence_after();
      const SmallUnit su = small_unit(p, u);
      small_mma_ss(tmem, smem_u32(sA), smem_u32(sW + (u & 1) * kSmallWBuf), su.nrows, su.K);
      mma_commit(mma_bar);
      ++n_commit;
    }
    mma_wait(305);
    small_load_unit(p, u + 2, total_units, sW);
    ++u;
    if (!ok) break;
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      uint32_t v[32];
      tmem_ld32(t_lane + (uint32_t)(half * 64 + c0), v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = half * 64 + c0 + i;
        if (col < D) xr[c0 + i] += __half2float(__float2half_rn(__uint_as_float(v[i]) + Lw.b_ffn_out[col]));
      }
    }
#pragma unroll
    for (int c = 0; c < 64; ++c)
      if (!row_valid) xr[c] = 0.f;
    tc_fence_before();
  }

  // ---- final LayerNorm (fp32) and store; padded rows are exact zeros
  if (ok) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < 64; ++c)
      if (half * 64 + c < D) s += xr[c];
    const float mean = small_row_sum(s, xchg, row, half) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < 64; ++c)
      if (half * 64 + c < D) {
        const float d = xr[c] - mean;
        q += d * d;
      }
    const float rstd = 1.0f / sqrtf(small_row_sum(q, xchg, row, half) / (float)D + p.eps);
    if (row < S) {
      float* orow = p.out + ((size_t)b * S + row) * D;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int col = half * 64 + c;
        if (col < D) orow[col] = row_valid ? (xr[c] - mean) * rstd * p.final_gamma[col] + p.final_beta[col] : 0.f;
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  pdl_trigger();
  // Every MMA issued has completed before TMEM is released, also after an
  // abort (a wait that gave up may have left one in flight).
  if (threadIdx.x == 0) {
    mma_commit(mma_bar);  // one more phase, after every MMA issued so far
    const unsigned long long t0 = globaltimer_ns();
    for (int ph = n_done; ph <= n_commit; ++ph)  // phases complete in order
      while (!mbar_try_wait(mma_bar, (uint32_t)(ph & 1)) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Off by default: the single-CTA path is still slower than the layer-by-layer
// kernels on the shapes measured (its per-sample latency is not yet hidden).
static bool g_small_enabled = false;

bool small_encoder_fits(const tj_encoder_desc* d) {
  if (!g_small_enabled) return false;
  const int dh = d->d_model / d->num_heads;
  return d->seq_len <= 128 && d->d_model <= 128 && d->ffn_dim <= 128 && dh <= 128 &&
         d->num_layers <= kSmallMaxLayers && d->batch <= 2147483647;
}

int set_small_encoder(int enabled) {
  const int prev = g_small_enabled ? 1 : 0;
  g_small_enabled = enabled != 0;
  return prev;
}

size_t small_encoder_smem(int dhp) {
  const int qch = dhp > 64 ? 2 : 1;
  return 1024 + (size_t)(2 + 2 + 2 * qch) * kSmallChunk + 2 * (size_t)dhp * 128 + 2 * kSmallWBuf + 256 * 4 + 128 + 64;
}

int launch_small_encoder(const tj_encoder_desc* d, const tj_layer_weights* layers, const float* final_gamma,
                         const float* final_beta, const float* x, const uint8_t* mask, float* out,
                         cudaStream_t stream) {
  SmallEncParams p{};
  p.x = x;
  p.mask = mask;
  p.out = out;
  p.S = d->seq_len;
  p.D = d->d_model;
  p.H = d->num_heads;
  p.F = d->ffn_dim;
  p.L = d->num_layers;
  p.causal = d->causal;
  p.eps = d->ln_eps;
  p.dh = d->d_model / d->num_heads;
  p.dhp = small_round16(p.dh);
  p.G = 384 / (3 * p.dhp);
  if (p.G > p.H) p.G = p.H;
  if (p.G < 1) return set_error(TJ_ERR_UNSUPPORTED, "small encoder: head dim %d", p.dh);
  p.qkv_units = 0;
  for (int g = 0; g * p.G < p.H; ++g) {
    const int gh = p.G < p.H - g * p.G ? p.G : p.H - g * p.G;
    p.qkv_units += (3 * gh * p.dhp + 127) / 128;
  }
  p.units_per_layer = p.qkv_units + 3;
  p.scale_log2 = (1.0f / sqrtf((float)p.dh)) * 1.4426950408889634f;
  p.final_gamma = final_gamma;
  p.final_beta = final_beta;
  for (int l = 0; l < p.L; ++l) p.layers[l] = layers[l];
  const size_t smem = small_encoder_smem(p.dhp);
  static bool attr_set[64] = {};
  const int dev = device_index();
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(small_encoder_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)small_encoder_smem(128));
    if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "small encoder smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  cudaError_t e = launch_pdl(small_encoder_kernel, dim3(d->batch), dim3(kSmallThreads), smem, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "small encoder launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

}  // namespace tj
