// Masked flash attention forward on tcgen05 (head_dim 64), replacing the SDPA
// call of v16_1_clean.py:505-514 (and the explicit softmax(QK^T*scale)V of the
// FP32 reference, torch_transformer_benchmark.py:97-117).
//
// Queries and keys are compact: the token plan packs the valid tokens of each
// sample densely, so a sample's keys are the rows [off, off+len) of its key
// segment(s) and padded keys never enter the loop.  A sample may have several
// key segments (context parallelism: one per rank, gathered by NCCL); they are
// walked in order as one key sequence.
//
// One CTA per (128-query tile, head, sample), 192 threads:
//   warp 0      TMA: Q once, then K and V tiles of 128 keys into a 3-stage ring
//   warp 1      TMEM allocation; one lane issues S_j = Q K_j^T (M=128,N=128,
//               K=16 x4) into one of two TMEM S buffers, and O_j = P_j V_j
//               (M=128,N=64,K=16 x8) into one of two TMEM O buffers
//   warps 2-5   softmax: thread = query row = TMEM lane.  Reads S_j, keeps the
//               running max/sum in fp32 (exp2 domain), writes P_j in fp16 to a
//               128-byte-swizzled shared tile, and folds O_{j-1} into a
//               register accumulator while the tensor core works on P_j V_j.
// The S_{j+1} product is issued before P_j V_j, so the tensor core computes the
// next scores while the softmax warps work on the current tile.
//
// Key rows of the last tile past the segment end are masked to -inf and the
// matching V rows are zeroed in shared memory before P V, so whatever the
// buffer holds past the segment (another sample's rows, stale memory) cannot
// reach the output even as 0 * NaN.
#include "common.cuh"
#include "internal.h"

namespace tj {

int make_tmap_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_elems, const uint32_t* box);

constexpr int kAttnThreads = 192;
constexpr int kAttnBM = 128;     // queries per CTA
constexpr int kAttnBN = 128;     // keys per tile
constexpr int kDH = 64;          // head dim
constexpr int kKVStages = 3;
constexpr uint32_t kQBytes = kAttnBM * kDH * 2;   // 16 KB
constexpr uint32_t kKVBytes = kAttnBN * kDH * 2;  // 16 KB
constexpr uint32_t kPBytes = kAttnBM * kAttnBN * 2;  // 32 KB (two 64-key swizzle atoms)
constexpr size_t kAttnSmem = 1024 + kQBytes + 2 * kKVStages * kKVBytes + 2 * kPBytes + 512;
constexpr uint32_t kAttnTmemCols = 512;  // S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384)

struct AttnKernelParams {
  int H, B, G;
  const int32_t* q_cu;
  const int32_t* kv_off;
  const int32_t* kv_len;
  int64_t kv_len_stride;
  float scale_log2;
  int causal;
  const int32_t* q_pos0;
  __half* ctx;
  int ld_ctx;
};

// Walks the key tiles of one sample in order: segment g, tile i inside it.
// All three roles walk the same sequence, so tile j means the same keys to each.
struct KvWalk {
  const int32_t* off;
  const int32_t* len;
  int G;
  int g, i, seg_len, seg_off, pos_base;  // pos_base = key position of segment start
  __device__ void init(const int32_t* o, const int32_t* l, int G_) {
    off = o;
    len = l;
    G = G_;
    g = 0;
    i = 0;
    pos_base = 0;
    load_segment();
  }
  __device__ void load_segment() {
    while (g < G && len[g] <= 0) ++g;
    if (g < G) {
      seg_len = len[g];
      seg_off = off[g];
    }
  }
  __device__ int row() const { return seg_off + i * kAttnBN; }
  __device__ int valid() const { return min(kAttnBN, seg_len - i * kAttnBN); }
  __device__ int first_pos() const { return pos_base + i * kAttnBN; }
  __device__ void next() {
    if (g >= G) return;
    ++i;
    if (i * kAttnBN >= seg_len) {
      pos_base += seg_len;
      ++g;
      i = 0;
      load_segment();
    }
  }
};

__device__ __forceinline__ int count_kv_tiles(const int32_t* len, int G) {
  int t = 0;
  for (int g = 0; g < G; ++g) {
    const int l = len[g];
    if (l > 0) t += (l + kAttnBN - 1) / kAttnBN;
  }
  return t;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_tcgen05_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const AttnKernelParams p) {
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q_begin = p.q_cu[b];
  const int nq = p.q_cu[b + 1] - q_begin;
  if (qt * kAttnBM >= nq) return;  // uniform for the CTA
  const int32_t* kv_off = p.kv_off + (int64_t)b * p.kv_len_stride;
  const int32_t* kv_len = p.kv_len + (int64_t)b * p.kv_len_stride;
  const int T = count_kv_tiles(kv_len, p.G);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;
  uint8_t* sV = sK + kKVStages * kKVBytes;
  uint8_t* sP = sV + kKVStages * kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  // q_full, k_full[3], v_full[3], k_empty[3], v_empty[3], s_full[2], s_empty[2],
  // p_full[2], p_empty[2], o_full[2], o_empty[2], final
  const uint32_t q_full = smem_u32(bars + 0);
  auto k_full = [&](int s) { return smem_u32(bars + 1 + s); };
  auto v_full = [&](int s) { return smem_u32(bars + 4 + s); };
  auto k_empty = [&](int s) { return smem_u32(bars + 7 + s); };
  auto v_empty = [&](int s) { return smem_u32(bars + 10 + s); };
  auto s_full = [&](int i) { return smem_u32(bars + 13 + i); };
  auto s_empty = [&](int i) { return smem_u32(bars + 15 + i); };
  auto p_full = [&](int i) { return smem_u32(bars + 17 + i); };
  auto p_empty = [&](int i) { return smem_u32(bars + 19 + i); };
  auto o_full = [&](int i) { return smem_u32(bars + 21 + i); };
  auto o_empty = [&](int i) { return smem_u32(bars + 23 + i); };
  const uint32_t final_bar = smem_u32(bars + 25);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_idx();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_empty(i), 4);
      mbar_init(p_full(i), 4);
      mbar_init(p_empty(i), 1);
      mbar_init(o_full(i), 1);
      mbar_init(o_empty(i), 4);
    }
    mbar_init(final_bar, 1);
    *abort_flag = device_failed() ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int last_k[kKVStages], last_v[kKVStages];
      for (int s = 0; s < kKVStages; ++s) last_k[s] = last_v[s] = -1;
      bool q_issued = false;
      if (!*abort_flag) {
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_3d(smem_u32(sQ), &tmQ, q_full, 0, q_begin + qt * kAttnBM, h);
        q_issued = true;
      }
      KvWalk w;
      w.init(kv_off, kv_len, p.G);
      for (int j = 0; j < T && !*abort_flag; ++j, w.next()) {
        const int s = j % kKVStages;
        const uint32_t ph = (uint32_t)((j / kKVStages) & 1);
        if (!mbar_wait(k_empty(s), ph ^ 1, abort_flag, 200)) break;
        mbar_arrive_expect_tx(k_full(s), kKVBytes);
        tma_load_4d(smem_u32(sK + s * kKVBytes), &tmK, k_full(s), 0, w.row(), h, w.g);
        last_k[s] = (int)ph;
        if (!mbar_wait(v_empty(s), ph ^ 1, abort_flag, 201)) break;
        mbar_arrive_expect_tx(v_full(s), kKVBytes);
        tma_load_4d(smem_u32(sV + s * kKVBytes), &tmV, v_full(s), 0, w.row(), h, w.g);
        last_v[s] = (int)ph;
      }
      if (q_issued) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
      for (int s = 0; s < kKVStages; ++s) {
        const unsigned long long t0 = globaltimer_ns();
        if (last_k[s] >= 0)
          while (!mbar_try_wait(k_full(s), (uint32_t)last_k[s]) &&
                 globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        if (last_v[s] >= 0)
          while (!mbar_try_wait(v_full(s), (uint32_t)last_v[s]) &&
                 globaltimer_ns() - t0 < kWaitLimitNs) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kAttnBM, kAttnBN, 0, 0);
      constexpr uint32_t idesc_o = idesc_f16_f32(kAttnBM, kDH, 0, 1);  // V is MN-major
      bool issued = false;
      bool ok = mbar_wait(q_full, 0, abort_flag, 210);
      if (ok) tc_fence_after();
      const uint64_t q_desc = sw128_desc(smem_u32(sQ), 16, 1024);

      auto issue_pv = [&](int i) -> bool {
        const int s = i % kKVStages;
        const uint32_t ph = (uint32_t)((i / kKVStages) & 1);
        const int buf = i & 1;
        if (!mbar_wait(v_full(s), ph, abort_flag, 211)) return false;
        if (!mbar_wait(p_full(buf), (uint32_t)((i >> 1) & 1), abort_flag, 212)) return false;
        if (i >= 2 && !mbar_wait(o_empty(buf), (uint32_t)(((i - 2) >> 1) & 1), abort_flag, 213))
          return false;
        tc_fence_after();
        const uint32_t d = tmem_base + 256u + (uint32_t)(buf * kDH);
        const uint32_t p_base = smem_u32(sP + buf * kPBytes);
        const uint32_t v_base = smem_u32(sV + s * kKVBytes);
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k) {
          // A = P (K-major, two 64-key atoms of 16 KB), B = V (MN-major, 16 key
          // rows of 128 bytes per K=16 step).
          const uint64_t a_desc =
              sw128_desc(p_base + (uint32_t)((k >> 2) * (kAttnBM * 128)) + (uint32_t)((k & 3) * 32),
                         16, 1024);
          const uint64_t b_desc = sw128_desc(v_base + (uint32_t)(k * 16 * 128), 1024, 1024);
          mma_f16_ss(d, a_desc, b_desc, idesc_o, k != 0 ? 1u : 0u);
        }
        mma_commit(o_full(buf));
        mma_commit(v_empty(s));
        mma_commit(p_empty(buf));
        return true;
      };

      for (int j = 0; ok && j < T; ++j) {
        const int s = j % kKVStages;
        const uint32_t ph = (uint32_t)((j / kKVStages) & 1);
        const int buf = j & 1;
        if (!mbar_wait(k_full(s), ph, abort_flag, 214)) break;
        if (j >= 2 && !mbar_wait(s_empty(buf), (uint32_t)(((j - 2) >> 1) & 1), abort_flag, 215))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * kAttnBN);
        const uint64_t k_desc = sw128_desc(smem_u32(sK + s * kKVBytes), 16, 1024);
#pragma unroll
        for (int k = 0; k < kDH / 16; ++k)
          mma_f16_ss(d, q_desc + (uint64_t)(2 * k), k_desc + (uint64_t)(2 * k), idesc_s,
                     k != 0 ? 1u : 0u);
        issued = true;
        mma_commit(s_full(buf));
        mma_commit(k_empty(s));
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && T > 0 && !*abort_flag) issue_pv(T - 1);
      if (issued) {
        mma_commit(final_bar);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(final_bar, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // Softmax warps.
    const int quarter = warp & 3;
    const int row = quarter * 32 + (int)lane;  // query row in the tile = TMEM lane
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const int q_local = qt * kAttnBM + row;
    const int q_pos = (p.causal && p.q_pos0 ? p.q_pos0[b] : 0) + q_local;
    float m_run = -INFINITY;  // running max of s*sl2
    float l_run = 0.f;
    float alpha_prev = 0.f;
    float acc[kDH];
#pragma unroll
    for (int d = 0; d < kDH; ++d) acc[d] = 0.f;
    bool ok = true;

    auto fold_o = [&](int i) -> bool {
      const int buf = i & 1;
      if (!mbar_wait(o_full(buf), (uint32_t)((i >> 1) & 1), abort_flag, 220)) return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(t_lane + 256u + (uint32_t)(buf * kDH), r0);
      tmem_ld32(t_lane + 256u + (uint32_t)(buf * kDH) + 32u, r1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty(buf));
#pragma unroll
      for (int d = 0; d < 32; ++d) acc[d] = fmaf(acc[d], alpha_prev, __uint_as_float(r0[d]));
#pragma unroll
      for (int d = 0; d < 32; ++d)
        acc[32 + d] = fmaf(acc[32 + d], alpha_prev, __uint_as_float(r1[d]));
      return true;
    };

    KvWalk w;
    w.init(kv_off, kv_len, p.G);
    for (int j = 0; j < T; ++j, w.next()) {
      const int buf = j & 1;
      const int s = j % kKVStages;
      if (!mbar_wait(s_full(buf), (uint32_t)((j >> 1) & 1), abort_flag, 221)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[kAttnBN];
      tmem_ld32(t_lane + (uint32_t)(buf * kAttnBN) + 0u, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
      tmem_ld32(t_lane + (uint32_t)(buf * kAttnBN) + 32u, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld32(t_lane + (uint32_t)(buf * kAttnBN) + 64u, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
      tmem_ld32(t_lane + (uint32_t)(buf * kAttnBN) + 96u, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty(buf));

      const int nvalid = w.valid();
      const int kp0 = w.first_pos();
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAttnBN; ++c) {
        float x = __uint_as_float(sr[c]);
        if (c >= nvalid || (p.causal && kp0 + c > q_pos)) x = -INFINITY;
        sr[c] = __float_as_uint(x);
        mx = fmaxf(mx, x);
      }
      const float m_new = fmaxf(m_run, mx * sl2);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2_approx(m_run - m_use);
      m_run = m_new;

      // P_j -> shared (wait until P_{j-2} V_{j-2} has finished reading it).
      if (j >= 2 && !mbar_wait(p_empty(buf), (uint32_t)(((j - 2) >> 1) & 1), abort_flag, 222)) {
        ok = false;
        break;
      }
      float rowsum = 0.f;
      uint8_t* prow = sP + buf * kPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          e[u] = exp2_approx(fmaf(__uint_as_float(sr[8 * c + u]), sl2, -m_use));
          rowsum += e[u];
        }
        const uint4 v4 = make_uint4(pack_half2(e[0], e[1]), pack_half2(e[2], e[3]),
                                    pack_half2(e[4], e[5]), pack_half2(e[6], e[7]));
        const int atom = c >> 3, cc = c & 7;
        *reinterpret_cast<uint4*>(prow + atom * (kAttnBM * 128) + ((cc ^ (row & 7)) << 4)) = v4;
      }
      l_run = l_run * alpha + rowsum;
      if (nvalid < kAttnBN) {
        // Zero the V rows past the segment end (thread `row` owns key row `row`).
        if (!mbar_wait(v_full(s), (uint32_t)((j / kKVStages) & 1), abort_flag, 223)) {
          ok = false;
          break;
        }
        if (row >= nvalid) {
          uint4* vrow = reinterpret_cast<uint4*>(sV + s * kKVBytes + row * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) vrow[c] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(buf));

      if (j >= 1 && !fold_o(j - 1)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && T > 0 && fold_o(T - 1)) {
      // done
    } else {
      ok = false;
    }
    if (ok && q_local < nq) {
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      __half* dst = p.ctx + (int64_t)(q_begin + q_local) * p.ld_ctx + h * kDH;
#pragma unroll
      for (int c = 0; c < kDH / 8; ++c) {
        uint4 o;
        o.x = pack_half2(acc[8 * c + 0] * inv_l, acc[8 * c + 1] * inv_l);
        o.y = pack_half2(acc[8 * c + 2] * inv_l, acc[8 * c + 3] * inv_l);
        o.z = pack_half2(acc[8 * c + 4] * inv_l, acc[8 * c + 5] * inv_l);
        o.w = pack_half2(acc[8 * c + 6] * inv_l, acc[8 * c + 7] * inv_l);
        reinterpret_cast<uint4*>(dst)[c] = o;
      }
    } else if (T == 0 && q_local < nq) {
      __half* dst = p.ctx + (int64_t)(q_begin + q_local) * p.ld_ctx + h * kDH;
#pragma unroll
      for (int c = 0; c < kDH / 8; ++c) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0, 0, 0, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnTmemCols);
  }
}

int launch_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_dim != kDH)
    return set_error(TJ_ERR_UNSUPPORTED, "flash_attn_fwd: head_dim %d (only 64 is built)", a.head_dim);
  if (a.H <= 0 || a.B <= 0 || a.G <= 0 || a.q_rows < 0 || a.kv_rows < 0 || a.max_q_per_sample < 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: bad sizes H=%d B=%d G=%d", a.H, a.B, a.G);
  if (!a.q || !a.k || !a.v || !a.ctx || !a.q_cu || !a.kv_off || !a.kv_len)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: null pointer");
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
       reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.ctx)) & 15u)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: operands must be 16-byte aligned");
  if (a.kv_stride_h % 8 != 0 || a.kv_stride_g % 8 != 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: K/V strides must be multiples of 8 elements");
  if (a.causal && a.G > 1 && a.q_pos0 == nullptr)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: causal with key segments needs q_pos0");
  if (a.q_rows == 0 || a.max_q_per_sample == 0 || a.kv_rows == 0) return TJ_OK;

  CUtensorMap tq, tk, tv;
  {
    uint64_t d[3] = {(uint64_t)kDH, (uint64_t)a.q_rows, (uint64_t)a.H};
    uint64_t s[2] = {(uint64_t)kDH, (uint64_t)kDH * a.q_rows};
    uint32_t bx[3] = {kDH, kAttnBM, 1};
    int rc = make_tmap_f16(&tq, a.q, 3, d, s, bx);
    if (rc) return rc;
  }
  {
    uint64_t d[4] = {(uint64_t)kDH, (uint64_t)a.kv_rows, (uint64_t)a.H, (uint64_t)a.G};
    uint64_t s[3] = {(uint64_t)kDH, (uint64_t)a.kv_stride_h, (uint64_t)a.kv_stride_g};
    uint32_t bx[4] = {kDH, kAttnBN, 1, 1};
    int rc = make_tmap_f16(&tk, a.k, 4, d, s, bx);
    if (rc) return rc;
    rc = make_tmap_f16(&tv, a.v, 4, d, s, bx);
    if (rc) return rc;
  }
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(attention_tcgen05_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmem);
    if (e != cudaSuccess)
      return set_error(TJ_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  AttnKernelParams kp{};
  kp.H = a.H;
  kp.B = a.B;
  kp.G = a.G;
  kp.q_cu = a.q_cu;
  kp.kv_off = a.kv_off;
  kp.kv_len = a.kv_len;
  kp.kv_len_stride = a.kv_len_stride;
  kp.scale_log2 = a.scale * 1.4426950408889634f;
  kp.causal = a.causal;
  kp.q_pos0 = a.q_pos0;
  kp.ctx = static_cast<__half*>(a.ctx);
  kp.ld_ctx = a.H * kDH;
  dim3 grid((a.max_q_per_sample + kAttnBM - 1) / kAttnBM, a.H, a.B);
  if (grid.y > 65535 || grid.z > 65535)
    return set_error(TJ_ERR_UNSUPPORTED, "flash_attn_fwd: H=%d or B=%d above 65535", a.H, a.B);
  attention_tcgen05_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>(tq, tk, tv, kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

}  // namespace tj
