// Masked flash attention forward on tcgen05, replacing the SDPA call of
// v16_1_clean.py:505-514 (non-causal, [B,1,1,S] key mask) and :491-504
// (causal), i.e. softmax(QK^T*scale)V of the FP32 reference,
// torch_transformer_benchmark.py:97-117, with the score matrix never stored.
// Heads are zero-padded to P = 64, 128 or 256 columns (AttnCfg below); the
// description here is the P = 64 instance, the one the dense layers run.
//
// Queries and keys are compact: the token plan packs the valid tokens of each
// sample densely, so a sample's keys are the rows [off, off+len) of its key
// segment(s) and padded keys never enter the loop.  A sample may have several
// key segments (context parallelism: one per rank, gathered by NCCL), walked
// in order as one key sequence.
//
// One CTA = two 128-query tiles of one (sample, head); 384 threads:
//   warp 0        TMA producer: Q tiles once, K/V tiles of 128 keys into a
//                 4-stage ring.  For the last, partial tile of a segment it
//                 also zeroes the V rows past the segment end in shared memory,
//                 so stale or foreign rows cannot reach P V even as 0 * NaN.
//   warp 1        TMEM allocation and MMA issue (one lane):
//                   S_t = Q_t K_j^T    (SS, M=128 N=128, 4 x K=16)
//                   O_t += P_t V_j     (TS: P from TMEM, V from shared, 8 x K=16)
//   warps 4-7     softmax for query tile 0, warps 8-11 for query tile 1;
//                 thread = query row = TMEM lane.
// TMEM (512 columns): tile t uses O [256t, +64) (fp32), S [256t+64, +128) and
// P [256t+192, +64) (fp16 pairs).
//
// Softmax per key tile: load the S row, mask only on partial/causal tiles,
// tree max; the running max is only raised when the new max exceeds it by
// more than 8 (log2 units), in which case O (in TMEM) and the row sum are
// rescaled -- otherwise P = exp2(s*scale*log2e - m) stays <= 2^8, safe in fp16.
// P goes back to TMEM as fp16 and the tensor core accumulates O += P V; the
// two query tiles' softmax warpgroups take turns on the exponentials while the
// tensor core works for the other tile.
#include "common.cuh"
#include "internal.h"

namespace tj {

int make_tmap_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_elems, const uint32_t* box);

constexpr int kAttnBM = 128;     // queries per tile

// Per padded head dim DH (the q/k/v row length: 64, 128 or 256; head dims
// below it are zero-padded): 64-column chunks CH (one 128-byte swizzle atom
// each), keys per tile BN, query tiles per CTA NT and K/V pipeline stages,
// chosen so shared memory (<= 227 KB) and TMEM (512 columns) hold them.
// TMEM per query tile: O [0, DH), S [DH, DH+BN), P [DH+BN, DH+BN+BN/2) (fp16
// pairs); DH=64 packs two tiles at a 256-column stride.
// SHORT (DH=64, at most 128 queries per sample): one query tile, two stages,
// 256 threads and 256 TMEM columns, so two CTAs share an SM and one CTA's
// pipeline fill and drain overlap the other's work -- short sequences have a
// single key tile per (sample, head), so that latency is most of a CTA's life.
template <int DH_, bool SHORT = false>
struct AttnCfg {
  static constexpr int DH = DH_;
  static constexpr int CH = DH / 64;
  static constexpr int BN = DH <= 128 ? 128 : 64;
  static constexpr int NT = (DH == 64 && !SHORT) ? 2 : 1;
  static constexpr int STAGES = SHORT ? 2 : (DH == 64 ? 4 : (DH == 128 ? 3 : 2));
  static constexpr int kThreads = SHORT ? 256 : 384;
  static constexpr int kMinBlocks = SHORT ? 2 : 1;
  static constexpr uint32_t kTmemCols = SHORT ? 256 : 512;
  // Register split: the producer/MMA warpgroup gives registers to the softmax
  // warpgroup(s).  kLaunchRegs is what ptxas must allocate (the launcher checks
  // the built kernel); 128*kRegsLow + (kThreads-128)*kRegsHigh may not exceed
  // kThreads*kLaunchRegs or setmaxnreg.inc would wait forever.
  static constexpr int kLaunchRegs = SHORT ? 128 : 168;
  static constexpr int kRegsLow = 56;
  static constexpr int kRegsHigh = SHORT ? 200 : 224;
  static_assert(128 * kRegsLow + (kThreads - 128) * kRegsHigh <= kThreads * kLaunchRegs, "register split");
  static_assert(kThreads * kLaunchRegs * kMinBlocks <= 65536, "register file");
  static constexpr uint32_t kQChunk = kAttnBM * 128;   // 128 rows x 64 halves
  static constexpr uint32_t kQBytes = CH * kQChunk;    // one query tile
  static constexpr uint32_t kKVChunk = BN * 128;       // BN rows x 64 halves
  static constexpr uint32_t kKVBytes = CH * kKVChunk;  // one K (or V) stage
  static constexpr uint32_t kTileStride = 256;         // TMEM columns between query tiles
  static constexpr uint32_t kOCol = 0, kSCol = DH, kPCol = DH + BN;
  static constexpr size_t kSmem = 1024 + (size_t)NT * kQBytes + 2 * (size_t)STAGES * kKVBytes + 512;
  static_assert(NT == 1 || kPCol + BN / 2 <= kTileStride, "two query tiles must fit in TMEM");
  static_assert(kPCol + BN / 2 <= kTmemCols, "query tile must fit in TMEM");
  static_assert(kSmem * kMinBlocks <= 232448, "shared memory");
  static_assert(STAGES <= 8, "barrier slots");
};
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P <= 256 between rescales
// Of every 8 exponential pairs, this many run as a polynomial on the FMA pipe
// and the rest on the MUFU unit (which alone would be the softmax bottleneck).
#ifndef TJ_ATTN_POLY_PAIRS_PER_8
#define TJ_ATTN_POLY_PAIRS_PER_8 2
#endif
constexpr int kPolyPairsPer8 = TJ_ATTN_POLY_PAIRS_PER_8;

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
  int dh_out;  // real head dim (<= DH): columns of ctx written per head
  const int32_t* order;  // optional: sample handled by grid row z (longest first)
  int z0;                // first grid row of this launch (batches above 65535 take several)
  int q_rows, kv_rows;   // rows of the Q slab and of one K/V slab (bounds of the row tables)
  // Split attention over two launches (context parallelism: the rank's own
  // keys first, the other ranks' keys once they have arrived).  part_mode 1
  // writes this launch's partial result instead of ctx: the normalised fp32
  // context part_o [q_rows][H*dh_out] and part_lse [q_rows][H] = log2 of the
  // softmax denominator in base-2 units (log2 sum 2^(s*scale*log2e)), -inf
  // for a row without keys.  part_mode 2 merges its own keys' result with
  // that partial and writes ctx.  part_mode 0: ctx only.
  float* part_o;
  float* part_lse;
  int part_mode;
};

// The row tables (q_cu, kv_off, kv_len, order) live in device memory, written
// by the caller or an earlier kernel, so the host cannot check them without a
// synchronise.  Every CTA checks the entries it uses before any load or store:
// an out-of-range entry is recorded as kDevBadArgument (wait site 230) in the
// status word and the CTA returns without touching memory.
__device__ __forceinline__ bool attn_tables_ok(const AttnKernelParams& p, int zb, int* b_out) {
  const int b = p.order ? p.order[zb] : zb;
  if (b < 0 || b >= p.B) return false;
  const int q0 = p.q_cu[b], q1 = p.q_cu[b + 1];
  if (q0 < 0 || q1 < q0 || q1 > p.q_rows) return false;
  const int32_t* off = p.kv_off + (int64_t)b * p.kv_len_stride;
  const int32_t* len = p.kv_len + (int64_t)b * p.kv_len_stride;
  for (int g = 0; g < p.G; ++g) {
    const int n = len[g];
    if (n > 0 && (off[g] < 0 || (int64_t)off[g] + n > p.kv_rows)) return false;
  }
  *b_out = b;
  return true;
}

// Walks the key tiles of one sample in order: segment g, tile i inside it.
// Every role walks the same sequence, so tile j means the same keys to each.
struct KvWalk {
  const int32_t* off;
  const int32_t* len;
  int G, bn;
  int g, i, seg_len, seg_off, pos_base;  // pos_base = key position of segment start
  __device__ void init(const int32_t* o, const int32_t* l, int G_, int bn_) {
    off = o;
    len = l;
    G = G_;
    bn = bn_;
    g = 0;
    i = 0;
    pos_base = 0;
    seg_len = 0;
    seg_off = 0;
    load_segment();
  }
  __device__ void load_segment() {
    while (g < G && len[g] <= 0) ++g;
    if (g < G) {
      seg_len = len[g];
      seg_off = off[g];
    }
  }
  __device__ int row() const { return seg_off + i * bn; }
  __device__ int valid() const { return min(bn, seg_len - i * bn); }
  __device__ int first_pos() const { return pos_base + i * bn; }
  __device__ void next() {
    if (g >= G) return;
    ++i;
    if (i * bn >= seg_len) {
      pos_base += seg_len;
      ++g;
      i = 0;
      load_segment();
    }
  }
};

// Number of key tiles to visit; with causal masking, tiles whose first key is
// after the last query of the CTA are skipped.
__device__ __forceinline__ int count_kv_tiles(const int32_t* off, const int32_t* len, int G, int bn,
                                              bool causal, int max_q_pos) {
  KvWalk w;
  w.init(off, len, G, bn);
  int t = 0;
  while (w.g < G) {
    if (causal && w.first_pos() > max_q_pos) break;
    ++t;
    w.next();
  }
  return t;
}

template <int DH, bool SHORT>
__global__ void __launch_bounds__(AttnCfg<DH, SHORT>::kThreads, AttnCfg<DH, SHORT>::kMinBlocks)
    attention_tcgen05_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const AttnKernelParams p) {
  using Cfg = AttnCfg<DH, SHORT>;
  constexpr int kRegsLow = Cfg::kRegsLow, kRegsHigh = Cfg::kRegsHigh;
  constexpr uint32_t kAttnTmemCols = Cfg::kTmemCols;
  constexpr int BN = Cfg::BN, CH = Cfg::CH, NT = Cfg::NT, kKVStages = Cfg::STAGES;
  constexpr uint32_t kQBytes = Cfg::kQBytes, kKVBytes = Cfg::kKVBytes;
  const int h = blockIdx.y;
  pdl_wait();  // q/k/v and the token plan come from earlier kernels
  const int zb = p.z0 + (int)blockIdx.z;
  int b = 0;
  if (!attn_tables_ok(p, zb, &b)) {  // uniform for the CTA
    if (threadIdx.x == 0) report_error(kDevBadArgument, 230);
    return;
  }
  const int q_begin = p.q_cu[b];
  const int nq = p.q_cu[b + 1] - q_begin;
  const int q_tile0 = blockIdx.x * NT;
  if (q_tile0 * kAttnBM >= nq) return;  // uniform for the CTA
  const int ntile = (NT == 2 && (q_tile0 + 1) * kAttnBM < nq) ? 2 : 1;
  const int32_t* kv_off = p.kv_off + (int64_t)b * p.kv_len_stride;
  const int32_t* kv_len = p.kv_len + (int64_t)b * p.kv_len_stride;
  const int q_pos0 = (p.causal && p.q_pos0) ? p.q_pos0[b] : 0;
  const int max_q_pos = q_pos0 + min(nq, (q_tile0 + ntile) * kAttnBM) - 1;
  const int T = count_kv_tiles(kv_off, kv_len, p.G, BN, p.causal != 0, max_q_pos);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = smem;                       // NT query tiles of CH chunks
  uint8_t* sK = sQ + NT * kQBytes;          // kKVStages x CH chunks of BN rows
  uint8_t* sV = sK + kKVStages * kKVBytes;  // kKVStages x CH chunks of BN rows
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKVStages * kKVBytes);
  // Barriers (8-byte slots, room for 8 K/V stages): q_full, k_full[8],
  // v_full[8], k_empty[8], v_empty[8], vfix[8], s_full[2], s_empty[2],
  // p_full[2], pv_done[2], final, exp_done0[4], exp_done1[4]; then the TMEM
  // base address and the abort flag.
  const uint32_t q_full = smem_u32(bars + 0);
  auto k_full = [&](int s) { return smem_u32(bars + 1 + s); };
  auto v_full = [&](int s) { return smem_u32(bars + 9 + s); };
  auto k_empty = [&](int s) { return smem_u32(bars + 17 + s); };
  auto v_empty = [&](int s) { return smem_u32(bars + 25 + s); };
  // vfix[s]: the producer has zeroed the V rows past the segment end of the
  // partial tile in stage s (one phase per partial tile that used the stage).
  auto vfix = [&](int s) { return smem_u32(bars + 33 + s); };
  auto s_full = [&](int t) { return smem_u32(bars + 41 + t); };
  auto s_empty = [&](int t) { return smem_u32(bars + 43 + t); };
  auto p_full = [&](int t) { return smem_u32(bars + 45 + t); };
  auto pv_done = [&](int t) { return smem_u32(bars + 47 + t); };
  const uint32_t final_bar = smem_u32(bars + 49);
  // exp_done{t}[q]: the softmax warp of query tile t on SM sub-partition q has
  // issued the exponentials of its current key tile (see the softmax loop).
  auto exp_done = [&](int t, int q) { return smem_u32(bars + 50 + 4 * t + q); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 58);
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
      mbar_init(vfix(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(s_empty(t), 4);
      mbar_init(p_full(t), 4);
      mbar_init(pv_done(t), 1);
    }
    mbar_init(final_bar, 1);
    for (int q = 0; q < 4; ++q) {
      mbar_init(exp_done(0, q), 1);
      mbar_init(exp_done(1, q), 1);
    }
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

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      int last_k[kKVStages], last_v[kKVStages];
      for (int s = 0; s < kKVStages; ++s) last_k[s] = last_v[s] = -1;
      bool q_issued = false;
      if (lane == 0 && !*abort_flag) {
        mbar_arrive_expect_tx(q_full, ntile * kQBytes);
        for (int t = 0; t < ntile; ++t)
          for (int c = 0; c < CH; ++c)
            tma_load_3d(smem_u32(sQ + t * kQBytes + c * Cfg::kQChunk), &tmQ, q_full, 64 * c,
                        q_begin + (q_tile0 + t) * kAttnBM, h);
        q_issued = true;
      }
      KvWalk w;
      w.init(kv_off, kv_len, p.G, BN);
      bool ok = true;
      for (int j = 0; j < T && ok; ++j, w.next()) {
        const int s = j % kKVStages;
        const uint32_t ph = (uint32_t)((j / kKVStages) & 1);
        const int nvalid = w.valid();
        if (lane == 0) {
          ok = mbar_wait(k_empty(s), ph ^ 1, abort_flag, 200);
          if (ok) {
            mbar_arrive_expect_tx(k_full(s), kKVBytes);
            for (int c = 0; c < CH; ++c)
              tma_load_4d(smem_u32(sK + s * kKVBytes + c * Cfg::kKVChunk), &tmK, k_full(s), 64 * c,
                          w.row(), h, w.g);
            last_k[s] = (int)ph;
            ok = mbar_wait(v_empty(s), ph ^ 1, abort_flag, 201);
          }
          if (ok) {
            mbar_arrive_expect_tx(v_full(s), kKVBytes);
            for (int c = 0; c < CH; ++c)
              tma_load_4d(smem_u32(sV + s * kKVBytes + c * Cfg::kKVChunk), &tmV, v_full(s), 64 * c,
                          w.row(), h, w.g);
            last_v[s] = (int)ph;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok && nvalid < BN) {
          // Zero V rows [nvalid, BN) of every chunk once the tile has landed.
          ok = mbar_wait(v_full(s), ph, abort_flag, 202);
          ok = __all_sync(0xffffffffu, ok ? 1 : 0) != 0;
          if (ok) {
            for (int c = 0; c < CH; ++c)
              for (int r = nvalid + (int)lane; r < BN; r += 32) {
                uint4* vrow = reinterpret_cast<uint4*>(sV + s * kKVBytes + c * Cfg::kKVChunk + r * 128);
#pragma unroll
                for (int u = 0; u < 8; ++u) vrow[u] = make_uint4(0u, 0u, 0u, 0u);
              }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(vfix(s));
          }
        }
      }
      if (lane == 0) {
        // Let every issued load land before the CTA can exit.
        if (q_issued) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
        for (int s = 0; s < kKVStages; ++s) {
          const unsigned long long t0 = globaltimer_ns();
          if (last_k[s] >= 0)
            while (!mbar_try_wait(k_full(s), (uint32_t)last_k[s]) && globaltimer_ns() - t0 < kWaitLimitNs) {
            }
          if (last_v[s] >= 0)
            while (!mbar_try_wait(v_full(s), (uint32_t)last_v[s]) && globaltimer_ns() - t0 < kWaitLimitNs) {
            }
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc_s = idesc_f16_f32(kAttnBM, BN, 0, 0);
        constexpr uint32_t idesc_o = idesc_f16_f32(kAttnBM, 64, 0, 1);  // one 64-column V chunk, MN-major
        bool issued = false;
        bool ok = mbar_wait(q_full, 0, abort_flag, 210);
        if (ok) tc_fence_after();
        int nfix[kKVStages];
        for (int s = 0; s < kKVStages; ++s) nfix[s] = 0;
        // S_t(j) = Q_t K_j^T into the tile's S columns.
        auto issue_s = [&](int t, int j, uint32_t k_base) -> bool {
          if (j >= 1 && !mbar_wait(s_empty(t), (uint32_t)((j - 1) & 1), abort_flag, 215)) return false;
          tc_fence_after();
          const uint32_t s_tmem = tmem_base + (uint32_t)(t * Cfg::kTileStride + Cfg::kSCol);
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            // head-dim chunk c: K=64 of the contraction, 4 x K=16
            const uint64_t q_desc = sw128_desc(smem_u32(sQ + t * kQBytes + c * Cfg::kQChunk), 16, 1024);
            const uint64_t k_desc = sw128_desc(k_base + c * Cfg::kKVChunk, 16, 1024);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16_ss(s_tmem, q_desc + (uint64_t)(2 * k), k_desc + (uint64_t)(2 * k), idesc_s,
                         (c | k) != 0 ? 1u : 0u);
          }
          mma_commit(s_full(t));
          issued = true;
          return true;
        };
        // O_t += P_t(i) V_i.  The first user of V_i waits for the tile (and, for
        // a partial tile, for the zeroed rows); the last user releases the stage.
        auto issue_pv = [&](int t, int i, bool boundary) -> bool {
          const int s = i % kKVStages;
          if (t == 0) {
            if (!mbar_wait(v_full(s), (uint32_t)((i / kKVStages) & 1), abort_flag, 211)) return false;
            if (boundary) {
              if (!mbar_wait(vfix(s), (uint32_t)(nfix[s] & 1), abort_flag, 212)) return false;
              ++nfix[s];
            }
          }
          if (!mbar_wait(p_full(t), (uint32_t)(i & 1), abort_flag, 213)) return false;
          tc_fence_after();
          const uint32_t v_base = smem_u32(sV + s * kKVBytes);
          const uint32_t o_tmem = tmem_base + (uint32_t)(t * Cfg::kTileStride + Cfg::kOCol);
          const uint32_t p_tmem = tmem_base + (uint32_t)(t * Cfg::kTileStride + Cfg::kPCol);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              // B = V chunk c (MN-major): K=16 keys = 16 rows of 128 bytes per step;
              // it accumulates into O columns [64c, 64c+64).
              const uint64_t b_desc =
                  sw128_desc(v_base + c * Cfg::kKVChunk + (uint32_t)(k * 16 * 128), 1024, 1024);
              mma_f16_ts(o_tmem + (uint32_t)(64 * c), p_tmem + (uint32_t)(k * 8), b_desc, idesc_o,
                         (i | k) != 0 ? 1u : 0u);
            }
          }
          mma_commit(pv_done(t));
          if (t == ntile - 1) mma_commit(v_empty(s));
          return true;
        };

        // S is issued one key tile ahead: S0(j+1), S1(j+1), then PV0(j),
        // PV1(j).  A softmax warpgroup releases S(j) as soon as it has the row
        // in registers, so S(j+1) is computed while it still works on tile j
        // and its next step can start the moment P(j) is stored.
        auto issue_s_pair = [&](int j) -> bool {
          const int s = j % kKVStages;
          if (!mbar_wait(k_full(s), (uint32_t)((j / kKVStages) & 1), abort_flag, 214)) return false;
          const uint32_t k_base = smem_u32(sK + s * kKVBytes);
          for (int t = 0; t < ntile; ++t)
            if (!issue_s(t, j, k_base)) return false;
          mma_commit(k_empty(s));
          return true;
        };
        KvWalk w;
        w.init(kv_off, kv_len, p.G, BN);
        if (ok && T > 0) ok = issue_s_pair(0);
        for (int j = 0; ok && j < T; ++j, w.next()) {
          if (j + 1 < T) ok = issue_s_pair(j + 1);
          const bool boundary = w.valid() < BN;
          for (int t = 0; ok && t < ntile; ++t) ok = issue_pv(t, j, boundary);
        }
        if (issued) {
          mma_commit(final_bar);
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(final_bar, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + (int)lane;
    if (t < ntile) {
      const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(t * Cfg::kTileStride);
      const uint32_t s_tmem = t_lane + Cfg::kSCol, p_tmem = t_lane + Cfg::kPCol, o_tmem = t_lane + Cfg::kOCol;
      const float sl2 = p.scale_log2;
      const int q_local = (q_tile0 + t) * kAttnBM + row;
      const int q_pos = q_pos0 + q_local;
      float m_run = -INFINITY;  // running max (log2 units, stale by at most 8)
      float l_run = 0.f;
      bool ok = true;
      // test-only: the first warpgroup withholds its first "P ready" arrive
      const bool withhold = t == 0 && *((volatile int*)&g_debug_withhold) == kWithholdAttnPFull;

      KvWalk w;
      w.init(kv_off, kv_len, p.G, BN);
      for (int j = 0; j < T; ++j, w.next()) {
        if (!mbar_wait(s_full(t), (uint32_t)(j & 1), abort_flag, 220)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32(s_tmem + (uint32_t)(32 * c), *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty(t));

        // Keys c >= lim are masked: the segment end, and for causal masking
        // the keys after this query.
        int lim = w.valid();
        if (p.causal) lim = min(lim, q_pos - w.first_pos() + 1);
        if (lim < BN) {
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = __uint_as_float(sr[u]);
#pragma unroll
        for (int c = 8; c < BN - 8; c += 16)
#pragma unroll
          for (int u = 0; u < 8; ++u)
            pm[u] = fmax3(pm[u], __uint_as_float(sr[c + u]), __uint_as_float(sr[c + 8 + u]));
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = fmaxf(pm[u], __uint_as_float(sr[BN - 8 + u]));
        const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                               fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        const float m_cand = fmaxf(m_run, mx * sl2);

        // The running max moves only when it would grow by more than the
        // threshold; O and the row sum are then rescaled by alpha below.
        const bool need = __any_sync(0xffffffffu, m_cand > m_run + kRescaleThreshold);
        float alpha = 1.f;
        if (need) {
          alpha = (m_cand == -INFINITY) ? 1.f : exp2_approx(m_run - m_cand);
          l_run *= alpha;
          if (m_cand != -INFINITY) m_run = m_cand;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sl2v = make_float2(sl2, sl2);
        const float2 negm = make_float2(-m_use, -m_use);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        // The two softmax warps of an SM sub-partition (one per query tile)
        // take turns on the exponentials, tile 0 first: while one holds the
        // MUFU and FMA pipes, the other loads its next S row and takes its
        // max, instead of both reaching the exponentials at the same time.
        if (ntile == 2 && (t == 1 || j >= 1)) {
          const uint32_t bar = t == 0 ? exp_done(1, quarter) : exp_done(0, quarter);
          const uint32_t parity = (uint32_t)((t == 0 ? j - 1 : j) & 1);
          if (!mbar_wait(bar, parity, abort_flag, 223)) {
            ok = false;
            break;
          }
        }
        // P is computed into registers first, so the exponentials overlap the
        // tensor core's P_{j-1} V_{j-1}; only the TMEM stores wait for it.
        uint32_t pk[BN / 2];
#pragma unroll
        for (int c = 0; c < BN / 2; ++c) {
          float2 x = ffma2(make_float2(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), sl2v, negm);
          if ((c & 7) < kPolyPairsPer8) {
            x = exp2_poly2(x);  // FMA pipe
          } else {
            x.x = exp2_approx(x.x);  // MUFU
            x.y = exp2_approx(x.y);
          }
          acc[c & 3] = fadd2(acc[c & 3], x);
          pk[c] = pack_half2(x.x, x.y);
        }
        if (ntile == 2) {
          __syncwarp();
          if (lane == 0) mbar_arrive(exp_done(t, quarter));
        }

        // P_{j-1} V_{j-1} must be done: it reads the P buffer and writes O.
        if (j >= 1) {
          if (!mbar_wait(pv_done(t), (uint32_t)((j - 1) & 1), abort_flag, 221)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (need) {
#pragma unroll 1
            for (int c = 0; c < DH / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(o_tmem + (uint32_t)(32 * c), o);
              tmem_ld_wait();
#pragma unroll
              for (int d = 0; d < 32; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * alpha);
              tmem_st32(o_tmem + (uint32_t)(32 * c), o);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tmem_st32(p_tmem + (uint32_t)(32 * c), *reinterpret_cast<uint32_t(*)[32]>(pk + 32 * c));
        tmem_st_wait();
        const float2 a01 = fadd2(acc[0], acc[1]), a23 = fadd2(acc[2], acc[3]);
        const float2 a = fadd2(a01, a23);
        l_run += a.x + a.y;
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && !(withhold && j == 0)) mbar_arrive(p_full(t));
      }
      if (ok && T > 0) {
        ok = mbar_wait(pv_done(t), (uint32_t)((T - 1) & 1), abort_flag, 222);
        if (ok) tc_fence_after();
      }
      ok = __all_sync(0xffffffffu, ok ? 1 : 0) != 0;
      if (ok) {  // warp-uniform: the TMEM loads below are warp-collective
        // out = O * f_o + prior * f_p, prior = the partial result of an
        // earlier launch over other keys (part_mode 2).  O and l_run are
        // relative to 2^m_run, so this launch's log2-sum-exp is
        // m_run + log2(l_run) (-inf without keys).
        const bool row_ok = q_local < nq;
        const int64_t row = (int64_t)q_begin + q_local;
        const float e_cur = l_run > 0.f ? m_run : -INFINITY;
        float f_o = l_run > 0.f ? 1.0f / l_run : 0.f, f_p = 0.f;
        if (p.part_mode == 2 && row_ok) {
          const float lse_p = p.part_lse[row * p.H + h];
          const float mx = fmaxf(e_cur, lse_p);
          if (mx == -INFINITY) {
            f_o = 0.f;
          } else {
            const float a = e_cur == -INFINITY ? 0.f : exp2_approx(e_cur - mx);
            const float b2 = lse_p == -INFINITY ? 0.f : exp2_approx(lse_p - mx);
            const float inv = 1.0f / (l_run * a + b2);
            f_o = a * inv;
            f_p = b2 * inv;
          }
        }
        if (p.part_mode == 1 && row_ok)
          p.part_lse[row * p.H + h] = l_run > 0.f ? e_cur + __log2f(l_run) : -INFINITY;
        const int ld_part = p.H * p.dh_out;
        float* prow = p.part_mode ? p.part_o + row * ld_part + h * p.dh_out : nullptr;
        const bool vec_part = (p.dh_out & 3) == 0;
        __half* dst = p.part_mode == 1 ? nullptr : p.ctx + row * p.ld_ctx + h * p.dh_out;
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          if (32 * c >= p.dh_out) break;
          uint32_t o[32];
          if (T > 0) {
            tmem_ld32(o_tmem + (uint32_t)(32 * c), o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] = 0u;
          }
          if (!row_ok) continue;
          const bool full = 32 * c + 32 <= p.dh_out;
          float val[32];
#pragma unroll
          for (int d = 0; d < 32; ++d) val[d] = __uint_as_float(o[d]) * f_o;
          if (p.part_mode == 1) {
            if (vec_part && full) {
#pragma unroll
              for (int g = 0; g < 8; ++g)
                reinterpret_cast<float4*>(prow + 32 * c)[g] =
                    make_float4(val[4 * g], val[4 * g + 1], val[4 * g + 2], val[4 * g + 3]);
            } else {
#pragma unroll
              for (int d = 0; d < 32; ++d)
                if (32 * c + d < p.dh_out) prow[32 * c + d] = val[d];
            }
            continue;
          }
          if (p.part_mode == 2) {
            if (vec_part && full) {
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                const float4 q4 = reinterpret_cast<const float4*>(prow + 32 * c)[g];
                val[4 * g] += q4.x * f_p;
                val[4 * g + 1] += q4.y * f_p;
                val[4 * g + 2] += q4.z * f_p;
                val[4 * g + 3] += q4.w * f_p;
              }
            } else {
#pragma unroll
              for (int d = 0; d < 32; ++d)
                if (32 * c + d < p.dh_out) val[d] += prow[32 * c + d] * f_p;
            }
          }
          if ((p.dh_out & 7) == 0 && full) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 v;
              v.x = pack_half2(val[8 * g + 0], val[8 * g + 1]);
              v.y = pack_half2(val[8 * g + 2], val[8 * g + 3]);
              v.z = pack_half2(val[8 * g + 4], val[8 * g + 5]);
              v.w = pack_half2(val[8 * g + 6], val[8 * g + 7]);
              reinterpret_cast<uint4*>(dst + 32 * c)[g] = v;
            }
          } else {
            // Head dims that are not a multiple of 32 (or of 8): the padded
            // columns are dropped.
#pragma unroll
            for (int d = 0; d < 32; ++d)
              if (32 * c + d < p.dh_out) dst[32 * c + d] = __float2half_rn(val[d]);
          }
        }
      }
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnTmemCols);
  }
}

// Row length (halves) of the q/k/v buffers for a head dim: heads are
// zero-padded to 64, 128 or 256.
int attn_head_pad(int head_dim) { return head_dim <= 64 ? 64 : (head_dim <= 128 ? 128 : 256); }

template <int DH, bool SHORT>
static int launch_attention_t(const AttnArgs& a, cudaStream_t stream) {
  using Cfg = AttnCfg<DH, SHORT>;
  CUtensorMap tq, tk, tv;
  {
    uint64_t d[3] = {(uint64_t)DH, (uint64_t)a.q_rows, (uint64_t)a.H};
    uint64_t s[2] = {(uint64_t)DH, (uint64_t)DH * a.q_rows};
    uint32_t bx[3] = {64, kAttnBM, 1};
    int rc = make_tmap_f16(&tq, a.q, 3, d, s, bx);
    if (rc) return rc;
  }
  {
    uint64_t d[4] = {(uint64_t)DH, (uint64_t)a.kv_rows, (uint64_t)a.H, (uint64_t)a.G};
    uint64_t s[3] = {(uint64_t)DH, (uint64_t)a.kv_stride_h, (uint64_t)a.kv_stride_g};
    uint32_t bx[4] = {64, (uint32_t)Cfg::BN, 1, 1};
    int rc = make_tmap_f16(&tk, a.k, 4, d, s, bx);
    if (rc) return rc;
    rc = make_tmap_f16(&tv, a.v, 4, d, s, bx);
    if (rc) return rc;
  }
  {
    int num_sms = 0;
    int rc = ensure_device_props(&num_sms);
    if (rc) return rc;
  }
  static bool attr_set[64] = {};
  const int dev = device_index();
  if (!attr_set[dev]) {
    cudaFuncAttributes fa;
    cudaError_t e0 = cudaFuncGetAttributes(&fa, attention_tcgen05_kernel<DH, SHORT>);
    if (e0 != cudaSuccess)
      return set_error(TJ_ERR_CUDA, "attention attributes: %s", cudaGetErrorString(e0));
    if (fa.numRegs != Cfg::kLaunchRegs)
      return set_error(TJ_ERR_UNSUPPORTED,
                       "attention kernel (head dim %d%s) built with %d registers per thread, the "
                       "register split assumes %d; refusing to launch",
                       DH, SHORT ? ", short" : "", fa.numRegs, Cfg::kLaunchRegs);
    cudaError_t e = cudaFuncSetAttribute(attention_tcgen05_kernel<DH, SHORT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
    if (e != cudaSuccess)
      return set_error(TJ_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
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
  kp.ld_ctx = a.ld_ctx ? (int)a.ld_ctx : a.H * a.head_dim;
  kp.dh_out = a.head_dim;
  kp.order = a.order;
  kp.q_rows = a.q_rows;
  kp.kv_rows = a.kv_rows;
  kp.part_o = a.part_o;
  kp.part_lse = a.part_lse;
  kp.part_mode = a.part_mode;
  constexpr int kQPerCta = Cfg::NT * kAttnBM;
  if (a.H > 65535) return set_error(TJ_ERR_UNSUPPORTED, "flash_attn_fwd: H=%d above 65535", a.H);
  // Grid rows are samples; a batch above the 65535-row limit runs as several
  // launches, each starting at its first row z0.
  for (int z0 = 0; z0 < a.B; z0 += 65535) {
    kp.z0 = z0;
    dim3 grid((a.max_q_per_sample + kQPerCta - 1) / kQPerCta, a.H, a.B - z0 < 65535 ? a.B - z0 : 65535);
    cudaError_t e = launch_pdl(attention_tcgen05_kernel<DH, SHORT>, grid, dim3(Cfg::kThreads), Cfg::kSmem,
                               stream, tq, tk, tv, kp);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  }
  return TJ_OK;
}

int launch_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_dim <= 0 || a.head_dim > 256)
    return set_error(TJ_ERR_UNSUPPORTED, "flash_attn_fwd: head_dim %d (1..256 supported)", a.head_dim);
  if (a.H <= 0 || a.B <= 0 || a.G <= 0 || a.q_rows < 0 || a.kv_rows < 0 || a.max_q_per_sample < 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: bad sizes H=%d B=%d G=%d", a.H, a.B, a.G);
  if (a.part_mode < 0 || a.part_mode > 2)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: part_mode %d (0, 1 or 2)", a.part_mode);
  if (!a.q || !a.k || !a.v || (a.part_mode != 1 && !a.ctx) || !a.q_cu || !a.kv_off || !a.kv_len ||
      (a.part_mode != 0 && (!a.part_o || !a.part_lse)))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: null pointer");
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
       reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.ctx) |
       reinterpret_cast<uintptr_t>(a.part_o)) & 15u)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: operands must be 16-byte aligned");
  if (a.kv_stride_h % 8 != 0 || a.kv_stride_g % 8 != 0)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: K/V strides must be multiples of 8 elements");
  if (a.causal && a.G > 1 && a.q_pos0 == nullptr)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "flash_attn_fwd: causal with key segments needs q_pos0");
  if (a.ld_ctx != 0 && (a.ld_ctx < (int64_t)a.H * a.head_dim || a.ld_ctx > INT32_MAX ||
                        ((a.head_dim & 7) == 0 && (a.ld_ctx & 7) != 0)))
    return set_error(TJ_ERR_INVALID_ARGUMENT,
                     "flash_attn_fwd: context row stride %lld (at least H*head_dim = %d, a multiple "
                     "of 8 when head_dim is)",
                     (long long)a.ld_ctx, a.H * a.head_dim);
  if (a.q_rows == 0 || a.max_q_per_sample == 0 || a.kv_rows == 0) return TJ_OK;
  switch (attn_head_pad(a.head_dim)) {
    case 64:
      if (a.max_q_per_sample <= kAttnBM) return launch_attention_t<64, true>(a, stream);
      return launch_attention_t<64, false>(a, stream);
    case 128:
      return launch_attention_t<128, false>(a, stream);
    default:
      return launch_attention_t<256, false>(a, stream);
  }
}

}  // namespace tj
