// moe_prefill.cu — MoE expert GEMMs for large token counts (prefill) on the
// 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Same computation as moe_decode.cu (MLP::forward, src/model.rs:1088-1184,
// with the gpt-oss interleaved mlp1 and clamped SwiGLU), organised as two
// grouped GEMMs over the expert-sorted token slots:
//   GEMM1  D[2I rows, n cols] = W1_e[2I, H] . X_e^T  -> bias + SwiGLU -> h (f16 hi + lo)
//   GEMM2  D[H rows, n cols]  = W2_e[H, I] . (h_hi + h_lo)^T -> bias -> y_slot (f32)
// Weights are operand A (M = 128 rows per tile) and token activations operand
// B (N <= 256 columns per tile, the slots of one expert).
//
// One persistent CTA per SM walks the tile list (expert, token tile, weight
// tile), weight tile fastest so CTAs running side by side share the token
// tile in L2. Warp roles:
//   warp 0      TMA producer: token tiles (K-major, 128-byte swizzle) into the
//               stage ring;
//   warp 1      TMEM owner and MMA issuer: one thread issues
//               tcgen05.mma.kind::f16 (f16 x f16 -> f32) into a double-buffered
//               TMEM accumulator and commits to the stage / accumulator barriers;
//   warps 2-9   converters: stream the MXFP4 codes and E8M0 scales through a
//               per-thread cp.async ring, decode with cvt.rn.f16x2.e2m1x2,
//               multiply each 32-element block by its scale in f16 (exact for
//               scales 2^-23..2^14, which the upload checks) and store the
//               weight tile in the tensor cores' swizzled K-major layout;
//   warps 10-13 epilogue: tcgen05.ld of the accumulator (one TMEM lane per
//               weight row), bias, then for GEMM1 the gate/up pairing across
//               adjacent lanes, the 2^sigma token scale and the clamped SwiGLU
//               (h split into f16 hi + lo), for GEMM2 the f32 slot rows.
// Every wait on an mbarrier is bounded; a timeout sets an error code and the
// CTA winds down (waiting, again bounded, for its own copies and MMAs).
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace oxg {
namespace {

using namespace sm100;

constexpr int BM = 128;             // weight rows per CTA (the pair's MMA has M = 256)
constexpr int BN = 256;             // token columns per tile (MMA N)
constexpr int BNH = BN / 2;         // token rows of the tile each CTA loads
constexpr int BK = 64;              // K per stage (one 128-byte swizzle atom of f16)
constexpr int kConvWarps = 8;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, alternating 32-column chunks
// Warp layout (warp w runs on sub-partition w % 4): 0 TMA producer, 1 MMA
// issuer, converters on warps 2-4, 6-8, 10-11 (none beside the MMA issuer, so
// its tensor-core instructions do not queue behind their shared-memory
// traffic), 5 and 9 idle, epilogue on 12-19 (two per TMEM lane quarter).
constexpr int kEpiWarp0 = 12;
constexpr int kThreadsP = (kEpiWarp0 + kEpiWarps) * 32;  // 640
__device__ __forceinline__ int converter_index(int warp) {
  // warps 2, 3, 4, 6, 7, 8, 10, 11 -> 0..7; -1 otherwise
  return (warp >= 2 && warp < kEpiWarp0 && warp != 5 && warp != 9) ? warp - 2 - (warp > 5) - (warp > 9)
                                                                   : -1;
}
constexpr int kConvThreads = kConvWarps * 32;
// The converter warps form kGroups groups; group g fills the A tiles of the
// k-steps it with it % kGroups == g, so each warp pays the per-step waits and
// fences once per kGroups k-steps and decodes kTasks (row, q) tasks per step.
constexpr int kGroups = 2;
constexpr int kGroupThreads = kConvThreads / kGroups;
constexpr int kTasks = BM * 4 / kGroupThreads;
constexpr int kTmemCols = 512;
constexpr int kMaxExpertsP = 256;
constexpr int kCombMaxK = kPrefillCombineMaxK;  // top-k of the fused combine

struct PrefillArgs {
  const uint8_t *codes;   // tile chunks of [E, rows, K] (codes + scales, relayout.cu)
  const uint16_t *bias;   // [E, rows]
  int K, rows;
  size_t item_bytes;      // bytes of one 16-row tile
  int pair_adj;           // row pairing of the tile chunks (1: rows 2g, 2g + 1)
  const int32_t *counts, *offsets;
  int n_segments;  // runs of slot rows sharing one expert (counts/offsets index)
  int weight_mod;  // segment v multiplies by the layer's local expert v % weight_mod
  // GEMM1 epilogue
  const float *pos_scale;  // [S] 2^sigma of the token in each slot position
  uint16_t *h_hi, *h_lo;   // [S, I] f16
  int I;
  float alpha, limit;
  // GEMM2 epilogue: row p of segment v goes to y_seg[v] + p * H when y_seg is
  // given (expert parallel: the source rank's buffer, possibly a peer GPU's),
  // else to y_slot + (offsets[v] + p) * H
  float *y_slot;  // [S, H]
  float *const *y_seg;
  int H;
  int *err;
  // fused weighted combine (GEMM2, y_slot only): see PrefillIO
  float *y;
  const int32_t *perm, *slot_pos;
  const float *wts;
  uint32_t *comb_cnt;
  int topk;
};

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Alignment self-check: records `code` (first one wins) and tells the caller
// to skip the access.
__device__ __forceinline__ bool misaligned(uint64_t addr, uint64_t align, int *err, int code) {
  if (addr & (align - 1)) {
    atomicCAS(err, 0, code);
    return true;
  }
  return false;
}

struct Coords {
  int e;       // local expert
  int n0;      // first slot of the token tile within the expert
  int nvalid;  // valid columns of the tile
  int m0;      // first weight row of the tile
};

template <int GEMM, int STAGES>
__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tm0,
                        const __grid_constant__ CUtensorMap tm1, const PrefillArgs a) {
  constexpr int NB = GEMM == 1 ? 1 : 2;  // token tiles per stage (GEMM2: h hi and lo)
  constexpr int A_BYTES = BM * BK * 2;   // this CTA's 128 weight rows
  constexpr int B_BYTES = BNH * BK * 2;  // this CTA's half of the token tile
  constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
  constexpr int kLead = 2;  // a converter group's own k-steps whose codes are in registers
  static_assert(STAGES % kGroups == 0, "every converter group owns the same stages");
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment of the shared-space offset (the swizzle atoms of the
  // TMA tiles and the MMA descriptors assume it); the same in both CTAs
  uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t *tiles = smem;

  // full_, acc_empty and mma_done are used in rank 0 only; empty_ and
  // acc_full in both CTAs
  __shared__ uint64_t full_[STAGES], empty_[STAGES];
  __shared__ uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int ntile_prefix[kMaxExpertsP + 1];
  __shared__ int epi_ok;
  __shared__ float col_scale[BN];  // GEMM1: 2^sigma of each column of the current item
  __shared__ int comb_tok[GEMM == 2 ? BN : 1], comb_n;  // GEMM2: tokens this CTA combines

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int E = a.n_segments;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // both CTAs' converter groups + rank 0's expect_tx arrival
      mbar_init(&full_[s], 2 * (kConvWarps / kGroups) + 1);
      mbar_init(&empty_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
    int run = 0;
    for (int e = 0; e < E; ++e) {
      ntile_prefix[e] = run;
      run += (a.counts[e] + BN - 1) / BN;
    }
    ntile_prefix[E] = run;
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  const int MT = (a.rows + 2 * BM - 1) / (2 * BM);  // 256-row tiles of the pair
  const int total = ntile_prefix[E] * MT;
  const int KSTEPS = a.K / BK;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  auto coords = [&](int item) {
    Coords c;
    const int ntg = item / MT;
    c.m0 = (item - ntg * MT) * 2 * BM;
    int e = 0;
    while (e + 1 < E && ntile_prefix[e + 1] <= ntg) ++e;
    c.e = e;
    c.n0 = (ntg - ntile_prefix[e]) * BN;
    c.nvalid = min(BN, a.counts[e] - c.n0);
    return c;
  };
  // rank 0's full barriers as seen from either CTA
  auto full_cl = [&](int s) { return mapa_shared(smem_addr(&full_[s]), 0); };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // Each CTA loads its half of the token tile: rank 0 columns [0, n/2),
    // rank 1 [n/2, n) of the n-column MMA (n = valid columns rounded up to
    // 16); the bytes of both are counted on rank 0's full barrier.
    if (lane == 0) {
      prefetch_tmap(&tm0);
      if (NB == 2) prefetch_tmap(&tm1);
      int it = 0;
      int last_round[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_round[s] = -1;
      bool ok = true;
      for (int item = pair; ok && item < total; item += n_pairs) {
        const Coords c = coords(item);
        const int n_mma = (c.nvalid + 15) / 16 * 16;
        const int row0 = a.offsets[c.e] + c.n0 + (rank ? n_mma / 2 : 0);
        for (int ks = 0; ks < KSTEPS; ++ks, ++it) {
          const int s = it % STAGES, r = it / STAGES;
          if (r > 0) {
            if (!(ok = mbar_wait_cl(&empty_[s], (r - 1) & 1, a.err, 1))) break;
            // rank 0's stage is free only once the pair MMAs reading both
            // CTAs' halves of it are done: pass that on to rank 1
            if (rank == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&empty_[s]), 1));
          }
          uint8_t *st = tiles + s * STAGE_BYTES;
          if (misaligned(smem_addr(st + A_BYTES), 1024, a.err, 101) ||
              misaligned((uint64_t)&tm0, 64, a.err, 102)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_[s], 2 * NB * B_BYTES);
          tma_load_2d_pair(st + A_BYTES, &tm0, full_cl(s), ks * BK, row0);
          if (NB == 2) tma_load_2d_pair(st + A_BYTES + B_BYTES, &tm1, full_cl(s), ks * BK, row0);
          last_round[s] = r;
        }
      }
      if (!ok && rank == 0) {  // let copies still in flight land before the pair exits
        for (int s = 0; s < STAGES; ++s)
          if (last_round[s] >= 0) mbar_wait_cl(&full_[s], last_round[s] & 1, a.err, 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && rank == 0) {
      int it = 0, j = 0;
      bool ok = true;
      // stage s's A tile starts at tiles + s * STAGE_BYTES, its B tile(s) A_BYTES
      // later; shared addresses stay below 2^18, so adding to the 14-bit start
      // field of the descriptor never carries into the next field
      const uint64_t desc_a0 = desc_sw128_kmajor(smem_addr(tiles));
      // one commit per k-step, to rank 0's barrier (rank 0's TMA producer
      // and epilogue pass the news on to rank 1); stage and phase counters
      // advance without divisions
      int s = 0, phase = 0;
      const uint32_t empty0 = smem_addr(&empty_[0]);
      for (int item = pair; ok && item < total; item += n_pairs, ++j) {
        const Coords c = coords(item);
        const int buf = j & 1, rr = j >> 1;
        if (rr > 0 && !(ok = mbar_wait_cl(&acc_empty[buf], (rr - 1) & 1, a.err, 3))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        const int n_mma = (c.nvalid + 15) / 16 * 16;
        const uint32_t idesc = idesc_f16_f32(2 * BM, n_mma);
        for (int ks = 0; ks < KSTEPS; ++ks, ++it) {
          if (!(ok = mbar_wait_cl(&full_[s], phase, a.err, 2))) break;
          tc_fence_after();
          // descriptors of k16 slice 0; slice kk starts 32 B (2 units) further
          const uint64_t ad = desc_a0 + (uint64_t)(s * (STAGE_BYTES >> 4));
          const uint64_t bd = ad + (uint64_t)(A_BYTES >> 4);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_f16_pair(d, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0);
            if (NB == 2) umma_f16_pair(d, ad + 2 * kk, bd + (B_BYTES >> 4) + 2 * kk, idesc, 1);
          }
          umma_commit_pair(empty0 + (uint32_t)(s * sizeof(uint64_t)));
          if (++s == STAGES) {
            s = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(smem_addr(&acc_full[buf]));
      }
      // nothing may be left in flight when TMEM is released
      umma_commit_pair(mapa_shared(smem_addr(&mma_done), 0));
      mbar_wait_cl(&mma_done, 0, a.err, 2);
    }
  } else if (converter_index(warp) >= 0) {
    // ------------------------------------------------------------ converters
    // Thread gt of group grp owns kTasks (row, q) pairs of each of its weight
    // tiles: row (gt + t * kGroupThreads) / 4, 16-byte chunks q (block 2hf of
    // the k-step pair) and 4 + q (block 2hf + 1). Its codes (8 B: word q of
    // the two blocks, adjacent in the tile-chunk order) and the two scale
    // bytes are loaded into registers kLead of its k-steps before use.
    const int ct = converter_index(warp) * 32 + lane;
    const int grp = ct / kGroupThreads, gt = ct % kGroupThreads;
    const int q = gt & 3;
    const int full = a.K / 128;  // complete 4-block groups per row
    const int tail = (a.K / 32) % 4;
    // The tasks' rows are 32 apart, so they share the tile row lr = row % 16
    // and with it the offsets inside each group chunk (part p, lane row gr).
    static_assert(kGroupThreads / 4 == 32, "task rows must be a whole number of tiles apart");
    const int lr = (gt >> 2) & 15;
    const int pp = a.pair_adj ? (lr & 1) : (lr >> 3), gr = a.pair_adj ? (lr >> 1) : (lr & 7);
    const int c_full = pp * 512 + (4 * gr + q) * 16, s_full = 1024 + pp * 32 + 4 * gr;
    const int c_tail = pp * 128 * tail + (4 * gr + q) * 4 * tail, s_tail = 256 * tail + pp * 32 + 4 * gr;
    // issue cursor: this group's k-steps as (item, ks), kGroups steps apart
    int i_item = pair, i_ks = grp;
    // task t's row is row0 + t * 32: its tile starts at crow + t * cstep
    const uint8_t *crow = a.codes;
    const size_t cstep = 2 * a.item_bytes;
    int n_rows_ok = 0;  // tasks 0 .. n_rows_ok - 1 lie inside the matrix
    auto set_rows = [&](int item) {
      const Coords c = coords(item);
      const int R0 = c.m0 + (int)rank * BM + (gt >> 2);
      crow = a.codes + ((size_t)(c.e % a.weight_mod) * (a.rows / 16) + (R0 >> 4)) * a.item_bytes;
      n_rows_ok = R0 < a.rows ? min(kTasks, (a.rows - R0 + kGroupThreads / 4 - 1) / (kGroupThreads / 4)) : 0;
    };
    auto normalise = [&]() {
      while (i_item < total && i_ks >= KSTEPS) {
        i_ks -= KSTEPS;
        i_item += n_pairs;
      }
    };
    normalise();
    if (i_item < total) set_rows(i_item);
    auto load_step = [&](uint2 (&cw)[kTasks], uint32_t (&sw)[kTasks]) {
      const int G = i_ks >> 1, hf = i_ks & 1;
      const int off = G * 1088 + (G < full ? c_full + hf * 8 : c_tail);
      const int soff = G * 1088 + (G < full ? s_full : s_tail) + 2 * hf;
#pragma unroll
      for (int t = 0; t < kTasks; ++t) {
        cw[t] = make_uint2(0u, 0u);
        sw[t] = 0u;
        if (i_item < total && t < n_rows_ok) {
          cw[t] = __ldg(reinterpret_cast<const uint2 *>(crow + t * cstep + off));
          sw[t] = __ldg(reinterpret_cast<const unsigned short *>(crow + t * cstep + soff));
        }
      }
      if (i_item < total) {
        const int prev = i_item;
        i_ks += kGroups;
        normalise();
        if (i_item != prev && i_item < total) set_rows(i_item);
      }
    };
    uint2 rc[kLead][kTasks];
    uint32_t rs[kLead][kTasks];
#pragma unroll
    for (int u = 0; u < kLead; ++u) load_step(rc[u], rs[u]);

    const int my_items = pair < total ? (total - 1 - pair) / n_pairs + 1 : 0;
    const int n_steps = my_items * KSTEPS;
    bool ok = true;
    for (int m0 = 0; ok && grp + m0 * kGroups < n_steps; m0 += kLead) {
#pragma unroll
      for (int u = 0; u < kLead; ++u) {
        const int it = grp + (m0 + u) * kGroups;
        if (it >= n_steps) break;
        const int s = it % STAGES, r = it / STAGES;
        // decode first (rows beyond the matrix load zero codes and scales)
        uint4 o[kTasks][2];
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          const uint32_t s0 = rs[u][t] & 0xFFu, s1 = rs[u][t] >> 8;
          const uint32_t h0 = pack_f16x2(e8m0_to_f32(s0), e8m0_to_f32(s0));
          const uint32_t h1 = pack_f16x2(e8m0_to_f32(s1), e8m0_to_f32(s1));
          uint32_t f[4];
          e2m1x8_to_f16x8(rc[u][t].x, f);
          o[t][0] = make_uint4(hmul2(f[0], h0), hmul2(f[1], h0), hmul2(f[2], h0), hmul2(f[3], h0));
          e2m1x8_to_f16x8(rc[u][t].y, f);
          o[t][1] = make_uint4(hmul2(f[0], h1), hmul2(f[1], h1), hmul2(f[2], h1), hmul2(f[3], h1));
        }
        load_step(rc[u], rs[u]);  // this group's step kLead ahead
        if (r > 0) {  // one lane waits for the MMAs to free the stage; the warp follows
          int w_ok = 1;
          if (lane == 0) w_ok = mbar_wait_cl(&empty_[s], (r - 1) & 1, a.err, 5);
          if (!(ok = __shfl_sync(0xFFFFFFFFu, w_ok, 0) != 0)) break;
        }
        uint8_t *atile = tiles + s * STAGE_BYTES;
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          const int r_ = (gt + t * kGroupThreads) >> 2;
          // chunks q and 4 + q of the row under the 128-byte swizzle. Odd rows
          // store their two chunks in the opposite order, so the 8 lanes (two
          // rows) of each store wavefront hit 8 different bank groups.
          const int x7 = r_ & 7;
          uint8_t *rowp = atile + (r_ >> 3) * 1024 + x7 * 128;
          const bool odd = r_ & 1;
          *reinterpret_cast<uint4 *>(rowp + (((odd ? 4 + q : q) ^ x7) << 4)) = odd ? o[t][1] : o[t][0];
          *reinterpret_cast<uint4 *>(rowp + (((odd ? q : 4 + q) ^ x7) << 4)) = odd ? o[t][0] : o[t][1];
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(full_cl(s));
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int lq = warp & 3;            // TMEM lane quarter this warp may access
    const int ew = warp - kEpiWarp0;
    const int half = ew >> 2;           // which 32-column chunks: 2m + half
    const int r = lq * 32 + lane;       // accumulator row = weight row within the tile
    const int up_row = lane & 1;
    int j = 0;
    for (int item = pair; item < total; item += n_pairs, ++j) {
      const Coords c = coords(item);
      const int buf = j & 1, rr = j >> 1;
      const int eg = c.e % a.weight_mod;
      const int pos_base = a.offsets[c.e] + c.n0;
      // one thread waits; the four epilogue warps follow its verdict together
      if (ew == 0 && lane == 0) {
        epi_ok = mbar_wait_cl(&acc_full[buf], rr & 1, a.err, 4);
        // the MMAs of the item are done in both CTAs' TMEM: tell rank 1
        if (epi_ok && rank == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&acc_full[buf]), 1));
      }
      named_bar_sync(1, kEpiWarps * 32);
      const bool ok = epi_ok != 0;
      if (GEMM == 1)  // every warp is past the previous item: refill the column scales
        for (int col = ew * 32 + lane; col < BN; col += kEpiWarps * 32)
          col_scale[col] = col < c.nvalid ? a.pos_scale[pos_base + col] : 0.f;
      named_bar_sync(1, kEpiWarps * 32);
      if (!ok) break;
      tc_fence_after();
      const int R = c.m0 + (int)rank * BM + r;
      const float bias_own = R < a.rows ? bf16_to_f32(a.bias[(size_t)eg * a.rows + R]) : 0.f;
      const float bias_other = __shfl_xor_sync(0xFFFFFFFFu, bias_own, 1);
      const float bg = up_row ? bias_other : bias_own, bu = up_row ? bias_own : bias_other;
      const bool row_ok = R < a.rows;

      // one 32-column chunk of the accumulator, straight to global memory
      auto process = [&](const uint32_t(&v)[32], int c0) {
        const int ncol = min(32, c.nvalid - c0);
        if (GEMM == 2) {
          if (row_ok) {
            float *dst = (a.y_seg ? a.y_seg[c.e] + (size_t)(c.n0 + c0) * a.H
                                  : a.y_slot + (size_t)(pos_base + c0) * a.H) + R;
#pragma unroll
            for (int cc = 0; cc < 32; ++cc)
              if (cc < ncol) dst[(size_t)cc * a.H] = __uint_as_float(v[cc]) + bias_own;
          }
        } else {
          // Gate (even lane) and up (odd lane) rows of pair R / 2: for each
          // column pair the even lane finishes the even column and the odd
          // lane the odd one, so all 32 lanes run the SwiGLU together. Each
          // store writes 16 consecutive f16 of two token rows.
          const size_t cstride = (size_t)a.I;
          uint16_t *hh = a.h_hi + (size_t)(pos_base + c0) * cstride + (R >> 1);
          uint16_t *hl = a.h_lo + (size_t)(pos_base + c0) * cstride + (R >> 1);
#pragma unroll
          for (int cp = 0; cp < 16; ++cp) {
            const float ve = __uint_as_float(v[2 * cp]), vo = __uint_as_float(v[2 * cp + 1]);
            const float oe = __shfl_xor_sync(0xFFFFFFFFu, ve, 1);
            const float oo = __shfl_xor_sync(0xFFFFFFFFu, vo, 1);
            const int cc = 2 * cp + up_row;
            const float sc = col_scale[c0 + cc];
            const float g = up_row ? oo : ve, u = up_row ? vo : oe;
            const float hv = swiglu_clamped_fast(fmaf(g, sc, bg), fmaf(u, sc, bu), a.alpha, a.limit);
            const uint32_t hi2 = pack_f16x2(hv, 0.f);
            const uint32_t lo2 = pack_f16x2(hv - unpack_f16x2(hi2).x, 0.f);
            if (row_ok && cc < ncol) {
              hh[(size_t)cc * cstride] = (uint16_t)(hi2 & 0xFFFFu);
              hl[(size_t)cc * cstride] = (uint16_t)(lo2 & 0xFFFFu);
            }
          }
        }
      };
      // this warp's chunks start at 32 * half, 64 columns apart (the other
      // warp of the lane quarter takes the ones in between)
      const uint32_t tbase = tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(buf * BN);
      for (int c0 = 32 * half; c0 < c.nvalid; c0 += 64) {
        uint32_t v[32];
        tmem_ld_32_async(tbase + (uint32_t)c0, v);
        tmem_wait_ld(v);
        process(v, c0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&acc_empty[buf]), 0));
      if (GEMM == 2 && a.y) {
        // Fused weighted top-k combine (src/moe.rs:90-96). Each (token,
        // 128-row tile of H) has an arrival counter; the CTA that stores the
        // last of the token's k slot rows for its 128 rows sums the k rows in
        // j order with the combine's arithmetic (so the result does not
        // depend on which CTA came last) and resets the counter to zero for
        // the next call. The accumulator buffer is already released, so the
        // MMAs of the next item overlap this.
        const int f0 = c.m0 + (int)rank * BM;
        __threadfence();  // this thread's slot-row stores before the arrivals
        if (ew == 0 && lane == 0) comb_n = 0;
        named_bar_sync(1, kEpiWarps * 32);
        const int col = ew * 32 + lane;
        if (f0 < a.rows && col < c.nvalid) {
          const int t = a.perm[pos_base + col] / a.topk;
          uint32_t *cnt = a.comb_cnt + (size_t)t * ((a.rows + BM - 1) / BM) + f0 / BM;
          if (atomicAdd(cnt, 1u) == (uint32_t)a.topk - 1u) {
            *cnt = 0u;
            comb_tok[atomicAdd(&comb_n, 1)] = t;
          }
        }
        __threadfence();  // the other CTAs' rows are visible past the arrivals
        named_bar_sync(1, kEpiWarps * 32);
        const int nf = min(BM, a.rows - f0);  // a multiple of 64
        const int n_comb = comb_n, K = a.topk;  // K <= kCombMaxK (checked at launch)
        // Two tokens per warp and round: lanes 4u + j fetch slot j's position
        // and weight of token u, then every lane issues the 2 x K row loads
        // of its 4 features before the first use, so a round costs two
        // memory round trips whatever K is.
        for (int i0 = 2 * ew; i0 < n_comb; i0 += 2 * kEpiWarps) {
          const int mu = lane >> 2, mj = lane & 3;
          int mp = -1;
          float mw = 0.f;
          if (lane < 8 && i0 + mu < n_comb && mj < K) {
            const int t = comb_tok[i0 + mu];
            mp = a.slot_pos[t * K + mj];
            mw = a.wts[t * K + mj];
          }
          const bool cols_ok = 4 * lane < nf;
          float4 v[2][kCombMaxK];
          int pj[2][kCombMaxK];
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int jj = 0; jj < kCombMaxK; ++jj) {
              pj[u][jj] = __shfl_sync(0xFFFFFFFFu, mp, 4 * u + jj);
              v[u][jj] = pj[u][jj] >= 0 && cols_ok
                             ? __ldcg(reinterpret_cast<const float4 *>(a.y_slot + (size_t)pj[u][jj] * a.H + f0) + lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            float wj[kCombMaxK];
#pragma unroll
            for (int jj = 0; jj < kCombMaxK; ++jj) wj[jj] = __shfl_sync(0xFFFFFFFFu, mw, 4 * u + jj);
            if (i0 + u >= n_comb || !cols_ok) continue;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int jj = 0; jj < kCombMaxK; ++jj) {
              if (pj[u][jj] < 0) continue;  // j >= K, or an unrouted slot
              acc.x = fmaf(wj[jj], v[u][jj].x, acc.x);
              acc.y = fmaf(wj[jj], v[u][jj].y, acc.y);
              acc.z = fmaf(wj[jj], v[u][jj].z, acc.z);
              acc.w = fmaf(wj[jj], v[u][jj].w, acc.w);
            }
            reinterpret_cast<float4 *>(a.y + (size_t)comb_tok[i0 + u] * a.H + f0)[lane] = acc;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs, loads and remote arrives are all done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// x rows in slot-position order, as f16 x * 2^-sigma (exact for bf16 input
// within the token's range, see router.cu), plus the per-position 2^sigma.
__global__ void __launch_bounds__(256) gather_f16_kernel(const uint16_t *__restrict__ x,
                                                         const int32_t *__restrict__ perm,
                                                         const int32_t *__restrict__ sigma,
                                                         int S, int H, int topk,
                                                         uint16_t *__restrict__ xp,
                                                         float *__restrict__ pos_scale, int *err) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < S; p += gridDim.x * warps) {
    const int t = perm[p] / topk;
    const int sg = sigma[t];
    const float inv = __uint_as_float((uint32_t)(127 - sg) << 23);
    if (lane == 0) pos_scale[p] = __uint_as_float((uint32_t)(127 + sg) << 23);
    if (misaligned((uint64_t)(x + (size_t)t * H), 16, err, 108) ||
        misaligned((uint64_t)(xp + (size_t)p * H), 8, err, 109))
      continue;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t * H);
    uint2 *dst = reinterpret_cast<uint2 *>(xp + (size_t)p * H);
    for (int c = lane; c < H / 8; c += 32) {
      const uint4 v = src[c];
      const uint32_t o0 = pack_f16x2(bf16_to_f32(v.x & 0xFFFFu) * inv, bf16_to_f32(v.x >> 16) * inv);
      const uint32_t o1 = pack_f16x2(bf16_to_f32(v.y & 0xFFFFu) * inv, bf16_to_f32(v.y >> 16) * inv);
      const uint32_t o2 = pack_f16x2(bf16_to_f32(v.z & 0xFFFFu) * inv, bf16_to_f32(v.z >> 16) * inv);
      const uint32_t o3 = pack_f16x2(bf16_to_f32(v.w & 0xFFFFu) * inv, bf16_to_f32(v.w >> 16) * inv);
      dst[2 * c] = make_uint2(o0, o1);
      dst[2 * c + 1] = make_uint2(o2, o3);
    }
  }
}

// min (over non-zero codes) and max of E8M0 scale bytes
__global__ void scale_range_kernel(const uint8_t *__restrict__ s, size_t n,
                                   unsigned *__restrict__ out) {
  unsigned lo = 255u, hi = 0u;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const unsigned v = s[i];
    if (v) lo = min(lo, v);
    hi = max(hi, v);
  }
  atomicMin(out, lo);
  atomicMax(out + 1, hi);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [rows, cols] f16 row-major matrix, box [64 cols, box_rows], 128-byte swizzle.
cudaError_t make_tmap(CUtensorMap *m, const void *base, size_t rows, int cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int GEMM, int STAGES>
size_t gemm_smem_bytes() {
  constexpr int NB = GEMM == 1 ? 1 : 2;
  return 1024 + (size_t)STAGES * (BM * BK * 2 + NB * BNH * BK * 2);
}

// Persistent grid of CTA pairs: as many clusters of 2 as fit at once (asked of
// the occupancy calculator once per device and kernel).
template <int GEMM, int STAGES>
cudaError_t launch_gemm(const CUtensorMap &m0, const CUtensorMap &m1, const PrefillArgs &a,
                        cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes<GEMM, STAGES>();
  auto fn = prefill_gemm_kernel<GEMM, STAGES>;
  cudaError_t st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (st != cudaSuccess) return st;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int pairs_of_device[64] = {0};
  int dev = 0;
  if ((st = cudaGetDevice(&dev)) != cudaSuccess) return st;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (pairs_of_device[dev] == 0) {
    cfg.gridDim = dim3(2);
    int n_clusters = 0;
    st = cudaOccupancyMaxActiveClusters(&n_clusters, fn, &cfg);
    if (st != cudaSuccess) return st;
    if (n_clusters < 1) return cudaErrorLaunchOutOfResources;
    pairs_of_device[dev] = n_clusters;
  }
  cfg.gridDim = dim3(2 * pairs_of_device[dev]);
  return cudaLaunchKernelEx(&cfg, fn, m0, m1, a);
}

}  // namespace

cudaError_t launch_scale_range(const uint8_t *scales, size_t n, unsigned *minmax,
                               cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  scale_range_kernel<<<148 * 4, 256, 0, stream>>>(scales, n, minmax);
  return cudaGetLastError();
}

cudaError_t launch_gather_f16(const uint16_t *x, const int32_t *perm, const int32_t *sigma, int S,
                              int H, int topk, uint16_t *xp, float *pos_scale, int *err,
                              cudaStream_t stream) {
  if (S == 0) return cudaSuccess;
  const int warps = 8;
  int grid = (S + warps - 1) / warps;
  if (grid > 148 * 16) grid = 148 * 16;
  gather_f16_kernel<<<grid, warps * 32, 0, stream>>>(x, perm, sigma, S, H, topk, xp, pos_scale,
                                                     err);
  return cudaGetLastError();
}

cudaError_t launch_prefill_mlp1(const MoeDeviceWeights &w, const PrefillIO &io, int n_sms,
                                cudaStream_t stream) {
  if (io.S == 0) return cudaSuccess;
  if (w.H % BK || w.I % BK || io.n_segments > kMaxExpertsP || io.n_segments < 1 ||
      io.weight_mod < 1)
    return cudaErrorInvalidValue;
  // the converters load 8-byte code words and 2-byte scale pairs, the
  // epilogue stores 4-byte h pairs
  if (((uintptr_t)w.w1 & 15) || ((uintptr_t)io.h_hi & 3) || ((uintptr_t)io.h_lo & 3))
    return cudaErrorInvalidValue;
  CUtensorMap m0, m1;
  cudaError_t st = make_tmap(&m0, io.xp, io.S, w.H, BNH);
  if (st != cudaSuccess) return st;
  m1 = m0;
  PrefillArgs a{};
  a.codes = w.w1;
  a.bias = w.b1;
  a.K = w.H;
  a.rows = 2 * w.I;
  a.item_bytes = tile_item_bytes(w.H);
  a.pair_adj = 1;
  a.counts = io.counts;
  a.offsets = io.offsets;
  a.n_segments = io.n_segments;
  a.weight_mod = io.weight_mod;
  a.pos_scale = io.pos_scale;
  a.h_hi = io.h_hi;
  a.h_lo = io.h_lo;
  a.I = w.I;
  a.alpha = w.alpha;
  a.limit = w.limit;
  a.H = w.H;
  a.err = io.err;
  (void)n_sms;
  return launch_gemm<1, 6>(m0, m1, a, stream);
}

cudaError_t launch_prefill_mlp2(const MoeDeviceWeights &w, const PrefillIO &io, int n_sms,
                                cudaStream_t stream) {
  if (io.S == 0) return cudaSuccess;
  if (w.H % BK || w.I % BK || io.n_segments > kMaxExpertsP || io.n_segments < 1 ||
      io.weight_mod < 1)
    return cudaErrorInvalidValue;
  if ((uintptr_t)w.w2 & 15) return cudaErrorInvalidValue;
  CUtensorMap m0, m1;
  cudaError_t st = make_tmap(&m0, io.h_hi, io.S, w.I, BNH);
  if (st != cudaSuccess) return st;
  st = make_tmap(&m1, io.h_lo, io.S, w.I, BNH);
  if (st != cudaSuccess) return st;
  PrefillArgs a{};
  a.codes = w.w2;
  a.bias = w.b2;
  a.K = w.I;
  a.rows = w.H;
  a.item_bytes = tile_item_bytes(w.I);
  a.pair_adj = 0;
  a.counts = io.counts;
  a.offsets = io.offsets;
  a.n_segments = io.n_segments;
  a.weight_mod = io.weight_mod;
  a.y_slot = io.y_slot;
  a.y_seg = io.y_seg;
  a.I = w.I;
  a.H = w.H;
  a.err = io.err;
  if (io.y) {  // fused combine: one GPU's slot rows only, float4 rows
    if (io.y_seg || !io.y_slot || !io.perm || !io.slot_pos || !io.wts || !io.comb_cnt || io.topk < 1 ||
        io.topk > kCombMaxK ||
        ((uintptr_t)io.y & 15) || ((uintptr_t)io.y_slot & 15))
      return cudaErrorInvalidValue;
    a.y = io.y;
    a.perm = io.perm;
    a.slot_pos = io.slot_pos;
    a.wts = io.wts;
    a.comb_cnt = io.comb_cnt;
    a.topk = io.topk;
  }
  (void)n_sms;
  return launch_gemm<2, 4>(m0, m1, a, stream);
}

}  // namespace oxg
