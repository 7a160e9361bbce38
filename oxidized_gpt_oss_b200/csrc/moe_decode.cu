// moe_decode.cu — MoE expert kernels for small token counts (decode):
// in-register MXFP4 dequantisation feeding warp-level f16 tensor-core MMAs.
//
// Reference computation (MLP::forward, src/model.rs:1088-1184, called per
// (token, expert) from src/moe.rs:81-93), with the gpt-oss layout and
// activation (mlp1 rows interleaved gate/up, clamped SwiGLU):
//   h1 = x . W1^T + b1          W1 [2I, H]; gate = even rows, up = odd rows
//   h  = swiglu(gate, up)       alpha, limit
//   y  = h . W2^T + b2          W2 [H, I]
//
// Design (HBM-bound: every expert weight byte is read once per step):
//  * A warp computes 16 weight rows x 8 token columns with mma.m16n8k16
//    (f16 in, f32 out); CTAs are 16 warps, one per SM.
//  * Weights stream from HBM in the tile-chunk order of relayout.cu: a 16-row
//    tile is one contiguous run, 1088 bytes (codes + scales) per 128-element
//    group, and one 16-byte copy per lane and row half gives a lane the
//    A-operand codes of all four blocks of the group. Each warp runs one
//    continuous cp.async pipeline through a shared-memory ring (6 groups in
//    flight per lane) across all the tiles it processes, so HBM latency is
//    covered without holding registers and without a refill gap between
//    tiles. cvt.rn.f16x2.e2m1x2 turns two codes into two exact f16 values;
//    the E8M0 scale of each 32-element block multiplies that block's f32 MMA
//    result (an exact power of two).
//  * The per-lane K order inside a block is permuted consistently on A (by the
//    byte order of the code word) and B (by the shared-memory "fragment order"
//    of the activations), so no shuffles are needed.
//  * mlp1: A rows g and g+8 of a tile are the gate and up rows of one
//    intermediate unit, so a lane holds both and applies bias + clamped SwiGLU
//    in registers. x enters as f16 x * 2^-sigma (exact for bf16 input) and the
//    products are scaled back by 2^sigma. With at most 8 tokens, all tokens
//    are staged once per CTA and every tile computes all 8 columns (the MMA
//    has 8 columns either way), so any warp can take any (expert, tile) and a
//    persistent grid keeps every SM busy; the epilogue keeps the columns of
//    the tokens routed to the tile's expert.
//  * mlp2: the f32 SwiGLU output is split into f16 hi + lo (h = hi + lo to
//    ~2^-22 relative), so the intermediate is not rounded to 16 bits. For an
//    expert with at most 4 tokens, hi and lo of token j sit in MMA columns 2j
//    and 2j+1 (one MMA per k-step); otherwise each half takes its own MMA.
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace oxg {
namespace {

// Per-warp ring of weight groups in flight: STAGES slots of one group's
// chunk (2 row halves x 32 lanes x 16 B of codes + 64 B of scales).
constexpr int kStageBytes = 1088;
// CTA shapes (warps, ring stages): the all-token mlp1 kernel, the per-expert
// kernel (mlp1 above 8 tokens, mlp2 above 8 tokens) and mlp2 for at most 8
// tokens (persistent grid, packed h stage).
#ifndef OXG_DEC_W1
#define OXG_DEC_W1 28
#define OXG_DEC_S1 5
#endif
#ifndef OXG_DEC_W2
#define OXG_DEC_W2 16
#define OXG_DEC_S2 6
#endif
#ifndef OXG_DEC_BULK
#define OXG_DEC_BULK 0
#endif
constexpr bool kBulk = OXG_DEC_BULK != 0;
#ifndef OXG_DEC_W3
#define OXG_DEC_W3 32
#define OXG_DEC_S3 5
#endif
constexpr int kW1 = OXG_DEC_W1, kS1 = OXG_DEC_S1;
constexpr int kW2 = OXG_DEC_W2, kS2 = OXG_DEC_S2;
constexpr int kW3 = OXG_DEC_W3, kS3 = OXG_DEC_S3;  // mlp2 with at most 8 tokens
// At most kDeepTokens tokens (4-8 active experts): each tile's K is split
// over 4 warps — mlp1 28 warps x 5 stages (7 tiles in flight per SM), mlp2
// 20 x 7 (5 tiles, a band being ~5 tiles of one expert).
#ifndef OXG_DEEP_TOKENS
#define OXG_DEEP_TOKENS 2
#endif
constexpr int kDeepTokens = OXG_DEEP_TOKENS;
// mlp1: 5 groups of 4 warps splitting K, 7 ring stages each. At one token
// (4 experts x 360 tiles) 5 groups per SM take 1440 / 740 = 1.95 rounds of
// tiles (7 groups: 1.39 rounds, the second mostly idle): 18.9 against 21.0 us.
constexpr int kW1d = 20, kS1d = 7, kK1d = 4;
constexpr int kW3d = 20, kS3d = 7, kK3d = 4;  // mlp2: 5 groups of 4 warps splitting K
constexpr int kMaxAllTokActive = 128;  // active experts of an all-token mlp1 launch (T*k <= 128)
// Flat-split kernels: warps x ring stages per CTA, one CTA per SM. mlp1
// stages 8 activation rows, mlp2 16 (two column groups of four slots' hi / lo
// halves); the rest of shared memory is the warps' rings.
#ifndef OXG_FLAT_W1
#define OXG_FLAT_W1 24
#define OXG_FLAT_S1 6
#endif
#ifndef OXG_FLAT_W2B
#define OXG_FLAT_W2B 20
#define OXG_FLAT_S2B 6
#endif
constexpr int kWf1 = OXG_FLAT_W1, kSf1 = OXG_FLAT_S1;
constexpr int kWf2b = OXG_FLAT_W2B, kSf2b = OXG_FLAT_S2B;
#ifndef OXG_DEC_FLAT
#define OXG_DEC_FLAT 1
#endif
// Token counts from which mlp2 runs the flat-split kernel over virtual
// experts (below: the persistent per-expert band kernel).
#ifndef OXG_FLAT2_MIN_TOKENS
#define OXG_FLAT2_MIN_TOKENS 9
#endif
constexpr bool kUseFlat = OXG_DEC_FLAT != 0;
constexpr size_t kMaxFlatSmem = 220 * 1024;  // dynamic shared memory (static arrays take the rest of 227 KB)

struct DecodeArgs {
  const uint8_t *codes;   // tile chunks of [E, rows, K] (codes + scales)
  const uint16_t *bias;   // [E, rows] bf16
  int K, rows;
  size_t item_bytes;      // bytes of one 16-row tile
  // mlp1 input: x [T, K] bf16, token of position p = perm[p] / topk
  const uint16_t *x;
  const int32_t *perm;
  const int32_t *sigma;
  const int32_t *idx;  // routing [T, topk] (all-token mlp1)
  int topk;
  // mlp2 input: h [n_slots, K] f32 in position order
  const float *h;
  const int32_t *counts, *offsets;
  int expert_base;
  float *out;  // mlp1: h [n_slots, I]; mlp2: y_slot [n_slots, H]
  int out_ld;
  float alpha, limit;
  // scheduling: blockIdx.y indexes `active` (ids of experts with tokens,
  // *n_active of them) when it is set, else expert_base + blockIdx.y;
  // blockIdx.x is one of `bands` equal bands of an expert's 16-row tiles
  const int32_t *active, *n_active;
  int bands;
  // dyn_bands: a 1-D grid of gridDim.x CTAs split on the device into
  // min(tiles, gridDim.x / n_active) bands per active expert (every SM busy
  // whatever the number of active experts); `bands` is then unused
  int dyn_bands;
  int pdl;  // launched as a programmatic dependent: wait before reading inputs
  int T;
  // mlp2 only: fused weighted combine when band_done is set
  uint32_t *band_done;
  const int32_t *slot_pos;
  const float *wts;
  float *y;
  int *err;  // error word: bounded waits that ran out record their code here
  // flat split (flat kernels): per grid warp two float4 x 32 partial-sum
  // slots, and per grid warp one arrival counter (zero between launches)
  float4 *parts;
  uint32_t *flat_cnt;
  // grouped kernels: virtual experts (expert id, first position, slot count
  // of each group of at most kVirtualTokens slots, and their number)
  const int32_t *v_expert, *v_pos0, *v_count, *n_virtual;
  // received-rows mode (expert parallelism): mlp1 reads f16 rows x * 2^-sigma
  // [pos, K] with their 2^sigma instead of gathering x through perm, and mlp2
  // writes each group's rows from v_out[group] (another rank's return rows)
  const uint16_t *xrows;
  const float *row_scale;
  float *const *v_out;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Byte offset of the 8-element group (n-tile nt, block blk, half s, token g,
// lane-in-quad q) in the fragment-ordered activation buffer.
__device__ __forceinline__ int frag_off(int nt, int nb, int blk, int s, int g, int q, int bytes) {
  return ((((nt * nb + blk) * 2 + s) * 8 + g) * 4 + q) * bytes;
}

// A warp's ring of STAGES group slots. Bulk mode: lane 0 fetches each group
// chunk with one cp.async.bulk (TMA engine) that completes on the slot's
// mbarrier; phase holds the parity each slot waits for next. Otherwise the
// lanes copy their own 16-byte pieces with cp.async.
struct WarpRing {
  uint8_t *ring;
  uint64_t *bars;
  uint32_t phase;
};
constexpr int kErrDecodeWait = 21;  // error word: a decode weight copy did not land

// Streams the chunks of n_items 16-row tiles through the warp's ring.
// item_ptr(i) gives the first byte of item i's tile; group_fn(blk0, nblk,
// wa, wb, sxa, sxb) consumes one group of nblk <= 4 blocks starting at block
// blk0 (the code words of the lane's rows a/b per block, and their four scale
// bytes); done_fn(i) runs after the last group of item i. Returns
// false (error word set) if a bulk copy did not complete within the wait
// budget; the copies still in flight have then been waited for (bounded).
template <int STAGES, bool BULK, class ItemPtr, class GroupFn, class DoneFn>
__device__ __forceinline__ bool stream_items(int n_items, int K, WarpRing &wr, int *err, ItemPtr item_ptr,
                                             GroupFn group_fn, DoneFn done_fn, int g_begin = 0,
                                             int g_count = -1) {
  if (n_items <= 0) return true;
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const int nb = K / 32, full = nb / 4, tail = nb % 4, ngroups = full + (tail ? 1 : 0);
  // groups [g_begin, g_begin + ng) of every item (all of them by default)
  const int ng = g_count < 0 ? ngroups - g_begin : g_count;
  if (ng <= 0) {  // an empty share of K: nothing to stream, partial sums stay zero
    for (int i = 0; i < n_items; ++i) done_fn(i);
    return true;
  }
  const uint32_t tail_bytes = 256u * tail + 64u;
  // Issue side: runs STAGES groups ahead of the consumer.
  int i_item = 0, i_grp = 0, i_slot = 0, pending = 0;
  const uint8_t *ip = item_ptr(0);
  auto issue_next = [&]() {
    if (i_item < n_items) {
      uint8_t *st = wr.ring + i_slot * kStageBytes;
      const uint8_t *ch = ip + (size_t)(g_begin + i_grp) * 1088;
      if (BULK) {
        if (lane == 0) {
          const uint32_t bytes = g_begin + i_grp < full ? 1088u : tail_bytes;
          sm100::mbar_arrive_expect_tx(&wr.bars[i_slot], bytes);
          sm100::bulk_copy(st, ch, bytes, &wr.bars[i_slot]);
        }
        ++pending;
      } else if (g_begin + i_grp < full) {
        cp_async_16(st + lane * 16, ch + lane * 16);
        cp_async_16(st + 512 + lane * 16, ch + 512 + lane * 16);
        if (lane < 4) cp_async_16(st + 1024 + lane * 16, ch + 1024 + lane * 16);
      } else {
        for (int b = 0; b < tail; ++b) {
          cp_async_4(st + lane * 16 + b * 4, ch + lane * 4 * tail + b * 4);
          cp_async_4(st + 512 + lane * 16 + b * 4, ch + 128 * tail + lane * 4 * tail + b * 4);
        }
        if (lane < 4) cp_async_16(st + 1024 + lane * 16, ch + 256 * tail + lane * 16);
      }
      if (++i_grp == ng) {
        i_grp = 0;
        if (++i_item < n_items) ip = item_ptr(i_item);
      }
    }
    if (!BULK) cp_async_commit();
    if (++i_slot == STAGES) i_slot = 0;
  };
#pragma unroll
  for (int u = 0; u < STAGES; ++u) issue_next();
  int c_item = 0, c_grp = 0, c_slot = 0;
  bool ok = true;
#pragma unroll 1
  while (c_item < n_items) {
    const uint8_t *st = wr.ring + c_slot * kStageBytes;
    uint32_t wa[4], wb[4], sxa, sxb;
    if (BULK) {
      const bool landed = sm100::mbar_wait(&wr.bars[c_slot], (wr.phase >> c_slot) & 1u, err, kErrDecodeWait);
      if (!__all_sync(0xFFFFFFFFu, landed)) {
        ok = false;
        break;
      }
      wr.phase ^= 1u << c_slot;
      --pending;
      // a bulk copy lands the chunk as stored: narrow groups keep their
      // packed layout (4 * tail bytes per lane and row half)
      if (g_begin + c_grp < full) {
        const uint4 va = *reinterpret_cast<const uint4 *>(st + lane * 16);
        const uint4 vb = *reinterpret_cast<const uint4 *>(st + 512 + lane * 16);
        wa[0] = va.x; wa[1] = va.y; wa[2] = va.z; wa[3] = va.w;
        wb[0] = vb.x; wb[1] = vb.y; wb[2] = vb.z; wb[3] = vb.w;
        sxa = *reinterpret_cast<const uint32_t *>(st + 1024 + g * 4);
        sxb = *reinterpret_cast<const uint32_t *>(st + 1056 + g * 4);
      } else {
#pragma unroll
        for (int b = 0; b < 3; ++b) {
          wa[b] = b < tail ? *reinterpret_cast<const uint32_t *>(st + lane * 4 * tail + 4 * b) : 0u;
          wb[b] = b < tail ? *reinterpret_cast<const uint32_t *>(st + 128 * tail + lane * 4 * tail + 4 * b) : 0u;
        }
        wa[3] = wb[3] = 0u;
        sxa = *reinterpret_cast<const uint32_t *>(st + 256 * tail + g * 4);
        sxb = *reinterpret_cast<const uint32_t *>(st + 256 * tail + 32 + g * 4);
      }
      // the slot's reads are done before the async proxy refills it
      sm100::fence_proxy_async_smem();
      __syncwarp();
    } else {
      cp_async_wait<STAGES - 1>();
      const uint4 va = *reinterpret_cast<const uint4 *>(st + lane * 16);
      const uint4 vb = *reinterpret_cast<const uint4 *>(st + 512 + lane * 16);
      wa[0] = va.x; wa[1] = va.y; wa[2] = va.z; wa[3] = va.w;
      wb[0] = vb.x; wb[1] = vb.y; wb[2] = vb.z; wb[3] = vb.w;
      sxa = *reinterpret_cast<const uint32_t *>(st + 1024 + g * 4);
      sxb = *reinterpret_cast<const uint32_t *>(st + 1056 + g * 4);
    }
    issue_next();
    if (g_begin + c_grp < full)
      group_fn((g_begin + c_grp) * 4, 4, wa, wb, sxa, sxb);
    else
      group_fn((g_begin + c_grp) * 4, tail, wa, wb, sxa, sxb);
    if (++c_grp == ng) {
      done_fn(c_item);
      c_grp = 0;
      ++c_item;
    }
    if (++c_slot == STAGES) c_slot = 0;
  }
  if (BULK) {
    // after a failed wait: the copies still in flight land (or time out)
    // before the warp leaves, so none writes into a reused shared buffer
    for (; pending > 0; --pending) {
      sm100::mbar_wait(&wr.bars[c_slot], (wr.phase >> c_slot) & 1u, err, kErrDecodeWait);
      wr.phase ^= 1u << c_slot;
      if (++c_slot == STAGES) c_slot = 0;
    }
    __syncwarp();
  } else {
    cp_async_wait<0>();
  }
  return ok;
}

// Per-warp barriers of the bulk ring: initialised once per CTA by the warp's
// lane 0 (all phases start at parity 0).
template <int STAGES>
__device__ __forceinline__ WarpRing make_ring(uint8_t *ring, uint64_t *bars) {
  if ((threadIdx.x & 31) == 0)
    for (int u = 0; u < STAGES; ++u) sm100::mbar_init(&bars[u], 1);
  sm100::fence_mbar_init();
  __syncwarp();
  return WarpRing{ring, bars, 0u};
}

// Decodes two rows' code words into the m16n8k16 A operands of the block's
// two k-steps.
__device__ __forceinline__ void a_operands(uint32_t wa, uint32_t wb, uint32_t (&A0)[4],
                                           uint32_t (&A1)[4]) {
  uint32_t fa[4], fb[4];
  e2m1x8_to_f16x8(wa, fa);
  e2m1x8_to_f16x8(wb, fb);
  A0[0] = fa[0]; A0[1] = fb[0]; A0[2] = fa[1]; A0[3] = fb[1];
  A1[0] = fa[2]; A1[1] = fb[2]; A1[2] = fa[3]; A1[3] = fb[3];
}

// One group of nblk <= 4 blocks against n-tile nt of the staged activations
// (KF bytes per fragment: 8 = one f16 pair per k-step, 16 = f16 hi and lo
// pairs), block by block: decode the A operands, the block's MMAs, then its
// E8M0 scales applied in f32. (Decoding all four blocks first and running
// their MMA chains side by side measured slower: 55 vs 52 us for mlp1.)
template <int KF>
__device__ __forceinline__ void mma_group(const uint8_t *bsm, int nb, int nt, int blk0, int nblk,
                                          const uint32_t (&wa)[4], const uint32_t (&wb)[4], uint32_t sxa,
                                          uint32_t sxb, int g, int q, float (&acc)[4]) {
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int b = 0; b < 4; ++b)
    if (b < nblk) {
      const int blk = blk0 + b;
      uint32_t A0[4], A1[4];
      a_operands(wa[b], wb[b], A0, A1);
      float d[4];
      if (KF == 8) {
        const uint2 b0 = *reinterpret_cast<const uint2 *>(bsm + frag_off(nt, nb, blk, 0, g, q, 8));
        const uint2 b1 = *reinterpret_cast<const uint2 *>(bsm + frag_off(nt, nb, blk, 1, g, q, 8));
        mma_f16_16816(d, A0, b0.x, b0.y, zero4);
        mma_f16_16816(d, A1, b1.x, b1.y, d);
      } else {
        const uint4 b0 = *reinterpret_cast<const uint4 *>(bsm + frag_off(nt, nb, blk, 0, g, q, 16));
        const uint4 b1 = *reinterpret_cast<const uint4 *>(bsm + frag_off(nt, nb, blk, 1, g, q, 16));
        mma_f16_16816(d, A0, b0.x, b0.y, zero4);
        mma_f16_16816(d, A0, b0.z, b0.w, d);
        mma_f16_16816(d, A1, b1.x, b1.y, d);
        mma_f16_16816(d, A1, b1.z, b1.w, d);
      }
      const float s_a = e8m0_to_f32(sxa >> (8 * b)), s_b = e8m0_to_f32(sxb >> (8 * b));
      acc[0] = fmaf(s_a, d[0], acc[0]);
      acc[1] = fmaf(s_a, d[1], acc[1]);
      acc[2] = fmaf(s_b, d[2], acc[2]);
      acc[3] = fmaf(s_b, d[3], acc[3]);
    }
}

// Stages tokens [tok0, tok0 + n) of x (rows of `x` given by row_of(tok))
// as f16 x * 2^-sigma into fragment order, 8 tokens per n-tile; tokens
// beyond `valid` are zero.
template <int NT, class RowOf>
__device__ __forceinline__ void stage_x(const DecodeArgs &a, uint8_t *smem, int nb, int valid,
                                        RowOf row_of, const int32_t *sigma) {
  const int K = a.K;
  const int units = NT * 8 * (K / 8);
#pragma unroll 4
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int tok = u / (K / 8), k0 = (u % (K / 8)) * 8;
    const int blk = k0 >> 5, qq = (k0 & 31) >> 3, nt = tok >> 3, gg = tok & 7;
    uint32_t o0 = 0, o1 = 0, o2 = 0, o3 = 0;
    if (tok < valid) {
      const int t = row_of(tok);
      const float inv = __uint_as_float((uint32_t)(127 - sigma[t]) << 23);
      const uint4 v = *reinterpret_cast<const uint4 *>(a.x + (size_t)t * K + k0);
      o0 = pack_f16x2(bf16_to_f32(v.x & 0xFFFFu) * inv, bf16_to_f32(v.x >> 16) * inv);
      o1 = pack_f16x2(bf16_to_f32(v.y & 0xFFFFu) * inv, bf16_to_f32(v.y >> 16) * inv);
      o2 = pack_f16x2(bf16_to_f32(v.z & 0xFFFFu) * inv, bf16_to_f32(v.z >> 16) * inv);
      o3 = pack_f16x2(bf16_to_f32(v.w & 0xFFFFu) * inv, bf16_to_f32(v.w >> 16) * inv);
    }
    *reinterpret_cast<uint2 *>(smem + frag_off(nt, nb, blk, 0, gg, qq, 8)) = make_uint2(o0, o1);
    *reinterpret_cast<uint2 *>(smem + frag_off(nt, nb, blk, 1, gg, qq, 8)) = make_uint2(o2, o3);
  }
}

// ---------------------------------------------------------------------------
// mlp1 over all tokens (T <= 8): persistent grid over (active expert, tile).
// ---------------------------------------------------------------------------
// KS > 1: KS consecutive warps share each tile, warp kq of a group streams
// the kq-th share of K's 128-wide groups; at the end of a tile the partial
// sums meet in shared memory and the group's first warp adds them in warp
// order (the same order every run) and runs the epilogue. At one or two
// tokens there are only ~4 experts x 360 tiles, so this keeps every warp of
// the SM busy instead of one warp per tile.
template <int WARPS, int STAGES, int KS = 1>
__global__ void __launch_bounds__(WARPS * 32, 1) mlp1_alltok_kernel(const DecodeArgs a) {
  static_assert(WARPS % KS == 0, "warps come in groups of KS");
  constexpr int kThreads = WARPS * 32;
  constexpr int kGroups = WARPS / KS;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ __align__(16) float red_s[KS > 1 ? WARPS * 32 * 4 : 4];
  __shared__ float tok_scale[8];
  __shared__ int act_s[kMaxAllTokActive];
  __shared__ int act_of[256];
  __shared__ int col_pos[kMaxAllTokActive * 8];  // position of (active expert, token), or -1
  __shared__ uint64_t ring_bars[WARPS * STAGES];

  if (a.pdl) pdl_wait();
  const int K = a.K, nb = K / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int T = a.T, k = a.topk;
  const int n_act = *a.n_active;
  const int n_tiles = a.rows / 16;

  for (int i = tid; i < n_act; i += kThreads) {
    act_s[i] = a.active[i];
    act_of[a.active[i]] = i;
  }
  for (int i = tid; i < n_act * 8; i += kThreads) col_pos[i] = -1;
  stage_x<1>(a, smem, nb, T, [](int tok) { return tok; }, a.sigma);
  if (tid < 8) tok_scale[tid] = tid < T ? __uint_as_float((uint32_t)(127 + a.sigma[tid]) << 23) : 1.f;
  __syncthreads();
  for (int p = tid; p < T * k; p += kThreads) {
    const int s = a.perm[p];
    col_pos[act_of[a.idx[s]] * 8 + s / k] = p;
  }
  __syncthreads();
  if (a.pdl) pdl_launch();

  const int gw = warp / KS, kq = warp % KS;
  const int W = gridDim.x * kGroups, wg = blockIdx.x * kGroups + gw;
  const int total = n_act * n_tiles;
  const int n_items = wg < total ? (total - wg + W - 1) / W : 0;
  const int n_grp = nb / 4 + (nb % 4 ? 1 : 0);
  const int g_begin = kq * n_grp / KS, g_end = (kq + 1) * n_grp / KS;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  auto item_ptr = [&](int i) {
    const int w = wg + i * W, ai = w / n_tiles, tile = w - ai * n_tiles;
    return a.codes + ((size_t)act_s[ai] * n_tiles + tile) * a.item_bytes;
  };
  auto group_fn = [&](int blk0, int nblk, const uint32_t(&wa)[4], const uint32_t(&wb)[4], uint32_t sxa,
                      uint32_t sxb) { mma_group<8>(smem, nb, 0, blk0, nblk, wa, wb, sxa, sxb, g, q, acc); };
  auto done_fn = [&](int i) {
    if constexpr (KS > 1) {
      float4 *slot = reinterpret_cast<float4 *>(red_s) + (gw * KS + kq) * 32 + lane;
      *slot = make_float4(acc[0], acc[1], acc[2], acc[3]);
      asm volatile("bar.sync %0, %1;" ::"r"(1 + gw), "r"(KS * 32) : "memory");
      if (kq == 0) {
        const float4 *g0 = reinterpret_cast<const float4 *>(red_s) + gw * KS * 32 + lane;
        float4 t = g0[0];
#pragma unroll
        for (int r = 1; r < KS; ++r) {
          const float4 v = g0[r * 32];
          t.x += v.x;
          t.y += v.y;
          t.z += v.z;
          t.w += v.w;
        }
        acc[0] = t.x;
        acc[1] = t.y;
        acc[2] = t.z;
        acc[3] = t.w;
      }
      asm volatile("bar.sync %0, %1;" ::"r"(1 + gw), "r"(KS * 32) : "memory");
      if (kq != 0) {
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        return;
      }
    }
    const int w = wg + i * W, ai = w / n_tiles, tile = w - ai * n_tiles;
    const int e = act_s[ai];
    const int pr = tile * 8 + g;  // intermediate unit (gate row 2pr, up row 2pr + 1)
    const float bg = bf16_to_f32(a.bias[(size_t)e * a.rows + 2 * pr]);
    const float bu = bf16_to_f32(a.bias[(size_t)e * a.rows + 2 * pr + 1]);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int t = 2 * q + c;
      const int p = col_pos[ai * 8 + t];
      if (p >= 0) {
        const float gate = fmaf(acc[c], tok_scale[t], bg);
        const float up = fmaf(acc[2 + c], tok_scale[t], bu);
        a.out[(size_t)p * a.out_ld + pr] = swiglu_clamped(gate, up, a.alpha, a.limit);
      }
    }
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  };
  WarpRing wr = make_ring<STAGES>(smem + nb * 2 * 32 * 8 + warp * (STAGES * kStageBytes),
                                  ring_bars + warp * STAGES);
  stream_items<STAGES, kBulk>(n_items, K, wr, a.err, item_ptr, group_fn, done_fn, g_begin, g_end - g_begin);
}

// ---------------------------------------------------------------------------
// Flat split (T <= 8 tokens). The launch's work is one sequence of weight
// chunks — (item, group) with item an (active expert, 16-row tile) and group
// one 128-element step of K — cut into equal contiguous ranges, one per warp
// of the grid, so every warp streams the same number of bytes whatever the
// number of active experts and tiles (a per-tile split leaves the warps of a
// last, partial round idle: at one token 1440 mlp1 tiles over 1036 warp
// groups). An item split between warps is summed by the warp that finishes
// its part last: each part lands in its warp's slot, and the last arrival adds
// the parts in range order — the same order every run, whichever warp is last.
// ---------------------------------------------------------------------------
// Balanced partition in 32-bit arithmetic (64-bit divisions are long
// instruction sequences on the GPU): the first r warps take q + 1 chunks, the
// other W - r take q, with q = C / W and r = C % W.
struct FlatRange {
  int C;  // chunks of the launch (or of one expert)
  int W;  // warps sharing them (<= C)
  int q, r;
  // warp w (< W) streams chunks [first(w), first(w + 1))
  __device__ __forceinline__ int first(int w) const { return w * q + min(w, r); }
  // the warp whose range holds chunk x
  __device__ __forceinline__ int owner(int x) const {
    const int b = r * (q + 1);
    return x < b ? x / (q + 1) : r + (x - b) / q;
  }
  // first(w) for any warp of the grid: warps w >= W (when the grid has more
  // warps than there are chunks) get the empty range [C, C)
  __device__ __forceinline__ int lo(int w) const { return w >= W ? C : first(w); }
};
// At most one warp per chunk, so that every warp of the range has a non-empty
// share and the owners of an item's chunks are consecutive warps.
__device__ __forceinline__ FlatRange flat_range(int chunks, int grid_warps) {
  FlatRange R;
  R.C = chunks;
  R.W = chunks < grid_warps ? (chunks > 0 ? chunks : 1) : grid_warps;
  R.q = chunks / R.W;
  R.r = chunks - R.q * R.W;
  return R;
}

// Arrival on a counter that publishes this warp's earlier stores and, for the
// last arrival, acquires every other arrival's (one atom.acq_rel by lane 0
// after a warp barrier, instead of two full fences).
__device__ __forceinline__ bool arrive_last(uint32_t *cnt, uint32_t n) {
  __syncwarp();
  uint32_t old = 0u;
  if ((threadIdx.x & 31) == 0)
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
  const bool last = __shfl_sync(0xFFFFFFFFu, old, 0) == n - 1;
  __syncwarp();
  return last;
}

// Row pitch (bytes) of an activation stage of K f16 values per row: a
// multiple of 64 that is 64 mod 128, so the eight lanes of one 16-byte
// shared-memory wavefront (two rows x four quarters) hit distinct banks.
__host__ __device__ constexpr int flat_row_pitch(int K) { return (2 * K) % 128 == 0 ? 2 * K + 64 : 2 * K; }

// The E2M1 codes of one word (byte i: codes 2i, 2i + 1, low nibble first)
// as four exact f16x2 values. OXG_E2M1_SHR 1: each byte reaches the
// conversion by a shift of the word; 0: by unpacking the word into bytes.
#ifndef OXG_E2M1_SHR
#define OXG_E2M1_SHR 0
#endif
__device__ __forceinline__ void e2m1_word(uint32_t w, uint32_t (&o)[4]) {
#if OXG_E2M1_SHR
  o[0] = e2m1x2_to_f16x2(w);
  o[1] = e2m1x2_to_f16x2(w >> 8);
  o[2] = e2m1x2_to_f16x2(w >> 16);
  o[3] = e2m1x2_to_f16x2(w >> 24);
#else
  e2m1x8_to_f16x8(w, o);
#endif
}

// The four E8M0 scales of a word (byte b: block b) as f32 powers of two,
// byte << 23 exactly as e8m0_to_f32 (0 -> 0.0, 255 -> +inf).
__device__ __forceinline__ void e8m0x4(uint32_t sx, float (&s)[4]) {
  s[0] = __uint_as_float((sx << 23) & 0x7F800000u);
  s[1] = __uint_as_float((sx << 15) & 0x7F800000u);
  s[2] = __uint_as_float((sx << 7) & 0x7F800000u);
  s[3] = __uint_as_float((sx >> 1) & 0x7F800000u);
}

// The m16n8k16 A operands of one block's two k-steps from the lane's code
// words of rows a and b (see a_operands).
__device__ __forceinline__ void a_ops(uint32_t wa, uint32_t wb, uint32_t (&A0)[4], uint32_t (&A1)[4]) {
  uint32_t fa[4], fb[4];
  e2m1_word(wa, fa);
  e2m1_word(wb, fb);
  A0[0] = fa[0]; A0[1] = fb[0]; A0[2] = fa[1]; A0[3] = fb[1];
  A1[0] = fa[2]; A1[1] = fb[2]; A1[2] = fa[3]; A1[3] = fb[3];
}

// One block's two k-steps against a row-major f16 activation stage: bv holds
// the lane's row's 8 values of the block (elements 8q .. 8q + 7, the K order
// the code words use, one 16-byte load); acc += scale * (A . B).
__device__ __forceinline__ void mma_blk(const uint32_t (&A0)[4], const uint32_t (&A1)[4], const uint4 &bv, float s_a,
                                        float s_b, float (&acc)[4]) {
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  float d[4];
  mma_f16_16816(d, A0, bv.x, bv.y, zero4);
  mma_f16_16816(d, A1, bv.z, bv.w, d);
  acc[0] = fmaf(s_a, d[0], acc[0]);
  acc[1] = fmaf(s_a, d[1], acc[1]);
  acc[2] = fmaf(s_b, d[2], acc[2]);
  acc[3] = fmaf(s_b, d[3], acc[3]);
}

// One slot of a warp's ring as the consumer reads it: the lane's 16 code
// bytes of rows a and b (word b = block b) and the four scale bytes of each.
struct SlotData {
  uint4 va, vb;
  uint32_t sxa, sxb;
};

// Shared-window helpers of the flat stream: 32-bit shared addresses with
// immediate offsets keep the per-chunk address arithmetic to a few adds.
__device__ __forceinline__ void cp16_s(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4_s(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}

// A warp's stream of chunks [c0, c1) (n_grp groups per item: `full` groups of
// four blocks, then one narrow group of `tail` blocks when K % 128 != 0)
// through its cp.async ring of STAGES slots, continuing across item
// boundaries, in two phases: prefill() puts the first STAGES chunks in flight
// (it needs only the weights), consume() runs the rest. item_ptr(i): first
// byte of item i's tile (consecutive chunks of an item are contiguous).
// consume(start_fn, full_fn, tail_fn, end_fn): start_fn(i) runs before the
// warp's first group of item i (to prefetch what the item's epilogue needs),
// full_fn(grp, slot) takes a group of four blocks, tail_fn(grp, slot) the
// item's narrow group, end_fn(i) runs after the warp's last group of item i. Per chunk the issue side does three 16-byte
// copies per lane, the consumer four shared loads; everything else is a few
// counters (no division, no 64-bit index arithmetic).
template <int STAGES, class ItemPtr>
struct FlatStream {
  static constexpr uint32_t kLast = (STAGES - 1) * kStageBytes;
  int full, tail, lane;
  // issue side: this lane's 16 bytes of the next chunk, chunks left to issue,
  // full groups left in the issuing item, its index, the next slot's offset
  const uint8_t *src;
  int i_left, i_full, i_item;
  uint32_t i_off;
  // consume side
  int c_left, c_full, c_grp, c_item;
  uint32_t ring_lane, ring_g;  // shared addresses of the lane's code bytes and scale word in slot 0
  ItemPtr item_ptr;

  __device__ __forceinline__ FlatStream(int c0, int c1, int K, uint8_t *ring, ItemPtr ptr)
      : item_ptr(ptr) {
    lane = threadIdx.x & 31;
    const int nb = K / 32;
    full = nb / 4;
    tail = nb % 4;
    const int n_grp = full + (tail ? 1 : 0);
    const int n = c1 > c0 ? (int)(c1 - c0) : 0;
    const int item = n > 0 ? (int)(c0 / n_grp) : 0;
    const int grp = n > 0 ? c0 - item * n_grp : 0;
    i_left = c_left = n;
    i_item = c_item = item;
    i_full = c_full = full - grp;  // 0 when the range starts at the narrow group
    c_grp = grp;
    i_off = 0u;
    src = n > 0 ? item_ptr(item) + (size_t)grp * 1088 + lane * 16 : nullptr;
    ring_lane = smem_u32(ring) + lane * 16;
    ring_g = smem_u32(ring) + 1024 + (lane >> 2) * 4;
  }

  __device__ __forceinline__ void next_item_issue() {
    ++i_item;
    src = item_ptr(i_item) + lane * 16;
    i_full = full;
  }

  __device__ __forceinline__ void issue() {
    if (i_left > 0) {
      const uint32_t d = ring_lane + i_off;
      if (i_full > 0) {
        cp16_s(d, src);
        cp16_s(d + 512, src + 512);
        if (lane < 4) cp16_s(d + 1024, src + 1024);
        src += 1088;
        if (--i_full == 0 && tail == 0 && i_left > 1) next_item_issue();
      } else {
        // the narrow group is stored packed (4 * tail bytes per lane and row
        // half, then 64 scale bytes): spread it into the full layout
        const uint8_t *ch = src - lane * 16;
        for (int b = 0; b < tail; ++b) {
          cp4_s(d + b * 4, ch + lane * 4 * tail + b * 4);
          cp4_s(d + 512 + b * 4, ch + 128 * tail + lane * 4 * tail + b * 4);
        }
        if (lane < 4) cp16_s(d + 1024, ch + 256 * tail + lane * 16);
        if (i_left > 1) next_item_issue();
      }
      --i_left;
    }
    cp_async_commit();
    i_off = i_off == kLast ? 0u : i_off + kStageBytes;
  }

  __device__ __forceinline__ void prefill() {
#pragma unroll
    for (int u = 0; u < STAGES; ++u) issue();
  }

  template <class StartFn, class FullFn, class TailFn, class EndFn>
  __device__ __forceinline__ void consume(StartFn start_fn, FullFn full_fn, TailFn tail_fn, EndFn end_fn) {
    uint32_t off = 0u;
    if (c_left > 0) start_fn(c_item);
#pragma unroll 1
    for (int n = c_left; n > 0; --n) {
      cp_async_wait<STAGES - 1>();
      __syncwarp();  // the scale bytes were copied by lanes 0-3
      SlotData d;
      d.va = lds128(ring_lane + off);
      d.vb = lds128(ring_lane + off + 512);
      d.sxa = lds32(ring_g + off);
      d.sxb = lds32(ring_g + off + 32);
      issue();  // the warp read the slot above (converged) before any lane refills it
      bool ends;
      if (c_full > 0) {
        full_fn(c_grp, d);
        ends = (--c_full == 0 && tail == 0) || n == 1;
        ++c_grp;
      } else {
        tail_fn(c_grp, d);
        ends = true;
      }
      if (ends) {
        end_fn(c_item);
        ++c_item;
        c_grp = 0;
        c_full = full;
        if (n > 1) start_fn(c_item);
      }
      off = off == kLast ? 0u : off + kStageBytes;
    }
    cp_async_wait<0>();
  }
};

// A warp's parts of the (at most two) items its range shares with other
// warps: slot 0 the item that began before the range, slot 1 the one that
// ends after it. They stay in registers while the weights stream and are
// settled once the warp's ring is empty (settle()): a memory fence inside the
// streaming loop would stall the warp until its copies in flight landed.
template <int NCG>
struct SplitParts {
  float4 v[2][NCG];  // indexed with compile-time slots only (registers)
  float2 bias[2];    // the item's epilogue values the warp prefetched
  int item[2];
  bool has[2];
  __device__ __forceinline__ SplitParts() { has[0] = has[1] = false; }

  // True when item [ia, ib) lies wholly in the warp's range [c0, c1) (write
  // it now); otherwise keeps the warp's part (and the item's prefetched
  // epilogue values) and returns false.
  __device__ __forceinline__ bool take(int c0, int c1, int ia, int ib, int it,
                                       const float4 (&p)[NCG], float2 b) {
    if (ia >= c0 && ib <= c1) return true;
    if (ia < c0) {
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) v[0][cg] = p[cg];
      bias[0] = b;
      item[0] = it;
      has[0] = true;
    } else {
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) v[1][cg] = p[cg];
      bias[1] = b;
      item[1] = it;
      has[1] = true;
    }
    return false;
  }

  // Publishes the parts, then for each: the last warp to arrive adds every
  // part of the item in range order (the same order every run, whichever warp
  // is last) and calls finish(item, sum, epilogue values). Parts live in the warp's two slots
  // of `parts`, arrival counters in cnt[slot_base + first owner] (left at zero).
  template <class Finish>
  __device__ __forceinline__ void settle(const FlatRange &R, int w, int n_grp, float4 *parts, uint32_t *cnt,
                                         int slot_base, Finish finish) {
    const int lane = threadIdx.x & 31;
    if (!has[0] && !has[1]) return;
#pragma unroll
    for (int s = 0; s < 2; ++s)
      if (has[s])
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) parts[((slot_base + w) * 2 + s) * NCG * 32 + cg * 32 + lane] = v[s][cg];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (!has[s]) continue;
      const int ia = item[s] * n_grp, ib = ia + n_grp;
      const int wf = R.owner(ia), wl = R.owner(ib - 1);
      if (!arrive_last(&cnt[slot_base + wf], (uint32_t)(wl - wf + 1))) continue;
      if (lane == 0) cnt[slot_base + wf] = 0u;  // zero again for the next launch
      float4 t[NCG];
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) t[cg] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int wp = wf; wp <= wl; ++wp) {
        const int sp = ia < R.first(wp) ? 0 : 1;
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
          const float4 u = wp == w ? v[s][cg] : __ldcg(&parts[((slot_base + wp) * 2 + sp) * NCG * 32 + cg * 32 + lane]);
          t[cg].x += u.x;
          t[cg].y += u.y;
          t[cg].z += u.z;
          t[cg].w += u.w;
        }
      }
      finish(item[s], t, bias[s]);
    }
  }
};

// mlp1 + bias + clamped SwiGLU over all tokens (T <= 8), flat split over the
// whole grid: x is staged once per CTA (row-major f16 x * 2^-sigma, 8 rows,
// rows >= T zero) and every tile computes all 8 token columns; the epilogue
// keeps the columns of the tokens routed to the tile's expert. The weight
// ring is filled before the activations are staged, so the first weight
// bytes are in flight while x is converted.
template <int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1) mlp1_flat_kernel(const DecodeArgs a) {
  constexpr int kThreads = WARPS * 32;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float tok_scale[8];
  __shared__ int act_s[kMaxAllTokActive];
  __shared__ int act_of[256];
  __shared__ int col_pos[kMaxAllTokActive * 8];  // position of (active expert, token), or -1

  if (a.pdl) pdl_wait();
  const int K = a.K, XS = flat_row_pitch(K);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int T = a.T, k = a.topk;
  const int n_act = *a.n_active;
  const int n_tiles = a.rows / 16;
  const int nb = K / 32, n_grp = nb / 4 + (nb % 4 ? 1 : 0), fs_tail = nb % 4;

  for (int i = tid; i < n_act; i += kThreads) {
    act_s[i] = a.active[i];
    act_of[a.active[i]] = i;
  }
  for (int i = tid; i < n_act * 8; i += kThreads) col_pos[i] = -1;
  __syncthreads();

  const FlatRange R = flat_range(n_act * n_tiles * n_grp, (int)gridDim.x * WARPS);
  const int w = (int)blockIdx.x * WARPS + warp;
  const int c0 = R.lo(w), c1 = R.lo(w + 1);
  uint8_t *ring = smem + 8 * XS + warp * (STAGES * kStageBytes);
  auto item_ptr = [&](int i) {
    const int ai = i / n_tiles, tile = i - ai * n_tiles;
    return a.codes + ((size_t)act_s[ai] * n_tiles + tile) * a.item_bytes;
  };
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const uint8_t *brow = smem + g * XS + q * 16;
  // one block of the group: its A operands, the activation load, the MMAs
  auto block = [&](const uint8_t *bp, uint32_t wa, uint32_t wb, float s_a, float s_b) {
    uint32_t A0[4], A1[4];
    a_ops(wa, wb, A0, A1);
    mma_blk(A0, A1, *reinterpret_cast<const uint4 *>(bp), s_a, s_b, acc);
  };
  auto full_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    block(bp, d.va.x, d.vb.x, sa[0], sb[0]);
    block(bp + 64, d.va.y, d.vb.y, sa[1], sb[1]);
    block(bp + 128, d.va.z, d.vb.z, sa[2], sb[2]);
    block(bp + 192, d.va.w, d.vb.w, sa[3], sb[3]);
  };
  auto tail_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    const uint32_t wa[4] = {d.va.x, d.va.y, d.va.z, d.va.w}, wb[4] = {d.vb.x, d.vb.y, d.vb.z, d.vb.w};
#pragma unroll
    for (int b = 0; b < 3; ++b)
      if (b < fs_tail) block(bp + 64 * b, wa[b], wb[b], sa[b], sb[b]);
  };
  // bias + clamped SwiGLU of one finished tile, for the tokens routed to its expert
  auto write_tile = [&](int item, const float4 (&v)[1], float2 bias) {
    const int ai = item / n_tiles, tile = item - ai * n_tiles;
    const int pr = tile * 8 + g;  // intermediate unit (gate row 2pr, up row 2pr + 1)
    const float gate[2] = {v[0].x, v[0].y}, up[2] = {v[0].z, v[0].w};
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int t = 2 * q + c;
      const int p = col_pos[ai * 8 + t];
      if (p >= 0)
        a.out[(size_t)p * a.out_ld + pr] = swiglu_clamped(fmaf(gate[c], tok_scale[t], bias.x),
                                                          fmaf(up[c], tok_scale[t], bias.y), a.alpha, a.limit);
    }
  };
  // the gate / up biases of the lane's unit, loaded when the warp starts an
  // item so their latency hides behind the item's weight stream
  float2 cur_bias = make_float2(0.f, 0.f);
  auto start_fn = [&](int item) {
    const int ai = item / n_tiles, tile = item - ai * n_tiles;
    const uint16_t *bp = a.bias + (size_t)act_s[ai] * a.rows + 2 * (tile * 8 + g);
    cur_bias = make_float2(bf16_to_f32(bp[0]), bf16_to_f32(bp[1]));
  };
  SplitParts<1> split;
  auto end_fn = [&](int item) {
    const float4 v[1] = {make_float4(acc[0], acc[1], acc[2], acc[3])};
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    const int ia = item * n_grp;
    if (split.take(c0, c1, ia, ia + n_grp, item, v, cur_bias)) write_tile(item, v, cur_bias);
  };

  // the weight stream does not depend on x: put it in flight first
  FlatStream<STAGES, decltype(item_ptr)> fs(c0, c1, K, ring, item_ptr);
  fs.prefill();

  // the per-(active expert, token) output positions (two dependent loads:
  // started first so that their latency overlaps the staging)
  for (int p = tid; p < T * k; p += kThreads) {
    const int s = a.perm[p];
    col_pos[act_of[a.idx[s]] * 8 + s / k] = p;
  }
  if (tid < 8) tok_scale[tid] = tid < T ? __uint_as_float((uint32_t)(127 + a.sigma[tid]) << 23) : 1.f;
  // stage x (row-major f16 x * 2^-sigma; conflict-free 16-byte stores), the
  // loads of kU units per thread issued together
  constexpr int kU = 4;
  const int units = 8 * (K / 8);
  for (int u0 = tid; u0 < units; u0 += kU * kThreads) {
    uint4 v[kU];
    float inv[kU];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, tok = u / (K / 8), c8 = u - tok * (K / 8);
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      inv[j] = 0.f;
      if (u < units && tok < T) {
        v[j] = *reinterpret_cast<const uint4 *>(a.x + (size_t)tok * K + c8 * 8);
        inv[j] = __uint_as_float((uint32_t)(127 - a.sigma[tok]) << 23);
      }
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, tok = u / (K / 8), c8 = u - tok * (K / 8);
      if (u < units) {
        uint4 o;
        o.x = pack_f16x2(bf16_to_f32(v[j].x & 0xFFFFu) * inv[j], bf16_to_f32(v[j].x >> 16) * inv[j]);
        o.y = pack_f16x2(bf16_to_f32(v[j].y & 0xFFFFu) * inv[j], bf16_to_f32(v[j].y >> 16) * inv[j]);
        o.z = pack_f16x2(bf16_to_f32(v[j].z & 0xFFFFu) * inv[j], bf16_to_f32(v[j].z >> 16) * inv[j]);
        o.w = pack_f16x2(bf16_to_f32(v[j].w & 0xFFFFu) * inv[j], bf16_to_f32(v[j].w >> 16) * inv[j]);
        *reinterpret_cast<uint4 *>(smem + tok * XS + c8 * 16) = o;
      }
    }
  }
  __syncthreads();
  if (a.pdl) pdl_launch();
  fs.consume(start_fn, full_fn, tail_fn, end_fn);
  split.settle(R, w, n_grp, a.parts, a.flat_cnt, 0, write_tile);
}

// mlp1 + bias + clamped SwiGLU over the virtual experts (groups of at most 8
// consecutive slots of one expert): the grid's CTAs are dealt to the groups in
// equal numbers, each CTA stages its group's x rows (gathered through perm,
// f16 x * 2^-sigma, row j = slot pos0 + j, rows beyond n_e zero) and the
// group's warps split the expert's weight chunks flat; the epilogue writes
// h[pos] for the group's slots. Used above 8 tokens, where one expert can hold
// many of the batch's tokens.
template <int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1) mlp1_group_kernel(const DecodeArgs a) {
  constexpr int kThreads = WARPS * 32;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float tok_scale[8];

  if (a.pdl) pdl_wait();
  const int K = a.K, XS = flat_row_pitch(K);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int n_v = *a.n_virtual;
  // one group of `per` CTAs per virtual expert; with more virtual experts
  // than CTAs, CTA c takes virtual experts c, c + gridDim.x, ... alone
  const bool spread = n_v <= (int)gridDim.x;
  const int per = spread ? (int)gridDim.x / max(n_v, 1) : 1;
  const int band = spread ? (int)blockIdx.x % per : 0;
  const int stride = spread ? (int)gridDim.x / per : (int)gridDim.x;
  const int n_tiles = a.rows / 16;
  const int nb = K / 32, n_grp = nb / 4 + (nb % 4 ? 1 : 0), fs_tail = nb % 4;
#pragma unroll 1
  for (int ai = (int)blockIdx.x / per; ai < n_v; ai += stride) {
  const int e = a.v_expert[ai];
  const int n_e = a.v_count[ai], pos0 = a.v_pos0[ai];

  const FlatRange R = flat_range(n_tiles * n_grp, per * WARPS);
  const int w = band * WARPS + warp;
  const int c0 = R.lo(w), c1 = R.lo(w + 1);
  const int slot_base = (spread ? ai * per : (int)blockIdx.x) * WARPS;  // the group's first warp
  uint8_t *ring = smem + 8 * XS + warp * (STAGES * kStageBytes);
  auto item_ptr = [&](int tile) { return a.codes + ((size_t)e * n_tiles + tile) * a.item_bytes; };
  FlatStream<STAGES, decltype(item_ptr)> fs(c0, c1, K, ring, item_ptr);
  fs.prefill();

  // stage the group's x rows (the loads of kU units per thread issued
  // together): gathered from x through perm, or the received f16 rows as they are
  if (tid < 8) {
    float sc = 1.f;
    if (tid < n_e)
      sc = a.xrows ? a.row_scale[pos0 + tid]
                   : __uint_as_float((uint32_t)(127 + a.sigma[a.perm[pos0 + tid] / a.topk]) << 23);
    tok_scale[tid] = sc;
  }
  constexpr int kU = 4;
  const int units = 8 * (K / 8);
  for (int u0 = tid; u0 < units; u0 += kU * kThreads) {
    uint4 v[kU];
    float inv[kU];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, row = u / (K / 8), c8 = u - row * (K / 8);
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      inv[j] = 0.f;
      if (u < units && row < n_e) {
        if (a.xrows) {
          v[j] = *reinterpret_cast<const uint4 *>(a.xrows + (size_t)(pos0 + row) * K + c8 * 8);
        } else {
          const int t = a.perm[pos0 + row] / a.topk;
          v[j] = *reinterpret_cast<const uint4 *>(a.x + (size_t)t * K + c8 * 8);
          inv[j] = __uint_as_float((uint32_t)(127 - a.sigma[t]) << 23);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, row = u / (K / 8), c8 = u - row * (K / 8);
      if (u < units && a.xrows) {
        *reinterpret_cast<uint4 *>(smem + row * XS + c8 * 16) = v[j];  // already f16 x * 2^-sigma
      } else if (u < units) {
        uint4 o;
        o.x = pack_f16x2(bf16_to_f32(v[j].x & 0xFFFFu) * inv[j], bf16_to_f32(v[j].x >> 16) * inv[j]);
        o.y = pack_f16x2(bf16_to_f32(v[j].y & 0xFFFFu) * inv[j], bf16_to_f32(v[j].y >> 16) * inv[j]);
        o.z = pack_f16x2(bf16_to_f32(v[j].z & 0xFFFFu) * inv[j], bf16_to_f32(v[j].z >> 16) * inv[j]);
        o.w = pack_f16x2(bf16_to_f32(v[j].w & 0xFFFFu) * inv[j], bf16_to_f32(v[j].w >> 16) * inv[j]);
        *reinterpret_cast<uint4 *>(smem + row * XS + c8 * 16) = o;
      }
    }
  }
  __syncthreads();
  if (a.pdl) pdl_launch();

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const uint8_t *brow = smem + g * XS + q * 16;
  auto block = [&](const uint8_t *bp, uint32_t wa, uint32_t wb, float s_a, float s_b) {
    uint32_t A0[4], A1[4];
    a_ops(wa, wb, A0, A1);
    mma_blk(A0, A1, *reinterpret_cast<const uint4 *>(bp), s_a, s_b, acc);
  };
  auto full_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    block(bp, d.va.x, d.vb.x, sa[0], sb[0]);
    block(bp + 64, d.va.y, d.vb.y, sa[1], sb[1]);
    block(bp + 128, d.va.z, d.vb.z, sa[2], sb[2]);
    block(bp + 192, d.va.w, d.vb.w, sa[3], sb[3]);
  };
  auto tail_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    const uint32_t wa[4] = {d.va.x, d.va.y, d.va.z, d.va.w}, wb[4] = {d.vb.x, d.vb.y, d.vb.z, d.vb.w};
#pragma unroll
    for (int b = 0; b < 3; ++b)
      if (b < fs_tail) block(bp + 64 * b, wa[b], wb[b], sa[b], sb[b]);
  };
  // bias + clamped SwiGLU of a finished tile for the group's slots (columns 2q, 2q + 1)
  auto write_tile = [&](int tile, const float4 (&v)[1], float2 bias) {
    const int pr = tile * 8 + g;  // intermediate unit (gate row 2pr, up row 2pr + 1)
    const float gate[2] = {v[0].x, v[0].y}, up[2] = {v[0].z, v[0].w};
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int j = 2 * q + c;
      if (j < n_e)
        a.out[(size_t)(pos0 + j) * a.out_ld + pr] = swiglu_clamped(fmaf(gate[c], tok_scale[j], bias.x),
                                                                   fmaf(up[c], tok_scale[j], bias.y), a.alpha,
                                                                   a.limit);
    }
  };
  float2 cur_bias = make_float2(0.f, 0.f);
  auto start_fn = [&](int tile) {
    const uint16_t *bp = a.bias + (size_t)e * a.rows + 2 * (tile * 8 + g);
    cur_bias = make_float2(bf16_to_f32(bp[0]), bf16_to_f32(bp[1]));
  };
  SplitParts<1> split;
  auto end_fn = [&](int tile) {
    const float4 v[1] = {make_float4(acc[0], acc[1], acc[2], acc[3])};
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    const int ia = tile * n_grp;
    if (split.take(c0, c1, ia, ia + n_grp, tile, v, cur_bias)) write_tile(tile, v, cur_bias);
  };
  fs.consume(start_fn, full_fn, tail_fn, end_fn);
  split.settle(R, w, n_grp, a.parts, a.flat_cnt, slot_base, write_tile);
  __syncthreads();  // the next virtual expert reuses the stage and the rings
  }
}

// mlp2 + bias over the virtual experts (groups of at most 8 consecutive
// slots of one expert, from the routing kernel), with the weighted top-k
// combine fused. The grid's CTAs are dealt to the virtual experts in equal
// groups of gridDim.x / n_virtual (the remainder idles), so an expert with
// many tokens gets one CTA group per 8 of them instead of looping over its
// tokens in one place; inside a group the expert's weight chunks are split
// flat over the group's warps. The group's n_e <= 4 * NCG slots are staged
// once per CTA as f16 hi / lo rows of the SwiGLU output (row 2t: hi, 2t + 1:
// lo, rows beyond 2 n_e zero), so an MMA column group of 8 holds the hi and lo
// halves of four slots and y = hi part + lo part keeps ~22 bits of h.
// Combine: when the last virtual expert finishes a 16-row tile, that warp
// writes y[t, rows] = sum_j wts[t, j] * y_slot[slot_pos[t, j], rows] in j
// order (the same expression as combine_kernel), so the result does not
// depend on which group finishes last.
template <int WARPS, int STAGES, int NCG>
__global__ void __launch_bounds__(WARPS * 32, 1) mlp2_flat_kernel(const DecodeArgs a) {
  constexpr int kThreads = WARPS * 32;
  extern __shared__ __align__(16) uint8_t smem[];

  if (a.pdl) pdl_wait();
  const int K = a.K, XS = flat_row_pitch(K);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int n_act = *a.n_virtual;  // groups that finish every tile (the combine's count)
  // one group of `per` CTAs per virtual expert; with more virtual experts
  // than CTAs, CTA c takes virtual experts c, c + gridDim.x, ... alone
  const bool spread = n_act <= (int)gridDim.x;
  const int per = spread ? (int)gridDim.x / max(n_act, 1) : 1;
  const int band = spread ? (int)blockIdx.x % per : 0;
  const int stride = spread ? (int)gridDim.x / per : (int)gridDim.x;
  const int n_tiles = a.rows / 16;
  const int nb = K / 32, n_grp = nb / 4 + (nb % 4 ? 1 : 0);
#pragma unroll 1
  for (int ai = (int)blockIdx.x / per; ai < n_act; ai += stride) {
  const int e = a.v_expert[ai];
  const int n_e = a.v_count[ai], pos0 = a.v_pos0[ai];
  const int ngc = (2 * n_e + 7) / 8;  // column groups in use (<= NCG)

  const FlatRange R = flat_range(n_tiles * n_grp, per * WARPS);
  const int w = band * WARPS + warp;
  const int c0 = R.lo(w), c1 = R.lo(w + 1);
  const int slot_base = (spread ? ai * per : (int)blockIdx.x) * WARPS;  // the group's first warp
  uint8_t *ring = smem + 8 * NCG * XS + warp * (STAGES * kStageBytes);
  auto item_ptr = [&](int tile) { return a.codes + ((size_t)e * n_tiles + tile) * a.item_bytes; };
  FlatStream<STAGES, decltype(item_ptr)> fs(c0, c1, K, ring, item_ptr);
  fs.prefill();

  // stage the expert's h rows as f16 hi / lo (conflict-free 16-byte stores),
  // the loads of kU units per thread issued together
  constexpr int kU = 4;
  const int units = 4 * NCG * (K / 8);
  for (int u0 = tid; u0 < units; u0 += kU * kThreads) {
    float4 v[kU][2];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, tok = u / (K / 8), c8 = u - tok * (K / 8);
      v[j][0] = v[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u < units && tok < n_e) {
        const float4 *src = reinterpret_cast<const float4 *>(a.h + (size_t)(pos0 + tok) * K + c8 * 8);
        v[j][0] = src[0];
        v[j][1] = src[1];
      }
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = u0 + j * kThreads, tok = u / (K / 8), c8 = u - tok * (K / 8);
      if (u >= units) continue;
      const float f[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w, v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hw[i] = pack_f16x2(f[2 * i], f[2 * i + 1]);
        const float2 r = unpack_f16x2(hw[i]);
        lw[i] = pack_f16x2(f[2 * i] - r.x, f[2 * i + 1] - r.y);
      }
      *reinterpret_cast<uint4 *>(smem + (2 * tok) * XS + c8 * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4 *>(smem + (2 * tok + 1) * XS + c8 * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  __syncthreads();
  if (a.pdl) pdl_launch();

  float acc[NCG][4];
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg) acc[cg][0] = acc[cg][1] = acc[cg][2] = acc[cg][3] = 0.f;
  const uint8_t *brow = smem + g * XS + q * 16;
  const int fs_tail = nb % 4;
  // one block: its A operands once, then the MMAs of each column group in use
  auto block = [&](const uint8_t *bp, uint32_t wa, uint32_t wb, float s_a, float s_b) {
    uint32_t A0[4], A1[4];
    a_ops(wa, wb, A0, A1);
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg)
      if (cg < ngc) mma_blk(A0, A1, *reinterpret_cast<const uint4 *>(bp + cg * 8 * XS), s_a, s_b, acc[cg]);
  };
  auto full_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    block(bp, d.va.x, d.vb.x, sa[0], sb[0]);
    block(bp + 64, d.va.y, d.vb.y, sa[1], sb[1]);
    block(bp + 128, d.va.z, d.vb.z, sa[2], sb[2]);
    block(bp + 192, d.va.w, d.vb.w, sa[3], sb[3]);
  };
  auto tail_fn = [&](int grp, const SlotData &d) {
    float sa[4], sb[4];
    e8m0x4(d.sxa, sa);
    e8m0x4(d.sxb, sb);
    const uint8_t *bp = brow + grp * 256;
    const uint32_t wa[4] = {d.va.x, d.va.y, d.va.z, d.va.w}, wb[4] = {d.vb.x, d.vb.y, d.vb.z, d.vb.w};
#pragma unroll
    for (int b = 0; b < 3; ++b)
      if (b < fs_tail) block(bp + 64 * b, wa[b], wb[b], sa[b], sb[b]);
  };
  // bias + store of one finished tile's rows for the group's slots (to
  // y_slot, or from the group's output pointer: another rank's return rows)
  float *const out0 = a.v_out ? a.v_out[ai] : a.out + (size_t)pos0 * a.out_ld;
  auto write_tile = [&](int tile, const float4 (&v)[NCG], float2 bias) {
    const int ra = tile * 16 + g, rb = ra + 8;  // rows g and g + 8 of the tile
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg) {
      const int tok = cg * 4 + q;  // columns 2q (hi) and 2q + 1 (lo) of the group
      if (cg < ngc && tok < n_e) {
        out0[(size_t)tok * a.out_ld + ra] = (v[cg].x + v[cg].y) + bias.x;
        out0[(size_t)tok * a.out_ld + rb] = (v[cg].z + v[cg].w) + bias.y;
      }
    }
  };
  // the biases of the lane's two rows, loaded when the warp starts a tile
  float2 cur_bias = make_float2(0.f, 0.f);
  auto start_fn = [&](int tile) {
    const uint16_t *bp = a.bias + (size_t)e * a.rows + tile * 16 + g;
    cur_bias = make_float2(bf16_to_f32(bp[0]), bf16_to_f32(bp[8]));
  };
  // a tile's rows are in y_slot (fenced): the last active expert to get there
  // writes y[t, rows] = sum_j wts[t, j] * y_slot[slot_pos[t, j], rows]
  auto combine_tile = [&](int tile) {
    if (!arrive_last(&a.band_done[tile], (uint32_t)n_act)) return;
    if (lane == 0) a.band_done[tile] = 0u;  // zero again for the next launch
    const int k = a.topk;
    for (int i = lane; i < a.T * 4; i += 32) {
      const int t = i >> 2, r = tile * 16 + 4 * (i & 3);
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < k; ++j) {
        const int p = __ldcg(a.slot_pos + t * k + j);
        if (p < 0) continue;
        const float wj = __ldcg(a.wts + t * k + j);
        const float4 y4 = __ldcg(reinterpret_cast<const float4 *>(a.out + (size_t)p * a.out_ld + r));
        s.x = fmaf(wj, y4.x, s.x);
        s.y = fmaf(wj, y4.y, s.y);
        s.z = fmaf(wj, y4.z, s.z);
        s.w = fmaf(wj, y4.w, s.w);
      }
      *reinterpret_cast<float4 *>(a.y + (size_t)t * a.out_ld + r) = s;
    }
  };
  SplitParts<NCG> split;
  auto end_fn = [&](int tile) {
    float4 v[NCG];
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg) {
      v[cg] = make_float4(acc[cg][0], acc[cg][1], acc[cg][2], acc[cg][3]);
      acc[cg][0] = acc[cg][1] = acc[cg][2] = acc[cg][3] = 0.f;
    }
    const int ia = tile * n_grp;
    if (split.take(c0, c1, ia, ia + n_grp, tile, v, cur_bias)) write_tile(tile, v, cur_bias);
  };
  fs.consume(start_fn, full_fn, tail_fn, end_fn);

  // the ring is empty: publish the whole tiles, then settle the split ones
  if (c1 > c0) {
    const int t_lo = (int)((c0 + n_grp - 1) / n_grp), t_hi = (int)(c1 / n_grp);  // tiles wholly in range
    if (a.band_done)
      for (int t = t_lo; t < t_hi; ++t) combine_tile(t);
    split.settle(R, w, n_grp, a.parts, a.flat_cnt, slot_base, [&](int tile, const float4 (&v)[NCG], float2 bias) {
      write_tile(tile, v, bias);
      if (a.band_done) combine_tile(tile);
    });
  }
  __syncthreads();  // the next virtual expert reuses the stage and the rings
  }
}

// One band of one expert's tiles x its n_e tokens.
//   MODE 1: mlp1 + bias + clamped SwiGLU -> a.out = h
//   MODE 2: mlp2 + bias -> a.out = y_slot
// PACKED (MODE 2, n_e <= 4): f16 hi/lo of token j in MMA columns 2j / 2j+1.
// The activation stage occupies the first stage_bytes of smem (the kernel's
// layout: NT n-tiles of 8-byte fragments for mlp1 and packed mlp2, 16-byte
// ones otherwise); the warps' rings follow it.
// KS > 1: groups of KS warps share each tile, warp kq streaming the kq-th
// share of K; the group's first warp adds the partial sums in warp order and
// writes the tile (see mlp1_alltok_kernel).
template <int MODE, int NT, bool PACKED, int WARPS, int STAGES, int KS = 1>
__device__ __forceinline__ void expert_band(const DecodeArgs &a, uint8_t *smem, int stage_bytes, float *tok_scale,
                                            uint64_t *ring_bars, int e, int n_e, int pos0, int t_begin,
                                            int t_end) {
  static_assert(WARPS % KS == 0, "warps come in groups of KS");
  constexpr int kGroups = WARPS / KS;
  constexpr int kTokPerPass = PACKED ? 4 : NT * 8;
  constexpr int kFrag = (MODE == 1 || PACKED) ? 8 : 16;  // bytes per staged fragment
  constexpr int kNT = PACKED ? 1 : NT;
  const int K = a.K, nb = K / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const size_t rbase = (size_t)e * a.rows;
  constexpr int kThreads = WARPS * 32;
  WarpRing wr = make_ring<STAGES>(smem + stage_bytes + warp * (STAGES * kStageBytes), ring_bars + warp * STAGES);
  bool ok = true;
  // tiles of this warp's group: t_begin + gw, t_begin + gw + kGroups, ...
  const int gw = warp / KS, kq = warp % KS;
  const int n_items = t_begin + gw < t_end ? (t_end - t_begin - gw + kGroups - 1) / kGroups : 0;
  const int n_grp = nb / 4 + (nb % 4 ? 1 : 0);
  const int g_begin = kq * n_grp / KS, g_end = (kq + 1) * n_grp / KS;
  __shared__ __align__(16) float red_s[KS > 1 ? WARPS * 32 * 4 * kNT : 4];

  for (int tok0 = 0; tok0 < n_e; tok0 += kTokPerPass) {
    // ---- stage this pass's activations in fragment order ----
    if (MODE == 1) {
      stage_x<NT>(a, smem, nb, n_e - tok0, [&](int tok) { return a.perm[pos0 + tok0 + tok] / a.topk; }, a.sigma);
      if (tid < NT * 8) {
        float sc = 1.f;
        if (tok0 + tid < n_e)
          sc = __uint_as_float((uint32_t)(127 + a.sigma[a.perm[pos0 + tok0 + tid] / a.topk]) << 23);
        tok_scale[tid] = sc;
      }
    } else {
      const int units = kTokPerPass * (K / 8);
#pragma unroll 4
      for (int u = tid; u < units; u += kThreads) {
        const int tok = u / (K / 8), k0 = (u % (K / 8)) * 8;
        const int blk = k0 >> 5, qq = (k0 & 31) >> 3;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (tok0 + tok < n_e) {
          const float4 *src = reinterpret_cast<const float4 *>(a.h + (size_t)(pos0 + tok0 + tok) * K + k0);
          const float4 v0 = src[0], v1 = src[1];
          f[0] = v0.x; f[1] = v0.y; f[2] = v0.z; f[3] = v0.w;
          f[4] = v1.x; f[5] = v1.y; f[6] = v1.z; f[7] = v1.w;
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const uint32_t h01 = pack_f16x2(f[4 * s], f[4 * s + 1]);
          const uint32_t h23 = pack_f16x2(f[4 * s + 2], f[4 * s + 3]);
          const float2 r01 = unpack_f16x2(h01), r23 = unpack_f16x2(h23);
          const uint32_t l01 = pack_f16x2(f[4 * s] - r01.x, f[4 * s + 1] - r01.y);
          const uint32_t l23 = pack_f16x2(f[4 * s + 2] - r23.x, f[4 * s + 3] - r23.y);
          if (PACKED) {
            *reinterpret_cast<uint2 *>(smem + frag_off(0, nb, blk, s, 2 * tok, qq, 8)) = make_uint2(h01, h23);
            *reinterpret_cast<uint2 *>(smem + frag_off(0, nb, blk, s, 2 * tok + 1, qq, 8)) = make_uint2(l01, l23);
          } else {
            *reinterpret_cast<uint4 *>(smem + frag_off(tok >> 3, nb, blk, s, tok & 7, qq, 16)) =
                make_uint4(h01, h23, l01, l23);
          }
        }
      }
    }
    __syncthreads();
    // Once every CTA of this grid has passed here, the next kernel in the
    // stream may start taking the SM slots that free up; it waits for this
    // grid's results before it reads them.
    if (a.pdl && tok0 == 0) pdl_launch();

    float acc[kNT][4];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    auto tile_of = [&](int i) { return t_begin + gw + i * kGroups; };
    auto item_ptr = [&](int i) { return a.codes + ((size_t)e * (a.rows / 16) + tile_of(i)) * a.item_bytes; };
    auto group_fn = [&](int blk0, int nblk, const uint32_t(&wa)[4], const uint32_t(&wb)[4], uint32_t sxa,
                        uint32_t sxb) {
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
        mma_group<kFrag>(smem, nb, nt, blk0, nblk, wa, wb, sxa, sxb, g, q, acc[nt]);
    };
    auto done_fn = [&](int i) {
      if constexpr (KS > 1) {
        float4 *slot = reinterpret_cast<float4 *>(red_s) + ((gw * KS + kq) * kNT) * 32 + lane;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) slot[nt * 32] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
        asm volatile("bar.sync %0, %1;" ::"r"(1 + gw), "r"(KS * 32) : "memory");
        if (kq == 0) {
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt) {
            const float4 *g0 = reinterpret_cast<const float4 *>(red_s) + (gw * KS * kNT + nt) * 32 + lane;
            float4 t = g0[0];
#pragma unroll
            for (int r = 1; r < KS; ++r) {
              const float4 v = g0[r * kNT * 32];
              t.x += v.x;
              t.y += v.y;
              t.z += v.z;
              t.w += v.w;
            }
            acc[nt][0] = t.x;
            acc[nt][1] = t.y;
            acc[nt][2] = t.z;
            acc[nt][3] = t.w;
          }
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + gw), "r"(KS * 32) : "memory");
        if (kq != 0) {
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
          return;
        }
      }
      const int tile = tile_of(i);
      const int row_a = MODE == 1 ? 2 * (tile * 8 + g) : tile * 16 + g;
      const int row_b = MODE == 1 ? row_a + 1 : row_a + 8;
      const float ba = bf16_to_f32(a.bias[rbase + row_a]), bb = bf16_to_f32(a.bias[rbase + row_b]);
      if (PACKED) {
        const int tok = tok0 + q;  // columns 2q (hi) and 2q + 1 (lo)
        if (tok < n_e) {
          const size_t pos = (size_t)(pos0 + tok);
          a.out[pos * a.out_ld + row_a] = (acc[0][0] + acc[0][1]) + ba;
          a.out[pos * a.out_ld + row_b] = (acc[0][2] + acc[0][3]) + bb;
        }
      } else {
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int col = nt * 8 + 2 * q + c;
            const int tok = tok0 + col;
            if (tok >= n_e) continue;
            const size_t pos = (size_t)(pos0 + tok);
            if (MODE == 1) {
              const float sc = tok_scale[col];
              a.out[pos * a.out_ld + tile * 8 + g] =
                  swiglu_clamped(fmaf(acc[nt][c], sc, ba), fmaf(acc[nt][2 + c], sc, bb), a.alpha, a.limit);
            } else {
              a.out[pos * a.out_ld + row_a] = acc[nt][c] + ba;
              a.out[pos * a.out_ld + row_b] = acc[nt][2 + c] + bb;
            }
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    };
    if (ok) ok = stream_items<STAGES, kBulk>(n_items, K, wr, a.err, item_ptr, group_fn, done_fn, g_begin,
                                             g_end - g_begin);
    __syncthreads();
  }
}

// Bytes of the per-expert kernel's activation stage: NT n-tiles of K / 32
// blocks x 2 k-steps x 32 lanes of 8-byte (mlp1, packed mlp2) or 16-byte
// (mlp2 with separate hi / lo columns) fragments.
__host__ __device__ constexpr int decode_stage_bytes(int mode, int nt, bool packed_only, int K) {
  return nt * (K / 32) * 2 * 32 * ((mode == 1 || packed_only) ? 8 : 16);
}

// PACKED_ONLY (mlp2): h is always staged as f16 hi/lo column pairs, four
// tokens per pass, so the stage needs half the shared memory and the ring
// gets the rest.
template <int MODE, int NT, int WARPS, int STAGES, bool PACKED_ONLY, int KS = 1>
__global__ void __launch_bounds__(WARPS * 32, 1) moe_decode_kernel(const DecodeArgs a) {
  constexpr int kThreads = WARPS * 32;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float tok_scale[NT * 8];
  __shared__ int band_last;
  __shared__ uint64_t ring_bars[WARPS * STAGES];

  if (a.pdl) pdl_wait();
  const int n_tiles = a.rows / 16;
  int e, band = blockIdx.x, bands = a.bands;
  if (a.dyn_bands) {
    const int n_act = *a.n_active;
    bands = min(n_tiles, (int)gridDim.x / max(n_act, 1));
    if (bands < 1 || (int)blockIdx.x >= n_act * bands) return;
    e = a.active[blockIdx.x / bands];
    band = blockIdx.x % bands;
  } else if (a.active) {
    if ((int)blockIdx.y >= *a.n_active) return;
    e = a.active[blockIdx.y];
  } else {
    e = a.expert_base + blockIdx.y;
  }
  const int n_e = a.counts[e];
  if (n_e == 0) return;
  const int pos0 = a.offsets[e];
  const int t_begin = (int)(((long long)band * n_tiles) / bands);
  const int t_end = (int)(((long long)(band + 1) * n_tiles) / bands);
  const int tid = threadIdx.x;

  // shared memory: the activation stage, then the rings (launch size
  // stage_bytes + WARPS * STAGES * kStageBytes)
  const int stage_bytes = decode_stage_bytes(MODE, NT, PACKED_ONLY, a.K);
  if constexpr (MODE == 2 && PACKED_ONLY)
    expert_band<MODE, NT, true, WARPS, STAGES, KS>(a, smem, stage_bytes, tok_scale, ring_bars, e, n_e, pos0,
                                                   t_begin, t_end);
  else if (MODE == 2 && n_e <= 4)
    expert_band<MODE, NT, true, WARPS, STAGES>(a, smem, stage_bytes, tok_scale, ring_bars, e, n_e, pos0, t_begin,
                                               t_end);
  else
    expert_band<MODE, NT, false, WARPS, STAGES>(a, smem, stage_bytes, tok_scale, ring_bars, e, n_e, pos0, t_begin,
                                                t_end);

  // ---- mlp2: the last expert to finish a band of rows combines it ----
  // out[t, r] = sum_j wts[t, j] * y_slot[slot_pos[t, j], r], j in order (the
  // same expression as combine_kernel), so the result does not depend on
  // which CTA finishes last.
  if (MODE == 2 && a.band_done) {
    if (tid == 0) {
      __threadfence();
      band_last = atomicAdd(&a.band_done[band], 1u) == (unsigned)(*a.n_active - 1);
    }
    __syncthreads();
    if (band_last) {
      __threadfence();
      // the routing of all T tokens into shared memory (the activation stage
      // is free now), then 4 rows per thread with every slot row load of a
      // token issued together
      const int S = a.T * a.topk;
      int *sp_s = reinterpret_cast<int *>(smem);
      float *w_s = reinterpret_cast<float *>(smem) + S;
      for (int i = tid; i < S; i += kThreads) {
        sp_s[i] = __ldcg(a.slot_pos + i);
        w_s[i] = __ldcg(a.wts + i);
      }
      __syncthreads();
      const int r0 = t_begin * 16, nq = (t_end - t_begin) * 4;  // float4 columns of the band
      for (int i = tid; i < nq * a.T; i += kThreads) {
        const int t = i / nq, r = r0 + 4 * (i % nq);
        float4 v[4];
        int p[4];
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = 0; j0 < a.topk; j0 += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            p[u] = j0 + u < a.topk ? sp_s[t * a.topk + j0 + u] : -1;
            if (p[u] >= 0) v[u] = __ldcg(reinterpret_cast<const float4 *>(a.out + (size_t)p[u] * a.out_ld + r));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (p[u] >= 0) {
              const float w = w_s[t * a.topk + j0 + u];
              acc.x = fmaf(w, v[u].x, acc.x);
              acc.y = fmaf(w, v[u].y, acc.y);
              acc.z = fmaf(w, v[u].z, acc.z);
              acc.w = fmaf(w, v[u].w, acc.w);
            }
        }
        *reinterpret_cast<float4 *>(a.y + (size_t)t * a.out_ld + r) = acc;
      }
    }
  }
}

__global__ void __launch_bounds__(256) combine_kernel(const float *__restrict__ y_slot,
                                                      const int32_t *__restrict__ slot_pos,
                                                      const float *__restrict__ wts, int T, int H,
                                                      int k, float *__restrict__ out) {
  const int h4 = H / 4;
  const size_t n = (size_t)T * h4;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int t = (int)(i / h4), c = (int)(i % h4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const int p = slot_pos[t * k + j];
      if (p < 0) continue;
      const float w = wts[t * k + j];
      const float4 v = reinterpret_cast<const float4 *>(y_slot + (size_t)p * H)[c];
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    reinterpret_cast<float4 *>(out + (size_t)t * H)[c] = acc;
  }
}

template <class Kern>
cudaError_t launch_ex(Kern fn, dim3 grid, int threads, size_t smem, bool pdl, cudaStream_t stream,
                      const DecodeArgs &a) {
  if (smem > 48 * 1024) {
    cudaError_t st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int MODE, int NT>
cudaError_t launch_decode(const DecodeArgs &a, int grid_y, cudaStream_t stream) {
  const size_t smem = (size_t)decode_stage_bytes(MODE, NT, false, a.K) + (size_t)kW2 * kS2 * kStageBytes;
  return launch_ex(moe_decode_kernel<MODE, NT, kW2, kS2, false>, dim3(a.bands, grid_y), kW2 * 32, smem, a.pdl,
                   stream, a);
}

int bands_for_tpw(int rows, int tpw) { return (rows / 16 + kW2 * tpw - 1) / (kW2 * tpw); }

DecodeArgs mlp1_args(const MoeDeviceWeights &w, const uint16_t *x, const int32_t *perm,
                     const int32_t *sigma, const int32_t *counts, const int32_t *offsets,
                     float *h) {
  DecodeArgs a{};
  a.codes = w.w1;
  a.bias = w.b1;
  a.K = w.H;
  a.rows = 2 * w.I;
  a.item_bytes = tile_item_bytes(w.H);
  a.x = x;
  a.perm = perm;
  a.sigma = sigma;
  a.topk = w.k;
  a.counts = counts;
  a.offsets = offsets;
  a.out = h;
  a.out_ld = w.I;
  a.alpha = w.alpha;
  a.limit = w.limit;
  a.bands = bands_for_tpw(a.rows, 2);
  return a;
}

DecodeArgs mlp2_args(const MoeDeviceWeights &w, const float *h, const int32_t *counts,
                     const int32_t *offsets, float *y_slot) {
  DecodeArgs a{};
  a.codes = w.w2;
  a.bias = w.b2;
  a.K = w.I;
  a.rows = w.H;
  a.item_bytes = tile_item_bytes(w.I);
  a.h = h;
  a.topk = w.k;
  a.counts = counts;
  a.offsets = offsets;
  a.out = y_slot;
  a.out_ld = w.H;
  a.bands = bands_for_tpw(a.rows, 2);
  return a;
}

}  // namespace

// Shared memory of the activation stage, per token n-tile: nb * 2 * 32 * 8 (mlp1)
// or * 16 (mlp2) bytes, plus the warps' cp.async rings. One n-tile (8 tokens)
// per pass; larger groups of tokens take several passes.
cudaError_t launch_moe_mlp1_decode(const MoeDeviceWeights &w, const uint16_t *x,
                                   const int32_t *perm, const int32_t *sigma,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *h, int *err,
                                   cudaStream_t stream) {
  if (n_slots == 0 || n_local_experts == 0) return cudaSuccess;
  DecodeArgs a = mlp1_args(w, x, perm, sigma, counts, offsets, h);
  a.expert_base = expert_base;
  a.err = err;
  return launch_decode<1, 1>(a, n_local_experts, stream);
}

cudaError_t launch_moe_mlp2_decode(const MoeDeviceWeights &w, const float *h,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *y_slot, int *err,
                                   cudaStream_t stream) {
  if (n_slots == 0 || n_local_experts == 0) return cudaSuccess;
  DecodeArgs a = mlp2_args(w, h, counts, offsets, y_slot);
  a.expert_base = expert_base;
  a.err = err;
  return launch_decode<2, 1>(a, n_local_experts, stream);
}

int decode_bands(int rows, int expected_active, int n_sms) {
  const int tiles = rows / 16;
  int bands = n_sms / (expected_active > 0 ? expected_active : 1);
  if (bands < 1) bands = 1;
  if (bands > tiles) bands = tiles;
  return bands;
}

cudaError_t launch_moe_mlp1_sched(const MoeDeviceWeights &w, const uint16_t *x,
                                  const int32_t *perm, const int32_t *sigma, const int32_t *idx,
                                  const int32_t *counts, const int32_t *offsets,
                                  const DecodeSched &s, int T, float *h, cudaStream_t stream) {
  if (s.max_active == 0 || T == 0) return cudaSuccess;
  DecodeArgs a = mlp1_args(w, x, perm, sigma, counts, offsets, h);
  a.active = s.active;
  a.n_active = s.n_active;
  a.pdl = s.pdl;
  a.T = T;
  a.idx = idx;
  a.err = s.err;
  a.parts = s.parts;
  a.flat_cnt = s.flat_cnt;
  a.v_expert = s.v_expert;
  a.v_pos0 = s.v_pos0;
  a.v_count = s.v_count;
  a.n_virtual = s.n_virtual;
  const size_t flat_smem = (size_t)8 * flat_row_pitch(a.K) + (size_t)kWf1 * kSf1 * kStageBytes;
  const bool flat_ok = kUseFlat && s.parts && s.flat_cnt && s.n_sms * kWf1 <= kFlatMaxWarps &&
                       flat_smem <= kMaxFlatSmem;
  if (T <= 8 && T * w.k <= kMaxAllTokActive && w.E <= 256) {
    if (T <= kDeepTokens) {
      const size_t smem = (size_t)(a.K / 32) * 2 * 32 * 8 + (size_t)kW1d * kS1d * kStageBytes;
      return launch_ex(mlp1_alltok_kernel<kW1d, kS1d, kK1d>, dim3(s.n_sms), kW1d * 32, smem, a.pdl, stream, a);
    }
    // The all-token kernel gives each warp whole tiles: measured fastest when
    // the expected tiles fill its warps evenly (at 8 tokens, ~22 experts x
    // 360 tiles over 148 x 28 warps: 1.9 rounds), slower than the flat split
    // when the last round is half empty (4 tokens: ~14 experts, 1.2 rounds).
    const double rounds = (double)s.exp_active * (a.rows / 16) / ((double)s.n_sms * kW1);
    if (flat_ok && rounds / std::ceil(rounds) < 0.8)
      return launch_ex(mlp1_flat_kernel<kWf1, kSf1>, dim3(s.n_sms), kWf1 * 32, flat_smem, a.pdl, stream, a);
    const size_t smem = (size_t)(a.K / 32) * 2 * 32 * 8 + (size_t)kW1 * kS1 * kStageBytes;
    return launch_ex(mlp1_alltok_kernel<kW1, kS1>, dim3(s.n_sms), kW1 * 32, smem, a.pdl, stream, a);
  }
  // above 8 tokens: equal CTA groups per virtual expert (at most 8 of an
  // expert's slots each), so a hot expert's tokens spread over the GPU
  if (flat_ok && s.v_expert)
    return launch_ex(mlp1_group_kernel<kWf1, kSf1>, dim3(s.n_sms), kWf1 * 32, flat_smem, a.pdl, stream, a);
  a.bands = s.bands1;
  return launch_decode<1, 1>(a, s.max_active, stream);
}

cudaError_t launch_moe_mlp2_sched(const MoeDeviceWeights &w, const float *h,
                                  const int32_t *counts, const int32_t *offsets,
                                  const DecodeSched &s, uint32_t *band_done, int T,
                                  const int32_t *slot_pos, const float *wts, float *y_slot,
                                  float *y, cudaStream_t stream) {
  if (s.max_active == 0) return cudaSuccess;
  DecodeArgs a = mlp2_args(w, h, counts, offsets, y_slot);
  a.active = s.active;
  a.n_active = s.n_active;
  a.bands = s.bands2;
  a.pdl = s.pdl;
  a.err = s.err;
  a.band_done = band_done;
  a.T = T;
  a.slot_pos = slot_pos;
  a.wts = wts;
  a.y = y;
  a.parts = s.parts;
  a.flat_cnt = s.flat_cnt;
  a.v_expert = s.v_expert;
  a.v_pos0 = s.v_pos0;
  a.v_count = s.v_count;
  a.n_virtual = s.n_virtual;
  if (T >= OXG_FLAT2_MIN_TOKENS && kUseFlat && s.parts && s.flat_cnt && s.v_expert) {
    // equal CTA groups per virtual expert (at most 8 slots: two column groups
    // of four slots' hi / lo halves), flat split inside each group
    const size_t smem = (size_t)16 * flat_row_pitch(a.K) + (size_t)kWf2b * kSf2b * kStageBytes;
    if (s.n_sms * kWf2b <= kFlatMaxWarps && smem <= kMaxFlatSmem)
      return launch_ex(mlp2_flat_kernel<kWf2b, kSf2b, 2>, dim3(s.n_sms), kWf2b * 32, smem, a.pdl, stream, a);
  }
  if (T <= 8 && s.max_active <= s.n_sms) {
    // persistent grid, bands per expert from the device's active count
    a.dyn_bands = 1;
    if (T <= kDeepTokens) {
      const size_t smem = (size_t)decode_stage_bytes(2, 1, true, a.K) + (size_t)kW3d * kS3d * kStageBytes;
      return launch_ex(moe_decode_kernel<2, 1, kW3d, kS3d, true, kK3d>, dim3(s.n_sms), kW3d * 32, smem, a.pdl,
                       stream, a);
    }
    const size_t smem = (size_t)decode_stage_bytes(2, 1, true, a.K) + (size_t)kW3 * kS3 * kStageBytes;
    return launch_ex(moe_decode_kernel<2, 1, kW3, kS3, true>, dim3(s.n_sms), kW3 * 32, smem, a.pdl, stream, a);
  }
  return launch_decode<2, 1>(a, s.max_active, stream);
}

cudaError_t launch_combine(const float *y_slot, const int32_t *slot_pos, const float *wts, int T,
                           int H, int k, float *out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const size_t n = (size_t)T * (H / 4);
  size_t want = (n + 255) / 256;
  unsigned grid = (unsigned)(want < 148 * 8 ? want : 148 * 8);
  combine_kernel<<<grid, 256, 0, stream>>>(y_slot, slot_pos, wts, T, H, k, out);
  return cudaGetLastError();
}

}  // namespace oxg

namespace oxg {

bool ep_decode_supported(int H, int I, int n_sms, int max_groups) {
  const size_t s1 = (size_t)8 * flat_row_pitch(H) + (size_t)kWf1 * kSf1 * kStageBytes;
  const size_t s2 = (size_t)16 * flat_row_pitch(I) + (size_t)kWf2b * kSf2b * kStageBytes;
  (void)max_groups;  // any number: with more groups than CTAs each CTA takes several in turn
  return kUseFlat && s1 <= kMaxFlatSmem && s2 <= kMaxFlatSmem && n_sms * kWf1 <= kFlatMaxWarps &&
         n_sms * kWf2b <= kFlatMaxWarps;
}

cudaError_t launch_ep_decode(const MoeDeviceWeights &w, const uint16_t *rows, const float *row_scale, float *h,
                             const EpVirtual &virt, const DecodeSched &s, cudaStream_t stream) {
  if (!ep_decode_supported(w.H, w.I, s.n_sms, virt.cap) || !s.parts || !s.flat_cnt) return cudaErrorInvalidValue;
  DecodeArgs a = mlp1_args(w, nullptr, nullptr, nullptr, nullptr, nullptr, h);
  a.pdl = s.pdl;
  a.err = s.err;
  a.parts = s.parts;
  a.flat_cnt = s.flat_cnt;
  a.v_expert = virt.expert;
  a.v_pos0 = virt.row0;
  a.v_count = virt.count;
  a.n_virtual = virt.n;
  a.xrows = rows;
  a.row_scale = row_scale;
  cudaError_t st = launch_ex(mlp1_group_kernel<kWf1, kSf1>, dim3(s.n_sms), kWf1 * 32,
                             (size_t)8 * flat_row_pitch(a.K) + (size_t)kWf1 * kSf1 * kStageBytes, a.pdl, stream, a);
  if (st != cudaSuccess) return st;
  DecodeArgs b = mlp2_args(w, h, nullptr, nullptr, nullptr);
  b.pdl = s.pdl;
  b.err = s.err;
  b.parts = s.parts;
  b.flat_cnt = s.flat_cnt;
  b.v_expert = virt.expert;
  b.v_pos0 = virt.row0;
  b.v_count = virt.count;
  b.n_virtual = virt.n;
  b.v_out = virt.out;
  return launch_ex(mlp2_flat_kernel<kWf2b, kSf2b, 2>, dim3(s.n_sms), kWf2b * 32,
                   (size_t)16 * flat_row_pitch(b.K) + (size_t)kWf2b * kSf2b * kStageBytes, b.pdl, stream, b);
}

}  // namespace oxg
