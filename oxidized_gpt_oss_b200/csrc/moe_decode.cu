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
constexpr int kDeepTokens = 2;
constexpr int kW1d = 28, kS1d = 5, kK1d = 4;  // mlp1: 7 groups of 4 warps splitting K
constexpr int kW3d = 20, kS3d = 7, kK3d = 4;  // mlp2: 5 groups of 4 warps splitting K
constexpr int kMaxAllTokActive = 128;  // active experts of an all-token mlp1 launch (T*k <= 128)

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
// Per-expert kernel: CTA = (expert, band of tiles); tokens staged per expert.
// ---------------------------------------------------------------------------

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
  if (T <= 8 && T * w.k <= kMaxAllTokActive && w.E <= 256) {
    if (T <= kDeepTokens) {
      const size_t smem = (size_t)(a.K / 32) * 2 * 32 * 8 + (size_t)kW1d * kS1d * kStageBytes;
      return launch_ex(mlp1_alltok_kernel<kW1d, kS1d, kK1d>, dim3(s.n_sms), kW1d * 32, smem, a.pdl, stream, a);
    }
    const size_t smem = (size_t)(a.K / 32) * 2 * 32 * 8 + (size_t)kW1 * kS1 * kStageBytes;
    return launch_ex(mlp1_alltok_kernel<kW1, kS1>, dim3(s.n_sms), kW1 * 32, smem, a.pdl, stream, a);
  }
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
