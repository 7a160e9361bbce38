// kernels.h — host-side launchers of the sm_100a kernels (internal to the
// library; the public surface is include/oxg_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace oxg {

// ---- dequant (dequant.cu) ---------------------------------------------------
// out[i] = bf16(e2m1(code_i) * scale[i / 32]) over n_blocks 32-element blocks.
// scale_fmt: 0 = E8M0 bytes, 1 = bf16 bit patterns.
cudaError_t launch_dequant_mxfp4(const uint8_t *codes, const void *scales, int scale_fmt,
                                 size_t n_blocks, uint16_t *out, cudaStream_t stream);

// ---- SwiGLU (swiglu.cu) -----------------------------------------------------
cudaError_t launch_swiglu(const float *gate, const float *up, size_t n, float alpha, float limit,
                          float *out, cudaStream_t stream);

// ---- weight re-layout (relayout.cu) ----------------------------------------
// Packed codes [rows, K/2] and scales [rows, K/32] in the checkpoint order ->
// the "tile chunk" order the f16 MoE kernels read (described in relayout.cu):
// one run of tile_item_bytes(K) bytes per 16-row tile, codes and scales of
// each 128-element group together. pair_adj selects the row pairing (1: the
// gate/up interleaved mlp1 rows 2g, 2g + 1; 0: rows g, g + 8). Either source
// may be null (that half is not written). rows % 16 == 0, K % 32 == 0.
__host__ __device__ inline size_t tile_item_bytes(int K) {
  const int nb = K / 32, tail = nb % 4;
  return (size_t)(nb / 4) * 1088 + (tail ? 256 * tail + 64 : 0);
}
cudaError_t launch_tile_weights(const uint8_t *codes, const uint8_t *scales, uint8_t *dst,
                                size_t rows, int K, int pair_adj, cudaStream_t stream);

// ---- routing (router.cu) ----------------------------------------------------
// logits may be null. sigma[T] receives the per-token power-of-two exponent
// that puts max|x| * 2^-sigma in [2^14, 2^15) (f16 operand range).
cudaError_t launch_router_topk(const uint16_t *x, const uint16_t *w, const uint16_t *b, int T, int H,
                               int E, int k, int32_t *idx, float *wts, float *logits,
                               int32_t *sigma, cudaStream_t stream);

// Batched router on the tensor cores for E a multiple of 16 (<= 64) and H a
// multiple of 16: the same outputs as launch_router_topk plus, per unit of 64
// tokens (router_mma_ctas(T) units), the expert histogram cta_hist[unit, E]
// and each slot's rank among the unit's slots of its expert, local_rank[T*k]
// (slot order). With err (a pipeline error word) and H a multiple of 64 it
// runs on tcgen05 (TMA-fed, bounded waits), else on mma.sync.
bool router_mma_supported(int H, int E, int k);
int router_mma_ctas(int T);
cudaError_t launch_router_mma(const uint16_t *x, const uint16_t *w, const uint16_t *b, int T, int H,
                              int E, int k, int32_t *idx, float *wts, float *logits,
                              int32_t *sigma, int32_t *cta_hist, int32_t *local_rank,
                              cudaStream_t stream, int *err = nullptr);

// ---- permutation (permute.cu) -------------------------------------------------
// Stable counting sort of the T*k (token, j) slots by expert.
//   counts[E], offsets[E+1], perm[T*k] (position -> slot), slot_pos[T*k]
//   (slot -> position).
// pad > 1: each expert's positions start at a multiple of pad (offsets[E]
// is the padded total; perm is defined on the occupied positions only).
cudaError_t launch_permute(const int32_t *idx, int n_slots, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                           cudaStream_t stream, int pad = 1);

// Positions from launch_router_mma's histograms and ranks (same result as
// launch_permute) and, when xp is not null, the prefill gather: xp[p] = f16
// x[token of slot perm[p]] * 2^-sigma, pos_scale[p] = 2^sigma.
// With terms: each expert's positions start at a multiple of 128 (offsets
// padded; offsets[E] the padded total) and x rows are written as the
// block-scaled prefill operand (two E4M3 planes [2][rows_cap][H] and scale
// atoms [2][rows_cap / 128][ceil(H / 128)][512]).
struct ScatterTerms {
  uint8_t *xq, *xsf;
  int rows_cap;  // multiple of 128, >= T * k + E * 127
};
cudaError_t launch_scatter(const int32_t *cta_hist, int n_cta, const int32_t *idx,
                           const int32_t *local_rank, int T, int k, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos, const uint16_t *x,
                           const int32_t *sigma, int H, uint16_t *xp, float *pos_scale,
                           cudaStream_t stream, const ScatterTerms *terms = nullptr);
// The same operand rows from slot_pos (after launch_permute with pad 128).
cudaError_t launch_gather_e4m3(const uint16_t *x, const int32_t *slot_pos, int S, int k, int H,
                               const ScatterTerms &terms, cudaStream_t stream);

// ---- fused routing for small batches (route_small.cu) -------------------------
constexpr int kMaxRouteTokens = 64;

struct RouteSmallArgs {
  const uint16_t *x, *router_w, *router_b;
  int T, H, E, k;
  float *logits;   // [T, E]
  int32_t *sigma;  // [T]
  int32_t *idx;    // [T, k]
  float *wts;      // [T, k]
  int32_t *counts, *offsets, *perm, *slot_pos;
  int32_t *active, *n_active;  // active expert ids (ascending) and their number
  uint32_t *done;              // CTA completion counter (zero between calls)
  uint32_t *band_done;         // per-band counters of the mlp2 kernel, zeroed here
  int n_bands;
  // optional (block-scaled expert path): x as two E4M3 terms per element,
  // rows 2t + term of xq [2T, H], and their UE8M0 scale atoms xsf
  // [ceil(H/128)][512] (row 2t + term, one byte per 32-element block), and
  // per expert the bit mask of the tokens routed to it (T <= 32)
  uint8_t *xq, *xsf;
  uint32_t *tok_mask;
  // optional: the active experts cut into groups of at most kVirtualTokens
  // consecutive slots ("virtual experts", expert order then slot order):
  // expert id, first position and slot count of each, and their number
  int32_t *v_expert, *v_pos0, *v_count, *n_virtual;
  // optional (expert-parallel dispatch, the batched router's outputs for one
  // CTA of <= 64 tokens): per expert the slot count [E], and per slot its
  // rank among the earlier slots of its expert [T, k]
  int32_t *cta_hist, *local_rank;
};
constexpr int kVirtualTokens = 8;
// Upper bound on the virtual experts of T tokens routed top-k over E experts.
inline int max_virtual(int E, int T, int k) {
  const int S = T * k, a = E < S ? E : S;
  return a + S / kVirtualTokens;
}
// pdl: launch with programmatic stream serialisation (overlaps the previous
// kernel's tail; the kernel waits for it before touching memory).
cudaError_t launch_route_small(const RouteSmallArgs &a, cudaStream_t stream, bool pdl);

// ---- block-scaled decode MoE (moe_mxf.cu) -------------------------------------
constexpr int kMaxMxfTokens = 8;
constexpr int kMxfPrefillTileN = 192;  // weight rows per prefill GEMM tile (the pair's MMA N)

// Weights as the block-scaled path reads them: the checkpoint's packed codes
// (64 bytes of slack after each matrix) and UE8M0 scale atoms
// [E][ceil(rows/128)][ceil(K/128)][512].
struct MxfWeights {
  int H, I, E, k;
  float alpha, limit;
  const uint8_t *q1, *a1;  // [E, 2I, H/2], atoms of [E, 2I, H/32]
  const uint16_t *b1;
  const uint8_t *q2, *a2;  // [E, H, I/2], atoms of [E, H, I/32]
  const uint16_t *b2;
};
struct MxfScratch {
  const int32_t *active, *n_active, *counts, *offsets, *idx, *slot_pos;
  const uint32_t *tok_mask;  // per expert: bit t set if token t is routed to it
  const float *wts;
  const uint8_t *xq, *xsf;   // from route_small
  uint8_t *hq, *hsf;         // [4 T k, I] terms, [E][ceil(I/128)][512] atoms
  float *y_slot;             // [T k, H]
  uint32_t *band_done;       // 4 per 128-row band of H, zero between calls
  float *y;                  // [T, H]
  int *err;
};
bool mxf_decode_supported(int H, int I, int T, int k);
// scale atoms of [E][rows][K/32] for weight tiles of tile_rows rows (128:
// decode, one atom per tile; 192: prefill, two)
size_t sf_atoms_bytes(int E, int rows, int K, int tile_rows);
cudaError_t launch_sf_atoms(const uint8_t *scales, int E, int rows, int K, int tile_rows, uint8_t *atoms,
                            cudaStream_t stream);
cudaError_t launch_mxf_mlp1(const MxfWeights &w, const MxfScratch &s, int T, int n_sms, bool pdl,
                            cudaStream_t stream);
cudaError_t launch_mxf_mlp2(const MxfWeights &w, const MxfScratch &s, int T, int n_sms, bool pdl,
                            cudaStream_t stream);

// ---- block-scaled prefill GEMMs (moe_mxf_prefill.cu) ---------------------------
// Operand buffers: x terms [2][rows_cap][H] with atoms [2][rows_cap/128][ceil(H/128)][512]
// (from launch_scatter / launch_gather_e4m3), h terms [4][rows_cap][I] with
// atoms [4][rows_cap/128][ceil(I/128)][512], y_slot [rows_cap][H] f32;
// counts/offsets with every expert's first position a multiple of 128.
struct MxfPrefillIO {
  const int32_t *counts, *offsets;
  const uint8_t *xq, *xsf;
  uint8_t *hq, *hsf;
  int rows_cap;
  float *y_slot;
  int *err;
};
bool mxf_prefill_supported(int H, int I, int E);
int mxf_rows_cap(int n_slots, int E);
// gemm 1 (x terms -> h terms) or 2 (h terms -> y_slot); p_atoms: that
// GEMM's weight scale atoms for 192-row tiles (sf_atoms_bytes(.., 192))
cudaError_t launch_mxf_prefill(const MxfWeights &w, const uint8_t *p_atoms, const MxfPrefillIO &io, int gemm,
                               int n_sms, cudaStream_t stream);

// ---- decode MoE (moe_decode.cu) ---------------------------------------------
struct MoeDeviceWeights {
  int H, I, E, k;
  float alpha, limit;
  const uint16_t *router_w, *router_b;
  const uint8_t *w1;    // tile chunks (codes + scales) of [E, 2I, H], gate/up pairing
  const uint16_t *b1;   // [E, 2I]
  const uint8_t *w2;    // tile chunks of [E, H, I], rows g / g + 8 pairing
  const uint16_t *b2;   // [E, H]
};

// mlp1 + bias + clamped SwiGLU for every (expert, slot) -> h [n_slots, I] f32
// (rows in expert-sorted position order; the token of position p is
// perm[p] / k).
cudaError_t launch_moe_mlp1_decode(const MoeDeviceWeights &w, const uint16_t *x,
                                   const int32_t *perm, const int32_t *sigma,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *h, int *err,
                                   cudaStream_t stream);
// mlp2 + bias -> y_slot [n_slots, H] f32 (position order)
cudaError_t launch_moe_mlp2_decode(const MoeDeviceWeights &w, const float *h,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *y_slot, int *err,
                                   cudaStream_t stream);
// Scheduled variants (decode fast path): blockIdx.y walks the active-expert
// list written by the routing kernel, the grid is sized to one resident
// wave, pdl chains the launches.
struct DecodeSched {
  const int32_t *active, *n_active;
  int max_active;  // grid.y: upper bound on the number of active experts
  int exp_active;  // expected number of active experts (uniform routing)
  int bands1;      // per-expert bands of the mlp1 kernel (when not all-token)
  int bands2;      // per-expert bands of the mlp2 kernel
  int n_sms;       // persistent grid of the all-token mlp1 kernel
  bool pdl;
  int *err;        // error word (bounded waits of the weight streams)
  // flat-split kernels: partial sums, flat_parts_bytes(n_sms) bytes, and
  // kFlatMaxWarps arrival counters, zero between launches
  float4 *parts;
  uint32_t *flat_cnt;
  // virtual experts from the routing kernel (8 < T <= 64): expert, first
  // position, slot count, number; max_virtual bounds the number
  const int32_t *v_expert, *v_pos0, *v_count, *n_virtual;
  int max_virtual;
};
constexpr int kFlatMaxWarps = 8192;  // grid warps a flat-split launch may use (n_sms x warps per CTA)
// Partial-sum scratch of the flat-split decode kernels on a GPU with n_sms SMs.
inline size_t flat_parts_bytes(int n_sms) { return (size_t)n_sms * 32 * 2 * 2 * 32 * 16; }
// Bands (CTAs per expert) so that expected_active experts fill n_sms SMs.
int decode_bands(int rows, int expected_active, int n_sms);
// mlp2's fused combine counts finished experts per row band in band_done,
// which must hold max(bands2, min(H / 16, n_sms)) zeroed counters.
// mlp1 + bias + clamped SwiGLU. With T <= 8 all tokens are staged once per
// CTA and a persistent grid of n_sms CTAs walks (active expert, tile) pairs;
// idx is the routing [T, k]. Otherwise one CTA per (active expert, band).
cudaError_t launch_moe_mlp1_sched(const MoeDeviceWeights &w, const uint16_t *x,
                                  const int32_t *perm, const int32_t *sigma, const int32_t *idx,
                                  const int32_t *counts, const int32_t *offsets,
                                  const DecodeSched &s, int T, float *h, cudaStream_t stream);
// mlp2 + bias into y_slot, then, per band of rows, the CTA of the last expert
// to finish writes y[t, band] = sum_j wts[t, j] * y_slot[slot_pos[t, j], band]
// (band_done: one zeroed counter per band).
cudaError_t launch_moe_mlp2_sched(const MoeDeviceWeights &w, const float *h,
                                  const int32_t *counts, const int32_t *offsets,
                                  const DecodeSched &s, uint32_t *band_done, int T,
                                  const int32_t *slot_pos, const float *wts, float *y_slot,
                                  float *y, cudaStream_t stream);

// ---- prefill MoE (moe_prefill.cu) -------------------------------------------
// Buffers of one prefill pass over S expert-sorted slots.
struct PrefillIO {
  int S;
  // The S slot rows are n_segments runs (counts[v] rows from offsets[v]); run v
  // is multiplied by the layer's local expert v % weight_mod. One GPU: the
  // runs are the experts. Expert parallel: (source rank, local expert) pairs.
  const int32_t *counts, *offsets;
  int n_segments, weight_mod;
  const uint16_t *xp;               // [S, H] f16 x * 2^-sigma in slot order (gather)
  const float *pos_scale;           // [S] 2^sigma of each slot's token
  uint16_t *h_hi, *h_lo;            // [S, I] f16 SwiGLU output, hi + lo
  float *y_slot;                    // [S, H] f32 expert outputs
  float *const *y_seg;              // or per segment: its rows' destination (null: y_slot)
  int *err;                         // pipeline timeout code (0 = none)
  // GEMM2 with the weighted top-k combine fused (one GPU, y_seg null): the
  // layer output y [T, H] f32, each token's k slot positions and weights,
  // the slot of each position, and one arrival counter per (token, 128-row
  // tile of H), zero on entry and left at zero (comb_mtiles = ceil(H / 128))
  float *y;
  const int32_t *perm, *slot_pos;
  const float *wts;
  uint32_t *comb_cnt;
  int topk;
};
// 128-row tiles of H: the fused combine's counters per token.
constexpr int prefill_comb_mtiles(int H) { return (H + 127) / 128; }
// The fused combine handles top-k up to this (larger k: combine_kernel).
constexpr int kPrefillCombineMaxK = 4;
// min over non-zero and max of E8M0 scale bytes into minmax[0..1] (which
// must hold 255 and 0 on entry).
cudaError_t launch_scale_range(const uint8_t *scales, size_t n, unsigned *minmax,
                               cudaStream_t stream);
cudaError_t launch_gather_f16(const uint16_t *x, const int32_t *perm, const int32_t *sigma, int S,
                              int H, int topk, uint16_t *xp, float *pos_scale, int *err,
                              cudaStream_t stream);
// tcgen05 grouped GEMMs (persistent grid of CTA pairs). Need H and I
// multiples of 64, every E8M0 scale 0 or in [104, 140] and n_segments <= 256.
cudaError_t launch_prefill_mlp1(const MoeDeviceWeights &w, const PrefillIO &io, int n_sms,
                                cudaStream_t stream);
cudaError_t launch_prefill_mlp2(const MoeDeviceWeights &w, const PrefillIO &io, int n_sms,
                                cudaStream_t stream);

// ---- expert-parallel exchange over peer memory (ep_p2p.cu) ---------------------
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxExperts = 64;
constexpr int kEpMaxSegments = 256;
// One rank's symmetric buffer (the same layout on every rank): flags
// [3][kEpMaxRanks] u32 (counts / rows / returns, indexed by the rank that
// raised them), counts inbox [kEpMaxRanks][kEpMaxExperts] i32, receive scales
// [max_recv] f32, receive rows [max_recv, H] f16, return rows
// [max_tokens * k, H] f32.
struct EpLayout {
  int W, E, H, k, rank, per;
  long long max_tokens, max_recv;
  long long wait_cycles;  // budget of every wait on another rank's flag (SM clock cycles)
  size_t off_flags, off_inbox, off_recv_scale, off_recv_rows, off_ret_rows, bytes;
};
struct EpPeers {
  char *base[kEpMaxRanks];  // every rank's symmetric buffer as mapped here ([rank]: own)
};
EpLayout ep_layout(int W, int E, int H, int k, int rank, long long max_tokens, long long max_recv);
// The counts into every rank's inbox, then (the same launch) the wait for
// every rank's counts flag; a wait that runs out records `code` in err.
cudaError_t launch_ep_counts(const EpLayout &L, const EpPeers &P, const int32_t *cta_hist, int n_cta,
                             int32_t *counts, int32_t *offsets, int *ok_word, uint32_t epoch, int *err,
                             int code, cudaStream_t stream);
cudaError_t launch_ep_scatter(const EpLayout &L, const EpPeers &P, const int32_t *cta_hist, int n_cta,
                              const int32_t *idx, const int32_t *local_rank, int T, const uint16_t *x,
                              const int32_t *sigma, int32_t *slot_pos, uint32_t *done_ctr,
                              int *ok_word, int *err, uint32_t epoch, cudaStream_t stream);
// Groups of at most kVirtualTokens received rows of one segment (the
// grouped decode kernels' virtual experts): resident expert, first row, row
// count and first output row (in the source's return rows) of each.
struct EpVirtual {
  int32_t *expert, *row0, *count, *n;
  float **out;
  int cap;  // entries the arrays hold
};
// seg: counts [kEpMaxSegments] then offsets [kEpMaxSegments + 1]; seg_ptr
// [kEpMaxSegments]; virt (optional, its arrays may be null): the groups
cudaError_t launch_ep_segments(const EpLayout &L, const EpPeers &P, uint32_t epoch, int *err,
                               int *ok_word, int32_t *seg, float **seg_ptr, const EpVirtual &virt,
                               cudaStream_t stream);
// Raises flag `kind` (1: rows, 2: returns) on every rank; with err, the same
// launch then waits for every rank's flag of that kind (code on a timeout).
cudaError_t launch_ep_signal(const EpLayout &L, const EpPeers &P, int kind, uint32_t epoch, int *ok_word,
                             int *err, int code, cudaStream_t stream);

// Expert-parallel decode on the receiving rank: the resident experts' MLPs
// over the received rows (f16 x * 2^-sigma [R, H] with their 2^sigma), in the
// groups of EpVirtual (grouped mlp1 into h [R, I], grouped mlp2 storing each
// group's output rows from its out pointer). ep_decode_supported is false when
// the grouped kernels' shared memory does not fit these widths.
bool ep_decode_supported(int H, int I, int n_sms, int max_groups);
cudaError_t launch_ep_decode(const MoeDeviceWeights &w, const uint16_t *rows, const float *row_scale, float *h,
                             const EpVirtual &virt, const DecodeSched &s, cudaStream_t stream);

// out[t, :] = sum_j wts[t, j] * y_slot[slot_pos[t*k + j], :], j in order.
cudaError_t launch_combine(const float *y_slot, const int32_t *slot_pos, const float *wts, int T,
                           int H, int k, float *out, cudaStream_t stream);

// ---- tensor-core issue rate (peak.cu) ------------------------------------------
// kind 0 kind::f16, 1 kind::mxf8f6f4 (E2M1 x E4M3), 2 kind::mxf4; n_ctas CTAs
// each issue `iters` M 128 x N 256 MMAs; err receives 31 if the final wait ran out.
double mma_flops_per_instr(int kind);
cudaError_t launch_mma_rate(int kind, int iters, int n_ctas, int *err, cudaStream_t stream);

}  // namespace oxg
