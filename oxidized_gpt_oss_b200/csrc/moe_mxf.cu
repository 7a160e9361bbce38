// moe_mxf.cu — decode-sized MoE expert layers on the block-scaled tensor
// cores: MXFP4 weights go from HBM into shared memory by TMA exactly as they
// are stored and into tcgen05.mma.kind::mxf8f6f4 with their E8M0 scales; no
// instruction of the SM touches a weight code.
//
// Reference computation (MLP::forward, src/model.rs:1088-1184, per (token,
// expert) from src/moe.rs:81-93; mlp1 rows interleaved gate/up, clamped
// SwiGLU, weighted combine in j order):
//   h = swiglu(x . W1^T + b1),  y_j = h . W2^T + b2,  out = sum_j w_j y_j
//
// One persistent CTA per SM walks (active expert, 128-row weight tile)
// items; each item runs the whole K of its rows:
//   warp 0     TMA producer: per 128-wide k-step, the 128 x 128 E2M1 weight
//              tile (8 KB from HBM), the activation tile (all tokens' E4M3
//              terms, L2-resident), and the two 512-byte scale atoms; two
//              k-steps per shared-memory stage, one barrier each;
//   warp 1     TMEM owner and MMA issuer: copies the scale atoms to TMEM
//              (tcgen05.cp) and issues 4 MMAs of M=128, N=nb, K=32 per
//              k-step into one of two accumulator buffers;
//   warps 2-5  epilogue (one TMEM lane quarter each), overlapping the next
//              item's MMAs.
// mlp1 (x = 2 E4M3 terms per token, MMA columns 2t and 2t+1): bias, gate/up
// pairing across adjacent lanes, clamped SwiGLU, then h of the tokens routed
// to the item's expert is split into 4 E4M3 terms per 32-feature block (the
// block spans the two warps of a lane-quarter pair, which exchange maxima
// through shared memory) and written as mlp2's operand rows 4p + term of
// slot position p, with the scale atoms.
// mlp2 (B = the expert's slots, columns 4i + term): the sum of the four
// term columns + bias is y_slot (four terms carry 16 significant bits and
// cost nothing here: the MMA has 8-column granularity and the kernel is
// bound by the weight stream); the CTA finishing the last expert of a
// 128-row band (completion counter per band) sums the k weighted rows of
// every token in j order.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"

namespace oxg {
namespace {

using namespace sm100;
using namespace mxf;

constexpr int kThreadsM = 192;
constexpr int kMaxStagesM = 10;
// k-tiles per pipeline stage: each stage's copies complete on one barrier,
// and TMA streams markedly faster with >= 16 KB per barrier than with the
// 8 KB of one 128 x 128 E2M1 tile (64 bytes per row)
constexpr int kStepsPerStage = 2;
constexpr int kSmemBudgetM = 225 * 1024;
constexpr int kAccCols = 32;                   // one accumulator buffer (N <= 32)
constexpr int kSfaCol = 2 * kAccCols, kSfbCol = kSfaCol + 4;
constexpr int kTmemColsM = 128;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

struct MxfDecodeArgs {
  int mode;                 // 1: gate/up + SwiGLU -> h terms; 2: down + bias -> y_slot, combine
  int T, k, H, I;
  int rows;                 // weight rows per expert (2I or H)
  int row_tiles, k_tiles, k_main;
  int sf_item_bytes;        // one item's scale atoms: k_tiles weight atoms, then k_tiles activation atoms
  int nb;                   // MMA N
  int stages, stage_bytes;
  const int32_t *active, *n_active, *counts, *offsets, *idx, *slot_pos;
  const uint32_t *tok_mask;
  const float *wts;
  const uint8_t *sfa;       // weight scale atoms [E][row_tiles][k_tiles][512]
  const uint8_t *sfb;       // mode 1: x atoms [k_tiles][512]; mode 2: h atoms [E][k_tiles][512]
  const uint16_t *bias;     // [E][rows] bf16
  float alpha, limit;
  uint8_t *hq;              // mode 1 out: [4 S][I] E4M3 terms, row 4p + term
  uint8_t *hsf;             // mode 1 out: [E][ceil(I/128)][512]
  float *y_slot;            // mode 2 out: [S][H]
  uint32_t *band_done;      // mode 2: per (128-row band, lane quarter), left at zero
  float *y;                 // mode 2 out: [T][H]
  int *err;
};

__global__ void __launch_bounds__(kThreadsM, 1)
    mxf_decode_kernel(const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_a_tail, const __grid_constant__ CUtensorMap tm_b2,
                      const __grid_constant__ CUtensorMap tm_b, const MxfDecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  // [stages x (A tiles, B tiles)][2 item scale buffers]
  uint8_t *sf_items = sm + a.stages * a.stage_bytes;
  __shared__ uint64_t full_[kMaxStagesM], empty_[kMaxStagesM], acc_full[2], acc_empty[2], mma_done, pair_bar[2];
  __shared__ uint64_t ifull[2], iempty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t pair_max[2][4][kMaxMxfTokens];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full_[s], 1);
      mbar_init(&empty_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(&mma_done, 1);
    mbar_init(&pair_bar[0], 2);
    mbar_init(&pair_bar[1], 2);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ifull[b], 1);
      mbar_init(&iempty[b], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a2);
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_a_tail);
    prefetch_tmap(&tm_b2);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemColsM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  // routing, x terms (mlp1) and h terms (mlp2) come from the previous kernels
  pdl_wait();
  pdl_launch();
  const int n_act = *a.n_active;
  const int n_items = n_act * a.row_tiles;
  const uint32_t b_bytes = (uint32_t)a.nb * 128u;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      int j = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++j) {
        const int e = a.active[item / a.row_tiles], rt = item % a.row_tiles;
        const int row0 = e * a.rows + rt * kTileM;
        const int brow0 = a.mode == 1 ? 0 : 4 * a.offsets[e];
        const uint8_t *sfa = a.sfa + (size_t)(e * a.row_tiles + rt) * a.k_tiles * kAtomBytes;
        const uint8_t *sfb = a.mode == 1 ? a.sfb : a.sfb + (size_t)e * a.k_tiles * kAtomBytes;
        // the item's scale atoms, both operands, two bulk copies into one of
        // two item buffers
        const int ib = j & 1;
        if (!(ok = mbar_wait(&iempty[ib], (((uint32_t)j >> 1) & 1u) ^ 1u, a.err, 8))) break;
        const uint32_t half = (uint32_t)a.sf_item_bytes / 2;
        mbar_arrive_expect_tx(&ifull[ib], 2u * half);
        bulk_load(sf_items + ib * a.sf_item_bytes, sfa, half, &ifull[ib]);
        bulk_load(sf_items + ib * a.sf_item_bytes + half, sfb, half, &ifull[ib]);
        for (int kp = 0; kp < a.k_tiles;) {
          // main k-tiles two at a time through the 3-D maps (one copy per
          // operand), a last odd main tile alone, then the tail tile
          const int nt = kp + 1 < a.k_main ? 2 : 1;
          if (!(ok = mbar_wait(&empty_[s], ph ^ 1u, a.err, 1))) break;
          uint8_t *st = sm + s * a.stage_bytes;
          uint8_t *sb = st + kStepsPerStage * kATileBytes;
          mbar_arrive_expect_tx(&full_[s], (uint32_t)nt * ((uint32_t)kATileTx + b_bytes));
          if (nt == 2) {
            tma_load_3d(st, &tm_a2, &full_[s], 0, row0, kp);
            tma_load_3d(sb, &tm_b2, &full_[s], 0, brow0, kp);
          } else {
            if (kp < a.k_main) tma_load_2d(st, &tm_a, &full_[s], kp * kTileK, row0);
            else tma_load_2d(st, &tm_a_tail, &full_[s], 0, row0);
            tma_load_2d(sb, &tm_b, &full_[s], kp * kTileK, brow0);
          }
          kp += nt;
          ++issued;
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // let every copy issued so far land before the CTA can exit
        for (int i = 0; i < a.stages && i < issued; ++i) {
          s = s == 0 ? a.stages - 1 : s - 1;
          if (s == a.stages - 1) ph ^= 1u;
          mbar_wait(&full_[s], ph, a.err, 2);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0, j = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t sfa_t = tmem + kSfaCol, sfb_t = tmem + kSfbCol;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++j) {
        const int buf = j & 1;
        if (!(ok = mbar_wait(&acc_empty[buf], (((uint32_t)j >> 1) & 1u) ^ 1u, a.err, 3))) break;
        if (!(ok = mbar_wait(&ifull[buf], ((uint32_t)j >> 1) & 1u, a.err, 9))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * kAccCols);
        const uint32_t sfi = smem_addr(sf_items + buf * a.sf_item_bytes);
        const uint32_t half = (uint32_t)a.sf_item_bytes / 2;
        for (int kp = 0; kp < a.k_tiles;) {
          const int n = kp + 1 < a.k_main ? 2 : 1;
          if (!(ok = mbar_wait(&full_[s], ph, a.err, 4))) break;
          tc_fence_after();
          const uint32_t st = smem_addr(sm + s * a.stage_bytes);
          for (int i = 0; i < n; ++i) {
            const uint32_t sa = st + i * kATileBytes;
            const uint32_t sb = st + kStepsPerStage * kATileBytes + i * b_bytes;
            const uint32_t sf = sfi + (uint32_t)(kp + i) * kAtomBytes;
            utccp_atom(sfa_t, sf);
            utccp_atom(sfb_t, sf + half);
            const uint64_t ad = desc_sw128_kmajor(sa), bd = desc_sw128_kmajor(sb);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_mxf(d, ad + 2 * kk, bd + 2 * kk, idesc_e2m1_e4m3(kTileM, a.nb, kk, kk),
                       sfa_t | ((uint32_t)kk << 30), sfb_t | ((uint32_t)kk << 30), (kp | i | kk) != 0);
          }
          umma_commit(&empty_[s]);
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
          }
          kp += n;
        }
        if (ok) {
          umma_commit(&iempty[buf]);
          umma_commit(&acc_full[buf]);
        }
      }
      umma_commit(&mma_done);
      mbar_wait(&mma_done, 0, a.err, 5);
    }
  } else {
    // ---- epilogue: warp w owns TMEM lanes 32 (w % 4) .. +31 ----
    const int q = warp & 3;
    const int ml = q * 32 + lane;  // row inside the 128-row tile
    int j = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++j) {
      const int buf = j & 1;
      // every lane waits; the warp leaves together if any lane timed out
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[buf], ((uint32_t)j >> 1) & 1u, a.err, 6))) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32_async(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kAccCols), r);
      tmem_wait_ld(r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);

      const int e = a.active[item / a.row_tiles], rt = item % a.row_tiles;
      const int m = rt * kTileM + ml;
      if (a.mode == 1) {
        // ---- gate/up + SwiGLU -> 4 E4M3 terms of h for the routed tokens ----
        const float bias = bf16_to_f32(a.bias[(size_t)e * a.rows + m]);
        const int off = a.offsets[e];
        // expert e's positions are its tokens in token order (stable grouping)
        const uint32_t tmask = __ldg(a.tok_mask + e);
        float h[kMaxMxfTokens];
        int pos[kMaxMxfTokens];
#pragma unroll
        for (int t = 0; t < kMaxMxfTokens; ++t) {
          const float v = __uint_as_float(r[2 * t]) + __uint_as_float(r[2 * t + 1]) + bias;
          const float u = __shfl_down_sync(0xFFFFFFFFu, v, 1);
          h[t] = (lane & 1) ? 0.f : swiglu_clamped_fast(v, u, a.alpha, a.limit);
          pos[t] = (tmask >> t) & 1u ? off + __popc(tmask & ((1u << t) - 1u)) : -1;
          uint32_t mx = __float_as_uint(h[t]) & 0x7FFFFFFFu;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
          if (lane == 0) pair_max[buf][q][t] = mx;
        }
        // exchange with the other warp of this 32-feature block (a warp can
        // run at most one item ahead of its partner, so two buffers suffice)
        __syncwarp();
        if (lane == 0) mbar_arrive(&pair_bar[q >> 1]);
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&pair_bar[q >> 1], (uint32_t)j & 1u, a.err, 7))) break;
        const int fl = ml >> 1;                  // feature inside the tile's 64
        const int f = rt * (kTileM / 2) + fl;    // intermediate feature
        const int fb = f >> 5;                   // its 32-feature block
#pragma unroll
        for (int t = 0; t < kMaxMxfTokens; ++t) {
          if (pos[t] < 0) continue;  // uniform across the warp
          const uint32_t mx = max(pair_max[buf][q][t], pair_max[buf][q ^ 1][t]);
          const int sb = term_scale_byte(mx);
          uint32_t tb[4];
          split_terms2<4>(h[t], 0.f, sb, tb);
          const int n0 = 4 * (pos[t] - off);
#pragma unroll
          for (int term = 0; term < 4; ++term) {
            // even lanes hold features fl; pack 4 consecutive features per word
            const uint32_t b0 = tb[term] & 0xFFu;
            const uint32_t b1 = __shfl_down_sync(0xFFFFFFFFu, b0, 2);
            const uint32_t b2 = __shfl_down_sync(0xFFFFFFFFu, b0, 4);
            const uint32_t b3 = __shfl_down_sync(0xFFFFFFFFu, b0, 6);
            if ((lane & 7) == 0)
              *reinterpret_cast<uint32_t *>(a.hq + (size_t)(4 * pos[t] + term) * a.I + f) =
                  b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
            if ((q & 1) == 0 && lane == 0)
              a.hsf[((size_t)e * ((a.I + kTileK - 1) / kTileK) + (fb >> 2)) * kAtomBytes +
                    atom_offset(n0 + term, fb & 3)] = (uint8_t)(sb - 5 * term);
          }
        }
      } else {
        // ---- down + bias -> y_slot; the band's last expert combines ----
        const bool valid = m < a.rows;
        const float bias = valid ? bf16_to_f32(a.bias[(size_t)e * a.rows + m]) : 0.f;
        const int cnt = a.counts[e], off = a.offsets[e];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < cnt && valid)
            a.y_slot[(size_t)(off + i) * a.H + m] = ((__uint_as_float(r[4 * i]) + __uint_as_float(r[4 * i + 1])) +
                                                     (__uint_as_float(r[4 * i + 2]) + __uint_as_float(r[4 * i + 3]))) +
                                                    bias;
        // this warp's 32 rows of the band are done for expert e; the warp
        // that completes them for the last expert combines them
        __threadfence();
        __syncwarp();
        uint32_t prev = 0;
        if (lane == 0) prev = atomicAdd(a.band_done + 4 * rt + q, 1u);
        prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
        if (prev == (uint32_t)(n_act - 1)) {
          __threadfence();
          // tokens in batches of 32 / k: lane l fetches the position and
          // weight of the batch's slot l, then every lane issues the loads
          // of a token's k rows together (two memory round trips per batch)
          const int tb = 32 / a.k;
          for (int t0 = 0; t0 < a.T; t0 += tb) {
            const int sl = t0 * a.k + lane;
            const bool have = lane < tb * a.k && sl < a.T * a.k;
            const int p_l = have ? __ldcg(a.slot_pos + sl) : 0;
            const float w_l = have ? __ldcg(a.wts + sl) : 0.f;
            for (int t = t0; t < min(a.T, t0 + tb); ++t) {
              const int base = (t - t0) * a.k;
              float v[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int p = __shfl_sync(0xFFFFFFFFu, p_l, (base + jj) & 31);
                v[jj] = (jj < a.k && valid) ? __ldcg(a.y_slot + (size_t)p * a.H + m) : 0.f;
              }
              float acc = 0.f;
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const float w = __shfl_sync(0xFFFFFFFFu, w_l, (base + jj) & 31);
                if (jj < a.k) acc = fmaf(w, v[jj], acc);
              }
              if (valid) a.y[(size_t)t * a.H + m] = acc;
            }
          }
          if (lane == 0) a.band_done[4 * rt + q] = 0u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemColsM);
}

// Scale atoms of a weight matrix for tiles of tile_rows rows: src
// [E][rows][K/32] -> dst [E][row_tiles][k_tiles][n_atoms][512] with
// n_atoms = ceil(tile_rows / 128) (atom a holds tile rows 128a ..), zero
// outside the matrix and the tile.
__global__ void sf_atoms_kernel(const uint8_t *__restrict__ src, int E, int rows, int kb, int tile_rows,
                                int row_tiles, int k_tiles, uint8_t *__restrict__ dst) {
  const int n_atoms = (tile_rows + kTileM - 1) / kTileM;
  const size_t total = (size_t)E * row_tiles * k_tiles * n_atoms * kAtomBytes;
  for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
    const int off = (int)(o % kAtomBytes);
    size_t q = o / kAtomBytes;
    const int at = (int)(q % n_atoms);
    q /= n_atoms;
    const int kt = (int)(q % k_tiles);
    q /= k_tiles;
    const int rt = (int)(q % row_tiles);
    const int e = (int)(q / row_tiles);
    const int rin = at * kTileM + 32 * ((off & 15) >> 2) + (off >> 4);
    const int r = rt * tile_rows + rin;
    const int b = kt * 4 + (off & 3);
    dst[o] = (rin < tile_rows && r < rows && b < kb) ? src[((size_t)e * rows + r) * kb + b] : (uint8_t)0;
  }
}

typedef CUresult (*EncodeTiledFnM)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFnM encode_fn_m() {
  static EncodeTiledFnM fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnM>(p);
  }
  return fn;
}

// 2-D map, 128-byte swizzle. E2M1 codes (16U4_ALIGN16B, box 128 x 128) or
// bytes (box 128 x box_rows).
cudaError_t make_map(CUtensorMap *m, const void *base, bool e2m1, uint64_t cols, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_rows) {
  EncodeTiledFnM fn = encode_fn_m();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {cols, rows}, strides[1] = {row_bytes};
  cuuint32_t box[2] = {128u, box_rows}, es[2] = {1u, 1u};
  CUresult r = fn(m, e2m1 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                  const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 3-D map over k-tiles: dims (128 elements of one k-tile, rows, k-tiles)
// with row stride row_bytes and k-tile stride 64 bytes (E2M1) or 128 bytes;
// box (128, box_rows, kStepsPerStage): consecutive whole k-tiles, each landing
// as its own 128-byte-swizzled tile.
cudaError_t make_map3(CUtensorMap *m, const void *base, bool e2m1, uint64_t rows, uint64_t row_bytes,
                      uint64_t k_tiles, uint32_t box_rows) {
  EncodeTiledFnM fn = encode_fn_m();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[3] = {128u, rows, k_tiles}, strides[2] = {row_bytes, e2m1 ? 64u : 128u};
  cuuint32_t box[3] = {128u, box_rows, (cuuint32_t)kStepsPerStage}, es[3] = {1u, 1u, 1u};
  CUresult r = fn(m, e2m1 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3,
                  const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_mxf(MxfDecodeArgs &a, const uint8_t *codes, int E, const uint8_t *b_base,
                       uint64_t b_rows, int grid, bool pdl, cudaStream_t stream) {
  const int K = a.mode == 1 ? a.H : a.I;
  a.k_tiles = (K + kTileK - 1) / kTileK;
  a.k_main = K / kTileK;
  a.row_tiles = (a.rows + kTileM - 1) / kTileM;
  a.stage_bytes = (kStepsPerStage * (kATileBytes + a.nb * 128) + 1023) / 1024 * 1024;
  a.sf_item_bytes = 2 * a.k_tiles * kAtomBytes;
  a.stages = std::min(kMaxStagesM, (kSmemBudgetM - 2 * a.sf_item_bytes) / a.stage_bytes);
  if (a.stages < 2) return cudaErrorInvalidValue;
  CUtensorMap ta2, ta, tt, tb2, tb;
  const uint64_t wrows = (uint64_t)E * a.rows;
  cudaError_t st = make_map(&ta, codes, true, (uint64_t)a.k_main * kTileK, wrows, (uint64_t)K / 2, kTileM);
  if (st) return st;
  if ((st = make_map(&tb, b_base, false, (uint64_t)K, b_rows, (uint64_t)K, (uint32_t)a.nb))) return st;
  if (a.k_main < a.k_tiles)
    st = make_map(&tt, codes + (size_t)a.k_main * (kTileK / 2), true, kTileK, wrows, (uint64_t)K / 2, kTileM);
  else
    tt = ta;
  if (st) return st;
  if (a.k_main >= 2) {
    // pairs of main k-tiles: dims (128 codes | bytes of a k-tile, rows, k-tile)
    if ((st = make_map3(&ta2, codes, true, wrows, (uint64_t)K / 2, (uint64_t)a.k_main, kTileM))) return st;
    if ((st = make_map3(&tb2, b_base, false, b_rows, (uint64_t)K, (uint64_t)a.k_main, (uint32_t)a.nb))) return st;
  } else {
    ta2 = ta;
    tb2 = tb;
  }
  const size_t smem = (size_t)a.stages * a.stage_bytes + 2 * (size_t)a.sf_item_bytes + 1024;
  static bool attr_set = false;
  if (!attr_set) {
    if ((st = cudaFuncSetAttribute(mxf_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBudgetM + 1024)))
      return st;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsM);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mxf_decode_kernel, ta2, ta, tt, tb2, tb, a);
}

}  // namespace

bool mxf_decode_supported(int H, int I, int T, int k) {
  return T >= 1 && T <= kMaxMxfTokens && H % 64 == 0 && I % 64 == 0 && H >= kTileK && I >= kTileK &&
         k >= 1 && k <= 16;
}

cudaError_t launch_sf_atoms(const uint8_t *scales, int E, int rows, int K, int tile_rows, uint8_t *atoms,
                            cudaStream_t stream) {
  const int kb = K / 32, row_tiles = (rows + tile_rows - 1) / tile_rows, k_tiles = (K + kTileK - 1) / kTileK;
  const size_t total = sf_atoms_bytes(E, rows, K, tile_rows);
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 65535);
  sf_atoms_kernel<<<blocks, 256, 0, stream>>>(scales, E, rows, kb, tile_rows, row_tiles, k_tiles, atoms);
  return cudaGetLastError();
}

size_t sf_atoms_bytes(int E, int rows, int K, int tile_rows) {
  return (size_t)E * ((rows + tile_rows - 1) / tile_rows) * ((K + kTileK - 1) / kTileK) *
         ((tile_rows + kTileM - 1) / kTileM) * kAtomBytes;
}

cudaError_t launch_mxf_mlp1(const MxfWeights &w, const MxfScratch &s, int T, int n_sms, bool pdl,
                            cudaStream_t stream) {
  MxfDecodeArgs a{};
  a.mode = 1;
  a.T = T;
  a.k = w.k;
  a.H = w.H;
  a.I = w.I;
  a.rows = 2 * w.I;
  a.nb = (2 * T + 15) / 16 * 16;
  a.active = s.active;
  a.n_active = s.n_active;
  a.counts = s.counts;
  a.offsets = s.offsets;
  a.idx = s.idx;
  a.slot_pos = s.slot_pos;
  a.tok_mask = s.tok_mask;
  a.wts = s.wts;
  a.sfa = w.a1;
  a.sfb = s.xsf;
  a.bias = w.b1;
  a.alpha = w.alpha;
  a.limit = w.limit;
  a.hq = s.hq;
  a.hsf = s.hsf;
  a.err = s.err;
  const int max_items = std::min(w.E, T * w.k) * ((a.rows + kTileM - 1) / kTileM);
  return launch_mxf(a, w.q1, w.E, s.xq, (uint64_t)2 * T, std::min(n_sms, max_items), pdl, stream);
}

cudaError_t launch_mxf_mlp2(const MxfWeights &w, const MxfScratch &s, int T, int n_sms, bool pdl,
                            cudaStream_t stream) {
  MxfDecodeArgs a{};
  a.mode = 2;
  a.T = T;
  a.k = w.k;
  a.H = w.H;
  a.I = w.I;
  a.rows = w.H;
  a.nb = (4 * T + 15) / 16 * 16;
  a.active = s.active;
  a.n_active = s.n_active;
  a.counts = s.counts;
  a.offsets = s.offsets;
  a.idx = s.idx;
  a.slot_pos = s.slot_pos;
  a.wts = s.wts;
  a.sfa = w.a2;
  a.sfb = s.hsf;
  a.bias = w.b2;
  a.y_slot = s.y_slot;
  a.band_done = s.band_done;
  a.y = s.y;
  a.err = s.err;
  const int max_items = std::min(w.E, T * w.k) * ((a.rows + kTileM - 1) / kTileM);
  return launch_mxf(a, w.q2, w.E, s.hq, (uint64_t)4 * T * w.k, std::min(n_sms, max_items), pdl, stream);
}

}  // namespace oxg
