// moe_mxf_prefill.cu — prefill MoE expert GEMMs on the block-scaled tensor
// cores, two SMs per tile (cta_group::2).
//
// Same computation as moe_prefill.cu (MLP::forward, src/model.rs:1088-1184;
// gpt-oss interleaved mlp1, clamped SwiGLU), with the MXFP4 weights consumed
// as they are stored: tcgen05.mma.kind::mxf8f6f4.block_scale multiplies E4M3
// activation terms (A, M = 256 slot rows, 128 per CTA) by E2M1 weights (B,
// N = 192 weight rows, 96 loaded by each CTA), each side with one UE8M0
// scale per 32 elements of K, accumulating in f32 in TMEM:
//   GEMM1  D[slots, 192 rows of W1_e] = sum over x's 2 terms   -> bias, SwiGLU -> h terms
//   GEMM2  D[slots, 192 rows of W2_e] = sum over h's 4 terms   -> bias -> y_slot (f32)
// Every pipeline stage holds two activation terms with one weight tile, so
// GEMM2 runs each 128-wide k-step as two passes (terms 0-1, then 2-3, the
// weight tile loaded for both) and keeps four 46 KB stages in flight.
// The activation rows of each expert start at a multiple of 128 (padded
// positions), so a CTA's 128 rows share one scale atom per k-step.
//
// Warp roles (one pair of CTAs per tile; 10 warps per CTA):
//   warp 0     TMA producer (both CTAs): the activation term tiles, the CTA's
//              half of the weight tile (TMA 16U4_ALIGN16B: 16 codes per 16
//              bytes of shared memory), the activation scale atoms of its
//              rows and the two weight scale atoms of the whole tile, all
//              counted on rank 0's stage barrier;
//   warp 1     TMEM owner (both CTAs) and, in rank 0, the MMA issuer: per
//              k-step the scale atoms go to TMEM (tcgen05.cp, both CTAs) and
//              4 x (terms) MMAs of K = 32 are issued;
//   warps 2-9  epilogue: warps 2-5 drain accumulator buffer 0, warps 6-9
//              buffer 1 (one TMEM lane quarter each), so each warp has two
//              tiles' worth of MMA time for its tile. GEMM1: bias + SwiGLU
//              on gate/up column pairs, then h (32 features per block,
//              thread-local) as four E4M3 terms + scales for GEMM2; GEMM2:
//              bias, f32 rows to y_slot.
// Every mbarrier wait is bounded; a timeout records a code in the error word
// and the pair winds down.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"

namespace oxg {
namespace {

using namespace sm100;
using namespace mxf;

constexpr int PM = 128;                // slot rows per CTA (pair M = 256)
constexpr int PN = kMxfPrefillTileN;   // weight rows per tile (pair N)
constexpr int PNH = PN / 2;            // weight rows each CTA loads
constexpr int kEpiWarpsX = 8;
constexpr int kThreadsX = (2 + kEpiWarpsX) * 32;
constexpr int kTmemColsX = 512;
constexpr int kTermsX = 2;                // activation terms per stage
constexpr int kSfaColX = 2 * PN;          // kTermsX terms x 4 columns
constexpr int kSfbColX = kSfaColX + 16;   // 2 atoms x 4 columns
constexpr int kMaxExpertsX = 256;
constexpr int kBTx = PNH * kTileK / 2;    // bytes the TMA moves for a CTA's weight half

struct MxfPrefillArgs {
  int K;                  // reduction length (H or I)
  int rows;               // weight rows per expert (2I or H)
  int n_tiles;            // ceil(rows / PN)
  int k_tiles, k_main;
  int n_experts;
  const int32_t *counts, *offsets;  // offsets padded to multiples of 128
  const uint16_t *bias;   // [E][rows]
  float alpha, limit;
  // GEMM1 out: h terms [4][rows_cap][I], atoms [4][rows_cap/128][ceil(I/128)][512]
  uint8_t *hq, *hsf;
  int I, rows_cap;
  // GEMM2 out
  float *y_slot;          // [rows_cap][H]
  int H;
  int *err;
};

template <int NT>
struct StageX {
  static constexpr int A = NT * kATileBytes;                // activation term tiles
  static constexpr int B = PNH * kTileK;                    // this CTA's weight half (padded codes)
  static constexpr int SFA = NT * kAtomBytes;
  static constexpr int SFB = 2 * kAtomBytes;
  static constexpr int BYTES = (A + B + SFA + SFB + 1023) / 1024 * 1024;
  static constexpr uint32_t TX_PAIR = 2u * (A + kBTx + SFA + SFB);
};

__device__ __forceinline__ void utccp_atom_pair(uint32_t taddr, uint32_t atom_saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((atom_saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}
__device__ __forceinline__ void umma_mxf_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void *smem_dst, const void *tmap, uint32_t bar_cl, int c0, int c1,
                                                 int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(tmap), "r"(bar_cl), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Instruction descriptor: A = E4M3 activations, B = E2M1 weights.
__host__ __device__ constexpr uint32_t idesc_e4m3_e2m1(int m, int n, int a_sf, int b_sf) {
  return ((uint32_t)b_sf << 4) | (0u << 7) | (5u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
         ((uint32_t)(m >> 4) << 24) | ((uint32_t)a_sf << 29);
}

struct CoordsX {
  int e, row0, nvalid, nt;
};

template <int GEMM, int STAGES>
__global__ void __launch_bounds__(kThreadsX, 1)
    mxf_prefill_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_wt, const __grid_constant__ CUtensorMap tm_sfa,
                       const __grid_constant__ CUtensorMap tm_sfb, const MxfPrefillArgs a) {
  constexpr int NT = kTermsX;             // activation terms per stage
  constexpr int PASSES = GEMM == 1 ? 1 : 2;  // stages per k-step (x: 2 terms, h: 4)
  using S = StageX<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *tiles = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full_[STAGES], empty_[STAGES];
  __shared__ uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int tile_prefix[kMaxExpertsX + 1];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int E = a.n_experts;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_[s], 1);
      mbar_init(&empty_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * (kEpiWarpsX / 2));
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
    int run = 0;
    for (int e = 0; e < E; ++e) {
      tile_prefix[e] = run;
      run += (a.counts[e] + 2 * PM - 1) / (2 * PM);
    }
    tile_prefix[E] = run;
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, kTmemColsX);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  const int total = tile_prefix[E] * a.n_tiles;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  auto coords = [&](int item) {
    CoordsX c;
    const int g = item / a.n_tiles;
    c.nt = item - g * a.n_tiles;
    int e = 0;
    while (e + 1 < E && tile_prefix[e + 1] <= g) ++e;
    c.e = e;
    const int i0 = (g - tile_prefix[e]) * 2 * PM;
    c.row0 = a.offsets[e] + i0;
    c.nvalid = min(2 * PM, a.counts[e] - i0);
    return c;
  };
  auto full_cl = [&](int s) { return mapa_shared(smem_addr(&full_[s]), 0); };
  const int rt_cap = a.rows_cap / PM;  // activation row tiles per term plane

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_act);
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_wt);
      prefetch_tmap(&tm_sfa);
      prefetch_tmap(&tm_sfb);
      int s = 0, r = 0;
      int last_round[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) last_round[i] = -1;
      bool ok = true;
      for (int item = pair; ok && item < total; item += n_pairs) {
        const CoordsX c = coords(item);
        const int arow = c.row0 + (int)rank * PM;
        const int wrow = c.e * a.rows + c.nt * PN + (int)rank * PNH;
        const int atile = arow / PM;
        for (int step = 0; step < a.k_tiles * PASSES; ++step) {
          const int ks = step / PASSES, t0 = (step % PASSES) * NT;
          if (r > 0) {
            if (!(ok = mbar_wait_cl(&empty_[s], (r - 1) & 1, a.err, 1))) break;
            if (rank == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&empty_[s]), 1));
          }
          uint8_t *st = tiles + s * S::BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full_[s], S::TX_PAIR);
#pragma unroll
          for (int t = 0; t < NT; ++t)
            tma_load_3d_pair(st + t * kATileBytes, &tm_act, full_cl(s), ks * kTileK, arow, t0 + t);
          if (ks < a.k_main) tma_load_2d_pair(st + S::A, &tm_w, full_cl(s), ks * kTileK, wrow);
          else tma_load_2d_pair(st + S::A, &tm_wt, full_cl(s), 0, wrow);
#pragma unroll
          for (int t = 0; t < NT; ++t)
            tma_load_2d_pair(st + S::A + S::B + t * kAtomBytes, &tm_sfa, full_cl(s), 0,
                             2 * (((t0 + t) * rt_cap + atile) * a.k_tiles + ks));
          tma_load_2d_pair(st + S::A + S::B + S::SFA, &tm_sfb, full_cl(s), 0,
                           4 * ((c.e * a.n_tiles + c.nt) * a.k_tiles + ks));
          last_round[s] = r;
          if (++s == STAGES) {
            s = 0;
            ++r;
          }
        }
      }
      if (!ok && rank == 0) {
        for (int i = 0; i < STAGES; ++i)
          if (last_round[i] >= 0) mbar_wait_cl(&full_[i], last_round[i] & 1, a.err, 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && rank == 0) {
      int s = 0, phase = 0, j = 0;
      bool ok = true;
      const uint32_t empty0 = smem_addr(&empty_[0]);
      const uint32_t sfb_t = tmem + kSfbColX;
      for (int item = pair; ok && item < total; item += n_pairs, ++j) {
        const int buf = j & 1, rr = j >> 1;
        if (rr > 0 && !(ok = mbar_wait_cl(&acc_empty[buf], (rr - 1) & 1, a.err, 3))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * PN);
        for (int step = 0; step < a.k_tiles * PASSES; ++step) {
          if (!(ok = mbar_wait_cl(&full_[s], phase, a.err, 2))) break;
          tc_fence_after();
          const uint32_t st = smem_addr(tiles + s * S::BYTES);
#pragma unroll
          for (int t = 0; t < NT; ++t) utccp_atom_pair(tmem + kSfaColX + 4 * t, st + S::A + S::B + t * kAtomBytes);
          utccp_atom_pair(sfb_t, st + S::A + S::B + S::SFA);
          utccp_atom_pair(sfb_t + 4, st + S::A + S::B + S::SFA + kAtomBytes);
          const uint64_t bd = desc_sw128_kmajor(st + S::A);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int t = 0; t < NT; ++t)
              umma_mxf_pair(d, desc_sw128_kmajor(st + t * kATileBytes) + 2 * kk, bd + 2 * kk,
                            idesc_e4m3_e2m1(2 * PM, PN, kk, kk),
                            (tmem + kSfaColX + 4 * t) | ((uint32_t)kk << 30), sfb_t | ((uint32_t)kk << 30),
                            (step | kk | t) != 0);
          umma_commit_pair(empty0 + (uint32_t)(s * sizeof(uint64_t)));
          if (++s == STAGES) {
            s = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(smem_addr(&acc_full[buf]));
      }
      umma_commit_pair(mapa_shared(smem_addr(&mma_done), 0));
      mbar_wait_cl(&mma_done, 0, a.err, 2);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int mybuf = ew / 4;             // accumulator buffer this warp drains
    const int q = warp & 3;               // TMEM lane quarter
    int j = 0;
    for (int item = pair; item < total; item += n_pairs, ++j) {
      if ((j & 1) != mybuf) continue;
      const int buf = mybuf, rr = j >> 1;
      const CoordsX c = coords(item);
      if (!mbar_wait_cl(&acc_full[buf], rr & 1, a.err, 4)) break;
      if (rank == 0 && q == 0 && lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&acc_full[buf]), 1));
      tc_fence_after();
      const int rloc = (int)rank * PM + q * 32 + lane;  // row inside the 256-row tile
      const bool row_ok = rloc < c.nvalid;
      const int p = c.row0 + rloc;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * PN);
      const int n0 = c.nt * PN;
      if (GEMM == 1) {
        const uint32_t *bias2 = reinterpret_cast<const uint32_t *>(a.bias + (size_t)c.e * a.rows);
        const int kt2 = (a.I + kTileK - 1) / kTileK;
        const size_t plane = (size_t)a.rows_cap * a.I;
        const size_t sf_plane = (size_t)rt_cap * kt2 * kAtomBytes;
        uint8_t *arow = a.hsf + (size_t)(p >> 7) * kt2 * kAtomBytes;
#pragma unroll 1
        for (int blk = 0; blk < PN / 64; ++blk) {
          const int c0 = blk * 64;
          if (n0 + c0 >= a.rows) break;  // uniform: past the matrix
          uint32_t v0[32], v1[32];
          tmem_ld_32_async(tbase + (uint32_t)c0, v0);
          tmem_ld_32_async(tbase + (uint32_t)c0 + 32, v1);
          tmem_wait_ld(v0);
          tmem_wait_ld(v1);
          const int f0 = (n0 + c0) >> 1;  // first feature of the block
          float h[32];
          uint32_t mx = 0u;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t bb = __ldg(bias2 + ((n0 + c0) >> 1) + i);
            const float g = __uint_as_float(i < 16 ? v0[2 * i] : v1[2 * i - 32]) + bf16_to_f32(bb & 0xFFFFu);
            const float u = __uint_as_float(i < 16 ? v0[2 * i + 1] : v1[2 * i - 31]) + bf16_to_f32(bb >> 16);
            h[i] = swiglu_clamped_fast(g, u, a.alpha, a.limit);
            mx = max(mx, __float_as_uint(h[i]) & 0x7FFFFFFFu);
          }
          if (row_ok) {
            const int sb = term_scale_byte(mx);
            uint32_t w[4][8];
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              uint32_t t0[4], t1[4];
              split_terms2<4>(h[i], h[i + 1], sb, t0);
              split_terms2<4>(h[i + 2], h[i + 3], sb, t1);
#pragma unroll
              for (int t = 0; t < 4; ++t) w[t][i >> 2] = t0[t] | (t1[t] << 16);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              uint4 *dst = reinterpret_cast<uint4 *>(a.hq + t * plane + (size_t)p * a.I + f0);
              dst[0] = make_uint4(w[t][0], w[t][1], w[t][2], w[t][3]);
              dst[1] = make_uint4(w[t][4], w[t][5], w[t][6], w[t][7]);
            }
            const int fb = f0 >> 5;
            const size_t o = (size_t)(fb >> 2) * kAtomBytes + atom_offset(p & 127, fb & 3);
#pragma unroll
            for (int t = 0; t < 4; ++t) arow[t * sf_plane + o] = (uint8_t)(sb - 5 * t);
            if (f0 + 32 == a.I)  // scale 0 for the blocks past I in the last k-tile
              for (int kb = a.I / 32; kb < 4 * kt2; ++kb) {
                const size_t o2 = (size_t)(kb >> 2) * kAtomBytes + atom_offset(p & 127, kb & 3);
#pragma unroll
                for (int t = 0; t < 4; ++t) arow[t * sf_plane + o2] = 0;
              }
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < PN; c0 += 32) {
          if (n0 + c0 >= a.rows) break;
          uint32_t v[32];
          tmem_ld_32_async(tbase + (uint32_t)c0, v);
          tmem_wait_ld(v);
          if (row_ok) {
            const uint32_t *bias2 = reinterpret_cast<const uint32_t *>(a.bias + (size_t)c.e * a.rows + n0 + c0);
            float4 *dst = reinterpret_cast<float4 *>(a.y_slot + (size_t)p * a.H + n0 + c0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t b01 = __ldg(bias2 + 2 * i), b23 = __ldg(bias2 + 2 * i + 1);
              dst[i] = make_float4(__uint_as_float(v[4 * i]) + bf16_to_f32(b01 & 0xFFFFu),
                                   __uint_as_float(v[4 * i + 1]) + bf16_to_f32(b01 >> 16),
                                   __uint_as_float(v[4 * i + 2]) + bf16_to_f32(b23 & 0xFFFFu),
                                   __uint_as_float(v[4 * i + 3]) + bf16_to_f32(b23 >> 16));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&acc_empty[buf]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemColsX);
}

typedef CUresult (*EncodeFnX)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFnX encode_x() {
  static EncodeFnX fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFnX>(p);
  }
  return fn;
}
cudaError_t encode(CUtensorMap *m, CUtensorMapDataType ty, int rank, const void *base, const cuuint64_t *dims,
                   const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle sw) {
  EncodeFnX fn = encode_x();
  if (!fn) return cudaErrorNotSupported;
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = fn(m, ty, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int GEMM, int STAGES>
cudaError_t launch_x(MxfPrefillArgs &a, const uint8_t *act, const uint8_t *act_sf, const uint8_t *codes,
                     const uint8_t *w_sf, int n_sms, cudaStream_t stream) {
  constexpr int NT = kTermsX;
  constexpr int PLANES = GEMM == 1 ? 2 : 4;  // activation term planes
  a.k_tiles = (a.K + kTileK - 1) / kTileK;
  a.k_main = a.K / kTileK;
  a.n_tiles = (a.rows + PN - 1) / PN;
  const int E = a.n_experts;
  CUtensorMap t_act, t_w, t_wt, t_sfa, t_sfb;
  cudaError_t st;
  {
    cuuint64_t dims[3] = {(cuuint64_t)a.K, (cuuint64_t)a.rows_cap, (cuuint64_t)PLANES};
    cuuint64_t strides[2] = {(cuuint64_t)a.K, (cuuint64_t)a.K * a.rows_cap};
    cuuint32_t box[3] = {128u, (cuuint32_t)PM, 1u};
    if ((st = encode(&t_act, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, act, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)a.k_main * kTileK, (cuuint64_t)E * a.rows};
    cuuint64_t strides[1] = {(cuuint64_t)a.K / 2};
    cuuint32_t box[2] = {128u, (cuuint32_t)PNH};
    if ((st = encode(&t_w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, codes, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if (a.k_main < a.k_tiles) {
      cuuint64_t dims2[2] = {(cuuint64_t)kTileK, (cuuint64_t)E * a.rows};
      if ((st = encode(&t_wt, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, codes + (size_t)a.k_main * (kTileK / 2),
                       dims2, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    } else {
      t_wt = t_w;
    }
  }
  {
    // activation scale atoms [PLANES][rows_cap/128][k_tiles][512] as 256-byte rows
    cuuint64_t dims[2] = {256u, (cuuint64_t)PLANES * (a.rows_cap / PM) * a.k_tiles * 2};
    cuuint64_t strides[1] = {256u};
    cuuint32_t box[2] = {256u, 2u};
    if ((st = encode(&t_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act_sf, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
    // weight scale atoms [E][n_tiles][k_tiles][2][512]
    cuuint64_t dims2[2] = {256u, (cuuint64_t)E * a.n_tiles * a.k_tiles * 4};
    cuuint32_t box2[2] = {256u, 4u};
    if ((st = encode(&t_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w_sf, dims2, strides, box2,
                     CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  }
  const size_t smem = (size_t)STAGES * StageX<NT>::BYTES + 1024;
  static int max_clusters[2] = {0, 0};
  int &mc = max_clusters[GEMM - 1];
  auto kern = mxf_prefill_kernel<GEMM, STAGES>;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreadsX);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!mc) {
    if ((st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))) return st;
    cfg.gridDim = dim3(2 * n_sms / 2);
    if ((st = cudaOccupancyMaxActiveClusters(&mc, kern, &cfg))) return st;
    if (mc < 1) return cudaErrorInvalidConfiguration;
  }
  cfg.gridDim = dim3(2 * std::min(mc, n_sms / 2));
  return cudaLaunchKernelEx(&cfg, kern, t_act, t_w, t_wt, t_sfa, t_sfb, a);
}

}  // namespace

bool mxf_prefill_supported(int H, int I, int E) {
  return H % 64 == 0 && I % 64 == 0 && H >= kTileK && I >= kTileK && E >= 1 && E <= kMaxExpertsX;
}

int mxf_rows_cap(int n_slots, int E) { return (n_slots + E * (PM - 1) + PM - 1) / PM * PM; }

cudaError_t launch_mxf_prefill(const MxfWeights &w, const uint8_t *p_atoms, const MxfPrefillIO &io, int gemm,
                               int n_sms, cudaStream_t stream) {
  if (!mxf_prefill_supported(w.H, w.I, w.E) || io.rows_cap % PM) return cudaErrorInvalidValue;
  MxfPrefillArgs a{};
  a.n_experts = w.E;
  a.counts = io.counts;
  a.offsets = io.offsets;
  a.alpha = w.alpha;
  a.limit = w.limit;
  a.hq = io.hq;
  a.hsf = io.hsf;
  a.I = w.I;
  a.H = w.H;
  a.rows_cap = io.rows_cap;
  a.y_slot = io.y_slot;
  a.err = io.err;
  if (gemm == 1) {
    a.K = w.H;
    a.rows = 2 * w.I;
    a.bias = w.b1;
    return launch_x<1, 4>(a, io.xq, io.xsf, w.q1, p_atoms, n_sms, stream);
  }
  a.K = w.I;
  a.rows = w.H;
  a.bias = w.b2;
  return launch_x<2, 4>(a, io.hq, io.hsf, w.q2, p_atoms, n_sms, stream);
}

}  // namespace oxg
