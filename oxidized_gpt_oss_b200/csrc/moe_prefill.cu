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

constexpr int BM = 128;             // weight rows per tile (MMA M)
constexpr int BK = 64;              // K per stage (one 128-byte swizzle atom of f16)
constexpr int kStagesP = 3;         // A/B stage ring
constexpr int kCodeStages = 6;      // converter cp.async ring (k-steps in flight)
constexpr int kConvWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kThreadsP = (2 + kConvWarps + kEpiWarps) * 32;  // 448
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kTasks = BM * 4 / kConvThreads;  // (row, lane-in-quad) tasks per converter thread
constexpr int kTmemCols = 512;
constexpr int kCodeStageBytes = kTasks * kConvThreads * 12;  // 8 B codes + 4 B scales per task
constexpr int kMaxExpertsP = 256;

struct PrefillArgs {
  const uint8_t *codes;   // relaid codes [E, rows, K/2]
  const uint8_t *scales;  // padded scales [E, rows, kb_pad]
  const uint16_t *bias;   // [E, rows]
  int K, rows, kb_pad;
  const int32_t *counts, *offsets;
  int n_experts, expert_base;
  // GEMM1 epilogue
  const float *pos_scale;  // [S] 2^sigma of the token in each slot position
  uint16_t *h_hi, *h_lo;   // [S, I] f16
  int I;
  float alpha, limit;
  // GEMM2 epilogue
  float *y_slot;  // [S, H]
  int H;
  int *err;
};

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void cp_async_8(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(smem)), "l"(gmem)
               : "memory");
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

template <int GEMM, int BN>
__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tm0,
                        const __grid_constant__ CUtensorMap tm1, const PrefillArgs a) {
  constexpr int NB = GEMM == 1 ? 1 : 2;  // token tiles per stage (GEMM2: h hi and lo)
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment of the shared-space offset (the swizzle atoms of the
  // TMA tiles and the MMA descriptors assume it)
  uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t *tiles = smem;
  uint8_t *code_ring = tiles + kStagesP * STAGE_BYTES;
  uint8_t *epi = code_ring + kCodeStages * kCodeStageBytes;  // GEMM1 output staging

  __shared__ uint64_t full_a[kStagesP], full_b[kStagesP], empty_[kStagesP];
  __shared__ uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int ntile_prefix[kMaxExpertsP + 1];
  __shared__ int epi_ok;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.n_experts;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesP; ++s) {
      mbar_init(&full_a[s], kConvWarps);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
    int run = 0;
    for (int e = 0; e < E; ++e) {
      ntile_prefix[e] = run;
      run += (a.counts[a.expert_base + e] + BN - 1) / BN;
    }
    ntile_prefix[E] = run;
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  const int MT = (a.rows + BM - 1) / BM;
  const int total = ntile_prefix[E] * MT;
  const int KSTEPS = a.K / BK;
  auto coords = [&](int item) {
    Coords c;
    const int ntg = item / MT;
    c.m0 = (item - ntg * MT) * BM;
    int e = 0;
    while (e + 1 < E && ntile_prefix[e + 1] <= ntg) ++e;
    c.e = e;
    c.n0 = (ntg - ntile_prefix[e]) * BN;
    c.nvalid = min(BN, a.counts[a.expert_base + e] - c.n0);
    return c;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm0);
      if (NB == 2) prefetch_tmap(&tm1);
      int it = 0;
      int last_round[kStagesP] = {-1, -1, -1};
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
        const Coords c = coords(item);
        const int row0 = a.offsets[a.expert_base + c.e] + c.n0;
        for (int ks = 0; ks < KSTEPS; ++ks, ++it) {
          const int s = it % kStagesP, r = it / kStagesP;
          if (r > 0 && !(ok = mbar_wait(&empty_[s], (r - 1) & 1, a.err, 1))) break;
          uint8_t *st = tiles + s * STAGE_BYTES;
          if (misaligned(smem_addr(st + A_BYTES), 1024, a.err, 101) ||
              misaligned((uint64_t)&tm0, 64, a.err, 102)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_b[s], NB * B_BYTES);
          tma_load_2d(st + A_BYTES, &tm0, &full_b[s], ks * BK, row0);
          if (NB == 2) tma_load_2d(st + A_BYTES + B_BYTES, &tm1, &full_b[s], ks * BK, row0);
          last_round[s] = r;
        }
      }
      if (!ok) {  // let copies still in flight land before the CTA exits
        for (int s = 0; s < kStagesP; ++s)
          if (last_round[s] >= 0) mbar_wait(&full_b[s], last_round[s] & 1, a.err, 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, j = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < total; item += gridDim.x, ++j) {
        const Coords c = coords(item);
        const int buf = j & 1, rr = j >> 1;
        if (rr > 0 && !(ok = mbar_wait(&acc_empty[buf], (rr - 1) & 1, a.err, 3))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        const int n_mma = (c.nvalid + 15) / 16 * 16;
        const uint32_t idesc = idesc_f16_f32(BM, n_mma);
        for (int ks = 0; ks < KSTEPS; ++ks, ++it) {
          const int s = it % kStagesP, r = it / kStagesP;
          if (!(ok = mbar_wait(&full_a[s], r & 1, a.err, 2))) break;
          if (!(ok = mbar_wait(&full_b[s], r & 1, a.err, 2))) break;
          tc_fence_after();
          const uint32_t sa = smem_addr(tiles + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = desc_sw128_kmajor(sa + kk * 32);
            umma_f16(d, ad, desc_sw128_kmajor(sb + kk * 32), idesc, (ks | kk) != 0);
            if (NB == 2) umma_f16(d, ad, desc_sw128_kmajor(sb + B_BYTES + kk * 32), idesc, 1);
          }
          umma_commit(&empty_[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // nothing may be left in flight when TMEM is released
      umma_commit(&mma_done);
      mbar_wait(&mma_done, 0, a.err, 2);
    }
  } else if (warp < 2 + kConvWarps) {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x - 64;
    const int q = ct & 3;
    const int nb = a.K / 32, full = nb / 4;
    // issue side of the per-thread code ring: runs kCodeStages k-steps ahead
    int i_item = blockIdx.x, i_ks = 0, i_slot = 0;
    Coords ic = i_item < total ? coords(i_item) : Coords{0, 0, 0, 0};
    auto issue_next = [&]() {
      if (i_item < total) {
        uint8_t *slot = code_ring + i_slot * kCodeStageBytes;
        const int G = i_ks >> 1, hf = i_ks & 1;
        const size_t ebase = (size_t)(a.expert_base + ic.e) * a.rows;
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          const int r = (ct + t * kConvThreads) >> 2;
          const int R = ic.m0 + r;
          if (R < a.rows) {
            const uint8_t *row = a.codes + (ebase + R) * (size_t)(a.K / 2);
            const int off = G < full ? G * 64 + q * 16 + hf * 8 : G * 64 + q * 8;
            uint8_t *d8 = slot + (t * kConvThreads + ct) * 8;
            uint8_t *d4 = slot + kTasks * kConvThreads * 8 + (t * kConvThreads + ct) * 4;
            const uint8_t *s4 = a.scales + (ebase + R) * (size_t)a.kb_pad + G * 4;
            if (!misaligned((uint64_t)(row + off), 8, a.err, 103) &&
                !misaligned(smem_addr(d8), 8, a.err, 104))
              cp_async_8(d8, row + off);
            if (!misaligned((uint64_t)s4, 4, a.err, 105) && !misaligned(smem_addr(d4), 4, a.err, 106))
              cp_async_4(d4, s4);
          }
        }
        if (++i_ks == KSTEPS) {
          i_ks = 0;
          i_item += gridDim.x;
          if (i_item < total) ic = coords(i_item);
        }
      }
      cp_async_commit();
      if (++i_slot == kCodeStages) i_slot = 0;
    };
#pragma unroll 1
    for (int u = 0; u < kCodeStages; ++u) issue_next();
    int it = 0, c_slot = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
      const Coords c = coords(item);
      for (int ks = 0; ks < KSTEPS; ++ks, ++it) {
        const int s = it % kStagesP, r = it / kStagesP;
        cp_async_wait<kCodeStages - 1>();
        const uint8_t *slot = code_ring + c_slot * kCodeStageBytes;
        uint2 cw[kTasks];
        uint32_t sw[kTasks];
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          cw[t] = *reinterpret_cast<const uint2 *>(slot + (t * kConvThreads + ct) * 8);
          sw[t] = *reinterpret_cast<const uint32_t *>(slot + kTasks * kConvThreads * 8 +
                                                      (t * kConvThreads + ct) * 4);
        }
        issue_next();
        if (++c_slot == kCodeStages) c_slot = 0;
        if (r > 0) {  // one lane waits, the warp follows its verdict
          int w_ok = 1;
          if (lane == 0) w_ok = mbar_wait(&empty_[s], (r - 1) & 1, a.err, 5);
          if (!(ok = __shfl_sync(0xFFFFFFFFu, w_ok, 0) != 0)) break;
        }
        uint8_t *atile = tiles + s * STAGE_BYTES;
        const int hf = ks & 1;
#pragma unroll
        for (int t = 0; t < kTasks; ++t) {
          const int r_ = (ct + t * kConvThreads) >> 2;
          const int R = c.m0 + r_;
          uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
          if (R < a.rows) {
            const uint32_t s0 = (sw[t] >> (16 * hf)) & 0xFFu, s1 = (sw[t] >> (16 * hf + 8)) & 0xFFu;
            const uint32_t h0 = pack_f16x2(e8m0_to_f32(s0), e8m0_to_f32(s0));
            const uint32_t h1 = pack_f16x2(e8m0_to_f32(s1), e8m0_to_f32(s1));
            uint32_t f[4];
            e2m1x8_to_f16x8(cw[t].x, f);
            o0 = make_uint4(hmul2(f[0], h0), hmul2(f[1], h0), hmul2(f[2], h0), hmul2(f[3], h0));
            e2m1x8_to_f16x8(cw[t].y, f);
            o1 = make_uint4(hmul2(f[0], h1), hmul2(f[1], h1), hmul2(f[2], h1), hmul2(f[3], h1));
          }
          // chunks q (block 2hf) and 4 + q (block 2hf + 1), 128-byte swizzle.
          // Odd rows store their two chunks in the opposite order, so the 8
          // lanes (two rows) of each store wavefront hit 8 different banks.
          const int x7 = r_ & 7;
          uint8_t *rowp = atile + (r_ >> 3) * 1024 + x7 * 128;
          const bool odd = r_ & 1;
          *reinterpret_cast<uint4 *>(rowp + (((odd ? 4 + q : q) ^ x7) << 4)) = odd ? o1 : o0;
          *reinterpret_cast<uint4 *>(rowp + (((odd ? q : 4 + q) ^ x7) << 4)) = odd ? o0 : o1;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------------ epilogue
    const int lq = warp & 3;            // TMEM lane quarter this warp may access
    const int ew = warp - (2 + kConvWarps);
    const int r = lq * 32 + lane;       // accumulator row = weight row within the tile
    int j = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++j) {
      const Coords c = coords(item);
      const int buf = j & 1, rr = j >> 1;
      // one thread waits; the four epilogue warps follow its verdict together
      if (ew == 0 && lane == 0) epi_ok = mbar_wait(&acc_full[buf], rr & 1, a.err, 4);
      named_bar_sync(1, kEpiWarps * 32);
      const bool ok = epi_ok != 0;
      named_bar_sync(1, kEpiWarps * 32);
      if (!ok) break;
      tc_fence_after();
      const int eg = a.expert_base + c.e;
      const int pos_base = a.offsets[eg] + c.n0;
      const int R = c.m0 + r;
      const float bias_own = R < a.rows ? bf16_to_f32(a.bias[(size_t)eg * a.rows + R]) : 0.f;
      const float bias_other = __shfl_xor_sync(0xFFFFFFFFu, bias_own, 1);
      const bool up_row = lane & 1;
      for (int c0 = 0; c0 < c.nvalid; c0 += 32) {
        float v[32];
        tmem_ld_32(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        if (GEMM == 2) {
          if (R < a.H) {
            const int ncol = min(32, c.nvalid - c0);
            for (int cc = 0; cc < ncol; ++cc)
              a.y_slot[(size_t)(pos_base + c0 + cc) * a.H + R] = v[cc] + bias_own;
          }
        } else {
          // gate (even lane) and up (odd lane) of pair p = R / 2; each lane of
          // the pair computes the SwiGLU for every other column
          uint16_t *st_hi = reinterpret_cast<uint16_t *>(epi);
          uint16_t *st_lo = st_hi + 32 * 64;
          const float bg = up_row ? bias_other : bias_own, bu = up_row ? bias_own : bias_other;
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, v[cc], 1);
            if ((cc & 1) == (int)up_row) {
              const int col = c0 + cc;
              float hv = 0.f;
              if (col < c.nvalid) {
                const float sc = a.pos_scale[pos_base + col];
                const float g = up_row ? other : v[cc], u = up_row ? v[cc] : other;
                hv = swiglu_clamped(fmaf(g, sc, bg), fmaf(u, sc, bu), a.alpha, a.limit);
              }
              const uint32_t hi2 = pack_f16x2(hv, 0.f);
              const float hi = unpack_f16x2(hi2).x;
              const uint32_t lo2 = pack_f16x2(hv - hi, 0.f);
              st_hi[cc * 64 + (r >> 1)] = (uint16_t)(hi2 & 0xFFFFu);
              st_lo[cc * 64 + (r >> 1)] = (uint16_t)(lo2 & 0xFFFFu);
            }
          }
          named_bar_sync(1, kEpiWarps * 32);
          // each warp writes 8 token rows of 64 pairs (128 B) per half
          const int p0 = c.m0 >> 1;
          for (int cc = ew * 8; cc < ew * 8 + 8; ++cc) {
            const int col = c0 + cc;
            if (col < c.nvalid) {
              const size_t o = (size_t)(pos_base + col) * a.I + p0 + 2 * lane;
              if (!misaligned((uint64_t)(a.h_hi + o), 4, a.err, 107) &&
                  !misaligned((uint64_t)(a.h_lo + o), 4, a.err, 107)) {
                *reinterpret_cast<uint32_t *>(a.h_hi + o) =
                    *reinterpret_cast<const uint32_t *>(st_hi + cc * 64 + 2 * lane);
                *reinterpret_cast<uint32_t *>(a.h_lo + o) =
                    *reinterpret_cast<const uint32_t *>(st_lo + cc * 64 + 2 * lane);
              }
            }
          }
          named_bar_sync(1, kEpiWarps * 32);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
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

template <int GEMM, int BN>
size_t gemm_smem_bytes() {
  constexpr int NB = GEMM == 1 ? 1 : 2;
  return 1024 + (size_t)kStagesP * (BM * BK * 2 + NB * BN * BK * 2) +
         (size_t)kCodeStages * kCodeStageBytes + 2 * 32 * 64 * 2;
}

template <int GEMM, int BN>
cudaError_t launch_gemm(const CUtensorMap &m0, const CUtensorMap &m1, const PrefillArgs &a,
                        int n_sms, cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes<GEMM, BN>();
  auto fn = prefill_gemm_kernel<GEMM, BN>;
  cudaError_t st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (st != cudaSuccess) return st;
  fn<<<n_sms, kThreadsP, smem, stream>>>(m0, m1, a);
  return cudaGetLastError();
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
  if (w.H % BK || w.I % BK || w.E > kMaxExpertsP) return cudaErrorInvalidValue;
  CUtensorMap m0, m1;
  cudaError_t st = make_tmap(&m0, io.xp, io.S, w.H, 256);
  if (st != cudaSuccess) return st;
  m1 = m0;
  PrefillArgs a{};
  a.codes = w.w1;
  a.scales = w.s1;
  a.bias = w.b1;
  a.K = w.H;
  a.rows = 2 * w.I;
  a.kb_pad = (w.H / 32 + 3) / 4 * 4;
  a.counts = io.counts;
  a.offsets = io.offsets;
  a.n_experts = io.n_local_experts;
  a.expert_base = io.expert_base;
  a.pos_scale = io.pos_scale;
  a.h_hi = io.h_hi;
  a.h_lo = io.h_lo;
  a.I = w.I;
  a.alpha = w.alpha;
  a.limit = w.limit;
  a.H = w.H;
  a.err = io.err;
  return launch_gemm<1, 256>(m0, m1, a, n_sms, stream);
}

cudaError_t launch_prefill_mlp2(const MoeDeviceWeights &w, const PrefillIO &io, int n_sms,
                                cudaStream_t stream) {
  if (io.S == 0) return cudaSuccess;
  if (w.H % BK || w.I % BK || w.E > kMaxExpertsP) return cudaErrorInvalidValue;
  CUtensorMap m0, m1;
  cudaError_t st = make_tmap(&m0, io.h_hi, io.S, w.I, 128);
  if (st != cudaSuccess) return st;
  st = make_tmap(&m1, io.h_lo, io.S, w.I, 128);
  if (st != cudaSuccess) return st;
  PrefillArgs a{};
  a.codes = w.w2;
  a.scales = w.s2;
  a.bias = w.b2;
  a.K = w.I;
  a.rows = w.H;
  a.kb_pad = (w.I / 32 + 3) / 4 * 4;
  a.counts = io.counts;
  a.offsets = io.offsets;
  a.n_experts = io.n_local_experts;
  a.expert_base = io.expert_base;
  a.y_slot = io.y_slot;
  a.I = w.I;
  a.H = w.H;
  a.err = io.err;
  return launch_gemm<2, 128>(m0, m1, a, n_sms, stream);
}

}  // namespace oxg
