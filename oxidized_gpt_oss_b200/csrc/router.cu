// router.cu — router GEMV + bias, top-k selection and softmax over the k.
//
// Follows MoELayer::forward of the reference (src/moe.rs:40-73):
//   logits[t, e] = x[t, :] . W[e, :]          (W stored [E, H], A*B^T, src/utils.rs:34-89)
//                 + b[e]                       (gpt-oss router bias; the reference has none)
//   take the k largest logits in the order of a stable descending sort, i.e.
//   ties go to the lower expert index (src/moe.rs:53-60);
//   softmax over those k (max-subtracted, sum accumulated in j order, uniform
//   if the sum is 0; src/utils.rs:91-111).
//
// One CTA of 256 threads per token: the x row is staged in shared memory as
// f32, warp w computes the logits of experts w, w+8, ... with lanes striding
// over H in 16-byte bf16 chunks, and warp 0 selects and normalises.
//
// The kernel also emits, per token, the power-of-two exponent sigma that puts
// max|x| * 2^-sigma in [2^14, 2^15); the MoE kernels feed x to f16 tensor-core
// operands as x * 2^-sigma and multiply the products back by 2^sigma. A bf16
// value (8 significant bits) converts to f16 exactly down to 2^-17, so every
// element of magnitude >= 2^-31 max|x| is exact; smaller ones are rounded to
// the f16 subnormal grid with absolute error <= 2^-39 max|x|.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace oxg {
namespace {

constexpr int kRouterThreads = 256;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;

// One warp selects the k largest of E logits (logit_s, shared memory) in the
// order of a stable descending sort and writes their softmax: each lane owns
// experts lane, lane+32, ...; a repeated arg-max with ties to the lower index
// reproduces the stable sort's first k. Optionally also the ids to idx_smem.
__device__ __forceinline__ void select_topk_softmax(const float *logit_s, int E, int k, int lane,
                                                    int32_t *__restrict__ idx_out,
                                                    float *__restrict__ wts_out,
                                                    int32_t *idx_smem) {
  constexpr int kPer = kMaxExperts / 32;
  float v[kPer];
  bool taken[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? logit_s[e] : -INFINITY;
    taken[i] = !(e < E);
  }
  float top_v[kMaxTopK];
  int top_e[kMaxTopK];
  for (int j = 0; j < k; ++j) {
    float bv = 0.f;
    int be = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (!taken[i] && (be == 0x7FFFFFFF || v[i] > bv)) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
      const bool other_better =
          oe != 0x7FFFFFFF && (be == 0x7FFFFFFF || ov > bv || (ov == bv && oe < be));
      if (other_better) {
        bv = ov;
        be = oe;
      }
    }
    top_v[j] = bv;
    top_e[j] = be;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == be) taken[i] = true;
  }
  if (lane == 0) {
    float mx = -INFINITY;
    for (int j = 0; j < k; ++j) mx = fmaxf(mx, top_v[j]);
    float sum = 0.f;
    for (int j = 0; j < k; ++j) {
      top_v[j] = expf(top_v[j] - mx);
      sum += top_v[j];
    }
    for (int j = 0; j < k; ++j) {
      idx_out[j] = top_e[j];
      wts_out[j] = sum == 0.f ? 1.0f / (float)k : top_v[j] / sum;
      if (idx_smem) idx_smem[j] = top_e[j];
    }
  }
}

// sigma from the biased exponent of max|x| (as f32 bits >> 23): max|x| <
// 2^(ex - 126), so max|x| * 2^-sigma < 2^15; clamped to [-110, 100].
__device__ __forceinline__ int sigma_of(uint32_t ex) {
  const int sg = (int)ex - 141;
  return sg < -110 ? -110 : (sg > 100 ? 100 : sg);
}

__global__ void __launch_bounds__(kRouterThreads) router_topk_kernel(
    const uint16_t *__restrict__ x, const uint16_t *__restrict__ w, const uint16_t *__restrict__ b,
    int H, int E, int k, int32_t *__restrict__ idx, float *__restrict__ wts,
    float *__restrict__ logits_out, int32_t *__restrict__ sigma_out) {
  extern __shared__ float xs[];  // [H]
  __shared__ float logit_s[kMaxExperts];
  __shared__ uint32_t amax_s;
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t *xr = x + (size_t)t * H;
  if (tid == 0) amax_s = 0u;
  __syncthreads();
  uint32_t amax = 0u;
  for (int i = tid; i < H / 2; i += kRouterThreads) {
    uint32_t pair = reinterpret_cast<const uint32_t *>(xr)[i];
    float lo = bf16_to_f32(pair & 0xFFFFu), hi = bf16_to_f32(pair >> 16);
    xs[2 * i] = lo;
    xs[2 * i + 1] = hi;
    amax = max(amax, max(__float_as_uint(lo) & 0x7FFFFFFFu, __float_as_uint(hi) & 0x7FFFFFFFu));
  }
  atomicMax(&amax_s, amax);
  __syncthreads();

  for (int e = warp; e < E; e += kRouterThreads / 32) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)e * H);
    float acc = 0.f;
    for (int c = lane; c < H / 8; c += 32) {
      uint4 q = __ldg(wr + c);
      const float *xv = xs + 8 * c;
      acc = fmaf(xv[0], bf16_to_f32(q.x & 0xFFFFu), acc);
      acc = fmaf(xv[1], bf16_to_f32(q.x >> 16), acc);
      acc = fmaf(xv[2], bf16_to_f32(q.y & 0xFFFFu), acc);
      acc = fmaf(xv[3], bf16_to_f32(q.y >> 16), acc);
      acc = fmaf(xv[4], bf16_to_f32(q.z & 0xFFFFu), acc);
      acc = fmaf(xv[5], bf16_to_f32(q.z >> 16), acc);
      acc = fmaf(xv[6], bf16_to_f32(q.w & 0xFFFFu), acc);
      acc = fmaf(xv[7], bf16_to_f32(q.w >> 16), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) {
      if (b) acc += bf16_to_f32(b[e]);
      logit_s[e] = acc;
      if (logits_out) logits_out[(size_t)t * E + e] = acc;
    }
  }
  __syncthreads();

  if (warp == 0) {
    select_topk_softmax(logit_s, E, k, lane, idx + (size_t)t * k, wts + (size_t)t * k, nullptr);
    if (lane == 0) sigma_out[t] = sigma_of(amax_s >> 23);
  }
}


// ---- batched router on the tensor cores -------------------------------------
// CTAs of 64 tokens and 16 warps: warp w computes the logits of token block
// w % 4 (16 tokens) against expert n-tiles w / 4 and w / 4 + 4 (8 experts
// each) with mma.sync.m16n8k16 on bf16 operands (exact products, f32
// accumulation), streaming x and W through a kRmStages-deep shared-memory
// ring of 128-column chunks (cp.async, 16-byte chunks XOR-swizzled by row so
// the ldmatrix reads are conflict-free; one barrier per chunk). max|x| per
// token comes from the A fragments. After the bias, each warp selects the
// top k of 4 tokens (rank_topk_softmax, the same selection and softmax as
// above); then warp 0 ranks the CTA's T*k slots per expert in slot order
// (the counting sort's first half): local_rank of each slot and the CTA's
// histogram, which scatter_kernel turns into positions. (Four warps of 16
// tokens x all experts each measured issue-bound: one warp per scheduler.)
constexpr int kRmTokens = 64;
constexpr int kRmWarps = 16;
constexpr int kRmThreads = kRmWarps * 32;
constexpr int kRmKC = 128;  // columns per chunk
constexpr int kRmMaxE = 64;
constexpr int kRmStages = 4;

__global__ void __launch_bounds__(kRmThreads) router_mma_kernel(
    const uint16_t *__restrict__ x, const uint16_t *__restrict__ w, const uint16_t *__restrict__ b,
    int T, int H, int E, int k, int32_t *__restrict__ idx, float *__restrict__ wts,
    float *__restrict__ logits_out, int32_t *__restrict__ sigma_out,
    int32_t *__restrict__ cta_hist, int32_t *__restrict__ local_rank) {
  extern __shared__ __align__(128) uint8_t rm_smem[];
  __shared__ float logit_s[kRmTokens][kRmMaxE];
  __shared__ int32_t idx_s[kRmTokens * kMaxTopK];
  __shared__ int cnt_s[kRmMaxE];
  __shared__ float top_v_s[kRmWarps][kMaxTopK];
  __shared__ int top_e_s[kRmWarps][kMaxTopK];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tb = warp & 3, eq = warp >> 2;  // token block (16 rows), first expert n-tile
  const int t0 = blockIdx.x * kRmTokens;
  const int stage_bytes = (kRmTokens + E) * kRmKC * 2;
  const int n_chunks = (H + kRmKC - 1) / kRmKC;
  const int NT = E / 8;  // n-tiles of 8 experts (E is a multiple of 16)
  const bool has0 = eq < NT, has1 = eq + 4 < NT;

  // chunk c into ring slot c % kRmStages (one commit group per call, empty
  // past the last chunk so the group count stays uniform)
  auto load_chunk = [&](int c) {
    if (c < n_chunks) {
      uint8_t *xs = rm_smem + (c % kRmStages) * stage_bytes;
      uint8_t *ws = xs + kRmTokens * kRmKC * 2;
      const int k0 = c * kRmKC;
      for (int i = threadIdx.x; i < (kRmTokens + E) * 16; i += kRmThreads) {
        const int r = i >> 4, ch = i & 15, col = k0 + ch * 8;
        const bool is_x = r < kRmTokens;
        const int row = is_x ? r : r - kRmTokens;
        const bool ok = col < H && (!is_x || t0 + row < T);
        const uint16_t *src = is_x ? x + (size_t)(ok ? t0 + row : 0) * H + (ok ? col : 0)
                                   : w + (size_t)row * H + (ok ? col : 0);
        uint8_t *dst = (is_x ? xs : ws) + row * (kRmKC * 2) + ((ch ^ (row & 7)) << 4);
        cp_async_16_zfill(dst, src, ok ? 16u : 0u);
      }
    }
    cp_async_commit();
  };

  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  uint32_t amax_lo = 0u, amax_hi = 0u;  // |x| bf16 bits of rows g and g + 8, two per register
  const int mi = lane >> 3, ri = lane & 7;
  const int arow = tb * 16 + ri + 8 * (mi & 1);
  // B matrices 0, 1: n-tile eq (k 0-7, 8-15); 2, 3: n-tile eq + 4 (or eq again)
  const int brow = 8 * ((mi >> 1) && has1 ? eq + 4 : eq) + ri;

#pragma unroll
  for (int c = 0; c < kRmStages - 1; ++c) load_chunk(c);
  for (int c = 0; c < n_chunks; ++c) {
    cp_async_wait<kRmStages - 2>();  // chunk c has landed (this thread's copies)
    __syncthreads();                 // ... everyone's; and slot (c - 1) % S is free
    load_chunk(c + kRmStages - 1);
    if (!has0) continue;
    const uint8_t *xs = rm_smem + (c % kRmStages) * stage_bytes;
    const uint8_t *ws = xs + kRmTokens * kRmKC * 2;
#pragma unroll
    for (int kk = 0; kk < kRmKC / 16; ++kk) {
      const int ach = 2 * kk + (mi >> 1), bch = 2 * kk + (mi & 1);
      uint32_t a[4], bq[4];
      ldmatrix_x4(a, xs + arow * (kRmKC * 2) + ((ach ^ (arow & 7)) << 4));
      ldmatrix_x4(bq, ws + brow * (kRmKC * 2) + ((bch ^ (brow & 7)) << 4));
      if (eq == 0) {
        amax_lo = __vmaxu2(amax_lo, __vmaxu2(a[0] & 0x7FFF7FFFu, a[2] & 0x7FFF7FFFu));
        amax_hi = __vmaxu2(amax_hi, __vmaxu2(a[1] & 0x7FFF7FFFu, a[3] & 0x7FFF7FFFu));
      }
      mma_bf16_16816(acc[0], a, bq[0], bq[1]);
      if (has1) mma_bf16_16816(acc[1], a, bq[2], bq[3]);
    }
  }
  cp_async_wait<0>();

  // logits (+ bias) of rows g and g + 8 of token block tb, experts
  // 8 tile + 2q + {0, 1}
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (u == 0 ? has0 : has1) {
      const int e0 = 8 * (eq + 4 * u) + 2 * q;
      const float b0 = b ? bf16_to_f32(b[e0]) : 0.f, b1 = b ? bf16_to_f32(b[e0 + 1]) : 0.f;
      logit_s[tb * 16 + g][e0] = acc[u][0] + b0;
      logit_s[tb * 16 + g][e0 + 1] = acc[u][1] + b1;
      logit_s[tb * 16 + g + 8][e0] = acc[u][2] + b0;
      logit_s[tb * 16 + g + 8][e0 + 1] = acc[u][3] + b1;
    }
  }
  if (eq == 0) {
    // max|x| of the rows: halves of the packed maxima, then over the quad
    uint32_t mlo = max(amax_lo & 0xFFFFu, amax_lo >> 16), mhi = max(amax_hi & 0xFFFFu, amax_hi >> 16);
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      mlo = max(mlo, __shfl_xor_sync(0xFFFFFFFFu, mlo, o));
      mhi = max(mhi, __shfl_xor_sync(0xFFFFFFFFu, mhi, o));
    }
    if (q == 0) {
      const int ta = t0 + tb * 16 + g, tbb = ta + 8;
      if (ta < T) sigma_out[ta] = sigma_of(mlo >> 7);  // bf16 bits >> 7 = f32 exponent
      if (tbb < T) sigma_out[tbb] = sigma_of(mhi >> 7);
    }
  }
  __syncthreads();  // every expert column of every token is in logit_s
  const int n_tok = min(kRmTokens, T - t0);
  constexpr int kTokPerWarp = kRmTokens / kRmWarps;
  for (int tl = warp * kTokPerWarp; tl < (warp + 1) * kTokPerWarp && tl < n_tok; ++tl) {
    const size_t t = (size_t)t0 + tl;
    rank_topk_softmax(logit_s[tl], E, k, lane, idx + t * k, wts + t * k, idx_s + tl * k, top_v_s[warp],
                      top_e_s[warp]);
  }
  __syncthreads();
  if (logits_out)
    for (int i = threadIdx.x; i < n_tok * E; i += kRmThreads)
      logits_out[(size_t)t0 * E + i] = logit_s[i / E][i % E];
  if (warp == 0) {
    for (int e = lane; e < E; e += 32) cnt_s[e] = 0;
    __syncwarp();
    const int n_slots = n_tok * k;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int s0 = 0; s0 < n_slots; s0 += 32) {
      const int sl = s0 + lane;
      const bool valid = sl < n_slots;
      const int e = valid ? idx_s[sl] : E + lane;  // distinct dummies never match
      const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
      const int prior = valid ? cnt_s[e] : 0;
      __syncwarp();
      if (valid) {
        local_rank[(size_t)t0 * k + sl] = prior + __popc(peers & lt_mask);
        if ((peers & lt_mask) == 0u) cnt_s[e] = prior + __popc(peers);
      }
      __syncwarp();
    }
    for (int e = lane; e < E; e += 32) cta_hist[(size_t)blockIdx.x * E + e] = cnt_s[e];
  }
}


// ---- batched router on tcgen05 -------------------------------------------------
// One CTA per 128 tokens (M = 128 of a kind::f16 MMA with bf16 operands, N =
// E experts, f32 accumulator in TMEM), the x tile and the router rows (both
// K-major, 64 columns per stage, 128-byte swizzle) streamed by TMA through a
// kTcStages-deep ring:
//   warp 0     TMA producer (one thread)
//   warp 1     TMEM owner and MMA issuer (one thread): 4 MMAs of K 16 per stage
//   warps 2-5  one token row per thread (the thread's TMEM lane): max|x| of
//              its row from each stage's x tile (a stage is free once the
//              MMAs and these four warps are done with it); then the logits
//              from TMEM, bias, top-k and softmax of its token (the same
//              selection and arithmetic as rank_topk_softmax), and per 64-token
//              half of the tile the histogram and slot ranks of the counting
//              sort (the batched router's outputs, in its 64-token units).
// Every wait is bounded: a timeout records code 14 in *err and the pipeline
// drains without hanging.
constexpr int kTcTokens = 128;
constexpr int kTcBK = 64;
constexpr int kTcStages = 6;
constexpr int kTcThreads = 192;
constexpr uint32_t kTcXBytes = kTcTokens * kTcBK * 2;  // 16 KB

__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                          // D format: f32
         | (1u << 7) | (1u << 10)           // A, B format: bf16
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

template <int EMAX>
__global__ void __launch_bounds__(kTcThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                     const uint16_t *__restrict__ b, int T, int H, int E, int k, int32_t *__restrict__ idx,
                     float *__restrict__ wts, float *__restrict__ logits_out, int32_t *__restrict__ sigma_out,
                     int32_t *__restrict__ cta_hist, int32_t *__restrict__ local_rank, int *err) {
  extern __shared__ uint8_t tc_raw[];
  uint8_t *smem = tc_raw + ((1024u - (sm100::smem_addr(tc_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full_[kTcStages], empty_[kTcStages], acc_full;
  __shared__ uint32_t tmem_slot;
  __shared__ int idx_s[kTcTokens * kMaxTopK];
  __shared__ int cnt_s[2][EMAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kTcTokens;
  const uint32_t w_bytes = (uint32_t)E * kTcBK * 2;
  const uint32_t stage_bytes = kTcXBytes + EMAX * kTcBK * 2;
  const int KSTEPS = H / kTcBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      sm100::mbar_init(&full_[s], 1);
      sm100::mbar_init(&empty_[s], 1 + 4);  // the MMA commit + the four row warps
    }
    sm100::mbar_init(&acc_full, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(&tmem_slot, EMAX);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      sm100::prefetch_tmap(&xmap);
      sm100::prefetch_tmap(&wmap);
      int issued = 0;
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int s = ks % kTcStages, r = ks / kTcStages;
        if (r > 0 && !sm100::mbar_wait(&empty_[s], (r - 1) & 1, err, 14)) break;
        uint8_t *st = smem + (size_t)s * stage_bytes;
        sm100::mbar_arrive_expect_tx(&full_[s], kTcXBytes + w_bytes);
        sm100::tma_load_2d(st, &xmap, &full_[s], ks * kTcBK, t0);
        sm100::tma_load_2d(st + kTcXBytes, &wmap, &full_[s], ks * kTcBK, 0);
        issued = ks + 1;
      }
      // after a timeout elsewhere: the copies still in flight land before the CTA exits
      for (int ks = issued - 1; ks >= 0 && ks >= issued - kTcStages; --ks)
        if (!sm100::mbar_wait(&full_[ks % kTcStages], (ks / kTcStages) & 1, err, 14)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTcTokens, E);
      const uint64_t d0 = sm100::desc_sw128_kmajor(sm100::smem_addr(smem));
      bool ok = true;
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int s = ks % kTcStages;
        if (!(ok = sm100::mbar_wait(&full_[s], (ks / kTcStages) & 1, err, 14))) break;
        sm100::tc_fence_after();
        const uint64_t ad = d0 + (uint64_t)(s * (stage_bytes >> 4));
        const uint64_t bd = ad + (uint64_t)(kTcXBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk) sm100::umma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0);
        sm100::umma_commit(&empty_[s]);
      }
      sm100::umma_commit(&acc_full);  // also after a timeout
      sm100::mbar_wait(&acc_full, 0, err, 14);  // no MMA in flight when TMEM is released
    }
  } else {
    // ---- row warps: thread = token row = TMEM lane
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int t = t0 + row;
    uint32_t amax = 0u;  // max |x| of the row as two packed bf16 magnitudes
    bool ok = true;
    for (int ks = 0; ks < KSTEPS && ok; ++ks) {
      const int s = ks % kTcStages;
      if (!(ok = sm100::mbar_wait(&full_[s], (ks / kTcStages) & 1, err, 14))) break;
      // the row's 128 bytes (its 16-byte chunks are swizzled within the row
      // and the maximum does not care about their order): iteration c reads
      // chunk c ^ (row & 7), so the 8 rows of a quarter warp hit 8 distinct
      // bank groups (all at chunk c: an 8-way conflict)
      const uint4 *rp = reinterpret_cast<const uint4 *>(smem + (size_t)s * stage_bytes + (size_t)row * 128);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = rp[c ^ (row & 7)];
        amax = __vmaxu2(amax, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                       __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty_[s]);
    }
    sm100::mbar_wait(&acc_full, 0, err, 14);
    sm100::tc_fence_after();
    float v[EMAX];
    {
      uint32_t r[32];
      sm100::tmem_ld_32_async(tmem + ((uint32_t)(q * 32) << 16), r);
      sm100::tmem_wait_ld(r);
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
      if constexpr (EMAX > 32) {
        sm100::tmem_ld_32_async(tmem + ((uint32_t)(q * 32) << 16) + 32u, r);
        sm100::tmem_wait_ld(r);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[32 + e] = __uint_as_float(r[e]);
      }
    }
    sm100::tc_fence_before();
    const bool valid = t < T;
#pragma unroll
    for (int e = 0; e < EMAX; ++e) {
      if (e < E) {
        v[e] += b ? bf16_to_f32(b[e]) : 0.f;
        if (valid && logits_out) logits_out[(size_t)t * E + e] = v[e];
        if (v[e] != v[e]) v[e] = -INFINITY;  // NaN ranks last, as in rank_topk_softmax
      }
    }
    if (valid) {
      const uint32_t m = max(amax & 0xFFFFu, amax >> 16);
      sigma_out[t] = sigma_of(m >> 7);  // bf16 bits >> 7 = f32 exponent
      // the k largest, ties to the lower expert (a stable descending sort)
      float top_v[kMaxTopK];
      int top_e[kMaxTopK];
      uint64_t taken = 0ull;
      for (int j = 0; j < k; ++j) {
        int be = -1;
        float bv = -INFINITY;
#pragma unroll
        for (int e = 0; e < EMAX; ++e)
          if (e < E && !((taken >> e) & 1ull) && (be < 0 || v[e] > bv)) {
            be = e;
            bv = v[e];
          }
        taken |= 1ull << be;
        top_v[j] = bv;
        top_e[j] = be;
      }
      float mx = -INFINITY;
      for (int j = 0; j < k; ++j) mx = fmaxf(mx, top_v[j]);
      float sum = 0.f;
      for (int j = 0; j < k; ++j) {
        top_v[j] = expf(top_v[j] - mx);
        sum += top_v[j];
      }
      for (int j = 0; j < k; ++j) {
        idx[(size_t)t * k + j] = top_e[j];
        wts[(size_t)t * k + j] = sum == 0.f ? 1.0f / (float)k : top_v[j] / sum;
        idx_s[row * k + j] = top_e[j];
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four row warps: every idx_s entry is written
    // the counting sort's first half per 64-token unit: warp of quarter 0
    // (rows 0-63) and of quarter 2 (rows 64-127)
    if (q == 0 || q == 2) {
      const int h = q >> 1, n_tok = min(64, T - (t0 + 64 * h));
      if (n_tok > 0) {
        int *cnt = cnt_s[h];
        for (int e = lane; e < E; e += 32) cnt[e] = 0;
        __syncwarp();
        const int n_slots = n_tok * k;
        const unsigned lt_mask = (1u << lane) - 1u;
        for (int s0 = 0; s0 < n_slots; s0 += 32) {
          const int sl = s0 + lane;
          const bool sv = sl < n_slots;
          const int e = sv ? idx_s[64 * h * k + sl] : E + lane;  // distinct dummies never match
          const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
          const int prior = sv ? cnt[e] : 0;
          __syncwarp();
          if (sv) {
            local_rank[(size_t)(t0 + 64 * h) * k + sl] = prior + __popc(peers & lt_mask);
            if ((peers & lt_mask) == 0u) cnt[e] = prior + __popc(peers);
          }
          __syncwarp();
        }
        for (int e = lane; e < E; e += 32) cta_hist[(size_t)(2 * blockIdx.x + h) * E + e] = cnt[e];
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, EMAX);
  }
}
}  // namespace

cudaError_t launch_router_topk(const uint16_t *x, const uint16_t *w, const uint16_t *b, int T, int H,
                               int E, int k, int32_t *idx, float *wts, float *logits,
                               int32_t *sigma, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (E > kMaxExperts || k > kMaxTopK || k > E || H % 8) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * sizeof(float);
  // opt in unconditionally: static plus dynamic shared memory is what counts
  cudaError_t st = cudaFuncSetAttribute(router_topk_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (st != cudaSuccess) return st;
  router_topk_kernel<<<T, kRouterThreads, smem, stream>>>(x, w, b, H, E, k, idx, wts, logits,
                                                          sigma);
  return cudaGetLastError();
}

bool router_mma_supported(int H, int E, int k) {
  return E % 16 == 0 && E <= kRmMaxE && k <= kMaxTopK && k <= E && H % 16 == 0;
}

int router_mma_ctas(int T) { return (T + kRmTokens - 1) / kRmTokens; }

namespace {
typedef CUresult (*RouterEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
RouterEncodeFn router_encode_fn() {
  static RouterEncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<RouterEncodeFn>(p);
  }
  return fn;
}
// [rows, cols] bf16 row-major, box [64 cols, box_rows], 128-byte swizzle (rows
// past the end read as zeros).
bool router_tmap(CUtensorMap *m, const void *base, int rows, int cols, int box_rows) {
  RouterEncodeFn fn = router_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_router_mma(const uint16_t *x, const uint16_t *w, const uint16_t *b, int T, int H,
                              int E, int k, int32_t *idx, float *wts, float *logits,
                              int32_t *sigma, int32_t *cta_hist, int32_t *local_rank,
                              cudaStream_t stream, int *err) {
  if (T == 0) return cudaSuccess;
  if (!router_mma_supported(H, E, k)) return cudaErrorInvalidValue;
  if ((uintptr_t)x & 15 || (uintptr_t)w & 15) return cudaErrorInvalidValue;
  CUtensorMap xm, wm;
  if (err && H % kTcBK == 0 && router_tmap(&xm, x, T, H, kTcTokens) && router_tmap(&wm, w, E, H, E)) {
    // tcgen05: one CTA per 128 tokens
    const int emax = E <= 32 ? 32 : 64;
    const size_t smem = 1024 + (size_t)kTcStages * (kTcXBytes + (size_t)emax * kTcBK * 2);
    const int grid = (T + kTcTokens - 1) / kTcTokens;
    cudaError_t st;
    if (emax == 32) {
      st = cudaFuncSetAttribute(router_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (st != cudaSuccess) return st;
      router_tc_kernel<32><<<grid, kTcThreads, smem, stream>>>(xm, wm, b, T, H, E, k, idx, wts, logits, sigma,
                                                                cta_hist, local_rank, err);
    } else {
      st = cudaFuncSetAttribute(router_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (st != cudaSuccess) return st;
      router_tc_kernel<64><<<grid, kTcThreads, smem, stream>>>(xm, wm, b, T, H, E, k, idx, wts, logits, sigma,
                                                                cta_hist, local_rank, err);
    }
    return cudaGetLastError();
  }
  const size_t smem = (size_t)kRmStages * (kRmTokens + E) * kRmKC * 2;
  cudaError_t st = cudaFuncSetAttribute(router_mma_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (st != cudaSuccess) return st;
  router_mma_kernel<<<router_mma_ctas(T), kRmThreads, smem, stream>>>(
      x, w, b, T, H, E, k, idx, wts, logits, sigma, cta_hist, local_rank);
  return cudaGetLastError();
}

}  // namespace oxg
