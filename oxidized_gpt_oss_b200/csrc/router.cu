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
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

constexpr int kRouterThreads = 256;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;

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
    // Each lane owns experts lane, lane+32, ...; repeated arg-max with ties to
    // the lower index reproduces the stable descending sort's first k.
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
        idx[(size_t)t * k + j] = top_e[j];
        wts[(size_t)t * k + j] = sum == 0.f ? 1.0f / (float)k : top_v[j] / sum;
      }
      const int ex = (int)(amax_s >> 23);  // max|x| < 2^(ex - 126)
      const int sg = ex - 141;             // max|x| * 2^-sg < 2^15
      sigma_out[t] = sg < -110 ? -110 : (sg > 100 ? 100 : sg);
    }
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

}  // namespace oxg
