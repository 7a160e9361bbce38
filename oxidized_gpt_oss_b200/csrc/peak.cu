// peak.cu — issue-rate measurement of the tensor-core instruction kinds the
// MoE kernels use, to give the prefill GEMMs a measured denominator.
//
// One CTA per SM; one thread issues `iters` back-to-back MMAs of one kind
// into a single TMEM accumulator from one A tile and one B tile that stay in
// shared memory (zero-filled; the scale factors of the block-scaled kinds
// are zero bytes copied into TMEM once), then commits and waits (bounded)
// for them to finish. No global memory is read, so the time is the tensor
// pipe's alone:
//   kind 0: tcgen05.mma.kind::f16 (f16 x f16 -> f32),           M 128, N 256, K 16
//   kind 1: tcgen05.mma.kind::mxf8f6f4.block_scale (E2M1 x E4M3), M 128, N 256, K 32
//   kind 2: tcgen05.mma.kind::mxf4.block_scale.block32 (E2M1 x E2M1, packed), M 128, N 256, K 64
// Both operand tiles are K-major with the 128-byte swizzle (one 128-byte
// row per operand row, 8-row atoms of 1024 bytes); consecutive MMAs walk
// the four 32-byte K slices of the row (16 f16, 32 one-byte or 64 packed
// four-bit elements each).
#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"
#include "sm100.cuh"

namespace oxg {
namespace {

using namespace sm100;

constexpr int kPeakM = 128, kPeakN = 256;
constexpr int kPeakA = kPeakM * 128, kPeakB = kPeakN * 128;  // bytes of the two tiles
constexpr int kPeakErr = 31;  // error word: the final commit did not arrive

// kind::mxf4 instruction descriptor: A and B E2M1 (format 1 of this kind),
// UE8M0 scales, K-major, dense K = 64.
__host__ __device__ constexpr uint32_t idesc_mxf4(int m, int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_mxf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

template <int KIND>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int iters, int *err) {
  extern __shared__ uint8_t peak_raw[];
  uint8_t *sm = peak_raw + ((1024u - (smem_addr(peak_raw) & 1023u)) & 1023u);
  uint8_t *a_tile = sm, *b_tile = sm + kPeakA, *atoms = sm + kPeakA + kPeakB;  // 2 scale atoms
  __shared__ uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kPeakA + kPeakB + 2 * mxf::kAtomBytes) / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(sm)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t sfa = tmem + 256, sfb = tmem + 260;  // scale columns past the accumulator
    if (KIND != 0) {
      mxf::utccp_atom(sfa, smem_addr(atoms));
      mxf::utccp_atom(sfb, smem_addr(atoms + mxf::kAtomBytes));
    }
    const uint64_t ad = desc_sw128_kmajor(smem_addr(a_tile)), bd = desc_sw128_kmajor(smem_addr(b_tile));
    for (int i = 0; i < iters; ++i) {
      const int kk = i & 3;  // 32-byte K slice of the 128-byte rows
      if (KIND == 0)
        umma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc_f16_f32(kPeakM, kPeakN), i != 0);
      else if (KIND == 1)
        mxf::umma_mxf(tmem, ad + 2 * kk, bd + 2 * kk, mxf::idesc_e2m1_e4m3(kPeakM, kPeakN, 0, 0), sfa, sfb, i != 0);
      else
        umma_mxf4(tmem, ad + 2 * kk, bd + 2 * kk, idesc_mxf4(kPeakM, kPeakN), sfa, sfb, i != 0);
    }
    umma_commit(&done_bar);
    mbar_wait(&done_bar, 0, err, kPeakErr);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace

double mma_flops_per_instr(int kind) {
  const int K = kind == 0 ? 16 : (kind == 1 ? 32 : 64);
  return 2.0 * kPeakM * kPeakN * K;
}

cudaError_t launch_mma_rate(int kind, int iters, int n_ctas, int *err, cudaStream_t stream) {
  if (kind < 0 || kind > 2 || iters < 1 || n_ctas < 1) return cudaErrorInvalidValue;
  const size_t smem = 1024 + kPeakA + kPeakB + 2 * mxf::kAtomBytes;
  auto launch = [&](auto fn) {
    cudaError_t st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
    fn<<<n_ctas, 128, smem, stream>>>(iters, err);
    return cudaGetLastError();
  };
  if (kind == 0) return launch(mma_rate_kernel<0>);
  if (kind == 1) return launch(mma_rate_kernel<1>);
  return launch(mma_rate_kernel<2>);
}

}  // namespace oxg
