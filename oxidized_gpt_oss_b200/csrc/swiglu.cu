// swiglu.cu — standalone clamped SwiGLU over device arrays.
//
// The reference's helper is ffn::swiglu (src/ffn.rs:5-13): silu(g) * u. The
// gpt-oss expert activation that this library implements is the clamped form
// g <- min(g, limit); u <- clamp(u, -limit, limit); out = g * sigmoid(alpha*g) * (u + 1),
// with alpha = 1.702 and limit = 7.0. limit = +inf, alpha = 1 and an "up" of
// u - 1 recover the reference's plain form. The same expression is fused into
// the mlp1 epilogue of the MoE kernels (moe_decode.cu).
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {
__global__ void __launch_bounds__(256) swiglu_kernel(const float *__restrict__ gate,
                                                     const float *__restrict__ up, size_t n,
                                                     float alpha, float limit,
                                                     float *__restrict__ out) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = swiglu_clamped(gate[i], up[i], alpha, limit);
}
}  // namespace

cudaError_t launch_swiglu(const float *gate, const float *up, size_t n, float alpha, float limit,
                          float *out, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  size_t want = (n + 255) / 256;
  unsigned grid = (unsigned)(want < 148 * 16 ? want : 148 * 16);
  swiglu_kernel<<<grid, 256, 0, stream>>>(gate, up, n, alpha, limit, out);
  return cudaGetLastError();
}

}  // namespace oxg
