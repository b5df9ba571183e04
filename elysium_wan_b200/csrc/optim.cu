// Sharded AdamW step: fp32 master, first and second moments, gradient; writes
// the bf16 working copy in the same pass so no separate cast kernel (and no
// per-use fp32->bf16 cast in the forward) is needed.
//
// Reference: torch.optim.AdamW / the chunked recipe in
// src/wantrain/runtime/optim.py:45-56,277-298 (betas 0.9/0.95, eps 1e-8, wd 0
// by default, src/wantrain/runtime/spec.py:27). The update order follows
// torch's AdamW: decoupled decay p *= 1 - lr*wd, then
// p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps). sqrtf is CUDA's own.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

__global__ void __launch_bounds__(256)
    adamw_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                 const float* __restrict__ g, __nv_bfloat16* __restrict__ pb, int64_t n, float lr,
                 float b1, float b2, float eps, float wd, float bc1, float sqrt_bc2) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float step = lr / bc1;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = g[i];
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    float pi = p[i];
    if (wd != 0.0f) pi = pi * (1.0f - lr * wd);
    const float denom = sqrtf(vi) / sqrt_bc2 + eps;
    pi = pi - step * (mi / denom);
    m[i] = mi;
    v[i] = vi;
    p[i] = pi;
    if (pb != nullptr) pb[i] = __float2bfloat16_rn(pi);
  }
}

}  // namespace

int adamw_step(const AdamWArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return 0;
  int64_t blocks = (a.n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  adamw_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      a.p, a.m, a.v, a.g, a.p_bf16, a.n, a.lr, a.beta1, a.beta2, a.eps, a.wd, a.bc1, sqrtf(a.bc2));
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
