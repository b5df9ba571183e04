// Softmax cross-entropy over a vocabulary row, fwd + bwd in one pass pair.
//
// Reference op: F.cross_entropy(logits.float(), targets) with mean reduction
// (src/wantrain/model/gpt.py:556-557, logits made fp32 at gpt.py:418). Here the
// head GEMM writes fp32 logits directly (tcgen05 epilogue kEpiF32), one CTA
// per row computes the log-sum-exp with an online (max, sum) pair and a fixed
// reduction tree, and the same CTA writes the bf16 gradient
// (softmax - onehot) * grad_scale that feeds the head's dX / dW GEMMs.
// Deterministic: fixed per-thread strides and a fixed tree, no atomics.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

constexpr int kCeThreads = 256;

__device__ __forceinline__ void lse_combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

__global__ void __launch_bounds__(kCeThreads)
    ce_kernel(const float* __restrict__ logits, int ldl, const int64_t* __restrict__ targets,
              int V, float* __restrict__ loss_rows, __nv_bfloat16* __restrict__ dlogits, int ldg,
              float grad_scale) {
  __shared__ float sm_m[kCeThreads / 32];
  __shared__ float sm_s[kCeThreads / 32];
  const int row = blockIdx.x;
  const float* x = logits + static_cast<size_t>(row) * ldl;
  float m = -INFINITY, s = 0.f;
  for (int j = threadIdx.x; j < V; j += kCeThreads) {
    const float v = x[j];
    if (v > m) {
      s = s * expf(m - v) + 1.0f;
      m = v;
    } else {
      s += expf(v - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_combine(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm_m[w] = m;
    sm_s[w] = s;
  }
  __syncthreads();
  float M = sm_m[0], Ssum = sm_s[0];
  for (int k = 1; k < kCeThreads / 32; ++k) lse_combine(M, Ssum, sm_m[k], sm_s[k]);
  const float lse = M + logf(Ssum);
  const int64_t tgt = targets[row];
  if (threadIdx.x == 0) loss_rows[row] = lse - x[tgt];
  if (dlogits != nullptr) {
    __nv_bfloat16* g = dlogits + static_cast<size_t>(row) * ldg;
    for (int j = threadIdx.x; j < ldg; j += kCeThreads) {
      float v = 0.f;
      if (j < V) v = (expf(x[j] - lse) - (j == tgt ? 1.0f : 0.0f)) * grad_scale;
      g[j] = __float2bfloat16_rn(v);
    }
  }
}

__global__ void __launch_bounds__(1024) mean_kernel(const float* __restrict__ x, int n,
                                                    float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += 1024) s += x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) out[0] = v / static_cast<float>(n);
  }
}

}  // namespace

int cross_entropy(const CeArgs& a, cudaStream_t stream) {
  if (a.T <= 0 || a.V <= 0 || a.ldl < a.V || (a.dlogits && a.ldg < a.V)) return 1;
  ce_kernel<<<a.T, kCeThreads, 0, stream>>>(a.logits, a.ldl, a.targets, a.V, a.loss_rows,
                                            a.dlogits, a.ldg, a.grad_scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int mean_reduce(const float* x, int n, float* out, cudaStream_t stream) {
  if (n <= 0) return 1;
  mean_kernel<<<1, 1024, 0, stream>>>(x, n, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
