// Softmax cross-entropy over a vocabulary row, fwd + bwd in one kernel.
//
// Reference op: F.cross_entropy(logits.float(), targets) with mean reduction
// (src/wantrain/model/gpt.py:556-557, logits made fp32 at gpt.py:418). Here the
// head GEMM writes fp32 logits directly (tcgen05 epilogue kEpiF32) and one CTA
// per row writes the loss and the bf16 gradient (softmax - onehot) * grad_scale
// that feeds the head's dX / dW GEMMs.
//
// Main path (rows up to 56K fp32, the GPT-2 vocabulary among them): the CTA
// copies its whole row into shared memory with bulk copies (one HBM read of
// the logits; a 2048 x 50257 fp32 block is 3x the L2, so a second pass would
// go to DRAM again), then max, sum of exp(x - max) (kept in place) and the
// gradient run from shared memory. Other rows: an online (max, sum) pass and a
// gradient pass over global memory.
// Deterministic: fixed per-thread element sets and fixed reduction trees.
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
              float grad_scale, int* status) {
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
  // A target outside the vocabulary is reported (status record) and gives a
  // NaN loss instead of a read outside the row.
  const bool tgt_ok = tgt >= 0 && tgt < V;
  if (threadIdx.x == 0) {
    if (!tgt_ok) record_check(status, kStatusBadArgument, kSiteCeTarget, row, tgt);
    loss_rows[row] = tgt_ok ? lse - x[tgt] : __int_as_float(0x7fc00000);
  }
  if (dlogits != nullptr) {
    __nv_bfloat16* g = dlogits + static_cast<size_t>(row) * ldg;
    for (int j = threadIdx.x; j < ldg; j += kCeThreads) {
      float v = 0.f;
      if (j < V) v = (expf(x[j] - lse) - (j == tgt ? 1.0f : 0.0f)) * grad_scale;
      g[j] = __float2bfloat16_rn(v);
    }
  }
}

constexpr int kCeSmemThreads = 1024;
constexpr int kCeSmemMaxBytes = 225 * 1024;  // row buffer; 16 bytes of barrier follow
constexpr int kCeCopyChunk = 32768;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  // fixed tree: xor butterfly in each warp, then warp 0 over the 32 warp results
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read from the previous reduction
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = red[l];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, u) : v + u;
    }
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

__global__ void __launch_bounds__(kCeSmemThreads, 1)
    ce_smem_kernel(const float* __restrict__ logits, int ldl, const int64_t* __restrict__ targets,
                   int V, float* __restrict__ loss_rows, __nv_bfloat16* __restrict__ dlogits,
                   int ldg, float grad_scale, int row_bytes, int* status) {
  extern __shared__ __align__(16) uint8_t ce_smem[];
  float* xs = reinterpret_cast<float*>(ce_smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(ce_smem + row_bytes);
  __shared__ float red[33];
  const int row = blockIdx.x;
  const float* x = logits + static_cast<size_t>(row) * ldl;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(row_bytes));
    for (int off = 0; off < row_bytes; off += kCeCopyChunk)
      bulk_load(ce_smem + off, reinterpret_cast<const uint8_t*>(x) + off,
                static_cast<uint32_t>(min(kCeCopyChunk, row_bytes - off)), bar);
  }
  const bool landed = __syncthreads_and(mbar_wait(bar, 0, status, kStatusTimeoutSmemFull));
  if (!landed) {
    // status recorded; give the copies in flight one more bounded wait before exiting
    if (threadIdx.x == 0) mbar_wait(bar, 0, nullptr, kStatusTimeoutDrain);
    return;
  }
  const int n4 = (V + 3) >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n4; i += kCeSmemThreads) {
    const float4 v = x4[i];
    const int j = 4 * i;
    m = fmaxf(m, v.x);
    if (j + 1 < V) m = fmaxf(m, v.y);
    if (j + 2 < V) m = fmaxf(m, v.z);
    if (j + 3 < V) m = fmaxf(m, v.w);
  }
  const float M = block_reduce(m, red, true);
  float s = 0.f;
  float4* e4 = reinterpret_cast<float4*>(xs);
  for (int i = threadIdx.x; i < n4; i += kCeSmemThreads) {
    float4 v = x4[i];
    const int j = 4 * i;
    v.x = expf(v.x - M);
    v.y = (j + 1 < V) ? expf(v.y - M) : 0.f;
    v.z = (j + 2 < V) ? expf(v.z - M) : 0.f;
    v.w = (j + 3 < V) ? expf(v.w - M) : 0.f;
    s += (v.x + v.y) + (v.z + v.w);
    e4[i] = v;
  }
  const float S = block_reduce(s, red, false);
  const float lse = M + logf(S);
  const int64_t tgt = targets[row];
  // A target outside the vocabulary is reported (status record) and gives a
  // NaN loss instead of a read outside the row.
  const bool tgt_ok = tgt >= 0 && tgt < V;
  if (threadIdx.x == 0) {
    if (!tgt_ok) record_check(status, kStatusBadArgument, kSiteCeTarget, row, tgt);
    loss_rows[row] = tgt_ok ? lse - x[tgt] : __int_as_float(0x7fc00000);
  }
  if (dlogits == nullptr) return;
  const float inv = 1.0f / S;
  __nv_bfloat16* g = dlogits + static_cast<size_t>(row) * ldg;
  for (int i = threadIdx.x; i < n4; i += kCeSmemThreads) {
    const float4 e = e4[i];
    const int j = 4 * i;
    float p[4] = {e.x * inv, e.y * inv, e.z * inv, e.w * inv};
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = (p[k] - ((j + k) == tgt ? 1.0f : 0.0f)) * grad_scale;
    uint2 w;
    w.x = pack_bf16x2(p[0], (j + 1 < V) ? p[1] : 0.f);
    w.y = pack_bf16x2((j + 2 < V) ? p[2] : 0.f, (j + 3 < V) ? p[3] : 0.f);
    *reinterpret_cast<uint2*>(g + j) = w;
  }
  for (int j = 4 * n4 + threadIdx.x; j < ldg; j += kCeSmemThreads) g[j] = __float2bfloat16_rn(0.f);
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

// Fused head + cross-entropy, second half (the first is the kEpiLse epilogue
// of the logits GEMM, which leaves per 256-wide vocabulary tile k of a row its
// max m_k and sum s_k of exp(x - m_k), the fp32 target logit, and fp16
// e = exp(x - m_k) in the gradient buffer). One CTA per row:
//   LSE  = M + log(sum_k s_k exp(m_k - M)),  M = max_k m_k  (fixed trees)
//   loss = LSE - x[target]
//   grad = (e * exp(m_k - LSE) - onehot) * grad_scale, rounded once to bf16 and
//          written over e in place; columns V .. ld are zeroed.
// The fp32 logits never exist in memory.
constexpr int kFinThreads = 256;
constexpr int kFinMaxTiles = 1024;  // vocabularies up to 256K

__device__ __forceinline__ float block_reduce_fin(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < kFinThreads / 32 ? red[l] : (is_max ? -INFINITY : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, u) : v + u;
    }
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

__global__ void __launch_bounds__(kFinThreads)
    ce_lse_finalize_kernel(const float2* __restrict__ part, int nt, int ld_part,
                           const float* __restrict__ tgt_logit, const int64_t* __restrict__ targets,
                           int V, uint16_t* __restrict__ buf, int ld, float grad_scale,
                           float* __restrict__ loss_rows, int* status) {
  __shared__ float fac[kFinMaxTiles];
  __shared__ float red[33];
  const int row = blockIdx.x;
  const float2* pr = part + static_cast<size_t>(row) * ld_part;
  float m = -INFINITY;
  for (int k = threadIdx.x; k < nt; k += kFinThreads) m = fmaxf(m, pr[k].x);
  const float M = block_reduce_fin(m, red, true);
  float s = 0.f;
  for (int k = threadIdx.x; k < nt; k += kFinThreads) {
    const float2 p = pr[k];
    s += p.y * expf(p.x - M);
  }
  const float S = block_reduce_fin(s, red, false);
  const float lse = M + logf(S);
  const int64_t tgt = targets[row];
  if (threadIdx.x == 0) {
    const bool tgt_ok = tgt >= 0 && tgt < V;
    if (!tgt_ok) record_check(status, kStatusBadArgument, kSiteCeTarget, row, tgt);
    loss_rows[row] = tgt_ok ? lse - tgt_logit[row] : __int_as_float(0x7fc00000);
  }
  for (int k = threadIdx.x; k < nt; k += kFinThreads) fac[k] = expf(pr[k].x - lse);
  __syncthreads();
  uint16_t* g = buf + static_cast<size_t>(row) * ld;
  // 8 columns (16 bytes) per thread and iteration; ld is a multiple of 8 and
  // a 256-wide tile holds whole groups of 8.
  for (int j = threadIdx.x * 8; j < ld; j += kFinThreads * 8) {
    uint4 w = *reinterpret_cast<const uint4*>(g + j);
    uint32_t u[4] = {w.x, w.y, w.z, w.w};
    const float f = j < V ? fac[j >> 8] : 0.f;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const __half2 e = *reinterpret_cast<const __half2*>(&u[h]);
      const float2 ef = __half22float2(e);
      const int c0 = j + 2 * h;
      float d0 = 0.f, d1 = 0.f;
      if (c0 < V) d0 = (ef.x * f - (c0 == tgt ? 1.0f : 0.0f)) * grad_scale;
      if (c0 + 1 < V) d1 = (ef.y * f - (c0 + 1 == tgt ? 1.0f : 0.0f)) * grad_scale;
      u[h] = pack_bf16x2(d0, d1);
    }
    *reinterpret_cast<uint4*>(g + j) = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

}  // namespace

int ce_lse_finalize(const float* part, int nt, int ld_part, const float* tgt_logit,
                    const int64_t* targets, int T, int V, void* buf, int ld, float grad_scale,
                    float* loss_rows, int* status, cudaStream_t stream) {
  if (T <= 0 || V <= 0 || nt != (V + 255) / 256 || nt > kFinMaxTiles || ld_part < nt ||
      ld < V || ld % 8 || (reinterpret_cast<uintptr_t>(buf) & 15))
    return 1;
  ce_lse_finalize_kernel<<<T, kFinThreads, 0, stream>>>(
      reinterpret_cast<const float2*>(part), nt, ld_part, tgt_logit, targets, V,
      reinterpret_cast<uint16_t*>(buf), ld, grad_scale, loss_rows, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int cross_entropy(const CeArgs& a, cudaStream_t stream) {
  if (a.T <= 0 || a.V <= 0 || a.ldl < a.V || (a.dlogits && a.ldg < a.V)) return 1;
  // the shared-memory path copies ceil(V / 4) float4 per row: in bounds when
  // the row pitch covers them; the gradient rows take 8-byte stores
  const int n4 = (a.V + 3) / 4;
  const int row_bytes = n4 * 16;
  const bool smem_ok = row_bytes <= kCeSmemMaxBytes && a.ldl >= 4 * n4 && (a.ldl % 4) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0 &&
                       (a.dlogits == nullptr ||
                        (a.ldg >= 4 * n4 && (a.ldg % 4) == 0 &&
                         (reinterpret_cast<uintptr_t>(a.dlogits) & 7) == 0));
  if (smem_ok) {
    const int smem = row_bytes + 16;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
      if (cudaFuncSetAttribute(ce_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kCeSmemMaxBytes + 16) != cudaSuccess)
        return 2;
      attr[dev & 63] = true;
    }
    ce_smem_kernel<<<a.T, kCeSmemThreads, smem, stream>>>(a.logits, a.ldl, a.targets, a.V,
                                                          a.loss_rows, a.dlogits, a.ldg,
                                                          a.grad_scale, row_bytes, a.status);
  } else {
    ce_kernel<<<a.T, kCeThreads, 0, stream>>>(a.logits, a.ldl, a.targets, a.V, a.loss_rows,
                                              a.dlogits, a.ldg, a.grad_scale, a.status);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int mean_reduce(const float* x, int n, float* out, cudaStream_t stream) {
  if (n <= 0) return 1;
  mean_kernel<<<1, 1024, 0, stream>>>(x, n, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
