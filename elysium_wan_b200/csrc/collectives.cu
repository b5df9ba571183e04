// ZeRO-1 collectives over NVLink peer memory (the parts that are not fused into
// the W GEMM epilogue, see kEpiAccF32Peer in gemm.cu).
//
// Layout: a wide stage's flat parameter buffer is cut into contiguous owner
// shards [lo[k], lo[k+1]). Every replica keeps, in symmetric (peer-mapped)
// memory: the full fp32 master, the full bf16 working copy and, as owner of
// shard k, `world` slots of that shard's length (slot r receives replica r's
// partial gradient).
//
//   push_partials   replica r copies the flat ranges the fused epilogue does
//                   not cover (LayerNorm, bias, embedding gradients) from its
//                   local partial into the owners' slots.
//   fold_slots      owner k: g = ((s_0 + s_1) + s_2) + ... in rank order, the
//                   declared fold tree (deterministic).
//   adamw_push      owner k: AdamW over its shard, writing the new fp32 and
//                   bf16 values into every replica's master / working copy
//                   (the all-gather, fused into the optimizer's stores).
// Synchronisation between these phases is a one-element NCCL all-reduce on
// the stage group issued by the host; no kernel here waits on a peer.
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace ewb {
namespace {

struct Owners {
  float* slots[kMaxPeers];
  long long lo[kMaxPeers + 1];
  long long stride;
  int rank;
  int world;
};

__global__ void push_partials_kernel(const float* __restrict__ partial, const long long* __restrict__ ranges,
                                     int nranges, Owners o) {
  // ranges: [start, end) pairs of flat indices
  for (int r = 0; r < nranges; ++r) {
    const long long a = ranges[2 * r], b = ranges[2 * r + 1];
    for (long long f = a + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; f < b;
         f += static_cast<long long>(gridDim.x) * blockDim.x) {
      int k = 0;
      while (k + 1 < o.world && f >= o.lo[k + 1]) ++k;
      o.slots[k][static_cast<long long>(o.rank) * o.stride + (f - o.lo[k])] = partial[f];
    }
  }
}

__global__ void fold_slots_kernel(const float* __restrict__ slots, long long stride, int world,
                                  long long n, float* __restrict__ out) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float acc = slots[i];
    for (int r = 1; r < world; ++r) acc += slots[static_cast<long long>(r) * stride + i];
    out[i] = acc;
  }
}

struct Replicas {
  float* master[kMaxPeers];
  __nv_bfloat16* work[kMaxPeers];
  int world;
};

// Same update as adamw_kernel (optim.cu), written to every replica.
__global__ void adamw_push_kernel(const float* __restrict__ p_in, float* __restrict__ m,
                                  float* __restrict__ v, const float* __restrict__ g, long long lo,
                                  long long n, Replicas rep, float lr, float b1, float b2, float eps,
                                  float wd, float bc1, float sqrt_bc2) {
  const float step = lr / bc1;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float gi = g[i];
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    float pi = p_in[lo + i];
    if (wd != 0.0f) pi = pi * (1.0f - lr * wd);
    const float denom = sqrtf(vi) / sqrt_bc2 + eps;
    pi = pi - step * (mi / denom);
    m[i] = mi;
    v[i] = vi;
    const __nv_bfloat16 pb = __float2bfloat16_rn(pi);
    for (int r = 0; r < rep.world; ++r) {
      rep.master[r][lo + i] = pi;
      rep.work[r][lo + i] = pb;
    }
  }
}

int grid_for(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148 * 8) b = 148 * 8;
  return static_cast<int>(b < 1 ? 1 : b);
}

}  // namespace

int zero1_push_partials(const float* partial, const long long* ranges_dev, int nranges,
                        float* const* slots, const long long* lo, long long stride, int rank,
                        int world, long long total, cudaStream_t stream) {
  if (world < 1 || world > kMaxPeers) return 1;
  Owners o{};
  for (int k = 0; k < world; ++k) o.slots[k] = slots[k];
  for (int k = 0; k <= world; ++k) o.lo[k] = lo[k];
  o.stride = stride;
  o.rank = rank;
  o.world = world;
  push_partials_kernel<<<grid_for(total), 256, 0, stream>>>(partial, ranges_dev, nranges, o);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int zero1_fold_slots(const float* slots, long long stride, int world, long long n, float* out,
                     cudaStream_t stream) {
  if (n <= 0) return 0;
  fold_slots_kernel<<<grid_for(n), 256, 0, stream>>>(slots, stride, world, n, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int zero1_adamw_push(const float* master, float* m, float* v, const float* g, long long lo,
                     long long n, float* const* masters, __nv_bfloat16* const* works, int world,
                     float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                     cudaStream_t stream) {
  if (n <= 0) return 0;
  if (world < 1 || world > kMaxPeers) return 1;
  Replicas rep{};
  for (int r = 0; r < world; ++r) {
    rep.master[r] = masters[r];
    rep.work[r] = works[r];
  }
  rep.world = world;
  adamw_push_kernel<<<grid_for(n), 256, 0, stream>>>(master, m, v, g, lo, n, rep, lr, b1, b2, eps,
                                                     wd, bc1, sqrtf(bc2));
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
