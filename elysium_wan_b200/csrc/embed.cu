// Token + learned position embedding, forward and deterministic backward.
//
// Reference op: Embed (src/wantrain/model/gpt.py:320-338): x = wte[idx] +
// wpe[pos], cast to the compute dtype, then the boundary narrowing. Forward
// reads the fp32 master tables directly and writes the boundary format: bf16,
// fp16, or fp8 (e4m3 / e5m2) with 1x128 scales (the quantisation is this
// kernel's epilogue).
//
// Backward without atomics: one CTA ranks every position by (token, position),
// so equal tokens form runs in position order; a second kernel gives each run
// head one CTA that sums the run's rows in that order into the fp32 table
// gradient. Position gradients sum the batch rows in batch order.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

__global__ void __launch_bounds__(128)
    embed_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ wte,
                     const float* __restrict__ wpe, int S, int d, int V, void* __restrict__ out,
                     int fmt, float* __restrict__ out_scale, int* status) {
  const int t = blockIdx.x;
  int64_t tok = idx[t];
  const int pos = t % S;
  // A token id outside the table is reported (status record) and reads row 0
  // instead of memory outside the table.
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0) record_check(status, kStatusBadArgument, kSiteEmbedToken, t, tok);
    tok = 0;
  }
  const float* er = wte + static_cast<size_t>(tok) * d;
  const float* pr = wpe != nullptr ? wpe + static_cast<size_t>(pos) * d : nullptr;  // rope: none
  for (int c0 = 0; c0 < d; c0 += 1024) {
    const int c = c0 + threadIdx.x * 8;
    float v[8];
    const bool ok = c < d;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = ok ? er[c + i] + (pr != nullptr ? pr[c + i] : 0.f) : 0.f;
    if (fmt_q8(fmt)) {
      // 16 consecutive threads cover one 128-column block.
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float scale = q8_block_scale(amax, fmt);
      const float inv = 1.0f / scale;
      if (ok) {
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
          w[h] = q8x2(v[4 * h] * inv, v[4 * h + 1] * inv, fmt) |
                 (q8x2(v[4 * h + 2] * inv, v[4 * h + 3] * inv, fmt) << 16);
        *reinterpret_cast<uint2*>(static_cast<uint8_t*>(out) + static_cast<size_t>(t) * d + c) =
            make_uint2(w[0], w[1]);
        if ((threadIdx.x & 15) == 0) out_scale[static_cast<size_t>(t) * (d / 128) + c / 128] = scale;
      }
    } else if (ok) {
      uint4 w;
      if (fmt == kFmtF16) {
        w = make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]),
                       pack_f16x2(v[6], v[7]));
      } else {
        w = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                       pack_bf16x2(v[6], v[7]));
      }
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (static_cast<size_t>(t) * d + c) * 2) = w;
    }
  }
}

// order[rank(t)] = t with rank by (token, position); T <= 16384.
// Rank of position t under the order (token, position); each CTA stages all
// T ids in shared memory and ranks kRankPer positions (one per thread), so the
// O(T^2) comparisons spread over T / kRankPer CTAs.
constexpr int kRankPer = 128;
__global__ void __launch_bounds__(kRankPer) embed_rank_kernel(const int64_t* __restrict__ idx,
                                                              int T, int* __restrict__ order) {
  extern __shared__ int sidx[];
  for (int i = threadIdx.x; i < T; i += kRankPer) sidx[i] = static_cast<int>(idx[i]);
  __syncthreads();
  const int t = blockIdx.x * kRankPer + threadIdx.x;
  if (t >= T) return;
  const int v = sidx[t];
  int r = 0;
  for (int u = 0; u < T; ++u) {
    const int w = sidx[u];
    r += (w < v) || (w == v && u < t);
  }
  order[r] = t;
}

__global__ void __launch_bounds__(256)
    embed_wte_bwd_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ dx,
                         const int* __restrict__ order, int T, int d, int V, float* __restrict__ dwte,
                         int* status) {
  const int i = blockIdx.x;
  const int t0 = order[i];
  const int64_t tok = idx[t0];
  if (i > 0 && idx[order[i - 1]] == tok) return;  // not a run head
  if (tok < 0 || tok >= V) {  // reported, never written outside the table
    if (threadIdx.x == 0) record_check(status, kStatusBadArgument, kSiteEmbedToken, t0, tok);
    return;
  }
  int end = i + 1;
  while (end < T && idx[order[end]] == tok) ++end;
  float* g = dwte + static_cast<size_t>(tok) * d;
  if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(dwte) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(dx) & 7) == 0) {
    // 4 columns per thread per pass: 16-byte fp32 and 8-byte bf16 accesses,
    // the passes independent so their loads overlap
#pragma unroll 4
    for (int c = 4 * threadIdx.x; c < d; c += 1024) {
      float4 s = *reinterpret_cast<const float4*>(g + c);
      for (int k = i; k < end; ++k) {
        const uint2 u = *reinterpret_cast<const uint2*>(dx + static_cast<size_t>(order[k]) * d + c);
        s.x += __uint_as_float(u.x << 16);
        s.y += __uint_as_float(u.x & 0xffff0000u);
        s.z += __uint_as_float(u.y << 16);
        s.w += __uint_as_float(u.y & 0xffff0000u);
      }
      *reinterpret_cast<float4*>(g + c) = s;
    }
    return;
  }
  for (int c = threadIdx.x; c < d; c += 256) {
    float s = g[c];
    for (int k = i; k < end; ++k) s += __bfloat162float(dx[static_cast<size_t>(order[k]) * d + c]);
    g[c] = s;
  }
}

__global__ void __launch_bounds__(256)
    embed_wpe_bwd_kernel(const __nv_bfloat16* __restrict__ dx, int T, int S, int d,
                         float* __restrict__ dwpe) {
  const int s = blockIdx.x;
  const int nb = T / S;
  for (int c = threadIdx.x; c < d; c += 256) {
    float acc = dwpe[static_cast<size_t>(s) * d + c];
    for (int b = 0; b < nb; ++b) acc += __bfloat162float(dx[(static_cast<size_t>(b) * S + s) * d + c]);
    dwpe[static_cast<size_t>(s) * d + c] = acc;
  }
}

}  // namespace

int embed_fwd(const EmbedArgs& a, cudaStream_t stream) {
  if (a.d % 8 || a.V <= 0 || (fmt_q8(a.out_fmt) && (a.d % 128 || a.out_scale == nullptr)) || a.T % a.S ||
      a.out_fmt < kFmtBf16 || a.out_fmt > kFmtF16)
    return 1;
  embed_fwd_kernel<<<a.T, 128, 0, stream>>>(a.idx, a.wte, a.wpe, a.S, a.d, a.V, a.out, a.out_fmt,
                                            a.out_scale, a.status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int embed_bwd(const EmbedBwdArgs& a, cudaStream_t stream) {
  if (a.T > 16384 || a.T % a.S) return 1;
  embed_rank_kernel<<<(a.T + kRankPer - 1) / kRankPer, kRankPer, a.T * sizeof(int), stream>>>(
      a.idx, a.T, a.order);
  embed_wte_bwd_kernel<<<a.T, 256, 0, stream>>>(a.idx, a.dx, a.order, a.T, a.d, a.V, a.dwte,
                                                a.status);
  if (a.dwpe != nullptr) embed_wpe_bwd_kernel<<<a.S, 256, 0, stream>>>(a.dx, a.T, a.S, a.d, a.dwpe);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
