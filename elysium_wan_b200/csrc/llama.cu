// Elementwise kernels of the Llama-family block for sm_100a: rotary position
// embedding on the fused qkv rows and the SwiGLU gate (forward and backward).
//
// Reference ops: apply_rope / rope_cache (adjacent-pair rotation, theta^(-2i/hd)
// frequencies) and SwiGLUMLP (down(silu(gate(x)) * up(x))) in
// src/wantrain/model/arch.py:49-92. Both are memory-bound passes: 16-byte
// vector loads and stores, fp32 math, one rounding to bf16 per output.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

// One thread rotates 8 consecutive columns (4 adjacent pairs) of one row.
// Columns [0, ncols) of each row hold the q heads then the k heads, hd wide;
// pair (2i, 2i + 1) of a head at position p turns by p * inv_freq[i]. The
// tables are [S][hd / 2] fp32 (cos, sin of that angle). inverse = rotate by
// minus the angle (the backward of a rotation is its transpose).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int ld, int rows, int S, int ncols,
                            int hd, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int inverse) {
  const int per_row = ncols / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(rows) * per_row) return;
  const int row = static_cast<int>(idx / per_row);
  const int col = static_cast<int>(idx % per_row) * 8;
  const int pos = row % S;
  const int i0 = (col % hd) / 2;  // first pair index within the head
  __nv_bfloat16* p = x + static_cast<size_t>(row) * ld + col;
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  __nv_bfloat16* b = reinterpret_cast<__nv_bfloat16*>(&raw);
  const float* c = cos_t + static_cast<size_t>(pos) * (hd / 2) + i0;
  const float* s = sin_t + static_cast<size_t>(pos) * (hd / 2) + i0;
  const float sg = inverse ? -1.f : 1.f;
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float x1 = __bfloat162float(b[2 * k]), x2 = __bfloat162float(b[2 * k + 1]);
    const float cc = c[k], ss = sg * s[k];
    o[k] = pack_bf16x2(x1 * cc - x2 * ss, x1 * ss + x2 * cc);
  }
  *reinterpret_cast<uint4*>(p) = out;
}

__device__ __forceinline__ float sigmoidf_(float g) { return 1.0f / (1.0f + expf(-g)); }

// h[t][j] = silu(gu[t][j]) * gu[t][f + j]; 8 columns per thread.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, int ldgu,
                                  __nv_bfloat16* __restrict__ h, int ldh, int rows, int f) {
  const int per_row = f / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(rows) * per_row) return;
  const int row = static_cast<int>(idx / per_row);
  const int col = static_cast<int>(idx % per_row) * 8;
  const __nv_bfloat16* gp = gu + static_cast<size_t>(row) * ldgu + col;
  uint4 graw = *reinterpret_cast<const uint4*>(gp);
  uint4 uraw = *reinterpret_cast<const uint4*>(gp + f);
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&graw);
  const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uraw);
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float r[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float gv = __bfloat162float(g[2 * k + e]);
      r[e] = gv * sigmoidf_(gv) * __bfloat162float(u[2 * k + e]);
    }
    o[k] = pack_bf16x2(r[0], r[1]);
  }
  *reinterpret_cast<uint4*>(h + static_cast<size_t>(row) * ldh + col) = out;
}

// dgu[t][j] = dh * u * silu'(g), dgu[t][f + j] = dh * silu(g), with
// silu'(g) = s (1 + g (1 - s)), s = sigmoid(g).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, int lddh,
                                  const __nv_bfloat16* __restrict__ gu, int ldgu,
                                  __nv_bfloat16* __restrict__ dgu, int lddgu, int rows, int f) {
  const int per_row = f / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(rows) * per_row) return;
  const int row = static_cast<int>(idx / per_row);
  const int col = static_cast<int>(idx % per_row) * 8;
  const __nv_bfloat16* gp = gu + static_cast<size_t>(row) * ldgu + col;
  uint4 graw = *reinterpret_cast<const uint4*>(gp);
  uint4 uraw = *reinterpret_cast<const uint4*>(gp + f);
  uint4 draw = *reinterpret_cast<const uint4*>(dh + static_cast<size_t>(row) * lddh + col);
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&graw);
  const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uraw);
  const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(&draw);
  uint4 og, ou;
  uint32_t* pg = reinterpret_cast<uint32_t*>(&og);
  uint32_t* pu = reinterpret_cast<uint32_t*>(&ou);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float rg[2], ru[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float gv = __bfloat162float(g[2 * k + e]);
      const float uv = __bfloat162float(u[2 * k + e]);
      const float dv = __bfloat162float(d[2 * k + e]);
      const float s = sigmoidf_(gv);
      rg[e] = dv * uv * s * (1.0f + gv * (1.0f - s));
      ru[e] = dv * gv * s;
    }
    pg[k] = pack_bf16x2(rg[0], rg[1]);
    pu[k] = pack_bf16x2(ru[0], ru[1]);
  }
  __nv_bfloat16* op = dgu + static_cast<size_t>(row) * lddgu + col;
  *reinterpret_cast<uint4*>(op) = og;
  *reinterpret_cast<uint4*>(op + f) = ou;
}

inline int grid_for(long long n, int tb) { return static_cast<int>((n + tb - 1) / tb); }

}  // namespace

int rope_apply(const RopeArgs& a, cudaStream_t stream) {
  if (a.ncols % 8 || a.hd % 8 || a.ncols % a.hd || a.ld % 8 || a.S <= 0) return 1;
  const long long n = static_cast<long long>(a.rows) * (a.ncols / 8);
  if (n == 0) return 0;
  rope_kernel<<<grid_for(n, 256), 256, 0, stream>>>(a.x, a.ld, a.rows, a.S, a.ncols, a.hd, a.cos,
                                                    a.sin, a.inverse);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int swiglu_fwd(const SwigluArgs& a, cudaStream_t stream) {
  if (a.f % 8 || a.ldgu % 8 || a.ldh % 8) return 1;
  const long long n = static_cast<long long>(a.rows) * (a.f / 8);
  if (n == 0) return 0;
  swiglu_fwd_kernel<<<grid_for(n, 256), 256, 0, stream>>>(a.gu, a.ldgu, a.h, a.ldh, a.rows, a.f);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int swiglu_bwd(const SwigluBwdArgs& a, cudaStream_t stream) {
  if (a.f % 8 || a.ldgu % 8 || a.lddh % 8 || a.lddgu % 8) return 1;
  const long long n = static_cast<long long>(a.rows) * (a.f / 8);
  if (n == 0) return 0;
  swiglu_bwd_kernel<<<grid_for(n, 256), 256, 0, stream>>>(a.dh, a.lddh, a.gu, a.ldgu, a.dgu,
                                                          a.lddgu, a.rows, a.f);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
