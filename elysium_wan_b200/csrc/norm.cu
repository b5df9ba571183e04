// LayerNorm forward / backward for sm_100a (reference op: nn.LayerNorm in
// src/wantrain/model/gpt.py:346-389,402-415, fp32 statistics under autocast).
//
// Forward: one CTA of 128 threads per row; the row is held in registers as
// fp32 (8 contiguous elements per thread per 1024-column slice), mean and
// variance are two-pass over the registers with a fixed reduction tree, so the
// result is deterministic. The input is any boundary format: bf16, fp16, or
// fp8 (e4m3 / e5m2) with one power-of-two scale per 128 columns; the
// conversion is the prologue of this kernel (the next stage's first op after a
// stage cut).
//
// Backward: dx with one warp per row (warp-shuffle row sums, no block
// barrier); dgamma/dbeta as per-chunk column partials (each thread owns 8
// columns over the chunk's rows, summed in row order) that a third kernel
// folds in chunk order into the fp32 gradients. No atomics anywhere.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

constexpr int kLnThreads = 128;
constexpr int kLnMaxSlices = 8;  // d <= 8192 (S = ceil(d / 1024) slices per thread)

__device__ __forceinline__ float block_sum_128(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

// Load 8 contiguous input elements of a boundary format (bf16, fp16, or
// e4m3 / e5m2 with a 1x128 block scale) as fp32.
__device__ __forceinline__ void load8(const void* x, const float* xs, int fmt, int ld, int lds,
                                      int row, int col, float* v) {
  if (fmt_q8(fmt)) {
    const uint8_t* p = reinterpret_cast<const uint8_t*>(x) + static_cast<size_t>(row) * ld + col;
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float s = xs[static_cast<size_t>(row) * lds + (col >> 7)];
    unpack8_fmt(make_uint4(raw.x, raw.y, 0u, 0u), fmt, s, v);
  } else {
    const uint8_t* p = reinterpret_cast<const uint8_t*>(x) + (static_cast<size_t>(row) * ld + col) * 2;
    unpack8_fmt(*reinterpret_cast<const uint4*>(p), fmt, 1.f, v);
  }
}

// 8 consecutive fp32 parameters (gamma / beta) as two 16-byte loads.
__device__ __forceinline__ void load8_f32(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float* v) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]);
  w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]);
  w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = w;
}

template <int S, bool RMS>
__global__ void __launch_bounds__(kLnThreads)
    layernorm_fwd_kernel(const void* __restrict__ x, const float* __restrict__ xs, int x_fmt,
                         int ldx, int ldxs, const float* __restrict__ gamma,
                         const float* __restrict__ beta, __nv_bfloat16* __restrict__ y, int ldy,
                         float* __restrict__ mean_out, float* __restrict__ rstd_out, int d,
                         float eps) {
  __shared__ float red[4];
  const int row = blockIdx.x;
  float v[S][8];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < S; ++j) {
    const int col = j * 1024 + threadIdx.x * 8;
    if (col < d) {
      load8(x, xs, x_fmt, ldx, ldxs, row, col, v[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[j][i];
    }
  }
  // RMSNorm: no centring (mean 0), no shift.
  const float mean = RMS ? 0.f : block_sum_128(s, red) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < S; ++j) {
    const int col = j * 1024 + threadIdx.x * 8;
    if (col < d) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float c = v[j][i] - mean;
        q += c * c;
      }
    }
  }
  const float var = block_sum_128(q, red) / static_cast<float>(d);
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < S; ++j) {
    const int col = j * 1024 + threadIdx.x * 8;
    if (col < d) {
      float o[8], gm[8], bt[8];
      load8_f32(gamma + col, gm);
      if (!RMS) load8_f32(beta + col, bt);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * rstd * gm[i] + (RMS ? 0.f : bt[i]);
      store8_bf16(y + static_cast<size_t>(row) * ldy + col, o);
    }
  }
  if (threadIdx.x == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)) (+ dres), g = dy * gamma.
// RMSNorm (RMS = true): mean = 0 and no centring of g, dx = rstd * (g - xhat * mean(g * xhat)).
//
// Two warps per row (four rows per CTA of eight warps): thread t of the row's
// 64 owns columns 512 j + 8 t (16-byte loads). Its share of x and dy is loaded
// once into registers (raw 16-byte words, so the whole row is in flight at
// once); the two row sums are per-thread sums in column order, a fixed warp
// butterfly, then the two warps' sums added in warp order through shared
// memory; dx is computed from the registers. NS = the most 512-column slices a
// row may have (d <= 512 NS).
constexpr int kLnBwdWarps = 8;

__device__ __forceinline__ void unpack8(const uint4& w, const float* xs_row, int fmt, int col,
                                        float* v) {
  unpack8_fmt(w, fmt, fmt_q8(fmt) ? xs_row[col >> 7] : 1.f, v);
}

template <int NS, bool RMS>
__global__ void __launch_bounds__(kLnBwdWarps * 32)
    layernorm_bwd_dx_kernel(const __nv_bfloat16* __restrict__ dy, int lddy, const void* __restrict__ x,
                            const float* __restrict__ xs, int x_fmt, int ldx, int ldxs,
                            const float* __restrict__ mean, const float* __restrict__ rstd,
                            const float* __restrict__ gamma, const __nv_bfloat16* __restrict__ dres,
                            int lddres, __nv_bfloat16* __restrict__ dx, int lddx, int rows, int d) {
  __shared__ float red[kLnBwdWarps][2];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int half = warp & 1;
  const int t = half * 32 + lane;  // thread index within the row's 64
  const int row = blockIdx.x * (kLnBwdWarps / 2) + (warp >> 1);
  const bool live = row < rows;
  uint4 xw[NS], dw[NS];
  const uint8_t* xrow = reinterpret_cast<const uint8_t*>(x) +
                        static_cast<size_t>(live ? row : 0) * ldx * fmt_bytes(x_fmt);
  const __nv_bfloat16* dyrow = dy + static_cast<size_t>(live ? row : 0) * lddy;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int col = j * 512 + t * 8;
    if (live && col < d) {
      if (fmt_q8(x_fmt)) {
        const uint2 r = __ldg(reinterpret_cast<const uint2*>(xrow + col));
        xw[j] = make_uint4(r.x, r.y, 0u, 0u);
      } else {
        xw[j] = __ldg(reinterpret_cast<const uint4*>(xrow + 2 * col));
      }
      dw[j] = __ldg(reinterpret_cast<const uint4*>(dyrow + col));
    }
  }
  const float* xs_row = (fmt_q8(x_fmt) && live) ? xs + static_cast<size_t>(row) * ldxs : nullptr;
  const float mu = (RMS || !live) ? 0.f : mean[row];
  const float rs = live ? rstd[row] : 0.f;
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int col = j * 512 + t * 8;
    if (live && col < d) {
      float xv[8], dv[8], gm[8];
      unpack8(xw[j], xs_row, x_fmt, col, xv);
      unpack8(dw[j], nullptr, 0, col, dv);
      load8_f32(gamma + col, gm);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g = dv[i] * gm[i];
        s1 += g;
        s2 += g * ((xv[i] - mu) * rs);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  if (lane == 0) {
    red[warp][0] = s1;
    red[warp][1] = s2;
  }
  __syncthreads();
  if (!live) return;
  const int w0 = warp & ~1;
  s1 = red[w0][0] + red[w0 + 1][0];
  s2 = red[w0][1] + red[w0 + 1][1];
  const float m1 = RMS ? 0.f : s1 / static_cast<float>(d);
  const float m2 = s2 / static_cast<float>(d);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int col = j * 512 + t * 8;
    if (col < d) {
      float xv[8], dv[8], gm[8], o[8];
      unpack8(xw[j], xs_row, x_fmt, col, xv);
      unpack8(dw[j], nullptr, 0, col, dv);
      load8_f32(gamma + col, gm);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = (xv[i] - mu) * rs;
        o[i] = rs * (dv[i] * gm[i] - m1 - xh * m2);
      }
      if (dres != nullptr) {
        float rv[8];
        load8(dres, nullptr, 0, lddres, 0, row, col, rv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rv[i];
      }
      store8_bf16(dx + static_cast<size_t>(row) * lddx + col, o);
    }
  }
}

// dgamma / dbeta partial sums of one chunk of rows: thread t of CTA (bx, chunk)
// owns columns 1024 bx + 8 t and sums dy * xhat and dy over the chunk's rows
// in row order; the chunks are folded in chunk order by fold_partials_kernel.
template <bool RMS>
__global__ void __launch_bounds__(kLnThreads)
    layernorm_bwd_param_kernel(const __nv_bfloat16* __restrict__ dy, int lddy,
                               const void* __restrict__ x, const float* __restrict__ xs, int x_fmt,
                               int ldx, int ldxs, const float* __restrict__ mean,
                               const float* __restrict__ rstd, float* __restrict__ part_g,
                               float* __restrict__ part_b, int rows, int d, int rows_per_chunk) {
  const int col = blockIdx.x * 1024 + threadIdx.x * 8;
  const int chunk = blockIdx.y;
  if (col >= d) return;
  const int r0 = chunk * rows_per_chunk;
  const int r1 = min(rows, r0 + rows_per_chunk);
  float pg[8], pb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    pg[i] = 0.f;
    pb[i] = 0.f;
  }
  // eight rows' raw 16-byte loads in flight per thread, then their sums in
  // row order
  const size_t xb = fmt_bytes(x_fmt);
  for (int rb = r0; rb < r1; rb += 8) {
    uint4 xw[8], dw[8];
    float mu[8], rs[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = rb + k;
      if (row < r1) {
        const uint8_t* xp = reinterpret_cast<const uint8_t*>(x) + (static_cast<size_t>(row) * ldx + col) * xb;
        if (fmt_q8(x_fmt)) {
          const uint2 r = __ldg(reinterpret_cast<const uint2*>(xp));
          xw[k] = make_uint4(r.x, r.y, 0u, 0u);
        } else {
          xw[k] = __ldg(reinterpret_cast<const uint4*>(xp));
        }
        dw[k] = __ldg(reinterpret_cast<const uint4*>(dy + static_cast<size_t>(row) * lddy + col));
        mu[k] = RMS ? 0.f : __ldg(mean + row);
        rs[k] = __ldg(rstd + row);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = rb + k;
      if (row < r1) {
        float xv[8], dv[8];
        unpack8(xw[k], fmt_q8(x_fmt) ? xs + static_cast<size_t>(row) * ldxs : nullptr, x_fmt, col, xv);
        unpack8(dw[k], nullptr, 0, col, dv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pg[i] += dv[i] * ((xv[i] - mu[k]) * rs[k]);
          pb[i] += dv[i];
        }
      }
    }
  }
  float4* g4 = reinterpret_cast<float4*>(part_g + static_cast<size_t>(chunk) * d + col);
  g4[0] = make_float4(pg[0], pg[1], pg[2], pg[3]);
  g4[1] = make_float4(pg[4], pg[5], pg[6], pg[7]);
  if (!RMS) {
    float4* b4 = reinterpret_cast<float4*>(part_b + static_cast<size_t>(chunk) * d + col);
    b4[0] = make_float4(pb[0], pb[1], pb[2], pb[3]);
    b4[1] = make_float4(pb[4], pb[5], pb[6], pb[7]);
  }
}

// grad[c] (+)= sum over chunks of part[chunk][c] in a fixed tree: a CTA owns
// 32 columns; warp w sums chunks w, w + 8, w + 16, ... in order (lane = column,
// 128-byte rows), then the eight warp sums are added in warp order. 8 warps x
// d / 32 CTAs instead of one serial chain per column over all chunks.
constexpr int kFoldWarps = 8;
__global__ void __launch_bounds__(kFoldWarps * 32)
    fold_partials_kernel(const float* __restrict__ part, int chunks, int d,
                         float* __restrict__ grad, int accumulate) {
  __shared__ float red[kFoldWarps][32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int c = blockIdx.x * 32 + l;
  float s = 0.f;
  if (c < d)
    for (int k = w; k < chunks; k += kFoldWarps) s += part[static_cast<size_t>(k) * d + c];
  red[w][l] = s;
  __syncthreads();
  if (w == 0 && c < d) {
    float t = red[0][l];
#pragma unroll
    for (int i = 1; i < kFoldWarps; ++i) t += red[i][l];
    grad[c] = accumulate ? grad[c] + t : t;
  }
}

}  // namespace

int layernorm_fwd(const LnArgs& a, cudaStream_t stream) {
  if (a.d % 8 || a.d > 1024 * kLnMaxSlices || (fmt_q8(a.x_fmt) && a.d % 128) ||
      a.x_fmt < kFmtBf16 || a.x_fmt > kFmtF16) return 1;
  const int S = (a.d + 1023) / 1024;
#define EWB_LN_FWD(SS)                                                                       \
  (a.rms ? layernorm_fwd_kernel<SS, true><<<a.rows, kLnThreads, 0, stream>>>(                 \
               a.x, a.x_scale, a.x_fmt, a.ldx, a.ldxs, a.gamma, a.beta, a.y, a.ldy, a.mean,   \
               a.rstd, a.d, a.eps)                                                            \
         : layernorm_fwd_kernel<SS, false><<<a.rows, kLnThreads, 0, stream>>>(                \
               a.x, a.x_scale, a.x_fmt, a.ldx, a.ldxs, a.gamma, a.beta, a.y, a.ldy, a.mean,   \
               a.rstd, a.d, a.eps))
  switch (S) {
    case 1: EWB_LN_FWD(1); break;
    case 2: EWB_LN_FWD(2); break;
    case 3: EWB_LN_FWD(3); break;
    case 4: EWB_LN_FWD(4); break;
    case 5: EWB_LN_FWD(5); break;
    case 6: EWB_LN_FWD(6); break;
    case 7: EWB_LN_FWD(7); break;
    default: EWB_LN_FWD(8); break;
  }
#undef EWB_LN_FWD
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int layernorm_bwd_rows_per_chunk(int rows) {
  // Chunks of 16 rows (at most 256 chunks) for the dgamma / dbeta partials:
  // d / 1024 x chunks CTAs of 128 threads, two batches of eight rows each.
  int rpc = rows > 256 * 16 ? (rows + 255) / 256 : 16;
  return rpc;
}

int layernorm_bwd(const LnBwdArgs& a, cudaStream_t stream) {
  if (a.d % 8 || a.d > 1024 * kLnMaxSlices || (fmt_q8(a.x_fmt) && a.d % 128) ||
      a.x_fmt < kFmtBf16 || a.x_fmt > kFmtF16) return 1;
  const int rpc = a.rows_per_chunk;
  if (rpc < 1) return 1;
  const int chunks = (a.rows + rpc - 1) / rpc;
  const int dx_grid = (a.rows + kLnBwdWarps / 2 - 1) / (kLnBwdWarps / 2);
  const dim3 pgrid((a.d + 1023) / 1024, chunks);
  const int ns = (a.d + 511) / 512;
#define EWB_LN_DX(NSV, R)                                                                     \
  layernorm_bwd_dx_kernel<NSV, R><<<dx_grid, kLnBwdWarps * 32, 0, stream>>>(                   \
      a.dy, a.lddy, a.x, a.x_scale, a.x_fmt, a.ldx, a.ldxs, a.mean, a.rstd, a.gamma, a.dres,     \
      a.lddres, a.dx, a.lddx, a.rows, a.d)
#define EWB_LN_DX_NS(R)                     \
  if (ns <= 2) EWB_LN_DX(2, R);             \
  else if (ns <= 4) EWB_LN_DX(4, R);        \
  else if (ns <= 6) EWB_LN_DX(6, R);        \
  else if (ns <= 8) EWB_LN_DX(8, R);        \
  else if (ns <= 10) EWB_LN_DX(10, R);      \
  else if (ns <= 12) EWB_LN_DX(12, R);      \
  else EWB_LN_DX(16, R)
  if (a.rms) {
    EWB_LN_DX_NS(true);
    layernorm_bwd_param_kernel<true><<<pgrid, kLnThreads, 0, stream>>>(
        a.dy, a.lddy, a.x, a.x_scale, a.x_fmt, a.ldx, a.ldxs, a.mean, a.rstd, a.part_g, a.part_b,
        a.rows, a.d, rpc);
  } else {
    EWB_LN_DX_NS(false);
    layernorm_bwd_param_kernel<false><<<pgrid, kLnThreads, 0, stream>>>(
        a.dy, a.lddy, a.x, a.x_scale, a.x_fmt, a.ldx, a.ldxs, a.mean, a.rstd, a.part_g, a.part_b,
        a.rows, a.d, rpc);
  }
#undef EWB_LN_DX_NS
#undef EWB_LN_DX
  if (cudaGetLastError() != cudaSuccess) return 2;
  const int fb = (a.d + 31) / 32;
  fold_partials_kernel<<<fb, kFoldWarps * 32, 0, stream>>>(a.part_g, chunks, a.d, a.dgamma,
                                                           a.accumulate);
  if (!a.rms)
    fold_partials_kernel<<<fb, kFoldWarps * 32, 0, stream>>>(a.part_b, chunks, a.d, a.dbeta,
                                                             a.accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb

// ---------------------------------------------------------------- allocation-free entry point
// ewb_layernorm_bwd_noalloc (declared and documented in noalloc.h): the
// partial-sum scratch lives in this file-scope device array instead of a
// caller-allocated buffer. Host code must not use the array's name as a
// device address; the address comes from cudaGetSymbolAddress, per device.
#include <mutex>

#include "noalloc.h"

static __device__ __align__(256) float
    g_ln_bwd_noalloc_scratch[2 * EWB_NOALLOC_LN_MAX_CHUNKS * EWB_NOALLOC_LN_MAX_D];

namespace {

std::mutex g_noalloc_mu;
float* g_noalloc_addr[64] = {nullptr};

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
float* noalloc_scratch(int* err) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = EWB_NOALLOC_ERR_SETUP;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_ln_bwd_noalloc_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      *err = EWB_NOALLOC_ERR_SETUP;
      return nullptr;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  return g_noalloc_addr[dev];
}

}  // namespace

extern "C" int ewb_layernorm_bwd_noalloc(const void* dy, int lddy, const void* x,
                                         const float* x_scale, int x_fmt, int ldx, int ldxs,
                                         const float* mean, const float* rstd, const float* gamma,
                                         const void* dres, int lddres, void* dx, int lddx,
                                         float* dgamma, float* dbeta, int accumulate, int rows,
                                         int d, void* stream) {
  if (dy == nullptr || x == nullptr || mean == nullptr || rstd == nullptr || gamma == nullptr ||
      dx == nullptr || dgamma == nullptr || dbeta == nullptr || rows <= 0 || d <= 0 || d % 8 ||
      x_fmt < ewb::kFmtBf16 || x_fmt > ewb::kFmtF16 ||
      (ewb::fmt_q8(x_fmt) && (x_scale == nullptr || d % 128)))
    return EWB_NOALLOC_ERR_ARGUMENT;
  if (d > EWB_NOALLOC_LN_MAX_D) return EWB_NOALLOC_ERR_TOO_LARGE;
  int err = EWB_NOALLOC_OK;
  float* scratch = noalloc_scratch(&err);
  if (scratch == nullptr) return err;
  ewb::LnBwdArgs a{};
  a.dy = static_cast<const __nv_bfloat16*>(dy);
  a.lddy = lddy;
  a.x = x;
  a.x_scale = x_scale;
  a.x_fmt = x_fmt;
  a.ldx = ldx;
  a.ldxs = ldxs;
  a.mean = mean;
  a.rstd = rstd;
  a.gamma = gamma;
  a.dres = static_cast<const __nv_bfloat16*>(dres);
  a.lddres = lddres;
  a.dx = static_cast<__nv_bfloat16*>(dx);
  a.lddx = lddx;
  a.part_g = scratch;
  a.part_b = scratch + EWB_NOALLOC_LN_MAX_CHUNKS * EWB_NOALLOC_LN_MAX_D;
  a.dgamma = dgamma;
  a.dbeta = dbeta;
  a.accumulate = accumulate ? 1 : 0;
  a.rows = rows;
  a.d = d;
  a.rows_per_chunk = (rows + EWB_NOALLOC_LN_MAX_CHUNKS - 1) / EWB_NOALLOC_LN_MAX_CHUNKS;
  const int rc = ewb::layernorm_bwd(a, static_cast<cudaStream_t>(stream));
  if (rc == 0) return EWB_NOALLOC_OK;
  return rc == 1 ? EWB_NOALLOC_ERR_ARGUMENT : EWB_NOALLOC_ERR_LAUNCH;
}
