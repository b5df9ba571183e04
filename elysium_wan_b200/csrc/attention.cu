// Causal self-attention forward / backward, bf16 in, fp32 softmax statistics.
//
// Reference op: F.scaled_dot_product_attention(q, k, v, is_causal=True)
// (src/wantrain/model/gpt.py:374-386), or the naive softmax(QK^T/sqrt(hd))V.
//
// Layout: Q, K and V are read in place from the fused qkv projection output
// [T, 3d] (token-major, head h of Q at column h*hd, of K at d + h*hd, of V at
// 2d + h*hd); O is written as [T, d] with heads concatenated, so neither side
// needs a transpose kernel. The softmax statistic kept for the backward is the
// base-2 log-sum-exp of the scaled scores, lse2 = max + log2(sum 2^(x - max)),
// x = (q.k) * log2(e) / sqrt(hd).
//
// Tiles: 128 (or 64) query rows per CTA, one warp per 16 rows, keys in blocks
// of 64 double-buffered by cp.async, bf16 mma.sync m16n8k16 with fp32
// accumulation; exponentials on the hardware ex2 unit.
// Backward: dK/dV in one kernel (a CTA owns a key block and walks the query
// blocks), dQ in another (a CTA owns a query block and walks the key blocks).
// Every output element is produced by one thread in a fixed order: there are
// no atomics, so gradients are bitwise reproducible.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Copy a [ROWS][HD] bf16 tile (row stride ld elements in global) into shared
// memory with row stride HD + 8 (the padding makes ldmatrix conflict-free).
template <int HD, int ROWS = 64>
__device__ __forceinline__ void load_tile_async(__nv_bfloat16* s, const __nv_bfloat16* g, int ld) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int LD = HD + 8;
  for (int i = threadIdx.x; i < ROWS * CH; i += blockDim.x) {
    const int r = i / CH, c = i % CH;
    cp_async16(smem_u32(s + r * LD + c * 8), g + static_cast<size_t>(r) * ld + c * 8);
  }
}

// 2^x with the hardware approximation (ex2.approx.ftz.f32): the softmax's
// exponent; its error (2 ulp) is far below the bf16 rounding of P.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A-operand fragments (16 rows x HD) of rows [row0, row0+16) of a smem tile.
template <int HD>
__device__ __forceinline__ void load_a_frags(const __nv_bfloat16* s, int row0, uint32_t (*f)[4]) {
  constexpr int LD = HD + 8;
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk)
    ldsm_x4(smem_u32(s + (row0 + (l & 15)) * LD + kk * 16 + (l >> 4) * 8), f[kk]);
}

// acc[16 x 64] += A[16 x HD] * T^T where T is a [64][HD] smem tile (T rows are
// the output columns): the "scores" product Q K^T / K Q^T / dO V^T / V dO^T.
template <int HD>
__device__ __forceinline__ void mma_a_tileT(const uint32_t (*a)[4], const __nv_bfloat16* t,
                                            float (*acc)[4]) {
  constexpr int LD = HD + 8;
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t b[4];
      ldsm_x4(smem_u32(t + (16 * p + (l & 7) + (l >> 4) * 8) * LD + kk * 16 + ((l >> 3) & 1) * 8),
              b);
      mma16816(acc[2 * p], a[kk], b[0], b[1]);
      mma16816(acc[2 * p + 1], a[kk], b[2], b[3]);
    }
  }
}

// Same product with the A fragments streamed from a smem tile (rows row0..+16).
template <int HD>
__device__ __forceinline__ void mma_tile_tileT(const __nv_bfloat16* a_s, int row0,
                                               const __nv_bfloat16* t, float (*acc)[4]) {
  constexpr int LD = HD + 8;
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(smem_u32(a_s + (row0 + (l & 15)) * LD + kk * 16 + (l >> 4) * 8), a);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      uint32_t b[4];
      ldsm_x4(smem_u32(t + (16 * p + (l & 7) + (l >> 4) * 8) * LD + kk * 16 + ((l >> 3) & 1) * 8),
              b);
      mma16816(acc[2 * p], a, b[0], b[1]);
      mma16816(acc[2 * p + 1], a, b[2], b[3]);
    }
  }
}

// out[16 x HD] += P[16 x 64] * T where T is a [64][HD] smem tile and P is held
// as fp32 accumulators of the scores layout (8 n-tiles of 8 columns).
template <int HD>
__device__ __forceinline__ void mma_p_tile(const float (*p)[4], const __nv_bfloat16* t,
                                           float (*out)[4]) {
  constexpr int LD = HD + 8;
  const int l = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16x2(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_bf16x2(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_bf16x2(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_bf16x2(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int q = 0; q < HD / 16; ++q) {
      uint32_t b[4];
      ldsm_x4_t(smem_u32(t + (16 * kk + (l & 7) + ((l >> 3) & 1) * 8) * LD + 16 * q + (l >> 4) * 8),
                b);
      mma16816(out[2 * q], a, b[0], b[1]);
      mma16816(out[2 * q + 1], a, b[2], b[3]);
    }
  }
}

// Forward: a CTA owns BQ = 16 * WARPS query rows (one warp per 16 rows) and
// walks the causal key blocks of 64 (double-buffered by cp.async).
template <int HD, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ o,
                    float* __restrict__ lse2, int S, int H, int Hkv, int d, float scale_log2) {
  constexpr int LD = HD + 8;
  constexpr int BQ = 16 * WARPS;
  constexpr int KT = 64 * LD;
  extern __shared__ __align__(16) __nv_bfloat16 sm_attn[];
  __nv_bfloat16* sQ = sm_attn;
  __nv_bfloat16* sK = sQ + BQ * LD;  // [2] tiles of 64 keys
  __nv_bfloat16* sV = sK + 2 * KT;

  const int qb = gridDim.x - 1 - blockIdx.x;  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int dkv = Hkv * HD, hk = h / (H / Hkv);  // grouped-query: kv head of this q head
  const int ldq = d + 2 * dkv;
  const size_t tok0 = static_cast<size_t>(b) * S;
  const __nv_bfloat16* Qg = qkv + (tok0 + qb * BQ) * ldq + h * HD;
  const __nv_bfloat16* Kg = qkv + tok0 * ldq + d + hk * HD;
  const __nv_bfloat16* Vg = qkv + tok0 * ldq + d + dkv + hk * HD;

  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int g = l >> 2, t4 = l & 3;
  const int row_base = qb * BQ + warp * 16;  // first global query row of this warp

  load_tile_async<HD, BQ>(sQ, Qg, ldq);
  load_tile_async<HD>(sK, Kg, ldq);
  load_tile_async<HD>(sV, Vg, ldq);
  cp_async_commit();

  uint32_t qf[HD / 16][4];
  float acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY};
  float lsum[2] = {0.f, 0.f};

  const int nblk = ((qb + 1) * BQ) / 64;  // key blocks up to the block diagonal
  for (int j = 0; j < nblk; ++j) {
    const int buf = j & 1;
    if (j + 1 < nblk) {
      load_tile_async<HD>(sK + (buf ^ 1) * KT, Kg + static_cast<size_t>(j + 1) * 64 * ldq, ldq);
      load_tile_async<HD>(sV + (buf ^ 1) * KT, Vg + static_cast<size_t>(j + 1) * 64 * ldq, ldq);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) load_a_frags<HD>(sQ, warp * 16, qf);
    // Key blocks entirely above this warp's rows contribute nothing.
    if (j * 64 <= row_base + 15) {
      float sc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
      mma_a_tileT<HD>(qf, sK + buf * KT, sc);
      const bool diag = (j * 64 + 63 > row_base);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int qrow = row_base + g + 8 * r;
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kcol = j * 64 + nt * 8 + 2 * t4 + e;
            float x = sc[nt][2 * r + e] * scale_log2;
            if (diag && kcol > qrow) x = -INFINITY;
            sc[nt][2 * r + e] = x;
            mx = fmaxf(mx, x);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(m[r], mx);
        const float alpha = (m[r] == -INFINITY) ? 0.f : fast_exp2(m[r] - mnew);
        m[r] = mnew;
        float rs = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float pv = fast_exp2(sc[nt][2 * r + e] - mnew);
            sc[nt][2 * r + e] = pv;
            rs += pv;
          }
        lsum[r] = lsum[r] * alpha + rs;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          acc[i][2 * r] *= alpha;
          acc[i][2 * r + 1] *= alpha;
        }
      }
      mma_p_tile<HD>(sc, sV + buf * KT, acc);
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float ls = lsum[r];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    const float inv = 1.0f / ls;
    const int qrow = row_base + g + 8 * r;
    __nv_bfloat16* orow = o + (tok0 + qrow) * d + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      *reinterpret_cast<uint32_t*>(orow + 8 * i + 2 * t4) =
          pack_bf16x2(acc[i][2 * r] * inv, acc[i][2 * r + 1] * inv);
    }
    if (t4 == 0) lse2[(static_cast<size_t>(b) * H + h) * S + qrow] = m[r] + log2f(ls);
  }
}

// D[b, h, s] = sum_j dO[t, h*hd + j] * O[t, h*hd + j] (one warp per (t, h)).
__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ o,
                                    const __nv_bfloat16* __restrict__ dout, float* __restrict__ D,
                                    int T, int S, int H, int hd, int d) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int l = threadIdx.x & 31;
  if (w >= T * H) return;
  const int t = w / H, h = w % H;
  const __nv_bfloat16* op = o + static_cast<size_t>(t) * d + h * hd;
  const __nv_bfloat16* dp = dout + static_cast<size_t>(t) * d + h * hd;
  float s = 0.f;
  for (int j = l; j < hd; j += 32) s += __bfloat162float(op[j]) * __bfloat162float(dp[j]);
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
  if (l == 0) {
    const int b = t / S, si = t % S;
    D[(static_cast<size_t>(b) * H + h) * S + si] = s;
  }
}

// dQ: a CTA owns BQ = 16 * WARPS query rows and walks the key blocks of 64.
template <int HD, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    attn_bwd_dq_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                       const float* __restrict__ lse2, const float* __restrict__ Dv,
                       __nv_bfloat16* __restrict__ dqkv, int S, int H, int Hkv, int d,
                       float scale_log2, float scale) {
  constexpr int LD = HD + 8;
  constexpr int BQ = 16 * WARPS;
  constexpr int KT = 64 * LD;
  extern __shared__ __align__(16) __nv_bfloat16 sm_attn[];
  __nv_bfloat16* sQ = sm_attn;
  __nv_bfloat16* sdO = sQ + BQ * LD;
  __nv_bfloat16* sK = sdO + BQ * LD;  // [2]
  __nv_bfloat16* sV = sK + 2 * KT;

  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int dkv = Hkv * HD, hk = h / (H / Hkv);
  const int ldq = d + 2 * dkv;
  const size_t tok0 = static_cast<size_t>(b) * S;
  const __nv_bfloat16* Qg = qkv + (tok0 + qb * BQ) * ldq + h * HD;
  const __nv_bfloat16* dOg = dout + (tok0 + qb * BQ) * d + h * HD;
  const __nv_bfloat16* Kg = qkv + tok0 * ldq + d + hk * HD;
  const __nv_bfloat16* Vg = qkv + tok0 * ldq + d + dkv + hk * HD;
  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int g = l >> 2, t4 = l & 3;
  const int row_base = qb * BQ + warp * 16;

  load_tile_async<HD, BQ>(sQ, Qg, ldq);
  load_tile_async<HD, BQ>(sdO, dOg, d);
  load_tile_async<HD>(sK, Kg, ldq);
  load_tile_async<HD>(sV, Vg, ldq);
  cp_async_commit();

  float lr[2], dr[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const size_t idx = (static_cast<size_t>(b) * H + h) * S + row_base + g + 8 * r;
    lr[r] = lse2[idx];
    dr[r] = Dv[idx];
  }
  uint32_t qf[HD / 16][4];
  uint32_t of[HD / 16][4];
  float dq[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  const int nblk = ((qb + 1) * BQ) / 64;
  for (int j = 0; j < nblk; ++j) {
    const int buf = j & 1;
    if (j + 1 < nblk) {
      load_tile_async<HD>(sK + (buf ^ 1) * KT, Kg + static_cast<size_t>(j + 1) * 64 * ldq, ldq);
      load_tile_async<HD>(sV + (buf ^ 1) * KT, Vg + static_cast<size_t>(j + 1) * 64 * ldq, ldq);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
      load_a_frags<HD>(sQ, warp * 16, qf);
      load_a_frags<HD>(sdO, warp * 16, of);
    }
    if (j * 64 <= row_base + 15) {
      float sc[8][4], dp[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
        dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
      }
      mma_a_tileT<HD>(qf, sK + buf * KT, sc);
      mma_a_tileT<HD>(of, sV + buf * KT, dp);
      const bool diag = (j * 64 + 63 > row_base);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = e >> 1;
          const int qrow = row_base + g + 8 * r;
          const int kcol = j * 64 + nt * 8 + 2 * t4 + (e & 1);
          float pv = fast_exp2(sc[nt][e] * scale_log2 - lr[r]);
          if (diag && kcol > qrow) pv = 0.f;
          sc[nt][e] = pv * (dp[nt][e] - dr[r]);  // dS
        }
      mma_p_tile<HD>(sc, sK + buf * KT, dq);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qrow = row_base + g + 8 * r;
    __nv_bfloat16* out = dqkv + (tok0 + qrow) * ldq + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
      *reinterpret_cast<uint32_t*>(out + 8 * i + 2 * t4) =
          pack_bf16x2(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
  }
}

// dK / dV: a CTA owns BKV = 16 * WARPS key rows and walks the query blocks of 64.
template <int HD, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    attn_bwd_dkdv_kernel(const __nv_bfloat16* __restrict__ qkv,
                         const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse2,
                         const float* __restrict__ Dv, __nv_bfloat16* __restrict__ dqkv, int S,
                         int H, int Hkv, int d, float scale_log2, float scale) {
  constexpr int LD = HD + 8;
  constexpr int BKV = 16 * WARPS;
  constexpr int QT = 64 * LD;
  extern __shared__ __align__(16) __nv_bfloat16 sm_attn[];
  __nv_bfloat16* sK = sm_attn;
  __nv_bfloat16* sV = sK + BKV * LD;
  __nv_bfloat16* sQ = sV + BKV * LD;  // [2]
  __nv_bfloat16* sdO = sQ + 2 * QT;   // [2]
  float* sL = reinterpret_cast<float*>(sdO + 2 * QT);  // [2][64]
  float* sD = sL + 128;                                 // [2][64]

  const int nkb = gridDim.x;
  const int kb = nkb - 1 - blockIdx.x;  // the heaviest key blocks (earliest keys) last
  // Grid y runs over kv heads; a kv head sums the rep = H / Hkv query heads
  // of its group in head order (deterministic, no atomics).
  const int hk = blockIdx.y, b = blockIdx.z;
  const int rep = H / Hkv, dkv = Hkv * HD;
  const int ldq = d + 2 * dkv;
  const size_t tok0 = static_cast<size_t>(b) * S;
  const __nv_bfloat16* Kg = qkv + (tok0 + kb * BKV) * ldq + d + hk * HD;
  const __nv_bfloat16* Vg = qkv + (tok0 + kb * BKV) * ldq + d + dkv + hk * HD;
  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int g = l >> 2, t4 = l & 3;
  const int krow_base = kb * BKV + warp * 16;
  const int nq = S / 64;
  const int q0 = (kb * BKV) / 64;  // first query block that sees these keys
  const int nqs = nq - q0;
  const int steps = rep * nqs;  // (query head of the group, query block) pairs

  // Stage step `it` (query head hk * rep + it / nqs, block q0 + it % nqs) into buffer nb.
  auto stage = [&](int it, int nb) {
    const int h = hk * rep + it / nqs, qi = q0 + it % nqs;
    load_tile_async<HD>(sQ + nb * QT, qkv + (tok0 + static_cast<size_t>(qi) * 64) * ldq + h * HD,
                        ldq);
    load_tile_async<HD>(sdO + nb * QT, dout + (tok0 + static_cast<size_t>(qi) * 64) * d + h * HD,
                        d);
    if (threadIdx.x < 64) {
      const size_t row = (static_cast<size_t>(b) * H + h) * S + qi * 64 + threadIdx.x;
      sL[nb * 64 + threadIdx.x] = lse2[row];
      sD[nb * 64 + threadIdx.x] = Dv[row];
    }
  };

  load_tile_async<HD, BKV>(sK, Kg, ldq);
  load_tile_async<HD, BKV>(sV, Vg, ldq);
  stage(0, 0);
  cp_async_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  for (int it = 0; it < steps; ++it) {
    const int qi = q0 + it % nqs;
    const int buf = it & 1;
    if (it + 1 < steps) {
      stage(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* q_s = sQ + buf * QT;
    const __nv_bfloat16* do_s = sdO + buf * QT;
    const float* l_s = sL + buf * 64;
    const float* d_s = sD + buf * 64;
    // Query blocks entirely before this warp's keys contribute nothing.
    if (qi * 64 + 63 >= krow_base) {
      // S^T[kv, q] = K Q^T for this warp's 16 key rows.
      float st[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
      mma_tile_tileT<HD>(sK, warp * 16, q_s, st);
      const bool diag = (qi * 64 < krow_base + 16);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int krow = krow_base + g + 8 * (e >> 1);
          const int qcol = nt * 8 + 2 * t4 + (e & 1);
          float pv = fast_exp2(st[nt][e] * scale_log2 - l_s[qcol]);
          if (diag && krow > qi * 64 + qcol) pv = 0.f;
          st[nt][e] = pv;  // P^T
        }
      mma_p_tile<HD>(st, do_s, dv);  // dV += P^T dO
      float dpt[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
      mma_tile_tileT<HD>(sV, warp * 16, do_s, dpt);  // dP^T = V dO^T
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qcol = nt * 8 + 2 * t4 + (e & 1);
          st[nt][e] = st[nt][e] * (dpt[nt][e] - d_s[qcol]);  // dS^T
        }
      mma_p_tile<HD>(st, q_s, dk);  // dK += dS^T Q
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int krow = krow_base + g + 8 * r;
    __nv_bfloat16* outk = dqkv + (tok0 + krow) * ldq + d + hk * HD;
    __nv_bfloat16* outv = dqkv + (tok0 + krow) * ldq + d + dkv + hk * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      *reinterpret_cast<uint32_t*>(outk + 8 * i + 2 * t4) =
          pack_bf16x2(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(outv + 8 * i + 2 * t4) =
          pack_bf16x2(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

template <typename K>
int set_smem(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
                 cudaSuccess
             ? 0
             : 1;
}

template <int HD, int WARPS>
int attn_fwd_hd(const AttnArgs& a, cudaStream_t stream) {
  constexpr int LD = HD + 8;
  const int smem = (16 * WARPS * LD + 4 * 64 * LD) * 2;
  if (set_smem(attn_fwd_kernel<HD, WARPS>, smem)) return 2;
  dim3 grid(a.S / (16 * WARPS), a.H, a.B);
  attn_fwd_kernel<HD, WARPS><<<grid, WARPS * 32, smem, stream>>>(
      a.qkv, a.o, a.lse, a.S, a.H, a.Hkv > 0 ? a.Hkv : a.H, a.d, a.scale * kLog2e);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

template <int HD, int WARPS>
int attn_bwd_hd(const AttnBwdArgs& a, cudaStream_t stream) {
  constexpr int LD = HD + 8;
  const int T = a.B * a.S;
  const int warps = T * a.H;
  attn_bwd_dot_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(a.o, a.dout, a.Dbuf, T, a.S,
                                                                    a.H, HD, a.d);
  const int smem_dq = (2 * 16 * WARPS * LD + 4 * 64 * LD) * 2;
  const int smem_kv = (2 * 16 * WARPS * LD + 4 * 64 * LD) * 2 + 4 * 64 * 4;
  if (set_smem(attn_bwd_dq_kernel<HD, WARPS>, smem_dq)) return 2;
  if (set_smem(attn_bwd_dkdv_kernel<HD, WARPS>, smem_kv)) return 2;
  const int hkv = a.Hkv > 0 ? a.Hkv : a.H;
  dim3 grid_kv(a.S / (16 * WARPS), hkv, a.B);
  dim3 grid_q(a.S / (16 * WARPS), a.H, a.B);
  attn_bwd_dkdv_kernel<HD, WARPS><<<grid_kv, WARPS * 32, smem_kv, stream>>>(
      a.qkv, a.dout, a.lse, a.Dbuf, a.dqkv, a.S, a.H, hkv, a.d, a.scale * kLog2e, a.scale);
  attn_bwd_dq_kernel<HD, WARPS><<<grid_q, WARPS * 32, smem_dq, stream>>>(
      a.qkv, a.dout, a.lse, a.Dbuf, a.dqkv, a.S, a.H, hkv, a.d, a.scale * kLog2e, a.scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace

// Sequences that are a multiple of 128 use 8-warp CTAs (128 rows); others 4.
int attention_fwd(const AttnArgs& a, cudaStream_t stream) {
  if (a.S % 64 || a.d != a.H * a.hd || (a.Hkv > 0 && a.H % a.Hkv)) return 1;
  if (a.impl == 0 && a.hd == 128 && a.S % 128 == 0) {
    const int rc = attention_fwd_tc(a, a.status, stream);
    if (rc != 1) return rc;
  }
  const bool big = a.S % 128 == 0;
  switch (a.hd) {
    case 64: return big ? attn_fwd_hd<64, 8>(a, stream) : attn_fwd_hd<64, 4>(a, stream);
    case 80: return big ? attn_fwd_hd<80, 8>(a, stream) : attn_fwd_hd<80, 4>(a, stream);
    case 128: return big ? attn_fwd_hd<128, 8>(a, stream) : attn_fwd_hd<128, 4>(a, stream);
    default: return 1;
  }
}

int attention_bwd(const AttnBwdArgs& a, cudaStream_t stream) {
  if (a.S % 64 || a.d != a.H * a.hd || (a.Hkv > 0 && a.H % a.Hkv)) return 1;
  if (a.impl == 0 && a.hd == 128 && a.S % 128 == 0) {
    const int T = a.B * a.S;
    const int warps = T * a.H;
    attn_bwd_dot_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(a.o, a.dout, a.Dbuf, T,
                                                                      a.S, a.H, a.hd, a.d);
    if (cudaGetLastError() != cudaSuccess) return 2;
    const int rc = attention_bwd_tc(a, a.status, stream);
    if (rc != 1) return rc;
  }
  const bool big = a.S % 128 == 0;
  switch (a.hd) {
    case 64: return big ? attn_bwd_hd<64, 8>(a, stream) : attn_bwd_hd<64, 4>(a, stream);
    case 80: return big ? attn_bwd_hd<80, 8>(a, stream) : attn_bwd_hd<80, 4>(a, stream);
    case 128: return big ? attn_bwd_hd<128, 8>(a, stream) : attn_bwd_hd<128, 4>(a, stream);
    default: return 1;
  }
}

}  // namespace ewb
