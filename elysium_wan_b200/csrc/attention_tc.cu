// Causal attention forward on the 5th-generation tensor cores (tcgen05 + TMEM
// + TMA) for sm_100a, head_dim 128, sequence lengths a multiple of 128.
//
// Reference op: scaled_dot_product_attention(q, k, v, is_causal=True) in
// src/wantrain/model/gpt.py:366-389 (arch.py:163-176 for grouped-query heads).
// Same contract as the mma.sync kernels of attention.cu (fused q | k | v rows
// in, o and the base-2 log-sum-exp out), which remain the path for other
// shapes and the backward.
//
// One CTA owns 128 query rows of one (batch, head) and walks the causal key
// blocks of 128. Ten warps:
//   warp 0     TMA producer: Q once, then K and V tiles into a 2-stage ring;
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//              S buffers, then O += P_{j-1} V_{j-1} into the TMEM O
//              accumulator; S_{j+1} is issued before P_j exists, so the
//              tensor core works while the softmax warps do;
//   warps 2-9  softmax in two warpgroups: warpgroup g owns key columns
//              64 g .. 64 g + 63 of every row, one query row per thread (warp
//              w reads TMEM lanes 32 (w % 4) .. +31, so each lane quarter has
//              one warp of each group). Its half of the S row is read once
//              into registers (the TMEM buffer is released at once), the two
//              halves' maxima meet through shared memory (a 64-thread named
//              barrier per lane quarter), exp2 of the half row, P rounded to
//              bf16 and written into its 64-column chunk of shared memory in the
//              128-byte-swizzled K-major layout the MMA reads, the running O
//              (its 64 columns) rescaled in TMEM only when the row max grows by
//              more than 2^8 (P and l use the same stale max, so O / l is
//              unchanged), and its half of the final O / l written out; the
//              row sum l is kept per half and added once at the end.
// TMEM: S0 | S1 | O = 384 of 512 columns. Shared memory: Q 32 KB, K 2 x 32 KB,
// V 2 x 32 KB, P 2 x 32 KB (224 KB). Every mbarrier wait is bounded (a
// status word records a timeout and every role returns).
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace ewb {
namespace {

constexpr int kTcHD = 128;
constexpr int kTcBlk = 128;
constexpr uint32_t kTile = 32768;  // one 128 x 128 bf16 tile (two 64-column chunks)
constexpr uint32_t kChunk = 16384;
constexpr uint32_t kOffQ = 0, kOffK = kTile, kOffV = 3 * kTile, kOffP = 5 * kTile;
constexpr uint32_t kOffBar = 7 * kTile;
constexpr uint32_t kOffXch = 7 * kTile + 256;  // [2 groups][128 rows] fp32 exchange
constexpr int kTcSmem = 7 * kTile + 256 + 1024 + 1024;
constexpr int kTcFwdThreads = 320;
constexpr float kLog2eTc = 1.4426950408889634f;
constexpr float kRescale = 8.0f;  // log2 of the largest P the lazy rescale allows

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kTcFwdThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_qk,
                       const __grid_constant__ CUtensorMap map_v, __nv_bfloat16* __restrict__ o,
                       float* __restrict__ lse2, int S, int H, int Hkv, int d, float scale_log2,
                       int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;   // [2]
  uint64_t* kempty = bars + 3;  // [2]
  uint64_t* vfull = bars + 5;   // [2]
  uint64_t* vempty = bars + 7;  // [2]
  uint64_t* sfull = bars + 9;   // [2]
  uint64_t* sfree = bars + 11;  // [2]
  uint64_t* pfull = bars + 13;  // [2]
  uint64_t* ofull = bars + 15;  // [2]: O += P_i V_i commits to ofull[i & 1]
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  // Longest rows first across all heads (blockIdx.x, the fastest launch
  // dimension, walks the heads): the greedy CTA scheduler then ends within
  // about one short tile of the ideal instead of one long tile.
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int h = blockIdx.x, b = blockIdx.z;
  const int hk = h / (H / Hkv);
  const int dkv = Hkv * kTcHD;
  const int row0 = b * S;
  const int nblk = qb + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    mbar_init(qfull, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], 8);
      mbar_init(&pfull[i], 8);
      mbar_init(&ofull[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map_qk);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint8_t* sq = smem + kOffQ;
      mbar_arrive_expect_tx(qfull, kTile);
      for (int c = 0; c < 2; ++c)
        tma_load_2d(sq + c * kChunk, &map_qk, qfull, h * kTcHD + c * 64, row0 + qb * kTcBlk, status);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nblk && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        uint8_t* sk = smem + kOffK + s * kTile;
        uint8_t* sv = smem + kOffV + s * kTile;
        if (!mbar_wait(&kempty[s], ph, status, kStatusTimeoutSmemEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kfull[s], kTile);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sk + c * kChunk, &map_qk, &kfull[s], d + hk * kTcHD + c * 64,
                      row0 + j * kTcBlk, status);
        if (!mbar_wait(&vempty[s], ph, status, kStatusTimeoutSmemEmpty)) {
          ok = false;
          issued = 2 * j + 1;
          break;
        }
        mbar_arrive_expect_tx(&vfull[s], kTile);
        for (int kb = 0; kb < 2; ++kb)
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sv + kb * kChunk + c * 8192, &map_v, &vfull[s],
                        d + dkv + hk * kTcHD + c * 64, row0 + j * kTcBlk + kb * 64, status);
        issued = 2 * j + 2;
      }
      // Drain: loads already issued must land before this CTA's memory goes away.
      mbar_wait(qfull, 0, nullptr, kStatusTimeoutDrain);
      if (!ok) {
        for (int i = issued - 1; i >= 0 && i >= issued - 4; --i) {
          const int j = i >> 1;
          uint64_t* bar = (i & 1) ? &vfull[j & 1] : &kfull[j & 1];
          mbar_wait(bar, (j >> 1) & 1, nullptr, kStatusTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IS = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t IP = idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(smem + kOffQ);
      bool ok = mbar_wait(qfull, 0, status, kStatusTimeoutSmemFull);
      auto pv = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&pfull[s], ph, status, kStatusTimeoutTmemFull)) return false;
        if (!mbar_wait(&vfull[s], ph, status, kStatusTimeoutSmemFull)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + kOffP + s * kTile);
        const uint32_t v_addr = smem_u32(smem + kOffV + s * kTile);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + 256, sdesc_sw128(p_addr + kb * kChunk + kk * 32, 16, 1024),
                     sdesc_sw128(v_addr + kb * kChunk + kk * 2048, 8192, 1024), IP,
                     (i > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&vempty[s]);
        umma_commit(&ofull[s]);
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kfull[s], ph, status, kStatusTimeoutSmemFull) ||
            !mbar_wait(&sfree[s], ph ^ 1, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + s * kTile);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + s * 128, sdesc_sw128(q_addr + c * kChunk + kk * 32, 16, 1024),
                     sdesc_sw128(k_addr + c * kChunk + kk * 32, 16, 1024), IS,
                     (c > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kempty[s]);
        umma_commit(&sfull[s]);
        if (j > 0 && !pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) pv(nblk - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, kStatusTimeoutDrain);
    }
  } else {
    const int wq = warp & 3;
    const int g = (warp - 2) >> 2;  // column half of this warpgroup
    const int c0 = g * 64;
    const int r = wq * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lanes = static_cast<uint32_t>(wq * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + kOffXch);  // [2][128]
    const int bar_id = 1 + wq;  // the two warps of this lane quarter
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (ok && !mbar_wait(&sfull[s], ph, status, kStatusTimeoutTmemFull)) ok = false;
      uint32_t v[64];
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        const uint32_t s_t = tmem + s * 128 + c0 + lanes;
        const bool diag = (j == qb);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld16(s_t + c * 16, v + c * 16);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          float x = __uint_as_float(v[i]) * scale_log2;
          if (diag && c0 + i > r) x = -INFINITY;
          v[i] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
        // this half of S is in registers: the buffer can take S_{j+2}
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[s]);
      }
      // The row max over both halves. Every warp passes the same sequence of
      // named barriers whatever happens (a failed wait only skips work), so the
      // two warps of a quarter can never meet at different barriers.
      xch[g * 128 + r] = ok ? mx : INFINITY;
      named_bar_sync(bar_id, 64);
      const float other = xch[(g ^ 1) * 128 + r];
      named_bar_sync(bar_id, 64);
      if (other == INFINITY) ok = false;
      if (!ok) continue;
      mx = fmaxf(mx, other);
      // Lazy rescaling: the running max moves only when it grows by more than
      // kRescale (log2 units); P and l use the same stale max, so O / l is the
      // same quantity (P <= 2^kRescale, well inside bf16 and fp32 range). The
      // two warps of a quarter see the same rows, so they decide alike.
      float mnew = m;
      if (__any_sync(0xffffffffu, mx > m + kRescale)) mnew = fmaxf(m, mx);
      const float alpha = (m == -INFINITY) ? 0.f : ex2f(m - mnew);
      // P_j reuses the buffer of P_{j-2}: O += P_{j-2} V_{j-2} must be
      // complete. O += P_{j-1} V_{j-1} may still run while exp2 fills P_j;
      // only a rescale of O (below) waits for it.
      if (j > 1 && !mbar_wait(&ofull[s], ((j - 2) >> 1) & 1, status, kStatusTimeoutTmemFull)) {
        ok = false;
        continue;
      }
      const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha != 1.0f);
      tc_fence_after();
      uint8_t* prow = smem + kOffP + s * kTile + g * kChunk + r * 128;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 8 keys per 16-byte unit
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = ex2f(__uint_as_float(v[c * 8 + 2 * i]) - mnew);
          const float p1 = ex2f(__uint_as_float(v[c * 8 + 2 * i + 1]) - mnew);
          rs += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l = l * alpha + rs;
      if (rescale) {
        if (!mbar_wait(&ofull[s ^ 1], ((j - 1) >> 1) & 1, status, kStatusTimeoutTmemFull)) {
          ok = false;
          continue;
        }
        tc_fence_after();
        const uint32_t o_t = tmem + 256 + c0 + lanes;
        uint32_t ov[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(o_t + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st16(o_t + c * 32, ov);
          tmem_st16(o_t + c * 32 + 16, ov + 16);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[s]);
      m = mnew;
    }
    // the row sum over both halves (both warps of the quarter get here)
    xch[g * 128 + r] = ok ? l : -1.0f;
    named_bar_sync(bar_id, 64);
    const float l_other = xch[(g ^ 1) * 128 + r];
    if (ok && l_other >= 0.f &&
        mbar_wait(&ofull[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, status,
                  kStatusTimeoutTmemFull)) {
      tc_fence_after();
      l = g == 0 ? l + l_other : l_other + l;  // the same sum in both halves
      const float inv = 1.0f / l;
      const int qrow = qb * kTcBlk + r;
      __nv_bfloat16* orow = o + (static_cast<size_t>(row0) + qrow) * d + h * kTcHD + c0;
      const uint32_t o_t = tmem + 256 + c0 + lanes;
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(o_t + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          uint4 w4;
          w4.x = pack_bf16x2(__uint_as_float(v[8 * t]) * inv, __uint_as_float(v[8 * t + 1]) * inv);
          w4.y = pack_bf16x2(__uint_as_float(v[8 * t + 2]) * inv, __uint_as_float(v[8 * t + 3]) * inv);
          w4.z = pack_bf16x2(__uint_as_float(v[8 * t + 4]) * inv, __uint_as_float(v[8 * t + 5]) * inv);
          w4.w = pack_bf16x2(__uint_as_float(v[8 * t + 6]) * inv, __uint_as_float(v[8 * t + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + t * 8) = w4;
        }
      }
      if (g == 0) lse2[(static_cast<size_t>(b) * H + h) * S + qrow] = m + log2f(l);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------------
// Backward. D = rowsum(dO * O) comes from the dot kernel of attention.cu.
//
// dK / dV: a CTA owns 128 keys of one (batch, kv head) and walks the
// (query head of its group, query block of 64) pairs in order, so a kv
// head's gradient is summed over its query heads in head order (no atomics):
//   S^T = K Q^T and dP^T = V dO^T (M 128 keys, N 64 queries) into one of two
//   TMEM buffer pairs; the softmax warps (one key row per thread) form
//   P^T = exp2(S^T - lse) and dS^T = P^T (dP^T - D), round both to bf16 and
//   write them K-major into shared memory; then dV += P^T dO and
//   dK += dS^T Q (M 128 keys, N 128, K 64) accumulate in TMEM. The MMA issuer
//   starts S^T / dP^T of the next pair before the grads of this one, so the
//   tensor core overlaps the softmax warps.
// TMEM: S^T x2 | dP^T x2 (64 columns each) | dV | dK = 512 columns.
// Shared memory: K 32 KB, V 32 KB, Q / dO / lse / D 2 stages, P^T / dS^T 2
// buffers (196 KB).
constexpr uint32_t kBwOffK = 0, kBwOffV = 32768, kBwOffQ = 65536, kBwOffDO = 98304;
constexpr uint32_t kBwOffL = 131072, kBwOffD = 131584, kBwOffP = 135168, kBwOffS = 167936;
constexpr uint32_t kBwOffBar = 200704;
constexpr int kBwSmem = 200704 + 256 + 1024;

constexpr int kBwThreads = 320;  // producer, MMA issuer, two warpgroups of four softmax warps

__global__ void __launch_bounds__(kBwThreads, 1)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap map_kv,
                            const __grid_constant__ CUtensorMap map_q,
                            const __grid_constant__ CUtensorMap map_do,
                            const float* __restrict__ lse2, const float* __restrict__ Dv,
                            __nv_bfloat16* __restrict__ dqkv, int S, int H, int Hkv, int d,
                            float scale_log2, float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBwOffBar);
  uint64_t* kvfull = bars;
  uint64_t* qfull = bars + 1;  // [2]
  uint64_t* done = bars + 3;   // [2]  grads MMAs of a pair finished (stage and P/dS free)
  uint64_t* sfull = bars + 5;  // [2]
  uint64_t* sfree = bars + 7;  // [2]
  uint64_t* pfull = bars + 9;  // [2]
  uint64_t* fin = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int kb = blockIdx.y;  // earliest keys (most query blocks) first, across all kv heads
  const int hk = blockIdx.x, bz = blockIdx.z;
  const int rep = H / Hkv, dkv = Hkv * kTcHD, ldq = d + 2 * dkv;
  const int row0 = bz * S;
  const int nq = S / 64, i0 = 2 * kb, nqs = nq - i0;
  const int steps = rep * nqs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    mbar_init(kvfull, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&done[i], 1);
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], 8);
      mbar_init(&pfull[i], 8);
    }
    mbar_init(fin, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map_kv);
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_do);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kvfull, 2 * kTile);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + kBwOffK + c * kChunk, &map_kv, kvfull, d + hk * kTcHD + c * 64,
                    row0 + kb * kTcBlk, status);
        tma_load_2d(smem + kBwOffV + c * kChunk, &map_kv, kvfull, d + dkv + hk * kTcHD + c * 64,
                    row0 + kb * kTcBlk, status);
      }
      int issued = 0;
      for (int t = 0; t < steps; ++t) {
        const int sb = t & 1;
        const int h = hk * rep + t / nqs, i = i0 + t % nqs;
        if (!mbar_wait(&done[sb], ((t >> 1) & 1) ^ 1, status, kStatusTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&qfull[sb], 2 * 16384 + 512);
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(smem + kBwOffQ + sb * 16384 + c * 8192, &map_q, &qfull[sb],
                      h * kTcHD + c * 64, row0 + i * 64, status);
          tma_load_2d(smem + kBwOffDO + sb * 16384 + c * 8192, &map_do, &qfull[sb],
                      h * kTcHD + c * 64, row0 + i * 64, status);
        }
        const size_t li = (static_cast<size_t>(bz) * H + h) * S + i * 64;
        bulk_load(smem + kBwOffL + sb * 256, lse2 + li, 256, &qfull[sb]);
        bulk_load(smem + kBwOffD + sb * 256, Dv + li, 256, &qfull[sb]);
        issued = t + 1;
      }
      mbar_wait(kvfull, 0, nullptr, kStatusTimeoutDrain);
      for (int t = issued - 1; t >= 0 && t >= issued - 2; --t)
        mbar_wait(&qfull[t & 1], (t >> 1) & 1, nullptr, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IS = idesc_bf16_f32(128, 64, false, false);
      constexpr uint32_t IG = idesc_bf16_f32(128, 128, false, true);
      const uint32_t k_addr = smem_u32(smem + kBwOffK), v_addr = smem_u32(smem + kBwOffV);
      bool ok = mbar_wait(kvfull, 0, status, kStatusTimeoutSmemFull);
      auto grads = [&](int t) -> bool {
        const int sb = t & 1;
        if (!mbar_wait(&pfull[sb], (t >> 1) & 1, status, kStatusTimeoutTmemFull)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + kBwOffP + sb * 16384);
        const uint32_t s_addr = smem_u32(smem + kBwOffS + sb * 16384);
        const uint32_t q_addr = smem_u32(smem + kBwOffQ + sb * 16384);
        const uint32_t o_addr = smem_u32(smem + kBwOffDO + sb * 16384);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_f16(tmem + 256, sdesc_sw128(p_addr + kk * 32, 16, 1024),
                   sdesc_sw128(o_addr + kk * 2048, 8192, 1024), IG, (t > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tmem + 384, sdesc_sw128(s_addr + kk * 32, 16, 1024),
                   sdesc_sw128(q_addr + kk * 2048, 8192, 1024), IG, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&done[sb]);
        return true;
      };
      for (int t = 0; t < steps && ok; ++t) {
        const int sb = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&qfull[sb], ph, status, kStatusTimeoutSmemFull) ||
            !mbar_wait(&sfree[sb], ph ^ 1, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + kBwOffQ + sb * 16384);
        const uint32_t o_addr = smem_u32(smem + kBwOffDO + sb * 16384);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (c > 0 || kk > 0) ? 1u : 0u;
            umma_f16(tmem + sb * 64, sdesc_sw128(k_addr + c * kChunk + kk * 32, 16, 1024),
                     sdesc_sw128(q_addr + c * 8192 + kk * 32, 16, 1024), IS, acc);
            umma_f16(tmem + 128 + sb * 64, sdesc_sw128(v_addr + c * kChunk + kk * 32, 16, 1024),
                     sdesc_sw128(o_addr + c * 8192 + kk * 32, 16, 1024), IS, acc);
          }
        umma_commit(&sfull[sb]);
        if (t > 0 && !grads(t - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && steps > 0 && grads(steps - 1)) umma_commit(fin);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, kStatusTimeoutDrain);
    }
  } else {
    const int wq = warp & 3;
    const int g = (warp - 2) >> 2;  // this warpgroup's half of the 64 query columns
    const int q0 = g * 32;
    const int r = wq * 32 + lane;  // key row within the block = TMEM lane
    const int kpos = kb * kTcBlk + r;
    const uint32_t lanes = static_cast<uint32_t>(wq * 32) << 16;
    bool ok = true;
    for (int t = 0; t < steps; ++t) {
      const int sb = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      const int i = i0 + t % nqs;
      if (!mbar_wait(&sfull[sb], ph, status, kStatusTimeoutTmemFull) ||
          !mbar_wait(&qfull[sb], ph, status, kStatusTimeoutSmemFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[32], pv[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld16(tmem + sb * 64 + q0 + lanes + c * 16, sv + c * 16);
        tmem_ld16(tmem + 128 + sb * 64 + q0 + lanes + c * 16, pv + c * 16);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[sb]);
      // P^T / dS^T buffer sb was read by the grads of pair t - 2.
      if (!mbar_wait(&done[sb], ph ^ 1, status, kStatusTimeoutSmemEmpty)) {
        ok = false;
        break;
      }
      const float* Ls = reinterpret_cast<const float*>(smem + kBwOffL + sb * 256);
      const float* Ds = reinterpret_cast<const float*>(smem + kBwOffD + sb * 256);
      uint8_t* prow = smem + kBwOffP + sb * 16384 + r * 128;
      uint8_t* srow = smem + kBwOffS + sb * 16384 + r * 128;
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        const int u8 = g * 4 + u4;  // 16-byte unit of the 64-query row
        uint32_t pk[4], dk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float pp[2], dd[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            const int ql = u4 * 8 + 2 * e + z;  // within this half
            const int q = q0 + ql;
            float p = ex2f(__uint_as_float(sv[ql]) * scale_log2 - Ls[q]);
            if (kpos > i * 64 + q) p = 0.f;
            pp[z] = p;
            dd[z] = p * (__uint_as_float(pv[ql]) - Ds[q]);
          }
          pk[e] = pack_bf16x2(pp[0], pp[1]);
          dk[e] = pack_bf16x2(dd[0], dd[1]);
        }
        const uint32_t off = static_cast<uint32_t>((u8 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(prow + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(srow + off) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[sb]);
    }
    if (ok && steps > 0 && mbar_wait(fin, 0, status, kStatusTimeoutTmemFull)) {
      tc_fence_after();
      __nv_bfloat16* dk_row = dqkv + (static_cast<size_t>(row0) + kpos) * ldq + d + hk * kTcHD;
      __nv_bfloat16* dv_row = dk_row + dkv;
      uint32_t v[32];
      {  // warpgroup 0 writes dV, warpgroup 1 dK
        __nv_bfloat16* out = g ? dk_row : dv_row;
        const float mul = g ? scale : 1.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + 256 + g * 128 + lanes + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int t4 = 0; t4 < 4; ++t4) {
            uint4 w4;
            w4.x = pack_bf16x2(__uint_as_float(v[8 * t4]) * mul, __uint_as_float(v[8 * t4 + 1]) * mul);
            w4.y = pack_bf16x2(__uint_as_float(v[8 * t4 + 2]) * mul, __uint_as_float(v[8 * t4 + 3]) * mul);
            w4.z = pack_bf16x2(__uint_as_float(v[8 * t4 + 4]) * mul, __uint_as_float(v[8 * t4 + 5]) * mul);
            w4.w = pack_bf16x2(__uint_as_float(v[8 * t4 + 6]) * mul, __uint_as_float(v[8 * t4 + 7]) * mul);
            *reinterpret_cast<uint4*>(out + c * 32 + t4 * 8) = w4;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ: a CTA owns 128 query rows of one (batch, head) and walks the causal key
// blocks of 128: S = Q K^T and dP = dO V^T (two N = 64 halves each) into
// TMEM, the softmax warps (one query row per thread, its lse and D in
// registers) form dS = P (dP - D) in bf16 into shared memory, then
// dQ += dS K (M 128, N 128, K 128) in TMEM. S and dP are released as soon as
// they are read, and dQ of block j - 1 is issued after S / dP of block j. K and V tiles are loaded as four
// 64 x 64 boxes, which both the K-major (S, dP) and the MN-major (dQ) operand
// views read. TMEM: S | dP | dQ = 384 of 512 columns. Shared memory: Q, dO,
// K x2, V x2, dS (224 KB).
constexpr uint32_t kDqOffQ = 0, kDqOffDO = 32768, kDqOffK = 65536, kDqOffV = 131072;
constexpr uint32_t kDqOffS = 196608, kDqOffBar = 229376;
constexpr int kDqSmem = 229376 + 256 + 1024;

__global__ void __launch_bounds__(kBwThreads, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap map_q128,
                          const __grid_constant__ CUtensorMap map_do128,
                          const __grid_constant__ CUtensorMap map_kv64,
                          const float* __restrict__ lse2, const float* __restrict__ Dv,
                          __nv_bfloat16* __restrict__ dqkv, int S, int H, int Hkv, int d,
                          float scale_log2, float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDqOffBar);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;   // [2]
  uint64_t* kempty = bars + 3;  // [2]
  uint64_t* sfull = bars + 5;
  uint64_t* sfree = bars + 6;   // S read into registers
  uint64_t* pfull = bars + 7;
  uint64_t* dsfree = bars + 8;  // dQ MMA of the previous block finished
  uint64_t* drain = bars + 9;
  uint64_t* dpfree = bars + 10;  // dP read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int qb = gridDim.y - 1 - blockIdx.y;  // longest rows first, across all heads
  const int h = blockIdx.x, bz = blockIdx.z;
  const int hk = h / (H / Hkv);
  const int dkv = Hkv * kTcHD, ldq = d + 2 * dkv;
  const int row0 = bz * S;
  const int nblk = qb + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    mbar_init(qfull, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
    }
    mbar_init(sfull, 1);
    mbar_init(sfree, 8);
    mbar_init(dpfree, 8);
    mbar_init(pfull, 8);
    mbar_init(dsfree, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map_q128);
    tma_prefetch_desc(&map_do128);
    tma_prefetch_desc(&map_kv64);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(qfull, 2 * kTile);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + kDqOffQ + c * kChunk, &map_q128, qfull, h * kTcHD + c * 64,
                    row0 + qb * kTcBlk, status);
        tma_load_2d(smem + kDqOffDO + c * kChunk, &map_do128, qfull, h * kTcHD + c * 64,
                    row0 + qb * kTcBlk, status);
      }
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int sb = j & 1;
        if (!mbar_wait(&kempty[sb], ((j >> 1) & 1) ^ 1, status, kStatusTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&kfull[sb], 2 * kTile);
        for (int kh = 0; kh < 2; ++kh)
          for (int c = 0; c < 2; ++c) {
            const int y = row0 + j * kTcBlk + kh * 64;
            tma_load_2d(smem + kDqOffK + sb * kTile + kh * kChunk + c * 8192, &map_kv64,
                        &kfull[sb], d + hk * kTcHD + c * 64, y, status);
            tma_load_2d(smem + kDqOffV + sb * kTile + kh * kChunk + c * 8192, &map_kv64,
                        &kfull[sb], d + dkv + hk * kTcHD + c * 64, y, status);
          }
        issued = j + 1;
      }
      mbar_wait(qfull, 0, nullptr, kStatusTimeoutDrain);
      for (int j = issued - 1; j >= 0 && j >= issued - 2; --j)
        mbar_wait(&kfull[j & 1], (j >> 1) & 1, nullptr, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IS = idesc_bf16_f32(128, 64, false, false);
      constexpr uint32_t IQ = idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(smem + kDqOffQ), o_addr = smem_u32(smem + kDqOffDO);
      const uint32_t ds_addr = smem_u32(smem + kDqOffS);
      bool ok = mbar_wait(qfull, 0, status, kStatusTimeoutSmemFull);
      // dQ += dS_i K_i, issued after S / dP of the next block so the tensor
      // core overlaps the softmax warps.
      auto dq = [&](int i) -> bool {
        const int sb = i & 1;
        if (!mbar_wait(pfull, i & 1, status, kStatusTimeoutTmemFull)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kDqOffK + sb * kTile);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + 256, sdesc_sw128(ds_addr + kh * kChunk + kk * 32, 16, 1024),
                     sdesc_sw128(k_addr + kh * kChunk + kk * 2048, 8192, 1024), IQ,
                     (i > 0 || kh > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kempty[sb]);
        umma_commit(dsfree);
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        const int sb = j & 1;
        const uint32_t fr = (j & 1) ^ 1;
        if (!mbar_wait(&kfull[sb], (j >> 1) & 1, status, kStatusTimeoutSmemFull) ||
            !mbar_wait(sfree, fr, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kDqOffK + sb * kTile);
        const uint32_t v_addr = smem_u32(smem + kDqOffV + sb * kTile);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16(tmem + kh * 64, sdesc_sw128(q_addr + c * kChunk + kk * 32, 16, 1024),
                       sdesc_sw128(k_addr + kh * kChunk + c * 8192 + kk * 32, 16, 1024), IS,
                       (c > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait(dpfree, fr, status, kStatusTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16(tmem + 128 + kh * 64,
                       sdesc_sw128(o_addr + c * kChunk + kk * 32, 16, 1024),
                       sdesc_sw128(v_addr + kh * kChunk + c * 8192 + kk * 32, 16, 1024), IS,
                       (c > 0 || kk > 0) ? 1u : 0u);
        umma_commit(sfull);
        if (j > 0 && !dq(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) dq(nblk - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, kStatusTimeoutDrain);
    }
  } else {
    const int wq = warp & 3;
    const int g = (warp - 2) >> 2;  // this warpgroup's half of the 128 key columns
    const int k0 = g * 64;
    const int r = wq * 32 + lane;
    const int qrow = qb * kTcBlk + r;
    const uint32_t lanes = static_cast<uint32_t>(wq * 32) << 16;
    const size_t li = (static_cast<size_t>(bz) * H + h) * S + qrow;
    const float lr = lse2[li], dr = Dv[li];
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(sfull, j & 1, status, kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16(tmem + lanes + k0 + c * 16, sv + c * 16);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree);
      const bool diag = (j == qb);
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        float p = ex2f(__uint_as_float(sv[k]) * scale_log2 - lr);
        if (diag && k0 + k > r) p = 0.f;
        sv[k] = __float_as_uint(p);
      }
      uint32_t dp[32];
      // dS buffer: the dQ MMA of block j - 1 must be done reading it.
      if (j > 0 && !mbar_wait(dsfree, (j - 1) & 1, status, kStatusTimeoutSmemEmpty)) {
        ok = false;
        break;
      }
      uint8_t* srow = smem + kDqOffS + g * kChunk + r * 128;  // this half's 64-key chunk
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tmem + 128 + lanes + k0 + c * 32, dp);
        tmem_wait_ld();
#pragma unroll
        for (int t4 = 0; t4 < 4; ++t4) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = c * 32 + t4 * 8 + 2 * e;
            pk[e] = pack_bf16x2(__uint_as_float(sv[k]) * (__uint_as_float(dp[t4 * 8 + 2 * e]) - dr),
                                __uint_as_float(sv[k + 1]) *
                                    (__uint_as_float(dp[t4 * 8 + 2 * e + 1]) - dr));
          }
          const int unit = c * 4 + t4;
          *reinterpret_cast<uint4*>(srow + ((unit ^ (r & 7)) << 4)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dpfree);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull);
    }
    if (ok && mbar_wait(dsfree, (nblk - 1) & 1, status, kStatusTimeoutTmemFull)) {
      tc_fence_after();
      __nv_bfloat16* out = dqkv + (static_cast<size_t>(row0) + qrow) * ldq + h * kTcHD + k0;
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // this warpgroup's 64 of the 128 columns
        tmem_ld32(tmem + 256 + lanes + k0 + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int t4 = 0; t4 < 4; ++t4) {
          uint4 w4;
          w4.x = pack_bf16x2(__uint_as_float(v[8 * t4]) * scale, __uint_as_float(v[8 * t4 + 1]) * scale);
          w4.y = pack_bf16x2(__uint_as_float(v[8 * t4 + 2]) * scale, __uint_as_float(v[8 * t4 + 3]) * scale);
          w4.z = pack_bf16x2(__uint_as_float(v[8 * t4 + 4]) * scale, __uint_as_float(v[8 * t4 + 5]) * scale);
          w4.w = pack_bf16x2(__uint_as_float(v[8 * t4 + 6]) * scale, __uint_as_float(v[8 * t4 + 7]) * scale);
          *reinterpret_cast<uint4*>(out + c * 32 + t4 * 8) = w4;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int attention_fwd_tc(const AttnArgs& a, int* status, cudaStream_t stream) {
  const int hkv = a.Hkv > 0 ? a.Hkv : a.H;
  if (a.hd != kTcHD || a.S % kTcBlk || a.d != a.H * a.hd || a.H % hkv) return 1;
  const int ldq = a.d + 2 * hkv * a.hd;
  const uint64_t rows = static_cast<uint64_t>(a.B) * a.S;
  CUtensorMap mqk, mv;
  if (!tma_map_bf16_2d(&mqk, a.qkv, ldq, rows, ldq, 64, 128) ||
      !tma_map_bf16_2d(&mv, a.qkv, ldq, rows, ldq, 64, 64))
    return 1;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kTcSmem) != cudaSuccess)
      return 2;
    attr = true;
  }
  dim3 grid(a.H, a.S / kTcBlk, a.B);
  attn_fwd_tc_kernel<<<grid, kTcFwdThreads, kTcSmem, stream>>>(mqk, mv, a.o, a.lse, a.S, a.H, hkv,
                                                                a.d, a.scale * kLog2eTc, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb

namespace ewb {

// dK, dV, dQ on the tensor cores; D (rowsum dO * O) must already be in a.Dbuf.
int attention_bwd_tc(const AttnBwdArgs& a, int* status, cudaStream_t stream) {
  const int hkv = a.Hkv > 0 ? a.Hkv : a.H;
  if (a.hd != kTcHD || a.S % kTcBlk || a.d != a.H * a.hd || a.H % hkv) return 1;
  const int ldq = a.d + 2 * hkv * a.hd;
  const uint64_t rows = static_cast<uint64_t>(a.B) * a.S;
  CUtensorMap m_kv128, m_q64, m_do64, m_q128, m_do128, m_kv64;
  if (!tma_map_bf16_2d(&m_kv128, a.qkv, ldq, rows, ldq, 64, 128) ||
      !tma_map_bf16_2d(&m_q64, a.qkv, ldq, rows, ldq, 64, 64) ||
      !tma_map_bf16_2d(&m_do64, a.dout, a.d, rows, a.d, 64, 64) ||
      !tma_map_bf16_2d(&m_q128, a.qkv, ldq, rows, ldq, 64, 128) ||
      !tma_map_bf16_2d(&m_do128, a.dout, a.d, rows, a.d, 64, 128) ||
      !tma_map_bf16_2d(&m_kv64, a.qkv, ldq, rows, ldq, 64, 64))
    return 1;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kBwSmem) != cudaSuccess ||
        cudaFuncSetAttribute(attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kDqSmem) != cudaSuccess)
      return 2;
    attr = true;
  }
  const float sl2 = a.scale * kLog2eTc;
  attn_bwd_dkdv_tc_kernel<<<dim3(hkv, a.S / kTcBlk, a.B), kBwThreads, kBwSmem, stream>>>(
      m_kv128, m_q64, m_do64, a.lse, a.Dbuf, a.dqkv, a.S, a.H, hkv, a.d, sl2, a.scale, status);
  attn_bwd_dq_tc_kernel<<<dim3(a.H, a.S / kTcBlk, a.B), kBwThreads, kDqSmem, stream>>>(
      m_q128, m_do128, m_kv64, a.lse, a.Dbuf, a.dqkv, a.S, a.H, hkv, a.d, sl2, a.scale, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
