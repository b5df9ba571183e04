// tcgen05 / TMEM GEMM for sm_100a with fused epilogues.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]      (bf16 inputs, fp32 accumulation in TMEM)
//
// A is either K-major (stored [M][lda], k contiguous) or MN-major (stored
// [K][lda], m contiguous); the same holds for B. With these two flags one
// kernel covers every GEMM of a transformer block:
//   forward   Y  = X W^T      A = X (K-major),   B = W  (K-major)
//   B pass    dX = dY W       A = dY (K-major),  B = W  (MN-major)
//   W pass    dW = dY^T X     A = dY (MN-major), B = X  (MN-major)
// which is the deferred weight-gradient split of the zero-bubble schedule
// (reference: src/wantrain/model/wgrad.py:193-249, where the same three
// products run through cuBLAS).
//
// Structure: a persistent kernel, one CTA per SM, 6 warps.
//   warp 0      TMA producer: 128B-swizzled boxes of A and B into a ring of
//               shared-memory stages (local memory only, no broadcast).
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=16) and commits to mbarriers.
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (each warp owns
//               32 TMEM lanes = 32 rows), fused math, stores to global.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1.
//
// A second kernel runs the same GEMM on pairs of SMs (tcgen05 cta_group::2,
// 256-row tiles, see gemm_pair_kernel); the launcher picks single or pair
// tiles per shape with a wave model (measured on B200: the pair tiles are
// 6-19% faster on the forward and weight-gradient shapes of the 15.8B layer).
//
// Determinism: each output tile is produced by exactly one CTA (or CTA pair)
// with a fixed k order, so results do not depend on the grid size or on
// scheduling; a given shape always takes the same kernel and tile width.
#include "common.cuh"
#include "gemm.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace ewb {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kGroupM = 16;

// Epilogues whose output leaves through shared memory and TMA (bf16 / fp32
// stores, fp32 reduce-add); the others store from registers.
template <int EPI>
struct EpiTraits {
  static constexpr bool kTma = (EPI == kEpiBf16 || EPI == kEpiF32 || EPI == kEpiAccF32);
  // shared-memory staging: TMA epilogues, and the peer scatter (rows regrouped
  // so each warp stores whole 128-byte row segments)
  static constexpr bool kStage = kTma || EPI == kEpiAccF32Peer;
};

// Tile widths: 256 (the default), 192 (an output 5120 wide splits into 27
// tiles of 192 per 128 rows, so a 2048-row GEMM fills 3 waves of 148 SMs at 97%
// instead of 72% with 256-wide tiles) and 128.
template <int BN, int EPI>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // Two 16 KB staging buffers for the TMA epilogues. (Four buffers with three
  // operand stages made the 256-wide gradient fold slower: 0.409 vs 0.372 ms.)
  static constexpr int OUT_BUFS = EpiTraits<EPI>::kStage ? 2 : 0;
  static constexpr int OUT_BYTES = OUT_BUFS * 16384;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 192) ? (EpiTraits<EPI>::kStage ? 4 : 5) : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  // two accumulators of BN columns; the allocation is a power of two
  static constexpr int TMEM_COLS = (BN == 192) ? 512 : 2 * BN;
  static_assert(SMEM <= 232448, "shared memory over the 227 KB per-CTA limit");
};

constexpr int kTileQueue = 4;  // depth of the producer -> MMA/epilogue tile-id ring

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

__device__ __forceinline__ float ld_bf16(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// Residual value (boundary format resid_fmt: bf16, fp16, or fp8 with a 1x128
// block scale) at (row, col).
__device__ __forceinline__ float resid_at(const GemmEpilogue& ep, int row, int col) {
  const size_t i = static_cast<size_t>(row) * ep.ldr + col;
  if (fmt_q8(ep.resid_fmt)) {
    const float s = ep.resid_scale[static_cast<size_t>(row) * ep.ld_resid_scale + (col >> 7)];
    return q8_value(reinterpret_cast<const uint8_t*>(ep.resid)[i], ep.resid_fmt) * s;
  }
  if (ep.resid_fmt == kFmtF16) return __half2float(reinterpret_cast<const __half*>(ep.resid)[i]);
  return ld_bf16(reinterpret_cast<const __nv_bfloat16*>(ep.resid) + i);
}

// Load 32 consecutive bf16 values of one row as fp32; vectorised (4 x 16 B)
// when the whole chunk is in range and 16-byte aligned.
__device__ __forceinline__ void load_bf16_32(const __nv_bfloat16* src, float* f, int valid) {
  if (valid >= 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = __ldg(s4 + j);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        f[8 * j + 2 * h] = __uint_as_float(u[h] << 16);
        f[8 * j + 2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = (i < valid) ? ld_bf16(src + i) : 0.f;
  }
}

// Residual values at (row, col0 .. col0 + 31) as fp32 (any boundary format; a
// 32-column chunk never straddles an fp8 scale block).
__device__ __forceinline__ void resid_32(const GemmEpilogue& ep, int row, int col0, float* f,
                                         int valid) {
  const int fmt = ep.resid_fmt;
  if (fmt == kFmtBf16) {
    load_bf16_32(reinterpret_cast<const __nv_bfloat16*>(ep.resid) + static_cast<size_t>(row) * ep.ldr +
                     col0,
                 f, valid);
    return;
  }
  const int eb = fmt_bytes(fmt);
  const uint8_t* src =
      reinterpret_cast<const uint8_t*>(ep.resid) + (static_cast<size_t>(row) * ep.ldr + col0) * eb;
  if (valid >= 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const float s = fmt_q8(fmt)
                        ? ep.resid_scale[static_cast<size_t>(row) * ep.ld_resid_scale + (col0 >> 7)]
                        : 1.f;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    if (eb == 1) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 w = __ldg(s4 + j);
        unpack8_fmt(make_uint4(w.x, w.y, 0u, 0u), fmt, s, f + 16 * j);
        unpack8_fmt(make_uint4(w.z, w.w, 0u, 0u), fmt, s, f + 16 * j + 8);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) unpack8_fmt(__ldg(s4 + j), fmt, s, f + 8 * j);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = (i < valid) ? resid_at(ep, row, col0 + i) : 0.f;
  }
}

// Store 32 consecutive fp16 values of one row (the fp16 boundary format).
__device__ __forceinline__ void store_f16_32(__half* dst, const float* f, int valid) {
  if (valid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      d4[j] = make_uint4(pack_f16x2(f[8 * j + 0], f[8 * j + 1]), pack_f16x2(f[8 * j + 2], f[8 * j + 3]),
                         pack_f16x2(f[8 * j + 4], f[8 * j + 5]), pack_f16x2(f[8 * j + 6], f[8 * j + 7]));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = __float2half_rn(f[i]);
  }
}

// Store 32 consecutive bf16 values of one row; vectorised when the whole chunk
// is in range and 16-byte aligned.
__device__ __forceinline__ void store_bf16_32(__nv_bfloat16* dst, const float* f, int valid) {
  if (valid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16x2(f[8 * j + 0], f[8 * j + 1]);
      w.y = pack_bf16x2(f[8 * j + 2], f[8 * j + 3]);
      w.z = pack_bf16x2(f[8 * j + 4], f[8 * j + 5]);
      w.w = pack_bf16x2(f[8 * j + 6], f[8 * j + 7]);
      d4[j] = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = __float2bfloat16_rn(f[i]);
  }
}

// Where the epilogue reads a tile's fp32 accumulator: TMEM, or, for the CTA
// that finishes a K-split tail tile, the sum of the splits' partials in split
// order (p0 + p1 + ... in that order whichever CTA finishes, so the result is
// bitwise the same run to run).
struct AccSrc {
  uint32_t taddr;   // this warp's TMEM lane quarter of the accumulator
  const float* ws;  // the tile's first partial ([kBM][BN] fp32), or nullptr
  int ns;           // number of partials
  int row;          // this thread's row of the tile
};

template <int BN>
__device__ __forceinline__ void acc_ld32(const AccSrc& a, int c, float* f) {
  if (a.ws == nullptr) {
    uint32_t v[32];
    tmem_ld32(a.taddr + c, v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
    return;
  }
  const float4* p = reinterpret_cast<const float4*>(a.ws + static_cast<size_t>(a.row) * BN + c);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 x = __ldcg(p + j);
    f[4 * j] = x.x;
    f[4 * j + 1] = x.y;
    f[4 * j + 2] = x.z;
    f[4 * j + 3] = x.w;
  }
#pragma unroll 1
  for (int k = 1; k < a.ns; ++k) {
    p += kBM * BN / 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 x = __ldcg(p + j);
      f[4 * j] += x.x;
      f[4 * j + 1] += x.y;
      f[4 * j + 2] += x.z;
      f[4 * j + 3] += x.w;
    }
  }
}

// A K-split tail unit's partial: this thread's accumulator row -> slot[row][*].
template <int BN>
__device__ __forceinline__ void write_partial(uint32_t taddr, float* slot, int row) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t v[32];
    tmem_ld32(taddr + c, v);
    tmem_wait_ld();
    float4* d = reinterpret_cast<float4*>(slot + static_cast<size_t>(row) * BN + c);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcg(d + j, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
  }
}

// Work units: tiles [0, full) whole, then each tail tile in `ns` K-splits.
struct Unit {
  int tile, split, ns, kb0, kb1;
};

__device__ __forceinline__ Unit decode_unit(int u, int full, int ns, int kblocks) {
  if (u < full) return {u, 0, 1, 0, kblocks};
  const int v = u - full;
  const int sp = v % ns;
  return {full + v / ns, sp, ns, sp * kblocks / ns, (sp + 1) * kblocks / ns};
}

// Register epilogues (everything but the TMA-staged kinds). `taddr` is this
// warp's TMEM lane quarter of the accumulator; `gm` this thread's row.
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile_regs(const AccSrc& acc, int gm, int nbase, int M, int N,
                                                   const GemmEpilogue& ep) {
  const bool row_ok = gm < M;
  if constexpr (EPI == kEpiLse) {
    // Fused head + cross-entropy, first half: this row's part of one 256-wide
    // vocabulary tile. Two passes over TMEM: the tile max m, then e = exp(x - m)
    // stored as fp16 (the finalize kernel turns it into the gradient in place)
    // and summed in column order; (m, sum) goes to the partials, and the tile
    // that holds the row's target also records the target's fp32 logit.
    // Every lane runs both passes (tcgen05.ld is warp-collective); a row past
    // M only skips its stores.
    const long long tgt = row_ok ? ep.targets[gm] : -1;
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float f[32];
      acc_ld32<BN>(acc, c, f);
      const int n0 = nbase + c;
      const int valid = (row_ok && n0 < N) ? min(32, N - n0) : 0;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i < valid) mx = fmaxf(mx, f[i]);
        if (n0 + i == tgt && i < valid) ep.tgt_logit[gm] = f[i];
      }
    }
    float sum = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float f[32];
      acc_ld32<BN>(acc, c, f);
      const int n0 = nbase + c;
      if (!row_ok || n0 >= N) continue;
      const int valid = min(32, N - n0);
      uint32_t w[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float e0 = (2 * h < valid) ? expf(f[2 * h] - mx) : 0.f;
        const float e1 = (2 * h + 1 < valid) ? expf(f[2 * h + 1] - mx) : 0.f;
        sum += e0;
        sum += e1;
        const __half2 hv = __floats2half2_rn(e0, e1);
        w[h] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      __half* dst = reinterpret_cast<__half*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
      if (valid == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          if (2 * h < valid) dst[2 * h] = __ushort_as_half(static_cast<unsigned short>(w[h] & 0xffffu));
          if (2 * h + 1 < valid) dst[2 * h + 1] = __ushort_as_half(static_cast<unsigned short>(w[h] >> 16));
        }
      }
    }
    if (row_ok)
      reinterpret_cast<float2*>(ep.lse_part)[static_cast<size_t>(gm) * ep.ld_part + nbase / BN] =
          make_float2(mx, sum);
  } else if constexpr (EPI == kEpiResidQ8) {
    // fp8 (e4m3 or e5m2, out_fmt) with one power-of-two scale per 128 columns
    // of a row, in two passes over TMEM (amax, then quantise) so no 128-value
    // array is held.
    const int nblk = ep.ld_scale_out;
#pragma unroll 1
    for (int c = 0; c < BN; c += 128) {
      const int n0 = nbase + c;
      float amax = 0.f;
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        float v[32];
        acc_ld32<BN>(acc, c + 32 * j, v);
        if (row_ok && n0 < N) {
          float r[32];
          resid_32(ep, gm, n0 + 32 * j, r, 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int n = n0 + 32 * j + i;
            const float b = ep.bias ? ep.bias[n] : 0.f;
            amax = fmaxf(amax, fabsf(r[i] + (v[i] + b)));
          }
        }
      }
      const float scale = q8_block_scale(amax, ep.out_fmt);
      const float inv = 1.0f / scale;  // exact: scale is a power of two
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        float v[32];
        acc_ld32<BN>(acc, c + 32 * j, v);
        if (row_ok && n0 < N) {
          float r[32];
          resid_32(ep, gm, n0 + 32 * j, r, 32);
          uint32_t w[8];
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 4 * h + e;
              const int n = n0 + 32 * j + i;
              const float b = ep.bias ? ep.bias[n] : 0.f;
              y[e] = (r[i] + (v[i] + b)) * inv;
            }
            w[h] = q8x2(y[0], y[1], ep.out_fmt) | (q8x2(y[2], y[3], ep.out_fmt) << 16);
          }
          uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(ep.out) +
                                               static_cast<size_t>(gm) * ep.ldo + n0 + 32 * j);
          d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
          d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (row_ok && n0 < N) ep.scale_out[static_cast<size_t>(gm) * nblk + (n0 >> 7)] = scale;
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float f[32];
      acc_ld32<BN>(acc, c, f);
      const int n0 = nbase + c;
      if (!row_ok || n0 >= N) continue;
      const int valid = min(32, N - n0);
      if constexpr (EPI == kEpiAccF32Peer) {
        // ZeRO-1 reduce-scatter from the epilogue: this replica's final partial
        // (its earlier microbatches, already folded in `out`, plus this tile)
        // goes straight into the owning replica's slot over NVLink.
        const float* lp = reinterpret_cast<const float*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
        const PeerScatter& ps = ep.peer;
        const long long f0 = ps.flat_off + static_cast<long long>(gm) * ep.ldo + n0;
        int k = 0;
        while (k + 1 < ps.world && f0 >= ps.shard_lo[k + 1]) ++k;
        const bool one_owner = (k + 1 >= ps.world) || (f0 + valid <= ps.shard_lo[k + 1]);
        float* dst0 = ps.slots[k] + static_cast<long long>(ps.rank) * ps.slot_stride + (f0 - ps.shard_lo[k]);
        if (one_owner && valid == 32 && (reinterpret_cast<uintptr_t>(dst0) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(lp) & 15) == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 a = reinterpret_cast<const float4*>(lp)[j];
            reinterpret_cast<float4*>(dst0)[j] = make_float4(a.x + f[4 * j], a.y + f[4 * j + 1],
                                                             a.z + f[4 * j + 2], a.w + f[4 * j + 3]);
          }
        } else {
          for (int i = 0; i < valid; ++i) {
            const long long fi = f0 + i;
            while (k + 1 < ps.world && fi >= ps.shard_lo[k + 1]) ++k;
            ps.slots[k][static_cast<long long>(ps.rank) * ps.slot_stride + (fi - ps.shard_lo[k])] =
                lp[i] + f[i];
          }
        }
        continue;
      }
      if (ep.bias != nullptr && EPI != kEpiDGelu) {
        const float* bp = ep.bias + n0;
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] += (i < valid) ? bp[i] : 0.f;
      }
      if constexpr (EPI == kEpiGelu) {
        // aux keeps the bf16 pre-activation u for the backward; out = gelu(u).
        __nv_bfloat16* aux =
            reinterpret_cast<__nv_bfloat16*>(ep.aux) + static_cast<size_t>(gm) * ep.ldaux + n0;
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = bf16_round(f[i]);
        store_bf16_32(aux, f, valid);
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = gelu_erf(f[i]);
      } else if constexpr (EPI == kEpiDGelu) {
        float u[32];
        load_bf16_32(reinterpret_cast<const __nv_bfloat16*>(ep.aux) +
                         static_cast<size_t>(gm) * ep.ldaux + n0,
                     u, valid);
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = f[i] * gelu_erf_grad(u[i]);
      } else if constexpr (EPI == kEpiResid) {
        float r[32];
        resid_32(ep, gm, n0, r, valid);
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = r[i] + f[i];
        if (ep.out_fmt == kFmtF16) {
          store_f16_32(reinterpret_cast<__half*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0, f,
                       valid);
          continue;
        }
      }
      __nv_bfloat16* dst =
          reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
      store_bf16_32(dst, f, valid);
    }
  }
}

// ZeRO-1 reduce-scatter from the epilogue (kEpiAccF32Peer): this replica's
// final partial of a tile (its earlier microbatches, already folded in `out`,
// plus the accumulator) goes straight into the owning replica's slot over
// NVLink. A thread holds one accumulator row, so storing from registers
// would send 32 rows' 16-byte pieces per warp instruction; instead each warp
// parks its 32 rows x 32 columns in shared memory (rows padded to 36 floats)
// and then writes them out row segment by row segment: 8 lanes cover one
// row's 128 contiguous bytes, a warp instruction four rows, for both the
// local partial it reads and the peer slot it writes.
template <int BN>
__device__ __forceinline__ void epilogue_tile_peer(const AccSrc& acc, int row, int m0, int nbase,
                                                   int M, int N, const GemmEpilogue& ep,
                                                   uint8_t* out_smem) {
  const int warp_q = row >> 5, lane = row & 31;
  float* stage = reinterpret_cast<float*>(out_smem) + warp_q * (32 * 36);
  const PeerScatter& ps = ep.peer;
  const int sub = lane >> 3;      // which of 4 rows this lane serves per pass
  const int c4 = (lane & 7) * 4;  // its 4 columns within the 32-column chunk
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float f[32];
    acc_ld32<BN>(acc, c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(stage + lane * 36 + 4 * j) =
          make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
    __syncwarp();
    const int n = nbase + c + c4;
    // All eight rows' local-partial loads go out before any store, so their
    // latencies overlap instead of adding up pass by pass.
    float4 l4[8];
    float* dst[8];
    unsigned fast = 0u, live = 0u;
#pragma unroll
    for (int pass = 0; pass < 8; ++pass) {
      const int gm = m0 + warp_q * 32 + pass * 4 + sub;
      dst[pass] = nullptr;
      if (gm < M && n < N) {
        live |= 1u << pass;
        const float* lp = reinterpret_cast<const float*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n;
        const long long f0 = ps.flat_off + static_cast<long long>(gm) * ep.ldo + n;
        int k = 0;
        while (k + 1 < ps.world && f0 >= ps.shard_lo[k + 1]) ++k;
        const bool one_owner = (k + 1 >= ps.world) || (f0 + 4 <= ps.shard_lo[k + 1]);
        float* d = ps.slots[k] + static_cast<long long>(ps.rank) * ps.slot_stride + (f0 - ps.shard_lo[k]);
        if (one_owner && n + 4 <= N && (reinterpret_cast<uintptr_t>(d) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(lp) & 15) == 0) {
          fast |= 1u << pass;
          dst[pass] = d;
          l4[pass] = __ldcs(reinterpret_cast<const float4*>(lp));
        }
      }
    }
#pragma unroll
    for (int pass = 0; pass < 8; ++pass) {
      if (!(live & (1u << pass))) continue;
      const int lr = pass * 4 + sub;  // row within this warp's 32
      const float4 a = *reinterpret_cast<const float4*>(stage + lr * 36 + c4);
      if (fast & (1u << pass)) {
        *reinterpret_cast<float4*>(dst[pass]) =
            make_float4(l4[pass].x + a.x, l4[pass].y + a.y, l4[pass].z + a.z, l4[pass].w + a.w);
        continue;
      }
      // ragged edge or a shard boundary inside these four columns
      const int gm = m0 + warp_q * 32 + lr;
      const float* lp = reinterpret_cast<const float*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n;
      const long long f0 = ps.flat_off + static_cast<long long>(gm) * ep.ldo + n;
      const int valid = min(4, N - n);
      const float av[4] = {a.x, a.y, a.z, a.w};
      int k = 0;
      for (int q = 0; q < valid; ++q) {
        const long long fi = f0 + q;
        while (k + 1 < ps.world && fi >= ps.shard_lo[k + 1]) ++k;
        ps.slots[k][static_cast<long long>(ps.rank) * ps.slot_stride + (fi - ps.shard_lo[k])] =
            lp[q] + av[q];
      }
    }
    __syncwarp();  // the next chunk overwrites this warp's staging rows
  }
}

// TMA-staged epilogue: each 128-byte-wide column chunk of the tile (32 fp32 or
// 64 bf16 columns x 128 rows) goes TMEM -> registers -> 128B-swizzled shared
// memory -> one bulk tensor store (or fp32 reduce-add for the gradient fold).
// Two staging buffers alternate; `leader` is the one thread that issues and
// tracks the bulk groups. Each output element receives exactly one store or
// add per launch, so the fold stays deterministic.
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile_tma(const AccSrc& acc, int row, int m0, int nbase, int N,
                                                  const GemmEpilogue& ep, const CUtensorMap* tmC,
                                                  uint8_t* out_smem, bool leader, int& chunk) {
  constexpr int CW = (EPI == kEpiBf16) ? 64 : 32;
  const bool reduce = (EPI == kEpiAccF32) && ep.beta != 0.f;
#pragma unroll 1
  for (int c = 0; c < BN; c += CW) {
    float f[CW];
#pragma unroll
    for (int j = 0; j < CW / 32; ++j) acc_ld32<BN>(acc, c + 32 * j, f + 32 * j);
    const int n0 = nbase + c;
    if (EPI != kEpiAccF32 && ep.bias != nullptr) {
#pragma unroll
      for (int i = 0; i < CW; ++i) f[i] += (n0 + i < N) ? ep.bias[n0 + i] : 0.f;
    }
    constexpr int NB = GemmCfg<BN, EPI>::OUT_BUFS;
    uint8_t* buf = out_smem + (chunk % NB) * 16384;
    if (leader) bulk_wait_read<NB - 1>();  // this buffer's store from NB chunks ago has read it
    named_bar_sync(1, 128);
    uint8_t* rowp = buf + row * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 w;
      if constexpr (EPI == kEpiBf16) {
        w.x = pack_bf16x2(f[8 * j + 0], f[8 * j + 1]);
        w.y = pack_bf16x2(f[8 * j + 2], f[8 * j + 3]);
        w.z = pack_bf16x2(f[8 * j + 4], f[8 * j + 5]);
        w.w = pack_bf16x2(f[8 * j + 6], f[8 * j + 7]);
      } else {
        w.x = __float_as_uint(f[4 * j + 0]);
        w.y = __float_as_uint(f[4 * j + 1]);
        w.z = __float_as_uint(f[4 * j + 2]);
        w.w = __float_as_uint(f[4 * j + 3]);
      }
      *reinterpret_cast<uint4*>(rowp + ((j ^ (row & 7)) << 4)) = w;
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 128);
    if (leader) {
      if (reduce)
        tma_reduce_add_2d(tmC, buf, n0, m0);
      else
        tma_store_2d(tmC, buf, n0, m0);
      bulk_commit();
    }
    ++chunk;
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC,
                        const __grid_constant__ CUtensorMap tmA2,
                        const __grid_constant__ CUtensorMap tmB2, const GemmEpilogue ep, int M,
                        int N, int K, int K2, int* status, int* sched, int nfull, int ns,
                        float* ws) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* out_smem = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(out_smem + Cfg::OUT_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tq_full = drain + 1;
  uint64_t* tq_empty = tq_full + kTileQueue;
  int* tile_ring = reinterpret_cast<int*>(tq_empty + kTileQueue);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_ring + kTileQueue);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    for (int q = 0; q < kTileQueue; ++q) {
      mbar_init(&tq_full[q], 1);
      mbar_init(&tq_empty[q], 5);  // the MMA thread + the four epilogue warps
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (K2 > 0) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
    if (EpiTraits<EPI>::kTma) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // K runs over one operand pair, or over two (A2, B2 after A, B: the weight
  // gradients of two microbatches folded by one launch).
  const int kb1 = (K + kBK - 1) / kBK;
  const int kblocks = kb1 + (K2 + kBK - 1) / kBK;
  // Units: tiles [0, nfull) whole, the other tiles each as `ns` K-splits (the
  // tail of the last wave spread over all SMs; see decode_unit).
  const int num_units = nfull + (num_tiles - nfull) * ns;
  int* tail_cnt = sched + 2;

  // Tiles are claimed dynamically from sched[0]; the claimed id travels to the
  // MMA and epilogue roles through a small ring guarded by mbarriers; -1 ends.
  auto next_tile = [&](int k) -> int {
    const int q = k % kTileQueue;
    if (!mbar_wait(&tq_full[q], (k / kTileQueue) & 1, status, kStatusTimeoutSmemFull)) return -1;
    return *reinterpret_cast<volatile int*>(&tile_ring[q]);
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        int t = atomicAdd(&sched[0], 1);
        if (t >= num_units) t = -1;
        const int q = k % kTileQueue;
        if (!mbar_wait(&tq_empty[q], ((k / kTileQueue) & 1) ^ 1, status, kStatusTimeoutSmemEmpty)) {
          ok = false;
          break;
        }
        tile_ring[q] = t;
        mbar_arrive(&tq_full[q]);
        if (t < 0) break;
        const Unit un = decode_unit(t, nfull, ns, kblocks);
        int mb, nb;
        tile_coords(un.tile, num_m, num_n, mb, nb);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, status, kStatusTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          const bool seg2 = kb >= kb1;
          const CUtensorMap* mA = seg2 ? &tmA2 : &tmA;
          const CUtensorMap* mB = seg2 ? &tmB2 : &tmB;
          const int kc = (seg2 ? kb - kb1 : kb) * kBK;
          if constexpr (!A_MN) {
            tma_load_2d(sa, mA, &full[s], kc, mb * kBM, status);
          } else {
            tma_load_2d(sa, mA, &full[s], mb * kBM, kc, status);
            tma_load_2d(sa + 8192, mA, &full[s], mb * kBM + 64, kc, status);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sb, mB, &full[s], kc, nb * BN, status);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192, mB, &full[s], nb * BN + j * 64, kc, status);
          }
        }
      }
      // Drain: every stage armed above must land before this CTA may exit.
      if (!ok) {
        for (int j = 0; j < STAGES && j < it; ++j) {
          const int i2 = it - 1 - j;
          mbar_wait(&full[i2 % STAGES], (i2 / STAGES) & 1, nullptr, kStatusTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      int it = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = next_tile(k);
        mbar_arrive(&tq_empty[k % kTileQueue]);
        if (t < 0) break;
        const int b = k & 1;
        const uint32_t use = static_cast<uint32_t>(k >> 1);
        if (!mbar_wait(&tempty[b], (use & 1) ^ 1, status, kStatusTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        const Unit un = decode_unit(t, nfull, ns, kblocks);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, status, kStatusTimeoutSmemFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(b_addr + kk * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, IDESC, (kb > un.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[b]);
      }
      // Every MMA this thread issued must complete before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, kStatusTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader = (warp == 2 && lane == 0);
    int chunk = 0;
    for (int k = 0;; ++k) {
      const int t = next_tile(k);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[k % kTileQueue]);
      if (t < 0) break;
      const Unit un = decode_unit(t, nfull, ns, kblocks);
      int mb, nb;
      tile_coords(un.tile, num_m, num_n, mb, nb);
      const int b = k & 1;
      const uint32_t use = static_cast<uint32_t>(k >> 1);
      if (!mbar_wait(&tfull[b], use & 1, status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(b * BN) + (static_cast<uint32_t>(q * 32) << 16);
      AccSrc acc{taddr, nullptr, 1, row};
      if (un.ns > 1) {
        // K-split tail unit: publish the partial; the CTA whose split lands
        // last sums all of them in split order and runs the epilogue.
        const int tail = un.tile - nfull;
        float* tile_ws = ws + static_cast<size_t>(tail) * un.ns * kBM * BN;
        write_partial<BN>(taddr, tile_ws + static_cast<size_t>(un.split) * kBM * BN, row);
        __threadfence();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        named_bar_sync(2, 128);
        if (warp == 2 && lane == 0) {
          const int prev = atomicAdd(&tail_cnt[tail], 1);
          const bool last = prev == un.ns - 1;
          if (last) tail_cnt[tail] = 0;  // every split has arrived: ready for the next launch
          __threadfence();
          *reinterpret_cast<volatile int*>(last_flag) = last ? 1 : 0;
        }
        named_bar_sync(2, 128);
        const bool last = *reinterpret_cast<volatile int*>(last_flag) != 0;
        named_bar_sync(2, 128);  // the flag is read before the next unit rewrites it
        if (!last) continue;
        acc = AccSrc{0u, tile_ws, un.ns, row};
      }
      if constexpr (EPI == kEpiAccF32Peer) {
        epilogue_tile_peer<BN>(acc, row, mb * kBM, nb * BN, M, N, ep, out_smem);
      } else if constexpr (EpiTraits<EPI>::kTma) {
        epilogue_tile_tma<EPI, BN>(acc, row, mb * kBM, nb * BN, N, ep, &tmC, out_smem, leader,
                                   chunk);
      } else {
        epilogue_tile_regs<EPI, BN>(acc, mb * kBM + row, nb * BN, M, N, ep);
      }
      if (un.ns > 1) continue;  // TMEM was released above
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (EpiTraits<EPI>::kTma && leader) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  // The last CTA to finish resets the tile counter for the next launch on this
  // stream (launches on one stream are ordered, so no other CTA can still read it).
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(&sched[1], 1);
    if (done == static_cast<int>(gridDim.x) - 1) {
      sched[0] = 0;
      sched[1] = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------- CTA-pair kernel
// The same GEMM on pairs of SMs (a cluster of two CTAs, tcgen05 cta_group::2):
// one pair computes a 256 x BN tile; CTA r of the pair holds rows 128 r ..
// 128 r + 127 of the tile (its A half) and columns BN/2 r .. of B (its B half)
// in its own shared memory, and its 128 rows of the fp32 accumulator in its
// own TMEM. The leader (rank 0) issues every MMA; the hardware reads both
// CTAs' operand halves, so each SM streams 2/3 of the operand bytes per FLOP of
// the single-CTA 128 x 256 tile. Both CTAs' TMA loads complete on the leader's
// stage barrier (no broadcast: each CTA loads only its own halves); the
// leader's MMA commits release both CTAs' stages and accumulators; both CTAs'
// epilogue warps free an accumulator by arriving on the leader's barrier.
// Tiles are assigned statically (pair p takes tiles p, p + pairs, ...), so the
// two CTAs and their roles walk the same sequence without exchanging ids.
template <int BN, int EPI>
struct PairCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = (BN / 2) * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_BUFS = EpiTraits<EPI>::kStage ? 2 : 0;
  static constexpr int OUT_BYTES = OUT_BUFS * 16384;
  static constexpr int STAGES = (227 * 1024 - OUT_BYTES - 1536) / STAGE_BYTES > 8
                                    ? 8
                                    : (227 * 1024 - OUT_BYTES - 1536) / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_BYTES + 1024 + 512;
  static constexpr int TMEM_COLS = (BN == 192) ? 512 : 2 * BN;
  static_assert(SMEM <= 232448, "shared memory over the 227 KB per-CTA limit");
  static_assert(BN == 128 || BN == 192 || BN == 256, "pair tiles are 256 x {128, 192, 256}");
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmEpilogue ep, int M, int N,
                     int K, int* status, int* sched, int nfull, int ns, float* ws) {
  using Cfg = PairCfg<BN, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* out_smem = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(out_smem + Cfg::OUT_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tq_full = drain + 1;
  uint64_t* tq_empty = tq_full + kTileQueue;
  int* tile_ring = reinterpret_cast<int*>(tq_empty + kTileQueue);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_ring + kTileQueue);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* tail_cnt = sched + 2;  // arrivals per (tail tile, CTA rank)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // four epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    for (int q = 0; q < kTileQueue; ++q) {
      mbar_init(&tq_full[q], 1);
      // the leader's ring slot is free again once every reader of both CTAs
      // took the id: its MMA thread and four epilogue warps, the peer's
      // producer and four epilogue warps
      mbar_init(&tq_empty[q], 10);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EpiTraits<EPI>::kTma) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;
  // Units: tiles [0, nfull) whole, then each tail tile as `ns` K-splits (the
  // last partial wave spread over every pair; ns = 1: no split).
  const int num_units = nfull + (num_tiles - nfull) * ns;

  // Units are claimed dynamically by the leader's producer (a pair that
  // starts late takes fewer) and published to both CTAs' roles through a ring
  // in each CTA's shared memory; -1 ends.
  auto next_tile = [&](int k) -> int {
    const int q = k % kTileQueue;
    if (!mbar_wait_cluster(&tq_full[q], (k / kTileQueue) & 1, status, kStatusTimeoutSmemFull))
      return -1;
    return *reinterpret_cast<volatile int*>(&tile_ring[q]);
  };
  auto took_tile = [&](int k) {
    mbar_arrive_cluster(peer_smem(smem_u32(&tq_empty[k % kTileQueue]), 0));
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        int t;
        if (lead) {
          t = atomicAdd(&sched[0], 1);
          if (t >= num_units) t = -1;
          const int q = k % kTileQueue;
          if (!mbar_wait(&tq_empty[q], ((k / kTileQueue) & 1) ^ 1, status,
                         kStatusTimeoutSmemEmpty)) {
            ok = false;
            t = -1;
          }
          // publish to this CTA and to the peer (store, then release-arrive)
          tile_ring[q] = t;
          const uint32_t peer_slot = peer_smem(smem_u32(&tile_ring[q]), 1);
          asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_slot), "r"(t) : "memory");
          mbar_arrive(&tq_full[q]);
          mbar_arrive_cluster(peer_smem(smem_u32(&tq_full[q]), 1));
        } else {
          t = next_tile(k);
          took_tile(k);
        }
        if (t < 0) break;
        const Unit un = decode_unit(t, nfull, ns, kblocks);
        int mb, nb;
        tile_coords(un.tile, num_m, num_n, mb, nb);
        const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int n0 = nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, status, kStatusTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          // the leader's stage barrier counts both CTAs' bytes
          if (lead) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
          const uint32_t lbar = peer_smem(smem_u32(&full[s]), 0);
          const int kc = kb * kBK;
          if constexpr (!A_MN) {
            tma_load_2d_pair(sa, &tmA, lbar, kc, m0, status);
          } else {
            tma_load_2d_pair(sa, &tmA, lbar, m0, kc, status);
            tma_load_2d_pair(sa + 8192, &tmA, lbar, m0 + 64, kc, status);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(sb, &tmB, lbar, kc, n0, status);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d_pair(sb + j * 8192, &tmB, lbar, n0 + j * 64, kc, status);
          }
        }
      }
      // Drain after a failure: the stages armed last must land before exit.
      if (!ok && lead) {
        for (int j = 0; j < STAGES && j < it; ++j) {
          const int i2 = it - 1 - j;
          mbar_wait(&full[i2 % STAGES], (i2 / STAGES) & 1, nullptr, kStatusTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (lead && lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(2 * kBM, BN, A_MN, B_MN);
      int it = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = next_tile(k);
        took_tile(k);
        if (t < 0) break;
        const Unit un = decode_unit(t, nfull, ns, kblocks);
        const int b = k & 1;
        const uint32_t use = static_cast<uint32_t>(k >> 1);
        if (!mbar_wait(&tempty[b], (use & 1) ^ 1, status, kStatusTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, status, kStatusTimeoutSmemFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(b_addr + kk * 32, 16, 1024);
            umma_f16_pair(d_tmem, ad, bd, IDESC, (kb > un.kb0 || kk > 0) ? 1u : 0u);
          }
          // this stage is free again in both CTAs once these MMAs complete
          umma_commit_pair(peer_smem(smem_u32(&empty[s]), 0));
          umma_commit_pair(peer_smem(smem_u32(&empty[s]), 1));
        }
        if (ok) {
          umma_commit_pair(peer_smem(smem_u32(&tfull[b]), 0));
          umma_commit_pair(peer_smem(smem_u32(&tfull[b]), 1));
        }
      }
      umma_commit_pair(peer_smem(smem_u32(drain), 0));
      mbar_wait(drain, 0, nullptr, kStatusTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader_thread = (warp == 2 && lane == 0);
    int chunk = 0;
    for (int k = 0;; ++k) {
      const int t = next_tile(k);
      __syncwarp();
      if (lane == 0) took_tile(k);
      if (t < 0) break;
      const Unit un = decode_unit(t, nfull, ns, kblocks);
      int mb, nb;
      tile_coords(un.tile, num_m, num_n, mb, nb);
      const int b = k & 1;
      const uint32_t use = static_cast<uint32_t>(k >> 1);
      if (!mbar_wait(&tfull[b], use & 1, status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(b * BN) + (static_cast<uint32_t>(q * 32) << 16);
      AccSrc acc{taddr, nullptr, 1, row};
      if (un.ns > 1) {
        // K-split tail unit: this CTA's half-tile partial goes to the
        // workspace and the accumulator is released; the CTA whose split of
        // this half lands last sums all of them in split order and runs the
        // epilogue (the same sum whichever CTA finishes last).
        const int tail = un.tile - nfull;
        const int slot = tail * 2 + static_cast<int>(rank);
        float* tile_ws = ws + static_cast<size_t>(slot) * un.ns * kBM * BN;
        write_partial<BN>(taddr, tile_ws + static_cast<size_t>(un.split) * kBM * BN, row);
        __threadfence();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(peer_smem(smem_u32(&tempty[b]), 0));
        named_bar_sync(2, 128);
        if (warp == 2 && lane == 0) {
          const int prev = atomicAdd(&tail_cnt[slot], 1);
          const bool last = prev == un.ns - 1;
          if (last) tail_cnt[slot] = 0;  // every split arrived: ready for the next launch
          __threadfence();
          *reinterpret_cast<volatile int*>(last_flag) = last ? 1 : 0;
        }
        named_bar_sync(2, 128);
        const bool last = *reinterpret_cast<volatile int*>(last_flag) != 0;
        named_bar_sync(2, 128);  // the flag is read before the next unit rewrites it
        if (!last) continue;
        acc = AccSrc{0u, tile_ws, un.ns, row};
      }
      const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
      if constexpr (EPI == kEpiAccF32Peer) {
        epilogue_tile_peer<BN>(acc, row, m0, nb * BN, M, N, ep, out_smem);
      } else if constexpr (EpiTraits<EPI>::kTma) {
        epilogue_tile_tma<EPI, BN>(acc, row, m0, nb * BN, N, ep, &tmC, out_smem, leader_thread,
                                   chunk);
      } else {
        epilogue_tile_regs<EPI, BN>(acc, m0 + row, nb * BN, M, N, ep);
      }
      if (un.ns > 1) continue;  // the accumulator was released above
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_smem(smem_u32(&tempty[b]), 0));
    }
    if (EpiTraits<EPI>::kTma && leader_thread) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its pair may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  // The last CTA to finish resets the tile counter for the next launch on
  // this stream (launches on one stream are ordered).
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(&sched[1], 1);
    if (done == static_cast<int>(gridDim.x) - 1) {
      sched[0] = 0;
      sched[1] = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D map: `inner` contiguous elements per row, `outer` rows, row stride `ld`
// elements of `esize` bytes, 128-byte swizzle.
bool make_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
              uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(esize)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer) {
  return make_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, inner, outer, ld, box_inner,
                  box_outer);
}

int num_sms_cached() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev];
}

// Per (device, stream) state, zeroed once; each launch leaves it zeroed for
// the next launch on the same stream (launches on one stream are ordered):
// [0] next unit, [1] CTAs done, [2 ..] arrivals per K-split tail tile. Plus a
// lazily allocated workspace for the tail tiles' fp32 partials.
constexpr int kSchedSlots = 256;
constexpr int kSchedInts = 256;      // >= 2 + the most tail tiles (one per SM)
constexpr int kMaxTailUnits = 160;   // >= SMs: tail units fill at most one wave
struct StreamState {
  int* counters;
  float* ws;  // kMaxTailUnits x [kBM][256] fp32, or nullptr
};

StreamState stream_state(cudaStream_t stream, bool want_ws) {
  static std::mutex mu;
  static int* base[64] = {nullptr};
  static cudaStream_t owner[64][kSchedSlots];
  static float* wsp[64][kSchedSlots] = {{nullptr}};
  static int used[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return {nullptr, nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (base[dev] == nullptr) {
    const size_t bytes = static_cast<size_t>(kSchedSlots) * kSchedInts * sizeof(int);
    if (cudaMalloc(&base[dev], bytes) != cudaSuccess) return {nullptr, nullptr};
    if (cudaMemset(base[dev], 0, bytes) != cudaSuccess) return {nullptr, nullptr};
  }
  int i = 0;
  while (i < used[dev] && owner[dev][i] != stream) ++i;
  if (i == used[dev]) {
    if (used[dev] >= kSchedSlots) return {nullptr, nullptr};
    owner[dev][used[dev]++] = stream;
  }
  if (want_ws && wsp[dev][i] == nullptr) {
    const size_t bytes = static_cast<size_t>(kMaxTailUnits) * kBM * 256 * sizeof(float);
    if (cudaMalloc(&wsp[dev][i], bytes) != cudaSuccess) {
      cudaGetLastError();  // clear: the launch runs without K-splits
      wsp[dev][i] = nullptr;
    }
  }
  return {base[dev] + static_cast<size_t>(i) * kSchedInts, wsp[dev][i]};
}

// K-split of a grid that fills less than one wave: the `tiles` tiles split
// along K into ns = sms / tiles parts (each at least kMinSplitKb k-blocks), so
// the launch uses ns times as many SMs. Returns ns (1: no split) and the number
// of whole tiles in `full`.
//
// Only single partial waves split. Splitting the last wave of a multi-wave
// grid measured slower on B200 (qkv projection 0.254 vs 0.237 ms, logits GEMM
// 0.823 vs 0.761 ms): the dynamic tile counter already balances the CTAs to
// within one tile, and a split tile ends with the CTA that claimed its last
// split, which is one of the CTAs that finished their whole tiles last.
constexpr int kMinSplitKb = 8;
int split_plan(long tiles, int sms, int kblocks, int* full) {
  *full = static_cast<int>(tiles);
  if (tiles >= sms / 2) return 1;
  const long r = tiles;
  int ns = static_cast<int>(sms / r);
  ns = std::min(ns, kblocks / kMinSplitKb);
  ns = std::min(ns, 16);
  if (ns < 2 || r * ns > kMaxTailUnits) return 1;
  *full = static_cast<int>(tiles - r);
  return ns;
}

// K-split of the pair kernel's last partial wave: when the tiles leave a
// tail of r <= pairs / 4 tiles after their whole waves (or the whole grid is
// that small), each tail tile splits along K into ns = pairs / r parts, so the
// tail takes about 1 / ns of a tile instead of a whole tile while most pairs
// idle. A 2048 x 5120 output is 160 pair tiles of 256 x 256: two waves of 74
// pairs and a tail of 12 tiles, which would otherwise hold the launch for a
// third tile time (72 % of the machine busy). The whole tiles are claimed
// first, so the split units start when every pair finishes its whole tiles.
// Returns ns (1: no split) and the number of whole tiles in `full`.
//
// Off unless EWB_GEMM_PAIR_SPLIT=1: measured on B200 it made the launches it
// touched slower (5120-wide projection 0.162 vs 0.098 ms, qkv weight
// gradient 0.397 vs 0.272 ms). Each thread writes and re-reads its whole
// accumulator row of every partial (1 KB strided rows, uncoalesced), and the
// last arrival's fixup sits on the launch's critical path.
int& pair_split_flag() {
  static int on = [] {
    const char* e = std::getenv("EWB_GEMM_PAIR_SPLIT");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  return on;
}
bool pair_split_enabled() { return pair_split_flag() != 0; }

int pair_split_plan(bool allow, long tiles, int pairs, int kblocks, int bn, int* full) {
  *full = static_cast<int>(tiles);
  if (!allow || !pair_split_enabled() || pairs < 2) return 1;
  const long r = tiles >= pairs ? tiles % pairs : tiles;
  if (r == 0 || 4 * r > pairs) return 1;
  int ns = static_cast<int>(pairs / r);
  ns = std::min(ns, kblocks / kMinSplitKb);
  ns = std::min(ns, 16);
  // workspace: r tiles x ns splits x 2 CTAs x [kBM][bn] fp32
  if (ns < 2 || r * ns * 2 * bn > static_cast<long>(kMaxTailUnits) * 256) return 1;
  *full = static_cast<int>(tiles - r);
  return ns;
}

// EWB_TRACE=1 prints each launch step to stderr (flushed), to localise host faults.
bool trace_on() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("EWB_TRACE");
    on = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return on == 1;
}
#define EWB_TRACE(...)                   \
  do {                                   \
    if (trace_on()) {                    \
      std::fprintf(stderr, __VA_ARGS__); \
      std::fflush(stderr);               \
    }                                    \
  } while (0)

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_cfg(const GemmArgs& g, cudaStream_t stream, int* sched, float* ws) {
  using Cfg = GemmCfg<BN, EPI>;
  EWB_TRACE("[gemm] BN=%d a_mn=%d b_mn=%d epi=%d M=%d N=%d K=%d lda=%d ldb=%d ldo=%d smem=%d\n",
            BN, (int)A_MN, (int)B_MN, EPI, g.M, g.N, g.K, g.lda, g.ldb, g.ep.ldo, Cfg::SMEM);
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
        cudaSuccess)
      return kGemmErrLaunch;
    attr_set[dev & 63] = true;
  }
  CUtensorMap ma, mbm, mc;
  const bool ok_a = A_MN ? make_map_bf16(&ma, g.a, g.M, g.K, g.lda, 64, 64)
                         : make_map_bf16(&ma, g.a, g.K, g.M, g.lda, 64, kBM);
  const bool ok_b = B_MN ? make_map_bf16(&mbm, g.b, g.N, g.K, g.ldb, 64, 64)
                         : make_map_bf16(&mbm, g.b, g.K, g.N, g.ldb, 64, BN);
  bool ok_c = true;
  if constexpr (EPI == kEpiBf16) {
    ok_c = make_map_bf16(&mc, g.ep.out, g.N, g.M, g.ep.ldo, 64, kBM);
  } else if constexpr (EPI == kEpiF32 || EPI == kEpiAccF32) {
    ok_c = make_map(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.ep.out, g.N, g.M, g.ep.ldo, 32, kBM);
  } else {
    mc = ma;  // unused by register epilogues
  }
  CUtensorMap ma2 = ma, mb2 = mbm;
  if (g.K2 > 0) {
    const bool ok_a2 = A_MN ? make_map_bf16(&ma2, g.a2, g.M, g.K2, g.lda2, 64, 64)
                            : make_map_bf16(&ma2, g.a2, g.K2, g.M, g.lda2, 64, kBM);
    const bool ok_b2 = B_MN ? make_map_bf16(&mb2, g.b2, g.N, g.K2, g.ldb2, 64, 64)
                            : make_map_bf16(&mb2, g.b2, g.K2, g.N, g.ldb2, 64, BN);
    if (!ok_a2 || !ok_b2) return kGemmErrTensorMap;
  }
  if (!ok_a || !ok_b || !ok_c) return kGemmErrTensorMap;
  const int sms = num_sms_cached();
  const long tiles = static_cast<long>((g.M + kBM - 1) / kBM) * ((g.N + BN - 1) / BN);
  int full = static_cast<int>(tiles);
  const int kbt = (g.K + kBK - 1) / kBK + (g.K2 + kBK - 1) / kBK;
  const int ns = (ws != nullptr && g.split) ? split_plan(tiles, sms, kbt, &full) : 1;
  const long units = full + (tiles - full) * ns;
  const int grid = static_cast<int>(std::max(1L, std::min(units, static_cast<long>(sms))));
  kern<<<grid, kThreads, Cfg::SMEM, stream>>>(ma, mbm, mc, ma2, mb2, g.ep, g.M, g.N, g.K, g.K2,
                                              g.status, sched, full, ns, ws);
  const cudaError_t err = cudaGetLastError();
  EWB_TRACE("[gemm] launched grid=%d ns=%d full=%d: %s\n", grid, ns, full, cudaGetErrorString(err));
  return err == cudaSuccess ? kGemmOk : kGemmErrLaunch;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_pair(const GemmArgs& g, cudaStream_t stream) {
  using Cfg = PairCfg<BN, EPI>;
  auto kern = gemm_pair_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
        cudaSuccess)
      return kGemmErrLaunch;
    attr_set[dev & 63] = true;
  }
  CUtensorMap ma, mbm, mc;
  const bool ok_a = A_MN ? make_map_bf16(&ma, g.a, g.M, g.K, g.lda, 64, 64)
                         : make_map_bf16(&ma, g.a, g.K, g.M, g.lda, 64, kBM);
  const bool ok_b = B_MN ? make_map_bf16(&mbm, g.b, g.N, g.K, g.ldb, 64, 64)
                         : make_map_bf16(&mbm, g.b, g.K, g.N, g.ldb, 64, BN / 2);
  bool ok_c = true;
  if constexpr (EPI == kEpiBf16) {
    ok_c = make_map_bf16(&mc, g.ep.out, g.N, g.M, g.ep.ldo, 64, kBM);
  } else if constexpr (EPI == kEpiF32 || EPI == kEpiAccF32) {
    ok_c = make_map(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.ep.out, g.N, g.M, g.ep.ldo, 32, kBM);
  } else {
    mc = ma;
  }
  if (!ok_a || !ok_b || !ok_c) return kGemmErrTensorMap;
  const int sms = num_sms_cached() & ~1;
  const long tiles = static_cast<long>((g.M + 2 * kBM - 1) / (2 * kBM)) * ((g.N + BN - 1) / BN);
  const int grid = static_cast<int>(std::max(2L, std::min(2 * tiles, static_cast<long>(sms))));
  EWB_TRACE("[gemm-pair] BN=%d a_mn=%d b_mn=%d epi=%d M=%d N=%d K=%d grid=%d smem=%d\n", BN,
            (int)A_MN, (int)B_MN, EPI, g.M, g.N, g.K, grid, Cfg::SMEM);
  const int kblocks = (g.K + kBK - 1) / kBK;
  int nfull = static_cast<int>(tiles);
  const int ns = pair_split_plan(g.split != 0, tiles, sms / 2, kblocks, BN, &nfull);
  const StreamState st = stream_state(stream, ns > 1);
  if (st.counters == nullptr) return kGemmErrLaunch;
  const bool split = ns > 1 && st.ws != nullptr;
  kern<<<grid, kThreads, Cfg::SMEM, stream>>>(ma, mbm, mc, g.ep, g.M, g.N, g.K, g.status,
                                              st.counters, split ? nfull : static_cast<int>(tiles),
                                              split ? ns : 1, st.ws);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kGemmOk : kGemmErrLaunch;
}

template <int BN>
int dispatch_pair(const GemmArgs& g, cudaStream_t s) {
  const int e = g.ep.kind;
  // an MN-major B half is whole 64-column swizzle panels: not with 192
  if (BN == 192 && g.b_mn) return kGemmErrUnsupported;
  if (!g.a_mn && !g.b_mn) {
    switch (e) {
      case kEpiBf16: return launch_pair<BN, false, false, kEpiBf16>(g, s);
      case kEpiGelu: return launch_pair<BN, false, false, kEpiGelu>(g, s);
      case kEpiResid: return launch_pair<BN, false, false, kEpiResid>(g, s);
      case kEpiResidQ8:
        if constexpr (BN == 256) return launch_pair<BN, false, false, kEpiResidQ8>(g, s);
        break;
      case kEpiF32: return launch_pair<BN, false, false, kEpiF32>(g, s);
      case kEpiLse:
        if constexpr (BN == 256) return launch_pair<BN, false, false, kEpiLse>(g, s);
        break;
      default: break;
    }
  } else if (!g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiBf16:
        if constexpr (BN != 192) return launch_pair<BN, false, true, kEpiBf16>(g, s);
        break;
      case kEpiDGelu:
        if constexpr (BN != 192) return launch_pair<BN, false, true, kEpiDGelu>(g, s);
        break;
      default: break;
    }
  } else if (g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiAccF32:
        if constexpr (BN != 192) return launch_pair<BN, true, true, kEpiAccF32>(g, s);
        break;
      case kEpiAccF32Peer:
        if constexpr (BN != 192) return launch_pair<BN, true, true, kEpiAccF32Peer>(g, s);
        break;
      default: break;
    }
  }
  return kGemmErrUnsupported;
}

template <int BN>
int dispatch_bn(const GemmArgs& g, cudaStream_t s, int* sc, float* ws) {
  const int e = g.ep.kind;
  if (!g.a_mn && !g.b_mn) {
    switch (e) {
      case kEpiBf16: return launch_cfg<BN, false, false, kEpiBf16>(g, s, sc, ws);
      case kEpiGelu: return launch_cfg<BN, false, false, kEpiGelu>(g, s, sc, ws);
      case kEpiResid: return launch_cfg<BN, false, false, kEpiResid>(g, s, sc, ws);
      case kEpiResidQ8: return launch_cfg<BN, false, false, kEpiResidQ8>(g, s, sc, ws);
      case kEpiF32: return launch_cfg<BN, false, false, kEpiF32>(g, s, sc, ws);
      case kEpiAccF32: return launch_cfg<BN, false, false, kEpiAccF32>(g, s, sc, ws);
      case kEpiLse:
        if constexpr (BN == 256) return launch_cfg<BN, false, false, kEpiLse>(g, s, sc, ws);
        break;
      default: break;
    }
  } else if (!g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiBf16: return launch_cfg<BN, false, true, kEpiBf16>(g, s, sc, ws);
      case kEpiDGelu: return launch_cfg<BN, false, true, kEpiDGelu>(g, s, sc, ws);
      case kEpiAccF32: return launch_cfg<BN, false, true, kEpiAccF32>(g, s, sc, ws);
      case kEpiF32: return launch_cfg<BN, false, true, kEpiF32>(g, s, sc, ws);
      default: break;
    }
  } else if (g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiAccF32: return launch_cfg<BN, true, true, kEpiAccF32>(g, s, sc, ws);
      case kEpiAccF32Peer: return launch_cfg<BN, true, true, kEpiAccF32Peer>(g, s, sc, ws);
      case kEpiBf16: return launch_cfg<BN, true, true, kEpiBf16>(g, s, sc, ws);
      case kEpiF32: return launch_cfg<BN, true, true, kEpiF32>(g, s, sc, ws);
      default: break;
    }
  }
  return kGemmErrUnsupported;
}

}  // namespace

int gemm_pick_bn(int M, int N, int K, bool split) {
  const int kblocks = (K + kBK - 1) / kBK;
  // Modelled time of a launch = whole waves x (time of one tile) / (the tile
  // width's tensor rate). A 128x128 tile streams as many operand bytes per FLOP
  // as the shared-memory port can feed (measured ~0.6 of the 128x256 tile's
  // rate on B200); a 128x192 tile needs 83% of the port (rate taken as 0.92).
  // The wave term is what picks 192 for the 5120-wide outputs of a 2048-row
  // microbatch (3 full waves instead of 2.16).
  const int sms = num_sms_cached();
  const long mt = (M + kBM - 1) / kBM;
  const int widths[3] = {256, 192, 128};
  const double rate[3] = {1.0, 0.82, 0.6};
  int best = 256;
  double best_t = 0.0;
  for (int i = 0; i < 3; ++i) {
    const int bn = widths[i];
    const long tiles = mt * ((N + bn - 1) / bn);
    int full = 0;
    const int ns = split ? split_plan(tiles, sms, kblocks, &full) : 1;
    // waves of whole tiles, plus 1/ns of one for a K-split last wave
    const double waves = ns > 1 ? static_cast<double>(full / sms) + 1.0 / ns + 0.05
                                : static_cast<double>((tiles + sms - 1) / sms);
    // columns computed per SM, including the padding of a partial last tile
    const double t = waves * bn / rate[i];
    if (i == 0 || t < best_t * 0.97) {
      best = bn;
      best_t = t;
    }
  }
  return best;
}

int& gemm_pair_mode() {
  static int mode = [] {
    const char* e = std::getenv("EWB_GEMM_PAIR");
    return e == nullptr ? 2 : std::atoi(e);
  }();
  return mode;
}

void set_gemm_pair_split(bool on) { pair_split_flag() = on ? 1 : 0; }

void set_gemm_pair_mode(int mode) { gemm_pair_mode() = mode; }

// Tile width of a CTA-pair launch (0: single-CTA tiles model faster). Same
// wave model as gemm_pick_bn: a pair tile is 256 rows and occupies two SMs;
// its rate relative to the single-CTA 128 x 256 tile is kPairRate.
constexpr double kPairRate = 1.08;
int gemm_pick_pair_bn(int M, int N, int K, int single_bn, bool split, bool b_mn) {
  const int sms = num_sms_cached();
  const int pairs = sms / 2;
  const double rate1[3] = {1.0, 0.82, 0.6};
  const int widths[3] = {256, 192, 128};
  double best1 = 0.0;
  for (int i = 0; i < 3; ++i) {
    if (widths[i] != single_bn) continue;
    const long tiles = static_cast<long>((M + kBM - 1) / kBM) * ((N + widths[i] - 1) / widths[i]);
    int full = 0;
    const int ns = split ? split_plan(tiles, sms, (K + kBK - 1) / kBK, &full) : 1;
    const double waves = ns > 1 ? static_cast<double>(full / sms) + 1.0 / ns + 0.05
                                : static_cast<double>((tiles + sms - 1) / sms);
    best1 = waves * widths[i] / rate1[i];
  }
  int best = 0;
  double best_t = best1;
  const int pw[3] = {256, 192, 128};
  const double prate[3] = {kPairRate, kPairRate * 0.92, kPairRate * 0.75};
  for (int i = 0; i < 3; ++i) {
    if (pw[i] == 192 && b_mn) continue;
    const long tiles = static_cast<long>((M + 2 * kBM - 1) / (2 * kBM)) * ((N + pw[i] - 1) / pw[i]);
    int full = 0;
    const int ns = pair_split_plan(split, tiles, pairs, (K + kBK - 1) / kBK, pw[i], &full);
    const double waves = ns > 1 ? static_cast<double>(full / pairs) + 1.0 / ns + 0.05
                                : static_cast<double>((tiles + pairs - 1) / pairs);
    // a pair tile is two single-CTA tiles of work per SM pair
    const double t = waves * pw[i] / prate[i];
    if (t < best_t * 0.97) {
      best = pw[i];
      best_t = t;
    }
  }
  return best;
}

int gemm_launch(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return kGemmErrShape;
  if ((reinterpret_cast<uintptr_t>(g.a) & 15) || (reinterpret_cast<uintptr_t>(g.b) & 15))
    return kGemmErrAlign;
  if ((g.lda % 8) || (g.ldb % 8)) return kGemmErrAlign;
  if (g.K2 < 0) return kGemmErrShape;
  if (g.K2 > 0 && ((reinterpret_cast<uintptr_t>(g.a2) & 15) ||
                   (reinterpret_cast<uintptr_t>(g.b2) & 15) || (g.lda2 % 8) || (g.ldb2 % 8)))
    return kGemmErrAlign;
  if (g.ep.kind == kEpiResidQ8 && (g.N % 128 || g.ep.ldo % 16 || !fmt_q8(g.ep.out_fmt)))
    return kGemmErrShape;
  if (g.ep.kind == kEpiResid && g.ep.out_fmt != kFmtBf16 && g.ep.out_fmt != kFmtF16) return kGemmErrShape;
  if ((g.ep.kind == kEpiResid || g.ep.kind == kEpiResidQ8) &&
      (g.ep.resid_fmt < kFmtBf16 || g.ep.resid_fmt > kFmtF16 ||
       (fmt_q8(g.ep.resid_fmt) && g.ep.resid_scale == nullptr)))
    return kGemmErrShape;
  if (reinterpret_cast<uintptr_t>(g.ep.out) & 15) return kGemmErrAlign;
  if ((g.ep.kind == kEpiBf16 && g.ep.ldo % 8) ||
      ((g.ep.kind == kEpiF32 || g.ep.kind == kEpiAccF32) && g.ep.ldo % 4))
    return kGemmErrAlign;
  int bn = g.bn;
  if (bn != 128 && bn != 192 && bn != 256) bn = gemm_pick_bn(g.M, g.N, g.K + g.K2, g.split != 0);
  if (g.ep.kind == kEpiResidQ8) bn = 256;  // a tile covers whole 128-column scale blocks
  if (g.ep.kind == kEpiLse) {
    // the partials are indexed by 256-wide vocabulary tile
    if (g.ep.targets == nullptr || g.ep.lse_part == nullptr || g.ep.tgt_logit == nullptr ||
        g.ep.ld_part < (g.N + 255) / 256 || g.ep.ldo % 8 || g.a_mn || g.b_mn)
      return kGemmErrShape;
    bn = 256;
  }
  // CTA pairs: whole operand pairs only (no second pair), tiles of 256 rows,
  // a small last wave split along K (pair_split_plan); gemm_pair_mode() 0 =
  // never, 1 = always when supported, 2 = when the wave model prefers it.
  if (g.K2 == 0 && gemm_pair_mode() != 0) {
    int pbn = 0;
    if (gemm_pair_mode() == 1) {
      pbn = (g.ep.kind == kEpiResidQ8 || g.ep.kind == kEpiLse) ? 256 : (g.N <= 128 ? 128 : 256);
    } else {
      pbn = gemm_pick_pair_bn(g.M, g.N, g.K, bn, g.split != 0, g.b_mn);
      if ((g.ep.kind == kEpiResidQ8 || g.ep.kind == kEpiLse) && pbn != 256) pbn = 0;
    }
    if (pbn == 256 || pbn == 192 || pbn == 128) {
      const int rc = pbn == 256   ? dispatch_pair<256>(g, stream)
                     : pbn == 192 ? dispatch_pair<192>(g, stream)
                                  : dispatch_pair<128>(g, stream);
      if (rc != kGemmErrUnsupported) return rc;
    }
  }
  const StreamState st = stream_state(stream, g.split != 0);
  if (st.counters == nullptr) return kGemmErrLaunch;
  if (bn == 128) return dispatch_bn<128>(g, stream, st.counters, st.ws);
  if (bn == 192) return dispatch_bn<192>(g, stream, st.counters, st.ws);
  return dispatch_bn<256>(g, stream, st.counters, st.ws);
}

// Exported for the other tcgen05 kernels (attention): a bf16 2D tensor map
// with 128-byte swizzle over [outer][ld] memory.
bool tma_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t ld, uint32_t box_inner, uint32_t box_outer) {
  return make_map_bf16(map, base, inner, outer, ld, box_inner, box_outer);
}

}  // namespace ewb
