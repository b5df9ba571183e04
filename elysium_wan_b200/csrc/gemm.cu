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
//               shared-memory stages (local memory only, no multicast).
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=16) and commits to mbarriers.
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (each warp owns
//               32 TMEM lanes = 32 rows), fused math, stores to global.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1.
//
// Determinism: each output tile is produced by exactly one CTA with a fixed
// k order, so results do not depend on the grid size or on scheduling.
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

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int TMEM_COLS = 2 * BN;
};

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

// Residual value (bf16, or fp8 e4m3 with a 1x128 block scale) at (row, col).
__device__ __forceinline__ float resid_at(const GemmEpilogue& ep, int row, int col) {
  if (ep.resid_fp8) {
    const __nv_fp8_e4m3 q =
        reinterpret_cast<const __nv_fp8_e4m3*>(ep.resid)[static_cast<size_t>(row) * ep.ldr + col];
    const float s = ep.resid_scale[static_cast<size_t>(row) * ep.ld_resid_scale + (col >> 7)];
    return static_cast<float>(q) * s;
  }
  return ld_bf16(reinterpret_cast<const __nv_bfloat16*>(ep.resid) +
                 static_cast<size_t>(row) * ep.ldr + col);
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

template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile(uint32_t taddr, int gm, int nbase, int M, int N,
                                              const GemmEpilogue& ep) {
  const bool row_ok = gm < M;
  if constexpr (EPI == kEpiResidQ8) {
    // fp8 e4m3 with one power-of-two scale per 128 columns of a row.
    const int nblk = ep.ld_scale_out;
#pragma unroll 1
    for (int c = 0; c < BN; c += 128) {
      float y[128];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t v[32];
        tmem_ld32(taddr + c + 32 * j, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) y[32 * j + i] = __uint_as_float(v[i]);
      }
      const int n0 = nbase + c;
      if (row_ok && n0 < N) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const int n = n0 + i;
          const float b = ep.bias ? ep.bias[n] : 0.f;
          y[i] = resid_at(ep, gm, n) + (y[i] + b);
          amax = fmaxf(amax, fabsf(y[i]));
        }
        const float scale = e4m3_block_scale(amax);
        const float inv = 1.0f / scale;  // exact: scale is a power of two
        uint8_t* dst = reinterpret_cast<uint8_t*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const int i = 16 * j + 4 * h;
            const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
                make_float2(y[i] * inv, y[i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
            const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
                make_float2(y[i + 2] * inv, y[i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
            w[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
          }
          d4[j] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        ep.scale_out[static_cast<size_t>(gm) * nblk + (n0 >> 7)] = scale;
      }
    }
    return;
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t v[32];
      tmem_ld32(taddr + c, v);
      tmem_wait_ld();
      const int n0 = nbase + c;
      if (!row_ok || n0 >= N) continue;
      const int valid = min(32, N - n0);
      float f[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
      if constexpr (EPI == kEpiAccF32) {
        float* dst = reinterpret_cast<float*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
        if (valid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
          float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 o = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
            if (ep.beta != 0.f) {
              const float4 p = d4[j];
              o.x = p.x + o.x;
              o.y = p.y + o.y;
              o.z = p.z + o.z;
              o.w = p.w + o.w;
            }
            d4[j] = o;
          }
        } else {
          for (int i = 0; i < valid; ++i) dst[i] = (ep.beta != 0.f) ? dst[i] + f[i] : f[i];
        }
      } else if constexpr (EPI == kEpiF32) {
        float* dst = reinterpret_cast<float*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < valid) {
            const float b = ep.bias ? ep.bias[n0 + i] : 0.f;
            dst[i] = f[i] + b;
          }
        }
      } else {
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
          const __nv_bfloat16* aux = reinterpret_cast<const __nv_bfloat16*>(ep.aux) +
                                     static_cast<size_t>(gm) * ep.ldaux + n0;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < valid) f[i] = f[i] * gelu_erf_grad(ld_bf16(aux + i));
        } else if constexpr (EPI == kEpiResid) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < valid) f[i] = resid_at(ep, gm, n0 + i) + f[i];
        }
        __nv_bfloat16* dst =
            reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<size_t>(gm) * ep.ldo + n0;
        store_bf16_32(dst, f, valid);
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmEpilogue ep, int M,
                        int N, int K, int* status) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

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
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
  const int kblocks = (K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, status, kStatusTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          if constexpr (!A_MN) {
            tma_load_2d(sa, &tmA, &full[s], kb * kBK, mb * kBM);
          } else {
            tma_load_2d(sa, &tmA, &full[s], mb * kBM, kb * kBK);
            tma_load_2d(sa + 8192, &tmA, &full[s], mb * kBM + 64, kb * kBK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sb, &tmB, &full[s], kb * kBK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192, &tmB, &full[s], nb * BN + j * 64, kb * kBK);
          }
        }
      }
      // Drain: every stage armed above must land before this CTA may exit.
      if (!ok) {
        for (int j = 0; j < STAGES && j < it; ++j) {
          const int i2 = it - 1 - j;
          mbar_wait(&full[i2 % STAGES], (i2 / STAGES) & 1, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      int it = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int b = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&tempty[b], (use & 1) ^ 1, status, kStatusTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
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
            umma_f16(d_tmem, ad, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
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
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int b = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tfull[b], use & 1, status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(b * BN) + (static_cast<uint32_t>(q * 32) << 16);
      epilogue_tile<EPI, BN>(taddr, mb * kBM + row, nb * BN, M, N, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
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

// bf16 2D map: `inner` contiguous elements per row, `outer` rows, row stride ld.
bool make_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms_cached() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev];
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
#define EWB_TRACE(...)                  \
  do {                                  \
    if (trace_on()) {                   \
      std::fprintf(stderr, __VA_ARGS__); \
      std::fflush(stderr);              \
    }                                   \
  } while (0)

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_cfg(const GemmArgs& g, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  EWB_TRACE("[gemm] BN=%d a_mn=%d b_mn=%d epi=%d M=%d N=%d K=%d lda=%d ldb=%d ldo=%d smem=%d\n",
            BN, (int)A_MN, (int)B_MN, EPI, g.M, g.N, g.K, g.lda, g.ldb, g.ep.ldo, Cfg::SMEM);
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    EWB_TRACE("[gemm] set smem attribute\n");
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
        cudaSuccess)
      return kGemmErrLaunch;
    attr_set[dev & 63] = true;
  }
  EWB_TRACE("[gemm] encode maps\n");
  CUtensorMap ma, mbm;
  const bool ok_a = A_MN ? make_map_bf16(&ma, g.a, g.M, g.K, g.lda, 64, 64)
                         : make_map_bf16(&ma, g.a, g.K, g.M, g.lda, 64, kBM);
  const bool ok_b = B_MN ? make_map_bf16(&mbm, g.b, g.N, g.K, g.ldb, 64, 64)
                         : make_map_bf16(&mbm, g.b, g.K, g.N, g.ldb, 64, BN);
  if (!ok_a || !ok_b) return kGemmErrTensorMap;
  EWB_TRACE("[gemm] maps ok\n");
  const int tiles = ((g.M + kBM - 1) / kBM) * ((g.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms_cached()));
  EWB_TRACE("[gemm] launch grid=%d\n", grid);
  kern<<<grid, kThreads, Cfg::SMEM, stream>>>(ma, mbm, g.ep, g.M, g.N, g.K, g.status);
  const cudaError_t err = cudaGetLastError();
  EWB_TRACE("[gemm] launched: %s\n", cudaGetErrorString(err));
  return err == cudaSuccess ? kGemmOk : kGemmErrLaunch;
}

template <int BN>
int dispatch_bn(const GemmArgs& g, cudaStream_t s) {
  const int e = g.ep.kind;
  if (!g.a_mn && !g.b_mn) {
    switch (e) {
      case kEpiBf16: return launch_cfg<BN, false, false, kEpiBf16>(g, s);
      case kEpiGelu: return launch_cfg<BN, false, false, kEpiGelu>(g, s);
      case kEpiResid: return launch_cfg<BN, false, false, kEpiResid>(g, s);
      case kEpiResidQ8: return launch_cfg<BN, false, false, kEpiResidQ8>(g, s);
      case kEpiF32: return launch_cfg<BN, false, false, kEpiF32>(g, s);
      case kEpiAccF32: return launch_cfg<BN, false, false, kEpiAccF32>(g, s);
      default: break;
    }
  } else if (!g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiBf16: return launch_cfg<BN, false, true, kEpiBf16>(g, s);
      case kEpiDGelu: return launch_cfg<BN, false, true, kEpiDGelu>(g, s);
      case kEpiAccF32: return launch_cfg<BN, false, true, kEpiAccF32>(g, s);
      case kEpiF32: return launch_cfg<BN, false, true, kEpiF32>(g, s);
      default: break;
    }
  } else if (g.a_mn && g.b_mn) {
    switch (e) {
      case kEpiAccF32: return launch_cfg<BN, true, true, kEpiAccF32>(g, s);
      case kEpiBf16: return launch_cfg<BN, true, true, kEpiBf16>(g, s);
      case kEpiF32: return launch_cfg<BN, true, true, kEpiF32>(g, s);
      default: break;
    }
  }
  return kGemmErrUnsupported;
}

// Fraction of the last wave of a persistent grid that has work.
double wave_efficiency(long tiles, int sms) {
  const long waves = (tiles + sms - 1) / sms;
  return static_cast<double>(tiles) / static_cast<double>(waves * sms);
}

}  // namespace

int gemm_pick_bn(int M, int N) {
  const int sms = num_sms_cached();
  const long t256 = static_cast<long>((M + kBM - 1) / kBM) * ((N + 255) / 256);
  const long t128 = static_cast<long>((M + kBM - 1) / kBM) * ((N + 127) / 128);
  // A 128x128 tile streams as many operand bytes per FLOP as the shared-memory
  // port can feed (measured ~0.6 of the 128x256 tile's rate on B200), so it
  // only wins when the 128x256 grid leaves most of the last wave idle.
  const double e256 = wave_efficiency(t256, sms) * (N >= 256 ? 1.0 : 0.5);
  const double e128 = wave_efficiency(t128, sms) * 0.6;
  return e128 > e256 ? 128 : 256;
}

int gemm_launch(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return kGemmErrShape;
  if ((reinterpret_cast<uintptr_t>(g.a) & 15) || (reinterpret_cast<uintptr_t>(g.b) & 15))
    return kGemmErrAlign;
  if ((g.lda % 8) || (g.ldb % 8)) return kGemmErrAlign;
  if (g.ep.kind == kEpiResidQ8 && (g.N % 128 || g.ep.ldo % 16)) return kGemmErrShape;
  int bn = g.bn;
  if (g.ep.kind == kEpiResidQ8) bn = 256;
  if (bn != 128 && bn != 256) bn = gemm_pick_bn(g.M, g.N);
  return bn == 128 ? dispatch_bn<128>(g, stream) : dispatch_bn<256>(g, stream);
}

}  // namespace ewb
