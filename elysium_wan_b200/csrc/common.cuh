// Shared device helpers for the sm_100a kernels of elysium_wan_b200.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
//   * mbarrier init / arrive / expect-tx / bounded try-wait,
//   * TMA tiled 2D loads of this GPU's own memory, one CTA's box each (no broadcast form),
//   * tcgen05 TMEM alloc / dealloc, the kind::f16 MMA with a shared-memory
//     descriptor pair, commit-to-mbarrier, and tcgen05.ld of 32 lanes x 32 bits.
//
// Every wait is bounded: after kWaitLimitNs of global time the waiter records a
// status code in a device status word (an int in global memory that the host
// reads after the step) and gives up, so a bug can never leave a GPU spinning.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "boundary.h"

namespace ewb {

// ---------------------------------------------------------------- status word
enum StatusCode : int {
  kStatusOk = 0,
  kStatusTimeoutSmemFull = 1,
  kStatusTimeoutSmemEmpty = 2,
  kStatusTimeoutTmemFull = 3,
  kStatusTimeoutTmemEmpty = 4,
  kStatusTimeoutPeer = 5,
  kStatusBadArgument = 6,
  kStatusTimeoutDrain = 7,
  kStatusBoundsCheck = 8,  // a check of a bounds-checked build (EWB_KCHECK) failed
};

// Where a check failed (the status record's site word).
enum CheckSite : int {
  kSiteNone = 0,
  kSiteEmbedToken = 1,   // a token id outside [0, V): a = position, b = id
  kSiteCeTarget = 2,     // a target outside [0, V): a = row, b = target
  kSiteTmaInnerX = 3,    // a tiled TMA load whose inner coordinate is not 16-byte aligned: a = x, b = y
};

// Two seconds: long enough for any legitimate wait inside one kernel (a GEMM
// stage or a peer flag of a collective), short enough that a wedged kernel
// returns quickly and leaves the context usable.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ bool status_failed(const int* status) {
  return status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0;
}

// The status record is 32 bytes: the status word, the failing site, and two
// 64-bit values naming the failing index (first failure wins).
__device__ __forceinline__ void record_check(int* status, int code, int site, long long a,
                                             long long b) {
  if (status != nullptr && atomicCAS(status, 0, code) == 0) {
    status[1] = site;
    reinterpret_cast<long long*>(status)[1] = a;
    reinterpret_cast<long long*>(status)[2] = b;
  }
}

// Bounds-checked builds (-DEWB_KCHECK): `ok` false records the site and the
// two values and returns false so the caller skips the access. In a regular
// build the check compiles away (always true).
#ifdef EWB_KCHECK
constexpr bool kKcheck = true;
#else
constexpr bool kKcheck = false;
#endif
__device__ __forceinline__ bool kcheck(int* status, bool ok, int site, long long a, long long b) {
  if (kKcheck && !ok) {
    record_check(status, kStatusBoundsCheck, site, a, b);
    return false;
  }
  return true;
}

// ---------------------------------------------------------------- smem / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false when the
// global-time limit (limit_ns, kWaitLimitNs unless a caller passes its own) ran
// out or another role of this launch already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (status_failed(status)) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      record_status(status, code);
      return false;
    }
  }
}

// Wait until the int at `flag` (global memory, written by another CTA, kernel
// or GPU) equals `want`, with the same bound and status record as mbar_wait.
__device__ __forceinline__ bool flag_wait(const int* flag, int want, int* status, int code,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  const volatile int* f = reinterpret_cast<const volatile int*>(flag);
  const unsigned long long t0 = globaltimer_ns();
  while (*f != want) {
    if (status_failed(status)) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      record_status(status, code);
      return false;
    }
    __nanosleep(256);
  }
  return true;
}

// ---------------------------------------------------------------- TMA (local memory only)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tiled load of one box into this CTA's shared memory; completion is
// signalled as transaction bytes on `bar`. x is the innermost coordinate.
// Every tiled load of this library reads a 2-byte map, so its inner
// coordinate x must be a multiple of 8 (16 bytes); a bounds-checked build
// records a violation (site kSiteTmaInnerX) and skips the copy, so the waiting
// consumer's bounded wait expires instead of the GPU raising an illegal
// instruction.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int* status = nullptr) {
  if (!kcheck(status, (x & 7) == 0, kSiteTmaInnerX, x, y)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk-tensor store / reduce-add of one box from this CTA's shared memory to
// global memory (tracked by bulk async-groups of the issuing thread). x is the
// innermost coordinate; out-of-range parts of the box are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src,
                                                  int x, int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N bulk groups of this thread are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], bf16/f16 inputs, one elected thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp receives
// lane (base_lane + t), columns [col, col + 16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  tmem_ld16(taddr, r);
  tmem_ld16(taddr + 16, r + 16);
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp writes lane
// (base_lane + t), columns [col, col + 16). Complete with tmem_wait_st().
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor (sm100 "version 1" layout) for a 128-byte
// swizzled operand tile. Fields: start address >> 4 in bits [0,14), leading
// byte offset >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1 in
// [46,48), base offset 0, layout type SWIZZLE_128B (=2) in [61,64).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16 with bf16 A/B and fp32 D.
// Bits: D format [4,6)=1 (f32), A format [7,10)=1 (bf16), B format [10,13)=1,
// A major [15] (0 = K-major, 1 = MN-major), B major [16], N>>3 in [17,23),
// M>>4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on two SMs computes one 256-row tile: the even CTA
// (rank 0, the leader) issues the MMAs, which read A and B halves from both
// CTAs' shared memory at the same offsets and accumulate into both CTAs' TMEM.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of both CTAs (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t peer_smem(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// One 256 x N x 16 MMA across the pair, issued by one thread of the leader.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// Arrive once on the mbarrier at shared::cluster address `bar` (this CTA's or
// the peer's) when every earlier pair MMA of this thread completes.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 2D tiled load into this CTA's shared memory whose completion (transaction
// bytes) is signalled on the leader CTA's mbarrier `leader_bar` (a
// shared::cluster address). No broadcast: each CTA loads its own half.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int x, int y,
                                                 int* status = nullptr) {
  if (!kcheck(status, (x & 7) == 0, kSiteTmaInnerX, x, y)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

// mbar_wait with cluster-scope acquire: the phase was completed by arrivals
// from the other CTA of a pair, and data it stored into this CTA's shared
// memory before arriving must be visible after the wait.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status,
                                                  int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (status_failed(status)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(status, code);
      return false;
    }
  }
}

// Arrive once on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Exact (erf) GELU and its derivative, written from the definition
// gelu(x) = x * Phi(x), Phi(x) = (1 + erf(x / sqrt 2)) / 2,
// gelu'(x) = Phi(x) + x * phi(x), phi(x) = exp(-x^2 / 2) / sqrt(2 pi).
// erff / expf are CUDA's own functions, called, not re-implemented.
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
  const float pdf = expf(-0.5f * x * x) * 0.39894228040143267794f;
  return cdf + x * pdf;
}

// fp8 e4m3 1x128 block scale: a power of two 2^(e - 8) where amax = f * 2^e,
// f in [0.5, 1) (frexp convention), so |x| / scale < 256 <= 448 (e4m3 max).
// Division and multiplication by a power of two are exact, so the only
// rounding is the e4m3 cast. amax == 0 gives scale 1.
__device__ __forceinline__ float e4m3_block_scale(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
  int e;
  frexpf(amax, &e);
  return ldexpf(1.0f, e - 8);
}

// 1x128 block scale of either fp8 format: 2^(e - 8) for e4m3 (|x| / scale <
// 256 <= 448) and 2^(e - 15) for e5m2 (|x| / scale < 32768 <= 57344).
__device__ __forceinline__ float q8_block_scale(float amax, int fmt) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
  int e;
  frexpf(amax, &e);
  return ldexpf(1.0f, e - (fmt == kFmtE5m2 ? 15 : 8));
}

// Two fp32 values (already divided by the block scale) as two fp8 bytes.
__device__ __forceinline__ uint32_t q8x2(float a, float b, int fmt) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
      make_float2(a, b), __NV_SATFINITE, fmt == kFmtE5m2 ? __NV_E5M2 : __NV_E4M3));
}

__device__ __forceinline__ float q8_value(uint8_t byte, int fmt) {
  const __half_raw h =
      __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(byte), fmt == kFmtE5m2 ? __NV_E5M2 : __NV_E4M3);
  return __half2float(__half(h));
}

// Eight boundary elements packed in 16 bytes (bf16 / fp16) or 8 bytes (fp8,
// the low half of w) as fp32; `scale` multiplies fp8 values.
__device__ __forceinline__ void unpack8_fmt(const uint4& w, int fmt, float scale, float* v) {
  if (fmt_q8(fmt)) {
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = q8_value(b[i], fmt) * scale;
  } else if (fmt == kFmtF16) {
    const __half* h = reinterpret_cast<const __half*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __half2float(h[i]);
  } else {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(u[i] << 16);
      v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace ewb
