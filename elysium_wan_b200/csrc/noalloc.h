// Allocation-free LayerNorm backward: a C entry point for callers that cannot
// allocate device memory.
//
// This entry point has no counterpart in the reference (virgiliolrf/
// elysium-wan has no native code at all); it is an addition of this library.
//
// Who needs it: callers that cannot call cudaMalloc or any allocating routine
// (torch's caching allocator included) at the point where they need the op --
// for example a framework whose own memory pool already owns the GPU's memory,
// so a fresh allocation would fail or fragment it, or a caller on a path that
// must neither fail nor wait on an allocation. They pass their own inputs and
// outputs; the per-chunk dgamma/dbeta partial sums that the regular entry
// point keeps in a caller-allocated scratch buffer live here in a fixed device
// array that the library reserves once, when it is loaded.
//
// Limits and behaviour:
//   * d (the normalised width) must be a multiple of 8 and at most
//     EWB_NOALLOC_LN_MAX_D (8192); a larger d is rejected with
//     EWB_NOALLOC_ERR_TOO_LARGE. The scratch array holds 2 x 64 x 8192 fp32
//     values (4 MiB), and every GPU that loads the library keeps it until the
//     process exits.
//   * The first call on a device looks up the array's device address (with
//     that device current) and caches it; make that first call before any
//     stream capture.
//   * Every call, on every stream, shares the one scratch array and leaves the
//     last call's partial sums in it. Each call overwrites every partial it
//     reads, so nothing needs to start at zero; calls that overlap on the GPU
//     (different streams, no ordering between them) race on the array and
//     must not be issued.
//   * dx equals the regular entry point's; dgamma / dbeta fold the rows in at
//     most 64 fixed chunks (the regular entry point uses up to 296), so their
//     last bits can differ from it while staying deterministic call to call.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum {
  EWB_NOALLOC_OK = 0,
  EWB_NOALLOC_ERR_ARGUMENT = 1,
  EWB_NOALLOC_ERR_LAUNCH = 2,
  EWB_NOALLOC_ERR_TOO_LARGE = 3,
  EWB_NOALLOC_ERR_SETUP = 4,
};

#define EWB_NOALLOC_LN_MAX_D 8192
#define EWB_NOALLOC_LN_MAX_CHUNKS 64

// dx = LayerNorm backward of dy (+ dres when non-null); dgamma / dbeta get the
// row sums of dy * xhat and dy (added to their contents when accumulate != 0).
// x_fp8 names x's format: 0 bf16, 1 e4m3 or 2 e5m2 with one fp32 scale per
// 128 columns (scales in x_scale with row stride ldxs), 3 fp16. dy, dres and dx are bf16. mean and
// rstd are the forward's per-row statistics. Leading dimensions are in
// elements. stream is a cudaStream_t (null for the legacy default stream).
// The scratch address is looked up once per device and cached; the cache does
// not survive cudaDeviceReset (call this entry point only in a context that
// has not been reset since its first call).
int ewb_layernorm_bwd_noalloc(const void* dy, int lddy, const void* x, const float* x_scale,
                              int x_fp8, int ldx, int ldxs, const float* mean, const float* rstd,
                              const float* gamma, const void* dres, int lddres, void* dx, int lddx,
                              float* dgamma, float* dbeta, int accumulate, int rows, int d,
                              void* stream);

#ifdef __cplusplus
}
#endif
