// Boundary formats: how an activation crosses an entry boundary (the input of
// every block and of the head). Plain C++ so host code can name them; the
// Python side names a format by the tensor's dtype (bf16, fp16, and e4m3 /
// e5m2 with one fp32 power-of-two scale per 128 columns of a row).
#pragma once

#ifdef __CUDACC__
#define EWB_HD __host__ __device__ __forceinline__
#else
#define EWB_HD inline
#endif

namespace ewb {

enum BoundaryFmt : int { kFmtBf16 = 0, kFmtE4m3 = 1, kFmtE5m2 = 2, kFmtF16 = 3 };

EWB_HD bool fmt_q8(int fmt) { return fmt == kFmtE4m3 || fmt == kFmtE5m2; }
EWB_HD int fmt_bytes(int fmt) { return fmt_q8(fmt) ? 1 : 2; }

}  // namespace ewb

#undef EWB_HD
