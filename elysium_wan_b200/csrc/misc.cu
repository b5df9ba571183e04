// Small deterministic helpers: bias-gradient column sums, standalone fp8
// (e4m3 / e5m2) 1x128 quantise / dequantise, fp32 -> bf16 cast.
#include "common.cuh"
#include "kernels.h"

namespace ewb {
namespace {

constexpr int kColRows = 64;  // rows per partial-sum chunk

__global__ void __launch_bounds__(256)
    colsum_part_kernel(const __nv_bfloat16* __restrict__ x, int T, int N, int ld,
                       float* __restrict__ part) {
  const int n = blockIdx.x * 256 + threadIdx.x;
  const int chunk = blockIdx.y;
  if (n >= N) return;
  const int r0 = chunk * kColRows, r1 = min(T, r0 + kColRows);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += __bfloat162float(x[static_cast<size_t>(r) * ld + n]);
  part[static_cast<size_t>(chunk) * N + n] = s;
}

__global__ void __launch_bounds__(256)
    colsum_fold_kernel(const float* __restrict__ part, int chunks, int N, float* __restrict__ grad,
                       int accumulate) {
  const int n = blockIdx.x * 256 + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += part[static_cast<size_t>(k) * N + n];
  grad[n] = accumulate ? grad[n] + s : s;
}

// One warp per 128-column block of a row.
__global__ void quant_kernel(const __nv_bfloat16* __restrict__ x, int T, int d, int fmt,
                             uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int l = threadIdx.x & 31;
  const int nb = d / 128;
  if (w >= T * nb) return;
  const int row = w / nb, blk = w % nb;
  const __nv_bfloat16* p = x + static_cast<size_t>(row) * d + blk * 128 + 4 * l;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(p[i]);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = q8_block_scale(amax, fmt);
  const float inv = 1.0f / s;
  *reinterpret_cast<uint32_t*>(q + static_cast<size_t>(row) * d + blk * 128 + 4 * l) =
      q8x2(v[0] * inv, v[1] * inv, fmt) | (q8x2(v[2] * inv, v[3] * inv, fmt) << 16);
  if (l == 0) scale[static_cast<size_t>(row) * nb + blk] = s;
}

__global__ void dequant_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                               int64_t n, int d, int fmt, __nv_bfloat16* __restrict__ y) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t row = i / d;
  const int col = static_cast<int>(i % d);
  y[i] = __float2bfloat16_rn(q8_value(q[i], fmt) * scale[row * (d / 128) + col / 128]);
}

__global__ void cast_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __float2bfloat16_rn(x[i]);
}

// The bounded waits in one launch: an mbarrier phase (mode 0) or a global
// flag (mode 1) that completes only if `release` is set, waited on with the
// caller's limit. out[0] = 1 if the wait completed, 0 if it gave up;
// out[1] = nanoseconds spent waiting.
__global__ void wait_probe_kernel(int mode, int release, int* flag, unsigned long long limit_ns,
                                  int* status, long long* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  if (release) {
    if (mode == 0) mbar_arrive(&bar);
    else atomicExch(flag, 1);
  }
  const unsigned long long t0 = globaltimer_ns();
  const bool ok = mode == 0 ? mbar_wait(&bar, 0, status, kStatusTimeoutSmemFull, limit_ns)
                            : flag_wait(flag, 1, status, kStatusTimeoutPeer, limit_ns);
  out[0] = ok ? 1 : 0;
  out[1] = static_cast<long long>(globaltimer_ns() - t0);
}

}  // namespace

int wait_probe(int mode, int release, int* flag, unsigned long long limit_ns, int* status,
               long long* out, cudaStream_t stream) {
  if (mode != 0 && mode != 1) return 1;
  wait_probe_kernel<<<1, 32, 0, stream>>>(mode, release, flag, limit_ns, status, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int colsum_part_rows(int T) { return (T + kColRows - 1) / kColRows; }

int colsum_bf16(const __nv_bfloat16* x, int T, int N, int ld, float* part, float* grad,
                int accumulate, cudaStream_t stream) {
  if (T <= 0 || N <= 0) return 1;
  const int chunks = colsum_part_rows(T);
  dim3 g1((N + 255) / 256, chunks);
  colsum_part_kernel<<<g1, 256, 0, stream>>>(x, T, N, ld, part);
  colsum_fold_kernel<<<(N + 255) / 256, 256, 0, stream>>>(part, chunks, N, grad, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int quant_q8_rows(const __nv_bfloat16* x, int T, int d, int fmt, uint8_t* q, float* scale,
                  cudaStream_t stream) {
  if (d % 128 || !fmt_q8(fmt)) return 1;
  const int warps = T * (d / 128);
  quant_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(x, T, d, fmt, q, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int dequant_q8_rows(const uint8_t* q, const float* scale, int T, int d, int fmt, __nv_bfloat16* y,
                    cudaStream_t stream) {
  if (d % 128 || !fmt_q8(fmt)) return 1;
  const int64_t n = static_cast<int64_t>(T) * d;
  dequant_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(q, scale, n, d, fmt, y);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int cast_f32_bf16(const float* x, __nv_bfloat16* y, int64_t n, cudaStream_t stream) {
  if (n <= 0) return 0;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cast_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace ewb
