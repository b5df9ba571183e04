// Host-visible launchers of the non-GEMM kernels. Plain C++ (no torch), so the
// same entry points serve the Python bindings and any native caller. Every
// launcher returns 0 on success, 1 for a rejected argument, 2 for a launch
// error.
#pragma once

#include "boundary.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ewb {

// ---------------------------------------------------------------- LayerNorm
struct LnArgs {
  const void* x;  // [rows][ldx] in boundary format x_fmt (BoundaryFmt)
  const float* x_scale;  // fp8 block scales [rows][ldxs]
  int x_fmt, ldx, ldxs;
  const float* gamma;
  const float* beta;
  __nv_bfloat16* y;
  int ldy;
  float* mean;
  float* rstd;
  int rows, d;
  float eps;
  int rms;  // RMSNorm: no centring, beta unused (may be null)
};
int layernorm_fwd(const LnArgs& a, cudaStream_t stream);

struct LnBwdArgs {
  const __nv_bfloat16* dy;
  int lddy;
  const void* x;
  const float* x_scale;
  int x_fmt, ldx, ldxs;
  const float* mean;
  const float* rstd;
  const float* gamma;
  const __nv_bfloat16* dres;  // optional residual-stream gradient added to dx
  int lddres;
  __nv_bfloat16* dx;
  int lddx;
  float* part_g;  // [chunks][d] scratch
  float* part_b;
  float* dgamma;  // fp32 gradients, accumulated when `accumulate`
  float* dbeta;
  int accumulate;
  int rows, d, rows_per_chunk;
  int rms;  // RMSNorm: part_b / dbeta unused (may be null)
};
int layernorm_bwd(const LnBwdArgs& a, cudaStream_t stream);
int layernorm_bwd_rows_per_chunk(int rows);

// ---------------------------------------------------------------- attention
// qkv rows are [q (H heads) | k (Hkv heads) | v (Hkv heads)], hd columns per
// head; Hkv = 0 means Hkv = H (multi-head), H % Hkv == 0 (grouped-query).
struct AttnArgs {
  const __nv_bfloat16* qkv;  // [B*S][d + 2 * Hkv * hd]
  __nv_bfloat16* o;  // [B*S][d]
  float* lse;  // [B][H][S] base-2 log-sum-exp
  int B, S, H, hd, d;
  float scale;  // softmax scale, 1/sqrt(hd)
  int Hkv;
  int* status;  // device status word of the bounded waits (may be null)
  int impl;     // 0 = best available, 1 = mma.sync kernels only
};
int attention_fwd(const AttnArgs& a, cudaStream_t stream);
// tcgen05 / TMEM / TMA forward (hd 128, S % 128 == 0); 1 = shape not supported.
int attention_fwd_tc(const AttnArgs& a, int* status, cudaStream_t stream);

struct AttnBwdArgs {
  const __nv_bfloat16* qkv;
  const __nv_bfloat16* o;
  const __nv_bfloat16* dout;
  const float* lse;
  float* Dbuf;  // [B][H][S] scratch
  __nv_bfloat16* dqkv;  // same layout as qkv
  int B, S, H, hd, d;
  float scale;
  int Hkv;
  int* status;  // device status word of the bounded waits (may be null)
  int impl;     // 0 = best available, 1 = mma.sync kernels only
};
int attention_bwd(const AttnBwdArgs& a, cudaStream_t stream);
// tcgen05 backward (hd 128, S % 128 == 0; D already in a.Dbuf); 1 = unsupported.
int attention_bwd_tc(const AttnBwdArgs& a, int* status, cudaStream_t stream);

// ---------------------------------------------------------------- cross-entropy
// Row-wise softmax cross-entropy over fp32 logits [T][ldl] (V valid columns).
// Writes loss_rows[T], and when dlogits != null the bf16 gradient
// (softmax - onehot) * grad_scale into [T][ldg] (pad columns zeroed).
struct CeArgs {
  const float* logits;
  int ldl;
  const int64_t* targets;
  int T, V;
  float* loss_rows;
  __nv_bfloat16* dlogits;
  int ldg;
  float grad_scale;
  int* status;  // device status word for the bounded waits (may be null)
};
int cross_entropy(const CeArgs& a, cudaStream_t stream);
// Second half of the fused head + cross-entropy (after the kEpiLse logits
// GEMM): per-row LSE from the 256-wide tile partials, loss rows, and the bf16
// gradient written over the fp16 exp(x - tile max) values in `buf` ([T][ld]).
int ce_lse_finalize(const float* part, int nt, int ld_part, const float* tgt_logit,
                    const int64_t* targets, int T, int V, void* buf, int ld, float grad_scale,
                    float* loss_rows, int* status, cudaStream_t stream);
// out[0] = sum(x[0..n)) / n, fixed-order tree (deterministic).
int mean_reduce(const float* x, int n, float* out, cudaStream_t stream);

// ---------------------------------------------------------------- embedding
struct EmbedArgs {
  const int64_t* idx;  // [B*S]
  const float* wte;  // [V][d] fp32 master
  const float* wpe;  // [S][d]
  int T, S, d, V;
  void* out;  // [T][d] in boundary format out_fmt (bf16, fp16, or fp8 + 1x128 scales)
  int out_fmt;
  float* out_scale;
  int* status;  // status record: a token id outside [0, V) is reported here
};
int embed_fwd(const EmbedArgs& a, cudaStream_t stream);

struct EmbedBwdArgs {
  const int64_t* idx;
  const __nv_bfloat16* dx;  // [T][d]
  int T, S, d, V;
  int* order;  // [T] scratch: positions sorted by (token, position)
  float* dwte;  // [V][d] fp32 gradient (accumulated)
  float* dwpe;  // [S][d]
  int* status;  // status record: a token id outside [0, V) is reported here
};
int embed_bwd(const EmbedBwdArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- optimizer
struct AdamWArgs {
  float* p;  // fp32 master
  float* m;
  float* v;
  const float* g;
  __nv_bfloat16* p_bf16;  // optional working copy
  int64_t n;
  float lr, beta1, beta2, eps, wd;
  float bc1, bc2;  // 1 - beta^t
};
int adamw_step(const AdamWArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- misc
// grad[n] (+)= sum_t x[t][n] in row order (bias gradients), deterministic.
int colsum_bf16(const __nv_bfloat16* x, int T, int N, int ld, float* part, float* grad,
                int accumulate, cudaStream_t stream);
int colsum_part_rows(int T);
// fp8 (fmt kFmtE4m3 / kFmtE5m2) with 1x128 power-of-two scales, standalone
// (tests, boundary tooling).
int quant_q8_rows(const __nv_bfloat16* x, int T, int d, int fmt, uint8_t* q, float* scale,
                  cudaStream_t stream);
int dequant_q8_rows(const uint8_t* q, const float* scale, int T, int d, int fmt, __nv_bfloat16* y,
                    cudaStream_t stream);
int cast_f32_bf16(const float* x, __nv_bfloat16* y, int64_t n, cudaStream_t stream);
// One bounded wait (mode 0: mbarrier phase, 1: global flag) with a caller
// limit; completes only if `release`. out[2]: {completed, waited ns}.
int wait_probe(int mode, int release, int* flag, unsigned long long limit_ns, int* status,
               long long* out, cudaStream_t stream);

// ---------------------------------------------------------------- ZeRO-1 over peer memory
int zero1_push_partials(const float* partial, const long long* ranges_dev, int nranges,
                        float* const* slots, const long long* lo, long long stride, int rank,
                        int world, long long total, cudaStream_t stream);
int zero1_fold_slots(const float* slots, long long stride, int world, long long n, float* out,
                     cudaStream_t stream);
int zero1_adamw_push(const float* master, float* m, float* v, const float* g, long long lo,
                     long long n, float* const* masters, __nv_bfloat16* const* works, int world,
                     float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                     cudaStream_t stream);

// ---------------------------------------------------------------- Llama family
// Rotary embedding, in place on columns [0, ncols) of each row (q heads then
// k heads, hd wide); row r sits at position r % S. Tables [S][hd / 2] fp32.
struct RopeArgs {
  __nv_bfloat16* x;
  int ld, rows, S, ncols, hd;
  const float* cos;
  const float* sin;
  int inverse;  // 1 = rotate back (the backward)
};
int rope_apply(const RopeArgs& a, cudaStream_t stream);

// h = silu(gu[:, :f]) * gu[:, f:2f].
struct SwigluArgs {
  const __nv_bfloat16* gu;
  int ldgu;
  __nv_bfloat16* h;
  int ldh, rows, f;
};
int swiglu_fwd(const SwigluArgs& a, cudaStream_t stream);

// dgu[:, :f] = dh * u * silu'(g), dgu[:, f:] = dh * silu(g).
struct SwigluBwdArgs {
  const __nv_bfloat16* dh;
  int lddh;
  const __nv_bfloat16* gu;
  int ldgu;
  __nv_bfloat16* dgu;
  int lddgu, rows, f;
};
int swiglu_bwd(const SwigluBwdArgs& a, cudaStream_t stream);

}  // namespace ewb
