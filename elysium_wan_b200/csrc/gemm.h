// Host-visible interface of the tcgen05 GEMM (gemm.cu). Plain C++: no torch
// headers, so the launcher can be reached from any host code.
#pragma once

#include "boundary.h"

#include <cuda_runtime.h>

namespace ewb {

enum GemmEpilogueKind : int {
  kEpiBf16 = 0,     // out bf16 = acc (+ bias)
  kEpiGelu = 1,     // aux bf16 = acc + bias; out bf16 = gelu(aux)
  kEpiResid = 2,    // out bf16 / fp16 (out_fmt) = resid + acc (+ bias)  (resid: any boundary fmt)
  kEpiResidQ8 = 3,  // out e4m3 / e5m2 (out_fmt) + 1x128 scales = quant(resid + acc (+ bias))
  kEpiAccF32 = 4,   // out f32 = (beta != 0 ? out : 0) + acc     (ordered gradient fold)
  kEpiDGelu = 5,    // out bf16 = acc * gelu'(aux)
  kEpiF32 = 6,      // out f32 = acc (+ bias)
  kEpiAccF32Peer = 7,  // owner slot (peer memory) = out (local f32 partial) + acc: ZeRO-1 RS
  kEpiLse = 8,  // logits tile -> per-row (tile max, sum exp) partials, target logit,
                // out fp16 = exp(acc - tile max); the logits themselves are never stored
};

constexpr int kMaxPeers = 8;

// Where a flat parameter index lands in the ZeRO-1 owners' slot buffers:
// owner k holds flat range [shard_lo[k], shard_lo[k+1]); replica `rank`
// writes its partial at slots[k] + rank * slot_stride + (f - shard_lo[k]).
struct PeerScatter {
  float* slots[kMaxPeers];
  long long shard_lo[kMaxPeers + 1];
  long long slot_stride;
  long long flat_off;  // flat index of out[0][0]
  int rank;
  int world;
};

enum GemmStatus : int {
  kGemmOk = 0,
  kGemmErrShape = 1,
  kGemmErrAlign = 2,
  kGemmErrTensorMap = 3,
  kGemmErrLaunch = 4,
  kGemmErrUnsupported = 5,
};

struct GemmEpilogue {
  int kind;
  void* out;
  int ldo;
  const float* bias;  // fp32 [N] or null
  const void* resid;  // [M][ldr] in boundary format resid_fmt (BoundaryFmt, common.cuh)
  int ldr;
  int resid_fmt;
  const float* resid_scale;  // [M][ld_resid_scale] when resid_fmt is an fp8 format
  int out_fmt;  // kEpiResid: 0 bf16 / 3 fp16; kEpiResidQ8: 1 e4m3 / 2 e5m2
  int ld_resid_scale;
  void* aux;  // bf16 [M][ldaux]
  int ldaux;
  float* scale_out;  // [M][ld_scale_out] for kEpiResidQ8
  int ld_scale_out;
  float beta;
  PeerScatter peer;  // kEpiAccF32Peer only
  // kEpiLse only (tiles are 256 wide): targets[M] (int64), lse_part[M][ld_part]
  // float2 (tile max, sum of exp over the tile), tgt_logit[M] fp32.
  const long long* targets;
  float* lse_part;
  int ld_part;
  float* tgt_logit;
};

struct GemmArgs {
  const void* a;  // bf16
  int lda;
  bool a_mn;  // false: A stored [M][lda] (K contiguous); true: [K][lda] (M contiguous)
  const void* b;
  int ldb;
  bool b_mn;  // false: B stored [N][ldb]; true: [K][ldb]
  int M, N, K;
  int bn;  // 128 / 192 / 256, anything else = pick by the wave model
  GemmEpilogue ep;
  int* status;  // device status word (may be null)
  int split;    // nonzero: a partial single wave may be split along K
  // Optional second operand pair over K2 more reduction steps (0: none):
  // C (epi)= A B^T + A2 B2^T accumulated in one pass, same layouts as A / B.
  const void* a2;
  int lda2;
  const void* b2;
  int ldb2;
  int K2;
};

int gemm_launch(const GemmArgs& args, cudaStream_t stream);
int gemm_pick_bn(int M, int N, int K, bool split);
// CTA-pair (cta_group::2) tiles: 0 = never, 1 = whenever supported, 2 = when
// the wave model prefers them (initial value from EWB_GEMM_PAIR, default 2).
// K-split of the pair kernel's small last wave (off by default; EWB_GEMM_PAIR_SPLIT=1).
void set_gemm_pair_split(bool on);
void set_gemm_pair_mode(int mode);

// bf16 2D tensor map with 128-byte swizzle (inner = contiguous extent in
// elements, ld = row pitch in elements); false if the driver refuses it.
bool tma_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t ld, uint32_t box_inner, uint32_t box_outer);

}  // namespace ewb
