// Python bindings of the sm_100a kernels (module elysium_wan_b200._C).
//
// Thin: each function checks dtypes, contiguity of the innermost dimension and
// alignment, derives leading dimensions from tensor strides, launches on the
// current CUDA stream and raises on any rejected argument or launch error.
// The launch counter is how the benchmark reports how many of this library's
// kernels ran inside its timed region.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <atomic>
#include <cstdlib>
#include <string>
#include <vector>

#include "gemm.h"
#include "kernels.h"

namespace {

std::atomic<long long> g_launches{0};

void count(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// One device status word per GPU (an int in device memory): kernels that time
// out on a bounded wait record a code there; the host reads it after a step.
// EWB_ATTN_IMPL=mma forces the mma.sync attention kernels (comparisons).
int attn_impl() {
  static int v = [] {
    const char* e = std::getenv("EWB_ATTN_IMPL");
    return (e != nullptr && std::string(e) == "mma") ? 1 : 0;
  }();
  return v;
}

// K-split of a GEMM's last wave (EWB_GEMM_SPLIT=0 turns it off; settable at
// run time for A/B timing).
int& gemm_split_flag() {
  static int v = [] {
    const char* e = std::getenv("EWB_GEMM_SPLIT");
    return (e != nullptr && std::string(e) == "0") ? 0 : 1;
  }();
  return v;
}
void set_gemm_split(bool on) { gemm_split_flag() = on ? 1 : 0; }

int* status_word(int dev) {
  static int* words[64] = {nullptr};
  if (dev < 0 || dev >= 64) return nullptr;
  if (words[dev] == nullptr) {
    int* p = nullptr;
    // the 32-byte status record: status word, failing site, two 64-bit values
    TORCH_CHECK(cudaMalloc(&p, 32) == cudaSuccess, "status word allocation failed");
    TORCH_CHECK(cudaMemset(p, 0, 32) == cudaSuccess, "status word init failed");
    words[dev] = p;
  }
  return words[dev];
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void check_2d_rowmajor(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a contiguous inner dimension");
}

void ok(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }

template <typename T>
T* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// C[m, n] = sum_k A[m, k] B[n, k]; A is [M, K] (a_mn=False) or [K, M]; B is
// [N, K] (b_mn=False) or [K, N].
void gemm_impl(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor out, int64_t epi,
               c10::optional<at::Tensor> bias, c10::optional<at::Tensor> resid,
               c10::optional<at::Tensor> resid_scale, c10::optional<at::Tensor> aux,
               c10::optional<at::Tensor> scale_out, double beta, int64_t bn,
               const ewb::PeerScatter* peer, c10::optional<at::Tensor> a2 = c10::nullopt,
               c10::optional<at::Tensor> b2 = c10::nullopt);

// The boundary format a tensor's dtype names (BoundaryFmt in common.cuh).
int boundary_fmt(const at::Tensor& t, const char* what) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return ewb::kFmtBf16;
    case at::kFloat8_e4m3fn: return ewb::kFmtE4m3;
    case at::kFloat8_e5m2: return ewb::kFmtE5m2;
    case at::kHalf: return ewb::kFmtF16;
    default: TORCH_CHECK(false, what, " must be bf16, fp16, e4m3 or e5m2"); return -1;
  }
}

void gemm(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor out, int64_t epi,
          c10::optional<at::Tensor> bias, c10::optional<at::Tensor> resid,
          c10::optional<at::Tensor> resid_scale, c10::optional<at::Tensor> aux,
          c10::optional<at::Tensor> scale_out, double beta, int64_t bn) {
  gemm_impl(a, a_mn, b, b_mn, out, epi, bias, resid, resid_scale, aux, scale_out, beta, bn, nullptr);
}

// Weight gradient of two microbatches in one launch (A, B and A2, B2 both
// MN-major, [K][M] and [K][N]): out (+)= A^T B + A2^T B2, accumulated over
// K + K2 in TMEM, then one fold into out.
void gemm_pair(at::Tensor a, at::Tensor b, at::Tensor a2, at::Tensor b2, at::Tensor out,
               double beta, int64_t bn) {
  gemm_impl(a, true, b, true, out, ewb::kEpiAccF32, c10::nullopt, c10::nullopt, c10::nullopt,
            c10::nullopt, c10::nullopt, beta, bn, nullptr, a2, b2);
}

// dW GEMM whose epilogue scatters (local partial + tile) into the ZeRO-1
// owners' slots: slots = peer pointers (int64), lo = world+1 flat bounds.
// Optional a2 / b2: a second microbatch folded by the same launch.
void gemm_peer_scatter(at::Tensor a, at::Tensor b, at::Tensor out, std::vector<int64_t> slots,
                       std::vector<int64_t> lo, int64_t stride, int64_t flat_off, int64_t rank,
                       int64_t bn, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2) {
  TORCH_CHECK(slots.size() >= 1 && slots.size() <= ewb::kMaxPeers, "1..8 owners");
  TORCH_CHECK(lo.size() == slots.size() + 1, "lo must have world+1 bounds");
  ewb::PeerScatter ps{};
  for (size_t k = 0; k < slots.size(); ++k) ps.slots[k] = reinterpret_cast<float*>(slots[k]);
  for (size_t k = 0; k < lo.size(); ++k) ps.shard_lo[k] = lo[k];
  ps.slot_stride = stride;
  ps.flat_off = flat_off;
  ps.rank = static_cast<int>(rank);
  ps.world = static_cast<int>(slots.size());
  gemm_impl(a, true, b, true, out, ewb::kEpiAccF32Peer, c10::nullopt, c10::nullopt, c10::nullopt,
            c10::nullopt, c10::nullopt, 1.0, bn, &ps, a2, b2);
}

void gemm_impl(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor out, int64_t epi,
               c10::optional<at::Tensor> bias, c10::optional<at::Tensor> resid,
               c10::optional<at::Tensor> resid_scale, c10::optional<at::Tensor> aux,
               c10::optional<at::Tensor> scale_out, double beta, int64_t bn,
               const ewb::PeerScatter* peer, c10::optional<at::Tensor> a2,
               c10::optional<at::Tensor> b2) {
  check_2d_rowmajor(a, "a");
  check_2d_rowmajor(b, "b");
  check_2d_rowmajor(out, "out");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "gemm operands must be bf16");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  const int Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm K mismatch: ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm out shape mismatch");
  c10::cuda::CUDAGuard guard(a.device());
  ewb::GemmArgs g{};
  g.a = a.data_ptr();
  g.lda = a.stride(0);
  g.a_mn = a_mn;
  g.b = b.data_ptr();
  g.ldb = b.stride(0);
  g.b_mn = b_mn;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bn = bn;
  g.split = gemm_split_flag();
  if (a2.has_value() && a2->defined()) {
    TORCH_CHECK(b2.has_value() && b2->defined(), "gemm: a2 needs b2");
    check_2d_rowmajor(*a2, "a2");
    check_2d_rowmajor(*b2, "b2");
    TORCH_CHECK(a2->scalar_type() == at::kBFloat16 && b2->scalar_type() == at::kBFloat16,
                "gemm operands must be bf16");
    const int M2 = a_mn ? a2->size(1) : a2->size(0);
    const int K2 = a_mn ? a2->size(0) : a2->size(1);
    const int N2 = b_mn ? b2->size(1) : b2->size(0);
    const int K2b = b_mn ? b2->size(0) : b2->size(1);
    TORCH_CHECK(M2 == M && N2 == N && K2 == K2b, "gemm: the second pair must match M, N and its K");
    g.a2 = a2->data_ptr();
    g.lda2 = a2->stride(0);
    g.b2 = b2->data_ptr();
    g.ldb2 = b2->stride(0);
    g.K2 = K2;
  }
  g.status = status_word(a.get_device());
  ewb::GemmEpilogue& e = g.ep;
  e.kind = static_cast<int>(epi);
  e.out = out.data_ptr();
  e.ldo = out.stride(0);
  e.bias = ptr_or_null<const float>(bias);
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() >= N, "bias must be fp32 [N]");
  if (resid.has_value() && resid->defined()) {
    check_2d_rowmajor(*resid, "resid");
    e.resid = resid->data_ptr();
    e.ldr = resid->stride(0);
    e.resid_fmt = boundary_fmt(*resid, "resid");
    if (ewb::fmt_q8(e.resid_fmt)) {
      TORCH_CHECK(resid_scale.has_value() && resid_scale->defined(), "fp8 resid needs scales");
      e.resid_scale = resid_scale->data_ptr<float>();
      e.ld_resid_scale = resid_scale->stride(0);
    }
  }
  if (aux.has_value() && aux->defined()) {
    check_2d_rowmajor(*aux, "aux");
    e.aux = aux->data_ptr();
    e.ldaux = aux->stride(0);
  }
  if (scale_out.has_value() && scale_out->defined()) {
    e.scale_out = scale_out->data_ptr<float>();
    e.ld_scale_out = scale_out->stride(0);
  }
  e.beta = static_cast<float>(beta);
  if (peer != nullptr) e.peer = *peer;
  switch (e.kind) {
    case ewb::kEpiBf16:
    case ewb::kEpiGelu:
    case ewb::kEpiDGelu:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16, "out must be bf16 for this epilogue");
      break;
    case ewb::kEpiResid:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kHalf,
                  "out must be bf16 or fp16 for the residual epilogue");
      e.out_fmt = boundary_fmt(out, "out");
      break;
    case ewb::kEpiAccF32:
    case ewb::kEpiF32:
    case ewb::kEpiAccF32Peer:
      TORCH_CHECK(out.scalar_type() == at::kFloat, "out must be fp32 for this epilogue");
      break;
    case ewb::kEpiResidQ8:
      e.out_fmt = boundary_fmt(out, "out");
      TORCH_CHECK(ewb::fmt_q8(e.out_fmt), "out must be e4m3 or e5m2");
      TORCH_CHECK(e.scale_out != nullptr, "scale_out required");
      break;
    default: TORCH_CHECK(false, "unknown epilogue ", epi);
  }
  if (e.kind == ewb::kEpiGelu || e.kind == ewb::kEpiDGelu) TORCH_CHECK(e.aux, "aux required");
  if (e.kind == ewb::kEpiResid || e.kind == ewb::kEpiResidQ8) TORCH_CHECK(e.resid, "resid required");
  ok(ewb::gemm_launch(g, cur_stream()), "gemm");
  count(1);
}

// Fused head + cross-entropy, the GEMM half: logits of h [T][d] x W [V][d]
// never stored; per 256-wide vocabulary tile each row leaves (max, sum exp) in
// part [T][nt][2], the target logit in tgt_logit [T], and fp16 exp(x - tile
// max) in buf [T][ld] (a 2-byte buffer the finalize turns into the bf16
// gradient in place).
void gemm_lse(at::Tensor h, at::Tensor w, at::Tensor buf, int64_t V, at::Tensor targets,
              at::Tensor part, at::Tensor tgt_logit) {
  check_2d_rowmajor(h, "h");
  check_2d_rowmajor(w, "w");
  check_2d_rowmajor(buf, "buf");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm operands must be bf16");
  TORCH_CHECK(buf.element_size() == 2 && buf.size(0) == h.size(0) && buf.size(1) >= V,
              "buf must be a 2-byte [T][>= V] buffer");
  TORCH_CHECK(w.size(0) == V && w.size(1) == h.size(1), "w must be [V][d]");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == h.size(0), "targets int64 [T]");
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous() && part.dim() == 3 &&
                  part.size(0) == h.size(0) && part.size(1) == (V + 255) / 256 && part.size(2) == 2,
              "part must be fp32 [T][ceil(V/256)][2]");
  TORCH_CHECK(tgt_logit.scalar_type() == at::kFloat && tgt_logit.numel() == h.size(0),
              "tgt_logit fp32 [T]");
  c10::cuda::CUDAGuard guard(h.device());
  ewb::GemmArgs g{};
  g.a = h.data_ptr();
  g.lda = h.stride(0);
  g.b = w.data_ptr();
  g.ldb = w.stride(0);
  g.M = h.size(0);
  g.N = static_cast<int>(V);
  g.K = h.size(1);
  g.bn = 256;
  g.split = gemm_split_flag();
  g.status = status_word(h.get_device());
  ewb::GemmEpilogue& e = g.ep;
  e.kind = ewb::kEpiLse;
  e.out = buf.data_ptr();
  e.ldo = buf.stride(0);
  e.targets = reinterpret_cast<const long long*>(targets.data_ptr<int64_t>());
  e.lse_part = part.data_ptr<float>();
  e.ld_part = part.size(1);
  e.tgt_logit = tgt_logit.data_ptr<float>();
  ok(ewb::gemm_launch(g, cur_stream()), "gemm_lse");
  count(1);
}

void ce_lse_finalize(at::Tensor part, at::Tensor tgt_logit, at::Tensor targets, int64_t V,
                     at::Tensor buf, double grad_scale, at::Tensor loss_rows) {
  check_2d_rowmajor(buf, "buf");
  TORCH_CHECK(buf.is_contiguous() && buf.element_size() == 2, "buf: dense 2-byte [T][ld]");
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous(), "part fp32");
  c10::cuda::CUDAGuard guard(buf.device());
  ok(ewb::ce_lse_finalize(part.data_ptr<float>(), part.size(1), part.size(1),
                          tgt_logit.data_ptr<float>(), targets.data_ptr<int64_t>(), buf.size(0),
                          static_cast<int>(V), buf.data_ptr(), buf.size(1),
                          static_cast<float>(grad_scale), loss_rows.data_ptr<float>(),
                          status_word(buf.get_device()), cur_stream()),
     "ce_lse_finalize");
  count(1);
}

int64_t gemm_pick_bn(int64_t M, int64_t N, int64_t K) {
  return ewb::gemm_pick_bn(M, N, K, gemm_split_flag() != 0);
}

// beta absent = RMSNorm (no centring, no shift).
void layernorm_fwd(at::Tensor x, c10::optional<at::Tensor> x_scale, at::Tensor gamma,
                   c10::optional<at::Tensor> beta, at::Tensor y, at::Tensor mean, at::Tensor rstd,
                   double eps) {
  check_2d_rowmajor(x, "x");
  check_2d_rowmajor(y, "y");
  c10::cuda::CUDAGuard guard(x.device());
  ewb::LnArgs a{};
  a.x = x.data_ptr();
  a.x_fmt = boundary_fmt(x, "x");
  a.ldx = x.stride(0);
  if (ewb::fmt_q8(a.x_fmt)) {
    TORCH_CHECK(x_scale.has_value() && x_scale->defined(), "fp8 input needs scales");
    a.x_scale = x_scale->data_ptr<float>();
    a.ldxs = x_scale->stride(0);
  }
  a.gamma = gamma.data_ptr<float>();
  a.rms = !(beta.has_value() && beta->defined());
  a.beta = a.rms ? nullptr : beta->data_ptr<float>();
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldy = y.stride(0);
  a.mean = mean.data_ptr<float>();
  a.rstd = rstd.data_ptr<float>();
  a.rows = x.size(0);
  a.d = x.size(1);
  a.eps = static_cast<float>(eps);
  ok(ewb::layernorm_fwd(a, cur_stream()), "layernorm_fwd");
  count(1);
}

int64_t layernorm_bwd_chunks(int64_t rows) {
  const int rpc = ewb::layernorm_bwd_rows_per_chunk(rows);
  return (rows + rpc - 1) / rpc;
}

void layernorm_bwd(at::Tensor dy, at::Tensor x, c10::optional<at::Tensor> x_scale, at::Tensor mean,
                   at::Tensor rstd, at::Tensor gamma, c10::optional<at::Tensor> dres,
                   at::Tensor dx, at::Tensor part_g, c10::optional<at::Tensor> part_b,
                   at::Tensor dgamma, c10::optional<at::Tensor> dbeta, bool accumulate) {
  check_2d_rowmajor(dy, "dy");
  check_2d_rowmajor(x, "x");
  check_2d_rowmajor(dx, "dx");
  c10::cuda::CUDAGuard guard(x.device());
  ewb::LnBwdArgs a{};
  a.dy = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  a.lddy = dy.stride(0);
  a.x = x.data_ptr();
  a.x_fmt = boundary_fmt(x, "x");
  a.ldx = x.stride(0);
  if (ewb::fmt_q8(a.x_fmt)) {
    TORCH_CHECK(x_scale.has_value() && x_scale->defined(), "fp8 input needs scales");
    a.x_scale = x_scale->data_ptr<float>();
    a.ldxs = x_scale->stride(0);
  }
  a.mean = mean.data_ptr<float>();
  a.rstd = rstd.data_ptr<float>();
  a.gamma = gamma.data_ptr<float>();
  if (dres.has_value() && dres->defined()) {
    a.dres = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
    a.lddres = dres->stride(0);
  }
  a.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  a.lddx = dx.stride(0);
  a.rows = x.size(0);
  a.d = x.size(1);
  a.rows_per_chunk = ewb::layernorm_bwd_rows_per_chunk(a.rows);
  const int chunks = (a.rows + a.rows_per_chunk - 1) / a.rows_per_chunk;
  TORCH_CHECK(part_g.numel() >= static_cast<int64_t>(chunks) * a.d, "part_g too small");
  a.rms = !(dbeta.has_value() && dbeta->defined());  // no beta gradient = RMSNorm
  a.part_g = part_g.data_ptr<float>();
  a.dgamma = dgamma.data_ptr<float>();
  if (!a.rms) {
    TORCH_CHECK(part_b.has_value() &&
                    part_b->numel() >= static_cast<int64_t>(chunks) * a.d,
                "part_b too small");
    a.part_b = part_b->data_ptr<float>();
    a.dbeta = dbeta->data_ptr<float>();
  }
  a.accumulate = accumulate ? 1 : 0;
  ok(ewb::layernorm_bwd(a, cur_stream()), "layernorm_bwd");
  count(3);
}

void attention_fwd(at::Tensor qkv, at::Tensor o, at::Tensor lse, int64_t B, int64_t S, int64_t H,
                   int64_t hd, double scale, int64_t Hkv) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.is_contiguous() && o.is_contiguous() && lse.is_contiguous(), "contiguous");
  c10::cuda::CUDAGuard guard(qkv.device());
  ewb::AttnArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.B = B;
  a.S = S;
  a.H = H;
  a.hd = hd;
  a.d = H * hd;
  a.scale = static_cast<float>(scale);
  a.Hkv = static_cast<int>(Hkv);
  a.status = status_word(qkv.device().index());
  a.impl = attn_impl();
  const int64_t hkv = Hkv > 0 ? Hkv : H;
  TORCH_CHECK(qkv.numel() == B * S * (a.d + 2 * hkv * hd), "qkv shape");
  ok(ewb::attention_fwd(a, cur_stream()), "attention_fwd");
  count(1);
}

void attention_bwd(at::Tensor qkv, at::Tensor o, at::Tensor dout, at::Tensor lse, at::Tensor Dbuf,
                   at::Tensor dqkv, int64_t B, int64_t S, int64_t H, int64_t hd, double scale,
                   int64_t Hkv) {
  TORCH_CHECK(qkv.is_contiguous() && o.is_contiguous() && dout.is_contiguous() &&
                  dqkv.is_contiguous(),
              "contiguous");
  c10::cuda::CUDAGuard guard(qkv.device());
  ewb::AttnBwdArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.Dbuf = Dbuf.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.B = B;
  a.S = S;
  a.H = H;
  a.hd = hd;
  a.d = H * hd;
  a.scale = static_cast<float>(scale);
  a.Hkv = static_cast<int>(Hkv);
  a.status = status_word(qkv.device().index());
  a.impl = attn_impl();
  TORCH_CHECK(dqkv.numel() == qkv.numel(), "dqkv shape");
  ok(ewb::attention_bwd(a, cur_stream()), "attention_bwd");
  count(3);
}

void rope(at::Tensor x, int64_t S, int64_t ncols, int64_t hd, at::Tensor cos_t, at::Tensor sin_t,
          bool inverse) {
  check_2d_rowmajor(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "rope: x must be bf16");
  TORCH_CHECK(cos_t.is_cuda() && sin_t.is_cuda() && cos_t.scalar_type() == at::kFloat &&
                  cos_t.numel() >= S * (hd / 2) && sin_t.numel() >= S * (hd / 2),
              "rope: tables must be fp32 [S][hd/2] on the device");
  TORCH_CHECK(ncols <= x.size(1), "rope: ncols exceeds the row");
  c10::cuda::CUDAGuard guard(x.device());
  ewb::RopeArgs a{};
  a.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  a.ld = x.stride(0);
  a.rows = x.size(0);
  a.S = S;
  a.ncols = ncols;
  a.hd = hd;
  a.cos = cos_t.data_ptr<float>();
  a.sin = sin_t.data_ptr<float>();
  a.inverse = inverse ? 1 : 0;
  ok(ewb::rope_apply(a, cur_stream()), "rope");
  count(1);
}

void swiglu_fwd(at::Tensor gu, at::Tensor h) {
  check_2d_rowmajor(gu, "gu");
  check_2d_rowmajor(h, "h");
  TORCH_CHECK(gu.size(1) == 2 * h.size(1) && gu.size(0) == h.size(0), "swiglu shapes");
  c10::cuda::CUDAGuard guard(gu.device());
  ewb::SwigluArgs a{};
  a.gu = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr());
  a.ldgu = gu.stride(0);
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.ldh = h.stride(0);
  a.rows = h.size(0);
  a.f = h.size(1);
  ok(ewb::swiglu_fwd(a, cur_stream()), "swiglu_fwd");
  count(1);
}

void swiglu_bwd(at::Tensor dh, at::Tensor gu, at::Tensor dgu) {
  check_2d_rowmajor(dh, "dh");
  check_2d_rowmajor(gu, "gu");
  check_2d_rowmajor(dgu, "dgu");
  TORCH_CHECK(gu.sizes() == dgu.sizes() && gu.size(1) == 2 * dh.size(1), "swiglu_bwd shapes");
  c10::cuda::CUDAGuard guard(gu.device());
  ewb::SwigluBwdArgs a{};
  a.dh = reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr());
  a.lddh = dh.stride(0);
  a.gu = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr());
  a.ldgu = gu.stride(0);
  a.dgu = reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr());
  a.lddgu = dgu.stride(0);
  a.rows = dh.size(0);
  a.f = dh.size(1);
  ok(ewb::swiglu_bwd(a, cur_stream()), "swiglu_bwd");
  count(1);
}

void cross_entropy(at::Tensor logits, int64_t V, at::Tensor targets, at::Tensor loss_rows,
                   c10::optional<at::Tensor> dlogits, double grad_scale) {
  check_2d_rowmajor(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "logits fp32");
  TORCH_CHECK(targets.scalar_type() == at::kLong, "targets int64");
  c10::cuda::CUDAGuard guard(logits.device());
  ewb::CeArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ldl = logits.stride(0);
  a.targets = targets.data_ptr<int64_t>();
  a.T = logits.size(0);
  a.V = V;
  a.loss_rows = loss_rows.data_ptr<float>();
  if (dlogits.has_value() && dlogits->defined()) {
    check_2d_rowmajor(*dlogits, "dlogits");
    a.dlogits = reinterpret_cast<__nv_bfloat16*>(dlogits->data_ptr());
    a.ldg = dlogits->size(1);
    TORCH_CHECK(dlogits->stride(0) == a.ldg, "dlogits must be dense");
  }
  a.grad_scale = static_cast<float>(grad_scale);
  a.status = status_word(logits.get_device());
  ok(ewb::cross_entropy(a, cur_stream()), "cross_entropy");
  count(1);
}

void mean_reduce(at::Tensor x, at::Tensor out) {
  c10::cuda::CUDAGuard guard(x.device());
  ok(ewb::mean_reduce(x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), cur_stream()),
     "mean_reduce");
  count(1);
}

// out's dtype names the boundary format (fp8 outputs also fill out_scale).
void embed_fwd(at::Tensor idx, at::Tensor wte, c10::optional<at::Tensor> wpe, int64_t S,
               at::Tensor out, c10::optional<at::Tensor> out_scale) {
  c10::cuda::CUDAGuard guard(idx.device());
  ewb::EmbedArgs a{};
  a.idx = idx.data_ptr<int64_t>();
  a.wte = wte.data_ptr<float>();
  a.wpe = ptr_or_null<float>(wpe);
  a.T = idx.numel();
  a.S = S;
  a.d = wte.size(1);
  a.V = wte.size(0);
  a.status = status_word(idx.get_device());
  check_2d_rowmajor(out, "out");
  TORCH_CHECK(out.stride(0) == a.d, "out must be contiguous [T][d]");
  a.out = out.data_ptr();
  a.out_fmt = boundary_fmt(out, "out");
  a.out_scale = ptr_or_null<float>(out_scale);
  TORCH_CHECK(!ewb::fmt_q8(a.out_fmt) || a.out_scale != nullptr, "fp8 output needs out_scale");
  ok(ewb::embed_fwd(a, cur_stream()), "embed_fwd");
  count(1);
}

void embed_bwd(at::Tensor idx, at::Tensor dx, int64_t S, at::Tensor order, at::Tensor dwte,
               c10::optional<at::Tensor> dwpe) {
  c10::cuda::CUDAGuard guard(idx.device());
  ewb::EmbedBwdArgs a{};
  a.idx = idx.data_ptr<int64_t>();
  a.dx = reinterpret_cast<const __nv_bfloat16*>(dx.data_ptr());
  a.T = idx.numel();
  a.S = S;
  a.d = dwte.size(1);
  a.V = dwte.size(0);
  a.order = order.data_ptr<int>();
  a.dwte = dwte.data_ptr<float>();
  a.dwpe = ptr_or_null<float>(dwpe);
  a.status = status_word(idx.get_device());
  ok(ewb::embed_bwd(a, cur_stream()), "embed_bwd");
  count(3);
}

void adamw(at::Tensor p, at::Tensor m, at::Tensor v, at::Tensor g,
           c10::optional<at::Tensor> p_bf16, double lr, double b1, double b2, double eps,
           double wd, int64_t step) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat,
              "adamw state must be fp32");
  TORCH_CHECK(p.numel() == m.numel() && p.numel() == v.numel() && p.numel() == g.numel(),
              "adamw size mismatch");
  c10::cuda::CUDAGuard guard(p.device());
  ewb::AdamWArgs a{};
  a.p = p.data_ptr<float>();
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.g = g.data_ptr<float>();
  a.p_bf16 = ptr_or_null<__nv_bfloat16>(p_bf16);
  a.n = p.numel();
  a.lr = lr;
  a.beta1 = b1;
  a.beta2 = b2;
  a.eps = eps;
  a.wd = wd;
  a.bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  a.bc2 = static_cast<float>(1.0 - std::pow(b2, static_cast<double>(step)));
  ok(ewb::adamw_step(a, cur_stream()), "adamw");
  count(1);
}

int64_t colsum_chunks(int64_t T) { return ewb::colsum_part_rows(T); }

void colsum(at::Tensor x, at::Tensor part, at::Tensor grad, bool accumulate) {
  check_2d_rowmajor(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(part.numel() >= ewb::colsum_part_rows(x.size(0)) * x.size(1), "part too small");
  ok(ewb::colsum_bf16(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.size(0), x.size(1),
                      x.stride(0), part.data_ptr<float>(), grad.data_ptr<float>(),
                      accumulate ? 1 : 0, cur_stream()),
     "colsum");
  count(2);
}

// fp8 with 1x128 scales; q's dtype (e4m3 / e5m2) names the format.
void quant_q8(at::Tensor x, at::Tensor q, at::Tensor scale) {
  TORCH_CHECK(x.is_contiguous() && q.is_contiguous() && scale.is_contiguous(), "contiguous");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bf16");
  c10::cuda::CUDAGuard guard(x.device());
  ok(ewb::quant_q8_rows(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.size(0), x.size(1),
                        boundary_fmt(q, "q"), reinterpret_cast<uint8_t*>(q.data_ptr()),
                        scale.data_ptr<float>(), cur_stream()),
     "quant_q8");
  count(1);
}

void dequant_q8(at::Tensor q, at::Tensor scale, at::Tensor y) {
  TORCH_CHECK(y.is_contiguous() && q.is_contiguous() && scale.is_contiguous(), "contiguous");
  c10::cuda::CUDAGuard guard(q.device());
  ok(ewb::dequant_q8_rows(reinterpret_cast<const uint8_t*>(q.data_ptr()), scale.data_ptr<float>(),
                          q.size(0), q.size(1), boundary_fmt(q, "q"),
                          reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), cur_stream()),
     "dequant_q8");
  count(1);
}

void cast_bf16(at::Tensor x, at::Tensor y) {
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel(), "cast shapes");
  c10::cuda::CUDAGuard guard(x.device());
  ok(ewb::cast_f32_bf16(x.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
                        x.numel(), cur_stream()),
     "cast_bf16");
  count(1);
}

int64_t launch_count() { return g_launches.load(); }

// A bounded device wait that nothing releases (or that is released before it
// starts, release=true): returns {completed, waited ns}; a timeout records its
// code in the device status word and the kernel returns normally.
std::vector<int64_t> wait_probe(int64_t mode, bool release, int64_t limit_ns) {
  int dev = 0;
  cudaGetDevice(&dev);
  auto opts = at::TensorOptions().device(at::kCUDA, dev);
  at::Tensor flag = at::zeros({1}, opts.dtype(at::kInt));
  at::Tensor out = at::zeros({2}, opts.dtype(at::kLong));
  ok(ewb::wait_probe(static_cast<int>(mode), release ? 1 : 0, flag.data_ptr<int>(),
                     static_cast<unsigned long long>(limit_ns), status_word(dev),
                     reinterpret_cast<long long*>(out.data_ptr<int64_t>()), cur_stream()),
     "wait_probe");
  count(1);
  at::Tensor h = out.cpu();
  return {h[0].item<int64_t>(), h[1].item<int64_t>()};
}

void zero1_push_partials(at::Tensor partial, at::Tensor ranges, std::vector<int64_t> slots,
                         std::vector<int64_t> lo, int64_t stride, int64_t rank) {
  c10::cuda::CUDAGuard guard(partial.device());
  std::vector<float*> sp;
  for (auto s : slots) sp.push_back(reinterpret_cast<float*>(s));
  std::vector<long long> l(lo.begin(), lo.end());
  TORCH_CHECK(ranges.scalar_type() == at::kLong && ranges.is_cuda(), "ranges: int64 cuda");
  ok(ewb::zero1_push_partials(partial.data_ptr<float>(),
                              reinterpret_cast<const long long*>(ranges.data_ptr<int64_t>()),
                              ranges.numel() / 2, sp.data(), l.data(), stride, rank,
                              static_cast<int>(slots.size()), partial.numel(), cur_stream()),
     "zero1_push_partials");
  count(1);
}

void zero1_fold_slots(at::Tensor slots, int64_t stride, int64_t world, int64_t n, at::Tensor out) {
  c10::cuda::CUDAGuard guard(slots.device());
  ok(ewb::zero1_fold_slots(slots.data_ptr<float>(), stride, world, n, out.data_ptr<float>(),
                           cur_stream()),
     "zero1_fold_slots");
  count(1);
}

void zero1_adamw_push(at::Tensor master, at::Tensor m, at::Tensor v, at::Tensor g, int64_t lo,
                      int64_t n, std::vector<int64_t> masters, std::vector<int64_t> works,
                      double lr, double b1, double b2, double eps, double wd, int64_t step) {
  c10::cuda::CUDAGuard guard(master.device());
  std::vector<float*> mp;
  std::vector<__nv_bfloat16*> wp;
  for (auto x : masters) mp.push_back(reinterpret_cast<float*>(x));
  for (auto x : works) wp.push_back(reinterpret_cast<__nv_bfloat16*>(x));
  const float bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  const float bc2 = static_cast<float>(1.0 - std::pow(b2, static_cast<double>(step)));
  ok(ewb::zero1_adamw_push(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                           g.data_ptr<float>(), lo, n, mp.data(), wp.data(),
                           static_cast<int>(mp.size()), lr, b1, b2, eps, wd, bc1, bc2,
                           cur_stream()),
     "zero1_adamw_push");
  count(1);
}

// Opt-in diagnostics: print the native backtrace of a host SIGSEGV to stderr.
void segv_backtrace(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "\n[ewb] native backtrace of the fatal signal:\n";
  (void)!write(2, msg, sizeof(msg) - 1);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

void install_segv_backtrace() {
  signal(SIGSEGV, segv_backtrace);
  signal(SIGBUS, segv_backtrace);
}

// Read and clear the device status word of the current device (synchronises).
int64_t status_read_clear() {
  int dev = 0;
  cudaGetDevice(&dev);
  int* p = status_word(dev);
  int v = 0;
  TORCH_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess,
              "status read failed");
  if (v != 0) cudaMemset(p, 0, 32);
  return v;
}

// The status record of the current device without clearing it (synchronises):
// [status, site, a, b] (site and values name the first failed check).
std::vector<int64_t> status_record() {
  int dev = 0;
  cudaGetDevice(&dev);
  int* p = status_word(dev);
  int32_t w[8] = {0};
  TORCH_CHECK(cudaMemcpy(w, p, 32, cudaMemcpyDeviceToHost) == cudaSuccess, "status read failed");
  const long long* q = reinterpret_cast<const long long*>(w);
  return {w[0], w[1], q[1], q[2]};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of elysium_wan_b200";
  m.def("gemm", &gemm);
  m.def("gemm_pick_bn", &gemm_pick_bn);
  m.def("set_gemm_split", &set_gemm_split);
  m.def("set_gemm_pair", [](int64_t mode) { ewb::set_gemm_pair_mode(static_cast<int>(mode)); });
  m.def("set_gemm_pair_split", [](bool on) { ewb::set_gemm_pair_split(on); });
  m.def("gemm_peer_scatter", &gemm_peer_scatter);
  m.def("gemm_pair", &gemm_pair);
  m.def("gemm_lse", &gemm_lse);
  m.def("ce_lse_finalize", &ce_lse_finalize);
  m.def("zero1_push_partials", &zero1_push_partials);
  m.def("zero1_fold_slots", &zero1_fold_slots);
  m.def("zero1_adamw_push", &zero1_adamw_push);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd);
  m.def("layernorm_bwd_chunks", &layernorm_bwd_chunks);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_bwd", &attention_bwd);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("cross_entropy", &cross_entropy);
  m.def("mean_reduce", &mean_reduce);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("adamw", &adamw);
  m.def("colsum", &colsum);
  m.def("colsum_chunks", &colsum_chunks);
  m.def("quant_q8", &quant_q8);
  m.def("dequant_q8", &dequant_q8);
  m.def("cast_bf16", &cast_bf16);
  m.def("launch_count", &launch_count);
  m.def("install_segv_backtrace", &install_segv_backtrace);
  m.def("status_read_clear", &status_read_clear);
  m.def("status_record", &status_record);
#ifdef EWB_KCHECK
  m.attr("KCHECK") = true;
#else
  m.attr("KCHECK") = false;
#endif
  m.def("wait_probe", &wait_probe);
  m.attr("EPI_BF16") = static_cast<int>(ewb::kEpiBf16);
  m.attr("EPI_GELU") = static_cast<int>(ewb::kEpiGelu);
  m.attr("EPI_RESID") = static_cast<int>(ewb::kEpiResid);
  m.attr("EPI_RESID_Q8") = static_cast<int>(ewb::kEpiResidQ8);
  m.attr("EPI_ACC_F32") = static_cast<int>(ewb::kEpiAccF32);
  m.attr("EPI_DGELU") = static_cast<int>(ewb::kEpiDGelu);
  m.attr("EPI_F32") = static_cast<int>(ewb::kEpiF32);
  m.attr("EPI_ACC_F32_PEER") = static_cast<int>(ewb::kEpiAccF32Peer);
}
