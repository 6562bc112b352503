// Torch bindings for the sm_100a kernel library. The .cu files expose a plain C ABI (no torch
// headers, so they compile quickly and can be linked from non-torch hosts); this file adapts
// torch tensors to it and checks shapes, dtypes and alignment before any launch.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "api.h"

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_DT(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has wrong dtype")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() >= 1 && (x).stride(-1) == 1, #x " must have unit inner stride")

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Launchers return their C status code to Python (miles_b200/ops/_lib.py raises on non-zero)
// instead of throwing from C++ once CUDA calls have run.

// ------------------------------------------------------------------ GEMM
// a: stored 2-D [a_rows, a_cols]; b: stored 2-D [b_rows, b_cols]; c: output buffer (any shape,
// row stride ldc). See gemm_sm100.cu for the modes.
int64_t gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor c, int64_t M,
          int64_t N, int64_t K, int64_t mode, c10::optional<torch::Tensor> group_offsets,
          int64_t num_groups, int64_t b_rows_per_group, int64_t c_group_stride, int64_t epi,
          double alpha, int64_t bn, c10::optional<torch::Tensor> group_counts, torch::Tensor err) {
  CHECK_CUDA(a); CHECK_CUDA(b); CHECK_CUDA(c);
  CHECK_DT(a, at::kBFloat16); CHECK_DT(b, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "gemm operands must be 2-D views");
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(b); CHECK_ROWMAJOR(c);
  TORCH_CHECK((epi & 1) ? c.scalar_type() == at::kFloat : c.scalar_type() == at::kBFloat16,
              "output dtype does not match epilogue");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "operands must be 16-byte aligned");
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
  const int64_t ldc = c.dim() >= 2 ? c.stride(-2) : N;
  TORCH_CHECK(ldc % 8 == 0 || (epi & 1), "ldc must be a multiple of 8");
  const int* go = nullptr;
  if (mode != 0) {
    TORCH_CHECK(group_offsets.has_value(), "grouped modes need group_offsets");
    CHECK_DT(group_offsets.value(), at::kInt);
    go = group_offsets.value().data_ptr<int>();
  }
  c10::cuda::CUDAGuard g(a.device());
  int rc = mb_gemm_bf16(a.data_ptr(), a.size(0), a.size(1), a.stride(0), a_mn, b.data_ptr(),
                        b.size(0), b.size(1), b.stride(0), b_mn, c.data_ptr(), ldc, (int)M, (int)N,
                        (int)K, (int)mode, go, (int)num_groups, (int)b_rows_per_group,
                        c_group_stride, (int)epi, (float)alpha, (int)bn,
                        group_counts.has_value() ? group_counts.value().data_ptr<int>() : nullptr,
                        err.data_ptr<int>(), cur_stream());
  return rc;
}

// Block-scaled fp8: x bf16 [M, K] -> q (uint8 view of e4m3) [M, K], s fp32 [K/128, lds].
int64_t fp8_act_quant(torch::Tensor x, torch::Tensor q, torch::Tensor s,
                      c10::optional<torch::Tensor> offsets, c10::optional<torch::Tensor> counts) {
  CHECK_CUDA(x); CHECK_CUDA(q); CHECK_CUDA(s);
  CHECK_DT(x, at::kBFloat16); CHECK_DT(q, at::kByte); CHECK_DT(s, at::kFloat);
  TORCH_CHECK(x.dim() == 2 && q.dim() == 2 && s.dim() == 2, "fp8_act_quant operands must be 2-D");
  CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(s);
  TORCH_CHECK(q.is_contiguous(), "q must be contiguous");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(q.size(0) == M && q.size(1) == K, "q shape");
  TORCH_CHECK(K % 128 == 0 && s.size(0) == K / 128 && s.size(1) >= M, "s shape");
  TORCH_CHECK(x.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 8 == 0, "x misaligned");
  const int* op = nullptr;
  const int* cp = nullptr;
  int E = 0;
  if (offsets.has_value()) {
    CHECK_DT(offsets.value(), at::kInt);
    op = offsets.value().data_ptr<int>();
    E = (int)offsets.value().numel() - 1;
    if (counts.has_value()) {
      CHECK_DT(counts.value(), at::kInt);
      TORCH_CHECK(counts.value().numel() == E, "counts must have E entries");
      cp = counts.value().data_ptr<int>();
    }
  }
  c10::cuda::CUDAGuard g(x.device());
  return mb_fp8_act_quant(x.data_ptr(), x.stride(0), (int)M, (int)K, q.data_ptr(), s.data_ptr<float>(),
                          s.stride(0), op, cp, E, cur_stream());
}

// Block-scaled fp8 GEMM: a [a_rows, K] e4m3 (uint8) with sa [K/128, >= a_rows]; b [b_rows, K]
// with sb [b_rows/128, K/128]; c bf16. epi 0: c [M, N]; epi 4: SwiGLU, N = 2F, c [M, F],
// optional gu [M, 2F].
int64_t gemm_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb,
                 torch::Tensor c, c10::optional<torch::Tensor> gu, int64_t M, int64_t N, int64_t K,
                 int64_t mode, c10::optional<torch::Tensor> group_offsets,
                 c10::optional<torch::Tensor> group_counts, int64_t num_groups,
                 int64_t b_rows_per_group, int64_t epi, int64_t swiglu_f, int64_t bn,
                 torch::Tensor err) {
  CHECK_CUDA(a); CHECK_CUDA(b); CHECK_CUDA(c); CHECK_CUDA(sa); CHECK_CUDA(sb);
  CHECK_DT(a, at::kByte); CHECK_DT(b, at::kByte); CHECK_DT(c, at::kBFloat16);
  CHECK_DT(sa, at::kFloat); CHECK_DT(sb, at::kFloat);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_fp8 operands must be 2-D");
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(b); CHECK_ROWMAJOR(c);
  TORCH_CHECK(sa.is_contiguous() && sb.is_contiguous(), "scales must be contiguous");
  TORCH_CHECK(a.size(1) == K && b.size(1) == K && K % 128 == 0, "K mismatch / K % 128");
  TORCH_CHECK(sa.dim() == 2 && sa.size(0) == K / 128 && sa.size(1) >= std::min<int64_t>(M, a.size(0)),
              "sa shape");
  TORCH_CHECK(sb.numel() == (b.size(0) / 128) * (K / 128) && b.size(0) % 128 == 0, "sb shape");
  TORCH_CHECK(a.stride(0) % 16 == 0 && b.stride(0) % 16 == 0, "row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "operands must be 16-byte aligned");
  TORCH_CHECK(c.stride(0) % 8 == 0, "ldc must be a multiple of 8");
  TORCH_CHECK(mode == 0 ? (M <= a.size(0) && N <= b.size(0)) : (M <= a.size(0)), "M / N out of range");
  const int* go = nullptr;
  const int* gc = nullptr;
  if (mode != 0) {
    TORCH_CHECK(group_offsets.has_value(), "grouped mode needs group_offsets");
    CHECK_DT(group_offsets.value(), at::kInt);
    go = group_offsets.value().data_ptr<int>();
    TORCH_CHECK(b.size(0) == num_groups * b_rows_per_group, "b rows != groups * rows per group");
    if (group_counts.has_value()) {
      CHECK_DT(group_counts.value(), at::kInt);
      gc = group_counts.value().data_ptr<int>();
    }
  }
  void* gup = nullptr;
  int64_t ldgu = 0;
  if (gu.has_value()) {
    CHECK_CUDA(gu.value()); CHECK_DT(gu.value(), at::kBFloat16); CHECK_ROWMAJOR(gu.value());
    gup = gu.value().data_ptr();
    ldgu = gu.value().stride(0);
  }
  c10::cuda::CUDAGuard g(a.device());
  return mb_gemm_fp8(a.data_ptr(), a.size(0), a.stride(0), sa.data_ptr<float>(), sa.size(1),
                     b.data_ptr(), b.size(0), b.stride(0), sb.data_ptr<float>(), c.data_ptr(),
                     c.stride(0), (int)M, (int)N, (int)K, (int)mode, go, gc, (int)num_groups,
                     (int)b_rows_per_group, (int)epi, (int)swiglu_f, gup, ldgu, (int)bn,
                     err.data_ptr<int>(), cur_stream());
}

// out[M, F] = silu(a @ b_gate^T) * (a @ b_up^T), b: [groups * 2F, K] ([gate; up] per group);
// gu (optional) receives the [M, 2F] product.
int64_t gemm_swiglu(torch::Tensor a, torch::Tensor b, torch::Tensor out,
                    c10::optional<torch::Tensor> gu, int64_t M, int64_t F, int64_t K, int64_t mode,
                    c10::optional<torch::Tensor> group_offsets, int64_t num_groups, int64_t bn,
                    c10::optional<torch::Tensor> group_counts, torch::Tensor err) {
  CHECK_CUDA(a); CHECK_CUDA(b); CHECK_CUDA(out);
  CHECK_DT(a, at::kBFloat16); CHECK_DT(b, at::kBFloat16); CHECK_DT(out, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm_swiglu operands must be 2-D");
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(b); CHECK_ROWMAJOR(out);
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && out.stride(0) % 8 == 0,
              "row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "operands must be 16-byte aligned");
  void* gup = nullptr;
  int64_t ldgu = 0;
  if (gu.has_value()) {
    CHECK_CUDA(gu.value()); CHECK_DT(gu.value(), at::kBFloat16); CHECK_ROWMAJOR(gu.value());
    gup = gu.value().data_ptr();
    ldgu = gu.value().stride(0);
    TORCH_CHECK(ldgu % 8 == 0 && reinterpret_cast<uintptr_t>(gup) % 16 == 0, "gu misaligned");
  }
  const int* go = nullptr;
  if (mode != 0) {
    TORCH_CHECK(group_offsets.has_value(), "grouped mode needs group_offsets");
    CHECK_DT(group_offsets.value(), at::kInt);
    go = group_offsets.value().data_ptr<int>();
  }
  c10::cuda::CUDAGuard g(a.device());
  return mb_gemm_bf16_swiglu(a.data_ptr(), a.size(0), a.stride(0), b.data_ptr(), b.size(0),
                             b.stride(0), out.data_ptr(), out.stride(0), gup, ldgu, (int)M, (int)F,
                             (int)K, (int)mode, go, (int)num_groups, (int)bn,
                             group_counts.has_value() ? group_counts.value().data_ptr<int>() : nullptr,
                             err.data_ptr<int>(), cur_stream());
}

// ------------------------------------------------------------------ thin wrappers
// Optional tensors are passed as None; shapes are validated in miles_b200/ops/*.py and the
// essential invariants again here.
using OT = c10::optional<torch::Tensor>;
static void* P(const OT& t) { return t.has_value() ? t.value().data_ptr() : nullptr; }
static void* P(const torch::Tensor& t) { return t.data_ptr(); }
template <typename T> static T* PT(const OT& t) { return t.has_value() ? (T*)t.value().data_ptr() : nullptr; }
template <typename T> static T* PT(const torch::Tensor& t) { return (T*)t.data_ptr(); }

int64_t rmsnorm_fwd(torch::Tensor x, OT res, torch::Tensor w, OT h_out, torch::Tensor y, OT rstd,
                 double eps) {
  CHECK_CUDA(x); CHECK_DT(x, at::kBFloat16); TORCH_CHECK(x.is_contiguous());
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  return mb_rmsnorm_fwd(P(x), P(res), P(w), P(h_out), P(y), PT<float>(rstd), rows, H, (float)eps,
                          cur_stream());
}

int64_t rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, OT dres,
                 torch::Tensor dx, torch::Tensor dw_part, OT dw_f32, OT dw_bf16, bool accumulate) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous());
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  const int nparts = dw_part.size(0);
  return mb_rmsnorm_bwd(P(dy), P(x), P(w), PT<float>(rstd), P(dres), P(dx), PT<float>(dw_part),
                          nparts, PT<float>(dw_f32), P(dw_bf16), accumulate, rows, H, cur_stream());
}

int64_t qk_norm_rope_fwd(torch::Tensor qkv, OT qw, OT kw, torch::Tensor pos, torch::Tensor cos_t,
                      torch::Tensor sin_t, torch::Tensor q_out, torch::Tensor k_out,
                      torch::Tensor v_out, OT slot, int64_t ld_kv, OT rstd, int64_t nq,
                      int64_t nkv, double eps, bool use_norm) {
  TORCH_CHECK(qkv.stride(-1) == 1);
  // the kernel reads cos / sin as float2 pairs of a [positions, 64] table
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(-1) == 64 &&
                  sin_t.size(-1) == 64 && reinterpret_cast<uintptr_t>(cos_t.data_ptr()) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(sin_t.data_ptr()) % 8 == 0,
              "qk_norm_rope: cos / sin must be contiguous [positions, 64] fp32 tables");
  TORCH_CHECK(qkv.stride(0) % 2 == 0 && reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 4 == 0,
              "qk_norm_rope: qkv rows must be 4-byte aligned");
  const int T = qkv.size(0);
  return mb_qk_norm_rope_fwd(P(qkv), qkv.stride(0), P(qw), P(kw), PT<int>(pos),
                               PT<float>(cos_t), PT<float>(sin_t), P(q_out), P(k_out), P(v_out),
                               PT<long long>(slot), ld_kv, PT<float>(rstd), T, nq, nkv,
                               (float)eps, use_norm, cur_stream());
}

int64_t qk_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                      OT qw, OT kw, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t,
                      OT rstd, torch::Tensor dqkv, torch::Tensor dw_part, torch::Tensor dw_out,
                      int64_t nq, int64_t nkv, bool use_norm) {
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous());
  const int T = qkv.size(0);
  return mb_qk_norm_rope_bwd(P(dq), P(dk), P(dv), P(qkv), qkv.stride(0), P(qw), P(kw),
                               PT<int>(pos), PT<float>(cos_t), PT<float>(sin_t), PT<float>(rstd),
                               P(dqkv), PT<float>(dw_part), dw_part.size(0), PT<float>(dw_out), T,
                               nq, nkv, use_norm, cur_stream());
}

int64_t swiglu_fwd(torch::Tensor gu, torch::Tensor out, OT nrows) {
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous());
  const int I = out.size(-1);
  return mb_swiglu_fwd(P(gu), P(out), out.numel() / I, I, PT<int>(nrows), cur_stream());
}
int64_t swiglu_bwd(torch::Tensor gu, torch::Tensor dout, torch::Tensor dgu, OT nrows) {
  TORCH_CHECK(gu.is_contiguous() && dout.is_contiguous() && dgu.is_contiguous());
  const int I = dout.size(-1);
  return mb_swiglu_bwd(P(gu), P(dout), P(dgu), dout.numel() / I, I, PT<int>(nrows), cur_stream());
}

int64_t router_fwd(torch::Tensor logits, OT bias, OT idx_in, torch::Tensor idx_out,
                torch::Tensor w_out, int64_t k, int64_t score_fn, bool renorm, int64_t n_group,
                int64_t topk_group, double scale) {
  CHECK_DT(logits, at::kFloat); TORCH_CHECK(logits.is_contiguous());
  if (bias.has_value()) CHECK_DT(bias.value(), at::kFloat);
  return mb_router_fwd(PT<float>(logits), PT<float>(bias), PT<int>(idx_in), PT<int>(idx_out),
                         PT<float>(w_out), logits.size(0), logits.size(1), k, score_fn, renorm,
                         n_group, topk_group, (float)scale, cur_stream());
}
int64_t moe_route_dispatch(torch::Tensor logits, OT bias, OT idx_in, torch::Tensor x,
                           torch::Tensor idx_out, torch::Tensor w_out, torch::Tensor counts,
                           torch::Tensor offsets, torch::Tensor dest, torch::Tensor xs, int64_t k,
                           int64_t score_fn, bool renorm, int64_t n_group, int64_t topk_group,
                           double scale, int64_t align) {
  CHECK_DT(logits, at::kFloat); TORCH_CHECK(logits.is_contiguous() && x.is_contiguous());
  if (bias.has_value()) CHECK_DT(bias.value(), at::kFloat);
  return mb_moe_route_dispatch(PT<float>(logits), PT<float>(bias), PT<int>(idx_in), P(x),
                               logits.size(0), logits.size(1), k, x.size(1), score_fn, renorm,
                               n_group, topk_group, (float)scale, align, PT<int>(idx_out),
                               PT<float>(w_out), PT<int>(counts), PT<int>(offsets), PT<int>(dest),
                               P(xs), cur_stream());
}
int64_t router_bwd(torch::Tensor logits, torch::Tensor idx, torch::Tensor dw, torch::Tensor dlogits,
                int64_t score_fn, bool renorm, double scale) {
  return mb_router_bwd(PT<float>(logits), PT<int>(idx), PT<float>(dw), P(dlogits),
                         logits.size(0), logits.size(1), idx.size(1), score_fn, renorm,
                         (float)scale, cur_stream());
}
int64_t moe_permute_plan(torch::Tensor idx, int64_t E, int64_t align, torch::Tensor hist,
                      torch::Tensor chunk_base, torch::Tensor counts, torch::Tensor offsets,
                      torch::Tensor dest) {
  CHECK_DT(idx, at::kInt);
  return mb_moe_permute_plan(PT<int>(idx), idx.numel(), E, align, PT<int>(hist),
                               PT<int>(chunk_base), PT<int>(counts), PT<int>(offsets),
                               PT<int>(dest), cur_stream());
}
int64_t moe_zero_pad(torch::Tensor counts, torch::Tensor offsets, torch::Tensor buf) {
  return mb_moe_zero_pad(PT<int>(counts), PT<int>(offsets), P(buf), counts.size(0), buf.size(1),
                           cur_stream());
}
int64_t moe_gather(torch::Tensor x, torch::Tensor dest, int64_t k, torch::Tensor xs) {
  return mb_moe_gather(P(x), PT<int>(dest), dest.numel(), k, x.size(1), P(xs), (int)xs.size(0),
                       cur_stream());
}
int64_t moe_gather_bwd(torch::Tensor dxs, torch::Tensor dest, int64_t k, torch::Tensor dx) {
  return mb_moe_gather_bwd(P(dxs), PT<int>(dest), dx.size(0), k, dx.size(1), P(dx), cur_stream());
}
int64_t moe_combine(torch::Tensor ys, torch::Tensor dest, torch::Tensor w, OT add, torch::Tensor y) {
  return mb_moe_combine(P(ys), PT<int>(dest), PT<float>(w), P(add), y.size(0), w.size(1),
                          y.size(1), P(y), cur_stream());
}
int64_t moe_combine_bwd(torch::Tensor dy, torch::Tensor ys, torch::Tensor dest, torch::Tensor w,
                     torch::Tensor dys, torch::Tensor dw) {
  return mb_moe_combine_bwd(P(dy), P(ys), PT<int>(dest), PT<float>(w), dy.size(0), w.size(1),
                              dy.size(1), P(dys), PT<float>(dw), cur_stream());
}

int64_t attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, OT lse,
              torch::Tensor cu, torch::Tensor tile_seq, torch::Tensor tile_idx, int64_t nq,
              int64_t nkv, double scale, torch::Tensor err) {
  TORCH_CHECK(q.stride(-1) == 1 && k.stride(-1) == 1 && v.stride(-1) == 1 && o.stride(-1) == 1);
  TORCH_CHECK(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0,
              "attention row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(k.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0, "q/k/v must be 16-byte aligned");
  c10::cuda::CUDAGuard g(q.device());
  return mb_attn_fwd(P(q), P(k), P(v), P(o), PT<float>(lse), PT<int>(cu), PT<int>(tile_seq),
                       PT<int>(tile_idx), tile_seq.numel(), q.stride(0), k.stride(0), v.stride(0),
                       o.stride(0), nq, nkv, q.size(0), (float)scale, err.data_ptr<int>(),
                       cur_stream());
}
int64_t attn_decode_nsplit(int64_t max_pages) { return mb_attn_decode_nsplit(max_pages); }
int64_t attn_decode(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor o,
                 torch::Tensor page_table, torch::Tensor ctx_lens, int64_t nq, int64_t nkv,
                 double scale, OT ws_o, OT ws_ml, torch::Tensor err) {
  TORCH_CHECK(q.is_contiguous() && kc.is_contiguous() && vc.is_contiguous(),
              "decode attention needs contiguous q and caches");
  c10::cuda::CUDAGuard g(q.device());
  return mb_attn_decode(P(q), P(kc), P(vc), P(o), PT<int>(page_table), PT<int>(ctx_lens),
                          q.size(0), page_table.size(1), kc.size(0), nq, nkv, (float)scale,
                          PT<float>(ws_o), PT<float>(ws_ml), err.data_ptr<int>(), cur_stream());
}
int64_t attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
              torch::Tensor dout, torch::Tensor lse, torch::Tensor delta, torch::Tensor dq,
              torch::Tensor dk, torch::Tensor dv, torch::Tensor cu, torch::Tensor blk_seq,
              torch::Tensor blk_idx, int64_t nq, int64_t nkv, double scale, torch::Tensor err) {
  TORCH_CHECK(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0 &&
              dout.stride(0) % 8 == 0, "attention row strides must be 16-byte multiples");
  c10::cuda::CUDAGuard g(q.device());
  return mb_attn_bwd(P(q), P(k), P(v), P(o), P(dout), PT<float>(lse), PT<float>(delta), P(dq),
                       P(dk), P(dv), PT<int>(cu), PT<int>(blk_seq), PT<int>(blk_idx),
                       blk_seq.numel(), q.stride(0), k.stride(0), v.stride(0), o.stride(0),
                       dout.stride(0), dq.stride(0), dk.stride(0), dv.stride(0), nq, nkv,
                       q.size(0), (float)scale, err.data_ptr<int>(), cur_stream());
}

int64_t logprob_fwd(torch::Tensor logits, torch::Tensor target, double inv_temp, OT logp, OT ent,
                 OT lse) {
  CHECK_DT(logits, at::kFloat); TORCH_CHECK(logits.stride(-1) == 1);
  return mb_logprob_fwd(PT<float>(logits), logits.stride(0), PT<int>(target), logits.size(0),
                          logits.size(1), (float)inv_temp, PT<float>(logp), PT<float>(ent),
                          PT<float>(lse), cur_stream());
}
int64_t logprob_part(torch::Tensor logits, torch::Tensor target, int64_t lo, double inv_temp,
                     torch::Tensor part) {
  CHECK_DT(logits, at::kFloat); TORCH_CHECK(logits.stride(-1) == 1);
  CHECK_DT(target, at::kInt); CHECK_DT(part, at::kFloat);
  const int64_t n = logits.size(0);
  TORCH_CHECK(target.is_contiguous() && target.numel() >= n, "logprob_part: target");
  TORCH_CHECK(part.is_contiguous() && part.numel() >= 4 * n, "logprob_part: part needs [4, n]");
  return mb_logprob_part(PT<float>(logits), logits.stride(0), PT<int>(target), lo, n,
                         logits.size(1), (float)inv_temp, PT<float>(part), cur_stream());
}
int64_t logprob_combine(torch::Tensor parts, int64_t world, OT logp, OT ent, OT lse) {
  CHECK_DT(parts, at::kFloat);
  TORCH_CHECK(parts.is_contiguous() && world >= 1 && parts.numel() % (4 * world) == 0,
              "logprob_combine: parts must be [world, 4, n]");
  const int64_t n = parts.numel() / (4 * world);
  for (const OT* o : {&logp, &ent, &lse})
    if (o->has_value()) {
      CHECK_DT(o->value(), at::kFloat);
      TORCH_CHECK(o->value().is_contiguous() && o->value().numel() >= n, "logprob_combine: output");
    }
  return mb_logprob_combine(PT<float>(parts), world, n, PT<float>(logp), PT<float>(ent),
                            PT<float>(lse), cur_stream());
}
int64_t logprob_bwd(torch::Tensor logits, torch::Tensor target, double inv_temp, torch::Tensor lse,
                 OT g_lp, OT g_ent, OT ent, torch::Tensor dlogits) {
  return mb_logprob_bwd(PT<float>(logits), logits.stride(0), PT<int>(target), logits.size(0),
                          logits.size(1), (float)inv_temp, PT<float>(lse), PT<float>(g_lp),
                          PT<float>(g_ent), PT<float>(ent), P(dlogits), dlogits.stride(0),
                          cur_stream());
}
int64_t sample(torch::Tensor logits, torch::Tensor inv_temps, torch::Tensor seeds,
            torch::Tensor positions, torch::Tensor tokens, OT logp, OT thr) {
  CHECK_DT(logits, at::kFloat);
  if (thr.has_value()) CHECK_DT(thr.value(), at::kFloat);
  return mb_sample(PT<float>(logits), logits.stride(0), logits.size(0), logits.size(1),
                     PT<float>(inv_temps), PT<unsigned long long>(seeds), PT<int>(positions),
                     PT<int>(tokens), PT<float>(logp), PT<float>(thr), cur_stream());
}
int64_t policy_loss(torch::Tensor logp, torch::Tensor old_logp, torch::Tensor adv,
                 torch::Tensor weight, OT rollout_logp, OT ref_logp, torch::Tensor dlogp,
                 OT pg_out, torch::Tensor part, torch::Tensor metrics, double eps, double eps_hi,
                 double eps_c, double tis_lo, double tis_hi, double kl_coef, int64_t kl_type,
                 int64_t use_tis) {
  // the kernel reads the rollout log-probs under TIS / IcePop and the reference log-probs under
  // a KL term: reject the call on the host when they are missing (a null read would fault)
  TORCH_CHECK(use_tis == 0 || rollout_logp.has_value(), "policy_loss: TIS needs rollout_logp");
  TORCH_CHECK(kl_type == 0 || ref_logp.has_value(), "policy_loss: a KL term needs ref_logp");
  const int64_t n = logp.numel();
  for (const torch::Tensor* t : {&old_logp, &adv, &weight, &dlogp})
    TORCH_CHECK(t->numel() == n, "policy_loss: operand sizes differ");
  if (rollout_logp.has_value()) TORCH_CHECK(rollout_logp.value().numel() == n, "rollout_logp size");
  if (ref_logp.has_value()) TORCH_CHECK(ref_logp.value().numel() == n, "ref_logp size");
  return mb_policy_loss(PT<float>(logp), PT<float>(old_logp), PT<float>(adv), PT<float>(weight),
                          PT<float>(rollout_logp), PT<float>(ref_logp), PT<float>(dlogp),
                          PT<float>(pg_out), PT<float>(part), PT<float>(metrics), logp.numel(),
                          eps, eps_hi, eps_c, tis_lo, tis_hi, kl_coef, kl_type, (int)use_tis,
                          cur_stream());
}
int64_t gae(torch::Tensor rewards, torch::Tensor values, torch::Tensor cu, double gamma, double lam,
         torch::Tensor adv, torch::Tensor ret) {
  return mb_gae(PT<float>(rewards), PT<float>(values), PT<int>(cu), cu.numel() - 1, gamma, lam,
                  PT<float>(adv), PT<float>(ret), cur_stream());
}
int64_t grpo_adv(torch::Tensor r, int64_t gsize, bool norm_std, double eps, torch::Tensor adv) {
  return mb_grpo_adv(PT<float>(r), r.numel() / gsize, gsize, norm_std, eps, PT<float>(adv),
                       cur_stream());
}
int64_t sqnorm(torch::Tensor x, torch::Tensor part, torch::Tensor out) {
  return mb_sqnorm(P(x), x.numel(), x.scalar_type() == at::kBFloat16, PT<float>(part),
                     PT<float>(out), cur_stream());
}
int64_t nonfinite(torch::Tensor x, torch::Tensor flag) {
  return mb_nonfinite(P(x), x.numel(), x.scalar_type() == at::kBFloat16, PT<float>(flag),
                        cur_stream());
}
int64_t adam(torch::Tensor param, OT master, torch::Tensor m, torch::Tensor v, torch::Tensor grad,
          double lr, double b1, double b2, double eps, double wd, int64_t step, OT sq,
          double max_norm, double inv_loss_scale, int64_t seed, OT skip) {
  CHECK_DT(param, at::kBFloat16);
  TORCH_CHECK(param.numel() == grad.numel() && m.numel() == param.numel() && v.numel() == param.numel());
  return mb_adam(P(param), PT<float>(master), P(m), P(v), P(grad), param.numel(),
                   grad.scalar_type() == at::kBFloat16, m.scalar_type() == at::kBFloat16, lr, b1,
                   b2, eps, wd, step, PT<float>(sq), max_norm, inv_loss_scale,
                   (unsigned long long)seed, PT<float>(skip), cur_stream());
}

// ------------------------------------------------------------------ quantization
int64_t fp8_block_cast(torch::Tensor x, int64_t bm, int64_t bn, torch::Tensor y,
                       torch::Tensor scale_inv, bool ue8m0) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2);
  return mb_fp8_block_cast(P(x), x.size(0), x.size(1), bm, bn, P(y), PT<float>(scale_inv), ue8m0,
                           cur_stream());
}
int64_t fp8_group_cast(torch::Tensor x, int64_t group, torch::Tensor y, torch::Tensor scale,
                       bool ue8m0) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2);
  return mb_fp8_group_cast(P(x), x.size(0), x.size(1), group, P(y), PT<float>(scale), ue8m0,
                           cur_stream());
}
int64_t int4_fake_quant(torch::Tensor x, int64_t group, bool sym, torch::Tensor q,
                        torch::Tensor scale, OT zero) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2);
  const int dt = x.scalar_type() == at::kBFloat16 ? 0 : (x.scalar_type() == at::kHalf ? 1 : 2);
  return mb_int4_fake_quant(P(x), x.size(0), x.size(1), group, sym, dt, P(q), P(scale), P(zero),
                            cur_stream());
}
int64_t nvfp4_quant(torch::Tensor x, double global_scale, torch::Tensor packed,
                    torch::Tensor bscale) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2);
  return mb_nvfp4_quant(P(x), x.size(0), x.size(1), (float)global_scale, P(packed), P(bscale),
                        cur_stream());
}
int64_t mxfp8_quant(torch::Tensor x, torch::Tensor y, torch::Tensor sexp) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2);
  return mb_mxfp8_quant(P(x), x.size(0), x.size(1), P(y), P(sexp), cur_stream());
}

// ------------------------------------------------------------------ symmetric memory
// Raw device allocations shared with peer processes through CUDA IPC handles. Pointers cross
// the binding as int64 addresses; peer pointer lists as std::vector<int64_t>.
int64_t symm_malloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  long long p = 0;
  int rc = mb_symm_malloc(bytes, &p);
  TORCH_CHECK(rc == 0, "symm_malloc failed");
  return p;
}
int64_t symm_free(int64_t ptr) { return mb_symm_free(ptr); }
torch::Tensor ipc_get_handle(int64_t ptr) {
  auto t = torch::empty({mb_ipc_handle_size()}, torch::dtype(torch::kUInt8));
  TORCH_CHECK(mb_ipc_get_handle(ptr, t.data_ptr()) == 0, "cudaIpcGetMemHandle failed");
  return t;
}
// (handle of the containing allocation, byte offset of ptr in it)
std::tuple<torch::Tensor, int64_t> ipc_get_handle_range(int64_t ptr) {
  auto t = torch::empty({mb_ipc_handle_size()}, torch::dtype(torch::kUInt8));
  long long off = 0;
  TORCH_CHECK(mb_ipc_get_handle_range(ptr, t.data_ptr(), &off) == 0, "IPC handle lookup failed");
  return {t, off};
}
int64_t ipc_open(torch::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == mb_ipc_handle_size() && handle.is_contiguous());
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  long long p = 0;
  TORCH_CHECK(mb_ipc_open(handle.data_ptr(), &p) == 0, "cudaIpcOpenMemHandle failed");
  return p;
}
int64_t ipc_close(int64_t ptr) { return mb_ipc_close(ptr); }
// Wrap a raw device address as a tensor view (no ownership).
torch::Tensor from_ptr(int64_t ptr, std::vector<int64_t> shape, c10::ScalarType dt, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dt).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}
int64_t symm_barrier(std::vector<int64_t> flag_ptrs, torch::Tensor my_flags, torch::Tensor ctl,
                     int64_t rank, int64_t world, int64_t timeout_ns, torch::Tensor err) {
  return mb_symm_barrier((const long long*)flag_ptrs.data(), PT<int>(my_flags), PT<int>(ctl), rank,
                         world, timeout_ns, PT<int>(err), cur_stream());
}
int64_t symm_allreduce(std::vector<int64_t> flag_ptrs, std::vector<int64_t> stage_ptrs,
                       torch::Tensor my_flags, torch::Tensor ctl, torch::Tensor my_stage,
                       int64_t cap, OT src, int64_t rows, int64_t H, int64_t rank, int64_t world,
                       OT res, OT norm_w, double eps, torch::Tensor out, OT h_out, OT rstd,
                       int64_t timeout_ns, torch::Tensor err) {
  if (src.has_value()) { CHECK_DT(src.value(), at::kBFloat16); TORCH_CHECK(src.value().is_contiguous()); }
  CHECK_DT(out, at::kBFloat16);
  TORCH_CHECK(out.is_contiguous() && out.numel() >= rows * H);
  return mb_symm_allreduce((const long long*)flag_ptrs.data(), (const long long*)stage_ptrs.data(),
                           PT<int>(my_flags), PT<int>(ctl), P(my_stage), cap, P(src), rows, H,
                           rank, world, P(res), P(norm_w), (float)eps, P(out), P(h_out),
                           PT<float>(rstd), timeout_ns, PT<int>(err), cur_stream());
}
int64_t symm_collective(int64_t kind, std::vector<int64_t> flag_ptrs, std::vector<int64_t> stage_ptrs,
                        torch::Tensor my_flags, torch::Tensor ctl, torch::Tensor my_stage,
                        int64_t cap, OT src, int64_t rows, int64_t H, int64_t rank, int64_t world,
                        OT res, OT norm_w, double eps, torch::Tensor out, OT h_out, OT rstd,
                        int64_t timeout_ns, torch::Tensor err) {
  if (src.has_value()) { CHECK_DT(src.value(), at::kBFloat16); TORCH_CHECK(src.value().is_contiguous()); }
  CHECK_DT(out, at::kBFloat16);
  TORCH_CHECK(out.is_contiguous());
  TORCH_CHECK(out.numel() >= (kind == 2 ? world : 1) * rows * H, "output too small");
  return mb_symm_collective((int)kind, (const long long*)flag_ptrs.data(),
                            (const long long*)stage_ptrs.data(), PT<int>(my_flags), PT<int>(ctl),
                            P(my_stage), cap, P(src), rows, H, rank, world, P(res), P(norm_w),
                            (float)eps, P(out), P(h_out), PT<float>(rstd), timeout_ns,
                            PT<int>(err), cur_stream());
}
int64_t symm_copy(torch::Tensor src, int64_t dst_ptr, int64_t bytes) {
  return mb_symm_copy(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), bytes, cur_stream());
}
int64_t symm_copy_ptr(int64_t src_ptr, int64_t dst_ptr, int64_t bytes) {
  return mb_symm_copy(reinterpret_cast<void*>(src_ptr), reinterpret_cast<void*>(dst_ptr), bytes,
                      cur_stream());
}
// Fused gradient reduce-scatter over peer memory (symm.cu grad_rs_kernel).
int64_t grad_rs(std::vector<int64_t> g_ptrs, int64_t lo, int64_t n, double scale, torch::Tensor out,
                torch::Tensor partial, torch::Tensor counter, torch::Tensor sq) {
  CHECK_DT(out, at::kBFloat16);
  CHECK_DT(partial, at::kFloat);
  CHECK_DT(counter, at::kInt);
  CHECK_DT(sq, at::kFloat);
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() >= n, "grad_rs: out");
  TORCH_CHECK(partial.is_cuda() && partial.numel() >= 148 * 4, "grad_rs: partial needs 592 floats");
  TORCH_CHECK(counter.is_cuda() && counter.numel() >= 1 && sq.is_cuda() && sq.numel() >= 1);
  TORCH_CHECK(!g_ptrs.empty() && g_ptrs.size() <= 8, "grad_rs: 1..8 ranks");
  return mb_grad_rs((const long long*)g_ptrs.data(), (int)g_ptrs.size(), lo, n, (float)scale,
                    P(out), PT<float>(partial), PT<int>(counter), PT<float>(sq), cur_stream());
}
// Refit: quantise a local bf16 weight into (possibly peer) fp8 + scale buffers, and dequantise
// from (possibly peer) buffers into a local bf16 weight.
int64_t fp8_block_cast_ptr(torch::Tensor x, int64_t bm, int64_t bn, int64_t y_ptr, int64_t s_ptr,
                           bool ue8m0) {
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2 && x.scalar_type() == at::kBFloat16);
  return mb_fp8_block_cast(P(x), x.size(0), x.size(1), bm, bn, reinterpret_cast<void*>(y_ptr),
                           reinterpret_cast<float*>(s_ptr), ue8m0, cur_stream());
}
int64_t fp8_block_dequant_ptr(int64_t q_ptr, int64_t s_ptr, int64_t bm, int64_t bn,
                              torch::Tensor out) {
  TORCH_CHECK(out.is_contiguous() && out.dim() == 2 && out.scalar_type() == at::kBFloat16);
  return mb_fp8_block_dequant(reinterpret_cast<void*>(q_ptr), reinterpret_cast<float*>(s_ptr),
                              out.size(0), out.size(1), bm, bn, P(out), cur_stream());
}

// Fused GEMM + all-reduce, GEMM half: y = a @ b^T (b_mn: a @ b) stored into peer staging areas.
int64_t gemm_peer(torch::Tensor a, torch::Tensor b, bool b_mn, int64_t M, int64_t N, int64_t K,
                  std::vector<int64_t> peer_ptrs, int64_t ldc, torch::Tensor par_word,
                  int64_t par_stride, int64_t scatter_rows, int64_t bn, torch::Tensor err) {
  CHECK_CUDA(a); CHECK_CUDA(b);
  CHECK_DT(a, at::kBFloat16); CHECK_DT(b, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2);
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(b);
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && N % 8 == 0 && ldc % 8 == 0);
  c10::cuda::CUDAGuard g(a.device());
  return mb_gemm_bf16_peer(a.data_ptr(), a.size(0), a.size(1), a.stride(0), false, b.data_ptr(),
                           b.size(0), b.size(1), b.stride(0), b_mn, (int)M, (int)N, (int)K,
                           (const long long*)peer_ptrs.data(), (int)peer_ptrs.size(), ldc,
                           PT<int>(par_word), par_stride, (int)scatter_rows, (int)bn, PT<int>(err),
                           cur_stream());
}

// ------------------------------------------------------------------ expert-parallel dispatch
#define LLP(v) ((const long long*)(v).data())
int64_t ep_publish(torch::Tensor counts, int64_t E_local, int64_t rank,
                   std::vector<int64_t> table_ptrs) {
  return mb_ep_publish(PT<int>(counts), counts.numel(), E_local, rank, table_ptrs.size(),
                       LLP(table_ptrs), cur_stream());
}
int64_t ep_offsets(torch::Tensor table, int64_t world, int64_t E_local, int64_t align,
                   torch::Tensor offsets, torch::Tensor counts, torch::Tensor base, int64_t cap,
                   torch::Tensor err) {
  return mb_ep_offsets(PT<int>(table), world, E_local, align, PT<int>(offsets), PT<int>(counts),
                       PT<int>(base), cap, PT<int>(err), cur_stream());
}
int64_t ep_dispatch(torch::Tensor x, torch::Tensor idx, torch::Tensor dest_g, torch::Tensor off_g,
                    int64_t E_local, int64_t rank, std::vector<int64_t> base_ptrs,
                    std::vector<int64_t> xs_ptrs, int64_t cap, torch::Tensor pos, torch::Tensor err) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && idx.is_contiguous());
  return mb_ep_dispatch(P(x), PT<int>(idx), PT<int>(dest_g), PT<int>(off_g), x.size(0),
                        idx.size(1), x.size(1), E_local, rank, base_ptrs.size(), LLP(base_ptrs),
                        LLP(xs_ptrs), cap, PT<int>(pos), PT<int>(err), cur_stream());
}
int64_t ep_combine(std::vector<int64_t> ys_ptrs, torch::Tensor idx, torch::Tensor pos,
                   torch::Tensor w, OT add, int64_t H, int64_t E_local, torch::Tensor y, OT saved) {
  TORCH_CHECK(y.is_contiguous() && y.scalar_type() == at::kBFloat16);
  return mb_ep_combine(LLP(ys_ptrs), ys_ptrs.size(), PT<int>(idx), PT<int>(pos), PT<float>(w),
                       P(add), idx.size(0), idx.size(1), H, E_local, P(y), P(saved), cur_stream());
}
int64_t ep_combine_bwd(torch::Tensor dy, torch::Tensor saved, torch::Tensor idx, torch::Tensor pos,
                       torch::Tensor w, int64_t E_local, std::vector<int64_t> dys_ptrs,
                       torch::Tensor dw) {
  TORCH_CHECK(dy.is_contiguous() && saved.is_contiguous());
  return mb_ep_combine_bwd(P(dy), P(saved), PT<int>(idx), PT<int>(pos), PT<float>(w), idx.size(0),
                           idx.size(1), dy.size(1), E_local, dys_ptrs.size(), LLP(dys_ptrs),
                           PT<float>(dw), cur_stream());
}
int64_t ep_gather_bwd(std::vector<int64_t> dxs_ptrs, torch::Tensor idx, torch::Tensor pos,
                      int64_t H, int64_t E_local, torch::Tensor dx) {
  TORCH_CHECK(dx.is_contiguous());
  return mb_ep_gather_bwd(LLP(dxs_ptrs), dxs_ptrs.size(), PT<int>(idx), PT<int>(pos), idx.size(0),
                          idx.size(1), H, E_local, P(dx), cur_stream());
}

// ------------------------------------------------------------------ Gated DeltaNet decode
int64_t gdn_decode(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor beta,
                   torch::Tensor g, torch::Tensor rows, torch::Tensor S, torch::Tensor out,
                   double scale) {
  for (auto* t : {&q, &k, &v, &beta, &g, &S, &out}) {
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kFloat,
                "gdn_decode: fp32 contiguous CUDA tensors expected");
  }
  TORCH_CHECK(rows.scalar_type() == at::kLong && rows.is_contiguous());
  TORCH_CHECK(q.dim() == 3 && S.dim() == 4 && S.size(1) == q.size(1) && S.size(2) == q.size(2));
  return mb_gdn_decode(PT<float>(q), PT<float>(k), PT<float>(v), PT<float>(beta), PT<float>(g),
                       (const long long*)rows.data_ptr(), PT<float>(S), PT<float>(out), q.size(0),
                       q.size(1), q.size(2), S.size(3), (float)scale, cur_stream());
}

// ------------------------------------------------------------------ MLA decode
int64_t mla_decode(torch::Tensor q_lat, torch::Tensor q_pe, torch::Tensor cache,
                   torch::Tensor page_table, torch::Tensor ctx_lens, OT bias, double scale,
                   torch::Tensor out) {
  TORCH_CHECK(q_lat.is_contiguous() && q_pe.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(q_lat.scalar_type() == at::kFloat && q_pe.scalar_type() == at::kFloat &&
              out.scalar_type() == at::kFloat && cache.scalar_type() == at::kBFloat16);
  TORCH_CHECK(page_table.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt &&
              page_table.is_contiguous());
  if (bias.has_value()) TORCH_CHECK(bias.value().scalar_type() == at::kFloat && bias.value().stride(-1) == 1);
  const long long row_stride = cache.stride(0);
  return mb_mla_decode(PT<float>(q_lat), PT<float>(q_pe), cache.data_ptr(), row_stride,
                       PT<int>(page_table), page_table.size(1), PT<int>(ctx_lens), PT<float>(bias),
                       bias.has_value() ? bias.value().stride(0) : 0, q_lat.size(0), q_lat.size(1),
                       q_lat.size(2), q_pe.size(2), (float)scale, PT<float>(out), cur_stream());
}


// ------------------------------------------------------------------ device-resident decode
// st: dict-free positional state (see engine/engine.py DecodeState): slot arrays [S+1, ...]
int64_t decode_prep(torch::Tensor rows, int64_t spare, torch::Tensor s_tok, torch::Tensor s_pos,
                    torch::Tensor s_done, torch::Tensor s_pt, torch::Tensor s_invt,
                    torch::Tensor s_seed, torch::Tensor tokens, torch::Tensor positions,
                    torch::Tensor ctx, torch::Tensor slots, torch::Tensor pt, torch::Tensor invt,
                    torch::Tensor seeds, OT state_rows, int64_t state_spare) {
  CHECK_DT(rows, at::kInt); CHECK_DT(s_tok, at::kInt); CHECK_DT(s_pos, at::kInt);
  CHECK_DT(s_done, at::kInt); CHECK_DT(s_pt, at::kInt); CHECK_DT(s_seed, at::kLong);
  CHECK_DT(slots, at::kLong); CHECK_DT(pt, at::kInt); CHECK_DT(seeds, at::kLong);
  const int B = rows.numel();
  TORCH_CHECK(pt.size(0) >= B && pt.size(1) == s_pt.size(1), "page-table shapes");
  TORCH_CHECK(rows.is_contiguous() && s_pt.is_contiguous() && pt.is_contiguous());
  if (state_rows.has_value()) CHECK_DT(state_rows.value(), at::kLong);
  return mb_decode_prep(PT<int>(rows), B, (int)spare, PT<int>(s_tok), PT<int>(s_pos),
                        PT<int>(s_done), PT<int>(s_pt), (int)s_pt.size(1), PT<float>(s_invt),
                        PT<long long>(s_seed), PT<int>(tokens), PT<int>(positions), PT<int>(ctx),
                        PT<long long>(slots), PT<int>(pt), PT<float>(invt), PT<long long>(seeds),
                        PT<long long>(state_rows), (int)state_spare, cur_stream());
}
int64_t decode_commit(torch::Tensor rows, int64_t spare, torch::Tensor tok, torch::Tensor lp,
                      OT experts, torch::Tensor s_tok, torch::Tensor s_pos, torch::Tensor s_done,
                      torch::Tensor s_nout, torch::Tensor s_maxnew, torch::Tensor s_stop,
                      torch::Tensor out_tok, torch::Tensor out_lp, OT out_exp, torch::Tensor s_rec) {
  CHECK_DT(tok, at::kInt); CHECK_DT(lp, at::kFloat); CHECK_DT(out_tok, at::kInt);
  CHECK_DT(out_lp, at::kFloat); CHECK_DT(s_stop, at::kInt); CHECK_DT(s_rec, at::kInt);
  const int B = rows.numel();
  int n_moe = 0, topk = 0, max_len = 0;
  if (experts.has_value() && out_exp.has_value()) {
    CHECK_DT(experts.value(), at::kInt);
    CHECK_DT(out_exp.value(), at::kByte);
    TORCH_CHECK(experts.value().is_contiguous() && out_exp.value().is_contiguous());
    TORCH_CHECK(experts.value().dim() == 3 && experts.value().size(1) == B,
                "experts must be [n_moe, B, k]");
    n_moe = experts.value().size(0);
    topk = experts.value().size(2);
    max_len = out_exp.value().size(1);
    TORCH_CHECK(out_exp.value().numel() == out_exp.value().size(0) * (int64_t)max_len * n_moe * topk,
                "out_exp must be [slots, max_len, n_moe, k]");
  }
  return mb_decode_commit(PT<int>(rows), B, (int)spare, PT<int>(tok), PT<float>(lp),
                          n_moe ? PT<int>(experts) : nullptr, n_moe, topk, PT<int>(s_tok), PT<int>(s_pos),
                          PT<int>(s_done), PT<int>(s_nout), PT<int>(s_maxnew), PT<int>(s_stop),
                          (int)s_stop.size(1), PT<int>(out_tok), PT<float>(out_lp),
                          (int)out_tok.size(1), n_moe ? PT<unsigned char>(out_exp) : nullptr,
                          PT<int>(s_rec), max_len, cur_stream());
}


// ------------------------------------------------------------------ virtual-memory arenas
// Status codes are returned first; values follow (ptr / handle as int64).
std::tuple<int64_t, int64_t> vmm_granularity(int64_t device) {
  size_t g = 0;
  const int rc = mb_vmm_granularity((int)device, &g);
  return {rc, (int64_t)g};
}
std::tuple<int64_t, int64_t> vmm_reserve(int64_t bytes) {
  unsigned long long p = 0;
  const int rc = mb_vmm_reserve((size_t)bytes, &p);
  return {rc, (int64_t)p};
}
int64_t vmm_free(int64_t ptr, int64_t bytes) { return mb_vmm_free((unsigned long long)ptr, (size_t)bytes); }
std::tuple<int64_t, int64_t> vmm_map(int64_t ptr, int64_t bytes, int64_t device) {
  unsigned long long h = 0;
  const int rc = mb_vmm_map((unsigned long long)ptr, (size_t)bytes, (int)device, &h);
  return {rc, (int64_t)h};
}
int64_t vmm_unmap(int64_t ptr, int64_t bytes, int64_t handle) {
  return mb_vmm_unmap((unsigned long long)ptr, (size_t)bytes, (unsigned long long)handle);
}
// A tensor view of `numel` elements at device address `ptr` (no ownership: the arena owns it).
torch::Tensor vmm_tensor(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel},
                          torch::TensorOptions().dtype(dtype).device(torch::kCUDA, (int)device));
}

// Page-lock / release a byte range of a CPU tensor's storage.
int64_t host_register(torch::Tensor t, int64_t offset, int64_t bytes) {
  TORCH_CHECK(t.device().is_cpu() && t.is_contiguous());
  TORCH_CHECK(offset >= 0 && offset + bytes <= (int64_t)(t.numel() * t.element_size()));
  return mb_host_register(static_cast<char*>(t.data_ptr()) + offset, (size_t)bytes);
}
int64_t host_unregister(torch::Tensor t, int64_t offset) {
  return mb_host_unregister(static_cast<char*>(t.data_ptr()) + offset);
}

// Guard words of the checked build: {moe, engine_step} (zeros in the regular build).
std::vector<int64_t> check_words(bool clear) {
  int a = 0, b = 0;
  mb_checks_moe(&a, clear);
  mb_checks_engine(&b, clear);
  return {a, b};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("mla_decode", &mla_decode, "absorbed MLA decode over the paged latent cache");
  m.def("gdn_decode", &gdn_decode, "Gated DeltaNet decode step (state updated in place)");
  m.def("ep_publish", &ep_publish);
  m.def("ep_offsets", &ep_offsets);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_combine", &ep_combine);
  m.def("ep_combine_bwd", &ep_combine_bwd);
  m.def("ep_gather_bwd", &ep_gather_bwd);
  m.def("symm_malloc", &symm_malloc);
  m.def("symm_free", &symm_free);
  m.def("ipc_get_handle", &ipc_get_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_get_handle_range", &ipc_get_handle_range);
  m.def("ipc_close", &ipc_close);
  m.def("from_ptr", &from_ptr);
  m.def("symm_barrier", &symm_barrier);
  m.def("symm_allreduce", &symm_allreduce);
  m.def("symm_collective", &symm_collective);
  m.def("symm_copy", &symm_copy);
  m.def("symm_copy_ptr", &symm_copy_ptr);
  m.def("grad_rs", &grad_rs);
  m.def("fp8_block_cast_ptr", &fp8_block_cast_ptr);
  m.def("fp8_block_dequant_ptr", &fp8_block_dequant_ptr);
  m.def("gemm_peer", &gemm_peer, "tcgen05 GEMM storing its tiles into peer staging areas");
  m.def("fp8_block_cast", &fp8_block_cast);
  m.def("fp8_group_cast", &fp8_group_cast);
  m.def("int4_fake_quant", &int4_fake_quant);
  m.def("nvfp4_quant", &nvfp4_quant);
  m.def("mxfp8_quant", &mxfp8_quant);
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM (dense / grouped)");
  m.def("fp8_act_quant", &fp8_act_quant, "1 x 128 fp8 activation quantisation (K-block-major scales)");
  m.def("gemm_fp8", &gemm_fp8, "tcgen05 block-scaled fp8 GEMM (dense / grouped, SwiGLU epilogue)");
  m.def("gemm_swiglu", &gemm_swiglu, "tcgen05 bf16 GEMM with fused SwiGLU epilogue");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("router_fwd", &router_fwd);
  m.def("moe_route_dispatch", &moe_route_dispatch);
  m.def("router_bwd", &router_bwd);
  m.def("moe_permute_plan", &moe_permute_plan);
  m.def("moe_zero_pad", &moe_zero_pad);
  m.def("moe_gather", &moe_gather);
  m.def("moe_gather_bwd", &moe_gather_bwd);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_decode", &attn_decode);
  m.def("attn_decode_nsplit", &attn_decode_nsplit);
  m.def("attn_bwd", &attn_bwd);
  m.def("logprob_fwd", &logprob_fwd);
  m.def("logprob_bwd", &logprob_bwd);
  m.def("logprob_part", &logprob_part);
  m.def("logprob_combine", &logprob_combine);
  m.def("sample", &sample);
  m.def("policy_loss", &policy_loss);
  m.def("gae", &gae);
  m.def("grpo_adv", &grpo_adv);
  m.def("sqnorm", &sqnorm);
  m.def("nonfinite", &nonfinite);
  m.def("adam", &adam);
  m.def("decode_prep", &decode_prep);
  m.def("check_words", &check_words);
  m.def("vmm_granularity", &vmm_granularity);
  m.def("vmm_reserve", &vmm_reserve);
  m.def("vmm_free", &vmm_free);
  m.def("vmm_map", &vmm_map);
  m.def("vmm_unmap", &vmm_unmap);
  m.def("vmm_tensor", &vmm_tensor);
  m.def("host_register", &host_register);
  m.def("host_unregister", &host_unregister);
  m.def("decode_commit", &decode_commit);
}
