// Deterministic causal attention for head_dim 128, bf16 in / fp32 softmax, GQA (sm_100a).
//
//  * forward and paged decode: tcgen05 kernels in csrc/attention_sm100.cu (entry points and
//    the decode split-KV combine kernel here)
//  * backward: the delta = rowsum(dO * O) kernel here, then the tcgen05 dK/dV and dQ kernels of
//    csrc/attention_sm100.cu (deterministic: each output tile has one owner)
//
// Bitwise train/rollout parity of the forward is a property of the tcgen05 kernel (one code
// path for prefill and decode rows); the backward only needs the forward's LSE.
//
// Reference roles replaced: TE/cuDNN fused attention and flash-attn varlen (E5,
// `--attention-backend flash`), SGLang paged decode attention (E7).
#include "common.cuh"
#include "api.h"

namespace mb {
namespace attn {

constexpr int D = 128;       // head dim
MB_DEVICE uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ---------------------------------------------------------------------------------------------
// Canonical split-KV combination. Keys are processed in chunks of 1024 (csrc/attention_sm100.cu);
// each chunk's (m, l, o) starts from scratch and the chunk partials are merged in increasing
// chunk order. The prefill kernel merges in TMEM; the decode kernel writes one partial per chunk
// and the combine kernel below merges them with the very same non-contracted float operations,
// so both give identical bits.
// ---------------------------------------------------------------------------------------------

// (M, L) <- merge((M, L), (m, l)); returns the factors applied to the old total and the chunk.
MB_DEVICE void merge_stats(float& M, float& L, float m, float l, float& fa, float& fb) {
  if (m == -INFINITY) { fa = 1.f; fb = 0.f; return; }
  if (M == -INFINITY) { M = m; L = l; fa = 0.f; fb = 1.f; return; }
  const float Mn = fmaxf(M, m);
  fa = exp2f(__fsub_rn(M, Mn));
  fb = exp2f(__fsub_rn(m, Mn));
  L = __fadd_rn(__fmul_rn(L, fa), __fmul_rn(l, fb));
  M = Mn;
}
MB_DEVICE float merge_val(float O, float o, float fa, float fb) {
  if (fb == 0.f) return O;
  if (fa == 0.f) return o;
  return __fadd_rn(__fmul_rn(O, fa), __fmul_rn(o, fb));
}

struct CombineParams {
  __nv_bfloat16* o;         // [B, nq, 128]
  const int* ctx_lens;      // [B]
  const float* ws_o;        // [B, nq, nsplit_max, 128]
  const float* ws_ml;       // [B, nq, nsplit_max, 2]
  int nq, nsplit_max;
};

// Merge the chunk partials of every (sequence, query head) in chunk order (same operations as
// the prefill kernel's in-register merge) and write the bf16 output. One warp per row; lane
// owns columns lane*4 .. lane*4+3.
__global__ void attn_decode_combine_kernel(const CombineParams p, int B) {
  pdl_trigger();
  pdl_wait();
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)B * p.nq) return;
  const int b = (int)(w / p.nq);
  const int ctx = p.ctx_lens[b];
  if (ctx <= 0) return;
  const int nsplit = (ctx + 1023) / 1024;
  if (nsplit <= 1) return;
  float M = -INFINITY, L = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < nsplit; ++s) {
    const long long base = w * p.nsplit_max + s;
    float fa, fb;
    merge_stats(M, L, p.ws_ml[base * 2], p.ws_ml[base * 2 + 1], fa, fb);
#pragma unroll
    for (int i = 0; i < 4; ++i) O[i] = merge_val(O[i], p.ws_o[base * D + lane * 4 + i], fa, fb);
  }
  const float inv = L > 0.f ? __frcp_rn(L) : 0.f;
  __nv_bfloat16* out = p.o + w * D + lane * 4;
  *reinterpret_cast<uint32_t*>(out) = pack2(__fmul_rn(O[0], inv), __fmul_rn(O[1], inv));
  *reinterpret_cast<uint32_t*>(out + 2) = pack2(__fmul_rn(O[2], inv), __fmul_rn(O[3], inv));
}

// ---------------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------------
// delta[h, t] = sum_d dO[t,h,d] * O[t,h,d]; one warp per (t, h).
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o,
                                      const __nv_bfloat16* __restrict__ dout,
                                      long long o_stride, long long do_stride, int T, int nq,
                                      float* __restrict__ delta) {
  pdl_trigger();
  pdl_wait();
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)T * nq) return;
  const int t = (int)(w / nq), h = (int)(w % nq);
  const __nv_bfloat16* a = o + (long long)t * o_stride + (long long)h * D + lane * 4;
  const __nv_bfloat16* b = dout + (long long)t * do_stride + (long long)h * D + lane * 4;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) s += __bfloat162float(a[i]) * __bfloat162float(b[i]);
  s = warp_sum(s);
  if (lane == 0) delta[(long long)h * T + t] = s;
}

}  // namespace attn
}  // namespace mb

using namespace mb::attn;
using mb::mb_launch;

// Forward: tcgen05 kernel of csrc/attention_sm100.cu over 128-row tiles (tile_seq/tile_idx).
extern "C" int mb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                           const int* cu_seqlens, const int* tile_seq, const int* tile_idx,
                           int ntiles, long long q_stride, long long k_stride, long long v_stride,
                           long long o_stride, int nq, int nkv, int T, float softmax_scale,
                           int* err, cudaStream_t st) {
  return mb_fa_fwd(q, k, v, o, lse, cu_seqlens, tile_seq, tile_idx, ntiles, q_stride, k_stride,
                   v_stride, o_stride, nq, nkv, T, softmax_scale, err, st);
}

// Number of 1024-key chunks a decode over `max_pages` 64-token pages can need (workspace sizing).
extern "C" int mb_attn_decode_nsplit(int max_pages) { return (max_pages + 15) / 16; }

// ws_o: float [B, nq, nsplit_max, 128]; ws_ml: float [B, nq, nsplit_max, 2] (only touched when a
// sequence spans more than one 1024-key chunk). num_slots = rows of the caches.
extern "C" int mb_attn_decode(const void* q, const void* kc, const void* vc, void* o,
                              const int* page_table, const int* ctx_lens, int B, int max_pages,
                              long long num_slots, int nq, int nkv, float softmax_scale,
                              float* ws_o, float* ws_ml, int* err, cudaStream_t st) {
  if (B == 0) return 0;
  int rc = mb_fa_decode(q, kc, vc, o, page_table, ctx_lens, B, max_pages, num_slots, nq, nkv,
                        softmax_scale, ws_o, ws_ml, err, st);
  if (rc) return rc;
  const int nsplit_max = mb_attn_decode_nsplit(max_pages);
  if (nsplit_max > 1) {
    CombineParams p{(__nv_bfloat16*)o, ctx_lens, ws_o, ws_ml, nq, nsplit_max};
    const long long w = (long long)B * nq;
    mb_launch(attn_decode_combine_kernel, (unsigned)((w + 7) / 8), 256, 0, st, p, B);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                           const void* dout, const float* lse, float* delta, void* dq, void* dk,
                           void* dv, const int* cu_seqlens, const int* blk_seq, const int* blk_idx,
                           int nblocks, long long q_stride, long long k_stride, long long v_stride,
                           long long o_stride, long long do_stride, long long dq_stride,
                           long long dk_stride, long long dv_stride, int nq, int nkv, int T,
                           float softmax_scale, int* err, cudaStream_t st) {
  // blk_seq / blk_idx: the 128-row tile table of the forward (tcgen05 backward kernels)
  if (nblocks == 0) return 0;
  if (nq % nkv) return -1;
  const long long warps = (long long)T * nq;
  mb_launch(attn_bwd_delta_kernel, (unsigned)((warps + 7) / 8), 256, 0, st, 
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, o_stride, do_stride, T, nq, delta);
  return mb_fa_bwd(q, k, v, dout, lse, delta, dq, dk, dv, cu_seqlens, blk_seq, blk_idx, nblocks,
                   q_stride, k_stride, v_stride, do_stride, dq_stride, dk_stride, dv_stride, nq,
                   nkv, T, softmax_scale, err, st);
}

// =============================================================================================
// Allocation-free decode attention.
//
// Some callers cannot allocate device memory at the point where they run decode attention:
// code executing inside another framework's memory pool or under a strict memory budget, and
// C/C++ hosts that link this library without a caching allocator (calling cudaMalloc there
// would synchronise the device or fail once the pool has claimed the GPU). For them this entry
// point takes only inputs and outputs; the split-KV workspace that mb_attn_decode receives from
// its caller lives instead in the fixed device array below.
//
//  * Limit: kNoAllocWsFloats floats (4 MiB) shared by the partial outputs and the (m, l)
//    pairs; a call needing more (B * nq * nsplit * 130 floats, nsplit = ceil(max_pages / 16))
//    is rejected with MB_NOALLOC_TOO_LARGE before anything is launched.
//  * Every GPU that loads the library holds the array until the process exits.
//  * Set-up: the first call on each device (with that device current) resolves the array's
//    device address with cudaGetSymbolAddress and caches it; make that first call before any
//    stream capture starts.
//  * The array is shared by every call and keeps the last call's contents. No part of it has
//    to start at zero (each call writes every slot it later reads), but calls whose kernels
//    overlap on the GPU (different streams, no ordering) race on it: order them.
// =============================================================================================
//  * Errors inside the kernels (a bounded wait that ran out: code 2) are recorded in a fixed
//    device int beside the workspace; read it with mb_attn_decode_noalloc_error (which also
//    clears it). It is zero until a kernel reports something.
constexpr long long kNoAllocWsFloats = 1ll << 20;
static __device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
static __device__ int g_noalloc_err;
static float* g_noalloc_ws_ptr[128] = {nullptr};
static int* g_noalloc_err_ptr[128] = {nullptr};

// Resolves (once per device, with that device current) the device addresses of the fixed
// workspace and error word. Returns 0, or -10 / -11 on a device or symbol lookup failure.
static int noalloc_setup(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return -10;
  if (g_noalloc_ws_ptr[dev] == nullptr) {
    void* ws = nullptr;
    void* e = nullptr;
    if (cudaGetSymbolAddress(&ws, g_noalloc_ws) != cudaSuccess || ws == nullptr) return -11;
    if (cudaGetSymbolAddress(&e, g_noalloc_err) != cudaSuccess || e == nullptr) return -11;
    g_noalloc_err_ptr[dev] = static_cast<int*>(e);
    g_noalloc_ws_ptr[dev] = static_cast<float*>(ws);
  }
  *dev_out = dev;
  return 0;
}

// Copies the error word of the current device into *code (0 = no error) and clears it. Ordered
// on stream `st` and synchronous with it (it waits for the stream's earlier work).
extern "C" int mb_attn_decode_noalloc_error(int* code, cudaStream_t st) {
  int dev = 0;
  const int rc = noalloc_setup(&dev);
  if (rc) return rc;
  if (cudaMemcpyAsync(code, g_noalloc_err_ptr[dev], sizeof(int), cudaMemcpyDeviceToHost, st) !=
      cudaSuccess)
    return -12;
  if (cudaMemsetAsync(g_noalloc_err_ptr[dev], 0, sizeof(int), st) != cudaSuccess) return -12;
  return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -12;
}

extern "C" int mb_attn_decode_noalloc(const void* q, const void* kc, const void* vc, void* o,
                                      const int* page_table, const int* ctx_lens, int B,
                                      int max_pages, long long num_slots, int nq, int nkv,
                                      float softmax_scale, cudaStream_t st) {
  if (B == 0) return 0;
  const long long nsplit = mb_attn_decode_nsplit(max_pages);
  const long long need = nsplit > 1 ? (long long)B * nq * nsplit * (D + 2) : 0;
  if (need > kNoAllocWsFloats) return -9;  // MB_NOALLOC_TOO_LARGE
  int dev = 0;
  const int rc = noalloc_setup(&dev);
  if (rc) return rc;
  float* ws_o = g_noalloc_ws_ptr[dev];
  float* ws_ml = ws_o + (long long)B * nq * nsplit * D;
  return mb_attn_decode(q, kc, vc, o, page_table, ctx_lens, B, max_pages, num_slots, nq, nkv,
                        softmax_scale, ws_o, ws_ml, g_noalloc_err_ptr[dev], st);
}
