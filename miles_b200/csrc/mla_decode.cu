// Absorbed multi-head latent attention decode over the paged latent cache (sm_100a).
//
// For sequence b and head h, with q_lat = W_uk^T q_nope (latent query, r wide) and the rotary
// query q_pe (dr wide), every cached token t (row [c_t | k_pe_t | ...] of the cache) scores
//     s_t = (q_lat . c_t + q_pe . k_pe_t) * scale (+ bias[b, t])
// and the output is the latent mix o_lat = sum_t softmax(s)_t c_t (W_uv is applied outside).
// One CTA per (sequence, head): the scores of the whole context live in shared memory (one
// float per cached token), pass 1 computes them (one key per thread at a time, bf16 rows read
// as 16-byte vectors), pass 2 mixes the latent rows with the threads spread over the r latent
// columns (each key's row is read contiguously across the CTA). The cache is read straight
// through the page table: nothing is gathered or expanded per head.
//
// Reference role: SGLang's MLA decode backends (FlashMLA / flashinfer MLA) serving the
// reference's DeepSeek-V3 / GLM-5 rollouts.
#include "common.cuh"

namespace mb {

__global__ void mla_decode_kernel(const float* __restrict__ q_lat, const float* __restrict__ q_pe,
                                  const __nv_bfloat16* __restrict__ cache, long long row_stride,
                                  const int* __restrict__ page_table, int max_pages,
                                  const int* __restrict__ ctx_lens, const float* __restrict__ bias,
                                  long long bias_stride, int nh, int r, int dr, float scale,
                                  float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sh[];
  float* q = sh;                 // r + dr
  float* sc = sh + r + dr;       // one score per cached token
  __shared__ float red[32];
  const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const long long bh = (long long)b * nh + h;
  for (int i = tid; i < r; i += nt) q[i] = q_lat[bh * r + i];
  for (int i = tid; i < dr; i += nt) q[r + i] = q_pe[bh * dr + i];
  __syncthreads();
  const int L = min(ctx_lens[b], max_pages * 64);  // never past the page-table row
  const int* pt = page_table + (long long)b * max_pages;
  // pass 1: scores and their max
  float mx = -INFINITY;
  for (int t = tid; t < L; t += nt) {
    const __nv_bfloat16* row = cache + ((long long)pt[t >> 6] * 64 + (t & 63)) * row_stride;
    float s = 0.f;
    for (int c = 0; c < r + dr; c += 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + c);
      const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int u = 0; u < 8; ++u) s += q[c + u] * __bfloat162float(vb[u]);
    }
    s *= scale;
    if (bias) s += bias[(long long)b * bias_stride + t];
    sc[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int w = 0; w < (nt + 31) / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int t = tid; t < L; t += nt) {
    const float p = sc[t] == -INFINITY ? 0.f : expf(sc[t] - mx);
    sc[t] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  if ((tid & 31) == 0) red[tid >> 5] = sum;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < (nt + 31) / 32; ++w) tot += red[w];
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  // pass 2: latent mix, threads over the latent columns
  for (int c = tid; c < r; c += nt) {
    float acc = 0.f;
    for (int t = 0; t < L; ++t) {
      const float p = sc[t];
      if (p == 0.f) continue;
      const __nv_bfloat16* row = cache + ((long long)pt[t >> 6] * 64 + (t & 63)) * row_stride;
      acc += p * __bfloat162float(row[c]);
    }
    out[bh * r + c] = acc * inv;
  }
}

}  // namespace mb

using namespace mb;

// Largest context one call serves: the per-token scores sit in shared memory.
static constexpr int kMlaMaxCtx = 48 * 1024;  // 192 KB of fp32 scores

extern "C" int mb_mla_decode(const float* q_lat, const float* q_pe, const void* cache,
                             long long row_stride, const int* page_table, int max_pages,
                             const int* ctx_lens, const float* bias, long long bias_stride, int B,
                             int nh, int r, int dr, float scale, float* out, cudaStream_t st) {
  if (B == 0) return 0;
  if ((r + dr) % 8 || row_stride % 8 || max_pages * 64 > kMlaMaxCtx) return -1;
  if (reinterpret_cast<uintptr_t>(cache) % 16) return -1;
  const size_t smem = (size_t)(r + dr + max_pages * 64) * sizeof(float);
  if (smem > 200 * 1024) return -1;
  if (cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           200 * 1024) != cudaSuccess)
    return -2;
  mb_launch(mla_decode_kernel, dim3(B, nh), dim3(256), smem, st, q_lat, q_pe,
            (const __nv_bfloat16*)cache, row_stride, page_table, max_pages, ctx_lens, bias,
            bias_stride, nh, r, dr, scale, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
