// Gated DeltaNet decode step (sm_100a): one token per sequence advances the recurrent state
// in place and produces the head outputs.
//
//   S' = exp(g) S;  e = beta (v - S'^T k);  S'' = S' + k e^T;  o = S''^T q * scale
//
// One CTA per (sequence, value head), one thread per value column j: the thread walks its
// column of the [dk, dv] fp32 state twice (k . S' first, then the update and q . S''), so the
// state is read twice and written once with coalesced accesses across the CTA and never has
// to fit in registers or shared memory. q / k (already L2-normalised and repeated to the value
// heads) are staged in shared memory.
//
// Reference role: the recurrent decode step of the fla gated-delta-rule kernels used by the
// reference's Qwen3-Next support (miles_plugins/models/qwen3_next.py).
#include "common.cuh"

namespace mb {

__global__ void gdn_decode_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                  const float* __restrict__ v, const float* __restrict__ beta,
                                  const float* __restrict__ g, const long long* __restrict__ rows,
                                  float* __restrict__ S, float* __restrict__ out, int nv, int dk,
                                  int dv, float scale) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sh[];
  float* qs = sh;
  float* ks = sh + dk;
  const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const long long bh = (long long)b * nv + h;
  for (int i = threadIdx.x; i < dk; i += blockDim.x) {
    qs[i] = q[bh * dk + i];
    ks[i] = k[bh * dk + i];
  }
  __syncthreads();
  if (j >= dv) return;
  const float eg = expf(g[bh]);
  const float bt = beta[bh];
  float* col = S + (rows[b] * nv + h) * (long long)dk * dv + j;
  float kS = 0.f;
  for (int i = 0; i < dk; ++i) kS += ks[i] * (col[(long long)i * dv] * eg);
  const float e = bt * (v[bh * dv + j] - kS);
  float o = 0.f;
  for (int i = 0; i < dk; ++i) {
    const float s = col[(long long)i * dv] * eg + ks[i] * e;
    col[(long long)i * dv] = s;
    o += qs[i] * s;
  }
  out[bh * dv + j] = o * scale;
}

}  // namespace mb

using namespace mb;

extern "C" int mb_gdn_decode(const float* q, const float* k, const float* v, const float* beta,
                             const float* g, const long long* rows, float* S, float* out, int B,
                             int nv, int dk, int dv, float scale, cudaStream_t st) {
  if (B == 0) return 0;
  if (dv < 1 || dv > 1024 || dk < 1 || dk > 4096) return -1;
  const int threads = (dv + 31) / 32 * 32;
  mb_launch(gdn_decode_kernel, dim3(B, nv), dim3(threads), (size_t)2 * dk * sizeof(float), st, q, k,
            v, beta, g, rows, S, out, nv, dk, dv, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
