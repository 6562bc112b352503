// Mixture-of-experts routing kernels (sm_100a): router top-k (softmax or sigmoid-grouped, fp32),
// replayed routing (Rollout Routing Replay), deterministic token permutation into
// expert-sorted, 128-row padded segments, and the weighted combine. Every ordering decision is
// a pure function of (token, slot): ranks inside an expert follow token order, and the combine
// sums the k expert outputs of a token in slot order, so MoE layers are bitwise reproducible.
//
// Reference roles replaced: Megatron TopKRouter / topk_routing_with_score_function with the R3
// hook (megatron.patch:514-541), moe_align_block_size + fused_moe permute/sum-reduce
// (fsdp_utils/kernels/fused_experts.py:15-200,360-381).
#include "common.cuh"

namespace mb {

constexpr int kMaxE = 256;
constexpr int kMaxK = 16;

// One warp per token. score_fn 0: softmax over E, top-k, optional renorm.
// score_fn 1: sigmoid scores; selection by (score + bias) restricted to the best `topk_group`
// of `n_group` groups (group score = sum of its top-2 biased scores); weights are the unbiased
// sigmoid scores of the selected experts, renormalised if `renorm`, times `scale`.
// replay: when idx_in != nullptr the selection is read from it (R3) instead of computed.
// Routing of token t by one warp (all 32 lanes call it). `gscore` is 32 floats of shared
// memory owned by the calling warp (group scores of the group-limited selection). Both the
// training router kernel and the fused decode route+dispatch kernel use this function, so
// their selections and weights are bitwise equal.
__device__ __forceinline__ void route_token(const float* __restrict__ logits,
                                            const float* __restrict__ bias,
                                            const int* __restrict__ idx_in, int* __restrict__ idx_out,
                                            float* __restrict__ w_out, int t, int E, int k,
                                            int score_fn, int renorm, int n_group, int topk_group,
                                            float scale, float* gscore, int lane) {
  constexpr int PER = kMaxE / 32;
  const int per = (E + 31) / 32;
  float sc[PER], sel[PER];
  const float* lr = logits + (long long)t * E;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    sc[i] = (i < per && e < E) ? lr[e] : -INFINITY;
    mx = fmaxf(mx, sc[i]);
  }
  if (score_fn == 0) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      sc[i] = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - mx);
      s += sc[i];
    }
    s = warp_sum(s);
    const float inv = 1.f / s;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      sc[i] *= inv;
      const int e = i * 32 + lane;
      sel[i] = (i < per && e < E) ? sc[i] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      const bool ok = i < per && e < E;
      sc[i] = ok ? 1.f / (1.f + expf(-sc[i])) : 0.f;
      sel[i] = ok ? sc[i] + (bias ? bias[e] : 0.f) : -INFINITY;
    }
    if (n_group > 1) {
      const int gsz = E / n_group;
      for (int g = 0; g < n_group; ++g) {
        float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int e = i * 32 + lane;
          if (i < per && e < E && e / gsz == g) {
            const float v = sel[i];
            if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
          }
        }
        for (int o = 16; o > 0; o >>= 1) {  // warp top-2 merge
          const float o1 = __shfl_xor_sync(0xffffffff, b1, o);
          const float o2 = __shfl_xor_sync(0xffffffff, b2, o);
          const float n1 = fmaxf(b1, o1);
          const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
          b1 = n1; b2 = n2;
        }
        if (lane == 0) gscore[g] = b1 + b2;
      }
      __syncwarp();
      unsigned keep = 0;  // best topk_group groups, ties -> lower group index
      if (lane == 0) {
        for (int r = 0; r < topk_group; ++r) {
          int best = -1;
          float bv = -INFINITY;
          for (int g = 0; g < n_group; ++g)
            if (!((keep >> g) & 1u) && (best < 0 || gscore[g] > bv)) { best = g; bv = gscore[g]; }
          keep |= 1u << best;
        }
      }
      keep = __shfl_sync(0xffffffff, keep, 0);
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        if (i < per && e < E && !((keep >> (e / gsz)) & 1u)) sel[i] = -INFINITY;
      }
    }
  }
  int chosen[kMaxK];
  float wsel[kMaxK];
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    int e_best;
    if (idx_in) {
      e_best = idx_in[(long long)t * k + j];
    } else {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        if (sel[i] > bv || (sel[i] == bv && e < bi)) { bv = sel[i]; bi = e; }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffff, bv, o);
        const int oi = __shfl_xor_sync(0xffffffff, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      e_best = bi;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (i * 32 + lane == e_best) sel[i] = -INFINITY;
    }
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == e_best) v = sc[i];
    v = __shfl_sync(0xffffffff, v, e_best & 31);
    chosen[j] = e_best;
    wsel[j] = v;
    wsum += v;
  }
  if (lane == 0) {
    const float inv = renorm ? 1.f / wsum : 1.f;
    for (int j = 0; j < k; ++j) {
      idx_out[(long long)t * k + j] = chosen[j];
      w_out[(long long)t * k + j] = wsel[j] * inv * scale;
    }
  }
}

__global__ void router_fwd_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                  const int* __restrict__ idx_in, int* __restrict__ idx_out,
                                  float* __restrict__ w_out, int T, int E, int k, int score_fn,
                                  int renorm, int n_group, int topk_group, float scale) {
  pdl_trigger();
  pdl_wait();
  __shared__ float gscore_sh[32][32];
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  route_token(logits, bias, idx_in, idx_out, w_out, t, E, k, score_fn, renorm, n_group,
              topk_group, scale, gscore_sh[threadIdx.x / 32], lane);
}

// Backward of router_fwd (softmax or sigmoid) to d(logits), written as bf16 for the router GEMM.
__global__ void router_bwd_kernel(const float* __restrict__ logits, const int* __restrict__ idx,
                                  const float* __restrict__ dw, __nv_bfloat16* __restrict__ dlogits,
                                  int T, int E, int k, int score_fn, int renorm, float scale) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  constexpr int PER = kMaxE / 32;
  const int per = (E + 31) / 32;
  const float* lr = logits + (long long)t * E;
  float sc[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    sc[i] = (i < per && e < E) ? lr[e] : -INFINITY;
    mx = fmaxf(mx, sc[i]);
  }
  if (score_fn == 0) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      sc[i] = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - mx);
      s += sc[i];
    }
    s = warp_sum(s);
#pragma unroll
    for (int i = 0; i < PER; ++i) sc[i] /= s;
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) sc[i] = (sc[i] == -INFINITY) ? 0.f : 1.f / (1.f + expf(-sc[i]));
  }
  float S = 0.f, dot = 0.f;
  float pj[kMaxK], gj[kMaxK];
  int ej[kMaxK];
  for (int j = 0; j < k; ++j) {
    ej[j] = idx[(long long)t * k + j];
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == ej[j]) v = sc[i];
    pj[j] = __shfl_sync(0xffffffff, v, ej[j] & 31);
    gj[j] = dw[(long long)t * k + j] * scale;
    S += pj[j];
  }
  for (int j = 0; j < k; ++j) dot += gj[j] * pj[j];
  float dp[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) dp[i] = 0.f;
  for (int j = 0; j < k; ++j) {
    const float d = renorm ? (gj[j] - dot / S) / S : gj[j];
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == ej[j]) dp[i] += d;
  }
  if (score_fn == 0) {
    float sdp = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) sdp += sc[i] * dp[i];
    sdp = warp_sum(sdp);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (i < per && e < E) dlogits[(long long)t * E + e] = __float2bfloat16(sc[i] * (dp[i] - sdp));
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (i < per && e < E)
        dlogits[(long long)t * E + e] = __float2bfloat16(dp[i] * sc[i] * (1.f - sc[i]));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Deterministic permutation. Entries i = t*k + j (token t, slot j) with expert idx[i].
//  1. chunk histograms  hist[c][e]
//  2. scan: counts, 128-padded offsets[E+1], chunk_base[c][e]
//  3. scatter: dest[i] = chunk_base[c][e] + (entries before i in chunk c with expert e)
// ---------------------------------------------------------------------------------------------
constexpr int kChunk = 1024;

__global__ void moe_hist_kernel(const int* __restrict__ idx, int n, int E, int* __restrict__ hist) {
  pdl_trigger();
  pdl_wait();
  __shared__ int h[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int i = blockIdx.x * kChunk + threadIdx.x;
  if (i < n && MB_GUARD(idx[i] >= 0 && idx[i] < E, 42)) atomicAdd(&h[idx[i]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[blockIdx.x * E + e] = h[e];
}

__global__ void moe_scan_kernel(const int* __restrict__ hist, int nchunks, int E, int align,
                                int* __restrict__ counts, int* __restrict__ offsets,
                                int* __restrict__ chunk_base) {
  pdl_trigger();
  pdl_wait();
  __shared__ int padded[kMaxE + 1];
  const int e = threadIdx.x;
  int total = 0;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) total += hist[c * E + e];
    counts[e] = total;
    padded[e] = (total + align - 1) / align * align;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      const int p = padded[i];
      offsets[i] = acc;
      acc += p;
    }
    offsets[E] = acc;
  }
  __syncthreads();
  if (e < E) {
    int run = offsets[e];
    for (int c = 0; c < nchunks; ++c) {
      chunk_base[c * E + e] = run;
      run += hist[c * E + e];
    }
  }
}

__global__ void moe_scatter_kernel(const int* __restrict__ idx, int n, int E,
                                   const int* __restrict__ chunk_base, int* __restrict__ dest) {
  pdl_trigger();
  pdl_wait();
  __shared__ int wcnt[32][kMaxE];
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wcnt[i / E][i % E] = 0;
  __syncthreads();
  const int i = blockIdx.x * kChunk + threadIdx.x;
  const bool valid = i < n;
  const int e = valid ? idx[i] : -1 - lane;  // distinct dummies never match real experts
  const unsigned peers = __match_any_sync(0xffffffff, e);
  const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
  if (valid && rank_in_warp == 0) wcnt[wid][e] = __popc(peers);
  __syncthreads();
  if (valid) {
    int base = chunk_base[blockIdx.x * E + e];
    for (int w = 0; w < wid; ++w) base += wcnt[w][e];
    dest[i] = base + rank_in_warp;
  }
}

// Zero the padding rows of every expert segment: [offsets[e] + counts[e], offsets[e+1]).
__global__ void moe_zero_pad_kernel(const int* __restrict__ counts, const int* __restrict__ offsets,
                                    __nv_bfloat16* __restrict__ buf, int H) {
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x;
  const int r0 = offsets[e] + counts[e], r1 = offsets[e + 1];
  const int nvec = H / 8;
  for (int r = r0; r < r1; ++r)
    for (int c = threadIdx.x; c < nvec; c += blockDim.x)
      reinterpret_cast<uint4*>(buf + (long long)r * H)[c] = make_uint4(0, 0, 0, 0);
}

// x_sorted[dest[t*k+j]] = x[t]; one warp per entry.
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ dest,
                                  int n, int k, int H, __nv_bfloat16* __restrict__ xs, int rows) {
  pdl_trigger();
  pdl_wait();
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  if (!MB_GUARD(dest[w] >= 0 && dest[w] < rows, 41)) return;  // destination row outside xs
  const int t = (int)(w / k);
  const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * H);
  uint4* dst = reinterpret_cast<uint4*>(xs + (long long)dest[w] * H);
  for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

// dx[t] = sum_j dxs[dest[t*k+j]] (slot order), one warp per (token, 256-column chunk). The k
// row indices and then the k rows are loaded before the sum (independent loads in flight
// instead of a dependent index -> row chain per slot); the sum order is unchanged.
constexpr int kGatherMaxK = 8;
__global__ void moe_gather_bwd_kernel(const __nv_bfloat16* __restrict__ dxs,
                                      const int* __restrict__ dest, int T, int k, int H,
                                      __nv_bfloat16* __restrict__ dx) {
  pdl_trigger();
  pdl_wait();
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nch = H / 256;
  if (gw >= (long long)T * nch) return;
  const int t = (int)(gw / nch);
  const int c = (int)(gw % nch) * 256 + lane * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j0 = 0; j0 < k; j0 += kGatherMaxK) {
    long long row[kGatherMaxK];
    uint4 v[kGatherMaxK];
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j)
      if (j0 + j < k) row[j] = __ldg(dest + (long long)t * k + j0 + j);
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j)
      if (j0 + j < k) v[j] = *reinterpret_cast<const uint4*>(dxs + row[j] * H + c);
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j) {
      if (j0 + j >= k) break;
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v[j]);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(b[q]);
    }
  }
  uint4 o;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(acc[q]);
  *reinterpret_cast<uint4*>(dx + (long long)t * H + c) = o;
}

// y[t] = sum_j w[t,j] * ys[dest[t*k+j]] (+ add[t]); fp32 accumulation in slot order.
// One warp per (token, 256-column chunk) so small decode batches still spread over the GPU.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ ys, const int* __restrict__ dest,
                                   const float* __restrict__ w, const __nv_bfloat16* __restrict__ add,
                                   int T, int k, int H, __nv_bfloat16* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nch = H / 256;
  if (gw >= (long long)T * nch) return;
  const int t = (int)(gw / nch);
  const int c = (int)(gw % nch) * 256 + lane * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  // indices and weights, then rows, all in flight before the slot-ordered sum
  for (int j0 = 0; j0 < k; j0 += kGatherMaxK) {
    long long row[kGatherMaxK];
    float wj[kGatherMaxK];
    uint4 v[kGatherMaxK];
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j)
      if (j0 + j < k) {
        row[j] = __ldg(dest + (long long)t * k + j0 + j);
        wj[j] = __ldg(w + (long long)t * k + j0 + j);
      }
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j)
      if (j0 + j < k) v[j] = *reinterpret_cast<const uint4*>(ys + row[j] * H + c);
#pragma unroll
    for (int j = 0; j < kGatherMaxK; ++j) {
      if (j0 + j >= k) break;
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v[j]);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wj[j] * __bfloat162float(b[q]);
    }
  }
  if (add) {
    const uint4 v = *reinterpret_cast<const uint4*>(add + (long long)t * H + c);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(b[q]);
  }
  uint4 o;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(acc[q]);
  *reinterpret_cast<uint4*>(y + (long long)t * H + c) = o;
}

// Backward of the combine: dys[dest] = w * dy[t]; dw[t,j] = <dy[t], ys[dest]>. One warp/token.
__global__ void moe_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                       const __nv_bfloat16* __restrict__ ys,
                                       const int* __restrict__ dest, const float* __restrict__ w,
                                       int T, int k, int H, __nv_bfloat16* __restrict__ dys,
                                       float* __restrict__ dw) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int j = 0; j < k; ++j) {
    const long long r = dest[t * k + j];
    const float wj = w[t * k + j];
    float dot = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 g = *reinterpret_cast<const uint4*>(dy + (long long)t * H + c);
      const uint4 v = *reinterpret_cast<const uint4*>(ys + r * H + c);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&g);
      const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float gv = __bfloat162float(gb[q]);
        dot += gv * __bfloat162float(vb[q]);
        ob[q] = __float2bfloat16(wj * gv);
      }
      *reinterpret_cast<uint4*>(dys + r * H + c) = o;
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[t * k + j] = dot;
  }
}

}  // namespace mb

using namespace mb;


// ---------------------------------------------------------------------------------------------
// Fused routing + dispatch for small batches (decode): one launch replaces router top-k,
// histogram, scan, scatter and gather. Every CTA routes all T tokens itself (route_token, the
// training router's arithmetic) and builds the whole plan in shared memory; CTA 0 publishes
// idx / weights / counts / offsets / dest, and the CTAs split the row gather. Row order inside
// an expert segment is ascending (token, slot), as in the multi-kernel plan.
// Shared memory: idx[n] | dest[n] | w[n] | cnt[E] | run[E] | offs[E+1] | wc[8][E].
// ---------------------------------------------------------------------------------------------
constexpr int kRDWarps = 8;
constexpr int kRDMaxN = 4096;

__global__ void __launch_bounds__(kRDWarps * 32)
moe_route_dispatch_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                          const int* __restrict__ idx_in, const __nv_bfloat16* __restrict__ x,
                          int T, int E, int k, int H, int score_fn, int renorm, int n_group,
                          int topk_group, float scale, int align, int* __restrict__ idx_out,
                          float* __restrict__ w_out, int* __restrict__ counts_out,
                          int* __restrict__ offsets_out, int* __restrict__ dest_out,
                          __nv_bfloat16* __restrict__ xs) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int rd_smem[];
  const int n = T * k;
  int* idx_s = rd_smem;
  int* dest_s = idx_s + n;
  float* w_s = reinterpret_cast<float*>(dest_s + n);
  int* cnt = reinterpret_cast<int*>(w_s + n);
  int* run = cnt + E;
  int* offs = run + E;
  int* wc = offs + E + 1;  // [kRDWarps][E]
  __shared__ float gscore_sh[kRDWarps][32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool routed = logits == nullptr;  // idx_out already holds the routing (plan + gather only)
  if (routed) {
    for (int i = tid; i < n; i += blockDim.x) idx_s[i] = idx_out[i];
  } else {
    for (int t = warp; t < T; t += kRDWarps)
      route_token(logits, bias, idx_in, idx_s, w_s, t, E, k, score_fn, renorm, n_group,
                  topk_group, scale, gscore_sh[warp], lane);
  }
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  for (int i = tid; i < kRDWarps * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) atomicAdd(&cnt[idx_s[i]], 1);
  __syncthreads();
  {  // exclusive scan of the padded counts: per-warp shuffle scan, then warp totals in order
    const int pc = tid < E ? (cnt[tid] + align - 1) / align * align : 0;
    int incl = pc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffff, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) wc[warp] = incl;  // wc is free until the rank loop (re-zeroed below)
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wc[w];
    if (tid < E) {
      offs[tid] = before + incl - pc;
      run[tid] = before + incl - pc;
    }
    if (tid == E - 1) offs[E] = before + incl;
    __syncthreads();
    if (tid < kRDWarps) wc[tid] = 0;
    __syncthreads();
  }
  // stable ranks, one block-sized chunk of entries at a time
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    const bool valid = i < n;
    const int e = valid ? idx_s[i] : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffff, e);
    const int r = __popc(peers & ((1u << lane) - 1u));
    if (valid && r == 0) wc[warp * E + e] = __popc(peers);
    __syncthreads();
    if (valid) {
      int b = run[e];
      for (int w = 0; w < warp; ++w) b += wc[w * E + e];
      dest_s[i] = b + r;
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kRDWarps; ++w) {
        add += wc[w * E + ee];
        wc[w * E + ee] = 0;
      }
      run[ee] += add;
    }
    __syncthreads();
  }
  // every CTA has read idx_out (when pre-routed) before this point: the grid never writes it then
  if (blockIdx.x == 0) {
    for (int i = tid; i < n; i += blockDim.x) {
      if (!routed) {
        idx_out[i] = idx_s[i];
        w_out[i] = w_s[i];
      }
      dest_out[i] = dest_s[i];
    }
    for (int e = tid; e < E; e += blockDim.x) counts_out[e] = cnt[e];
    if (tid == 0) offsets_out[E] = offs[E];
    for (int e = tid; e < E; e += blockDim.x) offsets_out[e] = offs[e];
  }
  // gather: CTA b copies rows b, b + gridDim.x, ...
  const int nvec = H / 8;
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)(i / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(xs + (long long)dest_s[i] * H);
    for (int c = tid; c < nvec; c += blockDim.x) dst[c] = src[c];
  }
}

extern "C" int mb_router_fwd(const float* logits, const float* bias, const int* idx_in, int* idx_out,
                             float* w_out, int T, int E, int k, int score_fn, int renorm,
                             int n_group, int topk_group, float scale, cudaStream_t st) {
  if (T == 0) return 0;
  if (E > kMaxE || k > kMaxK || (n_group > 1 && (n_group > 32 || E % n_group))) return -1;
  mb_launch(router_fwd_kernel, (T + 7) / 8, 256, 0, st, logits, bias, idx_in, idx_out, w_out, T, E, k,
                                                 score_fn, renorm, n_group, topk_group, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_router_bwd(const float* logits, const int* idx, const float* dw, void* dlogits,
                             int T, int E, int k, int score_fn, int renorm, float scale,
                             cudaStream_t st) {
  if (T == 0) return 0;
  if (E > kMaxE || k > kMaxK) return -1;
  mb_launch(router_bwd_kernel, (T + 7) / 8, 256, 0, st, logits, idx, dw, (__nv_bfloat16*)dlogits, T, E, k,
                                                 score_fn, renorm, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// workspace: hist [nchunks*E], chunk_base [nchunks*E] ints. nchunks = ceil(n / 1024).
extern "C" int mb_moe_permute_plan(const int* idx, int n, int E, int align, int* hist,
                                   int* chunk_base, int* counts, int* offsets, int* dest,
                                   cudaStream_t st) {
  if (E > kMaxE || align <= 0) return -1;
  const int nchunks = (n + kChunk - 1) / kChunk;
  if (n > 0) mb_launch(moe_hist_kernel, nchunks, kChunk, 0, st, idx, n, E, hist);
  mb_launch(moe_scan_kernel, 1, kMaxE, 0, st, hist, n > 0 ? nchunks : 0, E, align, counts, offsets,
                                       chunk_base);
  if (n > 0) mb_launch(moe_scatter_kernel, nchunks, kChunk, 0, st, idx, n, E, chunk_base, dest);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_moe_zero_pad(const int* counts, const int* offsets, void* buf, int E, int H,
                               cudaStream_t st) {
  if (H % 8) return -1;
  mb_launch(moe_zero_pad_kernel, E, 128, 0, st, counts, offsets, (__nv_bfloat16*)buf, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_moe_gather(const void* x, const int* dest, int n, int k, int H, void* xs,
                             int rows, cudaStream_t st) {
  if (n == 0) return 0;
  if (H % 8) return -1;
  mb_launch(moe_gather_kernel, (n + 7) / 8, 256, 0, st, (const __nv_bfloat16*)x, dest, n, k, H,
                                                 (__nv_bfloat16*)xs, rows);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_moe_gather_bwd(const void* dxs, const int* dest, int T, int k, int H, void* dx,
                                 cudaStream_t st) {
  if (T == 0) return 0;
  if (H % 256) return -1;
  const long long wg = (long long)T * (H / 256);
  mb_launch(moe_gather_bwd_kernel, (unsigned)((wg + 7) / 8), 256, 0, st, (const __nv_bfloat16*)dxs, dest, T, k, H,
                                                     (__nv_bfloat16*)dx);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_moe_combine(const void* ys, const int* dest, const float* w, const void* add,
                              int T, int k, int H, void* y, cudaStream_t st) {
  if (T == 0) return 0;
  if (H % 256) return -1;
  const long long wc = (long long)T * (H / 256);
  mb_launch(moe_combine_kernel, (unsigned)((wc + 7) / 8), 256, 0, st, (const __nv_bfloat16*)ys, dest, w,
                                                  (const __nv_bfloat16*)add, T, k, H,
                                                  (__nv_bfloat16*)y);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_moe_combine_bwd(const void* dy, const void* ys, const int* dest, const float* w,
                                  int T, int k, int H, void* dys, float* dw, cudaStream_t st) {
  if (T == 0) return 0;
  if (H % 256) return -1;
  mb_launch(moe_combine_bwd_kernel, (T + 7) / 8, 256, 0, st, (const __nv_bfloat16*)dy,
                                                      (const __nv_bfloat16*)ys, dest, w, T, k, H,
                                                      (__nv_bfloat16*)dys, dw);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Fused route + dispatch for n = T * k <= 4096 (decode batches). Outputs as mb_router_fwd +
// mb_moe_permute_plan + mb_moe_gather (padding rows of xs are not written).
extern "C" int mb_moe_route_dispatch(const float* logits, const float* bias, const int* idx_in,
                                     const void* x, int T, int E, int k, int H, int score_fn,
                                     int renorm, int n_group, int topk_group, float scale,
                                     int align, int* idx_out, float* w_out, int* counts,
                                     int* offsets, int* dest, void* xs, cudaStream_t st) {
  if (T == 0) return 0;
  const int n = T * k;
  if (E > kMaxE || k > kMaxK || n > kRDMaxN || H % 8 || align <= 0 ||
      (n_group > 1 && (n_group > 32 || E % n_group)))
    return -1;
  const size_t smem = (size_t)(3 * n + 3 * E + 1 + kRDWarps * E) * sizeof(int);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(moe_route_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((3 * kRDMaxN + 3 * kMaxE + 1 + kRDWarps * kMaxE) * sizeof(int))) != cudaSuccess)
      return -3;
    attr = true;
  }
  // one row per CTA up to the SM count: the plan is rebuilt redundantly per CTA (cheap), the
  // gather latency is not
  const int grid = n < 148 ? n : 148;
  // Every CTA routes all T tokens itself; past one warp-pass of tokens that redundant work
  // costs more than a separate, fully parallel router launch, so larger batches route first and
  // run this kernel for the plan + gather only.
  if (T > kRDWarps) {
    mb_launch(router_fwd_kernel, (T + 7) / 8, 256, 0, st, logits, bias, idx_in, idx_out, w_out,
              T, E, k, score_fn, renorm, n_group, topk_group, scale);
    logits = nullptr;
  }
  mb_launch(moe_route_dispatch_kernel, grid, kRDWarps * 32, smem, st, logits, bias, idx_in,
            (const __nv_bfloat16*)x, T, E, k, H, score_fn, renorm, n_group, topk_group, scale,
            align, idx_out, w_out, counts, offsets, dest, (__nv_bfloat16*)xs);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

MB_CHECK_GETTER(mb_checks_moe)
