// RL-specific kernels (sm_100a): vocab log-softmax / target log-prob / entropy (forward and
// backward), token sampling with the SAME log-softmax reduction (so rollout log-probs equal the
// trainer's bit for bit), the fused PPO/GSPO clipped policy loss with TIS and KL terms, GAE,
// GRPO group advantages, deterministic squared-norm reduction and the Adam update.
//
// Reference roles replaced: ppo_utils.py compute_policy_loss (:124-148), compute_approx_kl
// (:11-51), vocab-parallel log-prob / entropy (:151-194, :687-717), chunked GAE (:505-645),
// the SGLang sampler log-softmax (sglang.patch:500-523) and Megatron's distributed Adam.
#include "common.cuh"

namespace mb {

// ---------------------------------------------------------------------------------------------
// Row statistics of softmax(z * inv_temp): max m, sum s = sum exp(z' - m), sz = sum exp(z'-m) z'.
// One CTA of 512 threads per row; each thread keeps an online (m, s, sz) over a fixed strided
// subset, then a fixed-order tree combines them. Shared by the trainer's log-prob kernel and
// the rollout sampler: identical inputs give identical lse bits.
// ---------------------------------------------------------------------------------------------
constexpr int LS_THREADS = 512;

struct SoftStats {
  float m, s, sz;
};

MB_DEVICE SoftStats combine(SoftStats a, SoftStats b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  if (a.m >= b.m) {
    const float f = __expf(b.m - a.m);
    return {a.m, a.s + b.s * f, a.sz + b.sz * f};
  }
  const float f = __expf(a.m - b.m);
  return {b.m, b.s + a.s * f, b.sz + a.sz * f};
}

MB_DEVICE SoftStats row_stats(const float* __restrict__ z, int V, float inv_temp) {
  __shared__ SoftStats sh[LS_THREADS];
  SoftStats st{-INFINITY, 0.f, 0.f};
  for (int i = threadIdx.x; i < V; i += LS_THREADS) {
    const float x = z[i] * inv_temp;
    if (x > st.m) {
      const float f = (st.m == -INFINITY) ? 0.f : __expf(st.m - x);
      st.s = st.s * f + 1.f;
      st.sz = st.sz * f + x;
      st.m = x;
    } else {
      const float e = __expf(x - st.m);
      st.s += e;
      st.sz += e * x;
    }
  }
  sh[threadIdx.x] = st;
  __syncthreads();
  for (int off = LS_THREADS / 2; off > 0; off >>= 1) {
    if (threadIdx.x < off) sh[threadIdx.x] = combine(sh[threadIdx.x], sh[threadIdx.x + off]);
    __syncthreads();
  }
  const SoftStats r = sh[0];
  __syncthreads();
  return r;
}

// logp[r] = z[t]/T - lse; ent[r] = lse - E_p[z/T]; lse[r] saved for the backward.
__global__ void __launch_bounds__(LS_THREADS) logprob_fwd_kernel(
    const float* __restrict__ logits, long long ld, const int* __restrict__ target, int V,
    float inv_temp, float* __restrict__ logp, float* __restrict__ ent, float* __restrict__ lse) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const float* z = logits + r * ld;
  const SoftStats st = row_stats(z, V, inv_temp);
  if (threadIdx.x == 0) {
    const float l = st.m + logf(st.s);
    if (lse) lse[r] = l;
    if (logp) logp[r] = z[target[r]] * inv_temp - l;
    if (ent) ent[r] = l - st.sz / st.s;
  }
}

// Vocabulary-parallel log-prob, part 1: the softmax statistics of this rank's vocabulary slice
// [lo, lo + V) of every row (row_stats, the same reduction as logprob_fwd_kernel) and the
// target's scaled logit when the target falls in the slice (0 otherwise).
// part = [4][n]: {m, s, sz, tz}. The ranks' parts are then exchanged and combined.
__global__ void __launch_bounds__(LS_THREADS) logprob_part_kernel(
    const float* __restrict__ logits, long long ld, const int* __restrict__ target, int lo, int V,
    float inv_temp, float* __restrict__ part, int n) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const float* z = logits + r * ld;
  const SoftStats st = row_stats(z, V, inv_temp);
  if (threadIdx.x == 0) {
    const int t = target[r] - lo;
    part[r] = st.m;
    part[n + r] = st.s;
    part[2LL * n + r] = st.sz;
    part[3LL * n + r] = (t >= 0 && t < V) ? z[t] * inv_temp : 0.f;
  }
}

// Part 2: combine the parts of `world` slices ([world][4][n], in rank order, the same order on
// every rank, so every rank gets the same bits) into lse, the target log-prob and the entropy.
// With one slice this reproduces logprob_fwd_kernel exactly.
__global__ void logprob_combine_kernel(const float* __restrict__ parts, int world, int n,
                                       float* __restrict__ logp, float* __restrict__ ent,
                                       float* __restrict__ lse) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  SoftStats a{-INFINITY, 0.f, 0.f};
  float tz = 0.f;
  for (int w = 0; w < world; ++w) {
    const float* p = parts + (long long)w * 4 * n;
    a = combine(a, SoftStats{p[r], p[n + r], p[2LL * n + r]});
    tz += p[3LL * n + r];
  }
  const float l = a.m + logf(a.s);
  if (lse) lse[r] = l;
  if (logp) logp[r] = tz - l;
  if (ent) ent[r] = l - a.sz / a.s;
}

// dz_i = inv_temp * [ g_lp (1[i==t] - p_i) - g_ent p_i (z'_i - E_p z') ]  (bf16 output)
__global__ void __launch_bounds__(LS_THREADS) logprob_bwd_kernel(
    const float* __restrict__ logits, long long ld, const int* __restrict__ target, int V,
    float inv_temp, const float* __restrict__ lse, const float* __restrict__ g_lp,
    const float* __restrict__ g_ent, const float* __restrict__ ent,
    __nv_bfloat16* __restrict__ dlogits, long long ldd) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const float* z = logits + r * ld;
  const float l = lse[r];
  const float gl = g_lp ? g_lp[r] : 0.f;
  const float ge = g_ent ? g_ent[r] : 0.f;
  const float ez = ent ? l - ent[r] : 0.f;  // E_p[z'] = lse - H
  const int t = target[r];
  __nv_bfloat16* d = dlogits + r * ldd;
  for (int i = threadIdx.x; i < V; i += LS_THREADS) {
    const float x = z[i] * inv_temp;
    const float p = __expf(x - l);
    float g = gl * ((i == t ? 1.f : 0.f) - p);
    if (ge != 0.f) g -= ge * p * (x - ez);
    d[i] = __float2bfloat16(g * inv_temp);
  }
}

// ---------------------------------------------------------------------------------------------
// Sampling: Gumbel-max over z/T with a counter-based hash RNG (SplitMix64 finaliser, Steele,
// Lea & Flood 2014) keyed by (seed, position, vocab index). Writes the token and its log-prob
// computed from the same row_stats as the trainer. inv_temp <= 0 => greedy argmax.
// ---------------------------------------------------------------------------------------------
MB_DEVICE uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void __launch_bounds__(LS_THREADS) sample_kernel(
    const float* __restrict__ logits, long long ld, int V, const float* __restrict__ inv_temps,
    const unsigned long long* __restrict__ seeds, const int* __restrict__ positions,
    int* __restrict__ tokens, float* __restrict__ logp, const float* __restrict__ thr) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const float* z = logits + r * ld;
  // top-k / top-p: only logits >= thr[r] take part in the draw (the reported log-prob stays the
  // full-distribution one, which is what the trainer computes)
  const float cut = thr ? thr[r] : -INFINITY;
  const float itemp = inv_temps[r];
  const bool greedy = itemp <= 0.f;
  const float it = greedy ? 1.f : itemp;
  __shared__ float bv[LS_THREADS];
  __shared__ int bi[LS_THREADS];
  const uint64_t key = splitmix64(seeds[r] ^ splitmix64((uint64_t)(uint32_t)positions[r] + 0x1234567ull));
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += LS_THREADS) {
    if (z[i] < cut) continue;
    float score = z[i] * it;
    if (!greedy) {
      const uint64_t h = splitmix64(key ^ (uint64_t)i);
      const float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0,1)
      score += -logf(-logf(u));
    }
    if (score > best || (score == best && i < besti)) { best = score; besti = i; }
  }
  bv[threadIdx.x] = best;
  bi[threadIdx.x] = besti;
  __syncthreads();
  for (int off = LS_THREADS / 2; off > 0; off >>= 1) {
    if (threadIdx.x < off) {
      const float ov = bv[threadIdx.x + off];
      const int oi = bi[threadIdx.x + off];
      if (ov > bv[threadIdx.x] || (ov == bv[threadIdx.x] && oi < bi[threadIdx.x])) {
        bv[threadIdx.x] = ov;
        bi[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  const int tok = bi[0];
  const SoftStats st = row_stats(z, V, it);
  if (threadIdx.x == 0) {
    tokens[r] = tok;
    if (logp) logp[r] = z[tok] * it - (st.m + logf(st.s));
  }
}

// ---------------------------------------------------------------------------------------------
// Fused policy loss. Per token i (weight w_i already contains the loss mask and the reduction
// normaliser):
//   ppo_kl = old - logp, ratio = exp(-ppo_kl)
//   pg = max(-A r, -A clip(r, 1-eps, 1+eps_hi)); if eps_c > 1 and A < 0: pg = min(pg, -A eps_c)
//   pg *= tis, a constant: use_tis 1 = TIS (clamp(exp(old - rollout), tis_lo, tis_hi)),
//   use_tis 2 = IcePop (exp(old - rollout) inside [tis_lo, tis_hi], else 0)
//   kl term: kl_coef * KL(logp || ref) of type k1 / k2 / k3 (low_var_kl, clamped to [-10, 10])
// loss = sum_i w_i (pg_i + kl_coef kl_i); dlogp_i = w_i (dpg_i + kl_coef dkl_i).
// Metric partials per block: [sum w*pg, sum w*clipfrac, sum w*ppo_kl, sum w*kl, sum w*tis,
//  sum w*tis_clipped, sum w].
// ---------------------------------------------------------------------------------------------
constexpr int PL_METRICS = 7;

struct PolicyLossParams {
  const float *logp, *old_logp, *adv, *weight, *rollout_logp, *ref_logp;
  float* dlogp;
  float* pg_out;
  float* part;  // [gridDim.x, PL_METRICS]
  int n;
  float eps, eps_hi, eps_c, tis_lo, tis_hi, kl_coef;
  int kl_type;  // 0 none, 1 k1, 2 k2, 3 k3/low_var_kl
  int use_tis;  // 0 off, 1 TIS (clamp), 2 IcePop (mask)
};

__global__ void policy_loss_kernel(const PolicyLossParams p) {
  pdl_trigger();
  pdl_wait();
  float acc[PL_METRICS] = {0, 0, 0, 0, 0, 0, 0};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += gridDim.x * blockDim.x) {
    const float w = p.weight[i];
    const float lp = p.logp[i];
    const float kl_ppo = p.old_logp[i] - lp;
    const float ratio = expf(-kl_ppo);
    const float A = p.adv[i];
    const float pg1 = -A * ratio;
    const float rc = fminf(fmaxf(ratio, 1.f - p.eps), 1.f + p.eps_hi);
    const float pg2 = -A * rc;
    float pg, dpg;
    if (pg1 >= pg2) { pg = pg1; dpg = -A * ratio; } else { pg = pg2; dpg = (rc == ratio) ? -A * ratio : 0.f; }
    const float clipped = pg2 > pg1 ? 1.f : 0.f;
    if (p.eps_c > 1.f && A < 0.f) {
      const float pg3 = -A * p.eps_c;
      if (pg3 < pg) { pg = pg3; dpg = 0.f; }
    }
    float tis = 1.f, tis_clip = 0.f;
    if (p.use_tis) {
      const float raw = expf(p.old_logp[i] - p.rollout_logp[i]);
      tis = p.use_tis == 2 ? ((raw >= p.tis_lo && raw <= p.tis_hi) ? raw : 0.f)
                           : fminf(fmaxf(raw, p.tis_lo), p.tis_hi);
      tis_clip = (tis != raw) ? 1.f : 0.f;
      pg *= tis;
      dpg *= tis;
    }
    float kl = 0.f, dkl = 0.f;
    if (p.kl_type) {
      const float lr = lp - p.ref_logp[i];
      if (p.kl_type == 1) { kl = lr; dkl = 1.f; }
      else if (p.kl_type == 2) { kl = 0.5f * lr * lr; dkl = lr; }
      else {
        const float e = expf(-lr);
        kl = e + lr - 1.f;
        dkl = 1.f - e;
        if (kl > 10.f) { kl = 10.f; dkl = 0.f; }
        if (kl < -10.f) { kl = -10.f; dkl = 0.f; }
      }
    }
    if (p.pg_out) p.pg_out[i] = pg;
    p.dlogp[i] = w * (dpg + p.kl_coef * dkl);
    acc[0] += w * pg;
    acc[1] += w * clipped;
    acc[2] += w * kl_ppo;
    acc[3] += w * kl;
    acc[4] += w * tis;
    acc[5] += w * tis_clip;
    acc[6] += w;
  }
  __shared__ float sh[PL_METRICS][256];
#pragma unroll
  for (int k = 0; k < PL_METRICS; ++k) sh[k][threadIdx.x] = acc[k];
  __syncthreads();
  for (int off = 128; off > 0; off >>= 1) {
    if (threadIdx.x < off)
#pragma unroll
      for (int k = 0; k < PL_METRICS; ++k) sh[k][threadIdx.x] += sh[k][threadIdx.x + off];
    __syncthreads();
  }
  if (threadIdx.x < PL_METRICS) p.part[blockIdx.x * PL_METRICS + threadIdx.x] = sh[threadIdx.x][0];
}

// Sum [nparts, n] partials in fixed order into out[n] (single CTA).
__global__ void sum_parts_kernel(const float* __restrict__ part, int nparts, int n,
                                 float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < nparts; ++q) s += part[q * n + c];
    out[c] = s;
  }
}

// ---------------------------------------------------------------------------------------------
// GAE, one thread per sequence walking backwards (deterministic, exact recurrence):
//   delta_t = r_t + gamma V_{t+1} - V_t ;  A_t = delta_t + gamma lambda A_{t+1}
// Values/rewards packed by cu; returns = A + V.
// ---------------------------------------------------------------------------------------------
__global__ void gae_kernel(const float* __restrict__ rewards, const float* __restrict__ values,
                           const int* __restrict__ cu, int B, float gamma, float lam,
                           float* __restrict__ adv, float* __restrict__ ret) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int s = cu[b], e = cu[b + 1];
  float last = 0.f, next_v = 0.f;
  for (int t = e - 1; t >= s; --t) {
    const float v = values[t];
    const float delta = rewards[t] + gamma * next_v - v;
    last = delta + gamma * lam * last;
    adv[t] = last;
    ret[t] = last + v;
    next_v = v;
  }
}

// GRPO: per group of `gsize` rewards, adv = r - mean (optionally / (std + eps)); unbiased std.
__global__ void grpo_adv_kernel(const float* __restrict__ r, int ngroups, int gsize, int norm_std,
                                float eps, float* __restrict__ adv) {
  pdl_trigger();
  pdl_wait();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  const float* x = r + (long long)g * gsize;
  float mean = 0.f;
  for (int i = 0; i < gsize; ++i) mean += x[i];
  mean /= gsize;
  float var = 0.f;
  for (int i = 0; i < gsize; ++i) var += (x[i] - mean) * (x[i] - mean);
  const float std = gsize > 1 ? sqrtf(var / (gsize - 1)) : 0.f;
  for (int i = 0; i < gsize; ++i) {
    const float a = x[i] - mean;
    adv[(long long)g * gsize + i] = norm_std ? a / (std + eps) : a;
  }
}

// ---------------------------------------------------------------------------------------------
// Squared L2 norm of a flat buffer (fp32 or bf16), deterministic two-stage; out[0] += result.
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void sqnorm_part_kernel(const T* __restrict__ x, long long n, float* __restrict__ part) {
  pdl_trigger();
  pdl_wait();
  float s = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = (float)x[i];
    s += v * v;
  }
  __shared__ float sh[256];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int off = 128; off > 0; off >>= 1) {
    if (threadIdx.x < off) sh[threadIdx.x] += sh[threadIdx.x + off];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

__global__ void sqnorm_final_kernel(const float* __restrict__ part, int nparts, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sh[256];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 256) s += part[i];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int off = 128; off > 0; off >>= 1) {
    if (threadIdx.x < off) sh[threadIdx.x] += sh[threadIdx.x + off];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] += sh[0];
}

// ---------------------------------------------------------------------------------------------
// Adam(W). Gradient scale = inv_loss_scale * min(1, max_norm / (||g|| + 1e-6)) read from device
// memory (no host sync). master != nullptr: fp32 master weights; otherwise the bf16 params are
// the master and the update is stochastically rounded (hash RNG keyed by (seed, index)).
// m, v in fp32 or bf16; grad in fp32 or bf16.
// ---------------------------------------------------------------------------------------------
struct AdamParams {
  __nv_bfloat16* param;
  float* master;
  void* m;
  void* v;
  const void* grad;
  long long n;
  int grad_bf16, mv_bf16;
  float lr, b1, b2, eps, wd, bc1, bc2;  // bc = 1 - beta^step
  const float* sqnorm;
  float max_norm, inv_loss_scale;
  unsigned long long seed;
  const float* skip;  // if non-null and *skip != 0: skip the update (non-finite guard)
};

MB_DEVICE __nv_bfloat16 sr_bf16(float x, uint32_t rnd) {
  uint32_t bits = __float_as_uint(x);
  if ((bits & 0x7f800000u) == 0x7f800000u) return __float2bfloat16(x);  // inf / nan
  bits += (rnd & 0xffffu);
  bits &= 0xffff0000u;
  return __float2bfloat16(__uint_as_float(bits));  // exact: low bits already zero
}

__global__ void adam_kernel(const AdamParams p) {
  pdl_trigger();
  pdl_wait();
  if (p.skip && *p.skip != 0.f) return;
  float gscale = p.inv_loss_scale;
  if (p.sqnorm && p.max_norm > 0.f) {
    const float nrm = sqrtf(*p.sqnorm) * p.inv_loss_scale;
    gscale *= fminf(1.f, p.max_norm / (nrm + 1e-6f));
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n;
       i += (long long)gridDim.x * blockDim.x) {
    const float g = (p.grad_bf16 ? __bfloat162float(((const __nv_bfloat16*)p.grad)[i])
                                 : ((const float*)p.grad)[i]) * gscale;
    float m = p.mv_bf16 ? __bfloat162float(((__nv_bfloat16*)p.m)[i]) : ((float*)p.m)[i];
    float v = p.mv_bf16 ? __bfloat162float(((__nv_bfloat16*)p.v)[i]) : ((float*)p.v)[i];
    m = p.b1 * m + (1.f - p.b1) * g;
    v = p.b2 * v + (1.f - p.b2) * g * g;
    const float upd = (m / p.bc1) / (sqrtf(v / p.bc2) + p.eps);
    const float w0 = p.master ? p.master[i] : __bfloat162float(p.param[i]);
    const float w1 = w0 - p.lr * (upd + p.wd * w0);
    if (p.master) {
      p.master[i] = w1;
      p.param[i] = __float2bfloat16(w1);
    } else {
      const uint32_t r = (uint32_t)splitmix64(p.seed ^ (uint64_t)i);
      p.param[i] = sr_bf16(w1, r);
    }
    if (p.mv_bf16) {
      ((__nv_bfloat16*)p.m)[i] = __float2bfloat16(m);
      ((__nv_bfloat16*)p.v)[i] = __float2bfloat16(v);
    } else {
      ((float*)p.m)[i] = m;
      ((float*)p.v)[i] = v;
    }
  }
}

// Non-finite check of a flat fp32/bf16 buffer: sets *flag = 1 if any element is inf/nan.
template <typename T>
__global__ void nonfinite_kernel(const T* __restrict__ x, long long n, float* __restrict__ flag) {
  pdl_trigger();
  pdl_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    if (!isfinite((float)x[i])) { *flag = 1.f; return; }
  }
}

}  // namespace mb

using namespace mb;

static int gsz(long long n, int block, int cap = 148 * 8) {
  long long g = (n + block - 1) / block;
  return (int)(g > cap ? cap : (g < 1 ? 1 : g));
}

extern "C" int mb_logprob_fwd(const float* logits, long long ld, const int* target, int n, int V,
                              float inv_temp, float* logp, float* ent, float* lse, cudaStream_t st) {
  if (n == 0) return 0;
  mb_launch(logprob_fwd_kernel, n, LS_THREADS, 0, st, logits, ld, target, V, inv_temp, logp, ent, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_logprob_part(const float* logits, long long ld, const int* target, int lo, int n,
                               int V, float inv_temp, float* part, cudaStream_t st) {
  if (n == 0) return 0;
  mb_launch(logprob_part_kernel, n, LS_THREADS, 0, st, logits, ld, target, lo, V, inv_temp, part, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_logprob_combine(const float* parts, int world, int n, float* logp, float* ent,
                                  float* lse, cudaStream_t st) {
  if (n == 0) return 0;
  if (world < 1) return -1;
  mb_launch(logprob_combine_kernel, (n + 255) / 256, 256, 0, st, parts, world, n, logp, ent, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_logprob_bwd(const float* logits, long long ld, const int* target, int n, int V,
                              float inv_temp, const float* lse, const float* g_lp,
                              const float* g_ent, const float* ent, void* dlogits, long long ldd,
                              cudaStream_t st) {
  if (n == 0) return 0;
  mb_launch(logprob_bwd_kernel, n, LS_THREADS, 0, st, logits, ld, target, V, inv_temp, lse, g_lp, g_ent,
                                               ent, (__nv_bfloat16*)dlogits, ldd);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_sample(const float* logits, long long ld, int n, int V, const float* inv_temps,
                         const unsigned long long* seeds, const int* positions, int* tokens,
                         float* logp, const float* thr, cudaStream_t st) {
  if (n == 0) return 0;
  mb_launch(sample_kernel, n, LS_THREADS, 0, st, logits, ld, V, inv_temps, seeds, positions, tokens,
            logp, thr);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// part: scratch of at least 256 * 7 floats; metrics: 7 floats out.
extern "C" int mb_policy_loss(const float* logp, const float* old_logp, const float* adv,
                              const float* weight, const float* rollout_logp, const float* ref_logp,
                              float* dlogp, float* pg_out, float* part, float* metrics, int n,
                              float eps, float eps_hi, float eps_c, float tis_lo, float tis_hi,
                              float kl_coef, int kl_type, int use_tis, cudaStream_t st) {
  const int grid = gsz(n, 256, 256);
  PolicyLossParams p{logp, old_logp, adv, weight, rollout_logp, ref_logp, dlogp, pg_out, part, n,
                     eps, eps_hi, eps_c, tis_lo, tis_hi, kl_coef, kl_type, use_tis};
  mb_launch(policy_loss_kernel, grid, 256, 0, st, p);
  mb_launch(sum_parts_kernel, 1, 32, 0, st, part, grid, PL_METRICS, metrics);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_gae(const float* rewards, const float* values, const int* cu, int B, float gamma,
                      float lam, float* adv, float* ret, cudaStream_t st) {
  if (B == 0) return 0;
  mb_launch(gae_kernel, (B + 127) / 128, 128, 0, st, rewards, values, cu, B, gamma, lam, adv, ret);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_grpo_adv(const float* r, int ngroups, int gsize, int norm_std, float eps,
                           float* adv, cudaStream_t st) {
  if (ngroups == 0) return 0;
  mb_launch(grpo_adv_kernel, (ngroups + 127) / 128, 128, 0, st, r, ngroups, gsize, norm_std, eps, adv);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// part: scratch of >= 1184 floats. out[0] += sum(x^2).
extern "C" int mb_sqnorm(const void* x, long long n, int is_bf16, float* part, float* out,
                         cudaStream_t st) {
  if (n == 0) return 0;
  const int grid = gsz(n, 256);
  if (is_bf16)
    mb_launch(sqnorm_part_kernel<__nv_bfloat16>, grid, 256, 0, st, (const __nv_bfloat16*)x, n, part);
  else
    mb_launch(sqnorm_part_kernel<float>, grid, 256, 0, st, (const float*)x, n, part);
  mb_launch(sqnorm_final_kernel, 1, 256, 0, st, part, grid, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_nonfinite(const void* x, long long n, int is_bf16, float* flag, cudaStream_t st) {
  if (n == 0) return 0;
  const int grid = gsz(n, 256);
  if (is_bf16) mb_launch(nonfinite_kernel<__nv_bfloat16>, grid, 256, 0, st, (const __nv_bfloat16*)x, n, flag);
  else mb_launch(nonfinite_kernel<float>, grid, 256, 0, st, (const float*)x, n, flag);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_adam(void* param, float* master, void* m, void* v, const void* grad, long long n,
                       int grad_bf16, int mv_bf16, float lr, float b1, float b2, float eps, float wd,
                       int step, const float* sqnorm, float max_norm, float inv_loss_scale,
                       unsigned long long seed, const float* skip, cudaStream_t st) {
  if (n == 0) return 0;
  AdamParams p;
  p.param = (__nv_bfloat16*)param; p.master = master; p.m = m; p.v = v; p.grad = grad; p.n = n;
  p.grad_bf16 = grad_bf16; p.mv_bf16 = mv_bf16; p.lr = lr; p.b1 = b1; p.b2 = b2; p.eps = eps;
  p.wd = wd;
  p.bc1 = 1.f - powf(b1, (float)step);
  p.bc2 = 1.f - powf(b2, (float)step);
  p.sqnorm = sqnorm; p.max_norm = max_norm; p.inv_loss_scale = inv_loss_scale; p.seed = seed;
  p.skip = skip;
  mb_launch(adam_kernel, gsz(n, 256, 148 * 16), 256, 0, st, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
