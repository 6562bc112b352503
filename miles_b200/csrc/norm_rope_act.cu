// Normalisation, rotary embedding and activation kernels (sm_100a).
//
// All reductions use a fixed lane/thread assignment and a fixed tree order, so each output is a
// pure function of its own row: the trainer (packed micro-batches) and the rollout engine
// (one token per sequence per step) produce bitwise identical activations.
//
// Reference roles replaced: TE/Megatron fused RMSNorm, QK-layernorm + RoPE (megatron.patch
// rope hunks, model_provider.py TE spec) and SwiGLU (fused_experts.py:173-200 SiluAndMul).
#include "common.cuh"

namespace mb {

// ----------------------------------------------------------------------------------------------
// RMSNorm over rows of length H (H % 256 == 0, H <= 8192), one warp per row.
//   optional fused residual: h = x + res (bf16), y = norm(h)
// ----------------------------------------------------------------------------------------------
// One CTA per row: NT = H / 8 / CPT threads, each owning CPT 16-byte chunks (chunk c of the
// row at c = tid + j * NT). Sum of squares: per thread in chunk/element order, then the warp
// xor tree, then the warps in index order (fixed, so every launch gives the same bits).
template <int H>
struct RmsShape {
  static constexpr int NCH = H / 8;
  static constexpr int CPT = NCH / 128 > 1 ? NCH / 128 : 1;
  static constexpr int NT = NCH / CPT;
  static_assert(NCH % CPT == 0 && NT % 32 == 0, "unsupported hidden size");
};

template <int H>
__global__ void __launch_bounds__(RmsShape<H>::NT)
rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ h_out,
                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int rows,
                   float eps) {
  pdl_trigger();
  pdl_wait();
  using S = RmsShape<H>;
  constexpr int NW = S::NT / 32;
  __shared__ float wsum[NW];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  if (row >= rows) return;
  const long long base = (long long)row * H;
  float v[S::CPT * 8];
#pragma unroll
  for (int j = 0; j < S::CPT; ++j) {
    const int col = (tid + j * S::NT) * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(x + base + col);
    const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&a);
    if (res) {
      const uint4 r = *reinterpret_cast<const uint4*>(res + base + col);
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ob[e] = __float2bfloat16(__bfloat162float(ab[e]) + __bfloat162float(rb[e]));
        v[j * 8 + e] = __bfloat162float(ob[e]);
      }
      *reinterpret_cast<uint4*>(h_out + base + col) = o;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j * 8 + e] = __bfloat162float(ab[e]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < S::CPT * 8; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) wsum[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) tot += wsum[i];
  const float rstd = rsqrtf(tot / (float)H + eps);
  if (tid == 0 && rstd_out) rstd_out[row] = rstd;
#pragma unroll
  for (int j = 0; j < S::CPT; ++j) {
    const int col = (tid + j * S::NT) * 8;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + col);
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 o;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float nrm = __bfloat162float(__float2bfloat16(v[j * 8 + e] * rstd));
      ob[e] = __float2bfloat16(nrm * __bfloat162float(wb[e]));
    }
    *reinterpret_cast<uint4*>(y + base + col) = o;
  }
}

// dx = rstd * (g - xhat * mean(g * xhat)), g = dy * w. Two passes over the row (the second
// re-reads x/dy from L1/L2) keep register use flat in H; each warp accumulates its d(w)
// contribution in its own shared-memory row, reduced across warps in a fixed order.
template <int H>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                   const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w,
                                   const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dres,  // optional: added to dx
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part,
                                   int rows, int rows_per_block) {
  pdl_trigger();
  pdl_wait();
  const int warps = blockDim.x / 32;
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  extern __shared__ float sh[];
  float* mine = sh + wid * H;
  for (int c = lane; c < H; c += 32) mine[c] = 0.f;
  __syncwarp();
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + wid; row < r1; row += warps) {
    const float rs = rstd[row];
    const __nv_bfloat16* xr = x + (long long)row * H;
    const __nv_bfloat16* dr = dy + (long long)row * H;
    float dot = 0.f;
    for (int col = lane * 8; col < H; col += 256) {
      uint4 a = *reinterpret_cast<const uint4*>(xr + col);
      uint4 d = *reinterpret_cast<const uint4*>(dr + col);
      uint4 wv = *reinterpret_cast<const uint4*>(w + col);
      const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&d);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dot += __bfloat162float(db[j]) * __bfloat162float(wb[j]) * (__bfloat162float(ab[j]) * rs);
    }
    dot = warp_sum(dot) / (float)H;
    for (int col = lane * 8; col < H; col += 256) {
      uint4 a = *reinterpret_cast<const uint4*>(xr + col);
      uint4 d = *reinterpret_cast<const uint4*>(dr + col);
      uint4 wv = *reinterpret_cast<const uint4*>(w + col);
      const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&d);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
      float extra[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (dres) {
        uint4 r = *reinterpret_cast<const uint4*>(dres + (long long)row * H + col);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
        for (int j = 0; j < 8; ++j) extra[j] = __bfloat162float(rb[j]);
      }
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xv = __bfloat162float(ab[j]) * rs;
        const float dv = __bfloat162float(db[j]);
        const float g = dv * __bfloat162float(wb[j]);
        mine[col + j] += dv * __bfloat162float(__float2bfloat16(xv));
        ob[j] = __float2bfloat16(rs * (g - xv * dot) + extra[j]);
      }
      *reinterpret_cast<uint4*>(dx + (long long)row * H + col) = o;
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < warps; ++k) s += sh[k * H + col];
    dw_part[(long long)blockIdx.x * H + col] = s;
  }
}

// Sum per-block partial rows [nparts, n] into out[n] (fixed order), optionally accumulating.
__global__ void reduce_parts_kernel(const float* __restrict__ parts, int nparts, int n,
                                    float* __restrict__ out_f32, __nv_bfloat16* __restrict__ out_bf16,
                                    int accumulate) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += parts[(long long)p * n + c];
  if (out_f32) out_f32[c] = (accumulate ? out_f32[c] : 0.f) + s;
  if (out_bf16)
    out_bf16[c] = __float2bfloat16((accumulate ? __bfloat162float(out_bf16[c]) : 0.f) + s);
}

// ----------------------------------------------------------------------------------------------
// Fused per-head RMSNorm (QK-norm) + rotary embedding (rotate-half convention), head_dim D=128.
// in: qkv [T, (nq + 2*nkv) * D] rows with stride ld_in. Writes q [T, nq, D], k/v to
// k_out/v_out rows `slot[t]` (identity when slot == nullptr) with row stride ld_kv elements.
// cos/sin tables: [max_pos, D/2] fp32. One warp per (token, head); lane owns 4 dims:
// d = lane*2 + {0,1} in the first half and the same + D/2 in the second half.
// ----------------------------------------------------------------------------------------------
// One warp handles R consecutive heads of one token (R divides the head count): the R rows
// are loaded before any of them is processed (more loads in flight per warp) and the token's
// position / cos / sin are read once. Per element the arithmetic is that of one row at a time.
template <int R>
__global__ void qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, long long ld_in,
                                        const __nv_bfloat16* __restrict__ qw,
                                        const __nv_bfloat16* __restrict__ kw,
                                        const int* __restrict__ pos,
                                        const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t,
                                        __nv_bfloat16* __restrict__ q_out,
                                        __nv_bfloat16* __restrict__ k_out,
                                        __nv_bfloat16* __restrict__ v_out,
                                        const long long* __restrict__ slot, long long ld_kv,
                                        float* __restrict__ rstd_out, int T, int nq, int nkv,
                                        float eps, int use_norm) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128, HALF = 64;
  const int nh = nq + 2 * nkv;
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw * R >= (long long)T * nh) return;
  const int t = (int)(gw * R / nh), h0 = (int)(gw * R % nh);
  const __nv_bfloat16* src = qkv + (long long)t * ld_in + (long long)h0 * D;
  const int d0 = lane * 2;
  __nv_bfloat162 a[R], b[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    a[r] = *reinterpret_cast<const __nv_bfloat162*>(src + r * D + d0);
    b[r] = *reinterpret_cast<const __nv_bfloat162*>(src + r * D + HALF + d0);
  }
  const long long dst_row = slot ? slot[t] : (long long)t;
  const int p = pos[t];
  const float2 cs = *reinterpret_cast<const float2*>(cos_t + (long long)p * HALF + d0);
  const float2 sn = *reinterpret_cast<const float2*>(sin_t + (long long)p * HALF + d0);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int h = h0 + r;
    if (h >= nq + nkv) {  // V: plain copy into the cache / v buffer
      __nv_bfloat16* dst = v_out + dst_row * ld_kv + (long long)(h - nq - nkv) * D;
      *reinterpret_cast<__nv_bfloat162*>(dst + d0) = a[r];
      *reinterpret_cast<__nv_bfloat162*>(dst + HALF + d0) = b[r];
      continue;
    }
    float x0 = __low2float(a[r]), x1 = __high2float(a[r]);
    float y0 = __low2float(b[r]), y1 = __high2float(b[r]);
    const bool isq = h < nq;
    if (use_norm) {
      float ss = x0 * x0 + x1 * x1 + y0 * y0 + y1 * y1;
      ss = warp_sum(ss);
      const float rs = rsqrtf(ss / (float)D + eps);
      if (lane == 0 && rstd_out) rstd_out[(long long)t * (nq + nkv) + h] = rs;
      const __nv_bfloat16* nw = isq ? qw : kw;
      x0 = __bfloat162float(__float2bfloat16(x0 * rs)) * __bfloat162float(nw[d0]);
      x1 = __bfloat162float(__float2bfloat16(x1 * rs)) * __bfloat162float(nw[d0 + 1]);
      y0 = __bfloat162float(__float2bfloat16(y0 * rs)) * __bfloat162float(nw[HALF + d0]);
      y1 = __bfloat162float(__float2bfloat16(y1 * rs)) * __bfloat162float(nw[HALF + d0 + 1]);
      x0 = __bfloat162float(__float2bfloat16(x0));
      x1 = __bfloat162float(__float2bfloat16(x1));
      y0 = __bfloat162float(__float2bfloat16(y0));
      y1 = __bfloat162float(__float2bfloat16(y1));
    }
    const float c0 = cs.x, c1 = cs.y, s0 = sn.x, s1 = sn.y;
    const float o0 = x0 * c0 - y0 * s0, o1 = x1 * c1 - y1 * s1;
    const float p0 = y0 * c0 + x0 * s0, p1 = y1 * c1 + x1 * s1;
    __nv_bfloat16* dst = isq ? q_out + ((long long)t * nq + h) * D
                             : k_out + dst_row * ld_kv + (long long)(h - nq) * D;
    *reinterpret_cast<__nv_bfloat162*>(dst + d0) = __floats2bfloat162_rn(o0, o1);
    *reinterpret_cast<__nv_bfloat162*>(dst + HALF + d0) = __floats2bfloat162_rn(p0, p1);
  }
}

// Backward of the above for q and k heads; dv is copied through. Produces d(qkv) and per-block
// partial d(q_norm_w), d(k_norm_w).
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq,
                                        const __nv_bfloat16* __restrict__ dk,
                                        const __nv_bfloat16* __restrict__ dv,
                                        const __nv_bfloat16* __restrict__ qkv, long long ld_in,
                                        const __nv_bfloat16* __restrict__ qw,
                                        const __nv_bfloat16* __restrict__ kw,
                                        const int* __restrict__ pos,
                                        const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t,
                                        const float* __restrict__ rstd,
                                        __nv_bfloat16* __restrict__ dqkv,
                                        float* __restrict__ dw_part,  // [gridDim.x, 2, D]
                                        int T, int nq, int nkv, int use_norm) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128, HALF = 64;
  const int nh = nq + 2 * nkv;
  const int warps = blockDim.x / 32;
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int d0 = lane * 2;
  float dwq[4] = {0, 0, 0, 0}, dwk[4] = {0, 0, 0, 0};
  const long long total = (long long)T * nh;
  for (long long gw = (long long)blockIdx.x * warps + wid; gw < total;
       gw += (long long)gridDim.x * warps) {
    const int t = (int)(gw / nh), h = (int)(gw % nh);
    __nv_bfloat16* dst = dqkv + (long long)t * ld_in + (long long)h * D;
    if (h >= nq + nkv) {
      const __nv_bfloat16* g = dv + ((long long)t * nkv + (h - nq - nkv)) * D;
      *reinterpret_cast<__nv_bfloat162*>(dst + d0) = *reinterpret_cast<const __nv_bfloat162*>(g + d0);
      *reinterpret_cast<__nv_bfloat162*>(dst + HALF + d0) =
          *reinterpret_cast<const __nv_bfloat162*>(g + HALF + d0);
      continue;
    }
    const bool isq = h < nq;
    const __nv_bfloat16* g = isq ? dq + ((long long)t * nq + h) * D
                                 : dk + ((long long)t * nkv + (h - nq)) * D;
    const __nv_bfloat162 ga = *reinterpret_cast<const __nv_bfloat162*>(g + d0);
    const __nv_bfloat162 gb = *reinterpret_cast<const __nv_bfloat162*>(g + HALF + d0);
    const float go0 = __low2float(ga), go1 = __high2float(ga);
    const float gp0 = __low2float(gb), gp1 = __high2float(gb);
    const int p = pos[t];
    const float c0 = cos_t[(long long)p * HALF + d0], c1 = cos_t[(long long)p * HALF + d0 + 1];
    const float s0 = sin_t[(long long)p * HALF + d0], s1 = sin_t[(long long)p * HALF + d0 + 1];
    // inverse rotation
    float gx0 = go0 * c0 + gp0 * s0, gx1 = go1 * c1 + gp1 * s1;
    float gy0 = gp0 * c0 - go0 * s0, gy1 = gp1 * c1 - go1 * s1;
    const __nv_bfloat16* src = qkv + (long long)t * ld_in + (long long)h * D;
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(src + d0);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(src + HALF + d0);
    if (use_norm) {
      const float rs = rstd[(long long)t * (nq + nkv) + h];
      const float xh[4] = {__low2float(a) * rs, __high2float(a) * rs, __low2float(b) * rs,
                           __high2float(b) * rs};
      const __nv_bfloat16* nw = isq ? qw : kw;
      const float wv[4] = {__bfloat162float(nw[d0]), __bfloat162float(nw[d0 + 1]),
                           __bfloat162float(nw[HALF + d0]), __bfloat162float(nw[HALF + d0 + 1])};
      const float gn[4] = {gx0, gx1, gy0, gy1};
      float gg[4];
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        gg[i] = gn[i] * wv[i];
        dot += gg[i] * xh[i];
        const float contrib = gn[i] * __bfloat162float(__float2bfloat16(xh[i]));
        if (isq) dwq[i] += contrib; else dwk[i] += contrib;
      }
      dot = warp_sum(dot) / (float)D;
      gx0 = rs * (gg[0] - xh[0] * dot);
      gx1 = rs * (gg[1] - xh[1] * dot);
      gy0 = rs * (gg[2] - xh[2] * dot);
      gy1 = rs * (gg[3] - xh[3] * dot);
    }
    *reinterpret_cast<__nv_bfloat162*>(dst + d0) = __floats2bfloat162_rn(gx0, gx1);
    *reinterpret_cast<__nv_bfloat162*>(dst + HALF + d0) = __floats2bfloat162_rn(gy0, gy1);
  }
  if (!dw_part) return;
  __shared__ float sh[2][32][128];
  const int cols[4] = {d0, d0 + 1, HALF + d0, HALF + d0 + 1};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sh[0][wid][cols[i]] = dwq[i];
    sh[1][wid][cols[i]] = dwk[i];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D; c += blockDim.x) {
    const int which = c / D, col = c % D;
    float s = 0.f;
    for (int k = 0; k < warps; ++k) s += sh[which][k][col];
    dw_part[(long long)blockIdx.x * 2 * D + c] = s;
  }
}

// ----------------------------------------------------------------------------------------------
// SwiGLU: out = silu(gate) * up, gate/up halves of each row of gu [T, 2I] (row stride 2I).
// ----------------------------------------------------------------------------------------------
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ out, long long T, int I,
                                  const int* __restrict__ nrows) {
  pdl_trigger();
  pdl_wait();
  if (nrows) T = min(T, (long long)*nrows);  // rows beyond the live MoE segments are skipped
  const long long n8 = T * I / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 8;
    const long long t = e / I;
    const int c = (int)(e % I);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + I + c);
    const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uv);
    uint4 o;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = __bfloat162float(gb[j]);
      const float s = g / (1.f + expf(-g));
      ob[j] = __float2bfloat16(__bfloat162float(__float2bfloat16(s)) * __bfloat162float(ub[j]));
    }
    *reinterpret_cast<uint4*>(out + t * I + c) = o;
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  const __nv_bfloat16* __restrict__ dout,
                                  __nv_bfloat16* __restrict__ dgu, long long T, int I,
                                  const int* __restrict__ nrows) {
  pdl_trigger();
  pdl_wait();
  if (nrows) T = min(T, (long long)*nrows);
  const long long n8 = T * I / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 8;
    const long long t = e / I;
    const int c = (int)(e % I);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + c);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + I + c);
    uint4 dv = *reinterpret_cast<const uint4*>(dout + t * I + c);
    const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uv);
    const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&dv);
    uint4 og, ou;
    __nv_bfloat16* ogb = reinterpret_cast<__nv_bfloat16*>(&og);
    __nv_bfloat16* oub = reinterpret_cast<__nv_bfloat16*>(&ou);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = __bfloat162float(gb[j]);
      const float u = __bfloat162float(ub[j]);
      const float d = __bfloat162float(db[j]);
      const float sig = 1.f / (1.f + expf(-g));
      const float s = g * sig;
      oub[j] = __float2bfloat16(d * s);
      ogb[j] = __float2bfloat16(d * u * sig * (1.f + g * (1.f - sig)));
    }
    *reinterpret_cast<uint4*>(dgu + t * 2 * I + c) = og;
    *reinterpret_cast<uint4*>(dgu + t * 2 * I + I + c) = ou;
  }
}

}  // namespace mb

using namespace mb;

static int grid_for(long long n, int block) {
  long long g = (n + block - 1) / block;
  return (int)(g > 148 * 16 ? 148 * 16 : (g < 1 ? 1 : g));
}

extern "C" int mb_rmsnorm_fwd(const void* x, const void* res, const void* w, void* h_out, void* y,
                              float* rstd, int rows, int H, float eps, cudaStream_t st) {
  if (rows == 0) return 0;
#define RMS_CASE(HH)                                                                           \
  case HH:                                                                                     \
    mb_launch(rmsnorm_fwd_kernel<HH>, rows, RmsShape<HH>::NT, 0, st,                           \
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)res, (const __nv_bfloat16*)w,           \
        (__nv_bfloat16*)h_out, (__nv_bfloat16*)y, rstd, rows, eps);                            \
    break;
  switch (H) {
    RMS_CASE(256) RMS_CASE(512) RMS_CASE(1024) RMS_CASE(2048) RMS_CASE(2560) RMS_CASE(4096)
    RMS_CASE(5120) RMS_CASE(7168) RMS_CASE(8192)
    default: return -1;
  }
#undef RMS_CASE
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd,
                              const void* dres, void* dx, float* dw_part, int nparts, float* dw_f32,
                              void* dw_bf16, int accumulate, int rows, int H, cudaStream_t st) {
  if (rows == 0) return 0;
  const int block = H >= 7168 ? 128 : 256;  // per-warp d(w) rows must fit in shared memory
  const int rpb = (rows + nparts - 1) / nparts;
  const int grid = (rows + rpb - 1) / rpb;
  const size_t smem = (size_t)(block / 32) * H * sizeof(float);
#define RMSB_CASE(HH)                                                                          \
  case HH: {                                                                                   \
    auto k = rmsnorm_bwd_kernel<HH>;                                                           \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                               (int)smem);                                     \
    mb_launch(k, grid, block, smem, st, (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x,           \
                                 (const __nv_bfloat16*)w, rstd, (const __nv_bfloat16*)dres,   \
                                 (__nv_bfloat16*)dx, dw_part, rows, rpb);                      \
  } break;
  switch (H) {
    RMSB_CASE(256) RMSB_CASE(512) RMSB_CASE(1024) RMSB_CASE(2048) RMSB_CASE(2560)
    RMSB_CASE(4096) RMSB_CASE(5120) RMSB_CASE(7168) RMSB_CASE(8192)
    default: return -1;
  }
#undef RMSB_CASE
  mb_launch(reduce_parts_kernel, (H + 255) / 256, 256, 0, st, dw_part, grid, H, dw_f32,
                                                       (__nv_bfloat16*)dw_bf16, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_qk_norm_rope_fwd(const void* qkv, long long ld_in, const void* qw, const void* kw,
                                   const int* pos, const float* cos_t, const float* sin_t,
                                   void* q_out, void* k_out, void* v_out, const long long* slot,
                                   long long ld_kv, float* rstd, int T, int nq, int nkv, float eps,
                                   int use_norm, cudaStream_t st) {
  if (T == 0) return 0;
  const int nh = nq + 2 * nkv;
  const int R = nh % 4 == 0 ? 4 : nh % 2 == 0 ? 2 : 1;  // heads per warp
  const long long warps = (long long)T * nh / R;
  const int block = 256;
  const long long grid = (warps + 7) / 8;
  auto kern = R == 4 ? qk_norm_rope_fwd_kernel<4> : R == 2 ? qk_norm_rope_fwd_kernel<2>
                                                            : qk_norm_rope_fwd_kernel<1>;
  mb_launch(kern, (unsigned)grid, block, 0, st, 
      (const __nv_bfloat16*)qkv, ld_in, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw, pos,
      cos_t, sin_t, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, slot,
      ld_kv, rstd, T, nq, nkv, eps, use_norm);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// dw_out: 256 floats = [d(q_norm_w) (128), d(k_norm_w) (128)]
extern "C" int mb_qk_norm_rope_bwd(const void* dq, const void* dk, const void* dv, const void* qkv,
                                   long long ld_in, const void* qw, const void* kw, const int* pos,
                                   const float* cos_t, const float* sin_t, const float* rstd,
                                   void* dqkv, float* dw_part, int nparts, float* dw_out,
                                   int T, int nq, int nkv, int use_norm, cudaStream_t st) {
  if (T == 0) return 0;
  const int block = 256;
  mb_launch(qk_norm_rope_bwd_kernel, nparts, block, 0, st, 
      (const __nv_bfloat16*)dq, (const __nv_bfloat16*)dk, (const __nv_bfloat16*)dv,
      (const __nv_bfloat16*)qkv, ld_in, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw, pos,
      cos_t, sin_t, rstd, (__nv_bfloat16*)dqkv, use_norm ? dw_part : nullptr, T, nq, nkv,
      use_norm);
  if (use_norm) mb_launch(reduce_parts_kernel, 1, 256, 0, st, dw_part, nparts, 256, dw_out, nullptr, 0);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_swiglu_fwd(const void* gu, void* out, long long T, int I, const int* nrows,
                             cudaStream_t st) {
  if (T == 0) return 0;
  if (I % 8) return -1;
  const long long n8 = T * I / 8;
  mb_launch(swiglu_fwd_kernel, grid_for(n8, 256), 256, 0, st, (const __nv_bfloat16*)gu,
                                                       (__nv_bfloat16*)out, T, I, nrows);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_swiglu_bwd(const void* gu, const void* dout, void* dgu, long long T, int I,
                             const int* nrows, cudaStream_t st) {
  if (T == 0) return 0;
  if (I % 8) return -1;
  const long long n8 = T * I / 8;
  mb_launch(swiglu_bwd_kernel, grid_for(n8, 256), 256, 0, st, 
      (const __nv_bfloat16*)gu, (const __nv_bfloat16*)dout, (__nv_bfloat16*)dgu, T, I, nrows);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
