// Deterministic causal attention for head_dim 128, bf16 in / fp32 softmax, GQA (sm_100a).
//
//  * forward and paged decode: tcgen05 kernels in csrc/attention_sm100.cu (entry points and
//    the decode split-KV combine kernel here)
//  * attn_bwd_dkdv / attn_bwd_dq : deterministic backward (no atomics; each output tile is
//    owned by one CTA that walks its inputs in a fixed order)
//
// Bitwise train/rollout parity of the forward is a property of the tcgen05 kernel (one code
// path for prefill and decode rows); the backward only needs the forward's LSE.
//
// Backward tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) fed by ldmatrix from
// XOR-swizzled shared memory and cp.async double buffering.
//
// Reference roles replaced: TE/cuDNN fused attention and flash-attn varlen (E5,
// `--attention-backend flash`), SGLang paged decode attention (E7).
#include "common.cuh"
#include "api.h"

namespace mb {
namespace attn {

constexpr int D = 128;       // head dim
constexpr int BM = 64;       // query rows per CTA (4 warps x 16)
constexpr int BN = 64;       // keys per block
constexpr int TILE_BYTES = 64 * D * 2;  // one 64x128 bf16 tile = 16 KB

MB_DEVICE uint32_t swz(int row, int chunk) {  // byte offset inside a 64x128 bf16 tile
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

MB_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
MB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MB_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

MB_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
MB_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
MB_DEVICE void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load a 64-row x 128 tile whose row r lives at base + row_off(r) (elements), rows >= nvalid
// zero-filled. `nthreads` threads cooperate (thread index tid).
template <typename RowFn>
MB_DEVICE void load_tile(uint32_t smem, const __nv_bfloat16* base, RowFn row_off, int nvalid,
                         int tid, int nthreads) {
  for (int i = tid; i < 64 * 16; i += nthreads) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < nvalid;
    const __nv_bfloat16* src = ok ? base + row_off(r) + c * 8 : base;
    cp_async16(smem + swz(r, c), src, ok);
  }
}

// A-fragment (16 rows x 16 k) of a tile for the warp's 16 rows starting at row0, k-step ks.
MB_DEVICE void load_a(uint32_t tile, int row0, int ks, int lane, uint32_t (&a)[4]) {
  const int r = row0 + (lane & 15);
  const int ch = 2 * ks + (lane >> 4);
  ldsm_x4(tile + swz(r, ch), a[0], a[1], a[2], a[3]);
}

// B-fragments for two n8 tiles (rows n0..n0+15 of a [n][k] tile), k-step ks (non-transposed).
MB_DEVICE void load_b_nt(uint32_t tile, int n0, int ks, int lane, uint32_t& b00, uint32_t& b01,
                         uint32_t& b10, uint32_t& b11) {
  const int mi = lane >> 3;
  const int r = n0 + (mi >> 1) * 8 + (lane & 7);
  const int ch = 2 * ks + (mi & 1);
  ldsm_x4(tile + swz(r, ch), b00, b01, b10, b11);
}

// B-fragments for two n8 tiles of columns (chunks 2p, 2p+1) of a [k][n] tile, k rows k0..k0+15.
MB_DEVICE void load_b_t(uint32_t tile, int k0, int p, int lane, uint32_t& b00, uint32_t& b01,
                        uint32_t& b10, uint32_t& b11) {
  const int mi = lane >> 3;
  const int r = k0 + (mi & 1) * 8 + (lane & 7);
  const int ch = 2 * p + (mi >> 1);
  ldsm_x4_t(tile + swz(r, ch), b00, b01, b10, b11);
}

MB_DEVICE uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ---------------------------------------------------------------------------------------------
// Canonical split-KV combination. Keys are processed in chunks of 1024 (csrc/attention_sm100.cu);
// each chunk's (m, l, o) starts from scratch and the chunk partials are merged in increasing
// chunk order. The prefill kernel merges in TMEM; the decode kernel writes one partial per chunk
// and the combine kernel below merges them with the very same non-contracted float operations,
// so both give identical bits.
// ---------------------------------------------------------------------------------------------
constexpr int CHUNK_BLOCKS = 16;  // 1024 keys per chunk

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

struct BwdParams {
  const __nv_bfloat16 *q, *k, *v, *dout;
  const float *lse, *delta;  // [nq, T]
  __nv_bfloat16 *dq, *dk, *dv;
  const int* cu_seqlens;
  const int* blk_seq;
  const int* blk_idx;
  long long q_stride, k_stride, v_stride, do_stride, dq_stride, dk_stride, dv_stride;
  int nq, nkv, T;
  float scale_log2, scale;
};

// CTA = (key block of 64, kv head). Warp w owns keys kb*64 + 16w .. +15. Loops over the query
// heads of the group and over query blocks qb >= kb in a fixed order; accumulates dK, dV in
// registers.
__global__ void __launch_bounds__(128, 1) attn_bwd_dkdv_kernel(const BwdParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sk = smem_u32(smem), sv = sk + TILE_BYTES;
  const uint32_t sq = sk + 2 * TILE_BYTES, sdo = sk + 3 * TILE_BYTES;
  float* s_lse = reinterpret_cast<float*>(smem + 4 * TILE_BYTES);
  float* s_delta = s_lse + 64;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = p.blk_seq[blockIdx.x], kb = p.blk_idx[blockIdx.x];
  const int hk = blockIdx.y, G = p.nq / p.nkv;
  const int start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - start;
  const int n0 = kb * BN;
  const int kvalid = min(BN, len - n0);
  load_tile(sk, p.k + (long long)(start + n0) * p.k_stride + (long long)hk * D,
            [&](int r) { return (long long)r * p.k_stride; }, kvalid, tid, 128);
  load_tile(sv, p.v + (long long)(start + n0) * p.v_stride + (long long)hk * D,
            [&](int r) { return (long long)r * p.v_stride; }, kvalid, tid, 128);
  cp_async_commit();
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) dk[n][i] = dv[n][i] = 0.f;
  const int g = lane >> 2, c = lane & 3;
  const int key0 = n0 + warp * 16 + g, key1 = key0 + 8;  // this thread's S^T rows (keys)
  const int nqb = (len + BM - 1) / BM;
  for (int hh = 0; hh < G; ++hh) {
    const int h = hk * G + hh;
    for (int qb = kb; qb < nqb; ++qb) {
      const int m0 = qb * BM;
      const int qvalid = min(BM, len - m0);
      __syncthreads();
      load_tile(sq, p.q + (long long)(start + m0) * p.q_stride + (long long)h * D,
                [&](int r) { return (long long)r * p.q_stride; }, qvalid, tid, 128);
      load_tile(sdo, p.dout + (long long)(start + m0) * p.do_stride + (long long)h * D,
                [&](int r) { return (long long)r * p.do_stride; }, qvalid, tid, 128);
      cp_async_commit();
      if (tid < 64) {
        const bool ok = tid < qvalid;
        s_lse[tid] = ok ? p.lse[(long long)h * p.T + start + m0 + tid] : INFINITY;
        s_delta[tid] = ok ? p.delta[(long long)h * p.T + start + m0 + tid] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      // S^T = K Q^T (16 keys x 64 queries)
      float st[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a[4];
        load_a(sk, warp * 16, ks, lane, a);
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          uint32_t b00, b01, b10, b11;
          load_b_nt(sq, pp * 16, ks, lane, b00, b01, b10, b11);
          mma16816(st[2 * pp], a, b00, b01);
          mma16816(st[2 * pp + 1], a, b10, b11);
        }
      }
      // P^T = exp(S^T * scale - lse[query]); mask query < key
      const float ln2inv = 1.4426950408889634f;
      uint32_t pa[4][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int qi = j * 8 + 2 * c;
        const int qp0 = m0 + qi, qp1 = qp0 + 1;
        const float l0 = s_lse[qi] * ln2inv, l1 = s_lse[qi + 1] * ln2inv;
        const float p00 = (qp0 < key0) ? 0.f : exp2f(st[j][0] * p.scale_log2 - l0);
        const float p01 = (qp1 < key0) ? 0.f : exp2f(st[j][1] * p.scale_log2 - l1);
        const float p10 = (qp0 < key1) ? 0.f : exp2f(st[j][2] * p.scale_log2 - l0);
        const float p11 = (qp1 < key1) ? 0.f : exp2f(st[j][3] * p.scale_log2 - l1);
        st[j][0] = p00; st[j][1] = p01; st[j][2] = p10; st[j][3] = p11;
        const int kk = j >> 1;
        if ((j & 1) == 0) { pa[kk][0] = pack2(p00, p01); pa[kk][1] = pack2(p10, p11); }
        else { pa[kk][2] = pack2(p00, p01); pa[kk][3] = pack2(p10, p11); }
      }
      // dV += P^T dO
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int pp = 0; pp < 8; ++pp) {
          uint32_t b00, b01, b10, b11;
          load_b_t(sdo, kk * 16, pp, lane, b00, b01, b10, b11);
          mma16816(dv[2 * pp], pa[kk], b00, b01);
          mma16816(dv[2 * pp + 1], pa[kk], b10, b11);
        }
      // dP^T = V dO^T
      float dpt[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a[4];
        load_a(sv, warp * 16, ks, lane, a);
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          uint32_t b00, b01, b10, b11;
          load_b_nt(sdo, pp * 16, ks, lane, b00, b01, b10, b11);
          mma16816(dpt[2 * pp], a, b00, b01);
          mma16816(dpt[2 * pp + 1], a, b10, b11);
        }
      }
      // dS^T = P^T * (dP^T - delta[query])
      uint32_t dsa[4][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int qi = j * 8 + 2 * c;
        const float d0 = s_delta[qi], d1 = s_delta[qi + 1];
        const float v00 = st[j][0] * (dpt[j][0] - d0), v01 = st[j][1] * (dpt[j][1] - d1);
        const float v10 = st[j][2] * (dpt[j][2] - d0), v11 = st[j][3] * (dpt[j][3] - d1);
        const int kk = j >> 1;
        if ((j & 1) == 0) { dsa[kk][0] = pack2(v00, v01); dsa[kk][1] = pack2(v10, v11); }
        else { dsa[kk][2] = pack2(v00, v01); dsa[kk][3] = pack2(v10, v11); }
      }
      // dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int pp = 0; pp < 8; ++pp) {
          uint32_t b00, b01, b10, b11;
          load_b_t(sq, kk * 16, pp, lane, b00, b01, b10, b11);
          mma16816(dk[2 * pp], dsa[kk], b00, b01);
          mma16816(dk[2 * pp + 1], dsa[kk], b10, b11);
        }
    }
  }
  const bool ok0 = key0 < len, ok1 = key1 < len;
  __nv_bfloat16* dk0 = p.dk + (long long)(start + key0) * p.dk_stride + (long long)hk * D;
  __nv_bfloat16* dk1 = p.dk + (long long)(start + key1) * p.dk_stride + (long long)hk * D;
  __nv_bfloat16* dv0 = p.dv + (long long)(start + key0) * p.dv_stride + (long long)hk * D;
  __nv_bfloat16* dv1 = p.dv + (long long)(start + key1) * p.dv_stride + (long long)hk * D;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * c;
    if (ok0) {
      *reinterpret_cast<uint32_t*>(dk0 + col) = pack2(dk[n][0] * p.scale, dk[n][1] * p.scale);
      *reinterpret_cast<uint32_t*>(dv0 + col) = pack2(dv[n][0], dv[n][1]);
    }
    if (ok1) {
      *reinterpret_cast<uint32_t*>(dk1 + col) = pack2(dk[n][2] * p.scale, dk[n][3] * p.scale);
      *reinterpret_cast<uint32_t*>(dv1 + col) = pack2(dv[n][2], dv[n][3]);
    }
  }
}

// CTA = (query block, query head). dQ = scale * sum_j dS_j K_j over key blocks 0..qb.
__global__ void __launch_bounds__(128, 1) attn_bwd_dq_kernel(const BwdParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sq = smem_u32(smem), sdo = sq + TILE_BYTES;
  const uint32_t sk = sq + 2 * TILE_BYTES, sv = sq + 3 * TILE_BYTES;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = p.blk_seq[blockIdx.x], qb = p.blk_idx[blockIdx.x];
  const int h = blockIdx.y, hk = h / (p.nq / p.nkv);
  const int start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - start;
  const int m0 = qb * BM;
  const int qvalid = min(BM, len - m0);
  load_tile(sq, p.q + (long long)(start + m0) * p.q_stride + (long long)h * D,
            [&](int r) { return (long long)r * p.q_stride; }, qvalid, tid, 128);
  load_tile(sdo, p.dout + (long long)(start + m0) * p.do_stride + (long long)h * D,
            [&](int r) { return (long long)r * p.do_stride; }, qvalid, tid, 128);
  cp_async_commit();
  const int g = lane >> 2, c = lane & 3;
  const int qpos0 = m0 + warp * 16 + g, qpos1 = qpos0 + 8;
  const bool ok0 = qpos0 < len, ok1 = qpos1 < len;
  const float ln2inv = 1.4426950408889634f;
  const float lse0 = ok0 ? p.lse[(long long)h * p.T + start + qpos0] * ln2inv : INFINITY;
  const float lse1 = ok1 ? p.lse[(long long)h * p.T + start + qpos1] * ln2inv : INFINITY;
  const float del0 = ok0 ? p.delta[(long long)h * p.T + start + qpos0] : 0.f;
  const float del1 = ok1 ? p.delta[(long long)h * p.T + start + qpos1] : 0.f;
  float dq[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
  for (int j = 0; j <= qb; ++j) {
    const int kv = min(BN, len - j * BN);
    __syncthreads();
    load_tile(sk, p.k + (long long)(start + j * BN) * p.k_stride + (long long)hk * D,
              [&](int r) { return (long long)r * p.k_stride; }, kv, tid, 128);
    load_tile(sv, p.v + (long long)(start + j * BN) * p.v_stride + (long long)hk * D,
              [&](int r) { return (long long)r * p.v_stride; }, kv, tid, 128);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[jj][i] = dp[jj][i] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4], a2[4];
      load_a(sq, warp * 16, ks, lane, a);
      load_a(sdo, warp * 16, ks, lane, a2);
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        uint32_t b00, b01, b10, b11;
        load_b_nt(sk, pp * 16, ks, lane, b00, b01, b10, b11);
        mma16816(s[2 * pp], a, b00, b01);
        mma16816(s[2 * pp + 1], a, b10, b11);
        load_b_nt(sv, pp * 16, ks, lane, b00, b01, b10, b11);
        mma16816(dp[2 * pp], a2, b00, b01);
        mma16816(dp[2 * pp + 1], a2, b10, b11);
      }
    }
    uint32_t dsa[4][4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int k0 = j * BN + jj * 8 + 2 * c;
      const float p00 = (k0 > qpos0) ? 0.f : exp2f(s[jj][0] * p.scale_log2 - lse0);
      const float p01 = (k0 + 1 > qpos0) ? 0.f : exp2f(s[jj][1] * p.scale_log2 - lse0);
      const float p10 = (k0 > qpos1) ? 0.f : exp2f(s[jj][2] * p.scale_log2 - lse1);
      const float p11 = (k0 + 1 > qpos1) ? 0.f : exp2f(s[jj][3] * p.scale_log2 - lse1);
      const float v00 = p00 * (dp[jj][0] - del0), v01 = p01 * (dp[jj][1] - del0);
      const float v10 = p10 * (dp[jj][2] - del1), v11 = p11 * (dp[jj][3] - del1);
      const int kk = jj >> 1;
      if ((jj & 1) == 0) { dsa[kk][0] = pack2(v00, v01); dsa[kk][1] = pack2(v10, v11); }
      else { dsa[kk][2] = pack2(v00, v01); dsa[kk][3] = pack2(v10, v11); }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int pp = 0; pp < 8; ++pp) {
        uint32_t b00, b01, b10, b11;
        load_b_t(sk, kk * 16, pp, lane, b00, b01, b10, b11);
        mma16816(dq[2 * pp], dsa[kk], b00, b01);
        mma16816(dq[2 * pp + 1], dsa[kk], b10, b11);
      }
  }
  __nv_bfloat16* d0 = p.dq + (long long)(start + qpos0) * p.dq_stride + (long long)h * D;
  __nv_bfloat16* d1 = p.dq + (long long)(start + qpos1) * p.dq_stride + (long long)h * D;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * c;
    if (ok0) *reinterpret_cast<uint32_t*>(d0 + col) = pack2(dq[n][0] * p.scale, dq[n][1] * p.scale);
    if (ok1) *reinterpret_cast<uint32_t*>(d1 + col) = pack2(dq[n][2] * p.scale, dq[n][3] * p.scale);
  }
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
constexpr long long kNoAllocWsFloats = 1ll << 20;
static __device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
static float* g_noalloc_ws_ptr[128] = {nullptr};

extern "C" int mb_attn_decode_noalloc(const void* q, const void* kc, const void* vc, void* o,
                                      const int* page_table, const int* ctx_lens, int B,
                                      int max_pages, long long num_slots, int nq, int nkv,
                                      float softmax_scale, cudaStream_t st) {
  if (B == 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return -10;
  const long long nsplit = mb_attn_decode_nsplit(max_pages);
  const long long need = nsplit > 1 ? (long long)B * nq * nsplit * (D + 2) : 0;
  if (need > kNoAllocWsFloats) return -9;  // MB_NOALLOC_TOO_LARGE
  if (g_noalloc_ws_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_ws) != cudaSuccess || ptr == nullptr) return -11;
    g_noalloc_ws_ptr[dev] = static_cast<float*>(ptr);
  }
  float* ws_o = g_noalloc_ws_ptr[dev];
  float* ws_ml = ws_o + (long long)B * nq * nsplit * D;
  return mb_attn_decode(q, kc, vc, o, page_table, ctx_lens, B, max_pages, num_slots, nq, nkv,
                        softmax_scale, ws_o, ws_ml, nullptr, st);
}
