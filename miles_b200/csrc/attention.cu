// Deterministic causal attention for head_dim 128, bf16 in / fp32 softmax, GQA (sm_100a).
//
//  * attn_fwd      : packed variable-length sequences (training and rollout prefill)
//  * attn_decode   : one query token per sequence against a paged KV cache (rollout decode)
//  * attn_bwd_dkdv / attn_bwd_dq : deterministic backward (no atomics; each output tile is
//    owned by one CTA that walks its inputs in a fixed order)
//
// Bitwise train/rollout parity: attn_fwd and attn_decode both call `kv_block_update` for every
// 64-key block 0..floor(qpos/64) of a query row, with the same fragment layout, the same
// masking rule (key position > query position => -inf, rows beyond the valid keys are
// zero-filled) and the same online-softmax arithmetic. A query row therefore gets the same
// bits whether it is one row of a 64-row training tile (rows = tokens of one head) or one
// row of a decode tile (rows = the query heads sharing a KV head).
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) fed by ldmatrix from
// XOR-swizzled shared memory and cp.async double buffering.
//
// Reference roles replaced: TE/cuDNN fused attention and flash-attn varlen (E5,
// `--attention-backend flash`), SGLang paged decode attention (E7).
#include "common.cuh"

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

// Online-softmax update of one warp's 16 query rows with one 64-key block.
//   qf      : Q A-fragments (8 k-steps)
//   ktile/vtile : swizzled smem tiles of the block's keys/values (invalid rows zero-filled)
//   kbase   : absolute position of key 0 of the block
//   qpos0/1 : absolute positions of this thread's rows g and g+8 (mask key > qpos)
//   m, l    : running max (scaled, log2 domain) and sum for rows g, g+8
//   o       : 16 n8-tiles x 4 fp32 accumulators
MB_DEVICE void kv_block_update(const uint32_t (&qf)[8][4], uint32_t ktile, uint32_t vtile,
                               int kbase, int qpos0, int qpos1, float scale_log2, float (&m)[2],
                               float (&l)[2], float (&o)[16][4], int lane) {
  float s[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      uint32_t b00, b01, b10, b11;
      load_b_nt(ktile, p * 16, ks, lane, b00, b01, b10, b11);
      mma16816(s[2 * p], qf[ks], b00, b01);
      mma16816(s[2 * p + 1], qf[ks], b10, b11);
    }
  }
  const int c = lane & 3;
  float mx0 = m[0], mx1 = m[1];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int k0 = kbase + j * 8 + 2 * c;
    s[j][0] = (k0 > qpos0) ? -INFINITY : s[j][0] * scale_log2;
    s[j][1] = (k0 + 1 > qpos0) ? -INFINITY : s[j][1] * scale_log2;
    s[j][2] = (k0 > qpos1) ? -INFINITY : s[j][2] * scale_log2;
    s[j][3] = (k0 + 1 > qpos1) ? -INFINITY : s[j][3] * scale_log2;
    mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
    mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
  // rows that have seen no valid key yet keep max -inf; use 0 as the subtrahend so exp2 = 0
  const float sub0 = (mx0 == -INFINITY) ? 0.f : mx0;
  const float sub1 = (mx1 == -INFINITY) ? 0.f : mx1;
  const float alpha0 = exp2f(((m[0] == -INFINITY) ? sub0 : m[0]) - sub0);
  const float alpha1 = exp2f(((m[1] == -INFINITY) ? sub1 : m[1]) - sub1);
  m[0] = mx0;
  m[1] = mx1;
  float rs0 = 0.f, rs1 = 0.f;
  uint32_t pa[4][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float p0 = exp2f(s[j][0] - sub0), p1 = exp2f(s[j][1] - sub0);
    const float p2 = exp2f(s[j][2] - sub1), p3 = exp2f(s[j][3] - sub1);
    // round P to bf16 first so the normaliser sums exactly what the PV product consumes
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(p0, p1);
    const __nv_bfloat162 h23 = __floats2bfloat162_rn(p2, p3);
    rs0 += __low2float(h01) + __high2float(h01);
    rs1 += __low2float(h23) + __high2float(h23);
    const int kk = j >> 1;
    if ((j & 1) == 0) {
      pa[kk][0] = *reinterpret_cast<const uint32_t*>(&h01);
      pa[kk][1] = *reinterpret_cast<const uint32_t*>(&h23);
    } else {
      pa[kk][2] = *reinterpret_cast<const uint32_t*>(&h01);
      pa[kk][3] = *reinterpret_cast<const uint32_t*>(&h23);
    }
  }
  rs0 += __shfl_xor_sync(0xffffffff, rs0, 1);
  rs0 += __shfl_xor_sync(0xffffffff, rs0, 2);
  rs1 += __shfl_xor_sync(0xffffffff, rs1, 1);
  rs1 += __shfl_xor_sync(0xffffffff, rs1, 2);
  l[0] = l[0] * alpha0 + rs0;
  l[1] = l[1] * alpha1 + rs1;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    o[n][0] *= alpha0; o[n][1] *= alpha0;
    o[n][2] *= alpha1; o[n][3] *= alpha1;
  }
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      uint32_t b00, b01, b10, b11;
      load_b_t(vtile, kk * 16, p, lane, b00, b01, b10, b11);
      mma16816(o[2 * p], pa[kk], b00, b01);
      mma16816(o[2 * p + 1], pa[kk], b10, b11);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Canonical split-KV combination. Keys are processed in chunks of CHUNK_BLOCKS blocks; each
// chunk's (m, l, o) starts from scratch and the chunk partials are merged in increasing chunk
// order into a running total. The prefill kernel performs the merges in registers/shared
// memory; the decode path computes chunks in separate CTAs and merges them in a combine
// kernel with the very same non-contracted float operations, so both give identical bits.
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

// Write normalised output rows and LSE (natural log).
MB_DEVICE void finish_rows(const float (&o)[16][4], const float (&m)[2], const float (&l)[2],
                           __nv_bfloat16* out0, __nv_bfloat16* out1, bool ok0, bool ok1,
                           float* lse0, float* lse1, int lane) {
  const int c = lane & 3;
  const float inv0 = l[0] > 0.f ? __frcp_rn(l[0]) : 0.f;
  const float inv1 = l[1] > 0.f ? __frcp_rn(l[1]) : 0.f;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * c;
    if (ok0)
      *reinterpret_cast<uint32_t*>(out0 + col) =
          pack2(__fmul_rn(o[n][0], inv0), __fmul_rn(o[n][1], inv0));
    if (ok1)
      *reinterpret_cast<uint32_t*>(out1 + col) =
          pack2(__fmul_rn(o[n][2], inv1), __fmul_rn(o[n][3], inv1));
  }
  if (c == 0) {
    const float ln2 = 0.69314718055994530942f;
    if (ok0 && lse0) *lse0 = (l[0] > 0.f) ? (m[0] + log2f(l[0])) * ln2 : -INFINITY;
    if (ok1 && lse1) *lse1 = (l[1] > 0.f) ? (m[1] + log2f(l[1])) * ln2 : -INFINITY;
  }
}

struct FwdParams {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16* o;
  float* lse;               // [nq, total_tokens]
  const int* cu_seqlens;    // [B+1]
  const int* blk_seq;       // per q-block: sequence index
  const int* blk_idx;       // per q-block: block index inside the sequence
  long long q_stride, k_stride, v_stride, o_stride;  // token row strides (elements)
  int nq, nkv, total_tokens;
  float scale_log2;
};

__global__ void __launch_bounds__(128) attn_fwd_kernel(const FwdParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sq = smem_u32(smem);
  const uint32_t sk[2] = {sq + TILE_BYTES, sq + 3 * TILE_BYTES};
  const uint32_t sv[2] = {sq + 2 * TILE_BYTES, sq + 4 * TILE_BYTES};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = p.blk_seq[blockIdx.x], qb = p.blk_idx[blockIdx.x];
  const int h = blockIdx.y, hk = h / (p.nq / p.nkv);
  const int start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - start;
  const int m0 = qb * BM;
  const int qvalid = min(BM, len - m0);
  const __nv_bfloat16* qbase = p.q + (long long)(start + m0) * p.q_stride + (long long)h * D;
  load_tile(sq, qbase, [&](int r) { return (long long)r * p.q_stride; }, qvalid, tid, 128);
  const __nv_bfloat16* kb = p.k + (long long)start * p.k_stride + (long long)hk * D;
  const __nv_bfloat16* vb = p.v + (long long)start * p.v_stride + (long long)hk * D;
  const int nblocks = qb + 1;  // causal: key blocks 0..qb
  auto load_kv = [&](int j, int buf) {
    const int kv = min(BN, len - j * BN);
    load_tile(sk[buf], kb + (long long)j * BN * p.k_stride,
              [&](int r) { return (long long)r * p.k_stride; }, kv, tid, 128);
    load_tile(sv[buf], vb + (long long)j * BN * p.v_stride,
              [&](int r) { return (long long)r * p.v_stride; }, kv, tid, 128);
  };
  load_kv(0, 0);
  cp_async_commit();
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int g = lane >> 2;
  const int qpos0 = m0 + warp * 16 + g, qpos1 = qpos0 + 8;
  uint32_t qf[8][4];
  // running total of merged chunks: O in shared memory laid out [element][thread]
  float* otot = reinterpret_cast<float*>(smem + 5 * TILE_BYTES);
  float Mt[2] = {-INFINITY, -INFINITY}, Lt[2] = {0.f, 0.f};
  auto merge_chunk = [&]() {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float fa, fb;
      merge_stats(Mt[r], Lt[r], m[r], l[r], fa, fb);
#pragma unroll
      for (int n = 0; n < 16; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int i = n * 4 + r * 2 + e;
          otot[i * 128 + tid] = merge_val(otot[i * 128 + tid], o[n][r * 2 + e], fa, fb);
        }
    }
  };
  for (int j = 0; j < nblocks; ++j) {
    if (j + 1 < nblocks) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) load_a(sq, warp * 16, ks, lane, qf[ks]);
    }
    if (j > 0 && j % CHUNK_BLOCKS == 0) {  // chunk boundary: fold the finished chunk in
      merge_chunk();
#pragma unroll
      for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m[0] = m[1] = -INFINITY;
      l[0] = l[1] = 0.f;
    }
    kv_block_update(qf, sk[j & 1], sv[j & 1], j * BN, qpos0, qpos1, p.scale_log2, m, l, o, lane);
    __syncthreads();
  }
  cp_async_wait<0>();
  if (nblocks > CHUNK_BLOCKS) {
    merge_chunk();
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[n][i] = otot[(n * 4 + i) * 128 + tid];
    m[0] = Mt[0]; m[1] = Mt[1];
    l[0] = Lt[0]; l[1] = Lt[1];
  }
  const bool ok0 = qpos0 < len, ok1 = qpos1 < len;
  __nv_bfloat16* out0 = p.o + (long long)(start + qpos0) * p.o_stride + (long long)h * D;
  __nv_bfloat16* out1 = p.o + (long long)(start + qpos1) * p.o_stride + (long long)h * D;
  float* lse0 = p.lse ? p.lse + (long long)h * p.total_tokens + start + qpos0 : nullptr;
  float* lse1 = p.lse ? p.lse + (long long)h * p.total_tokens + start + qpos1 : nullptr;
  finish_rows(o, m, l, out0, out1, ok0, ok1, lse0, lse1, lane);
}

// ---------------------------------------------------------------------------------------------
// Decode: CTA = (sequence, kv head, chunk), four warps; rows = the G query heads of the group
// (G <= 16).
// KV cache layout: [num_slots, nkv, 128] with slot = page * 64 + offset; block j of a sequence
// is page page_table[b][j].
// ---------------------------------------------------------------------------------------------
struct DecParams {
  const __nv_bfloat16* q;   // [B, nq, 128]
  const __nv_bfloat16 *kc, *vc;
  __nv_bfloat16* o;         // [B, nq, 128]
  const int* page_table;    // [B, max_pages]
  const int* ctx_lens;      // [B] number of valid keys (query position = ctx_len - 1)
  int max_pages, nq, nkv;
  float scale_log2;
  float* ws_o;              // [B, nq, nsplit_max, 128] chunk partial outputs (unnormalised)
  float* ws_ml;             // [B, nq, nsplit_max, 2]   chunk partial (m, l)
  int nsplit_max;
};

constexpr int DEC_STAGES = 3;
constexpr int DEC_WARPS = 4;
// shared memory: Q (16 rows) | DEC_STAGES x (K tile, V tile) | P fragments | row-max partials
constexpr int DEC_Q_BYTES = 16 * D * 2;
constexpr int DEC_P_OFF = DEC_Q_BYTES + 2 * DEC_STAGES * TILE_BYTES;
constexpr int DEC_RED_OFF = DEC_P_OFF + 4 * 4 * 32 * 4;
constexpr int DEC_SMEM = DEC_RED_OFF + DEC_WARPS * 2 * 32 * 4;

// kv_block_update computed by four warps of one CTA, with bit-identical results. Warp w owns
// keys 16w..16w+15 of the score tile (score fragments s[2w], s[2w+1] of the one-warp version,
// accumulated over the same k-steps) and output columns 32w..32w+31 (n-tiles 4w..4w+3, fed by
// the same P fragments in the same k order). The row max is exact in any order; the row sum is
// recomputed by every warp from the shared P fragments in the one-warp order (j = 0..7, then
// the two xor shuffles), so every warp holds the same (m, l) as kv_block_update would.
MB_DEVICE void kv_block_update_4w(const uint32_t (&qf)[8][4], uint32_t ktile, uint32_t vtile,
                                  uint32_t* __restrict__ pbuf, float* __restrict__ red, int kbase,
                                  int qpos, float scale_log2, float (&m)[2], float (&l)[2],
                                  float (&o)[4][4], int warp, int lane) {
  float s[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t b00, b01, b10, b11;
    load_b_nt(ktile, warp * 16, ks, lane, b00, b01, b10, b11);
    mma16816(s[0], qf[ks], b00, b01);
    mma16816(s[1], qf[ks], b10, b11);
  }
  const int c = lane & 3;
  float mx0 = m[0], mx1 = m[1];
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int k0 = kbase + (2 * warp + jj) * 8 + 2 * c;
    s[jj][0] = (k0 > qpos) ? -INFINITY : s[jj][0] * scale_log2;
    s[jj][1] = (k0 + 1 > qpos) ? -INFINITY : s[jj][1] * scale_log2;
    s[jj][2] = (k0 > qpos) ? -INFINITY : s[jj][2] * scale_log2;
    s[jj][3] = (k0 + 1 > qpos) ? -INFINITY : s[jj][3] * scale_log2;
    mx0 = fmaxf(mx0, fmaxf(s[jj][0], s[jj][1]));
    mx1 = fmaxf(mx1, fmaxf(s[jj][2], s[jj][3]));
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
  red[(warp * 2 + 0) * 32 + lane] = mx0;
  red[(warp * 2 + 1) * 32 + lane] = mx1;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < DEC_WARPS; ++w) {
    mx0 = fmaxf(mx0, red[(w * 2 + 0) * 32 + lane]);
    mx1 = fmaxf(mx1, red[(w * 2 + 1) * 32 + lane]);
  }
  const float sub0 = (mx0 == -INFINITY) ? 0.f : mx0;
  const float sub1 = (mx1 == -INFINITY) ? 0.f : mx1;
  const float alpha0 = exp2f(((m[0] == -INFINITY) ? sub0 : m[0]) - sub0);
  const float alpha1 = exp2f(((m[1] == -INFINITY) ? sub1 : m[1]) - sub1);
  m[0] = mx0;
  m[1] = mx1;
  // this warp's P fragments: kk = warp; registers 0/1 from jj = 0, registers 2/3 from jj = 1
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const float p0 = exp2f(s[jj][0] - sub0), p1 = exp2f(s[jj][1] - sub0);
    const float p2 = exp2f(s[jj][2] - sub1), p3 = exp2f(s[jj][3] - sub1);
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(p0, p1);
    const __nv_bfloat162 h23 = __floats2bfloat162_rn(p2, p3);
    pbuf[(warp * 4 + jj * 2 + 0) * 32 + lane] = *reinterpret_cast<const uint32_t*>(&h01);
    pbuf[(warp * 4 + jj * 2 + 1) * 32 + lane] = *reinterpret_cast<const uint32_t*>(&h23);
  }
  __syncthreads();
  uint32_t pa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
#pragma unroll
    for (int r = 0; r < 4; ++r) pa[kk][r] = pbuf[(kk * 4 + r) * 32 + lane];
  float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int kk = j >> 1, r = (j & 1) * 2;
    const __nv_bfloat162 h01 = *reinterpret_cast<const __nv_bfloat162*>(&pa[kk][r]);
    const __nv_bfloat162 h23 = *reinterpret_cast<const __nv_bfloat162*>(&pa[kk][r + 1]);
    rs0 += __low2float(h01) + __high2float(h01);
    rs1 += __low2float(h23) + __high2float(h23);
  }
  rs0 += __shfl_xor_sync(0xffffffff, rs0, 1);
  rs0 += __shfl_xor_sync(0xffffffff, rs0, 2);
  rs1 += __shfl_xor_sync(0xffffffff, rs1, 1);
  rs1 += __shfl_xor_sync(0xffffffff, rs1, 2);
  l[0] = l[0] * alpha0 + rs0;
  l[1] = l[1] * alpha1 + rs1;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    o[n][0] *= alpha0; o[n][1] *= alpha0;
    o[n][2] *= alpha1; o[n][3] *= alpha1;
  }
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      uint32_t b00, b01, b10, b11;
      load_b_t(vtile, kk * 16, warp * 2 + pp, lane, b00, b01, b10, b11);
      mma16816(o[2 * pp], pa[kk], b00, b01);
      mma16816(o[2 * pp + 1], pa[kk], b10, b11);
    }
  }
}

// One CTA of four warps per (sequence, kv head, 1024-key chunk).
__global__ void __launch_bounds__(DEC_WARPS * 32) attn_decode_kernel(const DecParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sq = smem_u32(smem);
  uint32_t* pbuf = reinterpret_cast<uint32_t*>(smem + DEC_P_OFF);
  float* red = reinterpret_cast<float*>(smem + DEC_RED_OFF);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x, hk = blockIdx.y;
  const int G = p.nq / p.nkv;
  const int ctx = p.ctx_lens[b];
  if (ctx <= 0) return;
  const int qpos = ctx - 1;
  const int nblocks_all = qpos / BN + 1;
  const int nsplit = (nblocks_all + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS;
  const int split = blockIdx.z;
  if (split >= nsplit) return;
  const int jbeg = split * CHUNK_BLOCKS;
  const int nblocks = min(nblocks_all - jbeg, CHUNK_BLOCKS);
  const __nv_bfloat16* qbase = p.q + ((long long)b * p.nq + (long long)hk * G) * D;
  for (int i = tid; i < 16 * 16; i += DEC_WARPS * 32) {  // 16 query rows, rows >= G zero
    const int r = i >> 4, ch = i & 15;
    const bool ok = r < G;
    cp_async16(sq + swz(r, ch), ok ? qbase + (long long)r * D + ch * 8 : qbase, ok);
  }
  const long long kstride = (long long)p.nkv * D;
  auto kv_tile = [&](int j, int which) {
    return sq + DEC_Q_BYTES + (uint32_t)((j % DEC_STAGES) * 2 + which) * TILE_BYTES;
  };
  auto load_kv = [&](int j) {  // j: block index local to this split
    const int jj = jbeg + j;
    const int page = p.page_table[(long long)b * p.max_pages + jj];
    const int kv = min(BN, ctx - jj * BN);
    const long long slot0 = (long long)page * BN;
    load_tile(kv_tile(j, 0), p.kc + slot0 * kstride + (long long)hk * D,
              [&](int r) { return (long long)r * kstride; }, kv, tid, DEC_WARPS * 32);
    load_tile(kv_tile(j, 1), p.vc + slot0 * kstride + (long long)hk * D,
              [&](int r) { return (long long)r * kstride; }, kv, tid, DEC_WARPS * 32);
  };
#pragma unroll
  for (int s = 0; s < DEC_STAGES - 1; ++s) {
    if (s < nblocks) load_kv(s);
    cp_async_commit();
  }
  float o[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  uint32_t qf[8][4];
  for (int j = 0; j < nblocks; ++j) {
    if (j + DEC_STAGES - 1 < nblocks) load_kv(j + DEC_STAGES - 1);
    cp_async_commit();
    cp_async_wait<DEC_STAGES - 1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) load_a(sq, 0, ks, lane, qf[ks]);
    }
    kv_block_update_4w(qf, kv_tile(j, 0), kv_tile(j, 1), pbuf, red, (jbeg + j) * BN, qpos,
                       p.scale_log2, m, l, o, warp, lane);
    __syncthreads();  // the stage and P buffers are rewritten next iteration
  }
  cp_async_wait<0>();
  const int g = lane >> 2, c = lane & 3;
  if (nsplit == 1) {
    // same arithmetic as finish_rows, for this warp's 32 columns
    const float inv0 = l[0] > 0.f ? __frcp_rn(l[0]) : 0.f;
    const float inv1 = l[1] > 0.f ? __frcp_rn(l[1]) : 0.f;
    __nv_bfloat16* out0 = p.o + ((long long)b * p.nq + (long long)hk * G + g) * D;
    __nv_bfloat16* out1 = out0 + 8 * D;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int col = (warp * 4 + n) * 8 + 2 * c;
      if (g < G)
        *reinterpret_cast<uint32_t*>(out0 + col) =
            pack2(__fmul_rn(o[n][0], inv0), __fmul_rn(o[n][1], inv0));
      if (g + 8 < G)
        *reinterpret_cast<uint32_t*>(out1 + col) =
            pack2(__fmul_rn(o[n][2], inv1), __fmul_rn(o[n][3], inv1));
    }
    return;
  }
  // several chunks: publish this chunk's partial for the combine kernel
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + r * 8;
    if (row >= G) continue;
    const long long base = ((long long)b * p.nq + (long long)hk * G + row) * p.nsplit_max + split;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int col = (warp * 4 + n) * 8 + 2 * c;
      p.ws_o[base * D + col] = o[n][r * 2];
      p.ws_o[base * D + col + 1] = o[n][r * 2 + 1];
    }
    if (c == 0 && warp == 0) {
      p.ws_ml[base * 2] = m[r];
      p.ws_ml[base * 2 + 1] = l[r];
    }
  }
}

// Merge the chunk partials of every (sequence, query head) in chunk order (same operations as
// the prefill kernel's in-register merge) and write the bf16 output. One warp per row; lane
// owns columns lane*4 .. lane*4+3.
__global__ void attn_decode_combine_kernel(const DecParams p, int B) {
  pdl_trigger();
  pdl_wait();
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)B * p.nq) return;
  const int b = (int)(w / p.nq);
  const int ctx = p.ctx_lens[b];
  if (ctx <= 0) return;
  const int nsplit = ((ctx - 1) / BN + 1 + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS;
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

extern "C" int mb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                           const int* cu_seqlens, const int* blk_seq, const int* blk_idx,
                           int nblocks, long long q_stride, long long k_stride, long long v_stride,
                           long long o_stride, int nq, int nkv, int T, float softmax_scale,
                           cudaStream_t st) {
  if (nblocks == 0) return 0;
  if (nq % nkv) return -1;
  FwdParams p{(const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
              (__nv_bfloat16*)o, lse, cu_seqlens, blk_seq, blk_idx, q_stride, k_stride, v_stride,
              o_stride, nq, nkv, T, softmax_scale * 1.4426950408889634f};
  const int smem = 5 * TILE_BYTES + 64 * 128 * (int)sizeof(float);  // + merged-chunk totals
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    set = true;
  }
  mb_launch(attn_fwd_kernel, dim3(nblocks, nq), 128, smem, st, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Number of 1024-key chunks a decode over `max_pages` pages can need (workspace sizing).
extern "C" int mb_attn_decode_nsplit(int max_pages) {
  return (max_pages + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS;
}

// ws_o: float [B, nq, nsplit_max, 128]; ws_ml: float [B, nq, nsplit_max, 2] (only touched when a
// sequence spans more than one 1024-key chunk).
extern "C" int mb_attn_decode(const void* q, const void* kc, const void* vc, void* o,
                              const int* page_table, const int* ctx_lens, int B, int max_pages,
                              int nq, int nkv, float softmax_scale, float* ws_o, float* ws_ml,
                              cudaStream_t st) {
  if (B == 0) return 0;
  if (nq % nkv || nq / nkv > 16) return -1;
  const int nsplit_max = (max_pages + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS;
  if (nsplit_max > 1 && (!ws_o || !ws_ml)) return -3;
  DecParams p{(const __nv_bfloat16*)q, (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc,
              (__nv_bfloat16*)o, page_table, ctx_lens, max_pages, nq, nkv,
              softmax_scale * 1.4426950408889634f, ws_o, ws_ml, nsplit_max};
  const int smem = DEC_SMEM;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    set = true;
  }
  mb_launch(attn_decode_kernel, dim3(B, nkv, nsplit_max), DEC_WARPS * 32, smem, st, p);
  if (nsplit_max > 1) {
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
                           float softmax_scale, cudaStream_t st) {
  if (nblocks == 0) return 0;
  if (nq % nkv) return -1;
  const long long warps = (long long)T * nq;
  mb_launch(attn_bwd_delta_kernel, (unsigned)((warps + 7) / 8), 256, 0, st, 
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, o_stride, do_stride, T, nq, delta);
  BwdParams p{(const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
              (const __nv_bfloat16*)dout, lse, delta, (__nv_bfloat16*)dq, (__nv_bfloat16*)dk,
              (__nv_bfloat16*)dv, cu_seqlens, blk_seq, blk_idx, q_stride, k_stride, v_stride,
              do_stride, dq_stride, dk_stride, dv_stride, nq, nkv, T,
              softmax_scale * 1.4426950408889634f, softmax_scale};
  const int smem_kv = 4 * TILE_BYTES + 128 * sizeof(float);
  const int smem_q = 4 * TILE_BYTES;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
    cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
    set = true;
  }
  mb_launch(attn_bwd_dkdv_kernel, dim3(nblocks, nkv), 128, smem_kv, st, p);
  mb_launch(attn_bwd_dq_kernel, dim3(nblocks, nq), 128, smem_q, st, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
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
                                      int max_pages, int nq, int nkv, float softmax_scale,
                                      cudaStream_t st) {
  if (B == 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return -10;
  const long long nsplit = (max_pages + CHUNK_BLOCKS - 1) / CHUNK_BLOCKS;
  const long long need = nsplit > 1 ? (long long)B * nq * nsplit * (D + 2) : 0;
  if (need > kNoAllocWsFloats) return -9;  // MB_NOALLOC_TOO_LARGE
  if (g_noalloc_ws_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_ws) != cudaSuccess || ptr == nullptr) return -11;
    g_noalloc_ws_ptr[dev] = static_cast<float*>(ptr);
  }
  float* ws_o = g_noalloc_ws_ptr[dev];
  float* ws_ml = ws_o + (long long)B * nq * nsplit * D;
  return mb_attn_decode(q, kc, vc, o, page_table, ctx_lens, B, max_pages, nq, nkv, softmax_scale,
                        ws_o, ws_ml, st);
}
