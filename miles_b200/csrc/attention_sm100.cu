// Causal attention forward on the 5th-generation tensor cores (sm_100a): tcgen05.mma with
// TMEM accumulators, TMA-fed K/V pipelines and warp-specialised roles. Head dim 128, bf16 in,
// fp32 softmax, GQA.
//
//  * fa_fwd_kernel<0>: packed variable-length sequences (training forward, rollout prefill,
//    log-prob passes). Work item = (128-query tile of one sequence, query head).
//  * fa_fwd_kernel<1>: one query token per sequence against the paged KV cache (decode).
//    Work item = (sequence, KV head, 1024-key chunk); the tile's rows are the query heads
//    sharing the KV head (rows >= G are discarded; warps holding none of them idle).
//  Both are persistent: one CTA per SM walks a strided list of work items, so the barrier /
//  TMEM set-up is paid once per SM and the K/V pipeline runs across item boundaries.
//
// Canonical per-row arithmetic (identical in both modes, hence bitwise train/rollout parity):
//   keys are taken in blocks of 128 (positions 128j .. 128j+127 of the sequence) and in chunks
//   of 8 blocks (1024 keys). Per block:
//     S   = Q K^T                 one tcgen05 chain of 8 UMMAs (K = 16 head dims each)
//     m'  = max(m, max(S over keys <= qpos) * scale_log2);  sub = m' (0 if -inf)
//     alpha = 2^(m - sub)  (1 for the first block)
//     p   = key > qpos ? 0 : bf16(ex2.approx(fma(S, scale_log2, -sub)))
//           rs = fixed-tree sum of p: per 32-key group four interleaved
//           partial sums ((a0+a1)+(a2+a3)), groups combined as ((g0+g1)+(g2+g3))
//     l   = fma(l, alpha, rs)
//     O_j = P V                    one tcgen05 chain of 8 UMMAs (K = 16 keys each), fresh
//     O   = fma(O, alpha, O_j)     (O kept in registers, one row per thread)
//   Chunks start from (m, l, O) = (-inf, 0, 0) and are merged in chunk order with
//   non-contracted float operations: by the prefill CTA itself (running total in TMEM) or, for
//   decode, by attn_decode_combine_kernel (csrc/attention.cu) from per-chunk partials.
//
// Roles (320 threads): warp 0 = TMA producer (Q once, then K_j / V_j through a 2-stage ring),
// warp 1 = TMEM owner and MMA issuer (S_j into a double-buffered S, O_j into a single O_j
// buffer), warps 2-9 = softmax / output: two threads per row (TMEM lane), each owning 64 of
// the 128 columns. TMEM: S0 | S1 | O_j | Otot, 128 columns each. P_j (bf16) is written over its
// S buffer (keys 0-63 in columns 0-31, keys 64-127 in columns 64-95: each thread overwrites only
// scores it has already read) and fed to the P.V UMMA straight from tensor memory; the
// O_j fold is deferred to the end of the next block so the softmax never waits for P.V.
//
// Reference roles replaced: flash-attention / cuDNN fused attention forward used by Megatron
// (`--attention-backend flash`) and SGLang's paged decode attention.
#include "common.cuh"

#include <cstdio>

namespace mb {
namespace fa {

constexpr int D = 128;
constexpr int BM = 128;      // query rows per tile
constexpr int BN = 128;      // keys per block
constexpr int CHUNK = 8;     // blocks per canonical chunk (1024 keys)
constexpr int SUB = 128 * 64 * 2;   // one [128][64] bf16 SW128 sub-tile = 16 KB
constexpr int TILE = 2 * SUB;       // [128][128] bf16 = 32 KB
// shared memory map (offsets from a 1024-aligned base)
constexpr int NST = 2;       // K/V pipeline stages
constexpr int OFF_Q = 0;
constexpr int OFF_K = TILE;                  // NST stages
constexpr int OFF_V = OFF_K + NST * TILE;    // NST stages
constexpr int OFF_P = OFF_V + NST * TILE;    // fast decode (mode 2): two P tiles (SS P.V)
constexpr int OFF_RED = OFF_P + 2 * TILE;    // softmax row max / sum exchange, 2 x [2][128] f32
constexpr int OFF_BAR = OFF_RED + 2048;
constexpr int NTHREADS = 320;              // producer, MMA, 8 softmax warps
// The dynamic shared memory of this kernel starts 1024-aligned (it has no static shared
// memory); the kernel checks that and exits with error 2 otherwise, so no slack is requested.
constexpr int SMEM_BYTES = OFF_BAR + 256 /*barriers*/;
static_assert(SMEM_BYTES <= 232448, "fa_fwd_kernel shared memory exceeds the 227 KB limit");

struct Params {
  // mode 0
  const int* cu_seqlens;   // [B+1]
  const int* tile_seq;     // per CTA x: sequence index
  const int* tile_idx;     // per CTA x: 128-row tile index inside the sequence
  float* lse;              // [nq, total_tokens] (natural log), may be null
  long long o_stride;      // output token row stride (elements)
  int total_tokens;
  // mode 1
  const int* page_table;   // [B, max_pages] (64-token pages)
  const int* ctx_lens;     // [B]
  int max_pages;
  float* ws_o;             // [B, nq, nsplit_max, 128]
  float* ws_ml;            // [B, nq, nsplit_max, 2]
  int nsplit_max;
  int q_rows;              // query rows loaded per item (the G valid heads, rounded up to 8)
  // common
  __nv_bfloat16* o;
  int nq, nkv;
  float scale_log2;
  int* err;
};

MB_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A (M = 128 lanes x K = 16 bf16 packed in 8
// 32-bit columns, lower k in the low half) is read from tensor memory.
MB_DEVICE void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// 2^x with the hardware approximation (ex2.approx.ftz): one MUFU op; 2^-inf = +0.
MB_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
MB_DEVICE void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
MB_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
MB_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// chunk merge (same operations as the decode combine kernel)
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

// Bounded wait shared by all roles: gives up (and records code 2) after the wait limit.
MB_DEVICE bool wait_bar(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait(bar, parity, err, 2);
}
// Warp-uniform bounded wait (every lane polls; the result is true only if all lanes saw the
// phase complete), for warps that go on to warp-collective tcgen05.ld / tcgen05.st.
MB_DEVICE bool wait_warp(uint64_t* bar, uint32_t parity, int* err, int code) {
  return __all_sync(0xffffffff, mbar_wait(bar, parity, err, code));
}

// Work item of a persistent CTA. Mode 0: item = (128-row tile, query head), heads fastest so
// that CTAs running at the same time share K/V tiles through L2. Mode 1: item = (sequence, KV
// head, chunk). nblk == 0 marks an empty item (decode chunk past the context end).
struct Item {
  int seq_start, len, m0, h, hk, b, split, qpos, jbeg, nblk, nsplit;
};

template <int MODE>
MB_DEVICE Item get_item(const Params& p, int t) {
  Item it{};
  const int G = p.nq / p.nkv;
  if (MODE == 0) {
    const int tile = t / p.nq;
    it.h = t - tile * p.nq;
    it.hk = it.h / G;
    it.b = p.tile_seq[tile];
    const int qt = p.tile_idx[tile];
    it.seq_start = p.cu_seqlens[it.b];
    it.len = p.cu_seqlens[it.b + 1] - it.seq_start;
    it.m0 = qt * BM;
    it.nblk = qt + 1;  // causal: key blocks 0..qt (BM == BN)
    it.nsplit = 1;
  } else {
    const int per_b = p.nkv * p.nsplit_max;
    it.b = t / per_b;
    const int r = t - it.b * per_b;
    it.hk = r / p.nsplit_max;
    it.split = r - it.hk * p.nsplit_max;
    const int ctx = __ldg(p.ctx_lens + it.b);
    it.nblk = 0;
    it.nsplit = 1;
    if (ctx > 0) {
      it.qpos = ctx - 1;
      const int nb_all = it.qpos / BN + 1;
      it.nsplit = (nb_all + CHUNK - 1) / CHUNK;
      if (it.split < it.nsplit) {
        it.jbeg = it.split * CHUNK;
        it.nblk = min(nb_all - it.jbeg, CHUNK);
      }
    }
  }
  return it;
}

// Persistent: CTA x processes items x, x + gridDim.x, ... Buffer indices and mbarrier parities
// follow running counters (blocks `g`, non-empty items `n`) that every role advances alike.
template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 1) fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                        const __grid_constant__ CUtensorMap tmK,
                                                        const __grid_constant__ CUtensorMap tmV,
                                                        const Params p, int n_items) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                // [NST]
  uint64_t* k_empty = k_full + NST;           // [NST]
  uint64_t* v_full = k_empty + NST;           // [NST]
  uint64_t* v_empty = v_full + NST;           // [NST]
  uint64_t* s_full = v_empty + NST;           // [2]
  uint64_t* p_full = s_full + 2;              // [2] one per S/P buffer
  uint64_t* q_empty = p_full + 2;
  uint64_t* o_full = q_empty + 1;
  uint64_t* o_empty = o_full + 1;
  uint64_t* red_bar = o_empty + 1;            // [2] fast decode: max / sum exchange of 4 warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 2);
  if (smem != smem_raw) {  // not 1024-aligned: the shared-memory budget has no slack for it
    if (threadIdx.x == 0) report_error(p.err, 2);
    return;
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.nq / p.nkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_full + s, MODE == 2 ? 4 : 8);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, MODE == 2 ? 4 : 8);
    mbar_init(red_bar, 4);
    mbar_init(red_bar + 1, 4);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // device inputs (including the work tables) are read only after this point

  if (warp == 0) {
    // ================= TMA producer =================
    if (elect_one()) {
      int g = 0, n = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x) {
        const Item it = get_item<MODE>(p, t);
        if (it.nblk == 0) continue;
        uint8_t* sq = smem + OFF_Q;
        if (!wait_bar(q_empty, (n & 1) ^ 1, p.err)) break;
        // decode loads only the G query heads of the item (rows past them stay stale; every row
        // of S, P and O depends only on its own query row, and those rows are discarded)
        mbar_arrive_expect_tx(q_full, MODE == 0 ? TILE : MODE == 2 ? 8 * 1024 : 2 * p.q_rows * 128);
        if (MODE == 0) {
          tma_load_2d(sq, &tmQ, q_full, it.h * D, it.seq_start + it.m0);
          tma_load_2d(sq + SUB, &tmQ, q_full, it.h * D + 64, it.seq_start + it.m0);
        } else if (MODE == 2) {
          // fast decode: the G (<= 8) heads four times, in tile rows 32q + h (q = 0..3): row
          // 32q + h of S is head h's scores, read by lane h of softmax warp 4 + q
          const int row = it.b * p.nq + it.hk * G;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tma_load_2d(sq + c * 4096, &tmQ, q_full, 0, row);
            tma_load_2d(sq + SUB + c * 4096, &tmQ, q_full, 64, row);
          }
        } else {
          const int row = it.b * p.nq + it.hk * G;
          tma_load_2d(sq, &tmQ, q_full, 0, row);
          tma_load_2d(sq + SUB, &tmQ, q_full, 64, row);
        }
        ++n;
        // decode: the item's page-table entries (at most 2 * CHUNK pages) are fetched up front
        // as independent loads, instead of two dependent global loads before every block
        int pgs[2 * CHUNK];
        if (MODE != 0) {
          const int* pt = p.page_table + (long long)it.b * p.max_pages;
#pragma unroll
          for (int c = 0; c < 2 * CHUNK; ++c) {
            const int pg = 2 * it.jbeg + c;
            pgs[c] = (c < 2 * it.nblk && pg < p.max_pages) ? __ldg(pt + pg) : 0;
          }
        }
        for (int j = 0; j < it.nblk; ++j, ++g) {
          const int s = g % NST;  // K/V stage
          const uint32_t ph = ((g / NST) & 1) ^ 1;
          const int jj = it.jbeg + j;
          int y0, y1;  // rows of the two 64-key halves of the block
          if (MODE == 0) {
            y0 = it.seq_start + jj * BN;
            y1 = y0 + 64;
          } else {
            y0 = pgs[2 * j] * 64;
            y1 = pgs[2 * j + 1] * 64;
          }
          // K block: K-major sub-tiles [128 keys][64 dims]; key half at +8KB
          if (!wait_bar(k_empty + s, ph, p.err)) { ok = false; break; }
          uint8_t* sk = smem + OFF_K + s * TILE;
          mbar_arrive_expect_tx(k_full + s, TILE);
          tma_load_2d(sk, &tmK, k_full + s, it.hk * D, y0);
          tma_load_2d(sk + SUB, &tmK, k_full + s, it.hk * D + 64, y0);
          tma_load_2d(sk + SUB / 2, &tmK, k_full + s, it.hk * D, y1);
          tma_load_2d(sk + SUB + SUB / 2, &tmK, k_full + s, it.hk * D + 64, y1);
          // V block: MN-major boxes [64 keys][64 dims]; key half at +16KB, dim half at +8KB
          if (!wait_bar(v_empty + s, ph, p.err)) { ok = false; break; }
          uint8_t* sv = smem + OFF_V + s * TILE;
          mbar_arrive_expect_tx(v_full + s, TILE);
          tma_load_2d(sv, &tmV, v_full + s, it.hk * D, y0);
          tma_load_2d(sv + SUB / 2, &tmV, v_full + s, it.hk * D + 64, y0);
          tma_load_2d(sv + SUB, &tmV, v_full + s, it.hk * D, y1);
          tma_load_2d(sv + SUB + SUB / 2, &tmV, v_full + s, it.hk * D + 64, y1);
        }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(BM, D, false, true);
    const uint32_t sq = smem_u32(smem + OFF_Q);
    // O_i = P_i V_i with P_i (bf16) in TMEM columns 0..63 of S buffer i&1 (i: running block)
    auto issue_pv = [&](int i) -> bool {
      if (!wait_bar(p_full + (i & 1), (i >> 1) & 1, p.err)) return false;
      if (!wait_bar(o_empty, (i & 1) ^ 1, p.err)) return false;
      if (!wait_bar(v_full + i % NST, (i / NST) & 1, p.err)) return false;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sv = smem_u32(smem + OFF_V + (i % NST) * TILE);
        const uint32_t pa = tmem_base + (i & 1) * 128;
        const uint32_t ps = smem_u32(smem + OFF_P + (i & 1) * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bd = make_sdesc_sw128(sv + (kk >> 2) * SUB + (kk & 3) * 2048, 8192, 1024);
          if (MODE == 2) {
            // keys 16kk..16kk+15 of the P tile in shared memory (K-major SW128, like Q)
            const uint64_t ad = make_sdesc_sw128(ps + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
            umma_f16(tmem_base + 256, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
          } else {
            // keys 16kk..16kk+15: packed P columns (kk>>2)*64 + (kk&3)*8 of the S buffer
            umma_f16_ts(tmem_base + 256, pa + (kk >> 2) * 64 + (kk & 3) * 8, bd, idesc_o,
                        kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(o_full);
        umma_commit(v_empty + i % NST);
      }
      __syncwarp();
      return true;
    };
    int g = 0, n = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x) {
      const Item it = get_item<MODE>(p, t);
      if (it.nblk == 0) continue;
      if (!wait_bar(q_full, n & 1, p.err)) break;
      ++n;
      for (int j = 0; j < it.nblk; ++j, ++g) {
        const int s = g & 1;     // S / P buffer in tensor memory
        const int ks = g % NST;  // K stage in shared memory
        if (!wait_bar(k_full + ks, (g / NST) & 1, p.err)) { ok = false; break; }
        // S buffer s last held P_{g-2}: wait until PV_{g-2} has consumed it (fast decode keeps
        // P in shared memory: the softmax finished reading S_{g-2} before PV_{g-2} was issued)
        if (MODE != 2 && g >= 2 && !wait_bar(o_full, (g - 2) & 1, p.err)) { ok = false; break; }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sk = smem_u32(smem + OFF_K + ks * TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = make_sdesc_sw128(sq + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(sk + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
            umma_f16(tmem_base + s * 128, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(s_full + s);
          umma_commit(k_empty + ks);
          if (j == it.nblk - 1) umma_commit(q_empty);  // last S of the item: Q may be reloaded
        }
        __syncwarp();
        if (g >= 1 && !issue_pv(g - 1)) { ok = false; break; }
      }
    }
    if (ok && g > 0) issue_pv(g - 1);
  } else if (MODE == 2) {
    // ================= fast decode softmax / output (four warps) =================
    // Warps 4..7, warp 4 + q reading TMEM lanes 32q..32q+31. Q was loaded four times, at tile
    // rows 32q + h (h < G <= 8), so every warp finds head h's scores in its own lane h. Warp q
    // handles keys 32q .. 32q+31 of every block and output columns 32q .. 32q+31. The row
    // maximum and sum combine the four key groups through shared memory (bounded mbarrier
    // exchange) in the same order as the two-thread rows of the other modes:
    // rs = (g0 + g1) + (g2 + g3), so the results are bitwise those of the prefill kernel. Each
    // warp writes its 32 P values (bf16) into all four row copies 32q' + h of the block's
    // shared-memory P tile, so the SS P.V leaves head h's output in lane h of every lane
    // quarter; warp q folds its 32 output columns into registers.
    if (warp >= 4 && warp < 8) {
      const int q = warp & 3;
      const int h = lane & 7;
      const bool live_row = lane < G;
      const uint32_t lane_off = (uint32_t)(32 * q) << 16;
      float* red_max = reinterpret_cast<float*>(smem + OFF_RED);  // [4 groups][8 heads]
      float* red_sum = red_max + 32;                              // [4 groups][8 heads]
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x) {
        const Item it = get_item<MODE>(p, t);
        if (it.nblk == 0) continue;
        const int qpos = it.qpos;
        float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
        bool first_fold = true;
        float ot[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) ot[e] = 0.f;
        // Otot <- fma(Otot, alpha_prev, O_i) over this warp's 32 columns (Otot = 0 at first)
        auto fold_pv = [&](int i) -> bool {
          if (!wait_warp(o_full, i & 1, p.err, 2)) return false;
          tc_fence_after();
          uint32_t oj[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + 256 + 32 * q, oj);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            ot[e] = __fmaf_rn(first_fold ? 0.f : ot[e], alpha_prev, __uint_as_float(oj[e]));
          first_fold = false;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_empty);
          return true;
        };
        for (int j = 0; j < it.nblk; ++j, ++g) {
          const int s = g & 1;
          ok = ok && wait_warp(s_full + s, (g >> 1) & 1, p.err, 2);
          if (!ok) break;
          tc_fence_after();
          const int kbase = (it.jbeg + j) * BN + q * 32;
          const bool masked = j == it.nblk - 1;
          float sv[32];
          {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_off + s * 128 + q * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) sv[e] = __uint_as_float(r[e]);
          }
          float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float v = masked && kbase + e > qpos ? -INFINITY : sv[e];
            mx4[e & 3] = fmaxf(mx4[e & 3], v);
          }
          if (lane < 8) red_max[q * 8 + lane] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          __syncwarp();
          if (lane == 0) mbar_arrive(red_bar);
          ok = ok && wait_warp(red_bar, g & 1, p.err, 2);
          if (!ok) break;
          const float raw = fmaxf(fmaxf(red_max[h], red_max[8 + h]), fmaxf(red_max[16 + h], red_max[24 + h]));
          const float mnew = fmaxf(m, raw == -INFINITY ? -INFINITY : __fmul_rn(raw, p.scale_log2));
          const float sub = mnew == -INFINITY ? 0.f : mnew;
          const float alpha = exp2f(__fsub_rn(m == -INFINITY ? sub : m, sub));
          const float nsub = -sub;
          float a4[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float p0 = ex2_approx(__fmaf_rn(sv[e], p.scale_log2, nsub));
            float p1 = ex2_approx(__fmaf_rn(sv[e + 1], p.scale_log2, nsub));
            if (masked) {
              p0 = kbase + e > qpos ? 0.f : p0;
              p1 = kbase + e + 1 > qpos ? 0.f : p1;
            }
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            a4[e & 3] = __fadd_rn(a4[e & 3], __low2float(h2));
            a4[(e + 1) & 3] = __fadd_rn(a4[(e + 1) & 3], __high2float(h2));
            pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          // P rows 32q' + h (q' = 0..3), keys 32q .. 32q+31: sub-tile q >> 1, 16-byte chunks
          // (q & 1) * 4 + c of the 128-byte row, SW128-swizzled (chunk ^ (row & 7) = chunk ^ h)
          if (lane < 8) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              uint8_t* prow = smem + OFF_P + s * TILE + (q >> 1) * SUB + (32 * qq + h) * 128;
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const int chunk = ((q & 1) * 4 + c) ^ h;
                *reinterpret_cast<uint4*>(prow + chunk * 16) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
              }
            }
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full + s);
          if (lane < 8) red_sum[q * 8 + lane] = __fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]));
          __syncwarp();
          if (lane == 0) mbar_arrive(red_bar + 1);
          ok = ok && wait_warp(red_bar + 1, g & 1, p.err, 2);
          if (!ok) break;
          const float cs = __fadd_rn(__fadd_rn(red_sum[h], red_sum[8 + h]),
                                     __fadd_rn(red_sum[16 + h], red_sum[24 + h]));
          l = __fmaf_rn(l, alpha, cs);
          m = mnew;
          if (j >= 1) ok = ok && fold_pv(g - 1);
          alpha_prev = alpha;
        }
        ok = ok && fold_pv(g - 1);
        if (!ok) break;
        // lanes 0..G-1 (one per head) write this warp's 32 output columns
        if (live_row) {
          const long long w = (long long)it.b * p.nq + (long long)it.hk * G + h;
          if (it.nsplit == 1) {
            const float inv = l > 0.f ? __frcp_rn(l) : 0.f;
            __nv_bfloat16* out = p.o + w * D + q * 32;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint4 v;
              v.x = pack_bf16x2(__fmul_rn(ot[c * 8 + 0], inv), __fmul_rn(ot[c * 8 + 1], inv));
              v.y = pack_bf16x2(__fmul_rn(ot[c * 8 + 2], inv), __fmul_rn(ot[c * 8 + 3], inv));
              v.z = pack_bf16x2(__fmul_rn(ot[c * 8 + 4], inv), __fmul_rn(ot[c * 8 + 5], inv));
              v.w = pack_bf16x2(__fmul_rn(ot[c * 8 + 6], inv), __fmul_rn(ot[c * 8 + 7], inv));
              reinterpret_cast<uint4*>(out)[c] = v;
            }
          } else {
            const long long base = w * p.nsplit_max + it.split;
            float4* wo = reinterpret_cast<float4*>(p.ws_o + base * D + q * 32);
#pragma unroll
            for (int c = 0; c < 8; ++c)
              wo[c] = make_float4(ot[c * 4], ot[c * 4 + 1], ot[c * 4 + 2], ot[c * 4 + 3]);
            if (q == 0) {
              p.ws_ml[base * 2] = m;
              p.ws_ml[base * 2 + 1] = l;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
      }
    }
  } else {
    // ================= softmax / output =================
    // 8 warps: thread (quad, half) owns row quad*32+lane and columns [64*half, 64*half+64) of
    // S, P and O; the two halves of a row exchange partial maxima / sums through shared memory.
    const int sw = warp - 2;
    const int quad = warp & 3, half = sw >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int col0 = half * 64;
    // decode tiles hold G valid rows: warps of lane quadrants past them only keep the
    // barrier protocol (their rows are computed by nobody and discarded)
    const bool idle = MODE == 1 && quad * 32 >= G;
    float* red_max = reinterpret_cast<float*>(smem + OFF_RED);  // [2][128]
    float* red_sum = red_max + 256;                               // [2][128]
    auto softmax_sync = [] { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < n_items; t += gridDim.x) {
      const Item it = get_item<MODE>(p, t);
      if (it.nblk == 0) continue;
      const int qpos = MODE == 0 ? it.m0 + row : it.qpos;
      float O[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) O[i] = 0.f;
      float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
      float Mt = -INFINITY, Lt = 0.f;  // merged-chunk totals (mode 0, more than one chunk)

      // O <- fma(O, alpha_prev, O_i) for running block i (its PV product is in the O_j buffer)
      auto fold_pv = [&](int i) -> bool {
        if (!wait_warp(o_full, i & 1, p.err, 2)) return false;
        tc_fence_after();
        if (!idle) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_off + 256 + col0 + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              O[c * 32 + e] = __fmaf_rn(O[c * 32 + e], alpha_prev, __uint_as_float(r[e]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_empty);
        return true;
      };
      // merge the finished chunk (m, l, O) into the running total in TMEM columns 384..511
      auto merge_chunk = [&](bool first) {
        float fa, fb;
        merge_stats(Mt, Lt, m, l, fa, fb);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          const uint32_t ta = tmem_base + lane_off + 384 + col0 + c * 32;
          if (!first) {
            tmem_ld_32x32b_x32(ta, r);
            tmem_ld_wait();
          }
#pragma unroll
          for (int e = 0; e < 32; ++e)
            r[e] = __float_as_uint(first ? O[c * 32 + e]
                                         : merge_val(__uint_as_float(r[e]), O[c * 32 + e], fa, fb));
          tmem_st_32x32b_x32(ta, r);
        }
        tmem_st_wait();
      };

      // Block j: S_j -> P_j (into the S buffer) while PV_{j-1} runs; O_{j-1} is folded in at
      // the end of the block (at the start at chunk boundaries, where the chunk must be
      // complete).
      // A failed wait (ok = false) skips the TMEM work but keeps executing the named barriers,
      // so the other softmax warps never block on a barrier this warp stopped reaching.
      for (int j = 0; j < it.nblk; ++j, ++g) {
        const int s = g & 1;
        ok = ok && wait_warp(s_full + s, (g >> 1) & 1, p.err, 2);
        tc_fence_after();
        const bool boundary = MODE == 0 && j > 0 && j % CHUNK == 0;
        if (boundary) {
          ok = ok && fold_pv(g - 1);
          if (ok) merge_chunk(j == CHUNK);
#pragma unroll
          for (int i = 0; i < 64; ++i) O[i] = 0.f;
          m = -INFINITY;
          l = 0.f;
          alpha_prev = 1.f;
        }
        const int kbase = (it.jbeg + j) * BN + col0;
        const uint32_t ts = tmem_base + lane_off + s * 128 + col0;
        // Only the last block of a row's key range can hold keys past the query position (for
        // prefill tiles the diagonal block, for decode the block holding the context end).
        const bool masked = j == it.nblk - 1;
        // pass 1: row max of the raw scores (scaling is monotonic, so max(S) * scale equals
        // the max of the scaled scores bit for bit; max is exact in any order)
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (!idle && ok) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(ts + c * 32, r);
            tmem_ld_wait();
            if (masked) {
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const float sv = kbase + c * 32 + e > qpos ? -INFINITY : __uint_as_float(r[e]);
                mx4[e & 3] = fmaxf(mx4[e & 3], sv);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(r[e]));
            }
          }
        }
        red_max[half * 128 + row] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        softmax_sync();
        const float raw = fmaxf(red_max[row], red_max[128 + row]);
        const float mnew = fmaxf(m, raw == -INFINITY ? -INFINITY : __fmul_rn(raw, p.scale_log2));
        const float sub = mnew == -INFINITY ? 0.f : mnew;
        const float alpha = exp2f(__fsub_rn(m == -INFINITY ? sub : m, sub));
        const float nsub = -sub;
        // pass 2: P = bf16(2^fma(S, scale, -sub)) and its row sum. This thread's 64 keys are
        // packed into columns half*64 .. half*64+31 of the S buffer (inside the columns it has
        // itself just read), one 32-key group at a time.
        float cs[2] = {0.f, 0.f};
        if (!idle && ok) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(ts + c * 32, r);
            tmem_ld_wait();
            float a4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float p0 = ex2_approx(__fmaf_rn(__uint_as_float(r[e]), p.scale_log2, nsub));
              float p1 = ex2_approx(__fmaf_rn(__uint_as_float(r[e + 1]), p.scale_log2, nsub));
              if (masked) {
                const int kp = kbase + c * 32 + e;
                p0 = kp > qpos ? 0.f : p0;
                p1 = kp + 1 > qpos ? 0.f : p1;
              }
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
              a4[e & 3] = __fadd_rn(a4[e & 3], __low2float(h2));
              a4[(e + 1) & 3] = __fadd_rn(a4[(e + 1) & 3], __high2float(h2));
              pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            cs[c] = __fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]));
            tmem_st_32x32b_x16(tmem_base + lane_off + s * 128 + half * 64 + c * 16, pk);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(p_full + s);
        red_sum[half * 128 + row] = __fadd_rn(cs[0], cs[1]);
        softmax_sync();
        const float rs = __fadd_rn(red_sum[row], red_sum[128 + row]);
        l = __fmaf_rn(l, alpha, rs);
        m = mnew;
        if (j >= 1 && !boundary) ok = ok && fold_pv(g - 1);
        alpha_prev = alpha;
      }
      ok = ok && fold_pv(g - 1);
      if (!ok) continue;  // every softmax warp runs the same iterations (named barriers)
      if (MODE == 0) {
        if (it.nblk > CHUNK) {
          merge_chunk(false);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_off + 384 + col0 + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) O[c * 32 + e] = __uint_as_float(r[e]);
          }
          m = Mt;
          l = Lt;
        }
        if (qpos < it.len) {
          const float inv = l > 0.f ? __frcp_rn(l) : 0.f;
          __nv_bfloat16* out =
              p.o + (long long)(it.seq_start + qpos) * p.o_stride + (long long)it.h * D + col0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint4 v;
            v.x = pack_bf16x2(__fmul_rn(O[q * 8 + 0], inv), __fmul_rn(O[q * 8 + 1], inv));
            v.y = pack_bf16x2(__fmul_rn(O[q * 8 + 2], inv), __fmul_rn(O[q * 8 + 3], inv));
            v.z = pack_bf16x2(__fmul_rn(O[q * 8 + 4], inv), __fmul_rn(O[q * 8 + 5], inv));
            v.w = pack_bf16x2(__fmul_rn(O[q * 8 + 6], inv), __fmul_rn(O[q * 8 + 7], inv));
            reinterpret_cast<uint4*>(out)[q] = v;
          }
          if (p.lse && half == 0) {
            const float ln2 = 0.69314718055994530942f;
            p.lse[(long long)it.h * p.total_tokens + it.seq_start + qpos] =
                l > 0.f ? (m + log2f(l)) * ln2 : -INFINITY;
          }
        }
      } else if (row < G) {
        const long long w = (long long)it.b * p.nq + (long long)it.hk * G + row;
        if (it.nsplit == 1) {
          const float inv = l > 0.f ? __frcp_rn(l) : 0.f;
          __nv_bfloat16* out = p.o + w * D + col0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint4 v;
            v.x = pack_bf16x2(__fmul_rn(O[q * 8 + 0], inv), __fmul_rn(O[q * 8 + 1], inv));
            v.y = pack_bf16x2(__fmul_rn(O[q * 8 + 2], inv), __fmul_rn(O[q * 8 + 3], inv));
            v.z = pack_bf16x2(__fmul_rn(O[q * 8 + 4], inv), __fmul_rn(O[q * 8 + 5], inv));
            v.w = pack_bf16x2(__fmul_rn(O[q * 8 + 6], inv), __fmul_rn(O[q * 8 + 7], inv));
            reinterpret_cast<uint4*>(out)[q] = v;
          }
        } else {
          const long long base = w * p.nsplit_max + it.split;
          float4* wo = reinterpret_cast<float4*>(p.ws_o + base * D + col0);
#pragma unroll
          for (int q = 0; q < 16; ++q)
            wo[q] = make_float4(O[q * 4], O[q * 4 + 1], O[q * 4 + 2], O[q * 4 + 3]);
          if (half == 0) {
            p.ws_ml[base * 2] = m;
            p.ws_ml[base * 2 + 1] = l;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// =============================================================================================
// Backward (tcgen05). Two deterministic kernels (no atomics: every output tile has one owner
// that walks its inputs in a fixed order):
//   fa_bwd_dkdv_kernel: CTA = (128-key block j of one sequence, KV head). For every query head
//     of the group and every query tile i >= j:
//       S^T = K Q^T, dP^T = V dO^T (UMMA, keys x queries), P^T = 2^(S^T scale - lse2),
//       dS^T = P^T (dP^T - delta); dV += P^T dO, dK += dS^T Q (P^T / dS^T from TMEM).
//   fa_bwd_dq_kernel:   CTA = (128-query tile i, query head). For every key block j <= i:
//       S = Q K^T, dP = dO V^T, P, dS as above (rows = queries); dQ += dS K.
// dK and dQ are scaled by the softmax scale at the end. Q / dO / K tiles are loaded once in
// the K-major SW128 layout and read both as K-major operands (contraction over the head dim)
// and as MN-major operands (contraction over tokens: leading byte offset = one 16 KB d-half
// sub-tile).
// Roles: warp 0 TMA, warp 1 TMEM + MMA, warps 2-9 elementwise (two threads per TMEM lane, 64
// columns each), the same warps write the outputs.
// =============================================================================================
struct BwdParams {
  const int* cu_seqlens;
  const int* tile_seq;
  const int* tile_idx;
  const float* lse;    // [nq, T] natural log
  const float* delta;  // [nq, T]
  __nv_bfloat16 *dq, *dk, *dv;
  long long dq_stride, dk_stride, dv_stride;
  int nq, nkv, T;
  float scale_log2, scale;
  int* err;
};

constexpr int BW_THREADS = 320;
// dkdv smem: K | V (32 KB each) | 2 stages x (Q | dO) | 2 x (lse2 | delta) [128 f32 each] | bars
constexpr int BW_OFF_K = 0;
constexpr int BW_OFF_V = TILE;
constexpr int BW_OFF_STAGE = 2 * TILE;            // stage s: Q at +s*2*TILE, dO at +TILE
constexpr int BW_OFF_LD = 6 * TILE;               // [2][2][128] floats = 2 KB
constexpr int BW_OFF_BAR = BW_OFF_LD + 2048;
constexpr int BW_SMEM = BW_OFF_BAR + 256 + 1024;

MB_DEVICE void load_tile_kmajor(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  tma_load_2d(dst, map, bar, x, y);
  tma_load_2d(dst + SUB, map, bar, x + 64, y);
}

__global__ void __launch_bounds__(BW_THREADS, 1)
fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BW_OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* st_full = bars + 1;   // [2]
  uint64_t* st_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pd_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(st_full + s, 1);
      mbar_init(st_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(pd_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  const int G = p.nq / p.nkv;
  const int b = p.tile_seq[blockIdx.x], j = p.tile_idx[blockIdx.x];
  const int hk = blockIdx.y;
  const int seq_start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - seq_start;
  const int ntile = (len + BM - 1) / BM;
  const int nq_tiles = ntile - j;          // query tiles j .. ntile-1
  const int nsteps = G * nq_tiles;         // (head, query tile) pairs, head-major
  auto step_hi = [&](int n, int& h, int& i) { h = hk * G + n / nq_tiles; i = j + n % nq_tiles; };

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      load_tile_kmajor(smem + BW_OFF_K, &tmK, kv_full, hk * D, seq_start + j * BN);
      load_tile_kmajor(smem + BW_OFF_V, &tmV, kv_full, hk * D, seq_start + j * BN);
      for (int n = 0; n < nsteps; ++n) {
        const int s = n & 1;
        if (!mbar_wait(st_empty + s, ((n >> 1) & 1) ^ 1, p.err, 21)) break;
        int h, i;
        step_hi(n, h, i);
        uint8_t* st = smem + BW_OFF_STAGE + s * 2 * TILE;
        mbar_arrive_expect_tx(st_full + s, 2 * TILE);
        load_tile_kmajor(st, &tmQ, st_full + s, h * D, seq_start + i * BM);
        load_tile_kmajor(st + TILE, &tmDO, st_full + s, h * D, seq_start + i * BM);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_mn = make_idesc_bf16(128, 128, false, true);
    const uint32_t sk = smem_u32(smem + BW_OFF_K), sv = smem_u32(smem + BW_OFF_V);
    bool ok = mbar_wait(kv_full, 0, p.err, 22);
    for (int n = 0; ok && n < nsteps; ++n) {
      const int s = n & 1;
      if (!mbar_wait(st_full + s, (n >> 1) & 1, p.err, 23)) break;
      if (n >= 1 && !mbar_wait(pd_done, (n - 1) & 1, p.err, 24)) break;  // P^T / dS^T consumed
      tc_fence_after();
      const uint32_t sq = smem_u32(smem + BW_OFF_STAGE + s * 2 * TILE), sdo = sq + TILE;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // S^T = K Q^T (contract over d)
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem_base, make_sdesc_sw128(sk + off, 16, 1024),
                   make_sdesc_sw128(sq + off, 16, 1024), idesc_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dP^T = V dO^T
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem_base + 128, make_sdesc_sw128(sv + off, 16, 1024),
                   make_sdesc_sw128(sdo + off, 16, 1024), idesc_s, kk > 0);
        }
        umma_commit(s_full);
      }
      __syncwarp();
      if (!mbar_wait(p_full, n & 1, p.err, 25)) break;
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dV += P^T dO (contract over queries)
          const uint32_t pa = (kk >> 2) * 64 + (kk & 3) * 8;
          umma_f16_ts(tmem_base + 256, tmem_base + pa,
                      make_sdesc_sw128(sdo + kk * 2048, SUB, 1024), idesc_mn,
                      (n > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T Q
          const uint32_t pa = (kk >> 2) * 64 + (kk & 3) * 8;
          umma_f16_ts(tmem_base + 384, tmem_base + 128 + pa,
                      make_sdesc_sw128(sq + kk * 2048, SUB, 1024), idesc_mn,
                      (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pd_done);
        umma_commit(st_empty + s);
      }
      __syncwarp();
    }
  } else {
    const int sw = warp - 2, quad = warp & 3, half = sw >> 2;
    const int row = quad * 32 + lane;  // key within the block
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int kpos = j * BN + row;
    float* ld = reinterpret_cast<float*>(smem + BW_OFF_LD);  // [2 bufs][lse2 128 | delta 128]
    const int tid = threadIdx.x - 64;                          // 0..255
    auto sync256 = [] { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    const float LOG2E = 1.4426950408889634f;
    auto fetch = [&](int n) -> float {  // value this thread stores for step n
      int h, i;
      step_hi(n, h, i);
      const int q = i * BM + (tid & 127);
      if (q >= len) return 0.f;
      const long long at = (long long)h * p.T + seq_start + q;
      return tid < 128 ? p.lse[at] * LOG2E : p.delta[at];
    };
    bool ok = true;
    if (nsteps > 0) {
      ld[tid] = fetch(0);
      sync256();
    }
    for (int n = 0; n < nsteps; ++n) {
      const float nxt = n + 1 < nsteps ? fetch(n + 1) : 0.f;  // prefetch next step's vectors
      int h, i;
      step_hi(n, h, i);
      const float* lse2 = ld + (n & 1) * 256;
      const float* dlt = lse2 + 128;
      ok = ok && wait_warp(s_full, n & 1, p.err, 26);  // on failure keep the barrier protocol
      tc_fence_after();
      const bool edge = (i == j) || (i == ntile - 1);
#pragma unroll
      for (int c = 0; c < 2 && ok; ++c) {
        uint32_t rs[32], rp[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + half * 64 + c * 32, rs);
        tmem_ld_32x32b_x32(tmem_base + lane_off + 128 + half * 64 + c * 32, rp);
        tmem_ld_wait();
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pv[2], dv2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int ql = half * 64 + c * 32 + e + u;  // query within the tile
            float pp = ex2_approx(__fmaf_rn(__uint_as_float(rs[e + u]), p.scale_log2, -lse2[ql]));
            if (edge) {
              const int qpos = i * BM + ql;
              if (qpos < kpos || qpos >= len) pp = 0.f;
            }
            pv[u] = pp;
            dv2[u] = pp * (__uint_as_float(rp[e + u]) - dlt[ql]);
          }
          const __nv_bfloat162 hp = __floats2bfloat162_rn(pv[0], pv[1]);
          const __nv_bfloat162 hd = __floats2bfloat162_rn(dv2[0], dv2[1]);
          pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
          dk[e >> 1] = *reinterpret_cast<const uint32_t*>(&hd);
        }
        tmem_st_32x32b_x16(tmem_base + lane_off + half * 64 + c * 16, pk);
        tmem_st_32x32b_x16(tmem_base + lane_off + 128 + half * 64 + c * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(p_full);
      ld[((n + 1) & 1) * 256 + tid] = nxt;
      sync256();  // next step's vectors visible; this step's reads done
    }
    if (__all_sync(0xffffffff, ok) && nsteps > 0 && wait_warp(pd_done, (nsteps - 1) & 1, p.err, 27)) {
      tc_fence_after();
      // tcgen05.ld is warp-collective: every lane loads, only rows inside the sequence store
      const bool kok = kpos < len;
      const long long r = seq_start + (kok ? kpos : 0);
      __nv_bfloat16* dv_out = p.dv + r * p.dv_stride + (long long)hk * D + half * 64;
      __nv_bfloat16* dk_out = p.dk + r * p.dk_stride + (long long)hk * D + half * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t a[32], bb[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + 256 + half * 64 + c * 32, a);
        tmem_ld_32x32b_x32(tmem_base + lane_off + 384 + half * 64 + c * 32, bb);
        tmem_ld_wait();
        if (!kok) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 ov, okv;
          ov.x = pack_bf16x2(__uint_as_float(a[q * 8 + 0]), __uint_as_float(a[q * 8 + 1]));
          ov.y = pack_bf16x2(__uint_as_float(a[q * 8 + 2]), __uint_as_float(a[q * 8 + 3]));
          ov.z = pack_bf16x2(__uint_as_float(a[q * 8 + 4]), __uint_as_float(a[q * 8 + 5]));
          ov.w = pack_bf16x2(__uint_as_float(a[q * 8 + 6]), __uint_as_float(a[q * 8 + 7]));
          okv.x = pack_bf16x2(__uint_as_float(bb[q * 8 + 0]) * p.scale, __uint_as_float(bb[q * 8 + 1]) * p.scale);
          okv.y = pack_bf16x2(__uint_as_float(bb[q * 8 + 2]) * p.scale, __uint_as_float(bb[q * 8 + 3]) * p.scale);
          okv.z = pack_bf16x2(__uint_as_float(bb[q * 8 + 4]) * p.scale, __uint_as_float(bb[q * 8 + 5]) * p.scale);
          okv.w = pack_bf16x2(__uint_as_float(bb[q * 8 + 6]) * p.scale, __uint_as_float(bb[q * 8 + 7]) * p.scale);
          reinterpret_cast<uint4*>(dv_out + c * 32)[q] = ov;
          reinterpret_cast<uint4*>(dk_out + c * 32)[q] = okv;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// dq smem: Q | dO (32 KB each) | 2 stages x (K | V) | bars
constexpr int BQ_OFF_Q = 0;
constexpr int BQ_OFF_DO = TILE;
constexpr int BQ_OFF_STAGE = 2 * TILE;
constexpr int BQ_OFF_BAR = 6 * TILE;
constexpr int BQ_SMEM = BQ_OFF_BAR + 256 + 1024;

__global__ void __launch_bounds__(BW_THREADS, 1)
fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                 const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BQ_OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* st_full = bars + 1;   // [2]
  uint64_t* st_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pd_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(st_full + s, 1);
      mbar_init(st_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(pd_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  const int G = p.nq / p.nkv;
  const int b = p.tile_seq[blockIdx.x], i = p.tile_idx[blockIdx.x];
  const int h = blockIdx.y, hk = h / G;
  const int seq_start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - seq_start;
  const int nsteps = i + 1;  // key blocks 0..i

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, 2 * TILE);
      load_tile_kmajor(smem + BQ_OFF_Q, &tmQ, q_full, h * D, seq_start + i * BM);
      load_tile_kmajor(smem + BQ_OFF_DO, &tmDO, q_full, h * D, seq_start + i * BM);
      for (int n = 0; n < nsteps; ++n) {
        const int s = n & 1;
        if (!mbar_wait(st_empty + s, ((n >> 1) & 1) ^ 1, p.err, 28)) break;
        uint8_t* st = smem + BQ_OFF_STAGE + s * 2 * TILE;
        mbar_arrive_expect_tx(st_full + s, 2 * TILE);
        load_tile_kmajor(st, &tmK, st_full + s, hk * D, seq_start + n * BN);
        load_tile_kmajor(st + TILE, &tmV, st_full + s, hk * D, seq_start + n * BN);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_mn = make_idesc_bf16(128, 128, false, true);
    const uint32_t sq = smem_u32(smem + BQ_OFF_Q), sdo = smem_u32(smem + BQ_OFF_DO);
    bool ok = mbar_wait(q_full, 0, p.err, 29);
    for (int n = 0; ok && n < nsteps; ++n) {
      const int s = n & 1;
      if (!mbar_wait(st_full + s, (n >> 1) & 1, p.err, 30)) break;
      if (n >= 1 && !mbar_wait(pd_done, (n - 1) & 1, p.err, 31)) break;
      tc_fence_after();
      const uint32_t sk = smem_u32(smem + BQ_OFF_STAGE + s * 2 * TILE), sv = sk + TILE;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // S = Q K^T
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem_base, make_sdesc_sw128(sq + off, 16, 1024),
                   make_sdesc_sw128(sk + off, 16, 1024), idesc_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dP = dO V^T
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem_base + 128, make_sdesc_sw128(sdo + off, 16, 1024),
                   make_sdesc_sw128(sv + off, 16, 1024), idesc_s, kk > 0);
        }
        umma_commit(s_full);
      }
      __syncwarp();
      if (!mbar_wait(p_full, n & 1, p.err, 32)) break;
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dQ += dS K (contract over keys)
          const uint32_t pa = (kk >> 2) * 64 + (kk & 3) * 8;
          umma_f16_ts(tmem_base + 256, tmem_base + 128 + pa,
                      make_sdesc_sw128(sk + kk * 2048, SUB, 1024), idesc_mn,
                      (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pd_done);
        umma_commit(st_empty + s);
      }
      __syncwarp();
    }
  } else {
    const int sw = warp - 2, quad = warp & 3, half = sw >> 2;
    const int row = quad * 32 + lane;  // query within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qpos = i * BM + row;
    const bool qok = qpos < len;
    const long long at = (long long)h * p.T + seq_start + (qok ? qpos : 0);
    const float lse2 = qok ? p.lse[at] * 1.4426950408889634f : 0.f;
    const float dlt = qok ? p.delta[at] : 0.f;
    bool ok = true;
    for (int n = 0; n < nsteps; ++n) {
      if (!wait_warp(s_full, n & 1, p.err, 33)) { ok = false; break; }
      tc_fence_after();
      const bool diag = n == i;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t rs[32], rp[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + half * 64 + c * 32, rs);
        tmem_ld_32x32b_x32(tmem_base + lane_off + 128 + half * 64 + c * 32, rp);
        tmem_ld_wait();
        uint32_t dk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float d2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            float pp = ex2_approx(__fmaf_rn(__uint_as_float(rs[e + u]), p.scale_log2, -lse2));
            if (!qok || (diag && n * BN + half * 64 + c * 32 + e + u > qpos)) pp = 0.f;
            d2[u] = pp * (__uint_as_float(rp[e + u]) - dlt);
          }
          const __nv_bfloat162 hd = __floats2bfloat162_rn(d2[0], d2[1]);
          dk[e >> 1] = *reinterpret_cast<const uint32_t*>(&hd);
        }
        tmem_st_32x32b_x16(tmem_base + lane_off + 128 + half * 64 + c * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (__all_sync(0xffffffff, ok) && nsteps > 0 && wait_warp(pd_done, (nsteps - 1) & 1, p.err, 34)) {
      tc_fence_after();
      // tcgen05.ld is warp-collective: every lane loads, only rows inside the sequence store
      __nv_bfloat16* out = p.dq + (long long)(seq_start + (qok ? qpos : 0)) * p.dq_stride +
                           (long long)h * D + half * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t a[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + 256 + half * 64 + c * 32, a);
        tmem_ld_wait();
        if (!qok) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(a[q * 8 + 0]) * p.scale, __uint_as_float(a[q * 8 + 1]) * p.scale);
          v.y = pack_bf16x2(__uint_as_float(a[q * 8 + 2]) * p.scale, __uint_as_float(a[q * 8 + 3]) * p.scale);
          v.z = pack_bf16x2(__uint_as_float(a[q * 8 + 4]) * p.scale, __uint_as_float(a[q * 8 + 5]) * p.scale);
          v.w = pack_bf16x2(__uint_as_float(a[q * 8 + 6]) * p.scale, __uint_as_float(a[q * 8 + 7]) * p.scale);
          reinterpret_cast<uint4*>(out + c * 32)[q] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace fa
}  // namespace mb

using namespace mb;
using namespace mb::fa;

namespace {
int fwd_attr_set[3] = {0, 0, 0};  // one flag per MODE (0 prefill, 1 decode, 2 fast decode)
int g_sms = 0;
template <int MODE>
int launch_fa(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
              const Params& p, int n_items, cudaStream_t st) {
  if (!fwd_attr_set[MODE]) {
    if (cudaFuncSetAttribute(fa_fwd_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return -3;
    fwd_attr_set[MODE] = 1;
  }
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int grid = n_items < g_sms ? n_items : g_sms;
  mb_launch(fa_fwd_kernel<MODE>, dim3(grid), dim3(NTHREADS), SMEM_BYTES, st, tq, tk, tv, p,
            n_items);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, fa_fwd_kernel<MODE>);
    fprintf(stderr, "fa_fwd_kernel launch failed: %s (regs %d, max threads %d, smem %d)\n",
            cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, SMEM_BYTES);
    return -2;
  }
  return 0;
}
int current_ctx() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return -8;
  return 0;
}
}  // namespace

// Packed variable-length causal attention forward (head dim 128). q/k/v: token-major with row
// strides q_stride/k_stride/v_stride (elements, multiples of 8), heads contiguous inside a row.
// tile_seq/tile_idx list the (sequence, 128-row tile) work items; lse may be null.
extern "C" int mb_fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                         const int* cu_seqlens, const int* tile_seq, const int* tile_idx,
                         int ntiles, long long q_stride, long long k_stride, long long v_stride,
                         long long o_stride, int nq, int nkv, int T, float softmax_scale, int* err,
                         cudaStream_t st) {
  if (ntiles == 0 || T == 0) return 0;
  if (nq % nkv) return -1;
  if (int rc = current_ctx()) return rc;
  CUtensorMap tq, tk, tv;
  int rc = make_map(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nq * D, q_stride, 64, 128);
  if (rc) return rc;
  rc = make_map(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nkv * D, k_stride, 64, 64);
  if (rc) return rc;
  rc = make_map(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nkv * D, v_stride, 64, 64);
  if (rc) return rc;
  Params p{};
  p.cu_seqlens = cu_seqlens;
  p.tile_seq = tile_seq;
  p.tile_idx = tile_idx;
  p.lse = lse;
  p.o_stride = o_stride;
  p.total_tokens = T;
  p.o = (__nv_bfloat16*)o;
  p.nq = nq;
  p.nkv = nkv;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = err;
  return launch_fa<0>(tq, tk, tv, p, ntiles * nq, st);
}

// Paged decode: one query token per sequence. q: [B, nq, 128]; caches [num_slots, nkv, 128]
// with slot = page * 64 + offset. Sequences spanning several 1024-key chunks write per-chunk
// partials to ws_o/ws_ml, merged by the decode combine kernel (mb_attn_decode_combine).
extern "C" int mb_fa_decode(const void* q, const void* kc, const void* vc, void* o,
                            const int* page_table, const int* ctx_lens, int B, int max_pages,
                            long long num_slots, int nq, int nkv, float softmax_scale,
                            float* ws_o, float* ws_ml, int* err, cudaStream_t st) {
  if (B == 0) return 0;
  if (nq % nkv || nq / nkv > BM) return -1;
  const int nsplit_max = (max_pages + 2 * CHUNK - 1) / (2 * CHUNK);
  if (nsplit_max > 1 && (!ws_o || !ws_ml)) return -3;
  if (int rc = current_ctx()) return rc;
  CUtensorMap tq, tk, tv;
  // G <= 8 query heads per KV head: the one-warp softmax path (mode 2); larger groups: mode 1
  const bool fast = nq / nkv <= 8;
  const int q_rows = fast ? 8 : ((nq / nkv + 7) / 8) * 8;
  int rc = make_map(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)B * nq, D, D, 64, q_rows);
  if (rc) return rc;
  rc = make_map(&tk, kc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, (uint64_t)nkv * D,
                (uint64_t)nkv * D, 64, 64);
  if (rc) return rc;
  rc = make_map(&tv, vc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, (uint64_t)nkv * D,
                (uint64_t)nkv * D, 64, 64);
  if (rc) return rc;
  Params p{};
  p.page_table = page_table;
  p.ctx_lens = ctx_lens;
  p.max_pages = max_pages;
  p.ws_o = ws_o;
  p.ws_ml = ws_ml;
  p.nsplit_max = nsplit_max;
  p.q_rows = q_rows;
  p.o = (__nv_bfloat16*)o;
  p.nq = nq;
  p.nkv = nkv;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = err;
  return fast ? launch_fa<2>(tq, tk, tv, p, B * nkv * nsplit_max, st)
              : launch_fa<1>(tq, tk, tv, p, B * nkv * nsplit_max, st);
}

// Backward of mb_fa_fwd: dq [T, nq, 128], dk / dv [T, nkv, 128] (row strides given; every row
// is written). delta = rowsum(dO * O) [nq, T] and lse [nq, T] come from the caller.
extern "C" int mb_fa_bwd(const void* q, const void* k, const void* v, const void* dout,
                         const float* lse, const float* delta, void* dq, void* dk, void* dv,
                         const int* cu_seqlens, const int* tile_seq, const int* tile_idx,
                         int ntiles, long long q_stride, long long k_stride, long long v_stride,
                         long long do_stride, long long dq_stride, long long dk_stride,
                         long long dv_stride, int nq, int nkv, int T, float softmax_scale,
                         int* err, cudaStream_t st) {
  if (ntiles == 0 || T == 0) return 0;
  if (nq % nkv) return -1;
  if (int rc = current_ctx()) return rc;
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_map(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nq * D, q_stride, 64, 128);
  if (rc) return rc;
  rc = make_map(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nkv * D, k_stride, 64, 128);
  if (rc) return rc;
  rc = make_map(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nkv * D, v_stride, 64, 128);
  if (rc) return rc;
  rc = make_map(&tdo, dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (uint64_t)nq * D, do_stride, 64, 128);
  if (rc) return rc;
  BwdParams p{cu_seqlens, tile_seq, tile_idx, lse, delta, (__nv_bfloat16*)dq, (__nv_bfloat16*)dk,
              (__nv_bfloat16*)dv, dq_stride, dk_stride, dv_stride, nq, nkv, T,
              softmax_scale * 1.4426950408889634f, softmax_scale, err};
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(fa_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(fa_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BQ_SMEM) != cudaSuccess)
      return -3;
    attr = true;
  }
  mb_launch(fa_bwd_dkdv_kernel, dim3(ntiles, nkv), dim3(BW_THREADS), BW_SMEM, st, tq, tk, tv, tdo, p);
  mb_launch(fa_bwd_dq_kernel, dim3(ntiles, nq), dim3(BW_THREADS), BQ_SMEM, st, tq, tk, tv, tdo, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "fa_bwd launch failed: %s\n", cudaGetErrorString(e));
    return -2;
  }
  return 0;
}
