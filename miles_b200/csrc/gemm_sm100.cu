// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M,N] (=|+=) alpha * A[M,K] * B[N,K]^T        bf16 in, fp32 accumulate in TMEM
//
// A and B are each either K-major (row-major [rows, K]) or MN-major (row-major [K, rows]); the
// UMMA shared-memory descriptors express both, so forward (K,K), data-grad (K,MN) and weight-grad
// (MN,MN) products all run without a transpose pass.
//
// Modes
//   0  dense
//   1  grouped-M  (MoE expert forward / data-grad): A rows are tokens sorted by expert, each
//      expert's segment padded to a multiple of 128 rows (`group_offsets`, device array, E+1);
//      B is E stacked matrices; each 128-row tile belongs to exactly one expert.
//   2  grouped-K  (MoE expert weight-grad): C is E stacked [M,N] matrices and the contraction of
//      group g runs over rows [group_offsets[g], group_offsets[g+1]) of the MN-major operands.
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (TMEM -> registers -> global). The accumulator is double-buffered in
// TMEM so the epilogue of tile i overlaps the MMAs of tile i+1. Every output element is the
// same K-ordered sequence of 16-wide MMAs regardless of M, N-tile width or grid size (no
// split-K), which keeps results batch-invariant: a token's projection is bitwise identical
// whether it is computed in a 16k-token training micro-batch or a 1-token decode step.
//
// Reference roles replaced: TE/cuBLASLt dense GEMMs (megatron_utils/model_provider.py:146-183)
// and the MoE grouped GEMMs (--moe-grouped-gemm; fsdp_utils/kernels/fused_experts.py:15-170,
// fused_moe_triton_backward_kernels.py:10-271).
#include "common.cuh"
#include <stdio.h>
#include <stdlib.h>
#include <mutex>
#include <unordered_map>

namespace mb {

struct GemmParams {
  int M, N, K;               // logical sizes (mode 1: M = padded row upper bound)
  void* C;
  long long ldc;             // row stride of C in elements
  long long c_group_stride;  // mode 2: elements between consecutive groups' C
  const int* group_offsets;  // modes 1,2
  int num_groups;
  int b_rows_per_group;      // mode 1: rows of B's 2-D view per group
  int epi;                   // 0 store bf16, 1 store f32, 2 accumulate into bf16, 3 accumulate into f32,
                             // 4 SwiGLU (below), 5 store bf16 to peers (below)
  float alpha;
  int* err;                  // device error word (may be null)
  int a_stage_bytes;         // bytes TMA writes for one A stage (K-major A may load < BM rows)
  // Fused SwiGLU epilogue (epi 4): B holds [gate; up] rows per group (F each, N = 2F). An N tile
  // of width BN takes BN/2 gate rows and the matching BN/2 up rows, so the epilogue sees both
  // halves of its output columns and writes silu(gate) * up (width F, row stride ldc); when C2
  // is set it also writes the [gate | up] product (width 2F, row stride ldc2) for the backward.
  int swiglu_f;
  void* C2;
  long long ldc2;
  // mode 1, optional: rows per group before padding; padding rows of the output are then not
  // written (callers that run no backward over the padded buffer)
  const int* group_counts;
  // epi 5: store bf16 tiles into `npeers` destinations (peer ranks' staging areas of a fused
  // GEMM + all-reduce). Destination d is peer_c[d] + (par_word[0] & 1) * par_stride, row stride
  // ldc; the parity word is the collective's epoch counter, read after the PDL wait.
  void* peer_c[8];
  int npeers;
  int scatter_rows;  // > 0: row r goes only to peer r / scatter_rows, at row r % scatter_rows
                     // (GEMM + reduce-scatter); 0: every row to every peer (GEMM + all-reduce)
  const int* par_word;
  long long par_stride;
};

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
  // narrow N tiles serve small-M (decode) GEMMs, which are bound by the B stream: keep more
  // stages in flight for them
  static constexpr int STAGE_CAP = BN <= 32 ? 12 : 8;
  static constexpr int STAGES = STAGES_RAW > STAGE_CAP ? STAGE_CAP : STAGES_RAW;
  // two accumulators of BN columns; tcgen05.alloc takes a power of two >= 32
  static constexpr int TMEM_COLS = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128
                                 : (2 * BN) <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct TileInfo {
  int m0, n0, g, kbeg, kend;
  long long c_off;
  int brow0;
  bool valid;
};

template <int BN, int MODE>
MB_DEVICE int num_tiles(const GemmParams& p) {
  const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
  return MODE == 2 ? p.num_groups * mt * nt : mt * nt;
}

template <int BN, int MODE>
MB_DEVICE TileInfo get_tile(const GemmParams& p, int t) {
  TileInfo ti;
  const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
  ti.valid = true;
  ti.c_off = 0;
  ti.brow0 = 0;
  ti.g = 0;
  if (MODE == 2) {
    const int per = mt * nt;
    ti.g = t / per;
    const int r = t - ti.g * per;
    ti.m0 = (r % mt) * BM;
    ti.n0 = (r / mt) * BN;
    ti.kbeg = __ldg(p.group_offsets + ti.g);
    ti.kend = __ldg(p.group_offsets + ti.g + 1);
    ti.c_off = (long long)ti.g * p.c_group_stride;
  } else {
    if (MODE == 1) {
      // N-fastest: the N-tiles of one expert segment run on neighbouring CTAs at the same time
      // and share the segment's A-tile through L2 (instead of re-reading it from DRAM once per
      // N-tile sweep over all experts).
      ti.m0 = (t / nt) * BM;
      ti.n0 = (t % nt) * BN;
    } else {
      ti.m0 = (t % mt) * BM;
      ti.n0 = (t / mt) * BN;
    }
    ti.kbeg = 0;
    ti.kend = p.K;
    if (MODE == 1) {
      const int total = __ldg(p.group_offsets + p.num_groups);
      if (ti.m0 >= total) {
        ti.valid = false;
      } else {
        // largest g with offsets[g] <= m0 (binary search over E+1 sorted offsets)
        int lo = 0, hi = p.num_groups - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (__ldg(p.group_offsets + mid) <= ti.m0) lo = mid; else hi = mid - 1;
        }
        ti.g = lo;
        ti.brow0 = lo * p.b_rows_per_group;
      }
    }
  }
  return ti;
}

// Bounded wait that also gives up promptly once another role has aborted.
MB_DEVICE bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && (*abort_flag || global_ns() - t0 > kWaitLimitNs)) {
      if (*abort_flag) return false;
      break;
    }
  }
  report_error(err, 1);
  *abort_flag = 1;
  return false;
}

// SwiGLU epilogue of one accumulator (see GemmParams::swiglu_f). The gate/up products are
// rounded to bf16 first and then combined with the same expression as the stand-alone SwiGLU
// kernel, so the fused result is bitwise equal to GEMM followed by SwiGLU.
template <int BN>
MB_DEVICE void swiglu_epilogue(const GemmParams& p, const TileInfo& ti, uint32_t tbase, int row,
                               bool row_ok, bool empty_k) {
  constexpr int HB = BN / 2;
  constexpr int CW = HB < 32 ? 16 : 32;
#pragma unroll 1
  for (int c = 0; c < HB / CW; ++c) {
    uint32_t rg[32], ru[32];
    __syncwarp();
    if (!empty_k) {
      if constexpr (CW == 32) {
        tmem_ld_32x32b_x32(tbase + c * CW, rg);
        tmem_ld_32x32b_x32(tbase + HB + c * CW, ru);
      } else {
        tmem_ld_32x32b_x16(tbase + c * CW, rg);
        tmem_ld_32x32b_x16(tbase + HB + c * CW, ru);
      }
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < CW; ++i) rg[i] = ru[i] = 0u;
    }
    if (!row_ok) continue;
    const int col0 = (ti.n0 >> 1) + c * CW;  // column inside [0, F)
    if (col0 >= p.swiglu_f) continue;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.C) + ti.c_off + (long long)row * p.ldc + col0;
    __nv_bfloat16* gu = p.C2 ? reinterpret_cast<__nv_bfloat16*>(p.C2) + (long long)row * p.ldc2 + col0
                             : nullptr;
#pragma unroll
    for (int q = 0; q < CW / 8; ++q) {
      uint4 og, ou, oa;
      __nv_bfloat16* gb = reinterpret_cast<__nv_bfloat16*>(&og);
      __nv_bfloat16* ub = reinterpret_cast<__nv_bfloat16*>(&ou);
      __nv_bfloat16* ab = reinterpret_cast<__nv_bfloat16*>(&oa);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        gb[i] = __float2bfloat16(__uint_as_float(rg[q * 8 + i]) * p.alpha);
        ub[i] = __float2bfloat16(__uint_as_float(ru[q * 8 + i]) * p.alpha);
        const float g = __bfloat162float(gb[i]);
        const float sg = g / (1.f + expf(-g));
        ab[i] = __float2bfloat16(__bfloat162float(__float2bfloat16(sg)) * __bfloat162float(ub[i]));
      }
      reinterpret_cast<uint4*>(out)[q] = oa;
      if (gu) {
        reinterpret_cast<uint4*>(gu)[q] = og;
        reinterpret_cast<uint4*>(gu + p.swiglu_f)[q] = ou;
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int MODE>
__global__ void __launch_bounds__(192, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar + a, 1);
      mbar_init(tempty_bar + a, 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // inputs are read only after the previous kernel completes

  const int ntiles = num_tiles<BN, MODE>(p);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const TileInfo ti = get_tile<BN, MODE>(p, t);
        if (!ti.valid) continue;
        for (int k = ti.kbeg; k < ti.kend; k += BK) {
          if (!wait_or_abort(empty_bar + s, phase ^ 1, abort_flag, p.err)) goto producer_done;
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(full_bar + s, p.a_stage_bytes + Cfg::B_BYTES);
          if (A_MN) {
            tma_load_2d(sa, &tmA, full_bar + s, ti.m0, k);
            tma_load_2d(sa + 64 * 128, &tmA, full_bar + s, ti.m0 + 64, k);
          } else {
            tma_load_2d(sa, &tmA, full_bar + s, k, ti.m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 64 * 128, &tmB, full_bar + s, ti.n0 + 64 * j, ti.brow0 + k);
          } else if (p.swiglu_f) {
            const int nh = ti.n0 >> 1;
            tma_load_2d(sb, &tmB, full_bar + s, k, ti.brow0 + nh);
            tma_load_2d(sb + (BN / 2) * 128, &tmB, full_bar + s, k, ti.brow0 + p.swiglu_f + nh);
          } else {
            tma_load_2d(sb, &tmB, full_bar + s, k, ti.brow0 + ti.n0);
          }
          if (++s == STAGES) { s = 0; phase ^= 1; }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
    int s = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const TileInfo ti = get_tile<BN, MODE>(p, t);
      if (!ti.valid) continue;
      if (!wait_or_abort(tempty_bar + acc, acc_phase ^ 1, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      bool first = true;
      for (int k = ti.kbeg; k < ti.kend; k += BK) {
        if (!wait_or_abort(full_bar + s, phase, abort_flag, p.err)) goto mma_done;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sa = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sdesc_sw128(sa + kk * 2048, 64 * 128, 1024)
                                     : make_sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(sb + kk * 2048, 64 * 128, 1024)
                                     : make_sdesc_sw128(sb + kk * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (first && kk == 0) ? 0u : 1u);
          }
          umma_commit(empty_bar + s);  // frees the smem stage once these MMAs retire
        }
        __syncwarp();
        first = false;
        if (++s == STAGES) { s = 0; phase ^= 1; }
      }
      if (elect_one()) umma_commit(tfull_bar + acc);
      __syncwarp();
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  mma_done:;
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const long long par_off =
        p.epi == 5 ? (long long)(*reinterpret_cast<const volatile int*>(p.par_word) & 1) * p.par_stride : 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const TileInfo ti = get_tile<BN, MODE>(p, t);
      if (!ti.valid) continue;
      // warp-uniform: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffff, wait_or_abort(tfull_bar + acc, acc_phase, abort_flag, p.err))) break;
      tc_fence_after();
      const bool empty_k = ti.kend <= ti.kbeg;
      const int row = ti.m0 + quad * 32 + lane;
      bool row_ok = row < p.M;
      if (MODE == 1 && p.group_counts)
        row_ok = row_ok && row - __ldg(p.group_offsets + ti.g) < __ldg(p.group_counts + ti.g);
      const long long rbase = ti.c_off + (long long)row * p.ldc;
      if constexpr (BN >= 32) {
        if (p.epi == 4) {
          swiglu_epilogue<BN>(p, ti, tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN, row,
                              row_ok, empty_k);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar + acc);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
          continue;
        }
      }
      constexpr int CW = BN < 32 ? 16 : 32;  // columns per TMEM load
#pragma unroll 1
      for (int c = 0; c < BN / CW; ++c) {
        uint32_t r[32];
        __syncwarp();
        if (!empty_k) {
          const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * CW;
          if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr, r);
          else tmem_ld_32x32b_x16(taddr, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < CW; ++i) r[i] = 0u;
        }
        if (!row_ok) continue;
        if (empty_k && (p.epi & 2)) continue;  // accumulate nothing
        const int col0 = ti.n0 + c * CW;
        if (col0 >= p.N) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < CW; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
        const bool full_cols = col0 + CW <= p.N;
        if (p.epi == 0 || p.epi == 2 || p.epi == 5) {
         int d0 = 0, d1 = 1;
         long long rb = rbase;
         if (p.epi == 5) {
           if (p.scatter_rows > 0) {
             d0 = row / p.scatter_rows;
             d1 = d0 + 1;
             rb = (long long)(row - d0 * p.scatter_rows) * p.ldc;
           } else {
             d1 = p.npeers;
           }
         }
         for (int d = d0; d < d1; ++d) {
          __nv_bfloat16* out = (p.epi == 5 ? reinterpret_cast<__nv_bfloat16*>(p.peer_c[d]) + par_off
                                           : reinterpret_cast<__nv_bfloat16*>(p.C)) + rb + col0;
          if (full_cols) {
            uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
            for (int q = 0; q < CW / 8; ++q) {
              float w[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) w[i] = v[q * 8 + i];
              if (p.epi == 2) {
                uint4 old = o4[q];
                const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&old);
#pragma unroll
                for (int i = 0; i < 8; ++i) w[i] += __bfloat162float(ob[i]);
              }
              uint4 pk;
              pk.x = pack_bf16x2(w[0], w[1]);
              pk.y = pack_bf16x2(w[2], w[3]);
              pk.z = pack_bf16x2(w[4], w[5]);
              pk.w = pack_bf16x2(w[6], w[7]);
              o4[q] = pk;
            }
          } else {
            for (int i = 0; i < CW && col0 + i < p.N; ++i) {
              float w = v[i];
              if (p.epi == 2) w += __bfloat162float(out[i]);
              out[i] = __float2bfloat16(w);
            }
          }
         }
        } else {
          float* out = reinterpret_cast<float*>(p.C) + rbase + col0;
          if (full_cols) {
            float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
            for (int q = 0; q < CW / 4; ++q) {
              float4 w = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
              if (p.epi == 3) {
                const float4 o = o4[q];
                w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
              }
              o4[q] = w;
            }
          } else {
            for (int i = 0; i < CW && col0 + i < p.N; ++i) {
              out[i] = (p.epi == 3 ? out[i] : 0.f) + v[i];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar + acc);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// =============================================================================================
// Host side
// =============================================================================================
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major [rows, cols] map with a {box_cols, box_rows} box and 128-byte swizzle.
int make_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize,
                    uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols,
                    uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

static int g_num_sms = 0;

template <int BN, bool A_MN, bool B_MN, int MODE>
static int launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                      cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, MODE>;
  static bool attr_set = false;  // per instantiation; device-agnostic attribute
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::SMEM_BYTES) != cudaSuccess)
      return -3;
    attr_set = true;
  }
  if (g_num_sms == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
  const int tiles = MODE == 2 ? p.num_groups * mt * nt : mt * nt;
  if (tiles == 0) return 0;
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  mb_launch(kern, grid, 192, Cfg::SMEM_BYTES, st, ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int BN, int MODE>
static int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmParams& p, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_cfg<BN, false, false, MODE>(ta, tb, p, st);
  // narrow tiles (BN < 64) are built for K-major operands only (an MN-major B tile needs
  // 64-element rows for the 128-byte swizzle)
  if constexpr (BN < 64) return -5;
  else if (!a_mn && b_mn) return launch_cfg<BN, false, true, MODE>(ta, tb, p, st);
  else if (a_mn && b_mn) return launch_cfg<BN, true, true, MODE>(ta, tb, p, st);
  return -5;  // (MN, K) is not instantiated
}

template <int MODE>
static int dispatch_bn(int bn, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                       const GemmParams& p, cudaStream_t st) {
  switch (bn) {
    case 16: return dispatch_major<16, MODE>(a_mn, b_mn, ta, tb, p, st);
    case 32: return dispatch_major<32, MODE>(a_mn, b_mn, ta, tb, p, st);
    case 64: return dispatch_major<64, MODE>(a_mn, b_mn, ta, tb, p, st);
    case 128: return dispatch_major<128, MODE>(a_mn, b_mn, ta, tb, p, st);
    case 192: return dispatch_major<192, MODE>(a_mn, b_mn, ta, tb, p, st);
    case 256: return dispatch_major<256, MODE>(a_mn, b_mn, ta, tb, p, st);
  }
  return -6;
}

}  // namespace mb

// ---------------------------------------------------------------------------------------------
// C ABI used by the torch bindings.
//   a: pointer + stored shape [a_rows, a_cols] row-major (a_mn: a_rows = K, a_cols = M)
//   b: pointer + stored shape [b_rows, b_cols]          (b_mn: b_rows = K(*groups), b_cols = N)
// Returns 0 on success, negative on a configuration error.
// ---------------------------------------------------------------------------------------------
static int gemm_entry(const void* a, long long a_rows, long long a_cols, long long lda, bool a_mn,
                      const void* b, long long b_rows, long long b_cols, long long ldb, bool b_mn,
                      void* c, long long ldc, int M, int N, int K, int mode,
                      const int* group_offsets, int num_groups, int b_rows_per_group,
                      long long c_group_stride, int epi, float alpha, int bn, int swiglu_f,
                      void* c2, long long ldc2, const int* group_counts, int* err,
                      cudaStream_t stream, const long long* peer_ptrs = nullptr, int npeers = 0,
                      const int* par_word = nullptr, long long par_stride = 0,
                      int scatter_rows = 0) {
  using namespace mb;
  if (a_mn && !b_mn) return -5;
  // The driver's tensor-map encoder needs a current context in the calling thread; a thread
  // that has not made a runtime call yet (e.g. the autograd worker) has none. cudaSetDevice
  // makes the device's primary context current.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return -8;
  CUtensorMap ta, tb;
  // Dense GEMMs with M < 128 (decode) load only the first round_up(M, 8) rows of each A tile:
  // the remaining rows of the UMMA tile hold stale shared memory and produce output rows that
  // are never stored (each output row depends on its own A row only).
  const uint32_t a_box_rows = a_mn ? BK : (mode == 0 && M < BM ? (uint32_t)((M + 7) / 8 * 8) : BM);
  const uint32_t b_box_rows = b_mn ? BK : (uint32_t)(swiglu_f ? bn / 2 : bn);
  int rc = make_map(&ta, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a_rows, a_cols, lda, 64, a_box_rows);
  if (rc) return rc;
  rc = make_map(&tb, b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b_rows, b_cols, ldb, 64, b_box_rows);
  if (rc) return rc;
  GemmParams p;
  p.M = M; p.N = N; p.K = K;
  p.C = c; p.ldc = ldc; p.c_group_stride = c_group_stride;
  p.group_offsets = group_offsets; p.num_groups = num_groups;
  p.b_rows_per_group = b_rows_per_group;
  p.epi = epi; p.alpha = alpha; p.err = err;
  p.a_stage_bytes = a_mn ? BM * BK * 2 : (int)a_box_rows * BK * 2;
  p.swiglu_f = swiglu_f; p.C2 = c2; p.ldc2 = ldc2;
  p.group_counts = mode == 1 ? group_counts : nullptr;
  p.npeers = 0; p.par_word = par_word; p.par_stride = par_stride; p.scatter_rows = 0;
  for (int i = 0; i < 8; ++i) p.peer_c[i] = nullptr;
  if (epi == 5) {
    if (npeers < 1 || npeers > 8 || !par_word) return -1;
    p.npeers = npeers;
    for (int i = 0; i < npeers; ++i) p.peer_c[i] = reinterpret_cast<void*>(peer_ptrs[i]);
    if (scatter_rows < 0 || (scatter_rows > 0 && (long long)scatter_rows * npeers != M)) return -1;
    p.scatter_rows = scatter_rows;
    p.C = p.peer_c[0];
  }
  switch (mode) {
    case 0: return dispatch_bn<0>(bn, a_mn, b_mn, ta, tb, p, stream);
    case 1: return dispatch_bn<1>(bn, a_mn, b_mn, ta, tb, p, stream);
    case 2: return dispatch_bn<2>(bn, a_mn, b_mn, ta, tb, p, stream);
  }
  return -7;
}


extern "C" int mb_gemm_bf16(const void* a, long long a_rows, long long a_cols, long long lda,
                            bool a_mn, const void* b, long long b_rows, long long b_cols,
                            long long ldb, bool b_mn, void* c, long long ldc, int M, int N, int K,
                            int mode, const int* group_offsets, int num_groups,
                            int b_rows_per_group, long long c_group_stride, int epi, float alpha,
                            int bn, const int* group_counts, int* err, cudaStream_t stream) {
  if (epi == 4 || epi == 5) return -7;
  return gemm_entry(a, a_rows, a_cols, lda, a_mn, b, b_rows, b_cols, ldb, b_mn, c, ldc, M, N, K,
                    mode, group_offsets, num_groups, b_rows_per_group, c_group_stride, epi, alpha,
                    bn, 0, nullptr, 0, group_counts, err, stream);
}

// out[M, F] = silu(A B_gate^T) * (A B_up^T) with B = [gate; up] ([2F, K] per group, K-major),
// optionally also storing the [M, 2F] product into gu (row stride ldgu). Dense (mode 0) or
// grouped-M (mode 1). Requires F % (bn / 2) == 0 and bn >= 32.
extern "C" int mb_gemm_bf16_swiglu(const void* a, long long a_rows, long long lda, const void* b,
                                   long long b_rows, long long ldb, void* out, long long ldo,
                                   void* gu, long long ldgu, int M, int F, int K, int mode,
                                   const int* group_offsets, int num_groups, int bn,
                                   const int* group_counts, int* err, cudaStream_t stream) {
  if (bn < 32 || F % (bn / 2) || (mode != 0 && mode != 1)) return -1;
  return gemm_entry(a, a_rows, K, lda, false, b, b_rows, K, ldb, false, out, ldo, M, 2 * F, K,
                    mode, group_offsets, num_groups, 2 * F, 0, 4, 1.f, bn, F, gu, ldgu, group_counts,
                    err, stream);
}

// Fused GEMM + all-reduce / reduce-scatter, GEMM half: C = A B^T (dense, mode 0) with every
// bf16 output tile stored straight into peer staging areas over NVLink (epi 5): all `npeers`
// of them (all-reduce), or only the owner of the row (scatter_rows = M / npeers rows per rank,
// reduce-scatter). The reduce half is mb_symm_collective with src = null (symm.cu).
extern "C" int mb_gemm_bf16_peer(const void* a, long long a_rows, long long a_cols, long long lda,
                                 bool a_mn, const void* b, long long b_rows, long long b_cols,
                                 long long ldb, bool b_mn, int M, int N, int K,
                                 const long long* peer_ptrs, int npeers, long long ldc,
                                 const int* par_word, long long par_stride, int scatter_rows,
                                 int bn, int* err, cudaStream_t stream) {
  return gemm_entry(a, a_rows, a_cols, lda, a_mn, b, b_rows, b_cols, ldb, b_mn, nullptr, ldc, M, N,
                    K, 0, nullptr, 1, 0, 0, 5, 1.f, bn, 0, nullptr, 0, nullptr, err, stream,
                    peer_ptrs, npeers, par_word, par_stride, scatter_rows);
}
