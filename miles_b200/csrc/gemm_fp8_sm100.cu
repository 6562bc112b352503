// Block-scaled fp8 (e4m3) GEMM for sm_100a: the "unified blockwise fp8" recipe.
//
//   C[M,N] = sum_kb  sa[kb][m] * sb[n/128][kb] * (Aq[m, kb*128 : kb*128+128] . Bq[n, same])
//
// A holds activations quantised in 1 x 128 groups along K (one fp32 scale per row and 128-wide
// K block, stored K-block-major: sa[kb * lds + m]); B holds weights quantised in 128 x 128 blocks
// (fp32 scales [B_rows / 128, K / 128], row-major). Both operands are K-major e4m3.
//
// Because the scales change with every 128-wide K block, the tensor cores cannot accumulate
// the whole K range in one TMEM accumulator. Each K block is instead a fresh 128 x BN x 128
// product (4 kind::f8f6f4 UMMAs of K = 32) written into one of NBUF TMEM buffers; the
// epilogue warps read the buffer back (tcgen05.ld), release it to the MMA warp at once, and
// fold it into fp32 register accumulators with the block's combined scale. The MMA of K block
// j+1..j+NBUF-1 runs while the epilogue scales K block j. Rows and columns are independent and
// every output element is the same K-ordered chain, whatever M, the grid or the tile width, so
// the kernel is batch-invariant like the bf16 GEMM (a decode step and a training micro-batch
// produce bitwise the same row).
//
// Modes: 0 dense, 1 grouped-M (MoE experts: A rows sorted by expert, segments padded to 128
// rows, B = E stacked [N, K] matrices, sb stacked the same way). Epilogues: 0 store bf16,
// 4 SwiGLU (B = [gate; up] per group, output silu(gate) * up, optionally the [gate | up]
// product for the backward), both with the bf16 rounding points of the bf16 kernels.
//
// Roles: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, then NSETS sets of four
// epilogue warps (NSETS = 2: 320 threads). Warp w may only read TMEM lanes
// 32*(w%4)..+31, so every set covers the 128 rows once; the sets split the columns. Several
// warps per SM sub-partition hide the TMEM-load and scale-load latency of each K block.
//
// Reference roles replaced: the blockwise fp8 GEMMs of TransformerEngine (--fp8-recipe
// blockwise, examples/low_precision/README.md:17-18) and of DeepGEMM in the rollout engine
// (fp8 w8a8 block 128 x 128 serving after refit, megatron_to_hf/processors/quantizer_fp8.py).
#include "common.cuh"
#include <cuda_fp8.h>
#include <mutex>

namespace mb {
namespace f8 {

constexpr int BM = 128;
constexpr int BK = 128;  // 128 e4m3 = 128 bytes = one swizzle row = one scale block

struct Params {
  int M, N, K;
  void* C;
  long long ldc;
  const float* sa;  // [K/128][lds]
  long long lds;
  const float* sb;  // [B_rows/128][K/128]
  const int* group_offsets;
  const int* group_counts;
  int num_groups;
  int b_rows_per_group;
  int epi;       // 0 store bf16, 4 SwiGLU
  int swiglu_f;  // epi 4: F (gate rows per group; B rows per group = 2F)
  void* C2;      // epi 4, optional: [gate | up] product (width 2F, row stride ldc2)
  long long ldc2;
  int a_stage_bytes;
  int* err;
};

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_RAW = (196 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 12 ? 12 : STAGES_RAW;
  static constexpr int NBUF = BN >= 128 ? 4 : 8;  // TMEM buffers of BN columns (K blocks in flight)
  static constexpr int TMEM_COLS = NBUF * BN <= 32 ? 32 : NBUF * BN <= 64 ? 64 : NBUF * BN <= 128 ? 128
                                 : NBUF * BN <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int NSETS = 2;  // sets of four epilogue warps (measured: 2 beat 4)
  static constexpr int THREADS = 64 + 128 * NSETS;
  static constexpr int Q = BN / (2 * NSETS);  // columns per epilogue warp and range (two ranges)
};

struct Tile {
  int m0, n0, g, brow0;
  bool valid;
};

template <int BN, int MODE>
MB_DEVICE Tile get_tile(const Params& p, int t) {
  Tile ti;
  const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
  ti.valid = true;
  ti.g = 0;
  ti.brow0 = 0;
  if (MODE == 1) {
    // N-fastest: the N tiles of one expert segment run side by side and share its A tile in L2
    ti.m0 = (t / nt) * BM;
    ti.n0 = (t % nt) * BN;
    const int total = __ldg(p.group_offsets + p.num_groups);
    if (ti.m0 >= total) {
      ti.valid = false;
    } else {
      int lo = 0, hi = p.num_groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.group_offsets + mid) <= ti.m0) lo = mid; else hi = mid - 1;
      }
      ti.g = lo;
      ti.brow0 = lo * p.b_rows_per_group;
    }
  } else {
    ti.m0 = (t % mt) * BM;
    ti.n0 = (t / mt) * BN;
  }
  return ti;
}

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

template <int W>
MB_DEVICE void tld(uint32_t taddr, uint32_t* r) {
  if constexpr (W == 32) tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else if constexpr (W == 16) tmem_ld_32x32b_x16(taddr, r);
  else tmem_ld_32x32b_x8(taddr, r);
}

// bf16 store of W consecutive columns (vectorised when the whole run is in bounds and aligned)
template <int W>
MB_DEVICE void store_row(__nv_bfloat16* out, const float* v, int valid_cols) {
  if (valid_cols >= W && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < W / 8; ++q) {
      uint4 pk;
      pk.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      pk.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      pk.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      pk.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      reinterpret_cast<uint4*>(out)[q] = pk;
    }
  } else {
#pragma unroll
    for (int i = 0; i < W; ++i)
      if (i < valid_cols) out[i] = __float2bfloat16(v[i]);
  }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(Cfg<BN>::THREADS, 1)
gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const Params p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::NBUF;
  constexpr int Q = C::Q;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [NBUF]
  uint64_t* tempty_bar = tfull_bar + NBUF;   // [NBUF]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(tfull_bar + b, 1);
      mbar_init(tempty_bar + b, 4 * C::NSETS);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
  const int ntiles = mt * nt;
  const int nkb = p.K / BK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const Tile ti = get_tile<BN, MODE>(p, t);
        if (!ti.valid) continue;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!wait_or_abort(empty_bar + s, phase ^ 1, abort_flag, p.err)) goto producer_done;
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(full_bar + s, p.a_stage_bytes + C::B_BYTES);
          tma_load_2d(sa, &tmA, full_bar + s, kb * BK, ti.m0);
          if (p.epi == 4) {
            const int nh = ti.n0 >> 1;
            tma_load_2d(sb, &tmB, full_bar + s, kb * BK, ti.brow0 + nh);
            tma_load_2d(sb + (BN / 2) * BK, &tmB, full_bar + s, kb * BK, ti.brow0 + p.swiglu_f + nh);
          } else {
            tma_load_2d(sb, &tmB, full_bar + s, kb * BK, ti.brow0 + ti.n0);
          }
          if (++s == STAGES) { s = 0; phase ^= 1; }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_e4m3(BM, BN);
    int s = 0;
    uint32_t phase = 0;
    int buf = 0;
    uint32_t bphase = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const Tile ti = get_tile<BN, MODE>(p, t);
      if (!ti.valid) continue;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!wait_or_abort(tempty_bar + buf, bphase ^ 1, abort_flag, p.err)) goto mma_done;
        if (!wait_or_abort(full_bar + s, phase, abort_flag, p.err)) goto mma_done;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t d = tmem_base + buf * BN;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            umma_f8(d, make_sdesc_sw128(sa + kk * 32, 16, 1024),
                    make_sdesc_sw128(sb + kk * 32, 16, 1024), idesc, kk == 0 ? 0u : 1u);
          umma_commit(empty_bar + s);
          umma_commit(tfull_bar + buf);
        }
        __syncwarp();
        if (++s == STAGES) { s = 0; phase ^= 1; }
        if (++buf == NBUF) { buf = 0; bphase ^= 1; }
      }
    }
  mma_done:;
  } else {
    // ---------------- Epilogue / scale-and-accumulate (warps 2..9) ----------------
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // epilogue set
    const int c0 = half * Q;           // first range: tile columns [c0, c0 + Q)
    const int c1 = BN / 2 + half * Q;  // second range: [c1, c1 + Q)
    int buf = 0;
    uint32_t bphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const Tile ti = get_tile<BN, MODE>(p, t);
      if (!ti.valid) continue;
      const int row = ti.m0 + quad * 32 + lane;
      const bool row_in = row < p.M;
      bool row_ok = row_in;
      if (MODE == 1 && p.group_counts)
        row_ok = row_ok && row - __ldg(p.group_offsets + ti.g) < __ldg(p.group_counts + ti.g);
      // B row of each range's first column -> its 128 x 128 scale block row
      int brow_r0, brow_r1;
      if (p.epi == 4) {
        brow_r0 = ti.brow0 + (ti.n0 >> 1);
        brow_r1 = ti.brow0 + p.swiglu_f + (ti.n0 >> 1);
      } else {
        brow_r0 = ti.brow0 + ti.n0 + c0;
        brow_r1 = ti.brow0 + ti.n0 + c1;
      }
      const float* sb0 = p.sb + (long long)(brow_r0 / 128) * nkb;
      const float* sb1 = p.sb + (long long)(brow_r1 / 128) * nkb;
      float acc0[Q], acc1[Q];
#pragma unroll
      for (int i = 0; i < Q; ++i) acc0[i] = acc1[i] = 0.f;
      // The three scales of K block kb are loaded PF blocks ahead (a ring of registers indexed
      // by kb % PF after unrolling), so the global-load latency overlaps the previous blocks'
      // TMEM reads instead of stalling every block's FMAs.
      constexpr int PF = 4;
      float pa[PF], pb0[PF], pb1[PF];
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const bool in = u < nkb;
        pa[u] = in && row_in ? __ldg(p.sa + (long long)u * p.lds + row) : 0.f;
        pb0[u] = in ? __ldg(sb0 + u) : 0.f;
        pb1[u] = in ? __ldg(sb1 + u) : 0.f;
      }
      for (int kb0 = 0; kb0 < nkb && ok; kb0 += PF) {
#pragma unroll
        for (int u = 0; u < PF; ++u) {
          const int kb = kb0 + u;
          if (kb >= nkb) break;
          const float s0 = pa[u] * pb0[u];
          const float s1 = pa[u] * pb1[u];
          const int nk = kb + PF;  // refill this slot
          if (nk < nkb) {
            pa[u] = row_in ? __ldg(p.sa + (long long)nk * p.lds + row) : 0.f;
            pb0[u] = __ldg(sb0 + nk);
            pb1[u] = __ldg(sb1 + nk);
          }
          if (!__all_sync(0xffffffff, wait_or_abort(tfull_bar + buf, bphase, abort_flag, p.err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t r0[Q], r1[Q];
          const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * BN;
          tld<Q>(taddr + c0, r0);
          tld<Q>(taddr + c1, r1);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar + buf);
#pragma unroll
          for (int i = 0; i < Q; ++i) {
            acc0[i] = fmaf(__uint_as_float(r0[i]), s0, acc0[i]);
            acc1[i] = fmaf(__uint_as_float(r1[i]), s1, acc1[i]);
          }
          if (++buf == NBUF) { buf = 0; bphase ^= 1; }
        }
      }
      if (!ok || !row_ok) continue;
      if (p.epi == 4) {
        // silu(gate) * up with the bf16 rounding points of the stand-alone SwiGLU kernel
        const int col = (ti.n0 >> 1) + half * Q;  // output column inside [0, F)
        if (col >= p.swiglu_f) continue;
        float o[Q];
#pragma unroll
        for (int i = 0; i < Q; ++i) {
          const float g = __bfloat162float(__float2bfloat16(acc0[i]));
          const float u = __bfloat162float(__float2bfloat16(acc1[i]));
          const float sg = g / (1.f + expf(-g));
          o[i] = __bfloat162float(__float2bfloat16(sg)) * u;
        }
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + col;
        store_row<Q>(out, o, p.swiglu_f - col);
        if (p.C2) {
          __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(p.C2) + (long long)row * p.ldc2 + col;
          store_row<Q>(gu, acc0, p.swiglu_f - col);
          store_row<Q>(gu + p.swiglu_f, acc1, p.swiglu_f - col);
        }
      } else {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + ti.n0;
        store_row<Q>(out + c0, acc0, p.N - (ti.n0 + c0));
        store_row<Q>(out + c1, acc1, p.N - (ti.n0 + c1));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

static int g_num_sms = 0;

template <int BN, int MODE>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  using C = Cfg<BN>;
  auto kern = gemm_fp8_kernel<BN, MODE>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
        cudaSuccess)
      return -3;
    attr_set = true;
  }
  if (g_num_sms == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  if (tiles == 0) return 0;
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  mb_launch(kern, grid, C::THREADS, C::SMEM_BYTES, st, ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int MODE>
static int dispatch(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                    cudaStream_t st) {
  switch (bn) {
    case 32: return launch<32, MODE>(ta, tb, p, st);
    case 64: return launch<64, MODE>(ta, tb, p, st);
    case 128: return launch<128, MODE>(ta, tb, p, st);
  }
  return -6;
}

// ---------------------------------------------------------------------------------------------
// Activation quantisation: x bf16 [M, K] (row stride ldx) -> q e4m3 [M, K] contiguous and
// s fp32 [K/128][lds] (K-block-major, the layout the GEMM epilogue reads coalesced).
// One warp per (row, 128-wide block): 4 elements per lane, warp max, scale = amax / 448
// (amax floored at 1e-12), q = saturate(x * (1 / scale)). Grid-stride over the items.
// Grouped buffers (offsets [E+1] and counts [E] on the device, optional): only rows below
// offsets[E] that are not segment padding are quantised (padding rows of an inference buffer
// hold stale data and their GEMM outputs are never stored).
// ---------------------------------------------------------------------------------------------
__global__ void act_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int M, int K,
                                 __nv_fp8_e4m3* __restrict__ q, float* __restrict__ s,
                                 long long lds, const int* __restrict__ offsets,
                                 const int* __restrict__ counts, int E) {
  pdl_trigger();
  pdl_wait();
  const int nkb = K / 128;
  const int lane = threadIdx.x & 31;
  int rows = M;
  if (offsets) rows = min(rows, __ldg(offsets + E));
  const int items = rows * nkb;  // < 2^31 (checked on the host)
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  // U consecutive items (row-major over (row, kb)) per warp and iteration, all loaded before any
  // is reduced; one 32-bit division per iteration locates the first of them
  constexpr int U = 4;
  for (int base = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * U; base < items;
       base += nwarps * U) {
    int row[U], kb[U];
    row[0] = base / nkb;
    kb[0] = base - row[0] * nkb;
#pragma unroll
    for (int u = 1; u < U; ++u) {
      kb[u] = kb[u - 1] + 1;
      row[u] = row[u - 1];
      if (kb[u] == nkb) { kb[u] = 0; ++row[u]; }
    }
    uint2 raw[U];
    bool use[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      use[u] = base + u < items;
      if (use[u] && offsets && counts) {
        int lo = 0, hi = E - 1;  // segment of this row: largest g with offsets[g] <= row
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (__ldg(offsets + mid) <= row[u]) lo = mid; else hi = mid - 1;
        }
        use[u] = row[u] - __ldg(offsets + lo) < __ldg(counts + lo);  // warp-uniform
      }
      if (use[u])
        raw[u] = *reinterpret_cast<const uint2*>(x + (long long)row[u] * ldx + kb[u] * 128 + lane * 4);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!use[u]) continue;
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw[u]);
      float v[4];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = __bfloat162float(h[i]);
        amax = fmaxf(amax, fabsf(v[i]));
      }
      amax = warp_max(amax);
      const float sc = fmaxf(amax, 1e-12f) / 448.f;
      const float inv = 1.f / sc;
      uint32_t packed = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_fp8_e4m3 e(fminf(fmaxf(v[i] * inv, -448.f), 448.f));
        packed |= (uint32_t)(*reinterpret_cast<const uint8_t*>(&e)) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(q) + (long long)row[u] * K + kb[u] * 128 +
                                   lane * 4) = packed;
      if (lane == 0) s[(long long)kb[u] * lds + row[u]] = sc;
    }
  }
}



}  // namespace f8
}  // namespace mb

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------
// Activation quantisation (see act_quant_kernel). K % 128 == 0, ldx % 4 == 0, lds >= M.
// offsets / counts (device, E+1 / E entries) are optional (grouped expert buffers).
extern "C" int mb_fp8_act_quant(const void* x, long long ldx, int M, int K, void* q, float* s,
                                long long lds, const int* offsets, const int* counts, int E,
                                cudaStream_t st) {
  if (K % 128 || ldx % 4 || lds < M || (offsets && E < 1)) return -1;
  if ((long long)M * (K / 128) >= (1ll << 31)) return -1;
  if (M == 0) return 0;
  const long long items = (long long)M * (K / 128);
  const int per_block = 8;
  long long blocks = (items + 4 * per_block - 1) / (4 * per_block);
  if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 blocks per SM
  mb::mb_launch(mb::f8::act_quant_kernel, dim3((unsigned)blocks), dim3(per_block * 32), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K,
                reinterpret_cast<__nv_fp8_e4m3*>(q), s, lds, offsets, counts, E);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// Block-scaled fp8 GEMM (see the header). a: e4m3 [a_rows, K] row stride lda (bytes = elements);
// b: e4m3 [b_rows, K] row stride ldb; sa [K/128][lds]; sb [b_rows/128][K/128].
// mode 0: dense, M <= a_rows, N <= b_rows. mode 1: grouped-M (group_offsets [E+1] on the
// device, 128-row aligned; M = padded row bound; b_rows_per_group rows of B per group).
// epi 0: c bf16 [M, N] (row stride ldc). epi 4: SwiGLU, B = [gate F; up F] per group, c bf16
// [M, F], optional c2 [M, 2F]. bn in {32, 64, 128}; K % 128 == 0; b_rows_per_group % 128 == 0
// in mode 1; F % 128 == 0 for SwiGLU.
extern "C" int mb_gemm_fp8(const void* a, long long a_rows, long long lda, const float* sa,
                           long long lds, const void* b, long long b_rows, long long ldb,
                           const float* sb, void* c, long long ldc, int M, int N, int K, int mode,
                           const int* group_offsets, const int* group_counts, int num_groups,
                           int b_rows_per_group, int epi, int swiglu_f, void* c2, long long ldc2,
                           int bn, int* err, cudaStream_t stream) {
  using namespace mb;
  using namespace mb::f8;
  if (K % BK || K <= 0 || (mode != 0 && mode != 1) || (epi != 0 && epi != 4)) return -1;
  if (lda % 16 || ldb % 16 || b_rows % 128) return -1;
  if (epi == 4 && (swiglu_f % 128 || N != 2 * swiglu_f)) return -1;
  if (mode == 1 && b_rows_per_group % 128) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return -8;
  CUtensorMap ta, tb;
  const uint32_t a_box_rows = (mode == 0 && M < BM) ? (uint32_t)((M + 7) / 8 * 8) : BM;
  const uint32_t b_box_rows = (uint32_t)(epi == 4 ? bn / 2 : bn);
  int rc = make_map(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a_rows, K, lda, 128, a_box_rows);
  if (rc) return rc;
  rc = make_map(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, b_rows, K, ldb, 128, b_box_rows);
  if (rc) return rc;
  Params p;
  p.M = M; p.N = N; p.K = K;
  p.C = c; p.ldc = ldc;
  p.sa = sa; p.lds = lds; p.sb = sb;
  p.group_offsets = group_offsets;
  p.group_counts = mode == 1 ? group_counts : nullptr;
  p.num_groups = num_groups;
  p.b_rows_per_group = b_rows_per_group;
  p.epi = epi; p.swiglu_f = swiglu_f; p.C2 = c2; p.ldc2 = ldc2;
  p.a_stage_bytes = (int)a_box_rows * BK;
  p.err = err;
  return mode == 0 ? dispatch<0>(bn, ta, tb, p, stream) : dispatch<1>(bn, ta, tb, p, stream);
}
