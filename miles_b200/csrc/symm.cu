// Symmetric peer memory and in-kernel collectives over NVLink / NVSwitch (sm_100a).
//
// A "symmetric buffer" is one cudaMalloc'd region per rank whose CUDA IPC handle has been
// exchanged with every other rank of the group; each rank then holds device pointers to all
// peers' copies (opened with cudaIpcOpenMemHandle, lazy peer access). Kernels load from and
// store to those pointers directly: the data crosses NVLink / NVSwitch from inside the kernel,
// with no library collective and no copy engine.
//
// Synchronisation between ranks uses monotonically increasing epochs:
//   * every rank owns a control word pair ctl = {epoch, done, arrived} in its local memory;
//   * every rank owns a symmetric flag array flags[world] (flags[r] = last epoch rank r
//     announced to this rank);
//   * one collective call = one epoch e = ctl.epoch + 1. A rank announces e to every peer with
//     a system-scope release store into the peer's flags[rank] once its data is in place, and
//     waits (system-scope acquire loads) until its own flags[0..world) all reach e.
//   * the staging area is double-buffered by the parity of the epoch, so the data of call e+1
//     can land while a slow peer still reads call e: a rank writes call e+2's data only after
//     it has seen every peer announce e+1, which each peer does after finishing call e.
//   * the last CTA of the call to finish advances ctl.epoch; the epoch therefore lives on the
//     device, and a captured CUDA graph replays the collective correctly.
// Every wait is bounded (wall clock, `timeout_ns`); on expiry the kernel records error code 3
// in the library's device error word, skips the reduction and still advances the epoch, so the
// context stays usable and the host reports the failure.
//
// Kernels here never use TMA, so no tensor-memory-accelerator load ever reads a peer's memory.
//
// Reduction order is fixed (rank 0, 1, ..., world-1, fp32 accumulation, one rounding), so every
// rank obtains bitwise the same result and repeated calls are deterministic.
//
// Reference roles: NCCL all-reduce after row-parallel linears (Megatron TP,
// megatron_utils/model_provider.py) and SGLang's custom all-reduce in TP decode; NCCL barrier /
// broadcast in update_weight/broadcast.py.
#include "common.cuh"
#include <cstring>
#include <cuda_fp8.h>

namespace mb {

constexpr int kMaxPeers = 8;
struct Peers {
  void* p[kMaxPeers];
};

MB_DEVICE void st_release_sys(int* a, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
MB_DEVICE int ld_acquire_sys(const int* a) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
// Loads of data that other GPUs wrote during this collective: never through the non-coherent
// read-only path.
MB_DEVICE uint4 ld_volatile_v4(const void* a) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a)
               : "memory");
  return v;
}

// Announce epoch e to every rank (including this one).
MB_DEVICE void announce(const Peers& flags, int rank, int world, int e) {
  __threadfence_system();
  for (int r = threadIdx.x; r < world; r += blockDim.x)
    st_release_sys(reinterpret_cast<int*>(flags.p[r]) + rank, e);
}

// Wait until every rank announced epoch e to this rank. CTA-collective; returns false on
// timeout (after recording code 3).
MB_DEVICE bool wait_all(const int* my_flags, int world, int e, long long timeout_ns, int* err) {
  bool ok = true;
  if ((int)threadIdx.x < world) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(my_flags + threadIdx.x) - e < 0) {
      if ((long long)(global_ns() - t0) > timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(100);
    }
  }
  ok = __syncthreads_and(ok);
  if (!ok && threadIdx.x == 0) report_error(err, 3);
  return ok;
}

// Finish the call: the last CTA advances the epoch.
MB_DEVICE void finish(int* ctl, int e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int d = atomicAdd(ctl + 1, 1);
    if (d == (int)gridDim.x - 1) {
      ctl[1] = 0;
      ctl[2] = 0;
      __threadfence();
      atomicExch(ctl, e);
    }
  }
}

struct ReduceArgs {
  Peers flags;          // flags[r] -> rank r's flag array
  Peers stage;          // stage[r] -> rank r's staging area (push mode writes there)
  int* my_flags;        // this rank's flag array
  int* ctl;             // this rank's control words {epoch, done, arrived}
  const __nv_bfloat16* my_stage;  // this rank's staging area: [2][world][cap][H]
  const __nv_bfloat16* src;       // push mode: this rank's partial [rows, H]; null: data already staged
  const __nv_bfloat16* res;       // optional residual [rows, H] (norm mode)
  const __nv_bfloat16* w;         // norm weight [H] (norm mode)
  __nv_bfloat16* out;             // sum [rows, H] (plain) or normed y (norm mode)
  __nv_bfloat16* h_out;           // norm mode with residual: h = sum + res
  float* rstd_out;                // optional
  long long cap;                  // rows per staging slot
  int rows, H, rank, world;       // rows: rows of each slot the consumer reads
  int scatter_rows;               // push: 0 = every peer gets all `rows` rows of src;
                                  // 1 = peer r gets rows [r*rows, (r+1)*rows) (reduce-scatter)
  float eps;
  long long timeout_ns;
  int* err;
};

// Push phase of a stand-alone all-reduce: copy this rank's partial into slot `rank` of every
// peer's staging (parity par); the last CTA to finish announces the epoch.
MB_DEVICE void push_and_announce(const ReduceArgs& a, int par, int e) {
  const long long n8 = (long long)a.rows * a.H / 8;
  const long long slot = (long long)a.cap * a.H;
  const long long my_slot = ((long long)par * a.world + a.rank) * slot;
  if (a.scatter_rows) {
    // row block r of src -> peer r (each element crosses NVLink once)
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8 * a.world;
         i += (long long)gridDim.x * blockDim.x) {
      const int r = (int)(i / n8);
      const uint4 v = *reinterpret_cast<const uint4*>(a.src + i * 8);
      __nv_bfloat16* dst =
          reinterpret_cast<__nv_bfloat16*>(a.stage.p[r]) + my_slot + (i - r * n8) * 8;
      *reinterpret_cast<uint4*>(dst) = v;
    }
  } else {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x) {
      const uint4 v = *reinterpret_cast<const uint4*>(a.src + i * 8);
      for (int r = 0; r < a.world; ++r) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.stage.p[r]) + my_slot + i * 8;
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(a.ctl + 2, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (last) announce(a.flags, a.rank, a.world, e);
}

// Plain all-reduce: out = sum over ranks of the staged partials (rank order, fp32).
__global__ void __launch_bounds__(256) symm_allreduce_kernel(ReduceArgs a) {
  pdl_trigger();
  pdl_wait();
  const int e = *reinterpret_cast<volatile int*>(a.ctl) + 1;
  const int par = (e - 1) & 1;
  if (a.src) push_and_announce(a, par, e);
  else if (blockIdx.x == 0) announce(a.flags, a.rank, a.world, e);
  if (wait_all(a.my_flags, a.world, e, a.timeout_ns, a.err)) {
    const long long n8 = (long long)a.rows * a.H / 8;
    const long long slot = (long long)a.cap * a.H;
    const __nv_bfloat16* base = a.my_stage + (long long)par * a.world * slot;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x) {
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      for (int r = 0; r < a.world; ++r) {
        const uint4 v = ld_volatile_v4(base + r * slot + i * 8);
        const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(vb[k]);
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(a.out + i * 8) = o;
    }
  }
  finish(a.ctl, e);
}

// All-gather: out[r * rows + i] = slot_r[i] (rows of every rank, in rank order).
__global__ void __launch_bounds__(256) symm_allgather_kernel(ReduceArgs a) {
  pdl_trigger();
  pdl_wait();
  const int e = *reinterpret_cast<volatile int*>(a.ctl) + 1;
  const int par = (e - 1) & 1;
  push_and_announce(a, par, e);
  if (wait_all(a.my_flags, a.world, e, a.timeout_ns, a.err)) {
    const long long n8 = (long long)a.rows * a.H / 8;
    const long long slot = (long long)a.cap * a.H;
    const __nv_bfloat16* base = a.my_stage + (long long)par * a.world * slot;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8 * a.world;
         i += (long long)gridDim.x * blockDim.x) {
      const int r = (int)(i / n8);
      *reinterpret_cast<uint4*>(a.out + i * 8) = ld_volatile_v4(base + r * slot + (i - r * n8) * 8);
    }
  }
  finish(a.ctl, e);
}

// All-reduce fused with the residual add and RMSNorm that follow a row-parallel projection:
//   s = sum_r partial_r (bf16), h = s + res (bf16), y = rmsnorm(h) * w.
// Same per-row arithmetic (and bits) as rmsnorm_fwd_kernel applied to (s, res). One CTA per
// row, grid-stride over rows.
template <int H>
struct RowShape {
  static constexpr int NCH = H / 8;
  static constexpr int CPT = NCH / 128 > 1 ? NCH / 128 : 1;
  static constexpr int NT = NCH / CPT;
  static_assert(NCH % CPT == 0 && NT % 32 == 0, "unsupported hidden size");
};

// ROWS rows per CTA at once (NT threads each, the per-row thread assignment and reduction tree
// of rmsnorm_fwd_kernel), so short rows still keep enough loads in flight.
template <int H>
struct RowTile {
  static constexpr int ROWS = RowShape<H>::NT >= 512 ? 1 : 512 / RowShape<H>::NT;
  static constexpr int THREADS = ROWS * RowShape<H>::NT;
};

template <int H>
__global__ void __launch_bounds__(RowTile<H>::THREADS) symm_allreduce_norm_kernel(ReduceArgs a) {
  pdl_trigger();
  pdl_wait();
  using S = RowShape<H>;
  constexpr int NW = S::NT / 32;
  constexpr int ROWS = RowTile<H>::ROWS;
  __shared__ float wsum[ROWS][NW];
  const int e = *reinterpret_cast<volatile int*>(a.ctl) + 1;
  const int par = (e - 1) & 1;
  if (a.src) push_and_announce(a, par, e);
  else if (blockIdx.x == 0) announce(a.flags, a.rank, a.world, e);
  const int sub = threadIdx.x / S::NT;  // which of the CTA's rows
  const int tid = threadIdx.x % S::NT;  // thread within the row
  if (wait_all(a.my_flags, a.world, e, a.timeout_ns, a.err)) {
    const long long slot = a.cap * H;
    const __nv_bfloat16* base = a.my_stage + (long long)par * a.world * slot;
    for (int row0 = blockIdx.x * ROWS; row0 < a.rows; row0 += gridDim.x * ROWS) {
      const int row = row0 + sub;
      const bool active = row < a.rows;
      const long long rb = (long long)row * H;
      float v[S::CPT * 8];
#pragma unroll
      for (int j = 0; j < S::CPT; ++j) {
        const int col = (tid + j * S::NT) * 8;
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.f;
        if (active) {
          for (int r = 0; r < a.world; ++r) {
            const uint4 x = ld_volatile_v4(base + r * slot + rb + col);
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&x);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(xb[k]);
          }
        }
        if (a.res && active) {
          const uint4 rr = *reinterpret_cast<const uint4*>(a.res + rb + col);
          const __nv_bfloat16* rbf = reinterpret_cast<const __nv_bfloat16*>(&rr);
          uint4 o;
          __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float s = __bfloat162float(__float2bfloat16(acc[k]));
            ob[k] = __float2bfloat16(s + __bfloat162float(rbf[k]));
            v[j * 8 + k] = __bfloat162float(ob[k]);
          }
          *reinterpret_cast<uint4*>(a.h_out + rb + col) = o;
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) v[j * 8 + k] = __bfloat162float(__float2bfloat16(acc[k]));
        }
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < S::CPT * 8; ++i) ss += v[i] * v[i];
      ss = warp_sum(ss);
      if ((tid & 31) == 0) wsum[sub][tid >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < NW; ++i) tot += wsum[sub][i];
      __syncthreads();  // wsum is reused by the next rows
      if (!active) continue;
      const float rstd = rsqrtf(tot / (float)H + a.eps);
      if (tid == 0 && a.rstd_out) a.rstd_out[row] = rstd;
#pragma unroll
      for (int j = 0; j < S::CPT; ++j) {
        const int col = (tid + j * S::NT) * 8;
        const uint4 wv = *reinterpret_cast<const uint4*>(a.w + col);
        const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
        uint4 o;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float nrm = __bfloat162float(__float2bfloat16(v[j * 8 + k] * rstd));
          ob[k] = __float2bfloat16(nrm * __bfloat162float(wb[k]));
        }
        *reinterpret_cast<uint4*>(a.out + rb + col) = o;
      }
    }
  }
  finish(a.ctl, e);
}

// Barrier over the group (no data): announce, wait, advance.
__global__ void symm_barrier_kernel(Peers flags, int* my_flags, int* ctl, int rank, int world,
                                    long long timeout_ns, int* err) {
  pdl_trigger();
  pdl_wait();
  const int e = *reinterpret_cast<volatile int*>(ctl) + 1;
  announce(flags, rank, world, e);
  wait_all(my_flags, world, e, timeout_ns, err);
  finish(ctl, e);
}

// Copy `n` 16-byte chunks from a (possibly peer) source to a (possibly peer) destination with SM
// loads/stores; used for refit pushes where the copy is fused with other per-element work.
__global__ void symm_copy_kernel(const uint4* src, uint4* dst, long long n) {
  pdl_trigger();
  pdl_wait();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// 128x128-block fp8 (e4m3) -> bf16 with per-block fp32 scales; q and s may live in a peer's
// memory (refit: the trainer quantised straight into the owner engine's staging). 16 elements
// (one 16-byte fp8 load, two 16-byte bf16 stores) per thread step; N % 16 == 0.
__global__ void fp8_block_dequant_kernel(const uint8_t* q, const float* s, int M, int N, int bm,
                                         int bn, __nv_bfloat16* out) {
  pdl_trigger();
  pdl_wait();
  const int gn = (N + bn - 1) / bn;
  const long long n16 = (long long)M * N / 16;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
       i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 16;
    const int row = (int)(e / N), col = (int)(e % N);
    const float sc = s[(long long)(row / bm) * gn + col / bn];
    const uint4 v = ld_volatile_v4(q + e);
    const __nv_fp8_e4m3* f = reinterpret_cast<const __nv_fp8_e4m3*>(&v);
    uint4 o[2];
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(o);
#pragma unroll
    for (int k = 0; k < 16; ++k) ob[k] = __float2bfloat16(float(f[k]) * sc);
    *reinterpret_cast<uint4*>(out + e) = o[0];
    *reinterpret_cast<uint4*>(out + e + 8) = o[1];
  }
}

// Gradient reduce-scatter fused with the cast / scale and the squared norm of the result: this
// rank's shard [lo, lo + 8 * n8) of the flat bf16 gradient is summed over every rank's copy,
// read straight from the peers' memory (rank order, fp32, one rounding: bitwise the same on
// every run), scaled, rounded to bf16 and stored in place into this rank's own copy (a range no
// peer reads); the squared norm of the stored values goes to *sq_out (per-CTA partials reduced
// in CTA order by the last CTA: deterministic). All loads of a chunk are issued before the
// accumulation, so `world` 16-byte loads per thread are in flight. The caller orders the call
// after every rank's backward (a barrier) and keeps its own gradient buffer unchanged until
// every rank's call has finished (the parameter all-gather that follows).
__global__ void __launch_bounds__(256) grad_rs_kernel(Peers g, long long lo, long long n8,
                                                      float scale, int world, __nv_bfloat16* out,
                                                      float* partial, int* counter, float* sq_out) {
  pdl_trigger();
  pdl_wait();
  float sq = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    uint4 v[kMaxPeers];
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < world) v[r] = ld_volatile_v4(reinterpret_cast<const __nv_bfloat16*>(g.p[r]) + lo + i * 8);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r < world) {
        const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v[r]);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(vb[k]);
      }
    }
    uint4 o;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      ob[k] = __float2bfloat16(acc[k] * scale);
      const float f = __bfloat162float(ob[k]);
      sq += f * f;
    }
    *reinterpret_cast<uint4*>(out + i * 8) = o;
  }
  // CTA sum in a fixed tree, then the last CTA adds the partials in CTA order
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, d);
  __shared__ float ws[8];
  __shared__ int last;
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += ws[w];
    partial[blockIdx.x] = t;
    __threadfence();
    last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    float t = 0.f;
    for (int b = 0; b < (int)gridDim.x; ++b) t += *reinterpret_cast<volatile float*>(partial + b);
    *sq_out = t;
    *counter = 0;
  }
}

}  // namespace mb

using namespace mb;

static Peers to_peers(const long long* ptrs, int n) {
  Peers p{};
  for (int i = 0; i < n && i < kMaxPeers; ++i) p.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return p;
}

// Every CTA of a collective must be resident at once (a CTA waits for announcements that other
// CTAs of the peers' grids make), so a grid never exceeds what the GPU holds at once: the
// occupancy of the kernel at its block size times the SM count, at most 2 CTAs per SM (other
// work sharing the GPU keeps room), at least one per SM.
template <typename K>
static int coll_grid(K kernel, int block, long long work, int per_cta) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  int occ = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, 0) != cudaSuccess || occ < 1)
    occ = 1;
  if (occ > 2) occ = 2;
  long long g = (work + per_cta - 1) / per_cta;
  const long long cap = (long long)occ * sms;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

extern "C" {
int mb_symm_collective(int kind, const long long* flag_ptrs, const long long* stage_ptrs,
                       int* my_flags, int* ctl, const void* my_stage, long long cap,
                       const void* src, int rows, int H, int rank, int world, const void* res,
                       const void* norm_w, float eps, void* out, void* h_out, float* rstd,
                       long long timeout_ns, int* err, cudaStream_t st);

int mb_ipc_handle_size() { return (int)sizeof(cudaIpcMemHandle_t); }

int mb_symm_malloc(long long bytes, long long* ptr_out) {
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return -2;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) return -2;
  *ptr_out = reinterpret_cast<long long>(p);
  return 0;
}

int mb_symm_free(long long ptr) {
  return cudaFree(reinterpret_cast<void*>(ptr)) == cudaSuccess ? 0 : -2;
}

int mb_ipc_get_handle(long long ptr, void* handle_out) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)) != cudaSuccess) return -2;
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

// Handle of the allocation that contains `ptr` (e.g. a tensor inside a caching-allocator block)
// and ptr's byte offset from the allocation's base; the importer adds the offset to the base
// that cudaIpcOpenMemHandle returns.
int mb_ipc_get_handle_range(long long ptr, void* handle_out, long long* offset_out) {
  typedef CUresult (*range_fn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static range_fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return -3;
    fn = reinterpret_cast<range_fn>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return -3;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return -2;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = ptr - (long long)base;
  return 0;
}

int mb_ipc_open(const void* handle, long long* ptr_out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return -2;
  *ptr_out = reinterpret_cast<long long>(p);
  return 0;
}

int mb_ipc_close(long long ptr) {
  return cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)) == cudaSuccess ? 0 : -2;
}

int mb_symm_barrier(const long long* flag_ptrs, int* my_flags, int* ctl, int rank, int world,
                    long long timeout_ns, int* err, cudaStream_t st) {
  if (world < 1 || world > kMaxPeers) return -1;
  mb_launch(symm_barrier_kernel, 1, 32, 0, st, to_peers(flag_ptrs, world), my_flags, ctl, rank,
            world, timeout_ns, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// out = sum over ranks of partials. If src is given it is pushed into the peers' staging first;
// otherwise the partials are already staged (e.g. by a GEMM epilogue that stored its tiles into
// the peers' staging). norm_w != null selects the fused residual + RMSNorm form.
int mb_symm_allreduce(const long long* flag_ptrs, const long long* stage_ptrs, int* my_flags,
                      int* ctl, const void* my_stage, long long cap, const void* src, int rows,
                      int H, int rank, int world, const void* res, const void* norm_w,
                      float eps, void* out, void* h_out, float* rstd, long long timeout_ns,
                      int* err, cudaStream_t st) {
  return mb_symm_collective(0, flag_ptrs, stage_ptrs, my_flags, ctl, my_stage, cap, src, rows, H,
                            rank, world, res, norm_w, eps, out, h_out, rstd, timeout_ns, err, st);
}

// kind 0: all-reduce (above); 1: reduce-scatter (src holds world * rows rows, row block r
// goes to rank r, out = this rank's summed block of `rows` rows; norm_w / res fuse the
// residual + RMSNorm on that block); 2: all-gather (src holds `rows` rows, out world * rows).
int mb_symm_collective(int kind, const long long* flag_ptrs, const long long* stage_ptrs,
                       int* my_flags, int* ctl, const void* my_stage, long long cap,
                       const void* src, int rows, int H, int rank, int world, const void* res,
                       const void* norm_w, float eps, void* out, void* h_out, float* rstd,
                       long long timeout_ns, int* err, cudaStream_t st) {
  if (world < 1 || world > kMaxPeers || rows > cap || H % 8 || kind < 0 || kind > 2) return -1;
  if (kind == 2 && (!src || norm_w)) return -1;
  if (rows == 0) return 0;
  ReduceArgs a;
  a.flags = to_peers(flag_ptrs, world);
  a.stage = to_peers(stage_ptrs, world);
  a.my_flags = my_flags; a.ctl = ctl;
  a.my_stage = (const __nv_bfloat16*)my_stage;
  a.src = (const __nv_bfloat16*)src;
  a.res = (const __nv_bfloat16*)res;
  a.w = (const __nv_bfloat16*)norm_w;
  a.out = (__nv_bfloat16*)out;
  a.h_out = (__nv_bfloat16*)h_out;
  a.rstd_out = rstd;
  a.cap = cap; a.rows = rows; a.H = H; a.rank = rank; a.world = world; a.eps = eps;
  a.timeout_ns = timeout_ns; a.err = err;
  a.scatter_rows = kind == 1;
  if (kind == 2) {
    mb_launch(symm_allgather_kernel, coll_grid(symm_allgather_kernel, 256, (long long)rows * H / 8 * world, 256 * 4),
              256, 0, st, a);
  } else if (!norm_w) {
    mb_launch(symm_allreduce_kernel, coll_grid(symm_allreduce_kernel, 256, (long long)rows * H / 8, 256 * 4),
              256, 0, st, a);
  } else {
    if (res && !h_out) return -1;
#define AR_CASE(HH)                                                                            \
  case HH:                                                                                     \
    mb_launch(symm_allreduce_norm_kernel<HH>,                                                 \
              coll_grid(symm_allreduce_norm_kernel<HH>, RowTile<HH>::THREADS, rows,             \
                        RowTile<HH>::ROWS),                                                   \
              RowTile<HH>::THREADS, 0, st, a);                                                 \
    break;
    switch (H) {
      AR_CASE(256) AR_CASE(512) AR_CASE(1024) AR_CASE(2048) AR_CASE(2560) AR_CASE(4096)
      AR_CASE(5120) AR_CASE(7168) AR_CASE(8192)
      default: return -1;
    }
#undef AR_CASE
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_symm_copy(const void* src, void* dst, long long bytes, cudaStream_t st) {
  if (bytes % 16 || (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16)
    return -1;
  if (bytes == 0) return 0;
  const long long n = bytes / 16;
  long long g = (n + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  mb_launch(symm_copy_kernel, (int)g, 256, 0, st, (const uint4*)src, (uint4*)dst, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_fp8_block_dequant(const void* q, const float* s, int M, int N, int bm, int bn, void* out,
                         cudaStream_t st) {
  if (N % 16 || bn % 16 || (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) % 16)
    return -1;
  if (M == 0) return 0;
  const long long n16 = (long long)M * N / 16;
  long long g = (n16 + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  mb_launch(fp8_block_dequant_kernel, (int)g, 256, 0, st, (const uint8_t*)q, s, M, N, bm, bn,
            (__nv_bfloat16*)out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Fused gradient reduce-scatter (grad_rs_kernel). g_ptrs: every rank's flat gradient base
// (this rank's own at index rank); out = this rank's base + lo. partial: >= 148 * 4 floats.
int mb_grad_rs(const long long* g_ptrs, int world, long long lo, long long n, float scale,
               void* out, float* partial, int* counter, float* sq_out, cudaStream_t st) {
  if (world < 1 || world > kMaxPeers || n % 8 || lo % 8) return -1;
  for (int r = 0; r < world; ++r)
    if (g_ptrs[r] % 16) return -1;
  if (reinterpret_cast<uintptr_t>(out) % 16) return -1;
  const long long n8 = n / 8;
  long long grid = (n8 + 255) / 256;
  if (grid > 148 * 4) grid = 148 * 4;
  if (grid < 1) grid = 1;
  mb_launch(grad_rs_kernel, (int)grid, 256, 0, st, to_peers(g_ptrs, world), lo, n8, scale, world,
            (__nv_bfloat16*)out, partial, counter, sq_out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"
