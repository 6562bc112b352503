// Expert-parallel MoE dispatch / combine over symmetric peer memory (sm_100a).
//
// Every rank of an EP group of `world` ranks owns E_local = E / world experts and maps every
// peer's symmetric region (parallel/symm.py):
//   table [world][E_local] int32   rows each source rank sends to each of my experts
//   base  [E_local][world] int32   where source s's rows of my expert e start in my buffer
//   xs    [cap][H] bf16            my experts' input rows, expert-sorted, 128-row aligned
//   ys    [cap][H] bf16            my experts' output rows (same positions)
// Forward of one layer (the host inserts device barriers between the steps):
//   1. ep_publish : the source writes its per-expert row counts into each owner's table
//   2. ep_offsets : the owner lays out its buffer (expert segments padded to 128 rows; inside a
//                   segment, source ranks in rank order) and publishes base[e][s]
//   3. ep_dispatch: the source copies every (token, slot) row straight into the owner's xs at
//                   base[e][s] + (rank of the entry among this source's entries of expert e,
//                   in token-then-slot order), and remembers that position
//   4. the owner runs its grouped GEMMs on xs (output into ys)
//   5. ep_combine : the source reads its k rows of every token from the owners' ys and sums
//                   w_j * row_j in slot order (fp32) - the arithmetic of the local combine
// Backward: ep_combine_bwd writes w * dy into the owners' dys (the ys buffer) and forms dw from
// the rows saved by the forward combine; the owner runs the grouped data / weight-grad GEMMs
// (dxs into the xs buffer); ep_gather_bwd sums the k rows of every token from the owners' dxs.
// Every row therefore crosses NVLink once per direction, with no all-to-all, no host
// synchronisation and no intermediate send/receive buffers; positions are pure functions of
// (source rank, token, slot), so results are deterministic and equal to the single-GPU layer.
//
// Reference roles: Megatron's alltoall token dispatcher / DeepEP dispatch-combine
// (--moe-token-dispatcher-type alltoall, --moe-enable-deepep) for expert parallelism.
#include "common.cuh"

namespace mb {

struct EpPeers {
  void* p[8];
};

MB_DEVICE uint4 ep_ld(const void* a) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a)
               : "memory");
  return v;
}

// counts[E] (this source's rows per global expert) -> owner d's table[rank][e_local].
__global__ void ep_publish_kernel(const int* counts, int E, int E_local, int rank, EpPeers table) {
  pdl_trigger();
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / E_local;
    reinterpret_cast<volatile int*>(table.p[d])[rank * E_local + (e % E_local)] = counts[e];
  }
}

// Owner: table[world][E_local] -> offsets[E_local + 1] (segments padded to `align`),
// counts[E_local], base[E_local][world]. One CTA; thread e handles expert e.
__global__ void ep_offsets_kernel(const int* table, int world, int E_local, int align,
                                  int* offsets, int* counts, int* base, long long cap, int* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ int seg[1024];
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) {
    int tot = 0;
    for (int s = 0; s < world; ++s) tot += reinterpret_cast<const volatile int*>(table)[s * E_local + e];
    counts[e] = tot;
    seg[e] = (tot + align - 1) / align * align;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E_local; ++e) {
      const int len = seg[e];
      seg[e] = o;
      offsets[e] = o;
      o += len;
    }
    offsets[E_local] = o;
    if (o > cap) report_error(err, 4);  // receive buffer too small: rows are dropped
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) {
    int b = seg[e];
    for (int s = 0; s < world; ++s) {
      base[e * world + s] = b;
      b += reinterpret_cast<const volatile int*>(table)[s * E_local + e];
    }
  }
}

// Source: one warp per (token, slot) entry. dest_g / off_g come from the permute plan of this
// source's entries over the global experts (dest_g[i] - off_g[e] = rank of entry i among this
// source's entries of expert e). Writes the row into the owner's xs and its position to pos[i].
__global__ void ep_dispatch_kernel(const __nv_bfloat16* x, const int* idx, const int* dest_g,
                                   const int* off_g, int n, int k, int H, int E_local, int rank,
                                   int world, EpPeers base, EpPeers xs, long long cap, int* pos,
                                   int* err) {
  pdl_trigger();
  pdl_wait();
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const int e = idx[w];
  const int d = e / E_local, el = e % E_local;
  const int b = reinterpret_cast<const volatile int*>(base.p[d])[el * world + rank];
  const long long p = (long long)b + (dest_g[w] - off_g[e]);
  if (p >= cap) {
    if (lane == 0) {
      report_error(err, 4);
      pos[w] = -1;
    }
    return;
  }
  if (lane == 0) pos[w] = (int)p;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long long)(w / k) * H);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(xs.p[d]) + p * H);
  for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

// Source: y[t] = sum_j w[t,j] * ys_{owner(t,j)}[pos[t,j]] (+ add[t]), fp32 in slot order; with
// `saved` also stores the k rows it read ([T*k, H]) for the backward. One warp per (token,
// 256-column chunk), as the local combine.
__global__ void ep_combine_kernel(EpPeers ys, const int* idx, const int* pos, const float* w,
                                  const __nv_bfloat16* add, int T, int k, int H, int E_local,
                                  __nv_bfloat16* y, __nv_bfloat16* saved) {
  pdl_trigger();
  pdl_wait();
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nch = H / 256;
  if (gw >= (long long)T * nch) return;
  const int t = (int)(gw / nch);
  const int c = (int)(gw % nch) * 256 + lane * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j = 0; j < k; ++j) {
    const int i = t * k + j;
    const float wj = w[i];
    const int p = pos[i];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (p >= 0)
      v = ep_ld(reinterpret_cast<const __nv_bfloat16*>(ys.p[idx[i] / E_local]) + (long long)p * H + c);
    if (saved) *reinterpret_cast<uint4*>(saved + (long long)i * H + c) = v;
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] += wj * __bfloat162float(b[q]);
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

// Source, backward of the combine: dys_{owner}[pos] = w * dy[t] (stored into the owner's
// buffer), dw[t,j] = <dy[t], saved[t*k+j]>. One warp per token, as the local kernel.
__global__ void ep_combine_bwd_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* saved,
                                      const int* idx, const int* pos, const float* w, int T,
                                      int k, int H, int E_local, EpPeers dys, float* dw) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int j = 0; j < k; ++j) {
    const int i = t * k + j;
    const int p = pos[i];
    const float wj = w[i];
    __nv_bfloat16* out = p >= 0 ? reinterpret_cast<__nv_bfloat16*>(dys.p[idx[i] / E_local]) + (long long)p * H
                                : nullptr;
    float dot = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 g = *reinterpret_cast<const uint4*>(dy + (long long)t * H + c);
      const uint4 v = *reinterpret_cast<const uint4*>(saved + (long long)i * H + c);
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
      if (out) *reinterpret_cast<uint4*>(out + c) = o;
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[i] = dot;
  }
}

// Source, backward of the dispatch: dx[t] = sum_j dxs_{owner}[pos[t,j]] in slot order.
__global__ void ep_gather_bwd_kernel(EpPeers dxs, const int* idx, const int* pos, int T, int k,
                                     int H, int E_local, __nv_bfloat16* dx) {
  pdl_trigger();
  pdl_wait();
  const long long gw = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nch = H / 256;
  if (gw >= (long long)T * nch) return;
  const int t = (int)(gw / nch);
  const int c = (int)(gw % nch) * 256 + lane * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j = 0; j < k; ++j) {
    const int i = t * k + j;
    const int p = pos[i];
    if (p < 0) continue;
    const uint4 v = ep_ld(reinterpret_cast<const __nv_bfloat16*>(dxs.p[idx[i] / E_local]) + (long long)p * H + c);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(b[q]);
  }
  uint4 o;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(acc[q]);
  *reinterpret_cast<uint4*>(dx + (long long)t * H + c) = o;
}

}  // namespace mb

using namespace mb;

static EpPeers ep_peers(const long long* p, int n) {
  EpPeers r{};
  for (int i = 0; i < n && i < 8; ++i) r.p[i] = reinterpret_cast<void*>(p[i]);
  return r;
}

extern "C" {

int mb_ep_publish(const int* counts, int E, int E_local, int rank, int world,
                  const long long* table_ptrs, cudaStream_t st) {
  if (world < 1 || world > 8 || E != E_local * world) return -1;
  mb_launch(ep_publish_kernel, 1, 256, 0, st, counts, E, E_local, rank, ep_peers(table_ptrs, world));
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_ep_offsets(const int* table, int world, int E_local, int align, int* offsets, int* counts,
                  int* base, long long cap, int* err, cudaStream_t st) {
  if (E_local > 1024 || world > 8) return -1;
  mb_launch(ep_offsets_kernel, 1, 256, 0, st, table, world, E_local, align, offsets, counts, base,
            cap, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_ep_dispatch(const void* x, const int* idx, const int* dest_g, const int* off_g, int T,
                   int k, int H, int E_local, int rank, int world, const long long* base_ptrs,
                   const long long* xs_ptrs, long long cap, int* pos, int* err, cudaStream_t st) {
  if (H % 8 || world > 8) return -1;
  const long long n = (long long)T * k;
  if (n == 0) return 0;
  mb_launch(ep_dispatch_kernel, (unsigned)((n + 7) / 8), 256, 0, st, (const __nv_bfloat16*)x, idx,
            dest_g, off_g, (int)n, k, H, E_local, rank, world, ep_peers(base_ptrs, world),
            ep_peers(xs_ptrs, world), cap, pos, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_ep_combine(const long long* ys_ptrs, int world, const int* idx, const int* pos,
                  const float* w, const void* add, int T, int k, int H, int E_local, void* y,
                  void* saved, cudaStream_t st) {
  if (H % 256 || world > 8) return -1;
  if (T == 0) return 0;
  const long long wc = (long long)T * (H / 256);
  mb_launch(ep_combine_kernel, (unsigned)((wc + 7) / 8), 256, 0, st, ep_peers(ys_ptrs, world), idx,
            pos, w, (const __nv_bfloat16*)add, T, k, H, E_local, (__nv_bfloat16*)y,
            (__nv_bfloat16*)saved);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_ep_combine_bwd(const void* dy, const void* saved, const int* idx, const int* pos,
                      const float* w, int T, int k, int H, int E_local, int world,
                      const long long* dys_ptrs, float* dw, cudaStream_t st) {
  if (H % 256 || world > 8) return -1;
  if (T == 0) return 0;
  mb_launch(ep_combine_bwd_kernel, (T + 7) / 8, 256, 0, st, (const __nv_bfloat16*)dy,
            (const __nv_bfloat16*)saved, idx, pos, w, T, k, H, E_local, ep_peers(dys_ptrs, world), dw);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int mb_ep_gather_bwd(const long long* dxs_ptrs, int world, const int* idx, const int* pos, int T,
                     int k, int H, int E_local, void* dx, cudaStream_t st) {
  if (H % 256 || world > 8) return -1;
  if (T == 0) return 0;
  const long long wg = (long long)T * (H / 256);
  mb_launch(ep_gather_bwd_kernel, (unsigned)((wg + 7) / 8), 256, 0, st, ep_peers(dxs_ptrs, world),
            idx, pos, T, k, H, E_local, (__nv_bfloat16*)dx);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"
