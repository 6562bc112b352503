// Device-resident decode state for the rollout engine.
//
// The engine keeps every live sequence's decode state in device arrays indexed by a sequence
// slot (last token, position, page-table row, sampling parameters, generated-token count, done
// flag, stop tokens) and records each step's outputs (token, log-prob, routed experts) into
// per-slot device buffers. A captured CUDA graph then runs several decode steps back to back:
//
//   prep (this file) -> forward -> sampler -> commit (this file)   (x steps per graph)
//
// with no host involvement between steps: `prep` gathers the batch rows' inputs from their
// slots, `commit` appends the sampled token and advances the slot (or marks it done on a stop
// token / length limit; a done slot is frozen and its later rows write nothing). The host reads
// the done flags once per graph replay.
//
// Batch row j of a bucket of B rows serves slot rows[j]; rows[j] == spare (the last slot) is a
// padding row: it reads and writes only the trash KV page 0.
//
// Reference role: SGLang's scheduler loop + output processor (one host round trip per step
// there); here the loop state lives on the device.
#include "common.cuh"

namespace es {
using namespace mb;

__global__ void decode_prep_kernel(const int* __restrict__ rows, int B, int spare,
                                   const int* __restrict__ s_tok, const int* __restrict__ s_pos,
                                   const int* __restrict__ s_done,
                                   const int* __restrict__ s_pt, int max_pages,
                                   const float* __restrict__ s_invt,
                                   const long long* __restrict__ s_seed,
                                   int* __restrict__ tokens, int* __restrict__ positions,
                                   int* __restrict__ ctx, long long* __restrict__ slots,
                                   int* __restrict__ pt, float* __restrict__ invt,
                                   long long* __restrict__ seeds,
                                   long long* __restrict__ state_rows, int state_spare) {
  pdl_trigger();
  pdl_wait();
  const int j = blockIdx.x;
  if (j >= B) return;
  const int s = rows[j];
  if (!MB_GUARD(s >= 0 && s <= spare, 51)) return;  // batch row mapped to no slot
  const bool live = s != spare && !s_done[s];
  int p = live ? s_pos[s] : 0;
  // a position past the page table would index outside the row: treat the row as padding
  if (live && (p >> 6) >= max_pages) p = 0;
  const bool real = live && p > 0;
  for (int c = threadIdx.x; c < max_pages; c += blockDim.x)
    pt[(long long)j * max_pages + c] = real ? s_pt[(long long)s * max_pages + c] : 0;
  if (threadIdx.x == 0) {
    tokens[j] = real ? s_tok[s] : 0;
    positions[j] = p;
    ctx[j] = p + 1;
    slots[j] = real ? (long long)s_pt[(long long)s * max_pages + (p >> 6)] * 64 + (p & 63)
                    : (long long)(j & 63);
    invt[j] = real ? s_invt[s] : 1.f;
    seeds[j] = real ? s_seed[s] : 0;
    if (state_rows) state_rows[j] = real ? s : state_spare;
  }
}

// experts: [n_moe, B, k] int32 routing of the token fed at row j (layer-major, as the router
// writes it; nullptr without MoE / R3); out_exp: [slots, max_len, n_moe, k] uint8, written at
// the fed token's position.
__global__ void decode_commit_kernel(const int* __restrict__ rows, int B, int spare,
                                     const int* __restrict__ tok, const float* __restrict__ lp,
                                     const int* __restrict__ experts, int n_moe, int topk,
                                     int* __restrict__ s_tok, int* __restrict__ s_pos,
                                     int* __restrict__ s_done, int* __restrict__ s_nout,
                                     const int* __restrict__ s_maxnew,
                                     const int* __restrict__ s_stop, int nstop,
                                     int* __restrict__ out_tok, float* __restrict__ out_lp,
                                     int max_new, unsigned char* __restrict__ out_exp,
                                     const int* __restrict__ s_rec, int max_len) {
  pdl_trigger();
  pdl_wait();
  const int j = blockIdx.x;
  if (j >= B) return;
  const int s = rows[j];
  if (!MB_GUARD(s >= 0 && s <= spare, 52)) return;
  if (s == spare) return;
  __shared__ int live_sh, pos_sh;
  if (threadIdx.x == 0) {
    live_sh = !s_done[s] && s_pos[s] > 0;
    pos_sh = s_pos[s];
  }
  __syncthreads();
  if (!live_sh) return;
  const int p = pos_sh;
  if (experts && out_exp && s_rec[s] && p < max_len) {
    const int nk = n_moe * topk;
    unsigned char* dst = out_exp + ((long long)s * max_len + p) * nk;
    for (int c = threadIdx.x; c < nk; c += blockDim.x) {
      const int l = c / topk, kk = c - l * topk;
      dst[c] = (unsigned char)experts[((long long)l * B + j) * topk + kk];
    }
  }
  __syncthreads();  // every thread has read s_pos before thread 0 advances it
  if (threadIdx.x == 0) {
    const int n = s_nout[s];
    const int t = tok[j];
    if (n < max_new) {
      out_tok[(long long)s * max_new + n] = t;
      out_lp[(long long)s * max_new + n] = lp[j];
    }
    bool stop = n + 1 >= s_maxnew[s] || n + 1 >= max_new;
    for (int c = 0; c < nstop; ++c) stop |= (s_stop[(long long)s * nstop + c] == t);
    s_nout[s] = n + 1;
    s_tok[s] = t;
    s_pos[s] = p + 1;
    if (stop) s_done[s] = 1;
  }
}

}  // namespace es

extern "C" int mb_decode_prep(const int* rows, int B, int spare, const int* s_tok,
                              const int* s_pos, const int* s_done, const int* s_pt, int max_pages,
                              const float* s_invt, const long long* s_seed, int* tokens,
                              int* positions, int* ctx, long long* slots, int* pt, float* invt,
                              long long* seeds, long long* state_rows, int state_spare,
                              cudaStream_t st) {
  if (B == 0) return 0;
  return (int)mb::mb_launch(es::decode_prep_kernel, B, 128, 0, st, rows, B, spare, s_tok, s_pos, s_done, s_pt,
            max_pages, s_invt, s_seed, tokens, positions, ctx, slots, pt, invt, seeds, state_rows,
            state_spare);
}

extern "C" int mb_decode_commit(const int* rows, int B, int spare, const int* tok, const float* lp,
                                const int* experts, int n_moe, int topk, int* s_tok, int* s_pos, int* s_done,
                                int* s_nout, const int* s_maxnew, const int* s_stop, int nstop,
                                int* out_tok, float* out_lp, int max_new, unsigned char* out_exp,
                                const int* s_rec, int max_len, cudaStream_t st) {
  if (B == 0) return 0;
  return (int)mb::mb_launch(es::decode_commit_kernel, B, 128, 0, st, rows, B, spare, tok, lp, experts, n_moe, topk, s_tok,
            s_pos, s_done, s_nout, s_maxnew, s_stop, nstop, out_tok, out_lp, max_new, out_exp,
            s_rec, max_len);
}

MB_CHECK_GETTER(mb_checks_engine)
