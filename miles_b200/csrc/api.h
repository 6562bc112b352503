// C ABI of the sm_100a kernel library (implemented in the .cu files of this directory).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int mb_gemm_bf16(const void* a, long long a_rows, long long a_cols, long long lda, bool a_mn,
                 const void* b, long long b_rows, long long b_cols, long long ldb, bool b_mn,
                 void* c, long long ldc, int M, int N, int K, int mode, const int* group_offsets,
                 int num_groups, int b_rows_per_group, long long c_group_stride, int epi,
                 float alpha, int bn, const int* group_counts, int* err, cudaStream_t stream);
// Block-scaled fp8 GEMM and 1 x 128 activation quantisation (gemm_fp8_sm100.cu).
int mb_fp8_act_quant(const void* x, long long ldx, int M, int K, void* q, float* s, long long lds,
                     const int* offsets, const int* counts, int E, cudaStream_t st);
int mb_gemm_fp8(const void* a, long long a_rows, long long lda, const float* sa, long long lds,
                const void* b, long long b_rows, long long ldb, const float* sb, void* c,
                long long ldc, int M, int N, int K, int mode, const int* group_offsets,
                const int* group_counts, int num_groups, int b_rows_per_group, int epi,
                int swiglu_f, void* c2, long long ldc2, int bn, int* err, cudaStream_t stream);
int mb_gemm_bf16_swiglu(const void* a, long long a_rows, long long lda, const void* b,
                        long long b_rows, long long ldb, void* out, long long ldo, void* gu,
                        long long ldgu, int M, int F, int K, int mode, const int* group_offsets,
                        int num_groups, int bn, const int* group_counts, int* err,
                        cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
extern "C" {
#endif
int mb_rmsnorm_fwd(const void* x, const void* res, const void* w, void* h_out, void* y, float* rstd,
                   int rows, int H, float eps, cudaStream_t st);
int mb_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, const void* dres,
                   void* dx, float* dw_part, int nparts, float* dw_f32, void* dw_bf16, int accumulate,
                   int rows, int H, cudaStream_t st);
int mb_qk_norm_rope_fwd(const void* qkv, long long ld_in, const void* qw, const void* kw,
                        const int* pos, const float* cos_t, const float* sin_t, void* q_out,
                        void* k_out, void* v_out, const long long* slot, long long ld_kv,
                        float* rstd, int T, int nq, int nkv, float eps, int use_norm,
                        cudaStream_t st);
int mb_qk_norm_rope_bwd(const void* dq, const void* dk, const void* dv, const void* qkv,
                        long long ld_in, const void* qw, const void* kw, const int* pos,
                        const float* cos_t, const float* sin_t, const float* rstd, void* dqkv,
                        float* dw_part, int nparts, float* dw_out, int T, int nq, int nkv,
                        int use_norm, cudaStream_t st);
int mb_swiglu_fwd(const void* gu, void* out, long long T, int I, const int* nrows, cudaStream_t st);
int mb_swiglu_bwd(const void* gu, const void* dout, void* dgu, long long T, int I, const int* nrows,
                  cudaStream_t st);
int mb_router_fwd(const float* logits, const float* bias, const int* idx_in, int* idx_out,
                  float* w_out, int T, int E, int k, int score_fn, int renorm, int n_group,
                  int topk_group, float scale, cudaStream_t st);
int mb_router_bwd(const float* logits, const int* idx, const float* dw, void* dlogits, int T, int E,
                  int k, int score_fn, int renorm, float scale, cudaStream_t st);
int mb_moe_permute_plan(const int* idx, int n, int E, int align, int* hist, int* chunk_base,
                        int* counts, int* offsets, int* dest, cudaStream_t st);
int mb_moe_route_dispatch(const float* logits, const float* bias, const int* idx_in, const void* x,
                          int T, int E, int k, int H, int score_fn, int renorm, int n_group,
                          int topk_group, float scale, int align, int* idx_out, float* w_out,
                          int* counts, int* offsets, int* dest, void* xs, cudaStream_t st);
int mb_moe_zero_pad(const int* counts, const int* offsets, void* buf, int E, int H, cudaStream_t st);
int mb_moe_gather(const void* x, const int* dest, int n, int k, int H, void* xs, int rows, cudaStream_t st);
int mb_moe_gather_bwd(const void* dxs, const int* dest, int T, int k, int H, void* dx,
                      cudaStream_t st);
int mb_moe_combine(const void* ys, const int* dest, const float* w, const void* add, int T, int k,
                   int H, void* y, cudaStream_t st);
int mb_moe_combine_bwd(const void* dy, const void* ys, const int* dest, const float* w, int T,
                       int k, int H, void* dys, float* dw, cudaStream_t st);
int mb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                const int* cu_seqlens, const int* tile_seq, const int* tile_idx, int ntiles,
                long long q_stride, long long k_stride, long long v_stride, long long o_stride,
                int nq, int nkv, int T, float softmax_scale, int* err, cudaStream_t st);
int mb_attn_decode_nsplit(int max_pages);
int mb_attn_decode(const void* q, const void* kc, const void* vc, void* o, const int* page_table,
                   const int* ctx_lens, int B, int max_pages, long long num_slots, int nq, int nkv,
                   float softmax_scale, float* ws_o, float* ws_ml, int* err, cudaStream_t st);
int mb_fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
              const int* cu_seqlens, const int* tile_seq, const int* tile_idx, int ntiles,
              long long q_stride, long long k_stride, long long v_stride, long long o_stride,
              int nq, int nkv, int T, float softmax_scale, int* err, cudaStream_t st);
int mb_fa_decode(const void* q, const void* kc, const void* vc, void* o, const int* page_table,
                 const int* ctx_lens, int B, int max_pages, long long num_slots, int nq, int nkv,
                 float softmax_scale, float* ws_o, float* ws_ml, int* err, cudaStream_t st);
int mb_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, float* delta, void* dq, void* dk, void* dv,
                const int* cu_seqlens, const int* blk_seq, const int* blk_idx, int nblocks,
                long long q_stride, long long k_stride, long long v_stride, long long o_stride,
                long long do_stride, long long dq_stride, long long dk_stride,
                long long dv_stride, int nq, int nkv, int T, float softmax_scale, int* err,
                cudaStream_t st);
int mb_fa_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse,
              const float* delta, void* dq, void* dk, void* dv, const int* cu_seqlens,
              const int* tile_seq, const int* tile_idx, int ntiles, long long q_stride,
              long long k_stride, long long v_stride, long long do_stride, long long dq_stride,
              long long dk_stride, long long dv_stride, int nq, int nkv, int T,
              float softmax_scale, int* err, cudaStream_t st);
int mb_logprob_fwd(const float* logits, long long ld, const int* target, int n, int V,
                   float inv_temp, float* logp, float* ent, float* lse, cudaStream_t st);
// Vocabulary-parallel log-prob: per-slice softmax statistics part [4][n] = {m, s, sz, target
// logit or 0} of logits [n, V] holding vocabulary ids [lo, lo + V); then the rank-order combine of
// `world` parts [world][4][n] into logp / ent / lse.
int mb_logprob_part(const float* logits, long long ld, const int* target, int lo, int n, int V,
                    float inv_temp, float* part, cudaStream_t st);
int mb_logprob_combine(const float* parts, int world, int n, float* logp, float* ent, float* lse,
                       cudaStream_t st);
int mb_logprob_bwd(const float* logits, long long ld, const int* target, int n, int V,
                   float inv_temp, const float* lse, const float* g_lp, const float* g_ent,
                   const float* ent, void* dlogits, long long ldd, cudaStream_t st);
int mb_sample(const float* logits, long long ld, int n, int V, const float* inv_temps,
              const unsigned long long* seeds, const int* positions, int* tokens, float* logp,
              const float* thr, cudaStream_t st);
int mb_policy_loss(const float* logp, const float* old_logp, const float* adv, const float* weight,
                   const float* rollout_logp, const float* ref_logp, float* dlogp, float* pg_out,
                   float* part, float* metrics, int n, float eps, float eps_hi, float eps_c,
                   float tis_lo, float tis_hi, float kl_coef, int kl_type, int use_tis,
                   cudaStream_t st);
int mb_gae(const float* rewards, const float* values, const int* cu, int B, float gamma, float lam,
           float* adv, float* ret, cudaStream_t st);
int mb_grpo_adv(const float* r, int ngroups, int gsize, int norm_std, float eps, float* adv,
                cudaStream_t st);
int mb_sqnorm(const void* x, long long n, int is_bf16, float* part, float* out, cudaStream_t st);
int mb_nonfinite(const void* x, long long n, int is_bf16, float* flag, cudaStream_t st);
int mb_adam(void* param, float* master, void* m, void* v, const void* grad, long long n,
            int grad_bf16, int mv_bf16, float lr, float b1, float b2, float eps, float wd, int step,
            const float* sqnorm, float max_norm, float inv_loss_scale, unsigned long long seed,
            const float* skip, cudaStream_t st);
#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
extern "C" {
#endif
int mb_fp8_block_cast(const void* x, int M, int N, int bm, int bn, void* y, float* scale_inv,
                      int ue8m0, cudaStream_t st);
int mb_fp8_group_cast(const void* x, long long M, int N, int group, void* y, float* scale,
                      int ue8m0, cudaStream_t st);
int mb_int4_fake_quant(const void* x, long long M, int N, int group, int sym, int dtype, void* q,
                       void* scale, void* zero, cudaStream_t st);
int mb_nvfp4_quant(const void* x, long long M, int N, float global_scale, void* packed,
                   void* bscale, cudaStream_t st);
int mb_mxfp8_quant(const void* x, long long M, int N, void* y, void* sexp, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Allocation-free decode attention (no counterpart in the reference implementation; an
// addition of this library). Same inputs/outputs as mb_attn_decode, but the split-KV workspace
// is a fixed 4 MiB device array inside the library instead of caller memory, for callers that
// cannot allocate device memory. Returns -9 if the call would need more than that workspace,
// -10/-11 on device / symbol lookup failure. The first call on a device resolves the array's
// address (do it before any stream capture); concurrent calls on unordered streams race on the
// shared workspace.
#ifdef __cplusplus
extern "C" {
#endif
#define MB_NOALLOC_TOO_LARGE (-9)
int mb_attn_decode_noalloc(const void* q, const void* kc, const void* vc, void* o,
                           const int* page_table, const int* ctx_lens, int B, int max_pages,
                           long long num_slots, int nq, int nkv, float softmax_scale,
                           cudaStream_t st);
// Error word of the allocation-free entry point on the current device (0 = none, 2 = a bounded
// wait inside the kernel ran out and the output is incomplete); reading it clears it.
int mb_attn_decode_noalloc_error(int* code, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Symmetric peer memory and in-kernel collectives (symm.cu) and the fused GEMM + all-reduce
// GEMM half (gemm_sm100.cu, epilogue 5).
#ifdef __cplusplus
extern "C" {
#endif
int mb_ipc_handle_size();
int mb_symm_malloc(long long bytes, long long* ptr_out);
int mb_symm_free(long long ptr);
int mb_ipc_get_handle(long long ptr, void* handle_out);
int mb_ipc_get_handle_range(long long ptr, void* handle_out, long long* offset_out);
int mb_ipc_open(const void* handle, long long* ptr_out);
int mb_ipc_close(long long ptr);
int mb_symm_barrier(const long long* flag_ptrs, int* my_flags, int* ctl, int rank, int world,
                    long long timeout_ns, int* err, cudaStream_t st);
int mb_symm_allreduce(const long long* flag_ptrs, const long long* stage_ptrs, int* my_flags,
                      int* ctl, const void* my_stage, long long cap, const void* src, int rows,
                      int H, int rank, int world, const void* res, const void* norm_w,
                      float eps, void* out, void* h_out, float* rstd, long long timeout_ns,
                      int* err, cudaStream_t st);
int mb_symm_copy(const void* src, void* dst, long long bytes, cudaStream_t st);
// Fused gradient reduce-scatter + cast/scale + squared norm over peer memory: out[0, n) =
// bf16(scale * sum_r g_r[lo, lo + n)), *sq_out = sum of the squares of out. n, lo multiples of 8,
// pointers 16-byte aligned, partial >= 592 floats, counter one zeroed int.
int mb_grad_rs(const long long* g_ptrs, int world, long long lo, long long n, float scale,
               void* out, float* partial, int* counter, float* sq_out, cudaStream_t st);
int mb_fp8_block_dequant(const void* q, const float* s, int M, int N, int bm, int bn, void* out,
                         cudaStream_t st);
int mb_gemm_bf16_peer(const void* a, long long a_rows, long long a_cols, long long lda, bool a_mn,
                      const void* b, long long b_rows, long long b_cols, long long ldb, bool b_mn,
                      int M, int N, int K, const long long* peer_ptrs, int npeers, long long ldc,
                      const int* par_word, long long par_stride, int scatter_rows, int bn, int* err,
                      cudaStream_t stream);
int mb_symm_collective(int kind, const long long* flag_ptrs, const long long* stage_ptrs,
                       int* my_flags, int* ctl, const void* my_stage, long long cap,
                       const void* src, int rows, int H, int rank, int world, const void* res,
                       const void* norm_w, float eps, void* out, void* h_out, float* rstd,
                       long long timeout_ns, int* err, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Expert-parallel dispatch / combine over symmetric peer memory (moe_ep.cu).
#ifdef __cplusplus
extern "C" {
#endif
int mb_ep_publish(const int* counts, int E, int E_local, int rank, int world,
                  const long long* table_ptrs, cudaStream_t st);
int mb_ep_offsets(const int* table, int world, int E_local, int align, int* offsets, int* counts,
                  int* base, long long cap, int* err, cudaStream_t st);
int mb_ep_dispatch(const void* x, const int* idx, const int* dest_g, const int* off_g, int T,
                   int k, int H, int E_local, int rank, int world, const long long* base_ptrs,
                   const long long* xs_ptrs, long long cap, int* pos, int* err, cudaStream_t st);
int mb_ep_combine(const long long* ys_ptrs, int world, const int* idx, const int* pos,
                  const float* w, const void* add, int T, int k, int H, int E_local, void* y,
                  void* saved, cudaStream_t st);
int mb_ep_combine_bwd(const void* dy, const void* saved, const int* idx, const int* pos,
                      const float* w, int T, int k, int H, int E_local, int world,
                      const long long* dys_ptrs, float* dw, cudaStream_t st);
int mb_ep_gather_bwd(const long long* dxs_ptrs, int world, const int* idx, const int* pos, int T,
                     int k, int H, int E_local, void* dx, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Gated DeltaNet decode step (gdn.cu).
#ifdef __cplusplus
extern "C" {
#endif
int mb_gdn_decode(const float* q, const float* k, const float* v, const float* beta,
                  const float* g, const long long* rows, float* S, float* out, int B, int nv,
                  int dk, int dv, float scale, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Absorbed MLA decode over the paged latent cache (mla_decode.cu).
#ifdef __cplusplus
extern "C" {
#endif
int mb_mla_decode(const float* q_lat, const float* q_pe, const void* cache, long long row_stride,
                  const int* page_table, int max_pages, const int* ctx_lens, const float* bias,
                  long long bias_stride, int B, int nh, int r, int dr, float scale, float* out,
                  cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Device-resident decode loop state (engine_step.cu): gather a bucket's inputs from the
// sequence slots, and commit the sampled tokens back into them.
#ifdef __cplusplus
extern "C" {
#endif
int mb_decode_prep(const int* rows, int B, int spare, const int* s_tok, const int* s_pos,
                   const int* s_done, const int* s_pt, int max_pages, const float* s_invt,
                   const long long* s_seed, int* tokens, int* positions, int* ctx,
                   long long* slots, int* pt, float* invt, long long* seeds,
                   long long* state_rows, int state_spare, cudaStream_t st);
int mb_decode_commit(const int* rows, int B, int spare, const int* tok, const float* lp,
                     const int* experts, int n_moe, int topk, int* s_tok, int* s_pos, int* s_done, int* s_nout,
                     const int* s_maxnew, const int* s_stop, int nstop, int* out_tok,
                     float* out_lp, int max_new, unsigned char* out_exp, const int* s_rec,
                     int max_len, cudaStream_t st);
#ifdef __cplusplus
}
#endif

// Virtual-memory arenas (vmm.cu): reserved device address ranges with physical memory mapped in
// and out (addresses stay fixed across release / resume).
#ifdef __cplusplus
extern "C" {
#endif
int mb_vmm_granularity(int device, size_t* gran);
int mb_vmm_reserve(size_t bytes, unsigned long long* ptr);
int mb_vmm_free(unsigned long long ptr, size_t bytes);
int mb_vmm_map(unsigned long long ptr, size_t bytes, int device, unsigned long long* handle);
int mb_vmm_unmap(unsigned long long ptr, size_t bytes, unsigned long long handle);
int mb_host_register(void* ptr, size_t bytes);
int mb_host_unregister(void* ptr);
#ifdef __cplusplus
}
#endif

// Checked-build guard words (MB_GUARD in common.cuh; always 0 in the regular build).
#ifdef __cplusplus
extern "C" {
#endif
int mb_checks_moe(int* out, int clear);
int mb_checks_engine(int* out, int clear);
#ifdef __cplusplus
}
#endif
