// Shared device helpers for the sm_100a kernel library: mbarriers, TMA (plain loads only),
// tcgen05 (TMEM alloc / MMA / commit / ld) and bounded waits that report an error status
// instead of trapping.
//
// Design rules enforced here:
//  * Every spin wait has an iteration limit. On expiry the wait returns false and the caller
//    records a code in the library's device error word (read by the host via
//    miles_b200.ops.check_device_error()). No __trap(), no device assert.
//  * TMA loads are plain per-CTA loads (no cluster-wide broadcast qualifier in any form), so
//    this code is safe in multi-GPU jobs and never broadcasts a peer's memory through TMA.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define MB_DEVICE __device__ __forceinline__

#include <cstdlib>
#include <utility>

namespace mb {

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel of the library is launched with programmatic
// stream serialization; inside, `pdl_trigger()` lets the next kernel in the stream start
// launching immediately and `pdl_wait()` (griddepcontrol.wait) blocks until the previous kernel
// has completed and its memory is visible. The next kernel's launch latency and prologue
// (barrier init, TMEM allocation, descriptor prefetch) therefore overlap the previous kernel's
// tail. Kernels call pdl_wait() before touching any input. MB_NO_PDL=1 disables it.
// ---------------------------------------------------------------------------------------------
MB_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MB_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = std::getenv("MB_NO_PDL") == nullptr;
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t mb_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------------------------
// Error reporting
// ---------------------------------------------------------------------------------------------
// Codes: 1 = GEMM pipeline wait timed out, 2 = attention wait timed out, 3 = comm flag timed out.
// `err` is a device int owned by the caller (one per device, see miles_b200/ops/_lib.py); the
// first error code sticks until the host clears it.
MB_DEVICE void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Checked builds (-DMB_CHECKS=1, the miles_b200._C_checked extension): MB_GUARD(cond, code)
// evaluates `cond`; when it is false the code is recorded in this translation unit's check word
// (the first code sticks) and the caller skips the guarded access instead of faulting. In the
// regular build MB_GUARD is the constant `true` and `cond` is not evaluated. MB_CHECK_GETTER
// defines the C function that copies (and optionally clears) this unit's check word.
#ifdef MB_CHECKS
static __device__ int mb_check_word;
MB_DEVICE bool mb_guard(bool ok, int code) {
  if (!ok) atomicCAS(&mb_check_word, 0, code);
  return ok;
}
#define MB_GUARD(cond, code) ::mb::mb_guard((cond), (code))
#define MB_CHECK_GETTER(fn)                                                                      \
  extern "C" int fn(int* out, int clear) {                                                       \
    if (cudaMemcpyFromSymbol(out, ::mb::mb_check_word, sizeof(int)) != cudaSuccess) return -1;   \
    const int zero = 0;                                                                          \
    if (clear && cudaMemcpyToSymbol(::mb::mb_check_word, &zero, sizeof(int)) != cudaSuccess)     \
      return -1;                                                                                 \
    return 0;                                                                                    \
  }
#else
#define MB_GUARD(cond, code) true
#define MB_CHECK_GETTER(fn)                \
  extern "C" int fn(int* out, int clear) { \
    (void)clear;                           \
    *out = 0;                              \
    return 0;                              \
  }
#endif

// Spin limit for mbarrier waits: with the suspend hint of mbar_try_wait, 1<<22 polls is about
// 2 s of wall time, far beyond any legitimate stall.
constexpr uint32_t kSpinLimit = 1u << 22;

// Host: 2-D row-major [rows, cols] tensor map with a {box_cols, box_rows} box and 128-byte
// swizzle (defined in gemm_sm100.cu). Returns 0 on success.
int make_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, uint64_t rows,
             uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows);

// ---------------------------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------------------------
MB_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

MB_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
MB_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

MB_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

MB_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

MB_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One poll; a waiting thread may be suspended for up to kSuspendHintNs before it returns, which
// bounds the wall time of kSpinLimit polls (about 2 s) independently of the hardware default.
constexpr uint32_t kSuspendHintNs = 500;
MB_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

MB_DEVICE uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wall-clock limit of one bounded wait (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Bounded wait; returns false (and records `code`) if the phase did not complete within
// kWaitLimitNs of wall time (or kSpinLimit polls, whichever comes first).
MB_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && global_ns() - t0 > kWaitLimitNs) break;
  }
  report_error(err, code);
  return false;
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled, plain per-CTA loads)
// ---------------------------------------------------------------------------------------------
MB_DEVICE void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into this CTA's shared memory. x = innermost coordinate (elements); callers
// guarantee x * elem_size is a multiple of 16 bytes.
MB_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
MB_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
MB_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
MB_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
MB_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
MB_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 in, f32 accumulate).
MB_DEVICE void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f8f6f4 (e4m3 in, f32 accumulate).
MB_DEVICE void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread have completed.
MB_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

MB_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp receives lane (base_lane + i).
MB_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
MB_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns.
MB_DEVICE void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// ---------------------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 format): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), base_offset [49,52), lbo_mode [52], layout [61,64).
// Layout 2 = 128-byte swizzle.
MB_DEVICE uint64_t make_sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and f32 accumulation.
// c_format [4,6)=1 (f32); a_format [7,10)=1 (bf16); b_format [10,13)=1 (bf16);
// a_major [15], b_major [16] (0 = K-major, 1 = MN-major); N>>3 at [17,23); M>>4 at [24,29).
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor for kind::f8f6f4 with e4m3 A/B (format code 0), f32 accumulation.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------------------------
MB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
MB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

MB_DEVICE uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace mb
