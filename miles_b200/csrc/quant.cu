// Quantization kernels (sm_100a) used by the weight refit and the offline converters.
//
//  * block fp8 (e4m3), 2-D blocks of bm x bn (default 128x128): scale = absmax / 448 (fp32 or
//    rounded up to a power of two for ue8m0), y = sat(x / scale); returns the inverse scales
//    [ceil(M/bm), ceil(N/bn)] ("weight_scale_inv").
//  * token-group fp8 (1 x 128 activation groups).
//  * int4 fake quantization (quantize + dequantize in the input dtype) over groups of
//    `group` elements along rows, symmetric (scale = absmax/7) or asymmetric
//    (scale = (max-min)/15, zero = clamp(-round(min/scale), 0, 15)); q, scale, zero out.
//  * NVFP4: e2m1 values packed two per byte, e4m3 scale per 16 elements, fp32 global scale.
//  * MXFP8: e4m3 values with one ue8m0 (power-of-two) scale per 32 elements.
//
// Reference roles replaced: utils/fp8_kernel.py:24-79 (Triton block cast),
// kernels/int4_qat/fake_int4_quant_cuda.cu:29-367, quantizer_nvfp4.py:146-254,
// quantizer_mxfp8.py:84-97 (sglang mxfp8_group_quantize).
#include "common.cuh"
#include <cuda_fp8.h>

namespace mb {

constexpr float FP8_MAX = 448.f;

MB_DEVICE float ue8m0_round_up(float s) {
  // smallest power of two >= s (exact: exponent manipulation of the float bits)
  if (s <= 0.f) return 1.f;
  uint32_t b = __float_as_uint(s);
  const uint32_t mant = b & 0x7fffffu;
  uint32_t e = (b >> 23) & 0xffu;
  if (mant) e += 1;
  return __uint_as_float(e << 23);
}

// One CTA (256 threads) per (bm x bn) block. Two passes: absmax, then scale + convert.
__global__ void fp8_block_cast_kernel(const __nv_bfloat16* __restrict__ x, int M, int N, int bm,
                                      int bn, __nv_fp8_e4m3* __restrict__ y,
                                      float* __restrict__ scale_inv, int ue8m0) {
  const int br = blockIdx.y, bc = blockIdx.x;
  const int r0 = br * bm, c0 = bc * bn;
  const int rows = min(bm, M - r0), cols = min(bn, N - c0);
  float amax = 0.f;
  for (int i = threadIdx.x; i < rows * cols; i += blockDim.x) {
    const int r = i / cols, c = i % cols;
    amax = fmaxf(amax, fabsf(__bfloat162float(x[(long long)(r0 + r) * N + c0 + c])));
  }
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = fmaxf(red[0], 1e-12f);
  float s = amax / FP8_MAX;
  if (ue8m0) s = ue8m0_round_up(s);
  if (threadIdx.x == 0) scale_inv[br * gridDim.x + bc] = s;
  const float inv = 1.f / s;
  for (int i = threadIdx.x; i < rows * cols; i += blockDim.x) {
    const int r = i / cols, c = i % cols;
    const long long idx = (long long)(r0 + r) * N + c0 + c;
    const float v = fminf(fmaxf(__bfloat162float(x[idx]) * inv, -FP8_MAX), FP8_MAX);
    y[idx] = __nv_fp8_e4m3(v);
  }
}

// Fast path of the 128 x 128 block cast (full blocks, 16-byte aligned rows): thread t of the
// CTA holds row t / 2, columns (t & 1) * 64 .. +63 of the block in registers (eight 16-byte
// loads), so the block is read once; same scale and conversion as fp8_block_cast_kernel.
__global__ void __launch_bounds__(256) fp8_block_cast128_kernel(
    const __nv_bfloat16* __restrict__ x, int N, __nv_fp8_e4m3* __restrict__ y,
    float* __restrict__ scale_inv, int ue8m0) {
  const int br = blockIdx.y, bc = blockIdx.x;
  const int r = threadIdx.x >> 1, c0 = (threadIdx.x & 1) * 64;
  const long long base = (long long)(br * 128 + r) * N + bc * 128 + c0;
  uint4 raw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) raw[i] = reinterpret_cast<const uint4*>(x + base)[i];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__bfloat162float(h[j])));
  }
  __shared__ float red[8];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  amax = fmaxf(m, 1e-12f);
  float sc = amax / FP8_MAX;
  if (ue8m0) sc = ue8m0_round_up(sc);
  if (threadIdx.x == 0) scale_inv[br * gridDim.x + bc] = sc;
  const float inv = 1.f / sc;
  uint4 out[4];
  uint8_t* ob = reinterpret_cast<uint8_t*>(out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_fp8_e4m3 e(fminf(fmaxf(__bfloat162float(h[j]) * inv, -FP8_MAX), FP8_MAX));
      ob[i * 8 + j] = *reinterpret_cast<const uint8_t*>(&e);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(y) + base);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = out[i];
}

// 1 x group activation quantization: one warp per (row, group).
__global__ void fp8_group_cast_kernel(const __nv_bfloat16* __restrict__ x, long long M, int N,
                                      int group, __nv_fp8_e4m3* __restrict__ y,
                                      float* __restrict__ scale, int ue8m0) {
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int gpr = (N + group - 1) / group;
  if (w >= M * gpr) return;
  const long long r = w / gpr;
  const int g = (int)(w % gpr);
  const int c0 = g * group, c1 = min(N, c0 + group);
  float amax = 0.f;
  for (int c = c0 + lane; c < c1; c += 32) amax = fmaxf(amax, fabsf(__bfloat162float(x[r * N + c])));
  amax = fmaxf(warp_max(amax), 1e-12f);
  float s = amax / FP8_MAX;
  if (ue8m0) s = ue8m0_round_up(s);
  if (lane == 0) scale[r * gpr + g] = s;
  const float inv = 1.f / s;
  for (int c = c0 + lane; c < c1; c += 32)
    y[r * N + c] = __nv_fp8_e4m3(fminf(fmaxf(__bfloat162float(x[r * N + c]) * inv, -FP8_MAX), FP8_MAX));
}

// int4 fake quantization along rows in groups of `group` columns; one warp per (row, group).
template <typename T>
__global__ void int4_fake_quant_kernel(const T* __restrict__ x, long long M, int N, int group,
                                       int sym, T* __restrict__ q, T* __restrict__ scale,
                                       T* __restrict__ zero) {
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int gpr = N / group;
  if (w >= M * gpr) return;
  const long long r = w / gpr;
  const int c0 = (int)(w % gpr) * group;
  float mx = -INFINITY, mn = INFINITY, am = 0.f;
  for (int c = lane; c < group; c += 32) {
    const float v = (float)x[r * N + c0 + c];
    mx = fmaxf(mx, v);
    mn = fminf(mn, v);
    am = fmaxf(am, fabsf(v));
  }
  mx = warp_max(mx);
  mn = -warp_max(-mn);
  am = warp_max(am);
  float s, z = 0.f;
  if (sym) {
    s = fmaxf(am / 7.f, 1e-8f);
  } else {
    s = fmaxf((mx - mn) / 15.f, 1e-8f);
    z = fminf(fmaxf(-rintf(mn / s), 0.f), 15.f);
  }
  for (int c = lane; c < group; c += 32) {
    const long long idx = r * N + c0 + c;
    const float v = (float)x[idx];
    float qq;
    if (sym) qq = fminf(fmaxf(rintf(v / s), -8.f), 7.f);
    else qq = fminf(fmaxf(rintf(v / s) + z, 0.f), 15.f);
    q[idx] = (T)qq;
  }
  if (lane == 0) {
    scale[r * gpr + c0 / group] = (T)s;
    if (zero) zero[r * gpr + c0 / group] = (T)z;
  }
}

// e2m1 magnitude code of |v| (already scaled): representable values 0,.5,1,1.5,2,3,4,6;
// round to nearest with ties to even code.
MB_DEVICE uint32_t e2m1_code(float v) {
  // midpoints 0.25 .75 1.25 1.75 2.5 3.5 5 between consecutive codes; a tie goes to the even code
  const float a = fabsf(v);
  uint32_t c;
  if (a <= 0.25f) c = 0;
  else if (a < 0.75f) c = 1;
  else if (a <= 1.25f) c = 2;
  else if (a < 1.75f) c = 3;
  else if (a <= 2.5f) c = 4;
  else if (a < 3.5f) c = 5;
  else if (a <= 5.f) c = 6;
  else c = 7;
  return c | ((v < 0.f && c) ? 8u : 0u);
}

// NVFP4: groups of 16 along rows; block scale (e4m3) = absmax / 6 / global_scale.
__global__ void nvfp4_quant_kernel(const __nv_bfloat16* __restrict__ x, long long M, int N,
                                   float global_scale, uint8_t* __restrict__ packed,
                                   __nv_fp8_e4m3* __restrict__ bscale) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int gpr = N / 16;
  if (g >= M * gpr) return;
  const long long r = g / gpr;
  const int c0 = (int)(g % gpr) * 16;
  float v[16], am = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = __bfloat162float(x[r * N + c0 + i]);
    am = fmaxf(am, fabsf(v[i]));
  }
  const __nv_fp8_e4m3 sc(fminf(am / 6.f / global_scale, FP8_MAX));
  bscale[g] = sc;
  const float s = float(sc) * global_scale;
  const float inv = s > 0.f ? 1.f / s : 0.f;
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const uint32_t lo = e2m1_code(v[i] * inv), hi = e2m1_code(v[i + 1] * inv);
    packed[(r * N + c0 + i) / 2] = (uint8_t)(lo | (hi << 4));
  }
}

// MXFP8: groups of 32 along rows, ue8m0 scale (stored as the biased exponent byte).
__global__ void mxfp8_quant_kernel(const __nv_bfloat16* __restrict__ x, long long M, int N,
                                   __nv_fp8_e4m3* __restrict__ y, uint8_t* __restrict__ sexp) {
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int gpr = N / 32;
  if (w >= M * gpr) return;
  const long long r = w / gpr;
  const int c = (int)(w % gpr) * 32 + lane;
  const float v = __bfloat162float(x[r * N + c]);
  const float am = fmaxf(warp_max(fabsf(v)), 1e-30f);
  const float s = ue8m0_round_up(am / FP8_MAX);
  if (lane == 0) sexp[w] = (uint8_t)((__float_as_uint(s) >> 23) & 0xff);
  y[r * N + c] = __nv_fp8_e4m3(fminf(fmaxf(v / s, -FP8_MAX), FP8_MAX));
}

}  // namespace mb

using namespace mb;

extern "C" int mb_fp8_block_cast(const void* x, int M, int N, int bm, int bn, void* y,
                                 float* scale_inv, int ue8m0, cudaStream_t st) {
  if (M == 0 || N == 0) return 0;
  dim3 grid((N + bn - 1) / bn, (M + bm - 1) / bm);
  if (bm == 128 && bn == 128 && M % 128 == 0 && N % 128 == 0 &&
      reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0) {
    fp8_block_cast128_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, N, (__nv_fp8_e4m3*)y,
                                                    scale_inv, ue8m0);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  fp8_block_cast_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, M, N, bm, bn,
                                               (__nv_fp8_e4m3*)y, scale_inv, ue8m0);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_fp8_group_cast(const void* x, long long M, int N, int group, void* y,
                                 float* scale, int ue8m0, cudaStream_t st) {
  if (M == 0) return 0;
  const long long warps = M * ((N + group - 1) / group);
  fp8_group_cast_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      (const __nv_bfloat16*)x, M, N, group, (__nv_fp8_e4m3*)y, scale, ue8m0);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// dtype: 0 = bf16, 1 = fp16, 2 = fp32
extern "C" int mb_int4_fake_quant(const void* x, long long M, int N, int group, int sym, int dtype,
                                  void* q, void* scale, void* zero, cudaStream_t st) {
  if (M == 0) return 0;
  if (N % group) return -1;
  const long long warps = M * (N / group);
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (dtype == 0)
    int4_fake_quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        (const __nv_bfloat16*)x, M, N, group, sym, (__nv_bfloat16*)q, (__nv_bfloat16*)scale,
        (__nv_bfloat16*)zero);
  else if (dtype == 1)
    int4_fake_quant_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, M, N, group, sym,
                                                         (__half*)q, (__half*)scale, (__half*)zero);
  else
    int4_fake_quant_kernel<float><<<grid, 256, 0, st>>>((const float*)x, M, N, group, sym,
                                                        (float*)q, (float*)scale, (float*)zero);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_nvfp4_quant(const void* x, long long M, int N, float global_scale, void* packed,
                              void* bscale, cudaStream_t st) {
  if (M == 0) return 0;
  if (N % 16) return -1;
  const long long groups = M * (N / 16);
  nvfp4_quant_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, st>>>(
      (const __nv_bfloat16*)x, M, N, global_scale, (uint8_t*)packed, (__nv_fp8_e4m3*)bscale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int mb_mxfp8_quant(const void* x, long long M, int N, void* y, void* sexp,
                              cudaStream_t st) {
  if (M == 0) return 0;
  if (N % 32) return -1;
  const long long warps = M * (N / 32);
  mxfp8_quant_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      (const __nv_bfloat16*)x, M, N, (__nv_fp8_e4m3*)y, (uint8_t*)sexp);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
