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
                 float alpha, int bn, int* err, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
