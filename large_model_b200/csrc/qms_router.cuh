// qms_router.cuh - F32 dot products in the reference's exact summation order (sm_100a).
//
// qms_vec_dot_f32 (src/kernels.c:202-219) keeps two 8-lane FMA accumulators over 16-element
// steps, so element i always lands in lane i % 16 and each lane is a sequential FMA chain.
// It then adds the two accumulators lane-wise and reduces with hsum256:
//   c_m = a0_m + a1_m,  result = ((c0+c4)+(c2+c6)) + ((c1+c5)+(c3+c7)),
// followed by a scalar tail for n % 16 that is a separate multiply and add (no FMA). Sixteen CUDA threads reproduce it bit for bit:
// thread k runs lane k's chain, and shuffles with offsets 8, 4, 2, 1 inside the 16-thread
// group add exactly the pairs above in the same order.
#pragma once

#include "qms_common.cuh"

namespace qms {

// One dot of length n, computed by the 16 threads of a group (k = lane within the group,
// 0..15). All 32 lanes of the warp must call it. The result is valid in the group's k == 0.
__device__ __forceinline__ float dot_f32_exact16(const float *__restrict__ w, const float *__restrict__ x,
                                                 int64_t n, int k) {
    float acc = 0.0f;
    const int64_t n16 = n / 16 * 16;
#pragma unroll 8
    for (int64_t i = k; i < n16; i += 16) acc = __fmaf_rn(w[i], x[i], acc);
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8, 16));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 16));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2, 16));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1, 16));
    if (k == 0)
        for (int64_t i = n16; i < n; i++) acc = __fadd_rn(acc, __fmul_rn(w[i], x[i]));
    return acc;
}

// y[t][r] for every (row, token) pair; 16 threads per pair.
static __global__ void k_matvec_f32_exact(const float *__restrict__ w, int64_t rows, int64_t cols,
                                   const float *__restrict__ x, int T, float *__restrict__ y) {
    const int64_t pair = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const int k = threadIdx.x & 15;
    const bool valid = pair < rows * T;
    const int64_t r = valid ? pair % rows : 0, t = valid ? pair / rows : 0;
    const float v = dot_f32_exact16(w + r * cols, x + t * cols, cols, k);
    if (valid && k == 0) y[t * rows + r] = v;
}

inline int launch_matvec_f32_exact(const float *w, int64_t rows, int64_t cols, const float *x, int T, float *y,
                                   cudaStream_t s) {
    const int64_t threads = rows * T * 16;
    k_matvec_f32_exact<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(w, rows, cols, x, T, y);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

}  // namespace qms
