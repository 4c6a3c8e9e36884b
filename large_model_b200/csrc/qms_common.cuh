// qms_common.cuh - shared helpers of libqms_cuda (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/qms_cuda.h"

// ---- error reporting ------------------------------------------------------------------------

namespace qms {

void set_error(const char *fmt, ...);
void clear_error();

}  // namespace qms

#define QMS_CK(call)                                                                          \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) {                                                              \
            qms::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
            return QMS_CUDA_ECUDA;                                                            \
        }                                                                                     \
    } while (0)

#define QMS_REQUIRE(cond, code, ...)     \
    do {                                 \
        if (!(cond)) {                   \
            qms::set_error(__VA_ARGS__); \
            return (code);               \
        }                                \
    } while (0)

namespace qms {

// ---- repacked Q4_0 rows ---------------------------------------------------------------------
// A ggml Q4_0 row is nb blocks of {f16 d; u8 qs[16]} (18 bytes, not 16-byte aligned). On the
// device each row is stored as its nibble plane (nb x 16 bytes: block b at 16*b, so one 128-bit
// load fetches a whole block) followed by its scale plane (nb halves), padded to 16 bytes.
// The bytes and their meaning are unchanged; only their order differs.
__host__ __device__ inline size_t q4_row_stride(int nb) {
    return (size_t)nb * 16 + (((size_t)nb * 2 + 15) & ~(size_t)15);
}

// ---- device helpers -------------------------------------------------------------------------

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// 128-bit streaming load of read-only weights: not kept in L1, 256-byte L2 fetch granularity.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint16_t ld_stream2(const void *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Integer dot of one Q4_0 block: sum_j nib_j * q_j over 32 elements. Element j < 16 is the low
// nibble of qs[j], element j >= 16 the high nibble of qs[j-16] (ggml Q4_0); word m of the
// nibble plane holds qs[4m..4m+3], activation words m and m+4 hold q[4m..] and q[16+4m..].
__device__ __forceinline__ int q4_block_isum(uint4 nib, const int4 xa0, const int4 xa1) {
    const uint32_t m = 0x0F0F0F0Fu;
    int s = 0;
    s = __dp4a((int)(nib.x & m), xa0.x, s);
    s = __dp4a((int)(nib.y & m), xa0.y, s);
    s = __dp4a((int)(nib.z & m), xa0.z, s);
    s = __dp4a((int)(nib.w & m), xa0.w, s);
    s = __dp4a((int)((nib.x >> 4) & m), xa1.x, s);
    s = __dp4a((int)((nib.y >> 4) & m), xa1.y, s);
    s = __dp4a((int)((nib.z >> 4) & m), xa1.z, s);
    s = __dp4a((int)((nib.w >> 4) & m), xa1.w, s);
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The reference's per-32 quantiser (src/kernels.c:34-53) for one block held one value per
// lane: d = amax/127 (IEEE division), id = 1/d (0 when d == 0), q = round-half-even(x*id).
// fmaxf over |x| is order-independent, so the warp reduction gives the reference's amax.
struct Q8Lane {
    int q;      // this lane's int8 value
    float d;    // block scale
    int sum;    // sum of the block's 32 q values
    int sum_lo; // sum of q[0..15]
};

__device__ __forceinline__ Q8Lane quantize_lane(float x) {
    const float amax = warp_max(fabsf(x));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    Q8Lane r;
    r.q = __float2int_rn(__fmul_rn(x, id));
    r.d = d;
    r.sum = warp_sum_i(r.q);
    const int lane = threadIdx.x & 31;
    r.sum_lo = warp_sum_i(lane < 16 ? r.q : 0);
    return r;
}

// ---- release / acquire atomics (gpu scope) -------------------------------------------------
// A release add publishes every write this thread has made and, through a preceding barrier
// (__syncwarp / __syncthreads), every write of the threads that took part in it; an acquire read
// (or acq_rel add) makes those writes visible to the reader. No separate membar stalls the thread.
__device__ __forceinline__ void red_add_release(int *p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int atom_add_acq_rel(int *p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- flagged words ----------------------------------------------------------------------------
// A 64-bit word holding 32 data bits and a 32-bit call stamp, written and read with single-copy
// atomic 64-bit accesses: a reader that sees the current stamp sees the data written with it, so
// producers publish with a plain store (no fence, no counter) and consumers poll the data itself.
__device__ __forceinline__ void st_flagged(unsigned long long *p, uint32_t data, uint32_t stamp) {
    const unsigned long long v = ((unsigned long long)stamp << 32) | data;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_flagged(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// ---- packed pairs of fp32 (sm_100 f32x2 instructions): two lanes of work per instruction ---------
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
    return ((unsigned long long)__float_as_uint(v.y) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 f2_from(unsigned long long b) {
    return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32)));
}
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_from(d);
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_from(d);
}
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_from(d);
}

// ---- programmatic dependent launch ---------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace qms
