// qms_trunk.cu - the rest of a Qwen3-MoE token step on B200 (sm_100a): embedding, RMSNorm,
// Q4_0/Q4_1/Q6_K projections against Q8 activations, QK-norm + NEOX RoPE + fp32 KV append,
// causal GQA attention, and the output head with a fused greedy argmax.
//
// Reference: qms_forward and attention() in src/model.c:403-497, 1252-1296; the integer dots of
// src/kernels.c:82-195 (through qms_matmul_n, src/quant.c:128-170); qms_dequant_row (src/quant.c).
//
//   k_embed       one CTA per token: dequantise row ids[t] of token_embd (src/model.c:1273)
//   k_rmsnorm     one CTA per row: double sum of squares, y = (float)(x * inv) * w
//                 (src/model.c:403-409), optionally also the row's Q8 blocks (src/kernels.c:34-53)
//   k_gemv        y = W x for W in repacked Q4_0 / Q4_1 / Q6_K rows (qms_matmul_n's integer path):
//                 lanes of a warp split a row's blocks, dp4a dots per 32-block, fp32 accumulation;
//                 the first rows' weights are loaded before griddepcontrol.wait, so the stream of
//                 a projection starts while the previous kernel finishes. For one token the
//                 prologue RMS-normalises and quantises x itself; the head variant also keeps a
//                 running argmax and the last CTA writes the token (greedy decode on device).
//   k_qk_rope     one warp per head row: QK-norm (RMSNorm over head_dim), NEOX rotation from
//                 host-computed cos/sin tables (the reference's own double-precision angles), and
//                 the K/V append to the fp32 cache (src/model.c:436-462)
//   k_attention   one warp per q head, a CTA per group of heads sharing a KV head; scores in
//                 qms_vec_dot_f32's exact order (sixteen FMA chains + the hsum tree), double
//                 softmax, float accumulation of the V rows. One-token calls split the positions
//                 over CTAs and the last CTA of a head group merges the splits.
#include <math.h>
#include <string.h>

#include <algorithm>

#include "qms_async.cuh"
#include "qms_moe.cuh"
#include "qms_trunk.cuh"

namespace qms {

constexpr int kGemvWarps = 16;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr unsigned kFull = 0xffffffffu;

// ---- load-time repack -------------------------------------------------------------------------------
__global__ void k_repack_q4rows(const uint8_t *__restrict__ src, int64_t rows, int nb, int q1, size_t stride,
                                uint8_t *__restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    const int64_t r = i / nb;
    const int b = (int)(i % nb);
    const int bs = q1 ? 20 : 18;
    const uint16_t *s = reinterpret_cast<const uint16_t *>(src + (size_t)r * nb * bs + (size_t)b * bs);
    uint8_t *row = dst + (size_t)r * stride;
    const uint16_t *qs = s + 1 + q1;
    uint4 v;
    v.x = (uint32_t)qs[0] | ((uint32_t)qs[1] << 16);
    v.y = (uint32_t)qs[2] | ((uint32_t)qs[3] << 16);
    v.z = (uint32_t)qs[4] | ((uint32_t)qs[5] << 16);
    v.w = (uint32_t)qs[6] | ((uint32_t)qs[7] << 16);
    *reinterpret_cast<uint4 *>(row + (size_t)b * 16) = v;
    *reinterpret_cast<uint16_t *>(row + (size_t)nb * 16 + 2 * b) = s[0];
    if (q1) *reinterpret_cast<uint16_t *>(row + (size_t)nb * 16 + pad16((size_t)nb * 2) + 2 * b) = s[1];
}

__global__ void k_repack_q6k(const uint8_t *__restrict__ src, int64_t rows, int nsb, size_t stride,
                             uint8_t *__restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nsb) return;
    const int64_t r = i / nsb;
    const int sb = (int)(i % nsb);
    const uint16_t *s = reinterpret_cast<const uint16_t *>(src + ((size_t)r * nsb + sb) * 210);
    uint8_t *row = dst + (size_t)r * stride;
    uint32_t *body = reinterpret_cast<uint32_t *>(row + (size_t)sb * 208);
#pragma unroll 4
    for (int k = 0; k < 52; k++) body[k] = (uint32_t)s[2 * k] | ((uint32_t)s[2 * k + 1] << 16);
    *reinterpret_cast<uint16_t *>(row + (size_t)nsb * 208 + 2 * sb) = s[104];
}

int repack_rows(int type, const uint8_t *src, int64_t rows, int ncol, uint8_t *dst, cudaStream_t s) {
    const size_t stride = rows_stride(type, ncol);
    if (type == QMS_T_Q6_K) {
        const int nsb = ncol / 256;
        const int64_t n = rows * nsb;
        k_repack_q6k<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, rows, nsb, stride, dst);
    } else {
        const int nb = ncol / 32;
        const int64_t n = rows * nb;
        k_repack_q4rows<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, rows, nb, type == QMS_T_Q4_1, stride, dst);
    }
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

// ---- shared pieces ------------------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// 1 / sqrt(sum(x^2) / n + eps) in double for one row, by the whole CTA (src/model.c:405-407).
// red: nwarps doubles of shared memory. Every thread returns the same value.
__device__ double row_inv_rms(const float *__restrict__ x, int n, float eps, double *red) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)x[i];
        ss = fma(v, v, ss);
    }
    ss = warp_sum_d(ss);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < nw; i++) tot += red[i];
    return 1.0 / sqrt(tot / n + (double)eps);
}

// The reference's normalised element: (float)(x * inv) * w, two roundings (src/model.c:408).
__device__ __forceinline__ float norm_elem(float x, double inv, const float *w, int i) {
    return w ? __fmul_rn((float)((double)x * inv), w[i]) : x;
}

// Q8 block meta as packed in GemvArgs::xs: q-sum of elements 0..15 (low half) and 16..31 (high half).
__device__ __forceinline__ int pack_sums(const Q8Lane &r) { return (r.sum_lo & 0xffff) | ((r.sum - r.sum_lo) << 16); }
__device__ __forceinline__ int sum_lo(int s) { return (int)(int16_t)(s & 0xffff); }
__device__ __forceinline__ int sum_hi(int s) { return s >> 16; }

// KV cache elements: fp32 (the reference's cache, src/model.c:459-460) or fp16 (compacted: each K / V
// value rounded once when appended, read back as fp32).
__device__ __forceinline__ void kv_st(float *p, float v) { *p = v; }
__device__ __forceinline__ void kv_st(__half *p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ float kv_ld(const float *p) { return __ldcg(p); }
__device__ __forceinline__ float kv_ld(const __half *p) { return __half2float(__ldcg(p)); }
__device__ __forceinline__ float4 kv_ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 kv_ld4(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float2 kv_ld2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ float2 kv_ld2(const __half *p) { return __half22float2(*reinterpret_cast<const __half2 *>(p)); }
// the same from global memory through L2 only
__device__ __forceinline__ float4 kv_ldg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ float4 kv_ldg4(const __half *p) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(p));
    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float2 kv_ldg2(const float *p) { return __ldcg(reinterpret_cast<const float2 *>(p)); }
__device__ __forceinline__ float2 kv_ldg2(const __half *p) {
    const uint32_t u = __ldcg(reinterpret_cast<const unsigned int *>(p));
    return __half22float2(*reinterpret_cast<const __half2 *>(&u));
}

// 16-byte asynchronous copy global -> shared (L2 only; no register staging).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 8-byte asynchronous copy (through L1: the 16-byte form is the only L2-only one).
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Four cache elements: 16 bytes of fp32 or 8 bytes of fp16.
__device__ __forceinline__ void cp_async_kv4(float *dst, const float *src) { cp_async16(dst, src); }
__device__ __forceinline__ void cp_async_kv4(__half *dst, const __half *src) { cp_async8(dst, src); }
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}


// ---- embedding ---------------------------------------------------------------------------------------
__device__ __forceinline__ float dequant_elem(int type, const uint8_t *row, int i) {
    switch (type) {
    case QMS_T_F32: return reinterpret_cast<const float *>(row)[i];
    case QMS_T_F16: return h2f(reinterpret_cast<const uint16_t *>(row)[i]);
    case QMS_T_Q4_0: {
        const uint8_t *b = row + (size_t)(i >> 5) * 18;
        const int j = i & 31;
        const int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
        return __fmul_rn((float)(q - 8), h2f(*reinterpret_cast<const uint16_t *>(b)));
    }
    case QMS_T_Q4_1: {
        const uint8_t *b = row + (size_t)(i >> 5) * 20;
        const int j = i & 31;
        const int q = j < 16 ? (b[4 + j] & 0x0F) : (b[4 + j - 16] >> 4);
        return __fmaf_rn((float)q, h2f(*reinterpret_cast<const uint16_t *>(b)),
                         h2f(*reinterpret_cast<const uint16_t *>(b + 2)));
    }
    case QMS_T_Q8_0: {
        const uint8_t *b = row + (size_t)(i >> 5) * 34;
        return __fmul_rn((float)(int8_t)b[2 + (i & 31)], h2f(*reinterpret_cast<const uint16_t *>(b)));
    }
    default: {  // Q6_K, src/quant.c deq_q6_k
        const uint8_t *b = row + (size_t)(i >> 8) * 210;
        const int idx = i & 255, half = idx >> 7, r = idx & 127, quarter = r >> 5, l = r & 31;
        const uint8_t *ql = b + half * 64, *qh = b + 128 + half * 32;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + half * 8);
        const int lo = (quarter & 1) ? ql[l + 32] : ql[l];
        const int q = ((quarter < 2 ? lo & 0xF : lo >> 4) | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
        const float d = h2f(*reinterpret_cast<const uint16_t *>(b + 208));
        return __fmul_rn(__fmul_rn(d, (float)sc[(l >> 4) + 2 * quarter]), (float)q);
    }
    }
}

__global__ void __launch_bounds__(256) k_embed(int type, const uint8_t *__restrict__ embd, size_t rb, int vocab, int n,
                                               const int *__restrict__ ids, float *__restrict__ h, int *err) {
    const int t = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    const int id = ids[t];
    float *out = h + (size_t)t * n;
    if (id < 0 || id >= vocab) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = 0.0f;
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const uint8_t *row = embd + (size_t)id * rb;
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = dequant_elem(type, row, i);
}

int launch_embed(int type, const uint8_t *embd, int vocab, int n, const int *ids, int T, float *h, int *err,
                 cudaStream_t s) {
    QMS_CK(launch_pdl(k_embed, dim3(T), dim3(256), 0, s, type, embd, ggml_row_bytes(type, n), vocab, n, ids, h, err));
    return QMS_CUDA_OK;
}

// ---- RMSNorm (+ Q8 rows) ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float eps,
                                                 int n, float *__restrict__ y, int8_t *__restrict__ xq,
                                                 float *__restrict__ xd, int *__restrict__ xs) {
    __shared__ double red[8];
    const int t = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    const float *xr = x + (size_t)t * n;
    const double inv = w ? row_inv_rms(xr, n, eps, red) : 1.0;
    if (y)
        for (int i = threadIdx.x; i < n; i += blockDim.x) y[(size_t)t * n + i] = norm_elem(xr[i], inv, w, i);
    if (xq) {
        const int lane = threadIdx.x & 31, nb = n / 32;
        for (int b = threadIdx.x >> 5; b < nb; b += blockDim.x >> 5) {
            const Q8Lane r = quantize_lane(norm_elem(xr[32 * b + lane], inv, w, 32 * b + lane));
            xq[(size_t)t * n + 32 * b + lane] = (int8_t)r.q;
            if (lane == 0) {
                xd[(size_t)t * nb + b] = r.d;
                xs[(size_t)t * nb + b] = pack_sums(r);
            }
        }
    }
}

int launch_rmsnorm(const float *x, const float *w, float eps, int T, int n, float *y, int8_t *xq, float *xd, int *xs,
                   cudaStream_t s) {
    QMS_CK(launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, s, x, w, eps, n, y, xq, xd, xs));
    return QMS_CUDA_OK;
}

// ---- matrix-vector products ------------------------------------------------------------------------------
// Units: a Q4 row is split into 32-blocks, a Q6_K row into half super-blocks (128 values = four
// Q8 blocks). LPR lanes share a row (all 32 when the row has >= 32 units), each taking NU units.
template <int WT, int NU>
struct WRegs {
    uint4 nib[WT == 2 ? 6 : NU];      // Q4: nibble planes; Q6_K: ql (4) and qh (2)
    uint32_t sc[WT == 2 ? 2 : 1];     // Q6_K sub-scales
    uint16_t d[NU];
    uint16_t m[WT == 1 ? NU : 1];
};

__device__ __forceinline__ uint2 ld_stream8(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

template <int WT, int NU>
__device__ __forceinline__ void load_row(const GemvArgs &a, int r, int li, int LPR, WRegs<WT, NU> &w) {
    const uint8_t *row = a.w + (size_t)r * a.stride;
    if constexpr (WT == 2) {
        const int nsb = a.ncol / 256;
        const int u = li, sb = u >> 1, h = u & 1;
        const uint8_t *body = row + (size_t)sb * 208;
#pragma unroll
        for (int k = 0; k < 4; k++) w.nib[k] = ld_stream16(body + h * 64 + 16 * k);
#pragma unroll
        for (int k = 0; k < 2; k++) w.nib[4 + k] = ld_stream16(body + 128 + h * 32 + 16 * k);
        const uint2 s = ld_stream8(body + 192 + h * 8);
        w.sc[0] = s.x;
        w.sc[1] = s.y;
        w.d[0] = ld_stream2(row + (size_t)nsb * 208 + 2 * sb);
    } else {
        const int nb = a.ncol / 32;
#pragma unroll
        for (int j = 0; j < NU; j++) {
            const int b = li + LPR * j;
            w.nib[j] = ld_stream16(row + (size_t)b * 16);
            w.d[j] = ld_stream2(row + (size_t)nb * 16 + 2 * b);
            if constexpr (WT == 1) w.m[j] = ld_stream2(row + (size_t)nb * 16 + pad16((size_t)nb * 2) + 2 * b);
        }
    }
}

// dot of the lane's units against token tt of the staged Q8 tile
template <int WT, int NU>
__device__ __forceinline__ float lane_dot(const WRegs<WT, NU> &w, const int8_t *sq, const float *sd, const int *ss,
                                          int ncol, int li, int LPR) {
    const int nb = ncol / 32;
    float acc = 0.0f;
    if constexpr (WT == 2) {
        const int sb = li >> 1, h = li & 1;
        const float d6 = h2f(w.d[0]);
        const uint32_t *qlw = reinterpret_cast<const uint32_t *>(&w.nib[0]);
        const uint32_t *qhw = reinterpret_cast<const uint32_t *>(&w.nib[4]);
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const int b = sb * 8 + h * 4 + g;
            const int4 *x4 = reinterpret_cast<const int4 *>(sq + 32 * b);
            const int4 xa0 = x4[0], xa1 = x4[1];
            const int xw[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
            int dlo = 0, dhi = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t q6 = ((qlw[(g & 1) * 8 + k] >> (4 * (g >> 1))) & 0x0F0F0F0Fu) |
                                    (((qhw[k] >> (2 * g)) & 0x03030303u) << 4);
                if (k < 4) dlo = __dp4a((int)q6, xw[k], dlo);
                else dhi = __dp4a((int)q6, xw[k], dhi);
            }
            const uint32_t scw = w.sc[g >> 1];
            const int sa = (int)(int8_t)(scw >> (16 * (g & 1))), sbv = (int)(int8_t)(scw >> (16 * (g & 1) + 8));
            const int s = ss[b];
            const int isum = sa * (dlo - 32 * sum_lo(s)) + sbv * (dhi - 32 * sum_hi(s));
            acc = __fmaf_rn((float)isum, __fmul_rn(d6, sd[b]), acc);
        }
    } else {
#pragma unroll
        for (int j = 0; j < NU; j++) {
            const int b = li + LPR * j;
            const int4 *x4 = reinterpret_cast<const int4 *>(sq + 32 * b);
            const int isum = q4_block_isum(w.nib[j], x4[0], x4[1]);
            const float dx = sd[b];
            const int s = ss[b], sum = sum_lo(s) + sum_hi(s);
            const float dw = h2f(w.d[j]);
            if constexpr (WT == 0) {
                acc = __fmaf_rn((float)(isum - 8 * sum), __fmul_rn(dw, dx), acc);
            } else {
                acc = __fmaf_rn((float)isum, __fmul_rn(dw, dx), acc);
                acc = __fmaf_rn(h2f(w.m[j]), __fmul_rn(dx, (float)sum), acc);
            }
        }
    }
    (void)nb;
    return acc;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int r) {
    if (v != v) return 0ull;                                   // NaN never wins (argmax uses '>')
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xffffffffu - (uint32_t)r);   // ties: the lower index wins
}

template <int WT, int NU, bool F32IN>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) unsigned char gsm[];
    __shared__ double red[kGemvWarps];
    __shared__ unsigned long long s_best;
    __shared__ int s_last;
    const int ncol = a.ncol, nb = ncol / 32;
    int8_t *sq = reinterpret_cast<int8_t *>(gsm);                        // [kGemvTile][ncol]
    float *sd = reinterpret_cast<float *>(gsm + (size_t)kGemvTile * ncol);   // [kGemvTile][nb]
    int *ss = reinterpret_cast<int *>(sd + (size_t)kGemvTile * nb);     // [kGemvTile][nb]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int units = WT == 2 ? ncol / 128 : nb;
    const int LPR = units >= 32 ? 32 : units;
    const int RPW = 32 / LPR, seg = lane / LPR, li = lane % LPR;
    const int ngroups = (a.rows + RPW - 1) / RPW;
    const int gw = blockIdx.x * kGemvWarps + warp, nwg = gridDim.x * kGemvWarps;
    const bool argmax = a.amax != nullptr;
    if (tid == 0) s_best = 0ull;

    WRegs<WT, NU> cur, nxt;
    auto row_of = [&](int g) { const int r = g * RPW + seg; return r < a.rows ? r : a.rows - 1; };
    if (gw < ngroups) load_row<WT, NU>(a, row_of(gw), li, LPR, cur);   // weights never depend on earlier kernels
    pdl_trigger();
    pdl_wait();
    unsigned long long best = 0ull;
    for (int t0 = 0; t0 < a.T; t0 += kGemvTile) {
        const int tn = min(kGemvTile, a.T - t0);
        if (t0 > 0) {
            __syncthreads();
            if (gw < ngroups) load_row<WT, NU>(a, row_of(gw), li, LPR, cur);
        }
        if constexpr (F32IN) {
            for (int t = 0; t < tn; t++) {
                const float *xr = a.x + (size_t)(t0 + t) * a.ldx;
                const double inv = a.nw ? row_inv_rms(xr, ncol, a.eps, red) : 1.0;
                for (int b = warp; b < nb; b += kGemvWarps) {
                    const Q8Lane r = quantize_lane(norm_elem(xr[32 * b + lane], inv, a.nw, 32 * b + lane));
                    sq[(size_t)t * ncol + 32 * b + lane] = (int8_t)r.q;
                    if (lane == 0) {
                        sd[t * nb + b] = r.d;
                        ss[t * nb + b] = pack_sums(r);
                    }
                }
            }
        } else {
            const int4 *src = reinterpret_cast<const int4 *>(a.xq + (size_t)t0 * ncol);
            int4 *dst = reinterpret_cast<int4 *>(sq);
            for (int i = tid; i < tn * ncol / 16; i += kGemvThreads) dst[i] = __ldcg(src + i);
            for (int i = tid; i < tn * nb; i += kGemvThreads) {
                sd[i] = __ldcg(a.xd + (size_t)t0 * nb + i);
                ss[i] = __ldcg(a.xs + (size_t)t0 * nb + i);
            }
        }
        __syncthreads();
        for (int g = gw; g < ngroups; g += nwg) {
            const bool more = g + nwg < ngroups;
            if (more) load_row<WT, NU>(a, row_of(g + nwg), li, LPR, nxt);
            const int r = g * RPW + seg;
            for (int t = 0; t < tn; t++) {
                float acc = lane_dot<WT, NU>(cur, sq + (size_t)t * ncol, sd + t * nb, ss + t * nb, ncol, li, LPR);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
                    if (o < LPR) acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, o));
                if (li == 0 && r < a.rows) {
                    const size_t at = (size_t)(t0 + t) * a.ldy + r;
                    const float v = a.resid ? __fadd_rn(a.resid[at], acc) : acc;
                    a.y[at] = v;
                    if (argmax) {
                        const unsigned long long k = argmax_key(v, r);
                        best = k > best ? k : best;
                    }
                }
            }
            if (more) cur = nxt;
        }
    }
    if (!argmax) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(kFull, best, o);
        best = k > best ? k : best;
    }
    if (lane == 0) atomicMax(&s_best, best);
    __syncthreads();
    if (tid == 0) {
        atomicMax(a.amax, s_best);
        __threadfence();
        s_last = atomicAdd(a.ticket, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (tid == 0 && s_last) {
        __threadfence();
        const unsigned long long k = atomicExch(a.amax, 0ull);
        *a.tok = (int)(0xffffffffu - (uint32_t)k);
        if (a.pos) *a.pos += 1;
        *a.ticket = 0;
    }
}

constexpr int kGemvMaxCol = 8192;     // 256 Q4 blocks per row (the largest NU * 32)
constexpr size_t kGemvMaxSmem = (size_t)kGemvTile * (kGemvMaxCol + kGemvMaxCol / 32 * 8);

// Once per process and device: the variants' shared-memory limit and the SM count.
static int gemv_setup(int *nsm) {
    static int s_dev_nsm[64];
    static bool s_attr[64];
    int dev = 0;
    QMS_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) dev = 0;
    if (!s_dev_nsm[dev]) {
        int n = 148;
        QMS_CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        s_dev_nsm[dev] = n;
    }
    if (!s_attr[dev]) {
#define QMS_GEMV_ATTR(WT, NU)                                                                                    \
    QMS_CK(cudaFuncSetAttribute(k_gemv<WT, NU, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvMaxSmem)); \
    QMS_CK(cudaFuncSetAttribute(k_gemv<WT, NU, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvMaxSmem));
        QMS_GEMV_ATTR(0, 1) QMS_GEMV_ATTR(0, 2) QMS_GEMV_ATTR(0, 4) QMS_GEMV_ATTR(0, 8)
        QMS_GEMV_ATTR(1, 1) QMS_GEMV_ATTR(1, 2) QMS_GEMV_ATTR(1, 4) QMS_GEMV_ATTR(1, 8)
        QMS_GEMV_ATTR(2, 1)
#undef QMS_GEMV_ATTR
        s_attr[dev] = true;
    }
    *nsm = s_dev_nsm[dev];
    return QMS_CUDA_OK;
}

template <int WT, int NU>
static int launch_gemv_t(const GemvArgs &a, cudaStream_t s) {
    const int ncol = a.ncol, nb = ncol / 32;
    const size_t smem = (size_t)kGemvTile * (ncol + (size_t)nb * 8);
    auto kern = a.x != nullptr ? k_gemv<WT, NU, true> : k_gemv<WT, NU, false>;
    int nsm = 148;
    int rc = gemv_setup(&nsm);
    if (rc) return rc;
    const int units = WT == 2 ? ncol / 128 : nb;
    const int LPR = units >= 32 ? 32 : units;
    const int ngroups = (a.rows + 32 / LPR - 1) / (32 / LPR);
    int grid = (ngroups + kGemvWarps - 1) / kGemvWarps;
    grid = std::min(grid, 2 * nsm);
    QMS_CK(launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem, s, a));
    return QMS_CUDA_OK;
}

int launch_gemv(int type, const GemvArgs &a, cudaStream_t s) {
    QMS_REQUIRE(a.x == nullptr || a.T <= kGemvTile, QMS_CUDA_EINVAL, "gemv: fp32 input limited to %d tokens", kGemvTile);
    QMS_REQUIRE(a.amax == nullptr || a.T == 1, QMS_CUDA_EINVAL, "gemv: fused argmax needs T == 1");
    if (type == QMS_T_Q6_K) {
        const int units = a.ncol / 128;
        QMS_REQUIRE(a.ncol % 256 == 0 && units <= 32 && (units & (units - 1)) == 0, QMS_CUDA_EUNSUPPORTED,
                    "gemv: Q6_K rows of %d values not supported", a.ncol);
        return launch_gemv_t<2, 1>(a, s);
    }
    const int nb = a.ncol / 32;
    QMS_REQUIRE(a.ncol % 32 == 0 && (nb < 32 ? (nb & (nb - 1)) == 0 : nb % 32 == 0 && nb <= 256),
                QMS_CUDA_EUNSUPPORTED, "gemv: Q4 rows of %d values not supported", a.ncol);
    const int nu = nb < 32 ? 1 : nb / 32;
    QMS_REQUIRE(nu == 1 || nu == 2 || nu == 4 || nu == 8, QMS_CUDA_EUNSUPPORTED, "gemv: %d blocks per row", nb);
    if (type == QMS_T_Q4_0) {
        switch (nu) {
        case 1: return launch_gemv_t<0, 1>(a, s);
        case 2: return launch_gemv_t<0, 2>(a, s);
        case 4: return launch_gemv_t<0, 4>(a, s);
        default: return launch_gemv_t<0, 8>(a, s);
        }
    }
    QMS_REQUIRE(type == QMS_T_Q4_1, QMS_CUDA_EUNSUPPORTED, "gemv: type %d", type);
    switch (nu) {
    case 1: return launch_gemv_t<1, 1>(a, s);
    case 2: return launch_gemv_t<1, 2>(a, s);
    case 4: return launch_gemv_t<1, 4>(a, s);
    default: return launch_gemv_t<1, 8>(a, s);
    }
}

// ---- multi-token projections on int8 mma.sync ------------------------------------------------------
// y[t][r] = (resid) + sum_b d_w[r][b] * d_x[t][b] * (sum_k w[r][b][k] * x[t][b][k]) (+ the Q4_1 min
// term), each 32-block's integer dot exact and scaled in fp32 block by block, as in the one-token
// kernels (src/kernels.c:82-134). A warp owns 16 rows x 32 tokens: per block one
// mma.m16n8k32.s8 per 8 tokens (A = the rows' nibbles - 8 for Q4_0, B = the tokens' Q8 bytes),
// then the int32 results are scaled into fp32 registers. A CTA's warps share one 32-token tile:
// its Q8 bytes and block scales are staged in shared memory by cp.async, chunks of kGqKB blocks in
// two buffers (the next chunk loads while this one is used); token rows padded to kGqXS bytes and
// scale rows to kGqKB + 1 floats, so the fragment reads are conflict-free. Weights come straight
// from global memory (four lanes read a row's 16 bytes of a block: each weight byte once per tile).
constexpr int kGqKB = 8;                          // blocks per staged chunk
constexpr int kGqXS = kGqKB * 32 + 16;            // bytes of one token's chunk (+ pad)
constexpr int kGqDS = kGqKB + 1;                  // floats of one token's chunk scales (+ pad)

template <int Q1>
__global__ void __launch_bounds__(128) k_gemm_q4(const GemvArgs a) {
    // blockIdx.z: this CTA's share of the blocks when they are split over gridDim.z CTAs (each
    // writes its partial sums to kpart[z][t][r]; k_sum_parts adds them in order)
    __shared__ __align__(16) int8_t sxq[2][32 * kGqXS];
    __shared__ float sdx[2][32 * kGqDS];
    __shared__ int ssx[2][Q1 ? 32 * kGqDS : 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    const int g = lane >> 2, tg = lane & 3;
    const int r0 = (blockIdx.x * (nthr >> 5) + warp) * 16, t0 = blockIdx.y * 32;
    const int nb = a.ncol / 32, nchall = (nb + kGqKB - 1) / kGqKB, KS = gridDim.z, z = blockIdx.z;
    const int cb0 = z * nchall / KS, nch = (z + 1) * nchall / KS - cb0;   // this CTA's chunks [cb0, cb0 + nch)
    pdl_trigger();
    pdl_wait();
    auto stage = [&](int cl, int buf) {                        // chunk cb0 + cl of the tile into buffer buf
        const int c = cb0 + cl;
        const int c0 = c * kGqKB, kn = min(kGqKB, nb - c0);
        for (int i = tid; i < 32 * kn * 2; i += nthr) {
            const int t = i / (kn * 2), kb = (i >> 1) % kn, h = i & 1;
            const int tt = min(t0 + t, a.T - 1);               // rows past T are copies of the last (not stored)
            cp_async16(&sxq[buf][t * kGqXS + kb * 32 + 16 * h], a.xq + (size_t)tt * a.ncol + (size_t)(c0 + kb) * 32 + 16 * h);
        }
        for (int i = tid; i < 32 * kn; i += nthr) {
            const int t = i / kn, kb = i % kn, tt = min(t0 + t, a.T - 1);
            cp_async4(&sdx[buf][t * kGqDS + kb], a.xd + (size_t)tt * nb + c0 + kb);
            if (Q1) cp_async4(&ssx[buf][t * kGqDS + kb], a.xs + (size_t)tt * nb + c0 + kb);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const uint8_t *wr0 = a.w + (size_t)(r0 + g) * a.stride, *wr1 = wr0 + (size_t)8 * a.stride;
    const size_t dpl = (size_t)nb * 16, mpl = dpl + pad16((size_t)nb * 2);
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[j][i] = 0.0f;
    stage(0, 0);
    for (int cl = 0; cl < nch; cl++) {
        const int buf = cl & 1, c = cb0 + cl;
        // the chunk's weights into registers first: their round trip overlaps the activations' wait
        const int c0 = c * kGqKB, kn = min(kGqKB, nb - c0);
        uint32_t wq0[kGqKB], wq1[kGqKB];
        float dq0[kGqKB], dq1[kGqKB], mq0[kGqKB], mq1[kGqKB];
#pragma unroll
        for (int kb = 0; kb < kGqKB; kb++) {
            const int b = c0 + (kb < kn ? kb : 0);
            wq0[kb] = __ldg(reinterpret_cast<const uint32_t *>(wr0 + (size_t)b * 16 + 4 * tg));
            wq1[kb] = __ldg(reinterpret_cast<const uint32_t *>(wr1 + (size_t)b * 16 + 4 * tg));
            dq0[kb] = h2f(__ldg(reinterpret_cast<const uint16_t *>(wr0 + dpl) + b));
            dq1[kb] = h2f(__ldg(reinterpret_cast<const uint16_t *>(wr1 + dpl) + b));
            mq0[kb] = Q1 ? h2f(__ldg(reinterpret_cast<const uint16_t *>(wr0 + mpl) + b)) : 0.0f;
            mq1[kb] = Q1 ? h2f(__ldg(reinterpret_cast<const uint16_t *>(wr1 + mpl) + b)) : 0.0f;
        }
        if (cl + 1 < nch) {
            stage(cl + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int kb = 0; kb < kGqKB; kb++) {
            if (kb >= kn) break;
            const uint32_t w0 = wq0[kb], w1 = wq1[kb];
            uint32_t a0 = w0 & 0x0F0F0F0Fu, a2 = (w0 >> 4) & 0x0F0F0F0Fu, a1 = w1 & 0x0F0F0F0Fu, a3 = (w1 >> 4) & 0x0F0F0F0Fu;
            if (!Q1) {                                              // q - 8 in [-8, 7], bytewise
                a0 = __vsub4(a0, 0x08080808u);
                a1 = __vsub4(a1, 0x08080808u);
                a2 = __vsub4(a2, 0x08080808u);
                a3 = __vsub4(a3, 0x08080808u);
            }
            const float dw0 = dq0[kb], dw1 = dq1[kb], mw0 = mq0[kb], mw1 = mq1[kb];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int8_t *xb = &sxq[buf][(8 * j + g) * kGqXS + kb * 32 + 4 * tg];
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xb);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xb + 16);
                int c0r, c1r, c2r, c3r;
                asm volatile(
                    "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                    "{%10,%10,%10,%10};"
                    : "=r"(c0r), "=r"(c1r), "=r"(c2r), "=r"(c3r)
                    : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
                const int ta = 8 * j + 2 * tg;
                const float dx0 = sdx[buf][ta * kGqDS + kb], dx1 = sdx[buf][(ta + 1) * kGqDS + kb];
                acc[j][0] = __fmaf_rn((float)c0r, __fmul_rn(dw0, dx0), acc[j][0]);
                acc[j][1] = __fmaf_rn((float)c1r, __fmul_rn(dw0, dx1), acc[j][1]);
                acc[j][2] = __fmaf_rn((float)c2r, __fmul_rn(dw1, dx0), acc[j][2]);
                acc[j][3] = __fmaf_rn((float)c3r, __fmul_rn(dw1, dx1), acc[j][3]);
                if (Q1) {
                    const int s0 = ssx[buf][ta * kGqDS + kb], s1 = ssx[buf][(ta + 1) * kGqDS + kb];
                    const float f0 = __fmul_rn(dx0, (float)(sum_lo(s0) + sum_hi(s0)));
                    const float f1 = __fmul_rn(dx1, (float)(sum_lo(s1) + sum_hi(s1)));
                    acc[j][0] = __fmaf_rn(mw0, f0, acc[j][0]);
                    acc[j][1] = __fmaf_rn(mw0, f1, acc[j][1]);
                    acc[j][2] = __fmaf_rn(mw1, f0, acc[j][2]);
                    acc[j][3] = __fmaf_rn(mw1, f1, acc[j][3]);
                }
            }
        }
        __syncthreads();                                       // buffer buf is refilled next iteration
    }
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = t0 + 8 * j + 2 * tg + (i & 1), r = r0 + g + 8 * (i >> 1);
            if (t < a.T) {
                if (KS > 1) {
                    a.kpart[((size_t)z * a.T + t) * a.rows + r] = acc[j][i];
                } else {
                    const size_t at = (size_t)t * a.ldy + r;
                    a.y[at] = a.resid ? __fadd_rn(a.resid[at], acc[j][i]) : acc[j][i];
                }
            }
        }
}

// y[t][r] = (resid) + sum over z in order of part[z][t][r]: the split projections' partial sums.
__global__ void __launch_bounds__(256) k_sum_parts(const float *__restrict__ part, int KS, int T, int rows, float *y,
                                                  int ldy, const float *resid) {
    pdl_trigger();
    pdl_wait();
    const size_t n = (size_t)T * rows;
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256) {
        float v = part[i];
        for (int z = 1; z < KS; z++) v = __fadd_rn(v, part[(size_t)z * n + i]);
        const int t = (int)(i / rows), r = (int)(i % rows);
        const size_t at = (size_t)t * ldy + r;
        y[at] = resid ? __fadd_rn(resid[at], v) : v;
    }
}

// Q6_K rows (the head) on int8 mma.sync, several tokens. A 256-value super-block holds 16
// sub-blocks of 16 with int8 scales; a 32-value Q8 activation block covers two of them, so each
// block takes two m16n8k16 products (A = q6 - 32, exact int32), combined as sa * c_lo + sb * c_hi in
// integers and scaled by d6 * d_x in fp32: the arithmetic of the one-token head kernel
// (src/kernels.c:139-195). Element layout of a super-block (ggml): half n = e / 128; within it
// quarter qq = (e % 128) / 32 and l = e % 32; low 4 bits in ql[64 n + 32 (qq & 1) + l] at shift
// 4 (qq >> 1), high 2 bits in qh[32 n + l] at shift 2 qq; scale sc[8 n + 2 qq + l / 16].
__global__ void __launch_bounds__(128) k_gemm_q6k(const GemvArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tg = lane & 3;
    const int r0 = (blockIdx.x * (blockDim.x >> 5) + warp) * 16, t0 = blockIdx.y * 32;
    const int nsb = a.ncol / 256, nb = a.ncol / 32;
    pdl_trigger();
    pdl_wait();
    if (r0 >= a.rows) return;
    const uint8_t *wr[2] = {a.w + (size_t)(r0 + g) * a.stride, a.w + (size_t)(r0 + g + 8) * a.stride};
    const int8_t *xr[4];
    const float *dr[4][2];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        xr[j] = a.xq + (size_t)min(t0 + 8 * j + g, a.T - 1) * a.ncol + 4 * tg;
#pragma unroll
        for (int h = 0; h < 2; h++) dr[j][h] = a.xd + (size_t)min(t0 + 8 * j + 2 * tg + h, a.T - 1) * nb;
    }
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[j][i] = 0.0f;
    for (int sb = 0; sb < nsb; sb++) {
        uint32_t ql[2][2][2][2], qh[2][2][2];     // [row][half n][ql: qq & 1 / -][k0 / 16]
        int8_t sc[2][16];
        float d6[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint8_t *body = wr[r] + (size_t)sb * 208;
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    ql[r][n][0][k] = __ldg(reinterpret_cast<const uint32_t *>(body + 64 * n + 16 * k + 4 * tg));
                    ql[r][n][1][k] = __ldg(reinterpret_cast<const uint32_t *>(body + 64 * n + 32 + 16 * k + 4 * tg));
                    qh[r][n][k] = __ldg(reinterpret_cast<const uint32_t *>(body + 128 + 32 * n + 16 * k + 4 * tg));
                }
            const uint4 s4 = __ldg(reinterpret_cast<const uint4 *>(body + 192));
            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int i = 0; i < 16; i++) sc[r][i] = (int8_t)(sw[i >> 2] >> (8 * (i & 3)));
            d6[r] = h2f(__ldg(reinterpret_cast<const uint16_t *>(wr[r] + (size_t)nsb * 208) + sb));
        }
#pragma unroll
        for (int n = 0; n < 2; n++)
#pragma unroll
            for (int qq = 0; qq < 4; qq++) {
                const int bq = sb * 8 + 4 * n + qq;          // the Q8 block of these 32 values
                uint32_t A[2][2];                            // [k0 / 16][row]
#pragma unroll
                for (int k = 0; k < 2; k++)
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        const uint32_t lw = ql[r][n][qq & 1][k];
                        const uint32_t q6 = ((lw >> (4 * (qq >> 1))) & 0x0F0F0F0Fu) | (((qh[r][n][k] >> (2 * qq)) & 0x03030303u) << 4);
                        A[k][r] = __vsub4(q6, 0x20202020u);
                    }
                const int sa0 = sc[0][8 * n + 2 * qq], sb0 = sc[0][8 * n + 2 * qq + 1];
                const int sa1 = sc[1][8 * n + 2 * qq], sb1 = sc[1][8 * n + 2 * qq + 1];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    int c[2][4];
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        const uint32_t b0 = __ldg(reinterpret_cast<const uint32_t *>(xr[j] + (size_t)bq * 32 + 16 * k));
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
                            "{%7,%7,%7,%7};"
                            : "=r"(c[k][0]), "=r"(c[k][1]), "=r"(c[k][2]), "=r"(c[k][3])
                            : "r"(A[k][0]), "r"(A[k][1]), "r"(b0), "r"(0));
                    }
                    const float dx0 = __ldg(dr[j][0] + bq), dx1 = __ldg(dr[j][1] + bq);
                    acc[j][0] = __fmaf_rn((float)(sa0 * c[0][0] + sb0 * c[1][0]), __fmul_rn(d6[0], dx0), acc[j][0]);
                    acc[j][1] = __fmaf_rn((float)(sa0 * c[0][1] + sb0 * c[1][1]), __fmul_rn(d6[0], dx1), acc[j][1]);
                    acc[j][2] = __fmaf_rn((float)(sa1 * c[0][2] + sb1 * c[1][2]), __fmul_rn(d6[1], dx0), acc[j][2]);
                    acc[j][3] = __fmaf_rn((float)(sa1 * c[0][3] + sb1 * c[1][3]), __fmul_rn(d6[1], dx1), acc[j][3]);
                }
            }
    }
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = t0 + 8 * j + 2 * tg + (i & 1), r = r0 + g + 8 * (i >> 1);
            if (t < a.T) {
                const size_t at = (size_t)t * a.ldy + r;
                a.y[at] = a.resid ? __fadd_rn(a.resid[at], acc[j][i]) : acc[j][i];
            }
        }
}

// Multi-token projection of Q8 rows (xq / xd / xs) on mma.sync: Q4_0 / Q4_1 / Q6_K rows, a multiple of 16.
int launch_gemm_q(int type, const GemvArgs &a, cudaStream_t s) {
    QMS_REQUIRE((type == QMS_T_Q4_0 || type == QMS_T_Q4_1 || type == QMS_T_Q6_K) && a.x == nullptr && a.xq &&
                    a.rows % 16 == 0 && a.ncol % (type == QMS_T_Q6_K ? 256 : 32) == 0 && a.T >= 1 &&
                    a.amax == nullptr && a.stride % 16 == 0,
                QMS_CUDA_EINVAL, "gemm_q: type %d, %d rows of %d", type, a.rows, a.ncol);
    const int wpc = a.rows % 64 == 0 ? 4 : 1;                      // warps (16 rows each) per CTA
    dim3 grid(a.rows / (16 * wpc), (a.T + 31) / 32);
    if (type == QMS_T_Q6_K) {
        QMS_CK(launch_pdl(k_gemm_q6k, grid, dim3(32 * wpc), 0, s, a));
        return QMS_CUDA_OK;
    }
    // Few tiles (a few dozen tokens): split the blocks over up to 4 CTAs per tile so that ~4 CTAs
    // per SM hide the load latency; the partial sums are added in order by k_sum_parts.
    int nsm = 148;
    const int rc = gemv_setup(&nsm);
    if (rc) return rc;
    const int tiles = (int)(grid.x * grid.y), nch = (a.ncol / 32 + kGqKB - 1) / kGqKB;
    int ks = 1;
    while (ks < 4 && tiles * ks * 2 <= 4 * nsm && ks * 2 <= nch && a.kpart &&
           (size_t)ks * 2 * a.T * a.rows <= a.kpart_n)
        ks *= 2;
    grid.z = ks;
    if (type == QMS_T_Q4_0) QMS_CK(launch_pdl(k_gemm_q4<0>, grid, dim3(32 * wpc), 0, s, a));
    else QMS_CK(launch_pdl(k_gemm_q4<1>, grid, dim3(32 * wpc), 0, s, a));
    if (ks > 1) {
        const size_t n = (size_t)a.T * a.rows;
        const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)4 * nsm);
        QMS_CK(launch_pdl(k_sum_parts, dim3(blocks), dim3(256), 0, s, (const float *)a.kpart, ks, a.T, a.rows, a.y,
                          a.ldy, a.resid));
    }
    return QMS_CUDA_OK;
}

// ---- QK-norm, RoPE, KV append ------------------------------------------------------------------------------
template <int D, typename KT>
__global__ void __launch_bounds__(256) k_qk_rope(const AttnArgs a) {
    constexpr int J = D / 32, JH = J / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = blockIdx.x * 8 + warp, t = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    if (hh >= a.H + 2 * a.Hk) return;
    const int p = a.pos_vec ? a.pos_vec[t] : *a.pos + t;
    if (p < 0 || p >= a.ctx) {
        if (lane == 0) atomicOr(a.err, 1);
        return;
    }
    const int KD = a.Hk * D;
    const size_t cb = a.pos_vec ? (size_t)t * a.seq_stride : 0;   // this token's sequence
    float *row = a.qkv + (size_t)t * a.ldq + (size_t)hh * D;
    float x[J];
#pragma unroll
    for (int j = 0; j < J; j++) x[j] = row[lane + 32 * j];
    if (hh >= a.H + a.Hk) {                                    // v head: append as is
        KT *dst = static_cast<KT *>(a.vc) + cb + (size_t)p * KD + (size_t)(hh - a.H - a.Hk) * D;
#pragma unroll
        for (int j = 0; j < J; j++) kv_st(dst + lane + 32 * j, x[j]);
        return;
    }
    const float *nw = hh < a.H ? a.q_norm : a.k_norm;
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < J; j++) ss = fma((double)x[j], (double)x[j], ss);
    ss = warp_sum_d(ss);
    const double inv = 1.0 / sqrt(ss / D + (double)a.eps);
#pragma unroll
    for (int j = 0; j < J; j++) x[j] = norm_elem(x[j], inv, nw, lane + 32 * j);
    const float *cs = a.rope_cos + (size_t)p * (D / 2), *sn = a.rope_sin + (size_t)p * (D / 2);
#pragma unroll
    for (int j = 0; j < JH; j++) {                             // element i pairs with i + D/2
        const int i = lane + 32 * j;
        const float c = cs[i], s = sn[i], x1 = x[j], x2 = x[j + JH];
        x[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        x[j + JH] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
    if (hh < a.H) {
#pragma unroll
        for (int j = 0; j < J; j++) row[lane + 32 * j] = x[j];
        return;
    }
    KT *dst = static_cast<KT *>(a.kc) + cb + (size_t)p * KD + (size_t)(hh - a.H) * D;
#pragma unroll
    for (int j = 0; j < J; j++) kv_st(dst + lane + 32 * j, x[j]);
}

int launch_qk_rope(const AttnArgs &a, cudaStream_t s) {
    const dim3 grid((a.H + 2 * a.Hk + 7) / 8, a.T);
    if (a.D == 128) {
        if (a.kv16) QMS_CK(launch_pdl(k_qk_rope<128, __half>, grid, dim3(256), 0, s, a));
        else QMS_CK(launch_pdl(k_qk_rope<128, float>, grid, dim3(256), 0, s, a));
    } else {
        if (a.kv16) QMS_CK(launch_pdl(k_qk_rope<64, __half>, grid, dim3(256), 0, s, a));
        else QMS_CK(launch_pdl(k_qk_rope<64, float>, grid, dim3(256), 0, s, a));
    }
    return QMS_CUDA_OK;
}

// ---- attention -------------------------------------------------------------------------------------------------
int attention_heads_per_cta(int group) { return group < 4 ? group : 4; }

template <int D, typename KT>
__global__ void __launch_bounds__(128) k_attention(const AttnArgs a) {
    constexpr int NQ = D / 16;                   // elements of q per lane (lane k of 16: 16i + k)
    constexpr int DPL = D / 32;                  // output dims per lane
    const int HB = blockDim.x >> 5;
    const int group = a.H / a.Hk, nhb = group / HB;
    const int g = blockIdx.x / nhb, hb = blockIdx.x % nhb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g * group + hb * HB + warp;
    const int t = blockIdx.z;
    pdl_trigger();
    pdl_wait();
    const int pt = a.pos_vec ? a.pos_vec[t] : *a.pos + t;
    if (pt < 0 || pt >= a.ctx) return;           // k_qk_rope has flagged it
    const size_t cb = a.pos_vec ? (size_t)t * a.seq_stride : 0;
    const int p1 = pt + 1;                       // positions 0 .. pt (causal)
    const int KD = a.Hk * D;
    const float *qh = a.qkv + (size_t)t * a.ldq + (size_t)h * D;
    const int k16 = lane & 15, half = lane >> 4;
    float qr[NQ];
#pragma unroll
    for (int i = 0; i < NQ; i++) qr[i] = qh[16 * i + k16];
    const KT *kb = static_cast<const KT *>(a.kc) + cb + (size_t)g * D, *vb = static_cast<const KT *>(a.vc) + cb + (size_t)g * D;
    float o[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) o[d] = 0.0f;
    double m = -INFINITY, l = 0.0;
    for (int pc = 0; pc < p1; pc += 32) {
        float mydot = 0.0f;
#pragma unroll 4
        for (int j = 0; j < 16; j++) {
            const int p = pc + 2 * j + half;
            float acc = 0.0f;
            if (p < p1) {
                const KT *kp = kb + (size_t)p * KD;
#pragma unroll
                for (int i = 0; i < NQ; i++) acc = __fmaf_rn(qr[i], kv_ld(kp + 16 * i + k16), acc);
            }
            acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, 8, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, 4, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, 2, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, 1, 16));
            const float d0 = __shfl_sync(kFull, acc, 0), d1 = __shfl_sync(kFull, acc, 16);
            if (lane == 2 * j) mydot = d0;
            if (lane == 2 * j + 1) mydot = d1;
        }
        const bool valid = pc + lane < p1;
        const double sc = valid ? (double)mydot * a.scale : -INFINITY;
        const double mn = fmax(m, warp_max_d(sc));
        const double alpha = m == -INFINITY ? 0.0 : exp(m - mn);
        const double e = valid ? exp(sc - mn) : 0.0;
        l = fma(l, alpha, warp_sum_d(e));
        m = mn;
        const float fa = (float)alpha, fe = (float)e;
#pragma unroll
        for (int d = 0; d < DPL; d++) o[d] = __fmul_rn(o[d], fa);
        const int np = min(32, p1 - pc);
        for (int q = 0; q < np; q++) {
            const float w = __shfl_sync(kFull, fe, q);
            const KT *vp = vb + (size_t)(pc + q) * KD + lane * DPL;
            if constexpr (DPL == 4) {
                const float4 v = kv_ldg4(vp);
                o[0] = __fmaf_rn(w, v.x, o[0]);
                o[1] = __fmaf_rn(w, v.y, o[1]);
                o[2] = __fmaf_rn(w, v.z, o[2]);
                o[3] = __fmaf_rn(w, v.w, o[3]);
            } else {
                const float2 v = kv_ldg2(vp);
                o[0] = __fmaf_rn(w, v.x, o[0]);
                o[1] = __fmaf_rn(w, v.y, o[1]);
            }
        }
    }
    float *out = a.out + (size_t)t * a.H * D + (size_t)h * D + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; d++) out[d] = (float)((double)o[d] / l);
}

// One CTA per row: the largest argmax_key (NaN never wins, ties to the lower index).
__global__ void __launch_bounds__(256) k_argmax_rows(const float *__restrict__ logits, int ld, int V, int *tok,
                                                     int *pos) {
    __shared__ unsigned long long s_best[8];
    const int b = blockIdx.x, tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const float *row = logits + (size_t)b * ld;
    unsigned long long best = 0ull;
    for (int i = tid; i < V; i += 256) {
        const unsigned long long k = argmax_key(__ldcg(row + i), i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(kFull, best, o);
        best = k > best ? k : best;
    }
    if ((tid & 31) == 0) s_best[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; w++) best = s_best[w] > best ? s_best[w] : best;
        tok[b] = (int)(0xffffffffu - (uint32_t)best);
        if (pos) pos[b] += 1;
    }
}

int launch_argmax_rows(const float *logits, int ld, int B, int V, int *tok, int *pos, cudaStream_t s) {
    QMS_REQUIRE(B >= 1 && V >= 1 && ld >= V, QMS_CUDA_EINVAL, "argmax_rows: %d rows of %d", B, V);
    QMS_CK(launch_pdl(k_argmax_rows, dim3(B), dim3(256), 0, s, logits, ld, V, tok, pos));
    return QMS_CUDA_OK;
}

int launch_attention(const AttnArgs &a, cudaStream_t s) {
    const int group = a.H / a.Hk, HB = attention_heads_per_cta(group);
    const dim3 grid(a.Hk * (group / HB), 1, a.T);
    if (a.D == 128) {
        if (a.kv16) QMS_CK(launch_pdl(k_attention<128, __half>, grid, dim3(32 * HB), 0, s, a));
        else QMS_CK(launch_pdl(k_attention<128, float>, grid, dim3(32 * HB), 0, s, a));
    } else {
        if (a.kv16) QMS_CK(launch_pdl(k_attention<64, __half>, grid, dim3(32 * HB), 0, s, a));
        else QMS_CK(launch_pdl(k_attention<64, float>, grid, dim3(32 * HB), 0, s, a));
    }
    return QMS_CUDA_OK;
}

}  // namespace qms

// ---- one-token projections: persistent CTAs streaming their rows through a bulk-copy ring ---------
#include "qms_async.cuh"

namespace qms {

constexpr int kG1Warps = 16;                         // consumer warps (+ one producer warp), also for the head
constexpr int kG1WarpsHead = 16;
constexpr uint32_t kG1Stage = 32 * 1024;             // bytes per ring slot (whole rows)
constexpr int kG1MaxRing = 8;
constexpr size_t kG1SmemBudget = 160 * 1024;         // leaves room for a co-resident attention CTA
constexpr uint32_t kG1Spin = 1u << 22;               // polls before a wait gives up (>= 0.1 s)
enum { G1_ERR_WAIT = 64 };

struct G1Layout {
    int rps;          // rows per stage (a multiple of the rows one warp pass covers)
    int nst;          // ring slots
    uint32_t act;     // bytes of the activation area
};

__host__ __device__ inline int g1_lpr(int type, int ncol) {
    const int units = type == QMS_T_Q6_K ? ncol / 128 : ncol / 32;
    return units >= 32 ? 32 : units;
}

// Wait for `parity` of `bar` with a bound; on timeout raise *abort and the error bit.
__device__ __forceinline__ bool g1_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (++n == kG1Spin) {
            *abort = 1;
            atomicOr(err, G1_ERR_WAIT);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Activations in shared memory: q[0..15] and q[16..31] of block b at sqa + 16 b and sqb + 16 b
// (lanes reading consecutive blocks read consecutive 16-byte words), d and packed sums per block.
template <int WT, int NU>
__device__ __forceinline__ float g1_row_dot(const uint8_t *row, int ncol, const uint8_t *sqa, const uint8_t *sqb,
                                            const float *sd, const int *ss, int li, int LPR) {
    float acc = 0.0f;
    const int nb = ncol / 32;
    if constexpr (WT == 2) {
        const int nsb = ncol / 256, sb = li >> 1, h = li & 1;
        const uint8_t *body = row + (size_t)sb * 208;
        uint32_t qlw[16], qhw[8];
#pragma unroll
        for (int k = 0; k < 4; k++) *reinterpret_cast<uint4 *>(&qlw[4 * k]) = *reinterpret_cast<const uint4 *>(body + h * 64 + 16 * k);
#pragma unroll
        for (int k = 0; k < 2; k++) *reinterpret_cast<uint4 *>(&qhw[4 * k]) = *reinterpret_cast<const uint4 *>(body + 128 + h * 32 + 16 * k);
        const uint2 scw = *reinterpret_cast<const uint2 *>(body + 192 + h * 8);
        const float d6 = h2f(*reinterpret_cast<const uint16_t *>(row + (size_t)nsb * 208 + 2 * sb));
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const int b = g * (nb >> 2) + sb * 2 + h;               // g1_act_pos of block 8 sb + 4 h + g
            const int4 xa0 = *reinterpret_cast<const int4 *>(sqa + 16 * b), xa1 = *reinterpret_cast<const int4 *>(sqb + 16 * b);
            const int xw[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
            int dlo = 0, dhi = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t q6 = ((qlw[(g & 1) * 8 + k] >> (4 * (g >> 1))) & 0x0F0F0F0Fu) |
                                    (((qhw[k] >> (2 * g)) & 0x03030303u) << 4);
                if (k < 4) dlo = __dp4a((int)q6, xw[k], dlo);
                else dhi = __dp4a((int)q6, xw[k], dhi);
            }
            const uint32_t w = (g >> 1) ? scw.y : scw.x;
            const int sa = (int)(int8_t)(w >> (16 * (g & 1))), sbv = (int)(int8_t)(w >> (16 * (g & 1) + 8));
            const int s = ss[b];
            const int isum = sa * (dlo - 32 * sum_lo(s)) + sbv * (dhi - 32 * sum_hi(s));
            acc = __fmaf_rn((float)isum, __fmul_rn(d6, sd[b]), acc);
        }
    } else {
#pragma unroll
        for (int j = 0; j < NU; j++) {
            const int b = li + LPR * j;
            const uint4 nib = *reinterpret_cast<const uint4 *>(row + (size_t)b * 16);
            const float dw = h2f(*reinterpret_cast<const uint16_t *>(row + (size_t)nb * 16 + 2 * b));
            const int isum = q4_block_isum(nib, *reinterpret_cast<const int4 *>(sqa + 16 * b),
                                           *reinterpret_cast<const int4 *>(sqb + 16 * b));
            const float dx = sd[b];
            const int s = ss[b], sum = sum_lo(s) + sum_hi(s);
            if constexpr (WT == 0) {
                acc = __fmaf_rn((float)(isum - 8 * sum), __fmul_rn(dw, dx), acc);
            } else {
                const float mw = h2f(*reinterpret_cast<const uint16_t *>(row + (size_t)nb * 16 + pad16((size_t)nb * 2) + 2 * b));
                acc = __fmaf_rn((float)isum, __fmul_rn(dw, dx), acc);
                acc = __fmaf_rn(mw, __fmul_rn(dx, (float)sum), acc);
            }
        }
    }
    return acc;
}

// Where activation block b sits in shared memory. A Q6_K unit (lane li) reads blocks 4 li .. 4 li + 3,
// so for Q6_K rows block b goes to (b % 4) * nb / 4 + b / 4: for each of the four groups the lanes
// then read consecutive 16-byte words (no bank conflicts). Q4 lanes read consecutive blocks as is.
template <int WT>
__device__ __forceinline__ int g1_act_pos(int b, int nb) { return WT == 2 ? (b & 3) * (nb >> 2) + (b >> 2) : b; }

template <int NWC>
__device__ __forceinline__ void g1_consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NWC * 32) : "memory"); }

template <int WT, int NU, int NWC>
__global__ void __launch_bounds__((NWC + 1) * 32, NWC > 8 ? 1 : 2) k_gemv1(const GemvArgs a, const G1Layout lay, int *err) {
    constexpr int kG1Warps = NWC;
    extern __shared__ __align__(128) uint8_t g1sm[];
    __shared__ __align__(8) uint64_t full[kG1MaxRing], empty[kG1MaxRing];
    __shared__ double red[NWC];
    __shared__ unsigned long long s_best;
    __shared__ int s_abort, s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int r0 = (int)((int64_t)c * a.rows / G), r1 = (int)((int64_t)(c + 1) * a.rows / G), nr = r1 - r0;
    const int ncol = a.ncol, nb = ncol / 32;
    const int LPR = g1_lpr(WT == 2 ? QMS_T_Q6_K : QMS_T_Q4_0, ncol), RPW = 32 / LPR;
    const int nstage = (nr + lay.rps - 1) / lay.rps;
    uint8_t *ring = g1sm + lay.act;
    uint8_t *sqa = g1sm, *sqb = g1sm + (size_t)nb * 16;
    float *sd = reinterpret_cast<float *>(g1sm + (size_t)nb * 32);
    int *ss = reinterpret_cast<int *>(g1sm + (size_t)nb * 36);
    if (tid == 0) {
        for (int i = 0; i < lay.nst; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], lay.rps / RPW);
        }
        fence_mbar_init();
        s_abort = 0;
        s_best = 0ull;
    }
    __syncthreads();
    volatile int *abort = &s_abort;
    if (warp == kG1Warps) {                                   // producer: the weights never depend on
        if (lane == 0) {                                      // earlier kernels, so they stream at once
            const uint64_t pol = evict_first_policy();
            int issued = 0;
            for (int k = 0; k < nstage; k++) {
                const int slot = k % lay.nst;
                if (k >= lay.nst && !g1_wait(&empty[slot], ((k / lay.nst) - 1) & 1, abort, err)) break;
                const int rows = min(lay.rps, nr - k * lay.rps);
                const uint32_t bytes = (uint32_t)((size_t)rows * a.stride);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load(ring + (size_t)slot * kG1Stage, a.w + (size_t)(r0 + k * lay.rps) * a.stride, bytes, &full[slot], pol);
                issued = k + 1;
            }
            // every copy this CTA issued must land before the CTA may exit
            for (int k = issued > lay.nst ? issued - lay.nst : 0; k < issued; k++) {
                uint32_t n = 0;
                while (!mbar_try_wait(&full[k % lay.nst], (k / lay.nst) & 1))
                    if (++n == kG1Spin) {
                        atomicOr(err, G1_ERR_WAIT);
                        break;
                    }
            }
        }
        pdl_trigger();
        pdl_wait();
        return;
    }
    pdl_trigger();
    pdl_wait();
    // ---- activations: Q8 blocks of x (RMS-normed first with nw) or copied Q8 rows
    if (a.x) {
        // item v = (block v / 4, quarter v % 4): eight consecutive values; a thread takes items
        // tid + 256 k, all loaded before any is used (one round trip), and the four threads of a
        // block are consecutive lanes. The sum of squares has one fixed order in every CTA.
        constexpr int kItems = 4;                       // nb * 4 <= 4 * 256: ncol <= 8192
        const int nitems = nb * 4;
        float xv[kItems][8];
#pragma unroll
        for (int k = 0; k < kItems; k++) {
            const int v = tid + kG1Warps * 32 * k;
            if (v < nitems) {
                const float4 x0 = __ldcg(reinterpret_cast<const float4 *>(a.x + 8 * v));
                const float4 x1 = __ldcg(reinterpret_cast<const float4 *>(a.x + 8 * v + 4));
                xv[k][0] = x0.x; xv[k][1] = x0.y; xv[k][2] = x0.z; xv[k][3] = x0.w;
                xv[k][4] = x1.x; xv[k][5] = x1.y; xv[k][6] = x1.z; xv[k][7] = x1.w;
            }
        }
        if (a.nw) {
            float wv[kItems][8];
#pragma unroll
            for (int k = 0; k < kItems; k++) {
                const int v = tid + kG1Warps * 32 * k;
                if (v < nitems) {
                    const float4 w0 = __ldg(reinterpret_cast<const float4 *>(a.nw + 8 * v));
                    const float4 w1 = __ldg(reinterpret_cast<const float4 *>(a.nw + 8 * v + 4));
                    wv[k][0] = w0.x; wv[k][1] = w0.y; wv[k][2] = w0.z; wv[k][3] = w0.w;
                    wv[k][4] = w1.x; wv[k][5] = w1.y; wv[k][6] = w1.z; wv[k][7] = w1.w;
                }
            }
            double s2 = 0.0;
#pragma unroll
            for (int k = 0; k < kItems; k++)
                if (tid + kG1Warps * 32 * k < nitems)
#pragma unroll
                    for (int m = 0; m < 8; m++) s2 = fma((double)xv[k][m], (double)xv[k][m], s2);
            s2 = warp_sum_d(s2);
            if (lane == 0) red[warp] = s2;
            g1_consumer_sync<NWC>();
            double tot = 0.0;
            for (int i = 0; i < kG1Warps; i++) tot += red[i];
            const double inv = 1.0 / sqrt(tot / ncol + (double)a.eps);
#pragma unroll
            for (int k = 0; k < kItems; k++)
#pragma unroll
                for (int m = 0; m < 8; m++) xv[k][m] = __fmul_rn((float)((double)xv[k][m] * inv), wv[k][m]);
        }
#pragma unroll
        for (int k = 0; k < kItems; k++) {
            const int v = tid + kG1Warps * 32 * k;
            if (k * kG1Warps * 32 >= nitems) break;           // uniform: nitems is a multiple of 32
            const int b = v >> 2, p = v & 3;
            float amax = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; m++) amax = fmaxf(amax, fabsf(xv[k][m]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            uint32_t w0 = 0, w1 = 0;
            int sum = 0;
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int q = __float2int_rn(__fmul_rn(xv[k][m], id));
                sum += q;
                if (m < 4) w0 |= (uint32_t)(q & 0xff) << (8 * m);
                else w1 |= (uint32_t)(q & 0xff) << (8 * (m - 4));
            }
            const int s_pair = sum + __shfl_xor_sync(0xffffffffu, sum, 1);   // quarters 0+1: elements 0..15
            const int s_all = s_pair + __shfl_xor_sync(0xffffffffu, s_pair, 2);
            if (v < nitems) {
                const int bp = g1_act_pos<WT>(b, nb);
                uint8_t *dst = (p < 2 ? sqa : sqb) + 16 * bp + 8 * (p & 1);
                *reinterpret_cast<uint2 *>(dst) = make_uint2(w0, w1);
                if (p == 0) {
                    sd[bp] = d;
                    ss[bp] = (s_pair & 0xffff) | ((s_all - s_pair) << 16);
                }
            }
        }
    } else {
        for (int b = tid; b < nb; b += kG1Warps * 32) {
            const int4 *src = reinterpret_cast<const int4 *>(a.xq + 32 * (size_t)b);
            const int bp = g1_act_pos<WT>(b, nb);
            *reinterpret_cast<int4 *>(sqa + 16 * bp) = __ldcg(src);
            *reinterpret_cast<int4 *>(sqb + 16 * bp) = __ldcg(src + 1);
            sd[bp] = __ldcg(a.xd + b);
            ss[bp] = __ldcg(a.xs + b);
        }
    }
    g1_consumer_sync<NWC>();
    // ---- rows: warp pass g covers local rows [g*RPW, g*RPW + RPW), all inside one stage; a warp
    // takes passes g and g + NWC together so two rows' shared-memory loads are in flight at once
    const int seg = lane / LPR, li = lane % LPR;
    const int npass = (nr + RPW - 1) / RPW, ppst = lay.rps / RPW;
    unsigned long long best = 0ull;
    auto finish = [&](int g, int slot, float acc) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            if (o < LPR) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);             // this pass no longer reads the slot
        const int lr = g * RPW + seg;
        if (li == 0 && lr < nr) {
            const int r = r0 + lr;
            const float v = a.resid ? __fadd_rn(a.resid[r], acc) : acc;
            a.y[r] = v;
            if (a.amax) {
                const unsigned long long key = argmax_key(v, r);
                best = key > best ? key : best;
            }
        }
    };
    for (int g = warp; g < npass; g += 2 * NWC) {
        const int g2 = g + NWC;
        const bool two = g2 < npass;
        const int k1 = g / ppst, s1 = k1 % lay.nst, k2 = g2 / ppst, s2 = k2 % lay.nst;
        if (!g1_wait(&full[s1], (k1 / lay.nst) & 1, abort, err)) break;
        if (two && !g1_wait(&full[s2], (k2 / lay.nst) & 1, abort, err)) break;
        const int lr1 = g * RPW + seg, lr2 = g2 * RPW + seg;
        const uint8_t *row1 = ring + (size_t)s1 * kG1Stage + (size_t)(lr1 - k1 * lay.rps) * a.stride;
        const uint8_t *row2 = ring + (size_t)s2 * kG1Stage + (size_t)(lr2 - k2 * lay.rps) * a.stride;
        const float acc1 = lr1 < nr ? g1_row_dot<WT, NU>(row1, ncol, sqa, sqb, sd, ss, li, LPR) : 0.0f;
        const float acc2 = two && lr2 < nr ? g1_row_dot<WT, NU>(row2, ncol, sqa, sqb, sd, ss, li, LPR) : 0.0f;
        finish(g, s1, acc1);
        if (two) finish(g2, s2, acc2);
    }
    if (!a.amax) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long key = __shfl_xor_sync(0xffffffffu, best, o);
        best = key > best ? key : best;
    }
    if (lane == 0) atomicMax(&s_best, best);
    g1_consumer_sync<NWC>();
    if (tid == 0) {
        atomicMax(a.amax, s_best);
        __threadfence();
        s_last = atomicAdd(a.ticket, 1) == G - 1;
    }
    g1_consumer_sync<NWC>();
    if (tid == 0 && s_last) {
        __threadfence();
        const unsigned long long key = atomicExch(a.amax, 0ull);
        *a.tok = (int)(0xffffffffu - (uint32_t)key);
        if (a.pos) *a.pos += 1;
        *a.ticket = 0;
    }
}

template <int WT, int NU, int NWC = (WT == 2 ? kG1WarpsHead : kG1Warps)>
static int launch_gemv1_t(const GemvArgs &a, int *err, cudaStream_t s) {
    int nsm = 148;
    int rc = gemv_setup(&nsm);
    if (rc) return rc;
    const int type = WT == 2 ? QMS_T_Q6_K : WT == 1 ? QMS_T_Q4_1 : QMS_T_Q4_0;
    const int RPW = 32 / g1_lpr(type, a.ncol);
    G1Layout lay;
    lay.act = (uint32_t)(((size_t)(a.ncol / 32) * 40 + 127) & ~(size_t)127);
    lay.rps = (int)(kG1Stage / a.stride) / RPW * RPW;
    QMS_REQUIRE(lay.rps >= RPW, QMS_CUDA_EUNSUPPORTED, "gemv1: rows of %zu bytes", a.stride);
    const int G = std::min(nsm, a.rows);
    const int per_cta = (a.rows + G - 1) / G;
    const int stages = (per_cta + lay.rps - 1) / lay.rps;
    lay.nst = (int)std::min<size_t>(std::min(kG1MaxRing, stages), (kG1SmemBudget - lay.act) / kG1Stage);
    if (lay.nst < 1) lay.nst = 1;
    const size_t smem = lay.act + (size_t)lay.nst * kG1Stage;
    auto kern = k_gemv1<WT, NU, NWC>;
    static bool s_attr[64];
    int dev = 0;
    QMS_CK(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !s_attr[dev]) {
        QMS_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kG1SmemBudget + 16384)));
        s_attr[dev] = true;
    }
    QMS_CK(launch_pdl(kern, dim3(G), dim3((NWC + 1) * 32), smem, s, a, lay, err));
    return QMS_CUDA_OK;
}

int launch_gemv1(int type, const GemvArgs &a, int *err, cudaStream_t s) {
    QMS_REQUIRE(a.T == 1 && a.stride % 16 == 0 && ((uintptr_t)a.w & 15) == 0, QMS_CUDA_EINVAL,
                "gemv1: one token, 16-byte aligned rows");
    QMS_REQUIRE(a.ncol / 32 * 40 + 128 < 64 * 1024, QMS_CUDA_EUNSUPPORTED, "gemv1: rows of %d values", a.ncol);
    if (type == QMS_T_Q6_K) {
        const int units = a.ncol / 128;
        QMS_REQUIRE(a.ncol % 256 == 0 && units <= 32 && (units & (units - 1)) == 0, QMS_CUDA_EUNSUPPORTED,
                    "gemv1: Q6_K rows of %d values", a.ncol);
        return launch_gemv1_t<2, 1>(a, err, s);
    }
    const int nb = a.ncol / 32;
    QMS_REQUIRE(a.ncol % 32 == 0 && (nb < 32 ? (nb & (nb - 1)) == 0 : nb % 32 == 0 && nb <= 256),
                QMS_CUDA_EUNSUPPORTED, "gemv1: Q4 rows of %d values", a.ncol);
    const int nu = nb < 32 ? 1 : nb / 32;
    if (type == QMS_T_Q4_0) {
        switch (nu) {
        case 1: return launch_gemv1_t<0, 1>(a, err, s);
        case 2: return launch_gemv1_t<0, 2>(a, err, s);
        case 4: return launch_gemv1_t<0, 4>(a, err, s);
        case 8: return launch_gemv1_t<0, 8>(a, err, s);
        default: break;
        }
    } else if (type == QMS_T_Q4_1) {
        switch (nu) {
        case 1: return launch_gemv1_t<1, 1>(a, err, s);
        case 2: return launch_gemv1_t<1, 2>(a, err, s);
        case 4: return launch_gemv1_t<1, 4>(a, err, s);
        case 8: return launch_gemv1_t<1, 8>(a, err, s);
        default: break;
        }
    }
    set_error("gemv1: type %d with %d blocks per row not supported", type, nb);
    return QMS_CUDA_EUNSUPPORTED;
}

}  // namespace qms

// ---- one-token attention: QK-norm + RoPE + KV append fused, K/V staged in shared memory ------------
namespace qms {

// RMSNorm over one head row (D values, D/32 per lane at lane + 32 j) and the NEOX rotation at
// position p (src/model.c:403-422, 441-447); the warp returns the row in x.
template <int D>
__device__ __forceinline__ void norm_rope_row(float (&x)[D / 32], const float *nw, float eps, const float *cs,
                                              const float *sn, int lane) {
    constexpr int J = D / 32, JH = J / 2;
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < J; j++) ss = fma((double)x[j], (double)x[j], ss);
    ss = warp_sum_d(ss);
    const double inv = 1.0 / sqrt(ss / D + (double)eps);
#pragma unroll
    for (int j = 0; j < J; j++) x[j] = norm_elem(x[j], inv, nw, lane + 32 * j);
#pragma unroll
    for (int j = 0; j < JH; j++) {
        const int i = lane + 32 * j;
        const float c = cs[i], s = sn[i], x1 = x[j], x2 = x[j + JH];
        x[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        x[j + JH] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
}

// RMSNorm + NEOX rotation of one head row from preloaded values: x (the row), w (norm weights) and
// c / s (cos / sin of the position) as lane + 32 j (src/model.c:403-422, 441-447).
template <int D>
__device__ __forceinline__ void norm_rope_pre(float (&x)[D / 32], const float (&w)[D / 32], const float (&c)[D / 64],
                                              const float (&sn)[D / 64], float eps) {
    constexpr int J = D / 32, JH = J / 2;
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < J; j++) ss = fma((double)x[j], (double)x[j], ss);
    ss = warp_sum_d(ss);
    const double inv = 1.0 / sqrt(ss / D + (double)eps);
#pragma unroll
    for (int j = 0; j < J; j++) x[j] = __fmul_rn((float)((double)x[j] * inv), w[j]);
#pragma unroll
    for (int j = 0; j < JH; j++) {
        const float x1 = x[j], x2 = x[j + JH];
        x[j] = __fsub_rn(__fmul_rn(x1, c[j]), __fmul_rn(x2, sn[j]));
        x[j + JH] = __fadd_rn(__fmul_rn(x2, c[j]), __fmul_rn(x1, sn[j]));
    }
}

// CTA (kv head g, block s of kAttnBlock positions, sequence z) with group / HB warps; warp w owns q
// heads g * group + w * HB .. + HB. Scores: lane = position, each of the block's K rows read once
// from shared memory (rows padded to D + 4 floats: 16-byte aligned for cp.async, conflict-free
// float4 reads) for the warp's HB heads, each dot in qms_vec_dot_f32's order (sixteen FMA chains,
// then the hsum tree). P.V: lane = output dims, each V row read once for the HB heads. Every head's
// arithmetic is the same as with one warp per head; only the loads are shared. KT: the cache's
// element (fp32, or fp16 converted on each read); rows padded to D + 4 elements either way.
template <int D, int HB, typename KT>
__global__ void __launch_bounds__(512) k_attn_decode(const AttnArgs a) {
    constexpr int PB = kAttnBlock, KP = D + 4, J = D / 32, JH = J / 2, DPL = D / 32;
    __shared__ __align__(16) KT sk[PB * KP];
    __shared__ __align__(16) KT sv[PB * KP];
    __shared__ __align__(16) float sq[16 * D];
    const int group = a.H / a.Hk, g = blockIdx.x, s = blockIdx.y, z = blockIdx.z;   // z: sequence (batch)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x, nthr = blockDim.x;
    const int nwarps = nthr >> 5;
    pdl_trigger();
    pdl_wait();
    const int pos = a.pos_vec ? a.pos_vec[z] : *a.pos;
    if (pos < 0 || pos >= a.ctx) {
        if (tid == 0 && s == 0 && g == 0) atomicOr(a.err, 1);
        return;
    }
    const int npos = pos + 1, S = (npos + PB - 1) / PB;
    if (s >= S) {                                        // no positions here: an empty block for the merge
        if (lane == 0)
            for (int k = 0; k < HB; k++) {
                const size_t slot = ((size_t)z * a.H + g * group + warp * HB + k) * a.max_splits + s;
                a.part_ml[slot * 2] = -INFINITY;
                a.part_ml[slot * 2 + 1] = 0.0;
            }
        return;
    }
    const int p0 = s * PB, p1 = min(npos, p0 + PB), np = p1 - p0;
    const int KD = a.Hk * D;
    const size_t cb = (size_t)z * a.seq_stride;          // this sequence's caches (0 for one sequence)
    const float *qkv = a.qkv + (size_t)z * a.ldq;
    const bool has_new = p1 == npos && !a.q_ready;
    const int nc = a.q_ready ? np : min(p1, pos) - p0;   // cached rows (else the new one comes from qkv)
    for (int i = tid; i < nc * (D / 4); i += nthr) {
        const int p = i / (D / 4), d = 4 * (i % (D / 4));
        const size_t at = cb + (size_t)(p0 + p) * KD + (size_t)g * D + d;
        cp_async_kv4(sk + p * KP + d, static_cast<const KT *>(a.kc) + at);
        cp_async_kv4(sv + p * KP + d, static_cast<const KT *>(a.vc) + at);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // while the rows land: the group's q heads (QK-norm + NEOX RoPE) and the new position's rows
    const float *cs = a.rope_cos + (size_t)pos * (D / 2), *snp = a.rope_sin + (size_t)pos * (D / 2);
    float qw[J], kw[J], c[JH], sn[JH];
#pragma unroll
    for (int j = 0; j < J; j++) {
        qw[j] = __ldg(a.q_norm + lane + 32 * j);
        kw[j] = __ldg(a.k_norm + lane + 32 * j);
    }
#pragma unroll
    for (int j = 0; j < JH; j++) {
        c[j] = __ldg(cs + lane + 32 * j);
        sn[j] = __ldg(snp + lane + 32 * j);
    }
    for (int hh = warp; hh < group; hh += nwarps) {
        float qx[J];
#pragma unroll
        for (int j = 0; j < J; j++) qx[j] = __ldcg(qkv + (size_t)(g * group + hh) * D + lane + 32 * j);
        if (!a.q_ready) norm_rope_pre<D>(qx, qw, c, sn, a.eps);
#pragma unroll
        for (int j = 0; j < J; j++) sq[hh * D + lane + 32 * j] = qx[j];
    }
    if (has_new && warp == 0) {                               // the new position's K row, appended
        float kx[J];
#pragma unroll
        for (int j = 0; j < J; j++) kx[j] = __ldcg(qkv + (size_t)a.H * D + (size_t)g * D + lane + 32 * j);
        norm_rope_pre<D>(kx, kw, c, sn, a.eps);
#pragma unroll
        for (int j = 0; j < J; j++) {
            kv_st(sk + (pos - p0) * KP + lane + 32 * j, kx[j]);
            kv_st(static_cast<KT *>(a.kc) + cb + (size_t)pos * KD + (size_t)g * D + lane + 32 * j, kx[j]);
        }
    }
    if (has_new && warp == (nwarps > 1 ? 1 : 0)) {            // and its V row
#pragma unroll
        for (int j = 0; j < J; j++) {
            const float v = __ldcg(qkv + (size_t)(a.H + a.Hk) * D + (size_t)g * D + lane + 32 * j);
            kv_st(sv + (pos - p0) * KP + lane + 32 * j, v);
            kv_st(static_cast<KT *>(a.vc) + cb + (size_t)pos * KD + (size_t)g * D + lane + 32 * j, v);
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int h0 = warp * HB;                                 // this warp's first head within the group
    const bool valid = lane < np;
    double m[HB], l[HB];
    float fe[HB];
    {
        float acc[HB][16];
#pragma unroll
        for (int k = 0; k < HB; k++)
#pragma unroll
            for (int c2 = 0; c2 < 16; c2++) acc[k][c2] = 0.0f;
        if (valid) {
            const KT *kr = sk + lane * KP;
#pragma unroll
            for (int i = 0; i < D / 16; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 kv = kv_ld4(kr + 4 * (4 * i + j));
#pragma unroll
                    for (int k = 0; k < HB; k++) {
                        const float4 qv = reinterpret_cast<const float4 *>(sq + (h0 + k) * D)[4 * i + j];
                        acc[k][4 * j + 0] = __fmaf_rn(qv.x, kv.x, acc[k][4 * j + 0]);
                        acc[k][4 * j + 1] = __fmaf_rn(qv.y, kv.y, acc[k][4 * j + 1]);
                        acc[k][4 * j + 2] = __fmaf_rn(qv.z, kv.z, acc[k][4 * j + 2]);
                        acc[k][4 * j + 3] = __fmaf_rn(qv.w, kv.w, acc[k][4 * j + 3]);
                    }
                }
        }
#pragma unroll
        for (int k = 0; k < HB; k++) {
            float t[8];
#pragma unroll
            for (int c2 = 0; c2 < 8; c2++) t[c2] = __fadd_rn(acc[k][c2], acc[k][c2 + 8]);
#pragma unroll
            for (int c2 = 0; c2 < 4; c2++) t[c2] = __fadd_rn(t[c2], t[c2 + 4]);
            t[0] = __fadd_rn(t[0], t[2]);
            t[1] = __fadd_rn(t[1], t[3]);
            const double sc = valid ? (double)__fadd_rn(t[0], t[1]) * a.scale : -INFINITY;
            m[k] = warp_max_d(sc);
            const double e = valid ? exp(sc - m[k]) : 0.0;
            l[k] = warp_sum_d(e);
            fe[k] = (float)e;
        }
    }
    float o[HB][DPL];
#pragma unroll
    for (int k = 0; k < HB; k++)
#pragma unroll
        for (int d = 0; d < DPL; d++) o[k][d] = 0.0f;
    for (int q = 0; q < np; q++) {
        const KT *vp = sv + q * KP + lane * DPL;
        float v[DPL];
        if constexpr (DPL == 4) {
            const float4 t4 = kv_ld4(vp);
            v[0] = t4.x; v[1] = t4.y; v[2] = t4.z; v[3] = t4.w;
        } else {
            const float2 t2 = kv_ld2(vp);
            v[0] = t2.x; v[1] = t2.y;
        }
#pragma unroll
        for (int k = 0; k < HB; k++) {
            const float w = __shfl_sync(0xffffffffu, fe[k], q);
#pragma unroll
            for (int d = 0; d < DPL; d++) o[k][d] = __fmaf_rn(w, v[d], o[k][d]);
        }
    }
#pragma unroll
    for (int k = 0; k < HB; k++) {
        const int h = g * group + h0 + k;
        const size_t slot = ((size_t)z * a.H + h) * a.max_splits + s;
#pragma unroll
        for (int d = 0; d < DPL; d++) a.part_o[slot * D + lane * DPL + d] = o[k][d];
        if (lane == 0) {
            a.part_ml[slot * 2] = m[k];
            a.part_ml[slot * 2 + 1] = l[k];
        }
    }
}

// One CTA per q head: merge the S position blocks (flash-decoding), divide by the softmax sum and
// write the head's Q8 blocks (the O projection's input, src/kernels.c:34-53).
template <int D>
__global__ void __launch_bounds__(4 * D) k_attn_merge(const AttnArgs a, int8_t *xq, float *xd, int *xs) {
    constexpr int NT = 4 * D, NW = NT / 32;
    __shared__ float f[kAttnMaxCtx / kAttnBlock];
    __shared__ double red[NW];
    __shared__ float part[4][D];
    const int h = blockIdx.x, z = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    pdl_wait();
    // every block slot: the ones past the position hold an empty block (m = -inf, l = 0), so the
    // position need not be read first (one dependent round trip less); their weights are zero
    const int S = a.max_splits;                         // <= NT (the launch checks ctx)
    const size_t base = ((size_t)z * a.H + h) * a.max_splits;
    const bool own = tid < S;
    const double mq = own ? __ldcg(a.part_ml + (base + tid) * 2) : -INFINITY;
    const double lq = own ? __ldcg(a.part_ml + (base + tid) * 2 + 1) : 0.0;
    double mx = warp_max_d(mq);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    double M = red[0];
    for (int i = 1; i < NW; i++) M = fmax(M, red[i]);
    const double fq = own ? exp(mq - M) : 0.0;
    if (own) f[tid] = (float)fq;
    const double zw = warp_sum_d(lq * fq);
    __syncthreads();
    if (lane == 0) red[warp] = zw;
    __syncthreads();
    double Z = 0.0;
    for (int i = 0; i < NW; i++) Z += red[i];
    // quarter pt of the splits for dimension d, loads issued eight at a time
    const int pt = tid / D, d = tid % D;
    float acc = 0.0f;
    for (int q0 = pt; q0 < S; q0 += 32) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int q = q0 + 4 * u;
            v[u] = q < S && f[q] != 0.0f ? __ldcg(a.part_o + (base + q) * D + d) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (q0 + 4 * u < S) acc = __fmaf_rn(f[q0 + 4 * u], v[u], acc);
    }
    part[pt][d] = acc;
    __syncthreads();
    if (tid >= D) return;
    const float o = __fadd_rn(__fadd_rn(part[0][tid], part[1][tid]), __fadd_rn(part[2][tid], part[3][tid]));
    const float val = (float)((double)o / Z);
    const Q8Lane r = quantize_lane(val);
    const size_t e = (size_t)z * a.H * D + (size_t)h * D + tid;
    xq[e] = (int8_t)r.q;
    if (lane == 0) {
        xd[e / 32] = r.d;
        xs[e / 32] = pack_sums(r);
    }
}

template <int D>
static cudaError_t launch_attn_decode_d(const AttnArgs &a, int hb, dim3 grid, dim3 block, cudaStream_t s) {
    if (a.kv16) {
        if (hb == 4) return launch_pdl(k_attn_decode<D, 4, __half>, grid, block, 0, s, a);
        if (hb == 2) return launch_pdl(k_attn_decode<D, 2, __half>, grid, block, 0, s, a);
        return launch_pdl(k_attn_decode<D, 1, __half>, grid, block, 0, s, a);
    }
    if (hb == 4) return launch_pdl(k_attn_decode<D, 4, float>, grid, block, 0, s, a);
    if (hb == 2) return launch_pdl(k_attn_decode<D, 2, float>, grid, block, 0, s, a);
    return launch_pdl(k_attn_decode<D, 1, float>, grid, block, 0, s, a);
}

int launch_attn_decode(const AttnArgs &a, int8_t *xq, float *xd, int *xs, cudaStream_t s) {
    const int group = a.H / a.Hk;
    QMS_REQUIRE(group <= 16 && (a.T == 1 || a.pos_vec) && a.T <= 65535 && a.max_splits <= kAttnMaxCtx / kAttnBlock &&
                    a.max_splits * kAttnBlock >= a.ctx && a.max_splits <= 4 * a.D,
                QMS_CUDA_EUNSUPPORTED, "attn_decode: %d q heads per kv head, ctx %d", group, a.ctx);
    // heads per warp: 2 for one sequence (more warps shorten the latency-bound chain: 13.8 / 16.7 us
    // per 235B layer at positions 1024 / 2900 against 16.1 / 18.2 with 4), 4 for a batch (shared-
    // memory traffic bounds the throughput)
    const int hmax = a.pos_vec ? 4 : 2, hb = group < hmax ? group : hmax;
    QMS_REQUIRE(group % hb == 0, QMS_CUDA_EUNSUPPORTED, "attn_decode: %d q heads per kv head", group);
    const dim3 grid(a.Hk, a.max_splits, a.T), block(32 * (group / hb));
    if (a.D == 128) QMS_CK(launch_attn_decode_d<128>(a, hb, grid, block, s));
    else QMS_CK(launch_attn_decode_d<64>(a, hb, grid, block, s));
    if (a.D == 128) QMS_CK(launch_pdl(k_attn_merge<128>, dim3(a.H, a.T), dim3(512), 0, s, a, xq, xd, xs));
    else QMS_CK(launch_pdl(k_attn_merge<64>, dim3(a.H, a.T), dim3(256), 0, s, a, xq, xd, xs));
    return QMS_CUDA_OK;
}

}  // namespace qms

