// qms_moe.cu - the Qwen3-MoE feed-forward block on B200 (sm_100a): layer lifetime, the general
// (any T) kernels and the host entry points.
//
// Reference: moe() in src/model.c:1032-1167 with moe_group_fast (src/model.c:969-1007).
// Batch-1 decode (T == 1) runs the streaming kernels of qms_moe_stream.cu. Other T run:
//   k_moe_router   T <= 4: X CTAs: Q8 quantisation of xn (src/kernels.c:34-53), router logits
//                  in the reference's exact F32 order (src/kernels.c:202-219); the last CTA to
//                  finish does softmax / top-k / renormalisation (src/model.c:1045-1064).
//   larger T       k_quantize_rows, k_router_tiled (the same exact-order logits, tiled over
//                  up to 32 tokens x 32 experts in shared memory), k_moe_topk (one CTA per token).
// T >= 5 then runs the expert-grouped kernels (qms_moe_gemv.cu while experts average <= 24 slots,
// qms_moe_mma.cu above); T = 2..4 the per-slot kernels below:
//   k_moe_gate_up  one warp per (slot, f): gate row f and up row f of the slot's expert against
//                  the token's Q8 row (phase 1, :979-988), a = silu(g) * u (:994); the CTA that
//                  completes a 32-row group re-quantises it to Q8 (phase 2, :995).
//   k_moe_down     one CTA per (token, 32 output rows): down rows of all n_used experts
//                  (phase 3, :998-1005), then the weighted sum in selection order with one
//                  fused multiply-add per expert (:1152-1162), plus the optional residual.
// Expert weights are repacked at load into the staged layouts of qms_moe.cuh; from host memory
// they stream through a pinned staging ring (upload_q4).
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "qms_moe.cuh"
#include "qms_router.cuh"

using namespace qms;

namespace qms {

constexpr int kGateUpRows = 8;         // f values per gate/up CTA (one per warp)
constexpr int kDownRows = 32;          // output rows per down CTA (one per lane)
constexpr int kMmaMinT = 5;            // tokens from which the expert-grouped kernels run (GEMV, tensor cores):
                                        // measured 158 vs 325 us (T = 8) and 190 vs 463 us (T = 12) against
                                        // the per-slot dp4a kernels on a 235B layer

// ---- load-time repack: GGUF rows -> staged layouts (qms_moe.cuh) --------------------------------
// gate (which 0) / up (which 1) Q4_0 rows of a stacked [X][F] tensor -> chunks
// (rows row0 .. row0 + nrows - 1 of the tensor; src points at row row0)
__global__ void k_repack_gu(const uint8_t *__restrict__ src, int64_t row0, int64_t nrows, int nb, int F, int which,
                            Chunked c, uint8_t *__restrict__ dst, size_t expert_bytes) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nrows * nb) return;
    const int64_t R = row0 + idx / nb;
    const int b = (int)(idx % nb);
    const int e = (int)(R / F), row = (int)(R % F);
    const uint16_t *s = reinterpret_cast<const uint16_t *>(src + idx * 18);
    const int rr = (which * 32 + (row & 31)) & 7;
    uint8_t *cp = dst + (size_t)e * expert_bytes + gu_chunk(c, row, which, b) * c.GB;
    uint4 v;
    v.x = (uint32_t)s[1] | ((uint32_t)s[2] << 16);
    v.y = (uint32_t)s[3] | ((uint32_t)s[4] << 16);
    v.z = (uint32_t)s[5] | ((uint32_t)s[6] << 16);
    v.w = (uint32_t)s[7] | ((uint32_t)s[8] << 16);
    *reinterpret_cast<uint4 *>(cp + chunk_nib_off(c.SB, rr, b % c.SB)) = v;
    *reinterpret_cast<uint16_t *>(cp + chunk_scale_off(c.SB, rr, b % c.SB)) = s[0];
}

// down Q4_0 / Q4_1 rows of a stacked [X][E] tensor -> column stages; a Q4_1 block {d, m, qs[16]}
// keeps d in the scale plane and m in the min plane
__global__ void k_repack_dn(const uint8_t *__restrict__ src, int64_t row0, int64_t nrows, int nb, int E, DnCols d,
                            uint8_t *__restrict__ dst, size_t expert_bytes) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nrows * nb) return;
    const int64_t R = row0 + idx / nb;
    const int b = (int)(idx % nb);
    const int e = (int)(R / E), row = (int)(R % E);
    const uint16_t *s = reinterpret_cast<const uint16_t *>(src + idx * (d.q1 ? 20 : 18)) + d.q1;
    uint8_t *sp = dst + (size_t)e * expert_bytes + dn_stage_off(d, b, row);
    uint4 v;
    v.x = (uint32_t)s[1] | ((uint32_t)s[2] << 16);
    v.y = (uint32_t)s[3] | ((uint32_t)s[4] << 16);
    v.z = (uint32_t)s[5] | ((uint32_t)s[6] << 16);
    v.w = (uint32_t)s[7] | ((uint32_t)s[8] << 16);
    *reinterpret_cast<uint4 *>(sp + dn_nib_off(d, row)) = v;
    *reinterpret_cast<uint16_t *>(sp + dn_scale_off(d, row)) = s[-d.q1];
    if (d.q1) *reinterpret_cast<uint16_t *>(sp + dn_min_off(d, row)) = s[0];
}

// ---- router: quantise xn, logits, (last CTA) top-k --------------------------------------------
__global__ void __launch_bounds__(256) k_moe_router(const float *__restrict__ W, int X, int E, const float *__restrict__ xn,
                                                    int T, int K, int8_t *__restrict__ xq_q, float *__restrict__ xq_d,
                                                    int *__restrict__ xq_s, float *__restrict__ logits,
                                                    int *__restrict__ sel, float *__restrict__ wts,
                                                    int *__restrict__ cnt, int do_topk) {
    extern __shared__ float4 smem4[];
    float *srow = reinterpret_cast<float *>(smem4);
    __shared__ int s_last;
    pdl_trigger();
    const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nbE = E / 32;
    // (0) Q8 rows of xn: block b = e + X*m, one warp per block
    for (int64_t b = e + (int64_t)X * warp; b < (int64_t)T * nbE; b += (int64_t)X * 8) {
        const Q8Lane r = quantize_lane(xn[b * 32 + lane]);
        xq_q[b * 32 + lane] = (int8_t)r.q;
        if (lane == 0) {
            xq_d[b] = r.d;
            xq_s[b] = r.sum;
        }
    }
    // (1) router row e into shared memory
    const float4 *src = reinterpret_cast<const float4 *>(W + (size_t)e * E);
    for (int i = tid; i < E / 4; i += blockDim.x) smem4[i] = __ldg(src + i);
    __syncthreads();
    // (2) logits[t][e], 16 threads per token
    const int grp = tid >> 4, k = tid & 15;
    for (int t0 = 0; t0 < T; t0 += 16) {
        const int t = t0 + grp;
        const bool valid = t < T;
        const float v = dot_f32_exact16(srow, xn + (size_t)(valid ? t : 0) * E, E, k);
        if (valid && k == 0) {
            logits[(size_t)t * X + e] = v;
            __threadfence();
        }
    }
    if (!do_topk) return;
    // (3) the last CTA to finish ranks the experts of every token
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(cnt, 1) == X - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    __shared__ int s_sel[64];
    for (int t = 0; t < T; t++) topk_token(logits + (size_t)t * X, X, K, sel + t * K, wts + t * K, s_sel);
    if (tid == 0) *cnt = 0;
}

__global__ void __launch_bounds__(256) k_moe_topk(const float *__restrict__ logits, int X, int K, int *__restrict__ sel,
                                                  float *__restrict__ wts) {
    __shared__ int s_sel[64];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    topk_token(logits + (size_t)t * X, X, K, sel + t * K, wts + t * K, s_sel);
}

// QmsQ8 blocks (the reference's activation block, src/kernels.h:7-12) -> the planar Q8 rows the
// grouped kernels read: values, scale, block sum (s16[0] + s16[1]). One thread per block.
__global__ void __launch_bounds__(256) k_unpack_q8(const QmsQ8 *__restrict__ x, int64_t nblocks, int8_t *__restrict__ xq_q,
                                                   float *__restrict__ xq_d, int *__restrict__ xq_s) {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
        const QmsQ8 *blk = x + b;
        const int *q = reinterpret_cast<const int *>(blk->q);             // 4-byte aligned inside the 44-byte block
        int4 *dst = reinterpret_cast<int4 *>(xq_q + b * 32);
        dst[0] = make_int4(__ldg(q + 0), __ldg(q + 1), __ldg(q + 2), __ldg(q + 3));
        dst[1] = make_int4(__ldg(q + 4), __ldg(q + 5), __ldg(q + 6), __ldg(q + 7));
        xq_d[b] = __ldg(&blk->d);
        xq_s[b] = (int)__ldg(&blk->s16[0]) + (int)__ldg(&blk->s16[1]);
    }
}

// ---- router for larger T: Q8 rows, then logits tiled over (tokens x experts) ----------------------
// One warp per 32-block of xn: the quantiser of src/kernels.c:34-53.
__global__ void __launch_bounds__(256) k_quantize_rows(const float *__restrict__ xn, int64_t nblocks,
                                                       int8_t *__restrict__ xq_q, float *__restrict__ xq_d,
                                                       int *__restrict__ xq_s) {
    const int lane = threadIdx.x & 31;
    pdl_wait();
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; b < nblocks;
         b += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const Q8Lane r = quantize_lane(xn[b * 32 + lane]);
        xq_q[b * 32 + lane] = (int8_t)r.q;
        if (lane == 0) {
            xq_d[b] = r.d;
            xq_s[b] = r.sum;
        }
    }
}

// logits[t][e] for a tile of 4A tokens x 4A experts per CTA, in qms_vec_dot_f32's exact order
// (src/kernels.c:202-219): thread (k, g) runs lane k's FMA chain for A tokens x A experts over
// shared-memory chunks of 1024/A elements (the next chunk is loaded into registers while this one
// is used), then the 16 lanes of a pair reduce with offsets 8, 4, 2, 1. A = 8 for large T; smaller
// tiles give small batches more CTAs.
template <int A>
__global__ void __launch_bounds__(256) k_router_tiled(const float *__restrict__ W, int X, int E,
                                                      const float *__restrict__ xn, int T, float *__restrict__ logits) {
    constexpr int R = 4 * A, C = 1024 / A, S = C + 4, NV = R * C / 4 / 256;   // rows, chunk, stride, float4 per thread
    __shared__ __align__(16) float xs[R * S], ws[R * S];
    const int tid = threadIdx.x, k = tid & 15, g = tid >> 4, gt = g >> 2, ge = g & 3;
    const int t0 = blockIdx.x * R, e0 = blockIdx.y * R;
    pdl_wait();
    float acc[A][A];
#pragma unroll
    for (int a = 0; a < A; a++)
#pragma unroll
        for (int b = 0; b < A; b++) acc[a][b] = 0.0f;
    float4 px[NV], pw[NV];
    auto fetch = [&](int c0) {
#pragma unroll
        for (int v = 0; v < NV; v++) {
            const int i = tid + 256 * v, r = i / (C / 4), c = (i % (C / 4)) * 4;
            const int t = t0 + r, e = e0 + r;
            const bool in = c0 + c < E;
            px[v] = in && t < T ? __ldg(reinterpret_cast<const float4 *>(xn + (size_t)t * E + c0 + c))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            pw[v] = in && e < X ? __ldg(reinterpret_cast<const float4 *>(W + (size_t)e * E + c0 + c))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    fetch(0);
    for (int c0 = 0; c0 < E; c0 += C) {
        __syncthreads();
#pragma unroll
        for (int v = 0; v < NV; v++) {
            const int i = tid + 256 * v, r = i / (C / 4), c = (i % (C / 4)) * 4;
            *reinterpret_cast<float4 *>(xs + r * S + c) = px[v];
            *reinterpret_cast<float4 *>(ws + r * S + c) = pw[v];
        }
        __syncthreads();
        if (c0 + C < E) fetch(c0 + C);
        const int len = min(C, E - c0);
#pragma unroll 2
        for (int st = 0; st < len / 16; st++) {
            const int c = 16 * st + k;
            float xv[A], wv[A];
#pragma unroll
            for (int a = 0; a < A; a++) xv[a] = xs[(gt * A + a) * S + c];
#pragma unroll
            for (int b = 0; b < A; b++) wv[b] = ws[(ge * A + b) * S + c];
#pragma unroll
            for (int a = 0; a < A; a++)
#pragma unroll
                for (int b = 0; b < A; b++) acc[a][b] = __fmaf_rn(xv[a], wv[b], acc[a][b]);
        }
    }
#pragma unroll
    for (int a = 0; a < A; a++)
#pragma unroll
        for (int b = 0; b < A; b++) {
            float v = acc[a][b];
            v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8, 16));
            v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 16));
            v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 16));
            v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 16));
            const int t = t0 + gt * A + a, e = e0 + ge * A + b;
            if (k == 0 && t < T && e < X) logits[(size_t)t * X + e] = v;
        }
}

// CTAs of the tiled router for tile side 4A
static int64_t router_ctas(int T, int X, int A) { return (int64_t)((T + 4 * A - 1) / (4 * A)) * ((X + 4 * A - 1) / (4 * A)); }

// Router stage for any T: the fused one-kernel router for T <= kTopkInRouterMaxT, else quantiser,
// tiled logits and one top-k CTA per token.
static int launch_router(const float *router, int X, int E, const float *xn, int T, int K, int8_t *xq_q, float *xq_d,
                         int *xq_s, float *lg, int *sel, float *wts, int *cnt, cudaStream_t s) {
    if (T <= kTopkInRouterMaxT || ((uintptr_t)xn & 15) || ((uintptr_t)router & 15)) {
        const int fused = T <= kTopkInRouterMaxT;
        k_moe_router<<<X, 256, (size_t)E * 4, s>>>(router, X, E, xn, T, K, xq_q, xq_d, xq_s, lg, sel, wts, cnt, fused);
        QMS_CK(cudaGetLastError());
        if (!fused) QMS_CK(launch_pdl(k_moe_topk, dim3(T), dim3(256), 0, s, (const float *)lg, X, K, sel, wts));
        return QMS_CUDA_OK;
    }
    const int64_t nblocks = (int64_t)T * (E / 32);
    const unsigned qgrid = (unsigned)std::min<int64_t>((nblocks + 7) / 8, 4096);
    k_quantize_rows<<<qgrid, 256, 0, s>>>(xn, nblocks, xq_q, xq_d, xq_s);
    QMS_CK(cudaGetLastError());
    const int A = router_ctas(T, X, 8) >= 296 ? 8 : router_ctas(T, X, 4) >= 296 ? 4 : 2;
    const dim3 rgrid((T + 4 * A - 1) / (4 * A), (X + 4 * A - 1) / (4 * A));
    if (A == 8) QMS_CK(launch_pdl(k_router_tiled<8>, rgrid, dim3(256), 0, s, router, X, E, xn, T, lg));
    else if (A == 4) QMS_CK(launch_pdl(k_router_tiled<4>, rgrid, dim3(256), 0, s, router, X, E, xn, T, lg));
    else QMS_CK(launch_pdl(k_router_tiled<2>, rgrid, dim3(256), 0, s, router, X, E, xn, T, lg));
    QMS_CK(launch_pdl(k_moe_topk, dim3(T), dim3(256), 0, s, (const float *)lg, X, K, sel, wts));
    return QMS_CUDA_OK;
}

// ---- gate/up + SwiGLU + Q8 re-quantisation (any T) -------------------------------------------
template <int NBL>
__global__ void __launch_bounds__(256) k_moe_gate_up(const uint8_t *__restrict__ gu, size_t gu_expert, Chunked c,
                                                     int nbE, int F, int K, const int8_t *__restrict__ xq_q,
                                                     const float *__restrict__ xq_d, const int *__restrict__ xq_s,
                                                     const int *__restrict__ sel, float *__restrict__ act,
                                                     int8_t *__restrict__ aq_q, float *__restrict__ aq_d,
                                                     int *__restrict__ aq_s, int *__restrict__ gcnt) {
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int f = blockIdx.x * kGateUpRows + warp;
    const int slot = blockIdx.y, t = slot / K;
    pdl_wait();
    const int e = __ldcg(sel + slot);
    const uint8_t *ge = gu + (size_t)e * gu_expert;
    const int rr = f & 7;
    uint4 ng[NBL], nu[NBL];
    uint16_t sg[NBL], su[NBL];
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        const int b = lane + 32 * i;
        if (b < nbE) {
            const uint8_t *cg = ge + gu_chunk(c, f, 0, b) * c.GB;
            const uint8_t *cu = cg + 4 * (size_t)c.GB;          // up rows: chunks 4-7 of the stage
            const int bl = b % c.SB;
            ng[i] = ld_stream16(cg + chunk_nib_off(c.SB, rr, bl));
            nu[i] = ld_stream16(cu + chunk_nib_off(c.SB, rr, bl));
            sg[i] = ld_stream2(cg + chunk_scale_off(c.SB, rr, bl));
            su[i] = ld_stream2(cu + chunk_scale_off(c.SB, rr, bl));
        }
    }
    const int8_t *xq = xq_q + (size_t)t * nbE * 32;
    float g = 0.0f, u = 0.0f;
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        const int b = lane + 32 * i;
        if (b < nbE) {
            const int4 xa0 = __ldcg(reinterpret_cast<const int4 *>(xq + b * 32));
            const int4 xa1 = __ldcg(reinterpret_cast<const int4 *>(xq + b * 32 + 16));
            const float xd = __ldcg(xq_d + (size_t)t * nbE + b);
            const int xs8 = 8 * __ldcg(xq_s + (size_t)t * nbE + b);
            g = fmaf((float)(q4_block_isum(ng[i], xa0, xa1) - xs8), h2f(sg[i]) * xd, g);
            u = fmaf((float)(q4_block_isum(nu[i], xa0, xa1) - xs8), h2f(su[i]) * xd, u);
        }
    }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) {
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        act[(size_t)slot * F + f] = __fmul_rn(s, u);
        __threadfence();
    }
    __syncthreads();
    pdl_trigger();
    const int nbF = F / 32, grp = f / 32;
    int *cn = gcnt + (size_t)slot * nbF + grp;
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(cn, kGateUpRows) == 32 - kGateUpRows;
    }
    __syncthreads();
    if (s_last && warp == 0) {
        __threadfence();
        const size_t base = (size_t)slot * F + (size_t)grp * 32;
        const Q8Lane r = quantize_lane(__ldcg(act + base + lane));
        aq_q[base + lane] = (int8_t)r.q;
        if (lane == 0) {
            aq_d[(size_t)slot * nbF + grp] = r.d;
            aq_s[(size_t)slot * nbF + grp] = r.sum;
            *cn = 0;
        }
    }
}

// ---- down + weighted combine (+ residual), any T ----------------------------------------------
// One CTA per (kDownRows output rows, token): warp k computes those rows of expert slot k (lane =
// row), blocks in order, reading 512 contiguous bytes of nibbles per block from the column
// stages; the token's K Q8 activation rows are staged in shared memory first.
__global__ void __launch_bounds__(256) k_moe_down(const uint8_t *__restrict__ dn, size_t dn_expert, DnCols dc,
                                                  int nbF, int E, int K, const int8_t *__restrict__ aq_q,
                                                  const float *__restrict__ aq_d, const int *__restrict__ aq_s,
                                                  const int *__restrict__ sel, const float *__restrict__ wts,
                                                  const float *resid, float *out) {
    extern __shared__ __align__(16) uint8_t sdm[];
    const int F = nbF * 32, t = blockIdx.y, i0 = blockIdx.x * kDownRows;
    int8_t *sq = reinterpret_cast<int8_t *>(sdm);                   // [K][F]
    float *sd = reinterpret_cast<float *>(sdm + (size_t)K * F);     // [K][nbF]
    int *ss = reinterpret_cast<int *>(sd + K * nbF);                // [K][nbF] block sums
    float *sdn = reinterpret_cast<float *>(ss + K * nbF);           // [K][kDownRows]
    pdl_wait();
    const int4 *gq = reinterpret_cast<const int4 *>(aq_q + (size_t)t * K * F);
    for (int i = threadIdx.x; i < K * F / 16; i += blockDim.x) reinterpret_cast<int4 *>(sq)[i] = __ldcg(gq + i);
    for (int i = threadIdx.x; i < K * nbF; i += blockDim.x) {
        sd[i] = __ldcg(aq_d + (size_t)t * K * nbF + i);
        ss[i] = __ldcg(aq_s + (size_t)t * K * nbF + i);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = i0 + lane;
    for (int k = warp; k < K; k += blockDim.x >> 5) {
        const uint8_t *de = dn + (size_t)__ldcg(sel + t * K + k) * dn_expert;
        const int8_t *xq = sq + (size_t)k * F;
        float acc = 0.0f;
#pragma unroll 4
        for (int b = 0; b < nbF; b++) {
            const uint8_t *st = de + dn_stage_off(dc, b, row);
            const uint4 nib = ld_stream16(st + dn_nib_off(dc, row));
            const float dw = h2f(ld_stream2(st + dn_scale_off(dc, row)));
            const int4 xa0 = *reinterpret_cast<const int4 *>(xq + b * 32);
            const int4 xa1 = *reinterpret_cast<const int4 *>(xq + b * 32 + 16);
            const float xd = sd[k * nbF + b];
            const int xs = ss[k * nbF + b];
            if (dc.q1) {                            // d q + m: d dx isum + m ds (src/kernels.c:109-121)
                const float mw = h2f(ld_stream2(st + dn_min_off(dc, row)));
                acc = fmaf((float)q4_block_isum(nib, xa0, xa1), dw * xd, acc);
                acc = fmaf(mw, xd * (float)xs, acc);
            } else {                                // d (q - 8): the -8 folded into the block sum
                acc = fmaf((float)(q4_block_isum(nib, xa0, xa1) - 8 * xs), dw * xd, acc);
            }
        }
        sdn[k * kDownRows + lane] = acc;
    }
    __syncthreads();
    if (threadIdx.x < kDownRows) {
        const int i = i0 + threadIdx.x;
        float o = 0.0f;
        for (int j = 0; j < K; j++) o = __fmaf_rn(__ldcg(wts + t * K + j), sdn[j * kDownRows + threadIdx.x], o);
        if (resid) o = __fadd_rn(resid[(size_t)t * E + i], o);
        out[(size_t)t * E + i] = o;
    }
}

static size_t down_smem(const QmsCudaMoe *m) {
    return (size_t)m->K * m->F + (size_t)m->K * m->nbF * 8 + (size_t)m->K * kDownRows * 4;
}

// Lane-major copy of the router for the batch-1 kernel: row e, element 16*i + k at [e][k][i].
__global__ void k_router_lane_major(const float *__restrict__ W, int X, int E, float *__restrict__ Wlm) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)X * E) return;
    const int64_t e = idx / E;
    const int j = (int)(idx % E), L = E / 16;
    Wlm[e * E + (int64_t)(j & 15) * L + (j >> 4)] = W[idx];
}

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

static int ensure_device(int dev) {
    int cur = -1;
    QMS_CK(cudaGetDevice(&cur));
    if (cur != dev) QMS_CK(cudaSetDevice(dev));
    return QMS_CUDA_OK;
}

// Upload one stacked expert tensor (host or device source) and repack it: which = 0 / 1 gate / up
// rows into chunks, which = 2 down rows into column stages.
// Host-memory uploads go through a ring of two pinned host buffers and two device buffers of
// kStageBytes: host threads copy chunk i + 1 into pinned memory while chunk i's DMA and repack
// run on the upload stream, so a layer streams at the link rate instead of through the driver's
// pageable-copy path, and no device buffer the size of a whole tensor is needed.
constexpr size_t kStageBytes = 64u << 20;
constexpr int kStageThreads = 8;

struct UploadRing {
    uint8_t *h[2] = {nullptr, nullptr};   // pinned host
    uint8_t *d[2] = {nullptr, nullptr};   // device
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaStream_t s = nullptr;
    size_t cap = 0;                       // bytes per buffer
    int used[2] = {0, 0};

    int open(size_t largest) {            // largest: bytes of the biggest tensor to upload
        cap = std::min(kStageBytes, (largest + 4095) & ~(size_t)4095);
        for (int i = 0; i < 2; i++) {
            if (cudaHostAlloc(&h[i], cap, cudaHostAllocDefault) != cudaSuccess || cudaMalloc(&d[i], cap) != cudaSuccess ||
                cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                set_error("moe_create: cannot set up the %zu-byte upload ring", cap);
                return QMS_CUDA_ENOMEM;
            }
        }
        QMS_CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        return QMS_CUDA_OK;
    }
    ~UploadRing() {
        if (s) cudaStreamSynchronize(s);
        for (int i = 0; i < 2; i++) {
            if (h[i]) cudaFreeHost(h[i]);
            if (d[i]) cudaFree(d[i]);
            if (ev[i]) cudaEventDestroy(ev[i]);
        }
        if (s) cudaStreamDestroy(s);
    }
};

// memcpy of n bytes split over up to kStageThreads host threads
static void parallel_copy(uint8_t *dst, const uint8_t *src, size_t n) {
    const int nt = (int)std::min<size_t>(kStageThreads, std::max<size_t>(1, n >> 22));
    if (nt <= 1) {
        memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    const size_t per = (n + nt - 1) / nt;
    for (int t = 0; t < nt; t++) {
        const size_t a = (size_t)t * per, b = std::min(n, a + per);
        if (a < b) th.emplace_back([=] { memcpy(dst + a, src + a, b - a); });
    }
    for (auto &x : th) x.join();
}

static int launch_repack(const QmsCudaMoe *m, int which, const uint8_t *src, int64_t row0, int64_t nrows, uint8_t *dst,
                         cudaStream_t s) {
    const int nb = which == 2 ? m->nbF : m->nbE;
    const int64_t n = nrows * nb;
    const unsigned grid = (unsigned)((n + 255) / 256);
    if (which == 2) k_repack_dn<<<grid, 256, 0, s>>>(src, row0, nrows, nb, m->E, m->dcol, dst, m->dn_expert);
    else k_repack_gu<<<grid, 256, 0, s>>>(src, row0, nrows, nb, m->F, which, m->cgu, dst, m->gu_expert);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

static int upload_q4(const QmsCudaMoe *m, const void *src, int on_device, int which, uint8_t *dst, UploadRing *ring) {
    const int64_t nrows = (int64_t)m->n_local * (which == 2 ? m->E : m->F);
    const int nb = which == 2 ? m->nbF : m->nbE;
    const size_t rb = (size_t)nb * (which == 2 && m->dcol.q1 ? 20 : 18);
    int rc;
    if (on_device) {
        if ((rc = launch_repack(m, which, (const uint8_t *)src, 0, nrows, dst, 0))) return rc;
    } else {
        const int64_t per = (int64_t)(ring->cap / rb);
        int slot = 0;
        for (int64_t r0 = 0; r0 < nrows; r0 += per, slot ^= 1) {
            const int64_t nr = std::min<int64_t>(per, nrows - r0);
            if (ring->used[slot]) QMS_CK(cudaEventSynchronize(ring->ev[slot]));   // its last DMA and repack are done
            parallel_copy(ring->h[slot], (const uint8_t *)src + (size_t)r0 * rb, (size_t)nr * rb);
            QMS_CK(cudaMemcpyAsync(ring->d[slot], ring->h[slot], (size_t)nr * rb, cudaMemcpyHostToDevice, ring->s));
            if ((rc = launch_repack(m, which, ring->d[slot], r0, nr, dst, ring->s))) return rc;
            QMS_CK(cudaEventRecord(ring->ev[slot], ring->s));
            ring->used[slot] = 1;
        }
        QMS_CK(cudaStreamSynchronize(ring->s));
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_error("moe_create: repack failed: %s", cudaGetErrorString(e));
        return QMS_CUDA_ECUDA;
    }
    return QMS_CUDA_OK;
}

}  // namespace qms

extern "C" {

void qms_cuda_moe_destroy(QmsCudaMoe *m) {
    if (!m) return;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(m->device);
    cudaFree(m->router);
    cudaFree(m->router_lm);
    cudaFree(m->gu);
    cudaFree(m->dn);
    cudaFree(m->scratch);
    cudaFree(m->d_in);
    cudaFree(m->d_out);
    if (m->hstream) cudaStreamDestroy(m->hstream);
    if (cur >= 0) cudaSetDevice(cur);
    free(m);
}

static int create_impl(const QmsCudaMoeDesc *d, int base, int n_local, QmsCudaMoe **out) {
    clear_error();
    QMS_REQUIRE(d && out, QMS_CUDA_EINVAL, "moe_create: NULL argument");
    *out = nullptr;
    const int E = d->n_embd, X = d->n_expert, K = d->n_used, F = d->n_ff;
    QMS_REQUIRE(base >= 0 && n_local >= 1 && base + n_local <= X, QMS_CUDA_EINVAL,
                "moe_create_shard: experts [%d, %d) outside 0..%d", base, base + n_local, X);
    QMS_REQUIRE(d->router && d->gate && d->up && d->down, QMS_CUDA_EINVAL, "moe_create: NULL tensor");
    QMS_REQUIRE(E > 0 && X > 0 && K > 0 && F > 0 && K <= X, QMS_CUDA_EINVAL, "moe_create: bad dimensions");
    // the reference's integer fast path condition (src/model.c:1090-1093)
    QMS_REQUIRE(E % 256 == 0 && F % 32 == 0, QMS_CUDA_EUNSUPPORTED,
                "moe_create: n_embd %% 256 and n_ff %% 32 must be 0 (integer fast path)");
    QMS_REQUIRE(F % 256 == 0, QMS_CUDA_EUNSUPPORTED,
                "moe_create: n_ff %% 256 must be 0 (staged expert layout; all Qwen3-MoE shapes qualify)");
    QMS_REQUIRE(d->gate_type == QMS_T_Q4_0 && d->up_type == QMS_T_Q4_0 &&
                    (d->down_type == QMS_T_Q4_0 || d->down_type == QMS_T_Q4_1),
                QMS_CUDA_EUNSUPPORTED, "moe_create: expert types %d/%d/%d not supported (Q4_0 gate/up, Q4_0 or Q4_1 down)",
                d->gate_type, d->up_type, d->down_type);
    QMS_REQUIRE(E <= 4096 && F <= 2048 && X <= 256 && K <= 64 && 2 * X <= E, QMS_CUDA_EUNSUPPORTED,
                "moe_create: n_embd <= 4096, n_ff <= 2048, n_expert <= min(256, n_embd/2), n_used <= 64 required");
    int dev = 0;
    QMS_CK(cudaGetDevice(&dev));
    QmsCudaMoe *m = (QmsCudaMoe *)calloc(1, sizeof(QmsCudaMoe));
    QMS_REQUIRE(m, QMS_CUDA_ENOMEM, "moe_create: out of host memory");
    m->device = dev;
    if (cudaDeviceGetAttribute(&m->nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) m->nsm = 148;
    m->E = E; m->X = X; m->K = K; m->F = F;
    m->n_local = n_local; m->expert_base = base;
    m->nbE = E / 32; m->nbF = F / 32;
    m->gate_type = d->gate_type; m->up_type = d->up_type; m->down_type = d->down_type;
    m->cgu = make_chunked(m->nbE);
    m->dcol = make_dncols(E, d->down_type == QMS_T_Q4_1);
    m->gu_expert = (size_t)2 * F * m->nbE * 18;
    m->dn_expert = (size_t)E * m->nbF * (m->dcol.q1 ? 20 : 18);
    const size_t rb = (size_t)X * E * 4, gb = m->gu_expert * n_local, db = m->dn_expert * n_local;
    m->weight_bytes = rb + gb + db;
    if (cudaMalloc(&m->router, rb) != cudaSuccess || cudaMalloc(&m->router_lm, rb) != cudaSuccess ||
        cudaMalloc(&m->gu, gb) != cudaSuccess || cudaMalloc(&m->dn, db) != cudaSuccess) {
        cudaGetLastError();
        qms_cuda_moe_destroy(m);
        set_error("moe_create: cannot allocate %.2f GB of weights", (rb + gb + db) / 1e9);
        return QMS_CUDA_ENOMEM;
    }
    int rc = QMS_CUDA_OK;
    if (cudaMemcpy(m->router, d->router, rb, d->src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice) !=
        cudaSuccess) {
        set_error("moe_create: %s", cudaGetErrorString(cudaGetLastError()));
        rc = QMS_CUDA_ECUDA;
    }
    if (rc == QMS_CUDA_OK) {
        k_router_lane_major<<<(unsigned)(((int64_t)X * E + 255) / 256), 256>>>(m->router, X, E, m->router_lm);
        if (cudaGetLastError() != cudaSuccess) {
            set_error("moe_create: router layout kernel failed");
            rc = QMS_CUDA_ECUDA;
        }
    }
    {
        UploadRing ring;
        const size_t gu_bytes = (size_t)n_local * F * (E / 32) * 18;
        const size_t dn_bytes = (size_t)n_local * E * (F / 32) * (m->dcol.q1 ? 20 : 18);
        if (rc == QMS_CUDA_OK && !d->src_on_device) rc = ring.open(std::max(gu_bytes, dn_bytes));
        if (rc == QMS_CUDA_OK) rc = upload_q4(m, d->gate, d->src_on_device, 0, m->gu, &ring);
        if (rc == QMS_CUDA_OK) rc = upload_q4(m, d->up, d->src_on_device, 1, m->gu, &ring);
        if (rc == QMS_CUDA_OK) rc = upload_q4(m, d->down, d->src_on_device, 2, m->dn, &ring);
    }
    if (rc == QMS_CUDA_OK && down_smem(m) > 48 * 1024 &&
        cudaFuncSetAttribute(k_moe_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)down_smem(m)) != cudaSuccess) {
        set_error("moe_create: %s", cudaGetErrorString(cudaGetLastError()));
        rc = QMS_CUDA_ECUDA;
    }
    if (rc == QMS_CUDA_OK && n_local == X) rc = stream_prepare(m);   // a shard has no batch-1 path
    if (rc == QMS_CUDA_OK && mma_supported(m)) {
        m->mma_min_t = kMmaMinT;
        if (const char *env = getenv("QMS_MMA_MIN_T")) m->mma_min_t = atoi(env);   // 0 turns the path off
        if (m->mma_min_t > 0) rc = mma_prepare(m);
        const char *gv = getenv("QMS_GEMV");                                          // 0 turns the GEMV off
        m->gemv = m->mma_min_t > 0 && gv_supported(m) && !(gv && atoi(gv) == 0);
        if (rc == QMS_CUDA_OK && m->gemv) rc = gv_prepare(m);
    }
    if (rc != QMS_CUDA_OK) {
        qms_cuda_moe_destroy(m);
        return rc;
    }
    *out = m;
    return QMS_CUDA_OK;
}

int qms_cuda_moe_create(const QmsCudaMoeDesc *d, QmsCudaMoe **out) {
    return create_impl(d, 0, d ? d->n_expert : 0, out);
}

int qms_cuda_moe_create_shard(const QmsCudaMoeDesc *d, int expert_base, int n_local, QmsCudaMoe **out) {
    return create_impl(d, expert_base, n_local, out);
}

int64_t qms_cuda_moe_device_bytes(const QmsCudaMoe *m) {
    if (!m) return 0;
    return (int64_t)(m->weight_bytes + m->scratch_bytes) + (int64_t)m->io_cap_T * m->E * 8;
}

// Scratch for calls of up to T tokens (forward, route: T Q8 rows, T * K slots) and expert calls of
// up to `rows` slots (qms_cuda_moe_experts*: one Q8 row and one SwiGLU row per slot). Both only grow.
static int reserve_scratch(QmsCudaMoe *m, int T, int rows) {
    T = std::max(T, m->cap_T);
    rows = std::max(rows, m->cap_rows);
    if (m->scratch && T == m->cap_T && rows == m->cap_rows) return QMS_CUDA_OK;
    const size_t TK = (size_t)T * m->K;
    const size_t R = std::max((size_t)T, (size_t)rows);        // Q8 activation rows
    const size_t RS = std::max(TK, (size_t)rows);               // slot rows (SwiGLU, Q8 groups, arrivals)
    size_t off = 0;
    const size_t o_xq_q = off; off += al256(R * m->E);
    const size_t o_xq_d = off; off += al256(R * m->nbE * 4);
    const size_t o_xq_s = off; off += al256(R * m->nbE * 4);
    const size_t o_log = off; off += al256((size_t)T * m->X * 4);
    const size_t o_sel = off; off += al256(TK * 4);
    const size_t o_wts = off; off += al256(TK * 4);
    const size_t o_act = off; off += al256(RS * m->F * 4);
    const size_t o_aq_q = off; off += al256(RS * m->F);
    const size_t o_aq_d = off; off += al256(RS * m->nbF * 4);
    const size_t o_aq_s = off; off += al256(RS * m->nbF * 4);
    const size_t o_cnt = off; off += al256((1 + RS * m->nbF) * 4);
    const size_t o_err = off; off += 256;
    StreamScratch ss;
    stream_scratch_sizes(m, &ss);
    const size_t o_lgf = off; off += al256(ss.lg_flagged);
    const size_t o_stamps = off; off += al256(ss.stamps);
    const size_t o_aqf = off; off += al256(ss.aq_flagged);
    const size_t o_pgu = off; off += al256(ss.part_gu);
    const size_t o_fin = off; off += al256(ss.fin);
    void *p = nullptr;
    if (cudaMalloc(&p, off) != cudaSuccess) {
        cudaGetLastError();
        set_error("moe_reserve: cannot allocate %zu bytes of scratch for T=%d", off, T);
        return QMS_CUDA_ENOMEM;
    }
    if (cudaMemset(p, 0, off) != cudaSuccess) {
        cudaFree(p);
        set_error("moe_reserve: memset failed");
        return QMS_CUDA_ECUDA;
    }
    cudaFree(m->scratch);
    char *b = (char *)p;
    m->scratch = p;
    m->scratch_bytes = off;
    m->xq_q = (int8_t *)(b + o_xq_q);
    m->xq_d = (float *)(b + o_xq_d);
    m->xq_s = (int *)(b + o_xq_s);
    m->logits = (float *)(b + o_log);
    m->sel = (int *)(b + o_sel);
    m->wts = (float *)(b + o_wts);
    m->act = (float *)(b + o_act);
    m->aq_q = (int8_t *)(b + o_aq_q);
    m->aq_d = (float *)(b + o_aq_d);
    m->aq_s = (int *)(b + o_aq_s);
    m->cnt = (int *)(b + o_cnt);
    m->err = m->err_ext ? m->err_ext : (int *)(b + o_err);
    m->lg_flagged = (unsigned long long *)(b + o_lgf);
    m->stamps = (unsigned *)(b + o_stamps);
    m->aq_flagged = (unsigned long long *)(b + o_aqf);
    m->part_gu = (unsigned long long *)(b + o_pgu);
    m->fin = (unsigned long long *)(b + o_fin);
    m->cap_T = T;
    m->cap_rows = rows;
    return QMS_CUDA_OK;
}

int qms_cuda_moe_reserve(QmsCudaMoe *m, int T) {
    QMS_REQUIRE(m && T >= 0, QMS_CUDA_EINVAL, "moe_reserve: bad arguments");
    QMS_REQUIRE((int64_t)T * m->K <= 65535, QMS_CUDA_EINVAL, "moe: T * n_used must be <= 65535");
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if (m->mma_min_t > 0 && T >= m->mma_min_t && (rc = mma_reserve(m, T))) return rc;
    if (T <= m->cap_T) return QMS_CUDA_OK;
    return reserve_scratch(m, T, 0);
}

// Rows of one expert call: the grouped kernels' tile grids (S / 64 + X tiles) stay within 65535.
constexpr int kMaxExpertRows = 1 << 21;

// Expert calls of S slots: S Q8 rows and S SwiGLU rows in the scratch (the grouped kernels'
// workspace is sized by mma_core itself). Outside graph capture only.
static int reserve_expert_rows(QmsCudaMoe *m, int S, cudaStream_t s, const char *who) {
    if (S <= std::max(m->cap_T, m->cap_rows)) return QMS_CUDA_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    QMS_CK(cudaStreamIsCapturing(s, &cs));
    QMS_REQUIRE(cs == cudaStreamCaptureStatusNone, QMS_CUDA_EINVAL,
                "%s: scratch for %d slots must be reserved before graph capture", who, S);
    return reserve_scratch(m, 0, S);           // (cudaFree of the old scratch waits for the device)
}

int qms_cuda_moe_forward(QmsCudaMoe *m, const float *xn, int T, float *out, int *sel, float *wts, float *logits,
                         const float *resid, void *stream) {
    QMS_REQUIRE(m && T >= 0, QMS_CUDA_EINVAL, "moe_forward: bad arguments");
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(xn && out, QMS_CUDA_EINVAL, "moe_forward: NULL xn or out");
    QMS_REQUIRE(m->n_local == m->X, QMS_CUDA_EUNSUPPORTED,
                "moe_forward: a shard layer holds experts [%d, %d) only; run route, experts and combine",
                m->expert_base, m->expert_base + m->n_local);
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if (T > m->cap_T) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QMS_CK(cudaStreamIsCapturing((cudaStream_t)stream, &cs));
        QMS_REQUIRE(cs == cudaStreamCaptureStatusNone, QMS_CUDA_EINVAL,
                    "moe_forward: scratch for T=%d must be reserved before graph capture", T);
        if ((rc = qms_cuda_moe_reserve(m, T))) return rc;
    }
    const cudaStream_t s = (cudaStream_t)stream;
    if (T == 1 && m->stream_ok && ((uintptr_t)xn & 15) == 0) {
        if ((rc = stream_forward_bs1(m, xn, out, resid, s))) return rc;
    } else {
        if (m->timing) QMS_CK(cudaEventRecord(m->ev[0], s));
        if ((rc = launch_router(m->router, m->X, m->E, xn, T, m->K, m->xq_q, m->xq_d, m->xq_s, m->logits, m->sel,
                                m->wts, m->cnt, s)))
            return rc;
        if (m->timing) {
            QMS_CK(cudaEventRecord(m->ev[1], s));
            QMS_CK(cudaEventRecord(m->ev[2], s));
        }
        if (m->mma_min_t > 0 && T >= m->mma_min_t) {
            if ((rc = mma_forward(m, T, resid, out, s))) return rc;
        } else {
        const dim3 ggrid(m->F / kGateUpRows, T * m->K);
        const int nbl = (m->nbE + 31) / 32;
        auto gk = nbl == 1 ? k_moe_gate_up<1> : nbl == 2 ? k_moe_gate_up<2> : nbl == 3 ? k_moe_gate_up<3>
                                                                                         : k_moe_gate_up<4>;
        QMS_CK(launch_pdl(gk, ggrid, dim3(256), 0, s, (const uint8_t *)m->gu, m->gu_expert, m->cgu, m->nbE, m->F,
                          m->K, (const int8_t *)m->xq_q, (const float *)m->xq_d, (const int *)m->xq_s,
                          (const int *)m->sel, m->act, m->aq_q, m->aq_d, m->aq_s, m->cnt + 1));
        if (m->timing) {
            QMS_CK(cudaEventRecord(m->ev[3], s));
            QMS_CK(cudaEventRecord(m->ev[4], s));
        }
        const dim3 dgrid(m->E / kDownRows, T);
        QMS_CK(launch_pdl(k_moe_down, dgrid, dim3(256), down_smem(m), s, (const uint8_t *)m->dn, m->dn_expert,
                          m->dcol, m->nbF, m->E, m->K, (const int8_t *)m->aq_q, (const float *)m->aq_d,
                          (const int *)m->aq_s, (const int *)m->sel, (const float *)m->wts, resid, out));
        if (m->timing) QMS_CK(cudaEventRecord(m->ev[5], s));
        }
    }
    const size_t TK = (size_t)T * m->K;
    if (sel) QMS_CK(cudaMemcpyAsync(sel, m->sel, TK * 4, cudaMemcpyDeviceToDevice, s));
    if (wts) QMS_CK(cudaMemcpyAsync(wts, m->wts, TK * 4, cudaMemcpyDeviceToDevice, s));
    if (logits) QMS_CK(cudaMemcpyAsync(logits, m->logits, (size_t)T * m->X * 4, cudaMemcpyDeviceToDevice, s));
    return QMS_CUDA_OK;
}

}  // extern "C"

namespace qms {
int moe_forward_normed_bs1(QmsCudaMoe *m, const float *h, const float *nw, float eps, float *out,
                           const float *resid, int *sel, cudaStream_t s) {
    if (!m->stream_ok || m->n_local != m->X || m->E % 512 || ((uintptr_t)h & 15) || m->cap_T < 1)
        return QMS_CUDA_EUNSUPPORTED;
    int rc = stream_forward_bs1(m, h, out, resid, s, nw, eps);
    if (rc) return rc;
    if (sel) QMS_CK(cudaMemcpyAsync(sel, m->sel, (size_t)m->K * 4, cudaMemcpyDeviceToDevice, s));
    return QMS_CUDA_OK;
}
}  // namespace qms

extern "C" {

int qms_cuda_moe_route(QmsCudaMoe *m, const float *xn, int T, int *sel, float *wts, float *logits, void *stream) {
    QMS_REQUIRE(m && T >= 0, QMS_CUDA_EINVAL, "moe_route: bad arguments");
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(xn && sel && wts, QMS_CUDA_EINVAL, "moe_route: NULL xn, sel or wts");
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if (T > m->cap_T) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QMS_CK(cudaStreamIsCapturing((cudaStream_t)stream, &cs));
        QMS_REQUIRE(cs == cudaStreamCaptureStatusNone, QMS_CUDA_EINVAL,
                    "moe_route: scratch for T=%d must be reserved before graph capture", T);
        if ((rc = qms_cuda_moe_reserve(m, T))) return rc;
    }
    const cudaStream_t s = (cudaStream_t)stream;
    if ((rc = launch_router(m->router, m->X, m->E, xn, T, m->K, m->xq_q, m->xq_d, m->xq_s, m->logits, m->sel, m->wts,
                            m->cnt, s)))
        return rc;
    const size_t TK = (size_t)T * m->K;
    QMS_CK(cudaMemcpyAsync(sel, m->sel, TK * 4, cudaMemcpyDeviceToDevice, s));
    QMS_CK(cudaMemcpyAsync(wts, m->wts, TK * 4, cudaMemcpyDeviceToDevice, s));
    if (logits) QMS_CK(cudaMemcpyAsync(logits, m->logits, (size_t)T * m->X * 4, cudaMemcpyDeviceToDevice, s));
    return QMS_CUDA_OK;
}

int qms_cuda_moe_experts(QmsCudaMoe *m, const float *x, const int *expert, int S, float *dn, void *stream) {
    QMS_REQUIRE(m && S >= 0, QMS_CUDA_EINVAL, "moe_experts: bad arguments");
    if (S == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(x && expert && dn, QMS_CUDA_EINVAL, "moe_experts: NULL x, expert or dn");
    QMS_REQUIRE(m->mma_min_t > 0, QMS_CUDA_EUNSUPPORTED, "moe_experts: the grouped tensor-core path is off for this layer");
    QMS_REQUIRE(S <= kMaxExpertRows, QMS_CUDA_EINVAL, "moe_experts: %d rows (at most %d per call)", S, kMaxExpertRows);
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if ((rc = reserve_expert_rows(m, S, (cudaStream_t)stream, "moe_experts"))) return rc;
    const cudaStream_t s = (cudaStream_t)stream;
    const int64_t nblocks = (int64_t)S * m->nbE;
    k_quantize_rows<<<(unsigned)std::min<int64_t>((nblocks + 7) / 8, 4096), 256, 0, s>>>(x, nblocks, m->xq_q, m->xq_d,
                                                                                        m->xq_s);
    QMS_CK(cudaGetLastError());
    return mma_experts(m, S, expert, dn, s);
}

int qms_cuda_moe_experts_q8(QmsCudaMoe *m, const QmsQ8 *xq, const int *expert, int S, float *dn, void *stream) {
    QMS_REQUIRE(m && S >= 0, QMS_CUDA_EINVAL, "moe_experts_q8: bad arguments");
    if (S == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(xq && expert && dn, QMS_CUDA_EINVAL, "moe_experts_q8: NULL xq, expert or dn");
    QMS_REQUIRE(m->mma_min_t > 0, QMS_CUDA_EUNSUPPORTED, "moe_experts_q8: the grouped path is off for this layer");
    QMS_REQUIRE(S <= kMaxExpertRows, QMS_CUDA_EINVAL, "moe_experts_q8: %d rows (at most %d per call)", S, kMaxExpertRows);
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if ((rc = reserve_expert_rows(m, S, (cudaStream_t)stream, "moe_experts_q8"))) return rc;
    const cudaStream_t s = (cudaStream_t)stream;
    const int64_t nblocks = (int64_t)S * m->nbE;
    k_unpack_q8<<<(unsigned)std::min<int64_t>((nblocks + 255) / 256, 4096), 256, 0, s>>>(xq, nblocks, m->xq_q, m->xq_d,
                                                                                        m->xq_s);
    QMS_CK(cudaGetLastError());
    return mma_experts(m, S, expert, dn, s);
}

int qms_cuda_moe_combine(const float *dn, const float *wts, int T, int n_used, int n_embd, const float *resid,
                         float *out, void *stream) {
    QMS_REQUIRE(T >= 0 && n_used > 0 && n_embd > 0, QMS_CUDA_EINVAL, "moe_combine: bad arguments");
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(dn && wts && out, QMS_CUDA_EINVAL, "moe_combine: NULL dn, wts or out");
    return mma_combine(dn, wts, T, n_used, n_embd, resid, out, (cudaStream_t)stream);
}

int qms_cuda_moe_set_kernel_events(QmsCudaMoe *m, void **events) {
    QMS_REQUIRE(m, QMS_CUDA_EINVAL, "moe_set_kernel_events: NULL layer");
    m->timing = events != nullptr;
    for (int i = 0; i < 6; i++) m->ev[i] = events ? (cudaEvent_t)events[i] : nullptr;
    return QMS_CUDA_OK;
}

int qms_cuda_moe_status(QmsCudaMoe *m) {
    QMS_REQUIRE(m, QMS_CUDA_EINVAL, "moe_status: NULL layer");
    if (!m->err) return QMS_CUDA_OK;
    int rc = ensure_device(m->device);
    if (rc) return rc;
    int flags = 0;
    QMS_CK(cudaMemcpy(&flags, m->err, sizeof flags, cudaMemcpyDeviceToHost));
    if (flags) {
        QMS_CK(cudaMemset(m->err, 0, sizeof(int)));
        set_error("moe: a bounded wait inside the decode kernels gave up (flags 0x%x); outputs of that call are "
                  "invalid", flags);
        return QMS_CUDA_ETIMEOUT;
    }
    return QMS_CUDA_OK;
}

int qms_cuda_moe_forward_host(QmsCudaMoe *m, const float *xn, int T, float *out, int *sel, float *wts, float *logits) {
    QMS_REQUIRE(m && T >= 0, QMS_CUDA_EINVAL, "moe_forward_host: bad arguments");
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(xn && out, QMS_CUDA_EINVAL, "moe_forward_host: NULL xn or out");
    int rc = ensure_device(m->device);
    if (rc) return rc;
    if (!m->hstream) QMS_CK(cudaStreamCreateWithFlags(&m->hstream, cudaStreamNonBlocking));
    if ((rc = qms_cuda_moe_reserve(m, T))) return rc;
    if (T > m->io_cap_T) {
        cudaFree(m->d_in);
        cudaFree(m->d_out);
        m->d_in = m->d_out = nullptr;
        m->io_cap_T = 0;
        if (cudaMalloc(&m->d_in, (size_t)T * m->E * 4) != cudaSuccess ||
            cudaMalloc(&m->d_out, (size_t)T * m->E * 4) != cudaSuccess) {
            cudaGetLastError();
            set_error("moe_forward_host: cannot allocate I/O buffers for T=%d", T);
            return QMS_CUDA_ENOMEM;
        }
        m->io_cap_T = T;
    }
    const cudaStream_t s = m->hstream;
    const size_t xb = (size_t)T * m->E * 4;
    QMS_CK(cudaMemcpyAsync(m->d_in, xn, xb, cudaMemcpyHostToDevice, s));
    if ((rc = qms_cuda_moe_forward(m, m->d_in, T, m->d_out, nullptr, nullptr, nullptr, nullptr, s))) return rc;
    QMS_CK(cudaMemcpyAsync(out, m->d_out, xb, cudaMemcpyDeviceToHost, s));
    const size_t TK = (size_t)T * m->K;
    if (sel) QMS_CK(cudaMemcpyAsync(sel, m->sel, TK * 4, cudaMemcpyDeviceToHost, s));
    if (wts) QMS_CK(cudaMemcpyAsync(wts, m->wts, TK * 4, cudaMemcpyDeviceToHost, s));
    if (logits) QMS_CK(cudaMemcpyAsync(logits, m->logits, (size_t)T * m->X * 4, cudaMemcpyDeviceToHost, s));
    QMS_CK(cudaStreamSynchronize(s));
    return QMS_CUDA_OK;
}

}  // extern "C"

// ---- routing without allocation --------------------------------------------------------------
// Some callers may not call cudaMalloc at all: code running inside another framework's memory
// pool or allocator hooks, plugin hosts that forbid device allocation after start-up, and
// deployments that pin every byte of HBM up front. qms_cuda_moe_route_noalloc serves them:
// it runs the same router kernel (Q8 rows, exact-order logits, softmax/top-k) with its scratch
// in the fixed array below instead of a layer handle's cudaMalloc'd scratch. The array holds
// at most kNoAllocMaxT tokens of n_embd <= 4096 and n_expert <= 256 (384.25 KiB); every GPU
// that loads the library keeps it until the process exits.
namespace qms {

constexpr int kNoAllocMaxT = 64;
constexpr int kNoAllocMaxE = 4096;
constexpr int kNoAllocMaxX = 256;
constexpr size_t kNaXqQ = (size_t)kNoAllocMaxT * kNoAllocMaxE;              // int8 rows
constexpr size_t kNaXqD = (size_t)kNoAllocMaxT * (kNoAllocMaxE / 32) * 4;   // block scales
constexpr size_t kNaXqS = kNaXqD;                                           // block sums
constexpr size_t kNaLogits = (size_t)kNoAllocMaxT * kNoAllocMaxX * 4;       // router logits
constexpr size_t kNaCnt = 256;                                              // arrival counter
constexpr size_t kNoAllocScratchBytes = kNaXqQ + kNaXqD + kNaXqS + kNaLogits + kNaCnt;

static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

// Device address of g_route_scratch in the current context, looked up on every call: the lookup
// is a host-side query once the module is loaded (no allocation, no device work), and a cached
// address would go stale after a device reset or a new primary context. qms_cuda_init makes the
// first lookup, which loads the module and so places the array.
constexpr int kNoAllocMaxDevices = 64;

int route_scratch_ptr(int dev, unsigned char **out) {
    QMS_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, QMS_CUDA_EINVAL, "moe_route_noalloc: device %d unsupported", dev);
    unsigned char *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress((void **)&p, g_route_scratch);
    if (e != cudaSuccess || !p) {
        set_error("moe_route_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
        return QMS_CUDA_ECUDA;
    }
    *out = p;
    return QMS_CUDA_OK;
}

}  // namespace qms

extern "C" int qms_cuda_moe_route_noalloc(const float *router, int n_expert, int n_embd, int n_used, const float *xn,
                                          int T, int *sel, float *wts, float *logits, void *stream) {
    const int X = n_expert, E = n_embd, K = n_used;
    QMS_REQUIRE(router && xn && sel && wts && T >= 0, QMS_CUDA_EINVAL, "moe_route_noalloc: bad arguments");
    QMS_REQUIRE(T <= kNoAllocMaxT, QMS_CUDA_EINVAL,
                "moe_route_noalloc: T=%d exceeds the fixed scratch limit of %d tokens per call", T, kNoAllocMaxT);
    QMS_REQUIRE(E > 0 && E % 256 == 0 && E <= kNoAllocMaxE, QMS_CUDA_EINVAL,
                "moe_route_noalloc: n_embd=%d must be a multiple of 256 and at most %d", E, kNoAllocMaxE);
    QMS_REQUIRE(X > 0 && X <= kNoAllocMaxX && 2 * X <= E && K > 0 && K <= X && K <= 64, QMS_CUDA_EINVAL,
                "moe_route_noalloc: need 0 < n_used <= min(n_expert, 64) and n_expert <= min(%d, n_embd/2)",
                kNoAllocMaxX);
    QMS_REQUIRE(((uintptr_t)router & 15) == 0, QMS_CUDA_EINVAL, "moe_route_noalloc: router must be 16-byte aligned");
    if (T == 0) return QMS_CUDA_OK;
    int dev = -1;
    QMS_CK(cudaGetDevice(&dev));
    unsigned char *p = nullptr;
    const int rc = route_scratch_ptr(dev, &p);
    if (rc) return rc;
    int8_t *xq_q = (int8_t *)p;
    float *xq_d = (float *)(p + kNaXqQ);
    int *xq_s = (int *)(p + kNaXqQ + kNaXqD);
    float *lg = logits ? logits : (float *)(p + kNaXqQ + kNaXqD + kNaXqS);
    int *cnt = (int *)(p + kNaXqQ + kNaXqD + kNaXqS + kNaLogits);
    const cudaStream_t s = (cudaStream_t)stream;
    QMS_CK(cudaMemsetAsync(cnt, 0, sizeof(int), s));   // the arrival counter must start at zero
    return launch_router(router, X, E, xn, T, K, xq_q, xq_d, xq_s, lg, sel, wts, cnt, s);
}
