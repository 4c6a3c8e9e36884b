// qms_moe_stream.cu - batch-1 decode of the MoE block, streamed from HBM with TMA bulk copies.
//
// A decode token reads 8 experts x 10.6 MB of Q4_0 weights per 235B layer and does ~3.5 integer
// ops per byte, so the block is bound by HBM bandwidth, and on B200 every separately launched
// stream of a few tens of MB loses several microseconds to ramp-up and tail. So a call is two
// kernels chained with programmatic dependent launch (PDL):
//   k_router_bs1   one CTA per router row. Its weight row (16 KB, stored lane-major) is
//                  bulk-copied into shared memory BEFORE griddepcontrol.wait, i.e. while the
//                  previous kernel still runs; then xn is read, quantised to Q8, the logit is
//                  computed in the reference's exact F32 order and the last CTA to finish ranks
//                  the experts.
//   k_stream_ffn   persistent, one CTA per SM, ONE continuous stream of all the call's expert
//                  bytes: a producer thread bulk-copies (cp.async.bulk) first the CTA's share of
//                  gate/up stages (eight chunks of 8 rows x 16 blocks, 18 KB) and then, without
//                  waiting, its share of down stages into an mbarrier ring; eight consumer warps
//                  run dp4a dots against the token's Q8 row. A gate/up tile is 32 gate + 32 up
//                  rows, i.e. one SwiGLU + Q8 re-quantisation group (src/model.c:989-997). The
//                  down phase needs every group's Q8 values, so the consumers wait (bounded) on a
//                  grid-wide counter while the ring keeps filling with down chunks; a down tile
//                  is 8 output rows x 8 experts, combined in selection order with one FMA per
//                  expert (src/model.c:1152-1162) plus the optional residual.
// Work is split over the CTAs by stages, not tiles, so every SM streams the same number of bytes
// (+-1 stage). A tile split between CTAs leaves partial row sums in global memory; the CTA that
// completes it adds them in segment order, so results do not depend on timing. The grid (one
// CTA per SM) is always fully resident: the kernel needs most of an SM's shared memory and
// nothing it waits for runs behind it; a wait that still runs out sets an error bit.
// Every mbarrier wait is bounded: on timeout the kernel records an error bit in *err, stops
// issuing copies, waits (bounded) for the copies it already issued and returns.
#include <algorithm>

#include "qms_moe.cuh"
#include "qms_router.cuh"

namespace qms {

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 2) * 32;   // + producer warp + epilogue warp
constexpr int kMaxSegments = 4;                    // CTAs a tile may be split across
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr size_t kSmemOptIn = 232448;              // 227 KB: per-block dynamic shared memory on sm_100
constexpr size_t kRouterReserve = 40 * 1024;       // left free for the next call's router CTA

enum { ERR_CONSUMER = 1, ERR_PRODUCER = 2, ERR_GRID = 4, ERR_ROUTER = 16, ERR_DRAIN = 32 };

// ---- mbarrier / bulk-copy helpers --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Fetch [src, src + bytes) into L2 without waiting for it (16-byte aligned, multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Wait for phase `parity` of `bar`; give up when another thread set *abort or after kSpinLimit
// polls (then set *abort and the error bit). Returns true when the phase completed.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort, int *err, int code) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (++n == kSpinLimit) {
            *abort = 1;
            atomicOr(err, code);
            return false;
        }
    }
    return true;
}

// After an abort: wait (bounded) for every copy this producer issued into the ring to land,
// so no bulk copy is still writing into shared memory when the CTA exits.
__device__ __forceinline__ void drain_issued(uint64_t *full, int nst, int issued, int *err) {
    for (int j = issued > nst ? issued - nst : 0; j < issued; j++) {
        uint32_t n = 0;
        while (!mbar_try_wait(&full[j % nst], (j / nst) & 1))
            if (++n == kSpinLimit) {
                atomicOr(err, ERR_DRAIN);
                return;
            }
    }
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Static split of U stage-units over G CTAs: CTA c owns [lo(c), lo(c+1)).
__host__ __device__ inline int part_lo(int c, int U, int G) { return (int)((int64_t)c * U / G); }
__host__ __device__ inline int part_owner(int u, int U, int G) { return (int)(((int64_t)(u + 1) * G - 1) / U); }

// Ring position: slot and phase of the it-th stage, advanced incrementally.
struct Ring {
    int slot = 0;
    uint32_t phase = 0;
    int nst;
    __device__ explicit Ring(int n) : nst(n) {}
    __device__ void next() {
        if (++slot == nst) {
            slot = 0;
            phase ^= 1;
        }
    }
};

// One consumer warp's share of a stage: its chunk (8 rows x SB blocks) against one Q8 row.
template <int SB>
__device__ __forceinline__ void chunk_dot(const uint8_t *chunk, const int8_t *xq, const float *xd, const int *xs8,
                                          int s, int bl, int rs, float (&acc)[SB / 4]) {
    constexpr int P = SB / 4, RSTEP = 32 / SB;
    const int b = s * SB + bl;
    const int4 xa0 = *reinterpret_cast<const int4 *>(xq + b * 32);
    const int4 xa1 = *reinterpret_cast<const int4 *>(xq + b * 32 + 16);
    const float d = xd[b];
    const int s8 = xs8[b];
#pragma unroll
    for (int p = 0; p < P; p++) {
        const int rr = rs + p * RSTEP;
        const uint4 nib = *reinterpret_cast<const uint4 *>(chunk + chunk_nib_off(SB, rr, bl));
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(chunk + chunk_scale_off(SB, rr, bl)));
        acc[p] = fmaf((float)(q4_block_isum(nib, xa0, xa1) - s8), dw * d, acc[p]);
    }
}

// ---- router (batch 1) --------------------------------------------------------------------------
// The row is stored lane-major ([k][i] = element 16*i + k), so lane k of the exact-order dot reads
// its 256-long FMA chain with 128-bit loads; shared memory pads each lane's run by 16 bytes so
// the 16 lanes hit different banks.
__global__ void __launch_bounds__(256) k_router_bs1(const float *__restrict__ Wlm, int X, int E,
                                                    const float *__restrict__ xn, int K, int8_t *__restrict__ xq_q,
                                                    float *__restrict__ xq_d, int *__restrict__ xq_s,
                                                    float *__restrict__ logits, int *__restrict__ sel,
                                                    float *__restrict__ wts, int *__restrict__ cnt,
                                                    int *__restrict__ err) {
    extern __shared__ __align__(128) float rsm[];
    const int L = E / 16, PS = L + 4;
    float *srow = rsm;            // [16][PS]
    float *sx = rsm + 16 * PS;    // [16][PS]
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_sel[64];
    __shared__ int s_last, s_abort;
    const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_abort = 0;
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar, (uint32_t)E * 4);
        const uint64_t pol = evict_first_policy();
        for (int k = 0; k < 16; k++)
            bulk_load(srow + k * PS, Wlm + (size_t)e * E + (size_t)k * L, (uint32_t)L * 4, &bar, pol);
    }
    pdl_trigger();
    pdl_wait();                                    // xn comes from the previous kernel
    for (int q = tid; q < E / 4; q += blockDim.x) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(xn) + q);
        const int j = 4 * q;
        sx[((j + 0) & 15) * PS + ((j + 0) >> 4)] = v.x;
        sx[((j + 1) & 15) * PS + ((j + 1) >> 4)] = v.y;
        sx[((j + 2) & 15) * PS + ((j + 2) >> 4)] = v.z;
        sx[((j + 3) & 15) * PS + ((j + 3) >> 4)] = v.w;
    }
    __syncthreads();
    for (int b = e + X * (warp - 1); warp > 0 && b < E / 32; b += X * 7) {   // warp 0 runs the chain
        const int j = b * 32 + lane;
        const Q8Lane r = quantize_lane(sx[(j & 15) * PS + (j >> 4)]);
        xq_q[j] = (int8_t)r.q;
        if (lane == 0) {
            xq_d[b] = r.d;
            xq_s[b] = r.sum;
        }
    }
    if (warp == 0) {
        const bool ok = __all_sync(0xffffffffu, wait_bounded(&bar, 0, &s_abort, err, ERR_ROUTER));
        const int k = lane & 15;
        const float *w = srow + k * PS, *x = sx + k * PS;
        float acc = 0.0f;
        int i = 0;
        for (; i + 32 <= L; i += 32) {             // 8 loads of each operand in flight per batch
            float4 w4[8], x4[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                w4[q] = *reinterpret_cast<const float4 *>(w + i + 4 * q);
                x4[q] = *reinterpret_cast<const float4 *>(x + i + 4 * q);
            }
#pragma unroll
            for (int q = 0; q < 8; q++) {
                acc = __fmaf_rn(w4[q].x, x4[q].x, acc);
                acc = __fmaf_rn(w4[q].y, x4[q].y, acc);
                acc = __fmaf_rn(w4[q].z, x4[q].z, acc);
                acc = __fmaf_rn(w4[q].w, x4[q].w, acc);
            }
        }
        for (; i < L; i += 4) {
            const float4 w4 = *reinterpret_cast<const float4 *>(w + i);
            const float4 x4 = *reinterpret_cast<const float4 *>(x + i);
            acc = __fmaf_rn(w4.x, x4.x, acc);
            acc = __fmaf_rn(w4.y, x4.y, acc);
            acc = __fmaf_rn(w4.z, x4.z, acc);
            acc = __fmaf_rn(w4.w, x4.w, acc);
        }
        acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8, 16));
        acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 16));
        acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2, 16));
        acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1, 16));
        if (lane == 0) {
            logits[e] = ok ? acc : 0.0f;
            s_last = atom_add_acq_rel(cnt, 1) == X - 1;   // publishes the logit, sees the others'
        }
    }
    __syncthreads();
    if (!s_last) return;
    topk_token(logits, X, K, sel, wts, s_sel);
    if (tid == 0) *cnt = 0;
}

// ---- gate/up + SwiGLU + Q8, then down + combine, in one stream (batch 1) ------------------------
struct FfnArgs {
    const uint8_t *gu, *dn;
    size_t gu_expert, dn_expert;
    int nbE, nbF, F, E, K, nst;
    const int8_t *xq_q;
    const float *xq_d;
    const int *xq_s;
    int8_t *aq_q;
    float *aq_d;
    int *aq_s;
    float *part_gu, *part_dn;
    int *tcnt_gu, *tcnt_dn;
    const int *sel;
    const float *wts;
    const float *resid;
    float *out;
    int *grid_cnt;    // [0]: gate/up tiles whose Q8 group is written, [1]: CTAs past the wait
    int *err;
};

// Epilogue-warp half of a tile split across CTAs: publish this CTA's 64 partial sums; the CTA
// whose segment arrives last gets true and `v` (2 values per lane: [lane], [32 + lane]) holding
// the full sums, added in segment order so the result does not depend on arrival order.
__device__ __forceinline__ bool merge_partial(float *part, int *tcnt, int tile, int S, int U, int G, int c,
                                              float (&v)[2]) {
    const int lane = threadIdx.x & 31;
    const int first = part_owner(tile * S, U, G);
    const int segs = part_owner(tile * S + S - 1, U, G) - first + 1;
    float *pt = part + (size_t)tile * kMaxSegments * 64;
    pt[(c - first) * 64 + lane] = v[0];
    pt[(c - first) * 64 + 32 + lane] = v[1];
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atom_add_acq_rel(tcnt + tile, 1) == segs - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return false;
    float a0 = 0.0f, a1 = 0.0f;
    for (int q = 0; q < segs; q++) {
        a0 += __ldcg(pt + q * 64 + lane);
        a1 += __ldcg(pt + q * 64 + 32 + lane);
    }
    v[0] = a0;
    v[1] = a1;
    if (lane == 0) tcnt[tile] = 0;
    return true;
}

constexpr int kSumBufs = 4;        // tile-sum hand-off buffers between consumer and epilogue warps

template <int SBG, int SBD>
__global__ void __launch_bounds__(kStreamThreads, 1) k_stream_ffn(const FfnArgs a) {
    constexpr uint32_t GBG = 8 * SBG * 18, STG = 8 * GBG, GBD = 8 * SBD * 18, STD = 8 * GBD;
    constexpr uint32_t SLOT = STG > STD ? STG : STD;
    constexpr int PG = SBG / 4, RSG = 32 / SBG, PD = SBD / 4, RSD = 32 / SBD;
    extern __shared__ __align__(128) uint8_t smem[];
    const int nst = a.nst, K = a.K, F = a.F, nbE = a.nbE, nbF = a.nbF;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nst * SLOT);
    uint64_t *empty = full + nst;
    uint64_t *sfull = empty + nst;                                  // [kSumBufs] sums written
    uint64_t *sempty = sfull + kSumBufs;                            // [kSumBufs] sums consumed
    int8_t *sxq = reinterpret_cast<int8_t *>(sempty + kSumBufs);   // [nbE*32]
    float *sxd = reinterpret_cast<float *>(sxq + nbE * 32);         // [nbE]
    int *sxs = reinterpret_cast<int *>(sxd + nbE);                  // [nbE], 8 * sum
    int8_t *saq = reinterpret_cast<int8_t *>(sxs + nbE);            // [K][F]
    float *sad = reinterpret_cast<float *>(saq + K * F);            // [K][nbF]
    int *sas = reinterpret_cast<int *>(sad + K * nbF);              // [K][nbF], 8 * sum
    float *sbuf = reinterpret_cast<float *>(sas + K * nbF);         // [kSumBufs][64] tile sums
    __shared__ int s_abort, s_ok;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x, c = blockIdx.x;
    const int Sg = nbE / SBG, tps = F / 32, ntg = K * tps, Ug = ntg * Sg;
    const int Sd = nbF / SBD, RBE = 8 / K, RT = 8 * RBE, Ud = (a.E / RT) * Sd;
    const int ug0 = part_lo(c, Ug, G), ug1 = part_lo(c + 1, Ug, G);
    const int ud0 = part_lo(c, Ud, G), ud1 = part_lo(c + 1, Ud, G);
    const size_t tile_bytes = (size_t)Sg * STG;
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < nst; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        for (int i = 0; i < kSumBufs; i++) {
            mbar_init(&sfull[i], kConsumerWarps);
            mbar_init(&sempty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();                                  // the next router may prefetch its weights
    pdl_wait();                                     // selection and Q8 row come from the router
    volatile int *abort_flag = &s_abort;

    if (warp == kConsumerWarps) {                   // ---- producer: one stream, gate/up then down
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            int ex[8];
            for (int j = 0; j < 8; j++) ex[j] = j < K ? __ldcg(a.sel + j) : 0;
            Ring r(nst);
            int issued = 0;
            bool ok = true;
            for (int u = ug0; u < ug1 && ok; u++) {
                const int tile = u / Sg, s = u - tile * Sg;
                const uint8_t *src = a.gu + (size_t)ex[tile / tps] * a.gu_expert + (size_t)(tile % tps) * tile_bytes;
                if (issued >= nst && !(ok = wait_bounded(&empty[r.slot], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER)))
                    break;
                mbar_arrive_expect_tx(&full[r.slot], STG);
                bulk_load(ring + (size_t)r.slot * SLOT, src + (size_t)s * STG, STG, &full[r.slot], pol);
                issued++;
                r.next();
            }
            const uint8_t *base[8];
            for (int gi = 0; gi < 8; gi++) base[gi] = a.dn + (size_t)ex[gi / RBE] * a.dn_expert;
            for (int u = ud0; u < ud1 && ok; u++) {
                const int tile = u / Sd, s = u - tile * Sd;
                if (issued >= nst && !(ok = wait_bounded(&empty[r.slot], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER)))
                    break;
                mbar_arrive_expect_tx(&full[r.slot], STD);
                uint8_t *dst = ring + (size_t)r.slot * SLOT;
                for (int gi = 0; gi < 8; gi++) {
                    const size_t rb = (size_t)tile * RBE + gi % RBE;
                    bulk_load(dst + gi * GBD, base[gi] + (rb * Sd + s) * GBD, GBD, &full[r.slot], pol);
                }
                issued++;
                r.next();
            }
            if (!ok || *abort_flag) drain_issued(full, nst, issued, a.err);
        }
        return;
    }

    if (warp == kConsumerWarps + 1) {               // ---- epilogue warp: SwiGLU/Q8, merges, combine
        Ring sr(kSumBufs);
        bool ok = true;
        for (int pass = 0; pass < 2; pass++) {
            const bool gate = pass == 0;
            const int S = gate ? Sg : Sd, U = gate ? Ug : Ud;
            const int u0 = gate ? ug0 : ud0, u1 = gate ? ug1 : ud1;
            float w[8];
            if (!gate)
                for (int j = 0; j < 8; j++) w[j] = j < K ? __ldcg(a.wts + j) : 0.0f;
            for (int u = u0; u < u1;) {
                const int tile = u / S, s0 = u - tile * S, s1 = min(S, s0 + (u1 - u));
                u += s1 - s0;
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&sfull[sr.slot], sr.phase, abort_flag, a.err,
                                                                  ERR_CONSUMER));
                float v[2] = {sbuf[sr.slot * 64 + lane], sbuf[sr.slot * 64 + 32 + lane]};
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[sr.slot]);
                sr.next();
                if (!ok) continue;
                bool mine = true;
                if (!(s0 == 0 && s1 == S))
                    mine = merge_partial(gate ? a.part_gu : a.part_dn, gate ? a.tcnt_gu : a.tcnt_dn, tile, S, U, G, c,
                                         v);
                if (!mine) continue;
                if (gate) {                         // rows 0-31: gate f0+lane, rows 32-63: up f0+lane
                    const int slot = tile / tps, t = tile % tps;
                    const float av = __fmul_rn(__fdiv_rn(v[0], __fadd_rn(1.0f, expf(-v[0]))), v[1]);
                    const Q8Lane q8 = quantize_lane(av);
                    const size_t base = (size_t)slot * F + (size_t)t * 32;
                    a.aq_q[base + lane] = (int8_t)q8.q;
                    if (lane == 0) {
                        a.aq_d[(size_t)slot * tps + t] = q8.d;
                        a.aq_s[(size_t)slot * tps + t] = q8.sum;
                    }
                    __syncwarp();
                    if (lane == 0) red_add_release(a.grid_cnt, 1);   // one more Q8 group is visible
                } else {                            // sum index (j*RBE + rbi)*8 + rr: expert j, row rr of block rbi
                    const int rbi = (lane >> 3) & 7, rr = lane & 7;
                    float o = 0.0f;
                    for (int jj = 0; jj < K; jj++) {
                        const int idx = (jj * RBE + rbi) * 8 + rr;
                        const float lo = __shfl_sync(0xffffffffu, v[0], idx & 31);
                        const float hi = __shfl_sync(0xffffffffu, v[1], idx & 31);
                        o = __fmaf_rn(w[jj], idx < 32 ? lo : hi, o);
                    }
                    if (lane < RT) {
                        const int i = tile * RT + lane;
                        if (a.resid) o = __fadd_rn(a.resid[i], o);
                        a.out[i] = o;
                    }
                }
            }
        }
        return;
    }

    // ---- consumers, phase A: gate/up
    const int tid = threadIdx.x;
    for (int i = tid; i < nbE * 2; i += kConsumerWarps * 32)
        reinterpret_cast<int4 *>(sxq)[i] = __ldcg(reinterpret_cast<const int4 *>(a.xq_q) + i);
    for (int i = tid; i < nbE; i += kConsumerWarps * 32) {
        sxd[i] = __ldcg(a.xq_d + i);
        sxs[i] = 8 * __ldcg(a.xq_s + i);
    }
    consumer_sync();
    const int g = warp;
    Ring r(nst), sr(kSumBufs);
    int handed = 0;
    bool ok = true;
    // hand a tile's 64 sums (8 per warp) to the epilogue warp
    auto hand_off = [&](const float *acc, int P, int RS, int bl, int rs) {
        if (handed >= kSumBufs && ok)
            ok = __all_sync(0xffffffffu, wait_bounded(&sempty[sr.slot], sr.phase ^ 1, abort_flag, a.err, ERR_CONSUMER));
        if (bl == 0)
            for (int p = 0; p < P; p++) sbuf[sr.slot * 64 + g * 8 + rs + p * RS] = acc[p];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfull[sr.slot]);
        sr.next();
        handed++;
    };
    {
        const int bl = lane % SBG, rs = lane / SBG;
        for (int u = ug0; u < ug1;) {
            const int tile = u / Sg, s0 = u - tile * Sg, s1 = min(Sg, s0 + (ug1 - u));
            float acc[PG];
#pragma unroll
            for (int p = 0; p < PG; p++) acc[p] = 0.0f;
            for (int s = s0; s < s1; s++, r.next()) {
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
                if (ok) {
                    chunk_dot<SBG>(ring + (size_t)r.slot * SLOT + g * GBG, sxq, sxd, sxs, s, bl, rs, acc);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[r.slot]);
                }
            }
            u += s1 - s0;
#pragma unroll
            for (int p = 0; p < PG; p++)
#pragma unroll
                for (int o = SBG / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(0xffffffffu, acc[p], o);
            hand_off(acc, PG, RSG, bl, rs);
        }
    }

    // ---- phase B: wait until every CTA's Q8 groups are written, then down + combine
    if (tid == 0) {
        int okg = 1;
        uint32_t n = 0;
        while (ld_acquire(a.grid_cnt) < ntg) {
            if (*abort_flag || ++n == kSpinLimit) {
                okg = 0;
                if (!*abort_flag) atomicOr(a.err, ERR_GRID);
                *abort_flag = 1;
                break;
            }
            __nanosleep(32);
        }
        // the last CTA past the wait re-arms both counters for the next call
        if (atomicAdd(a.grid_cnt + 1, 1) == G - 1) {
            atomicExch(a.grid_cnt, 0);
            atomicExch(a.grid_cnt + 1, 0);
        }
        s_ok = okg;
    }
    consumer_sync();
    ok = ok && s_ok;
    if (ok) {
        for (int i = tid; i < K * F / 16; i += kConsumerWarps * 32)
            reinterpret_cast<int4 *>(saq)[i] = __ldcg(reinterpret_cast<const int4 *>(a.aq_q) + i);
        for (int i = tid; i < K * nbF; i += kConsumerWarps * 32) {
            sad[i] = __ldcg(a.aq_d + i);
            sas[i] = 8 * __ldcg(a.aq_s + i);
        }
    }
    consumer_sync();
    {
        const int j = g / RBE, bl = lane % SBD, rs = lane / SBD;
        const int8_t *xq = saq + (size_t)j * F;
        const float *xdv = sad + j * nbF;
        const int *xsv = sas + j * nbF;
        for (int u = ud0; u < ud1;) {
            const int tile = u / Sd, s0 = u - tile * Sd, s1 = min(Sd, s0 + (ud1 - u));
            float acc[PD];
#pragma unroll
            for (int p = 0; p < PD; p++) acc[p] = 0.0f;
            for (int s = s0; s < s1; s++, r.next()) {
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
                if (ok) {
                    chunk_dot<SBD>(ring + (size_t)r.slot * SLOT + g * GBD, xq, xdv, xsv, s, bl, rs, acc);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[r.slot]);
                }
            }
            u += s1 - s0;
#pragma unroll
            for (int p = 0; p < PD; p++)
#pragma unroll
                for (int o = SBD / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(0xffffffffu, acc[p], o);
            hand_off(acc, PD, RSD, bl, rs);
        }
    }
}

// ---- host side -----------------------------------------------------------------------------------
static uint32_t ffn_slot(const QmsCudaMoe *m) { return 8 * std::max(m->cgu.GB, m->cdn.GB); }
static size_t ffn_fixed(const QmsCudaMoe *m) {
    return 2 * kSumBufs * 8 + (size_t)m->nbE * 40 + (size_t)m->K * m->F + (size_t)m->K * m->nbF * 8 +
           kSumBufs * 64 * 4;
}
static size_t ffn_smem(const QmsCudaMoe *m) { return (size_t)m->gu_nst * (ffn_slot(m) + 16) + ffn_fixed(m); }
static size_t router_smem(int E) { return (size_t)2 * 16 * (E / 16 + 4) * 4; }

static int max_segments(int U, int S, int G) {
    int worst = 1;
    for (int tile = 0; tile * S < U; tile++)
        worst = std::max(worst, part_owner(tile * S + S - 1, U, G) - part_owner(tile * S, U, G) + 1);
    return worst;
}

typedef void (*FfnKernel)(const FfnArgs);
static FfnKernel ffn_kernel(const QmsCudaMoe *m) {
    if (m->cgu.SB == 16) return m->cdn.SB == 16 ? k_stream_ffn<16, 16> : k_stream_ffn<16, 8>;
    return m->cdn.SB == 16 ? k_stream_ffn<8, 16> : k_stream_ffn<8, 8>;
}

int stream_prepare(QmsCudaMoe *m) {
    m->stream_ok = 0;
    if (!(m->K == 1 || m->K == 2 || m->K == 4 || m->K == 8) || m->X > 256 || 2 * m->X > m->E) return QMS_CUDA_OK;
    if (m->nbE % m->cgu.SB || m->nbF % m->cdn.SB) return QMS_CUDA_OK;
    // the deepest ring that still leaves room for the next call's router CTA on the same SM
    m->gu_nst = (int)std::min<size_t>(12, (kSmemOptIn - kRouterReserve - ffn_fixed(m)) / (ffn_slot(m) + 16));
    m->dn_nst = m->gu_nst;
    if (m->gu_nst < 4) return QMS_CUDA_OK;
    const int Ugu = m->K * (m->F / 32) * m->cgu.S, Udn = (m->E / (64 / m->K)) * m->cdn.S;
    if (max_segments(Ugu, m->cgu.S, m->nsm) > kMaxSegments || max_segments(Udn, m->cdn.S, m->nsm) > kMaxSegments)
        return QMS_CUDA_OK;
    const FfnKernel fk = ffn_kernel(m);
    QMS_CK(cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ffn_smem(m)));
    QMS_CK(cudaFuncSetAttribute(k_router_bs1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)router_smem(m->E)));
    // one shared-memory carveout for both kernels: no L1/shared reconfiguration between them
    QMS_CK(cudaFuncSetAttribute(fk, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    QMS_CK(cudaFuncSetAttribute(k_router_bs1, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    m->stream_ok = 1;
    return QMS_CUDA_OK;
}

int stream_scratch_sizes(const QmsCudaMoe *m, size_t *part_gu, size_t *part_dn, size_t *cnt_gu, size_t *cnt_dn) {
    const int tiles_gu = m->K * (m->F / 32), tiles_dn = m->E / (64 / std::max(1, std::min(8, m->K)));
    *part_gu = (size_t)tiles_gu * kMaxSegments * 64 * 4;
    *part_dn = (size_t)tiles_dn * kMaxSegments * 64 * 4;
    *cnt_gu = (size_t)tiles_gu * 4 + 64;           // + the two grid counters
    *cnt_dn = (size_t)tiles_dn * 4;
    return QMS_CUDA_OK;
}

int stream_forward_bs1(QmsCudaMoe *m, const float *xn, float *out, const float *resid, cudaStream_t s) {
    if (m->timing) QMS_CK(cudaEventRecord(m->ev[0], s));
    QMS_CK(launch_pdl(k_router_bs1, dim3(m->X), dim3(256), router_smem(m->E), s, (const float *)m->router_lm, m->X,
                      m->E, xn, m->K, m->xq_q, m->xq_d, m->xq_s, m->logits, m->sel, m->wts, m->cnt, m->err));
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[1], s));
        QMS_CK(cudaEventRecord(m->ev[2], s));
    }
    FfnArgs a;
    a.gu = m->gu;
    a.dn = m->dn;
    a.gu_expert = m->gu_expert;
    a.dn_expert = m->dn_expert;
    a.nbE = m->nbE;
    a.nbF = m->nbF;
    a.F = m->F;
    a.E = m->E;
    a.K = m->K;
    a.nst = m->gu_nst;
    a.xq_q = m->xq_q;
    a.xq_d = m->xq_d;
    a.xq_s = m->xq_s;
    a.aq_q = m->aq_q;
    a.aq_d = m->aq_d;
    a.aq_s = m->aq_s;
    a.part_gu = m->part_gu;
    a.part_dn = m->part_dn;
    a.tcnt_gu = m->tcnt_gu;
    a.tcnt_dn = m->tcnt_dn;
    a.sel = m->sel;
    a.wts = m->wts;
    a.resid = resid;
    a.out = out;
    a.grid_cnt = m->tcnt_gu + m->K * (m->F / 32);
    a.err = m->err;
    QMS_CK(launch_pdl(ffn_kernel(m), dim3(m->nsm), dim3(kStreamThreads), ffn_smem(m), s, a));
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[3], s));
        QMS_CK(cudaEventRecord(m->ev[4], s));
        QMS_CK(cudaEventRecord(m->ev[5], s));
    }
    return QMS_CUDA_OK;
}

}  // namespace qms
