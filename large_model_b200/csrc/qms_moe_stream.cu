// qms_moe_stream.cu - batch-1 decode of the MoE block as ONE kernel per call, streamed from HBM
// with TMA bulk copies.
//
// A decode token reads 8 experts x 10.6 MB of Q4_0 weights per 235B layer and does ~3.5 integer
// ops per byte, so the block is bound by HBM bandwidth; on B200 every separately launched stream
// of a few tens of MB loses microseconds to launch, ramp-up and tail, and every global round trip
// taken while the stream saturates HBM costs a microsecond or more. k_decode_bs1 is persistent
// (one CTA per SM: 16 consumer warps, a producer warp, an epilogue warp) and does:
//   routing   CTA e < X bulk-copies router row e (stored lane-major) into shared memory before
//             griddepcontrol.wait, computes logit e in the reference's exact F32 order and
//             publishes it; every CTA quantises xn to Q8 itself, gathers the X logits and selects
//             the experts itself, so no CTA waits for a designated one and no second kernel runs;
//   gate/up   the CTA's share of all K experts' gate/up stages (eight chunks of 8 rows x 16
//             blocks, 18 KB) is bulk-copied into an mbarrier ring; consumer warps run dp4a dots
//             against the token's Q8 row. A tile is 32 gate + 32 up rows, i.e. one SwiGLU + Q8
//             re-quantisation group (src/model.c:989-997), finished by the epilogue warp;
//   down      the consumers gather every CTA's Q8 groups (bounded polls) while the ring keeps
//             filling with down chunks; a down tile is 8 output rows x 8 experts, combined in
//             selection order with one FMA per expert (src/model.c:1152-1162) plus the optional
//             residual.
// Work is split over the CTAs by stages, not tiles, so every SM streams the same number of bytes
// (+-1 stage). A tile split between CTAs leaves partial row sums in global memory; the tile's last
// CTA adds them in CTA order, so results do not depend on timing. Everything exchanged between
// CTAs (logits, partial sums, Q8 groups) travels as flagged words: 32 data bits and a call stamp in
// one 64-bit store, so a reader polls the data itself and no fence, atomic or counter sits on the
// critical path. Each CTA keeps its own stamp word (all CTAs run every call, so they agree). The
// grid (one CTA per SM) is always fully resident: the kernel needs most of an SM's shared memory
// and nothing it waits for runs behind it. Every wait is bounded: on timeout the kernel records an
// error bit in *err, stops issuing copies, waits (bounded) for the copies it already issued and
// returns.
#include <algorithm>

#include "qms_moe.cuh"
#include "qms_router.cuh"

namespace qms {

constexpr int kChunkWarps = 2;                     // consumer warps per chunk (8 rows / kChunkWarps each)
constexpr int kConsumerWarps = 8 * kChunkWarps;    // a stage is 8 chunks
constexpr int kStreamThreads = (kConsumerWarps + 2) * 32;   // + producer warp + epilogue warp
constexpr int kMaxSegments = 4;                    // CTAs a tile may be split across
constexpr uint32_t kSpinLimit = 1u << 22;           // polls before a wait gives up (>= 0.1 s with backoff)
constexpr uint32_t kPollBackoffNs = 100;
constexpr size_t kSmemOptIn = 232448;              // 227 KB: per-block dynamic shared memory on sm_100
#ifndef QMS_STREAM_MAX_RING
#define QMS_STREAM_MAX_RING 12
#endif

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
// A failed poll backs off briefly: mbarrier polls and the consumers' shared-memory loads and
// shuffles share one pipe, so 17 warps polling flat out slow down the warps that have work.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort, int *err, int code) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (++n == kSpinLimit) {
            *abort = 1;
            atomicOr(err, code);
            return false;
        }
        __nanosleep(kPollBackoffNs);
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

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

// Static split of U stage-units over G CTAs: CTA c owns [lo(c), lo(c+1)).
__host__ __device__ inline int part_lo(int c, int U, int G) { return (int)((int64_t)c * U / G); }
__host__ __device__ inline int part_owner(int u, int U, int G) { return (int)(((int64_t)(u + 1) * G - 1) / U); }

// A CTA's units [u0, u1) form tile segments: a head segment (the end of a tile started by the
// previous CTA), a tail segment (the start of a tile finished by the next CTA) and whole tiles in
// between. Segments of split tiles are processed first, so the cross-CTA merges they need happen
// early and a CTA's last work is a whole tile, which needs no merge.
struct Segs {
    int u0, u1, S, t_first, t_last, head_s0, tail_s1, nfull, full0, n;
    __device__ Segs(int u0_, int u1_, int S_) : u0(u0_), u1(u1_), S(S_) {
        n = 0;
        if (u0 >= u1) return;
        t_first = u0 / S;
        t_last = (u1 - 1) / S;
        head_s0 = u0 - t_first * S;
        tail_s1 = u1 - t_last * S;                 // end stage (exclusive) of the last tile
        const bool head = head_s0 != 0 || (t_first == t_last && tail_s1 != S);
        const bool tail = t_last != t_first && tail_s1 != S;
        full0 = head ? t_first + 1 : t_first;
        const int full1 = tail ? t_last : t_last + 1;
        nfull = full1 - full0;
        n = (tail ? 1 : 0) + (head ? 1 : 0) + nfull;
        has_head = head;
        has_tail = tail;
    }
    bool has_head = false, has_tail = false;
    // k-th segment in processing order: tail, head, then whole tiles
    __device__ void get(int k, int &tile, int &s0, int &s1) const {
        if (has_tail) {
            if (k == 0) { tile = t_last; s0 = 0; s1 = tail_s1; return; }
            k--;
        }
        if (has_head) {
            if (k == 0) { tile = t_first; s0 = head_s0; s1 = t_first == t_last ? tail_s1 : S; return; }
            k--;
        }
        tile = full0 + k;
        s0 = 0;
        s1 = S;
    }
};

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

// One consumer warp's share of a stage: rows rs + RSTEP * (r0 + p) of its chunk (8 rows x SB
// blocks, lane = row set rs x block bl) against one Q8 row.
template <int SB>
__device__ __forceinline__ void chunk_dot(const uint8_t *chunk, const int8_t *xq, const float *xd, const int *xs8,
                                          int s, int bl, int rs, int r0, float (&acc)[SB / 4 / kChunkWarps]) {
    constexpr int P = SB / 4 / kChunkWarps, RSTEP = 32 / SB;
    const int b = s * SB + bl;
    const int4 xa0 = *reinterpret_cast<const int4 *>(xq + b * 32);
    const int4 xa1 = *reinterpret_cast<const int4 *>(xq + b * 32 + 16);
    const float d = xd[b];
    const int s8 = xs8[b];
#pragma unroll
    for (int p = 0; p < P; p++) {
        const int rr = rs + (r0 + p) * RSTEP;
        const uint4 nib = *reinterpret_cast<const uint4 *>(chunk + chunk_nib_off(SB, rr, bl));
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(chunk + chunk_scale_off(SB, rr, bl)));
        acc[p] = fmaf((float)(q4_block_isum(nib, xa0, xa1) - s8), dw * d, acc[p]);
    }
}

// The same for Q4_1 chunks (value d q + m): d dx isum + m ds with ds = dx * (float)sum, the
// activation block's sum term of src/kernels.c:109-121; xs holds the plain block sums.
template <int SB>
__device__ __forceinline__ void chunk_dot_q41(const uint8_t *chunk, const int8_t *xq, const float *xd, const int *xs,
                                              int s, int bl, int rs, int r0, float (&acc)[SB / 4 / kChunkWarps]) {
    constexpr int P = SB / 4 / kChunkWarps, RSTEP = 32 / SB;
    const int b = s * SB + bl;
    const int4 xa0 = *reinterpret_cast<const int4 *>(xq + b * 32);
    const int4 xa1 = *reinterpret_cast<const int4 *>(xq + b * 32 + 16);
    const float d = xd[b];
    const float ds = d * (float)xs[b];
#pragma unroll
    for (int p = 0; p < P; p++) {
        const int rr = rs + (r0 + p) * RSTEP;
        const uint4 nib = *reinterpret_cast<const uint4 *>(chunk + chunk_nib_off(SB, rr, bl));
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(chunk + chunk_scale_off(SB, rr, bl)));
        const float mw = h2f(*reinterpret_cast<const uint16_t *>(chunk + chunk_min_off(SB, rr, bl)));
        acc[p] = fmaf((float)q4_block_isum(nib, xa0, xa1), dw * d, acc[p]);
        acc[p] = fmaf(mw, ds, acc[p]);
    }
}

// ---- routing inside the decode kernel -----------------------------------------------------------
// The reference (src/model.c:1045-1064) takes prob[e] = exp((double)l_e - max) / z in double,
// picks the top k by repeated strict-'>' argmax over prob (ties, including probabilities that
// underflow to 0, go to the lower index) and weighs them (float)(p_j / sum_j p_j), the sum in
// selection order. On B200 a dependent double operation costs ~90 cycles, so the critical path
// ranks the float logits instead (ties to the lower index; exp(l - max) / z is non-decreasing in
// l, so the order agrees) and proves the agreement from the double exponentials of the top K+1
// alone: if each exceeds the next by more than the rounding of one division, their
// probabilities are strictly decreasing. Only when that proof fails does the selection wait for
// the exact double ranking; z, the probabilities and the weights are computed after the experts
// are known, while the first weights stream in.

// Float rank of every logit (ties to the lower index), split over tpl = 512 / X threads per logit
// (lanes tpl*e .. tpl*e + tpl - 1). Thread `part` of a logit reads float4 groups part, part + tpl,
// ... so the lanes of a warp hit different banks (contiguous spans per part would all map to the
// same banks and serialise). lg is padded with -inf up to kLogitPad entries; t_cand[r] = the logit
// of rank r for r <= K. Called by all consumer threads.
constexpr int kLogitPad = 256;
__device__ __forceinline__ void rank_candidates(const float *lg, int X, int K, int tid, int *t_cand) {
    const int tpl = X <= 128 ? 4 : 2;
    const int e = tid / tpl, part = tid % tpl;
    const int n4 = (X + 4 * tpl - 1) / (4 * tpl);    // float4 groups per thread; 4 * tpl * n4 <= kLogitPad
    int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
    if (e < X) {
        const float v = lg[e];
        const float4 *l4 = reinterpret_cast<const float4 *>(lg);
#pragma unroll 8
        for (int q = 0; q < n4; q++) {
            const int f = part + tpl * q;
            const float4 u = l4[f];
            const int jj = 4 * f;
            r0 += (u.x > v) | ((u.x == v) & (jj + 0 < e));
            r1 += (u.y > v) | ((u.y == v) & (jj + 1 < e));
            r2 += (u.z > v) | ((u.z == v) & (jj + 2 < e));
            r3 += (u.w > v) | ((u.w == v) & (jj + 3 < e));
        }
    }
    int rank = r0 + r1 + r2 + r3;
    rank += __shfl_xor_sync(0xffffffffu, rank, 1);
    if (tpl == 4) rank += __shfl_xor_sync(0xffffffffu, rank, 2);
    if (e < X && part == 0 && rank <= K) t_cand[rank] = e;
}

// The exact ranking of the double probabilities (ties, underflow, NaN): cold, kept out of line.
__device__ __noinline__ void route_exact(const float *lg, int X, int K, double mx, int *s_sel, double *t_ex,
                                         double *t_pj, double &z) {
    const int lane = threadIdx.x & 31;
    z = 0.0;                                        // z in topk_token's order (qms_moe.cuh)
    for (int b = 0; b < X; b += 32) {
        const int e = b + lane;
        const double x = e < X ? exp((double)lg[e] - mx) : 0.0;
        if (e < X) t_ex[e] = x;
        double zb = x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) zb += __shfl_xor_sync(0xffffffffu, zb, o);
        z += zb;
    }
    __syncwarp();
    for (int e = lane; e < X; e += 32) t_ex[e] = t_ex[e] / z;   // probabilities
    __syncwarp();
    for (int e = lane; e < X; e += 32) {            // exact ranking of the doubles
        const double p = t_ex[e];
        int rk = 0;
        for (int j = 0; j < e; j++) rk += t_ex[j] >= p;
        for (int j = e + 1; j < X; j++) rk += t_ex[j] > p;
        if (rk < K) {
            s_sel[rk] = e;
            t_pj[rk] = p;
        }
    }
    z = -1.0;                                       // t_pj is final
    __syncwarp();
}

// Warp 0: turns the float candidates into the reference's selection. Returns after s_sel holds
// it (verified, or ranked exactly); route_weights then finishes the probabilities and weights.
__device__ void route_select(const float *lg, int X, int K, const int *t_cand, int *s_sel, double *t_ex,
                             double *t_pj, double &z) {
    const int lane = threadIdx.x & 31;
    const int nc = K < X ? K + 1 : K, nchk = K < X ? K : K - 1;
    const double mx = (double)lg[t_cand[0]];        // the largest logit
    bool exact = nc > 32;
    if (!exact) {
        const double ex = lane < nc ? exp((double)lg[t_cand[lane]] - mx) : 0.0;
        const double nx = __shfl_down_sync(0xffffffffu, ex, 1);
        // p_r > p_{r+1} is certain once ex_r > ex_{r+1} (1 + 2^-48) and ex_r is far from the
        // subnormal range (then p = ex / z >= 2^-1008 is normal too): one division by z rounds
        // by at most 2^-53 relative. NaN logits fail the test and take the exact path.
        exact = __any_sync(0xffffffffu, (lane < nchk && !(ex > nx * (1.0 + 0x1p-48))) || (lane < nc && !(ex >= 0x1p-1000)));
        if (!exact && lane < K) s_sel[lane] = t_cand[lane];
    }
    z = 0.0;
    if (exact) route_exact(lg, X, K, mx, s_sel, t_ex, t_pj, z);
}

// Warp 0, after route_select: the weights (float)(p_j / sum_j p_j), sum in selection order.
__device__ void route_weights(const float *lg, int X, int K, const int *s_sel, double *t_pj, double z,
                              float *s_w, int *sel, float *wts) {
    const int lane = threadIdx.x & 31;
    if (z >= 0.0) {                                 // verified selection: z and p_j still to come
        const double mx = (double)lg[s_sel[0]];
        for (int b = 0; b < X; b += 32) {
            const int e = b + lane;
            double zb = e < X ? exp((double)lg[e] - mx) : 0.0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) zb += __shfl_xor_sync(0xffffffffu, zb, o);
            z += zb;
        }
        for (int t = lane; t < K; t += 32) t_pj[t] = exp((double)lg[s_sel[t]] - mx) / z;
        __syncwarp();
    }
    for (int t = lane; t < K; t += 32) {
        double ws = 0.0;
        for (int j = 0; j < K; j++) ws += t_pj[j];
        const float w = (float)(t_pj[t] / ws);
        s_w[t] = w;
        if (sel) sel[t] = s_sel[t];
        if (wts) wts[t] = w;
    }
    __syncwarp();
}

// ---- gate/up + SwiGLU + Q8, then down + combine, in one stream (batch 1) ------------------------
struct DecodeArgs {
    const float *router_lm;               // [X][16][E/16]: element 16*i + k of a row at [k][i]
    const float *xn, *resid;
    float *out;
    const uint8_t *gu, *dn;               // staged experts
    size_t gu_expert, dn_expert;
    int nbE, nbF, F, E, K, X, nst;
    unsigned long long *lgf;              // [X] flagged logits
    unsigned long long *aq;               // [K*F/32 groups][10] flagged Q8 groups: q (8 words), d, sum
    unsigned long long *part_gu, *part_dn;   // flagged partial sums of tiles split across CTAs
    unsigned *stamps;                     // [G] per-CTA call stamps
    float *logits;                        // optional outputs (NULL to skip): [X]
    int *sel;                             // [K] (written by CTA 0)
    float *wts;                           // [K] (written by CTA 0)
    int *err;
};

constexpr int kAqWords = 10;              // flagged words per Q8 group

// Poll a flagged word until it carries `stamp`; bounded like every other wait.
__device__ __forceinline__ bool wait_flagged(const unsigned long long *p, uint32_t stamp, unsigned long long &v,
                                             volatile int *abort, int *err, int code) {
    uint32_t n = 0;
    while ((uint32_t)(v >> 32) != stamp) {
        if (*abort) return false;
        if (++n == kSpinLimit) {
            *abort = 1;
            atomicOr(err, code);
            return false;
        }
        __nanosleep(32);
        v = ld_flagged(p);
    }
    return true;
}

// Epilogue-warp half of a tile split across CTAs (2 sums per lane: [lane], [32 + lane]). Every
// CTA but the tile's last publishes its partial sums as flagged words and returns false; the last
// CTA polls them and returns true with the full sums, added in CTA order so the result does not
// depend on timing. A CTA's non-last segments of split tiles are the first work it does, so the
// last CTA rarely waits.
__device__ __forceinline__ bool merge_partial(unsigned long long *part, int tile, int S, int U, int G, int c,
                                              uint32_t stamp, float (&v)[2], volatile int *abort, int *err) {
    const int lane = threadIdx.x & 31;
    const int first = part_owner(tile * S, U, G), last = part_owner(tile * S + S - 1, U, G);
    unsigned long long *pt = part + (size_t)tile * kMaxSegments * 64;
    if (c != last) {
        st_flagged(pt + (c - first) * 64 + lane, __float_as_uint(v[0]), stamp);
        st_flagged(pt + (c - first) * 64 + 32 + lane, __float_as_uint(v[1]), stamp);
        return false;
    }
    float a0 = 0.0f, a1 = 0.0f;
    bool ok = true;
    for (int q = 0; q < last - first; q++) {
        unsigned long long w0 = ld_flagged(pt + q * 64 + lane), w1 = ld_flagged(pt + q * 64 + 32 + lane);
        ok = ok && wait_flagged(pt + q * 64 + lane, stamp, w0, abort, err, ERR_GRID) &&
             wait_flagged(pt + q * 64 + 32 + lane, stamp, w1, abort, err, ERR_GRID);
        a0 += __uint_as_float((uint32_t)w0);
        a1 += __uint_as_float((uint32_t)w1);
    }
    v[0] = a0 + v[0];
    v[1] = a1 + v[1];
    return __all_sync(0xffffffffu, ok);
}

constexpr int kSumBufs = 4;        // tile-sum hand-off buffers between consumer and epilogue warps

template <int SBG, int SBD, int DQ1>
__global__ void __launch_bounds__(kStreamThreads, 1) k_decode_bs1(const DecodeArgs a) {
    // DQ1: down weights are Q4_1 (chunks carry a min plane), else Q4_0
    constexpr uint32_t GBG = 8 * SBG * 18, STG = 8 * GBG, GBD = 8 * SBD * (DQ1 ? 20 : 18), STD = 8 * GBD;
    constexpr uint32_t SLOT = STG > STD ? STG : STD;
    constexpr int PG = SBG / 4 / kChunkWarps, RSG = 32 / SBG, PD = SBD / 4 / kChunkWarps, RSD = 32 / SBD;
    extern __shared__ __align__(128) uint8_t smem[];
    const int nst = a.nst, K = a.K, F = a.F, E = a.E, X = a.X, nbE = a.nbE, nbF = a.nbF;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nst * SLOT);
    uint64_t *empty = full + nst;
    uint64_t *sfull = empty + nst;                                  // [kSumBufs] sums written
    uint64_t *sempty = sfull + kSumBufs;                            // [kSumBufs] sums consumed
    uint64_t *rbar = sempty + kSumBufs;                             // router row landed
    uint64_t *selbar = rbar + 1;                                    // experts chosen
    int8_t *sxq = reinterpret_cast<int8_t *>(selbar + 1);          // [nbE*32] the token's Q8 row
    float *sxd = reinterpret_cast<float *>(sxq + nbE * 32);         // [nbE]
    int *sxs = reinterpret_cast<int *>(sxd + nbE);                  // [nbE], 8 * sum
    int8_t *saq = reinterpret_cast<int8_t *>(sxs + nbE);            // [K][F]
    float *sad = reinterpret_cast<float *>(saq + K * F);            // [K][nbF]
    int *sas = reinterpret_cast<int *>(sad + K * nbF);              // [K][nbF], 8 * sum
    float *sbuf = reinterpret_cast<float *>(sas + K * nbF);         // [kSumBufs][64] tile sums
    float *slg = sbuf + kSumBufs * 64;                              // [kLogitPad] this call's logits
    // routing scratch inside the ring, which carries no stage before the experts are known
    const int L = E / 16, PS = L + 4;
    float *srow = reinterpret_cast<float *>(ring);                  // [16][PS] router row, lane-major
    float *sx = srow + 16 * PS;                                     // [16][PS] xn, lane-major
    __shared__ int s_abort;
    __shared__ const uint8_t *s_gu_base[8], *s_dn_base[8];   // producer: selected experts' weights
    __shared__ int s_sel[64];
    __shared__ float s_w[64];                                  // epilogue: routing weights
    __shared__ uint32_t s_stamp;
    __shared__ int t_cand[65];                                 // routing: float rank -> logit
    __shared__ double t_ex[256], t_pj[64], s_z;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x, c = blockIdx.x;
    const int Sg = nbE / SBG, tps = F / 32, ntg = K * tps, Ug = ntg * Sg;
    const int Sd = nbF / SBD, RBE = 8 / K, RT = 8 * RBE, Ud = (a.E / RT) * Sd;
    const uint32_t WSD = (uint32_t)Sd * GBD;        // one chunk's share of a down stage (Sd slots)
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
        mbar_init(rbar, 1);
        mbar_init(selbar, 1);
        fence_mbar_init();
        if (c < X) {                                // router row c, lane-major, before the wait
            mbar_arrive_expect_tx(rbar, (uint32_t)E * 4);
            const uint64_t pol = evict_first_policy();
            for (int k = 0; k < 16; k++)
                bulk_load(srow + k * PS, a.router_lm + (size_t)c * E + (size_t)k * L, (uint32_t)L * 4, rbar, pol);
        }
    }
    __syncthreads();
    pdl_trigger();                                  // the next call's kernel may stage its router row
    pdl_wait();                                     // xn comes from the previous kernel
    volatile int *abort_flag = &s_abort;

    if (warp == kConsumerWarps) {                   // ---- producer: one stream, gate/up then down
        if (lane == 0) {
            bool ok = wait_bounded(selbar, 0, abort_flag, a.err, ERR_PRODUCER) && !*abort_flag;
            const uint64_t pol = evict_first_policy();
            // expert bases live in shared memory: a local array would sit in local memory, and
            // every load from it that misses L1 queues behind the stream in L2
            for (int j = 0; j < 8; j++) s_gu_base[j] = a.gu + (size_t)(j < K ? s_sel[j] : 0) * a.gu_expert;
            for (int gi = 0; gi < 8; gi++) s_dn_base[gi] = a.dn + (size_t)s_sel[gi / RBE] * a.dn_expert;
            Ring r(nst);
            int issued = 0;
            const Segs sg(ug0, ug1, Sg), sd(ud0, ud1, Sd);
            for (int k = 0; k < sg.n && ok; k++) {
                int tile, s0, s1;
                sg.get(k, tile, s0, s1);
                const uint8_t *src = s_gu_base[tile / tps] + (size_t)(tile % tps) * tile_bytes;
                for (int s = s0; s < s1 && ok; s++) {
                    if (issued >= nst &&
                        !(ok = wait_bounded(&empty[r.slot], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER)))
                        break;
                    mbar_arrive_expect_tx(&full[r.slot], STG);
                    bulk_load(ring + (size_t)r.slot * SLOT, src + (size_t)s * STG, STG, &full[r.slot], pol);
                    issued++;
                    r.next();
                }
            }
            // The ring fills with down chunks while the consumers wait for every CTA's SwiGLU groups.
            // First pad to a multiple of Sd slots with stages that carry no data.
            while (r.slot % Sd != 0 && ok) {
                if (issued >= nst &&
                    !(ok = wait_bounded(&empty[r.slot], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER)))
                    break;
                mbar_arrive(&full[r.slot]);
                issued++;
                r.next();
            }
            for (int k = 0; k < sd.n && ok; k++) {
                int tile, s0, s1;
                sd.get(k, tile, s0, s1);
                // A down stage is one tile segment: per chunk (expert / row block) its stages s0..s1
                // are adjacent in HBM, so it is ONE copy of up to Sd * GBD bytes (many small copies
                // stream far slower). It takes Sd whole slots starting at a multiple of Sd (nst is
                // one, so it never wraps).
                for (int q = 0; q < Sd && ok; q++)
                    if (issued + q >= nst)
                        ok = wait_bounded(&empty[r.slot + q], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER);
                if (!ok) break;
                const uint32_t bytes = (uint32_t)(s1 - s0) * GBD;
                mbar_arrive_expect_tx(&full[r.slot], 8 * bytes);
                uint8_t *dst = ring + (size_t)r.slot * SLOT;
                for (int gi = 0; gi < 8; gi++) {
                    const size_t rb = (size_t)tile * RBE + gi % RBE;
                    bulk_load(dst + gi * WSD, s_dn_base[gi] + (rb * Sd + s0) * GBD, bytes, &full[r.slot], pol);
                }
                for (int q = 1; q < Sd; q++) mbar_arrive(&full[r.slot + q]);
                issued += Sd;
                for (int q = 0; q < Sd; q++) r.next();
            }
            if (!ok || *abort_flag) drain_issued(full, nst, issued, a.err);
        }
        return;
    }

    if (warp == kConsumerWarps + 1) {               // ---- epilogue warp: SwiGLU/Q8, merges, combine
        // first the routing weights (the combine needs them, the experts' gate/up does not)
        bool ok = __all_sync(0xffffffffu, wait_bounded(selbar, 0, abort_flag, a.err, ERR_CONSUMER)) && !*abort_flag;
        if (ok) route_weights(slg, X, K, s_sel, t_pj, s_z, s_w, c == 0 ? a.sel : nullptr, c == 0 ? a.wts : nullptr);
        Ring sr(kSumBufs);
        const uint32_t stamp = s_stamp;
        for (int pass = 0; pass < 2; pass++) {
            const bool gate = pass == 0;
            const int S = gate ? Sg : Sd, U = gate ? Ug : Ud;
            const Segs sq(gate ? ug0 : ud0, gate ? ug1 : ud1, S);
            for (int k = 0; k < sq.n; k++) {
                int tile, s0, s1;
                sq.get(k, tile, s0, s1);
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&sfull[sr.slot], sr.phase, abort_flag, a.err,
                                                                  ERR_CONSUMER));
                float v[2] = {sbuf[sr.slot * 64 + lane], sbuf[sr.slot * 64 + 32 + lane]};
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[sr.slot]);
                sr.next();
                if (!ok) continue;
                bool mine = true;
                if (!(s0 == 0 && s1 == S))
                    mine = merge_partial(gate ? a.part_gu : a.part_dn, tile, S, U, G, c, stamp, v, abort_flag, a.err);
                if (!mine) continue;
                if (gate) {                         // rows 0-31: gate f0+lane, rows 32-63: up f0+lane
                    // Q8 group `tile` (expert slot tile / tps, values f0..f0+31) as flagged words
                    const float av = __fmul_rn(__fdiv_rn(v[0], __fadd_rn(1.0f, expf(-v[0]))), v[1]);
                    const Q8Lane q8 = quantize_lane(av);
                    uint32_t b4 = (uint32_t)(q8.q & 0xff) << (8 * (lane & 3));
                    b4 |= __shfl_xor_sync(0xffffffffu, b4, 1);
                    b4 |= __shfl_xor_sync(0xffffffffu, b4, 2);
                    unsigned long long *dst = a.aq + (size_t)tile * kAqWords;
                    if ((lane & 3) == 0) st_flagged(dst + (lane >> 2), b4, stamp);
                    if (lane == 1) st_flagged(dst + 8, __float_as_uint(q8.d), stamp);
                    if (lane == 2) st_flagged(dst + 9, (uint32_t)q8.sum, stamp);
                } else {                            // sum index (j*RBE + rbi)*8 + rr: expert j, row rr of block rbi
                    const int rbi = (lane >> 3) & 7, rr = lane & 7;
                    float o = 0.0f;
                    for (int jj = 0; jj < K; jj++) {
                        const int idx = (jj * RBE + rbi) * 8 + rr;
                        const float lo = __shfl_sync(0xffffffffu, v[0], idx & 31);
                        const float hi = __shfl_sync(0xffffffffu, v[1], idx & 31);
                        o = __fmaf_rn(s_w[jj], idx < 32 ? lo : hi, o);
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

    // ---- consumers: routing first (the producer and the epilogue wait for it)
    const int tid = threadIdx.x;
    if (tid == 0) {
        const unsigned next = __ldcg(a.stamps + c) + 1;   // never 0: zeroed words are never current
        s_stamp = next ? next : 1;
        a.stamps[c] = s_stamp;
    }
    for (int q = tid; q < E / 4; q += kConsumerWarps * 32) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.xn) + q);
        const int j = 4 * q;
        sx[((j + 0) & 15) * PS + ((j + 0) >> 4)] = v.x;
        sx[((j + 1) & 15) * PS + ((j + 1) >> 4)] = v.y;
        sx[((j + 2) & 15) * PS + ((j + 2) >> 4)] = v.z;
        sx[((j + 3) & 15) * PS + ((j + 3) >> 4)] = v.w;
    }
    consumer_sync();
    const uint32_t stamp = s_stamp;
    bool ok = true;
    if (warp == 0) {
        if (c < X) {                                // logit c in qms_vec_dot_f32's exact order
            ok = __all_sync(0xffffffffu, wait_bounded(rbar, 0, abort_flag, a.err, ERR_ROUTER));
            const int k = lane & 15;
            const float *w = srow + k * PS, *x = sx + k * PS;
            float acc = 0.0f;
            int i = 0;
            for (; i + 32 <= L; i += 32) {         // 8 loads of each operand in flight per batch
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
            if (lane == 0 && ok) {
                st_flagged(a.lgf + c, __float_as_uint(acc), stamp);
                if (a.logits) a.logits[c] = acc;
            }
        }
    } else {                                        // the token's Q8 row (src/kernels.c:34-53)
        for (int b = warp - 1; b < nbE; b += kConsumerWarps - 1) {
            const int j = b * 32 + lane;
            const Q8Lane r = quantize_lane(sx[(j & 15) * PS + (j >> 4)]);
            sxq[j] = (int8_t)r.q;
            if (lane == 0) {
                sxd[b] = r.d;
                sxs[b] = 8 * r.sum;
            }
        }
    }
    if (tid < X) {                                  // every CTA's logit
        unsigned long long v = ld_flagged(a.lgf + tid);
        if (wait_flagged(a.lgf + tid, stamp, v, abort_flag, a.err, ERR_ROUTER)) slg[tid] = __uint_as_float((uint32_t)v);
    } else if (tid < kLogitPad) {
        slg[tid] = -INFINITY;                       // padding the rank loop may read
    }
    consumer_sync();
    rank_candidates(slg, X, K, tid, t_cand);
    consumer_sync();
    if (warp == 0) {
        double z = 0.0;
        if (!*abort_flag) route_select(slg, X, K, t_cand, s_sel, t_ex, t_pj, z);
        if (lane == 0) s_z = z;
        __syncwarp();
        if (lane == 0) mbar_arrive(selbar);         // producer and epilogue may start (they check the abort flag)
    }
    ok = !*abort_flag;

    // ---- consumers, phase A: gate/up
    const int g = warp / kChunkWarps, half = warp % kChunkWarps;   // chunk of the stage, row part
    Ring r(nst), sr(kSumBufs);
    int handed = 0;
    // hand a tile's 64 sums (8 per chunk) to the epilogue warp
    auto hand_off = [&](const float *acc, int P, int RS, int bl, int rs) {
        if (handed >= kSumBufs && ok)
            ok = __all_sync(0xffffffffu, wait_bounded(&sempty[sr.slot], sr.phase ^ 1, abort_flag, a.err, ERR_CONSUMER));
        if (bl == 0)
            for (int p = 0; p < P; p++) sbuf[sr.slot * 64 + g * 8 + rs + (half * P + p) * RS] = acc[p];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfull[sr.slot]);
        sr.next();
        handed++;
    };
    {
        const int bl = lane % SBG, rs = lane / SBG;
        const Segs sq(ug0, ug1, Sg);
        for (int k = 0; k < sq.n; k++) {
            int tile, s0, s1;
            sq.get(k, tile, s0, s1);
            float acc[PG];
#pragma unroll
            for (int p = 0; p < PG; p++) acc[p] = 0.0f;
            for (int s = s0; s < s1; s++, r.next()) {
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
                if (ok) {
                    chunk_dot<SBG>(ring + (size_t)r.slot * SLOT + g * GBG, sxq, sxd, sxs, s, bl, rs, half * PG, acc);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[r.slot]);
                }
            }
#pragma unroll
            for (int p = 0; p < PG; p++)
#pragma unroll
                for (int o = SBG / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(0xffffffffu, acc[p], o);
            hand_off(acc, PG, RSG, bl, rs);
        }
    }

    // the producer's padding slots before the first down stage, released before the wait so the
    // ring can fill with down stages meanwhile
    for (; r.slot % Sd != 0; r.next()) {
        if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&empty[r.slot]);
    }

    // ---- phase B: gather every CTA's Q8 groups as they appear, then down + combine. Each thread
    // keeps all its words in flight and re-polls only the pending ones, one round trip per round.
    if (ok) {
        const int nw = ntg * kAqWords;
        constexpr int kBatch = 8;
        for (int i0 = tid; i0 < nw && ok; i0 += kBatch * kConsumerWarps * 32) {
            unsigned long long v[kBatch];
            uint32_t pending = 0;
#pragma unroll
            for (int b = 0; b < kBatch; b++) {
                const int i = i0 + b * kConsumerWarps * 32;
                v[b] = i < nw ? ld_flagged(a.aq + i) : 0ull;
            }
            uint32_t n = 0;
            for (;;) {
#pragma unroll
                for (int b = 0; b < kBatch; b++) {
                    const int i = i0 + b * kConsumerWarps * 32;
                    if (i < nw && (uint32_t)(v[b] >> 32) != stamp) pending |= 1u << b;
                }
                if (!pending) break;
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                if (++n == kSpinLimit) {
                    *abort_flag = 1;
                    atomicOr(a.err, ERR_GRID);
                    ok = false;
                    break;
                }
                __nanosleep(64);
#pragma unroll
                for (int b = 0; b < kBatch; b++)
                    if (pending & (1u << b)) v[b] = ld_flagged(a.aq + i0 + b * kConsumerWarps * 32);
                pending = 0;
            }
            if (!ok) break;
#pragma unroll
            for (int b = 0; b < kBatch; b++) {
                const int i = i0 + b * kConsumerWarps * 32;
                if (i >= nw) continue;
                const int gi = i / kAqWords, w = i - gi * kAqWords;
                const uint32_t d = (uint32_t)v[b];
                if (w < 8) reinterpret_cast<uint32_t *>(saq)[gi * 8 + w] = d;
                else if (w == 8) sad[gi] = __uint_as_float(d);
                else sas[gi] = DQ1 ? (int)d : 8 * (int)d;   // block sum (Q4_1) or 8 x it (Q4_0)
            }
        }
    }
    consumer_sync();
    ok = ok && !*abort_flag;                        // every failed wait raised the abort flag
    {
        const int j = g / RBE, bl = lane % SBD, rs = lane / SBD;
        const int8_t *xq = saq + (size_t)j * F;
        const float *xdv = sad + j * nbF;
        const int *xsv = sas + j * nbF;
        const Segs sq(ud0, ud1, Sd);
        for (int k = 0; k < sq.n; k++) {
            int tile, s0, s1;
            sq.get(k, tile, s0, s1);
            float acc[PD];
#pragma unroll
            for (int p = 0; p < PD; p++) acc[p] = 0.0f;
            if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
            if (ok) {
                const uint8_t *chunk = ring + (size_t)r.slot * SLOT + g * WSD;   // [chunk][stage s0..s1]
                for (int s = s0; s < s1; s++)
                    if (DQ1) chunk_dot_q41<SBD>(chunk + (s - s0) * GBD, xq, xdv, xsv, s, bl, rs, half * PD, acc);
                    else chunk_dot<SBD>(chunk + (s - s0) * GBD, xq, xdv, xsv, s, bl, rs, half * PD, acc);
                __syncwarp();
                if (lane == 0)
                    for (int q = 0; q < Sd; q++) mbar_arrive(&empty[r.slot + q]);
            }
            for (int q = 0; q < Sd; q++) r.next();
#pragma unroll
            for (int p = 0; p < PD; p++)
#pragma unroll
                for (int o = SBD / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(0xffffffffu, acc[p], o);
            hand_off(acc, PD, RSD, bl, rs);
        }
    }
}

// ---- host side -----------------------------------------------------------------------------------
static uint32_t dec_slot(const QmsCudaMoe *m) { return 8 * std::max(m->cgu.GB, m->cdn.GB); }
static size_t dec_fixed(const QmsCudaMoe *m) {
    return (2 * kSumBufs + 2) * 8 + (size_t)m->nbE * 40 + (size_t)m->K * m->F + (size_t)m->K * m->nbF * 8 +
           kSumBufs * 64 * 4 + (size_t)kLogitPad * 4;
}
static size_t dec_smem(const QmsCudaMoe *m) { return (size_t)m->gu_nst * (dec_slot(m) + 16) + dec_fixed(m); }

static int max_segments(int U, int S, int G) {
    int worst = 1;
    for (int tile = 0; tile * S < U; tile++)
        worst = std::max(worst, part_owner(tile * S + S - 1, U, G) - part_owner(tile * S, U, G) + 1);
    return worst;
}

typedef void (*DecodeKernel)(const DecodeArgs);
static DecodeKernel dec_kernel(const QmsCudaMoe *m) {
    if (m->cdn.q1) {
        if (m->cgu.SB == 16) return m->cdn.SB == 16 ? k_decode_bs1<16, 16, 1> : k_decode_bs1<16, 8, 1>;
        return m->cdn.SB == 16 ? k_decode_bs1<8, 16, 1> : k_decode_bs1<8, 8, 1>;
    }
    if (m->cgu.SB == 16) return m->cdn.SB == 16 ? k_decode_bs1<16, 16, 0> : k_decode_bs1<16, 8, 0>;
    return m->cdn.SB == 16 ? k_decode_bs1<8, 16, 0> : k_decode_bs1<8, 8, 0>;
}

int stream_prepare(QmsCudaMoe *m) {
    m->stream_ok = 0;
    if (!(m->K == 1 || m->K == 2 || m->K == 4 || m->K == 8) || m->X > 256 || 2 * m->X > m->E) return QMS_CUDA_OK;
    if (m->nbE % m->cgu.SB || m->nbF % m->cdn.SB) return QMS_CUDA_OK;
    const uint32_t slot = dec_slot(m);
    cudaFuncAttributes fa;
    QMS_CK(cudaFuncGetAttributes(&fa, dec_kernel(m)));
    // the deepest ring that fits, a multiple of the down stage width cdn.S so a down stage never
    // wraps around it; routing scratch (router row + xn, lane-major) lives in its first slots
    const size_t avail = kSmemOptIn - fa.sharedSizeBytes - dec_fixed(m);
    const int fit = (int)std::min<size_t>(QMS_STREAM_MAX_RING, avail / (slot + 16));
    m->gu_nst = fit / m->cdn.S * m->cdn.S;
    m->dn_nst = m->gu_nst;
    if (m->gu_nst < 4 || m->gu_nst < m->cdn.S) return QMS_CUDA_OK;
    if ((size_t)2 * 16 * (m->E / 16 + 4) * 4 > (size_t)m->gu_nst * slot) return QMS_CUDA_OK;
    const int Ugu = m->K * (m->F / 32) * m->cgu.S, Udn = (m->E / (64 / m->K)) * m->cdn.S;
    if (max_segments(Ugu, m->cgu.S, m->nsm) > kMaxSegments || max_segments(Udn, m->cdn.S, m->nsm) > kMaxSegments)
        return QMS_CUDA_OK;
    const DecodeKernel dk = dec_kernel(m);
    QMS_CK(cudaFuncSetAttribute(dk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec_smem(m)));
    QMS_CK(cudaFuncSetAttribute(dk, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    m->stream_ok = 1;
    return QMS_CUDA_OK;
}

int stream_scratch_sizes(const QmsCudaMoe *m, StreamScratch *sz) {
    const int tiles_gu = m->K * (m->F / 32), tiles_dn = m->E / (64 / std::max(1, std::min(8, m->K)));
    sz->lg_flagged = (size_t)m->X * 8;
    sz->stamps = (size_t)m->nsm * 4;
    sz->aq_flagged = (size_t)tiles_gu * kAqWords * 8;
    sz->part_gu = (size_t)tiles_gu * kMaxSegments * 64 * 8;
    sz->part_dn = (size_t)tiles_dn * kMaxSegments * 64 * 8;
    return QMS_CUDA_OK;
}

int stream_forward_bs1(QmsCudaMoe *m, const float *xn, float *out, const float *resid, cudaStream_t s) {
    DecodeArgs a;
    a.router_lm = m->router_lm;
    a.xn = xn;
    a.resid = resid;
    a.out = out;
    a.gu = m->gu;
    a.dn = m->dn;
    a.gu_expert = m->gu_expert;
    a.dn_expert = m->dn_expert;
    a.nbE = m->nbE;
    a.nbF = m->nbF;
    a.F = m->F;
    a.E = m->E;
    a.K = m->K;
    a.X = m->X;
    a.nst = m->gu_nst;
    a.lgf = m->lg_flagged;
    a.aq = m->aq_flagged;
    a.part_gu = m->part_gu;
    a.part_dn = m->part_dn;
    a.stamps = m->stamps;
    a.logits = m->logits;
    a.sel = m->sel;
    a.wts = m->wts;
    a.err = m->err;
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[0], s));
        QMS_CK(cudaEventRecord(m->ev[1], s));
        QMS_CK(cudaEventRecord(m->ev[2], s));
    }
    QMS_CK(launch_pdl(dec_kernel(m), dim3(m->nsm), dim3(kStreamThreads), dec_smem(m), s, a));
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[3], s));
        QMS_CK(cudaEventRecord(m->ev[4], s));
        QMS_CK(cudaEventRecord(m->ev[5], s));
    }
    return QMS_CUDA_OK;
}

}  // namespace qms
