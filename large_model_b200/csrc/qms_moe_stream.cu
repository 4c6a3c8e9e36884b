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
//   tiles     a tile is one 32-value group of one selected expert's intermediate activation,
//             i.e. one SwiGLU + Q8 group (src/model.c:989-997). Its work is Sg gate/up stages (32
//             gate + 32 up rows over all E/32 blocks: eight chunks of 8 rows x 16 blocks, 18 KB)
//             followed by Rq down stages (the group's block column of the expert's down matrix,
//             RD rows x one block each). All tiles' stages are split evenly over the CTAs, so every
//             SM streams the same bytes (+-1 stage), and a CTA does the down work of the tiles it
//             finished itself: nothing grid-wide separates gate/up from down, and the producer
//             streams gate/up of tile k+1 before down of tile k so the SwiGLU never stalls it;
//   gate/up   consumer warps run dp4a dots against the token's Q8 row; the epilogue warp turns a
//             tile's 64 sums into silu(g)*u and its Q8 group;
//   down      the consumers add w_j * (the group's down dots) into a partial output vector in
//             shared memory (the down product split over the intermediate dimension);
//   combine   every CTA publishes its partial vector; CTA c then sums its share of the E rows over
//             all CTAs in CTA order, adds the optional residual and writes them.
// A tile split between two CTAs hands over its partial gate/up sums or its finished Q8 group
// through global memory: the CTA that produces the hand-over processes that tile first, the CTA
// that takes it processes that tile last. Everything exchanged between CTAs travels as flagged
// words: 32 data bits and a call stamp in one 64-bit store, so a reader polls the data itself and
// no fence, atomic or counter sits on the critical path. Each CTA keeps its own stamp word (all
// CTAs run every call, so they agree). The grid (one CTA per SM) is always fully resident: the
// kernel needs most of an SM's shared memory and nothing it waits for runs behind it. Results do
// not depend on timing: every sum has a fixed order. Every wait is bounded: on timeout the kernel
// records an error bit in *err, stops issuing copies, waits (bounded) for the copies it already
// issued and returns.
#include <stdlib.h>

#include <algorithm>

#include "qms_async.cuh"
#include "qms_moe.cuh"
#include "qms_router.cuh"

namespace qms {

constexpr int kChunkWarps = 2;                     // consumer warps per chunk (8 rows / kChunkWarps each)
constexpr int kConsumerWarps = 8 * kChunkWarps;    // a stage is 8 chunks
constexpr int kStreamThreads = (kConsumerWarps + 2) * 32;   // + producer warp + epilogue warp
constexpr int kMaxSegments = 4;                    // CTAs a tile may be split across
constexpr int kMaxGrid = 256;                      // CTAs (SMs) the combine tables cover
constexpr int kLogitCopies = 16;                   // copies of the logit words (readers spread over lines)
constexpr uint32_t kSpinLimit = 1u << 22;           // polls before a wait gives up (>= 0.1 s with backoff)
constexpr uint32_t kPollBackoffNs = 100;
constexpr size_t kSmemOptIn = 232448;              // 227 KB: per-block dynamic shared memory on sm_100
// Ring slots (stages in flight per SM). 148 SMs x 6 x 18 KB = 16 MB in flight already covers
// HBM's bandwidth-latency product; deeper rings only lengthen the queue a late-starting SM waits
// behind. The environment variable QMS_STREAM_RING (2..32) overrides it for tuning.
#ifndef QMS_STREAM_MAX_RING
#define QMS_STREAM_MAX_RING 6
#endif

enum { ERR_CONSUMER = 1, ERR_PRODUCER = 2, ERR_GRID = 4, ERR_ROUTER = 16, ERR_DRAIN = 32 };

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

// Static split of U units over G CTAs: CTA c owns [lo(c), lo(c+1)). 32-bit arithmetic (a 64-bit
// division is a long instruction sequence on the GPU): the host checks U * G < 2^31.
__host__ __device__ inline int part_lo(int c, int U, int G) { return c * U / G; }
__host__ __device__ inline int part_owner(int u, int U, int G) { return ((u + 1) * G - 1) / U; }

constexpr int kMaxTiles = 8;                       // tiles one CTA touches (checked on the host)

// The tiles CTA range [u0, u1) of the unit sequence touches (UT units per tile), in processing
// order: the tile it shares with the next CTA first (the next CTA needs its hand-over), then whole
// tiles, then the tile it shares with the previous CTA (it takes that CTA's hand-over); s0/s1 are
// the CTA's units [s0, s1) within each tile. Writes at most kMaxTiles entries, returns the count.
__host__ __device__ inline int make_jobs(int u0, int u1, int UT, int *tile, int *s0, int *s1) {
    if (u0 >= u1) return 0;
    const int tf = u0 / UT, tl = (u1 - 1) / UT;
    const bool split = tf != tl;
    const bool tail = split && u1 < (tl + 1) * UT, head = split && u0 > tf * UT;
    int n = 0;
    for (int k = 0; k < tl - tf + 1; k++) {
        int t = tf + k;
        if (tail) t = k == 0 ? tl : tf + k - 1 + (head ? 1 : 0);
        else if (head) t = tf + k + 1;
        if (head && k == tl - tf) t = tf;
        if (n < kMaxTiles) {
            tile[n] = t;
            s0[n] = u0 > t * UT ? u0 - t * UT : 0;
            s1[n] = u1 < (t + 1) * UT ? u1 - t * UT : UT;
        }
        n++;
    }
    return n;
}

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

// ---- gate/up + SwiGLU + Q8, down, combine in one stream (batch 1) ------------------------------
struct DecodeArgs {
    const float *router_lm;               // [X][16][E/16]: element 16*i + k of a row at [k][i]
    const float *xn, *resid;
    const float *nw;                      // optional: xn = RMSNorm(xn) * nw first (ffn_norm, src/model.c:1283)
    float eps;
    float *out;
    const uint8_t *gu, *dn;               // staged experts: gate/up chunks, down column stages
    size_t gu_expert, dn_expert;
    int nbE, F, E, K, X, nst, RD;
    uint32_t slot;                        // ring slot bytes
    unsigned long long *lgf;              // [kLogitCopies][X] flagged logits
    unsigned long long *aq;               // [tiles][10] flagged Q8 groups: q (8 words), d, sum
    unsigned long long *part_gu;          // [tiles][kMaxSegments][64] flagged partial gate/up sums
    unsigned long long *fin;              // [G][E] flagged partial outputs, one vector per CTA
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

// Epilogue warp, tile whose gate/up this CTA finishes after `nprev` earlier CTAs: adds their
// flagged partial sums (slots 0 .. nprev-1, 2 per lane) in CTA order before its own, so the result
// does not depend on timing. The earlier CTAs published them as the first work of their call.
__device__ __forceinline__ bool add_partials(const unsigned long long *part, int tile, int nprev, uint32_t stamp,
                                             float (&v)[2], volatile int *abort, int *err) {
    const int lane = threadIdx.x & 31;
    const unsigned long long *pt = part + (size_t)tile * kMaxSegments * 64;
    float a0 = 0.0f, a1 = 0.0f;
    bool ok = true;
    for (int q = 0; q < nprev; q++) {
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

template <int SBG, int DQ1>
__global__ void __launch_bounds__(kStreamThreads, 1) k_decode_bs1(const DecodeArgs a) {
    // SBG: blocks per gate/up chunk row; DQ1: down weights are Q4_1 (stages carry a min plane)
    constexpr uint32_t GBG = 8 * SBG * 18, STG = 8 * GBG;
    constexpr int PG = SBG / 4 / kChunkWarps, RSG = 32 / SBG;
    extern __shared__ __align__(128) uint8_t smem[];
    const int nst = a.nst, K = a.K, F = a.F, E = a.E, X = a.X, nbE = a.nbE, RD = a.RD;
    const uint32_t SLOT = a.slot, STD = (uint32_t)RD * (DQ1 ? 20 : 18);
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nst * SLOT);
    uint64_t *empty = full + nst;
    uint64_t *sfull = empty + nst;                                  // [kSumBufs] sums written
    uint64_t *sempty = sfull + kSumBufs;                            // [kSumBufs] sums consumed
    uint64_t *rbar = sempty + kSumBufs;                             // router row landed
    uint64_t *selbar = rbar + 1;                                    // experts chosen
    uint64_t *specbar = selbar + 1;                                 // float ranking done (t_cand)
    uint64_t *ringbar = specbar + 1;                                // the ring holds the chosen experts
    uint64_t *qbar = ringbar + 1;                                   // [kMaxTiles] tile's Q8 group ready
    float *sacc = reinterpret_cast<float *>(qbar + kMaxTiles);     // [E] this CTA's partial output
    int8_t *sxq = reinterpret_cast<int8_t *>(sacc + E);             // [nbE*32] the token's Q8 row
    float *sxd = reinterpret_cast<float *>(sxq + nbE * 32);         // [nbE]
    int *sxs = reinterpret_cast<int *>(sxd + nbE);                  // [nbE], 8 * sum
    int8_t *sq8 = reinterpret_cast<int8_t *>(sxs + nbE);            // [kMaxTiles][32] tiles' Q8 groups
    float *sq8d = reinterpret_cast<float *>(sq8 + kMaxTiles * 32);  // [kMaxTiles]
    int *sq8s = reinterpret_cast<int *>(sq8d + kMaxTiles);          // [kMaxTiles] sum (Q4_1) or 8 x sum
    float *sbuf = reinterpret_cast<float *>(sq8s + kMaxTiles);      // [kSumBufs][64] tile sums
    float *slg = sbuf + kSumBufs * 64;                              // [kLogitPad] this call's logits
    // routing scratch inside the ring, which carries no stage before the experts are known
    const int L = E / 16, PS = L + 4;
    float *srow = reinterpret_cast<float *>(ring);                  // [16][PS] router row, lane-major
    float *sx = srow + 16 * PS;                                     // [16][PS] xn, lane-major
    __shared__ int s_abort;
    __shared__ double s_nrm[kConsumerWarps];
    __shared__ const uint8_t *s_gu_base[8], *s_dn_base[8];   // producer: streamed experts' weights
    __shared__ int s_spec[8];                                  // producer: the experts being streamed
    __shared__ int s_sel[64];
    __shared__ float s_w[64];                                  // routing weights
    __shared__ uint32_t s_stamp;
    __shared__ int t_cand[65];                                 // routing: float rank -> logit
    __shared__ double t_ex[256], t_pj[64], s_z;
    __shared__ int s_jn, s_jt[kMaxTiles], s_j0[kMaxTiles], s_j1[kMaxTiles];   // this CTA's tiles
    __shared__ int s_rb[kMaxGrid + 1];                         // combine: CTA r reduces rows [s_rb[r], s_rb[r+1])

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x, c = blockIdx.x;
    const int Sg = nbE / SBG, tps = F / 32, Rq = E / RD, UT = Sg + Rq, U = K * tps * UT;
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
        mbar_init(specbar, 1);
        mbar_init(ringbar, 1);
        for (int i = 0; i <= K; i++) t_cand[i] = 0;
        for (int i = 0; i < kMaxTiles; i++) mbar_init(&qbar[i], 1);
        fence_mbar_init();
        s_jn = make_jobs(part_lo(c, U, G), part_lo(c + 1, U, G), UT, s_jt, s_j0, s_j1);
        if (c < X) {                                // router row c, lane-major, before the wait
            mbar_arrive_expect_tx(rbar, (uint32_t)E * 4);
            const uint64_t pol = evict_first_policy();
            for (int k = 0; k < 16; k++)
                bulk_load(srow + k * PS, a.router_lm + (size_t)c * E + (size_t)k * L, (uint32_t)L * 4, rbar, pol);
        }
    }
    for (int i = threadIdx.x; i <= G; i += blockDim.x) s_rb[i] = part_lo(i, E, G);
    __syncthreads();
    pdl_trigger();                                  // the next call's kernel may stage its router row
    pdl_wait();                                     // xn comes from the previous kernel
    volatile int *abort_flag = &s_abort;
    const int nj = s_jn;

    if (warp == kConsumerWarps) {                   // ---- producer: one stream of stages
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            // The stream starts on the float ranking's top K (t_cand) while warp 0 still proves it
            // against the double probabilities; the selection is checked before the ring is handed
            // to the consumers (ringbar). If they differ (ties of the exact ranking, NaN logits),
            // the copies issued so far land, the ring is reset and the stream restarts.
            bool ok = wait_bounded(specbar, 0, abort_flag, a.err, ERR_PRODUCER) && !*abort_flag;
            bool valid = false;                     // the experts in use are the selection
            for (int pass = 0; pass < 2 && ok; pass++) {
                // expert bases live in shared memory: a local array would sit in local memory,
                // and every load from it that misses L1 queues behind the stream in L2
                for (int j = 0; j < K; j++) {
                    int e = valid ? s_sel[j] : t_cand[j];
                    if ((unsigned)e >= (unsigned)X) e = 0;   // speculative only: the check rejects it
                    s_spec[j] = e;
                    s_gu_base[j] = a.gu + (size_t)e * a.gu_expert;
                    s_dn_base[j] = a.dn + (size_t)e * a.dn_expert;
                }
                bool restart = false;
                auto check = [&]() {                // the proof is done: same experts?
                    ok = wait_bounded(selbar, 0, abort_flag, a.err, ERR_PRODUCER) && !*abort_flag;
                    if (!ok) return;
                    bool same = true;
                    for (int j = 0; j < K; j++) same = same && s_sel[j] == s_spec[j];
                    if (same) {
                        valid = true;
                        mbar_arrive(ringbar);
                    } else {
                        restart = true;
                    }
                };
                Ring r(nst);
                int issued = 0;
                // step k: gate/up stages of tile k, then down stages of tile k - 1
                for (int k = 0; k <= nj && ok && !restart; k++) {
                    for (int h = 0; h < 2 && ok && !restart; h++) {
                        const int kk = k - h;
                        if (h == 0 ? k == nj : k == 0) continue;
                        const int t = s_jt[kk], s0 = s_j0[kk], s1 = s_j1[kk];
                        int lo, hi;
                        const uint8_t *src;
                        uint32_t bytes;
                        if (h == 0) {
                            lo = s0;
                            hi = s1 < Sg ? s1 : Sg;
                            src = s_gu_base[t / tps] + (size_t)(t % tps) * tile_bytes;
                            bytes = STG;
                        } else {
                            lo = (s0 > Sg ? s0 : Sg) - Sg;
                            hi = s1 - Sg;
                            src = s_dn_base[t / tps] + (size_t)(t % tps) * Rq * STD;
                            bytes = STD;
                        }
                        for (int q = lo; q < hi && ok; q++) {
                            if (issued >= nst) {
                                if (!valid && (check(), restart || !ok)) break;
                                if (!(ok = wait_bounded(&empty[r.slot], r.phase ^ 1, abort_flag, a.err, ERR_PRODUCER)))
                                    break;
                            }
                            mbar_arrive_expect_tx(&full[r.slot], bytes);
                            bulk_load(ring + (size_t)r.slot * SLOT, src + (size_t)q * bytes, bytes, &full[r.slot], pol);
                            issued++;
                            r.next();
                        }
                    }
                }
                if (ok && !valid && !restart) check();
                if (!ok || *abort_flag) {
                    drain_issued(full, nst, issued, a.err);
                    break;
                }
                if (!restart) break;
                // wrong experts: let the speculative copies land, reset the ring, start over
                drain_issued(full, nst, issued, a.err);
                for (int i = 0; i < nst; i++) {
                    mbar_init(&full[i], 1);
                    mbar_init(&empty[i], kConsumerWarps);
                }
                fence_mbar_init();
                valid = true;
                mbar_arrive(ringbar);
            }
        }
        return;
    }

    if (warp == kConsumerWarps + 1) {               // ---- epilogue warp: merges, SwiGLU, Q8 groups
        // first the routing weights (the down work needs them, gate/up does not)
        bool ok = __all_sync(0xffffffffu, wait_bounded(selbar, 0, abort_flag, a.err, ERR_CONSUMER)) && !*abort_flag;
        if (ok) route_weights(slg, X, K, s_sel, t_pj, s_z, s_w, c == 0 ? a.sel : nullptr, c == 0 ? a.wts : nullptr);
        Ring sr(kSumBufs);
        const uint32_t stamp = s_stamp;
        for (int k = 0; k < nj; k++) {
            const int t = s_jt[k], s0 = s_j0[k], s1 = s_j1[k];
            unsigned long long *gq = a.aq + (size_t)t * kAqWords;
            if (s0 < Sg) {                          // gate/up sums of this CTA's part of the tile
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&sfull[sr.slot], sr.phase, abort_flag, a.err,
                                                                  ERR_CONSUMER));
                float v[2] = {sbuf[sr.slot * 64 + lane], sbuf[sr.slot * 64 + 32 + lane]};
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[sr.slot]);
                sr.next();
                if (!ok) continue;
                const int first = part_owner(t * UT, U, G);
                if (s1 < Sg) {                      // a later CTA finishes this tile's gate/up
                    unsigned long long *pt = a.part_gu + ((size_t)t * kMaxSegments + (c - first)) * 64;
                    st_flagged(pt + lane, __float_as_uint(v[0]), stamp);
                    st_flagged(pt + 32 + lane, __float_as_uint(v[1]), stamp);
                    continue;
                }
                if (c > first) ok = add_partials(a.part_gu, t, c - first, stamp, v, abort_flag, a.err);
                if (!ok) continue;
                // rows 0-31: gate f0+lane, rows 32-63: up f0+lane -> a = silu(g) * u, its Q8 group
                const float av = __fmul_rn(__fdiv_rn(v[0], __fadd_rn(1.0f, expf(-v[0]))), v[1]);
                const Q8Lane q8 = quantize_lane(av);
                sq8[k * 32 + lane] = (int8_t)q8.q;
                if (lane == 0) {
                    sq8d[k] = q8.d;
                    sq8s[k] = DQ1 ? q8.sum : 8 * q8.sum;
                }
                if (s1 < UT) {                      // a later CTA does part of the tile's down work
                    uint32_t b4 = (uint32_t)(q8.q & 0xff) << (8 * (lane & 3));
                    b4 |= __shfl_xor_sync(0xffffffffu, b4, 1);
                    b4 |= __shfl_xor_sync(0xffffffffu, b4, 2);
                    if ((lane & 3) == 0) st_flagged(gq + (lane >> 2), b4, stamp);
                    if (lane == 1) st_flagged(gq + 8, __float_as_uint(q8.d), stamp);
                    if (lane == 2) st_flagged(gq + 9, (uint32_t)q8.sum, stamp);
                }
            } else {                                // down work only: the Q8 group of an earlier CTA
                if (!ok) continue;
                unsigned long long w = lane < kAqWords ? ld_flagged(gq + lane) : 0ull;
                ok = __all_sync(0xffffffffu, lane >= kAqWords || wait_flagged(gq + lane, stamp, w, abort_flag, a.err,
                                                                              ERR_GRID));
                if (!ok) continue;
                const uint32_t d = (uint32_t)w;
                if (lane < 8) reinterpret_cast<uint32_t *>(sq8 + k * 32)[lane] = d;
                else if (lane == 8) sq8d[k] = __uint_as_float(d);
                else if (lane == 9) sq8s[k] = DQ1 ? (int)d : 8 * (int)d;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&qbar[k]);
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
    // every CTA reads all of xn: start each CTA at a different 128-byte line so the 148 readers
    // of each line do not arrive at once
    const int n4 = E / 4, rot = (c * 8) % n4;
    for (int q0 = tid; q0 < n4; q0 += kConsumerWarps * 32) {
        const int q = q0 + rot < n4 ? q0 + rot : q0 + rot - n4;
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.xn) + q);
        const int j = 4 * q;
        sx[((j + 0) & 15) * PS + ((j + 0) >> 4)] = v.x;
        sx[((j + 1) & 15) * PS + ((j + 1) >> 4)] = v.y;
        sx[((j + 2) & 15) * PS + ((j + 2) >> 4)] = v.z;
        sx[((j + 3) & 15) * PS + ((j + 3) >> 4)] = v.w;
        reinterpret_cast<float4 *>(sacc)[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    consumer_sync();
    if (a.nw) {
        // the block's input is RMSNorm(h) * ffn_norm: the sum of squares in one fixed order, the
        // same in every CTA (each CTA routes and quantises its own copy, so all copies must agree)
        const int per = E / (kConsumerWarps * 32);          // E % 512 == 0 when nw is passed
        double s2 = 0.0;
        for (int k = 0; k < per; k++) {
            const int j = tid * per + k;
            const double v = (double)sx[(j & 15) * PS + (j >> 4)];
            s2 = fma(v, v, s2);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if ((tid & 31) == 0) s_nrm[tid >> 5] = s2;
        consumer_sync();
        double tot = 0.0;
        for (int i = 0; i < kConsumerWarps; i++) tot += s_nrm[i];
        const double inv = 1.0 / sqrt(tot / E + (double)a.eps);
        for (int k = 0; k < per; k++) {
            const int j = tid * per + k;
            float *px = sx + (j & 15) * PS + (j >> 4);
            *px = __fmul_rn((float)((double)*px * inv), __ldg(a.nw + j));
        }
        consumer_sync();
    }
    const uint32_t stamp = s_stamp;
    bool ok = true;
    if (warp == 0) {
        if (c < X) {                                // logit c in qms_vec_dot_f32's exact order
            ok = __all_sync(0xffffffffu, wait_bounded(rbar, 0, abort_flag, a.err, ERR_ROUTER));
            const int k = lane & 15;
            const float *w = srow + k * PS, *x = sx + k * PS;
            // the chain is 256 dependent FMAs (E = 4096): operands of the next 8 elements are
            // loaded while the current 8 multiply, so no shared-memory latency sits in the chain
            float acc = 0.0f;
            const int nch = L / 8;                  // L % 16 == 0 (E % 256 == 0): nch is even
            float4 wa[2], xa[2], wb[2], xb[2];
#pragma unroll
            for (int q = 0; q < 2; q++) {
                wa[q] = *reinterpret_cast<const float4 *>(w + 4 * q);
                xa[q] = *reinterpret_cast<const float4 *>(x + 4 * q);
            }
            for (int ch = 0; ch < nch; ch += 2) {
                const int ib = (ch + 1) * 8;
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    wb[q] = *reinterpret_cast<const float4 *>(w + ib + 4 * q);
                    xb[q] = *reinterpret_cast<const float4 *>(x + ib + 4 * q);
                }
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    acc = __fmaf_rn(wa[q].x, xa[q].x, acc);
                    acc = __fmaf_rn(wa[q].y, xa[q].y, acc);
                    acc = __fmaf_rn(wa[q].z, xa[q].z, acc);
                    acc = __fmaf_rn(wa[q].w, xa[q].w, acc);
                }
                if (ch + 2 < nch) {
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        wa[q] = *reinterpret_cast<const float4 *>(w + ib + 8 + 4 * q);
                        xa[q] = *reinterpret_cast<const float4 *>(x + ib + 8 + 4 * q);
                    }
                }
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    acc = __fmaf_rn(wb[q].x, xb[q].x, acc);
                    acc = __fmaf_rn(wb[q].y, xb[q].y, acc);
                    acc = __fmaf_rn(wb[q].z, xb[q].z, acc);
                    acc = __fmaf_rn(wb[q].w, xb[q].w, acc);
                }
            }
            acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2, 16));
            acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1, 16));
            acc = __shfl_sync(0xffffffffu, acc, 0);
            if (lane < kLogitCopies && ok) st_flagged(a.lgf + lane * X + c, __float_as_uint(acc), stamp);
            if (lane == 0 && ok && a.logits) a.logits[c] = acc;
        }
    } else {                                        // the token's Q8 row (src/kernels.c:34-53)
        // four threads per 32-block, eight values each: a warp-wide reduction per block would make
        // each warp run ~9 blocks of dependent shuffles back to back
        for (int v = tid - 32; v < nbE * 4; v += (kConsumerWarps - 1) * 32) {   // warp-uniform: nbE % 8 == 0
            const int b = v >> 2, p = v & 3;
            const float *xs = sx + 8 * (p & 1) * PS + 2 * b + (p >> 1);   // element 32b + 8p + m at xs[m * PS]
            float x[8], amax = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; m++) {
                x[m] = xs[m * PS];
                amax = fmaxf(amax, fabsf(x[m]));
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            uint32_t w0 = 0, w1 = 0;
            int sum = 0;
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int q = __float2int_rn(__fmul_rn(x[m], id));
                sum += q;
                if (m < 4) w0 |= (uint32_t)(q & 0xff) << (8 * m);
                else w1 |= (uint32_t)(q & 0xff) << (8 * (m - 4));
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            *reinterpret_cast<uint2 *>(sxq + 32 * b + 8 * p) = make_uint2(w0, w1);
            if (p == 0) {
                sxd[b] = d;
                sxs[b] = 8 * sum;
            }
        }
    }
    if (tid < X) {                                  // every CTA's logit, from this CTA's copy
        const unsigned long long *lw = a.lgf + (c % kLogitCopies) * X + tid;
        unsigned long long v = ld_flagged(lw);
        if (wait_flagged(lw, stamp, v, abort_flag, a.err, ERR_ROUTER)) slg[tid] = __uint_as_float((uint32_t)v);
    } else if (tid < kLogitPad) {
        slg[tid] = -INFINITY;                       // padding the rank loop may read
    }
    consumer_sync();
    rank_candidates(slg, X, K, tid, t_cand);
    consumer_sync();
    if (tid == 0) mbar_arrive(specbar);             // the producer may start on the float ranking
    if (warp == 0) {
        double z = 0.0;
        if (!*abort_flag) route_select(slg, X, K, t_cand, s_sel, t_ex, t_pj, z);
        if (lane == 0) s_z = z;
        __syncwarp();
        if (lane == 0) mbar_arrive(selbar);         // producer and epilogue may start (they check the abort flag)
    }
    ok = !*abort_flag;

    // ---- consumers: the stream, in the producer's order, once it carries the selected experts
    if (ok) ok = __all_sync(0xffffffffu, wait_bounded(ringbar, 0, abort_flag, a.err, ERR_CONSUMER));
    const int g = warp / kChunkWarps, half = warp % kChunkWarps;   // chunk of a gate/up stage, row part
    Ring r(nst), sr(kSumBufs);
    int handed = 0;
    // the partial output row q*RD + i belongs to thread i % 512 throughout: that thread updates it
    // and publishes it (fin[c][row]) once the CTA's last down stage touching it is done
    unsigned long long *fin_c = a.fin + (size_t)c * E;
    bool published = false;
    auto publish_rows = [&](int qa, int qb) {
        for (int q = qa; q < qb; q++)
            for (int i = tid; i < RD; i += kConsumerWarps * 32)
                st_flagged(fin_c + q * RD + i, __float_as_uint(sacc[q * RD + i]), stamp);
    };
    const int bl = lane % SBG, rs = lane / SBG;
    for (int k = 0; k <= nj; k++) {
        if (k < nj) {                               // gate/up stages of tile k
            const int s0 = s_j0[k], s1 = s_j1[k] < Sg ? s_j1[k] : Sg;
            if (s0 < s1) {
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
                // hand the tile's 64 sums (8 per chunk) to the epilogue warp
                if (handed >= kSumBufs && ok)
                    ok = __all_sync(0xffffffffu, wait_bounded(&sempty[sr.slot], sr.phase ^ 1, abort_flag, a.err,
                                                              ERR_CONSUMER));
                if (bl == 0)
                    for (int p = 0; p < PG; p++) sbuf[sr.slot * 64 + g * 8 + rs + (half * PG + p) * RSG] = acc[p];
                __syncwarp();
                if (lane == 0) mbar_arrive(&sfull[sr.slot]);
                sr.next();
                handed++;
            }
        }
        if (k > 0) {                                // down stages of tile k - 1
            const int kk = k - 1, t = s_jt[kk];
            const int q0 = (s_j0[kk] > Sg ? s_j0[kk] : Sg) - Sg, q1 = s_j1[kk] - Sg;
            // the last tile's down stages come last in the stream: rows outside them are final
            // now, and each of its stages finishes its rows (a row is only ever updated by the
            // thread that publishes it, so no barrier is needed)
            const bool last = kk == nj - 1;
            if (last && ok) publish_rows(0, q0 > 0 ? q0 : 0);
            if (q0 < q1) {
                if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&qbar[kk], 0, abort_flag, a.err, ERR_CONSUMER));
                int4 xa0 = make_int4(0, 0, 0, 0), xa1 = xa0;
                float xd = 0.0f, wj = 0.0f;
                int xs = 0;
                if (ok) {
                    xa0 = *reinterpret_cast<const int4 *>(sq8 + kk * 32);
                    xa1 = *reinterpret_cast<const int4 *>(sq8 + kk * 32 + 16);
                    xd = sq8d[kk];
                    xs = sq8s[kk];
                    wj = s_w[t / tps];
                }
                for (int q = q0; q < q1; q++, r.next()) {
                    if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&full[r.slot], r.phase, abort_flag, a.err, ERR_CONSUMER));
                    if (!ok) continue;
                    const uint8_t *st = ring + (size_t)r.slot * SLOT;
                    float *pa = sacc + q * RD;
#pragma unroll 2
                    for (int i = tid; i < RD; i += kConsumerWarps * 32) {
                        const uint4 nib = *reinterpret_cast<const uint4 *>(st + i * 16);
                        const float dw = h2f(*reinterpret_cast<const uint16_t *>(st + RD * 16 + i * 2));
                        const int isum = q4_block_isum(nib, xa0, xa1);
                        float term;
                        if (DQ1) {                  // d q + m: d dx isum + m ds (src/kernels.c:109-121)
                            const float mw = h2f(*reinterpret_cast<const uint16_t *>(st + RD * 18 + i * 2));
                            term = fmaf((float)isum, dw * xd, mw * (xd * (float)xs));
                        } else {                    // d (q - 8): the -8 folded into the block sum
                            term = (float)(isum - xs) * (dw * xd);
                        }
                        const float o = fmaf(wj, term, pa[i]);
                        pa[i] = o;
                        if (last) st_flagged(fin_c + q * RD + i, __float_as_uint(o), stamp);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[r.slot]);
                }
            }
            if (last && ok) {
                publish_rows(q1 > q0 ? q1 : q0, Rq);
                published = true;
            }
        }
    }
    if (!published && ok) publish_rows(0, Rq);      // no down work came last (or none at all)

    // ---- combine: CTA c sums rows R0 .. R0+nr-1 over every CTA's partial vector, in CTA order
    consumer_sync();                                // the ring is idle: it receives the partials
    const int R0 = s_rb[c], nr = s_rb[c + 1] - R0;
    float *red = reinterpret_cast<float *>(ring);   // [G][nr]
    if (!*abort_flag) {
        // warp w polls CTAs w, w + 16, ... (lane = row), all words in flight, stale ones re-polled
        constexpr int kSrc = (kMaxGrid + kConsumerWarps - 1) / kConsumerWarps;
        for (int i0 = 0; i0 < nr; i0 += 32) {
            const int i = i0 + lane;
            unsigned long long v[kSrc];
#pragma unroll
            for (int j = 0; j < kSrc; j++) {
                const int q = warp + j * kConsumerWarps;
                v[j] = q < G && i < nr ? ld_flagged(a.fin + (size_t)q * E + R0 + i) : 0ull;
            }
            uint32_t n = 0;
            bool done = false;
            while (!done) {
                uint32_t pending = 0;
#pragma unroll
                for (int j = 0; j < kSrc; j++) {
                    const int q = warp + j * kConsumerWarps;
                    if (q < G && i < nr && (uint32_t)(v[j] >> 32) != stamp) pending |= 1u << j;
                }
                if (!pending) {
                    done = true;
                    break;
                }
                if (*abort_flag) break;
                if (++n == kSpinLimit) {
                    *abort_flag = 1;
                    atomicOr(a.err, ERR_GRID);
                    break;
                }
                __nanosleep(64);
#pragma unroll
                for (int j = 0; j < kSrc; j++)
                    if (pending & (1u << j)) v[j] = ld_flagged(a.fin + (size_t)(warp + j * kConsumerWarps) * E + R0 + i);
            }
            if (!done) break;
#pragma unroll
            for (int j = 0; j < kSrc; j++) {
                const int q = warp + j * kConsumerWarps;
                if (q < G && i < nr) red[q * nr + i] = __uint_as_float((uint32_t)v[j]);
            }
        }
    }
    consumer_sync();
    if (*abort_flag) return;
    // 16 threads per row, each sums every 16th CTA in order, then a fixed tree
    for (int i0 = 0; i0 < nr; i0 += kConsumerWarps * 2) {
        const int i = i0 + (tid >> 4), p = tid & 15;
        float sum = 0.0f;
        if (i < nr)
            for (int q = p; q < G; q += 16) sum += red[q * nr + i];
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (p == 0 && i < nr) {
            float o = sum;
            if (a.resid) o = __fadd_rn(a.resid[R0 + i], o);
            a.out[R0 + i] = o;
        }
    }
}

// ---- host side -----------------------------------------------------------------------------------
static uint32_t dec_slot(const QmsCudaMoe *m) {
    const uint32_t stg = 8 * m->cgu.GB, std_ = m->dcol.STD;
    return stg > std_ ? stg : std_;
}
static size_t dec_fixed(const QmsCudaMoe *m) {
    return (2 * kSumBufs + 4 + kMaxTiles) * 8 + (size_t)m->E * 4 + (size_t)m->nbE * 40 + kMaxTiles * 40 +
           kSumBufs * 64 * 4 + (size_t)kLogitPad * 4;
}
static size_t dec_smem(const QmsCudaMoe *m) { return (size_t)m->nst * (dec_slot(m) + 16) + dec_fixed(m); }

typedef void (*DecodeKernel)(const DecodeArgs);
static DecodeKernel dec_kernel(const QmsCudaMoe *m) {
    if (m->dcol.q1) return m->cgu.SB == 16 ? k_decode_bs1<16, 1> : k_decode_bs1<8, 1>;
    return m->cgu.SB == 16 ? k_decode_bs1<16, 0> : k_decode_bs1<8, 0>;
}

// Largest number of tiles one CTA touches, and of CTAs one tile's gate/up part spans.
static void job_bounds(const QmsCudaMoe *m, int *max_tiles, int *max_segs) {
    const int G = m->nsm, Sg = m->cgu.S, UT = Sg + m->dcol.Rq, ntg = m->K * (m->F / 32), U = ntg * UT;
    int jt[kMaxTiles], j0[kMaxTiles], j1[kMaxTiles];
    *max_tiles = 0;
    for (int c = 0; c < G; c++) *max_tiles = std::max(*max_tiles, make_jobs(part_lo(c, U, G), part_lo(c + 1, U, G), UT, jt, j0, j1));
    *max_segs = 1;
    for (int t = 0; t < ntg; t++)
        *max_segs = std::max(*max_segs, part_owner(t * UT + Sg - 1, U, G) - part_owner(t * UT, U, G) + 1);
}

int stream_prepare(QmsCudaMoe *m) {
    m->stream_ok = 0;
    if (m->K > 8 || m->X > 256 || 2 * m->X > m->E || m->nsm > kMaxGrid) return QMS_CUDA_OK;
    const int64_t units = (int64_t)m->K * (m->F / 32) * (m->cgu.S + m->dcol.Rq);
    if ((units + 1) * m->nsm >= (1ll << 31) || (int64_t)(m->E + 1) * m->nsm >= (1ll << 31)) return QMS_CUDA_OK;
    if (m->nbE % m->cgu.SB) return QMS_CUDA_OK;
    const uint32_t slot = dec_slot(m);
    cudaFuncAttributes fa;
    QMS_CK(cudaFuncGetAttributes(&fa, dec_kernel(m)));
    const size_t avail = kSmemOptIn - fa.sharedSizeBytes - dec_fixed(m);
    int want = QMS_STREAM_MAX_RING;
    if (const char *env = getenv("QMS_STREAM_RING")) {
        const int v = atoi(env);
        if (v >= 2 && v <= 32) want = v;
    }
    m->nst = (int)std::min<size_t>((size_t)want, avail / (slot + 16));
    if (m->nst < 2) return QMS_CUDA_OK;
    const size_t ring = (size_t)m->nst * slot;
    if ((size_t)2 * 16 * (m->E / 16 + 4) * 4 > ring) return QMS_CUDA_OK;             // routing scratch
    if ((size_t)m->nsm * ((m->E + m->nsm - 1) / m->nsm) * 4 > ring) return QMS_CUDA_OK;   // combine scratch
    int max_tiles, max_segs;
    job_bounds(m, &max_tiles, &max_segs);
    if (max_tiles > kMaxTiles || max_segs > kMaxSegments) return QMS_CUDA_OK;
    const DecodeKernel dk = dec_kernel(m);
    QMS_CK(cudaFuncSetAttribute(dk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec_smem(m)));
    QMS_CK(cudaFuncSetAttribute(dk, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    // CTAs of this kernel wait for one another, so the whole grid (one CTA per SM) must be
    // resident at once: if an SM cannot hold a CTA, batch-1 calls take the per-slot kernels
    // instead (they never wait across CTAs). QMS_PERSISTENT=0 forces that choice.
    int per_sm = 0;
    QMS_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dk, kStreamThreads, dec_smem(m)));
    if (!persistent_grid_fits(per_sm, m->nsm, m->nsm)) return QMS_CUDA_OK;
    if (const char *env = getenv("QMS_PERSISTENT"))
        if (atoi(env) == 0) return QMS_CUDA_OK;
    m->stream_ok = 1;
    return QMS_CUDA_OK;
}

int stream_scratch_sizes(const QmsCudaMoe *m, StreamScratch *sz) {
    const int tiles = m->K * (m->F / 32);
    sz->lg_flagged = (size_t)kLogitCopies * m->X * 8;
    sz->stamps = (size_t)m->nsm * 4;
    sz->aq_flagged = (size_t)tiles * kAqWords * 8;
    sz->part_gu = (size_t)tiles * kMaxSegments * 64 * 8;
    sz->fin = (size_t)m->nsm * m->E * 8;
    return QMS_CUDA_OK;
}

int stream_forward_bs1(QmsCudaMoe *m, const float *xn, float *out, const float *resid, cudaStream_t s,
                       const float *nw, float eps) {
    DecodeArgs a;
    a.router_lm = m->router_lm;
    a.xn = xn;
    a.nw = nw;
    a.eps = eps;
    a.resid = resid;
    a.out = out;
    a.gu = m->gu;
    a.dn = m->dn;
    a.gu_expert = m->gu_expert;
    a.dn_expert = m->dn_expert;
    a.nbE = m->nbE;
    a.F = m->F;
    a.E = m->E;
    a.K = m->K;
    a.X = m->X;
    a.nst = m->nst;
    a.RD = m->dcol.RD;
    a.slot = dec_slot(m);
    a.lgf = m->lg_flagged;
    a.aq = m->aq_flagged;
    a.part_gu = m->part_gu;
    a.fin = m->fin;
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
