// qms_moe_gemv.cu - the MoE block for batched decode: expert-grouped GEMV on the CUDA cores.
//
// At batched-decode sizes the T*K slots spread over the X experts a few at a time, so a call is
// one read of every selected expert's weights; on N = 1..16 columns the tensor cores would idle
// while the per-block scale work dominates. Here each expert's weights stream from HBM once per
// call and serve all of its slots. After the slots are grouped by expert (k_mma_group, tiles of
// up to 16 slots of one expert, the reference's grouping of src/model.c:1066-1088):
//   k_gv_gate_up  persistent, one CTA per SM, owning a contiguous, cost-balanced range of
//                 (tile, 32-f) items. A producer warp streams each item's gate/up stages (one
//                 bulk copy each, the staged chunk layout) through a ring in shared memory; 16
//                 consumer warps hold the tile's Q8 activation rows in shared memory and form
//                 every (row, slot) dot with dp4a, each 32-block's int32 sum scaled in fp32
//                 (src/kernels.c:82-107); then SwiGLU and the Q8 group of each slot's 32 f values
//                 (src/model.c:989-997).
//   k_gv_down     the same over (tile, column-stage rows, K half) items: whole column stages
//                 (one bulk copy each) of one half of the F/32 block columns, against the slots'
//                 Q8 activation groups; writes each slot's unweighted partial down row per half
//                 (src/model.c:999-1004); the combine adds the halves and sums the slots in
//                 selection order. Q4_0 and Q4_1 down.
// A 32-block's integer dot is exact; only the fp32 summation order differs from the reference.
#include <string.h>

#include <algorithm>

#include "qms_async.cuh"
#include "qms_moe.cuh"

namespace qms {

constexpr int kGvSlots = 16;                 // slots per tile (k_mma_group width)
constexpr int kGvConsWarps = 16;
constexpr int kGvCons = kGvConsWarps * 32;
constexpr int kGvThreads = kGvCons + 32;     // + producer warp
constexpr int kGvMaxRing = 16;
constexpr size_t kGvSmemCap = 216 * 1024;     // dynamic; + ~2.6 KB static stays under 227 KB
constexpr uint32_t kGvSpin = 1u << 22;
constexpr int kGvMagic = 0x4B400000;         // float bits of 2^23 + 2^22: int v -> float exactly for |v| < 2^22
constexpr float kGvMagicF = 12582912.0f;
constexpr int kGvMaxTiles = 640;             // tiles of a GEMV call: S / 16 + nx with S <= 24 nx, nx <= 256
constexpr int kGvItemCost0 = 3;              // cost of an item beyond its slot pairs (the weight stream), in slots
constexpr int kGvXRow = kGvSlots * 32 + 16;  // shared-memory bytes of one block's activation values (all slots + pad)
constexpr int kGvSRow = kGvSlots * 8 + 8;    // bytes of one block's {scale, second word} pairs (+ pad)
constexpr int kGvKParts = 2;                 // down items split the F/32 block columns in halves

enum { GV_ERR = 128 };

struct GvArgs {
    const uint8_t *w;          // staged experts: gate/up chunks or down column stages
    size_t w_expert;
    Chunked c;
    DnCols dc;
    int nb;                    // blocks along K: E/32 (gate/up) or F/32 (down)
    int F, E;
    MmaWork wk;                // slot groups: tiles, cnt, off, slots, ntiles
    const int8_t *xq;          // activation rows [rows][nb * 32]
    const float *xd;           // [rows][nb] block scales
    const int *xs;             // [rows][nb] block sums
    int rdiv;                  // activation row of slot s: s / rdiv
    int ring;                  // stages in the shared-memory ring
    uint32_t sst;              // bytes of one ring stage (multiple of 128)
    int8_t *aq_q;              // gate/up out: [S][F] Q8 values
    float *aq_d;               // [S][F/32]
    int *aq_s;                 // [S][F/32]
    float *dn;                 // down out: [S][E] partial rows of the first K half
    float *dn2;                //           [S][E] of the second half
    int *err;
};

// Bounded wait on an mbarrier phase; on timeout set the CTA's abort flag and the error bit.
__device__ __forceinline__ bool gv_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (++n == kGvSpin) {
            *abort = 1;
            atomicOr(err, GV_ERR);
            return false;
        }
        if (n > 64) __nanosleep(32);
    }
    return true;
}

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kGvCons) : "memory"); }

// bias + integer dot of one 32-block from pre-split nibble words (w[0..3] low nibbles = elements
// 0-15, w[4..7] high nibbles = 16-31) against the two 16-byte halves of a Q8 block; one dp4a chain.
__device__ __forceinline__ int gv_dot(const uint32_t (&w)[8], uint4 x0, uint4 x1, int bias) {
    int s = __dp4a((int)w[0], (int)x0.x, bias);
    s = __dp4a((int)w[1], (int)x0.y, s);
    s = __dp4a((int)w[2], (int)x0.z, s);
    s = __dp4a((int)w[3], (int)x0.w, s);
    s = __dp4a((int)w[4], (int)x1.x, s);
    s = __dp4a((int)w[5], (int)x1.y, s);
    s = __dp4a((int)w[6], (int)x1.z, s);
    s = __dp4a((int)w[7], (int)x1.w, s);
    return s;
}

__device__ __forceinline__ void gv_split(uint4 v, uint32_t (&w)[8]) {
    const uint32_t m = 0x0F0F0F0Fu;
    w[0] = v.x & m;
    w[1] = v.y & m;
    w[2] = v.z & m;
    w[3] = v.w & m;
    w[4] = (v.x >> 4) & m;
    w[5] = (v.y >> 4) & m;
    w[6] = (v.z >> 4) & m;
    w[7] = (v.w >> 4) & m;
}

// Two magic-encoded integer dots (kGvMagic + v) as the floats v, exactly (|v| < 2^22).
__device__ __forceinline__ float2 gv_unmagic(int a, int b) {
    return f2_add(make_float2(__int_as_float(a), __int_as_float(b)), make_float2(-kGvMagicF, -kGvMagicF));
}

struct GvTile {
    int e, off, ns;            // expert, first slot in the grouped list, slots in the tile
};

__device__ __forceinline__ GvTile gv_tile(const MmaWork &w, int tl) {
    const int t = __ldcg(w.tiles + tl);
    GvTile g;
    g.e = t & 0xFFFF;
    const int n0 = (t >> 16) * kGvSlots;
    g.off = __ldcg(w.off + g.e) + n0;
    g.ns = min(kGvSlots, __ldcg(w.cnt + g.e) - n0);
    return g;
}

// All threads: this CTA's contiguous range [lo, hi) of the ntiles * ipt items, split by cost (an
// item of a tile with n slots costs n rounded up to pairs + kGvItemCost0): the CTA owns the items whose starting cost
// falls in its share. s_pre: kGvMaxTiles + 1 ints of shared memory.
__device__ __forceinline__ void gv_split_items(const MmaWork &w, int ntiles, int ipt, int *s_pre, int *s_lh,
                                               int &lo, int &hi) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int t = tid; t < ntiles; t += nt) s_pre[t] = ((gv_tile(w, t).ns + 1) & ~1) + kGvItemCost0;
    if (tid < 2) s_lh[tid] = ntiles * ipt;
    __syncthreads();
    if (tid < 32) {                                       // exclusive prefix of the per-item costs
        const int per = (ntiles + 31) / 32, t0 = tid * per, t1 = min(ntiles, t0 + per);
        int sum = 0;
        for (int t = t0; t < t1; t++) sum += s_pre[t];
        int inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (tid >= o) inc += v;
        }
        int run = inc - sum;
        for (int t = t0; t < t1; t++) {
            const int c = s_pre[t];
            s_pre[t] = run;
            run += c;
        }
        if (tid == 31) s_pre[ntiles] = inc;
    }
    __syncthreads();
    const long long P = gridDim.x, tot = (long long)ipt * s_pre[ntiles];
    for (int t = tid; t < ntiles; t += nt) {
        const long long c0 = (long long)ipt * s_pre[t], wt = s_pre[t + 1] - s_pre[t];
        for (int k = 0; k < 2; k++) {                     // first item with start * P >= bound
            const long long bound = (long long)(blockIdx.x + k) * tot;
            const long long need = bound - c0 * P;
            const long long j = need <= 0 ? 0 : (need + wt * P - 1) / (wt * P);
            if (j < ipt) atomicMin(&s_lh[k], t * ipt + (int)j);
        }
    }
    __syncthreads();
    lo = s_lh[0];
    hi = s_lh[1];
}

// Consumers: the tile's activation rows into shared memory, block-major: block b's 16-byte halves
// of slot j at b * kGvXRow + j * 32 + h * 16, its {scale bits, second word} at b * kGvSRow + j * 8
// (the pads put consecutive blocks in different banks; a thread's slots sit at fixed offsets).
// The second word is the dp4a chain's starting value kGvMagic - 8 * sum for Q4_0 weights, or for
// Q4_1 the product d * sum as float bits. An odd slot count is padded with a zero row (its results
// are never stored), so slots go in pairs.
template <bool Q1>
__device__ __forceinline__ void gv_stage_x(const GvArgs &a, const GvTile &g, int8_t *sx, uint8_t *sxs) {
    const int nb = a.nb, K32 = nb * 32, nsp = (g.ns + 1) & ~1;
    for (int idx = threadIdx.x; idx < nsp * nb * 2; idx += kGvCons) {
        const int j = idx / (2 * nb), rem = idx - j * 2 * nb, h = rem / nb, b = rem - h * nb;
        uint4 v = make_uint4(0, 0, 0, 0);
        float d = 0.0f;
        int sm = 0;
        if (j < g.ns) {
            const int row = __ldcg(a.wk.slots + g.off + j) / a.rdiv;
            v = __ldcg(reinterpret_cast<const uint4 *>(a.xq + (size_t)row * K32 + b * 32 + h * 16));
            d = __ldcg(a.xd + (size_t)row * nb + b);
            sm = __ldcg(a.xs + (size_t)row * nb + b);
        }
        *reinterpret_cast<uint4 *>(sx + (size_t)b * kGvXRow + j * 32 + h * 16) = v;
        if (h == 0)
            *reinterpret_cast<uint2 *>(sxs + (size_t)b * kGvSRow + j * 8) =
                make_uint2(__float_as_uint(d), Q1 ? __float_as_uint(d * (float)sm) : (uint32_t)(kGvMagic - 8 * sm));
    }
}

// Producer (one thread): for each item of [lo, hi), nst ring stages; src(expert base, item's
// index within its tile, stage, ring slot, full barrier, policy) issues one stage's bulk copies.
// Waits are bounded.
template <typename Src>
__device__ __forceinline__ void gv_produce(const GvArgs &a, int lo, int hi, int ipt, int nst, uint8_t *ring,
                                           uint64_t *full, uint64_t *empty, volatile int *abort, Src src) {
    const uint64_t pol = evict_first_policy();
    int r = 0;
    uint32_t par = 0, issued = 0;
    bool ok = true;
    int cur = -1;
    const uint8_t *base = nullptr;
    for (int item = lo; item < hi && ok; item++) {
        const int tl = item / ipt, sub = item - tl * ipt;
        if (tl != cur) {
            cur = tl;
            base = a.w + (size_t)(__ldcg(a.wk.tiles + tl) & 0xFFFF) * a.w_expert;
        }
        for (int st = 0; st < nst; st++) {
            if (issued >= (uint32_t)a.ring && !(ok = gv_wait(&empty[r], par ^ 1, abort, a.err))) break;
            if (*abort) {                  // consumers stopped: they no longer free stages
                ok = false;
                break;
            }
            src(base, sub, st, ring + (size_t)r * a.sst, &full[r], pol);
            issued++;
            if (++r == a.ring) {
                r = 0;
                par ^= 1;
            }
        }
    }
    // Copies still in flight land before the CTA exits (after a normal run every one of them has
    // been consumed and these waits return at once). A consumer frees a stage only after it saw
    // the stage's copy land, so no stage ever holds two copies.
    const uint32_t n = issued < (uint32_t)a.ring ? issued : (uint32_t)a.ring;
    for (uint32_t k = issued - n; k < issued; k++) {
        uint32_t spin = 0;
        while (!mbar_try_wait(&full[k % a.ring], (k / a.ring) & 1) && ++spin < kGvSpin) __nanosleep(64);
    }
}

// Ring position and status of a consumer thread, kept across items.
struct GvRing {
    int r;
    uint32_t par;
    bool ok;
};

// Consumer side of one ring stage: wait for it (bounded); the stage's shared memory, or nullptr once
// the CTA has aborted. gv_release frees it after this thread's weights are in registers.
__device__ __forceinline__ const uint8_t *gv_acquire(const GvArgs &a, GvRing &c, const uint8_t *ring, uint64_t *full,
                                                     volatile int *abort) {
    if (c.ok) c.ok = gv_wait(&full[c.r], c.par, abort, a.err);
    return c.ok ? ring + (size_t)c.r * a.sst : nullptr;
}

__device__ __forceinline__ void gv_release(GvRing &c, uint64_t *empty, int lane, int nring) {
    __syncwarp();
    if (c.ok && lane == 0) mbar_arrive(&empty[c.r]);
    if (++c.r == nring) {
        c.r = 0;
        c.par ^= 1;
    }
}

// ---- gate/up + SwiGLU + Q8 ---------------------------------------------------------------------------
// Item (tile, ft): f values ft*32 .. +31 of the tile's expert; its nb/16 stages are the staged chunks
// (8 chunks of 8 rows x 16 blocks: chunks 0-3 gate rows, 4-7 up rows). Consumer thread t: block
// b = t % 16 of every stage and f value t / 16; its gate and up rows go as a pair.
constexpr int kGvSB = 16;
constexpr uint32_t kGvGB = 8u * kGvSB * 18;

// One item with NP slot pairs: the stage loop, then the sums over the 16 threads of each f (adjacent
// lanes) and SwiGLU (src/model.c:989-997) into sa[slot][32].
template <int NP>
__device__ __forceinline__ void gv_gu_item(const GvArgs &a, GvRing &c, uint8_t *ring, uint64_t *full, uint64_t *empty,
                                        volatile int *abort, const int8_t *sx, const uint8_t *sxs, float *sa, int nst) {
    const int tid = threadIdx.x, lane = tid & 31, b = tid % kGvSB, f = tid / kGvSB;
    const uint32_t o = (uint32_t)((f & 7) * kGvSB + b), cgo = (uint32_t)(f >> 3) * kGvGB;
    float2 acc[2 * NP];                                   // (gate, up) of slot j
#pragma unroll
    for (int j = 0; j < 2 * NP; j++) acc[j] = make_float2(0.0f, 0.0f);
    for (int st = 0; st < nst; st++) {
        const uint8_t *stg = gv_acquire(a, c, ring, full, abort);
        uint4 ng = make_uint4(0, 0, 0, 0), nu = ng;
        float2 dgu = make_float2(0.0f, 0.0f);
        if (stg) {
            const uint8_t *cg = stg + cgo, *cu = cg + 4 * kGvGB;
            ng = *reinterpret_cast<const uint4 *>(cg + o * 16);
            nu = *reinterpret_cast<const uint4 *>(cu + o * 16);
            dgu = make_float2(h2f(*reinterpret_cast<const uint16_t *>(cg + 8 * kGvSB * 16 + o * 2)),
                              h2f(*reinterpret_cast<const uint16_t *>(cu + 8 * kGvSB * 16 + o * 2)));
        }
        gv_release(c, empty, lane, a.ring);
        if (!stg) continue;
        uint32_t wg[8], wu[8];
        gv_split(ng, wg);
        gv_split(nu, wu);
        const int gb = st * kGvSB + b;
        const int8_t *xb = sx + (size_t)gb * kGvXRow;
        const uint8_t *sb = sxs + (size_t)gb * kGvSRow;
#pragma unroll
        for (int j = 0; j < 2 * NP; j++) {
            const uint4 x0 = *reinterpret_cast<const uint4 *>(xb + j * 32);
            const uint4 x1 = *reinterpret_cast<const uint4 *>(xb + j * 32 + 16);
            const uint2 xv = *reinterpret_cast<const uint2 *>(sb + j * 8);
            const float xd = __uint_as_float(xv.x);
            const int bias = (int)xv.y;                         // kGvMagic - 8 * sum: Q4_0 is d (q - 8)
            const float2 p = gv_unmagic(gv_dot(wg, x0, x1, bias), gv_dot(wu, x0, x1, bias));
            acc[j] = f2_fma(p, f2_mul(dgu, make_float2(xd, xd)), acc[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < 2 * NP; j++) {
        float gs = acc[j].x, us = acc[j].y;
#pragma unroll
        for (int m = kGvSB / 2; m > 0; m >>= 1) {
            gs += __shfl_xor_sync(0xffffffffu, gs, m);
            us += __shfl_xor_sync(0xffffffffu, us, m);
        }
        if (b == 0) {
            const float sg = __fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs)));
            sa[j * 32 + f] = __fmul_rn(sg, us);
        }
    }
}

__global__ void __launch_bounds__(kGvThreads, 1) k_gv_gate_up(const GvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort, s_lh[2], s_pre[kGvMaxTiles + 1];
    const int nb = a.nb, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t *ring = smem;
    int8_t *sx = reinterpret_cast<int8_t *>(smem + (size_t)a.ring * a.sst);
    uint8_t *sxs = reinterpret_cast<uint8_t *>(sx + (size_t)nb * kGvXRow);
    float *sact = reinterpret_cast<float *>(sxs + (size_t)nb * kGvSRow);   // [2][slot][32]
    uint64_t *full = reinterpret_cast<uint64_t *>(sact + 2 * kGvSlots * 32);
    uint64_t *empty = full + a.ring;
    if (tid == 0) {
        s_abort = 0;
        for (int r = 0; r < a.ring; r++) {
            mbar_init(&full[r], 1);
            mbar_init(&empty[r], kGvConsWarps);
        }
        fence_mbar_init();
    }
    pdl_wait();
    pdl_trigger();
    const int ipt = a.F / 32, nst = nb / kGvSB;
    int lo, hi;
    gv_split_items(a.wk, min(__ldcg(a.wk.ntiles), kGvMaxTiles), ipt, s_pre, s_lh, lo, hi);
    if (warp == kGvConsWarps) {
        if (lane == 0)
            gv_produce(a, lo, hi, ipt, nst, ring, full, empty, &s_abort,
                       [&](const uint8_t *base, int sub, int st, uint8_t *dst, uint64_t *bar, uint64_t pol) {
                           mbar_arrive_expect_tx(bar, 8 * kGvGB);
                           bulk_load(dst, base + ((size_t)(sub * nst + st) * 8) * kGvGB, 8 * kGvGB, bar, pol);
                       });
        return;
    }
    GvRing c{0, 0, true};
    int cur = -1, buf = 0;
    GvTile g{0, 0, 0};
    for (int item = lo; item < hi; item++) {
        const int tl = item / ipt, sub = item - tl * ipt;
        if (tl != cur) {
            cons_sync();                                   // every consumer is done with the old rows
            cur = tl;
            g = gv_tile(a.wk, tl);
            gv_stage_x<false>(a, g, sx, sxs);
            cons_sync();
        }
        float *sa = sact + buf * kGvSlots * 32;
        switch ((g.ns + 1) >> 1) {
            case 1: gv_gu_item<1>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 2: gv_gu_item<2>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 3: gv_gu_item<3>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 4: gv_gu_item<4>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 5: gv_gu_item<5>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 6: gv_gu_item<6>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            case 7: gv_gu_item<7>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
            default: gv_gu_item<8>(a, c, ring, full, empty, &s_abort, sx, sxs, sa, nst); break;
        }
        cons_sync();
        for (int j = warp; j < g.ns; j += kGvConsWarps) {   // Q8 group of each slot's 32 f values
            const Q8Lane q = quantize_lane(sa[j * 32 + lane]);
            if (c.ok) {
                const int slot = __ldcg(a.wk.slots + g.off + j);
                a.aq_q[(size_t)slot * a.F + sub * 32 + lane] = (int8_t)q.q;
                if (lane == 0) {
                    a.aq_d[(size_t)slot * ipt + sub] = q.d;
                    a.aq_s[(size_t)slot * ipt + sub] = q.sum;
                }
            }
        }
        buf ^= 1;
    }
}

// ---- down ------------------------------------------------------------------------------------------
// Item (tile, q, kh): down rows q*RD .. +RD-1 of the tile's expert (column stage row range q) over
// block columns kh*nb/2 .. +nb/2-1; stage st = the whole column stage (kh*nb/2 + st, q). Consumer
// thread t: rows t + 512 i, i < RPT = RD / 512 (two rows go as a pair).
template <bool Q1, int RPT, int NP>
__device__ __forceinline__ void gv_dn_item(const GvArgs &a, GvRing &c, uint8_t *ring, uint64_t *full, uint64_t *empty,
                                        volatile int *abort, const int8_t *sx, const uint8_t *sxs, int nst, int kh,
                                        int q, const GvTile &g) {
    constexpr int RD = 512 * RPT;
    constexpr uint32_t NIB = RD * 16, SCL = RD * 2;
    const int tid = threadIdx.x, lane = tid & 31, r1 = RPT == 2 ? tid + 512 : tid;
    float2 acc[2 * NP];                                   // RPT 2: rows (t, t + 512); 1: .x only
#pragma unroll
    for (int j = 0; j < 2 * NP; j++) acc[j] = make_float2(0.0f, 0.0f);
    for (int st = 0; st < nst; st++) {
        const uint8_t *stg = gv_acquire(a, c, ring, full, abort);
        uint4 n0 = make_uint4(0, 0, 0, 0), n1 = n0;
        float2 dw = make_float2(0.0f, 0.0f), mw = dw;
        if (stg) {
            n0 = *reinterpret_cast<const uint4 *>(stg + tid * 16);
            n1 = *reinterpret_cast<const uint4 *>(stg + r1 * 16);
            dw = make_float2(h2f(*reinterpret_cast<const uint16_t *>(stg + NIB + tid * 2)),
                             h2f(*reinterpret_cast<const uint16_t *>(stg + NIB + r1 * 2)));
            if (Q1)
                mw = make_float2(h2f(*reinterpret_cast<const uint16_t *>(stg + NIB + SCL + tid * 2)),
                                 h2f(*reinterpret_cast<const uint16_t *>(stg + NIB + SCL + r1 * 2)));
        }
        gv_release(c, empty, lane, a.ring);
        if (!stg) continue;
        uint32_t w0[8], w1[8];
        gv_split(n0, w0);
        gv_split(n1, w1);
        const int bc = kh * nst + st;
        const int8_t *xb = sx + (size_t)bc * kGvXRow;
        const uint8_t *sb = sxs + (size_t)bc * kGvSRow;
#pragma unroll
        for (int j = 0; j < 2 * NP; j++) {
            const uint4 x0 = *reinterpret_cast<const uint4 *>(xb + j * 32);
            const uint4 x1 = *reinterpret_cast<const uint4 *>(xb + j * 32 + 16);
            const uint2 xv = *reinterpret_cast<const uint2 *>(sb + j * 8);
            const float xd = __uint_as_float(xv.x);
            if (Q1) {                                  // d q + m: d dx isum + m (dx sum)  (src/kernels.c:109-121)
                const float2 p = gv_unmagic(gv_dot(w0, x0, x1, kGvMagic), RPT == 2 ? gv_dot(w1, x0, x1, kGvMagic) : kGvMagic);
                acc[j] = f2_fma(p, f2_mul(dw, make_float2(xd, xd)), acc[j]);
                const float ds = __uint_as_float(xv.y);
                acc[j] = f2_fma(mw, make_float2(ds, ds), acc[j]);
            } else {                                   // d (q - 8): the -8 sits in the chain's start
                const int bias = (int)xv.y;
                const float2 p = gv_unmagic(gv_dot(w0, x0, x1, bias), RPT == 2 ? gv_dot(w1, x0, x1, bias) : kGvMagic);
                acc[j] = f2_fma(p, f2_mul(dw, make_float2(xd, xd)), acc[j]);
            }
        }
    }
    if (c.ok) {
        float *dst = kh ? a.dn2 : a.dn;
#pragma unroll
        for (int j = 0; j < 2 * NP; j++) {
            if (j < 2 * NP - 1 || j < g.ns) {             // not the padding slot
                float *o = dst + (size_t)__ldcg(a.wk.slots + g.off + j) * a.E + q * RD + tid;
                o[0] = acc[j].x;
                if (RPT == 2) o[512] = acc[j].y;
            }
        }
    }
}

template <bool Q1, int RPT>
__global__ void __launch_bounds__(kGvThreads, 1) k_gv_down(const GvArgs a) {
    constexpr int RD = 512 * RPT;
    constexpr uint32_t STD = RD * (Q1 ? 20 : 18);
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort, s_lh[2], s_pre[kGvMaxTiles + 1];
    const int nb = a.nb, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t *ring = smem;
    int8_t *sx = reinterpret_cast<int8_t *>(smem + (size_t)a.ring * a.sst);
    uint8_t *sxs = reinterpret_cast<uint8_t *>(sx + (size_t)nb * kGvXRow);
    uint64_t *full = reinterpret_cast<uint64_t *>(sxs + (size_t)nb * kGvSRow);
    uint64_t *empty = full + a.ring;
    if (tid == 0) {
        s_abort = 0;
        for (int r = 0; r < a.ring; r++) {
            mbar_init(&full[r], 1);
            mbar_init(&empty[r], kGvConsWarps);
        }
        fence_mbar_init();
    }
    pdl_wait();
    pdl_trigger();
    const int Rq = a.dc.Rq, ipt = Rq * kGvKParts, nst = nb / kGvKParts;
    int lo, hi;
    gv_split_items(a.wk, min(__ldcg(a.wk.ntiles), kGvMaxTiles), ipt, s_pre, s_lh, lo, hi);
    if (warp == kGvConsWarps) {
        if (lane == 0)
            gv_produce(a, lo, hi, ipt, nst, ring, full, empty, &s_abort,
                       [&](const uint8_t *base, int sub, int st, uint8_t *dst, uint64_t *bar, uint64_t pol) {
                           const int kh = sub / Rq, q = sub - kh * Rq, bc = kh * nst + st;
                           mbar_arrive_expect_tx(bar, STD);
                           bulk_load(dst, base + (size_t)(bc * Rq + q) * STD, STD, bar, pol);
                       });
        return;
    }
    GvRing c{0, 0, true};
    int cur = -1;
    GvTile g{0, 0, 0};
    for (int item = lo; item < hi; item++) {
        const int tl = item / ipt, sub = item - tl * ipt, kh = sub / Rq, q = sub - kh * Rq;
        if (tl != cur) {
            cons_sync();
            cur = tl;
            g = gv_tile(a.wk, tl);
            gv_stage_x<Q1>(a, g, sx, sxs);
            cons_sync();
        }
        switch ((g.ns + 1) >> 1) {
            case 1: gv_dn_item<Q1, RPT, 1>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 2: gv_dn_item<Q1, RPT, 2>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 3: gv_dn_item<Q1, RPT, 3>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 4: gv_dn_item<Q1, RPT, 4>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 5: gv_dn_item<Q1, RPT, 5>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 6: gv_dn_item<Q1, RPT, 6>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            case 7: gv_dn_item<Q1, RPT, 7>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
            default: gv_dn_item<Q1, RPT, 8>(a, c, ring, full, empty, &s_abort, sx, sxs, nst, kh, q, g); break;
        }
    }
}

// dn[s] += dn2[s] for every grouped slot s (rows whose expert id was out of range stay as they
// were): the two K halves of the down rows into one (expert-parallel entry point). nx experts.
__global__ void __launch_bounds__(256) k_gv_add(float *__restrict__ dn, const float *__restrict__ dn2, MmaWork w,
                                                int nx, int E) {
    pdl_wait();
    const int nvalid = __ldcg(w.off + nx - 1) + __ldcg(w.cnt + nx - 1);
    const int q = E / 4;                                    // float4 per row
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)nvalid * q;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / q), c = (int)(i - (int64_t)r * q);
        const size_t at = (size_t)__ldcg(w.slots + r) * q + c;
        float4 a = reinterpret_cast<float4 *>(dn)[at];
        const float4 b = __ldcg(reinterpret_cast<const float4 *>(dn2) + at);
        a.x = __fadd_rn(a.x, b.x);
        a.y = __fadd_rn(a.y, b.y);
        a.z = __fadd_rn(a.z, b.z);
        a.w = __fadd_rn(a.w, b.w);
        reinterpret_cast<float4 *>(dn)[at] = a;
    }
}

// ---- host side -------------------------------------------------------------------------------------
static uint32_t al128(size_t n) { return (uint32_t)((n + 127) & ~(size_t)127); }

static uint32_t gv_stage_bytes(const QmsCudaMoe *m, bool gu) {
    return al128(gu ? 8 * (size_t)m->cgu.GB : (size_t)m->dcol.STD);
}

static size_t gv_fixed(const QmsCudaMoe *m, bool gu) {
    const int nb = gu ? m->nbE : m->nbF;
    return (size_t)nb * (kGvXRow + kGvSRow) + (gu ? 2 * kGvSlots * 32 * 4 : 0);
}

static int gv_ring(const QmsCudaMoe *m, bool gu) {
    const size_t fixed = gv_fixed(m, gu), sst = gv_stage_bytes(m, gu);
    if (fixed + 2 * (sst + 16) > kGvSmemCap) return 0;
    return (int)std::min<size_t>(kGvMaxRing, (kGvSmemCap - fixed) / (sst + 16));
}

static size_t gv_smem(const QmsCudaMoe *m, bool gu) {
    const int ring = gv_ring(m, gu);
    return (size_t)ring * gv_stage_bytes(m, gu) + gv_fixed(m, gu) + (size_t)ring * 16;
}

// Shapes the grouped GEMV covers: staged gate/up chunks of 16 blocks (n_embd % 512 == 0), down
// column stages of 512 or 1024 rows, F a multiple of 64 (two K halves of whole blocks), both rings
// at least 2 stages deep.
int gv_supported(const QmsCudaMoe *m) {
    return m->cgu.SB == 16 && m->F % 64 == 0 && (m->dcol.RD == 512 || m->dcol.RD == 1024) && m->X <= 256 &&
           gv_ring(m, true) >= 2 && gv_ring(m, false) >= 2;
}

static const void *gv_down_kernel(const QmsCudaMoe *m) {
    const bool q1 = m->dcol.q1, r2 = m->dcol.RD == 1024;
    return q1 ? (r2 ? (const void *)k_gv_down<true, 2> : (const void *)k_gv_down<true, 1>)
              : (r2 ? (const void *)k_gv_down<false, 2> : (const void *)k_gv_down<false, 1>);
}

int gv_prepare(QmsCudaMoe *m) {
    QMS_CK(cudaFuncSetAttribute(k_gv_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gv_smem(m, true)));
    QMS_CK(cudaFuncSetAttribute(gv_down_kernel(m), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gv_smem(m, false)));
    return QMS_CUDA_OK;
}

// gate/up + SwiGLU + Q8 into m's aq scratch, then the two K halves of the down rows into dn and
// dn2, for the slots grouped in w (at most maxT tiles of kGvSlots); activation row of slot s: s / rdiv
// of m's xq scratch. With sum_halves the second half is added into dn (S slots).
int gv_gemms(QmsCudaMoe *m, const MmaWork &w, int maxT, int S, int nx, int rdiv, float *dn, float *dn2,
             bool sum_halves, cudaStream_t s) {
    QMS_REQUIRE(maxT <= kGvMaxTiles, QMS_CUDA_EINVAL, "moe: %d tiles exceed the grouped GEMV's %d", maxT, kGvMaxTiles);
    GvArgs g;
    memset(&g, 0, sizeof g);
    g.w = m->gu;
    g.w_expert = m->gu_expert;
    g.c = m->cgu;
    g.dc = m->dcol;
    g.nb = m->nbE;
    g.F = m->F;
    g.E = m->E;
    g.wk = w;
    g.xq = m->xq_q;
    g.xd = m->xq_d;
    g.xs = m->xq_s;
    g.rdiv = rdiv;
    g.ring = gv_ring(m, true);
    g.sst = gv_stage_bytes(m, true);
    g.aq_q = m->aq_q;
    g.aq_d = m->aq_d;
    g.aq_s = m->aq_s;
    g.err = m->err;
    const dim3 grid(m->nsm), block(kGvThreads);
    QMS_CK(launch_pdl(k_gv_gate_up, grid, block, gv_smem(m, true), s, g));
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[3], s));
        QMS_CK(cudaEventRecord(m->ev[4], s));
    }
    GvArgs d = g;
    d.w = m->dn;
    d.w_expert = m->dn_expert;
    d.nb = m->nbF;
    d.xq = m->aq_q;
    d.xd = m->aq_d;
    d.xs = m->aq_s;
    d.rdiv = 1;
    d.ring = gv_ring(m, false);
    d.sst = gv_stage_bytes(m, false);
    d.dn = dn;
    d.dn2 = dn2;
    const size_t sm = gv_smem(m, false);
    if (m->dcol.q1) {
        if (m->dcol.RD == 1024) QMS_CK(launch_pdl(k_gv_down<true, 2>, grid, block, sm, s, d));
        else QMS_CK(launch_pdl(k_gv_down<true, 1>, grid, block, sm, s, d));
    } else {
        if (m->dcol.RD == 1024) QMS_CK(launch_pdl(k_gv_down<false, 2>, grid, block, sm, s, d));
        else QMS_CK(launch_pdl(k_gv_down<false, 1>, grid, block, sm, s, d));
    }
    if (sum_halves) {
        const int64_t n = (int64_t)S * m->E / 4;
        QMS_CK(launch_pdl(k_gv_add, dim3((unsigned)std::min<int64_t>((n + 255) / 256, 4 * m->nsm)), dim3(256), 0, s,
                          dn, (const float *)dn2, w, nx, m->E));
    }
    return QMS_CUDA_OK;
}

}  // namespace qms
