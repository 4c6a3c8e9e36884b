// qms_moe_mma.cu - the MoE block for T >= 5 tokens (batched decode, prefill): slot grouping, and
// the expert-grouped GEMMs on tcgen05 tensor cores, one kind::i8 MMA per 32-element block with a
// per-block scale epilogue.
//
// The reference's moe_group_fast (src/model.c:969-1007) groups the T*K (token, expert) slots by
// expert (:1066-1088) and runs each expert's gate/up rows and down rows once over all of its slots.
// Here every (expert, NW-slot tile) pair is one GEMM column tile (NW = 16 while the experts average
// <= 24 slots, else 64; the 16-slot calls go to the grouped GEMV of qms_moe_gemv.cu when it covers
// the shape):
//   k_mma_group    counting sort of the slots by expert; tile list (expert, tile index)
//   k_mma_gather   each tile's activations as MMA operands: the slots' Q8 rows rearranged into the
//                  tensor core's K-major core-matrix layout (one block of NW x 32 bytes per 32
//                  values), plus the per-block activation scales (and block sums for Q4_1 down)
//   k_mma_gemm<GU> 128 gate/up rows x NW slots per CTA: per 32-block, converter warps expand the
//                  Q4_0 nibbles to int8 (q - 8), one thread issues tcgen05.mma kind::i8 into a
//                  TMEM buffer (int32, exact), and 16 epilogue warps add P * (d_w * d_x) into fp32
//                  registers in block order (the reference's per-block scaling, src/kernels.c:82-107).
//                  Then silu(g) * u and its Q8 groups per slot (src/model.c:989-997).
//   k_mma_gemm<dn> 128 down rows x NW slots per CTA, the same pipeline over the F/32 blocks of the
//                  SwiGLU activations (Q4_1 down: q and the block sums, d q + m).
//   k_mma_combine  out[t] = sum_j w[t][j] * dn[t*K + j] in selection order (+ residual).
// A 32-block's int32 dot product is exact, so the per-block scaling happens in fp32 exactly as in
// the dp4a kernels; only the float summation order differs from the reference.
#include <string.h>

#include <algorithm>

#include "qms_async.cuh"
#include "qms_moe.cuh"

namespace qms {

constexpr int kMmaM = 128;                 // weight rows per tile (tensor-core M)
constexpr int kMmaN = 64;                  // slots per tile (tensor-core N) at larger loads
constexpr int kMmaNs = 16;                 // slots per tile when experts average few slots (batched decode)
constexpr int kMmaRaw = 2;                 // raw stages in flight (TMA ring)
constexpr int kMmaA = 16;                  // converted A blocks in flight
constexpr int kMmaGrp = 4;                 // blocks a converter pass expands (one fence, one wait)
#ifndef QMS_MMA_TMEM_BUFS
#define QMS_MMA_TMEM_BUFS 8
#endif
constexpr int kMmaTm = QMS_MMA_TMEM_BUFS;  // TMEM int32 buffers (64 columns each; 8 fill all 512)
#ifndef QMS_MMA_CONV_WARPS
#define QMS_MMA_CONV_WARPS 4
#endif
constexpr int kMmaConvWarps = QMS_MMA_CONV_WARPS;   // Q4 -> int8 converter warps (4: one row per thread)
#ifndef QMS_MMA_EPI_WARPS
#define QMS_MMA_EPI_WARPS 16
#endif
constexpr int kMmaEpiWarps = QMS_MMA_EPI_WARPS;     // per TMEM lane quarter kMmaEpiWarps / 4 column groups
constexpr int kMmaColGroups = kMmaEpiWarps / 4;
static_assert(kMmaEpiWarps % 4 == 0, "whole lane quarters");
constexpr int kMmaEpi0 = 2 + kMmaConvWarps;         // first epilogue warp
constexpr int kMmaThreads = (2 + kMmaConvWarps + kMmaEpiWarps) * 32;   // warp 0 TMA, 1 MMA, converters, epilogue
static_assert(kMmaConvWarps * 32 == kMmaM, "one A row per converter thread");
static_assert(kMmaA % kMmaGrp == 0 && 8 % kMmaGrp == 0, "converter groups tile the ring and every stage");
constexpr uint32_t kMmaSpin = 1u << 22;
constexpr uint32_t kABlock = 4096;         // one block of the A operand: 128 rows x 32 bytes
constexpr uint32_t kChunkPad = 16;         // gap after each raw gate/up chunk: rows of different
                                           // chunks start in different shared-memory banks

enum { MMA_ERR = 64 };

// ---- tcgen05 helpers ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8 rows x 16 bytes (rows
// 16 bytes apart); lbo = byte distance between the two 16-byte K halves, sbo = between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor: s8 x s8 -> s32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_s8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc) {
    const uint32_t zero = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(zero), "r"(zero)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 TMEM lanes (this warp's quarter) x C consecutive 32-bit columns, C = 4, 8, 16 or 32 (not waited).
template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[C]) {
    if constexpr (C == 32) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
              "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
    } else if constexpr (C == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    } else if constexpr (C == 8) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                     : "r"(taddr));
    } else {
        static_assert(C == 4, "4, 8, 16 or 32 columns");
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                     : "r"(taddr));
    }
}

// Bounded wait on an mbarrier phase; on timeout set the CTA's abort flag and the error bit.
__device__ __forceinline__ bool mma_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (++n == kMmaSpin) {
            *abort = 1;
            atomicOr(err, MMA_ERR);
            return false;
        }
        if (n > 64) __nanosleep(32);
    }
    return true;
}

// Q4 nibbles of one 32-block (16 bytes) -> 32 int8 values in element order: elements 0-15 are the
// low nibbles (first K half), 16-31 the high nibbles. Q4_0 subtracts 8 (src/quant.c:19-28).
__device__ __forceinline__ void nib_to_s8(uint4 v, bool minus8, uint4 &lo, uint4 &hi) {
    const uint32_t m = 0x0F0F0F0Fu;
    uint32_t w[8] = {v.x & m, v.y & m, v.z & m, v.w & m, (v.x >> 4) & m, (v.y >> 4) & m, (v.z >> 4) & m, (v.w >> 4) & m};
    if (minus8) {
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = ((w[i] | 0x80808080u) - 0x08080808u) ^ 0x80808080u;   // bytewise q - 8
    }
    lo = make_uint4(w[0], w[1], w[2], w[3]);
    hi = make_uint4(w[4], w[5], w[6], w[7]);
}

// ---- slot grouping -------------------------------------------------------------------------------
// One CTA: slots s = t*K + j grouped by expert sel[s]; tiles of nw slots per expert.
__global__ void __launch_bounds__(1024) k_mma_group(const int *__restrict__ sel, int S, int X, int maxT, int nw, MmaWork w) {
    __shared__ int s_cnt[256], s_off[257], s_toff[257];
    const int tid = threadIdx.x;
    pdl_wait();
    for (int e = tid; e < X; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    for (int s = tid; s < S; s += blockDim.x) {
        const int e = __ldcg(sel + s);
        w.pos[s] = (unsigned)e < (unsigned)X ? atomicAdd(&s_cnt[e], 1) : -1;
    }
    __syncthreads();
    if (tid == 0) {
        int o = 0, t = 0;
        for (int e = 0; e < X; e++) {
            s_off[e] = o;
            s_toff[e] = t;
            o += s_cnt[e];
            t += (s_cnt[e] + nw - 1) / nw;
        }
        s_off[X] = o;
        s_toff[X] = t < maxT ? t : maxT;
        *w.ntiles = s_toff[X];
    }
    __syncthreads();
    for (int e = tid; e < X; e += blockDim.x) {
        w.cnt[e] = s_cnt[e];
        w.off[e] = s_off[e];
        w.toff[e] = s_toff[e];
        for (int i = 0; s_toff[e] + i < s_toff[e + 1] && s_toff[e] + i < maxT; i++)
            w.tiles[s_toff[e] + i] = e | (i << 16);
    }
    for (int s = tid; s < S; s += blockDim.x) {
        const int e = __ldcg(sel + s);
        if ((unsigned)e < (unsigned)X) w.slots[s_off[e] + w.pos[s]] = s;
    }
}

// B operands of every tile: column j of tile (e, n0) is slot slots[off[e] + n0 + j] (zeros past
// the expert's count). Source row of slot s: s / rdiv (gate/up reads the token's Q8 row, down the
// slot's). Block b of a tile of nw slots: [K half][nw/8 slot groups][8 slots][16 bytes]. One thread
// per (slot, K half): blockDim = 2 * nw.
__global__ void __launch_bounds__(128) k_mma_gather(const int8_t *__restrict__ q, const float *__restrict__ d,
                                                    const int *__restrict__ sums, int nb, int rdiv, int nw, MmaWork w) {
    const int tl = blockIdx.x;
    pdl_wait();
    if (tl >= __ldcg(w.ntiles)) return;
    const int tile = __ldcg(w.tiles + tl), e = tile & 0xFFFF, n0 = (tile >> 16) * nw;
    const int n = min(nw, __ldcg(w.cnt + e) - n0);
    const int j = threadIdx.x >> 1, h = threadIdx.x & 1;
    const int slot = j < n ? __ldcg(w.slots + __ldcg(w.off + e) + n0 + j) : -1;
    const size_t row = slot >= 0 ? (size_t)(slot / rdiv) : 0;
    const int K = nb * 32;
    const size_t bt = (size_t)nw * 32;                      // bytes of one block of the tile
    for (int b = blockIdx.y; b < nb; b += gridDim.y) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (slot >= 0) v = __ldcg(reinterpret_cast<const uint4 *>(q + row * K + b * 32 + h * 16));
        int8_t *dst = w.bg + ((size_t)tl * nb + b) * bt;
        *reinterpret_cast<uint4 *>(dst + h * (nw * 16) + (j >> 3) * 128 + (j & 7) * 16) = v;
        if (h == 0) {
            w.bs[((size_t)tl * nb + b) * nw + j] = slot >= 0 ? __ldcg(d + row * nb + b) : 0.0f;
            if (sums) w.bsum[((size_t)tl * nb + b) * nw + j] = slot >= 0 ? __ldcg(sums + row * nb + b) : 0;
        }
    }
}

// ---- the grouped GEMM ------------------------------------------------------------------------------
// One template for both products. GU: A = 128 gate/up rows of the staged chunks (two 64-row tiles,
// rows 0-31 gate / 32-63 up of each), K = E/32 blocks; epilogue = SwiGLU + Q8 groups. !GU: A = 128
// down rows from the column stages, K = F/32 blocks; epilogue = fp32 rows per slot.
struct MmaArgs {
    const uint8_t *w;          // staged experts (gate/up chunks or down column stages)
    size_t w_expert;
    Chunked cgu;               // GU layout
    DnCols dc;                 // !GU layout
    int nb, SB;                // blocks along K, blocks per stage
    int F, E, K;               // model shape
    MmaWork wk;
    int8_t *aq_q;              // GU out: [T*K][F] Q8 values
    float *aq_d;               // GU out: [T*K][F/32]
    int *aq_s;                 // GU out: [T*K][F/32] block sums
    int *err;
};

// raw A bytes of one stage in shared memory: 16 gate/up chunks (+ gaps), or SB down blocks of
// 128 rows (nibbles 2048 B, scales 256 B, Q4_1 mins 256 B)
__host__ __device__ inline uint32_t raw_a_bytes(bool gu, uint32_t chunk_bytes, int SB, bool q1) {
    return gu ? 16u * (chunk_bytes + kChunkPad) : (uint32_t)SB * (q1 ? 2560u : 2304u);
}

template <bool GU, bool Q1, int NW>
__global__ void __launch_bounds__(kMmaThreads, 1) k_mma_gemm(const MmaArgs a) {
    constexpr int EC = NW / kMmaColGroups;                      // columns per epilogue warp
    constexpr uint32_t BT = NW * 32;                            // one block of the B operand
    extern __shared__ __align__(1024) uint8_t smem[];
    const int SB = a.SB, nb = a.nb;
    const uint32_t GB = a.cgu.GB, CP = GB + kChunkPad;       // gate/up chunk bytes, chunk stride
    const uint32_t RA = raw_a_bytes(GU, GB, SB, Q1);           // raw A bytes per stage
    const uint32_t RB = (uint32_t)SB * BT;                     // B operand bytes per stage
    const uint32_t RS = (uint32_t)SB * NW * 4;                 // activation scales per stage
    const uint32_t RU = Q1 ? RS : 0;                           // activation block sums per stage
    const uint32_t RSLOT = (RA + RB + RS + RU + 127) & ~127u;
    uint8_t *raw = smem;                                       // [kMmaRaw][RSLOT]
    uint8_t *abuf = smem + kMmaRaw * RSLOT;                    // [kMmaA][kABlock]
    uint64_t *bars = reinterpret_cast<uint64_t *>(abuf + kMmaA * kABlock);
    uint64_t *raw_full = bars, *raw_empty = raw_full + kMmaRaw;
    uint64_t *a_full = raw_empty + kMmaRaw, *a_empty = a_full + kMmaA;
    uint64_t *tm_full = a_empty + kMmaA, *tm_empty = tm_full + kMmaTm;
    float *xch = reinterpret_cast<float *>(raw);               // after the K loop: [2][groups][32][EC + 1] up sums
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int tl = blockIdx.y, mt = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();                                                 // the tile list and operands come from the previous kernels
    if (tl >= __ldcg(a.wk.ntiles)) return;                     // uniform per CTA, before any barrier
    const int tile = __ldcg(a.wk.tiles + tl), e = tile & 0xFFFF, n0 = (tile >> 16) * NW;
    const int ncol = min(NW, __ldcg(a.wk.cnt + e) - n0);
    const int soff = __ldcg(a.wk.off + e) + n0;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < kMmaRaw; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kMmaConvWarps + kMmaEpiWarps);
        }
        for (int i = 0; i < kMmaA; i++) {
            mbar_init(&a_full[i], kMmaConvWarps);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kMmaTm; i++) {
            mbar_init(&tm_full[i], 1);
            mbar_init(&tm_empty[i], kMmaEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kMmaTm * NW)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    volatile int *abort_flag = &s_abort;
    const int nst = nb / SB;

    if (warp == 0) {                                            // ---- TMA producer
        if (lane == 0) {
            const uint8_t *we = a.w + (size_t)e * a.w_expert;
            const int8_t *bg = a.wk.bg + (size_t)tl * nb * BT;
            const float *bs = a.wk.bs + (size_t)tl * nb * NW;
            const int *bu = a.wk.bsum + (size_t)tl * nb * NW;
            const uint64_t pol = evict_first_policy();
            int issued = 0;
            bool ok = true;
            for (int s = 0; s < nst && ok; s++) {
                const int slot = s % kMmaRaw;
                if (s >= kMmaRaw && !(ok = mma_wait(&raw_empty[slot], ((s / kMmaRaw) & 1) ^ 1, abort_flag, a.err)))
                    break;
                uint8_t *dst = raw + (size_t)slot * RSLOT;
                mbar_arrive_expect_tx(&raw_full[slot], (GU ? 16u * GB : RA) + RB + RS + RU);
                if (GU) {
                    const size_t tile_bytes = (size_t)a.cgu.S * 8 * GB;
                    for (int c = 0; c < 16; c++) {                  // 2 tiles x 8 chunks of stage s
                        const uint8_t *src = we + (size_t)(2 * mt + c / 8) * tile_bytes + ((size_t)s * 8 + (c & 7)) * GB;
                        bulk_load(dst + c * CP, src, GB, &raw_full[slot], pol);
                    }
                } else {
                    const int r0 = mt * kMmaM;
                    const uint32_t per = Q1 ? 2560u : 2304u;
                    for (int bl = 0; bl < SB; bl++) {
                        const uint8_t *st = we + dn_stage_off(a.dc, s * SB + bl, r0);
                        uint8_t *db = dst + bl * per;
                        bulk_load(db, st + dn_nib_off(a.dc, r0), 2048, &raw_full[slot], pol);
                        bulk_load(db + 2048, st + dn_scale_off(a.dc, r0), 256, &raw_full[slot], pol);
                        if (Q1) bulk_load(db + 2304, st + dn_min_off(a.dc, r0), 256, &raw_full[slot], pol);
                    }
                }
                bulk_load(dst + RA, bg + (size_t)s * RB, RB, &raw_full[slot], pol);
                bulk_load(dst + RA + RB, bs + (size_t)s * SB * NW, RS, &raw_full[slot], pol);
                if (Q1) bulk_load(dst + RA + RB + RS, bu + (size_t)s * SB * NW, RU, &raw_full[slot], pol);
                issued++;
            }
            // copies still in flight after an abort must land before the CTA exits
            for (int j = issued > kMmaRaw ? issued - kMmaRaw : 0; j < issued && !ok; j++) {
                uint32_t n = 0;
                while (!mbar_try_wait(&raw_full[j % kMmaRaw], (j / kMmaRaw) & 1) && ++n < kMmaSpin) {
                }
            }
        }
    } else if (warp == 1) {                                     // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_s8(kMmaM, NW);
            // one pass per converter group: the last slot's barrier implies the group's earlier ones
            // (every converter warp arrives them in order), likewise for the epilogue's TMEM buffers
            const uint32_t a0 = smem_u32(abuf), r0 = smem_u32(raw) + RA;
            int issued = 0, s = 0, bl0 = 0;
            for (int b0 = 0; b0 < nb; b0 += kMmaGrp) {
                const int bl = b0 + kMmaGrp - 1;
                if (!mma_wait(&a_full[bl % kMmaA], (bl / kMmaA) & 1, abort_flag, a.err)) break;
                if (bl >= kMmaTm) {                             // TMEM buffers read out by the epilogue
                    if (!mma_wait(&tm_empty[bl % kMmaTm], ((bl / kMmaTm) & 1) ^ 1, abort_flag, a.err)) break;
                    tc_fence_after();
                }
                const uint32_t rb = r0 + (uint32_t)(s % kMmaRaw) * RSLOT + (uint32_t)bl0 * BT;
#pragma unroll
                for (int g = 0; g < kMmaGrp; g++) {
                    const int b = b0 + g;
                    const uint64_t da = umma_desc(a0 + (uint32_t)(b % kMmaA) * kABlock, 2048, 128);
                    const uint64_t db = umma_desc(rb + (uint32_t)g * BT, NW * 16, 128);
                    umma_s8(tmem + (b % kMmaTm) * NW, da, db, idesc);
                    umma_commit(&tm_full[b % kMmaTm]);
                }
                issued += kMmaGrp;
                bl0 += kMmaGrp;
                if (bl0 == SB) {
                    bl0 = 0;
                    s++;
                }
            }
            // the tensor core must be idle before TMEM is freed
            if (issued > 0) {
                uint32_t n = 0;
                const int lb = issued - 1;
                while (!mbar_try_wait(&tm_full[lb % kMmaTm], (lb / kMmaTm) & 1) && ++n < kMmaSpin) {
                }
            }
        }
    } else if (warp < kMmaEpi0) {                               // ---- converters: Q4 -> int8 A blocks
        // thread ct expands row ct of kMmaGrp blocks per pass: one fence and one barrier arrival
        // per block group rather than per block
        const int R = threadIdx.x - 64;                         // 0..127 (kMmaConvWarps == 4)
        bool ok = true;
        int s = 0, bl0 = 0;
        for (int b0 = 0; b0 < nb && ok; b0 += kMmaGrp) {
            if (bl0 == 0) ok = __all_sync(0xffffffffu, mma_wait(&raw_full[s % kMmaRaw], (s / kMmaRaw) & 1, abort_flag, a.err));
            for (int g = 0; g < kMmaGrp && ok; g++) {
                const int b = b0 + g;
                if (b >= kMmaA) ok = __all_sync(0xffffffffu, mma_wait(&a_empty[b % kMmaA], ((b / kMmaA) & 1) ^ 1, abort_flag, a.err));
            }
            if (!ok) break;
            const uint8_t *rs = raw + (size_t)(s % kMmaRaw) * RSLOT;
            const uint8_t *src;
            uint32_t bstride;                                   // bytes from block bl to bl + 1 in the raw stage
            if (GU) {
                const int c = (R >> 6) * 8 + ((R & 63) >> 3), rr = R & 7;
                src = rs + c * CP + (rr * SB + bl0) * 16;
                bstride = 16;
            } else {
                src = rs + bl0 * (Q1 ? 2560 : 2304) + R * 16;
                bstride = Q1 ? 2560 : 2304;
            }
            uint4 v[kMmaGrp];
#pragma unroll
            for (int g = 0; g < kMmaGrp; g++) v[g] = *reinterpret_cast<const uint4 *>(src + g * bstride);
#pragma unroll
            for (int g = 0; g < kMmaGrp; g++) {
                uint4 lo, hi;
                nib_to_s8(v[g], !Q1, lo, hi);
                uint8_t *ab = abuf + ((b0 + g) % kMmaA) * kABlock;
                *reinterpret_cast<uint4 *>(ab + (R >> 3) * 128 + (R & 7) * 16) = lo;
                *reinterpret_cast<uint4 *>(ab + 2048 + (R >> 3) * 128 + (R & 7) * 16) = hi;
            }
            fence_async_smem();                                 // generic-proxy writes -> tensor core
            __syncwarp();
            if (lane == 0)
                for (int g = 0; g < kMmaGrp; g++) mbar_arrive(&a_full[(b0 + g) % kMmaA]);
            bl0 += kMmaGrp;
            if (bl0 == SB) {
                if (lane == 0) mbar_arrive(&raw_empty[s % kMmaRaw]);
                bl0 = 0;
                s++;
            }
        }
    } else {                                                    // ---- epilogue: 8 warps
        // two blocks per pass: one wait, one TMEM round trip and one release per pair, so the
        // per-block bookkeeping stays small next to the 2 x EC columns of scaling
        const int q = warp & 3, cq = (warp - kMmaEpi0) >> 2, R = 32 * q + lane;   // lane quarter, column group (EC columns)
        float acc[EC];
#pragma unroll
        for (int j = 0; j < EC; j++) acc[j] = 0.0f;
        bool ok = true;
        int s = 0, bl = 0;
        for (int b = 0; b < nb && ok; b += 2) {
            const int b1 = b + 1;                               // nb % 8 == 0: pairs never straddle the end
            ok = __all_sync(0xffffffffu, mma_wait(&tm_full[b1 % kMmaTm], (b1 / kMmaTm) & 1, abort_flag, a.err));
            if (!ok) break;
            if (warp == kMmaEpi0 && lane == 0) {                // the MMAs have read their A blocks
                mbar_arrive(&a_empty[b % kMmaA]);
                mbar_arrive(&a_empty[b1 % kMmaA]);
            }
            tc_fence_after();
            uint32_t r[2][EC];
#pragma unroll
            for (int i = 0; i < 2; i++)
                tmem_ld<EC>(tmem + ((uint32_t)(32 * q) << 16) + ((b + i) % kMmaTm) * NW + cq * EC, r[i]);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tm_empty[b % kMmaTm]);
                mbar_arrive(&tm_empty[b1 % kMmaTm]);
            }
            const uint8_t *rs = raw + (size_t)(s % kMmaRaw) * RSLOT;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                float dw, mw = 0.0f;
                if (GU) {
                    const int c = (R >> 6) * 8 + ((R & 63) >> 3), rr = R & 7;
                    dw = h2f(*reinterpret_cast<const uint16_t *>(rs + c * CP + 8 * SB * 16 + (rr * SB + bl + i) * 2));
                } else {
                    const uint8_t *pb = rs + (bl + i) * (Q1 ? 2560 : 2304);
                    dw = h2f(*reinterpret_cast<const uint16_t *>(pb + 2048 + R * 2));
                    if (Q1) mw = h2f(*reinterpret_cast<const uint16_t *>(pb + 2304 + R * 2));
                }
                const float *sx = reinterpret_cast<const float *>(rs + RA + RB) + (bl + i) * NW + cq * EC;
                const int *su = reinterpret_cast<const int *>(rs + RA + RB + RS) + (bl + i) * NW + cq * EC;
                // int32 -> float without the conversion unit: |P| < 2^22, so 2^23 + 2^22 + P is exact
                // in a float's mantissa; pairs of columns go through the packed f32x2 pipe
#pragma unroll
                for (int j = 0; j < EC; j += 2) {
                    const float2 xd = *reinterpret_cast<const float2 *>(sx + j);
                    float2 p2 = make_float2(__int_as_float((int)r[i][j] + 0x4B400000),
                                            __int_as_float((int)r[i][j + 1] + 0x4B400000));
                    p2 = f2_add(p2, make_float2(-12582912.0f, -12582912.0f));
                    const float2 sc = f2_mul(make_float2(dw, dw), xd);
                    float2 ac = make_float2(acc[j], acc[j + 1]);
                    if (Q1) {
                        const float2 mc = f2_mul(make_float2(mw, mw), make_float2(xd.x * (float)su[j], xd.y * (float)su[j + 1]));
                        ac = f2_add(ac, mc);
                    }
                    ac = f2_fma(p2, sc, ac);
                    acc[j] = ac.x;
                    acc[j + 1] = ac.y;
                }
            }
            __syncwarp();
            bl += 2;
            if (bl == SB) {
                if (lane == 0) mbar_arrive(&raw_empty[s % kMmaRaw]);
                bl = 0;
                s++;
            }
        }
        // every epilogue warp is done with the raw stages before they hold the exchange
        asm volatile("bar.sync 1, %0;" ::"n"(kMmaEpiWarps * 32) : "memory");
        if (GU) {
            // rows 0-31 / 64-95 (lane quarters 0, 2) are gate rows f, 32-63 / 96-127 the up rows of
            // the same f: the up warps hand their sums over, the gate warps finish the groups
            const int th = q >> 1;                                // which 64-row tile
            float *xu = xch + ((th * kMmaColGroups + cq) * 32 + lane) * (EC + 1);
            if (q & 1)
#pragma unroll
                for (int j = 0; j < EC; j++) xu[j] = acc[j];
            asm volatile("bar.sync 1, %0;" ::"n"(kMmaEpiWarps * 32) : "memory");
            if (!(q & 1) && ok && !*abort_flag) {
                const int f = 64 * mt + 32 * th + lane, grp = f >> 5;
#pragma unroll
                for (int j = 0; j < EC; j++) {
                    const int col = cq * EC + j;
                    if (col >= ncol) continue;                   // warp-uniform
                    const float g = acc[j], u = xu[j];
                    const float av = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                    const Q8Lane q8 = quantize_lane(av);
                    const int slot = __ldcg(a.wk.slots + soff + col);
                    a.aq_q[(size_t)slot * a.F + f] = (int8_t)q8.q;
                    if (lane == 0) {
                        a.aq_d[(size_t)slot * (a.F / 32) + grp] = q8.d;
                        a.aq_s[(size_t)slot * (a.F / 32) + grp] = q8.sum;
                    }
                }
            }
        } else if (ok && !*abort_flag) {
            const int row = mt * kMmaM + R;
#pragma unroll
            for (int j = 0; j < EC; j++) {
                const int col = cq * EC + j;
                if (col >= ncol) continue;
                const int slot = __ldcg(a.wk.slots + soff + col);
                a.wk.dn[(size_t)slot * a.E + row] = acc[j];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kMmaTm * NW) : "memory");
    }
}

// out[t][i] = sum_j w[t][j] * dn[t*K + j][i] in selection order (src/model.c:1152-1162), + resid.
// dn2 (optional): second K half of each down row, added to the first before weighting.
__global__ void __launch_bounds__(256) k_mma_combine(const float *__restrict__ dn, const float *__restrict__ dn2,
                                                     const float *__restrict__ wts, int K, int E, const float *resid,
                                                     float *out) {
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    if (i >= E) return;
    float o = 0.0f;
    for (int j = 0; j < K; j++) {
        const size_t at = ((size_t)t * K + j) * E + i;
        const float d = dn2 ? __fadd_rn(__ldcg(dn + at), __ldcg(dn2 + at)) : __ldcg(dn + at);
        o = __fmaf_rn(__ldcg(wts + t * K + j), d, o);
    }
    if (resid) o = __fadd_rn(resid[(size_t)t * E + i], o);
    out[(size_t)t * E + i] = o;
}

// ---- host side -------------------------------------------------------------------------------------
static size_t mma_smem(const QmsCudaMoe *m, int SB, bool gu, bool q1, int nw) {
    const size_t RA = raw_a_bytes(gu, m->cgu.GB, SB, q1);
    const size_t RSLOT = (RA + (size_t)SB * nw * 32 + (size_t)SB * nw * 4 * (q1 ? 2 : 1) + 127) & ~(size_t)127;
    return kMmaRaw * RSLOT + kMmaA * kABlock + (2 * kMmaRaw + 2 * kMmaA + 2 * kMmaTm) * 8;
}

// Device workspace shared by every layer of the process (layers run one after another on a stream).
static struct {
    void *p = nullptr;
    size_t bytes = 0;
    int dev = -1;
} g_mma_ws;

// Tile width for S slots over nx experts: 16 slots while the experts average <= 24 slots, else 64.
static int mma_width(int S, int nx) { return (int64_t)S <= (int64_t)24 * nx ? kMmaNs : kMmaN; }

static int mma_layout(const QmsCudaMoe *m, int T, MmaWork *w, size_t *bytes, char *base) {
    const size_t S = (size_t)T * m->K;
    const size_t maxT = S / kMmaNs + m->X;                                  // tiles at the narrower width
    const size_t bcols = std::max(maxT * kMmaNs, (S / kMmaN + m->X) * kMmaN);   // B columns at either width
    const int nbmax = std::max(m->nbE, m->nbF);
    size_t off = 0;
    auto take = [&](size_t n) { size_t o = off; off += (n + 255) & ~(size_t)255; return base + o; };
    w->cnt = (int *)take(m->X * 4);
    w->off = (int *)take((m->X + 1) * 4);
    w->toff = (int *)take((m->X + 1) * 4);
    w->ntiles = (int *)take(4);
    w->pos = (int *)take(S * 4);
    w->slots = (int *)take(S * 4);
    w->tiles = (int *)take(maxT * 4);
    w->bg = (int8_t *)take(bcols * nbmax * 32);
    w->bs = (float *)take(bcols * nbmax * 4);
    w->bsum = (int *)take(bcols * nbmax * 4);
    w->dn = (float *)take(S * m->E * 4);
    w->dn2 = (float *)take(std::min(S, (size_t)24 * m->X) * m->E * 4);
    *bytes = off;
    return QMS_CUDA_OK;
}

// Is the grouped tensor-core path usable for this layer (shapes the tiling covers)?
int mma_supported(const QmsCudaMoe *m) {
    return m->F % 64 == 0 && m->E % kMmaM == 0 && m->X <= 256 && m->nbE % m->cgu.SB == 0 && m->nbF % 8 == 0 &&
           m->dcol.RD % kMmaM == 0;
}

int mma_prepare(QmsCudaMoe *m) {
    const int SBd = 8;
    auto set = [](const void *k, size_t smem) -> int {
        QMS_CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        return QMS_CUDA_OK;
    };
    int rc;
    if ((rc = set((const void *)k_mma_gemm<true, false, kMmaN>, mma_smem(m, m->cgu.SB, true, false, kMmaN)))) return rc;
    if ((rc = set((const void *)k_mma_gemm<false, false, kMmaN>, mma_smem(m, SBd, false, false, kMmaN)))) return rc;
    if ((rc = set((const void *)k_mma_gemm<false, true, kMmaN>, mma_smem(m, SBd, false, true, kMmaN)))) return rc;
    if ((rc = set((const void *)k_mma_gemm<true, false, kMmaNs>, mma_smem(m, m->cgu.SB, true, false, kMmaNs)))) return rc;
    if ((rc = set((const void *)k_mma_gemm<false, false, kMmaNs>, mma_smem(m, SBd, false, false, kMmaNs)))) return rc;
    if ((rc = set((const void *)k_mma_gemm<false, true, kMmaNs>, mma_smem(m, SBd, false, true, kMmaNs)))) return rc;
    return QMS_CUDA_OK;
}

template <int NW>
static int mma_gemms(QmsCudaMoe *m, const MmaArgs &g, const MmaArgs &d, int maxT, cudaStream_t s) {
    const int SBd = d.SB;
    QMS_CK(launch_pdl(k_mma_gemm<true, false, NW>, dim3(2 * m->F / kMmaM, maxT), dim3(kMmaThreads),
                      mma_smem(m, g.SB, true, false, NW), s, g));
    if (m->timing) {
        QMS_CK(cudaEventRecord(m->ev[3], s));
        QMS_CK(cudaEventRecord(m->ev[4], s));
    }
    QMS_CK(launch_pdl(k_mma_gather, dim3(maxT, 8), dim3(2 * NW), 0, s, (const int8_t *)m->aq_q, (const float *)m->aq_d,
                      (const int *)m->aq_s, m->nbF, 1, NW, g.wk));
    if (m->dcol.q1)
        QMS_CK(launch_pdl(k_mma_gemm<false, true, NW>, dim3(m->E / kMmaM, maxT), dim3(kMmaThreads),
                          mma_smem(m, SBd, false, true, NW), s, d));
    else
        QMS_CK(launch_pdl(k_mma_gemm<false, false, NW>, dim3(m->E / kMmaM, maxT), dim3(kMmaThreads),
                          mma_smem(m, SBd, false, false, NW), s, d));
    return QMS_CUDA_OK;
}

// The expert FFNs of S slots: slot s has Q8 row s / rdiv in m's xq scratch and expert sel[s]
// (0 .. nx-1); dn[s][E] receives its down row. Slots whose expert is out of range are skipped.
static int mma_core(QmsCudaMoe *m, int S, const int *sel, int nx, int rdiv, float *dn, cudaStream_t s) {
    const int T = (S + m->K - 1) / m->K;                 // workspace is sized in tokens of K slots
    MmaWork w;
    size_t need = 0;
    mma_layout(m, T, &w, &need, nullptr);
    if (need > g_mma_ws.bytes || g_mma_ws.dev != m->device) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QMS_CK(cudaStreamIsCapturing(s, &cs));
        QMS_REQUIRE(cs == cudaStreamCaptureStatusNone, QMS_CUDA_EINVAL,
                    "moe: tensor-core workspace for %d slots must be reserved before graph capture", S);
        QMS_CK(cudaStreamSynchronize(s));
        if (g_mma_ws.p) cudaFree(g_mma_ws.p);
        g_mma_ws.p = nullptr;
        g_mma_ws.bytes = 0;
        if (cudaMalloc(&g_mma_ws.p, need) != cudaSuccess) {
            cudaGetLastError();
            set_error("moe: cannot allocate %zu bytes of tensor-core workspace", need);
            return QMS_CUDA_ENOMEM;
        }
        g_mma_ws.bytes = need;
        g_mma_ws.dev = m->device;
    }
    mma_layout(m, T, &w, &need, (char *)g_mma_ws.p);
    if (dn) w.dn = dn;
    const int nw = mma_width(S, nx), maxT = S / nw + nx;
    QMS_CK(launch_pdl(k_mma_group, dim3(1), dim3(1024), 0, s, sel, S, nx, maxT, nw, w));
    if (m->gemv && nw == kMmaNs)                       // few slots per expert: CUDA cores
        return gv_gemms(m, w, maxT, S, nx, rdiv, w.dn, w.dn2, dn != nullptr, s);
    QMS_CK(launch_pdl(k_mma_gather, dim3(maxT, 8), dim3(2 * nw), 0, s, (const int8_t *)m->xq_q, (const float *)m->xq_d,
                      (const int *)nullptr, m->nbE, rdiv, nw, w));
    MmaArgs g;
    memset(&g, 0, sizeof g);
    g.w = m->gu;
    g.w_expert = m->gu_expert;
    g.cgu = m->cgu;
    g.dc = m->dcol;
    g.nb = m->nbE;
    g.SB = m->cgu.SB;
    g.F = m->F;
    g.E = m->E;
    g.K = m->K;
    g.wk = w;
    g.aq_q = m->aq_q;
    g.aq_d = m->aq_d;
    g.aq_s = m->aq_s;
    g.err = m->err;
    MmaArgs d = g;
    d.w = m->dn;
    d.w_expert = m->dn_expert;
    d.nb = m->nbF;
    d.SB = 8;                                           // down stages: 8 blocks (F/32 % 8 == 0)
    return nw == kMmaNs ? mma_gemms<kMmaNs>(m, g, d, maxT, s) : mma_gemms<kMmaN>(m, g, d, maxT, s);
}

// T > 1 tokens: router output (xq, sel, wts) already in m's scratch.
int mma_forward(QmsCudaMoe *m, int T, const float *resid, float *out, cudaStream_t s) {
    int rc = mma_core(m, T * m->K, m->sel, m->X, m->K, nullptr, s);
    if (rc) return rc;
    MmaWork w;
    size_t need = 0;
    mma_layout(m, T, &w, &need, (char *)g_mma_ws.p);
    const bool halves = m->gemv && mma_width(T * m->K, m->X) == kMmaNs;   // the grouped GEMV ran
    QMS_CK(launch_pdl(k_mma_combine, dim3((m->E + 255) / 256, T), dim3(256), 0, s, (const float *)w.dn,
                      halves ? (const float *)w.dn2 : nullptr, (const float *)m->wts, m->K, m->E, resid, out));
    if (m->timing) QMS_CK(cudaEventRecord(m->ev[5], s));
    return QMS_CUDA_OK;
}

// Expert FFNs of S slots whose rows are already quantised in m's xq scratch (row s) - the expert
// side of expert parallelism. expert[s] is a local expert id (0 .. n_local - 1).
int mma_experts(QmsCudaMoe *m, int S, const int *expert, float *dn, cudaStream_t s) {
    return mma_core(m, S, expert, m->n_local, 1, dn, s);
}

// out[t] = sum_j w[t][j] * dn[t*K + j] in selection order (+ resid)
int mma_combine(const float *dn, const float *wts, int T, int K, int E, const float *resid, float *out,
                cudaStream_t s) {
    QMS_CK(launch_pdl(k_mma_combine, dim3((E + 255) / 256, T), dim3(256), 0, s, dn, (const float *)nullptr, wts, K, E,
                      resid, out));
    return QMS_CUDA_OK;
}

int mma_reserve(QmsCudaMoe *m, int T) {
    MmaWork w;
    size_t need = 0;
    mma_layout(m, T, &w, &need, nullptr);
    if (need <= g_mma_ws.bytes && g_mma_ws.dev == m->device) return QMS_CUDA_OK;
    QMS_CK(cudaDeviceSynchronize());
    if (g_mma_ws.p) cudaFree(g_mma_ws.p);
    g_mma_ws.p = nullptr;
    g_mma_ws.bytes = 0;
    if (cudaMalloc(&g_mma_ws.p, need) != cudaSuccess) {
        cudaGetLastError();
        set_error("moe_reserve: cannot allocate %zu bytes of tensor-core workspace", need);
        return QMS_CUDA_ENOMEM;
    }
    g_mma_ws.bytes = need;
    g_mma_ws.dev = m->device;
    return QMS_CUDA_OK;
}

}  // namespace qms
