// qms_moe.cuh - internal declarations shared by the MoE sources (not part of the C ABI).
#pragma once

#include <string.h>

#include "qms_common.cuh"

namespace qms {

// ---- staged expert layouts ---------------------------------------------------------------------
// gate/up rows are repacked at load into "chunks" of 8 rows x SB blocks (SB = 16 or 8):
//   [8 rows][SB blocks][16 bytes]  nibble planes (block b of row rr at (rr*SB + b)*16)
//   [8 rows][SB blocks][2 bytes]   fp16 scales
// so a chunk is 8*SB*18 bytes, the same bytes as the 8*SB ggml blocks it holds. The gate/up rows
// of one expert form tiles of 32 f-values; a tile is nb/SB stages; a stage is 8 chunks: chunks 0-3
// hold gate rows f0..f0+31, chunks 4-7 the up rows of the same f (row r of the tile = 8*chunk +
// rr; r < 32 gate row f0+r, r >= 32 up row f0+r-32). One stage is one contiguous bulk copy.
struct Chunked {
    int SB;        // blocks per chunk row
    int S;         // chunks along one row (nb / SB)
    uint32_t GB;   // chunk bytes
};

__host__ __device__ inline Chunked make_chunked(int nb) {
    Chunked c;
    c.SB = nb % 16 == 0 ? 16 : 8;
    c.S = nb / c.SB;
    c.GB = (uint32_t)(8 * c.SB * 18);
    return c;
}

// chunk index of (gate/up row pair f, which) at block b, within one expert
__host__ __device__ inline size_t gu_chunk(const Chunked &c, int f, int which, int b) {
    const int t = f >> 5, r = which * 32 + (f & 31);
    return ((size_t)t * c.S + b / c.SB) * 8 + (r >> 3);
}

__host__ __device__ inline uint32_t chunk_nib_off(int SB, int rr, int bl) { return (uint32_t)(rr * SB + bl) * 16; }
__host__ __device__ inline uint32_t chunk_scale_off(int SB, int rr, int bl) {
    return (uint32_t)(8 * SB * 16 + (rr * SB + bl) * 2);
}

// down rows (E rows of nbF blocks, Q4_0 or Q4_1) are repacked into "column stages": for each
// block column b (32 values of the intermediate activation, i.e. one SwiGLU/Q8 group) the
// expert's rows are stored in Rq = E/RD stages of RD consecutive rows:
//   [RD rows][16 bytes] nibbles, [RD rows][2 bytes] fp16 d, (Q4_1 only) [RD rows][2 bytes] fp16 m
// Stage (b, q) sits at (b*Rq + q)*STD within the expert, so the down work of one Q8 group is Rq
// adjacent stages and a warp reading 32 consecutive rows of one block reads 512 contiguous bytes.
struct DnCols {
    int RD;        // rows per stage
    int Rq;        // stages per block column (E / RD)
    int q1;        // 1: Q4_1 blocks, 0: Q4_0
    uint32_t STD;  // stage bytes, RD * (20 or 18)
};

__host__ __device__ inline DnCols make_dncols(int E, int q1) {
    DnCols d;
    d.RD = E % 1024 == 0 ? 1024 : E % 512 == 0 ? 512 : 256;
    d.Rq = E / d.RD;
    d.q1 = q1;
    d.STD = (uint32_t)(d.RD * (q1 ? 20 : 18));
    return d;
}

// byte offset of stage (block column b, row i) and of row i's fields within it
__host__ __device__ inline size_t dn_stage_off(const DnCols &d, int b, int i) {
    return (size_t)(b * d.Rq + i / d.RD) * d.STD;
}
__host__ __device__ inline uint32_t dn_nib_off(const DnCols &d, int i) { return (uint32_t)(i % d.RD) * 16; }
__host__ __device__ inline uint32_t dn_scale_off(const DnCols &d, int i) { return (uint32_t)(d.RD * 16 + (i % d.RD) * 2); }
__host__ __device__ inline uint32_t dn_min_off(const DnCols &d, int i) { return (uint32_t)(d.RD * 18 + (i % d.RD) * 2); }

constexpr int kTopkInRouterMaxT = 4;   // above this, k_moe_topk runs one CTA per token

// ---- top-k of one token by a whole CTA (blockDim.x >= X, X <= 256) --------------------------
// The reference (src/model.c:1045-1064): prob[e] = exp((double)l_e - max) / z in double, then
// top-k by repeated strict-'>' argmax over prob, so ties (including probabilities that
// underflow to exactly 0) go to the lower expert index; weights (float)(p_j / sum_j p_j) with
// the sum taken in selection order. exp(l - max) / z is non-decreasing in l, so ranking the float
// logits (ties to the lower index) gives the same selection and order whenever the double
// probabilities of the top k+1 candidates are strictly decreasing; that is checked, and only if
// two of them tie does every thread fall back to ranking the doubles themselves. z is summed as a
// tree (the reference sums sequentially); the difference is ~1e-16 relative, below the float
// resolution of the weights. Writes sel[0..K) and wts[0..K); s_sel receives sel as well.
__device__ inline void topk_token(const float *__restrict__ lg, int X, int K, int *__restrict__ sel,
                                  float *__restrict__ wts, int *s_sel) {
    __shared__ double t_p[256];
    __shared__ __align__(16) float t_v[256];
    __shared__ double t_red[8];
    __shared__ double t_pj[64];
    __shared__ int t_cand[65];
    __shared__ int t_tie;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const float v = tid < X ? __ldcg(lg + tid) : -INFINITY;
    if (tid < X) t_v[tid] = v;
    if (tid == 0) t_tie = 0;
    float mx = warp_max(v);
    if (lane == 0) t_red[warp] = mx;
    __syncthreads();
    mx = (float)t_red[0];
    for (int i = 1; i < nw; i++) mx = fmaxf(mx, (float)t_red[i]);
    const double ex = tid < X ? exp((double)v - (double)mx) : 0.0;
    double z = ex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    __syncthreads();
    if (lane == 0) t_red[warp] = z;
    __syncthreads();
    z = 0.0;
    for (int i = 0; i < nw; i++) z += t_red[i];
    const double p = ex / z;
    if (tid < X) {
        t_p[tid] = p;
        int r0 = 0, r1 = 0, r2 = 0, r3 = 0;               // float rank, ties to the lower index
        const float4 *v4 = reinterpret_cast<const float4 *>(t_v);
        int j = 0;
#pragma unroll 8
        for (; j + 4 <= X; j += 4) {
            const float4 u = v4[j >> 2];
            r0 += (u.x > v) | ((u.x == v) & (j + 0 < tid));
            r1 += (u.y > v) | ((u.y == v) & (j + 1 < tid));
            r2 += (u.z > v) | ((u.z == v) & (j + 2 < tid));
            r3 += (u.w > v) | ((u.w == v) & (j + 3 < tid));
        }
        for (; j < X; j++) r0 += (t_v[j] > v) | ((t_v[j] == v) & (j < tid));
        const int rank = r0 + r1 + r2 + r3;
        if (rank <= K) t_cand[rank] = tid;
    }
    __syncthreads();
    const int nchk = K < X ? K : K - 1;                   // pairs (r, r+1) that decide the selection
    if (tid < nchk && !(t_p[t_cand[tid]] > t_p[t_cand[tid + 1]])) t_tie = 1;
    __syncthreads();
    if (!t_tie) {
        if (tid < K) {
            const int e = t_cand[tid];
            sel[tid] = e;
            s_sel[tid] = e;
            t_pj[tid] = t_p[e];
        }
    } else if (tid < X) {                                 // exact ranking of the doubles
        int rank = 0;
        for (int j = 0; j < tid; j++) rank += t_p[j] >= p;
        for (int j = tid + 1; j < X; j++) rank += t_p[j] > p;
        if (rank < K) {
            sel[rank] = tid;
            s_sel[rank] = tid;
            t_pj[rank] = p;
        }
    }
    __syncthreads();
    if (tid < K) {                                        // every thread sums in selection order
        double ws = 0.0;
        for (int j = 0; j < K; j++) ws += t_pj[j];
        wts[tid] = (float)(t_pj[tid] / ws);
    }
    __syncthreads();
}

}  // namespace qms

struct QmsCudaMoe {
    int device, nsm;
    int E, X, K, F, nbE, nbF;
    int n_local, expert_base;  // experts held: [expert_base, expert_base + n_local) of the X routed
    int gate_type, up_type, down_type;
    qms::Chunked cgu;    // gate/up chunks
    qms::DnCols dcol;    // down column stages
    float *router;       // [X][E] F32
    float *router_lm;    // [X][16][E/16]: element 16*i + k of a row at [k][i] (lane-major, batch-1 router)
    uint8_t *gu;         // [X] experts of staged gate/up chunks
    uint8_t *dn;         // [X] experts of down column stages
    size_t gu_expert, dn_expert, weight_bytes;
    int stream_ok;       // batch-1 streaming kernels usable for this shape
    int mma_min_t;       // T from which the grouped kernels run (0: never)
    int gemv;            // grouped GEMV (CUDA cores) for calls of few slots per expert
    // scratch, sized for cap_T tokens and for expert calls of cap_rows slots
    int cap_T;
    int cap_rows;
    void *scratch;
    size_t scratch_bytes;
    int8_t *xq_q;
    float *xq_d;
    int *xq_s;
    float *logits;
    int *sel;
    float *wts;
    float *act;
    int8_t *aq_q;
    float *aq_d;
    int *aq_s;
    int *cnt;            // [0]: router arrivals; [1 + slot*nbF + g]: gate/up group arrivals
    int *err;            // device error flags (bounded waits that gave up)
    int *err_ext;        // when set (a model owns the layer): the flag word to use instead of the scratch one
    // batch-1 kernel exchange buffers, in flagged words (data | call stamp << 32)
    unsigned long long *lg_flagged;          // [copies][X] router logits
    unsigned long long *aq_flagged;          // [K*F/32 groups][10]: 8 words of q, d, sum
    unsigned long long *part_gu;             // [tile][segments][64] partial gate/up sums of split tiles
    unsigned long long *fin;                 // [nsm * E] per-CTA partial outputs
    unsigned *stamps;                        // [nsm] per-CTA call stamps
    int nst;                    // ring depth (slots) of the batch-1 kernel
    // host-buffer entry point
    cudaStream_t hstream;
    float *d_in, *d_out;
    int io_cap_T;
    // optional per-kernel timing events (qms_cuda_moe_set_kernel_events)
    cudaEvent_t ev[6];
    int timing;
};

namespace qms {

template <typename... P, typename... A>
static cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, ((P)args)...);
}

// A grid whose CTAs wait for one another is safe only if all of it is resident at once: `grid`
// CTAs against `per_sm` resident CTAs per SM on `nsm` SMs.
inline bool persistent_grid_fits(int per_sm, int nsm, int grid) {
    return per_sm >= 1 && nsm >= 1 && (long long)per_sm * nsm >= grid;
}

// batch-1 decode kernels (qms_moe_stream.cu)
int stream_prepare(QmsCudaMoe *m);     // shape check + kernel attributes; sets m->stream_ok
int stream_forward_bs1(QmsCudaMoe *m, const float *xn, float *out, const float *resid, cudaStream_t s,
                       const float *nw = nullptr, float eps = 0.0f);
// One token through the layer with its input RMS-normed inside the batch-1 kernel:
// out = resid + moe(RMSNorm(h) * nw). Returns QMS_CUDA_EUNSUPPORTED when the batch-1 kernel does
// not serve this layer (the caller then normalises separately).
int moe_forward_normed_bs1(QmsCudaMoe *m, const float *h, const float *nw, float eps, float *out,
                           const float *resid, int *sel, cudaStream_t s);
struct StreamScratch {                 // bytes of the batch-1 kernel's exchange buffers
    size_t lg_flagged, stamps, aq_flagged, part_gu, fin;
};
int stream_scratch_sizes(const QmsCudaMoe *m, StreamScratch *sz);

// batched tensor-core kernels (qms_moe_mma.cu), T >= mma_min_t
int mma_supported(const QmsCudaMoe *m);
int mma_prepare(QmsCudaMoe *m);
int mma_reserve(QmsCudaMoe *m, int T);
int mma_forward(QmsCudaMoe *m, int T, const float *resid, float *out, cudaStream_t s);
int mma_experts(QmsCudaMoe *m, int S, const int *expert, float *dn, cudaStream_t s);
int mma_combine(const float *dn, const float *wts, int T, int K, int E, const float *resid, float *out,
                cudaStream_t s);

// Slots grouped by expert (k_mma_group): per expert its count, first position and first tile;
// the tile list (expert | tile index << 16) and the slot ids in expert order.
struct MmaWork {
    int *cnt, *off, *toff, *ntiles, *pos, *slots, *tiles;
    int8_t *bg;        // [tiles][nb][2048] tensor-core B operands
    float *bs;         // [tiles][nb][64] activation scales
    int *bsum;         // [tiles][nb][64] activation block sums (Q4_1 down)
    float *dn;         // [T*K][E] down rows per slot
    float *dn2;        // [min(T*K, 24 X)][E] second K half of the grouped GEMV's down rows
};

// batched expert-grouped GEMV kernels (qms_moe_gemv.cu), the grouped path when experts average
// <= 24 slots per call (16-slot tiles)
int gv_supported(const QmsCudaMoe *m);
int gv_prepare(QmsCudaMoe *m);
int gv_gemms(QmsCudaMoe *m, const MmaWork &w, int maxT, int S, int nx, int rdiv, float *dn, float *dn2,
             bool sum_halves, cudaStream_t s);

}  // namespace qms
