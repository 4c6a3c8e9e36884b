// qms_sample.cu - the chat path's token sampler on the device (the reference's sample(),
// src/chat.c:27-69), so a decode step hands back one token id instead of copying the whole
// logit row (151,936 floats for Qwen3) to the host.
//
// One cluster of 8 CTAs x 1024 threads, each CTA scanning an eighth of the row; histograms,
// counts and candidates meet in distributed shared memory:
//   greedy (temp <= 0): argmax, the first index among equal maxima (chat.c:38-40);
//   tempered: the K largest logits (K = top_k when 0 < top_k < V, else min(V, 1024)) by a
//   4-pass radix select on order-preserving 32-bit keys, the keys equal to the K-th taken in
//   index order; the K sorted by (value descending, index ascending), which is the order the
//   reference's insertion sort produces (chat.c:44-50); weights exp((l_j - l_0) / temp) in
//   double; the normalised cumulative sum, the top-p cut, one pcg32 draw and the pick run
//   sequentially on one thread in the reference's order (chat.c:51-66), with IEEE double
//   additions and divisions, so they round as the host's. exp() is CUDA's double exp (at most
//   1 ulp from the host's), which could move a pick only if a draw fell within ~1e-16 of a
//   cumulative boundary.
#include <cooperative_groups.h>

#include "qms_common.cuh"

namespace cg = cooperative_groups;

namespace qms {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;
constexpr int kSampleCtas = 8;             // one cluster shares the passes over the row

// float -> unsigned key with the same order (-0 and +0 equal, as in float comparisons)
__device__ __forceinline__ uint32_t sample_key(float f) {
    if (f == 0.0f) f = 0.0f;
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// PCG-XSH-RR step of the chat sampler's generator (chat.c:27-33)
__device__ __forceinline__ uint32_t sample_pcg32(uint64_t &s) {
    const uint64_t x = s;
    s = x * 6364136223846793005ull + 1442695040888963407ull;
    const uint32_t v = (uint32_t)(((x >> 18) ^ x) >> 27);
    const uint32_t r = (uint32_t)(x >> 59);
    return (v >> r) | (v << ((32u - r) & 31u));
}

// exclusive prefix over the 1024 threads of the CTA
__device__ __forceinline__ int block_exclusive_scan(int v, int *s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = s_warp[lane], wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        s_warp[lane] = wi - w;
    }
    __syncthreads();
    const int r = s_warp[warp] + inc - v;
    __syncthreads();                                       // s_warp reusable afterwards
    return r;
}

// One cluster of kSampleCtas CTAs; CTA r scans logits [r V / n, (r + 1) V / n). Every CTA takes
// the same cluster barriers in the same order; CTA 0 finishes the draw.
__global__ void __cluster_dims__(kSampleCtas, 1, 1) __launch_bounds__(kSampleThreads, 1)
    k_sample(const float *__restrict__ l, int V, float temp, float top_p, int K, uint64_t *rng, int *token) {
    __shared__ unsigned long long s_k[kSampleMaxK];       // CTA 0: (~key << 32) | index, sorted ascending
    __shared__ double s_w[kSampleMaxK];
    __shared__ double s_q[kSampleMaxK];                    // s_w / z
    __shared__ unsigned s_hist[256];                       // this CTA's slice
    __shared__ unsigned s_tot[256];                        // the cluster's
    __shared__ int s_warp[32];
    __shared__ float s_bv[32];
    __shared__ int s_bi[32];
    __shared__ float s_cbv[kSampleCtas];                   // CTA 0: each CTA's maximum and its index
    __shared__ int s_cbi[kSampleCtas];
    __shared__ int s_cnt[2];                               // this CTA's keys above / equal to T
    __shared__ unsigned s_digit, s_kk;
    __shared__ double s_z;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lo = (int)((long long)V * rank / kSampleCtas), hi = (int)((long long)V * (rank + 1) / kSampleCtas);
    cluster.sync();                                        // every CTA of the cluster runs before any remote access

    if (!(temp > 0.0f)) {                                  // greedy: first index of the maximum
        float bv = -INFINITY;
        int bi = V;
        for (int i = lo + tid; i < hi; i += kSampleThreads) {
            const float v = __ldg(l + i);
            if (bi == V || v > bv) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi < V && (bi == V || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            s_bv[warp] = bv;
            s_bi[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float v = s_bv[0];
            int b = s_bi[0];
            for (int w = 1; w < kSampleThreads / 32; w++)
                if (s_bi[w] < V && (b == V || s_bv[w] > v || (s_bv[w] == v && s_bi[w] < b))) {
                    v = s_bv[w];
                    b = s_bi[w];
                }
            *cluster.map_shared_rank(&s_cbv[rank], 0) = v;     // CTA 0's slots, one per CTA
            *cluster.map_shared_rank(&s_cbi[rank], 0) = b;
        }
        cluster.sync();
        if (rank == 0 && tid == 0) {
            float v = s_cbv[0];
            int b = s_cbi[0];
            for (int r = 1; r < kSampleCtas; r++)              // slices ascend, so ties keep the lower rank
                if (s_cbi[r] < V && (b == V || s_cbv[r] > v)) {
                    v = s_cbv[r];
                    b = s_cbi[r];
                }
            *token = b;
        }
        return;
    }

    // ---- radix select of the K-th largest key over the cluster, 8 bits per pass from the top
    uint32_t prefix = 0, pmask = 0;
    unsigned kk = (unsigned)K;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int j = tid; j < 256; j += kSampleThreads) s_hist[j] = 0;
        __syncthreads();
        for (int i = lo + tid; i < hi; i += kSampleThreads) {
            const uint32_t u = sample_key(__ldg(l + i));
            if ((u & pmask) == prefix) atomicAdd(&s_hist[(u >> shift) & 255u], 1u);
        }
        cluster.sync();                                    // every slice's histogram is complete
        if (tid < 256) {
            unsigned c = 0;
            for (int r = 0; r < kSampleCtas; r++) c += *cluster.map_shared_rank(&s_hist[tid], r);
            s_tot[tid] = c;
        }
        cluster.sync();                                    // every CTA has read them (before the next reset)
        if (tid == 0) {
            unsigned cum = 0;
            int d = 255;
            for (; d > 0; d--) {
                if (cum + s_tot[d] >= kk) break;
                cum += s_tot[d];
            }
            s_digit = (unsigned)d;
            s_kk = kk - cum;
        }
        __syncthreads();
        prefix |= s_digit << shift;
        pmask |= 255u << shift;
        kk = s_kk;
        __syncthreads();
    }
    const uint32_t T = prefix;                             // the K-th largest key
    const int need = (int)kk, ngt = K - need;              // keys == T to take, keys > T

    // ---- the K in index order into CTA 0: all keys above T, then the first `need` equal to T
    const int n = hi - lo, chunk = (n + kSampleThreads - 1) / kSampleThreads;
    const int i0 = lo + min(n, tid * chunk), i1 = lo + min(n, tid * chunk + chunk);
    int gt = 0, eq = 0;
    for (int i = i0; i < i1; i++) {
        const uint32_t u = sample_key(__ldg(l + i));
        gt += u > T;
        eq += u == T;
    }
    int pg = block_exclusive_scan(gt, s_warp);
    int pe = block_exclusive_scan(eq, s_warp);
    if (tid == kSampleThreads - 1) {
        s_cnt[0] = pg + gt;
        s_cnt[1] = pe + eq;
    }
    cluster.sync();                                        // every CTA's counts are published
    for (int r = 0; r < rank; r++) {                       // keys of the lower slices come first
        pg += *cluster.map_shared_rank(&s_cnt[0], r);
        pe += *cluster.map_shared_rank(&s_cnt[1], r);
    }
    unsigned long long *dk = cluster.map_shared_rank(s_k, 0);
    for (int i = i0; i < i1; i++) {
        const uint32_t u = sample_key(__ldg(l + i));
        if (u > T) {
            dk[pg++] = ((unsigned long long)(~u) << 32) | (unsigned)i;
        } else if (u == T) {
            if (pe < need) dk[ngt + pe] = ((unsigned long long)(~u) << 32) | (unsigned)i;
            pe++;
        }
    }
    cluster.sync();                                        // the candidates are in CTA 0
    if (rank != 0) return;
    for (int j = K + tid; j < kSampleMaxK; j += kSampleThreads) s_k[j] = ~0ull;
    __syncthreads();

    // ---- bitonic sort of the 1024 composite keys (ascending: value descending, index ascending)
    for (int size = 2; size <= kSampleMaxK; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int j = tid ^ stride;
            if (j > tid) {
                const unsigned long long a = s_k[tid], b = s_k[j];
                const bool up = (tid & size) == 0;
                if ((a > b) == up) {
                    s_k[tid] = b;
                    s_k[j] = a;
                }
            }
            __syncthreads();
        }
    }

    // ---- weights, then the reference's sequential sums on one thread
    const double l0 = (double)__ldg(l + (int)(s_k[0] & 0xFFFFFFFFu));
    if (tid < K) {
        const double d = __dsub_rn((double)__ldg(l + (int)(s_k[tid] & 0xFFFFFFFFu)), l0);
        s_w[tid] = exp(__ddiv_rn(d, (double)temp));
    }
    __syncthreads();
    if (tid == 0) {
        double z = 0.0;
        for (int j = 0; j < K; j++) z = __dadd_rn(z, s_w[j]);
        s_z = z;
    }
    __syncthreads();
    if (tid < K) s_q[tid] = __ddiv_rn(s_w[tid], s_z);       // IEEE division: the host's quotients
    __syncthreads();
    if (tid == 0) {
        int keep = K;
        double c = 0.0;
        for (int j = 0; j < K; j++) {
            c = __dadd_rn(c, s_q[j]);
            if (c >= (double)top_p) {
                keep = j + 1;
                break;
            }
        }
        double zk = 0.0;
        for (int j = 0; j < keep; j++) zk = __dadd_rn(zk, s_w[j]);
        uint64_t st = *rng;
        const double r = __dmul_rn((double)sample_pcg32(st) / 4294967296.0, zk);
        *rng = st;
        int pick = (int)(s_k[keep - 1] & 0xFFFFFFFFu);
        double acc = 0.0;
        for (int j = 0; j < keep; j++) {
            acc = __dadd_rn(acc, s_w[j]);
            if (r < acc) {
                pick = (int)(s_k[j] & 0xFFFFFFFFu);
                break;
            }
        }
        *token = pick;
    }
}

}  // namespace qms

extern "C" int qms_cuda_sample(const float *logits, int vocab, float temp, float top_p, int top_k, uint64_t *rng,
                               int *token, void *stream) {
    QMS_REQUIRE(logits && token && vocab > 0, QMS_CUDA_EINVAL, "sample: NULL logits or token, or vocab <= 0");
    const int K = (top_k > 0 && top_k < vocab) ? top_k : (vocab < qms::kSampleMaxK ? vocab : qms::kSampleMaxK);
    if (temp > 0.0f) {
        QMS_REQUIRE(rng, QMS_CUDA_EINVAL, "sample: NULL rng state with temp > 0");
        QMS_REQUIRE(K <= qms::kSampleMaxK, QMS_CUDA_EUNSUPPORTED,
                    "sample: top_k=%d exceeds the device sampler's %d candidates", top_k, qms::kSampleMaxK);
    }
    qms::k_sample<<<qms::kSampleCtas, qms::kSampleThreads, 0, (cudaStream_t)stream>>>(logits, vocab, temp, top_p, K, rng,
                                                                                     token);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}
