// qms_ep.cu - expert-parallel dispatch and combine on the device, with fixed-capacity buffers.
//
// Rank r of N holds experts [r * X/N, (r+1) * X/N). A layer call sends every (token, slot) row to
// the rank owning the slot's expert and brings the down rows back. Here both directions move
// fixed-size segments: rank r's send buffer holds N segments of `cap` rows, segment o for owner o,
// each slot at its rank (in slot order) among the slots of the same owner. Nothing about the
// routing has to reach the host, so the exchange is a plain fixed-size all-to-all (NCCL
// grouped send/recv from C, or all_to_all_single), and the whole layer can run in a CUDA graph.
//   k_ep_index     one CTA: owner and segment index of every slot (a stable counting sort),
//                  the local expert id of every used entry, -1 in every unused one
//   k_ep_pack      one CTA per token: its row quantised once (the reference's quantiser,
//                  src/kernels.c:34-53, QmsQ8 blocks of src/kernels.h:7-12), written to each
//                  of its slots' entries
//   k_ep_combine   out[t] = resid[t] + sum_j wts[t][j] * ret[slot[t*K + j]] in selection order
//                  (src/model.c:1152-1162), the arithmetic of the unsharded grouped path
#include <limits.h>

#include "qms_common.cuh"

namespace qms {

constexpr int kEpMaxRanks = 64;
constexpr int kEpIndexThreads = 1024;

// Slots i = t * K + j in chunks of 1024 (one per thread). Within a warp, lanes with the same owner
// find each other with __match_any_sync; the per-warp counts of a chunk, summed over the warps
// before this one and added to the owner's running base, give the slot's index in its segment.
// So the order inside a segment is slot order, whatever the chunking.
__global__ void __launch_bounds__(kEpIndexThreads) k_ep_index(const int *__restrict__ sel, int S, int n_expert,
                                                              int n_rank, int cap, int *__restrict__ slot,
                                                              int *__restrict__ send_e, int *err) {
    __shared__ int wcnt[kEpIndexThreads / 32][kEpMaxRanks];
    __shared__ int base[kEpMaxRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = n_expert / n_rank;
    if (tid < n_rank) base[tid] = 0;
    __syncthreads();
    bool bad = false;
    for (int c0 = 0; c0 < S; c0 += kEpIndexThreads) {
        for (int j = tid; j < (kEpIndexThreads / 32) * kEpMaxRanks; j += kEpIndexThreads)
            wcnt[j / kEpMaxRanks][j % kEpMaxRanks] = 0;
        __syncthreads();
        const int i = c0 + tid;
        int e = -1, o = -1;
        if (i < S) {
            e = sel[i];
            if (e >= 0 && e < n_expert) o = e / per;
            else bad = true;
        }
        const unsigned same = __match_any_sync(0xffffffffu, o);
        const int before = __popc(same & ((1u << lane) - 1u));
        if (o >= 0 && before == 0) wcnt[warp][o] = __popc(same);
        __syncthreads();
        if (o >= 0) {
            int p = base[o] + before;
            for (int w = 0; w < warp; w++) p += wcnt[w][o];
            if (p < cap) {
                slot[i] = o * cap + p;
                send_e[(size_t)o * cap + p] = e - o * per;
            } else {
                slot[i] = -1;                          // past the segment's capacity: dropped, flagged
                bad = true;
            }
        } else if (i < S) {
            slot[i] = -1;
        }
        __syncthreads();
        if (tid < n_rank) {
            int t = 0;
            for (int w = 0; w < kEpIndexThreads / 32; w++) t += wcnt[w][tid];
            base[tid] += t;
        }
        __syncthreads();
    }
    for (int r = 0; r < n_rank; r++)
        for (int j = min(base[r], cap) + tid; j < cap; j += kEpIndexThreads) send_e[(size_t)r * cap + j] = -1;
    if (__syncthreads_or(bad) && tid == 0 && err) atomicOr(err, 1);
}

// One CTA per token, a warp per 32-block: quantise once, then write the block into every entry
// the token's K slots were given (k_ep_index ran before on the same stream).
__global__ void __launch_bounds__(256) k_ep_pack(const float *__restrict__ xn, const int *__restrict__ slot, int K,
                                                 int nb, QmsQ8 *__restrict__ send_x) {
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int b = warp; b < nb; b += nw) {
        const Q8Lane r = quantize_lane(xn[((size_t)t * nb + b) * 32 + lane]);
        for (int j = 0; j < K; j++) {
            const int s = __ldg(slot + (size_t)t * K + j);
            if (s < 0) continue;
            QmsQ8 *o = send_x + (size_t)s * nb + b;
            o->q[lane] = (int8_t)r.q;
            if (lane == 0) {
                o->d = r.d;
                o->ds = __fmul_rn(r.d, (float)r.sum);
                o->s16[0] = (int16_t)r.sum_lo;
                o->s16[1] = (int16_t)(r.sum - r.sum_lo);
            }
        }
    }
}

// The fixed-order FMA chain of the unsharded combine, reading each slot's down row where the
// exchange put it. A dropped slot (-1) contributes NaN, so an overflowed call cannot pass as valid.
__global__ void __launch_bounds__(256) k_ep_combine(const float *__restrict__ ret, const int *__restrict__ slot,
                                                    const float *__restrict__ wts, int K, int E,
                                                    const float *resid, float *out) {
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= E) return;
    float o = 0.0f;
    for (int j = 0; j < K; j++) {
        const int s = __ldg(slot + (size_t)t * K + j);
        const float d = s >= 0 ? __ldcg(ret + (size_t)s * E + i) : __int_as_float(0x7fc00000);
        o = __fmaf_rn(__ldcg(wts + (size_t)t * K + j), d, o);
    }
    if (resid) o = __fadd_rn(resid[(size_t)t * E + i], o);
    out[(size_t)t * E + i] = o;
}

}  // namespace qms

using namespace qms;

extern "C" {

int qms_cuda_ep_pack(const float *xn, const int *sel, int T, int n_used, int n_embd, int n_expert, int n_rank,
                     int cap, QmsQ8 *send_x, int *send_e, int *slot, int *err, void *stream) {
    QMS_REQUIRE(T >= 0 && n_used >= 1 && n_embd > 0 && n_embd % 32 == 0 && n_expert >= 1 && cap >= 1,
                QMS_CUDA_EINVAL, "ep_pack: bad shape (T %d, n_used %d, n_embd %d, n_expert %d, cap %d)", T, n_used,
                n_embd, n_expert, cap);
    QMS_REQUIRE(n_rank >= 1 && n_rank <= kEpMaxRanks && n_expert % n_rank == 0, QMS_CUDA_EUNSUPPORTED,
                "ep_pack: %d experts over %d ranks (1..%d ranks, an even split)", n_expert, n_rank, kEpMaxRanks);
    QMS_REQUIRE((int64_t)T * n_used <= INT_MAX && (int64_t)n_rank * cap <= INT_MAX, QMS_CUDA_EINVAL,
                "ep_pack: %d x %d slots or %d x %d entries overflow an int", T, n_used, n_rank, cap);
    QMS_REQUIRE(send_x && send_e && (T == 0 || (xn && sel && slot)), QMS_CUDA_EINVAL,
                "ep_pack: NULL xn, sel, send_x, send_e or slot");
    QMS_REQUIRE(((uintptr_t)send_x & 3) == 0 && ((uintptr_t)send_e & 3) == 0, QMS_CUDA_EINVAL,
                "ep_pack: send_x and send_e must be 4-byte aligned");
    const cudaStream_t s = (cudaStream_t)stream;
    k_ep_index<<<1, kEpIndexThreads, 0, s>>>(sel, T * n_used, n_expert, n_rank, cap, slot, send_e, err);
    QMS_CK(cudaGetLastError());
    if (T == 0) return QMS_CUDA_OK;
    k_ep_pack<<<T, 256, 0, s>>>(xn, slot, n_used, n_embd / 32, send_x);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

int qms_cuda_ep_combine(const float *ret, const int *slot, const float *wts, int T, int n_used, int n_embd,
                        const float *resid, float *out, void *stream) {
    QMS_REQUIRE(T >= 0 && T <= 65535 && n_used >= 1 && n_embd > 0, QMS_CUDA_EINVAL,
                "ep_combine: bad shape (T %d, n_used %d, n_embd %d)", T, n_used, n_embd);
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE(ret && slot && wts && out, QMS_CUDA_EINVAL, "ep_combine: NULL ret, slot, wts or out");
    k_ep_combine<<<dim3((n_embd + 255) / 256, T), 256, 0, (cudaStream_t)stream>>>(ret, slot, wts, n_used, n_embd,
                                                                                  resid, out);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

}  // extern "C"
