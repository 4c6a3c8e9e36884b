// qms_model.cu - a whole Qwen3-MoE model resident in HBM and its token step on B200 (sm_100a):
// the device counterpart of qms_model_load / qms_forward (reference src/model.c:314-387, 1252-1296).
//
// One forward over T tokens at positions pos..pos+T-1 launches, on one stream:
//   k_embed                                   embedding rows (src/model.c:1273)
//   per layer:
//     QKV projection   T == 1: k_gemv with RMSNorm(attn_norm) + Q8 in its prologue
//                      T > 1 : k_rmsnorm (-> Q8 rows) + k_gemv over tiles of 8 tokens
//     k_qk_rope        QK-norm, NEOX RoPE, fp32 K/V append (src/model.c:436-462)
//     k_attention      causal GQA (src/model.c:465-492)
//     O projection     k_gemv (+ residual into h in place, src/model.c:1282)
//     k_rmsnorm        ffn_norm (src/model.c:1283)
//     MoE block        qms_cuda_moe_forward with the residual fused (src/model.c:1284-1285)
//   final RMSNorm + head   k_gemv over the output rows (src/model.c:1288-1292); the greedy decode
//                          step also takes the argmax in the same kernel and advances the position
// Every kernel is launched with programmatic dependent launch; weights are the only memory read
// before griddepcontrol.wait. Positions are read from device memory, so a captured decode step can
// be replayed as the sequence grows. Long prompts run in chunks of up to kChunk tokens; every
// token's arithmetic is the same whatever the chunking (attention reads earlier tokens from the
// KV cache), so chunking changes no result of the reference's formulas.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "qms_moe.cuh"
#include "qms_trunk.cuh"

using namespace qms;

namespace qms {
constexpr int kChunk = 256;          // tokens per forward pass over the layers (prefill)
constexpr int kSplit = kAttnBlock;   // positions per attention CTA in one-token steps

struct DevLayer {
    float *norms = nullptr;          // attn_norm [E], ffn_norm [E], q_norm [D], k_norm [D]
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    int qkv_type = 0, o_type = 0;
    uint8_t *wqkv = nullptr, *wo = nullptr;
    QmsCudaMoe *moe = nullptr;
    bool set = false;
};
}  // namespace qms

struct QmsCudaModel {
    int device, nsm;
    int L, E, H, Hk, D, X, K, F, V, ctx;
    float eps;
    double rope_base;
    int QD, KD, NQKV, group;
    int embd_type;
    uint8_t *embd;                   // GGUF rows
    float *out_norm;
    int head_type;
    uint8_t *head;                   // repacked rows
    float *rope_cos, *rope_sin;      // [ctx][D/2]
    void *kc, *vc;                   // [n_seq][L][ctx][KD] elements of kv_es bytes
    int kv_type;                     // QMS_T_F32 (the reference's cache) or QMS_T_F16 (compacted)
    size_t kv_es;
    int n_seq;                       // sequences with a KV cache of ctx positions each
    float *bpart_o;                  // batched one-token attention partials (set_sequences)
    double *bpart_ml;
    size_t seq_stride;               // floats between two sequences' caches (L * ctx * KD)
    std::vector<DevLayer> layers;
    // forward scratch for cap_T tokens
    int cap_T;
    void *scratch;
    size_t scratch_bytes;
    float *h, *xn, *qkv, *att, *logits;
    int8_t *xq;
    float *xd;
    int *xs;
    int *ids, *pos, *sel;
    int *pos_vec;                    // [cap_T] positions of a batched host call
    float *kpart;                    // partial sums of split multi-token projections
    size_t kpart_n;
    float *part_o;
    double *part_ml;
    int *amax_ticket, *err;
    unsigned long long *amax;
    int max_splits;
    int *h_pinned;                   // host mirror of ids + pos for the host entry point
    int *flags;                      // device [1 + L]: the trunk's error word, then each MoE layer's
    int *h_flags;                    // pinned host mirror of flags, read once per host call
    cudaStream_t stream;
    size_t weight_bytes;
    // QMS_PROF sections
    int prof;
    double prof_ms[7];
    std::vector<cudaEvent_t> ev;
};

namespace qms {

static int ensure_dev(int dev) {
    int cur = -1;
    QMS_CK(cudaGetDevice(&cur));
    if (cur != dev) QMS_CK(cudaSetDevice(dev));
    return QMS_CUDA_OK;
}

static size_t al256m(size_t x) { return (x + 255) & ~(size_t)255; }

// cudaMalloc with the failure as a status
static int dmalloc(void **p, size_t n, const char *what) {
    *p = nullptr;
    if (n == 0) return QMS_CUDA_OK;
    if (cudaMalloc(p, n) != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        set_error("model: cannot allocate %.3f GB for %s", n / 1e9, what);
        return QMS_CUDA_ENOMEM;
    }
    return QMS_CUDA_OK;
}

// copy `n` bytes of a host or device source into device memory
static int to_device(void *dst, const void *src, size_t n, int src_on_device) {
    QMS_CK(cudaMemcpy(dst, src, n, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    return QMS_CUDA_OK;
}

// Repack `rows` GGUF rows (host or device source; several sources concatenated) into dst.
static int upload_rows(int type, const void *const *srcs, const int64_t *rows, int nsrc, int ncol, int on_dev,
                       uint8_t *dst) {
    const size_t rb = ggml_row_bytes(type, ncol);
    int64_t total = 0;
    for (int i = 0; i < nsrc; i++) total += rows[i];
    void *stage = nullptr;
    int rc = dmalloc(&stage, (size_t)total * rb, "a staging buffer");
    if (rc) return rc;
    size_t off = 0;
    for (int i = 0; i < nsrc && rc == QMS_CUDA_OK; i++) {
        rc = to_device((uint8_t *)stage + off, srcs[i], (size_t)rows[i] * rb, on_dev);
        off += (size_t)rows[i] * rb;
    }
    if (rc == QMS_CUDA_OK) rc = repack_rows(type, (const uint8_t *)stage, total, ncol, dst, 0);
    if (rc == QMS_CUDA_OK && cudaDeviceSynchronize() != cudaSuccess) {
        set_error("model: repack failed: %s", cudaGetErrorString(cudaGetLastError()));
        rc = QMS_CUDA_ECUDA;
    }
    cudaFree(stage);
    return rc;
}

static bool gemv_cols_ok(int ncol, int type) {
    if (type == QMS_T_Q6_K) {
        const int u = ncol / 128;
        return ncol % 256 == 0 && u <= 32 && (u & (u - 1)) == 0;
    }
    const int nb = ncol / 32;
    return ncol % 32 == 0 && nb >= 1 && (nb < 32 ? (nb & (nb - 1)) == 0 : nb % 32 == 0 && nb <= 256 &&
                                                                              (nb / 32 & (nb / 32 - 1)) == 0);
}

static int model_reserve(QmsCudaModel *m, int T) {
    if (T <= m->cap_T) return QMS_CUDA_OK;
    const size_t wq = (size_t)std::max(m->E, m->QD);
    size_t off = 0;
    auto take = [&](size_t n) { const size_t o = off; off += al256m(n); return o; };
    const size_t o_h = take((size_t)T * m->E * 4), o_xn = take((size_t)T * m->E * 4);
    const size_t o_qkv = take((size_t)T * m->NQKV * 4), o_att = take((size_t)T * m->QD * 4);
    const size_t o_lg = take((size_t)T * m->V * 4);
    const size_t o_xq = take((size_t)T * wq), o_xd = take((size_t)T * wq / 32 * 4), o_xs = take((size_t)T * wq / 32 * 4);
    const size_t o_ids = take((size_t)T * 4), o_pos = take(4), o_posv = take((size_t)T * 4);
    const size_t o_sel = take((size_t)m->L * T * m->K * 4);
    const size_t o_po = take((size_t)m->H * m->max_splits * m->D * 4), o_pml = take((size_t)m->H * m->max_splits * 16);
    const size_t o_at = take(4), o_amax = take(8);
    const size_t kpart_n = (size_t)4 * 64 * std::max(m->NQKV, m->E), o_kp = take(kpart_n * 4);
    void *p = nullptr;
    int rc = dmalloc(&p, off, "forward scratch");
    if (rc) return rc;
    if (cudaMemset(p, 0, off) != cudaSuccess) {
        cudaFree(p);
        set_error("model: memset failed");
        return QMS_CUDA_ECUDA;
    }
    int *hp = nullptr;
    if (cudaMallocHost(&hp, (size_t)(2 * T + 1) * 4) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        set_error("model: cannot allocate pinned host memory");
        return QMS_CUDA_ENOMEM;
    }
    if (m->scratch) {
        QMS_CK(cudaDeviceSynchronize());
        cudaFree(m->scratch);
    }
    if (m->h_pinned) cudaFreeHost(m->h_pinned);
    m->h_pinned = hp;
    char *b = (char *)p;
    m->scratch = p;
    m->scratch_bytes = off;
    m->h = (float *)(b + o_h);
    m->xn = (float *)(b + o_xn);
    m->qkv = (float *)(b + o_qkv);
    m->att = (float *)(b + o_att);
    m->logits = (float *)(b + o_lg);
    m->xq = (int8_t *)(b + o_xq);
    m->xd = (float *)(b + o_xd);
    m->xs = (int *)(b + o_xs);
    m->ids = (int *)(b + o_ids);
    m->pos = (int *)(b + o_pos);
    m->pos_vec = (int *)(b + o_posv);
    m->kpart = (float *)(b + o_kp);
    m->kpart_n = kpart_n;
    m->sel = (int *)(b + o_sel);
    m->part_o = (float *)(b + o_po);
    m->part_ml = (double *)(b + o_pml);
    m->amax_ticket = (int *)(b + o_at);
    m->err = m->flags;
    m->amax = (unsigned long long *)(b + o_amax);
    m->cap_T = T;
    for (auto &L : m->layers)
        if (L.moe && (rc = qms_cuda_moe_reserve(L.moe, T))) return rc;
    return QMS_CUDA_OK;
}

static int layers_ready(const QmsCudaModel *m) {
    for (int l = 0; l < m->L; l++)
        QMS_REQUIRE(m->layers[l].set, QMS_CUDA_EINVAL, "forward: layer %d was never set", l);
    return QMS_CUDA_OK;
}

static int prof_mark(QmsCudaModel *m, size_t i, cudaStream_t s) {
    if (!m->prof) return QMS_CUDA_OK;
    QMS_CK(cudaEventRecord(m->ev[i], s));
    return QMS_CUDA_OK;
}

// One pass over the layers for T <= cap_T tokens. ids, pos: device. logits: device
// [all ? T : 1][V]. tok != NULL: fused greedy argmax (T == 1) into *tok, and *pos advances.
// A projection of several tokens' Q8 rows: Q4 / Q6_K weights on the mma.sync kernels, others on the GEMV.
static int launch_proj(int type, const GemvArgs &g, cudaStream_t s) {
    const bool q4 = type == QMS_T_Q4_0 || type == QMS_T_Q4_1, q6 = type == QMS_T_Q6_K && g.ncol % 256 == 0;
    if ((q4 || q6) && g.rows % 16 == 0 && g.x == nullptr && g.amax == nullptr) return launch_gemm_q(type, g, s);
    return launch_gemv(type, g, s);
}

// One pass over the layers for T tokens. Single sequence `seq`: tokens at *pos + t. Batch
// (pos_vec != NULL): token t is sequence t at position pos_vec[t]. tok != NULL: greedy argmax of
// the head into tok (T == 1 fused into the head; batch per row) and pos_adv += 1.
static int forward_core(QmsCudaModel *m, const int *ids, int T, const int *pos, float *logits, int all, int *sel,
                        int *tok, int *pos_adv, cudaStream_t s, int seq = 0, const int *pos_vec = nullptr) {
    int rc;
    const int E = m->E;
    size_t ei = 0;
    if ((rc = prof_mark(m, ei++, s))) return rc;
    if ((rc = launch_embed(m->embd_type, m->embd, m->V, E, ids, T, m->h, m->err, s))) return rc;
    AttnArgs at;
    memset(&at, 0, sizeof at);
    at.qkv = m->qkv;
    at.ldq = m->NQKV;
    at.eps = m->eps;
    at.rope_cos = m->rope_cos;
    at.rope_sin = m->rope_sin;
    at.pos = pos;
    at.pos_vec = pos_vec;
    at.seq_stride = m->seq_stride;
    at.T = T;
    at.ctx = m->ctx;
    at.H = m->H;
    at.Hk = m->Hk;
    at.D = m->D;
    at.scale = 1.0 / sqrt((double)m->D);
    at.max_splits = m->max_splits;
    at.part_o = m->part_o;
    at.part_ml = m->part_ml;
    at.out = m->att;
    at.err = m->err;
    for (int l = 0; l < m->L; l++) {
        const DevLayer &L = m->layers[l];
        at.q_norm = L.q_norm;
        at.k_norm = L.k_norm;
        const size_t kvo = m->kv_es * ((size_t)seq * m->seq_stride + (size_t)l * m->ctx * m->KD);
        at.kc = static_cast<char *>(m->kc) + kvo;
        at.vc = static_cast<char *>(m->vc) + kvo;
        at.kv16 = m->kv_type == QMS_T_F16;
        int *sel_l = sel ? sel + (size_t)l * T * m->K : nullptr;
        GemvArgs g;
        memset(&g, 0, sizeof g);
        const bool one = T == 1 && !pos_vec;
        if (one) {
            // one token: streaming projections, fused attention, RMSNorm inside the MoE kernel
            g.w = L.wqkv;
            g.stride = rows_stride(L.qkv_type, E);
            g.rows = m->NQKV;
            g.ncol = E;
            g.T = 1;
            g.x = m->h;
            g.nw = L.attn_norm;
            g.eps = m->eps;
            g.y = m->qkv;
            if ((rc = launch_gemv1(L.qkv_type, g, m->err, s))) return rc;
            if ((rc = prof_mark(m, ei++, s))) return rc;
            if ((rc = launch_attn_decode(at, m->xq, m->xd, m->xs, s))) return rc;
            if ((rc = prof_mark(m, ei++, s))) return rc;
            memset(&g, 0, sizeof g);
            g.w = L.wo;
            g.stride = rows_stride(L.o_type, m->QD);
            g.rows = E;
            g.ncol = m->QD;
            g.T = 1;
            g.xq = m->xq;
            g.xd = m->xd;
            g.xs = m->xs;
            g.y = m->h;
            g.resid = m->h;
            if ((rc = launch_gemv1(L.o_type, g, m->err, s))) return rc;
            if ((rc = prof_mark(m, ei++, s))) return rc;
        }
        if (one) {
            rc = moe_forward_normed_bs1(L.moe, m->h, L.ffn_norm, m->eps, m->h, m->h, sel_l, s);
            if (rc == QMS_CUDA_EUNSUPPORTED) {
                clear_error();
                if ((rc = launch_rmsnorm(m->h, L.ffn_norm, m->eps, 1, E, m->xn, nullptr, nullptr, nullptr, s))) return rc;
                rc = qms_cuda_moe_forward(L.moe, m->xn, 1, m->h, sel_l, nullptr, nullptr, m->h, s);
            }
            if (rc) return rc;
            if ((rc = prof_mark(m, ei++, s))) return rc;
            continue;
        }
        // several tokens: RMSNorm(attn_norm) -> Q8 rows -> QKV
        g.w = L.wqkv;
        g.stride = rows_stride(L.qkv_type, E);
        g.rows = m->NQKV;
        g.ncol = E;
        g.T = T;
        g.eps = m->eps;
        g.y = m->qkv;
        g.ldy = m->NQKV;
        if ((rc = launch_rmsnorm(m->h, L.attn_norm, m->eps, T, E, nullptr, m->xq, m->xd, m->xs, s))) return rc;
        g.xq = m->xq;
        g.xd = m->xd;
        g.xs = m->xs;
        g.kpart = m->kpart;
        g.kpart_n = m->kpart_n;
        if ((rc = launch_proj(L.qkv_type, g, s))) return rc;
        if ((rc = prof_mark(m, ei++, s))) return rc;
        if (pos_vec) {                  // one token per sequence: the decode kernels, Q8 rows out
            AttnArgs ab = at;
            if (m->bpart_o) {           // else one sequence: the scratch's partials cover it
                ab.part_o = m->bpart_o;
                ab.part_ml = m->bpart_ml;
            }
            // QK-norm, RoPE and the K / V appends once per head row, not in every position block
            if ((rc = launch_qk_rope(at, s))) return rc;
            ab.q_ready = 1;
            if ((rc = launch_attn_decode(ab, m->xq, m->xd, m->xs, s))) return rc;
        } else {
            if ((rc = launch_qk_rope(at, s))) return rc;
            if ((rc = launch_attention(at, s))) return rc;
        }
        if ((rc = prof_mark(m, ei++, s))) return rc;
        // O projection + residual (h += O att)
        memset(&g, 0, sizeof g);
        g.w = L.wo;
        g.stride = rows_stride(L.o_type, m->QD);
        g.rows = E;
        g.ncol = m->QD;
        g.T = T;
        g.y = m->h;
        g.ldy = E;
        g.resid = m->h;
        if (!pos_vec && (rc = launch_rmsnorm(m->att, nullptr, 0.0f, T, m->QD, nullptr, m->xq, m->xd, m->xs, s)))
            return rc;
        g.xq = m->xq;
        g.xd = m->xd;
        g.xs = m->xs;
        g.kpart = m->kpart;
        g.kpart_n = m->kpart_n;
        if ((rc = launch_proj(L.o_type, g, s))) return rc;
        if ((rc = prof_mark(m, ei++, s))) return rc;
        // MoE block + residual
        if ((rc = launch_rmsnorm(m->h, L.ffn_norm, m->eps, T, E, m->xn, nullptr, nullptr, nullptr, s))) return rc;
        if ((rc = qms_cuda_moe_forward(L.moe, m->xn, T, m->h, sel_l, nullptr, nullptr, m->h, s))) return rc;
        if ((rc = prof_mark(m, ei++, s))) return rc;
    }
    // final norm + head: the last token, or all of them
    GemvArgs g;
    memset(&g, 0, sizeof g);
    g.w = m->head;
    g.stride = rows_stride(m->head_type, E);
    g.rows = m->V;
    g.ncol = E;
    g.eps = m->eps;
    g.y = logits;
    g.ldy = m->V;
    const int nT = all || pos_vec ? T : 1;
    g.T = nT;
    if (tok && !pos_vec) {
        g.amax = m->amax;
        g.ticket = m->amax_ticket;
        g.tok = tok;
        g.pos = pos_adv;
    }
    if (nT == 1 && !pos_vec) {
        g.x = m->h + (size_t)(T - 1) * E;
        g.ldx = E;
        g.nw = m->out_norm;
        if ((rc = launch_gemv1(m->head_type, g, m->err, s))) return rc;
    } else {
        if ((rc = launch_rmsnorm(m->h, m->out_norm, m->eps, nT, E, nullptr, m->xq, m->xd, m->xs, s))) return rc;
        g.xq = m->xq;
        g.xd = m->xd;
        g.xs = m->xs;
        if ((rc = launch_proj(m->head_type, g, s))) return rc;
        if (tok && pos_vec && (rc = launch_argmax_rows(logits, m->V, T, m->V, tok, pos_adv, s))) return rc;
    }
    if ((rc = prof_mark(m, ei++, s))) return rc;
    return QMS_CUDA_OK;
}

// The section timers' events, created when profiling is switched on.
static int prof_events(QmsCudaModel *m) {
    if (m->prof && m->ev.size() < (size_t)4 * m->L + 2) {
        for (size_t i = m->ev.size(); i < (size_t)4 * m->L + 2; i++) {
            cudaEvent_t e;
            QMS_CK(cudaEventCreate(&e));
            m->ev.push_back(e);
        }
    }
    return QMS_CUDA_OK;
}

// Sum the recorded sections into prof_ms (after the stream has finished).
static int prof_collect(QmsCudaModel *m) {
    if (!m->prof) return QMS_CUDA_OK;
    float ms = 0.0f;
    size_t e = 0;
    for (int l = 0; l < m->L; l++, e += 4) {
        const int sec[4] = {0, 1, 2, 5};            // qkv, attn, o_proj, moe
        for (int k = 0; k < 4; k++) {
            QMS_CK(cudaEventElapsedTime(&ms, m->ev[e + k], m->ev[e + k + 1]));
            m->prof_ms[sec[k]] += ms;
        }
    }
    QMS_CK(cudaEventElapsedTime(&ms, m->ev[e], m->ev[e + 1]));
    m->prof_ms[6] += ms;
    return QMS_CUDA_OK;
}

}  // namespace qms

extern "C" {

void qms_cuda_model_free(QmsCudaModel *m) {
    if (!m) return;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(m->device);
    cudaDeviceSynchronize();
    for (auto &L : m->layers) {
        cudaFree(L.norms);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
        qms_cuda_moe_destroy(L.moe);
    }
    cudaFree(m->embd);
    cudaFree(m->out_norm);
    cudaFree(m->head);
    cudaFree(m->rope_cos);
    cudaFree(m->rope_sin);
    cudaFree(m->kc);
    cudaFree(m->vc);
    cudaFree(m->scratch);
    if (m->h_pinned) cudaFreeHost(m->h_pinned);
    cudaFree(m->flags);
    cudaFree(m->bpart_o);
    cudaFree(m->bpart_ml);
    if (m->h_flags) cudaFreeHost(m->h_flags);
    for (cudaEvent_t e : m->ev) cudaEventDestroy(e);
    if (m->stream) cudaStreamDestroy(m->stream);
    if (cur >= 0) cudaSetDevice(cur);
    delete m;
}

int qms_cuda_model_create(const QmsCudaModelDesc *d, QmsCudaModel **out) {
    clear_error();
    QMS_REQUIRE(d && out, QMS_CUDA_EINVAL, "model_create: NULL argument");
    *out = nullptr;
    QMS_REQUIRE(d->embd && d->out_norm, QMS_CUDA_EINVAL, "model_create: NULL embd or out_norm");
    QMS_REQUIRE(d->n_layer > 0 && d->n_embd > 0 && d->n_head > 0 && d->n_head_kv > 0 && d->head_dim > 0 &&
                    d->n_expert > 0 && d->n_used > 0 && d->n_ff > 0 && d->vocab > 0 && d->ctx > 0,
                QMS_CUDA_EINVAL, "model_create: bad dimensions");
    QMS_REQUIRE(d->n_head % d->n_head_kv == 0 && d->n_used <= d->n_expert, QMS_CUDA_EINVAL,
                "model_create: inconsistent config (n_head %% n_head_kv, n_used <= n_expert)");
    QMS_REQUIRE(d->ctx <= kAttnMaxCtx && d->ctx <= 4 * d->head_dim * kAttnBlock, QMS_CUDA_EUNSUPPORTED,
                "model_create: ctx %d above what the one-token attention merges (%d)", d->ctx,
                std::min(kAttnMaxCtx, 4 * d->head_dim * kAttnBlock));
    QMS_REQUIRE(d->n_head / d->n_head_kv <= 16, QMS_CUDA_EUNSUPPORTED, "model_create: more than 16 q heads per kv head");
    QMS_REQUIRE(d->head_dim == 64 || d->head_dim == 128, QMS_CUDA_EUNSUPPORTED,
                "model_create: head_dim %d (64 or 128 supported)", d->head_dim);
    const int group = d->n_head / d->n_head_kv, HB = attention_heads_per_cta(group);
    QMS_REQUIRE(group % HB == 0, QMS_CUDA_EUNSUPPORTED, "model_create: %d q heads per kv head not supported", group);
    QMS_REQUIRE(d->n_embd % 256 == 0, QMS_CUDA_EUNSUPPORTED, "model_create: n_embd %% 256 must be 0");
    const int QD = d->n_head * d->head_dim;
    QMS_REQUIRE(gemv_cols_ok(d->n_embd, QMS_T_Q4_0) && gemv_cols_ok(QD, QMS_T_Q4_0), QMS_CUDA_EUNSUPPORTED,
                "model_create: projection widths %d / %d not supported", d->n_embd, QD);
    const int et = d->embd_type;
    QMS_REQUIRE(et == QMS_T_Q4_0 || et == QMS_T_Q4_1 || et == QMS_T_Q8_0 || et == QMS_T_Q6_K || et == QMS_T_F16 ||
                    et == QMS_T_F32,
                QMS_CUDA_EUNSUPPORTED, "model_create: token_embd type %d not supported", et);
    const int ht = d->output ? d->output_type : et;
    QMS_REQUIRE(ht == QMS_T_Q4_0 || ht == QMS_T_Q4_1 || ht == QMS_T_Q6_K, QMS_CUDA_EUNSUPPORTED,
                "model_create: output type %d not supported (Q4_0, Q4_1, Q6_K)", ht);
    QMS_REQUIRE(gemv_cols_ok(d->n_embd, ht), QMS_CUDA_EUNSUPPORTED, "model_create: head rows of %d", d->n_embd);
    int dev = 0;
    QMS_CK(cudaGetDevice(&dev));
    QmsCudaModel *m = new (std::nothrow) QmsCudaModel();
    QMS_REQUIRE(m, QMS_CUDA_ENOMEM, "model_create: out of host memory");
    m->device = dev;
    if (cudaDeviceGetAttribute(&m->nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) m->nsm = 148;
    m->L = d->n_layer;
    m->E = d->n_embd;
    m->H = d->n_head;
    m->Hk = d->n_head_kv;
    m->D = d->head_dim;
    m->X = d->n_expert;
    m->K = d->n_used;
    m->F = d->n_ff;
    m->V = d->vocab;
    m->ctx = d->ctx;
    m->eps = d->eps;
    m->rope_base = d->rope_base;
    m->QD = QD;
    m->KD = d->n_head_kv * d->head_dim;
    m->NQKV = QD + 2 * m->KD;
    m->group = group;
    m->embd_type = et;
    m->head_type = ht;
    m->max_splits = (d->ctx + kSplit - 1) / kSplit;
    m->layers.resize(d->n_layer);
    int rc = QMS_CUDA_OK;
    const size_t erb = ggml_row_bytes(et, m->E);
    m->n_seq = 1;
    m->kv_type = QMS_T_F32;
    m->kv_es = 4;
    m->seq_stride = (size_t)m->L * m->ctx * m->KD;
    const size_t kv = (size_t)m->L * m->ctx * m->KD * 4;
    const size_t rope = (size_t)m->ctx * (m->D / 2) * 4;
    if (!rc) rc = dmalloc((void **)&m->embd, (size_t)m->V * erb, "token_embd");
    if (!rc) rc = dmalloc((void **)&m->out_norm, (size_t)m->E * 4, "output_norm");
    if (!rc) rc = dmalloc((void **)&m->head, (size_t)m->V * rows_stride(ht, m->E), "the output head");
    if (!rc) rc = dmalloc((void **)&m->rope_cos, rope, "RoPE tables");
    if (!rc) rc = dmalloc((void **)&m->rope_sin, rope, "RoPE tables");
    if (!rc) rc = dmalloc((void **)&m->flags, (size_t)(1 + m->L) * 4, "error flags");
    if (!rc && (cudaMemset(m->flags, 0, (size_t)(1 + m->L) * 4) != cudaSuccess ||
                cudaMallocHost(&m->h_flags, (size_t)(1 + m->L) * 4) != cudaSuccess)) {
        cudaGetLastError();
        set_error("model_create: cannot set up the error flags");
        rc = QMS_CUDA_ENOMEM;
    }
    if (!rc) rc = dmalloc((void **)&m->kc, kv, "the K cache");
    if (!rc) rc = dmalloc((void **)&m->vc, kv, "the V cache");
    if (!rc) rc = to_device(m->embd, d->embd, (size_t)m->V * erb, d->src_on_device);
    if (!rc) rc = to_device(m->out_norm, d->out_norm, (size_t)m->E * 4, d->src_on_device);
    if (!rc) {
        const void *src = d->output ? d->output : d->embd;
        const int64_t rows = m->V;
        rc = upload_rows(ht, &src, &rows, 1, m->E, d->src_on_device, m->head);
    }
    if (!rc) {
        // NEOX angles exactly as the reference computes them (src/model.c:411-422, 446-447):
        // inv_freq[i] = base^(-2i/D) and cos / sin of pos * inv_freq[i] in double, rounded to float
        std::vector<float> c((size_t)m->ctx * (m->D / 2)), sn(c.size());
        std::vector<double> inv(m->D / 2);
        for (int i = 0; i < m->D / 2; i++) inv[i] = pow(m->rope_base, -2.0 * i / m->D);
        for (int p = 0; p < m->ctx; p++)
            for (int i = 0; i < m->D / 2; i++) {
                const double ang = (double)p * inv[i];
                c[(size_t)p * (m->D / 2) + i] = (float)cos(ang);
                sn[(size_t)p * (m->D / 2) + i] = (float)sin(ang);
            }
        rc = to_device(m->rope_cos, c.data(), rope, 0);
        if (!rc) rc = to_device(m->rope_sin, sn.data(), rope, 0);
    }
    if (!rc && (cudaMemset(m->kc, 0, kv) != cudaSuccess || cudaMemset(m->vc, 0, kv) != cudaSuccess)) {
        set_error("model_create: memset failed");
        rc = QMS_CUDA_ECUDA;
    }
    if (!rc && cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_error("model_create: cannot create a stream");
        rc = QMS_CUDA_ECUDA;
    }
    m->weight_bytes = (size_t)m->V * (erb + rows_stride(ht, m->E)) + (size_t)m->E * 4;
    // the whole prefill chunk at once: the scratch never moves afterwards, so decode steps captured
    // in a CUDA graph stay valid whatever the caller runs next
    if (!rc) rc = model_reserve(m, kChunk);
    if (rc) {
        qms_cuda_model_free(m);
        return rc;
    }
    *out = m;
    return QMS_CUDA_OK;
}

int qms_cuda_model_set_layer(QmsCudaModel *m, int l, const QmsCudaLayerDesc *ld) {
    clear_error();
    QMS_REQUIRE(m && ld, QMS_CUDA_EINVAL, "model_set_layer: NULL argument");
    QMS_REQUIRE(l >= 0 && l < m->L, QMS_CUDA_EINVAL, "model_set_layer: layer %d outside 0..%d", l, m->L - 1);
    QMS_REQUIRE(ld->attn_norm && ld->q_norm && ld->k_norm && ld->ffn_norm && ld->q && ld->k && ld->v && ld->o,
                QMS_CUDA_EINVAL, "model_set_layer: NULL tensor");
    QMS_REQUIRE(ld->q_type == ld->k_type && ld->q_type == ld->v_type &&
                    (ld->q_type == QMS_T_Q4_0 || ld->q_type == QMS_T_Q4_1) &&
                    (ld->o_type == QMS_T_Q4_0 || ld->o_type == QMS_T_Q4_1),
                QMS_CUDA_EUNSUPPORTED, "model_set_layer: attention types %d/%d/%d/%d (Q4_0 or Q4_1, q = k = v)",
                ld->q_type, ld->k_type, ld->v_type, ld->o_type);
    const QmsCudaMoeDesc &md = ld->moe;
    QMS_REQUIRE(md.n_embd == m->E && md.n_expert == m->X && md.n_used == m->K && md.n_ff == m->F, QMS_CUDA_EINVAL,
                "model_set_layer: MoE shape %d/%d/%d/%d differs from the model's", md.n_embd, md.n_expert, md.n_used,
                md.n_ff);
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    DevLayer &L = m->layers[l];
    const int on_dev = md.src_on_device;
    if (L.set) {                                      // replacing a layer
        QMS_CK(cudaDeviceSynchronize());
        cudaFree(L.norms);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
        qms_cuda_moe_destroy(L.moe);
        L = DevLayer();
    }
    const size_t nn = (size_t)2 * m->E + 2 * m->D;
    if (!rc) rc = dmalloc((void **)&L.norms, nn * 4, "layer norms");
    if (!rc) rc = dmalloc((void **)&L.wqkv, (size_t)m->NQKV * rows_stride(ld->q_type, m->E), "QKV weights");
    if (!rc) rc = dmalloc((void **)&L.wo, (size_t)m->E * rows_stride(ld->o_type, m->QD), "O weights");
    if (!rc) {
        L.attn_norm = L.norms;
        L.ffn_norm = L.norms + m->E;
        L.q_norm = L.norms + 2 * m->E;
        L.k_norm = L.q_norm + m->D;
        rc = to_device(L.attn_norm, ld->attn_norm, (size_t)m->E * 4, on_dev);
    }
    if (!rc) rc = to_device(L.ffn_norm, ld->ffn_norm, (size_t)m->E * 4, on_dev);
    if (!rc) rc = to_device(L.q_norm, ld->q_norm, (size_t)m->D * 4, on_dev);
    if (!rc) rc = to_device(L.k_norm, ld->k_norm, (size_t)m->D * 4, on_dev);
    if (!rc) {
        const void *srcs[3] = {ld->q, ld->k, ld->v};
        const int64_t rows[3] = {m->QD, m->KD, m->KD};
        rc = upload_rows(ld->q_type, srcs, rows, 3, m->E, on_dev, L.wqkv);
    }
    if (!rc) {
        const void *src = ld->o;
        const int64_t rows = m->E;
        rc = upload_rows(ld->o_type, &src, &rows, 1, m->QD, on_dev, L.wo);
    }
    if (!rc) rc = qms_cuda_moe_create(&md, &L.moe);
    if (!rc) {
        L.moe->err_ext = m->flags + 1 + l;    // one read of the model's flags covers every layer
        L.moe->err = L.moe->err_ext;
        QMS_CK(cudaMemset(L.moe->err, 0, 4));
        rc = qms_cuda_moe_reserve(L.moe, m->cap_T);
    }
    if (rc) {
        cudaFree(L.norms);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
        qms_cuda_moe_destroy(L.moe);
        L = DevLayer();
        return rc;
    }
    L.qkv_type = ld->q_type;
    L.o_type = ld->o_type;
    L.set = true;
    return QMS_CUDA_OK;
}

int64_t qms_cuda_model_device_bytes(const QmsCudaModel *m) {
    if (!m) return 0;
    int64_t b = (int64_t)m->weight_bytes + (int64_t)m->scratch_bytes;
    b += (int64_t)2 * m->n_seq * m->seq_stride * m->kv_es + (int64_t)2 * m->ctx * (m->D / 2) * 4;
    for (const auto &L : m->layers) {
        if (!L.set) continue;
        b += (int64_t)((2 * m->E + 2 * m->D) * 4) + (int64_t)m->NQKV * rows_stride(L.qkv_type, m->E) +
             (int64_t)m->E * rows_stride(L.o_type, m->QD) + qms_cuda_moe_device_bytes(L.moe);
    }
    return b;
}

int qms_cuda_model_reserve(QmsCudaModel *m, int T) {
    QMS_REQUIRE(m && T >= 0, QMS_CUDA_EINVAL, "model_reserve: bad arguments");
    QMS_REQUIRE(T <= kChunk, QMS_CUDA_EINVAL, "model_reserve: at most %d tokens per pass", kChunk);
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    return model_reserve(m, T);
}

int qms_cuda_forward_dev(QmsCudaModel *m, const int *ids, int T, const int *pos, float *logits, int all_logits,
                         void *stream) {
    QMS_REQUIRE(m && ids && pos && logits && T >= 1, QMS_CUDA_EINVAL, "forward_dev: bad arguments");
    QMS_REQUIRE(T <= m->cap_T, QMS_CUDA_EINVAL, "forward_dev: T=%d exceeds the reserved %d tokens", T, m->cap_T);
    int rc = ensure_dev(m->device);
    if (rc || (rc = layers_ready(m))) return rc;
    return forward_core(m, ids, T, pos, logits, all_logits, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

int qms_cuda_decode_step(QmsCudaModel *m, int *tok, int *pos, float *logits, void *stream) {
    QMS_REQUIRE(m && tok && pos, QMS_CUDA_EINVAL, "decode_step: bad arguments");
    int rc = ensure_dev(m->device);
    if (rc || (rc = layers_ready(m))) return rc;
    return forward_core(m, tok, 1, pos, logits ? logits : m->logits, 0, nullptr, tok, pos, (cudaStream_t)stream);
}

static int flags_check(QmsCudaModel *m);

int qms_cuda_forward(QmsCudaModel *m, const int *ids, int T, int pos0, float *logits, int all_logits, int *sel_trace) {
    return qms_cuda_forward_seq(m, 0, ids, T, pos0, logits, all_logits, sel_trace);
}

int qms_cuda_forward_seq(QmsCudaModel *m, int seq, const int *ids, int T, int pos0, float *logits, int all_logits,
                         int *sel_trace) {
    clear_error();
    QMS_REQUIRE(m && ids && logits && T >= 0 && pos0 >= 0, QMS_CUDA_EINVAL, "forward: bad arguments");
    QMS_REQUIRE(seq >= 0 && seq < m->n_seq, QMS_CUDA_EINVAL, "forward: sequence %d of %d", seq, m->n_seq);
    if (T == 0) return QMS_CUDA_OK;
    QMS_REQUIRE((int64_t)pos0 + T <= m->ctx, QMS_CUDA_EINVAL, "forward: context %d exceeded", m->ctx);
    for (int t = 0; t < T; t++) QMS_REQUIRE(ids[t] >= 0 && ids[t] < m->V, QMS_CUDA_EINVAL, "forward: bad id %d", ids[t]);
    int rc = ensure_dev(m->device);
    if (rc || (rc = layers_ready(m))) return rc;
    if ((rc = model_reserve(m, std::min(T, kChunk)))) return rc;
    const cudaStream_t s = m->stream;
    if ((rc = prof_events(m))) return rc;
    for (int c0 = 0; c0 < T; c0 += m->cap_T) {
        const int Tc = std::min(m->cap_T, T - c0);
        const bool last = c0 + Tc == T;
        QMS_CK(cudaStreamSynchronize(s));          // the pinned mirror is reused
        memcpy(m->h_pinned, ids + c0, (size_t)Tc * 4);
        m->h_pinned[Tc] = pos0 + c0;
        QMS_CK(cudaMemcpyAsync(m->ids, m->h_pinned, (size_t)Tc * 4, cudaMemcpyHostToDevice, s));
        QMS_CK(cudaMemcpyAsync(m->pos, m->h_pinned + Tc, 4, cudaMemcpyHostToDevice, s));
        const int want = all_logits || last;
        if ((rc = forward_core(m, m->ids, Tc, m->pos, m->logits, all_logits, sel_trace ? m->sel : nullptr, nullptr,
                               nullptr, s, seq)))
            return rc;
        if (want) {
            const size_t n = (size_t)(all_logits ? Tc : 1) * m->V;
            float *dst = logits + (all_logits ? (size_t)c0 * m->V : 0);
            QMS_CK(cudaMemcpyAsync(dst, m->logits, n * 4, cudaMemcpyDeviceToHost, s));
        }
        if (sel_trace)
            for (int l = 0; l < m->L; l++)
                QMS_CK(cudaMemcpyAsync(sel_trace + ((size_t)l * T + c0) * m->K, m->sel + (size_t)l * Tc * m->K,
                                       (size_t)Tc * m->K * 4, cudaMemcpyDeviceToHost, s));
        if (last) QMS_CK(cudaMemcpyAsync(m->h_flags, m->flags, (size_t)(1 + m->L) * 4, cudaMemcpyDeviceToHost, s));
        QMS_CK(cudaStreamSynchronize(s));
        if ((rc = prof_collect(m))) return rc;
    }
    return flags_check(m);
}

// The flags in h_flags (copied after the stream's last kernel): the trunk's word, then each MoE
// layer's. A raised flag is reported once and cleared.
static int flags_check(QmsCudaModel *m) {
    int trunk = m->h_flags[0], moe = 0, layer = -1;
    for (int l = 0; l < m->L; l++)
        if (m->h_flags[1 + l] && layer < 0) {
            moe = m->h_flags[1 + l];
            layer = l;
        }
    if (!trunk && layer < 0) return QMS_CUDA_OK;
    QMS_CK(cudaMemset(m->flags, 0, (size_t)(1 + m->L) * 4));
    memset(m->h_flags, 0, (size_t)(1 + m->L) * 4);
    if (trunk & ~3) {
        set_error("forward: a bounded wait inside the decode kernels gave up (flags 0x%x: 64 = a weight stream, "
                  "128 = attention); outputs of that call are invalid", trunk);
        return QMS_CUDA_ETIMEOUT;
    }
    if (trunk) {
        set_error("forward: a device-side check refused work (flags 0x%x: 1 = position beyond ctx %d, 2 = bad token id)",
                  trunk, m->ctx);
        return QMS_CUDA_EINVAL;
    }
    set_error("moe: layer %d: a bounded wait inside the decode kernels gave up (flags 0x%x); outputs of that call "
              "are invalid", layer, moe);
    return QMS_CUDA_ETIMEOUT;
}

// (Re)allocate the KV caches of n_seq sequences with elements of kv_type (cleared), and the batched
// attention's partials for up to min(n_seq, 256) sequences (here, so that no batched call
// allocates: they may be captured in a CUDA graph).
static int realloc_caches(QmsCudaModel *m, int n_seq, int kv_type) {
    const size_t es = kv_type == QMS_T_F16 ? 2 : 4, kv = (size_t)n_seq * m->seq_stride * es;
    void *kc = nullptr, *vc = nullptr;
    int rc = dmalloc(&kc, kv, "the K caches");
    if (!rc) rc = dmalloc(&vc, kv, "the V caches");
    if (!rc && (cudaMemset(kc, 0, kv) != cudaSuccess || cudaMemset(vc, 0, kv) != cudaSuccess)) {
        set_error("KV caches: memset failed");
        rc = QMS_CUDA_ECUDA;
    }
    const int nb = std::min(n_seq, kChunk), ms = (m->ctx + kAttnBlock - 1) / kAttnBlock;
    float *po = nullptr;
    double *pml = nullptr;
    if (!rc && n_seq > 1) {
        rc = dmalloc((void **)&po, (size_t)nb * m->H * ms * m->D * 4, "batched attention partials");
        if (!rc) rc = dmalloc((void **)&pml, (size_t)nb * m->H * ms * 16, "batched attention partials");
    }
    if (rc) {
        cudaFree(kc);
        cudaFree(vc);
        cudaFree(po);
        cudaFree(pml);
        return rc;
    }
    QMS_CK(cudaDeviceSynchronize());
    cudaFree(m->kc);
    cudaFree(m->vc);
    cudaFree(m->bpart_o);
    cudaFree(m->bpart_ml);
    m->kc = kc;
    m->vc = vc;
    m->bpart_o = po;
    m->bpart_ml = pml;
    m->n_seq = n_seq;
    m->kv_type = kv_type;
    m->kv_es = es;
    return QMS_CUDA_OK;
}

int qms_cuda_model_set_sequences(QmsCudaModel *m, int n_seq) {
    clear_error();
    QMS_REQUIRE(m && n_seq >= 1, QMS_CUDA_EINVAL, "set_sequences: bad arguments");
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    if (n_seq == m->n_seq) return QMS_CUDA_OK;
    return realloc_caches(m, n_seq, m->kv_type);
}

int qms_cuda_model_set_kv_type(QmsCudaModel *m, int kv_type) {
    clear_error();
    QMS_REQUIRE(m, QMS_CUDA_EINVAL, "set_kv_type: NULL model");
    QMS_REQUIRE(kv_type == QMS_T_F32 || kv_type == QMS_T_F16, QMS_CUDA_EUNSUPPORTED,
                "set_kv_type: type %d (F32 or F16)", kv_type);
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    if (kv_type == m->kv_type) return QMS_CUDA_OK;
    return realloc_caches(m, m->n_seq, kv_type);
}

int qms_cuda_model_copy_sequence(QmsCudaModel *m, int src, int dst, int npos) {
    clear_error();
    QMS_REQUIRE(m && src >= 0 && dst >= 0 && src < m->n_seq && dst < m->n_seq && src != dst && npos >= 0 &&
                    npos <= m->ctx,
                QMS_CUDA_EINVAL, "copy_sequence: bad arguments");
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    const size_t es = m->kv_es, layer = (size_t)m->ctx * m->KD, n = (size_t)npos * m->KD * es;
    char *kc = static_cast<char *>(m->kc), *vc = static_cast<char *>(m->vc);
    for (int l = 0; l < m->L && n; l++) {
        const size_t so = es * ((size_t)src * m->seq_stride + l * layer), d = es * ((size_t)dst * m->seq_stride + l * layer);
        QMS_CK(cudaMemcpyAsync(kc + d, kc + so, n, cudaMemcpyDeviceToDevice, m->stream));
        QMS_CK(cudaMemcpyAsync(vc + d, vc + so, n, cudaMemcpyDeviceToDevice, m->stream));
    }
    QMS_CK(cudaStreamSynchronize(m->stream));
    return QMS_CUDA_OK;
}

int qms_cuda_forward_batch(QmsCudaModel *m, int B, const int *ids, const int *pos, float *logits) {
    clear_error();
    QMS_REQUIRE(m && ids && pos && logits && B >= 1, QMS_CUDA_EINVAL, "forward_batch: bad arguments");
    QMS_REQUIRE(B <= m->n_seq && B <= m->cap_T, QMS_CUDA_EINVAL, "forward_batch: %d sequences (%d with caches, %d per pass)",
                B, m->n_seq, m->cap_T);
    for (int b = 0; b < B; b++) {
        QMS_REQUIRE(ids[b] >= 0 && ids[b] < m->V, QMS_CUDA_EINVAL, "forward_batch: bad id %d", ids[b]);
        QMS_REQUIRE(pos[b] >= 0 && pos[b] < m->ctx, QMS_CUDA_EINVAL, "forward_batch: context %d exceeded", m->ctx);
    }
    int rc = ensure_dev(m->device);
    if (rc || (rc = layers_ready(m))) return rc;
    const cudaStream_t s = m->stream;
    if ((rc = prof_events(m))) return rc;
    QMS_CK(cudaStreamSynchronize(s));
    memcpy(m->h_pinned, ids, (size_t)B * 4);
    memcpy(m->h_pinned + B, pos, (size_t)B * 4);
    QMS_CK(cudaMemcpyAsync(m->ids, m->h_pinned, (size_t)B * 4, cudaMemcpyHostToDevice, s));
    QMS_CK(cudaMemcpyAsync(m->pos_vec, m->h_pinned + B, (size_t)B * 4, cudaMemcpyHostToDevice, s));
    if ((rc = forward_core(m, m->ids, B, nullptr, m->logits, 1, nullptr, nullptr, nullptr, s, 0, m->pos_vec))) return rc;
    QMS_CK(cudaMemcpyAsync(logits, m->logits, (size_t)B * m->V * 4, cudaMemcpyDeviceToHost, s));
    QMS_CK(cudaMemcpyAsync(m->h_flags, m->flags, (size_t)(1 + m->L) * 4, cudaMemcpyDeviceToHost, s));
    QMS_CK(cudaStreamSynchronize(s));
    if ((rc = prof_collect(m))) return rc;
    return flags_check(m);
}

int qms_cuda_decode_batch(QmsCudaModel *m, int B, int *tok, int *pos, float *logits, void *stream) {
    QMS_REQUIRE(m && tok && pos && B >= 1, QMS_CUDA_EINVAL, "decode_batch: bad arguments");
    QMS_REQUIRE(B <= m->n_seq && B <= m->cap_T, QMS_CUDA_EINVAL, "decode_batch: %d sequences (%d with caches, %d per pass)",
                B, m->n_seq, m->cap_T);
    int rc = ensure_dev(m->device);
    if (rc || (rc = layers_ready(m))) return rc;
    return forward_core(m, tok, B, nullptr, logits ? logits : m->logits, 1, nullptr, tok, pos, (cudaStream_t)stream, 0,
                        pos);
}

int qms_cuda_model_status(QmsCudaModel *m) {
    QMS_REQUIRE(m, QMS_CUDA_EINVAL, "model_status: NULL model");
    int rc = ensure_dev(m->device);
    if (rc) return rc;
    QMS_CK(cudaDeviceSynchronize());
    QMS_CK(cudaMemcpy(m->h_flags, m->flags, (size_t)(1 + m->L) * 4, cudaMemcpyDeviceToHost));
    return flags_check(m);
}

int qms_cuda_model_profile(QmsCudaModel *m, int on, double *ms) {
    QMS_REQUIRE(m, QMS_CUDA_EINVAL, "model_profile: NULL model");
    if (ms) {
        for (int i = 0; i < 7; i++) ms[i] = m->prof_ms[i];
        for (int i = 0; i < 7; i++) m->prof_ms[i] = 0.0;
    }
    m->prof = on != 0;
    return QMS_CUDA_OK;
}

}  // extern "C"
