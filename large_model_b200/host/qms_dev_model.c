/* qms_dev_model.c - the device build of qms's model layer: qms_forward runs on the B200 through
 * libqms_cuda (include/qms_cuda.h); qms_model_load, the GGUF reader, the tokenizer and the CLI
 * stay the reference's own code, compiled unchanged from its source tree.
 *
 * This is the binding a maintainer adds to the reference (the reference is C and links the
 * library directly): the reference's src/model.c is compiled inside this translation unit with
 * its qms_forward and qms_model_free renamed, and the two functions below take their place.
 *   qms_forward    (src/model.h:141, src/model.c:1252-1296): on the first call the loaded host
 *                  tensors are uploaded once (qms_cuda_model_create / _set_layer); every call then
 *                  runs qms_cuda_forward. --trace records (src/model.c:1102-1110) are written from
 *                  the device's expert selections; QMS_PROF sections (src/model.h:143-150) come
 *                  from CUDA events.
 *   qms_model_free (src/model.h:136): frees the device model, then the host model.
 * There is no CPU fallback: a device failure is a -1 return with the reason on stderr, as the
 * reference reports its own failures. --exact (the fp32 dequantise-then-dot path) is refused;
 * the device implements the reference's default integer path. */
#define qms_forward qms_forward_host
#define qms_model_free qms_model_free_host
#include "model.c"
#undef qms_forward
#undef qms_model_free

#include "qms_cuda.h"

static QmsCudaModel *g_dev;          /* one model per process, like the CLI's one QmsModel */
static const QmsModel *g_dev_owner;

static int dev_upload(QmsModel *m)
{
    const QmsCfg *c = &m->c;
    if (qms_cuda_init(0) != QMS_CUDA_OK) { fprintf(stderr, "device: %s\n", qms_cuda_last_error()); return -1; }
    QmsCudaModelDesc d;
    memset(&d, 0, sizeof d);
    d.n_layer = c->n_layer; d.n_embd = c->n_embd; d.n_head = c->n_head; d.n_head_kv = c->n_head_kv;
    d.head_dim = c->head_dim; d.n_expert = c->n_expert; d.n_used = c->n_used; d.n_ff = c->n_ff_exp;
    d.vocab = c->vocab; d.eps = c->eps; d.rope_base = c->rope_base; d.ctx = m->ctx;
    d.embd_type = m->embd.type; d.embd = m->embd.data;
    d.out_norm = m->out_norm;
    /* tied embeddings: load points output at embd (src/model.c:333-335) */
    d.output_type = m->output.type;
    d.output = m->output.data == m->embd.data ? NULL : m->output.data;
    d.src_on_device = 0;
    if (!d.embd) { fprintf(stderr, "device: token embeddings are not resident\n"); return -1; }
    double t0 = qms_now();
    if (qms_cuda_model_create(&d, &g_dev) != QMS_CUDA_OK) {
        fprintf(stderr, "device: %s\n", qms_cuda_last_error());
        return -1;
    }
    for (int l = 0; l < c->n_layer; l++) {
        const QmsLayer *L = &m->L[l];
        QmsCudaLayerDesc ld;
        memset(&ld, 0, sizeof ld);
        ld.attn_norm = L->attn_norm; ld.q_norm = L->q_norm; ld.k_norm = L->k_norm; ld.ffn_norm = L->ffn_norm;
        ld.q_type = L->q.type; ld.k_type = L->k.type; ld.v_type = L->v.type; ld.o_type = L->o.type;
        ld.q = L->q.data; ld.k = L->k.data; ld.v = L->v.data; ld.o = L->o.data;
        ld.moe.n_embd = c->n_embd; ld.moe.n_expert = c->n_expert; ld.moe.n_used = c->n_used;
        ld.moe.n_ff = c->n_ff_exp;
        ld.moe.gate_type = L->gate.m.type; ld.moe.up_type = L->up.m.type; ld.moe.down_type = L->down.m.type;
        ld.moe.router = (const float *)L->router.data;
        ld.moe.gate = L->gate.m.data; ld.moe.up = L->up.m.data; ld.moe.down = L->down.m.data;
        ld.moe.src_on_device = 0;
        if (!ld.q || !ld.moe.gate) {
            fprintf(stderr, "device: layer %d is not resident (streaming modes are host-only)\n", l);
            return -1;
        }
        if (qms_cuda_model_set_layer(g_dev, l, &ld) != QMS_CUDA_OK) {
            fprintf(stderr, "device: layer %d: %s\n", l, qms_cuda_last_error());
            return -1;
        }
    }
    fprintf(stderr, "device: %d layers uploaded, %.2f GB on the GPU, %.1f s\n", c->n_layer,
            qms_cuda_model_device_bytes(g_dev) / 1e9, qms_now() - t0);
    g_dev_owner = m;
    return 0;
}

int qms_forward(QmsModel *m, const int *ids, int T, int pos0, float *logits, int all_logits)
{
    const QmsCfg *c = &m->c;
    m->trace_step++;
    if (pos0 + T > m->ctx) { fprintf(stderr, "forward: context %d exceeded\n", m->ctx); return -1; }
    if (qms_exact_math) { fprintf(stderr, "forward: --exact is not implemented by the device build\n"); return -1; }
    if (!g_dev && dev_upload(m) != 0) return -1;
    if (g_dev_owner != m) { fprintf(stderr, "forward: the device holds another model\n"); return -1; }
    int *sel = NULL;
    if (m->trace) {
        sel = (int *)malloc((size_t)c->n_layer * T * c->n_used * sizeof(int));
        if (!sel) return -1;
    }
    qms_cuda_model_profile(g_dev, qms_prof_on, NULL);
    if (qms_cuda_forward(g_dev, ids, T, pos0, logits, all_logits, sel) != QMS_CUDA_OK) {
        fprintf(stderr, "forward: %s\n", qms_cuda_last_error());
        free(sel);
        return -1;
    }
    if (qms_prof_on) {   /* device milliseconds per section into the reference's second counters */
        double ms[7];
        qms_cuda_model_profile(g_dev, 1, ms);
        for (int k = 0; k < 7 && k < QMS_PROF_N; k++) qms_prof[k] += ms[k] / 1e3;
    }
    if (sel) {           /* one record per distinct expert of each layer, in expert order */
        unsigned char *seen = (unsigned char *)calloc((size_t)c->n_expert, 1);
        for (int l = 0; l < c->n_layer && seen; l++) {
            memset(seen, 0, (size_t)c->n_expert);
            for (int i = 0; i < T * c->n_used; i++) {
                const int e = sel[(size_t)l * T * c->n_used + i];
                if (e >= 0 && e < c->n_expert) seen[e] = 1;
            }
            for (int e = 0; e < c->n_expert; e++) {
                if (!seen[e]) continue;
                const int32_t st = m->trace_step;
                const int16_t ly = (int16_t)l, ex = (int16_t)e;
                fwrite(&st, 4, 1, m->trace);
                fwrite(&ly, 2, 1, m->trace);
                fwrite(&ex, 2, 1, m->trace);
            }
        }
        free(seen);
        free(sel);
    }
    return 0;
}

void qms_model_free(QmsModel *m)
{
    if (g_dev && g_dev_owner == m) {
        qms_cuda_model_free(g_dev);
        g_dev = NULL;
        g_dev_owner = NULL;
    }
    qms_model_free_host(m);
}
