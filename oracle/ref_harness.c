/* ref_harness.c - exposes the reference's own MoE block for parity checks (test infrastructure).
 *
 * Compiled by oracle/Makefile together with the reference's unmodified sources, read in place
 * from the reference tree: src/model.c is included here so that its static moe() (model.c:1032)
 * can be called on a one-layer resident QmsModel. The library lands in oracle/_ref/ and is
 * only ever used as a checker (tests/golden/make_golden.py, tests/, bench.py's reference arm).
 */
#include "model.c"

#include <stdio.h>

void ref_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int ref_get_threads(void) { return omp_get_max_threads(); }
void ref_set_exact(int on) { qms_exact_math = on; }

static QmsMat mat(int type, int64_t rows, int64_t cols, const void *data)
{
    QmsMat m;
    m.type = type;
    m.rows = rows;
    m.cols = cols;
    m.row_bytes = qms_row_bytes(type, cols);
    m.data = (const unsigned char *)data;
    return m;
}

/* Run moe() on T tokens of xn [T][E]; out [T][E]. When trace is non-NULL it receives the
 * reference's own --trace records for this call (distinct experts in ascending order, one
 * int per record) and *n_trace their count (capacity: X). Returns moe()'s status. */
int ref_moe(int E, int X, int K, int F, int gate_type, int up_type, int down_type,
            const float *router, const void *gate, const void *up, const void *down,
            const float *xn, int T, float *out, int *trace, int *n_trace)
{
    QmsModel m;
    QmsLayer L;
    memset(&m, 0, sizeof m);
    memset(&L, 0, sizeof L);
    m.c.n_layer = 1;
    m.c.n_embd = E;
    m.c.n_expert = X;
    m.c.n_used = K;
    m.c.n_ff_exp = F;
    m.L = &L;
    L.router = mat(QMS_T_F32, X, E, router);
    L.gate.m = mat(gate_type, F, E, gate);
    L.gate.expert_bytes = L.gate.m.row_bytes * (uint64_t)F;
    L.up.m = mat(up_type, F, E, up);
    L.up.expert_bytes = L.up.m.row_bytes * (uint64_t)F;
    L.down.m = mat(down_type, E, F, down);
    L.down.expert_bytes = L.down.m.row_bytes * (uint64_t)E;
    m.eptr = (const unsigned char **)calloc(3 * (size_t)X, sizeof(*m.eptr));
    if (!m.eptr) return -1;
    if (trace) m.trace = tmpfile();
    const int rc = moe(&m, 0, xn, xn, T, out);
    if (trace && m.trace) {
        fflush(m.trace);
        rewind(m.trace);
        int n = 0;
        int32_t st;
        int16_t ly, ex;
        while (n < X && fread(&st, 4, 1, m.trace) == 1 && fread(&ly, 2, 1, m.trace) == 1 &&
               fread(&ex, 2, 1, m.trace) == 1)
            trace[n++] = ex;
        *n_trace = n;
        fclose(m.trace);
    }
    free((void *)m.eptr);
    return rc;
}

/* ---- the reference's whole forward pass on a model built from host arrays ----------------------
 * qms_model_load (src/model.c:314-387) without the file: the caller passes each tensor's host
 * buffer (GGUF layout), which the model points at (not copied); KV cache and expert pointers are
 * allocated as load does. ref_forward is the reference's own qms_forward (src/model.c:1252). */
QmsModel *ref_model_new(int n_layer, int n_embd, int n_head, int n_head_kv, int head_dim, int n_expert,
                        int n_used, int n_ff, int vocab, float eps, double rope_base, int ctx)
{
    QmsModel *m = (QmsModel *)calloc(1, sizeof *m);
    if (!m) return NULL;
    QmsCfg *c = &m->c;
    c->n_layer = n_layer; c->n_embd = n_embd; c->n_head = n_head; c->n_head_kv = n_head_kv;
    c->head_dim = head_dim; c->n_expert = n_expert; c->n_used = n_used; c->n_ff_exp = n_ff;
    c->vocab = vocab; c->eps = eps; c->rope_base = rope_base;
    m->ctx = ctx;
    m->tr.n_pin = n_layer;
    m->tr.slot_layer[0] = m->tr.slot_layer[1] = -1;
    m->L = (QmsLayer *)calloc((size_t)n_layer, sizeof(QmsLayer));
    m->eptr = (const unsigned char **)calloc(3 * (size_t)n_expert, sizeof(*m->eptr));
    const size_t kv = (size_t)n_layer * ctx * n_head_kv * head_dim;
    m->kc = (float *)calloc(kv, sizeof(float));
    m->vc = (float *)calloc(kv, sizeof(float));
    if (!m->L || !m->eptr || !m->kc || !m->vc) return NULL;
    return m;
}

void ref_model_set_trunk(QmsModel *m, int embd_type, const void *embd, const float *out_norm, int out_type,
                         const void *output)
{
    const QmsCfg *c = &m->c;
    m->embd = mat(embd_type, c->vocab, c->n_embd, embd);
    m->out_norm = (float *)out_norm;
    m->output = output ? mat(out_type, c->vocab, c->n_embd, output) : m->embd;   /* tied (src/model.c:335) */
}

void ref_model_set_layer(QmsModel *m, int l, const float *attn_norm, const float *q_norm, const float *k_norm,
                         const float *ffn_norm, int att_type, const void *q, const void *k, const void *v,
                         int o_type, const void *o, const float *router, int gate_type, const void *gate,
                         const void *up, int down_type, const void *down)
{
    const QmsCfg *c = &m->c;
    QmsLayer *L = &m->L[l];
    const int E = c->n_embd, QD = c->n_head * c->head_dim, KD = c->n_head_kv * c->head_dim, F = c->n_ff_exp;
    L->attn_norm = (float *)attn_norm; L->q_norm = (float *)q_norm; L->k_norm = (float *)k_norm;
    L->ffn_norm = (float *)ffn_norm;
    L->q = mat(att_type, QD, E, q);
    L->k = mat(att_type, KD, E, k);
    L->v = mat(att_type, KD, E, v);
    L->o = mat(o_type, E, QD, o);
    L->router = mat(QMS_T_F32, c->n_expert, E, router);
    L->gate.m = mat(gate_type, F, E, gate);
    L->gate.expert_bytes = L->gate.m.row_bytes * (uint64_t)F;
    L->up.m = mat(gate_type, F, E, up);
    L->up.expert_bytes = L->up.m.row_bytes * (uint64_t)F;
    L->down.m = mat(down_type, E, F, down);
    L->down.expert_bytes = L->down.m.row_bytes * (uint64_t)E;
}

int ref_forward(QmsModel *m, const int *ids, int T, int pos0, float *logits, int all_logits)
{
    return qms_forward(m, ids, T, pos0, logits, all_logits);
}

void ref_model_free(QmsModel *m)
{
    if (!m) return;
    free(m->L);
    free((void *)m->eptr);
    free(m->kc);
    free(m->vc);
    free(m);
}
