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
