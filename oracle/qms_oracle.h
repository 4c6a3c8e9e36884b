/* qms_oracle.h - CPU restatement of qms's Qwen3-MoE feed-forward path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is compared
 * against; nothing in the product (libqms_cuda) links, loads or calls it. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may use it.
 *
 * Every function restates the reference's integer ("fast") path, including its float
 * evaluation order as compiled by gcc -O2 with FMA (AVX2 lanes, hsum tree, contracted
 * multiply-adds), so that its outputs are bit-identical to the reference's own build.
 * That claim is pinned by tests/test_oracle_vs_ref.py against oracle/_ref (the reference
 * compiled from its own sources) and by tests/golden/ fixtures produced from oracle/_ref.
 */
#ifndef QMS_ORACLE_H
#define QMS_ORACLE_H

#include <stdint.h>

/* ggml tensor type ids (GGUF file format numbering; reference src/gguf.h:8-10). */
enum { ORC_T_F32 = 0, ORC_T_F16 = 1, ORC_T_Q4_0 = 2, ORC_T_Q4_1 = 3, ORC_T_Q8_0 = 8, ORC_T_Q6_K = 14 };

/* Activation block, 44 bytes: same layout as the reference's QmsQ8 (src/kernels.h:7-12). */
typedef struct {
    float d;
    float ds;
    int16_t s16[2];
    int8_t q[32];
} OrcQ8;

/* One resident MoE layer in GGUF layout (reference src/model.h:229-243, model.c:133-157):
 * router F32 [n_expert][n_embd]; gate/up stacked [n_expert][n_ff][n_embd/32 blocks];
 * down stacked [n_expert][n_embd][n_ff/32 blocks]. */
typedef struct {
    int n_embd, n_expert, n_used, n_ff;
    int gate_type, up_type, down_type;
    const float *router;
    const uint8_t *gate, *up, *down;
} OrcMoe;

float    orc_f16_to_f32(uint16_t h);
uint64_t orc_row_bytes(int type, int64_t ne0);
int      orc_dequant_row(int type, const void *src, float *dst, int64_t n);
void     orc_quantize_q8(const float *x, int64_t n, OrcQ8 *out);
float    orc_vec_dot_q8(int type, const uint8_t *w, const OrcQ8 *x, int64_t n);
float    orc_vec_dot_f32(const float *w, const float *x, int64_t n);
/* y[t][r] = W[r] . x[t] through the integer path (F32 weights: fp32 dot). */
void     orc_matmul(int type, int64_t rows, int64_t cols, const uint8_t *w, const float *x, int T, float *y);
void     orc_matmul_q8(int type, int64_t rows, int64_t cols, const uint8_t *w, const OrcQ8 *xq, int T, float *y);
int      orc_sample(const float *logits, int V, float temp, float top_p, int top_k, uint64_t *rng);
/* Router: logits, top-k ids in selection order, renormalised weights. */
void     orc_route(const float *router, int n_expert, int n_embd, int n_used, const float *xn, int T,
                   float *logits, int *sel, float *wts);
/* Whole MoE block, fast path. sel/wts/logits may be NULL. Returns 0, or -1 when the
 * reference would not take the fast path for this layer (it would use --exact math). */
int      orc_moe(const OrcMoe *L, const float *xn, int T, float *out, int *sel, float *wts, float *logits);
/* Reference SwiGLU activation a = silu(g) * u for one row (model.c:424, 994). */
void     orc_swiglu(const float *g, const float *u, int64_t n, float *a);
void     orc_set_threads(int n);

#endif /* QMS_ORACLE_H */
