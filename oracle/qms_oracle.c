/* qms_oracle.c - CPU restatement of qms's Qwen3-MoE feed-forward path (test infrastructure).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libqms_cuda, never part of the product path.
 *
 * Compiled with -ffp-contract=off so that every fused multiply-add below is an explicit
 * fmaf() placed exactly where gcc -O2 -mfma contracts the reference's source, and every
 * other float operation is rounded on its own. The eight AVX2 float lanes of the
 * reference's dot products are restated as arrays acc[8], reduced in hsum256's order.
 *
 * Citations are src/<file>:<line> inside the reference project (ZeningXiong/large_model).
 */
#include "qms_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* fp16 -> fp32, exact for every half (src/qms.h:11-33). */
float orc_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* subnormal half: shift the mantissa up until its leading one reaches bit 10 */
            int e = 1;
            while (!(mant & 0x400u)) { mant <<= 1; e--; }
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(e + 127 - 15) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float ld_f16(const uint8_t *p)
{
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

/* Bytes per row (src/gguf.c:85-96). */
uint64_t orc_row_bytes(int type, int64_t ne0)
{
    switch (type) {
    case ORC_T_F32:  return (uint64_t)ne0 * 4;
    case ORC_T_F16:  return (uint64_t)ne0 * 2;
    case ORC_T_Q4_0: return ne0 % 32 ? 0 : (uint64_t)ne0 / 32 * 18;
    case ORC_T_Q4_1: return ne0 % 32 ? 0 : (uint64_t)ne0 / 32 * 20;
    case ORC_T_Q8_0: return ne0 % 32 ? 0 : (uint64_t)ne0 / 32 * 34;
    case ORC_T_Q6_K: return ne0 % 256 ? 0 : (uint64_t)ne0 / 256 * 210;
    default:         return 0;
    }
}

/* Block dequantisers (src/quant.c:17-93). */
int orc_dequant_row(int type, const void *src, float *y, int64_t n)
{
    const uint8_t *b = (const uint8_t *)src;
    switch (type) {
    case ORC_T_F32:
        memcpy(y, b, (size_t)n * 4);
        return 0;
    case ORC_T_F16:
        for (int64_t i = 0; i < n; i++) y[i] = ld_f16(b + 2 * i);
        return 0;
    case ORC_T_Q4_0:                                   /* src/quant.c:17-28 */
        if (n % 32) return -1;
        for (int64_t i = 0; i < n; i += 32, b += 18, y += 32) {
            const float d = ld_f16(b);
            for (int j = 0; j < 16; j++) {
                y[j] = (float)((b[2 + j] & 0x0F) - 8) * d;
                y[j + 16] = (float)((b[2 + j] >> 4) - 8) * d;
            }
        }
        return 0;
    case ORC_T_Q4_1:                                   /* src/quant.c:30-41; q*d is exact */
        if (n % 32) return -1;
        for (int64_t i = 0; i < n; i += 32, b += 20, y += 32) {
            const float d = ld_f16(b), m = ld_f16(b + 2);
            for (int j = 0; j < 16; j++) {
                y[j] = fmaf((float)(b[4 + j] & 0x0F), d, m);
                y[j + 16] = fmaf((float)(b[4 + j] >> 4), d, m);
            }
        }
        return 0;
    case ORC_T_Q8_0:                                   /* src/quant.c:43-51 */
        if (n % 32) return -1;
        for (int64_t i = 0; i < n; i += 32, b += 34, y += 32) {
            const float d = ld_f16(b);
            for (int j = 0; j < 32; j++) y[j] = (float)(int8_t)b[2 + j] * d;
        }
        return 0;
    case ORC_T_Q6_K:                                   /* src/quant.c:53-79 */
        if (n % 256) return -1;
        for (int64_t i = 0; i < n; i += 256, b += 210) {
            const uint8_t *ql = b, *qh = b + 128;
            const int8_t *sc = (const int8_t *)(b + 192);
            const float d = ld_f16(b + 208);
            for (int half = 0; half < 2; half++) {
                for (int l = 0; l < 32; l++) {
                    const int is = l / 16;
                    const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    y[l] = d * (float)sc[is + 0] * (float)q1;
                    y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    y[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
                y += 128;
                ql += 64;
                qh += 32;
                sc += 8;
            }
        }
        return 0;
    default:
        return -1;
    }
}

/* Per-32 activation quantiser (src/kernels.c:34-53): d = amax/127, q = round-half-even(x/d). */
void orc_quantize_q8(const float *x, int64_t n, OrcQ8 *out)
{
    for (int64_t b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        int s0 = 0, s1 = 0;
        for (int j = 0; j < 32; j++) {
            const int q = (int)nearbyintf(xb[j] * id);
            out[b].q[j] = (int8_t)q;
            if (j < 16) s0 += q; else s1 += q;
        }
        out[b].d = d;
        out[b].s16[0] = (int16_t)s0;
        out[b].s16[1] = (int16_t)s1;
        out[b].ds = d * (float)(s0 + s1);
    }
}

/* hsum256 (src/kernels.c:66-72): fold the high 128 bits onto the low, then movehl, then
 * movehdup: ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)). */
static inline float hsum8(const float v[8])
{
    const float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    const float t0 = s0 + s2, t1 = s1 + s3;
    return t0 + t1;
}

/* Integer dot of one 32-block, split in the eight 4-element dpbusd lanes (src/kernels.c:56-64):
 * lane k covers elements 4k..4k+3 of the block. */
static inline void q4_lanes(const uint8_t *qs, const int8_t *q8, int lane[8])
{
    for (int k = 0; k < 8; k++) {
        int s = 0;
        for (int m = 0; m < 4; m++) {
            const int j = 4 * k + m;
            const int w = j < 16 ? (qs[j] & 0x0F) : (qs[j - 16] >> 4);
            s += w * q8[j];
        }
        lane[k] = s;
    }
}

/* Q4_0 x Q8 (src/kernels.c:82-94, AVX2 branch as compiled with FMA contraction). */
static float dot_q4_0(const uint8_t *w, const OrcQ8 *x, int64_t nb)
{
    float acc[8] = { 0 }, corr = 0.0f;
    int lane[8];
    for (int64_t b = 0; b < nb; b++, w += 18) {
        const float d = ld_f16(w);
        q4_lanes(w + 2, x[b].q, lane);
        const float dd = d * x[b].d;
        for (int k = 0; k < 8; k++) acc[k] = fmaf((float)lane[k], dd, acc[k]);
        corr = fmaf(d, x[b].ds, corr);
    }
    return hsum8(acc) - 8.0f * corr;
}

/* Q4_1 x Q8 (src/kernels.c:109-121). */
static float dot_q4_1(const uint8_t *w, const OrcQ8 *x, int64_t nb)
{
    float acc[8] = { 0 }, off = 0.0f;
    int lane[8];
    for (int64_t b = 0; b < nb; b++, w += 20) {
        const float d = ld_f16(w), m = ld_f16(w + 2);
        q4_lanes(w + 4, x[b].q, lane);
        const float dd = d * x[b].d;
        for (int k = 0; k < 8; k++) acc[k] = fmaf((float)lane[k], dd, acc[k]);
        off = fmaf(m, x[b].ds, off);
    }
    return hsum8(acc) + off;
}

/* Q6_K x Q8 (src/kernels.c:139-170): per 32-group g of a 128-half, lanes 0-3 (elements 0..15)
 * are scaled by sc[2g] and lanes 4-7 by sc[2g+1]; the -32 offset is folded into corr. */
static float dot_q6_k(const uint8_t *w, const OrcQ8 *x, int64_t nsb)
{
    float acc[8] = { 0 }, corr = 0.0f;
    for (int64_t sb = 0; sb < nsb; sb++, w += 210) {
        const float d = ld_f16(w + 208);
        const int8_t *scs = (const int8_t *)(w + 192);
        for (int half = 0; half < 2; half++) {
            const uint8_t *ql = w + half * 64;
            const uint8_t *qh = w + 128 + half * 32;
            const int8_t *sc = scs + half * 8;
            for (int g = 0; g < 4; g++) {
                const OrcQ8 *xb = &x[sb * 8 + half * 4 + g];
                const int sa = sc[2 * g], sbb = sc[2 * g + 1];
                const float dd = d * xb->d;
                for (int k = 0; k < 8; k++) {
                    int s = 0;
                    for (int m = 0; m < 4; m++) {
                        const int l = 4 * k + m;
                        const int lo = ql[(g & 1) * 32 + l];
                        const int q6 = (g < 2 ? lo & 0xF : lo >> 4) | (((qh[l] >> (2 * g)) & 3) << 4);
                        s += q6 * xb->q[l];
                    }
                    s *= k < 4 ? sa : sbb;
                    acc[k] = fmaf((float)s, dd, acc[k]);
                }
                corr = fmaf(dd, (float)(sa * xb->s16[0] + sbb * xb->s16[1]), corr);
            }
        }
    }
    return hsum8(acc) - 32.0f * corr;
}

float orc_vec_dot_q8(int type, const uint8_t *w, const OrcQ8 *x, int64_t n)
{
    switch (type) {                                    /* src/kernels.c:223-231 */
    case ORC_T_Q4_0: return dot_q4_0(w, x, n / 32);
    case ORC_T_Q4_1: return dot_q4_1(w, x, n / 32);
    case ORC_T_Q6_K: return dot_q6_k(w, x, n / 256);
    default: return NAN;
    }
}

/* F32 dot (src/kernels.c:202-219): two 8-lane FMA accumulators over 16-element steps,
 * a lane-wise add, hsum256, then a scalar tail that gcc leaves as a multiply and an add. */
float orc_vec_dot_f32(const float *w, const float *x, int64_t n)
{
    float a0[8] = { 0 }, a1[8] = { 0 }, c[8];
    int64_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int k = 0; k < 8; k++) {
            a0[k] = fmaf(w[i + k], x[i + k], a0[k]);
            a1[k] = fmaf(w[i + 8 + k], x[i + 8 + k], a1[k]);
        }
    for (int k = 0; k < 8; k++) c[k] = a0[k] + a1[k];
    float s = hsum8(c);
    for (; i < n; i++) s += w[i] * x[i];
    return s;
}

void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* qms_matmul fast path (src/quant.c:128-170): quantise x once, one dot per (row, token). */
void orc_matmul(int type, int64_t rows, int64_t cols, const uint8_t *w, const float *x, int T, float *y)
{
    const uint64_t rb = orc_row_bytes(type, cols);
    const int64_t nb = cols / 32;
    OrcQ8 *xq = NULL;
    if (type != ORC_T_F32) {
        xq = (OrcQ8 *)malloc((size_t)T * nb * sizeof(OrcQ8));
        for (int t = 0; t < T; t++) orc_quantize_q8(x + (size_t)t * cols, cols, xq + (size_t)t * nb);
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *wr = w + (uint64_t)r * rb;
        for (int t = 0; t < T; t++)
            y[(size_t)t * rows + r] = type == ORC_T_F32
                ? orc_vec_dot_f32((const float *)wr, x + (size_t)t * cols, cols)
                : orc_vec_dot_q8(type, wr, xq + (size_t)t * nb, cols);
    }
    free(xq);
}

/* The same from activations already quantised, T rows of cols/32 blocks each: the reference
 * quantises a slot's input once and dots every row against it (src/model.c:979-988). */
void orc_matmul_q8(int type, int64_t rows, int64_t cols, const uint8_t *w, const OrcQ8 *xq, int T, float *y)
{
    const uint64_t rb = orc_row_bytes(type, cols);
    const int64_t nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int t = 0; t < T; t++)
            y[(size_t)t * rows + r] = orc_vec_dot_q8(type, w + (uint64_t)r * rb, xq + (size_t)t * nb, cols);
}

/* Router softmax, top-k and renormalisation (src/model.c:1043-1064): double softmax over all
 * experts, top-k by repeated argmax with strict '>' (ties go to the lower index), then
 * weights (float)(p / sum of the selected p) in selection order. */
void orc_route(const float *router, int X, int E, int K, const float *xn, int T,
               float *logits_out, int *sel, float *wts)
{
    float *logits = logits_out ? logits_out : (float *)malloc((size_t)T * X * sizeof(float));
    double *prob = (double *)malloc((size_t)X * sizeof(double));
    orc_matmul(ORC_T_F32, X, E, (const uint8_t *)router, xn, T, logits);
    for (int t = 0; t < T; t++) {
        const float *lt = logits + (size_t)t * X;
        double mx = -INFINITY, z = 0.0;
        for (int e = 0; e < X; e++) if (lt[e] > mx) mx = lt[e];
        for (int e = 0; e < X; e++) { prob[e] = exp((double)lt[e] - mx); z += prob[e]; }
        for (int e = 0; e < X; e++) prob[e] /= z;
        int *s = sel + (size_t)t * K;
        double wsum = 0.0;
        for (int j = 0; j < K; j++) {
            int best = -1;
            for (int e = 0; e < X; e++) {
                int taken = 0;
                for (int i = 0; i < j; i++) if (s[i] == e) { taken = 1; break; }
                if (!taken && (best < 0 || prob[e] > prob[best])) best = e;
            }
            s[j] = best;
            wsum += prob[best];
        }
        for (int j = 0; j < K; j++) wts[(size_t)t * K + j] = (float)(prob[s[j]] / wsum);
    }
    free(prob);
    if (!logits_out) free(logits);
}

/* SwiGLU (src/model.c:424 silu, :994 a = silu(g) * u). */
void orc_swiglu(const float *g, const float *u, int64_t n, float *a)
{
    for (int64_t j = 0; j < n; j++) {
        const float s = g[j] / (1.0f + expf(-g[j]));
        a[j] = s * u[j];
    }
}

static int fast_supported(int type)
{
    return type == ORC_T_Q4_0 || type == ORC_T_Q4_1 || type == ORC_T_Q6_K || type == ORC_T_F32;
}

/* The MoE block (src/model.c:1032-1167), resident fast path. Each (token, chosen expert) pair
 * gets gate/up dots against the token's Q8 row (moe_group_fast phase 1, :979-988), SwiGLU and
 * a Q8 re-quantisation of the F-vector (phase 2, :989-997) and down dots (phase 3, :998-1005).
 * Grouping slots by expert does not change any value, so pairs are visited token by token.
 * The combine sums w_j * dn_j in selection order with a contracted multiply-add (:1152-1162). */
int orc_moe(const OrcMoe *L, const float *xn, int T, float *out, int *sel_out, float *wts_out,
            float *logits_out)
{
    const int E = L->n_embd, X = L->n_expert, K = L->n_used, F = L->n_ff;
    const int fast = fast_supported(L->gate_type) && fast_supported(L->up_type) &&
                     fast_supported(L->down_type) && L->gate_type != ORC_T_F32 &&
                     L->down_type != ORC_T_F32 && E % 256 == 0 && F % 32 == 0;   /* :1090-1093 */
    if (!fast) return -1;
    int *sel = sel_out ? sel_out : (int *)malloc((size_t)T * K * sizeof(int));
    float *wts = wts_out ? wts_out : (float *)malloc((size_t)T * K * sizeof(float));
    orc_route(L->router, X, E, K, xn, T, logits_out, sel, wts);

    const uint64_t rb_g = orc_row_bytes(L->gate_type, E), rb_u = orc_row_bytes(L->up_type, E);
    const uint64_t rb_d = orc_row_bytes(L->down_type, F);
    const int nbE = E / 32, nbF = F / 32;
    OrcQ8 *xq = (OrcQ8 *)malloc((size_t)nbE * sizeof(OrcQ8));
    OrcQ8 *aq = (OrcQ8 *)malloc((size_t)nbF * sizeof(OrcQ8));
    float *g = (float *)malloc((size_t)F * sizeof(float));
    float *u = (float *)malloc((size_t)F * sizeof(float));
    float *a = (float *)malloc((size_t)F * sizeof(float));
    float *dn = (float *)malloc((size_t)E * sizeof(float));
    for (int t = 0; t < T; t++) {
        orc_quantize_q8(xn + (size_t)t * E, E, xq);
        float *ot = out + (size_t)t * E;
        for (int i = 0; i < E; i++) ot[i] = 0.0f;
        for (int j = 0; j < K; j++) {
            const int e = sel[t * K + j];
            const uint8_t *gw = L->gate + (uint64_t)e * F * rb_g;
            const uint8_t *uw = L->up + (uint64_t)e * F * rb_u;
            const uint8_t *dw = L->down + (uint64_t)e * E * rb_d;
#pragma omp parallel for schedule(static)
            for (int r = 0; r < F; r++) {
                g[r] = orc_vec_dot_q8(L->gate_type, gw + (uint64_t)r * rb_g, xq, E);
                u[r] = orc_vec_dot_q8(L->up_type, uw + (uint64_t)r * rb_u, xq, E);
            }
            orc_swiglu(g, u, F, a);
            orc_quantize_q8(a, F, aq);
#pragma omp parallel for schedule(static)
            for (int r = 0; r < E; r++) dn[r] = orc_vec_dot_q8(L->down_type, dw + (uint64_t)r * rb_d, aq, F);
            const float wj = wts[t * K + j];
            for (int i = 0; i < E; i++) ot[i] = fmaf(wj, dn[i], ot[i]);
        }
    }
    free(xq); free(aq); free(g); free(u); free(a); free(dn);
    if (!sel_out) free(sel);
    if (!wts_out) free(wts);
    (void)nbF;
    return 0;
}

/* ---- token sampler (src/chat.c:27-69) ------------------------------------------------------ */
/* PCG-XSH-RR step of the chat sampler's generator (chat.c:27-33). */
static uint32_t orc_pcg32(uint64_t *s)
{
    const uint64_t x = *s;
    *s = x * 6364136223846793005ull + 1442695040888963407ull;
    const uint32_t v = (uint32_t)(((x >> 18) ^ x) >> 27);
    const uint32_t r = (uint32_t)(x >> 59);
    return (v >> r) | (v << ((32u - r) & 31u));
}

/* Restatement of sample() (chat.c:36-69): argmax when temp <= 0 (first maximum); otherwise the
 * K largest logits (K = top_k when 0 < top_k < V, else min(V, 1024)) ordered by value descending,
 * lower index first among equals; weights exp((l_j - l_0) / temp) in double; the shortest prefix
 * whose normalised cumulative weight reaches top_p; one pcg32 draw scaled by that prefix's weight
 * picks the token. *rng advances once per tempered draw. */
int orc_sample(const float *l, int V, float temp, float top_p, int top_k, uint64_t *rng)
{
    int best = 0;
    for (int i = 1; i < V; i++)
        if (l[i] > l[best]) best = i;
    if (temp <= 0.0f) return best;
    const int K = (top_k > 0 && top_k < V) ? top_k : (V < 1024 ? V : 1024);
    int *ix = (int *)malloc((size_t)K * sizeof(int));
    double *w = (double *)malloc((size_t)K * sizeof(double));
    int n = 0;
    for (int i = 0; i < V; i++) {                 /* sorted insertion, ties keep the lower index first */
        if (n == K && !(l[i] > l[ix[K - 1]])) continue;
        int j = n < K ? n++ : K - 1;
        for (; j > 0 && l[ix[j - 1]] < l[i]; j--) ix[j] = ix[j - 1];
        ix[j] = i;
    }
    double z = 0.0;
    for (int j = 0; j < n; j++) {
        w[j] = exp(((double)l[ix[j]] - (double)l[ix[0]]) / (double)temp);
        z += w[j];
    }
    int keep = n;
    double c = 0.0;
    for (int j = 0; j < n; j++) {
        c += w[j] / z;
        if (c >= (double)top_p) {
            keep = j + 1;
            break;
        }
    }
    double zk = 0.0;
    for (int j = 0; j < keep; j++) zk += w[j];
    const double r = ((double)orc_pcg32(rng) / 4294967296.0) * zk;
    int pick = ix[keep - 1];
    double acc = 0.0;
    for (int j = 0; j < keep; j++) {
        acc += w[j];
        if (r < acc) {
            pick = ix[j];
            break;
        }
    }
    free(ix);
    free(w);
    return pick;
}
