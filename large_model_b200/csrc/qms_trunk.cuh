// qms_trunk.cuh - internal declarations of the trunk kernels (qms_trunk.cu): everything of a token
// step outside the MoE block. Not part of the C ABI.
#pragma once

#include "qms_common.cuh"

namespace qms {

// ---- repacked projection rows ------------------------------------------------------------------
// Q4_0 / Q4_1 row of nb blocks: nibble plane [nb][16 B], d plane [nb] fp16 (padded to 16 B),
// Q4_1 also an m plane [nb] fp16 (padded). Q6_K row of nsb super-blocks: body [nsb][208 B]
// (ql[128], qh[64], scales[16] as in ggml) then the d plane [nsb] fp16 (padded). The bytes and
// their meaning are the GGUF rows' own; only their order differs, so 128-bit loads stay aligned.
__host__ __device__ inline size_t pad16(size_t x) { return (x + 15) & ~(size_t)15; }
__host__ __device__ inline size_t rows_stride(int type, int ncol) {
    if (type == QMS_T_Q6_K) return (size_t)(ncol / 256) * 208 + pad16((size_t)(ncol / 256) * 2);
    const size_t nb = (size_t)ncol / 32;
    return nb * 16 + pad16(nb * 2) * (type == QMS_T_Q4_1 ? 2 : 1);
}
__host__ __device__ inline size_t ggml_row_bytes(int type, int ncol) {
    switch (type) {
    case QMS_T_F32: return (size_t)ncol * 4;
    case QMS_T_F16: return (size_t)ncol * 2;
    case QMS_T_Q4_0: return (size_t)ncol / 32 * 18;
    case QMS_T_Q4_1: return (size_t)ncol / 32 * 20;
    case QMS_T_Q8_0: return (size_t)ncol / 32 * 34;
    case QMS_T_Q6_K: return (size_t)ncol / 256 * 210;
    default: return 0;
    }
}

// Repack `rows` GGUF rows (device source) of type Q4_0 / Q4_1 / Q6_K into the layout above.
int repack_rows(int type, const uint8_t *src, int64_t rows, int ncol, uint8_t *dst, cudaStream_t s);

// ---- matrix-vector products over repacked rows ---------------------------------------------------
constexpr int kGemvTile = 8;          // tokens per pass (activations staged in shared memory)

struct GemvArgs {
    const uint8_t *w;                 // repacked rows
    size_t stride;                    // bytes per row
    int rows, ncol, T;
    // input, either fp32 rows x [T][ldx] quantised to Q8 in the prologue (optionally RMS-normed
    // with weight nw first; T <= kGemvTile), or Q8 rows already in global memory
    const float *x;
    int ldx;
    const float *nw;
    float eps;
    const int8_t *xq;                 // [T][ncol]
    const float *xd;                  // [T][ncol/32]
    const int *xs;                    // [T][ncol/32]: q-sum of the first 16 | second 16 << 16
    float *y;                         // y[t * ldy + r]
    int ldy;
    const float *resid;               // optional, same indexing as y (may equal y)
    // fused greedy argmax of y (T == 1): key slot, CTA ticket, token out, position to advance
    unsigned long long *amax;
    int *ticket;
    int *tok;
    int *pos;
    // multi-token projections: scratch for the partial sums when the blocks are split over CTAs
    // (kpart_n floats; NULL: no split)
    float *kpart;
    size_t kpart_n;
};
int launch_gemv(int type, const GemvArgs &a, cudaStream_t s);
// Several tokens (Q8 rows in xq / xd / xs) through Q4_0 / Q4_1 / Q6_K rows on int8 mma.sync;
// rows % 16 == 0.
int launch_gemm_q(int type, const GemvArgs &a, cudaStream_t s);

// One-token projection (decode): a persistent CTA per SM owns a contiguous range of rows and
// streams it through a ring of TMA bulk copies issued before griddepcontrol.wait. Input: fp32 x
// (RMS-normed with nw first when nw != NULL) quantised in the prologue, or Q8 rows (xq/xd/xs).
// y[r] = (resid ? resid[r] : 0) + dot; optional fused greedy argmax as in GemvArgs.
int launch_gemv1(int type, const GemvArgs &a, int *err, cudaStream_t s);

// ---- norms, embedding, attention ----------------------------------------------------------------
// y = RMSNorm(x) * w per row (src/model.c:403-409), optionally also as Q8 rows (xq / xd / xs as in
// GemvArgs); w == NULL quantises x unchanged.
int launch_rmsnorm(const float *x, const float *w, float eps, int T, int n, float *y, int8_t *xq, float *xd, int *xs,
                   cudaStream_t s);
// h[t] = dequant(embd row ids[t]) (src/model.c:1273); ids outside [0, vocab) write zeros and set err bit 2.
int launch_embed(int type, const uint8_t *embd, int vocab, int n, const int *ids, int T, float *h, int *err,
                 cudaStream_t s);

struct AttnArgs {
    float *qkv;                       // [T][ldq]: q (H*D) | k (Hk*D) | v (Hk*D) per token, from the projections
    int ldq;
    const float *q_norm, *k_norm;
    float eps;
    const float *rope_cos, *rope_sin; // [ctx][D/2]
    void *kc, *vc;                    // this layer's cache [ctx][Hk*D]: fp32, or fp16 when kv16
    int kv16;
    const int *pos;                   // device: position of token 0
    // several sequences (batched decode): token t belongs to sequence t, sits at position pos_vec[t]
    // and uses the caches at kc / vc + t * seq_stride; NULL: every token of one sequence
    const int *pos_vec;
    size_t seq_stride;
    int q_ready;                      // one-token attention: q rows already QK-normed and rotated and
                                      // the new K / V rows already in the cache (k_qk_rope ran)
    int T, ctx, H, Hk, D;
    double scale;                     // 1/sqrt(D)
    int max_splits;
    float *part_o;                    // one-token attention partials [T][H][max_splits][D]
    double *part_ml;                  // [T][H][max_splits][2]
    float *out;                       // [T][H*D]
    int *err;
};
// One-token attention (decode): CTA (kv head, 32 positions, sequence) with QK-norm, RoPE and the
// K/V append of the new position fused in; partials merged by k_attn_merge, which writes the Q8
// rows of the attention output for the O projection (xq / xd / xs as in GemvArgs). T == 1, or a
// batch (pos_vec): one token for each of T sequences.
int launch_attn_decode(const AttnArgs &a, int8_t *xq, float *xd, int *xs, cudaStream_t s);
constexpr int kAttnBlock = 32;        // positions per decode-attention CTA
constexpr int kAttnMaxCtx = 16384;    // longest context the one-token attention merges

// QK-norm + NEOX RoPE of every q / k head and the fp32 K/V append (src/model.c:441-462).
int launch_qk_rope(const AttnArgs &a, cudaStream_t s);
// Causal GQA attention with the reference's score order (src/model.c:465-492).
int launch_attention(const AttnArgs &a, cudaStream_t s);
// Greedy argmax of each of B rows of logits [B][ld] over V columns (ties: the lower index, as the
// reference's '>' scan): tok[b] = the winner, pos[b] += 1 when pos is not NULL.
int launch_argmax_rows(const float *logits, int ld, int B, int V, int *tok, int *pos, cudaStream_t s);
int attention_heads_per_cta(int group);

}  // namespace qms
