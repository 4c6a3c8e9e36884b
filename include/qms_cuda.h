/* qms_cuda.h - C ABI of libqms_cuda: the B200 (sm_100a) Qwen3-MoE feed-forward path.
 *
 * Plain C types only (pointers, sizes, ints); streams are passed as `void *` (a cudaStream_t,
 * NULL = the legacy default stream). Every function returns an int status (QMS_CUDA_OK = 0,
 * negative on failure) and records a one-line reason readable with qms_cuda_last_error(),
 * like the reference's 0 / -1 returns with the reason printed to stderr (src/model.h:135-141).
 * There is no CPU fallback: without a usable sm_100 device every compute call fails.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   qms_quantize_q8            src/kernels.h:15   (src/kernels.c:34-53)
 *   qms_vec_dot_q8/qms_matmul  src/kernels.h:19, src/quant.h:23-26 (src/quant.c:128-170)
 *   qms_vec_dot_f32            src/kernels.h:21   (src/kernels.c:202-221)
 *   moe()                      src/model.c:1032-1167, called from qms_forward (src/model.c:1284)
 *   sample() (chat sampler)    src/chat.c:36-69 with pcg32() src/chat.c:27-33
 */
#ifndef QMS_CUDA_H
#define QMS_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor type ids, GGUF numbering (src/gguf.h:8-10). A translation unit that also includes
 * the reference's gguf.h (include guard QMS_GGUF_H) gets the same values from there. */
#ifndef QMS_GGUF_H
enum { QMS_T_F32 = 0, QMS_T_F16 = 1, QMS_T_Q4_0 = 2, QMS_T_Q4_1 = 3, QMS_T_Q8_0 = 8, QMS_T_Q6_K = 14 };
#endif

/* Status codes. */
enum {
    QMS_CUDA_OK = 0,
    QMS_CUDA_EINVAL = -1,       /* bad argument or shape */
    QMS_CUDA_ECUDA = -2,        /* a CUDA runtime call failed */
    QMS_CUDA_ENOMEM = -3,       /* device allocation failed */
    QMS_CUDA_EUNSUPPORTED = -4, /* type/shape outside what the kernels implement */
    QMS_CUDA_ENODEV = -5,       /* no sm_100 device */
    QMS_CUDA_ETIMEOUT = -6      /* a bounded wait inside a kernel gave up (see qms_cuda_moe_status) */
};

/* Activation block: 32 int8 values with one fp32 scale; same 44-byte layout as the
 * reference's QmsQ8 (src/kernels.h:7-12), which a translation unit that includes the reference's
 * kernels.h (include guard QMS_KERNELS_H) uses instead. */
#ifndef QMS_KERNELS_H
typedef struct {
    float d;         /* scale: x ~= q * d */
    float ds;        /* d * sum(q[0..31]) */
    int16_t s16[2];  /* sum(q[0..15]), sum(q[16..31]) */
    int8_t q[32];
} QmsQ8;
#endif

/* ---- library ---------------------------------------------------------------------------- */

/* Reason for the last failure on the calling thread ("" when none). */
const char *qms_cuda_last_error(void);
/* Select and check `device` (must be sm_100). Replaces nothing in the reference (CPU only). */
int qms_cuda_init(int device);
/* Number of visible CUDA devices, or a negative status. */
int qms_cuda_device_count(void);
/* Wait for all work queued on `stream`. */
int qms_cuda_stream_sync(void *stream);

/* ---- kernel-level mirrors (device pointers) ------------------------------------------------ */

/* Quantise `rows` rows of n floats (n % 32 == 0) to n/32 QmsQ8 blocks each, bit-identical to
 * qms_quantize_q8 (src/kernels.h:15, src/kernels.c:34-53). */
int qms_cuda_quantize_q8(const float *x, int64_t n, int64_t rows, QmsQ8 *out, void *stream);

/* y[t][r] = dot(W row r, xq[t]) for a GGUF-layout weight matrix (rows x cols, type Q4_0, Q4_1
 * or Q6_K) and T quantised activation rows: the integer fast path of qms_matmul / qms_vec_dot_q8
 * (src/quant.h:23, src/kernels.h:19, src/quant.c:128-170). */
int qms_cuda_matvec_q8(int type, const void *w, int64_t rows, int64_t cols, const QmsQ8 *xq,
                       int T, float *y, void *stream);

/* y[t][r] = dot(W row r, x[t]) for an F32 matrix, in qms_vec_dot_f32's exact AVX2 summation
 * order (src/kernels.h:21, src/kernels.c:202-221), so router logits are bit-identical. */
int qms_cuda_matvec_f32(const float *w, int64_t rows, int64_t cols, const float *x, int T,
                        float *y, void *stream);

/* ---- MoE feed-forward block (src/model.c:1032-1167) ---------------------------------------- */

/* One MoE layer as the reference loads it (src/model.c:359-362, model.h:229-243):
 * router F32 [n_expert][n_embd]; gate/up stacked [n_expert][n_ff] rows of n_embd;
 * down stacked [n_expert][n_embd] rows of n_ff; ggml block layouts. */
typedef struct {
    int n_embd, n_expert, n_used, n_ff;
    int gate_type, up_type, down_type;
    const float *router;
    const void *gate, *up, *down;
    int src_on_device;          /* 1: the five pointers are device memory; 0: host memory */
} QmsCudaMoeDesc;

typedef struct QmsCudaMoe QmsCudaMoe;

/* Upload (or copy from device) and repack one layer into HBM on the current device. The
 * source buffers are not retained. Replaces load_experts / load_mat for one layer
 * (src/model.c:133-157, 359-362). Types: gate and up Q4_0; down Q4_0 or Q4_1 (the GGUF mixes
 * that store ffn_down_exps one step wider); anything else is QMS_CUDA_EUNSUPPORTED. */
int qms_cuda_moe_create(const QmsCudaMoeDesc *desc, QmsCudaMoe **out);
void qms_cuda_moe_destroy(QmsCudaMoe *m);
/* Bytes of device memory held by the layer (weights + scratch). */
int64_t qms_cuda_moe_device_bytes(const QmsCudaMoe *m);
/* Make sure scratch for T tokens exists (T * n_used <= 65535). Forward calls do this themselves;
 * call it before capturing forward calls into a CUDA graph (no allocation may happen during
 * capture). Growing the scratch moves it, so graphs captured on this layer before any call that
 * grows it (a larger T, or an expert call with more rows) no longer apply. */
int qms_cuda_moe_reserve(QmsCudaMoe *m, int T);

/* out[t] = sum_j w[t][j] * FFN_{sel[t][j]}(xn[t]) for T tokens: moe(m, l, xn, h, T, out)
 * (src/model.c:1032). xn, out: device fp32 [T][n_embd]. Optional device outputs (NULL to skip):
 * sel [T][n_used] selected experts in selection order, wts [T][n_used] renormalised weights,
 * logits [T][n_expert] router logits. resid (optional, device [T][n_embd]): when non-NULL
 * out = resid + moe(xn), the residual add of qms_forward (src/model.c:1285). */
int qms_cuda_moe_forward(QmsCudaMoe *m, const float *xn, int T, float *out, int *sel,
                         float *wts, float *logits, const float *resid, void *stream);

/* ---- expert parallelism: route, expert FFNs, combine (no reference counterpart; the reference
 * runs every expert in one process). A full layer runs them inside qms_cuda_moe_forward; a
 * shard runs them under the caller's dispatch (all-to-all of rows, see large_model_b200/ep.py). */

/* A layer holding experts [expert_base, expert_base + n_local) of the desc's n_expert routed
 * ones: desc->router has all n_expert rows; desc->gate/up/down hold only the n_local experts
 * (stacked in expert order). qms_cuda_moe_forward is refused on a shard. */
int qms_cuda_moe_create_shard(const QmsCudaMoeDesc *desc, int expert_base, int n_local, QmsCudaMoe **out);
/* Routing only (src/model.c:1043-1064): sel [T][n_used] (global expert ids, selection order) and
 * wts [T][n_used], optional logits [T][n_expert]; device buffers. */
int qms_cuda_moe_route(QmsCudaMoe *m, const float *xn, int T, int *sel, float *wts, float *logits, void *stream);
/* Expert FFNs of S rows (moe_group_fast's phases 1-3 for one slot each, src/model.c:979-1005):
 * x [S][n_embd] fp32, expert[S] local ids (0 .. n_local - 1), dn [S][n_embd] receives each row's
 * down projection before weighting. Rows with an out-of-range id are skipped (dn left as is).
 * S <= 2^21; the layer's scratch grows to S rows on the first call that needs it (outside graph
 * capture). Runs the grouped tensor-core kernels; device buffers. */
int qms_cuda_moe_experts(QmsCudaMoe *m, const float *x, const int *expert, int S, float *dn, void *stream);
/* The same from rows already quantised: xq [S][n_embd/32] QmsQ8 blocks (e.g. from
 * qms_cuda_quantize_q8, bit-identical to the reference's quantiser), so a dispatch sends 44 bytes
 * per 32 values instead of 128 (moe_group_fast quantises each slot's input once, src/model.c:979-988).
 * The results equal qms_cuda_moe_experts on the fp32 rows. */
int qms_cuda_moe_experts_q8(QmsCudaMoe *m, const QmsQ8 *xq, const int *expert, int S, float *dn, void *stream);
/* out[t] = resid[t] + sum_j wts[t][j] * dn[t * n_used + j] in selection order (src/model.c:1152-1162);
 * resid may be NULL; device buffers. */
int qms_cuda_moe_combine(const float *dn, const float *wts, int T, int n_used, int n_embd, const float *resid,
                         float *out, void *stream);

/* ---- expert parallelism with fixed-capacity buffers (no counterpart in the CPU-only reference;
 * each slot's arithmetic is moe_group_fast's, src/model.c:979-1005, and the combine order is
 * src/model.c:1152-1162) -------------------------------------------------------------------------
 * Rank r of n_rank holds experts [r * n_expert / n_rank, (r + 1) * n_expert / n_rank) as a shard
 * layer. One layer call on every rank, with nothing read back to the host:
 *   1. qms_cuda_moe_route                      sel, wts for its T tokens;
 *   2. qms_cuda_ep_pack                        send_x / send_e: n_rank segments of cap entries;
 *   3. all-to-all of segment o to rank o       send_x (cap * n_embd/32 QmsQ8 blocks per segment)
 *                                              and send_e (cap ints per segment) -> recv_x, recv_e;
 *   4. qms_cuda_moe_experts_q8(shard, recv_x, recv_e, n_rank * cap, dn_recv): unused entries
 *      carry id -1 and are skipped;
 *   5. all-to-all of dn_recv (cap * n_embd floats per segment) back -> ret;
 *   6. qms_cuda_ep_combine(ret, slot, wts, ...).
 * Every segment has the same size on every rank, so the exchange needs no counts: NCCL
 * send/recv pairs in one group from C, or all_to_all_single. cap = (largest T of any rank) *
 * n_used never overflows; a smaller cap moves fewer bytes, and a slot past its segment's capacity
 * is dropped, sets *err (when err is not NULL) and makes its token's output NaN.
 *
 * Pack: sel [T][n_used] global expert ids (selection order), xn [T][n_embd] fp32; writes the
 * owner's local expert id of every used entry and -1 of every unused one into send_e
 * [n_rank][cap], each token's Q8 row (the reference's quantiser) into send_x [n_rank][cap][n_embd/32]
 * at every entry one of its slots was given, and slot [T][n_used] = o * cap + (index of the slot
 * among the slots owned by o, in slot order), or -1 when dropped. T may be 0 (send_e is still
 * cleared). n_rank <= 64 and n_expert % n_rank == 0. Device buffers; no host synchronisation. */
int qms_cuda_ep_pack(const float *xn, const int *sel, int T, int n_used, int n_embd, int n_expert, int n_rank,
                     int cap, QmsQ8 *send_x, int *send_e, int *slot, int *err, void *stream);
/* out[t] = resid[t] + sum_j wts[t][j] * ret[slot[t][j]] in selection order, the arithmetic of
 * qms_cuda_moe_combine: ret [n_rank * cap][n_embd] holds the down rows returned by step 5;
 * resid may be NULL. T <= 65535. Device buffers. */
int qms_cuda_ep_combine(const float *ret, const int *slot, const float *wts, int T, int n_used, int n_embd,
                        const float *resid, float *out, void *stream);

/* ---- chat path: token sampling on the device (src/chat.c:27-69) -------------------------------- */

/* One draw of the reference's sampler, sample() (src/chat.c:36-69), on device memory: logits
 * [vocab] fp32; temp <= 0 gives the argmax (first index among equal maxima); otherwise the K
 * largest logits (K = top_k when 0 < top_k < vocab, else min(vocab, 1024)), weights
 * exp((l - l_max) / temp) in double, the top-p prefix and one pcg32 draw (chat.c:27-33) from
 * *rng, which is advanced. rng (device uint64) may be NULL when temp <= 0; *token (device int)
 * receives the id. K above 1024 is QMS_CUDA_EUNSUPPORTED. Logits must be finite. */
int qms_cuda_sample(const float *logits, int vocab, float temp, float top_p, int top_k, uint64_t *rng,
                    int *token, void *stream);

/* Waits for the device and reports whether any bounded wait inside the layer's kernels gave up
 * since the last call (QMS_CUDA_ETIMEOUT; the outputs of the affected call are invalid), then
 * clears the flag. The batch-1 kernels never spin without a limit, so a stuck pipeline turns into
 * this status instead of a hung GPU. No reference counterpart (the reference has no device). */
int qms_cuda_moe_status(QmsCudaMoe *m);

/* Kernel timing hook: with events non-NULL (an array of 6 cudaEvent_t), every following forward
 * records events[2i] before and events[2i+1] after its stage i on the launch stream. For T == 1
 * the whole block is one kernel (routing, gate/up, SwiGLU, down, combine): it is stage 1, and
 * stages 0 and 2 are empty. For T > 1 stage 0 is routing, stage 1 gate/up + SwiGLU and stage 2
 * down + combine. The events serialise the kernels (no programmatic overlap). NULL turns the
 * hook off. */
int qms_cuda_moe_set_kernel_events(QmsCudaMoe *m, void **events);

/* Same through host buffers (xn, out and the optional outputs in host memory): copies in,
 * runs, copies out and waits; the drop-in for the reference's host-memory moe() call. */
int qms_cuda_moe_forward_host(QmsCudaMoe *m, const float *xn, int T, float *out, int *sel,
                              float *wts, float *logits);

/* ---- whole model on the device: qms_model_load / qms_forward (src/model.h:135-141) ------------- */

/* Model configuration and the trunk tensors, as read_cfg and qms_model_load hold them
 * (src/model.c:279-312, :314-338). Tensors are in GGUF/ggml block layout, host memory
 * (src_on_device 0) or device memory (1); they are copied (and repacked) on the current device and
 * not retained. output == NULL means tied embeddings (the head multiplies by token_embd, as
 * src/model.c:333-335 does). Supported types: embd Q4_0, Q4_1, Q8_0, Q6_K, F16 or F32; output
 * (or tied embd) Q4_0, Q4_1 or Q6_K; n_embd % 256 == 0, head_dim 64 or 128 (<= QMS_MAX_HEAD_DIM). */
typedef struct {
    int n_layer, n_embd, n_head, n_head_kv, head_dim;
    int n_expert, n_used, n_ff, vocab;
    float eps;                 /* RMSNorm epsilon (the reference stores (float) of the GGUF value) */
    double rope_base;          /* NEOX RoPE base */
    int ctx;                   /* KV cache capacity in positions (fp32 K and V, [layer][pos][n_head_kv*head_dim]) */
    int embd_type;
    const void *embd;          /* token_embd.weight [vocab] rows of n_embd */
    const float *out_norm;     /* output_norm.weight [n_embd] */
    int output_type;
    const void *output;        /* output.weight [vocab] rows of n_embd, or NULL (tied) */
    int src_on_device;
} QmsCudaModelDesc;

/* One layer's tensors (QmsLayer, src/model.h:37-45): norms F32; q [n_head*head_dim], k and v
 * [n_head_kv*head_dim] rows of n_embd, o [n_embd] rows of n_head*head_dim, all Q4_0 or Q4_1;
 * moe.* the MoE block exactly as for qms_cuda_moe_create (its n_* fields must match the model). */
typedef struct {
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
    int q_type, k_type, v_type, o_type;
    const void *q, *k, *v, *o;
    QmsCudaMoeDesc moe;
} QmsCudaLayerDesc;

typedef struct QmsCudaModel QmsCudaModel;

/* Allocate the model on the current device: trunk tensors, KV cache for desc->ctx positions and
 * the forward's scratch. Layers are added with qms_cuda_model_set_layer; a forward before every
 * layer is set fails. Replaces qms_model_load's allocation and reads (src/model.c:314-387). */
int qms_cuda_model_create(const QmsCudaModelDesc *desc, QmsCudaModel **out);
/* Upload layer l (0 <= l < n_layer); the source buffers may be freed afterwards, so a loader can
 * stream a GGUF file layer by layer with one layer of host memory. */
int qms_cuda_model_set_layer(QmsCudaModel *m, int l, const QmsCudaLayerDesc *ld);
void qms_cuda_model_free(QmsCudaModel *m);
/* Device bytes held (weights, KV cache, scratch). */
int64_t qms_cuda_model_device_bytes(const QmsCudaModel *m);

/* qms_forward (src/model.c:1252-1296) on host buffers: T tokens ids[0..T) at positions
 * pos0..pos0+T-1, appending to the KV cache; logits (host fp32) receives [vocab] for the last
 * position, or [T][vocab] when all_logits. Embedding dequant, per layer RMSNorm -> attention
 * (QKV projections, QK-norm, NEOX RoPE, fp32 KV append, causal GQA, O projection) -> residual ->
 * RMSNorm -> MoE -> residual, final RMSNorm and the head, all on the device; returns after the
 * logits are on the host. pos0 + T > ctx or an id outside [0, vocab) is QMS_CUDA_EINVAL (the
 * reference returns -1, src/model.c:1257,1264). sel_trace, when non-NULL (host int
 * [n_layer][T][n_used]), receives every layer's selected experts in selection order, from which a
 * caller writes the reference's --trace records (src/model.c:1102-1110). */
int qms_cuda_forward(QmsCudaModel *m, const int *ids, int T, int pos0, float *logits, int all_logits,
                     int *sel_trace);

/* The same on device buffers, asynchronously on `stream`: ids (device int [T]); *pos (device int)
 * is the position of ids[0] and is read by the kernels, so a captured graph can be replayed as
 * the position advances. logits: device fp32 [all_logits ? T : 1][vocab]. 1 <= T <= 256; positions
 * beyond ctx or invalid ids are not written and set the error reported by qms_cuda_model_status. */
int qms_cuda_forward_dev(QmsCudaModel *m, const int *ids, int T, const int *pos, float *logits,
                         int all_logits, void *stream);
/* One greedy decode step entirely on the device (src/main.c:198-207, inc mode): the token *tok at
 * position *pos (device ints) runs through the model; the argmax of its logits (first index
 * among equal maxima, as argmax() in src/main.c) is written back to *tok, *pos is incremented,
 * and logits (device fp32 [vocab], optional) receive the step's logits. Graph-capturable: a graph
 * of N steps generates N tokens with no host round trip. */
int qms_cuda_decode_step(QmsCudaModel *m, int *tok, int *pos, float *logits, void *stream);

/* Several sequences. The reference serves one sequence per model (src/model.h:116-118,
 * qms_forward's KV cache); the device model can hold n_seq KV caches of ctx positions each.
 * set_sequences reallocates them (all positions cleared; sequence 0 is the one qms_cuda_forward
 * uses); n_seq * n_layer * ctx * 4 KB of device memory for 235B-shape layers. No other call may
 * be running, and CUDA graphs captured before no longer apply. */
int qms_cuda_model_set_sequences(QmsCudaModel *m, int n_seq);
/* The KV caches' element type: QMS_T_F32 (default: the reference's fp32 cache, src/model.c:459-460)
 * or QMS_T_F16 (compacted: half the memory and the attention's cache traffic; each K / V value is
 * rounded to fp16 once when appended, so results depart from the reference's by that rounding).
 * Reallocates and clears every sequence's cache, like set_sequences. */
int qms_cuda_model_set_kv_type(QmsCudaModel *m, int kv_type);
/* Copy positions [0, npos) of sequence src's cache to sequence dst (a shared prompt prefix). */
int qms_cuda_model_copy_sequence(QmsCudaModel *m, int src, int dst, int npos);
/* qms_cuda_forward on sequence seq's cache (qms_cuda_forward is seq 0). */
int qms_cuda_forward_seq(QmsCudaModel *m, int seq, const int *ids, int T, int pos0, float *logits,
                         int all_logits, int *sel_trace);
/* One token for each of B sequences in one pass (batched decode): sequence b (0 <= b < B) takes
 * ids[b] at position pos[b]; logits: host fp32 [B][vocab]. Host buffers, synchronous; each row is
 * what qms_cuda_forward_seq(m, b, &ids[b], 1, pos[b], ...) would return, up to the float
 * summation order of the multi-token kernels. B <= n_seq and B <= 256. */
int qms_cuda_forward_batch(QmsCudaModel *m, int B, const int *ids, const int *pos, float *logits);
/* The same on the device, greedy: tok[B], pos[B] device ints; each row's argmax (first index among
 * equal maxima) is written back to tok[b] and pos[b] is incremented; logits (device fp32 [B][vocab])
 * optional. Graph-capturable. */
int qms_cuda_decode_batch(QmsCudaModel *m, int B, int *tok, int *pos, float *logits, void *stream);
/* The forward's scratch covers up to 256 tokens per pass from creation on (longer calls run in
 * passes of 256), so device pointers never move and captured graphs stay valid; T > 256 is
 * QMS_CUDA_EINVAL. */
int qms_cuda_model_reserve(QmsCudaModel *m, int T);
/* Waits for the device; QMS_CUDA_EINVAL if a device-side check (position beyond ctx, bad id)
 * refused work since the last call, QMS_CUDA_ETIMEOUT if a MoE kernel's bounded wait gave up. */
int qms_cuda_model_status(QmsCudaModel *m);
/* QMS_PROF-style section timers (src/model.h:143-150): with on != 0, every following
 * qms_cuda_forward records CUDA events around its sections and adds their device time in ms to
 * ms[0..6] = qkv, attn, o_proj, router, fetch (always 0: weights are resident), moe, output.
 * For one-token calls routing runs inside the MoE kernel and is counted under moe. ms may be NULL
 * to only switch; reading (ms non-NULL) returns the sums and clears them. */
int qms_cuda_model_profile(QmsCudaModel *m, int on, double *ms);

/* Routing that allocates nothing. It has no counterpart in the reference (the reference
 * allocates freely on the host); it exists for callers that may not call cudaMalloc, such as
 * code running under another framework's memory pool or allocator hooks, plugin hosts that
 * forbid device allocation after start-up, or deployments that reserve all of HBM up front.
 * Computes what qms_cuda_moe_forward reports as sel / wts / logits: router F32 [n_expert][n_embd]
 * (16-byte aligned) against xn [T][n_embd]; sel [T][n_used] in selection order, wts [T][n_used],
 * logits [T][n_expert] (optional, NULL to skip); all device pointers supplied by the caller.
 * Its scratch lives in one fixed device array inside the library (384.25 KiB on every GPU that
 * loads it, kept until exit): T <= 64, n_embd <= 4096 (multiple of 256), n_expert <= 256 and
 * <= n_embd / 2, n_used <= min(n_expert, 64); larger sizes return QMS_CUDA_EINVAL with a message.
 * qms_cuda_init(device) loads the library's device code (and so the array) and looks up the
 * array's address for that device, so a caller that reserves the rest of HBM afterwards still has
 * it; without qms_cuda_init, the first call on each device does that (make it before any stream
 * capture). Every call looks the address up in the current context (a host-side query), so a
 * device reset or a new context never leaves a stale address. All calls share the one array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller. */
int qms_cuda_moe_route_noalloc(const float *router, int n_expert, int n_embd, int n_used,
                               const float *xn, int T, int *sel, float *wts, float *logits,
                               void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QMS_CUDA_H */
