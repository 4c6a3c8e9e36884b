/* A plain C (C99) caller of libqms_cuda, compiled against include/qms_cuda.h the way the
 * reference's sources would be: checks that the header is valid C, that the block layout is the
 * reference's, and that the entry points refuse bad arguments on the host before any device call.
 * It makes no compute call, so it runs on a machine without a GPU (argv[1] "nogpu": qms_cuda_init
 * must then fail with QMS_CUDA_ENODEV and leave a reason). Exit status 0 when every check holds. */
#include <stddef.h>
#include <stdio.h>
#include <string.h>

#include "qms_cuda.h"

static int failures = 0;

#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            fprintf(stderr, "FAIL line %d: %s (last error: %s)\n", __LINE__, #cond,   \
                    qms_cuda_last_error());                                           \
            failures++;                                                               \
        }                                                                             \
    } while (0)

static QmsCudaModelDesc model_desc(void) {
    static float norm[512];
    static unsigned char rows[16];
    QmsCudaModelDesc d;
    memset(&d, 0, sizeof d);
    d.n_layer = 2;
    d.n_embd = 512;
    d.n_head = 8;
    d.n_head_kv = 2;
    d.head_dim = 64;
    d.n_expert = 32;
    d.n_used = 4;
    d.n_ff = 256;
    d.vocab = 4096;
    d.eps = 1e-6f;
    d.rope_base = 1e6;
    d.ctx = 64;
    d.embd_type = QMS_T_Q4_0;
    d.embd = rows;
    d.out_norm = norm;
    d.output_type = QMS_T_Q6_K;
    d.output = rows;
    d.src_on_device = 0;
    return d;
}

int main(int argc, char **argv) {
    const int no_gpu = argc > 1 && strcmp(argv[1], "nogpu") == 0;
    float f[64];
    int i[64];
    QmsQ8 q[4];

    /* the reference's activation block (src/kernels.h:7-12): 44 bytes, d first, q last */
    CHECK(sizeof(QmsQ8) == 44);
    CHECK(offsetof(QmsQ8, d) == 0 && offsetof(QmsQ8, ds) == 4 && offsetof(QmsQ8, s16) == 8 &&
          offsetof(QmsQ8, q) == 12);

    if (no_gpu) {
        CHECK(qms_cuda_init(0) == QMS_CUDA_ENODEV);
        CHECK(qms_cuda_last_error()[0] != '\0');
    }

    /* kernel mirrors */
    CHECK(qms_cuda_quantize_q8(NULL, 32, 1, q, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_quantize_q8(f, 33, 1, q, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_matvec_q8(QMS_T_Q6_K, f, 4, 32, q, 1, f, NULL) == QMS_CUDA_EINVAL);

    /* MoE block and its expert-parallel phases */
    CHECK(qms_cuda_moe_forward(NULL, f, 1, f, NULL, NULL, NULL, NULL, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_moe_experts_q8(NULL, q, i, 4, f, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_ep_pack(f, i, 4, 4, 500, 32, 2, 16, q, i, i, NULL, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_ep_pack(f, i, 4, 4, 512, 32, 3, 16, q, i, i, NULL, NULL) == QMS_CUDA_EUNSUPPORTED);
    CHECK(qms_cuda_ep_pack(f, NULL, 4, 4, 512, 32, 2, 16, q, i, i, NULL, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_ep_combine(NULL, i, f, 4, 4, 512, NULL, f, NULL) == QMS_CUDA_EINVAL);
    CHECK(qms_cuda_ep_combine(f, i, f, 0, 4, 512, NULL, f, NULL) == QMS_CUDA_OK);

    /* routing without allocation: sizes past its fixed scratch */
    CHECK(qms_cuda_moe_route_noalloc(f, 128, 4096, 8, f, 65, i, f, NULL, NULL) == QMS_CUDA_EINVAL);

    /* chat sampler */
    CHECK(qms_cuda_sample(NULL, 10, 1.0f, 0.9f, 0, NULL, i, NULL) == QMS_CUDA_EINVAL);

    /* whole model: the configuration is checked before any device work */
    {
        QmsCudaModel *m = NULL;
        QmsCudaModelDesc d = model_desc();
        d.head_dim = 96;
        CHECK(qms_cuda_model_create(&d, &m) == QMS_CUDA_EUNSUPPORTED && m == NULL);
        d = model_desc();
        d.n_head = 6;
        d.n_head_kv = 4;
        CHECK(qms_cuda_model_create(&d, &m) == QMS_CUDA_EINVAL && m == NULL);
        d = model_desc();
        d.ctx = 0;
        CHECK(qms_cuda_model_create(&d, &m) == QMS_CUDA_EINVAL && m == NULL);
        CHECK(qms_cuda_forward(NULL, i, 1, 0, f, 0, NULL) == QMS_CUDA_EINVAL);
        CHECK(qms_cuda_forward_batch(NULL, 1, i, i, f) == QMS_CUDA_EINVAL);
        CHECK(qms_cuda_model_status(NULL) == QMS_CUDA_EINVAL);
        qms_cuda_model_free(NULL);
    }

    if (failures) {
        fprintf(stderr, "%d check(s) failed\n", failures);
        return 1;
    }
    printf("ok\n");
    return 0;
}
