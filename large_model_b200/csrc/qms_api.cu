// qms_api.cu - library state and the kernel-level mirrors of src/kernels.h (sm_100a).
#include <stdarg.h>
#include <string.h>

#include "qms_common.cuh"
#include "qms_router.cuh"

namespace qms {

int route_scratch_ptr(int dev, unsigned char **out);   // qms_moe.cu

static thread_local char g_err[512];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

// ---- qms_quantize_q8 (src/kernels.c:34-53): one warp per 32-block -------------------------
__global__ void k_quantize_q8_aos(const float *__restrict__ x, int64_t nblocks, QmsQ8 *__restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (b >= nblocks) return;
    const int lane = threadIdx.x & 31;
    const Q8Lane r = quantize_lane(x[b * 32 + lane]);
    QmsQ8 *o = out + b;
    o->q[lane] = (int8_t)r.q;
    if (lane == 0) {
        o->d = r.d;
        o->ds = __fmul_rn(r.d, (float)r.sum);
        o->s16[0] = (int16_t)r.sum_lo;
        o->s16[1] = (int16_t)(r.sum - r.sum_lo);
    }
}

// ---- qms_vec_dot_q8 on GGUF-layout rows: one warp per (row, token) -----------------------
// Q4_0/Q4_1 blocks are 18/20 bytes (2-byte aligned), read as halves; a lane takes blocks
// lane, lane+32, ...; the warp sum is the row's dot. Accumulation order differs from the AVX2
// lanes, so results agree with the reference to float rounding (|d| / sum|terms| ~ 1e-7).
__device__ __forceinline__ uint32_t ld_u32_from_halves(const uint16_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 16);
}

__device__ __forceinline__ int4 ld_q8_words(const QmsQ8 *x, int half) {
    const int *q = reinterpret_cast<const int *>(x->q) + half * 4;
    return make_int4(q[0], q[1], q[2], q[3]);
}

__global__ void k_matvec_q8_gguf(int type, const uint8_t *__restrict__ w, int64_t rows, int64_t cols,
                                 size_t rb, const QmsQ8 *__restrict__ xq, float *__restrict__ y) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int t = blockIdx.y;
    if (r >= rows) return;
    const int lane = threadIdx.x & 31;
    const uint8_t *row = w + (size_t)r * rb;
    const QmsQ8 *xt = xq + (size_t)t * (cols / 32);
    float acc = 0.0f;
    if (type == QMS_T_Q4_0 || type == QMS_T_Q4_1) {
        const int bs = type == QMS_T_Q4_0 ? 18 : 20;
        const int nb = (int)(cols / 32);
        for (int b = lane; b < nb; b += 32) {
            const uint16_t *blk = reinterpret_cast<const uint16_t *>(row + (size_t)b * bs);
            const float dw = h2f(blk[0]);
            const uint16_t *qs = blk + (type == QMS_T_Q4_0 ? 1 : 2);
            const uint4 nib = make_uint4(ld_u32_from_halves(qs), ld_u32_from_halves(qs + 2),
                                         ld_u32_from_halves(qs + 4), ld_u32_from_halves(qs + 6));
            const QmsQ8 *xb = xt + b;
            const int isum = q4_block_isum(nib, ld_q8_words(xb, 0), ld_q8_words(xb, 1));
            if (type == QMS_T_Q4_0) {
                const int sq = (int)xb->s16[0] + (int)xb->s16[1];
                acc = fmaf((float)(isum - 8 * sq), dw * xb->d, acc);
            } else {
                const float mw = h2f(blk[1]);
                acc = fmaf((float)isum, dw * xb->d, acc);
                acc = fmaf(mw, xb->ds, acc);
            }
        }
    } else {  // Q6_K: 256-element super-blocks of 210 bytes; a lane takes one 32-group at a time
        const int ng = (int)(cols / 32);
        for (int gi = lane; gi < ng; gi += 32) {
            const int sb = gi / 8, half = (gi / 4) & 1, g = gi & 3;
            const uint8_t *s = row + (size_t)sb * 210;
            const uint8_t *ql = s + half * 64 + (g & 1) * 32;
            const uint8_t *qh = s + 128 + half * 32;
            const int8_t *sc = reinterpret_cast<const int8_t *>(s + 192 + half * 8 + 2 * g);
            const float d = h2f(*reinterpret_cast<const uint16_t *>(s + 208));
            const QmsQ8 *xb = xt + gi;
            int s_lo = 0, s_hi = 0;
            for (int l = 0; l < 32; l++) {
                const int lo = ql[l];
                const int q6 = (g < 2 ? lo & 0xF : lo >> 4) | (((qh[l] >> (2 * g)) & 3) << 4);
                if (l < 16) s_lo += q6 * xb->q[l]; else s_hi += q6 * xb->q[l];
            }
            const int isum = sc[0] * (s_lo - 32 * xb->s16[0]) + sc[1] * (s_hi - 32 * xb->s16[1]);
            acc = fmaf((float)isum, d * xb->d, acc);
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) y[(size_t)t * rows + r] = acc;
}

}  // namespace qms

using namespace qms;

extern "C" {

const char *qms_cuda_last_error(void) { return g_err; }

int qms_cuda_device_count(void) {
    int n = 0;
    QMS_CK(cudaGetDeviceCount(&n));
    return n;
}

int qms_cuda_init(int device) {
    clear_error();
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        set_error("no CUDA device");
        return QMS_CUDA_ENODEV;
    }
    QMS_REQUIRE(device >= 0 && device < n, QMS_CUDA_EINVAL, "device %d out of range (%d devices)", device, n);
    QMS_CK(cudaSetDevice(device));
    cudaDeviceProp p;
    QMS_CK(cudaGetDeviceProperties(&p, device));
    QMS_REQUIRE(p.major == 10 && p.minor == 0, QMS_CUDA_ENODEV,
                "device %d is sm_%d%d; libqms_cuda is built for sm_100a only", device, p.major, p.minor);
    // load the module holding the fixed routing scratch now (lazy module loading would otherwise
    // allocate it at the first qms_cuda_moe_route_noalloc call) and cache its address
    unsigned char *scratch = nullptr;
    return route_scratch_ptr(device, &scratch);
}

int qms_cuda_stream_sync(void *stream) {
    QMS_CK(cudaStreamSynchronize((cudaStream_t)stream));
    return QMS_CUDA_OK;
}

int qms_cuda_quantize_q8(const float *x, int64_t n, int64_t rows, QmsQ8 *out, void *stream) {
    QMS_REQUIRE(x && out && n > 0 && n % 32 == 0 && rows >= 0, QMS_CUDA_EINVAL,
                "quantize_q8: n must be a positive multiple of 32");
    const int64_t nblocks = rows * (n / 32);
    if (nblocks == 0) return QMS_CUDA_OK;
    const int wpb = 8;
    k_quantize_q8_aos<<<(unsigned)((nblocks + wpb - 1) / wpb), wpb * 32, 0, (cudaStream_t)stream>>>(x, nblocks, out);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

int qms_cuda_matvec_q8(int type, const void *w, int64_t rows, int64_t cols, const QmsQ8 *xq, int T, float *y,
                       void *stream) {
    QMS_REQUIRE(w && xq && y && rows > 0 && T >= 0, QMS_CUDA_EINVAL, "matvec_q8: bad arguments");
    QMS_REQUIRE(type == QMS_T_Q4_0 || type == QMS_T_Q4_1 || type == QMS_T_Q6_K, QMS_CUDA_EUNSUPPORTED,
                "matvec_q8: type %d not supported (Q4_0, Q4_1, Q6_K)", type);
    QMS_REQUIRE(cols % (type == QMS_T_Q6_K ? 256 : 32) == 0, QMS_CUDA_EINVAL,
                "matvec_q8: cols %lld not a multiple of the block size", (long long)cols);
    QMS_REQUIRE(((uintptr_t)w & 1) == 0 && ((uintptr_t)xq & 3) == 0, QMS_CUDA_EINVAL,
                "matvec_q8: misaligned weight or activation pointer");
    QMS_REQUIRE(T <= 65535, QMS_CUDA_EINVAL, "matvec_q8: T %d > 65535", T);
    if (T == 0) return QMS_CUDA_OK;
    const size_t rb = type == QMS_T_Q4_0 ? (size_t)cols / 32 * 18
                      : type == QMS_T_Q4_1 ? (size_t)cols / 32 * 20 : (size_t)cols / 256 * 210;
    const int wpb = 8;
    dim3 grid((unsigned)((rows + wpb - 1) / wpb), (unsigned)T);
    k_matvec_q8_gguf<<<grid, wpb * 32, 0, (cudaStream_t)stream>>>(type, (const uint8_t *)w, rows, cols, rb, xq, y);
    QMS_CK(cudaGetLastError());
    return QMS_CUDA_OK;
}

int qms_cuda_matvec_f32(const float *w, int64_t rows, int64_t cols, const float *x, int T, float *y, void *stream) {
    QMS_REQUIRE(w && x && y && rows > 0 && cols > 0 && T >= 0, QMS_CUDA_EINVAL, "matvec_f32: bad arguments");
    QMS_REQUIRE(cols <= (1 << 20), QMS_CUDA_EINVAL, "matvec_f32: cols too large");
    if (T == 0) return QMS_CUDA_OK;
    return launch_matvec_f32_exact(w, rows, cols, x, T, y, (cudaStream_t)stream);
}

}  // extern "C"
