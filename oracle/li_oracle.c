/*
 * CPU oracle for the LeanInfer fused-kernel path. TEST INFRASTRUCTURE ONLY:
 * the checker for the CUDA kernels (tests/, __graft_entry__.smoke) and the
 * timed CPU baseline of bench.py. The product never links or calls it.
 *
 * Reference citations are paths inside the LeanInfer repository. Block
 * formats follow gguf-py 0.19.0 (gguf/quants.py), the only source of the
 * Q8_0/Q4_K formats available here (ggml itself is not vendored by the
 * reference). Build with -ffp-contract=off: the block decoders reproduce
 * gguf-py's separately rounded fp32 multiply and subtract.
 *
 * Floating-point ops other than block decode accumulate in double: the
 * oracle is the exact value the fp32 kernels are measured against.
 */
#include "li_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- minimal parallel-for over host threads (LIO_THREADS overrides) ---- */
typedef void (*lio_body)(void *ctx, int64_t i);

typedef struct {
    lio_body fn;
    void *ctx;
    int64_t n, chunk;
    int64_t next;              /* shared counter, atomically advanced */
} lio_job;

int lio_num_threads(void) {
    const char *e = getenv("LIO_THREADS");
    if (e && atoi(e) > 0) return atoi(e);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void *lio_worker(void *arg) {
    lio_job *j = (lio_job *)arg;
    for (;;) {
        const int64_t b = __atomic_fetch_add(&j->next, j->chunk, __ATOMIC_RELAXED);
        if (b >= j->n) break;
        const int64_t e = b + j->chunk < j->n ? b + j->chunk : j->n;
        for (int64_t i = b; i < e; ++i) j->fn(j->ctx, i);
    }
    return NULL;
}

static void parallel_for(int64_t n, int64_t chunk, lio_body fn, void *ctx) {
    if (n <= 0) return;
    lio_job job = {fn, ctx, n, chunk > 0 ? chunk : 1, 0};
    int T = lio_num_threads();
    if (T > 256) T = 256;
    if ((int64_t)T > (n + job.chunk - 1) / job.chunk) T = (int)((n + job.chunk - 1) / job.chunk);
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < T; ++t)
        if (pthread_create(&th[started], NULL, lio_worker, &job) == 0) ++started;
    lio_worker(&job);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* IEEE binary16 -> binary32, exact for every input (numpy astype). */
float lio_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {                       /* subnormal: m * 2^-24 */
            float f = (float)m * 5.9604644775390625e-08f;
            return sign ? -f : f;
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

float lio_bf16_to_fp32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t lio_fp32_to_bf16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

size_t lio_row_bytes(int wtype, int64_t k) {
    switch (wtype) {
    case 0: return (size_t)k * 4;
    case 1: return (size_t)k * 2;
    case 8: return (k % 32) ? 0 : (size_t)(k / 32) * 34;
    case 12: return (k % 256) ? 0 : (size_t)(k / 256) * 144;
    default: return 0;
    }
}

/* Q8_0 block: value = fp32(d) * fp32(q). gguf/quants.py:396-402. */
static void deq_q8_0_block(const uint8_t *b, float *out) {
    uint16_t dh;
    memcpy(&dh, b, 2);
    float d = lio_fp16_to_fp32(dh);
    const int8_t *q = (const int8_t *)(b + 2);
    for (int i = 0; i < 32; ++i) out[i] = (float)q[i] * d;
}

/* Q4_K 6-bit scale/min unpack. gguf/quants.py:479-500 (get_scale_min). */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K block: value = fl(fl(d*sc) * q) - fl(dmin*m), sub-block 2i from the
 * low nibbles of qs[32i..32i+31], sub-block 2i+1 from their high nibbles.
 * gguf/quants.py:503-522. */
static void deq_q4_k_block(const uint8_t *b, float *out) {
    uint16_t dh, mh;
    memcpy(&dh, b, 2);
    memcpy(&mh, b + 2, 2);
    const float d = lio_fp16_to_fp32(dh), dmin = lio_fp16_to_fp32(mh);
    const uint8_t *sc6 = b + 4, *qs = b + 16;
    for (int j = 0; j < 8; ++j) {
        int sc, mn;
        q4k_scale_min(sc6, j, &sc, &mn);
        const float dl = d * (float)sc;
        const float ml = dmin * (float)mn;
        const uint8_t *src = qs + 32 * (j / 2);
        const int shift = (j & 1) ? 4 : 0;
        for (int i = 0; i < 32; ++i) {
            const float qv = (float)((src[i] >> shift) & 0x0f);
            const float t = dl * qv;
            out[32 * j + i] = t - ml;
        }
    }
}

static void deq_row(int wtype, const uint8_t *row, float *out, int64_t k) {
    switch (wtype) {
    case 0: memcpy(out, row, (size_t)k * 4); break;
    case 1:
        for (int64_t i = 0; i < k; ++i) {
            uint16_t h;
            memcpy(&h, row + 2 * i, 2);
            out[i] = lio_fp16_to_fp32(h);
        }
        break;
    case 8:
        for (int64_t b = 0; b < k / 32; ++b) deq_q8_0_block(row + 34 * b, out + 32 * b);
        break;
    case 12:
        for (int64_t b = 0; b < k / 256; ++b) deq_q4_k_block(row + 144 * b, out + 256 * b);
        break;
    }
}

typedef struct { int wtype; const uint8_t *src; float *dst; int64_t bs; size_t bb; } deq_ctx;

static void deq_body(void *c, int64_t b) {
    deq_ctx *d = (deq_ctx *)c;
    deq_row(d->wtype, d->src + d->bb * b, d->dst + d->bs * b, d->bs);
}

int lio_dequantize(int wtype, const void *src, float *dst, int64_t n) {
    int64_t bs = (wtype == 8) ? 32 : (wtype == 12) ? 256 : 1;
    if (lio_row_bytes(wtype, bs) == 0 || n % bs) return -1;
    deq_ctx c = {wtype, (const uint8_t *)src, dst, bs, lio_row_bytes(wtype, bs)};
    parallel_for(n / bs, 1024, deq_body, &c);
    return 0;
}

static double dot_fd(const float *a, const double *b, int64_t k) {
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t i = 0;
    for (; i + 4 <= k; i += 4) {
        s0 += (double)a[i] * b[i];
        s1 += (double)a[i + 1] * b[i + 1];
        s2 += (double)a[i + 2] * b[i + 2];
        s3 += (double)a[i + 3] * b[i + 3];
    }
    for (; i < k; ++i) s0 += (double)a[i] * b[i];
    return (s0 + s1) + (s2 + s3);
}

/* x_norm = x * gamma * rsqrt(mean(x^2) + eps): the reference's RMSNorm,
 * cuda/leaninfer-fused-ffn.cu:62-83 (CPU form cuda/benchmark_fused.cu:99-110).
 * gamma NULL: copy. */
static void rms_norm_d(const float *x, const float *gamma, double *xn, int K,
                       float eps) {
    if (!gamma) {
        for (int i = 0; i < K; ++i) xn[i] = x[i];
        return;
    }
    double sq = 0;
    for (int i = 0; i < K; ++i) sq += (double)x[i] * x[i];
    const double r = 1.0 / sqrt(sq / K + (double)eps);
    for (int i = 0; i < K; ++i) xn[i] = (double)x[i] * gamma[i] * r;
}

static double silu_d(double v) { return v / (1.0 + exp(-v)); }

/* fp32 -> nearest binary16 value (round to nearest even), as __float2half:
 * the value's fp16 step is found from its exponent. */
static float fp16_round(float f) {
    const float a = fabsf(f);
    float out;
    if (a >= 65520.0f) {
        out = INFINITY;
    } else if (a < 6.103515625e-05f) {     /* subnormal range: step 2^-24 */
        out = nearbyintf(a * 16777216.0f) / 16777216.0f;
    } else {
        int e;
        frexpf(a, &e);                      /* a = m * 2^e, m in [0.5, 1) */
        const float step = ldexpf(1.0f, e - 11);
        out = nearbyintf(a / step) * step;
    }
    return signbit(f) ? -out : out;
}

typedef struct {
    int wtype;
    const uint8_t *W;
    size_t rb;
    const double *xn;
    float *dst;
    int K, N, n_rows;
} mm_ctx;

static void mm_body(void *cp, int64_t n) {
    mm_ctx *c = (mm_ctx *)cp;
    float *wrow = (float *)malloc(sizeof(float) * c->K);
    deq_row(c->wtype, c->W + c->rb * n, wrow, c->K);
    for (int r = 0; r < c->n_rows; ++r)
        c->dst[(size_t)r * c->N + n] = (float)dot_fd(wrow, c->xn + (size_t)r * c->K, c->K);
    free(wrow);
}

/* dst[r][n] = <x_norm[r], W[n]>: cuda/leaninfer-fused-ffn.cu:41-97 with
 * quantized rows decoded first (ggml MUL_MAT semantics). */
int lio_rms_norm_matmul(int wtype, const float *x, const float *gamma,
                        const void *W, float *dst, int K, int N, int n_rows,
                        float eps) {
    const size_t rb = lio_row_bytes(wtype, K);
    if (!rb) return -1;
    double *xn = (double *)malloc(sizeof(double) * (size_t)K * n_rows);
    for (int r = 0; r < n_rows; ++r)
        rms_norm_d(x + (size_t)r * K, gamma, xn + (size_t)r * K, K, eps);
    mm_ctx c = {wtype, (const uint8_t *)W, rb, xn, dst, K, N, n_rows};
    parallel_for(N, 16, mm_body, &c);
    free(xn);
    return 0;
}

/* ---- ggml-style quantized activations (UNPINNED) ----------------------
 * ggml's CPU MUL_MAT of a quantized matrix first quantizes the activation
 * row and takes integer dot products: Q4_K weights against q8_K
 * activations (256-value blocks, scale 1/iscale with iscale = -127/v where v
 * is the element of largest magnitude, q = nearest(iscale * x) capped at 127,
 * 16-value block sums for the min term), Q8_0 weights against q8_0
 * activations (32-value blocks, d = max|x| / 127 stored as fp16, q =
 * nearest(x / d) with the fp32 d). Restated from ggml's published
 * quantize_row_q8_K / quantize_row_q8_0 and vec_dot_q4_K_q8_K /
 * vec_dot_q8_0_q8_0 arithmetic; no reference test or vector pins ggml's CPU
 * results, so this variant only measures how far that arithmetic lies from
 * the exact dot products. The row is RMS-normalised in fp32 first, as
 * ggml's RMS_NORM + MUL produce it. Block sums are exact integers; the
 * per-block scaling is in double. */
static void q8act_row(const double *xn, int K, int qk, int8_t *q, float *d) {
    for (int b = 0; b < K / qk; ++b) {
        float xb[256];
        float amax = 0.f, vmax = 0.f;
        for (int j = 0; j < qk; ++j) {
            xb[j] = (float)xn[(size_t)b * qk + j];
            if (fabsf(xb[j]) > amax) { amax = fabsf(xb[j]); vmax = xb[j]; }
        }
        int8_t *qb = q + (size_t)b * qk;
        if (amax == 0.f) {
            d[b] = 0.f;
            memset(qb, 0, (size_t)qk);
        } else if (qk == 256) {             /* q8_K */
            const float iscale = -127.f / vmax;
            for (int j = 0; j < qk; ++j) {
                long v = lrintf(iscale * xb[j]);
                qb[j] = (int8_t)(v > 127 ? 127 : v);
            }
            d[b] = 1.f / iscale;
        } else {                            /* q8_0 */
            const float db = amax / 127.f, id = 1.f / db;
            for (int j = 0; j < qk; ++j) qb[j] = (int8_t)lrintf(xb[j] * id);
            d[b] = fp16_round(db);
        }
    }
}

typedef struct {
    int wtype;
    const uint8_t *W;
    size_t rb;
    const int8_t *q;
    const float *d;
    const int32_t *bs;   /* per activation row: sums of its 32-value groups (ggml's q8_K bsums) */
    float *dst;
    int K, N, n_rows;
} q8_ctx;

/* One weight row against every activation row. The row is unpacked once
 * (4-bit codes to int8, scales and mins to ints), then each row's dot is a
 * plain int8 x int8 -> int32 loop per 32-value group, which the compiler
 * vectorises (the integer dots of ggml's vec_dot kernels); the integer sums
 * and their float combination are the same as before, so the result is
 * unchanged bit for bit. */
static void q8_body(void *cp, int64_t n) {
    q8_ctx *c = (q8_ctx *)cp;
    const uint8_t *row = c->W + c->rb * n;
    const int K = c->K;
    int8_t *wq = (int8_t *)malloc((size_t)K);
    if (c->wtype == 12) {
        const int nb = K / 256;
        int *sc = (int *)malloc(sizeof(int) * 16 * (size_t)nb);
        int *mn = sc + 8 * nb;
        double *dd = (double *)malloc(sizeof(double) * 2 * (size_t)nb);
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = row + 144 * (size_t)b;
            uint16_t dh, mh;
            memcpy(&dh, blk, 2);
            memcpy(&mh, blk + 2, 2);
            dd[2 * b] = lio_fp16_to_fp32(dh);
            dd[2 * b + 1] = lio_fp16_to_fp32(mh);
            for (int j = 0; j < 8; ++j) {
                q4k_scale_min(blk + 4, j, &sc[8 * b + j], &mn[8 * b + j]);
                const uint8_t *src = blk + 16 + 32 * (j / 2);
                for (int i = 0; i < 32; ++i) wq[256 * b + 32 * j + i] = (int8_t)((src[i] >> ((j & 1) ? 4 : 0)) & 0x0f);
            }
        }
        for (int r = 0; r < c->n_rows; ++r) {
            const int8_t *q = c->q + (size_t)r * K;
            const float *d = c->d + (size_t)r * nb;
            const int32_t *bs = c->bs + (size_t)r * (K / 32);
            double acc = 0;
            for (int b = 0; b < nb; ++b) {
                int32_t s_sc = 0, s_mn = 0;
                for (int j = 0; j < 8; ++j) {
                    const int8_t *wj = wq + 256 * b + 32 * j, *qj = q + 256 * b + 32 * j;
                    int32_t dot = 0;
                    for (int i = 0; i < 32; ++i) dot += (int32_t)wj[i] * (int32_t)qj[i];
                    s_sc += sc[8 * b + j] * dot;
                    s_mn += mn[8 * b + j] * bs[8 * b + j];
                }
                acc += dd[2 * b] * d[b] * (double)s_sc - dd[2 * b + 1] * d[b] * (double)s_mn;
            }
            c->dst[(size_t)r * c->N + n] = (float)acc;
        }
        free(dd);
        free(sc);
    } else {
        const int nb = K / 32;
        double *dd = (double *)malloc(sizeof(double) * (size_t)nb);
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = row + 34 * (size_t)b;
            uint16_t dh;
            memcpy(&dh, blk, 2);
            dd[b] = lio_fp16_to_fp32(dh);
            memcpy(wq + 32 * b, blk + 2, 32);
        }
        for (int r = 0; r < c->n_rows; ++r) {
            const int8_t *q = c->q + (size_t)r * K;
            const float *d = c->d + (size_t)r * nb;
            double acc = 0;
            for (int b = 0; b < nb; ++b) {
                int32_t dot = 0;
                for (int i = 0; i < 32; ++i) dot += (int32_t)wq[32 * b + i] * (int32_t)q[32 * b + i];
                acc += dd[b] * d[b] * (double)dot;
            }
            c->dst[(size_t)r * c->N + n] = (float)acc;
        }
        free(dd);
    }
    free(wq);
}

int lio_rms_norm_matmul_q8act(int wtype, const float *x, const float *gamma,
                              const void *W, float *dst, int K, int N,
                              int n_rows, float eps) {
    const size_t rb = lio_row_bytes(wtype, K);
    if (!rb || (wtype != 8 && wtype != 12)) return -1;
    const int qk = wtype == 12 ? 256 : 32;
    double *xn = (double *)malloc(sizeof(double) * (size_t)K);
    int8_t *q = (int8_t *)malloc((size_t)K * n_rows);
    float *d = (float *)malloc(sizeof(float) * (size_t)(K / qk) * n_rows);
    for (int r = 0; r < n_rows; ++r) {
        const float *xr = x + (size_t)r * K;
        if (gamma) {                         /* fp32 RMS_NORM (double sum), then MUL */
            double sq = 0;
            for (int i = 0; i < K; ++i) sq += (double)xr[i] * xr[i];
            const float scale = 1.0f / sqrtf((float)(sq / K) + eps);
            for (int i = 0; i < K; ++i) xn[i] = (double)((xr[i] * scale) * gamma[i]);
        } else {
            for (int i = 0; i < K; ++i) xn[i] = xr[i];
        }
        q8act_row(xn, K, qk, q + (size_t)r * K, d + (size_t)r * (K / qk));
    }
    int32_t *bs = (int32_t *)malloc(sizeof(int32_t) * (size_t)(K / 32) * n_rows);
    for (int64_t g = 0; g < (int64_t)(K / 32) * n_rows; ++g) {
        int32_t t = 0;
        for (int i = 0; i < 32; ++i) t += q[32 * g + i];
        bs[g] = t;
    }
    q8_ctx c = {wtype, (const uint8_t *)W, rb, q, d, bs, dst, K, N, n_rows};
    parallel_for(N, 16, q8_body, &c);
    free(bs);
    free(xn);
    free(q);
    free(d);
    return 0;
}

typedef struct {
    int wtype;
    const uint8_t *Wg, *Wu;
    size_t rb;
    const double *xn;
    float *h;
    int K, N, n_rows;
} sw_ctx;

static void sw_body(void *cp, int64_t n) {
    sw_ctx *c = (sw_ctx *)cp;
    float *g = (float *)malloc(sizeof(float) * c->K * 2);
    float *u = g + c->K;
    deq_row(c->wtype, c->Wg + c->rb * n, g, c->K);
    deq_row(c->wtype, c->Wu + c->rb * n, u, c->K);
    for (int r = 0; r < c->n_rows; ++r) {
        const double *xr = c->xn + (size_t)r * c->K;
        c->h[(size_t)r * c->N + n] = (float)(silu_d(dot_fd(g, xr, c->K)) * dot_fd(u, xr, c->K));
    }
    free(g);
}

/* h[n] = silu(gate) * up: cuda/leaninfer-fused-ffn.cu:116-180 (f32) and
 * :188-252 (f16 weights, x_norm rounded to fp16 at :230). */
int lio_rms_norm_swiglu(int wtype, const float *x, const float *gamma,
                        const void *Wg, const void *Wu, float *h, int K, int N,
                        int n_rows, float eps, int round_xn_f16) {
    const size_t rb = lio_row_bytes(wtype, K);
    if (!rb) return -1;
    double *xn = (double *)malloc(sizeof(double) * (size_t)K * n_rows);
    for (int r = 0; r < n_rows; ++r) {
        double *xr = xn + (size_t)r * K;
        rms_norm_d(x + (size_t)r * K, gamma, xr, K, eps);
        if (round_xn_f16)
            for (int i = 0; i < K; ++i) xr[i] = fp16_round((float)xr[i]);
    }
    sw_ctx c = {wtype, (const uint8_t *)Wg, (const uint8_t *)Wu, rb, xn, h, K, N, n_rows};
    parallel_for(N, 16, sw_body, &c);
    free(xn);
    return 0;
}

int lio_ffn(int wtype, const float *x, const float *gamma, const void *Wg,
            const void *Wu, const void *Wd, float *y, int K, int N, int n_rows,
            float eps) {
    float *h = (float *)malloc(sizeof(float) * (size_t)N * n_rows);
    int rc = lio_rms_norm_swiglu(wtype, x, gamma, Wg, Wu, h, K, N, n_rows, eps, 0);
    if (!rc) rc = lio_rms_norm_matmul(wtype, h, NULL, Wd, y, N, K, n_rows, 0.f);
    free(h);
    return rc;
}

/* Gated RMSNorm: cuda/leaninfer-fused-gate.cu:39-85; CPU form
 * scripts/patch_fused_gate.sh:89-110. */
void lio_silu_gate(const float *o, const float *z, const float *gamma,
                   float *dst, int K, int n_rows, float eps) {
    for (int r = 0; r < n_rows; ++r) {
        const float *orow = o + (size_t)r * K, *zrow = z + (size_t)r * K;
        double sq = 0;
        for (int i = 0; i < K; ++i) sq += (double)orow[i] * orow[i];
        const double rs = 1.0 / sqrt(sq / K + (double)eps);
        for (int i = 0; i < K; ++i)
            dst[(size_t)r * K + i] = (float)(silu_d(zrow[i]) * ((double)orow[i] * gamma[i] * rs));
    }
}

/* One token of the gated delta rule on one head, reference arithmetic of
 * cuda/leaninfer-fused-deltanet.cu:217-288 (scale :196, beta :235,
 * decay :236, sums :238-255, v' :257, output :258, update+clamp :281-287).
 * S is [D(k)][D(v)] (S[c*D + r]), updated in place. qs is q * scale. */
static void gdr_token(double *S, const double *qs, const double *kk,
                      const double *vv, double beta_sig, double decay,
                      double *o, int D, int clamp, double *u, double *w) {
    double attn = 0;
    for (int c = 0; c < D; ++c) attn += kk[c] * qs[c];
    for (int r = 0; r < D; ++r) u[r] = w[r] = 0;
    for (int c = 0; c < D; ++c) {
        const double *Sc = S + (size_t)c * D;
        for (int r = 0; r < D; ++r) {
            u[r] += Sc[r] * kk[c];
            w[r] += Sc[r] * qs[c];
        }
    }
    for (int r = 0; r < D; ++r) {
        const double vn = beta_sig * (vv[r] - decay * u[r]);
        o[r] = decay * w[r] + vn * attn;
        u[r] = vn;                                   /* reuse: v' */
    }
    for (int c = 0; c < D; ++c) {
        double *Sc = S + (size_t)c * D;
        for (int r = 0; r < D; ++r) {
            double s = decay * Sc[r] + u[r] * kk[c];
            if (clamp) s = s < -1e6 ? -1e6 : (s > 1e6 ? 1e6 : s);
            Sc[r] = s;
        }
    }
}

typedef struct {
    const float *q, *k, *v, *g, *beta, *state_in;
    float *out, *state_out;
    double *o_all;
    int64_t D, n_tokens, n_heads, gqa, nkq;
    int repeat_type;
    size_t vnb1, vnb2, vnb3;
    double scale;
} rec_ctx;

static void rec_body(void *cp, int64_t idx) {
    rec_ctx *c = (rec_ctx *)cp;
    const int64_t D = c->D, s = idx / c->n_heads, h = idx % c->n_heads;
    /* head mapping: cuda/leaninfer-fused-deltanet.cu:165-167 */
    const int64_t hk = c->repeat_type == 0 ? h / c->gqa : h % c->nkq;
    double *S = (double *)malloc(sizeof(double) * D * D);
    double *qs = (double *)malloc(sizeof(double) * D * 6);
    double *kk = qs + D, *vv = kk + D, *o = vv + D, *u = o + D, *w = u + D;
    const float *Sin = c->state_in + (s * c->n_heads + h) * D * D;
    for (int64_t i = 0; i < D * D; ++i) S[i] = Sin[i];
    for (int64_t t = 0; t < c->n_tokens; ++t) {
        const float *qp = c->q + ((s * c->nkq + hk) * c->n_tokens + t) * D;
        const float *kp = c->k + ((s * c->nkq + hk) * c->n_tokens + t) * D;
        const float *vp = c->v + s * c->vnb3 + h * c->vnb2 + t * c->vnb1;
        for (int64_t i = 0; i < D; ++i) {
            qs[i] = (double)qp[i] * c->scale;
            kk[i] = kp[i];
            vv[i] = vp[i];
        }
        const double gb = c->g[(s * c->n_tokens + t) * c->n_heads + h];
        const double bb = c->beta[(s * c->n_tokens + t) * c->n_heads + h];
        const double bsig = 1.0 / (1.0 + exp(-bb));
        const double decay = exp(gb < 50.0 ? gb : 50.0);
        gdr_token(S, qs, kk, vv, bsig, decay, o, (int)D, 1, u, w);
        float *op = c->out + ((s * c->n_tokens + t) * c->n_heads + h) * D;
        double *oa = c->o_all + ((s * c->n_tokens + t) * c->n_heads + h) * D;
        for (int64_t i = 0; i < D; ++i) {
            op[i] = (float)o[i];
            oa[i] = o[i];
        }
    }
    float *Sout = c->state_out + (s * c->n_heads + h) * D * D;
    for (int64_t i = 0; i < D * D; ++i) Sout[i] = (float)S[i];
    free(S);
    free(qs);
}

typedef struct {
    const float *W_out;
    const double *o_all;
    float *proj_out;
    int64_t n_tokens, n_seqs, HD;
} proj_ctx;

/* Intended projection of cuda/leaninfer-fused-deltanet.cu:260-279:
 * proj[d][t] = sum_s sum_{h,j} W_out[d][h*D+j] * o[s][t][h][j]
 * (the reference's lane mapping there covers only D/32 of the terms). */
static void proj_body(void *cp, int64_t d) {
    proj_ctx *c = (proj_ctx *)cp;
    for (int64_t t = 0; t < c->n_tokens; ++t) {
        double acc = 0;
        for (int64_t s = 0; s < c->n_seqs; ++s) {
            const double *oa = c->o_all + (s * c->n_tokens + t) * c->HD;
            for (int64_t j = 0; j < c->HD; ++j) acc += (double)c->W_out[d * c->HD + j] * oa[j];
        }
        c->proj_out[d * c->n_tokens + t] = (float)acc;
    }
}

int lio_deltanet_recurrent(const float *q, const float *k, const float *v,
                           const float *g, const float *beta,
                           const float *state_in, float *out, float *state_out,
                           const float *W_out, float *proj_out,
                           int64_t D, int64_t n_tokens, int64_t n_heads,
                           int64_t gqa, int repeat_type, int64_t n_seqs,
                           int64_t hidden, size_t vnb1, size_t vnb2,
                           size_t vnb3) {
    if (D <= 0 || gqa <= 0 || n_heads % gqa) return -1;
    rec_ctx c = {q, k, v, g, beta, state_in, out, state_out, NULL, D, n_tokens, n_heads, gqa,
                 n_heads / gqa, repeat_type, vnb1, vnb2, vnb3, 1.0 / sqrt((double)D)};
    c.o_all = (double *)calloc((size_t)(n_seqs * n_tokens * n_heads * D) + 1, sizeof(double));
    parallel_for(n_seqs * n_heads, 1, rec_body, &c);
    if (W_out && proj_out) {
        proj_ctx pc = {W_out, c.o_all, proj_out, n_tokens, n_seqs, n_heads * D};
        parallel_for(hidden, 8, proj_body, &pc);
    }
    free(c.o_all);
    return 0;
}

size_t lio_deltanet_taps_per_seq(const lio_deltanet_layer *L) {
    const size_t D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads;
    return (2 * Hk * D + Hv * D) + Hv * D + 2 * Hv + 2 * Hv * D;
}

typedef struct {
    const lio_deltanet_layer *L;
    const float *p;        /* [n_seqs][NI] in-projection */
    const double *act;     /* [n_seqs][C] post-conv activations */
    const double *qkn;     /* [n_seqs][2*Hk*D] l2-normalised q | k */
    float *state, *og, *taps;
    int C, NI;
    size_t tps;
} layer_ctx;

/* One (sequence, v-head) of the layer: beta, g, recurrence, gated RMSNorm. */
static void layer_head_body(void *cp, int64_t idx) {
    layer_ctx *c = (layer_ctx *)cp;
    const lio_deltanet_layer *L = c->L;
    const int D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads, C = c->C;
    const int s = (int)(idx / Hv), h = (int)(idx % Hv);
    const int gqa = Hv / Hk;
    const int hk = L->repeat_type == 0 ? h / gqa : h % Hk;
    const float *ps = c->p + (size_t)s * c->NI;
    const double *act = c->act + (size_t)s * C;
    const double *qn = c->qkn + (size_t)s * 2 * Hk * D, *kn = qn + Hk * D;
    const double scale = 1.0 / sqrt((double)D);
    double *S = (double *)malloc(sizeof(double) * D * D);
    double *buf = (double *)malloc(sizeof(double) * D * 6);
    double *qs = buf, *kk = qs + D, *vv = kk + D, *o = vv + D, *u = o + D, *w = u + D;
    float *Sg = c->state + ((size_t)s * Hv + h) * D * D;
    for (int i = 0; i < D * D; ++i) S[i] = Sg[i];
    for (int i = 0; i < D; ++i) {
        qs[i] = qn[hk * D + i] * scale;
        kk[i] = kn[hk * D + i];
        vv[i] = act[2 * Hk * D + h * D + i];
    }
    const double bsig = 1.0 / (1.0 + exp(-(double)ps[C + Hv * D + h]));
    const double av = (double)ps[C + Hv * D + Hv + h] + L->dt_bias[h];
    const double sp = av > 20.0 ? av : log1p(exp(av));       /* softplus */
    const double gval = -exp((double)L->a_log[h]) * sp;
    const double decay = exp(gval < 50.0 ? gval : 50.0);
    gdr_token(S, qs, kk, vv, bsig, decay, o, D, 1, u, w);
    for (int i = 0; i < D * D; ++i) Sg[i] = (float)S[i];
    /* gated RMSNorm of this head (cuda/leaninfer-fused-gate.cu:39-85); z is
     * the raw in-projection z */
    double sq = 0;
    for (int i = 0; i < D; ++i) sq += o[i] * o[i];
    const double rs = 1.0 / sqrt(sq / D + L->norm_eps);
    float *og = c->og + (size_t)s * Hv * D + (size_t)h * D;
    for (int i = 0; i < D; ++i) {
        const double zv = ps[C + h * D + i];
        og[i] = (float)(silu_d(zv) * o[i] * L->norm_w[i] * rs);
    }
    if (c->taps) {
        float *tp = c->taps + c->tps * s;
        tp[C + Hv * D + h] = (float)bsig;
        tp[C + Hv * D + Hv + h] = (float)gval;
        for (int i = 0; i < D; ++i) {
            tp[C + Hv * D + 2 * Hv + h * D + i] = (float)o[i];
            tp[C + 2 * Hv * D + 2 * Hv + h * D + i] = og[i];
        }
    }
    free(S);
    free(buf);
}

/* One decode step of a Gated DeltaNet layer. The op order is the one of the
 * reference product's decode graph (node names in traces/qwen35_9b_run.json:
 * qkv_mixed, conv_output_raw, conv_output_silu, q_conv/k_conv, alpha_biased,
 * a_softplus, g_in, delta_net_fused_raw, attn_out_norm, linear_attn_out);
 * the recurrence is gdr_token (reference kernel arithmetic), the gated norm
 * lio_silu_gate's, the projections lio_rms_norm_matmul's. */
typedef int (*lio_matmul_fn)(int, const float *, const float *, const void *, float *, int, int, int, float);

static int layer_decode_impl(const lio_deltanet_layer *L, const float *x,
                             float *y, float *conv_state, float *state,
                             int n_seqs, float *taps, lio_matmul_fn mm);

int lio_deltanet_layer_decode(const lio_deltanet_layer *L, const float *x,
                              float *y, float *conv_state, float *state,
                              int n_seqs, float *taps) {
    return layer_decode_impl(L, x, y, conv_state, state, n_seqs, taps, lio_rms_norm_matmul);
}

/* The same step with both projections in ggml's CPU arithmetic (activations
 * quantized to q8_K / q8_0, integer dots: lio_rms_norm_matmul_q8act), the
 * form ggml's CPU backend runs; UNPINNED, for the timed CPU baseline only. */
int lio_deltanet_layer_decode_q8act(const lio_deltanet_layer *L, const float *x,
                                    float *y, float *conv_state, float *state,
                                    int n_seqs) {
    return layer_decode_impl(L, x, y, conv_state, state, n_seqs, NULL, lio_rms_norm_matmul_q8act);
}

static int layer_decode_impl(const lio_deltanet_layer *L, const float *x,
                             float *y, float *conv_state, float *state,
                             int n_seqs, float *taps, lio_matmul_fn mm) {
    const int D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads;
    const int K = L->conv_kernel, hid = L->hidden;
    if (Hk <= 0 || Hv % Hk) return -1;
    const int C = 2 * Hk * D + Hv * D;                 /* conv channels   */
    const int NI = C + Hv * D + 2 * Hv;                /* in-proj rows    */
    float *p = (float *)malloc(sizeof(float) * (size_t)NI * n_seqs);
    int rc = mm(L->w_in_type, x, L->in_norm_w, L->w_in, p, hid, NI, n_seqs, L->in_norm_eps);
    if (rc) { free(p); return rc; }
    float *og = (float *)malloc(sizeof(float) * (size_t)Hv * D * n_seqs);
    double *act = (double *)malloc(sizeof(double) * (size_t)C * n_seqs);
    double *qkn = (double *)malloc(sizeof(double) * (size_t)2 * Hk * D * n_seqs);
    const size_t tps = lio_deltanet_taps_per_seq(L);
    for (int s = 0; s < n_seqs; ++s) {
        const float *ps = p + (size_t)s * NI;
        double *as = act + (size_t)s * C;
        float *cs = conv_state + (size_t)s * C * (K - 1);
        for (int c = 0; c < C; ++c) {          /* causal conv1d + silu */
            double acc = 0;
            for (int j = 0; j < K - 1; ++j) acc += (double)L->conv_w[c * K + j] * cs[c * (K - 1) + j];
            acc += (double)L->conv_w[c * K + K - 1] * ps[c];
            for (int j = 0; j < K - 2; ++j) cs[c * (K - 1) + j] = cs[c * (K - 1) + j + 1];
            cs[c * (K - 1) + K - 2] = ps[c];
            as[c] = silu_d(acc);
        }
        double *qn = qkn + (size_t)s * 2 * Hk * D, *kn = qn + Hk * D;
        for (int h = 0; h < Hk; ++h) {         /* per-head l2norm of q, k */
            double sq = 0, sk = 0;
            for (int i = 0; i < D; ++i) {
                sq += as[h * D + i] * as[h * D + i];
                sk += as[Hk * D + h * D + i] * as[Hk * D + h * D + i];
            }
            const double rq = 1.0 / sqrt(sq + L->l2_eps), rk = 1.0 / sqrt(sk + L->l2_eps);
            for (int i = 0; i < D; ++i) {
                qn[h * D + i] = as[h * D + i] * rq;
                kn[h * D + i] = as[Hk * D + h * D + i] * rk;
            }
        }
        if (taps) {
            float *tp = taps + tps * s;
            for (int c = 0; c < C; ++c) tp[c] = (float)as[c];
            for (int i = 0; i < Hv * D; ++i) tp[C + i] = ps[C + i];
        }
    }
    layer_ctx lc = {L, p, act, qkn, state, og, taps, C, NI, tps};
    parallel_for((int64_t)n_seqs * Hv, 1, layer_head_body, &lc);
    rc = mm(L->w_out_type, og, NULL, L->w_out, y, Hv * D, hid, n_seqs, 0.f);
    free(qkn);
    free(act);
    free(og);
    free(p);
    return rc;
}

typedef struct {
    const uint16_t *q, *k, *v;
    const float *g, *beta;
    float *state, *o;
    int T, Hk, Hv, D;
    double scale;
} pf_ctx;

static void pf_body(void *cp, int64_t hh) {
    pf_ctx *c = (pf_ctx *)cp;
    const int D = c->D, h = (int)hh, hk = h / (c->Hv / c->Hk);
    double *S = (double *)malloc(sizeof(double) * D * D);
    double *buf = (double *)malloc(sizeof(double) * D * 6);
    double *qs = buf, *kk = qs + D, *vv = kk + D, *ot = vv + D, *u = ot + D, *w = u + D;
    float *Sg = c->state + (size_t)h * D * D;
    for (int i = 0; i < D * D; ++i) S[i] = Sg[i];
    for (int t = 0; t < c->T; ++t) {
        for (int i = 0; i < D; ++i) {
            qs[i] = (double)lio_bf16_to_fp32(c->q[((size_t)t * c->Hk + hk) * D + i]) * c->scale;
            kk[i] = lio_bf16_to_fp32(c->k[((size_t)t * c->Hk + hk) * D + i]);
            vv[i] = lio_bf16_to_fp32(c->v[((size_t)t * c->Hv + h) * D + i]);
        }
        gdr_token(S, qs, kk, vv, c->beta[(size_t)t * c->Hv + h],
                  exp((double)c->g[(size_t)t * c->Hv + h]), ot, D, 0, u, w);
        for (int i = 0; i < D; ++i) c->o[((size_t)t * c->Hv + h) * D + i] = (float)ot[i];
    }
    for (int i = 0; i < D * D; ++i) Sg[i] = (float)S[i];
    free(S);
    free(buf);
}

/* Token-by-token gated delta rule (no clamp), the semantics the chunked WY
 * prefill must reproduce; cross-checked against flash-linear-attention's
 * naive_recurrent_gated_delta_rule in the golden fixtures. */
int lio_gdr_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                    const float *g, const float *beta, float *state, float *o,
                    int T, int Hk, int Hv, int D, float scale) {
    if (Hk <= 0 || Hv % Hk) return -1;
    pf_ctx c = {q, k, v, g, beta, state, o, T, Hk, Hv, D, (double)scale};
    parallel_for(Hv, 1, pf_body, &c);
    return 0;
}

/* ---------------------------------------------------------------------- */
/* Gated GQA attention decode layer (no kernel of the reference: the hybrid
 * stack's attention layers, reference docs/ASSESSMENT.md:1077 and
 * :1086-1087, "standard grouped-query attention ... RoPE" with a normal KV
 * cache). The norm is the reference's RMSNorm form
 * (cuda/leaninfer-fused-ffn.cu:62-83); the output gate sigmoid(gate) and the
 * per-head q/k RMSNorm follow the Qwen3.5 gated-attention convention, the
 * RoPE is NeoX rotate-half: choices, not pinned by the reference. */

uint16_t lio_fp32_to_fp16(float f) {
    const float r = fp16_round(f);
    uint32_t b;
    memcpy(&b, &r, 4);
    const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    const float a = fabsf(r);
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    if (isinf(a)) return (uint16_t)(sign | 0x7c00u);
    if (a == 0.0f) return sign;
    if (a < 6.103515625e-05f) return (uint16_t)(sign | (uint16_t)(a * 16777216.0f));   /* subnormal: m * 2^-24 */
    int e;
    const float m = frexpf(a, &e);            /* a = m * 2^e, m in [0.5, 1) */
    const uint16_t ebits = (uint16_t)(e - 1 + 15);
    const uint16_t mbits = (uint16_t)((m * 2.0f - 1.0f) * 1024.0f);
    return (uint16_t)(sign | (ebits << 10) | mbits);
}

static void head_rms_rope(double *v, const float *w, int D, float eps, int rope_dim, double theta, int pos) {
    if (w) {
        double sq = 0;
        for (int i = 0; i < D; ++i) sq += v[i] * v[i];
        const double r = 1.0 / sqrt(sq / D + (double)eps);
        for (int i = 0; i < D; ++i) v[i] = v[i] * w[i] * r;
    }
    const int half = rope_dim / 2;
    for (int i = 0; i < half; ++i) {
        const double ang = (double)pos * pow(theta, -2.0 * i / rope_dim);
        const double c = cos(ang), sn = sin(ang);
        const double x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c - x2 * sn;
        v[i + half] = x2 * c + x1 * sn;
    }
}

typedef struct {
    const lio_attn_layer *L;
    const float *p;            /* [n][NP] projections */
    const uint16_t *kc, *vc;
    const int32_t *pos;
    float *og;                 /* [n][Hq*D] */
    int NP, max_ctx;
} attn_ctx;

static double sigmoid_d(double v) { return 1.0 / (1.0 + exp(-v)); }

static void attn_head_body(void *cp, int64_t idx) {
    attn_ctx *c = (attn_ctx *)cp;
    const lio_attn_layer *L = c->L;
    const int D = L->head_dim, Hq = L->n_q_heads, Hkv = L->n_kv_heads;
    const int s = (int)(idx / Hq), h = (int)(idx % Hq), j = h / (Hq / Hkv);
    const int pos = c->pos[s];
    const float *ps = c->p + (size_t)s * c->NP;
    double *q = (double *)malloc(sizeof(double) * D);
    double *acc = (double *)calloc(D, sizeof(double));
    double *sc = (double *)malloc(sizeof(double) * (pos + 1));
    for (int i = 0; i < D; ++i) q[i] = ps[h * D + i];
    head_rms_rope(q, L->q_norm_w, D, L->qk_norm_eps, L->rope_dim, L->rope_theta, pos);
    const double scale = 1.0 / sqrt((double)D);
    double mx = -INFINITY;
    for (int t = 0; t <= pos; ++t) {
        const uint16_t *kr = c->kc + (((size_t)s * c->max_ctx + t) * Hkv + j) * D;
        double d = 0;
        for (int i = 0; i < D; ++i) d += q[i] * lio_fp16_to_fp32(kr[i]);
        sc[t] = d * scale;
        if (sc[t] > mx) mx = sc[t];
    }
    double l = 0;
    for (int t = 0; t <= pos; ++t) {
        const double w = exp(sc[t] - mx);
        l += w;
        const uint16_t *vr = c->vc + (((size_t)s * c->max_ctx + t) * Hkv + j) * D;
        for (int i = 0; i < D; ++i) acc[i] += w * lio_fp16_to_fp32(vr[i]);
    }
    const float *gate = ps + (size_t)Hq * D + h * D;
    for (int i = 0; i < D; ++i)
        c->og[(size_t)s * Hq * D + h * D + i] = (float)(acc[i] / l * sigmoid_d(gate[i]));
    free(sc);
    free(acc);
    free(q);
}

int lio_attn_layer_decode(const lio_attn_layer *L, const float *x, float *y,
                          uint16_t *k_cache, uint16_t *v_cache,
                          const int32_t *pos, int n_seqs, int max_ctx) {
    const int D = L->head_dim, Hq = L->n_q_heads, Hkv = L->n_kv_heads, hid = L->hidden;
    if (Hkv <= 0 || Hq % Hkv || L->rope_dim % 2 || L->rope_dim > D) return -1;
    const int NP = 2 * Hq * D + 2 * Hkv * D;
    for (int s = 0; s < n_seqs; ++s)
        if (pos[s] < 0 || pos[s] >= max_ctx) return -1;
    float *p = (float *)malloc(sizeof(float) * (size_t)NP * n_seqs);
    int rc = lio_rms_norm_matmul(L->w_in_type, x, L->in_norm_w, L->w_in, p, hid, NP, n_seqs, L->in_norm_eps);
    if (rc) { free(p); return rc; }
    double *kv = (double *)malloc(sizeof(double) * D);
    for (int s = 0; s < n_seqs; ++s) {      /* the new token's k, v into the caches */
        const float *ps = p + (size_t)s * NP;
        for (int j = 0; j < Hkv; ++j) {
            const size_t off = (((size_t)s * max_ctx + pos[s]) * Hkv + j) * D;
            for (int i = 0; i < D; ++i) kv[i] = ps[2 * Hq * D + j * D + i];
            head_rms_rope(kv, L->k_norm_w, D, L->qk_norm_eps, L->rope_dim, L->rope_theta, pos[s]);
            for (int i = 0; i < D; ++i) {
                k_cache[off + i] = lio_fp32_to_fp16((float)kv[i]);
                v_cache[off + i] = lio_fp32_to_fp16(ps[2 * Hq * D + Hkv * D + j * D + i]);
            }
        }
    }
    free(kv);
    float *og = (float *)malloc(sizeof(float) * (size_t)Hq * D * n_seqs);
    attn_ctx ac = {L, p, k_cache, v_cache, pos, og, NP, max_ctx};
    parallel_for((int64_t)n_seqs * Hq, 1, attn_head_body, &ac);
    rc = lio_rms_norm_matmul(L->w_out_type, og, NULL, L->w_out, y, Hq * D, hid, n_seqs, 0.f);
    free(og);
    free(p);
    return rc;
}
