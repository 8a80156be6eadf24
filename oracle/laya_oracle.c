/*
 * laya_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the laya-rust reference CPU backend for the encoder
 * forward pass.  It is the parity checker for the CUDA engine and the timed CPU
 * baseline; nothing in the shipped library links or calls it.
 *
 * What it restates (paths are inside the zerodegress/laya-rust project):
 *   - weights.rs:8-64      f2h / h2f (f16 <-> f32, round-to-nearest-even)
 *   - gguf.rs:289-357      GGUF v3 header reader with its validation rules
 *   - gguf.rs:550-571      tensor decode (F32 / F16 / BF16 -> f32)
 *   - weights.rs:270-295   role-driven transpose (arch.rs:306-322 set)
 *   - backend/cpu/mod.rs:47-466  every op of the ops::Backend trait
 *   - graph.rs:62-186      rope tables and the forward graph, with taps
 *   - convert.rs:16-21     rope frequency table
 *
 * Numerics follow the reference exactly: f32 tensors, f64 layer-norm
 * statistics, Abramowitz & Stegun 7.1.26 erf in f64, k-outer f32 GEMM
 * (gemm_nt) and per-output dot products (gemm_t), rows split across
 * LAYA_CPU_THREADS threads, single-threaded attention, glibc expf/logf/cosf/
 * sinf/powf (what Rust's f32 methods call on linux-gnu).  Build without
 * -ffast-math and with -ffp-contract=off so no multiply-add is fused.
 *
 * LAYA_ORACLE_FAST=1 (set by the test suite, never by the timed CPU
 * baseline) computes the same values faster: gemm_nt in register tiles and
 * the attention's (sequence, head) pairs on all threads.  Every output
 * element keeps the reference's operation sequence; tests check bit
 * equality with the reference traversal.
 *
 * Parity status: the op functions are pinned by the reference's own op
 * known-answer tests (tests/ops.rs:42-267) and the f16 conversion by
 * tests/gguf.rs:122-170.  The reference itself (Rust) cannot be compiled in
 * this image, so whole-forward outputs are pinned only through those op KATs.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define H 1024
#define NH 16
#define HD 64
#define NLAYER 28
#define INTER 2624
#define NVOCAB 50368
#define WINDOW 64
#define HEAD_LAYERS 2
#define HEAD_INTER 4096
#define ACT_HIDDEN 256
#define ACT_INPUT (H + 4)
#define QTYPES 3
#define GLOBAL_EVERY 3
static const float SCALE = 0.3535533845424652f; /* arch.rs:7 */
static const float EPS = 1e-5f;                 /* arch.rs:8 */
static const float NEG_BIG = -3.4e38f;          /* cpu/mod.rs:323 */

/* ------------------------------------------------------------------ */
/* f16 <-> f32 (weights.rs:8-64)                                       */
/* ------------------------------------------------------------------ */
uint16_t lo_f2h(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
    int32_t e32 = (int32_t)((b >> 23) & 0xff);
    uint32_t mant = b & 0x7fffff;
    if (e32 == 0xff) return sign | 0x7c00 | (mant ? 0x200 : 0);
    int32_t e = e32 - 112;
    if (e >= 31) return sign | 0x7c00;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = mant | 0x800000;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) r += 1;
        return sign | (uint16_t)r;
    }
    uint32_t r = ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r += 1;
    return sign | (uint16_t)r;
}

float lo_h2f(uint16_t h) {
    uint32_t s = ((uint32_t)(h >> 15)) << 31;
    int32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {
            int32_t ee = -14;
            while (!(m & 0x400)) { m <<= 1; ee -= 1; }
            bits = s | ((uint32_t)(ee + 127) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000 | (m << 13);
    } else {
        bits = s | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ------------------------------------------------------------------ */
/* threads (cpu/mod.rs:47-57)                                          */
/* ------------------------------------------------------------------ */
int lo_nthreads(void) {
    const char *v = getenv("LAYA_CPU_THREADS");
    if (v && *v) {
        long t = strtol(v, NULL, 10);
        if (t > 0) return (int)t;
    }
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c > 0 ? (int)c : 1;
}

/* ------------------------------------------------------------------ */
/* erf / gelu (cpu/mod.rs:59-78)                                       */
/* ------------------------------------------------------------------ */
static float erf_as(float xf) {
    double x = (double)xf;
    const double p = 0.3275911;
    const double a0 = 0.254829592, a1 = -0.284496736, a2 = 1.421413741, a3 = -1.453152027,
                 a4 = 1.061405429;
    double sign = x < 0.0 ? -1.0 : 1.0;
    x = fabs(x);
    double t = 1.0 / (1.0 + p * x);
    double poly = t * (a0 + t * (a1 + t * (a2 + t * (a3 + t * a4))));
    return (float)(sign * (1.0 - poly * exp(-x * x)));
}

static float gelu1(float v) { return 0.5f * v * (1.0f + erf_as(v / 1.4142135381698608f)); }

/* ------------------------------------------------------------------ */
/* GEMMs (cpu/mod.rs:80-126)                                           */
/* ------------------------------------------------------------------ */
typedef struct {
    const float *x, *w;
    float *y;
    size_t row0, row1, kk, n;
} gemm_job;

static void *gemm_nt_worker(void *arg) {
    gemm_job *j = (gemm_job *)arg;
    for (size_t r = j->row0; r < j->row1; r++) {
        const float *xr = j->x + r * j->kk;
        float *yrow = j->y + r * j->n;
        for (size_t kx = 0; kx < j->kk; kx++) {
            const float a = xr[kx];
            const float *wr = j->w + kx * j->n;
            for (size_t ni = 0; ni < j->n; ni++) yrow[ni] += a * wr[ni];
        }
    }
    return NULL;
}

/* Test infrastructure: the same sums as gemm_nt_worker, element by element
 * (y starts at 0 and adds the rounded a*w over k = 0, 1, ... in order, one
 * rounding per multiply and per add: SSE2 multiplies and adds, never fused),
 * computed 4 rows x 8 columns at a time in registers from a copy of the 8
 * columns of w laid out k-major.  A job is a range of 8-column blocks over
 * every row, so w is packed once per GEMM. */
typedef struct {
    const float *x, *w;
    float *y;
    size_t r, kk, n, cb0, cb1;
} tile_job;

#if defined(__x86_64__)
/* The same 4-row tile over 16 columns in 8-wide AVX registers (vmulps and
 * vaddps, never fused), on CPUs that have AVX. */
__attribute__((target("avx"))) static size_t tile16_avx(const float *x, const float *pk, float *y, size_t r,
                                                        size_t kk, size_t n, size_t c0) {
    size_t r0 = 0;
    for (; r0 + 4 <= r; r0 += 4) {
        const float *x0 = x + r0 * kk, *x1 = x0 + kk, *x2 = x1 + kk, *x3 = x2 + kk;
        float *y0 = y + r0 * n + c0;
        __m256 a00 = _mm256_loadu_ps(y0), a01 = _mm256_loadu_ps(y0 + 8);
        __m256 a10 = _mm256_loadu_ps(y0 + n), a11 = _mm256_loadu_ps(y0 + n + 8);
        __m256 a20 = _mm256_loadu_ps(y0 + 2 * n), a21 = _mm256_loadu_ps(y0 + 2 * n + 8);
        __m256 a30 = _mm256_loadu_ps(y0 + 3 * n), a31 = _mm256_loadu_ps(y0 + 3 * n + 8);
        const float *wp = pk;
        for (size_t kx = 0; kx < kk; kx++, wp += 16) {
            const __m256 w0 = _mm256_load_ps(wp), w1 = _mm256_load_ps(wp + 8);
            __m256 b = _mm256_set1_ps(x0[kx]);
            a00 = _mm256_add_ps(a00, _mm256_mul_ps(b, w0));
            a01 = _mm256_add_ps(a01, _mm256_mul_ps(b, w1));
            b = _mm256_set1_ps(x1[kx]);
            a10 = _mm256_add_ps(a10, _mm256_mul_ps(b, w0));
            a11 = _mm256_add_ps(a11, _mm256_mul_ps(b, w1));
            b = _mm256_set1_ps(x2[kx]);
            a20 = _mm256_add_ps(a20, _mm256_mul_ps(b, w0));
            a21 = _mm256_add_ps(a21, _mm256_mul_ps(b, w1));
            b = _mm256_set1_ps(x3[kx]);
            a30 = _mm256_add_ps(a30, _mm256_mul_ps(b, w0));
            a31 = _mm256_add_ps(a31, _mm256_mul_ps(b, w1));
        }
        _mm256_storeu_ps(y0, a00);
        _mm256_storeu_ps(y0 + 8, a01);
        _mm256_storeu_ps(y0 + n, a10);
        _mm256_storeu_ps(y0 + n + 8, a11);
        _mm256_storeu_ps(y0 + 2 * n, a20);
        _mm256_storeu_ps(y0 + 2 * n + 8, a21);
        _mm256_storeu_ps(y0 + 3 * n, a30);
        _mm256_storeu_ps(y0 + 3 * n + 8, a31);
    }
    return r0;
}
#endif

/* 16-column blocks on AVX CPUs (then the 8-column SSE2 tile for a last odd
 * block), 8-column blocks otherwise; rows left over after the 4-row tiles
 * go one at a time, k in order. */
static void *gemm_nt_tiled_worker(void *arg) {
    tile_job *j = (tile_job *)arg;
    const size_t r = j->r, kk = j->kk, n = j->n;
    float *pk = (float *)aligned_alloc(32, ((kk * 16 * sizeof(float) + 31) / 32) * 32 + 32);
#if defined(__x86_64__)
    const int avx = __builtin_cpu_supports("avx");
#else
    const int avx = 0;
#endif
    for (size_t cb = j->cb0; cb < j->cb1;) {
        const size_t c0 = cb * 8;
        size_t r0 = 0;
#if defined(__x86_64__)
        if (avx && cb + 2 <= j->cb1) {
            for (size_t kx = 0; kx < kk; kx++)
                for (int c = 0; c < 16; c++) pk[kx * 16 + c] = j->w[kx * n + c0 + c];
            r0 = tile16_avx(j->x, pk, j->y, r, kk, n, c0);
            for (; r0 < r; r0++) {
                float *yr = j->y + r0 * n + c0;
                for (size_t kx = 0; kx < kk; kx++) {
                    const float a = j->x[r0 * kk + kx];
                    for (int c = 0; c < 16; c++) yr[c] += a * pk[kx * 16 + c];
                }
            }
            cb += 2;
            continue;
        }
#endif
        for (size_t kx = 0; kx < kk; kx++)
            for (int c = 0; c < 8; c++) pk[kx * 8 + c] = j->w[kx * n + c0 + c];
#if defined(__SSE2__)
        for (; r0 + 4 <= r; r0 += 4) {
            const float *x0 = j->x + r0 * kk, *x1 = x0 + kk, *x2 = x1 + kk, *x3 = x2 + kk;
            float *y0 = j->y + r0 * n + c0;
            __m128 a00 = _mm_loadu_ps(y0), a01 = _mm_loadu_ps(y0 + 4);
            __m128 a10 = _mm_loadu_ps(y0 + n), a11 = _mm_loadu_ps(y0 + n + 4);
            __m128 a20 = _mm_loadu_ps(y0 + 2 * n), a21 = _mm_loadu_ps(y0 + 2 * n + 4);
            __m128 a30 = _mm_loadu_ps(y0 + 3 * n), a31 = _mm_loadu_ps(y0 + 3 * n + 4);
            const float *wp = pk;
            for (size_t kx = 0; kx < kk; kx++, wp += 8) {
                const __m128 w0 = _mm_load_ps(wp), w1 = _mm_load_ps(wp + 4);
                __m128 b = _mm_set1_ps(x0[kx]);
                a00 = _mm_add_ps(a00, _mm_mul_ps(b, w0));
                a01 = _mm_add_ps(a01, _mm_mul_ps(b, w1));
                b = _mm_set1_ps(x1[kx]);
                a10 = _mm_add_ps(a10, _mm_mul_ps(b, w0));
                a11 = _mm_add_ps(a11, _mm_mul_ps(b, w1));
                b = _mm_set1_ps(x2[kx]);
                a20 = _mm_add_ps(a20, _mm_mul_ps(b, w0));
                a21 = _mm_add_ps(a21, _mm_mul_ps(b, w1));
                b = _mm_set1_ps(x3[kx]);
                a30 = _mm_add_ps(a30, _mm_mul_ps(b, w0));
                a31 = _mm_add_ps(a31, _mm_mul_ps(b, w1));
            }
            _mm_storeu_ps(y0, a00);
            _mm_storeu_ps(y0 + 4, a01);
            _mm_storeu_ps(y0 + n, a10);
            _mm_storeu_ps(y0 + n + 4, a11);
            _mm_storeu_ps(y0 + 2 * n, a20);
            _mm_storeu_ps(y0 + 2 * n + 4, a21);
            _mm_storeu_ps(y0 + 3 * n, a30);
            _mm_storeu_ps(y0 + 3 * n + 4, a31);
        }
#endif
        for (; r0 < r; r0++) {
            float *yr = j->y + r0 * n + c0;
            for (size_t kx = 0; kx < kk; kx++) {
                const float a = j->x[r0 * kk + kx];
                for (int c = 0; c < 8; c++) yr[c] += a * pk[kx * 8 + c];
            }
        }
        cb += 1;
    }
    free(pk);
    return NULL;
}

static int lo_fast(void) {
    const char *v = getenv("LAYA_ORACLE_FAST");
    return v && v[0] == '1';
}

static void run_gemm_tiled(const float *x, const float *w, float *y, size_t r, size_t kk, size_t n) {
    memset(y, 0, sizeof(float) * r * n);
    const size_t nb = n / 8;
    size_t nt = (size_t)lo_nthreads();
    if (nt > nb) nt = nb ? nb : 1;
    tile_job *jobs = (tile_job *)calloc(nt, sizeof(tile_job));
    pthread_t *tid = (pthread_t *)calloc(nt, sizeof(pthread_t));
    const size_t chunk = (nb + nt - 1) / nt;
    for (size_t t = 0; t < nt; t++) {
        tile_job *j = &jobs[t];
        j->x = x; j->w = w; j->y = y; j->r = r; j->kk = kk; j->n = n;
        j->cb0 = t * chunk < nb ? t * chunk : nb;
        j->cb1 = (t + 1) * chunk < nb ? (t + 1) * chunk : nb;
        if (nt == 1) gemm_nt_tiled_worker(j);
        else pthread_create(&tid[t], NULL, gemm_nt_tiled_worker, j);
    }
    if (nt > 1)
        for (size_t t = 0; t < nt; t++) pthread_join(tid[t], NULL);
    /* the last n % 8 columns, k in order */
    for (size_t ri = 0; ri < r; ri++)
        for (size_t kx = 0; kx < kk; kx++) {
            const float a = x[ri * kk + kx];
            for (size_t c = nb * 8; c < n; c++) y[ri * n + c] += a * w[kx * n + c];
        }
    free(tid);
    free(jobs);
}

static void *gemm_t_worker(void *arg) {
    gemm_job *j = (gemm_job *)arg;
    for (size_t r = j->row0; r < j->row1; r++) {
        const float *xr = j->x + r * j->kk;
        float *yrow = j->y + r * j->n;
        for (size_t ni = 0; ni < j->n; ni++) {
            const float *wr = j->w + ni * j->kk;
            float acc = 0.0f;
            for (size_t kx = 0; kx < j->kk; kx++) acc += xr[kx] * wr[kx];
            yrow[ni] = acc;
        }
    }
    return NULL;
}

static void run_gemm(void *(*fn)(void *), const float *x, const float *w, float *y, size_t r,
                     size_t kk, size_t n) {
    memset(y, 0, sizeof(float) * r * n);
    size_t rr = r > 0 ? r : 1;
    size_t threads = (size_t)lo_nthreads();
    if (threads > rr) threads = rr;
    size_t chunk = (r + threads - 1) / threads;
    if (chunk == 0) chunk = 1;
    size_t nt = (r + chunk - 1) / chunk;
    pthread_t *tid = (pthread_t *)calloc(nt ? nt : 1, sizeof(pthread_t));
    gemm_job *jobs = (gemm_job *)calloc(nt ? nt : 1, sizeof(gemm_job));
    for (size_t t = 0; t < nt; t++) {
        jobs[t].x = x;
        jobs[t].w = w;
        jobs[t].y = y;
        jobs[t].row0 = t * chunk;
        jobs[t].row1 = (t + 1) * chunk < r ? (t + 1) * chunk : r;
        jobs[t].kk = kk;
        jobs[t].n = n;
        if (nt == 1) fn(&jobs[t]);
        else pthread_create(&tid[t], NULL, fn, &jobs[t]);
    }
    if (nt > 1)
        for (size_t t = 0; t < nt; t++) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

/* matmul: x [r, kk] . w [kk, n]  (w in graph layout, out contiguous) */
void lo_matmul(const float *x, size_t r, size_t kk, const float *w, size_t n, float *y) {
    if (lo_fast()) run_gemm_tiled(x, w, y, r, kk, n);
    else run_gemm(gemm_nt_worker, x, w, y, r, kk, n);
}

/* Both traversals by name, for the test that they agree bit for bit. */
void lo_matmul_order(int tiled, const float *x, size_t r, size_t kk, const float *w, size_t n, float *y) {
    if (tiled) run_gemm_tiled(x, w, y, r, kk, n);
    else run_gemm(gemm_nt_worker, x, w, y, r, kk, n);
}

/* matmul_t: x [r, kk] . w[n, kk]^T */
void lo_matmul_t(const float *x, size_t r, size_t kk, const float *w, size_t n, float *y) {
    run_gemm(gemm_t_worker, x, w, y, r, kk, n);
}

/* ------------------------------------------------------------------ */
/* element ops (cpu/mod.rs:145-465)                                    */
/* ------------------------------------------------------------------ */
void lo_embedding(const float *table, size_t dim, const int64_t *ids, size_t nids, float *out) {
    for (size_t r = 0; r < nids; r++)
        memcpy(out + r * dim, table + (size_t)ids[r] * dim, sizeof(float) * dim);
}

void lo_layernorm(const float *x, size_t rows, size_t dim, const float *w, const float *b,
                  float eps, float *out) {
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        float *orow = out + r * dim;
        double sum = 0.0;
        for (size_t i = 0; i < dim; i++) sum += (double)xr[i];
        double mean = sum / (double)dim;
        double vs = 0.0;
        for (size_t i = 0; i < dim; i++) {
            double d = (double)xr[i] - mean;
            vs += d * d;
        }
        double var = vs / (double)dim;
        double rstd = 1.0 / sqrt(var + (double)eps);
        for (size_t i = 0; i < dim; i++) {
            float v = (float)(((double)xr[i] - mean) * rstd) * w[i];
            if (b) v += b[i];
            orow[i] = v;
        }
    }
}

/* split_qkv_rope: qkv [n*len, 3*nh*hd] -> q,k,v [n, nh, len, hd] */
void lo_split_qkv_rope(const float *qkv, size_t rows, const float *cosb, const float *sinb,
                       float scale, size_t nh, size_t hd, size_t len, float *q, float *k,
                       float *v) {
    size_t n = rows / len;
    size_t half = hd / 2;
    size_t stride = 3 * nh * hd;
    for (size_t b = 0; b < n; b++)
        for (size_t s = 0; s < len; s++)
            for (size_t h = 0; h < nh; h++) {
                size_t base = (b * len + s) * stride + h * hd;
                for (size_t d = 0; d < hd; d++) {
                    float qx = qkv[base + d], kx = qkv[base + nh * hd + d];
                    if (cosb && sinb) {
                        size_t j = d % half;
                        float c = cosb[s * half + j];
                        float sn = sinb[s * half + j];
                        float qr = d < half ? -qkv[base + d + half] : qkv[base + d - half];
                        float kr = d < half ? -qkv[base + nh * hd + d + half]
                                            : qkv[base + nh * hd + d - half];
                        qx = qx * c + qr * sn;
                        kx = kx * c + kr * sn;
                    }
                    size_t o = ((b * nh + h) * len + s) * hd + d;
                    q[o] = qx * scale;
                    k[o] = kx * scale;
                    v[o] = qkv[base + 2 * nh * hd + d];
                }
            }
}

/* attention for one (sequence b, head h): cpu/mod.rs:257-314 */
static void attn_one(const float *q, const float *k, const float *v, const float *mask, size_t b, size_t h,
                     size_t nh, size_t len, size_t hd, float *scores, float *out) {
    size_t head = ((b * nh + h) * len) * hd;
    const float *qb = q + head, *kb = k + head, *vb = v + head;
    const float *mb = mask + b * len * len;
    for (size_t s = 0; s < len; s++) {
        const float *qs = qb + s * hd;
        const float *ms = mb + s * len;
        float mx = -3.4e38f;
        for (size_t t = 0; t < len; t++) {
            const float *kt = kb + t * hd;
            float acc = 0.0f;
            for (size_t d = 0; d < hd; d++) acc += qs[d] * kt[d];
            float sc = acc + ms[t];
            scores[t] = sc;
            if (sc > mx) mx = sc;
        }
        float sum = 0.0f;
        for (size_t t = 0; t < len; t++) {
            float e = expf(scores[t] - mx);
            scores[t] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        for (size_t t = 0; t < len; t++) scores[t] *= inv;
        for (size_t d = 0; d < hd; d++) {
            float acc = 0.0f;
            for (size_t t = 0; t < len; t++) acc += scores[t] * vb[t * hd + d];
            out[(b * len + s) * nh * hd + h * hd + d] = acc;
        }
    }
}

typedef struct {
    const float *q, *k, *v, *mask;
    size_t nh, len, hd, p0, p1;
    float *out;
} attn_job;

static void *attn_worker(void *arg) {
    attn_job *j = (attn_job *)arg;
    float *scores = (float *)malloc(sizeof(float) * (j->len ? j->len : 1));
    for (size_t p = j->p0; p < j->p1; p++)
        attn_one(j->q, j->k, j->v, j->mask, p / j->nh, p % j->nh, j->nh, j->len, j->hd, scores, j->out);
    free(scores);
    return NULL;
}

/* With LAYA_ORACLE_FAST=1 (test infrastructure) the (sequence, head) pairs
 * are split across LAYA_CPU_THREADS threads.  Every output element is
 * computed by the same code either way, so the results are identical; the
 * timed CPU baseline keeps the reference's single thread. */

/* attention: q,k,v [n, nh, len, hd], mask [n, len, len] -> out [n*len, nh*hd] */
void lo_attention(const float *q, const float *k, const float *v, const float *mask, size_t n,
                  size_t nh, size_t len, size_t hd, float *out) {
    const size_t pairs = n * nh;
    size_t nt = lo_fast() ? (size_t)lo_nthreads() : 1;
    if (nt > pairs) nt = pairs ? pairs : 1;
    attn_job *jobs = (attn_job *)calloc(nt, sizeof(attn_job));
    pthread_t *tid = (pthread_t *)calloc(nt, sizeof(pthread_t));
    const size_t chunk = (pairs + nt - 1) / nt;
    for (size_t t = 0; t < nt; t++) {
        attn_job *j = &jobs[t];
        j->q = q; j->k = k; j->v = v; j->mask = mask;
        j->nh = nh; j->len = len; j->hd = hd; j->out = out;
        j->p0 = t * chunk < pairs ? t * chunk : pairs;
        j->p1 = (t + 1) * chunk < pairs ? (t + 1) * chunk : pairs;
        if (nt == 1) attn_worker(j);
        else pthread_create(&tid[t], NULL, attn_worker, j);
    }
    if (nt > 1)
        for (size_t t = 0; t < nt; t++) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

/* window_mask: window < 0 means "no window" */
void lo_window_mask(const int64_t *att, size_t n, size_t len, long window, float *m) {
    for (size_t b = 0; b < n; b++)
        for (size_t s = 0; s < len; s++)
            for (size_t t = 0; t < len; t++) {
                size_t diff = s > t ? s - t : t - s;
                int drop = att[b * len + t] == 0 || (window >= 0 && diff > (size_t)window);
                m[(b * len + s) * len + t] = drop ? NEG_BIG : 0.0f;
            }
}

void lo_add(const float *a, const float *b, size_t count, float *out) {
    for (size_t i = 0; i < count; i++) out[i] = a[i] + b[i];
}

void lo_add_bias(const float *x, size_t count, const float *b, size_t dim, float *out) {
    for (size_t i = 0; i < count; i++) out[i] = x[i] + b[i % dim];
}

void lo_gelu(const float *x, size_t count, float *out) {
    for (size_t i = 0; i < count; i++) out[i] = gelu1(x[i]);
}

void lo_gelu_mul(const float *x, size_t rows, size_t half, float *out) {
    size_t stride = 2 * half;
    for (size_t r = 0; r < rows; r++)
        for (size_t c = 0; c < half; c++) {
            float gate = gelu1(x[r * stride + c]);
            out[r * half + c] = gate * x[r * stride + half + c];
        }
}

void lo_relu(const float *x, size_t count, float *out) {
    for (size_t i = 0; i < count; i++) out[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

void lo_add_type(const float *x, size_t rows, size_t dim, const float *type_emb,
                 const int64_t *qtype, size_t len, float *out) {
    for (size_t i = 0; i < rows * dim; i++) {
        size_t seq = (i / dim) / len;
        out[i] = x[i] + type_emb[(size_t)qtype[seq] * dim + (i % dim)];
    }
}

void lo_gather_markers(const float *x, size_t rows, size_t dim, const int64_t *mpos, size_t nm,
                       size_t k, float *out) {
    size_t len = rows / (nm / k);
    for (size_t r = 0; r < nm; r++) {
        size_t b = r / k;
        size_t src = (b * len + (size_t)mpos[r]) * dim;
        memcpy(out + r * dim, x + src, sizeof(float) * dim);
    }
}

void lo_post(const float *sc, size_t count, const int64_t *mmask, size_t k, float *logits,
             float *feats) {
    size_t n = count / k;
    float *pb = (float *)malloc(sizeof(float) * (k ? k : 1));
    for (size_t b = 0; b < n; b++) {
        const float *s = sc + b * k;
        const int64_t *m = mmask + b * k;
        for (size_t j = 0; j < k; j++) {
            float v = m[j] != 0 ? s[j] : -10000.0f;
            logits[b * k + j] = v;
            pb[j] = v;
        }
        float mx = -3.4e38f;
        for (size_t j = 0; j < k; j++) mx = fmaxf(mx, pb[j]);
        float sum = 0.0f;
        for (size_t j = 0; j < k; j++) {
            float e = expf(pb[j] - mx);
            pb[j] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        float t1 = -1.0f, t2 = -1.0f, ent = 0.0f;
        size_t nv = 0;
        for (size_t j = 0; j < k; j++) {
            float p = pb[j] * inv;
            if (p > t1) {
                t2 = t1;
                t1 = p;
            } else if (p > t2) {
                t2 = p;
            }
            ent -= p * logf(fmaxf(p, 1e-9f));
            if (m[j] != 0) nv++;
        }
        if (t2 < 0.0f) t2 = 0.0f;
        float nn = (float)(nv < 2 ? 2 : nv);
        feats[b * 4] = t1;
        feats[b * 4 + 1] = t1 - t2;
        feats[b * 4 + 2] = ent / logf(nn);
        feats[b * 4 + 3] = nn / 255.0f;
    }
    free(pb);
}

void lo_act_input(const float *x, size_t dim, const float *feats, size_t n, size_t nf,
                  size_t len, float *out) {
    for (size_t b = 0; b < n; b++) {
        memcpy(out + b * (dim + nf), x + b * len * dim, sizeof(float) * dim);
        memcpy(out + b * (dim + nf) + dim, feats + b * nf, sizeof(float) * nf);
    }
}

/* convert.rs:16-21 */
void lo_rope_freq(float theta, size_t half, float *out) {
    float d = (float)(2 * half);
    for (size_t j = 0; j < half; j++) out[j] = 1.0f / powf(theta, (float)(2 * j) / d);
}

/* graph.rs:62-84 */
void lo_rope_tables(const float *freq, size_t len, float *cs, float *sn) {
    size_t half = HD / 2;
    for (size_t p = 0; p < len; p++)
        for (size_t j = 0; j < half; j++) {
            float a = (float)p * freq[j];
            cs[p * half + j] = cosf(a);
            sn[p * half + j] = sinf(a);
        }
}

/* ------------------------------------------------------------------ */
/* GGUF v3 reader (gguf.rs:289-357) and tensor decode                  */
/* ------------------------------------------------------------------ */
typedef struct {
    char *name;
    uint32_t nd;
    uint64_t dims[4];
    uint32_t ty;
    uint64_t offset;
} lo_tinfo;

typedef struct {
    FILE *f;
    uint64_t pos, len;
    char *err;
    size_t errlen;
    int bad;
} lo_rd;

static int rd_take(lo_rd *r, void *dst, uint64_t n) {
    if (r->bad) return -1;
    if (r->pos + n > r->len || r->pos + n < r->pos) {
        snprintf(r->err, r->errlen, "gguf: read of %llu bytes at %llu passes end of file (%llu)",
                 (unsigned long long)n, (unsigned long long)r->pos, (unsigned long long)r->len);
        r->bad = 1;
        return -1;
    }
    if (n && fread(dst, 1, (size_t)n, r->f) != n) {
        snprintf(r->err, r->errlen, "gguf: short read");
        r->bad = 1;
        return -1;
    }
    r->pos += n;
    return 0;
}

static uint64_t rd_u64(lo_rd *r) {
    uint64_t v = 0;
    rd_take(r, &v, 8);
    return v;
}
static uint32_t rd_u32(lo_rd *r) {
    uint32_t v = 0;
    rd_take(r, &v, 4);
    return v;
}

static char *rd_string(lo_rd *r) {
    uint64_t n = rd_u64(r);
    if (r->bad) return NULL;
    if (r->pos + n > r->len) {
        snprintf(r->err, r->errlen, "gguf: string of %llu bytes passes end of file",
                 (unsigned long long)n);
        r->bad = 1;
        return NULL;
    }
    char *s = (char *)malloc((size_t)n + 1);
    if (rd_take(r, s, n)) {
        free(s);
        return NULL;
    }
    s[n] = 0;
    return s;
}

/* metadata values are skipped except the few the loader checks */
typedef struct {
    char *key;
    uint32_t ty;
    uint64_t u;    /* integer value (as_u64) */
    double f;      /* float value (as_f32 source) */
    char *s;       /* string value */
} lo_kv;

static int skip_value(lo_rd *r, uint32_t ty, lo_kv *out, int depth) {
    uint8_t b1;
    uint16_t b2;
    uint32_t b4;
    uint64_t b8;
    switch (ty) {
    case 0: rd_take(r, &b1, 1); if (out) out->u = b1; break;
    case 1: rd_take(r, &b1, 1); if (out) out->u = (uint64_t)(int64_t)(int8_t)b1; break;
    case 2: rd_take(r, &b2, 2); if (out) out->u = b2; break;
    case 3: rd_take(r, &b2, 2); if (out) out->u = (uint64_t)(int64_t)(int16_t)b2; break;
    case 4: rd_take(r, &b4, 4); if (out) out->u = b4; break;
    case 5: rd_take(r, &b4, 4); if (out) out->u = (uint64_t)(int64_t)(int32_t)b4; break;
    case 6: {
        float f;
        rd_take(r, &f, 4);
        if (out) out->f = f;
        break;
    }
    case 7: rd_take(r, &b1, 1); break;
    case 8: {
        char *s = rd_string(r);
        if (out) out->s = s;
        else free(s);
        break;
    }
    case 9: {
        uint32_t et = rd_u32(r);
        uint64_t n = rd_u64(r);
        if (r->bad) return -1;
        if (n > (r->len - 1) / 8) {
            snprintf(r->err, r->errlen, "gguf: array of %llu elements is not plausible",
                     (unsigned long long)n);
            r->bad = 1;
            return -1;
        }
        if (depth > 8) {
            snprintf(r->err, r->errlen, "gguf: arrays nested too deep");
            r->bad = 1;
            return -1;
        }
        for (uint64_t i = 0; i < n && !r->bad; i++) skip_value(r, et, NULL, depth + 1);
        break;
    }
    case 10: rd_take(r, &b8, 8); if (out) out->u = b8; break;
    case 11: rd_take(r, &b8, 8); if (out) out->u = b8; break;
    case 12: {
        double d;
        rd_take(r, &d, 8);
        if (out) out->f = d;
        break;
    }
    default:
        snprintf(r->err, r->errlen, "gguf: unknown metadata value type %u", ty);
        r->bad = 1;
        return -1;
    }
    return r->bad ? -1 : 0;
}

/* ------------------------------------------------------------------ */
/* the model (graph.rs:19-46 load, 86-186 forward)                     */
/* ------------------------------------------------------------------ */
typedef struct {
    char name[72];
    float *data;
    size_t dims[2];
    int nd;
} lo_weight;

#define NWEIGHTS 207
typedef struct {
    lo_weight w[NWEIGHTS];
    int nw;
} lo_model;

static char g_names[NWEIGHTS][72];
static int g_transpose[NWEIGHTS];
static int g_names_ready = 0;

/* arch.rs:263-322: the 207 names in load order plus the 120-entry transpose set */
static void build_names(void) {
    if (g_names_ready) return;
    int i = 0;
    const char *fixed[] = {"encoder.embeddings.tok_embeddings.weight", "type_emb.weight",
                           "encoder.final_norm.weight", "rope.freq_full", "rope.freq_sliding",
                           "scorer.0.weight", "scorer.0.bias", "scorer.1.weight", "scorer.1.bias",
                           "scorer.3.weight", "scorer.3.bias", "act_head.0.weight",
                           "act_head.0.bias", "act_head.2.weight", "act_head.2.bias"};
    for (int j = 0; j < 15; j++) {
        snprintf(g_names[i], 72, "%s", fixed[j]);
        g_transpose[i] = (j == 7 || j == 9);
        i++;
    }
    for (int l = 0; l < NLAYER; l++) {
        if (l == 0) snprintf(g_names[i], 72, "encoder.embeddings.norm.weight");
        else snprintf(g_names[i], 72, "encoder.layers.%d.attn_norm.weight", l);
        g_transpose[i++] = 0;
        snprintf(g_names[i], 72, "encoder.layers.%d.mlp_norm.weight", l);
        g_transpose[i++] = 0;
        snprintf(g_names[i], 72, "encoder.layers.%d.attn.Wqkv.weight", l);
        g_transpose[i++] = 1;
        snprintf(g_names[i], 72, "encoder.layers.%d.attn.Wo.weight", l);
        g_transpose[i++] = 1;
        snprintf(g_names[i], 72, "encoder.layers.%d.mlp.Wi.weight", l);
        g_transpose[i++] = 1;
        snprintf(g_names[i], 72, "encoder.layers.%d.mlp.Wo.weight", l);
        g_transpose[i++] = 1;
    }
    for (int l = 0; l < HEAD_LAYERS; l++) {
        const char *suf[] = {"norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias",
                             "self_attn.in_proj_weight", "self_attn.in_proj_bias",
                             "self_attn.out_proj.weight", "self_attn.out_proj.bias",
                             "linear1.weight", "linear1.bias", "linear2.weight", "linear2.bias"};
        const int tr[] = {0, 0, 0, 0, 1, 0, 0, 0, 1, 0, 1, 0};
        for (int j = 0; j < 12; j++) {
            snprintf(g_names[i], 72, "head.layers.%d.%s", l, suf[j]);
            g_transpose[i++] = tr[j];
        }
    }
    g_names_ready = 1;
}

int lo_weight_count(void) {
    build_names();
    return NWEIGHTS;
}
const char *lo_weight_name(int i) {
    build_names();
    return (i >= 0 && i < NWEIGHTS) ? g_names[i] : NULL;
}
int lo_weight_transposed(int i) {
    build_names();
    return (i >= 0 && i < NWEIGHTS) ? g_transpose[i] : -1;
}

static const lo_weight *W(const lo_model *m, const char *name) {
    for (int i = 0; i < m->nw; i++)
        if (strcmp(m->w[i].name, name) == 0) return &m->w[i];
    fprintf(stderr, "weight %s was not loaded\n", name);
    abort();
}

/* A loaded weight's f32 data in graph layout, or NULL (for harnesses that
 * copy the oracle's weights elsewhere). */
const float *lo_weight_data(const lo_model *m, const char *name, size_t *count) {
    for (int i = 0; i < m->nw; i++)
        if (strcmp(m->w[i].name, name) == 0) {
            if (count) *count = m->w[i].nd == 1 ? m->w[i].dims[0] : m->w[i].dims[0] * m->w[i].dims[1];
            return m->w[i].data;
        }
    return NULL;
}

void lo_close(lo_model *m) {
    if (!m) return;
    for (int i = 0; i < m->nw; i++) free(m->w[i].data);
    free(m);
}

/* Loads every weight as f32 in graph layout (Tensors::f32, weights.rs:278-295). */
lo_model *lo_open(const char *path, char *err, size_t errlen) {
    build_names();
    lo_rd r = {0};
    r.err = err;
    r.errlen = errlen;
    r.f = fopen(path, "rb");
    if (!r.f) {
        snprintf(err, errlen, "%s: cannot open", path);
        return NULL;
    }
    fseek(r.f, 0, SEEK_END);
    r.len = (uint64_t)ftell(r.f);
    fseek(r.f, 0, SEEK_SET);
    lo_model *m = NULL;
    lo_tinfo *ti = NULL;
    lo_kv *kv = NULL;
    uint64_t tc = 0, kc = 0;
    uint32_t magic = rd_u32(&r), version = rd_u32(&r);
    if (r.bad) goto fail;
    if (magic != 0x46554747u) {
        snprintf(err, errlen, "%s: not a GGUF file (magic %#010x)", path, magic);
        goto fail;
    }
    if (version != 3) {
        snprintf(err, errlen, "%s: GGUF version %u, want 3", path, version);
        goto fail;
    }
    tc = rd_u64(&r);
    kc = rd_u64(&r);
    if (r.bad) goto fail;
    if (tc > r.len / 64 || kc > r.len / 16 || tc * 64 + kc * 16 > r.len) {
        snprintf(err, errlen, "%s: header claims %llu tensors and %llu metadata entries", path,
                 (unsigned long long)tc, (unsigned long long)kc);
        goto fail;
    }
    kv = (lo_kv *)calloc(kc ? kc : 1, sizeof(lo_kv));
    for (uint64_t i = 0; i < kc; i++) {
        kv[i].key = rd_string(&r);
        kv[i].ty = rd_u32(&r);
        if (r.bad) goto fail;
        if (skip_value(&r, kv[i].ty, &kv[i], 0)) goto fail;
    }
    ti = (lo_tinfo *)calloc(tc ? tc : 1, sizeof(lo_tinfo));
    for (uint64_t i = 0; i < tc; i++) {
        ti[i].name = rd_string(&r);
        ti[i].nd = rd_u32(&r);
        if (r.bad) goto fail;
        if (ti[i].nd == 0 || ti[i].nd > 4) {
            snprintf(err, errlen, "gguf: tensor %s has %u dimensions", ti[i].name, ti[i].nd);
            goto fail;
        }
        for (uint32_t d = 0; d < ti[i].nd; d++) ti[i].dims[d] = rd_u64(&r);
        ti[i].ty = rd_u32(&r);
        ti[i].offset = rd_u64(&r);
        if (r.bad) goto fail;
    }
    uint64_t data_off = (r.pos + 31) / 32 * 32;
    if (data_off > r.len) {
        snprintf(err, errlen, "%s: tensor data starts past end of file", path);
        goto fail;
    }
    for (uint64_t i = 0; i < tc; i++) {
        uint64_t es = ti[i].ty == 0 ? 4 : (ti[i].ty == 1 || ti[i].ty == 30) ? 2 : 0;
        if (!es) {
            snprintf(err, errlen, "gguf: unsupported tensor type %u", ti[i].ty);
            goto fail;
        }
        uint64_t el = 1;
        for (uint32_t d = 0; d < ti[i].nd; d++) el *= ti[i].dims[d];
        if (ti[i].offset % 32) {
            snprintf(err, errlen, "gguf: tensor %s offset %llu is not a multiple of 32",
                     ti[i].name, (unsigned long long)ti[i].offset);
            goto fail;
        }
        if (data_off + ti[i].offset + el * es > r.len) {
            snprintf(err, errlen, "gguf: tensor %s data is outside the file", ti[i].name);
            goto fail;
        }
    }
    /* general.architecture must be "laya" (weights.rs:139-145) */
    {
        int ok = 0;
        for (uint64_t i = 0; i < kc; i++)
            if (kv[i].key && strcmp(kv[i].key, "general.architecture") == 0 && kv[i].s &&
                strcmp(kv[i].s, "laya") == 0)
                ok = 1;
        if (!ok) {
            snprintf(err, errlen, "%s: general.architecture is not \"laya\"", path);
            goto fail;
        }
    }
    m = (lo_model *)calloc(1, sizeof(lo_model));
    for (int wi = 0; wi < NWEIGHTS; wi++) {
        const lo_tinfo *t = NULL;
        for (uint64_t i = 0; i < tc; i++)
            if (strcmp(ti[i].name, g_names[wi]) == 0) t = &ti[i];
        if (!t) {
            snprintf(err, errlen, "%s: no tensor named %s", path, g_names[wi]);
            goto fail;
        }
        /* stored dims are the reverse of the GGUF dims (weights.rs:261-268) */
        size_t sd[4];
        for (uint32_t d = 0; d < t->nd; d++) sd[d] = (size_t)t->dims[t->nd - 1 - d];
        size_t el = 1;
        for (uint32_t d = 0; d < t->nd; d++) el *= sd[d];
        size_t es = t->ty == 0 ? 4 : 2;
        unsigned char *raw = (unsigned char *)malloc(el * es);
        fseek(r.f, (long)(data_off + t->offset), SEEK_SET);
        if (fread(raw, 1, el * es, r.f) != el * es) {
            free(raw);
            snprintf(err, errlen, "%s: short read of %s", path, g_names[wi]);
            goto fail;
        }
        float *v = (float *)malloc(sizeof(float) * el);
        for (size_t i = 0; i < el; i++) {
            if (t->ty == 0) {
                memcpy(&v[i], raw + 4 * i, 4);
            } else if (t->ty == 1) {
                uint16_t h;
                memcpy(&h, raw + 2 * i, 2);
                v[i] = lo_h2f(h);
            } else {
                uint16_t h;
                memcpy(&h, raw + 2 * i, 2);
                uint32_t bits = (uint32_t)h << 16;
                memcpy(&v[i], &bits, 4);
            }
        }
        free(raw);
        lo_weight *w = &m->w[m->nw++];
        snprintf(w->name, 72, "%s", g_names[wi]);
        w->nd = (int)t->nd;
        w->dims[0] = sd[0];
        w->dims[1] = t->nd > 1 ? sd[1] : 1;
        if (g_transpose[wi] && t->nd == 2) {
            size_t a = sd[0], c = sd[1];
            float *o = (float *)malloc(sizeof(float) * el);
            for (size_t i = 0; i < a; i++)
                for (size_t j = 0; j < c; j++) o[j * a + i] = v[i * c + j];
            free(v);
            v = o;
            w->dims[0] = c;
            w->dims[1] = a;
        }
        w->data = v;
    }
    for (uint64_t i = 0; i < tc; i++) free(ti[i].name);
    for (uint64_t i = 0; i < kc; i++) {
        free(kv[i].key);
        free(kv[i].s);
    }
    free(ti);
    free(kv);
    fclose(r.f);
    return m;
fail:
    if (ti)
        for (uint64_t i = 0; i < tc; i++) free(ti[i].name);
    if (kv)
        for (uint64_t i = 0; i < kc; i++) {
            free(kv[i].key);
            free(kv[i].s);
        }
    free(ti);
    free(kv);
    lo_close(m);
    fclose(r.f);
    return NULL;
}

typedef void (*lo_tap_fn)(void *user, const char *stage, const float *data, size_t count);

static float *fa(size_t n) {
    float *p = (float *)malloc(sizeof(float) * (n ? n : 1));
    if (!p) {
        fprintf(stderr, "oracle: out of memory (%zu floats)\n", n);
        abort();
    }
    return p;
}

/* One encoder layer 0..NLAYER-1 in place on the padded residual stream
 * x [n*l, H]: the body of the layer loop of graph.rs:104-123 (layer 0 norms
 * with the embedding norm and adds the attention output to the normed input,
 * later layers add it to x).  Returns -1 on bad arguments. */
int lo_encoder_layer(const lo_model *m, size_t n, size_t l, const int64_t *att, int layer,
                     float *x) {
    if (!(n > 0 && l > 0) || layer < 0 || layer >= NLAYER) return -1;
    size_t rows = n * l, half = HD / 2;
    int global = layer % GLOBAL_EVERY == 0;
    float *cs = fa(l * half), *sn = fa(l * half), *mask = fa(n * l * l);
    lo_rope_tables(W(m, global ? "rope.freq_full" : "rope.freq_sliding")->data, l, cs, sn);
    lo_window_mask(att, n, l, global ? -1 : WINDOW, mask);
    float *t = fa(rows * H), *qkv = fa(rows * 3 * H), *q = fa(rows * H), *kk = fa(rows * H),
          *v = fa(rows * H), *ctx = fa(rows * H), *p = fa(rows * H), *mlp = fa(rows * 2 * INTER),
          *gate = fa(rows * INTER);
    char nm[96];
    if (layer == 0) snprintf(nm, sizeof nm, "encoder.embeddings.norm.weight");
    else snprintf(nm, sizeof nm, "encoder.layers.%d.attn_norm.weight", layer);
    lo_layernorm(x, rows, H, W(m, nm)->data, NULL, EPS, t);
    snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wqkv.weight", layer);
    lo_matmul(t, rows, H, W(m, nm)->data, 3 * H, qkv);
    lo_split_qkv_rope(qkv, rows, cs, sn, SCALE, NH, HD, l, q, kk, v);
    lo_attention(q, kk, v, mask, n, NH, l, HD, ctx);
    snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wo.weight", layer);
    lo_matmul(ctx, rows, H, W(m, nm)->data, H, p);
    lo_add(layer == 0 ? t : x, p, rows * H, x);
    snprintf(nm, sizeof nm, "encoder.layers.%d.mlp_norm.weight", layer);
    lo_layernorm(x, rows, H, W(m, nm)->data, NULL, EPS, t);
    snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wi.weight", layer);
    lo_matmul(t, rows, H, W(m, nm)->data, 2 * INTER, mlp);
    lo_gelu_mul(mlp, rows, INTER, gate);
    snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wo.weight", layer);
    lo_matmul(gate, rows, INTER, W(m, nm)->data, H, p);
    lo_add(x, p, rows * H, x);
    free(cs); free(sn); free(mask); free(t); free(qkv); free(q); free(kk); free(v); free(ctx);
    free(p); free(mlp); free(gate);
    return 0;
}

/* graph.rs:86-186.  layer_limit < 0 runs all NLAYER encoder layers. */
int lo_forward_ex(const lo_model *m, size_t n, size_t l, size_t k, const int64_t *ids,
                  const int64_t *att, const int64_t *mpos, const int64_t *mmask,
                  const int64_t *qtype, float *logits_out, float *act_out, lo_tap_fn tap,
                  void *user) {
    if (!(n > 0 && l > 0 && k > 0)) return -1;
    size_t rows = n * l;
    size_t half = HD / 2;
    float *cos_a = fa(l * half), *sin_a = fa(l * half), *cos_b = fa(l * half),
          *sin_b = fa(l * half);
    lo_rope_tables(W(m, "rope.freq_full")->data, l, cos_a, sin_a);
    lo_rope_tables(W(m, "rope.freq_sliding")->data, l, cos_b, sin_b);
    float *mask_g = fa(n * l * l), *mask_l = fa(n * l * l);
    lo_window_mask(att, n, l, -1, mask_g);
    lo_window_mask(att, n, l, WINDOW, mask_l);

    float *x = fa(rows * H), *t = fa(rows * H), *qkv = fa(rows * 3 * H);
    float *q = fa(rows * H), *kk = fa(rows * H), *v = fa(rows * H), *ctx = fa(rows * H);
    float *p = fa(rows * H), *mlp = fa(rows * 2 * INTER), *gate = fa(rows * INTER);
    float *hmlp = fa(rows * HEAD_INTER), *tmp = fa(rows * HEAD_INTER);
    const lo_weight *emb = W(m, "encoder.embeddings.tok_embeddings.weight");
    lo_embedding(emb->data, H, ids, rows, x);
    if (tap) tap(user, "embed", x, rows * H);
    char nm[96];
    for (int layer = 0; layer < NLAYER; layer++) {
        int global = layer % GLOBAL_EVERY == 0;
        if (layer == 0) snprintf(nm, sizeof nm, "encoder.embeddings.norm.weight");
        else snprintf(nm, sizeof nm, "encoder.layers.%d.attn_norm.weight", layer);
        lo_layernorm(x, rows, H, W(m, nm)->data, NULL, EPS, t);
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wqkv.weight", layer);
        lo_matmul(t, rows, H, W(m, nm)->data, 3 * H, qkv);
        lo_split_qkv_rope(qkv, rows, global ? cos_a : cos_b, global ? sin_a : sin_b, SCALE, NH,
                          HD, l, q, kk, v);
        lo_attention(q, kk, v, global ? mask_g : mask_l, n, NH, l, HD, ctx);
        snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wo.weight", layer);
        lo_matmul(ctx, rows, H, W(m, nm)->data, H, p);
        if (layer == 0) lo_add(t, p, rows * H, x);
        else lo_add(x, p, rows * H, x);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp_norm.weight", layer);
        lo_layernorm(x, rows, H, W(m, nm)->data, NULL, EPS, t);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wi.weight", layer);
        lo_matmul(t, rows, H, W(m, nm)->data, 2 * INTER, mlp);
        lo_gelu_mul(mlp, rows, INTER, gate);
        snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wo.weight", layer);
        lo_matmul(gate, rows, INTER, W(m, nm)->data, H, p);
        lo_add(x, p, rows * H, x);
        if (tap) {
            snprintf(nm, sizeof nm, "enc.%d", layer);
            tap(user, nm, x, rows * H);
        }
    }
    lo_layernorm(x, rows, H, W(m, "encoder.final_norm.weight")->data, NULL, EPS, t);
    lo_add_type(t, rows, H, W(m, "type_emb.weight")->data, qtype, l, x);
    if (tap) tap(user, "final", x, rows * H);
    for (int layer = 0; layer < HEAD_LAYERS; layer++) {
#define HN(s) (snprintf(nm, sizeof nm, "head.layers.%d." s, layer), W(m, nm)->data)
        lo_layernorm(x, rows, H, HN("norm1.weight"), HN("norm1.bias"), EPS, t);
        lo_matmul(t, rows, H, HN("self_attn.in_proj_weight"), 3 * H, qkv);
        lo_add_bias(qkv, rows * 3 * H, HN("self_attn.in_proj_bias"), 3 * H, qkv);
        lo_split_qkv_rope(qkv, rows, NULL, NULL, SCALE, NH, HD, l, q, kk, v);
        lo_attention(q, kk, v, mask_g, n, NH, l, HD, ctx);
        lo_matmul_t(ctx, rows, H, HN("self_attn.out_proj.weight"), H, p);
        lo_add_bias(p, rows * H, HN("self_attn.out_proj.bias"), H, p);
        lo_add(x, p, rows * H, x);
        lo_layernorm(x, rows, H, HN("norm2.weight"), HN("norm2.bias"), EPS, t);
        lo_matmul(t, rows, H, HN("linear1.weight"), HEAD_INTER, hmlp);
        lo_add_bias(hmlp, rows * HEAD_INTER, HN("linear1.bias"), HEAD_INTER, hmlp);
        lo_relu(hmlp, rows * HEAD_INTER, tmp);
        lo_matmul(tmp, rows, HEAD_INTER, HN("linear2.weight"), H, p);
        lo_add_bias(p, rows * H, HN("linear2.bias"), H, p);
        lo_add(x, p, rows * H, x);
#undef HN
        if (tap) {
            snprintf(nm, sizeof nm, "head.%d", layer);
            tap(user, nm, x, rows * H);
        }
    }
    size_t nk = n * k;
    float *mrow = fa(nk * H), *mt = fa(nk * H), *hid = fa(nk * H), *hg = fa(nk * H),
          *sc = fa(nk), *feats = fa(n * 4);
    lo_gather_markers(x, rows, H, mpos, nk, k, mrow);
    lo_layernorm(mrow, nk, H, W(m, "scorer.0.weight")->data, W(m, "scorer.0.bias")->data, EPS,
                 mt);
    lo_matmul(mt, nk, H, W(m, "scorer.1.weight")->data, H, hid);
    lo_add_bias(hid, nk * H, W(m, "scorer.1.bias")->data, H, hid);
    lo_gelu(hid, nk * H, hg);
    lo_matmul(hg, nk, H, W(m, "scorer.3.weight")->data, 1, sc);
    lo_add_bias(sc, nk, W(m, "scorer.3.bias")->data, 1, sc);
    lo_post(sc, nk, mmask, k, logits_out, feats);
    if (tap) tap(user, "logits", logits_out, nk);
    float *aact = fa(n * ACT_INPUT), *ap = fa(n * ACT_HIDDEN), *apg = fa(n * ACT_HIDDEN);
    lo_act_input(x, H, feats, n, 4, l, aact);
    lo_matmul_t(aact, n, ACT_INPUT, W(m, "act_head.0.weight")->data, ACT_HIDDEN, ap);
    lo_add_bias(ap, n * ACT_HIDDEN, W(m, "act_head.0.bias")->data, ACT_HIDDEN, ap);
    lo_gelu(ap, n * ACT_HIDDEN, apg);
    lo_matmul_t(apg, n, ACT_HIDDEN, W(m, "act_head.2.weight")->data, 2, act_out);
    lo_add_bias(act_out, n * 2, W(m, "act_head.2.bias")->data, 2, act_out);
    if (tap) tap(user, "act", act_out, n * 2);

    free(cos_a); free(sin_a); free(cos_b); free(sin_b); free(mask_g); free(mask_l);
    free(x); free(t); free(qkv); free(q); free(kk); free(v); free(ctx); free(p); free(mlp);
    free(gate); free(hmlp); free(tmp); free(mrow); free(mt); free(hid); free(hg); free(sc);
    free(feats); free(aact); free(ap); free(apg);
    return 0;
}
