/*
 * CPU restatement of the reference's short-context / masked decode branch:
 * dequantize K and V to the query dtype, then scaled dot-product attention
 * (mlx_qsdpa/__init__.py:49-60 and mlx_qsdpa/dispatch.py:68-83 of
 * Thump604/mlx-qsdpa v0.3.1).
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/ as a large-size checker and by
 * bench.py as the timed CPU baseline ("port" of the reference CPU path, whose
 * own implementation -- MLX's CPU backend -- is not installable here).  The
 * shipped library never links or calls it.
 *
 * Numerics: dequantised values are rounded once to the query dtype
 * (scale*code+bias evaluated in double, then rounded), scores / softmax /
 * output accumulate in float32 (MLX's CPU fallback graph accumulates its
 * matmuls in float32), the output is rounded to the query dtype.
 *
 * Parallelism: a plain pthreads parallel-for over rows (no OpenMP runtime is
 * needed).  Build: see oracle/Makefile (gcc -O3 -shared -pthread).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>


/* ---- minimal pthreads parallel-for: body(lo, hi, ctx) over [0, n) ---- */
typedef void (*range_fn)(long lo, long hi, void* ctx);
typedef struct { range_fn fn; void* ctx; long lo, hi; } range_job;
static void* range_run(void* a) {
    range_job* j = (range_job*)a;
    j->fn(j->lo, j->hi, j->ctx);
    return NULL;
}
static int default_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
static void parallel_for(long n, int threads, range_fn fn, void* ctx) {
    if (threads <= 0) threads = default_threads();
    if (threads > 256) threads = 256;
    if (n < threads) threads = (int)(n > 0 ? n : 1);
    pthread_t tid[256];
    range_job jobs[256];
    long chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].lo = t * chunk; jobs[t].hi = (t + 1) * chunk < n ? (t + 1) * chunk : n;
        if (t > 0) pthread_create(&tid[t], NULL, range_run, &jobs[t]);
    }
    range_run(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
}

static inline float f16_to_f32(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}
static inline uint16_t f64_to_f16(double d) {
    _Float16 x = (_Float16)d;
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}
static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float to_f32(uint16_t v, int dtype) {
    return dtype == 0 ? f16_to_f32(v) : bf16_to_f32(v);
}
static inline uint16_t from_f64(double d, int dtype) {
    return dtype == 0 ? f64_to_f16(d) : f32_to_bf16((float)d);
}

/* Dequantise rows (R, D) of MLX-layout packed codes into dtype bit patterns. */
typedef struct {
    const uint32_t* packed; const uint16_t* scales; const uint16_t* biases;
    uint16_t* out; int D, bits, group_size, dtype;
} deq_ctx;

static void deq_rows(long lo, long hi, void* p) {
    const deq_ctx* c = (const deq_ctx*)p;
    const int epw = 32 / c->bits;
    const int pd = c->D / epw;
    const int G = c->D / c->group_size;
    const uint32_t mask = (1u << c->bits) - 1u;
    for (long r = lo; r < hi; ++r) {
        const uint32_t* w = c->packed + r * pd;
        const uint16_t* s = c->scales + r * G;
        const uint16_t* b = c->biases ? c->biases + r * G : NULL;
        uint16_t* o = c->out + r * (long)c->D;
        for (int d = 0; d < c->D; ++d) {
            uint32_t code = (w[d / epw] >> (c->bits * (d % epw))) & mask;
            int g = d / c->group_size;
            double v = (double)to_f32(s[g], c->dtype) * (double)code +
                       (b ? (double)to_f32(b[g], c->dtype) : 0.0);
            o[d] = from_f64(v, c->dtype);
        }
    }
}

void oracle_dequantize(const uint32_t* packed, const uint16_t* scales,
                       const uint16_t* biases, uint16_t* out, long rows, int D,
                       int bits, int group_size, int dtype, int threads) {
    deq_ctx c = {packed, scales, biases, out, D, bits, group_size, dtype};
    parallel_for(rows, threads, deq_rows, &c);
}

/*
 * Decode attention over dequantised K/V (all arrays contiguous):
 *   q (B, Hq, D), kd/vd (B, Hkv, N, D) dtype bits, out (B, Hq, D) dtype bits.
 */
typedef struct {
    const uint16_t *q, *kd, *vd; uint16_t* out;
    int Hq, Hkv; long N; int D, dtype; float scale;
} att_ctx;

static void att_rows(long lo, long hi, void* p) {
    const att_ctx* c = (const att_ctx*)p;
    const int D = c->D;
    const long N = c->N;
    const int rep = c->Hq / c->Hkv;
    float* sc = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
    float* acc = (float*)malloc(sizeof(float) * (size_t)D);
    for (long bh = lo; bh < hi; ++bh) {
        long b = bh / c->Hq;
        int h = (int)(bh % c->Hq), kvh = h / rep;
        const uint16_t* K = c->kd + (b * c->Hkv + kvh) * N * D;
        const uint16_t* V = c->vd + (b * c->Hkv + kvh) * N * D;
        for (int d = 0; d < D; ++d) qf[d] = to_f32(c->q[bh * D + d], c->dtype) * c->scale;
        float mx = -INFINITY;
        for (long n = 0; n < N; ++n) {
            const uint16_t* kr = K + n * D;
            float s = 0.f;
            for (int d = 0; d < D; ++d) s += qf[d] * to_f32(kr[d], c->dtype);
            sc[n] = s;
            if (s > mx) mx = s;
        }
        float l = 0.f;
        for (int d = 0; d < D; ++d) acc[d] = 0.f;
        for (long n = 0; n < N; ++n) {
            float pr = expf(sc[n] - mx);
            l += pr;
            const uint16_t* vr = V + n * D;
            for (int d = 0; d < D; ++d) acc[d] += pr * to_f32(vr[d], c->dtype);
        }
        for (int d = 0; d < D; ++d)
            c->out[bh * D + d] = from_f64(l > 0.f ? (double)(acc[d] / l) : 0.0, c->dtype);
    }
    free(sc);
    free(qf);
    free(acc);
}

void oracle_attend(const uint16_t* q, const uint16_t* kd, const uint16_t* vd,
                   uint16_t* out, int B, int Hq, int Hkv, long N, int D,
                   int dtype, float scale, int threads) {
    att_ctx c = {q, kd, vd, out, Hq, Hkv, N, D, dtype, scale};
    parallel_for((long)B * Hq, threads, att_rows, &c);
}

/* Full branch: dequantise K and V into caller buffers, then attend. */
void oracle_decode(const uint16_t* q, const uint32_t* pk, const uint32_t* pv,
                   const uint16_t* ks, const uint16_t* vs, const uint16_t* kb,
                   const uint16_t* vb, uint16_t* out, uint16_t* kd, uint16_t* vd,
                   int B, int Hq, int Hkv, long N, int D, int bits,
                   int group_size, int dtype, float scale, int threads) {
    long rows = (long)B * Hkv * N;
    oracle_dequantize(pk, ks, kb, kd, rows, D, bits, group_size, dtype, threads);
    oracle_dequantize(pv, vs, vb, vd, rows, D, bits, group_size, dtype, threads);
    oracle_attend(q, kd, vd, out, B, Hq, Hkv, N, D, dtype, scale, threads);
}

int oracle_max_threads(void) { return default_threads(); }
