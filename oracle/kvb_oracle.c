/*
 * kvb_oracle.c -- CPU restatement of kv-cache-bench's fp64 decode-attention oracle.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path, never part of it:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it. The product
 * library (kv_cache_bench_b200/libkvbcuda.so) neither links nor calls anything here, and it
 * fails loudly when its CUDA code is missing instead of falling back to this file.
 *
 * Parity pinning: tests/test_oracle.py checks every function below against golden vectors
 * that the reference's own compiled code wrote (tests/golden/, generator in
 * tests/golden/make_golden.cpp, recipe in oracle/Makefile).
 *
 * What each function restates (paths relative to the reference project root):
 *   kvb_oracle_paged_attention   src/reference.cpp:65-100 (attention_reference: two-pass fp64
 *                                softmax, sequential sums), read through the paged layout of
 *                                src/reference.hpp:44-58 (paged_index) instead of the contiguous
 *                                copy; int8 values are dequantized to fp32 first exactly as
 *                                src/reference.cpp:52-62 (float(int8) * scale) does.
 *   kvb_oracle_contig_attention  src/reference.cpp:65-100 on the contiguous [B][Hkv][max_len][D]
 *                                layout (src/reference.hpp:38-40).
 *   kvb_oracle_quantize_i8       src/reference.cpp:32-51 (per (sequence block, KV head) absmax/127).
 *   kvb_oracle_dequantize_i8     src/reference.cpp:52-62.
 *   kvb_oracle_fp16_bound        tests/gpu_tests.cpp:22-38 (fp16 storage error bound).
 *   kvb_oracle_i8_bound          tests/gpu_tests.cpp:43-62 (int8 storage error bound).
 *
 * Element types: 0 = fp32, 1 = fp16 (IEEE binary16 bits), 2 = int8 with fp32 scales per
 * (physical block, KV head).
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 kvb_half;

enum { KVB_ORACLE_F32 = 0, KVB_ORACLE_F16 = 1, KVB_ORACLE_I8 = 2 };

/* ---- element access -------------------------------------------------------------------- */

/* The value the reference's attention reads for element `i` of a cache of type `type`. For
 * int8 it is the fp32 product float(x) * scale (src/reference.cpp:60), widened to double. */
static inline double load_elem(int type, const void* base, size_t i, float scale) {
    switch (type) {
    case KVB_ORACLE_F32: return (double)((const float*)base)[i];
    case KVB_ORACLE_F16: return (double)((const kvb_half*)base)[i];
    default: return (double)((float)((const int8_t*)base)[i] * scale);
    }
}

/* ---- attention ------------------------------------------------------------------------- */

typedef struct {
    /* shape */
    int B, H, Hkv, D;
    int type;
    /* paged layout (page > 0) or contiguous layout (page == 0, row stride max_len) */
    int page, max_blocks, max_len;
    const float* q;
    const void* k;
    const void* v;
    const int32_t* table;
    const int32_t* lens;
    const float* k_scale;
    const float* v_scale;
    float* out;
    int threads;
} attn_job;

typedef struct {
    const attn_job* job;
    int worker;
} attn_task;

/* Offset of element (b, kvh, t, 0) and the int8 scale slot of its block. */
static inline size_t row_offset(const attn_job* j, int b, int kvh, int t, size_t* scale_slot) {
    if (j->page == 0) {
        *scale_slot = 0;
        return (((size_t)b * j->Hkv + kvh) * (size_t)j->max_len + (size_t)t) * (size_t)j->D;
    }
    const size_t blk = (size_t)j->table[(size_t)b * j->max_blocks + t / j->page];
    *scale_slot = blk * (size_t)j->Hkv + (size_t)kvh;
    return ((blk * (size_t)j->Hkv + (size_t)kvh) * (size_t)j->page + (size_t)(t % j->page)) * (size_t)j->D;
}

static void* attn_worker(void* arg) {
    const attn_task* task = (const attn_task*)arg;
    const attn_job* j = task->job;
    const int D = j->D, H = j->H, G = j->H / j->Hkv, rows = j->B * j->H;
    const float scale = 1.0f / sqrtf((float)D);
    int cap = 0;
    double* p = NULL;
    double* acc = (double*)malloc(sizeof(double) * (size_t)D);
    for (int row = task->worker; row < rows; row += j->threads) {
        const int b = row / H, h = row % H, kvh = h / G, len = j->lens[b];
        const float* qr = j->q + (size_t)row * D;
        if (len > cap) {
            free(p);
            cap = len;
            p = (double*)malloc(sizeof(double) * (size_t)cap);
        }
        double mx = -INFINITY;
        for (int t = 0; t < len; ++t) {
            size_t slot;
            const size_t off = row_offset(j, b, kvh, t, &slot);
            const float ks = j->type == KVB_ORACLE_I8 ? j->k_scale[slot] : 1.0f;
            double dot = 0;
            for (int d = 0; d < D; ++d) dot += (double)qr[d] * load_elem(j->type, j->k, off + (size_t)d, ks);
            p[t] = dot * scale;
            if (p[t] > mx) mx = p[t];
        }
        double sum = 0;
        for (int t = 0; t < len; ++t) sum += (p[t] = exp(p[t] - mx));
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int t = 0; t < len; ++t) {
            size_t slot;
            const size_t off = row_offset(j, b, kvh, t, &slot);
            const float vs = j->type == KVB_ORACLE_I8 ? j->v_scale[slot] : 1.0f;
            for (int d = 0; d < D; ++d) acc[d] += p[t] * load_elem(j->type, j->v, off + (size_t)d, vs);
        }
        for (int d = 0; d < D; ++d) j->out[(size_t)row * D + d] = len ? (float)(acc[d] / sum) : 0.0f;
    }
    free(p);
    free(acc);
    return NULL;
}

static void run_attention(attn_job* j) {
    const int rows = j->B * j->H;
    if (rows <= 0) return;
    if (j->threads < 1) j->threads = 1;
    if (j->threads > rows) j->threads = rows;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)j->threads);
    attn_task* tasks = (attn_task*)malloc(sizeof(attn_task) * (size_t)j->threads);
    for (int w = 0; w < j->threads; ++w) {
        tasks[w].job = j;
        tasks[w].worker = w;
        if (w > 0) pthread_create(&tid[w], NULL, attn_worker, &tasks[w]);
    }
    attn_worker(&tasks[0]);
    for (int w = 1; w < j->threads; ++w) pthread_join(tid[w], NULL);
    free(tid);
    free(tasks);
}

/* out[b][h][:] = softmax_t(q.k_t / sqrt(D)) . v_t over the paged cache (pool [blocks][Hkv][page][D],
 * table [B][max_blocks]). An empty sequence gives exactly 0. */
void kvb_oracle_paged_attention(int B, int H, int Hkv, int D, int type, int page, int max_blocks,
                                const float* q, const void* k, const void* v, const int32_t* table,
                                const int32_t* lens, const float* k_scale, const float* v_scale,
                                float* out, int threads) {
    attn_job j = {B, H, Hkv, D, type, page, max_blocks, 0, q, k, v, table, lens, k_scale, v_scale, out, threads};
    run_attention(&j);
}

/* The same over the contiguous cache [B][Hkv][max_len][D] (fp32 or fp16 only). */
void kvb_oracle_contig_attention(int B, int H, int Hkv, int D, int type, int max_len, const float* q,
                                 const void* k, const void* v, const int32_t* lens, float* out, int threads) {
    attn_job j = {B, H, Hkv, D, type, 0, 0, max_len, q, k, v, NULL, lens, NULL, NULL, out, threads};
    run_attention(&j);
}

/* ---- int8 quantization ----------------------------------------------------------------- */

static inline size_t contig_index(int Hkv, int D, int max_len, int b, int kvh, int t, int d) {
    return (((size_t)b * Hkv + kvh) * (size_t)max_len + (size_t)t) * (size_t)D + (size_t)d;
}

static inline size_t paged_index(int Hkv, int D, int page, int max_blocks, const int32_t* table, int b, int kvh,
                                 int t, int d) {
    const size_t blk = (size_t)table[(size_t)b * max_blocks + t / page];
    return ((blk * (size_t)Hkv + (size_t)kvh) * (size_t)page + (size_t)(t % page)) * (size_t)D + (size_t)d;
}

/* Per (sequence, logical block, KV head): amax over the live tokens, scale = amax / 127 (fp32),
 * x -> clamp(nearbyint(x / scale), -127, 127), or 0 when the scale is 0. Writes the pool
 * [blocks][Hkv][page][D] and scales [blocks][Hkv] at the physical block of the table. */
void kvb_oracle_quantize_i8(int B, int Hkv, int D, int page, int max_blocks, int max_len, const int32_t* table,
                            const int32_t* lens, const float* contig, int8_t* paged, float* scales) {
    for (int b = 0; b < B; ++b)
        for (int i = 0; i * page < lens[b]; ++i)
            for (int kvh = 0; kvh < Hkv; ++kvh) {
                const int t0 = i * page, t1 = lens[b] < t0 + page ? lens[b] : t0 + page;
                float amax = 0;
                for (int t = t0; t < t1; ++t)
                    for (int d = 0; d < D; ++d) {
                        const float a = fabsf(contig[contig_index(Hkv, D, max_len, b, kvh, t, d)]);
                        if (a > amax) amax = a;
                    }
                const float scale = amax / 127.0f;
                scales[(size_t)table[(size_t)b * max_blocks + i] * Hkv + kvh] = scale;
                for (int t = t0; t < t1; ++t)
                    for (int d = 0; d < D; ++d) {
                        const float x = contig[contig_index(Hkv, D, max_len, b, kvh, t, d)];
                        int8_t qv = 0;
                        if (scale > 0) {
                            float r = nearbyintf(x / scale);
                            if (r < -127.0f) r = -127.0f;
                            if (r > 127.0f) r = 127.0f;
                            qv = (int8_t)r;
                        }
                        paged[paged_index(Hkv, D, page, max_blocks, table, b, kvh, t, d)] = qv;
                    }
            }
}

/* Live tokens of the int8 pool back to fp32 in the contiguous layout: float(x) * scale. */
void kvb_oracle_dequantize_i8(int B, int Hkv, int D, int page, int max_blocks, int max_len, const int32_t* table,
                              const int32_t* lens, const int8_t* paged, const float* scales, float* contig) {
    for (int b = 0; b < B; ++b)
        for (int kvh = 0; kvh < Hkv; ++kvh)
            for (int t = 0; t < lens[b]; ++t) {
                const float scale = scales[(size_t)table[(size_t)b * max_blocks + t / page] * Hkv + kvh];
                for (int d = 0; d < D; ++d)
                    contig[contig_index(Hkv, D, max_len, b, kvh, t, d)] =
                        (float)paged[paged_index(Hkv, D, page, max_blocks, table, b, kvh, t, d)] * scale;
            }
}

/* ---- storage error bounds (test tolerances) -------------------------------------------- */

#define KVB_TOL_KERNEL 2e-5
#define KVB_HALF_UNIT (1.0 / 2048)

/* Bound on |out_f16_storage - out_exact|: each score moves by at most
 * E = u * scale * max_t sum_d |q_d k_td|, every softmax weight by a factor within exp(+-2E),
 * and V by u * max|v|; plus the kernel tolerance. k32/v32 are the unrounded fp32 values in the
 * contiguous layout. */
double kvb_oracle_fp16_bound(int B, int H, int Hkv, int D, int max_len, const int32_t* lens, const float* q,
                             const float* k32, const float* v32) {
    const double scale = 1.0 / sqrt((double)D);
    const int G = H / Hkv;
    double E = 0, vmax = 0;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
            for (int t = 0; t < lens[b]; ++t) {
                double acc = 0;
                for (int d = 0; d < D; ++d) {
                    const size_t i = contig_index(Hkv, D, max_len, b, h / G, t, d);
                    acc += fabs((double)q[((size_t)b * H + h) * D + d]) * fabs((double)k32[i]);
                    if (fabs((double)v32[i]) > vmax) vmax = fabs((double)v32[i]);
                }
                if (KVB_HALF_UNIT * scale * acc > E) E = KVB_HALF_UNIT * scale * acc;
            }
    return vmax * (KVB_HALF_UNIT + expm1(2 * E)) + KVB_TOL_KERNEL;
}

/* The int8 version: element moves by at most s/2 for a slice with scale s, so score t moves by
 * scale * sum_d|q_d| * s_k / 2 (max over t is E), V by s_v / 2; max|v| of a slice is 127 s_v. */
double kvb_oracle_i8_bound(int B, int H, int Hkv, int D, int page, int max_blocks, const int32_t* table,
                           const int32_t* lens, const float* q, const float* k_scale, const float* v_scale) {
    const double scale = 1.0 / sqrt((double)D);
    const int G = H / Hkv;
    double E = 0, vq = 0, vmax = 0;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            double q1 = 0;
            for (int d = 0; d < D; ++d) q1 += fabs((double)q[((size_t)b * H + h) * D + d]);
            for (int i = 0; i * page < lens[b]; ++i) {
                const size_t slot = (size_t)table[(size_t)b * max_blocks + i] * Hkv + (size_t)(h / G);
                if (scale * q1 * k_scale[slot] / 2 > E) E = scale * q1 * k_scale[slot] / 2;
                if ((double)v_scale[slot] / 2 > vq) vq = (double)v_scale[slot] / 2;
                if (127.0 * v_scale[slot] > vmax) vmax = 127.0 * v_scale[slot];
            }
        }
    return vmax * expm1(2 * E) + vq + KVB_TOL_KERNEL;
}

/* NaN-aware max |a - b| (src/reference.hpp:27-35): any NaN difference counts as infinite. */
double kvb_oracle_max_abs_diff(const float* a, const float* b, size_t n) {
    double m = 0;
    for (size_t i = 0; i < n; ++i) {
        const double e = fabs((double)a[i] - (double)b[i]);
        if (isnan(e)) return INFINITY;
        if (e > m) m = e;
    }
    return m;
}
