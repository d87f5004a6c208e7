/*
 * gxo.c — CPU oracle for the Gyro routed-MoE layer. TEST INFRASTRUCTURE ONLY (see gxo.h).
 *
 * Built twice by oracle/Makefile:
 *   liboracle.so       -O2 -ffp-contract=off, serial: the parity checker.
 *   liboracle_fast.so  -O3 -DGXO_THREADS -pthread: the timed CPU baseline (the reference's
 *                      own CPU engine is Zig, and no Zig toolchain exists on these machines).
 * Every function names the reference lines it restates.
 */
#ifdef GXO_THREADS
#define _GNU_SOURCE /* syscall() for the futex waits of the worker pool */
#endif
#include "gxo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef GXO_THREADS
#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>
#endif

static float g_codebook[4096]; /* f32 expansion of the table, src/kernels.zig:15-23 */
static int g_codebook_ready = 0;

int gxo_set_codebook(const void *table, size_t bytes) {
    if (!table || bytes != 8192) return -1;
    const uint8_t *b = (const uint8_t *)table;
    for (int i = 0; i < 4096; ++i)
        g_codebook[i] = gxo_fp16_to_fp32((uint16_t)(b[2 * i] | (b[2 * i + 1] << 8)));
    g_codebook_ready = 1;
    return 0;
}

int gxo_max_threads(void) {
#ifdef GXO_THREADS
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
#else
    return 1;
#endif
}

/* Chunked parallel-for in the manner of src/pool.zig:84-114: an atomic cursor hands out
 * [start, start + chunk) ranges and the calling thread participates. The fast build keeps one
 * pool of parked worker threads for the life of the process, as the reference engine does
 * (src/pool.zig:63-81: a generation counter wakes the workers, a pending count tells the caller
 * when they are done; both waits spin briefly, then sleep on a futex), so a call pays a wake-up,
 * not a thread start. */
typedef void (*range_fn)(void *ctx, size_t start, size_t end);
#ifdef GXO_THREADS
#include <linux/futex.h>
#include <sys/syscall.h>

#define GXO_MAX_WORKERS 255
typedef struct pool_state {
    pthread_mutex_t init_lock;
    int workers;                 /* parked threads, started once */
    int active;                  /* workers that drain the current job */
    range_fn fn;
    void *ctx;
    size_t count, chunk;
    atomic_size_t next;
    atomic_uint generation;      /* bumped once per job */
    atomic_uint pending;         /* workers still inside the current job */
} pool_state;
static pool_state g_pool = {PTHREAD_MUTEX_INITIALIZER, 0, 0, NULL, NULL, 0, 0, 0, 0, 0};

static void futex_wait_u32(atomic_uint *addr, unsigned expected) {
    syscall(SYS_futex, (unsigned *)addr, FUTEX_WAIT_PRIVATE, expected, NULL, NULL, 0);
}
static void futex_wake_u32(atomic_uint *addr, int n) {
    syscall(SYS_futex, (unsigned *)addr, FUTEX_WAKE_PRIVATE, n, NULL, NULL, 0);
}

static void pool_drain(void) {
    for (;;) {
        size_t start = atomic_fetch_add_explicit(&g_pool.next, g_pool.chunk, memory_order_relaxed);
        if (start >= g_pool.count) break;
        size_t end = start + g_pool.chunk < g_pool.count ? start + g_pool.chunk : g_pool.count;
        g_pool.fn(g_pool.ctx, start, end);
    }
}

static void *pool_worker(void *arg) {
    const int index = (int)(intptr_t)arg;
    unsigned seen = 0;
    for (;;) {
        unsigned spins = 0, g;
        while ((g = atomic_load_explicit(&g_pool.generation, memory_order_acquire)) == seen) {
            if (++spins < 4096) continue;
            futex_wait_u32(&g_pool.generation, seen);
        }
        seen = g;
        if (index < g_pool.active) pool_drain();
        if (atomic_fetch_sub_explicit(&g_pool.pending, 1, memory_order_acq_rel) == 1)
            futex_wake_u32(&g_pool.pending, 1);
    }
    return NULL;
}

/* Starts the parked workers once (threads - 1 of them, at most GXO_MAX_WORKERS). */
static int pool_start(int threads) {
    pthread_mutex_lock(&g_pool.init_lock);
    if (g_pool.workers == 0) {
        int want = threads - 1 < GXO_MAX_WORKERS ? threads - 1 : GXO_MAX_WORKERS;
        for (int i = 0; i < want; ++i) {
            pthread_t t;
            if (pthread_create(&t, NULL, pool_worker, (void *)(intptr_t)i) != 0) break;
            pthread_detach(t);
            g_pool.workers++;
        }
    }
    pthread_mutex_unlock(&g_pool.init_lock);
    return g_pool.workers;
}
#endif

static void pool_run(int threads, size_t count, size_t chunk, range_fn fn, void *ctx) {
    if (count == 0) return;
    if (chunk == 0) chunk = 1;
#ifdef GXO_THREADS
    if (threads > 1 && count > chunk && pool_start(threads) > 0) {
        g_pool.fn = fn;
        g_pool.ctx = ctx;
        g_pool.count = count;
        g_pool.chunk = chunk;
        g_pool.active = threads - 1 < g_pool.workers ? threads - 1 : g_pool.workers;
        atomic_store_explicit(&g_pool.next, 0, memory_order_relaxed);
        atomic_store_explicit(&g_pool.pending, (unsigned)g_pool.workers, memory_order_release);
        atomic_fetch_add_explicit(&g_pool.generation, 1, memory_order_acq_rel);
        futex_wake_u32(&g_pool.generation, GXO_MAX_WORKERS);
        pool_drain();
        unsigned spins = 0, left;
        while ((left = atomic_load_explicit(&g_pool.pending, memory_order_acquire)) != 0) {
            if (++spins < (1u << 16)) continue;
            futex_wait_u32(&g_pool.pending, left);
        }
        return;
    }
#else
    (void)threads;
#endif
    fn(ctx, 0, count);
}

/* src/gyro.zig:32-41 */
int gxo_type_info(uint32_t type_id, int *k, int *steps, int *block_bytes) {
    int kk, ss, bb;
    switch (type_id) {
        case 144: kk = 8; ss = 32; bb = 34; break; /* TQ2_T */
        case 145: kk = 6; ss = 32; bb = 26; break; /* TQK6 */
        case 146: kk = 7; ss = 32; bb = 30; break; /* TQK7 */
        case 147: kk = 5; ss = 64; bb = 42; break; /* TQP5 */
        case 148: kk = 6; ss = 64; bb = 50; break; /* TQP6 */
        case 149: kk = 7; ss = 64; bb = 58; break; /* TQP7 */
        case 150: kk = 5; ss = 32; bb = 22; break; /* TQK5 */
        case 151: kk = 4; ss = 32; bb = 18; break; /* TQK4 */
        default: return -1;
    }
    if (k) *k = kk;
    if (steps) *steps = ss;
    if (block_bytes) *block_bytes = bb;
    return 0;
}

static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* src/gyro.zig:128-141: exact conversion of every binary16 pattern, subnormals included. */
float gxo_fp16_to_fp32(uint16_t half) {
    uint32_t sign = (uint32_t)(half & 0x8000u) << 16;
    uint32_t exponent = (half >> 10) & 31u;
    uint32_t mantissa = half & 1023u;
    if (exponent == 31) return bits_to_f32(sign | 0x7f800000u | (mantissa << 13));
    if (exponent != 0) return bits_to_f32(sign | ((exponent + 112u) << 23) | (mantissa << 13));
    if (mantissa == 0) return bits_to_f32(sign);
    uint32_t out_exp = 113;
    while ((mantissa & 1024u) == 0) { mantissa <<= 1; out_exp -= 1; }
    return bits_to_f32(sign | (out_exp << 23) | ((mantissa & 1023u) << 13));
}

/* src/gyro.zig:107-117. TQ2_T: previous byte (circular) : this byte. Otherwise a 16-bit
 * window at bit (steps-1-step)*K of the circular LSB-first stream. */
uint32_t gxo_state(uint32_t type_id, const uint8_t *stream, int stream_len, int step) {
    if (type_id == 144) return ((uint32_t)stream[(step + 31) % 32] << 8) | stream[step];
    int k, steps;
    gxo_type_info(type_id, &k, &steps, NULL);
    uint32_t offset = (uint32_t)(steps - 1 - step) * (uint32_t)k;
    uint32_t byte = offset >> 3;
    uint32_t word = (uint32_t)stream[byte] |
                    ((uint32_t)stream[(byte + 1) % (uint32_t)stream_len] << 8) |
                    ((uint32_t)stream[(byte + 2) % (uint32_t)stream_len] << 16);
    return (word >> (offset & 7)) & 0xffffu;
}

/* src/gyro.zig:81-105 (strict): w = d * CB[...] as one binary32 multiply. */
int gxo_decode_row(uint32_t type_id, int state_bits, const uint8_t *src, size_t src_len,
                   float *dst, size_t n) {
    if (state_bits < 0) return -2;
    if (state_bits != 15) return -3;
    int k, steps, bb;
    if (gxo_type_info(type_id, &k, &steps, &bb)) return -1;
    if (n % 128) return -4;
    if (src_len != n / 128 * (size_t)bb) return -5;
    size_t out = 0;
    for (size_t off = 0; off < src_len; off += (size_t)bb) {
        const uint8_t *block = src + off;
        float scale = gxo_fp16_to_fp32((uint16_t)(block[0] | (block[1] << 8)));
        const uint8_t *stream = block + 2;
        int pairs = steps == 64 ? 1 : 2;
        for (int step = 0; step < steps; ++step) {
            uint32_t state = gxo_state(type_id, stream, bb - 2, step);
            uint32_t hash = (state & 0x7fffu) * 0x9e3779b1u;
            for (int pair = 0; pair < pairs; ++pair) {
                uint32_t index = pair == 0 ? hash >> 21 : (hash >> 10) & 2047u;
                volatile float a = scale * g_codebook[index * 2];
                volatile float b = scale * g_codebook[index * 2 + 1];
                dst[out] = a;
                dst[out + 1] = b;
                out += 2;
            }
        }
    }
    return 0;
}

/* src/gyro.zig:143-150 */
static int validate_transform(size_t n, size_t block, const int8_t *signs) {
    if (block == 0 || (block & (block - 1))) return -1;
    if (n % block) return -4;
    if (signs)
        for (size_t i = 0; i < n; ++i)
            if (signs[i] != 1 && signs[i] != -1) return -7;
    return 0;
}

/* src/gyro.zig:152-172: strict butterflies, then one multiply by 1/sqrt(b) per value. */
static void hadamard(float *v, size_t n, size_t block) {
    const float norm = 1.0f / sqrtf((float)block);
    for (size_t start = 0; start < n; start += block) {
        float *b = v + start;
        for (size_t width = 1; width < block; width *= 2)
            for (size_t s = 0; s < block; s += 2 * width)
                for (size_t j = 0; j < width; ++j) {
                    float p = b[s + j], q = b[s + j + width];
                    b[s + j] = p + q;
                    b[s + j + width] = p - q;
                }
        for (size_t j = 0; j < block; ++j) b[j] *= norm;
    }
}

/* src/gyro.zig:177-184 */
int gxo_rotate(float *v, size_t n, size_t block, const int8_t *signs) {
    int rc = validate_transform(n, block, signs);
    if (rc) return rc;
    if (signs) for (size_t i = 0; i < n; ++i) v[i] *= (float)signs[i];
    hadamard(v, n, block);
    return 0;
}

/* src/gyro.zig:188-195 */
int gxo_unrotate(float *v, size_t n, size_t block, const int8_t *signs) {
    int rc = validate_transform(n, block, signs);
    if (rc) return rc;
    hadamard(v, n, block);
    if (signs) for (size_t i = 0; i < n; ++i) v[i] *= (float)signs[i];
    return 0;
}

/* src/kernels.zig:317-338 */
void gxo_rotate_f32(float *x, size_t n, size_t block, const float *signs) {
    if (signs) for (size_t i = 0; i < n; ++i) x[i] *= signs[i];
    hadamard(x, n, block);
}

/* src/kernels.zig:56-67 (f32 and Gyro types only: the non-expert types are out of scope). */
size_t gxo_row_bytes(uint32_t type_id, size_t cols) {
    if (type_id == 0) return cols * 4;
    if (type_id == 1 || type_id == 30) return cols * 2;
    if (type_id == 8) return cols % 32 ? 0 : cols / 32 * 34;
    int bb;
    if (gxo_type_info(type_id, NULL, NULL, &bb) || cols % 128) return 0;
    return cols / 128 * (size_t)bb;
}

/* 8-lane vector reduction of the Zig @reduce(.Add) on a V8. */
static float reduce8(const float a[8]) {
    return ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
}

/* src/kernels.zig:72-84 */
static float dot_f32(const uint8_t *row, const float *x, size_t n) {
    float acc[8] = {0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; ++j) {
            float w;
            memcpy(&w, row + (i + j) * 4, 4);
            acc[j] += w * x[i + j];
        }
    float sum = reduce8(acc);
    for (; i < n; ++i) { float w; memcpy(&w, row + i * 4, 4); sum += w * x[i]; }
    return sum;
}

/* src/kernels.zig:253-261 */
static float dot_dense(const float *a, const float *b, size_t n) {
    float acc[8] = {0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] += a[i + j] * b[i + j];
    float sum = reduce8(acc);
    for (; i < n; ++i) sum += a[i] * b[i];
    return sum;
}

/* src/kernels.zig:136-159: one block in the stored basis (fast-path decode, w = d * cb). */
static void decode_block(uint32_t type_id, int steps, int bb, const uint8_t *block, float *out) {
    const float scale = gxo_fp16_to_fp32((uint16_t)(block[0] | (block[1] << 8)));
    const uint8_t *stream = block + 2;
    if (steps == 32) {
        for (int step = 0; step < 32; ++step) {
            uint32_t state = gxo_state(type_id, stream, bb - 2, step);
            uint32_t h = (state & 0x7fffu) * 0x9e3779b1u;
            uint32_t a = (h >> 21) * 2, b = ((h >> 10) & 2047u) * 2;
            out[step * 4 + 0] = scale * g_codebook[a];
            out[step * 4 + 1] = scale * g_codebook[a + 1];
            out[step * 4 + 2] = scale * g_codebook[b];
            out[step * 4 + 3] = scale * g_codebook[b + 1];
        }
    } else {
        for (int step = 0; step < 64; ++step) {
            uint32_t state = gxo_state(type_id, stream, bb - 2, step);
            uint32_t h = (state & 0x7fffu) * 0x9e3779b1u;
            uint32_t a = (h >> 21) * 2;
            out[step * 2 + 0] = scale * g_codebook[a];
            out[step * 2 + 1] = scale * g_codebook[a + 1];
        }
    }
}

/* src/kernels.zig:161-183: fused TQ2_T dot, per block a 4-lane accumulator times the scale. */
static float dot_tq2(const uint8_t *row, const float *x, size_t cols) {
    float total = 0;
    for (size_t bi = 0; bi < cols / 128; ++bi) {
        const uint8_t *block = row + bi * 34;
        const float scale = gxo_fp16_to_fp32((uint16_t)(block[0] | (block[1] << 8)));
        const uint8_t *stream = block + 2;
        const float *xb = x + bi * 128;
        float acc[4] = {0, 0, 0, 0};
        for (int step = 0; step < 32; ++step) {
            uint32_t state = ((uint32_t)stream[(step + 31) & 31] << 8) | stream[step];
            uint32_t h = (state & 0x7fffu) * 0x9e3779b1u;
            uint32_t a = (h >> 21) * 2, b = ((h >> 10) & 2047u) * 2;
            acc[0] += g_codebook[a] * xb[step * 4 + 0];
            acc[1] += g_codebook[a + 1] * xb[step * 4 + 1];
            acc[2] += g_codebook[b] * xb[step * 4 + 2];
            acc[3] += g_codebook[b + 1] * xb[step * 4 + 3];
        }
        total += scale * ((acc[0] + acc[2]) + (acc[1] + acc[3]));
    }
    return total;
}

/* src/kernels.zig:185-199 */
static float dot_gyro_generic(uint32_t type_id, const uint8_t *row, const float *x, size_t cols) {
    int steps, bb;
    gxo_type_info(type_id, NULL, &steps, &bb);
    float total = 0, tmp[128];
    for (size_t bi = 0; bi < cols / 128; ++bi) {
        decode_block(type_id, steps, bb, row + bi * (size_t)bb, tmp);
        float acc[8] = {0};
        for (int i = 0; i < 128; i += 8)
            for (int j = 0; j < 8; ++j) acc[j] += tmp[i + j] * x[bi * 128 + i + j];
        total += reduce8(acc);
    }
    return total;
}

/* src/kernels.zig:201-210 */
/* src/kernels.zig:86-105 (dotHalf): bf16 widened by a 16-bit shift, f16 converted exactly. */
static float dot_half(int bf, const uint8_t *row, const float *x, size_t n) {
    float sum = 0;
    for (size_t i = 0; i < n; ++i) {
        uint16_t bits = (uint16_t)(row[2 * i] | (row[2 * i + 1] << 8));
        float w = bf ? bits_to_f32((uint32_t)bits << 16) : gxo_fp16_to_fp32(bits);
        sum += w * x[i];
    }
    return sum;
}

/* src/kernels.zig:107-120 (dotQ8): per 32-weight block, d * sum(q * x). */
static float dot_q8(const uint8_t *row, const float *x, size_t n) {
    float total = 0;
    for (size_t b = 0; b < n / 32; ++b) {
        const uint8_t *block = row + b * 34;
        float d = gxo_fp16_to_fp32((uint16_t)(block[0] | (block[1] << 8)));
        float acc = 0;
        for (int j = 0; j < 32; ++j) acc += (float)(int8_t)block[2 + j] * x[b * 32 + j];
        total += d * acc;
    }
    return total;
}

float gxo_dot_row(uint32_t type_id, const uint8_t *row, const float *x, size_t cols) {
    if (type_id == 0) return dot_f32(row, x, cols);
    if (type_id == 1 || type_id == 30) return dot_half(type_id == 30, row, x, cols);
    if (type_id == 8) return dot_q8(row, x, cols);
    if (type_id == 144) return dot_tq2(row, x, cols);
    return dot_gyro_generic(type_id, row, x, cols);
}

/* src/kernels.zig:213-235 (Gyro branch) */
void gxo_decode_row_fast(uint32_t type_id, const uint8_t *row, float *out, size_t cols) {
    int steps, bb;
    gxo_type_info(type_id, NULL, &steps, &bb);
    for (size_t b = 0; b < cols / 128; ++b) decode_block(type_id, steps, bb, row + b * (size_t)bb, out + b * 128);
}

/* src/kernels.zig:281-291 (weight = 1) */
void gxo_rms_norm(float *out, const float *x, size_t n, float eps) {
    float ss = 0;
    for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale;
}

/* src/kernels.zig:340-349 */
void gxo_softmax(float *x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; ++i) m = x[i] > m ? x[i] : m;
    float sum = 0;
    for (size_t i = 0; i < n; ++i) { x[i] = expf(x[i] - m); sum += x[i]; }
    for (size_t i = 0; i < n; ++i) x[i] /= sum;
}

/* src/engine.zig:671-686: insertion top-k; ties prefer the lower index. */
void gxo_topk(const float *values, size_t n, uint32_t *ids, float *weights, size_t k) {
    const uint32_t none = 0xffffffffu;
    for (size_t j = 0; j < k; ++j) { ids[j] = none; weights[j] = -INFINITY; }
    for (size_t i = 0; i < n; ++i) {
        float v = values[i];
        if (v <= weights[k - 1] && ids[k - 1] != none) continue;
        size_t pos = k - 1;
        while (pos > 0 && (v > weights[pos - 1] || ids[pos - 1] == none)) {
            weights[pos] = weights[pos - 1];
            ids[pos] = ids[pos - 1];
            pos -= 1;
        }
        weights[pos] = v;
        ids[pos] = (uint32_t)i;
    }
}

/* src/kernels.zig:307-309 */
static float silu(float x) { return x / (1.0f + expf(-x)); }

/* Shared state of one gxo_moe_ffn call for the parallel ranges. */
typedef struct ffn_ctx {
    const gxo_layer *l;
    const float *x, *xh;
    size_t n, E, F, U, NE, gate_row, down_row;
    float *router, *act, *act_up, *down;
    const uint32_t *start, *order;
} ffn_ctx;

/* Router rows: kernels.matmul, src/engine.zig:526 -> src/kernels.zig:239-268. */
static void router_range(void *p, size_t a, size_t b) {
    ffn_ctx *c = (ffn_ctx *)p;
    for (size_t r = a; r < b; ++r)
        for (size_t t = 0; t < c->n; ++t)
            c->router[t * c->NE + r] =
                dot_f32((const uint8_t *)(c->l->router + r * c->E), c->x + t * c->E, c->E);
}

/* Phase 1, one task per (expert, row), src/engine.zig:568-602. */
static void gate_up_range(void *p, size_t a, size_t b) {
    ffn_ctx *c = (ffn_ctx *)p;
    const size_t E = c->E, F = c->F, U = c->U;
    float *wbuf = malloc(sizeof(float) * E);
    for (size_t task = a; task < b; ++task) {
        size_t e = task / F, row = task % F;
        uint32_t first = c->start[e], last = c->start[e + 1];
        if (first == last) continue;
        const uint8_t *g = c->l->gate + (e * F + row) * c->gate_row;
        const uint8_t *u = c->l->up + (e * F + row) * c->gate_row;
        if (last - first == 1) {
            uint32_t slot = c->order[first];
            const float *xs = c->xh + (slot / U) * E;
            c->act[slot * F + row] = gxo_dot_row(c->l->type_id, g, xs, E);
            c->act_up[slot * F + row] = gxo_dot_row(c->l->type_id, u, xs, E);
            continue;
        }
        gxo_decode_row_fast(c->l->type_id, g, wbuf, E);
        for (uint32_t i = first; i < last; ++i) {
            uint32_t slot = c->order[i];
            c->act[slot * F + row] = dot_dense(wbuf, c->xh + (slot / U) * E, E);
        }
        gxo_decode_row_fast(c->l->type_id, u, wbuf, E);
        for (uint32_t i = first; i < last; ++i) {
            uint32_t slot = c->order[i];
            c->act_up[slot * F + row] = dot_dense(wbuf, c->xh + (slot / U) * E, E);
        }
    }
    free(wbuf);
}

/* Phase 2, one task per (expert, output row), src/engine.zig:609-633. */
static void down_range(void *p, size_t a, size_t b) {
    ffn_ctx *c = (ffn_ctx *)p;
    const size_t E = c->E, F = c->F;
    float *wbuf = malloc(sizeof(float) * F);
    for (size_t task = a; task < b; ++task) {
        size_t e = task / E, row = task % E;
        uint32_t first = c->start[e], last = c->start[e + 1];
        if (first == last) continue;
        const uint8_t *d = c->l->down + (e * E + row) * c->down_row;
        if (last - first == 1) {
            uint32_t slot = c->order[first];
            c->down[slot * E + row] = gxo_dot_row(c->l->type_id, d, c->act + slot * F, F);
            continue;
        }
        gxo_decode_row_fast(c->l->type_id, d, wbuf, F);
        for (uint32_t i = first; i < last; ++i) {
            uint32_t slot = c->order[i];
            c->down[slot * E + row] = dot_dense(wbuf, c->act + slot * F, F);
        }
    }
    free(wbuf);
}

/* Expert phase of src/engine.zig:547-641 for a given routing (ids/weights [n][U]): rotation,
 * grouping, gate/up, SwiGLU, down rotation, down, weighted sum. Slots whose id is not below
 * n_expert are skipped; the expert-parallel model of the tests uses them for slots served by
 * another rank. */
static int experts_phase(const gxo_layer *l, const float *x, size_t n, const uint32_t *ids,
                         const float *weights, float *out, int threads) {
    const size_t E = l->n_embd, F = l->n_ff, U = l->n_used, NE = l->n_expert;
    size_t gate_row = gxo_row_bytes(l->type_id, E), down_row = gxo_row_bytes(l->type_id, F);
    float *xh = malloc(sizeof(float) * n * E);
    float *act = malloc(sizeof(float) * n * U * F);
    float *act_up = malloc(sizeof(float) * n * U * F);
    float *down = malloc(sizeof(float) * n * U * E);
    uint32_t *order = malloc(sizeof(uint32_t) * n * U);
    if (!xh || !act || !act_up || !down || !order) {
        free(xh); free(act); free(act_up); free(down); free(order);
        return -1;
    }
    uint32_t start[513];
    ffn_ctx c = {l, x, xh, n, E, F, U, NE, gate_row, down_row, NULL, act, act_up, down, start, order};
    /* Rotated expert input shared by gate and up, src/engine.zig:547-551. */
    memcpy(xh, x, sizeof(float) * n * E);
    if (l->gate_signs) for (size_t t = 0; t < n; ++t) gxo_rotate_f32(xh + t * E, E, 128, l->gate_signs);
    /* Counting sort of slots by expert, src/engine.zig:553-564. */
    memset(out, 0, sizeof(float) * n * E);
    memset(start, 0, sizeof(start));
    for (size_t i = 0; i < n * U; ++i) if (ids[i] < NE) start[ids[i] + 1] += 1;
    for (size_t e = 0; e < NE; ++e) start[e + 1] += start[e];
    uint32_t fill[513];
    memcpy(fill, start, sizeof(fill));
    for (size_t i = 0; i < n * U; ++i) if (ids[i] < NE) order[fill[ids[i]]++] = (uint32_t)i;
    /* Phase 1: gate/up, chunk 16, src/engine.zig:568. */
    pool_run(threads, NE * F, 16, gate_up_range, &c);
    /* SwiGLU and down-input rotation, src/engine.zig:603-607. */
    for (size_t slot = 0; slot < n * U; ++slot) {
        if (ids[slot] >= NE) continue;
        float *a = act + slot * F;
        const float *up = act_up + slot * F;
        for (size_t i = 0; i < F; ++i) a[i] = silu(a[i]) * up[i];
        if (l->down_signs) gxo_rotate_f32(a, F, 128, l->down_signs);
    }
    /* Phase 2: down, chunk 64, src/engine.zig:609. */
    pool_run(threads, NE * E, 64, down_range, &c);
    /* Weighted sum, src/engine.zig:634-641. */
    for (size_t t = 0; t < n; ++t) {
        float *o = out + t * E;
        for (size_t k = 0; k < U; ++k) {
            size_t slot = t * U + k;
            if (ids[slot] >= NE) continue;
            float wgt = weights[slot];
            const float *v = down + slot * E;
            for (size_t i = 0; i < E; ++i) o[i] += wgt * v[i];
        }
    }
    free(xh); free(act); free(act_up); free(down); free(order);
    return 0;
}

static int layer_ok(const gxo_layer *l) {
    if (!l || !g_codebook_ready || l->type_id == 0) return 0;
    const size_t E = l->n_embd, F = l->n_ff, U = l->n_used, NE = l->n_expert;
    return gxo_row_bytes(l->type_id, E) && gxo_row_bytes(l->type_id, F) && U && NE <= 512 && E && F;
}

/* src/engine.zig:520-642 */
int gxo_moe_ffn(const gxo_layer *l, const float *x, size_t n, float *out,
                uint32_t *ids, float *weights, int threads) {
    if (!layer_ok(l) || !x || !out || !ids || !weights || !l->router || n == 0 || l->n_used > l->n_expert)
        return -1;
    const size_t E = l->n_embd, U = l->n_used, NE = l->n_expert;
    float *router = malloc(sizeof(float) * n * NE);
    if (!router) return -1;
    ffn_ctx c = {l, x, NULL, n, E, l->n_ff, U, NE, 0, 0, router, NULL, NULL, NULL, NULL, NULL};
    /* Router, chunk as kernels.matmul picks it (pool.chunkFor(rows, 8)). */
    size_t router_chunk = threads > 1 ? NE / ((size_t)threads * 4) : NE;
    pool_run(threads, NE, router_chunk > 8 ? router_chunk : 8, router_range, &c);
    /* Softmax, top-k, renormalisation, src/engine.zig:527-540. The optional bias is a
     * harness hook (skewed expert popularity) with no reference counterpart. */
    for (size_t t = 0; t < n; ++t) {
        float *probs = router + t * NE;
        if (l->router_bias) for (size_t e = 0; e < NE; ++e) probs[e] += l->router_bias[e];
        gxo_softmax(probs, NE);
        uint32_t *id = ids + t * U;
        float *w = weights + t * U;
        gxo_topk(probs, NE, id, w, U);
        float sum = 0;
        for (size_t j = 0; j < U; ++j) sum += w[j];
        sum = sum > 6.103515625e-5f ? sum : 6.103515625e-5f;
        for (size_t j = 0; j < U; ++j) {
            w[j] /= sum;
            if (l->expert_weights_scale != 0 && l->expert_weights_scale != 1) w[j] *= l->expert_weights_scale;
        }
    }
    free(router);
    return experts_phase(l, x, n, ids, weights, out, threads);
}

int gxo_moe_experts(const gxo_layer *l, const float *x, size_t n, const uint32_t *ids,
                    const float *weights, float *out, int threads) {
    if (!layer_ok(l) || !x || !out || !ids || !weights) return -1;
    if (n == 0) return 0;
    return experts_phase(l, x, n, ids, weights, out, threads);
}

/* ---- shared expert, src/engine.zig:644-653 ------------------------------------------------
 * out[t] += sigmoid(gate_inp . x[t]) * Down(silu(Gate x[t]) * Up x[t]); the three matrices are
 * plain row-major (kernels.matmul over dotRow, src/kernels.zig:239-268). */
typedef struct shared_ctx {
    const gxo_shared *s;
    const float *x;
    size_t n, E, SF, row_in, row_f;
    float *g, *u, *d;
} shared_ctx;

static void shared_gate_up_range(void *p, size_t a, size_t b) {
    shared_ctx *c = (shared_ctx *)p;
    for (size_t r = a; r < b; ++r)
        for (size_t t = 0; t < c->n; ++t) {
            c->g[t * c->SF + r] = gxo_dot_row(c->s->type_id, c->s->gate + r * c->row_in, c->x + t * c->E, c->E);
            c->u[t * c->SF + r] = gxo_dot_row(c->s->type_id, c->s->up + r * c->row_in, c->x + t * c->E, c->E);
        }
}

static void shared_down_range(void *p, size_t a, size_t b) {
    shared_ctx *c = (shared_ctx *)p;
    for (size_t r = a; r < b; ++r)
        for (size_t t = 0; t < c->n; ++t)
            c->d[t * c->E + r] = gxo_dot_row(c->s->type_id, c->s->down + r * c->row_f, c->g + t * c->SF, c->SF);
}

/* src/kernels.zig:303-305 */
static float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

int gxo_shared_expert(const gxo_shared *s, const float *x, size_t n, size_t E, float *out, int threads) {
    if (!s || !x || !out || !s->gate || !s->up || !s->down || !s->gate_inp || s->n_ff == 0) return -1;
    const size_t SF = s->n_ff;
    const size_t row_in = gxo_row_bytes(s->type_id, E), row_f = gxo_row_bytes(s->type_id, SF);
    if (!row_in || !row_f || (s->type_id != 0 && s->type_id != 1 && s->type_id != 8 && s->type_id != 30)) return -1;
    float *g = malloc(sizeof(float) * n * SF), *u = malloc(sizeof(float) * n * SF), *d = malloc(sizeof(float) * n * E);
    if (!g || !u || !d) { free(g); free(u); free(d); return -1; }
    shared_ctx c = {s, x, n, E, SF, row_in, row_f, g, u, d};
    pool_run(threads, SF, 8, shared_gate_up_range, &c);
    for (size_t i = 0; i < n * SF; ++i) g[i] = silu(g[i]) * u[i];
    pool_run(threads, E, 8, shared_down_range, &c);
    for (size_t t = 0; t < n; ++t) {
        const float gate = sigmoid(dot_f32((const uint8_t *)s->gate_inp, x + t * E, E));
        float *o = out + t * E;
        const float *v = d + t * E;
        for (size_t i = 0; i < E; ++i) o[i] += v[i] * gate;
    }
    free(g); free(u); free(d);
    return 0;
}

/* ---- hyper-connection mixer around the FFN block, src/engine.zig:184-228 ------------------
 * res [n][hc*E] holds hc residual streams per token. hc_mix: per stream RMSNorm with its weight,
 * lo = silu((Down xn) / hc), gate = Up lo, out = mean over streams of xn * sigmoid(gate), and the
 * injection weights Inject xn; hc_combine: res[c] += block_out * 2 sigmoid(inject[c] / hc). */
typedef struct hc_ctx {
    const gxo_hc *w;
    size_t n, HD, R, rb_hd, rb_r;
    const float *xn, *lo;
    float *lo_out, *gate, *inj;
} hc_ctx;

static void hc_down_range(void *p, size_t a, size_t b) {
    hc_ctx *c = (hc_ctx *)p;
    for (size_t r = a; r < b; ++r)
        for (size_t t = 0; t < c->n; ++t)
            c->lo_out[t * c->R + r] = gxo_dot_row(c->w->type_id, c->w->down + r * c->rb_hd, c->xn + t * c->HD, c->HD);
}

static void hc_up_range(void *p, size_t a, size_t b) {
    hc_ctx *c = (hc_ctx *)p;
    for (size_t r = a; r < b; ++r)
        for (size_t t = 0; t < c->n; ++t)
            c->gate[t * c->HD + r] = gxo_dot_row(c->w->type_id, c->w->up + r * c->rb_r, c->lo + t * c->R, c->R);
}

int gxo_hc_mix(const gxo_hc *w, const float *res, size_t n, float *out, float *inject, int threads) {
    if (!w || !res || !out || !w->norm || !w->down || !w->up || w->n_streams == 0 || w->rank == 0) return -1;
    const size_t E = w->n_embd, H = w->n_streams, HD = H * E, R = w->rank;
    const size_t rb_hd = gxo_row_bytes(w->type_id, HD), rb_r = gxo_row_bytes(w->type_id, R);
    if (!rb_hd || !rb_r) return -1;
    float *xn = malloc(sizeof(float) * n * HD), *lo = malloc(sizeof(float) * n * R), *gate = malloc(sizeof(float) * n * HD);
    if (!xn || !lo || !gate) { free(xn); free(lo); free(gate); return -1; }
    const float hcf = (float)H;
    for (size_t t = 0; t < n; ++t)
        for (size_t c = 0; c < H; ++c) {
            const size_t o = t * HD + c * E;
            /* src/kernels.zig:281-291 with the stream's weight */
            float ss = 0;
            for (size_t i = 0; i < E; ++i) ss += res[o + i] * res[o + i];
            const float scale = 1.0f / sqrtf(ss / (float)E + w->eps);
            for (size_t i = 0; i < E; ++i) xn[o + i] = res[o + i] * scale * w->norm[c * E + i];
        }
    hc_ctx c = {w, n, HD, R, rb_hd, rb_r, xn, lo, lo, gate, NULL};
    pool_run(threads, R, 8, hc_down_range, &c);
    for (size_t i = 0; i < n * R; ++i) lo[i] = silu(lo[i] / hcf);
    pool_run(threads, HD, 64, hc_up_range, &c);
    for (size_t t = 0; t < n; ++t) {
        float *dst = out + t * E;
        memset(dst, 0, sizeof(float) * E);
        for (size_t ci = 0; ci < H; ++ci) {
            const size_t o = t * HD + ci * E;
            for (size_t i = 0; i < E; ++i) dst[i] += xn[o + i] * sigmoid(gate[o + i]);
        }
        for (size_t i = 0; i < E; ++i) dst[i] /= hcf;
    }
    if (inject) {
        if (!w->inject) { free(xn); free(lo); free(gate); return -1; }
        for (size_t t = 0; t < n; ++t)
            for (size_t ci = 0; ci < H; ++ci)
                inject[t * H + ci] = gxo_dot_row(w->type_id, w->inject + ci * rb_hd, xn + t * HD, HD);
    }
    free(xn); free(lo); free(gate);
    return 0;
}

int gxo_hc_combine(const gxo_hc *w, float *res, size_t n, const float *block_out, const float *inject) {
    if (!w || !res || !block_out || !inject) return -1;
    const size_t E = w->n_embd, H = w->n_streams, HD = H * E;
    const float hcf = (float)H;
    for (size_t t = 0; t < n; ++t)
        for (size_t c = 0; c < H; ++c) {
            const float wgt = 2.0f * sigmoid(inject[t * H + c] / hcf);
            float *dst = res + t * HD + c * E;
            for (size_t i = 0; i < E; ++i) dst[i] += block_out[t * E + i] * wgt;
        }
    return 0;
}
