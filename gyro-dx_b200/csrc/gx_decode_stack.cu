// gx_decode_stack.cu — the whole decode stack (few tokens, many layers) as one persistent
// cooperative kernel.
//
// Per layer, in order (src/engine.zig:520-642 per layer; the pre-norm residual between layers):
//   R  router rows of this CTA: raw logits W_r x for every token, and the token's sum of squares
//      (RMSNorm scale) from the same loads                                  -> grid barrier
//   T  every CTA selects the experts of every token from the logits (softmax, top-U with
//      lower-index ties, renormalisation), one warp per token, into shared memory
//   G  gate/up units of this CTA: bulk-copied tiles, rotated input, trellis decode on mma.sync,
//      SwiGLU -> act; the next layer's router rows are prefetched into L2   -> grid barrier
//   D  down units of this CTA: rotated act, decode GEMV over all U slots, weighted sum plus the
//      residual -> next layer's input (or the output)                      -> grid barrier
//
// A chain of per-phase kernels pays a launch transition and a codebook staging per phase; here
// the codebook is staged once per stack and phases meet at grid barriers. The barrier is a
// monotonic counter in global memory (zeroed before the launch); every wait on it is bounded
// by kWaitLimitNs and ends the kernel with KERR_WAIT. The launch is cooperative, so all CTAs are
// resident. Data other CTAs wrote during the kernel (logits, act, layer inputs) is read with
// L2-coherent loads (ld.global.cg), never through the non-coherent or L1 paths.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "gx_device.cuh"
#include "gx_gemv.cuh"
#include "gx_internal.h"

namespace gx {

#ifdef GX_TRACE
// Instrumented builds: %globaltimer at the phase boundaries of one layer, per CTA.
__device__ long long gx_stack_trace[160][20];
#define GX_STACK_MARK(l, trace_l, p)                                                                \
    do {                                                                                            \
        if ((l) == (trace_l) && threadIdx.x == 0 && blockIdx.x < 160)                               \
            gx_stack_trace[blockIdx.x][p] = (long long)globaltimer_ns();                            \
    } while (0)
#define GX_STACK_MARK_IF(on, p) GX_STACK_MARK((on) ? 0 : 1, 0, p)
// SM cycle counter at a point, for intra-phase durations (slots 17..19 hold clock64 values)
#define GX_STACK_CLK_IF(on, p)                                                                      \
    do {                                                                                            \
        if ((on) && threadIdx.x == 0 && blockIdx.x < 160) gx_stack_trace[blockIdx.x][p] = clock64(); \
    } while (0)
#else
#define GX_STACK_MARK(l, trace_l, p) do {} while (0)
#define GX_STACK_MARK_IF(on, p) do {} while (0)
#define GX_STACK_CLK_IF(on, p) do {} while (0)
#endif

namespace {

constexpr int kThreads = 512, kWarps = 16, kNC = 16;
constexpr int kKBWD = 2;  // down: (slot, block) pairs per warp (U * F / 128 <= 32)
// Dynamic shared memory cap: 227 KB per block less room for the kernel's static shared memory.
constexpr int kSmemBudget = 226 * 1024;

__device__ __forceinline__ float ldcg_act(const void *p, int bf16, size_t i) {
    if (bf16) {
        const unsigned short b = __ldcg(reinterpret_cast<const unsigned short *>(p) + i);
        return __uint_as_float((uint32_t)b << 16);
    }
    return __ldcg(reinterpret_cast<const float *>(p) + i);
}

__device__ __forceinline__ void store_act(void *p, int bf16, size_t i, float v) {
    if (bf16)
        reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float *>(p)[i] = v;
}

// Grid-wide barrier number `n` (1, 2, ...): every CTA adds one to the counter and waits until
// it reaches n * gridDim.x. Returns false for every thread of the CTA if the wait expired.
__device__ __forceinline__ bool grid_barrier(unsigned *counter, unsigned n, int *err) {
    __syncthreads();
    int ok = 1;
    if (threadIdx.x == 0) {
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
        const unsigned target = n * gridDim.x;
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
            if (v >= target) break;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicExch(err, KERR_WAIT);
                ok = 0;
                break;
            }
            __nanosleep(20);
        }
        __threadfence();
    }
    return __syncthreads_and(ok) != 0;
}

// An opaque copy of v: values derived from it inside a phase are recomputed per layer instead of
// being hoisted out of the layer loop, where every phase's geometry would stay live at once.
__device__ __forceinline__ int opaque(int v) {
    asm volatile("" : "+r"(v));
    return v;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Rotated 128-column block of one activation row into xs (this warp's 128 floats), reading
// data another CTA may have written in this kernel: xs = H128(signs * scale * v) / sqrt(128).
__device__ __forceinline__ void rotated_block_cg(const void *src, int bf16, size_t base, float scale,
                                                 const float *signs, int sbase, float *xs, int lane) {
    float v[4];
    if (bf16) {
        const uint2 q = __ldcg(reinterpret_cast<const uint2 *>(reinterpret_cast<const unsigned short *>(src) + base +
                                                               4 * lane));
        v[0] = __uint_as_float(q.x << 16);
        v[1] = __uint_as_float(q.x & 0xffff0000u);
        v[2] = __uint_as_float(q.y << 16);
        v[3] = __uint_as_float(q.y & 0xffff0000u);
    } else {
        const float4 q = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(src) + base + 4 * lane));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= scale;
    if (signs) {
        const float4 g = __ldg(reinterpret_cast<const float4 *>(signs + sbase + 4 * lane));
        v[0] *= g.x; v[1] *= g.y; v[2] *= g.z; v[3] *= g.w;
        fwht128_warp(v, lane);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) xs[4 * lane + j] = v[j];
    __syncwarp();
}

// Expert selection of one token by the whole CTA, one expert per thread (NE <= 512): softmax of
// scale * logit + bias (src/kernels.zig:340-349), the rank of every expert by (probability, lower
// index first) (src/engine.zig:671-686), the U best in rank order, renormalisation by
// max(sum, 2^-14) and the optional expert_weights_scale (src/engine.zig:533-539).
// red: 32 floats, keys: 512 slots of shared memory.
__device__ void select_token_block(const float *logits, const float *bias, int NE, int U, float scale, float wscale,
                                   uint32_t *ids, float *w, float *red, unsigned long long *keys, bool tr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool live = tid < NE;
    GX_STACK_CLK_IF(tr, 17);
    const float l = live ? __ldcg(logits + tid) * scale + (bias ? __ldg(bias + tid) : 0.f) : -INFINITY;
    float m = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) m = fmaxf(m, red[i]);
    GX_STACK_MARK_IF(tr, 12);
    const float e = live ? expf(l - m) : 0.f;
    float s = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[16 + warp] = s;
    __syncthreads();
    s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += red[16 + i];
    const float p = e / s;
    // key order = probability, then lower index: keys are unique, so ranks are a permutation
    const unsigned long long key = live ? ((unsigned long long)__float_as_uint(p) << 32) | (0xffffffffu - (uint32_t)tid)
                                        : 0ull;
    keys[tid] = key;
    __syncthreads();
    GX_STACK_MARK_IF(tr, 13);
    if (live) {
        // keys past NE are zero (threads >= NE store 0), so whole groups of 8 can be read
        int rank = 0;
        const ulonglong2 *k2 = reinterpret_cast<const ulonglong2 *>(keys);
        for (int j = 0; j < (NE + 7) / 8 && rank < U; ++j) {
            const ulonglong2 q0 = k2[4 * j], q1 = k2[4 * j + 1], q2 = k2[4 * j + 2], q3 = k2[4 * j + 3];
            rank += (q0.x > key) + (q0.y > key) + (q1.x > key) + (q1.y > key) + (q2.x > key) + (q2.y > key) +
                    (q3.x > key) + (q3.y > key);
        }
        if (rank < U) {
            ids[rank] = (uint32_t)tid;
            w[rank] = p;
        }
    }
    __syncthreads();
    GX_STACK_MARK_IF(tr, 14);
    GX_STACK_CLK_IF(tr, 18);
    if (warp == 0) {
        const float wk = lane < U ? w[lane] : 0.f;
        float total = 0.f;
        for (int k = 0; k < U; ++k) total += __shfl_sync(0xffffffffu, wk, k);
        total = fmaxf(total, 6.103515625e-5f);
        if (lane < U) {
            float v = wk / total;
            if (wscale != 0.f && wscale != 1.f) v *= wscale;
            w[lane] = v;
        }
    }
    __syncthreads();
    GX_STACK_CLK_IF(tr, 19);
}

}  // namespace

extern __shared__ __align__(128) uint8_t gx_stack_smem[];


// Geometry and shared-memory carve-up of the stack kernel, recomputed where needed so that no
// phase keeps it live in registers.
struct StackGeo {
    int E, F, U, NE, n_tok, NB, NBF, WB, RG, NT, UPS, unit_proj, gu_unit, NTD, slot_bytes, dn_unit, NPAIR, P,
        stage_bytes;
    uint32_t *cb;
    uint8_t *stage;
    float *part;       // [P][32][8]
    float *xs;         // [16 warps][128]
    float *red;        // [16 warps][5][16 tokens]
    uint32_t *sel_ids; // [16 tokens][16]
    float *sel_w;      // [16 tokens][16]
    float *sel_scale;  // [16 tokens]
    float *tred;       // [32] selection reductions
    uint64_t *bar;     // [2]
};

template <uint32_t T>
__device__ __forceinline__ StackGeo stack_geo(const StackArgs &a, int P) {
    constexpr int TB = tile_bytes(T);
    StackGeo g;
    g.E = a.E; g.F = a.F; g.U = a.U; g.NE = a.NE; g.n_tok = a.n_tok;
    g.NB = a.E >> 7;
    g.NBF = a.F >> 7;
    g.WB = g.NB < 16 ? g.NB : 16;
    g.RG = 16 / g.WB;
    g.NT = a.F >> 3;
    g.UPS = (g.NT + g.RG - 1) / g.RG;
    g.unit_proj = g.RG * g.NB * TB;
    g.gu_unit = 2 * g.unit_proj;
    g.NTD = a.E >> 3;
    g.slot_bytes = g.NBF * TB;
    g.dn_unit = a.U * g.slot_bytes;
    g.NPAIR = a.U * g.NBF;
    g.P = P;
    const int unit_max = g.gu_unit > g.dn_unit ? g.gu_unit : g.dn_unit;
    g.stage_bytes = ((P * unit_max + 127) / 128) * 128;
    g.cb = reinterpret_cast<uint32_t *>(gx_stack_smem);
    g.stage = gx_stack_smem + Codebook<kNC>::BYTES;
    g.part = reinterpret_cast<float *>(g.stage + 2 * g.stage_bytes);
    g.xs = g.part + P * 32 * 8;
    g.red = g.xs + kWarps * 128;
    g.sel_ids = reinterpret_cast<uint32_t *>(g.red + kWarps * 80);
    g.sel_w = reinterpret_cast<float *>(g.sel_ids + 256);
    g.sel_scale = g.sel_w + 256;
    g.tred = g.sel_scale + 16;
    g.bar = reinterpret_cast<uint64_t *>(g.tred + 32);
    return g;
}

// Waits for absolute stage s; on expiry every thread sees false after the copies still in
// flight into this CTA's shared memory (stages s and s+1, up to `last`) got one more bounded wait.
__device__ __forceinline__ bool wait_stage(uint64_t *bar, int s, int last, int *err) {
    const bool ok = mbar_wait(&bar[s & 1], (uint32_t)((s >> 1) & 1), err);
    if (__syncthreads_and(ok)) return true;
    if (threadIdx.x == 0)
        for (int t = s; t <= s + 1 && t <= last; ++t) mbar_wait(&bar[t & 1], (uint32_t)((t >> 1) & 1), nullptr);
    __syncthreads();
    return false;
}

// ---- R: raw logits of this CTA's router rows and every token's RMSNorm scale ---------------
__device__ __forceinline__ void phase_router(const StackArgs &a, const float *router, const void *cur, int cur_bf16,
                                          float *sel_scale, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x, E = a.E, NE = a.NE, n_tok = a.n_tok;
    const int chunk = E / kWarps;  // columns per warp (a multiple of 8)
    const int c0 = warp * chunk + 4 * lane;
    const bool on = 4 * lane < chunk;
    int rows[4];
    int nr = 0;
    for (int e = cta; e < NE && nr < 4; e += G) rows[nr++] = e;
    float4 wv[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
        if (r < nr && on) wv[r] = __ldg(reinterpret_cast<const float4 *>(router + (size_t)rows[r] * E + c0));
    for (int t = 0; t < n_tok; ++t) {
        float xv[4] = {0.f, 0.f, 0.f, 0.f};
        if (on) {
            const size_t o = (size_t)t * E + c0;
            if (cur_bf16) {
                const uint2 q = __ldcg(reinterpret_cast<const uint2 *>(reinterpret_cast<const unsigned short *>(cur) + o));
                xv[0] = __uint_as_float(q.x << 16);
                xv[1] = __uint_as_float(q.x & 0xffff0000u);
                xv[2] = __uint_as_float(q.y << 16);
                xv[3] = __uint_as_float(q.y & 0xffff0000u);
            } else {
                const float4 q = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(cur) + o));
                xv[0] = q.x; xv[1] = q.y; xv[2] = q.z; xv[3] = q.w;
            }
        }
        float acc[5];
        acc[4] = xv[0] * xv[0] + xv[1] * xv[1] + xv[2] * xv[2] + xv[3] * xv[3];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            acc[r] = (r < nr && on) ? wv[r].x * xv[0] + wv[r].y * xv[1] + wv[r].z * xv[2] + wv[r].w * xv[3] : 0.f;
#pragma unroll
        for (int r = 0; r < 5; ++r)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 5; ++r) red[(warp * 5 + r) * 16 + t] = acc[r];
        }
    }
    __syncthreads();
    if (tid < n_tok * 5) {
        const int t = tid % n_tok, r = tid / n_tok;
        float s = 0.f;
        for (int w = 0; w < kWarps; ++w) s += red[(w * 5 + r) * 16 + t];
        if (r == 4) sel_scale[t] = a.norm_eps > 0.f ? 1.0f / sqrtf(s / (float)E + a.norm_eps) : 1.f;
        else if (r < nr) a.logits[(size_t)t * NE + rows[r]] = s;
    }
}

// Issues down stage s (absolute stage index s_abs) of this CTA's down units: one bulk copy per
// (unit, slot) into the stage buffer of s_abs. Called by warp 0.
template <uint32_t T>
__device__ __forceinline__ void issue_down_stage(const StackGeo &g, const StackLayer &L, int v0, int v1, int s,
                                                 int s_abs) {
    const int lane = threadIdx.x & 31, U = g.U;
    uint8_t *buf = g.stage + (s_abs & 1) * g.stage_bytes;
    const int ua = v0 + s * g.P, ub = min(ua + g.P, v1);
    if (lane == 0) mbar_expect_tx(&g.bar[s_abs & 1], (uint32_t)((ub - ua) * g.dn_unit));
    __syncwarp();
    for (int q = lane; q < (ub - ua) * U; q += 32) {
        const int u = ua + q / U, k = q % U;
        const int t = u / g.NTD, i = u % g.NTD;
        const uint32_t e = g.sel_ids[t * 16 + k];
        bulk_g2s(buf + (u - ua) * g.dn_unit + k * g.slot_bytes,
                 L.down + (uint64_t)e * L.down_expert_bytes + (uint64_t)i * g.slot_bytes, (uint32_t)g.slot_bytes,
                 &g.bar[s_abs & 1]);
    }
}

__device__ __forceinline__ void down_range(const StackGeo &g, int &v0, int &v1) {
    const int n_units = g.n_tok * g.NTD;
    v0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
    v1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
}

// ---- G: gate/up units of this CTA, SwiGLU into act -------------------------------------------
template <uint32_t T>
__device__ __forceinline__ bool phase_gate_up(const StackArgs &a, const StackLayer &L, const void *cur, int cur_bf16,
                                           int P, int sbase, const float *next_router, const float *next_bias,
                                           bool early_down, bool tr) {
    constexpr int TB = tile_bytes(T);
    P = opaque(P);
    const StackGeo g = stack_geo<T>(a, P);
    const int tid = opaque((int)threadIdx.x), lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x, U = g.U;
    const int n_units = g.n_tok * U * g.UPS;
    const int u0 = (int)((long long)cta * n_units / G), u1 = (int)((long long)(cta + 1) * n_units / G);
    const int n_st = (u1 - u0 + P - 1) / P;
    auto issue = [&](int s) {  // warp 0
        uint8_t *buf = g.stage + ((sbase + s) & 1) * g.stage_bytes;
        const int ua = u0 + s * P, ub = min(ua + P, u1);
        if (lane == 0) {
            uint32_t total = 0;
            for (int u = ua; u < ub; ++u) total += 2u * (uint32_t)(min(g.RG, g.NT - (u % g.UPS) * g.RG) * g.NB * TB);
            mbar_expect_tx(&g.bar[(sbase + s) & 1], total);
        }
        __syncwarp();
        for (int k = lane; k < (ub - ua) * 2; k += 32) {
            const int u = ua + (k >> 1), proj = k & 1;
            const int slot = u / g.UPS, ui = u % g.UPS;
            const uint32_t bytes = (uint32_t)(min(g.RG, g.NT - ui * g.RG) * g.NB * TB);
            const uint32_t e = g.sel_ids[(slot / U) * 16 + slot % U];
            const uint64_t off = (uint64_t)e * L.gate_expert_bytes + (uint64_t)ui * g.unit_proj;
            bulk_g2s(buf + (u - ua) * g.gu_unit + proj * g.unit_proj, (proj ? L.up : L.gate) + off, bytes,
                     &g.bar[(sbase + s) & 1]);
        }
    };
    if (warp == 0) {
        if (n_st > 0) issue(0);
        if (n_st > 1) issue(1);
        // the down phase's first stage, when gate/up leaves its buffer free, streams in now
        if (early_down) {
            int v0, v1;
            down_range(g, v0, v1);
            issue_down_stage<T>(g, L, v0, v1, 0, sbase + n_st);
        }
    }
    // the next layer's router rows (and bias) stream into L2 behind this phase
    if (next_router && tid == kThreads - 1) {
        for (int e = cta; e < g.NE; e += G) prefetch_l2(next_router + (size_t)e * g.E, (uint32_t)g.E * 4u);
        if (cta == 0 && next_bias && (g.NE & 3) == 0) prefetch_l2(next_bias, (uint32_t)g.NE * 4u);
    }
    const bool active = warp < g.WB * g.RG;
    const int kcol = warp % g.WB, rg = warp / g.WB;
    const uint32_t copy_off = Codebook<kNC>::copy_off(lane);
    float *xw = g.xs + warp * 128;
    uint32_t A[1][8][4];
    int cur_tok = -1;
    auto build_a = [&](int tok) {
        rotated_block_cg(cur, cur_bf16, (size_t)tok * g.E + kcol * 128, g.sel_scale[tok], L.gate_signs, kcol * 128, xw,
                         lane);
        build_a_single(xw, lane, A[0]);
        __syncwarp();
    };
    if (active && n_st > 0) {
        cur_tok = (u0 / g.UPS) / U;
        build_a(cur_tok);
    }
    GX_STACK_MARK_IF(tr, 16);
    #pragma unroll 1
    for (int s = 0; s < n_st; ++s) {
        if (!wait_stage(g.bar, sbase + s, sbase + n_st - 1, a.err)) return false;
        if (s == 0) GX_STACK_MARK_IF(tr, 8);
        const int ua = u0 + s * P, ub = min(ua + P, u1);
        const uint8_t *buf = g.stage + ((sbase + s) & 1) * g.stage_bytes;
        #pragma unroll 1
        for (int u = ua; u < ub; ++u) {
            const int slot = u / g.UPS, ui = u % g.UPS, tok = slot / U;
            if (active && tok != cur_tok) {
                build_a(tok);
                cur_tok = tok;
            }
            const int nt = min(g.RG, g.NT - ui * g.RG);
            if (active && rg < nt) {
                const uint8_t *ubase = buf + (u - ua) * g.gu_unit;
#pragma unroll
                for (int proj = 0; proj < 2; ++proj) {
                    float acc[1][2] = {{0.f, 0.f}};
                    tile_mma<T, 1, kNC>(ubase + proj * g.unit_proj + (rg * g.NB + kcol) * TB, g.cb, copy_off, lane, A,
                                        acc);
                    if (lane < 4) {
                        float *p = g.part + (((u - ua) * 2 + proj) * 16 + rg * g.WB + kcol) * 8 + 2 * lane;
                        p[0] = acc[0][0];
                        p[1] = acc[0][1];
                    }
                }
            }
        }
        __syncthreads();
        if (s == n_st - 1) GX_STACK_MARK_IF(tr, 9);
        if (warp == 0 && s + 2 < n_st) issue(s + 2);
        #pragma unroll 1
        for (int r = tid; r < (ub - ua) * g.RG * 8; r += kThreads) {
            const int j = r / (g.RG * 8), rgi = (r >> 3) % g.RG, n = r & 7;
            const int u = ua + j, slot = u / g.UPS, ui = u % g.UPS;
            if (rgi >= min(g.RG, g.NT - ui * g.RG)) continue;
            float gs = 0.f, up = 0.f;
            #pragma unroll 1
            for (int kc = 0; kc < g.WB; ++kc) {
                gs += g.part[((j * 2 + 0) * 16 + rgi * g.WB + kc) * 8 + n];
                up += g.part[((j * 2 + 1) * 16 + rgi * g.WB + kc) * 8 + n];
            }
            a.act[(size_t)slot * g.F + (ui * g.RG + rgi) * 8 + n] = silu_ref(gs) * up;
        }
        __syncthreads();
    }
    return true;
}

// ---- D: down units of this CTA, weighted sum over the slots, residual ----------------------
template <uint32_t T>
__device__ __forceinline__ bool phase_down(const StackArgs &a, const StackLayer &L, const void *cur, int cur_bf16,
                                        void *dst, int dst_bf16, int P, int sbase, bool early, bool tr) {
    constexpr int TB = tile_bytes(T);
    P = opaque(P);
    const StackGeo g = stack_geo<T>(a, P);
    const int tid = opaque((int)threadIdx.x), lane = tid & 31, warp = tid >> 5;
    const int U = g.U;
    int v0, v1;
    down_range(g, v0, v1);
    const int n_st = (v1 - v0 + P - 1) / P;
    auto issue = [&](int s) { issue_down_stage<T>(g, L, v0, v1, s, sbase + s); };  // warp 0
    if (warp == 0) {
        if (n_st > 0 && !early) issue(0);
        if (n_st > 1) issue(1);
    }
    // residual of this thread's first output row, loaded while the weights stream in
    float resid0 = 0.f;
    if (a.residual && n_st > 0 && tid < (min(v0 + P, v1) - v0) * 8) {
        const int u = v0 + (tid >> 3);
        resid0 = ldcg_act(cur, cur_bf16, (size_t)(u / g.NTD) * g.E + (u % g.NTD) * 8 + (tid & 7));
    }
    const uint32_t copy_off = Codebook<kNC>::copy_off(lane);
    float *xw = g.xs + warp * 128;
    uint32_t A[kKBWD][1][8][4];
    int cur_tok = -1;
    auto build_a = [&](int t) {
#pragma unroll
        for (int j = 0; j < kKBWD; ++j) {
            const int p = warp + kWarps * j;
            if (p < g.NPAIR) {
                const int k = p / g.NBF, b = p % g.NBF;
                rotated_block_cg(a.act, 0, (size_t)(t * U + k) * g.F + b * 128, 1.f, L.down_signs, b * 128, xw, lane);
                build_a_single(xw, lane, A[j][0]);
                __syncwarp();
            }
        }
    };
    if (n_st > 0) {
        cur_tok = v0 / g.NTD;
        build_a(cur_tok);
    }
    GX_STACK_MARK_IF(tr, 15);
    #pragma unroll 1
    for (int s = 0; s < n_st; ++s) {
        if (!wait_stage(g.bar, sbase + s, sbase + n_st - 1, a.err)) return false;
        if (s == 0) GX_STACK_MARK_IF(tr, 10);
        const int ua = v0 + s * P, ub = min(ua + P, v1);
        const uint8_t *buf = g.stage + ((sbase + s) & 1) * g.stage_bytes;
        #pragma unroll 1
        for (int u = ua; u < ub; ++u) {
            const int t = u / g.NTD;
            if (t != cur_tok) {
                build_a(t);
                cur_tok = t;
            }
#pragma unroll
            for (int j = 0; j < kKBWD; ++j) {
                const int p = warp + kWarps * j;
                if (p < g.NPAIR) {
                    const int k = p / g.NBF, b = p % g.NBF;
                    float acc[1][2] = {{0.f, 0.f}};
                    tile_mma<T, 1, kNC>(buf + (u - ua) * g.dn_unit + k * g.slot_bytes + b * TB, g.cb, copy_off, lane,
                                        A[j], acc);
                    if (lane < 4) {
                        float *q = g.part + ((u - ua) * 32 + p) * 8 + 2 * lane;
                        q[0] = acc[0][0];
                        q[1] = acc[0][1];
                    }
                }
            }
        }
        __syncthreads();
        if (s == n_st - 1) GX_STACK_MARK_IF(tr, 11);
        if (warp == 0 && s + 2 < n_st) issue(s + 2);
        #pragma unroll 1
        for (int r = tid; r < (ub - ua) * 8; r += kThreads) {
            const int j = r >> 3, n = r & 7;
            const int u = ua + j, t = u / g.NTD, i = u % g.NTD;
            const int row = i * 8 + n;
            float v = 0.f;
            #pragma unroll 1
            for (int k = 0; k < U; ++k) {
                float dk = 0.f;
                #pragma unroll 1
                for (int b = 0; b < g.NBF; ++b) dk += g.part[(j * 32 + k * g.NBF + b) * 8 + n];
                v += g.sel_w[t * 16 + k] * dk;
            }
            const size_t o = (size_t)t * g.E + row;
            if (a.residual) v = (s == 0 && r == tid ? resid0 : ldcg_act(cur, cur_bf16, o)) + v;
            if (!(fabsf(v) <= 3.4028235e38f)) atomicExch(a.err, KERR_RANGE);   // Inf or NaN
            store_act(dst, dst_bf16, o, v);
        }
        __syncthreads();
    }
    return true;
}

template <uint32_t T>
__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(StackArgs a, int P) {
    {
        const StackGeo g = stack_geo<T>(a, P);
        if (threadIdx.x == 0) {
            mbar_init(&g.bar[0], 1);
            mbar_init(&g.bar[1], 1);
            fence_barrier_init();
        }
        Codebook<kNC>::stage(g.cb, a.codebook, threadIdx.x, kThreads);
    }
    __shared__ StackLayer Ls[2];  // table entries of this layer and the next (loaded one layer ahead)
    if (threadIdx.x == 0) Ls[0] = a.layers[0];
    unsigned n_sync = 0;
    int sbase = 0;  // stages used so far by this CTA (mbarrier phase bookkeeping)
    for (int l = 0; l < a.n_layers; ++l) {
        __syncthreads();
        const StackLayer &L = Ls[l & 1];
        const bool last = l + 1 == a.n_layers;
        const void *cur = l == 0 ? a.x : (const void *)((l & 1) ? a.xa : a.xb);
        const int cur_bf16 = l == 0 ? a.x_bf16 : 0;
        GX_STACK_MARK(l, a.n_layers / 2, 0);
        {
            const StackGeo g = stack_geo<T>(a, P);
            phase_router(a, L.router, cur, cur_bf16, g.sel_scale, g.red);
        }
        if (!last && threadIdx.x == 32) Ls[(l + 1) & 1] = a.layers[l + 1];
        GX_STACK_MARK(l, a.n_layers / 2, 1);
        if (!grid_barrier(a.sync, ++n_sync, a.err)) return;
        GX_STACK_MARK(l, a.n_layers / 2, 2);
        // T: expert selection of the tokens this CTA's gate/up and down units touch
        {
            const StackGeo g = stack_geo<T>(a, P);
            const int n_gu = a.n_tok * a.U * g.UPS, n_dn = a.n_tok * g.NTD;
            const int u0 = (int)((long long)blockIdx.x * n_gu / gridDim.x);
            const int u1 = (int)((long long)(blockIdx.x + 1) * n_gu / gridDim.x);
            const int v0 = (int)((long long)blockIdx.x * n_dn / gridDim.x);
            const int v1 = (int)((long long)(blockIdx.x + 1) * n_dn / gridDim.x);
            int t_lo = a.n_tok, t_hi = -1;
            if (u1 > u0) {
                t_lo = (u0 / g.UPS) / a.U;
                t_hi = ((u1 - 1) / g.UPS) / a.U;
            }
            if (v1 > v0) {
                t_lo = min(t_lo, v0 / g.NTD);
                t_hi = max(t_hi, (v1 - 1) / g.NTD);
            }
            for (int t = t_lo; t <= t_hi; ++t)
                select_token_block(a.logits + (size_t)t * a.NE, L.bias, a.NE, a.U, g.sel_scale[t], L.scale,
                                   g.sel_ids + t * 16, g.sel_w + t * 16, g.tred,
                                   reinterpret_cast<unsigned long long *>(g.red), l == a.n_layers / 2);
        }
        GX_STACK_MARK(l, a.n_layers / 2, 3);
        bool early_down;
        {
            const StackGeo g = stack_geo<T>(a, P);
            const int n_gu = a.n_tok * a.U * g.UPS;
            const int gu_st = ((int)((long long)(blockIdx.x + 1) * n_gu / gridDim.x) -
                               (int)((long long)blockIdx.x * n_gu / gridDim.x) + P - 1) / P;
            int v0, v1;
            down_range(g, v0, v1);
            early_down = gu_st <= 1 && v1 > v0;
        }
        if (!phase_gate_up<T>(a, L, cur, cur_bf16, P, sbase, last ? nullptr : Ls[(l + 1) & 1].router,
                              last ? nullptr : Ls[(l + 1) & 1].bias, early_down, l == a.n_layers / 2))
            return;
        {
            const int n_gu = a.n_tok * a.U * stack_geo<T>(a, P).UPS;
            sbase += ((int)((long long)(blockIdx.x + 1) * n_gu / gridDim.x) -
                      (int)((long long)blockIdx.x * n_gu / gridDim.x) + P - 1) / P;
        }
        GX_STACK_MARK(l, a.n_layers / 2, 4);
        if (!grid_barrier(a.sync, ++n_sync, a.err)) return;
        GX_STACK_MARK(l, a.n_layers / 2, 5);
        if (!phase_down<T>(a, L, cur, cur_bf16, last ? a.out : (void *)((l & 1) ? a.xb : a.xa), last ? a.out_bf16 : 0, P,
                           sbase, early_down, l == a.n_layers / 2))
            return;
        {
            const int n_dn = a.n_tok * (a.E >> 3);
            sbase += ((int)((long long)(blockIdx.x + 1) * n_dn / gridDim.x) -
                      (int)((long long)blockIdx.x * n_dn / gridDim.x) + P - 1) / P;
        }
        GX_STACK_MARK(l, a.n_layers / 2, 6);
        if (!last && !grid_barrier(a.sync, ++n_sync, a.err)) return;
        GX_STACK_MARK(l, a.n_layers / 2, 7);
    }
}

namespace {

template <uint32_t T>
cudaError_t stack_t(const StackArgs &a, int sm_count, int P, int smem, cudaStream_t s) {
    static const cudaError_t once =
        cudaFuncSetAttribute(decode_stack_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (once != cudaSuccess) return once;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_stack_kernel<T>, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    e = cudaMemsetAsync(a.sync, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)sm_count);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_stack_kernel<T>, a, P);
}

}  // namespace

// Shared memory of the stack kernel for P units per stage (0 if it does not fit).
int decode_stack_smem(uint32_t type, int E, int F, int U, int P) {
    const int TB = tile_bytes(type);
    const int NB = E >> 7, WB = NB < 16 ? NB : 16, RG = 16 / WB;
    const int gu = 2 * RG * NB * TB, dn = U * (F >> 7) * TB;
    const int unit = gu > dn ? gu : dn;
    const int stage = ((P * unit + 127) / 128) * 128;
    const int bytes = Codebook<kNC>::BYTES + 2 * stage + P * 32 * 8 * 4 + kWarps * 128 * 4 + kWarps * 80 * 4 +
                      256 * 4 * 2 + 16 * 4 + 32 * 4 + 2 * 8;
    return bytes <= kSmemBudget ? bytes : 0;
}

bool decode_stack_supported(uint32_t type, int E, int F, int U, int NE, int n_tok) {
    if (!type_k(type) || n_tok < 1 || n_tok > 16 || E % 128 || F % 128 || E > 2048 || NE > 512 || U > 16)
        return false;
    if (U * (F / 128) > kWarps * kKBWD) return false;
    if (16 % ((E / 128) < 16 ? (E / 128) : 16)) return false;  // warps split evenly over column blocks
    return decode_stack_smem(type, E, F, U, 1) > 0;
}

cudaError_t launch_decode_stack(const StackArgs &a, uint32_t type, int sm_count, cudaStream_t s) {
    if (!decode_stack_supported(type, a.E, a.F, a.U, a.NE, a.n_tok)) return cudaErrorInvalidValue;
    if (a.NE > 4 * sm_count) return cudaErrorInvalidValue;  // at most 4 router rows per CTA
    int P = 8;
    while (P > 1 && decode_stack_smem(type, a.E, a.F, a.U, P) == 0) --P;
    const int smem = decode_stack_smem(type, a.E, a.F, a.U, P);
    switch (type) {
        case 144: return stack_t<144>(a, sm_count, P, smem, s);
        case 145: return stack_t<145>(a, sm_count, P, smem, s);
        case 146: return stack_t<146>(a, sm_count, P, smem, s);
        case 147: return stack_t<147>(a, sm_count, P, smem, s);
        case 148: return stack_t<148>(a, sm_count, P, smem, s);
        case 149: return stack_t<149>(a, sm_count, P, smem, s);
        case 150: return stack_t<150>(a, sm_count, P, smem, s);
        case 151: return stack_t<151>(a, sm_count, P, smem, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gx

#ifdef GX_TRACE
extern "C" __attribute__((visibility("default"))) int gx_stack_trace_read(long long *out, int clear) {
    if (cudaMemcpyFromSymbol(out, gx::gx_stack_trace, sizeof(gx::gx_stack_trace)) != cudaSuccess) return -1;
    if (clear) {
        static long long zeros[160][20] = {};
        if (cudaMemcpyToSymbol(gx::gx_stack_trace, zeros, sizeof(zeros)) != cudaSuccess) return -1;
    }
    return 0;
}
#endif
