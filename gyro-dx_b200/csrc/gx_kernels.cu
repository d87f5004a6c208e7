// gx_kernels.cu — sm_100a kernels of the routed-MoE decode path.
//
//   router_kernel      logits = W_r x (+ bias), then softmax / top-k / renormalisation in the
//                      last CTA to finish (src/engine.zig:526-540, :671-686;
//                      shaders/engine/mv.hlsl:157-182 + moe.hlsl:20-80)
//   topk_kernel        the same selection, one warp per token, for large token counts
//   gate_up_kernel     per slot: Hadamard-rotated input (src/engine.zig:547-551), fused Gyro
//                      decode + gate and up GEMV, SwiGLU epilogue (:567-606;
//                      moe.hlsl:108-211 proj 0/1 + moe_act:222-254 first half)
//   down_kernel        per token: down-input signs + FWHT prologue (:606), fused decode + down
//                      GEMV for all U slots, weighted combine (+ residual) epilogue
//                      (:608-641; moe.hlsl proj 2 + moe_combine:292-305)
//   matvec_kernel      standalone decode GEMV of one matrix for up to 16 tokens
//   decode_blocks_kernel  strict per-weight decode, bit-exact conformance (gyro_decode.hlsl)
//   repack_kernel      reference block layout -> HBM tile layout (gx_tile.h)
//
// The decode GEMVs keep the packed weights in the tile layout of gx_tile.h: a CTA streams its
// tiles into shared memory with 1-D bulk async copies (TMA engine, mbarrier completion, no
// multicast), keeps 16 bank-interleaved copies of the 8 KB codebook in shared memory, and
// feeds the looked-up fp16 codebook pairs straight into mma.sync B fragments. Activations enter
// the A fragments as fp16 hi + lo halves (rows 0-7 hi, rows 8-15 lo), so the products carry
// about 22 bits of the fp32 activation while the weights are exact.
#include <cuda_runtime.h>
#include <math.h>

#include "gx_device.cuh"
#include "gx_internal.h"

namespace gx {

using CB = Codebook<kCodebookCopies>;

// One 8-row x 128-column tile against NG groups of 8 tokens. acc[g][0..1] accumulates, for
// token (8g + lane/4), rows 2*(lane%4) and 2*(lane%4)+1 of the tile (scaled by d).
template <uint32_t T, int NG>
__device__ __forceinline__ void tile_mma(const uint8_t *tile, const uint32_t *cb, uint32_t copy_off, int lane,
                                         const uint32_t (&A)[NG][8][4], float (&acc)[NG][2]) {
    uint32_t own[4];
    load_run<T>(tile, lane, own);
    const int nbr = (lane & ~3) | ((lane + 3) & 3);
    const uint32_t nv = __shfl_sync(0xffffffffu, (T == T_TQ2_T) ? own[1] : own[0], nbr);
    const uint32_t nb = (T == T_TQ2_T) ? (nv >> 24) : (nv & 0xffffu);
    uint32_t i0[8], i1[8];
    quarter_indices<T>(own, nb, i0, i1);
    uint32_t b0[8], b1[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        b0[c] = cb[CB::word(i0[c], copy_off)];
        b1[c] = cb[CB::word(i1[c], copy_off)];
    }
    float d[NG][4];
#pragma unroll
    for (int g = 0; g < NG; ++g) d[g][0] = d[g][1] = d[g][2] = d[g][3] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int g = 0; g < NG; ++g) mma16816(d[g], A[g][c], b0[c], b1[c]);
    const uint32_t sc = *reinterpret_cast<const uint32_t *>(tile + tile_code_bytes(T) + 4 * (lane & 3));
    const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&sc));
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        acc[g][0] += s.x * (d[g][0] + d[g][2]);
        acc[g][1] += s.y * (d[g][1] + d[g][3]);
    }
}

// A fragments of one token for one 128-column block from 128 fp32 values in shared memory
// (xs[0..127]); lanes 0-3 carry the token (row 0 hi, row 8 lo), the other lanes zeros.
__device__ __forceinline__ void build_a_single(const float *xs, int lane, uint32_t (&A)[8][4]) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        if (lane < 4) {
            const float *p = xs + 32 * lane + 4 * c;
            float h0, l0, h1, l1, h2, l2, h3, l3;
            split_hilo(p[0], h0, l0);
            split_hilo(p[1], h1, l1);
            split_hilo(p[2], h2, l2);
            split_hilo(p[3], h3, l3);
            A[c][0] = pack_half2(h0, h1);
            A[c][1] = pack_half2(l0, l1);
            A[c][2] = pack_half2(h2, h3);
            A[c][3] = pack_half2(l2, l3);
        } else {
            A[c][0] = A[c][1] = A[c][2] = A[c][3] = 0u;
        }
    }
}

// Rotated block of one activation row into xs (per-warp scratch of 128 floats):
// xs = H128(signs * v) / sqrt(128) for v = src[base .. base+128).
__device__ __forceinline__ void rotated_block_to_smem(const void *src, int bf16, size_t base, const float *signs,
                                                      int sbase, float *xs, int lane) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = load_act(src, bf16, base + 4 * lane + j);
        if (signs) v[j] *= signs[sbase + 4 * lane + j];
    }
    if (signs) fwht128_warp(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) xs[4 * lane + j] = v[j];
    __syncwarp();
}

// ------------------------------------------------------------------------------------------
// Router: one warp per expert row; the last CTA to finish runs the per-token selection.
// ------------------------------------------------------------------------------------------
__device__ void topk_token(const float *row, int NE, int U, float scale, uint32_t *ids, float *weights, int lane) {
    float v[16];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < NE ? __ldcg(row + i) : -INFINITY;
        m = fmaxf(m, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < NE ? expf(v[j] - m) : 0.f;
        s += v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (lane + 32 * j) < NE ? v[j] / s : -1.f;
    float wk[16];
    uint32_t ik[16];
    for (int k = 0; k < U; ++k) {
        float bv = -2.f;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (v[j] > bv) { bv = v[j]; bi = (uint32_t)(lane + 32 * j); }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if ((uint32_t)(lane + 32 * j) == bi) v[j] = -1.f;
        wk[k & 15] = bv;
        ik[k & 15] = bi;
    }
    if (lane == 0) {
        float total = 0.f;
        for (int k = 0; k < U; ++k) total += wk[k];
        total = fmaxf(total, 6.103515625e-5f);
        for (int k = 0; k < U; ++k) {
            float w = wk[k] / total;
            if (scale != 0.f && scale != 1.f) w *= scale;
            ids[k] = ik[k];
            weights[k] = w;
        }
    }
}

__global__ void __launch_bounds__(64) router_kernel(RouterArgs a, int fused_topk) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    const int r = blockIdx.x * wpb + warp;
    if (r < a.NE) {
        const float *w = a.W + (size_t)r * a.E;
        const float bias = a.bias ? a.bias[r] : 0.f;
        for (int cbase = 0; cbase < a.E; cbase += 2048) {
            float4 wv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int c = cbase + 128 * j + 4 * lane;
                wv[j] = c < a.E ? __ldg(reinterpret_cast<const float4 *>(w + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            for (int t0 = 0; t0 < a.n_tok; t0 += 8) {
                float acc[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int c = cbase + 128 * j + 4 * lane;
                    if (c >= a.E) break;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        if (t0 + t < a.n_tok) {
                            const size_t base = (size_t)(t0 + t) * a.E + c;
                            float x0, x1, x2, x3;
                            if (a.x_bf16) {
                                const __nv_bfloat162 *p = reinterpret_cast<const __nv_bfloat162 *>(
                                    reinterpret_cast<const __nv_bfloat16 *>(a.x) + base);
                                const float2 u0 = __bfloat1622float2(p[0]), u1 = __bfloat1622float2(p[1]);
                                x0 = u0.x; x1 = u0.y; x2 = u1.x; x3 = u1.y;
                            } else {
                                const float4 xv = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + base);
                                x0 = xv.x; x1 = xv.y; x2 = xv.z; x3 = xv.w;
                            }
                            acc[t] = fmaf(wv[j].x, x0, acc[t]);
                            acc[t] = fmaf(wv[j].y, x1, acc[t]);
                            acc[t] = fmaf(wv[j].z, x2, acc[t]);
                            acc[t] = fmaf(wv[j].w, x3, acc[t]);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < 8; ++t) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
                }
                if (lane == 0) {
                    for (int t = 0; t < 8 && t0 + t < a.n_tok; ++t) {
                        float *dst = a.logits + (size_t)(t0 + t) * a.NE + r;
                        // Columns beyond the first 2048 accumulate onto the stored partial.
                        *dst = (cbase == 0 ? bias : *dst) + acc[t];
                    }
                }
            }
        }
    }
    if (!fused_topk) return;
    __shared__ int is_last;
    __threadfence();  // every logits writer publishes before the CTA takes its ticket
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.counter, 1u);
        is_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int t = warp; t < a.n_tok; t += wpb)
        topk_token(a.logits + (size_t)t * a.NE, a.NE, a.U, a.scale, a.ids + (size_t)t * a.U,
                   a.weights + (size_t)t * a.U, lane);
    if (threadIdx.x == 0) *a.counter = 0u;
}

__global__ void __launch_bounds__(256) topk_kernel(RouterArgs a) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.n_tok) return;
    topk_token(a.logits + (size_t)t * a.NE, a.NE, a.U, a.scale, a.ids + (size_t)t * a.U,
               a.weights + (size_t)t * a.U, lane);
}

// ------------------------------------------------------------------------------------------
// Shared shape of the streamed decode GEMVs: a CTA owns a contiguous range of work units,
// fetches P units per stage with bulk copies into one of two stage buffers, and reduces the
// per-warp partial sums of a stage in shared memory.
// ------------------------------------------------------------------------------------------
struct StageCtl {
    uint64_t *bar;
    int u0, u1, P, n_stages;
};

// Waits for stage s. On an expired wait every thread of the CTA sees false; before the CTA
// returns, the copies still in flight into its shared memory get one more bounded wait.
__device__ __forceinline__ bool stage_wait(const StageCtl &c, int s, int *err) {
    bool ok = mbar_wait(&c.bar[s & 1], (uint32_t)((s >> 1) & 1), err);
    if (__syncthreads_and(ok)) return true;
    if (threadIdx.x == 0) {
        for (int t = s; t < s + 2 && t < c.n_stages; ++t) mbar_wait(&c.bar[t & 1], (uint32_t)((t >> 1) & 1), nullptr);
    }
    __syncthreads();
    return false;
}

// ---- gate/up: unit = (slot, RG row-groups of both projections) ---------------------------
template <uint32_t T, int KBW>
__global__ void __launch_bounds__(512, 1) gate_up_kernel(GateUpArgs a, int P) {
    constexpr int TB = tile_bytes(T);
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NB = a.E >> 7;
    const int WB = NB < 16 ? NB : 16;
    const int RG = 16 / WB;
    const int NT = a.F >> 3;
    const int UPS = (NT + RG - 1) / RG;
    const int unit_proj = RG * NB * TB;
    const int stage_bytes = P * 2 * unit_proj;

    uint32_t *cb = reinterpret_cast<uint32_t *>(smem);
    uint8_t *stage = smem + CB::BYTES;
    float *part = reinterpret_cast<float *>(stage + 2 * stage_bytes);  // [P][2][16][8]
    float *xs = part + P * 2 * 16 * 8;                                  // [16][128]
    uint64_t *bar = reinterpret_cast<uint64_t *>(xs + 16 * 128);

    const int n_units = a.n_slots * UPS;
    StageCtl ctl;
    ctl.bar = bar;
    ctl.P = P;
    ctl.u0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
    ctl.u1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
    ctl.n_stages = (ctl.u1 - ctl.u0 + P - 1) / P;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();

    auto issue = [&](int s) {
        uint8_t *buf = stage + (s & 1) * stage_bytes;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        uint32_t total = 0;
        for (int u = ua; u < ub; ++u) {
            const int ui = u % UPS;
            total += 2u * (uint32_t)(min(RG, NT - ui * RG) * NB * TB);
        }
        mbar_expect_tx(&bar[s & 1], total);
        for (int u = ua; u < ub; ++u) {
            const int slot = u / UPS, ui = u % UPS;
            const uint32_t bytes = (uint32_t)(min(RG, NT - ui * RG) * NB * TB);
            uint32_t e = a.ids[slot];
            if (e >= (uint32_t)a.n_expert) {
                atomicExch(a.err, KERR_BOUNDS);
                e = 0;
            }
            const uint64_t off = (uint64_t)e * a.expert_bytes + (uint64_t)ui * unit_proj;
            uint8_t *dst = buf + (u - ua) * 2 * unit_proj;
            bulk_g2s(dst, a.gate + off, bytes, &bar[s & 1]);
            bulk_g2s(dst + unit_proj, a.up + off, bytes, &bar[s & 1]);
        }
    };
    if (tid == 0) {
        if (ctl.n_stages > 0) issue(0);
        if (ctl.n_stages > 1) issue(1);
    }
    CB::stage(cb, a.codebook, tid, blockDim.x);
    __syncthreads();

    const bool active = warp < WB * RG;
    const int kcol = warp % WB, rg = warp / WB;
    const uint32_t copy_off = CB::copy_off(lane);
    uint32_t A[KBW][1][8][4];
    int cur_tok = -1;
    float *xw = xs + warp * 128;

    for (int s = 0; s < ctl.n_stages; ++s) {
        if (!stage_wait(ctl, s, a.err)) return;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        const uint8_t *buf = stage + (s & 1) * stage_bytes;
        for (int u = ua; u < ub; ++u) {
            const int slot = u / UPS, ui = u % UPS;
            const int tok = slot / a.U;
            if (active && tok != cur_tok) {
#pragma unroll
                for (int j = 0; j < KBW; ++j) {
                    const int b = kcol + WB * j;
                    if (b < NB) {
                        rotated_block_to_smem(a.x, a.x_bf16, (size_t)tok * a.E + b * 128, a.signs, b * 128, xw, lane);
                        build_a_single(xw, lane, A[j][0]);
                        __syncwarp();
                    }
                }
                cur_tok = tok;
            }
            const int nt = min(RG, NT - ui * RG);
            if (active && rg < nt) {
                const uint8_t *ubase = buf + (u - ua) * 2 * unit_proj;
#pragma unroll
                for (int proj = 0; proj < 2; ++proj) {
                    float acc[1][2] = {{0.f, 0.f}};
#pragma unroll
                    for (int j = 0; j < KBW; ++j) {
                        const int b = kcol + WB * j;
                        if (b < NB)
                            tile_mma<T, 1>(ubase + proj * unit_proj + (rg * NB + b) * TB, cb, copy_off, lane, A[j], acc);
                    }
                    if (lane < 4) {
                        float *p = part + (((u - ua) * 2 + proj) * 16 + rg * WB + kcol) * 8 + 2 * lane;
                        p[0] = acc[0][0];
                        p[1] = acc[0][1];
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && s + 2 < ctl.n_stages) issue(s + 2);
        for (int r = tid; r < (ub - ua) * RG * 8; r += blockDim.x) {
            const int j = r / (RG * 8), rgi = (r >> 3) % RG, n = r & 7;
            const int u = ua + j, slot = u / UPS, ui = u % UPS;
            if (rgi >= min(RG, NT - ui * RG)) continue;
            float g = 0.f, up = 0.f;
            for (int kc = 0; kc < WB; ++kc) {
                g += part[((j * 2 + 0) * 16 + rgi * WB + kc) * 8 + n];
                up += part[((j * 2 + 1) * 16 + rgi * WB + kc) * 8 + n];
            }
            a.act[(size_t)slot * a.F + (ui * RG + rgi) * 8 + n] = silu_ref(g) * up;
        }
        __syncthreads();
    }
}

// ---- down: unit = (token, one row group); warps own (slot, block) pairs -------------------
template <uint32_t T, int KBW>
__global__ void __launch_bounds__(512, 1) down_kernel(DownArgs a, int P) {
    constexpr int TB = tile_bytes(T);
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NBF = a.F >> 7;
    const int NPAIR = a.U * NBF;
    const int NT = a.E >> 3;
    const int slot_bytes = NBF * TB;
    const int unit_bytes = a.U * slot_bytes;
    const int stage_bytes = P * unit_bytes;
    constexpr int PMAX = 16 * KBW;

    uint32_t *cb = reinterpret_cast<uint32_t *>(smem);
    uint8_t *stage = smem + CB::BYTES;
    float *part = reinterpret_cast<float *>(stage + 2 * stage_bytes);  // [P][PMAX][8]
    float *xs = part + P * PMAX * 8;                                    // [16][128]
    uint64_t *bar = reinterpret_cast<uint64_t *>(xs + 16 * 128);

    const int n_units = a.n_tok * NT;
    StageCtl ctl;
    ctl.bar = bar;
    ctl.P = P;
    ctl.u0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
    ctl.u1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
    ctl.n_stages = (ctl.u1 - ctl.u0 + P - 1) / P;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();

    auto issue = [&](int s) {
        uint8_t *buf = stage + (s & 1) * stage_bytes;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        mbar_expect_tx(&bar[s & 1], (uint32_t)((ub - ua) * unit_bytes));
        for (int u = ua; u < ub; ++u) {
            const int t = u / NT, i = u % NT;
            for (int k = 0; k < a.U; ++k) {
                uint32_t e = a.ids[t * a.U + k];
                if (e >= (uint32_t)a.n_expert) {
                    atomicExch(a.err, KERR_BOUNDS);
                    e = 0;
                }
                bulk_g2s(buf + (u - ua) * unit_bytes + k * slot_bytes,
                         a.down + (uint64_t)e * a.expert_bytes + (uint64_t)i * slot_bytes, (uint32_t)slot_bytes,
                         &bar[s & 1]);
            }
        }
    };
    if (tid == 0) {
        if (ctl.n_stages > 0) issue(0);
        if (ctl.n_stages > 1) issue(1);
    }
    CB::stage(cb, a.codebook, tid, blockDim.x);
    __syncthreads();

    const uint32_t copy_off = CB::copy_off(lane);
    uint32_t A[KBW][1][8][4];
    int cur_tok = -1;
    float *xw = xs + warp * 128;

    for (int s = 0; s < ctl.n_stages; ++s) {
        if (!stage_wait(ctl, s, a.err)) return;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        const uint8_t *buf = stage + (s & 1) * stage_bytes;
        for (int u = ua; u < ub; ++u) {
            const int t = u / NT;
            if (t != cur_tok) {
#pragma unroll
                for (int j = 0; j < KBW; ++j) {
                    const int p = warp + 16 * j;
                    if (p < NPAIR) {
                        const int k = p / NBF, b = p % NBF;
                        rotated_block_to_smem(a.act, 0, (size_t)(t * a.U + k) * a.F + b * 128, a.signs, b * 128, xw,
                                              lane);
                        build_a_single(xw, lane, A[j][0]);
                        __syncwarp();
                    }
                }
                cur_tok = t;
            }
#pragma unroll
            for (int j = 0; j < KBW; ++j) {
                const int p = warp + 16 * j;
                if (p < NPAIR) {
                    const int k = p / NBF, b = p % NBF;
                    float acc[1][2] = {{0.f, 0.f}};
                    tile_mma<T, 1>(buf + (u - ua) * unit_bytes + k * slot_bytes + b * TB, cb, copy_off, lane, A[j],
                                   acc);
                    if (lane < 4) {
                        float *q = part + ((u - ua) * PMAX + p) * 8 + 2 * lane;
                        q[0] = acc[0][0];
                        q[1] = acc[0][1];
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && s + 2 < ctl.n_stages) issue(s + 2);
        for (int r = tid; r < (ub - ua) * 8; r += blockDim.x) {
            const int j = r >> 3, n = r & 7;
            const int u = ua + j, t = u / NT, i = u % NT;
            const int row = i * 8 + n;
            float v = 0.f;
            for (int k = 0; k < a.U; ++k) {
                float dk = 0.f;
                for (int b = 0; b < NBF; ++b) dk += part[(j * PMAX + k * NBF + b) * 8 + n];
                v += a.weights[t * a.U + k] * dk;
            }
            const size_t o = (size_t)t * a.E + row;
            if (a.resid) v = load_act(a.resid, a.resid_bf16, o) + v;
            if (a.out_bf16)
                reinterpret_cast<__nv_bfloat16 *>(a.out)[o] = __float2bfloat16_rn(v);
            else
                reinterpret_cast<float *>(a.out)[o] = v;
        }
        __syncthreads();
    }
}

// ---- standalone matvec: unit = RG row groups; up to 16 tokens (2 groups of 8) -----------
template <uint32_t T, int KBW, int NG>
__global__ void __launch_bounds__(512, 1) matvec_kernel(MatvecArgs a, int t0, int P) {
    constexpr int TB = tile_bytes(T);
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NB = a.cols >> 7;
    const int WB = NB < 16 ? NB : 16;
    const int RG = 16 / WB;
    const int NT = a.rows >> 3;
    const int n_units = (NT + RG - 1) / RG;
    const int unit_bytes = RG * NB * TB;
    const int stage_bytes = P * unit_bytes;
    const int ntok = min(16, a.n_tok - t0);

    uint32_t *cb = reinterpret_cast<uint32_t *>(smem);
    uint8_t *stage = smem + CB::BYTES;
    float *part = reinterpret_cast<float *>(stage + 2 * stage_bytes);  // [P][16 warps][16 tok][8]
    uint64_t *bar = reinterpret_cast<uint64_t *>(part + P * 16 * 16 * 8);

    StageCtl ctl;
    ctl.bar = bar;
    ctl.P = P;
    ctl.u0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
    ctl.u1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
    ctl.n_stages = (ctl.u1 - ctl.u0 + P - 1) / P;
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int s) {
        uint8_t *buf = stage + (s & 1) * stage_bytes;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        uint32_t total = 0;
        for (int u = ua; u < ub; ++u) total += (uint32_t)(min(RG, NT - u * RG) * NB * TB);
        mbar_expect_tx(&bar[s & 1], total);
        for (int u = ua; u < ub; ++u)
            bulk_g2s(buf + (u - ua) * unit_bytes, a.tiles + (uint64_t)u * unit_bytes,
                     (uint32_t)(min(RG, NT - u * RG) * NB * TB), &bar[s & 1]);
    };
    if (tid == 0) {
        if (ctl.n_stages > 0) issue(0);
        if (ctl.n_stages > 1) issue(1);
    }
    CB::stage(cb, a.codebook, tid, blockDim.x);

    const bool active = warp < WB * RG;
    const int kcol = warp % WB, rg = warp / WB;
    const uint32_t copy_off = CB::copy_off(lane);
    // A fragments straight from global x: lane (g, q) holds token 8*grp + g.
    uint32_t A[KBW][NG][8][4];
#pragma unroll
    for (int j = 0; j < KBW; ++j)
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
            const int b = kcol + WB * j;
            const int tok = 8 * grp + (lane >> 2), q = lane & 3;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (active && b < NB && tok < ntok) {
                    const float4 xv = *reinterpret_cast<const float4 *>(a.x + (size_t)(t0 + tok) * a.cols + b * 128 +
                                                                        32 * q + 4 * c);
                    float h0, l0, h1, l1, h2, l2, h3, l3;
                    split_hilo(xv.x, h0, l0);
                    split_hilo(xv.y, h1, l1);
                    split_hilo(xv.z, h2, l2);
                    split_hilo(xv.w, h3, l3);
                    A[j][grp][c][0] = pack_half2(h0, h1);
                    A[j][grp][c][1] = pack_half2(l0, l1);
                    A[j][grp][c][2] = pack_half2(h2, h3);
                    A[j][grp][c][3] = pack_half2(l2, l3);
                } else {
                    A[j][grp][c][0] = A[j][grp][c][1] = A[j][grp][c][2] = A[j][grp][c][3] = 0u;
                }
            }
        }
    __syncthreads();

    for (int s = 0; s < ctl.n_stages; ++s) {
        if (!stage_wait(ctl, s, a.err)) return;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        const uint8_t *buf = stage + (s & 1) * stage_bytes;
        for (int u = ua; u < ub; ++u) {
            const int nt = min(RG, NT - u * RG);
            if (active && rg < nt) {
                float acc[NG][2];
#pragma unroll
                for (int grp = 0; grp < NG; ++grp) acc[grp][0] = acc[grp][1] = 0.f;
#pragma unroll
                for (int j = 0; j < KBW; ++j) {
                    const int b = kcol + WB * j;
                    if (b < NB) tile_mma<T, NG>(buf + (u - ua) * unit_bytes + (rg * NB + b) * TB, cb, copy_off, lane, A[j], acc);
                }
#pragma unroll
                for (int grp = 0; grp < NG; ++grp) {
                    float *p = part + (((u - ua) * 16 + warp) * 16 + 8 * grp + (lane >> 2)) * 8 + 2 * (lane & 3);
                    p[0] = acc[grp][0];
                    p[1] = acc[grp][1];
                }
            }
        }
        __syncthreads();
        if (tid == 0 && s + 2 < ctl.n_stages) issue(s + 2);
        for (int r = tid; r < (ub - ua) * RG * 16 * 8; r += blockDim.x) {
            const int j = r / (RG * 128), rgi = (r / 128) % RG, tok = (r >> 3) & 15, n = r & 7;
            const int u = ua + j;
            if (rgi >= min(RG, NT - u * RG) || tok >= ntok) continue;
            float v = 0.f;
            for (int kc = 0; kc < WB; ++kc) v += part[(((j * 16) + rgi * WB + kc) * 16 + tok) * 8 + n];
            a.y[(size_t)(t0 + tok) * a.rows + (u * RG + rgi) * 8 + n] = v;
        }
        __syncthreads();
    }
}

// ---- strict decode (conformance): one thread per (block, step) --------------------------
__global__ void decode_blocks_kernel(uint32_t type, const uint8_t *__restrict__ packed, uint32_t nblocks,
                                     const uint16_t *__restrict__ cbh, float *__restrict__ out) {
    const int S = type_steps(type), K = type_k(type), BB = type_block_bytes(type), Q = BB - 2;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (K == 0 || gid >= (uint64_t)nblocks * S) return;
    const uint32_t blk = (uint32_t)(gid / S), t = (uint32_t)(gid % S);
    const uint8_t *b = packed + (size_t)blk * BB;
    const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
    const uint8_t *qs = b + 2;
    uint32_t state;
    if (type == T_TQ2_T) {
        state = ((uint32_t)qs[(t + 31) & 31] << 8) | qs[t];
    } else {
        const uint32_t off = (uint32_t)(S - 1 - (int)t) * (uint32_t)K, byte = off >> 3;
        const uint32_t w = (uint32_t)qs[byte] | ((uint32_t)qs[(byte + 1) % Q] << 8) | ((uint32_t)qs[(byte + 2) % Q] << 16);
        state = (w >> (off & 7)) & 0xffffu;
    }
    const uint32_t h = hash_state(state);
    float *o = out + (size_t)blk * 128 + t * (S == 32 ? 4 : 2);
    const uint32_t i0 = h >> 21;
    o[0] = __fmul_rn(d, __half2float(__ushort_as_half(cbh[2 * i0])));
    o[1] = __fmul_rn(d, __half2float(__ushort_as_half(cbh[2 * i0 + 1])));
    if (S == 32) {
        const uint32_t i1 = (h >> 10) & 2047u;
        o[2] = __fmul_rn(d, __half2float(__ushort_as_half(cbh[2 * i1])));
        o[3] = __fmul_rn(d, __half2float(__ushort_as_half(cbh[2 * i1 + 1])));
    }
}

__global__ void repack_kernel(uint32_t type, const uint8_t *__restrict__ raw, uint64_t row_bytes, uint32_t rows,
                              uint32_t nb, uint8_t *__restrict__ tiles) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t n_tiles = (uint64_t)(rows / 8) * nb;
    if (gid >= n_tiles * 32) return;
    const int lane = (int)(gid & 31);
    const uint64_t tile = gid >> 5;
    const uint64_t i = tile / nb, b = tile % nb;
    const uint8_t *block = raw + (i * 8 + (lane >> 2)) * row_bytes + b * (uint64_t)type_block_bytes(type);
    repack_lane(type, block, tiles + tile * (uint64_t)tile_bytes(type), lane);
}

__global__ void residual_copy_kernel(const void *x, int x_bf16, float *out, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = load_act(x, x_bf16, i);
}

// ------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------
namespace {

constexpr int kSmemLimit = 227 * 1024;

// Raises a kernel's dynamic shared-memory limit once (never inside a stream capture: the
// first launch of every instantiation happens in an eager call).
template <typename K>
cudaError_t set_smem(K kernel, int) {
    static cudaError_t once = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    return once;
}

template <uint32_t T, int KBW>
cudaError_t gate_up_t(const GateUpArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.E / 128, WB = NB < 16 ? NB : 16, RG = 16 / WB;
    const int unit_proj = RG * NB * tile_bytes(T);
    const int fixed = CB::BYTES + 16 * 128 * 4 + 64;
    int P = 4;
    while (P > 1 && fixed + 2 * P * 2 * unit_proj + P * 2 * 16 * 8 * 4 > kSmemLimit) --P;
    const int smem = fixed + 2 * P * 2 * unit_proj + P * 2 * 16 * 8 * 4;
    if (smem > kSmemLimit) return cudaErrorInvalidValue;
    const int NT = a.F / 8, UPS = (NT + RG - 1) / RG;
    const int n_units = a.n_slots * UPS;
    if (n_units == 0) return cudaSuccess;
    const int grid = n_units < sm_count ? n_units : sm_count;
    auto k = gate_up_kernel<T, KBW>;
    cudaError_t e = set_smem(k, smem);
    if (e != cudaSuccess) return e;
    k<<<grid, 512, smem, s>>>(a, P);
    return cudaGetLastError();
}

template <uint32_t T, int KBW>
cudaError_t down_t(const DownArgs &a, int sm_count, cudaStream_t s) {
    const int NBF = a.F / 128;
    const int unit_bytes = a.U * NBF * tile_bytes(T);
    const int PMAX = 16 * KBW;
    const int fixed = CB::BYTES + 16 * 128 * 4 + 64;
    int P = 4;
    while (P > 1 && fixed + 2 * P * unit_bytes + P * PMAX * 8 * 4 > kSmemLimit) --P;
    const int smem = fixed + 2 * P * unit_bytes + P * PMAX * 8 * 4;
    if (smem > kSmemLimit) return cudaErrorInvalidValue;
    const int n_units = a.n_tok * (a.E / 8);
    if (n_units == 0) return cudaSuccess;
    const int grid = n_units < sm_count ? n_units : sm_count;
    auto k = down_kernel<T, KBW>;
    cudaError_t e = set_smem(k, smem);
    if (e != cudaSuccess) return e;
    k<<<grid, 512, smem, s>>>(a, P);
    return cudaGetLastError();
}

template <uint32_t T, int KBW, int NG>
cudaError_t matvec_t(const MatvecArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.cols / 128, WB = NB < 16 ? NB : 16, RG = 16 / WB;
    const int unit_bytes = RG * NB * tile_bytes(T);
    const int fixed = CB::BYTES + 64;
    int P = 4;
    while (P > 1 && fixed + 2 * P * unit_bytes + P * 16 * 16 * 8 * 4 > kSmemLimit) --P;
    const int smem = fixed + 2 * P * unit_bytes + P * 16 * 16 * 8 * 4;
    if (smem > kSmemLimit) return cudaErrorInvalidValue;
    const int NT = a.rows / 8, n_units = (NT + RG - 1) / RG;
    const int grid = n_units < sm_count ? n_units : sm_count;
    auto k = matvec_kernel<T, KBW, NG>;
    cudaError_t e = set_smem(k, smem);
    if (e != cudaSuccess) return e;
    for (int t0 = 0; t0 < a.n_tok; t0 += 16) {
        k<<<grid, 512, smem, s>>>(a, t0, P);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

#define GX_TYPE_SWITCH(type, CALL)                 \
    switch (type) {                                \
        case 144: { constexpr uint32_t T = 144; CALL; } \
        case 145: { constexpr uint32_t T = 145; CALL; } \
        case 146: { constexpr uint32_t T = 146; CALL; } \
        case 147: { constexpr uint32_t T = 147; CALL; } \
        case 148: { constexpr uint32_t T = 148; CALL; } \
        case 149: { constexpr uint32_t T = 149; CALL; } \
        case 150: { constexpr uint32_t T = 150; CALL; } \
        case 151: { constexpr uint32_t T = 151; CALL; } \
        default: return cudaErrorInvalidValue;     \
    }

}  // namespace

cudaError_t launch_router(const RouterArgs &a, cudaStream_t s) {
    const int wpb = 2;
    const int grid = (a.NE + wpb - 1) / wpb;
    const int fused = a.n_tok <= 32;
    router_kernel<<<grid, 32 * wpb, 0, s>>>(a, fused);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || fused) return e;
    topk_kernel<<<(a.n_tok + 7) / 8, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gate_up(const GateUpArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.E / 128;
    if (NB <= 16) { GX_TYPE_SWITCH(a.type, return (gate_up_t<T, 1>(a, sm_count, s))) }
    if (NB <= 32) { GX_TYPE_SWITCH(a.type, return (gate_up_t<T, 2>(a, sm_count, s))) }
    return cudaErrorInvalidValue;
}

cudaError_t launch_down(const DownArgs &a, int sm_count, cudaStream_t s) {
    const int npair = a.U * (a.F / 128);
    if (npair <= 16) { GX_TYPE_SWITCH(a.type, return (down_t<T, 1>(a, sm_count, s))) }
    if (npair <= 32) { GX_TYPE_SWITCH(a.type, return (down_t<T, 2>(a, sm_count, s))) }
    if (npair <= 64) { GX_TYPE_SWITCH(a.type, return (down_t<T, 4>(a, sm_count, s))) }
    return cudaErrorInvalidValue;
}

cudaError_t launch_matvec(const MatvecArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.cols / 128;
    if (NB > 16) return cudaErrorInvalidValue;
    if (a.n_tok <= 8) { GX_TYPE_SWITCH(a.type, return (matvec_t<T, 1, 1>(a, sm_count, s))) }
    GX_TYPE_SWITCH(a.type, return (matvec_t<T, 1, 2>(a, sm_count, s)))
}

cudaError_t launch_repack(uint32_t type, const uint8_t *raw, uint64_t row_bytes, uint32_t rows, uint32_t cols,
                          uint8_t *tiles, cudaStream_t s) {
    const uint32_t nb = cols / 128;
    const uint64_t threads = (uint64_t)(rows / 8) * nb * 32;
    if (threads == 0) return cudaSuccess;
    repack_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(type, raw, row_bytes, rows, nb, tiles);
    return cudaGetLastError();
}

cudaError_t launch_decode_blocks(uint32_t type, const uint8_t *packed, uint32_t nblocks, const uint16_t *codebook,
                                 float *out, cudaStream_t s) {
    const uint64_t threads = (uint64_t)nblocks * type_steps(type);
    if (threads == 0) return cudaSuccess;
    decode_blocks_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(type, packed, nblocks, codebook, out);
    return cudaGetLastError();
}

cudaError_t launch_residual_copy(const void *x, int x_bf16, float *out, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    residual_copy_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, x_bf16, out, n);
    return cudaGetLastError();
}

}  // namespace gx
