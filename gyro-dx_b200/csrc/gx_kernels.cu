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
//   matvec_kernel      standalone decode GEMV of one matrix, a warp per 16-row unit, up to 16 tokens
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

#include <algorithm>

#define GX_TRACE_OWNER
#include "gx_device.cuh"
#include "gx_gemv.cuh"
#include "gx_internal.h"

namespace gx {

// ------------------------------------------------------------------------------------------
// Router GEMV (one warp per expert row) and expert selection.
// ------------------------------------------------------------------------------------------
// Selection for one token (one warp): optional RMSNorm scale of x (src/kernels.zig:281-291 with
// unit weight), logits = scale * (W x) + bias, softmax (src/kernels.zig:340-349), top-U with
// lower-index ties (src/engine.zig:671-686), renormalisation by max(sum, 2^-14) and the optional
// expert_weights_scale (src/engine.zig:533-539).
// Tree reductions over a lane's slots (depth log2 N instead of a chain of N).
template <int N>
__device__ __forceinline__ float tree_max(const float (&v)[N]) {
    float t[N];
#pragma unroll
    for (int j = 0; j < N; ++j) t[j] = v[j];
#pragma unroll
    for (int w = N / 2; w > 0; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) t[j] = fmaxf(t[j], t[j + w]);
    return t[0];
}
template <int N>
__device__ __forceinline__ float tree_sum(const float (&v)[N]) {
    float t[N];
#pragma unroll
    for (int j = 0; j < N; ++j) t[j] = v[j];
#pragma unroll
    for (int w = N / 2; w > 0; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) t[j] = t[j] + t[j + w];
    return t[0];
}
template <int N>
__device__ __forceinline__ unsigned long long tree_max_u64(const unsigned long long (&v)[N]) {
    unsigned long long t[N];
#pragma unroll
    for (int j = 0; j < N; ++j) t[j] = v[j];
#pragma unroll
    for (int w = N / 2; w > 0; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) t[j] = t[j] > t[j + w] ? t[j] : t[j + w];
    return t[0];
}

template <int NV>
__device__ void topk_token_nv(const RouterArgs &a, int t, int lane) {
    const float *row = a.logits + (size_t)t * a.NE;
    float ss = 0.f;
    if (a.norm_eps > 0.f) {
        if (a.ss_from_x) {
            // 8 values per lane per step (E is a multiple of 128): independent 16-byte loads
#pragma unroll 4
            for (int i = 8 * lane; i < a.E; i += 256) {
                float v[8];
                const size_t g = (size_t)t * a.E + i;
                if (a.x_bf16) {
                    const uint4 q = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(a.x) + g);
                    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        v[2 * j] = __uint_as_float(w4[j] << 16);
                        v[2 * j + 1] = __uint_as_float(w4[j] & 0xffff0000u);
                    }
                } else {
                    const float4 p0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + g);
                    const float4 p1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + g + 4);
                    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
                    v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        } else {
            ss = __ldcg(a.ss + t);
        }
    }
    const float scale = a.norm_eps > 0.f ? 1.0f / sqrtf(ss / (float)a.E + a.norm_eps) : 1.f;
    // Expert lane + 32 j in slot j (NV slots per lane, NE <= 32 NV). Every logit and bias load of
    // the lane goes out before the first is used (one round trip), then the split-K partials in
    // split order.
    float v[NV], bias[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int i = lane + 32 * j;
        const bool on = i < a.NE;
        v[j] = on ? __ldcg(row + i) : 0.f;
        bias[j] = on && a.bias ? __ldg(a.bias + i) : 0.f;
    }
    for (int z = 1; z < a.logit_splits; ++z) {
        const float *rz = row + (size_t)z * a.n_tok * a.NE;
        float p[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) p[j] = lane + 32 * j < a.NE ? __ldcg(rz + lane + 32 * j) : 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] += p[j];
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = lane + 32 * j < a.NE ? v[j] * scale + bias[j] : -INFINITY;
    // softmax (src/kernels.zig:340-349): the maximum by one warp-wide integer maximum of the
    // order-preserving image of the floats, the sum by a tree in the lane and across lanes
    float m = tree_max(v);
    {
        int o = __float_as_int(m);
        o = __reduce_max_sync(0xffffffffu, o >= 0 ? o : o ^ 0x7fffffff);
        m = __int_as_float(o >= 0 ? o : o ^ 0x7fffffff);
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = lane + 32 * j < a.NE ? expf(v[j] - m) : 0.f;
    float s = tree_sum(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    // Selection key: probability bits (order-preserving for p >= 0) above the complemented index,
    // so the largest key is the largest probability and, among equal ones, the lowest index (the
    // tie rule of src/engine.zig:671-686). A round takes the lane's largest key by a tree, then
    // two warp-wide unsigned maxima (probability, then index among equal probabilities). Absent
    // and taken experts have key 0; present ones have a nonzero complemented index.
    unsigned long long key[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int i = lane + 32 * j;
        key[j] = i < a.NE ? ((unsigned long long)__float_as_uint(v[j] / s) << 32) | (0xffffffffu - (uint32_t)i) : 0ull;
    }
    float my_w = 0.f, total = 0.f;
    uint32_t my_id = 0;
    for (int k = 0; k < a.U; ++k) {
        const unsigned long long best = tree_max_u64(key);
        const uint32_t hm = __reduce_max_sync(0xffffffffu, (uint32_t)(best >> 32));
        const uint32_t lm = __reduce_max_sync(0xffffffffu, (uint32_t)(best >> 32) == hm ? (uint32_t)best : 0u);
        const unsigned long long win = ((unsigned long long)hm << 32) | lm;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (key[j] == win) key[j] = 0ull;
        // renormalisation sum in selection order (src/engine.zig:533-539)
        total += __uint_as_float(hm);
        if (lane == k) {
            my_w = __uint_as_float(hm);
            my_id = 0xffffffffu - lm;
        }
    }
    total = fmaxf(total, 6.103515625e-5f);
    if (lane < a.U) {
        float w = my_w / total;
        if (a.scale != 0.f && a.scale != 1.f) w *= a.scale;
        a.ids[(size_t)t * a.U + lane] = my_id;
        a.weights[(size_t)t * a.U + lane] = w;
    }
    if (lane == 0) a.xscale[t] = scale;
}

__device__ __forceinline__ void topk_token(const RouterArgs &a, int t, int lane) {
    if (a.NE <= 256)
        topk_token_nv<8>(a, t, lane);
    else
        topk_token_nv<16>(a, t, lane);
}

// Block-wide selection for one token by a 512-thread CTA (thread i scores expert i): the same
// arithmetic as topk_token, then every warp keeps its own top-U and warp 0 merges them.
// Results go to sel_ids / sel_w (U entries) and *sel_scale; cand and red are shared scratch.
__device__ void block_topk(const GateUpArgs &a, int t, uint32_t *sel_ids, float *sel_w, float *sel_scale,
                           unsigned long long *cand, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float scale = a.norm_eps > 0.f ? 1.0f / sqrtf(__ldcg(a.ss + t) / (float)a.E + a.norm_eps) : 1.f;
    const bool live = tid < a.NE;
    const float l = live ? __ldcg(a.logits + (size_t)t * a.NE + tid) * scale + (a.bias ? __ldg(a.bias + tid) : 0.f)
                         : -INFINITY;
    float m = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int w = 1; w < 16; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    const float e = live ? expf(l - m) : 0.f;
    float s = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.f;
#pragma unroll
    for (int w = 0; w < 16; ++w) s += red[w];
    unsigned long long key = live ? ((unsigned long long)__float_as_uint(e / s) << 32) | (0xffffffffu - (uint32_t)tid) : 0ull;
    unsigned long long mine = 0ull;
    for (int k = 0; k < a.U; ++k) {
        unsigned long long best = key;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (key == best) key = 0ull;
        if (lane == k) mine = best;
    }
    if (lane < 16) cand[warp * 16 + lane] = lane < a.U ? mine : 0ull;
    __syncthreads();
    if (warp == 0) {
        unsigned long long c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = cand[lane + 32 * j];
        float my_w = 0.f;
        uint32_t my_id = 0;
        for (int k = 0; k < a.U; ++k) {
            unsigned long long b = c[0];
#pragma unroll
            for (int j = 1; j < 8; ++j) b = c[j] > b ? c[j] : b;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
                b = other > b ? other : b;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (c[j] == b) c[j] = 0ull;
            if (lane == k) {
                my_w = __uint_as_float((uint32_t)(b >> 32));
                my_id = 0xffffffffu - (uint32_t)b;
            }
        }
        float total = 0.f;
        for (int k = 0; k < a.U; ++k) total += __shfl_sync(0xffffffffu, my_w, k);
        total = fmaxf(total, 6.103515625e-5f);
        if (lane < a.U) {
            float w = my_w / total;
            if (a.wscale != 0.f && a.wscale != 1.f) w *= a.wscale;
            sel_ids[lane] = my_id;
            sel_w[lane] = w;
        }
        if (lane == 0) *sel_scale = scale;
    }
    __syncthreads();
}

constexpr int kRouterTok = 4;       // tokens staged in shared memory per pass
constexpr int kRouterWarps = 2;     // expert rows per CTA

// W rows are loaded into registers before pdl_wait(), so they stream while the previous kernel
// (the last layer's down GEMV) still runs. x is staged in shared memory as f32.
template <int NJ>
__global__ void __launch_bounds__(64) router_kernel(RouterArgs a) {
    extern __shared__ __align__(16) float xsm[];          // [kRouterTok][E]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x * kRouterWarps + warp;
    GX_TRACE_START(0);
    pdl_launch_dependents();
    const bool has_row = r < a.NE;
    const float *w = a.W + (size_t)(has_row ? r : 0) * a.E;
    float4 wv[NJ];                                       // E <= 128 * NJ
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int c = 128 * j + 4 * lane;
        wv[j] = (has_row && c < a.E) ? __ldg(reinterpret_cast<const float4 *>(w + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    GX_TRACE_POINT(0);
    pdl_wait();
    GX_TRACE_POINT(1);
    if (NJ <= 16 && a.n_tok <= kRouterTok) {
        // Few tokens: every warp reads the token rows straight into registers (all loads of a row
        // out at once), four independent FMA chains, and warp 0 of CTA 0 takes the sums of squares.
        // (E <= 2048: a row and the warp's weights fit in registers.)
        for (int t = 0; t < (NJ <= 16 ? a.n_tok : 0); ++t) {
            float4 xv[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int c = 128 * j + 4 * lane;
                if (c < a.E) {
                    const size_t g = (size_t)t * a.E + c;
                    if (a.x_bf16) {
                        const uint2 q = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(a.x) + g);
                        xv[j] = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u),
                                            __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xffff0000u));
                    } else {
                        xv[j] = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + g);
                    }
                } else {
                    xv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                float &q = acc[j & 3];
                q = fmaf(wv[j].x, xv[j].x, q);
                q = fmaf(wv[j].y, xv[j].y, q);
                q = fmaf(wv[j].z, xv[j].z, q);
                q = fmaf(wv[j].w, xv[j].w, q);
            }
            float dot = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0 && has_row) a.logits[(size_t)t * a.NE + r] = dot;
            if (a.norm_eps > 0.f && blockIdx.x == 0 && warp == 0) {
                float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    float &q = sq[j & 3];
                    q = fmaf(xv[j].x, xv[j].x, q);
                    q = fmaf(xv[j].y, xv[j].y, q);
                    q = fmaf(xv[j].z, xv[j].z, q);
                    q = fmaf(xv[j].w, xv[j].w, q);
                }
                float ss = (sq[0] + sq[1]) + (sq[2] + sq[3]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                if (lane == 0) a.ss[t] = ss;
            }
        }
    } else
    for (int t0 = 0; t0 < a.n_tok; t0 += kRouterTok) {
        const int nt = min(kRouterTok, a.n_tok - t0);
        __syncthreads();
        // 8 values per thread per iteration (E is a multiple of 128): independent 16-byte loads.
#pragma unroll 4
        for (int i = threadIdx.x * 8; i < nt * a.E; i += blockDim.x * 8) {
            const size_t g = (size_t)t0 * a.E + i;
            float v[8];
            if (a.x_bf16) {
                const uint4 q = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(a.x) + g);
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[2 * j] = __uint_as_float(w4[j] << 16);
                    v[2 * j + 1] = __uint_as_float(w4[j] & 0xffff0000u);
                }
            } else {
                const float4 p0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + g);
                const float4 p1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + g + 4);
                v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
                v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
            }
            *reinterpret_cast<float4 *>(xsm + i) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4 *>(xsm + i + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
        __syncthreads();
        GX_TRACE_POINT(5);
        // CTA 0 publishes each token's sum of squares for the RMSNorm scale (read by top-k).
        if (a.norm_eps > 0.f && blockIdx.x == 0 && warp == 0) {
            for (int t = 0; t < nt; ++t) {
                float ss = 0.f;
                for (int i = lane * 4; i < a.E; i += 128) {
                    const float4 v = *reinterpret_cast<const float4 *>(xsm + t * a.E + i);
                    ss = fmaf(v.x, v.x, ss);
                    ss = fmaf(v.y, v.y, ss);
                    ss = fmaf(v.z, v.z, ss);
                    ss = fmaf(v.w, v.w, ss);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                if (lane == 0) a.ss[t0 + t] = ss;
            }
        }
        float acc[kRouterTok];
#pragma unroll
        for (int t = 0; t < kRouterTok; ++t) acc[t] = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int c = 128 * j + 4 * lane;
            if (c < a.E) {
#pragma unroll
                for (int t = 0; t < kRouterTok; ++t) {
                    if (t < nt) {
                        const float4 xv = *reinterpret_cast<const float4 *>(xsm + t * a.E + c);
                        acc[t] = fmaf(wv[j].x, xv.x, acc[t]);
                        acc[t] = fmaf(wv[j].y, xv.y, acc[t]);
                        acc[t] = fmaf(wv[j].z, xv.z, acc[t]);
                        acc[t] = fmaf(wv[j].w, xv.w, acc[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kRouterTok; ++t)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
        if (lane == 0 && has_row)
            for (int t = 0; t < nt; ++t) a.logits[(size_t)(t0 + t) * a.NE + r] = acc[t];
    }
    GX_TRACE_POINT(2);
    if (a.done) {
        // Lane 0 of every warp wrote this warp's logits (and CTA 0's warp 0 the sums of squares);
        // it counts the warp done with one acquire-release add. The warp that counts last has
        // acquired every other warp's writes: it selects the experts of every token and resets
        // the count for the next launch.
        unsigned old = 0;
        if (lane == 0) asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.done) : "memory");
        old = __shfl_sync(0xffffffffu, old, 0);
        __syncwarp();  // the other lanes read after lane 0's acquire
        if (old == gridDim.x * kRouterWarps - 1) {
            for (int t = 0; t < a.n_tok; ++t) topk_token(a, t, lane);
            if (lane == 0) *a.done = 0u;
        }
    }
}

__global__ void __launch_bounds__(256) topk_kernel(RouterArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.n_tok) return;
    topk_token(a, t, lane);
}

// ---- gate/up: unit = (slot, RG row-groups of both projections) ---------------------------
template <uint32_t T, int KBW, int NC>
__global__ void __launch_bounds__(512, 1) gate_up_kernel(GateUpArgs a, int P) {
    using CB = Codebook<NC>;
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
    unsigned long long *cand = reinterpret_cast<unsigned long long *>(xs + 16 * 128);  // [256]
    uint32_t *sel_ids = reinterpret_cast<uint32_t *>(cand + 256);      // [8][16]
    float *sel_w = reinterpret_cast<float *>(sel_ids + 128);           // [8][16]
    float *sel_scale = sel_w + 128;                                    // [8]
    float *red = sel_scale + 8;                                        // [16]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 16);

    GX_TRACE_START(1);
    pdl_launch_dependents();
    const int n_units = a.n_slots * UPS;
    StageCtl ctl;
    ctl.bar = bar;
    ctl.P = P;
    ctl.u0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
    ctl.u1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
    ctl.n_stages = (ctl.u1 - ctl.u0 + P - 1) / P;
    const int tok_first = (ctl.u0 / UPS) / a.U;
    const int n_tok_cta = ctl.n_stages > 0 ? ((ctl.u1 - 1) / UPS) / a.U - tok_first + 1 : 0;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 1);
        fence_barrier_init();
        // the codebook streams in from its prebuilt image while the router still runs
        CB::stage_bulk(cb, a.codebook_image, &bar[2]);
    }
    __syncthreads();

    // Warp 0 fills stage s: lane 0 posts the byte count, then every lane loads one slot's
    // expert id and issues that copy, so the id loads and copies go out in parallel.
    auto issue = [&](int s) {
        uint8_t *buf = stage + (s & 1) * stage_bytes;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        if (lane == 0) {
            uint32_t total = 0;
            for (int u = ua; u < ub; ++u) total += 2u * (uint32_t)(min(RG, NT - (u % UPS) * RG) * NB * TB);
            mbar_expect_tx(&bar[s & 1], total);
        }
        __syncwarp();
        for (int k = lane; k < (ub - ua) * 2; k += 32) {
            const int u = ua + (k >> 1), proj = k & 1;
            const int slot = u / UPS, ui = u % UPS;
            const uint32_t bytes = (uint32_t)(min(RG, NT - ui * RG) * NB * TB);
            uint32_t e = a.fused_topk ? sel_ids[(slot / a.U - tok_first) * 16 + slot % a.U] : a.ids[slot];
            if (e >= (uint32_t)a.n_expert) {
                atomicExch(a.err, KERR_BOUNDS);
                e = 0;
            }
            const uint64_t off = (uint64_t)e * a.expert_bytes + (uint64_t)ui * unit_proj;
            bulk_g2s(buf + (u - ua) * 2 * unit_proj + proj * unit_proj, (proj ? a.up : a.gate) + off, bytes,
                     &bar[s & 1]);
        }
    };
    GX_TRACE_POINT(0);
    pdl_wait();
    GX_TRACE_POINT(1);
    if (a.fused_topk) {
        // Expert selection for the tokens of this CTA's units; the CTA holding a token's first
        // unit publishes it for the down kernel.
        for (int tt = 0; tt < n_tok_cta; ++tt)
            block_topk(a, tok_first + tt, sel_ids + tt * 16, sel_w + tt * 16, sel_scale + tt, cand, red);
        if (tid < n_tok_cta * a.U) {
            const int tt = tid / a.U, k = tid % a.U, t = tok_first + tt;
            const int first_unit = t * a.U * UPS;
            if (first_unit >= ctl.u0 && first_unit < ctl.u1) {
                a.ids_out[t * a.U + k] = sel_ids[tt * 16 + k];
                a.weights_out[t * a.U + k] = sel_w[tt * 16 + k];
            }
        }
    }
    // no CTA barrier here: the other warps rotate their input while warp 0 issues the copies
    if (warp == 0) {
        if (ctl.n_stages > 0) issue(0);
        if (ctl.n_stages > 1) issue(1);
    }

    GX_TRACE_POINT(2);
    const bool active = warp < WB * RG;
    const int kcol = warp % WB, rg = warp / WB;
    const uint32_t copy_off = CB::copy_off(lane);
    uint32_t A[KBW][1][8][4];
    int cur_tok = -1;
    float *xw = xs + warp * 128;
    // The first unit's activations are prepared while its weights are still in flight.
    auto build_a = [&](int tok) {
#pragma unroll
        for (int j = 0; j < KBW; ++j) {
            const int b = kcol + WB * j;
            if (b < NB) {
                rotated_block_to_smem(a.x, a.x_bf16, (size_t)tok * a.E + b * 128,
                                      a.fused_topk ? sel_scale[tok - tok_first] : (a.xscale ? a.xscale[tok] : 1.f),
                                      a.signs, b * 128, xw, lane);
                build_a_single(xw, lane, A[j][0]);
                __syncwarp();
            }
        }
    };
    if (active && ctl.n_stages > 0) {
        cur_tok = (ctl.u0 / UPS) / a.U;
        build_a(cur_tok);
    }
    GX_TRACE_POINT(3);
    if (!codebook_wait(&bar[2], ctl, a.err)) return;

    for (int s = 0; s < ctl.n_stages; ++s) {
        if (!stage_wait(ctl, s, a.err)) return;
        if (s == 0) GX_TRACE_POINT(4);
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        const uint8_t *buf = stage + (s & 1) * stage_bytes;
        for (int u = ua; u < ub; ++u) {
            const int slot = u / UPS, ui = u % UPS;
            const int tok = slot / a.U;
            if (active && tok != cur_tok) {
                build_a(tok);
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
                            tile_mma<T, 1, NC>(ubase + proj * unit_proj + (rg * NB + b) * TB, cb, copy_off, lane, A[j], acc);
                    }
                    if (lane < 4) {
                        float *p = part + (((u - ua) * 2 + proj) * 16 + rg * WB + kcol) * 8 + 2 * lane;
                        p[0] = acc[0][0];
                        p[1] = acc[0][1];
                    }
                }
            }
        }
        if (s == 0) GX_TRACE_POINT(5);
        __syncthreads();
        if (warp == 0 && s + 2 < ctl.n_stages) issue(s + 2);
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
    GX_TRACE_POINT(6);
}

// ---- down: unit = (token, one row group); warps own (slot, block) pairs -------------------
template <uint32_t T, int KBW, int NC>
__global__ void __launch_bounds__(512, 1) down_kernel(DownArgs a, int P) {
    using CB = Codebook<NC>;
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
    float *wsm = xs + 16 * 128;                                         // [P][16] routing weights
    uint64_t *bar = reinterpret_cast<uint64_t *>(wsm + 4 * 16);

    GX_TRACE_START(2);
    pdl_launch_dependents();
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
        mbar_init(&bar[2], 1);
        fence_barrier_init();
        CB::stage_bulk(cb, a.codebook_image, &bar[2]);
    }
    __syncthreads();

    // Warp 0 fills stage s, one (unit, slot) copy per lane (see gate_up_kernel).
    auto issue = [&](int s) {
        uint8_t *buf = stage + (s & 1) * stage_bytes;
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        if (lane == 0) mbar_expect_tx(&bar[s & 1], (uint32_t)((ub - ua) * unit_bytes));
        __syncwarp();
        for (int q = lane; q < (ub - ua) * a.U; q += 32) {
            const int u = ua + q / a.U, k = q % a.U;
            const int t = u / NT, i = u % NT;
            uint32_t e = a.ids[t * a.U + k];
            if (e >= (uint32_t)a.n_expert) {
                atomicExch(a.err, KERR_BOUNDS);
                e = 0;
            }
            bulk_g2s(buf + (u - ua) * unit_bytes + k * slot_bytes,
                     a.down + (uint64_t)e * a.expert_bytes + (uint64_t)i * slot_bytes, (uint32_t)slot_bytes, &bar[s & 1]);
        }
    };
    GX_TRACE_POINT(0);
    pdl_wait();
    GX_TRACE_POINT(1);
    if (warp == 0) {
        if (ctl.n_stages > 0) issue(0);
        if (ctl.n_stages > 1) issue(1);
    }

    GX_TRACE_POINT(2);
    const uint32_t copy_off = CB::copy_off(lane);
    uint32_t A[KBW][1][8][4];
    int cur_tok = -1;
    float *xw = xs + warp * 128;
    // Down input of token t: signs + FWHT of silu(g)*u per (slot, block) pair of this warp. All
    // pairs' loads go out before the first transform.
    auto build_a = [&](int t) {
        float v[KBW][4], sg[KBW][4];
#pragma unroll
        for (int j = 0; j < KBW; ++j) {
            const int p = warp + 16 * j;
            if (p < NPAIR) {
                const int k = p / NBF, b = p % NBF;
                const float4 q = *reinterpret_cast<const float4 *>(a.act + (size_t)(t * a.U + k) * a.F + b * 128 + 4 * lane);
                v[j][0] = q.x; v[j][1] = q.y; v[j][2] = q.z; v[j][3] = q.w;
                if (a.signs) {
                    const float4 g = *reinterpret_cast<const float4 *>(a.signs + b * 128 + 4 * lane);
                    sg[j][0] = g.x; sg[j][1] = g.y; sg[j][2] = g.z; sg[j][3] = g.w;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < KBW; ++j) {
            const int p = warp + 16 * j;
            if (p < NPAIR) {
                if (a.signs) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[j][q] *= sg[j][q];
                    fwht128_warp(v[j], lane);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) xw[4 * lane + q] = v[j][q];
                __syncwarp();
                build_a_single(xw, lane, A[j][0]);
                __syncwarp();
            }
        }
    };
    if (ctl.n_stages > 0) {
        cur_tok = ctl.u0 / NT;
        build_a(cur_tok);
    }
    GX_TRACE_POINT(3);
    if (!codebook_wait(&bar[2], ctl, a.err)) return;

    for (int s = 0; s < ctl.n_stages; ++s) {
        if (!stage_wait(ctl, s, a.err)) return;
        if (s == 0) GX_TRACE_POINT(4);
        const int ua = ctl.u0 + s * P, ub = min(ua + P, ctl.u1);
        const uint8_t *buf = stage + (s & 1) * stage_bytes;
        for (int u = ua; u < ub; ++u) {
            const int t = u / NT;
            if (t != cur_tok) {
                build_a(t);
                cur_tok = t;
            }
            if (warp == 0 && lane < a.U) wsm[(u - ua) * 16 + lane] = a.weights[t * a.U + lane];
#pragma unroll
            for (int j = 0; j < KBW; ++j) {
                const int p = warp + 16 * j;
                if (p < NPAIR) {
                    const int k = p / NBF, b = p % NBF;
                    float acc[1][2] = {{0.f, 0.f}};
                    tile_mma<T, 1, NC>(buf + (u - ua) * unit_bytes + k * slot_bytes + b * TB, cb, copy_off, lane, A[j],
                                   acc);
                    if (lane < 4) {
                        float *q = part + ((u - ua) * PMAX + p) * 8 + 2 * lane;
                        q[0] = acc[0][0];
                        q[1] = acc[0][1];
                    }
                }
            }
        }
        if (s == 0) GX_TRACE_POINT(5);
        __syncthreads();
        if (warp == 0 && s + 2 < ctl.n_stages) issue(s + 2);
        for (int r = tid; r < (ub - ua) * 8; r += blockDim.x) {
            const int j = r >> 3, n = r & 7;
            const int u = ua + j, t = u / NT, i = u % NT;
            const int row = i * 8 + n;
            float v = 0.f;
            for (int k = 0; k < a.U; ++k) {
                float dk = 0.f;
                for (int b = 0; b < NBF; ++b) dk += part[(j * PMAX + k * NBF + b) * 8 + n];
                v += wsm[j * 16 + k] * dk;
            }
            const size_t o = (size_t)t * a.E + row;
            if (a.extra) v += a.extra[o];
            if (a.resid) v = load_act(a.resid, a.resid_bf16, o) + v;
            if (!(fabsf(v) <= 3.4028235e38f)) atomicExch(a.err, KERR_RANGE);   // Inf or NaN
            if (a.out_bf16)
                reinterpret_cast<__nv_bfloat16 *>(a.out)[o] = __float2bfloat16_rn(v);
            else
                reinterpret_cast<float *>(a.out)[o] = v;
        }
        __syncthreads();
    }
    GX_TRACE_POINT(6);
}

// ---- standalone matvec: one warp per 16-row unit across all column blocks -----------------
// The weights are the MMA's A operand (m16n8k16: rows g and g+8 of a lane are the same row of
// two consecutive 8-row tiles, so a lane decodes one quarter of two rows) and the activations
// the B operand: the token dimension n holds (token, hi/lo part) pairs, four tokens per MMA
// group. Every warp streams its own units with the next blocks' codes loaded into registers two
// blocks ahead (no shared-memory staging, no barriers, no cross-warp reduction); shared memory
// holds the codebook copies and the activations in B-fragment order.
template <uint32_t T>
struct TileCodes {
    uint32_t own0[4], own1[4];   // the lane's run in the unit's two tiles
    uint32_t sc;                 // scales of row g in the two tiles (low / high half)
};

template <uint32_t T>
__device__ __forceinline__ void load_codes(const uint8_t *t0, const uint8_t *t1, int lane, TileCodes<T> &c) {
    load_run<T>(t0, lane, c.own0);
    load_run<T>(t1, lane, c.own1);
    const int g = lane >> 2;
    const uint32_t s0 = *reinterpret_cast<const uint16_t *>(t0 + tile_code_bytes(T) + 2 * g);
    const uint32_t s1 = *reinterpret_cast<const uint16_t *>(t1 + tile_code_bytes(T) + 2 * g);
    c.sc = s0 | (s1 << 16);
}

template <uint32_t T, int NG, int NC, int THREADS>
__global__ void __launch_bounds__(THREADS, 1) matvec_kernel(MatvecArgs a, int t0) {
    using CB = Codebook<NC>;
    constexpr int TB = tile_bytes(T);
    extern __shared__ __align__(128) uint8_t smem[];
    uint32_t *cb = reinterpret_cast<uint32_t *>(smem);
    uint2 *xf = reinterpret_cast<uint2 *>(smem + CB::BYTES);   // [block][chunk][group][lane]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int NB = a.cols >> 7;
    const int ntok = min(4 * NG, a.n_tok - t0);
    GX_TRACE_START(3);

    CB::stage(cb, a.codebook, tid, blockDim.x);
    // Activation fragments: lane (g, q) of group ng carries token 4ng + g/2, part g%2 (hi or lo
    // fp16 half of the f32 value) at columns 32q + 4c + {0,1} (b0) and {2,3} (b1).
    for (int i = tid; i < NB * 8 * NG * 32; i += blockDim.x) {
        const int ln = i & 31, ng = (i >> 5) % NG, c = (i / (32 * NG)) & 7, b = i / (256 * NG);
        const int tok = 4 * ng + ((ln >> 2) >> 1), part = (ln >> 2) & 1, qq = ln & 3;
        uint2 v = make_uint2(0u, 0u);
        if (tok < ntok) {
            const float4 x4 = *reinterpret_cast<const float4 *>(a.x + (size_t)(t0 + tok) * a.cols + b * 128 + 32 * qq + 4 * c);
            float h0, l0, h1, l1, h2, l2, h3, l3;
            split_hilo(x4.x, h0, l0);
            split_hilo(x4.y, h1, l1);
            split_hilo(x4.z, h2, l2);
            split_hilo(x4.w, h3, l3);
            v.x = part ? pack_half2(l0, l1) : pack_half2(h0, h1);
            v.y = part ? pack_half2(l2, l3) : pack_half2(h2, h3);
        }
        xf[i] = v;
    }
    __syncthreads();

    const int n_units = (a.rows + 15) >> 4;     // the tiles hold a zero row group past an odd count
    const int wid = blockIdx.x * (blockDim.x >> 5) + warp, nw = gridDim.x * (blockDim.x >> 5);
    const int n_mine = wid < n_units ? (n_units - 1 - wid) / nw + 1 : 0;
    const int steps = n_mine * NB;            // (unit, block) pairs of this warp, in order
    const uint32_t lane_off = 4u * CB::copy_off(lane);
    const uint8_t *cbb = smem;
    const int nbr = (lane & ~3) | ((lane + 3) & 3);
    // (unit, block) positions advance by counting, no division in the loop: the prefetch runs two
    // steps ahead of the step being decoded
    const size_t unit_stride = (size_t)2 * NB * TB;      // bytes of one 16-row unit
    const uint8_t *pf_unit = a.tiles + (size_t)wid * unit_stride;
    int pf_b = 0;
    auto prefetch = [&](TileCodes<T> &dst) {
        load_codes<T>(pf_unit + (size_t)pf_b * TB, pf_unit + (size_t)(NB + pf_b) * TB, lane, dst);
        if (++pf_b == NB) {
            pf_b = 0;
            pf_unit += (size_t)nw * unit_stride;
        }
    };
    TileCodes<T> nx0, nx1;
    if (steps > 0) prefetch(nx0);
    if (steps > 1) prefetch(nx1);
    float acc[NG][2];
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) acc[ng][0] = acc[ng][1] = 0.f;
    bool xon[NG];                             // lanes whose (token, part) is live load activations
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) xon[ng] = 4 * ng + (g >> 1) < ntok;
    int b = 0, u = wid;
    for (int step = 0; step < steps; ++step) {
        const TileCodes<T> cur = nx0;
        nx0 = nx1;
        if (step + 2 < steps) prefetch(nx1);
        const uint32_t v0 = __shfl_sync(0xffffffffu, (T == T_TQ2_T) ? cur.own0[1] : cur.own0[0], nbr);
        const uint32_t v1 = __shfl_sync(0xffffffffu, (T == T_TQ2_T) ? cur.own1[1] : cur.own1[0], nbr);
        uint32_t o0a[8], o1a[8], o0b[8], o1b[8];
        quarter_offsets<T, NC>(cur.own0, (T == T_TQ2_T) ? (v0 >> 24) : (v0 & 0xffffu), lane_off, o0a, o1a);
        quarter_offsets<T, NC>(cur.own1, (T == T_TQ2_T) ? (v1 >> 24) : (v1 & 0xffffu), lane_off, o0b, o1b);
        float d[NG][4];
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) d[ng][0] = d[ng][1] = d[ng][2] = d[ng][3] = 0.f;
        const uint2 *xb = xf + (size_t)b * 8 * NG * 32 + lane;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t w[4] = {lds_u32(cbb, o0a[c]), lds_u32(cbb, o0b[c]), lds_u32(cbb, o1a[c]),
                                   lds_u32(cbb, o1b[c])};
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) {
                const uint2 xv = xon[ng] ? xb[(c * NG + ng) * 32] : make_uint2(0u, 0u);
                mma16816(d[ng], w, xv.x, xv.y);
            }
        }
        const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&cur.sc));
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
            acc[ng][0] = fmaf(s.x, d[ng][0] + d[ng][1], acc[ng][0]);
            acc[ng][1] = fmaf(s.y, d[ng][2] + d[ng][3], acc[ng][1]);
        }
        if (++b == NB) {
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) {
                const int tok = 4 * ng + q;
                if (tok < ntok) {
                    float *y = a.y + (size_t)(t0 + tok) * a.rows + 16 * u + g;
                    y[0] = acc[ng][0];
                    if (16 * u + 8 < a.rows) y[8] = acc[ng][1];
                }
                acc[ng][0] = acc[ng][1] = 0.f;
            }
            b = 0;
            u += nw;
        }
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

// Raises the dynamic shared-memory limit of kernel instantiation K once per process (never
// inside a stream capture: the first launch of every instantiation happens in an eager call).
template <auto K, int Bytes = kSmemLimit>
cudaError_t set_smem() {
    static const cudaError_t once = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, Bytes);
    return once;
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), int grid, int block, int smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Stage count P per buffer: as many units as fit under the budget (at most 4).
int pick_stages(int fixed, int per_stage, int budget) {
    int P = 4;
    while (P > 1 && fixed + 2 * P * per_stage > budget) --P;
    return fixed + 2 * P * per_stage <= budget ? P : 0;
}

template <uint32_t T, int KBW, int NC>
cudaError_t gate_up_t(const GateUpArgs &a, int sm_count, cudaStream_t s, bool pdl) {
    const int NB = a.E / 128, WB = NB < 16 ? NB : 16, RG = 16 / WB;
    const int unit_proj = RG * NB * tile_bytes(T);
    // codebook + per-warp activation scratch + selection scratch + barriers
    const int fixed = Codebook<NC>::BYTES + 16 * 128 * 4 + (256 * 8 + 128 * 4 * 2 + 8 * 4 + 16 * 4) + 64;
    // per stage: P units x 2 projections, plus the partials of those units
    const int per_unit = 2 * unit_proj + 2 * 16 * 8 * 4 / 2;
    const int P = pick_stages(fixed, per_unit, kSmemLimit);
    if (P == 0) return cudaErrorInvalidValue;
    const int smem = fixed + 2 * P * 2 * unit_proj + P * 2 * 16 * 8 * 4;
    const int NT = a.F / 8, UPS = (NT + RG - 1) / RG;
    const int n_units = a.n_slots * UPS;
    if (n_units == 0) return cudaSuccess;
    // 512 threads at ~120 registers fill an SM's register file: one CTA per SM.
    const int grid = n_units < sm_count ? n_units : sm_count;
    cudaError_t e = set_smem<gate_up_kernel<T, KBW, NC>>();
    if (e != cudaSuccess) return e;
    return launch(gate_up_kernel<T, KBW, NC>, grid, 512, smem, s, pdl, a, P);
}

template <uint32_t T, int KBW, int NC>
cudaError_t down_t(const DownArgs &a, int sm_count, cudaStream_t s, bool pdl) {
    const int NBF = a.F / 128;
    const int unit_bytes = a.U * NBF * tile_bytes(T);
    const int PMAX = 16 * KBW;
    const int fixed = Codebook<NC>::BYTES + 16 * 128 * 4 + 4 * 16 * 4 + 64;
    const int per_unit = unit_bytes + PMAX * 8 * 4 / 2;
    const int P = pick_stages(fixed, per_unit, kSmemLimit);
    if (P == 0) return cudaErrorInvalidValue;
    const int smem = fixed + 2 * P * unit_bytes + P * PMAX * 8 * 4;
    const int n_units = a.n_tok * (a.E / 8);
    if (n_units == 0) return cudaSuccess;
    // 512 threads at ~120 registers fill an SM's register file: one CTA per SM.
    const int grid = n_units < sm_count ? n_units : sm_count;
    cudaError_t e = set_smem<down_kernel<T, KBW, NC>>();
    if (e != cudaSuccess) return e;
    return launch(down_kernel<T, KBW, NC>, grid, 512, smem, s, pdl, a, P);
}

template <uint32_t T, int NG, int NC, int THREADS>
cudaError_t matvec_t(const MatvecArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.cols / 128;
    const int smem = Codebook<NC>::BYTES + NB * 8 * NG * 32 * 8;
    if (smem > kSmemLimit) return cudaErrorInvalidValue;
    const int n_units = (a.rows + 15) / 16;
    const int grid = std::max(1, std::min(sm_count, (n_units + THREADS / 32 - 1) / (THREADS / 32)));
    cudaError_t e = set_smem<matvec_kernel<T, NG, NC, THREADS>>();
    if (e != cudaSuccess) return e;
    for (int t0 = 0; t0 < a.n_tok; t0 += 4 * NG) {
        e = launch(matvec_kernel<T, NG, NC, THREADS>, grid, THREADS, smem, s, false, a, t0);
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

bool gate_up_fuses_topk(int E, int F, int U, int n_tok, int sm_count) {
    const int NB = E / 128, WB = NB < 16 ? NB : 16, RG = 16 / WB;
    const int UPS = (F / 8 + RG - 1) / RG;
    const long long units = (long long)n_tok * U * UPS;
    if (units == 0) return false;
    const long long grid = units < sm_count ? units : sm_count;
    const long long per_cta = (units + grid - 1) / grid;
    const long long per_tok = (long long)U * UPS;
    return (per_cta + per_tok - 1) / per_tok + 1 <= 8;
}

cudaError_t launch_router(const RouterArgs &a, cudaStream_t s, bool pdl, bool with_topk) {
    const int grid = (a.NE + kRouterWarps - 1) / kRouterWarps;
    const int smem = kRouterTok * a.E * 4;
    cudaError_t e;
    if (a.E <= 2048) {
        e = set_smem<router_kernel<16>, kRouterTok * 4096 * 4>();
        if (e == cudaSuccess) e = launch(router_kernel<16>, grid, 32 * kRouterWarps, smem, s, pdl, a);
    } else {
        e = set_smem<router_kernel<32>, kRouterTok * 4096 * 4>();
        if (e == cudaSuccess) e = launch(router_kernel<32>, grid, 32 * kRouterWarps, smem, s, pdl, a);
    }
    if (e != cudaSuccess || !with_topk) return e;
    return launch(topk_kernel, (a.n_tok + 7) / 8, 256, 0, s, pdl, a);
}

cudaError_t launch_topk(const RouterArgs &a, cudaStream_t s) {
    if (a.n_tok == 0) return cudaSuccess;
    return launch(topk_kernel, (a.n_tok + 7) / 8, 256, 0, s, chain_pdl_enabled(), a);
}

cudaError_t launch_gate_up(const GateUpArgs &a, int sm_count, cudaStream_t s, bool pdl) {
    constexpr int NC = kCodebookCopies;
    const int NB = a.E / 128;
    if (NB <= 16) { GX_TYPE_SWITCH(a.type, return (gate_up_t<T, 1, NC>(a, sm_count, s, pdl))) }
    if (NB <= 32) { GX_TYPE_SWITCH(a.type, return (gate_up_t<T, 2, NC>(a, sm_count, s, pdl))) }
    return cudaErrorInvalidValue;
}

cudaError_t launch_down(const DownArgs &a, int sm_count, cudaStream_t s, bool pdl) {
    constexpr int NC = kCodebookCopies;
    const int npair = a.U * (a.F / 128);
    if (npair <= 16) { GX_TYPE_SWITCH(a.type, return (down_t<T, 1, NC>(a, sm_count, s, pdl))) }
    if (npair <= 32) { GX_TYPE_SWITCH(a.type, return (down_t<T, 2, NC>(a, sm_count, s, pdl))) }
    if (npair <= 64) { GX_TYPE_SWITCH(a.type, return (down_t<T, 4, NC>(a, sm_count, s, pdl))) }
    return cudaErrorInvalidValue;
}

cudaError_t launch_matvec(const MatvecArgs &a, int sm_count, cudaStream_t s) {
    const int NB = a.cols / 128;
    if (NB > 16 || a.rows % 8) return cudaErrorInvalidValue;
    // Up to 4 tokens: one MMA group; up to 8: two; beyond, four groups per launch with half the
    // codebook copies (the activation fragments take the room).
    // 32 warps per SM hide the code loads for one and two groups (64 registers a thread); four
    // groups need more registers and run 16 warps.
    if (a.n_tok <= 4) { GX_TYPE_SWITCH(a.type, return (matvec_t<T, 1, kCodebookCopies, 1024>(a, sm_count, s))) }
    if (a.n_tok <= 8) { GX_TYPE_SWITCH(a.type, return (matvec_t<T, 2, kCodebookCopies, 1024>(a, sm_count, s))) }
    GX_TYPE_SWITCH(a.type, return (matvec_t<T, 4, kCodebookCopies / 2, 512>(a, sm_count, s)))
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

#ifdef GX_TRACE
// Trace readout for instrumented builds only (not part of the C ABI of include/gyro_moe.h).
extern "C" __attribute__((visibility("default"))) int gx_trace_read(long long *out, int clear) {
    if (cudaMemcpyFromSymbol(out, gx::gx_trace, sizeof(gx::gx_trace)) != cudaSuccess) return -1;
    if (clear) {
        static long long zeros[gx::kTraceKernels][gx::kTraceCtas][gx::kTracePoints] = {};
        if (cudaMemcpyToSymbol(gx::gx_trace, zeros, sizeof(zeros)) != cudaSuccess) return -1;
    }
    return 0;
}
#endif
