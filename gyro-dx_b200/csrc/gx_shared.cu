// gx_shared.cu — the shared expert of a routed layer with its sigmoid gate (src/engine.zig:644-653;
// on the reference GPU: the three shared-expert mv calls and the gate mv of src/gpu_engine.zig:
// 1061-1063, :1074 and the shared term of moe_combine, shaders/engine/moe.hlsl:302-303):
//
//   out[t] += sigmoid(gate_inp . x[t]) * Down(silu(Gate x[t]) * Up x[t])
//
// x is the layer input (unrotated: the shared expert is not a Gyro tensor). The matrices are Q8_0
// (int8 weights with one fp16 scale per 32) or fp16. On the decode path (few tokens) they are
// memory-bound GEMVs on the CUDA cores, one warp per output row with all of the call's tokens
// (up to 8 at a time in registers), coalesced 8-weight loads and fp32 accumulation; the gated down
// product goes to an f32 term that the routed down kernel adds in its epilogue. Many-token calls
// use the tensor-core grouped GEMM (moe_gemm_kernel with the W_Q8 / W_F16 decoders) instead, and
// only the gate logits and the tile list come from here.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gx_dense.cuh"
#include "gx_device.cuh"
#include "gx_internal.h"

namespace gx {

using namespace dense;

namespace {

constexpr int kSharedWarps = 4;     // rows per CTA (one warp each)
constexpr int kSharedTok = 8;       // tokens held in registers at a time


// The scale the routed experts see for token t (the selection computes the same expression).
__device__ __forceinline__ float token_scale(const SharedArgs &a, int t) {
    if (a.xscale) return a.xscale[t];
    return a.norm_eps > 0.f ? 1.0f / sqrtf(a.ss[t] / (float)a.E + a.norm_eps) : 1.f;
}

// Gate logits: one warp per token (grid-stride over the calling CTA's warps).
__device__ void gate_logits(const SharedArgs &a, int warp0, int warps) {
    const int lane = threadIdx.x & 31;
    for (int t = warp0; t < a.n_tok; t += warps) {
        float s = 0.f;
        for (int c = lane * 8; c < a.E; c += 256) {
            float v[8];
            load_x8(a.x, a.x_bf16, (size_t)t * a.E + c, v);
            const float4 g0 = *reinterpret_cast<const float4 *>(a.gate_inp + c);
            const float4 g1 = *reinterpret_cast<const float4 *>(a.gate_inp + c + 4);
            s = fmaf(g0.x, v[0], s); s = fmaf(g0.y, v[1], s); s = fmaf(g0.z, v[2], s); s = fmaf(g0.w, v[3], s);
            s = fmaf(g1.x, v[4], s); s = fmaf(g1.y, v[5], s); s = fmaf(g1.z, v[6], s); s = fmaf(g1.w, v[7], s);
        }
        s = warp_sum(s);
        if (lane == 0) a.logit[t] = s * token_scale(a, t);
    }
}

// act[t][r] = silu(Gate[r] . x~[t]) * (Up[r] . x~[t]) with x~ = x * xscale; the last CTA computes
// the gate logits.
template <uint32_t WT>
__global__ void __launch_bounds__(kSharedWarps * 32) shared_gate_up_kernel(SharedArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == gridDim.x - 1) {
        gate_logits(a, warp, kSharedWarps);
        return;
    }
    const int r = blockIdx.x * kSharedWarps + warp;
    if (r >= a.SF) return;
    for (int t0 = 0; t0 < a.n_tok; t0 += kSharedTok) {
        const int nt = min(kSharedTok, a.n_tok - t0);
        float g[kSharedTok], u[kSharedTok];
#pragma unroll
        for (int t = 0; t < kSharedTok; ++t) g[t] = u[t] = 0.f;
        for (int c = lane * 8; c < a.E; c += 256) {
            float wg[8], wu[8];
            load_w8<WT>(a.gate, r, a.E, c, wg);
            load_w8<WT>(a.up, r, a.E, c, wu);
#pragma unroll
            for (int t = 0; t < kSharedTok; ++t) {
                if (t < nt) {
                    float v[8];
                    load_x8(a.x, a.x_bf16, (size_t)(t0 + t) * a.E + c, v);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        g[t] = fmaf(wg[j], v[j], g[t]);
                        u[t] = fmaf(wu[j], v[j], u[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kSharedTok; ++t) {
            if (t < nt) {
                const float sc = token_scale(a, t0 + t);
                const float gt = warp_sum(g[t]) * sc, ut = warp_sum(u[t]) * sc;
                if (lane == 0) a.act[(size_t)(t0 + t) * a.SF + r] = silu_ref(gt) * ut;
            }
        }
    }
}

// y[t][r] = sigmoid(logit[t]) * (Down[r] . act[t]).
template <uint32_t WT>
__global__ void __launch_bounds__(kSharedWarps * 32) shared_down_kernel(SharedArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * kSharedWarps + warp;
    if (r >= a.E) return;
    for (int t0 = 0; t0 < a.n_tok; t0 += kSharedTok) {
        const int nt = min(kSharedTok, a.n_tok - t0);
        float acc[kSharedTok];
#pragma unroll
        for (int t = 0; t < kSharedTok; ++t) acc[t] = 0.f;
        for (int c = lane * 8; c < a.SF; c += 256) {
            float w[8];
            load_w8<WT>(a.down, r, a.SF, c, w);
#pragma unroll
            for (int t = 0; t < kSharedTok; ++t) {
                if (t < nt) {
                    float v[8];
                    load_x8(a.act, 0, (size_t)(t0 + t) * a.SF + c, v);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[t] = fmaf(w[j], v[j], acc[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kSharedTok; ++t) {
            if (t < nt) {
                const float s = warp_sum(acc[t]);
                if (lane == 0) a.y[(size_t)(t0 + t) * a.E + r] = sigmoid_ref(a.logit[t0 + t]) * s;
            }
        }
    }
}

__global__ void __launch_bounds__(256) shared_logits_kernel(SharedArgs a) {
    gate_logits(a, blockIdx.x * 8 + (threadIdx.x >> 5), gridDim.x * 8);
}

__global__ void shared_tiles_kernel(int n_tok, int *tile_expert, int *tile_rows, int *n_mtiles) {
    const int tiles = (n_tok + 127) / 128;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < tiles; t += gridDim.x * blockDim.x) {
        tile_expert[t] = 0;
        tile_rows[t] = min(128, n_tok - 128 * t);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_mtiles = tiles;
}

bool shared_shape_ok(const SharedArgs &a) {
    return a.E > 0 && a.E % 128 == 0 && a.SF > 0 && a.SF % 128 == 0 && (a.wt == W_Q8 || a.wt == W_F16);
}

}  // namespace

cudaError_t launch_shared_gate_up(const SharedArgs &a, cudaStream_t s, bool pdl) {
    if (!shared_shape_ok(a)) return cudaErrorInvalidValue;
    if (a.n_tok == 0) return cudaSuccess;
    const int grid = (a.SF + kSharedWarps - 1) / kSharedWarps + 1;
    return a.wt == W_Q8 ? launch_pdl(shared_gate_up_kernel<W_Q8>, grid, kSharedWarps * 32, s, pdl, a)
                        : launch_pdl(shared_gate_up_kernel<W_F16>, grid, kSharedWarps * 32, s, pdl, a);
}

cudaError_t launch_shared_down(const SharedArgs &a, cudaStream_t s, bool pdl) {
    if (!shared_shape_ok(a)) return cudaErrorInvalidValue;
    if (a.n_tok == 0) return cudaSuccess;
    const int grid = (a.E + kSharedWarps - 1) / kSharedWarps;
    return a.wt == W_Q8 ? launch_pdl(shared_down_kernel<W_Q8>, grid, kSharedWarps * 32, s, pdl, a)
                        : launch_pdl(shared_down_kernel<W_F16>, grid, kSharedWarps * 32, s, pdl, a);
}

cudaError_t launch_shared_logits(const SharedArgs &a, cudaStream_t s) {
    if (a.E % 128) return cudaErrorInvalidValue;
    if (a.n_tok == 0) return cudaSuccess;
    shared_logits_kernel<<<(a.n_tok + 7) / 8, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_shared_tiles(int n_tok, int *tile_expert, int *tile_rows, int *n_mtiles, cudaStream_t s) {
    const int tiles = (n_tok + 127) / 128;
    shared_tiles_kernel<<<(tiles + 255) / 256 > 0 ? (tiles + 255) / 256 : 1, 256, 0, s>>>(n_tok, tile_expert, tile_rows,
                                                                                         n_mtiles);
    return cudaGetLastError();
}

}  // namespace gx
