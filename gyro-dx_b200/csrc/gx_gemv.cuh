// gx_gemv.cuh — the decode-GEMV building blocks shared by the per-phase kernels (gx_kernels.cu)
// and the persistent decode-stack kernel (gx_decode_stack.cu): the tile product on mma.sync
// with in-register trellis decode, activation fragments, and the staged bulk-copy pipeline.
#pragma once
#include <cuda_runtime.h>

#include "gx_device.cuh"

namespace gx {

// One 8-row x 128-column tile against NG groups of 8 tokens. acc[g][0..1] accumulates, for
// token (8g + lane/4), rows 2*(lane%4) and 2*(lane%4)+1 of the tile (scaled by d).
template <uint32_t T, int NG, int NC>
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
        b0[c] = cb[Codebook<NC>::word(i0[c], copy_off)];
        b1[c] = cb[Codebook<NC>::word(i1[c], copy_off)];
    }
    // Two independent accumulator chains (even / odd chunks) halve the mma dependency chain.
    float d[2][NG][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int g = 0; g < NG; ++g) d[h][g][0] = d[h][g][1] = d[h][g][2] = d[h][g][3] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int g = 0; g < NG; ++g) mma16816(d[c & 1][g], A[g][c], b0[c], b1[c]);
    const uint32_t sc = *reinterpret_cast<const uint32_t *>(tile + tile_code_bytes(T) + 4 * (lane & 3));
    const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&sc));
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        acc[g][0] += s.x * ((d[0][g][0] + d[1][g][0]) + (d[0][g][2] + d[1][g][2]));
        acc[g][1] += s.y * ((d[0][g][1] + d[1][g][1]) + (d[0][g][3] + d[1][g][3]));
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
__device__ __forceinline__ void rotated_block_to_smem(const void *src, int bf16, size_t base, float scale,
                                                      const float *signs, int sbase, float *xs, int lane) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = load_act(src, bf16, base + 4 * lane + j) * scale;
        if (signs) v[j] *= signs[sbase + 4 * lane + j];
    }
    if (signs) fwht128_warp(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) xs[4 * lane + j] = v[j];
    __syncwarp();
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

// Waits for the bulk-staged codebook (barrier cb_bar, phase 0). On an expired wait every thread
// sees false; the stage copies this CTA issued (up to two) and the codebook copy get one more
// bounded wait before the CTA returns.
__device__ __forceinline__ bool codebook_wait(uint64_t *cb_bar, const StageCtl &c, int *err) {
    const bool ok = mbar_wait(cb_bar, 0u, err);
    if (__syncthreads_and(ok)) return true;
    if (threadIdx.x == 0) {
        mbar_wait(cb_bar, 0u, nullptr);
        for (int t = 0; t < 2 && t < c.n_stages; ++t) mbar_wait(&c.bar[t & 1], 0u, nullptr);
    }
    __syncthreads();
    return false;
}

}  // namespace gx
