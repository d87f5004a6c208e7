// gx_gemv.cuh — the decode-GEMV building blocks shared by the per-phase kernels (gx_kernels.cu)
// and the persistent decode-stack kernel (gx_decode_stack.cu): the tile product on mma.sync
// with in-register trellis decode, activation fragments, and the staged bulk-copy pipeline.
#pragma once
#include <cuda_runtime.h>

#include "gx_device.cuh"

namespace gx {

// ---- codebook lookups by byte offset -------------------------------------------------------
// prmt.b32 in its default mode: a selector nibble with bit 3 set replicates the sign bit of the
// chosen byte, which yields a zero byte from a byte below 0x80.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Byte offsets into a Codebook<NC> array of the two codebook pairs of each of the 8 chunks of a
// lane's quarter (the values quarter_indices computes, as offsets): o0[c] for weights
// 32q + 4c + {0,1}, o1[c] for 32q + 4c + {2,3}. lane_off = 4 * (the lane's copy). The index of a
// pair times 4 * NC is taken straight from the hash by one shift and one masked OR (the copy
// offset lies below the index bits), so a lookup costs two integer operations and the load.
// TQ2_T builds each 15-bit state with one prmt from the run and a copy whose bytes have bit 7
// cleared (the previous byte's high bit is not part of the state, the sign bytes are zero).
template <uint32_t T, int NC>
__device__ __forceinline__ void quarter_offsets(const uint32_t own[4], uint32_t nb, uint32_t lane_off, uint32_t (&o0)[8],
                                                uint32_t (&o1)[8]) {
    constexpr int SH = NC == 16 ? 6 : NC == 8 ? 5 : NC == 4 ? 4 : -1;
    static_assert(SH > 0, "codebook copies: 4, 8 or 16");
    constexpr uint32_t M = 2047u << SH;
    auto offsets = [&](uint32_t s15, uint32_t &a, uint32_t &b) {
        const uint32_t h = s15 * 0x9e3779b1u;
        a = ((h >> (21 - SH)) & M) | lane_off;
        b = ((h >> (10 - SH)) & M) | lane_off;
    };
    if constexpr (T == T_TQ2_T) {
        const uint32_t m0 = own[0] & 0x7f7f7f7fu, m1 = own[1] & 0x7f7f7f7fu, mn = nb & 0x7fu;
        // step c: this byte (low) and the byte before it (high, bit 7 cleared), upper bytes zero
        offsets(prmt(own[0], mn, 0x5540u), o0[0], o1[0]);
        offsets(prmt(own[0], m0, 0xcc41u), o0[1], o1[1]);
        offsets(prmt(own[0], m0, 0xdd52u), o0[2], o1[2]);
        offsets(prmt(own[0], m0, 0xee63u), o0[3], o1[3]);
        offsets(prmt(own[1], m0, 0xff70u), o0[4], o1[4]);
        offsets(prmt(own[1], m1, 0xcc41u), o0[5], o1[5]);
        offsets(prmt(own[1], m1, 0xdd52u), o0[6], o1[6]);
        offsets(prmt(own[1], m1, 0xee63u), o0[7], o1[7]);
    } else {
        uint32_t i0[8], i1[8];
        quarter_indices<T>(own, nb, i0, i1);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            o0[c] = (i0[c] << SH) | lane_off;
            o1[c] = (i1[c] << SH) | lane_off;
        }
    }
}

__device__ __forceinline__ uint32_t lds_u32(const uint8_t *base, uint32_t off) {
    return *reinterpret_cast<const uint32_t *>(base + off);
}

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
    uint32_t o0[8], o1[8];
    quarter_offsets<T, NC>(own, nb, 4u * copy_off, o0, o1);
    const uint8_t *cbb = reinterpret_cast<const uint8_t *>(cb);
    uint32_t b0[8], b1[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        b0[c] = lds_u32(cbb, o0[c]);
        b1[c] = lds_u32(cbb, o1[c]);
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
