// gx_tile.h — HBM tile layout of packed Gyro expert matrices and the per-lane trellis decode
// that feeds mma.sync B fragments. Host and device code: the CPU emulation in
// tests/tile_emu.cpp compiles this header with g++ to check the layout without a GPU.
//
// Format (normative, SPEC.md sections 3-6 of agention-gyro; src/gyro.zig:32-117):
//   block = fp16 scale d + stream of S steps of K new bits (TQ2_T: K=8, S=32, one byte per
//   step, state = prev byte : this byte; TQK: S=32, 16-bit window at bit (S-1-t)K of the
//   circular LSB-first stream; TQP: S=64, same window rule, one codebook pair per step).
//   hash = (state & 0x7fff) * 0x9E3779B1; idx0 = hash >> 21; idx1 = (hash >> 10) & 2047.
//
// Tile layout (this project's, chosen for the decode GEMV):
//   A matrix [R rows x C cols] becomes tiles of 8 rows x one 128-column block, ordered
//   [row group i][block b]. Tile bytes = 8 * block_bytes (no padding; always a multiple of 16):
//     codes: 8 rows x (block_bytes - 2) stream bytes, then scales: 8 fp16 (row g at 2g).
//   Lane L = 4g + q of a warp owns row g, quarter q of the block: the 32 weights
//   [32q, 32q + 32) = a run of R = (block_bytes - 2) / 4 contiguous stream bytes starting at
//   run_start(q). A run is split into parts of 8/4/2/1 bytes; part p of all 32 lanes is stored
//   together (lane L at 32 * part_offset(p) + L * part_size(p)), so every part load of a
//   warp is one coalesced access. The bits a lane needs beyond its run (TQ2_T: the byte
//   before it; TQK/TQP: the first 16-K bits after it, circularly) sit in the run of quarter
//   (q + 3) % 4 of the same row, which the lane fetches with one warp shuffle.
//
// K permutation for mma.m16n8k16 (row.col, f16 inputs, f32 accumulate): chunk c (0..7) of
// a block gives lane (g, q) the B registers
//     b0 = codebook pair for weights 32q + 4c + {0, 1} of row g (k = 2q, 2q+1)
//     b1 = codebook pair for weights 32q + 4c + {2, 3} of row g (k = 2q+8, 2q+9)
// so A must hold x[32q + 4c + {0,1}] at k = 2q, 2q+1 and x[32q + 4c + {2,3}] at k = 2q+8, 2q+9.
// For S=32 types chunk c is step 8q + c (pairs 0 and 1); for S=64 types it is steps
// 16q + 2c and 16q + 2c + 1 (pair 0 of each).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define GX_HD __host__ __device__ __forceinline__
#else
#define GX_HD inline
#endif

namespace gx {

enum : uint32_t {
    T_TQ2_T = 144, T_TQK6 = 145, T_TQK7 = 146, T_TQP5 = 147,
    T_TQP6 = 148, T_TQP7 = 149, T_TQK5 = 150, T_TQK4 = 151
};

GX_HD constexpr int type_k(uint32_t t) {
    return t == 144 ? 8 : t == 145 ? 6 : t == 146 ? 7 : t == 147 ? 5 : t == 148 ? 6 :
           t == 149 ? 7 : t == 150 ? 5 : t == 151 ? 4 : 0;
}
GX_HD constexpr int type_steps(uint32_t t) { return (t >= 147 && t <= 149) ? 64 : 32; }
GX_HD constexpr int type_block_bytes(uint32_t t) { return type_k(t) ? 2 + type_steps(t) * type_k(t) / 8 : 0; }
GX_HD constexpr int run_bytes(uint32_t t) { return (type_block_bytes(t) - 2) / 4; }
GX_HD constexpr int tile_bytes(uint32_t t) { return 8 * type_block_bytes(t); }
GX_HD constexpr int tile_code_bytes(uint32_t t) { return 8 * (type_block_bytes(t) - 2); }

// Greedy split of a run into 8/4/2/1-byte parts.
GX_HD constexpr int part_size(int run, int p) {
    int off = 0;
    for (int i = 0; i < p; ++i) {
        int rem = run - off;
        off += rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : rem;
    }
    int rem = run - off;
    return rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : rem;
}
GX_HD constexpr int part_offset(int run, int p) {
    int off = 0;
    for (int i = 0; i < p; ++i) off += part_size(run, i);
    return off;
}
GX_HD constexpr int part_count(int run) {
    int n = 0, off = 0;
    while (off < run) { off += part_size(run, n); ++n; }
    return n;
}

// First stream byte of quarter q's run.
GX_HD constexpr int run_start(uint32_t t, int q) {
    return t == 144 ? 8 * q : (3 - q) * run_bytes(t);
}

// Portable byte permute / funnel shift (host emulation of the PTX prmt / shf.r).
GX_HD uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t s) {
#if defined(__CUDA_ARCH__)
    return __byte_perm(a, b, s);
#else
    uint64_t v = ((uint64_t)b << 32) | a;
    uint32_t r = 0;
    for (int i = 0; i < 4; ++i) {
        uint32_t sel = (s >> (4 * i)) & 7;
        r |= (uint32_t)((v >> (8 * sel)) & 0xff) << (8 * i);
    }
    return r;
#endif
}
GX_HD uint32_t funnel_r(uint32_t lo, uint32_t hi, uint32_t sh) {
#if defined(__CUDA_ARCH__)
    return __funnelshift_r(lo, hi, sh);
#else
    sh &= 31;
    return sh ? (lo >> sh) | (hi << (32 - sh)) : lo;
#endif
}

GX_HD uint32_t hash_state(uint32_t s) { return (s & 0x7fffu) * 0x9e3779b1u; }

// Codebook indices of the 8 chunks of one lane's quarter.
//   own[0..3]: the lane's run bytes, little-endian (run byte j in own[j/4] bits 8(j%4)..)
//   nb:        TQ2_T: the neighbour run's last byte in bits 0..7;
//              TQK/TQP: the neighbour run's first two bytes in bits 0..15.
// i0[c] feeds b0 (k = 2q, 2q+1), i1[c] feeds b1 (k = 2q+8, 2q+9).
template <uint32_t T>
GX_HD void quarter_indices(const uint32_t own[4], uint32_t nb, uint32_t i0[8], uint32_t i1[8]) {
    if constexpr (T == T_TQ2_T) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            uint32_t s;
            if (c == 0) s = byte_perm(own[0], nb, 0x40u);
            else if (c < 4) s = byte_perm(own[0], 0u, (uint32_t)(c | ((c - 1) << 4)));
            else if (c == 4) s = byte_perm(own[1], own[0], 0x70u);
            else s = byte_perm(own[1], 0u, (uint32_t)((c - 4) | ((c - 5) << 4)));
            uint32_t h = hash_state(s);
            i0[c] = h >> 21;
            i1[c] = (h >> 10) & 2047u;
        }
    } else {
        constexpr int K = type_k(T);
        constexpr int S = type_steps(T);
        constexpr int R = run_bytes(T);
        // Bit string: run bytes [0, R) then the neighbour's two bytes.
        uint32_t w[5] = {own[0], own[1], own[2], own[3], 0u};
        constexpr int wi = R / 4, sh = 8 * (R % 4);
        w[wi] |= nb << sh;
        if constexpr (sh > 16) w[wi + 1] |= nb >> (32 - sh);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if constexpr (S == 32) {
                constexpr int dummy = 0; (void)dummy;
                const int o = (7 - c) * K;
                uint32_t s = funnel_r(w[o >> 5], w[(o >> 5) + 1], (uint32_t)(o & 31));
                uint32_t h = hash_state(s);
                i0[c] = h >> 21;
                i1[c] = (h >> 10) & 2047u;
            } else {
                const int o0 = (15 - 2 * c) * K, o1 = (14 - 2 * c) * K;
                uint32_t s0 = funnel_r(w[o0 >> 5], w[(o0 >> 5) + 1], (uint32_t)(o0 & 31));
                uint32_t s1 = funnel_r(w[o1 >> 5], w[(o1 >> 5) + 1], (uint32_t)(o1 & 31));
                i0[c] = hash_state(s0) >> 21;
                i1[c] = hash_state(s1) >> 21;
            }
        }
    }
}

// Neighbour bits a lane takes from the run of quarter (q + 3) % 4 (see quarter_indices).
template <uint32_t T>
GX_HD uint32_t neighbour_bits(const uint32_t nbr_own[4]) {
    if constexpr (T == T_TQ2_T) return nbr_own[1] >> 24;
    else return nbr_own[0] & 0xffffu;
}

// Byte offset of part p of lane L inside a tile's code region.
template <uint32_t T>
GX_HD constexpr int part_lane_offset(int p, int lane) {
    return 32 * part_offset(run_bytes(T), p) + lane * part_size(run_bytes(T), p);
}

// Writes lane L's run (row L/4, quarter L%4) of one reference-layout block (scale + stream)
// into a tile, and the row's scale when L%4 == 0. Used by the upload repack kernel and by
// the CPU emulation.
GX_HD void repack_lane(uint32_t t, const uint8_t *block, uint8_t *tile, int lane) {
    const int R = run_bytes(t), q = lane & 3, g = lane >> 2;
    const uint8_t *run = block + 2 + run_start(t, q);
    const int np = part_count(R);
    for (int p = 0; p < np; ++p) {
        const int sz = part_size(R, p), off = part_offset(R, p);
        uint8_t *dst = tile + 32 * off + lane * sz;
        for (int j = 0; j < sz; ++j) dst[j] = run[off + j];
    }
    if (q == 0) {
        tile[tile_code_bytes(t) + 2 * g] = block[0];
        tile[tile_code_bytes(t) + 2 * g + 1] = block[1];
    }
}

// Reads lane L's run from a tile (shared or global memory) into own[] (little-endian).
template <uint32_t T>
GX_HD void load_run(const uint8_t *tile, int lane, uint32_t own[4]) {
    constexpr int R = run_bytes(T);
    constexpr int NP = part_count(R);
    own[0] = own[1] = own[2] = own[3] = 0u;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int sz = part_size(R, p), off = part_offset(R, p);
        const uint8_t *src = tile + 32 * off + lane * sz;
        if (sz == 8) {
#if defined(__CUDA_ARCH__)
            const uint2 v = *reinterpret_cast<const uint2 *>(src);
            own[off / 4] = v.x;
            own[off / 4 + 1] = v.y;
#else
            uint32_t v[2];
            for (int j = 0; j < 2; ++j)
                v[j] = (uint32_t)src[4 * j] | ((uint32_t)src[4 * j + 1] << 8) |
                       ((uint32_t)src[4 * j + 2] << 16) | ((uint32_t)src[4 * j + 3] << 24);
            own[off / 4] = v[0];
            own[off / 4 + 1] = v[1];
#endif
        } else if (sz == 4) {
#if defined(__CUDA_ARCH__)
            own[off / 4] |= *reinterpret_cast<const uint32_t *>(src);
#else
            own[off / 4] |= (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) |
                            ((uint32_t)src[3] << 24);
#endif
        } else if (sz == 2) {
#if defined(__CUDA_ARCH__)
            own[off / 4] |= (uint32_t)(*reinterpret_cast<const uint16_t *>(src)) << (8 * (off % 4));
#else
            own[off / 4] |= ((uint32_t)src[0] | ((uint32_t)src[1] << 8)) << (8 * (off % 4));
#endif
        } else {
            own[off / 4] |= (uint32_t)src[0] << (8 * (off % 4));
        }
    }
}

}  // namespace gx
