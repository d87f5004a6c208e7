// CPU emulation of one warp of the decode GEMV: repack a reference-layout 8-row slab into the
// HBM tile layout, read each lane's run back, decode the trellis indices, and multiply the
// resulting mma.m16n8k16 B fragments with the matching A fragments of up to 8 tokens (fp16
// hi/lo split, rows 0-7 hi and 8-15 lo). Compiled by tests/test_tile_layout.py with g++; it
// exercises gyro-dx_b200/csrc/gx_tile.h exactly as the kernels use it.
#include <cstdint>
#include <cstring>
#include <vector>

#include "../gyro-dx_b200/csrc/gx_tile.h"

static double h2d(uint16_t h) {
    const uint32_t s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
    double v;
    if (e == 0) v = m * (1.0 / 16777216.0);
    else if (e == 31) v = m ? 0.0 / 0.0 : 1.0 / 0.0;
    else v = (1.0 + m / 1024.0) * ((e >= 15) ? (double)(1u << (e - 15)) : 1.0 / (double)(1u << (15 - e)));
    return s ? -v : v;
}

template <uint32_t T>
static void run(int NB, const uint8_t *raw, const uint16_t *xhi, const uint16_t *xlo, int ntok,
                const uint16_t *cb, double *out, uint8_t *tiles_out) {
    constexpr int BB = gx::type_block_bytes(T);
    constexpr int TB = gx::tile_bytes(T);
    const int C = NB * 128;
    std::vector<uint8_t> tiles((size_t)NB * TB, 0xEE);
    for (int b = 0; b < NB; ++b)
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2;
            gx::repack_lane(T, raw + (size_t)g * NB * BB + (size_t)b * BB, tiles.data() + (size_t)b * TB, lane);
        }
    if (tiles_out) std::memcpy(tiles_out, tiles.data(), tiles.size());
    for (int i = 0; i < ntok * 8; ++i) out[i] = 0;
    for (int b = 0; b < NB; ++b) {
        const uint8_t *tile = tiles.data() + (size_t)b * TB;
        uint32_t own[32][4];
        for (int lane = 0; lane < 32; ++lane) gx::load_run<T>(tile, lane, own[lane]);
        uint32_t i0[32][8], i1[32][8];
        for (int lane = 0; lane < 32; ++lane) {
            const int nbr = (lane & ~3) | ((lane + 3) & 3);
            gx::quarter_indices<T>(own[lane], gx::neighbour_bits<T>(own[nbr]), i0[lane], i1[lane]);
        }
        double D[16][8] = {};
        for (int c = 0; c < 8; ++c) {
            double A[16][16] = {}, B[16][8] = {};
            for (int lane = 0; lane < 32; ++lane) {
                const int g = lane >> 2, q = lane & 3;
                B[2 * q][g] = h2d(cb[2 * i0[lane][c]]);
                B[2 * q + 1][g] = h2d(cb[2 * i0[lane][c] + 1]);
                B[2 * q + 8][g] = h2d(cb[2 * i1[lane][c]]);
                B[2 * q + 9][g] = h2d(cb[2 * i1[lane][c] + 1]);
                if (g < ntok) {
                    const int base = g * C + b * 128 + 32 * q + 4 * c;
                    A[g][2 * q] = h2d(xhi[base]);
                    A[g][2 * q + 1] = h2d(xhi[base + 1]);
                    A[g][2 * q + 8] = h2d(xhi[base + 2]);
                    A[g][2 * q + 9] = h2d(xhi[base + 3]);
                    A[g + 8][2 * q] = h2d(xlo[base]);
                    A[g + 8][2 * q + 1] = h2d(xlo[base + 1]);
                    A[g + 8][2 * q + 8] = h2d(xlo[base + 2]);
                    A[g + 8][2 * q + 9] = h2d(xlo[base + 3]);
                }
            }
            for (int m = 0; m < 16; ++m)
                for (int n = 0; n < 8; ++n)
                    for (int k = 0; k < 16; ++k) D[m][n] += A[m][k] * B[k][n];
        }
        for (int t = 0; t < ntok; ++t)
            for (int n = 0; n < 8; ++n) {
                const uint8_t *sc = tile + gx::tile_code_bytes(T) + 2 * n;
                const double d = h2d((uint16_t)(sc[0] | (sc[1] << 8)));
                out[t * 8 + n] += d * (D[t][n] + D[t + 8][n]);
            }
    }
}

extern "C" int emu_tile_gemv(uint32_t type, int NB, const uint8_t *raw, const uint16_t *xhi,
                             const uint16_t *xlo, int ntok, const uint16_t *cb, double *out,
                             uint8_t *tiles_out) {
    switch (type) {
        case 144: run<144>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 145: run<145>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 146: run<146>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 147: run<147>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 148: run<148>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 149: run<149>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 150: run<150>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        case 151: run<151>(NB, raw, xhi, xlo, ntok, cb, out, tiles_out); return 0;
        default: return -1;
    }
}

extern "C" int emu_tile_bytes(uint32_t type) {
    return gx::tile_bytes(type);
}
