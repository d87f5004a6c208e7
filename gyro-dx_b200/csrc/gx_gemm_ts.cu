// gx_gemm_ts.cu — grouped GEMM of the routed experts with the decoded weights in tensor memory.
//
// D[weight row][token] = sum_k W[row][k] * X[token][k] per (token tile, weight pair) work item,
// issued as tcgen05.mma.kind::f16 with A = decoded Gyro weights in TMEM and B = the token tile in
// shared memory:
//   - the weights are decoded straight from the packed codes into registers and stored into
//     TMEM with tcgen05.st, so decoded weights never pass through shared memory (the codebook
//     lookups are the only shared-memory reads of the decoders);
//   - the MMA's N is the token count of the tile rounded up to 16, not a fixed 128;
//   - a work item covers two 128-row weight tiles against one token tile, so each token byte
//     brought in feeds 256 weight rows: gate/up = gate rows [f0, f0+128) in accumulator 0 and
//     the same up rows in accumulator 1 (silu(g) * u pairs the same TMEM lane of the two), down
//     = rows [e0, e0+256) as two tiles.
// The token tiles are the 128-row tiles pack_rows_kernel writes in its compact form
// ([tile][K/64][rows16 x 128 B], 128-byte swizzle); the outputs have moe_gemm_kernel's layout:
// act [tiles*128][F] f32 (silu(g) * u) and Y [tiles*128][E] f16.
//
// Roles (832 threads):
//   warp 0      token tiles: as many 64-wide k-steps of the tile as fit 32 KB per bulk copy
//   warp 1      TMEM allocation; the whole warp runs the issue loop, one elected lane issues the
//               MMAs (8 per k-step) and the commits
//   warps 2-17  decoders in 2 sets of 8 warps: set j decodes the CTA's k-steps n = j, j + 2, ...
//               (over its items in order); (warp - 2) / 4 % 2 picks the weight tile and warp % 4
//               the TMEM lane quarter; one thread decodes one weight row's 64 weights of a k-step
//   warps 18-25 epilogue in two groups of 4 (alternate 16-token chunks): the accumulators to act,
//               to the down operand tiles, or to Y; then the MMAs of the next item start
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>

#include "gx_device.cuh"
#include "gx_gemv.cuh"
#include "gx_internal.h"
#include "gx_umma.cuh"

namespace gx {

namespace {

constexpr int kTsSets = 2;                     // decoder sets (8 warps each: 2 tiles x 4 lane quarters)
constexpr int kTsTStages = 4;                  // token stages in shared memory (one bulk copy each)
constexpr int kTsWStages = 4;                  // decoded k-steps (both weight tiles) in TMEM
constexpr int kTsCopies = 8;
constexpr int kTsDecWarps = 8 * kTsSets;
constexpr int kTsEpiWarp = 2 + kTsDecWarps;
constexpr int kTsEpiWarps = 8;                 // two groups of 4 (one warp per TMEM lane quarter)
constexpr int kTsThreads = 32 * (kTsEpiWarp + kTsEpiWarps);
constexpr int kTsTok = 32768;                  // as many k-steps of the tile's rows as fit (>= 2)
// TMEM columns: accumulators of tiles 0 and 1 at 0 and 128 (up to 128 tokens each), weight
// stage s of tile w at 256 + 32 (2 s + w)
constexpr uint32_t kTsW = 256, kTsCols = 512;
static_assert(kTsW + 64 * kTsWStages <= kTsCols, "TMEM plan");
static_assert(kTsWStages % kTsSets == 0, "each decoder set owns the weight stages s = set (mod sets)");
static_assert((kTsTStages & (kTsTStages - 1)) == 0 && (kTsWStages & (kTsWStages - 1)) == 0, "ring sizes");

struct TsSmem {
    static constexpr int TOK = 0;                                   // per stage +kTsTok
    static constexpr int CB = kTsTStages * kTsTok;
    static constexpr int XT = CB + Codebook<kTsCopies>::BYTES;      // 2 groups x 2 x [16 tokens][128 columns] f32
    static constexpr int BARS = XT + 2 * 2 * 16 * 128 * 4;
    static constexpr int BYTES = BARS + 256;
};

__device__ __forceinline__ uint32_t tile_cols(int rows) { return rows <= 16 ? 16u : (uint32_t)((rows + 15) & ~15); }

// k-steps per token stage for a tile of `cols` rows: the largest power of two that fits kTsTok
// and divides KS (KS is even, and one k-step is at most 16 KB, so at least 2)
__device__ __forceinline__ int stage_ksteps(uint32_t cols, int KS) {
    int kps = 2;
    while (2 * kps * (int)cols * 128 <= kTsTok && KS % (2 * kps) == 0) kps *= 2;
    return kps;
}

// silu(x) = x / (1 + e^-x) with the fast exponential and division (a few ulp from the
// correctly rounded form; the operands of the products are f16)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

template <uint32_t T, int MODE>
__global__ void __launch_bounds__(kTsThreads, 1) moe_gemm_ts_kernel(GemmArgs a) {
    using CBk = Codebook<kTsCopies>;
    extern __shared__ __align__(1024) uint8_t tsm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)tsm_raw + 1023) & ~(uintptr_t)1023);
    uint32_t *cb = reinterpret_cast<uint32_t *>(sm + TsSmem::CB);
    uint64_t *full_tok = reinterpret_cast<uint64_t *>(sm + TsSmem::BARS);
    uint64_t *empty_tok = full_tok + kTsTStages;
    uint64_t *full_w = empty_tok + kTsTStages;
    uint64_t *empty_w = full_w + kTsWStages;
    uint64_t *acc_full = empty_w + kTsWStages;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *xt_full = acc_empty + 1;         // fused down packing, per group and buffer: a chunk
    uint64_t *xt_free = xt_full + 4;           // of act rows in xt / read by the group's 4 warps
    uint64_t *done = xt_free + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int TB = tile_bytes(T);
    const int NB = a.K / 128;
    const int KS = a.K / 64;
    const int n_p = MODE == 0 ? a.F / 128 : a.E / 256;   // weight pairs per token tile
    if (tid == 0) {
        for (int s = 0; s < kTsTStages; ++s) {
            mbar_init(&full_tok[s], 1);
            mbar_init(&empty_tok[s], 1);
        }
        for (int s = 0; s < kTsWStages; ++s) {
            mbar_init(&full_w[s], 8);
            mbar_init(&empty_w[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kTsEpiWarps);
        for (int b = 0; b < 4; ++b) {
            mbar_init(&xt_full[b], 4);
            mbar_init(&xt_free[b], 4);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    if (warp == 1) tmem_alloc(tmem_slot, kTsCols);
    CBk::stage(cb, a.codebook, tid, kTsThreads);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // everything above is independent of the predecessor kernels; their outputs are read below
    pdl_wait();
    const uint32_t tmem_base = *tmem_slot;
    const int n_items = *a.n_mtiles * n_p;

    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (mbar_wait(bar, parity, a.err)) return true;
        *abort_flag = 1;
        return false;
    };
    auto rows_of = [&](int t) -> int {
        const int r = a.tile_rows[t];
        return r < 0 ? 0 : (r > 128 ? 128 : r);
    };

    if (warp == 0) {
        // ---- token tiles: stage_ksteps k-steps of the tile's rows (rounded up to 16) per bulk
        // copy (compact tiles: the k-step blocks of a tile lie back to back, rows16 x 128 B each)
        if (lane == 0) {
            int m = 0;
            for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
                const int t = it / n_p;
                const uint32_t cols = tile_cols(rows_of(t)), kblock = cols * 128u;
                const int kps = stage_ksteps(cols, KS);
                const uint8_t *src = a.A + (size_t)t * KS * 16384u;
                for (int ks = 0; ks < KS; ks += kps, ++m) {
                    const int s = m & (kTsTStages - 1);
                    if (!wait(&empty_tok[s], ((m / kTsTStages) & 1) ^ 1)) break;
                    mbar_expect_tx(&full_tok[s], (uint32_t)kps * kblock);
                    bulk_g2s(sm + TsSmem::TOK + s * kTsTok, src + (size_t)ks * kblock, (uint32_t)kps * kblock, &full_tok[s]);
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: the whole warp runs the loop and takes every wait (a warp vote makes
        // each outcome uniform), one elected lane issues the MMAs (8 per k-step: 2 tiles x K =
        // 16 x 4) and the commits. With the loop state uniform across the warp an MMA issues in
        // about half the cycles it takes from a loop that only lane 0 runs.
        const bool leader = elect_one();
        {
            const uint64_t dtmpl = sw128_desc(0);
            const uint32_t tok0 = smem_u32(sm + TsSmem::TOK);
            // the fast path of a wait is one try_wait; the bounded wait only when it fails
            auto wait_q = [&](uint64_t *bar, uint32_t parity) -> bool {
                return __all_sync(0xffffffffu, mbar_try_wait(bar, parity) || wait(bar, parity));
            };
            int n = 0, m = 0, cnt = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++cnt) {
                const uint32_t cols = tile_cols(rows_of(it / n_p)), kblock = cols * 128u;
                const int kps = stage_ksteps(cols, KS);
                const uint32_t idesc = f16_idesc(128, cols);
                for (int ks0 = 0; ok && ks0 < KS; ks0 += kps, ++m) {
                    const int st = m & (kTsTStages - 1);
                    if (!wait_q(&full_tok[st], (m / kTsTStages) & 1)) { ok = false; break; }
                    // the accumulators are free once the previous item's epilogue has read them
                    if (ks0 == 0 && !wait_q(acc_empty, (cnt & 1) ^ 1)) { ok = false; break; }
                    uint32_t baddr = tok0 + (uint32_t)st * kTsTok;
                    for (int j = 0; j < kps; ++j, ++n, baddr += kblock) {
                        const int sw = n & (kTsWStages - 1);
                        if (!wait_q(&full_w[sw], (n / kTsWStages) & 1)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t bd = dtmpl | (uint64_t)((baddr >> 4) & 0x3FFFu);
                        const uint32_t at = tmem_base + kTsW + 64u * (uint32_t)sw;
                        const uint32_t acc0 = (ks0 | j) != 0;
                        if (leader) {
                            umma_f16_ts(tmem_base, at, bd, idesc, acc0);
                            umma_f16_ts(tmem_base + 128u, at + 32u, bd, idesc, acc0);
                            umma_f16_ts(tmem_base, at + 8u, bd + 2u, idesc, 1u);
                            umma_f16_ts(tmem_base + 128u, at + 40u, bd + 2u, idesc, 1u);
                            umma_f16_ts(tmem_base, at + 16u, bd + 4u, idesc, 1u);
                            umma_f16_ts(tmem_base + 128u, at + 48u, bd + 4u, idesc, 1u);
                            umma_f16_ts(tmem_base, at + 24u, bd + 6u, idesc, 1u);
                            umma_f16_ts(tmem_base + 128u, at + 56u, bd + 6u, idesc, 1u);
                        }
                        __syncwarp();
                        if (leader) umma_commit(&empty_w[sw]);
                        __syncwarp();
                    }
                    if (ok && leader) umma_commit(&empty_tok[st]);
                    __syncwarp();
                }
                if (ok && leader) umma_commit(acc_full);
                __syncwarp();
            }
            // all issued MMAs complete before TMEM is released (a commit covers the MMAs of the
            // thread that issues it)
            if (leader) {
                umma_commit(done);
                mbar_wait(done, 0, nullptr);
            }
            __syncwarp();
        }
    } else if (warp < kTsEpiWarp) {
        // ---- decoders: row i of weight tile w of the item's pair; the set's k-steps ----------
        const int set = (warp - 2) >> 3, w = ((warp - 2) >> 2) & 1, lg = warp & 3;
        const int i = 32 * lg + lane;                      // TMEM lane = row of the weight tile
        const int r8 = i & 7;                              // the row's place in its 8-row code tile
        const uint32_t lane_off = 4u * CBk::copy_off(lane);
        const uint8_t *cbb = reinterpret_cast<const uint8_t *>(cb);
        auto rowtiles_of = [&](int it) -> const uint8_t * {
            const int t = it / n_p, p = it % n_p;
            uint32_t e = (uint32_t)a.tile_expert[t];
            if (e >= (uint32_t)a.n_expert) {
                atomicExch(a.err, KERR_BOUNDS);
                e = 0;
            }
            const uint8_t *mat = MODE == 0 ? (w == 0 ? a.w0 : a.w1) : a.w0;
            const int row = MODE == 0 ? p * 128 + i : p * 256 + w * 128 + i;
            return mat + (uint64_t)e * a.expert_bytes + (size_t)(row >> 3) * NB * TB;
        };
        // Codes of one k-step (half h of a block): the two own quarters 2h, 2h+1, the neighbour
        // run of quarter (2h+3)%4 and the block scale. The next k-step of the set is fetched
        // while this one is decoded (kTsSets k-steps of the CTA ahead), across items.
        struct Codes {
            uint32_t own0[4], own1[4], nbr[4];
            uint32_t d;
        };
        int pf_cnt = 0, pf_ks = set;
        while (pf_ks >= KS) { pf_ks -= KS; ++pf_cnt; }
        int pf_rt_cnt = -1;
        const uint8_t *pf_rt = nullptr;
        auto fetch = [&](Codes &cd) -> bool {
            const int it = blockIdx.x + pf_cnt * gridDim.x;
            if (it >= n_items) return false;
            if (pf_rt_cnt != pf_cnt) {
                pf_rt_cnt = pf_cnt;
                pf_rt = rowtiles_of(it);
            }
            const int h = pf_ks & 1;
            const uint8_t *tile = pf_rt + (size_t)(pf_ks >> 1) * TB;
            load_run<T>(tile, 4 * r8 + 2 * h, cd.own0);
            load_run<T>(tile, 4 * r8 + 2 * h + 1, cd.own1);
            load_run<T>(tile, 4 * r8 + ((2 * h + 3) & 3), cd.nbr);
            cd.d = *reinterpret_cast<const uint16_t *>(tile + tile_code_bytes(T) + 2 * r8);
            pf_ks += kTsSets;
            while (pf_ks >= KS) { pf_ks -= KS; ++pf_cnt; }
            return true;
        };
        Codes cur;
        bool have = fetch(cur);
        for (int n = set; have; n += kTsSets) {
            Codes nxt;
            const bool more = fetch(nxt);
            const int s = n & (kTsWStages - 1), round = n / kTsWStages;
            const __half2 d2 = __halves2half2(__ushort_as_half((uint16_t)cur.d), __ushort_as_half((uint16_t)cur.d));
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * lg) << 16) + kTsW + 32u * (uint32_t)(2 * s + w);
            bool ok = true;
            // quarter qq of the k-step: column 16 qq + 2c holds weights 32 qq + 4c + {0, 1},
            // column 16 qq + 2c + 1 holds 32 qq + 4c + {2, 3} (the lower k in the low half)
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                uint32_t o0[8], o1[8];
                if (qq == 0) quarter_offsets<T, kTsCopies>(cur.own0, neighbour_bits<T>(cur.nbr), lane_off, o0, o1);
                else quarter_offsets<T, kTsCopies>(cur.own1, neighbour_bits<T>(cur.own0), lane_off, o0, o1);
                uint32_t v[16];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t p0 = lds_u32(cbb, o0[c]);
                    const uint32_t p1 = lds_u32(cbb, o1[c]);
                    const __half2 w0 = __hmul2(*reinterpret_cast<const __half2 *>(&p0), d2);
                    const __half2 w1 = __hmul2(*reinterpret_cast<const __half2 *>(&p1), d2);
                    v[2 * c] = *reinterpret_cast<const uint32_t *>(&w0);
                    v[2 * c + 1] = *reinterpret_cast<const uint32_t *>(&w1);
                }
                if (qq == 0) {
                    if (!wait(&empty_w[s], (round & 1) ^ 1)) { ok = false; break; }
                    tc_fence_after();
                }
                tmem_st16(taddr + 16u * qq, v);
            }
            if (!ok) break;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_w[s]);
            cur = nxt;
            have = more;
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 of both accumulators; group g
        // (4 warps) takes the 16-token chunks c with c % 2 == g ----------------------------------
        const int lg = warp & 3, eg = (warp - kTsEpiWarp) >> 2;
        float *xt = reinterpret_cast<float *>(sm + TsSmem::XT) + eg * 2 * 16 * 128;
        uint64_t *xfull = xt_full + 2 * eg, *xfree = xt_free + 2 * eg;
        int cnt = 0, ch = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++cnt) {
            const int t = it / n_p, p = it % n_p;
            const int rows = rows_of(t);
            if (!wait(acc_full, cnt & 1)) break;
            tc_fence_after();
            const uint32_t base = tmem_base + ((uint32_t)(32 * lg) << 16);
            bool ok = true;
            if (MODE == 0 && a.down_A) {
                // act = silu(g) * u of columns [128 p, 128 p + 128) for 16 tokens at a time: each
                // warp of the group puts its 32 columns (times the down signs) into xt, then each
                // takes 4 tokens: 128-point Hadamard across the warp (with signs only, as
                // pack_rows_kernel), f16, into the down operand tiles (k-steps 2p and 2p + 1 of the
                // token tile; pack_rows_kernel's compact layout)
                const int f = p * 128 + 32 * lg + lane;
                const float sgn = a.down_signs ? a.down_signs[f] : 1.f;
                const uint32_t kblock = tile_cols(rows) * 128u;
                uint8_t *tile_out = a.down_A + (size_t)t * (a.F / 64) * 16384u;
                for (int c0 = 16 * eg; c0 < rows; c0 += 32, ++ch) {
                    const int b = ch & 1;
                    uint32_t g[16], u[16];
                    tmem_ld16(base + (uint32_t)c0, g);
                    tmem_ld16(base + 128u + (uint32_t)c0, u);
                    tmem_wait_ld();
                    if (!wait(&xfree[b], ((ch >> 1) & 1) ^ 1)) { ok = false; break; }
                    float *xb = xt + b * 16 * 128;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        xb[j * 128 + 32 * lg + lane] = silu_fast(__uint_as_float(g[j])) * __uint_as_float(u[j]) * sgn;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xfull[b]);
                    if (!wait(&xfull[b], (ch >> 1) & 1)) { ok = false; break; }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int jj = 4 * lg + q;
                        const float4 x4 = *reinterpret_cast<const float4 *>(xb + jj * 128 + 4 * lane);
                        float v[4] = {x4.x, x4.y, x4.z, x4.w};
                        if (a.down_signs) fwht128_warp(v, lane);   // unrotated layers: no transform
                        if (c0 + jj < rows) {
                            const int col = 4 * lane;             // column of the 128 block
                            uint8_t *blk = tile_out + (size_t)(2 * p + (col >> 6)) * kblock;
                            uint2 o;
                            o.x = pack_half2(v[0], v[1]);
                            o.y = pack_half2(v[2], v[3]);
                            *reinterpret_cast<uint2 *>(blk + sw128_offset((uint32_t)(c0 + jj), (uint32_t)(col & 63))) = o;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xfree[b]);
                }
            } else if (MODE == 0) {
                // lane i: gate row and up row f of the pair, both in TMEM lane i
                float *dst = a.act + ((size_t)t * 128 + 16 * eg) * a.F + p * 128 + 32 * lg + lane;
                for (int c0 = 16 * eg; c0 < rows; c0 += 32) {
                    uint32_t g[16], u[16];
                    tmem_ld16(base + (uint32_t)c0, g);
                    tmem_ld16(base + 128u + (uint32_t)c0, u);
                    tmem_wait_ld();
                    const int n = min(16, rows - c0);
                    float *d0 = dst;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (j < n) *d0 = silu_fast(__uint_as_float(g[j])) * __uint_as_float(u[j]);
                        d0 += a.F;
                    }
                    dst += (size_t)32 * a.F;
                }
            } else {
                __half *dst = a.Y + ((size_t)t * 128 + 16 * eg) * a.E + p * 256 + 32 * lg + lane;
                for (int c0 = 16 * eg; c0 < rows; c0 += 32) {
                    uint32_t y0[16], y1[16];
                    tmem_ld16(base + (uint32_t)c0, y0);
                    tmem_ld16(base + 128u + (uint32_t)c0, y1);
                    tmem_wait_ld();
                    const int n = min(16, rows - c0);
                    __half *d0 = dst;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (j < n) {
                            d0[0] = __float2half_rn(__uint_as_float(y0[j]));
                            d0[128] = __float2half_rn(__uint_as_float(y1[j]));
                        }
                        d0 += a.E;
                    }
                    dst += (size_t)32 * a.E;
                }
            }
            if (!ok) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTsCols);
    }
}

template <uint32_t T, int MODE>
cudaError_t gemm_ts_t(const GemmArgs &a, int sm_count, cudaStream_t s) {
    const int smem = TsSmem::BYTES + 1024;
    static const cudaError_t once =
        cudaFuncSetAttribute(moe_gemm_ts_kernel<T, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (once != cudaSuccess) return once;
    return launch_chain(moe_gemm_ts_kernel<T, MODE>, dim3(sm_count), dim3(kTsThreads), smem, s, a);
}

}  // namespace

bool gemm_ts_routed(uint32_t type) {
    static const bool smem_b = [] {
        const char *v = std::getenv("GX_GEMM_SMEM");
        return v && v[0] == '1';
    }();
    return !smem_b && type_k(type) != 0;
}

bool gemm_ts_supports(const GemmArgs &a, int mode) {
    if (type_k(a.type) == 0 || a.K % 128 != 0) return false;
    return mode == 0 ? a.F % 128 == 0 : a.E % 256 == 0;
}

cudaError_t launch_moe_gemm_ts(const GemmArgs &a, int mode, int sm_count, cudaStream_t s) {
#define GX_TS_CASE(TT)                                                                       \
    case TT:                                                                                 \
        return mode == 0 ? gemm_ts_t<TT, 0>(a, sm_count, s) : gemm_ts_t<TT, 1>(a, sm_count, s);
    switch (a.type) {
        GX_TS_CASE(144)
        GX_TS_CASE(145)
        GX_TS_CASE(146)
        GX_TS_CASE(147)
        GX_TS_CASE(148)
        GX_TS_CASE(149)
        GX_TS_CASE(150)
        GX_TS_CASE(151)
        default:
            return cudaErrorInvalidValue;
    }
#undef GX_TS_CASE
}

}  // namespace gx
