// gx_prefill.cu — the many-token (prefill) path of the routed layer on sm_100a tensor cores.
//
//   router_gemm_kernel   logits = X W_r^T in fp32 on CUDA cores (tiled SGEMM), raw (before the
//                        RMSNorm scale and bias, which the selection applies)
//   group_kernel         count / prefix / stable fill of slots by expert (src/engine.zig:553-564),
//                        expert segments padded to 128-row tiles
//   pack_rows_kernel     gathers token rows per tile, applies scale, signs and the 128-point
//                        Hadamard transform, writes f16 operand tiles in the 128-byte-swizzled
//                        K-major layout the tensor core reads
//   moe_gemm_kernel      grouped GEMM per (expert row tile, weight column tile): decoder warps
//                        expand Gyro trellis codes into f16 B tiles in shared memory, one thread
//                        issues tcgen05.mma into a TMEM accumulator, epilogue warps read TMEM:
//                        gate/up -> SwiGLU, down -> f16 rows
//   combine_kernel       weighted un-permute of the down rows (src/engine.zig:634-641) + residual
//
// f16 is used for both operands: every codebook value is exact in f16, d * CB is rounded once
// (2^-11 relative), activations keep 11 mantissa bits; accumulation is f32 in TMEM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gx_device.cuh"
#include "gx_gemv.cuh"
#include "gx_internal.h"
#include "gx_umma.cuh"

namespace gx {

// ------------------------------------------------------------------------------------------
// Router GEMM: C[z][t][e] = sum over the z-th K slice of X[t][c] W[e][c] (split-K partials,
// summed in a fixed order by the selection). CTA tile 64 tokens x 32 experts, 256 threads, each
// 4 tokens x 2 experts, K chunks of 32 staged in shared memory with the next chunk prefetched.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) router_gemm_kernel(const float *__restrict__ W, const void *__restrict__ x,
                                                          int x_bf16, int n_tok, int NE, int E, float *__restrict__ C) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ __align__(16) float xs[32][64 + 4];
    __shared__ __align__(16) float ws[32][32 + 4];
    const int t0 = blockIdx.y * 64, e0 = blockIdx.x * 32;
    const int ksplit = E / gridDim.z, kbeg = blockIdx.z * ksplit, kend = kbeg + ksplit;
    C += (size_t)blockIdx.z * n_tok * NE;
    const int tid = threadIdx.x;
    const int tt = (tid & 15) * 4, ee = (tid >> 4) * 2;
    // loader mapping: x tile 64 x 32 -> 8 values per thread (rows lr + 8j, column lc);
    // w tile 32 x 32 -> 4 values per thread (rows lr + 8j)
    const int lc = tid & 31, lr = tid >> 5;
    float xr[8], wr[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int t = t0 + lr + 8 * j;
            xr[j] = t < n_tok ? load_act(x, x_bf16, (size_t)t * E + k0 + lc) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + lr + 8 * j;
            wr[j] = e < NE ? __ldg(W + (size_t)e * E + k0 + lc) : 0.f;
        }
    };
    float acc[4][2] = {};
    load(kbeg);
    for (int k0 = kbeg; k0 < kend; k0 += 32) {
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[lc][lr + 8 * j] = xr[j];
#pragma unroll
        for (int j = 0; j < 4; ++j) ws[lc][lr + 8 * j] = wr[j];
        __syncthreads();
        if (k0 + 32 < kend) load(k0 + 32);   // next chunk in flight while this one is consumed
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[k][tt]);
            const float2 wv = *reinterpret_cast<const float2 *>(&ws[k][ee]);
            acc[0][0] = fmaf(xv.x, wv.x, acc[0][0]); acc[0][1] = fmaf(xv.x, wv.y, acc[0][1]);
            acc[1][0] = fmaf(xv.y, wv.x, acc[1][0]); acc[1][1] = fmaf(xv.y, wv.y, acc[1][1]);
            acc[2][0] = fmaf(xv.z, wv.x, acc[2][0]); acc[2][1] = fmaf(xv.z, wv.y, acc[2][1]);
            acc[3][0] = fmaf(xv.w, wv.x, acc[3][0]); acc[3][1] = fmaf(xv.w, wv.y, acc[3][1]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int t = t0 + tt + i, e = e0 + ee + j;
            if (t < n_tok && e < NE) C[(size_t)t * NE + e] = acc[i][j];
        }
}

// ------------------------------------------------------------------------------------------
// Grouping (the counting sort of src/engine.zig:553-564 without its stable order, which no
// result depends on: every output row is computed from its own input row). Three kernels:
//   count  per-expert slot counts (warp-aggregated atomics)
//   scan   one CTA: 128-row tiles per expert, tile list, each expert's first row; it leaves
//          the counts at zero for the next grouping (they start at zero when allocated)
//   place  each slot takes the next row of its expert (warp-aggregated atomics)
// Slots whose id is kNoSlot (expert-parallel rows carry them for experts of other ranks) get no
// row; any other id outside [0, NE) is reported as KERR_BOUNDS.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) group_count_kernel(GroupArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int s = blockIdx.x * 1024 + threadIdx.x;
    const bool live = s < a.n_slots;
    const uint32_t e = live ? a.ids[s] : kNoSlot;
    const bool ok = live && e < (uint32_t)a.NE;
    if (live && !ok && e != kNoSlot) atomicExch(a.err, KERR_BOUNDS);
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : 0xffffffffu);
    if (ok && __ffs(peers) - 1 == (int)(threadIdx.x & 31)) atomicAdd(&a.expert_count[e], __popc(peers));
}

__global__ void __launch_bounds__(512) group_scan_kernel(GroupArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int wsum[16];
    const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
    const int cnt = e < a.NE ? a.expert_count[e] : 0;
    if (e < a.NE) a.expert_count[e] = 0;       // zero again for the next grouping (no memset node)
    const int nt = (cnt + 127) / 128;
    int incl = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    const int base = before + incl - nt;  // exclusive prefix of tiles
    if (e < a.NE) {
        for (int m = 0; m < nt; ++m) {
            a.tile_expert[base + m] = e;
            a.tile_rows[base + m] = min(128, cnt - m * 128);
        }
        a.cursor[e] = base * 128;
    }
    if (e == 511) *a.n_mtiles = before + incl;
}

__global__ void __launch_bounds__(1024) group_place_kernel(GroupArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int s = blockIdx.x * 1024 + threadIdx.x, lane = threadIdx.x & 31;
    const bool live = s < a.n_slots;
    const uint32_t e = live ? a.ids[s] : kNoSlot;
    const bool ok = live && e < (uint32_t)a.NE;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : 0xffffffffu);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (ok && lane == leader) base = atomicAdd(&a.cursor[e], __popc(peers));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (ok) {
        const int row = base + __popc(peers & ((1u << lane) - 1u));
        a.row_slot[row] = s;
        a.slot_row[s] = row;
    } else if (live) {
        a.slot_row[s] = -1;
    }
}

// ------------------------------------------------------------------------------------------
// Token rotation, once per token: xh[t] = f16(H128((x[t] * scale[t]) * signs) / sqrt(128)) per
// 128-column block (src/engine.zig:547-551), one warp per (token, 4 blocks). With scatter, the
// row goes instead to rows scatter[t][0..n_dst) of xh that are >= 0 (the expert-parallel send
// buffer: one copy per destination rank that serves one of the token's experts).
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rotate_tokens_kernel(const void *x, int x_bf16, const float *xscale,
                                                            const float *signs, int n_tok, int E, __half *xh,
                                                            const int *scatter, int n_dst) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int nb = E / 128, groups = (nb + 3) / 4;
    if (w >= (long long)n_tok * groups) return;
    const int t = (int)(w / groups), b0 = (int)(w % groups) * 4;
    const float sc = xscale ? xscale[t] : 1.f;
    float v[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int b = b0 + q;
        if (b >= nb) break;
        const size_t base = (size_t)t * E + b * 128 + 4 * lane;
#pragma unroll
        for (int j = 0; j < 4; ++j) v[q][j] = load_act(x, x_bf16, base + j) * sc;
        if (signs) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[q][j] *= signs[b * 128 + 4 * lane + j];
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int b = b0 + q;
        if (b >= nb) break;
        if (signs) fwht128_warp(v[q], lane);
        uint2 o;
        o.x = pack_half2(v[q][0], v[q][1]);
        o.y = pack_half2(v[q][2], v[q][3]);
        if (!scatter) {
            *reinterpret_cast<uint2 *>(xh + (size_t)t * E + b * 128 + 4 * lane) = o;
            continue;
        }
        for (int d = 0; d < n_dst; ++d) {
            const int row = scatter[(size_t)t * n_dst + d];
            if (row >= 0) *reinterpret_cast<uint2 *>(xh + (size_t)row * E + b * 128 + 4 * lane) = o;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Rotation and packing in one pass (the single-GPU many-token path): one warp per (token, 4
// blocks) rotates as rotate_tokens_kernel does and stores the f16 row into the tile row of each
// of the token's slots, in the layout pack_rows_kernel writes. The rows a tile has past its
// tokens are not written: the MMA columns they feed are never stored.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rotate_pack_kernel(RotPackArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int nb = a.E / 128, groups = (nb + 3) / 4;
    if (w >= (long long)a.n_tok * groups) return;
    const int t = (int)(w / groups), b0 = (int)(w % groups) * 4;
    const float sc = a.xscale ? a.xscale[t] : 1.f;
    uint2 o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int b = b0 + q;
        if (b >= nb) break;
        const size_t base = (size_t)t * a.E + b * 128 + 4 * lane;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = load_act(a.x, a.x_bf16, base + j) * sc;
        if (a.signs) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] *= a.signs[b * 128 + 4 * lane + j];
            fwht128_warp(v, lane);
        }
        o[q].x = pack_half2(v[0], v[1]);
        o[q].y = pack_half2(v[2], v[3]);
    }
    const int ks_lo = lane >> 4, col = 4 * (lane & 15);
    for (int k = 0; k < a.U; ++k) {
        const int row = a.slot_row[(size_t)t * a.U + k];
        if (row < 0) continue;
        const int tile = row >> 7, i = row & 127;
        const int rows_t = a.tile_rows[tile];
        const int np = a.compact ? (rows_t <= 16 ? 16 : (rows_t + 15) & ~15) : 128;
        uint8_t *base = a.dst + (size_t)tile * (a.E / 64) * 16384u;
        const size_t kblock = (size_t)np * 128u;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int b = b0 + q;
            if (b >= nb) break;
            *reinterpret_cast<uint2 *>(base + (size_t)(2 * b + ks_lo) * kblock + sw128_offset((uint32_t)i, (uint32_t)col)) =
                o[q];
        }
    }
}

// ------------------------------------------------------------------------------------------
// Row packing: one warp per padded row. Source row = token of the slot (gate/up input, x) or
// the padded row itself (down input, act). v = src * scale, * signs, then H128 / sqrt(128) per
// 128-column block when signs are given; f16 into the swizzled K-major tile layout
// [tile][K/64][128 rows x 64 cols]. Four blocks' loads are in flight at a time.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pack_rows_kernel(PackArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int nb = a.K / 128;
    if (row >= (long long)*a.n_mtiles * 128) return;
    const int t = (int)(row >> 7), i = (int)(row & 127);
    const int rows_t = a.tile_rows[t];
    const bool valid = i < rows_t;
    // compact tiles keep rows16(rows) rows per k-step block; the rows past that are not stored
    const int np = a.compact ? (rows_t <= 16 ? 16 : (rows_t + 15) & ~15) : 128;
    if (i >= np) return;
    uint8_t *tile_base = a.dst + (size_t)t * (a.K / 64) * 16384u;
    const size_t kblock = (size_t)np * 128u;
    size_t src_row = (size_t)row;
    float sc = 1.f;
    if (valid && a.by_token) {
        const int tok = a.row_slot[row] / a.U;
        src_row = (size_t)tok;
        if (a.xscale) sc = a.xscale[tok];
    } else if (valid && a.xscale) {
        sc = a.xscale[row];
    }
    const int ks_lo = lane >> 4, col = 4 * (lane & 15);
    if (a.by_token) {
        // gate/up input: copy the token's rotated f16 row (rotate_tokens_kernel) into the tile
        const __half *xr = a.xh + src_row * a.K;
        for (int b = 0; b < nb; ++b) {
            uint2 w = make_uint2(0u, 0u);
            if (valid) w = *reinterpret_cast<const uint2 *>(xr + b * 128 + 4 * lane);
            uint8_t *tile = tile_base + (size_t)(2 * b + ks_lo) * kblock;
            *reinterpret_cast<uint2 *>(tile + sw128_offset((uint32_t)i, (uint32_t)col)) = w;
        }
        return;
    }
    for (int b0 = 0; b0 < nb; b0 += 4) {
        float v[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int b = b0 + q;
            if (valid && b < nb) {
                const size_t base = src_row * a.K + b * 128 + 4 * lane;
                if (a.src_bf16) {
                    const uint2 w = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(a.src) + base);
                    v[q][0] = __uint_as_float(w.x << 16);
                    v[q][1] = __uint_as_float(w.x & 0xffff0000u);
                    v[q][2] = __uint_as_float(w.y << 16);
                    v[q][3] = __uint_as_float(w.y & 0xffff0000u);
                } else {
                    const float4 w = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.src) + base);
                    v[q][0] = w.x; v[q][1] = w.y; v[q][2] = w.z; v[q][3] = w.w;
                }
                if (a.signs) {
                    const float4 g = *reinterpret_cast<const float4 *>(a.signs + b * 128 + 4 * lane);
                    v[q][0] *= g.x * sc; v[q][1] *= g.y * sc; v[q][2] *= g.z * sc; v[q][3] *= g.w * sc;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[q][j] *= sc;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[q][j] = 0.f;
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int b = b0 + q;
            if (b >= nb) break;
            if (a.signs) fwht128_warp(v[q], lane);
            uint8_t *tile = tile_base + (size_t)(2 * b + ks_lo) * kblock;
            uint2 w;
            w.x = pack_half2(v[q][0], v[q][1]);
            w.y = pack_half2(v[q][2], v[q][3]);
            *reinterpret_cast<uint2 *>(tile + sw128_offset((uint32_t)i, (uint32_t)col)) = w;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Grouped GEMM on tcgen05. 448 threads: warp 0 loads A tiles (bulk copies), warp 1 owns TMEM
// and issues the MMAs, warps 2-9 decode B tiles (one weight row per thread per 64-column
// step), warps 10-13 drain the accumulator. Work item = (row tile, column tile); the
// accumulator is double-buffered in TMEM (2 x 256 columns).
// MODE 0: B rows = 128 gate rows + 128 up rows of F-columns [nt*128, +128); epilogue writes
//         act = silu(g) * u (f32) per padded row. MODE 1: B rows = 256 down rows
//         [nt*256, +256); epilogue writes f16 rows of the expert output.
// ------------------------------------------------------------------------------------------
constexpr int kGemmStages = 3;
constexpr int kGemmCopies = 8;
constexpr int kStageBytes = 16384 + 32768;
constexpr int kGemmThreads = 448;

struct GemmSmem {
    static constexpr int A = 0;                                   // per stage +kStageBytes
    static constexpr int B = 16384;
    static constexpr int CB = kGemmStages * kStageBytes;
    static constexpr int BARS = CB + Codebook<kGemmCopies>::BYTES;
    static constexpr int BYTES = BARS + 256;
};

template <uint32_t T, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) moe_gemm_kernel(GemmArgs a) {
    using CBk = Codebook<kGemmCopies>;
    extern __shared__ __align__(1024) uint8_t gsmem_raw[];
    // 1024-byte alignment of the operand tiles (the swizzle pattern is address based)
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)gsmem_raw + 1023) & ~(uintptr_t)1023);
    uint32_t *cb = reinterpret_cast<uint32_t *>(sm + GemmSmem::CB);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(sm + GemmSmem::BARS);
    uint64_t *full_b = full_a + kGemmStages;
    uint64_t *empty = full_b + kGemmStages;
    uint64_t *acc_full = empty + kGemmStages;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int TB = tile_bytes(T);
    const int NB = a.K / 128;
    const int KS = a.K / 64;
    if (tid == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_b[s], 8);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    CBk::stage(cb, a.codebook, tid, kGemmThreads);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // everything above is independent of the predecessor kernels; their outputs are read below
    pdl_wait();
    const uint32_t tmem_base = *tmem_slot;
    const int n_items = *a.n_mtiles * a.n_ntiles;

    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (mbar_wait(bar, parity, a.err)) return true;
        *abort_flag = 1;
        return false;
    };

    if (warp == 0) {
        // ---- A producer ------------------------------------------------------------------
        if (lane == 0) {
            int n = 0;
            for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
                const int t = it / a.n_ntiles;
                for (int ks = 0; ks < KS; ++ks, ++n) {
                    const int s = n % kGemmStages, round = n / kGemmStages;
                    if (!wait(&empty[s], (round & 1) ^ 1)) break;
                    mbar_expect_tx(&full_a[s], 16384);
                    bulk_g2s(sm + s * kStageBytes + GemmSmem::A, a.A + ((size_t)t * KS + ks) * 16384u, 16384, &full_a[s]);
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer --------------------------------------------------------------------
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(128, 256);
            int n = 0, cnt = 0;
            for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++cnt) {
                const int ab = cnt & 1;
                if (!wait(&acc_empty[ab], ((cnt >> 1) & 1) ^ 1)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * 256);
                bool ok = true;
                for (int ks = 0; ks < KS; ++ks, ++n) {
                    const int s = n % kGemmStages, round = n / kGemmStages;
                    if (!wait(&full_a[s], round & 1) || !wait(&full_b[s], round & 1)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sm + s * kStageBytes + GemmSmem::A);
                    const uint32_t b_addr = smem_u32(sm + s * kStageBytes + GemmSmem::B);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_f16(d_tmem, sw128_desc(a_addr + 32 * k), sw128_desc(b_addr + 32 * k), idesc,
                                 (ks | k) != 0);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&acc_full[ab]);
            }
            // all issued MMAs complete before TMEM is released
            umma_commit(done);
            mbar_wait(done, 0, nullptr);
        }
    } else if (warp < 10) {
      if constexpr (T == W_Q8 || T == W_F16) {
        // ---- B from a plain matrix (the shared expert): thread d writes row d of the B tile,
        // Q8_0 as fp16(d * q) (one rounding, as d * CB for the Gyro types), fp16 as stored. The
        // row's 64 weights are loaded before the stage is free, hiding part of their latency.
        const int d = tid - 64;
        int n = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const int nt = it % a.n_ntiles;
            const bool second = MODE == 0 && d >= 128;
            const uint8_t *mat = second ? a.w1 : a.w0;
            const __half *dsc = second ? a.d1 : a.d0;
            const int row = MODE == 0 ? nt * 128 + (d & 127) : nt * 256 + d;
            bool ok = true;
            for (int ks = 0; ks < KS; ++ks, ++n) {
                const int s = n % kGemmStages, round = n / kGemmStages;
                uint4 v[8];
                if constexpr (T == W_Q8) {
                    const uint4 *q = reinterpret_cast<const uint4 *>(mat + (size_t)row * a.K + 64 * ks);
                    const uint4 q4[4] = {q[0], q[1], q[2], q[3]};
                    const float dd[2] = {__half2float(dsc[(size_t)row * (a.K / 32) + 2 * ks]),
                                         __half2float(dsc[(size_t)row * (a.K / 32) + 2 * ks + 1])};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {       // weights 8j .. 8j+7
                        const uint32_t lo = (&q4[j >> 1].x)[(j & 1) * 2], hi = (&q4[j >> 1].x)[(j & 1) * 2 + 1];
                        const float sc = dd[j >> 2];
                        uint32_t h[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t word = k < 2 ? lo : hi;
                            const int sh = 16 * (k & 1);
                            const float a0 = sc * (float)(int8_t)((word >> sh) & 0xffu);
                            const float a1 = sc * (float)(int8_t)((word >> (sh + 8)) & 0xffu);
                            h[k] = pack_half2(a0, a1);
                        }
                        v[j] = make_uint4(h[0], h[1], h[2], h[3]);
                    }
                } else {
                    const uint4 *w = reinterpret_cast<const uint4 *>(mat + ((size_t)row * a.K + 64 * ks) * 2);
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = w[j];
                }
                if (!wait(&empty[s], (round & 1) ^ 1)) { ok = false; break; }
                uint8_t *bt = sm + s * kStageBytes + GemmSmem::B;
#pragma unroll
                for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4 *>(bt + sw128_offset((uint32_t)d, (uint32_t)(8 * j))) = v[j];
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_b[s]);
            }
            if (!ok) break;
        }
      } else {
        // ---- B decoders: thread d builds row d of the 256-row B tile -----------------------
        const int d = tid - 64;
        const uint32_t lane_off = 4u * CBk::copy_off(lane);
        const uint8_t *cbb = reinterpret_cast<const uint8_t *>(cb);
        const int r8 = d & 7;                  // row within its 8-row tile (the same in every item)
        // The thread's row of an item's B tile: its 8-row tiles, one per 128-column block.
        auto rowtiles_of = [&](int it) -> const uint8_t * {
            const int t = it / a.n_ntiles, nt = it % a.n_ntiles;
            uint32_t e = (uint32_t)a.tile_expert[t];
            if (e >= (uint32_t)a.n_expert) {
                atomicExch(a.err, KERR_BOUNDS);
                e = 0;
            }
            const uint8_t *mat = (MODE == 0 ? (d < 128 ? a.w0 : a.w1) : a.w0) + (uint64_t)e * a.expert_bytes;
            const int row = MODE == 0 ? nt * 128 + (d & 127) : nt * 256 + d;
            return mat + (size_t)(row >> 3) * NB * TB;
        };
        // Codes of one k-step: the two own quarters (2h, 2h+1), the neighbour run of quarter
        // (2h+3)%4 and the row's block scale. They are fetched kPrefetch k-steps ahead, across
        // item boundaries, so the global-load latency hides behind the decoding of the steps
        // between.
        struct Codes {
            uint32_t own0[4], own1[4], nbr[4];
            uint16_t d;
        };
        constexpr int kPrefetch = 3;
        int pf_it = blockIdx.x, pf_ks = 0;
        const uint8_t *pf_rt = pf_it < n_items ? rowtiles_of(pf_it) : nullptr;
        auto fetch_next = [&](Codes &cd) {
            if (pf_it >= n_items) return;
            const int h = pf_ks & 1;
            const uint8_t *tile = pf_rt + (size_t)(pf_ks >> 1) * TB;
            load_run<T>(tile, 4 * r8 + 2 * h, cd.own0);
            load_run<T>(tile, 4 * r8 + 2 * h + 1, cd.own1);
            load_run<T>(tile, 4 * r8 + ((2 * h + 3) & 3), cd.nbr);
            cd.d = *reinterpret_cast<const uint16_t *>(tile + tile_code_bytes(T) + 2 * r8);
            if (++pf_ks == KS) {
                pf_ks = 0;
                pf_it += gridDim.x;
                if (pf_it < n_items) pf_rt = rowtiles_of(pf_it);
            }
        };
        Codes cq[kPrefetch];
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i) fetch_next(cq[i]);
        int n = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            bool ok = true;
            for (int ks = 0; ks < KS; ++ks, ++n) {
                const int s = n % kGemmStages, round = n / kGemmStages;
                uint32_t own0[4], own1[4], nbr[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) { own0[j] = cq[0].own0[j]; own1[j] = cq[0].own1[j]; nbr[j] = cq[0].nbr[j]; }
                const uint16_t dh = cq[0].d;
#pragma unroll
                for (int i = 0; i + 1 < kPrefetch; ++i) cq[i] = cq[i + 1];
                fetch_next(cq[kPrefetch - 1]);
                const __half2 d2 = __halves2half2(__ushort_as_half(dh), __ushort_as_half(dh));
                uint32_t o0[2][8], o1[2][8];
                quarter_offsets<T, kGemmCopies>(own0, neighbour_bits<T>(nbr), lane_off, o0[0], o1[0]);
                quarter_offsets<T, kGemmCopies>(own1, neighbour_bits<T>(own0), lane_off, o0[1], o1[1]);
                if (!wait(&empty[s], (round & 1) ^ 1)) { ok = false; break; }
                uint8_t *bt = sm + s * kStageBytes + GemmSmem::B;
#pragma unroll
                for (int qq = 0; qq < 2; ++qq)
#pragma unroll
                    for (int c = 0; c < 8; c += 2) {
                        uint32_t w[4];
                        const uint32_t p0 = lds_u32(cbb, o0[qq][c]);
                        const uint32_t p1 = lds_u32(cbb, o1[qq][c]);
                        const uint32_t p2 = lds_u32(cbb, o0[qq][c + 1]);
                        const uint32_t p3 = lds_u32(cbb, o1[qq][c + 1]);
                        const uint32_t pp[4] = {p0, p1, p2, p3};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const __half2 v = __hmul2(*reinterpret_cast<const __half2 *>(&pp[j]), d2);
                            w[j] = *reinterpret_cast<const uint32_t *>(&v);
                        }
                        const int col = 32 * qq + 4 * c;  // 8 consecutive weights: chunk col/8
                        *reinterpret_cast<uint4 *>(bt + sw128_offset((uint32_t)d, (uint32_t)col)) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_b[s]);
            }
            if (!ok) break;
        }
      }
    } else {
        // ---- epilogue: warp (10..13) reads TMEM lanes 32*(warp%4) .. +31 -------------------
        const int lg = warp & 3;
        const int r = 32 * lg + lane;
        int cnt = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++cnt) {
            const int t = it / a.n_ntiles, nt = it % a.n_ntiles;
            const int ab = cnt & 1;
            if (!wait(&acc_full[ab], (cnt >> 1) & 1)) break;
            tc_fence_after();
            const bool valid = r < a.tile_rows[t];
            const uint32_t base = tmem_base + ((uint32_t)(32 * lg) << 16) + (uint32_t)(ab * 256);
            const size_t prow = (size_t)t * 128 + r;
            if (MODE == 0) {
                float *dst = a.act + prow * a.F + nt * 128;
#pragma unroll 1
                for (int j = 0; j < 8; ++j) {
                    uint32_t g[16], u[16];
                    tmem_ld16(base + 16 * j, g);
                    tmem_ld16(base + 128 + 16 * j, u);
                    tmem_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float4 o;
                            o.x = silu_ref(__uint_as_float(g[4 * q + 0])) * __uint_as_float(u[4 * q + 0]);
                            o.y = silu_ref(__uint_as_float(g[4 * q + 1])) * __uint_as_float(u[4 * q + 1]);
                            o.z = silu_ref(__uint_as_float(g[4 * q + 2])) * __uint_as_float(u[4 * q + 2]);
                            o.w = silu_ref(__uint_as_float(g[4 * q + 3])) * __uint_as_float(u[4 * q + 3]);
                            *reinterpret_cast<float4 *>(dst + 16 * j + 4 * q) = o;
                        }
                    }
                }
            } else {
                __half *dst = a.Y + prow * a.E + nt * 256;
#pragma unroll 1
                for (int j = 0; j < 16; ++j) {
                    uint32_t y[16];
                    tmem_ld16(base + 16 * j, y);
                    tmem_wait_ld();
                    if (valid) {
                        uint4 o0, o1;
                        o0.x = pack_half2(__uint_as_float(y[0]), __uint_as_float(y[1]));
                        o0.y = pack_half2(__uint_as_float(y[2]), __uint_as_float(y[3]));
                        o0.z = pack_half2(__uint_as_float(y[4]), __uint_as_float(y[5]));
                        o0.w = pack_half2(__uint_as_float(y[6]), __uint_as_float(y[7]));
                        o1.x = pack_half2(__uint_as_float(y[8]), __uint_as_float(y[9]));
                        o1.y = pack_half2(__uint_as_float(y[10]), __uint_as_float(y[11]));
                        o1.z = pack_half2(__uint_as_float(y[12]), __uint_as_float(y[13]));
                        o1.w = pack_half2(__uint_as_float(y[14]), __uint_as_float(y[15]));
                        *reinterpret_cast<uint4 *>(dst + 16 * j) = o0;
                        *reinterpret_cast<uint4 *>(dst + 16 * j + 8) = o1;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

// ------------------------------------------------------------------------------------------
// Combine: out[t] = sum_k w[t][k] * Y[row(t, k)] (+ resid[t]); 4 columns per thread. Slots
// without a row (row < 0: served by another rank) add nothing.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    const int per_row = a.E / 4;
    if (i >= (long long)a.n_tok * per_row) return;
    const int t = (int)(i / per_row), c = (int)(i % per_row) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < a.U; ++k) {
        const int row = a.slot_row[t * a.U + k];
        if (row < 0) continue;
        const float w = a.weights[t * a.U + k];
        const uint2 q = *reinterpret_cast<const uint2 *>(a.Y + (size_t)row * a.E + c);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
        v[0] += w * f0.x;
        v[1] += w * f0.y;
        v[2] += w * f1.x;
        v[3] += w * f1.y;
    }
    if (a.Ysh) {
        // the shared expert with its sigmoid gate (src/engine.zig:649-652)
        const float g = 1.0f / (1.0f + expf(-a.sh_logit[t]));
        const uint2 q = *reinterpret_cast<const uint2 *>(a.Ysh + (size_t)t * a.E + c);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
        v[0] += f0.x * g;
        v[1] += f0.y * g;
        v[2] += f1.x * g;
        v[3] += f1.y * g;
    }
    const size_t o = (size_t)t * a.E + c;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (a.resid) v[j] = load_act(a.resid, a.resid_bf16, o + j) + v[j];
        bad |= !(fabsf(v[j]) <= (a.out_f16 ? 65504.f : 3.4028235e38f));   // NaN fails the test too
        if (a.out_f16)
            reinterpret_cast<__half *>(a.out)[o + j] = __float2half_rn(v[j]);
        else if (a.out_bf16)
            reinterpret_cast<__nv_bfloat16 *>(a.out)[o + j] = __float2bfloat16_rn(v[j]);
        else
            reinterpret_cast<float *>(a.out)[o + j] = v[j];
    }
    if (bad && a.err) atomicExch(a.err, KERR_RANGE);
}

// ------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------
namespace {
thread_local bool t_chain_pdl = false;   // the calling thread's current forward call
}
void set_chain_pdl(bool on) {
    static const bool allowed = [] {
        const char *v = getenv("GX_PDL");
        return !(v && v[0] == '0');
    }();
    t_chain_pdl = allowed && on;
}
bool chain_pdl_enabled() { return t_chain_pdl; }

cudaError_t launch_router_gemm(const float *W, const void *x, int x_bf16, int n_tok, int NE, int E, float *C,
                               int splits, cudaStream_t s) {
    dim3 grid((NE + 31) / 32, (n_tok + 63) / 64, splits);
    return launch_chain(router_gemm_kernel, grid, dim3(256), 0, s, W, x, x_bf16, n_tok, NE, E, C);
}

cudaError_t launch_group(const GroupArgs &a, cudaStream_t s) {
    if (a.NE > 512) return cudaErrorInvalidValue;
    const unsigned blocks = (unsigned)((a.n_slots + 1023) / 1024);
    cudaError_t e = cudaSuccess;
    if (blocks) e = launch_chain(group_count_kernel, dim3(blocks), dim3(1024), 0, s, a);
    if (e == cudaSuccess) e = launch_chain(group_scan_kernel, dim3(1), dim3(512), 0, s, a);
    if (e == cudaSuccess && blocks) e = launch_chain(group_place_kernel, dim3(blocks), dim3(1024), 0, s, a);
    return e;
}

cudaError_t launch_rotate_pack(const RotPackArgs &a, cudaStream_t s) {
    const long long warps = (long long)a.n_tok * ((a.E / 128 + 3) / 4);
    if (warps == 0) return cudaSuccess;
    return launch_chain(rotate_pack_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, a);
}

cudaError_t launch_pack_rows(const PackArgs &a, int max_tiles, cudaStream_t s) {
    const long long warps = (long long)max_tiles * 128;
    if (warps == 0) return cudaSuccess;
    return launch_chain(pack_rows_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, a);
}

namespace {
template <uint32_t T, int MODE>
cudaError_t gemm_t(const GemmArgs &a, int sm_count, cudaStream_t s) {
    const int smem = GemmSmem::BYTES + 1024;
    static const cudaError_t once =
        cudaFuncSetAttribute(moe_gemm_kernel<T, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (once != cudaSuccess) return once;
    return launch_chain(moe_gemm_kernel<T, MODE>, dim3(sm_count), dim3(kGemmThreads), smem, s, a);
}
}  // namespace

cudaError_t launch_moe_gemm(const GemmArgs &a, int mode, int sm_count, cudaStream_t s) {
    if (gemm_ts_routed(a.type))
        return gemm_ts_supports(a, mode) ? launch_moe_gemm_ts(a, mode, sm_count, s) : cudaErrorInvalidValue;
#define GX_GEMM_CASE(TT)                                                                 \
    case TT:                                                                             \
        return mode == 0 ? gemm_t<TT, 0>(a, sm_count, s) : gemm_t<TT, 1>(a, sm_count, s);
    switch (a.type) {
        GX_GEMM_CASE(144)
        GX_GEMM_CASE(145)
        GX_GEMM_CASE(146)
        GX_GEMM_CASE(147)
        GX_GEMM_CASE(148)
        GX_GEMM_CASE(149)
        GX_GEMM_CASE(150)
        GX_GEMM_CASE(151)
        GX_GEMM_CASE(W_Q8)
        GX_GEMM_CASE(W_F16)
        default:
            return cudaErrorInvalidValue;
    }
#undef GX_GEMM_CASE
}

cudaError_t launch_rotate_tokens(const void *x, int x_bf16, const float *xscale, const float *signs, int n_tok,
                                int E, __half *xh, cudaStream_t s, const int *scatter, int n_dst) {
    const long long warps = (long long)n_tok * ((E / 128 + 3) / 4);
    if (warps == 0) return cudaSuccess;
    return launch_chain(rotate_tokens_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, x, x_bf16, xscale,
                        signs, n_tok, E, xh, scatter, n_dst);
}

cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s) {
    const long long n = (long long)a.n_tok * (a.E / 4);
    if (n == 0) return cudaSuccess;
    return launch_chain(combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, a);
}

}  // namespace gx
