// gx_router_tc.cu — the many-token router GEMM (logits = W_r x, src/engine.zig:526 through
// kernels.matmul, src/kernels.zig:72-84 and :264-268) on the tcgen05 tensor cores at fp32
// accuracy.
//
// The f32 router matrix is stored as three bf16 parts, W = W0 + W1 + W2 (each part the bf16
// rounding of what the previous parts leave), which together carry its 24-bit significand.
// bf16 activations are used as they are; f32 activations are split the same way into x0, x1, x2.
// Every product of parts is exact in f32, and the tensor core accumulates in f32. The products
// kept are those with i + j <= 2 (x_i W_j is about 2^-8(i+j) of x W), so the dropped terms are
// ~2^-24 of the result, the size of fp32 rounding itself.
//
// Tile: 128 tokens x 128 experts, K split over gridDim.z (partial logits [split][token][expert],
// summed by the selection kernel). Warps 0-3 build the activation parts of each 64-column step
// in shared memory (128-byte swizzled K-major, as the MMA descriptors expect) and afterwards
// drain the accumulator; warp 4 streams the pre-swizzled weight parts with one bulk copy per
// step; warp 5 owns TMEM and issues the MMAs. Every wait is bounded.
#include <cuda_bf16.h>

#include <algorithm>
#include <cuda_runtime.h>

#include "gx_device.cuh"
#include "gx_internal.h"
#include "gx_umma.cuh"

namespace gx {

namespace {

constexpr int kRtThreads = 192;
constexpr int kRtPart = 16384;  // one 128-row x 64-column bf16 operand part

struct RtArgs {
    const void *x;
    int x_bf16, n_tok, E, NE, ks_per_split;
    const uint8_t *wparts;  // [NE/128][E/64][3][16384]
    float *logits;          // [split][n_tok][NE]
    int *err;
};

__device__ __forceinline__ uint32_t bf16_bits_rn(float v) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    return (uint32_t)(*reinterpret_cast<const unsigned short *>(&b));
}
__device__ __forceinline__ float bf16_value(uint32_t bits) { return __uint_as_float(bits << 16); }

template <int AP>
__global__ void __launch_bounds__(kRtThreads, 1) router_tc_kernel(RtArgs a) {
    constexpr int ST = AP == 1 ? 3 : 2;                 // pipeline stages
    constexpr int STAGE = (AP + 3) * kRtPart;           // activation parts + three weight parts
    extern __shared__ __align__(1024) uint8_t rt_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)rt_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(sm + ST * STAGE);
    uint64_t *full_b = full_a + ST;
    uint64_t *empty = full_b + ST;
    uint64_t *acc_full = empty + ST;
    uint64_t *done = acc_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m0 = blockIdx.x * 128, nt = blockIdx.y, split = blockIdx.z;
    const int KS = a.E / 64, ks0 = split * a.ks_per_split, nks = a.ks_per_split;
    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full_a[s], 4);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    if (warp == 5) tmem_alloc(tmem_slot, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // everything above is independent of the predecessor kernels; their outputs are read below
    pdl_wait();
    const uint32_t tmem_base = *tmem_slot;

    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (mbar_wait(bar, parity, a.err)) return true;
        *abort_flag = 1;
        return false;
    };

    if (warp < 4) {
        // ---- activation parts: thread r writes row r (token m0 + r) of each part; the row's
        // next 64 columns are loaded while this step waits for its stage ----------------------
        const int r = tid;
        const int tok = m0 + r;
        const bool live = tok < a.n_tok;
        constexpr int NV = AP == 1 ? 8 : 16;  // 16-byte loads per row and step
        uint4 nx[NV];
        auto fetch = [&](int i) {
            const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.x) +
                                                               ((size_t)tok * a.E + (size_t)(ks0 + i) * 64) * (AP == 1 ? 2 : 4));
#pragma unroll
            for (int v = 0; v < NV; ++v) nx[v] = live ? src[v] : make_uint4(0u, 0u, 0u, 0u);
        };
        if (nks > 0) fetch(0);
        bool ok = true;
        const uint32_t rowoff = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
        for (int i = 0; i < nks; ++i) {
            const int s = i % ST, round = i / ST;
            uint4 cur[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) cur[v] = nx[v];
            if (i + 1 < nks) fetch(i + 1);
            if (!wait(&empty[s], (round & 1) ^ 1)) { ok = false; break; }
            uint8_t *at = sm + s * STAGE;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = columns 8c .. 8c+7
                uint32_t p[AP][4];
                if (AP == 1) {
                    p[0][0] = cur[c].x; p[0][1] = cur[c].y; p[0][2] = cur[c].z; p[0][3] = cur[c].w;
                } else {
                    const uint4 u0 = cur[2 * c], u1 = cur[(2 * c + 1) % NV];
                    const float f[8] = {__uint_as_float(u0.x), __uint_as_float(u0.y), __uint_as_float(u0.z),
                                        __uint_as_float(u0.w), __uint_as_float(u1.x), __uint_as_float(u1.y),
                                        __uint_as_float(u1.z), __uint_as_float(u1.w)};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        uint32_t lo[AP], hi[AP];
                        float rl = f[2 * h], rh = f[2 * h + 1];
#pragma unroll
                        for (int q = 0; q < AP; ++q) {
                            lo[q] = bf16_bits_rn(rl);
                            hi[q] = bf16_bits_rn(rh);
                            rl -= bf16_value(lo[q]);
                            rh -= bf16_value(hi[q]);
                        }
#pragma unroll
                        for (int q = 0; q < AP; ++q) p[q][h] = lo[q] | (hi[q] << 16);
                    }
                }
                const uint32_t off = rowoff + (uint32_t)((c ^ (r & 7)) << 4);
#pragma unroll
                for (int q = 0; q < AP; ++q)
                    *reinterpret_cast<uint4 *>(at + q * kRtPart + off) = make_uint4(p[q][0], p[q][1], p[q][2], p[q][3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_a[s]);
        }
        // ---- epilogue: TMEM lanes 32*warp .. +31, 128 columns ------------------------------
        if (ok && wait(acc_full, 0)) {
            tc_fence_after();
            float *dst = a.logits + ((size_t)split * a.n_tok + tok) * a.NE;
            const uint32_t base = tmem_base + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
                uint32_t v[16];
                tmem_ld16(base + 16 * j, v);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const int e = nt * 128 + 16 * j + q;
                        if (e < a.NE) dst[e] = __uint_as_float(v[q]);
                    }
                }
            }
        }
    } else if (warp == 4) {
        // ---- weight parts: one 48 KB bulk copy per step -------------------------------------
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nks; ++i) {
                const int s = i % ST, round = i / ST;
                if (!wait(&empty[s], (round & 1) ^ 1)) break;
                mbar_expect_tx(&full_b[s], 3 * kRtPart);
                bulk_g2s(sm + s * STAGE + AP * kRtPart, a.wparts + ((size_t)nt * KS + ks0 + i) * 3 * kRtPart,
                         3 * kRtPart, &full_b[s]);
                ++issued;
            }
            if (*abort_flag) {  // copies still in flight land before the CTA leaves
                for (int i = (issued > ST ? issued - ST : 0); i < issued; ++i)
                    mbar_wait(&full_b[i % ST], (uint32_t)((i / ST) & 1), nullptr);
            }
        }
    } else {
        // ---- MMA issuer: the whole warp runs the loop and takes the waits (a warp vote makes
        // each outcome uniform); one elected lane issues the MMAs and the commits ---------------
        const bool leader = elect_one();
        const uint32_t idesc = f16_idesc(128, 128) | (1u << 7) | (1u << 10);  // A and B bf16
        bool ok = true;
        for (int i = 0; i < nks; ++i) {
            const int s = i % ST, round = i / ST;
            const bool ready = wait(&full_a[s], round & 1) && wait(&full_b[s], round & 1);
            if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
            tc_fence_after();
            const uint32_t at = smem_u32(sm + s * STAGE), bt = at + AP * kRtPart;
            if (leader) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
#pragma unroll
                    for (int xi = 0; xi < AP; ++xi)
#pragma unroll
                        for (int wj = 0; wj < 3 - xi; ++wj)
                            umma_f16(tmem_base, sw128_desc(at + xi * kRtPart + 32 * k),
                                     sw128_desc(bt + wj * kRtPart + 32 * k), idesc, (i | k | xi | wj) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (leader) {
            if (ok) umma_commit(acc_full);
            umma_commit(done);
            mbar_wait(done, 0, nullptr);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 128);
    }
}

template <int AP>
cudaError_t router_tc_t(const RtArgs &a, dim3 grid, cudaStream_t s) {
    constexpr int ST = AP == 1 ? 3 : 2;
    constexpr int SMEM = ST * (AP + 3) * kRtPart + 1024 + 256;
    static const cudaError_t once =
        cudaFuncSetAttribute(router_tc_kernel<AP>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (once != cudaSuccess) return once;
    return launch_chain(router_tc_kernel<AP>, grid, dim3(kRtThreads), SMEM, s, a);
}

}  // namespace

// K splits of the router GEMM: as many as keep the grid to one wave of CTAs (each CTA streams
// its slice of the three router parts, so more CTAs means more SMs pulling them in), limited by
// the partial-logit scratch of the context (4 x 512 columns per token) and by E / 64.
int router_tc_splits(int n_tok, int NE, int E, int sm_count) {
    const int tiles = ((n_tok + 127) / 128) * ((NE + 127) / 128);
    const int KS = E / 64;
    const int cap = std::min(16, 4 * 512 / (((NE + 127) / 128) * 128));
    int splits = 1;
    while (splits * 2 <= cap && tiles * splits * 2 <= sm_count && KS % (splits * 2) == 0) splits *= 2;
    return splits;
}

size_t router_parts_bytes(int NE, int E) { return (size_t)((NE + 127) / 128) * (E / 64) * 3 * kRtPart; }

cudaError_t launch_router_tc(const void *x, int x_bf16, int n_tok, int NE, int E, const uint8_t *wparts,
                             float *logits, int splits, int *err, cudaStream_t s) {
    if (n_tok <= 0) return cudaSuccess;
    if (E % 64 || (E / 64) % splits || NE > 512) return cudaErrorInvalidValue;
    RtArgs a{};
    a.x = x;
    a.x_bf16 = x_bf16;
    a.n_tok = n_tok;
    a.E = E;
    a.NE = NE;
    a.ks_per_split = E / 64 / splits;
    a.wparts = wparts;
    a.logits = logits;
    a.err = err;
    const dim3 grid((unsigned)((n_tok + 127) / 128), (unsigned)((NE + 127) / 128), (unsigned)splits);
    return x_bf16 ? router_tc_t<1>(a, grid, s) : router_tc_t<3>(a, grid, s);
}

}  // namespace gx
