// gx_device.cuh — device building blocks shared by the sm_100a kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "gx_internal.h"
#include "gx_tile.h"

namespace gx {

// Wall-clock bound of every mbarrier / flag wait: after this many nanoseconds the wait gives
// up, records an error for the host, and the kernel returns.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- shared-memory codebook with NCOPY interleaved copies ---------------------------------
// Word i of copy c sits at i * NCOPY + c, and a lane reads copy (lane % NCOPY): two lanes of a
// warp can only meet in a bank when they share a copy (at most 32 / NCOPY lanes), and the
// address of a lookup is one multiply-add of the index.
template <int NCOPY>
struct Codebook {
    static constexpr int WORDS = 2048 * NCOPY;
    static constexpr int BYTES = WORDS * 4;

    // Consecutive threads write consecutive shared words (no bank conflicts); each reads its
    // word's codebook entry from the L1-resident 8 KB global table. The loads of a thread are
    // independent, so they overlap.
    __device__ static void stage(uint32_t *smem, const uint32_t *__restrict__ global_table, int tid, int nthreads) {
#pragma unroll 16
        for (int w = tid; w < WORDS; w += nthreads) smem[w] = __ldg(global_table + w / NCOPY);
    }
    // The same words by bulk copies of a prebuilt image (image[w] = table[w / NCOPY]) into
    // shared memory, completing on mbarrier bar (initialised, count 1). Thread 0 only.
    __device__ static void stage_bulk(uint32_t *smem, const uint32_t *image, uint64_t *bar);
    // Word index of codebook entry idx in this lane's copy (copy_off = lane % NCOPY).
    __device__ static __forceinline__ uint32_t word(uint32_t idx, uint32_t copy_off) { return idx * NCOPY + copy_off; }
    __device__ static __forceinline__ uint32_t copy_off(int lane) { return (uint32_t)(lane % NCOPY); }
};

// ---- tensor-core dot product: mma.sync m16n8k16, f16 x f16 -> f32 -------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// fp32 -> (hi, lo) fp16 pair with x ~= hi + lo to about 22 bits.
__device__ __forceinline__ void split_hilo(float x, float &hi, float &lo) {
    hi = __half2float(__float2half_rn(x));
    lo = x - hi;
}

// ---- mbarrier + bulk async copy (TMA engine, 1-D, no multicast) --------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
template <int NCOPY>
__device__ void Codebook<NCOPY>::stage_bulk(uint32_t *smem, const uint32_t *image, uint64_t *bar) {
    constexpr uint32_t kChunk = 16384;
    static_assert(BYTES % kChunk == 0, "codebook image in whole chunks");
    mbar_expect_tx(bar, (uint32_t)BYTES);
    for (uint32_t o = 0; o < (uint32_t)BYTES; o += kChunk)
        bulk_g2s(reinterpret_cast<uint8_t *>(smem) + o, reinterpret_cast<const uint8_t *>(image) + o, kChunk, bar);
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; returns false (and records KERR_WAIT) once kWaitLimitNs have passed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - start > kWaitLimitNs) break;
    }
    if (err) atomicExch(err, KERR_WAIT);
    return false;
}

// ---- 128-point normalised Walsh-Hadamard transform across one warp ----------------------
// Lane l holds v[0..3] = x[4l .. 4l+3]. Butterfly widths 1, 2, 4, ..., 64 in the order of
// src/kernels.zig:317-338 (pairs (j, j + width) -> (a + b, a - b)), then * 1/sqrt(128).
__device__ __forceinline__ void fwht128_warp(float (&v)[4], int lane) {
    float a, b;
    a = v[0]; b = v[1]; v[0] = a + b; v[1] = a - b;
    a = v[2]; b = v[3]; v[2] = a + b; v[3] = a - b;
    a = v[0]; b = v[2]; v[0] = a + b; v[2] = a - b;
    a = v[1]; b = v[3]; v[1] = a + b; v[3] = a - b;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float p = __shfl_xor_sync(0xffffffffu, v[j], m);
            v[j] = upper ? p - v[j] : v[j] + p;
        }
    }
    const float norm = 1.0f / sqrtf(128.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= norm;
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while its predecessor still runs; pdl_wait() blocks until the predecessor grid has
// completed and its memory is visible. Every CTA calls pdl_wait() before it reads anything the
// predecessor wrote or writes anything a predecessor reads. Without the launch attribute both
// instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch of a kernel of the many-token chain (router .. combine, and the expert-parallel
// exchange kernels) with programmatic dependent launch: the kernel may be scheduled while its
// predecessor on the stream still runs, and every such kernel calls pdl_launch_dependents() first
// and pdl_wait() before it reads anything a predecessor wrote. The host enables it per call
// (set_chain_pdl): it pays off when the chain's kernels are short (measured on B200: +7 % on one
// 1,024-token layer, -1.4 % on a 4,067-token one); GX_PDL=0 in the environment turns it off.
// (chain_pdl_enabled / set_chain_pdl: gx_internal.h)
template <typename... KArgs, typename... Args>
cudaError_t launch_chain_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    return launch_chain_pdl(chain_pdl_enabled(), kernel, grid, block, smem, s, args...);
}

// Optional phase trace (build with -DGX_TRACE): thread 0 of each CTA stores %globaltimer (ns) at
// numbered points into gx_trace[kernel][cta][point], and the CTA's start at point 7. Off in normal
// builds; the array lives in the translation unit that defines GX_TRACE_OWNER (gx_kernels.cu).
#if defined(GX_TRACE) && defined(GX_TRACE_OWNER)
constexpr int kTraceKernels = 4, kTraceCtas = 160, kTracePoints = 8;
__device__ long long gx_trace[kTraceKernels][kTraceCtas][kTracePoints];
#define GX_TRACE_START(k)                                                                   \
    const int gx_tk_ = (k);                                                                 \
    do {                                                                                    \
        if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) gx_trace[gx_tk_][blockIdx.x][7] = (long long)globaltimer_ns(); \
    } while (0)
#define GX_TRACE_POINT(p)                                                                  \
    do {                                                                                   \
        if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) gx_trace[gx_tk_][blockIdx.x][p] = (long long)globaltimer_ns(); \
    } while (0)
#else
#define GX_TRACE_START(k) do {} while (0)
#define GX_TRACE_POINT(p) do {} while (0)
#endif

__device__ __forceinline__ float load_act(const void *p, int bf16, size_t i) {
    if (bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    return reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ float silu_ref(float x) { return x / (1.0f + expf(-x)); }

}  // namespace gx
