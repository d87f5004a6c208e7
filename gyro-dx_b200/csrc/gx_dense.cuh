// gx_dense.cuh — device helpers for plain (non-Gyro) weight matrices: the shared expert and the
// hyper-connection mixer. Weights are Q8_0 split into int8 [rows][cols] and fp16 block scales
// [rows][cols/32] (W_Q8), or fp16 [rows][cols] (W_F16); activations f32 or bf16.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gx_internal.h"

namespace gx {
namespace dense {

// 8 consecutive weights of row r starting at column c (c a multiple of 8) as f32: Q8_0 as d * q
// (exact in f32), fp16 widened.
template <uint32_t WT>
__device__ __forceinline__ void load_w8(const SharedMat &m, int r, int cols, int c, float (&w)[8]) {
    if constexpr (WT == W_Q8) {
        const uint2 q = *reinterpret_cast<const uint2 *>(m.w + (size_t)r * cols + c);
        const float d = __half2float(m.d[(size_t)r * (cols / 32) + c / 32]);
        const uint32_t qq[2] = {q.x, q.y};
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = d * (float)(int8_t)((qq[j >> 2] >> (8 * (j & 3))) & 0xffu);
    } else {
        const uint4 h = *reinterpret_cast<const uint4 *>(m.w + ((size_t)r * cols + c) * 2);
        const __half2 *p = reinterpret_cast<const __half2 *>(&h);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(p[j]);
            w[2 * j] = f.x;
            w[2 * j + 1] = f.y;
        }
    }
}

__device__ __forceinline__ void load_x8(const void *x, int bf16, size_t i, float (&v)[8]) {
    if (bf16) {
        const uint4 q = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(x) + i);
        const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = __uint_as_float(w4[j] << 16);
            v[2 * j + 1] = __uint_as_float(w4[j] & 0xffff0000u);
        }
    } else {
        const float4 p0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + i);
        const float4 p1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + i + 4);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
        v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float sigmoid_ref_f(float x) { return sigmoid_ref(x); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), int grid, int block, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace dense
}  // namespace gx
