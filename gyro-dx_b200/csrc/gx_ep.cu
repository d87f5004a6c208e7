// gx_ep.cu — expert-parallel dispatch plan and the sum of returned partial rows.
//
// With W ranks, rank d serves experts [d*NE/W, (d+1)*NE/W), except the experts a route table
// marks as replicated, which every rank serves for its own tokens. A token travels once to every
// rank that serves at least one of its U selected experts, carrying its U slots as destination-local
// expert ids (kNoSlot for experts served elsewhere) and routing weights. The destination
// computes sum_k w_k * Expert_k(x) over its own slots and returns one partial row, and the source
// adds the partial rows of all destinations. This is the scatter / gather around the expert
// phase of src/engine.zig:547-641; the grouping, GEMMs and per-row combine are the same kernels as
// the single-GPU many-token path.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gx_device.cuh"
#include "gx_internal.h"

namespace gx {

// Rank that serves expert e (< NE) and the expert's index among that rank's local experts: the
// route table when the layer has one (replicated experts are served where the token is), else
// the contiguous shard of e.
__device__ __forceinline__ int serving_rank(const EpPlanArgs &a, uint32_t e, uint32_t per) {
    if (a.route) {
        const int r = a.route[e].x;
        return r < 0 ? a.rank : r;
    }
    return (int)(e / per);
}
__device__ __forceinline__ uint32_t local_expert(const EpPlanArgs &a, uint32_t e, uint32_t lo) {
    return a.route ? (uint32_t)a.route[e].y : e - lo;
}

// One CTA of 1024 threads per destination rank d: send rows for d are the tokens with a slot on
// d, in token order (so each destination sees a stable order), at rows [d*stride, d*stride+count);
// rows [count, pad_rows) are filled with empty slots, since a destination receives pad_rows rows
// from every source without learning the count first.
__global__ void __launch_bounds__(1024) ep_plan_kernel(EpPlanArgs a) {
    __shared__ int wsum[32];
    __shared__ int base, chunk;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t per = (uint32_t)(a.NE / a.W), lo = (uint32_t)d * per;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int t0 = 0; t0 < a.n_tok; t0 += 1024) {
        const int t = t0 + tid;
        bool mine = false;
        if (t < a.n_tok) {
            for (int k = 0; k < a.U; ++k) {
                const uint32_t e = a.ids[(size_t)t * a.U + k];
                if (e >= (uint32_t)a.NE) {
                    atomicExch(a.err, KERR_BOUNDS);
                    continue;
                }
                if (d == 0 && a.expert_count) atomicAdd(a.expert_count + e, 1u);
                if (serving_rank(a, e, per) == d) mine = true;
            }
        }
        const unsigned vote = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) wsum[warp] = __popc(vote);
        __syncthreads();
        if (warp == 0) {
            const int v = wsum[lane];
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            wsum[lane] = incl - v;  // exclusive prefix of warp counts
            if (lane == 31) chunk = incl;
        }
        __syncthreads();
        const int pos = base + wsum[warp] + __popc(vote & ((1u << lane) - 1u));
        if (t < a.n_tok) {
            if (mine) {
                const size_t row = (size_t)d * a.stride + pos;
                a.pos_of[(size_t)t * a.W + d] = (int)row;
                for (int k = 0; k < a.U; ++k) {
                    const uint32_t e = a.ids[(size_t)t * a.U + k];
                    const bool here = e < (uint32_t)a.NE && serving_rank(a, e, per) == d;
                    a.send_ids[row * a.U + k] = here ? local_expert(a, e, lo) : kNoSlot;
                    a.send_w[row * a.U + k] = here ? a.weights[(size_t)t * a.U + k] : 0.f;
                }
            } else {
                a.pos_of[(size_t)t * a.W + d] = -1;
            }
        }
        __syncthreads();
        if (tid == 0) base += chunk;
        __syncthreads();
    }
    if (tid == 0) a.send_count[d] = base;
    // every destination receives pad_rows rows from this rank; the unused ones carry no slot
    for (int r = base + tid; r < a.pad_rows; r += 1024) {
        const size_t row = (size_t)d * a.stride + r;
        for (int k = 0; k < a.U; ++k) {
            a.send_ids[row * a.U + k] = kNoSlot;
            a.send_w[row * a.U + k] = 0.f;
        }
    }
}

// out[t] = resid[t] + sum over destinations of the returned partial row of (t, d).
__global__ void __launch_bounds__(256) ep_combine_kernel(EpCombineArgs a) {
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    const int per_row = a.E / 4;
    if (i >= (long long)a.n_tok * per_row) return;
    const int t = (int)(i / per_row), c = (int)(i % per_row) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < a.W; ++d) {
        const int row = a.pos_of[(size_t)t * a.W + d];
        if (row < 0) continue;
        const uint2 q = *reinterpret_cast<const uint2 *>(a.ret + (size_t)row * a.E + c);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
        v[0] += f0.x;
        v[1] += f0.y;
        v[2] += f1.x;
        v[3] += f1.y;
    }
    const size_t o = (size_t)t * a.E + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (a.resid) v[j] = load_act(a.resid, a.resid_bf16, o + j) + v[j];
        if (a.out_bf16)
            reinterpret_cast<__nv_bfloat16 *>(a.out)[o + j] = __float2bfloat16_rn(v[j]);
        else
            reinterpret_cast<float *>(a.out)[o + j] = v[j];
    }
}

cudaError_t launch_ep_plan(const EpPlanArgs &a, cudaStream_t s) {
    if (a.W <= 0 || a.NE % a.W) return cudaErrorInvalidValue;
    ep_plan_kernel<<<a.W, 1024, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpCombineArgs &a, cudaStream_t s) {
    const long long n = (long long)a.n_tok * (a.E / 4);
    if (n == 0) return cudaSuccess;
    ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace gx
