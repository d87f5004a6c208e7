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
#include <algorithm>

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

// The plan is two token-parallel passes over CTAs of kPlanTok tokens. Pass 1 marks, per token,
// the ranks that serve one of its slots (bit d of dest_mask) and counts them per CTA; pass 2 gives
// each marked (token, d) its row: the CTA's base for d (the counts of the CTAs before it) plus its
// rank among the CTA's marked tokens. So the send rows for d are the tokens with a slot on d, in
// token order (each destination sees a stable order), at rows [d*stride, d*stride+count); rows
// [count, pad_rows) are marked empty, since with NCCL rows a destination receives pad_rows rows
// from every source without learning the count first.
__global__ void __launch_bounds__(kPlanTok) ep_plan_mask_kernel(EpPlanArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int cnt[kMaxEpWorld];
    const int tid = threadIdx.x, lane = tid & 31;
    const int t = blockIdx.x * kPlanTok + tid;
    const uint32_t per = (uint32_t)(a.NE / a.W);
    for (int d = tid; d < a.W; d += kPlanTok) cnt[d] = 0;
    __syncthreads();
    uint64_t mask = 0;
    if (t < a.n_tok) {
        for (int k = 0; k < a.U; ++k) {
            const uint32_t e = a.ids[(size_t)t * a.U + k];
            if (e >= (uint32_t)a.NE) {
                atomicExch(a.err, KERR_BOUNDS);
                continue;
            }
            mask |= 1ull << serving_rank(a, e, per);
        }
        a.dest_mask[t] = mask;
    }
    if (a.expert_count) {
        // routed-slot counts, one atomic per distinct expert in the warp
        for (int k = 0; k < a.U; ++k) {
            const uint32_t e = t < a.n_tok ? a.ids[(size_t)t * a.U + k] : kNoSlot;
            const unsigned same = __match_any_sync(0xffffffffu, e);
            if (e < (uint32_t)a.NE && lane == __ffs(same) - 1) atomicAdd(a.expert_count + e, (unsigned)__popc(same));
        }
    }
    for (int d = 0; d < a.W; ++d) {
        const unsigned v = __ballot_sync(0xffffffffu, (mask >> d) & 1);
        if (lane == 0 && v) atomicAdd(&cnt[d], __popc(v));
    }
    __syncthreads();
    for (int d = tid; d < a.W; d += kPlanTok) a.block_count[(size_t)blockIdx.x * kMaxEpWorld + d] = cnt[d];
}

__global__ void __launch_bounds__(kPlanTok) ep_plan_place_kernel(EpPlanArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int kWarps = kPlanTok / 32;
    __shared__ int base[kMaxEpWorld], total[kMaxEpWorld];
    __shared__ int wcnt[kMaxEpWorld][kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t = blockIdx.x * kPlanTok + tid;
    const uint32_t per = (uint32_t)(a.NE / a.W);
    // base and total of every destination: warp w sums destinations w, w + kWarps, ...
    for (int d = warp; d < a.W; d += kWarps) {
        int before = 0, all = 0;
        for (int j = lane; j < (int)gridDim.x; j += 32) {
            const int v = a.block_count[(size_t)j * kMaxEpWorld + d];
            all += v;
            if (j < (int)blockIdx.x) before += v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            before += __shfl_xor_sync(0xffffffffu, before, o);
            all += __shfl_xor_sync(0xffffffffu, all, o);
        }
        if (lane == 0) {
            base[d] = before;
            total[d] = all;
        }
    }
    const uint64_t mask = t < a.n_tok ? a.dest_mask[t] : 0;
    for (int d = 0; d < a.W; ++d) {
        const unsigned v = __ballot_sync(0xffffffffu, (mask >> d) & 1);
        if (lane == 0) wcnt[d][warp] = __popc(v);
    }
    __syncthreads();
    if (blockIdx.x == 0)
        for (int d = tid; d < a.W; d += kPlanTok) a.send_count[d] = total[d];
    for (int d = 0; d < a.W; ++d) {
        const unsigned v = __ballot_sync(0xffffffffu, (mask >> d) & 1);
        if (t >= a.n_tok) continue;
        if (!((mask >> d) & 1)) {
            a.pos_of[(size_t)t * a.W + d] = -1;
            continue;
        }
        int pos = base[d] + __popc(v & ((1u << lane) - 1u));
        for (int w = 0; w < warp; ++w) pos += wcnt[d][w];
        const size_t row = (size_t)d * a.stride + pos;
        a.pos_of[(size_t)t * a.W + d] = (int)row;
        const uint32_t lo = (uint32_t)d * per;
        for (int k = 0; k < a.U; ++k) {
            const uint32_t e = a.ids[(size_t)t * a.U + k];
            const bool here = e < (uint32_t)a.NE && serving_rank(a, e, per) == d;
            a.send_ids[row * a.U + k] = here ? local_expert(a, e, lo) : kNoSlot;
            a.send_w[row * a.U + k] = here ? a.weights[(size_t)t * a.U + k] : 0.f;
        }
    }
    // every destination receives pad_rows rows from this rank (NCCL rows); the unused ones carry no slot
    for (int d = 0; d < a.W; ++d)
        for (int r = total[d] + (int)blockIdx.x * kPlanTok + tid; r < a.pad_rows; r += (int)gridDim.x * kPlanTok) {
            const size_t row = (size_t)d * a.stride + r;
            for (int k = 0; k < a.U; ++k) {
                a.send_ids[row * a.U + k] = kNoSlot;
                a.send_w[row * a.U + k] = 0.f;
            }
        }
}

// out[t] = resid[t] + sum over destinations of the returned partial row of (t, d) (+ the gated
// shared-expert row of t).
__global__ void __launch_bounds__(256) ep_combine_kernel(EpCombineArgs a) {
    pdl_launch_dependents();
    pdl_wait();
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
    if (a.Ysh) {
        // this rank's shared expert for its own token, with its sigmoid gate (src/engine.zig:649-652)
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
        bad |= !(fabsf(v[j]) <= 3.4028235e38f);   // Inf or NaN
        if (a.out_bf16)
            reinterpret_cast<__nv_bfloat16 *>(a.out)[o + j] = __float2bfloat16_rn(v[j]);
        else
            reinterpret_cast<float *>(a.out)[o + j] = v[j];
    }
    if (bad && a.err) atomicExch(a.err, KERR_RANGE);
}

cudaError_t launch_ep_plan(const EpPlanArgs &a, cudaStream_t s) {
    if (a.W <= 0 || a.W > kMaxEpWorld || a.NE % a.W || a.n_tok < 0) return cudaErrorInvalidValue;
    const int grid = std::max(1, ep_plan_ctas(a.n_tok));
    cudaError_t e = launch_chain(ep_plan_mask_kernel, dim3(grid), dim3(kPlanTok), 0, s, a);
    if (e == cudaSuccess) e = launch_chain(ep_plan_place_kernel, dim3(grid), dim3(kPlanTok), 0, s, a);
    return e;
}

cudaError_t launch_ep_combine(const EpCombineArgs &a, cudaStream_t s) {
    const long long n = (long long)a.n_tok * (a.E / 4);
    if (n == 0) return cudaSuccess;
    return launch_chain(ep_combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, a);
}

// ---- exchange over NVLink peer memory -------------------------------------------------------
// A source writes only the rows a destination needs, straight into the destination's memory
// (plain stores through the IPC mapping; no TMA and no multicast), and publishes them with a
// release store of the epoch into the destination's flag word after a system-scope fence. The
// destination acquires the flag before it reads. Every wait is bounded (EpPeerArgs::wait_ns),
// and a failure travels on: a rank whose receive failed publishes its return flags with
// kFlagFailed, so no rank completes the call with another rank's rows missing.

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until the flag carries this epoch (or a later one); false (and KERR_WAIT) when the
// limit passes or the peer published the epoch with kFlagFailed.
__device__ bool wait_flag(const unsigned *flag, unsigned epoch, uint64_t wait_ns, int *err) {
    const uint64_t t0 = globaltimer_ns();
    unsigned v;
    while (((v = ld_acquire_sys(flag)) & ~kFlagFailed) < epoch) {
        if (globaltimer_ns() - t0 > wait_ns) {
            atomicExch(err, KERR_WAIT);
            return false;
        }
        __nanosleep(64);
    }
    if (v & kFlagFailed) {
        atomicExch(err, KERR_WAIT);
        return false;
    }
    return true;
}

// The CTA that finishes last (every thread's writes fenced at system scope first) returns true.
__device__ bool last_cta(unsigned *done) {
    __threadfence_system();
    __syncthreads();
    __shared__ bool is_last;
    if (threadIdx.x == 0) is_last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (is_last && threadIdx.x == 0) {
        __threadfence();
        *done = 0;  // every CTA has counted: ready for the next transfer
    }
    return is_last;
}

__global__ void __launch_bounds__(256) ep_push_kernel(EpPushArgs a, int row_ctas) {
    pdl_launch_dependents();
    pdl_wait();
    const EpPeerArgs &p = a.p;
    const int lane = threadIdx.x & 31;
    if ((int)blockIdx.x < row_ctas) {
        // rows: one warp per (token, 4 column blocks) in a grid-stride loop, rotation as
        // rotate_tokens_kernel
        const int nb = p.E / 128, groups = (nb + 3) / 4;
        const long long n_w = (long long)a.n_tok * groups, step = (long long)row_ctas * 8;
        for (long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); w < n_w; w += step) {
            const int t = (int)(w / groups), b0 = (int)(w % groups) * 4;
            const float sc = a.xscale ? a.xscale[t] : 1.f;
            float v[4][4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int b = b0 + q;
                if (b >= nb) break;
                const size_t base = (size_t)t * p.E + b * 128 + 4 * lane;
#pragma unroll
                for (int j = 0; j < 4; ++j) v[q][j] = load_act(a.x, a.x_bf16, base + j) * sc;
                if (a.signs) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[q][j] *= a.signs[b * 128 + 4 * lane + j];
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int b = b0 + q;
                if (b >= nb) break;
                if (a.signs) fwht128_warp(v[q], lane);
                uint2 o;
                o.x = pack_half2(v[q][0], v[q][1]);
                o.y = pack_half2(v[q][2], v[q][3]);
                for (int d = 0; d < p.W; ++d) {
                    const int row = a.pos_of[(size_t)t * p.W + d];
                    if (row < 0) continue;
                    const size_t pos = (size_t)(row - d * p.T);
                    __half *dst = reinterpret_cast<__half *>(p.peer[d] + p.off.rx_rows) +
                                  ((size_t)p.rank * p.T + pos) * p.E + b * 128 + 4 * lane;
                    *reinterpret_cast<uint2 *>(dst) = o;
                }
            }
        }
    } else {
        // slot metadata: thread per (destination, position) of this call's T rows per source,
        // grid-stride; rows past the destination's count carry no slot
        const long long n_r = (long long)p.W * p.T;
        const long long step = (long long)(gridDim.x - row_ctas) * 256;
        for (long long r = (long long)(blockIdx.x - row_ctas) * 256 + threadIdx.x; r < n_r; r += step) {
            const int d = (int)(r / p.T), pos = (int)(r % p.T);
            const size_t src = ((size_t)d * p.T + pos) * p.U;
            const size_t dst = ((size_t)p.rank * p.T + pos) * p.U;
            uint32_t *ids = reinterpret_cast<uint32_t *>(p.peer[d] + p.off.rx_ids);
            float *wts = reinterpret_cast<float *>(p.peer[d] + p.off.rx_w);
            if (pos < a.send_count[d]) {
                for (int k = 0; k < p.U; ++k) {
                    ids[dst + k] = a.send_ids[src + k];
                    wts[dst + k] = a.send_w[src + k];
                }
            } else {
                for (int k = 0; k < p.U; ++k) ids[dst + k] = kNoSlot;
            }
        }
    }
    unsigned *done = reinterpret_cast<unsigned *>(p.peer[p.rank] + p.off.done);
    if (last_cta(done) && threadIdx.x < (unsigned)p.W) {
        const int d = threadIdx.x;
        *reinterpret_cast<volatile int *>(p.peer[d] + p.off.rx_count + 4 * p.rank) = a.send_count[d];
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned *>(p.peer[d] + p.off.rx_flag) + p.rank, p.epoch);
    }
}

__global__ void __launch_bounds__(1024) ep_wait_rx_kernel(EpPeerArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int failed[kMaxPeers];
    __shared__ int any_failed;
    uint8_t *own = a.peer[a.rank];
    if (threadIdx.x == 0) any_failed = 0;
    __syncthreads();
    if (threadIdx.x < (unsigned)a.W) {
        const int s = threadIdx.x;
        const bool ok = wait_flag(reinterpret_cast<const unsigned *>(own + a.off.rx_flag) + s, a.epoch, a.wait_ns, a.err);
        failed[s] = !ok;
        if (!ok) atomicExch(&any_failed, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<volatile int *>(own + a.off.status) = any_failed;
    if (!any_failed) return;
    // the rows of a source that never published this call hold another call's slots: none of
    // them takes part (the sources that did publish marked their own rows past the count)
    int *cnt = reinterpret_cast<int *>(own + a.off.rx_count);
    uint32_t *ids = reinterpret_cast<uint32_t *>(own + a.off.rx_ids);
    for (int s = 0; s < a.W; ++s) {
        if (!failed[s]) continue;
        if (threadIdx.x == 0) cnt[s] = 0;
        const long long n = (long long)a.T * a.U, base = (long long)s * a.T * a.U;
        for (long long i = threadIdx.x; i < n; i += blockDim.x) ids[base + i] = kNoSlot;
    }
}

// One warp per received row (grid-stride): the row's U slots are read once (lane k holds slot k)
// and every lane sums 8 columns at a time into one 16-byte store to the source's ret region.
__global__ void __launch_bounds__(256) ep_return_kernel(EpPeerArgs a, const __half *Y, const int *slot_row) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    uint8_t *own = a.peer[a.rank];
    const int *cnt = reinterpret_cast<const int *>(own + a.off.rx_count);
    const float *rw = reinterpret_cast<const float *>(own + a.off.rx_w);
    const bool failed = *reinterpret_cast<volatile const int *>(own + a.off.status) != 0;
    const long long n_r = failed ? 0 : (long long)a.W * a.T, step = (long long)gridDim.x * 8;
    for (long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); r < n_r; r += step) {
        const int s = (int)(r / a.T), pos = (int)(r % a.T);
        if (pos >= min(cnt[s], a.T)) continue;  // the same for the whole warp
        int row_k = -1;
        float w_k = 0.f;
        if (lane < a.U) {
            row_k = slot_row[(size_t)r * a.U + lane];
            w_k = rw[(size_t)r * a.U + lane];
        }
        __half *dst = reinterpret_cast<__half *>(a.peer[s] + a.off.ret_rows) + ((size_t)a.rank * a.T + pos) * a.E;
        for (int c = lane * 8; c < a.E; c += 256) {
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int k = 0; k < a.U; ++k) {
                const int row = __shfl_sync(0xffffffffu, row_k, k);
                const float wk = __shfl_sync(0xffffffffu, w_k, k);
                if (row < 0) continue;
                const uint4 q = *reinterpret_cast<const uint4 *>(Y + (size_t)row * a.E + c);
                const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h[j]);
                    v[2 * j] += wk * f.x;
                    v[2 * j + 1] += wk * f.y;
                }
            }
            uint4 o;
            o.x = pack_half2(v[0], v[1]);
            o.y = pack_half2(v[2], v[3]);
            o.z = pack_half2(v[4], v[5]);
            o.w = pack_half2(v[6], v[7]);
            *reinterpret_cast<uint4 *>(dst + c) = o;
        }
    }
    unsigned *done = reinterpret_cast<unsigned *>(own + a.off.done) + 1;
    if (last_cta(done) && threadIdx.x < (unsigned)a.W) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned *>(a.peer[threadIdx.x] + a.off.ret_flag) + a.rank,
                       a.epoch | (failed ? kFlagFailed : 0u));
    }
}

__global__ void ep_wait_ret_kernel(EpPeerArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x < (unsigned)a.W)
        wait_flag(reinterpret_cast<const unsigned *>(a.peer[a.rank] + a.off.ret_flag) + threadIdx.x, a.epoch,
                  a.wait_ns, a.err);
}

size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

// grid bounds of the exchange kernels (CTAs of 256 threads; a few per SM of 148)
constexpr long long kPushRowCtas = 148 * 6, kPushMetaCtas = 148, kReturnCtas = 148 * 6;

}  // namespace

EpBlock ep_block_layout(int W, int T, int E, int U) {
    EpBlock b{};
    size_t off = 0;
    b.rx_rows = off; off = align_up(off + (size_t)W * T * E * 2);
    b.rx_ids = off; off = align_up(off + (size_t)W * T * U * 4);
    b.rx_w = off; off = align_up(off + (size_t)W * T * U * 4);
    b.ret_rows = off; off = align_up(off + (size_t)W * T * E * 2);
    b.rx_count = off; off = align_up(off + (size_t)W * 4);
    b.rx_flag = off; off = align_up(off + (size_t)W * 4);
    b.ret_flag = off; off = align_up(off + (size_t)W * 4);
    b.done = off; off = align_up(off + 8);
    b.status = off; off = align_up(off + 4);
    b.bytes = off;
    return b;
}

cudaError_t launch_ep_push(const EpPushArgs &a, cudaStream_t s) {
    if (a.p.W > kMaxPeers || a.p.W > 256) return cudaErrorInvalidValue;
    // grid-stride kernels: a bounded grid keeps the completion count (one atomic per CTA) small
    if (a.n_tok > a.p.T || a.p.epoch == 0 || a.p.epoch >= kFlagFailed) return cudaErrorInvalidValue;
    const long long warps = (long long)a.n_tok * ((a.p.E / 128 + 3) / 4);
    const int row_ctas = (int)std::min<long long>((warps + 7) / 8, kPushRowCtas);
    const int meta_ctas = (int)std::min<long long>(((long long)a.p.W * a.p.T + 255) / 256, kPushMetaCtas);
    const int grid = row_ctas + meta_ctas > 0 ? row_ctas + meta_ctas : 1;
    return launch_chain(ep_push_kernel, dim3(grid), dim3(256), 0, s, a, row_ctas);
}

cudaError_t launch_ep_wait_rx(const EpPeerArgs &a, cudaStream_t s) {
    if (a.W > kMaxPeers) return cudaErrorInvalidValue;
    return launch_chain(ep_wait_rx_kernel, dim3(1), dim3(1024), 0, s, a);
}

cudaError_t launch_ep_return(const EpPeerArgs &a, const __half *Y, const int *slot_row, cudaStream_t s) {
    if (a.W > kMaxPeers || a.W > 256) return cudaErrorInvalidValue;
    if (a.E % 8 || a.U > 32) return cudaErrorInvalidValue;
    const long long warps = (long long)a.W * a.T;
    const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>((warps + 7) / 8, kReturnCtas));
    return launch_chain(ep_return_kernel, dim3(grid), dim3(256), 0, s, a, Y, slot_row);
}

cudaError_t launch_ep_wait_ret(const EpPeerArgs &a, cudaStream_t s) {
    if (a.W > kMaxPeers) return cudaErrorInvalidValue;
    return launch_chain(ep_wait_ret_kernel, dim3(1), dim3(32), 0, s, a);
}

}  // namespace gx

