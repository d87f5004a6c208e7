// gx_hc.cu — the hyper-connection mixer around the routed layer, the producer of the layer's input
// and the consumer of its output in the reference model (src/engine.zig:162-165 and :184-228;
// on the reference GPU the fused hc_pre / hc_post kernels of shaders/engine/hc.hlsl):
//
//   xn[c]   = RMSNorm(res[c]) * norm[c]                 for each of the H residual streams
//   lo      = silu((Down xn) / H)                        Down [R][H*E]
//   gate    = Up lo                                       Up   [H*E][R]
//   cur     = (1/H) sum_c xn[c] * sigmoid(gate[c])       the routed layer's input
//   inj     = Inject xn                                   Inject [H][H*E]
//   ... y = routed + shared experts of cur ...
//   res[c] += y * 2 sigmoid(inj[c] / H)
//
// Few tokens run on the CUDA cores (one warp per weight row, up to 8 tokens in registers, fp32
// accumulation). Many tokens take the Down and Up products through the tensor-core grouped GEMM
// (moe_gemm_kernel with the plain-matrix decoders); the norm, the SiLU, the mix, the injection
// weights and the combine stay here.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gx_dense.cuh"
#include "gx_device.cuh"
#include "gx_internal.h"

namespace gx {

using namespace dense;

namespace {

constexpr int kHcWarps = 4;
constexpr int kHcTok = 8;

// xn[t][c][:] = res[t][c][:] * rsqrt(mean(res[t][c]^2) + eps) * norm[c][:] (src/kernels.zig:281-291);
// one CTA per (token, stream).
__global__ void __launch_bounds__(256) hc_norm_kernel(HcArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x / a.H, c = blockIdx.x % a.H;
    const size_t base = (size_t)t * a.H * a.E + (size_t)c * a.E;
    __shared__ float red[8];
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < a.E; i += 1024) {
        const float4 v = *reinterpret_cast<const float4 *>(a.res + base + i);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float scale = 1.0f / sqrtf(tot / (float)a.E + a.eps);
    for (int i = threadIdx.x * 4; i < a.E; i += 1024) {
        const float4 v = *reinterpret_cast<const float4 *>(a.res + base + i);
        const float4 g = *reinterpret_cast<const float4 *>(a.norm + (size_t)c * a.E + i);
        *reinterpret_cast<float4 *>(a.xn + base + i) =
            make_float4(v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w);
    }
}

// Rows [row0, R + H) of (Down | Inject) against xn: lo[t][r] = silu(dot / H) for r < R,
// inj[t][r - R] = dot for the injection rows. One warp per row, 8 tokens at a time.
template <uint32_t WT>
__global__ void __launch_bounds__(kHcWarps * 32) hc_down_kernel(HcArgs a, int row0) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = row0 + blockIdx.x * kHcWarps + warp;
    if (r >= a.R + a.H) return;
    const bool inj = r >= a.R;
    const SharedMat &m = inj ? a.inject : a.down;
    const int row = inj ? r - a.R : r, HD = a.H * a.E;
    for (int t0 = 0; t0 < a.n_tok; t0 += kHcTok) {
        const int nt = min(kHcTok, a.n_tok - t0);
        float acc[kHcTok];
#pragma unroll
        for (int t = 0; t < kHcTok; ++t) acc[t] = 0.f;
        for (int c = lane * 8; c < HD; c += 256) {
            float w[8];
            load_w8<WT>(m, row, HD, c, w);
#pragma unroll
            for (int t = 0; t < kHcTok; ++t) {
                if (t < nt) {
                    float v[8];
                    load_x8(a.xn, 0, (size_t)(t0 + t) * HD + c, v);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[t] = fmaf(w[j], v[j], acc[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kHcTok; ++t) {
            if (t < nt) {
                const float s = warp_sum(acc[t]);
                if (lane == 0) {
                    if (inj) a.inj[(size_t)(t0 + t) * a.H + row] = s;
                    else a.lo[(size_t)(t0 + t) * a.R + row] = silu_ref(s / (float)a.H);
                }
            }
        }
    }
}

// cur[t][i] = (1/H) sum_c xn[t][c][i] * sigmoid(Up[c*E + i] . lo[t]); one warp per i.
template <uint32_t WT>
__global__ void __launch_bounds__(kHcWarps * 32) hc_up_mix_kernel(HcArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * kHcWarps + warp;
    if (i >= a.E) return;
    const int HD = a.H * a.E;
    for (int t0 = 0; t0 < a.n_tok; t0 += kHcTok) {
        const int nt = min(kHcTok, a.n_tok - t0);
        float out[kHcTok];
#pragma unroll
        for (int t = 0; t < kHcTok; ++t) out[t] = 0.f;
        for (int c = 0; c < a.H; ++c) {
            const int row = c * a.E + i;
            float g[kHcTok];
#pragma unroll
            for (int t = 0; t < kHcTok; ++t) g[t] = 0.f;
            for (int k = lane * 8; k < a.R; k += 256) {
                float w[8];
                load_w8<WT>(a.up, row, a.R, k, w);
#pragma unroll
                for (int t = 0; t < kHcTok; ++t) {
                    if (t < nt) {
                        float v[8];
                        load_x8(a.lo, 0, (size_t)(t0 + t) * a.R + k, v);
#pragma unroll
                        for (int j = 0; j < 8; ++j) g[t] = fmaf(w[j], v[j], g[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kHcTok; ++t) {
                if (t < nt) {
                    const float gt = warp_sum(g[t]);
                    out[t] += a.xn[(size_t)(t0 + t) * HD + row] * sigmoid_ref(gt);
                }
            }
        }
        if (lane == 0)
            for (int t = 0; t < nt; ++t) a.cur[(size_t)(t0 + t) * a.E + i] = out[t] / (float)a.H;
    }
}

// Tensor-core path: lo[t][r] = silu(Ylo[t][r] / H) from the Down GEMM's f16 rows (row stride Rp).
__global__ void __launch_bounds__(256) hc_lo_kernel(HcArgs a, const __half *Ylo, int Rp) {
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i >= (long long)a.n_tok * a.R) return;
    const int t = (int)(i / a.R), r = (int)(i % a.R);
    a.lo[i] = silu_ref(__half2float(Ylo[(size_t)t * Rp + r]) / (float)a.H);
}

// Tensor-core path: cur[t][i] = (1/H) sum_c xn[t][c][i] * sigmoid(gate[t][c][i]) from the Up GEMM's
// f16 rows.
__global__ void __launch_bounds__(256) hc_mix_kernel(HcArgs a, const __half *gate) {
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i >= (long long)a.n_tok * a.E) return;
    const int t = (int)(i / a.E), e = (int)(i % a.E);
    const size_t base = (size_t)t * a.H * a.E + e;
    float acc = 0.f;
    for (int c = 0; c < a.H; ++c)
        acc += a.xn[base + (size_t)c * a.E] * sigmoid_ref(__half2float(gate[base + (size_t)c * a.E]));
    a.cur[i] = acc / (float)a.H;
}

// res[t][c][i] += y[t][i] * 2 sigmoid(inj[t][c] / H).
__global__ void __launch_bounds__(256) hc_combine_kernel(HcArgs a, const float *y) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    const long long HD = (long long)a.H * a.E;
    if (i >= (long long)a.n_tok * HD) return;
    const int t = (int)(i / HD), c = (int)((i % HD) / a.E), e = (int)(i % a.E);
    const float w = 2.0f * sigmoid_ref(a.inj[(size_t)t * a.H + c] / (float)a.H);
    a.res_out[i] += y[(size_t)t * a.E + e] * w;
}

bool hc_shape_ok(const HcArgs &a) {
    return a.E > 0 && a.E % 256 == 0 && a.H >= 1 && a.H <= 8 && a.R > 0 && a.R % 128 == 0 &&
           (a.wt == W_Q8 || a.wt == W_F16);
}

}  // namespace

cudaError_t launch_hc_norm(const HcArgs &a, cudaStream_t s, bool pdl) {
    if (!hc_shape_ok(a)) return cudaErrorInvalidValue;
    if (a.n_tok == 0) return cudaSuccess;
    return launch_pdl(hc_norm_kernel, a.n_tok * a.H, 256, s, pdl, a);
}

cudaError_t launch_hc_down(const HcArgs &a, int row0, cudaStream_t s, bool pdl) {
    if (!hc_shape_ok(a)) return cudaErrorInvalidValue;
    if (a.n_tok == 0 || row0 >= a.R + a.H) return cudaSuccess;
    const int grid = (a.R + a.H - row0 + kHcWarps - 1) / kHcWarps;
    return a.wt == W_Q8 ? launch_pdl(hc_down_kernel<W_Q8>, grid, kHcWarps * 32, s, pdl, a, row0)
                        : launch_pdl(hc_down_kernel<W_F16>, grid, kHcWarps * 32, s, pdl, a, row0);
}

cudaError_t launch_hc_up_mix(const HcArgs &a, cudaStream_t s, bool pdl) {
    if (!hc_shape_ok(a)) return cudaErrorInvalidValue;
    if (a.n_tok == 0) return cudaSuccess;
    const int grid = (a.E + kHcWarps - 1) / kHcWarps;
    return a.wt == W_Q8 ? launch_pdl(hc_up_mix_kernel<W_Q8>, grid, kHcWarps * 32, s, pdl, a)
                        : launch_pdl(hc_up_mix_kernel<W_F16>, grid, kHcWarps * 32, s, pdl, a);
}

cudaError_t launch_hc_lo(const HcArgs &a, const __half *Ylo, int Rp, cudaStream_t s) {
    const long long n = (long long)a.n_tok * a.R;
    if (n == 0) return cudaSuccess;
    hc_lo_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, Ylo, Rp);
    return cudaGetLastError();
}

cudaError_t launch_hc_mix(const HcArgs &a, const __half *gate, cudaStream_t s) {
    const long long n = (long long)a.n_tok * a.E;
    if (n == 0) return cudaSuccess;
    hc_mix_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, gate);
    return cudaGetLastError();
}

cudaError_t launch_hc_combine(const HcArgs &a, const float *y, cudaStream_t s, bool pdl) {
    const long long n = (long long)a.n_tok * a.H * a.E;
    if (n == 0) return cudaSuccess;
    return launch_pdl(hc_combine_kernel, (int)((n + 255) / 256), 256, s, pdl, a, y);
}

}  // namespace gx
