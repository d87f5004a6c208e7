// gx_internal.h — launchers shared between the kernels (gx_kernels.cu) and the C ABI
// (gx_abi.cu). Host-only declarations.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gx {

// Shared-memory codebook copies used by the decode-GEMV kernels.
constexpr int kCodebookCopies = 16;

struct RouterArgs {
    const float *W;          // [NE][E] f32
    const float *bias;       // [NE] or nullptr
    const void *x;           // [n_tok][E]
    int x_bf16;
    int n_tok, NE, E, U;
    float scale;             // expert_weights_scale
    float *logits;           // [n_tok][NE] scratch
    uint32_t *ids;           // [n_tok][U]
    float *weights;          // [n_tok][U]
    unsigned *counter;       // zero at rest; reset by the last CTA
    int *err;
};

struct GateUpArgs {
    uint32_t type;
    const uint8_t *gate;     // tiles of local expert 0; expert e at + e * expert_bytes
    const uint8_t *up;
    uint64_t expert_bytes;   // tiles of one projection of one expert
    const void *x;           // [n_tok][E]
    int x_bf16;
    const float *signs;      // [E] or nullptr
    const uint32_t *ids;     // [n_slots] local expert of each slot
    float *act;              // [n_slots][F] silu(gate) * up
    const uint32_t *codebook;// 2048 words in global memory
    int E, F, U, n_slots, n_expert;
    int *err;
};

struct DownArgs {
    uint32_t type;
    const uint8_t *down;     // tiles of local expert 0
    uint64_t expert_bytes;
    const float *act;        // [n_slots][F]
    const float *signs;      // [F] or nullptr
    const uint32_t *ids;     // [n_tok][U]
    const float *weights;    // [n_tok][U]
    const void *resid;       // [n_tok][E] or nullptr (residual added to the output)
    int resid_bf16;
    void *out;               // [n_tok][E]
    int out_bf16;
    const uint32_t *codebook;
    int E, F, U, n_tok, n_expert;
    int *err;
};

struct MatvecArgs {
    uint32_t type;
    const uint8_t *tiles;
    const float *x;          // [n_tok][cols]
    float *y;                // [n_tok][rows]
    const uint32_t *codebook;
    int rows, cols, n_tok;
    int *err;
};

cudaError_t launch_router(const RouterArgs &a, cudaStream_t s);
cudaError_t launch_gate_up(const GateUpArgs &a, int sm_count, cudaStream_t s);
cudaError_t launch_down(const DownArgs &a, int sm_count, cudaStream_t s);
cudaError_t launch_matvec(const MatvecArgs &a, int sm_count, cudaStream_t s);
cudaError_t launch_repack(uint32_t type, const uint8_t *raw, uint64_t row_bytes, uint32_t rows,
                          uint32_t cols, uint8_t *tiles, cudaStream_t s);
cudaError_t launch_decode_blocks(uint32_t type, const uint8_t *packed, uint32_t nblocks,
                                 const uint16_t *codebook, float *out, cudaStream_t s);
cudaError_t launch_residual_copy(const void *x, int x_bf16, float *out, size_t n, cudaStream_t s);

}  // namespace gx
