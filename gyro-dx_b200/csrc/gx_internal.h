// gx_internal.h — launchers shared between the kernels (gx_kernels.cu) and the C ABI
// (gx_abi.cu). Host-only declarations.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gx {

// Error codes a kernel can leave in the context's device error word.
// KERR_RANGE: a layer output is not finite (an f16 operand or intermediate overflowed, or the
// input held Inf/NaN); the output writers record it.
enum : int { KERR_NONE = 0, KERR_WAIT = 1, KERR_BOUNDS = 2, KERR_RANGE = 3 };

// Shared-memory codebook copies of the decode-GEMV kernels (2 banks per copy, so at most two
// lanes of a warp contend for a bank during a lookup).
constexpr int kCodebookCopies = 16;

struct RouterArgs {
    const float *W;          // [NE][E] f32
    const float *bias;       // [NE] or nullptr
    const void *x;           // [n_tok][E]
    int x_bf16;
    int n_tok, NE, E, U;
    float scale;             // expert_weights_scale
    float norm_eps;          // > 0: route RMSNorm(x) (unit weight)
    float *ss;               // [n_tok] sum of squares of x (written when norm_eps > 0)
    int ss_from_x;           // selection computes the sum of squares from x itself (prefill)
    int logit_splits;        // > 1: logits holds that many split-K partials [split][n_tok][NE]
    float *xscale;           // [n_tok] per-token input scale (written by topk_kernel)
    float *logits;           // [n_tok][NE] scratch (raw W x, before scale and bias)
    uint32_t *ids;           // [n_tok][U]
    float *weights;          // [n_tok][U]
    int *err;
    // Selection in the router's last CTA (few tokens): every CTA counts itself done here, and the
    // last one selects the experts of every token and sets the counter back to 0. nullptr: a
    // separate selection kernel (or gate_up_kernel) selects.
    unsigned *done;
};

// Tokens up to which router_kernel selects the experts itself (in its last CTA).
constexpr int kRouterSelectTok = 4;

struct GateUpArgs {
    uint32_t type;
    const uint8_t *gate;     // tiles of local expert 0; expert e at + e * expert_bytes
    const uint8_t *up;
    uint64_t expert_bytes;   // tiles of one projection of one expert
    const void *x;           // [n_tok][E]
    int x_bf16;
    const float *signs;      // [E] or nullptr
    const float *xscale;     // [n_tok] input scale from topk_kernel, or nullptr (unfused only)
    const uint32_t *ids;     // [n_slots] local expert of each slot (unfused only)
    float *act;              // [n_slots][F] silu(gate) * up
    const uint32_t *codebook;// 2048 words in global memory
    const uint32_t *codebook_image;  // the shared-memory codebook image (kCodebookCopies copies)
    int E, F, U, n_slots, n_expert;
    int *err;
    // Fused selection (few tokens): each CTA selects the experts of its own tokens from the
    // router's raw logits, and the CTA holding a token's first unit publishes ids/weights.
    int fused_topk;
    const float *logits;     // [n_tok][NE] raw W x
    const float *bias;       // [NE] or nullptr
    const float *ss;         // [n_tok] sum of squares of x (norm_eps > 0)
    int NE;
    float norm_eps, wscale;  // RMSNorm epsilon (0: none), expert_weights_scale
    uint32_t *ids_out;       // [n_tok][U]
    float *weights_out;      // [n_tok][U]
};

// Whether gate_up_kernel can select experts itself for n_tok tokens (at most 8 tokens per CTA).
bool gate_up_fuses_topk(int E, int F, int U, int n_tok, int sm_count);

// ---- the shared expert of a layer (src/engine.zig:644-653) -----------------------------------
// Device encodings of its three plain row-major matrices: Q8_0 split into int8 weights
// [rows][cols] and fp16 block scales [rows][cols/32] (one per 32 weights), or fp16 weights
// [rows][cols] (bf16 and f32 matrices are converted at upload). The values double as the
// weight "type" of moe_gemm_kernel's shared-expert decoders; they are not Gyro type ids.
enum : uint32_t { W_F16 = 1, W_Q8 = 8 };

struct SharedMat {
    const uint8_t *w;        // int8 (W_Q8) or fp16 (W_F16) weights [rows][cols]
    const __half *d;         // W_Q8: fp16 scales [rows][cols/32]; nullptr for W_F16
};

// Decode path (few tokens, CUDA cores): act = silu(Gate x) * Up x and the gate logits, then
// y = sigmoid(logit) * Down act, an f32 [n_tok][E] term the routed down kernel adds.
struct SharedArgs {
    uint32_t wt;             // W_Q8 or W_F16
    SharedMat gate, up, down;
    const float *gate_inp;   // [E] f32
    const void *x;           // [n_tok][E] layer input (unrotated)
    int x_bf16;
    // RMSNorm scale of token t: xscale[t] when given, else 1/sqrt(ss[t]/E + norm_eps) when
    // norm_eps > 0 (ss from the router), else 1
    const float *xscale;
    const float *ss;
    float norm_eps;
    int n_tok, E, SF;
    float *act;              // [n_tok][SF]
    float *logit;            // [n_tok] gate_inp . (x * xscale)
    float *y;                // [n_tok][E]
};
cudaError_t launch_shared_gate_up(const SharedArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_shared_down(const SharedArgs &a, cudaStream_t s, bool pdl);
// Only the gate logits (the tensor-core path computes the rest with moe_gemm_kernel).
cudaError_t launch_shared_logits(const SharedArgs &a, cudaStream_t s);
// Tile list of the shared expert on the tensor-core path: every token in order, 128 per tile.
cudaError_t launch_shared_tiles(int n_tok, int *tile_expert, int *tile_rows, int *n_mtiles, cudaStream_t s);

// Hyper-connection mixer of the FFN block (H residual streams of E, low rank R).
struct HcArgs {
    uint32_t wt;             // W_Q8 or W_F16
    SharedMat down;          // [R][H*E]
    SharedMat up;            // [H*E][R]
    SharedMat inject;        // [H][H*E]
    const float *norm;       // [H*E] per-stream RMSNorm weights
    float eps;
    int n_tok, H, E, R;
    const float *res;        // [n_tok][H*E] residual streams (read by the norm)
    float *res_out;          // the same streams, updated by the combine
    float *xn;               // [n_tok][H*E] normed streams
    float *lo;               // [n_tok][R]
    float *inj;              // [n_tok][H]
    float *cur;              // [n_tok][E] the routed layer's input
};
cudaError_t launch_hc_norm(const HcArgs &a, cudaStream_t s, bool pdl);
// Rows [row0, R + H) of Down | Inject on the CUDA cores (row0 = R: the injection rows alone).
cudaError_t launch_hc_down(const HcArgs &a, int row0, cudaStream_t s, bool pdl);
cudaError_t launch_hc_up_mix(const HcArgs &a, cudaStream_t s, bool pdl);
// Tensor-core path: lo from the Down GEMM's f16 rows (stride Rp), cur from the Up GEMM's f16 rows.
cudaError_t launch_hc_lo(const HcArgs &a, const __half *Ylo, int Rp, cudaStream_t s);
cudaError_t launch_hc_mix(const HcArgs &a, const __half *gate, cudaStream_t s);
cudaError_t launch_hc_combine(const HcArgs &a, const float *y, cudaStream_t s, bool pdl);

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
    const float *extra;      // [n_tok][E] or nullptr: the gated shared-expert term, added too
    void *out;               // [n_tok][E]
    int out_bf16;
    const uint32_t *codebook;
    const uint32_t *codebook_image;  // the shared-memory codebook image (kCodebookCopies copies)
    int E, F, U, n_tok, n_expert;
    int *err;
};

// ---- prefill (many tokens): grouping, row packing, tcgen05 grouped GEMM, combine ----------
struct GroupArgs {
    const uint32_t *ids;     // [n_slots] expert of each slot (local numbering)
    int n_slots, NE;
    int *expert_count;       // [NE]
    int *cursor;             // [NE] scratch: next free padded row of each expert
    int *tile_expert;        // [max_tiles] expert of each 128-row tile
    int *tile_rows;          // [max_tiles] valid rows in the tile
    int *n_mtiles;           // [1]
    int *row_slot;           // [max_tiles * 128] slot of each valid padded row
    int *slot_row;           // [n_slots] padded row of each slot
    int *err;
};

struct PackArgs {
    const void *src;         // by_token: x [n_tok][K]; else act [padded rows][K]
    int src_bf16;
    int by_token, U, K;
    const float *xscale;     // by_token: [n_tok] per-token scale; else [padded rows] row scale, or nullptr
    const __half *xh;        // by_token: rotated f16 token rows [n_tok][K] (rotate_tokens)
    const float *signs;      // [K] or nullptr (then no Hadamard transform)
    const int *row_slot, *tile_rows, *n_mtiles;
    uint8_t *dst;            // [tiles][K/64][16384] f16 swizzled
    int compact;             // k-step blocks of rows16(tile rows) x 128 B each, back to back
                             // (moe_gemm_ts_kernel), instead of 16384 B each
};

// Token rotation fused with the token pack (single-GPU many-token path): each token is rotated
// once and its f16 row written straight into the tile row of each of its slots.
struct RotPackArgs {
    const void *x;
    int x_bf16;
    const float *xscale;     // [n_tok] per-token scale, or nullptr
    const float *signs;      // [E] or nullptr (then no Hadamard transform)
    int n_tok, E, U;
    const int *slot_row;     // [n_tok * U] padded row of each slot, -1 for none
    const int *tile_rows;    // rows of each 128-row tile
    uint8_t *dst;            // token tiles [tiles][E/64][16384]
    int compact;             // as PackArgs::compact
};

struct GemmArgs {
    uint32_t type;           // Gyro type id, or W_Q8 / W_F16 for the shared expert's matrices
    const uint8_t *w0, *w1;  // gate + up (mode 0) or down (mode 1) tiles of local expert 0
    const __half *d0, *d1;   // W_Q8: block scales of w0 / w1
    uint64_t expert_bytes;   // tiles of one projection of one expert
    int K, n_ntiles, n_expert;
    const uint8_t *A;        // packed operand tiles [tile][K/64][16384]
    const int *tile_expert, *tile_rows, *n_mtiles;
    float *act;              // mode 0 output [tiles*128][F]
    int F;
    __half *Y;               // mode 1 output [tiles*128][E]
    int E;
    const uint32_t *codebook;
    int *err;
    // moe_gemm_ts_kernel, mode 0: when set, the epilogue writes the down GEMM's operand tiles
    // (act * down signs, 128-point Hadamard per block, f16, compact layout of pack_rows_kernel)
    // instead of act
    uint8_t *down_A;
    const float *down_signs;
};

struct CombineArgs {
    const __half *Y;
    const int *slot_row;
    const float *weights;
    const __half *Ysh;       // [n_tok][E] shared-expert rows, or nullptr
    const float *sh_logit;   // [n_tok] their gate logits (added as sigmoid(logit) * Ysh)
    const void *resid;
    int resid_bf16;
    void *out;
    int out_bf16;
    int out_f16;             // f16 output (expert-parallel partial rows); overrides out_bf16
    int n_tok, U, E;
    int *err;                // KERR_RANGE when an output is not finite (or beyond f16 for out_f16)
};

cudaError_t launch_router_gemm(const float *W, const void *x, int x_bf16, int n_tok, int NE, int E, float *C,
                               int splits, cudaStream_t s);
// Router GEMM on tcgen05 (gx_router_tc.cu): wparts holds the router as three bf16 parts in
// 128-expert x 64-column swizzled tiles (router_parts_bytes); logits are [splits][n_tok][NE].
size_t router_parts_bytes(int NE, int E);
int router_tc_splits(int n_tok, int NE, int E, int sm_count);
cudaError_t launch_router_tc(const void *x, int x_bf16, int n_tok, int NE, int E, const uint8_t *wparts,
                             float *logits, int splits, int *err, cudaStream_t s);
cudaError_t launch_rotate_tokens(const void *x, int x_bf16, const float *xscale, const float *signs, int n_tok,
                                int E, __half *xh, cudaStream_t s, const int *scatter = nullptr, int n_dst = 0);

// ---- decode stack as one persistent cooperative kernel (gx_decode_stack.cu) ----------------
struct StackLayer {
    const float *router;     // [NE][E]
    const float *bias;       // [NE]
    const float *gate_signs; // [E] or nullptr
    const float *down_signs; // [F] or nullptr
    const uint8_t *gate, *up, *down;
    uint64_t gate_expert_bytes, down_expert_bytes;
    float scale;             // expert_weights_scale
};

struct StackArgs {
    const StackLayer *layers;  // device table, n_layers entries
    int n_layers;
    const void *x;           // [n_tok][E] input
    int x_bf16;
    void *out;               // [n_tok][E] output of the last layer
    int out_bf16;
    float *xa, *xb;          // [n_tok][E] f32 inputs of the inner layers
    float *logits;           // [n_tok][NE]
    float *act;              // [n_tok * U][F]
    const uint32_t *codebook;
    unsigned *sync;          // grid-barrier counter, zeroed by the launcher
    int n_tok, NE, E, F, U;
    float norm_eps;          // > 0: experts and router see RMSNorm(x)
    int residual;            // 1: x_{l+1} = x_l + MoE_l(.); 0: out = MoE(x)
    int *err;
};

bool decode_stack_supported(uint32_t type, int E, int F, int U, int NE, int n_tok);
cudaError_t launch_decode_stack(const StackArgs &a, uint32_t type, int sm_count, cudaStream_t s);

// ---- expert parallelism: dispatch plan and the source-side sum of returned rows ----------
// Slot id meaning "no expert of this rank" in expert-parallel rows.
constexpr uint32_t kNoSlot = 0xffffffffu;

// Expert-parallel groups hold at most kMaxEpWorld ranks; the plan handles kPlanTok tokens per CTA.
constexpr int kMaxEpWorld = 64;
constexpr int kPlanTok = 256;
inline int ep_plan_ctas(int n_tok) { return (n_tok + kPlanTok - 1) / kPlanTok; }

struct EpPlanArgs {
    const uint32_t *ids;     // [n_tok][U] global expert ids from the selection
    const float *weights;    // [n_tok][U]
    int n_tok, U, NE, W;     // without a route table rank d serves experts [d*NE/W, (d+1)*NE/W)
    int rank;                // this rank (route entries with rank -1 mean "here")
    const int2 *route;       // [NE] (serving rank or -1, local expert id there), or nullptr
    unsigned *expert_count;  // [NE] slots routed to each expert, accumulated, or nullptr
    int stride;              // send-buffer rows reserved per destination (>= n_tok)
    int pad_rows;            // rows [count, pad_rows) of every destination are marked empty
    int *pos_of;             // [n_tok][W] send row of (token, destination), -1 if none
    uint32_t *send_ids;      // [W*stride][U] destination-local expert id or kNoSlot
    float *send_w;           // [W*stride][U] routing weight (0 for kNoSlot)
    int *send_count;         // [W] rows per destination
    uint64_t *dest_mask;     // [n_tok] scratch: bit d set if rank d serves one of the token's slots
    int *block_count;        // [ep_plan_ctas(n_tok)][kMaxEpWorld] scratch: marked tokens per CTA
    int *err;
};

struct EpCombineArgs {
    const __half *ret;       // returned partial rows, laid out as the send buffer
    const int *pos_of;       // [n_tok][W]
    int W;
    const __half *Ysh;       // [n_tok][E] this rank's shared-expert rows, or nullptr
    const float *sh_logit;   // [n_tok]
    const void *resid;       // [n_tok][E] or nullptr
    int resid_bf16;
    void *out;               // [n_tok][E]
    int out_bf16;
    int n_tok, E;    int *err;                // KERR_RANGE when an output is not finite
};

// ---- expert-parallel exchange over NVLink peer memory -------------------------------------
// Every rank owns one exchange block, mapped into every other rank by CUDA IPC, laid out alike
// on all ranks for W ranks, up to T rows per source and E, U of the largest layer:
//   rx_rows [W src][T][E] f16 | rx_ids [W][T][U] | rx_w [W][T][U] | ret_rows [W dst][T][E] f16 |
//   rx_count [W] | rx_flag [W] | ret_flag [W] | done [2] | status [1]
// A call uses the first S <= T rows of every source's region, S = the largest token count of any
// rank in that call (every rank knows all counts), so the rows a call touches are [W][S]
// contiguous. A flag holds the epoch (layer call number) of the last transfer from that rank;
// kFlagFailed set beside the epoch means that rank's side of the exchange failed (an expired
// wait), and the rank that reads it fails the call too instead of using the rows.
constexpr int kMaxPeers = 16;
constexpr unsigned kFlagFailed = 0x80000000u;

struct EpBlock {
    size_t rx_rows, rx_ids, rx_w, ret_rows, rx_count, rx_flag, ret_flag, done, status, bytes;
};
EpBlock ep_block_layout(int W, int T, int E, int U);

struct EpPeerArgs {
    uint8_t *peer[kMaxPeers];  // every rank's exchange block in this process's address space
    EpBlock off;
    int W, rank;
    int T;                     // row stride of a source's region in this call (S above)
    int E, U;
    unsigned epoch;            // < kFlagFailed
    uint64_t wait_ns;          // bound of every flag wait
    int *err;
};

// Rotated f16 rows of this rank's tokens straight into the destinations' rx regions (row
// positions from the plan, stride T), the slot metadata beside them (rows [count, T) of every
// destination marked kNoSlot), then count + flag per destination from the last CTA.
struct EpPushArgs {
    EpPeerArgs p;
    const void *x;
    int x_bf16, n_tok;
    const float *xscale;     // [n_tok] or nullptr
    const float *signs;      // [E] or nullptr
    const int *pos_of;       // [n_tok][W] = d * T + position, or -1
    const uint32_t *send_ids;
    const float *send_w;     // [W * T][U] plan output
    const int *send_count;   // [W]
};

cudaError_t launch_ep_plan(const EpPlanArgs &a, cudaStream_t s);
cudaError_t launch_ep_push(const EpPushArgs &a, cudaStream_t s);
// Waits (bounded) for every source's flag of this epoch. A source whose wait expires or whose
// flag carries kFlagFailed gives KERR_WAIT, its rows are marked as carrying no slot, and the
// block's status word records the failure for ep_return.
cudaError_t launch_ep_wait_rx(const EpPeerArgs &a, cudaStream_t s);
// Weighted sum of the U expert rows of every received row (Y, slot_row as the combine kernel)
// written as f16 into the source's ret region, then a flag per source from the last CTA. After a
// failed receive it writes no rows and publishes the epoch with kFlagFailed, so every source
// fails the call as well.
cudaError_t launch_ep_return(const EpPeerArgs &a, const __half *Y, const int *slot_row, cudaStream_t s);
// Waits (bounded) for every destination's return flag of this epoch (kFlagFailed: KERR_WAIT).
cudaError_t launch_ep_wait_ret(const EpPeerArgs &a, cudaStream_t s);
cudaError_t launch_ep_combine(const EpCombineArgs &a, cudaStream_t s);
cudaError_t launch_group(const GroupArgs &a, cudaStream_t s);
cudaError_t launch_pack_rows(const PackArgs &a, int max_tiles, cudaStream_t s);
cudaError_t launch_rotate_pack(const RotPackArgs &a, cudaStream_t s);
cudaError_t launch_moe_gemm(const GemmArgs &a, int mode, int sm_count, cudaStream_t s);
// The routed experts' grouped GEMM with the decoded weights in tensor memory (gx_gemm_ts.cu):
// launch_moe_gemm uses it for the Gyro types (gemm_ts_routed) unless GX_GEMM_SMEM=1 selects
// moe_gemm_kernel; its token tiles are packed compact (PackArgs::compact).
bool gemm_ts_routed(uint32_t type);
// Programmatic dependent launch of the many-token chain's kernels, chosen per forward call by the
// calling thread (launch_chain in gx_device.cuh).
bool chain_pdl_enabled();
void set_chain_pdl(bool on);
bool gemm_ts_supports(const GemmArgs &a, int mode);
cudaError_t launch_moe_gemm_ts(const GemmArgs &a, int mode, int sm_count, cudaStream_t s);
cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s);

struct MatvecArgs {
    uint32_t type;
    const uint8_t *tiles;
    const float *x;          // [n_tok][cols]
    float *y;                // [n_tok][rows]
    const uint32_t *codebook;
    int rows, cols, n_tok;
    int *err;
};

// pdl: launch with programmatic stream serialization (overlap with the previous kernel).
// with_topk: also launch the per-token selection kernel (when gate_up does not fuse it).
cudaError_t launch_router(const RouterArgs &a, cudaStream_t s, bool pdl, bool with_topk);
// Per-token selection (one warp per token) from raw logits.
cudaError_t launch_topk(const RouterArgs &a, cudaStream_t s);
cudaError_t launch_gate_up(const GateUpArgs &a, int sm_count, cudaStream_t s, bool pdl);
cudaError_t launch_down(const DownArgs &a, int sm_count, cudaStream_t s, bool pdl);
cudaError_t launch_matvec(const MatvecArgs &a, int sm_count, cudaStream_t s);
cudaError_t launch_repack(uint32_t type, const uint8_t *raw, uint64_t row_bytes, uint32_t rows,
                          uint32_t cols, uint8_t *tiles, cudaStream_t s);
cudaError_t launch_decode_blocks(uint32_t type, const uint8_t *packed, uint32_t nblocks,
                                 const uint16_t *codebook, float *out, cudaStream_t s);
cudaError_t launch_residual_copy(const void *x, int x_bf16, float *out, size_t n, cudaStream_t s);

}  // namespace gx
