/*
 * gyro_moe.h — C ABI of the B200 (sm_100a) routed-expert MoE layer for Gyro trellis experts.
 *
 * Drop-in replacement, for the routed-MoE path, of the Direct3D 12 bridge of mattneel/gyro-dx:
 * native/include/gyro_native.h:65-137 (mirrored in Zig by src/native_abi.zig:50-95 and wrapped
 * by src/gpu.zig). The Zig caller is Engine.ffn (src/gpu_engine.zig:1052-1119); the tensors it
 * hands over are the Matrix.data slices of src/model.zig:97-124 (stacked expert tensors, rows of
 * packed 128-weight Gyro blocks), unchanged.
 *
 * Conventions kept from gyro_native.h:65-70:
 *   - every call returns int32, negative = failure (GX_E_*), 0 = success;
 *   - a context is used by one thread at a time (serialized access per context);
 *   - every blocking call takes timeout_ms and returns GX_E_TIMEOUT instead of hanging;
 *   - a failed or timed-out destroy keeps the handle valid for a retry;
 *   - structs are plain C with fixed layouts (sizes asserted in the Zig mirror);
 *   - work is enqueued asynchronously; tickets are monotonic u64 (gd_submit,
 *     native/gyro_native.cpp:919-934) and become complete in order.
 * Device pointers are CUDA device addresses of the context's device; host pointers are plain
 * process memory (pinned or pageable).
 */
#ifndef GYRO_MOE_H
#define GYRO_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32) && defined(GX_EXPORTS)
#define GX_API __declspec(dllexport)
#elif defined(_WIN32)
#define GX_API __declspec(dllimport)
#else
#define GX_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GX_ABI_VERSION 1u

typedef struct gx_context gx_context;
typedef int32_t gx_result;

enum {
    GX_OK = 0,
    GX_E_INVALIDARG = -1,   /* bad pointer, size, type id, layer index or shape */
    GX_E_OUTOFMEMORY = -2,  /* device or pinned host allocation failed */
    GX_E_TIMEOUT = -3,      /* a blocking call reached timeout_ms; the work is still queued */
    GX_E_DEVICE = -4,       /* CUDA reported an error; the context should be destroyed */
    GX_E_UNSUPPORTED = -5,  /* device is not sm_100 or the request is not supported */
    GX_E_STATE = -6,        /* call out of order (layer not uploaded, context closed) */
    GX_E_MISMATCH = -7,     /* gx_decode_blocks: an output differs from the expected bits */
    GX_E_COMM = -8,         /* NCCL failure or peer loss in the expert-parallel group */
    GX_E_KERNEL = -9,       /* a kernel's bounded wait expired; its outputs are invalid */
    GX_E_RANGE = -10        /* a layer output is not finite: the input held Inf/NaN, or an
                               activation outgrew the f16 operands of the tensor-core path (or the
                               f16 hi/lo split of the decode path); the outputs are invalid */
};

/* Activation encodings, and the weight encodings of a shared expert (the type ids of
 * src/kernels.zig:7-10). */
enum { GX_F32 = 0, GX_Q8_0 = 8, GX_BF16 = 30 };

/* Options: mirrors the role of gd_options (native/include/gyro_native.h:25-31). */
enum {
    GX_FLAG_PROFILE = 1u      /* record per-phase device times (gx_read_timings) */
};

typedef struct gx_options {
    uint32_t device;          /* CUDA device ordinal */
    uint32_t rank;            /* expert-parallel rank in [0, world) */
    uint32_t world;           /* expert-parallel group size, 1..64; 1 = single GPU */
    uint32_t max_tokens;      /* largest n_tok of one forward call on this rank */
    uint32_t max_layers;      /* number of layer slots (gx_upload_layer indices) */
    uint32_t flags;           /* GX_FLAG_* */
    const void *codebook;     /* the normative 8192-byte table (src/gyro_codebook.f16) */
    uint64_t codebook_bytes;  /* must be 8192 */
    uint8_t nccl_id[128];     /* ncclUniqueId from rank 0 when world > 1, else ignored */
} gx_options;                 /* 168 bytes */

/* Replaces gd_caps (native/include/gyro_native.h:33-46). */
typedef struct gx_caps {
    uint32_t abi_version;
    uint32_t sm_count;
    uint32_t cc_major, cc_minor;
    uint32_t rank, world;
    uint32_t max_tokens, max_layers;
    uint64_t hbm_bytes;       /* total device memory */
    uint64_t free_bytes;      /* free device memory now */
    uint64_t l2_bytes;
    uint64_t arena_bytes;     /* bytes held by uploaded layers on this device */
    char device_name[120];
    uint32_t ep_exchange;     /* expert-parallel rows: GX_EP_NONE until the first layer, then one of
                                 GX_EP_PEER (NVLink peer memory) or GX_EP_NCCL */
    uint32_t ep_peer_layers;  /* layer calls so far whose rows crossed by NVLink peer memory */
} gx_caps;                    /* 192 bytes */

#define GX_EP_NONE 0u
#define GX_EP_NCCL 1u
#define GX_EP_PEER 2u

/* One routed-expert layer as the Zig host holds it (src/model.zig:97-124, :408-421). */
typedef struct gx_layer_desc {
    uint32_t type_id;             /* Gyro type of gate/up/down, 144..151 */
    uint32_t n_expert;            /* experts in the layer (<= 512) */
    uint32_t n_embd;              /* E: hidden width, multiple of 128 */
    uint32_t n_ff;                /* F: expert FFN width, multiple of 128 */
    uint32_t n_used;              /* U: experts per token (top-k), 1..16 */
    float expert_weights_scale;   /* applied unless 0 or 1 (src/engine.zig:538) */
    const void *gate;             /* [n_expert*F rows][E/128 blocks] packed, host memory */
    const void *up;               /* same shape as gate */
    const void *down;             /* [n_expert*E rows][F/128 blocks] packed, host memory */
    uint64_t gate_bytes, up_bytes, down_bytes;
    const float *router;          /* [n_expert][E] f32, host memory */
    const float *gate_signs;      /* [E] +-1, or NULL when the experts are not rotated */
    const float *up_signs;        /* must equal gate_signs (src/gpu_engine.zig:404) or be NULL */
    const float *down_signs;      /* [F] +-1, or NULL */
    const float *router_bias;     /* [n_expert] additive logit bias, or NULL (benchmark hook:
                                     skewed expert popularity; no reference counterpart) */
} gx_layer_desc;

/* The shared expert of a routed layer and its sigmoid gate, as the Zig host binds them
 * (ffn_{gate,up,down}_shexp and ffn_gate_inp_shexp, src/model.zig:418-421). Plain row-major
 * matrices in one of the encodings the reference GPU engine multiplies them in
 * (src/gpu_engine.zig:846-850): GX_Q8_0 (blocks of an fp16 scale and 32 int8), GX_BF16 or GX_F32.
 * On the device Q8_0 stays Q8_0; bf16 and f32 matrices are stored as fp16 (bf16 values convert
 * exactly within the fp16 range, f32 values are rounded once). */
typedef struct gx_shared_desc {
    uint32_t type_id;             /* GX_Q8_0, GX_BF16 or GX_F32 */
    uint32_t n_ff;                /* SF = n_ff_shexp: multiple of 128, at most 4096 */
    const void *gate;             /* [SF rows][n_embd], host memory */
    const void *up;               /* [SF][n_embd] */
    const void *down;             /* [n_embd rows][SF] */
    uint64_t gate_bytes, up_bytes, down_bytes;
    const float *gate_inp;        /* [n_embd] f32 weights of the sigmoid gate */
} gx_shared_desc;

/* Per-phase device times, in nanoseconds, of the most recent forward call (gx_moe_forward*, or
 * all layers of the most recent gx_stack_forward*) on a context created with GX_FLAG_PROFILE.
 * Measured with CUDA events recorded on the context's stream between the kernels (inside the
 * captured graph for stacks). Replaces gd_timestamp / gd_read_timestamps and the phase marks of
 * Engine.mark (native/gyro_native.cpp:911-917, src/gpu_engine.zig:150-166). */
typedef struct gx_timings {
    uint64_t router_ns;     /* router GEMV + softmax/top-k */
    uint64_t gate_up_ns;    /* fused decode gate/up GEMV + SwiGLU */
    uint64_t down_ns;       /* fused decode down GEMV + weighted combine */
    uint64_t experts_ns;    /* gate_up_ns + down_ns (+ dispatch/combine when world > 1) */
    uint64_t total_ns;
    uint64_t layers;        /* layers covered by these sums */
} gx_timings;

/* Opens a context on one device (replaces gd_create, native/include/gyro_native.h:71).
 * With world > 1 every rank (one process or thread per GPU) calls it with the same nccl_id, and
 * the call returns once all ranks have joined (GX_E_COMM if they have not within the
 * communication timeout: GX_COMM_TIMEOUT_MS in the environment, default 120000). Experts are
 * then sharded: rank r holds experts [r*n_expert/world, (r+1)*n_expert/world) of every layer,
 * and every forward call is a collective (see gx_moe_forward). NCCL (libnccl.so.2) is loaded
 * only for world > 1; GX_E_UNSUPPORTED if it cannot be found. */
GX_API gx_result gx_create(const gx_options *options, gx_context **out_context);

/* No counterpart in the reference (its bridge drives one GPU). Writes a new NCCL unique id
 * (bytes must be 128) for gx_options.nccl_id: rank 0 calls it and hands the bytes to the other
 * ranks over the host's own channel. */
GX_API gx_result gx_comm_unique_id(uint8_t *out_id, uint64_t bytes);

/* Replaces gd_get_caps (native/include/gyro_native.h:72). */
GX_API gx_result gx_get_caps(gx_context *context, gx_caps *out_caps);

/* Copies one layer's router, signs and (local) experts from host memory into this device's
 * HBM arena; the caller keeps ownership of its buffers. Replaces the resident-expert upload
 * of Engine.setupExperts / loadBundle and the sign/codebook upload
 * (src/gpu_engine.zig:447-458, :593-668). Blocking. */
GX_API gx_result gx_upload_layer(gx_context *context, uint32_t layer, const gx_layer_desc *desc,
                                 uint32_t timeout_ms);

/* Adds the shared expert to an uploaded layer (desc NULL removes it). From then on every forward
 * call of the layer returns ffn_out instead of ffn_moe_out (src/engine.zig:642-653):
 *   y[t] = routed[t] + sigmoid(gate_inp . x[t]) * Down(silu(Gate x[t]) * Up x[t])
 * with x the layer input (unrotated). gx_upload_layer of the same index removes it again. With
 * world > 1 every rank holds the whole shared expert and computes it for its own tokens (it is
 * not exchanged). Needs n_embd to be a multiple of 256. Blocking. No counterpart function in the
 * reference bridge: its host binds these tensors next to the routed ones (src/gpu_engine.zig:
 * 397-401) and multiplies them with its generic mv (:1061-1063, :1074). */
GX_API gx_result gx_upload_shared(gx_context *context, uint32_t layer, const gx_shared_desc *desc,
                                  uint32_t timeout_ms);

/* ---- the FFN block with its hyper-connection mixer -----------------------------------------
 * The reference model keeps hc residual streams per token and reaches each routed layer through a
 * low-rank mixer (src/engine.zig:162-165, :184-228; src/gpu_engine.zig:891-928 with the hc_pre /
 * hc_post / hc_mix / hc_combine kernels of its engine shaders). The mixer weights of one layer's
 * FFN block are blk.L.hc_ffn_{norm,down,up,inject}.weight (src/model.zig:361-366) in one
 * non-expert encoding: GX_Q8_0, GX_BF16 or GX_F32 (stored on the device as for the shared expert). */
typedef struct gx_hc_desc {
    uint32_t n_streams;           /* hc: 1..8 residual streams of n_embd each (HD = hc * n_embd) */
    uint32_t rank;                /* hc_rank: multiple of 64, at most 4096 (320 in the reference model) */
    uint32_t type_id;             /* GX_Q8_0, GX_BF16 or GX_F32 of down / up / inject */
    float eps;                    /* RMSNorm epsilon of the per-stream norm */
    const float *norm;            /* [HD] f32 per-stream norm weights, host memory */
    const void *down;             /* [rank rows][HD], host memory */
    const void *up;               /* [HD rows][rank] */
    const void *inject;           /* [hc rows][HD] */
    uint64_t down_bytes, up_bytes, inject_bytes;
} gx_hc_desc;

/* Attaches the FFN block's mixer to an uploaded layer (desc NULL removes it). Needs n_embd to be a
 * multiple of 256. Blocking. No counterpart function in the reference bridge: its host binds these
 * tensors with the rest of the layer (src/gpu_engine.zig:351-354). */
GX_API gx_result gx_upload_hc(gx_context *context, uint32_t layer, const gx_hc_desc *desc, uint32_t timeout_ms);

/* One FFN block on device-resident residual streams, enqueued on the context's stream:
 *   cur, inj = hcMix(res)        xn_c = RMSNorm(res_c) * norm_c, lo = silu(Down xn / hc),
 *                                cur = mean_c xn_c * sigmoid((Up lo)_c), inj = Inject xn
 *   y = the layer on cur         routed experts (+ shared expert), as gx_moe_forward
 *   res_c += y * 2 sigmoid(inj_c / hc)
 * res: [n_tok][hc * n_embd] f32 device, updated in place. mixed: optional device [n_tok][n_embd]
 * f32 output of cur (the hc_mixed observation, src/engine.zig:210), or NULL. The layer needs
 * gx_upload_hc. With world > 1 it is a collective like gx_moe_forward (the mixer itself runs on
 * each rank's own tokens). out_ticket: optional; completes when res is written. */
GX_API gx_result gx_ffn_block(gx_context *context, uint32_t layer, float *res, uint32_t n_tok, float *mixed,
                              uint64_t *out_ticket);

/* ---- layers from a GGUF model file ---------------------------------------------------------
 * Replaces, for this path, the Zig host's GGUF reader and tensor binding (src/gguf.zig:263-334,
 * src/model.zig:395-421) and its expert-arena setup (src/gpu_engine.zig:593-668). Layer L of the
 * file is blk.L.ffn_{gate,up,down}_exps.weight (one Gyro type, stacked experts [E,F,NE] / [F,E,NE]),
 * blk.L.ffn_gate_inp.weight (router [E,NE], f32, f16 or bf16), optionally the shared expert
 * blk.L.ffn_{gate,up,down}_shexp.weight and blk.L.ffn_gate_inp_shexp.weight, with U from
 * <general.architecture>.expert_used_count, expert_weights_scale when present, and the Hadamard
 * signs the prism.hadamard.* metadata assigns to the expert tensors (by input width). The header
 * is validated as src/gguf.zig does; a malformed file gives GX_E_INVALIDARG, a well-formed one this
 * path cannot take (other tensor types, other prism.hadamard versions) GX_E_UNSUPPORTED; with
 * GX_DEBUG=1 in the environment the reason is printed. */
#define GX_SHARED_NONE 0xffffffffu
typedef struct gx_gguf_layer_info {
    uint32_t type_id;             /* Gyro type of the expert tensors */
    uint32_t n_expert, n_embd, n_ff, n_used;
    float expert_weights_scale;
    uint32_t shared_type;         /* GX_Q8_0 / GX_BF16 / GX_F32, or GX_SHARED_NONE */
    uint32_t shared_ff;           /* n_ff_shexp (0 without a shared expert) */
    uint32_t rotated;             /* bit 0: gate/up carry signs, bit 1: down carries signs */
    uint32_t reserved;
} gx_gguf_layer_info;             /* 40 bytes */

/* Shapes and types of layer gguf_layer of a file (no device needed), so the host can size its
 * context before creating it. */
GX_API gx_result gx_gguf_inspect_layer(const char *path, uint32_t gguf_layer, gx_gguf_layer_info *out_info);

/* gx_upload_layer (and gx_upload_shared when the layer has a shared expert) of layer gguf_layer
 * of the file into slot layer of the context, reading only the tensors it needs. Blocking. */
GX_API gx_result gx_upload_layer_gguf(gx_context *context, uint32_t layer, const char *path, uint32_t gguf_layer,
                                      uint32_t timeout_ms);

/* Routed-expert layer on device-resident activations, enqueued on the context's stream
 * (replaces the dispatch chain of Engine.ffn, src/gpu_engine.zig:1059-1116, through
 * gd_dispatch, native/gyro_native.cpp:891-900):
 *   y[t] = sum_k w[t][k] * Down_e(act(Gate_e(Hx[t]), Up_e(Hx[t])))   (src/engine.zig:520-642)
 * x: [n_tok][E] device, x_dtype GX_F32/GX_BF16; y: [n_tok][E] device, y_dtype GX_F32/GX_BF16.
 * ids/weights: optional device outputs [n_tok][U] (the ffn_moe_topk observation), or NULL.
 * out_ticket: optional; completes when y is written. With world > 1 this is a collective:
 * every rank calls it for its own tokens (n_tok may differ, may be 0) with the same layer, in the
 * same order. Each token's rotated row goes once to every rank that holds one of its experts,
 * each such rank returns one weighted partial row, and the source adds them. The call blocks
 * until the per-rank row counts are known (one short host round trip per layer); a peer that
 * stops answering for the communication timeout gives GX_E_COMM, after which only gx_destroy
 * is valid. With world > 1 every token count takes the tensor-core path, and n_embd must be a
 * multiple of 256 (gx_upload_layer returns GX_E_UNSUPPORTED otherwise). */
GX_API gx_result gx_moe_forward(gx_context *context, uint32_t layer, const void *x, uint32_t x_dtype,
                                uint32_t n_tok, void *y, uint32_t y_dtype, uint32_t *ids, float *weights,
                                uint64_t *out_ticket);

/* Same on host buffers: copies x in and y (and ids/weights if non-NULL) out, then waits.
 * This is the end-to-end call the host uses when its activations live in host memory. */
GX_API gx_result gx_moe_forward_host(gx_context *context, uint32_t layer, const void *x, uint32_t x_dtype,
                                     uint32_t n_tok, void *y, uint32_t y_dtype, uint32_t *ids,
                                     float *weights, uint32_t timeout_ms);

/* A stack of consecutive layers with a pre-norm residual between them,
 *   x_{l+1} = x_l + MoE_l(RMSNorm(x_l)),  RMSNorm(x) = x / sqrt(mean(x^2) + 1e-6) (unit weight,
 *   src/kernels.zig:281-291),
 * for n_tok tokens: the benchmark stand-in for the norm and hyper-connection mixer between the
 * reference model's layers, which lie outside this ABI. Device pointers; the chain of kernels is
 * captured into a CUDA graph on the first call and replayed on later calls with the same
 * (first_layer, n_layers, n_tok, dtypes, flags). With world > 1 it is a collective like
 * gx_moe_forward, and the layers run without a graph. */
GX_API gx_result gx_stack_forward(gx_context *context, uint32_t first_layer, uint32_t n_layers,
                                  const void *x, uint32_t x_dtype, uint32_t n_tok, void *y,
                                  uint32_t y_dtype, uint64_t *out_ticket);
GX_API gx_result gx_stack_forward_host(gx_context *context, uint32_t first_layer, uint32_t n_layers,
                                       const void *x, uint32_t x_dtype, uint32_t n_tok, void *y,
                                       uint32_t y_dtype, uint32_t timeout_ms);

/* Ticket completion (replaces gd_wait_compute / gd_poll, native/include/gyro_native.h:84,126).
 * gx_wait returns GX_E_TIMEOUT if the ticket is not complete after timeout_ms, GX_E_DEVICE on a
 * CUDA error and GX_E_KERNEL if a kernel reported an expired bounded wait. */
GX_API gx_result gx_wait(gx_context *context, uint64_t ticket, uint32_t timeout_ms);
GX_API gx_result gx_poll(gx_context *context, uint64_t *out_completed);

/* The context's CUDA stream (cudaStream_t), so the host can order its own work. */
GX_API gx_result gx_get_stream(gx_context *context, void **out_stream);

/* Gyro decode conformance hook (replaces gd_validate_gyro, native/gyro_native.cpp:597-730 and
 * its shader shaders/gyro_decode.hlsl). Decodes value_count weights (a positive multiple of
 * 128, at most 16777216) of packed blocks (host memory, exactly value_count/128 blocks of the
 * type) into out (host, f32, stored basis, w = d * CB as one binary32 multiply). If expected is
 * non-NULL the call returns GX_E_MISMATCH when any output differs bitwise and writes the
 * largest absolute difference to max_abs_error (may be NULL). Blocking. */
GX_API gx_result gx_decode_blocks(gx_context *context, uint32_t type_id, const void *packed,
                                  uint64_t packed_bytes, float *out, uint32_t value_count,
                                  const float *expected, float *max_abs_error, uint32_t timeout_ms);

/* Standalone decode GEMV on one packed matrix, the per-slot product of moe_gyro
 * (shaders/engine/moe.hlsl:108-211) and Engine.mv for Gyro weights:
 *   y[t][r] = sum_c W[r][c] * x[t][c],  W [rows][cols] packed (reference layout, host),
 * x [n_tok][cols] f32 device, y [n_tok][rows] f32 device, n_tok <= 64. gx_upload_matrix returns
 * a handle (index) owned by the context. */
GX_API gx_result gx_upload_matrix(gx_context *context, uint32_t type_id, uint32_t rows, uint32_t cols,
                                  const void *packed, uint64_t packed_bytes, uint32_t *out_handle,
                                  uint32_t timeout_ms);
GX_API gx_result gx_matvec(gx_context *context, uint32_t handle, const float *x, uint32_t n_tok,
                           float *y, uint64_t *out_ticket);

GX_API gx_result gx_read_timings(gx_context *context, gx_timings *out_timings);

/* No counterpart in the reference (its bridge drives one GPU). Expert-parallel contexts only
 * (world > 1, else GX_E_UNSUPPORTED). Copies into counts[n_expert] the number of this rank's
 * routed slots per global expert of the layer since the last reset (reset != 0 zeroes them after
 * the copy). Blocking. The host sums them over ranks to find the experts worth replicating. */
GX_API gx_result gx_read_expert_counts(gx_context *context, uint32_t layer, uint32_t *counts, uint32_t reset,
                                       uint32_t timeout_ms);

/* No counterpart in the reference. Collective over the expert-parallel group: every rank passes
 * the same list of n distinct global experts of the layer (n <= 32 and below the number of experts
 * outside one rank's shard). Each listed expert's rank broadcasts its packed tiles into a replica
 * slot on every other rank, and from then on every rank serves the listed experts for its own
 * tokens, so their rows cross no link and the load of popular experts spreads over the group.
 * A later call replaces the list (n = 0 restores plain sharding). Blocking; GX_E_COMM if a peer
 * does not take part within the communication timeout. */
GX_API gx_result gx_replicate_experts(gx_context *context, uint32_t layer, const uint32_t *experts, uint32_t n,
                                      uint32_t timeout_ms);

/* No counterpart in the reference. The routed-expert layer for decode batches that allocates no
 * device or host memory on any call. It is meant for hosts that may not allocate once they are
 * stepping: a serving host that hands all free HBM to its own pools (expert arena, caches) at
 * start-up, where a later cudaMalloc would fail, and step loops that must not stall the device,
 * which cudaMalloc and cudaFree do because they synchronise it. gx_moe_forward can allocate on a
 * call (buffers of the many-token path are sized on first use); this call never does.
 *
 * Same arguments, outputs, ticket and error reporting as gx_moe_forward, for
 * n_tok <= GX_NOALLOC_MAX_TOKENS; a larger n_tok returns GX_E_INVALIDARG (with GX_DEBUG=1 set,
 * the reason is printed). It runs the same decode kernels, always, and records no phase times.
 *
 * Its scratch (router logits, selected experts and weights, gate/up activations) is one fixed
 * array of GX_NOALLOC_SCRATCH_BYTES bytes in the library's device image, one per device, shared
 * by every context and every call on that device. Nothing in it needs to start at zero: a call
 * writes each word before it reads it. Calls that overlap on the GPU (on different streams or
 * contexts of one device, not ordered by the host) race on the array and give wrong results;
 * calls through one context are ordered on its stream and do not overlap.
 *
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress),
 * which loads the library's device code on that device if needed; make that first call before
 * any stream capture and before the host's no-allocation phase begins. */
#define GX_NOALLOC_MAX_TOKENS 16u
#define GX_NOALLOC_SCRATCH_BYTES 559616u
GX_API gx_result gx_moe_forward_noalloc(gx_context *context, uint32_t layer, const void *x, uint32_t x_dtype,
                                        uint32_t n_tok, void *y, uint32_t y_dtype, uint32_t *ids, float *weights,
                                        uint64_t *out_ticket);

/* Replaces the context's GX_FLAG_* set (e.g. to switch phase timing on for a profiled replay).
 * Phase events serialise the kernels they separate, so timed calls should run without it. */
GX_API gx_result gx_set_flags(gx_context *context, uint32_t flags);

/* Closes the context (replaces gd_destroy, native/include/gyro_native.h:137). Waits up to
 * timeout_ms for queued work; on GX_E_TIMEOUT the context stays valid. */
GX_API gx_result gx_destroy(gx_context *context, uint32_t timeout_ms);

#ifdef __cplusplus
}
#endif
#endif /* GYRO_MOE_H */
