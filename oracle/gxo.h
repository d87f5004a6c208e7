/*
 * gxo — CPU oracle for the Gyro routed-MoE layer.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path: only the tests,
 * the smoke check and bench.py's cpu_baseline / reference arm may load it. The product path
 * (the gx_* C ABI in include/gyro_moe.h) never calls into it.
 *
 * It restates, in plain C, the reference CPU engine of mattneel/gyro-dx:
 *   - Gyro decode and rotation:  src/gyro.zig:81-195 (normative, strict float mode)
 *   - CPU kernels:               src/kernels.zig:56-349
 *   - routed-expert layer:       src/engine.zig:520-642 (Session.ffn) and topK :671-686
 * Parity of the decode and rotation parts is pinned bit-for-bit against the vendored C decoder
 * third_party/agention-gyro/src/tq_ref.c (compiled from the reference tree into oracle/_ref)
 * and against the reference fixture tests/gyro_vectors.bin (SHA-256 8f739c3e...818c).
 * The layer composition has no reference golden vectors (the reference pins it only with
 * whole-model dumps of a 75.8 GB model); it is restated step by step from engine.zig.
 */
#ifndef GXO_H
#define GXO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Installs the normative 8192-byte codebook (4096 little-endian binary16 values,
 * src/gyro_codebook.f16, SHA-256 ee481f15...e588). Must be called before decoding.
 * Returns 0, or -1 if bytes != 8192. */
int gxo_set_codebook(const void *table, size_t bytes);

/* Type table, src/gyro.zig:32-41. Returns 0 on success, -1 for an unknown id. */
int gxo_type_info(uint32_t type_id, int *k, int *steps, int *block_bytes);

/* Exact binary16 -> binary32, src/gyro.zig:128-141. */
float gxo_fp16_to_fp32(uint16_t half);

/* 16-bit trellis state of step t of one block's stream, src/gyro.zig:107-117. */
uint32_t gxo_state(uint32_t type_id, const uint8_t *stream, int stream_len, int step);

/* Strict decode of packed blocks, src/gyro.zig:81-105. Error codes mirror gyro.Error:
 * -1 UnsupportedType, -2 MissingStateBits, -3 UnsupportedStateBits, -4 InvalidRowLength,
 * -5 InvalidSourceLength. state_bits < 0 means "missing". */
int gxo_decode_row(uint32_t type_id, int state_bits, const uint8_t *src, size_t src_len,
                   float *dst, size_t n);

/* T(x) = H_b(s * x) and T^-1(x) = s * H_b(x), src/gyro.zig:143-195 (int8 signs, NULL = +1).
 * -1 InvalidBlockSize, -4 InvalidRowLength, -6 InvalidSignsLength (unused: caller passes n),
 * -7 InvalidSign; on error the values are unchanged. */
int gxo_rotate(float *v, size_t n, size_t block, const int8_t *signs);
int gxo_unrotate(float *v, size_t n, size_t block, const int8_t *signs);

/* src/kernels.zig:317-338: x *= signs (f32), then normalised block FWHT. */
void gxo_rotate_f32(float *x, size_t n, size_t block, const float *signs);

/* Row bytes of a matrix row, src/kernels.zig:56-67 (0 for f32 routers is cols*4). */
size_t gxo_row_bytes(uint32_t type_id, size_t cols);

/* dotRow for f32, f16, bf16, Q8_0 and the eight Gyro types, src/kernels.zig:72-120, 161-210. */
float gxo_dot_row(uint32_t type_id, const uint8_t *row, const float *x, size_t cols);

/* decodeRow for Gyro types (fast path of the engine), src/kernels.zig:136-159, 213-235. */
void gxo_decode_row_fast(uint32_t type_id, const uint8_t *row, float *out, size_t cols);

/* src/kernels.zig:281-291 with a unit weight: out = x / sqrt(mean(x^2) + eps). In place allowed. */
void gxo_rms_norm(float *out, const float *x, size_t n, float eps);

/* src/kernels.zig:340-349 and src/engine.zig:671-686. */
void gxo_softmax(float *x, size_t n);
void gxo_topk(const float *values, size_t n, uint32_t *ids, float *weights, size_t k);

/* One routed-expert layer. Matrices use the reference layout: the stacked 3-D expert tensor
 * of src/model.zig:115-123 (expert e = rows [e*F, (e+1)*F) of gate/up, rows [e*E, (e+1)*E)
 * of down), each row a run of packed 128-weight blocks. */
typedef struct gxo_layer {
    uint32_t type_id;
    uint32_t n_expert, n_embd, n_ff, n_used;
    float expert_weights_scale;
    const uint8_t *gate, *up, *down;     /* stacked expert matrices */
    const float *router;                 /* [n_expert][n_embd] f32 */
    const float *gate_signs;             /* [n_embd] +-1 or NULL (shared by gate and up) */
    const float *down_signs;             /* [n_ff]  +-1 or NULL */
    const float *router_bias;            /* harness-only logit bias [n_expert] or NULL */
} gxo_layer;

/* src/engine.zig:520-642 for n tokens. x [n][E] f32; out [n][E]; ids/weights [n][U].
 * threads <= 1 runs serially; otherwise the router and the two expert phases run on a
 * pthread chunk pool with the reference's chunk sizes (16 for gate/up tasks, 64 for down
 * tasks) when the library was built with GXO_THREADS. Returns 0, or -1 on bad arguments. */
int gxo_moe_ffn(const gxo_layer *layer, const float *x, size_t n, float *out,
                uint32_t *ids, float *weights, int threads);

/* The expert half of gxo_moe_ffn for a given routing: ids/weights [n][n_used] (ids local to
 * this layer's experts). Slots with ids[slot] >= n_expert contribute nothing (the slots another
 * rank serves in the expert-parallel model). The router fields of the layer are not used. */
int gxo_moe_experts(const gxo_layer *layer, const float *x, size_t n, const uint32_t *ids,
                    const float *weights, float *out, int threads);

/* The shared expert of a layer, src/engine.zig:644-653: three plain row-major matrices in a
 * non-expert encoding (0 f32, 1 f16, 8 Q8_0, 30 bf16; src/kernels.zig:7-10, :56-67) and the f32
 * vector of its sigmoid gate. Bindings of src/model.zig:418-421. */
typedef struct gxo_shared {
    uint32_t type_id;
    uint32_t n_ff;                       /* n_ff_shexp */
    const uint8_t *gate, *up;            /* [n_ff][n_embd] */
    const uint8_t *down;                 /* [n_embd][n_ff] */
    const float *gate_inp;               /* [n_embd] */
} gxo_shared;

/* out[t] += sigmoid(gate_inp . x[t]) * Down(silu(Gate x[t]) * Up x[t]) for n tokens x [n][E]
 * (the unrotated layer input). Returns 0, or -1 on bad arguments. */
int gxo_shared_expert(const gxo_shared *s, const float *x, size_t n, size_t E, float *out, int threads);

/* Hyper-connection mixer weights around the FFN block (src/model.zig:55-60, :362-367): n_streams
 * residual streams of n_embd, a per-stream RMSNorm weight, the low-rank down [rank][hc*E], up
 * [hc*E][rank] and inject [hc][hc*E] matrices in one non-expert encoding (8 Q8_0, 0 f32, 30 bf16,
 * 1 f16), the norm epsilon. */
typedef struct gxo_hc {
    uint32_t n_streams, rank, n_embd, type_id;
    float eps;
    const float *norm;                   /* [hc*E] */
    const uint8_t *down, *up, *inject;
} gxo_hc;

/* src/engine.zig:184-215 (hcMix): res [n][hc*E] -> out [n][E] and, if inject is not NULL,
 * inject [n][hc]. Returns 0, or -1 on bad arguments. */
int gxo_hc_mix(const gxo_hc *w, const float *res, size_t n, float *out, float *inject, int threads);

/* src/engine.zig:217-228 (hcCombine): res[t][c] += block_out[t] * 2 sigmoid(inject[t][c] / hc). */
int gxo_hc_combine(const gxo_hc *w, float *res, size_t n, const float *block_out, const float *inject);

/* Threads the library can use (1 when built without GXO_THREADS). */
int gxo_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
