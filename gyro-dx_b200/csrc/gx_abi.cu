// gx_abi.cu — the C ABI of include/gyro_moe.h: context, HBM arena upload, forward calls,
// tickets and timeouts. One CUDA stream per context; work is asynchronous and ordered.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>
#include <thread>
#include <tuple>
#include <vector>

#include "../../include/gyro_moe.h"
#include "gx_comm.h"
#include "gx_internal.h"
#include "gx_tile.h"

namespace {

constexpr int kEvents = 64;
// Token count from which a forward call takes the tensor-core prefill path (grouped GEMM over
// expert row tiles) instead of the per-slot decode GEMVs.
constexpr uint32_t kPrefillMinTokens = 64;
constexpr uint32_t kChainPdlMaxTokens = 2048;
// RMSNorm epsilon of the stack's pre-norm residual x_{l+1} = x_l + MoE_l(RMSNorm(x_l)).
constexpr float kStackNormEps = 1e-6f;

struct Layer {
    bool ready = false;
    uint32_t type = 0, n_expert = 0, local_experts = 0, first_expert = 0, E = 0, F = 0, U = 0;
    float scale = 0.f;
    uint8_t *arena = nullptr;
    uint64_t bytes = 0;
    uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    uint64_t gate_expert_bytes = 0, down_expert_bytes = 0;
    float *router = nullptr, *bias = nullptr, *gate_signs = nullptr, *down_signs = nullptr;
    uint8_t *router_parts = nullptr;  // router as three bf16 parts, tcgen05 tiles (many-token path)
    // expert parallelism: slots after the local shard that hold copies of hot experts, the
    // route of every global expert (serving rank or -1 = the token's own rank, local index),
    // and this rank's routed-slot count per global expert
    uint32_t replica_slots = 0;
    std::vector<uint32_t> replicas;
    int2 *route = nullptr;
    unsigned *expert_count = nullptr;
    // shared expert (gx_upload_shared), in an arena of its own: W_Q8 or W_F16 matrices
    uint32_t sh_wt = 0, SF = 0;
    uint8_t *sh_arena = nullptr;
    uint64_t sh_bytes = 0;
    gx::SharedMat sh_gate{}, sh_up{}, sh_down{};
    float *sh_gate_inp = nullptr;
    // hyper-connection mixer of the FFN block (gx_upload_hc), in an arena of its own: H streams,
    // rank padded with zeros to R (a multiple of 128), Down padded with zero rows to Rp (a
    // multiple of 256) for the tensor-core path
    uint32_t hc_wt = 0, H = 0, R = 0, Rp = 0;
    float hc_eps = 0.f;
    uint8_t *hc_arena = nullptr;
    uint64_t hc_bytes = 0;
    gx::SharedMat hc_down{}, hc_up{}, hc_inject{};
    float *hc_norm = nullptr;
};

// Copies of hot experts one expert-parallel rank can hold per layer, beside its own shard.
constexpr uint32_t kMaxReplicas = 32;

struct Matrix {
    uint32_t type = 0, rows = 0, cols = 0;
    uint8_t *tiles = nullptr;
};

using GraphKey = std::tuple<uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t>;

}  // namespace

struct gx_context {
    int device = 0;
    uint32_t rank = 0, world = 1, max_tokens = 0, max_layers = 0, flags = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    uint32_t *codebook = nullptr;  // 2048 words = 4096 fp16
    uint32_t *codebook_image = nullptr;  // the decode kernels' shared-memory codebook (interleaved copies)
    unsigned *router_done = nullptr;     // completion count of the selecting router launch (0 between launches)
    std::vector<Layer> layers;
    std::vector<Matrix> mats;
    // scratch sized for max_tokens
    float *logits = nullptr, *weights = nullptr, *act = nullptr, *xbuf[2] = {nullptr, nullptr};
    float *xscale = nullptr, *ss = nullptr;
    // prefill buffers, sized on first use for the largest (E, F, U, NE) seen
    struct Prefill {
        size_t max_tiles = 0, E = 0, F = 0, slots = 0;
        uint8_t *A = nullptr, *A2 = nullptr;
        float *act = nullptr;
        __half *Y = nullptr;
        int *ints = nullptr;  // expert_count | cursor | tile_expert | tile_rows | n_mtiles | row_slot | slot_row
        int *expert_count = nullptr, *cursor = nullptr, *tile_expert = nullptr, *tile_rows = nullptr,
            *n_mtiles = nullptr;
        int *row_slot = nullptr, *slot_row = nullptr;
    } pf;
    // shared-expert work buffers for max_tokens tokens of the widest shared expert uploaded:
    // decode path (act, gated output term), tensor-core path (operand tiles, act, f16 rows, tile
    // list), and the gate logits of both
    struct Shared {
        size_t E = 0, SF = 0;
        float *logit = nullptr, *act = nullptr, *y = nullptr;
        uint8_t *A = nullptr, *A2 = nullptr;
        float *pact = nullptr;
        __half *Ysh = nullptr;
        int *ints = nullptr;  // tile_expert | tile_rows | n_mtiles
    } sh;
    // FFN-block mixer work buffers for max_tokens tokens of the widest mixer uploaded: normed
    // streams, low-rank activations, injection logits, the layer's input and output; tensor-core
    // path: operand tiles of xn and lo, f16 rows of Down xn and Up lo, tile list
    struct Hc {
        size_t HD = 0, Rp = 0, E = 0;
        float *xn = nullptr, *lo = nullptr, *inj = nullptr, *cur = nullptr, *y = nullptr;
        uint8_t *A = nullptr, *A2 = nullptr;
        __half *Ylo = nullptr, *gate = nullptr;
        int *ints = nullptr;  // tile_expert | tile_rows | n_mtiles
    } hc;
    uint32_t *ids = nullptr;
    int *err = nullptr;
    void *x_stage = nullptr, *y_stage = nullptr;     // device staging (graphs, host calls)
    void *h_in = nullptr, *h_out = nullptr;          // pinned host staging
    size_t stage_bytes = 0;
    cudaEvent_t events[kEvents] = {};
    uint64_t submitted = 0;
    std::vector<cudaEvent_t> prof;   // 4 per layer slot: start, router done, gate/up done, down done
    uint32_t prof_layers = 0;        // layers recorded by the most recent forward call
    uint32_t prof_stack = 0;         // > 0: the last call was one stack kernel over this many layers
    gx::StackLayer *stack_table = nullptr;  // device table of uploaded layers (decode-stack kernel)
    unsigned *stack_sync = nullptr;  // grid-barrier counter of the decode-stack kernel
    std::map<GraphKey, std::pair<cudaGraph_t, cudaGraphExec_t>> graphs;
    bool broken = false;
    // expert-parallel group (world > 1)
    const gx::NcclApi *nccl = nullptr;
    ncclComm_t comm = nullptr;
    uint32_t comm_timeout_ms = 120000;
    struct Ep {
        size_t src_cap = 0, recv_cap = 0, E = 0, U = 0;   // rows the buffers hold
        int *pos_of = nullptr;                          // [max_tokens][world]
        uint64_t *dest_mask = nullptr;                  // plan scratch [max_tokens]
        int *block_count = nullptr;                     // plan scratch [CTAs][kMaxEpWorld]
        uint32_t *send_ids = nullptr;                   // [world * max_tokens][U]
        float *send_w = nullptr;
        __half *send_rows = nullptr, *ret_rows = nullptr;   // [world * max_tokens][E]
        __half *recv_rows = nullptr, *part_rows = nullptr;  // [recv_cap][E]
        uint32_t *recv_ids = nullptr;                   // [recv_rows][U]
        float *recv_w = nullptr;
        int *counts = nullptr;                          // device: send counts [world], recv counts [world]
        std::vector<int> src_ntok;                      // tokens of every rank in the current call
        // exchange over NVLink peer memory (state 0: not set up, 1: in use, -1: NCCL rows instead)
        int peer_state = 0;
        int T = 0, pE = 0, pU = 0;
        uint8_t *block = nullptr;                       // this rank's exchange block
        uint8_t *peers[gx::kMaxPeers] = {};             // every rank's block, mapped here
        gx::EpBlock off{};
        unsigned epoch = 0;
        uint64_t wait_ns = 2000000000ull;               // bound of the device-side flag waits
        unsigned fault_skip_push = 0;                   // test hook: epoch whose push is not launched
        uint32_t peer_layers = 0;                       // layer calls that took the peer exchange
        int *h_counts = nullptr;                        // pinned copy
        cudaEvent_t counts_ready = nullptr;
    } ep;
};

namespace {

// GX_DEBUG=1 in the environment prints the failing CUDA call to stderr.
bool debug_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("GX_DEBUG");
        return v && v[0] && v[0] != '0';
    }();
    return on;
}

gx_result fail_cuda_at(gx_context *c, cudaError_t e, const char *what, int line) {
    if (e != cudaSuccess && debug_enabled())
        std::fprintf(stderr, "gyro_moe: %s failed at gx_abi.cu:%d: %s (%s)\n", what, line, cudaGetErrorName(e),
                     cudaGetErrorString(e));
    if (e == cudaSuccess) return GX_OK;
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return GX_E_OUTOFMEMORY;
    }
    if (e == cudaErrorInvalidValue) {
        cudaGetLastError();
        return GX_E_INVALIDARG;
    }
    if (c) c->broken = true;
    return GX_E_DEVICE;
}

#define fail_cuda(c, e) fail_cuda_at((c), (e), "CUDA call", __LINE__)
#define GX_CUDA(expr)                                                       \
    do {                                                                    \
        cudaError_t gx_e_ = (expr);                                         \
        if (gx_e_ != cudaSuccess) return fail_cuda_at(c, gx_e_, #expr, __LINE__); \
    } while (0)

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

bool known_type(uint32_t t) { return gx::type_k(t) != 0; }

// Waits for an event with a wall-clock limit; checks the kernels' error word when done.
gx_result wait_event(gx_context *c, cudaEvent_t ev, uint32_t timeout_ms) {
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return fail_cuda(c, q);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - start).count();
        if ((uint64_t)ms >= timeout_ms) return GX_E_TIMEOUT;
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    int err = 0;
    cudaError_t e = cudaMemcpy(&err, c->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(c, e);
    if (err != 0) {
        if (debug_enabled())
            std::fprintf(stderr, "gyro_moe: kernel error word %d (1 = expired wait, 2 = bad expert id, 3 = output not finite)\n", err);
        cudaMemset(c->err, 0, sizeof(int));
        // an expired wait in an expert-parallel group means a peer fell out of step: the exchange
        // epochs of the ranks no longer agree, so the context takes no further calls
        if (c->world > 1 && err == gx::KERR_WAIT) c->broken = true;
        return err == gx::KERR_RANGE ? GX_E_RANGE : GX_E_KERNEL;
    }
    return GX_OK;
}

gx_result record_ticket(gx_context *c, uint64_t *out_ticket) {
    const uint64_t t = ++c->submitted;
    GX_CUDA(cudaEventRecord(c->events[t % kEvents], c->stream));
    if (out_ticket) *out_ticket = t;
    return GX_OK;
}

gx_result sync_all(gx_context *c, uint32_t timeout_ms) {
    uint64_t t = 0;
    gx_result r = record_ticket(c, &t);
    if (r != GX_OK) return r;
    return wait_event(c, c->events[t % kEvents], timeout_ms);
}

// The router as three bf16 parts W = W0 + W1 + W2 (each the bf16 rounding of what the parts before
// it leave), laid out as the router tensor-core kernel reads them: tiles of 128 experts x 64
// columns, [expert tile][column step][part], each 128-byte swizzled K-major (row r of a tile at
// (r/8)*1024 + (r%8)*128, its 16-byte chunk c at position c ^ (r%8)). Experts past NE are zero.
uint16_t bf16_bits_rn_host(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float bf16_value_host(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
std::vector<uint16_t> router_parts(const float *W, uint64_t NE, uint64_t E) {
    const uint64_t NT = (NE + 127) / 128, KS = E / 64;
    std::vector<uint16_t> out(gx::router_parts_bytes((int)NE, (int)E) / 2, 0);
    for (uint64_t nt = 0; nt < NT; ++nt)
        for (uint64_t ks = 0; ks < KS; ++ks)
            for (uint32_t r = 0; r < 128; ++r) {
                const uint64_t e = nt * 128 + r;
                if (e >= NE) continue;
                for (uint32_t col = 0; col < 64; ++col) {
                    float rest = W[e * E + ks * 64 + col];
                    const uint32_t off = (r >> 3) * 1024u + (r & 7u) * 128u + ((((col * 2u) >> 4) ^ (r & 7u)) << 4) +
                                         ((col * 2u) & 15u);
                    for (int j = 0; j < 3; ++j) {
                        const uint16_t b = bf16_bits_rn_host(rest);
                        rest -= bf16_value_host(b);
                        out[(((nt * KS + ks) * 3 + (uint64_t)j) * 16384u + off) / 2] = b;
                    }
                }
            }
    return out;
}

gx_result ensure_scratch(gx_context *c) {
    const size_t T = c->max_tokens ? c->max_tokens : 1;
    // Sized for the largest shapes the ABI accepts: E <= 4096, F <= 1024, NE <= 512, U <= 16.
    const size_t E = 4096, F = 1024, NE = 512, U = 16;
    GX_CUDA(cudaMalloc(&c->logits, 4 * T * NE * sizeof(float)));  // up to 4 split-K partials
    GX_CUDA(cudaMalloc(&c->weights, T * U * sizeof(float)));
    GX_CUDA(cudaMalloc(&c->xscale, T * sizeof(float)));
    GX_CUDA(cudaMalloc(&c->ss, T * sizeof(float)));
    GX_CUDA(cudaMalloc(&c->ids, T * U * sizeof(uint32_t)));
    GX_CUDA(cudaMalloc(&c->act, T * U * F * sizeof(float)));
    GX_CUDA(cudaMalloc(&c->xbuf[0], T * E * sizeof(float)));
    GX_CUDA(cudaMalloc(&c->xbuf[1], T * E * sizeof(float)));
    c->stage_bytes = T * E * sizeof(float);
    GX_CUDA(cudaMalloc(&c->x_stage, c->stage_bytes));
    GX_CUDA(cudaMalloc(&c->y_stage, c->stage_bytes));
    GX_CUDA(cudaMallocHost(&c->h_in, c->stage_bytes));
    GX_CUDA(cudaMallocHost(&c->h_out, c->stage_bytes + T * U * 8));
    GX_CUDA(cudaMalloc(&c->err, sizeof(int)));
    GX_CUDA(cudaMemset(c->err, 0, sizeof(int)));
    GX_CUDA(cudaMalloc(&c->stack_table, c->max_layers * sizeof(gx::StackLayer)));
    GX_CUDA(cudaMemset(c->stack_table, 0, c->max_layers * sizeof(gx::StackLayer)));
    GX_CUDA(cudaMalloc(&c->stack_sync, 64));
    return GX_OK;
}

void release_all(gx_context *c) {
    for (auto &kv : c->graphs) {
        if (kv.second.second) cudaGraphExecDestroy(kv.second.second);
        if (kv.second.first) cudaGraphDestroy(kv.second.first);
    }
    c->graphs.clear();
    for (auto &l : c->layers) {
        if (l.arena) cudaFree(l.arena);
        if (l.sh_arena) cudaFree(l.sh_arena);
        if (l.hc_arena) cudaFree(l.hc_arena);
    }
    void *sh[] = {c->sh.logit, c->sh.act, c->sh.y, c->sh.A, c->sh.A2, c->sh.pact, c->sh.Ysh, c->sh.ints,
                  c->hc.xn, c->hc.lo, c->hc.inj, c->hc.cur, c->hc.y, c->hc.A, c->hc.A2, c->hc.Ylo, c->hc.gate,
                  c->hc.ints};
    for (void *p : sh) if (p) cudaFree(p);
    void *pf[] = {c->pf.A, c->pf.A2, c->pf.act, c->pf.Y, c->pf.ints};
    for (void *p : pf) if (p) cudaFree(p);
    for (auto &m : c->mats) if (m.tiles) cudaFree(m.tiles);
    void *dev[] = {c->codebook, c->codebook_image, c->router_done, c->logits, c->weights, c->xscale, c->ss, c->ids,
                   c->act, c->xbuf[0], c->xbuf[1], c->x_stage, c->y_stage, c->err, c->stack_table, c->stack_sync};
    for (void *p : dev) if (p) cudaFree(p);
    if (c->h_in) cudaFreeHost(c->h_in);
    if (c->h_out) cudaFreeHost(c->h_out);
    for (uint32_t r = 0; r < c->world && r < (uint32_t)gx::kMaxPeers; ++r)
        if (c->ep.peers[r] && r != c->rank) cudaIpcCloseMemHandle(c->ep.peers[r]);
    if (c->ep.block) cudaFree(c->ep.block);
    void *ep[] = {c->ep.pos_of, c->ep.send_ids, c->ep.send_w, c->ep.send_rows, c->ep.ret_rows, c->ep.recv_rows,
                  c->ep.part_rows, c->ep.recv_ids, c->ep.recv_w, c->ep.counts, c->ep.dest_mask,
                  c->ep.block_count};
    for (void *p : ep) if (p) cudaFree(p);
    if (c->ep.h_counts) cudaFreeHost(c->ep.h_counts);
    if (c->ep.counts_ready) cudaEventDestroy(c->ep.counts_ready);
    if (c->comm) {
        // Abort is local (no peer takes part) and also ends an operation stuck on a lost peer;
        // the stream has been drained before this point unless the context is broken.
        c->nccl->CommAbort(c->comm);
        c->comm = nullptr;
    }
    for (auto &e : c->events) if (e) cudaEventDestroy(e);
    for (auto &e : c->prof) if (e) cudaEventDestroy(e);
    c->prof.clear();
    if (c->stream) cudaStreamDestroy(c->stream);
}

size_t dtype_size(uint32_t dt) { return dt == GX_BF16 ? 2 : 4; }

// Phase event: a plain record on the stream, or an event-record node (external record) while
// the stream is being captured into a graph (a plain record there only orders graph nodes).
cudaError_t record_phase(cudaEvent_t ev, cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(s, &st);
    if (e != cudaSuccess) return e;
    return st == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal)
                                               : cudaEventRecord(ev, s);
}

// Prefill buffers for max_tokens tokens of a layer shape. Rows are padded per expert to
// 128-row tiles: at most slots/128 + min(NE, slots) tiles.
gx_result ensure_prefill(gx_context *c, const Layer &L, size_t slots) {
    const size_t tiles = (slots + 127) / 128 + std::min<size_t>(L.local_experts + L.replica_slots, slots);
    auto &p = c->pf;
    if (p.max_tiles >= tiles && p.E >= L.E && p.F >= L.F && p.slots >= slots) return GX_OK;
    void *old[] = {p.A, p.A2, p.act, p.Y, p.ints};
    bool had = false;
    for (void *q : old) if (q) { cudaFree(q); had = true; }
    p = gx_context::Prefill{};
    if (had) {  // captured stacks point at the old buffers
        for (auto &kv : c->graphs) {
            cudaGraphExecDestroy(kv.second.second);
            cudaGraphDestroy(kv.second.first);
        }
        c->graphs.clear();
    }
    GX_CUDA(cudaMalloc(&p.A, tiles * (L.E / 64) * 16384));
    GX_CUDA(cudaMalloc(&p.A2, tiles * (L.F / 64) * 16384));
    GX_CUDA(cudaMalloc(&p.act, tiles * 128 * L.F * sizeof(float)));
    GX_CUDA(cudaMalloc(&p.Y, tiles * 128 * L.E * sizeof(__half)));
    const size_t n_ints = 1024 + 2 * tiles + 1 + tiles * 128 + slots;
    GX_CUDA(cudaMalloc(&p.ints, n_ints * sizeof(int)));
    // the per-expert counts start at zero; the grouping's scan kernel leaves them at zero
    GX_CUDA(cudaMemsetAsync(p.ints, 0, 512 * sizeof(int), c->stream));
    p.expert_count = p.ints;
    p.cursor = p.expert_count + 512;
    p.tile_expert = p.cursor + 512;
    p.tile_rows = p.tile_expert + tiles;
    p.n_mtiles = p.tile_rows + tiles;
    p.row_slot = p.n_mtiles + 1;
    p.slot_row = p.row_slot + tiles * 128;
    p.max_tiles = tiles;
    p.E = L.E;
    p.F = L.F;
    p.slots = slots;
    return GX_OK;
}

// Work buffers of the shared expert for max_tokens tokens of shape (E, SF), grown only (any
// captured stack is dropped, since it points at the old buffers).
gx_result ensure_shared(gx_context *c, size_t E, size_t SF) {
    auto &sh = c->sh;
    if (sh.E >= E && sh.SF >= SF) return GX_OK;
    E = std::max(E, sh.E);
    SF = std::max(SF, sh.SF);
    void *old[] = {sh.logit, sh.act, sh.y, sh.A, sh.A2, sh.pact, sh.Ysh, sh.ints};
    for (void *q : old) if (q) cudaFree(q);
    sh = gx_context::Shared{};
    for (auto &kv : c->graphs) {
        cudaGraphExecDestroy(kv.second.second);
        cudaGraphDestroy(kv.second.first);
    }
    c->graphs.clear();
    const size_t T = c->max_tokens, Td = std::min<size_t>(T, kPrefillMinTokens), tiles = (T + 127) / 128;
    GX_CUDA(cudaMalloc(&sh.logit, T * sizeof(float)));
    GX_CUDA(cudaMalloc(&sh.act, Td * SF * sizeof(float)));
    GX_CUDA(cudaMalloc(&sh.y, Td * E * sizeof(float)));
    if (T >= kPrefillMinTokens || c->world > 1) {
        GX_CUDA(cudaMalloc(&sh.A, tiles * (E / 64) * 16384));
        GX_CUDA(cudaMalloc(&sh.A2, tiles * (SF / 64) * 16384));
        GX_CUDA(cudaMalloc(&sh.pact, tiles * 128 * SF * sizeof(float)));
        GX_CUDA(cudaMalloc(&sh.Ysh, tiles * 128 * E * sizeof(__half)));
        GX_CUDA(cudaMalloc(&sh.ints, (2 * tiles + 1) * sizeof(int)));
    }
    sh.E = E;
    sh.SF = SF;
    return GX_OK;
}

// Work buffers of the FFN-block mixer for max_tokens tokens (E, HD = H * E, Rp), grown only.
gx_result ensure_hc(gx_context *c, size_t E, size_t HD, size_t Rp) {
    auto &h = c->hc;
    if (h.E >= E && h.HD >= HD && h.Rp >= Rp) return GX_OK;
    E = std::max(E, h.E);
    HD = std::max(HD, h.HD);
    Rp = std::max(Rp, h.Rp);
    void *old[] = {h.xn, h.lo, h.inj, h.cur, h.y, h.A, h.A2, h.Ylo, h.gate, h.ints};
    for (void *q : old) if (q) cudaFree(q);
    h = gx_context::Hc{};
    const size_t T = c->max_tokens, tiles = (T + 127) / 128;
    GX_CUDA(cudaMalloc(&h.xn, T * HD * sizeof(float)));
    GX_CUDA(cudaMalloc(&h.lo, T * Rp * sizeof(float)));
    GX_CUDA(cudaMalloc(&h.inj, T * 8 * sizeof(float)));
    GX_CUDA(cudaMalloc(&h.cur, T * E * sizeof(float)));
    GX_CUDA(cudaMalloc(&h.y, T * E * sizeof(float)));
    if (T >= kPrefillMinTokens) {
        GX_CUDA(cudaMalloc(&h.A, tiles * (HD / 64) * 16384));
        GX_CUDA(cudaMalloc(&h.A2, tiles * (Rp / 64) * 16384));
        GX_CUDA(cudaMalloc(&h.Ylo, tiles * 128 * Rp * sizeof(__half)));
        GX_CUDA(cudaMalloc(&h.gate, tiles * 128 * HD * sizeof(__half)));
        GX_CUDA(cudaMalloc(&h.ints, (2 * tiles + 1) * sizeof(int)));
    }
    h.E = E;
    h.HD = HD;
    h.Rp = Rp;
    return GX_OK;
}

gx::HcArgs hc_args(gx_context *c, const Layer &L, float *res, uint32_t n_tok) {
    gx::HcArgs a{};
    a.wt = L.hc_wt;
    a.down = L.hc_down;
    a.up = L.hc_up;
    a.inject = L.hc_inject;
    a.norm = L.hc_norm;
    a.eps = L.hc_eps;
    a.n_tok = (int)n_tok;
    a.H = (int)L.H;
    a.E = (int)L.E;
    a.R = (int)L.R;
    a.res = res;
    a.res_out = res;
    a.xn = c->hc.xn;
    a.lo = c->hc.lo;
    a.inj = c->hc.inj;
    a.cur = c->hc.cur;
    return a;
}

// The mixer in front of the routed layer (src/engine.zig:184-215): per-stream norm, then the two
// low-rank products and the gated mean into c->hc.cur, and the injection logits into c->hc.inj.
// Few tokens on the CUDA cores; many tokens through the grouped GEMM with the plain-matrix
// decoders (one "expert", 128 tokens per row tile), as the reference switches to its tiled
// products above gemm_min_tok (src/gpu_engine.zig:896, :909-922).
gx_result enqueue_hc_mix(gx_context *c, const Layer &L, const gx::HcArgs &a) {
    const uint32_t n_tok = (uint32_t)a.n_tok;
    GX_CUDA(gx::launch_hc_norm(a, c->stream, false));
    if (n_tok < kPrefillMinTokens) {
        GX_CUDA(gx::launch_hc_down(a, 0, c->stream, true));
        GX_CUDA(gx::launch_hc_up_mix(a, c->stream, true));
        return GX_OK;
    }
    auto &h = c->hc;
    const int tiles = (int)((c->max_tokens + 127) / 128);
    const int HD = (int)(L.H * L.E);
    int *tile_expert = h.ints, *tile_rows = h.ints + tiles, *n_mtiles = h.ints + 2 * tiles;
    GX_CUDA(gx::launch_shared_tiles((int)n_tok, tile_expert, tile_rows, n_mtiles, c->stream));
    gx::PackArgs pa{};
    pa.src = h.xn;
    pa.U = 1;
    pa.K = HD;
    pa.tile_rows = tile_rows;
    pa.n_mtiles = n_mtiles;
    pa.dst = h.A;
    GX_CUDA(gx::launch_pack_rows(pa, tiles, c->stream));
    gx::GemmArgs gm{};
    gm.type = L.hc_wt;
    gm.w0 = L.hc_down.w;
    gm.d0 = L.hc_down.d;
    gm.K = HD;
    gm.n_ntiles = (int)(L.Rp / 256);
    gm.n_expert = 1;
    gm.A = h.A;
    gm.tile_expert = tile_expert;
    gm.tile_rows = tile_rows;
    gm.n_mtiles = n_mtiles;
    gm.Y = h.Ylo;
    gm.E = (int)L.Rp;
    gm.codebook = c->codebook;
    gm.err = c->err;
    GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
    GX_CUDA(gx::launch_hc_down(a, (int)L.R, c->stream, false));   // the injection rows
    GX_CUDA(gx::launch_hc_lo(a, h.Ylo, (int)L.Rp, c->stream));
    gx::PackArgs pl{};
    pl.src = h.lo;
    pl.U = 1;
    pl.K = (int)L.R;
    pl.tile_rows = tile_rows;
    pl.n_mtiles = n_mtiles;
    pl.dst = h.A2;
    GX_CUDA(gx::launch_pack_rows(pl, tiles, c->stream));
    gm.w0 = L.hc_up.w;
    gm.d0 = L.hc_up.d;
    gm.K = (int)L.R;
    gm.n_ntiles = HD / 256;
    gm.A = h.A2;
    gm.Y = h.gate;
    gm.E = HD;
    GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
    GX_CUDA(gx::launch_hc_mix(a, h.gate, c->stream));
    return GX_OK;
}

gx::SharedArgs shared_args(gx_context *c, const Layer &L, const void *x, int xb, uint32_t n_tok) {
    gx::SharedArgs a{};
    a.wt = L.sh_wt;
    a.gate = L.sh_gate;
    a.up = L.sh_up;
    a.down = L.sh_down;
    a.gate_inp = L.sh_gate_inp;
    a.x = x;
    a.x_bf16 = xb;
    a.n_tok = (int)n_tok;
    a.E = (int)L.E;
    a.SF = (int)L.SF;
    a.act = c->sh.act;
    a.logit = c->sh.logit;
    a.y = c->sh.y;
    return a;
}

// Shared expert of a few-token call on the CUDA cores: act and gate logits, then the gated down
// product into c->sh.y, which the routed down kernel adds. The token scale comes from the
// router's sums of squares.
gx_result enqueue_shared_decode(gx_context *c, const Layer &L, const void *x, int xb, uint32_t n_tok, float norm_eps,
                                bool pdl) {
    gx::SharedArgs a = shared_args(c, L, x, xb, n_tok);
    a.ss = c->ss;
    a.norm_eps = norm_eps;
    GX_CUDA(gx::launch_shared_gate_up(a, c->stream, pdl));
    GX_CUDA(gx::launch_shared_down(a, c->stream, pdl));
    return GX_OK;
}

// Shared expert of a many-token call on the tensor cores: every token is a row of one "expert"
// (tiles of 128 tokens in order), through the same grouped GEMM as the routed experts with the
// Q8_0 / fp16 decoders, into f16 rows c->sh.Ysh; the gate logits into c->sh.logit. xscale: the
// per-token scale the selection wrote.
gx_result enqueue_shared_gemm(gx_context *c, const Layer &L, const void *x, int xb, uint32_t n_tok,
                              const float *xscale) {
    auto &sh = c->sh;
    if (n_tok == 0) return GX_OK;
    const int tiles = (int)((c->max_tokens + 127) / 128);
    int *tile_expert = sh.ints, *tile_rows = sh.ints + tiles, *n_mtiles = sh.ints + 2 * tiles;
    GX_CUDA(gx::launch_shared_tiles((int)n_tok, tile_expert, tile_rows, n_mtiles, c->stream));
    gx::PackArgs pa{};
    pa.src = x;
    pa.src_bf16 = xb;
    pa.by_token = 0;
    pa.U = 1;
    pa.K = (int)L.E;
    pa.xscale = xscale;
    pa.tile_rows = tile_rows;
    pa.n_mtiles = n_mtiles;
    pa.dst = sh.A;
    GX_CUDA(gx::launch_pack_rows(pa, tiles, c->stream));
    gx::GemmArgs gm{};
    gm.type = L.sh_wt;
    gm.w0 = L.sh_gate.w;
    gm.w1 = L.sh_up.w;
    gm.d0 = L.sh_gate.d;
    gm.d1 = L.sh_up.d;
    gm.K = (int)L.E;
    gm.n_ntiles = (int)(L.SF / 128);
    gm.n_expert = 1;
    gm.A = sh.A;
    gm.tile_expert = tile_expert;
    gm.tile_rows = tile_rows;
    gm.n_mtiles = n_mtiles;
    gm.act = sh.pact;
    gm.F = (int)L.SF;
    gm.Y = sh.Ysh;
    gm.E = (int)L.E;
    gm.codebook = c->codebook;
    gm.err = c->err;
    GX_CUDA(gx::launch_moe_gemm(gm, 0, c->sm_count, c->stream));
    gx::PackArgs pd{};
    pd.src = sh.pact;
    pd.by_token = 0;
    pd.U = 1;
    pd.K = (int)L.SF;
    pd.tile_rows = tile_rows;
    pd.n_mtiles = n_mtiles;
    pd.dst = sh.A2;
    GX_CUDA(gx::launch_pack_rows(pd, tiles, c->stream));
    gm.w0 = L.sh_down.w;
    gm.w1 = nullptr;
    gm.d0 = L.sh_down.d;
    gm.d1 = nullptr;
    gm.K = (int)L.SF;
    gm.n_ntiles = (int)(L.E / 256);
    gm.A = sh.A2;
    GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
    gx::SharedArgs a = shared_args(c, L, x, xb, n_tok);
    a.xscale = xscale;
    GX_CUDA(gx::launch_shared_logits(a, c->stream));
    return GX_OK;
}

// Raw router logits of n_tok tokens into c->logits as *splits partial sums: on the tensor cores
// when the layer carries its bf16 router parts, else the fp32 CUDA-core GEMM.
cudaError_t launch_router_logits(gx_context *c, const Layer &L, const void *x, int xb, uint32_t n_tok, int *splits) {
    if (L.router_parts && L.n_expert <= 512) {
        *splits = gx::router_tc_splits((int)n_tok, (int)L.n_expert, (int)L.E, c->sm_count);
        return gx::launch_router_tc(x, xb, (int)n_tok, (int)L.n_expert, (int)L.E, L.router_parts, c->logits, *splits,
                                    c->err, c->stream);
    }
    *splits = (L.E % (4 * 32) == 0) ? 4 : 1;
    return gx::launch_router_gemm(L.router, x, xb, (int)n_tok, (int)L.n_expert, (int)L.E, c->logits, *splits,
                                  c->stream);
}

// Many-token layer on tensor cores: router GEMM, per-token selection, grouping, packed f16
// operand tiles, two grouped tcgen05 GEMMs with trellis decoding, combine.
// ev (GX_FLAG_PROFILE): start, after selection/grouping/packing, after the gate/up GEMM, end.
gx_result enqueue_layer_prefill(gx_context *c, const Layer &L, const void *x, uint32_t x_dtype, uint32_t n_tok,
                                const void *resid, uint32_t resid_dtype, void *out, uint32_t out_dtype,
                                float norm_eps, cudaEvent_t *ev) {
    gx_result r = ensure_prefill(c, L, (size_t)c->max_tokens * L.U);
    if (r != GX_OK) return r;
    auto &p = c->pf;
    const int xb = x_dtype == GX_BF16;
    if (ev) GX_CUDA(record_phase(ev[0], c->stream));
    int splits;
    GX_CUDA(launch_router_logits(c, L, x, xb, n_tok, &splits));
    gx::RouterArgs ra{};
    ra.W = L.router;
    ra.bias = L.bias;
    ra.x = x;
    ra.x_bf16 = xb;
    ra.n_tok = (int)n_tok;
    ra.NE = (int)L.n_expert;
    ra.E = (int)L.E;
    ra.U = (int)L.U;
    ra.scale = L.scale;
    ra.norm_eps = norm_eps;
    ra.ss = c->ss;
    ra.ss_from_x = 1;
    ra.logit_splits = splits;
    ra.xscale = c->xscale;
    ra.logits = c->logits;
    ra.ids = c->ids;
    ra.weights = c->weights;
    ra.err = c->err;
    GX_CUDA(gx::launch_topk(ra, c->stream));
    if (L.sh_wt) {
        r = enqueue_shared_gemm(c, L, x, xb, n_tok, c->xscale);
        if (r != GX_OK) return r;
    }
    gx::GroupArgs ga{};
    ga.ids = c->ids;
    ga.n_slots = (int)(n_tok * L.U);
    ga.NE = (int)L.local_experts;
    ga.expert_count = p.expert_count;
    ga.cursor = p.cursor;
    ga.tile_expert = p.tile_expert;
    ga.tile_rows = p.tile_rows;
    ga.n_mtiles = p.n_mtiles;
    ga.row_slot = p.row_slot;
    ga.slot_row = p.slot_row;
    ga.err = c->err;
    GX_CUDA(gx::launch_group(ga, c->stream));
    // each token rotated once and stored into the tile rows of its slots
    gx::RotPackArgs rp{};
    rp.x = x;
    rp.x_bf16 = xb;
    rp.xscale = norm_eps > 0.f ? c->xscale : nullptr;
    rp.signs = L.gate_signs;
    rp.n_tok = (int)n_tok;
    rp.E = (int)L.E;
    rp.U = (int)L.U;
    rp.slot_row = p.slot_row;
    rp.tile_rows = p.tile_rows;
    rp.dst = p.A;
    rp.compact = gx::gemm_ts_routed(L.type);
    GX_CUDA(gx::launch_rotate_pack(rp, c->stream));
    if (ev) GX_CUDA(record_phase(ev[1], c->stream));
    gx::GemmArgs gm{};
    gm.type = L.type;
    gm.w0 = L.gate;
    gm.w1 = L.up;
    gm.expert_bytes = L.gate_expert_bytes;
    gm.K = (int)L.E;
    gm.n_ntiles = (int)(L.F / 128);
    gm.n_expert = (int)L.local_experts;
    gm.A = p.A;
    gm.tile_expert = p.tile_expert;
    gm.tile_rows = p.tile_rows;
    gm.n_mtiles = p.n_mtiles;
    gm.act = p.act;
    gm.F = (int)L.F;
    gm.Y = p.Y;
    gm.E = (int)L.E;
    gm.codebook = c->codebook;
    gm.err = c->err;
    if (gx::gemm_ts_routed(L.type)) {
        gm.down_A = p.A2;   // the gate/up epilogue packs the down operand
        gm.down_signs = L.down_signs;
    }
    GX_CUDA(gx::launch_moe_gemm(gm, 0, c->sm_count, c->stream));
    if (ev) GX_CUDA(record_phase(ev[2], c->stream));
    gx::PackArgs pd{};
    pd.src = p.act;
    pd.src_bf16 = 0;
    pd.by_token = 0;
    pd.U = (int)L.U;
    pd.K = (int)L.F;
    pd.signs = L.down_signs;
    pd.row_slot = p.row_slot;
    pd.tile_rows = p.tile_rows;
    pd.n_mtiles = p.n_mtiles;
    pd.dst = p.A2;
    pd.compact = gx::gemm_ts_routed(L.type);
    if (!gx::gemm_ts_routed(L.type)) GX_CUDA(gx::launch_pack_rows(pd, (int)p.max_tiles, c->stream));
    gm.w0 = L.down;
    gm.w1 = nullptr;
    gm.expert_bytes = L.down_expert_bytes;
    gm.K = (int)L.F;
    gm.n_ntiles = (int)(L.E / 256);
    gm.A = p.A2;
    GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
    gx::CombineArgs ca{};
    ca.err = c->err;
    ca.Y = p.Y;
    ca.slot_row = p.slot_row;
    ca.weights = c->weights;
    ca.Ysh = L.sh_wt ? c->sh.Ysh : nullptr;
    ca.sh_logit = c->sh.logit;
    ca.resid = resid;
    ca.resid_bf16 = resid_dtype == GX_BF16;
    ca.out = out;
    ca.out_bf16 = out_dtype == GX_BF16;
    ca.n_tok = (int)n_tok;
    ca.U = (int)L.U;
    ca.E = (int)L.E;
    GX_CUDA(gx::launch_combine(ca, c->stream));
    if (ev) GX_CUDA(record_phase(ev[3], c->stream));
    return GX_OK;
}

// ---- expert parallelism (world > 1) ------------------------------------------------------
// Rank r serves experts [r*NE/W, (r+1)*NE/W) (and, after gx_replicate_experts, the replicated
// experts for its own tokens). A forward call first exchanges every rank's token count (one host
// round trip per call). Per layer, every rank then takes the same NCCL steps in the same order,
// also with no tokens of its own: dispatch of n_tok rotated token rows (with their
// destination-local slots; rows no slot of the destination needs carry none) to every rank, the
// expert phase on what it received, and the return of one weighted partial row per received row;
// the source adds the partial rows (+ residual). No step waits on the host, so the layers of a
// stack queue back to back.

gx_result comm_result(gx_context *c, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return GX_OK;
    if (debug_enabled())
        std::fprintf(stderr, "gyro_moe: %s: %s\n", what,
                     r == ncclInProgress ? "no progress within the communication timeout" : c->nccl->GetErrorString(r));
    c->broken = true;  // a lost peer leaves NCCL work queued; only gx_destroy (abort) is valid now
    return GX_E_COMM;
}

gx_result comm_group_end(gx_context *c, const char *what) {
    ncclResult_t r = c->nccl->GroupEnd();
    if (r == ncclSuccess || r == ncclInProgress) r = gx::nccl_settle(c->nccl, c->comm, c->comm_timeout_ms);
    return comm_result(c, r, what);
}

template <typename T>
void free_dev(T *&p) {
    if (p) cudaFree(p);
    p = nullptr;
}

// Send-side buffers for world * max_tokens rows of the largest layer shape seen.
gx_result ensure_ep_send(gx_context *c, const Layer &L) {
    auto &e = c->ep;
    const size_t W = c->world, T = c->max_tokens, rows = W * T;
    if (!e.counts) {
        GX_CUDA(cudaMalloc(&e.counts, 2 * W * sizeof(int)));
        GX_CUDA(cudaMallocHost(&e.h_counts, 2 * W * sizeof(int)));
        GX_CUDA(cudaEventCreateWithFlags(&e.counts_ready, cudaEventDisableTiming));
    }
    if (e.src_cap >= rows && e.E >= L.E && e.U >= L.U) return GX_OK;
    free_dev(e.pos_of);
    free_dev(e.send_ids);
    free_dev(e.send_w);
    free_dev(e.send_rows);
    free_dev(e.ret_rows);
    free_dev(e.dest_mask);
    free_dev(e.block_count);
    e.src_cap = 0;
    const size_t E = std::max<size_t>(e.E, L.E), U = std::max<size_t>(e.U, L.U);
    GX_CUDA(cudaMalloc(&e.pos_of, T * W * sizeof(int)));
    GX_CUDA(cudaMalloc(&e.dest_mask, T * sizeof(uint64_t)));
    GX_CUDA(cudaMalloc(&e.block_count, (size_t)std::max(1, gx::ep_plan_ctas((int)T)) * gx::kMaxEpWorld * sizeof(int)));
    GX_CUDA(cudaMalloc(&e.send_ids, rows * U * sizeof(uint32_t)));
    GX_CUDA(cudaMalloc(&e.send_w, rows * U * sizeof(float)));
    GX_CUDA(cudaMalloc(&e.send_rows, rows * E * sizeof(__half)));
    GX_CUDA(cudaMalloc(&e.ret_rows, rows * E * sizeof(__half)));
    e.src_cap = rows;
    e.E = E;
    e.U = U;
    // receive buffers are sized for E and U too
    free_dev(e.recv_rows);
    free_dev(e.part_rows);
    free_dev(e.recv_ids);
    free_dev(e.recv_w);
    e.recv_cap = 0;
    return GX_OK;
}

// Receive-side buffers for R rows (grown geometrically, at most world * max_tokens).
gx_result ensure_ep_recv(gx_context *c, size_t R) {
    auto &e = c->ep;
    if (e.recv_cap >= R) return GX_OK;
    const size_t cap = std::min<size_t>(std::max<size_t>(R, 2 * e.recv_cap), e.src_cap);
    free_dev(e.recv_rows);
    free_dev(e.part_rows);
    free_dev(e.recv_ids);
    free_dev(e.recv_w);
    e.recv_cap = 0;
    GX_CUDA(cudaMalloc(&e.recv_rows, cap * e.E * sizeof(__half)));
    GX_CUDA(cudaMalloc(&e.part_rows, cap * e.E * sizeof(__half)));
    GX_CUDA(cudaMalloc(&e.recv_ids, cap * e.U * sizeof(uint32_t)));
    GX_CUDA(cudaMalloc(&e.recv_w, cap * e.U * sizeof(float)));
    e.recv_cap = cap;
    return GX_OK;
}

// Exchanges every rank's token count for the call that follows (a collective; blocking).
gx_result ep_sync_ntok(gx_context *c, uint32_t n_tok) {
    auto &e = c->ep;
    const int W = (int)c->world;
    if (!e.counts) {
        GX_CUDA(cudaMalloc(&e.counts, 2 * W * sizeof(int)));
        GX_CUDA(cudaMallocHost(&e.h_counts, 2 * W * sizeof(int)));
        GX_CUDA(cudaEventCreateWithFlags(&e.counts_ready, cudaEventDisableTiming));
    }
    e.h_counts[0] = (int)n_tok;
    GX_CUDA(cudaMemcpyAsync(e.counts, e.h_counts, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    c->nccl->GroupStart();
    for (int d = 0; d < W; ++d) {
        c->nccl->Send(e.counts, 1, ncclInt32, d, c->comm, c->stream);
        c->nccl->Recv(e.counts + W + d, 1, ncclInt32, d, c->comm, c->stream);
    }
    gx_result r = comm_group_end(c, "token-count exchange");
    if (r != GX_OK) return r;
    GX_CUDA(cudaMemcpyAsync(e.h_counts + W, e.counts + W, W * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    GX_CUDA(cudaEventRecord(e.counts_ready, c->stream));
    r = wait_event(c, e.counts_ready, c->comm_timeout_ms);
    if (r == GX_E_TIMEOUT) return comm_result(c, ncclInProgress, "token-count exchange");
    if (r != GX_OK) return r;
    e.src_ntok.assign(e.h_counts + W, e.h_counts + 2 * W);
    for (int v : e.src_ntok)
        if (v < 0 || (uint32_t)v > c->max_tokens) return comm_result(c, ncclInvalidUsage, "token-count exchange");
    return GX_OK;
}

// Exchanges `bytes` of this rank's device buffer src with every rank into dst[W][bytes] (a
// collective; blocking).
gx_result ep_allgather(gx_context *c, const void *src, void *dst, size_t bytes, const char *what) {
    c->nccl->GroupStart();
    for (int d = 0; d < (int)c->world; ++d) {
        c->nccl->Send(src, bytes, ncclUint8, d, c->comm, c->stream);
        c->nccl->Recv(static_cast<uint8_t *>(dst) + (size_t)d * bytes, bytes, ncclUint8, d, c->comm, c->stream);
    }
    gx_result r = comm_group_end(c, what);
    if (r != GX_OK) return r;
    GX_CUDA(cudaEventRecord(c->ep.counts_ready, c->stream));
    r = wait_event(c, c->ep.counts_ready, c->comm_timeout_ms);
    return r == GX_E_TIMEOUT ? comm_result(c, ncclInProgress, what) : r;
}

// Releases this rank's exchange block and its mappings of the other ranks' blocks, after the
// work queued on the stream (which may still use them) has finished.
gx_result ep_peer_teardown(gx_context *c) {
    auto &e = c->ep;
    GX_CUDA(cudaStreamSynchronize(c->stream));
    for (int p = 0; p < (int)c->world && p < gx::kMaxPeers; ++p)
        if (e.peers[p] && p != (int)c->rank) cudaIpcCloseMemHandle(e.peers[p]);
    for (auto &p : e.peers) p = nullptr;
    if (e.block) cudaFree(e.block);
    e.block = nullptr;
    e.peer_state = 0;
    return GX_OK;
}

// Sets up the exchange over peer memory (a collective, on the first expert-parallel layer, and
// again when a later layer is wider than the blocks): every
// rank allocates its block for T = max_tokens rows per source and the largest E and U uploaded,
// shares it by CUDA IPC, and maps every other rank's block. Every rank takes the peer path only
// if every rank could map every block and all agree on T, E, U; otherwise all keep the NCCL rows
// (GX_EP_NCCL=1 asks for those).
gx_result ep_peer_setup(gx_context *c) {
    auto &e = c->ep;
    const int W = (int)c->world;
    int E = 0, U = 0;
    for (const Layer &L : c->layers)
        if (L.ready) {
            E = std::max<int>(E, (int)L.E);
            U = std::max<int>(U, (int)L.U);
        }
    const char *force = std::getenv("GX_EP_NCCL");
    int ok = W <= gx::kMaxPeers && !(force && force[0] == '1') ? 1 : 0;
    cudaIpcMemHandle_t handle{};
    if (ok) {
        e.off = gx::ep_block_layout(W, (int)c->max_tokens, E, U);
        if (cudaMalloc(&e.block, e.off.bytes) != cudaSuccess ||
            cudaMemset(e.block, 0, e.off.bytes) != cudaSuccess ||
            cudaIpcGetMemHandle(&handle, e.block) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
        }
    }
    // record: ok, T, E, U, handle
    // ranks whose waits depend on each other must be on different GPUs (device UUIDs compared)
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, c->device) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
    }
    struct Rec {
        int ok, T, E, U;
        cudaIpcMemHandle_t h;
        char uuid[16];
    } mine{ok, (int)c->max_tokens, E, U, handle, {}};
    std::memcpy(mine.uuid, prop.uuid.bytes, 16);
    std::vector<Rec> all(W);
    uint8_t *dev = nullptr;
    GX_CUDA(cudaMalloc(&dev, sizeof(Rec) * (W + 1)));
    gx_result r = GX_OK;
    do {
        if (cudaMemcpy(dev, &mine, sizeof(Rec), cudaMemcpyHostToDevice) != cudaSuccess) { r = GX_E_DEVICE; break; }
        r = ep_allgather(c, dev, dev + sizeof(Rec), sizeof(Rec), "exchange setup");
        if (r != GX_OK) break;
        if (cudaMemcpy(all.data(), dev + sizeof(Rec), sizeof(Rec) * W, cudaMemcpyDeviceToHost) != cudaSuccess) {
            r = GX_E_DEVICE;
            break;
        }
        for (const Rec &x : all) ok = ok && x.ok && x.T == mine.T && x.E == E && x.U == U;
        for (int p = 0; p < W; ++p)
            for (int q = p + 1; q < W; ++q)
                if (std::memcmp(all[p].uuid, all[q].uuid, 16) == 0) ok = 0;
        for (int p = 0; ok && p < W; ++p) {
            if (p == (int)c->rank) { e.peers[p] = e.block; continue; }
            void *m = nullptr;
            if (cudaIpcOpenMemHandle(&m, all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
            } else {
                e.peers[p] = static_cast<uint8_t *>(m);
            }
        }
        // all ranks agree on the outcome
        int flag = ok;
        if (cudaMemcpy(dev, &flag, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) { r = GX_E_DEVICE; break; }
        r = ep_allgather(c, dev, dev + sizeof(Rec), sizeof(int), "exchange setup");
        if (r != GX_OK) break;
        std::vector<int> flags(W);
        if (cudaMemcpy(flags.data(), dev + sizeof(Rec), sizeof(int) * W, cudaMemcpyDeviceToHost) != cudaSuccess) {
            r = GX_E_DEVICE;
            break;
        }
        for (int f : flags) ok = ok && f;
    } while (false);
    cudaFree(dev);
    if (r != GX_OK) return r;
    if (!ok) {
        for (int p = 0; p < W; ++p)
            if (e.peers[p] && p != (int)c->rank) cudaIpcCloseMemHandle(e.peers[p]);
        for (auto &p : e.peers) p = nullptr;
        if (e.block) cudaFree(e.block);
        e.block = nullptr;
        e.peer_state = -1;
        return GX_OK;
    }
    e.T = (int)c->max_tokens;
    e.pE = E;
    e.pU = U;
    e.peer_state = 1;
    return GX_OK;
}

// The layer's exchange over peer memory, after selection and the plan (stride T): push the rows,
// wait for every source's rows, the expert phase on the rx region ([W][T] rows, empty ones carry
// no slot), partial rows straight into the sources' ret regions, wait for every destination,
// and the source sum.
gx_result enqueue_layer_ep_peer(gx_context *c, const Layer &L, const void *x, int xb, uint32_t n_tok, size_t S,
                                const void *resid, uint32_t resid_dtype, void *out, uint32_t out_dtype, float norm_eps,
                                cudaEvent_t *ev) {
    auto &e = c->ep;
    const int W = (int)c->world;
    const size_t E = L.E, U = L.U, T = S;
    // buffers of the expert phase first: growing them synchronises the device, which must not
    // happen between this rank's push and the peers' waits for it
    const size_t rows = (size_t)W * T;
    {
        const size_t cap = (size_t)W * e.T * U;
        size_t want = rows * U;
        if (c->pf.slots < want) want = std::min(cap, std::max(want, c->pf.slots + c->pf.slots / 2));
        gx_result r0 = ensure_prefill(c, L, want);
        if (r0 != GX_OK) return r0;
    }
    gx::EpPeerArgs pa{};
    for (int p = 0; p < W; ++p) pa.peer[p] = e.peers[p];
    pa.off = e.off;
    pa.W = W;
    pa.rank = (int)c->rank;
    pa.T = (int)T;
    pa.E = (int)E;
    pa.U = (int)U;
    pa.epoch = ++e.epoch;
    pa.wait_ns = e.wait_ns;
    pa.err = c->err;
    ++e.peer_layers;
    // the blocks are laid out for the largest E and U; a smaller layer uses the same offsets
    gx::EpPushArgs ps{};
    ps.p = pa;
    ps.x = x;
    ps.x_bf16 = xb;
    ps.n_tok = (int)n_tok;
    ps.xscale = norm_eps > 0.f ? c->xscale : nullptr;
    ps.signs = L.gate_signs;
    ps.pos_of = e.pos_of;
    ps.send_ids = e.send_ids;
    ps.send_w = e.send_w;
    ps.send_count = e.counts;
    // GX_EP_FAULT_SKIP_PUSH=<n> (failure-detection tests): this rank does not send its rows of its
    // n-th peer-exchange layer call, so its peers' bounded waits run out
    if (pa.epoch != e.fault_skip_push) GX_CUDA(gx::launch_ep_push(ps, c->stream));
    GX_CUDA(gx::launch_ep_wait_rx(pa, c->stream));
    if (ev) GX_CUDA(record_phase(ev[1], c->stream));
    auto &p = c->pf;
    gx::GroupArgs ga{};
    ga.ids = reinterpret_cast<const uint32_t *>(e.block + e.off.rx_ids);
    ga.n_slots = (int)(rows * U);
    ga.NE = (int)(L.local_experts + L.replica_slots);
    ga.expert_count = p.expert_count;
    ga.cursor = p.cursor;
    ga.tile_expert = p.tile_expert;
    ga.tile_rows = p.tile_rows;
    ga.n_mtiles = p.n_mtiles;
    ga.row_slot = p.row_slot;
    ga.slot_row = p.slot_row;
    ga.err = c->err;
    GX_CUDA(gx::launch_group(ga, c->stream));
    gx::PackArgs pk{};
    pk.by_token = 1;
    pk.U = (int)U;
    pk.K = (int)E;
    pk.xh = reinterpret_cast<const __half *>(e.block + e.off.rx_rows);
    pk.row_slot = p.row_slot;
    pk.tile_rows = p.tile_rows;
    pk.n_mtiles = p.n_mtiles;
    pk.dst = p.A;
    pk.compact = gx::gemm_ts_routed(L.type);
    GX_CUDA(gx::launch_pack_rows(pk, (int)p.max_tiles, c->stream));
    gx::GemmArgs gm{};
    gm.type = L.type;
    gm.w0 = L.gate;
    gm.w1 = L.up;
    gm.expert_bytes = L.gate_expert_bytes;
    gm.K = (int)L.E;
    gm.n_ntiles = (int)(L.F / 128);
    gm.n_expert = (int)(L.local_experts + L.replica_slots);
    gm.A = p.A;
    gm.tile_expert = p.tile_expert;
    gm.tile_rows = p.tile_rows;
    gm.n_mtiles = p.n_mtiles;
    gm.act = p.act;
    gm.F = (int)L.F;
    gm.Y = p.Y;
    gm.E = (int)L.E;
    gm.codebook = c->codebook;
    gm.err = c->err;
    if (gx::gemm_ts_routed(L.type)) {
        gm.down_A = p.A2;   // the gate/up epilogue packs the down operand
        gm.down_signs = L.down_signs;
    }
    GX_CUDA(gx::launch_moe_gemm(gm, 0, c->sm_count, c->stream));
    if (ev) GX_CUDA(record_phase(ev[2], c->stream));
    gx::PackArgs pd{};
    pd.src = p.act;
    pd.by_token = 0;
    pd.U = (int)U;
    pd.K = (int)L.F;
    pd.signs = L.down_signs;
    pd.row_slot = p.row_slot;
    pd.tile_rows = p.tile_rows;
    pd.n_mtiles = p.n_mtiles;
    pd.dst = p.A2;
    pd.compact = gx::gemm_ts_routed(L.type);
    if (!gx::gemm_ts_routed(L.type)) GX_CUDA(gx::launch_pack_rows(pd, (int)p.max_tiles, c->stream));
    gm.w0 = L.down;
    gm.w1 = nullptr;
    gm.expert_bytes = L.down_expert_bytes;
    gm.K = (int)L.F;
    gm.n_ntiles = (int)(L.E / 256);
    gm.A = p.A2;
    GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
    GX_CUDA(gx::launch_ep_return(pa, p.Y, p.slot_row, c->stream));
    GX_CUDA(gx::launch_ep_wait_ret(pa, c->stream));
    gx::EpCombineArgs ec{};
    ec.err = c->err;
    ec.ret = reinterpret_cast<const __half *>(e.block + e.off.ret_rows);
    ec.pos_of = e.pos_of;
    ec.W = W;
    ec.Ysh = L.sh_wt && n_tok ? c->sh.Ysh : nullptr;
    ec.sh_logit = c->sh.logit;
    ec.resid = resid;
    ec.resid_bf16 = resid_dtype == GX_BF16;
    ec.out = out;
    ec.out_bf16 = out_dtype == GX_BF16;
    ec.n_tok = (int)n_tok;
    ec.E = (int)E;
    GX_CUDA(gx::launch_ep_combine(ec, c->stream));
    if (ev) GX_CUDA(record_phase(ev[3], c->stream));
    return GX_OK;
}

// One layer across the expert-parallel group. ev (GX_FLAG_PROFILE): start, after the dispatch
// exchange (selection, rotation, plan, counts, rows), after the gate/up GEMM, end (down GEMM,
// partial rows, return exchange, sum).
gx_result enqueue_layer_ep(gx_context *c, const Layer &L, const void *x, uint32_t x_dtype, uint32_t n_tok,
                           const void *resid, uint32_t resid_dtype, void *out, uint32_t out_dtype, float norm_eps,
                           cudaEvent_t *ev) {
    const int W = (int)c->world;
    const size_t E = L.E, U = L.U;
    gx_result r = ensure_ep_send(c, L);
    if (r != GX_OK) return r;
    auto &e = c->ep;
    if (e.peer_state == 1 && ((int)L.E > e.pE || (int)L.U > e.pU)) {
        // a layer wider than the blocks (uploaded after the set-up): every rank reaches this
        // point in the same call, so all of them set the exchange up again at the new size
        r = ep_peer_teardown(c);
        if (r != GX_OK) return r;
    }
    if (e.peer_state == 0) {
        r = ep_peer_setup(c);
        if (r != GX_OK) return r;
    }
    const bool peer = e.peer_state == 1;
    const int xb = x_dtype == GX_BF16;
    // send rows reserved per destination: with peer memory, the largest token count of any rank
    // in this call (every rank knows all counts from ep_sync_ntok), the stride of the rx regions
    size_t S = 1;
    for (int v : e.src_ntok) S = std::max<size_t>(S, (size_t)v);
    if ((int)e.src_ntok.size() != W || S > (size_t)c->max_tokens) return GX_E_STATE;
    const size_t stride = peer ? S : (n_tok ? n_tok : 1);
    if (ev) GX_CUDA(record_phase(ev[0], c->stream));
    if (n_tok > 0) {
        int splits;
        GX_CUDA(launch_router_logits(c, L, x, xb, n_tok, &splits));
        gx::RouterArgs ra{};
        ra.W = L.router;
        ra.bias = L.bias;
        ra.x = x;
        ra.x_bf16 = xb;
        ra.n_tok = (int)n_tok;
        ra.NE = (int)L.n_expert;
        ra.E = (int)L.E;
        ra.U = (int)L.U;
        ra.scale = L.scale;
        ra.norm_eps = norm_eps;
        ra.ss = c->ss;
        ra.ss_from_x = 1;
        ra.logit_splits = splits;
        ra.xscale = c->xscale;
        ra.logits = c->logits;
        ra.ids = c->ids;
        ra.weights = c->weights;
        ra.err = c->err;
        GX_CUDA(gx::launch_topk(ra, c->stream));
        if (L.sh_wt) {
            // the shared expert is replicated: every rank computes it for its own tokens
            r = enqueue_shared_gemm(c, L, x, xb, n_tok, c->xscale);
            if (r != GX_OK) return r;
        }
    }
    gx::EpPlanArgs pa{};
    pa.ids = c->ids;
    pa.weights = c->weights;
    pa.n_tok = (int)n_tok;
    pa.U = (int)U;
    pa.NE = (int)L.n_expert;
    pa.W = W;
    pa.rank = (int)c->rank;
    pa.route = L.route;
    pa.expert_count = L.expert_count;
    pa.stride = (int)stride;
    pa.pad_rows = peer ? 0 : (int)n_tok;
    pa.pos_of = e.pos_of;
    pa.send_ids = e.send_ids;
    pa.send_w = e.send_w;
    pa.send_count = e.counts;
    pa.dest_mask = e.dest_mask;
    pa.block_count = e.block_count;
    pa.err = c->err;
    GX_CUDA(gx::launch_ep_plan(pa, c->stream));
    if (peer) return enqueue_layer_ep_peer(c, L, x, xb, n_tok, S, resid, resid_dtype, out, out_dtype, norm_eps, ev);
    GX_CUDA(gx::launch_rotate_tokens(x, xb, norm_eps > 0.f ? c->xscale : nullptr, L.gate_signs, (int)n_tok, (int)E,
                                     e.send_rows, c->stream, e.pos_of, W));
    // every source sends its n_tok rows to every rank (rows without a slot there are empty)
    if ((int)e.src_ntok.size() != W) return GX_E_STATE;
    std::vector<size_t> scnt(W, n_tok), rcnt(W), roff(W);
    size_t R = 0;
    for (int d = 0; d < W; ++d) {
        rcnt[d] = (size_t)e.src_ntok[d];
        roff[d] = R;
        R += rcnt[d];
    }
    if (R > e.src_cap) return comm_result(c, ncclInvalidUsage, "received more rows than the group can hold");
    r = ensure_ep_recv(c, R);
    if (r != GX_OK) return r;
    if (R > 0) {
        r = ensure_prefill(c, L, R * U);
        if (r != GX_OK) return r;
    }
    c->nccl->GroupStart();
    for (int d = 0; d < W; ++d) {
        const size_t so = (size_t)d * stride;
        if (scnt[d]) {
            c->nccl->Send(e.send_rows + so * E, scnt[d] * E, ncclFloat16, d, c->comm, c->stream);
            c->nccl->Send(e.send_ids + so * U, scnt[d] * U, ncclUint32, d, c->comm, c->stream);
            c->nccl->Send(e.send_w + so * U, scnt[d] * U, ncclFloat32, d, c->comm, c->stream);
        }
        if (rcnt[d]) {
            c->nccl->Recv(e.recv_rows + roff[d] * E, rcnt[d] * E, ncclFloat16, d, c->comm, c->stream);
            c->nccl->Recv(e.recv_ids + roff[d] * U, rcnt[d] * U, ncclUint32, d, c->comm, c->stream);
            c->nccl->Recv(e.recv_w + roff[d] * U, rcnt[d] * U, ncclFloat32, d, c->comm, c->stream);
        }
    }
    r = comm_group_end(c, "dispatch");
    if (r != GX_OK) return r;
    if (ev) GX_CUDA(record_phase(ev[1], c->stream));
    if (R > 0) {
        auto &p = c->pf;
        gx::GroupArgs ga{};
        ga.ids = e.recv_ids;
        ga.n_slots = (int)(R * U);
        ga.NE = (int)(L.local_experts + L.replica_slots);
        ga.expert_count = p.expert_count;
        ga.cursor = p.cursor;
        ga.tile_expert = p.tile_expert;
        ga.tile_rows = p.tile_rows;
        ga.n_mtiles = p.n_mtiles;
        ga.row_slot = p.row_slot;
        ga.slot_row = p.slot_row;
        ga.err = c->err;
        GX_CUDA(gx::launch_group(ga, c->stream));
        gx::PackArgs pk{};
        pk.by_token = 1;
        pk.U = (int)U;
        pk.K = (int)E;
        pk.xh = e.recv_rows;
        pk.row_slot = p.row_slot;
        pk.tile_rows = p.tile_rows;
        pk.n_mtiles = p.n_mtiles;
        pk.dst = p.A;
        pk.compact = gx::gemm_ts_routed(L.type);
        GX_CUDA(gx::launch_pack_rows(pk, (int)p.max_tiles, c->stream));
        gx::GemmArgs gm{};
        gm.type = L.type;
        gm.w0 = L.gate;
        gm.w1 = L.up;
        gm.expert_bytes = L.gate_expert_bytes;
        gm.K = (int)L.E;
        gm.n_ntiles = (int)(L.F / 128);
        gm.n_expert = (int)(L.local_experts + L.replica_slots);
        gm.A = p.A;
        gm.tile_expert = p.tile_expert;
        gm.tile_rows = p.tile_rows;
        gm.n_mtiles = p.n_mtiles;
        gm.act = p.act;
        gm.F = (int)L.F;
        gm.Y = p.Y;
        gm.E = (int)L.E;
        gm.codebook = c->codebook;
        gm.err = c->err;
        if (gx::gemm_ts_routed(L.type)) {
            gm.down_A = p.A2;   // the gate/up epilogue packs the down operand
            gm.down_signs = L.down_signs;
        }
        GX_CUDA(gx::launch_moe_gemm(gm, 0, c->sm_count, c->stream));
        if (ev) GX_CUDA(record_phase(ev[2], c->stream));
        gx::PackArgs pd{};
        pd.src = p.act;
        pd.by_token = 0;
        pd.U = (int)U;
        pd.K = (int)L.F;
        pd.signs = L.down_signs;
        pd.row_slot = p.row_slot;
        pd.tile_rows = p.tile_rows;
        pd.n_mtiles = p.n_mtiles;
        pd.dst = p.A2;
        pd.compact = gx::gemm_ts_routed(L.type);
        if (!gx::gemm_ts_routed(L.type)) GX_CUDA(gx::launch_pack_rows(pd, (int)p.max_tiles, c->stream));
        gm.w0 = L.down;
        gm.w1 = nullptr;
        gm.expert_bytes = L.down_expert_bytes;
        gm.K = (int)L.F;
        gm.n_ntiles = (int)(L.E / 256);
        gm.A = p.A2;
        GX_CUDA(gx::launch_moe_gemm(gm, 1, c->sm_count, c->stream));
        gx::CombineArgs ca{};
        ca.err = c->err;
        ca.Y = p.Y;
        ca.slot_row = p.slot_row;
        ca.weights = e.recv_w;
        ca.out = e.part_rows;
        ca.out_f16 = 1;
        ca.n_tok = (int)R;
        ca.U = (int)U;
        ca.E = (int)E;
        GX_CUDA(gx::launch_combine(ca, c->stream));
    } else if (ev) {
        GX_CUDA(record_phase(ev[2], c->stream));
    }
    c->nccl->GroupStart();
    for (int d = 0; d < W; ++d) {
        if (rcnt[d]) c->nccl->Send(e.part_rows + roff[d] * E, rcnt[d] * E, ncclFloat16, d, c->comm, c->stream);
        if (scnt[d])
            c->nccl->Recv(e.ret_rows + (size_t)d * stride * E, scnt[d] * E, ncclFloat16, d, c->comm, c->stream);
    }
    r = comm_group_end(c, "combine");
    if (r != GX_OK) return r;
    gx::EpCombineArgs ec{};
    ec.err = c->err;
    ec.ret = e.ret_rows;
    ec.pos_of = e.pos_of;
    ec.W = W;
    ec.Ysh = L.sh_wt && n_tok ? c->sh.Ysh : nullptr;
    ec.sh_logit = c->sh.logit;
    ec.resid = resid;
    ec.resid_bf16 = resid_dtype == GX_BF16;
    ec.out = out;
    ec.out_bf16 = out_dtype == GX_BF16;
    ec.n_tok = (int)n_tok;
    ec.E = (int)E;
    GX_CUDA(gx::launch_ep_combine(ec, c->stream));
    if (ev) GX_CUDA(record_phase(ev[3], c->stream));
    return GX_OK;
}

// One routed layer: router + top-k, gate/up + SwiGLU, down + combine (+ residual).
// prof_slot >= 0 records the phase events of layer slot prof_slot (GX_FLAG_PROFILE).
// norm_eps > 0 routes and feeds the experts RMSNorm(x) (unit weight); the residual stays x.
// chained: the previous operation on the stream is this library's down kernel.
gx_result enqueue_layer(gx_context *c, const Layer &L, const void *x, uint32_t x_dtype, uint32_t n_tok,
                        const void *resid, uint32_t resid_dtype, void *out, uint32_t out_dtype, int prof_slot,
                        float norm_eps, bool chained) {
    // programmatic dependent launch along the many-token chain for calls of up to
    // kChainPdlMaxTokens tokens on this rank, where its kernels are short enough for the launch
    // gaps to matter
    gx::set_chain_pdl(n_tok <= kChainPdlMaxTokens);
    if (c->world > 1) {
        cudaEvent_t *pev = prof_slot >= 0 ? &c->prof[4 * (size_t)prof_slot] : nullptr;
        return enqueue_layer_ep(c, L, x, x_dtype, n_tok, resid, resid_dtype, out, out_dtype, norm_eps, pev);
    }
    if (n_tok >= kPrefillMinTokens && L.n_expert <= 512 && L.E % 256 == 0) {
        cudaEvent_t *pev = prof_slot >= 0 ? &c->prof[4 * (size_t)prof_slot] : nullptr;
        return enqueue_layer_prefill(c, L, x, x_dtype, n_tok, resid, resid_dtype, out, out_dtype, norm_eps, pev);
    }
    cudaEvent_t *ev = prof_slot >= 0 ? &c->prof[4 * (size_t)prof_slot] : nullptr;
    if (ev) GX_CUDA(record_phase(ev[0], c->stream));
    gx::RouterArgs ra{};
    ra.W = L.router;
    ra.bias = L.bias;
    ra.x = x;
    ra.x_bf16 = x_dtype == GX_BF16;
    ra.n_tok = (int)n_tok;
    ra.NE = (int)L.n_expert;
    ra.E = (int)L.E;
    ra.U = (int)L.U;
    ra.scale = L.scale;
    ra.norm_eps = norm_eps;
    ra.ss = c->ss;
    ra.logit_splits = 1;
    ra.xscale = c->xscale;
    ra.logits = c->logits;
    ra.ids = c->ids;
    ra.weights = c->weights;
    ra.err = c->err;
    // the router's last CTA selects for a few tokens; otherwise gate_up_kernel or topk_kernel
    const bool sel_router = n_tok <= (uint32_t)gx::kRouterSelectTok;
    ra.done = sel_router ? c->router_done : nullptr;
    const bool fused = !sel_router && gx::gate_up_fuses_topk((int)L.E, (int)L.F, (int)L.U, (int)n_tok, c->sm_count);
    // Programmatic overlap only between kernels of this chain: never across the phase events
    // of a profiled call, and not for the first kernel of a call (its predecessor is a copy).
    const bool pdl = ev == nullptr && chained;
    GX_CUDA(gx::launch_router(ra, c->stream, pdl, !fused && !sel_router));
    if (ev) GX_CUDA(record_phase(ev[1], c->stream));
    if (L.sh_wt) {
        gx_result r = enqueue_shared_decode(c, L, x, x_dtype == GX_BF16, n_tok, norm_eps, ev == nullptr);
        if (r != GX_OK) return r;
    }

    gx::GateUpArgs ga{};
    ga.type = L.type;
    ga.gate = L.gate;
    ga.up = L.up;
    ga.expert_bytes = L.gate_expert_bytes;
    ga.x = x;
    ga.x_bf16 = x_dtype == GX_BF16;
    ga.signs = L.gate_signs;
    ga.xscale = norm_eps > 0.f ? c->xscale : nullptr;
    ga.ids = c->ids;
    ga.fused_topk = fused;
    ga.logits = c->logits;
    ga.bias = L.bias;
    ga.ss = c->ss;
    ga.NE = (int)L.n_expert;
    ga.norm_eps = norm_eps;
    ga.wscale = L.scale;
    ga.ids_out = c->ids;
    ga.weights_out = c->weights;
    ga.act = c->act;
    ga.codebook = c->codebook;
    ga.codebook_image = c->codebook_image;
    ga.E = (int)L.E;
    ga.F = (int)L.F;
    ga.U = (int)L.U;
    ga.n_slots = (int)(n_tok * L.U);
    ga.n_expert = (int)L.local_experts;
    ga.err = c->err;
    GX_CUDA(gx::launch_gate_up(ga, c->sm_count, c->stream, ev == nullptr));
    if (ev) GX_CUDA(record_phase(ev[2], c->stream));

    gx::DownArgs da{};
    da.type = L.type;
    da.down = L.down;
    da.expert_bytes = L.down_expert_bytes;
    da.act = c->act;
    da.signs = L.down_signs;
    da.ids = c->ids;
    da.weights = c->weights;
    da.resid = resid;
    da.resid_bf16 = resid_dtype == GX_BF16;
    da.extra = L.sh_wt ? c->sh.y : nullptr;
    da.out = out;
    da.out_bf16 = out_dtype == GX_BF16;
    da.codebook = c->codebook;
    da.codebook_image = c->codebook_image;
    da.E = (int)L.E;
    da.F = (int)L.F;
    da.U = (int)L.U;
    da.n_tok = (int)n_tok;
    da.n_expert = (int)L.local_experts;
    da.err = c->err;
    GX_CUDA(gx::launch_down(da, c->sm_count, c->stream, ev == nullptr));
    if (ev) GX_CUDA(record_phase(ev[3], c->stream));
    return GX_OK;
}

gx_result check_forward(gx_context *c, uint32_t layer, uint32_t x_dtype, uint32_t n_tok, uint32_t y_dtype) {
    if (!c) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    if ((x_dtype != GX_F32 && x_dtype != GX_BF16) || (y_dtype != GX_F32 && y_dtype != GX_BF16)) return GX_E_INVALIDARG;
    if (n_tok > c->max_tokens) return GX_E_INVALIDARG;
    return GX_OK;
}

gx_result stack_enqueue(gx_context *c, uint32_t first, uint32_t n_layers, const void *x, uint32_t x_dtype,
                        uint32_t n_tok, void *y, uint32_t y_dtype) {
    const void *cur = x;
    uint32_t cur_dtype = x_dtype;
    if (c->flags & GX_FLAG_PROFILE) {
        c->prof_layers = n_layers;
        c->prof_stack = 0;
    }
    for (uint32_t i = 0; i < n_layers; ++i) {
        const Layer &L = c->layers[first + i];
        const bool last = i + 1 == n_layers;
        void *out = last ? y : c->xbuf[i & 1];
        const uint32_t out_dtype = last ? y_dtype : GX_F32;
        const int slot = (c->flags & GX_FLAG_PROFILE) ? (int)i : -1;
        gx_result r = enqueue_layer(c, L, cur, cur_dtype, n_tok, cur, cur_dtype, out, out_dtype, slot, kStackNormEps,
                                    i > 0);
        if (r != GX_OK) return r;
        cur = out;
        cur_dtype = out_dtype;
    }
    return GX_OK;
}

// Whether a stack call runs as one persistent decode-stack kernel instead of the PDL-chained
// per-phase kernels: opt-in with GX_STACK_KERNEL=1 (at batch 1 on B200 the chained kernels are
// faster: its phases are short serial sections separated by grid barriers), one GPU, few tokens,
// and every layer of the same type and shape within the kernel's limits.
bool stack_kernel_fits(gx_context *c, uint32_t first, uint32_t n_layers, uint32_t n_tok) {
    const char *opt = std::getenv("GX_STACK_KERNEL");
    if (!opt || opt[0] != '1') return false;
    if (c->world != 1 || n_tok == 0 || n_tok >= kPrefillMinTokens) return false;
    const Layer &L0 = c->layers[first];
    for (uint32_t i = 0; i < n_layers; ++i) {
        const Layer &L = c->layers[first + i];
        if (L.type != L0.type || L.E != L0.E || L.F != L0.F || L.U != L0.U || L.n_expert != L0.n_expert) return false;
        if (L.sh_wt) return false;  // the persistent kernel has no shared-expert phase
    }
    return L0.n_expert <= 4u * (uint32_t)c->sm_count &&
           gx::decode_stack_supported(L0.type, (int)L0.E, (int)L0.F, (int)L0.U, (int)L0.n_expert, (int)n_tok);
}

// The whole stack (pre-norm residual chain) as one cooperative kernel launch.
gx_result enqueue_stack_kernel(gx_context *c, uint32_t first, uint32_t n_layers, const void *x, uint32_t x_dtype,
                               uint32_t n_tok, void *y, uint32_t y_dtype) {
    const Layer &L0 = c->layers[first];
    const bool prof = (c->flags & GX_FLAG_PROFILE) != 0;
    if (prof) {
        c->prof_layers = 0;
        c->prof_stack = n_layers;
        GX_CUDA(record_phase(c->prof[0], c->stream));
    }
    gx::StackArgs a{};
    a.layers = c->stack_table + first;
    a.n_layers = (int)n_layers;
    a.x = x;
    a.x_bf16 = x_dtype == GX_BF16;
    a.out = y;
    a.out_bf16 = y_dtype == GX_BF16;
    a.xa = c->xbuf[0];
    a.xb = c->xbuf[1];
    a.logits = c->logits;
    a.act = c->act;
    a.codebook = c->codebook;
    a.sync = c->stack_sync;
    a.n_tok = (int)n_tok;
    a.NE = (int)L0.n_expert;
    a.E = (int)L0.E;
    a.F = (int)L0.F;
    a.U = (int)L0.U;
    a.norm_eps = kStackNormEps;
    a.residual = 1;
    a.err = c->err;
    GX_CUDA(gx::launch_decode_stack(a, L0.type, c->sm_count, c->stream));
    if (prof) GX_CUDA(record_phase(c->prof[3], c->stream));
    return GX_OK;
}

// Joins the expert-parallel group: a non-blocking NCCL communicator over all ranks' contexts,
// bounded by the communication timeout (GX_COMM_TIMEOUT_MS in the environment, default 120 s).
gx_result open_group(gx_context *c, const gx_options *o) {
    c->nccl = gx::nccl_api();
    if (!c->nccl) return GX_E_UNSUPPORTED;
    if (const char *v = std::getenv("GX_COMM_TIMEOUT_MS")) {
        const long ms = std::strtol(v, nullptr, 10);
        if (ms > 0) c->comm_timeout_ms = (uint32_t)ms;
    }
    ncclUniqueId id;
    std::memcpy(id.internal, o->nccl_id, sizeof(id.internal));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t nr = c->nccl->CommInitRankConfig(&c->comm, (int)c->world, id, (int)c->rank, &cfg);
    if (nr == ncclSuccess || nr == ncclInProgress) nr = gx::nccl_settle(c->nccl, c->comm, c->comm_timeout_ms);
    if (nr != ncclSuccess) {
        if (debug_enabled())
            std::fprintf(stderr, "gyro_moe: joining the expert-parallel group failed: %s\n",
                         nr == ncclInProgress ? "not all ranks joined within the timeout" : c->nccl->GetErrorString(nr));
        if (c->comm) c->nccl->CommAbort(c->comm);
        c->comm = nullptr;
        return GX_E_COMM;
    }
    return GX_OK;
}

}  // namespace

extern "C" {

GX_API gx_result gx_comm_unique_id(uint8_t *out_id, uint64_t bytes) {
    if (!out_id || bytes != sizeof(ncclUniqueId)) return GX_E_INVALIDARG;
    const gx::NcclApi *api = gx::nccl_api();
    if (!api) return GX_E_UNSUPPORTED;
    ncclUniqueId id;
    if (api->GetUniqueId(&id) != ncclSuccess) return GX_E_COMM;
    std::memcpy(out_id, id.internal, sizeof(id.internal));
    return GX_OK;
}

GX_API gx_result gx_create(const gx_options *o, gx_context **out) {
    if (!o || !out || !o->codebook || o->codebook_bytes != 8192 || o->world == 0 || o->rank >= o->world ||
        o->max_tokens == 0 || o->max_layers == 0 || o->max_tokens > (1u << 20) || o->world > (uint32_t)gx::kMaxEpWorld)
        return GX_E_INVALIDARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || (int)o->device >= n) return GX_E_INVALIDARG;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, (int)o->device) != cudaSuccess) return GX_E_DEVICE;
    if (prop.major != 10) return GX_E_UNSUPPORTED;
    gx_context *c = new (std::nothrow) gx_context();
    if (!c) return GX_E_OUTOFMEMORY;
    c->device = (int)o->device;
    c->rank = o->rank;
    c->world = o->world;
    c->max_tokens = o->max_tokens;
    c->max_layers = o->max_layers;
    c->flags = o->flags;
    c->sm_count = prop.multiProcessorCount;
    c->layers.resize(o->max_layers);
    gx_result r = GX_OK;
    do {
        if (cudaSetDevice(c->device) != cudaSuccess) { r = GX_E_DEVICE; break; }
        if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) { r = GX_E_DEVICE; break; }
        bool ok = true;
        for (auto &e : c->events) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
        c->prof.assign(4 * (size_t)c->max_layers, nullptr);
        for (auto &e : c->prof) ok = ok && cudaEventCreate(&e) == cudaSuccess;
        if (!ok) { r = GX_E_DEVICE; break; }
        if (cudaMalloc(&c->codebook, 8192) != cudaSuccess) { r = GX_E_OUTOFMEMORY; break; }
        if (cudaMemcpy(c->codebook, o->codebook, 8192, cudaMemcpyHostToDevice) != cudaSuccess) { r = GX_E_DEVICE; break; }
        {
            // word w of the image is codebook word w / kCodebookCopies (copy w % kCodebookCopies)
            std::vector<uint32_t> image(2048 * (size_t)gx::kCodebookCopies);
            const uint32_t *words = static_cast<const uint32_t *>(o->codebook);
            for (size_t w = 0; w < image.size(); ++w) image[w] = words[w / gx::kCodebookCopies];
            const size_t bytes = image.size() * sizeof(uint32_t);
            if (cudaMalloc(&c->codebook_image, bytes) != cudaSuccess) { r = GX_E_OUTOFMEMORY; break; }
            if (cudaMemcpy(c->codebook_image, image.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
                r = GX_E_DEVICE;
                break;
            }
        }
        if (cudaMalloc(&c->router_done, sizeof(unsigned)) != cudaSuccess) { r = GX_E_OUTOFMEMORY; break; }
        if (cudaMemset(c->router_done, 0, sizeof(unsigned)) != cudaSuccess) { r = GX_E_DEVICE; break; }
        r = ensure_scratch(c);
        if (r != GX_OK || c->world == 1) break;
        if (const char *v = std::getenv("GX_EP_WAIT_MS")) {
            const long ms = std::strtol(v, nullptr, 10);
            if (ms > 0) c->ep.wait_ns = (uint64_t)ms * 1000000ull;
        }
        if (const char *v = std::getenv("GX_EP_FAULT_SKIP_PUSH")) c->ep.fault_skip_push = (unsigned)std::strtoul(v, nullptr, 10);
        r = open_group(c, o);
    } while (false);
    if (r != GX_OK) {
        release_all(c);
        delete c;
        return r;
    }
    *out = c;
    return GX_OK;
}

GX_API gx_result gx_get_caps(gx_context *c, gx_caps *caps) {
    if (!c || !caps) return GX_E_INVALIDARG;
    std::memset(caps, 0, sizeof(*caps));
    cudaDeviceProp prop{};
    GX_CUDA(cudaGetDeviceProperties(&prop, c->device));
    size_t free_b = 0, total_b = 0;
    GX_CUDA(cudaSetDevice(c->device));
    GX_CUDA(cudaMemGetInfo(&free_b, &total_b));
    caps->abi_version = GX_ABI_VERSION;
    caps->sm_count = (uint32_t)prop.multiProcessorCount;
    caps->cc_major = (uint32_t)prop.major;
    caps->cc_minor = (uint32_t)prop.minor;
    caps->rank = c->rank;
    caps->world = c->world;
    caps->max_tokens = c->max_tokens;
    caps->max_layers = c->max_layers;
    caps->hbm_bytes = total_b;
    caps->free_bytes = free_b;
    caps->l2_bytes = (uint64_t)prop.l2CacheSize;
    for (auto &l : c->layers) caps->arena_bytes += l.bytes + l.sh_bytes + l.hc_bytes;
    for (auto &m : c->mats) caps->arena_bytes += (uint64_t)m.rows / 8 * (m.cols / 128) * gx::tile_bytes(m.type);
    std::strncpy(caps->device_name, prop.name, sizeof(caps->device_name) - 1);
    caps->ep_exchange = c->ep.peer_state == 1 ? GX_EP_PEER : c->ep.peer_state == -1 ? GX_EP_NCCL : GX_EP_NONE;
    caps->ep_peer_layers = c->ep.peer_layers;
    return GX_OK;
}

GX_API gx_result gx_upload_layer(gx_context *c, uint32_t layer, const gx_layer_desc *d, uint32_t timeout_ms) {
    if (!c || !d) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size()) return GX_E_INVALIDARG;
    if (!known_type(d->type_id) || d->n_expert == 0 || d->n_expert > 512 || d->n_embd == 0 || d->n_embd % 128 ||
        d->n_embd > 4096 || d->n_ff == 0 || d->n_ff % 128 || d->n_ff > 1024 || d->n_used == 0 || d->n_used > 16 ||
        d->n_used > d->n_expert || !d->gate || !d->up || !d->down || !d->router)
        return GX_E_INVALIDARG;
    if (d->n_used * (d->n_ff / 128) > 64) return GX_E_UNSUPPORTED;
    if (d->n_expert % c->world) return GX_E_INVALIDARG;
    if (c->world > 1 && d->n_embd % 256) return GX_E_UNSUPPORTED;  // expert-parallel rows use the GEMM path
    const uint64_t bb = (uint64_t)gx::type_block_bytes(d->type_id);
    const uint64_t E = d->n_embd, F = d->n_ff, NE = d->n_expert;
    const uint64_t gate_row = E / 128 * bb, down_row = F / 128 * bb;
    if (d->gate_bytes != NE * F * gate_row || d->up_bytes != NE * F * gate_row || d->down_bytes != NE * E * down_row)
        return GX_E_INVALIDARG;
    if (d->up_signs && (!d->gate_signs || std::memcmp(d->up_signs, d->gate_signs, E * sizeof(float)) != 0))
        return GX_E_INVALIDARG;  // gate and up share one rotated input (src/gpu_engine.zig:404)
    if (d->up_signs == nullptr && d->gate_signs != nullptr) return GX_E_INVALIDARG;
    const float *signs[2] = {d->gate_signs, d->down_signs};
    const uint64_t widths[2] = {E, F};
    for (int s = 0; s < 2; ++s)
        if (signs[s])
            for (uint64_t i = 0; i < widths[s]; ++i)
                if (signs[s][i] != 1.0f && signs[s][i] != -1.0f) return GX_E_INVALIDARG;

    GX_CUDA(cudaSetDevice(c->device));
    Layer &L = c->layers[layer];
    if (L.arena) {
        gx_result r = sync_all(c, timeout_ms);
        if (r != GX_OK) return r;
        cudaFree(L.arena);
        if (L.sh_arena) cudaFree(L.sh_arena);
        if (L.hc_arena) cudaFree(L.hc_arena);
        L = Layer{};
    }
    const uint64_t NEl = NE / c->world, first = c->rank * NEl;
    const uint64_t gate_local = NEl * F * gate_row, down_local = NEl * E * down_row;
    const uint64_t R = c->world > 1 ? std::min<uint64_t>(kMaxReplicas, NE - NEl) : 0;  // replica slots
    uint64_t off = 0;
    const uint64_t o_gate = off; off = align256(off + (NEl + R) * F * gate_row);
    const uint64_t o_up = off; off = align256(off + (NEl + R) * F * gate_row);
    const uint64_t o_down = off; off = align256(off + (NEl + R) * E * down_row);
    const uint64_t o_route = off; off = align256(off + (c->world > 1 ? NE * sizeof(int2) : 0));
    const uint64_t o_count = off; off = align256(off + (c->world > 1 ? NE * sizeof(unsigned) : 0));
    const uint64_t o_router = off; off = align256(off + NE * E * 4);
    const uint64_t o_bias = off; off = align256(off + NE * 4);
    const uint64_t o_gs = off; off = align256(off + E * 4);
    const uint64_t o_ds = off; off = align256(off + F * 4);
    const bool with_parts = E % 64 == 0;
    const uint64_t o_rp = off; off = align256(off + (with_parts ? gx::router_parts_bytes((int)NE, (int)E) : 0));
    uint8_t *arena = nullptr;
    GX_CUDA(cudaMalloc(&arena, off));
    uint8_t *raw = nullptr;
    cudaError_t e = cudaMalloc(&raw, gate_local > down_local ? gate_local : down_local);
    if (e != cudaSuccess) {
        cudaFree(arena);
        return fail_cuda(c, e);
    }
    struct Part { const void *src; uint64_t row_bytes, rows, cols, dst; };
    const Part parts[3] = {
        {static_cast<const uint8_t *>(d->gate) + first * F * gate_row, gate_row, NEl * F, E, o_gate},
        {static_cast<const uint8_t *>(d->up) + first * F * gate_row, gate_row, NEl * F, E, o_up},
        {static_cast<const uint8_t *>(d->down) + first * E * down_row, down_row, NEl * E, F, o_down},
    };
    for (const Part &p : parts) {
        if (e == cudaSuccess) e = cudaMemcpyAsync(raw, p.src, p.rows * p.row_bytes, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess)
            e = gx::launch_repack(d->type_id, raw, p.row_bytes, (uint32_t)p.rows, (uint32_t)p.cols, arena + p.dst, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(arena + o_router, d->router, NE * E * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        if (d->router_bias) e = cudaMemcpyAsync(arena + o_bias, d->router_bias, NE * 4, cudaMemcpyHostToDevice, c->stream);
        else e = cudaMemsetAsync(arena + o_bias, 0, NE * 4, c->stream);
    }
    if (e == cudaSuccess && d->gate_signs)
        e = cudaMemcpyAsync(arena + o_gs, d->gate_signs, E * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && d->down_signs)
        e = cudaMemcpyAsync(arena + o_ds, d->down_signs, F * 4, cudaMemcpyHostToDevice, c->stream);
    std::vector<int2> route;
    if (e == cudaSuccess && c->world > 1) {
        route.resize(NE);
        for (uint64_t x = 0; x < NE; ++x) route[x] = make_int2((int)(x / NEl), (int)(x % NEl));
        e = cudaMemcpyAsync(arena + o_route, route.data(), NE * sizeof(int2), cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(arena + o_count, 0, NE * sizeof(unsigned), c->stream);
    }
    std::vector<uint16_t> rparts;
    if (e == cudaSuccess && with_parts) {
        rparts = router_parts(d->router, NE, E);
        e = cudaMemcpyAsync(arena + o_rp, rparts.data(), rparts.size() * 2, cudaMemcpyHostToDevice, c->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(raw);
    if (e != cudaSuccess) {
        cudaFree(arena);
        return fail_cuda(c, e);
    }
    L.ready = true;
    L.type = d->type_id;
    L.n_expert = (uint32_t)NE;
    L.local_experts = (uint32_t)NEl;
    L.first_expert = (uint32_t)first;
    L.E = (uint32_t)E;
    L.F = (uint32_t)F;
    L.U = d->n_used;
    L.scale = d->expert_weights_scale;
    L.arena = arena;
    L.bytes = off;
    L.gate = arena + o_gate;
    L.up = arena + o_up;
    L.down = arena + o_down;
    L.gate_expert_bytes = F * gate_row;
    L.down_expert_bytes = E * down_row;
    L.router = reinterpret_cast<float *>(arena + o_router);
    L.bias = reinterpret_cast<float *>(arena + o_bias);
    L.gate_signs = d->gate_signs ? reinterpret_cast<float *>(arena + o_gs) : nullptr;
    L.down_signs = d->down_signs ? reinterpret_cast<float *>(arena + o_ds) : nullptr;
    L.router_parts = with_parts ? arena + o_rp : nullptr;
    L.replica_slots = (uint32_t)R;
    L.replicas.clear();
    L.route = c->world > 1 ? reinterpret_cast<int2 *>(arena + o_route) : nullptr;
    L.expert_count = c->world > 1 ? reinterpret_cast<unsigned *>(arena + o_count) : nullptr;
    {
        gx::StackLayer sl{};
        sl.router = L.router;
        sl.bias = L.bias;
        sl.gate_signs = L.gate_signs;
        sl.down_signs = L.down_signs;
        sl.gate = L.gate;
        sl.up = L.up;
        sl.down = L.down;
        sl.gate_expert_bytes = L.gate_expert_bytes;
        sl.down_expert_bytes = L.down_expert_bytes;
        sl.scale = L.scale;
        GX_CUDA(cudaMemcpy(c->stack_table + layer, &sl, sizeof(sl), cudaMemcpyHostToDevice));
    }
    // A re-uploaded layer invalidates captured stacks.
    for (auto &kv : c->graphs) {
        cudaGraphExecDestroy(kv.second.second);
        cudaGraphDestroy(kv.second.first);
    }
    c->graphs.clear();
    return GX_OK;
}

namespace {

// Bytes of one source row of cols values in a non-expert encoding (0: not one of them).
uint64_t dense_row_bytes(uint32_t type, uint64_t cols) {
    if (type == GX_Q8_0) return cols % 32 ? 0 : cols / 32 * 34;
    if (type == GX_BF16) return cols * 2;
    if (type == GX_F32) return cols * 4;
    return 0;
}

// A plain row-major matrix in host memory (src/gguf.zig's row layout of Q8_0, bf16 and f32).
struct DenseMat {
    const uint8_t *src;
    uint64_t rows, cols, row_bytes;
};

// Arena offsets of a matrix's device encoding: weights at *o_w, Q8_0 block scales at *o_d.
void dense_place(uint32_t type, const DenseMat &m, uint64_t *off, uint64_t *o_w, uint64_t *o_d) {
    const bool q8 = type == GX_Q8_0;
    *o_w = *off;
    *off = align256(*off + m.rows * m.cols * (q8 ? 1 : 2));
    *o_d = *off;
    *off = align256(*off + (q8 ? m.rows * (m.cols / 32) * 2 : 0));
}

// Device encoding into zeroed host memory: Q8_0 split into int8 weights w [rows][ld] and fp16
// block scales d [rows][ld/32]; bf16 and f32 as fp16 w [rows][ld] (bf16 values convert exactly
// within the fp16 range, f32 values are rounded once). ld >= cols (0: cols); columns past cols
// stay zero.
void dense_encode(uint32_t type, const DenseMat &M, uint8_t *w_out, uint8_t *d_out, uint64_t ld = 0) {
    if (ld == 0) ld = M.cols;
    for (uint64_t r = 0; r < M.rows; ++r) {
        const uint8_t *row = M.src + r * M.row_bytes;
        if (type == GX_Q8_0) {
            int8_t *w = reinterpret_cast<int8_t *>(w_out) + r * ld;
            uint16_t *sc = reinterpret_cast<uint16_t *>(d_out) + r * (ld / 32);
            for (uint64_t b = 0; b < M.cols / 32; ++b) {
                std::memcpy(&sc[b], row + 34 * b, 2);
                std::memcpy(&w[32 * b], row + 34 * b + 2, 32);
            }
        } else {
            __half *w = reinterpret_cast<__half *>(w_out) + r * ld;
            for (uint64_t i = 0; i < M.cols; ++i) {
                float v;
                if (type == GX_BF16) {
                    const uint32_t bits = ((uint32_t)row[2 * i] | ((uint32_t)row[2 * i + 1] << 8)) << 16;
                    std::memcpy(&v, &bits, 4);
                } else {
                    std::memcpy(&v, row + 4 * i, 4);
                }
                w[i] = __float2half_rn(v);
            }
        }
    }
}

void drop_graphs(gx_context *c) {
    for (auto &kv : c->graphs) {
        cudaGraphExecDestroy(kv.second.second);
        cudaGraphDestroy(kv.second.first);
    }
    c->graphs.clear();
}

}  // namespace

GX_API gx_result gx_upload_shared(gx_context *c, uint32_t layer, const gx_shared_desc *d, uint32_t timeout_ms) {
    if (!c) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    Layer &L = c->layers[layer];
    const uint64_t E = L.E;
    uint64_t row_in = 0, row_sf = 0, SF = 0;
    if (d) {
        SF = d->n_ff;
        if (SF == 0 || SF % 128 || SF > 4096 || !d->gate || !d->up || !d->down || !d->gate_inp) return GX_E_INVALIDARG;
        row_in = dense_row_bytes(d->type_id, E);
        row_sf = dense_row_bytes(d->type_id, SF);
        if (!row_in || !row_sf) return GX_E_INVALIDARG;
        if (d->gate_bytes != SF * row_in || d->up_bytes != SF * row_in || d->down_bytes != E * row_sf)
            return GX_E_INVALIDARG;
        if (E % 256) return GX_E_UNSUPPORTED;
    }
    GX_CUDA(cudaSetDevice(c->device));
    if (L.sh_arena) {
        gx_result r = sync_all(c, timeout_ms);  // queued calls may still read the old matrices
        if (r != GX_OK) return r;
        cudaFree(L.sh_arena);
    }
    L.sh_arena = nullptr;
    L.sh_wt = 0;
    L.SF = 0;
    L.sh_bytes = 0;
    L.sh_gate = L.sh_up = L.sh_down = gx::SharedMat{};
    L.sh_gate_inp = nullptr;
    for (auto &kv : c->graphs) {  // captured stacks of this layer ran without (or with the old) shared expert
        cudaGraphExecDestroy(kv.second.second);
        cudaGraphDestroy(kv.second.first);
    }
    c->graphs.clear();
    if (!d) return GX_OK;

    const bool q8 = d->type_id == GX_Q8_0;
    const DenseMat mats[3] = {{static_cast<const uint8_t *>(d->gate), SF, E, row_in},
                              {static_cast<const uint8_t *>(d->up), SF, E, row_in},
                              {static_cast<const uint8_t *>(d->down), E, SF, row_sf}};
    uint64_t off = 0, o_w[3], o_d[3];
    for (int m = 0; m < 3; ++m) dense_place(d->type_id, mats[m], &off, &o_w[m], &o_d[m]);
    const uint64_t o_gi = off;
    off = align256(off + E * 4);
    std::vector<uint8_t> host(off, 0);
    for (int m = 0; m < 3; ++m) dense_encode(d->type_id, mats[m], host.data() + o_w[m], host.data() + o_d[m]);
    std::memcpy(host.data() + o_gi, d->gate_inp, E * 4);
    gx_result r = ensure_shared(c, E, SF);
    if (r != GX_OK) return r;
    uint8_t *arena = nullptr;
    GX_CUDA(cudaMalloc(&arena, off));
    cudaError_t e = cudaMemcpy(arena, host.data(), off, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(arena);
        return fail_cuda(c, e);
    }
    L.sh_arena = arena;
    L.sh_bytes = off;
    L.sh_wt = q8 ? gx::W_Q8 : gx::W_F16;
    L.SF = (uint32_t)SF;
    gx::SharedMat *dst[3] = {&L.sh_gate, &L.sh_up, &L.sh_down};
    for (int m = 0; m < 3; ++m) {
        dst[m]->w = arena + o_w[m];
        dst[m]->d = q8 ? reinterpret_cast<const __half *>(arena + o_d[m]) : nullptr;
    }
    L.sh_gate_inp = reinterpret_cast<float *>(arena + o_gi);
    return GX_OK;
}

GX_API gx_result gx_upload_hc(gx_context *c, uint32_t layer, const gx_hc_desc *d, uint32_t timeout_ms) {
    if (!c) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    Layer &L = c->layers[layer];
    const uint64_t E = L.E;
    uint64_t H = 0, R = 0, HD = 0, row_hd = 0, row_r = 0;
    if (d) {
        H = d->n_streams;
        R = d->rank;
        HD = H * E;
        if (H == 0 || H > 8 || R == 0 || R % 64 || R > 4096 || !d->norm || !d->down || !d->up || !d->inject ||
            !(d->eps > 0.f))
            return GX_E_INVALIDARG;
        row_hd = dense_row_bytes(d->type_id, HD);
        row_r = dense_row_bytes(d->type_id, R);
        if (!row_hd || !row_r) return GX_E_INVALIDARG;
        if (d->down_bytes != R * row_hd || d->up_bytes != HD * row_r || d->inject_bytes != H * row_hd)
            return GX_E_INVALIDARG;
        if (E % 256) return GX_E_UNSUPPORTED;
    }
    GX_CUDA(cudaSetDevice(c->device));
    if (L.hc_arena) {
        gx_result r = sync_all(c, timeout_ms);  // queued blocks may still read the old weights
        if (r != GX_OK) return r;
        cudaFree(L.hc_arena);
    }
    L.hc_arena = nullptr;
    L.hc_bytes = 0;
    L.hc_wt = L.H = L.R = L.Rp = 0;
    L.hc_down = L.hc_up = L.hc_inject = gx::SharedMat{};
    L.hc_norm = nullptr;
    if (!d) return GX_OK;

    // The rank is padded with zeros to Rk (a multiple of 128, the operand packing's block): Up gets
    // zero columns, Down zero rows, and lo = silu(0) = 0 there, so every sum is unchanged. Down has
    // Rp >= Rk rows (a multiple of 256) for the tensor-core path's column tiles of Down xn.
    const uint64_t Rk = (R + 127) / 128 * 128, Rp = (R + 255) / 256 * 256;
    const DenseMat mats[3] = {{static_cast<const uint8_t *>(d->down), R, HD, row_hd},
                              {static_cast<const uint8_t *>(d->up), HD, R, row_r},
                              {static_cast<const uint8_t *>(d->inject), H, HD, row_hd}};
    const DenseMat shapes[3] = {{nullptr, Rp, HD, 0}, {nullptr, HD, Rk, 0}, mats[2]};
    uint64_t off = 0, o_w[3], o_d[3];
    for (int m = 0; m < 3; ++m) dense_place(d->type_id, shapes[m], &off, &o_w[m], &o_d[m]);
    const uint64_t o_norm = off;
    off = align256(off + HD * 4);
    std::vector<uint8_t> host(off, 0);
    for (int m = 0; m < 3; ++m)
        dense_encode(d->type_id, mats[m], host.data() + o_w[m], host.data() + o_d[m], shapes[m].cols);
    std::memcpy(host.data() + o_norm, d->norm, HD * 4);
    gx_result r = ensure_hc(c, E, HD, Rp);
    if (r != GX_OK) return r;
    uint8_t *arena = nullptr;
    GX_CUDA(cudaMalloc(&arena, off));
    cudaError_t e = cudaMemcpy(arena, host.data(), off, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(arena);
        return fail_cuda(c, e);
    }
    const bool q8 = d->type_id == GX_Q8_0;
    L.hc_arena = arena;
    L.hc_bytes = off;
    L.hc_wt = q8 ? gx::W_Q8 : gx::W_F16;
    L.H = (uint32_t)H;
    L.R = (uint32_t)Rk;
    L.Rp = (uint32_t)Rp;
    L.hc_eps = d->eps;
    gx::SharedMat *dst[3] = {&L.hc_down, &L.hc_up, &L.hc_inject};
    for (int m = 0; m < 3; ++m) {
        dst[m]->w = arena + o_w[m];
        dst[m]->d = q8 ? reinterpret_cast<const __half *>(arena + o_d[m]) : nullptr;
    }
    L.hc_norm = reinterpret_cast<float *>(arena + o_norm);
    return GX_OK;
}

GX_API gx_result gx_moe_forward(gx_context *c, uint32_t layer, const void *x, uint32_t x_dtype, uint32_t n_tok,
                                void *y, uint32_t y_dtype, uint32_t *ids, float *weights, uint64_t *out_ticket) {
    gx_result r = check_forward(c, layer, x_dtype, n_tok, y_dtype);
    if (r != GX_OK) return r;
    if (n_tok > 0 && (!x || !y)) return GX_E_INVALIDARG;
    // Vector loads need 16-byte aligned activations; outputs are written as 4-byte words.
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 3) || ((uintptr_t)ids & 3) || ((uintptr_t)weights & 3))
        return GX_E_INVALIDARG;
    GX_CUDA(cudaSetDevice(c->device));
    const Layer &L = c->layers[layer];
    if (n_tok > 0 || c->world > 1) {  // with world > 1 every rank takes part in the exchange
        if (c->world > 1) {
            r = ep_sync_ntok(c, n_tok);
            if (r != GX_OK) return r;
        }
        const bool prof = (c->flags & GX_FLAG_PROFILE) != 0;
        if (prof) {
            c->prof_layers = 1;
            c->prof_stack = 0;
        }
        r = enqueue_layer(c, L, x, x_dtype, n_tok, nullptr, GX_F32, y, y_dtype, prof ? 0 : -1, 0.f, false);
        if (r != GX_OK) return r;
    }
    if (n_tok > 0) {
        if (ids) GX_CUDA(cudaMemcpyAsync(ids, c->ids, (size_t)n_tok * L.U * 4, cudaMemcpyDeviceToDevice, c->stream));
        if (weights)
            GX_CUDA(cudaMemcpyAsync(weights, c->weights, (size_t)n_tok * L.U * 4, cudaMemcpyDeviceToDevice, c->stream));
    }
    return record_ticket(c, out_ticket);
}

GX_API gx_result gx_ffn_block(gx_context *c, uint32_t layer, float *res, uint32_t n_tok, float *mixed,
                              uint64_t *out_ticket) {
    gx_result r = check_forward(c, layer, GX_F32, n_tok, GX_F32);
    if (r != GX_OK) return r;
    const Layer &L = c->layers[layer];
    if (!L.hc_wt) return GX_E_STATE;
    if (n_tok > 0 && (!res || ((uintptr_t)res & 15) || ((uintptr_t)mixed & 3))) return GX_E_INVALIDARG;
    GX_CUDA(cudaSetDevice(c->device));
    if (c->world > 1) {  // every rank takes part in the layer's exchange, also with no tokens
        r = ep_sync_ntok(c, n_tok);
        if (r != GX_OK) return r;
    } else if (n_tok == 0) {
        return record_ticket(c, out_ticket);
    }
    const gx::HcArgs a = hc_args(c, L, res, n_tok);
    if (n_tok > 0) {
        r = enqueue_hc_mix(c, L, a);
        if (r != GX_OK) return r;
        if (mixed)
            GX_CUDA(cudaMemcpyAsync(mixed, c->hc.cur, (size_t)n_tok * L.E * sizeof(float), cudaMemcpyDeviceToDevice,
                                    c->stream));
    }
    r = enqueue_layer(c, L, c->hc.cur, GX_F32, n_tok, nullptr, GX_F32, c->hc.y, GX_F32, -1, 0.f, false);
    if (r != GX_OK) return r;
    if (n_tok > 0) GX_CUDA(gx::launch_hc_combine(a, c->hc.y, c->stream, false));
    return record_ticket(c, out_ticket);
}

GX_API gx_result gx_moe_forward_host(gx_context *c, uint32_t layer, const void *x, uint32_t x_dtype, uint32_t n_tok,
                                     void *y, uint32_t y_dtype, uint32_t *ids, float *weights, uint32_t timeout_ms) {
    gx_result r = check_forward(c, layer, x_dtype, n_tok, y_dtype);
    if (r != GX_OK) return r;
    if (n_tok == 0 && c->world == 1) return GX_OK;
    if (n_tok > 0 && (!x || !y)) return GX_E_INVALIDARG;
    GX_CUDA(cudaSetDevice(c->device));
    const Layer &L = c->layers[layer];
    const size_t in_b = (size_t)n_tok * L.E * dtype_size(x_dtype), out_b = (size_t)n_tok * L.E * dtype_size(y_dtype);
    if (in_b) {
        std::memcpy(c->h_in, x, in_b);
        GX_CUDA(cudaMemcpyAsync(c->x_stage, c->h_in, in_b, cudaMemcpyHostToDevice, c->stream));
    }
    if (c->world > 1) {
        r = ep_sync_ntok(c, n_tok);
        if (r != GX_OK) return r;
    }
    const bool prof = (c->flags & GX_FLAG_PROFILE) != 0;
    if (prof) {
        c->prof_layers = 1;
        c->prof_stack = 0;
    }
    r = enqueue_layer(c, L, c->x_stage, x_dtype, n_tok, nullptr, GX_F32, c->y_stage, y_dtype, prof ? 0 : -1, 0.f,
                      false);
    if (r != GX_OK) return r;
    uint8_t *ho = static_cast<uint8_t *>(c->h_out);
    const size_t sel_b = (size_t)n_tok * L.U * 4;
    if (out_b) GX_CUDA(cudaMemcpyAsync(ho, c->y_stage, out_b, cudaMemcpyDeviceToHost, c->stream));
    if (ids) GX_CUDA(cudaMemcpyAsync(ho + c->stage_bytes, c->ids, sel_b, cudaMemcpyDeviceToHost, c->stream));
    if (weights) GX_CUDA(cudaMemcpyAsync(ho + c->stage_bytes + sel_b, c->weights, sel_b, cudaMemcpyDeviceToHost, c->stream));
    r = sync_all(c, timeout_ms);
    if (r != GX_OK) return r;
    if (out_b) std::memcpy(y, ho, out_b);
    if (ids && sel_b) std::memcpy(ids, ho + c->stage_bytes, sel_b);
    if (weights && sel_b) std::memcpy(weights, ho + c->stage_bytes + sel_b, sel_b);
    return GX_OK;
}

GX_API gx_result gx_stack_forward(gx_context *c, uint32_t first, uint32_t n_layers, const void *x, uint32_t x_dtype,
                                  uint32_t n_tok, void *y, uint32_t y_dtype, uint64_t *out_ticket) {
    if (!c || n_layers == 0 || (uint64_t)first + n_layers > c->layers.size()) return GX_E_INVALIDARG;
    for (uint32_t i = 0; i < n_layers; ++i) {
        gx_result r = check_forward(c, first + i, x_dtype, n_tok, y_dtype);
        if (r != GX_OK) return r;
        if (c->layers[first + i].E != c->layers[first].E) return GX_E_INVALIDARG;
    }
    if (n_tok == 0 && c->world == 1) return record_ticket(c, out_ticket);
    if (n_tok > 0 && (!x || !y || ((uintptr_t)y & 3))) return GX_E_INVALIDARG;
    GX_CUDA(cudaSetDevice(c->device));
    const size_t E = c->layers[first].E;
    const size_t in_b = n_tok * E * dtype_size(x_dtype), out_b = n_tok * E * dtype_size(y_dtype);
    if (stack_kernel_fits(c, first, n_layers, n_tok)) {
        // One launch for the whole stack; the input is staged if it aliases the output or the
        // kernel's layer buffers, or is not 16-byte aligned (the kernel reads it with vector loads).
        const void *src = x;
        if (x == y || x == c->xbuf[0] || x == c->xbuf[1] || ((uintptr_t)x & 15)) {
            GX_CUDA(cudaMemcpyAsync(c->x_stage, x, in_b, cudaMemcpyDeviceToDevice, c->stream));
            src = c->x_stage;
        }
        gx_result r = enqueue_stack_kernel(c, first, n_layers, src, x_dtype, n_tok, y, y_dtype);
        if (r != GX_OK) return r;
        return record_ticket(c, out_ticket);
    }
    if (c->world > 1) {
        // One token-count exchange per call, then the layers queue without host round trips.
        gx_result rs = ep_sync_ntok(c, n_tok);
        if (rs != GX_OK) return rs;
        if (in_b) GX_CUDA(cudaMemcpyAsync(c->x_stage, x, in_b, cudaMemcpyDeviceToDevice, c->stream));
        gx_result r = stack_enqueue(c, first, n_layers, c->x_stage, x_dtype, n_tok, c->y_stage, y_dtype);
        if (r != GX_OK) return r;
        if (out_b) GX_CUDA(cudaMemcpyAsync(y, c->y_stage, out_b, cudaMemcpyDeviceToDevice, c->stream));
        return record_ticket(c, out_ticket);
    }
    // The graph reads x_stage and writes y_stage; the caller's buffers are copied around it.
    GX_CUDA(cudaMemcpyAsync(c->x_stage, x, in_b, cudaMemcpyDeviceToDevice, c->stream));
    const GraphKey key{first, n_layers, n_tok, x_dtype, y_dtype, c->flags};
    auto it = c->graphs.find(key);
    if (it == c->graphs.end()) {
        // First call runs eagerly (sets kernel attributes), then the chain is captured.
        gx_result r = stack_enqueue(c, first, n_layers, c->x_stage, x_dtype, n_tok, c->y_stage, y_dtype);
        if (r != GX_OK) return r;
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ge = nullptr;
        GX_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        r = stack_enqueue(c, first, n_layers, c->x_stage, x_dtype, n_tok, c->y_stage, y_dtype);
        cudaError_t e = cudaStreamEndCapture(c->stream, &g);
        if (r != GX_OK) {
            if (g) cudaGraphDestroy(g);
            return r;
        }
        GX_CUDA(e);
        e = cudaGraphInstantiate(&ge, g, 0);
        if (e != cudaSuccess) {
            cudaGraphDestroy(g);
            return fail_cuda(c, e);
        }
        c->graphs[key] = {g, ge};
    } else {
        GX_CUDA(cudaGraphLaunch(it->second.second, c->stream));
    }
    GX_CUDA(cudaMemcpyAsync(y, c->y_stage, out_b, cudaMemcpyDeviceToDevice, c->stream));
    return record_ticket(c, out_ticket);
}

GX_API gx_result gx_stack_forward_host(gx_context *c, uint32_t first, uint32_t n_layers, const void *x,
                                       uint32_t x_dtype, uint32_t n_tok, void *y, uint32_t y_dtype,
                                       uint32_t timeout_ms) {
    if (!c || n_layers == 0 || (uint64_t)first + n_layers > c->layers.size()) return GX_E_INVALIDARG;
    if (n_tok == 0 && c->world == 1) return GX_OK;
    if ((n_tok > 0 && (!x || !y)) || n_tok > c->max_tokens) return GX_E_INVALIDARG;
    if (!c->layers[first].ready) return GX_E_STATE;
    const size_t E = c->layers[first].E;
    const size_t in_b = n_tok * E * dtype_size(x_dtype), out_b = n_tok * E * dtype_size(y_dtype);
    GX_CUDA(cudaSetDevice(c->device));
    if (in_b) {
        std::memcpy(c->h_in, x, in_b);
        GX_CUDA(cudaMemcpyAsync(c->xbuf[0], c->h_in, in_b, cudaMemcpyHostToDevice, c->stream));
    }
    // xbuf[0] holds the input only until the stack's staging copy has read it.
    gx_result r = gx_stack_forward(c, first, n_layers, c->xbuf[0], x_dtype, n_tok, c->y_stage, y_dtype, nullptr);
    if (r != GX_OK) return r;
    if (out_b) GX_CUDA(cudaMemcpyAsync(c->h_out, c->y_stage, out_b, cudaMemcpyDeviceToHost, c->stream));
    r = sync_all(c, timeout_ms);
    if (r != GX_OK) return r;
    if (out_b) std::memcpy(y, c->h_out, out_b);
    return GX_OK;
}

GX_API gx_result gx_wait(gx_context *c, uint64_t ticket, uint32_t timeout_ms) {
    if (!c) return GX_E_INVALIDARG;
    if (ticket > c->submitted) return GX_E_INVALIDARG;
    if (ticket == 0) return GX_OK;
    GX_CUDA(cudaSetDevice(c->device));
    return wait_event(c, c->events[ticket % kEvents], timeout_ms);
}

GX_API gx_result gx_poll(gx_context *c, uint64_t *out_completed) {
    if (!c || !out_completed) return GX_E_INVALIDARG;
    uint64_t done = c->submitted > kEvents ? c->submitted - kEvents : 0;
    for (uint64_t t = c->submitted; t > done; --t) {
        cudaError_t q = cudaEventQuery(c->events[t % kEvents]);
        if (q == cudaSuccess) {
            done = t;
            break;
        }
        if (q != cudaErrorNotReady) return fail_cuda(c, q);
    }
    *out_completed = done;
    return GX_OK;
}

GX_API gx_result gx_get_stream(gx_context *c, void **out_stream) {
    if (!c || !out_stream) return GX_E_INVALIDARG;
    *out_stream = c->stream;
    return GX_OK;
}

GX_API gx_result gx_decode_blocks(gx_context *c, uint32_t type_id, const void *packed, uint64_t packed_bytes,
                                  float *out, uint32_t value_count, const float *expected, float *max_abs_error,
                                  uint32_t timeout_ms) {
    // Argument rules of gd_validate_gyro (native/gyro_native.cpp:597-607).
    if (!c || !packed || !out || !known_type(type_id) || value_count == 0 || value_count % 128 ||
        value_count > 16777216u)
        return GX_E_INVALIDARG;
    const uint32_t blocks = value_count / 128;
    if (packed_bytes != (uint64_t)blocks * gx::type_block_bytes(type_id)) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    GX_CUDA(cudaSetDevice(c->device));
    uint8_t *din = nullptr;
    float *dout = nullptr;
    GX_CUDA(cudaMalloc(&din, packed_bytes));
    cudaError_t e = cudaMalloc(&dout, (size_t)value_count * 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(din, packed, packed_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = gx::launch_decode_blocks(type_id, din, blocks, reinterpret_cast<const uint16_t *>(c->codebook), dout, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, (size_t)value_count * 4, cudaMemcpyDeviceToHost, c->stream);
    gx_result r = e == cudaSuccess ? sync_all(c, timeout_ms) : fail_cuda(c, e);
    if (r != GX_E_TIMEOUT) {
        cudaFree(din);
        cudaFree(dout);
    }
    if (r != GX_OK) return r;
    if (expected) {
        float worst = 0.f;
        bool same = true;
        for (uint32_t i = 0; i < value_count; ++i) {
            uint32_t a, b;
            std::memcpy(&a, &out[i], 4);
            std::memcpy(&b, &expected[i], 4);
            if (a != b) {
                same = false;
                const float diff = out[i] > expected[i] ? out[i] - expected[i] : expected[i] - out[i];
                if (!(diff <= worst)) worst = diff;
            }
        }
        if (max_abs_error) *max_abs_error = worst;
        if (!same) return GX_E_MISMATCH;
    } else if (max_abs_error) {
        *max_abs_error = 0.f;
    }
    return GX_OK;
}

GX_API gx_result gx_upload_matrix(gx_context *c, uint32_t type_id, uint32_t rows, uint32_t cols, const void *packed,
                                  uint64_t packed_bytes, uint32_t *out_handle, uint32_t timeout_ms) {
    if (!c || !packed || !out_handle || !known_type(type_id) || rows == 0 || rows % 8 || cols == 0 || cols % 128 ||
        cols > 2048)
        return GX_E_INVALIDARG;
    const uint64_t row_bytes = (uint64_t)cols / 128 * gx::type_block_bytes(type_id);
    if (packed_bytes != row_bytes * rows) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    GX_CUDA(cudaSetDevice(c->device));
    // the GEMV takes rows 16 at a time: an odd count of 8-row groups gets a zero group after it
    const uint64_t pad = rows % 16 ? (uint64_t)gx::tile_bytes(type_id) * (cols / 128) : 0;
    uint8_t *raw = nullptr, *tiles = nullptr;
    GX_CUDA(cudaMalloc(&tiles, packed_bytes + pad));
    cudaError_t e = cudaMalloc(&raw, packed_bytes);
    if (e == cudaSuccess && pad) e = cudaMemsetAsync(tiles + packed_bytes, 0, pad, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(raw, packed, packed_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = gx::launch_repack(type_id, raw, row_bytes, rows, cols, tiles, c->stream);
    gx_result r = e == cudaSuccess ? sync_all(c, timeout_ms) : fail_cuda(c, e);
    if (r != GX_E_TIMEOUT) cudaFree(raw);
    if (r != GX_OK) {
        if (r != GX_E_TIMEOUT) cudaFree(tiles);
        return r;
    }
    Matrix m;
    m.type = type_id;
    m.rows = rows;
    m.cols = cols;
    m.tiles = tiles;
    c->mats.push_back(m);
    *out_handle = (uint32_t)(c->mats.size() - 1);
    return GX_OK;
}

GX_API gx_result gx_matvec(gx_context *c, uint32_t handle, const float *x, uint32_t n_tok, float *y,
                           uint64_t *out_ticket) {
    if (!c || handle >= c->mats.size() || (n_tok && (!x || !y)) || n_tok > 64) return GX_E_INVALIDARG;
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 3)) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    GX_CUDA(cudaSetDevice(c->device));
    if (n_tok) {
        const Matrix &m = c->mats[handle];
        gx::MatvecArgs a{};
        a.type = m.type;
        a.tiles = m.tiles;
        a.x = x;
        a.y = y;
        a.codebook = c->codebook;
        a.rows = (int)m.rows;
        a.cols = (int)m.cols;
        a.n_tok = (int)n_tok;
        a.err = c->err;
        GX_CUDA(gx::launch_matvec(a, c->sm_count, c->stream));
    }
    return record_ticket(c, out_ticket);
}

GX_API gx_result gx_read_timings(gx_context *c, gx_timings *t) {
    if (!c || !t) return GX_E_INVALIDARG;
    std::memset(t, 0, sizeof(*t));
    if (!(c->flags & GX_FLAG_PROFILE)) return GX_OK;
    if (c->prof_stack > 0) {  // one stack kernel: only its total is known
        float ms = 0.f;
        GX_CUDA(cudaEventSynchronize(c->prof[3]));
        GX_CUDA(cudaEventElapsedTime(&ms, c->prof[0], c->prof[3]));
        t->total_ns = (uint64_t)(ms * 1e6);
        t->layers = c->prof_stack;
        return GX_OK;
    }
    if (c->prof_layers == 0) return GX_OK;
    GX_CUDA(cudaEventSynchronize(c->prof[4 * (size_t)(c->prof_layers - 1) + 3]));
    for (uint32_t l = 0; l < c->prof_layers; ++l) {
        const cudaEvent_t *ev = &c->prof[4 * (size_t)l];
        float ms[3] = {0.f, 0.f, 0.f};
        for (int k = 0; k < 3; ++k) GX_CUDA(cudaEventElapsedTime(&ms[k], ev[k], ev[k + 1]));
        t->router_ns += (uint64_t)(ms[0] * 1e6);
        t->gate_up_ns += (uint64_t)(ms[1] * 1e6);
        t->down_ns += (uint64_t)(ms[2] * 1e6);
    }
    t->experts_ns = t->gate_up_ns + t->down_ns;
    t->total_ns = t->router_ns + t->experts_ns;
    t->layers = c->prof_layers;
    return GX_OK;
}

GX_API gx_result gx_set_flags(gx_context *c, uint32_t flags) {
    if (!c || (flags & ~(uint32_t)GX_FLAG_PROFILE)) return GX_E_INVALIDARG;
    c->flags = flags;
    c->prof_layers = 0;
    c->prof_stack = 0;
    return GX_OK;
}

GX_API gx_result gx_destroy(gx_context *c, uint32_t timeout_ms) {
    if (!c) return GX_E_INVALIDARG;
    if (!c->broken) {
        cudaSetDevice(c->device);
        gx_result r = sync_all(c, timeout_ms);
        if (r == GX_E_TIMEOUT) return r;
    }
    release_all(c);
    delete c;
    return GX_OK;
}

}  // extern "C"

// ---- gx_moe_forward_noalloc: decode layer on library-owned static scratch -----------------
// Some hosts may not allocate device memory once they start stepping: serving hosts that give
// all free HBM to their own pools at start-up (so a later cudaMalloc fails), and step loops that
// must not stall the device (cudaMalloc and cudaFree synchronise it). gx_moe_forward can
// allocate on a call (the tensor-core path sizes its buffers on first use), so this entry point
// runs the decode kernels on a fixed array that is part of the library image instead.
namespace {

constexpr uint32_t kNoAllocMaxTokens = GX_NOALLOC_MAX_TOKENS;
constexpr uint64_t na_align(uint64_t v) { return (v + 255) & ~uint64_t(255); }
// Per-token scratch at the ABI's largest accepted layer: 512 router logits, U*F <= 64*128
// activations; selections for U <= 16; one norm and one input scale.
constexpr size_t kNaLogits = 0;
constexpr size_t kNaSs = kNaLogits + na_align((uint64_t)kNoAllocMaxTokens * 512 * 4);
constexpr size_t kNaXscale = kNaSs + na_align((uint64_t)kNoAllocMaxTokens * 4);
constexpr size_t kNaIds = kNaXscale + na_align((uint64_t)kNoAllocMaxTokens * 4);
constexpr size_t kNaWeights = kNaIds + na_align((uint64_t)kNoAllocMaxTokens * 16 * 4);
constexpr size_t kNaAct = kNaWeights + na_align((uint64_t)kNoAllocMaxTokens * 16 * 4);
constexpr size_t kNaBytes = kNaAct + na_align((uint64_t)kNoAllocMaxTokens * 64 * 128 * 4);
static_assert(kNaBytes == GX_NOALLOC_SCRATCH_BYTES, "header limit out of date");

// The scratch: one array per device, shared by every context and every call on that device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNaBytes];

constexpr int kNaMaxDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_base[kNaMaxDevices] = {};

// Device address of the array on the current device (c->device), looked up on the first call
// for that device. The lookup loads the library's device code on that device if it is not
// loaded yet, which is why the first call should come before any stream capture.
gx_result noalloc_scratch(gx_context *c, uint8_t **out) {
    if (c->device < 0 || c->device >= kNaMaxDevices) return GX_E_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_base[c->device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return fail_cuda_at(c, e, "cudaGetSymbolAddress(g_noalloc_scratch)", __LINE__);
        g_noalloc_base[c->device] = static_cast<uint8_t *>(p);
    }
    *out = g_noalloc_base[c->device];
    return GX_OK;
}

}  // namespace

extern "C" {

GX_API gx_result gx_moe_forward_noalloc(gx_context *c, uint32_t layer, const void *x, uint32_t x_dtype,
                                        uint32_t n_tok, void *y, uint32_t y_dtype, uint32_t *ids, float *weights,
                                        uint64_t *out_ticket) {
    if (!c) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (c->world > 1) return GX_E_UNSUPPORTED;  // the decode kernels need every expert on this device
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    if ((x_dtype != GX_F32 && x_dtype != GX_BF16) || (y_dtype != GX_F32 && y_dtype != GX_BF16)) return GX_E_INVALIDARG;
    if (n_tok > kNoAllocMaxTokens) {
        if (debug_enabled())
            std::fprintf(stderr, "gyro_moe: gx_moe_forward_noalloc: n_tok %u exceeds the static scratch limit of %u\n",
                         n_tok, kNoAllocMaxTokens);
        return GX_E_INVALIDARG;
    }
    if (n_tok > 0 && (!x || !y)) return GX_E_INVALIDARG;
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 3) || ((uintptr_t)ids & 3) || ((uintptr_t)weights & 3))
        return GX_E_INVALIDARG;
    const Layer &L = c->layers[layer];
    if (L.n_expert > 512 || L.U > 16 || (uint64_t)L.U * L.F > 64 * 128) return GX_E_INVALIDARG;
    if (L.sh_wt) return GX_E_UNSUPPORTED;  // its scratch holds no shared-expert buffers
    GX_CUDA(cudaSetDevice(c->device));
    uint8_t *base = nullptr;
    gx_result r = noalloc_scratch(c, &base);
    if (r != GX_OK) return r;
    if (n_tok == 0) return record_ticket(c, out_ticket);

    // Every scratch word a kernel reads is written earlier in the same call (logits by the
    // router, selections by the top-k step, activations by gate/up), so nothing is cleared.
    // For up to kRouterSelectTok tokens the router's arrival count is the context's own
    // counter (allocated by gx_create, zero between launches), not a word of this array.
    float *logits = reinterpret_cast<float *>(base + kNaLogits);
    float *ss = reinterpret_cast<float *>(base + kNaSs);
    float *xscale = reinterpret_cast<float *>(base + kNaXscale);
    uint32_t *sel_ids = reinterpret_cast<uint32_t *>(base + kNaIds);
    float *sel_w = reinterpret_cast<float *>(base + kNaWeights);
    float *act = reinterpret_cast<float *>(base + kNaAct);

    gx::RouterArgs ra{};
    ra.W = L.router;
    ra.bias = L.bias;
    ra.x = x;
    ra.x_bf16 = x_dtype == GX_BF16;
    ra.n_tok = (int)n_tok;
    ra.NE = (int)L.n_expert;
    ra.E = (int)L.E;
    ra.U = (int)L.U;
    ra.scale = L.scale;
    ra.norm_eps = 0.f;
    ra.ss = ss;
    ra.logit_splits = 1;
    ra.xscale = xscale;
    ra.logits = logits;
    ra.ids = sel_ids;
    ra.weights = sel_w;
    ra.err = c->err;
    const bool sel_router = n_tok <= (uint32_t)gx::kRouterSelectTok;
    ra.done = sel_router ? c->router_done : nullptr;
    const bool fused = !sel_router && gx::gate_up_fuses_topk((int)L.E, (int)L.F, (int)L.U, (int)n_tok, c->sm_count);
    GX_CUDA(gx::launch_router(ra, c->stream, false, !fused && !sel_router));

    gx::GateUpArgs ga{};
    ga.type = L.type;
    ga.gate = L.gate;
    ga.up = L.up;
    ga.expert_bytes = L.gate_expert_bytes;
    ga.x = x;
    ga.x_bf16 = x_dtype == GX_BF16;
    ga.signs = L.gate_signs;
    ga.xscale = nullptr;
    ga.ids = sel_ids;
    ga.fused_topk = fused;
    ga.logits = logits;
    ga.bias = L.bias;
    ga.ss = ss;
    ga.NE = (int)L.n_expert;
    ga.norm_eps = 0.f;
    ga.wscale = L.scale;
    ga.ids_out = sel_ids;
    ga.weights_out = sel_w;
    ga.act = act;
    ga.codebook = c->codebook;
    ga.codebook_image = c->codebook_image;
    ga.E = (int)L.E;
    ga.F = (int)L.F;
    ga.U = (int)L.U;
    ga.n_slots = (int)(n_tok * L.U);
    ga.n_expert = (int)L.local_experts;
    ga.err = c->err;
    GX_CUDA(gx::launch_gate_up(ga, c->sm_count, c->stream, true));

    gx::DownArgs da{};
    da.type = L.type;
    da.down = L.down;
    da.expert_bytes = L.down_expert_bytes;
    da.act = act;
    da.signs = L.down_signs;
    da.ids = sel_ids;
    da.weights = sel_w;
    da.resid = nullptr;
    da.resid_bf16 = 0;
    da.out = y;
    da.out_bf16 = y_dtype == GX_BF16;
    da.codebook = c->codebook;
    da.codebook_image = c->codebook_image;
    da.E = (int)L.E;
    da.F = (int)L.F;
    da.U = (int)L.U;
    da.n_tok = (int)n_tok;
    da.n_expert = (int)L.local_experts;
    da.err = c->err;
    GX_CUDA(gx::launch_down(da, c->sm_count, c->stream, true));

    const size_t sel_b = (size_t)n_tok * L.U * 4;
    if (ids) GX_CUDA(cudaMemcpyAsync(ids, sel_ids, sel_b, cudaMemcpyDeviceToDevice, c->stream));
    if (weights) GX_CUDA(cudaMemcpyAsync(weights, sel_w, sel_b, cudaMemcpyDeviceToDevice, c->stream));
    return record_ticket(c, out_ticket);
}

}  // extern "C"

// ---- expert parallelism: usage counts and replicas of hot experts -------------------------
extern "C" {

GX_API gx_result gx_read_expert_counts(gx_context *c, uint32_t layer, uint32_t *counts, uint32_t reset,
                                       uint32_t timeout_ms) {
    if (!c || !counts) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    const Layer &L = c->layers[layer];
    if (!L.expert_count) return GX_E_UNSUPPORTED;
    GX_CUDA(cudaSetDevice(c->device));
    GX_CUDA(cudaMemcpyAsync(c->h_out, L.expert_count, L.n_expert * sizeof(unsigned), cudaMemcpyDeviceToHost,
                            c->stream));
    if (reset) GX_CUDA(cudaMemsetAsync(L.expert_count, 0, L.n_expert * sizeof(unsigned), c->stream));
    gx_result r = sync_all(c, timeout_ms);
    if (r != GX_OK) return r;
    std::memcpy(counts, c->h_out, L.n_expert * sizeof(unsigned));
    return GX_OK;
}

GX_API gx_result gx_replicate_experts(gx_context *c, uint32_t layer, const uint32_t *experts, uint32_t n,
                                      uint32_t timeout_ms) {
    if (!c || (n && !experts)) return GX_E_INVALIDARG;
    if (c->broken) return GX_E_DEVICE;
    if (layer >= c->layers.size() || !c->layers[layer].ready) return GX_E_STATE;
    Layer &L = c->layers[layer];
    if (!L.route) return GX_E_UNSUPPORTED;
    if (n > L.replica_slots) return GX_E_INVALIDARG;
    std::vector<char> seen(L.n_expert, 0);
    for (uint32_t i = 0; i < n; ++i) {
        if (experts[i] >= L.n_expert || seen[experts[i]]) return GX_E_INVALIDARG;
        seen[experts[i]] = 1;
    }
    GX_CUDA(cudaSetDevice(c->device));
    const uint32_t NEl = L.local_experts;
    // every rank's replica slot i receives expert experts[i] from the rank whose shard holds it
    const uint64_t dn_bytes = L.down_expert_bytes, gu_bytes = L.gate_expert_bytes;
    c->nccl->GroupStart();
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t e = experts[i], owner = e / NEl, k = e % NEl;
        uint8_t *bases[3] = {L.gate, L.up, L.down};
        const uint64_t bytes[3] = {gu_bytes, gu_bytes, dn_bytes};
        for (int p = 0; p < 3; ++p) {
            const uint8_t *src = bases[p] + (uint64_t)k * bytes[p];
            uint8_t *dst = bases[p] + (uint64_t)(NEl + i) * bytes[p];
            c->nccl->Broadcast(src, dst, bytes[p], ncclUint8, (int)owner, c->comm, c->stream);
        }
    }
    gx_result r = comm_group_end(c, "expert replication");
    if (r != GX_OK) return r;
    std::vector<int2> route(L.n_expert);
    for (uint32_t x = 0; x < L.n_expert; ++x) route[x] = make_int2((int)(x / NEl), (int)(x % NEl));
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t e = experts[i], owner = e / NEl;
        route[e] = make_int2(-1, owner == c->rank ? (int)(e % NEl) : (int)(NEl + i));
    }
    GX_CUDA(cudaMemcpyAsync(L.route, route.data(), route.size() * sizeof(int2), cudaMemcpyHostToDevice, c->stream));
    r = sync_all(c, timeout_ms);
    if (r != GX_OK) return r;
    L.replicas.assign(experts, experts + n);
    return GX_OK;
}

}  // extern "C"

