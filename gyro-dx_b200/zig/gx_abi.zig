//! Extern mirror of include/gyro_moe.h for the Zig host of gyro-dx, in the style of
//! src/native_abi.zig:1-95 (explicit extern structs and functions, comptime layout asserts).
//! It replaces native_abi.zig's gd_* declarations for the routed-expert path.
//! No Zig toolchain exists on the build machines, so this file is written against the C header
//! and checked only by the C/ctypes layout tests (tests/test_abi.py); it is not compiled here.
pub const gx_context = opaque {};
pub const gx_result = i32;

pub const ok: gx_result = 0;
pub const e_invalidarg: gx_result = -1;
pub const e_outofmemory: gx_result = -2;
pub const e_timeout: gx_result = -3;
pub const e_device: gx_result = -4;
pub const e_unsupported: gx_result = -5;
pub const e_state: gx_result = -6;
pub const e_mismatch: gx_result = -7;
pub const e_comm: gx_result = -8;
pub const e_kernel: gx_result = -9;
pub const e_range: gx_result = -10;

pub const dtype_f32: u32 = 0;
pub const dtype_q8_0: u32 = 8;
pub const dtype_bf16: u32 = 30;
pub const flag_profile: u32 = 1;
pub const ep_none: u32 = 0;
pub const ep_nccl: u32 = 1;
pub const ep_peer: u32 = 2;

pub const gx_options = extern struct {
    device: u32,
    rank: u32,
    world: u32,
    max_tokens: u32,
    max_layers: u32,
    flags: u32,
    codebook: ?*const anyopaque,
    codebook_bytes: u64,
    nccl_id: [128]u8,
};

pub const gx_caps = extern struct {
    abi_version: u32,
    sm_count: u32,
    cc_major: u32,
    cc_minor: u32,
    rank: u32,
    world: u32,
    max_tokens: u32,
    max_layers: u32,
    hbm_bytes: u64,
    free_bytes: u64,
    l2_bytes: u64,
    arena_bytes: u64,
    device_name: [120]u8,
    ep_exchange: u32,
    ep_peer_layers: u32,
};

pub const gx_layer_desc = extern struct {
    type_id: u32,
    n_expert: u32,
    n_embd: u32,
    n_ff: u32,
    n_used: u32,
    expert_weights_scale: f32,
    gate: ?*const anyopaque,
    up: ?*const anyopaque,
    down: ?*const anyopaque,
    gate_bytes: u64,
    up_bytes: u64,
    down_bytes: u64,
    router: ?[*]const f32,
    gate_signs: ?[*]const f32,
    up_signs: ?[*]const f32,
    down_signs: ?[*]const f32,
    router_bias: ?[*]const f32,
};

pub const gx_shared_desc = extern struct {
    type_id: u32,
    n_ff: u32,
    gate: ?*const anyopaque,
    up: ?*const anyopaque,
    down: ?*const anyopaque,
    gate_bytes: u64,
    up_bytes: u64,
    down_bytes: u64,
    gate_inp: ?[*]const f32,
};

pub const shared_none: u32 = 0xffffffff;

pub const gx_hc_desc = extern struct {
    n_streams: u32,
    rank: u32,
    type_id: u32,
    eps: f32,
    norm: ?[*]const f32,
    down: ?*const anyopaque,
    up: ?*const anyopaque,
    inject: ?*const anyopaque,
    down_bytes: u64,
    up_bytes: u64,
    inject_bytes: u64,
};

pub const gx_gguf_layer_info = extern struct {
    type_id: u32,
    n_expert: u32,
    n_embd: u32,
    n_ff: u32,
    n_used: u32,
    expert_weights_scale: f32,
    shared_type: u32,
    shared_ff: u32,
    rotated: u32,
    reserved: u32,
};

pub const gx_timings = extern struct {
    router_ns: u64,
    gate_up_ns: u64,
    down_ns: u64,
    experts_ns: u64,
    total_ns: u64,
    layers: u64,
};

pub extern fn gx_create(options: *const gx_options, context: *?*gx_context) gx_result;
pub extern fn gx_get_caps(context: *gx_context, caps: *gx_caps) gx_result;
pub extern fn gx_upload_layer(context: *gx_context, layer: u32, desc: *const gx_layer_desc, timeout_ms: u32) gx_result;
pub extern fn gx_upload_shared(context: *gx_context, layer: u32, desc: ?*const gx_shared_desc, timeout_ms: u32) gx_result;
pub extern fn gx_upload_hc(context: *gx_context, layer: u32, desc: ?*const gx_hc_desc, timeout_ms: u32) gx_result;
pub extern fn gx_ffn_block(context: *gx_context, layer: u32, res: ?[*]f32, n_tok: u32, mixed: ?[*]f32,
    ticket: ?*u64) gx_result;
pub extern fn gx_gguf_inspect_layer(path: [*:0]const u8, gguf_layer: u32, info: *gx_gguf_layer_info) gx_result;
pub extern fn gx_upload_layer_gguf(context: *gx_context, layer: u32, path: [*:0]const u8, gguf_layer: u32,
    timeout_ms: u32) gx_result;
pub extern fn gx_moe_forward(context: *gx_context, layer: u32, x: ?*const anyopaque, x_dtype: u32, n_tok: u32,
    y: ?*anyopaque, y_dtype: u32, ids: ?[*]u32, weights: ?[*]f32, ticket: ?*u64) gx_result;
pub extern fn gx_moe_forward_host(context: *gx_context, layer: u32, x: ?*const anyopaque, x_dtype: u32, n_tok: u32,
    y: ?*anyopaque, y_dtype: u32, ids: ?[*]u32, weights: ?[*]f32, timeout_ms: u32) gx_result;
pub extern fn gx_stack_forward(context: *gx_context, first_layer: u32, n_layers: u32, x: ?*const anyopaque,
    x_dtype: u32, n_tok: u32, y: ?*anyopaque, y_dtype: u32, ticket: ?*u64) gx_result;
pub extern fn gx_stack_forward_host(context: *gx_context, first_layer: u32, n_layers: u32, x: ?*const anyopaque,
    x_dtype: u32, n_tok: u32, y: ?*anyopaque, y_dtype: u32, timeout_ms: u32) gx_result;
pub extern fn gx_wait(context: *gx_context, ticket: u64, timeout_ms: u32) gx_result;
pub extern fn gx_poll(context: *gx_context, completed: *u64) gx_result;
pub extern fn gx_get_stream(context: *gx_context, stream: *?*anyopaque) gx_result;
pub extern fn gx_decode_blocks(context: *gx_context, type_id: u32, packed: [*]const u8, packed_bytes: u64,
    out: [*]f32, value_count: u32, expected: ?[*]const f32, max_abs_error: ?*f32, timeout_ms: u32) gx_result;
pub extern fn gx_upload_matrix(context: *gx_context, type_id: u32, rows: u32, cols: u32, packed: [*]const u8,
    packed_bytes: u64, handle: *u32, timeout_ms: u32) gx_result;
pub extern fn gx_matvec(context: *gx_context, handle: u32, x: [*]const f32, n_tok: u32, y: [*]f32,
    ticket: ?*u64) gx_result;
pub extern fn gx_read_timings(context: *gx_context, timings: *gx_timings) gx_result;
pub extern fn gx_comm_unique_id(out_id: [*]u8, bytes: u64) gx_result;
pub extern fn gx_read_expert_counts(context: *gx_context, layer: u32, counts: [*]u32, reset: u32,
    timeout_ms: u32) gx_result;
pub extern fn gx_replicate_experts(context: *gx_context, layer: u32, experts: ?[*]const u32, n: u32,
    timeout_ms: u32) gx_result;
pub extern fn gx_moe_forward_noalloc(context: *gx_context, layer: u32, x: ?*const anyopaque, x_dtype: u32,
    n_tok: u32, y: ?*anyopaque, y_dtype: u32, ids: ?[*]u32, weights: ?[*]f32, ticket: ?*u64) gx_result;
pub extern fn gx_set_flags(context: *gx_context, flags: u32) gx_result;
pub extern fn gx_destroy(context: *gx_context, timeout_ms: u32) gx_result;

comptime {
    const assert = @import("std").debug.assert;
    assert(@sizeOf(gx_options) == 168);
    assert(@offsetOf(gx_options, "nccl_id") == 40);
    assert(@sizeOf(gx_caps) == 192);
    assert(@offsetOf(gx_caps, "device_name") == 64);
    assert(@offsetOf(gx_caps, "ep_exchange") == 184);
    assert(@sizeOf(gx_layer_desc) == 112);
    assert(@offsetOf(gx_layer_desc, "router") == 72);
    assert(@sizeOf(gx_timings) == 48);
    assert(@sizeOf(gx_shared_desc) == 64);
    assert(@offsetOf(gx_shared_desc, "gate_inp") == 56);
    assert(@sizeOf(gx_gguf_layer_info) == 40);
    assert(@sizeOf(gx_hc_desc) == 72);
    assert(@offsetOf(gx_hc_desc, "down_bytes") == 48);
}
