//! gpu.zig for libchannel_b200 -- a drop-in replacement of Channel's Vulkan GPU module
//! (src/gpu.zig and src/gpu/*.zig) over the C-ABI in include/channel_cuda.h.
//!
//! Copy this file over src/gpu.zig.  It keeps the names and signatures the rest of the
//! reference uses:
//!   gpu.context.GpuContext.init / deinit             (main.zig:114)
//!   gpu.model_gpu.GpuModelContext.init / deinit      (main.zig:119)
//!   gpu.model_dispatch.gpuDispatchForwardToken       (model/forward.zig:47)
//!   gpu.batch_dispatch.gpuDispatchPrefillBatch       (server/prefill.zig:90)
//!   GpuModelContext.batch_prefill_ctx.max_tokens     (server/prefill.zig:61-66)
//!   GpuModelContext.buf_x / buf_topk_ids / buf_topk_vals .asSlice(T)
//!                                                    (server/decode.zig:13, prefill.zig:92-93,
//!                                                     memory_inject.zig:56, server.zig:78-80)
//! src/model, src/kernels.zig, src/quant.zig, src/ring_buffer.zig, src/sampler.zig and
//! server_queue.zig stay unchanged.
//!
//! What differs from the Vulkan module, and why:
//!   * The reference maps its buffers into host memory (UMA).  Device memory of a B200 is
//!     not host-visible, so buf_x and the top-64 are host mirrors that every dispatch
//!     refreshes (a few KB per token); writes into them do not reach the device.
//!   * The KV caches are read and written through GpuModelContext.kvRead / kvWrite
//!     (ch_kv_read / ch_kv_write).  The four places that slice layers[l].buf_k_cache /
//!     buf_v_cache directly (memory.zig:106-107, model/memory_inject.zig:20-27,
//!     hippocampus.zig:168-169, snapshot.zig:97-98) call these instead.
//!   * Weights are quantized on the device (ch_model_create_bf16): Q4_0 for every
//!     projection (QuantMode .q4 / .mixed), Q8_0 for the tied LM head, exactly as
//!     quant.zig would (model_gpu.zig:44-55,109-127,157).
//!   * The quiescence gate (model_dispatch.zig:47-101, quiescence_thresh > 0) is not
//!     implemented: every layer runs, as the reference does with the gate off.
//!
//! Untested here: this build has no Zig toolchain.  Written against Zig 0.14
//! (docs/quick-start.md:28).
const std = @import("std");
const c = @cImport(@cInclude("channel_cuda.h"));
const tensor = @import("tensor.zig");
const model_types = @import("model/types.zig");
const model_mod = @import("model.zig");
pub const quant = @import("quant.zig");

pub const GpuError = error{ InvalidArgument, OutOfMemory, Cuda, Timeout, BatchTooLarge, GpuError, State, Device, Comm, Unsupported };

fn check(rc: c_int) GpuError!void {
    return switch (rc) {
        c.CH_OK => {},
        c.CH_EINVAL => error.InvalidArgument,
        c.CH_ENOMEM => error.OutOfMemory,
        c.CH_ETIMEOUT => error.Timeout,
        c.CH_EBATCH => error.BatchTooLarge, // batch_dispatch.zig:42
        c.CH_ESTATE => error.State,
        c.CH_EDEVICE => error.Device,
        c.CH_ECOMM => error.Comm,
        else => error.Cuda,
    };
}

fn logLastError(what: []const u8) void {
    std.log.err("{s}: {s}", .{ what, std.mem.span(c.ch_last_error()) });
}

/// A host array standing in for one of the reference's mapped buffers.
pub const HostView = struct {
    bytes: []align(16) u8 = &.{},

    pub fn init(allocator: std.mem.Allocator, n_bytes: usize) !HostView {
        const b = try allocator.alignedAlloc(u8, 16, n_bytes);
        @memset(b, 0);
        return .{ .bytes = b };
    }
    pub fn deinit(self: *HostView, allocator: std.mem.Allocator) void {
        if (self.bytes.len > 0) allocator.free(self.bytes);
        self.bytes = &.{};
    }
    pub fn asSlice(self: HostView, comptime T: type) []T {
        const p: [*]T = @ptrCast(@alignCast(self.bytes.ptr));
        return p[0 .. self.bytes.len / @sizeOf(T)];
    }
};

// ---------------------------------------------------------------------------------
// GpuContext (src/gpu/context.zig:17-109)
pub const context = struct {
    pub const GpuContext = struct {
        allocator: std.mem.Allocator,
        h: *c.ch_ctx,
        device_name: [256]u8,

        pub fn init(allocator: std.mem.Allocator) !GpuContext {
            var h: ?*c.ch_ctx = null;
            check(c.ch_ctx_create(0, &h)) catch |e| {
                logLastError("ch_ctx_create");
                return e;
            };
            var name = [_]u8{0} ** 256;
            const label = "NVIDIA B200 (libchannel_b200, sm_100a)";
            @memcpy(name[0..label.len], label);
            return .{ .allocator = allocator, .h = h.?, .device_name = name };
        }
        pub fn deinit(self: *GpuContext) void {
            c.ch_ctx_destroy(self.h);
        }
    };
};

// ---------------------------------------------------------------------------------
// BatchPrefillContext (src/gpu/batch_prefill.zig): the chunk limit the server splits by
pub const batch_prefill = struct {
    pub const BatchPrefillContext = struct {
        max_tokens: usize,
        buf_x: HostView = .{},
    };
};

// ---------------------------------------------------------------------------------
// GpuModelContext (src/gpu/model_gpu.zig:30-216)
pub const model_gpu = struct {
    pub const GpuModelContext = struct {
        allocator: std.mem.Allocator,
        ctx: *const context.GpuContext,
        h: *c.ch_model,
        hidden: usize,
        vocab: usize,
        kv_dim: usize,
        buf_x: HostView,
        buf_normed_x: HostView,
        buf_topk_ids: HostView,
        buf_topk_vals: HostView,
        batch_prefill_ctx: ?*batch_prefill.BatchPrefillContext,
        prefill_ctx_storage: *batch_prefill.BatchPrefillContext,
        list_active: []u32,
        list_sliding: []u32,

        pub fn init(allocator: std.mem.Allocator, ctx: *const context.GpuContext, m: *const model_mod.Model,
                    config: model_types.ModelConfig, mode: quant.QuantMode, quiescence_thresh: f32) !GpuModelContext {
            _ = quiescence_thresh; // every layer runs (the gate is off)
            if (mode != .q4 and mode != .mixed) return error.Unsupported; // this backend is the Q4 path
            const L = config.num_hidden_layers;
            if (L == 0 or L > 64 or m.layers.len != L) return error.InvalidArgument;
            const head_dim = m.layers[0].head_dim;
            for (m.layers) |l| if (l.head_dim != head_dim or l.num_kv_heads != m.layers[0].num_kv_heads) return error.Unsupported;

            var cfg = std.mem.zeroes(c.ch_model_config);
            cfg.vocab_size = @intCast(config.vocab_size);
            cfg.hidden_size = @intCast(config.hidden_size);
            cfg.intermediate_size = @intCast(config.intermediate_size);
            cfg.num_hidden_layers = @intCast(L);
            cfg.num_attention_heads = @intCast(config.num_attention_heads);
            cfg.num_key_value_heads = @intCast(m.layers[0].num_kv_heads);
            cfg.head_dim = @intCast(head_dim);
            cfg.rotary_dim = @intCast(m.layers[0].rotary_dim);
            cfg.rms_norm_eps = config.rms_norm_eps;
            cfg.rope_theta = config.rope_theta;
            cfg.rope_theta_full = config.rope_theta_full;
            cfg.sliding_window = @intCast(config.sliding_window);
            cfg.max_prefill_tokens = 1024; // BatchPrefillContext max_tokens (model_gpu.zig:178)
            for (m.layers, 0..) |l, i| cfg.layer_types[i] = if (l.layer_type == .full_attention) 1 else 0;

            const lw = try allocator.alloc(c.ch_layer_weights_bf16, L);
            defer allocator.free(lw);
            for (m.layers, 0..) |l, i| {
                lw[i] = std.mem.zeroes(c.ch_layer_weights_bf16);
                lw[i].q_proj = bf16Ptr(l.q_proj);
                lw[i].k_proj = bf16Ptr(l.k_proj);
                lw[i].v_proj = if (l.k_eq_v or l.v_proj.len == 0) null else bf16Ptr(l.v_proj); // NULL: k_proj
                lw[i].o_proj = bf16Ptr(l.o_proj);
                lw[i].gate_proj = bf16Ptr(l.gate_proj);
                lw[i].up_proj = bf16Ptr(l.up_proj);
                lw[i].down_proj = bf16Ptr(l.down_proj);
                lw[i].input_norm = normPtr(l.input_layernorm, config.hidden_size);
                lw[i].q_norm = normPtr(l.q_norm, l.head_dim);
                lw[i].k_norm = normPtr(l.k_norm, l.head_dim);
                lw[i].pre_ffn_norm = normPtr(l.pre_feedforward_layernorm, config.hidden_size);
                lw[i].post_attn_norm = if (l.post_attention_layernorm) |p| bf16Ptr(p) else null;
                lw[i].post_ffn_norm = if (l.post_feedforward_layernorm) |p| bf16Ptr(p) else null;
                lw[i].layer_scalar = l.layer_scalar orelse 1.0;
            }
            var h: ?*c.ch_model = null;
            check(c.ch_model_create_bf16(ctx.h, &cfg, lw.ptr, bf16Ptr(m.embed_tokens),
                normPtr(m.final_norm, config.hidden_size), &h)) catch |e| {
                logLastError("ch_model_create_bf16");
                return e;
            };
            errdefer c.ch_model_destroy(h.?);
            const bp = try allocator.create(batch_prefill.BatchPrefillContext);
            errdefer allocator.destroy(bp);
            bp.* = .{ .max_tokens = cfg.max_prefill_tokens };
            const H = config.hidden_size;
            return .{
                .allocator = allocator,
                .ctx = ctx,
                .h = h.?,
                .hidden = H,
                .vocab = config.vocab_size,
                .kv_dim = m.layers[0].kv_dim,
                .buf_x = try HostView.init(allocator, H * 4),
                .buf_normed_x = try HostView.init(allocator, H * 4),
                .buf_topk_ids = try HostView.init(allocator, 64 * 4),
                .buf_topk_vals = try HostView.init(allocator, 64 * 4),
                .batch_prefill_ctx = bp,
                .prefill_ctx_storage = bp,
                .list_active = try allocator.alloc(u32, 4096),
                .list_sliding = try allocator.alloc(u32, 4096),
            };
        }

        pub fn deinit(self: *GpuModelContext) void {
            c.ch_model_destroy(self.h);
            self.buf_x.deinit(self.allocator);
            self.buf_normed_x.deinit(self.allocator);
            self.buf_topk_ids.deinit(self.allocator);
            self.buf_topk_vals.deinit(self.allocator);
            self.allocator.destroy(self.prefill_ctx_storage);
            self.allocator.free(self.list_active);
            self.allocator.free(self.list_sliding);
        }

        /// One slot's K and V rows of one layer (kv_dim floats each), replacing the
        /// mapped-buffer reads of memory.zig:106-107, hippocampus.zig:168-169 and
        /// snapshot.zig:97-98.
        pub fn kvRead(self: *GpuModelContext, layer: usize, slot: usize, k: []f32, v: []f32) GpuError!void {
            if (k.len < self.kv_dim or v.len < self.kv_dim) return error.InvalidArgument;
            try check(c.ch_kv_read(self.h, @intCast(layer), @intCast(slot), k.ptr, v.ptr));
        }
        /// The writes of model/memory_inject.zig:20-27 and snapshot restore.
        pub fn kvWrite(self: *GpuModelContext, layer: usize, slot: usize, k: []const f32, v: []const f32) GpuError!void {
            if (k.len < self.kv_dim or v.len < self.kv_dim) return error.InvalidArgument;
            try check(c.ch_kv_write(self.h, @intCast(layer), @intCast(slot), k.ptr, v.ptr));
        }
        /// Zero the KV caches and decode state (server.zig:76-82).
        pub fn zeroState(self: *GpuModelContext) GpuError!void {
            try check(c.ch_model_zero_state(self.h));
            @memset(self.buf_x.bytes, 0);
        }

        fn mirrorTopk(self: *GpuModelContext, top: *const [64]c.ch_topk) void {
            const ids = self.buf_topk_ids.asSlice(u32);
            const vals = self.buf_topk_vals.asSlice(f32);
            for (top, 0..) |t, i| {
                ids[i] = t.id;
                vals[i] = t.val;
            }
        }
        fn mirrorState(self: *GpuModelContext) GpuError!void {
            try check(c.ch_read_x(self.h, self.buf_x.asSlice(f32).ptr));
            try check(c.ch_read_normed_x(self.h, self.buf_normed_x.asSlice(f32).ptr));
        }
    };
};

fn bf16Ptr(s: []const tensor.bf16) [*c]const u16 {
    return @ptrCast(s.ptr);
}
// createNormBuffer (model_gpu.zig:57-66): a norm of the wrong length is all ones -> NULL
fn normPtr(s: []const tensor.bf16, n: usize) [*c]const u16 {
    return if (s.len == n) bf16Ptr(s) else null;
}

// ---------------------------------------------------------------------------------
// gpuDispatchForwardToken (src/gpu/model_dispatch.zig:128-153): same arguments, same
// u32 result, 0 on failure (model_dispatch.zig:144)
pub const model_dispatch = struct {
    pub fn gpuDispatchForwardToken(gpu: *model_gpu.GpuModelContext, config: *const model_types.ModelConfig,
                                   layers: []const model_types.LayerWeights, x: []const f32,
                                   topk_out: ?[]model_types.TopKCandidate, clock: usize, slot_idx: usize,
                                   active_slots: []const usize, sliding_slots: []const usize) u32 {
        _ = layers;
        if (x.len < config.hidden_size or active_slots.len > 4096 or sliding_slots.len > 4096) return 0;
        for (active_slots, 0..) |s, i| gpu.list_active[i] = @intCast(s);
        for (sliding_slots, 0..) |s, i| gpu.list_sliding[i] = @intCast(s);
        var top: [64]c.ch_topk = undefined;
        var tok: u32 = 0;
        check(c.ch_forward_token(gpu.h, x.ptr, @intCast(clock), @intCast(slot_idx), gpu.list_active.ptr,
            @intCast(active_slots.len), gpu.list_sliding.ptr, @intCast(sliding_slots.len),
            if (topk_out != null) &top else null, &tok)) catch {
            logLastError("ch_forward_token");
            return 0;
        };
        if (topk_out) |out| {
            gpu.mirrorTopk(&top);
            for (out[0..64], top) |*dst, t| dst.* = .{ .id = t.id, .val = t.val };
        }
        gpu.mirrorState() catch return 0; // buf_x is read after the step (server/decode.zig:13)
        _ = tok;
        return gpu.buf_topk_ids.asSlice(u32)[0]; // model_dispatch.zig:152

    }
};

// ---------------------------------------------------------------------------------
// gpuDispatchPrefillBatch (src/gpu/batch_dispatch.zig:25-172)
pub const batch_dispatch = struct {
    pub const ProgressFn = *const fn (layer_idx: usize, total_layers: usize, ctx: ?*anyopaque) void;

    const Progress = struct { f: ProgressFn, ctx: ?*anyopaque };
    fn progressTrampoline(layer_idx: usize, total: usize, ctx: ?*anyopaque) callconv(.C) void {
        const p: *const Progress = @ptrCast(@alignCast(ctx.?));
        p.f(layer_idx, total, p.ctx);
    }

    pub fn gpuDispatchPrefillBatch(
        prefill: *batch_prefill.BatchPrefillContext,
        gpu: *model_gpu.GpuModelContext,
        config: *const model_types.ModelConfig,
        layers: []const model_types.LayerWeights,
        tokens: []const u32,
        embed_tokens: []const tensor.bf16,
        slots: []const u32,
        start_clock: usize,
        num_prev_slots: usize,
        logits_out: []f32,
        progress_fn: ?ProgressFn,
        progress_ctx: ?*anyopaque,
    ) !void {
        _ = config;
        _ = layers;
        _ = embed_tokens; // the model keeps the table on the device (ch_model_create_bf16)
        if (tokens.len == 0 or tokens.len > prefill.max_tokens) return error.BatchTooLarge;
        if (slots.len < num_prev_slots + tokens.len) return error.GpuError;
        var top: [64]c.ch_topk = undefined;
        var prog: Progress = undefined;
        var cb: c.ch_progress_fn = null;
        var cb_ctx: ?*anyopaque = null;
        if (progress_fn) |f| {
            prog = .{ .f = f, .ctx = progress_ctx };
            cb = &progressTrampoline;
            cb_ctx = @ptrCast(&prog);
        }
        check(c.ch_prefill(gpu.h, tokens.ptr, @intCast(tokens.len), null, slots.ptr, @intCast(start_clock),
            @intCast(num_prev_slots), &top, if (logits_out.len > 0) logits_out.ptr else null, logits_out.len,
            cb, cb_ctx)) catch |e| {
            logLastError("ch_prefill");
            return if (e == error.BatchTooLarge) error.BatchTooLarge else error.GpuError;
        };
        gpu.mirrorTopk(&top); // read back by server/prefill.zig:92-96
        gpu.mirrorState() catch return error.GpuError;
    }
};
