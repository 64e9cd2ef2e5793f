"""ctypes binding of libchannel_b200.so (declarations mirror include/channel_cuda.h).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libchannel_b200.so"

u8, u16, u32, u64, f32 = C.c_uint8, C.c_uint16, C.c_uint32, C.c_uint64, C.c_float
vp, sz, i32 = C.c_void_p, C.c_size_t, C.c_int
P = C.POINTER

CH_IPC_HANDLE_BYTES = 64
CH_OK, CH_EINVAL, CH_ENOMEM, CH_ECUDA, CH_ETIMEOUT, CH_EBATCH, CH_ESTATE, CH_EDEVICE, CH_ECOMM = 0, -1, -2, -3, -4, -5, -6, -7, -8
STATUS_NAMES = {0: "CH_OK", -1: "CH_EINVAL", -2: "CH_ENOMEM", -3: "CH_ECUDA", -4: "CH_ETIMEOUT", -5: "CH_EBATCH",
                -6: "CH_ESTATE", -7: "CH_EDEVICE", -8: "CH_ECOMM"}


class ChTopk(C.Structure):
    _fields_ = [("id", u32), ("val", f32)]


class ChModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", u32), ("hidden_size", u32), ("intermediate_size", u32), ("num_hidden_layers", u32),
        ("num_attention_heads", u32), ("num_key_value_heads", u32), ("head_dim", u32), ("rotary_dim", u32),
        ("rms_norm_eps", f32), ("rope_theta", f32), ("rope_theta_full", f32),
        ("sliding_window", u32), ("max_prefill_tokens", u32), ("layer_types", u8 * 64),
    ]


class ChLayerWeights(C.Structure):
    _fields_ = [
        ("q_proj", P(u32)), ("k_proj", P(u32)), ("v_proj", P(u32)), ("o_proj", P(u32)),
        ("gate_proj", P(u32)), ("up_proj", P(u32)), ("down_proj", P(u32)),
        ("input_norm", P(f32)), ("q_norm", P(f32)), ("k_norm", P(f32)), ("post_attn_norm", P(f32)),
        ("pre_ffn_norm", P(f32)), ("post_ffn_norm", P(f32)), ("layer_scalar", f32),
    ]


class ChLayerWeightsBf16(C.Structure):
    _fields_ = [
        ("q_proj", P(u16)), ("k_proj", P(u16)), ("v_proj", P(u16)), ("o_proj", P(u16)),
        ("gate_proj", P(u16)), ("up_proj", P(u16)), ("down_proj", P(u16)),
        ("input_norm", P(u16)), ("q_norm", P(u16)), ("k_norm", P(u16)), ("post_attn_norm", P(u16)),
        ("pre_ffn_norm", P(u16)), ("post_ffn_norm", P(u16)), ("layer_scalar", f32),
    ]


class ChSamplerParams(C.Structure):
    _fields_ = [("temp", f32), ("top_p", f32), ("min_p", f32), ("repeat_penalty", f32), ("frequency_penalty", f32),
                ("presence_penalty", f32), ("top_k", u32), ("suppress_thinking", u8), ("suppress_critique", u8),
                ("suppress_channel_close", u8), ("reserved", u8)]


class ChStepDesc(C.Structure):
    _fields_ = [("clock", u32), ("slot", u32), ("n_active", u32), ("n_sliding", u32),
                ("active", P(u32)), ("sliding", P(u32))]


class ChStreamStep(C.Structure):
    _fields_ = [("stream", u32), ("token", u32), ("clock", u32), ("slot", u32),
                ("active", P(u32)), ("sliding", P(u32)), ("n_active", u32), ("n_sliding", u32)]


PROGRESS_FN = C.CFUNCTYPE(None, sz, sz, vp)

# name -> (restype, argtypes); every symbol declared in include/channel_cuda.h
SIGNATURES = {
    "ch_last_error": (C.c_char_p, []),
    "ch_api_version": (i32, []),
    "ch_ctx_create": (i32, [i32, P(vp)]),
    "ch_ctx_destroy": (None, [vp]),
    "ch_ctx_synchronize": (i32, [vp]),
    "ch_ctx_stream": (vp, [vp]),
    "ch_ctx_device_status": (i32, [vp, P(u32)]),
    "ch_model_create": (i32, [vp, P(ChModelConfig), P(ChLayerWeights), P(u32), P(f32), P(u16), P(vp)]),
    "ch_model_create_synthetic": (i32, [vp, P(ChModelConfig), u64, P(vp)]),
    "ch_model_create_bf16": (i32, [vp, P(ChModelConfig), P(ChLayerWeightsBf16), P(u16), P(u16), P(vp)]),
    "ch_model_create_synthetic_sharded": (i32, [vp, P(ChModelConfig), u64, u32, u32, P(vp)]),
    "ch_model_exchange_handle": (i32, [vp, vp]),
    "ch_model_attach_peers": (i32, [vp, vp]),
    "ch_model_destroy": (None, [vp]),
    "ch_model_zero_state": (i32, [vp]),
    "ch_model_weight_tiles": (i32, [vp, u32, i32, P(vp), P(u32), P(u32)]),
    "ch_forward_token": (i32, [vp, P(f32), u32, u32, P(u32), u32, P(u32), u32, P(ChTopk), P(u32)]),
    "ch_prefill": (i32, [vp, P(u32), u32, P(u16), P(u32), u32, u32, P(ChTopk), P(f32), sz, PROGRESS_FN, vp]),
    "ch_read_x": (i32, [vp, P(f32)]),
    "ch_read_normed_x": (i32, [vp, P(f32)]),
    "ch_kv_read": (i32, [vp, u32, u32, P(f32), P(f32)]),
    "ch_kv_write": (i32, [vp, u32, u32, P(f32), P(f32)]),
    "ch_decode_plan": (i32, [vp, P(ChStepDesc), u32]),
    "ch_streams_init": (i32, [vp, u32, u32]),
    "ch_stream_prefill": (i32, [vp, u32, P(u32), u32, P(u32), u32, u32, P(u32)]),
    "ch_streams_decode": (i32, [vp, P(ChStreamStep), u32, P(u32)]),
    "ch_streams_read_normed_x": (i32, [vp, u32, P(f32)]),
    "ch_sampler_create": (i32, [vp, P(ChSamplerParams), u64, u32, P(vp)]),
    "ch_sampler_destroy": (None, [vp]),
    "ch_sampler_set_recent": (i32, [vp, P(u32), u32]),
    "ch_sampler_sample_topk": (i32, [vp, vp, vp, u32, vp, u32, vp]),
    "ch_model_set_sampler": (i32, [vp, vp]),
    "ch_streams_read_logits": (i32, [vp, u32, P(f32)]),
    "ch_decode_run": (i32, [vp, u32, u32]),
    "ch_decode_continue": (i32, [vp, u32]),
    "ch_decode_tokens": (i32, [vp, P(u32), u32]),
    "ch_q4_tile_bytes": (sz, [u32, u32]),
    "ch_q8_tile_bytes": (sz, [u32, u32]),
    "ch_q4_pack": (i32, [vp, vp, u32, u32, vp]),
    "ch_q4_pack_gateup": (i32, [vp, vp, vp, u32, u32, vp]),
    "ch_q8_pack": (i32, [vp, vp, u32, u32, vp]),
    "ch_gemv_q4": (i32, [vp, vp, u32, u32, vp, vp]),
    "ch_gemv_q4_noalloc": (i32, [vp, u32, u32, vp, vp, vp, vp]),
    "ch_fused_mlp_q4": (i32, [vp, vp, u32, u32, vp, vp]),
    "ch_gemv_q8": (i32, [vp, vp, u32, u32, vp, vp]),
    "ch_rmsnorm": (i32, [vp, vp, vp, vp, u32, u32, f32]),
    "ch_add_rmsnorm": (i32, [vp, vp, vp, vp, vp, u32, u32, f32, f32]),
    "ch_decode_attention": (i32, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, f32, f32, f32, vp]),
    "ch_batch_causal_attention": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, f32, i32, vp]),
    "ch_topk64": (i32, [vp, vp, u32, vp, vp]),
    "ch_batch_gemm_q4": (i32, [vp, vp, u32, u32, vp, u32, vp]),
    "ch_batch_fused_mlp_q4": (i32, [vp, vp, u32, u32, vp, u32, vp]),
    "ch_batch_gemm_q4_mma": (i32, [vp, vp, u32, u32, vp, u32, vp]),
    "ch_batch_fused_mlp_q4_mma": (i32, [vp, vp, u32, u32, vp, u32, vp]),
    "ch_gen_q4_blocks": (i32, [vp, vp, u32, u32, u64, f32]),
    "ch_gen_bf16": (i32, [vp, vp, sz, u64, f32, f32]),
    "ch_quantize_q8_rows": (i32, [vp, vp, u32, u32, vp]),
    "ch_quantize_q4_rows": (i32, [vp, vp, u32, u32, vp]),
    "ch_tensor_seed": (u64, [u64, u32, u32]),
    "ch_ring_create": (vp, [u32, u32]),
    "ch_ring_destroy": (None, [vp]),
    "ch_ring_reset": (None, [vp]),
    "ch_ring_set_num_anchors": (None, [vp, sz]),
    "ch_ring_num_anchors": (sz, [vp]),
    "ch_ring_total_ingested": (sz, [vp]),
    "ch_ring_window_size": (sz, [vp, sz]),
    "ch_ring_get_slot_index": (sz, [vp, sz, sz]),
    "ch_ring_activate_slot": (sz, [vp, sz, sz]),
    "ch_ring_deactivate_slot": (None, [vp, sz, sz]),
    "ch_ring_activate_range": (None, [vp, sz, sz, P(u32)]),
    "ch_rings_fill_steps": (None, [P(vp), P(u32), P(u32), P(u32), u32, sz, P(ChStreamStep), P(u32)]),
    "ch_ring_rollback_clock": (None, [vp, sz]),
    "ch_ring_write_kv_meta": (None, [vp, sz, sz]),
    "ch_ring_write_recall_meta": (None, [vp, sz, sz, sz]),
    "ch_ring_clear_recall": (None, [vp]),
    "ch_ring_mark_boundary": (None, [vp, sz, i32, f32]),
    "ch_ring_is_active": (i32, [vp, sz, sz]),
    "ch_ring_slot_clock": (sz, [vp, sz, sz]),
    "ch_ring_active_slots": (sz, [vp, sz, sz, i32, sz, P(u32)]),
    "ch_ring_prefill_prev_slots": (sz, [vp, sz, sz, sz, P(u32)]),
    "ch_ring_dev_create": (i32, [vp, P(vp)]),
    "ch_ring_dev_destroy": (None, [vp]),
    "ch_ring_dev_upload": (i32, [vp, vp]),
    "ch_ring_dev_lists": (i32, [vp, u32, i32, sz, vp, vp, vp, vp, vp]),
    "ch_ring_dev_prefill_prev": (i32, [vp, u32, u32, vp, vp]),
    "ch_decode_run_ring": (i32, [vp, vp, vp, u32, u32, u32]),
}

_lib = None


def load() -> C.CDLL:
    """Load the in-tree shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} missing: run `python -m channel_b200.build` (no CPU fallback exists)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class ChannelError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def check(status: int) -> None:
    if status != CH_OK:
        raise ChannelError(status, load().ch_last_error().decode(errors="replace"))
