"""ctypes binding of ``libnkimoe.so`` (the C ABI in ``include/nkimoe.h``).

There is no fallback: if the shared library is missing or fails to load, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libnkimoe.so")

NKM_OK = 0
NKM_ERR_ARG = 1
NKM_ERR_CUDA = 2
NKM_ERR_TIMEOUT = 4
NKM_ERR_INDEX = 8

NKM_STAGE_ATTN = 1
NKM_STAGE_MOE = 2
NKM_STAGE_LMHEAD = 4
NKM_STAGE_QKV_IN = 8
NKM_STAGE_KV_FIRST = 16
NKM_MOE_WEIGHTS_BF16 = 0
NKM_MOE_WEIGHTS_MXFP8 = 1

NKM_PACK_PLAIN = 0
NKM_PACK_GATE_UP = 1


class nkm_qwen3_layer(ctypes.Structure):
    _fields_ = [("wqkv_ft", c_void_p), ("wo_ft", c_void_p), ("q_norm", c_void_p), ("k_norm", c_void_p),
                ("ln1", c_void_p), ("ln2", c_void_p), ("router", c_void_p), ("w13_ft", c_void_p),
                ("w2_ft", c_void_p), ("router_bias", c_void_p)]


class nkm_qwen3_desc(ctypes.Structure):
    _fields_ = [("hidden", c_int32), ("n_q_heads", c_int32), ("n_kv_heads", c_int32), ("head_dim", c_int32),
                ("n_experts", c_int32), ("top_k", c_int32), ("moe_inter", c_int32), ("n_layers", c_int32),
                ("vocab", c_int32), ("rms_eps", c_float), ("layers", POINTER(nkm_qwen3_layer)),
                ("final_norm", c_void_p), ("lm_head_ft", c_void_p), ("embed", c_void_p),
                ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("rope_max_pos", c_int32),
                ("k_pool", c_void_p), ("v_pool", c_void_p), ("num_blocks", c_int32),
                ("block_size", c_int32), ("max_batch", c_int32), ("n_ranks", c_int32), ("rank", c_int32),
                ("expert_begin", c_int32), ("n_local_experts", c_int32), ("xchg", c_void_p * 8)]


class nkm_qwen3_step(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("input_ids", c_void_p), ("x_in", c_void_p), ("positions", c_void_p),
                ("block_table", c_void_p), ("max_blocks_per_seq", c_int32), ("y_out", c_void_p),
                ("logits_out", c_void_p), ("first_layer", c_int32), ("num_layers", c_int32),
                ("stages", c_int32), ("residual", c_int32), ("trace_topk_idx", c_void_p),
                ("trace_topk_w", c_void_p), ("trace_router_logits", c_void_p), ("trace_qkv", c_void_p),
                ("trace_resid_mid", c_void_p), ("trace_resid_out", c_void_p), ("trace_stage_ns", c_void_p)]


class nkm_gptoss_layer(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("wqkv_ft", "bqkv", "wo_ft", "bo", "sinks", "ln1", "ln2", "router",
                                        "router_bias", "w13_fp4", "s13", "b13", "w2_fp4", "s2", "b2")] + \
        [("sliding", c_int32)]


class nkm_gptoss_desc(ctypes.Structure):
    _fields_ = [("hidden", c_int32), ("hidden_actual", c_int32), ("n_q_heads", c_int32), ("n_kv_heads", c_int32),
                ("head_dim", c_int32), ("n_experts", c_int32), ("top_k", c_int32), ("inter", c_int32),
                ("n_layers", c_int32), ("vocab", c_int32), ("rms_eps", c_float), ("swiglu_limit", c_float),
                ("swiglu_alpha", c_float), ("sliding_window", c_int32), ("layers", POINTER(nkm_gptoss_layer)),
                ("final_norm", c_void_p), ("lm_head_ft", c_void_p), ("embed", c_void_p),
                ("rope_cos", POINTER(c_float)), ("rope_sin", POINTER(c_float)), ("rope_max_pos", c_int32),
                ("k_pool", c_void_p), ("v_pool", c_void_p), ("num_blocks", c_int32), ("block_size", c_int32),
                ("max_batch", c_int32), ("max_context", c_int32), ("kv_fp8", c_int32), ("k_scale", c_float),
                ("v_scale", c_float), ("n_ranks", c_int32), ("rank", c_int32), ("expert_begin", c_int32),
                ("n_local_experts", c_int32), ("xchg", c_void_p * 8)]


class nkm_gptoss_step(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("input_ids", c_void_p), ("x_in", c_void_p), ("positions", c_void_p),
                ("block_table", c_void_p), ("max_blocks_per_seq", c_int32), ("y_out", c_void_p),
                ("logits_out", c_void_p), ("first_layer", c_int32), ("num_layers", c_int32),
                ("trace_qkv", c_void_p), ("trace_resid_mid", c_void_p), ("trace_resid_out", c_void_p),
                ("trace_router_logits", c_void_p), ("trace_topk_idx", c_void_p), ("trace_topk_w", c_void_p),
                ("trace_stage_ns", c_void_p)]


class nkm_moe_tc_desc(ctypes.Structure):
    _fields_ = [("hidden", c_int32), ("n_experts", c_int32), ("top_k", c_int32), ("moe_inter", c_int32),
                ("rms_eps", c_float), ("ln2", c_void_p), ("router", c_void_p), ("router_bias", c_void_p),
                ("w13", c_void_p), ("w2", c_void_p), ("max_tokens", c_int32), ("weight_format", c_int32),
                ("expert_begin", c_int32), ("n_local_experts", c_int32)]


class nkm_sample_params(ctypes.Structure):
    _fields_ = [("top_k", c_int32), ("top_p", c_float), ("temperature", c_float), ("seed", ctypes.c_uint64)]


# name -> (restype, argtypes); every symbol declared in include/nkimoe.h
SIGNATURES = {
    "nkm_qwen3_workspace_bytes": (c_size_t, [POINTER(nkm_qwen3_desc)]),
    "nkm_qwen3_xchg_bytes": (c_size_t, [POINTER(nkm_qwen3_desc)]),
    "nkm_qwen3_create": (c_int, [POINTER(nkm_qwen3_desc), c_void_p, c_size_t, POINTER(c_void_p)]),
    "nkm_qwen3_destroy": (None, [c_void_p]),
    "nkm_qwen3_decode_step": (c_int, [c_void_p, POINTER(nkm_qwen3_step), c_void_p]),
    "nkm_qwen3_status": (c_int, [c_void_p, c_void_p]),
    "nkm_qwen3_attention_block": (c_int, [c_void_p, c_int32, POINTER(nkm_qwen3_step), c_void_p]),
    "nkm_qwen3_moe_block": (c_int, [c_void_p, c_int32, POINTER(nkm_qwen3_step), c_void_p]),
    "nkm_qwen3_qkv_buffer": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_size_t)]),
    "nkm_qwen3_moe_block_noalloc": (c_int, [POINTER(nkm_qwen3_desc), c_int32, POINTER(nkm_qwen3_step), c_void_p,
                                            c_void_p]),
    "nkm_pack_ft": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p]),
    "nkm_sample_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "nkm_sample_logits": (c_int, [c_void_p, c_int32, c_int32, POINTER(nkm_sample_params), c_void_p, c_void_p,
                                  c_void_p, c_size_t, c_void_p]),
    "nkm_gptoss_workspace_bytes": (c_size_t, [POINTER(nkm_gptoss_desc)]),
    "nkm_gptoss_xchg_bytes": (c_size_t, [POINTER(nkm_gptoss_desc)]),
    "nkm_gptoss_create": (c_int, [POINTER(nkm_gptoss_desc), c_void_p, c_size_t, POINTER(c_void_p)]),
    "nkm_gptoss_destroy": (None, [c_void_p]),
    "nkm_gptoss_decode_step": (c_int, [c_void_p, POINTER(nkm_gptoss_step), c_void_p]),
    "nkm_gptoss_status": (c_int, [c_void_p, c_void_p]),
    "nkm_mxfp4_scale_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
    "nkm_pack_mxfp4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "nkm_moe_tc_workspace_bytes": (c_size_t, [POINTER(nkm_moe_tc_desc)]),
    "nkm_moe_block_tc": (c_int, [POINTER(nkm_moe_tc_desc), c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    "nkm_moe_tc_status": (c_int, [c_void_p, c_void_p]),
    "nkm_ep_push": (c_int, [c_void_p, ctypes.c_int64, c_void_p, c_int32, ctypes.c_int64, c_void_p, c_void_p]),
    "nkm_ep_arrivals_per_push": (c_int32, []),
    "nkm_ep_wait": (c_int, [c_void_p, ctypes.c_uint64, c_void_p, c_void_p]),
    "nkm_ep_reduce": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "nkm_moe_block_tc_partial": (c_int, [POINTER(nkm_moe_tc_desc), c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, ctypes.c_size_t, c_void_p]),
    "nkm_mxfp8_experts_bytes": (ctypes.c_size_t, [c_int32, c_int32, c_int32]),
    "nkm_pack_mxfp8_experts": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "nkm_last_error": (c_char_p, []),
    "nkm_version": (c_char_p, []),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load ``libnkimoe.so`` once (raises ``OSError`` if it is missing or broken)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python -m nki_moe_megakernel_b200.build`")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def last_error() -> str:
    return lib().nkm_last_error().decode()


class NkmError(RuntimeError):
    def __init__(self, code: int, where: str):
        super().__init__(f"{where} failed with status {code}: {last_error()}")
        self.code = code


def check(code: int, where: str) -> None:
    if code != NKM_OK:
        raise NkmError(code, where)
