"""ctypes binding of ``libdtree_b200.so`` (C ABI in ``include/dtree_b200.h``).

The shared object is built in-tree by ``dtree_mlx_b200.build``.  There is no
fallback: if the library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdtree_b200.so"

DTREE_MAX_TREE = 128
DTREE_MASK_WORDS = 2

STATUS_NAMES = {
    0: "DTREE_OK",
    -1: "DTREE_ERR_INVALID_ARG",
    -2: "DTREE_ERR_CUDA",
    -3: "DTREE_ERR_UNSUPPORTED",
    -4: "DTREE_ERR_CAPACITY",
    -5: "DTREE_ERR_TREE",
    -6: "DTREE_ERR_STATE",
}


class DTreeError(RuntimeError):
    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class StepState(C.Structure):
    """Mirror of ``dtree_step_state``."""

    _fields_ = [
        ("start", C.c_int32),
        ("root_token", C.c_int32),
        ("step", C.c_int32),
        ("n_accepted", C.c_int32),
        ("bonus_token", C.c_int32),
        ("n_output", C.c_int32),
        ("n_nodes", C.c_int32),
        ("reserved", C.c_int32),
    ]


STEP_STATE_FIELDS = [f[0] for f in StepState._fields_]


class Qwen3Layer(C.Structure):
    _fields_ = [
        ("input_norm", C.c_void_p),
        ("qkv", C.c_void_p),
        ("q_norm", C.c_void_p),
        ("k_norm", C.c_void_p),
        ("o_proj", C.c_void_p),
        ("post_norm", C.c_void_p),
        ("gate_up", C.c_void_p),
        ("down", C.c_void_p),
    ]


class Qwen3Q4Layer(C.Structure):
    _fields_ = [
        ("qkv_scales", C.c_void_p),
        ("qkv_biases", C.c_void_p),
        ("o_scales", C.c_void_p),
        ("o_biases", C.c_void_p),
        ("gate_up_scales", C.c_void_p),
        ("gate_up_biases", C.c_void_p),
        ("down_scales", C.c_void_p),
        ("down_biases", C.c_void_p),
    ]


class Qwen3Desc(C.Structure):
    _fields_ = [
        ("hidden", C.c_int),
        ("layers", C.c_int),
        ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("ffn", C.c_int),
        ("vocab", C.c_int),
        ("rope_theta", C.c_float),
        ("rms_eps", C.c_float),
        ("t_cap", C.c_int),
        ("kv_capacity", C.c_int),
        ("n_capture", C.c_int),
        ("capture_layers", C.c_int * 16),
        ("embed", C.c_void_p),
        ("final_norm", C.c_void_p),
        ("layer", C.POINTER(Qwen3Layer)),
        ("kv_cache", C.c_void_p),
        ("h", C.c_void_p),
        ("xn", C.c_void_p),
        ("q", C.c_void_p),
        ("attn", C.c_void_p),
        ("act", C.c_void_p),
        ("norm_out", C.c_void_p),
        ("capture", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("quant_bits", C.c_int),
        ("group_size", C.c_int),
        ("q4_layer", C.POINTER(Qwen3Q4Layer)),
        ("verify_path", C.c_int),
        ("embed_q4_packed", C.c_void_p),
        ("embed_q4_scales", C.c_void_p),
        ("embed_q4_biases", C.c_void_p),
    ]


class Qwen35LinearLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("input_norm", "in_proj", "conv_weight", "norm", "out_proj", "post_norm",
                                          "gate_up", "down")]


class Qwen35AttnLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up",
                                          "down")]


class Qwen35Desc(C.Structure):
    _fields_ = [
        *[(n, C.c_int) for n in ("hidden", "layers", "full_attention_interval", "ffn", "vocab", "n_heads",
                                  "n_kv_heads", "head_dim")],
        ("rope_theta", C.c_float),
        ("partial_rotary_factor", C.c_float),
        ("rms_eps", C.c_float),
        *[(n, C.c_int) for n in ("lin_k_heads", "lin_v_heads", "lin_k_dim", "lin_v_dim", "conv_kernel", "t_cap",
                                  "kv_capacity", "n_capture")],
        ("capture_layers", C.c_int * 16),
        ("embed", C.c_void_p),
        ("final_norm", C.c_void_p),
        ("linear_layers", C.POINTER(Qwen35LinearLayer)),
        ("attn_layers", C.POINTER(Qwen35AttnLayer)),
        ("a_log", C.c_void_p),
        ("dt_bias", C.c_void_p),
        *[(n, C.c_void_p) for n in ("kv_cache", "conv_state", "rec_state", "h", "xn", "q", "gate", "attn", "act",
                                     "norm_out", "capture", "lin_proj", "lin_qkv", "workspace")],
        ("workspace_bytes", C.c_size_t),
    ]


QWEN35_BUFFERS = ("kv_cache", "conv_state", "rec_state", "h", "xn", "q", "gate", "attn", "act", "norm_out",
                  "capture", "lin_proj", "lin_qkv", "workspace")

P = C.c_void_p
I = C.c_int
SZ = C.c_size_t

# name -> (restype, argtypes)
PROTOTYPES = {
    "dtree_last_error": (C.c_char_p, []),
    "dtree_version": (I, []),
    "dtree_device_error": (I, [C.POINTER(C.c_uint32), I]),
    "dtree_test_delayed_store": (I, [P, C.c_int32, I, P]),
    "dtree_tree_build_workspace_bytes": (SZ, [I, I, I]),
    "dtree_tree_build": (I, [P, I, I, I, P, P, SZ, P, P, P, P, P, P, P, P]),
    "dtree_tree_from_topk": (I, [P, P, I, I, I, P, P, P, P, P, P, P]),
    "dtree_tree_build_noalloc_max_bytes": (SZ, []),
    "dtree_tree_build_noalloc_max_vocab": (I, [I]),
    "dtree_tree_build_noalloc": (I, [P, I, I, I, P, P, P, P, P, P, P]),
    "dtree_chain_build": (I, [P, I, I, P, P, P, P, P, P, P]),
    "dtree_plant_draft_logits": (I, [P, I, I, C.c_uint32, P, P, I, C.c_float, P]),
    "dtree_accept_walk": (I, [P, P, P, P, P, P, I, P, I, P]),
    "dtree_kv_compact": (I, [P, I, I, I, I, P, P, P]),
    "dtree_gather_rows": (I, [P, SZ, P, P, P, I, P]),
    "dtree_step_commit": (I, [P, P]),
    "dtree_linear_workspace_bytes": (SZ, [I, I]),
    "dtree_linear_bf16": (I, [P, I, I, P, I, P, P, SZ, I, P]),
    "dtree_linear_q4": (I, [P, I, I, P, P, P, I, P, P, SZ, I, P]),
    "dtree_linear_q4_workspace_bytes": (SZ, [I, I, I]),
    "dtree_tree_conv1d": (I, [P, I, P, P, P, I, I, I, I, P, P, P]),
    "dtree_tree_gated_delta": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, I, P, P, P]),
    "dtree_gated_delta_commit": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, I, P, P]),
    "dtree_conv_state_commit": (I, [P, I, P, P, P, I, I, I, I, P, P]),
    "dtree_qwen35_buffer_bytes": (I, [C.POINTER(Qwen35Desc), C.POINTER(C.c_size_t)]),
    "dtree_qwen35_create": (I, [C.POINTER(Qwen35Desc), C.POINTER(C.c_void_p)]),
    "dtree_qwen35_destroy": (I, [P]),
    "dtree_qwen35_forward": (I, [P, P, P, P, P, I, I, P, P, P]),
    "dtree_qwen35_commit": (I, [P, P, P, P, P]),
    "dtree_dflash_context": (I, [P, P, P, P, I, I, I, I, P, P]),
    "dtree_dflash_context_ring": (I, [P, P, P, P, I, I, I, I, P, P, I, I, P]),
    "dtree_dflash_block": (I, [P, I, I, P, P, P]),
    "dtree_qwen3_forward_logits": (I, [P, P, P, P, I, P, P, P]),
    "dtree_tree_attention_workspace_bytes": (SZ, [I, I, I, I]),
    "dtree_tree_attention": (I, [P, I, P, P, I, I, I, I, I, P, P, P, I, P, SZ, P]),
    "dtree_lm_head_workspace_bytes": (SZ, [I]),
    "dtree_lm_head_argmax": (I, [P, I, I, I, P, I, P, P, SZ, P]),
    "dtree_lm_head_sample": (I, [P, I, I, I, P, I, C.c_float, C.c_uint32, P, P, P, SZ, P]),
    "dtree_chain_sample": (I, [P, I, I, C.c_float, C.c_uint32, P, P, P, P, P, P, P]),
    "dtree_qwen3_set_sampling": (I, [P, C.c_float, C.c_uint32]),
    "dtree_qwen3_set_attention_keys": (I, [P, I]),
    "dtree_qwen3_prefill_workspace_bytes": (C.c_size_t, [P, I]),
    "dtree_qwen3_prefill": (I, [P, P, P, I, P, P, I, P, P, P, C.c_size_t, P]),
    "dtree_qwen35_set_sampling": (I, [P, C.c_float, C.c_uint32]),
    "dtree_qwen35_prefill_workspace_bytes": (C.c_size_t, [P, I]),
    "dtree_qwen35_prefill": (I, [P, P, P, I, P, P, I, P, P, P, C.c_size_t, P]),
    "dtree_qwen3_buffer_bytes": (I, [C.POINTER(Qwen3Desc), C.POINTER(C.c_size_t)]),
    "dtree_qwen3_create": (I, [C.POINTER(Qwen3Desc), C.POINTER(C.c_void_p)]),
    "dtree_qwen3_destroy": (I, [P]),
    "dtree_qwen3_forward_tree": (I, [P, P, P, P, I, P, P, P]),
}

_lib = None


def load() -> C.CDLL:
    """Load the library once (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("DTREE_B200_LIB", str(LIB_PATH))
    if not Path(path).exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m dtree_mlx_b200.build` "
            "(the B200 CUDA library is required; there is no CPU fallback)"
        )
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().dtree_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> int:
    """Call an int-returning entry point and raise DTreeError on failure."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise DTreeError(rc, name, last_error())
    return rc


def device_error(clear: bool = True) -> int:
    code = C.c_uint32(0)
    call("dtree_device_error", C.byref(code), 1 if clear else 0)
    return int(code.value)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
