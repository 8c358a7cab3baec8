"""ctypes binding of the in-tree C-ABI libraries (no torch types cross it).

The product path is native: if libgpt2_w8a8.so is missing, importing this
module raises — there is no Python or CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIBDIR = Path(__file__).resolve().parent / "lib"
CORE_PATH = LIBDIR / "libgpt2_w8a8.so"

W8A8_OK = 0
W8A8_ERR_INVALID = -1
W8A8_ERR_UNSUPPORTED = -2
W8A8_ERR_CUDA = -3
W8A8_ERR_DEVICE = -4
W8A8_ERR_NOMEM = -5
W8A8_ERR_IO = -6

EPI_DEQUANT, EPI_BIAS, EPI_BIAS_RESID, EPI_BIAS_GELU = 0, 1, 2, 3

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_f = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes); must match include/gpt2_w8a8.h and gpt2_engine.h
SIGNATURES = {
    "w8a8_init": (_i, [_i]),
    "w8a8_status_string": (C.c_char_p, [_i]),
    "w8a8_device_error": (_i, [_i]),
    "w8a8_quant_rows": (_i, [_p, _i64, _i, _i, _p, _p, _p]),
    "w8a8_layernorm_quant": (_i, [_p, _i64, _i, _i, _p, _p, _f, _p, _i64, _p, _p, _p]),
    "w8a8_embed_layernorm_quant": (_i, [_p, _p, _p, _i, _i, _p, _i, _p, _p, _p, _f, _p, _p, _p, _p]),
    "w8a8_gemm_s32": (_i, [_p, _i, _i, _p, _i, _p, _p]),
    "w8a8_linear": (_i, [_p, _p, _i, _i, _p, _p, _p, _i, _i, _p, _i64, _p, _i64, _p, _sz, _p]),
    "w8a8_linear_workspace_size": (_sz, [_i, _i]),
    "w8a8_absmax_record_floats": (_sz, [_i, _i]),
    "w8a8_linear_absmax": (_i, [_p, _p, _i, _i, _p, _p, _p, _i, _i, _p, _i64, _p, _i64, _p, _sz,
                                _p, _p, _sz, _p]),
    "w8a8_linear_from_bf16": (_i, [_p, _i64, _p, _i, _i, _i, _p, _p, _p, _i, _i, _p, _i64, _p,
                                   _i64, _p, _p, _p, _sz, _p]),
    "w8a8_linear_noalloc": (_i, [_p, _p, _i, _i, _p, _p, _p, _i, _i, _p, _i64, _p, _i64, _p]),
    "w8a8_layernorm_linear_qkv": (_i, [_p, _i64, _p, _p, _f, _p, _p, _i, _i, _p, _p, _p, _p, _i64,
                                       _p, _p, _i64, _i, _p, _p, _sz, _p]),
    "w8a8_layernorm_linear_absmax": (_i, [_p, _i64, _p, _p, _f, _p, _p, _i, _i, _p, _p, _p, _i, _i,
                                          _p, _i64, _p, _i64, _p, _sz, _p, _p, _sz, _p]),
    "w8a8_linear_qkv": (_i, [_p, _p, _i, _i, _p, _p, _p, _p, _i64, _p, _p, _i64, _i, _p, _p,
                             _sz, _p]),
    "w8a8_linear_qkv_heads": (_i, [_p, _p, _i, _i, _i, _p, _p, _p, _p, _i64, _p, _p, _i64, _i,
                                   _p, _p, _sz, _p]),
    "w8a8_row_amax": (_i, [_p, _i64, _i, _i, _p, _p]),
    "w8a8_quant_rows_amax": (_i, [_p, _i64, _i, _i, _p, _i, _i64, _p, _i64, _p, _p]),
    "w8a8_reduce_residual_layernorm_quant": (_i, [_p, _i64, _i, _i64, _i, _i, _p, _p, _p, _p, _i64,
                                                  _p, _i64, _p, _p, _f, _p, _i64, _p, _p]),
    "w8a8_row_amax_to": (_i, [_p, _i64, _i, _i, _p, _i, _p]),
    "w8a8_reduce_residual_layernorm_quant_bcast": (_i, [_p, _i64, _i, _i64, _i, _i, _p, _p, _p, _p,
                                                        _i64, _p, _i64, _p, _p, _f, _p, _i64, _p,
                                                        _p, _p, _i, _i64, _p]),
    "w8a8_gemm_s32_scatter": (_i, [_p, _i, _i, _p, _i, _p, _i, _i, _p]),
    "w8a8_peer_alloc": (_i, [_sz, _p, _p]),
    "w8a8_peer_open": (_i, [_p, _p]),
    "w8a8_peer_close": (_i, [_p]),
    "w8a8_peer_free": (_i, [_p]),
    "w8a8_peer_copy": (_i, [_p, _p, _sz, _p]),
    "w8a8_peer_signal": (_i, [_p, _i, C.c_uint32, _p]),
    "w8a8_peer_wait": (_i, [_p, _i, C.c_uint32, _p]),
    "w8a8_attention_prefill": (_i, [_p, _i64, _p, _p, _i64, _i, _i, _i, _i, _p, _i64, _p]),
    "w8a8_attention_decode_workspace_size": (_sz, [_i, _i, _i]),
    "w8a8_attention_decode": (_i, [_p, _i64, _p, _p, _i64, _i, _p, _i, _i, _i, _p, _i64, _p, _sz, _p]),
    "w8a8_attention_decode_launches": (_i, [_i, _i, _i]),
    "w8a8_attention_decode_workspace_reset": (_i, [_p, _sz, _p]),
    "w8a8_attention_decode_quant": (_i, [_p, _i64, _p, _p, _i64, _i, _p, _i, _i, _i, _p, _i64, _p,
                                         _p, _p, _sz, _p]),
    "w8a8_lm_head": (_i, [_p, _i64, _i, _i, _p, _i, _p, _i64, _p]),
    "w8a8_sample_greedy": (_i, [_p, _i64, _i, _i, _p, _p, _i64, _p, _p]),
    "w8a8_sample_topk": (_i, [_p, _i64, _i, _i, _f, _i, _p, _i64, _p, _p, _p, _i64, _p, _p,
                              _i64, _p]),
    "w8a8_advance_positions": (_i, [_p, _p, _i, _i, _p]),
    "w8a8_ref_embeddings": (_i, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "w8a8_ref_add_bias": (_i, [_p, _i, _i, _p, _p]),
    "w8a8_ref_add_2d": (_i, [_p, _i, _i, _p, _p, _p]),
    "w8a8_ref_gelu": (_i, [_p, _i, _i, _p]),
    "w8a8_ref_dequant": (_i, [_p, _p, _p, _p, _i, _i, _p]),
    "w8a8_ref_causal_mask": (_i, [_p, _i, _i, _p]),
    "w8a8_ref_concat_heads": (_i, [_p, _p, _i, _i, _i, _i, _p]),
    "w8a8_ref_softmax": (_i, [_p, _i, _i, _i, _p, _f, _i, _p]),
    "gpt2_engine_create": (_i, [_p, _i, _p]),
    "gpt2_engine_destroy": (None, [_p]),
    "gpt2_engine_load_quant8": (_i, [_p, C.c_char_p]),
    "gpt2_engine_load_quant8_memory": (_i, [_p, _p, _sz]),
    "gpt2_engine_quant8_bytes": (_sz, [_p]),
    "gpt2_engine_generate": (_i, [_p, _p, _i, _i, _i, _p]),
    "gpt2_engine_generate_device": (_i, [_p, _p, _i, _i, _i, _p, _p]),
    "gpt2_engine_prefill": (_i, [_p, _p, _i, _i, _p, _i]),
    "gpt2_engine_decode_steps": (_i, [_p, _i]),
    "gpt2_engine_slots_begin": (_i, [_p, _i, _p, _i]),
    "gpt2_engine_slot_prefill": (_i, [_p, _i, _p, _i]),
    "gpt2_engine_slot_release": (_i, [_p, _i, _p]),
    "gpt2_engine_slot_tokens": (_i, [_p, _i]),
    "gpt2_engine_serve": (_i, [_p, _p, _i, _i]),
    "gpt2_engine_copy_logits": (_i, [_p, _p, _i]),
    "gpt2_engine_set_graphs": (_i, [_p, _i]),
    "gpt2_engine_set_decode_split": (_i, [_p, _i]),
    "w8a8_last_cuda_error": (C.c_char_p, []),
    "gpt2_engine_set_sampling": (_i, [_p, _f, _i]),
    "gpt2_quant8_check_manifest": (_i, [_p, C.c_char_p, C.c_char_p, C.c_size_t]),
    "gpt2_engine_set_draws": (_i, [_p, _i, _p, _i]),
    "gpt2_reference_draws": (_i, [C.c_uint, _p, _i]),
    "gpt2_engine_launches_per_decode_step": (_i, [_p]),
    "gpt2_engine_launches_per_prefill": (_i, [_p]),
    "gpt2_engine_stream": (_p, [_p]),
    "gpt2_engine_last_error": (C.c_char_p, [_p]),
}

# include/cuda_kernels.h, per model size (void functions)
COMPAT_SYMBOLS = [
    "embeddings_cuda", "layernorm_cuda", "add_bias_cuda", "softmax_cuda", "casual_masking_cuda",
    "gelu_cuda", "concat_heads_cuda", "add_2d_cuda", "per_token_quant_cuda",
    "dequant_int32_to_bf16_cuda", "dot_2d_int8_fused_cuda", "attention_prefill_cuda",
    "attention_decode_cuda", "lm_head_greedy_cuda", "lm_head_topk_cuda",
]
COMPAT_SIGNATURES = {
    "embeddings_cuda": [_p, _p, _p, _p, _i, _i],
    "layernorm_cuda": [_p, _i, _i, _p, _p, _p, _f],
    "add_bias_cuda": [_p, _i, _i, _p, _p],
    "softmax_cuda": [_p, _i, _i, _i, _p, _f, _i],
    "casual_masking_cuda": [_p, _i, _i],
    "gelu_cuda": [_p, _i, _i, _p],
    "concat_heads_cuda": [_p, _p, _i, _i, _i, _i],
    "add_2d_cuda": [_p, _i, _i, _p, _p],
    "per_token_quant_cuda": [_p, _p, _p, _i, _i],
    "dequant_int32_to_bf16_cuda": [_p, _p, _p, _p, _i, _i],
    "dot_2d_int8_fused_cuda": [_p, _i, _i, _p, _p, _p, _i, _p, _i, _p, _p, _p],
    "attention_prefill_cuda": [_p, _p, _p, _i, _p],
    "attention_decode_cuda": [_p, _p, _p, _i, _p, _p, _sz],
    "lm_head_greedy_cuda": [_p, _p, _p, _p],
    "lm_head_topk_cuda": [_p, _p, _p, _f, _i, _p, _p],
}


class EngineConfig(C.Structure):
    _fields_ = [("d_model", _i), ("n_layer", _i), ("n_head", _i), ("vocab", _i), ("ctx", _i),
                ("max_batch", _i), ("max_tokens", _i)]


class Request(C.Structure):
    """gpt2_request (include/gpt2_engine.h)."""
    _fields_ = [("prompt", _p), ("T", _i), ("n_gen", _i), ("out", _p), ("draws", _p)]


class W8A8Error(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {status_string(status)} ({status})")


_core = None
_compat: dict[str, C.CDLL] = {}


def core() -> C.CDLL:
    global _core
    if _core is None:
        if not CORE_PATH.exists():
            raise ImportError(
                f"{CORE_PATH} is missing: build it with `python -m c_gpt2_b200.build` "
                "(there is no fallback implementation)")
        lib = C.CDLL(str(CORE_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _core = lib
    return _core


def compat(size: str) -> C.CDLL:
    """The drop-in include/cuda_kernels.h library for one model size."""
    if size not in _compat:
        path = LIBDIR / f"libcuda_kernels_{size}.so"
        if not path.exists():
            raise ImportError(f"{path} is missing: run `python -m c_gpt2_b200.build`")
        core()
        lib = C.CDLL(str(path))
        for name, args in COMPAT_SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = None
            fn.argtypes = args
        _compat[size] = lib
    return _compat[size]


def status_string(st: int) -> str:
    s = core().w8a8_status_string(st)
    return s.decode() if s else "?"


def check(st: int, what: str) -> None:
    if st != W8A8_OK:
        raise W8A8Error(st, what)
