"""Weight formats of the reference, written from host arrays.

* FP32 ``.bin`` — the order gpt2.c:1703-1800 reads: wte, wpe, then per layer
  ln_1 γ/β, c_attn W [3d,d] (Q,K,V rows), c_attn b [3d], c_proj W [d,d], c_proj
  b, ln_2 γ/β, c_fc W [4d,d], c_fc b, mlp c_proj W [d,4d], b; then ln_f γ/β.
  All weights [OUT, IN] (extract_weights.py:42-64). No header, no padding.
* INT8 ``quant8.bin`` — the same order with the four GEMM weights replaced by
  an int8 block followed by its fp32 per-output-channel scale, every block
  zero-padded to 16 bytes (tools/offline_quant/src/writer.py:34-69).
* ``quant8.json`` — the manifest written beside it
  (tools/offline_quant/src/writer.py:72-124): scheme, scale convention, the
  quantized and preserved tensor names and a memory summary, all determined
  by the model's dimensions.

Per-channel symmetric quantization follows
tools/offline_quant/src/quantizer.py:52-64: scale = amax/127 per output row
(1.0 for an all-zero row), q = clip(rint(W/scale), ±127).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import BinaryIO, Iterable, Iterator

import numpy as np

INT8_MAX = 127
ALIGNMENT = 16
QUANTIZED = ("W_qkv", "attn_proj", "W1", "W2")
PRESERVED = ("wte", "wpe", "ln1_gamma", "ln1_beta", "b_qkv", "attn_proj_bias",
             "ln2_gamma", "ln2_beta", "b1", "b2", "lnf_gamma", "lnf_beta")
MANIFEST_TOOL_VERSION = "0.1"
MANIFEST_SCHEME = "int8_per_channel_symmetric"
MANIFEST_SCALE_CONVENTION = "amax/127"
MANIFEST_SCALE_DTYPE = "fp32"


@dataclass(frozen=True)
class GPT2Dims:
    d_model: int
    n_layer: int
    n_head: int
    vocab: int = 50257
    ctx: int = 1024

    @property
    def d_ff(self) -> int:
        return 4 * self.d_model


DIMS = {
    "small": GPT2Dims(768, 12, 12),
    "medium": GPT2Dims(1024, 24, 16),
    "large": GPT2Dims(1280, 36, 20),
}


# the reference's model names and FP32 weight files (tools/offline_quant/src/reader.py:36-43,
# include/model_config.h:14,22,30)
WEIGHTS_FILES = {"small": "gpt2_c_weights.bin", "medium": "gpt2_medium_c_weights.bin",
                 "large": "gpt2_large_c_weights.bin"}


def model_name(dims: GPT2Dims) -> str | None:
    for name, known in DIMS.items():
        if (known.d_model, known.n_layer, known.n_head) == (dims.d_model, dims.n_layer,
                                                            dims.n_head):
            return name
    return None


def tensor_layout(dims: GPT2Dims) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every tensor in file order."""
    d, f = dims.d_model, dims.d_ff
    out: list[tuple[str, tuple[int, ...]]] = [("wte", (dims.vocab, d)), ("wpe", (dims.ctx, d))]
    for l in range(dims.n_layer):
        out += [
            (f"h{l}.ln1_gamma", (d,)), (f"h{l}.ln1_beta", (d,)),
            (f"h{l}.W_qkv", (3 * d, d)), (f"h{l}.b_qkv", (3 * d,)),
            (f"h{l}.attn_proj", (d, d)), (f"h{l}.attn_proj_bias", (d,)),
            (f"h{l}.ln2_gamma", (d,)), (f"h{l}.ln2_beta", (d,)),
            (f"h{l}.W1", (f, d)), (f"h{l}.b1", (f,)),
            (f"h{l}.W2", (d, f)), (f"h{l}.b2", (d,)),
        ]
    out += [("lnf_gamma", (d,)), ("lnf_beta", (d,))]
    return out


def is_quantized(name: str) -> bool:
    return name.split(".")[-1] in QUANTIZED


def quantize_per_channel(W: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """FP32 [OUT, IN] -> (int8 [OUT, IN], fp32 scale [OUT])."""
    if W.dtype != np.float32 or W.ndim != 2:
        raise TypeError("expected a 2-D float32 weight")
    amax = np.max(np.abs(W), axis=1)
    scale = np.where(amax > 0, amax / np.float32(INT8_MAX), np.float32(1.0)).astype(np.float32)
    q = np.rint(W / scale[:, None])
    np.clip(q, -INT8_MAX, INT8_MAX, out=q)
    return q.astype(np.int8), scale


def _block(fp: BinaryIO, arr: np.ndarray) -> int:
    data = np.ascontiguousarray(arr).tobytes()
    fp.write(data)
    pad = (-len(data)) % ALIGNMENT
    if pad:
        fp.write(b"\x00" * pad)
    return len(data) + pad


def write_quant8(fp: BinaryIO, tensors: Iterable[tuple[str, np.ndarray]]) -> int:
    """Write the quant8 image of FP32 tensors given in file order."""
    n = 0
    for name, arr in tensors:
        arr = np.asarray(arr, dtype=np.float32)
        if is_quantized(name):
            q, s = quantize_per_channel(arr)
            n += _block(fp, q)
            n += _block(fp, s)
        else:
            n += _block(fp, arr)
    return n


def write_fp32(fp: BinaryIO, tensors: Iterable[tuple[str, np.ndarray]]) -> int:
    n = 0
    for _, arr in tensors:
        data = np.ascontiguousarray(arr, dtype=np.float32).tobytes()
        fp.write(data)
        n += len(data)
    return n


def quant8_nbytes(dims: GPT2Dims) -> int:
    n = 0
    for name, shape in tensor_layout(dims):
        count = int(np.prod(shape))
        if is_quantized(name):
            n += -(-count // ALIGNMENT) * ALIGNMENT + -(-shape[0] * 4 // ALIGNMENT) * ALIGNMENT
        else:
            n += -(-count * 4 // ALIGNMENT) * ALIGNMENT
    return n


def read_quant8(data: bytes | memoryview, dims: GPT2Dims) -> dict[str, np.ndarray]:
    """Parse a quant8 image: quantized tensors give name -> int8, name.scale -> fp32."""
    mv = memoryview(data)
    off = 0
    out: dict[str, np.ndarray] = {}

    def take(count: int, dtype) -> np.ndarray:
        nonlocal off
        nbytes = count * np.dtype(dtype).itemsize
        if off + nbytes > len(mv):
            raise ValueError("quant8 image truncated")
        a = np.frombuffer(mv[off:off + nbytes], dtype=dtype)
        off += -(-nbytes // ALIGNMENT) * ALIGNMENT
        return a

    for name, shape in tensor_layout(dims):
        count = int(np.prod(shape))
        if is_quantized(name):
            out[name] = take(count, np.int8).reshape(shape)
            out[name + ".scale"] = take(shape[0], np.float32)
        else:
            out[name] = take(count, np.float32).reshape(shape)
    return out


# ---- the quant8.json manifest (tools/offline_quant/src/writer.py:72-124) ----

def memory_summary(dims: GPT2Dims) -> dict[str, int]:
    """writer.py:72-96: byte counts of the unpadded tensors, rounded (Python's
    round, half to even) to MiB / KiB."""
    d, f, L = dims.d_model, dims.d_ff, dims.n_layer
    preserved = 4 * (dims.vocab * d + dims.ctx * d + 2 * d + L * (2 * d + 3 * d + d + 2 * d + f + d))
    quantized = L * (3 * d * d + d * d + f * d + d * f)
    scales = 4 * L * (3 * d + d + f + d)
    mib = 1024 * 1024
    return {
        "source_fp32_total_mb": round((preserved + 4 * quantized) / mib),
        "quantized_int8_mb": round(quantized / mib),
        "preserved_fp32_mb": round(preserved / mib),
        "scale_overhead_kb": round(scales / 1024),
        "artifact_total_mb": round((preserved + quantized + scales) / mib),
    }


def build_manifest(dims: GPT2Dims, name: str | None = None,
                   weights_filename: str | None = None) -> dict:
    """writer.py:99-111 for a model of these dimensions; name and weights file
    default to the reference's for GPT-2 small / medium / large."""
    name = name or model_name(dims)
    if name is None:
        raise ValueError("dimensions of no GPT-2 size: give the model name")
    weights_filename = weights_filename or WEIGHTS_FILES[name]
    return {
        "tool_version": MANIFEST_TOOL_VERSION,
        "model": f"gpt2-{name}",
        "scheme": MANIFEST_SCHEME,
        "scale_convention": MANIFEST_SCALE_CONVENTION,
        "scale_dtype": MANIFEST_SCALE_DTYPE,
        "source_weights_path": f"weights/{weights_filename}",
        "quantized_tensors": list(QUANTIZED),
        "preserved_tensors": list(PRESERVED),
        "memory_summary": memory_summary(dims),
    }


def manifest_text(manifest: dict) -> str:
    """The file's text as writer.py:120-122 writes it."""
    return json.dumps(manifest, indent=2) + "\n"


def write_manifest(path: str | os.PathLike, dims: GPT2Dims, name: str | None = None,
                   weights_filename: str | None = None) -> None:
    with open(path, "w") as f:
        f.write(manifest_text(build_manifest(dims, name, weights_filename)))


def check_manifest(manifest: dict, dims: GPT2Dims) -> None:
    """Raise ValueError unless the manifest describes this scheme and a model
    of these dimensions (the model name, where it names a GPT-2 size, and the
    memory summary)."""
    want = {"scheme": MANIFEST_SCHEME, "scale_convention": MANIFEST_SCALE_CONVENTION,
            "scale_dtype": MANIFEST_SCALE_DTYPE, "quantized_tensors": list(QUANTIZED),
            "preserved_tensors": list(PRESERVED), "memory_summary": memory_summary(dims)}
    for key, value in want.items():
        if manifest.get(key) != value:
            raise ValueError(f"quant8 manifest: {key} is {manifest.get(key)!r}, expected {value!r}")
    name = model_name(dims)
    if name is not None and manifest.get("model") != f"gpt2-{name}":
        raise ValueError(f"quant8 manifest: model {manifest.get('model')!r} for GPT-2 {name}")
