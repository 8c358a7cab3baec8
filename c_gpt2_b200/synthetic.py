"""Seeded synthetic weights and prompts for the benchmark and test workloads.

No checkpoint or dataset is available offline, so every workload uses
random-initialised weights of the real GPT-2 architecture: N(0, 0.02) for
embeddings, projection weights and biases, LayerNorm gain 1 and bias 0, from
a seeded generator, drawn tensor by tensor in file order. Prompt token ids
are uniform in [0, vocab).
"""
from __future__ import annotations

import io
from typing import Iterator

import numpy as np

from .quant8 import GPT2Dims, tensor_layout, write_fp32, write_quant8

INIT_STD = 0.02


def iter_fp32_weights(dims: GPT2Dims, seed: int = 0) -> Iterator[tuple[str, np.ndarray]]:
    rng = np.random.default_rng(seed)
    for name, shape in tensor_layout(dims):
        leaf = name.split(".")[-1]
        if leaf.endswith("gamma"):
            yield name, np.ones(shape, dtype=np.float32)
        elif leaf.endswith("beta"):
            yield name, np.zeros(shape, dtype=np.float32)
        else:
            a = rng.standard_normal(shape, dtype=np.float32)
            a *= np.float32(INIT_STD)
            yield name, a


def quant8_image(dims: GPT2Dims, seed: int = 0) -> bytes:
    buf = io.BytesIO()
    write_quant8(buf, iter_fp32_weights(dims, seed))
    return buf.getvalue()


def write_weight_files(dims: GPT2Dims, seed: int, fp32_path=None, quant8_path=None) -> None:
    """One pass over the generator writes the FP32 file and/or the quant8 file."""
    f32 = open(fp32_path, "wb") if fp32_path else None
    q8 = open(quant8_path, "wb") if quant8_path else None
    try:
        for name, arr in iter_fp32_weights(dims, seed):
            if f32:
                write_fp32(f32, [(name, arr)])
            if q8:
                write_quant8(q8, [(name, arr)])
    finally:
        if f32:
            f32.close()
        if q8:
            q8.close()


def iter_fp32_weights_gpu(dims: GPT2Dims, seed: int = 0, device="cuda"):
    """Same distributions drawn on the GPU (torch's seeded CUDA generator):
    the benchmark's way to make GPT-2 large's 774M weights in seconds.
    Yields (name, float32 CUDA tensor) in file order."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for name, shape in tensor_layout(dims):
        leaf = name.split(".")[-1]
        if leaf.endswith("gamma"):
            yield name, torch.ones(shape, dtype=torch.float32, device=device)
        elif leaf.endswith("beta"):
            yield name, torch.zeros(shape, dtype=torch.float32, device=device)
        else:
            yield name, torch.randn(shape, generator=g, dtype=torch.float32,
                                    device=device) * INIT_STD


def _quantize_gpu(W):
    """quant8.quantize_per_channel on a CUDA tensor (same fp32 arithmetic)."""
    import torch
    amax = W.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.clamp(torch.round(W / scale[:, None]), -127, 127).to(torch.int8)
    return q, scale


def quant8_image_gpu(dims: GPT2Dims, seed: int = 0, device="cuda",
                     fp32_path=None) -> np.ndarray:
    """quant8.bin image (numpy uint8) of GPU-drawn weights; optionally also
    writes the FP32 .bin of the same weights (for the reference's CPU build)."""
    import torch
    from .quant8 import ALIGNMENT, is_quantized, quant8_nbytes
    img = np.zeros(quant8_nbytes(dims), dtype=np.uint8)
    off = 0
    f32 = open(fp32_path, "wb") if fp32_path else None

    def put(t):
        nonlocal off
        b = t.contiguous().cpu().numpy().view(np.uint8).reshape(-1)
        img[off:off + b.size] = b
        off += -(-b.size // ALIGNMENT) * ALIGNMENT

    try:
        for name, W in iter_fp32_weights_gpu(dims, seed, device):
            if f32:
                f32.write(W.cpu().numpy().tobytes())
            if is_quantized(name):
                q, s = _quantize_gpu(W)
                put(q)
                put(s)
            else:
                put(W)
            del W
    finally:
        if f32:
            f32.close()
    assert off == img.size
    torch.cuda.synchronize()
    return img


def prompts(n_seq: int, T: int, vocab: int = 50257, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=(n_seq, T), dtype=np.int64).astype(np.int32)


def outlier_activations(M: int, K: int, seed: int = 0, frac: float = 0.01,
                        gain: float = 20.0) -> np.ndarray:
    """X ~ N(0,1) with a seeded 1% of channels scaled x20 (isolated-linear workload)."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K), dtype=np.float32)
    n_out = max(1, int(round(frac * K)))
    cols = rng.choice(K, size=n_out, replace=False)
    X[:, cols] *= np.float32(gain)
    return X
