"""The drop-in ABI (libcuda_kernels_<size>.so, include/cuda_kernels.h)
against the reference's own CUDA kernels, compiled from the reference tree
for sm_100a into oracle/_ref/libref_kernels_<size>.so and run on the same
device buffers. Both sides compute on the GPU with the same CUDA math
library, so every result is compared bit for bit."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from c_gpt2_b200 import _lib
from oracle import oracle
from tests.gpu_util import from_dev_bf16, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
D_MODEL = {"small": 768, "large": 1280}


def _ref_lib(size):
    path = ROOT / "oracle" / "_ref" / f"libref_kernels_{size}.so"
    if not path.exists():
        pytest.skip(f"{path.name} not built (make -C oracle ref needs the reference tree)")
    lib = C.CDLL(str(path))
    for name, args in _lib.COMPAT_SIGNATURES.items():
        if hasattr(lib, name):
            getattr(lib, name).argtypes = args
            getattr(lib, name).restype = None
    return lib


def _both(size):
    return _lib.compat(size), _ref_lib(size)


def _p(t):
    return t.data_ptr()


def _sync():
    torch.cuda.synchronize()


@pytest.mark.parametrize("size", ["small", "large"])
def test_per_token_quant(cuda, size):
    ours, ref = _both(size)
    rng = np.random.default_rng(1)
    for M, K in [(1, D_MODEL[size]), (77, D_MODEL[size]), (40, 4 * D_MODEL[size])]:
        x = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((M, K)).astype(np.float32) * 3))
        outs = []
        for lib in (ours, ref):
            q = torch.empty((M, K), dtype=torch.int8, device=cuda)
            s = torch.empty((M,), dtype=torch.float32, device=cuda)
            lib.per_token_quant_cuda(_p(x), _p(q), _p(s), M, K)
            _sync()
            outs.append((q.cpu().numpy(), s.cpu().numpy()))
        np.testing.assert_array_equal(outs[0][0], outs[1][0])
        np.testing.assert_array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("size", ["small", "large"])
def test_layernorm(cuda, size):
    ours, ref = _both(size)
    d = D_MODEL[size]
    rng = np.random.default_rng(2)
    M = 64
    x = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((M, d)).astype(np.float32) * 2 + 0.5))
    g = to_dev_bf16(oracle.bf16_bits(rng.uniform(0.5, 1.5, d).astype(np.float32)))
    b = to_dev_bf16(oracle.bf16_bits(rng.standard_normal(d).astype(np.float32) * 0.1))
    outs = []
    for lib in (ours, ref):
        y = torch.empty((M, d), dtype=torch.bfloat16, device=cuda)
        lib.layernorm_cuda(_p(x), M, d, _p(g), _p(b), _p(y), 1e-5)
        _sync()
        outs.append(from_dev_bf16(y))
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("size", ["small", "large"])
def test_gelu_bias_add_dequant(cuda, size):
    ours, ref = _both(size)
    rng = np.random.default_rng(3)
    M, N = 33, 4 * D_MODEL[size]
    base = oracle.bf16_bits(rng.standard_normal((M, N)).astype(np.float32) * 2)
    bias = to_dev_bf16(oracle.bf16_bits(rng.standard_normal(N).astype(np.float32) * 0.02))
    other = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((M, N)).astype(np.float32)))
    acc = to_dev(rng.integers(-2_000_000, 2_000_000, (M, N), dtype=np.int32))
    sw = to_dev(rng.uniform(1e-3, 1e-2, N).astype(np.float32))
    sx = to_dev(rng.uniform(1e-3, 1e-1, M).astype(np.float32))
    res = []
    for lib in (ours, ref):
        a = to_dev_bf16(base)
        lib.gelu_cuda(_p(a), N, M, None)
        lib.add_bias_cuda(_p(a), M, N, _p(bias), None)
        out = torch.empty_like(a)
        lib.add_2d_cuda(_p(a), M, N, _p(other), _p(out))
        lib.add_2d_cuda(_p(out), M, N, _p(other), None)  # in place
        dq = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
        lib.dequant_int32_to_bf16_cuda(_p(acc), _p(sw), _p(sx), _p(dq), M, N)
        _sync()
        res.append((from_dev_bf16(a), from_dev_bf16(out), from_dev_bf16(dq)))
    for u, v in zip(*res):
        np.testing.assert_array_equal(u, v)


@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("temperature", [1.0, 0.7])
def test_softmax(cuda, causal, temperature):
    ours, ref = _both("small")
    rng = np.random.default_rng(4)
    rows, cols, stride = 37, 300, 320
    x = oracle.bf16_bits(rng.standard_normal((rows, stride)).astype(np.float32) * 4)
    res = []
    for lib in (ours, ref):
        a = to_dev_bf16(x)
        out = to_dev_bf16(np.zeros((rows, stride), np.uint16))
        lib.softmax_cuda(_p(a), rows, cols, stride, _p(out), temperature, causal)
        _sync()
        res.append(from_dev_bf16(out))
    np.testing.assert_array_equal(res[0], res[1])
    # the vocabulary softmax is called in place (gpt2.c:2182)
    res = []
    for lib in (ours, ref):
        a = to_dev_bf16(x[:1, :300].copy())
        lib.softmax_cuda(_p(a), 1, 300, 300, _p(a), temperature, 0)
        _sync()
        res.append(from_dev_bf16(a))
    np.testing.assert_array_equal(res[0], res[1])


def test_embeddings_concat_mask(cuda):
    ours, ref = _both("small")
    rng = np.random.default_rng(5)
    d, V, Cx, H, hd = 768, 1000, 1024, 12, 64
    wte = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((V, d)).astype(np.float32) * 0.02))
    wpe = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((Cx, d)).astype(np.float32) * 0.02))
    tok = to_dev(rng.integers(0, V, Cx).astype(np.int32))
    src = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((H, Cx, hd)).astype(np.float32)))
    scores = oracle.bf16_bits(rng.standard_normal((64, 64)).astype(np.float32))
    res = []
    for lib in (ours, ref):
        emb = torch.zeros((Cx, d), dtype=torch.bfloat16, device=cuda)
        lib.embeddings_cuda(_p(wte), _p(wpe), _p(tok), _p(emb), 5, 20)
        dest = torch.zeros((Cx, d), dtype=torch.bfloat16, device=cuda)
        for t in (0, 3, 1023):
            lib.concat_heads_cuda(_p(src), _p(dest), t, H, hd, Cx)
        m = to_dev_bf16(scores)
        lib.casual_masking_cuda(_p(m), 64, 50)
        _sync()
        res.append((from_dev_bf16(emb), from_dev_bf16(dest), from_dev_bf16(m)))
    for u, v in zip(*res):
        np.testing.assert_array_equal(u, v)
