"""CPU tests: the oracle pinned against the reference's own outputs, the
oracle's restatements against independent numpy forms, and the C ABI
(libraries load, every declared symbol is exported, host-side validation)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"


# ---- oracle pinned by the reference ---------------------------------------

def test_oracle_prefill_logits_vs_reference_fp32():
    """The oracle's W8A8 prefill on GPT-2 small (seed-0 weights, 32-token
    prompt) against the reference's own CPU FP32 build on the same weights:
    same greedy token, logits within the W8A8 quantization error."""
    from c_gpt2_b200.quant8 import DIMS
    from c_gpt2_b200.synthetic import quant8_image
    z = np.load(GOLDEN / "ref_fp32_small.npz")
    img = quant8_image(DIMS["small"], 0)
    toks, lg = oracle.generate(img, DIMS["small"], z["prompt"], 1)
    ref = z["prefill_logits"].astype(np.float32)
    got = oracle.bf16_to_f32(lg)
    assert toks[0] == z["first_token"][0] == int(np.argmax(ref))
    err = np.abs(got - ref)
    assert err.mean() < 2e-2, err.mean()
    assert err.max() < 0.15, err.max()


def test_oracle_quant_semantics():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((6, 100)).astype(np.float32)
    x[1] = 0.0                      # zero row -> scale 1, all zeros
    x[2, 5] = 300.0                 # outlier
    xb = oracle.bf16_bits(x)
    xq, sx = oracle.quant_rows(xb)
    xf = oracle.bf16_to_f32(xb)
    amax = np.abs(xf).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(np.rint(xf * inv[:, None]), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(sx, scale)
    np.testing.assert_array_equal(xq, q)
    assert sx[1] == 1.0 and not xq[1].any()


def test_oracle_gemm_and_linear():
    rng = np.random.default_rng(1)
    xq = rng.integers(-127, 128, (5, 48), dtype=np.int8)
    W = rng.integers(-127, 128, (7, 48), dtype=np.int8)
    Y = oracle.gemm_s32(xq, W)
    np.testing.assert_array_equal(Y, xq.astype(np.int64) @ W.astype(np.int64).T)
    sx = rng.uniform(0.01, 0.1, 5).astype(np.float32)
    sw = rng.uniform(1e-3, 1e-2, 7).astype(np.float32)
    b = oracle.bf16_bits(rng.standard_normal(7).astype(np.float32) * 0.02)
    out = oracle.linear(xq, sx, W, sw, b, oracle.EPI_BIAS)
    t = oracle.bf16_to_f32(oracle.bf16_bits((Y.astype(np.float32) * sw[None]) * sx[:, None]))
    y = oracle.bf16_bits(t + oracle.bf16_to_f32(b)[None])
    np.testing.assert_array_equal(out, y)


def test_oracle_layernorm_close_to_float64():
    rng = np.random.default_rng(2)
    for d in (768, 1280):
        x = oracle.bf16_bits(rng.standard_normal((4, d)).astype(np.float32) * 3 + 1)
        g = oracle.bf16_bits(rng.uniform(0.5, 1.5, d).astype(np.float32))
        b = oracle.bf16_bits(rng.standard_normal(d).astype(np.float32) * 0.1)
        y = oracle.bf16_to_f32(oracle.layernorm(x, g, b))
        xf = oracle.bf16_to_f32(x).astype(np.float64)
        mu = xf.mean(1, keepdims=True)
        ref = (xf - mu) / np.sqrt(xf.var(1, keepdims=True) + 1e-5)
        ref = ref * oracle.bf16_to_f32(g) + oracle.bf16_to_f32(b)
        assert np.max(np.abs(y - ref) / (np.abs(ref) + 1e-2)) < 1e-2


def test_oracle_softmax_and_greedy():
    rng = np.random.default_rng(3)
    x = oracle.bf16_bits(rng.standard_normal(1000).astype(np.float32))
    p = oracle.bf16_to_f32(oracle.softmax_row(x))
    xf = oracle.bf16_to_f32(x).astype(np.float64)
    ref = np.exp(xf - xf.max())
    ref /= ref.sum()
    assert np.max(np.abs(p - ref) / ref) < 1e-2
    assert oracle.greedy(x) == int(np.argmax(p))
    # ties on bf16 probabilities: the first index wins (gpt2.c:2216-2221)
    tie = np.zeros(10, np.float32)
    tie[3] = tie[7] = 2.0
    assert oracle.greedy(oracle.bf16_bits(tie)) == 3


def test_oracle_gelu_formula():
    for v in (-3.0, -0.5, 0.0, 0.3, 1.7, 6.0):
        want = 0.5 * v * (1 + np.tanh(0.79788456 * (v + 0.044715 * v ** 3)))
        assert abs(oracle.lib().orc_gelu(v) - want) < 1e-5


def test_oracle_attention_causal_matches_numpy():
    rng = np.random.default_rng(4)
    T, H = 9, 2
    d = 64 * H
    Q = oracle.bf16_bits(rng.standard_normal((T, d)).astype(np.float32))
    K = oracle.bf16_bits(rng.standard_normal((T, d)).astype(np.float32))
    V = oracle.bf16_bits(rng.standard_normal((T, d)).astype(np.float32))
    O = oracle.bf16_to_f32(oracle.attention(Q, K, V, 0, H))
    q, k, v = (oracle.bf16_to_f32(a).astype(np.float64) for a in (Q, K, V))
    for h in range(H):
        sl = slice(64 * h, 64 * h + 64)
        s = q[:, sl] @ k[:, sl].T / 8.0
        s[np.triu_indices(T, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        ref = p @ v[:, sl]
        assert np.max(np.abs(O[:, sl] - ref)) < 3e-2


# ---- C ABI -------------------------------------------------------------------

def _declared_functions(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    text = re.sub(r"#.*", "", text)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", text)
    return sorted(set(n for n in names if n not in ("sizeof",)))


def test_core_library_exports_every_declared_symbol():
    from c_gpt2_b200 import _lib
    lib = _lib.core()
    for h in ("gpt2_w8a8.h", "gpt2_engine.h"):
        names = _declared_functions(ROOT / "include" / h)
        assert len(names) > 5
        for n in names:
            assert hasattr(lib, n), f"{n} declared in {h} but not exported"
    for n in _lib.SIGNATURES:
        assert hasattr(lib, n)


@pytest.mark.parametrize("size", ["small", "medium", "large"])
def test_compat_library_exports_reference_abi(size):
    from c_gpt2_b200 import _lib
    lib = _lib.compat(size)
    names = _declared_functions(ROOT / "include" / "cuda_kernels.h")
    # the ten symbols of the reference's include/cuda_kernels.h
    ref_abi = ["embeddings_cuda", "layernorm_cuda", "add_bias_cuda", "softmax_cuda",
               "casual_masking_cuda", "gelu_cuda", "concat_heads_cuda", "add_2d_cuda",
               "per_token_quant_cuda", "dequant_int32_to_bf16_cuda"]
    for n in ref_abi:
        assert n in names
    for n in names:
        assert hasattr(lib, n), n


def test_host_validation_without_gpu():
    """Argument checks run before any CUDA call and return W8A8_ERR_INVALID."""
    from c_gpt2_b200 import _lib
    lib = _lib.core()
    assert lib.w8a8_quant_rows(None, 8, 4, 8, None, None, None) == _lib.W8A8_ERR_INVALID
    assert lib.w8a8_linear(None, None, 4, 16, None, None, None, 8, 1, None, 0, None, 8,
                           None, 0, None) == _lib.W8A8_ERR_INVALID
    assert lib.w8a8_quant_rows(None, 8, 0, 8, None, None, None) == _lib.W8A8_OK  # empty
    # the LayerNorm-forming entry points: missing rows / gain, and an empty call
    assert lib.w8a8_layernorm_linear_qkv(None, 768, None, None, 1e-5, None, None, 1, 768, None,
                                         None, None, None, 768, None, None, 0, 1, None, None, 0,
                                         None) == _lib.W8A8_ERR_INVALID
    assert lib.w8a8_layernorm_linear_qkv(None, 768, None, None, 1e-5, None, None, 0, 768, None,
                                         None, None, None, 768, None, None, 0, 1, None, None, 0,
                                         None) == _lib.W8A8_OK
    n_part = C.c_int(7)
    assert lib.w8a8_layernorm_linear_absmax(None, 768, None, None, 1e-5, None, None, 1, 768, None,
                                            None, None, 3072, _lib.EPI_BIAS_GELU, None, 0, None,
                                            3072, None, 0, C.byref(n_part), None, 0,
                                            None) == _lib.W8A8_ERR_INVALID
    assert n_part.value == 0
    assert lib.w8a8_layernorm_linear_absmax(None, 768, None, None, 1e-5, None, None, 1, 768, None,
                                            None, None, 3072, _lib.EPI_BIAS_GELU, None, 0, None,
                                            3072, None, 0, None, None, 0,
                                            None) == _lib.W8A8_ERR_INVALID  # no n_part
    assert _lib.status_string(_lib.W8A8_ERR_DEVICE).startswith("a kernel")
    cfg = _lib.EngineConfig(768, 12, 10, 50257, 1024, 4, 4096)  # head_dim != 64
    h = C.c_void_p()
    assert lib.gpt2_engine_create(C.byref(cfg), 0, C.byref(h)) == _lib.W8A8_ERR_INVALID
    cfg = _lib.EngineConfig(768, 12, 12, 50257, 2048, 4, 4096)  # ctx > 1024
    assert lib.gpt2_engine_create(C.byref(cfg), 0, C.byref(h)) == _lib.W8A8_ERR_INVALID


def test_engine_quant8_size_matches_writer():
    from c_gpt2_b200 import _lib
    from c_gpt2_b200.quant8 import DIMS, GPT2Dims, quant8_nbytes
    for dims in (DIMS["small"], DIMS["large"], GPT2Dims(64, 2, 1, 100, 16)):
        cfg = _lib.EngineConfig(dims.d_model, dims.n_layer, dims.n_head, dims.vocab, dims.ctx,
                                1, 16)
        assert _lib.core().gpt2_engine_quant8_bytes(C.byref(cfg)) == quant8_nbytes(dims)
