"""CPU tests: weight formats against the reference's own quantizer/writer
outputs (tests/golden/), and the product quantizer's edge cases."""
import hashlib
import io
import json
from pathlib import Path

import numpy as np
import pytest

from c_gpt2_b200.quant8 import (DIMS, GPT2Dims, quant8_nbytes, quantize_per_channel,
                                read_quant8, tensor_layout, write_fp32, write_quant8)
from c_gpt2_b200.synthetic import iter_fp32_weights, outlier_activations, prompts, quant8_image

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_weight_quant_matches_reference_golden():
    z = np.load(GOLDEN / "weight_quant.npz")
    names = sorted({k.split(".")[0] for k in z.files})
    assert set(names) == {"normal", "outlier", "zero_row", "ties"}
    for n in names:
        q, s = quantize_per_channel(z[f"{n}.W"])
        np.testing.assert_array_equal(q, z[f"{n}.int8"], err_msg=n)
        np.testing.assert_array_equal(s.view(np.uint32), z[f"{n}.scale"].view(np.uint32),
                                      err_msg=n)


def test_weight_quant_edge_cases():
    z = np.load(GOLDEN / "weight_quant.npz")
    q, s = quantize_per_channel(z["zero_row.W"])
    assert s[2] == 1.0 and not q[2].any()            # all-zero row: scale 1, zeros
    q, s = quantize_per_channel(z["ties.W"])
    assert q.max() == 127 and q.min() >= -127         # -128 never used
    # ties to even: -5.5 -> -6, -4.5 -> -4, 0.5 -> 0, 1.5 -> 2, 2.5 -> 2
    row = z["ties.W"][0]
    for x, want in [(-5.5, -6), (-4.5, -4), (0.5, 0), (1.5, 2), (2.5, 2)]:
        (idx,) = np.nonzero(row == np.float32(x))
        assert q[0, idx[0]] == want, x


def test_quant8_writer_matches_reference_writer():
    meta = json.loads((GOLDEN / "quant8_tiny.json").read_text())
    dims = GPT2Dims(**meta["dims"])
    buf = io.BytesIO()
    write_quant8(buf, iter_fp32_weights(dims, meta["seed"]))
    data = buf.getvalue()
    assert len(data) == meta["bytes"] == quant8_nbytes(dims)
    assert hashlib.sha256(data).hexdigest() == meta["sha256"]


def test_quant8_read_roundtrip():
    dims = GPT2Dims(d_model=64, n_layer=2, n_head=1, vocab=100, ctx=16)
    src = dict(iter_fp32_weights(dims, 3))
    img = quant8_image(dims, 3)
    back = read_quant8(img, dims)
    for name, shape in tensor_layout(dims):
        if name.split(".")[-1] in ("W_qkv", "attn_proj", "W1", "W2"):
            q, s = quantize_per_channel(src[name])
            np.testing.assert_array_equal(back[name], q)
            np.testing.assert_array_equal(back[name + ".scale"], s)
        else:
            np.testing.assert_array_equal(back[name], src[name])
    with pytest.raises(ValueError):
        read_quant8(img[:-32], dims)


def test_fp32_layout_matches_reference_sizes():
    # gpt2.c reads exactly these counts (gpt2.c:1703-1800); the FP32 file of
    # GPT-2 small is 124,439,808 parameters.
    buf = io.BytesIO()
    dims = DIMS["small"]
    n = sum(int(np.prod(s)) for _, s in tensor_layout(dims))
    assert n == 124439808
    dims_t = GPT2Dims(d_model=64, n_layer=1, n_head=1, vocab=10, ctx=8)
    assert write_fp32(buf, iter_fp32_weights(dims_t, 0)) == 4 * sum(
        int(np.prod(s)) for _, s in tensor_layout(dims_t))


def test_synthetic_is_seeded():
    a = prompts(4, 8, seed=0)
    b = prompts(4, 8, seed=0)
    np.testing.assert_array_equal(a, b)
    assert a.min() >= 0 and a.max() < 50257
    x = outlier_activations(16, 768, seed=1)
    big = np.abs(x).max(axis=0) > 10
    assert 1 <= big.sum() <= 8  # 1% of 768 channels scaled x20
