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


# ---- the quant8.json manifest (tools/offline_quant/src/writer.py:72-124) ----

MANIFESTS = json.loads((GOLDEN / "quant8_manifests.json").read_text())
TINY_GOLDEN = GPT2Dims(d_model=64, n_layer=2, n_head=1, vocab=100, ctx=16)


def _manifest_cases():
    from c_gpt2_b200 import quant8
    yield "small", DIMS["small"], quant8.build_manifest(DIMS["small"])
    yield "medium", DIMS["medium"], quant8.build_manifest(DIMS["medium"])
    yield "large", DIMS["large"], quant8.build_manifest(DIMS["large"])
    yield "tiny", TINY_GOLDEN, quant8.build_manifest(TINY_GOLDEN, "tiny", "tiny.bin")


def test_manifest_matches_reference_writer(tmp_path):
    """The text the reference's writer writes, byte for byte."""
    from c_gpt2_b200 import quant8
    for name, dims, m in _manifest_cases():
        assert quant8.manifest_text(m) == MANIFESTS[name], name
        quant8.check_manifest(json.loads(MANIFESTS[name]), dims)
    path = tmp_path / "gpt2_large_quant8.json"
    quant8.write_manifest(path, DIMS["large"])
    assert path.read_text() == MANIFESTS["large"]


def _spoiled(text):
    """Manifests that must be refused: one field changed each."""
    m = json.loads(text)
    out = []
    for key, value in (("scheme", "int8_per_tensor"), ("scale_convention", "amax/128"),
                       ("scale_dtype", "fp16")):
        out.append({**m, key: value})
    out.append({**m, "quantized_tensors": m["quantized_tensors"][::-1]})
    out.append({**m, "preserved_tensors": m["preserved_tensors"][:-1]})
    ms = dict(m["memory_summary"])
    ms["scale_overhead_kb"] += 1
    out.append({**m, "memory_summary": ms})
    return out


def test_manifest_check_refuses_mismatches():
    from c_gpt2_b200 import quant8
    for m in _spoiled(MANIFESTS["large"]):
        with pytest.raises(ValueError):
            quant8.check_manifest(m, DIMS["large"])
    with pytest.raises(ValueError):  # a small model's manifest for the large model
        quant8.check_manifest(json.loads(MANIFESTS["small"]), DIMS["large"])
    with pytest.raises(ValueError):
        quant8.check_manifest({**json.loads(MANIFESTS["large"]), "model": "gpt2-xl"},
                              DIMS["large"])


def test_engine_manifest_check_in_c():
    """gpt2_quant8_check_manifest (the engine loader's check; host code only)."""
    import ctypes as C
    from c_gpt2_b200._lib import EngineConfig, W8A8_ERR_INVALID, W8A8_OK, core

    def check(dims, text):
        cfg = EngineConfig(dims.d_model, dims.n_layer, dims.n_head, dims.vocab, dims.ctx, 1, 1)
        err = C.create_string_buffer(160)
        st = core().gpt2_quant8_check_manifest(C.byref(cfg), text.encode(), err, 160)
        return st, err.value.decode()

    for name, dims, _ in _manifest_cases():
        assert check(dims, MANIFESTS[name]) == (W8A8_OK, ""), name
    for m in _spoiled(MANIFESTS["large"]):
        st, why = check(DIMS["large"], json.dumps(m, indent=2))
        assert st == W8A8_ERR_INVALID and why
    assert check(DIMS["large"], MANIFESTS["small"])[0] == W8A8_ERR_INVALID
    assert check(DIMS["large"], MANIFESTS["large"].replace("gpt2-large", "gpt2-xl"))[0] \
        == W8A8_ERR_INVALID
    assert check(DIMS["large"], "{}")[0] == W8A8_ERR_INVALID


def test_engine_manifest_check_any_json_layout():
    """The C check reads the fields wherever json.dump puts them: compact
    separators, reordered keys and CRLF line ends are the same manifest;
    an escaped string is refused rather than misread."""
    import ctypes as C
    from c_gpt2_b200._lib import EngineConfig, W8A8_ERR_INVALID, W8A8_OK, core

    dims = DIMS["medium"]
    cfg = EngineConfig(dims.d_model, dims.n_layer, dims.n_head, dims.vocab, dims.ctx, 1, 1)
    m = json.loads(MANIFESTS["medium"])
    texts = [json.dumps(m, separators=(",", ":")),
             json.dumps(dict(reversed(list(m.items()))), indent=4),
             MANIFESTS["medium"].replace("\n", "\r\n")]
    for t in texts:
        assert core().gpt2_quant8_check_manifest(C.byref(cfg), t.encode(), None, 0) == W8A8_OK
    bad = MANIFESTS["medium"].replace('"amax/127"', '"amax\\/127"')
    assert core().gpt2_quant8_check_manifest(C.byref(cfg), bad.encode(), None, 0) \
        == W8A8_ERR_INVALID
