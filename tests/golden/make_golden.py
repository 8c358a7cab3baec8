"""Regenerate the golden fixtures of tests/golden/ from the reference itself.

Runs only where the reference tree is mounted (its root in the REF_ROOT
environment variable); the tests read the fixtures it wrote and never run it.
Outputs:

  weight_quant.npz    the reference's per-channel quantizer
                      (tools/offline_quant/src/quantizer.py:52-64) applied to
                      seeded FP32 matrices, including edge cases (zero row,
                      exact .5 ties, a single large outlier)
  quant8_tiny.json    SHA-256 and size of the quant8.bin the reference's
                      writer (tools/offline_quant/src/writer.py:50-69)
                      produces for tiny seeded weights
  quant8_manifests.json  the text of the quant8.json manifest the reference's
                      writer (tools/offline_quant/src/writer.py:99-124) writes
                      for GPT-2 small / medium / large and the tiny model
                      (it depends on tensor sizes only: zero-filled tensors)
  ref_fp32_small.npz  the reference's CPU FP32 build (oracle/_ref, gpt2.c)
                      on GPT-2 small, seed-0 weights, a 32-token prompt of
                      seed-0 ids: the 64-token greedy stream and the logits
                      of the last prompt position (fp16)

usage: python tests/golden/make_golden.py [--skip-ref-run]
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF_ROOT = Path(os.environ.get("REF_ROOT", "/root/reference"))
sys.path.insert(0, str(ROOT))

TINY = dict(d_model=64, n_layer=2, n_head=1, vocab=100, ctx=16)
SEED = 0


def reference_quant_modules():
    sys.path.insert(0, str(REF_ROOT / "tools" / "offline_quant"))
    from src import quantizer, reader, writer  # noqa: E402  (the reference's own modules)
    return quantizer, reader, writer


def weight_quant_cases() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(1234)
    cases = {
        "normal": (rng.standard_normal((48, 96), dtype=np.float32) * np.float32(0.02)),
        "outlier": rng.standard_normal((16, 64), dtype=np.float32),
    }
    cases["outlier"][3, 7] = np.float32(40.0)
    z = rng.standard_normal((8, 32), dtype=np.float32)
    z[2, :] = 0.0
    cases["zero_row"] = z
    # rows whose values sit exactly on .5 multiples of the scale: amax 127
    # gives scale 1, so x/scale = x and rint's ties-to-even decides
    ties = np.tile(np.arange(-6.5, 6.5, 0.5, dtype=np.float32), (4, 1))
    ties[:, 0] = 127.0
    cases["ties"] = ties
    return cases


def make_weight_quant(quantizer) -> None:
    out = {}
    for name, W in weight_quant_cases().items():
        qt = quantizer.quantize_per_channel(np.ascontiguousarray(W))
        out[f"{name}.W"] = W
        out[f"{name}.int8"] = qt.int8
        out[f"{name}.scale"] = qt.scale
    np.savez_compressed(HERE / "weight_quant.npz", **out)


def make_quant8_tiny(quantizer, reader, writer) -> None:
    from c_gpt2_b200.quant8 import GPT2Dims
    from c_gpt2_b200.synthetic import iter_fp32_weights

    dims = GPT2Dims(**TINY)
    t = dict(iter_fp32_weights(dims, SEED))
    cfg = reader.ModelConfig("tiny", dims.d_model, dims.n_layer, dims.n_head, "tiny.bin")
    layers = []
    for l in range(dims.n_layer):
        p = f"h{l}."
        layers.append(reader.Layer(
            ln1_gamma=t[p + "ln1_gamma"], ln1_beta=t[p + "ln1_beta"], W_qkv=t[p + "W_qkv"],
            b_qkv=t[p + "b_qkv"], attn_proj=t[p + "attn_proj"],
            attn_proj_bias=t[p + "attn_proj_bias"], ln2_gamma=t[p + "ln2_gamma"],
            ln2_beta=t[p + "ln2_beta"], W1=t[p + "W1"], b1=t[p + "b1"], W2=t[p + "W2"],
            b2=t[p + "b2"]))
    w = reader.Weights(config=cfg, wte=t["wte"], wpe=t["wpe"], layers=layers,
                       lnf_gamma=t["lnf_gamma"], lnf_beta=t["lnf_beta"])
    qw = quantizer.quantize_weights(w)
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "tiny_quant8.bin"
        writer.write_bin(qw, path)
        data = path.read_bytes()
    meta = {"dims": TINY, "seed": SEED, "bytes": len(data),
            "sha256": hashlib.sha256(data).hexdigest(),
            "generator": "c_gpt2_b200.synthetic.iter_fp32_weights",
            "writer": "reference tools/offline_quant/src/writer.py write_bin"}
    (HERE / "quant8_tiny.json").write_text(json.dumps(meta, indent=2) + "\n")


def make_quant8_manifests(quantizer, reader, writer) -> None:
    def zeros_weights(cfg, vocab, ctx):
        d, f = cfg.d_model, 4 * cfg.d_model
        z = lambda *shape: np.zeros(shape, np.float32)
        qt = lambda o, i: quantizer.QuantizedTensor(int8=np.zeros((o, i), np.int8), scale=z(o))
        layers = [quantizer.QuantizedLayer(
            ln1_gamma=z(d), ln1_beta=z(d), W_qkv=qt(3 * d, d), b_qkv=z(3 * d),
            attn_proj=qt(d, d), attn_proj_bias=z(d), ln2_gamma=z(d), ln2_beta=z(d),
            W1=qt(f, d), b1=z(f), W2=qt(d, f), b2=z(d)) for _ in range(cfg.num_layers)]
        return quantizer.QuantizedWeights(config=cfg, wte=z(vocab, d), wpe=z(ctx, d),
                                          layers=layers, lnf_gamma=z(d), lnf_beta=z(d))

    out = {}
    cases = [(name, cfg, reader.VOCAB_SIZE, reader.CTX_LEN)
             for name, cfg in reader.MODEL_CONFIGS.items()]
    cases.append(("tiny", reader.ModelConfig("tiny", TINY["d_model"], TINY["n_layer"],
                                             TINY["n_head"], "tiny.bin"),
                  TINY["vocab"], TINY["ctx"]))
    for name, cfg, vocab, ctx in cases:
        buf = io.StringIO()  # as writer.write_quantized writes the file (writer.py:120-122)
        json.dump(writer.build_manifest(zeros_weights(cfg, vocab, ctx)), buf, indent=2)
        buf.write("\n")
        out[name] = buf.getvalue()
    (HERE / "quant8_manifests.json").write_text(json.dumps(out, indent=1) + "\n")


def make_ref_fp32_small() -> None:
    from c_gpt2_b200.quant8 import DIMS
    from c_gpt2_b200.synthetic import prompts, write_weight_files
    sys.path.insert(0, str(ROOT))
    from oracle.ref_runner import run_reference

    dims = DIMS["small"]
    T, n_gen = 32, 64
    ids = prompts(1, T, dims.vocab, SEED)[0]
    with tempfile.TemporaryDirectory() as td:
        f32 = Path(td) / "small.bin"
        write_weight_files(dims, SEED, fp32_path=f32)
        stream = run_reference("small", f32, ids, n_gen)
        pre = run_reference("small", f32, ids, 1, dump_logits_row=T - 1)
    np.savez_compressed(HERE / "ref_fp32_small.npz", prompt=ids, tokens=stream["tokens"],
                        prefill_logits=pre["logits"].astype(np.float16),
                        first_token=pre["tokens"])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-ref-run", action="store_true")
    args = ap.parse_args()
    quantizer, reader, writer = reference_quant_modules()
    make_weight_quant(quantizer)
    make_quant8_tiny(quantizer, reader, writer)
    make_quant8_manifests(quantizer, reader, writer)
    if not args.skip_ref_run:
        make_ref_fp32_small()


if __name__ == "__main__":
    main()
