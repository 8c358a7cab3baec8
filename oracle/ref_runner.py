"""Run the reference's own CPU FP32 build (oracle/_ref/gpt2_ref_<size>), and
the GPU builds of its gpt2.c (the reference's INT8 GPU build, and gpt2.c on
this repository's library), on seeded synthetic weights and prompt ids. TEST
INFRASTRUCTURE ONLY: used by tests/, the smoke check, c_gpt2_b200.profcase's
reference legs and bench.py's CPU-baseline leg as the checker and baseline,
never by the product path.

The reference reads weights from the relative path weights/<file>
(include/model_config.h:14,22,30) and tokenizes over TCP 127.0.0.1:65432
(gpt2.c:26-27, 198-235). A fake tokenizer answers `encode` with the seeded
prompt ids and records the ids of the final `decode` request — the greedy
stream (gpt2.c:2311-2325).
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
PORT = 65432
WEIGHT_FILES = {"small": "gpt2_c_weights.bin", "medium": "gpt2_medium_c_weights.bin",
                "large": "gpt2_large_c_weights.bin"}
# the INT8 GPU builds read the quant8.bin instead (include/model_config.h:15,23,31)
QUANT8_FILES = {"small": "gpt2_small_quant8.bin", "medium": "gpt2_medium_quant8.bin",
                "large": "gpt2_large_quant8.bin"}
# GPU builds of gpt2.c (oracle/Makefile):
#   gpu_int8    the reference's INT8 GPU build: its cuda/*.cu kernels + cuBLAS
#   ourkernels  the same gpt2.c object on this repository's libcuda_kernels
#   dropin      gpt2.c with its GPU layer and pick on this repository's entry
#               points (no cuBLAS)
GPU_BUILDS = {"gpu_int8": "gpt2_gpu_int8_{}", "ourkernels": "gpt2_gpu_ourkernels_{}",
              "dropin": "gpt2_dropin_{}"}


def ref_binary(size: str) -> Path:
    return REF_DIR / f"gpt2_ref_{size}"


def gpu_binary(build: str, size: str) -> Path:
    return REF_DIR / GPU_BUILDS[build].format(size)


class FakeTokenizer:
    """Single-connection-at-a-time JSON server with the reference's protocol
    (tokenizer.py: one request per connection, reply, close)."""

    def __init__(self, prompt_ids):
        self.prompt_ids = [int(t) for t in prompt_ids]
        self.decodes: list[list[int]] = []
        self._sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self._sock.bind(("127.0.0.1", PORT))
        self._sock.listen(8)
        self._stop = False
        self._t = threading.Thread(target=self._serve, daemon=True)
        self._t.start()

    def _serve(self):
        while not self._stop:
            try:
                conn, _ = self._sock.accept()
            except OSError:
                return
            with conn:
                buf = b""
                req = None
                while len(buf) < 1 << 20:
                    chunk = conn.recv(65536)
                    if not chunk:
                        break
                    buf += chunk
                    try:
                        req = json.loads(buf.decode())
                        break
                    except ValueError:
                        continue
                if req is None:
                    continue
                if req.get("mode") == "encode":
                    resp = {"tokens": self.prompt_ids}
                else:
                    toks = [int(t) for t in req.get("tokens", [])]
                    self.decodes.append(toks)
                    resp = {"text": " ".join(map(str, toks))}
                conn.sendall(json.dumps(resp).encode())

    def close(self):
        self._stop = True
        try:
            self._sock.shutdown(socket.SHUT_RDWR)  # wakes the blocked accept()
        except OSError:
            pass
        try:
            self._sock.close()
        except OSError:
            pass
        self._t.join(timeout=5)


def run_reference(size: str, fp32_weights: Path, prompt_ids, n_gen: int,
                  dump_logits_row: int | None = None, threads: int | None = None,
                  timeout: float = 3600.0) -> dict:
    """Run the reference's CPU FP32 build once; returns {"tokens", "perf",
    "logits", "wall_s"}."""
    return _run(ref_binary(size), WEIGHT_FILES[size], fp32_weights, prompt_ids, n_gen,
                dump_logits_row, threads, timeout)


def run_gpu_build(build: str, size: str, quant8_weights: Path, prompt_ids, n_gen: int,
                  temperature: float = 0.0, top_k: int = 40, timeout: float = 1800.0) -> dict:
    """Run one GPU build of gpt2.c (GPU_BUILDS) on a quant8.bin; returns
    {"tokens", "perf", "wall_s"}. At temperature > 0 the reference draws with
    its own unseeded rand()."""
    return _run(gpu_binary(build, size), QUANT8_FILES[size], quant8_weights, prompt_ids, n_gen,
                None, None, timeout, temperature=temperature, top_k=top_k)


def _run(exe: Path, weight_name: str, weights: Path, prompt_ids, n_gen: int,
         dump_logits_row: int | None, threads: int | None, timeout: float,
         temperature: float = 0.0, top_k: int | None = None) -> dict:
    if not exe.exists():
        raise FileNotFoundError(f"{exe} missing: run `make -C oracle ref`")
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        (td / "weights").mkdir()
        os.symlink(Path(weights).resolve(), td / "weights" / weight_name)
        (td / "logs").mkdir()
        env = dict(os.environ)
        n = threads or os.cpu_count() or 1
        env["OPENBLAS_NUM_THREADS"] = str(n)
        cmd = [str(exe)]
        if dump_logits_row is not None:
            cmd += ["--dump-logits", str(td / "logits.f32"), str(dump_logits_row)]
        cmd += ["--prompt", "synthetic prompt", "--temperature", repr(float(temperature)),
                "--no-stream", "--req_out_tokens", str(n_gen),
                "--json_out_file", str(td / "perf.json")]
        if top_k is not None:
            cmd += ["--top_k", str(top_k)]
        tok = FakeTokenizer(prompt_ids)
        try:
            t0 = time.perf_counter()
            r = subprocess.run(cmd, cwd=td, env=env, capture_output=True, text=True,
                               timeout=timeout)
            wall = time.perf_counter() - t0
        finally:
            tok.close()
        if r.returncode != 0:
            raise RuntimeError(f"reference exited {r.returncode}: {r.stderr[-2000:]}")
        perf = json.loads((td / "perf.json").read_text())
        logits = None
        if dump_logits_row is not None:
            logits = np.fromfile(td / "logits.f32", dtype=np.float32)
        if not tok.decodes:
            raise RuntimeError("reference made no decode request")
        return {"tokens": np.array(tok.decodes[-1], dtype=np.int32), "perf": perf,
                "logits": logits, "wall_s": wall, "threads": n}
