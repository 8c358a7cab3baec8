"""Python handle on the C host engine (include/gpt2_engine.h)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import EngineConfig, Request, W8A8Error, core
from .quant8 import GPT2Dims


class Engine:
    """Batched W8A8 GPT-2 on one GPU; all heavy work happens in native code."""

    def __init__(self, dims: GPT2Dims, max_batch: int, max_tokens: int | None = None,
                 device: int = 0):
        self.dims = dims
        self.max_batch = max_batch
        self.max_tokens = max_tokens or max_batch * dims.ctx
        self._cfg = EngineConfig(dims.d_model, dims.n_layer, dims.n_head, dims.vocab, dims.ctx,
                                 max_batch, self.max_tokens)
        h = C.c_void_p()
        st = core().gpt2_engine_create(C.byref(self._cfg), device, C.byref(h))
        if st != _lib.W8A8_OK:
            raise W8A8Error(st, "gpt2_engine_create")
        self._h = h

    # -- lifecycle ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            core().gpt2_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int, what: str) -> None:
        if st != _lib.W8A8_OK:
            msg = core().gpt2_engine_last_error(self._h)
            raise W8A8Error(st, f"{what} ({msg.decode() if msg else ''})")

    # -- weights -----------------------------------------------------------
    @property
    def quant8_bytes(self) -> int:
        return core().gpt2_engine_quant8_bytes(C.byref(self._cfg))

    def load_quant8(self, image) -> None:
        """image: bytes / numpy uint8 buffer in quant8.bin layout, or a path."""
        if isinstance(image, (str, os.PathLike)):
            self._check(core().gpt2_engine_load_quant8(self._h, os.fsencode(image)),
                        "gpt2_engine_load_quant8")
            return
        buf = np.frombuffer(image, dtype=np.uint8) if isinstance(image, bytes) else image
        buf = np.ascontiguousarray(buf)
        self._check(core().gpt2_engine_load_quant8_memory(self._h, buf.ctypes.data, buf.nbytes),
                    "gpt2_engine_load_quant8_memory")

    # -- generation --------------------------------------------------------
    def generate(self, prompts: np.ndarray, n_gen: int, out: np.ndarray | None = None
                 ) -> np.ndarray:
        """Host-buffer API: prompts [B, T] int32 -> generated ids [B, n_gen]
        (written into `out` when given, e.g. pinned memory)."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        B, T = p.shape
        if out is None:
            out = np.empty((B, n_gen), dtype=np.int32)
        if out.shape != (B, n_gen) or out.dtype != np.int32 or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous int32 [B, n_gen] array")
        self._check(core().gpt2_engine_generate(self._h, p.ctypes.data, B, T, n_gen,
                                                out.ctypes.data), "gpt2_engine_generate")
        return out

    def generate_device(self, prompts_d, n_gen: int, out_d, stream=None) -> None:
        """Device-buffer API (torch tensors): asynchronous on `stream`."""
        B, T = prompts_d.shape
        s = stream.cuda_stream if stream is not None else None
        self._check(core().gpt2_engine_generate_device(self._h, prompts_d.data_ptr(), B, T, n_gen,
                                                       out_d.data_ptr(), s),
                    "gpt2_engine_generate_device")

    def prefill(self, prompts_d, out_d, out_stride: int) -> None:
        B, T = prompts_d.shape
        self._check(core().gpt2_engine_prefill(self._h, prompts_d.data_ptr(), B, T,
                                               out_d.data_ptr(), out_stride),
                    "gpt2_engine_prefill")

    def decode_steps(self, steps: int) -> None:
        self._check(core().gpt2_engine_decode_steps(self._h, steps), "gpt2_engine_decode_steps")

    # -- continuous batching ------------------------------------------------
    def serve(self, requests: list[tuple], slots: int) -> list[np.ndarray]:
        """Serve (prompt ids, n_gen) or (prompt ids, n_gen, draws) requests over
        `slots` decode slots, admitted in order as slots free up
        (gpt2_engine_serve); draws (n_gen floats in [0, 1]) are used when top-k
        sampling is on. Returns each request's generated ids."""
        prompts = [np.ascontiguousarray(r[0], dtype=np.int32) for r in requests]
        outs = [np.zeros((r[1],), dtype=np.int32) for r in requests]
        draws = [np.ascontiguousarray(r[2], dtype=np.float32) if len(r) > 2 else None
                 for r in requests]
        for r, dr in zip(requests, draws):
            if dr is not None and dr.size != r[1]:
                raise ValueError("a request's draws must number its n_gen")
        reqs = (Request * len(requests))()
        for i, (r, p, o, dr) in enumerate(zip(requests, prompts, outs, draws)):
            reqs[i] = Request(p.ctypes.data, p.size, r[1], o.ctypes.data,
                              dr.ctypes.data if dr is not None else None)
        self._check(core().gpt2_engine_serve(self._h, reqs, len(requests), slots),
                    "gpt2_engine_serve")
        return outs

    def slots_begin(self, slots: int, out_d, out_stride: int) -> None:
        self._check(core().gpt2_engine_slots_begin(self._h, slots, out_d.data_ptr(), out_stride),
                    "gpt2_engine_slots_begin")

    def slot_prefill(self, slot: int, prompt_d) -> None:
        self._check(core().gpt2_engine_slot_prefill(self._h, slot, prompt_d.data_ptr(),
                                                    prompt_d.numel()),
                    "gpt2_engine_slot_prefill")

    def slot_release(self, slot: int) -> np.ndarray:
        """The slot's tokens so far; the slot is parked."""
        n = core().gpt2_engine_slot_tokens(self._h, slot)
        out = np.zeros((max(n, 0),), dtype=np.int32)
        self._check(core().gpt2_engine_slot_release(self._h, slot,
                                                    out.ctypes.data if n > 0 else None),
                    "gpt2_engine_slot_release")
        return out

    def slot_tokens(self, slot: int) -> int:
        return core().gpt2_engine_slot_tokens(self._h, slot)

    def logits(self, rows: int) -> np.ndarray:
        """bf16 logits of the last step as float32 [rows, vocab]."""
        raw = np.empty((rows, self.dims.vocab), dtype=np.uint16)
        self._check(core().gpt2_engine_copy_logits(self._h, raw.ctypes.data, rows),
                    "gpt2_engine_copy_logits")
        return (raw.astype(np.uint32) << 16).view(np.float32)

    def set_sampling(self, temperature: float, top_k: int = 40) -> None:
        """temperature <= 0: greedy (default); else top-k sampling at that temperature."""
        self._check(core().gpt2_engine_set_sampling(self._h, float(temperature), int(top_k)),
                    "gpt2_engine_set_sampling")

    def set_draws(self, slot: int, draws) -> None:
        """Slot `slot`'s draws in [0, 1], one per token from its first on."""
        d = np.ascontiguousarray(draws, dtype=np.float32)
        self._check(core().gpt2_engine_set_draws(self._h, slot, d.ctypes.data if d.size else None,
                                                 d.size), "gpt2_engine_set_draws")

    def set_decode_split(self, halves: int) -> None:
        """Decode steps as one chain over all slots (1) or two concurrent chains (2)."""
        self._check(core().gpt2_engine_set_decode_split(self._h, int(halves)),
                    "gpt2_engine_set_decode_split")

    @staticmethod
    def reference_draws(n: int, seed: int = 1) -> np.ndarray:
        """(float)rand() / RAND_MAX for n calls of glibc's rand() after srand(seed):
        the reference's draws (gpt2.c:2231; it never seeds: seed 1)."""
        out = np.zeros((n,), dtype=np.float32)
        st = core().gpt2_reference_draws(seed, out.ctypes.data if n else None, n)
        if st != _lib.W8A8_OK:
            raise ValueError(f"gpt2_reference_draws: status {st}")
        return out

    def set_graphs(self, enable: bool) -> None:
        self._check(core().gpt2_engine_set_graphs(self._h, 1 if enable else 0),
                    "gpt2_engine_set_graphs")

    @property
    def stream_handle(self) -> int:
        return core().gpt2_engine_stream(self._h)

    @property
    def launches_per_decode_step(self) -> int:
        return core().gpt2_engine_launches_per_decode_step(self._h)

    @property
    def launches_per_prefill(self) -> int:
        return core().gpt2_engine_launches_per_prefill(self._h)
