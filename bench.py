"""Benchmark: GPT-2 large W8A8 batched generation, data-parallel over GPUs.

Workload (the configuration the headline tok/s is quoted on at 1/2/4/8
GPUs): 64 independent sequences, each a 512-token random prompt followed by
512 greedy tokens (KV cache grows to 1023 rows), split data-parallel over the
GPUs of one node (64/N sequences per rank, strong scaling, no collective on
the data path). Weights: GPT-2 large architecture, random N(0, 0.02) init,
per-output-channel INT8 (synthetic; no checkpoint is available offline).

Outside the timed region, a second leg runs the GPT-2 large W8A8 prefill of
32 x 1024 tokens tensor-parallel over all ranks (`tp_prefill` in the JSON
line: device time, and bit-equality of its tokens and logits with the
single-GPU engine's prefill of the same batch).

One step = the whole job on a rank's shard: batched prefill of its prompts,
then 511 greedy decode steps (CUDA-graph replays). `value` = generated
tokens of all ranks / max-over-ranks device time (CUDA events on the
engine's stream); `e2e` = the same through the host-buffer API
(gpt2_engine_generate: pinned prompts in, generated ids out, per step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_SEQ, PROMPT, GEN = 64, 512, 512
METRIC = "GPT-2 W8A8 prefill & decode tok/s at 1/2/4/8 B200; INT8 GEMM % peak"
WORKLOAD = ("gpt2-large W8A8, 64 sequences x (512-token prompt + 512 greedy tokens), "
            "data-parallel over GPUs")
# CPU-baseline samples of one sequence of the same workload: the full
# 512-token prompt and the first 16 tokens of its generation (timed every
# step), and once a 1000-token prompt with 8 tokens, the context the
# generation ends at. The reference's CPU path recomputes the LM head over
# every row each step (gpt2.c:2168-2172), so its time per token grows with
# the context; the two samples bracket the 512 -> 1023 range.
REF_SAMPLE_GEN = 16
REF_LATE_PROMPT, REF_LATE_GEN = 1000, 8


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.seek(0)
        rows = [l.split(",") for l in self.f.read().strip().splitlines() if l.strip()]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_sample(dims, fp32_path: Path, prompt, n_gen: int) -> dict:
    """Time the reference's own CPU FP32 build on one sequence (rank 0)."""
    from oracle.ref_runner import run_reference
    r = run_reference("large", fp32_path, prompt, n_gen)
    perf = r["perf"]
    return {"value": n_gen / perf["total_seconds"], "ttft_s": perf["ttft_s"],
            "mean_tpot_s": perf["mean_tpot_s"], "threads": r["threads"]}


def reference_full_sequence(early: dict, late: dict) -> float:
    """tok/s of the reference on one whole sequence of the workload (512-token
    prompt + 512 tokens): the first token after the prefill (early sample's
    time to first token), then 511 tokens whose time per token grows linearly
    from the early sample's (context ~512) to the late sample's (~1000)."""
    per_token = 0.5 * (early["mean_tpot_s"] + late["mean_tpot_s"])
    return GEN / (early["ttft_s"] + (GEN - 1) * per_token)


def reference_late_sample(dims, fp32_path: Path) -> dict:
    from c_gpt2_b200.synthetic import prompts
    P = prompts(1, REF_LATE_PROMPT, dims.vocab, seed=1)[0]
    return reference_sample(dims, fp32_path, P, REF_LATE_GEN)


def reference_baseline(early: list[dict], late: dict) -> dict:
    """The cpu_baseline object from the early samples (median) and the late one."""
    e = {k: statistics.median(x[k] for x in early) for k in ("value", "ttft_s", "mean_tpot_s")}
    full = reference_full_sequence(e, late)
    sample = (f"one sequence of the workload: 512-token prompt + {REF_SAMPLE_GEN} greedy tokens "
              f"(median of {len(early)}: ttft {e['ttft_s']:.2f} s, {e['mean_tpot_s']:.3f} s per "
              f"token) and a {REF_LATE_PROMPT}-token prompt + {REF_LATE_GEN} tokens "
              f"({late['mean_tpot_s']:.3f} s per token); value = 512 tokens over the prefill plus "
              f"511 tokens at the mean of the two per-token times; reference gpt2.c FP32 CPU "
              f"build (OpenBLAS); {cpu_model()}")
    return {"value": round(full, 4), "unit": "tok/s", "cores": early[0]["threads"],
            "kind": "reference", "sample": sample,
            "early_sample_tok_s": round(e["value"], 4), "ttft_s": round(e["ttft_s"], 3),
            "tpot_s_ctx512": round(e["mean_tpot_s"], 4),
            "tpot_s_ctx1000": round(late["mean_tpot_s"], 4)}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_arm(args, rank: int, world: int) -> None:
    """--impl reference: the reference's own CPU implementation of the path
    (gpt2.c FP32, OpenBLAS, all host threads) on a bounded sample of the same
    workload; rank 0 alone runs and prints."""
    if rank != 0:
        return
    from c_gpt2_b200.quant8 import DIMS
    from c_gpt2_b200.synthetic import prompts, write_weight_files
    from oracle.ref_runner import ref_binary
    if not ref_binary("large").exists():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/gpt2_ref_large not built "
                                         "(make -C oracle ref needs the reference tree)"}))
        return
    dims = DIMS["large"]
    P = prompts(N_SEQ, PROMPT, dims.vocab, seed=0)
    with tempfile.TemporaryDirectory() as td:
        f32 = Path(td) / "large_fp32.bin"
        _write_fp32(dims, f32)
        for _ in range(args.warmup):
            reference_sample(dims, f32, P[0], REF_SAMPLE_GEN)
        t0 = time.perf_counter()
        vals = [reference_sample(dims, f32, P[0], REF_SAMPLE_GEN) for _ in range(args.steps)]
        t_steps = time.perf_counter() - t0
        late = reference_late_sample(dims, f32)
    cpu = reference_baseline(vals, late)
    v = cpu["value"]
    out = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(1000 * t_steps / args.steps, 2), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "impl": "reference", "config": workload_config(args.gpus, args.decode_split),
           "cpu_baseline": cpu,
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def workload_config(world: int, decode_split: int = 1) -> dict:
    return {"workload": WORKLOAD, "model": "gpt2-large", "n_seq": N_SEQ,
            "prompt_len": PROMPT, "gen_len": GEN, "seq_per_gpu": N_SEQ // world,
            "parallelism": f"dp{world}", "decode_chains": decode_split,
            "l2": "inputs larger than L2 (929 MB weights + 12 GB KV cache per step)"}


def _write_fp32(dims, path: Path) -> None:
    import torch
    if torch.cuda.is_available():
        from c_gpt2_b200.synthetic import quant8_image_gpu
        quant8_image_gpu(dims, 0, "cuda", fp32_path=path)
    else:
        from c_gpt2_b200.synthetic import write_weight_files
        write_weight_files(dims, 0, fp32_path=path)


def time_kernel(fn, iters: int, stream) -> float:
    """Average milliseconds of `fn` over `iters` launches (CUDA events on `stream`)."""
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


# DRAM bytes of one decode-attention launch (64 sequences, 20 heads, 768
# cached positions) measured with ncu: 251.85 MB read + 4.59 MB written,
# against 251.7 MB of K/V rows the kernel must read.
ATTN_DRAM_BYTES_B64 = 251_846_144 + 4_593_408


def kernel_rooflines(count: int, peaks: dict, dev) -> dict:
    """The dominant kernels of one step, timed alone at the workload's shapes.

    decode attention (both launches of one layer's call): B = this rank's
    sequences, 20 heads, 768 cached keys each (the mean context over the
    512-token decode phase). Algorithmic bytes = K and V rows read + q + o.

    prefill INT8 GEMM: the MLP up-projection of GPT-2 large over this rank's
    B x 512 prompt tokens (N = 5120, K = 1280), 2*M*N*K operations; and the
    four prefill GEMMs of a layer together (W_qkv with the bias epilogue,
    attn_proj and W2 with bias + residual, W1 with bias + GELU), each timed
    alone, reported as their summed operations over their summed times.
    """
    import torch
    from c_gpt2_b200 import _lib, ops
    H, C, hd, d = 20, 1024, 64, 1280
    n = 768
    B = count
    stream = torch.cuda.current_stream()
    K = torch.randn((B, C, d), device=dev).to(torch.bfloat16)
    V = torch.randn((B, C, d), device=dev).to(torch.bfloat16)
    q = torch.randn((B, d), device=dev).to(torch.bfloat16)
    o = torch.empty((B, d), dtype=torch.bfloat16, device=dev)
    nctx = torch.full((B,), n, dtype=torch.int32, device=dev)
    ws = torch.zeros((_lib.core().w8a8_attention_decode_workspace_size(B, H, C),),
                     dtype=torch.uint8, device=dev)
    ms = time_kernel(lambda: ops.attention_decode(q, K, V, C * d, nctx, C, H, out=o,
                                                  workspace=ws), 50, stream)
    attn_bytes = B * H * n * hd * 2 * 2 + 2 * B * d * 2
    attn_gbs = attn_bytes / (ms * 1e-3) / 1e9
    del K, V
    M, N, Kd = B * PROMPT, 5120, 1280
    xq = torch.randint(-127, 128, (M, Kd), dtype=torch.int8, device=dev)
    W = torch.randint(-127, 128, (N, Kd), dtype=torch.int8, device=dev)
    sx = torch.rand((M,), device=dev) * 0.01 + 1e-3
    sw = torch.rand((N,), device=dev) * 0.01 + 1e-3
    b = (torch.randn((N,), device=dev) * 0.02).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    gms = time_kernel(lambda: ops.linear(xq, sx, W, sw, b, _lib.EPI_BIAS_GELU, out=y), 20, stream)
    tops = 2.0 * M * N * Kd / (gms * 1e-3) / 1e12
    int8_peak = 2.0 * peaks["bf16_tflops"]
    del xq, W, y
    # the other three prefill GEMMs of a layer, each with inputs beyond L2
    per = {"w1": (round(gms, 4), 2.0 * M * N * Kd)}
    for name, n_out, k_in, epi in (("w_qkv", 3 * d, d, _lib.EPI_BIAS),
                                   ("attn_proj", d, d, _lib.EPI_BIAS_RESID),
                                   ("w2", d, 4 * d, _lib.EPI_BIAS_RESID)):
        x_ = torch.randint(-127, 128, (M, k_in), dtype=torch.int8, device=dev)
        w_ = torch.randint(-127, 128, (n_out, k_in), dtype=torch.int8, device=dev)
        sw_ = torch.rand((n_out,), device=dev) * 0.01 + 1e-3
        b_ = (torch.randn((n_out,), device=dev) * 0.02).to(torch.bfloat16)
        r_ = (torch.randn((M, n_out), device=dev).to(torch.bfloat16)
              if epi == _lib.EPI_BIAS_RESID else None)
        y_ = torch.empty((M, n_out), dtype=torch.bfloat16, device=dev)
        t_ = time_kernel(lambda: ops.linear(x_, sx, w_, sw_, b_, epi, R=r_, out=y_), 20, stream)
        per[name] = (round(t_, 4), 2.0 * M * n_out * k_in)
        del x_, w_, r_, y_
    all_ms = sum(t for t, _ in per.values())
    all_tops = sum(o for _, o in per.values()) / (all_ms * 1e-3) / 1e12
    return {
        "attention": {"ms": ms, "bytes": attn_bytes, "gbs": attn_gbs, "seqs": B},
        "gemm": {"workload": f"W1 prefill GEMM M={M} N={N} K={Kd} (+dequant, bias, GELU)",
                 "ms": round(gms, 4), "tops": round(tops, 1),
                 "peak_tops": round(int8_peak, 1),
                 "peak_note": f"2 x {peaks['source']} bf16 dense (INT8 runs the tensor pipe "
                              "at twice the bf16 rate)",
                 "frac": round(tops / int8_peak, 4)},
        "gemm_layer": {"workload": f"the four prefill GEMMs of one GPT-2 large layer at M={M} "
                                   "(W_qkv bias, attn_proj bias+residual, W1 bias+GELU, "
                                   "W2 bias+residual), each timed alone",
                       "ms": round(all_ms, 4), "tops": round(all_tops, 1),
                       "frac": round(all_tops / int8_peak, 4),
                       "ms_per_gemm": {k: t for k, (t, _) in per.items()}},
    }


# Tensor-parallel prefill leg (GPT-2 large, 32 prompts x 1024 tokens, split
# over every rank of the run).
TP_SEQ, TP_TOK = 32, 1024


def tp_prefill_leg(args, rank: int, world: int, local: int, dev) -> dict | None:
    """GPT-2 large W8A8 prefill of 32 x 1024 tokens, tensor-parallel over the
    run's ranks (W_qkv and W1 column-split; attn_proj and W2 over each rank's
    own sequences with the whole K, their int8 inputs brought by one NCCL
    all-to-all each; int8 all-gather of the LayerNorm rows, fp32 max
    all-reduce of the row maxima), timed
    on the device (max over ranks), and its next tokens and logits compared
    bit for bit with the single-GPU engine's prefill of the same batch, which
    rank 0 also times. Every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist
    from c_gpt2_b200.dp import max_over_ranks
    from c_gpt2_b200.engine import Engine
    from c_gpt2_b200.quant8 import DIMS, read_quant8
    from c_gpt2_b200.synthetic import prompts, quant8_image_gpu
    from c_gpt2_b200.tp import TPPlan, TPPrefill, shard_weights

    dims = DIMS["large"]
    img = quant8_image_gpu(dims, seed=0, device=dev)
    P = torch.from_numpy(prompts(TP_SEQ, TP_TOK, dims.vocab, seed=0)).to(dev)
    plan = TPPlan.make(dims, world)
    shard = shard_weights(read_quant8(img, dims), plan, rank, dev)
    tp = TPPrefill(plan, shard, rank)
    for _ in range(args.warmup):
        tp.run(P)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        nxt, logits = tp.run(P)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    full = logits
    if world > 1:
        full = torch.empty((TP_SEQ, dims.vocab), dtype=logits.dtype, device=dev)
        dist.all_gather_into_tensor(full, logits.contiguous())
    tp.close()
    del shard, tp
    out = None
    if rank == 0:
        eng = Engine(dims, max_batch=TP_SEQ, max_tokens=TP_SEQ * TP_TOK, device=local)
        eng.load_quant8(img)
        one = torch.empty((TP_SEQ,), dtype=torch.int32, device=dev)
        es = torch.cuda.ExternalStream(eng.stream_handle, device=dev)
        for _ in range(args.warmup):
            eng.prefill(P, one, 1)
        torch.cuda.synchronize()
        e0.record(es)
        for _ in range(args.steps):
            eng.prefill(P, one, 1)
        e1.record(es)
        torch.cuda.synchronize()
        ms1 = e0.elapsed_time(e1) / args.steps
        want = eng.logits(TP_SEQ)
        eng.close()
        got = (full.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
               .astype(np.uint32) << 16).view(np.float32)
        same_tok = bool(np.array_equal(nxt.cpu().numpy(), one.cpu().numpy()))
        same_logits = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
        M = TP_SEQ * TP_TOK
        gemm_ops = 2.0 * M * 12 * dims.d_model ** 2 * dims.n_layer
        out = {"workload": f"gpt2-large W8A8 prefill {TP_SEQ} x {TP_TOK} tokens, "
                           f"tensor-parallel tp{world} (heads per rank "
                           f"{[h1 - h0 for h0, h1 in plan.heads]})",
               "tp": world, "ms": round(ms, 3), "tok_per_s": round(M / (ms / 1e3), 1),
               "gemm_tops_effective": round(gemm_ops / (ms / 1e3) / 1e12, 1),
               "ms_1gpu_engine": round(ms1, 3), "vs_1gpu": round(ms1 / ms, 3),
               "bitexact": same_tok and same_logits, "tokens_equal": same_tok,
               "logits_equal": same_logits,
               "exchange": "int8 all-to-all to the rows' owners + int8 all-gather + fp32 max "
                           "all-reduce (NCCL)"}
    if world > 1:
        dist.barrier()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp-prefill", action="store_true",
                    help="skip the tensor-parallel 32 x 1024 prefill leg")
    ap.add_argument("--decode-split", type=int, choices=[1, 2], default=1,
                    help="decode each step as one chain of kernels or two concurrent chains")
    args = ap.parse_args()

    from c_gpt2_b200.dp import dist_env, max_over_ranks, shard
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from c_gpt2_b200 import ops
    from c_gpt2_b200.engine import Engine
    from c_gpt2_b200.quant8 import DIMS
    from c_gpt2_b200.synthetic import prompts, quant8_image_gpu

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)
    ops.init(local)
    peaks = load_peaks()
    dims = DIMS["large"]
    first, count = shard(N_SEQ, rank, world)
    img = quant8_image_gpu(dims, seed=0, device=dev)
    eng = Engine(dims, max_batch=count, max_tokens=count * PROMPT, device=local)
    eng.load_quant8(img)
    eng.set_decode_split(args.decode_split)
    del img
    P = prompts(N_SEQ, PROMPT, dims.vocab, seed=0)[first:first + count]
    pd = torch.from_numpy(np.ascontiguousarray(P)).to(dev)
    out = torch.empty((count, GEN), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        eng.generate_device(pd, GEN, out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        eng.generate_device(pd, GEN, out)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_step = max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    value = N_SEQ * GEN / (ms_step / 1e3)
    assert ops.device_error(reset=True) == 0

    # e2e through the host-buffer API: pinned prompts in, generated ids out
    Ph = torch.from_numpy(np.ascontiguousarray(P)).pin_memory().numpy()
    Oh = torch.empty((count, GEN), dtype=torch.int32).pin_memory().numpy()
    for _ in range(min(args.warmup, 1)):
        eng.generate(Ph, GEN, out=Oh)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.generate(Ph, GEN, out=Oh)
    t_e2e = (time.perf_counter() - t0) / args.steps
    barrier()
    t_e2e = max_over_ranks(t_e2e, dev)
    e2e = N_SEQ * GEN / t_e2e
    launches = args.steps * (eng.launches_per_prefill + (GEN - 1) * eng.launches_per_decode_step)
    eng.close()

    roof = kernel_rooflines(count, peaks, dev)
    achieved = roof["attention"]["gbs"]
    tp_line = None if args.no_tp_prefill else tp_prefill_leg(args, rank, world, local, dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle.ref_runner import ref_binary
            if ref_binary("large").exists():
                with tempfile.TemporaryDirectory() as td:
                    f32 = Path(td) / "large_fp32.bin"
                    quant8_image_gpu(dims, 0, dev, fp32_path=f32)
                    early = reference_sample(dims, f32, P[0], REF_SAMPLE_GEN)
                    late = reference_late_sample(dims, f32)
                cpu = reference_baseline([early], late)
        except Exception as exc:  # the baseline is reported, not required
            cpu = {"value": None, "error": str(exc)[:200]}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": workload_config(world, args.decode_split),
            "e2e": {"value": round(e2e, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(count * PROMPT * 4),
                    "d2h_bytes_per_step": int(count * GEN * 4)},
            "roofline": {"bound": "hbm", "kernel": "decode attention (scores + P.V, one layer)",
                         "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "traffic": round(ATTN_DRAM_BYTES_B64 * roof["attention"]["seqs"] / 64),
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum per launch "
                                         "from one ncu capture at 64 sequences x 20 heads x 768 "
                                         "positions, scaled by sequences per GPU",
                         "algorithmic_bytes": int(roof["attention"]["bytes"]),
                         "peak_source": peaks["source"]},
            "gemm": roof["gemm"],
            "gemm_layer": roof["gemm_layer"],
            "tp_prefill": tp_line,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": int(launches),
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
