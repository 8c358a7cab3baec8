"""Single-kernel cases for profiling: one kernel of the decode/prefill path on
seeded synthetic inputs, launched a few times and nothing else, so that a
profiler capture (`ncu -k <kernel> -c 1..3`) sees exactly that kernel at the
size of the large model (d_model 1280, 20 heads, context 1024).

    python -m c_gpt2_b200.profcase attention-decode [--batch 64] [--n-ctx 768]
    python -m c_gpt2_b200.profcase attention-prefill [--seqs 64] [--tokens 512]
    python -m c_gpt2_b200.profcase layernorm-quant [--m 32768] [--d 1280]
    python -m c_gpt2_b200.profcase quant-rows [--m 32768] [--k 5120]
    python -m c_gpt2_b200.profcase linear --m 32768 --n 5120 --k 1280 --epi gelu
    python -m c_gpt2_b200.profcase linear --m 64 --n 5120 --k 1280 --epi gelu
    python -m c_gpt2_b200.profcase decode [--model medium] [--batch 1] [--prompt 512] [--gen 256]
    python -m c_gpt2_b200.profcase gemv-chain [--model large] [--layers 36]
    python -m c_gpt2_b200.profcase mlp-pair [--model large] [--m 64] [--layers 36]
    python -m c_gpt2_b200.profcase sample [--rows 64] [--top-k 40] [--temperature 0.8]

Every case holds well under 1 GB on the device and exceeds the 126 MB L2 only
where the workload itself does (the attention KV cache, the prefill
activations, the weights of the GEMV chain). Prints one line with the
CUDA-event time per launch, measured after the profiled launches.
"""
from __future__ import annotations

import argparse
import ctypes

import torch

from . import _lib, ops

EPI = {"dequant": _lib.EPI_DEQUANT, "bias": _lib.EPI_BIAS, "resid": _lib.EPI_BIAS_RESID,
       "gelu": _lib.EPI_BIAS_GELU}


_FLUSH = None


def _graph(fn, reps: int, flush: bool):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            if flush:
                torch.amax(_FLUSH)
            if fn is not None:
                fn()
    return g


def _replay_ms(g) -> float:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g.replay()
    torch.cuda.synchronize()
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def _time(fn, reps: int) -> float:
    """Mean microseconds per launch on the device: the launches are captured
    in a CUDA graph and replayed, so no host launch overhead falls between
    them. With --flush every launch follows a 256 MB read that evicts the
    126 MB L2 (a read leaves no dirty lines to be written back during the
    launch), and the time of a graph of the reads alone is subtracted."""
    flush = _FLUSH is not None
    t = _replay_ms(_graph(fn, reps, flush))
    if flush:
        t -= _replay_ms(_graph(None, reps, True))
    return 1000.0 * t / reps


def attention_decode(a) -> None:
    B, H, C, n = a.batch, a.heads, a.ctx, a.n_ctx
    d = 64 * H
    g = torch.Generator(device="cuda").manual_seed(0)
    K = torch.randn((B, C, d), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, C, d), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B, d), device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty((B, d), dtype=torch.bfloat16, device="cuda")
    nctx = torch.full((B,), n, dtype=torch.int32, device="cuda")
    ws = torch.zeros((_lib.core().w8a8_attention_decode_workspace_size(B, H, C),),
                     dtype=torch.uint8, device="cuda")

    def run():
        ops.attention_decode(q, K, V, C * d, nctx, C, H, out=o, workspace=ws)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    kv = 2 * B * n * d * 2
    print(f"attention_decode B={B} H={H} n_ctx={n}: {us:.2f} us/launch, "
          f"KV {kv / 1e6:.1f} MB, {kv / us / 1e3:.0f} GB/s")


def attention_prefill(a) -> None:
    B, H, T = a.seqs, a.heads, a.tokens
    d = 64 * H
    g = torch.Generator(device="cuda").manual_seed(0)
    K = torch.randn((B, T, d), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, T, d), device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn((B * T, d), device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty((B * T, d), dtype=torch.bfloat16, device="cuda")

    def run():
        ops.attention_prefill(q, K, V, T * d, B, T, H, out=o)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    flops = B * H * 2.0 * 2 * 64 * T * (T + 1) / 2  # causal QK^T and PV
    print(f"attention_prefill seqs={B} T={T} H={H}: {us:.2f} us/launch, "
          f"{flops / us / 1e6:.1f} TFLOP/s (causal)")


def layernorm_quant(a) -> None:
    M, d = a.m, a.d
    g = torch.Generator(device="cuda").manual_seed(0)
    X = torch.randn((M, d), device="cuda", generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn((d,), device="cuda", generator=g)).to(torch.bfloat16)
    beta = (0.1 * torch.randn((d,), device="cuda", generator=g)).to(torch.bfloat16)

    def run():
        ops.layernorm_quant(X, gamma, beta, want_y=False)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    byts = M * d * 2 + M * d + M * 4
    print(f"layernorm_quant M={M} d={d}: {us:.2f} us/launch, {byts / us / 1e3:.0f} GB/s")


def quant_rows(a) -> None:
    M, K = a.m, a.k
    g = torch.Generator(device="cuda").manual_seed(0)
    X = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)

    def run():
        ops.per_token_quant(X)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    byts = M * K * 2 + M * K + M * 4
    print(f"quant_rows M={M} K={K}: {us:.2f} us/launch, {byts / us / 1e3:.0f} GB/s")


def linear(a) -> None:
    M, N, K = a.m, a.n, a.k
    g = torch.Generator(device="cuda").manual_seed(0)
    xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    sx = torch.rand((M,), device="cuda", generator=g) * 0.01 + 1e-3
    sw = torch.rand((N,), device="cuda", generator=g) * 0.01 + 1e-3
    b = (torch.randn((N,), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    R = torch.randn((M, N), device="cuda", generator=g).to(torch.bfloat16) \
        if a.epi == "resid" else None
    y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    # Only decode-sized GEMMs (M <= 128) split K and use the workspace.
    ws = ops.linear_workspace(M, N, "cuda") if M <= 128 else None
    epi = EPI[a.epi]

    def run():
        ops.linear(xq, sx, W, sw, b, epi, R=R, out=y, workspace=ws)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    ops_ = 2.0 * M * N * K
    byts = M * K + N * K + 2 * M * N + (2 * M * N if R is not None else 0)
    print(f"linear M={M} N={N} K={K} epi={a.epi}: {us:.2f} us/launch, "
          f"{ops_ / us / 1e6:.0f} TOP/s, {byts / us / 1e3:.0f} GB/s algorithmic")


def mlp_pair(a) -> None:
    """The decode MLP pair of a model, W1 (+GELU) then W2 (+residual), for
    --m tokens over --layers layers of distinct weights (streamed from HBM as
    in a decode step), in one CUDA graph per variant: W1 -> quant_rows -> W2
    against the fused pair (W1 with the row absmax record -> W2 quantizing
    its bf16 input), and each half of both alone."""
    from .quant8 import DIMS
    dims = DIMS[a.model]
    d, L, M = dims.d_model, a.layers, a.m
    f = 4 * d
    g = torch.Generator(device="cuda").manual_seed(0)
    W1 = [torch.randint(-127, 128, (f, d), dtype=torch.int8, device="cuda", generator=g)
          for _ in range(L)]
    W2 = [torch.randint(-127, 128, (d, f), dtype=torch.int8, device="cuda", generator=g)
          for _ in range(L)]
    sw1 = torch.rand((f,), device="cuda", generator=g) * 1e-3 + 1e-4
    sw2 = torch.rand((d,), device="cuda", generator=g) * 1e-3 + 1e-4
    b1 = (torch.randn((f,), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b2 = (torch.randn((d,), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    xq = torch.randint(-127, 128, (M, d), dtype=torch.int8, device="cuda", generator=g)
    sx = torch.full((M,), 1e-2, device="cuda")
    R = torch.randn((M, d), device="cuda", generator=g).to(torch.bfloat16)
    X1 = torch.empty((M, f), dtype=torch.bfloat16, device="cuda")
    Y = torch.empty((M, d), dtype=torch.bfloat16, device="cuda")
    q2 = torch.empty((M, f), dtype=torch.int8, device="cuda")
    s2 = torch.empty((M,), device="cuda")
    ws = ops.linear_workspace(M, f, "cuda")
    lib = _lib.core()
    cap = lib.w8a8_absmax_record_floats(M, f)
    rec = torch.empty(cap, dtype=torch.float32, device="cuda")
    n_part = ctypes.c_int(0)
    p = ops._ptr

    def w1_plain(i):
        ops.linear(xq, sx, W1[i], sw1, b1, EPI["gelu"], out=X1, workspace=ws)

    def quant():
        _lib.check(lib.w8a8_quant_rows(p(X1), f, M, f, p(q2), p(s2), ops._stream()), "quant")

    def w2_plain(i):
        ops.linear(q2, s2, W2[i], sw2, b2, EPI["resid"], R=R, out=Y, workspace=ws)

    def w1_absmax(i):
        _lib.check(lib.w8a8_linear_absmax(p(xq), p(sx), M, d, p(W1[i]), p(sw1), p(b1), f,
                                          EPI["gelu"], None, 0, p(X1), f, p(rec), cap,
                                          ctypes.byref(n_part), p(ws), ws.numel(),
                                          ops._stream()), "absmax")

    def w2_bf16(i):
        _lib.check(lib.w8a8_linear_from_bf16(p(X1), f, p(rec), n_part.value, M, f, p(W2[i]),
                                             p(sw2), p(b2), d, EPI["resid"], p(R), d, p(Y), d,
                                             p(q2), p(s2), p(ws), ws.numel(), ops._stream()),
                   "from_bf16")

    w1_absmax(0)
    torch.cuda.synchronize()
    variants = {
        "W1 -> quant -> W2": lambda: [(w1_plain(i), quant(), w2_plain(i)) for i in range(L)],
        "W1(absmax) -> W2(bf16 in)": lambda: [(w1_absmax(i), w2_bf16(i)) for i in range(L)],
        "W1 alone": lambda: [w1_plain(i) for i in range(L)],
        "W1(absmax) alone": lambda: [w1_absmax(i) for i in range(L)],
        "quant alone": lambda: [quant() for i in range(L)],
        "W2 alone": lambda: [w2_plain(i) for i in range(L)],
        "W2(bf16 in) alone": lambda: [w2_bf16(i) for i in range(L)],
    }
    for name, fn in variants.items():
        fn()
        torch.cuda.synchronize()
        ms = _replay_ms(_graph(fn, 1, False))
        print(f"mlp-pair {a.model} M={M} x{L} layers, {name}: {1000 * ms / L:.2f} us/layer "
              f"(parts {n_part.value})")


def gemv_chain(a) -> None:
    """The batch-1 decode GEMVs of a model back to back: per layer W_qkv,
    attn_proj, W1, W2 with their epilogues, each layer with its own weights
    (708 MB for GPT-2 large: every replay streams them from HBM), one CUDA
    graph. Per-GEMV time and the HBM bandwidth the weight stream reaches when
    each GEMV's weight loads overlap the previous launch (programmatic
    dependent launch), as inside a decode step."""
    from .quant8 import DIMS
    dims = DIMS[a.model]
    d, L = dims.d_model, a.layers
    g = torch.Generator(device="cuda").manual_seed(0)
    shapes = [(3 * d, d, "bias"), (d, d, "resid"), (4 * d, d, "gelu"), (d, 4 * d, "resid")]
    Ws = [[torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
           for n, k, _ in shapes] for _ in range(L)]
    xs = {k: torch.randint(-127, 128, (1, k), dtype=torch.int8, device="cuda", generator=g)
          for k in (d, 4 * d)}
    sx = torch.full((1,), 1e-3, device="cuda")
    sws = {n: torch.rand((n,), device="cuda", generator=g) * 0.01 + 1e-3 for n, _, _ in shapes}
    bs = {n: (torch.randn((n,), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
          for n, _, _ in shapes}
    R = torch.randn((1, d), device="cuda", generator=g).to(torch.bfloat16)
    ys = {n: torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for n, _, _ in shapes}

    def run():
        for layer in range(L):
            for (n, k, e), W in zip(shapes, Ws[layer]):
                ops.linear(xs[k], sx, W, sws[n], bs[n], EPI[e],
                           R=R if e == "resid" else None, out=ys[n])

    run()
    torch.cuda.synchronize()
    ms = _replay_ms(_graph(run, 1, False))
    n_launch = 4 * L
    wbytes = sum(n * k for n, k, _ in shapes) * L
    print(f"gemv-chain {a.model} x{L} layers: {1000 * ms / n_launch:.2f} us/GEMV, "
          f"{wbytes / 1e6:.0f} MB weights in {1000 * ms:.1f} us -> {wbytes / ms / 1e6:.0f} GB/s")


def decode(a) -> None:
    """Whole greedy decode steps of the engine (CUDA-graph replays): per-step
    time and the bytes a step must read (int8 weights + bf16 LM head + the KV
    cache at the mean context), i.e. the HBM roofline of batched decode."""
    from .engine import Engine
    from .quant8 import DIMS
    from .synthetic import prompts, quant8_image_gpu
    dims = DIMS[a.model]
    B, T, G = a.batch, a.prompt, a.gen
    eng = Engine(dims, max_batch=B, max_tokens=B * T)
    eng.load_quant8(quant8_image_gpu(dims, 0, "cuda"))
    P = torch.from_numpy(prompts(B, T, dims.vocab, 0)).cuda()
    out = torch.empty((B, G), dtype=torch.int32, device="cuda")
    s = torch.cuda.ExternalStream(eng.stream_handle)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(2):  # the first pass builds the decode graph
        e[0].record(s)
        eng.prefill(P, out, G)
        e[1].record(s)
        eng.decode_steps(G - 1)
        e[2].record(s)
        torch.cuda.synchronize()
    pre_ms, dec_ms = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])
    d, L = dims.d_model, dims.n_layer
    w_bytes = L * 12 * d * d + dims.vocab * d * 2
    kv_bytes = L * B * 2 * (T + G / 2) * d * 2
    us = 1000.0 * dec_ms / (G - 1)
    gbs = (w_bytes + kv_bytes) / us / 1e3
    print(f"decode {a.model} batch {B}, prompt {T}, {G} tokens: prefill {pre_ms:.2f} ms, "
          f"{us:.1f} us/step ({B / us * 1e6:.0f} tok/s); bytes/step {(w_bytes + kv_bytes) / 1e6:.0f}"
          f" MB -> {gbs:.0f} GB/s")


def sample(a) -> None:
    """The next-token pick of a decode step over rows x 50257 bf16 logits
    (N(0, 3)): greedy at temperature <= 0, else top-k sampling."""
    V = 50257
    g = torch.Generator(device="cuda").manual_seed(0)
    logits = (3 * torch.randn((a.rows, V), device="cuda", generator=g)).to(torch.bfloat16)
    rnd = torch.rand((a.rows,), device="cuda", generator=g)

    def run():
        if a.temperature > 0:
            ops.sample_topk(logits, a.temperature, a.top_k, rnd)
        else:
            ops.sample_greedy(logits)

    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    us = _time(run, a.timed)
    what = f"top-{a.top_k} at T={a.temperature}" if a.temperature > 0 else "greedy"
    print(f"sample {what}, {a.rows} rows x {V}: {us:.2f} us/launch, "
          f"{a.rows * V * 2 / us / 1e3:.0f} GB/s of logits")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="case", required=True)
    p = sub.add_parser("attention-decode")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--heads", type=int, default=20)
    p.add_argument("--ctx", type=int, default=1024)
    p.add_argument("--n-ctx", type=int, default=768)
    p = sub.add_parser("attention-prefill")
    p.add_argument("--seqs", type=int, default=64)
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--heads", type=int, default=20)
    p = sub.add_parser("layernorm-quant")
    p.add_argument("--m", type=int, default=32768)
    p.add_argument("--d", type=int, default=1280)
    p = sub.add_parser("quant-rows")
    p.add_argument("--m", type=int, default=32768)
    p.add_argument("--k", type=int, default=5120)
    p = sub.add_parser("decode")
    p.add_argument("--model", choices=["small", "medium", "large"], default="medium")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--gen", type=int, default=256)
    p = sub.add_parser("gemv-chain")
    p.add_argument("--model", choices=["small", "medium", "large"], default="large")
    p.add_argument("--layers", type=int, default=36)
    p = sub.add_parser("linear")
    p.add_argument("--m", type=int, required=True)
    p.add_argument("--n", type=int, required=True)
    p.add_argument("--k", type=int, required=True)
    p.add_argument("--epi", choices=sorted(EPI), default="bias")
    p = sub.add_parser("mlp-pair")
    p.add_argument("--model", choices=["small", "medium", "large"], default="large")
    p.add_argument("--m", type=int, default=64)
    p.add_argument("--layers", type=int, default=36)
    p = sub.add_parser("sample")
    p.add_argument("--rows", type=int, default=64)
    p.add_argument("--top-k", type=int, default=40)
    p.add_argument("--temperature", type=float, default=0.8)
    for p in sub.choices.values():
        p.add_argument("--launches", type=int, default=3, help="launches before timing")
        p.add_argument("--timed", type=int, default=20, help="launches timed after them")
        p.add_argument("--flush", action="store_true", help="evict L2 before each timed launch")
    a = ap.parse_args(argv)
    ops.init(0)
    if a.flush:
        global _FLUSH
        _FLUSH = torch.ones((64 << 20,), dtype=torch.float32, device="cuda")
    {"attention-decode": attention_decode, "attention-prefill": attention_prefill,
     "layernorm-quant": layernorm_quant, "linear": linear, "decode": decode,
     "gemv-chain": gemv_chain, "sample": sample, "mlp-pair": mlp_pair,
     "quant-rows": quant_rows}[a.case](a)
    st = ops.device_error()
    if st:
        raise SystemExit(f"device error word {st}")


if __name__ == "__main__":
    main()
