"""Host logic of the tensor-parallel prefill (c_gpt2_b200/tp.py) on CPU ranks.

The shard plan must cover every head, d_ff column and sequence exactly once,
and the exchange steps (all-gather of int8 rows, max-allreduce of row maxima,
int32 reduce-scatter) must reassemble the single-rank layer exactly. Here the
device kernels are replaced by plain torch CPU stand-ins with the same
contracts (integer GEMMs, per-row float work), and two gloo ranks must
reproduce the one-rank run bit for bit.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from c_gpt2_b200.quant8 import GPT2Dims, quantize_per_channel, tensor_layout
from c_gpt2_b200.tp import Collectives, TPPlan, TPPrefill, shard_weights, split_even

TINY = GPT2Dims(d_model=256, n_layer=2, n_head=4, vocab=97, ctx=64)


def test_split_even_covers_and_balances():
    assert split_even(20, 8) == [(0, 3), (3, 6), (6, 9), (9, 12), (12, 14), (14, 16), (16, 18),
                                 (18, 20)]
    for n, p in [(20, 2), (20, 4), (80, 8), (7, 7)]:
        parts = split_even(n, p)
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        sizes = [e - s for s, e in parts]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        split_even(3, 4)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_gpt2_large(world):
    dims = GPT2Dims(1280, 36, 20)
    plan = TPPlan.make(dims, world)
    rows = np.concatenate([plan.qkv_rows(r) for r in range(world)])
    assert sorted(rows.tolist()) == list(range(3 * dims.d_model))
    assert sum(plan.d_heads(r) for r in range(world)) == dims.d_model
    assert all(plan.d_heads(r) % 32 == 0 for r in range(world))
    ff = [plan.ff[r] for r in range(world)]
    assert ff[0][0] == 0 and ff[-1][1] == dims.d_ff
    assert all((e - s) % 64 == 0 for s, e in ff)
    seqs = [plan.seqs(32, r) for r in range(world)]
    assert seqs[0][0] == 0 and seqs[-1][1] == 32


def _weights(dims: GPT2Dims, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in tensor_layout(dims):
        leaf = name.split(".")[-1]
        if leaf.endswith("gamma"):
            a = 1.0 + 0.1 * rng.standard_normal(shape)
        elif leaf.endswith("beta"):
            a = 0.1 * rng.standard_normal(shape)
        else:
            a = 0.05 * rng.standard_normal(shape)
        a = a.astype(np.float32)
        if leaf in ("W_qkv", "attn_proj", "W1", "W2"):
            q, s = quantize_per_channel(a)
            w[name], w[name + ".scale"] = q, s
        else:
            w[name] = a
    return w


def test_shard_weights_slices():
    plan = TPPlan.make(TINY, 2)
    w = _weights(TINY)
    sh = shard_weights(w, plan, 1, "cpu")
    L = sh.layers[0]
    d = TINY.d_model
    assert L["W_qkv"].shape == (3 * d // 2, d)
    np.testing.assert_array_equal(L["W_qkv"].numpy()[:d // 2], w["h0.W_qkv"][d // 2:d])
    np.testing.assert_array_equal(L["W_qkv"].numpy()[d // 2:d], w["h0.W_qkv"][d + d // 2:2 * d])
    np.testing.assert_array_equal(L["attn_proj"].numpy(), w["h0.attn_proj"][:, d // 2:])
    f0, f1 = plan.ff[1]
    np.testing.assert_array_equal(L["W1"].numpy(), w["h0.W1"][f0:f1])
    np.testing.assert_array_equal(L["W2"].numpy(), w["h0.W2"][:, f0:f1])
    assert L["W2"].is_contiguous() and L["attn_proj"].is_contiguous()


# ---- torch CPU stand-ins for the device kernels (test infrastructure) -------

def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.float().to(torch.bfloat16)


def _quant(X: torch.Tensor, amax: torch.Tensor):
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.round(X.float() * (1.0 / scale)[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale


def _ln(X: torch.Tensor, g, b, eps):
    x = X.float()
    mu = x.mean(1, keepdim=True)
    var = ((x - mu) ** 2).mean(1, keepdim=True)
    return _bf((x - mu) * torch.rsqrt(var + eps) * g.float() + b.float())


def _acc(Xq, W):
    return (Xq.long() @ W.long().T).to(torch.int32)


def _deq_bias(acc, sX, sW, b):
    return _bf(_bf(acc.float() * sW[None, :] * sX[:, None]).float() + b.float())


class CPUKernels:
    @staticmethod
    def embed_layernorm_quant(wte, wpe, tok, T, pos0, g, b, eps):
        pos = torch.arange(tok.numel()) % T
        H = _bf(wte[tok].float() + wpe[pos].float())
        Y = _ln(H, g, b, eps)
        q, s = _quant(Y, Y.float().abs().amax(1))
        return H, Y, q, s

    @staticmethod
    def linear_qkv_heads(Xq, sX, W, sW, b, Q, Kc, Vc, seq_stride, T):
        y = _deq_bias(_acc(Xq, W), sX, sW, b)
        dh = W.shape[0] // 3
        Q.copy_(y[:, :dh])
        Kc.view(-1, dh).copy_(y[:, dh:2 * dh])
        Vc.view(-1, dh).copy_(y[:, 2 * dh:])

    @staticmethod
    def attention_prefill(Q, Kc, Vc, seq_stride, n_seq, T, hl):
        q = Q.float().view(n_seq, T, hl, 64).transpose(1, 2)
        k = Kc.float().view(n_seq, T, hl, 64).transpose(1, 2)
        v = Vc.float().view(n_seq, T, hl, 64).transpose(1, 2)
        s = q @ k.transpose(-1, -2) / 8.0
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
        o = torch.softmax(s, -1) @ v
        return _bf(o.transpose(1, 2).reshape(n_seq * T, hl * 64))

    @staticmethod
    def row_amax(X):
        return X.float().abs().amax(1)

    @staticmethod
    def quant_rows_amax(X, amax):
        return _quant(X, amax)

    gemm_s32 = staticmethod(_acc)

    @staticmethod
    def linear(Xq, sX, W, sW, b, epilogue, R=None, out=None):
        y = _deq_bias(_acc(Xq, W), sX, sW, b)
        if epilogue == 2:  # + residual
            y = _bf(R.float() + y.float())
        else:
            assert epilogue == 3
            y = y.float()
            y = _bf(0.5 * y * (1.0 + torch.tanh(0.79788456 * (y + 0.044715 * y ** 3))))
        if out is not None:
            out.copy_(y)
            return out
        return y

    @staticmethod
    def reduce_residual_layernorm_quant(acc, sX, sW, b, R, H, g=None, beta=None, eps=1e-5,
                                        Xq=None, sXq=None):
        H.copy_(_bf(R.float() + _deq_bias(acc, sX, sW, b).float()))
        if g is not None:
            Y = _ln(H, g, beta, eps)
            q, s = _quant(Y, Y.float().abs().amax(1))
            Xq.copy_(q)
            sXq.copy_(s)
        return H

    @staticmethod
    def layernorm_quant(X, g, b, eps, want_y=True, want_q=True):
        Y = _ln(X, g, b, eps)
        q, s = _quant(Y, Y.float().abs().amax(1)) if want_q else (None, None)
        return (Y if want_y else None), q, s

    @staticmethod
    def lm_head(Xf, wte):
        return _bf(Xf.float() @ wte.float().T)

    @staticmethod
    def sample_greedy(logits):
        return torch.argmax(logits.float(), dim=1).to(torch.int32)


def _tokens(n_seq, T):
    return torch.from_numpy(np.random.default_rng(3).integers(0, TINY.vocab, (n_seq, T))
                            ).to(torch.int32)


def _run_rank(rank, world, port, out_dir, exchange, halves, n_seq=4):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = TPPlan.make(TINY, world)
        shard = shard_weights(_weights(TINY), plan, rank, "cpu")
        nxt, logits = TPPrefill(plan, shard, rank, CPUKernels(), Collectives(),
                                exchange=exchange, halves=halves).run(_tokens(n_seq, 16))
        torch.save({"next": nxt, "logits": logits}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange,halves", [("alltoall", True), ("alltoall", False),
                                            ("collective", False)])
def test_tp_prefill_two_gloo_ranks_equal_one_rank(tmp_path, exchange, halves):
    """Two ranks, with the int8 inputs of the row-split GEMMs sent to the rows'
    owners (alltoall; the batch in two interleaved halves or whole) or their
    int32 partial sums reduce-scattered (collective): the one-rank result bit
    for bit."""
    plan1 = TPPlan.make(TINY, 1)
    shard1 = shard_weights(_weights(TINY), plan1, 0, "cpu")
    want_next, want_logits = TPPrefill(plan1, shard1, 0, CPUKernels(), Collectives(),
                                       exchange="collective").run(_tokens(4, 16))
    port = 29500 + os.getpid() % 300 + {"collective": 0, "alltoall": 300}[exchange] + 300 * halves
    mp.start_processes(_run_rank, args=(2, port, str(tmp_path), exchange, halves), nprocs=2,
                       join=True, start_method="spawn")
    got = [torch.load(tmp_path / f"r{r}.pt") for r in range(2)]
    for g in got:
        assert torch.equal(g["next"], want_next)
    logits = torch.cat([g["logits"] for g in got])
    assert torch.equal(logits, want_logits)


def test_tp_prefill_three_gloo_ranks_uneven_heads(tmp_path):
    """Three ranks: 4 heads as 2, 1, 1 and d_ff as 6, 5, 5 units of 64, so the
    all-to-all moves column blocks of different widths (the shape of 20 heads
    over 8 GPUs): the one-rank result bit for bit."""
    plan1 = TPPlan.make(TINY, 1)
    shard1 = shard_weights(_weights(TINY), plan1, 0, "cpu")
    want_next, want_logits = TPPrefill(plan1, shard1, 0, CPUKernels(), Collectives(),
                                       exchange="collective").run(_tokens(6, 16))
    plan3 = TPPlan.make(TINY, 3)
    assert [plan3.d_heads(r) for r in range(3)] == [128, 64, 64]
    port = 28400 + os.getpid() % 500
    mp.start_processes(_run_rank, args=(3, port, str(tmp_path), "alltoall", True, 6), nprocs=3,
                       join=True, start_method="spawn")
    got = [torch.load(tmp_path / f"r{r}.pt") for r in range(3)]
    for g in got:
        assert torch.equal(g["next"], want_next)
    assert torch.equal(torch.cat([g["logits"] for g in got]), want_logits)
