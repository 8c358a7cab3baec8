"""Tensor-parallel W8A8 prefill of GPT-2 over G GPUs (one process per GPU),
bit-identical to the single-GPU layer.

The reference runs every layer on one GPU (transformer_block_gpu,
gpt2.c:1124-1330). Here each layer is split the Megatron way, with the
exchange steps chosen so that no rounding changes:

* W_qkv is column-split by whole heads and attention runs on the local heads;
  W1 is column-split into a d_ff slice. Both read the full quantized LayerNorm
  output, which every GPU holds (all-gather of int8 rows + fp32 scales).
* attn_proj and W2 are row-split over the same head dims / d_ff slice. Their
  inputs are quantized per token over the WHOLE row (activation_quant.cu:
  75-91), so each GPU contributes its row maxima and the scale comes from a
  max-allreduce of [M] floats; quantizing the local columns with it gives
  exactly the single-GPU int8 values.
* The row-split GEMMs produce int32 partial sums, reduce-scattered (exact in
  any order) so that each GPU owns whole sequences of the residual stream.
  The owner applies dequant + bias + residual with the single-GPU rounding
  points, then the next LayerNorm + quant, and the int8 rows are all-gathered.

Per sub-block the exchange is an int32 reduce-scatter of [M, d] plus an int8
all-gather of [M, d] (5 bytes per element against the 4 of a bf16
all-reduce), in exchange for outputs equal to one GPU's bit for bit.

`Kernels` is the device side (the library's CUDA kernels through ops);
`Collectives` is the exchange (torch.distributed: NCCL on GPUs). Both are
parameters so that the host logic can be exercised on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .quant8 import GPT2Dims

HEAD_DIM = 64


def split_even(n: int, parts: int) -> list[tuple[int, int]]:
    """[start, end) of `parts` contiguous pieces of n, the first n % parts one
    larger (20 heads over 8 GPUs: 3,3,3,3,2,2,2,2)."""
    if parts <= 0 or n < parts:
        raise ValueError(f"cannot split {n} into {parts} non-empty parts")
    base, extra = divmod(n, parts)
    out, s = [], 0
    for r in range(parts):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


@dataclass(frozen=True)
class TPPlan:
    """Which heads, d_ff columns and sequences each rank owns."""
    dims: GPT2Dims
    world: int
    heads: tuple[tuple[int, int], ...]  # per rank [h0, h1)
    ff: tuple[tuple[int, int], ...]     # per rank [f0, f1) of d_ff, multiples of 64

    @staticmethod
    def make(dims: GPT2Dims, world: int) -> "TPPlan":
        heads = tuple(split_even(dims.n_head, world))
        units = split_even(dims.d_ff // HEAD_DIM, world)
        ff = tuple((a * HEAD_DIM, b * HEAD_DIM) for a, b in units)
        return TPPlan(dims, world, heads, ff)

    def d_heads(self, rank: int) -> int:
        h0, h1 = self.heads[rank]
        return (h1 - h0) * HEAD_DIM

    def qkv_rows(self, rank: int) -> np.ndarray:
        """Rows of the packed W_qkv [3d, d] (Q, K, V blocks) of rank's heads."""
        d = self.dims.d_model
        h0, h1 = self.heads[rank]
        cols = np.arange(h0 * HEAD_DIM, h1 * HEAD_DIM)
        return np.concatenate([cols, d + cols, 2 * d + cols])

    def seqs(self, n_seq: int, rank: int) -> tuple[int, int]:
        """Sequences [s0, s1) whose residual stream rank owns."""
        if n_seq % self.world:
            raise ValueError(f"{n_seq} sequences do not split evenly over {self.world} GPUs")
        per = n_seq // self.world
        return rank * per, (rank + 1) * per


@dataclass
class TPShard:
    """One rank's weights: replicated embeddings and norms, its slices of the
    four GEMM weights (int8 + fp32 scales) and biases (bf16)."""
    wte: torch.Tensor
    wpe: torch.Tensor
    lnf_gamma: torch.Tensor
    lnf_beta: torch.Tensor
    layers: list[dict[str, torch.Tensor]]


def _bf16(a: np.ndarray, device) -> torch.Tensor:
    # fp32 -> bf16 with round-to-nearest-even, as the weight loader does
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(
        torch.bfloat16)


def _dev(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def shard_weights(w: dict[str, np.ndarray], plan: TPPlan, rank: int, device) -> TPShard:
    """Slice a parsed quant8 image (quant8.read_quant8) for `rank`."""
    d = plan.dims.d_model
    h0, h1 = plan.heads[rank]
    c0, c1 = h0 * HEAD_DIM, h1 * HEAD_DIM
    f0, f1 = plan.ff[rank]
    rows = plan.qkv_rows(rank)
    layers = []
    for l in range(plan.dims.n_layer):
        p = f"h{l}."
        layers.append({
            "ln1_gamma": _bf16(w[p + "ln1_gamma"], device),
            "ln1_beta": _bf16(w[p + "ln1_beta"], device),
            "W_qkv": _dev(w[p + "W_qkv"][rows], device),
            "W_qkv.scale": _dev(w[p + "W_qkv.scale"][rows], device),
            "b_qkv": _bf16(w[p + "b_qkv"][rows], device),
            "attn_proj": _dev(w[p + "attn_proj"][:, c0:c1], device),
            "attn_proj.full": _dev(w[p + "attn_proj"], device),
            "attn_proj.scale": _dev(w[p + "attn_proj.scale"], device),
            "attn_proj_bias": _bf16(w[p + "attn_proj_bias"], device),
            "ln2_gamma": _bf16(w[p + "ln2_gamma"], device),
            "ln2_beta": _bf16(w[p + "ln2_beta"], device),
            "W1": _dev(w[p + "W1"][f0:f1], device),
            "W1.scale": _dev(w[p + "W1.scale"][f0:f1], device),
            "b1": _bf16(w[p + "b1"][f0:f1], device),
            "W2": _dev(w[p + "W2"][:, f0:f1], device),
            "W2.full": _dev(w[p + "W2"], device),
            "W2.scale": _dev(w[p + "W2.scale"], device),
            "b2": _bf16(w[p + "b2"], device),
        })
    assert d == w["wte"].shape[1]
    return TPShard(_bf16(w["wte"], device), _bf16(w["wpe"], device),
                   _bf16(w["lnf_gamma"], device), _bf16(w["lnf_beta"], device), layers)


class Collectives:
    """The three exchange steps, over a torch.distributed process group (none
    needed when the group has one rank)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def all_gather_rows(self, full: torch.Tensor, rank: int, world: int) -> None:
        """full [world*m, ...]: rank's chunk is filled in, every chunk comes back."""
        if self.world == 1:
            return
        m = full.shape[0] // world
        own = full[rank * m:(rank + 1) * m]
        # NCCL gathers in place when the input is this rank's chunk of the
        # output; other backends get a copy of the chunk
        if dist.get_backend(self.group) != "nccl":
            own = own.clone()
        dist.all_gather_into_tensor(full, own, group=self.group)

    def reduce_scatter_sum(self, out: torch.Tensor, full: torch.Tensor) -> None:
        if self.world == 1:
            out.copy_(full)
            return
        dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.SUM, group=self.group)

    def all_reduce_max(self, x: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(x, op=dist.ReduceOp.MAX, group=self.group)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int],
                   in_splits: list[int]) -> None:
        """1-D tensors: block j of inp (in_splits[j] elements) goes to rank j;
        block j of out comes from rank j."""
        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)


class Kernels:
    """Device side of one tensor-parallel layer: the library's CUDA kernels."""

    embed_layernorm_quant = staticmethod(ops.embed_layernorm_quant)
    linear_qkv_heads = staticmethod(ops.linear_qkv_heads)
    attention_prefill = staticmethod(ops.attention_prefill)
    row_amax = staticmethod(ops.row_amax)
    quant_rows_amax = staticmethod(ops.quant_rows_amax)
    gemm_s32 = staticmethod(ops.gemm_s32)
    linear = staticmethod(ops.linear)
    reduce_residual_layernorm_quant = staticmethod(ops.reduce_residual_layernorm_quant)
    layernorm_quant = staticmethod(ops.layernorm_quant)
    lm_head = staticmethod(ops.lm_head)
    sample_greedy = staticmethod(ops.sample_greedy)


class CollectiveExchange:
    """The exchange steps through collectives (NCCL on GPUs, gloo on CPU):
    fp32 max all-reduce of row maxima, int32 reduce-scatter of partial sums,
    all-gather of the owners' quantized rows."""

    def __init__(self, kernels, collectives: Collectives, rank: int, world: int, M: int, d: int,
                 device):
        self.k, self.c, self.rank, self.world = kernels, collectives, rank, world
        self.Mo = M // world
        self.Xq = torch.empty((M, d), dtype=torch.int8, device=device)
        self.sX = torch.empty((M,), dtype=torch.float32, device=device)
        self.P_own = torch.empty((self.Mo, d), dtype=torch.int32, device=device)

    def own_rows(self):
        m0 = self.rank * self.Mo
        return self.Xq[m0:m0 + self.Mo], self.sX[m0:m0 + self.Mo]

    def publish_rows(self) -> None:
        self.c.all_gather_rows(self.Xq, self.rank, self.world)
        self.c.all_gather_rows(self.sX, self.rank, self.world)

    def row_maxima(self, X: torch.Tensor, kind: int) -> torch.Tensor:
        amax = self.k.row_amax(X)
        self.c.all_reduce_max(amax)
        return amax

    def partial_sums(self, Xq: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
        P = self.k.gemm_s32(Xq, W)
        self.c.reduce_scatter_sum(self.P_own, P)
        return self.P_own

    def reduce(self, acc, sx, sW, b, H, gamma=None, beta=None, eps=1e-5) -> None:
        if gamma is None:
            self.k.reduce_residual_layernorm_quant(acc, sx, sW, b, H, H)
            return
        xq, sxq = self.own_rows()
        self.k.reduce_residual_layernorm_quant(acc, sx, sW, b, H, H, gamma, beta, eps, xq, sxq)
        self.publish_rows()

    def gather_tokens(self, nxt: torch.Tensor) -> None:
        self.c.all_gather_rows(nxt, self.rank, self.world)


class AllToAllExchange(CollectiveExchange):
    """Row-split GEMMs without partial sums: the int8 input columns each rank
    holds for every row (its heads' attention output, its d_ff slice of the
    GELU output) go to the rows' owners in one all-to-all, and each owner
    runs attn_proj and W2 over its own rows with the whole K. The owner's
    GEMM then computes exactly the one-GPU layer's rows (same int32 sums,
    same fused epilogue), and the exchange moves int8 inputs instead of int32
    partial sums: at G ranks each rank sends (G-1)/G of its column block."""

    def __init__(self, kernels, collectives: Collectives, rank: int, world: int, M: int, d: int,
                 device):
        super().__init__(kernels, collectives, rank, world, M, d, device)
        self.device = device

    def to_owners(self, X: torch.Tensor, cols: list[int]) -> torch.Tensor:
        """X [M, cols[rank]] int8 -> [Mo, sum(cols)] int8: this rank's rows with
        every rank's columns, in rank order."""
        Mo, c = self.Mo, X.shape[1]
        recv = torch.empty((Mo * sum(cols),), dtype=X.dtype, device=self.device)
        self.c.all_to_all(recv, X.reshape(-1), [Mo * cq for cq in cols], [Mo * c] * self.world)
        blocks, off = [], 0
        for cq in cols:
            blocks.append(recv[off:off + Mo * cq].view(Mo, cq))
            off += Mo * cq
        return torch.cat(blocks, dim=1) if len(blocks) > 1 else blocks[0]


class PeerExchange:
    """The same exchange steps done by the library's kernels over NVLink peer
    memory, with no collective on the data path:

    * row maxima: `w8a8_row_amax_to` stores this GPU's [M] maxima into slot
      `rank` of every GPU's [G][M] array; the quantization takes the max over
      the G slots;
    * partial sums: `w8a8_gemm_s32_scatter` stores the int32 rows each GPU owns
      straight into slot `rank` of that GPU's [G][M/G][d] receive area (16-byte
      peer stores from the GEMM epilogue); the owner's reduce kernel adds the
      G slots in rank order;
    * quantized rows: the owner's reduce + LayerNorm + quant kernel also stores
      its int8 rows and scales into every other GPU's [M][d] buffer.

    Each step ends with a flag per (kind, source) on every destination GPU
    (`w8a8_peer_signal`, system-scope release) and a bounded wait for the G
    flags of this GPU (`w8a8_peer_wait`). Flag values are per-kind epoch
    counters, so no flag is ever reset. Every buffer is reused only after a
    later exchange step has proven that all GPUs finished reading it."""

    KINDS = 5  # 0 partial sums, 1 quantized rows, 2 attention maxima, 3 GELU maxima, 4 tokens

    def __init__(self, rank: int, world: int, M: int, d: int, group=None):
        from . import peer
        self.peer = peer
        self.rank, self.world, self.M, self.d = rank, world, M, d
        self.Mo = Mo = M // world
        G = world
        off = 0

        def region(nbytes):
            nonlocal off
            o = off
            off += (nbytes + 255) & ~255
            return o

        self.o_acc = region(G * Mo * d * 4)
        self.o_xq = region(M * d)
        self.o_sx = region(M * 4)
        self.o_amax = [region(G * M * 4), region(G * M * 4)]
        self.o_tok = region(M * 4)
        self.o_flags = region(self.KINDS * G * 4)
        self.buf = peer.PeerBuffer(off, group)
        base = self.buf.local
        self.acc = peer.view(base + self.o_acc, (G, Mo, d), torch.int32)
        self.Xq = peer.view(base + self.o_xq, (M, d), torch.int8)
        self.sX = peer.view(base + self.o_sx, (M,), torch.float32)
        self.amax = [peer.view(base + o, (G, M), torch.float32) for o in self.o_amax]
        self.epoch = [0] * self.KINDS

    def close(self) -> None:
        self.buf.close()

    def _flag(self, r: int, kind: int, src: int) -> int:
        return self.buf.base[r] + self.o_flags + (kind * self.world + src) * 4

    def _step(self, kind: int) -> None:
        """Publish this GPU's part of step `kind`, then wait for everyone's."""
        self.epoch[kind] += 1
        e = self.epoch[kind]
        self.peer.signal([self._flag(r, kind, self.rank) for r in range(self.world)], e)
        self.peer.wait(self._flag(self.rank, kind, 0), self.world, e)

    def own_rows(self):
        m0 = self.rank * self.Mo
        return self.Xq[m0:m0 + self.Mo], self.sX[m0:m0 + self.Mo]

    def publish_rows(self) -> None:
        """Copy this GPU's rows of Xq/sX into every other GPU's buffers."""
        m0, Mo, d = self.rank * self.Mo, self.Mo, self.d
        for r in range(self.world):
            if r != self.rank:
                b = self.buf.base[r]
                self.peer.copy(b + self.o_xq + m0 * d, self.buf.local + self.o_xq + m0 * d, Mo * d)
                self.peer.copy(b + self.o_sx + m0 * 4, self.buf.local + self.o_sx + m0 * 4, Mo * 4)
        self._step(1)

    def row_maxima(self, X: torch.Tensor, kind: int) -> torch.Tensor:
        o = self.o_amax[kind]
        ops.row_amax_to(X, [self.buf.base[r] + o + self.rank * self.M * 4
                            for r in range(self.world)])
        self._step(2 + kind)
        return self.amax[kind]

    def partial_sums(self, Xq: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
        slot = self.rank * self.Mo * self.d * 4
        ops.gemm_s32_scatter(Xq, W, [self.buf.base[r] + self.o_acc + slot
                                     for r in range(self.world)], self.Mo)
        self._step(0)
        return self.acc

    def reduce(self, acc, sx, sW, b, H, gamma=None, beta=None, eps=1e-5) -> None:
        if gamma is None:
            ops.reduce_residual_layernorm_quant(acc, sx, sW, b, H, H)
            return
        xq, sxq = self.own_rows()
        others = [r for r in range(self.world) if r != self.rank]
        ops.reduce_residual_layernorm_quant_bcast(
            acc, sx, sW, b, H, H, gamma, beta, eps, xq, sxq,
            [self.buf.base[r] + self.o_xq for r in others],
            [self.buf.base[r] + self.o_sx for r in others], self.rank * self.Mo)
        self._step(1)

    def gather_tokens(self, nxt: torch.Tensor) -> None:
        n = nxt.numel() // self.world
        s0 = self.rank * n
        tok = self.buf.local + self.o_tok
        self.peer.copy(tok + s0 * 4, nxt[s0:s0 + n].data_ptr(), n * 4)
        for r in range(self.world):
            if r != self.rank:
                self.peer.copy(self.buf.base[r] + self.o_tok + s0 * 4, nxt[s0:s0 + n].data_ptr(),
                               n * 4)
        self._step(4)
        nxt.copy_(self.peer.view(tok, (nxt.numel(),), torch.int32))


class TPPrefill:
    """Prefill of n_seq prompts of T tokens on `world` ranks; returns the
    greedy next token of every sequence (on every rank) and the last-position
    logits of the sequences this rank owns.

    exchange: "alltoall" (int8 inputs to the rows' owners in one all-to-all,
    whole-K GEMMs there), "collective" (int32 partial sums reduce-scattered),
    both over NCCL / gloo collectives, or "peer" (partial sums through the
    library's own kernels over NVLink peer memory; GPUs only).

    halves (exchange "alltoall", more than one rank): the batch runs as two
    halves, each rank's first and second halves of its own sequences, each
    half with its own process group and (on GPUs) its own CUDA stream; their
    layers are issued alternately, so that one half's exchanges run while the
    other half computes. Each sequence's arithmetic is unchanged. Off by
    default: GPT-2 large 32 x 1024 on 2 GPUs took 50.4 ms in halves against
    48.2 ms as one batch."""

    def __init__(self, plan: TPPlan, shard: TPShard, rank: int, kernels=None,
                 collectives: Collectives | None = None, eps: float = 1e-5,
                 exchange: str = "alltoall", group=None, halves: bool = False):
        self.plan, self.w, self.rank = plan, shard, rank
        self.k = kernels or Kernels()
        self.c = collectives or Collectives(group)
        self.eps = eps
        self.mode = exchange
        self.group = group
        self._ex = None
        self._halves = None
        if halves and exchange == "alltoall" and plan.world > 1 and dist.is_initialized():
            # one process group per half, created in the same order on every rank
            ranks = list(range(plan.world))
            self._halves = [{"c": Collectives(dist.new_group(ranks)), "ex": None}
                            for _ in range(2)]

    def _exchange(self, M: int, d: int, device):
        ex = self._ex
        if ex is not None and ex.M_key == (M, d):
            return ex
        if ex is not None and hasattr(ex, "close"):
            ex.close()
        if self.mode == "peer":
            ex = PeerExchange(self.rank, self.plan.world, M, d, self.group)
        elif self.mode == "alltoall":
            ex = AllToAllExchange(self.k, self.c, self.rank, self.plan.world, M, d, device)
        else:
            ex = CollectiveExchange(self.k, self.c, self.rank, self.plan.world, M, d, device)
        ex.M_key = (M, d)
        self._ex = ex
        return ex

    def close(self) -> None:
        if self._ex is not None and hasattr(self._ex, "close"):
            self._ex.close()
        self._ex = None
        if self._halves:
            for h in self._halves:
                h["ex"] = None

    def _layers_alltoall(self, ex, H, Q, Kc, Vc, n_seq, T, hl, dh, m0, m1):
        """The blocks of TPPrefill.run for exchange "alltoall": QKV and W1 over the
        rank's column slices for all rows; attn_proj and W2 over the rank's own
        rows with the whole K, their inputs brought by AllToAllExchange.to_owners;
        LayerNorm + quantization of the own rows, published to every rank."""
        plan, w, k = self.plan, self.w, self.k
        Xq, sX = ex.Xq, ex.sX
        heads = [plan.d_heads(q) for q in range(plan.world)]
        ffs = [f1 - f0 for f0, f1 in plan.ff]
        R1 = torch.empty_like(H)
        n_layer = len(w.layers)
        for l, L in enumerate(w.layers):
            k.linear_qkv_heads(Xq, sX, L["W_qkv"], L["W_qkv.scale"], L["b_qkv"], Q, Kc, Vc,
                               T * dh, T)
            O = k.attention_prefill(Q, Kc, Vc, T * dh, n_seq, T, hl)
            Oq, sO = k.quant_rows_amax(O, ex.row_maxima(O, 0))
            del O
            yield
            Oq_own = ex.to_owners(Oq, heads)
            yield
            # attn_proj + bias + residual (gpt2.c:1235-1245), then LN2 + quantization
            k.linear(Oq_own, sO[m0:m1].contiguous(), L["attn_proj.full"], L["attn_proj.scale"],
                     L["attn_proj_bias"], epilogue=2, R=H, out=R1)
            xq, sxq = ex.own_rows()
            _, q, sq = k.layernorm_quant(R1, L["ln2_gamma"], L["ln2_beta"], self.eps, want_y=False)
            xq.copy_(q)
            sxq.copy_(sq)
            ex.publish_rows()
            yield
            Gk = k.linear(Xq, sX, L["W1"], L["W1.scale"], L["b1"], epilogue=3)
            Gq, sG = k.quant_rows_amax(Gk, ex.row_maxima(Gk, 1))
            del Gk
            yield
            Gq_own = ex.to_owners(Gq, ffs)
            yield
            # W2 + bias + residual (gpt2.c:1302-1325), then the next layer's LN1
            k.linear(Gq_own, sG[m0:m1].contiguous(), L["W2.full"], L["W2.scale"], L["b2"],
                     epilogue=2, R=R1, out=H)
            if l + 1 < n_layer:
                N = w.layers[l + 1]
                _, q, sq = k.layernorm_quant(H, N["ln1_gamma"], N["ln1_beta"], self.eps,
                                             want_y=False)
                xq.copy_(q)
                sxq.copy_(sq)
                ex.publish_rows()
                yield

    def _layers_partial_sums(self, ex, H, Q, Kc, Vc, n_seq, T, hl, dh, m0, m1) -> None:
        """The blocks for exchanges "collective" and "peer": attn_proj and W2
        over the rank's K slices for all rows, the int32 partial sums
        reduce-scattered to the rows' owners, which add bias and residual and
        form the LayerNorm + quantization of their rows."""
        w, k = self.w, self.k
        Xq, sX = ex.Xq, ex.sX
        n_layer = len(w.layers)
        for l, L in enumerate(w.layers):
            # attention on the local heads
            k.linear_qkv_heads(Xq, sX, L["W_qkv"], L["W_qkv.scale"], L["b_qkv"], Q, Kc, Vc,
                               T * dh, T)
            O = k.attention_prefill(Q, Kc, Vc, T * dh, n_seq, T, hl)
            # attn_proj, row-split: whole-row scale, int32 partials to the row owners
            Oq, sO = k.quant_rows_amax(O, ex.row_maxima(O, 0))
            acc = ex.partial_sums(Oq, L["attn_proj"])
            ex.reduce(acc, sO[m0:m1], L["attn_proj.scale"], L["attn_proj_bias"], H,
                      L["ln2_gamma"], L["ln2_beta"], self.eps)
            # MLP: W1 column-split with GELU, W2 row-split
            Gk = k.linear(Xq, sX, L["W1"], L["W1.scale"], L["b1"], epilogue=3)
            Gq, sG = k.quant_rows_amax(Gk, ex.row_maxima(Gk, 1))
            del Gk
            acc = ex.partial_sums(Gq, L["W2"])
            if l + 1 < n_layer:
                N = w.layers[l + 1]
                ex.reduce(acc, sG[m0:m1], L["W2.scale"], L["b2"], H, N["ln1_gamma"],
                          N["ln1_beta"], self.eps)
            else:
                ex.reduce(acc, sG[m0:m1], L["W2.scale"], L["b2"], H)

    def _steps(self, tokens: torch.Tensor, ex, out: dict):
        """The whole prefill of `tokens` as a generator that pauses after each
        exchange step; leaves (next tokens, own logits) in out["result"]."""
        plan, w, k, r = self.plan, self.w, self.k, self.rank
        n_seq, T = tokens.shape
        d = plan.dims.d_model
        dh = plan.d_heads(r)
        hl = dh // HEAD_DIM
        M = n_seq * T
        s0, s1 = plan.seqs(n_seq, r)
        m0, m1 = s0 * T, s1 * T
        dev = w.wte.device
        L0 = w.layers[0]
        Xq, sX = ex.Xq, ex.sX
        # residual stream of the owned sequences; int8 LayerNorm output of all rows
        own_tok = tokens[s0:s1].contiguous().reshape(-1)
        H, _, xq, sx = k.embed_layernorm_quant(w.wte, w.wpe, own_tok, T, None, L0["ln1_gamma"],
                                               L0["ln1_beta"], self.eps)
        Xq[m0:m1].copy_(xq)
        sX[m0:m1].copy_(sx)
        ex.publish_rows()
        yield
        Kc = torch.empty((n_seq, T, dh), dtype=torch.bfloat16, device=dev)
        Vc = torch.empty_like(Kc)
        Q = torch.empty((M, dh), dtype=torch.bfloat16, device=dev)
        if self.mode == "alltoall":
            yield from self._layers_alltoall(ex, H, Q, Kc, Vc, n_seq, T, hl, dh, m0, m1)
        else:
            self._layers_partial_sums(ex, H, Q, Kc, Vc, n_seq, T, hl, dh, m0, m1)
        # final LayerNorm of each owned sequence's last position, LM head, greedy
        last = H.view(s1 - s0, T, d)[:, T - 1, :]
        Xf, _, _ = k.layernorm_quant(last, w.lnf_gamma, w.lnf_beta, self.eps, want_q=False)
        logits = k.lm_head(Xf, w.wte)
        nxt = torch.empty((n_seq,), dtype=torch.int32, device=dev)
        nxt[s0:s1].copy_(k.sample_greedy(logits))
        ex.gather_tokens(nxt)
        out["result"] = (nxt, logits)

    def run(self, tokens: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        n_seq, T = tokens.shape
        world = self.plan.world
        if self._halves and n_seq % (2 * world) == 0:
            return self._run_halves(tokens)
        ex = self._exchange(n_seq * T, self.plan.dims.d_model, self.w.wte.device)
        out = {}
        for _ in self._steps(tokens, ex, out):
            pass
        return out["result"]

    def _run_halves(self, tokens: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        n_seq, T = tokens.shape
        world, d, dev = self.plan.world, self.plan.dims.d_model, self.w.wte.device
        per = n_seq // world
        half = per // 2
        cuda = dev.type == "cuda" if isinstance(dev, torch.device) else str(dev).startswith("cuda")
        main = torch.cuda.current_stream(dev) if cuda else None
        runs = []
        for i, h in enumerate(self._halves):
            # half i: the i-th half of every rank's own sequences, rank by rank
            idx = torch.cat([torch.arange(q * per + i * half, q * per + (i + 1) * half)
                             for q in range(world)]).to(tokens.device)
            if h["ex"] is None or h["ex"].M_key != (world * half * T, d):
                h["ex"] = AllToAllExchange(self.k, h["c"], self.rank, world, world * half * T, d,
                                           dev)
                h["ex"].M_key = (world * half * T, d)
            if cuda and "stream" not in h:
                h["stream"] = torch.cuda.Stream(dev)
            stream = h.get("stream")
            if stream is not None:
                stream.wait_stream(main)
            toks = tokens.index_select(0, idx)
            out = {}
            runs.append({"idx": idx, "out": out, "stream": stream,
                         "gen": self._steps(toks, h["ex"], out)})
        live = list(runs)
        while live:
            for run in list(live):
                ctx = torch.cuda.stream(run["stream"]) if run["stream"] is not None else None
                try:
                    if ctx is not None:
                        with ctx:
                            next(run["gen"])
                    else:
                        next(run["gen"])
                except StopIteration:
                    live.remove(run)
        if cuda:
            for run in runs:
                main.wait_stream(run["stream"])
        nxt = torch.empty((n_seq,), dtype=torch.int32, device=dev)
        for run in runs:
            nxt.index_copy_(0, run["idx"], run["out"]["result"][0])
        logits = torch.cat([run["out"]["result"][1] for run in runs])
        return nxt, logits


EXCHANGE_TEXT = {
    "alltoall": "int8 inputs of attn_proj / W2 to the rows' owners by all-to-all + int8 "
                "all-gather + fp32 max-allreduce (NCCL)",
    "collective": "int32 reduce-scatter + int8 all-gather + fp32 max-allreduce (NCCL)",
    "peer": "int32 partial sums stored into the owners' memory by the GEMM epilogue, int8 rows "
            "broadcast by the LayerNorm kernel, fp32 row maxima, over NVLink peer memory",
}


def main(argv=None) -> None:
    """Time the tensor-parallel prefill of GPT-2 large, 32 x 1024 tokens:
    python -m torch.distributed.run --nproc-per-node G --master-addr 127.0.0.1 \\
        -m c_gpt2_b200.tp [--n-seq 32] [--tokens 1024] [--steps 3] [--warmup 3]
    Prints one JSON line on rank 0 (device time, max over ranks)."""
    import argparse
    import json
    from datetime import timedelta

    from .dp import dist_env, max_over_ranks
    from .quant8 import DIMS, read_quant8
    from .synthetic import prompts, quant8_image_gpu

    ap = argparse.ArgumentParser()
    ap.add_argument("--n-seq", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=None, help="fewer layers (smoke runs only)")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--exchange", choices=["alltoall", "collective", "peer"], default="alltoall")
    ap.add_argument("--halves", action="store_true",
                    help="alltoall: run the batch as two interleaved halves")
    a = ap.parse_args(argv)
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=300))
    ops.init(local)
    dims = DIMS["large"]
    if a.layers:
        dims = GPT2Dims(dims.d_model, a.layers, dims.n_head, dims.vocab, dims.ctx)
    img = quant8_image_gpu(dims, seed=0, device=dev)
    plan = TPPlan.make(dims, world)
    shard = shard_weights(read_quant8(img, dims), plan, rank, dev)
    del img
    P = torch.from_numpy(prompts(a.n_seq, a.tokens, dims.vocab, seed=0)).to(dev)
    tp = TPPrefill(plan, shard, rank, exchange=a.exchange if world > 1 else "collective",
                   halves=a.halves)
    for _ in range(a.warmup):
        tp.run(P)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        nxt, _ = tp.run(P)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, dev)
    if world > 1:
        dist.barrier()
    M = a.n_seq * a.tokens
    gemm_ops = 2.0 * M * 12 * dims.d_model ** 2 * dims.n_layer
    if rank == 0:
        print(json.dumps({
            "workload": f"gpt2-large W8A8 prefill {a.n_seq} x {a.tokens} tokens, "
                        f"{dims.n_layer} layers, tensor-parallel tp{world}",
            "n_gpus": world, "ms_per_prefill": round(ms, 3),
            "tok_per_s": round(M / (ms / 1e3), 1),
            "gemm_tops_effective": round(gemm_ops / (ms / 1e3) / 1e12, 1),
            "exchange": EXCHANGE_TEXT[a.exchange if world > 1 else "collective"],
            "steps": a.steps, "warmup": a.warmup,
            "first_tokens": nxt[:4].tolist()}))
    tp.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
