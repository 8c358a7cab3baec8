"""Full-size stream parity against the oracle: the benchmark's own GPT-2 large
model and prompts, and GPT-2 medium with a 512-token prompt.

GPT-2 large: 36 layers, the seed-0 weights drawn as the benchmark draws them
(torch's seeded CUDA generator, then the reference's per-channel
quantization), the benchmark's seed-0 512-token prompts, at the per-GPU batch
of the 1-GPU run (64 sequences) and of the 8-GPU run (8 sequences). A few
sequences of each batch are compared with the oracle's stream for that prompt
alone (gpt2.c:2094-2247, the INT8 forward of gpt2.c:1124-1330).

The bar. The reference leaves the fp32 order of the attention and LM-head
sums to cuBLAS, so the oracle is run twice: in ascending index order and in
descending order (oracle.generate_steps(..., sum_order=1)), both equally
valid readings of the reference. On these random-weight models with 512-token
prompts the two already differ by up to ~0.1 in single logits (mean ~0.018):
a rounding difference anywhere flips int8 activations that the next layers
amplify. The GPU must stay inside that spread:

* every step, up to and including the first step where the streams differ:
  mean |GPU - oracle| <= max(2e-2, 1.25 x the oracle's own mean spread) and
  max |GPU - oracle| <= max(0.1, 1.25 x its max spread) (2e-2 is the logit
  tolerance the task states);
* at the first differing step, the GPU's token is a numerical tie: its oracle
  logit is below the oracle's best by no more than the oracle's own max
  spread at that step (at least one bf16 ulp).
"""
import numpy as np
import pytest
import torch

from c_gpt2_b200.engine import Engine
from c_gpt2_b200.quant8 import DIMS
from c_gpt2_b200.synthetic import prompts, quant8_image_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

N_SEQ, PROMPT = 64, 512      # the benchmark's workload
N_GEN_LARGE = 8
N_GEN_MEDIUM = 64


def engine_steps(eng, P, n_gen, rows, device):
    """Greedy tokens [B, n_gen] of a batched prefill + decode steps, and the
    logits [len(rows), n_gen, vocab] (float32) every token of `rows` was
    picked from."""
    B = P.shape[0]
    pd = torch.from_numpy(np.ascontiguousarray(P)).to(device)
    out = torch.zeros((B, n_gen), dtype=torch.int32, device=device)
    eng.prefill(pd, out, n_gen)
    lg = [eng.logits(B)[rows]]
    for _ in range(n_gen - 1):
        eng.decode_steps(1)
        lg.append(eng.logits(B)[rows])
    torch.cuda.synchronize()
    return out.cpu().numpy(), np.stack(lg, 1)


class OracleStream:
    """The oracle's stream in both summation orders and their spread."""

    def __init__(self, img, dims, prompt, n_gen):
        self.tokens, bits = oracle.generate_steps(img, dims, prompt, n_gen)
        alt_tokens, alt_bits = oracle.generate_steps(img, dims, prompt, n_gen, sum_order=1)
        self.logits = oracle.bf16_to_f32(bits)
        alt = oracle.bf16_to_f32(alt_bits)
        d = np.nonzero(alt_tokens != self.tokens)[0]
        sync = int(d[0]) + 1 if d.size else n_gen  # steps whose contexts agree
        e = np.abs(alt[:sync] - self.logits[:sync])
        self.spread_max = e.max(axis=1)            # per step
        self.spread_mean = e.mean(axis=1)

    def spread_at(self, s):
        s = min(s, len(self.spread_max) - 1)
        return float(self.spread_max[s]), float(self.spread_mean[s])


def compare_stream(tokens, logits, ref: OracleStream, label=""):
    """Returns (identical leading tokens, largest logit error up to there)."""
    n = len(ref.tokens)
    diff = np.nonzero(tokens != ref.tokens)[0]
    g = int(diff[0]) if diff.size else n
    worst = 0.0
    for s in range(min(g + 1, n)):  # the contexts agree through step g
        sp_max, sp_mean = ref.spread_at(s)
        e = np.abs(logits[s] - ref.logits[s])
        assert e.mean() <= max(2e-2, 1.25 * sp_mean), (label, s, e.mean(), sp_mean)
        assert e.max() <= max(0.1, 1.25 * sp_max), (label, s, e.max(), sp_max)
        worst = max(worst, float(e.max()))
    if g < n:
        w = ref.logits[g]
        best = w.max()
        ulp = np.float32(2.0) ** (np.floor(np.log2(abs(best))) - 7)
        gap = best - w[tokens[g]]
        assert gap <= max(ulp, ref.spread_at(g)[0]), (
            f"{label} step {g}: GPU token {tokens[g]} is {gap} below the oracle's best "
            f"{ref.tokens[g]} (spread {ref.spread_at(g)[0]})")
    print(f"{label}: {g}/{n} identical tokens, max |dlogit| {worst:.4f}")
    return g, worst


@pytest.fixture(scope="module")
def large(cuda):
    dims = DIMS["large"]
    img = quant8_image_gpu(dims, seed=0, device=cuda)
    P = prompts(N_SEQ, PROMPT, dims.vocab, seed=0)
    cache = {}

    def want(b):
        if b not in cache:
            cache[b] = OracleStream(img, dims, P[b], N_GEN_LARGE)
        return cache[b]

    eng = Engine(dims, max_batch=N_SEQ, max_tokens=N_SEQ * PROMPT)
    eng.load_quant8(img)
    yield dims, eng, P, want
    eng.close()


@pytest.mark.parametrize("batch,rows", [(64, [0, 42, 63]), (8, [0, 7])])
def test_gpt2_large_benchmark_streams(cuda, large, batch, rows):
    """The benchmark's model and prompts at the per-GPU batches of 1 and 8 GPUs."""
    dims, eng, P, want = large
    toks, lg = engine_steps(eng, P[:batch], N_GEN_LARGE, rows, cuda)
    for i, b in enumerate(rows):
        compare_stream(toks[b], lg[i], want(b), f"large batch {batch} seq {b}")


def test_gpt2_large_batch_sizes_agree(cuda, large):
    """The first 8 sequences decoded in a batch of 64 and in a batch of 8 (the
    1-GPU and 8-GPU shards). Decode attention sums P.V in a different fp32
    order at the two batch sizes, so a sequence may leave the other's stream
    only where both stay within the oracle's spread (checked against the
    oracle for every sequence whose streams differ)."""
    dims, eng, P, want = large
    rows = list(range(8))
    t64, l64 = engine_steps(eng, P, N_GEN_LARGE, rows, cuda)
    t8, l8 = engine_steps(eng, P[:8], N_GEN_LARGE, rows, cuda)
    same = 0
    for b in rows:
        if np.array_equal(t64[b], t8[b]):
            same += 1
            continue
        compare_stream(t64[b], l64[b], want(b), f"batch 64 seq {b}")
        compare_stream(t8[b], l8[b], want(b), f"batch 8 seq {b}")
    print(f"batch 64 vs 8: {same}/8 sequences identical")


def test_gpt2_medium_prompt512(cuda):
    """GPT-2 medium, batch 1: a 512-token prompt, then greedy tokens, every
    step's logits against the oracle."""
    dims = DIMS["medium"]
    img = quant8_image_gpu(dims, seed=0, device=cuda)
    P = prompts(1, PROMPT, dims.vocab, seed=3)
    eng = Engine(dims, max_batch=1, max_tokens=PROMPT)
    eng.load_quant8(img)
    toks, lg = engine_steps(eng, P, N_GEN_MEDIUM, [0], cuda)
    eng.close()
    compare_stream(toks[0], lg[0], OracleStream(img, dims, P[0], N_GEN_MEDIUM), "medium")
