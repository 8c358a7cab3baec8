"""Top-k sampling at a temperature on the GPU (w8a8_sample_topk) against the
oracle (gpt2.c:130-180 and 2223-2245) and against the reference's own
softmax_cuda kernel for the probabilities it samples from.

The kernel exposes the bf16 probabilities it forms; the token it draws must
equal the oracle's draw from those probabilities exactly (both put the lower
index first among equal probabilities), and the probabilities must equal the
reference kernel's softmax_cuda output bit for bit (same device math)."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from c_gpt2_b200 import _lib, ops
from oracle import oracle
from tests.gpu_util import bf16_ulp_diff, from_dev_bf16, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _logits(rng, M, V, kind):
    if kind == "normal":
        x = rng.standard_normal((M, V)).astype(np.float32) * 3.0
    elif kind == "ties":  # few distinct logits: long runs of equal probabilities
        x = np.round(rng.standard_normal((M, V)) * 2.0).astype(np.float32)
    else:  # "peaked": a handful of large logits over a flat floor
        x = np.zeros((M, V), np.float32)
        for m in range(M):
            x[m, rng.choice(V, 5, replace=False)] = rng.uniform(8, 12, 5)
    return oracle.bf16_bits(x)


def _sample(lg_bits, temp, k, r):
    M, V = lg_bits.shape
    probs = torch.zeros((M, V), dtype=torch.bfloat16, device="cuda:0")
    toks = ops.sample_topk(to_dev_bf16(lg_bits), temp, k, to_dev(np.asarray(r, np.float32)),
                           probs_out=probs)
    return toks.cpu().numpy(), from_dev_bf16(probs)


@pytest.mark.parametrize("kind", ["normal", "ties", "peaked"])
@pytest.mark.parametrize("temp", [0.7, 1.0, 1.6])
def test_topk_tokens_match_oracle(cuda, kind, temp):
    seed = {"normal": 100, "ties": 200, "peaked": 300}[kind] + int(temp * 10)
    rng = np.random.default_rng(seed)
    M, V = 6, 50257
    lg = _logits(rng, M, V, kind)
    want_p = [oracle.softmax_row(lg[m], temp) for m in range(M)]
    for k in (1, 40, 640, V):
        r = rng.random(M, dtype=np.float32)
        toks, probs = _sample(lg, temp, k, r)
        for m in range(M):
            # expf on the GPU against the C library's: within one bf16 ulp
            assert bf16_ulp_diff(probs[m], want_p[m]).max() <= 1
            assert toks[m] == oracle.sample_topk(probs[m], k, r[m]), (kind, temp, k, m)


def test_topk_draw_boundaries(cuda):
    """r exactly at a running sum of the renormalised probabilities takes the
    next token (gpt2.c:2236 tests r < cum); one float below it, this one."""
    rng = np.random.default_rng(3)
    V, k = 50257, 40
    lg = _logits(rng, 1, V, "normal")
    _, probs = _sample(lg, 1.0, k, [0.5])
    idx, q = oracle.top_k(probs[0], k)
    cum = np.cumsum(oracle.bf16_to_f32(q), dtype=np.float32)
    rs, want = [], []
    for i in (0, 1, 7, k - 2):
        rs += [cum[i], np.nextafter(cum[i], np.float32(0))]
        want += [idx[i + 1], idx[i]]
    # r = 1.0 may fall below the last running sum (the bf16 values can add up
    # to a little over 1); r equal to the last running sum never does
    rs += [0.0, 1.0, cum[-1]]
    want += [idx[0], oracle.sample_topk(probs[0], k, 1.0), idx[-1]]
    lg_rep = np.repeat(lg, len(rs), axis=0)
    toks, _ = _sample(lg_rep, 1.0, k, rs)
    assert list(toks) == [int(w) for w in want]


def test_topk_probabilities_match_reference_softmax(cuda):
    """The probabilities the sampler draws from are softmax_cuda's
    (cuda/softmax.cu) at the same temperature, bit for bit."""
    path = ROOT / "oracle" / "_ref" / "libref_kernels_small.so"
    if not path.exists():
        pytest.skip(f"{path.name} not built (make -C oracle ref needs the reference tree)")
    ref = C.CDLL(str(path))
    ref.softmax_cuda.argtypes = _lib.COMPAT_SIGNATURES["softmax_cuda"]
    ref.softmax_cuda.restype = None
    rng = np.random.default_rng(9)
    M, V = 4, 50257
    lg = _logits(rng, M, V, "normal")
    for temp in (0.5, 0.9, 1.0, 2.0):
        _, probs = _sample(lg, temp, 40, np.zeros(M, np.float32))
        a = to_dev_bf16(lg)
        ref.softmax_cuda(a.data_ptr(), M, V, V, a.data_ptr(), temp, 0)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(probs, from_dev_bf16(a))


def test_topk_k1_and_zero_temperature_are_greedy(cuda):
    rng = np.random.default_rng(4)
    M, V = 8, 50257
    lg = _logits(rng, M, V, "ties")
    greedy = ops.sample_greedy(to_dev_bf16(lg)).cpu().numpy()
    r = rng.random(M, dtype=np.float32)
    # top-1 at temperature 1: the largest probability, lowest index first
    assert list(_sample(lg, 1.0, 1, r)[0]) == list(greedy)
    # temperature <= 0 is greedy decoding (gpt2.c:2212)
    assert list(_sample(lg, 0.0, 40, r)[0]) == list(greedy)


def test_topk_small_vocab_and_uniform_fallback(cuda):
    rng = np.random.default_rng(6)
    for V in (1, 7, 300, 4099):
        M = 3
        lg = _logits(rng, M, V, "normal")
        for k in (1, 5, V):
            r = rng.random(M, dtype=np.float32)
            toks, probs = _sample(lg, 1.3, k, r)
            for m in range(M):
                assert 0 <= toks[m] < V
                assert toks[m] == oracle.sample_topk(probs[m], k, r[m])


def test_topk_appends_with_per_row_draw_positions(cuda):
    """The decode-loop form: r read at rnd[m, rnd_pos[m]], the token stored at
    append_to[m, append_pos[m]] and append_pos advanced."""
    rng = np.random.default_rng(8)
    M, V, S, k, temp = 5, 50257, 16, 40, 0.8
    lg = _logits(rng, M, V, "normal")
    rnd = rng.random((M, S), dtype=np.float32)
    pos = np.array([0, 3, 15, 7, 1], np.int32)
    d_lg, d_rnd, d_pos = to_dev_bf16(lg), to_dev(rnd), to_dev(pos)
    d_app = torch.full((M, S), -1, dtype=torch.int32, device="cuda:0")
    d_out = torch.empty((M,), dtype=torch.int32, device="cuda:0")
    probs = torch.zeros((M, V), dtype=torch.bfloat16, device="cuda:0")
    ops.check(ops.core().w8a8_sample_topk(
        d_lg.data_ptr(), V, M, V, temp, k, d_rnd.data_ptr(), S, d_pos.data_ptr(),
        d_out.data_ptr(), d_app.data_ptr(), S, d_pos.data_ptr(), probs.data_ptr(), V,
        torch.cuda.current_stream().cuda_stream), "w8a8_sample_topk")
    toks, app, new_pos = d_out.cpu().numpy(), d_app.cpu().numpy(), d_pos.cpu().numpy()
    p = from_dev_bf16(probs)
    np.testing.assert_array_equal(new_pos, pos + 1)
    for m in range(M):
        assert toks[m] == oracle.sample_topk(p[m], k, rnd[m, pos[m]])
        assert app[m, pos[m]] == toks[m]
        assert (np.delete(app[m], pos[m]) == -1).all()


def test_topk_rejects_bad_arguments(cuda):
    lib = ops.core()
    x = torch.zeros((2, 90000), dtype=torch.bfloat16, device="cuda:0")
    r = torch.zeros((2,), dtype=torch.float32, device="cuda:0")
    o = torch.zeros((2,), dtype=torch.int32, device="cuda:0")
    s = torch.cuda.current_stream().cuda_stream
    # vocabulary above the kernel's shared-memory capacity: refused before any launch
    assert lib.w8a8_sample_topk(x.data_ptr(), 90000, 2, 90000, 1.0, 40, r.data_ptr(), 1, None,
                                o.data_ptr(), None, 0, None, None, 0, s) == _lib.W8A8_ERR_UNSUPPORTED
    # no draws for a positive temperature; a row stride below the vocabulary
    assert lib.w8a8_sample_topk(x.data_ptr(), 90000, 2, 50257, 1.0, 40, None, 1, None,
                                o.data_ptr(), None, 0, None, None, 0, s) == _lib.W8A8_ERR_INVALID
    assert lib.w8a8_sample_topk(x.data_ptr(), 100, 2, 50257, 1.0, 40, r.data_ptr(), 1, None,
                                o.data_ptr(), None, 0, None, None, 0, s) == _lib.W8A8_ERR_INVALID
    assert lib.w8a8_sample_topk(x.data_ptr(), 90000, 0, 50257, 1.0, 40, r.data_ptr(), 1, None,
                                o.data_ptr(), None, 0, None, None, 0, s) == 0


def test_reference_abi_lm_head_picks(cuda):
    """lm_head_greedy_cuda and lm_head_topk_cuda (include/cuda_kernels.h, the
    per-size drop-in library) give the LM head's logits and the token that the
    runtime ABI's w8a8_lm_head + sampler give on the same buffers."""
    lib = _lib.compat("small")
    d, V = 768, 50257
    rng = np.random.default_rng(12)
    xf = to_dev_bf16(oracle.bf16_bits(rng.standard_normal(d).astype(np.float32)))
    wte = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((V, d)).astype(np.float32) * 0.08))
    want_logits = ops.lm_head(xf[None], wte)
    logits = torch.zeros((V,), dtype=torch.bfloat16, device="cuda:0")
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    lib.lm_head_greedy_cuda(xf.data_ptr(), wte.data_ptr(), logits.data_ptr(), tok.data_ptr())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(from_dev_bf16(logits), from_dev_bf16(want_logits[0]))
    assert tok.item() == ops.sample_greedy(want_logits).item()
    for temp, k, r in ((0.8, 40, 0.3), (1.3, 1000, 0.77), (0.6, 1, 0.5), (0.0, 40, 0.5)):
        r_d = torch.tensor([r], dtype=torch.float32, device="cuda:0")
        logits.zero_()
        lib.lm_head_topk_cuda(xf.data_ptr(), wte.data_ptr(), logits.data_ptr(), temp, k,
                              r_d.data_ptr(), tok.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(from_dev_bf16(logits), from_dev_bf16(want_logits[0]))
        probs = torch.zeros((1, V), dtype=torch.bfloat16, device="cuda:0")
        want = ops.sample_topk(want_logits, temp, k, r_d, probs_out=probs).item()
        assert tok.item() == want, (temp, k, r)
        if temp > 0:
            assert want == oracle.sample_topk(from_dev_bf16(probs)[0], k, r)


def test_topk_flat_row_ranks_across_the_cluster(cuda):
    """Every logit equal: one probability key held by all 50257 entries (the
    largest per-key count), so the drawn rank among equal probabilities runs
    across the CTAs that share the row; and a row with a single finite
    maximum among equal floor values."""
    V = 50257
    flat = np.zeros((4, V), np.float32)
    flat[2:, :] = -3.0
    flat[3, 31337] = 5.0
    lg = oracle.bf16_bits(flat)
    for k in (40, 20000, V):
        r = np.array([0.0, 0.999, 0.5, 0.25], np.float32)
        toks, probs = _sample(lg, 1.0, k, r)
        for m in range(4):
            assert toks[m] == oracle.sample_topk(probs[m], k, r[m]), (k, m)


def test_topk_vocab_above_the_cluster_kernel(cuda):
    """65536..81920 entries take the one-CTA kernel (the cluster kernel's
    per-key counts are 16 bits wide)."""
    rng = np.random.default_rng(12)
    M, V = 2, 70000
    lg = _logits(rng, M, V, "normal")
    for k in (40, V):
        r = rng.random(M, dtype=np.float32)
        toks, probs = _sample(lg, 0.9, k, r)
        for m in range(M):
            assert toks[m] == oracle.sample_topk(probs[m], k, r[m])
