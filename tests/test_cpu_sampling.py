"""The oracle's top-k sampling against the reference's own top_k_sample
(gpt2.c:130-180), compiled from the reference tree with bf16 activations as
in its GPU build (oracle/_ref/libref_host_bf16.so), and the draw loop of
gpt2.c:2231-2245 restated step by step.

The reference sorts with qsort, which leaves the order of equal
probabilities unspecified; everything else is compared bit for bit: the
probability at every sorted position, the renormalised bf16 values and the
set of tokens above the k-th probability."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
V = 50257


def _ref_host():
    path = ROOT / "oracle" / "_ref" / "libref_host_bf16.so"
    if not path.exists():
        pytest.skip(f"{path.name} not built (make -C oracle ref needs the reference tree)")
    lib = C.CDLL(str(path))
    lib.top_k_sample.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.top_k_sample.restype = None
    return lib


def _ref_top_k(lib, probs, k):
    p = np.ascontiguousarray(probs, np.uint16)
    n = p.size
    kk = n if (k <= 0 or k > n) else k
    idx = np.full((n,), -1, np.int32)
    q = np.zeros((n,), np.uint16)
    lib.top_k_sample(p.ctypes.data, n, k, idx.ctypes.data, q.ctypes.data)
    return idx[:kk], q[:kk]


def _draw(idx, q, r):
    """gpt2.c:2231-2245 over the outputs of top_k_sample."""
    cum = np.float32(0.0)
    r = np.float32(r)
    q32 = oracle.bf16_to_f32(q)
    for i in range(len(idx)):
        cum = np.float32(cum + q32[i])
        if r < cum:
            return int(idx[i])
    return int(idx[-1])


def _rows():
    rng = np.random.default_rng(11)
    rows = []
    for temp in (0.7, 1.0, 1.6):
        lg = oracle.bf16_bits(rng.standard_normal(V).astype(np.float32) * 3.0)
        rows.append(("normal", oracle.softmax_row(lg, temp)))
    # few distinct logits: long runs of equal probabilities
    lg = oracle.bf16_bits(np.round(rng.standard_normal(V) * 2.0).astype(np.float32))
    rows.append(("ties", oracle.softmax_row(lg, 1.0)))
    # one dominant token, the rest underflowing to zero
    lg = np.full(V, oracle.bf16_bits(np.float32([-200.0]))[0], np.uint16)
    lg[12345] = oracle.bf16_bits(np.float32([30.0]))[0]
    rows.append(("spike", oracle.softmax_row(lg, 1.0)))
    # all probabilities zero: the uniform fallback
    rows.append(("zeros", np.zeros(V, np.uint16)))
    return rows


@pytest.mark.parametrize("k", [1, 40, 640, V])
def test_top_k_matches_reference(k):
    lib = _ref_host()
    for name, p in _rows():
        ri, rq = _ref_top_k(lib, p, k)
        oi, oq = oracle.top_k(p, k)
        np.testing.assert_array_equal(rq, oq, err_msg=f"{name}: renormalised probabilities")
        np.testing.assert_array_equal(p[ri], p[oi], err_msg=f"{name}: sorted probabilities")
        assert len(set(ri.tolist())) == len(ri)
        edge = p[oi[-1]]  # tokens strictly above the k-th probability are the same set
        assert set(ri[p[ri] != edge].tolist()) == set(oi[p[oi] != edge].tolist()), name


def test_draw_matches_reference_loop():
    lib = _ref_host()
    libc = C.CDLL(None)
    libc.srand(1)  # the reference never seeds rand(): glibc starts at seed 1
    draws = [np.float32(libc.rand()) / np.float32(2147483647) for _ in range(6)]
    for k in (1, 40, 640):
        for name, p in _rows():
            ri, rq = _ref_top_k(lib, p, k)
            oi, oq = oracle.top_k(p, k)
            cum = np.cumsum(oracle.bf16_to_f32(oq), dtype=np.float32)  # sequential in fp32
            rs = draws + [0.0, 1.0, cum[0], np.nextafter(cum[0], np.float32(0)),
                          cum[len(cum) // 2]]
            for r in rs:
                want = _draw(ri, rq, r)
                got = oracle.sample_topk(p, k, r)
                assert p[got] == p[want], (name, k, r)  # the same probability ...
                if name != "zeros" and np.count_nonzero(p == p[want]) == 1:
                    assert got == want  # ... and the same token where it is unique


def test_top_k_clamps_k():
    p = oracle.softmax_row(oracle.bf16_bits(np.linspace(-3, 3, 100).astype(np.float32)), 1.0)
    # gpt2.c:1963-1968: top_k < 1 -> 1, top_k > vocab -> vocab
    assert oracle.sample_topk(p, 0, 0.5) == oracle.sample_topk(p, 1, 0.5) == 99
    i_all, _ = oracle.top_k(p, 10**6)
    assert len(i_all) == 100


def test_reference_draws_are_glibc_rand():
    """gpt2_reference_draws reproduces the reference's r = (float)rand() /
    RAND_MAX (gpt2.c:2231) from its own generator state."""
    from c_gpt2_b200.engine import Engine

    libc = C.CDLL(None)
    for seed in (1, 7, 123456789):
        libc.srand(seed)
        want = np.array([np.float32(libc.rand()) / np.float32(2147483647) for _ in range(2000)],
                        np.float32)
        got = Engine.reference_draws(2000, seed)
        np.testing.assert_array_equal(got, want)
        assert got.min() >= 0.0 and got.max() <= 1.0
    # the process's own rand() stream is untouched by the helper
    libc.srand(5)
    a = [libc.rand() for _ in range(3)]
    libc.srand(5)
    libc.rand()
    Engine.reference_draws(10, 5)
    assert [libc.rand(), libc.rand()] == a[1:]
    assert Engine.reference_draws(0).size == 0
