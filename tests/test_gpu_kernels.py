"""GPU parity of the sm_100a kernels against the CPU oracle (same seeded
inputs). Integer and quantization results are bit-exact; bf16 outputs that
pass through CUDA's tanhf/rsqrtf/expf or through reordered fp32 sums are
checked within the tolerance written in each test."""
import numpy as np
import pytest
import torch

from c_gpt2_b200 import _lib, ops
from c_gpt2_b200.synthetic import outlier_activations
from oracle import oracle
from tests.gpu_util import bf16_ulp_diff, from_dev_bf16, kernel_names_fresh, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu


def _rand_bf16(rng, shape, scale=1.0):
    return oracle.bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(scale))


@pytest.mark.parametrize("M,K", [(1, 768), (7, 3072), (64, 5120), (333, 1024), (5, 100),
                                 (3, 8), (1024, 768), (1024, 5120), (2048, 1280), (1024, 4104)])
def test_quant_rows_bit_exact(cuda, M, K):
    rng = np.random.default_rng(M * 7 + K)
    x = outlier_activations(M, K, seed=M + K)
    if M > 2:
        x[1] = 0.0  # zero row
    xb = oracle.bf16_bits(x)
    xq, sx = ops.per_token_quant(to_dev_bf16(xb))
    rq, rs = oracle.quant_rows(xb)
    np.testing.assert_array_equal(xq.cpu().numpy(), rq)
    np.testing.assert_array_equal(sx.cpu().numpy().view(np.uint32), rs.view(np.uint32))


# (M, N, K): decode GEMV (M < 16), tensor-core tiles with ragged M/N, K not a
# multiple of 128, and the CUDA-core fallback (K % 16 != 0).
GEMM_SHAPES = [(1, 768, 768), (4, 2304, 768), (15, 3072, 1024), (16, 768, 768),
               (33, 200, 768), (64, 5120, 1280), (100, 1280, 5120), (128, 2304, 768),
               (200, 384, 192), (257, 640, 768), (1024, 1024, 1024), (40, 96, 80),
               (20, 72, 40), (3, 130, 56)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_s32_bit_exact(cuda, M, N, K):
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    Y = ops.gemm_s32(to_dev(xq), to_dev(W)).cpu().numpy()
    np.testing.assert_array_equal(Y, oracle.gemm_s32(xq, W))


def test_gemm_s32_extreme_values(cuda):
    # |acc| up to 127*127*5120 = 8.3e7: still exact int32
    M, N, K = 32, 256, 5120
    xq = np.full((M, K), 127, np.int8)
    W = np.full((N, K), -127, np.int8)
    W[::2] = 127
    Y = ops.gemm_s32(to_dev(xq), to_dev(W)).cpu().numpy()
    np.testing.assert_array_equal(Y, oracle.gemm_s32(xq, W))


@pytest.mark.parametrize("M,N,K", [(1, 2304, 768), (9, 768, 3072), (16, 2304, 768),
                                   (128, 3072, 768), (300, 768, 3072), (1024, 2304, 768),
                                   (300, 320, 768), (129, 96, 256), (1, 1280, 5120),
                                   (1, 200, 3072), (1, 5120, 1280), (257, 288, 4736),
                                   (600, 1280, 5120), (256, 256, 64)])
@pytest.mark.parametrize("epi", [_lib.EPI_DEQUANT, _lib.EPI_BIAS, _lib.EPI_BIAS_RESID])
def test_linear_epilogues_bit_exact(cuda, M, N, K, epi):
    rng = np.random.default_rng(M + N + K + epi)
    x = oracle.bf16_bits(outlier_activations(M, K, seed=epi + M))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = _rand_bf16(rng, (N,), 0.02)
    R = _rand_bf16(rng, (M, N))
    want = oracle.linear(xq, sx, W, sw, b, epi, R if epi == _lib.EPI_BIAS_RESID else None)
    out = ops.linear(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b), epi,
                     R=to_dev_bf16(R) if epi == _lib.EPI_BIAS_RESID else None)
    np.testing.assert_array_equal(from_dev_bf16(out), want)


@pytest.mark.parametrize("M,N,K", [(16, 768, 768), (64, 1280, 5120), (64, 3840, 1280),
                                   (33, 5120, 1280), (100, 200, 3072)])
@pytest.mark.parametrize("epi", [_lib.EPI_BIAS, _lib.EPI_BIAS_RESID])
def test_linear_split_k_bit_exact(cuda, M, N, K, epi):
    """Decode-sized GEMMs split K over the SMs and meet in an int32 workspace
    through integer atomics: exact in any order. Two calls in a row check that
    the workspace is left zeroed."""
    rng = np.random.default_rng(M * N + K)
    x = oracle.bf16_bits(outlier_activations(M, K, seed=M + epi))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = _rand_bf16(rng, (N,), 0.02)
    R = _rand_bf16(rng, (M, N))
    Rr = R if epi == _lib.EPI_BIAS_RESID else None
    want = oracle.linear(xq, sx, W, sw, b, epi, Rr)
    ws = ops.linear_workspace(M, N, cuda)
    args = (to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b), epi)
    for _ in range(2):
        out = ops.linear(*args, R=to_dev_bf16(R) if Rr is not None else None, workspace=ws)
        np.testing.assert_array_equal(from_dev_bf16(out), want)
    assert not ws.any(), "workspace not returned to zero"


@pytest.mark.parametrize("B", [20, 8, 3])
def test_linear_qkv_scatter_split_k(cuda, B):
    """Packed QKV GEMM writing Q rows and K/V cache rows at per-sequence
    positions (decode: one token per sequence), split over K, at batch sizes
    20, 8 and 3."""
    rng = np.random.default_rng(11 + B)
    d, C = 768, 64
    x = oracle.bf16_bits(outlier_activations(B, d, seed=4))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (3 * d, d), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, 3 * d).astype(np.float32)
    b = _rand_bf16(rng, (3 * d,), 0.02)
    want = oracle.linear(xq, sx, W, sw, b, oracle.EPI_BIAS)
    pos = rng.integers(0, C, B).astype(np.int32)
    Q = torch.zeros((B, d), dtype=torch.bfloat16, device=cuda)
    Kc = torch.zeros((B, C, d), dtype=torch.bfloat16, device=cuda)
    Vc = torch.zeros((B, C, d), dtype=torch.bfloat16, device=cuda)
    ws = ops.linear_workspace(B, 3 * d, cuda)
    ops.linear_qkv(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b), Q, Kc, Vc,
                   C * d, 1, to_dev(pos), workspace=ws)
    q, k, v = from_dev_bf16(Q), from_dev_bf16(Kc), from_dev_bf16(Vc)
    np.testing.assert_array_equal(q, want[:, :d])
    for i in range(B):
        np.testing.assert_array_equal(k[i, pos[i]], want[i, d:2 * d])
        np.testing.assert_array_equal(v[i, pos[i]], want[i, 2 * d:])
        other = np.delete(np.arange(C), pos[i])
        assert not k[i, other].any() and not v[i, other].any()


@pytest.mark.parametrize("zero_acc", [True, False])
@pytest.mark.parametrize("M,K", [(256, 128), (256, 5120), (64, 128)])
def test_linear_resid_bf16_edge_values(cuda, zero_acc, M, K):
    """Bias and residual additions at the edges of bf16: subnormals, signed
    zeros, the largest finite values and infinities (token-major tiles at 256
    tokens, on CTA pairs with K = 5120, the cluster split-K path at 64). With
    zero weights every dequantized product is +0, so the sums see the edge
    values themselves; with random weights tiny biases meet normal values."""
    rng = np.random.default_rng(21 + zero_acc)
    N = 512
    x = oracle.bf16_bits(outlier_activations(M, K, seed=9))
    xq, sx = oracle.quant_rows(x)
    W = (np.zeros((N, K), np.int8) if zero_acc
         else rng.integers(-127, 128, (N, K), dtype=np.int8))
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    edge = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x007F, 0x807F, 0x0080, 0x8080, 0x7F7F,
                     0xFF7F, 0x3F80, 0xBF80], np.uint16)
    b = _rand_bf16(rng, (N,), 0.02)
    b[: 4 * len(edge)] = np.tile(edge, 4)
    R = _rand_bf16(rng, (M, N))
    pick = rng.random((M, N)) < 0.3
    R[pick] = rng.choice(np.r_[edge, [0x7F80, 0xFF80]].astype(np.uint16), pick.sum())
    # biases stay finite, so no sum is inf + -inf
    want = oracle.linear(xq, sx, W, sw, b, _lib.EPI_BIAS_RESID, R)
    got = from_dev_bf16(ops.linear(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b),
                                   _lib.EPI_BIAS_RESID, R=to_dev_bf16(R)))
    np.testing.assert_array_equal(got, want)


def test_linear_qkv_scatter_prefill(cuda):
    """Packed QKV GEMM of a prefill (token-major tiles): 3 sequences of 100
    tokens each written to Q and to K/V cache rows pos0[b] + t; tiles of 32
    rows straddle sequences."""
    rng = np.random.default_rng(12)
    B, T, d, C = 3, 100, 768, 256
    x = oracle.bf16_bits(outlier_activations(B * T, d, seed=5))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (3 * d, d), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, 3 * d).astype(np.float32)
    b = _rand_bf16(rng, (3 * d,), 0.02)
    want = oracle.linear(xq, sx, W, sw, b, oracle.EPI_BIAS)
    pos = rng.integers(0, C - T, B).astype(np.int32)
    Q = torch.zeros((B * T, d), dtype=torch.bfloat16, device=cuda)
    Kc = torch.zeros((B, C, d), dtype=torch.bfloat16, device=cuda)
    Vc = torch.zeros((B, C, d), dtype=torch.bfloat16, device=cuda)
    ops.linear_qkv(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b), Q, Kc, Vc,
                   C * d, T, to_dev(pos))
    q, k, v = from_dev_bf16(Q), from_dev_bf16(Kc), from_dev_bf16(Vc)
    np.testing.assert_array_equal(q, want[:, :d])
    for i in range(B):
        rows = slice(i * T, (i + 1) * T)
        np.testing.assert_array_equal(k[i, pos[i]:pos[i] + T], want[rows, d:2 * d])
        np.testing.assert_array_equal(v[i, pos[i]:pos[i] + T], want[rows, 2 * d:])
        other = np.r_[0:pos[i], pos[i] + T:C]
        assert not k[i, other].any() and not v[i, other].any()


def test_linear_qkv_heads_scatter_long_k(cuda):
    """QKV scatter of a head subset with a long reduction (K 4736), which
    takes the CTA-pair GEMM: 2 sequences of 150 tokens into Q and K/V cache
    rows pos0[b] + t, 128-column segments (one 256-channel unit straddles
    the Q/K boundary)."""
    rng = np.random.default_rng(31)
    B, T, K, dh, C = 2, 150, 4736, 128, 400
    x = oracle.bf16_bits(outlier_activations(B * T, K, seed=6))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (3 * dh, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, 3 * dh).astype(np.float32)
    b = _rand_bf16(rng, (3 * dh,), 0.02)
    want = oracle.linear(xq, sx, W, sw, b, oracle.EPI_BIAS)
    pos = np.array([7, 230], np.int32)
    Q = torch.zeros((B * T, dh), dtype=torch.bfloat16, device=cuda)
    Kc = torch.zeros((B, C, dh), dtype=torch.bfloat16, device=cuda)
    Vc = torch.zeros((B, C, dh), dtype=torch.bfloat16, device=cuda)
    ops.linear_qkv_heads(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b), Q, Kc, Vc,
                         C * dh, T, to_dev(pos))
    q, k, v = from_dev_bf16(Q), from_dev_bf16(Kc), from_dev_bf16(Vc)
    np.testing.assert_array_equal(q, want[:, :dh])
    for i in range(B):
        rows = slice(i * T, (i + 1) * T)
        np.testing.assert_array_equal(k[i, pos[i]:pos[i] + T], want[rows, dh:2 * dh])
        np.testing.assert_array_equal(v[i, pos[i]:pos[i] + T], want[rows, 2 * dh:])
        other = np.r_[0:pos[i], pos[i] + T:C]
        assert not k[i, other].any() and not v[i, other].any()
    assert ops.device_error(reset=True) == 0


@pytest.mark.parametrize("M,N,K", [(1, 3072, 768), (64, 5120, 1280), (512, 3072, 768),
                                   (333, 320, 768), (300, 512, 4864)])
def test_linear_gelu_within_one_ulp(cuda, M, N, K):
    """GELU uses CUDA's tanhf on the GPU and the C library's on the CPU:
    at most 1 bf16 ulp apart, almost always identical."""
    rng = np.random.default_rng(N + K)
    x = oracle.bf16_bits(outlier_activations(M, K, seed=3))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = _rand_bf16(rng, (N,), 0.02)
    want = oracle.linear(xq, sx, W, sw, b, oracle.EPI_BIAS_GELU)
    got = from_dev_bf16(ops.linear(to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw),
                                   to_dev_bf16(b), _lib.EPI_BIAS_GELU))
    ulp = bf16_ulp_diff(got, want)
    assert ulp.max() <= 1
    assert (ulp > 0).mean() < 1e-3


@pytest.mark.parametrize("M,d", [(1, 768), (37, 1024), (300, 1280), (8, 2000)])
def test_layernorm_quant(cuda, M, d):
    """LayerNorm within 1 bf16 ulp of the oracle (GPU rsqrtf vs CPU 1/sqrtf);
    quantization of the GPU's own LN output bit-exact."""
    rng = np.random.default_rng(d + M)
    x = _rand_bf16(rng, (M, d), 2.0)
    g = oracle.bf16_bits(rng.uniform(0.5, 1.5, d).astype(np.float32))
    b = _rand_bf16(rng, (d,), 0.1)
    Y, Xq, sX = ops.layernorm_quant(to_dev_bf16(x), to_dev_bf16(g), to_dev_bf16(b))
    y = from_dev_bf16(Y)
    want = oracle.layernorm(x, g, b)
    ulp = bf16_ulp_diff(y, want)
    assert ulp.max() <= 1, ulp.max()
    rq, rs = oracle.quant_rows(y)
    np.testing.assert_array_equal(Xq.cpu().numpy(), rq)
    np.testing.assert_array_equal(sX.cpu().numpy(), rs)


def test_embed_layernorm_quant(cuda):
    rng = np.random.default_rng(5)
    V, C, d, B, T = 300, 64, 768, 3, 5
    wte = _rand_bf16(rng, (V, d), 0.02)
    wpe = _rand_bf16(rng, (C, d), 0.02)
    g = oracle.bf16_bits(np.ones(d, np.float32))
    b = oracle.bf16_bits(np.zeros(d, np.float32))
    toks = rng.integers(0, V, B * T).astype(np.int32)
    pos0 = np.array([0, 7, 40], np.int32)
    H, Y, Xq, sX = ops.embed_layernorm_quant(to_dev_bf16(wte), to_dev_bf16(wpe), to_dev(toks), T,
                                             to_dev(pos0), to_dev_bf16(g), to_dev_bf16(b))
    pos = (pos0[:, None] + np.arange(T)[None]).reshape(-1)
    h = oracle.bf16_bits(oracle.bf16_to_f32(wte)[toks] + oracle.bf16_to_f32(wpe)[pos])
    np.testing.assert_array_equal(from_dev_bf16(H), h)
    assert bf16_ulp_diff(from_dev_bf16(Y), oracle.layernorm(h, g, b)).max() <= 1


def _attn_case(rng, n_seq, T_ctx, H):
    d = 64 * H
    Q = _rand_bf16(rng, (n_seq, T_ctx, d))
    K = _rand_bf16(rng, (n_seq, T_ctx, d))
    V = _rand_bf16(rng, (n_seq, T_ctx, d))
    return Q, K, V


def _attn_tolerance(got, want):
    """P.V and q.k sums are reordered relative to the oracle: bf16 outputs
    within 2e-2 absolute (|O| <= max|V|, here ~4) and 99% within 2 ulp."""
    g, w = oracle.bf16_to_f32(got), oracle.bf16_to_f32(want)
    assert np.max(np.abs(g - w)) < 2e-2
    assert (bf16_ulp_diff(got, want) <= 2).mean() > 0.99


@pytest.mark.parametrize("n_seq,T,H", [(1, 1, 1), (1, 37, 2), (2, 64, 12), (3, 130, 4),
                                       (1, 512, 16), (1, 1024, 2), (2, 1000, 3), (4, 256, 20)])
def test_attention_prefill(cuda, n_seq, T, H):
    rng = np.random.default_rng(T * 13 + H)
    Q, K, V = _attn_case(rng, n_seq, T, H)
    d = 64 * H
    O = ops.attention_prefill(to_dev_bf16(Q.reshape(-1, d)), to_dev_bf16(K), to_dev_bf16(V),
                              T * d, n_seq, T, H)
    got = from_dev_bf16(O).reshape(n_seq, T, d)
    for s in range(n_seq):
        _attn_tolerance(got[s], oracle.attention(Q[s], K[s], V[s], 0, H))


@pytest.mark.parametrize("n_seq,H,lens", [(1, 16, [300]), (1, 12, [1]), (3, 2, [5, 64, 129]),
                                          (64, 20, None), (2, 20, [1024, 513])])
def test_attention_decode(cuda, n_seq, H, lens):
    rng = np.random.default_rng(n_seq * 31 + H)
    C = 1024
    lens = lens or list(rng.integers(1, C + 1, n_seq))
    d = 64 * H
    K = _rand_bf16(rng, (n_seq, C, d))
    V = _rand_bf16(rng, (n_seq, C, d))
    q = _rand_bf16(rng, (n_seq, d))
    n_ctx = np.array(lens, np.int32)
    O = ops.attention_decode(to_dev_bf16(q), to_dev_bf16(K), to_dev_bf16(V), C * d,
                             to_dev(n_ctx), C, H)
    got = from_dev_bf16(O)
    for s in range(n_seq):
        n = lens[s]
        want = oracle.attention(q[s:s + 1], K[s, :n], V[s, :n], n - 1, H)
        _attn_tolerance(got[s:s + 1], want)


@pytest.mark.parametrize("n_seq,H", [(64, 20), (2, 20), (5, 12)])
def test_attention_decode_quant_fused(cuda, n_seq, H):
    """The fused output quantization equals quant_rows of the same output, on
    two calls in a row (the per-sequence tickets must come back to zero), for
    both the one-kernel (many sequences) and the split-key path."""
    rng = np.random.default_rng(n_seq + H)
    C, d = 1024, 64 * H
    K = to_dev_bf16(_rand_bf16(rng, (n_seq, C, d)))
    V = to_dev_bf16(_rand_bf16(rng, (n_seq, C, d)))
    q = to_dev_bf16(_rand_bf16(rng, (n_seq, d)))
    n_ctx = to_dev(rng.integers(1, C + 1, n_seq).astype(np.int32))
    ws = torch.zeros((_lib.core().w8a8_attention_decode_workspace_size(n_seq, H, C),),
                     dtype=torch.uint8, device=cuda)
    want = ops.attention_decode(q, K, V, C * d, n_ctx, C, H, workspace=ws)
    want_q, want_s = ops.per_token_quant(want)
    for _ in range(2):
        O, Xq, sX = ops.attention_decode_quant(q, K, V, C * d, n_ctx, C, H, ws)
        assert torch.equal(O, want)
        assert torch.equal(Xq, want_q) and torch.equal(sX, want_s)


@pytest.mark.parametrize("M", [1, 3, 16, 64])
def test_lm_head_and_greedy(cuda, M):
    rng = np.random.default_rng(M)
    V, d = 50257, 768
    wte = _rand_bf16(rng, (V, d), 0.02)
    xf = _rand_bf16(rng, (M, d))
    logits = ops.lm_head(to_dev_bf16(xf), to_dev_bf16(wte))
    got = from_dev_bf16(logits)
    toks = ops.sample_greedy(logits).cpu().numpy()
    for m in range(M):
        want = oracle.lm_head(xf[m], wte)
        g, w = oracle.bf16_to_f32(got[m]), oracle.bf16_to_f32(want)
        assert np.max(np.abs(g - w)) < 1e-2
        assert (bf16_ulp_diff(got[m], want) <= 1).mean() > 0.99
        # greedy on the GPU's own logits equals the oracle's greedy on them
        assert toks[m] == oracle.greedy(got[m])


def test_greedy_probability_rounding_ties(cuda):
    """Logits from a few adjacent bf16 values near the top: many entries share
    the largest bf16 probability after rounding (also entries whose logits
    differ), and the first of them must win, as in the reference."""
    rng = np.random.default_rng(5)
    V, M = 50257, 8
    top = oracle.bf16_bits(np.array([0.5], np.float32))[0]
    vals = (top - np.arange(4, dtype=np.uint16)).astype(np.uint16)
    lg = rng.choice(vals, (M, V)).astype(np.uint16)
    lg[:, ::7] = oracle.bf16_bits(np.full((1,), -4.0, np.float32))[0]
    toks = ops.sample_greedy(to_dev_bf16(lg)).cpu().numpy()
    assert list(toks) == [oracle.greedy(lg[m]) for m in range(M)]


def test_greedy_tie_break_first_index(cuda):
    V = 50257
    x = np.full((2, V), -3.0, np.float32)
    x[0, [17, 4000, 50000]] = 5.0
    x[1, [50256, 9]] = 1.0
    lg = oracle.bf16_bits(x)
    toks = ops.sample_greedy(to_dev_bf16(lg)).cpu().numpy()
    assert list(toks) == [17, 9] == [oracle.greedy(lg[0]), oracle.greedy(lg[1])]


def test_rejects_bad_arguments(cuda):
    x = torch.zeros((4, 8), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.W8A8Error):
        ops.layernorm_quant(x, x[0], x[0], want_y=False, want_q=False)
    q = torch.zeros((4, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.W8A8Error):  # max_ctx beyond the 1024-row cache
        ops.attention_decode(q, q, q, 0, None, 2048, 1)


# Row counts >= 1024 take the warp-per-row kernels (row in registers), fewer
# rows the block-per-row kernels: both must produce identical bits.
WARP_M = 1536


def _chunks(M, step=512):
    return [(i, min(M, i + step)) for i in range(0, M, step)]


@pytest.mark.parametrize("d", [768, 1024, 1280, 2000])
def test_layernorm_warp_rows_equal_block_rows(cuda, d):
    rng = np.random.default_rng(d)
    X = to_dev_bf16(_rand_bf16(rng, (WARP_M, d), 2.0))
    g = to_dev_bf16(oracle.bf16_bits(rng.uniform(0.5, 1.5, d).astype(np.float32)))
    b = to_dev_bf16(_rand_bf16(rng, (d,), 0.1))
    Y, Xq, sX = ops.layernorm_quant(X, g, b)
    for i, j in _chunks(WARP_M):
        y, q, s = ops.layernorm_quant(X[i:j], g, b)
        assert torch.equal(Y[i:j], y) and torch.equal(Xq[i:j], q) and torch.equal(sX[i:j], s)


@pytest.mark.parametrize("K", [768, 1280, 5120])
def test_quant_warp_rows_equal_block_rows(cuda, K):
    X = to_dev_bf16(oracle.bf16_bits(outlier_activations(WARP_M, K, seed=K)))
    Xq, sX = ops.per_token_quant(X)
    amax = ops.row_amax(X)
    Xq2, sX2 = ops.quant_rows_amax(X, amax)
    assert torch.equal(Xq, Xq2) and torch.equal(sX, sX2)
    for i, j in _chunks(WARP_M):
        q, s = ops.per_token_quant(X[i:j])
        assert torch.equal(Xq[i:j], q) and torch.equal(sX[i:j], s)
        assert torch.equal(amax[i:j], ops.row_amax(X[i:j]))


def test_embed_layernorm_warp_rows_equal_block_rows(cuda):
    rng = np.random.default_rng(9)
    V, C, d, B, T = 500, 1024, 1280, 3, 512
    wte = to_dev_bf16(_rand_bf16(rng, (V, d), 0.02))
    wpe = to_dev_bf16(_rand_bf16(rng, (C, d), 0.02))
    g = to_dev_bf16(oracle.bf16_bits(rng.uniform(0.5, 1.5, d).astype(np.float32)))
    b = to_dev_bf16(_rand_bf16(rng, (d,), 0.1))
    toks = to_dev(rng.integers(0, V, B * T).astype(np.int32))
    pos0 = to_dev(np.array([0, 100, 512], np.int32))
    H, Y, Xq, sX = ops.embed_layernorm_quant(wte, wpe, toks, T, pos0, g, b)
    for s in range(B):
        h, y, q, sx = ops.embed_layernorm_quant(wte, wpe, toks[s * T:(s + 1) * T], T,
                                                pos0[s:s + 1], g, b)
        r = slice(s * T, (s + 1) * T)
        assert torch.equal(H[r], h) and torch.equal(Y[r], y)
        assert torch.equal(Xq[r], q) and torch.equal(sX[r], sx)


def _mlp_operands(rng, M, d):
    f = 4 * d
    x = oracle.bf16_bits(outlier_activations(M, d, seed=M + d))
    xq, sx = oracle.quant_rows(x)
    W1 = rng.integers(-127, 128, (f, d), dtype=np.int8)
    W2 = rng.integers(-127, 128, (d, f), dtype=np.int8)
    sw1 = rng.uniform(1e-4, 1e-3, f).astype(np.float32)
    sw2 = rng.uniform(1e-4, 1e-3, d).astype(np.float32)
    b1 = _rand_bf16(rng, f, 0.02)
    b2 = _rand_bf16(rng, d, 0.02)
    R = _rand_bf16(rng, (M, d))
    dev = [to_dev(xq), to_dev(sx), to_dev(W1), to_dev(sw1), to_dev_bf16(b1), to_dev(W2),
           to_dev(sw2), to_dev_bf16(b2), to_dev_bf16(R)]
    return dev


@pytest.mark.parametrize("M", [1, 2, 8, 37, 64, 128, 200])
@pytest.mark.parametrize("d", [768, 1280])
def test_mlp_pair_fused_quantization(cuda, M, d):
    """W1 (+GELU) -> W2 with the quantization of W1's output fused
    (w8a8_linear_absmax -> w8a8_linear_from_bf16) against W1 -> quant_rows
    -> W2: bit-identical outputs; the record's row maxima are the rows'
    largest |y|; for one token (the fused GEMVs) no quantization or maxima
    kernel runs."""
    rng = np.random.default_rng(M * 5 + d)
    xq, sx, W1, sw1, b1, W2, sw2, b2, R = _mlp_operands(rng, M, d)
    ws = ops.linear_workspace(M, 4 * d, cuda)
    X1 = ops.linear(xq, sx, W1, sw1, b1, _lib.EPI_BIAS_GELU, workspace=ws)
    q2, s2 = ops.per_token_quant(X1)
    want = ops.linear(q2, s2, W2, sw2, b2, _lib.EPI_BIAS_RESID, R=R, workspace=ws)

    X1f, rec = ops.linear_absmax(xq, sx, W1, sw1, b1, _lib.EPI_BIAS_GELU, workspace=ws)
    Y = ops.linear_from_bf16(X1f, rec, W2, sw2, b2, _lib.EPI_BIAS_RESID, R=R, workspace=ws)
    assert torch.equal(X1f.view(torch.int16), X1.view(torch.int16))
    amax = X1.float().abs().amax(1)
    assert torch.equal(rec.amax(0), amax)
    assert torch.equal(Y.view(torch.int16), want.view(torch.int16))
    assert ops.device_error(reset=True) == 0
    if M == 1:  # the fused GEMV pair: two launches, no quantization or maxima kernel
        names = kernel_names_fresh("test_gpu_kernels", "mlp_pair_call", [[M, d]])[0]["names"]
        assert len(names) == 2, names
        assert not [n for n in names if "quant" in n or "amax" in n], names


def mlp_pair_call(M, d):
    """The fused W1 -> W2 pair on cuda:0 as the test above builds it, for
    kernel_names_fresh."""
    rng = np.random.default_rng(M * 5 + d)
    xq, sx, W1, sw1, b1, W2, sw2, b2, R = _mlp_operands(rng, M, d)
    ws = ops.linear_workspace(M, 4 * d, "cuda:0")

    def call():
        X1f, rec = ops.linear_absmax(xq, sx, W1, sw1, b1, _lib.EPI_BIAS_GELU, workspace=ws)
        ops.linear_from_bf16(X1f, rec, W2, sw2, b2, _lib.EPI_BIAS_RESID, R=R, workspace=ws)
        return 0
    return call


@pytest.mark.parametrize("M,K,n_part", [(1, 5120, 1), (1, 5120, 7), (3, 3072, 5), (64, 5120, 120),
                                        (128, 1024, 2), (300, 1024, 3)])
def test_linear_from_bf16_matches_quant_rows(cuda, M, K, n_part):
    """The in-kernel quantization against quant_rows on the same bf16 rows:
    zero rows (scale 1), outlier channels, the row maxima spread over n_part
    parts (each row's maximum in one part, the others below it)."""
    rng = np.random.default_rng(M + K + n_part)
    x = outlier_activations(M, K, seed=M * 3 + K)
    x[M // 2] = 0.0
    X = to_dev_bf16(oracle.bf16_bits(x))
    amax = X.float().abs().amax(1)
    rec = (amax[None, :] * torch.rand((n_part, M), device=cuda)).contiguous()
    rec[torch.from_numpy(rng.integers(0, n_part, M)).to(cuda), torch.arange(M, device=cuda)] = amax
    N = 768
    W = to_dev(rng.integers(-127, 128, (N, K), dtype=np.int8))
    sw = to_dev(rng.uniform(1e-4, 1e-3, N).astype(np.float32))
    b = to_dev_bf16(_rand_bf16(rng, N, 0.02))
    ws = ops.linear_workspace(M, N, cuda)
    xq, sx = ops.per_token_quant(X)
    want = ops.linear(xq, sx, W, sw, b, _lib.EPI_BIAS, workspace=ws)
    got = ops.linear_from_bf16(X, rec, W, sw, b, _lib.EPI_BIAS, workspace=ws)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert ops.device_error(reset=True) == 0


def _ln_operands(rng, M, d, N):
    X = _rand_bf16(rng, (M, d), 2.0)
    X[:, rng.choice(d, max(1, d // 100), replace=False)] = _rand_bf16(rng, (M, max(1, d // 100)), 40.0)
    g = _rand_bf16(rng, (d,), 1.0)
    b = _rand_bf16(rng, (d,), 0.1)
    W = rng.integers(-127, 128, (N, d), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    bias = _rand_bf16(rng, (N,), 0.02)
    return (to_dev_bf16(X), to_dev_bf16(g), to_dev_bf16(b), to_dev(W), to_dev(sw),
            to_dev_bf16(bias))


@pytest.mark.parametrize("M,d", [(1, 768), (1, 1024), (1, 1280), (1, 1600), (3, 1280)])
def test_layernorm_folded_into_qkv_gemv(cuda, M, d):
    """The QKV GEMV that forms the token's LayerNorm itself equals the
    LayerNorm kernel followed by the QKV GEMM, bit for bit: Q, the K/V cache
    rows and the quantized row it also writes (M = 3: the two kernels)."""
    rng = np.random.default_rng(d + M)
    X, g, b, W, sw, bias = _ln_operands(rng, M, d, 3 * d)
    C = 40
    pos = torch.tensor([17], dtype=torch.int32, device=cuda)
    T = M
    outs = []
    for fused in (False, True):
        Q = torch.zeros((M, d), dtype=torch.bfloat16, device=cuda)
        Kc = torch.zeros((1, C, d), dtype=torch.bfloat16, device=cuda)
        Vc = torch.zeros((1, C, d), dtype=torch.bfloat16, device=cuda)
        if fused:
            Xq, sX = ops.layernorm_linear_qkv(X, g, b, W, sw, bias, Q, Kc, Vc, C * d, T, pos)
        else:
            _, Xq, sX = ops.layernorm_quant(X, g, b, want_y=False)
            ops.linear_qkv(Xq, sX, W, sw, bias, Q, Kc, Vc, C * d, T, pos)
        outs.append([Q, Kc, Vc, Xq, sX])
    for a, f in zip(*outs):
        assert torch.equal(a.view(torch.uint8), f.view(torch.uint8))
    assert ops.device_error(reset=True) == 0
    if M == 1:
        names = kernel_names_fresh("test_gpu_kernels", "ln_qkv_call", [[d]])[0]["names"]
        assert len(names) == 1 and "gemv_ln" in names[0], names


def ln_qkv_call(d):
    """The fused LayerNorm + QKV GEMV of the test above on cuda:0."""
    rng = np.random.default_rng(d + 1)
    X, g, b, W, sw, bias = _ln_operands(rng, 1, d, 3 * d)
    Q = torch.zeros((1, d), dtype=torch.bfloat16, device="cuda:0")
    Kc = torch.zeros((1, 40, d), dtype=torch.bfloat16, device="cuda:0")
    Vc = torch.zeros((1, 40, d), dtype=torch.bfloat16, device="cuda:0")
    pos = torch.tensor([3], dtype=torch.int32, device="cuda:0")

    def call():
        ops.layernorm_linear_qkv(X, g, b, W, sw, bias, Q, Kc, Vc, 40 * d, 1, pos)
        return 0
    return call


@pytest.mark.parametrize("M,d", [(1, 768), (1, 1280), (1, 1600), (2, 1024)])
def test_layernorm_folded_into_w1_gemv(cuda, M, d):
    """W1 with the LayerNorm formed in the GEMV and the row absmax record
    equals the LayerNorm kernel followed by linear_absmax, bit for bit (the
    record's row maxima, the GELU output and the quantized row)."""
    rng = np.random.default_rng(3 * d + M)
    X, g, b, W, sw, bias = _ln_operands(rng, M, d, 4 * d)
    Y, rec, Xq, sX = ops.layernorm_linear_absmax(X, g, b, W, sw, bias, _lib.EPI_BIAS_GELU)
    _, Xq0, sX0 = ops.layernorm_quant(X, g, b, want_y=False)
    Y0, rec0 = ops.linear_absmax(Xq0, sX0, W, sw, bias, _lib.EPI_BIAS_GELU)
    assert torch.equal(Xq, Xq0) and torch.equal(sX.view(torch.int32), sX0.view(torch.int32))
    assert torch.equal(Y.view(torch.int16), Y0.view(torch.int16))
    assert torch.equal(rec.max(0).values, rec0.max(0).values)
    assert torch.equal(rec.max(0).values, Y.float().abs().max(1).values)
    assert ops.device_error(reset=True) == 0


def test_prefill_gelu_every_bf16_input(cuda):
    """The GELU of the prefill GEMM's fused epilogue against the reference-
    shaped element-wise GELU kernel (cuda/gelu.cu:10-15) for every one of the
    65536 bf16 inputs, bit for bit. The inputs enter as the biases of a GEMM
    whose accumulators are zero, so the epilogue's GELU input is each bias
    exactly."""
    M, K, N = 256, 16, 1 << 16  # more than 128 tokens: the token-major kernel
    xq = torch.zeros((M, K), dtype=torch.int8, device=cuda)
    sx = torch.ones(M, device=cuda)
    W = torch.ones((N, K), dtype=torch.int8, device=cuda)
    sw = torch.ones(N, device=cuda)
    bias = torch.arange(N, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).to(cuda)
    u = ops.linear(xq, sx, W, sw, bias, _lib.EPI_BIAS)  # the GELU input of each column
    keep = ~torch.isnan(bias) & (bias.view(torch.int16) != -0x8000)  # 0 + (-0) is +0
    assert torch.equal(u[0].view(torch.int16)[keep], bias.view(torch.int16)[keep])
    got = ops.linear(xq, sx, W, sw, bias, _lib.EPI_BIAS_GELU)
    want = u.clone()
    ops.ref_gelu(want)
    g, w = got.view(torch.int16), want.view(torch.int16)
    both_nan = torch.isnan(got) & torch.isnan(want)
    bad = (g != w) & ~both_nan
    assert not bool(bad.any()), [hex(int(b) & 0xffff) for b in bias.view(torch.int16)[bad[0]][:8]]
    # NaN out for the NaN inputs and for -inf (0.5 * -inf * (1 + -1))
    assert int(both_nan[0].sum()) == int(torch.isnan(bias).sum()) + 1
    assert ops.device_error(reset=True) == 0


@pytest.mark.parametrize("V", [2048, 3001, 70000])
def test_greedy_vocabulary_sizes(cuda, V):
    """The cluster pick over vocabularies whose four 256-aligned slices end
    short or empty-ish, with rows that start off a 16-byte boundary."""
    rng = np.random.default_rng(V)
    M = 5
    lg = oracle.bf16_bits(rng.standard_normal((M, V + 3)).astype(np.float32) * 2.0)
    d = to_dev_bf16(lg)[:, 3:]  # row stride V + 3: rows start at odd offsets
    toks = ops.sample_greedy(d).cpu().numpy()
    assert list(toks) == [oracle.greedy(lg[m, 3:]) for m in range(M)]
