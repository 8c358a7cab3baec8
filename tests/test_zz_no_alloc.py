"""w8a8_linear_noalloc: the linear layer for callers that cannot allocate
device memory (a host that sizes all of it once at start-up, as gpt2.c does,
or a plugin whose host owns the allocator). Where w8a8_linear would split a
few-token GEMM over K into a caller's workspace, this entry point uses a fixed
scratch array inside the library; its results must equal w8a8_linear's and
the oracle's, call after call, since every call shares that array.

The shapes below reach the split-K kernel: a few tokens whose output rows are
not 16-byte aligned, or whose N is not a multiple of 4, which the cluster
kernel does not take. The kernels each call launches are read back from the
CUDA activity record (torch.profiler, in a fresh process), which shows that
these shapes really run the channel-major tcgen05 GEMM that reads the
scratch.

This file is collected last so a run that stops at the first failure has
already run every other test."""
import re

import numpy as np
import pytest
import torch

from c_gpt2_b200 import _lib, ops
from c_gpt2_b200.synthetic import outlier_activations
from oracle import oracle
from tests.gpu_util import bf16_ulp_diff, from_dev_bf16, kernel_names_fresh, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu


def _noalloc(args, M, K, N, epi, R, Y):
    xq, sx, W, sw, b = args
    ldr = R.stride(0) if R is not None else 0
    return _lib.core().w8a8_linear_noalloc(
        xq.data_ptr(), sx.data_ptr(), M, K, W.data_ptr(), sw.data_ptr(), b.data_ptr(), N, epi,
        R.data_ptr() if R is not None else None, ldr, Y.data_ptr(), Y.stride(0),
        torch.cuda.current_stream().cuda_stream)


SCRATCH_BYTES = 4 << 20  # W8A8_NOALLOC_SCRATCH_BYTES of include/gpt2_w8a8.h
# channel-major tcgen05 GEMM (template arguments KIND = 0, EPI, CM = true)
SPLIT_K_KERNEL = re.compile(r"gemm_tc_kernel<0, \d+, true")


def _operands(M, N, K, epi, seed):
    rng = np.random.default_rng(seed)
    x = oracle.bf16_bits(outlier_activations(M, K, seed=7))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = oracle.bf16_bits(rng.standard_normal(N).astype(np.float32) * 0.02)
    r = oracle.bf16_bits(rng.standard_normal((M, N)).astype(np.float32))
    r = r if epi == _lib.EPI_BIAS_RESID else None
    return xq, sx, W, sw, b, r


def _out(M, N, pad, device):
    """[M, N] bf16 view with row pitch N + pad, filled with 7.0."""
    return torch.full((M, N + pad), 7.0, dtype=torch.bfloat16, device=device)[:, :N]


def noalloc_call(M, N, K, epi, pad):
    """One w8a8_linear_noalloc call of this shape on cuda:0 (operands as the
    tests build them), for kernel_names_fresh."""
    dev = torch.device("cuda", 0)
    xq, sx, W, sw, b, r = _operands(M, N, K, epi, M + N + K)
    args = (to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b))
    R = None
    if r is not None:
        R = torch.zeros((M, N + pad), dtype=torch.bfloat16, device=dev)[:, :N]
        R.copy_(to_dev_bf16(r))
    Y = _out(M, N, pad, dev)
    return lambda: _noalloc(args, M, K, N, epi, R, Y)


# (M, N, K, epilogue, extra elements per output row)
SPLIT_K_SHAPES = [
    (64, 1280, 5120, _lib.EPI_BIAS_RESID, 4),   # W2 of GPT-2 large, unaligned output rows
    (64, 5120, 1280, _lib.EPI_BIAS_GELU, 4),    # W1 of GPT-2 large
    (20, 2304, 768, _lib.EPI_BIAS, 4),          # W_qkv of GPT-2 small
    (16, 1282, 768, _lib.EPI_BIAS, 0),          # N % 4 != 0
]


@pytest.mark.parametrize("M,N,K,epi,pad", SPLIT_K_SHAPES)
def test_noalloc_split_k_matches_linear_and_oracle(cuda, M, N, K, epi, pad):
    xq, sx, W, sw, b, r = _operands(M, N, K, epi, M + N + K)
    args = (to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b))
    R = None
    if r is not None:
        R = torch.zeros((M, N + pad), dtype=torch.bfloat16, device=cuda)[:, :N]
        R.copy_(to_dev_bf16(r))
    # w8a8_linear with its own zeroed workspace
    ws = ops.linear_workspace(M, N, cuda)
    want = from_dev_bf16(ops.linear(*args, epi, R=R, out=_out(M, N, pad, cuda), workspace=ws))
    assert int(ws.count_nonzero()) == 0  # the split-K kernel leaves it zero
    # the oracle: bit-exact, GELU within one bf16 ulp (CUDA tanhf vs the C library's)
    ref = oracle.linear(xq, sx, W, sw, b, epi, R=r)
    if epi == _lib.EPI_BIAS_GELU:
        assert bf16_ulp_diff(want, ref).max() <= 1
    else:
        np.testing.assert_array_equal(want, ref)
    # two calls in a row: the shared scratch keeps the last call's contents
    for call in range(2):
        Y = _out(M, N, pad, cuda)
        assert _noalloc(args, M, K, N, epi, R, Y) == _lib.W8A8_OK
        np.testing.assert_array_equal(from_dev_bf16(Y), want)
    assert ops.device_error(reset=True) == 0
    # the call runs the split-K kernel, which reads the scratch
    rec = kernel_names_fresh("test_zz_no_alloc", "noalloc_call", [[M, N, K, epi, pad]])[0]
    assert rec["status"] == _lib.W8A8_OK
    assert any(SPLIT_K_KERNEL.search(n) for n in rec["names"]), rec["names"]


def test_noalloc_shapes_without_split_k(cuda):
    """One token (GEMV), aligned decode rows (cluster kernel) and prefill rows
    (token-major kernel) read no workspace: they run as w8a8_linear, whatever
    their size, including shapes whose partial sums would not fit the scratch."""
    shapes = [(1, 2304, 768), (64, 5120, 1280), (1024, 2048, 64), (256, 5120, 1280)]
    for M, N, K in shapes:
        xq, sx, W, sw, b, _ = _operands(M, N, K, _lib.EPI_BIAS, M + N + K)
        args = (to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b))
        want = from_dev_bf16(ops.linear(*args, _lib.EPI_BIAS))
        np.testing.assert_array_equal(want, oracle.linear(xq, sx, W, sw, b, _lib.EPI_BIAS))
        Y = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda)
        assert _noalloc(args, M, K, N, _lib.EPI_BIAS, None, Y) == _lib.W8A8_OK
        np.testing.assert_array_equal(from_dev_bf16(Y), want)
    recs = kernel_names_fresh("test_zz_no_alloc", "noalloc_call",
                              [[M, N, K, _lib.EPI_BIAS, 0] for M, N, K in shapes])
    for (M, N, K), rec in zip(shapes, recs):
        names = rec["names"]
        assert rec["status"] == _lib.W8A8_OK
        assert names and not any(SPLIT_K_KERNEL.search(n) for n in names), (M, N, K, names)
        assert not any("emset" in n for n in names), names  # no clearing either


def test_noalloc_rejects_split_k_beyond_the_scratch(cuda):
    """128 tokens x 9216 channels on the split-K path: 4.5 MiB of partial sums
    plus counters exceed the 4 MiB array. The call is refused and writes
    nothing."""
    M, N, K, pad = 128, 9216, 1280, 4
    assert M * N * 4 > SCRATCH_BYTES
    xq = torch.ones((M, K), dtype=torch.int8, device=cuda)
    sx = torch.ones(M, device=cuda)
    W = torch.ones((N, K), dtype=torch.int8, device=cuda)
    sw = torch.ones(N, device=cuda)
    b = torch.zeros(N, dtype=torch.bfloat16, device=cuda)
    Y = _out(M, N, pad, cuda)
    st = _noalloc((xq, sx, W, sw, b), M, K, N, _lib.EPI_BIAS, None, Y)
    assert st == _lib.W8A8_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert bool((Y == 7.0).all())
