"""w8a8_linear_noalloc: the linear layer for callers that cannot allocate
device memory. Its split-K scratch lives in a fixed array inside the library;
its results must equal those of w8a8_linear given a caller-allocated
workspace, call after call (the shared scratch must be cleared each time).
This file is collected last so a stopping run has run every other test."""
import numpy as np
import pytest
import torch

from c_gpt2_b200 import _lib, ops
from c_gpt2_b200.synthetic import outlier_activations
from oracle import oracle
from tests.gpu_util import from_dev_bf16, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu


def _noalloc(args, M, K, N, epi, R, Y):
    xq, sx, W, sw, b = args
    ldr = R.stride(0) if R is not None else 0
    return _lib.core().w8a8_linear_noalloc(
        xq.data_ptr(), sx.data_ptr(), M, K, W.data_ptr(), sw.data_ptr(), b.data_ptr(), N, epi,
        R.data_ptr() if R is not None else None, ldr, Y.data_ptr(), Y.stride(0),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,K,epi", [(64, 1280, 5120, _lib.EPI_BIAS_RESID),
                                       (64, 5120, 1280, _lib.EPI_BIAS_GELU),
                                       (20, 2304, 768, _lib.EPI_BIAS)])
def test_noalloc_linear_matches_linear(cuda, M, N, K, epi):
    rng = np.random.default_rng(M + N + K)
    x = oracle.bf16_bits(outlier_activations(M, K, seed=7))
    xq, sx = oracle.quant_rows(x)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = oracle.bf16_bits(rng.standard_normal(N).astype(np.float32) * 0.02)
    R = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((M, N)).astype(np.float32)))
    R = R if epi == _lib.EPI_BIAS_RESID else None
    args = (to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw), to_dev_bf16(b))
    ws = ops.linear_workspace(M, N, cuda)
    want = from_dev_bf16(ops.linear(*args, epi, R=R, workspace=ws))
    for _ in range(2):  # the shared scratch keeps the last call's contents
        Y = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda)
        assert _noalloc(args, M, K, N, epi, R, Y) == _lib.W8A8_OK
        np.testing.assert_array_equal(from_dev_bf16(Y), want)


def test_noalloc_rejects_shapes_beyond_the_scratch(cuda):
    M, N, K = 1024, 2048, 64  # 8 MiB of partial sums > 4 MiB of scratch
    xq = torch.zeros((M, K), dtype=torch.int8, device=cuda)
    sx = torch.ones(M, device=cuda)
    W = torch.zeros((N, K), dtype=torch.int8, device=cuda)
    sw = torch.ones(N, device=cuda)
    b = torch.zeros(N, dtype=torch.bfloat16, device=cuda)
    Y = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    st = _noalloc((xq, sx, W, sw, b), M, K, N, _lib.EPI_BIAS, None, Y)
    assert st == _lib.W8A8_ERR_UNSUPPORTED
