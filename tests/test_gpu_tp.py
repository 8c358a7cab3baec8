"""Tensor-parallel prefill on the GPU: its building-block kernels against the
single-GPU kernels they split, and the whole prefill against the single-GPU
engine, bit for bit (one rank on one GPU; two NCCL ranks when two GPUs are
present)."""
import os
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from c_gpt2_b200 import _lib, ops
from c_gpt2_b200.engine import Engine
from c_gpt2_b200.quant8 import GPT2Dims, read_quant8
from c_gpt2_b200.synthetic import outlier_activations, prompts, quant8_image_gpu
from c_gpt2_b200.tp import Collectives, TPPlan, TPPrefill, shard_weights
from oracle import oracle
from tests.gpu_util import from_dev_bf16, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu
# GPT-2 large layer shapes, two layers
LARGE2 = GPT2Dims(d_model=1280, n_layer=2, n_head=20)


def _bf16_rows(M, K, seed):
    return to_dev_bf16(oracle.bf16_bits(outlier_activations(M, K, seed=seed)))


def test_quant_with_split_row_maxima_equals_quant_rows(cuda):
    M, K = 300, 5120
    X = _bf16_rows(M, K, 1)
    want_q, want_s = ops.per_token_quant(X)
    parts = [(0, 1280), (1280, 3200), (3200, 5120)]
    amax = torch.stack([ops.row_amax(X[:, a:b]) for a, b in parts])
    np.testing.assert_array_equal(amax.amax(0).cpu().numpy(),
                                  X.float().abs().amax(1).cpu().numpy())
    for a, b in parts:
        q, s = ops.quant_rows_amax(X[:, a:b], amax)
        assert torch.equal(q, want_q[:, a:b])
        assert torch.equal(s, want_s)


@pytest.mark.parametrize("slots", [1, 2, 4])
def test_reduce_residual_layernorm_quant_equals_linear_then_layernorm(cuda, slots):
    M, K, d = 256, 2560, 1280
    rng = np.random.default_rng(slots)
    xq, sx = oracle.quant_rows(oracle.bf16_bits(outlier_activations(M, K, seed=3)))
    W = rng.integers(-127, 128, (d, K), dtype=np.int8)
    sw = rng.uniform(1e-3, 1e-2, d).astype(np.float32)
    b = to_dev_bf16(oracle.bf16_bits(rng.standard_normal(d).astype(np.float32) * 0.02))
    R = to_dev_bf16(oracle.bf16_bits(rng.standard_normal((M, d)).astype(np.float32)))
    g = to_dev_bf16(oracle.bf16_bits(1 + 0.1 * rng.standard_normal(d).astype(np.float32)))
    be = to_dev_bf16(oracle.bf16_bits(0.1 * rng.standard_normal(d).astype(np.float32)))
    Xq, sX, Wd, sW = to_dev(xq), to_dev(sx), to_dev(W), to_dev(sw)
    want_h = ops.linear(Xq, sX, Wd, sW, b, _lib.EPI_BIAS_RESID, R=R)
    _, want_q, want_s = ops.layernorm_quant(want_h, g, be, want_y=False)
    # partial sums over K slices, as the row-split GEMM on `slots` GPUs makes them
    cuts = np.linspace(0, K // 64, slots + 1).astype(int) * 64
    acc = torch.stack([ops.gemm_s32(Xq[:, a:c].contiguous(), Wd[:, a:c].contiguous())
                       for a, c in zip(cuts, cuts[1:])])
    H = R.clone()
    q = torch.empty((M, d), dtype=torch.int8, device=cuda)
    s = torch.empty((M,), dtype=torch.float32, device=cuda)
    ops.reduce_residual_layernorm_quant(acc, sX, sW, b, H, H, g, be, 1e-5, q, s)
    np.testing.assert_array_equal(from_dev_bf16(H), from_dev_bf16(want_h))
    assert torch.equal(q, want_q) and torch.equal(s, want_s)


@pytest.fixture(scope="module")
def large2_image():
    return quant8_image_gpu(LARGE2, seed=5)


def _engine_prefill(img, dims, P):
    n_seq, T = P.shape
    eng = Engine(dims, max_batch=n_seq, max_tokens=n_seq * T)
    eng.load_quant8(img)
    p_d = torch.from_numpy(P).cuda()
    out = torch.empty((n_seq,), dtype=torch.int32, device="cuda")
    eng.prefill(p_d, out, 1)
    torch.cuda.synchronize()
    logits = eng.logits(n_seq)
    eng.close()
    return out.cpu().numpy(), logits


def test_tp_one_rank_matches_engine(cuda, large2_image):
    P = prompts(4, 128, seed=9)
    want_next, want_logits = _engine_prefill(large2_image, LARGE2, P)
    plan = TPPlan.make(LARGE2, 1)
    shard = shard_weights(read_quant8(large2_image, LARGE2), plan, 0, cuda)
    nxt, logits = TPPrefill(plan, shard, 0).run(torch.from_numpy(P).cuda())
    np.testing.assert_array_equal(nxt.cpu().numpy(), want_next)
    got = (from_dev_bf16(logits).astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(got, want_logits)


def _tp_rank(rank, world, port, img_path, p_path, out_dir, exchange="collective"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        ops.init(rank)
        img = np.load(img_path)
        P = np.load(p_path)
        plan = TPPlan.make(LARGE2, world)
        shard = shard_weights(read_quant8(img, LARGE2), plan, rank, f"cuda:{rank}")
        tp = TPPrefill(plan, shard, rank, collectives=Collectives(), exchange=exchange)
        for _ in range(2):  # twice: the exchange buffers and flags are reused
            nxt, logits = tp.run(torch.from_numpy(P).cuda())
        torch.cuda.synchronize()
        tp.close()
        np.save(os.path.join(out_dir, f"next{rank}.npy"), nxt.cpu().numpy())
        np.save(os.path.join(out_dir, f"logits{rank}.npy"), from_dev_bf16(logits))
        assert ops.device_error() == 0
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["alltoall", "collective", "peer"])
def test_tp_two_ranks_match_engine(cuda, large2_image, tmp_path, exchange):
    """Two ranks, exchange through NCCL (int8 inputs to the rows' owners, or
    int32 partial sums) or through the library's peer-memory kernels over
    NVLink: the same logits and tokens as one GPU, bit for bit."""
    P = prompts(4, 128, seed=9)
    want_next, want_logits = _engine_prefill(large2_image, LARGE2, P)
    np.save(tmp_path / "img.npy", large2_image)
    np.save(tmp_path / "p.npy", P)
    port = 29600 + os.getpid() % 300 + {"collective": 0, "peer": 300, "alltoall": 600}[exchange]
    mp.start_processes(_tp_rank, args=(2, port, str(tmp_path / "img.npy"),
                                       str(tmp_path / "p.npy"), str(tmp_path), exchange),
                       nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"next{r}.npy"), want_next)
    bits = np.concatenate([np.load(tmp_path / f"logits{r}.npy") for r in range(2)])
    np.testing.assert_array_equal((bits.astype(np.uint32) << 16).view(np.float32), want_logits)


def test_reduce_warp_rows_equal_block_rows(cuda):
    """Row counts >= 1024 take the warp-per-row kernel, fewer rows the
    block-per-row kernel: identical bits."""
    M, d, slots = 1536, 1280, 2
    g = torch.Generator(device="cuda").manual_seed(1)
    acc = torch.randint(-2 ** 24, 2 ** 24, (slots, M, d), dtype=torch.int32, device=cuda,
                        generator=g)
    sX = torch.rand((M,), device=cuda, generator=g) * 1e-2 + 1e-4
    sW = torch.rand((d,), device=cuda, generator=g) * 1e-2 + 1e-4
    b = (torch.randn((d,), device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    R = torch.randn((M, d), device=cuda, generator=g).to(torch.bfloat16)
    gam = (1 + 0.1 * torch.randn((d,), device=cuda, generator=g)).to(torch.bfloat16)
    bet = (0.1 * torch.randn((d,), device=cuda, generator=g)).to(torch.bfloat16)
    H = torch.empty_like(R)
    q = torch.empty((M, d), dtype=torch.int8, device=cuda)
    s = torch.empty((M,), dtype=torch.float32, device=cuda)
    ops.reduce_residual_layernorm_quant(acc, sX, sW, b, R, H, gam, bet, 1e-5, q, s)
    for i in range(0, M, 512):
        j = i + 512
        h = torch.empty_like(R[i:j])
        q2 = torch.empty_like(q[i:j])
        s2 = torch.empty_like(s[i:j])
        ops.reduce_residual_layernorm_quant(acc[:, i:j], sX[i:j], sW, b, R[i:j], h, gam, bet,
                                            1e-5, q2, s2)
        assert torch.equal(H[i:j], h) and torch.equal(q[i:j], q2) and torch.equal(s[i:j], s2)
