"""Torch-tensor front end of the C ABI (include/gpt2_w8a8.h).

Each function takes CUDA tensors, checks dtypes/shapes on the host, and calls
the native entry point on the current torch stream. Names follow the
reference's kernel ABI (include/cuda_kernels.h of roeybenhayun/c_gpt2) where a
function has a counterpart there.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, core


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.data_ptr()


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor")


def init(device: int = 0) -> None:
    check(core().w8a8_init(device), "w8a8_init")


def device_error(reset: bool = True) -> int:
    return core().w8a8_device_error(1 if reset else 0)


def per_token_quant(X: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """activation_quant.cu:37-110 — X [M,K] bf16 -> (Xq int8 [M,K], sX f32 [M])."""
    _need(X, torch.bfloat16, "X")
    M, K = X.shape
    Xq = torch.empty((M, K), dtype=torch.int8, device=X.device)
    sX = torch.empty((M,), dtype=torch.float32, device=X.device)
    check(core().w8a8_quant_rows(_ptr(X), X.stride(0), M, K, _ptr(Xq), _ptr(sX), _stream()),
          "w8a8_quant_rows")
    return Xq, sX


def layernorm_quant(X: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                    want_y: bool = True, want_q: bool = True):
    """layernorm.cu:7-100 (+ per-token quant). Returns (Y, Xq, sX), None where not asked."""
    _need(X, torch.bfloat16, "X")
    M, d = X.shape
    Y = torch.empty((M, d), dtype=torch.bfloat16, device=X.device) if want_y else None
    Xq = torch.empty((M, d), dtype=torch.int8, device=X.device) if want_q else None
    sX = torch.empty((M,), dtype=torch.float32, device=X.device) if want_q else None
    check(core().w8a8_layernorm_quant(_ptr(X), X.stride(0), M, d, _ptr(gamma), _ptr(beta), eps,
                                      _ptr(Y), d, _ptr(Xq), _ptr(sX), _stream()),
          "w8a8_layernorm_quant")
    return Y, Xq, sX


def embed_layernorm_quant(wte, wpe, tokens, T, pos0, gamma, beta, eps=1e-5):
    """embeddings.cu + layernorm.cu + quant for M = B*T new tokens.
    Returns (H, Y, Xq, sX)."""
    _need(tokens, torch.int32, "tokens")
    M = tokens.numel()
    d = wte.shape[1]
    dev = wte.device
    H = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
    Y = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
    Xq = torch.empty((M, d), dtype=torch.int8, device=dev)
    sX = torch.empty((M,), dtype=torch.float32, device=dev)
    check(core().w8a8_embed_layernorm_quant(_ptr(wte), _ptr(wpe), _ptr(tokens), M, T, _ptr(pos0),
                                            d, _ptr(H), _ptr(gamma), _ptr(beta), eps, _ptr(Y),
                                            _ptr(Xq), _ptr(sX), _stream()),
          "w8a8_embed_layernorm_quant")
    return H, Y, Xq, sX


def gemm_s32(Xq: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """The reference's cublasGemmEx INT8 call: Xq [M,K] · W[N,K]^T -> int32 [M,N]."""
    _need(Xq, torch.int8, "Xq")
    _need(W, torch.int8, "W")
    M, K = Xq.shape
    N = W.shape[0]
    Y = torch.empty((M, N), dtype=torch.int32, device=Xq.device)
    check(core().w8a8_gemm_s32(_ptr(Xq), M, K, _ptr(W), N, _ptr(Y), _stream()), "w8a8_gemm_s32")
    return Y


def linear_workspace(M: int, N: int, device) -> torch.Tensor:
    """Zero-filled split-K workspace for w8a8_linear (reusable across calls)."""
    return torch.zeros((core().w8a8_linear_workspace_size(M, N),), dtype=torch.uint8,
                       device=device)


def linear(Xq, sX, W, sW, bias, epilogue=_lib.EPI_BIAS, R=None, out=None, workspace=None):
    """Fused W8A8 linear: dequant (+bias) (+residual | +GELU) -> bf16 [M,N]."""
    _need(Xq, torch.int8, "Xq")
    M, K = Xq.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=Xq.device)
    ldr = R.stride(0) if R is not None else 0
    ws_bytes = workspace.numel() if workspace is not None else 0
    check(core().w8a8_linear(_ptr(Xq), _ptr(sX), M, K, _ptr(W), _ptr(sW), _ptr(bias), N, epilogue,
                             _ptr(R), ldr, _ptr(Y), Y.stride(0), _ptr(workspace), ws_bytes,
                             _stream()), "w8a8_linear")
    return Y


def linear_absmax(Xq, sX, W, sW, bias, epilogue=_lib.EPI_BIAS_GELU, R=None, out=None,
                  workspace=None):
    """linear() that also returns the row absmax record of its output:
    (Y, record [n_part, M] float32) with record.max(0) = max_n |Y[m, n]|."""
    _need(Xq, torch.int8, "Xq")
    M, K = Xq.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=Xq.device)
    ldr = R.stride(0) if R is not None else 0
    ws_bytes = workspace.numel() if workspace is not None else 0
    cap = core().w8a8_absmax_record_floats(M, N)
    rec = torch.empty(cap, dtype=torch.float32, device=Xq.device)
    n_part = ctypes.c_int(0)
    check(core().w8a8_linear_absmax(_ptr(Xq), _ptr(sX), M, K, _ptr(W), _ptr(sW), _ptr(bias), N,
                                    epilogue, _ptr(R), ldr, _ptr(Y), Y.stride(0), _ptr(rec), cap,
                                    ctypes.byref(n_part), _ptr(workspace), ws_bytes, _stream()),
          "w8a8_linear_absmax")
    return Y, rec[: n_part.value * M].view(n_part.value, M)


def linear_from_bf16(X, record, W, sW, bias, epilogue=_lib.EPI_BIAS_RESID, R=None, out=None,
                     workspace=None, Xq=None, sX=None):
    """linear() on the per-token quantization of the bf16 rows X, whose row
    maxima are the parts of `record` ([n_part, M], from linear_absmax)."""
    _need(X, torch.bfloat16, "X")
    M, K = X.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=X.device)
    Xq = Xq if Xq is not None else torch.empty((M, K), dtype=torch.int8, device=X.device)
    sX = sX if sX is not None else torch.empty(M, dtype=torch.float32, device=X.device)
    ldr = R.stride(0) if R is not None else 0
    ws_bytes = workspace.numel() if workspace is not None else 0
    check(core().w8a8_linear_from_bf16(_ptr(X), X.stride(0), _ptr(record), record.shape[0], M, K,
                                       _ptr(W), _ptr(sW), _ptr(bias), N, epilogue, _ptr(R), ldr,
                                       _ptr(Y), Y.stride(0), _ptr(Xq), _ptr(sX),
                                       _ptr(workspace), ws_bytes, _stream()),
          "w8a8_linear_from_bf16")
    return Y


def linear_qkv(Xq, sX, Wqkv, sWqkv, bqkv, Q, Kc, Vc, seq_stride, T, pos0=None, workspace=None):
    M, d = Xq.shape
    ws_bytes = workspace.numel() if workspace is not None else 0
    check(core().w8a8_linear_qkv(_ptr(Xq), _ptr(sX), M, d, _ptr(Wqkv), _ptr(sWqkv), _ptr(bqkv),
                                 _ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc), seq_stride, T,
                                 _ptr(pos0), _ptr(workspace), ws_bytes, _stream()),
          "w8a8_linear_qkv")


def layernorm_linear_qkv(X, gamma, beta, Wqkv, sWqkv, bqkv, Q, Kc, Vc, seq_stride, T, pos0=None,
                         eps=1e-5, workspace=None):
    """layernorm_quant(X) then linear_qkv on its rows, as one kernel for a
    single token; returns the quantized rows (Xq, sX) it also writes."""
    _need(X, torch.bfloat16, "X")
    M, d = X.shape
    Xq = torch.empty((M, d), dtype=torch.int8, device=X.device)
    sX = torch.empty(M, dtype=torch.float32, device=X.device)
    ws_bytes = workspace.numel() if workspace is not None else 0
    check(core().w8a8_layernorm_linear_qkv(_ptr(X), X.stride(0), _ptr(gamma), _ptr(beta), eps,
                                           _ptr(Xq), _ptr(sX), M, d, _ptr(Wqkv), _ptr(sWqkv),
                                           _ptr(bqkv), _ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc),
                                           seq_stride, T, _ptr(pos0), _ptr(workspace), ws_bytes,
                                           _stream()), "w8a8_layernorm_linear_qkv")
    return Xq, sX


def layernorm_linear_absmax(X, gamma, beta, W, sW, bias, epilogue=_lib.EPI_BIAS_GELU, R=None,
                            eps=1e-5, out=None, workspace=None):
    """layernorm_quant(X) then linear_absmax on its rows, as one kernel for a
    single token: (Y, record [n_part, M], Xq, sX)."""
    _need(X, torch.bfloat16, "X")
    M, K = X.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=X.device)
    Xq = torch.empty((M, K), dtype=torch.int8, device=X.device)
    sX = torch.empty(M, dtype=torch.float32, device=X.device)
    ldr = R.stride(0) if R is not None else 0
    ws_bytes = workspace.numel() if workspace is not None else 0
    cap = core().w8a8_absmax_record_floats(M, N)
    rec = torch.empty(cap, dtype=torch.float32, device=X.device)
    n_part = ctypes.c_int(0)
    check(core().w8a8_layernorm_linear_absmax(_ptr(X), X.stride(0), _ptr(gamma), _ptr(beta), eps,
                                              _ptr(Xq), _ptr(sX), M, K, _ptr(W), _ptr(sW),
                                              _ptr(bias), N, epilogue, _ptr(R), ldr, _ptr(Y),
                                              Y.stride(0), _ptr(rec), cap, ctypes.byref(n_part),
                                              _ptr(workspace), ws_bytes, _stream()),
          "w8a8_layernorm_linear_absmax")
    return Y, rec[: n_part.value * M].view(n_part.value, M), Xq, sX


def linear_qkv_heads(Xq, sX, Wqkv, sWqkv, bqkv, Q, Kc, Vc, seq_stride, T, pos0=None,
                     workspace=None):
    """QKV projection of a subset of heads: Wqkv [3*d_heads, K]."""
    M, K = Xq.shape
    dh = Wqkv.shape[0] // 3
    ws_bytes = workspace.numel() if workspace is not None else 0
    check(core().w8a8_linear_qkv_heads(_ptr(Xq), _ptr(sX), M, K, dh, _ptr(Wqkv), _ptr(sWqkv),
                                       _ptr(bqkv), _ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc),
                                       seq_stride, T, _ptr(pos0), _ptr(workspace), ws_bytes,
                                       _stream()), "w8a8_linear_qkv_heads")


def row_amax(X, out=None):
    """Per-row max |x| of a bf16 [M, K] block -> f32 [M]."""
    _need(X, torch.bfloat16, "X")
    M, K = X.shape
    out = out if out is not None else torch.empty((M,), dtype=torch.float32, device=X.device)
    check(core().w8a8_row_amax(_ptr(X), X.stride(0), M, K, _ptr(out), _stream()), "w8a8_row_amax")
    return out


def quant_rows_amax(X, amax, Xq=None, sX=None):
    """Per-token quantization of X [M, K] with the row maxima amax ([M] or
    [n, M], the maximum over the n partial maxima)."""
    _need(X, torch.bfloat16, "X")
    M, K = X.shape
    amax2 = amax.reshape(-1, M)
    Xq = Xq if Xq is not None else torch.empty((M, K), dtype=torch.int8, device=X.device)
    sX = sX if sX is not None else torch.empty((M,), dtype=torch.float32, device=X.device)
    check(core().w8a8_quant_rows_amax(_ptr(X), X.stride(0), M, K, _ptr(amax2), amax2.shape[0],
                                      amax2.stride(0), _ptr(Xq), Xq.stride(0), _ptr(sX), _stream()),
          "w8a8_quant_rows_amax")
    return Xq, sX


def reduce_residual_layernorm_quant(acc, sX, sW, bias, R, H, gamma=None, beta=None, eps=1e-5,
                                    Xq=None, sXq=None):
    """H = R + dequant(sum of int32 partials acc [n, M, d] or [M, d]) + bias,
    then optionally LayerNorm + quant of H into Xq / sXq."""
    _need(acc, torch.int32, "acc")
    acc3 = acc if acc.dim() == 3 else acc.unsqueeze(0)
    n, M, d = acc3.shape
    check(core().w8a8_reduce_residual_layernorm_quant(
        _ptr(acc3), acc3.stride(1), n, acc3.stride(0), M, d, _ptr(sX), _ptr(sW), _ptr(bias),
        _ptr(R), R.stride(0), _ptr(H), H.stride(0), _ptr(gamma), _ptr(beta), eps, _ptr(Xq),
        Xq.stride(0) if Xq is not None else 0, _ptr(sXq), _stream()),
        "w8a8_reduce_residual_layernorm_quant")
    return H


def row_amax_to(X, out_ptrs):
    """Row maxima of X [M, K] into several [M] f32 arrays given by address."""
    from .peer import ptr_array
    M, K = X.shape
    check(core().w8a8_row_amax_to(_ptr(X), X.stride(0), M, K, ptr_array(out_ptrs), len(out_ptrs),
                                  _stream()), "w8a8_row_amax_to")


def gemm_s32_scatter(Xq, W, dst_ptrs, rows_per_dst):
    """Xq [M, K] . W[N, K]^T as int32, row m stored at dst[m // rows_per_dst]."""
    from .peer import ptr_array
    _need(Xq, torch.int8, "Xq")
    M, K = Xq.shape
    N = W.shape[0]
    check(core().w8a8_gemm_s32_scatter(_ptr(Xq), M, K, _ptr(W), N, ptr_array(dst_ptrs),
                                       len(dst_ptrs), rows_per_dst, _stream()),
          "w8a8_gemm_s32_scatter")


def reduce_residual_layernorm_quant_bcast(acc, sX, sW, bias, R, H, gamma, beta, eps, Xq, sXq,
                                          xq_bcast, sx_bcast, bcast_row0):
    """reduce_residual_layernorm_quant whose quantized rows are also stored
    into other GPUs' buffers (addresses) at row bcast_row0 + m."""
    from .peer import ptr_array
    acc3 = acc if acc.dim() == 3 else acc.unsqueeze(0)
    n, M, d = acc3.shape
    check(core().w8a8_reduce_residual_layernorm_quant_bcast(
        _ptr(acc3), acc3.stride(1), n, acc3.stride(0), M, d, _ptr(sX), _ptr(sW), _ptr(bias),
        _ptr(R), R.stride(0), _ptr(H), H.stride(0), _ptr(gamma), _ptr(beta), eps, _ptr(Xq),
        Xq.stride(0), _ptr(sXq), ptr_array(xq_bcast), ptr_array(sx_bcast), len(xq_bcast),
        bcast_row0, _stream()), "w8a8_reduce_residual_layernorm_quant_bcast")


def attention_prefill(Q, Kc, Vc, seq_stride, n_seq, T, n_head, out=None):
    d = n_head * 64
    O = out if out is not None else torch.empty((n_seq * T, d), dtype=torch.bfloat16,
                                                device=Q.device)
    check(core().w8a8_attention_prefill(_ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc), seq_stride,
                                        n_seq, T, n_head, 64, _ptr(O), O.stride(0), _stream()),
          "w8a8_attention_prefill")
    return O


def attention_decode(Q, Kc, Vc, seq_stride, n_ctx, max_ctx, n_head, out=None, workspace=None):
    n_seq = Q.shape[0]
    d = n_head * 64
    O = out if out is not None else torch.empty((n_seq, d), dtype=torch.bfloat16, device=Q.device)
    need = core().w8a8_attention_decode_workspace_size(n_seq, n_head, max_ctx)
    if workspace is None:  # zero-filled: the ticket counters must start at zero
        workspace = torch.zeros((need,), dtype=torch.uint8, device=Q.device)
    check(core().w8a8_attention_decode(_ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc), seq_stride,
                                       n_seq, _ptr(n_ctx), max_ctx, n_head, 64, _ptr(O),
                                       O.stride(0), _ptr(workspace), workspace.numel(),
                                       _stream()), "w8a8_attention_decode")
    return O


def attention_decode_quant(Q, Kc, Vc, seq_stride, n_ctx, max_ctx, n_head, workspace, out=None):
    """attention_decode + per-token quantization of each sequence's output
    row in the same launch. `workspace` must start zero-filled (it is left so).
    Returns (O, Xq, sX)."""
    n_seq = Q.shape[0]
    d = n_head * 64
    O = out if out is not None else torch.empty((n_seq, d), dtype=torch.bfloat16, device=Q.device)
    Xq = torch.empty((n_seq, d), dtype=torch.int8, device=Q.device)
    sX = torch.empty((n_seq,), dtype=torch.float32, device=Q.device)
    check(core().w8a8_attention_decode_quant(_ptr(Q), Q.stride(0), _ptr(Kc), _ptr(Vc), seq_stride,
                                             n_seq, _ptr(n_ctx), max_ctx, n_head, 64, _ptr(O),
                                             O.stride(0), _ptr(Xq), _ptr(sX), _ptr(workspace),
                                             workspace.numel(), _stream()),
          "w8a8_attention_decode_quant")
    return O, Xq, sX


def lm_head(Xf, wte):
    M, d = Xf.shape
    V = wte.shape[0]
    logits = torch.empty((M, V), dtype=torch.bfloat16, device=Xf.device)
    check(core().w8a8_lm_head(_ptr(Xf), Xf.stride(0), M, d, _ptr(wte), V, _ptr(logits), V,
                              _stream()), "w8a8_lm_head")
    return logits


def sample_greedy(logits):
    M, V = logits.shape
    out = torch.empty((M,), dtype=torch.int32, device=logits.device)
    check(core().w8a8_sample_greedy(_ptr(logits), logits.stride(0), M, V, _ptr(out), None, 0, None,
                                    _stream()), "w8a8_sample_greedy")
    return out


def sample_topk(logits, temperature, top_k, rnd, probs_out=None):
    """Top-k sampling at a temperature, one draw per row (``rnd`` float32 [M]
    on the device, each in [0, 1]); ``probs_out`` optionally receives the bf16
    probabilities. A temperature <= 0 gives the greedy token."""
    M, V = logits.shape
    out = torch.empty((M,), dtype=torch.int32, device=logits.device)
    check(core().w8a8_sample_topk(_ptr(logits), logits.stride(0), M, V, float(temperature),
                                  int(top_k), _ptr(rnd), 1, None, _ptr(out), None, 0, None,
                                  _ptr(probs_out) if probs_out is not None else None,
                                  probs_out.stride(0) if probs_out is not None else 0,
                                  _stream()), "w8a8_sample_topk")
    return out


# ---- reference-shaped element-wise operations (in place where the reference is) ----

def ref_softmax(a, rows, cols, stride, out, temperature=1.0, causal=0):
    check(core().w8a8_ref_softmax(_ptr(a), rows, cols, stride, _ptr(out), temperature, causal,
                                  _stream()), "w8a8_ref_softmax")


def ref_gelu(x):
    rows, cols = x.shape
    check(core().w8a8_ref_gelu(_ptr(x), cols, rows, _stream()), "w8a8_ref_gelu")


def ref_dequant(Y, sW, sX):
    M, N = Y.shape
    out = torch.empty((M, N), dtype=torch.bfloat16, device=Y.device)
    check(core().w8a8_ref_dequant(_ptr(Y), _ptr(sW), _ptr(sX), _ptr(out), M, N, _stream()),
          "w8a8_ref_dequant")
    return out


def ref_add_bias(a, b):
    rows, cols = a.shape
    check(core().w8a8_ref_add_bias(_ptr(a), rows, cols, _ptr(b), _stream()), "w8a8_ref_add_bias")


def ref_add_2d(a, b, out=None):
    rows, cols = a.shape
    out = a if out is None else out
    check(core().w8a8_ref_add_2d(_ptr(a), rows, cols, _ptr(b), _ptr(out), _stream()),
          "w8a8_ref_add_2d")
    return out
