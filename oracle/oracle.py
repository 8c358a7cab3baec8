"""ctypes binding of the CPU oracle (oracle/lib/liboracle_w8a8.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and bench.py's
CPU-baseline leg as the checker; never by the product path. Arrays are numpy;
bf16 values travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "lib" / "liboracle_w8a8.so"
EPI_DEQUANT, EPI_BIAS, EPI_BIAS_RESID, EPI_BIAS_GELU = 0, 1, 2, 3

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
        l = C.CDLL(str(LIB_PATH))
        p, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
        l.orc_quant_rows.argtypes = [p, i, i, p, p]
        l.orc_gemm_s32.argtypes = [p, i, i, p, i, p]
        l.orc_gelu.argtypes = [f]
        l.orc_gelu.restype = f
        l.orc_linear.argtypes = [p, p, i, i, p, p, p, i, i, p, p]
        l.orc_layernorm.argtypes = [p, i, i, p, p, f, p]
        l.orc_softmax_row.argtypes = [p, i, f, p]
        l.orc_attention.argtypes = [p, p, p, i, i, i, p]
        l.orc_lm_head.argtypes = [p, i, p, i, p]
        l.orc_greedy.argtypes = [p, i]
        l.orc_greedy.restype = i
        l.orc_top_k.argtypes = [p, i, i, p, p]
        l.orc_sample_topk.argtypes = [p, i, i, f]
        l.orc_sample_topk.restype = i
        l.orc_generate.argtypes = [p, sz, i, i, i, i, i, p, i, i, p, p]
        l.orc_generate.restype = i
        l.orc_generate_steps.argtypes = [p, sz, i, i, i, i, i, p, i, i, p, p, p]
        l.orc_generate_steps.restype = i
        l.orc_set_sum_order.argtypes = [i]
        l.orc_set_sum_order.restype = None
        _lib = l
    return _lib


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quant_rows(x_bf16: np.ndarray):
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    xq = np.empty((M, K), np.int8)
    sx = np.empty((M,), np.float32)
    lib().orc_quant_rows(x.ctypes.data, M, K, xq.ctypes.data, sx.ctypes.data)
    return xq, sx


def gemm_s32(xq: np.ndarray, W: np.ndarray) -> np.ndarray:
    xq, W = _c(xq, np.int8), _c(W, np.int8)
    M, K = xq.shape
    N = W.shape[0]
    Y = np.empty((M, N), np.int32)
    lib().orc_gemm_s32(xq.ctypes.data, M, K, W.ctypes.data, N, Y.ctypes.data)
    return Y


def linear(xq, sx, W, sw, bias, epi, R=None) -> np.ndarray:
    xq, W = _c(xq, np.int8), _c(W, np.int8)
    sx, sw = _c(sx, np.float32), _c(sw, np.float32)
    M, K = xq.shape
    N = W.shape[0]
    b = _c(bias, np.uint16) if bias is not None else None
    r = _c(R, np.uint16) if R is not None else None
    Y = np.empty((M, N), np.uint16)
    lib().orc_linear(xq.ctypes.data, sx.ctypes.data, M, K, W.ctypes.data, sw.ctypes.data,
                     b.ctypes.data if b is not None else None, N, epi,
                     r.ctypes.data if r is not None else None, Y.ctypes.data)
    return Y


def layernorm(x, gamma, beta, eps=1e-5) -> np.ndarray:
    x, g, b = _c(x, np.uint16), _c(gamma, np.uint16), _c(beta, np.uint16)
    M, d = x.shape
    y = np.empty((M, d), np.uint16)
    lib().orc_layernorm(x.ctypes.data, M, d, g.ctypes.data, b.ctypes.data, eps, y.ctypes.data)
    return y


def softmax_row(x, temperature=1.0) -> np.ndarray:
    x = _c(x, np.uint16)
    out = np.empty_like(x)
    lib().orc_softmax_row(x.ctypes.data, x.size, temperature, out.ctypes.data)
    return out


def attention(Q, K, V, q0, n_head) -> np.ndarray:
    """Rows [q0, q0+len(Q)) of one sequence; K/V hold cache rows [0, q0+len(Q))."""
    Q, K, V = _c(Q, np.uint16), _c(K, np.uint16), _c(V, np.uint16)
    nq = Q.shape[0]
    O = np.empty_like(Q)
    lib().orc_attention(Q.ctypes.data, K.ctypes.data, V.ctypes.data, q0, nq, n_head,
                        O.ctypes.data)
    return O


def lm_head(xf, wte) -> np.ndarray:
    xf, wte = _c(xf, np.uint16), _c(wte, np.uint16)
    V, d = wte.shape
    out = np.empty((V,), np.uint16)
    lib().orc_lm_head(xf.ctypes.data, d, wte.ctypes.data, V, out.ctypes.data)
    return out


def greedy(logits) -> int:
    x = _c(logits, np.uint16)
    return int(lib().orc_greedy(x.ctypes.data, x.size))


def top_k(probs, k):
    """gpt2.c:130-180: (indices [k], renormalised bf16 probabilities [k]) of one
    row of bf16 probabilities; equal probabilities in ascending index order."""
    p = _c(probs, np.uint16)
    kk = min(max(int(k), 1), p.size)
    idx = np.empty((kk,), np.int32)
    q = np.empty((kk,), np.uint16)
    lib().orc_top_k(p.ctypes.data, p.size, int(k), idx.ctypes.data, q.ctypes.data)
    return idx, q


def sample_topk(probs, k, r) -> int:
    """gpt2.c:2223-2245: the token drawn with r in [0, 1] from one row of bf16 probabilities."""
    p = _c(probs, np.uint16)
    return int(lib().orc_sample_topk(p.ctypes.data, p.size, int(k), float(r)))


def generate(image: bytes, dims, prompt, n_gen: int):
    """Greedy stream of one sequence; returns (tokens [n_gen], last logits bf16 bits)."""
    buf = np.frombuffer(image, dtype=np.uint8)
    p = _c(prompt, np.int32)
    out = np.empty((n_gen,), np.int32)
    logits = np.empty((dims.vocab,), np.uint16)
    st = lib().orc_generate(buf.ctypes.data, buf.nbytes, dims.d_model, dims.n_layer, dims.n_head,
                            dims.vocab, dims.ctx, p.ctypes.data, p.size, n_gen, out.ctypes.data,
                            logits.ctypes.data)
    if st != 0:
        raise RuntimeError(f"orc_generate failed ({st})")
    return out, logits


def generate_steps(image, dims, prompt, n_gen: int, sum_order: int = 0):
    """Greedy stream of one sequence with the bf16 logits every token was
    picked from: (tokens [n_gen], logits bits [n_gen, vocab]).

    sum_order 1 adds the fp32 sums the reference leaves to cuBLAS (attention
    dot products and P.V, LM head) in descending instead of ascending index
    order: an equally valid reading of the reference, for measuring how far
    two valid orders drift apart."""
    buf = np.frombuffer(image, dtype=np.uint8)
    p = _c(prompt, np.int32)
    out = np.empty((n_gen,), np.int32)
    logits = np.empty((n_gen, dims.vocab), np.uint16)
    lib().orc_set_sum_order(sum_order)
    try:
        st = lib().orc_generate_steps(buf.ctypes.data, buf.nbytes, dims.d_model, dims.n_layer,
                                      dims.n_head, dims.vocab, dims.ctx, p.ctypes.data, p.size,
                                      n_gen, out.ctypes.data, None, logits.ctypes.data)
    finally:
        lib().orc_set_sum_order(0)
    if st != 0:
        raise RuntimeError(f"orc_generate_steps failed ({st})")
    return out, logits
