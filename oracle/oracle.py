"""ctypes front end of the CPU oracle (oracle/relpos_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg. The product package never imports this module. Every function takes and returns float32 numpy
arrays in the reference's layouts (q [bh,n,hd], kt [bh,hd,n], v [bh,n,hd], table [(2h-1)+(2w-1),hd]).
"""
import ctypes
import os

import numpy as np

from . import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.OUT
        if not os.path.exists(path):
            build_oracle.build()
        l = ctypes.CDLL(path)
        f = ctypes.POINTER(ctypes.c_float)
        L, I, F = ctypes.c_long, ctypes.c_int, ctypes.c_float
        for name in ("oracle_attention_relpos_f32", "oracle_attention_relpos_bf16"):
            fn = getattr(l, name)
            fn.argtypes = [f, f, f, f, f, L, I, I, I, F, I]
            fn.restype = I
        l.oracle_relpos_softmax_f32.argtypes = [f, f, f, f, L, I, I, I, F, I]
        l.oracle_relpos_softmax_f32.restype = I
        l.oracle_qkv_split_f32.argtypes = [f, f, f, L, I, I, I]
        l.oracle_qkv_split_f32.restype = I
        l.oracle_cpu_has_bf16.restype = I
        l.oracle_max_threads.restype = I
        _lib = l
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def cpu_has_bf16() -> bool:
    return bool(lib().oracle_cpu_has_bf16())


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def attention_relpos(q, kt, v, table, h, w, scale, threads=0, mode="exact"):
    """Fused attention on the CPU. mode: "exact" (src/kernels.rs:131-225, f32) or "bf16"
    (src/cpu_gemm.rs path, AVX-512 BF16 hosts only)."""
    q, kt, v, table = _f32(q), _f32(kt), _f32(v), _f32(table)
    bh, n, hd = q.shape
    assert n == h * w and kt.shape == (bh, hd, n) and v.shape == (bh, n, hd)
    assert table.shape == ((2 * h - 1) + (2 * w - 1), hd)
    out = np.empty((bh, n, hd), np.float32)
    fn = lib().oracle_attention_relpos_f32 if mode == "exact" else lib().oracle_attention_relpos_bf16
    rc = fn(_p(q), _p(kt), _p(v), _p(table), _p(out), bh, h, w, hd, float(scale), int(threads))
    if rc != 0:
        raise RuntimeError(f"oracle attention ({mode}) failed: rc={rc}")
    return out


def relpos_softmax(s, q, table, h, w, scale, threads=0):
    """Probabilities [rows, n] (src/kernels.rs:62-105). s: [..., n], q: [..., hd] with the same rows."""
    n = h * w
    s2, q2, table = _f32(s).reshape(-1, n), _f32(q), _f32(table)
    hd = q2.shape[-1]
    q2 = q2.reshape(-1, hd)
    rows = s2.shape[0]
    assert q2.shape[0] == rows
    out = np.empty_like(s2)
    rc = lib().oracle_relpos_softmax_f32(_p(s2), _p(q2), _p(table), _p(out), rows, h, w, hd, float(scale),
                                         int(threads))
    if rc != 0:
        raise RuntimeError(f"oracle relpos_softmax failed: rc={rc}")
    return out.reshape(np.shape(s))


def qkv_split(y, bias, n, nh, hd):
    """(q [bh,n,hd], kt [bh,hd,n], v [bh,n,hd]) from y [tokens, 3*nh*hd] + bias (src/kernels.rs:234-263)."""
    y, bias = _f32(y), _f32(bias)
    tokens = y.shape[0]
    out = np.empty(3 * tokens * nh * hd, np.float32)
    rc = lib().oracle_qkv_split_f32(_p(y), _p(bias), _p(out), tokens, n, nh, hd)
    if rc != 0:
        raise RuntimeError("oracle qkv_split failed")
    bh = tokens // n * nh
    plane = tokens * nh * hd
    return (out[:plane].reshape(bh, n, hd), out[plane:2 * plane].reshape(bh, hd, n),
            out[2 * plane:].reshape(bh, n, hd))


def window_partition(x, ws):
    """[B, H, W, C] -> [B * nWh * nWw, ws, ws, C], zero-padding H and W up to multiples of ws
    (src/sam1/encoder.rs:132-140: pad, reshape [B, Hp/ws, ws, Wp/ws, ws, C], swap the two middle axes)."""
    x = np.asarray(x)
    b, h, w, c = x.shape
    hp, wp = -(-h // ws) * ws, -(-w // ws) * ws
    xp = np.zeros((b, hp, wp, c), x.dtype)
    xp[:, :h, :w] = x
    xp = xp.reshape(b, hp // ws, ws, wp // ws, ws, c).transpose(0, 1, 3, 2, 4, 5)
    return xp.reshape(-1, ws, ws, c)


def window_unpartition(xw, ws, h, w):
    """Inverse of window_partition, cropping the pads (src/sam1/encoder.rs:142-145): [B*nW, ws, ws, C] ->
    [B, H, W, C]."""
    xw = np.asarray(xw)
    c = xw.shape[-1]
    hp, wp = -(-h // ws) * ws, -(-w // ws) * ws
    b = xw.shape[0] // ((hp // ws) * (wp // ws))
    x = xw.reshape(b, hp // ws, wp // ws, ws, ws, c).transpose(0, 1, 3, 2, 4, 5).reshape(b, hp, wp, c)
    return x[:, :h, :w]


def qkv_split_window(y, bias, images, h, w, ws, nh, hd):
    """The reference's order for the windowed input side: the qkv projection y of the real tokens
    [images*h*w, 3C] (no bias) is laid on the token grid, window_partition pads with zero projections
    (a zero input token projects to 0), then qkv_split adds the bias and splits heads
    (src/sam1/encoder.rs:132-140, src/kernels.rs:234-263). ws = 0: one window of h x w."""
    y = _f32(y)
    c3 = y.shape[1]
    grid = y.reshape(images, h, w, c3)
    if ws:
        win = window_partition(grid, ws)
        n = ws * ws
    else:
        win, n = grid, h * w
    return qkv_split(np.ascontiguousarray(win.reshape(-1, c3)), bias, n, nh, hd)


def window_merge(attn, images, h, w, ws, nh, hd):
    """attn [bh, n, hd] -> heads back to [windows, n, C] (src/sam1/encoder.rs:82) -> window_unpartition crop
    (:142-145) -> [images*h*w, C]. ws = 0: one window of h x w."""
    attn = _f32(attn)
    bh, n, _ = attn.shape
    tok = attn.reshape(bh // nh, nh, n, hd).transpose(0, 2, 1, 3).reshape(bh // nh, n, nh * hd)
    if ws:
        grid = window_unpartition(tok.reshape(-1, ws, ws, nh * hd), ws, h, w)
    else:
        grid = tok.reshape(images, h, w, nh * hd)
    return np.ascontiguousarray(grid.reshape(images * h * w, nh * hd))


# ------------------------------------------------------------------------------------------------
# The rest of the encoder block (src/sam1/encoder.rs:89-129), restated in numpy (f64 arithmetic on the
# given values; the callers pass 16-bit-rounded inputs where the kernels see 16-bit inputs).
# ------------------------------------------------------------------------------------------------

def linear(a, w, bias=None):
    """a [M, K] . w[N, K]^T (+ bias): the reference's Linear holds w transposed and multiplies
    (src/cpu_gemm.rs:205-222, src/sam1/encoder.rs:61-63, 103-107)."""
    y = np.asarray(a, np.float64) @ np.asarray(w, np.float64).T
    return y if bias is None else y + np.asarray(bias, np.float64)


def bias_residual(res, y, bias):
    """res + y + bias[col] (src/kernels.rs:619-641)."""
    return np.asarray(res, np.float64) + np.asarray(y, np.float64) + np.asarray(bias, np.float64)


def bias_gelu(y, bias):
    """gelu_erf(y + bias[col]) = 0.5 x (1 + erf(x / sqrt 2)) (src/kernels.rs:643-665)."""
    from scipy.special import erf
    x = np.asarray(y, np.float64) + np.asarray(bias, np.float64)
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def layer_norm(x, weight, bias, eps=1e-6):
    """LayerNorm over the last dim with the biased variance (candle_nn::LayerNorm, as the blocks' norm1 /
    norm2 use it, src/sam1/encoder.rs:100-102)."""
    x = np.asarray(x, np.float64)
    mean = x.mean(-1, keepdims=True)
    var = ((x - mean) ** 2).mean(-1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * np.asarray(weight, np.float64) + np.asarray(bias, np.float64)


def attention_block(x, p, heads):
    """Attention::forward (src/sam1/encoder.rs:73-85): x [nW, H, W, C] -> the output projection without its
    bias [nW, H, W, C]; the attention itself is the exact-f32 oracle above."""
    nw, h, w, c = x.shape
    hd, n = c // heads, h * w
    y = linear(x.reshape(nw * n, c), p["qkv_w"])
    q, kt, v = qkv_split(y, p["qkv_b"], n, heads, hd)
    rel = np.concatenate([p["rel_pos_h"], p["rel_pos_w"]], 0)
    ctx = attention_relpos(q, kt, v, rel, h, w, hd ** -0.5)
    out = ctx.reshape(nw, heads, n, hd).transpose(0, 2, 1, 3).reshape(nw * n, c)
    return linear(out, p["proj_w"]).reshape(nw, h, w, c)


def block_forward(x, p, heads, window, eps=1e-6):
    """Block::forward (src/sam1/encoder.rs:115-129) in the reference's order: norm1, window_partition with
    zero pad (windowed blocks), attention, window_unpartition crop, bias_residual, norm2, lin1 + bias_gelu,
    lin2 + bias_residual. x [B, H, W, C] -> [B, H, W, C] (f64)."""
    b, h, w, c = x.shape
    y = layer_norm(x, p["norm1_w"], p["norm1_b"], eps)
    if window:
        parts = window_partition(y, window)
        y = window_unpartition(attention_block(parts, p, heads), window, h, w)
    else:
        y = attention_block(y, p, heads)
    x = bias_residual(x, y, p["proj_b"])
    t = b * h * w
    m = bias_gelu(linear(layer_norm(x, p["norm2_w"], p["norm2_b"], eps).reshape(t, c), p["lin1_w"]), p["lin1_b"])
    return bias_residual(x, linear(m, p["lin2_w"]).reshape(b, h, w, c), p["lin2_b"])
