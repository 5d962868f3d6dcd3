"""sam-rs_b200: B200 (sm_100a) implementation of sam-rs's decomposed-rel-pos attention path.

Host-side mirror of the reference's custom-op entry points (apiplant/sam-rs 0.1.1, src/kernels.rs),
over the C ABI of libsamrs_b200.so. Same names, argument meaning and error behaviour as the
reference; PyTorch CUDA tensors stand in for candle CUDA tensors (device memory and streams only).

    relpos_softmax(scores, q, table, h, w, scale)        src/kernels.rs:12-43
    attention_relpos(q, kt, v, table, h, w, scale)       src/kernels.rs:896-906 (the fused op, CUDA)
    qkv_split(y, bias, n, nh, hd) -> (q, kt, v)          src/kernels.rs:870-894
    bmm(a, b)                                            src/kernels.rs:917-924
    Attention / window_partition / window_unpartition    src/sam1/encoder.rs:45-85, 132-145
    linear(a, w, bias, res, epilogue)                    Linear + bias / bias_residual / bias_gelu
                                                         (src/cpu_gemm.rs:205-222, src/kernels.rs:1040-1061)
    qkv_linear_window(x, w, bias, ...)                   qkv Linear + window_partition + qkv_split, fused
    layer_norm(x, weight, bias, eps)                     the blocks' norm1 / norm2 (src/sam1/encoder.rs:100-102)
    Block                                                Block::forward (src/sam1/encoder.rs:89-129) on the
                                                         library's kernels

Every op runs a CUDA kernel of this package; a tensor that is not a contiguous CUDA tensor of
f32/f16/bf16 raises, as the reference's `bail!` does (src/kernels.rs:1092,1097-1102). There is no
CPU fallback: if libsamrs_b200.so is missing, the first op call raises.
"""
import ctypes
import math

import torch

from . import _abi
from ._abi import SamrsError

__all__ = ["relpos_softmax", "attention_relpos", "attention_relpos_cpu", "qkv_split", "qkv_split_window",
           "window_merge", "bmm", "Attention", "window_partition", "window_unpartition", "device_status",
           "recompute_count", "global_policy", "linear", "qkv_linear_window", "layer_norm", "Block", "SamrsError"]

_DTYPES = {torch.float32: _abi.F32, torch.float16: _abi.F16, torch.bfloat16: _abi.BF16}
_IMPLS = {"auto": _abi.IMPL_AUTO, "simt": _abi.IMPL_SIMT, "tc": _abi.IMPL_TC}


def _dtype_code(*ts):
    dt = ts[0].dtype
    if dt not in _DTYPES:
        raise SamrsError(_abi.ERR_INVALID, f"unsupported dtype {dt} for a sam-rs CUDA kernel")
    for t in ts:
        if t.dtype != dt:
            raise SamrsError(_abi.ERR_INVALID, f"mixed dtypes {dt} and {t.dtype}")
        if not t.is_cuda:
            raise SamrsError(_abi.ERR_INVALID, "sam-rs CUDA kernels need CUDA tensors")
        if not t.is_contiguous():
            raise SamrsError(_abi.ERR_INVALID, "sam-rs kernels need contiguous inputs")
    return _DTYPES[dt]


def _stream():
    return ctypes_stream(torch.cuda.current_stream())


def ctypes_stream(stream):
    return stream.cuda_stream


def attention_relpos(q, kt, v, table, h, w, scale, impl="auto", out=None):
    """Fused attention: softmax(scale*q.kt + relpos(q)) . v, shapes q/v [BH, h*w, hd], kt [BH, hd, h*w],
    table [(2h-1)+(2w-1), hd]. Returns [BH, h*w, hd] in the input dtype (src/kernels.rs:896-906)."""
    code = _dtype_code(q, kt, v, table)
    if q.dim() != 3 or kt.dim() != 3 or v.dim() != 3:
        raise SamrsError(_abi.ERR_INVALID, "attention_relpos: q, kt, v must be rank 3")
    bh, n, hd = q.shape
    if n != h * w or tuple(kt.shape) != (bh, hd, n) or tuple(v.shape) != (bh, n, hd):
        raise SamrsError(_abi.ERR_INVALID, f"attention_relpos: shapes q{tuple(q.shape)} kt{tuple(kt.shape)} "
                                           f"v{tuple(v.shape)} do not match h={h} w={w}")
    if tuple(table.shape) != ((2 * h - 1) + (2 * w - 1), hd):
        raise SamrsError(_abi.ERR_INVALID, f"attention_relpos: table {tuple(table.shape)} != "
                                           f"({(2 * h - 1) + (2 * w - 1)}, {hd})")
    if out is None:
        out = torch.empty_like(q)
    else:
        _dtype_code(out, q)
        if out.shape != q.shape:
            raise SamrsError(_abi.ERR_INVALID, "attention_relpos: out shape mismatch")
    _abi.check(_abi.lib().samrs_relpos_attn_fwd_ex(q.data_ptr(), kt.data_ptr(), v.data_ptr(), table.data_ptr(),
                                                   out.data_ptr(), bh, h, w, hd, float(scale), code, _IMPLS[impl],
                                                   _stream()))
    return out


def attention_relpos_cpu(q, kt, v, table, h, w, scale):
    """Signature twin of the reference's `attention_relpos_cpu` (src/kernels.rs:899): returns the fused
    attention for CUDA inputs, and None otherwise (the reference returns None off its own device)."""
    if not (q.is_cuda and q.dtype in _DTYPES):
        return None
    return attention_relpos(q.contiguous(), kt.contiguous(), v.contiguous(), table.contiguous(), h, w, scale)


def relpos_softmax(scores, q, table, h, w, scale):
    """Materialising biased softmax: scores [BH, h*w, h*w], q [BH, h*w, hd] -> probs [BH, h*w, h*w]
    (src/kernels.rs:12-43)."""
    code = _dtype_code(scores, q, table)
    n = h * w
    hd = q.shape[-1]
    rows = scores.numel() // n if n else 0
    if scores.shape[-1] != n or q.numel() != rows * hd:
        raise SamrsError(_abi.ERR_INVALID, f"relpos_softmax: scores {tuple(scores.shape)} / q {tuple(q.shape)} "
                                           f"do not match h={h} w={w}")
    if tuple(table.shape) != ((2 * h - 1) + (2 * w - 1), hd):
        raise SamrsError(_abi.ERR_INVALID, "relpos_softmax: bad table shape")
    out = torch.empty_like(scores)
    _abi.check(_abi.lib().samrs_relpos_softmax_fwd(scores.data_ptr(), q.data_ptr(), table.data_ptr(),
                                                   out.data_ptr(), rows, h, w, hd, float(scale), code, _stream()))
    return out


def qkv_split(y, bias, n, nh, hd):
    """y [T, 3*nh*hd] (bias-free qkv projection) + bias [3*nh*hd] -> (q [BH,n,hd], kt [BH,hd,n], v [BH,n,hd]),
    BH = (T/n)*nh (src/kernels.rs:870-894)."""
    code = _dtype_code(y, bias)
    t = y.shape[0]
    if y.dim() != 2 or y.shape[1] != 3 * nh * hd or bias.numel() != 3 * nh * hd:
        raise SamrsError(_abi.ERR_INVALID, "qkv_split: shape mismatch")
    packed = torch.empty(y.numel(), dtype=y.dtype, device=y.device)
    _abi.check(_abi.lib().samrs_qkv_split_fwd(y.data_ptr(), bias.data_ptr(), packed.data_ptr(), t, n, nh, hd, code,
                                              _stream()))
    bh = t // n * nh
    plane = t * nh * hd
    return (packed[:plane].view(bh, n, hd), packed[plane:2 * plane].view(bh, hd, n),
            packed[2 * plane:].view(bh, n, hd))


def _win_counts(h, w, ws):
    wh, ww = (ws, ws) if ws else (h, w)
    return wh * ww, ((h + wh - 1) // wh) * ((w + ww - 1) // ww)


def qkv_split_window(y, bias, images, h, w, ws, nh, hd):
    """window_partition (zero pad, src/sam1/encoder.rs:132-140) + qkv bias + qkv_split (src/kernels.rs:870-894)
    in one pass: y [images*h*w, 3*nh*hd] is the projection of the real tokens (no bias); returns
    (q [BH,n,hd], kt [BH,hd,n], v [BH,n,hd]), BH = images * windows * nh, n = ws*ws; pad tokens get the bias.
    ws = 0: one window of h x w (global layers)."""
    code = _dtype_code(y, bias)
    c = nh * hd
    if y.dim() != 2 or y.shape[0] != images * h * w or y.shape[1] != 3 * c or bias.numel() != 3 * c:
        raise SamrsError(_abi.ERR_INVALID, "qkv_split_window: shape mismatch")
    n, nwin = _win_counts(h, w, ws)
    bh = images * nwin * nh
    packed = torch.empty(3 * bh * n * hd, dtype=y.dtype, device=y.device)
    _abi.check(_abi.lib().samrs_qkv_split_window_fwd(y.data_ptr(), bias.data_ptr(), packed.data_ptr(), images, h, w,
                                                     ws, nh, hd, code, _stream()))
    plane = bh * n * hd
    return (packed[:plane].view(bh, n, hd), packed[plane:2 * plane].view(bh, hd, n),
            packed[2 * plane:].view(bh, n, hd))


def window_merge(attn, images, h, w, ws, nh, hd):
    """Heads back to tokens (src/sam1/encoder.rs:82) + window_unpartition crop (:142-145): attn [BH, n, hd] ->
    [images*h*w, nh*hd], the real tokens only."""
    code = _dtype_code(attn)
    n, nwin = _win_counts(h, w, ws)
    if attn.shape != (images * nwin * nh, n, hd) or not attn.is_contiguous():
        raise SamrsError(_abi.ERR_INVALID, "window_merge: shape mismatch")
    out = torch.empty(images * h * w, nh * hd, dtype=attn.dtype, device=attn.device)
    _abi.check(_abi.lib().samrs_window_merge_fwd(attn.data_ptr(), out.data_ptr(), images, h, w, ws, nh, hd, code,
                                                 _stream()))
    return out


_EPIS = {"bias": _abi.EPI_BIAS, "bias_residual": _abi.EPI_BIAS_RESIDUAL, "bias_gelu": _abi.EPI_BIAS_GELU}


def linear(a, w, bias, res=None, epilogue="bias", out=None):
    """Tensor-core Linear with a fused epilogue: a [M, K] . w[N, K]^T + bias [N], then
    "bias" (nothing more), "bias_residual" (+ res [M, N], src/kernels.rs:1040-1049) or "bias_gelu" (exact erf
    GELU, src/kernels.rs:1051-1061). w is the weight as stored ([out, in]). f16 / bf16."""
    if epilogue not in _EPIS:
        raise SamrsError(_abi.ERR_INVALID, f"linear: unknown epilogue {epilogue!r}")
    ts = (a, w, bias) if res is None else (a, w, bias, res)
    code = _dtype_code(*ts)
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1] or bias.numel() != w.shape[0]:
        raise SamrsError(_abi.ERR_INVALID, f"linear: shapes a{tuple(a.shape)} w{tuple(w.shape)} bias{tuple(bias.shape)}")
    m, k = a.shape
    n = w.shape[0]
    if epilogue == "bias_residual" and (res is None or tuple(res.shape) != (m, n)):
        raise SamrsError(_abi.ERR_INVALID, "linear: bias_residual needs res [M, N]")
    if out is None:
        out = torch.empty(m, n, dtype=a.dtype, device=a.device)
    _abi.check(_abi.lib().samrs_linear_fwd(a.data_ptr(), w.data_ptr(), bias.data_ptr(),
                                           res.data_ptr() if res is not None else None, out.data_ptr(), m, n, k,
                                           _EPIS[epilogue], code, _stream()))
    return out


def qkv_linear_window(x, w, bias, images, h, w_grid, ws, nh, hd):
    """qkv Linear + window partition (zero pad) + bias + head split in one tensor-core GEMM: x [images*h*w, C]
    (real tokens), w [3C, C], bias [3C] -> (q [BH,n,hd], kt [BH,hd,n], v [BH,n,hd]) as qkv_split_window returns
    them (pad tokens get the bias)."""
    code = _dtype_code(x, w, bias)
    c = nh * hd
    if x.dim() != 2 or tuple(x.shape) != (images * h * w_grid, c) or tuple(w.shape) != (3 * c, c) or \
            bias.numel() != 3 * c:
        raise SamrsError(_abi.ERR_INVALID, "qkv_linear_window: shape mismatch")
    n, nwin = _win_counts(h, w_grid, ws)
    bh = images * nwin * nh
    packed = torch.empty(3 * bh * n * hd, dtype=x.dtype, device=x.device)
    _abi.check(_abi.lib().samrs_qkv_linear_window_fwd(x.data_ptr(), w.data_ptr(), bias.data_ptr(), packed.data_ptr(),
                                                      images, h, w_grid, ws, nh, hd, code, _stream()))
    plane = bh * n * hd
    return (packed[:plane].view(bh, n, hd), packed[plane:2 * plane].view(bh, hd, n),
            packed[2 * plane:].view(bh, n, hd))


def layer_norm(x, weight, bias, eps=1e-6, out=None):
    """LayerNorm over the last dim (src/sam1/encoder.rs:100-102: candle_nn::LayerNorm, eps 1e-6)."""
    code = _dtype_code(x, weight, bias)
    c = x.shape[-1]
    if weight.numel() != c or bias.numel() != c:
        raise SamrsError(_abi.ERR_INVALID, "layer_norm: weight / bias size")
    if out is None:
        out = torch.empty_like(x)
    _abi.check(_abi.lib().samrs_layer_norm_fwd(x.data_ptr(), weight.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                               x.numel() // c, c, float(eps), code, _stream()))
    return out


def bmm(a, b):
    """Batched [B,m,k] x [B,k,n] (src/kernels.rs:917-924); a plain library GEMM, as in the reference."""
    return torch.bmm(a, b)


def device_status(clear=True):
    """Synchronise the current stream and return the device status word (0 = healthy)."""
    rc = _abi.lib().samrs_device_status(_stream(), 1 if clear else 0)
    if rc < 0:
        raise SamrsError(rc, _abi.lib().samrs_last_error().decode())
    return rc


def recompute_count(clear=True):
    """Synchronise the current stream and return how many bf16 global-layer CTAs (one head x 256 query rows)
    the exact second pass recomputed since the last clear."""
    n = ctypes.c_int64(0)
    _abi.check(_abi.lib().samrs_recompute_count(_stream(), ctypes.byref(n), 1 if clear else 0))
    return int(n.value)


def global_policy(table, reset=False):
    """The library's choice for the bf16 global layer whose rel-pos table is `table`: (last measured share of
    CTAs the exact second pass recomputed, -1 if none; True if its next call runs the exact kernel alone).
    reset=True first forgets every layer's history on the current device."""
    share, exact = ctypes.c_double(0.0), ctypes.c_int(0)
    _abi.check(_abi.lib().samrs_global_policy(ctypes.c_void_p(table.data_ptr()), ctypes.byref(share),
                                              ctypes.byref(exact), 1 if reset else 0))
    return float(share.value), bool(exact.value)


def window_partition(x, ws):
    """[B, H, W, C] -> ([B*nWh*nWw, ws, ws, C], Hp, Wp), zero-padding H, W up to multiples of ws
    (src/sam1/encoder.rs:132-140)."""
    b, h, w, c = x.shape
    ph, pw = (ws - h % ws) % ws, (ws - w % ws) % ws
    if ph or pw:
        x = torch.nn.functional.pad(x, (0, 0, 0, pw, 0, ph))
    hp, wp = h + ph, w + pw
    x = x.reshape(b, hp // ws, ws, wp // ws, ws, c).permute(0, 1, 3, 2, 4, 5).contiguous()
    return x.reshape(b * (hp // ws) * (wp // ws), ws, ws, c), hp, wp


def window_unpartition(x, ws, hp, wp, hw, b, c):
    """Inverse of window_partition, cropping back to hw (src/sam1/encoder.rs:142-145)."""
    x = x.reshape(b, hp // ws, wp // ws, ws, ws, c).permute(0, 1, 3, 2, 4, 5).contiguous().reshape(b, hp, wp, c)
    return x[:, : hw[0], : hw[1], :].contiguous()


class Attention:
    """SAM ViT attention block, `Attention::new` / `Attention::forward` of src/sam1/encoder.rs:45-85.

    Weights: qkv_w [3C, C], qkv_b [3C], proj_w [C, C], rel_pos_h / rel_pos_w [2*input-1, hd].
    The table is cat(rel_pos_h, rel_pos_w) and scale = hd^-0.5 (encoder.rs:56-69). forward() returns the
    output projection without its bias, as the reference does (the caller fuses the bias into the
    residual add, encoder.rs:71-72)."""

    def __init__(self, qkv_w, qkv_b, proj_w, proj_b, rel_pos_h, rel_pos_w, heads):
        dim = qkv_w.shape[1]
        self.heads = heads
        self.hd = dim // heads
        self.qkv_wt = qkv_w.t().contiguous()
        self.qkv_b = qkv_b.contiguous()
        self.proj_wt = proj_w.t().contiguous()
        self.proj_b = proj_b
        self.scale = float(self.hd) ** -0.5
        self.rel = torch.cat([rel_pos_h, rel_pos_w], 0).contiguous()

    def forward(self, x):
        nw, h, w, c = x.shape
        nh, n = self.heads, h * w
        hd = c // nh
        y = (x.reshape(nw * n, c) @ self.qkv_wt).contiguous()
        q, kt, v = qkv_split(y, self.qkv_b, n, nh, hd)
        ctx = attention_relpos(q, kt, v, self.rel, h, w, self.scale)
        out = ctx.reshape(nw, nh, n, hd).permute(0, 2, 1, 3).reshape(nw * n, c)
        return (out @ self.proj_wt).reshape(nw, h, w, c)


def vit_scale(hd):
    """scale = hd^-0.5 (src/sam1/encoder.rs:66)."""
    return 1.0 / math.sqrt(hd)


class Block:
    """SAM ViT encoder block, `Block::forward` of src/sam1/encoder.rs:89-129, on this library's kernels only:

        y   = norm1(x)                                   layer_norm
        q, kt, v = split(window_partition(y) Wqkv^T + b)  qkv_linear_window (pads get the bias)
        a   = attention_relpos(q, kt, v, rel)            the fused tcgen05 attention
        x   = x + merge(a) Wproj^T + bproj               window_merge, linear(bias_residual)
        x   = x + gelu(norm2(x) W1^T + b1) W2^T + b2     layer_norm, linear(bias_gelu), linear(bias_residual)

    The projections run on the real tokens only (a pad token's projection is the bias, and the crop drops
    the pads' outputs), so the result is the reference's. Weights as stored ([out, in]); x [B, H, W, C]."""

    def __init__(self, p, heads, window, eps=1e-6):
        self.p, self.heads, self.window, self.eps = p, heads, window, eps
        self.rel = torch.cat([p["rel_pos_h"], p["rel_pos_w"]], 0).contiguous()

    def forward(self, x):
        b, h, w, c = x.shape
        nh, p = self.heads, self.p
        hd = c // nh
        t = b * h * w
        xt = x.reshape(t, c)
        y = layer_norm(xt, p["norm1_w"], p["norm1_b"], self.eps)
        ws = self.window
        q, kt, v = qkv_linear_window(y, p["qkv_w"], p["qkv_b"], b, h, w, ws, nh, hd)
        wh, ww = (ws, ws) if ws else (h, w)
        a = attention_relpos(q, kt, v, self.rel, wh, ww, float(hd) ** -0.5)
        merged = window_merge(a, b, h, w, ws, nh, hd)
        x1 = linear(merged, p["proj_w"], p["proj_b"], res=xt, epilogue="bias_residual")
        y2 = layer_norm(x1, p["norm2_w"], p["norm2_b"], self.eps)
        m = linear(y2, p["lin1_w"], p["lin1_b"], epilogue="bias_gelu")
        return linear(m, p["lin2_w"], p["lin2_b"], res=x1, epilogue="bias_residual").reshape(b, h, w, c)
