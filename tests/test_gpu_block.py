"""The encoder block around the attention on the GPU (through the C ABI), against the oracle's restatement of
the reference (src/sam1/encoder.rs:89-129): the tensor-core Linear with its three fused epilogues, the qkv
projection fused with the window partition and head split, LayerNorm, one windowed and one global block, and
BASELINE config 2's ViT-B stack (12 blocks, f16)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle
from tests.helpers import HALF_TOL, parity_err, rel_max_err, mean_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def r(t):
    return t.float().cpu().numpy()


def rnd(shape, dt, dev, g, std=1.0):
    return (torch.randn(*shape, generator=g, device=dev) * std).to(DT[dt])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("epi", ["bias", "bias_residual", "bias_gelu"])
@pytest.mark.parametrize("m,n,k", [(300, 768, 768), (1000, 2304, 768), (257, 3072, 768), (129, 768, 3072),
                                   (64, 80, 40)])
def test_linear_epilogues(samrs, cuda, m, n, k, epi, dt):
    """out = epilogue(a . w^T + bias) against f64 on the same 16-bit inputs; M and N tails, K tails (40)."""
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    a, w = rnd((m, k), dt, cuda, g), rnd((n, k), dt, cuda, g, 0.05)
    bias, res = rnd((n,), dt, cuda, g, 0.1), rnd((m, n), dt, cuda, g)
    out = samrs.linear(a, w, bias, res=res if epi == "bias_residual" else None, epilogue=epi)
    assert samrs.device_status() == 0
    y = oracle.linear(r(a), r(w))
    want = {"bias": lambda: y + r(bias), "bias_residual": lambda: oracle.bias_residual(r(res), y, r(bias)),
            "bias_gelu": lambda: oracle.bias_gelu(y, r(bias))}[epi]()
    err = parity_err(r(out), want, dt)
    assert err < 1e-3, err


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("images,h,w,ws,nh,hd", [(2, 64, 64, 14, 12, 64), (1, 64, 64, 0, 16, 80),
                                                 (2, 13, 20, 7, 3, 32), (1, 14, 14, 14, 2, 16), (3, 14, 10, 4, 2, 32)])
def test_qkv_linear_window_bit_exact(samrs, cuda, images, h, w, ws, nh, hd, dt):
    """The fused qkv GEMM writes, element for element, what qkv_split_window makes of the same kernel's
    Linear output (round(a . w^T + b) in the I/O dtype): real tokens bit-exact, pad tokens = the bias."""
    g = torch.Generator(device=cuda).manual_seed(h * w + nh)
    c = nh * hd
    x, wt, bias = rnd((images * h * w, c), dt, cuda, g), rnd((3 * c, c), dt, cuda, g, 0.05), rnd((3 * c,), dt, cuda, g)
    got = samrs.qkv_linear_window(x, wt, bias, images, h, w, ws, nh, hd)
    y = samrs.linear(x, wt, bias)  # the same accumulation, + bias, rounded once
    assert samrs.device_status() == 0
    real = oracle.qkv_split_window(r(y), np.zeros(3 * c, np.float32), images, h, w, ws, nh, hd)
    pads = oracle.qkv_split_window(np.zeros((images * h * w, 3 * c), np.float32), r(bias), images, h, w, ws, nh, hd)
    mask = oracle.qkv_split_window(np.ones((images * h * w, 3 * c), np.float32), np.zeros(3 * c, np.float32),
                                   images, h, w, ws, nh, hd)
    for gt, re, pa, mk in zip(got, real, pads, mask):
        assert gt.shape == re.shape
        assert np.array_equal(r(gt), np.where(mk > 0, re, pa))


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,c", [(1000, 768), (77, 1280), (33, 100), (5, 2048)])
def test_layer_norm(samrs, cuda, rows, c, dt):
    g = torch.Generator(device=cuda).manual_seed(rows + c)
    tdt = torch.float32 if dt == "f32" else DT[dt]
    x = (torch.randn(rows, c, generator=g, device=cuda) * 2 + 0.5).to(tdt)
    wt = (torch.randn(c, generator=g, device=cuda) * 0.2 + 1).to(tdt)
    b = (torch.randn(c, generator=g, device=cuda) * 0.1).to(tdt)
    out = samrs.layer_norm(x, wt, b, 1e-6)
    assert samrs.device_status() == 0
    err = parity_err(r(out), oracle.layer_norm(r(x), r(wt), r(b), 1e-6), dt)
    assert err < (1e-5 if dt == "f32" else 1e-3), err


def block_params(c, heads, window, g, dev, dt):
    """ViT block weights ~ N(0, 0.02), norms around 1 / 0, rel-pos tables ~ N(0, 0.5)."""
    hd, size = c // heads, (window if window else 64)
    shapes = dict(qkv_w=(3 * c, c), qkv_b=(3 * c,), proj_w=(c, c), proj_b=(c,), lin1_w=(4 * c, c), lin1_b=(4 * c,),
                  lin2_w=(c, 4 * c), lin2_b=(c,))
    p = {k: rnd(s, dt, dev, g, 0.02) for k, s in shapes.items()}
    for nm in ("norm1", "norm2"):
        p[nm + "_w"] = (1 + torch.randn(c, generator=g, device=dev) * 0.1).to(DT[dt])
        p[nm + "_b"] = rnd((c,), dt, dev, g, 0.05)
    p["rel_pos_h"] = rnd((2 * size - 1, hd), dt, dev, g, 0.5)
    p["rel_pos_w"] = rnd((2 * size - 1, hd), dt, dev, g, 0.5)
    return p


@pytest.mark.parametrize("window", [14, 0])
def test_block_matches_oracle(samrs, cuda, window):
    """One ViT-B block (C 768, 12 heads, f16, 1 image of 64 x 64 tokens), windowed (pad 64 -> 70) and global."""
    g = torch.Generator(device=cuda).manual_seed(11 + window)
    p = block_params(768, 12, window, g, cuda, "f16")
    x = rnd((1, 64, 64, 768), "f16", cuda, g)
    got = samrs.Block(p, 12, window).forward(x)
    assert samrs.device_status() == 0
    want = oracle.block_forward(r(x), {k: r(v) for k, v in p.items()}, 12, window)
    assert rel_max_err(r(got), want) < 5e-3
    assert mean_rel_err(r(got), want) < 1e-3


def test_vitb_stack_config2(samrs, cuda):
    """BASELINE config 2's stack, 12 ViT-B blocks (global at 2, 5, 8, 11, src/sam1/encoder.rs:20), f16, inputs
    ~ N(0, 1), weights ~ N(0, 0.02), one image, against the oracle chain of the same 12 blocks."""
    g = torch.Generator(device=cuda).manual_seed(2)
    params = [block_params(768, 12, 0 if i in (2, 5, 8, 11) else 14, g, cuda, "f16") for i in range(12)]
    x = rnd((1, 64, 64, 768), "f16", cuda, g)
    y, ref = x, r(x).astype(np.float64)
    for i, p in enumerate(params):
        win = 0 if i in (2, 5, 8, 11) else 14
        y = samrs.Block(p, 12, win).forward(y)
        ref = oracle.block_forward(ref, {k: r(v) for k, v in p.items()}, 12, win)
    assert samrs.device_status() == 0
    assert rel_max_err(r(y), ref) < 1e-2
    assert mean_rel_err(r(y), ref) < 2e-3


_GEMM_CHILD = r"""
import importlib, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[2])
samrs = importlib.import_module("sam-rs_b200")
dev = torch.device("cuda:0")
g = torch.Generator(device=dev).manual_seed(11)
outs = {}
for dt in (torch.bfloat16, torch.float16):
    for m, n, k in ((1000, 2304, 768), (257, 1280, 5120), (4096, 3840, 1280), (64, 80, 40)):
        a = torch.randn(m, k, generator=g, device=dev).to(dt)
        w = (0.05 * torch.randn(n, k, generator=g, device=dev)).to(dt)
        b = (0.1 * torch.randn(n, generator=g, device=dev)).to(dt)
        res = torch.randn(m, n, generator=g, device=dev).to(dt)
        for epi in ("bias", "bias_residual", "bias_gelu"):
            y = samrs.linear(a, w, b, res=res if epi == "bias_residual" else None, epilogue=epi)
            outs[f"{dt}-{m}-{n}-{k}-{epi}"] = y.view(torch.int16).cpu().numpy()
    x = torch.randn(2 * 64 * 64, 768, generator=g, device=dev).to(dt)
    wq = (0.05 * torch.randn(3 * 768, 768, generator=g, device=dev)).to(dt)
    bq = torch.randn(3 * 768, generator=g, device=dev).to(dt)
    for i, t in enumerate(samrs.qkv_linear_window(x, wq, bq, 2, 64, 64, 14, 12, 64)):
        outs[f"{dt}-qkv-{i}"] = t.contiguous().view(torch.int16).cpu().numpy()
assert samrs.device_status() == 0
np.savez(sys.argv[1], **outs)
"""


def test_single_cta_gemm_matches_cta_pairs(tmp_path):
    """The single-CTA GEMM kernel (one CTA per 128 x 256 tile, used where no 2-CTA cluster can be resident;
    forced with SAMRS_GEMM_SINGLE_CTA=1) writes bit for bit what the CTA-pair kernel writes: the three Linear
    epilogues at ragged and ViT-H shapes (K 40 .. 5120) and the fused qkv window layout, bf16 and f16. Each
    path runs in a child process of its own, since the choice is made once per process."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    files = {}
    for single in ("0", "1"):
        env = dict(os.environ, SAMRS_GEMM_SINGLE_CTA=single)
        f = str(tmp_path / f"gemm_{single}.npz")
        subprocess.run([sys.executable, "-c", _GEMM_CHILD, f, root], env=env, check=True, timeout=600)
        files[single] = np.load(f)
    assert set(files["0"].files) == set(files["1"].files)
    for key in files["0"].files:
        assert np.array_equal(files["0"][key], files["1"][key]), key
