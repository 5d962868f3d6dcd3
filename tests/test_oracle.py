"""CPU oracle (oracle/relpos_oracle.c) against the golden fixtures and against the reference's own
CPU-side tests (tests/cpu_gemm.rs:29-50 bf16-vs-exact bar, src/kernels.rs:887-893 qkv_split fallback)."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle
from tests.golden.make_golden import digest, f16_round, make_inputs
from tests.helpers import make_inputs as make_rand, mean_rel_err, rel_max_err

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def load(path):
    g = np.load(path)
    h, w, bh, hd, seed = (int(g[k]) for k in ("h", "w", "bh", "hd", "seed"))
    q, kt, v, t = make_inputs(h, w, bh, hd, seed)
    assert digest(q, kt, v, t) == str(g["input_sha256"]), "fixture inputs no longer regenerate bit-identically"
    return g, (h, w, bh, hd), (q, kt, v, t)


def test_fixtures_present():
    assert len(GOLDEN) == 4


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_exact_attention_matches_golden(path):
    g, (h, w, bh, hd), (q, kt, v, t) = load(path)
    out = oracle.attention_relpos(q, kt, v, t, h, w, float(g["scale"]))
    assert rel_max_err(out[:, g["rows"], :], g["out_rows"]) < 1e-5


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_softmax_matches_golden(path):
    g, (h, w, bh, hd), (q, kt, v, t) = load(path)
    s = f16_round(np.matmul(q, kt))
    p = oracle.relpos_softmax(s, q, t, h, w, float(g["scale"]))
    assert np.abs(p[:, g["probs_row_ids"], :] - g["probs_rows"]).max() < 1e-5
    np.testing.assert_allclose(p.sum(-1), 1.0, rtol=1e-5)


@pytest.mark.skipif(not oracle.cpu_has_bf16(), reason="CPU lacks AVX-512 BF16")
@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 6, 64), (64, 64, 2, 64), (7, 11, 3, 80)])
def test_bf16_path_within_reference_bar(h, w, bh, hd):
    # tests/cpu_gemm.rs:29-50: N(0,1) inputs, scale 0.125, mean relative error < 1.5e-2
    q, kt, v, t = make_rand(h, w, bh, hd, seed=h * 1000 + w)
    exact = oracle.attention_relpos(q, kt, v, t, h, w, 0.125)
    fast = oracle.attention_relpos(q, kt, v, t, h, w, 0.125, mode="bf16")
    assert mean_rel_err(fast, exact) < 1.5e-2


def test_qkv_split_matches_tensor_fallback():
    # src/kernels.rs:890-893: broadcast_add, reshape (t/n, n, 3, nh, hd), permute (2, 0, 3, 1, 4)
    n, nh, hd, win = 196, 12, 64, 3
    rng = np.random.default_rng(5)
    y = rng.standard_normal((win * n, 3 * nh * hd), dtype=np.float32)
    b = rng.standard_normal(3 * nh * hd, dtype=np.float32)
    q, kt, v = oracle.qkv_split(y, b, n, nh, hd)
    qkv = (y + b).reshape(win, n, 3, nh, hd).transpose(2, 0, 3, 1, 4).reshape(3, win * nh, n, hd)
    np.testing.assert_array_equal(q, qkv[0])
    np.testing.assert_array_equal(kt, qkv[1].transpose(0, 2, 1))
    np.testing.assert_array_equal(v, qkv[2])


@pytest.mark.parametrize("h,w,bh,hd", [(1, 1, 2, 8), (3, 5, 2, 16), (2, 9, 1, 7), (14, 14, 1, 80)])
def test_ragged_shapes_match_float64(h, w, bh, hd):
    from tests.golden.make_golden import reference_attention
    q, kt, v, t = make_rand(h, w, bh, hd, seed=7 + h + w)
    out = oracle.attention_relpos(q, kt, v, t, h, w, 0.3)
    ref, _, _ = reference_attention(q, kt, v, t, h, w, 0.3)
    assert rel_max_err(out, ref) < 1e-5


def test_empty_batch():
    q, kt, v, t = make_rand(4, 4, 0, 8, seed=1)
    assert oracle.attention_relpos(q, kt, v, t, 4, 4, 0.5).shape == (0, 16, 8)


@pytest.mark.parametrize("b,h,w,ws", [(2, 64, 64, 14), (1, 13, 20, 7), (3, 14, 14, 14)])
def test_window_partition_matches_package_mirror(b, h, w, ws):
    """The oracle's numpy window_partition / window_unpartition (src/sam1/encoder.rs:132-145) against the
    package's torch mirror (the layout the model code uses), both ways."""
    import torch
    from tests.conftest import load_samrs
    s = load_samrs()
    x = np.random.default_rng(b + h + w).standard_normal((b, h, w, 5), dtype=np.float32)
    parts = oracle.window_partition(x, ws)
    tparts, hp, wp = s.window_partition(torch.from_numpy(x), ws)
    assert np.array_equal(parts, tparts.numpy())
    assert np.array_equal(oracle.window_unpartition(parts, ws, h, w), x)
    back = s.window_unpartition(tparts, ws, hp, wp, (h, w), b, 5)
    assert np.array_equal(back.numpy(), x)


@pytest.mark.parametrize("images,h,w,ws,nh,hd", [(2, 13, 20, 7, 3, 8), (1, 16, 16, 0, 2, 8)])
def test_window_merge_inverts_split(images, h, w, ws, nh, hd):
    """window_merge(q of qkv_split_window) is y_q + b_q on the real tokens; pad tokens hold the bias."""
    rng = np.random.default_rng(images * 7 + h)
    c = nh * hd
    y = rng.standard_normal((images * h * w, 3 * c), dtype=np.float32)
    b = rng.standard_normal(3 * c, dtype=np.float32)
    q, kt, v = oracle.qkv_split_window(y, b, images, h, w, ws, nh, hd)
    assert np.array_equal(oracle.window_merge(q, images, h, w, ws, nh, hd), y[:, :c] + b[:c])
    assert np.array_equal(oracle.window_merge(v, images, h, w, ws, nh, hd), y[:, 2 * c:] + b[2 * c:])
    if ws:
        # the last window of image 0 starts in the grid and runs past it: its pad tokens are the bias
        nww = -(-w // ws)
        last = (nww - 1) * nh  # window (0, nww-1), head 0
        tok_pad = ws - 1  # column (nww-1)*ws + ws-1 >= w
        assert np.array_equal(q[last, tok_pad], b[:hd])


def test_block_oracle_matches_torch_definitions():
    """oracle.block_forward (numpy, the reference's order) against the same block written with torch's own
    layer_norm / exact GELU / matmul on CPU, with the attention taken from the oracle in both."""
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(4)
    c, nh, ws = 64, 2, 7
    shapes = dict(qkv_w=(3 * c, c), qkv_b=(3 * c,), proj_w=(c, c), proj_b=(c,), lin1_w=(4 * c, c), lin1_b=(4 * c,),
                  lin2_w=(c, 4 * c), lin2_b=(c,), norm1_w=(c,), norm1_b=(c,), norm2_w=(c,), norm2_b=(c,),
                  rel_pos_h=(13, 32), rel_pos_w=(13, 32))
    p = {k: (rng.standard_normal(s) * 0.1).astype(np.float64) for k, s in shapes.items()}
    p["norm1_w"] += 1
    p["norm2_w"] += 1
    x = rng.standard_normal((1, 12, 12, c))
    got = oracle.block_forward(x, p, nh, ws)
    t = {k: torch.from_numpy(v) for k, v in p.items()}
    xt = torch.from_numpy(x)
    y = F.layer_norm(xt, (c,), t["norm1_w"], t["norm1_b"], 1e-6).numpy()
    parts = oracle.window_partition(y, ws)
    attn = oracle.window_unpartition(oracle.attention_block(parts, p, nh), ws, 12, 12)
    x1 = xt + torch.from_numpy(np.asarray(attn)) + t["proj_b"]
    hmid = F.gelu(F.layer_norm(x1, (c,), t["norm2_w"], t["norm2_b"], 1e-6) @ t["lin1_w"].T + t["lin1_b"])
    want = (x1 + hmid @ t["lin2_w"].T + t["lin2_b"]).numpy()
    assert np.abs(got - want).max() < 1e-9 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 3, 64), (7, 11, 2, 80), (8, 8, 2, 16)])
def test_bench_fp32_reference_matches_oracle(h, w, bh, hd):
    """bench.py's PyTorch fp32 reference (the per-rank sampled parity of the bench line) computes the op the
    oracle computes: square and non-square grids."""
    import torch
    import bench
    rng = np.random.default_rng(h * w + hd)
    n = h * w
    q = rng.standard_normal((bh, n, hd), dtype=np.float32)
    kt = rng.standard_normal((bh, hd, n), dtype=np.float32)
    v = rng.standard_normal((bh, n, hd), dtype=np.float32)
    t = 0.5 * rng.standard_normal((2 * h - 1 + 2 * w - 1, hd), dtype=np.float32)
    ref = oracle.attention_relpos(q, kt, v, t, h, w, 0.125)
    got = bench.relpos_attention_fp32(torch, *(torch.from_numpy(x) for x in (q, kt, v, t)), h, w, 0.125).numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-5
