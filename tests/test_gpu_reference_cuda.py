"""Parity against runs of the reference's own code: its CUDA kernels (kernels/sam.cu).

oracle/build_ref_cuda.py compiles that file, where it lies, with the flags of the reference's build.rs into
oracle/_ref/sam.cubin. oracle/ref_cuda.py launches the kernels with the reference's own launch
configurations (src/kernels.rs:1104-1131). These tests pin both the CPU oracle and this library's kernels
to that code:

* The reference's KAT `relpos_softmax_matches_fallback` (tests/kernels.rs:19-36) is re-run on the
  reference's kernel. It is checked against the oracle's restatement of the CPU fallback, at the KAT's own
  bar (max abs diff < 1e-3 with f16 inputs). The same is done in f32 and bf16, plus a ViT-H window shape.
  This library's softmax-only export is compared with the reference's kernel directly.
* qkv_split: this library's kernel and the oracle against the reference's kernel, bit for bit, in the
  reference test's shape (tests/kernels.rs:39-50) and at ViT-H.
* bias_residual / bias_gelu: the oracle's restatements against the reference's kernels (f32). The fused
  GEMM epilogues against the reference's unfused path (cuBLAS product rounded to the I/O dtype, then the
  reference's kernel), at the reference test's bar (max abs diff < 2e-2, tests/kernels.rs:52-58).
* The reference's CUDA attention path, bmm(relpos_softmax(bmm(q, kt)), v) (src/sam1/encoder.rs:81), is
  compared with the oracle and with the fused kernels. In f32 all three agree to 1e-4 (relative). In f16
  and bf16 the reference path rounds S and P to the I/O dtype; the fused kernels must be at least as close
  to the exact oracle as that path is.
"""
import os

import numpy as np
import pytest

from oracle import build_ref_cuda, oracle
from tests.helpers import F32_TOL, HALF_TOL, ROUNDING_SLACK, make_inputs, parity_err, rel_max_err

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(build_ref_cuda.OUT),
                                 reason="oracle/_ref/sam.cubin not built (the reference's kernels/sam.cu was absent "
                                        "at build time)")]

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
# the reference KAT's bar (f16 inputs, tests/kernels.rs:34); bf16 adds half an output ulp of a probability
# near 1 (2^-9); f32 (not in the reference's KAT) the fast-math exponential's error
SOFTMAX_BAR = {"f16": 1e-3, "bf16": 1e-3 + 2.0 ** -9, "f32": 1e-5}


@pytest.fixture(scope="module")
def ref(cuda):
    from oracle.ref_cuda import RefCuda
    return RefCuda()


def dev(a, dt, cuda):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(cuda).to(DT[dt])


def host(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 6, 64), (64, 64, 2, 64), (7, 11, 3, 80), (14, 14, 8, 80)])
def test_reference_softmax_kernel_vs_oracle(samrs, cuda, ref, h, w, bh, hd, dt):
    """tests/kernels.rs:19-36 on the reference's kernel: N(0,1) scores, q and table, scale 0.125."""
    n = h * w
    rng = np.random.default_rng(1000 + h * 7 + w + hd)
    s = rng.standard_normal((bh, n, n), dtype=np.float32)
    q = rng.standard_normal((bh, n, hd), dtype=np.float32)
    t = rng.standard_normal(((2 * h - 1) + (2 * w - 1), hd), dtype=np.float32)
    sd, qd, td = dev(s, dt, cuda), dev(q, dt, cuda), dev(t, dt, cuda)
    got_ref = ref.relpos_softmax(sd, qd, td, h, w, 0.125)
    got_ours = samrs.relpos_softmax(sd, qd, td, h, w, 0.125)
    torch.cuda.synchronize()
    want = oracle.relpos_softmax(host(sd), host(qd), host(td), h, w, 0.125)
    d_ref = float(np.abs(host(got_ref) - want).max())
    d_ours = float(np.abs(host(got_ours) - want).max())
    d_pair = float((got_ref.float() - got_ours.float()).abs().max())
    print(f"relpos_softmax {h}x{w} hd {hd} {dt}: max abs diff reference kernel vs oracle {d_ref:.2e}, "
          f"ours vs oracle {d_ours:.2e}, ours vs reference kernel {d_pair:.2e}")
    assert d_ref < SOFTMAX_BAR[dt], d_ref
    assert d_ours < SOFTMAX_BAR[dt], d_ours
    assert d_pair < SOFTMAX_BAR[dt], d_pair


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n,nh,hd,win", [(196, 12, 64, 3), (196, 16, 80, 2), (4096, 16, 80, 1)])
def test_qkv_split_bit_exact_vs_reference_kernel(samrs, cuda, ref, n, nh, hd, win, dt):
    """The reference test's shape (tests/kernels.rs:39-50: 196 tokens, 12 heads, hd 64, 3 windows) and ViT-H
    windowed and global shapes: identical bits from this library's kernel, the reference's kernel and (f32
    inputs) the oracle."""
    rng = np.random.default_rng(n + nh + hd)
    c = nh * hd
    y = dev(rng.standard_normal((win * n, 3 * c), dtype=np.float32), dt, cuda)
    b = dev(rng.standard_normal(3 * c, dtype=np.float32), dt, cuda)
    r = ref.qkv_split(y, b, n, nh, hd)
    o = samrs.qkv_split(y, b, n, nh, hd)
    torch.cuda.synchronize()
    for a, e in zip(o, r):
        assert a.shape == e.shape
        assert torch.equal(a, e)
    if dt == "f32":
        for a, e in zip(oracle.qkv_split(host(y), host(b), n, nh, hd), r):
            assert np.array_equal(a, host(e))


def test_bias_kernels_vs_oracle(cuda, ref):
    """The oracle's bias_residual and erf GELU (float64) against the reference's kernels in f32."""
    rng = np.random.default_rng(5)
    c = 768
    res = rng.standard_normal((64, c), dtype=np.float32)
    y = rng.standard_normal((64, c), dtype=np.float32) * 3
    b = rng.standard_normal(c, dtype=np.float32)
    got = host(ref.bias_residual(dev(res, "f32", cuda), dev(y, "f32", cuda), dev(b, "f32", cuda)))
    assert np.abs(got - oracle.bias_residual(res, y, b)).max() < 1e-5
    y4 = rng.standard_normal((64, 4 * c), dtype=np.float32) * 3
    b4 = rng.standard_normal(4 * c, dtype=np.float32)
    got = host(ref.bias_gelu(dev(y4, "f32", cuda), dev(b4, "f32", cuda)))
    d = float(np.abs(got - oracle.bias_gelu(y4, b4)).max())
    print(f"bias_gelu: reference kernel (f32, fast math) vs oracle (float64 erf): max abs diff {d:.2e}")
    assert d < 1e-5, d


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_gemm_epilogues_vs_reference_path(samrs, cuda, ref, dt):
    """The fused GEMM epilogues against the reference's unfused CUDA path: the cuBLAS product in the I/O
    dtype, then the reference's bias_residual / bias_gelu kernel (src/sam1/encoder.rs:83-84, 121-128). Both
    are held to the reference test's bar against the float64 oracle, and the fused epilogue (no rounding of
    the product before the bias) must be at least as close to the oracle as the reference's path."""
    rng = np.random.default_rng(17)
    m, k = 512, 768
    a = dev(rng.standard_normal((m, k), dtype=np.float32), dt, cuda)
    for n, epi in ((3072, "bias_gelu"), (768, "bias_residual")):
        w = dev(rng.standard_normal((n, k), dtype=np.float32) * 0.02, dt, cuda)
        b = dev(rng.standard_normal(n, dtype=np.float32) * 0.1, dt, cuda)
        res = dev(rng.standard_normal((m, n), dtype=np.float32), dt, cuda) if epi == "bias_residual" else None
        y = ref.matmul(a, w.t())
        ref_out = ref.bias_gelu(y, b) if epi == "bias_gelu" else ref.bias_residual(res, y, b)
        ours = samrs.linear(a, w, b, res=res, epilogue=epi)
        torch.cuda.synchronize()
        exact = oracle.linear(host(a), host(w))
        exact = oracle.bias_gelu(exact, host(b)) if epi == "bias_gelu" else oracle.bias_residual(host(res), exact,
                                                                                              host(b))
        e_ref = float(np.abs(host(ref_out) - exact).max())
        e_ours = float(np.abs(host(ours) - exact).max())
        print(f"{epi} {dt}: max abs diff vs float64 oracle: reference path {e_ref:.2e}, fused {e_ours:.2e}")
        assert e_ref < 2e-2 and e_ours < 2e-2
        assert e_ours <= e_ref * 1.05 + 1e-6, (e_ours, e_ref)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 37, 80), (64, 64, 2, 80), (14, 14, 50, 64), (64, 64, 3, 64),
                                       (7, 11, 3, 80)])
def test_reference_cuda_attention_path(samrs, cuda, ref, h, w, bh, hd, dt):
    """The reference's CUDA attention path against the exact oracle and the fused kernels (ViT scale
    hd^-0.5, tables N(0, 0.5))."""
    q, kt, v, t = make_inputs(h, w, bh, hd, seed=h * 31 + bh + hd, table_std=0.5)
    scale = hd ** -0.5
    qd, ktd, vd, td = (dev(x, dt, cuda) for x in (q, kt, v, t))
    path = ref.attention(qd, ktd, vd, td, h, w, scale)
    fused = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale)
    assert samrs.device_status() == 0
    exact = oracle.attention_relpos(host(qd), host(ktd), host(vd), host(td), h, w, scale)
    e_path = rel_max_err(host(path), exact)
    e_fused = rel_max_err(host(fused), exact)
    e_pair = rel_max_err(host(fused), host(path))
    print(f"attention {h}x{w} bh {bh} hd {hd} {dt}: max|x-oracle|/max|oracle|: reference CUDA path {e_path:.2e}, "
          f"fused {e_fused:.2e}; fused vs reference path {e_pair:.2e}")
    if dt == "f32":
        assert e_path < F32_TOL and e_fused < F32_TOL and e_pair < F32_TOL
    else:
        assert parity_err(host(fused), exact, dt) < HALF_TOL
        assert e_fused <= max(e_path, HALF_TOL + ROUNDING_SLACK[dt]), (e_fused, e_path)


GOLDEN = sorted(__import__("glob").glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_golden_fixtures_vs_reference_kernels(cuda, ref, path):
    """The committed golden fixtures (float64 restatement of the reference's tensor-op fallback) against the
    reference's own CUDA code in f32: its attention path for the stored output rows, its relpos_softmax
    kernel for the stored probability rows (scores rounded to f16 as the fixture's softmax KAT does)."""
    from tests.golden.make_golden import digest, f16_round, make_inputs as golden_inputs
    g = np.load(path)
    h, w, bh, hd, seed = (int(g[k]) for k in ("h", "w", "bh", "hd", "seed"))
    scale = float(g["scale"])
    q, kt, v, t = golden_inputs(h, w, bh, hd, seed)
    assert digest(q, kt, v, t) == str(g["input_sha256"])
    qd, ktd, vd, td = (dev(x, "f32", cuda) for x in (q, kt, v, t))
    out = host(ref.attention(qd, ktd, vd, td, h, w, scale))[:, g["rows"], :]
    e_out = rel_max_err(out, g["out_rows"])
    s16 = torch.from_numpy(f16_round(np.matmul(q.astype(np.float64), kt.astype(np.float64)).astype(np.float32)))
    probs = host(ref.relpos_softmax(s16.to(cuda).contiguous(), qd, td, h, w, scale))[:, g["probs_row_ids"], :]
    e_p = float(np.abs(probs - g["probs_rows"]).max())
    print(f"{os.path.basename(path)}: reference CUDA path vs fixture {e_out:.2e} (relative), reference softmax "
          f"kernel vs fixture {e_p:.2e} (abs)")
    assert e_out < 1e-5, e_out
    assert e_p < 1e-5, e_p
