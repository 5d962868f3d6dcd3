"""Parity of the CUDA path (through the C ABI) with the CPU oracle on the same seeded inputs.

Bars (tests/helpers.py): f32 I/O max|got-ref|/max|ref| <= 1e-4; f16/bf16 I/O: the error beyond half an
ulp of the I/O dtype, max(|got-ref| - ulp/2, 0)/max|ref|, <= 3e-3, against the exact-f32 oracle fed the
same 16-bit-rounded inputs (the reference's KAT rounds its inputs the same way, tests/kernels.rs:28-31). Geometries: the reference's KATs (tests/kernels.rs:23), config 1 at full
size, ViT-L/H shapes, ragged and edge shapes; full-size ViT-H batches through size-independent
properties (linearity in v, convex-combination bounds) plus oracle checks of sampled heads.
"""
import glob
import os

import numpy as np
import pytest

from oracle import oracle
from tests.golden.make_golden import digest, f16_round, make_inputs as golden_inputs
from tests.helpers import F32_TOL, HALF_TOL, excess_err, make_inputs, mean_rel_err, parity_err, rel_max_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def to_dev(a, dt, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(DT[dt])


def rounded(t):
    return t.float().cpu().numpy()


def run_case(samrs, dev, h, w, bh, hd, dt, impl, seed, scale=0.125, table_std=1.0):
    q, kt, v, t = make_inputs(h, w, bh, hd, seed, table_std)
    qd, ktd, vd, td = (to_dev(x, dt, dev) for x in (q, kt, v, t))
    out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale, impl=impl)
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), h, w, scale)
    got = out.float().cpu().numpy()
    assert mean_rel_err(got, ref) < (1e-5 if dt == "f32" else 3e-3)
    return parity_err(got, ref, dt)


def tol(dt):
    return F32_TOL if dt == "f32" else HALF_TOL


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_golden_fixtures(samrs, cuda, path, dt):
    # Fixture inputs are f16-representable, so f32 and f16 runs see identical values.
    g = np.load(path)
    h, w, bh, hd, seed = (int(g[k]) for k in ("h", "w", "bh", "hd", "seed"))
    q, kt, v, t = golden_inputs(h, w, bh, hd, seed)
    assert digest(q, kt, v, t) == str(g["input_sha256"])
    out = samrs.attention_relpos(*(to_dev(x, dt, cuda) for x in (q, kt, v, t)), h, w, float(g["scale"]))
    got = out.float().cpu().numpy()[:, g["rows"], :]
    assert parity_err(got, g["out_rows"], dt) < tol(dt)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("impl", ["auto", "simt"])
@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 6, 64), (64, 64, 2, 64), (7, 11, 3, 80)])
def test_reference_kat_geometries(samrs, cuda, h, w, bh, hd, dt, impl):
    err = run_case(samrs, cuda, h, w, bh, hd, dt, impl, seed=h * 100 + w + bh)
    assert err < tol(dt), err


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("h,w,bh,hd", [(64, 64, 3, 80), (14, 14, 37, 80), (14, 14, 50, 64), (64, 64, 4, 64)])
def test_vit_shapes_tensor_core_path(samrs, cuda, h, w, bh, hd, dt):
    err = run_case(samrs, cuda, h, w, bh, hd, dt, "auto", seed=bh * 7 + hd, table_std=0.5)
    assert err < HALF_TOL, err


@pytest.mark.parametrize("h,w,bh,hd,dt", [(1, 1, 3, 8, "f32"), (2, 3, 5, 1, "f32"), (3, 17, 2, 33, "bf16"),
                                          (5, 5, 1, 128, "f16"), (128, 1, 1, 16, "f32"), (9, 64, 2, 72, "bf16"),
                                          (32, 32, 1, 96, "f32")])
def test_ragged_and_edge_shapes(samrs, cuda, h, w, bh, hd, dt):
    err = run_case(samrs, cuda, h, w, bh, hd, dt, "auto", seed=h + w + hd)
    assert err < tol(dt), err


def test_config1_full_size_f32(samrs, cuda):
    # ViT-B op, f32, one image. Windowed: 25 windows x 12 heads, 196 tokens, hd 64;
    # global: 12 heads x 4096 tokens; rel tables ~ N(0, 0.5); scale 64^-0.5.
    for (h, w, bh) in [(14, 14, 300), (64, 64, 12)]:
        err = run_case(samrs, cuda, h, w, bh, 64, "f32", "auto", seed=bh, scale=64 ** -0.5, table_std=0.5)
        assert err < F32_TOL, (h, err)


@pytest.mark.parametrize("h,w,bh,hd", [(64, 64, 512, 80), (14, 14, 12800, 80), (64, 64, 256, 64), (14, 14, 6400, 64)],
                         ids=["config4-global", "config4-window", "config3-global", "config3-window"])
def test_full_batch_properties(samrs, cuda, h, w, bh, hd):
    """BASELINE configs 4 (ViT-H, 32 images: 16 heads, hd 80) and 3 (ViT-L, 16 images: 16 heads, hd 64) at full
    size, bf16: linearity in v and convex-combination bounds over every head, and the oracle on heads sampled
    evenly over the whole batch (32 per global layer, 64 per windowed layer)."""
    g = torch.Generator(device=cuda).manual_seed(1234 + h + hd)
    n = h * w
    q = torch.randn(bh, n, hd, device=cuda, generator=g).bfloat16()
    kt = torch.randn(bh, hd, n, device=cuda, generator=g).bfloat16()
    v1 = torch.randn(bh, n, hd, device=cuda, generator=g).bfloat16()
    v2 = torch.randn(bh, n, hd, device=cuda, generator=g).bfloat16()
    t = (torch.randn(4 * h - 2, hd, device=cuda, generator=g) * 0.5).bfloat16()
    scale = hd ** -0.5
    o1 = samrs.attention_relpos(q, kt, v1, t, h, w, scale)
    o2 = samrs.attention_relpos(q, kt, v2, t, h, w, scale)
    o12 = samrs.attention_relpos(q, kt, (v1.float() + v2.float()).bfloat16(), t, h, w, scale)
    assert samrs.device_status() == 0
    # softmax weights do not depend on v: out(v1+v2) = out(v1) + out(v2) up to bf16 rounding of v1+v2 and outputs
    lin = (o12.float() - o1.float() - o2.float()).abs().max().item() / o12.float().abs().max().item()
    assert lin < 2e-2, lin
    # each output row is a convex combination of the rows of v
    vmax = v1.float().amax(dim=1, keepdim=True)
    vmin = v1.float().amin(dim=1, keepdim=True)
    slack = 1e-2 * vmax.abs().clamp(min=1)
    assert bool(((o1.float() <= vmax + slack) & (o1.float() >= vmin - slack)).all())
    heads = np.unique(np.linspace(0, bh - 1, 32 if h == 64 else 64).round().astype(int))
    idx = torch.from_numpy(heads).to(cuda)
    ref = oracle.attention_relpos(rounded(q[idx]), rounded(kt[idx]), rounded(v1[idx]), rounded(t), h, w, scale)
    err = parity_err(o1[idx].float().cpu().numpy(), ref, "bf16")
    assert err < HALF_TOL, err


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("hd", [64, 80])
def test_global_late_max_jumps(samrs, cuda, hd, dt):
    """Row maxima that jump late in the key sequence (64x64 global layer): the online softmax's rescaling.

    Every query has a large first coordinate and a few keys have a large first coordinate, so that a
    query's max logit jumps by 25 to 30 log2 units at a later 128-key tile (far beyond the largest P a
    16-bit type holds against the earlier reference): in the first tiles, in the middle, and in the last
    tile only, per head; head 1 jumps by ~130 in the last tile (beyond an f32 P against the earlier
    reference: the bf16 single-pass CTA must be recomputed). Most rows end up dominated by one key, whose
    16-bit P rounding must cancel between the numerator and the row sum."""
    h = w = 64
    q, kt, v, t = make_inputs(h, w, 3, hd, seed=hd + 5, table_std=0.5)
    q[:, :, 0] = 4.0
    jumps = {0: {128 * 1 + 3: 40.0, 128 * 9 + 77: 80.0, 128 * 31 + 127: 120.0},
             1: {128 * 31 + 5: 200.0},
             2: {128 * 2 + 64: 40.0, 128 * 3 + 1: 80.0, 128 * 4 + 2: 120.0, 128 * 20 + 90: 160.0}}
    for b, keys in jumps.items():
        for key, big in keys.items():
            kt[b, 0, key] = big
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, dt, cuda) for x in (q, kt, v, t))
    samrs.global_policy(td, reset=True)  # bf16: the speculative pass and its fixup, whatever ran before
    out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale)
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), h, w, scale)
    err = parity_err(out.float().cpu().numpy(), ref, dt)
    assert err < tol(dt), err


@pytest.mark.parametrize("h,w,bh,hd", [(64, 64, 3, 80), (14, 14, 37, 80), (14, 14, 50, 64), (64, 64, 4, 64)])
def test_f32_tensor_core_path(samrs, cuda, h, w, bh, hd):
    """f32 I/O on the tensor cores (kind::tf32 MMAs on operands split in two TF32 terms), forced with
    impl="tc", against the oracle at the f32 bar: ViT-B/L (hd 64) and ViT-H (hd 80) global and windowed shapes."""
    err = run_case(samrs, cuda, h, w, bh, hd, "f32", "tc", seed=bh * 5 + hd, table_std=0.5)
    assert err < F32_TOL, err


@pytest.mark.parametrize("hd", [64, 80])
def test_window_f32_late_max(samrs, cuda, hd):
    """f32 windowed layers: row maxima that jump by 40-100 log2 units in the second, third or last (partly
    masked) 64-key tile, so that the lazily rescaled running maximum must rescale O."""
    h = w = 14
    q, kt, v, t = make_inputs(h, w, 12, hd, seed=hd + 3, table_std=0.5)
    q[:, :, 0] = 4.0
    for b in range(12):
        kt[b, 0, [70, 140, 195][b % 3]] = 40.0 + 20.0 * (b % 4)
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, "f32", cuda) for x in (q, kt, v, t))
    out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale, impl="tc")
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), h, w, scale)
    err = parity_err(out.float().cpu().numpy(), ref, "f32")
    assert err < F32_TOL, err


@pytest.mark.parametrize("table_std", [0.1, 0.5, 8.0])
@pytest.mark.parametrize("hd", [64, 80])
def test_window_bf16_single_pass(samrs, cuda, hd, table_std):
    """bf16 windowed layers take a single pass per row with the reference from the row's first 32 keys:
    small tables, the bench's N(0, 0.5), and N(0, 8), whose rh spreads of hundreds of log2 units make later
    key rows exceed the reference by more than 64 (the reference is raised, the P already written scaled).
    A few keys with large scores make rows dominated by one key."""
    h = w = 14
    q, kt, v, t = make_inputs(h, w, 40, hd, seed=hd + int(table_std * 10), table_std=table_std)
    kt[::3, :, 17] *= 6.0
    err = parity_err(*_run_window_bf16(samrs, cuda, q, kt, v, t, hd), "bf16")
    assert err < HALF_TOL, err


@pytest.mark.parametrize("hd", [64, 80])
def test_window_bf16_late_max_raises_reference(samrs, cuda, hd):
    """bf16 windowed layers: row maxima that jump past the single pass's reference (the max of the row's first
    32 keys) by more than 64 log2 units in a later 32-key chunk, once (chunk 1), twice (chunks 1 and 4), three
    times (chunks 1, 4 and the last, partly masked chunk 6) or only in the last chunk; heads whose jump stays
    below the limit (P up to 2^39, no raise) and heads without a jump. Only the even query rows see the jumps,
    so every warp mixes rows that raise the reference with rows that keep it."""
    h = w = 14
    bh = 24
    q, kt, v, t = make_inputs(h, w, bh, hd, seed=hd + 11, table_std=0.5)
    q[:, ::2, 0] = 4.0
    for b in range(bh):
        kind = b % 6
        keys = {0: [], 1: [40], 2: [40, 150], 3: [40, 150, 195], 4: [195], 5: [100]}[kind]
        bigs = {4: [120.0], 5: [60.0]}.get(kind, [120.0, 250.0, 400.0])
        for key, big in zip(keys, bigs):
            kt[b, 0, key] = big
    err = parity_err(*_run_window_bf16(samrs, cuda, q, kt, v, t, hd), "bf16")
    assert err < HALF_TOL, err


def _run_window_bf16(samrs, cuda, q, kt, v, t, hd):
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, "bf16", cuda) for x in (q, kt, v, t))
    out = samrs.attention_relpos(qd, ktd, vd, td, 14, 14, scale)
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), 14, 14, scale)
    return out.float().cpu().numpy(), ref


@pytest.mark.parametrize("hd", [64, 80])
def test_global_bf16_overflow_recompute(samrs, cuda, hd):
    """bf16 global layers: a CTA whose single-pass tiles would overflow is recomputed exactly.

    v ~ 1e35 and, per head, one key in a later tile whose logit jumps ~25-29 log2 units above the running
    max: the single-pass tile's P of that key reaches ~2^25, P.V overflows f32, and the CTA must take the
    exact pass (P <= 2^8 there, so O stays finite)."""
    h = w = 64
    q, kt, v, t = make_inputs(h, w, 2, hd, seed=hd + 11, table_std=0.5)
    q[:, :, 0] = 4.0
    v *= 1e35
    kt[0, 0, 128 * 5 + 17] = 40.0
    kt[1, 0, 128 * 30 + 101] = 40.0
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, "bf16", cuda) for x in (q, kt, v, t))
    samrs.global_policy(td, reset=True)
    out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale)
    assert samrs.device_status() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), h, w, scale)
    err = parity_err(got, ref, "bf16")
    assert err < HALF_TOL, err


def test_global_bf16_fixup_several_blocks_per_cta(samrs, cuda):
    """The bf16 fixup launch runs at most one CTA per SM, each recomputing every marked block of its share in
    turn: 24 heads x 16 blocks = 384 blocks, all marked (a key in a late tile jumps ~26 log2 units above the
    running max of every row and v ~ 1e35, so every single-pass block overflows), i.e. two or three blocks per
    CTA. Every block is counted once, and sampled heads match the oracle."""
    h = w = 64
    hd, bh = 80, 24
    q, kt, v, t = make_inputs(h, w, bh, hd, seed=31, table_std=0.5)
    q[:, :, 0] = 4.0
    v *= 1e35
    for b in range(bh):
        kt[b, 0, 128 * (20 + b % 12) + 7 * b % 128] = 40.0
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, "bf16", cuda) for x in (q, kt, v, t))
    samrs.global_policy(td, reset=True)
    samrs.recompute_count(clear=True)
    out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale)
    assert samrs.recompute_count(clear=True) == bh * 16
    assert samrs.device_status() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    heads = [0, 7, 16, 23]
    ref = oracle.attention_relpos(rounded(qd[heads]), rounded(ktd[heads]), rounded(vd[heads]), rounded(td), h, w, scale)
    err = parity_err(got[heads], ref, "bf16")
    assert err < HALF_TOL, err


def test_bf16_recompute_counter(samrs, cuda):
    """The recompute counter: random N(0,1) activations and N(0,0.5) tables need no exact second pass; the
    overflow case above marks some CTAs (one head x 256 rows each) and the counter sees them."""
    samrs.recompute_count(clear=True)
    q, kt, v, t = make_inputs(64, 64, 4, 80, seed=3, table_std=0.5)
    args = [to_dev(x, "bf16", cuda) for x in (q, kt, v, t)]
    samrs.global_policy(args[3], reset=True)
    samrs.attention_relpos(*args, 64, 64, 80 ** -0.5)
    assert samrs.recompute_count() == 0
    q, kt, v, t = make_inputs(64, 64, 2, 80, seed=91, table_std=0.5)
    q[:, :, 0] = 4.0
    v *= 1e35
    kt[0, 0, 128 * 5 + 17] = 40.0
    args = [to_dev(x, "bf16", cuda) for x in (q, kt, v, t)]
    samrs.global_policy(args[3], reset=True)
    samrs.attention_relpos(*args, 64, 64, 80 ** -0.5)
    assert samrs.device_status() == 0
    assert 1 <= samrs.recompute_count() <= 2 * 16


def test_global_bf16_policy_switches_to_exact(samrs, cuda):
    """A bf16 global layer whose CTAs mostly need the exact second pass (activations and rel-pos table of
    std 2: rel-pos bias spreads of hundreds of log2 units) is switched to the exact kernel alone once its
    measured recompute share is read back, returns to the speculative pass (measured again) after 32 exact
    calls, and stays speculative on ordinary data. Every output matches the oracle on sampled heads."""
    h = w = 64
    hd, bh = 80, 16
    q, kt, v, t = make_inputs(h, w, bh, hd, seed=123, table_std=2.0)
    q *= 2.0
    kt *= 2.0
    scale = hd ** -0.5
    qd, ktd, vd, td = (to_dev(x, "bf16", cuda) for x in (q, kt, v, t))
    heads = [0, 7, 15]
    ref = oracle.attention_relpos(rounded(qd)[heads], rounded(ktd)[heads], rounded(vd)[heads], rounded(td), h, w,
                                  scale)

    def run():
        out = samrs.attention_relpos(qd, ktd, vd, td, h, w, scale)
        assert samrs.device_status() == 0
        err = parity_err(out.float().cpu().numpy()[heads], ref, "bf16")
        assert err < HALF_TOL, err

    share, exact = samrs.global_policy(td, reset=True)
    assert (share, exact) == (-1.0, False)
    samrs.recompute_count(clear=True)
    run()  # speculative pass + fixup, measured
    recomputed = samrs.recompute_count(clear=True)
    share, exact = samrs.global_policy(td)
    assert share == recomputed / (bh * 16) and share > 0.15 and exact, (share, recomputed)
    for _ in range(32):
        run()  # the exact kernel alone: nothing for the fixup to count
    assert samrs.recompute_count(clear=True) == 0
    share2, exact2 = samrs.global_policy(td)
    assert not exact2 and share2 == share
    run()  # the probe: speculative again, measured again
    assert samrs.recompute_count(clear=True) == recomputed
    assert samrs.global_policy(td) == (share, True)
    # ordinary data (N(0,1) activations, N(0, 0.5) table) on its own table: measured, kept speculative
    q, kt, v, t = make_inputs(h, w, 4, hd, seed=124, table_std=0.5)
    args = [to_dev(x, "bf16", cuda) for x in (q, kt, v, t)]
    samrs.attention_relpos(*args, h, w, scale)
    assert samrs.recompute_count(clear=True) == 0
    assert samrs.global_policy(args[3]) == (0.0, False)


def test_ex2_polynomial_against_cuda_exp2f(samrs, cuda):
    """The windowed kernel's own exp2 (range reduction to [-1/2, 1/2] by rounding, degree-4 polynomial fitted
    to relative error, exponent-field insertion) against CUDA's exp2f: relative error <= 3e-6 on [-120, 127];
    below -120 the argument is clamped, so the result is 2^-120 (within the same relative error)."""
    x = torch.cat([torch.linspace(-120.0, 127.0, 1 << 20, device=cuda),
                   torch.rand(1 << 20, device=cuda) * 247.0 - 120.0,
                   torch.arange(-120, 128, device=cuda, dtype=torch.float32),
                   torch.arange(-120, 127, device=cuda, dtype=torch.float32) + 0.5]).contiguous()
    yp, yl = torch.empty_like(x), torch.empty_like(x)
    lib = samrs._abi.lib()
    samrs._abi.check(lib.samrs_selftest_ex2(x.data_ptr(), yp.data_ptr(), yl.data_ptr(), x.numel(),
                                            torch.cuda.current_stream().cuda_stream))
    xd = x.double().cpu().numpy()
    lib_rel = np.abs(yl.double().cpu().numpy() / np.exp2(xd) - 1).max()
    assert lib_rel < 1e-6, lib_rel  # exp2f itself is within a couple of f32 ulps
    rel = np.abs(yp.double().cpu().numpy() / yl.double().cpu().numpy() - 1).max()
    assert rel <= 3e-6, rel
    lo = torch.tensor([-121.0, -126.5, -150.0, -1e30], device=cuda)
    ylo, ylo2 = torch.empty_like(lo), torch.empty_like(lo)
    samrs._abi.check(lib.samrs_selftest_ex2(lo.data_ptr(), ylo.data_ptr(), ylo2.data_ptr(), lo.numel(),
                                            torch.cuda.current_stream().cuda_stream))
    assert np.abs(ylo.double().cpu().numpy() / 2.0 ** -120 - 1).max() <= 3e-6


def test_tc_and_simt_agree_bf16(samrs, cuda):
    for (h, w, bh, hd) in [(64, 64, 2, 80), (14, 14, 40, 80)]:
        q, kt, v, t = make_inputs(h, w, bh, hd, seed=99)
        args = [to_dev(x, "bf16", cuda) for x in (q, kt, v, t)]
        a = samrs.attention_relpos(*args, h, w, 0.125, impl="auto").float()
        b = samrs.attention_relpos(*args, h, w, 0.125, impl="simt").float()
        assert (a - b).abs().max().item() / b.abs().max().item() < 2 * HALF_TOL


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("h,w,bh,hd", [(14, 14, 6, 64), (64, 64, 2, 64), (7, 11, 3, 80)])
def test_relpos_softmax_kat(samrs, cuda, h, w, bh, hd, dt):
    # tests/kernels.rs:19-37: probs agree with the CPU op within 1e-3 absolute on 16-bit-rounded inputs
    n = h * w
    rng = np.random.default_rng(n + bh)
    s = rng.standard_normal((bh, n, n), dtype=np.float32)
    q = rng.standard_normal((bh, n, hd), dtype=np.float32)
    t = rng.standard_normal((2 * h - 1 + 2 * w - 1, hd), dtype=np.float32)
    sd, qd, td = (to_dev(x, dt, cuda) for x in (s, q, t))
    got = samrs.relpos_softmax(sd, qd, td, h, w, 0.125).float().cpu().numpy()
    want = oracle.relpos_softmax(rounded(sd), rounded(qd), rounded(td), h, w, 0.125)
    if dt == "bf16":
        # bf16 rounding of a probability near 1 alone is 2^-9 ~ 2e-3: bound what lies beyond half an ulp
        assert excess_err(got, want, "bf16") * np.abs(want).max() < 1e-3
    else:
        assert np.abs(got - want).max() < (1e-5 if dt == "f32" else 1e-3)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_qkv_split_matches_oracle(samrs, cuda, dt):
    n, nh, hd, win = 196, 12, 64, 3
    rng = np.random.default_rng(11)
    y = rng.standard_normal((win * n, 3 * nh * hd), dtype=np.float32)
    b = rng.standard_normal(3 * nh * hd, dtype=np.float32)
    yd, bd = to_dev(y, dt, cuda), to_dev(b, dt, cuda)
    got = samrs.qkv_split(yd, bd, n, nh, hd)
    want = oracle.qkv_split(rounded(yd), rounded(bd), n, nh, hd)
    for g_, w_ in zip(got, want):
        ref = torch.from_numpy(w_).to(DT[dt]).float().numpy()  # the sum rounds once to the I/O dtype
        assert np.array_equal(g_.float().cpu().numpy(), ref)


def test_attention_block_chain(samrs, cuda):
    """Attention::forward (src/sam1/encoder.rs:73-85) on a windowed ViT-B block: qkv GEMM -> qkv_split ->
    fused attention -> proj, against the same chain with the oracle for the attention."""
    torch.manual_seed(3)
    c, nh = 768, 12
    x = torch.randn(1, 64, 64, c, device=cuda)
    parts, hp, wp = samrs.window_partition(x, 14)
    assert parts.shape == (25, 14, 14, c) and hp == wp == 70
    back = samrs.window_unpartition(parts, 14, hp, wp, (64, 64), 1, c)
    assert torch.equal(back, x)
    att = samrs.Attention(torch.randn(3 * c, c, device=cuda) * 0.02, torch.randn(3 * c, device=cuda) * 0.02,
                          torch.randn(c, c, device=cuda) * 0.02, torch.zeros(c, device=cuda),
                          torch.randn(27, 64, device=cuda) * 0.5, torch.randn(27, 64, device=cuda) * 0.5, nh)
    y = att.forward(parts)
    assert y.shape == parts.shape
    qkv = (parts.reshape(-1, c) @ att.qkv_wt).cpu().numpy()
    q, kt, v = oracle.qkv_split(qkv, att.qkv_b.cpu().numpy(), 196, nh, 64)
    ctx = oracle.attention_relpos(q, kt, v, att.rel.cpu().numpy(), 14, 14, 64 ** -0.5)
    ref = torch.from_numpy(ctx).reshape(25, nh, 196, 64).permute(0, 2, 1, 3).reshape(-1, c) @ att.proj_wt.cpu()
    assert rel_max_err(y.reshape(-1, c).cpu().numpy(), ref.numpy()) < 1e-3


# ViT-H / ViT-B windowed (TMA path), pads along both axes with an odd window token count (vectorised
# path), global (one window), exact fit (TMA), ragged on both axes (TMA: zero-filled loads, clipped
# stores), hd 12 (scalar path in 16-bit, TMA in f32)
WIN_GEOMS = [(2, 64, 64, 14, 16, 80), (1, 64, 64, 14, 12, 64), (2, 13, 20, 7, 3, 24), (1, 16, 16, 0, 4, 32),
             (1, 14, 14, 14, 2, 16), (2, 30, 20, 8, 4, 32), (1, 9, 11, 4, 2, 12)]


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("images,h,w,ws,nh,hd", WIN_GEOMS)
def test_qkv_split_window_matches_oracle(samrs, cuda, images, h, w, ws, nh, hd, dt):
    """window_partition (zero pad) + qkv bias + qkv_split in one kernel, bit-exact against the oracle's
    restatement of the reference order (src/sam1/encoder.rs:132-140, src/kernels.rs:234-263)."""
    rng = np.random.default_rng(h * 31 + w + hd)
    c = nh * hd
    y = rng.standard_normal((images * h * w, 3 * c), dtype=np.float32)
    b = rng.standard_normal(3 * c, dtype=np.float32)
    yd, bd = to_dev(y, dt, cuda), to_dev(b, dt, cuda)
    got = samrs.qkv_split_window(yd, bd, images, h, w, ws, nh, hd)
    want = oracle.qkv_split_window(rounded(yd), rounded(bd), images, h, w, ws, nh, hd)
    for g_, w_ in zip(got, want):
        ref = torch.from_numpy(np.ascontiguousarray(w_)).to(DT[dt]).float().numpy()  # one rounding of the sum
        assert g_.shape == w_.shape
        assert np.array_equal(g_.float().cpu().numpy(), ref)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("images,h,w,ws,nh,hd", WIN_GEOMS)
def test_window_merge_matches_oracle(samrs, cuda, images, h, w, ws, nh, hd, dt):
    """Heads back to tokens + window_unpartition crop (src/sam1/encoder.rs:82,142-145), bit-exact."""
    wh, ww = (ws, ws) if ws else (h, w)
    bh = images * (-(-h // wh)) * (-(-w // ww)) * nh
    a = np.random.default_rng(h + w).standard_normal((bh, wh * ww, hd), dtype=np.float32)
    ad = to_dev(a, dt, cuda)
    got = samrs.window_merge(ad, images, h, w, ws, nh, hd)
    want = oracle.window_merge(rounded(ad), images, h, w, ws, nh, hd)
    assert np.array_equal(got.float().cpu().numpy(), want)


def test_windowed_block_fused_io_chain(samrs, cuda):
    """The windowed ViT-B block on the real tokens only: qkv GEMM on the 64x64 grid -> qkv_split_window ->
    fused attention -> window_merge -> proj, against the reference order (window_partition with zero pad ->
    qkv GEMM on all 70x70 tokens -> qkv_split -> attention -> proj -> window_unpartition) with the oracle
    for the attention."""
    torch.manual_seed(5)
    c, nh, hd = 768, 12, 64
    x = torch.randn(1, 64, 64, c, device=cuda)
    att = samrs.Attention(torch.randn(3 * c, c, device=cuda) * 0.02, torch.randn(3 * c, device=cuda) * 0.02,
                          torch.randn(c, c, device=cuda) * 0.02, torch.zeros(c, device=cuda),
                          torch.randn(27, 64, device=cuda) * 0.5, torch.randn(27, 64, device=cuda) * 0.5, nh)
    y = (x.reshape(-1, c) @ att.qkv_wt).contiguous()
    q, kt, v = samrs.qkv_split_window(y, att.qkv_b, 1, 64, 64, 14, nh, hd)
    ctx = samrs.attention_relpos(q, kt, v, att.rel, 14, 14, att.scale)
    got = samrs.window_merge(ctx, 1, 64, 64, 14, nh, hd) @ att.proj_wt
    parts = oracle.window_partition(x.cpu().numpy(), 14)
    qkv = parts.reshape(-1, c) @ att.qkv_wt.cpu().numpy()
    q2, kt2, v2 = oracle.qkv_split(qkv, att.qkv_b.cpu().numpy(), 196, nh, hd)
    ctx2 = oracle.attention_relpos(q2, kt2, v2, att.rel.cpu().numpy(), 14, 14, hd ** -0.5)
    tok = ctx2.reshape(25, nh, 196, hd).transpose(0, 2, 1, 3).reshape(-1, c) @ att.proj_wt.cpu().numpy()
    ref = oracle.window_unpartition(tok.reshape(25, 14, 14, c), 14, 64, 64).reshape(-1, c)
    assert rel_max_err(got.cpu().numpy(), ref) < 1e-3


def test_empty_and_status(samrs, cuda):
    q = torch.zeros(0, 16, 8, device=cuda)
    out = samrs.attention_relpos(q, torch.zeros(0, 8, 16, device=cuda), q, torch.zeros(14, 8, device=cuda), 4, 4, 1.0)
    assert out.shape == (0, 16, 8)
    assert samrs.device_status() == 0


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("h,hd", [(14, 64), (64, 80)])
def test_misaligned_buffers_fall_back_to_simt(samrs, cuda, h, hd, dt):
    """q, kt, v and out one element into larger buffers (not 16-byte aligned): the tensor-core kernels need
    16-byte alignment, so the default path takes the SIMT kernel (and matches the oracle), while forcing
    the tensor-core path is refused with SAMRS_ERR_UNSUPPORTED."""
    bh = 3
    q, kt, v, t = make_inputs(h, h, bh, hd, seed=h + hd, table_std=0.5)

    def offset_view(a):
        flat = torch.zeros(a.size + 1, dtype=DT[dt], device=cuda)
        flat[1:] = torch.from_numpy(np.ascontiguousarray(a)).reshape(-1).to(cuda).to(DT[dt])
        return flat[1:].view(a.shape)

    qd, ktd, vd = offset_view(q), offset_view(kt), offset_view(v)
    td = to_dev(t, dt, cuda)
    out = offset_view(np.zeros_like(q))
    assert qd.data_ptr() % 16 != 0
    scale = hd ** -0.5
    samrs.attention_relpos(qd, ktd, vd, td, h, h, scale, out=out)
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(rounded(qd), rounded(ktd), rounded(vd), rounded(td), h, h, scale)
    assert parity_err(out.float().cpu().numpy(), ref, dt) < tol(dt)
    with pytest.raises(samrs.SamrsError) as e:
        samrs.attention_relpos(qd, ktd, vd, td, h, h, scale, impl="tc", out=out)
    assert e.value.code == samrs._abi.ERR_UNSUPPORTED
