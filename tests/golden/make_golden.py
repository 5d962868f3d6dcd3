"""Generate the golden fixtures in this directory.

The reference (apiplant/sam-rs) ships no golden vectors for this path and cannot be built here (Rust),
so the fixtures come from an independent float64 restatement of the reference's *tensor-op fallback*
(src/kernels.rs:20-42: index_select of the rel-pos tables, two batched matmuls for rel_h / rel_w, a
5-D broadcast add onto scale*scores, softmax over the last dim), followed by the PV product of
src/sam1/encoder.rs:81. It shares no code with oracle/relpos_oracle.c (which restates the tiled CPU
op, src/kernels.rs:131-225), so agreement between the two pins the oracle.

Inputs: numpy PCG64 (default_rng(seed)) standard normals, rounded to float16 precision as the
reference's own KAT does (tests/kernels.rs:28-31), so the same fixture serves the f32, f16 and bf16
checks (f16-representable values are not all bf16-representable; bf16 tests round again and use the
oracle, not these fixtures). Geometries are the reference's KAT geometries (tests/kernels.rs:23,
tests/cpu_gemm.rs:35) at scale 0.125, plus one ViT-H windowed slice (hd 80).

    python tests/golden/make_golden.py   (rewrites golden_*.npz)
"""
import hashlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, h, w, bh, hd, seed, row_stride): row_stride subsamples stored output rows for big cases
CASES = [
    ("kat_14x14_bh6_hd64", 14, 14, 6, 64, 1401, 1),
    ("kat_64x64_bh2_hd64", 64, 64, 2, 64, 6402, 16),
    ("kat_7x11_bh3_hd80", 7, 11, 3, 80, 711, 1),
    ("vith_14x14_bh4_hd80", 14, 14, 4, 80, 1480, 1),
]
SCALE = 0.125


def f16_round(x):
    return x.astype(np.float16).astype(np.float32)


def make_inputs(h, w, bh, hd, seed):
    """Seeded inputs in the reference layouts: s [bh,n,n] raw scores for the softmax KAT,
    q [bh,n,hd], kt [bh,hd,n], v [bh,n,hd], table [(2h-1)+(2w-1), hd]."""
    n = h * w
    rng = np.random.default_rng(seed)
    q = f16_round(rng.standard_normal((bh, n, hd), dtype=np.float32))
    kt = f16_round(rng.standard_normal((bh, hd, n), dtype=np.float32))
    v = f16_round(rng.standard_normal((bh, n, hd), dtype=np.float32))
    table = f16_round(rng.standard_normal(((2 * h - 1) + (2 * w - 1), hd), dtype=np.float32))
    return q, kt, v, table


def tensor_fallback_probs(scores, q, table, h, w, scale):
    """float64 restatement of src/kernels.rs:20-42. scores [bh, n, n] -> probs [bh, n, n]."""
    scores = scores.astype(np.float64)
    q = q.astype(np.float64)
    table = table.astype(np.float64)
    bh, n, hd = q.shape

    def idx(size):
        qi = np.arange(size)[:, None]
        ki = np.arange(size)[None, :]
        return (qi + size - 1 - ki).reshape(-1)

    th = table[: 2 * h - 1]
    tw = table[2 * h - 1: 2 * h - 1 + 2 * w - 1]
    rh = th[idx(h)].reshape(h, h, hd)  # rh[i, kh] = Th[i + h - 1 - kh]
    rw = tw[idx(w)].reshape(w, w, hd)  # rw[j, kw] = Tw[j + w - 1 - kw]
    rq = q.reshape(bh, h, w, hd)
    rel_h = np.einsum("bijd,ikd->bijk", rq, rh)  # [bh, h, w, kh]
    rel_w = np.einsum("bijd,jkd->bijk", rq, rw)  # [bh, h, w, kw]
    a = (scores * scale).reshape(bh, h, w, h, w)
    a = a + rel_h[:, :, :, :, None] + rel_w[:, :, :, None, :]
    a = a.reshape(bh, n, n)
    a = a - a.max(axis=-1, keepdims=True)
    e = np.exp(a)
    return e / e.sum(axis=-1, keepdims=True)


def reference_attention(q, kt, v, table, h, w, scale):
    """bmm(relpos_softmax(bmm(q, kt)), v) in float64 (src/sam1/encoder.rs:81)."""
    s = np.matmul(q.astype(np.float64), kt.astype(np.float64))
    p = tensor_fallback_probs(s, q, table, h, w, scale)
    return np.matmul(p, v.astype(np.float64)), s, p


def digest(*arrays):
    hs = hashlib.sha256()
    for a in arrays:
        hs.update(np.ascontiguousarray(a).tobytes())
    return hs.hexdigest()


def main():
    for name, h, w, bh, hd, seed, stride in CASES:
        q, kt, v, table = make_inputs(h, w, bh, hd, seed)
        out, s, p = reference_attention(q, kt, v, table, h, w, SCALE)
        rows = np.arange(0, h * w, stride)
        prow = rows[:: max(1, len(rows) // 16)][:16]  # stored probability rows
        # softmax KAT: raw scores are themselves f16-rounded inputs in tests/kernels.rs:24-31
        s16 = f16_round(s.astype(np.float32))
        p16 = tensor_fallback_probs(s16, q, table, h, w, SCALE)
        np.savez_compressed(
            os.path.join(HERE, f"golden_{name}.npz"),
            h=h, w=w, bh=bh, hd=hd, seed=seed, scale=SCALE, rows=rows,
            input_sha256=digest(q, kt, v, table),
            out_rows=out[:, rows, :].astype(np.float32),
            probs_rows=p16[:, prow, :].astype(np.float32),
            probs_row_ids=prow,
        )
        print(name, out.shape, "max|out|", float(np.abs(out).max()))


if __name__ == "__main__":
    main()
