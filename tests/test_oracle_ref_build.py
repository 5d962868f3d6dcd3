"""The build recipe of the reference's own CUDA kernels (oracle/build_ref_cuda.py), on the CPU: it compiles the
reference's kernels/sam.cu where it lies when that tree is present, and builds nothing otherwise."""
import os

from oracle import build_ref_cuda


def test_ref_cuda_recipe_without_reference_tree(monkeypatch, tmp_path):
    monkeypatch.setattr(build_ref_cuda, "SRC", str(tmp_path / "absent" / "sam.cu"))
    monkeypatch.setattr(build_ref_cuda, "OUT", str(tmp_path / "_ref" / "sam.cubin"))
    assert build_ref_cuda.build(force=True) is None
    assert not os.path.exists(tmp_path / "_ref")


def test_ref_cuda_recipe_builds_when_reference_present():
    if not os.path.exists(build_ref_cuda.SRC):
        return  # the GPU box: only the prebuilt cubin travels
    out = build_ref_cuda.build()
    assert out == build_ref_cuda.OUT and os.path.getsize(out) > 0
    assert os.path.dirname(out).endswith(os.path.join("oracle", "_ref"))
