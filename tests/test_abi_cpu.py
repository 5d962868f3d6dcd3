"""The C-ABI library loads, exports every symbol that include/samrs_b200.h declares, and rejects bad
arguments before touching a device (no compute call runs here)."""
import ctypes

import pytest

from tests.conftest import load_samrs


def abi():
    return load_samrs()._abi


def test_library_exports_every_header_symbol():
    a = abi()
    names = a.header_symbols()
    assert set(names) >= {"samrs_relpos_attn_fwd", "samrs_relpos_attn_fwd_ex", "samrs_relpos_softmax_fwd",
                          "samrs_qkv_split_fwd", "samrs_qkv_split_window_fwd", "samrs_window_merge_fwd",
                          "samrs_last_error", "samrs_abi_version", "samrs_device_status",
                          "samrs_recompute_count", "samrs_selftest_ex2", "samrs_linear_fwd",
                          "samrs_qkv_linear_window_fwd", "samrs_layer_norm_fwd", "samrs_test_hooks",
                          "samrs_global_policy"}
    lib = ctypes.CDLL(a.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version():
    assert abi().lib().samrs_abi_version() == 1


@pytest.mark.parametrize("args,code", [
    (dict(dtype=7), -1),                 # unknown dtype
    (dict(bh=-1), -1),                   # negative batch
    (dict(h=0), -2), (dict(w=129), -2),  # grid outside 1..128
    (dict(hd=0), -2), (dict(hd=129), -2),
    (dict(impl=9), -1),
])
def test_attention_rejects_bad_arguments(args, code):
    a = abi()
    p = dict(bh=1, h=4, w=4, hd=8, dtype=0, impl=0)
    p.update(args)
    rc = a.lib().samrs_relpos_attn_fwd_ex(0, 0, 0, 0, 0, p["bh"], p["h"], p["w"], p["hd"], 0.5, p["dtype"], p["impl"],
                                          None)
    assert rc == code
    assert a.lib().samrs_last_error()


def test_null_pointers_rejected():
    a = abi()
    assert a.lib().samrs_relpos_attn_fwd(0, 0, 0, 0, 0, 1, 4, 4, 8, 0.5, 0, None) == -1
    assert a.lib().samrs_recompute_count(None, None, 0) == -1
    assert a.lib().samrs_global_policy(None, None, None, 0) == -1
    assert a.lib().samrs_selftest_ex2(0, 0, 0, 4, None) == -1
    assert a.lib().samrs_selftest_ex2(0, 0, 0, -1, None) == -1
    assert a.lib().samrs_selftest_ex2(0, 0, 0, 0, None) == 0


def test_empty_batch_is_noop():
    a = abi()
    assert a.lib().samrs_relpos_attn_fwd(0, 0, 0, 0, 0, 0, 4, 4, 8, 0.5, 2, None) == 0
    assert a.lib().samrs_relpos_softmax_fwd(0, 0, 0, 0, 0, 4, 4, 8, 0.5, 1, None) == 0


def test_softmax_rows_must_be_multiple_of_n():
    a = abi()
    assert a.lib().samrs_relpos_softmax_fwd(0, 0, 0, 0, 17, 4, 4, 8, 0.5, 0, None) == -1


def test_qkv_split_rejects_ragged_tokens():
    a = abi()
    assert a.lib().samrs_qkv_split_fwd(0, 0, 0, 197, 196, 12, 64, 0, None) == -1


def test_host_mirror_rejects_cpu_tensors():
    import torch
    s = load_samrs()
    q = torch.zeros(1, 16, 8)
    kt = torch.zeros(1, 8, 16)
    t = torch.zeros(14, 8)
    with pytest.raises(s.SamrsError):
        s.attention_relpos(q, kt, q, t, 4, 4, 0.5)
    assert s.attention_relpos_cpu(q, kt, q, t, 4, 4, 0.5) is None


@pytest.mark.parametrize("args", [dict(dtype=5), dict(images=-1), dict(h=0), dict(ws=-1), dict(nh=0), dict(hd=0)])
def test_window_io_rejects_bad_arguments(args):
    a = abi()
    p = dict(images=1, h=8, w=8, ws=4, nh=2, hd=8, dtype=2)
    p.update(args)
    rc = a.lib().samrs_qkv_split_window_fwd(0, 0, 0, p["images"], p["h"], p["w"], p["ws"], p["nh"], p["hd"],
                                            p["dtype"], None)
    assert rc == -1 and a.lib().samrs_last_error()
    rc = a.lib().samrs_window_merge_fwd(0, 0, p["images"], p["h"], p["w"], p["ws"], p["nh"], p["hd"], p["dtype"], None)
    assert rc == -1 and a.lib().samrs_last_error()


def test_window_io_empty_and_null():
    a = abi()
    assert a.lib().samrs_qkv_split_window_fwd(0, 0, 0, 0, 64, 64, 14, 16, 80, 2, None) == 0
    assert a.lib().samrs_window_merge_fwd(0, 0, 0, 64, 64, 14, 16, 80, 2, None) == 0
    assert a.lib().samrs_qkv_split_window_fwd(0, 0, 0, 1, 64, 64, 14, 16, 80, 2, None) == -1
    assert a.lib().samrs_window_merge_fwd(0, 0, 1, 64, 64, 14, 16, 80, 2, None) == -1


@pytest.mark.parametrize("args,code", [
    (dict(dtype=0), -2),                  # f32: no tensor-core GEMM
    (dict(k=100), -2), (dict(n=40), -2),  # k % 8, n % 16
    (dict(m=-1), -1), (dict(n=0), -1),
    (dict(epi=7), -1),
])
def test_linear_rejects_bad_arguments(args, code):
    a = abi()
    p = dict(m=4, n=32, k=64, epi=0, dtype=2)
    p.update(args)
    rc = a.lib().samrs_linear_fwd(0, 0, 0, 0, 0, p["m"], p["n"], p["k"], p["epi"], p["dtype"], None)
    assert rc == code and a.lib().samrs_last_error()


def test_linear_and_norm_empty_and_null():
    a = abi()
    assert a.lib().samrs_linear_fwd(0, 0, 0, 0, 0, 0, 32, 64, 1, 2, None) == 0
    assert a.lib().samrs_linear_fwd(0, 0, 0, 0, 0, 4, 32, 64, 0, 2, None) == -1
    assert a.lib().samrs_layer_norm_fwd(0, 0, 0, 0, 0, 768, 1e-6, 1, None) == 0
    assert a.lib().samrs_layer_norm_fwd(0, 0, 0, 0, 3, 768, 1e-6, 1, None) == -1
    assert a.lib().samrs_layer_norm_fwd(0, 0, 0, 0, 3, 768, -1.0, 1, None) == -1
    assert a.lib().samrs_qkv_linear_window_fwd(0, 0, 0, 0, 0, 64, 64, 14, 12, 64, 1, None) == 0
    assert a.lib().samrs_qkv_linear_window_fwd(0, 0, 0, 0, 1, 64, 64, 14, 12, 12, 1, None) == -2  # hd % 16
    assert a.lib().samrs_qkv_linear_window_fwd(0, 0, 0, 0, 1, 64, 64, 14, 12, 64, 1, None) == -1  # null


def test_header_compiles_as_c_and_links(tmp_path):
    """include/samrs_b200.h is a C header (what the reference's Rust FFI, or any C caller, binds): a C99 program
    that includes it compiles with gcc, links against the library and gets the error codes and messages of the
    argument checks (no GPU needed for those)."""
    import os
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    lib_dir = os.path.join(root, "sam-rs_b200")
    src = tmp_path / "probe.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "samrs_b200.h"
int main(void) {
  if (samrs_abi_version() != SAMRS_ABI_VERSION) return 1;
  int rc = samrs_relpos_attn_fwd(0, 0, 0, 0, 0, 1, 4, 4, 8, 0.5f, 7, 0);
  if (rc != SAMRS_ERR_INVALID || strlen(samrs_last_error()) == 0) return 2;
  rc = samrs_relpos_attn_fwd_ex(0, 0, 0, 0, 0, 1, 0, 4, 8, 0.5f, SAMRS_F32, SAMRS_IMPL_AUTO, 0);
  if (rc != SAMRS_ERR_UNSUPPORTED) return 3;
  rc = samrs_linear_fwd(0, 0, 0, 0, 0, 4, 16, 8, 9, SAMRS_BF16, 0);
  if (rc != SAMRS_ERR_INVALID) return 4;
  printf("%s\n", samrs_last_error());
  return 0;
}
''')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(root, "include"), str(src), "-o", str(exe),
                    "-L", lib_dir, "-lsamrs_b200", f"-Wl,-rpath,{lib_dir}"], check=True, timeout=120)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert "epilogue" in r.stdout
