"""Failure detection on the GPU without a fault: a bounded wait that runs out.

With the test hooks set (every wait bounded at ~0.1 ms, and CTA 0 of the global-layer kernel never issuing the
load of one key tile), the MMA issuer's wait for that tile runs out: the kernel records code 1 in the device
status word and every CTA returns, draining its own copies and freeing TMEM (nothing traps, faults or hangs).
The host then sees the status, every entry point refuses with SAMRS_ERR_DEVICE until the word is cleared, and
the next normal call matches the oracle."""
import time

import numpy as np
import pytest

from oracle import oracle
from tests.helpers import HALF_TOL, make_inputs, parity_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_bounded_wait_runs_out_and_the_library_recovers(samrs, cuda, dt):
    lib = samrs._abi.lib()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    q, kt, v, t = make_inputs(64, 64, 4, 80, seed=17, table_std=0.5)
    args = [torch.from_numpy(x).to(cuda).to(tdt) for x in (q, kt, v, t)]
    scale = 80 ** -0.5
    assert samrs.device_status() == 0
    try:
        samrs._abi.check(lib.samrs_test_hooks(200_000, 5))  # ~0.1 ms per wait; CTA 0 never loads key tile 5
        t0 = time.perf_counter()
        samrs.attention_relpos(*args, 64, 64, scale)
        status = samrs.device_status(clear=False)  # synchronises: the kernel returned
        elapsed = time.perf_counter() - t0
    finally:
        samrs._abi.check(lib.samrs_test_hooks(0, -1))
    assert status == 1, status  # kStatusWaitTimeout
    assert elapsed < 5.0, elapsed
    # the word has been seen and not cleared: every entry point refuses instead of launching a no-op
    with pytest.raises(samrs.SamrsError) as err:
        samrs.attention_relpos(*args, 64, 64, scale)
    assert err.value.code == samrs._abi.ERR_DEVICE
    assert samrs.device_status(clear=True) == 1
    assert samrs.device_status() == 0
    out = samrs.attention_relpos(*args, 64, 64, scale)
    assert samrs.device_status() == 0
    ref = oracle.attention_relpos(*(a.float().cpu().numpy() for a in args), 64, 64, scale)
    assert parity_err(out.float().cpu().numpy(), ref, dt) < HALF_TOL
