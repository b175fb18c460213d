"""A bounded device wait that runs out, on the GPU, without faulting it.

The streamed prefill's chain CTAs wait (bounded) on per-record ready flags that
prep workers in the same launch set.  gdn_test_prefill_hooks lowers the wait
budget and makes the prep workers leave one record unpublished: the chain CTA
of that sequence gives up, every role of it drains (its copies land, its MMAs
complete) and returns, the launch completes, gdn_check_device_error reports the
timeout, and the next prefill on the same device is correct again.  Nothing
here traps, faults or spins without a limit."""
import math
import time

import numpy as np
import pytest

from oracle import gdn_oracle as O
from tests._util import max_abs, to_dev, to_np

pytestmark = pytest.mark.gpu


def test_prefill_record_wait_times_out_and_recovers(cuda_device):
    import torch
    from gdn_18646_b200 import _lib, ops
    B, T, H, dk, dv = 1, 1024, 4, 128, 128            # 4 chains, 16 chunks: the streamed schedule
    inp = O.make_prefill_inputs(91, B, T, H, dk, dv, state_std=0.02)
    q, k, v, a, b = (to_dev(inp[x]) for x in ("q", "k", "v", "a", "b"))
    A_log, s0 = to_dev(inp["A_log"]), to_dev(inp["state_in"])
    lib = _lib.lib()

    def run():
        return ops.prefill(q, k, v, A_log, a, b, state_in=s0, scale=inp["scale"], schedule="stream")

    run()
    torch.cuda.synchronize()
    assert lib.gdn_check_device_error() == _lib.GDN_OK
    nchunks = T // 64
    try:
        # ~1 ms budget; sequence (b=0, h=1) waits for its chunk 7 forever otherwise
        _lib.call("gdn_test_prefill_hooks", 2_000_000, 1 * nchunks + 7)
        t0 = time.perf_counter()
        run()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        status = lib.gdn_check_device_error()
    finally:
        _lib.call("gdn_test_prefill_hooks", 0, -1)
    assert status == _lib.GDN_ERR_DEVICE_TIMEOUT
    assert elapsed < 1.0, f"the timed-out launch took {elapsed:.3f} s"
    # the device and the library are usable at once: the same call is correct again
    o, S = run()
    torch.cuda.synchronize()
    assert lib.gdn_check_device_error() == _lib.GDN_OK
    o_r, S_r = O.prefill(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["mask"],
                         state_in=inp["state_in"], scale=inp["scale"], chunk_size=64, dt=np.float64)
    assert max_abs(to_np(o), o_r) <= 2e-2
    assert O.rel_fro(to_np(S), S_r) <= 1e-3
