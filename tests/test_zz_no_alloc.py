"""gdn_prefill_fwd_noalloc, the prefill for callers that cannot allocate device
memory while they run (an engine that reserved the GPU's memory for its own
pools, a plugin whose host forbids allocation at execute time).  Its workspace
is a static 32 MiB device array inside the library.

CPU: a problem whose workspace exceeds the array is rejected with a clear error
before any device access.  GPU: two calls in a row (the second runs over the
first one's leftovers in the shared array), under every launch schedule, each
match gdn_prefill_fwd_ws within the prefill tolerance of the other tests, and
the oracle bar; a ragged problem after a larger one matches the workspace
entry point on a 0xFF-filled workspace; and a call allocates nothing (the
default memory pool's high-water mark stays at zero, while gdn_prefill_fwd on
the same problem raises it, and the device's free memory is unchanged).

This file is named to be collected last.
"""
import numpy as np
import pytest

from gdn_18646_b200 import _lib
from oracle import gdn_oracle as O

FAKE = 0x10000
O_TOL = 2e-2          # bf16 output max-abs, as in test_prefill_gpu.py
S_TOL = 1e-3          # fp32 state relative Frobenius, as in test_prefill_gpu.py


@pytest.fixture(scope="module")
def lib():
    return _lib.lib()


def _args(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, A_log=FAKE, a=FAKE, b=FAKE, gate=0, dtb=0.0, dtv=None, mask=None,
             s_in=None, out=FAKE, s_out=FAKE, B=4, T=4096, Hqk=16, Hv=16, dk=128, dv=128, layout=0, scale=0.0,
             stream=None)
    a.update(over)
    return list(a.values())


def test_noalloc_rejects_problems_beyond_the_static_scratch(lib):
    need = lib.gdn_prefill_workspace_bytes(4, 4096, 16, 128, 128)
    assert need > 32 << 20
    assert _lib.call_status("gdn_prefill_fwd_noalloc", *_args()) == _lib.GDN_ERR_UNSUPPORTED
    assert "static scratch" in _lib.last_error()
    assert _lib.call_status("gdn_prefill_fwd_noalloc", *_args(q=None)) == _lib.GDN_ERR_NULL


def _inputs(B, T, H, dk, dv, seed):
    return O.make_prefill_inputs(seed, B, T, H, dk, dv, state_std=0.02)


def _device(inp):
    """The call's device tensors, outputs NaN-poisoned (every element must be written)."""
    import torch
    from tests._util import to_dev
    t = dict(q=to_dev(inp["q"]), k=to_dev(inp["k"]), v=to_dev(inp["v"]), a=to_dev(inp["a"]), b=to_dev(inp["b"]),
             A_log=to_dev(inp["A_log"]), s_in=to_dev(np.asarray(inp["state_in"], np.float32)))
    B, H, T, dk = t["q"].shape
    t["out"] = torch.full_like(t["v"], float("nan"))
    t["s_out"] = torch.full((B, H, dk, t["v"].shape[-1]), float("nan"), dtype=torch.float32, device="cuda")
    return t


def _launch(name, inp, t, ws=None):
    """One prefill through the C ABI on prepared device tensors (no allocation here)."""
    import torch
    B, H, T, dk = t["q"].shape
    dv = t["v"].shape[-1]
    stream = torch.cuda.current_stream().cuda_stream
    common = [t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["A_log"].data_ptr(), t["a"].data_ptr(),
              t["b"].data_ptr(), 0, float(inp["dt_bias"]), None, None, t["s_in"].data_ptr(), t["out"].data_ptr(),
              t["s_out"].data_ptr(), B, T, H, H, dk, dv, 0, float(inp["scale"])]
    if name == "gdn_prefill_fwd_ws":
        _lib.call(name, *common, ws.data_ptr(), ws.numel(), stream)
    else:
        _lib.call(name, *common, stream)
    torch.cuda.synchronize()
    return t["out"], t["s_out"]


def _call(name, inp, ws=None):
    """One prefill through the C ABI on fresh device tensors; returns (o bf16, final state fp32)."""
    return _launch(name, inp, _device(inp), ws)


def _close(o, s, o_ref, s_ref):
    import torch
    assert torch.isfinite(o.float()).all() and torch.isfinite(s).all()
    err_o = float((o.float() - o_ref.float()).abs().max())
    err_s = float(torch.linalg.vector_norm(s - s_ref) / torch.linalg.vector_norm(s_ref))
    assert err_o <= O_TOL, f"o max-abs {err_o:.3e}"
    assert err_s <= S_TOL, f"state rel-Frobenius {err_s:.3e}"


def _pool_high_water(reset=False):
    from cuda.bindings import driver as drv
    from cuda.bindings import runtime as rt
    import torch
    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    attr = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    if reset:
        err, = rt.cudaMemPoolSetAttribute(pool, attr, drv.cuuint64_t(0))
        assert err == rt.cudaError_t.cudaSuccess
    err, val = rt.cudaMemPoolGetAttribute(pool, attr)
    assert err == rt.cudaError_t.cudaSuccess
    return int(val)


def _check_oracle(inp, o, s):
    from tests._util import to_np
    o_r, s_r = O.prefill(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                         inp["mask"], state_in=inp["state_in"], scale=float(inp["scale"]), chunk_size=64,
                         dt=np.float64)
    assert float(np.abs(O.bf16_to_f32(to_np(o)) - o_r).max()) <= O_TOL
    assert O.rel_fro(to_np(s), s_r) <= S_TOL


_SCHEDULES = {"auto": 0, "single": 1, "pieced": 2, "stream": 3}   # GDN_SCHEDULE_*


@pytest.mark.gpu
@pytest.mark.parametrize("schedule", ["auto", "single", "pieced", "stream"])
@pytest.mark.parametrize("B,T,H,dk,dv", [(1, 256, 2, 64, 64), (1, 1000, 4, 128, 256), (2, 4096, 4, 128, 128)])
def test_noalloc_two_calls_match_workspace_entry_point(cuda_device, lib, B, T, H, dk, dv, schedule):
    """Each launch schedule runs over the previous call's leftovers in the shared
    array (the streamed one reads per-record ready flags that a previous call
    left set: the gate kernel clears them first)."""
    import torch
    ws = torch.empty(lib.gdn_prefill_workspace_bytes(B, T, H, dk, dv), dtype=torch.uint8, device="cuda")
    first = _inputs(B, T, H, dk, dv, 900 + T)
    second = _inputs(B, T, H, dk, dv, 901 + T)
    _lib.call("gdn_prefill_set_schedule", _SCHEDULES[schedule])     # this thread's default: noalloc uses it
    try:
        for inp in (first, second):                   # back to back: the array keeps the first call's records
            o1, s1 = _call("gdn_prefill_fwd_noalloc", inp)
            o2, s2 = _call("gdn_prefill_fwd_ws", inp, ws)
            _close(o1, s1, o2, s2)
            _check_oracle(inp, o1, s1)
    finally:
        _lib.call("gdn_prefill_set_schedule", _lib.GDN_SCHEDULE_AUTO)


@pytest.mark.gpu
def test_noalloc_ragged_after_a_larger_problem(cuda_device, lib):
    """A ragged problem (T = 1000: a partial last chunk, dv = 256) right after a
    larger one, with nothing cleared in between: no record row or flag the
    larger call left behind is read back.  The reference is gdn_prefill_fwd_ws on
    a workspace filled with 0xFF."""
    import torch
    big = _inputs(2, 4096, 4, 128, 128, 905)
    _call("gdn_prefill_fwd_noalloc", big)
    small = _inputs(1, 1000, 4, 128, 256, 906)
    o1, s1 = _call("gdn_prefill_fwd_noalloc", small)
    ws = torch.full((lib.gdn_prefill_workspace_bytes(1, 1000, 4, 128, 256),), 0xFF, dtype=torch.uint8, device="cuda")
    o2, s2 = _call("gdn_prefill_fwd_ws", small, ws)
    _close(o1, s1, o2, s2)
    _check_oracle(small, o1, s1)


@pytest.mark.gpu
def test_noalloc_allocates_nothing(cuda_device, lib):
    """Neither the stream-ordered pool (its high-water mark stays at zero) nor any
    other allocation (the device's free memory is unchanged across the call)."""
    import torch
    inp = _inputs(1, 1000, 4, 128, 128, 77)
    t = _device(inp)
    _launch("gdn_prefill_fwd_noalloc", inp, t)               # first call: module load and symbol look-up
    _pool_high_water(reset=True)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    _launch("gdn_prefill_fwd_noalloc", inp, t)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, f"free device memory changed by {free_before - free_after} B"
    assert _pool_high_water() == 0
    _call("gdn_prefill_fwd", inp)                            # control: the allocating entry point shows up
    assert _pool_high_water() >= lib.gdn_prefill_workspace_bytes(1, 1000, 4, 128, 128)
