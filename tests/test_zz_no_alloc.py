"""gdn_prefill_fwd_noalloc: the prefill with its workspace in the library's
static 32 MiB device array, for callers that cannot allocate device memory.

CPU: problems whose workspace exceeds the array are rejected before any
device access.  GPU: results equal gdn_prefill_fwd_ws bit for bit and meet the
oracle bar, and the call takes nothing from the stream-ordered allocator (the
default memory pool's high-water mark stays at zero, while gdn_prefill_fwd on
the same problem raises it).
"""
import numpy as np
import pytest

from gdn_18646_b200 import _lib
from oracle import gdn_oracle as O

FAKE = 0x10000


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


def _call(name, inp, ws=None):
    import torch
    from tests._util import to_dev
    q, k, v = to_dev(inp["q"]), to_dev(inp["k"]), to_dev(inp["v"])
    a, b = to_dev(inp["a"]), to_dev(inp["b"])
    A_log = to_dev(inp["A_log"])
    s_in = to_dev(np.asarray(inp["state_in"], np.float32))
    B, H, T, dk = q.shape
    dv = v.shape[-1]
    out = torch.full_like(v, float("nan"))
    s_out = torch.empty(B, H, dk, dv, dtype=torch.float32, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    common = [q.data_ptr(), k.data_ptr(), v.data_ptr(), A_log.data_ptr(), a.data_ptr(), b.data_ptr(), 0,
              float(inp["dt_bias"]), None, None, s_in.data_ptr(), out.data_ptr(), s_out.data_ptr(),
              B, T, H, H, dk, dv, 0, float(inp["scale"])]
    if name == "gdn_prefill_fwd_ws":
        _lib.call(name, *common, ws.data_ptr(), ws.numel(), stream)
    else:
        _lib.call(name, *common, stream)
    torch.cuda.synchronize()
    return out, s_out


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


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,dk,dv", [(1, 256, 2, 64, 64), (1, 1000, 4, 128, 256), (2, 4096, 4, 128, 128)])
def test_noalloc_matches_workspace_call_and_oracle(cuda_device, lib, B, T, H, dk, dv):
    import torch
    from tests._util import to_np
    inp = _inputs(B, T, H, dk, dv, 900 + T)
    o1, s1 = _call("gdn_prefill_fwd_noalloc", inp)
    ws = torch.empty(lib.gdn_prefill_workspace_bytes(B, T, H, dk, dv), dtype=torch.uint8, device="cuda")
    o2, s2 = _call("gdn_prefill_fwd_ws", inp, ws)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    o_r, s_r = O.prefill(inp["q"], inp["k"], inp["v"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["mask"],
                         state_in=inp["state_in"], scale=float(inp["scale"]), chunk_size=64, dt=np.float64)
    assert float(np.abs(O.bf16_to_f32(to_np(o1)) - o_r).max()) <= 2e-2
    assert O.rel_fro(to_np(s1), s_r) <= 1e-3


@pytest.mark.gpu
def test_noalloc_allocates_nothing(cuda_device, lib):
    inp = _inputs(1, 1000, 4, 128, 128, 77)
    _call("gdn_prefill_fwd_noalloc", inp)                    # first call: module and symbol set-up
    _pool_high_water(reset=True)
    _call("gdn_prefill_fwd_noalloc", inp)
    assert _pool_high_water() == 0
    _call("gdn_prefill_fwd", inp)                            # control: the allocating entry point shows up
    assert _pool_high_water() >= lib.gdn_prefill_workspace_bytes(1, 1000, 4, 128, 128)
