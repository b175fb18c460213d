"""C ABI checks that need no GPU: the library loads, exports every entry point
declared in include/gdn_b200.h, and rejects bad arguments with status codes
(validation runs before any CUDA call, so no device is touched here; only
arguments that fail validation are used)."""
import ctypes
import os
import re

import pytest

from gdn_18646_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gdn_b200.h")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from gdn_18646_b200 import build
        build.build()
    return _lib.lib()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("gdn_prefill_fwd", "gdn_decode_step", "gdn_rmsnorm_fwd", "gdn_gated_rmsnorm_fwd",
              "gdn_proj_conv_silu_fwd", "gdn_last_error", "gdn_version", "gdn_check_device_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in gdn_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version(lib):
    assert b"sm_100a" in lib.gdn_version()


FAKE = 0x10000  # 16-byte aligned, never dereferenced: every call below fails validation first
ODD = 0x10002   # misaligned


def prefill_args(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, A_log=FAKE, a=FAKE, b=FAKE, gate=0, dtb=0.0, dtv=None, mask=None,
             s_in=None, out=FAKE, s_out=FAKE, B=1, T=64, Hqk=2, Hv=2, dk=128, dv=128, layout=0, scale=0.0,
             stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize("over,code", [
    (dict(q=None), _lib.GDN_ERR_NULL),
    (dict(out=None), _lib.GDN_ERR_NULL),
    (dict(B=0), _lib.GDN_ERR_SHAPE),
    (dict(T=0), _lib.GDN_ERR_SHAPE),
    (dict(Hqk=3, Hv=4), _lib.GDN_ERR_SHAPE),
    (dict(gate=5), _lib.GDN_ERR_DTYPE),
    (dict(layout=2), _lib.GDN_ERR_DTYPE),
    (dict(dk=96), _lib.GDN_ERR_UNSUPPORTED),
    (dict(dv=512), _lib.GDN_ERR_UNSUPPORTED),
    (dict(q=ODD), _lib.GDN_ERR_ALIGN),
    (dict(s_out=ODD), _lib.GDN_ERR_ALIGN),
])
def test_prefill_rejects(lib, over, code):
    assert _lib.call_status("gdn_prefill_fwd", *prefill_args(**over)) == code
    assert "gdn_prefill_fwd" in _lib.last_error()


def decode_args(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, a=FAKE, b=FAKE, gate=0, A_log=FAKE, dtb=None, s_in=FAKE, s_out=FAKE,
             out=FAKE, B=2, Hqk=2, Hv=2, dk=128, dv=128, scale=0.0, stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize("over,code", [
    (dict(s_in=None), _lib.GDN_ERR_NULL),
    (dict(B=-1), _lib.GDN_ERR_SHAPE),
    (dict(Hqk=4, Hv=2), _lib.GDN_ERR_SHAPE),
    (dict(gate=2), _lib.GDN_ERR_DTYPE),
    (dict(dk=100), _lib.GDN_ERR_UNSUPPORTED),
    (dict(s_out=ODD), _lib.GDN_ERR_ALIGN),
])
def test_decode_rejects(lib, over, code):
    assert _lib.call_status("gdn_decode_step", *decode_args(**over)) == code


@pytest.mark.parametrize("args,code", [
    ((None, FAKE, FAKE, 4, 2048, 1e-6, None), _lib.GDN_ERR_NULL),
    ((FAKE, FAKE, FAKE, 4, 2047, 1e-6, None), _lib.GDN_ERR_SHAPE),
    ((FAKE, FAKE, FAKE, 4, 16384, 1e-6, None), _lib.GDN_ERR_SHAPE),
    ((ODD, FAKE, FAKE, 4, 2048, 1e-6, None), _lib.GDN_ERR_ALIGN),
])
def test_rmsnorm_rejects(lib, args, code):
    assert _lib.call_status("gdn_rmsnorm_fwd", *args) == code


def test_gated_rmsnorm_rejects(lib):
    assert _lib.call_status("gdn_gated_rmsnorm_fwd", FAKE, 0, None, FAKE, FAKE, 4, 128, 1e-6, None) == \
        _lib.GDN_ERR_NULL
    assert _lib.call_status("gdn_gated_rmsnorm_fwd", FAKE, 9, FAKE, FAKE, FAKE, 4, 128, 1e-6, None) == \
        _lib.GDN_ERR_DTYPE


@pytest.mark.parametrize("over,code", [
    (dict(x=None), _lib.GDN_ERR_NULL),
    (dict(D=100), _lib.GDN_ERR_SHAPE),
    (dict(Dout=200), _lib.GDN_ERR_SHAPE),
    (dict(B=0), _lib.GDN_ERR_SHAPE),
    (dict(l2=100), _lib.GDN_ERR_SHAPE),
    (dict(y=ODD), _lib.GDN_ERR_ALIGN),
])
def test_proj_rejects(lib, over, code):
    a = dict(x=FAKE, W=FAKE, cw=FAKE, y=FAKE, B=1, T=8, D=256, Dout=256, csi=None, cso=None, l2=0, stream=None)
    a.update(over)
    assert _lib.call_status("gdn_proj_conv_silu_fwd", *a.values()) == code


def test_python_surface_raises_runtime_error(lib):
    with pytest.raises(_lib.GdnError) as ei:
        _lib.call("gdn_prefill_fwd", *prefill_args(dk=96))
    assert ei.value.status == _lib.GDN_ERR_UNSUPPORTED
    assert isinstance(ei.value, RuntimeError)


def test_prefill_workspace_and_schedule_entry_points(lib):
    rec = 2048 + 16384 + 2 * 128 * 128 + 8192 + 1024           # gate block, A1 lo/hi, W (tf32), P, gates

    def flags(n):                                               # one 4-byte ready flag per record, 128 B granules
        return (4 * n + 127) // 128 * 128
    assert lib.gdn_prefill_workspace_bytes(4, 4096, 16, 128, 128) == \
        4 * 16 * 64 * rec + 4 * 16 * 128 * 128 * 4 + flags(4 * 16 * 64)
    assert lib.gdn_prefill_workspace_bytes(1, 65, 2, 64, 64) == 2 * 2 * (2048 + 16384 + 2 * 64 * 128 + 9216) + \
        2 * 64 * 64 * 4 + flags(2 * 2)
    assert lib.gdn_prefill_workspace_bytes(1, 64, 2, 96, 64) == 0
    assert lib.gdn_prefill_workspace_bytes(0, 64, 2, 128, 128) == 0
    assert _lib.call_status("gdn_prefill_set_schedule", 7) == _lib.GDN_ERR_ARG
    assert _lib.call_status("gdn_prefill_set_schedule", _lib.GDN_SCHEDULE_AUTO) == _lib.GDN_OK
    assert lib.gdn_prefill_launch_count(1, 64, 2, 96, 64) == -1


def test_prefill_ws_rejects_small_workspace(lib):
    args = prefill_args()
    args = args[:-1] + [FAKE, 1024, None]                          # workspace, workspace_bytes, stream
    assert _lib.call_status("gdn_prefill_fwd_ws", *args) == _lib.GDN_ERR_SHAPE
    assert "workspace" in _lib.last_error()


def test_decode_proj_rejects(lib):
    def seg(**over):
        d = dict(W=FAKE, y=FAKE, conv_w=None, conv_state_in=None, conv_state_out=None, C=256, ldy=256, l2_group=0)
        d.update(over)
        return _lib.ProjSegment(**d)

    def call(segs, B=2, D=2048, x=FAKE):
        arr = (_lib.ProjSegment * max(1, len(segs)))(*segs)
        return _lib.call_status("gdn_decode_proj_fwd", x, None, 1e-6, B, D, arr, len(segs), None)

    assert call([seg()], x=None) == _lib.GDN_ERR_NULL
    assert call([seg()], B=9) == _lib.GDN_ERR_SHAPE
    assert call([seg()], D=2000) == _lib.GDN_ERR_SHAPE
    assert call([]) == _lib.GDN_ERR_SHAPE
    assert call([seg(C=40, ldy=40)]) == _lib.GDN_ERR_SHAPE
    assert call([seg()], D=1000) == _lib.GDN_ERR_SHAPE
    assert call([seg()], B=8, D=8192) == _lib.GDN_ERR_SHAPE
    assert call([seg(l2_group=128, C=192, ldy=192)]) == _lib.GDN_ERR_SHAPE
    assert call([seg(conv_state_in=FAKE)]) == _lib.GDN_ERR_NULL
    assert call([seg(W=ODD)]) == _lib.GDN_ERR_ALIGN
    assert "gdn_decode_proj_fwd" in _lib.last_error()


def varlen_args(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, A_log=FAKE, a=FAKE, b=FAKE, gate=0, dtb=0.0, dtv=None, cu=FAKE, N=2,
             Ttot=100, max_len=64, s_in=None, out=FAKE, s_out=FAKE, Hqk=2, Hv=2, dk=128, dv=128, scale=0.0,
             ws=FAKE, ws_bytes=1 << 30, stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize("over,code", [
    (dict(cu=None), _lib.GDN_ERR_NULL),
    (dict(cu=ODD), _lib.GDN_ERR_ALIGN),
    (dict(N=0), _lib.GDN_ERR_SHAPE),
    (dict(max_len=101), _lib.GDN_ERR_SHAPE),
    (dict(max_len=0), _lib.GDN_ERR_SHAPE),
    (dict(q=None), _lib.GDN_ERR_NULL),
    (dict(dk=96), _lib.GDN_ERR_UNSUPPORTED),
    (dict(Hqk=3, Hv=4), _lib.GDN_ERR_SHAPE),
])
def test_prefill_varlen_rejects(lib, over, code):
    assert _lib.call_status("gdn_prefill_varlen_fwd_ws", *varlen_args(**over)) == code
    assert "gdn_prefill" in _lib.last_error()


def test_prefill_varlen_workspace_matches_fixed_length(lib):
    assert lib.gdn_prefill_varlen_workspace_bytes(3, 1000, 4, 128, 128) == \
        lib.gdn_prefill_workspace_bytes(3, 1000, 4, 128, 128)


def test_decode_step_ex_rejects_unknown_flags(lib):
    args = [FAKE, FAKE, FAKE, FAKE, FAKE, 0, FAKE, None, FAKE, FAKE, FAKE, 1, 1, 1, 128, 128, 0.0]
    assert _lib.call_status("gdn_decode_step_ex", *args, 4, None) == _lib.GDN_ERR_DTYPE
    assert "flags" in _lib.last_error()


def test_outproj_rs_rejects(lib):
    import ctypes
    two = (ctypes.c_void_p * 2)(FAKE, FAKE)
    assert _lib.call_status("gdn_outproj_rs_fwd", None, FAKE, two, 1024, 256, 128, 0, 2, None) == _lib.GDN_ERR_NULL
    assert _lib.call_status("gdn_outproj_rs_fwd", FAKE, FAKE, two, 1000, 256, 128, 0, 2, None) == _lib.GDN_ERR_SHAPE
    assert _lib.call_status("gdn_outproj_rs_fwd", FAKE, FAKE, two, 1024, 200, 128, 0, 2, None) == _lib.GDN_ERR_SHAPE
    assert _lib.call_status("gdn_outproj_rs_fwd", FAKE, FAKE, two, 1024, 256, 128, 2, 2, None) == _lib.GDN_ERR_SHAPE
    odd = (ctypes.c_void_p * 2)(FAKE, ODD)
    assert _lib.call_status("gdn_outproj_rs_fwd", FAKE, FAKE, odd, 1024, 256, 128, 0, 2, None) == _lib.GDN_ERR_ALIGN
    assert _lib.call_status("gdn_outproj_reduce", FAKE, FAKE, 16, 100, 2, None) == _lib.GDN_ERR_SHAPE


def test_prefill_bwd_rejects(lib):
    base = [FAKE] * 6 + [0, 0.0, None, None, None, FAKE, 0, None] + [FAKE] * 7 + [None]
    def call(B=1, T=64, H=2, dk=64, dv=64, ws=FAKE, wsb=1 << 40, **over):
        args = list(base)
        for i, v in over.items():
            args[int(i[1:])] = v
        return _lib.call_status("gdn_prefill_bwd", *args, B, T, H, dk, dv, 0.0, ws, wsb, None)
    assert call(a0=None) == _lib.GDN_ERR_NULL
    assert call(T=0) == _lib.GDN_ERR_SHAPE
    assert call(dk=256) == _lib.GDN_ERR_UNSUPPORTED
    assert call(a6=7) == _lib.GDN_ERR_DTYPE
    assert call(a12=5) == _lib.GDN_ERR_DTYPE
    assert call(wsb=16) == _lib.GDN_ERR_SHAPE
    assert call(ws=ODD) == _lib.GDN_ERR_ALIGN
    assert lib.gdn_prefill_bwd_workspace_bytes(1, 64, 2, 96, 64) == 0
    # chunked (the default): per 64-token chunk the state entering it, its gradient
    # leaving it, the d and dd rows and the chunk's operand record
    n1 = 4 * 16 * 4096 // 64
    c1 = lib.gdn_prefill_bwd_workspace_bytes(4, 4096, 16, 128, 128)
    assert n1 * (2 * 128 * 128 + 2 * 64 * 128) * 4 <= c1 <= 1.5e9, c1   # config 1
    assert _lib.call_status("gdn_prefill_bwd_set_algorithm", 3) == _lib.GDN_ERR_ARG
    assert _lib.call_status("gdn_prefill_bwd_set_algorithm", _lib.GDN_BWD_TOKEN) == _lib.GDN_OK
    try:
        # token-recurrent in windows: checkpoints plus one window of per-token states
        t1 = lib.gdn_prefill_bwd_workspace_bytes(4, 4096, 16, 128, 128)
        assert t1 <= 1.5e9, t1                               # config 1 (one window: 17.2 GB)
        t4 = lib.gdn_prefill_bwd_workspace_bytes(8, 32768, 32, 128, 128)
        assert t4 <= 8e9, t4                                 # config 4 (one window: 275 GB)
        assert _lib.call_status("gdn_prefill_bwd_set_window", -1) == _lib.GDN_ERR_ARG
        assert _lib.call_status("gdn_prefill_bwd_set_window", 64) == _lib.GDN_OK
        small = lib.gdn_prefill_bwd_workspace_bytes(4, 4096, 16, 128, 128)
        assert small < t1                                    # 64-token windows hold fewer states
    finally:
        _lib.call_status("gdn_prefill_bwd_set_window", 0)
        _lib.call_status("gdn_prefill_bwd_set_algorithm", _lib.GDN_BWD_AUTO)
    assert lib.gdn_prefill_bwd_workspace_bytes(4, 4096, 16, 128, 128) == c1


def test_prefill_host_plan(lib):
    # config 1: segments of up to 1024 tokens (48 MiB of q, k, v), halving toward the end
    assert lib.gdn_prefill_host_segment(4, 4096, 16, 16, 128, 128, 1, 0) == 1024
    assert lib.gdn_prefill_host_segment(1, 100, 16, 16, 128, 128, 1, 512) == 128     # capped at T rounded up
    assert lib.gdn_prefill_host_segment(1, 100, 16, 16, 128, 128, 1, 96) == -1       # not a multiple of 64
    assert lib.gdn_prefill_host_segment(1, 100, 16, 16, 96, 128, 1, 0) == -1
    big = lib.gdn_prefill_host_workspace_bytes(4, 4096, 16, 16, 128, 128, 1, 0)
    small = lib.gdn_prefill_host_workspace_bytes(4, 4096, 16, 16, 128, 128, 1, 64)
    assert 0 < small < big
    # the segment prefill's own workspace is part of it
    assert small > lib.gdn_prefill_workspace_bytes(4, 64, 16, 128, 128)
    assert lib.gdn_prefill_host_workspace_bytes(4, 4096, 16, 16, 128, 128, 7, 0) == 0


def test_prefill_host_rejects(lib):
    def call(seg=0, ws=ODD, wsb=1 << 40, **over):
        args = prefill_args(**over)[:-1]                 # drop the stream
        return _lib.call_status("gdn_prefill_host", *args, seg, ws, wsb, None)
    assert call(q=None) == _lib.GDN_ERR_NULL
    assert call(T=0) == _lib.GDN_ERR_SHAPE
    assert call(dk=96) == _lib.GDN_ERR_SHAPE
    assert call(layout=5) == _lib.GDN_ERR_SHAPE
    assert call(seg=96) == _lib.GDN_ERR_SHAPE
    assert call(wsb=16) == _lib.GDN_ERR_SHAPE
    assert call(ws=None) == _lib.GDN_ERR_SHAPE
    assert call() == _lib.GDN_ERR_ALIGN
    assert "gdn_prefill_host" in _lib.last_error()


def _plan(lib, B, T, H, seg):
    starts = (ctypes.c_int * 4096)()
    n = lib.gdn_prefill_host_plan(B, T, H, H, 128, 128, 1, seg, starts, 4096)
    return [starts[i] for i in range(n + 1)]


@pytest.mark.parametrize("T", [1, 63, 64, 65, 1000, 4096, 5000, 70001])
def test_prefill_host_plan_segments(lib, T):
    auto = _plan(lib, 4, T, 16, 0)
    seg = lib.gdn_prefill_host_segment(4, T, 16, 16, 128, 128, 1, 0)
    assert auto[0] == 0 and auto[-1] == T
    lens = [b - a for a, b in zip(auto, auto[1:])]
    assert all(0 < x <= seg for x in lens)
    assert all(x % 64 == 0 for x in lens[:-1])          # chunk-aligned boundaries
    assert lens[-1] <= 64                                # the tail is one chunk
    if T == 4096:
        assert lens == [1024, 1024, 1024, 512, 256, 128, 64, 64]
    uni = _plan(lib, 4, T, 16, 128)                      # explicit: uniform, ragged last
    assert uni == list(range(0, T, 128)) + [T]


def test_decode_step_gated_rejects(lib):
    base = [FAKE, FAKE, FAKE, FAKE, FAKE, 0, FAKE, None, FAKE, FAKE, None]
    def call(z=FAKE, gamma=FAKE, y=FAKE, dk=128, flags=0):
        return _lib.call_status("gdn_decode_step_gated", *base, z, gamma, 1e-6, y, 1, 1, 1, dk, 128, 0.0, flags, None)
    assert call(y=None) == _lib.GDN_ERR_NULL
    assert call(z=None) == _lib.GDN_ERR_NULL
    assert call(gamma=None) == _lib.GDN_ERR_NULL
    assert call(dk=96) == _lib.GDN_ERR_UNSUPPORTED
    assert call(flags=8) == _lib.GDN_ERR_DTYPE
    assert call(y=ODD) == _lib.GDN_ERR_ALIGN
    assert "gdn_decode_step_gated" in _lib.last_error()


def test_proj_multi_rejects(lib):
    segs = (_lib.ProjOutSeg * 2)()
    for s_ in segs:
        s_.W, s_.y, s_.conv_w, s_.Dout, s_.l2norm_group = FAKE, FAKE, None, 128, 0
    assert _lib.call_status("gdn_proj_multi_fwd", None, 1, 8, 64, segs, 2, None) == _lib.GDN_ERR_NULL
    assert _lib.call_status("gdn_proj_multi_fwd", FAKE, 1, 8, 64, segs, 0, None) == _lib.GDN_ERR_SHAPE
    assert _lib.call_status("gdn_proj_multi_fwd", FAKE, 1, 8, 64, segs, 7, None) == _lib.GDN_ERR_SHAPE
    segs[1].Dout = 100
    assert _lib.call_status("gdn_proj_multi_fwd", FAKE, 1, 8, 64, segs, 2, None) == _lib.GDN_ERR_SHAPE
    segs[1].Dout, segs[1].y = 128, ODD
    assert _lib.call_status("gdn_proj_multi_fwd", FAKE, 1, 8, 64, segs, 2, None) == _lib.GDN_ERR_ALIGN
    segs[1].y, segs[1].W = FAKE, None
    assert _lib.call_status("gdn_proj_multi_fwd", FAKE, 1, 8, 64, segs, 2, None) == _lib.GDN_ERR_NULL


def test_prefill_window_rejects(lib):
    def call(t0=0, Tw=64, ws=ODD, wsb=1 << 40, **over):
        args = prefill_args(**over)
        head, tail = args[:15], args[15:-2]              # ... B, T | Hqk, Hv, dk, dv, layout
        scale = args[-2]
        return _lib.call_status("gdn_prefill_window_ws", *head, t0, Tw, *tail, scale, ws, wsb, None)
    assert call(q=None) == _lib.GDN_ERR_NULL
    assert call(T=128, t0=-64) == _lib.GDN_ERR_SHAPE
    assert call(T=128, t0=64, Tw=65) == _lib.GDN_ERR_SHAPE
    assert call(T=128, Tw=0) == _lib.GDN_ERR_SHAPE
    assert "window" in _lib.last_error()
    assert call(T=128, t0=64, Tw=64, wsb=16) == _lib.GDN_ERR_SHAPE   # workspace below the window's size
    assert call(T=128, t0=64, Tw=64) == _lib.GDN_ERR_ALIGN            # everything else valid: the workspace
    assert call(T=128, t0=64, Tw=64, dk=96) == _lib.GDN_ERR_UNSUPPORTED


def test_gather_window_rejects(lib):
    two = (ctypes.c_void_p * 2)(FAKE, FAKE)
    one_missing = (ctypes.c_void_p * 2)(FAKE, None)
    def call(g=FAKE, peers=two, world=2, rank=0, B=1, T=128, H=2, dv=128, layout=0, t0=0, Tw=64):
        return _lib.call_status("gdn_gather_window", g, peers, world, rank, B, T, H, dv, layout, t0, Tw, None)
    assert call(g=None) == _lib.GDN_ERR_NULL
    assert call(peers=None) == _lib.GDN_ERR_NULL
    assert call(peers=one_missing) == _lib.GDN_ERR_NULL               # rank 1's buffer is needed by rank 0
    assert call(rank=2) == _lib.GDN_ERR_SHAPE
    assert call(world=0) == _lib.GDN_ERR_SHAPE
    assert call(t0=64, Tw=128) == _lib.GDN_ERR_SHAPE
    assert call(layout=3) == _lib.GDN_ERR_DTYPE
    assert call(world=1, rank=0, peers=one_missing) == _lib.GDN_OK   # nothing to pull, nothing enqueued


def test_prefill_fwd_ex_rejects(lib):
    """Per-call options: unknown schedule or gate layout -> GDN_ERR_ARG, a token-row
    gate stride below Hv -> GDN_ERR_SHAPE; otherwise the _ws checks apply."""
    def call(schedule=0, gl=0, gld=0, ws=ODD, wsb=1 << 40, **over):
        args = prefill_args(**over)[:-1]                      # ... scale (stream goes last)
        opts = _lib.PrefillOpts(schedule, gl, gld)
        return _lib.call_status("gdn_prefill_fwd_ex", *args, ctypes.byref(opts), ws, wsb, None)
    assert call(schedule=4) == _lib.GDN_ERR_ARG
    assert call(schedule=-1) == _lib.GDN_ERR_ARG
    assert call(gl=2) == _lib.GDN_ERR_ARG
    assert "gate layout" in _lib.last_error()
    assert call(gl=1, gld=1) == _lib.GDN_ERR_SHAPE             # Hv = 2 gates per token row at least
    assert call(q=None) == _lib.GDN_ERR_NULL
    assert call(gl=1, gld=64) == _lib.GDN_ERR_ALIGN             # everything else valid: the workspace
    args = prefill_args()[:-1]
    assert _lib.call_status("gdn_prefill_fwd_ex", *args, None, ODD, 1 << 40, None) == _lib.GDN_ERR_ALIGN


def test_schedule_is_per_thread(lib):
    """gdn_prefill_set_schedule changes the calling thread's default only."""
    import threading
    seen = {}

    def other():
        seen["count"] = lib.gdn_prefill_launch_count_ex(1, 1000, 4, 128, 256, _lib.GDN_SCHEDULE_PIECED)
        seen["default"] = _lib.call_status("gdn_prefill_set_schedule", _lib.GDN_SCHEDULE_SINGLE)
    _lib.call("gdn_prefill_set_schedule", _lib.GDN_SCHEDULE_AUTO)
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["default"] == _lib.GDN_OK
    assert lib.gdn_prefill_launch_count_ex(1, 64, 2, 96, 64, 0) == -1
    assert lib.gdn_prefill_launch_count_ex(1, 64, 2, 128, 64, 9) == -1


def test_prefill_test_hooks_reject(lib):
    assert _lib.call_status("gdn_test_prefill_hooks", -1, -1) == _lib.GDN_ERR_ARG
    assert _lib.call_status("gdn_test_prefill_hooks", 0, -2) == _lib.GDN_ERR_ARG
