"""Torch-facing operators over the C ABI (libgdn_b200.so).

Two surfaces:

* functional ops (``prefill``, ``decode_step``, ``rmsnorm``, ``gated_rmsnorm``,
  ``proj_conv_silu``) taking torch CUDA tensors, shape-generic, launching on
  ``torch.cuda.current_stream()``;
* drop-in module objects with the reference's operator surface -- the
  ``exts`` dict consumed by ``gdn_layer.GDNLayerCustom`` (gdn_layer.py:206-217):
  ``exts()['prefill'].prefill(...)`` (kernels/prefill_chunked.cu:512-526),
  ``['decode'].forward(...)`` (kernels/decode.cu:172-218),
  ``['proj'].forward(...)`` (kernels/fused_proj_conv_silu.cu:298-360),
  ``['rmsnorm'].forward(...)`` (kernels/rmsnorm.cu:280-298).

torch is only the allocator / stream provider here; all arithmetic runs in
the sm_100a kernels of the library.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import (GDN_DTYPE_BF16, GDN_DTYPE_F32, GDN_LAYOUT_BHTD, GDN_LAYOUT_BTHD)

CHUNK = 64


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _gate_dtype(t: torch.Tensor, name: str) -> int:
    if t.dtype == torch.bfloat16:
        return GDN_DTYPE_BF16
    if t.dtype == torch.float32:
        return GDN_DTYPE_F32
    raise RuntimeError(f"{name}: gate tensors must be bfloat16 or float32, got {t.dtype}")


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda_contig(t: torch.Tensor, name: str, dtype=None) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")
    if dtype is not None:
        _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


# ---------------------------------------------------------------------------
# functional ops
# ---------------------------------------------------------------------------


_SCHEDULES = {None: 0, "auto": 0, "single": 1, "pieced": 2, "stream": 3}


def prefill(q, k, v, A_log, a, b_logits, *, dt_bias=0.0, mask=None, state_in=None,
            scale=0.0, layout="bhtd", out=None, state_out=None, return_state=True, gates="bht", schedule=None):
    """Chunked gated-delta-rule prefill (reference/prefill_ref.py semantics).

    layout "bhtd": q,k [B,Hqk,T,dk], v [B,Hv,T,dv]; "bthd": q,k [B,T,Hqk,dk], v [B,T,Hv,dv].
    a, b_logits [B,Hv,T] (bf16 or f32), or with gates="bth" [B,T,Hv] views whose
    token rows share one stride (read in place, e.g. the halves of a [B,T,2Hv]
    projection); A_log [Hv] f32; dt_bias float or f32 [Hv]; mask [B,T] f32 or None;
    state_in [B,Hv,dk,dv] f32 or None; schedule None/"auto", "single", "pieced" or
    "stream" for this call (gdn_prefill_fwd_ex).
    Returns (out bf16 in v's layout, state_out f32 [B,Hv,dk,dv] or None).
    """
    _need(gates in ("bht", "bth"), f"gates must be 'bht' or 'bth', got {gates!r}")
    _need(schedule in _SCHEDULES, f"schedule must be one of {sorted(k_ for k_ in _SCHEDULES if k_)}, got {schedule!r}")
    lay, B, T, Hqk, Hv, dk, dv, gdt, dt_scalar, dt_vec = _prefill_checks(q, k, v, A_log, a, b_logits, dt_bias, mask,
                                                                         state_in, layout, gates)
    if out is None:
        out = torch.empty_like(v)
    if state_out is None and return_state:
        state_out = torch.empty(B, Hv, dk, dv, dtype=torch.float32, device=q.device)
    ws_bytes = _lib.lib().gdn_prefill_workspace_bytes(B, T, Hv, dk, dv)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=q.device)
    opts = _lib.PrefillOpts(_SCHEDULES[schedule], _lib.GDN_GATES_BTH if gates == "bth" else _lib.GDN_GATES_BHT,
                            a.stride(1) if gates == "bth" else 0)
    _lib.call("gdn_prefill_fwd_ex", _ptr(q), _ptr(k), _ptr(v), _ptr(A_log), _ptr(a), _ptr(b_logits), gdt,
              dt_scalar, _ptr(dt_vec), _ptr(mask), _ptr(state_in), _ptr(out), _ptr(state_out),
              B, T, Hqk, Hv, dk, dv, lay, float(scale), ctypes.byref(opts), _ptr(ws), int(ws_bytes), _stream())
    return out, state_out


def prefill_window(q, k, v, A_log, a, b_logits, t0, Tw, *, out, dt_bias=0.0, mask=None, state_in=None,
                   state_out=None, scale=0.0, layout="bhtd", workspace=None):
    """``prefill`` over the tokens [t0, t0 + Tw) of the given (whole) tensors
    (gdn_prefill_window_ws): reads the window's q, k, v, gates and mask in place
    and writes its o into the same tokens of ``out``; ``state_in`` is the state
    before token t0, ``state_out`` the state after the window.  ``workspace``: a
    uint8 CUDA tensor of at least gdn_prefill_workspace_bytes(B, Tw, Hv, dk, dv)
    bytes (allocated per call if None)."""
    lay, B, T, Hqk, Hv, dk, dv, gdt, dt_scalar, dt_vec = _prefill_checks(q, k, v, A_log, a, b_logits, dt_bias, mask,
                                                                         state_in, layout)
    _cuda_contig(out, "out", torch.bfloat16)
    _need(tuple(out.shape) == tuple(v.shape), "out must have v's shape")
    if state_out is not None:
        _cuda_contig(state_out, "state_out", torch.float32)
    ws_bytes = int(_lib.lib().gdn_prefill_workspace_bytes(B, max(int(Tw), 1), Hv, dk, dv))
    if workspace is None:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    _need(workspace.is_cuda and workspace.dtype == torch.uint8 and workspace.numel() >= ws_bytes,
          f"workspace: uint8 CUDA tensor of at least {ws_bytes} bytes required")
    _lib.call("gdn_prefill_window_ws", _ptr(q), _ptr(k), _ptr(v), _ptr(A_log), _ptr(a), _ptr(b_logits), gdt,
              dt_scalar, _ptr(dt_vec), _ptr(mask), _ptr(state_in), _ptr(out), _ptr(state_out),
              B, T, int(t0), int(Tw), Hqk, Hv, dk, dv, lay, float(scale), _ptr(workspace), workspace.numel(),
              _stream())
    return out, state_out


def _prefill_checks(q, k, v, A_log, a, b_logits, dt_bias, mask, state_in, layout, gates="bht"):
    """Shape, dtype and device checks shared by the prefill wrappers; returns
    (layout code, B, T, Hqk, Hv, dk, dv, gate dtype code, dt_bias scalar, dt_bias vector).
    ``gates`` "bht": a, b_logits contiguous [B, Hv, T]; "bth": [B, T, Hv] views whose
    tokens are rows of one stride (e.g. the halves of a [B, T, 2 Hv] projection)."""
    lay = GDN_LAYOUT_BHTD if layout == "bhtd" else GDN_LAYOUT_BTHD
    for name, t in (("q", q), ("k", k), ("v", v)):
        _cuda_contig(t, name, torch.bfloat16)
    if lay == GDN_LAYOUT_BHTD:
        B, Hqk, T, dk = q.shape
        Hv, dv = v.shape[1], v.shape[3]
    else:
        B, T, Hqk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
    _need(tuple(k.shape) == tuple(q.shape), "k must have q's shape")
    gdt = _gate_dtype(a, "a")
    _need(b_logits.dtype == a.dtype, "a and b_logits must share a dtype")
    if gates == "bth":
        _need(a.is_cuda and b_logits.is_cuda, "a and b_logits must be CUDA tensors")
        _need(tuple(a.shape) == (B, T, Hv) and tuple(b_logits.shape) == (B, T, Hv),
              "a, b_logits must be [B, T, Hv] with gates='bth'")
        ld = a.stride(1)
        _need(a.stride(2) == 1 and tuple(b_logits.stride()) == tuple(a.stride()) and a.stride(0) == T * ld
              and ld >= Hv, "a, b_logits (gates='bth'): token rows of one stride, heads contiguous")
    else:
        _cuda_contig(a, "a")
        _cuda_contig(b_logits, "b_logits")
        _need(tuple(a.shape) == (B, Hv, T) and tuple(b_logits.shape) == (B, Hv, T), "a, b_logits must be [B, Hv, T]")
    _cuda_contig(A_log, "A_log", torch.float32)
    dt_vec = None
    dt_scalar = 0.0
    if isinstance(dt_bias, torch.Tensor) and dt_bias.numel() > 1:
        _cuda_contig(dt_bias, "dt_bias", torch.float32)
        dt_vec = dt_bias
    else:
        dt_scalar = float(dt_bias)
    if mask is not None:
        _cuda_contig(mask, "mask", torch.float32)
    if state_in is not None:
        _cuda_contig(state_in, "state_in", torch.float32)
    return lay, B, T, Hqk, Hv, dk, dv, gdt, dt_scalar, dt_vec


def _contig(t: torch.Tensor, name: str, dtype=None) -> None:
    _need(t.is_contiguous(), f"{name} must be contiguous")
    if dtype is not None:
        _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


def prefill_host(q, k, v, A_log, a, b_logits, *, dt_bias=0.0, mask=None, state_in=None, scale=0.0,
                 layout="bhtd", out=None, state_out=None, return_state=True, seg_tokens=0, device=None,
                 synchronize=True):
    """``prefill`` on host tensors (gdn_prefill_host): the inputs are copied to the
    GPU and the results back in token segments that overlap the prefill of the
    neighbouring segments.  Tensors may live on the host (pinned, for the copies
    to overlap) or on the device; outputs default to pinned host tensors.
    ``seg_tokens`` 0 picks the segment length.  With ``synchronize`` the current
    stream is synchronised before returning; without it the host outputs are
    valid once the stream completes, and the caller keeps the host inputs alive
    until then.  Same result as ``prefill`` on the whole sequence."""
    lay = GDN_LAYOUT_BHTD if layout == "bhtd" else GDN_LAYOUT_BTHD
    for name, t in (("q", q), ("k", k), ("v", v)):
        _contig(t, name, torch.bfloat16)
    if lay == GDN_LAYOUT_BHTD:
        B, Hqk, T, dk = q.shape
        Hv, dv = v.shape[1], v.shape[3]
    else:
        B, T, Hqk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
    _need(tuple(k.shape) == tuple(q.shape), "k must have q's shape")
    gdt = _gate_dtype(a, "a")
    _need(b_logits.dtype == a.dtype, "a and b_logits must share a dtype")
    _contig(a, "a")
    _contig(b_logits, "b_logits")
    _need(tuple(a.shape) == (B, Hv, T) and tuple(b_logits.shape) == (B, Hv, T), "a, b_logits must be [B, Hv, T]")
    _contig(A_log, "A_log", torch.float32)
    dt_vec, dt_scalar = None, 0.0
    if isinstance(dt_bias, torch.Tensor) and dt_bias.numel() > 1:
        _contig(dt_bias, "dt_bias", torch.float32)
        dt_vec = dt_bias
    else:
        dt_scalar = float(dt_bias)
    if mask is not None:
        _contig(mask, "mask", torch.float32)
    if state_in is not None:
        _contig(state_in, "state_in", torch.float32)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty(v.shape, dtype=torch.bfloat16, pin_memory=True)
    if state_out is None and return_state:
        state_out = torch.empty(B, Hv, dk, dv, dtype=torch.float32, pin_memory=True)
    ws_bytes = int(_lib.lib().gdn_prefill_host_workspace_bytes(B, T, Hqk, Hv, dk, dv, gdt, int(seg_tokens)))
    _need(ws_bytes > 0, f"prefill_host: unsupported shapes or seg_tokens={seg_tokens}")
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    ws_ptr = (ws.data_ptr() + 255) // 256 * 256
    with torch.cuda.device(dev):
        _lib.call("gdn_prefill_host", _ptr(q), _ptr(k), _ptr(v), _ptr(A_log), _ptr(a), _ptr(b_logits), gdt,
                  dt_scalar, _ptr(dt_vec), _ptr(mask), _ptr(state_in), _ptr(out), _ptr(state_out),
                  B, T, Hqk, Hv, dk, dv, lay, float(scale), int(seg_tokens), ws_ptr, ws_bytes, _stream())
        if synchronize:
            torch.cuda.current_stream().synchronize()
    return out, state_out


def prefill_varlen(q, k, v, A_log, a, b_logits, cu_seqlens, *, max_len=None, dt_bias=0.0, state_in=None,
                   scale=0.0, out=None, state_out=None, return_state=True):
    """Prefill of N sequences packed along the token axis (gdn_prefill_varlen_fwd_ws).

    q,k [Ttot,Hqk,dk], v [Ttot,Hv,dv] bf16; a, b_logits [Hv,Ttot]; cu_seqlens int32 [N+1]
    on the device (sequence i = tokens cu_seqlens[i]:cu_seqlens[i+1]); max_len = the
    longest sequence (read from cu_seqlens with a device->host copy when not given);
    state_in [N,Hv,dk,dv] f32 or None.  Returns (out [Ttot,Hv,dv] bf16, state_out
    [N,Hv,dk,dv] f32 or None); per sequence the result of ``prefill`` on it alone."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _cuda_contig(t, name, torch.bfloat16)
    _need(q.dim() == 3 and v.dim() == 3, "q, k, v must be [Ttot, H, D]")
    Ttot, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    _need(tuple(k.shape) == tuple(q.shape) and v.shape[0] == Ttot, "k must have q's shape, v Ttot rows")
    gdt = _gate_dtype(a, "a")
    _need(b_logits.dtype == a.dtype, "a and b_logits must share a dtype")
    _cuda_contig(a, "a")
    _cuda_contig(b_logits, "b_logits")
    _need(tuple(a.shape) == (Hv, Ttot) and tuple(b_logits.shape) == (Hv, Ttot), "a, b_logits must be [Hv, Ttot]")
    _cuda_contig(cu_seqlens, "cu_seqlens", torch.int32)
    N = cu_seqlens.numel() - 1
    _need(N >= 1, "cu_seqlens needs at least two entries")
    if max_len is None:
        max_len = int((cu_seqlens[1:] - cu_seqlens[:-1]).max())
    max_len = max(int(max_len), 1)
    _cuda_contig(A_log, "A_log", torch.float32)
    dt_vec, dt_scalar = None, 0.0
    if isinstance(dt_bias, torch.Tensor) and dt_bias.numel() > 1:
        _cuda_contig(dt_bias, "dt_bias", torch.float32)
        dt_vec = dt_bias
    else:
        dt_scalar = float(dt_bias)
    if state_in is not None:
        _cuda_contig(state_in, "state_in", torch.float32)
    if out is None:
        out = torch.empty_like(v)
    if state_out is None and return_state:
        state_out = torch.empty(N, Hv, dk, dv, dtype=torch.float32, device=q.device)
    ws_bytes = _lib.lib().gdn_prefill_varlen_workspace_bytes(N, max_len, Hv, dk, dv)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=q.device)
    _lib.call("gdn_prefill_varlen_fwd_ws", _ptr(q), _ptr(k), _ptr(v), _ptr(A_log), _ptr(a), _ptr(b_logits), gdt,
              dt_scalar, _ptr(dt_vec), _ptr(cu_seqlens), N, Ttot, max_len, _ptr(state_in), _ptr(out),
              _ptr(state_out), Hqk, Hv, dk, dv, float(scale), _ptr(ws), int(ws_bytes), _stream())
    return out, state_out


def prefill_backward(q, k, v, A_log, a, b_logits, dO, *, dt_bias=0.0, mask=None, state_in=None, dS_final=None,
                     scale=0.0, need_dstate=True, window=None, algorithm=None):
    """Gradients of ``prefill`` (gdn_prefill_bwd): q, k [B,H,T,dk], v [B,H,T,dv] bf16
    (layout "bhtd", Hqk == Hv), gates as ``prefill``, dO [B,H,T,dv] (bf16 or f32),
    dS_final [B,H,dk,dv] or None.  ``algorithm``: "token" (token-recurrent, in
    windows), "chunked" (64-token chunks) or None (the library's choice).
    ``window``: tokens per window of the token-recurrent backward (None: automatic,
    max(256, sqrt T)).  Returns a dict of fp32 tensors
    dq, dk, dv, da, db, dA_log [H], ddt_bias ([H] for a per-head dt_bias, a scalar
    tensor otherwise) and dstate_in (or None)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _cuda_contig(t, name, torch.bfloat16)
    B, H, T, dk = q.shape
    dv = v.shape[-1]
    gdt = _gate_dtype(a, "a")
    _need(b_logits.dtype == a.dtype, "a and b_logits must share a dtype")
    _cuda_contig(a, "a")
    _cuda_contig(b_logits, "b_logits")
    _need(dO.dtype in (torch.bfloat16, torch.float32), "dO must be bf16 or f32")
    _cuda_contig(dO, "dO")
    dod = GDN_DTYPE_BF16 if dO.dtype == torch.bfloat16 else GDN_DTYPE_F32
    dt_vec = dt_bias if isinstance(dt_bias, torch.Tensor) and dt_bias.numel() > 1 else None
    dt_scalar = 0.0 if dt_vec is not None else float(dt_bias)
    f32 = dict(dtype=torch.float32, device=q.device)
    g = dict(dq=torch.empty(B, H, T, dk, **f32), dk=torch.empty(B, H, T, dk, **f32), dv=torch.empty(B, H, T, dv, **f32),
             da=torch.empty(B, H, T, **f32), db=torch.empty(B, H, T, **f32), dA_log=torch.empty(H, **f32),
             ddt_bias=torch.empty(H, **f32),
             dstate_in=torch.empty(B, H, dk, dv, **f32) if need_dstate else None)
    _need(window is None or int(window) > 0, f"window must be a positive token count, got {window!r}")
    algos = {None: 0, "token": 1, "chunked": 2}
    _need(algorithm in algos, f"algorithm must be None, 'token' or 'chunked', got {algorithm!r}")
    lib = _lib.lib()
    _lib.call("gdn_prefill_bwd_set_window", 0 if window is None else int(window))
    _lib.call("gdn_prefill_bwd_set_algorithm", algos[algorithm])
    try:
        ws_bytes = lib.gdn_prefill_bwd_workspace_bytes(B, T, H, dk, dv)
        ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=q.device)
        _lib.call("gdn_prefill_bwd", _ptr(q), _ptr(k), _ptr(v), _ptr(A_log), _ptr(a), _ptr(b_logits), gdt,
                  dt_scalar, _ptr(dt_vec), _ptr(mask), _ptr(state_in), _ptr(dO), dod, _ptr(dS_final), _ptr(g["dq"]),
                  _ptr(g["dk"]), _ptr(g["dv"]), _ptr(g["da"]), _ptr(g["db"]), _ptr(g["dA_log"]),
                  _ptr(g["ddt_bias"]), _ptr(g["dstate_in"]), B, T, H, dk, dv, float(scale), _ptr(ws),
                  int(ws_bytes), _stream())
    finally:
        _lib.call("gdn_prefill_bwd_set_window", 0)
        _lib.call("gdn_prefill_bwd_set_algorithm", 0)
    if dt_vec is None:
        g["ddt_bias"] = g["ddt_bias"].sum()
    return g


class PrefillFunction(torch.autograd.Function):
    """``prefill`` as an autograd op (layout "bhtd", Hqk == Hv): forward is the
    chunked tcgen05 prefill, backward gdn_prefill_backward.  Differentiable
    inputs: q, k, v, A_log, a, b_logits, dt_bias (tensor) and state_in;
    outputs (o, state_out)."""

    @staticmethod
    def forward(ctx, q, k, v, A_log, a, b_logits, dt_bias, state_in, scale):
        o, S = prefill(q, k, v, A_log, a, b_logits, dt_bias=dt_bias, state_in=state_in, scale=scale)
        ctx.save_for_backward(q, k, v, A_log, a, b_logits, dt_bias, state_in)
        ctx.scale = scale
        return o, S

    @staticmethod
    def backward(ctx, do, dS):
        q, k, v, A_log, a, b_logits, dt_bias, state_in = ctx.saved_tensors
        if do is None:
            do = torch.zeros_like(v, dtype=torch.float32)
        g = prefill_backward(q, k, v, A_log, a, b_logits, do.contiguous(), dt_bias=dt_bias, state_in=state_in,
                             dS_final=None if dS is None else dS.contiguous(), scale=ctx.scale)
        ddt = g["ddt_bias"].reshape(dt_bias.shape).to(dt_bias.dtype)
        return (g["dq"].to(q.dtype), g["dk"].to(k.dtype), g["dv"].to(v.dtype), g["dA_log"], g["da"].to(a.dtype),
                g["db"].to(b_logits.dtype), ddt, g["dstate_in"], None)


def prefill_autograd(q, k, v, A_log, a, b_logits, dt_bias, state_in, scale=0.0):
    """Differentiable ``prefill`` (see PrefillFunction); dt_bias a tensor ([H] or [1])."""
    return PrefillFunction.apply(q, k, v, A_log, a, b_logits, dt_bias, state_in, scale)


def decode_step(q, k, v, a, b, A_log, dt_bias, state, *, scale=0.0, out=None, state_out=None, l2norm_qk=False):
    """One decode step; updates ``state`` in place unless ``state_out`` is given.
    q,k [B,Hqk,dk] bf16; v [B,Hv,dv] bf16; a,b [B,Hv]; state [B,Hv,dk,dv] f32.
    With ``l2norm_qk`` q and k are L2-normalised per head inside the kernel.
    Returns out f32 [B,Hv,dv]."""
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for name, t in (("q", q), ("k", k), ("v", v)):
        _cuda_contig(t, name, torch.bfloat16)
    _cuda_contig(state, "state", torch.float32)
    gdt = _gate_dtype(a, "a")
    if out is None:
        out = torch.empty(B, Hv, dv, dtype=torch.float32, device=q.device)
    if state_out is None:
        state_out = state
    _lib.call("gdn_decode_step_ex", _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), gdt, _ptr(A_log),
              _ptr(dt_bias), _ptr(state), _ptr(state_out), _ptr(out), B, Hqk, Hv, dk, dv, float(scale),
              _lib.GDN_DECODE_L2NORM_QK if l2norm_qk else 0, _stream())
    return out


def decode_step_gated(q, k, v, a, b, A_log, dt_bias, state, z, norm_gamma, eps, *, scale=0.0, y=None,
                      out=None, state_out=None, l2norm_qk=False):
    """``decode_step`` with the layer's gated output norm applied to each head's o row in
    the same kernel (gdn_decode_step_gated): y = rmsnorm_dv(o) * norm_gamma * silu(z), bf16.
    z [B,Hv,dv] bf16; norm_gamma [dv] bf16.  ``out`` (the fp32 o) is written only when
    given.  Returns y [B,Hv,dv] bf16."""
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for name, t in (("q", q), ("k", k), ("v", v), ("z", z), ("norm_gamma", norm_gamma)):
        _cuda_contig(t, name, torch.bfloat16)
    _cuda_contig(state, "state", torch.float32)
    _need(z.numel() == B * Hv * dv and norm_gamma.numel() == dv, "z must be [B, Hv, dv] and norm_gamma [dv]")
    gdt = _gate_dtype(a, "a")
    if y is None:
        y = torch.empty(B, Hv, dv, dtype=torch.bfloat16, device=q.device)
    if state_out is None:
        state_out = state
    _lib.call("gdn_decode_step_gated", _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), gdt, _ptr(A_log),
              _ptr(dt_bias), _ptr(state), _ptr(state_out), _ptr(out), _ptr(z), _ptr(norm_gamma), float(eps),
              _ptr(y), B, Hqk, Hv, dk, dv, float(scale), _lib.GDN_DECODE_L2NORM_QK if l2norm_qk else 0, _stream())
    return y


def outproj_rs(x, W, recv_ptrs, rank, world):
    """This rank's share of a head-sharded output projection, sent to its owners
    (gdn_outproj_rs_fwd): the partial product x [M, K] @ W[N, K]^T, cut into row
    blocks of M/world tokens, block s written into slot ``rank`` of the receive
    buffer at ``recv_ptrs[s]`` (device pointers of every rank's [world, M/world, N]
    bf16 buffer, peers' mapped into this process).  Only launches; ordering the
    reduction after every rank's call is the caller's job."""
    _cuda_contig(x, "x", torch.bfloat16)
    _cuda_contig(W, "W", torch.bfloat16)
    _need(x.dim() == 2 and W.dim() == 2 and x.shape[1] == W.shape[1], "x [M, K] and W [N, K] required")
    _need(len(recv_ptrs) == world, "one receive buffer per rank")
    arr = (ctypes.c_void_p * world)(*[int(p) for p in recv_ptrs])
    _lib.call("gdn_outproj_rs_fwd", _ptr(x), _ptr(W), arr, x.shape[0], W.shape[0], x.shape[1], int(rank), int(world),
              _stream())


def gather_window(gathered, peer_ptrs, rank, t0, Tw, layout="bhtd", stream=None):
    """Pull tokens [t0, t0 + Tw) of every peer's slot of a head-sharded o into the
    same slots of ``gathered`` [world, B, H_local, T, dv] ("bhtd") or [world, B, T,
    H_local, dv] ("bthd") (gdn_gather_window): one copy-engine transfer per peer
    from ``peer_ptrs[p]`` (rank p's gathered buffer, mapped into this process),
    enqueued on ``stream`` (default: the current stream).  Only enqueues; the
    caller orders it after the peers wrote the window."""
    _cuda_contig(gathered, "gathered", torch.bfloat16)
    _need(gathered.dim() == 5, "gathered must be [world, B, H, T, dv] or [world, B, T, H, dv]")
    _need(layout in ("bhtd", "bthd"), f"layout must be 'bhtd' or 'bthd', got {layout!r}")
    world = gathered.shape[0]
    _need(len(peer_ptrs) == world, "one peer pointer per rank")
    if layout == "bhtd":
        _, B, H, T, dv = gathered.shape
        lay = GDN_LAYOUT_BHTD
    else:
        _, B, T, H, dv = gathered.shape
        lay = GDN_LAYOUT_BTHD
    arr = (ctypes.c_void_p * world)(*[int(p) for p in peer_ptrs])
    s = stream.cuda_stream if stream is not None else _stream()
    _lib.call("gdn_gather_window", _ptr(gathered), arr, world, int(rank), B, T, H, dv, lay, int(t0), int(Tw), s)


def outproj_reduce(recv, out=None):
    """out [rows, N] = bf16(sum over slots of recv [world, rows, N]) (gdn_outproj_reduce)."""
    _cuda_contig(recv, "recv", torch.bfloat16)
    world, rows, N = recv.shape
    if out is None:
        out = torch.empty(rows, N, dtype=torch.bfloat16, device=recv.device)
    _lib.call("gdn_outproj_reduce", _ptr(recv), _ptr(out), rows, N, world, _stream())
    return out


def rmsnorm(x, gamma, eps=1e-6, out=None):
    """y = x * rsqrt(mean(x^2) + eps) * gamma over the last dim; bf16 in/out."""
    _cuda_contig(x, "x", torch.bfloat16)
    _cuda_contig(gamma, "gamma", torch.bfloat16)
    D = x.shape[-1]
    R = x.numel() // D
    if out is None:
        out = torch.empty_like(x)
    _lib.call("gdn_rmsnorm_fwd", _ptr(x), _ptr(gamma), _ptr(out), R, D, float(eps), _stream())
    return out


def gated_rmsnorm(x, z, gamma, eps=1e-6, out=None):
    """y = rmsnorm(x) * gamma * silu(z) over the last dim (x bf16 or f32, z bf16)."""
    _cuda_contig(x, "x")
    _cuda_contig(z, "z", torch.bfloat16)
    _cuda_contig(gamma, "gamma", torch.bfloat16)
    xdt = _gate_dtype(x, "x")
    D = x.shape[-1]
    R = x.numel() // D
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("gdn_gated_rmsnorm_fwd", _ptr(x), xdt, _ptr(z), _ptr(gamma), _ptr(out), R, D, float(eps),
              _stream())
    return out


def proj_conv_silu(x, W, conv_w, *, conv_state_in=None, conv_state_out=None, l2norm_group=0, out=None):
    """SiLU(causal_conv4(x @ W^T)) with optional conv history and per-group L2 norm.
    x [B,T,D] bf16; W [Dout,D] bf16; conv_w [Dout,4] bf16 -> [B,T,Dout] bf16."""
    _cuda_contig(x, "x", torch.bfloat16)
    _cuda_contig(W, "W", torch.bfloat16)
    _cuda_contig(conv_w, "conv_w", torch.bfloat16)
    B, T, D = x.shape
    Dout = W.shape[0]
    if out is None:
        out = torch.empty(B, T, Dout, dtype=torch.bfloat16, device=x.device)
    _lib.call("gdn_proj_conv_silu_fwd", _ptr(x), _ptr(W), _ptr(conv_w), _ptr(out), B, T, D, Dout,
              _ptr(conv_state_in), _ptr(conv_state_out), int(l2norm_group), _stream())
    return out


def proj_multi(x, segments):
    """Several projections of the same x [B,T,D] bf16 in one launch (gdn_proj_multi_fwd).
    ``segments``: up to 6 dicts with ``W`` [Dout, D] bf16 and optionally ``conv_w``
    [Dout, 4] (without it: a plain projection x @ W^T rounded to bf16),
    ``conv_state_in`` / ``conv_state_out`` [B, Dout, 3], ``l2norm_group`` and ``out``
    [B, T, Dout].  Returns the list of outputs, each as ``proj_conv_silu`` (or the
    plain projection) would give it."""
    _cuda_contig(x, "x", torch.bfloat16)
    _need(x.dim() == 3, "x must be [B, T, D]")
    B, T, D = x.shape
    segs = (_lib.ProjOutSeg * len(segments))()
    outs = []
    for i, sg in enumerate(segments):
        W = sg["W"]
        _cuda_contig(W, f"segments[{i}].W", torch.bfloat16)
        _need(W.dim() == 2 and W.shape[1] == D, f"segments[{i}].W must be [Dout, {D}]")
        Dout = W.shape[0]
        out = sg.get("out")
        if out is None:
            out = torch.empty(B, T, Dout, dtype=torch.bfloat16, device=x.device)
        _cuda_contig(out, f"segments[{i}].out", torch.bfloat16)
        cw = sg.get("conv_w")
        if cw is not None:
            _cuda_contig(cw, f"segments[{i}].conv_w", torch.bfloat16)
        segs[i].W, segs[i].y, segs[i].conv_w = _ptr(W), _ptr(out), _ptr(cw)
        segs[i].conv_state_in, segs[i].conv_state_out = _ptr(sg.get("conv_state_in")), _ptr(sg.get("conv_state_out"))
        segs[i].Dout, segs[i].l2norm_group = Dout, int(sg.get("l2norm_group", 0))
        outs.append(out)
    _lib.call("gdn_proj_multi_fwd", _ptr(x), B, T, D, segs, len(segments), _stream())
    return outs


def decode_proj(x, segments, *, norm_gamma=None, eps=1e-6):
    """Input projections of one decode step in one launch (gdn_decode_proj_fwd).

    x [B, D] bf16 (B <= 8); ``segments``: list of dicts with ``W`` [C, D] bf16 and
    optionally ``conv_w`` [C, 4], ``conv_state_in`` / ``conv_state_out`` [B, C, 3]
    (may be the same tensor: updated in place), ``l2_group`` and ``out`` [B, C].
    With ``norm_gamma`` x is RMS-normalised first.  Returns the list of outputs,
    each [B, C] bf16: SiLU(conv4) (L2-normalised per group when asked) for the
    segments with ``conv_w``, plain bf16(x W^T) rows for the others."""
    _cuda_contig(x, "x", torch.bfloat16)
    _need(x.dim() == 2, "x must be [B, D]")
    B, D = x.shape
    if norm_gamma is not None:
        _cuda_contig(norm_gamma, "norm_gamma", torch.bfloat16)
    segs = (_lib.ProjSegment * len(segments))()
    outs = []
    for i, sg in enumerate(segments):
        W = sg["W"]
        _cuda_contig(W, f"segments[{i}].W", torch.bfloat16)
        _need(W.shape[1] == D, f"segments[{i}].W must be [C, {D}]")
        C = W.shape[0]
        out = sg.get("out")
        if out is None:
            out = torch.empty(B, C, dtype=torch.bfloat16, device=x.device)
        _need(out.dtype == torch.bfloat16 and out.is_cuda and out.shape[-1] == C and out.stride(-1) == 1,
              f"segments[{i}].out must be bf16 [B, {C}] with unit inner stride")
        for name in ("conv_w", "conv_state_in", "conv_state_out"):
            if sg.get(name) is not None:
                _cuda_contig(sg[name], f"segments[{i}].{name}", torch.bfloat16)
        segs[i] = _lib.ProjSegment(_ptr(W), _ptr(out), _ptr(sg.get("conv_w")), _ptr(sg.get("conv_state_in")),
                                   _ptr(sg.get("conv_state_out")), C, out.stride(0) if B > 1 else C,
                                   int(sg.get("l2_group", 0)))
        outs.append(out)
    _lib.call("gdn_decode_proj_fwd", _ptr(x), _ptr(norm_gamma), float(eps), B, D, segs, len(segments), _stream())
    return outs


# ---------------------------------------------------------------------------
# reference-surface modules (drop-in for GDNLayerCustom's ``exts`` dict)
# ---------------------------------------------------------------------------


class PrefillModule:
    """``prefill(q,k,v,A_log,a,dt_bias,b_logits,mask,state_in,scale) -> (out, state_out)``
    with the argument meaning of kernels/prefill_chunked.cu:422-433 (q,k,v [B,H,T,*]
    bf16; a,b_logits [B,H,T] bf16; dt_bias float; mask [B,T] f32; state_in empty =
    zeros).  Shape-generic: H, dk in {64,128}, dv in {64,128,256}, any T."""

    # the reference layer's shapes (gdn_layer.py:24-28); C_DIM is the chunk length
    H_DIM = 16
    K_DIM = 128
    V_DIM = 256
    C_DIM = CHUNK

    def prefill(self, q, k, v, A_log, a, dt_bias, b_logits, mask, state_in, scale):
        for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b_logits", b_logits)):
            _need(t.is_cuda and t.is_contiguous() and t.dtype == torch.bfloat16,
                  f"{name}: contiguous bfloat16 CUDA required")
        s_in = state_in if (state_in is not None and state_in.numel() > 0) else None
        return prefill(q, k, v, A_log, a, b_logits, dt_bias=float(dt_bias), mask=mask, state_in=s_in,
                       scale=float(scale), layout="bhtd")


class DecodeModule:
    """``forward(q,k,v,a_sc,b_sc,A_log,dt_bias,S_in,scale,o_out,S_out) -> None``
    (kernels/decode.cu:172-214): q,k [B,H,K], v [B,H,V] bf16, a,b [B,H] bf16,
    A_log, dt_bias [H] f32, S_in/S_out [B,H,K,V] f32 (may alias), o_out [B,H,V] f32."""

    def forward(self, q, k, v, a_sc, b_sc, A_log, dt_bias, S_in, scale, o_out, S_out):
        for name, t in (("q", q), ("k", k), ("v", v), ("a_sc", a_sc), ("b_sc", b_sc), ("A_log", A_log),
                        ("dt_bias", dt_bias), ("S_in", S_in), ("o_out", o_out), ("S_out", S_out)):
            _need(t.is_cuda, f"{name} must be a CUDA tensor")
            _need(t.is_contiguous(), f"{name} must be contiguous")
        decode_step(q, k, v, a_sc, b_sc, A_log, dt_bias, S_in, scale=float(scale), out=o_out, state_out=S_out)


class ProjModule:
    """``forward(input [B,T,D], weight [D_out,D], conv_w [D_out,4]) -> [B,T,D_out]``
    bf16 (kernels/fused_proj_conv_silu.cu:298-355)."""

    def forward(self, input, weight, conv_w):
        _need(input.is_cuda and weight.is_cuda and conv_w.is_cuda, "all tensors must be on CUDA")
        _need(input.is_contiguous() and weight.is_contiguous() and conv_w.is_contiguous(),
              "all tensors must be contiguous")
        _need(input.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and conv_w.dtype == torch.bfloat16,
              "all tensors must be bfloat16")
        _need(weight.shape[1] == input.shape[2], "weight dim-1 must equal D")
        _need(conv_w.shape[0] == weight.shape[0], "conv_w dim-0 must equal D_out")
        _need(conv_w.shape[1] == 4, "conv_w dim-1 must equal CONV_K")
        return proj_conv_silu(input, weight, conv_w)


class RMSNormModule:
    """``forward(x [R,D] bf16, gamma [D] bf16, eps, block_threads, rows_per_block)``
    (kernels/rmsnorm.cu:280-293).  The launch-shape arguments are validated like the
    reference's (:133-144) and otherwise unused; any D % 8 == 0 up to 8192 works."""

    def forward(self, x, gamma, eps, block_threads, rows_per_block):
        _need(x.is_cuda, "x must be CUDA")
        _need(gamma.is_cuda, "gamma must be CUDA")
        _need(x.dtype == torch.bfloat16, "x must be BF16")
        _need(gamma.dtype == torch.bfloat16, "gamma must be BF16")
        _need(x.dim() == 2, "x must be [R, D]")
        _need(gamma.dim() == 1 and gamma.shape[0] == x.shape[1], "gamma must be [D]")
        _need(x.is_contiguous() and gamma.is_contiguous(), "inputs must be contiguous")
        _need(rows_per_block >= 1, "rows_per_block must be >= 1")
        _need(32 <= block_threads <= 1024, "block_threads must be in [32, 1024]")
        _need(block_threads % rows_per_block == 0, "block_threads must be divisible by rows_per_block")
        tpr = block_threads // rows_per_block
        _need(tpr >= 32 and tpr % 32 == 0, "threads_per_row must be a multiple of 32")
        return rmsnorm(x, gamma, float(eps))


def exts() -> dict:
    """The ``exts`` dict of gdn_layer.GDNLayerCustom (gdn_layer.py:209-217)."""
    _lib.lib()  # fail loudly now if the library is missing
    return dict(rmsnorm=RMSNormModule(), proj=ProjModule(), prefill=PrefillModule(), decode=DecodeModule())
