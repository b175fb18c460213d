"""Shared helpers for the parity tests (numpy oracle <-> torch CUDA tensors)."""
import os

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def to_dev(x, device="cuda"):
    """numpy -> torch on device; uint16 arrays are bf16 bit patterns."""
    import torch
    x = np.ascontiguousarray(x)
    if x.dtype == np.uint16:
        return torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(x).to(device)


def to_np(t):
    """torch -> numpy; bf16 -> uint16 bit patterns, others unchanged."""
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def bf16_f32(x):
    from oracle.gdn_oracle import bf16_to_f32
    return bf16_to_f32(x) if x.dtype == np.uint16 else x


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(bf16_f32(a), np.float64) - np.asarray(bf16_f32(b), np.float64))))


def ref_tol_ok(got, want, atol, rtol):
    """The reference harness's mixed tolerance |got - want| < atol + rtol*|want|
    (tests/test_prefill.py:61-62, bench_gdn.py:66-70)."""
    g = np.asarray(bf16_f32(got), np.float64)
    w = np.asarray(bf16_f32(want), np.float64)
    return bool(np.all(np.abs(g - w) < atol + rtol * np.abs(w)))
