"""Generate golden vectors by running the REFERENCE's own PyTorch functions.

Run here (where the reference checkout is mounted) with

    python tests/golden/make_golden.py /path/to/GDN_18646

It imports ``reference/prefill_ref.py``, ``reference/decode_ref.py``,
``reference/fused_proj_conv_silu_ref.py`` and ``reference/rmsnorm_ref.py``
from that checkout, feeds them seeded inputs (generated with the oracle's
helpers so the same distributions are used everywhere) on the CPU, and writes
one ``.npz`` per case next to this script.  bf16 arrays are stored as uint16
bit patterns.  Nothing at test time reads the reference checkout: the tests
only read the committed ``.npz`` files.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import gdn_oracle as O  # noqa: E402


def t_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def t_f32(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))


def gate_tensor(x):
    x = np.asarray(x)
    return t_bf16(x) if x.dtype == np.uint16 else t_f32(x)


def np_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    clean = {k: np.asarray(v) for k, v in arrays.items() if v is not None}
    np.savez_compressed(path, **clean)
    print(f"wrote {path} ({os.path.getsize(path)} B)")


def prefill_case(name, ref_prefill, inp, chunk, *, scale=None, Hqk_expand=None):
    q, k = inp["q"], inp["k"]
    H = inp["v"].shape[1]
    if Hqk_expand:
        qx, kx = O.expand_qk_heads(q, H), O.expand_qk_heads(k, H)
    else:
        qx, kx = q, k
    sc = inp["scale"] if scale is None else scale
    o, S = ref_prefill(
        t_bf16(qx), t_bf16(kx), t_bf16(inp["v"]), t_f32(inp["A_log"]),
        gate_tensor(inp["a"]), torch.tensor(float(inp["dt_bias"])), gate_tensor(inp["b"]),
        t_f32(inp["mask"]),
        state_in=None if inp["state_in"] is None else t_f32(inp["state_in"]),
        scale=sc, chunk_size=chunk)
    save(name, q=q, k=k, v=inp["v"], a=inp["a"], b=inp["b"], A_log=inp["A_log"],
         dt_bias=np.float32(inp["dt_bias"]), mask=inp["mask"], state_in=inp["state_in"],
         scale=np.float32(sc), chunk=np.int32(chunk), o=o.float().numpy(), state_out=S.numpy())


def main(ref_root):
    sys.path.insert(0, ref_root)
    from reference.prefill_ref import ref_prefill
    from reference.decode_ref import ref_decode
    from reference.fused_proj_conv_silu_ref import ref_proj_conv_silu
    from reference.rmsnorm_ref import ref_rmsnorm

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # config 0 exactly: B=1 T=256 H=2 dk=dv=64, chunk 64, zero state
    prefill_case("prefill_config0", ref_prefill, O.make_prefill_inputs(100, 1, 256, 2, 64, 64), 64)
    # config 1 reduced (B, T, H), full head dims 128/128, fp32 gates, N(0,0.02) state
    prefill_case("prefill_config1_small", ref_prefill,
                 O.make_prefill_inputs(101, 1, 192, 2, 128, 128, gate_dtype="f32", state_std=0.02), 64)
    # mask != 1 (the oracle masks k_beta/v_beta/o but not the decay)
    inp = O.make_prefill_inputs(102, 2, 128, 2, 64, 64, state_std=0.02)
    rng = np.random.default_rng(7)
    inp["mask"] = (rng.random((2, 128)) > 0.3).astype(np.float32)
    prefill_case("prefill_mask", ref_prefill, inp, 64)
    # ragged length (T % 64 != 0: the reference pads the last chunk)
    prefill_case("prefill_ragged", ref_prefill,
                 O.make_prefill_inputs(103, 1, 100, 2, 64, 64, state_std=0.02), 64)
    # scale == 0 -> 1/sqrt(K)
    prefill_case("prefill_scale0", ref_prefill, O.make_prefill_inputs(104, 1, 64, 1, 64, 64), 64,
                 scale=0.0)
    # grouped value heads: 2 q/k heads shared by 4 value heads (config 3 uses 16/32)
    prefill_case("prefill_gva", ref_prefill,
                 O.make_prefill_inputs(105, 1, 128, 4, 64, 64, state_std=0.02, Hqk=2), 64,
                 Hqk_expand=True)
    # the reference's own test shape: H=16 dk=128 dv=256, unnormalised N/sqrt(dk)
    # inputs, A_log=0, scale=1 (tests/test_prefill.py:30-39); H reduced 16 -> 4 to keep the fixture small
    g = torch.Generator().manual_seed(106)
    B, Hh, T, dk, dv = 1, 4, 64, 128, 256
    qt = (torch.randn(B, Hh, T, dk, generator=g) * dk ** -0.5).bfloat16()
    kt = (torch.randn(B, Hh, T, dk, generator=g) * dk ** -0.5).bfloat16()
    vt = (torch.randn(B, Hh, T, dv, generator=g) * dk ** -0.5).bfloat16()
    at = torch.randn(B, Hh, T, generator=g).bfloat16()
    bt = torch.randn(B, Hh, T, generator=g).bfloat16()
    inp = dict(q=np_bits(qt), k=np_bits(kt), v=np_bits(vt), a=np_bits(at), b=np_bits(bt),
               A_log=np.zeros(Hh, np.float32), dt_bias=0.0, mask=np.ones((B, T), np.float32),
               state_in=None, scale=1.0)
    prefill_case("prefill_refshape", ref_prefill, inp, 64)

    # decode: config 2 reduced (B, H), full 128/128, N(0,0.02) state, 3 chained steps
    steps, S0, A_log, dtb = O.make_decode_inputs(200, 2, 2, 128, 128, steps=3)
    S = t_f32(S0)
    outs, states = [], []
    for st in steps:
        o, S = ref_decode(t_bf16(st["q"])[:, None], t_bf16(st["k"])[:, None],
                          t_bf16(st["v"])[:, None], S, t_f32(A_log),
                          t_bf16(st["a"])[:, None], t_f32(dtb), t_bf16(st["b"])[:, None],
                          1.0 / math.sqrt(128))
        outs.append(o.numpy())
        states.append(S.numpy())
    save("decode_config2_small", state_in=S0, A_log=A_log, dt_bias=dtb,
         q=np.stack([s["q"] for s in steps]), k=np.stack([s["k"] for s in steps]),
         v=np.stack([s["v"] for s in steps]), a=np.stack([s["a"] for s in steps]),
         b=np.stack([s["b"] for s in steps]), o=np.stack(outs), state_out=np.stack(states))
    # decode, the reference's own test shape (tests/test_decode.py:27-36): dv=256;
    # B, H reduced to keep the fixture small
    g = torch.Generator().manual_seed(201)
    B, Hh, dk, dv = 1, 4, 128, 256
    q = (torch.randn(B, 1, Hh, dk, generator=g) * 0.02).bfloat16()
    k = (torch.randn(B, 1, Hh, dk, generator=g) * 0.02).bfloat16()
    v = (torch.randn(B, 1, Hh, dv, generator=g) * 0.02).bfloat16()
    a = (torch.randn(B, 1, Hh, generator=g) * 0.1).bfloat16()
    b = (torch.randn(B, 1, Hh, generator=g) * 0.1).bfloat16()
    A0 = torch.zeros(Hh)
    d0 = torch.zeros(Hh)
    S_in = torch.randn(B, Hh, dk, dv, generator=g) * 0.01
    o, S1 = ref_decode(q, k, v, S_in, A0, a, d0, b, 1.0 / math.sqrt(dk))
    save("decode_refshape", q=np_bits(q[:, 0]), k=np_bits(k[:, 0]), v=np_bits(v[:, 0]),
         a=np_bits(a[:, 0]), b=np_bits(b[:, 0]), A_log=A0.numpy(), dt_bias=d0.numpy(),
         state_in=S_in.numpy(), o=o.numpy(), state_out=S1.numpy())

    # fused projection + causal conv + SiLU (D % 64 == 0, Dout % 128 == 0; T=1 edge)
    for name, (B, T, D, Dout, seed) in {"proj_small": (2, 67, 256, 128, 300),
                                         "proj_t1": (3, 1, 128, 256, 301)}.items():
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(B, T, D, generator=g).bfloat16()
        W = (torch.randn(Dout, D, generator=g) * D ** -0.5).bfloat16()
        cw = (torch.randn(Dout, 4, generator=g) * 0.5).bfloat16()
        y = ref_proj_conv_silu(x, W, cw)
        save(name, x=np_bits(x), W=np_bits(W), conv_w=np_bits(cw), y=np_bits(y))

    # RMSNorm (D=2048 as the reference kernel, plus a non-2048 width)
    for name, (R, D, seed) in {"rmsnorm_2048": (5, 2048, 400), "rmsnorm_512": (3, 512, 401)}.items():
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(R, D, generator=g).bfloat16()
        gamma = (1.0 + 0.1 * torch.randn(D, generator=g)).bfloat16()
        y = ref_rmsnorm(x, gamma, 1e-6)
        save(name, x=np_bits(x), gamma=np_bits(gamma), eps=np.float32(1e-6), y=np_bits(y))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout root>")
    main(sys.argv[1])
