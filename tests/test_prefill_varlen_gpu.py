"""Variable-length prefill (gdn_prefill_varlen_fwd_ws): N sequences packed along
the token axis with cu_seqlens offsets.  Per sequence the result must be the
fixed-length prefill of that sequence alone -- bit for bit, since the rows a
sequence's last chunk reads past its end (the next sequence's tokens) enter
every product multiplied by exact zeros -- and the oracle's within the prefill
bar (bf16 o max-abs <= 2e-2, fp32 state relative Frobenius <= 1e-3).  Empty
sequences pass their state through; offsets that are inconsistent on the device
skip their sequence and are reported by gdn_check_device_error."""
import numpy as np
import pytest

from gdn_18646_b200 import _lib
from oracle import gdn_oracle as O
from tests._util import to_dev, to_np

pytestmark = pytest.mark.gpu

O_TOL = 2e-2
S_TOL = 1e-3


def _packed(lens, H, dk, dv, seed, Hqk=None, state_std=0.02):
    """Per-sequence oracle inputs (B = 1 each) and their packed concatenation."""
    Hqk = Hqk or H
    seqs = [O.make_prefill_inputs(seed + i, 1, max(L, 1), H, dk, dv, state_std=state_std, Hqk=Hqk)
            for i, L in enumerate(lens)]
    for s, L in zip(seqs, lens):                      # cut to the real length (0 allowed)
        s["q"], s["k"], s["v"] = s["q"][:, :, :L], s["k"][:, :, :L], s["v"][:, :, :L]
        s["a"], s["b"] = s["a"][:, :, :L], s["b"][:, :, :L]
        s["mask"] = s["mask"][:, :L]
    pack = dict(
        q=np.concatenate([s["q"][0].transpose(1, 0, 2) for s in seqs]),      # [Ttot, Hqk, dk]
        k=np.concatenate([s["k"][0].transpose(1, 0, 2) for s in seqs]),
        v=np.concatenate([s["v"][0].transpose(1, 0, 2) for s in seqs]),      # [Ttot, H, dv]
        a=np.concatenate([s["a"][0] for s in seqs], axis=1),                 # [H, Ttot]
        b=np.concatenate([s["b"][0] for s in seqs], axis=1),
        state_in=np.concatenate([s["state_in"] for s in seqs]),              # [N, H, dk, dv]
        cu=np.concatenate([[0], np.cumsum(lens)]).astype(np.int32))
    return seqs, pack


def _run_varlen(pack, A_log, scale):
    import torch
    from gdn_18646_b200 import ops
    o, s = ops.prefill_varlen(to_dev(pack["q"]), to_dev(pack["k"]), to_dev(pack["v"]), to_dev(A_log),
                              to_dev(pack["a"]), to_dev(pack["b"]), to_dev(pack["cu"]),
                              state_in=to_dev(pack["state_in"]), scale=scale)
    torch.cuda.synchronize()
    return o, s


def _run_single(seq, state_in):
    """The fixed-length prefill of one sequence, layout [1, T, H, D], single-launch schedule."""
    import torch
    from gdn_18646_b200 import ops
    q = to_dev(np.ascontiguousarray(seq["q"].transpose(0, 2, 1, 3)))
    k = to_dev(np.ascontiguousarray(seq["k"].transpose(0, 2, 1, 3)))
    v = to_dev(np.ascontiguousarray(seq["v"].transpose(0, 2, 1, 3)))
    o, s = ops.prefill(q, k, v, to_dev(seq["A_log"]), to_dev(seq["a"]), to_dev(seq["b"]),
                       state_in=to_dev(state_in), scale=seq["scale"], layout="bthd")
    torch.cuda.synchronize()
    return o[0], s[0]


@pytest.fixture
def single_schedule():
    lib = _lib.lib()
    lib.gdn_prefill_set_schedule(_lib.GDN_SCHEDULE_SINGLE)
    yield
    lib.gdn_prefill_set_schedule(_lib.GDN_SCHEDULE_AUTO)


@pytest.mark.parametrize("lens,H,Hqk,dk,dv", [
    ([1, 63, 64, 65, 200, 0, 1000, 128], 4, 4, 128, 128),
    ([300, 7, 129], 4, 2, 128, 128),                     # grouped value heads
    ([100, 64, 1, 250], 2, 2, 64, 64),
    ([130, 70], 2, 2, 128, 256),                         # two value tiles per head
])
def test_varlen_matches_each_sequence_alone(cuda_device, single_schedule, lens, H, Hqk, dk, dv):
    import torch
    seqs, pack = _packed(lens, H, dk, dv, seed=40 + sum(lens), Hqk=Hqk)
    o, s = _run_varlen(pack, seqs[0]["A_log"], seqs[0]["scale"])
    o_np, s_np = to_np(o), to_np(s)
    for i, (seq, L) in enumerate(zip(seqs, lens)):
        t0, t1 = pack["cu"][i], pack["cu"][i + 1]
        if L == 0:
            assert np.array_equal(s_np[i], pack["state_in"][i]), "an empty sequence passes its state through"
            continue
        o1, s1 = _run_single(seq, pack["state_in"][i:i + 1])
        assert np.array_equal(o_np[t0:t1], to_np(o1)), f"sequence {i}: o differs from the fixed-length prefill"
        assert np.array_equal(s_np[i], to_np(s1)), f"sequence {i}: state differs from the fixed-length prefill"
    assert torch.isfinite(o.float()).all()


def test_varlen_against_oracle(cuda_device):
    lens = [70, 1, 191, 64]
    seqs, pack = _packed(lens, 2, 128, 128, seed=7)
    o, s = _run_varlen(pack, seqs[0]["A_log"], seqs[0]["scale"])
    o_np, s_np = O.bf16_to_f32(to_np(o)), to_np(s)
    for i, seq in enumerate(seqs):
        t0, t1 = pack["cu"][i], pack["cu"][i + 1]
        o_r, s_r = O.prefill(seq["q"], seq["k"], seq["v"], seq["A_log"], seq["a"], seq["dt_bias"], seq["b"],
                             seq["mask"], state_in=seq["state_in"], scale=float(seq["scale"]), chunk_size=64,
                             dt=np.float64)
        assert float(np.abs(o_np[t0:t1] - o_r[0].transpose(1, 0, 2)).max()) <= O_TOL
        assert O.rel_fro(s_np[i], s_r[0]) <= S_TOL


def test_varlen_device_checks_offsets(cuda_device):
    """Offsets that decrease or pass Ttot skip their sequence (its outputs are not
    written, its state is passed through) and are reported after the call."""
    import torch
    lens = [100, 50, 50]
    seqs, pack = _packed(lens, 2, 128, 128, seed=3)
    pack["cu"] = np.array([0, 100, 90, 250], dtype=np.int32)       # sequence 1 decreases, 2 ends past Ttot
    lib = _lib.lib()
    assert lib.gdn_check_device_error() == _lib.GDN_OK
    o, s = _run_varlen(pack, seqs[0]["A_log"], seqs[0]["scale"])
    assert lib.gdn_check_device_error() == _lib.GDN_ERR_SHAPE
    assert "cu_seqlens" in _lib.last_error()
    assert lib.gdn_check_device_error() == _lib.GDN_OK             # the word was cleared
    assert np.array_equal(to_np(s)[1], pack["state_in"][1])
    assert np.array_equal(to_np(s)[2], pack["state_in"][2])
    assert torch.isfinite(s).all()


def test_varlen_streamed_schedule_equals_single(cuda_device):
    """The streamed schedule (prep workers and chain CTAs in one launch, records
    chunk-major behind ready flags) gives the single schedule's bits for packed
    sequences too, including a sequence whose prep tasks end early."""
    lib = _lib.lib()
    lens = [700, 5, 64, 1300, 0, 90]
    seqs, pack = _packed(lens, 4, 128, 128, seed=17)
    res = []
    for mode in (_lib.GDN_SCHEDULE_STREAM, _lib.GDN_SCHEDULE_SINGLE):
        lib.gdn_prefill_set_schedule(mode)
        try:
            res.append([to_np(t) for t in _run_varlen(pack, seqs[0]["A_log"], seqs[0]["scale"])])
        finally:
            lib.gdn_prefill_set_schedule(_lib.GDN_SCHEDULE_AUTO)
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])
