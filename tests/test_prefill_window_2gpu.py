"""Head-sharded prefill with the all-gather of o overlapped window by window
(sharding.WindowedHeadGather) across two real GPUs: each rank runs its half of
the value heads through chained windows whose o lands in its slot of a gathered
buffer, and pulls each window of the peer's slot over NVLink (copy-engine
transfers from the CUDA IPC mapping) while the next window computes.  Every
rank's gathered buffer must equal, bit for bit, the per-rank whole-sequence
prefill followed by an NCCL all-gather; twice in a row (the second call reuses
the buffers), for both layouts.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from gdn_18646_b200 import ops
    from gdn_18646_b200.sharding import WindowedHeadGather
    B, T, H, d = 2, 1000, 8, 128
    Hs = H // world
    results = []
    try:
        for layout in ("bhtd", "bthd"):
            gath = WindowedHeadGather(B, T, Hs, d, layout=layout)
            try:
                for it in range(2):
                    g = torch.Generator(device="cuda").manual_seed(1000 * rank + 10 * it + (layout == "bthd"))
                    shp = (B, Hs, T, d) if layout == "bhtd" else (B, T, Hs, d)
                    q = torch.nn.functional.normalize(torch.randn(shp, generator=g, device="cuda"), dim=-1).bfloat16()
                    k = torch.nn.functional.normalize(torch.randn(shp, generator=g, device="cuda"), dim=-1).bfloat16()
                    v = torch.randn(shp, generator=g, device="cuda").bfloat16()
                    a = torch.randn(B, Hs, T, generator=g, device="cuda")
                    b = torch.randn(B, Hs, T, generator=g, device="cuda")
                    A_log = torch.full((Hs,), -2.3, device="cuda")
                    s0 = torch.randn(B, Hs, d, d, generator=g, device="cuda") * 0.02
                    want_o, want_s = ops.prefill(q, k, v, A_log, a, b, state_in=s0, layout=layout)
                    want = torch.empty((world,) + tuple(want_o.shape), dtype=want_o.dtype, device="cuda")
                    dist.all_gather_into_tensor(want, want_o)
                    got, got_s = gath.prefill(q, k, v, A_log, a, b, state_in=s0, window_tokens=256)
                    torch.cuda.synchronize()
                    results.append(bool(torch.equal(got, want)) and bool(torch.equal(got_s, want_s)))
            finally:
                gath.close()
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(" ".join(str(int(r)) for r in results))


def test_windowed_gather_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        res = open(tmp_path / f"rank{r}.txt").read().split()
        assert res == ["1"] * 4, (r, res)
