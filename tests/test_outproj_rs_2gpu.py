"""The fused head-sharded output projection across real GPUs: two processes,
one GPU each, NCCL for the two ordering all-reduces, CUDA IPC for the receive
buffers (every tile of the partial product is stored straight into the owning
GPU's memory over NVLink).  Each rank checks its rows against the unsharded
projection of the same seeded inputs (torch fp32), twice in a row so the
second call reuses the buffers.  Skipped on a box with fewer than two GPUs."""
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
    from gdn_18646_b200.sharding import PeerBuffer, owned_rows, sharded_out_proj
    M, N, K = 2048, 2048, 1024
    kr = K // world
    errs = []
    buf = PeerBuffer(M // world, N)
    try:
        for it in range(2):
            g = torch.Generator(device="cuda").manual_seed(100 + it)
            x = torch.randn(M, K, generator=g, device="cuda").bfloat16()
            W = (torch.randn(N, K, generator=g, device="cuda") * K ** -0.5).bfloat16()
            y = sharded_out_proj(x[:, rank * kr:(rank + 1) * kr].contiguous(),
                                 W[:, rank * kr:(rank + 1) * kr].contiguous(), buf)
            ref = (x.float() @ W.float().T)[owned_rows(M, rank, world)]
            torch.cuda.synchronize()
            errs.append(((y.float() - ref).abs().max() / ref.abs().max()).item())
    finally:
        buf.close()
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(" ".join(f"{e:.6e}" for e in errs))


def test_outproj_rs_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        errs = [float(e) for e in open(tmp_path / f"rank{r}.txt").read().split()]
        assert len(errs) == 2 and max(errs) <= 0.02, (r, errs)
