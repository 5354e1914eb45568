"""The Ulysses path on two B200s over NCCL: sequence-sharded Q/K/V move to
head sharding with one all-to-all, each rank runs the fused forward on its
heads, one all-to-all brings the output back.  Heads are independent, so the
result must equal the single-GPU forward of the whole tensors byte for byte.

Skipped unless two GPUs are visible (the single-GPU suite runs it as a skip)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import has_b200

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not has_b200() or torch.cuda.device_count() < 2, reason="needs two B200 GPUs")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path):
    import datetime

    from vc_attention_b200 import Config, sharding
    from vc_attention_b200.synthetic import make_qkv

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        q, k, v = make_qkv("c4", 9, heads=4, seq=2048)
        s = q.shape[2] // world
        tok = slice(rank * s, (rank + 1) * s)
        cfg = Config(v_smooth=True, expcast=True)
        out, _ = sharding.attention_seq_sharded(*(x[:, :, tok].contiguous().cuda() for x in (q, k, v)), cfg)
        torch.save(out.cpu(), os.path.join(path, f"out{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ulysses_two_gpus_equals_single_gpu(tmp_path):
    from vc_attention_b200 import Config, attention
    from vc_attention_b200.synthetic import make_qkv

    world = 2
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, start_method="spawn")
    q, k, v = make_qkv("c4", 9, heads=4, seq=2048)
    want, _ = attention(q.cuda(), k.cuda(), v.cuda(), Config(v_smooth=True, expcast=True))
    got = torch.cat([torch.load(tmp_path / f"out{r}.pt") for r in range(world)], dim=2)
    assert torch.equal(got, want.cpu())
