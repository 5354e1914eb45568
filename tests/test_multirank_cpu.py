"""The N>1 path on CPU: head partitioning, the Ulysses all-to-alls and the
max-over-ranks timing, as world_size-2 gloo ranks.

Heads are independent, so a head-sharded forward must give the same bytes
as the unsharded one.  The per-head compute here is the CPU checker (the
GPU path needs a B200); what is under test is the partition and the data
movement around it."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vc_attention_b200 import sharding


@pytest.mark.parametrize("heads,world", [(40, 1), (40, 2), (40, 8), (24, 8), (7, 3), (2, 4), (0, 2)])
def test_head_ranges_cover_every_head_once(heads, world):
    ranges = [sharding.head_range(heads, world, r) for r in range(world)]
    covered = [h for a, b in ranges for h in range(a, b)]
    assert covered == list(range(heads))
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_head_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharding.head_range(40, 2, 2)
    with pytest.raises(ValueError):
        sharding.head_range(40, 0, 0)


def test_max_over_ranks_without_a_group_is_identity():
    assert sharding.max_over_ranks(3.5) == 3.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_inputs():
    g = torch.Generator().manual_seed(7)
    b, h, s, d = 1, 4, 512, 128
    q = torch.randn(b, h, s, d, generator=g) / d ** 0.5
    k = torch.randn(b, h, s, d, generator=g) / d ** 0.5 + torch.randn(b, h, 1, d, generator=g) * 1.5
    v = torch.randn(b, h, 8, d, generator=g)[:, :, torch.randint(0, 8, (s,), generator=g)] \
        + 0.3 * torch.randn(b, h, s, d, generator=g)
    return q, k, v


def _oracle_forward(q, k, v):
    """[B, H, S, D] float32 -> [B, H, S, D]: the CPU checker per head."""
    from oracle import oracle as O
    b, h, s, d = q.shape
    flat = [x.reshape(b * h, s, d).numpy() for x in (q, k, v)]
    pi, _, _ = O.group_values(flat[2], clusters=8, iterations=2)
    out = O.attention(flat[0], flat[1], flat[2], expcast=True, active=True, pi=pi)
    return torch.from_numpy(out).reshape(b, h, s, -1)


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _full_inputs()
        s = q.shape[2] // world
        tok = slice(rank * s, (rank + 1) * s)
        # sequence-sharded inputs -> head-sharded
        qh, kh, vh = (sharding.seq_to_heads(t[:, :, tok].contiguous()) for t in (q, k, v))
        a, b = sharding.head_range(q.shape[1], world, rank)
        for got, full in zip((qh, kh, vh), (q, k, v)):
            assert torch.equal(got, full[:, a:b])
            assert torch.equal(sharding.shard_heads(full, world, rank), got)
        # round trip back to sequence sharding
        assert torch.equal(sharding.heads_to_seq(qh), q[:, :, tok])
        # head-sharded forward, then back: equal to the unsharded forward
        out_local = sharding.heads_to_seq(_oracle_forward(qh, kh, vh))
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out_local.numpy())
        # slowest rank wins
        assert sharding.max_over_ranks(float(10 + rank)) == float(10 + world - 1)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_ulysses_and_head_sharded_forward(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    q, k, v = _full_inputs()
    want = _oracle_forward(q, k, v).numpy()
    s = q.shape[2] // world
    for r in range(world):
        got = np.load(tmp_path / f"out{r}.npy")
        assert np.array_equal(got, want[:, :, r * s:(r + 1) * s])
