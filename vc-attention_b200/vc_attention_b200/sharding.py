"""Multi-GPU partitioning of the forward: heads are independent.

Every (batch, head) pair is a separate attention problem: the K channel mean,
the Lloyd clustering, the quantisation scales and the online softmax are all
per head (reference: src/vc_attention/core.py:96, :138-163, :125-135;
csrc/kernels.cu:313 loops heads outermost).  N ranks therefore take
contiguous head ranges and run the forward with no collective on the data
path.

Inputs that arrive sequence-sharded (every rank holds S/N tokens of all heads,
the layout of the reference's LightX2V sequence-parallel path,
src/vc_attention/lightx2v.py:119 and :138-139) move to head sharding with one
all-to-all before the forward and back with one after it (Ulysses).  The
all-to-alls go through ``torch.distributed`` (NCCL over NVLink on B200, gloo
on CPU).
"""
from __future__ import annotations

import torch


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous head range [start, stop) of ``rank``; the first
    ``heads % world`` ranks take one extra head."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is outside a world of {world}")
    if heads < 0:
        raise ValueError("heads must be non-negative")
    base, extra = divmod(heads, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's heads of a BNSD tensor, contiguous."""
    start, stop = head_range(x.shape[1], world, rank)
    return x[:, start:stop].contiguous()


def _world(group):
    return torch.distributed.get_world_size(group)


def max_over_ranks(x: float, group=None) -> float:
    """The largest ``x`` over the ranks of ``group`` (x itself without a
    process group).  Multi-GPU times are reported this way: the job takes as
    long as its slowest rank."""
    if not torch.distributed.is_available() or not torch.distributed.is_initialized():
        return x
    backend = torch.distributed.get_backend(group)
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
    return float(t.item())


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, H, S/N, D] (this rank's token chunk, all heads) -> [B, H/N, S, D]
    (this rank's heads, all tokens in rank order).  H must divide by N."""
    n = _world(group)
    b, h, s, d = x.shape
    if h % n:
        raise ValueError(f"{h} heads do not split evenly over {n} ranks")
    send = x.reshape(b, n, h // n, s, d).transpose(0, 1).contiguous()     # chunk r -> rank r
    recv = torch.empty_like(send)                                          # chunk r <- rank r's tokens
    torch.distributed.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 2, 0, 3, 4).reshape(b, h // n, n * s, d)


def heads_to_seq(o: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of :func:`seq_to_heads`: [B, H/N, S, Dv] -> [B, H, S/N, Dv]."""
    n = _world(group)
    b, hl, s_full, d = o.shape
    if s_full % n:
        raise ValueError(f"{s_full} tokens do not split evenly over {n} ranks")
    s = s_full // n
    send = o.reshape(b, hl, n, s, d).permute(2, 0, 1, 3, 4).contiguous()   # token chunk r -> rank r
    recv = torch.empty_like(send)                                          # head group r <- rank r
    torch.distributed.all_to_all_single(recv, send, group=group)
    return recv.transpose(0, 1).reshape(b, n * hl, s, d)


def attention_seq_sharded(q, k, v, config=None, *, cache=None, group=None, **kwargs):
    """Attention on sequence-sharded inputs ([B, H, S/N, D] per rank): one
    all-to-all to head sharding, the local forward on H/N heads over all S
    tokens, one all-to-all back.  Returns this rank's [B, H, S/N, Dv] output
    and the local stats."""
    from .core import attention

    qh, kh, vh = (seq_to_heads(t, group) for t in (q, k, v))
    out, stats = attention(qh, kh, vh, config, cache=cache, **kwargs)
    return heads_to_seq(out, group), stats
