"""Capture and replay of real post-RoPE Q/K/V (the reference's adapter
capture, lightx2v.py:92-125, and its replay, replay.py:80-96): which calls
are saved, the byte budget, the file's contents and identity, the 128-row
query slice against the full K/V; on a B200 a capture made through the
adapter replays against the CPU checker."""
import hashlib
import types

import numpy as np
import pytest
import torch

from conftest import has_b200
from vc_attention_b200 import error_report as er
from vc_attention_b200.lightx2v import CaptureOptions, ExperimentAdapter, capture


class FakeAttention:
    def __call__(self, q, k, v, cfg, *, cache, step, total_steps, request_id, layer_id, scale):
        return q * 2, {"smoothing_active": False, "layout_refreshed": False, "expcast": cfg.expcast}


def scheduler(step, steps, marker):
    return types.SimpleNamespace(step_index=step, infer_steps=steps, layout_cpu=marker)


def snd(seed, s=256, h=3, d=16):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(s, h, d, generator=g).to(torch.bfloat16) for _ in range(3)]


def test_adapter_captures_the_selected_calls(tmp_path, monkeypatch):
    monkeypatch.setenv("RANK", "0")
    opts = CaptureOptions(output_dir=str(tmp_path), steps=(0, 2), layers=(1,), heads=2, max_captures=3)
    adapter = ExperimentAdapter("combined", attention_fn=FakeAttention(), capture=opts)
    marker = object()
    inputs = {}
    for step in range(4):
        for layer in range(3):
            q, k, v = snd(10 * step + layer)
            inputs[(step, layer)] = (q, k, v)
            adapter.apply(q, k, v, scheduler=scheduler(step, 4, marker), block_idx=layer, softmax_scale=0.25)
    assert sorted(adapter.audit["captures"]) == ["rank0_step0_layer1", "rank0_step2_layer1"]
    for step in (0, 2):
        path = tmp_path / "captures" / f"rank0_step{step}_layer1.pt"
        q, k, v, source = er.load_capture(path)
        want = [x.transpose(0, 1).unsqueeze(0)[:, :2] for x in inputs[(step, 1)]]   # BNSD, first 2 heads
        assert all(torch.equal(a, b) for a, b in zip((q, k, v), want))
        meta = source["metadata"]
        assert meta["step"] == step and meta["total_steps"] == 4 and meta["layer"] == 1 and meta["rank"] == 0
        assert meta["scale"] == 0.25 and meta["full_shape"] == [1, 3, 256, 16] and meta["layout"] == "BNSD"
        assert meta["post_rope"] and meta["full_kv_context"] and meta["dtype"] == "torch.bfloat16"
        assert source["sha256"] == hashlib.sha256(path.read_bytes()).hexdigest()
    assert adapter.audit["capture_bytes"] == 2 * 3 * (2 * 256 * 16 * 2)


def test_capture_limits(tmp_path):
    q, k, v = (x.transpose(0, 1).unsqueeze(0) for x in snd(1))
    audit = {"captures": {}, "capture_bytes": 0}
    opts = CaptureOptions(output_dir=str(tmp_path), steps=(0, 1, 2), layers=(0,), max_captures=2)
    assert capture(opts, audit, q, k, v, step=0, steps=3, layer=0, scale=1.0, rank=1) is None   # other rank
    assert capture(opts, audit, q, k, v, step=0, steps=3, layer=5, scale=1.0, rank=0) is None   # layer not chosen
    assert capture(opts, audit, q, k, v, step=0, steps=3, layer=0, scale=1.0, rank=0) is not None
    assert capture(opts, audit, q, k, v, step=0, steps=3, layer=0, scale=1.0, rank=0) is None   # same key again
    assert capture(opts, audit, q, k, v, step=1, steps=3, layer=0, scale=1.0, rank=0) is not None
    assert capture(opts, audit, q, k, v, step=2, steps=3, layer=0, scale=1.0, rank=0) is None   # max_captures
    tight = CaptureOptions(output_dir=str(tmp_path), steps=(0,), layers=(0,), max_capture_mib=1)
    big = torch.zeros(1, 1, 1 << 20, 1, dtype=torch.bfloat16)       # 2 MiB per tensor
    with pytest.raises(ValueError, match="budget"):
        capture(tight, {"captures": {}, "capture_bytes": 0}, big, big, big, step=0, steps=1, layer=0, scale=1.0,
                rank=0)
    with pytest.raises(ValueError, match="positive"):
        CaptureOptions(output_dir=str(tmp_path), heads=0)


def test_query_slice_keeps_block_boundaries():
    q = torch.zeros(1, 2, 1000, 8)
    assert er.query_slice(q, 128, 0).shape[2] == 872
    assert er.query_slice(q, 256, 128).shape[2] == 128
    assert er.query_slice(q, 896, 500).shape[2] == 104
    for bad in (64, 1024, -128):
        with pytest.raises(ValueError, match="block boundary"):
            er.query_slice(q, bad, 0)
    with pytest.raises(SystemExit):
        er.main(["--capture", "missing.pt", "--q-start", "100"])


@pytest.mark.gpu
@pytest.mark.skipif(not has_b200(), reason="needs a B200")
def test_capture_through_the_adapter_replays_against_the_checker(tmp_path, monkeypatch):
    """A capture taken by the adapter around the real B200 attention replays
    (error_report --capture) with its own scale and step, and the native
    output of the query slice matches the CPU checker within the tolerance."""
    from oracle import oracle as O
    from vc_attention_b200 import Config, attention
    from vc_attention_b200.synthetic import make_qkv

    monkeypatch.setenv("RANK", "0")
    q, k, v = make_qkv("c3", 7, heads=3, seq=2048)                      # BNSD bf16
    opts = CaptureOptions(output_dir=str(tmp_path), steps=(0,), layers=(4,), heads=2)
    adapter = ExperimentAdapter("combined", capture=opts)
    snd_in = [x[0].transpose(0, 1).contiguous().cuda() for x in (q, k, v)]
    adapter.apply(*snd_in, scheduler=scheduler(0, 8, object()), block_idx=4, softmax_scale=0.1)
    path = tmp_path / "captures" / "rank0_step0_layer4.pt"
    res = er.replay(path, q_start=512, q_limit=256, rows=32)
    assert res["q_rows"] == 256 and res["kv_tokens"] == 2048 and res["source"]["metadata"]["scale"] == 0.1
    for mode, entry in res["modes"].items():
        assert entry["native_vs_fp32"]["cosine"] > 0.99, (mode, entry)
    cq, ck, cv, _ = er.load_capture(path)
    cq = er.query_slice(cq, 512, 256)
    for smooth, cast in ((False, True), (True, True)):
        cfg = Config(v_smooth=smooth, expcast=cast)
        got, _ = attention(cq.cuda(), ck.cuda(), cv.cuda(), cfg, step=0, total_steps=8, scale=0.1)
        pi = None
        if smooth:
            pi, _, _ = O.group_values(cv[0].float().numpy(), clusters=8, iterations=2)
        ref = O.attention(cq[0].float().numpy(), ck[0].float().numpy(), cv[0].float().numpy(), expcast=cast,
                          active=smooth, pi=pi, scale=0.1)
        ref = torch.from_numpy(np.ascontiguousarray(ref)).to(torch.bfloat16).float().numpy()
        m = O.metrics(got[0].float().cpu().numpy(), ref)
        assert m["relative_rmse"] <= 1e-3 and m["cosine"] >= 0.9999, (smooth, cast, m)
