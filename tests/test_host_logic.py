"""Host-side logic of the b200_fp8 backend on CPU: Config contract, the
LayoutCache step schedule (checked against the sequence recorded from the
reference, tests/golden/schedule.json) and the no-fallback rules."""
import json
import pathlib

import pytest
import torch

import cases
from vc_attention_b200 import Config, LayoutCache, attention, core

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.fixture
def cpu_grouping(monkeypatch):
    """The schedule logic is host code; swap the GPU clustering for a stub
    that returns a fresh identity permutation, so `pi is` checks still work."""
    calls = []

    def fake(v, *, clusters, iterations, centers=None):
        calls.append(centers is None)
        b, h, s, d = v.shape
        return torch.arange(s).expand(b, h, s).clone(), torch.zeros(b, h, min(clusters, s), d)

    monkeypatch.setattr(core, "group_values", fake)
    return calls


def test_schedule_matches_reference_recording(cpu_grouping):
    records = json.loads((GOLDEN / "schedule.json").read_text())
    cache = LayoutCache(Config(v_smooth=True))
    base_v = cases.clustered_values(tokens=64, heads=1, dim=8)
    last_pi = None
    for rec, (request, step, total, trim) in zip(records, cases.schedule_script()):
        v = base_v[:, :, : base_v.shape[2] - trim]
        pi, active, refreshed = cache.layout(v, step=step, total_steps=total, request_id=request, layer_id=0)
        got = {"active": bool(active), "refreshed": bool(refreshed), "has_pi": pi is not None,
               "same_pi_as_previous": bool(pi is not None and pi is last_pi), "entries": cache.entries}
        assert got == {k: rec[k] for k in got}, (rec, got)
        last_pi = pi


def test_refresh_warm_starts_from_cached_centres(cpu_grouping):
    cache = LayoutCache(Config(v_smooth=True))
    v = torch.zeros(1, 1, 16, 4)
    for step in range(0, 13):
        cache.layout(v, step=step, total_steps=50, request_id="r", layer_id=3)
    # refreshes at 0, 4, 8, 12: cold start first, warm starts afterwards
    assert cpu_grouping == [True, False, False, False]


def test_window_is_ceil_of_active_fraction(cpu_grouping):
    cache = LayoutCache(Config(v_smooth=True))
    v = torch.zeros(1, 1, 16, 4)
    actives = [cache.layout(v, step=s, total_steps=50, request_id="r", layer_id=0)[1] for s in range(50)]
    assert actives == [s < 13 for s in range(50)]


def test_snapshot_restores_state(cpu_grouping):
    cache = LayoutCache(Config(v_smooth=True))
    v = torch.zeros(1, 1, 16, 4)
    cache.layout(v, step=0, total_steps=50, request_id="a", layer_id=0)
    snap = cache._snapshot(0)
    cache.layout(v, step=0, total_steps=50, request_id="b", layer_id=0)
    cache._restore(snap, 0)
    assert cache._request_id == "a" and cache._states[0]["refresh_step"] == 0


@pytest.mark.parametrize("kwargs", [
    {"kv_block": 0}, {"clusters": -1}, {"active_fraction": float("nan")}, {"backend": "automatic"},
    {"backend": "reference"}, {"quantize": False}, {"q_block": 7}, {"kv_block": 64}, {"q_block": 512},
    {"k_quant_block": 8192}, {"k_quant_block": 192}, {"clusters": 33}, {"mean_dtype": "int8"},
    {"k_smooth": 1}, {"iterations": True},
])
def test_config_rejects_invalid_contract(kwargs):
    with pytest.raises(ValueError):
        Config(**kwargs)


def test_config_accepts_reference_defaults():
    cfg = Config()
    assert (cfg.q_block, cfg.k_quant_block, cfg.kv_block, cfg.clusters, cfg.iterations) == (128, 256, 128, 8, 2)
    Config(q_block=64, k_quant_block=512, mean_dtype="bfloat16", v_smooth=True, expcast=True)


def test_rejects_cpu_tensors_without_fallback():
    x = torch.ones(1, 1, 3, 16)
    with pytest.raises(ValueError, match="requires CUDA"):
        attention(x, x, x, Config())


def test_unsupported_semantics_fail_explicitly():
    q, k, v = cases.reference_test_inputs((1, 2, 19, 35, 16, 16))
    with pytest.raises(ValueError, match="causal"):
        attention(q, k, v, Config(), causal=True)
    with pytest.raises(ValueError, match="mask"):
        attention(q, k, v, Config(), mask=torch.ones(19, 35))
    with pytest.raises(ValueError, match="heads"):
        attention(q, k[:, :1], v[:, :1], Config())
    with pytest.raises(ValueError, match="Empty"):
        attention(q[:, :, :0], k, v, Config())
    with pytest.raises(ValueError, match="FP16/BF16/FP32"):
        attention(q.double(), k.double(), v.double(), Config())


def test_layout_requires_request_id_and_valid_steps(cpu_grouping):
    cache = LayoutCache(Config(v_smooth=True))
    v = torch.zeros(1, 1, 8, 4)
    with pytest.raises(ValueError, match="request_id"):
        cache.layout(v, step=0, total_steps=4, request_id=None, layer_id=0)
    with pytest.raises(ValueError, match="step"):
        cache.layout(v, step=4, total_steps=4, request_id="r", layer_id=0)


def test_peek_predicts_layout_without_changing_the_cache(cpu_grouping):
    """LayoutCache.peek gives layout()'s decision for the same call (active,
    refresh, and the cached pi exactly when it would be reused) over the
    recorded schedule script, including the reversed step, the new request and
    the changed shape, and clusters nothing and changes nothing itself."""
    cache = LayoutCache(Config(v_smooth=True))
    base_v = cases.clustered_values(tokens=64, heads=1, dim=8)
    reused = 0
    for request, step, total, trim in cases.schedule_script():
        v = base_v[:, :, : base_v.shape[2] - trim]
        calls, rid, states = len(cpu_grouping), cache._request_id, dict(cache._states)
        fields = {k: dict(s) for k, s in states.items()}
        pi_p, active_p, refresh_p = cache.peek(v, step=step, total_steps=total, request_id=request, layer_id=0)
        assert len(cpu_grouping) == calls and cache._request_id == rid and cache._states == states
        assert all(dict(cache._states[k]) == f for k, f in fields.items())
        pi, active, refresh = cache.layout(v, step=step, total_steps=total, request_id=request, layer_id=0)
        assert (active_p, refresh_p) == (active, refresh), (request, step)
        if active and not refresh:
            assert pi_p is pi
            reused += 1
        else:
            assert pi_p is None
    assert reused > 0
    with pytest.raises(ValueError, match="request_id"):
        cache.peek(base_v, step=0, total_steps=1, request_id=None, layer_id=0)
    with pytest.raises(ValueError, match="step"):
        cache.peek(base_v, step=3, total_steps=3, request_id="a", layer_id=0)


def test_kv_order_must_be_known():
    q, k, v = cases.reference_test_inputs((1, 2, 19, 35, 16, 16))
    with pytest.raises(ValueError, match="kv_order"):
        attention(q, k, v, Config(), kv_order="sorted")


def test_to_layout_order_gathers_rows_through_pi():
    x = torch.arange(2 * 3 * 5 * 4, dtype=torch.float32).reshape(2, 3, 5, 4)
    pi = torch.stack([torch.randperm(5, generator=torch.Generator().manual_seed(i)) for i in range(6)])
    pi = pi.reshape(2, 3, 5).to(torch.int32)
    from vc_attention_b200 import to_layout_order
    y = to_layout_order(x, pi)
    for b in range(2):
        for h in range(3):
            for r in range(5):
                assert torch.equal(y[b, h, r], x[b, h, int(pi[b, h, r])])
