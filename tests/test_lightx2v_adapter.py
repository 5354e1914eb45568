"""The LightX2V attention adapter: call-layout checks, cache generations,
(layer, step) order, audit counters and the config patch, as in the
reference's src/vc_attention/lightx2v.py (host logic, a stand-in attention on
CPU); and on a B200 the adapter's output against a direct ``attention`` call."""
import json
import types

import pytest
import torch

from conftest import has_b200
from vc_attention_b200 import lightx2v
from vc_attention_b200.lightx2v import ExperimentAdapter, configure, validate_layout


class FakeAttention:
    """Records each call and returns a recognisable output: q scaled by 2,
    with the stats keys the adapter reads."""

    def __init__(self, smoothing=True, refreshed=False):
        self.calls = []
        self.smoothing, self.refreshed = smoothing, refreshed

    def __call__(self, q, k, v, cfg, *, cache, step, total_steps, request_id, layer_id, scale):
        self.calls.append(dict(shape=tuple(q.shape), step=step, total_steps=total_steps, request_id=request_id,
                               layer_id=layer_id, scale=scale, cache=cache))
        return q * 2, {"smoothing_active": self.smoothing, "layout_refreshed": self.refreshed,
                       "expcast": cfg.expcast}


def scheduler(step, steps=8, marker=None):
    return types.SimpleNamespace(step_index=step, infer_steps=steps, layout_cpu=marker if marker is not None else object())


def qkv(s=6, h=3, d=4, batch_dim=False):
    shape = (1, s, h, d) if batch_dim else (s, h, d)
    g = torch.Generator().manual_seed(0)
    return [torch.randn(shape, generator=g) for _ in range(3)]


def test_validate_layout_returns_bnsd_views():
    q, k, v = qkv()
    for args in ((q, k, v), [x.unsqueeze(0) for x in (q, k, v)]):
        out = validate_layout(*args, None, None, None, None, {})
        assert [tuple(x.shape) for x in out] == [(1, 3, 6, 4)] * 3
        assert torch.equal(out[0][0, 1], q[:, 1])
    cu = torch.tensor([0, 6], dtype=torch.int32)
    validate_layout(q, k, v, cu, cu, 6, 6, {"causal": False, "dropout": 0, "mask": None})


@pytest.mark.parametrize("kwargs, message", [
    ({"window": 4}, "Unknown attention options"),
    ({"causal": True}, "noncausal"),
    ({"dropout": 0.1}, "dropout"),
    ({"mask": torch.ones(1)}, "mask is unsupported"),
    ({"attn_mask": torch.ones(1)}, "attn_mask is unsupported"),
    ({"pse": torch.ones(1)}, "pse is unsupported"),
])
def test_validate_layout_refuses_options(kwargs, message):
    q, k, v = qkv()
    with pytest.raises(ValueError, match=message):
        validate_layout(q, k, v, None, None, None, None, kwargs)


def test_validate_layout_refuses_packed_and_mismatched():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="packed"):
        validate_layout(q, k, v, torch.tensor([0, 3, 6]), None, None, None, {})
    with pytest.raises(ValueError, match="max_seqlen"):
        validate_layout(q, k, v, None, None, 5, None, {})
    with pytest.raises(ValueError, match="equal Q/K/V"):
        validate_layout(q, k[:5], v, None, None, None, None, {})
    with pytest.raises(ValueError, match="SND or 1SND"):
        validate_layout(q[None, None], k[None, None], v[None, None], None, None, None, None, {})


def test_apply_layout_scale_and_audit():
    fake = FakeAttention(smoothing=True, refreshed=True)
    adapter = ExperimentAdapter("combined", attention_fn=fake)
    q, k, v = qkv()
    out = adapter.apply(q, k, v, scheduler=scheduler(0), block_idx=0)
    # [S, H*D] with each head's rows in place: the fake doubles q
    assert out.shape == (6, 12) and torch.equal(out, (q * 2).reshape(6, 12))
    call = fake.calls[0]
    assert call["shape"] == (1, 3, 6, 4) and call["scale"] == 4 ** -0.5 and call["total_steps"] == 8
    assert adapter.vc_config.v_smooth and adapter.vc_config.expcast
    adapter.apply(q, k, v, scheduler=scheduler(0), block_idx=1, softmax_scale=0.3)
    assert fake.calls[1]["scale"] == 0.3
    assert adapter.audit["calls"] == 2 and adapter.audit["smoothing_calls"] == 2
    assert adapter.audit["regroup_calls"] == 2 and adapter.audit["expcast_calls"] == 2


def test_generations_and_step_order():
    fake = FakeAttention()
    adapter = ExperimentAdapter("v_smooth", attention_fn=fake)
    q, k, v = qkv()
    marker = object()
    for step in range(3):
        for layer in range(2):
            adapter.apply(q, k, v, scheduler=scheduler(step, marker=marker), block_idx=layer)
    assert {c["request_id"] for c in fake.calls} == {1}
    # the same layer again at an earlier or equal step is refused
    with pytest.raises(ValueError, match="repeated or reversed"):
        adapter.apply(q, k, v, scheduler=scheduler(2, marker=marker), block_idx=0)
    # step 0 of a layer seen before starts a new generation (and resets the cache)
    adapter.cache._states[("x",)] = {"sentinel": True}
    adapter.apply(q, k, v, scheduler=scheduler(0, marker=marker), block_idx=0)
    assert fake.calls[-1]["request_id"] == 2 and ("x",) not in adapter.cache._states
    # a new layout marker starts a new generation at any step
    adapter.apply(q, k, v, scheduler=scheduler(5, marker=object()), block_idx=1)
    assert fake.calls[-1]["request_id"] == 3


def test_apply_requires_scheduler_and_marker():
    adapter = ExperimentAdapter("expcast", attention_fn=FakeAttention())
    q, k, v = qkv()
    with pytest.raises(ValueError, match="scheduler and block_idx"):
        adapter.apply(q, k, v, block_idx=0)
    with pytest.raises(ValueError, match="layout_cpu"):
        adapter.apply(q, k, v, scheduler=types.SimpleNamespace(step_index=0, infer_steps=4), block_idx=0)
    with pytest.raises(ValueError, match="mode"):
        ExperimentAdapter("fp16")


@pytest.mark.parametrize("patch, message", [
    ({"use_compile": True}, "use_compile"),
    ({"warmup": True}, "warmup"),
    ({"parallel": {"seq_p_head_parallel": True}}, "head_parallel"),
    ({"parallel": {"seq_p_attn_type": "ring"}}, "Ulysses"),
    ({"enable_cfg": True}, "CFG"),
])
def test_configure_refuses(patch, message):
    with pytest.raises(ValueError, match=message):
        configure({"attn_type": "flash_attn3", **patch})


def test_configure_and_prepare_only(tmp_path, capsys):
    base = {"attn_type": "flash_attn3", "parallel": {"seq_p_attn_type": "ulysses"}, "infer_steps": 40}
    assert configure(base)["attn_type"] == lightx2v.REGISTRY_KEY and base["attn_type"] == "flash_attn3"
    src = tmp_path / "h3.json"
    src.write_text(json.dumps(base))
    rc = lightx2v.main(["--mode", "combined", "--output-dir", str(tmp_path / "out"), "--prepare-only", "--",
                        "--model_cls", "x", "--config_json", str(src)])
    assert rc == 0
    patched = json.loads((tmp_path / "out" / "config.rank0.json").read_text())
    assert patched["attn_type"] == lightx2v.REGISTRY_KEY and patched["warmup"] is False
    assert capsys.readouterr().out.strip().endswith("config.rank0.json")


def test_register_mixes_in_the_template():
    registered = {}

    class Registry:
        def register(self, cls, key):
            registered[key] = cls

    class Template:
        pass

    audit = {"calls": 0, "smoothing_calls": 0, "regroup_calls": 0, "expcast_calls": 0}
    cls = lightx2v.register(Registry(), Template, "fp8_control", audit)
    adapter = registered[lightx2v.REGISTRY_KEY]()
    assert cls is registered[lightx2v.REGISTRY_KEY] and isinstance(adapter, Template)
    assert adapter.audit is audit and not adapter.vc_config.v_smooth and not adapter.vc_config.expcast


@pytest.mark.gpu
@pytest.mark.skipif(not has_b200(), reason="needs a B200")
def test_adapter_output_equals_direct_attention_on_b200():
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv

    q, k, v = (x.cuda() for x in make_qkv("c3", 5, heads=2, seq=1000))
    snd = [x[0].transpose(0, 1).contiguous() for x in (q, k, v)]          # [S, H, D]
    adapter = ExperimentAdapter("combined")
    marker = object()
    cfg = Config(v_smooth=True, expcast=True)
    cache = LayoutCache(cfg)
    for step in range(3):
        got = adapter.apply(*snd, scheduler=scheduler(step, steps=8, marker=marker), block_idx=7)
        want, _ = attention(q, k, v, cfg, cache=cache, step=step, total_steps=8, request_id=1, layer_id=7)
        assert got.dtype == q.dtype and got.shape == (1000, 256)
        assert torch.equal(got, want[0].transpose(0, 1).reshape(1000, 256))
    assert adapter.audit["calls"] == 3 and adapter.audit["regroup_calls"] == 1
