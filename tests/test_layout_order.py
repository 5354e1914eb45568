"""K and V handed over in the cached layout's order (the persistent
pre-permuted layout: a producer keeps K/V in pi order so that the forward
skips the gather the reference does on every call, cuda_backend.py:49-51).

On a step that reuses the cached layout, ``attention(..., kv_order="layout")``
on ``to_layout_order(k, pi)`` and ``to_layout_order(v, pi)`` must give the
call on K and V in token order:
- bit for bit without the K demean, since then every kernel reads the same
  bytes;
- with the K demean, within the usual tolerance (relative RMSE <= 1e-3,
  cosine >= 0.9999). The K channel sums run over the rows in the order
  given, as the reference's do after its gather, so their last bits may
  differ from the sums over token order.
On every other step the call is refused and the cache is left as it was."""
import pytest
import torch

from conftest import has_b200

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]


def _rel_rmse_cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    rmse = (a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()
    cos = torch.dot(a, b) / (a.norm() * b.norm())
    return rmse.item(), cos.item()


@pytest.mark.parametrize("k_smooth", [False, True])
@pytest.mark.parametrize("cast", [False, True])
def test_kv_in_layout_order_equals_the_gathering_call(cast, k_smooth):
    from vc_attention_b200 import Config, LayoutCache, attention, to_layout_order
    from vc_attention_b200.synthetic import make_qkv
    cfg = Config(v_smooth=True, expcast=cast, k_smooth=k_smooth)
    q, k, v = make_qkv("c3", 11, device="cuda", heads=3, seq=4096 + 200)
    natural, layout = LayoutCache(cfg), LayoutCache(cfg)
    kw = dict(total_steps=50, request_id="r", layer_id=0)
    for cache in (natural, layout):          # step 0 clusters V in both caches
        attention(q, k, v, cfg, cache=cache, step=0, **kw)
    for step in (1, 2):
        pi, active, refresh = layout.peek(v, step=step, **kw)
        assert pi is not None and active and not refresh
        assert torch.equal(pi, natural._states[0]["pi"])
        kp, vp = to_layout_order(k, pi), to_layout_order(v, pi)
        want, s_want = attention(q, k, v, cfg, cache=natural, step=step, **kw)
        got, s_got = attention(q, kp, vp, cfg, cache=layout, step=step, kv_order="layout", **kw)
        assert s_got["smoothing_active"] and not s_got["layout_refreshed"]
        assert s_got == s_want
        if not k_smooth:
            assert torch.equal(got, want), step
        else:
            rmse, cos = _rel_rmse_cos(got, want)
            print(f"cast={cast} step={step}: relative RMSE {rmse:.3e}, cosine {cos:.8f}, "
                  f"bit-equal {torch.equal(got, want)}")
            assert rmse <= 1e-3 and cos >= 0.9999


def test_kv_in_layout_order_is_refused_without_a_cached_layout():
    from vc_attention_b200 import Config, LayoutCache, attention, to_layout_order
    from vc_attention_b200.synthetic import make_qkv
    cfg = Config(v_smooth=True, expcast=True)
    q, k, v = make_qkv("c3", 12, device="cuda", heads=2, seq=2048)
    kw = dict(total_steps=50, request_id="r", layer_id=0)
    # a one-shot call has no cached layout
    with pytest.raises(ValueError, match="cached layout"):
        attention(q, k, v, cfg, kv_order="layout")
    cache = LayoutCache(cfg)
    # the first step of a request clusters: nothing cached yet, nothing changes
    with pytest.raises(ValueError, match="cached layout"):
        attention(q, k, v, cfg, cache=cache, step=0, kv_order="layout", **kw)
    assert cache.entries == 0
    attention(q, k, v, cfg, cache=cache, step=0, **kw)
    pi = cache._states[0]["pi"]
    kp, vp = to_layout_order(k, pi), to_layout_order(v, pi)
    attention(q, kp, vp, cfg, cache=cache, step=3, kv_order="layout", **kw)
    before = dict(cache._states[0])
    # step 4 refreshes the layout and step 13 is past the smoothing window:
    # both are refused, and the cached state is the same objects as before
    for step in (4, 13):
        p, _, _ = cache.peek(v, step=step, **kw)
        assert p is None
        with pytest.raises(ValueError, match="cached layout"):
            attention(q, kp, vp, cfg, cache=cache, step=step, kv_order="layout", **kw)
        state = cache._states[0]
        assert state.keys() == before.keys() and all(state[key] is before[key] for key in before)
