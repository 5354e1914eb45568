"""Stream behaviour of the B200 path (the reference's contract,
bindings.cpp:176 and test_cuda.py:176-189: work on the caller's current
stream, no device-wide synchronisation): the status read waits for the
caller's stream only, and the caller-owned status word defers it."""
import pytest
import torch

from conftest import has_b200

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]


def _inputs():
    import cases
    return [x.cuda() for x in cases.reference_test_inputs((1, 2, 300, 700, 128, 128))]


def _busy(stream, seconds=1.5):
    """Keeps `stream` busy for about `seconds` (a spinning kernel)."""
    rate = torch.cuda.get_device_properties(0).clock_rate * 1000     # kHz -> cycles per second
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(seconds * rate))


def test_attention_does_not_wait_for_another_busy_stream():
    """attention() on stream B reads its status word on B; a spinning kernel
    on an unrelated (blocking) stream A is still running when it returns.  A
    status read on the legacy default stream would have waited for A."""
    from vc_attention_b200 import Config, attention
    q, k, v = _inputs()
    cfg = Config(v_smooth=True, expcast=True)
    attention(q, k, v, cfg)                 # load the library and warm up outside the timed part
    torch.cuda.synchronize()
    a, b = torch.cuda.Stream(), torch.cuda.Stream()
    _busy(a)
    with torch.cuda.stream(b):
        out, _ = attention(q, k, v, cfg)
    still_busy = not a.query()
    assert b.query()                        # the call waited for its own stream
    a.synchronize()
    assert still_busy, "attention waited for an unrelated stream"
    assert torch.isfinite(out).all()


def test_caller_owned_status_defers_the_check_and_rolls_back():
    """With status=word the call only queues its work (the host does not wait
    for the stream), the flags land in the word, and rollback() restores the
    layout cache after a failed check."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.b200_backend import raise_for_status
    q, k, v = _inputs()
    cfg = Config(v_smooth=True)
    cache = LayoutCache(cfg)
    attention(q, k, v, cfg, cache=cache, step=0, total_steps=20, request_id="r")
    before = dict(cache._states[0])
    s = torch.cuda.Stream()
    _busy(s)
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = v.clone()
    bad[0, 0, 3, 3] = float("nan")
    with torch.cuda.stream(s):
        out, stats = attention(q, k, bad, cfg, cache=cache, step=4, total_steps=20, request_id="r", status=word)
    assert not s.query(), "the deferred call waited for its stream"
    assert cache._states[0]["refresh_step"] == 4        # the layout moved on before the check
    with torch.cuda.stream(s):
        with pytest.raises(ValueError, match="finite"):
            raise_for_status(word)
    stats["rollback"]()
    assert cache._states[0]["refresh_step"] == before["refresh_step"]
    assert cache._states[0]["pi"] is before["pi"]
