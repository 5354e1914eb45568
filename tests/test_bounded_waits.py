"""The attention kernel's bounded waits, exercised with no GPU fault.

`vcb_wait_selftest` holds what an attention CTA holds when a wait expires
(tensor memory, a bulk copy in flight, a tcgen05 commit) and waits through the
kernel's own `mbar_wait` on a barrier phase that nothing completes.  Every wait
gives up after the 2 s limit; the CTA drains, frees its tensor memory and sets
the timeout flag, which the host turns into the RuntimeError the forward
raises.  The same CUDA context then runs the fused path again."""
import pytest
import torch

from conftest import has_b200

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]


def test_completed_phase_gives_no_timeout():
    from vc_attention_b200.b200_backend import raise_for_status, wait_selftest

    r = wait_selftest(complete=True)
    assert (r["gave_up"], r["completed"], r["copy_intact"]) == (0, 4, True)
    assert r["elapsed_ms"] < 1000
    raise_for_status(r["status"])


def test_expired_wait_sets_the_timeout_flag_and_the_context_stays_usable():
    from vc_attention_b200 import Config, attention
    from vc_attention_b200.b200_backend import raise_for_status, wait_selftest

    r = wait_selftest(complete=False)
    assert (r["gave_up"], r["completed"], r["copy_intact"]) == (4, 0, True)
    assert 1900 <= r["elapsed_ms"] < 10000
    with pytest.raises(RuntimeError, match="bounded device wait expired"):
        raise_for_status(r["status"])

    # The context is intact and the tensor memory was freed: a forward whose
    # CTAs each allocate all 512 columns of an SM runs and gives the exact answer.
    q = torch.zeros(1, 2, 300, 128, device="cuda")
    k = torch.zeros(1, 2, 520, 128, device="cuda")
    v = torch.full((1, 2, 520, 128), 3.0, device="cuda")
    for cast in (False, True):
        out, _ = attention(q, k, v, Config(expcast=cast))
        torch.testing.assert_close(out, torch.full_like(out, 3), rtol=2e-5, atol=2e-5)
    torch.cuda.synchronize()
