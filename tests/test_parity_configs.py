"""Parity of the B200 path with the CPU checker (oracle/) on every benchmark
configuration at its stated size, the denoising schedule of configuration 5,
the query-slice replay, and the count of ExpCast bytes in which the fused
kernel's encode differs from the reference's FP64-intermediate one.

Full-size forwards run on the GPU; the checker recomputes one or two heads
and a few 128-row query slices of each (the replay semantics of the
reference, replay.py:95-99: a 128-aligned slice of Q against the full K/V).
Tolerance, as everywhere in these tests: relative RMSE <= 1e-3 and cosine
>= 0.9999; permutations, payloads and ExpCast codes bit for bit."""
import math

import numpy as np
import pytest
import torch

from conftest import has_b200
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]

RMSE_TOL = 1e-3
COS_TOL = 0.9999
D = 128


def _head_np(x, head):
    return x[:, head].float().cpu().numpy()           # [B=1, S, D] -> the checker's [heads, S, D]


def _cast(ref, dtype):
    return torch.from_numpy(np.ascontiguousarray(ref)).to(dtype).float().numpy()


def _check_rows(out, q, k, v, cfg, *, head, rows, pi=None, active=False, scale=D ** -0.5):
    """The checker's output for `rows` of one head against the GPU output."""
    prep = O.Prepared(_head_np(q, head), _head_np(k, head), _head_np(v, head),
                      pi=None if pi is None else pi[None], active=active, q_block=cfg.q_block,
                      k_quant_block=cfg.k_quant_block, kv_block=128, mean_dtype=cfg.mean_dtype,
                      k_smooth=cfg.k_smooth, qk_hadamard=cfg.qk_hadamard)
    results = []
    for r0 in rows:
        ref = O.stream(prep, slice(r0, r0 + 128), expcast=cfg.expcast, scale=scale)
        got = out[:, head, r0:r0 + 128].float().cpu().numpy()
        m = O.metrics(got, _cast(ref, q.dtype))
        assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, (head, r0, m)
        results.append(m)
    return results


# ------------------------------------------------------------------ config 2
@pytest.mark.parametrize("cast", [False, True], ids=["fp8_control", "expcast"])
def test_config2_full_size(cast):
    """B1 H24 S16384 bf16, Gaussian V, 128-token Q / 256-token K blocks, in
    the fp8_control and expcast modes: two heads x two query slices."""
    from vc_attention_b200 import Config, attention
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv("c2", 31, device="cuda")
    assert q.shape == (1, 24, 16384, 128)
    cfg = Config(v_smooth=False, expcast=cast)
    out, stats = attention(q, k, v, cfg)
    assert not stats["smoothing_active"]
    for head in (0, 23):
        print(head, _check_rows(out, q, k, v, cfg, head=head, rows=(0, 16384 - 128)))


# ------------------------------------------------------------------ config 4
def test_config4_single_gpu_one_head():
    """B1 S131072 bf16, combined mode at a refresh step, one head on one GPU:
    the whole permutation bit for bit and two query slices against the
    checker (the multi-GPU Ulysses form is checked by the bench line and by
    tests/test_multigpu.py)."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv("c4", 41, device="cuda", heads=1)
    assert q.shape == (1, 1, 131072, 128)
    cfg = Config(v_smooth=True, expcast=True)
    cache = LayoutCache(cfg)
    out, stats = attention(q, k, v, cfg, cache=cache, step=0, total_steps=50, request_id="c4")
    assert stats["layout_refreshed"] and stats["smoothing_active"]
    pi = cache._states[0]["pi"][0, 0].cpu().numpy()
    rpi, _, _ = O.group_values(_head_np(v, 0), clusters=8, iterations=2)
    assert np.array_equal(pi, rpi[0])
    print(_check_rows(out, q, k, v, cfg, head=0, rows=(0, 65536 + 4096), pi=rpi[0], active=True))


# ------------------------------------------------------------------ config 5
ARMS = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False),
        "combined": (True, True)}
CHECKED_STEPS = (0, 1, 4, 12, 13, 49)


@pytest.mark.parametrize("mode", sorted(ARMS))
def test_config5_schedule_phases(mode):
    """B1 H24 S65536, centres drifting per step, 50 steps through one
    LayoutCache (core.py:182-211): smoothing on steps 0-12, layout refreshed
    at 0/4/8/12 with warm-started centres, the cached permutation reused in
    between, no smoothing from step 13.  At steps 0, 1, 4, 12, 13 and 49 one
    head's permutation (bit for bit, warm start followed on the checker) and
    a query slice are compared with the checker; the cached permutation is
    the very tensor of the last refresh."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv
    smooth, cast = ARMS[mode]
    cfg = Config(v_smooth=smooth, expcast=cast)
    cache = LayoutCache(cfg)
    head, total = 5, 50
    ref_centers, ref_pi, last_pi = None, None, None
    phases = []
    for step in range(total):
        q, k, v = make_qkv("c5", 51, device="cuda", step=step)
        out, stats = attention(q, k, v, cfg, cache=cache, step=step, total_steps=total, request_id=mode,
                               layer_id=0)
        active = step < 13 and smooth
        assert stats["smoothing_active"] == active
        assert stats["layout_refreshed"] == (active and step % 4 == 0)
        if stats["layout_refreshed"]:
            # the checker follows every refresh, warm-started like the cache
            ref_pi, ref_centers, _ = O.group_values(_head_np(v, head), clusters=8, iterations=2,
                                                    centers=ref_centers)
            last_pi = cache._states[0]["pi"]
            assert np.array_equal(last_pi[0, head].cpu().numpy(), ref_pi[0]), step
        elif smooth:
            # cached (core.py:209-211), also after the window, where the
            # permutation stays and only the demean stops
            assert cache._states[0]["pi"] is last_pi
        if step in CHECKED_STEPS:
            m = _check_rows(out, q, k, v, cfg, head=head, rows=(4096,), pi=ref_pi[0] if smooth else None,
                            active=active)
            phases.append((step, stats["layout_refreshed"], active, m[0]["relative_rmse"]))
    print(mode, phases)


def test_query_slice_replay_equals_full_rows():
    """replay.py:95-99: Q rows [4096, 4224) against the full K/V through
    attention() give the same rows as the full call.  Q is quantised in
    128-row blocks, so the slice's bytes, and therefore its output, are
    identical; the check is bit for bit, which implies the tolerance."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv("c5", 61, device="cuda", step=0)
    for smooth, cast in ARMS.values():
        cfg = Config(v_smooth=smooth, expcast=cast)
        full, _ = attention(q, k, v, cfg, cache=LayoutCache(cfg), step=0, total_steps=50, request_id="full")
        part, _ = attention(q[:, :, 4096:4224], k, v, cfg, cache=LayoutCache(cfg), step=0, total_steps=50,
                            request_id="slice")
        assert part.shape == (1, 24, 128, 128)
        assert torch.equal(part, full[:, :, 4096:4224]), (smooth, cast)


# ------------------------------------------------------- small-scale edge
@pytest.mark.parametrize("scale", [1e-30, 1e-44])
@pytest.mark.parametrize("cast", [False, True])
def test_tiny_scale_with_ragged_keys(scale, cast):
    """A softmax scale so small that every logit rounds to zero (the reference
    then weighs all keys equally), with 300 keys so the last tile is ragged:
    the masked keys must stay out of the row mass and nothing may turn NaN."""
    from vc_attention_b200 import Config, attention
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, n, 64, generator=g) for n in (130, 300, 300))
    cfg = Config(v_smooth=False, expcast=cast)
    out, _ = attention(q.cuda(), k.cuda(), v.cuda(), cfg, scale=scale)
    assert torch.isfinite(out).all()
    ref = O.attention(q[0].numpy(), k[0].numpy(), v[0].numpy(), expcast=cast, active=False, scale=scale)
    m = O.metrics(out[0].cpu().numpy(), ref)
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


# ------------------------------------------------ fused ExpCast byte flips
def _probe(config, seq, seed, *, expcast, q_tile):
    from vc_attention_b200 import stages
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv(config, seed, device="cuda", heads=1, seq=seq)
    q, k, v = (x.to(torch.bfloat16) for x in (q, k, v))
    q8, qs, k8, ks = stages.quantize_qk(q, k)
    v8, meta, _ = stages.prepare_v(v, active=False)
    scale = D ** -0.5
    _, logits, codes, rowstat = stages.attention_fp8_probe(
        q8, qs, k8, ks, v8, meta, heads=1, sq=seq, sk=seq, dv=D, head=0, q_tile=q_tile, expcast=expcast,
        has_mean=False, scale=scale)
    rows = q_tile * 128 + np.arange(128)
    qsr = qs[0].cpu().numpy()[rows // 128].astype(np.float32)                  # [128]
    ksr = ks[0].cpu().numpy()[np.arange(logits.shape[0]) * 128 // 256].astype(np.float32)   # [tiles]
    return (logits.cpu().numpy(), codes.cpu().numpy(), rowstat.cpu().numpy(), qsr, ksr, np.float32(scale))


@pytest.mark.parametrize("config,seq,q_tile", [("c3", 32768, 77), ("c2", 16384, 5), ("c1", 2048, 3)])
def test_fused_expcast_byte_flips(config, seq, q_tile):
    """Counts the ExpCast bytes of one query tile over every KV tile of a
    head in which the fused kernel differs from the reference's encode.

    The kernel never forms S - m: it encodes rne(fma(s, A, B) * 2^24) with
    s = q8 . k8, A = fp32(c * 8 log2 e * 2^-24), B = fp32((119.65 - m * 8 log2
    e) * 2^-24) and c = fp32(fp32(qs * ks) * scale).  Three counts:
    - the kernel's own form on the host (vco_fused_codes) must equal the
      dumped bytes exactly: the dump and its emulation agree;
    - against the reference's FP64-intermediate encode (core.py:60-68,
      :326-328) of fp32(S - m), given the kernel's FP32 logits S = fp32(s c)
      and its running max m;
    - against the same encode of the reference's own logits
      fp32(fp32(qs ks s) * scale), with their running max.
    Differences must be single-code flips at rounding boundaries, at most
    1e-4 of the codes."""
    logits, codes, rowstat, qsr, ksr, scale = _probe(config, seq, 71, expcast=True, q_tile=q_tile)
    tiles = logits.shape[0]
    m, a, b = rowstat[..., 0], rowstat[..., 1], rowstat[..., 2]
    valid = np.isfinite(logits)
    own = O.fused_codes(logits, a[..., None], b[..., None])
    assert np.array_equal(own[valid], codes[valid])
    assert not codes[~valid].any()
    # the kernel's FP32 logits and running max
    c = (qsr[None, :] * ksr[:, None]).astype(np.float32) * scale                # [tiles, 128] fp32
    c = c.astype(np.float32)
    s_kernel = (logits.astype(np.float64) * c[..., None].astype(np.float64)).astype(np.float32)
    assert np.array_equal(np.maximum.accumulate(np.where(valid, s_kernel, -np.inf).max(-1), axis=0), m)
    shifted = (s_kernel - m[..., None]).astype(np.float32)
    fp64_codes = O.expcast_codes(np.where(valid, shifted, -np.inf), fp64=True)
    # the reference's own logits: exact dot product times the scales, rounded, times scale, rounded
    s_ref = (logits.astype(np.float64) * (qsr[None, :, None].astype(np.float64) * ksr[:, None, None])
             ).astype(np.float32)
    s_ref = (s_ref * scale).astype(np.float32)
    m_ref = np.maximum.accumulate(np.where(valid, s_ref, -np.inf).max(-1), axis=0)
    ref_codes = O.expcast_codes(np.where(valid, (s_ref - m_ref[..., None]).astype(np.float32), -np.inf), fp64=True)
    n = int(valid.sum())
    flips_same = int((fp64_codes != codes)[valid].sum())
    flips_ref = int((ref_codes != codes)[valid].sum())
    diff = np.abs(fp64_codes.astype(np.int16) - codes.astype(np.int16))[valid]
    print(f"{config}: {n} codes over {tiles} KV tiles; differ from the FP64 encode of the kernel's FP32 logits: "
          f"{flips_same} ({flips_same / n:.2e}); from the FP64 encode of the reference's logits: {flips_ref} "
          f"({flips_ref / n:.2e}); largest difference {int(diff.max()) if diff.size else 0}")
    assert diff.max() <= 1
    assert flips_same <= 1e-4 * n and flips_ref <= 1e-4 * n


@pytest.mark.parametrize("config,seq,q_tile", [("c3", 32768, 77)])
def test_fused_exp_p8_against_fp32_exp(config, seq, q_tile):
    """Without ExpCast, P8 = e4m3(exp(S - m) * 256) (core.py:330-333).  The
    kernel takes 2^(fma(s, A, B)) on MUFU.EX2 with the factor 256 folded into
    B; against torch's FP32 exp of the kernel's FP32 (S - m), at most 1e-3 of
    the bytes may differ, each by one E4M3 step."""
    logits, codes, rowstat, qsr, ksr, scale = _probe(config, seq, 73, expcast=False, q_tile=q_tile)
    m = rowstat[..., 0]
    valid = np.isfinite(logits)
    c = ((qsr[None, :] * ksr[:, None]).astype(np.float32) * scale).astype(np.float32)
    s_kernel = (logits.astype(np.float64) * c[..., None]).astype(np.float32)
    shifted = torch.from_numpy(np.where(valid, (s_kernel - m[..., None]).astype(np.float32), -np.inf))
    ref = (torch.exp(shifted) * 256.0).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    n = int(valid.sum())
    flips = int((ref != codes)[valid].sum())
    step = np.abs(ref.astype(np.int16) - codes.astype(np.int16))[valid]
    print(f"{config} non-ExpCast P8: {flips} of {n} bytes differ ({flips / n:.2e}); largest {int(step.max())}")
    assert step.max() <= 1 and flips <= 1e-3 * n
