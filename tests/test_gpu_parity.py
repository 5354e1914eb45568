"""Parity of the sm_100a path with the CPU checker (oracle/) and with outputs
recorded from the reference implementation (tests/golden).

Byte-level stages are compared bit for bit: ExpCast codes, E4M3 payloads and
block scales of Q/K, V tiles, cluster permutations and centres.  The fused
attention output is compared within the tolerance the contract states:
relative RMSE <= 1e-3 and cosine >= 0.9999 (FP32 accumulation order is the
only difference)."""
import math

import numpy as np
import pytest
import torch

import cases
from conftest import has_b200
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]

RMSE_TOL = 1e-3
COS_TOL = 0.9999


def _np(t):
    return t.detach().float().cpu().numpy()


def _flat_np(x):
    b, h, s, d = x.shape
    return x.float().reshape(b * h, s, d).cpu().numpy()


def _cast_like(ref, dtype):
    """The reference returns output.to(q.dtype) (core.py:341)."""
    return torch.from_numpy(np.ascontiguousarray(ref)).to(dtype).float().numpy()


# ----------------------------------------------------------------- ExpCast
def test_expcast_bytes_bit_exact():
    from vc_attention_b200.b200_backend import expcast_codes
    x = cases.expcast_inputs()
    got = expcast_codes(x.cuda()).cpu().numpy()
    assert np.array_equal(got, O.expcast_codes(x.numpy(), fp64=False))
    # count of bytes that differ from the reference's FP64-intermediate form
    golden = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "golden.npz")["expcast_codes"]
    assert int((got != golden).sum()) == 0


def test_expcast_known_answers_and_boundaries():
    from vc_attention_b200.b200_backend import expcast_codes
    u = torch.tensor(cases.KNOWN_U) / math.log2(math.e)
    assert expcast_codes(u.cuda()).tolist() == cases.KNOWN_CODES
    x = cases.expcast_inputs()[7:19]
    assert expcast_codes(x.cuda()).tolist() == cases.FMA_CODES


# ------------------------------------------------------------ Q/K stages
QK_CASES = [
    # dtype, heads, sq, sk, d, q_block, k_quant_block, k_smooth, hadamard, permuted
    (torch.bfloat16, 3, 1000, 1300, 128, 128, 256, True, True, True),
    (torch.float32, 2, 130, 260, 37, 128, 256, True, True, False),
    (torch.float16, 2, 300, 700, 64, 64, 512, True, True, True),
    (torch.bfloat16, 1, 256, 384, 128, 32, 128, False, True, False),
    (torch.float32, 2, 200, 300, 21, 96, 256, True, False, False),
    (torch.bfloat16, 1, 600, 5000, 128, 256, 4096, True, True, True),
    (torch.float16, 2, 500, 900, 128, 64, 256, True, True, True),
    (torch.bfloat16, 2, 100, 200, 128, 8, 16, True, True, True),     # blocks below one warp of rows
]


@pytest.mark.parametrize("case", QK_CASES)
def test_quantize_qk_bit_exact(case):
    from vc_attention_b200 import stages
    dtype, h, sq, sk, d, qb, kq, ks, had, perm = case
    g = torch.Generator().manual_seed(sq + sk + d)
    q = torch.randn(1, h, sq, d, generator=g).to(dtype)
    k = (torch.randn(1, h, sk, d, generator=g) + torch.randn(1, h, 1, d, generator=g) * 1.5).to(dtype)
    pi = torch.stack([torch.randperm(sk, generator=g) for _ in range(h)]).int().view(1, h, sk) if perm else None
    q8, qs, k8, kss = stages.quantize_qk(q.cuda(), k.cuda(), pi=None if pi is None else pi.cuda(), q_block=qb,
                                         k_quant_block=kq, k_smooth=ks, hadamard=had)
    qn, kn = _flat_np(q), _flat_np(k)
    qf, kf = O.preprocess_qk(qn, kn, k_smooth=ks, qk_hadamard=had, pi=pi.view(h, sk).numpy() if perm else None)
    rq8, rqs = O.quantize_blocks(qf, qb)
    rk8, rks = O.quantize_blocks(kf, kq)
    assert np.array_equal(qs.cpu().numpy(), rqs)
    assert np.array_equal(kss.cpu().numpy(), rks)
    assert np.array_equal(q8.cpu().numpy(), rq8)
    assert np.array_equal(k8.cpu().numpy(), rk8)


@pytest.mark.parametrize("dim", [37, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("k_smooth,rotate", [(False, False), (False, True), (True, False), (True, True)])
def test_preprocess_qk_matches_checker_and_explicit_matrix(dim, dtype, k_smooth, rotate):
    """test_paper_alignment.py:114-142 on the B200 path, on a side stream with
    non-contiguous inputs; bit-exact against the CPU checker."""
    from vc_attention_b200.b200_backend import preprocess_qk
    g = torch.Generator().manual_seed(14)
    q, k = [torch.randn(2, 2, n, dim, generator=g) for n in (13, 35)]
    k += torch.linspace(-2, 2, dim)
    q, k = q.to(dtype), k.to(dtype)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        qd, kd = [torch.stack([x.cuda(), x.cuda()], -1)[..., 0] for x in (q, k)]
        got = preprocess_qk(qd, kd, k_smooth, rotate)
        consumed = [x + 1 for x in got]
    stream.synchronize()
    rq, rk = O.preprocess_qk(_flat_np(q), _flat_np(k), k_smooth=k_smooth, qk_hadamard=rotate)
    assert np.array_equal(_np(got[0]).reshape(rq.shape), rq)
    assert np.array_equal(_np(got[1]).reshape(rk.shape), rk)
    width = 1 << (dim - 1).bit_length() if rotate else dim
    mat = torch.tensor([[(-1.0) ** bin(i & j).count("1") for j in range(width)] for i in range(width)]) / math.sqrt(width)
    eq, ek = q.float(), k.float()
    if k_smooth:
        ek = ek - ek.mean(-2, keepdim=True)
    if rotate:
        eq = torch.nn.functional.pad(eq, (0, width - dim)) @ mat
        ek = torch.nn.functional.pad(ek, (0, width - dim)) @ mat
    torch.testing.assert_close(consumed[0].cpu(), eq + 1, atol=3e-6, rtol=3e-5)
    torch.testing.assert_close(consumed[1].cpu(), ek + 1, atol=3e-6, rtol=3e-5)


# --------------------------------------------------------------- V stages
@pytest.mark.parametrize("mean_dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("active,perm,dtype,s,dv", [
    (True, True, torch.bfloat16, 1000, 128), (True, False, torch.float32, 300, 21),
    (False, True, torch.float16, 257, 128), (False, False, torch.bfloat16, 128, 64),
])
def test_prepare_v_bit_exact(mean_dtype, active, perm, dtype, s, dv):
    from vc_attention_b200 import stages
    g = torch.Generator().manual_seed(s + dv)
    h = 2
    v = (torch.randn(1, h, s, dv, generator=g) * 0.3 + torch.randn(1, h, 1, dv, generator=g) * 3).to(dtype)
    pi = torch.stack([torch.randperm(s, generator=g) for _ in range(h)]).int().view(1, h, s) if perm else None
    v8, meta, mop = stages.prepare_v(v.cuda(), pi=None if pi is None else pi.cuda(), active=active, mean_dtype=mean_dtype)
    r8, rvs, rmu = O.value_tiles(_flat_np(v), None if pi is None else pi.view(h, s).numpy(), active=active,
                                 mean_dtype=mean_dtype, kv_block=128)
    meta = meta.cpu().numpy()
    assert np.array_equal(meta[:, :, 0], rvs)
    assert np.array_equal(meta[:, :, 1], rmu)
    assert np.array_equal(v8.cpu().numpy(), r8)
    if active:
        # the mean operand of the row-mass x mean MMA: the stored mean as bf16
        # pieces u1 (truncated) + u2 + u3 (rounded remainders), which add up to
        # it exactly, in the row [u1, u2, u3, u1, u2, u1, 0 ...]
        stored = torch.from_numpy(rmu)
        u1 = (stored.view(torch.int32) & -65536).view(torch.float32)
        u2 = (stored - u1).to(torch.bfloat16).float()
        u3 = (stored - u1 - u2).to(torch.bfloat16).float()
        assert torch.equal(u1 + u2 + u3, stored)
        want = torch.zeros(*stored.shape, 16, dtype=torch.bfloat16)
        for slot, piece in enumerate((u1, u2, u3, u1, u2, u1)):
            want[..., slot] = piece.to(torch.bfloat16)
        assert torch.equal(mop.cpu(), want.view(torch.int16))
    else:
        assert mop is None


def test_prepare_v_reference_tiles(golden):
    """V bytes on the order-independent fixture equal the reference's own."""
    from vc_attention_b200 import stages
    tile = cases.exact_value_tile()          # [1, 2, 128, 21]
    for mean_dtype in ("float16", "bfloat16", "float32"):
        v8, meta, _ = stages.prepare_v(tile.cuda(), active=True, mean_dtype=mean_dtype)
        payload = v8.cpu().numpy()[:, 0, :21, :].transpose(0, 2, 1)
        assert np.array_equal(payload, golden[f"vtile_exact_{mean_dtype}_payload"][0])
        assert np.array_equal(meta.cpu().numpy()[:, 0, 0, :21], golden[f"vtile_exact_{mean_dtype}_scale"][0, :, 0])
        assert np.array_equal(meta.cpu().numpy()[:, 0, 1, :21], golden[f"vtile_exact_{mean_dtype}_stored"][0, :, 0])


# ------------------------------------------------------------- clustering
@pytest.mark.parametrize("dtype,s,d,clusters,iters,warm", [
    (torch.bfloat16, 4096, 128, 8, 2, False), (torch.float32, 1000, 16, 8, 2, False),
    (torch.float16, 777, 37, 3, 3, True), (torch.bfloat16, 300, 128, 1, 2, False),
    (torch.float32, 5, 16, 8, 2, False), (torch.bfloat16, 2048, 128, 32, 2, True),
])
def test_group_values_bit_exact(dtype, s, d, clusters, iters, warm):
    from vc_attention_b200.b200_backend import group_values
    from vc_attention_b200.synthetic import make_qkv
    if d == 128:
        _, _, v = make_qkv("c3", s + clusters, heads=2, seq=s)
        v = v.to(dtype)
    else:
        v = cases.clustered_values(tokens=s, heads=2, dim=d).to(dtype)
    count = min(clusters, s)
    centers = None
    if warm:
        centers = torch.randn(1, 2, count, d, generator=torch.Generator().manual_seed(3)) * 2
    pi, cen = group_values(v.cuda(), clusters=clusters, iterations=iters,
                           centers=None if centers is None else centers.cuda())
    rpi, rcen, _ = O.group_values(_flat_np(v), clusters=clusters, iterations=iters,
                                  centers=None if centers is None else centers.view(2, count, d).numpy())
    assert np.array_equal(pi.view(2, s).cpu().numpy(), rpi)
    assert np.array_equal(cen.view(2, count, d).cpu().numpy(), rcen)


def test_group_values_agreement_with_reference(golden):
    from vc_attention_b200.b200_backend import group_values
    v = cases.separated_values()
    pi, cen = group_values(v.cuda(), clusters=8, iterations=2)
    assert np.array_equal(pi[0].cpu().numpy(), golden["group_sep_pi"][0])
    np.testing.assert_allclose(cen[0].cpu().numpy(), golden["group_sep_centers"][0], rtol=1e-6, atol=1e-6)
    v = cases.clustered_values()
    pi, _ = group_values(v.cuda(), clusters=8, iterations=2)
    agreement = float((pi[0].cpu().numpy() == golden["group_pi"][0]).mean())
    print(f"permutation agreement with the reference on near-tie data: {agreement:.4f}")
    assert agreement > 0.95


# ----------------------------------------------------------- attention
def _oracle_forward(q, k, v, cfg, *, pi, active, scale=None):
    b, h = q.shape[:2]
    out = O.attention(_flat_np(q), _flat_np(k), _flat_np(v), expcast=cfg.expcast, active=active,
                      pi=None if pi is None else pi.view(b * h, -1).cpu().numpy(), q_block=cfg.q_block,
                      k_quant_block=cfg.k_quant_block, kv_block=128, mean_dtype=cfg.mean_dtype, scale=scale,
                      k_smooth=cfg.k_smooth, qk_hadamard=cfg.qk_hadamard)
    return out.reshape(b, h, q.shape[2], v.shape[3])


@pytest.mark.parametrize("name", sorted(cases.ATTENTION_CASES))
def test_attention_matches_reference_outputs(golden, name):
    """GPU output vs the output the reference implementation recorded."""
    from vc_attention_b200 import Config, attention
    shape, cfg_kw, call_kw = cases.ATTENTION_CASES[name]
    q, k, v = cases.attention_inputs(name)
    cfg = Config(**cfg_kw)
    out, stats = attention(q.cuda(), k.cuda(), v.cuda(), cfg, **call_kw)
    torch.cuda.synchronize()
    assert stats["native_fused_attention"] and stats["tiles"] == int(golden[f"attn_{name}_tiles"])
    got = _np(out)
    if shape == "c1":
        got = got[:, :, ::cases.C1_ROW_STRIDE]
    m = O.metrics(got, golden[f"attn_{name}"])
    print(name, m)
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


ARMS = [(False, False), (False, True), (True, False), (True, True)]


@pytest.mark.parametrize("smooth,cast", ARMS)
@pytest.mark.parametrize("config,heads,seq", [("c2", 2, 2048), ("c3", 2, 4096), ("c1", 2, 2048)])
def test_attention_matches_checker_on_benchmark_distributions(config, heads, seq, smooth, cast):
    from vc_attention_b200 import Config, LayoutCache, attention
    q, k, v = (x.cuda() for x in __import__("vc_attention_b200.synthetic", fromlist=["x"]).make_qkv(
        config, 11, heads=heads, seq=seq))
    cfg = Config(v_smooth=smooth, expcast=cast)
    cache = LayoutCache(cfg)
    out, stats = attention(q, k, v, cfg, cache=cache, step=0, total_steps=50, request_id="r")
    pi = cache._states[0]["pi"] if smooth else None
    ref = _oracle_forward(q, k, v, cfg, pi=pi, active=smooth)
    m = O.metrics(_np(out), _cast_like(ref, q.dtype))
    print(config, smooth, cast, m)
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


def test_constant_values_restored_exactly():
    """test_core.py:42-48 / cuda_backend.preflight: constant V is returned exactly."""
    from vc_attention_b200 import Config, attention
    q, k, v = cases.reference_test_inputs((1, 2, 300, 700, 128, 128))
    v.fill_(3.0)
    for cast in (False, True):
        out, _ = attention(q.cuda(), k.cuda(), v.cuda(), Config(v_smooth=True, expcast=cast))
        torch.testing.assert_close(out.cpu(), torch.full_like(out.cpu(), 3.0), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("cast", [False, True])
def test_running_max_mean_recovery_and_tail(cast):
    """test_cuda.py:141-150: a later key block dominates; the mean of the last
    (ragged) tile must be recovered exactly after the running-max rescale."""
    from vc_attention_b200 import Config, attention
    q = torch.ones(1, 1, 17, 16)
    k = torch.cat([torch.full((1, 1, 128, 16), -20.), torch.full((1, 1, 3, 16), 20.)], 2)
    v = torch.cat([torch.full((1, 1, 128, 16), 3.), torch.full((1, 1, 3, 16), 9.)], 2)
    out, _ = attention(q.cuda(), k.cuda(), v.cuda(), Config(v_smooth=True, expcast=cast, clusters=1))
    torch.testing.assert_close(out.cpu(), torch.full_like(out.cpu(), 9), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dtype_noncontiguous_and_distinct_value_width(dtype):
    """test_cuda.py:98-110."""
    from vc_attention_b200 import Config, attention
    q, k, v = [x.to(dtype) for x in cases.reference_test_inputs((1, 2, 35, 131, 64, 32))]

    def strided(x):
        return torch.stack([x, x], -1)[..., 0]
    cfg = Config(expcast=False)
    out, _ = attention(*[strided(x.cuda()) for x in (q, k, v)], cfg)
    assert out.dtype == dtype
    ref = _oracle_forward(q, k, v, cfg, pi=None, active=False)
    m = O.metrics(_np(out), _cast_like(ref, dtype))
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


def test_signed_values_and_shared_k_quantization_scale():
    """test_cuda.py:113-126."""
    from vc_attention_b200 import Config, attention
    q, k, v = cases.reference_test_inputs((1, 1, 35, 259, 37, 21))
    v = (v - 3) * 5
    k[:, :, :128] *= 0.1
    k[:, :, 128:256] *= 4
    cfg = Config(expcast=False)
    out, _ = attention(q.cuda(), k.cuda(), v.cuda(), cfg)
    ref = _oracle_forward(q, k, v, cfg, pi=None, active=False)
    m = O.metrics(_np(out), ref)
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


def test_current_stream_is_used():
    """test_cuda.py:176-189."""
    from vc_attention_b200 import Config, attention
    cfg = Config()
    q, k, v = cases.reference_test_inputs((1, 1, 17, 35, 16, 16))
    ref = _oracle_forward(q, k, v, cfg, pi=None, active=False)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        qd, kd, vd = [x.cuda(non_blocking=True) for x in (q, k, v)]
        out, _ = attention(qd, kd, vd, cfg)
        consumed = out + 1
    stream.synchronize()
    m = O.metrics(_np(consumed) - 1, ref)
    assert m["relative_rmse"] <= RMSE_TOL


@pytest.mark.parametrize("chunk_heads", [None, 2, 5])
def test_streamed_host_attention_equals_device_attention(chunk_heads):
    """attention_streamed (host tensors, transfers overlapped per head chunk)
    gives the same bytes as attention on the whole device tensors: heads are
    independent and every chunk runs the same forward.  Two steps with one
    cache check the per-chunk layout refresh and reuse."""
    from vc_attention_b200 import Config, LayoutCache, attention, attention_streamed
    from vc_attention_b200.synthetic import make_qkv
    cfg = Config(v_smooth=True, expcast=True)
    q, k, v = make_qkv("c3", 5, heads=7, seq=1000)
    hq, hk, hv = (x.pin_memory() for x in (q, k, v))
    cache_h, cache_d = LayoutCache(cfg), LayoutCache(cfg)
    for step in (0, 1):
        got, stats = attention_streamed(hq, hk, hv, cfg, cache=cache_h, step=step, total_steps=8, request_id="r",
                                        chunk_heads=chunk_heads)
        want, _ = attention(q.cuda(), k.cuda(), v.cuda(), cfg, cache=cache_d, step=step, total_steps=8,
                            request_id="r")
        assert got.device.type == "cpu" and got.is_pinned()
        assert torch.equal(got, want.cpu())
        assert stats["layout_refreshed"] == (step == 0)


def test_cache_refresh_reuse_and_window_with_native_clustering():
    """test_cuda.py:153-173: reused layout, current means, end of the window."""
    from vc_attention_b200 import Config, LayoutCache, attention
    q, k, v = [x.cuda() for x in cases.reference_test_inputs((1, 2, 19, 259, 16, 16))]
    cfg = Config(v_smooth=True, clusters=1)
    cache = LayoutCache(cfg)
    args = dict(cache=cache, total_steps=20, request_id="one", layer_id=0)
    first, first_info = attention(q, k, v, cfg, step=0, **args)
    second, second_info = attention(q, k, v + 8, cfg, step=1, **args)
    assert first_info["layout_refreshed"] and not second_info["layout_refreshed"]
    torch.testing.assert_close(second - first, torch.full_like(first, 8), atol=0.02, rtol=0)
    _, late_info = attention(q, k, v, cfg, step=5, **args)
    assert not late_info["smoothing_active"]


def test_nonfinite_input_is_rejected_and_cache_untouched():
    from vc_attention_b200 import Config, LayoutCache, attention
    q, k, v = [x.cuda() for x in cases.reference_test_inputs((1, 1, 40, 300, 64, 64))]
    cfg = Config(v_smooth=True)
    cache = LayoutCache(cfg)
    attention(q, k, v, cfg, cache=cache, step=0, total_steps=20, request_id="a")
    before = cache._states[0]
    for bad in ("q", "k", "v"):
        n, d = {"q": q, "k": k, "v": v}[bad].shape[2:]
        for value, where in ((float("nan"), (0, 0, 5, 3)), (float("inf"), (0, 0, n - 1, d - 1)),
                             (float("-inf"), (0, 0, n // 2, 0))):
            t = {"q": q, "k": k, "v": v}
            t[bad] = t[bad].clone()
            t[bad][where] = value
            with pytest.raises(ValueError, match="finite"):
                attention(t["q"], t["k"], t["v"], cfg, cache=cache, step=4, total_steps=20, request_id="a")
            assert cache._states[0] is before and cache._states[0]["step"] == 0
    # past the smoothing window (no V mean) the check still covers V
    for value in (float("nan"), float("inf")):
        tv = v.clone()
        tv[0, 0, 17, 9] = value
        with pytest.raises(ValueError, match="finite"):
            attention(q, k, tv, cfg, cache=LayoutCache(cfg), step=19, total_steps=20, request_id="b")


@pytest.mark.parametrize("k_smooth,rotate", [(False, False), (False, True), (True, False), (True, True)])
def test_qk_switches_with_custom_scale(k_smooth, rotate):
    """test_cuda.py:192-203."""
    from vc_attention_b200 import Config, attention
    q, k, v = cases.reference_test_inputs((1, 2, 17, 35, 37, 21))
    k += torch.linspace(-2, 2, 37)
    cfg = Config(v_smooth=True, expcast=True, clusters=1, k_smooth=k_smooth, qk_hadamard=rotate)
    out, stats = attention(q.cuda(), k.cuda(), v.cuda(), cfg, scale=0.07)
    assert stats["k_smooth"] == k_smooth and stats["qk_hadamard"] == rotate
    pi = torch.arange(35).view(1, 1, 35).expand(1, 2, 35).int()    # one cluster: identity
    ref = _oracle_forward(q, k, v, cfg, pi=pi, active=True, scale=0.07)
    m = O.metrics(_np(out), ref)
    assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, m


def test_preflight():
    from vc_attention_b200.b200_backend import preflight
    assert preflight()["preflight"] == "passed"


# ------------------------------------------------------ full-size checks
def test_full_size_c3_rows_match_checker():
    """Config 3 at full size (H=40, S=32768, combined, refresh step): the
    permutation of two heads is bit-exact and two 128-row query slices of
    each (replay.py:95-99 semantics: full K/V) agree with the checker."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv("c3", 3, device="cuda")
    cfg = Config(v_smooth=True, expcast=True)
    cache = LayoutCache(cfg)
    out, _ = attention(q, k, v, cfg, cache=cache, step=0, total_steps=50, request_id="full")
    pi = cache._states[0]["pi"]
    assert torch.equal(pi.sort(-1).values[0, :3], torch.arange(32768, device="cuda", dtype=torch.int32).expand(3, -1))
    for head in (0, 37):
        qh, kh, vh = (x[:, head:head + 1].float().cpu() for x in (q, k, v))
        rpi, _, _ = O.group_values(_flat_np(vh), clusters=8, iterations=2)
        assert np.array_equal(pi[0, head].cpu().numpy(), rpi[0])
        prep = O.Prepared(_flat_np(qh), _flat_np(kh), _flat_np(vh), pi=rpi, active=True, q_block=128,
                          k_quant_block=256, kv_block=128, mean_dtype="float16", k_smooth=True, qk_hadamard=True)
        for r0 in (0, 4096):
            ref = O.stream(prep, slice(r0, r0 + 128), expcast=True, scale=128 ** -0.5)
            got = _np(out[:, head, r0:r0 + 128])
            m = O.metrics(got, _cast_like(ref, torch.bfloat16))
            assert m["relative_rmse"] <= RMSE_TOL and m["cosine"] >= COS_TOL, (head, r0, m)


def test_full_size_properties():
    """Size-independent properties at config-3 size: the output is finite,
    a permutation of the query rows permutes the output rows exactly, and a
    constant shift of V (outside the demean window) shifts the output."""
    from vc_attention_b200 import Config, attention
    from vc_attention_b200.synthetic import make_qkv
    q, k, v = make_qkv("c3", 5, device="cuda", heads=8)
    cfg = Config(v_smooth=False, expcast=True)
    out, _ = attention(q, k, v, cfg)
    assert torch.isfinite(out).all()
    # Q tiles are independent: swapping two 128-row blocks swaps the output rows bit for bit.
    perm = torch.arange(q.shape[2], device="cuda")
    perm[:128], perm[128:256] = perm[128:256].clone(), perm[:128].clone()
    out2, _ = attention(q[:, :, perm], k, v, cfg)
    assert torch.equal(out2, out[:, :, perm])
