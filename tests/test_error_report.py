"""The error-report CLI (the reference's native / reference / FP32 comparison,
scripts/benchmark_cuda.py:152-183): sampling, the FP64 golden and the metrics
on CPU; the native report on a B200."""
import math

import pytest
import torch

from conftest import has_b200
from vc_attention_b200 import error_report as er


def test_query_rows_spread_and_bounds():
    assert er.query_rows(10, 20) == list(range(10))
    assert er.query_rows(100, 1) == [0]
    rows = er.query_rows(4096, 64)
    assert rows[0] == 0 and rows[-1] == 4095 and len(rows) == 64 and rows == sorted(set(rows))


def test_fp32_golden_matches_a_direct_softmax():
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 9, 4, generator=g) for _ in range(3))
    rows = [0, 4, 8]
    got = er.fp32_golden(q, k, v, rows, 0.5)
    for h in range(2):
        for i, r in enumerate(rows):
            w = [math.exp(0.5 * float(q[0, h, r].double() @ k[0, h, j].double())) for j in range(9)]
            want = sum(w[j] * v[0, h, j].double() for j in range(9)) / sum(w)
            assert torch.allclose(got[0, h, i], want, rtol=1e-12, atol=1e-12)


def test_metrics_definitions():
    g = torch.tensor([1.0, -2.0, 3.0, 0.5])
    m = er.metrics(g.clone(), g)
    assert m["relative_rmse"] == 0 and m["max_abs"] == 0 and abs(m["cosine"] - 1) < 1e-15
    s = g + torch.tensor([0.1, 0.0, -0.2, 0.0])
    m = er.metrics(s, g)
    rmse = math.sqrt((0.01 + 0.04) / 4)
    assert abs(m["relative_rmse"] - rmse / math.sqrt((1 + 4 + 9 + 0.25) / 4)) < 1e-7
    assert abs(m["max_abs"] - 0.2) < 1e-7
    with pytest.raises(ValueError, match="non-finite"):
        er.metrics(torch.tensor([float("nan")]), torch.tensor([1.0]))


def test_cli_rejects_bad_arguments():
    with pytest.raises(SystemExit):
        er.main(["--rows", "0"])
    with pytest.raises(SystemExit):
        er.main(["--step", "4", "--total-steps", "4"])


@pytest.mark.gpu
@pytest.mark.skipif(not has_b200(), reason="needs a B200")
def test_native_error_report_on_b200():
    res = er.report(config="c2", heads=2, seq=2048, rows=32)
    assert set(res["modes"]) == set(er.MODES) and res["rows"] == 32
    for mode, entry in res["modes"].items():
        m = entry["native_vs_fp32"]
        # FP8 attention on Gaussian V: a few percent relative RMSE against
        # exact FP32 (the reference's published CPU figures are 5.1-5.4 %)
        assert m["relative_rmse"] < 0.1 and m["cosine"] > 0.99, (mode, m)
