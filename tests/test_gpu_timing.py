"""CLB_BANK_TIMING: device spans of the synchronous host entry points, one JSON line per call
on stderr (schema clb-cuda-timing-v1) and the last span through clb_bank_last_timing."""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb(cuda):
    import crosslane_b200
    return crosslane_b200


def lines(err):
    return [json.loads(s) for s in err.splitlines() if s.startswith('{"schema":"clb-cuda-timing-v1"')]


def test_timing_spans(cb, orc, capfd):
    dim, ff, E, k = 1024, 512, 16, 4
    bank = cb.ExpertBank(n_layers=2, n_experts=E, dim=dim, ff=ff, max_picks=k, device=0, timing=True)
    try:
        bank.fill_synthetic(5, 2)
        rng = np.random.default_rng(0)
        ids, w = orc.route_sigmoid(rng.standard_normal(E).astype(np.float32), k)
        x = rng.standard_normal(dim).astype(np.float32)
        capfd.readouterr()
        bank.layer_execute(1, ids, w, x)
        t = bank.last_timing()
        assert t["ns"] > 0 and t["layer"] == 1 and t["layers"] == 1 and t["picks"] == k
        assert t["h2d_bytes"] == dim * 4 + k * 8 and t["d2h_bytes"] == dim * 4
        T = 6
        h = rng.standard_normal((T, dim)).astype(np.float32)
        lg = rng.standard_normal((2, T, E)).astype(np.float32)
        bank.stack_batch(0, 2, h, lg)
        t = bank.last_timing()
        assert t["layers"] == 2 and t["picks"] == 2 * T * k and t["d2h_bytes"] == T * dim * 4
        got = lines(capfd.readouterr().err)
        assert [g["call"] for g in got] == ["layer_execute", "stack_batch"]
        assert all(g["lane"] == "cuda" and g["device"] == 0 and g["ns"] > 0 for g in got)
    finally:
        bank.close()


def test_no_timing_lines_by_default(cb, orc, capfd):
    dim, ff, E, k = 1024, 512, 8, 2
    bank = cb.ExpertBank(n_layers=1, n_experts=E, dim=dim, ff=ff, max_picks=k, device=0)
    try:
        bank.fill_synthetic(5, 0)
        capfd.readouterr()
        bank.layer_execute(0, np.array([1, 4], np.int32), np.array([0.5, 0.5], np.float32), np.ones(dim, np.float32))
        assert lines(capfd.readouterr().err) == [] and bank.last_timing()["ns"] == 0
    finally:
        bank.close()
