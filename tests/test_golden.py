"""The oracle against golden vectors computed by crosslane's own arithmetic
(tests/golden/make_golden.py over oracle/_ref). Runs where the checkout is absent."""
import os

import numpy as np
import pytest

from oracle_lib import bits

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_vectors.npz")


@pytest.fixture(scope="module")
def gv():
    return np.load(GOLDEN)


def test_quant(orc, gv):
    assert np.array_equal(orc.quantize(gv["quant_x"]), gv["quant_q"])


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_row_dots(orc, gv, qtype):
    y = orc.mv(qtype, gv[f"mv{qtype}_w"], gv[f"mv{qtype}_q"], 24, 1024)
    assert np.array_equal(bits(y), bits(gv[f"mv{qtype}_y"]))


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_expert_chain(orc, gv, qtype):
    h, y = orc.expert(qtype, gv[f"ex{qtype}_g"], gv[f"ex{qtype}_u"], gv[f"ex{qtype}_d"], gv[f"ex{qtype}_x"], 512, 256,
                      10.0)
    assert np.array_equal(bits(h), bits(gv[f"ex{qtype}_h"]))
    assert np.array_equal(bits(y), bits(gv[f"ex{qtype}_y"]))


def test_combine(orc, gv):
    out = orc.combine(gv["comb_ids"], gv["comb_w"], gv["comb_rows"], gv["comb_shared"])
    assert np.array_equal(bits(out), bits(gv["comb_out"]))


def test_route_cpu(orc, gv):
    for t in range(8):
        ids, w = orc.route_sqrt_softplus(gv["route_logits"][t], gv["route_bias"], 6, 2.5)
        assert np.array_equal(ids, gv["route_ids"][t]) and np.array_equal(bits(w), bits(gv["route_w"][t]))


def test_synthetic_inputs_stable(orc, gv):
    """The synthetic generator still produces the committed input bytes."""
    assert np.array_equal(orc.synth_matrix(16, 555, 1, 16, 0, 24, 1024), gv["mv16_w"])
    assert np.array_equal(orc.synth_matrix(29, 9, 0, 29, 2, 512, 256), gv["ex29_d"])
