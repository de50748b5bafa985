"""Pin the C oracle to crosslane's own arithmetic, compiled from its sources into
oracle/_ref/libref.so (q8k_core.hpp, core.hpp, other_combine.hpp, route.cpp)."""
import numpy as np
import pytest

from oracle_lib import Q8K, bits, tie_probe


def test_half_all_encodings(orc, ref):
    for h in range(65536):
        a, b = orc.L.orc_half(h), ref.L.ref_half(h)
        if np.isnan(a):
            assert np.isnan(b)
        else:
            assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32), h


@pytest.mark.parametrize("case", ["normal", "zero", "tie", "wide", "signed_tie", "subnormal", "one_hot"])
def test_quant_block_bitexact(orc, ref, case):
    rng = np.random.default_rng(hash(case) % 2**32)
    n = 256 * 24
    x = {"normal": rng.standard_normal(n), "zero": np.zeros(n), "tie": tie_probe(n),
         "wide": rng.standard_normal(n) * np.exp(rng.uniform(-80, 80, n)),
         "signed_tie": np.tile(np.r_[2.0, -2.0, rng.uniform(-1, 1, 254)], 24),
         "subnormal": rng.standard_normal(n) * 1e-42,
         "one_hot": np.eye(256)[rng.integers(0, 256, 24)].ravel() * -3.5}[case].astype(np.float32)
    assert np.array_equal(orc.quantize(x), ref.quantize(x))


@pytest.mark.parametrize("qtype", [16, 17, 29])
@pytest.mark.parametrize("nb", [1, 6, 28])
def test_dot_bitexact(orc, ref, qtype, nb):
    rng = np.random.default_rng(qtype * 100 + nb)
    for trial in range(40):
        w = orc.synth_matrix(qtype, trial, 3, trial, trial % 3, 1, 256 * nb)
        x = (rng.standard_normal(256 * nb) * (1 + trial)).astype(np.float32)
        if trial % 5 == 0:
            x = tie_probe(256 * nb)
        qa = orc.quantize(x)
        assert bits(orc.dot(qtype, w, qa, nb)) == bits(ref.dot(qtype, w, qa, nb))


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_integer_lanes_random_bytes(orc, ref, qtype):
    rng = np.random.default_rng(7 + qtype)
    bb = {16: 66, 17: 74, 29: 56}[qtype]
    for trial in range(300):
        blk = rng.integers(0, 256, bb, dtype=np.uint8)
        qa = orc.quantize(rng.standard_normal(256).astype(np.float32))
        for lane in range(8):
            assert orc.integer_lane(qtype, blk, qa, lane) == ref.integer_lane(qtype, blk, qa, lane)


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_decode_sub_matches_reference_decoder(orc, ref, qtype):
    rng = np.random.default_rng(qtype)
    bb = {16: 66, 17: 74, 29: 56}[qtype]
    for trial in range(300):
        blk = rng.integers(0, 256, bb, dtype=np.uint8)
        if qtype != 29:
            blk[1] &= 0x7B  # finite scale
        for ib in range(8):
            qo, do, so = orc.decode_sub(qtype, blk, ib)
            qr, dr, sr = ref.decode_sub(qtype, blk, ib)
            assert np.array_equal(qo, qr) and np.array_equal(so, sr)
            assert bits(do) == bits(dr) or (np.isnan(do) and np.isnan(dr))


def test_swiglu_bitexact(orc, ref):
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(5000) * 8).astype(np.float32)
    u = (rng.standard_normal(5000) * 8).astype(np.float32)
    for limit in (0.0, 10.0):
        for a, b in zip(g, u):
            assert bits(orc.L.orc_swiglu(float(a), float(b), limit)) == bits(ref.L.ref_swiglu(float(a), float(b),
                                                                                               limit))


def test_combine_byte_oracle(orc, ref):
    """engine/strata/warm/other_combine_check.cpp:28-48: dims, pick counts, shuffled ids,
    signed zeros and subnormal rows; byte-identical to crosslane's other_combine."""
    rng = np.random.default_rng(72641)

    def value(n):
        b = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
        b = (b & 0x807FFFFF) | ((rng.integers(0, 190, n).astype(np.uint32)) << 23)
        return b.view(np.float32)

    for dim in (1, 7, 8, 9, 63, 256, 257, 4096):
        for n in (1, 2, 3, 6, 8, 16):
            ids = rng.permutation(n).astype(np.int32)
            w = value(n)
            shared = value(dim)
            rows = value(n * dim).reshape(n, dim)
            rows[:, 0] = np.where(np.arange(n) % 2, -0.0, 0.0)
            if dim > 1:
                rows[:, 1] = np.arange(1, n + 1, dtype=np.uint32).view(np.float32)
            assert np.array_equal(bits(orc.combine(ids, w, rows, shared)), bits(ref.combine(ids, w, rows, shared)))


def test_route_mode_b_matches_route_cpu(orc, ref):
    rng = np.random.default_rng(11)
    for trial in range(200):
        n, k = (384, 6) if trial % 2 else (64, 8)
        logits = (rng.standard_normal(n) * (1 + trial % 7)).astype(np.float32)
        if trial % 10 == 0:
            logits[:5] = 25.0  # softplus linear branch and exact ties
        bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
        scale = float(rng.uniform(0.5, 3.0))
        io, wo = orc.route_sqrt_softplus(logits, bias, k, scale)
        ir, wr = ref.route_cpu(logits, bias, k, scale)
        assert np.array_equal(io, ir) and np.array_equal(bits(wo), bits(wr))


def test_expert_chain_matches_reference(orc, ref):
    """One expert FFN end to end (quant, gate/up, SwiGLU, quant, down), both sides on
    the same ggml bytes, reference geometry 5120 x 2304 with clamp 10."""
    dim, ff = 5120, 2304
    rng = np.random.default_rng(5)
    for qtype in (16, 17, 29):
        g = orc.synth_matrix(qtype, 1, 0, qtype, 0, ff, dim)
        u = orc.synth_matrix(qtype, 1, 0, qtype, 1, ff, dim)
        d = orc.synth_matrix(qtype, 1, 0, qtype, 2, dim, ff)
        x = rng.standard_normal(dim).astype(np.float32)
        ho, yo = orc.expert(qtype, g, u, d, x, dim, ff, 10.0)
        hr, yr = ref.expert(qtype, g, u, d, x, dim, ff, 10.0, threads=4)
        assert np.array_equal(bits(ho), bits(hr)) and np.array_equal(bits(yo), bits(yr))


# ---- the timed CPU lane (oracle/liblane.so, AVX2) against the reference arithmetic ----

@pytest.fixture(scope="module")
def lane():
    import oracle_lib
    cl = oracle_lib.cpu_lane()
    if cl is None:
        pytest.skip("oracle/liblane.so not built")
    return cl


@pytest.mark.parametrize("qtype", [16, 17, 29])
@pytest.mark.parametrize("nb", [1, 6, 28])
def test_cpu_lane_dot_bitexact_to_reference(orc, ref, lane, qtype, nb):
    rng = np.random.default_rng(qtype * 31 + nb)
    bb = {16: 66, 17: 74, 29: 56}[qtype]
    for trial in range(60):
        if trial % 2:
            w = rng.integers(0, 256, bb * nb, dtype=np.uint8)  # arbitrary block bytes
            if qtype != 29:  # keep the fp16 super-scales finite
                for b in range(nb):
                    w[bb * b:bb * b + 2] = np.frombuffer(np.float16(rng.uniform(0.001, 0.1)).tobytes(), np.uint8)
            else:
                for b in range(nb):
                    hbits = int(np.float16(rng.uniform(0.001, 0.1)).view(np.uint16))
                    for j in range(4):  # super-scale nibbles in the top of the four scale words
                        w[bb * b + 49 + 2 * j] = (w[bb * b + 49 + 2 * j] & 0x0F) | (((hbits >> (4 * j)) & 15) << 4)
        else:
            w = orc.synth_matrix(qtype, trial, 5, trial, trial % 3, 1, 256 * nb)
        x = (rng.standard_normal(256 * nb) * (1 + trial)).astype(np.float32)
        if trial % 7 == 0:
            x = tie_probe(256 * nb)
        qa = ref.quantize(x)
        assert np.array_equal(lane.quantize(x), qa)
        assert bits(lane.dot(qtype, w, qa, nb)) == bits(ref.dot(qtype, w, qa, nb)), trial


def test_cpu_lane_layer_batch_bitexact_to_oracle(orc, lane):
    """A token-layer of 6 experts of mixed types through the batched lane equals the
    oracle's expert chain bit for bit (rows are independent; only the job order differs)."""
    dim, ff, seed = 2048, 768, 11
    types = [16, 17, 29, 16, 29, 17]
    mats = [[orc.synth_matrix(t, seed, 0, e, r, *((ff, dim) if r < 2 else (dim, ff))) for r in range(3)]
            for e, t in enumerate(types)]
    x = np.random.default_rng(3).standard_normal(dim).astype(np.float32)
    y, used = lane.experts(types, [m[0] for m in mats], [m[1] for m in mats], [m[2] for m in mats], x, dim, ff, 0.0,
                           threads=4)
    assert used == 4
    for e, t in enumerate(types):
        _, want = orc.expert(t, *mats[e], x, dim, ff)
        assert np.array_equal(bits(y[e]), bits(want)), e
