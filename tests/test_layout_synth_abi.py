"""CPU tests of the library surface that needs no GPU: packed layout, synthetic inputs,
host routing, and the exported C ABI."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import crosslane_b200 as cb
from oracle_lib import bits

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# ---------------------------------------------------------------- packed layout

@pytest.mark.parametrize("qtype", [16, 17, 29])
@pytest.mark.parametrize("n,k", [(1, 256), (3, 512), (16, 256), (33, 768), (96, 2048)])
def test_pack_roundtrip(qtype, n, k):
    rng = np.random.default_rng(n * k + qtype)
    bb = cb.BLOCK_BYTES[qtype]
    raw = rng.integers(0, 256, n * (k // 256) * bb, dtype=np.uint8).reshape(-1, bb)
    if qtype == 29:
        raw[:, 55] &= 0xBF  # fp16 bit 14 (exponent MSB) lives in word 3's top nibble: keep finite
    else:
        raw[:, 1] &= 0x7B
    raw = raw.ravel()
    packed = cb.pack(qtype, n, k, raw)
    assert packed.size == cb.packed_bytes(qtype, n, k) >= raw.size
    assert packed.size - raw.size < 3 * 256
    assert np.array_equal(cb.unpack(qtype, n, k, packed), raw)


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_pack_rejects_nonfinite_scale(qtype):
    bb = cb.BLOCK_BYTES[qtype]
    raw = np.zeros(4 * bb, np.uint8)
    if qtype == 29:
        for j in range(4):  # fp16 0x7c00 scattered over the scale words' top nibbles
            raw[bb + 49 + 2 * j] = ((0x7C00 >> (4 * j)) & 15) << 4
    else:
        raw[bb + 1] = 0x7C
    with pytest.raises(cb.ClbError):
        cb.pack(qtype, 4, 256, raw)


def test_pack_geometry_checks():
    assert cb.packed_bytes(16, 0, 256) == 0
    assert cb.packed_bytes(16, 4, 300) == 0
    assert cb.packed_bytes(12, 4, 256) == 0
    with pytest.raises(cb.ClbError):
        cb.pack(16, 4, 256, np.zeros(10, np.uint8))


def aux_to_signbytes(aux):
    out = 0
    for j in range(4):
        out |= (((aux >> (7 * j)) & 127) | (((aux >> (28 + j)) & 1) << 7)) << (8 * j)
    return out


@pytest.mark.parametrize("qtype", [16, 17])
def test_pack_plane_order(qtype):
    """Body piece q of block b of row r lands at ((b*4 + q)*n + r)*16 (clb_types.h); an
    IQ2_XXS chunk's u32 aux becomes 4 sign bytes carrying the sub-scale bits on top."""
    n, k = 5, 512
    bb = cb.BLOCK_BYTES[qtype]
    raw = (np.arange(n * 2 * bb, dtype=np.uint32) * 7 + 3).astype(np.uint8)
    raw.reshape(-1, bb)[:, 1] &= 0x7B
    packed = cb.pack(qtype, n, k, raw)
    blk = raw.reshape(n, 2, bb)
    for r in range(n):
        for b in range(2):
            for q in range(4):
                off = ((b * 4 + q) * n + r) * 16
                want = blk[r, b, 2 + 16 * q: 18 + 16 * q].copy()
                if qtype == 16:
                    for c in range(2):
                        aux = int(want[8 * c + 4: 8 * c + 8].view(np.uint32)[0])
                        want[8 * c + 4: 8 * c + 8] = np.frombuffer(np.uint32(aux_to_signbytes(aux)).tobytes(), np.uint8)
                assert np.array_equal(packed[off:off + 16], want)


# ---------------------------------------------------------------- synthetic inputs

def test_scale_table(orc):
    t = orc.scale_table().view(np.float16).astype(np.float64)
    assert np.all(np.diff(t) >= 0) and t[0] > 0
    assert abs(np.median(t) - 0.0067449) < 2e-5  # median of |N(0,1)| * 0.01
    assert abs(t.mean() - 0.01 * np.sqrt(2 / np.pi)) < 5e-5


def test_synth_deterministic_and_distinct(orc):
    a = orc.synth_matrix(16, 1, 2, 3, 0, 8, 512)
    assert np.array_equal(a, orc.synth_matrix(16, 1, 2, 3, 0, 8, 512))
    assert not np.array_equal(a, orc.synth_matrix(16, 1, 2, 3, 1, 8, 512))
    assert not np.array_equal(a, orc.synth_matrix(16, 1, 2, 4, 0, 8, 512))
    blocks = orc.synth_matrix(17, 5, 0, 0, 2, 256, 1024).reshape(-1, 74)
    counts = np.bincount(blocks[:, 2:66].ravel(), minlength=256)
    assert counts.min() > 0.8 * counts.mean()  # code bytes uniform


def test_type_policies(orc):
    assert {orc.expert_type(0, 9, 3, e) for e in range(384)} == {16}
    assert [orc.expert_type(1, 9, 0, e) for e in (0, 127, 128, 255, 256, 383)] == [16, 16, 17, 17, 29, 29]
    mix = np.bincount([orc.expert_type(2, 9, lay, e) for lay in range(40) for e in range(384)], minlength=30)
    assert all(abs(mix[t] / 15360 - 1 / 3) < 0.02 for t in (16, 17, 29))


# ---------------------------------------------------------------- host routing

def test_route_host_mode_a(orc):
    rng = np.random.default_rng(4)
    for trial in range(300):
        logits = rng.standard_normal(384).astype(np.float32)
        if trial % 9 == 0:
            logits[[3, 50, 7]] = 4.0
        ids, w = cb.route_host(0, logits, 6)
        oi, ow = orc.route_sigmoid(logits, 6)
        assert np.array_equal(ids, oi)
        assert np.array_equal(bits(w), bits(ow))
        assert abs(float(w.sum()) - 1.0) < 1e-6
    logits = np.zeros(384, np.float32)
    assert list(cb.route_host(0, logits, 6)[0]) == [0, 1, 2, 3, 4, 5]
    for k in (1, 2, 8, 16):  # one-pass top-k keeps the arg-max order for every k
        logits = rng.standard_normal(100).astype(np.float32)
        logits[[5, 60, 61]] = 3.0
        ids, w = cb.route_host(0, logits, k)
        oi, ow = orc.route_sigmoid(logits, k)
        assert np.array_equal(ids, oi) and np.array_equal(bits(w), bits(ow))


def test_route_host_mode_b(orc):
    rng = np.random.default_rng(5)
    for trial in range(200):
        logits = (rng.standard_normal(384) * 3).astype(np.float32)
        bias = (rng.standard_normal(384) * 0.2).astype(np.float32)
        ids, w = cb.route_host(1, logits, 6, bias=bias, scale=2.5)
        oi, ow = orc.route_sqrt_softplus(logits, bias, 6, 2.5)
        assert np.array_equal(ids, oi)
        assert np.abs(bits(w).astype(np.int64) - bits(ow).astype(np.int64)).max() <= 2


def test_route_host_rejects_bad_input():
    bad = np.zeros(384, np.float32)
    bad[3] = np.inf
    with pytest.raises(cb.ClbError):
        cb.route_host(0, bad, 6)
    with pytest.raises(cb.ClbError):
        cb.route_host(0, np.zeros(4, np.float32), 6)


# ---------------------------------------------------------------- exported ABI

def declared_functions():
    text = open(os.path.join(ROOT, "include", "crosslane_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(clb_[a-z0-9_]+)\s*\(", text)
    return sorted(set(n for n in names if not n.endswith("_fn")))


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(cb._capi.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 28
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(cb._capi.SIGNATURES), set(names) - set(cb._capi.SIGNATURES)


def test_abi_version_and_sizes():
    assert cb.lib.clb_abi_version() == 1
    assert C.sizeof(cb._capi.ErrorV1) == 516
    assert C.sizeof(cb._capi.BankConfigV1) == 64
    assert cb.lib.clb_q8k_activation_bytes(7168) == 28 * 292
    assert cb.lib.clb_q8k_activation_bytes(100) == 0


def test_library_has_sm100a_code():
    """The shared library embeds sm_100a device code (cubin ELF marker), not PTX only."""
    blob = open(cb._capi.LIB_PATH, "rb").read()
    assert b"sm_100a" in blob


def test_bank_create_rejects_bad_config():
    err = cb._capi.ErrorV1()
    h = C.c_void_p()
    cfg = cb._capi.BankConfigV1(device=0, n_layers=1, n_experts=8, dim=300, ff=256, max_picks=6)
    rc = cb.lib.clb_bank_create(C.byref(cfg), C.byref(h), C.byref(err))
    assert rc != 0 and not h.value and err.message


def test_device_primitives_validate_before_launch():
    assert cb.lib.clb_q8k_quantize(None, None, 256, None) == cb._capi.CLB_E_INVALID
    assert cb.lib.clb_q8k_mv(12, None, None, None, 1, 256, None) == cb._capi.CLB_E_INVALID
    assert cb.lib.clb_q8k_activate(None, None, None, 1, 0.0, None) == cb._capi.CLB_E_INVALID
    assert cb.lib.clb_route_device(0, None, 384, 6, 1, None, None, None) == cb._capi.CLB_E_INVALID
