"""Exhaustive CPU proofs of the decode, modelled on crosslane's engine/strata/warm/mmvq_proof.cpp:13-34.

1. The oracle's lane integers (q8k_core.hpp restatement) agree with an independent
   per-32 decoder (core.hpp restatement) for every IQ2_XXS index x sign pair, every
   IQ2_XS 9-bit index x sign word, every IQ1_M index x delta x scale pair.
2. The GPU kernels' decode -- nibble-selector tables from the library, the packed
   IQ2_XXS sign bytes, byte permute (PTX prmt.b32 semantics), and both ways of forming
   lanes (the row-per-thread dp4a lanes of clb_rowdot.cuh and the mma.sync m16n8k32
   fragments with per-lane activation masks of clb_device.cuh) -- reproduces the
   oracle's lane integers exactly. The kernels' algorithm restated in numpy, on every code.
"""
import ctypes as C

import numpy as np
import pytest

import crosslane_b200 as cb

PRMT_IQ2_POS, PRMT_IQ2_NEG, PRMT_IQ1 = 0x002B1908, 0x00D5E7F8, 0x000100FF


def tables():
    out = np.zeros(2944, np.uint32)
    assert cb.lib.clb_decode_tables(out.ctypes.data_as(C.c_void_p), out.size) == 2944
    return {"xxs": out[0:256], "xs": out[256:768], "iq1": out[768:2816], "sign": out[2816:2944]}


def prmt(a, b, sel):
    """PTX prmt.b32 default mode, vectorised over numpy arrays."""
    src = (np.asarray(b, np.uint64) << 32) | np.asarray(a, np.uint64)
    sel = np.asarray(sel, np.uint64)
    out = np.zeros(np.broadcast(src, sel).shape, np.uint64)
    for i in range(4):
        s = (sel >> np.uint64(4 * i)) & np.uint64(15)
        byte = (src >> (np.uint64(8) * (s & np.uint64(7)))) & np.uint64(255)
        byte = np.where(s & np.uint64(8), np.where(byte & np.uint64(128), np.uint64(255), np.uint64(0)), byte)
        out |= byte << np.uint64(8 * i)
    return out.astype(np.uint32)


def s8(word):
    """uint32 -> 4 int8 values (little endian)."""
    return np.asarray(word, np.uint32).view(np.uint8).reshape(-1, 4).astype(np.int8).astype(np.int32)


def aux_to_signbytes(aux):
    """clb_pack.h's IQ2_XXS chunk re-planing of the u32 aux."""
    out = 0
    for j in range(4):
        out |= (((aux >> (7 * j)) & 127) | (((aux >> (28 + j)) & 1) << 7)) << (8 * j)
    return out


def gpu_group_decode(qtype, tb, blocks, c, t):
    """decode_group<T> of clb_device.cuh for chunk c, group t over an array of AoS blocks.
    Returns (lo int8x4 as int32[...,4], hi, scale, delta)."""
    n = len(blocks)
    if qtype == 16:
        # packed chunk: [4 grid bytes][4 sign bytes; bit 7 of byte j = sub-scale bit j]
        gw = blocks[:, 2 + 8 * c: 6 + 8 * c].copy().view(np.uint32)[:, 0]
        aux = blocks[:, 6 + 8 * c: 10 + 8 * c].copy().view(np.uint32)[:, 0]
        sw = np.array([aux_to_signbytes(int(a)) for a in aux], np.uint32)
        gi = (gw >> (8 * t)) & 0xFF
        si = (sw >> (8 * t)) & 0x7F
        sel = tb["xxs"][gi] | tb["sign"][si]
        lo = prmt(PRMT_IQ2_POS, PRMT_IQ2_NEG, sel)
        hi = prmt(PRMT_IQ2_POS, PRMT_IQ2_NEG, sel >> 16)
        scale = ((((sw & 0x80808080) | 0x08000000).astype(np.uint64) * 0x00204081 >> 27) & 0x1F).astype(np.uint32)
        delta = np.zeros(n, np.int64)
    elif qtype == 17:
        w = blocks[:, 2 + 8 * c + 4 * (t >> 1): 6 + 8 * c + 4 * (t >> 1)].copy().view(np.uint32)[:, 0]
        code = (w >> (16 * (t & 1))) & 0xFFFF
        sel = tb["xs"][code & 511] | tb["sign"][code >> 9]
        lo = prmt(PRMT_IQ2_POS, PRMT_IQ2_NEG, sel)
        hi = prmt(PRMT_IQ2_POS, PRMT_IQ2_NEG, sel >> 16)
        sb = blocks[:, 66 + c].astype(np.uint32)
        scale = (((sb >> (4 * (t >> 1))) & 15) << 1) | 1
        delta = np.zeros(n, np.int64)
    else:
        qsw = blocks[:, 4 * c: 4 * c + 4].copy().view(np.uint32)[:, 0]
        qh = blocks[:, 32 + 2 * c + (t >> 1)].astype(np.uint32)
        nib = (qh >> (4 * (t & 1))) & 15
        idx = ((qsw >> (8 * t)) & 0xFF) | ((nib & 7) << 8)
        sel = tb["iq1"][idx]
        lo = prmt(PRMT_IQ1, 0, sel)
        hi = prmt(PRMT_IQ1, 0, sel >> 16)
        scw = blocks[:, 48 + 2 * (c >> 1): 50 + 2 * (c >> 1)].copy().view(np.uint16)[:, 0].astype(np.uint32)
        scale = (((scw >> (6 * (c & 1) + 3 * (t >> 1))) & 7) << 1) | 1
        delta = np.where(nib & 8, -1, 1)
    return s8(lo), s8(hi), scale.astype(np.int64), delta.astype(np.int64)


def gpu_lane_ints(qtype, tb, blocks, q):
    """The kernel's per-lane integer sums of one 256-block, via the MMA fragment model.

    Thread (g, t) supplies A rows g/g+8 at k-slots 4t.. (lane 2t) and 16+4t.. (lane 2t+1)
    and B column g with the activation masked to its lane; D = A @ B gives every row's 8
    lane sums of one chunk. Here a "row" is one block of `blocks`.
    """
    n = len(blocks)
    main = np.zeros((n, 8), np.int64)
    dl = np.zeros((n, 8), np.int64)
    for c in range(8):
        q32 = q[32 * c: 32 * c + 32].astype(np.int64)
        A = np.zeros((n, 32), np.int64)
        scale = np.zeros((n, 4), np.int64)
        delta = np.zeros((n, 4), np.int64)
        for t in range(4):
            lo, hi, sc, de = gpu_group_decode(qtype, tb, blocks, c, t)
            A[:, 4 * t: 4 * t + 4] = lo
            A[:, 16 + 4 * t: 16 + 4 * t + 4] = hi
            scale[:, t] = sc
            delta[:, t] = de
        B = np.zeros((32, 8), np.int64)
        for g in range(8):
            for t in range(4):
                if g == 2 * t:
                    B[4 * t: 4 * t + 4, g] = q32[8 * t: 8 * t + 4]
                if g == 2 * t + 1:
                    B[16 + 4 * t: 16 + 4 * t + 4, g] = q32[8 * t + 4: 8 * t + 8]
        D = A @ B
        for lane in range(8):
            t = lane // 2
            main[:, lane] += scale[:, t] * D[:, lane]
            lsum = int(q32[4 * lane: 4 * lane + 4].sum())
            dl[:, lane] += scale[:, t] * delta[:, t] * lsum
    return main, dl


def gpu_row_lane_ints(qtype, tb, blocks, q):
    """block_lanes<T> of clb_rowdot.cuh: one thread decodes all 4 groups of every chunk,
    lane 2j += scale * dp4a(lo_j, q lane 2j), lane 2j+1 += scale * dp4a(hi_j, q lane 2j+1);
    IQ1_M delta lanes += (+-scale) * sum of the lane's 4 activations."""
    n = len(blocks)
    main = np.zeros((n, 8), np.int64)
    dl = np.zeros((n, 8), np.int64)
    for c in range(8):
        q32 = q[32 * c: 32 * c + 32].astype(np.int64)
        for j in range(4):
            lo, hi, sc, de = gpu_group_decode(qtype, tb, blocks, c, j)
            main[:, 2 * j] += sc * (lo * q32[8 * j: 8 * j + 4]).sum(axis=1)
            main[:, 2 * j + 1] += sc * (hi * q32[8 * j + 4: 8 * j + 8]).sum(axis=1)
            dl[:, 2 * j] += sc * de * int(q32[8 * j: 8 * j + 4].sum())
            dl[:, 2 * j + 1] += sc * de * int(q32[8 * j + 4: 8 * j + 8].sum())
    return main, dl


def exhaustive_blocks(qtype, rng):
    """Blocks covering every grid index x sign word (IQ2) or index x delta x scale (IQ1_M)."""
    bb = {16: 66, 17: 74, 29: 56}[qtype]
    if qtype == 16:
        cases = [(i, s) for i in range(256) for s in range(128)]
    elif qtype == 17:
        cases = list(range(512 * 128))
    else:
        cases = [(i, d, s) for i in range(2048) for d in range(2) for s in range(64) if (i + s) % 4 == 0] + \
                [(i, d, s) for i in range(2048) for d in range(2) for s in range(64) if (i + s) % 4 != 0][::3]
    blocks = rng.integers(0, 256, (len(cases), bb), dtype=np.uint8)
    blocks[:, 0:2] = np.frombuffer(np.uint16(0x3555).tobytes(), np.uint8)
    for r, case in enumerate(cases):
        b = blocks[r]
        for c in range(8):
            if qtype == 16:
                i, s = case
                b[2 + 8 * c: 6 + 8 * c] = (i + c) % 256
                aux = ((c * 5 + s) % 16) << 28
                for j in range(4):
                    aux |= ((s + 37 * j) % 128) << (7 * j)
                b[6 + 8 * c: 10 + 8 * c] = np.frombuffer(np.uint32(aux).tobytes(), np.uint8)
            elif qtype == 17:
                for j in range(4):
                    code = (case + 7919 * (4 * c + j)) % 65536
                    b[2 + 8 * c + 2 * j: 4 + 8 * c + 2 * j] = np.frombuffer(np.uint16(code).tobytes(), np.uint8)
                b[66 + c] = (case + 31 * c) % 256
            else:
                i, d, s = case
                for j in range(4):
                    b[4 * c + j] = (i + 97 * j) & 255
                for j in range(2):
                    lo = ((i + 97 * 2 * j) >> 8) & 7 | (d << 3)
                    hi = ((i + 97 * (2 * j + 1)) >> 8) & 7 | ((1 - d) << 3)
                    b[32 + 2 * c + j] = lo | (hi << 4)
        if qtype == 29:
            i, d, s = case
            for j in range(4):
                word = (s | (((s + 11 * j) % 64) << 6)) | (0x3 << 12 if j < 2 else 0x5 << 12)
                b[48 + 2 * j: 50 + 2 * j] = np.frombuffer(np.uint16(word).tobytes(), np.uint8)
    return blocks


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_lane_integers_match_independent_decoder(orc, qtype):
    """Oracle lane integers == sum over the independent per-32 decode (both restate the reference)."""
    rng = np.random.default_rng(qtype)
    blocks = exhaustive_blocks(qtype, rng)[::97]  # every case is covered in the GPU-model test below
    x = rng.standard_normal(256).astype(np.float32) * 2
    qb = orc.quantize(x)
    qs = qb[4:260].view(np.int8).astype(np.int64)
    for blk in blocks:
        blk = np.ascontiguousarray(blk)
        lane_main = np.zeros(8, np.int64)
        lane_delta = np.zeros(8, np.int64)
        for ib in range(8):
            qv, d, s = orc.decode_sub(qtype, blk, ib)
            for lane in range(8):
                pos = slice(32 * ib + 4 * lane, 32 * ib + 4 * lane + 4)
                sub = qv[4 * lane: 4 * lane + 4].astype(np.int64)
                sc = s[0] if lane < 4 else s[1]
                if qtype == 29:
                    codes = (sub - np.where(sub % 8 == 7, -1, 1)) // 8  # q = 8*code + delta
                    dlt = sub - 8 * codes
                    lane_main[lane] += sc * int((codes * qs[pos]).sum())
                    lane_delta[lane] += sc * int((dlt * qs[pos]).sum())
                else:
                    lane_main[lane] += sc * int((sub * qs[pos]).sum())
        for lane in range(8):
            m, dd = orc.integer_lane(qtype, blk, qb, lane)
            assert m == lane_main[lane]
            if qtype == 29:
                assert dd == lane_delta[lane]


@pytest.mark.parametrize("qtype", [16, 17, 29])
def test_gpu_decode_model_exhaustive(orc, qtype):
    """The kernel's prmt + MMA-fragment decode equals the oracle's lane integers on every code."""
    tb = tables()
    rng = np.random.default_rng(100 + qtype)
    blocks = exhaustive_blocks(qtype, rng)
    for probe in range(2):
        x = rng.standard_normal(256).astype(np.float32) * 3 if probe == 0 else \
            np.array([127.0 if i == 0 else (i % 31) - 15 + 0.5 for i in range(256)], np.float32)
        qb = orc.quantize(x)
        qs = qb[4:260].view(np.int8)
        main, delta = gpu_lane_ints(qtype, tb, blocks, qs)
        rmain, rdelta = gpu_row_lane_ints(qtype, tb, blocks, qs)
        assert np.array_equal(main, rmain) and (qtype != 29 or np.array_equal(delta, rdelta))
        sample = range(0, len(blocks), max(1, len(blocks) // 400))
        for r in sample:
            blk = np.ascontiguousarray(blocks[r])
            for lane in range(8):
                m, d = orc.integer_lane(qtype, blk, qb, lane)
                assert main[r, lane] == m, (r, lane)
                if qtype == 29:
                    assert delta[r, lane] == d


def test_tables_match_codebooks(ref):
    """Selector tables decode back to crosslane's own codebooks (q8k_tables.inc) and ksigns."""
    tb = tables()
    for i in range(256):
        g = ref.L.ref_grid(16, i)
        sym = [(int(tb["xxs"][i]) >> (4 * j)) & 15 for j in range(8)]
        assert [[8, 25, 43][s] for s in sym] == [(g >> (8 * j)) & 255 for j in range(8)]
    for i in range(512):
        g = ref.L.ref_grid(17, i)
        sym = [(int(tb["xs"][i]) >> (4 * j)) & 15 for j in range(8)]
        assert [[8, 25, 43][s] for s in sym] == [(g >> (8 * j)) & 255 for j in range(8)]
    for i in range(2048):
        g = ref.L.ref_grid(29, i)
        sym = [(int(tb["iq1"][i]) >> (4 * j)) & 15 for j in range(8)]
        assert [s - 1 for s in sym] == [int(np.int8(np.uint8((g >> (8 * j)) & 255))) for j in range(8)]
    for s in range(128):
        k = ref.L.ref_ksigns(s)
        assert all(((int(tb["sign"][s]) >> (4 * j)) & 15) == (4 if (k >> j) & 1 else 0) for j in range(8))


def test_compact_codebook_assertion():
    """crosslane engine/strata/sycl/moe/iq2_codebook.hpp:23-29: every IQ2 magnitude is one of
    {8, 25, 43}, i.e. 8 + 17c + (c >> 1) for a 2-bit symbol c -- the premise of the
    3-symbol byte-permute decode."""
    tb = tables()
    for name in ("xxs", "xs"):
        for v in tb[name]:
            for j in range(8):
                c = (int(v) >> (4 * j)) & 15
                assert c <= 2 and 8 + 17 * c + (c >> 1) in (8, 25, 43)
