"""Strata pack ingestion (weight_source.hpp:1-5, pack_source.cpp:144-185): the library's
reader applies the reference's checks and returns the stored bytes; a bank loads every
placed expert matrix from a pack and its outputs equal the CPU oracle's on the same raw
ggml bytes (exact order: bit for bit), including mixed types within an expert and the
reference model's geometry (hidden 5120, intermediate 2304, SwiGLU clamp 10)."""
import os
import struct

import numpy as np
import pytest

import crosslane_b200 as cb
from crosslane_b200.strata_pack import StrataPack, expert_tensor, write_pack

BLOCK = {"IQ2_XXS": 66, "IQ2_XS": 74, "IQ1_M": 56}
GGML = {"IQ2_XXS": 16, "IQ2_XS": 17, "IQ1_M": 29}


def matrix_bytes(rng, dtype, n, k):
    """Random ggml blocks with a finite fp16 super-scale (+-0.333, as crosslane's fixture)."""
    bs = BLOCK[dtype]
    raw = bytearray(rng.integers(0, 256, n * (k // 256) * bs, dtype=np.uint8).tobytes())
    for b in range(n * (k // 256)):
        at, half = b * bs, (0x3555 if b % 2 else 0xB555)
        if dtype != "IQ1_M":
            struct.pack_into("<H", raw, at, half)
        else:
            for word in range(4):
                pos = at + 48 + 2 * word
                sc = struct.unpack_from("<H", raw, pos)[0]
                struct.pack_into("<H", raw, pos, (sc & 4095) | (((half >> (4 * word)) & 15) << 12))
    return bytes(raw)


def make_pack(path, layers, experts, dim, ff, sigs, seed=0, limit=0.0):
    rng = np.random.default_rng(seed)
    tensors, raw = [], {}
    for l in range(layers):
        for e in range(experts):
            sig = sigs[(l * experts + e) % len(sigs)]
            for role in range(3):
                n, k = (dim, ff) if role == 2 else (ff, dim)
                data = matrix_bytes(rng, sig[role], n, k)
                raw[l, e, role] = (sig[role], data)
                tensors.append((expert_tensor(l, e, role), sig[role], data, (n, k)))
    tensors.append(("layers.0.ffn.norm.weight", "F32", np.ones(dim, np.float32).tobytes(), (dim,)))
    write_pack(str(path), tensors, {"hidden_size": dim, "moe_intermediate_size": ff, "n_routed_experts": experts,
                                    "num_hidden_layers": layers, "swiglu_limit": limit})
    return raw


SIGS = [("IQ2_XXS", "IQ2_XXS", "IQ2_XXS"), ("IQ1_M", "IQ1_M", "IQ1_M"), ("IQ2_XS", "IQ2_XS", "IQ1_M"),
        ("IQ2_XXS", "IQ2_XXS", "IQ2_XS")]


def test_reader(tmp_path):
    raw = make_pack(tmp_path / "p", 2, 3, 512, 256, SIGS)
    with StrataPack(str(tmp_path / "p")) as pk:
        assert pk.meta("hidden_size") == "512" and pk.meta("format") == "gguf" and pk.meta("absent") is None
        for (l, e, role), (dtype, data) in raw.items():
            name = expert_tensor(l, e, role)
            info = pk.tensor(name)
            assert info[0] == dtype and info[1] == len(data)
            assert info[2] == ((512, 256) if role == 2 else (256, 512))
            assert pk.read(name) == data
            assert pk.read(name, 66, 100) == data[66:166]
        assert pk.tensor("missing") is None
        with pytest.raises(cb.ClbError):
            pk.read(expert_tensor(0, 0, 0), 10, 10 ** 9)


@pytest.mark.parametrize("case", ["no_model_dir", "not_gguf", "duplicate", "unknown_shard", "past_end", "gap",
                                  "bad_line", "missing_shard"])
def test_reader_rejects(tmp_path, case):
    d = tmp_path / "p"
    make_pack(d, 1, 1, 256, 256, SIGS)
    ds4, tens = (d / "ds4.txt").read_text(), (d / "tensors.txt").read_text()
    if case == "no_model_dir":
        ds4 = "\n".join(x for x in ds4.splitlines() if not x.startswith("model_dir")) + "\n"
    elif case == "not_gguf":
        ds4 = ds4.replace("format gguf", "format safetensors")
    elif case == "duplicate":
        tens += tens.splitlines()[1] + "\n"
    elif case == "unknown_shard":
        tens = tens.replace(" IQ2_XXS 0 ", " IQ2_XXS 3 ", 1)
    elif case == "past_end":  # the last tensor of the shard one byte longer
        last = tens.splitlines()[-1]
        line = last.split()
        line[5] = str(int(line[5]) + 1)
        tens = tens.replace(last, " ".join(line))
    elif case == "gap":
        tens = "file 2 other.gguf\n" + tens
    elif case == "bad_line":
        tens += "t broken IQ2_XXS zero\n"
    elif case == "missing_shard":
        os.remove(d / "model.gguf")
    (d / "ds4.txt").write_text(ds4)
    (d / "tensors.txt").write_text(tens)
    with pytest.raises(cb.ClbError):
        StrataPack(str(d))


def oracle_expert(orc, raw, l, e, x, dim, ff, limit):
    (tg, g), (tu, u), (td, dn) = (raw[l, e, r] for r in range(3))
    q = orc.quantize(x)
    gv = orc.mv(GGML[tg], np.frombuffer(g, np.uint8), q, ff, dim)
    uv = orc.mv(GGML[tu], np.frombuffer(u, np.uint8), q, ff, dim)
    h = orc.swiglu(gv, uv, limit)
    return orc.mv(GGML[td], np.frombuffer(dn, np.uint8), orc.quantize(h), dim, ff)


@pytest.mark.gpu
@pytest.mark.parametrize("dim,ff,limit", [(768, 512, 0.0), (5120, 2304, 10.0)])
def test_bank_loads_pack_bit_exact(cuda, orc, tmp_path, dim, ff, limit):
    layers, experts = (2, 4) if dim == 768 else (1, 2)
    raw = make_pack(tmp_path / "p", layers, experts, dim, ff, SIGS, limit=limit)
    bank = cb.ExpertBank(n_layers=layers, n_experts=experts, dim=dim, ff=ff, max_picks=experts, device=0, limit=limit,
                         exact_order=True)
    try:
        with StrataPack(str(tmp_path / "p")) as pk:
            bank.load_strata_pack(pk)
        rng = np.random.default_rng(3)
        for l in range(layers):
            x = rng.standard_normal(dim).astype(np.float32)
            ids = np.arange(experts, dtype=np.int32)
            got = bank.warm_compute_many(l, ids, x)
            for i, e in enumerate(ids):
                want = oracle_expert(orc, raw, l, int(e), x, dim, ff, limit)
                assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32)), (l, e)
    finally:
        bank.close()


@pytest.mark.gpu
def test_bank_pack_checks(cuda, tmp_path):
    make_pack(tmp_path / "p", 1, 2, 512, 256, SIGS)
    with StrataPack(str(tmp_path / "p")) as pk:
        bank = cb.ExpertBank(n_layers=1, n_experts=2, dim=768, ff=256, max_picks=2, device=0)
        try:
            with pytest.raises(cb.ClbError):  # hidden_size differs
                bank.load_strata_pack(pk)
        finally:
            bank.close()
        bank = cb.ExpertBank(n_layers=2, n_experts=2, dim=512, ff=256, max_picks=2, device=0)
        try:
            with pytest.raises(cb.ClbError):  # the pack has one layer
                bank.load_strata_pack(pk)
        finally:
            bank.close()
