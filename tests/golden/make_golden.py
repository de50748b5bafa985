"""Regenerate tests/golden/*.npz from crosslane's own arithmetic (oracle/_ref/libref.so).

    make -C oracle && python tests/golden/make_golden.py

Inputs are the synthetic blocks of crosslane_b200/csrc/synth.h plus seeded activations;
outputs (Q8_K bytes, row dots, expert chains, combine, route_cpu) come from the
reference build only, never from the oracle under test.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_lib  # noqa: E402


def main():
    ref = oracle_lib.reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libref.so missing: build it with `make -C oracle` next to a crosslane checkout")
    gen = oracle_lib.Oracle()  # used only for the synthetic input bytes
    rng = np.random.default_rng(20261201)
    out = {}
    # Q8_K quantisation probes
    xq = np.concatenate([rng.standard_normal(512), np.zeros(256), oracle_lib.tie_probe(256),
                         rng.standard_normal(256) * 1e-41, np.r_[3.0, -3.0, rng.uniform(-1, 1, 254)]]).astype(np.float32)
    out["quant_x"] = xq
    out["quant_q"] = ref.quantize(xq)
    # row dots per type
    for qtype in (16, 17, 29):
        n, k = 24, 1024
        w = gen.synth_matrix(qtype, 555, 1, qtype, 0, n, k)
        x = (rng.standard_normal(k) * 2).astype(np.float32)
        q = ref.quantize(x)
        bb = {16: 66, 17: 74, 29: 56}[qtype] * (k // 256)
        y = np.array([ref.dot(qtype, np.ascontiguousarray(w[r * bb:(r + 1) * bb]), q, k // 256) for r in range(n)],
                     np.float32)
        out[f"mv{qtype}_w"], out[f"mv{qtype}_q"], out[f"mv{qtype}_y"] = w, q, y
    # one expert chain per type (dim 512, ff 256, clamp 10)
    for qtype in (16, 17, 29):
        dim, ff = 512, 256
        g = gen.synth_matrix(qtype, 9, 0, qtype, 0, ff, dim)
        u = gen.synth_matrix(qtype, 9, 0, qtype, 1, ff, dim)
        d = gen.synth_matrix(qtype, 9, 0, qtype, 2, dim, ff)
        x = rng.standard_normal(dim).astype(np.float32)
        h, y = ref.expert(qtype, g, u, d, x, dim, ff, 10.0, threads=1)
        out.update({f"ex{qtype}_g": g, f"ex{qtype}_u": u, f"ex{qtype}_d": d, f"ex{qtype}_x": x,
                    f"ex{qtype}_h": h, f"ex{qtype}_y": y})
    # combine
    ids = np.array([5, 1, 9, 3], np.int32)
    w = rng.uniform(0, 1, 4).astype(np.float32)
    rows = rng.standard_normal((4, 300)).astype(np.float32)
    shared = rng.standard_normal(300).astype(np.float32)
    out.update({"comb_ids": ids, "comb_w": w, "comb_rows": rows, "comb_shared": shared,
                "comb_out": ref.combine(ids, w, rows, shared)})
    # route_cpu (mode B)
    logits = rng.standard_normal((8, 384)).astype(np.float32)
    bias = (rng.standard_normal(384) * 0.1).astype(np.float32)
    rid, rw = zip(*[ref.route_cpu(logits[t], bias, 6, 2.5) for t in range(8)])
    out.update({"route_logits": logits, "route_bias": bias, "route_ids": np.array(rid), "route_w": np.array(rw)})
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_vectors.npz"))


if __name__ == "__main__":
    main()
