"""The allocation-free expert entry point (clb_expert_forward_noalloc).

Some callers of the lane cannot call cudaMalloc -- a serving loop that must not risk an
allocation's device synchronisation, a plugin whose device memory is owned by another
allocator. This entry point takes packed
weights, x and y from the caller and keeps its own intermediates in a fixed array inside
the library. Here its output is checked against the bank's warm_compute on the same
expert and against the CPU oracle's expert, twice in a row (the second call reuses the
array with the first call's contents still in it), at the parity tolerance used
throughout the GPU tests; also at the largest shape the array covers (dim 16384, ff 8192).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import max_abs_rel, rel_l2

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
MAX_ABS_REL = 5e-3


def _call(cb, qtype, d_gate, d_up, d_down, d_x, d_y, dim, ff, limit):
    err = cb._capi.ErrorV1()
    rc = cb.lib.clb_expert_forward_noalloc(qtype, C.c_void_p(d_gate.data_ptr()), C.c_void_p(d_up.data_ptr()),
                                           C.c_void_p(d_down.data_ptr()), C.c_void_p(d_x.data_ptr()),
                                           C.c_void_p(d_y.data_ptr()), dim, ff, limit, None, C.byref(err))
    return rc, err.message.decode()


@pytest.mark.parametrize("qtype,dim,ff", [(16, 7168, 1536), (17, 7168, 1536), (29, 7168, 1536), (16, 16384, 8192)])
def test_noalloc_matches_bank_compute(cuda, orc, qtype, dim, ff):
    import crosslane_b200 as cb
    torch = cuda
    limit, seed = 0.0, 314
    mats = [orc.synth_matrix(qtype, seed, 0, 2, role, n, k)
            for role, (n, k) in enumerate([(ff, dim), (ff, dim), (dim, ff)])]
    bank = cb.ExpertBank(n_layers=1, n_experts=4, dim=dim, ff=ff, max_picks=1, limit=limit)
    try:
        for role, m in enumerate(mats):
            bank.load_matrix(0, 2, role, qtype, m)
        packed = [torch.from_numpy(cb.pack(qtype, n, k, m)).cuda()
                  for m, (n, k) in zip(mats, [(ff, dim), (ff, dim), (dim, ff)])]
        rng = np.random.default_rng(qtype)
        for call in range(2):
            x = rng.standard_normal(dim).astype(np.float32)
            want = bank.warm_compute(0, 2, x)
            _, ref_y = orc.expert(qtype, mats[0], mats[1], mats[2], x, dim, ff, limit)
            d_x = torch.from_numpy(x).cuda()
            d_y = torch.full((dim,), float("nan"), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            rc, msg = _call(cb, qtype, *packed, d_x, d_y, dim, ff, limit)
            assert rc == 0, msg
            torch.cuda.synchronize()
            got = d_y.cpu().numpy()
            assert np.all(np.isfinite(got)), f"call {call}"
            assert rel_l2(got, want) <= REL_L2 and max_abs_rel(got, want) <= MAX_ABS_REL, f"call {call}"
            assert rel_l2(got, ref_y) <= REL_L2 and max_abs_rel(got, ref_y) <= MAX_ABS_REL, f"call {call} vs oracle"
    finally:
        bank.close()


def test_noalloc_rejects_shapes_beyond_scratch(cuda):
    import crosslane_b200 as cb
    torch = cuda
    buf = torch.zeros(16, dtype=torch.float32, device="cuda")
    rc, msg = _call(cb, 16, buf, buf, buf, buf, buf, 16384 + 256, 1536, 0.0)
    assert rc == cb._capi.CLB_E_UNSUPPORTED and "16384" in msg
    rc, msg = _call(cb, 16, buf, buf, buf, buf, buf, 7168, 8192 + 256, 0.0)
    assert rc == cb._capi.CLB_E_UNSUPPORTED and "8192" in msg
