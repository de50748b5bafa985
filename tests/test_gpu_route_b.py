"""Device-side routing of the MoE block: the router GEMV against an fp64
reference, crosslane's route_cpu (mode 1) on the device against the host restatement
(clb_route_host, the oracle's route_cpu) bit for bit, and the whole MoE block on the device
(router -> route -> experts -> combine, no host round trip) against the oracle layer."""
import numpy as np
import pytest

from oracle_lib import max_abs_rel, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb(cuda):
    import crosslane_b200
    return crosslane_b200


def test_router_gemv_matches_fp64(cb, cuda):
    torch = cuda
    rng = np.random.default_rng(1)
    E, D, T = 384, 7168, 5
    W = (rng.standard_normal((E, D)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, D)).astype(np.float32)
    d_l = torch.empty((T, E), dtype=torch.float32, device="cuda")
    cb.router_device(torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda(), d_l)
    got = d_l.cpu().numpy()
    want = x.astype(np.float64) @ W.astype(np.float64).T
    scale = np.abs(x).astype(np.float64) @ np.abs(W).astype(np.float64).T  # |x| . |w| bounds the rounding error
    assert np.all(np.abs(got - want) <= 1e-5 * scale), np.max(np.abs(got - want) / scale)
    again = torch.empty_like(d_l)
    cb.router_device(torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda(), again)
    assert torch.equal(d_l, again)


@pytest.mark.parametrize("E,k,scale", [(384, 6, 2.5), (256, 8, 1.0), (1024, 16, 0.5), (16, 16, 1.0)])
def test_route_b_device_matches_host(cb, orc, cuda, E, k, scale):
    torch = cuda
    rng = np.random.default_rng(E + k)
    T = 600
    logits = (rng.standard_normal((T, E)) * 4).astype(np.float32)
    logits[:, :3] = np.array([25.0, 20.0, 19.999998], np.float32)  # both softplus branches, the boundary
    logits[1, :] = logits[1, 0]  # all scores equal: ties go to the lower id
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    bias[5:9] = 0.0
    d_ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    d_w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    d_st = torch.zeros(1, dtype=torch.int32, device="cuda")
    cb.route_b_device(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), k, scale, d_ids, d_w, d_st)
    ids, w = d_ids.cpu().numpy(), d_w.cpu().numpy()
    assert int(d_st.item()) == 0
    for t in range(T):
        hi, hw = cb.route_host(1, logits[t], k, bias=bias, scale=scale)
        oi, ow = orc.route_sqrt_softplus(logits[t], bias, k, scale)
        assert np.array_equal(ids[t], hi) and np.array_equal(hi, oi), t  # selection: bit for bit
        assert np.array_equal(hw.view(np.uint32), ow.view(np.uint32)), t
        # weights: the device's exp/log1p are the correctly rounded floats; glibc's expf and
        # log1pf are off by one ulp for some arguments (about 1.4 % of the scores at these
        # logit scales), and one score an ulp apart moves every weight of its token by an
        # ulp or two through the sum
        ulps = np.abs(w[t].view(np.int32).astype(np.int64) - hw.view(np.int32).astype(np.int64))
        assert ulps.max() <= 2, (t, w[t], hw)


def test_route_b_device_flags_nonfinite(cb, cuda):
    torch = cuda
    E, k = 32, 4
    logits = np.zeros((2, E), np.float32)
    bias = np.zeros(E, np.float32)
    bias[3] = np.inf
    d_ids = torch.empty((2, k), dtype=torch.int32, device="cuda")
    d_w = torch.empty((2, k), dtype=torch.float32, device="cuda")
    d_st = torch.zeros(1, dtype=torch.int32, device="cuda")
    cb.route_b_device(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), k, 1.0, d_ids, d_w, d_st)
    assert int(d_st.item()) == 1


def test_moe_block_device_matches_oracle(cb, orc, cuda):
    torch = cuda
    dim, ff, E, k, seed, policy, scale = 2048, 512, 24, 6, 8, 2, 2.5
    bank = cb.ExpertBank(n_layers=2, n_experts=E, dim=dim, ff=ff, max_picks=k, device=0)
    try:
        bank.fill_synthetic(seed, policy)
        rng = np.random.default_rng(3)
        W = (rng.standard_normal((E, dim)) * 0.03).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
        for trial in range(3):
            x = rng.standard_normal(dim).astype(np.float32)
            shared = rng.standard_normal(dim).astype(np.float32)
            resid = rng.standard_normal(dim).astype(np.float32)
            d_x, d_W, d_b = (torch.from_numpy(a).cuda() for a in (x, W, bias))
            d_sh, d_r = torch.from_numpy(shared).cuda(), torch.from_numpy(resid).cuda()
            d_out = torch.empty(dim, dtype=torch.float32, device="cuda")
            d_lg = torch.empty(E, dtype=torch.float32, device="cuda")
            d_ids = torch.empty(k, dtype=torch.int32, device="cuda")
            d_w = torch.empty(k, dtype=torch.float32, device="cuda")
            bank.moe_block_device(1, d_x, d_W, d_b, scale, d_out, d_lg, d_ids, d_w, d_shared=d_sh, d_resid=d_r)
            bank.synchronize()
            lg = d_lg.cpu().numpy()
            ids, w = cb.route_host(1, lg, k, bias=bias, scale=scale)  # the host's picks on the device's logits
            dw = d_w.cpu().numpy()
            assert np.array_equal(d_ids.cpu().numpy(), ids)
            assert np.abs(dw.view(np.int32).astype(np.int64) - w.view(np.int32).astype(np.int64)).max() <= 2
            want = orc.layer_synth(policy, seed, 1, ids, w, x, dim, ff, shared=shared)
            got = d_out.cpu().numpy() - resid
            assert rel_l2(got, want) <= 1e-3 and max_abs_rel(got, want) <= 5e-3, trial
    finally:
        bank.close()
