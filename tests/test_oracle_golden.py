"""Pin the CPU oracle to the reference: its outputs must match the golden fixtures that the
reference's own PyTorch code produced (tests/golden/make_golden.py) on the same seeded inputs.

Exact where the reference is deterministic on CPU (build sums, codes, new-token assignments and
codes, selected sets, tail counts, quotas, log n'); every differing expanded index must be a tie (or
a 1-ulp neighbour) of its cluster's threshold key, because the eager reference breaks ties by an
unspecified argsort order; float outputs within stated tolerances.
"""
import os

import numpy as np
import pytest

import cases
import oracle as O

HQ, HKV, D = 32, 8, 128


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, f"{name}.npz"))


def _ukey(b):
    b = b.astype(np.uint32)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)


def test_transcendentals_accuracy():
    """The oracle's own ln / exp / erf (the GPU kernels reproduce them) are accurate fp32 functions."""
    import math
    lib = O.lib()
    xs = np.concatenate([np.logspace(-30, 30, 997), np.arange(1, 5000, 7, dtype=np.float64)]).astype(np.float32)
    for x in xs:
        assert abs(lib.oro_logf(float(x)) - math.log(float(x))) <= 2e-7 * max(1.0, abs(math.log(float(x))))
    for x in np.linspace(-80, 20, 1001, dtype=np.float32):
        ref = math.exp(float(x))
        assert abs(lib.oro_expf(float(x)) - ref) <= 1.2e-7 * ref + 1e-38
    assert lib.oro_expf(float("-inf")) == 0.0
    for x in np.linspace(0, 7, 1401, dtype=np.float32):
        assert abs(lib.oro_erff(float(x)) - math.erf(float(x))) <= 1.2e-7


def test_flash_qhead_matches_reference_selftest_formula(golden_dir):
    """methods_eager.selftest's fp32 reference (inference/methods_eager.py:708-719) vs the oracle."""
    x = cases.flash_inputs("flash_qhead")
    z = _load(golden_dir, "flash_qhead")
    out = O.flash(O.bits(x["q"]), O.bits(x["k"]), O.bits(x["v"]), x["sel"].numpy(), x["exp"].numpy(),
                  O.bits(x["kbar"]), O.bits(x["vbar"]), x["log_n"].numpy(), D ** -0.5, per_qhead=True)
    ref = z["out"]
    assert np.abs(out - ref).max() < 2e-5
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-5


def test_flash_kvhead_matches_reference_unfused_path(golden_dir):
    """bench_flash_latency's ours_torch path (bf16 probabilities and bf16 matmuls) vs the fp64 oracle:
    agreement to bf16 precision."""
    x = cases.flash_inputs("flash_kvhead")
    z = _load(golden_dir, "flash_kvhead")
    out = O.flash(O.bits(x["q"]), O.bits(x["k"]), O.bits(x["v"]), x["sel"].numpy(), x["exp"].numpy(),
                  O.bits(x["kbar"]), O.bits(x["vbar"]), x["log_n"].numpy(), D ** -0.5, per_qhead=False)
    ref = z["out"]
    rel = np.linalg.norm(out - ref, axis=1) / np.linalg.norm(ref, axis=1)
    assert np.median(rel) < 1e-2 and rel.max() < 3e-2


def _state_from_fixture(x, z):
    B, n0, Lmax = x["B"], x["n0"], x["Lmax"]
    C = int(z["C"])
    st = O.new_state(B, Lmax, C)
    st["U"][:] = z["U"]
    st["scale"][:] = z["scale"].reshape(B, HKV, 32)
    st["codes"][:, :, :n0] = z["codes"][:, :, :n0]
    st["W"][:] = z["W"]
    st["colmean"][:] = z["colmean"].reshape(B, HQ, 16)
    st["cent"][:] = z["cent"]
    st["asg"][:, :, :n0] = z["asg"]
    st["nb"][:] = z["nb"]
    K, V = O.bits(x["K"]).copy(), O.bits(x["V"]).copy()
    for b in range(B):
        mem, cs, cl, Sk, Sk2, Sv = O.csr_sums(K[b], V[b], st["asg"][b], n0, C)
        st["Sk"][b], st["Sk2"][b], st["Sv"][b] = Sk, Sk2, Sv
        st["mem"][b], st["cstart"][b], st["clen"][b] = mem, cs, cl
    return st, K, V


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_build_matches_reference(golden_dir, name):
    """Codes and cluster sums restated from the reference's basis and assignments are bit-identical."""
    x = cases.decode_inputs(name)
    z = _load(golden_dir, name)
    st, K, V = _state_from_fixture(x, z)
    n0 = x["n0"]

    def same(name, got, want):
        got, want = np.asarray(got), np.asarray(want)
        if not np.array_equal(got, want):
            bad = np.argwhere(got != want)
            d = np.abs(got.astype(np.float64) - want.astype(np.float64))
            raise AssertionError(f"{name}: {len(bad)} of {got.size} differ, first at {bad[0].tolist()}, "
                                 f"max |diff| {d.max():.3e}")
    same("Sk_sum", st["Sk"].astype(np.float64).sum(-1), z["Sk_sum"])
    same("Sk2_sum", st["Sk2"].astype(np.float64).sum(-1), z["Sk2_sum"])
    same("Sv_sum", st["Sv"].astype(np.float64).sum(-1), z["Sv_sum"])
    same("Sk_rows", st["Sk"][:, ::16, ::4], z["Sk_rows"])
    for b in range(x["B"]):
        scale, codes = O.build_codes(K[b], z["U"][b], n0)
        same(f"scale[{b}]", scale, z["scale"][b].reshape(HKV, 32))
        same(f"codes[{b}]", codes[:, :n0], z["codes"][b][:, :n0])
        same(f"nb[{b}]", st["nb"][b], np.stack([np.bincount(st["asg"][b, h, :n0], minlength=int(z["C"]))
                                                for h in range(HQ)]).astype(np.float32))


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_decode_steps_match_reference(golden_dir, name):
    x = cases.decode_inputs(name)
    z = _load(golden_dir, name)
    st, K, V = _state_from_fixture(x, z)
    B, n0 = x["B"], x["n0"]
    R, C, E = B * HQ, int(z["C"]), int(z["E"])
    for s in range(x["steps"]):
        n = n0 + s + 1
        K[:, :, n - 1] = O.bits(x["new_k"][s])
        V[:, :, n - 1] = O.bits(x["new_v"][s])
        q = O.bits(x["qdec"][s].reshape(R, D))
        o = O.decode_step(st, q, K, V, n, x["rho"], C, E)
        # index update of the new token
        assert np.array_equal(st["asg"][..., n - 1], z[f"s{s}_asg_new"])
        assert np.array_equal(st["codes"][:, :, n - 1], z[f"s{s}_codes_new"])
        # QGS selection: same sets (the reference's topk order within the top is not specified)
        for a, b in zip(o["sel"], z[f"s{s}_sel"]):
            assert sorted(a.tolist()) == sorted(b.tolist())
        # ErrorGate tail counts exact, scores to fp32 rounding, quotas exact
        assert np.array_equal(o["nt"], z[f"s{s}_nt"])
        zs = z[f"s{s}_score"]
        assert np.all(np.abs(o["score"] - zs) <= 2e-6 * np.maximum(np.abs(zs), 1.0))
        assert np.array_equal(o["quota"], z[f"s{s}_quota"].astype(np.float32))
        # within-cluster top-q: every differing token sits at its cluster's threshold key (a tie)
        keys = _ukey(o["s_masked"])
        asg = st["asg"].reshape(R, -1)
        for r in range(R):
            mine, ref = set(o["exp_idx"][r].tolist()) - {-1}, set(z[f"s{s}_exp"][r].tolist()) - {-1}
            assert len(mine) == len(ref)
            for c in {int(asg[r, t]) for t in mine ^ ref}:
                took = [t for t in mine if asg[r, t] == c]
                T = min(int(keys[r, t]) for t in took)
                for t in (mine ^ ref):
                    if asg[r, t] == c:
                        assert abs(int(keys[r, t]) - T) <= 1, (r, c, t)
        # proxies and output on the REFERENCE's own indices
        kbar, vbar, logn = O.residual(K, V, asg, z[f"s{s}_sel"], z[f"s{s}_exp"].astype(np.int32),
                                      st["Sk"].reshape(R, C, D), st["Sv"].reshape(R, C, D), o["nt"], o["quota"])
        assert np.array_equal(logn, z[f"s{s}_logn"])
        assert np.array_equal(kbar[::16, ::4], z[f"s{s}_kbar_rows"])
        assert np.array_equal(vbar[::16, ::4], z[f"s{s}_vbar_rows"])
        out = O.flash(q, K.reshape(B * HKV, -1, D), V.reshape(B * HKV, -1, D), z[f"s{s}_sel"],
                      z[f"s{s}_exp"].astype(np.int32), kbar, vbar, logn, D ** -0.5, per_qhead=True)
        ref = z[f"s{s}_out"]   # OursUnfused.attend: bf16 probabilities, bf16 matmuls
        rel = np.linalg.norm(out - ref, axis=1) / np.linalg.norm(ref, axis=1)
        assert np.median(rel) < 1.5e-2 and rel.max() < 5e-2


# ------------------------------------------------------------------ the build against the reference
REF_ROOT = os.environ.get("OA_REFERENCE", "/root/reference")


def _reference_asset():
    p = os.path.join(REF_ROOT, "assets", "llama-3.1-8b-instruct.query_metric.triu.pt")
    if not os.path.exists(p):
        pytest.skip("the reference checkout (its static-metric asset) is not on this machine")
    import torch
    return torch.load(p, map_location="cpu", weights_only=False)


def test_metric_unpack_matches_reference_restore():
    """method.unpack_metric on the reference's shipped asset == the reference's own restore
    (assets/restore_query_metric.py:18-27, imported from the checkout), all 32 layers; the fixture
    metric_l0.npz is layer 0 of that asset."""
    import importlib.util
    import torch
    from openattention_b200 import method as Mth
    packed = _reference_asset()
    spec = importlib.util.spec_from_file_location("restore_query_metric",
                                                  os.path.join(REF_ROOT, "assets", "restore_query_metric.py"))
    rq = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rq)
    want = rq.unpack(packed)["M"]
    got = Mth.unpack_metric(packed)
    assert got.shape == (32, 32, 128, 128) and torch.equal(got, want)
    fx = cases.asset_packed()
    assert torch.equal(fx["M_triu"], packed["M_triu"][:1]) and torch.equal(fx["inv_freq"], packed["inv_freq"])


def test_load_static_metric_forms_and_missing():
    """The loader reads the packed and the unpacked asset form to the same M, and raises without a metric."""
    import types
    import torch
    from openattention_b200 import method as Mth
    packed = cases.asset_packed()
    M1, inv1, s1 = Mth.load_static_metric(types.SimpleNamespace(static_metric=packed), 1)
    M2, inv2, s2 = Mth.load_static_metric(types.SimpleNamespace(static_metric={"M": M1, "inv_freq": inv1}), 1)
    assert torch.equal(M1, M2) and torch.equal(inv1, inv2) and s1 == s2 == 1.0
    assert torch.equal(M1, M1.transpose(-1, -2))
    old = os.environ.pop("OA_STATIC_M", None)
    try:
        with pytest.raises(RuntimeError, match="no static query metric"):
            Mth.load_static_metric(types.SimpleNamespace(), 1)
        with pytest.raises(RuntimeError, match="holds 1 layers"):
            Mth.load_static_metric(types.SimpleNamespace(static_metric=packed), 2)
    finally:
        if old is not None:
            os.environ["OA_STATIC_M"] = old


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_basis_matches_reference(golden_dir, name):
    """The product's query metric (static metric rotated to the decode window + question rows) and its
    eigen-bases equal the reference's U (QGS) and W (QGC) bit for bit (inference/methods_eager.py:510-528);
    decode_real_l0 uses layer 0 of the reference's own asset."""
    from openattention_b200 import method as Mth
    x = cases.decode_inputs(name)
    z = _load(golden_dir, name)
    for b in range(x["B"]):
        M = Mth.query_metric(x["M"][0], x["inv_freq"], 1.0, x["qpre"][b], x["n0"], cases.QLEN)
        U, W = Mth.basis_from_host_metric(M.float())
        assert np.array_equal(U.numpy(), z["U"][b]), f"U[{b}]"
        assert np.array_equal(O.bits(W), z["W"][b]), f"W[{b}]"


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_kmeans_matches_reference(golden_dir, name):
    """The oracle's QGC projection and 4 Lloyd iterations (the GPU build equals the oracle bit for bit,
    tests/test_decode_gpu.py) from the reference's W reproduce the reference's cluster assignments and
    member counts exactly.  Centroids and column means differ only by the projection's rounding: the
    reference's projection is a bf16 matmul whose fp32 accumulation order is the library's, so a
    projected coordinate can differ by one bf16 ulp (2^-7 relative) where the exact sum sits near a
    rounding boundary; a mean of such values moves by at most one ulp of its largest member."""
    import torch
    x = cases.decode_inputs(name)
    z = _load(golden_dir, name)
    C, n0 = int(z["C"]), x["n0"]
    K = O.bits(x["K"])
    ulp = 2.0 ** -7
    for b in range(x["B"]):
        zP, colmean = O.project(K[b], z["W"][b], n0)
        asg, cent, nb = O.kmeans(zP, O.seeds(n0, C, 0), C)
        assert np.array_equal(asg, z["asg"][b].astype(np.int32)), f"asg[{b}]"
        assert np.array_equal(nb, z["nb"][b]), f"nb[{b}]"
        # the reference's own projection (methods_eager.py:530-531) evaluated here, for the bounds
        krep = x["K"][b, :, :n0].repeat_interleave(4, 0)
        zr = torch.matmul(krep, O.from_bits(z["W"][b])).float().numpy()          # (32, T, 16), bf16 values
        raw = zP.astype(np.float64) + colmean[:, None, :]   # the oracle's bf16 coordinates, up to fp32 rounding
        d = np.abs(raw - zr)
        # fp32 accumulation error of a 128-term dot is relative to the sum of |products|, which near a
        # zero coordinate exceeds the coordinate itself
        mag = np.abs(krep.float().numpy()) @ np.abs(O.from_bits(z["W"][b]).float().numpy())
        slack = 2.0 ** -23 * (np.abs(zr) + np.abs(colmean)[:, None, :]) + 2.0 ** -20 * mag
        assert np.all(d <= ulp * np.abs(zr) + slack), "projected coordinates differ by more than one bf16 ulp"
        print(f"{name}[{b}]: {(d > slack).mean():.2e} of the projected coordinates differ by one bf16 ulp")
        zc = z["colmean"][b].reshape(32, 16)
        assert np.all(np.abs(colmean - zc) <= ulp * np.abs(zr).max(1) + 1e-6), f"colmean[{b}]"
        for h in range(32):
            big = np.zeros(C)
            np.maximum.at(big, asg[h], np.abs(zr[h]).max(1))
            bound = ulp * big + ulp * np.abs(zr[h]).max() + 1e-5
            assert np.all(np.abs(cent[h] - z["cent"][b][h]) <= bound[:, None]), f"cent[{b}, {h}]"
