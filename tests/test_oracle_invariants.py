"""The oracle's water-filling and within-cluster top-q against the properties the reference states
for them, on seeded random rows (CPU only).

Water-filling (inference/methods_eager.py:558-581, invariants checked by the reference's own self-test
at :725-727): quotas are whole numbers, 0 <= quota <= cap with cap = n_t for live clusters (n_t > 1)
and 0 otherwise, and sum(quota) = min(E, sum(cap)).

Top-q (inference/ours_graph.py:93-166): each cluster's segment of exp_idx, at offset sum of the
earlier quotas, holds the q best candidates of the cluster by score (ties -> lower position) in
ascending position order, and -1 pads the rest.  Checked against a brute-force sort."""
import numpy as np
import pytest

import oracle as O


def _caps(nt):
    return np.where(nt > 1.0, nt, 0.0)


@pytest.mark.parametrize("C,E", [(64, 216), (192, 679), (192, 1335)])
def test_waterfill_invariants(C, E):
    rng = np.random.default_rng(C * 7 + E)
    rows = []
    for kind in range(6):
        for _ in range(8):
            score = rng.normal(0.0, 3.0, C).astype(np.float32)
            nt = rng.integers(0, 600, C).astype(np.float32)
            if kind == 1:    # total capacity below E: every live cluster gets its cap
                nt = rng.integers(0, max(2, 2 * E // C), C).astype(np.float32)
            elif kind == 2:  # no live cluster
                nt = rng.integers(0, 2, C).astype(np.float32)
            elif kind == 3:  # ties in the scores
                score = np.round(score).astype(np.float32)
            elif kind == 4:  # one cluster dominates the weights
                score[rng.integers(C)] += 40.0
            elif kind == 5:  # weights spanning many orders of magnitude
                score = rng.normal(0.0, 30.0, C).astype(np.float32)
            rows.append((score, nt))
    score = np.stack([r[0] for r in rows])
    nt = np.stack([r[1] for r in rows])
    quota = O.waterfill(score, nt, E)
    cap = _caps(nt)
    assert np.all(quota == np.floor(quota)), "quotas are whole numbers"
    assert np.all(quota >= 0) and np.all(quota <= cap)
    np.testing.assert_array_equal(quota.sum(1), np.minimum(float(E), cap.sum(1)))


def _bf16_bits(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_topq_is_the_exact_top_q():
    rng = np.random.default_rng(11)
    R, C, Lmax, n, E = 8, 16, 2048, 1900, 400
    asg = rng.integers(0, C, (R, Lmax)).astype(np.int32)
    # coarse scores: many exact ties between positions
    s = _bf16_bits(np.round(rng.normal(0.0, 2.0, (R, Lmax)) * 4) / 4)
    s[:, n:] = 0xFF80
    sel = rng.choice(n, (R, 12), replace=True)
    for r in range(R):
        s[r, sel[r]] = 0xFF80  # selected tokens are out of the race
    quota = np.zeros((R, C), np.float32)
    for r in range(R):
        live = s[r, :n] != 0xFF80
        avail = np.bincount(asg[r, :n][live], minlength=C)
        q = np.minimum(avail, rng.integers(0, 2 * E // C, C))
        while q.sum() > E:
            q[int(np.argmax(q))] -= 1
        quota[r] = q
    exp_idx = O.topq(s, asg, quota, n, E)
    sf = O.bf16_to_f32(s)
    for r in range(R):
        base = 0
        for c in range(C):
            q = int(quota[r, c])
            cand = np.flatnonzero(asg[r, :n] == c)
            order = sorted(cand.tolist(), key=lambda t: (-sf[r, t], t))
            want = sorted(order[:q])
            got = exp_idx[r, base:base + q].tolist()
            assert got == want, (r, c)
            base += q
        assert np.all(exp_idx[r, base:] == -1)


def _round_bf16(x32):
    """fp32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.asarray(x32, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_scan_is_bf16_of_the_once_rounded_exact_sum():
    """QGS scores (graph_runner.py:100-120) are bf16(fp32(sum_j code_j zq_j)) with the sum taken
    exactly and rounded once, so they do not depend on a summation order; sink, local and beyond-n
    positions are -inf.  zq rows here span fewer than 2^21 in magnitude, where every product is
    exact in the kernel's fixed-point limbs too."""
    rng = np.random.default_rng(5)
    B, Lmax, n, ns, nl = 1, 640, 600, 2, 3
    codes = rng.integers(-127, 128, (B, 8, Lmax, 32)).astype(np.int8)
    mag = 2.0 ** rng.uniform(-6, 2, (B * 32, 32))
    zq = _bf16_bits(mag * rng.choice([-1.0, 1.0], (B * 32, 32)))
    s = O.scan(codes, zq, n, ns, nl, sw=Lmax)
    zf = O.bf16_to_f32(zq).astype(np.float64)
    for r in range(B * 32):
        exact = codes[r // 128, (r % 32) // 4].astype(np.float64) @ zf[r]  # (Lmax,), exact in float64
        want = _round_bf16(exact.astype(np.float32))
        want[:ns] = 0xFF80
        want[n - nl:] = 0xFF80
        np.testing.assert_array_equal(s[r], want)


def test_errorgate_matches_the_formula_in_float64():
    """ErrorGate (ours_fused.py:122-154): per cluster b, the tail after removing the selected tokens
    Sk_t = Sk - sum k, Sk2_t = Sk2 - sum k^2, n_t = n_b - #selected; kbar = Sk_t / max(n_t, 1),
    var = max(Sk2_t / max(n_t, 1) - kbar^2, 0), zbar = s q.kbar, s2 = s^2 sum_d q_d^2 var_d and
    score = zbar + ln max(n_t, 1) + s2 / 2 + ln max(erf(sqrt(s2 / 2)), 1e-30), s = 128^-1/2.
    The oracle's fp32 evaluation is held to 2e-4 relative of the float64 formula; n_t exactly."""
    rng = np.random.default_rng(3)
    Lmax, C, NS, D = 256, 8, 6, 128
    K = _bf16_bits(rng.normal(0.0, 1.0, (1, 8, Lmax, D)))
    q = _bf16_bits(rng.normal(0.0, 1.0, (32, D)))
    asg = rng.integers(0, C - 1, (32, Lmax)).astype(np.int32)
    asg[:, :40] = 0  # one large cluster
    asg[:, 40] = C - 1  # and one whose single member is selected below: an empty tail
    Kf = O.bf16_to_f32(K[0]).astype(np.float64)
    qf = O.bf16_to_f32(q).astype(np.float64)
    Sk, Sk2 = np.zeros((32, C, D)), np.zeros((32, C, D))
    sel = np.zeros((32, NS), np.int32)
    for r in range(32):
        np.add.at(Sk[r], asg[r], Kf[r // 4])
        np.add.at(Sk2[r], asg[r], Kf[r // 4] ** 2)
        sel[r] = rng.choice(Lmax, NS, replace=False)
        sel[r, 0] = 40
    nb = np.stack([np.bincount(asg[r], minlength=C) for r in range(32)]).astype(np.float32)
    Sk32, Sk232 = Sk.astype(np.float32), Sk2.astype(np.float32)
    score, nt = O.errorgate(q, K, asg, sel, Sk32, Sk232, nb)
    from math import erf, log, sqrt
    sc = 128 ** -0.5
    for r in range(32):
        skt, sk2t = Sk32[r].astype(np.float64), Sk232[r].astype(np.float64)
        ntr = nb[r].astype(np.float64)
        for t in sel[r]:
            c = asg[r, t]
            skt[c] -= Kf[r // 4, t]
            sk2t[c] -= Kf[r // 4, t] ** 2
            ntr[c] -= 1
        np.testing.assert_array_equal(nt[r], ntr.astype(np.float32))
        for c in range(C):
            m = max(ntr[c], 1.0)
            kb = skt[c] / m
            var = np.maximum(sk2t[c] / m - kb * kb, 0.0)
            s2 = sc * sc * float((qf[r] ** 2) @ var)
            want = sc * float(qf[r] @ kb) + log(m) + s2 / 2 + log(max(erf(sqrt(s2 / 2)), 1e-30))
            assert abs(float(score[r, c]) - want) <= 2e-4 * max(1.0, abs(want)), (r, c, float(score[r, c]), want)


def test_residual_proxies_match_the_read_sets():
    """Residual proxies (ours_fused.py:367-407): per cluster, the pooled sums minus every token read
    (selected tokens by their assignment, expanded tokens by the quota segment their slot is in),
    n' = n_t - q, kbar' = bf16(Sk' / max(n', 1)), vbar' likewise, log n' = ln max(n', 1) when n' > 0.5
    else -inf.  Compared with the same sums in float64: log n' to 1e-6, the bf16 proxies to one bf16
    rounding plus the fp32 cancellation error of the pooled sums."""
    rng = np.random.default_rng(8)
    Lmax, C, NS, E, D = 512, 12, 5, 96, 128
    K = _bf16_bits(rng.normal(0.0, 1.0, (1, 8, Lmax, D)))
    V = _bf16_bits(rng.normal(0.0, 1.0, (1, 8, Lmax, D)))
    Kf, Vf = O.bf16_to_f32(K[0]).astype(np.float64), O.bf16_to_f32(V[0]).astype(np.float64)
    asg = rng.integers(0, C, (32, Lmax)).astype(np.int32)
    Sk, Sv = np.zeros((32, C, D)), np.zeros((32, C, D))
    sel = np.zeros((32, NS), np.int32)
    nt = np.zeros((32, C), np.float32)
    quota = np.zeros((32, C), np.float32)
    exp_idx = np.full((32, E), -1, np.int32)
    for r in range(32):
        kv = r // 4
        np.add.at(Sk[r], asg[r], Kf[kv])
        np.add.at(Sv[r], asg[r], Vf[kv])
        sel[r] = rng.choice(Lmax, NS, replace=False)
        tail = np.ones(Lmax, bool)
        tail[sel[r]] = False
        nt[r] = np.bincount(asg[r][tail], minlength=C)
        quota[r] = np.minimum(nt[r], rng.integers(0, 2 * E // C, C))
        quota[r, 0] = nt[r, 0]  # a cluster read completely: n' = 0, log n' = -inf
        while quota[r].sum() > E:
            quota[r, 1 + int(np.argmax(quota[r, 1:]))] -= 1
        j = 0
        for c in range(C):
            m = np.flatnonzero(tail & (asg[r] == c))[:int(quota[r, c])]
            exp_idx[r, j:j + len(m)] = m
            j += len(m)
    Sk32, Sv32 = Sk.astype(np.float32), Sv.astype(np.float32)
    kbar, vbar, logn = O.residual(K, V, asg, sel, exp_idx, Sk32, Sv32, nt, quota)
    Skr, Svr, nr = O.residual_sums(K, V, asg, sel, exp_idx, Sk32, Sv32, nt, quota)
    live = nr > 0.5
    want_ln = np.where(live, np.log(np.maximum(nr, 1.0)), -np.inf)
    assert np.array_equal(np.isinf(logn), ~live)
    np.testing.assert_allclose(logn[live], want_ln[live], rtol=0, atol=1e-6)
    inv = 1.0 / np.maximum(nr, 1.0)[..., None]
    for got, S, Sr in ((kbar, Sk, Skr), (vbar, Sv, Svr)):
        g = O.bf16_to_f32(got).astype(np.float64)
        want = Sr * inv
        tol = 2.0 ** -8 * np.abs(want) + 1e-5 * np.abs(S).max(-1, keepdims=True) * inv
        assert np.all(np.abs(g - want) <= tol)


def test_select_is_the_exact_top_k():
    """QGS select (graph_runner.py:123-159): sel = [0 .. ns-1, n-nl .. n-1, the k best scores ranked by
    (score desc, position asc)] and the chosen scores become -inf.  The best-tiles-first search of the
    reference is exact (every top-k score lies in one of the k best tiles by maximum), so the check
    is a brute-force sort over all positions below n, with many tied scores."""
    rng = np.random.default_rng(21)
    R, n, ns, nl, k = 16, 3000, 2, 3, 9
    s = _bf16_bits(np.round(rng.normal(0.0, 1.5, (R, n)) * 2) / 2)
    s[:, :ns] = 0xFF80
    s[:, n - nl:] = 0xFF80
    s[3, ns:n - nl] = s[3, ns]  # one row where every candidate ties
    s0 = s.copy()
    sel = O.select(s, n, ns, nl, k)
    sf = O.bf16_to_f32(s0)
    for r in range(R):
        order = sorted(range(n), key=lambda t: (-sf[r, t], t))[:k]
        assert sel[r].tolist() == list(range(ns)) + list(range(n - nl, n)) + order
        want = s0[r].copy()
        want[order] = 0xFF80
        np.testing.assert_array_equal(s[r], want)


def test_index_update_against_float64():
    """Index update of the new token (ours_graph.py:43-90): per KV head, code = clamp(rint(k.U / scale),
    +-127); per query head, zp = bf16(k.W) - colmean, cluster = argmax_c(zp.cent_c - |cent_c|^2 / 2)
    (ties -> lower id), then n_b += 1, Sk += k, Sk2 += k^2, Sv += v (one fp32 add each) and the position
    appended to the cluster's generated list while it has room (the count always advances).  Codes
    within one step of the float64 value; the cluster equal to the float64 choice unless the two best
    are within 1e-3; the sums exactly."""
    rng = np.random.default_rng(13)
    Lmax, C, D, pos, rmax = 64, 12, 128, 40, 256
    st = O.new_state(1, Lmax, C, rmax)
    st["U"][0] = (rng.normal(size=(8, D, 32)) / np.sqrt(D)).astype(np.float32)
    st["scale"][0] = (np.abs(rng.normal(size=(8, 32))) * 0.05 + 0.02).astype(np.float32)
    st["W"][0] = _bf16_bits(rng.normal(size=(32, D, 16)) / np.sqrt(D))
    st["colmean"][0] = (rng.normal(size=(32, 16)) * 0.1).astype(np.float32)
    st["cent"][0] = rng.normal(size=(32, C, 16)).astype(np.float32)
    st["nb"][0] = rng.integers(1, 20, (32, C)).astype(np.float32)
    for k_ in ("Sk", "Sk2", "Sv"):
        st[k_][0] = rng.normal(size=(32, C, D)).astype(np.float32)
    st["reccnt"][0] = rng.integers(0, 5, (32, C)).astype(np.int32)
    st["reccnt"][0, :8] = rmax  # the first KV head's query heads: lists already full
    K = _bf16_bits(rng.normal(size=(1, 8, Lmax, D)))
    V = _bf16_bits(rng.normal(size=(1, 8, Lmax, D)))
    snap = {k_: v.copy() for k_, v in st.items()}
    O.index_update(st, K, V, pos)
    kf = O.bf16_to_f32(K[0, :, pos]).astype(np.float64)  # (8, D)
    vf32, kf32 = O.bf16_to_f32(V[0, :, pos]), O.bf16_to_f32(K[0, :, pos])
    z = np.einsum("kd,kdj->kj", kf, st["U"][0].astype(np.float64)) / st["scale"][0]
    code_ref = np.clip(np.rint(z), -127, 127)
    assert np.abs(st["codes"][0, :, pos].astype(np.int64) - code_ref).max() <= 1
    assert (st["codes"][0, :, pos] != code_ref).sum() <= 2
    cent = st["cent"][0].astype(np.float64)
    for h in range(32):
        kv = h // 4
        proj = kf[kv] @ O.bf16_to_f32(st["W"][0, h]).astype(np.float64)
        zp = O.bf16_to_f32(_round_bf16(proj.astype(np.float32))).astype(np.float64) - st["colmean"][0, h]
        dist = cent[h] @ zp - 0.5 * (cent[h] ** 2).sum(1)
        cid = int(st["asg"][0, h, pos])
        best = int(np.argmax(dist))
        assert cid == best or dist[best] - dist[cid] < 1e-3, (h, cid, best)
        others = np.arange(C) != cid
        np.testing.assert_array_equal(st["nb"][0, h, others], snap["nb"][0, h, others])
        assert st["nb"][0, h, cid] == snap["nb"][0, h, cid] + 1
        np.testing.assert_array_equal(st["Sk"][0, h, cid], snap["Sk"][0, h, cid] + kf32[kv])
        np.testing.assert_array_equal(st["Sk2"][0, h, cid], snap["Sk2"][0, h, cid] + kf32[kv] * kf32[kv])
        np.testing.assert_array_equal(st["Sv"][0, h, cid], snap["Sv"][0, h, cid] + vf32[kv])
        np.testing.assert_array_equal(st["Sk"][0, h, others], snap["Sk"][0, h, others])
        cnt = int(snap["reccnt"][0, h, cid])
        assert st["reccnt"][0, h, cid] == cnt + 1
        if cnt < rmax:
            assert st["reclist"][0, h, cid, cnt] == pos
        np.testing.assert_array_equal(st["reclist"][0, h, others], snap["reclist"][0, h, others])


def test_erf_series_rounds_to_one_from_four():
    """The fp32 erf skips its double series from x = 4 on: the series rounded to fp32 is 1 there.
    Checked on every fp32 value in [4, 4.01] and on a grid up to the series' own cutoff at 6."""
    import ctypes
    lib = O.lib()
    lib.oro_erf_d.restype = ctypes.c_double
    lib.oro_erf_d.argtypes = [ctypes.c_double]
    lo = np.float32(4.0)
    dense = lo + np.arange(0, 40000, dtype=np.float32) * np.spacing(lo)  # every float from 4 upward
    grid = np.linspace(4.0, 6.0, 20001, dtype=np.float32)
    for x in np.concatenate([dense, grid]):
        assert np.float32(lib.oro_erf_d(float(x))) == np.float32(1.0), float(x)
        assert lib.oro_erff(float(x)) == 1.0
    # and the series is still used just below 4
    assert lib.oro_erff(3.5) < 1.0
