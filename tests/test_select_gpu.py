"""The QGS row top-k (qgs_select) and the within-cluster top-q (topq) through the C ABI against the
oracle on crafted score rows: random scores; all-equal scores (every choice is a tie, decided by the
lower position); and skewed rows whose large values sit in the tiles and in-tile offsets that one
half of a warp's lanes read, so the kernel's threshold pre-filter overflows and its radix select
runs.  k from 1 to 40 (above 32 the radix select always runs).  Bit-exact."""
import os

import numpy as np
import pytest
import torch

import cases
import oracle as O
from helpers import state_from_fixture, to_gpu_state, to_np
from openattention_b200 import selection as S
from openattention_b200.geometry import HQ

pytestmark = pytest.mark.gpu
NEG = 0xFF80


def _bits(v):
    return O.bits(torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(torch.bfloat16))


def _rows(kind, R, n, seed):
    rng = np.random.default_rng(seed)
    if kind == "random":
        v = rng.standard_normal((R, n)).astype(np.float32) * 3
    elif kind == "equal":
        v = np.full((R, n), 1.5, np.float32)
    else:  # skewed: tiles t % 32 < 16 and in-tile offsets < 16 hold the large values
        v = rng.standard_normal((R, n)).astype(np.float32) * 0.1
        t = np.arange(n)
        hot = ((t // 32) % 32 < 16) & (t % 32 < 16)
        v[:, hot] += 10 + rng.standard_normal((R, int(hot.sum()))).astype(np.float32)
    return _bits(v)


@pytest.mark.parametrize("kind", ["random", "equal", "skewed"])
@pytest.mark.parametrize("k_top", [1, 9, 31, 40])
def test_select_matches_oracle(kind, k_top):
    _check_select(kind, k_top, 64, 4101, 4160)


@pytest.mark.parametrize("kind", ["random", "equal", "skewed"])
@pytest.mark.parametrize("k_top", [9, 40])
def test_select_tile_maxima_not_bf16(kind, k_top):
    """Tile maxima that are not bf16 values (a caller's own) take the 64-bit tile words; the scan's
    are bf16 values and take the 32-bit ones.  Both pick the same tiles."""
    _check_select(kind, k_top, 64, 4101, 4160, nudge_tile_max=True)


@pytest.mark.parametrize("n,Lmax,k_top", [(65536, 65600, 20), (131072, 131104, 40)])
def test_select_long_rows_matches_oracle(n, Lmax, k_top):
    """Rows of 64K and 128K positions: the per-warp tile keys then take tens of KB of shared memory,
    which together with the kernel's static arrays passes the 48 KB default."""
    _check_select("random", k_top, 8, n, Lmax)


def _check_select(kind, k_top, R, n, Lmax, nudge_tile_max=False):
    ns, nl = 3, 3
    SW = S.padded_len(Lmax)
    NT = (Lmax + 31) // 32
    s = np.full((R, SW), NEG, np.uint16)
    s[:, :n] = _rows(kind, R, n, 7 + k_top)
    s[:, :ns] = NEG
    s[:, n - nl:n] = NEG
    tmax = O.bf16_to_f32(s[:, :NT * 32].reshape(R, NT, 32)).max(axis=2).astype(np.float32)
    if nudge_tile_max:  # one ulp up: the same order, but no longer bf16 values (the 64-bit tile words)
        tmax = np.nextafter(tmax, np.float32(np.inf)).astype(np.float32)
    ref = s.copy()
    sel_ref = O.select(ref, n, ns, nl, k_top)
    scores = O.from_bits(s).cuda()
    sel = torch.empty(R, ns + nl + k_top, dtype=torch.int32, device="cuda")
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    S.qgs_select(scores, torch.from_numpy(tmax).cuda(), Lmax, n_dev, ns, nl, k_top, sel)
    torch.cuda.synchronize()
    assert np.array_equal(sel.cpu().numpy(), sel_ref)
    assert np.array_equal(to_np(scores), ref)


@pytest.mark.parametrize("kind", ["random", "equal"])
def test_topq_matches_oracle_with_ties(golden_dir, kind):
    """Top-q over a fixture's CSR lists with crafted scores and quotas (up to 4 per cluster)."""
    x = cases.decode_inputs("decode_c0")
    z = np.load(os.path.join(golden_dir, "decode_c0.npz"))
    st_np, K, V = state_from_fixture(x, z)
    B, n0, Lmax = x["B"], x["n0"], x["Lmax"]
    C = st_np["nb"].shape[-1]
    E, R = 216, B * HQ
    n = n0  # no generated tokens
    SW = S.padded_len(Lmax)
    s = np.full((R, SW), NEG, np.uint16)
    s[:, :n] = _rows(kind, R, n, 11)
    clen = st_np["clen"].reshape(R, C)
    quota = np.zeros((R, C), np.float32)
    for r in range(R):
        left = E
        for c in np.random.default_rng(r).permutation(C):
            q = min(4, int(clen[r, c]), left)
            quota[r, c] = q
            left -= q
    exp_ref = O.topq(s, st_np["asg"].reshape(R, -1), quota, n, E)
    st = to_gpu_state(st_np)
    exp_idx = torch.empty(R, E, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    S.topq(O.from_bits(s).cuda(), st, torch.from_numpy(quota).cuda(), E,
           torch.tensor([n], dtype=torch.int32, device="cuda"), torch.tensor([n0], dtype=torch.int32, device="cuda"),
           exp_idx, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(exp_idx.cpu().numpy(), exp_ref)


@pytest.mark.parametrize("n0,use_ws", [(65536, True), (65536, False), (40000, False), (35300, False),
                                       (32768, False)])
def test_topq_long_rows_matches_oracle(n0, use_ws):
    """Top-q at each row length's kernel, quotas up to 40 (past the register path's 32): 32K and 35.3K
    positions (the pipelined kernel, two key buffers; 35.3K is near the most its shared memory holds),
    40K (one key buffer), and rows too long for shared memory
    (64K) with the workspace (keys permuted into CSR order, then selected from contiguous keys) and
    without it (keys read from global memory)."""
    import types
    from openattention_b200 import method as Mth
    from openattention_b200 import synth
    dev = torch.device("cuda")
    B, rho = 1, 0.01
    Lmax = n0 + 8
    K, V, _ = synth.kv_torch(51, B, n0, Lmax, dev)
    Mth.C.K, Mth.C.V, Mth.C.qlen = [K], [V], [40]
    m = Mth.OursB200(types.SimpleNamespace(rho=rho, static_metric=synth.static_metric_standin(7, 1)), B, Lmax, dev,
                     layers=1)
    g = torch.Generator(device=dev)
    g.manual_seed(52)
    qpre = torch.zeros(1, HQ, n0, 128, dtype=torch.bfloat16, device=dev)
    qpre[:, :, n0 - 64:] = torch.randn(1, HQ, 64, 128, generator=g, device=dev).to(torch.bfloat16)
    m.build(0, 0, qpre, n0)
    R, C, E = B * HQ, m.C, m.E
    st = m.st[0]
    clen = st["clen"].view(R, C).cpu().numpy()
    quota = np.zeros((R, C), np.float32)
    for r in range(R):
        left = E
        for c in np.random.default_rng(60 + r).permutation(C):
            q = min(int(np.random.default_rng(r * 97 + c).integers(0, 40)), int(clen[r, c]), left)
            quota[r, c] = q
            left -= q
    s = np.full((R, S.padded_len(Lmax)), NEG, np.uint16)
    s[:, :n0] = _rows("random", R, n0, 61)
    exp_ref = O.topq(s, st["asg"].view(R, -1).cpu().numpy(), quota, n0, E)
    ws = S.topq_workspace(R, Lmax, E, dev) if use_ws else None
    assert (ws is not None) == use_ws
    exp_idx = torch.empty(R, E, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    S.topq(O.from_bits(s).cuda(), st, torch.from_numpy(quota).cuda(), E, torch.tensor([n0], dtype=torch.int32,
           device=dev), torch.tensor([n0], dtype=torch.int32, device=dev), exp_idx, status, workspace=ws)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(exp_idx.cpu().numpy(), exp_ref)


@pytest.mark.parametrize("offset,advance", [(0, True), (-1, False)])
def test_append_kv_matches_index_copy(offset, advance):
    """The runner helper writes the new token's K/V rows where two index copies would, and advances
    the counters as the decode loop's increments do."""
    dev = torch.device("cuda")
    B, Lmax, n = 3, 200, 57
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    K = torch.randn(B, 8, Lmax, 128, generator=g, device=dev).to(torch.bfloat16)
    V = torch.randn(B, 8, Lmax, 128, generator=g, device=dev).to(torch.bfloat16)
    kn = torch.randn(B, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn(B, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    Kr, Vr = K.clone(), V.clone()
    n_dev = torch.tensor([n], dtype=torch.int32, device=dev)
    kv_idx = torch.tensor([n - 1], dtype=torch.int64, device=dev)
    S.append_kv(K, V, kn, vn, n_dev, offset=offset, advance=advance, kv_idx=kv_idx)
    p = n + offset
    Kr[:, :, p] = kn
    Vr[:, :, p] = vn
    torch.cuda.synchronize()
    assert torch.equal(K, Kr) and torch.equal(V, Vr)
    assert int(n_dev.item()) == (n + 1 if advance else n)
    assert int(kv_idx.item()) == (n if advance else n - 1)
