"""CPU ORACLE (test infrastructure, never the product): Python side of the C restatement in oa_oracle.c.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference arm may import this
module, and only as the checker or as the timed CPU restatement of the reference.

Stage wrappers take numpy arrays (bf16 data as uint16 bit patterns) and run the C restatement.
`decode_step` chains them in the order of the reference's deployed step (inference/methods_eager.py
Ours.decode :583-654; inference/ours_graph.py OursG2.decode :290-347) and `build_request` restates the
per-request build (methods_eager.py Ours.build :505-555, inference/ours_fastbuild.py :199-304, the
static-metric rotation of static_top_k.py StaticTopKMasker._rot_avg :102-131).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboa_oracle.so")
HQ, HKV, D, G, RQ, RC = 32, 8, 128, 4, 32, 16
SC = D ** -0.5
_lock = threading.Lock()
_lib = None


def build_lib(force: bool = False) -> str:
    src = os.path.join(HERE, "oa_oracle.c")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "liboa_oracle.so"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB):
                    build_lib()
                _lib = ctypes.CDLL(LIB)
                _lib.oro_logf.restype = ctypes.c_float
                _lib.oro_logf.argtypes = [ctypes.c_float]
                _lib.oro_expf.restype = ctypes.c_float
                _lib.oro_expf.argtypes = [ctypes.c_float]
                _lib.oro_erff.restype = ctypes.c_float
                _lib.oro_erff.argtypes = [ctypes.c_float]
    return _lib


def set_threads(n: int) -> int:
    """OpenMP threads of the oracle's parallel loops (its runtime may already be initialised by the
    host process, so the environment variable alone is not enough).  Returns the count in effect."""
    L = lib()
    L.omp_set_num_threads(ctypes.c_int(max(1, int(n))))
    L.omp_get_max_threads.restype = ctypes.c_int
    return int(L.omp_get_max_threads())


def _p(a):
    return ctypes.c_void_p(0) if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 torch tensor -> uint16 numpy bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a).astype(np.uint32) << 16).view(np.float32)


I, L, F = ctypes.c_int, ctypes.c_int64, ctypes.c_float


# ------------------------------------------------------------------ decode stages
def index_update(st, K, V, pos):
    """In place on the state dict (codes, asg, nb, Sk, Sk2, Sv, reclist, reccnt); K, V uint16 (B,8,Lmax,D)."""
    B, _, Lmax, _ = K.shape
    C = st["nb"].shape[-1]
    lib().oro_index_update(I(B), I(Lmax), I(C), I(pos), _p(K), _p(V), _p(st["codes"]), _p(st["U"]),
                           _p(st["scale"]), _p(st["W"]), _p(st["colmean"]), _p(st["cent"]), _p(st["asg"]),
                           _p(st["nb"]), _p(st["Sk"]), _p(st["Sk2"]), _p(st["Sv"]), _p(st.get("reclist")),
                           _p(st.get("reccnt")), I(st["reclist"].shape[-1] if "reclist" in st else 0))


def zq(q, U, scale):
    """q uint16 (R, D) -> zq uint16 (R, 32)."""
    R = q.shape[0]
    out = np.zeros((R, RQ), np.uint16)
    lib().oro_zq(I(R // HQ), _p(_c(q, np.uint16)), _p(_c(U, np.float32)), _p(_c(scale, np.float32)), _p(out))
    return out


def scan(codes, zqv, n, ns, nl, sw=None):
    """codes int8 (B,8,Lmax,32), zq uint16 (R,32) -> bf16 score bits (R, sw)."""
    B, _, Lmax, _ = codes.shape
    sw = n if sw is None else sw
    s = np.full((B * HQ, sw), 0xFF80, np.uint16)
    lib().oro_scan(I(B), I(Lmax), I(n), I(ns), I(nl), _p(_c(codes, np.int8)), _p(_c(zqv, np.uint16)), _p(s), L(sw))
    return s


def select(s, n, ns, nl, k_top):
    """In place on s (selected scores -> -inf); returns sel int32 (R, ns+nl+k_top)."""
    R, sw = s.shape
    sel = np.zeros((R, ns + nl + k_top), np.int32)
    lib().oro_select(I(R), I(n), I(ns), I(nl), I(k_top), _p(s), L(sw), _p(sel))
    return sel


def errorgate(q, K, asg, sel, Sk, Sk2, nb):
    B, _, Lmax, _ = K.shape
    R, C = nb.reshape(-1, nb.shape[-1]).shape
    NS = sel.shape[1]
    score = np.zeros((R, C), np.float32)
    nt = np.zeros((R, C), np.float32)
    lib().oro_errorgate(I(B), I(Lmax), I(C), I(NS), _p(_c(q, np.uint16)), _p(_c(K, np.uint16)),
                        _p(_c(asg, np.int32)), _p(_c(sel, np.int32)), _p(_c(Sk, np.float32)),
                        _p(_c(Sk2, np.float32)), _p(_c(nb, np.float32)), _p(score), _p(nt))
    return score, nt


def waterfill(score, nt, E):
    R, C = score.shape
    quota = np.zeros((R, C), np.float32)
    lib().oro_waterfill(I(R), I(C), F(float(E)), _p(_c(score, np.float32)), _p(_c(nt, np.float32)), _p(quota))
    return quota


def topq(s, asg, quota, n, E):
    R, sw = s.shape
    C = quota.shape[1]
    Lmax = asg.shape[-1]
    exp_idx = np.zeros((R, E), np.int32)
    lib().oro_topq(I(R), I(Lmax), I(C), I(E), I(n), _p(_c(s, np.uint16)), L(sw), _p(_c(asg, np.int32)),
                   _p(_c(quota, np.float32)), _p(exp_idx))
    return exp_idx


def residual(K, V, asg, sel, exp_idx, Sk, Sv, nt, quota):
    B, _, Lmax, _ = K.shape
    R, C = nt.shape
    kbar = np.zeros((R, C, D), np.uint16)
    vbar = np.zeros((R, C, D), np.uint16)
    logn = np.zeros((R, C), np.float32)
    lib().oro_residual(I(B), I(Lmax), I(C), I(sel.shape[1]), I(exp_idx.shape[1]), _p(_c(K, np.uint16)),
                       _p(_c(V, np.uint16)), _p(_c(asg, np.int32)), _p(_c(sel, np.int32)),
                       _p(_c(exp_idx, np.int32)), _p(_c(Sk, np.float32)), _p(_c(Sv, np.float32)),
                       _p(_c(nt, np.float32)), _p(_c(quota, np.float32)), _p(kbar), _p(vbar), _p(logn))
    return kbar, vbar, logn


def flash(q, k, v, sel, exp_idx, kbar, vbar, logn, sm_scale, per_qhead):
    """fp64 estimator.  q (BQ,D) uint16; k, v (BH,K,D) uint16; kbar/vbar (BQ|BH, NB, D) uint16."""
    BQ = q.shape[0]
    BH, Kd, _ = k.shape
    NB = 0 if kbar is None else kbar.shape[1]
    out = np.zeros((BQ, D), np.float64)
    lib().oro_flash(I(BQ), I(BH), L(Kd), I(sel.shape[1]), I(exp_idx.shape[1]), I(NB),
                    I(1 if per_qhead else BQ // BH), _p(_c(q, np.uint16)), _p(_c(k, np.uint16)),
                    _p(_c(v, np.uint16)), _p(_c(sel, np.int32)), _p(_c(exp_idx, np.int32)),
                    _p(None if kbar is None else _c(kbar, np.uint16)),
                    _p(None if vbar is None else _c(vbar, np.uint16)),
                    _p(None if logn is None else _c(logn, np.float32)), ctypes.c_double(sm_scale), _p(out))
    return out


def estimator_fp32(q, k, v, sel, exp_idx, Skr, Svr, nr, sm_scale=SC):
    """The fp32 estimator with UN-rounded proxies (kbar' = Skr/n', vbar' = Svr/n' kept in fp32):
    softmax([q.k*s over S and X, q.kbar'*s + ln n']) . [v, vbar'] evaluated in float64."""
    R = q.shape[0]
    qf = bf16_to_f32(q).astype(np.float64)
    out = np.zeros((R, D))
    Gq = R // k.shape[0]
    for r in range(R):
        idx = np.concatenate([sel[r], exp_idx[r]])
        idx = idx[idx >= 0]
        kr = bf16_to_f32(k[r // Gq, idx]).astype(np.float64)
        vr = bf16_to_f32(v[r // Gq, idx]).astype(np.float64)
        live = nr[r] > 0.5
        inv = 1.0 / np.maximum(nr[r][live], 1.0)
        kb = Skr[r][live].astype(np.float64) * inv[:, None]
        vb = Svr[r][live].astype(np.float64) * inv[:, None]
        z = np.concatenate([kr @ qf[r] * sm_scale, kb @ qf[r] * sm_scale + np.log(np.maximum(nr[r][live], 1.0))])
        p = np.exp(z - z.max())
        out[r] = (p[:len(idx)] @ vr + p[len(idx):] @ vb) / p.sum()
    return out


def residual_sums(K, V, asg, sel, exp_idx, Sk, Sv, nt, quota):
    """Unrounded residual sums in float64 (the inputs of estimator_fp32): Skr = Sk - the read tokens'
    k summed per cluster (selected tokens by their assignment, expanded tokens by the quota segment
    their slot falls in; pads skipped), Svr likewise, nr = nt - quota.  Same read sets as
    oro_residual (ours_fused.py:367-407)."""
    R, C, _ = Sk.shape
    B, _, Lmax, _ = K.shape
    Kf = K.reshape(B * HKV, Lmax, D)
    Vf = V.reshape(B * HKV, Lmax, D)
    Skr = Sk.astype(np.float64).copy()
    Svr = Sv.astype(np.float64).copy()
    for r in range(R):
        kv = r // (HQ // HKV)
        base = np.concatenate([[0], np.cumsum(quota[r].astype(np.int64))])
        toks, cls = [], []
        for t in sel[r]:
            if 0 <= t < Lmax:
                toks.append(t)
                cls.append(asg[r, t])
        for j, t in enumerate(exp_idx[r]):
            if 0 <= t < Lmax and j < base[C]:
                toks.append(t)
                cls.append(int(np.searchsorted(base, j, side="right") - 1))
        if toks:
            toks, cls = np.array(toks), np.array(cls)
            np.subtract.at(Skr[r], cls, bf16_to_f32(Kf[kv, toks]).astype(np.float64))
            np.subtract.at(Svr[r], cls, bf16_to_f32(Vf[kv, toks]).astype(np.float64))
    return Skr, Svr, (nt.astype(np.float64) - quota.astype(np.float64))


# ------------------------------------------------------------------ build stages (one request)
def build_codes(K1, U1, T):
    """K1 uint16 (8, Lmax, D), U1 (8, D, 32) -> scale (8, 32), codes (8, Lmax, 32) (first T rows)."""
    Lmax = K1.shape[1]
    scale = np.zeros((HKV, RQ), np.float32)
    codes = np.zeros((HKV, Lmax, RQ), np.int8)
    lib().oro_build_codes(I(T), I(Lmax), _p(_c(K1, np.uint16)), _p(_c(U1, np.float32)), _p(scale), _p(codes))
    return scale, codes


def project(K1, W1, T):
    Lmax = K1.shape[1]
    zP = np.zeros((HQ, T, RC), np.float32)
    colmean = np.zeros((HQ, RC), np.float32)
    lib().oro_project(I(T), I(Lmax), _p(_c(K1, np.uint16)), _p(_c(W1, np.uint16)), _p(zP), _p(colmean))
    return zP, colmean


def kmeans(zP, init, C, iters=4):
    """Lloyd iterations as methods_eager.py:533-545: returns asg (32, T), cent (32, C, 16), nb (32, C)."""
    T = zP.shape[1]
    init = np.ascontiguousarray(init, np.int64)
    cent = np.ascontiguousarray(zP[:, init, :])
    asg = np.zeros((HQ, T), np.int32)
    nb = np.zeros((HQ, C), np.float32)
    for _ in range(iters):
        lib().oro_kmeans_assign(I(T), I(C), _p(zP), _p(cent), _p(asg), L(T))
        lib().oro_kmeans_update(I(T), I(C), _p(zP), _p(asg), L(T), _p(init), _p(cent), _p(nb))
    return asg, cent, nb


def csr_sums(K1, V1, asg, T, C):
    Lmax = K1.shape[1]
    mem = np.zeros((HQ, Lmax), np.int32)
    cstart = np.zeros((HQ, C), np.int32)
    clen = np.zeros((HQ, C), np.int32)
    Sk = np.zeros((HQ, C, D), np.float32)
    Sk2 = np.zeros((HQ, C, D), np.float32)
    Sv = np.zeros((HQ, C, D), np.float32)
    lib().oro_csr_sums(I(T), I(Lmax), I(C), _p(_c(K1, np.uint16)), _p(_c(V1, np.uint16)), _p(_c(asg, np.int32)),
                       L(asg.shape[-1]), _p(mem), _p(cstart), _p(clen), _p(Sk), _p(Sk2), _p(Sv))
    return mem, cstart, clen, Sk, Sk2, Sv


# ------------------------------------------------------------------ metric and basis (torch, CPU)
def rot_avg(Mpre, inv_freq, scaling, p, w):
    """mean over t in [p, p+w) of R_t M R_t^T in closed form (static_top_k.py:102-131)."""
    th = torch.cat([inv_freq, inv_freq]).double()
    a, b = th.unsqueeze(1), th.unsqueeze(0)

    def mean_exp(alpha):
        if w <= 64:
            t = torch.arange(p, p + w, dtype=torch.float64)
            ph = alpha.unsqueeze(-1) * t
            return torch.complex(ph.cos().mean(-1), ph.sin().mean(-1))
        z = torch.polar(torch.ones_like(alpha), alpha)
        den = 1 - z
        small = den.abs() < 1e-9
        s = torch.where(small, torch.full_like(z, float(w)), (1 - z ** w) / torch.where(small, torch.ones_like(den), den))
        return s * torch.polar(torch.ones_like(alpha), alpha * p) / w

    Em, Ep = mean_exp(a - b), mean_exp(a + b)
    cc, ss = 0.5 * (Em.real + Ep.real), 0.5 * (Em.real - Ep.real)
    cs, sc = 0.5 * (Ep.imag - Em.imag), 0.5 * (Ep.imag + Em.imag)
    cc, ss, cs, sc = [x.float() * (scaling * scaling) for x in (cc, ss, cs, sc)]
    h = D // 2
    J = torch.zeros(D, D)
    J[:h, h:] = -torch.eye(h)
    J[h:, :h] = torch.eye(h)
    M = Mpre.float()
    return cc * M + cs * (M @ J.T) + sc * (J @ M) + ss * (J @ M @ J.T)


def metric(Mpre_l, inv_freq, scaling, qprefill, T, Qn, win=32, P=64):
    """M = 1/2 trnorm(static metric rotated to [T, T+win)) + 1/2 trnorm(question rows), (32, D, D)
    (methods_eager.py:510-518).  qprefill: (32, T, D) bf16 torch."""
    def nt(x):
        return x / torch.diagonal(x, dim1=-2, dim2=-1).sum(-1).clamp(min=1e-12)[..., None, None]
    Mst = rot_avg(Mpre_l, inv_freq, scaling, T, win)
    Pn = min(P, max(Qn - 2, 1))
    pi = torch.linspace(0, max(Qn - 3, 0), Pn).long().unique()
    qsel = qprefill[:, T - Qn:, :].index_select(1, pi).float()
    freqs = (Qn - pi).float().unsqueeze(-1) * inv_freq.unsqueeze(0)
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos() * scaling, emb.sin() * scaling
    h = D // 2
    qrot = qsel * cos + torch.cat([-qsel[..., h:], qsel[..., :h]], -1) * sin
    Mq = torch.matmul(qrot.transpose(-1, -2), qrot) / qrot.shape[1]
    return 0.5 * nt(Mst) + 0.5 * nt(Mq)


def basis(M):
    """U (8, D, 32) from the KV-head mean metric; W (32, D, 16) bf16 = U16 * sqrt(max(lambda, 0))
    (methods_eager.py:520-528)."""
    _, Ukv = torch.linalg.eigh(M.view(HKV, G, D, D).mean(1))
    U = Ukv[..., -RQ:].contiguous()
    ev, Uq = torch.linalg.eigh(M)
    W = (Uq[..., -RC:] * ev[..., -RC:].clamp(min=0).sqrt().unsqueeze(-2)).to(torch.bfloat16)
    return U, W


def seeds(T, C, layer):
    g = torch.Generator(device="cpu").manual_seed(31 * (layer + 1))
    return torch.randperm(T, generator=g)[:C].numpy().astype(np.int64)


# ------------------------------------------------------------------ whole-step orchestration
def step_split(n, rho, C, E):
    """sink = local = max(1, int(1e-4 n)); k_top from the heavy fraction (methods_eager.py:605-607)."""
    ns = nl = max(1, int(0.0001 * n))
    heavy = rho - 0.0002 - E / 32768 - 1.5 * C / 32768
    return ns, nl, max(1, int(heavy * n))


def new_state(B, Lmax, C, rmax=256):
    z = np.zeros
    return dict(codes=z((B, HKV, Lmax, RQ), np.int8), U=z((B, HKV, D, RQ), np.float32),
                scale=z((B, HKV, RQ), np.float32), W=z((B, HQ, D, RC), np.uint16),
                colmean=z((B, HQ, RC), np.float32), cent=z((B, HQ, C, RC), np.float32),
                asg=z((B, HQ, Lmax), np.int32), nb=z((B, HQ, C), np.float32), Sk=z((B, HQ, C, D), np.float32),
                Sk2=z((B, HQ, C, D), np.float32), Sv=z((B, HQ, C, D), np.float32),
                mem=z((B, HQ, Lmax), np.int32), cstart=z((B, HQ, C), np.int32), clen=z((B, HQ, C), np.int32),
                reclist=z((B, HQ, C, rmax), np.int32), reccnt=z((B, HQ, C), np.int32))


def build_from_basis(st, b, K1, V1, U1, W1, T, layer):
    """Everything of the build after the eigen-decomposition, for request b (K1, V1 uint16 (8, Lmax, D))."""
    C = st["nb"].shape[-1]
    scale, codes = build_codes(K1, U1, T)
    st["U"][b], st["scale"][b] = U1, scale
    st["codes"][b, :, :T] = codes[:, :T]
    zP, colmean = project(K1, W1, T)
    asg, cent, nb = kmeans(zP, seeds(T, C, layer), C)
    st["W"][b], st["colmean"][b], st["cent"][b], st["nb"][b] = W1, colmean, cent, nb
    st["asg"][b, :, :T] = asg
    mem, cstart, clen, Sk, Sk2, Sv = csr_sums(K1, V1, asg, T, C)
    st["mem"][b], st["cstart"][b], st["clen"][b] = mem, cstart, clen
    st["Sk"][b], st["Sk2"][b], st["Sv"][b] = Sk, Sk2, Sv
    st["reccnt"][b] = 0
    return zP


def decode_step(st, q, K, V, n, rho, C, E):
    """One deployed decode step at length n (new token already at n-1 in K/V).  q uint16 (R, D);
    K, V uint16 (B, 8, Lmax, D).  Returns every intermediate and the fp64 flash output."""
    ns, nl, k_top = step_split(n, rho, C, E)
    B = K.shape[0]
    R = B * HQ
    index_update(st, K, V, n - 1)
    zqv = zq(q, st["U"].reshape(B * HKV, D, RQ), st["scale"].reshape(B * HKV, RQ))
    s = scan(st["codes"], zqv, n, ns, nl)
    s_raw = s.copy()
    sel = select(s, n, ns, nl, k_top)
    asg = st["asg"].reshape(R, -1)
    score, nt = errorgate(q, K, asg, sel, st["Sk"].reshape(R, C, D), st["Sk2"].reshape(R, C, D),
                          st["nb"].reshape(R, C))
    quota = waterfill(score, nt, E)
    exp_idx = topq(s, asg, quota, n, E)
    kbar, vbar, logn = residual(K, V, asg, sel, exp_idx, st["Sk"].reshape(R, C, D), st["Sv"].reshape(R, C, D),
                                nt, quota)
    Kf = K.reshape(B * HKV, K.shape[2], D)
    Vf = V.reshape(B * HKV, V.shape[2], D)
    out = flash(q, Kf, Vf, sel, exp_idx, kbar, vbar, logn, SC, per_qhead=True)
    return dict(ns=ns, nl=nl, k_top=k_top, zq=zqv, s=s_raw, s_masked=s, sel=sel, score=score, nt=nt, quota=quota,
                exp_idx=exp_idx, kbar=kbar, vbar=vbar, logn=logn, out=out)
