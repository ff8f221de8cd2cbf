"""The deployed OpenAttention method on B200: the drop-in for the reference's `Method` classes
(inference/methods_eager.py:243-266 Method, :468-662 Ours; inference/ours_graph.py:265-347 OursG2;
inference/ours_fastbuild.py:143-307 OursG3 "ours3").

    C.K = [...]; C.V = [...]          # per layer (B, 8, Lmax, 128) bf16 caches, owned by the caller
    a = SimpleNamespace(rho=0.01, static_metric_path="llama-3.1-8b-instruct.query_metric.triu.pt")
    m = OursB200(a, B, Lmax, "cuda")  # the metric: the reference's asset (packed or unpacked form)
    m.build(l, b, q_prefill, T)       # prefill: per layer and batch row, after K/V[:, :, :T] are written
    out = m.decode(l, q, n)           # decode: q (B, 32, 1, 128) bf16, new token already at n - 1

Every compute step is a kernel of the C-ABI library (selection.py / flash.py / the build entry
points); torch only allocates memory, runs the per-request eigen-decomposition of the 128x128 query
metric (torch.linalg.eigh, as the reference) and draws the k-means seeds (CPU randperm, as the
reference).  The step is CUDA-graph safe: it reads the current length from `C.n_dev` and the
prefix length from `C.n0_dev` when the caller provides them (graph_runner.py:601-603), never syncs
with the host, and all per-step buffers are preallocated in __init__.
"""
from __future__ import annotations

import os

import torch

from . import _lib
from . import flash as flash_mod
from . import selection as S
from .geometry import D, G, HKV, HQ, ITERS, PQ, RC, RMAX, RQ, WIN, budget, llama31_inv_freq, step_split

NL = 32  # layers a method instance holds state for (methods_eager.NL)


class Ctx:
    """Run state shared with the attention hook (inference/methods_eager.py:176-189)."""
    phase = "prefill"
    brow = 0
    n = 0
    K = V = None        # per layer (B, HKV, Lmax, D)
    qlen = []           # question-chunk length per batch row
    method = None
    n_dev = None        # device int32 (1,): current length incl. the new token (graph mode)
    n0_dev = None       # device int32 (1,): prefix length at build (graph mode)
    kv_idx = None       # device int64 (1,): write position of the new token (graph mode)


C = Ctx()


# ------------------------------------------------------------------ static query metric
def rot_avg(Mpre: torch.Tensor, inv_freq: torch.Tensor, scaling: float, p: int, w: int) -> torch.Tensor:
    """mean over t in [p, p+w) of R_t M R_t^T in closed form, R_t the RoPE rotation at position t
    (StaticTopKMasker._rot_avg, static_top_k.py:102-131)."""
    dev = Mpre.device
    th = torch.cat([inv_freq, inv_freq]).double().to(dev)
    a, b = th.unsqueeze(1), th.unsqueeze(0)

    def mean_exp(alpha):
        if w <= 64:
            t = torch.arange(p, p + w, device=dev, dtype=torch.float64)
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
    J = torch.zeros(D, D, device=dev)
    J[:h, h:] = -torch.eye(h, device=dev)
    J[h:, :h] = torch.eye(h, device=dev)
    M = Mpre.float()
    return cc * M + cs * (M @ J.T) + sc * (J @ M) + ss * (J @ M @ J.T)


def question_rows(Qn: int, P: int = PQ) -> torch.Tensor:
    """Indices (into the last Qn prefill rows) of the question rows the metric uses: up to P rows spread
    over [0, Qn - 3] (inference/methods_eager.py:512-513).  A host tensor."""
    Pn = min(P, max(Qn - 2, 1))
    return torch.linspace(0, max(Qn - 3, 0), Pn).long().unique()


def metric_from_rows(Mst, qsel, pi, Qn, inv_freq, scaling):
    """M = 1/2 trnorm(Mst) + 1/2 trnorm(Mq), Mq the mean outer product of the question rows qsel
    (32, P, D) fp32 rotated back by RoPE at offsets Qn - pi (inference/methods_eager.py:514-518)."""
    def nt(x):
        return x / torch.diagonal(x, dim1=-2, dim2=-1).sum(-1).clamp(min=1e-12)[..., None, None]
    freqs = (Qn - pi).float().unsqueeze(-1) * inv_freq.unsqueeze(0)
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos() * scaling, emb.sin() * scaling
    h = D // 2
    qrot = qsel * cos + torch.cat([-qsel[..., h:], qsel[..., :h]], -1) * sin
    Mq = torch.matmul(qrot.transpose(-1, -2), qrot) / qrot.shape[1]
    return 0.5 * nt(Mst) + 0.5 * nt(Mq)


def query_metric(Mpre_l, inv_freq, scaling, q, T, Qn, win=WIN, P=PQ):
    """M = 1/2 trnorm(static metric rotated to [T, T+win)) + 1/2 trnorm(question rows)
    (inference/methods_eager.py:510-518), all on q's device.  q: (1, 32, T, D) prefill queries.
    OursB200 evaluates the same function on the host (rot_avg + metric_from_rows on CPU tensors), the
    reference's CPU arithmetic, so that its bases equal the reference's bit for bit."""
    Mst = rot_avg(Mpre_l, inv_freq, scaling, T, win)
    pi = question_rows(Qn, P)
    qsel = q[0, :, T - Qn:, :].index_select(1, pi.to(q.device)).float()
    return metric_from_rows(Mst, qsel, pi.to(q.device), Qn, inv_freq.to(q.device), scaling)


def basis_from_metric(M: torch.Tensor):
    """U (8, D, 32): top-32 eigenvectors of each KV head's mean metric; W (32, D, 16) bf16 =
    top-16 eigenvectors scaled by sqrt(max(eigenvalue, 0)) (inference/methods_eager.py:520-528).

    The 40 symmetric 128 x 128 eigen-decompositions run on the host (batched LAPACK, about 2.6 MB
    each way): the device solver takes the matrices one at a time and costs about 90 ms per layer.
    An eigenvector is defined up to its sign; a flipped column of U changes zq and the codes together
    (their products, the scores, do not change), and a flipped column of W changes the projected keys
    and the centroids together, so the selection is the same."""
    U, W = basis_from_host_metric(M.detach().to("cpu", torch.float32))
    return U.to(M.device), W.to(M.device)


def basis_from_host_metric(Mh: torch.Tensor):
    """basis_from_metric on a host copy of M (4 hkv, D, D) fp32 (32 heads, or a KV-head shard's query heads);
    returns host tensors U (hkv, D, 32) and W (4 hkv, D, 16)."""
    _, Ukv = torch.linalg.eigh(Mh.view(-1, G, D, D).mean(1))
    ev, Uq = torch.linalg.eigh(Mh)
    U = Ukv[..., -RQ:].contiguous()
    W = (Uq[..., -RC:] * ev[..., -RC:].clamp(min=0).sqrt().unsqueeze(-2)).to(torch.bfloat16).contiguous()
    return U, W


def kmeans_seeds(T: int, Cn: int, layer: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(31 * (layer + 1))
    return torch.randperm(T, generator=g)[:Cn]


def unpack_metric(packed: dict) -> torch.Tensor:
    """The full symmetric metric (..., d, d) from the shipped upper-triangle form {"M_triu": (..., d(d+1)/2),
    "dim": d} (assets/restore_query_metric.py:18-27): entry k of a row of M_triu is M[i, j] = M[j, i]
    for the k-th pair (i <= j) in row-major order of the upper triangle."""
    d = int(packed["dim"])
    tri = packed["M_triu"]
    if tri.shape[-1] != d * (d + 1) // 2:
        raise RuntimeError(f"M_triu has {tri.shape[-1]} entries per matrix, a {d}x{d} triangle has {d * (d + 1) // 2}")
    i, j = torch.triu_indices(d, d)
    M = tri.new_zeros(*tri.shape[:-1], d, d)
    M[..., i, j] = tri
    M[..., j, i] = tri
    return M


def load_static_metric(a, layers: int):
    """(M (L, 32, D, D) fp32 pre-RoPE query metric, inv_freq (64,), attention scaling).

    Source, first found: `a.static_metric` (a tensor, or a dict in either asset form), the file
    `a.static_metric_path`, the file named by OA_STATIC_M.  Both forms of the reference's asset are
    read: the shipped packed one (assets/llama-3.1-8b-instruct.query_metric.triu.pt: "M_triu", "dim",
    "inv_freq", "attention_scaling") and the unpacked one the reference writes on first use ("M", ...,
    inference/methods_eager.py:474-480).  Without a metric this raises: the QGS and QGC bases are
    derived from it, and a made-up metric would silently select different tokens."""
    src = getattr(a, "static_metric", None)
    path = getattr(a, "static_metric_path", None) or os.environ.get("OA_STATIC_M")
    if src is None and path:
        if not os.path.exists(path):
            raise RuntimeError(f"static query metric file {path!r} does not exist")
        src = torch.load(path, map_location="cpu", weights_only=False)
    if src is None:
        raise RuntimeError("no static query metric: pass a.static_metric (tensor or asset dict), "
                           "a.static_metric_path, or set OA_STATIC_M to the reference's asset "
                           "(llama-3.1-8b-instruct.query_metric.triu.pt or its unpacked form)")
    if isinstance(src, dict):
        M = unpack_metric(src) if "M_triu" in src else src["M"]
        inv = src.get("inv_freq")
        inv = llama31_inv_freq() if inv is None else inv
        M, scaling = M.float(), float(src.get("attention_scaling", 1.0))
    else:
        M, inv, scaling = src.float(), llama31_inv_freq(), 1.0
    if M.dim() != 4 or tuple(M.shape[1:]) != (HQ, D, D):
        raise RuntimeError(f"static metric must be (layers, {HQ}, {D}, {D}), got {tuple(M.shape)}")
    if M.shape[0] < layers:
        raise RuntimeError(f"static metric holds {M.shape[0]} layers, the method needs {layers}")
    return M[:layers].contiguous(), inv.float(), scaling


# ------------------------------------------------------------------ the method
class OursB200:
    """OpenAttention decode (QGS scan + top-k, ErrorGate + water-filling, within-cluster top-q,
    residual proxies, OpenAttention.flash) with the per-request QGC/QGS build.

    FUSED (default): the residual proxies and the attention run as one kernel (the K/V rows of the
    read tokens are gathered once); keep_proxies additionally writes kbar', vbar', ln n' out.
    FUSED = False runs oa_residual and then calls `flash.ours_flash` through the module attribute,
    the hook the reference's tests spy on; decode takes that path too whenever `flash.ours_flash` has
    been replaced, so a harness that installs a spy sees the step's sel / exp_idx / proxies."""
    name = "ours3"
    FUSED = True
    keep_proxies = False

    def __init__(self, a, B, Lmax, dev, layers: int | None = None, kv_heads: tuple[int, int] | None = None):
        """kv_heads = (k0, kc): this instance holds KV heads k0 .. k0+kc-1 of every request (a KV-head shard:
        caches C.K[l] / C.V[l] are (B, kc, Lmax, 128), decode queries (B, 4 kc, 1, 128) for query heads
        4 k0 .. 4 (k0+kc) - 1); default all 8."""
        self.a, self.B, self.Lmax = a, B, Lmax
        self.dev = torch.device(dev)
        if self.dev.type != "cuda":
            raise RuntimeError("OursB200 runs on CUDA devices only (no CPU fallback)")
        _lib.load()
        k0, kc = kv_heads if kv_heads is not None else getattr(a, "kv_heads", None) or (0, HKV)
        if not (0 <= k0 and 1 <= kc and k0 + kc <= HKV):
            raise RuntimeError(f"kv_heads {(k0, kc)} is not a range of the {HKV} KV heads")
        self.k0, self.hkv, self.hq = k0, kc, G * kc
        self.R = B * self.hq
        self.C, self.E = budget(a.rho)
        self.NL = layers or getattr(a, "layers", None) or NL
        Mpre, inv_freq, scaling = load_static_metric(a, self.NL)
        # the metric is evaluated on the host, in the reference's CPU arithmetic (see build_async)
        self.Mpre = Mpre.cpu()[:, G * k0:G * (k0 + kc)].contiguous()  # this shard's query heads
        self.inv_freq = inv_freq.cpu()
        self.scaling = scaling
        self._mst = {}  # layer -> (T, static metric rotated to T): shared by the requests of one prefill length
        self.st = [S.new_state(B, Lmax, self.C, self.dev, RMAX, hkv=kc) for _ in range(self.NL)]
        R, Cn, E, dev = self.R, self.C, self.E, self.dev
        self.NT = (Lmax + 31) // 32          # 32-token tiles of the QGS tile maxima
        self.SW = S.padded_len(Lmax)
        self.zq = torch.zeros(R, RQ, dtype=torch.bfloat16, device=dev)
        self.scores = torch.zeros(R, self.SW, dtype=torch.bfloat16, device=dev)
        self.tmax = torch.zeros(R, self.NT, dtype=torch.float32, device=dev)
        self.score = torch.zeros(R, Cn, device=dev)
        self.nt = torch.zeros(R, Cn, device=dev)
        self.zdot = torch.zeros(R, Cn, device=dev)  # ErrorGate's tail-mean dots, reused by the fused flash
        self.quota = torch.zeros(R, Cn, device=dev)
        self.exp_idx = torch.full((R, E), -1, dtype=torch.int32, device=dev)
        self.topq_ws = S.topq_workspace(R, Lmax, E, dev)  # only for rows too long for shared memory
        self.kbar = torch.zeros(R, Cn, D, dtype=torch.bfloat16, device=dev)
        self.vbar = torch.zeros(R, Cn, D, dtype=torch.bfloat16, device=dev)
        self.logn = torch.zeros(R, Cn, device=dev)
        self.out = torch.zeros(R, D, dtype=torch.bfloat16, device=dev)
        self._sel = {}
        self._n_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)  # kernel-side error flag (bounded waits)
        self._n0_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        lib = _lib.load()
        # the automatic split count depends on the list length (chunk rounding): size for the largest
        nbytes = max(lib.oa_flash_workspace_bytes(R, ns, E, Cn, 0) for ns in range(1, 513))
        self.flash_ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev) if nbytes else None
        self._quota = self.quota
        self.read_frac = 0.0

    # ---------------------------------------------------------------- build (prefill)
    def build(self, l, b, q, T):
        """Index of layer l, batch row b after the prefill wrote C.K[l][b, :, :T], C.V[l][b, :, :T];
        q: (1, 32, T, D) prefill queries (the last C.qlen[b] rows are the question); a KV-head shard takes
        either all 32 query heads or its own 4 kc."""
        self.build_async(l, b, q, T)()

    def build_async(self, l, b, q, T):
        """build() in two halves.  Now: the question rows of q (at most 64 per head) are copied to pinned
        host memory (q is not used after this returns).  The returned callable: the query metric and its
        eigen-decomposition on the host, then the device build.  A prefill loop calls it after enqueueing
        its next layer, so the host half overlaps device work.

        The metric is host arithmetic on purpose: it is the reference's own CPU computation, so the
        bases (and through them codes and clusters) are bit-identical to the reference's; a device
        evaluation would round its fp32 matmuls differently and perturb the eigenvectors."""
        Qn = C.qlen[b] if C.qlen else 40
        pi = question_rows(Qn)
        if q.shape[1] == HQ and self.hq != HQ:
            q = q[:, G * self.k0:G * self.k0 + self.hq]
        if q.shape[1] != self.hq:
            raise RuntimeError(f"prefill queries hold {q.shape[1]} heads; this instance builds {self.hq}")
        rows = q[0, :, T - Qn:, :].index_select(1, pi.pin_memory().to(q.device, non_blocking=True))
        rows_h = torch.empty(rows.shape, dtype=rows.dtype, pin_memory=True)
        rows_h.copy_(rows, non_blocking=True)
        done = torch.cuda.Event()
        done.record()

        def finish():
            hit = self._mst.get(l)
            if hit is None or hit[0] != T:
                hit = (T, rot_avg(self.Mpre[l], self.inv_freq, self.scaling, T, WIN))
                self._mst[l] = hit
            done.synchronize()
            M = metric_from_rows(hit[1], rows_h.float(), pi, Qn, self.inv_freq, self.scaling)
            U, W = basis_from_host_metric(M)
            self.build_from_basis(l, b, U.to(self.dev, non_blocking=True), W.to(self.dev, non_blocking=True), T)
        return finish

    def build_from_basis(self, l, b, U, W, T):
        """Everything of the build after the eigen-decomposition (QGS codes, QGC projection, Lloyd
        iterations, CSR member lists, cluster sums), all on the GPU."""
        st, dev, Cn, Lmax = self.st[l], self.dev, self.C, self.Lmax
        K1, V1 = C.K[l][b], C.V[l][b]
        stream = torch.cuda.current_stream(dev).cuda_stream
        p = _lib.ptr
        st["U"][b].copy_(U)
        st["W"][b].copy_(W)
        lib = _lib.load()
        hkv = self.hkv
        amax = torch.empty(hkv * RQ, dtype=torch.int32, device=dev)
        _lib.call("oa_build_codes", p(K1), hkv, Lmax, T, p(st["U"][b]), p(st["scale"][b]), p(st["codes"][b]), p(amax),
                  stream)
        zP = torch.empty(self.hq, T, RC, device=dev)
        ws = torch.empty(max(lib.oa_build_project_workspace_bytes(T), lib.oa_csr_workspace_bytes(T, Cn)),
                         dtype=torch.uint8, device=dev)
        _lib.call("oa_build_project", p(K1), hkv, Lmax, T, p(st["W"][b]), p(zP), p(st["colmean"][b]), p(ws),
                  ws.numel(), stream)
        init = kmeans_seeds(T, Cn, l).to(dev)
        cent = st["cent"][b]
        cent.copy_(zP.index_select(1, init))
        for _ in range(ITERS):
            _lib.call("oa_kmeans_assign", p(zP), hkv, T, Cn, p(cent), p(st["asg"][b]), Lmax, stream)
            _lib.call("oa_csr_build", p(st["asg"][b]), Lmax, hkv, T, Cn, p(st["mem"][b]), Lmax, p(st["cstart"][b]),
                      p(st["clen"][b]), p(ws), ws.numel(), stream)
            _lib.call("oa_kmeans_update", p(zP), hkv, T, Cn, p(st["mem"][b]), Lmax, p(st["cstart"][b]),
                      p(st["clen"][b]), p(init), p(cent), p(st["nb"][b]), stream)
        _lib.call("oa_cluster_sums", p(K1), p(V1), hkv, Lmax, Cn, p(st["mem"][b]), Lmax, p(st["cstart"][b]),
                  p(st["clen"][b]), p(st["Sk"][b]), p(st["Sk2"][b]), p(st["Sv"][b]), stream)
        if "reccnt" in st:
            st["reccnt"][b].zero_()
        self._n0_dev.fill_(T)

    # ---------------------------------------------------------------- decode step
    def _sel_buf(self, NS):
        if NS not in self._sel:
            self._sel[NS] = torch.zeros(self.R, NS, dtype=torch.int32, device=self.dev)
        return self._sel[NS]

    def select(self, l, q, n, residual=True, k_new=None, v_new=None):
        """Stages 1-5 of the step: index update + zq, QGS scan + top-k, ErrorGate + water-filling,
        within-cluster top-q and (residual=True) the residual proxies.  Returns (q rows, sel)."""
        st, Lmax = self.st[l], self.Lmax
        K, V = C.K[l], C.V[l]
        n_dev = C.n_dev if C.n_dev is not None else self._n_dev.fill_(n)
        ns, nl, k_top = step_split(n, self.a.rho, self.C, self.E)
        qr = q.reshape(self.R, D)
        if not qr.is_contiguous():
            qr = qr.contiguous()
        sel = self._sel_buf(ns + nl + k_top)
        S.index_update(K, V, st, n_dev, q=qr, zq=self.zq, k_new=k_new, v_new=v_new)
        S.qgs_scan(st["codes"], self.zq, n_dev, ns, nl, self.scores, self.tmax, self.status)
        S.qgs_select(self.scores, self.tmax, Lmax, n_dev, ns, nl, k_top, sel)
        S.errorgate_waterfill(qr, K, st, sel, self.E, self.score, self.nt, self.quota, self.status, zdot=self.zdot)
        n0_dev = C.n0_dev if C.n0_dev is not None else self._n0_dev
        S.topq(self.scores, st, self.quota, self.E, n_dev, n0_dev, self.exp_idx, self.status, workspace=self.topq_ws)
        if residual:
            S.residual(K, V, st, sel, self.exp_idx, self.nt, self.quota, self.kbar, self.vbar, self.logn,
                       self.status)
        self._quota = self.quota
        self.last_sel = sel
        self.read_frac = (ns + nl + k_top + self.E + 1.5 * self.C) / n
        return qr, sel

    def decode(self, l, q, n, k_new=None, v_new=None):
        """The reference's decode(l, q, n) (the new token's K/V already in C.K[l] / C.V[l] at n - 1).  With
        k_new, v_new (B, 8, 128) bf16 the caller leaves that write to the index update, which does it in
        the same launch (oa_index_update_append)."""
        if not self.FUSED or flash_mod.ours_flash is not _OURS_FLASH:
            # unfused, or a caller has replaced flash.ours_flash (the reference's equivalence harnesses
            # swap bl.ours_flash for a spy that records sel / exp_idx / the proxies): the residual proxies
            # are formed and the attention goes through that attribute, so the spy sees every call
            qr, sel = self.select(l, q, n, k_new=k_new, v_new=v_new)
            return self.attend(l, qr, sel, self.exp_idx, self.kbar, self.vbar, self.logn)
        qr, sel = self.select(l, q, n, residual=False, k_new=k_new, v_new=v_new)
        keep = self.keep_proxies
        S.residual_flash(qr, C.K[l], C.V[l], self.st[l], sel, self.exp_idx, self.nt, self.quota, self.out,
                         kbar=self.kbar if keep else None, vbar=self.vbar if keep else None,
                         logn=self.logn if keep else None, status=self.status, zdot=self.zdot)
        return self.out.view(self.B, self.hq, 1, D)

    def attend(self, l, qr, sel, exp_idx, kbar_r, vbar_r, logn):
        """OpenAttention.flash with per-query-head proxies, called through the module attribute
        flash.ours_flash so tests can spy on it (as the reference's bl.ours_flash)."""
        Lmax = self.Lmax
        out = flash_mod.ours_flash(qr, C.K[l].view(-1, Lmax, D), C.V[l].view(-1, Lmax, D), sel, exp_idx, kbar_r,
                                   vbar_r, logn, out=self.out, workspace=self.flash_ws)
        return out.view(self.B, self.hq, 1, D)


METHODS = {"ours3": OursB200, "ours": OursB200}
_OURS_FLASH = flash_mod.ours_flash  # the library's own operator (a replaced attribute is a caller's hook)
