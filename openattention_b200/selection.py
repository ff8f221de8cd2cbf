"""Torch-tensor wrappers over the C-ABI selection stages (one call = one kernel launch on the current
stream).  Shapes follow the state layout of include/openattention_b200.h; all tensors must be CUDA,
contiguous and of the stated dtype (checked here, so the C side only sees valid layouts).

A KV-head shard of the requests (hkv of their 8 KV heads, and the 4 hkv query heads that read them) uses
the same wrappers: the caches are (B, hkv, Lmax, 128), the per-query-head state (B, 4 hkv, ...), and
hkv is read from the cache shape."""
from __future__ import annotations

import torch

from . import _lib
from .geometry import D, G, HKV, RC, RQ

_ptr = _lib.ptr


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(name, t, dtype, shape=None):
    if t is None:
        return
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f"{name}: need a contiguous CUDA {dtype} tensor, got {t.dtype} "
                           f"{'cuda' if t.is_cuda else 'cpu'} contiguous={t.is_contiguous()}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name}: shape {tuple(t.shape)} != {tuple(shape)}")


def _on(dev, *named):
    """Every given (name, tensor) pair, None skipped, is a CUDA tensor on `dev`.  A kernel given a host
    tensor's address would fault or, on a GPU that can reach host memory, silently read the wrong
    memory; a tensor on another GPU would be read across the link, or not at all."""
    for name, t in named:
        if t is not None and (not t.is_cuda or t.device != dev):
            raise RuntimeError(f"{name}: need a tensor on {dev}, got one on {t.device}")


def _state_on(dev, st):
    _on(dev, *((f"state[{k!r}]", t) for k, t in st.items()))


def _rows(name, t, dtype, R, cols=None):
    """(R, cols) rows of `dtype` whose last dimension is contiguous (the row stride is passed on)."""
    if t.dtype != dtype or t.dim() != 2 or t.shape[0] != R or t.stride(1) != 1 or (cols is not None and t.shape[1] != cols):
        raise RuntimeError(f"{name}: need ({R}, {cols if cols is not None else 'n'}) {dtype} rows with a contiguous "
                           f"last dim, got {tuple(t.shape)} {t.dtype}")


def _heads(K):
    """(B, hkv, Lmax) of a cache (B, hkv, Lmax, 128): hkv KV heads per request (8, or a shard's subset)."""
    B, hkv, Lmax, _ = K.shape
    if not 1 <= hkv <= HKV:
        raise RuntimeError(f"K holds {hkv} KV heads per request; 1..{HKV} are supported")
    return B, hkv, Lmax


def append_kv(K, V, k_new, v_new, n_dev, offset=0, advance=True, kv_idx=None):
    """Writes the new token's K/V rows (B, hkv, 128) at position n_dev + offset of the caches (B, hkv, Lmax,
    128) in one launch; with advance, n_dev += 1 and kv_idx (int64, optional) = the old n_dev."""
    B, hkv, Lmax = _heads(K)
    _need("K", K, torch.bfloat16, (B, hkv, Lmax, D))
    _need("V", V, torch.bfloat16, (B, hkv, Lmax, D))
    _need("k_new", k_new, torch.bfloat16, (B, hkv, D))
    _need("v_new", v_new, torch.bfloat16, (B, hkv, D))
    _need("n_dev", n_dev, torch.int32, (1,))
    if kv_idx is not None:
        _need("kv_idx", kv_idx, torch.int64, (1,))
    _on(K.device, ("V", V), ("k_new", k_new), ("v_new", v_new), ("n_dev", n_dev), ("kv_idx", kv_idx))
    _lib.call("oa_append_kv", _ptr(K), _ptr(V), B, hkv, Lmax, _ptr(k_new), _ptr(v_new), _ptr(n_dev), int(offset),
              1 if advance else 0, _ptr(kv_idx), _stream(K))


def index_update(K, V, st, n_dev, q=None, zq=None, k_new=None, v_new=None):
    """New token at n-1 joins the index; with q (B*4*hkv, D) also writes zq (B*4*hkv, 32) bf16.  With
    k_new, v_new (B, hkv, 128) the token's rows are written into K, V at n-1 by the same launch."""
    B, hkv, Lmax = _heads(K)
    C = st["nb"].shape[-1]
    _need("K", K, torch.bfloat16, (B, hkv, Lmax, D))
    _need("V", V, torch.bfloat16, (B, hkv, Lmax, D))
    _need("n_dev", n_dev, torch.int32, (1,))
    if q is not None:
        if q.dtype != torch.bfloat16 or q.stride(-1) != 1 or q.shape != (B * G * hkv, D):
            raise RuntimeError(f"q must be ({B * G * hkv}, 128) bf16 with a contiguous last dim")
        _need("zq", zq, torch.bfloat16, (B * G * hkv, RQ))
    _on(K.device, ("V", V), ("n_dev", n_dev), ("q", q), ("zq", zq), ("k_new", k_new), ("v_new", v_new))
    _state_on(K.device, st)
    rec = st.get("reclist")
    rmax = 0 if rec is None else rec.shape[-1]
    tail = (_ptr(st["codes"]), _ptr(st["U"]), _ptr(st["scale"]), _ptr(st["W"]), _ptr(st["colmean"]), _ptr(st["cent"]),
            _ptr(st["asg"]), _ptr(st["nb"]), _ptr(st["Sk"]), _ptr(st["Sk2"]), _ptr(st["Sv"]), _ptr(rec),
            _ptr(st.get("reccnt")), rmax, _ptr(q), 0 if q is None else q.stride(0), _ptr(zq), _ptr(n_dev), _stream(K))
    if k_new is None:
        _lib.call("oa_index_update", _ptr(K), _ptr(V), B, hkv, Lmax, C, *tail)
        return
    _need("k_new", k_new, torch.bfloat16, (B, hkv, D))
    _need("v_new", v_new, torch.bfloat16, (B, hkv, D))
    _lib.call("oa_index_update_append", _ptr(K), _ptr(V), B, hkv, Lmax, C, _ptr(k_new), _ptr(v_new), *tail)


def qgs_scan(codes, zq, n_dev, ns, nl, scores, tile_max, status=None):
    B, hkv, Lmax = _heads(codes)
    _need("codes", codes, torch.int8)
    _need("zq", zq, torch.bfloat16, (B * G * hkv, RQ))
    if scores.dtype != torch.bfloat16 or tile_max.dtype != torch.float32 or scores.stride(1) != 1:
        raise RuntimeError("scores must be bf16 (R, >= Lmax) and tile_max fp32 (R, >= NT)")
    _on(codes.device, ("zq", zq), ("n_dev", n_dev), ("scores", scores), ("tile_max", tile_max), ("status", status))
    _lib.call("oa_qgs_scan", _ptr(codes), _ptr(zq), B, hkv, Lmax, _ptr(n_dev), int(ns), int(nl), _ptr(scores),
              scores.stride(0), _ptr(tile_max), tile_max.stride(0), _ptr(status), _stream(codes))


def qgs_select(scores, tile_max, Lmax, n_dev, ns, nl, k_top, sel):
    R = scores.shape[0]
    _need("sel", sel, torch.int32, (R, ns + nl + k_top))
    _rows("scores", scores, torch.bfloat16, R)
    _rows("tile_max", tile_max, torch.float32, R)
    _on(scores.device, ("tile_max", tile_max), ("n_dev", n_dev), ("sel", sel))
    _lib.call("oa_qgs_select", _ptr(scores), scores.stride(0), _ptr(tile_max), tile_max.stride(0), R, Lmax,
              _ptr(n_dev), int(ns), int(nl), int(k_top), _ptr(sel), _stream(scores))


def errorgate_waterfill(q, K, st, sel, E, score, nt, quota, status=None, zdot=None):
    """zdot (optional, (R, C) fp32): receives q . kbar of each cluster's tail mean, for residual_flash."""
    B, hkv, Lmax = _heads(K)
    C = st["nb"].shape[-1]
    R = B * G * hkv
    for nm, t in (("score", score), ("nt", nt), ("quota", quota), ("zdot", zdot)):
        _need(nm, t, torch.float32, (R, C))
    _need("sel", sel, torch.int32)
    _need("K", K, torch.bfloat16, (B, hkv, Lmax, D))
    _rows("q", q, torch.bfloat16, R, D)
    _on(K.device, ("q", q), ("sel", sel), ("score", score), ("nt", nt), ("quota", quota), ("zdot", zdot),
        ("status", status))
    _state_on(K.device, st)
    _lib.call("oa_errorgate_waterfill", _ptr(q), q.stride(0), _ptr(K), B, hkv, Lmax, C, _ptr(st["asg"]), _ptr(sel),
              sel.shape[1], _ptr(st["Sk"]), _ptr(st["Sk2"]), _ptr(st["nb"]), float(E), _ptr(score), _ptr(nt),
              _ptr(quota), _ptr(zdot), _ptr(status), _stream(K))


def topq_workspace(R: int, Lmax: int, E: int, device) -> torch.Tensor | None:
    """The workspace oa_topq uses for rows too long for its shared-memory kernel (None when not needed)."""
    nbytes = _lib.load().oa_topq_workspace_bytes(R, Lmax, E)
    return torch.empty(nbytes, dtype=torch.uint8, device=device) if nbytes else None


def topq_variant(Lmax: int, E: int, C: int) -> int:
    """The top-q kernel rows of Lmax positions take: 0 pipelined (two key buffers), 1 one key buffer,
    2 the long-row kernels."""
    return int(_lib.load().oa_topq_variant(Lmax, E, C))


def topq(scores, st, quota, E, n_dev, n0_dev, exp_idx, status=None, workspace=None):
    R = scores.shape[0]
    B, _, Lmax = st["asg"].shape
    C = st["nb"].shape[-1]
    _need("exp_idx", exp_idx, torch.int32, (R, E))
    _need("quota", quota, torch.float32, (R, C))
    _rows("scores", scores, torch.bfloat16, R)
    _on(scores.device, ("quota", quota), ("n_dev", n_dev), ("n0_dev", n0_dev), ("exp_idx", exp_idx),
        ("status", status), ("workspace", workspace))
    _state_on(scores.device, st)
    rec = st.get("reclist")
    _lib.call("oa_topq", _ptr(scores), scores.stride(0), R, Lmax, C, _ptr(st["mem"]), _ptr(st["cstart"]),
              _ptr(st["clen"]), _ptr(st["asg"]), _ptr(rec), _ptr(st.get("reccnt")),
              0 if rec is None else rec.shape[-1], _ptr(quota), E, _ptr(n_dev), _ptr(n0_dev), _ptr(exp_idx),
              _ptr(status), _ptr(workspace), 0 if workspace is None else workspace.numel(), _stream(scores))


def residual(K, V, st, sel, exp_idx, nt, quota, kbar, vbar, logn, status=None):
    B, hkv, Lmax = _heads(K)
    C = st["nb"].shape[-1]
    R = B * G * hkv
    _need("kbar", kbar, torch.bfloat16, (R, C, D))
    _need("vbar", vbar, torch.bfloat16, (R, C, D))
    _need("logn", logn, torch.float32, (R, C))
    _need("K", K, torch.bfloat16, (B, hkv, Lmax, D))
    _need("V", V, torch.bfloat16, (B, hkv, Lmax, D))
    _need("sel", sel, torch.int32)
    _need("exp_idx", exp_idx, torch.int32)
    _need("nt", nt, torch.float32, (R, C))
    _need("quota", quota, torch.float32, (R, C))
    _on(K.device, ("V", V), ("sel", sel), ("exp_idx", exp_idx), ("nt", nt), ("quota", quota), ("kbar", kbar),
        ("vbar", vbar), ("logn", logn), ("status", status))
    _state_on(K.device, st)
    _lib.call("oa_residual", _ptr(K), _ptr(V), B, hkv, Lmax, C, _ptr(st["asg"]), _ptr(sel), sel.shape[1], _ptr(exp_idx),
              exp_idx.shape[1], _ptr(st["Sk"]), _ptr(st["Sv"]), _ptr(nt), _ptr(quota), _ptr(kbar), _ptr(vbar),
              _ptr(logn), _ptr(status), _stream(K))


def residual_flash(q, K, V, st, sel, exp_idx, nt, quota, out, kbar=None, vbar=None, logn=None, sm_scale=128 ** -0.5,
                   status=None, zdot=None):
    """Residual proxies + OpenAttention.flash in one kernel; out (B*32, D) bf16 or fp32.  zdot: the
    step's errorgate_waterfill zdot output (optional; saves the Sk read)."""
    B, hkv, Lmax = _heads(K)
    C = st["nb"].shape[-1]
    R = B * G * hkv
    if out.shape != (R, D) or out.stride(1) != 1 or out.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"out must be ({R}, 128) bf16 or fp32 with a contiguous last dim")
    code = _lib.OA_F32 if out.dtype == torch.float32 else _lib.OA_BF16
    _need("zdot", zdot, torch.float32, (R, C))
    _need("K", K, torch.bfloat16, (B, hkv, Lmax, D))
    _need("V", V, torch.bfloat16, (B, hkv, Lmax, D))
    _rows("q", q, torch.bfloat16, R, D)
    _need("sel", sel, torch.int32)
    _need("exp_idx", exp_idx, torch.int32)
    _need("nt", nt, torch.float32, (R, C))
    _need("quota", quota, torch.float32, (R, C))
    _on(K.device, ("q", q), ("V", V), ("sel", sel), ("exp_idx", exp_idx), ("nt", nt), ("quota", quota), ("out", out),
        ("kbar", kbar), ("vbar", vbar), ("logn", logn), ("status", status), ("zdot", zdot))
    _state_on(K.device, st)
    _lib.call("oa_residual_flash", _ptr(q), q.stride(0), _ptr(K), _ptr(V), B, hkv, Lmax, C, _ptr(st["asg"]), _ptr(sel),
              sel.shape[1], _ptr(exp_idx), exp_idx.shape[1], _ptr(st["Sk"]), _ptr(st["Sv"]), _ptr(nt), _ptr(quota),
              _ptr(zdot), _ptr(kbar), _ptr(vbar), _ptr(logn), _ptr(out), out.stride(0), code, float(sm_scale),
              _ptr(status), _stream(K))


def padded_len(Lmax: int) -> int:
    """Row length of the per-token score buffer: Lmax rounded up to 256 tokens."""
    return (Lmax + 255) // 256 * 256


def new_state(B: int, Lmax: int, C: int, device, rmax: int = 256, hkv: int = HKV) -> dict:
    """Per-layer index state: the layout contract of methods_eager.Ours / OursG2 (int8 codes, CSR
    member lists, generated-token lists of rmax entries per cluster; rmax = 0 leaves them out, the
    top-q stage then finds generated tokens by scanning the assignments).  hkv < 8: the state of a
    KV-head shard (hkv KV heads and their 4 hkv query heads per request)."""
    z = lambda *s, dt=torch.float32: torch.zeros(*s, device=device, dtype=dt)  # noqa: E731
    hq = G * hkv
    st = dict(codes=z(B, hkv, Lmax, RQ, dt=torch.int8), U=z(B, hkv, D, RQ), scale=z(B, hkv, RQ),
              W=z(B, hq, D, RC, dt=torch.bfloat16), colmean=z(B, hq, RC), cent=z(B, hq, C, RC),
              asg=z(B, hq, Lmax, dt=torch.int32), nb=z(B, hq, C), Sk=z(B, hq, C, D), Sk2=z(B, hq, C, D),
              Sv=z(B, hq, C, D), mem=z(B, hq, Lmax, dt=torch.int32), cstart=z(B, hq, C, dt=torch.int32),
              clen=z(B, hq, C, dt=torch.int32))
    if rmax > 0:
        st["reclist"] = z(B, hq, C, rmax, dt=torch.int32)
        st["reccnt"] = z(B, hq, C, dt=torch.int32)
    return st
