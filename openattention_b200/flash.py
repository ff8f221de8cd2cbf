"""OpenAttention.flash operators with the reference's call signatures, backed by the sm_100a kernels.

`decode_expand_attention` is the drop-in for triton_expand_decode.decode_expand_attention
(triton_expand_decode.py:139-165): proxies (kbar, vbar) per KV head.
`ours_flash` is the drop-in for methods_eager.ours_flash (inference/methods_eager.py:161-172):
proxies per query head, sm_scale fixed to 128**-0.5, nb=0 disables the proxy stream.

Both return a new tensor shaped like q (q's dtype unless `out_dtype` says otherwise) and run on the
current CUDA stream.  The Triton tuning hints of the reference (block_n, block_b, num_warps) are
accepted and ignored.
"""
from __future__ import annotations

import torch

from . import _lib

SC = 128 ** -0.5

_ws_cache: dict = {}


def _workspace(device: torch.device, rows: int, nbytes: int, stream: int) -> torch.Tensor | None:
    """Zero-filled scratch for the split-K mode, cached per (device, stream, row count) and grown on
    demand (its leading per-row ticket counters are only guaranteed zero for the row count it served).
    Keyed by stream: calls on one stream run in order and may share a workspace, while calls on two
    streams can overlap on the GPU and would race on one workspace's counters and partial sums.
    Callers that pass `workspace=` themselves must give overlapping calls different workspaces."""
    if nbytes == 0:
        return None
    key = (device.type, device.index, stream, rows)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def _check(name, t, dtype, ndim):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != ndim:
        raise RuntimeError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")


def _same_device(dev, **tensors):
    for name, t in tensors.items():
        if t is not None and (not isinstance(t, torch.Tensor) or t.device != dev):
            where = t.device if isinstance(t, torch.Tensor) else type(t).__name__
            raise RuntimeError(f"{name} must be a tensor on {dev} (q's device), got {where}")


def _flash(entry, q, k, v, sel_idx, exp_idx, kbar, vbar, log_n, sm_scale, nb, out_dtype, nsplit, out,
           workspace):
    _check("q", q, torch.bfloat16, 2)
    _check("k", k, torch.bfloat16, 3)
    _check("v", v, torch.bfloat16, 3)
    BQ, D = q.shape
    BH, K, Dk = k.shape
    if D != 128 or Dk != 128 or v.shape != k.shape or v.stride() != k.stride():
        raise RuntimeError(f"head_dim must be 128 and k/v must share shape and strides: q {tuple(q.shape)}, "
                           f"k {tuple(k.shape)}, v {tuple(v.shape)}")
    if q.stride(1) != 1 or k.stride(2) != 1:
        raise RuntimeError("the last dim of q, k and v must be contiguous")
    # every tensor on q's GPU: a host tensor's address would fault in the kernel (or, where the GPU
    # can reach host memory, be read silently), and another GPU's would be read across the link
    dev = q.device
    _same_device(dev, k=k, v=v, sel_idx=sel_idx, exp_idx=exp_idx, out=out, workspace=workspace)
    sel_idx = sel_idx.to(torch.int32).contiguous()
    exp_idx = exp_idx.to(torch.int32).contiguous()
    if sel_idx.dim() != 2 or exp_idx.dim() != 2 or sel_idx.shape[0] != BQ or exp_idx.shape[0] != BQ:
        raise RuntimeError("sel_idx and exp_idx must be (BQ, n) int32")
    NB = kbar.shape[1] if nb is None else int(nb)
    if NB > 0:
        _check("kbar", kbar, torch.bfloat16, 3)
        _check("vbar", vbar, torch.bfloat16, 3)
        _check("log_n", log_n, torch.float32, 2)
        _same_device(dev, kbar=kbar, vbar=vbar, log_n=log_n)
        if log_n.stride(1) != 1:
            raise RuntimeError("log_n must have a contiguous last dim")
        if kbar.stride() != vbar.stride() or kbar.shape != vbar.shape or kbar.stride(2) != 1:
            raise RuntimeError("kbar/vbar must share shape and strides with a contiguous last dim")
        if NB > kbar.shape[1] or log_n.shape[1] < NB:
            raise RuntimeError("nb exceeds the proxy tensors")
        want_rows = BQ if entry == "oa_flash_qhead_proxies" else BH
        if kbar.shape[0] != want_rows or log_n.shape[0] != BQ:
            raise RuntimeError(f"kbar/vbar need {want_rows} rows and log_n {BQ} rows")
    if out_dtype is None:
        out_dtype = q.dtype
    if out is None:
        out = torch.empty(BQ, D, dtype=out_dtype, device=q.device)
    elif out.dtype not in (torch.bfloat16, torch.float32) or out.shape != (BQ, D) or out.stride(1) != 1:
        raise RuntimeError(f"out must be ({BQ}, {D}) bf16 or fp32 with a contiguous last dim, got "
                           f"{tuple(out.shape)} {out.dtype}")
    if workspace is not None and workspace.dtype != torch.uint8:
        raise RuntimeError("workspace must be a uint8 tensor (its size is its byte count)")
    code = {torch.bfloat16: _lib.OA_BF16, torch.float32: _lib.OA_F32}[out.dtype]
    lib = _lib.load()
    need = lib.oa_flash_workspace_bytes(BQ, sel_idx.shape[1], exp_idx.shape[1], NB, int(nsplit))
    stream = torch.cuda.current_stream(q.device).cuda_stream
    if need and workspace is None:
        workspace = _workspace(q.device, BQ, need, stream)
    _lib.call(entry, _lib.ptr(q), q.stride(0), _lib.ptr(k), _lib.ptr(v), k.stride(0), k.stride(1),
              _lib.ptr(sel_idx), sel_idx.shape[1], _lib.ptr(exp_idx), exp_idx.shape[1],
              _lib.ptr(kbar) if NB else 0, _lib.ptr(vbar) if NB else 0,
              kbar.stride(0) if NB else 0, kbar.stride(1) if NB else 0,
              _lib.ptr(log_n) if NB else 0, log_n.stride(0) if NB else 0,
              _lib.ptr(out), out.stride(0), code, BQ, BH, K, NB, float(sm_scale), int(nsplit),
              _lib.ptr(workspace), 0 if workspace is None else workspace.numel(), stream)
    return out


def decode_expand_attention(q, k, v, sel_idx, exp_idx, kbar, vbar, log_n, sm_scale=None, block_n=64,
                            block_b=64, num_warps=4, *, out_dtype=None, nsplit=0, out=None, workspace=None):
    """q:(BQ,D) k,v:(BH,K,D) sel_idx:(BQ,N_SEL) exp_idx:(BQ,N_EXP) kbar,vbar:(BH,NB,D) log_n:(BQ,NB) -> (BQ,D).

    Index lists may be padded with -1; log_n is the natural log of each bin's count, -inf for bins
    that were expanded.  sm_scale defaults to D**-0.5."""
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    return _flash("oa_flash_kvhead_proxies", q, k, v, sel_idx, exp_idx, kbar, vbar, log_n, sm_scale, None,
                  out_dtype, nsplit, out, workspace)


def ours_flash(q, k, v, sel_idx, exp_idx, kbar, vbar, log_n, nb=None, *, out_dtype=None, nsplit=0, out=None,
               workspace=None):
    """q:(R,D) k,v:(B*HKV,Lmax,D) sel:(R,Ns) exp:(R,Ne) int32 (-1 = pad); kbar,vbar:(R,C,D); log_n:(R,C)."""
    return _flash("oa_flash_qhead_proxies", q, k, v, sel_idx, exp_idx, kbar, vbar, log_n, SC, nb, out_dtype,
                  nsplit, out, workspace)
