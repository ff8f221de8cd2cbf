"""Model geometry, budget table and per-step budget split of the deployed method.

Constants follow inference/methods_eager.py:77-84 (HQ, HKV, D, SC, DEPLOYED, CTX_LEN) and
run_openattention.sh:28-31 (the 5% row, absent from DEPLOYED in the reference).  The per-step
split (sink, local, top-k) is methods_eager.py:605-607.
"""
from __future__ import annotations

import math

HQ, HKV, D = 32, 8, 128
G = HQ // HKV
RQ, RC = 32, 16          # QGS code rank, QGC projection rank
ITERS, WIN, PQ = 4, 32, 64  # Lloyd iterations, RoPE window of the static metric, question rows
SC = D ** -0.5
CTX_LEN = 32768          # accounting context the budgets were sized for
RMAX = 256               # generated tokens one cluster's list holds (inference/ours_graph.py:40)

# rho -> (clusters C, expansion budget E)
DEPLOYED = {0.01: (64, 216), 0.03: (192, 679), 0.05: (192, 1335)}


def budget(rho: float):
    key = round(rho, 4)
    if key not in DEPLOYED:
        raise KeyError(f"no deployed (C, E) for rho={rho}; known: {sorted(DEPLOYED)}")
    return DEPLOYED[key]


def step_split(n: int, rho: float, C: int, E: int):
    """(ns, nl, k_top) at current length n: sink = local = max(1, int(1e-4 n)),
    k_top = max(1, int((rho - 2e-4 - E/32768 - 1.5 C/32768) n))."""
    ns = nl = max(1, int(0.0001 * n))
    heavy = rho - 0.0002 - E / CTX_LEN - 1.5 * C / CTX_LEN
    k_top = max(1, int(heavy * n))
    return ns, nl, k_top


def realised_read(n: int, rho: float, C: int, E: int) -> float:
    """Fraction of the cache read per step, proxies charged 1.5 rows (methods_eager.py:653)."""
    ns, nl, k_top = step_split(n, rho, C, E)
    return (ns + nl + k_top + E + 1.5 * C) / n


def llama31_inv_freq(theta: float = 500000.0, dim: int = D, factor: float = 8.0, low_freq_factor: float = 1.0,
                     high_freq_factor: float = 4.0, original_max_position: int = 8192):
    """Llama-3.1 RoPE inverse frequencies (the 'llama3' rope scaling rule), as fp32 values."""
    import torch
    f = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    low_wl = original_max_position / low_freq_factor
    high_wl = original_max_position / high_freq_factor
    wl = 2 * math.pi / f
    out = torch.where(wl > low_wl, f / factor, f)
    smooth = (original_max_position / wl - low_freq_factor) / (high_freq_factor - low_freq_factor)
    smoothed = (1 - smooth) * out / factor + smooth * out
    mid = ~(wl < high_wl) * ~(wl > low_wl)
    return torch.where(mid, smoothed, out)
