"""Seeded synthetic workloads with the reference benchmark's shapes (no dataset or checkpoint is used).

Per request b (generator seeded with seed + b):
  keys    64 per-KV-head centroids mu_c ~ N(0, 4); token t picks c ~ U{0..63}; k = mu_c + N(0, 0.25);
          then RoPE at position t with the Llama-3.1 inverse frequencies
  values  ~ N(0, 1);   decode queries ~ N(0, 1);   prefill queries (32, T, D) ~ N(0, 1), qlen = 40
  caches  bf16, shape (B, 8, Lmax, 128)
The static query metric (the reference ships it as a data asset) is replaced by a seeded PSD stand-in
M = A diag(s^2) A^T / 64 per (layer, query head) with A ~ N(0, 1) of shape (128, 64) and s linear
from 2 to 0.1.

Two generators: numpy (PCG64; bit-stable across machines, used for fixtures and CPU checks) and
torch (on the target device; used for the large benchmark caches).
"""
from __future__ import annotations

import numpy as np
import torch

from .geometry import D, HKV, HQ, llama31_inv_freq

NCENT = 64
QLEN = 40


def rope_rotate(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """x (..., T, D) fp32 rotated by RoPE at positions pos (T,)."""
    freqs = pos.float().unsqueeze(-1) * inv_freq.to(x.device).unsqueeze(0)
    emb = torch.cat([freqs, freqs], -1)
    h = x.shape[-1] // 2
    return x * emb.cos() + torch.cat([-x[..., h:], x[..., :h]], -1) * emb.sin()


# ------------------------------------------------------------------ numpy (bit-stable)
def kv_numpy(seed: int, n: int, Lmax: int | None = None):
    """One request: K, V as torch bf16 (8, Lmax, D) with the first n positions filled (rest zero)."""
    Lmax = n if Lmax is None else Lmax
    rng = np.random.default_rng(seed)
    mu = rng.standard_normal((HKV, NCENT, D), dtype=np.float32) * 2.0
    cid = rng.integers(0, NCENT, size=(HKV, n))
    k = mu[np.arange(HKV)[:, None], cid] + rng.standard_normal((HKV, n, D), dtype=np.float32) * 0.5
    v = rng.standard_normal((HKV, n, D), dtype=np.float32)
    kt = rope_rotate(torch.from_numpy(k), torch.arange(n), llama31_inv_freq())
    K = torch.zeros(HKV, Lmax, D, dtype=torch.bfloat16)
    V = torch.zeros(HKV, Lmax, D, dtype=torch.bfloat16)
    K[:, :n] = kt.to(torch.bfloat16)
    V[:, :n] = torch.from_numpy(v).to(torch.bfloat16)
    return K, V, mu


def new_token_numpy(seed: int, mu: np.ndarray, pos: int):
    """The decode-step key/value of one request at position pos: (8, D) bf16 each."""
    rng = np.random.default_rng(seed)
    cid = rng.integers(0, NCENT, size=(HKV,))
    k = mu[np.arange(HKV), cid] + rng.standard_normal((HKV, D), dtype=np.float32) * 0.5
    v = rng.standard_normal((HKV, D), dtype=np.float32)
    kt = rope_rotate(torch.from_numpy(k).unsqueeze(1), torch.tensor([pos]), llama31_inv_freq())[:, 0]
    return kt.to(torch.bfloat16), torch.from_numpy(v).to(torch.bfloat16)


def queries_numpy(seed: int, rows: int, shape_tail=(D,)):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((rows, *shape_tail), dtype=np.float32)).to(torch.bfloat16)


def static_metric_numpy(seed: int, layers: int = 1):
    """Stand-in for the shipped pre-RoPE query metric: (layers, 32, D, D) fp32 symmetric PSD."""
    rng = np.random.default_rng(seed)
    s = np.linspace(2.0, 0.1, 64, dtype=np.float32)
    A = rng.standard_normal((layers, HQ, D, 64), dtype=np.float32) * s
    M = np.einsum("lhdk,lhek->lhde", A, A) / 64.0
    return torch.from_numpy(M.astype(np.float32))


def static_metric_standin(seed: int = 7, layers: int = 1) -> dict:
    """The stand-in in the reference asset's unpacked form, for OursB200(a, ...) with
    a.static_metric = static_metric_standin(...) (synthetic workloads only)."""
    return {"M": static_metric_numpy(seed, layers), "inv_freq": llama31_inv_freq(), "attention_scaling": 1.0}


# ------------------------------------------------------------------ torch (device, large caches)
def kv_torch(seed: int, B: int, n: int, Lmax: int, device, dtype=torch.bfloat16):
    """B requests of the same law, generated on `device`: K, V (B, 8, Lmax, D) and centroids (B, 8, 64, D)."""
    g = torch.Generator(device=device)
    K = torch.zeros(B, HKV, Lmax, D, dtype=dtype, device=device)
    V = torch.zeros(B, HKV, Lmax, D, dtype=dtype, device=device)
    mus = torch.empty(B, HKV, NCENT, D, device=device)
    inv = llama31_inv_freq().to(device)
    pos = torch.arange(n, device=device)
    for b in range(B):
        g.manual_seed(seed + b)
        mu = torch.randn(HKV, NCENT, D, generator=g, device=device) * 2.0
        cid = torch.randint(0, NCENT, (HKV, n), generator=g, device=device)
        k = torch.gather(mu, 1, cid.unsqueeze(-1).expand(-1, -1, D))
        k += torch.randn(HKV, n, D, generator=g, device=device) * 0.5
        K[b, :, :n] = rope_rotate(k, pos, inv).to(dtype)
        V[b, :, :n] = torch.randn(HKV, n, D, generator=g, device=device).to(dtype)
        mus[b] = mu
    return K, V, mus


def new_tokens_torch(seed: int, mus: torch.Tensor, pos: int):
    """Decode-step K/V rows for B requests at position pos: (B, 8, D) each."""
    device = mus.device
    B = mus.shape[0]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    cid = torch.randint(0, NCENT, (B, HKV), generator=g, device=device)
    k = torch.gather(mus, 2, cid[..., None, None].expand(-1, -1, 1, D))[:, :, 0]
    k = k + torch.randn(B, HKV, D, generator=g, device=device) * 0.5
    v = torch.randn(B, HKV, D, generator=g, device=device)
    kt = rope_rotate(k.unsqueeze(2), torch.tensor([pos], device=device), llama31_inv_freq().to(device))[:, :, 0]
    return kt.to(torch.bfloat16), v.to(torch.bfloat16)
