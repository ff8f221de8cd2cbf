"""Seeded input definitions shared by the golden-fixture generator and the tests.

Inputs are regenerated from these seeds (numpy PCG64, bit-stable across machines); the fixtures
(`*.npz` beside this file) hold only the reference's outputs on them.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from openattention_b200 import synth
from openattention_b200.geometry import D, HKV, HQ

FLASH_CASES = {
    # modelled on methods_eager.selftest (inference/methods_eager.py:693-728): per-query-head proxies,
    # 7 padded exp slots, 5 bins with log n = -inf
    "flash_qhead": dict(kind="qhead", B=2, Lmax=1024, C=64, Ns=14, Ne=216, pads=7, neg=5, seed=11),
    # modelled on bench_flash_latency.build (bench_flash_latency.py:49-73): per-KV-head proxies, a
    # constant ell = log((K - n_ours) / C), 1% read at K = 4096
    "flash_kvhead": dict(kind="kvhead", B=2, Lmax=4096, C=64, Ns=15, Ne=216, pads=0, neg=0, seed=12),
}

DECODE_CASES = {
    # config 0 of the benchmark: batch 1, one layer, 4096-token context, 1% read (C=64, E=216)
    "decode_c0": dict(B=1, n0=4096, steps=3, rho=0.01, seed=100, mseed=7),
    # two requests at 3% (C=192, E=679), 1024-token context
    "decode_b2_r3": dict(B=2, n0=1024, steps=2, rho=0.03, seed=200, mseed=8),
    # one request at 1% with the REFERENCE's static query metric (layer 0 of its shipped asset, kept in
    # metric_l0.npz in the asset's packed form) instead of the seeded stand-in
    "decode_real_l0": dict(B=1, n0=2048, steps=2, rho=0.01, seed=300, mseed="asset"),
}
METRIC_FIXTURE = "metric_l0.npz"
QLEN = 40


def flash_inputs(name):
    c = FLASH_CASES[name]
    rng = np.random.default_rng(c["seed"])
    B, Lmax, Cn, Ns, Ne = c["B"], c["Lmax"], c["C"], c["Ns"], c["Ne"]
    R, BH = B * HQ, B * HKV

    def bf(*shape):
        return torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(torch.bfloat16)

    k, v, q = bf(BH, Lmax, D), bf(BH, Lmax, D), bf(R, D)
    perm = np.stack([rng.permutation(Lmax) for _ in range(R)]).astype(np.int32)
    sel = torch.from_numpy(perm[:, :Ns].copy())
    ex = torch.from_numpy(perm[:, Ns:Ns + Ne].copy())
    if c["pads"]:
        ex[:, -c["pads"]:] = -1
    prow = R if c["kind"] == "qhead" else BH
    kb, vb = bf(prow, Cn, D), bf(prow, Cn, D)
    if c["kind"] == "qhead":
        ln = torch.from_numpy(rng.random((R, Cn), dtype=np.float32) * 5)
    else:
        ln = torch.full((R, Cn), math.log((Lmax - (Ns + Ne)) / Cn), dtype=torch.float32)
    if c["neg"]:
        ln[:, :c["neg"]] = float("-inf")
    return dict(q=q, k=k, v=v, sel=sel, exp=ex, kbar=kb, vbar=vb, log_n=ln, kind=c["kind"])


def decode_inputs(name):
    """Caches with the first n0 positions filled, per-request prefill queries, per-step new tokens
    and decode queries, and the static-metric stand-in."""
    c = DECODE_CASES[name]
    B, n0, steps, seed = c["B"], c["n0"], c["steps"], c["seed"]
    Lmax = n0 + steps + 8
    K = torch.zeros(B, HKV, Lmax, D, dtype=torch.bfloat16)
    V = torch.zeros(B, HKV, Lmax, D, dtype=torch.bfloat16)
    mus, qpre = [], []
    for b in range(B):
        Kb, Vb, mu = synth.kv_numpy(seed + b, n0, Lmax)
        K[b], V[b] = Kb, Vb
        mus.append(mu)
        qpre.append(synth.queries_numpy(seed + 1000 + b, HQ * n0).view(1, HQ, n0, D))
    new_k, new_v, qdec = [], [], []
    for s in range(steps):
        pos = n0 + s
        ks, vs = zip(*[synth.new_token_numpy(seed + 10000 + 100 * s + b, mus[b], pos) for b in range(B)])
        new_k.append(torch.stack(ks))
        new_v.append(torch.stack(vs))
        qdec.append(synth.queries_numpy(seed + 20000 + s, B * HQ).view(B, HQ, 1, D))
    if c["mseed"] == "asset":
        M, inv_freq = asset_metric()
    else:
        M, inv_freq = synth.static_metric_numpy(c["mseed"], layers=1), synth.llama31_inv_freq()
    return dict(B=B, n0=n0, steps=steps, Lmax=Lmax, rho=c["rho"], K=K, V=V, qpre=qpre, new_k=new_k, new_v=new_v,
                qdec=qdec, M=M, inv_freq=inv_freq)


def asset_packed():
    """Layer 0 of the reference's static-metric asset in its shipped packed form (a dict as the asset's)."""
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), METRIC_FIXTURE))
    return {"M_triu": torch.from_numpy(z["M_triu"]), "dim": int(z["dim"]), "inv_freq": torch.from_numpy(z["inv_freq"]),
            "attention_scaling": float(z["attention_scaling"])}


def asset_metric():
    """(M (1, 32, 128, 128), inv_freq) of asset_packed(), unpacked by this package's loader."""
    from openattention_b200.method import load_static_metric
    import types
    M, inv, _ = load_static_metric(types.SimpleNamespace(static_metric=asset_packed()), 1)
    return M, inv
