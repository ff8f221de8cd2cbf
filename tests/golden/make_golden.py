"""Generate the golden fixtures by running the REFERENCE's own PyTorch code on CPU.

    python tests/golden/make_golden.py --reference /path/to/OpenAttention

Needs a checkout of the reference (it is not available on GPU machines; the fixtures are committed).
The reference's package __init__ pulls in ray / matplotlib / seaborn, which are stubbed here; its
eager method class writes the unpacked static metric to OA_STATIC_M, which points at a temporary
file holding the case's metric: this repository's seeded stand-in, or (decode_real_l0) layer 0 of the
reference's own asset.  Nothing of the reference is copied: its
functions are executed and their outputs saved.

Fixtures:
  flash_qhead.npz   methods_eager.selftest's fp32 reference formula (inference/methods_eager.py:708-719)
                    evaluated on cases.flash_inputs("flash_qhead")
  flash_kvhead.npz  bench_flash_latency.make_paths(...)["ours_torch"] (bench_flash_latency.py:126-133),
                    the reference's unfused PyTorch path with per-KV-head proxies
  metric_l0.npz     layer 0 of the reference's shipped static query metric
                    (assets/llama-3.1-8b-instruct.query_metric.triu.pt, Apache-2.0), in its packed form
  decode_*.npz      methods_eager.Ours build + decode steps (inference/methods_eager.py:505-654) with the
                    attention stage of OursUnfused (:671-685): post-build state, and per step the
                    selected / expanded indices, ErrorGate scores, quotas, proxies and outputs
"""
from __future__ import annotations

import argparse
import inspect
import os
import sys
import tempfile
import textwrap
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)
import cases  # noqa: E402
from openattention_b200.geometry import D, G, HKV, HQ, llama31_inv_freq  # noqa: E402


def bits(t):
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def npc(t):
    """A numpy COPY (decode steps later update the method's state tensors in place)."""
    return t.detach().numpy().copy()


def import_reference(ref_root, metric_path):
    for m in ["ray", "ray.tune", "matplotlib", "matplotlib.pyplot", "seaborn"]:
        sys.modules.setdefault(m, types.ModuleType(m))
    sys.modules["ray"].tune = sys.modules["ray.tune"]
    os.environ["OA_STATIC_M"] = metric_path
    sys.path.insert(0, os.path.join(ref_root, "inference"))
    sys.path.insert(0, ref_root)
    import methods_eager as bl
    import bench_flash_latency as bfl
    return bl, bfl


def golden_flash_qhead(bl):
    x = cases.flash_inputs("flash_qhead")
    src = textwrap.dedent(inspect.getsource(bl.selftest)).splitlines()
    i0 = next(i for i, s in enumerate(src) if s.strip().startswith("off = "))
    i1 = next(i for i, s in enumerate(src) if s.strip().startswith("ref = "))
    body = textwrap.dedent("\n".join(src[i0:i1 + 1]))
    ns = dict(torch=torch, q=x["q"], k=x["k"], v=x["v"], sel=x["sel"].long(), ex=x["exp"].long(), kb=x["kbar"],
              vb=x["vbar"], ln=x["log_n"], R=x["q"].shape[0], Lmax=x["k"].shape[1], G=bl.G, D=bl.D, SC=bl.SC,
              NEG=bl.NEG, dev="cpu")
    exec(body, ns)
    return dict(out=npc(ns["ref"].double()), source_lines=np.array([i0, i1]))


def golden_flash_kvhead(bfl):
    x = cases.flash_inputs("flash_kvhead")
    q, k, v = x["q"], x["k"], x["v"]
    BQ, BH = q.shape[0], k.shape[0]
    allidx = torch.cat([x["sel"], x["exp"]], 1).int().contiguous()
    t = dict(B=BH // HKV, g=BQ // BH, BH=BH, BQ=BQ, sc=D ** -0.5, q=q, k=k, v=v, sel_base=allidx, sel_ours=allidx,
             sel_top=allidx, samp=allidx, kbar=x["kbar"], vbar=x["vbar"], ell=x["log_n"], sel_s=x["sel"],
             exp_x=x["exp"], n_base=allidx.shape[1], n_ours=allidx.shape[1], n_exp=x["exp"].shape[1],
             n_half=allidx.shape[1], K=k.shape[1], D=D, dt=torch.bfloat16, dev="cpu")
    out = bfl.make_paths(t)["ours_torch"]()
    return dict(out=npc(out.view(BQ, D).float()))


def golden_metric_l0(ref_root):
    """Layer 0 of the reference's shipped static-metric asset, kept in its packed (upper-triangle) form."""
    d = torch.load(os.path.join(ref_root, "assets", "llama-3.1-8b-instruct.query_metric.triu.pt"), map_location="cpu",
                   weights_only=False)
    return dict(M_triu=npc(d["M_triu"][:1]), dim=np.array(d["dim"]), inv_freq=npc(d["inv_freq"]),
                attention_scaling=np.array(float(d.get("attention_scaling", 1.0))),
                source=np.array(f"{d.get('source')} ({d.get('n_requests')} requests), layer 0 of 32"))


def golden_decode(bl, name, metric_path):
    x = cases.decode_inputs(name)
    torch.save({"M": x["M"], "inv_freq": x["inv_freq"], "attention_scaling": 1.0}, metric_path)
    bl.NL = 1
    bl.DEPLOYED[0.05] = (192, 1335)
    B, n0, Lmax = x["B"], x["n0"], x["Lmax"]
    bl.C.K = [x["K"].clone()]
    bl.C.V = [x["V"].clone()]
    bl.C.qlen = [cases.QLEN] * B
    bl.C.timing = False

    class Rec(bl.OursUnfused):
        def attend(self, l, q, sel, exp_idx, kbar_r, vbar_r, logn):
            self.rec = dict(sel=sel.clone(), exp_idx=exp_idx.clone(), kbar_r=kbar_r.clone(), vbar_r=vbar_r.clone(),
                            logn=logn.clone())
            return super().attend(l, q, sel, exp_idx, kbar_r, vbar_r, logn)

    m = Rec(types.SimpleNamespace(rho=x["rho"]), B, Lmax, "cpu")
    hq = bl.Ours.hier_quota

    def spy(score, cap, live, E):
        qb = hq(score, cap, live, E)
        m.rec_q = dict(score=score.clone(), nt=cap.clone(), quota=qb.clone())
        return qb
    m.hier_quota = spy
    for b in range(B):
        m.build(0, b, x["qpre"][b], n0)
    out = dict(U=npc(m.U[0]), scale=npc(m.scale[0]), codes=npc(m.codes[0].float()).astype(np.int8),
               W=bits(m.W[0]), colmean=npc(m.colmean[0]), cent=npc(m.cent[0]),
               asg=npc(m.asg[0][..., :n0]).astype(np.uint8 if m.C <= 255 else np.int16),
               nb=npc(m.nb[0]), Sk_sum=npc(m.Sk[0].double().sum(-1)), Sk2_sum=npc(m.Sk2[0].double().sum(-1)),
               Sv_sum=npc(m.Sv[0].double().sum(-1)), Sk_rows=npc(m.Sk[0][:, ::16, ::4]), C=np.array(m.C),
               E=np.array(m.E))
    for s in range(x["steps"]):
        n = n0 + s + 1
        bl.C.K[0][:, :, n - 1] = x["new_k"][s]
        bl.C.V[0][:, :, n - 1] = x["new_v"][s]
        o = m.decode(0, x["qdec"][s], n)
        r, rq = m.rec, m.rec_q
        out[f"s{s}_sel"] = npc(r["sel"]).astype(np.int32)
        out[f"s{s}_exp"] = npc(r["exp_idx"]).astype(np.int16 if n < 32768 else np.int32)
        out[f"s{s}_score"] = npc(rq["score"])
        out[f"s{s}_nt"] = npc(rq["nt"])
        out[f"s{s}_quota"] = npc(rq["quota"]).astype(np.int16)
        out[f"s{s}_kbar_sum"] = npc(r["kbar_r"].double().sum(-1))
        out[f"s{s}_vbar_sum"] = npc(r["vbar_r"].double().sum(-1))
        out[f"s{s}_kbar_rows"] = bits(r["kbar_r"][::16, ::4])
        out[f"s{s}_vbar_rows"] = bits(r["vbar_r"][::16, ::4])
        out[f"s{s}_logn"] = npc(r["logn"])
        out[f"s{s}_out"] = npc(o.view(B * HQ, D).float())
        out[f"s{s}_asg_new"] = npc(m.asg[0][..., n - 1]).astype(np.int16)
        out[f"s{s}_codes_new"] = npc(m.codes[0][:, :, n - 1].float()).astype(np.int8)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OA_REFERENCE"),
                    help="checkout of the reference (or set OA_REFERENCE)")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    if not a.reference:
        ap.error("--reference (or OA_REFERENCE) is required")
    torch.set_num_threads(os.cpu_count() or 1)
    tmp = tempfile.mkdtemp()
    metric_path = os.path.join(tmp, "static_metric.pt")
    torch.save({"M": torch.zeros(1, HQ, D, D), "inv_freq": llama31_inv_freq(), "attention_scaling": 1.0},
               metric_path)
    bl, bfl = import_reference(a.reference, metric_path)
    # the metric fixture first: the decode case that uses the real asset reads it through cases.py
    jobs = {"metric_l0": lambda: golden_metric_l0(a.reference), "flash_qhead": lambda: golden_flash_qhead(bl),
            "flash_kvhead": lambda: golden_flash_kvhead(bfl)}
    for name in cases.DECODE_CASES:
        jobs[name] = (lambda nm: (lambda: golden_decode(bl, nm, metric_path)))(name)
    for name, fn in jobs.items():
        if a.only and name not in a.only.split(","):
            continue
        res = fn()
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
