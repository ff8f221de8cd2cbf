#!/usr/bin/env python3
"""Decode-attention-stage benchmark of the OpenAttention deployed path on B200 (BASELINE config c2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B] [--ctx N]
    python bench.py --sweep [--sweep-b 1,32] [--sweep-n 8192,131072] [--sweep-rho 0.05]   (latency sweep)

Workload per GPU: B=32 requests, 32K-token bf16 KV caches (seeded synthetic, see
openattention_b200/synth.py), 1% read (C=64, E=216), ONE layer's decode step: index update + QGS
scan + top-k, ErrorGate + water-filling, within-cluster top-q, residual proxies, OpenAttention.flash.
Each step appends a token (n grows by one per step).  The step is one CUDA graph replay (the
reference's deployed graph mode); the timed region replays K steps, inputs resident in HBM
(`value`), and again with per-step host->device input copies and a device->host output copy through
the same public API (`e2e`): two step graphs with their own input/output buffers alternate, and a
copy stream moves step s+1's inputs in and step s's output out while the GPU computes.  Inputs (int8 codes 268 MB + bf16 K/V 4.3 GB per GPU) exceed the
126 MB L2, so no flush is needed between iterations.

Multi-GPU (torchrun): requests are sharded, every rank runs its own B=32 (weak scaling), no
collective on the data path; the step time is the max over ranks and `value` = that time / N
(µs per bs32 layer-step for the whole job).

--impl reference: the reference's CPU implementation of the path (this repository's C restatement
of it, oracle/oa_oracle.c -- the reference itself is Python and cannot run without a checkout), on
all host cores, on a bounded sample of the same workload, scaled to the same unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import types

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn-stage µs/step @32K ctx, bs32, 1% read; % HBM roofline; ms/token e2e"
UNIT = "µs/step"
B_PER_GPU, N_CTX, RHO = 32, 32768, 0.01
VALUE_SLOTS = 64  # step graphs the `value` loop takes in turn (their inputs are staged before timing)
SCAN_BYTES_PER_TOKEN = 32  # int8 codes per token per KV head (the scan's algorithmic bytes)
LAUNCHES_PER_STEP = 7      # append_kv, index_update, qgs_scan, qgs_select, errorgate_waterfill, topq, residual_flash
CLOCK_SOAK_S = 0.3         # step replays before warm-up while the clock sampler runs (state reset after)
CLOCK_SOAK_MAX_STEPS = 1024
CLOCK_SOAK_RUN = 128       # the soak resets the state every this many steps, so it needs only these extra
                           # positions in the KV buffer (the workload's own length decides the kernels)


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profiles(kernel):
    """DRAM bytes (read + write) per full-size launch of `kernel` from the committed ncu summary
    profiles/roofline_traffic.json (None when that kernel has not been captured)."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(p):
        try:
            v = json.load(open(p)).get(kernel)
            return v.get("bytes_per_launch") if isinstance(v, dict) else v
        except (ValueError, OSError):
            return None
    return None


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, max clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        idx = dev.index or 0
        self.index = ids[idx] if idx < len(ids) and ids[idx].isdigit() else str(idx)
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t_end = time.time() + 5.0
            while not self.lines and time.time() < t_end:  # sampling has started before the timed work
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0=None, t1=None, window=""):
        """Median SM clock, max clock and throttle reasons over the samples taken in [t0, t1] (host time)."""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines[1:]:  # the first sample predates the load
            if (t0 is not None and ts < t0) or (t1 is not None and ts > t1):
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9 or f[0] != self.index:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm)}
        if window:
            out["window"] = window
        return out


# ------------------------------------------------------------------ our arm
def build_workload(dev, seed, steps_total, extra_positions=0, B=None, kv_heads=(0, 8)):
    """B requests (default B_PER_GPU) of the synthetic law; with kv_heads = (k0, kc) this rank keeps only
    those KV heads of every request (and their query heads), the KV-head shard of a small batch."""
    from openattention_b200 import method as Mth
    from openattention_b200 import synth
    from openattention_b200.geometry import G, HQ
    B = B_PER_GPU if B is None else B
    n0 = N_CTX
    k0, kc = kv_heads
    Lmax = n0 + steps_total + extra_positions + 16
    K, V, mus = synth.kv_torch(seed, B, n0, Lmax, dev)
    if kc != 8:
        K, V = K[:, k0:k0 + kc].contiguous(), V[:, k0:k0 + kc].contiguous()
    Mth.C.K, Mth.C.V, Mth.C.qlen = [K], [V], [40] * B
    m = Mth.OursB200(types.SimpleNamespace(rho=RHO, static_metric=synth.static_metric_standin(7, 1)), B, Lmax, dev,
                     layers=1, kv_heads=(k0, kc))
    g = torch.Generator(device=dev)
    qpre = torch.empty(1, HQ, n0, 128, dtype=torch.bfloat16, device=dev)
    for b in range(B):
        g.manual_seed(seed + 5000 + b)
        qpre[:, :, n0 - 64:] = torch.randn(1, HQ, 64, 128, generator=g, device=dev).to(torch.bfloat16)
        m.build(0, b, qpre, n0)
    del qpre
    # per-step inputs: decode queries and the new K/V rows
    g.manual_seed(seed + 9000)
    qs = torch.randn(steps_total, B, HQ, 1, 128, generator=g, device=dev).to(torch.bfloat16)
    qs = qs[:, :, G * k0:G * (k0 + kc)].contiguous()
    nks, nvs = [], []
    for s in range(steps_total):
        nk, nv = synth.new_tokens_torch(seed + 20000 + s, mus, n0 + s)  # all 8 KV heads, then this rank's
        nks.append(nk[:, k0:k0 + kc])
        nvs.append(nv[:, k0:k0 + kc])
    torch.cuda.synchronize()
    return m, Mth, qs, torch.stack(nks), torch.stack(nvs), n0, Lmax


class GraphStep:
    """One decode step as a CUDA graph: write the new token at kv_idx, n_dev and kv_idx advance, decode.
    With copy_out the graph also copies the attention output into a buffer of its own (so a host
    read of one step can overlap the next step, which rewrites the method's output buffer)."""

    def __init__(self, m, Mth, n0, dev, copy_out=False, fresh=True):
        from openattention_b200.geometry import HQ
        B = m.B
        self.m, self.Mth = m, Mth
        self.q_in = torch.zeros(B, m.hq, 1, 128, dtype=torch.bfloat16, device=dev)
        self.k_in = torch.zeros(B, m.hkv, 128, dtype=torch.bfloat16, device=dev)
        self.v_in = torch.zeros(B, m.hkv, 128, dtype=torch.bfloat16, device=dev)
        # position counters: new ones for a new workload (fresh), else the ones of the graphs already
        # captured for this workload, which all advance the same counters
        if fresh or getattr(Mth.C, "kv_idx", None) is None or Mth.C.n_dev is None:
            Mth.C.n_dev = torch.full((1,), n0, dtype=torch.int32, device=dev)      # n before the step
            Mth.C.kv_idx = torch.full((1,), n0 - 1, dtype=torch.int64, device=dev)
            Mth.C.n0_dev = torch.full((1,), n0, dtype=torch.int32, device=dev)
        self.n_host = n0 + 1  # ns/nl/k_top are constant over the benchmark window
        self.copy_out = copy_out
        self.out_buf = torch.empty(B, m.hq, 1, 128, dtype=torch.bfloat16, device=dev) if copy_out else None
        snap = {k: v.clone() for k, v in m.st[0].items()}
        n_snap, kv_snap = Mth.C.n_dev.clone(), Mth.C.kv_idx.clone()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside capture
                self._body()
        torch.cuda.current_stream(dev).wait_stream(s)
        for k, v in snap.items():
            m.st[0][k].copy_(v)
        Mth.C.n_dev.copy_(n_snap)
        Mth.C.kv_idx.copy_(kv_snap)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()
        torch.cuda.synchronize()

    def _body(self):
        from openattention_b200 import selection as S
        C = self.Mth.C
        # the new token's K/V rows at position n, then n_dev = n + 1 and kv_idx = n (one launch)
        S.append_kv(C.K[0], C.V[0], self.k_in, self.v_in, C.n_dev, offset=0, advance=True, kv_idx=C.kv_idx)
        res = self.m.decode(0, self.q_in, self.n_host)
        if self.copy_out:
            self.out_buf.copy_(res)
            return self.out_buf
        return res

    def replay(self):
        self.graph.replay()


class StageGraphStep(GraphStep):
    """The decode step with a timing event between its kernels, captured as a graph of its own
    (external event-record nodes): each kernel's duration inside the step, with the L2 contents
    the kernels before it leave, as opposed to stage_profile's launches timed alone.  The body is
    the method's fused decode (OursB200.select + residual_flash) written out stage by stage."""

    NAMES = ("index_update_kernel", "qgs_scan_kernel", "qgs_select_kernel", "errorgate_waterfill_kernel",
             "topq_pipe_kernel", "proxy_flash_kernel")

    def __init__(self, m, Mth, n0, dev):
        self.ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(self.NAMES) + 1)]
        super().__init__(m, Mth, n0, dev, copy_out=False, fresh=False)

    def _body(self):
        from openattention_b200 import selection as S
        from openattention_b200.geometry import D, HQ, step_split
        C, m = self.Mth.C, self.m
        st, K, V = m.st[0], C.K[0], C.V[0]
        S.append_kv(K, V, self.k_in, self.v_in, C.n_dev, offset=0, advance=True, kv_idx=C.kv_idx)
        ns, nl, k_top = step_split(self.n_host, m.a.rho, m.C, m.E)
        qr = self.q_in.reshape(m.R, D)
        sel = m._sel_buf(ns + nl + k_top)
        ev = self.ev
        ev[0].record()
        S.index_update(K, V, st, C.n_dev, q=qr, zq=m.zq)
        ev[1].record()
        S.qgs_scan(st["codes"], m.zq, C.n_dev, ns, nl, m.scores, m.tmax, m.status)
        ev[2].record()
        S.qgs_select(m.scores, m.tmax, m.Lmax, C.n_dev, ns, nl, k_top, sel)
        ev[3].record()
        S.errorgate_waterfill(qr, K, st, sel, m.E, m.score, m.nt, m.quota, m.status, zdot=m.zdot)
        ev[4].record()
        S.topq(m.scores, st, m.quota, m.E, C.n_dev, C.n0_dev, m.exp_idx, m.status, workspace=m.topq_ws)
        ev[5].record()
        S.residual_flash(qr, K, V, st, sel, m.exp_idx, m.nt, m.quota, m.out, status=m.status, zdot=m.zdot)
        ev[6].record()
        return m.out


def in_graph_profile(m, Mth, n0, dev, qs, nks, nvs, reps):
    """Per-kernel milliseconds inside the step graph (mean over `reps` replays, after 3 untimed).  Each
    replay decodes the next of the workload's steps (its own query and new token), as the timed steps do:
    one token appended over and over would pile up in one cluster and change the quotas."""
    sg = StageGraphStep(m, Mth, n0, dev)
    tot = [0.0] * len(sg.NAMES)
    for i in range(reps + 3):
        sg.q_in.copy_(qs[i % qs.shape[0]])
        sg.k_in.copy_(nks[i % nks.shape[0]])
        sg.v_in.copy_(nvs[i % nvs.shape[0]])
        sg.replay()
        torch.cuda.synchronize()
        if i >= 3:
            for k in range(len(sg.NAMES)):
                tot[k] += sg.ev[k].elapsed_time(sg.ev[k + 1])
    del sg
    return {nm: t / reps for nm, t in zip(StageGraphStep.NAMES, tot)}


def stage_profile(m, Mth, gs, iters):
    """Each kernel of the step timed alone on the current stream: CUDA events around single launches,
    L2 flushed (a 256 MB write) before each and the GPU kept busy while the host enqueues the launch
    (so host launch overhead is not timed), mean over `iters`; with its algorithmic bytes per launch
    (unique bytes the stage must move: inputs read once, outputs written once, no on-chip intermediates)."""
    from openattention_b200 import selection as S
    from openattention_b200.geometry import D, HKV, HQ, step_split
    st, B, C, E = m.st[0], m.B, m.C, m.E
    R, Rkv = m.R, B * m.hkv
    n = int(Mth.C.n_dev.item())
    ns, nl, k_top = step_split(gs.n_host, RHO, C, E)
    NS = ns + nl + k_top
    sel = m._sel_buf(NS)
    K, V = Mth.C.K[0], Mth.C.V[0]
    qr = gs.q_in.reshape(R, D)
    n_dev, n0_dev = Mth.C.n_dev, Mth.C.n0_dev
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=K.device)
    scores_snap = m.scores.clone()

    def timed(fn, prep=None):
        for _ in range(3):
            if prep:
                prep()
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            if prep:
                prep()
            flush.zero_()
            # a bounded spin (about 0.2 ms) keeps the GPU busy while the host enqueues the launch, so
            # the events time the kernel and not the host's launch overhead
            torch.cuda._sleep(400_000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / iters

    upd_keys = [k for k in ("codes", "asg", "nb", "Sk", "Sk2", "Sv", "reclist", "reccnt") if k in st]
    upd_snap = {k: st[k].clone() for k in upd_keys}

    def upd_restore():  # the index update appends the step's token: put the state back before each launch
        for k in upd_keys:
            st[k].copy_(upd_snap[k])

    ms = {
        "index_update_kernel": timed(lambda: S.index_update(K, V, st, n_dev, q=qr, zq=m.zq), prep=upd_restore),
        "qgs_scan_kernel": timed(lambda: S.qgs_scan(st["codes"], m.zq, n_dev, ns, nl, m.scores, m.tmax, m.status)),
        "qgs_select_kernel": timed(lambda: S.qgs_select(m.scores, m.tmax, m.Lmax, n_dev, ns, nl, k_top, sel),
                                   prep=lambda: m.scores.copy_(scores_snap)),
        "errorgate_waterfill_kernel": timed(lambda: S.errorgate_waterfill(qr, K, st, sel, E, m.score, m.nt, m.quota,
                                                                          m.status, zdot=m.zdot)),
        "topq_pipe_kernel": timed(lambda: S.topq(m.scores, st, m.quota, E, n_dev, n0_dev, m.exp_idx, m.status,
                                                     workspace=m.topq_ws)),
        "proxy_flash_kernel": timed(lambda: S.residual_flash(qr, K, V, st, sel, m.exp_idx, m.nt, m.quota, m.out,
                                                                status=m.status, zdot=m.zdot)),
    }
    # data-dependent byte counts of this step
    quota = m.quota.view(B, m.hq, C)
    members = int((st["clen"].float() * (quota > 0)).sum().item())
    reads = int((m.exp_idx >= 0).sum().item()) + R * NS
    # GQA-unique rows: the union of the read lists of a KV head's query heads (they share little)
    G_ = m.hq // m.hkv
    lists = torch.cat([sel, m.exp_idx], 1).view(B * m.hkv, G_ * (NS + E)).long()
    lists = torch.where(lists >= 0, lists, torch.full_like(lists, -1)).sort(1).values
    uniq = (lists[:, 1:] != lists[:, :-1]) & (lists[:, 1:] >= 0)
    unique_reads = int(uniq.sum().item() + (lists[:, 0] >= 0).sum().item())
    nt_tiles = (n + 31) // 32
    alg = {
        "index_update_kernel": R * (D * 16 * 2 + C * 16 * 4 + 3 * D * 4 * 2 + D * 2) + Rkv * (D * 32 * 4 + 2 * D * 2),
        "qgs_scan_kernel": Rkv * n * 32,
        "qgs_select_kernel": R * (nt_tiles * 4 + NS * 4),
        "errorgate_waterfill_kernel": R * (2 * C * D * 4 + C * 4 + NS * (D * 2 + 4) + D * 2 + 4 * C * 4),
        "topq_pipe_kernel": members * 6 + R * (2 * C * 4 + E * 4),
        "proxy_flash_kernel": reads * 2 * D * 2 + R * (C * D * 4 + 3 * C * 4 + (NS + E) * 4 + 2 * D * 2),
    }
    # the whole step's algorithmic bytes: codes, the three fp32 sum arrays once, the read rows, the small
    # per-row arrays, the index-update operands and the chosen clusters' member lists
    step_alg = (Rkv * n * 32 + 3 * R * C * D * 4 + reads * 2 * D * 2 + R * C * 4 + R * (NS + E) * 4 + 2 * R * D * 2
                + R * (D * 16 * 2 + C * 16 * 4) + Rkv * D * 32 * 4 + members * 6)
    unique = {"proxy_flash_kernel": alg["proxy_flash_kernel"] - (reads - unique_reads) * 2 * D * 2}
    return ms, alg, step_alg, n, unique


def cpu_baseline_sample(m, Mth, qs, nks, nvs, budget_s=12.0):
    """The oracle (C restatement of the reference's per-step algorithm) on the host cores: decode
    steps of ONE request (request 0's state copied from the GPU), repeated until ~budget_s of CPU
    work; reported per bs32 layer-step (x32)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = use_all_host_threads(O)
    st_gpu = m.st[0]
    st = {}
    for k, v in st_gpu.items():
        t = v[0:1].detach()
        st[k] = O.bits(t).copy() if t.dtype == torch.bfloat16 else t.cpu().numpy().copy()
    K = O.bits(Mth.C.K[0][0:1]).copy()
    V = O.bits(Mth.C.V[0][0:1]).copy()
    n = int(Mth.C.n_dev.item())
    C, E = m.C, m.E
    times, steps = [], 0
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end and steps < 64:
        s = steps % qs.shape[0]
        n += 1
        if n > K.shape[2]:
            break
        K[:, :, n - 1] = O.bits(nks[s][0:1])
        V[:, :, n - 1] = O.bits(nvs[s][0:1])
        q = O.bits(qs[s][0:1].reshape(32, 128))
        t0 = time.perf_counter()
        O.decode_step(st, q, K, V, n, RHO, C, E)
        times.append(time.perf_counter() - t0)
        steps += 1
    per_req = statistics.median(times)
    return {"value": per_req * 1e6 * m.B, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} decode steps of 1 request (n~{N_CTX}, rho={RHO:g}), median x {m.B} requests; "
                      f"oracle/oa_oracle.c with OpenMP on {threads} threads"}


def run_ours(a):
    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = dist
    steps_total = a.warmup + 2 * a.steps + 8
    from openattention_b200 import shard
    if a.global_batch:
        # a fixed batch split over the ranks (strong scaling): whole requests while there are at least as
        # many as ranks, else every rank keeps all requests and a share of the 8 KV heads (shard.plan)
        plan = shard.plan(a.global_batch, world, rank)
        seed = 17 if plan.kind == "kvhead" else shard.request_seed(17, plan.req_start)
        m, Mth, qs, nks, nvs, n0, Lmax = build_workload(dev, seed=seed, steps_total=steps_total,
                                                        extra_positions=CLOCK_SOAK_RUN, B=plan.req_count,
                                                        kv_heads=(plan.kv_start, plan.kv_count))
    else:
        # every rank runs its own B=32 requests (request sharding, weak scaling)
        plan = None
        m, Mth, qs, nks, nvs, n0, Lmax = build_workload(dev, seed=shard.request_seed(17, rank),
                                                        steps_total=steps_total, extra_positions=CLOCK_SOAK_RUN)
    gs = GraphStep(m, Mth, n0, dev)
    # `value`: VALUE_SLOTS step graphs with input buffers of their own, filled once before timing and
    # taken in turn, so the timed steps read inputs already resident in HBM (no staging copies).  Each
    # holds a distinct decode step: with only a few, the same few tokens would be appended over and
    # over and pile up in their clusters, which no decode does.
    nslots = min(VALUE_SLOTS, qs.shape[0])
    gsv = [gs] + [GraphStep(m, Mth, n0, dev, fresh=False) for _ in range(nslots - 1)]
    for g, gv in enumerate(gsv):
        gv.q_in.copy_(qs[g])
        gv.k_in.copy_(nks[g])
        gv.v_in.copy_(nvs[g])
    snap = {k: v.clone() for k, v in m.st[0].items()}
    n_snap, kv_snap = Mth.C.n_dev.clone(), Mth.C.kv_idx.clone()
    Kc, Vc = Mth.C.K[0].clone(), Mth.C.V[0].clone()

    def reset():
        for k, v in snap.items():
            m.st[0][k].copy_(v)
        Mth.C.n_dev.copy_(n_snap)
        Mth.C.kv_idx.copy_(kv_snap)
        Mth.C.K[0].copy_(Kc)
        Mth.C.V[0].copy_(Vc)
        torch.cuda.synchronize()

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return shard.max_over_ranks(x, device=dev)

    # ---- value: device-resident inputs.  The nvidia-smi sampler (20 ms) runs from a clock soak through
    #      the timed region: the soak replays the step graphs for CLOCK_SOAK_S (the state reset every
    #      CLOCK_SOAK_RUN steps and after it), so the clock record covers the step under load even when
    #      K steps take only a few ms.
    clk = Clocks(dev).__enter__()
    t_soak = time.time()
    soak = 0
    while soak < CLOCK_SOAK_MAX_STEPS and time.time() - t_soak < CLOCK_SOAK_S:
        for _ in range(32):
            gsv[soak % nslots].replay()
            soak += 1
        torch.cuda.synchronize()
        if soak % CLOCK_SOAK_RUN == 0:
            reset()
    reset()
    for s in range(a.warmup):
        gsv[s % nslots].replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(a.steps):
        gsv[(a.warmup + s) % nslots].replay()
    e1.record()
    torch.cuda.synchronize()
    t_timed_end = time.time()
    clk.__exit__(None, None, None)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    # ---- e2e: host buffers, copies inside the timed region.  Two step graphs with their own input
    #      and output buffers alternate; a copy stream moves step s+1's inputs in and step s's output
    #      out while step s (or s+1) computes.
    reset()
    from openattention_b200.geometry import HQ
    hq = qs.cpu().pin_memory()
    hk = nks.cpu().pin_memory()
    hv = nvs.cpu().pin_memory()
    hout = torch.empty(max(a.steps, a.warmup), m.B, m.hq, 1, 128, dtype=torch.bfloat16).pin_memory()
    n_now0, kv_now0 = Mth.C.n_dev.clone(), Mth.C.kv_idx.clone()
    gsp = [GraphStep(m, Mth, n0, dev, copy_out=True, fresh=False) for _ in range(2)]
    Mth.C.n_dev.copy_(n_now0)
    Mth.C.kv_idx.copy_(kv_now0)
    cs = torch.cuda.Stream(dev)
    main = torch.cuda.current_stream(dev)

    def run(first, count, out_rows):
        ev_in = [torch.cuda.Event() for _ in range(count)]
        ev_done = [torch.cuda.Event() for _ in range(count)]

        def h2d(j):  # inputs of step j into graph j % 2, once that graph's previous replay is done
            g = gsp[j % 2]
            with torch.cuda.stream(cs):
                if j >= 2:
                    cs.wait_event(ev_done[j - 2])
                g.q_in.copy_(hq[first + j], non_blocking=True)
                g.k_in.copy_(hk[first + j], non_blocking=True)
                g.v_in.copy_(hv[first + j], non_blocking=True)
                ev_in[j].record(cs)

        for j in range(min(2, count)):
            h2d(j)
        for j in range(count):
            main.wait_event(ev_in[j])
            gsp[j % 2].replay()
            ev_done[j].record(main)
            with torch.cuda.stream(cs):
                cs.wait_event(ev_done[j])
                hout[out_rows(j)].copy_(gsp[j % 2].out_buf, non_blocking=True)
            if j + 2 < count:
                h2d(j + 2)
        main.wait_stream(cs)

    run(0, a.warmup, lambda j: 0)
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    run(a.warmup, a.steps, lambda j: j)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / a.steps)
    h2d = (qs[0].numel() + nks[0].numel() + nvs[0].numel()) * 2
    d2h = gsp[0].out_buf.numel() * 2
    del gsp
    # ---- every kernel of the step timed inside the step graph and alone; roofline of the dominant one
    reset()
    ig_ms = in_graph_profile(m, Mth, n0, dev, qs, nks, nvs, 20)
    ig_ms = {k: max_over_ranks(v) for k, v in ig_ms.items()}
    st_ms, st_alg, step_alg, n_now, st_unique = stage_profile(m, Mth, gs, max(10, min(a.steps, 50)))
    st_ms = {k: max_over_ranks(v) for k, v in st_ms.items()}
    peak, peak_kind = peaks()
    dom = max(ig_ms, key=ig_ms.get)
    achieved = st_alg[dom] / (ig_ms[dom] * 1e-3) / 1e9
    stages = {k: {"us": round(ig_ms[k] * 1e3, 2), "alone_us": round(st_ms[k] * 1e3, 2), "alg_bytes": st_alg[k],
                  "gbs": round(st_alg[k] / (ig_ms[k] * 1e-3) / 1e9, 1),
                  "frac": round(st_alg[k] / (ig_ms[k] * 1e-3) / 1e9 / peak, 4)} for k in st_ms}
    for k, ub in st_unique.items():  # bytes counting each K/V row once per KV head (GQA-unique)
        stages[k]["unique_alg_bytes"] = ub
        stages[k]["unique_frac"] = round(ub / (ig_ms[k] * 1e-3) / 1e9 / peak, 4)
    step_gbs = step_alg / (ms * 1e-3 * 1.0) / 1e9
    res = None
    if rank == 0:
        cpu = cpu_baseline_sample(m, Mth, qs, nks, nvs) if world == 1 else None
        Rkv_codes_mb = m.B * m.hkv * Lmax * 32 / 1e6
        kv_gb = 2 * m.B * m.hkv * Lmax * 128 * 2 / 1e9
        if plan is None:  # weak scaling: µs per bs32 layer-step for the whole job
            div, scaling, gb = world, "weak", B_PER_GPU * world
            workload = f"c2 decode-attn-stage: B={B_PER_GPU} requests/GPU"
            par = f"request-sharded x{world} (no data-path collective)"
        else:  # strong scaling: µs per step of the fixed batch (max over ranks)
            div, scaling, gb = 1, "strong", a.global_batch
            workload = f"decode-attn-stage: global batch {a.global_batch}"
            par = (f"{plan.kind}-sharded x{world}: rank 0 holds {plan.req_count} request(s) x {plan.kv_count} KV "
                   "head(s) (no data-path collective)")
        res = {
            "metric": METRIC, "value": round(ms * 1e3 / div, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 5), "higher_is_better": False, "scaling": scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded clustered RoPE keys, N(0,1) values/queries)",
            "config": {"workload": f"{workload}, n={N_CTX}+steps, rho={RHO:g} (C={m.C}, E={m.E}), one layer step as "
                                   "one CUDA graph",
                       "global_batch": gb, "seq_len": N_CTX, "parallelism": par,
                       "l2": (f"inputs larger than L2 (int8 codes {Rkv_codes_mb:.0f} MB + bf16 K/V {kv_gb:.2f} GB per GPU), "
                              "no flush" if Rkv_codes_mb > 126 else
                              f"int8 codes {Rkv_codes_mb:.0f} MB + bf16 K/V {kv_gb:.2f} GB per GPU; step reads about "
                              "1% of them, no flush")},
            "e2e": {"value": round(ms_e2e * 1e3 / div, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": LAUNCHES_PER_STEP * a.steps,
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         # the committed ncu traffic figures are for the default workload (B=32 per GPU) only
                         "traffic": traffic_from_profiles(dom) if plan is None and B_PER_GPU == 32 else None,
                         "alg_bytes_per_launch": st_alg[dom],
                         "launch_us": round(ig_ms[dom] * 1e3, 3), "launch_timing": "inside the step graph (event-record nodes)"},
            "stages": stages,
            "step_roofline": {"alg_bytes": step_alg, "achieved": round(step_gbs, 1), "unit": "GB/s",
                              "frac": round(step_gbs / peak, 4), "n": n_now},
            "clocks": clk.summary(t_soak, t_timed_end + 0.05,
                                  window=f"clock soak ({soak} replays of the step, {CLOCK_SOAK_S:g} s) through the timed "
                                         "region"),
            "cpu_baseline": cpu,
            "stage_us_per_step_per_gpu": round(ms * 1e3, 3),
        }
    if pg is not None:
        del gs
        pg.barrier()
        pg.destroy_process_group()
    return res


# ------------------------------------------------------------------ latency sweep (config c3)
SWEEP_B = (1, 4, 16, 32, 64)
SWEEP_N = (8192, 16384, 32768, 65536, 131072)
SWEEP_RHO = (0.01, 0.05)


def sweep_point(dev, B, n0, rho, steps, warmup):
    """One point of the latency sweep: one request of n0 tokens is built and replicated B times (the
    per-request work does not depend on which request it is), then `steps` graph-replayed decode
    steps are timed with CUDA events (inputs larger than L2 from B = 4 on; at B = 1 the step
    reads about 16 MB per step and the number is a latency)."""
    from openattention_b200 import method as Mth
    from openattention_b200 import synth
    from openattention_b200.geometry import HQ
    total = warmup + steps + 4
    Lmax = n0 + total + 16
    K1, V1, mus = synth.kv_torch(41, 1, n0, Lmax, dev)
    K = K1.expand(B, -1, -1, -1).contiguous()
    V = V1.expand(B, -1, -1, -1).contiguous()
    del K1, V1
    Mth.C.K, Mth.C.V, Mth.C.qlen = [K], [V], [40] * B
    m = Mth.OursB200(types.SimpleNamespace(rho=rho, static_metric=synth.static_metric_standin(7, 1)), B, Lmax, dev,
                     layers=1)
    g = torch.Generator(device=dev)
    g.manual_seed(43)
    qpre = torch.zeros(1, HQ, n0, 128, dtype=torch.bfloat16, device=dev)
    qpre[:, :, n0 - 64:] = torch.randn(1, HQ, 64, 128, generator=g, device=dev).to(torch.bfloat16)
    m.build(0, 0, qpre, n0)
    del qpre
    for k, v in m.st[0].items():
        if k in ("reclist", "reccnt"):
            v.zero_()
        v[1:].copy_(v[0:1].expand_as(v[1:]))
    gs = GraphStep(m, Mth, n0, dev)
    qs = torch.randn(total, B, HQ, 1, 128, generator=g, device=dev).to(torch.bfloat16)
    nk, nv = synth.new_tokens_torch(45, mus.expand(B, *mus.shape[1:]).contiguous(), n0)
    for s in range(warmup):
        gs.q_in.copy_(qs[s])
        gs.k_in.copy_(nk)
        gs.v_in.copy_(nv)
        gs.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        gs.q_in.copy_(qs[warmup + s])
        gs.k_in.copy_(nk)
        gs.v_in.copy_(nv)
        gs.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    R, Rkv, C, E = B * HQ, B * 8, m.C, m.E
    n = int(Mth.C.n_dev.item())
    from openattention_b200.geometry import step_split
    ns, nl, k_top = step_split(gs.n_host, rho, C, E)
    NS = ns + nl + k_top
    reads = int((m.exp_idx >= 0).sum().item()) + R * NS
    alg = (Rkv * n * 32 + 3 * R * C * 128 * 4 + reads * 512 + R * C * 4 + R * (NS + E) * 4 + 2 * R * 256
           + R * (128 * 16 * 2 + C * 16 * 4) + Rkv * 128 * 32 * 4)
    del gs, m, K, V
    torch.cuda.empty_cache()
    return {"sweep": "c3", "B": B, "n": n0, "rho": rho, "C": C, "E": E, "us_per_step": round(ms * 1e3, 2),
            "alg_bytes": alg, "achieved_gbs": round(alg / (ms * 1e-3) / 1e9, 1),
            "frac": round(alg / (ms * 1e-3) / 1e9 / peaks()[0], 4)}


def run_sweep(a):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Bs = [int(x) for x in a.sweep_b.split(",")] if a.sweep_b else SWEEP_B
    Ns = [int(x) for x in a.sweep_n.split(",")] if a.sweep_n else SWEEP_N
    rhos = [float(x) for x in a.sweep_rho.split(",")] if a.sweep_rho else SWEEP_RHO
    for rho in rhos:
        for n0 in Ns:
            for B in Bs:
                print(json.dumps(sweep_point(dev, B, n0, rho, a.steps, a.warmup)), flush=True)
    return None


# ------------------------------------------------------------------ end-to-end model decode (config c4)
def run_model_e2e(a):
    """Config c4: a random-initialised Llama-3.1-8B architecture with the OpenAttention path as its
    attention; dense prefill of a uniformly random prompt (plus the index build of every layer), then
    `--decode-steps` greedy decode steps replayed as one CUDA graph per step.  Reports ms per decode
    step (per token of each request) and the aggregate tokens/s.

    Under torchrun every rank is a batch replica (its own model copy, batch and prompt); after each step
    the ranks' new token ids are gathered with NCCL (all_gather_into_tensor over NVLink, the only
    collective), and the step time is the max over ranks."""
    from openattention_b200 import llama as L
    from openattention_b200 import shard
    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg = L.LlamaConfig()
    B, T, steps = B_PER_GPU, a.prompt, a.decode_steps
    model = L.RandomLlama(cfg, B, T + steps + a.warmup + 16, dev, rho=RHO, seed=1)
    g = torch.Generator(device=dev)
    g.manual_seed(2 + 1000 * rank)
    prompt = torch.randint(0, cfg.vocab, (B, T), generator=g, device=dev)
    model.prefill(prompt[:, :min(T, 1024)])  # warm-up: library handles, kernel selection, host buffers
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = model.prefill(prompt)
    torch.cuda.synchronize()
    t_prefill = time.perf_counter() - t0
    model.start_decode(T, first)
    model.capture()
    gathered = torch.empty(world * B, dtype=torch.long, device=dev)

    def step():
        tok = model.step_graph()
        if dist is not None:  # every replica's new tokens, in rank order
            dist.all_gather_into_tensor(gathered, tok)
        return tok

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = shard.max_over_ranks(e0.elapsed_time(e1) / steps, device=dev)
    t_prefill = shard.max_over_ranks(t_prefill, device=dev)
    status = int(model.method.status.item())
    if dist is not None:
        model.graph = None
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {"metric": "ms/token e2e (c4: random-init Llama-3.1-8B, OpenAttention 1% decode)", "value": round(ms, 4),
            "unit": "ms/token", "n_gpus": world, "steps": steps, "warmup": a.warmup, "higher_is_better": False,
            "tokens_per_s": round(world * B * 1000.0 / ms, 1), "dtype": "bf16",
            "data": "synthetic (uniform random prompt)",
            "prefill_incl_build_s": round(t_prefill, 2),
            "prefill_plus_128_steps_s": round(t_prefill + 128 * ms / 1e3, 2),  # the reference's e2e-seconds measure
            "config": {"workload": "c4 end-to-end decode", "model": "Llama-3.1-8B architecture, random init",
                       "global_batch": world * B, "prompt": T, "decode_steps": steps, "rho": RHO,
                       "parallelism": (f"batch replicas x{world}, new token ids gathered by NCCL each step"
                                       if world > 1 else "single GPU")},
            "status": status}


# ------------------------------------------------------------------ reference arm (CPU)
def use_all_host_threads(O):
    """The CPU legs use every host core (torchrun sets OMP_NUM_THREADS=1 per rank).  Returns the
    thread count in effect."""
    return O.set_threads(os.cpu_count() or 1)


def run_reference(a):
    rank, world, local = dist_env()
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = use_all_host_threads(O)
    from openattention_b200 import synth
    from openattention_b200.geometry import HQ, budget
    C, E = budget(RHO)
    B_s = 1  # requests per sample step (bounded CPU sample), scaled to bs32
    n0 = N_CTX
    Lmax = n0 + a.warmup + a.steps + 8
    st = O.new_state(B_s, Lmax, C)
    K = np.zeros((B_s, 8, Lmax, 128), np.uint16)
    V = np.zeros_like(K)
    mus = []
    t_build = time.perf_counter()
    Mpre = synth.static_metric_numpy(7, 1)[0]
    inv = synth.llama31_inv_freq()
    for b in range(B_s):
        Kb, Vb, mu = synth.kv_numpy(17 + b, n0, Lmax)
        K[b], V[b] = O.bits(Kb), O.bits(Vb)
        mus.append(mu)
        qpre = torch.zeros(HQ, n0, 128, dtype=torch.bfloat16)
        qpre[:, n0 - 64:] = synth.queries_numpy(5017 + b, HQ * 64).view(HQ, 64, 128)
        M = O.metric(Mpre, inv, 1.0, qpre, n0, 40)
        U, W = O.basis(M)
        O.build_from_basis(st, b, K[b], V[b], U.numpy(), O.bits(W), n0, layer=0)
    t_build = time.perf_counter() - t_build
    times = []
    n = n0
    for s in range(a.warmup + a.steps):
        n += 1
        for b in range(B_s):
            nk, nv = synth.new_token_numpy(20017 + 100 * s + b, mus[b], n - 1)
            K[b, :, n - 1], V[b, :, n - 1] = O.bits(nk), O.bits(nv)
        q = O.bits(synth.queries_numpy(9017 + s, B_s * HQ))
        t0 = time.perf_counter()
        O.decode_step(st, q, K, V, n, RHO, C, E)
        if s >= a.warmup:
            times.append(time.perf_counter() - t0)
    per = statistics.median(times) / B_s * B_PER_GPU * 1e6
    cores = threads
    sample = (f"{a.steps} timed decode steps of {B_s} request(s) at n={N_CTX}, 1% read (C={C}, E={E}); median "
              f"scaled x{B_PER_GPU // B_s} to bs32; build {t_build:.1f} s untimed")
    return {"metric": METRIC, "value": round(per, 1), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(per / 1e3, 4), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded clustered RoPE keys)",
            "impl": "reference",
            "config": {"workload": f"c2 decode-attn-stage: B={B_PER_GPU} requests, n={N_CTX}, rho={RHO:g} (C={C}, E={E}), "
                                   "one layer step", "global_batch": B_PER_GPU, "seq_len": N_CTX,
                       "parallelism": "host CPU"},
            "cpu_baseline": {"value": round(per, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(per, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    global B_PER_GPU, N_CTX, RHO
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model-e2e", action="store_true",
                    help="config c4: end-to-end decode of a random-init Llama-3.1-8B (ms/token); --batch sets B")
    ap.add_argument("--prompt", type=int, default=30000, help="prompt length for --model-e2e")
    ap.add_argument("--decode-steps", type=int, default=256, help="decode steps for --model-e2e")
    ap.add_argument("--sweep", action="store_true",
                    help="latency sweep of the decode step over batch x context x read (one JSON line per point)")
    ap.add_argument("--sweep-b", default="", help="comma list of batches for --sweep")
    ap.add_argument("--sweep-n", default="", help="comma list of contexts for --sweep")
    ap.add_argument("--sweep-rho", default="", help="comma list of read fractions for --sweep (0.01, 0.03, 0.05)")
    ap.add_argument("--ctx", type=int, default=N_CTX,
                    help="context length (default 32768, the benchmark config; others only for profiling)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="a fixed batch split over the GPUs (strong scaling): by request, or by KV head when it is "
                         "smaller than the GPU count (e.g. --gpus 8 --global-batch 1)")
    ap.add_argument("--batch", type=int, default=None,
                    help="requests per GPU (default 32, the benchmark config; smaller only for profiling; "
                         "--model-e2e defaults to 1, config c4)")
    ap.add_argument("--rho", type=float, default=RHO,
                    help="read fraction (default 0.01, the benchmark config; 0.03 / 0.05 only for profiling)")
    a = ap.parse_args()
    B_PER_GPU = a.batch if a.batch is not None else (1 if a.model_e2e else 32)
    N_CTX = a.ctx
    RHO = a.rho
    if a.warmup < 3:
        a.warmup = 3
    if a.sweep:
        run_sweep(a)
        return
    if a.model_e2e:
        res = run_model_e2e(a)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    res = run_reference(a) if a.impl == "reference" else run_ours(a)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
