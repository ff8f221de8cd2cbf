"""End-to-end decode of a random-initialised Llama-3.1-8B architecture whose attention is the
OpenAttention path of this package (the caller of the path: inference/graph_runner.py:469-482 attention
hook, :567-719 CUDA-graph decode loop; model shapes of Llama-3.1-8B).

The dense parts (embedding, RMSNorm, the QKV / O / MLP projections, the LM head) are plain PyTorch
(cuBLAS GEMMs).  Prefill writes the post-RoPE K/V cache, attends densely (PyTorch SDPA, causal,
grouped-query) and then builds each layer's index with `OursB200.build`; every decode step runs the
layers with `OursB200.decode` as the attention and picks the next token greedily.  A whole decode
step (all layers) is captured once as a CUDA graph: the write position and the current length are
device counters (C.kv_idx, C.n_dev), so the graph replays step after step.

Weights are random (there are no checkpoints in this environment); the numbers it produces are
timings and the sparse path's behaviour, not language-model quality.
"""
from __future__ import annotations

import types
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import method as Mth
from .geometry import D, HKV, HQ, llama31_inv_freq


_DENSE_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.CUDNN_ATTENTION]

# the index state the decode step's index update changes (besides the new position's code and
# assignment, which the next real step rewrites identically)
_STEP_STATE = ("nb", "Sk", "Sk2", "Sv", "reclist", "reccnt")


@dataclass
class LlamaConfig:
    layers: int = 32
    hidden: int = HQ * D        # 4096: the attention geometry of the path is fixed
    ffn: int = 14336
    vocab: int = 128256
    eps: float = 1e-5
    qlen: int = 40              # question rows the index build uses (C.qlen)


class RandomLlama:
    """Random bf16 weights (std 1/sqrt(fan-in)), caches and the OpenAttention method for B requests
    of up to Lmax positions."""

    def __init__(self, cfg: LlamaConfig, B: int, Lmax: int, dev, rho: float = 0.01, seed: int = 0,
                 static_metric=None):
        self.cfg, self.B, self.Lmax = cfg, B, Lmax
        self.dev = torch.device(dev)
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        H, Fd, V = cfg.hidden, cfg.ffn, cfg.vocab
        nqkv = (HQ + 2 * HKV) * D

        def w(rows, cols):
            return (torch.randn(rows, cols, generator=g, device=self.dev) * rows ** -0.5).to(torch.bfloat16)

        self.embed = (torch.randn(V, H, generator=g, device=self.dev)).to(torch.bfloat16)
        self.wqkv = [w(H, nqkv) for _ in range(cfg.layers)]
        self.wo = [w(HQ * D, H) for _ in range(cfg.layers)]
        self.wgu = [w(H, 2 * Fd) for _ in range(cfg.layers)]
        self.wdown = [w(Fd, H) for _ in range(cfg.layers)]
        self.ln1 = [torch.ones(H, dtype=torch.bfloat16, device=self.dev) for _ in range(cfg.layers)]
        self.ln2 = [torch.ones(H, dtype=torch.bfloat16, device=self.dev) for _ in range(cfg.layers)]
        self.norm = torch.ones(H, dtype=torch.bfloat16, device=self.dev)
        self.lm_head = w(H, V)
        # RoPE tables (Llama-3.1 frequency scaling), fp32, every position of the cache
        inv = llama31_inv_freq().to(self.dev).float()
        pos = torch.arange(Lmax, device=self.dev, dtype=torch.float32)
        emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], -1)
        self.cos, self.sin = emb.cos(), emb.sin()
        self.K = [torch.zeros(B, HKV, Lmax, D, dtype=torch.bfloat16, device=self.dev) for _ in range(cfg.layers)]
        self.V = [torch.zeros(B, HKV, Lmax, D, dtype=torch.bfloat16, device=self.dev) for _ in range(cfg.layers)]
        Mth.C.K, Mth.C.V, Mth.C.qlen = self.K, self.V, [cfg.qlen] * B
        # the weights are random, so the query metric of the real model means nothing here: the seeded
        # stand-in is the default (a real checkpoint would pass the reference's asset)
        if static_metric is None:
            from .synth import static_metric_standin
            static_metric = static_metric_standin(7, cfg.layers)
        self.method = Mth.OursB200(types.SimpleNamespace(rho=rho, static_metric=static_metric), B, Lmax, self.dev,
                                   layers=cfg.layers)
        self.graph = None

    # ------------------------------------------------------------------ pieces
    def _rms(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(torch.bfloat16) * w

    @staticmethod
    def _rope(x, cos, sin):
        """x (..., T, D) with cos / sin (T, D) broadcast over the leading dims."""
        h = D // 2
        xf = x.float()
        rot = torch.cat([-xf[..., h:], xf[..., :h]], -1)
        return (xf * cos + rot * sin).to(torch.bfloat16)

    def _mlp(self, x, l):
        gu = x @ self.wgu[l]
        gate, up = gu.chunk(2, dim=-1)
        return (F.silu(gate.float()) * up.float()).to(torch.bfloat16) @ self.wdown[l]

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, chunk: int = 8192) -> torch.Tensor:
        """tokens (B, T) int64.  Fills every layer's K/V cache for positions [0, T), builds the index of
        every layer and request, and returns the greedy next token (B,)."""
        B, T = tokens.shape
        cos, sin = self.cos[:T], self.sin[:T]
        nxt = torch.empty(B, dtype=torch.long, device=self.dev)
        for b in range(B):
            x = self.embed[tokens[b]]                                      # (T, H)
            pending = None  # the previous layer's build, finished once this layer's work is enqueued
            for l in range(self.cfg.layers):
                h = self._rms(x, self.ln1[l])
                qkv = h @ self.wqkv[l]
                q = qkv[:, :HQ * D].view(T, HQ, D).transpose(0, 1)          # (32, T, D)
                k = qkv[:, HQ * D:(HQ + HKV) * D].view(T, HKV, D).transpose(0, 1)
                v = qkv[:, (HQ + HKV) * D:].view(T, HKV, D).transpose(0, 1)
                q = self._rope(q, cos, sin)
                k = self._rope(k, cos, sin)
                self.K[l][b, :, :T] = k
                self.V[l][b, :, :T] = v
                g = HQ // HKV  # grouped-query: each KV head serves 4 query heads
                with sdpa_kernel(_DENSE_BACKENDS):  # never the T x T math path
                    o = F.scaled_dot_product_attention(q.unsqueeze(0), k.repeat_interleave(g, 0).unsqueeze(0),
                                                       v.repeat_interleave(g, 0).unsqueeze(0), is_causal=True)[0]
                x = x + o.transpose(0, 1).reshape(T, HQ * D) @ self.wo[l]
                for t0 in range(0, T, chunk):                            # MLP in row chunks (activation memory)
                    t1 = min(T, t0 + chunk)
                    x[t0:t1] = x[t0:t1] + self._mlp(self._rms(x[t0:t1], self.ln2[l]), l)
                finish = self.method.build_async(l, b, q.unsqueeze(0), T)
                if pending is not None:
                    pending()
                pending = finish
            pending()
            logits = self._rms(x[-1:], self.norm) @ self.lm_head
            nxt[b] = logits.float().argmax(-1)[0]
        return nxt

    # ------------------------------------------------------------------ decode
    def _decode_body(self, tok: torch.Tensor, n_host: int) -> torch.Tensor:
        """One decode step for the B requests: token tok (B,) at position C.kv_idx (= n - 1)."""
        C, B = Mth.C, self.B
        C.n_dev.add_(1)
        C.kv_idx.add_(1)
        cos = self.cos.index_select(0, C.kv_idx)                          # (1, D)
        sin = self.sin.index_select(0, C.kv_idx)
        x = self.embed.index_select(0, tok)                               # (B, H)
        for l in range(self.cfg.layers):
            h = self._rms(x, self.ln1[l])
            qkv = h @ self.wqkv[l]
            q = self._rope(qkv[:, :HQ * D].view(B, HQ, D), cos, sin)
            k = self._rope(qkv[:, HQ * D:(HQ + HKV) * D].view(B, HKV, D), cos, sin)
            v = qkv[:, (HQ + HKV) * D:].view(B, HKV, D)
            # this layer's new K/V rows are written at position n - 1 (the counters advanced at the step's
            # start) by the index update's launch
            o = self.method.decode(l, q.view(B, HQ, 1, D), n_host, k_new=k.contiguous(), v_new=v.contiguous())
            x = x + o.reshape(B, HQ * D) @ self.wo[l]
            x = x + self._mlp(self._rms(x, self.ln2[l]), l)
        logits = self._rms(x, self.norm) @ self.lm_head
        return logits.float().argmax(-1)

    @torch.no_grad()
    def start_decode(self, n0: int, first: torch.Tensor):
        """Device counters for a decode that starts after a prefix of n0 positions, with `first` (B,)
        the token to feed at position n0."""
        C = Mth.C
        C.n_dev = torch.full((1,), n0, dtype=torch.int32, device=self.dev)    # before the step
        C.kv_idx = torch.full((1,), n0 - 1, dtype=torch.int64, device=self.dev)
        C.n0_dev = torch.full((1,), n0, dtype=torch.int32, device=self.dev)
        self.n_host = n0 + 1  # ns / nl / k_top of the step (constant over a decode window)
        self.tok = first.to(self.dev).clone()

    @torch.no_grad()
    def step_eager(self) -> torch.Tensor:
        self.tok = self._decode_body(self.tok, self.n_host)
        return self.tok

    @torch.no_grad()
    def capture(self):
        """Capture one decode step (all layers) as a CUDA graph; the counters are restored after the
        warm-up, so the next replay is the next step."""
        C = Mth.C
        n_snap, kv_snap, tok_snap = C.n_dev.clone(), C.kv_idx.clone(), self.tok.clone()
        st_snap = [{k: st[k].clone() for k in _STEP_STATE if k in st} for st in self.method.st]
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self._decode_body(self.tok, self.n_host)   # warm-up outside capture (one extra token written)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize()
        C.n_dev.copy_(n_snap)
        C.kv_idx.copy_(kv_snap)
        self.tok.copy_(tok_snap)
        for st, snap in zip(self.method.st, st_snap):
            for k, v in snap.items():
                st[k].copy_(v)
        del st_snap
        self._tok_in = self.tok
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._tok_out = self._decode_body(self._tok_in, self.n_host)
        torch.cuda.synchronize()

    @torch.no_grad()
    def step_graph(self) -> torch.Tensor:
        self.graph.replay()
        self._tok_in.copy_(self._tok_out)
        return self._tok_out
