"""The end-to-end decode loop (random-initialised Llama-3.1 architecture, OpenAttention as attention) on
a small configuration: prefill + index build, then decode steps eagerly and as a replayed CUDA graph;
the two give the same tokens (same kernels, same order), and every step's hidden state is finite."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import to_np
from openattention_b200 import llama as L
from openattention_b200 import method as Mth

pytestmark = pytest.mark.gpu


def _run(graph: bool, steps: int = 6):
    cfg = L.LlamaConfig(layers=2, ffn=1024, vocab=2048)
    B, T = 2, 2048
    model = L.RandomLlama(cfg, B, T + steps + 16, "cuda", rho=0.01, seed=3)
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    prompt = torch.randint(0, cfg.vocab, (B, T), generator=g, device="cuda")
    first = model.prefill(prompt)
    model.start_decode(T, first)
    if graph:
        model.capture()
    toks = [first.clone()]
    for _ in range(steps):
        toks.append((model.step_graph() if graph else model.step_eager()).clone())
    torch.cuda.synchronize()
    assert int(model.method.status.item()) == 0
    assert torch.isfinite(model.method.out.float()).all()
    assert int(Mth.C.n_dev.item()) == T + steps
    return torch.stack(toks)


def test_graph_decode_matches_eager():
    eager = _run(False)
    graph = _run(True)
    assert torch.equal(eager, graph)
    assert eager.shape == (7, 2)
    assert bool(((eager >= 0) & (eager < 2048)).all())


def test_model_decode_layer_matches_oracle():
    """One decode step of the model, layer 0 checked against the oracle: the layer's query and new K/V
    rows (as the model produced them) and its index state before the step go through the oracle's step;
    the method's selected and expanded indices are bit-exact and its bf16 attention output is within
    2e-3 plus one bf16 rounding of the fp32 estimator."""
    cfg = L.LlamaConfig(layers=2, ffn=1024, vocab=2048)
    B, T, D = 2, 2048, 128
    model = L.RandomLlama(cfg, B, T + 16, "cuda", rho=0.01, seed=5)
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    prompt = torch.randint(0, cfg.vocab, (B, T), generator=g, device="cuda")
    first = model.prefill(prompt)
    model.start_decode(T, first)
    meth = model.method
    rec = {}
    orig = meth.decode

    def spy(l, q, n, k_new=None, v_new=None):
        if l != 0 or rec:
            return orig(l, q, n, k_new=k_new, v_new=v_new)
        torch.cuda.synchronize()
        rec.update(st={k: to_np(v).copy() for k, v in meth.st[0].items()}, K=O.bits(Mth.C.K[0]).copy(),
                   V=O.bits(Mth.C.V[0]).copy(), q=O.bits(q.reshape(B * 32, D)).copy(), k=O.bits(k_new),
                   v=O.bits(v_new), n=n)
        out = orig(l, q, n, k_new=k_new, v_new=v_new)
        torch.cuda.synchronize()
        rec.update(out=out.float().cpu().numpy().reshape(B * 32, D), sel=to_np(meth.last_sel).copy(),
                   exp=to_np(meth.exp_idx).copy())
        return out

    meth.decode = spy
    model.step_eager()
    torch.cuda.synchronize()
    n, st, K, V = rec["n"], rec["st"], rec["K"], rec["V"]
    K[:, :, n - 1], V[:, :, n - 1] = rec["k"], rec["v"]
    R, C = B * 32, meth.C
    o = O.decode_step(st, rec["q"], K, V, n, 0.01, C, meth.E)
    assert np.array_equal(rec["sel"], o["sel"])
    assert np.array_equal(rec["exp"], o["exp_idx"])
    Lmax = K.shape[2]
    Skr, Svr, nr = O.residual_sums(K, V, st["asg"].reshape(R, -1), o["sel"], o["exp_idx"], st["Sk"].reshape(R, C, D),
                                   st["Sv"].reshape(R, C, D), o["nt"], o["quota"])
    est = O.estimator_fp32(rec["q"], K.reshape(B * 8, Lmax, D), V.reshape(B * 8, Lmax, D), o["sel"], o["exp_idx"],
                           Skr, Svr, nr)
    assert np.all(np.abs(rec["out"] - est) <= 2e-3 + np.abs(est) * 2.0 ** -8)
