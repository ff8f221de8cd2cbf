"""The end-to-end decode loop (random-initialised Llama-3.1 architecture, OpenAttention as attention) on
a small configuration: prefill + index build, then decode steps eagerly and as a replayed CUDA graph;
the two give the same tokens (same kernels, same order), and every step's hidden state is finite."""
import pytest
import torch

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
