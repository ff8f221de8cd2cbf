"""The Python stage wrappers reject tensors a kernel cannot use before anything reaches the library:
host tensors (whose addresses a kernel would fault on, or on a GPU that can reach host memory read
silently), tensors on another device, and rows of the wrong dtype or layout.  CPU only: every call
here must raise before its first launch."""
import pytest
import torch

from openattention_b200 import selection as S
from openattention_b200.geometry import D, HKV, HQ, RQ

B, Lmax, C, E, NS = 1, 64, 8, 16, 5
R = B * HQ


def _host_inputs():
    bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
    st = S.new_state(B, Lmax, C, "cpu")
    return dict(
        K=torch.zeros(B, HKV, Lmax, D, dtype=bf), V=torch.zeros(B, HKV, Lmax, D, dtype=bf), st=st,
        q=torch.zeros(R, D, dtype=bf), zq=torch.zeros(R, RQ, dtype=bf), n_dev=torch.ones(1, dtype=i32),
        scores=torch.zeros(R, S.padded_len(Lmax), dtype=bf), tmax=torch.zeros(R, Lmax // 32, dtype=f32),
        sel=torch.zeros(R, NS, dtype=i32), exp_idx=torch.zeros(R, E, dtype=i32), nt=torch.zeros(R, C, dtype=f32),
        quota=torch.zeros(R, C, dtype=f32), score=torch.zeros(R, C, dtype=f32), out=torch.zeros(R, D, dtype=f32),
        kbar=torch.zeros(R, C, D, dtype=bf), vbar=torch.zeros(R, C, D, dtype=bf), logn=torch.zeros(R, C, dtype=f32),
        k_new=torch.zeros(B, HKV, D, dtype=bf), v_new=torch.zeros(B, HKV, D, dtype=bf))


CALLS = {
    "append_kv": lambda x: S.append_kv(x["K"], x["V"], x["k_new"], x["v_new"], x["n_dev"]),
    "index_update": lambda x: S.index_update(x["K"], x["V"], x["st"], x["n_dev"], q=x["q"], zq=x["zq"]),
    "qgs_scan": lambda x: S.qgs_scan(x["st"]["codes"], x["zq"], x["n_dev"], 1, 1, x["scores"], x["tmax"]),
    "qgs_select": lambda x: S.qgs_select(x["scores"], x["tmax"], Lmax, x["n_dev"], 1, 1, NS - 2, x["sel"]),
    "errorgate_waterfill": lambda x: S.errorgate_waterfill(x["q"], x["K"], x["st"], x["sel"], E, x["score"],
                                                           x["nt"], x["quota"]),
    "topq": lambda x: S.topq(x["scores"], x["st"], x["quota"], E, x["n_dev"], x["n_dev"], x["exp_idx"]),
    "residual": lambda x: S.residual(x["K"], x["V"], x["st"], x["sel"], x["exp_idx"], x["nt"], x["quota"],
                                     x["kbar"], x["vbar"], x["logn"]),
    "residual_flash": lambda x: S.residual_flash(x["q"], x["K"], x["V"], x["st"], x["sel"], x["exp_idx"], x["nt"],
                                                 x["quota"], x["out"]),
}


@pytest.mark.parametrize("name", list(CALLS))
def test_host_tensors_are_rejected(name):
    with pytest.raises(RuntimeError, match="CUDA|need a tensor on"):
        CALLS[name](_host_inputs())


def test_device_and_layout_helpers():
    cuda0 = torch.device("cuda", 0)
    with pytest.raises(RuntimeError, match="need a tensor on cuda:0"):
        S._on(cuda0, ("x", torch.zeros(2)))
    S._on(cuda0, ("none", None))  # absent optional tensors pass
    with pytest.raises(RuntimeError, match="state\\['nb'\\]"):
        S._state_on(cuda0, {"nb": torch.zeros(1)})
    S._rows("q", torch.zeros(4, 8, dtype=torch.bfloat16), torch.bfloat16, 4, 8)
    for bad in (torch.zeros(4, 8, dtype=torch.float32), torch.zeros(3, 8, dtype=torch.bfloat16),
                torch.zeros(8, 4, dtype=torch.bfloat16).t(), torch.zeros(4, 8, 1, dtype=torch.bfloat16)):
        with pytest.raises(RuntimeError, match="contiguous last dim"):
            S._rows("q", bad, torch.bfloat16, 4, 8)


def test_flash_entries_reject_host_and_foreign_tensors():
    from openattention_b200 import flash as F
    bf = torch.bfloat16
    q, k = torch.zeros(4, D, dtype=bf), torch.zeros(1, 16, D, dtype=bf)
    sel, ex = torch.zeros(4, 2, dtype=torch.int32), torch.zeros(4, 3, dtype=torch.int32)
    kb, ln = torch.zeros(1, 2, D, dtype=bf), torch.zeros(4, 2)
    for fn in (F.decode_expand_attention, F.ours_flash):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn(q, k, k, sel, ex, kb, kb, ln)
    cuda0 = torch.device("cuda", 0)
    F._same_device(cuda0, out=None, workspace=None)
    with pytest.raises(RuntimeError, match="sel_idx must be a tensor on cuda:0"):
        F._same_device(cuda0, sel_idx=sel)
    with pytest.raises(RuntimeError, match="exp_idx must be a tensor on cuda:0 .*list"):
        F._same_device(cuda0, exp_idx=[1, 2])


def test_topq_variant_by_row_length():
    """oa_topq_variant names the kernel rows of a length take, and the benchmark's default c2 workload
    (its KV buffer with the warm-up, twice the timed steps and the clock soak's positions) stays on
    the pipelined one: a longer buffer would measure the one-buffer kernel instead."""
    import bench
    from openattention_b200 import selection as S
    from openattention_b200.geometry import budget
    C, E = budget(bench.RHO)
    assert (C, E) == (64, 216)
    assert S.topq_variant(32768, E, C) == 0
    assert S.topq_variant(35308, E, C) == 0
    assert S.topq_variant(40000, E, C) == 1
    assert S.topq_variant(65536, E, C) == 2
    steps, warmup = 500, 20  # bench.py's defaults
    Lmax = bench.N_CTX + (warmup + 2 * steps + 8) + bench.CLOCK_SOAK_RUN + 16
    assert S.topq_variant(Lmax, E, C) == 0, Lmax
