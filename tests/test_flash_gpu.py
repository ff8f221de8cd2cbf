"""OpenAttention.flash on the GPU vs the fp64 CPU oracle (and the reference's golden output).

Tolerance (north star): fp32 output within 2e-3 max-abs and 1e-3 relative-L2 of the estimator;
bf16 output equal to the bf16 rounding of the estimator within one bf16 ulp per element."""
import math
import os

import numpy as np
import pytest
import torch

import cases
import oracle as O
from openattention_b200 import flash as F

pytestmark = pytest.mark.gpu
D = 128
MAX_ABS, REL_L2 = 2e-3, 1e-3


def _run(x, out_dtype, nsplit=0, k=None, v=None, nb=None):
    dev = "cuda"
    q = x["q"].to(dev)
    k = (x["k"] if k is None else k).to(dev)
    v = (x["v"] if v is None else v).to(dev)
    args = (q, k, v, x["sel"].to(dev), x["exp"].to(dev), x["kbar"].to(dev), x["vbar"].to(dev), x["log_n"].to(dev))
    if x["kind"] == "qhead":
        o = F.ours_flash(*args, nb=nb, out_dtype=out_dtype, nsplit=nsplit)
    else:
        o = F.decode_expand_attention(*args, out_dtype=out_dtype, nsplit=nsplit)
    torch.cuda.synchronize()
    return o.cpu()


def _oracle(x, nb=None):
    kb = x["kbar"] if nb != 0 else None
    return O.flash(O.bits(x["q"]), O.bits(x["k"]), O.bits(x["v"]), x["sel"].numpy(), x["exp"].numpy(),
                   None if kb is None else O.bits(kb), None if kb is None else O.bits(x["vbar"]),
                   None if kb is None else x["log_n"].numpy(), D ** -0.5, per_qhead=x["kind"] == "qhead")


def _check_f32(out, ref):
    out = out.double().numpy()
    assert np.abs(out - ref).max() <= MAX_ABS
    assert np.linalg.norm(out - ref) <= REL_L2 * np.linalg.norm(ref)


def _check_bf16(out, ref):
    r = torch.from_numpy(ref).float()
    rb = r.to(torch.bfloat16).float()
    o = out.float()
    ulp = torch.maximum(rb.abs(), torch.full_like(rb, 2.0 ** -126)) * 2.0 ** -7
    assert bool(((o - rb).abs() <= ulp * 1.01).all())


@pytest.mark.parametrize("name", list(cases.FLASH_CASES))
@pytest.mark.parametrize("nsplit", [1, 0, 2, 3, 8, 16])
def test_flash_matches_oracle(name, nsplit):
    x = cases.flash_inputs(name)
    ref = _oracle(x)
    _check_f32(_run(x, torch.float32, nsplit), ref)
    _check_bf16(_run(x, torch.bfloat16, nsplit), ref)


def test_flash_qhead_matches_reference_fixture(golden_dir):
    x = cases.flash_inputs("flash_qhead")
    ref = np.load(os.path.join(golden_dir, "flash_qhead.npz"))["out"]
    _check_f32(_run(x, torch.float32), ref)


def test_flash_edge_cases():
    x = cases.flash_inputs("flash_qhead")
    R = x["q"].shape[0]
    # a row with every index padded and every proxy skipped returns zeros
    x["sel"][3] = -1
    x["exp"][3] = -1
    x["log_n"][3] = -math.inf
    # out-of-range indices are pads
    x["exp"][5, :10] = 10 ** 6
    ref = _oracle(x)
    ref_pad = ref.copy()
    y = dict(x)
    y["exp"] = x["exp"].clone()
    y["exp"][5, :10] = -1
    assert np.allclose(_oracle(y), ref_pad)
    for ns in (1, 4):
        o = _run(x, torch.float32, ns)
        assert torch.all(o[3] == 0)
        _check_f32(o, ref)
    # nb = 0 disables the proxy stream
    _check_f32(_run(x, torch.float32, nb=0), _oracle(x, nb=0))
    assert R == 64


def test_flash_strided_cache():
    """k/v as a view of a larger cache (stride(0) > K * D), as C.K[l].view(-1, Lmax, D)[..., :K] gives."""
    x = cases.flash_inputs("flash_kvhead")
    BH, K, _ = x["k"].shape
    big_k = torch.zeros(BH, K + 64, D, dtype=torch.bfloat16)
    big_v = torch.zeros(BH, K + 64, D, dtype=torch.bfloat16)
    big_k[:, :K], big_v[:, :K] = x["k"], x["v"]
    o = _run(x, torch.float32, k=big_k.cuda()[:, :K], v=big_v.cuda()[:, :K])
    _check_f32(o, _oracle(x))


def test_flash_repeatable():
    """Two launches give bitwise identical outputs (split merge in fixed chunk order)."""
    x = cases.flash_inputs("flash_qhead")
    a = _run(x, torch.float32, 8)
    b = _run(x, torch.float32, 8)
    assert torch.equal(a, b)
