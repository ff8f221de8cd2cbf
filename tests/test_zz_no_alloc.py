"""The allocation-free flash entry point (oa_flash_qhead_proxies_noalloc) against oa_flash_qhead_proxies.

Both are called through the C ABI on the same inputs; the new entry point keeps its split-K scratch in
the library's own fixed array, the existing one gets a caller workspace.  Two calls in a row on one
stream, with different inputs and different split counts, check that the shared scratch carries
nothing from one call into the next.  Tolerance as the other flash tests: fp32 output within 2e-3
max-abs and 1e-3 relative-L2; bf16 output within one bf16 ulp per element."""
import pytest
import torch

import cases
from openattention_b200 import _lib
from openattention_b200 import flash as F

pytestmark = pytest.mark.gpu
MAX_ABS, REL_L2 = 2e-3, 1e-3
SCRATCH_LIMIT = 4 << 20


def _inputs(seed_shift):
    x = cases.flash_inputs("flash_qhead")
    if seed_shift:
        g = torch.Generator().manual_seed(seed_shift)
        x["q"] = torch.randn(x["q"].shape, generator=g).to(torch.bfloat16)
        x["exp"] = x["exp"].flip(1).contiguous()
        x["log_n"] = x["log_n"].flip(1).contiguous()
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def _noalloc(x, out_dtype, nsplit):
    q, k = x["q"], x["k"]
    BQ, BH, K = q.shape[0], k.shape[0], k.shape[1]
    kb = x["kbar"]
    NB = kb.shape[1]
    out = torch.empty(BQ, 128, dtype=out_dtype, device=q.device)
    code = _lib.OA_F32 if out_dtype == torch.float32 else _lib.OA_BF16
    _lib.call("oa_flash_qhead_proxies_noalloc", q.data_ptr(), q.stride(0), k.data_ptr(), x["v"].data_ptr(),
              k.stride(0), k.stride(1), x["sel"].data_ptr(), x["sel"].shape[1], x["exp"].data_ptr(),
              x["exp"].shape[1], kb.data_ptr(), x["vbar"].data_ptr(), kb.stride(0), kb.stride(1),
              x["log_n"].data_ptr(), x["log_n"].stride(0), out.data_ptr(), out.stride(0), code, BQ, BH, K, NB,
              float(F.SC), int(nsplit), torch.cuda.current_stream().cuda_stream)
    return out


def _existing(x, out_dtype, nsplit):
    return F.ours_flash(x["q"], x["k"], x["v"], x["sel"], x["exp"], x["kbar"], x["vbar"], x["log_n"],
                        out_dtype=out_dtype, nsplit=nsplit)


def _close(a, b, out_dtype):
    a, b = a.double().cpu(), b.double().cpu()
    if out_dtype == torch.float32:
        assert (a - b).abs().max().item() <= MAX_ABS
        assert torch.linalg.norm(a - b).item() <= REL_L2 * torch.linalg.norm(b).item()
    else:
        ulp = torch.maximum(b.abs(), torch.full_like(b, 2.0 ** -126)) * 2.0 ** -7
        assert bool(((a - b).abs() <= ulp * 1.01).all())


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("splits", [(8, 3), (0, 16), (1, 8)])
def test_noalloc_matches_existing_entry_two_calls(out_dtype, splits):
    xa, xb = _inputs(0), _inputs(5)
    # two calls in a row on one stream, no synchronisation between them
    oa_ = _noalloc(xa, out_dtype, splits[0])
    ob_ = _noalloc(xb, out_dtype, splits[1])
    torch.cuda.synchronize()
    ra = _existing(xa, out_dtype, splits[0])
    rb = _existing(xb, out_dtype, splits[1])
    torch.cuda.synchronize()
    _close(oa_, ra, out_dtype)
    _close(ob_, rb, out_dtype)
    assert not torch.equal(ra, rb)


def test_noalloc_rejects_split_beyond_scratch():
    """A split whose scratch exceeds the fixed array is refused with status 1 and a message.  Every
    buffer holds the BQ rows the call names (a few MB), so even a broken size check would only give a
    wrong answer, never an access outside them."""
    x = _inputs(0)
    BQ, BH = 4096, 16
    rep = BQ // x["q"].shape[0]
    q = x["q"].repeat(rep, 1).contiguous()
    sel = x["sel"].repeat(rep, 1).contiguous()
    ex = x["exp"].repeat(rep, 1).contiguous()
    ln = x["log_n"].repeat(rep, 1).contiguous()
    kb = x["kbar"].repeat(rep, 1, 1).contiguous()
    vb = x["vbar"].repeat(rep, 1, 1).contiguous()
    k = x["k"][:BH].contiguous()
    v = x["v"][:BH].contiguous()
    lib = _lib.load()
    need = lib.oa_flash_workspace_bytes(BQ, sel.shape[1], ex.shape[1], kb.shape[1], 64)
    assert need > SCRATCH_LIMIT
    out = torch.full((BQ, 128), 7.0, dtype=torch.float32, device=q.device)
    status = lib.oa_flash_qhead_proxies_noalloc(
        q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), sel.data_ptr(),
        sel.shape[1], ex.data_ptr(), ex.shape[1], kb.data_ptr(), vb.data_ptr(), kb.stride(0), kb.stride(1),
        ln.data_ptr(), ln.stride(0), out.data_ptr(), out.stride(0), _lib.OA_F32, BQ, BH, k.shape[1], kb.shape[1],
        float(F.SC), 64, torch.cuda.current_stream().cuda_stream)
    assert status == 1
    msg = lib.oa_last_error_string()
    assert b"scratch" in msg and b"oa_flash_qhead_proxies_noalloc" in msg
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()), "a rejected call must not write its output"


def test_noalloc_argument_error_names_the_entry_point():
    """An argument error found after the size check (BQ not a multiple of BH) is refused with status 1,
    its message names this entry point, and nothing is launched."""
    x = _inputs(0)
    q, k = x["q"], x["k"]
    BQ = q.shape[0]
    out = torch.full((BQ, 128), 7.0, dtype=torch.float32, device=q.device)
    lib = _lib.load()
    status = lib.oa_flash_qhead_proxies_noalloc(
        q.data_ptr(), q.stride(0), k.data_ptr(), x["v"].data_ptr(), k.stride(0), k.stride(1), x["sel"].data_ptr(),
        x["sel"].shape[1], x["exp"].data_ptr(), x["exp"].shape[1], x["kbar"].data_ptr(), x["vbar"].data_ptr(),
        x["kbar"].stride(0), x["kbar"].stride(1), x["log_n"].data_ptr(), x["log_n"].stride(0), out.data_ptr(),
        out.stride(0), _lib.OA_F32, BQ, 3, k.shape[1], x["kbar"].shape[1], float(F.SC), 4,
        torch.cuda.current_stream().cuda_stream)
    assert status == 1
    assert b"oa_flash_qhead_proxies_noalloc" in lib.oa_last_error_string()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
