"""Shared test plumbing: move oracle state (numpy) to GPU state (torch) and back."""
import numpy as np
import torch

import oracle as O

INT_KEYS = ("codes", "asg", "mem", "cstart", "clen", "reclist", "reccnt")


def to_gpu_state(st_np, dev="cuda"):
    from openattention_b200 import selection as S
    B, _, Lmax, _ = st_np["codes"].shape
    C = st_np["nb"].shape[-1]
    st = S.new_state(B, Lmax, C, dev, st_np["reclist"].shape[-1])
    for k, v in st_np.items():
        if k == "W":
            st[k].copy_(O.from_bits(v).to(dev))
        else:
            st[k].copy_(torch.from_numpy(np.ascontiguousarray(v)).to(dev))
    return st


def to_np(t):
    if t.dtype == torch.bfloat16:
        return O.bits(t)
    return t.detach().cpu().numpy()


def state_from_fixture(x, z):
    """Oracle state = the reference's post-build state (the fixture), sums restated from its assignments."""
    B, n0, Lmax = x["B"], x["n0"], x["Lmax"]
    C = int(z["C"])
    st = O.new_state(B, Lmax, C)
    st["U"][:] = z["U"]
    st["scale"][:] = z["scale"].reshape(B, 8, 32)
    st["codes"][:, :, :n0] = z["codes"][:, :, :n0]
    st["W"][:] = z["W"]
    st["colmean"][:] = z["colmean"].reshape(B, 32, 16)
    st["cent"][:] = z["cent"]
    st["asg"][:, :, :n0] = z["asg"]
    st["nb"][:] = z["nb"]
    K, V = O.bits(x["K"]).copy(), O.bits(x["V"]).copy()
    for b in range(B):
        mem, cs, cl, Sk, Sk2, Sv = O.csr_sums(K[b], V[b], st["asg"][b], n0, C)
        st["Sk"][b], st["Sk2"][b], st["Sv"][b] = Sk, Sk2, Sv
        st["mem"][b], st["cstart"][b], st["clen"][b] = mem, cs, cl
    return st, K, V
