"""CPU: the oracle against the reference's own outputs (golden vectors made by
tests/golden/make_golden.py from fast_triton_attn.FusedAttentionFunction)."""
import math
import os

import numpy as np
import pytest
import torch

from oracle.eager import (GRAD_NAMES, block_fwd_bwd, compare, cos_sim, make_inputs, rotary,
                          swap_even_odd, yarn_tables)

CASES = ["c1", "n64", "n128"]


def load_golden(path):
    z = np.load(path)
    B, T, C, H, N, seed, T_max = (int(v) for v in z["shape"])
    inp = {k[3:]: torch.from_numpy(z[k].view(np.int16)).view(torch.bfloat16).float()
           for k in z.files if k.startswith("in_")}
    want = {k: torch.from_numpy(z[k]) for k in ["y", *GRAD_NAMES]}
    return (B, T, C, H, N, seed, T_max), inp, want


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_golden(case, golden_dir):
    (B, T, C, H, N, seed, T_max), inp, want = load_golden(os.path.join(golden_dir, f"golden_{case}.npz"))
    got = block_fwd_bwd(inp, H, N)
    res = compare(got, want, ["y", *GRAD_NAMES])
    # The reference rounds to bf16 at its kernels' casts; the oracle is fp32 throughout.
    for name, r in res.items():
        assert r["cos"] > 0.9999, (name, r)
        assert r["max_rel"] < 3e-2, (name, r)


@pytest.mark.parametrize("case", CASES)
def test_golden_inputs_are_reproducible(case, golden_dir):
    (B, T, C, H, N, seed, T_max), inp, _ = load_golden(os.path.join(golden_dir, f"golden_{case}.npz"))
    again = make_inputs(B, T, C, H, N, seed=seed, T_max=T_max)
    for k, v in inp.items():
        assert torch.equal(v, again[k]), k


def test_golden_factor_grads_zero_beyond_T(golden_dir):
    (B, T, C, H, N, seed, T_max), _, want = load_golden(os.path.join(golden_dir, "golden_n64.npz"))
    assert T_max > T
    assert torch.count_nonzero(want["df1"][T:]) == 0 and torch.count_nonzero(want["df2"][T:]) == 0


def test_rotary_is_pairwise_rotation():
    f1, f2 = yarn_tables(8, 16)
    x = torch.randn(16, 8)
    y = rotary(x, f1, f2)
    # norms of every pair are preserved by an orthogonal table
    pn = lambda t: t.view(16, 4, 2).norm(dim=-1)
    assert torch.allclose(pn(x), pn(y), atol=1e-5)
    assert torch.equal(swap_even_odd(swap_even_odd(x)), x)


def test_oracle_fp32_vs_fp64():
    inp = make_inputs(1, 64, 64, 2, 32, seed=3)
    a = block_fwd_bwd(inp, 2, 32, dtype=torch.float32)
    b = block_fwd_bwd(inp, 2, 32, dtype=torch.float64)
    for k in ["y", *GRAD_NAMES]:
        assert cos_sim(a[k], b[k]) > 0.99999, k


def test_nonorthogonal_table_gradients_are_exact():
    """Autograd through the eager forward is exact for any table (finite differences)."""
    inp = make_inputs(1, 8, 16, 1, 8, seed=4, mscale=1.3, round_bf16=False)
    inp = {k: v.double() for k, v in inp.items()}
    out = block_fwd_bwd(inp, 1, 8, dtype=torch.float64)
    from oracle.eager import block_forward
    eps = 1e-6
    i, j = 3, 5
    xp = inp["x"].clone(); xp[0, i, j] += eps
    xm = inp["x"].clone(); xm[0, i, j] -= eps
    args = [inp[k] for k in ("wq", "wk", "wv", "wg", "wo", "f1", "f2")]
    fp = (block_forward(xp, *args, H=1, N=8) * inp["dy"]).sum()
    fm = (block_forward(xm, *args, H=1, N=8) * inp["dy"]).sum()
    assert math.isclose(float((fp - fm) / (2 * eps)), float(out["dx"][0, i, j]), rel_tol=1e-5, abs_tol=1e-8)
