"""GPU: the block against the reference's own GPU path, run unmodified on the
B200 (fast_triton_attn.fused_attn: its Triton kernels and ATen flash attention),
imported from baseline/_ref where the reference is installed; skipped when it is
not.

Both sides are bf16 pipelines that round at different points, so the bars are
those used against the reference's golden vectors: outputs max|a-b|/max|b| <=
3e-2 and every gradient cosine > 0.999.  Shapes keep C = H*N and unit-magnitude
rotary tables, where the reference's backward is exact (its rotated-frame norm
backward and table gradients assume an orthogonal table and C == H*N)."""
import os
import sys

import pytest
import torch

from gpu_util import DEV
from oracle.eager import GRAD_NAMES, make_inputs
from test_gpu_block import check, run_block

pytestmark = pytest.mark.gpu
REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _reference():
    if not os.path.exists(os.path.join(REF_DIR, "fast_triton_attn.py")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import fast_triton_attn

    return fast_triton_attn


class _Tables:
    def __init__(self, f1, f2):
        self.factor1, self.factor2 = f1, f2


def run_reference(ref, inp, H, N):
    x = inp["x"].to(device=DEV, dtype=torch.bfloat16).requires_grad_(True)
    lins = []
    for k in ("wq", "wk", "wv", "wg", "wo"):
        w = inp[k].to(device=DEV, dtype=torch.bfloat16)
        lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, device=DEV, dtype=torch.bfloat16)
        lin.weight = torch.nn.Parameter(w.contiguous())
        lins.append(lin)
    f1 = inp["f1"].to(device=DEV, dtype=torch.bfloat16).contiguous().requires_grad_(True)
    f2 = inp["f2"].to(device=DEV, dtype=torch.bfloat16).contiguous().requires_grad_(True)
    y = ref.fused_attn(x, *lins, _Tables(f1, f2), H, N)
    y.backward(inp["dy"].to(device=DEV, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    out = {"y": y.detach().float().cpu(), "dx": x.grad.float().cpu()}
    for name, lin in zip(GRAD_NAMES[1:6], lins):
        out[name] = lin.weight.grad.float().cpu()
    out["df1"], out["df2"] = f1.grad.float().cpu(), f2.grad.float().cpu()
    return out


@pytest.mark.parametrize("B,T,C,H,N", [(2, 256, 256, 4, 64), (1, 512, 512, 8, 64), (1, 256, 256, 2, 128)])
def test_block_matches_reference_triton_on_gpu(B, T, C, H, N):
    ref = _reference()
    inp = make_inputs(B, T, C, H, N, seed=31)
    want = run_reference(ref, inp, H, N)
    got = run_block(inp, H, N)
    check(got, want, ["y", *GRAD_NAMES], y_tol=3e-2)
