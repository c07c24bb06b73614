"""Generate golden vectors from the reference's own ``FusedAttentionFunction``.

Run where the reference source is available (read-only is fine), naming the
directory that holds its fast_triton_attn.py:

    python tests/golden/make_golden.py --ref <reference checkout>

The reference (fast_triton_attn.py) is imported unmodified and run on the CPU
under the Triton interpreter (TRITON_INTERPRET=1).  Two things make that work:

* The two ATen flash-attention ops it calls (fast_triton_attn.py:438 and :587)
  have no CPU kernel; they are redirected, through a stand-in for the module's
  ``torch`` global, to ATen's ``_scaled_dot_product_flash_attention_for_cpu``
  and ``..._for_cpu_backward`` (same math, same outputs O and logsumexp).
* Triton 3.6's interpreter mis-computes bf16 ``tl.dot`` and bf16 x bf16
  elementwise products, so the reference is run with fp32 tensors.  Its kernels
  still round to bf16 at every explicit ``.to(tl.bfloat16)`` site
  (fast_triton_attn.py:32, :103, :106, :108, :123), so the fixtures hold the
  reference's algorithm with fp32 storage in between.

Inputs are bf16-representable (``oracle.eager.make_inputs(round_bf16=True)``)
and are stored as bf16 bit patterns; outputs are stored as fp32.  Nothing on
the GPU box reads the reference: the tests read only the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.eager import make_inputs  # noqa: E402

# name -> (B, T, C, H, N, seed, T_max)
CASES = {
    "c1": (2, 256, 128, 4, 32, 0, 256),       # BASELINE config 1, head dim 32
    "n64": (1, 256, 128, 2, 64, 1, 320),      # head dim 64, factor table longer than T
    "n128": (1, 256, 256, 2, 128, 2, 256),    # head dim 128
}


def _load_reference(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import fast_triton_attn as fta  # the reference, unmodified

    aten = torch.ops.aten

    def flash_fwd(q, k, v, dropout_p=0.0, is_causal=False, return_debug_mask=False, scale=None):
        o, lse = aten._scaled_dot_product_flash_attention_for_cpu(q, k, v, dropout_p, is_causal, scale=scale)
        return o, lse, None, None, q.shape[2], k.shape[2], None, None, None

    def flash_bwd(do, q, k, v, o, lse, cq, ck, mq, mk, dropout_p=0.0, is_causal=False,
                  philox_seed=None, philox_offset=None, scale=None):
        return aten._scaled_dot_product_flash_attention_for_cpu_backward(
            do, q, k, v, o, lse, dropout_p, is_causal, scale=scale)

    class _Aten:
        def __getattr__(self, name):
            if name == "_scaled_dot_product_flash_attention":
                return flash_fwd
            if name == "_scaled_dot_product_flash_attention_backward":
                return flash_bwd
            return getattr(aten, name)

    class _Ops:
        aten = _Aten()

        def __getattr__(self, name):
            return getattr(torch.ops, name)

    class _Torch:
        ops = _Ops()

        def __getattr__(self, name):
            return getattr(torch, name)

    fta.torch = _Torch()
    return fta


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def run_case(fta, name, B, T, C, H, N, seed, T_max):
    inp = make_inputs(B, T, C, H, N, seed=seed, T_max=T_max)
    leaves = [inp[k].clone().requires_grad_(True) for k in ("x", "wq", "wk", "wv", "wg", "wo", "f1", "f2")]
    t0 = time.time()
    y = fta.FusedAttentionFunction.apply(*leaves, H, N, 1e-6)
    y.backward(inp["dy"])
    dt = time.time() - t0
    out = {f"in_{k}": _bf16_bits(v) for k, v in inp.items()}
    out["y"] = y.detach().numpy()
    for gname, leaf in zip(("dx", "dwq", "dwk", "dwv", "dwg", "dwo", "df1", "df2"), leaves):
        out[gname] = leaf.grad.detach().numpy()
    out["shape"] = np.array([B, T, C, H, N, seed, T_max], dtype=np.int64)
    path = os.path.join(HERE, f"golden_{name}.npz")
    np.savez_compressed(path, **out)
    print(f"{name}: wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB, reference ran {dt:.1f} s)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="directory holding the reference's fast_triton_attn.py")
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    args = ap.parse_args()
    fta = _load_reference(args.ref)
    for name in args.cases:
        run_case(fta, name, *CASES[name])


if __name__ == "__main__":
    main()
