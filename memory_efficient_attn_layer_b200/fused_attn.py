"""``fused_attn`` and its autograd function: the drop-in boundary.

Mirrors the reference's interface (fast_triton_attn.py:373-697): same names,
same argument order and meaning, same gradient tuple.  The work is done by
libmea.so (sm_100a kernels) through two calls, ``mea_block_forward`` and
``mea_block_backward``.  The forward keeps only x, the weights, the rotary
tables and the attention row log-sum-exp for the backward; everything else is
recomputed there (the reference additionally keeps the attention output,
fast_triton_attn.py:463-466).
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from . import dp as _dp

# Device timeouts are always reported: by default at the first call after the
# failing one whose asynchronous status copy has landed (no synchronisation);
# with MEA_CHECK_STATUS=1 at the failing call itself (one synchronisation per call).
_CHECK_STATUS = os.environ.get("MEA_CHECK_STATUS", "0") == "1"


def _dims(x: torch.Tensor, H: int, N: int, factor1: torch.Tensor, eps: float) -> _lib.MeaBlockDims:
    B, T, C = x.shape
    return _lib.MeaBlockDims(B, T, C, int(H), int(N), factor1.shape[0], float(eps))


def _check_inputs(x, weights, factor1, factor2, H, N):
    _lib.require_device(x.device)
    if x.dim() != 3:
        raise ValueError(f"x must be [B, T, C], got shape {tuple(x.shape)}")
    B, T, C = x.shape
    HN = H * N
    shapes = [(HN, C)] * 4 + [(C, HN)]
    for name, w, shp in zip(("q", "k", "v", "g", "o"), weights, shapes):
        if tuple(w.shape) != shp:
            raise ValueError(f"{name}_proj.weight must be {shp}, got {tuple(w.shape)}")
    for t in (x, *weights, factor1, factor2):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"fused_attn computes in bf16; got a {t.dtype} tensor")
        if t.device != x.device:
            raise ValueError("all tensors must be on the same device")
    if factor1.dim() != 2 or factor1.shape[1] != N or factor1.shape[0] < T or factor2.shape != factor1.shape:
        raise ValueError(f"rotary tables must be [T_max >= {T}, {N}], got {tuple(factor1.shape)} / "
                         f"{tuple(factor2.shape)}")


class FusedAttentionFunction(torch.autograd.Function):
    """Autograd node of the block (fast_triton_attn.py:373)."""

    @staticmethod
    def forward(ctx, x, q_weight, k_weight, v_weight, g_weight, o_weight, factor1, factor2, H, N, eps, save_o=False):
        """``save_o`` (no counterpart in the reference's signature; default off):
        also keep the attention output O [B,H,T,N] for the backward, as the
        reference does (fast_triton_attn.py:463-466), so the backward skips the
        attention recompute.  Off, only x, the weights, the tables and the row
        log-sum-exp are kept."""
        weights = [w.contiguous() for w in (q_weight, k_weight, v_weight, g_weight, o_weight)]
        x = x.contiguous()
        factor1 = factor1.contiguous()
        factor2 = factor2.contiguous()
        _check_inputs(x, weights, factor1, factor2, H, N)
        _lib.poll_status(x.device)  # a timeout of an earlier call whose status copy has landed
        B, T, C = x.shape
        L = _lib.lib()
        dims = _dims(x, H, N, factor1, eps)
        y = torch.empty_like(x)
        lse = torch.empty(B, H, T, dtype=torch.float32, device=x.device)
        ws_bytes = L.mea_forward_workspace_size(ctypes.byref(dims))
        if ws_bytes == 0:  # invalid dims: let the library say why
            _lib.check(L.mea_block_forward(ctypes.byref(dims), *([None] * 11), 0, None, None))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        status = _lib.status_buffer(x.device)
        head = (ctypes.byref(dims), _lib.ptr(x), *[_lib.ptr(w) for w in weights], _lib.ptr(factor1),
                _lib.ptr(factor2), _lib.ptr(y), _lib.ptr(lse))
        tail = (_lib.ptr(ws), ws_bytes, _lib.ptr(status), _lib.stream_ptr(x.device))
        o = None
        if save_o:
            o = torch.empty(B, H, T, N, dtype=torch.bfloat16, device=x.device)
            _lib.check(L.mea_block_forward_save_o(*head, _lib.ptr(o), *tail))
        else:
            _lib.check(L.mea_block_forward(*head, *tail))
        del ws
        if _CHECK_STATUS:
            _lib.read_status(x.device)
        else:
            _lib.note_status(x.device)
        ctx.save_o = o is not None
        ctx.save_for_backward(x, *weights, factor1, factor2, lse, *([o] if o is not None else []))
        ctx.H, ctx.N, ctx.eps = int(H), int(N), float(eps)
        ctx.exchange = _dp.active_exchange()
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, wq, wk, wv, wg, wo, factor1, factor2, lse = ctx.saved_tensors[:9]
        o = ctx.saved_tensors[9] if ctx.save_o else None
        H, N, eps = ctx.H, ctx.N, ctx.eps
        dy = grad_output.to(torch.bfloat16).contiguous()
        _lib.poll_status(x.device)
        L = _lib.lib()
        dims = _dims(x, H, N, factor1, eps)
        dx = torch.empty_like(x)
        want_df = ctx.needs_input_grad[6] or ctx.needs_input_grad[7]
        df1 = torch.empty(factor1.shape, dtype=torch.float32, device=x.device) if want_df else None
        df2 = torch.empty(factor2.shape, dtype=torch.float32, device=x.device) if want_df else None
        ws_bytes = L.mea_backward_workspace_size(ctypes.byref(dims))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        status = _lib.status_buffer(x.device)
        head = (ctypes.byref(dims), _lib.ptr(x), _lib.ptr(wq), _lib.ptr(wk), _lib.ptr(wv), _lib.ptr(wg),
                _lib.ptr(wo), _lib.ptr(factor1), _lib.ptr(factor2), _lib.ptr(lse))
        fn = L.mea_block_backward_ex
        if o is not None:  # the forward kept O: no attention recompute
            fn = L.mea_block_backward_from_o
            head = head + (_lib.ptr(o),)

        def call(dw_bf16, dw32, ev_dwo=None, ev_dw=None):
            _lib.check(fn(*head, _lib.ptr(dy), _lib.ptr(dx), *[_lib.ptr(d) for d in dw_bf16], _lib.ptr(df1),
                          _lib.ptr(df2), _lib.ptr(dw32), _lib.ptr(ws), ws_bytes, _lib.ptr(status),
                          _lib.stream_ptr(x.device), ev_dwo, ev_dw))

        sink = _dp.grad_sink_for((wq, wk, wv, wg, wo)) if all(ctx.needs_input_grad[1:6]) else None
        ex = ctx.exchange
        dws = None if sink is not None else [torch.empty_like(w) for w in (wq, wk, wv, wg, wo)]
        if sink is not None:
            # The sharded optimizer owns these weights: fp32 gradients go straight
            # into its buffer (added when it already holds this step's gradient).
            dst, fresh = sink
            out = dst if fresh else torch.empty_like(dst)
            call([None] * 5, out)
            if not fresh:
                dst.add_(out)
            dws = [None] * 5
        elif ex is None:
            call(dws, None)
        else:
            _exchange_backward(call, dws, x, ex)
        if _CHECK_STATUS:
            _lib.read_status(x.device)
        else:
            _lib.note_status(x.device)
        gf1 = df1.to(factor1.dtype) if want_df else None
        gf2 = df2.to(factor2.dtype) if want_df else None
        return (dx, *dws, gf1, gf2, None, None, None, None)


def _exchange_backward(call, dws, x, ex):
    """Backward whose fp32 weight gradients are all-reduced across the exchange's
    group on a side stream, each part from the moment the library marks it
    final; the bf16 gradients are written from the reduced buffer on that
    stream, and the caller's stream waits for it before anything after the
    backward runs."""
    main = torch.cuda.current_stream(x.device)
    side = _dp.side_stream(x.device)
    n_w = dws[0].numel()
    dw32 = torch.empty(5 * n_w, dtype=torch.float32, device=x.device)
    ev_dwo, ev_dw = torch.cuda.Event(), torch.cuda.Event()
    ev_dwo.record(main)  # creates the events; the library records them again at the right points
    ev_dw.record(main)
    call([None] * 5, dw32, ev_dwo._as_parameter_, ev_dw._as_parameter_)
    dw32.record_stream(side)
    for d in dws:
        d.record_stream(side)
    with torch.cuda.stream(side):
        side.wait_event(ev_dwo)
        _dp.reduce_weight_grads(dw32, 4 * n_w, ex.group, ex.average, before_qkvg=lambda: side.wait_event(ev_dw))
        for i, d in enumerate(dws):
            d.copy_(dw32[i * n_w:(i + 1) * n_w].view_as(d))
    if _exchange_waits is not None:
        reach, done = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reach.record(main)
        done.record(side)
        _exchange_waits.append((reach, done))
    main.wait_stream(side)


_exchange_waits = None


def record_exchange_waits(on: bool):
    """Instrument the overlapped gradient exchange: while on, every backward
    records when the caller's stream reaches the end of the backward and when
    the side stream's all-reduce finishes.  Turning it off returns, per
    backward, the milliseconds the caller's stream waited for the exchange
    (0 when the all-reduce was hidden under the rest of the backward)."""
    global _exchange_waits
    if on:
        _exchange_waits = []
        return None
    pairs, _exchange_waits = _exchange_waits or [], None
    out = []
    for reach, done in pairs:
        done.synchronize()
        out.append(max(0.0, reach.elapsed_time(done)))
    return out


def fused_attn(x, q_proj, k_proj, v_proj, g_proj, o_proj, yarn_module, H, N, eps=1e-6, save_o=False):
    """Gated causal attention block (fast_triton_attn.py:681-697).

    Reads ``.weight`` of the five bias-free ``nn.Linear`` projections and
    ``.factor1`` / ``.factor2`` of the rotary object, exactly as the reference.
    ``save_o`` (default off) keeps the attention output for the backward
    instead of recomputing it (see FusedAttentionFunction.forward).
    """
    return FusedAttentionFunction.apply(
        x, q_proj.weight, k_proj.weight, v_proj.weight, g_proj.weight, o_proj.weight,
        yarn_module.factor1, yarn_module.factor2, H, N, eps, save_o)
