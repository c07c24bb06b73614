"""GPU: every libmea kernel through the C ABI against a plain PyTorch fp32
reference of the same op (bf16 inputs, fp32 math)."""
import math

import pytest
import torch

from gpu_util import DEV, P, bf16, call, cos, dims, maxrel, status, stream
from oracle.eager import swap_even_odd, yarn_tables

pytestmark = pytest.mark.gpu
EPS = 1e-6
LOG2E = 1.4426950408889634


def rnd(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(*shape, device=DEV, generator=g) * scale


def unit_rms(t):
    return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True))


def attn_ref(q, k, v):
    N, T = q.shape[-1], q.shape[-2]
    s = q @ k.transpose(-1, -2) / math.sqrt(N)
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return torch.softmax(s, -1) @ v, torch.logsumexp(s, -1)


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 1), (0, 1), (1, 0)])
@pytest.mark.parametrize("N", [384, 512])
@pytest.mark.parametrize("M", [256, 384])
def test_gemm_operand_layouts(a_mn, b_mn, N, M):
    """M = 384 leaves the last CTA pair half outside the matrix (zero-filled
    loads, clipped stores)."""
    K = 320
    A, B = bf16(rnd(M, K, seed=1)), bf16(rnd(N, K, seed=2))
    a_st = A.t().contiguous() if a_mn else A
    b_st = B.t().contiguous() if b_mn else B
    out = torch.empty(M, N, device=DEV)
    s = status()
    call("mea_gemm", M, N, K, P(a_st), M if a_mn else K, a_mn, P(b_st), N if b_mn else K, b_mn, P(out), N, 0, P(s),
         stream(), status_buf=s)
    ref = A.float() @ B.float().t()
    assert maxrel(out, ref) < 1e-3


def test_gemm_split_k_accumulate():
    M, N, K = 256, 512, 8192
    A, B = bf16(rnd(M, K, seed=3)), bf16(rnd(N, K, seed=4))
    out = torch.zeros(M, N, device=DEV)
    s = status()
    call("mea_gemm", M, N, K, P(A.t().contiguous()), M, 1, P(B.t().contiguous()), N, 1, P(out), N, 1, P(s), stream(),
         status_buf=s)
    assert maxrel(out, A.float() @ B.float().t()) < 1e-3


# ------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("rows,C", [(512, 384), (512, 256), (4097, 512), (3001, 768), (515, 1024), (333, 2048)])
def test_rmsnorm_forward(rows, C):
    # C = 384: the one-row-per-warp loop; the others: the row-batched kernel (odd row counts leave the
    # last warp with one row)
    x = bf16(rnd(rows, C, scale=3.0, seed=5))
    xn = torch.empty_like(x)
    r = torch.empty(rows, device=DEV)
    call("mea_rmsnorm_forward", rows, C, EPS, P(x), P(xn), P(r), stream())
    rr = torch.rsqrt(x.float().pow(2).mean(-1) + EPS)
    assert maxrel(r, rr) < 1e-5
    assert maxrel(xn.float(), x.float() * rr[:, None]) < 8e-3
    assert torch.equal(xn, (x.float() * r[:, None]).to(torch.bfloat16))
    r_only = torch.full((rows,), float("nan"), device=DEV)
    call("mea_rmsnorm_forward", rows, C, EPS, P(x), None, P(r_only), stream())
    assert torch.equal(r_only, r)  # the forward (r only) and the recompute (r and x_n) agree bit for bit


def test_rmsnorm_backward():
    rows, C = 512, 384
    x = bf16(rnd(rows, C, scale=2.0, seed=6))
    g = bf16(rnd(rows, C, seed=7))
    r = torch.rsqrt(x.float().pow(2).mean(-1) + EPS).contiguous()
    dx = torch.empty_like(x)
    call("mea_rmsnorm_backward", rows, C, P(g), P(x), P(r), P(dx), stream())
    xf = x.float().requires_grad_(True)
    (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)).backward(g.float())
    assert cos(dx, xf.grad) > 0.9995 and maxrel(dx.float(), xf.grad) < 2e-2


# ------------------------------------------------------------------ projections
@pytest.mark.parametrize("H,N", [(4, 32), (2, 64), (1, 128), (4, 64)])
@pytest.mark.parametrize("B,T", [(2, 256), (3, 128)])
def test_qkvg_forward(H, N, B, T):
    C = 128
    HN = H * N
    xn = bf16(rnd(B * T, C, seed=8))
    W = [bf16(rnd(HN, C, scale=0.08, seed=9 + i)) for i in range(4)]
    f1, f2 = (bf16(t) for t in yarn_tables(N, T))
    q, k, v, gs = (torch.empty(B, H, T, N, dtype=torch.bfloat16, device=DEV) for _ in range(4))
    rq, rk = (torch.empty(B, H, T, device=DEV) for _ in range(2))
    s = status()
    call("mea_qkvg_forward", dims(B, T, C, H, N), P(xn), *[P(w) for w in W], P(f1), P(f2), P(q), P(k), P(v), P(gs),
         P(rq), P(rk), P(s), stream(), status_buf=s)
    acc = [(xn.float() @ w.float().t()).view(B, T, H, N).transpose(1, 2) for w in W]
    for a, out, r in ((acc[0], q, rq), (acc[1], k, rk)):
        rr = torch.rsqrt(a.pow(2).mean(-1) + EPS)
        qn = (a * rr[..., None]).bfloat16().float()
        want = qn * f1.float()[:T] + swap_even_odd(qn) * f2.float()[:T]
        assert maxrel(r, rr) < 1e-4
        assert maxrel(out.float(), want) < 1e-2
    assert maxrel(v.float(), acc[2]) < 1e-2
    assert maxrel(gs.float(), torch.sigmoid(acc[3])) < 1e-2


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("N", [32, 64, 128])
@pytest.mark.parametrize("B,H,T", [(2, 2, 128), (2, 2, 384), (40, 8, 1152), (64, 8, 640)])
@pytest.mark.parametrize("mag", [1.0, 3.0])
def test_attention_forward(N, B, H, T, mag):
    """Small grids (one work item per CTA) and grids with several work items per
    persistent CTA: 40*8 heads x 5 pairs and 64*8 heads x 3 pairs (odd tile
    counts, so one item of each head pairs with itself)."""
    q = bf16(unit_rms(rnd(B, H, T, N, seed=20)) * mag)
    k = bf16(unit_rms(rnd(B, H, T, N, seed=21)) * mag)
    v = bf16(rnd(B, H, T, N, seed=22))
    gs = bf16(torch.sigmoid(rnd(B, H, T, N, seed=23)))
    gated = torch.empty(B, T, H * N, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(B, H, T, device=DEV)
    o = torch.empty(B, H, T, N, dtype=torch.bfloat16, device=DEV)
    s = status()
    call("mea_attention_forward", B, H, T, N, P(q), P(k), P(v), P(gs), P(gated), P(lse), P(o), P(s), stream(),
         status_buf=s)
    O, L = attn_ref(q.float(), k.float(), v.float())
    assert maxrel(o.float(), O) < 2e-2, "attention output"
    assert (lse - L * LOG2E).abs().max().item() < 2e-3, "log-sum-exp (log2 units)"
    want = (O * gs.float()).transpose(1, 2).reshape(B, T, H * N)
    assert maxrel(gated.float(), want) < 2e-2, "gated output"


@pytest.mark.parametrize("B,H,T,N", [(2, 2, T, N) for N in (32, 64, 128) for T in (128, 384)]
                         + [(32, 8, 512, 64), (16, 4, 640, 128)])
def test_attention_backward(B, H, T, N):
    """The persistent backward walks pairs of key tiles (k, nq-1-k); the last two
    cases give every CTA several pairs of mixed lengths (K/V buffers reused
    across items, odd nq with a single middle tile)."""
    q = bf16(unit_rms(rnd(B, H, T, N, seed=30)))
    k = bf16(unit_rms(rnd(B, H, T, N, seed=31)))
    v = bf16(rnd(B, H, T, N, seed=32))
    dO = bf16(rnd(B, H, T, N, seed=33))
    ones = torch.ones_like(q)
    gated = torch.empty(B, T, H * N, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(B, H, T, device=DEV)
    o = torch.empty_like(q)
    s = status()
    call("mea_attention_forward", B, H, T, N, P(q), P(k), P(v), P(ones), P(gated), P(lse), P(o), P(s), stream(),
         status_buf=s)
    delta = (dO.float() * o.float()).sum(-1).contiguous()
    dq = torch.zeros(B, H, T, N, device=DEV)
    dk = torch.empty_like(q)
    dv = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=DEV)
    call("mea_attention_backward", B, H, T, N, P(q), P(k), P(v), P(dO), P(lse), P(delta), P(dq), P(dk), P(dv), H * N,
         P(s), stream(), status_buf=s)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    O, _ = attn_ref(qf, kf, vf)
    O.backward(dO.float())
    for name, got, want in (("dq", dq, qf.grad), ("dk", dk.float(), kf.grad), ("dv", dv.float().transpose(1, 2), vf.grad)):
        assert cos(got, want) > 0.999, name
        assert maxrel(got, want) < 3e-2, name


@pytest.mark.parametrize("H,N", [(2, 64), (4, 32), (2, 128)])
@pytest.mark.parametrize("B,T", [(2, 256), (3, 128)])
def test_gate_backward(H, N, B, T):
    C = 128
    HN = H * N
    dy = bf16(rnd(B * T, C, seed=40))
    wo = bf16(rnd(C, HN, scale=0.08, seed=41))
    o = bf16(rnd(B, H, T, N, seed=42))
    gs = bf16(torch.sigmoid(rnd(B, H, T, N, seed=43)))
    dO = torch.empty_like(o)
    dacc = torch.zeros(B * T, 4 * HN, dtype=torch.bfloat16, device=DEV)
    delta = torch.empty(B, H, T, device=DEV)
    s = status()
    call("mea_gate_backward", dims(B, T, C, H, N), P(dy), P(wo), P(o), P(gs), P(dO), P(dacc[:, 3 * HN:]), 4 * HN,
         P(delta), P(s), stream(), status_buf=s)
    dG = (dy.float() @ wo.float()).view(B, T, H, N).transpose(1, 2)
    g = gs.float()
    dO_ref = dG * g
    assert maxrel(dO.float(), dO_ref) < 1e-2
    dg_ref = (dG * o.float() * g * (1 - g)).transpose(1, 2).reshape(B * T, HN)
    assert maxrel(dacc[:, 3 * HN:].float(), dg_ref) < 1e-2
    assert torch.count_nonzero(dacc[:, :3 * HN]) == 0
    assert maxrel(delta, (dO_ref.bfloat16().float() * o.float()).sum(-1)) < 1e-3


@pytest.mark.parametrize("H,N", [(4, 32), (2, 64), (1, 128)])
@pytest.mark.parametrize("mscale", [1.0, 1.3])
def test_qk_norm_rope_backward(H, N, mscale):
    B, T = 2, 256
    HN = H * N
    f1, f2 = (bf16(t) for t in yarn_tables(N, T, mscale=mscale))
    accs = [rnd(B, H, T, N, scale=2.0, seed=50 + i) for i in range(2)]
    rots, rs = [], []
    for a in accs:
        r = torch.rsqrt(a.pow(2).mean(-1) + EPS)
        qn = (a * r[..., None]).bfloat16().float()
        rots.append(bf16(qn * f1.float() + swap_even_odd(qn) * f2.float()))
        rs.append(r.contiguous())
    dq = rnd(B, H, T, N, seed=60)
    dk = bf16(rnd(B, H, T, N, seed=61))
    dacc = torch.zeros(B * T, 4 * HN, dtype=torch.bfloat16, device=DEV)
    df1 = torch.zeros(T, N, device=DEV)
    df2 = torch.zeros(T, N, device=DEV)
    call("mea_qk_norm_rope_backward", dims(B, T, HN, H, N), P(dq), P(dk), P(rots[0]), P(rots[1]), P(rs[0]), P(rs[1]),
         P(f1), P(f2), P(dacc), 4 * HN, P(df1), P(df2), stream())
    F1 = f1.double().requires_grad_(True)
    F2 = f2.double().requires_grad_(True)
    grads = []
    for a, g in zip(accs, (dq.double(), dk.double())):
        A = a.double().requires_grad_(True)
        qn = A * torch.rsqrt(A.pow(2).mean(-1, keepdim=True) + EPS)
        (qn * F1 + swap_even_odd(qn) * F2).backward(g)
        grads.append(A.grad)
    for slot, want in enumerate(grads):
        got = dacc[:, slot * HN:(slot + 1) * HN].float().view(B, T, H, N).transpose(1, 2)
        assert cos(got, want) > 0.999 and maxrel(got, want) < 3e-2, slot
    assert cos(df1, F1.grad) > 0.999 and cos(df2, F2.grad) > 0.999


# ------------------------------------------------------------------ e4m3 GEMM
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (384, 128, 640), (1024, 512, 2048), (512, 768, 1024)])
@pytest.mark.parametrize("out_bf16", [0, 1])
def test_gemm_e4m3(M, N, K, out_bf16):
    """e4m3 operands (kind::f8f6f4 on CTA pairs) against torch's fp32 product of the
    same e4m3 values: the products are exact in fp32, so an fp32 output agrees to
    accumulation-order rounding and a bf16 output to its own rounding."""
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(N, K, device=DEV, generator=g).to(torch.float8_e4m3fn)
    out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16 if out_bf16 else torch.float32)
    s = status()
    call("mea_gemm_e4m3", M, N, K, P(a), K, P(b), K, P(out), N, out_bf16, P(s), stream(), status_buf=s)
    want = a.float() @ b.float().t()
    assert torch.isfinite(out.float()).all()
    assert maxrel(out.float(), want) < (1e-2 if out_bf16 else 1e-5)
