// Bandwidth-bound kernels of the block: the input RMSNorm forward and
// backward, the per-head q/k RMSNorm + rotary backward (with the optional
// rotary-table gradients), and an fp32 -> bf16 cast for the weight gradients.
// All are one pass over HBM with 16-byte vector accesses.
#include <cuda_bf16.h>

#include <algorithm>

#include "launch.h"
#include "ptx.cuh"

namespace mea {

// ---------------------------------------------------------------------------
// Input RMSNorm forward: xn = bf16(x * r), r = rsqrt(mean(x^2) + eps).
// One warp per row (fast_triton_attn.py:12-34 and the inv_rms store of
// :181-210).
// ---------------------------------------------------------------------------
__global__ void rmsnorm_fwd_kernel(int rows, int C, float eps, const __nv_bfloat16* __restrict__ x,
                                   __nv_bfloat16* __restrict__ xn, float* __restrict__ rout) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const __nv_bfloat16* xr = x + size_t(warp) * C;
  float ss = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf16_lo(w[e]), b = bf16_hi(w[e]);
      ss = fmaf(a, a, fmaf(b, b, ss));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / float(C) + eps);
  if (rout && lane == 0) rout[warp] = r;
  if (!xn) return;
  __nv_bfloat16* yr = xn + size_t(warp) * C;
  for (int c = lane * 8; c < C; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = pack_bf16(bf16_lo(w[e]) * r, bf16_hi(w[e]) * r);
    st_global_v4(yr + c, o[0], o[1], o[2], o[3]);
  }
}

// The same for C = 256*V (V 16-byte pieces per lane and row): rows taken
// grid-stride two at a time, every piece of both rows loaded before any is
// used and kept in registers for the xn store, so x is read from HBM once
// with 32*V bytes per lane in flight.  Same arithmetic, in the same order, as
// rmsnorm_fwd_kernel.
template <int V>
__global__ void __launch_bounds__(256) rmsnorm_fwd_rows_kernel(int rows, float eps, const __nv_bfloat16* __restrict__ x,
                                                               __nv_bfloat16* __restrict__ xn, float* __restrict__ rout) {
  constexpr int C = 256 * V;
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int row0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row0 < rows; row0 += 2 * nw) {
    const int row1 = row0 + nw;
    const bool two = row1 < rows;
    uint4 v[2][V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[0][i] = __ldg(reinterpret_cast<const uint4*>(x + size_t(row0) * C + 256 * i + lane * 8));
    if (two) {
#pragma unroll
      for (int i = 0; i < V; ++i)
        v[1][i] = __ldg(reinterpret_cast<const uint4*>(x + size_t(row1) * C + 256 * i + lane * 8));
    }
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const uint32_t w[4] = {v[q][i].x, v[q][i].y, v[q][i].z, v[q][i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16_lo(w[e]), b = bf16_hi(w[e]);
          ss[q] = fmaf(a, a, fmaf(b, b, ss[q]));
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], o);
      ss[1] += __shfl_xor_sync(0xffffffffu, ss[1], o);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (q == 1 && !two) break;
      const int row = q ? row1 : row0;
      const float r = rsqrtf(ss[q] / float(C) + eps);
      if (rout && lane == 0) rout[row] = r;
      if (!xn) continue;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const uint32_t w[4] = {v[q][i].x, v[q][i].y, v[q][i].z, v[q][i].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = pack_bf16(bf16_lo(w[e]) * r, bf16_hi(w[e]) * r);
        st_global_v4(xn + size_t(row) * C + 256 * i + lane * 8, o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Input RMSNorm backward (fast_triton_attn.py:663-669):
//   dx = r * (g - xn * sum(g * xn) / C),  xn = bf16(x * r), g = d xn.
// With `prescaled` the incoming rows are g' = r * g (the row scale applied
// where g was produced), and the same identity reads
//   dx = g' - xn * sum(g' * xn) / C.
// ---------------------------------------------------------------------------
__global__ void rmsnorm_bwd_kernel(int rows, int C, const __nv_bfloat16* __restrict__ dxn,
                                   const __nv_bfloat16* __restrict__ x, const float* __restrict__ rin,
                                   __nv_bfloat16* __restrict__ dx, bool prescaled) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const size_t off = size_t(warp) * C;
  const float r = rin[warp];
  const float s = prescaled ? 1.0f : r;  // factor on the output
  float dot = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
    const uint4 gv = *reinterpret_cast<const uint4*>(dxn + off + c);
    const uint4 xv = *reinterpret_cast<const uint4*>(x + off + c);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dot = fmaf(bf16_lo(gw[e]), round_bf16(bf16_lo(xw[e]) * r), dot);
      dot = fmaf(bf16_hi(gw[e]), round_bf16(bf16_hi(xw[e]) * r), dot);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  const float k = dot / float(C);
  for (int c = lane * 8; c < C; c += 256) {
    const uint4 gv = *reinterpret_cast<const uint4*>(dxn + off + c);
    const uint4 xv = *reinterpret_cast<const uint4*>(x + off + c);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float n0 = round_bf16(bf16_lo(xw[e]) * r), n1 = round_bf16(bf16_hi(xw[e]) * r);
      o[e] = pack_bf16(s * (bf16_lo(gw[e]) - n0 * k), s * (bf16_hi(gw[e]) - n1 * k));
    }
    st_global_v4(dx + off + c, o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// Per-head q/k RMSNorm + rotary backward, exact for any rotary table.
//
// Forward (per pair i of row (b,h,t)): qn = acc * r, q_rot = R_t qn with
//   R_t = [[f1[2i], f2[2i]], [f2[2i+1], f1[2i+1]]]   (fast_triton_attn.py:140).
// Backward from d q_rot:
//   dqn  = R_t^T dq_rot                                (inverse rotary, :614-619)
//   dot  = sum(dqn * qn) = sum(dq_rot * q_rot)          (holds for any R_t)
//   dacc = r * (dqn - qn * dot / N)                     (norm backward, :603-612)
// qn is recovered from the stored bf16 q_rot through R_t^{-1}; pairs with a
// singular 2x2 block contribute qn = 0 there.  The reference applies the norm
// backward in the rotated frame, which equals this only for orthogonal R_t.
// Table gradients (:622-639), exact form:
//   df1[t,n] += dq_rot[n] * qn[n],  df2[t,n] += dq_rot[n] * qn[n^1]  over (b,h), q and k.
// rq / rk are the factors from the projection accumulator row to qn: the q/k
// inverse RMS, times the input RMSNorm's r when the projection read x (the
// block backward), which puts r into dacc as the weight and input gradients
// then need.
//
// Grid: x = position t, y = chunk of the B*H rows; each block loops over its
// (b,h) rows at fixed t so the table gradients reduce in registers and leave
// the block with one atomic per (t, n).  Each thread owns 8 consecutive
// elements (4 pairs) of a row: 16-byte loads of q, k, dk and two of dq, and the
// loads of U rows are issued before any of them is used.
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) qk_bwd_kernel(int BH, int H, int T, int bh_per_block,
                                                     const float* __restrict__ dq_acc,
                                                     const __nv_bfloat16* __restrict__ dk,
                                                     const __nv_bfloat16* q_rot, const __nv_bfloat16* k_rot,
                                                     const float* __restrict__ rq, const float* __restrict__ rk,
                                                     const __nv_bfloat16* __restrict__ f1,
                                                     const __nv_bfloat16* __restrict__ f2, long long ldf,
                                                     __nv_bfloat16* out_q, __nv_bfloat16* out_k, long long o_sb,
                                                     long long o_sh, long long o_st,
                                                     float* __restrict__ df1, float* __restrict__ df2) {
  constexpr int EPT = 8;             // elements per thread
  constexpr int TPR = HD / EPT;      // threads per row (4, 8, 16)
  constexpr int RPB = 256 / TPR;     // rows per pass of the block
  constexpr int U = 2;               // passes whose loads are in flight together
  const int t = blockIdx.x;
  const int sub = threadIdx.x % TPR;
  const int grp = threadIdx.x / TPR;
  const int n0 = sub * EPT;

  // This position's table entries for our 4 pairs, and each pair's inverse (recovers qn from q_rot).
  float tf1[EPT], tf2[EPT], inv[EPT / 2];
  {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(f1 + size_t(t) * ldf + n0));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(f2 + size_t(t) * ldf + n0));
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tf1[2 * q] = bf16_lo(wa[q]);
      tf1[2 * q + 1] = bf16_hi(wa[q]);
      tf2[2 * q] = bf16_lo(wb[q]);
      tf2[2 * q + 1] = bf16_hi(wb[q]);
      const float det = tf1[2 * q] * tf1[2 * q + 1] - tf2[2 * q] * tf2[2 * q + 1];
      inv[q] = fabsf(det) > 1e-30f ? 1.0f / det : 0.f;
    }
  }
  float a1[EPT], a2[EPT];
#pragma unroll
  for (int e = 0; e < EPT; ++e) a1[e] = a2[e] = 0.f;

  const int bh_begin = blockIdx.y * bh_per_block;
  const int bh_end = min(bh_begin + bh_per_block, BH);
  // Trip count is uniform across the block so the row shuffles below always
  // see every lane; lanes past the end work on zeros and store nothing.
  for (int base = bh_begin; base < bh_end; base += U * RPB) {
    float4 gq[U][2];
    uint4 gk[U], yq[U], yk[U];
    float r_q[U], r_k[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int bh = base + u * RPB + grp;
      const size_t row = size_t(bh) * T + t;
      if (bh < bh_end) {
        const float4* dqp = reinterpret_cast<const float4*>(dq_acc + row * HD + n0);
        gq[u][0] = __ldg(dqp);
        gq[u][1] = __ldg(dqp + 1);
        gk[u] = __ldg(reinterpret_cast<const uint4*>(dk + row * HD + n0));
        // plain loads: the outputs may be q_rot / k_rot themselves
        yq[u] = *reinterpret_cast<const uint4*>(q_rot + row * HD + n0);
        yk[u] = *reinterpret_cast<const uint4*>(k_rot + row * HD + n0);
        r_q[u] = __ldg(rq + row);
        r_k[u] = __ldg(rk + row);
      } else {
        gq[u][0] = gq[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        gk[u] = yq[u] = yk[u] = make_uint4(0, 0, 0, 0);
        r_q[u] = r_k[u] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int bh = base + u * RPB + grp;
      const bool valid = bh < bh_end;
      const int b = valid ? bh / H : 0, h = valid ? bh - (bh / H) * H : 0;
      const size_t ooff = size_t(b) * o_sb + size_t(h) * o_sh + size_t(t) * o_st + n0;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float g[EPT], y[EPT];
        const uint4 yv = which == 0 ? yq[u] : yk[u];
        const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
        if (which == 0) {
          const float4 g0 = gq[u][0], g1 = gq[u][1];
          g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
          g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
        } else {
          const uint32_t gw[4] = {gk[u].x, gk[u].y, gk[u].z, gk[u].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            g[2 * q] = bf16_lo(gw[q]);
            g[2 * q + 1] = bf16_hi(gw[q]);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          y[2 * q] = bf16_lo(yw[q]);
          y[2 * q + 1] = bf16_hi(yw[q]);
        }
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) dot = fmaf(g[e], y[e], dot);
#pragma unroll
        for (int o = TPR / 2; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o, TPR);
        const float kk = dot / float(HD);
        const float r = which == 0 ? r_q[u] : r_k[u];
        uint32_t out[EPT / 2];
#pragma unroll
        for (int e = 0; e < EPT; e += 2) {
          const float fe1 = tf1[e], fo1 = tf1[e + 1], fe2 = tf2[e], fo2 = tf2[e + 1], iv = inv[e / 2];
          const float qa = (fo1 * y[e] - fe2 * y[e + 1]) * iv;
          const float qb = (fe1 * y[e + 1] - fo2 * y[e]) * iv;
          const float da = fe1 * g[e] + fo2 * g[e + 1];
          const float db = fe2 * g[e] + fo1 * g[e + 1];
          out[e / 2] = pack_bf16(r * (da - qa * kk), r * (db - qb * kk));
          a1[e] = fmaf(g[e], qa, a1[e]);
          a1[e + 1] = fmaf(g[e + 1], qb, a1[e + 1]);
          a2[e] = fmaf(g[e], qb, a2[e]);
          a2[e + 1] = fmaf(g[e + 1], qa, a2[e + 1]);
        }
        if (valid) st_global_v4((which == 0 ? out_q : out_k) + ooff, out[0], out[1], out[2], out[3]);
      }
    }
  }
  if (!df1) return;
  __shared__ float red[2][RPB][HD];
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    red[0][grp][n0 + e] = a1[e];
    red[1][grp][n0 + e] = a2[e];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * HD; i += blockDim.x) {
    const int w = i / HD, n = i % HD;
    float s = 0.f;
    for (int gI = 0; gI < RPB; ++gI) s += red[w][gI][n];
    atomicAdd((w == 0 ? df1 : df2) + size_t(t) * HD + n, s);
  }
}

__device__ __forceinline__ void cast4(long long i, long long n, const float* __restrict__ src,
                                      __nv_bfloat16* __restrict__ dst) {
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    *reinterpret_cast<uint2*>(dst + i) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
  } else {
    for (long long j = i; j < n; ++j) dst[j] = __float2bfloat16_rn(src[j]);
  }
}

__global__ void cast_f32_bf16_kernel(long long n, const float* __restrict__ src, __nv_bfloat16* __restrict__ dst) {
  cast4(((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4, n, src, dst);
}

// Up to kCastParts consecutive fp32 parts of n elements each (part y at src +
// y*n) into their own bf16 tensors in one launch (blockIdx.y = part; a NULL
// destination skips its part): the five weight gradients of the backward.
constexpr int kCastParts = 5;
struct CastParts {
  __nv_bfloat16* dst[kCastParts];
};
__global__ void cast_f32_bf16_parts_kernel(long long n, const float* __restrict__ src, const CastParts parts) {
  __nv_bfloat16* dst = parts.dst[blockIdx.y];
  if (!dst) return;
  cast4(((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4, n, src + (long long)blockIdx.y * n, dst);
}

// ---------------------------------------------------------------------------
// Upper bound on every scaled attention score, from the rotary tables.
//
// q and k reach the attention after the parameter-free per-head RMSNorm
// (||x_n||^2 = N ms / (ms + eps) < N) and the rotary x*f1 + swap(x)*f2, which
// maps each pair (x_2i, x_2i+1) through M = [[f1_2i, f2_2i], [f2_2i+1,
// f1_2i+1]].  Hence ||q_t|| <= sigma_max(t) sqrt(N) with sigma_max^2 the larger
// eigenvalue of M^T M, (F + sqrt(F^2 - 4 det^2)) / 2 with F = ||M||_F^2, and
// |q_t . k_s| * scale <= max_t sigma_max^2 * N / sqrt(N).  The bound (in log2
// units, with 1% + 0.05 of slack for the bf16 rounding of q and k) lets the
// attention forward use one fixed reference for exp2 instead of a running max.
// One CTA; every table row below T is read once.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float pair_sigma2(float a, float d, float b, float c) {
  const float fro = a * a + b * b + c * c + d * d;
  const float det = a * d - b * c;
  return 0.5f * (fro + sqrtf(fmaxf(fro * fro - 4.f * det * det, 0.f)));
}

// A grid of CTAs (256 threads) striding over the tables' 16-byte pieces (4
// rotary pairs of each table), every thread's loads issued before any is used.
// Each CTA maps its partial maximum through the bound's (increasing) formula
// and folds it into *out with an integer atomicMax: the bounds are positive, so
// integer order is float order, and the result equals the bound of the global
// maximum.  *out must be zero on entry.
__global__ void __launch_bounds__(256) rope_bound_kernel(int T, int HD, const __nv_bfloat16* __restrict__ f1,
                                                         const __nv_bfloat16* __restrict__ f2, long long ldf,
                                                         float* __restrict__ out) {
  __shared__ float red[8];
  const int per_row = HD / 8;  // 16-byte pieces per table row
  const int n = T * per_row;
  const int stride = gridDim.x * blockDim.x;
  float s2 = 0.f;
  constexpr int U = 4;
  for (int base = blockIdx.x * blockDim.x + threadIdx.x; base < n; base += U * stride) {
    uint4 a[U], b[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * stride;
      if (i < n) {
        const int t = i / per_row, e = (i - t * per_row) * 8;
        a[u] = __ldg(reinterpret_cast<const uint4*>(f1 + size_t(t) * ldf + e));
        b[u] = __ldg(reinterpret_cast<const uint4*>(f2 + size_t(t) * ldf + e));
      } else {
        a[u] = make_uint4(0, 0, 0, 0);
        b[u] = a[u];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t wa[4] = {a[u].x, a[u].y, a[u].z, a[u].w}, wb[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
      for (int q = 0; q < 4; ++q)  // pair (2i, 2i+1): f1 = (lo, hi) of wa[q], f2 = (lo, hi) of wb[q]
        s2 = fmaxf(s2, pair_sigma2(bf16_lo(wa[q]), bf16_hi(wa[q]), bf16_lo(wb[q]), bf16_hi(wb[q])));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s2 = fmaxf(s2, __shfl_xor_sync(0xffffffffu, s2, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s2;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0)
      atomicMax(reinterpret_cast<int*>(out), __float_as_int((m * sqrtf(float(HD)) * 1.4426950408889634f) * 1.01f + 0.05f));
  }
}

// ---------------------------------------------------------------------------
// Gate + repack (fast_triton_attn.py:146-176, :334-367):
//   gated[b, t, h*N + n] = O[b, h, t, n] * gs[b, h, t, n].
// Used by the backward when the forward kept O (no attention recompute).  One
// thread per 8 elements (16-byte loads and store); consecutive threads walk n,
// then t, so every warp reads and writes whole 16-byte-aligned row pieces.
// ---------------------------------------------------------------------------
__global__ void gate_repack_kernel(long long units, int H, int T, int N, const __nv_bfloat16* __restrict__ o,
                                   const __nv_bfloat16* __restrict__ gs, __nv_bfloat16* __restrict__ gated) {
  const int per_row = N / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < units;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / per_row;  // (b, h, t) row of O
    const int u = int(i - row * per_row);
    const int t = int(row % T);
    const long long bh = row / T;
    const int h = int(bh % H);
    const long long b = bh / H;
    const uint4 ov = __ldg(reinterpret_cast<const uint4*>(o) + i);
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gs) + i);
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t out[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      out[e] = pack_bf16(bf16_lo(ow[e]) * bf16_lo(gw[e]), bf16_hi(ow[e]) * bf16_hi(gw[e]));
    st_global_v4(gated + ((b * T + t) * H + h) * N + 8 * u, out[0], out[1], out[2], out[3]);
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
int run_gate_repack(int B, int H, int T, int HD, const void* o, const void* gs, void* gated, cudaStream_t st) {
  if (B <= 0 || H <= 0 || T <= 0 || HD % 8)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gate repack: bad shape (head dim %d must be a multiple of 8)", HD);
  if (!o || !gs || !gated ||
      (reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(gs) | reinterpret_cast<uintptr_t>(gated)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "gate repack: tensors must be non-NULL and 16-byte aligned");
  const long long units = (long long)B * H * T * (HD / 8);
  const int threads = 256;
  const long long want = (units + threads - 1) / threads;
  const int blocks = int(std::min<long long>(want, (long long)num_sms() * 8));
  gate_repack_kernel<<<blocks, threads, 0, st>>>(units, H, T, HD, static_cast<const __nv_bfloat16*>(o),
                                                 static_cast<const __nv_bfloat16*>(gs), static_cast<__nv_bfloat16*>(gated));
  return check_launch("gate_repack_kernel");
}

int run_rope_bound(int T, int HD, const void* f1, const void* f2, long long ldf, float* out, cudaStream_t st) {
  if (T <= 0 || HD % 8 || ldf % 8 || !f1 || !f2 || !out)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "rope bound: bad arguments");
  if ((reinterpret_cast<uintptr_t>(f1) | reinterpret_cast<uintptr_t>(f2)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "rope bound: tables must be 16-byte aligned");
  if (cudaMemsetAsync(out, 0, sizeof(float), st) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "rope bound: clearing the output failed");
  const int pieces = T * (HD / 8);
  const int blocks = std::max(1, std::min((pieces + 4 * 256 - 1) / (4 * 256), num_sms()));
  rope_bound_kernel<<<blocks, 256, 0, st>>>(T, HD, static_cast<const __nv_bfloat16*>(f1),
                                            static_cast<const __nv_bfloat16*>(f2), ldf, out);
  return check_launch("rope_bound_kernel");
}

template <int V>
static int rmsnorm_fwd_rows(int rows, float eps, const void* x, void* xn, float* r, cudaStream_t st) {
  const int threads = 256;
  static int resident = 0;  // CTAs per SM at this kernel's register count
  if (!resident) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, rmsnorm_fwd_rows_kernel<V>, threads, 0) != cudaSuccess || nb < 1)
      nb = 1;
    resident = nb;
  }
  const long long want = ((long long)rows + 15) / 16;  // 8 warps of two rows
  const int blocks = int(std::max<long long>(1, std::min<long long>(want, (long long)num_sms() * resident)));
  rmsnorm_fwd_rows_kernel<V><<<blocks, threads, 0, st>>>(rows, eps, static_cast<const __nv_bfloat16*>(x),
                                                         static_cast<__nv_bfloat16*>(xn), r);
  return check_launch("rmsnorm_fwd_rows_kernel");
}

int run_rmsnorm_fwd(int rows, int C, float eps, const void* x, void* xn, float* r, cudaStream_t st) {
  if (C % 8 || C <= 0 || rows <= 0) return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "rmsnorm: C=%d must be a multiple of 8", C);
  if (!x || (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(xn)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "rmsnorm: x (and xn) must be non-NULL and 16-byte aligned");
  switch (C) {
    case 256: return rmsnorm_fwd_rows<1>(rows, eps, x, xn, r, st);
    case 512: return rmsnorm_fwd_rows<2>(rows, eps, x, xn, r, st);
    case 768: return rmsnorm_fwd_rows<3>(rows, eps, x, xn, r, st);
    case 1024: return rmsnorm_fwd_rows<4>(rows, eps, x, xn, r, st);
    case 1536: return rmsnorm_fwd_rows<6>(rows, eps, x, xn, r, st);
    case 2048: return rmsnorm_fwd_rows<8>(rows, eps, x, xn, r, st);
    default: break;
  }
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  rmsnorm_fwd_kernel<<<blocks, threads, 0, st>>>(rows, C, eps, static_cast<const __nv_bfloat16*>(x),
                                                 static_cast<__nv_bfloat16*>(xn), r);
  return check_launch("rmsnorm_fwd_kernel");
}

int run_rmsnorm_bwd(int rows, int C, const void* dxn, const void* x, const float* r, void* dx, cudaStream_t st,
                    bool prescaled) {
  if (C % 8 || C <= 0 || rows <= 0) return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "rmsnorm bwd: C=%d must be a multiple of 8", C);
  if (!dxn || !x || !r || !dx ||
      (reinterpret_cast<uintptr_t>(dxn) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dx)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "rmsnorm bwd: dxn, x, dx must be non-NULL and 16-byte aligned");
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  rmsnorm_bwd_kernel<<<blocks, threads, 0, st>>>(rows, C, static_cast<const __nv_bfloat16*>(dxn),
                                                 static_cast<const __nv_bfloat16*>(x), r,
                                                 static_cast<__nv_bfloat16*>(dx), prescaled);
  return check_launch("rmsnorm_bwd_kernel");
}

// The q/k backward with its two outputs at out_q / out_k, element (b, h, t, n)
// at b*o_sb + h*o_sh + t*o_st + n.
static int qk_bwd_launch(int B, int H, int T, int HD, const float* dq_acc, const void* dk, const void* q_rot,
                         const void* k_rot, const float* rq, const float* rk, const void* f1, const void* f2,
                         long long ldf, void* out_q, void* out_k, long long o_sb, long long o_sh, long long o_st,
                         float* df1, float* df2, cudaStream_t st) {
  const int BH = B * H;
  // 2 passes x 256/(HD/8) rows per block iteration, 4 iterations per block at most
  const int rows_per_iter = 2 * 256 / (HD / 8);
  const int bh_per_block = BH < 4 * rows_per_iter ? BH : 4 * rows_per_iter;
  dim3 grid(T, (BH + bh_per_block - 1) / bh_per_block);
  if ((reinterpret_cast<uintptr_t>(dq_acc) | reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(q_rot) |
       reinterpret_cast<uintptr_t>(k_rot) | reinterpret_cast<uintptr_t>(f1) | reinterpret_cast<uintptr_t>(f2) |
       reinterpret_cast<uintptr_t>(out_q) | reinterpret_cast<uintptr_t>(out_k)) & 15 ||
      ldf % 8 || o_sb % 8 || o_sh % 8 || o_st % 8)
    return set_error(MEA_ERR_ALIGNMENT, "qk backward: operands must be 16-byte aligned");
  auto f1p = static_cast<const __nv_bfloat16*>(f1);
  auto f2p = static_cast<const __nv_bfloat16*>(f2);
  auto dkp = static_cast<const __nv_bfloat16*>(dk);
  auto qp = static_cast<const __nv_bfloat16*>(q_rot);
  auto kp = static_cast<const __nv_bfloat16*>(k_rot);
  auto oq = static_cast<__nv_bfloat16*>(out_q);
  auto ok = static_cast<__nv_bfloat16*>(out_k);
  switch (HD) {
    case 32:
      qk_bwd_kernel<32><<<grid, 256, 0, st>>>(BH, H, T, bh_per_block, dq_acc, dkp, qp, kp, rq, rk, f1p, f2p, ldf, oq,
                                              ok, o_sb, o_sh, o_st, df1, df2);
      break;
    case 64:
      qk_bwd_kernel<64><<<grid, 256, 0, st>>>(BH, H, T, bh_per_block, dq_acc, dkp, qp, kp, rq, rk, f1p, f2p, ldf, oq,
                                              ok, o_sb, o_sh, o_st, df1, df2);
      break;
    case 128:
      qk_bwd_kernel<128><<<grid, 256, 0, st>>>(BH, H, T, bh_per_block, dq_acc, dkp, qp, kp, rq, rk, f1p, f2p, ldf, oq,
                                               ok, o_sb, o_sh, o_st, df1, df2);
      break;
    default:
      return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "qk backward: head dim %d not in {32, 64, 128}", HD);
  }
  return check_launch("qk_bwd_kernel");
}

int run_qk_norm_rope_bwd(int B, int H, int T, int HD, const float* dq_acc, const void* dk, const void* q_rot,
                         const void* k_rot, const float* rq, const float* rk, const void* f1, const void* f2,
                         long long ldf, void* dacc, long long ld_dacc, float* df1, float* df2, cudaStream_t st) {
  // q part of row (b, t) at dacc + (b*T + t)*ld_dacc + h*HD, k part H*HD further on
  char* base = static_cast<char*>(dacc);
  return qk_bwd_launch(B, H, T, HD, dq_acc, dk, q_rot, k_rot, rq, rk, f1, f2, ldf, dacc,
                       base + size_t(H) * HD * 2, (long long)T * ld_dacc, HD, ld_dacc, df1, df2, st);
}

int run_qk_norm_rope_bwd_inplace(int B, int H, int T, int HD, const float* dq_acc, const void* dk, void* q_rot,
                                 void* k_rot, const float* rq, const float* rk, const void* f1, const void* f2,
                                 long long ldf, float* df1, float* df2, cudaStream_t st) {
  return qk_bwd_launch(B, H, T, HD, dq_acc, dk, q_rot, k_rot, rq, rk, f1, f2, ldf, q_rot, k_rot,
                       (long long)H * T * HD, (long long)T * HD, HD, df1, df2, st);
}

int run_cast_f32_bf16_parts(long long n, const float* src, void* const* dst, int parts, cudaStream_t st) {
  if (parts < 1 || parts > kCastParts)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "cast: %d parts (1..%d)", parts, kCastParts);
  if (n <= 0) return MEA_OK;
  CastParts cp{};
  bool any = false;
  for (int i = 0; i < parts; ++i) {
    cp.dst[i] = static_cast<__nv_bfloat16*>(dst[i]);
    any |= dst[i] != nullptr;
    if (reinterpret_cast<uintptr_t>(dst[i]) & 7)
      return set_error(MEA_ERR_ALIGNMENT, "cast: bf16 output %d must be 8-byte aligned", i);
  }
  if (any && ((reinterpret_cast<uintptr_t>(src) & 15) || n % 4))
    return set_error(MEA_ERR_ALIGNMENT, "cast: fp32 parts must be 16-byte aligned with n %% 4 == 0");
  if (!any) return MEA_OK;
  const long long threads = 256;
  const long long blocks = (n / 4 + threads) / threads;
  cast_f32_bf16_parts_kernel<<<dim3(unsigned(blocks), unsigned(parts)), unsigned(threads), 0, st>>>(n, src, cp);
  return check_launch("cast_f32_bf16_parts_kernel");
}

int run_cast_f32_bf16(long long n, const float* src, void* dst, cudaStream_t st) {
  if (n <= 0) return MEA_OK;
  if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 7))
    return set_error(MEA_ERR_ALIGNMENT, "cast: src must be 16-byte and dst 8-byte aligned");
  const long long threads = 256;
  const long long blocks = (n / 4 + threads) / threads;
  cast_f32_bf16_kernel<<<unsigned(blocks), unsigned(threads), 0, st>>>(n, src, static_cast<__nv_bfloat16*>(dst));
  return check_launch("cast_f32_bf16_kernel");
}

}  // namespace mea
