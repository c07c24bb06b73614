// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M, N] = sum_k A[m, k] * B[n, k]      (bf16 operands, fp32 accumulate in TMEM)
//
// One CTA per SM walks a static list of 128 x BN output tiles (optionally split
// along K).  Warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
// warp 1 issues tcgen05.mma from one elected lane into one of two TMEM
// accumulators (double-buffered, so the epilogue of tile i overlaps the
// mainloop of tile i+1), and warps 2..5 run the epilogue (one TMEM lane = one
// output row per thread).  Operands may be K-major or MN-major in global
// memory; both are staged with 128-byte swizzle and described to the tensor
// core with the matching smem descriptor, so no transposes are ever written.
//
// Epilogues carry the block's elementwise work so it never makes its own pass
// over HBM:
//   EPI_QKVG  : per-head q/k RMSNorm + interleaved rotary, v copy, sigmoid(g),
//               scatter to [B, H, T, N]   (fast_triton_attn.py:102-144)
//   EPI_DGATE : gate backward (dO = dGated*g, dg_pre = dGated*O*g(1-g)) and
//               delta = rowsum(dO*O) for the attention backward
//               (fast_triton_attn.py:581-584, :601)
//   EPI_BF16 / EPI_F32 / EPI_RED_F32 : plain stores / split-K fp32 reduction.
#pragma once
#include <cuda.h>

#include "ptx.cuh"

namespace mea {

enum AMode : int { A_K = 0, A_MN = 1 };
enum BMode : int { B_K = 0, B_MN = 1, B_SLABS = 2, B_MN_KSPLIT4 = 3 };
enum EpiMode : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_RED_F32 = 2, EPI_QKVG = 3, EPI_DGATE = 4 };

struct GemmMaps {
  CUtensorMap a;
  CUtensorMap b[4];
};

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_splits, kb_per_split, kb_total;
  int b_kb_per_src;  // B_MN_KSPLIT4: k-blocks taken from each of the 4 B tensors
  int slab_rows;     // B_SLABS: rows of one slab (= head dim)
  int* status;
  // EPI_BF16 / EPI_F32 / EPI_RED_F32: D[m, n] -> out[m * ldo + n]
  void* out;
  long long ldo;
  // EPI_QKVG
  __nv_bfloat16 *q, *k, *v, *g;
  const __nv_bfloat16 *f1, *f2;
  long long ldf;
  float *rq, *rk;
  const float* row_scale;
  int T, H, hd;
  float eps;
  // EPI_DGATE
  const __nv_bfloat16 *o_in, *gs_in;
  __nv_bfloat16 *do_out, *dg_out;
  long long ld_dg;
  float* delta;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr uint32_t GEMM_A_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KB

// EPI_QKVG runs eight epilogue warps (two groups splitting the q/k/v/g slabs)
// that stage each slab in shared memory and copy it out with coalesced stores;
// the other epilogues run four warps storing straight from registers.  Shared
// memory: stage ring, then the staging tile, then the barriers.
template <int BN, int EPI>
struct GemmCfg {
  static constexpr bool QKVG = EPI == EPI_QKVG;
  static constexpr int EPI_WARPS = QKVG ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGES = QKVG ? 3 : (BN >= 256 ? 4 : 6);
  static constexpr uint32_t STAGING_BYTES = QKVG ? GEMM_BM * BN * 2 : 0;
  static constexpr uint32_t B_BYTES = BN * GEMM_BK * 2;
  static constexpr uint32_t STAGE_BYTES = GEMM_A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = 1024 + size_t(STAGES) * STAGE_BYTES + STAGING_BYTES + 256;
};

__device__ __forceinline__ void gemm_decode(const GemmParams& p, int BN, int t, int& m0, int& n0, int& kb0, int& kb1) {
  const int mn = p.m_tiles * p.n_tiles;
  const int split = t / mn;
  const int r = t - split * mn;
  const int mt = r / p.n_tiles;
  const int nt = r - mt * p.n_tiles;
  m0 = mt * GEMM_BM;
  n0 = nt * BN;
  kb0 = split * p.kb_per_split;
  kb1 = min(kb0 + p.kb_per_split, p.kb_total);
}

// ---------------------------------------------------------------------------
// Epilogues.  `taddr` is this warp's TMEM lane block + accumulator column 0;
// `m` the output row this thread owns.
// ---------------------------------------------------------------------------
template <int BN>
__device__ __forceinline__ void epi_store(const GemmParams& p, int mode, uint32_t taddr, int m, int n0) {
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_load32(taddr + c, r);
    if (mode == EPI_BF16) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(m) * p.ldo + n0 + c;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        st_global_v4(dst + 8 * j, pack_bf16(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1])),
                     pack_bf16(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3])),
                     pack_bf16(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5])),
                     pack_bf16(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7])));
    } else if (mode == EPI_F32) {
      float* dst = reinterpret_cast<float*>(p.out) + size_t(m) * p.ldo + n0 + c;
#pragma unroll
      for (int j = 0; j < 8; ++j) st_global_v4(dst + 4 * j, r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    } else {
      float* dst = reinterpret_cast<float*>(p.out) + size_t(m) * p.ldo + n0 + c;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        red_add_v4_f32(dst + 4 * j, __uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                       __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
    }
  }
}

// Staging tile of one slab: 128 rows of 2*HD bytes; 16-byte unit u of row r sits
// at u ^ (r & 7) within the row (u ^ (r & 3) for HD = 32), so that the row-per-
// thread writes and the unit-per-thread copy-out both spread over the banks.
template <int HD>
__device__ __forceinline__ uint32_t stage_addr(uint32_t slab, int r, int u) {
  constexpr int UPR = HD / 8;  // 16-byte units per row
  constexpr int MASK = UPR >= 8 ? 7 : UPR - 1;
  return slab + r * (HD * 2) + ((u ^ (r & MASK)) << 4);
}
template <int HD>
__device__ __forceinline__ void stage_unit(uint32_t slab, int r, int u, const uint32_t* w) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(stage_addr<HD>(slab, r, u)), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3])
               : "memory");
}
// Copy a staged slab (128 consecutive rows of one [B,H,T,N] output) to global
// memory: the group's 128 threads move consecutive 16-byte units.
template <int HD>
__device__ __forceinline__ void copy_out_slab(uint32_t slab, __nv_bfloat16* dst, int ti) {
  constexpr int UPR = HD / 8;
#pragma unroll 4
  for (int i = ti; i < 128 * UPR; i += 128) {
    const int r = i / UPR, u = i - (i / UPR) * UPR;
    uint32_t w0, w1, w2, w3;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                 : "r"(stage_addr<HD>(slab, r, u)) : "memory");
    st_global_v4(dst + size_t(i) * 8, w0, w1, w2, w3);
  }
}

// Rotary-table columns [c, c+32) of one table row, as four 16-byte pieces per table.
template <int HD>
__device__ __forceinline__ void load_tab_chunk(const __nv_bfloat16* f1row, const __nv_bfloat16* f2row, int c,
                                               uint4 (&t1)[4], uint4 (&t2)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    t1[j] = *reinterpret_cast<const uint4*>(f1row + c + 8 * j);
    t2[j] = *reinterpret_cast<const uint4*>(f2row + c + 8 * j);
  }
}

// q/k RMSNorm over the head dim, bf16 rounding of the normed value, then
// interleaved rotary out[n] = qn[n]*f1[t,n] + qn[n^1]*f2[t,n]
// (fast_triton_attn.py:102-106, :132-141); v stored as is (fast_triton_attn.py:108)
// and g as sigmoid(g) (fast_triton_attn.py:123).  One slab (q, k, v or g of one
// head) of this thread's row, written bf16 to its [B,H,T,N] output row in
// 32-column chunks; rotary-table rows are loaded one chunk ahead of their use.
// QK: q or k (per-head RMSNorm + rotary, with the rotary rows of chunks 0 and 1
// preloaded in t1/t2 and later chunks streamed one ahead); else v or sigmoid(g).
template <int HD, bool QK>
__device__ __forceinline__ void qkvg_slab(const GemmParams& p, uint32_t tcol, uint32_t slab, int r, int typ, float rs,
                                          size_t bht, const __nv_bfloat16* f1row, const __nv_bfloat16* f2row,
                                          uint4 (&t1)[2][4], uint4 (&t2)[2][4]) {
  constexpr int NCH = HD / 32;
  float sc = rs;
  if (QK) {
    float ss = 0.f;
#pragma unroll
    for (int ci = 0; ci < NCH; ++ci) {
      uint32_t v[32];
      tmem_load32(tcol + 32 * ci, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = __uint_as_float(v[j]) * rs;
        ss = fmaf(x, x, ss);
      }
    }
    const float inv = rsqrtf(ss / float(HD) + p.eps);
    float* rdst = typ == 0 ? p.rq : p.rk;
    if (rdst) rdst[bht] = inv;
    sc = rs * inv;
  }
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    const int c = 32 * ci;
    if (QK && ci >= 1 && ci + 1 < NCH) load_tab_chunk<HD>(f1row, f2row, c + 32, t1[(ci + 1) & 1], t2[(ci + 1) & 1]);
    uint32_t v[32];
    tmem_load32(tcol + c, v);
    uint32_t pk[16];
    if (QK) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4) {
        const uint32_t w1[4] = {t1[ci & 1][v4].x, t1[ci & 1][v4].y, t1[ci & 1][v4].z, t1[ci & 1][v4].w};
        const uint32_t w2[4] = {t2[ci & 1][v4].x, t2[ci & 1][v4].y, t2[ci & 1][v4].z, t2[ci & 1][v4].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = v4 * 4 + e;
          const float qa = round_bf16(__uint_as_float(v[2 * j]) * sc);
          const float qb = round_bf16(__uint_as_float(v[2 * j + 1]) * sc);
          pk[j] = pack_bf16(qa * bf16_lo(w1[e]) + qb * bf16_lo(w2[e]), qb * bf16_hi(w1[e]) + qa * bf16_hi(w2[e]));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float a = __uint_as_float(v[2 * j]) * rs;
        float bb = __uint_as_float(v[2 * j + 1]) * rs;
        if (typ == 3) {
          a = __fdividef(1.0f, 1.0f + __expf(-a));
          bb = __fdividef(1.0f, 1.0f + __expf(-bb));
        }
        pk[j] = pack_bf16(a, bb);
      }
    }
    // 32 columns = 4 16-byte units of the row, in column chunk c / 64
#pragma unroll
    for (int j = 0; j < 4; ++j) stage_unit<HD>(slab, r, c / 8 + j, pk + 4 * j);
  }
}

// The same for head dims <= 64, with one TMEM round trip per slab: the whole
// row of the slab is loaded at once (both 32-column chunks in flight), the
// rotary-table row is fetched alongside so its latency overlaps the TMEM wait,
// and the values stay in registers from the sum of squares to the rotary.
template <int HD, bool QK>
__device__ __forceinline__ void qkvg_slab_row(const GemmParams& p, uint32_t tcol, uint32_t slab, int r, int typ,
                                              float rs, size_t bht, const __nv_bfloat16* f1row,
                                              const __nv_bfloat16* f2row) {
  static_assert(HD == 32 || HD == 64, "row-at-once slab: head dim 32 or 64");
  constexpr int NCH = HD / 32;
  uint32_t v[NCH][32];
  uint4 w1[HD / 8], w2[HD / 8];
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) tmem_ld32(tcol + 32 * ci, v[ci]);
  if (QK) {
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      w1[j] = __ldg(reinterpret_cast<const uint4*>(f1row) + j);
      w2[j] = __ldg(reinterpret_cast<const uint4*>(f2row) + j);
    }
  }
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) tmem_wait_ld_tied(v[ci]);
  float sc = rs;
  if (QK) {
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int ci = 0; ci < NCH; ++ci)
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float x0 = __uint_as_float(v[ci][j]) * rs, x1 = __uint_as_float(v[ci][j + 1]) * rs;
        ss0 = fmaf(x0, x0, ss0);
        ss1 = fmaf(x1, x1, ss1);
      }
    const float inv = rsqrtf((ss0 + ss1) / float(HD) + p.eps);
    float* rdst = typ == 0 ? p.rq : p.rk;
    if (rdst) rdst[bht] = inv;
    sc = rs * inv;
  }
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    const int c = 32 * ci;
    uint32_t pk[16];
    if (QK) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4) {
        const uint4 a1 = w1[ci * 4 + v4], a2 = w2[ci * 4 + v4];
        const uint32_t x1[4] = {a1.x, a1.y, a1.z, a1.w}, x2[4] = {a2.x, a2.y, a2.z, a2.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = v4 * 4 + e;
          const float qa = round_bf16(__uint_as_float(v[ci][2 * j]) * sc);
          const float qb = round_bf16(__uint_as_float(v[ci][2 * j + 1]) * sc);
          pk[j] = pack_bf16(qa * bf16_lo(x1[e]) + qb * bf16_lo(x2[e]), qb * bf16_hi(x1[e]) + qa * bf16_hi(x2[e]));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float a = __uint_as_float(v[ci][2 * j]) * rs;
        float bb = __uint_as_float(v[ci][2 * j + 1]) * rs;
        if (typ == 3) {
          a = __fdividef(1.0f, 1.0f + __expf(-a));
          bb = __fdividef(1.0f, 1.0f + __expf(-bb));
        }
        pk[j] = pack_bf16(a, bb);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) stage_unit<HD>(slab, r, c / 8 + j, pk + 4 * j);
  }
}

// q/k RMSNorm over the head dim, bf16 rounding of the normed value, then
// interleaved rotary out[n] = qn[n]*f1[t,n] + qn[n^1]*f2[t,n]
// (fast_triton_attn.py:102-106, :132-141); v stored as is (fast_triton_attn.py:108)
// and g as sigmoid(g) (fast_triton_attn.py:123).  This thread's row of each
// slab its group owns (slabs s with s % 2 == wg) goes straight to the slab's
// [B,H,T,N] output.  For N = 128 the q/k slabs go first, while the rotary rows
// preloaded by the caller are live, and v/g follow.
template <int BN, int HD>
__device__ __forceinline__ void epi_qkvg(const GemmParams& p, uint32_t taddr, int m, int n0, int wg, int r, int ti,
                                         uint32_t stg, uint4 (&t1)[2][4], uint4 (&t2)[2][4]) {
  constexpr int NSLAB = BN / HD;
  constexpr uint32_t SLAB_BYTES = GEMM_BM * HD * 2;
  const int b = m / p.T;
  const int t = m - b * p.T;
  const float rs = p.row_scale ? p.row_scale[m] : 1.0f;
  const __nv_bfloat16* f1row = p.f1 + size_t(t) * p.ldf;
  const __nv_bfloat16* f2row = p.f2 + size_t(t) * p.ldf;
  // the group's previous copy-out has read the staging tile
  named_bar_sync(1 + wg, 128);
  if constexpr (HD <= 64) {
#pragma unroll 1
    for (int s = wg; s < NSLAB; s += 2) {
      const int sg = n0 / HD + s;
      const size_t bht = (size_t(b) * p.H + (sg >> 2)) * p.T + t;
      if ((sg & 3) < 2)
        qkvg_slab_row<HD, true>(p, taddr + s * HD, stg + s * SLAB_BYTES, r, sg & 3, rs, bht, f1row, f2row);
      else
        qkvg_slab_row<HD, false>(p, taddr + s * HD, stg + s * SLAB_BYTES, r, sg & 3, rs, bht, f1row, f2row);
    }
  } else {
#pragma unroll 1
    for (int s = wg; s < NSLAB; s += 2) {
      const int sg = n0 / HD + s;
      if ((sg & 3) < 2)
        qkvg_slab<HD, true>(p, taddr + s * HD, stg + s * SLAB_BYTES, r, sg & 3, rs,
                            (size_t(b) * p.H + (sg >> 2)) * p.T + t, f1row, f2row, t1, t2);
    }
#pragma unroll 1
    for (int s = wg; s < NSLAB; s += 2) {
      const int sg = n0 / HD + s;
      if ((sg & 3) >= 2)
        qkvg_slab<HD, false>(p, taddr + s * HD, stg + s * SLAB_BYTES, r, sg & 3, rs,
                             (size_t(b) * p.H + (sg >> 2)) * p.T + t, f1row, f2row, t1, t2);
    }
  }
}

// Copy-out of the slabs staged by epi_qkvg (after the group's barrier).
template <int BN, int HD>
__device__ __forceinline__ void epi_qkvg_copy_out(const GemmParams& p, int m0, int n0, int wg, int ti, uint32_t stg) {
  constexpr int NSLAB = BN / HD;
  const int b = m0 / p.T, t0 = m0 - (m0 / p.T) * p.T;
  named_bar_sync(1 + wg, 128);
#pragma unroll 1
  for (int s = wg; s < NSLAB; s += 2) {
    const int sg = n0 / HD + s;
    const int typ = sg & 3;
    __nv_bfloat16* out = (typ == 0 ? p.q : typ == 1 ? p.k : typ == 2 ? p.v : p.g) +
                         ((size_t(b) * p.H + (sg >> 2)) * p.T + t0) * HD;
    copy_out_slab<HD>(stg + s * (GEMM_BM * HD * 2), out, ti);
  }
}


// Gate backward fused on the dGated = dY * Wo tile (fast_triton_attn.py:576-584, :601):
//   dO = dGated*g  -> [B,H,T,N] bf16 (input of the attention backward)
//   dg_pre = dGated*O*g*(1-g) -> the g slot of the projection-gradient buffer
//   delta = rowsum(dO*O) per (b,h,t)  (the attention backward's D term)
template <int BN, int HD>
__device__ __forceinline__ void epi_dgate(const GemmParams& p, uint32_t taddr, int m, int n0) {
  constexpr int hd = HD;
  const int b = m / p.T;
  const int t = m - b * p.T;
  constexpr int nslab = BN / hd;
  constexpr int nch = hd / 32;
#pragma unroll 1
  for (int s = 0; s < nslab; ++s) {
    const int head = n0 / hd + s;
    const size_t bht = (size_t(b) * p.H + head) * p.T + t;
    const __nv_bfloat16* orow = p.o_in + bht * hd;
    const __nv_bfloat16* grow = p.gs_in + bht * hd;
    __nv_bfloat16* dorow = p.do_out + bht * hd;
    __nv_bfloat16* dgrow = p.dg_out + size_t(m) * p.ld_dg + size_t(head) * hd;
    float dsum = 0.f;
    // O and sigmoid(g) of the row are loaded one 32-column chunk ahead of their use.
    uint4 ob[2][4], gb[2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ob[0][j] = *reinterpret_cast<const uint4*>(orow + 8 * j);
      gb[0][j] = *reinterpret_cast<const uint4*>(grow + 8 * j);
    }
#pragma unroll
    for (int ci = 0; ci < nch; ++ci) {
      const int c = 32 * ci;
      const int cur = ci & 1;
      if (ci + 1 < nch) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ob[cur ^ 1][j] = *reinterpret_cast<const uint4*>(orow + c + 32 + 8 * j);
          gb[cur ^ 1][j] = *reinterpret_cast<const uint4*>(grow + c + 32 + 8 * j);
        }
      }
      uint32_t r[32];
      tmem_load32(taddr + s * hd + c, r);
      uint32_t pd[16], pg[16];
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4) {
        const uint4 ov = ob[cur][v4];
        const uint4 gv = gb[cur][v4];
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = v4 * 4 + e;
          const float o0 = bf16_lo(ow[e]), o1 = bf16_hi(ow[e]);
          const float g0 = bf16_lo(gw[e]), g1 = bf16_hi(gw[e]);
          const float d0 = __uint_as_float(r[2 * j]), d1 = __uint_as_float(r[2 * j + 1]);
          const float do0 = round_bf16(d0 * g0), do1 = round_bf16(d1 * g1);
          dsum = fmaf(do0, o0, dsum);
          dsum = fmaf(do1, o1, dsum);
          pd[j] = pack_bf16(do0, do1);
          pg[j] = pack_bf16(d0 * o0 * g0 * (1.0f - g0), d1 * o1 * g1 * (1.0f - g1));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        st_global_v4(dorow + c + 8 * j, pd[4 * j], pd[4 * j + 1], pd[4 * j + 2], pd[4 * j + 3]);
        st_global_v4(dgrow + c + 8 * j, pg[4 * j], pg[4 * j + 1], pg[4 * j + 2], pg[4 * j + 3]);
      }
    }
    p.delta[bht] = dsum;
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
// HD: head dim for the per-head epilogues (EPI_QKVG, EPI_DGATE), 0 otherwise.
template <int BN, int AM, int BMD, int EPI, int HD>
__global__ void __launch_bounds__(GemmCfg<BN, EPI>::THREADS, 1) gemm_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16(GEMM_BM, BN, AM == A_MN ? 1u : 0u, (BMD == B_MN || BMD == B_MN_KSPLIT4) ? 1u : 0u);
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * GEMM_A_BYTES;
  // barriers after the stage ring and the staging tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING_BYTES);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto accf_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = p.m_tiles * p.n_tiles * p.k_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 32 * Cfg::EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.a);
    for (int i = 0; i < 4; ++i) tma_prefetch_desc(&maps.b[i]);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  Guard g(p.status, KID_GEMM);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      for (int t = blockIdx.x; t < ntiles && g.ok; t += gridDim.x) {
        int m0, n0, kb0, kb1;
        gemm_decode(p, BN, t, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, g, 1)) break;
          const uint32_t fb = full_bar(stage);
          mbar_expect_tx(fb, Cfg::STAGE_BYTES);
          const uint32_t a_dst = sA + stage * GEMM_A_BYTES;
          const uint32_t b_dst = sB + stage * Cfg::B_BYTES;
          if (AM == A_K) {
            tma_load_2d(a_dst, &maps.a, fb, kb * GEMM_BK, m0);
          } else {
            tma_load_2d(a_dst, &maps.a, fb, m0, kb * GEMM_BK);
            tma_load_2d(a_dst + 8192, &maps.a, fb, m0 + 64, kb * GEMM_BK);
          }
          if (BMD == B_K) {
            tma_load_2d(b_dst, &maps.b[0], fb, kb * GEMM_BK, n0);
          } else if (BMD == B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i) tma_load_2d(b_dst + 8192 * i, &maps.b[0], fb, n0 + 64 * i, kb * GEMM_BK);
          } else if (BMD == B_SLABS) {
            const int nsl = BN / p.slab_rows;
            for (int s = 0; s < nsl; ++s) {
              const int sg = n0 / p.slab_rows + s;
              tma_load_2d(b_dst + s * p.slab_rows * 128, &maps.b[sg & 3], fb, kb * GEMM_BK, (sg >> 2) * p.slab_rows);
            }
          } else {
            const int src = kb / p.b_kb_per_src;
            const int kr = (kb - src * p.b_kb_per_src) * GEMM_BK;
#pragma unroll
            for (int i = 0; i < BN / 64; ++i) tma_load_2d(b_dst + 8192 * i, &maps.b[src], fb, n0 + 64 * i, kr);
          }
          last_par[stage] = int(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!g.ok) {
        // Abort: let every copy this thread issued land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_drain(full_bar(s), uint32_t(last_par[s]));
      } else {
        // Tail: wait for the MMA warp's release (tcgen05.commit) of every stage's
        // last fill, so no asynchronous arrive targets this CTA's shared memory
        // after it exits.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(empty_bar(s), uint32_t(last_par[s]), g, 6);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool any = false;
      for (int t = blockIdx.x; t < ntiles && g.ok; t += gridDim.x, ++it) {
        int m0, n0, kb0, kb1;
        gemm_decode(p, BN, t, m0, n0, kb0, kb1);
        const int buf = it & 1;
        if (!mbar_wait(acce_bar(buf), ((it >> 1) & 1) ^ 1, g, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, g, 3)) break;
          tc_fence_after();
          const uint32_t a_base = sA + stage * GEMM_A_BYTES;
          const uint32_t b_base = sB + stage * Cfg::B_BYTES;
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = AM == A_K ? smem_desc(a_base + 32 * k, 16, 1024, SW_128B)
                                          : smem_desc(a_base + 2048 * k, 8192, 1024, SW_128B);
            const uint64_t bd = (BMD == B_K || BMD == B_SLABS) ? smem_desc(b_base + 32 * k, 16, 1024, SW_128B)
                                                                : smem_desc(b_base + 2048 * k, 8192, 1024, SW_128B);
            mma_ss(d, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          any = true;
          mma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!g.ok) break;
        mma_commit(accf_bar(buf));
      }
      if (!g.ok && any) {
        mma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ---------------- Epilogue: warps 2 .. 2+EPI_WARPS-1 ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int wg = (warp - 2) >> 2;  // epilogue group (QKVG: 0 or 1)
    const int ti = (warp - 2 - 4 * wg) * 32 + lane;  // thread index within the group
    const uint32_t stg = sA + STAGES * Cfg::STAGE_BYTES;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      int m0, n0, kb0, kb1;
      gemm_decode(p, BN, t, m0, n0, kb0, kb1);
      const int buf = it & 1;
      // Projection epilogue: the rotary-table rows of this thread's token are
      // loaded before the accumulator wait, which hides their latency.
      uint4 pre1[2][4], pre2[2][4];
      if constexpr (Cfg::QKVG && HD > 64) {
        const int t = (m0 + row) % p.T;
        const __nv_bfloat16* f1row = p.f1 + size_t(t) * p.ldf;
        const __nv_bfloat16* f2row = p.f2 + size_t(t) * p.ldf;
        load_tab_chunk<HD>(f1row, f2row, 0, pre1[0], pre2[0]);
        if (HD > 32) load_tab_chunk<HD>(f1row, f2row, 32, pre1[1], pre2[1]);
      }
      bool ok = mbar_wait(accf_bar(buf), (it >> 1) & 1, g, 4);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        g.ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + buf * BN;
      const int m = m0 + row;
      if constexpr (Cfg::QKVG) {
        epi_qkvg<BN, HD>(p, taddr, m, n0, wg, row, ti, stg, pre1, pre2);
        tc_fence_before();
        mbar_arrive(acce_bar(buf));
        epi_qkvg_copy_out<BN, HD>(p, m0, n0, wg, ti, stg);
      } else {
        if constexpr (EPI == EPI_DGATE)
          epi_dgate<BN, HD>(p, taddr, m, n0);
        else
          epi_store<BN>(p, EPI, taddr, m, n0);
        tc_fence_before();
        mbar_arrive(acce_bar(buf));
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace mea
