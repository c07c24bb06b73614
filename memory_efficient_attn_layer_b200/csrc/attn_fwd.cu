// Causal softmax attention forward on tcgen05, with the sigmoid gate and the
// [B,H,T,N] -> [B,T,H*N] repack fused into the epilogue.
//
// Replaces the reference's ATen flash-attention call plus gate_repack_kernel
// (fast_triton_attn.py:425-457) and, in the backward, the recompute gate
// (fast_triton_attn.py:559-570).
//
// One CTA = one (b, h, 128-row query tile), two CTAs per SM: each holds 256
// TMEM columns, so while one CTA's softmax warps work on exponentials the
// other CTA's MMAs keep the tensor core busy, and one CTA's prologue/epilogue
// overlaps the other's main loop.  Warp 0 loads Q once and streams K and V
// through separate TMA rings; warp 1 issues S_j = Q K_j^T and O += P_j V_j with
// P read straight from TMEM; warps 2..5 run the softmax, one query row per
// thread.  Key tiles above the diagonal are never loaded (causal skipping); the
// diagonal tile is masked.
//
// TMEM, N <= 64: S [0,128), P [128,192), O [192, 192+N).  S_j is computed in
// two 64-key halves with their own barriers; the softmax warps turn each half
// into bf16 P in registers, release it (so that half of S_{j+1} = Q K_{j+1}^T
// runs while they work on the other) and write its P columns once PV_{j-1} has
// consumed the previous P (pv_done): neither MMA sits on the per-tile chain.  N = 128 (O needs 128 columns): S
// [0,128) with P written over it in place, O [128,256); S_{j+1} is issued after
// PV_j (tcgen05 MMAs of one thread run in issue order).
//
// The reference value subtracted before exp2 is one of:
// * a bound on every scaled score of the call (forward of the block: q and k
//   are RMS-normalised per head, so the rotary tables bound |q.k|): one pass
//   over each score row, no row max, no rescaling of O;
// * the saved row log-sum-exp (the backward's recompute): P comes out
//   normalised, exactly the P the attention backward rebuilds;
// * the online running max, refreshed lazily: O and the row sum are rescaled
//   only when a row's max grows by more than 2^8 (every P value stays <= 256).
//
// Outputs: gated[b, t, h*N + n] = (O/l)[n] * gs[b,h,t,n] (bf16), the row
// log-sum-exp in log2 units lse2 = m + log2(l) (fp32, [B,H,T]), and
// optionally O itself in [B,H,T,N] bf16 (needed by the gate backward).
#include "attn_common.cuh"
#include "launch.h"
#include "tma.h"

namespace mea {

struct AttnFwdParams {
  int B, H, T;
  float scale_log2;         // softmax scale * log2(e)
  const __nv_bfloat16* gs;  // sigmoid(g), [B,H,T,N]
  __nv_bfloat16* gated;     // [B,T,H*N]
  float* lse2;              // [B,H,T]; NULL when lse_in is given
  __nv_bfloat16* o_out;     // optional [B,H,T,N]
  const float* bound;       // optional device scalar: bound on every scaled score (log2 units)
  const float* lse_in;      // optional saved lse2: normalised recompute
  float* dq_zero;           // optional fp32 [B,H,T,N] cleared by the epilogue (N <= 64)
  int* status;
};

struct AttnFwdMaps {
  CUtensorMap q, k, v;
  // (N <= 64) epilogue: sigmoid(g) tile in ([B*H*T, N], 128-row box), gated out
  // ([B*T, H*N], 32-row boxes), O out ([B*H*T, N], 32-row boxes)
  CUtensorMap gs, gated, o;
  CUtensorMap dqz;  // (N <= 64) dq_zero as [B*H*T, N] fp32, 32-column x 32-row boxes
};

template <int HD>
struct AttnFwdCfg {
  static constexpr int KS = HD <= 64 ? 2 : 1;  // K ring depth
  static constexpr int VS = HD <= 64 ? 2 : 1;  // V ring depth
  static constexpr uint32_t TILE_BYTES = 128 * HD * 2;
  static constexpr bool SEP_P = HD <= 64;  // P in its own TMEM columns
  static constexpr uint32_t S_COL = 0, P_COL = SEP_P ? 128 : 0, O_COL = SEP_P ? 192 : 128;
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr size_t SMEM = 1024 + TILE_BYTES * (1 + KS + VS) + 256;
};

// Max of 16 raw scores of key columns [16c, 16c+16) into four chains.
template <bool DIAG>
__device__ __forceinline__ void max_chunk(const uint32_t (&v)[16], int c, int r, float (&m)[4]) {
  float x[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) x[e] = (DIAG && 16 * c + e > r) ? -INFINITY : __uint_as_float(v[e]);
#pragma unroll
  for (int e = 0; e < 16; e += 8) {
    m[0] = max3f(m[0], x[e], x[e + 1]);
    m[1] = max3f(m[1], x[e + 2], x[e + 3]);
    m[2] = max3f(m[2], x[e + 4], x[e + 5]);
    m[3] = max3f(m[3], x[e + 6], x[e + 7]);
  }
}

// Row max of one 128-column score row held in TMEM (raw, unscaled scores),
// streamed in 16-column chunks with the next chunk's load in flight.
// DIAG: the diagonal tile, where key column c > query row r is masked out.
template <bool DIAG>
__device__ __forceinline__ float score_row_max(uint32_t sb, int r) {
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  uint32_t a[16], b[16];
  tmem_ld16(sb, a);
  tmem_wait_ld_tied(a);
#pragma unroll
  for (int c = 0; c < 8; c += 2) {
    tmem_ld16(sb + 16 * (c + 1), b);
    max_chunk<DIAG>(a, c, r, m);
    tmem_wait_ld_tied(b);
    if (c + 2 < 8) tmem_ld16(sb + 16 * (c + 2), a);
    max_chunk<DIAG>(b, c + 1, r, m);
    if (c + 2 < 8) tmem_wait_ld_tied(a);
  }
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// exp2 of 16 scores, packed bf16 P for key columns [16c, 16c+16) stored over the
// score buffer at packed columns [8c, 8c+8); accumulates the row sum.
template <bool DIAG>
__device__ __forceinline__ void exp_chunk(const uint32_t (&v)[16], uint32_t sb, int c, int r, float2 scale2, float2 bias2,
                                          float2& acc0, float2& acc1) {
  uint32_t pk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 t = ffma2(make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), scale2, bias2);
    const float2 pp = exp2_pair(t, (kPolyPairsFwd >> e) & 1);
    float p0 = pp.x, p1 = pp.y;
    if (DIAG) {
      const int c0 = 16 * c + 2 * e;
      p0 = c0 > r ? 0.f : p0;
      p1 = c0 + 1 > r ? 0.f : p1;
    }
    if (e & 1)
      acc1 = fadd2(acc1, make_float2(p0, p1));
    else
      acc0 = fadd2(acc0, make_float2(p0, p1));
    pk[e] = pack_bf16(p0, p1);
  }
  tmem_st8(sb + 8 * c, pk);
}

// P = exp2(s * sl2 - m) for one row, written back over the scores as packed
// bf16 pairs (columns [0, 64) of the S buffer); returns the row sum of P.
template <bool DIAG>
__device__ __forceinline__ float exp_pack_row(uint32_t sb, int r, float sl2, float neg_m) {
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  const float2 scale2 = make_float2(sl2, sl2), bias2 = make_float2(neg_m, neg_m);
  uint32_t a[16], b[16];
  tmem_ld16(sb, a);
  tmem_wait_ld_tied(a);
#pragma unroll
  for (int c = 0; c < 8; c += 2) {
    tmem_ld16(sb + 16 * (c + 1), b);
    exp_chunk<DIAG>(a, sb, c, r, scale2, bias2, acc0, acc1);
    tmem_wait_ld_tied(b);
    if (c + 2 < 8) tmem_ld16(sb + 16 * (c + 2), a);
    exp_chunk<DIAG>(b, sb, c + 1, r, scale2, bias2, acc0, acc1);
    if (c + 2 < 8) tmem_wait_ld_tied(a);
  }
  return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

// P = exp2(s * sl2 - m) of key columns [64*hh, 64*hh + 64) of query row r into
// registers (packed bf16 pairs, columns 64*hh + [2i, 2i+2) in pk[i]); returns
// this half's share of the row sum.  Every TMEM load has completed on return.
template <bool DIAG>
__device__ __forceinline__ float exp_half_regs(uint32_t sb, int hh, int r, float sl2, float neg_m, uint32_t (&pk)[32]) {
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  const float2 scale2 = make_float2(sl2, sl2), bias2 = make_float2(neg_m, neg_m);
  uint32_t a[16], b[16];
  auto chunk = [&](const uint32_t(&v)[16], int c) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float2 t = ffma2(make_float2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), scale2, bias2);
      const float2 pp = exp2_pair(t, (kPolyPairsFwd >> e) & 1);
      float p0 = pp.x, p1 = pp.y;
      if (DIAG) {
        const int c0 = 64 * hh + 16 * c + 2 * e;
        p0 = c0 > r ? 0.f : p0;
        p1 = c0 + 1 > r ? 0.f : p1;
      }
      if (e & 1)
        acc1 = fadd2(acc1, make_float2(p0, p1));
      else
        acc0 = fadd2(acc0, make_float2(p0, p1));
      pk[8 * c + e] = pack_bf16(p0, p1);
    }
  };
  tmem_ld16(sb + 64 * hh, a);
  tmem_wait_ld_tied(a);
#pragma unroll
  for (int c = 0; c < 4; c += 2) {
    tmem_ld16(sb + 64 * hh + 16 * (c + 1), b);
    chunk(a, c);
    tmem_wait_ld_tied(b);
    if (c + 2 < 4) tmem_ld16(sb + 64 * hh + 16 * (c + 2), a);
    chunk(b, c + 1);
    if (c + 2 < 4) tmem_wait_ld_tied(a);
  }
  return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

// RECOMP: the backward's recompute against the saved LSE (p.lse_in set): P comes
// out normalised, so no row max or row sum is formed and no LSE is written.
template <int HD, bool RECOMP>
__global__ void __launch_bounds__(192, 2) attn_fwd_kernel(const __grid_constant__ AttnFwdMaps maps, const AttnFwdParams p) {
  using Cfg = AttnFwdCfg<HD>;
  using Tile = HeadTile<HD>;
  constexpr int KS = Cfg::KS, VS = Cfg::VS;
  constexpr uint32_t TB = Cfg::TILE_BYTES;
  constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0, 0);
  constexpr uint32_t IDESC_SH = idesc_bf16(128, 64, 0, 0);  // (SEP_P) one 64-key half of S
  constexpr uint32_t IDESC_O = idesc_bf16(128, HD, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + TB;       // KS K tiles
  const uint32_t sV = sK + KS * TB;  // VS V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TB * (1 + KS + VS));
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0;
  auto k_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return b0 + 8u * (1 + KS + s); };
  auto v_full = [&](int s) { return b0 + 8u * (1 + 2 * KS + s); };
  auto v_empty = [&](int s) { return b0 + 8u * (1 + 2 * KS + VS + s); };
  const uint32_t s_full = b0 + 8u * (1 + 2 * KS + 2 * VS);
  const uint32_t p_full = s_full + 8;
  const uint32_t o_bar = s_full + 16;
  const uint32_t drain_bar = s_full + 24;
  const uint32_t s_empty = s_full + 32;  // (SEP_P) softmax has read the key half [0, 64) of S_j
  const uint32_t pv_done = s_full + 40;  // (SEP_P) PV_j has completed
  // (SEP_P) S_j is computed in two 64-key halves: s_full / s_empty for keys
  // [0, 64), s_full_b / s_empty_b for [64, 128)
  const uint32_t s_full_b = s_full + 48;
  const uint32_t s_empty_b = s_full + 56;
  const uint32_t q_free = s_full + 64;  // (SEP_P) the last score MMA has read Q
  const uint32_t gs_bar = s_full + 72;  // (SEP_P) sigmoid(g) tile landed in Q's buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11 + 2 * KS + 2 * VS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int nq = p.T / 128;
  // Head-major order: the query tiles of one (b,h) run side by side and share its
  // K/V in L2; within a head the longest (diagonal-most) tiles start first.
  const int bh = int(blockIdx.x) / nq;
  const int qt = nq - 1 - int(blockIdx.x) % nq;
  (void)BH;
  const int nkv = qt + 1;
  const int row0 = bh * p.T;  // first row of this (b,h) in the [B*H*T, HD] view

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(s_empty, 128);
    mbar_init(pv_done, 1);
    mbar_init(s_full_b, 1);
    mbar_init(s_empty_b, 128);
    mbar_init(q_free, 1);
    mbar_init(gs_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Guard g(p.status, KID_ATTN_FWD);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k);
      tma_prefetch_desc(&maps.v);
      mbar_expect_tx(q_full, TB);
#pragma unroll
      for (int c = 0; c < Tile::NCHUNK; ++c)
        tma_load_2d(sQ + c * 128 * Tile::SWB, &maps.q, q_full, c * Tile::CHUNK_ELEMS, row0 + qt * 128);
      int kpar[KS], vpar[VS];
      for (int s = 0; s < KS; ++s) kpar[s] = -1;
      for (int s = 0; s < VS; ++s) vpar[s] = -1;
      for (int j = 0; j < nkv; ++j) {
        const int sk = j % KS, sv = j % VS;
        const uint32_t pk = (j / KS) & 1, pv = (j / VS) & 1;
        if (!mbar_wait(k_empty(sk), pk ^ 1, g, 1)) break;
        mbar_expect_tx(k_full(sk), TB);
#pragma unroll
        for (int c = 0; c < Tile::NCHUNK; ++c)
          tma_load_2d(sK + sk * TB + c * 128 * Tile::SWB, &maps.k, k_full(sk), c * Tile::CHUNK_ELEMS, row0 + j * 128);
        kpar[sk] = int(pk);
        if (!mbar_wait(v_empty(sv), pv ^ 1, g, 9)) break;
        mbar_expect_tx(v_full(sv), TB);
#pragma unroll
        for (int c = 0; c < Tile::NCHUNK; ++c)
          tma_load_2d(sV + sv * TB + c * 128 * Tile::SWB, &maps.v, v_full(sv), c * Tile::CHUNK_ELEMS, row0 + j * 128);
        vpar[sv] = int(pv);
      }
      if (!g.ok) {
        mbar_drain(q_full, 0);
        for (int s = 0; s < KS; ++s)
          if (kpar[s] >= 0) mbar_drain(k_full(s), uint32_t(kpar[s]));
        for (int s = 0; s < VS; ++s)
          if (vpar[s] >= 0) mbar_drain(v_full(s), uint32_t(vpar[s]));
      } else {
        // Tail: wait for the MMA warp's release (tcgen05.commit) of the last K and
        // V tile of every ring slot, so no asynchronous arrive targets this CTA's
        // shared memory after it exits.
        for (int s = 0; s < KS; ++s)
          if (kpar[s] >= 0) mbar_wait(k_empty(s), uint32_t(kpar[s]), g, 13);
        for (int s = 0; s < VS; ++s)
          if (vpar[s] >= 0) mbar_wait(v_empty(s), uint32_t(vpar[s]), g, 14);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      bool any = false;
      auto issue_s = [&](int j) {
        const int sk = j % KS;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_ss(tmem + Cfg::S_COL, Tile::kmajor(sQ, 128, kk), Tile::kmajor(sK + sk * TB, 128, kk), IDESC_S,
                 kk > 0 ? 1u : 0u);
        mma_commit(k_empty(sk));
        mma_commit(s_full);
      };
      if constexpr (Cfg::SEP_P) {
        // S_j in two 64-key halves, each committed to its own barrier, so that the
        // half [0, 64) of S_{j+1} runs while the softmax warps work on keys
        // [64, 128) of S_j, and the other half while they start on S_{j+1}.
        auto issue_half = [&](int j, int hf) {
          const int sk = j % KS;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem + Cfg::S_COL + 64 * hf, Tile::kmajor(sQ, 128, kk),
                   Tile::kmajor(sK + sk * TB + hf * 64 * Tile::SWB, 128, kk), IDESC_SH, kk > 0 ? 1u : 0u);
          if (hf) mma_commit(k_empty(sk));
          mma_commit(hf ? s_full_b : s_full);
        };
        if (mbar_wait(q_full, 0, g, 5) && mbar_wait(k_full(0), 0, g, 2)) {
          tc_fence_after();
          issue_half(0, 0);
          issue_half(0, 1);
          if (nkv == 1) mma_commit(q_free);
          any = true;
          for (int j = 0; j < nkv; ++j) {
            const int sv = j % VS;
            if (j + 1 < nkv) {  // each half of S_{j+1} as soon as that half of S_j has been read
              if (!mbar_wait(s_empty, j & 1, g, 10)) break;
              if (!mbar_wait(k_full((j + 1) % KS), ((j + 1) / KS) & 1, g, 2)) break;
              tc_fence_after();
              issue_half(j + 1, 0);
              if (!mbar_wait(s_empty_b, j & 1, g, 16)) break;
              tc_fence_after();
              issue_half(j + 1, 1);
              if (j + 2 == nkv) mma_commit(q_free);
            } else {
              // Q is no longer read: bring the tile's sigmoid(g) into its buffer for
              // the epilogue while the last softmax tile runs.
              if (!mbar_wait(q_free, 0, g, 19)) break;
              mbar_expect_tx(gs_bar, TB);
              tma_load_2d(sQ, &maps.gs, gs_bar, 0, row0 + qt * 128);
            }
            if (!mbar_wait(p_full, j & 1, g, 3)) break;
            if (!mbar_wait(v_full(sv), (j / VS) & 1, g, 4)) break;
            tc_fence_after();
#pragma unroll
            for (int kc = 0; kc < 8; ++kc)
              mma_ts(tmem + Cfg::O_COL, tmem + Cfg::P_COL + kc * 8, Tile::mnmajor(sV + sv * TB, 128, kc), IDESC_O,
                     (j > 0 || kc > 0) ? 1u : 0u);
            mma_commit(v_empty(sv));
            mma_commit(pv_done);
          }
          if (g.ok) mma_commit(o_bar);
        }
      } else if (mbar_wait(q_full, 0, g, 5)) {
        for (int j = 0; j < nkv; ++j) {
          const int sk = j % KS, sv = j % VS;
          if (!mbar_wait(k_full(sk), (j / KS) & 1, g, 2)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem + Cfg::S_COL, Tile::kmajor(sQ, 128, kk), Tile::kmajor(sK + sk * TB, 128, kk), IDESC_S,
                   kk > 0 ? 1u : 0u);
          mma_commit(k_empty(sk));
          mma_commit(s_full);
          any = true;
          if (!mbar_wait(p_full, j & 1, g, 3)) break;
          if (!mbar_wait(v_full(sv), (j / VS) & 1, g, 4)) break;
          tc_fence_after();
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ts(tmem + Cfg::O_COL, tmem + Cfg::S_COL + kc * 8, Tile::mnmajor(sV + sv * TB, 128, kc), IDESC_O,
                   (j > 0 || kc > 0) ? 1u : 0u);
          mma_commit(v_empty(sv));
        }
        if (g.ok) mma_commit(o_bar);
      }
      if (!g.ok && any) {
        mma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ---------------- softmax + epilogue: warps 2..5 ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const int t = qt * 128 + r;
    const size_t bht = size_t(bh) * p.T + t;
    // Reference for exp2 (uniform over the CTA): 2 = saved LSE, 1 = score bound, 0 = online max.
    int mode = 0;
    float ref = 0.f;
    if constexpr (RECOMP) {
      mode = 2;
      ref = p.lse_in[bht];
    } else if (p.bound) {
      const float bnd = __ldg(p.bound);
      if (bnd <= ATTN_MAX_BOUND) {
        mode = 1;
        ref = bnd;
      }
    }
    float m_run = -INFINITY, l_run = 0.f;  // m_run in scaled log2 units
    bool ok = true;
    if constexpr (Cfg::SEP_P) {
      // S_j arrives in two 64-key halves; each half is released (s_empty,
      // s_empty_b) as soon as its exponentials are done, and its bf16 P
      // columns are written right away (once PV_{j-1} has consumed the
      // previous P).
      const uint32_t sb = lane_base + Cfg::S_COL;
      for (int j = 0; j < nkv && ok; ++j) {
        ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, g, 6));
        if (!ok) break;
        tc_fence_after();
        const bool diag = (j == qt);
        bool pv_seen = (j == 0);  // PV_{j-1} has completed (O and the P columns are free)
        bool have_b = false;      // the half [64, 128) of S_j has landed
        if (mode == 0) {
          // The online max needs the whole score row.
          ok = __all_sync(0xffffffffu, mbar_wait(s_full_b, j & 1, g, 17));
          if (!ok) break;
          tc_fence_after();
          have_b = true;
          const float mx = (diag ? score_row_max<true>(sb, r) : score_row_max<false>(sb, r)) * sl2;
          // Lazy rescale: refresh the reference max only when it grows by > 8 (log2 units).
          const bool need = mx > m_run + 8.0f;
          if (__any_sync(0xffffffffu, need)) {
            const float m_new = need ? mx : m_run;
            const float alpha = ex2(m_run - m_new);  // 0 when m_run = -inf
            if (j > 0) {
              ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, g, 11));
              if (!ok) break;
              tc_fence_after();
              pv_seen = true;
#pragma unroll
              for (int c = 0; c < HD; c += 16) {
                uint32_t ov[16];
                tmem_load16(lane_base + Cfg::O_COL + c, ov);
#pragma unroll
                for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                tmem_st16(lane_base + Cfg::O_COL + c, ov);
              }
            }
            l_run *= alpha;
            m_run = m_new;
          }
        }
        const float neg_m = mode != 0 ? -ref : -m_run;
        uint32_t pk[32];
        // Keys [0, 64), then [64, 128): one loop (not unrolled), so the exponential
        // code exists once and stays resident in the instruction cache.
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          if (hh == 1 && !have_b) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full_b, j & 1, g, 17));
            if (!ok) break;
            tc_fence_after();
          }
          l_run += diag ? exp_half_regs<true>(sb, hh, r, sl2, neg_m, pk) : exp_half_regs<false>(sb, hh, r, sl2, neg_m, pk);
          tc_fence_before();
          mbar_arrive(hh ? s_empty_b : s_empty);
          if (hh == 0 && !pv_seen) {
            ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, g, 12));
            if (!ok) break;
            tc_fence_after();
          }
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2)
            tmem_st16(lane_base + Cfg::P_COL + 32 * hh + 16 * q2, *reinterpret_cast<const uint32_t(*)[16]>(pk + 16 * q2));
          tmem_st_wait();  // the registers of pk are rewritten by the next half
        }
        if (!ok) break;
        tc_fence_before();
        mbar_arrive(p_full);
      }
    } else
    for (int j = 0; j < nkv && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, g, 6));
      if (!ok) break;
      tc_fence_after();
      const uint32_t sb = lane_base + Cfg::S_COL;
      const bool diag = (j == qt);
      if (mode != 0) {
        // Fixed reference: one pass, P = exp2(s*c - ref) <= 1 (up to bf16 rounding of q, k).
        l_run += diag ? exp_pack_row<true>(sb, r, sl2, -ref) : exp_pack_row<false>(sb, r, sl2, -ref);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full);
        continue;
      }
      const float mx = (diag ? score_row_max<true>(sb, r) : score_row_max<false>(sb, r)) * sl2;
      // Lazy rescale: refresh the reference max only when it grows by > 8 (log2 units).
      const bool need = mx > m_run + 8.0f;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_run;
        const float alpha = ex2(m_run - m_new);  // 0 when m_run = -inf
        if (j > 0) {
          // s_full(j) completing means PV_{j-1} (issued before S_j) completed: O is stable.
#pragma unroll
          for (int c = 0; c < HD; c += 16) {
            uint32_t ov[16];
            tmem_load16(lane_base + Cfg::O_COL + c, ov);
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st16(lane_base + Cfg::O_COL + c, ov);
          }
        }
        l_run *= alpha;
        m_run = m_new;
      }
      // P = exp2(s*c - m), its row sum, and bf16 P written over S for the PV MMA.
      l_run += diag ? exp_pack_row<true>(sb, r, sl2, -m_run) : exp_pack_row<false>(sb, r, sl2, -m_run);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- epilogue: O / l, gate, repack ----
    if constexpr (Cfg::SEP_P) {
      // The sigmoid(g) tile is in Q's buffer (gs_bar); each warp writes its 32
      // rows of gated and O into the first K / V slots (free after the last S and
      // PV MMAs) in the tensor maps' swizzle and stores them by TMA.
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_bar, 0, g, 8));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nkv - 1) & 1, g, 15));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(gs_bar, 0, g, 20));
      if (ok) {
        tc_fence_after();
        const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
        if (mode != 0) m_run = ref;
        const float inv_l = mode == 2 ? 1.0f : 1.0f / l_run;
        constexpr int ROWB = Tile::SWB;  // bytes per tile row (HD <= 64: one swizzle chunk)
        auto unit = [&](uint32_t tile, int u) -> uint32_t {
          return ROWB == 128 ? tile + r * 128 + ((u ^ (r & 7)) << 4) : tile + r * 64 + ((u ^ ((r >> 1) & 3)) << 4);
        };
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          uint32_t ov[16];
          tmem_load16(lane_base + Cfg::O_COL + c, ov);
#pragma unroll
          for (int u2 = 0; u2 < 2; ++u2) {
            const int u = c / 8 + u2;
            uint32_t gw[4];
            asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(gw[0]), "=r"(gw[1]), "=r"(gw[2]), "=r"(gw[3])
                         : "r"(unit(sQ, u)) : "memory");
            uint32_t go[4], oo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float o0 = __uint_as_float(ov[8 * u2 + 2 * e]) * inv_l;
              const float o1 = __uint_as_float(ov[8 * u2 + 2 * e + 1]) * inv_l;
              go[e] = pack_bf16(o0 * bf16_lo(gw[e]), o1 * bf16_hi(gw[e]));
              oo[e] = pack_bf16(o0, o1);
            }
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(unit(sK, u)), "r"(go[0]), "r"(go[1]), "r"(go[2]),
                         "r"(go[3]) : "memory");
            if (p.o_out)
              asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(unit(sV, u)), "r"(oo[0]), "r"(oo[1]),
                           "r"(oo[2]), "r"(oo[3]) : "memory");
          }
        }
        if (!RECOMP && p.lse2) p.lse2[bht] = m_run + __log2f(l_run);
        fence_proxy_async_smem();
        __syncwarp();
        if (p.dq_zero) {
          // Zero rows for the backward's dQ accumulator: a 32-row x 128-byte zero
          // tile per warp in the free second K / V slots, stored HD/32 times.
          const uint32_t zb = (quarter < 2 ? sK : sV) + TB + uint32_t((quarter & 1) * 4096);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(zb + lane * 128 + u * 16), "r"(0u) : "memory");
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) {
          const uint32_t box = uint32_t(quarter * 32 * ROWB);
          tma_store_2d(&maps.gated, sK + box, h * HD, b * p.T + qt * 128 + quarter * 32);
          if (p.o_out) tma_store_2d(&maps.o, sV + box, 0, row0 + qt * 128 + quarter * 32);
          if (p.dq_zero)
#pragma unroll
            for (int c = 0; c < HD; c += 32)
              tma_store_2d(&maps.dqz, (quarter < 2 ? sK : sV) + TB + uint32_t((quarter & 1) * 4096), c,
                           row0 + qt * 128 + quarter * 32);
          bulk_commit();
          bulk_wait0();
        }
        __syncwarp();
      }
    } else {
    // sigmoid(g) of this row is fetched while the last PV completes.
    uint4 gv[HD / 8];
    if (ok) {
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) gv[c] = __ldg(reinterpret_cast<const uint4*>(p.gs + bht * HD) + c);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_bar, 0, g, 8));
    if (ok) {
      tc_fence_after();
      const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
      if (mode != 0) m_run = ref;
      const float inv_l = mode == 2 ? 1.0f : 1.0f / l_run;
      __nv_bfloat16* grow = p.gated + (size_t(b) * p.T + t) * size_t(p.H * HD) + size_t(h) * HD;
      __nv_bfloat16* orow = p.o_out ? p.o_out + bht * HD : nullptr;
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        uint32_t ov[16];
        tmem_load16(lane_base + Cfg::O_COL + c, ov);
        const uint4 g0 = gv[c / 8], g1 = gv[c / 8 + 1];
        const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        uint32_t go[8], oo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float o0 = __uint_as_float(ov[2 * e]) * inv_l;
          const float o1 = __uint_as_float(ov[2 * e + 1]) * inv_l;
          go[e] = pack_bf16(o0 * bf16_lo(gw[e]), o1 * bf16_hi(gw[e]));
          oo[e] = pack_bf16(o0, o1);
        }
        st_global_v4(grow + c, go[0], go[1], go[2], go[3]);
        st_global_v4(grow + c + 8, go[4], go[5], go[6], go[7]);
        if (orow) {
          st_global_v4(orow + c, oo[0], oo[1], oo[2], oo[3]);
          st_global_v4(orow + c + 8, oo[4], oo[5], oo[6], oo[7]);
        }
      }
      if (!RECOMP && p.lse2) p.lse2[bht] = m_run + __log2f(l_run);
    }
    }
    if (!ok) g.ok = false;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int HD>
static int launch_attn_fwd_t(const AttnFwdMaps& maps, const AttnFwdParams& p, cudaStream_t st) {
  using Cfg = AttnFwdCfg<HD>;
  auto kern = p.lse_in ? attn_fwd_kernel<HD, true> : attn_fwd_kernel<HD, false>;
  if (!smem_attr_set(reinterpret_cast<const void*>(kern), int(Cfg::SMEM)))
    return set_error(MEA_ERR_CUDA, "cudaFuncSetAttribute(attn_fwd) failed");
  const int grid = p.B * p.H * (p.T / 128);
  kern<<<grid, 192, Cfg::SMEM, st>>>(maps, p);
  return check_launch("attn_fwd_kernel");
}

int run_attn_fwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* gs, void* gated,
                 float* lse2, void* o_out, const float* bound, const float* lse_in, int* status, cudaStream_t st,
                 float* dq_zero) {
  if (dq_zero && HD > 64)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "attention: dQ clearing is built for head dims <= 64");
  if (HD != 32 && HD != 64 && HD != 128)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention: head dim %d not in {32, 64, 128}", HD);
  if (T % 128 != 0 || T <= 0 || B <= 0 || H <= 0)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention: T=%d must be a positive multiple of 128", T);
  if (uint64_t(B) * H * T * HD > (uint64_t(1) << 31))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention: B*H*T*N must stay below 2^31");
  if (!q || !k || !v || !gs || !gated || (!lse2 && !lse_in))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "attention: NULL tensor pointer");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(gs) | reinterpret_cast<uintptr_t>(gated) | reinterpret_cast<uintptr_t>(o_out) |
       reinterpret_cast<uintptr_t>(dq_zero)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "attention: q/k/v/gs/gated/o/dq tensors must be 16-byte aligned");
  const uint64_t rows = uint64_t(B) * H * T;
  const int swb = HD * 2 >= 128 ? 128 : HD * 2;
  const int box_inner = swb / 2;
  AttnFwdMaps maps;
  const auto sw = swizzle_for(swb);
  int rc = make_tmap_2d(&maps.q, q, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.k, k, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.v, v, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  if (HD <= 64) {
    rc |= make_tmap_2d(&maps.gs, gs, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
    rc |= make_tmap_2d(&maps.gated, gated, uint64_t(H) * HD, uint64_t(B) * T, uint64_t(H) * HD * 2, box_inner, 32, sw);
    rc |= make_tmap_2d(&maps.o, o_out ? o_out : gated, HD, rows, uint64_t(HD) * 2, box_inner, 32, sw);
    if (dq_zero)
      rc |= make_tmap_2d(&maps.dqz, dq_zero, HD, rows, uint64_t(HD) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
  }
  if (rc) return set_error(MEA_ERR_CUDA, "attention: tensor map encode failed");
  AttnFwdParams p;
  p.B = B;
  p.H = H;
  p.T = T;
  p.scale_log2 = 1.4426950408889634f / sqrtf(float(HD));
  p.gs = static_cast<const __nv_bfloat16*>(gs);
  p.gated = static_cast<__nv_bfloat16*>(gated);
  p.o_out = static_cast<__nv_bfloat16*>(o_out);
  p.bound = lse_in ? nullptr : bound;
  p.lse_in = lse_in;
  p.dq_zero = dq_zero;
  p.lse2 = lse_in ? nullptr : lse2;
  p.status = status;
  switch (HD) {
    case 32: return launch_attn_fwd_t<32>(maps, p, st);
    case 64: return launch_attn_fwd_t<64>(maps, p, st);
    default: return launch_attn_fwd_t<128>(maps, p, st);
  }
}

}  // namespace mea
