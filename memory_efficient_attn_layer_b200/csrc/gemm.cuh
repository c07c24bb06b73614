// Persistent warp-specialised tcgen05 GEMM for sm_100a on CTA pairs.
//
//   D[M, N] = sum_k A[m, k] * B[n, k]      (bf16 operands, fp32 accumulate in TMEM)
//
// The grid is a set of 2-CTA clusters, one CTA per SM.  Each pair walks a
// static list of 256 x BN output tiles (optionally split along K): every CTA
// stages its own 128 rows of A and its own BN/2 columns of B, and the pair's
// leader issues one tcgen05.mma.cta_group::2 of M = 256 per 16-deep k-step,
// which reads both CTAs' shared memory and leaves each CTA's 128 accumulator
// rows in its own TMEM.  Per SM this halves the B traffic through shared
// memory, whose bandwidth (TMA writes plus tensor-core reads) is what bounds a
// 128 x BN single-CTA tile at K = 512.
//
// Roles per CTA: warp 0 issues the TMA loads into a STAGES-deep ring (counted
// on the leader's "full" barrier), warp 1 of the leader issues the MMAs into
// one of two TMEM accumulators (double-buffered, so the epilogue of tile i
// overlaps the mainloop of tile i+1), and the epilogue warps (one TMEM lane =
// one output row per thread) read the accumulator, release it to the leader,
// and write their results through a swizzled shared-memory staging tile with
// TMA stores, so that no epilogue access to global memory is row-per-thread.
// Operands may be K-major or MN-major in global memory; both are staged with
// 128-byte swizzle and described to the tensor core with the matching smem
// descriptor, so no transposes are ever written.
//
// Epilogues carry the block's elementwise work so it never makes its own pass
// over HBM:
//   EPI_QKVG  : row scale (the fused input RMSNorm), per-head q/k RMSNorm +
//               interleaved rotary, v copy, sigmoid(g), [B, H, T, N] outputs
//               (fast_triton_attn.py:102-144); rotary-table rows come in by TMA
//   EPI_DGATE : gate backward (dO = dGated*g, dg_pre = dGated*O*g(1-g), times
//               an optional row scale) and delta = rowsum(dO*O) for the
//               attention backward (fast_triton_attn.py:581-584, :601); O and g
//               rows come in by TMA
//   EPI_BF16 / EPI_F32 / EPI_RED_F32 : plain stores / split-K fp32 TMA reduce-add.
#pragma once
#include <cuda.h>

#include "ptx.cuh"

namespace mea {

// A_K_HEADS / A_MN_HEADS: A as A_K / A_MN, but stored as four [B*H*T, hd]
// tensors (per-head layout, hd a multiple of 64): logical column (A_K_HEADS)
// or row (A_MN_HEADS) j = part*H*hd + h*hd + n of token (b, t) lives in part
// `part` at row (b*H + h)*T + t, column n.  Every 64-wide chunk of j stays in
// one head, so each is one TMA box.
enum AMode : int { A_K = 0, A_MN = 1, A_K_HEADS = 2, A_MN_HEADS = 3 };
enum BMode : int { B_K = 0, B_MN = 1, B_SLABS = 2, B_MN_KSPLIT4 = 3 };
enum EpiMode : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_RED_F32 = 2, EPI_QKVG = 3, EPI_DGATE = 4 };

// out: EPI_BF16/F32/RED_F32 out[0] = D; EPI_QKVG out[0..3] = q, k, v, sigmoid(g)
// ([B*H*T, N] views); EPI_DGATE out[0] = dO ([B*H*T, N]), out[1] = dg_pre
// ([M, H*N] view of the g slot, or [B*H*T, N] with dg_heads).  in: EPI_QKVG the rotary tables f1, f2
// ([T_max, N]); EPI_DGATE O and sigmoid(g) ([B*H*T, N]).
struct GemmMaps {
  CUtensorMap a[4];  // [0] only, except A_K_HEADS / A_MN_HEADS (one per part)
  CUtensorMap b[4];
  CUtensorMap out[4];
  CUtensorMap in[2];
};

struct GemmParams {
  int M, N, K;
  int m_pairs, n_tiles, k_splits, kb_per_split, kb_total;
  int b_kb_per_src;  // B_MN_KSPLIT4: k-blocks taken from each of the 4 B tensors
  int slab_rows;     // B_SLABS: rows of one slab (= head dim)
  int* status;
  // EPI_QKVG (row_scale: x_n = diag(row_scale) x; rq, rk receive row_scale times
  // the q/k inverse RMS, the factor from an accumulator row to the normalised
  // row) and EPI_DGATE (row_scale on dg_pre).  row_scale may be NULL (1).
  float *rq, *rk;
  const float* row_scale;
  int T, H, hd;
  float eps;
  // EPI_DGATE
  float* delta;
  int dg_heads;  // dg_pre stored [B*H*T, hd] (like dO) instead of [M, H*hd]
};

// Logical index j of the 4*H*hd dimension of an A_*_HEADS operand -> part,
// head and column within the head.
__device__ __forceinline__ void heads_coord(const GemmParams& p, int j, int& part, int& h, int& n) {
  const int hn = p.H * p.hd;
  part = j / hn;
  const int rem = j - part * hn;
  h = rem / p.hd;
  n = rem - h * p.hd;
}

constexpr int GEMM_BM = 128;  // rows per CTA; a pair covers 256
constexpr int GEMM_BK = 64;
constexpr uint32_t GEMM_A_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KB
constexpr uint32_t GEMM_SMEM_LIMIT = 232448;              // 227 KB opt-in per block

// Shared memory: A ring, B ring, epilogue staging (per warp), epilogue inputs
// (rotary tables per TMEM lane quarter, or O / sigmoid(g) buffers per warp),
// barriers.  Every region starts on a 1024-byte boundary (128-byte swizzle
// atoms).  The ring takes whatever the epilogue leaves, up to 8 stages.
template <int BN, int EPI, int HD>
struct GemmCfg {
  static constexpr bool QKVG = EPI == EPI_QKVG;
  static constexpr bool DGATE = EPI == EPI_DGATE;
  // EPI_QKVG: QK_GROUPS groups of four warps (one per TMEM lane quarter), group
  // g taking the slabs s with s % QK_GROUPS == g: one slab per warp and tile for
  // N <= 64 (16 warps), one of the two for N = 128 (8 warps).
  static constexpr int QK_GROUPS = QKVG ? (HD >= 128 ? 2 : 4) : 1;
  // EPI_DGATE: DG_GROUPS groups of four warps, group g taking the heads s with
  // s % DG_GROUPS == g; each warp streams its heads through two in-place buffers.
  static constexpr int DG_GROUPS = DGATE ? (HD >= 128 ? 1 : 2) : 1;
  static constexpr int EPI_WARPS = 4 * QK_GROUPS * DG_GROUPS;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr uint32_t B_BYTES = (BN / 2) * GEMM_BK * 2;
  static constexpr uint32_t STAGE_BYTES = GEMM_A_BYTES + B_BYTES;
  static constexpr uint32_t WARP_STG = QKVG ? 64u * BN / QK_GROUPS
                                       : EPI == EPI_BF16 ? 64u * BN
                                       : DGATE ? 0u
                                               : 32u * (BN < 128 ? BN : 128) * 4;
  static constexpr uint32_t STAGING = EPI_WARPS * WARP_STG;
  // DGATE: per warp two buffers of one head's O and sigmoid(g) rows (32 x HD
  // each), overwritten in place by dO and dg_pre and stored from there.
  static constexpr uint32_t INPUTS = QKVG ? 512u * HD : DGATE ? EPI_WARPS * 2u * 128u * HD : 0;
  static constexpr int AUX_BARS = 16;
  static constexpr uint32_t FIXED = 1024 + STAGING + INPUTS + 512;
  static constexpr int STAGES_FIT = int((GEMM_SMEM_LIMIT - FIXED) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = FIXED + size_t(STAGES) * STAGE_BYTES;
  static_assert(STAGES >= 3, "GEMM: shared memory leaves fewer than 3 pipeline stages");
  static_assert(WARP_STG % 1024 == 0 && INPUTS % 1024 == 0, "GEMM: 1024-byte regions");
};

// Work unit u -> pair row base m0 (256 rows), column base n0, k-block range.
__device__ __forceinline__ void gemm_decode(const GemmParams& p, int BN, int u, int& m0, int& n0, int& kb0, int& kb1) {
  const int mn = p.m_pairs * p.n_tiles;
  const int split = u / mn;
  const int r = u - split * mn;
  const int mt = r / p.n_tiles;
  const int nt = r - mt * p.n_tiles;
  m0 = mt * 2 * GEMM_BM;
  n0 = nt * BN;
  kb0 = split * p.kb_per_split;
  kb1 = min(kb0 + p.kb_per_split, p.kb_total);
}

// ---------------------------------------------------------------------------
// Staging geometry.  A box is 32 rows (one warp's TMEM lane quarter) of a tile
// 64 elements wide (128-byte rows, 128-byte swizzle: 16-byte unit u of row r at
// u ^ (r & 7)) or 32 bf16 wide (64-byte rows, 64-byte swizzle: unit u at
// u ^ ((r >> 1) & 3)) -- the layouts TMA reads and writes for those swizzle
// modes.  With one row per lane, a warp's 16-byte accesses of one unit column
// touch every bank exactly four times (the minimum for 512 bytes).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t swz128(uint32_t box, int r, int u) { return box + r * 128 + ((u ^ (r & 7)) << 4); }
__device__ __forceinline__ uint32_t swz64(uint32_t box, int r, int u) {
  return box + r * 64 + ((u ^ ((r >> 1) & 3)) << 4);
}
// Unit u of row r in a 32-row tile HD bf16 wide (boxes of 64 columns, 4 KB each).
template <int HD>
__device__ __forceinline__ uint32_t hd_unit(uint32_t tile, int r, int u) {
  if constexpr (HD == 32) return swz64(tile, r, u);
  else return swz128(tile + (u >> 3) * 4096, r, u & 7);
}
__device__ __forceinline__ void sts_v4(uint32_t addr, const uint32_t* w) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
               : "memory");
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// Hand this warp's share of an accumulator buffer back to the pair's MMA issuer.
__device__ __forceinline__ void release_acc(uint32_t acce_cl, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(acce_cl);
}
// Before a warp rewrites its staging tile: its previous TMA stores have read it.
__device__ __forceinline__ void staging_acquire(int lane) {
  if (lane == 0) bulk_wait_read0();
  __syncwarp();
}
// After a warp's st.shared of a staging tile: visible to the TMA (async proxy).
__device__ __forceinline__ void staging_publish() {
  fence_proxy_async_smem();
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Epilogues.  `taddr` is this warp's TMEM lane quarter + accumulator column 0;
// `row0` the output row of lane 0, `stg` this warp's staging tile.
// ---------------------------------------------------------------------------
template <int BN>
__device__ __forceinline__ void epi_bf16(const GemmMaps& maps, uint32_t taddr, uint32_t stg, int lane, int row0, int n0,
                                         uint32_t acce_cl) {
  staging_acquire(lane);
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    uint32_t r0[32], r1[32];
    tmem_ld32(taddr + c, r0);
    tmem_ld32(taddr + c + 32, r1);
    tmem_wait_ld_tied2x32(r0, r1);
    const uint32_t box = stg + (c >> 6) * 4096;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* r = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
      const uint32_t w[4] = {pack_bf16(__uint_as_float(r[0]), __uint_as_float(r[1])),
                             pack_bf16(__uint_as_float(r[2]), __uint_as_float(r[3])),
                             pack_bf16(__uint_as_float(r[4]), __uint_as_float(r[5])),
                             pack_bf16(__uint_as_float(r[6]), __uint_as_float(r[7]))};
      sts_v4(swz128(box, lane, j), w);
    }
  }
  release_acc(acce_cl, lane);
  staging_publish();
  if (lane == 0) {
#pragma unroll
    for (int bx = 0; bx < BN / 64; ++bx) tma_store_2d(&maps.out[0], stg + bx * 4096, n0 + 64 * bx, row0);
    bulk_commit();
  }
}

// fp32 output (RED: TMA reduce-add into it), 128 columns per staging round.
template <int BN, bool RED>
__device__ __forceinline__ void epi_f32(const GemmMaps& maps, uint32_t taddr, uint32_t stg, int lane, int row0, int n0,
                                        uint32_t acce_cl) {
  constexpr int CH = BN < 128 ? BN : 128;
#pragma unroll 1
  for (int h = 0; h < BN; h += CH) {
    staging_acquire(lane);
#pragma unroll 1
    for (int c = 0; c < CH; c += 32) {
      uint32_t r[32];
      tmem_load32(taddr + h + c, r);
      const uint32_t box = stg + (c >> 5) * 4096;
#pragma unroll
      for (int j = 0; j < 8; ++j) sts_v4(swz128(box, lane, j), r + 4 * j);
    }
    if (h + CH >= BN) release_acc(acce_cl, lane);
    staging_publish();
    if (lane == 0) {
#pragma unroll
      for (int bx = 0; bx < CH / 32; ++bx) {
        if (RED) tma_reduce_add_2d(&maps.out[0], stg + bx * 4096, n0 + h + 32 * bx, row0);
        else tma_store_2d(&maps.out[0], stg + bx * 4096, n0 + h + 32 * bx, row0);
      }
      bulk_commit();
    }
  }
}

// q or k slab of this lane's row: per-head RMSNorm over the head dim, bf16
// rounding of the normed value, then interleaved rotary
//   out[n] = qn[n]*f1[t,n] + qn[n^1]*f2[t,n]      (fast_triton_attn.py:102-106, :132-141)
// with the rotary-table row read from the quarter's table tile.  `rs` is the
// row's input-norm scale (1 when the GEMM input is already normalised).
// EARLY (HD <= 64, the slab is the warp's last TMEM read of the tile): hand the
// accumulator back (release_acc on acce_cl) as soon as the slab is in registers.
template <int HD, bool EARLY = false>
__device__ __forceinline__ void qk_slab(const GemmParams& p, uint32_t tcol, uint32_t slab, uint32_t tab, int lane,
                                        int typ, float rs, size_t bht, bool valid, uint32_t acce_cl = 0) {
  static_assert(!EARLY || HD <= 64, "early release needs the whole slab in registers");
  constexpr int NCH = HD / 32;
  constexpr uint32_t TAB_BYTES = 32 * HD * 2;
  uint32_t v[HD <= 64 ? NCH : 1][32];
  float ss0 = 0.f, ss1 = 0.f;
  if constexpr (HD <= 64) {
    tmem_ld32(tcol, v[0]);
    if constexpr (NCH == 2) {
      tmem_ld32(tcol + 32, v[NCH - 1]);
      tmem_wait_ld_tied2x32(v[0], v[NCH - 1]);
    } else {
      tmem_wait_ld_tied(v[0]);
    }
    if constexpr (EARLY) release_acc(acce_cl, lane);
#pragma unroll
    for (int ci = 0; ci < NCH; ++ci)
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float x0 = __uint_as_float(v[ci][j]), x1 = __uint_as_float(v[ci][j + 1]);
        ss0 = fmaf(x0, x0, ss0);
        ss1 = fmaf(x1, x1, ss1);
      }
  } else {
#pragma unroll 1
    for (int ci = 0; ci < NCH; ++ci) {
      uint32_t w[32];
      tmem_load32(tcol + 32 * ci, w);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float x0 = __uint_as_float(w[j]), x1 = __uint_as_float(w[j + 1]);
        ss0 = fmaf(x0, x0, ss0);
        ss1 = fmaf(x1, x1, ss1);
      }
    }
  }
  const float inv = rsqrtf((ss0 + ss1) * (rs * rs) / float(HD) + p.eps);
  const float sc = rs * inv;  // accumulator row -> normalised row
  if (valid) {
    float* rdst = typ == 0 ? p.rq : p.rk;
    if (rdst) rdst[bht] = sc;
  }
#pragma unroll
  for (int ci = 0; ci < NCH; ++ci) {
    uint32_t wbuf[32];
    const uint32_t* w;
    if constexpr (HD <= 64) {
      w = v[ci];
    } else {
      tmem_load32(tcol + 32 * ci, wbuf);
      w = wbuf;
    }
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      const int u = 4 * ci + j4;
      const uint4 a1 = lds_v4(hd_unit<HD>(tab, lane, u));
      const uint4 a2 = lds_v4(hd_unit<HD>(tab + TAB_BYTES, lane, u));
      const uint32_t x1[4] = {a1.x, a1.y, a1.z, a1.w}, x2[4] = {a2.x, a2.y, a2.z, a2.w};
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 8 * j4 + 2 * e;
        const float qa = round_bf16(__uint_as_float(w[j]) * sc);
        const float qb = round_bf16(__uint_as_float(w[j + 1]) * sc);
        pk[e] = pack_bf16(qa * bf16_lo(x1[e]) + qb * bf16_lo(x2[e]), qb * bf16_hi(x1[e]) + qa * bf16_hi(x2[e]));
      }
      sts_v4(hd_unit<HD>(slab, lane, u), pk);
    }
  }
}

// v slab (stored as is, fast_triton_attn.py:108) or g slab (sigmoid, :123).
// 32 columns of one slab chunk from registers into the staging slab.
template <int HD>
__device__ __forceinline__ void vg_chunk(const uint32_t (&w)[32], int ci, uint32_t slab, int lane, bool sig, float rs) {
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4) {
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = 8 * j4 + 2 * e;
      float a = __uint_as_float(w[j]) * rs;
      float b = __uint_as_float(w[j + 1]) * rs;
      if (sig) {
        a = __fdividef(1.0f, 1.0f + __expf(-a));
        b = __fdividef(1.0f, 1.0f + __expf(-b));
      }
      pk[e] = pack_bf16(a, b);
    }
    sts_v4(hd_unit<HD>(slab, lane, 4 * ci + j4), pk);
  }
}
// EARLY (HD <= 64): the whole slab is loaded first and the accumulator handed
// back (release_acc on acce_cl) before the stores, as in qk_slab.
template <int HD, bool EARLY = false>
__device__ __forceinline__ void vg_slab(uint32_t tcol, uint32_t slab, int lane, bool sig, float rs,
                                        uint32_t acce_cl = 0) {
  if constexpr (EARLY) {
    static_assert(HD <= 64, "early release needs the whole slab in registers");
    constexpr int NCH = HD / 32;
    uint32_t v[NCH][32];
    tmem_ld32(tcol, v[0]);
    if constexpr (NCH == 2) {
      tmem_ld32(tcol + 32, v[NCH - 1]);
      tmem_wait_ld_tied2x32(v[0], v[NCH - 1]);
    } else {
      tmem_wait_ld_tied(v[0]);
    }
    release_acc(acce_cl, lane);
#pragma unroll
    for (int ci = 0; ci < NCH; ++ci) vg_chunk<HD>(v[ci], ci, slab, lane, sig, rs);
  } else {
#pragma unroll 1
    for (int ci = 0; ci < HD / 32; ++ci) {
      uint32_t w[32];
      tmem_load32(tcol + 32 * ci, w);
      vg_chunk<HD>(w, ci, slab, lane, sig, rs);
    }
  }
}

// Projection epilogue of one tile for this warp: its group's slabs (s % G ==
// wg) of its 32 rows, staged per slab and written by TMA to the slab's
// [B,H,T,N] output.  q/k slabs wait for the quarter's rotary-table tile.
template <int BN, int HD>
__device__ __forceinline__ void epi_qkvg(const GemmMaps& maps, const GemmParams& p, uint32_t taddr, uint32_t stg,
                                         uint32_t tab, uint32_t tab_full, uint32_t tab_empty, uint32_t tab_par,
                                         int lane, int wg, int mq, int n0, uint32_t acce_cl, Guard& g) {
  constexpr int G = HD >= 128 ? 2 : 4;  // warp groups splitting the slabs (GemmCfg::QK_GROUPS)
  constexpr int NJ = BN / HD / G;
  constexpr uint32_t SLAB_BYTES = 32 * HD * 2;
  // One slab per warp and tile (BN = 256, HD = 64): the slab's TMEM loads are the
  // warp's last reads of the accumulator, so it is handed back to the MMA issuer
  // right after them, before the norm / rotary / sigmoid math and the stores.
  constexpr bool EARLY = NJ == 1 && HD <= 64;
  const int b = mq / p.T;
  const int tq = mq - b * p.T;  // token of lane 0
  const int m = mq + lane;
  const bool valid = m < p.M;
  const float rs = p.row_scale ? __ldg(p.row_scale + (valid ? m : p.M - 1)) : 1.0f;
  staging_acquire(lane);
  bool any_qk = false;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int s = wg + G * j;
    const int sg = n0 / HD + s;
    const int typ = sg & 3;
    if (typ < 2) {
      if (!any_qk) {
        bool ok = mbar_wait(tab_full, tab_par, g, 7);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) g.ok = false;
        any_qk = true;
      }
      const size_t bht = (size_t(b) * p.H + (sg >> 2)) * p.T + tq + lane;
      qk_slab<HD, EARLY>(p, taddr + s * HD, stg + j * SLAB_BYTES, tab, lane, typ, rs, bht, valid, acce_cl);
    } else {
      vg_slab<HD, EARLY>(taddr + s * HD, stg + j * SLAB_BYTES, lane, typ == 3, rs, acce_cl);
    }
  }
  if (any_qk) {
    __syncwarp();
    if (lane == 0) mbar_arrive(tab_empty);
  }
  if constexpr (!EARLY) release_acc(acce_cl, lane);
  staging_publish();
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int sg = n0 / HD + wg + G * j;
      const int row = (b * p.H + (sg >> 2)) * p.T + tq;
#pragma unroll
      for (int bx = 0; bx < (HD + 63) / 64; ++bx)
        tma_store_2d(&maps.out[sg & 3], stg + j * SLAB_BYTES + bx * 4096, 64 * bx, row);
    }
    bulk_commit();
  }
}

// Gate backward on the dGated = dY * Wo tile (fast_triton_attn.py:576-584, :601):
//   dO = dGated*g  -> [B,H,T,N] bf16 (input of the attention backward)
//   dg_pre = dGated*O*g*(1-g) -> the g slot of the projection-gradient buffer
//   delta = rowsum(dO*O) per (b,h,t)  (the attention backward's D term)
// Each warp streams the heads s (s % G == its group) of its 32 rows through two
// buffers: O and sigmoid(g) of a head come in by TMA, are overwritten in place
// by dO and dg_pre (each lane reads and then writes the same 16-byte units of
// its own row) and go out by TMA from there.  The next head's load (of this
// tile, or the first of the warp's next tile) is issued while this head is
// processed.  `hc` counts the warp's heads (buffer hc & 1, phase (hc >> 1) & 1).
template <int HD>
__device__ __forceinline__ void dgate_issue(const GemmMaps& maps, uint32_t buf, uint32_t bar, int b, int H, int T,
                                            int tq, int head) {
  constexpr uint32_t TILE = 32 * HD * 2;
  const int row = (b * H + head) * T + tq;
  mbar_expect_tx(bar, 2 * TILE);
#pragma unroll
  for (int bx = 0; bx < (HD + 63) / 64; ++bx) {
    tma_load_2d(buf + bx * 4096, &maps.in[0], bar, 64 * bx, row);
    tma_load_2d(buf + TILE + bx * 4096, &maps.in[1], bar, 64 * bx, row);
  }
}

template <int BN, int HD, int G>
__device__ __forceinline__ void epi_dgate(const GemmMaps& maps, const GemmParams& p, uint32_t taddr, uint32_t inb,
                                          uint32_t in_bar, uint32_t& hc, int lane, int wg, int mq, int n0,
                                          bool has_next, int next_mq, int next_n0, uint32_t acce_cl, Guard& g) {
  constexpr int NJ = BN / HD / G;
  constexpr uint32_t TILE = 32 * HD * 2;
  const int b = mq / p.T;
  const int tq = mq - b * p.T;
  const bool valid = mq + lane < p.M;
  // Optional per-row factor on dg_pre (the input RMSNorm's r: the weight and
  // input gradients then read x instead of x_n).
  const float rs = p.row_scale ? __ldg(p.row_scale + (valid ? mq + lane : p.M - 1)) : 1.0f;
#pragma unroll 1
  for (int j = 0; j < NJ; ++j, ++hc) {
    const int head = n0 / HD + wg + G * j;
    const uint32_t buf = inb + (hc & 1) * 2 * TILE;
    const uint32_t bar = in_bar + 8 * (hc & 1);
    // The other buffer's last store has read it: refill it with the next head.
    staging_acquire(lane);
    if (lane == 0) {
      const uint32_t nbuf = inb + ((hc + 1) & 1) * 2 * TILE, nbar = in_bar + 8 * ((hc + 1) & 1);
      if (j + 1 < NJ) {
        dgate_issue<HD>(maps, nbuf, nbar, b, p.H, p.T, tq, head + G);
      } else if (has_next) {
        const int nb = next_mq / p.T;
        dgate_issue<HD>(maps, nbuf, nbar, nb, p.H, p.T, next_mq - nb * p.T, next_n0 / HD + wg);
      }
    }
    bool ok = mbar_wait(bar, (hc >> 1) & 1, g, 8);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      g.ok = false;
      break;
    }
    float dsum = 0.f;
#pragma unroll 1
    for (int ci = 0; ci < HD / 32; ++ci) {
      uint32_t r[32];
      tmem_load32(taddr + (wg + G * j) * HD + 32 * ci, r);
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        const int u = 4 * ci + j4;
        const uint32_t ao = hd_unit<HD>(buf, lane, u), ag = hd_unit<HD>(buf + TILE, lane, u);
        const uint4 ov = lds_v4(ao);
        const uint4 gv = lds_v4(ag);
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t pd[4], pg[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = 8 * j4 + 2 * e;
          const float o0 = bf16_lo(ow[e]), o1 = bf16_hi(ow[e]);
          const float g0 = bf16_lo(gw[e]), g1 = bf16_hi(gw[e]);
          const float d0 = __uint_as_float(r[jj]), d1 = __uint_as_float(r[jj + 1]);
          const float do0 = round_bf16(d0 * g0), do1 = round_bf16(d1 * g1);
          dsum = fmaf(do0, o0, dsum);
          dsum = fmaf(do1, o1, dsum);
          pd[e] = pack_bf16(do0, do1);
          pg[e] = pack_bf16(d0 * o0 * g0 * (1.0f - g0) * rs, d1 * o1 * g1 * (1.0f - g1) * rs);
        }
        sts_v4(ao, pd);
        sts_v4(ag, pg);
      }
    }
    if (valid) p.delta[(size_t(b) * p.H + head) * p.T + tq + lane] = dsum;
    if (j == NJ - 1) release_acc(acce_cl, lane);
    staging_publish();
    if (lane == 0) {
      const int row = (b * p.H + head) * p.T + tq;
#pragma unroll
      for (int bx = 0; bx < (HD + 63) / 64; ++bx) {
        tma_store_2d(&maps.out[0], buf + bx * 4096, 64 * bx, row);
        if (p.dg_heads)
          tma_store_2d(&maps.out[1], buf + TILE + bx * 4096, 64 * bx, row);
        else
          tma_store_2d(&maps.out[1], buf + TILE + bx * 4096, head * HD + 64 * bx, mq);
      }
      bulk_commit();
    }
  }
}

// ---------------------------------------------------------------------------
// The kernel (launched as 2-CTA clusters)
// ---------------------------------------------------------------------------
// HD: head dim for the per-head epilogues (EPI_QKVG, EPI_DGATE), 0 otherwise.
// E4M3: e4m3 operands (both K-major).  A stage still holds 128-byte rows, i.e.
// 2 * GEMM_BK one-byte elements of K, so only the K coordinate of the loads and
// the MMA kind change.
template <int BN, int AM, int BMD, int EPI, int HD, bool E4M3 = false>
__global__ void __launch_bounds__(GemmCfg<BN, EPI, HD>::THREADS, 1)
    gemm_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  using Cfg = GemmCfg<BN, EPI, HD>;
  constexpr int STAGES = Cfg::STAGES;
  static_assert(!E4M3 || (AM == A_K && BMD == B_K), "e4m3 GEMM: K-major operands only");
  constexpr int KBE = E4M3 ? 2 * GEMM_BK : GEMM_BK;  // K elements per stage
  constexpr bool A_MNMAJ = AM == A_MN || AM == A_MN_HEADS;  // A tiles M-major in shared memory
  constexpr uint32_t IDESC =
      E4M3 ? idesc_e4m3(2 * GEMM_BM, BN)
           : idesc_bf16(2 * GEMM_BM, BN, A_MNMAJ ? 1u : 0u, (BMD == B_MN || BMD == B_MN_KSPLIT4) ? 1u : 0u);
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  constexpr int HB = BN / 2;  // B columns staged by each CTA

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * GEMM_A_BYTES;
  const uint32_t sStg = sB + STAGES * Cfg::B_BYTES;
  const uint32_t sIn = sStg + Cfg::STAGING;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING + Cfg::INPUTS);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto accf_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  // QKVG: table full/empty per lane quarter; DGATE: input buffers per epilogue warp
  auto aux_bar = [&](int i) { return bar0 + 8u * (2 * STAGES + 5 + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5 + Cfg::AUX_BARS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int nunits = p.m_pairs * p.n_tiles * p.k_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 2 * Cfg::EPI_WARPS);  // every epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < Cfg::AUX_BARS; ++i) mbar_init(aux_bar(i), (Cfg::QKVG && i >= 4 && i < 8) ? 2 : 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 4; ++i) {
      tma_prefetch_desc(&maps.a[i]);
      tma_prefetch_desc(&maps.b[i]);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised before any cross-CTA copy, commit or arrive.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  Guard g(p.status, KID_GEMM);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      for (int u = pair; u < nunits && g.ok; u += npairs) {
        int m0, n0, kb0, kb1;
        gemm_decode(p, BN, u, m0, n0, kb0, kb1);
        const int mc = m0 + int(rank) * GEMM_BM;  // this CTA's rows
        const int nc = n0 + int(rank) * HB;       // this CTA's B columns
        // Per-head A and split B coordinates are set up once per unit and then
        // stepped per k-block: no integer division on this thread's k-loop.
        //  A_K_HEADS : (part, head, column) of the k-block; rows of one sequence.
        //  A_MN_HEADS: (part, head, column) of each 64-row chunk; (sequence, position) of the k-block.
        //  B_MN_KSPLIT4: source tensor and row of the k-block.
        int a_part[2] = {0, 0}, a_h[2] = {0, 0}, a_n[2] = {0, 0}, a_b = 0, a_t = 0, b_src = 0, b_kr = 0;
        if (AM == A_K_HEADS) {
          heads_coord(p, kb0 * GEMM_BK, a_part[0], a_h[0], a_n[0]);
          a_b = mc / p.T;
          a_t = mc - a_b * p.T;
        } else if (AM == A_MN_HEADS) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            // a chunk at or past M (a pair's second CTA past the end) reads part 0
            // one row past its end: zero fill, the full box still counted.
            if (mc + 64 * i < p.M) heads_coord(p, mc + 64 * i, a_part[i], a_h[i], a_n[i]);
            else a_h[i] = -1;
          }
          a_b = (kb0 * GEMM_BK) / p.T;
          a_t = kb0 * GEMM_BK - a_b * p.T;
        }
        if (BMD == B_MN_KSPLIT4) {
          b_src = kb0 / p.b_kb_per_src;
          b_kr = (kb0 - b_src * p.b_kb_per_src) * GEMM_BK;
        }
        // B_SLABS: slabs staged by each CTA, and the first one's index
        const int sl_half = BMD == B_SLABS ? BN / p.slab_rows / 2 : 0;
        const int sl_sg0 = BMD == B_SLABS ? nc / p.slab_rows : 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, g, 1)) break;
          // both CTAs' copies count on the leader's barrier; the leader expects their sum
          if (rank == 0) mbar_expect_tx(full_bar(stage), 2 * Cfg::STAGE_BYTES);
          const uint32_t fb = mapa_shared(full_bar(stage), 0);
          const uint32_t a_dst = sA + stage * GEMM_A_BYTES;
          const uint32_t b_dst = sB + stage * Cfg::B_BYTES;
          if (AM == A_K) {
            tma_load_2d_pair(a_dst, &maps.a[0], fb, kb * KBE, mc);
          } else if (AM == A_MN) {
            tma_load_2d_pair(a_dst, &maps.a[0], fb, mc, kb * GEMM_BK);
            tma_load_2d_pair(a_dst + 8192, &maps.a[0], fb, mc + 64, kb * GEMM_BK);
          } else if (AM == A_K_HEADS) {
            // 128 token rows (one sequence: T % 128 == 0) x the 64 columns of one head
            tma_load_2d_pair(a_dst, &maps.a[a_part[0]], fb, a_n[0], (a_b * p.H + a_h[0]) * p.T + a_t);
            if ((a_n[0] += GEMM_BK) == p.hd) {
              a_n[0] = 0;
              if (++a_h[0] == p.H) {
                a_h[0] = 0;
                ++a_part[0];
              }
            }
          } else {
            // 64 tokens (one sequence) x two 64-wide row chunks, each within one head
#pragma unroll
            for (int i = 0; i < 2; ++i)
              tma_load_2d_pair(a_dst + 8192 * i, &maps.a[a_part[i]], fb, a_n[i],
                               a_h[i] < 0 ? p.K * p.H : (a_b * p.H + a_h[i]) * p.T + a_t);
            if ((a_t += GEMM_BK) == p.T) {
              a_t = 0;
              ++a_b;
            }
          }
          if (BMD == B_K) {
            tma_load_2d_pair(b_dst, &maps.b[0], fb, kb * KBE, nc);
          } else if (BMD == B_MN) {
#pragma unroll
            for (int i = 0; i < HB / 64; ++i)
              tma_load_2d_pair(b_dst + 8192 * i, &maps.b[0], fb, nc + 64 * i, kb * GEMM_BK);
          } else if (BMD == B_SLABS) {
            for (int s = 0; s < sl_half; ++s) {
              const int sg = sl_sg0 + s;
              tma_load_2d_pair(b_dst + s * p.slab_rows * 128, &maps.b[sg & 3], fb, kb * GEMM_BK,
                               (sg >> 2) * p.slab_rows);
            }
          } else {
#pragma unroll
            for (int i = 0; i < HB / 64; ++i)
              tma_load_2d_pair(b_dst + 8192 * i, &maps.b[b_src], fb, nc + 64 * i, b_kr);
            if ((b_kr += GEMM_BK) == p.b_kb_per_src * GEMM_BK) {
              b_kr = 0;
              ++b_src;
            }
          }
          last_par[stage] = int(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Tail: every stage's last fill has been released by the MMA (the commits
      // that arrive on this CTA's empty barriers have landed).
      for (int s = 0; s < STAGES; ++s)
        if (last_par[s] >= 0 && g.ok) mbar_wait(empty_bar(s), uint32_t(last_par[s]), g, 6);
      if (!g.ok) {
        // Abort: let the copies in flight land (the leader's full barriers count
        // both CTAs' bytes) and the MMA's releases arrive, with short bounded waits.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) {
            if (rank == 0) mbar_drain(full_bar(s), uint32_t(last_par[s]));
            mbar_drain(empty_bar(s), uint32_t(last_par[s]));
          }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (rank == 0 && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool any = false;
      for (int u = pair; u < nunits && g.ok; u += npairs, ++it) {
        int m0, n0, kb0, kb1;
        gemm_decode(p, BN, u, m0, n0, kb0, kb1);
        const int buf = it & 1;
        if (!mbar_wait_cluster(acce_bar(buf), ((it >> 1) & 1) ^ 1, g, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, g, 3)) break;
          tc_fence_after();
          const uint32_t a_base = sA + stage * GEMM_A_BYTES;
          const uint32_t b_base = sB + stage * Cfg::B_BYTES;
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = !A_MNMAJ ? smem_desc(a_base + 32 * k, 16, 1024, SW_128B)
                                         : smem_desc(a_base + 2048 * k, 8192, 1024, SW_128B);
            const uint64_t bd = (BMD == B_K || BMD == B_SLABS) ? smem_desc(b_base + 32 * k, 16, 1024, SW_128B)
                                                                : smem_desc(b_base + 2048 * k, 8192, 1024, SW_128B);
            if constexpr (E4M3)
              mma_ss_pair_e4m3(d, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              mma_ss_pair(d, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          any = true;
          mma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!g.ok) break;
        mma_commit_pair(accf_bar(buf), 0x3);
      }
      if (!g.ok && any) {
        mma_commit_pair(drain_bar, 0x1);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ---------------- Epilogue: warps 2 .. 2+EPI_WARPS-1 (both CTAs) ----------------
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int wg = (warp - 2) >> 2;
    const uint32_t stg = sStg + (warp - 2) * Cfg::WARP_STG;
    const uint32_t acce_cl0 = mapa_shared(acce_bar(0), 0);
    const uint32_t acce_cl1 = mapa_shared(acce_bar(1), 0);
    // QKVG: the quarter's rotary-table tile (f1 then f2), loaded by the group-0 warp
    const uint32_t tab = sIn + quarter * (Cfg::QKVG ? 2 * 32 * HD * 2 : 0);
    uint32_t tab_par = 0;
    // DGATE: this warp's two head buffers and their barriers; the first head of
    // the warp's first tile is requested before the loop
    const uint32_t inb = sIn + (warp - 2) * (Cfg::DGATE ? 2 * 128 * HD : 0);
    const uint32_t in_bar = aux_bar(Cfg::DGATE ? 2 * (warp - 2) : 0);
    uint32_t hc = 0;
    if constexpr (Cfg::DGATE) {
      if (lane == 0 && pair < nunits) {
        int m0, n0, kb0, kb1;
        gemm_decode(p, BN, pair, m0, n0, kb0, kb1);
        const int mq = m0 + int(rank) * GEMM_BM + quarter * 32;
        const int b = mq / p.T;
        dgate_issue<HD>(maps, inb, in_bar, b, p.H, p.T, mq - b * p.T, n0 / HD + wg);
      }
    }
    int it = 0;
    for (int u = pair; u < nunits; u += npairs, ++it) {
      int m0, n0, kb0, kb1;
      gemm_decode(p, BN, u, m0, n0, kb0, kb1);
      const int buf = it & 1;
      const int mq = m0 + int(rank) * GEMM_BM + quarter * 32;  // row of lane 0
      if constexpr (Cfg::QKVG) {
        // rotary rows of this tile: requested before the accumulator wait
        const bool need_tab = ((n0 / HD) & 3) < 2 || (BN / HD > 2);  // the tile has q/k slabs
        const int tq = mq - (mq / p.T) * p.T;
        if (need_tab && wg == 0 && lane == 0 && mbar_wait(aux_bar(4 + quarter), tab_par ^ 1, g, 9)) {
          mbar_expect_tx(aux_bar(quarter), 2 * 32 * HD * 2);
#pragma unroll
          for (int bx = 0; bx < (HD + 63) / 64; ++bx) {
            tma_load_2d(tab + bx * 4096, &maps.in[0], aux_bar(quarter), 64 * bx, tq);
            tma_load_2d(tab + 32 * HD * 2 + bx * 4096, &maps.in[1], aux_bar(quarter), 64 * bx, tq);
          }
        }
      }
      bool ok = mbar_wait(accf_bar(buf), (it >> 1) & 1, g, 4);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        g.ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + buf * BN;
      const uint32_t acce_cl = buf ? acce_cl1 : acce_cl0;
      if constexpr (Cfg::QKVG) {
        const bool need_tab = ((n0 / HD) & 3) < 2 || (BN / HD > 2);  // the tile has q/k slabs
        epi_qkvg<BN, HD>(maps, p, taddr, stg, tab, aux_bar(quarter), aux_bar(4 + quarter), tab_par, lane, wg, mq, n0,
                         acce_cl, g);
        if (need_tab) tab_par ^= 1;
      } else if constexpr (Cfg::DGATE) {
        const bool has_next = u + npairs < nunits;
        int nm0 = 0, nn0 = 0;
        if (has_next) gemm_decode(p, BN, u + npairs, nm0, nn0, kb0, kb1);
        epi_dgate<BN, HD, Cfg::DG_GROUPS>(maps, p, taddr, inb, in_bar, hc, lane, wg, mq, n0, has_next,
                                          nm0 + int(rank) * GEMM_BM + quarter * 32, nn0, acce_cl, g);
      } else if constexpr (EPI == EPI_BF16) {
        epi_bf16<BN>(maps, taddr, stg, lane, mq, n0, acce_cl);
      } else {
        epi_f32<BN, EPI == EPI_RED_F32>(maps, taddr, stg, lane, mq, n0, acce_cl);
      }
      if (!g.ok) break;
    }
    // every TMA store / reduce of this warp has completed before the CTA exits
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  __syncthreads();
  // No CTA of the pair leaves (or frees TMEM) while the other may still use its
  // shared memory or barriers.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace mea
