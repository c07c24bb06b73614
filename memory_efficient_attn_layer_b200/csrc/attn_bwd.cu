// Causal softmax attention backward on tcgen05.
//
// Replaces the reference's ATen flash-attention backward
// (fast_triton_attn.py:586-596).  Inputs are the rotated q/k, v, dO, the
// saved row log-sum-exp (log2 units) and delta = rowsum(dO * O).
//
// One CTA = one (b, h, 128-row key tile); it walks the query tiles from the
// diagonal to the end (causal skipping).  Per query tile i:
//   S  = Q_i K^T,  dP = dO_i V^T         (tcgen05 into TMEM, one query row per lane)
//   P  = exp2(S*c - lse2),  dS = P (dP - delta)     (softmax warps; lse2 and delta
//                                                     are per-thread scalars)
//   dV += P^T dO_i   (P staged in swizzled shared memory, read MN-major)
//   dK += dS^T Q_i   (dS staged in shared memory, read MN-major)
//   dQ_i = dS K      (dS also written to TMEM as packed bf16: A operand from TMEM)
// dK and dV stay in TMEM for the whole walk.  The softmax warps also add each
// finished dQ_i tile (fp32) into the accumulator in global memory ([B,H,T,N],
// zeroed by the caller) and finally write dK and dV.  The dQ tile is staged in
// swizzled shared memory (64 columns at a time: two rounds for N = 128) and
// added by one TMA reduce-add per 32-column box, which keeps the reductions off
// the load/store unit that the P/dS tile stores need.
//
// Warps (four warpgroups, registers rebalanced with setmaxnreg): warpgroup 0 =
// warp 0 TMA, warp 1 MMA issue (warps 2, 3 idle); warpgroups 1-2 = softmax:
// query row = TMEM lane, warps 4..7 take key columns [0,64) and warps 8..11
// [64,128) (two warps per SM sub-partition, so one can issue while the other
// waits); warpgroup 3 = dQ read-out, one query row per thread, off the softmax
// warps' critical path.
//
// Schedules (TMEM has 512 columns):
//  * N <= 64 ("overlapped"): S [0,128), dP [128,256), dS [256,320), dV, dK, dQ
//    after it.  As soon as the softmax warps have read S_i and dP_i (st_empty),
//    the MMA warp issues S_{i+1}, dP_{i+1}, ahead of dV_i, dK_i, dQ_i, so the
//    next tile's scores are ready when the softmax warps finish storing P_i and
//    dS_i, and its exponentials overlap this tile's gradient MMAs.
//  * N = 128 ("serial"): S [0,128) (dS written over it), dP [128,256) (dQ written
//    over it after dP is read), dV [256,384), dK [384,512); S_{i+1} is issued
//    after dQ_i, and dP_{i+1} after the read-out of dQ_i.
#include "attn_common.cuh"
#include "launch.h"
#include "tma.h"

namespace mea {

struct AttnBwdParams {
  int B, H, T;
  float scale;       // softmax scale (1/sqrt(N))
  float scale_log2;  // scale * log2(e)
  const float* lse2;
  const float* delta;
  float* dq_acc;      // [B,H,T,N] fp32, accumulated
  __nv_bfloat16* dk;  // [B,H,T,N]
  __nv_bfloat16* dv;  // dv[(b*T + t)*ld_dv + h*N + n], or [B,H,T,N] like dk when dv_heads
  long long ld_dv;
  int dv_heads;
  const float* dv_scale;  // [B*T] factor on dV row (b, t), or NULL
  int* status;
};

struct AttnBwdMaps {
  CUtensorMap q, k, v, dO;
  CUtensorMap dq;  // dq_acc as [B*H*T, N] fp32, 32x128 boxes, 128-byte swizzle
  CUtensorMap dk;  // dk as [B*H*T, N] bf16, min(N,64) x 128 boxes
  CUtensorMap dv;  // dv as [B*T, ld_dv] bf16 (head h at column h*N), or as dk; min(N,64) x 128 boxes
};

template <int HD>
struct AttnBwdCfg {
  static constexpr bool OVERLAP = HD <= 64;
  static constexpr int STAGES = HD <= 64 ? 2 : 1;   // Q/dO ring depth
  static constexpr int KV_BUFS = HD <= 64 ? 2 : 1;  // K/V buffers: the next work item's load overlaps this one
  static constexpr uint32_t TB = 128 * HD * 2;
  static constexpr uint32_t PT = 128 * 128 * 2;  // one bf16 [128 x 128] P or dS tile
  static constexpr uint32_t S_COL = 0, DP_COL = 128;
  static constexpr uint32_t DS_COL = OVERLAP ? 256 : 0;
  static constexpr uint32_t DV_COL = OVERLAP ? 320 : 256;
  static constexpr uint32_t DK_COL = DV_COL + HD;
  static constexpr uint32_t DQ_COL = OVERLAP ? DK_COL + HD : DP_COL;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(!OVERLAP || DQ_COL + HD <= 512, "TMEM budget");
  // Registers per thread of each warpgroup after setmaxnreg (launched with 512
  // threads x 128 = 65536): 128 x REG_TMA_MMA + 256 x REG_SOFTMAX + 128 x
  // REG_READOUT = 65536.  At N = 128 the TMA/MMA warps' serial-schedule loop
  // needs more than 80 (it spilled to local memory there), the softmax warps
  // fit in 152.
  static constexpr int REG_TMA_MMA = HD >= 128 ? 112 : 80;
  static constexpr int REG_SOFTMAX = HD >= 128 ? 152 : 168;
  static constexpr int REG_READOUT = 96;
  static_assert(128 * REG_TMA_MMA + 256 * REG_SOFTMAX + 128 * REG_READOUT == 512 * 128, "register split");
  static constexpr uint32_t OFF_KV = 0;  // buffer b: K at OFF_KV + 2*TB*b, V right after it
  static constexpr uint32_t OFF_Q = KV_BUFS * 2 * TB, OFF_DO = OFF_Q + STAGES * TB;
  static constexpr uint32_t OFF_P = OFF_DO + STAGES * TB, OFF_DS = OFF_P + PT;
  static constexpr uint32_t OFF_LSE = OFF_DS + PT;
  static constexpr int DQ_COLS = HD <= 64 ? 32 : 64;            // dQ columns staged per round
  static constexpr int DQ_ROUNDS = HD / DQ_COLS;                // rounds per dQ tile
  static constexpr uint32_t OFF_DQ = OFF_LSE + STAGES * 1024;   // DQ_COLS/32 boxes of [128 x 32] fp32
  static constexpr uint32_t DQ_BYTES = DQ_COLS * 512;
  static constexpr uint32_t OFF_BAR = OFF_DQ + DQ_BYTES;
  static constexpr size_t SMEM = 1024 + OFF_BAR + 256;
};

// MN-major descriptor of a [128 q rows x 128 kv] bf16 tile stored as two
// 64-column chunks (16 KB apart) of 128-byte swizzled rows; k-step of 16 rows.
__device__ __forceinline__ uint64_t ptile_mn(uint32_t base, int kc) {
  return smem_desc(base + kc * 2048, 16384, 1024, SW_128B);
}

// Store 8 packed bf16 pairs of row r, key columns [16c, 16c+16), into a
// [128 x 128] tile with the swizzle the MN-major descriptor expects.
__device__ __forceinline__ void st_tile_row16(uint32_t tile, int r, int c, const uint32_t* w) {
  const uint32_t row_addr = tile + (c >> 2) * 16384 + r * 128;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int lu = (c & 3) * 2 + u;
    const uint32_t addr = row_addr + ((lu ^ (r & 7)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[4 * u]), "r"(w[4 * u + 1]),
                 "r"(w[4 * u + 2]), "r"(w[4 * u + 3])
                 : "memory");
  }
}

// P and dS for 16 key columns [16(cbase+c), 16(cbase+c)+16) of query row r.
template <bool DIAG>
__device__ __forceinline__ void bwd_chunk(const uint32_t (&sv)[16], const uint32_t (&dp)[16], int c, int cbase, int r,
                                          float2 scale2, float2 bias2, float dl, uint32_t (&pk)[32], uint32_t (&dsk)[32]) {
  const float2 dl2 = make_float2(dl, dl);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 t = ffma2(make_float2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), scale2, bias2);
    const float2 pp = exp2_pair(t, (kPolyPairsBwd >> e) & 1);
    float p0 = pp.x, p1 = pp.y;
    if (DIAG) {  // key column > query row: masked
      const int c0 = 16 * (cbase + c) + 2 * e;
      p0 = c0 > r ? 0.f : p0;
      p1 = c0 + 1 > r ? 0.f : p1;
    }
    pk[8 * c + e] = pack_bf16(p0, p1);
    const float2 ds = fmul2(make_float2(p0, p1),
                            fsub2(make_float2(__uint_as_float(dp[2 * e]), __uint_as_float(dp[2 * e + 1])), dl2));
    dsk[8 * c + e] = pack_bf16(ds.x, ds.y);
  }
}

// Half a row: key columns [64*hh, 64*hh + 64) of query row r.  S and dP stream
// out of TMEM in 16-column chunks with the next chunk's loads in flight while
// the current chunk is computed; P and dS are kept packed (bf16 pairs).
// `mid()` runs once the first two chunks are done (the caller stores them).
template <bool DIAG, class Mid>
__device__ __forceinline__ void bwd_half_row(uint32_t s_addr, uint32_t dp_addr, int hh, int r, float sl2, float neg_lse,
                                             float dl, uint32_t (&pk)[32], uint32_t (&dsk)[32], Mid&& mid) {
  const float2 scale2 = make_float2(sl2, sl2), bias2 = make_float2(neg_lse, neg_lse);
  const int col0 = 64 * hh;
  uint32_t s0[16], d0[16], s1[16], d1[16];
  tmem_ld16(s_addr + col0, s0);
  tmem_ld16(dp_addr + col0, d0);
  tmem_wait_ld_tied2(s0, d0);
#pragma unroll
  for (int c = 0; c < 4; c += 2) {
    tmem_ld16(s_addr + col0 + 16 * (c + 1), s1);
    tmem_ld16(dp_addr + col0 + 16 * (c + 1), d1);
    bwd_chunk<DIAG>(s0, d0, c, 4 * hh, r, scale2, bias2, dl, pk, dsk);
    tmem_wait_ld_tied2(s1, d1);
    if (c + 2 < 4) {
      tmem_ld16(s_addr + col0 + 16 * (c + 2), s0);
      tmem_ld16(dp_addr + col0 + 16 * (c + 2), d0);
    }
    bwd_chunk<DIAG>(s1, d1, c + 1, 4 * hh, r, scale2, bias2, dl, pk, dsk);
    if (c == 0) mid();  // chunks 0 and 1 are in pk / dsk; the next loads are in flight
    if (c + 2 < 4) tmem_wait_ld_tied2(s0, d0);
  }
}

// Stage columns [c0, c0 + NC) of row r of a dQ tile (scaled) into the fp32
// staging tile: NC/32 boxes of 128 rows x 128 bytes in the 128-byte swizzle the
// TMA reduce-add unswizzles (16-byte unit u of row r at u ^ (r & 7)).
template <int NC>
__device__ __forceinline__ void dq_stage(uint32_t dq_addr, int c0, int r, uint32_t stg, float scale) {
#pragma unroll
  for (int c = 0; c < NC; c += 16) {
    uint32_t v[16];
    tmem_load16(dq_addr + c0 + c, v);
    const int col0 = c;
    const uint32_t row = stg + (col0 >> 5) * 16384 + r * 128;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int unit = ((col0 & 31) >> 2) + u;
      asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(row + ((unit ^ (r & 7)) << 4)),
                   "f"(__uint_as_float(v[4 * u]) * scale), "f"(__uint_as_float(v[4 * u + 1]) * scale),
                   "f"(__uint_as_float(v[4 * u + 2]) * scale), "f"(__uint_as_float(v[4 * u + 3]) * scale)
                   : "memory");
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(512, 1) attn_bwd_kernel(const __grid_constant__ AttnBwdMaps maps, const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<HD>;
  using Tile = HeadTile<HD>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int KV_BUFS = Cfg::KV_BUFS;
  constexpr uint32_t TB = Cfg::TB;
  constexpr bool OVERLAP = Cfg::OVERLAP;
  constexpr uint32_t IDESC_SS = idesc_bf16(128, 128, 0, 0);  // S, dP
  constexpr uint32_t IDESC_KV = idesc_bf16(128, HD, 1, 1);   // dV, dK: A (P^T / dS^T) and B MN-major
  constexpr uint32_t IDESC_DQ = idesc_bf16(128, HD, 0, 1);   // dQ: A = dS from TMEM

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t base = smem_u32(smem);
  auto sK = [&](int b) { return base + Cfg::OFF_KV + 2 * TB * b; };
  auto sV = [&](int b) { return base + Cfg::OFF_KV + 2 * TB * b + TB; };
  auto sQ = [&](int s) { return base + Cfg::OFF_Q + s * TB; };
  auto sdO = [&](int s) { return base + Cfg::OFF_DO + s * TB; };
  const uint32_t sP = base + Cfg::OFF_P, sDS = base + Cfg::OFF_DS;
  float* lse_s = reinterpret_cast<float*>(smem + Cfg::OFF_LSE);  // [STAGES][2][128]: lse2, delta
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  const uint32_t b0 = smem_u32(bars);
  auto kv_full = [&](int b) { return b0 + 8u * b; };
  auto kv_empty = [&](int b) { return b0 + 8u * (2 + b); };
  auto qdo_full = [&](int s) { return b0 + 8u * (4 + s); };
  auto qdo_empty = [&](int s) { return b0 + 8u * (4 + STAGES + s); };
  const uint32_t st_full = b0 + 8u * (4 + 2 * STAGES);
  const uint32_t ds_full = st_full + 8;
  const uint32_t dq_full = st_full + 16;
  const uint32_t dq_empty = st_full + 24;
  const uint32_t drain_bar = st_full + 32;
  const uint32_t st_empty = st_full + 40;     // softmax warps have read S_n and dP_n
  const uint32_t stg_full = st_full + 48;     // dQ staging tile written
  const uint32_t stg_empty = st_full + 56;    // previous TMA reduce has read the staging tile
  const uint32_t kvacc_empty = st_full + 64;  // dK / dV of the previous work item read out of TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13 + 2 * STAGES);
  // (N <= 64) the dV MMAs have read the P tile / the dK MMAs the dS tile (the
  // slots after tmem_slot)
  const uint32_t p_free = st_full + 80;
  const uint32_t ds_free = st_full + 88;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nq = p.T / 128;
  const int BH = p.B * p.H;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(kv_full(b), 1);
      mbar_init(kv_empty(b), 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(qdo_full(s), 1);
      mbar_init(qdo_empty(s), 1);
    }
    mbar_init(st_full, 1);
    mbar_init(ds_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(drain_bar, 1);
    mbar_init(st_empty, 256);
    mbar_init(stg_full, 128);
    mbar_init(stg_empty, 1);
    mbar_init(kvacc_empty, 128);
    mbar_init(p_free, 1);
    mbar_init(ds_free, 1);
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
  Guard g(p.status, KID_ATTN_BWD);

  // Each warpgroup ends here: TMEM is freed once every warp is done with it.
  auto finish = [&]() {
    tc_fence_before();
    named_bar_sync(1, 512);
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
  };
  // Register shares per warpgroup: Cfg::REG_* (sum 65536).  Each role sets its
  // share first and ends in `finish`, so every role is compiled against its own
  // budget.
  if (warp < 4) {
    reg_dealloc<Cfg::REG_TMA_MMA>();
    if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k);
      tma_prefetch_desc(&maps.v);
      tma_prefetch_desc(&maps.dO);
      int last_par[STAGES];
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      int kv_par[2] = {-1, -1};
      int gstep = 0, item = 0;
      for (PairItems it(nq, BH, blockIdx.x, gridDim.x); it.valid() && g.ok; it.next(), ++item) {
        int bh, jt;
        it.get(bh, jt);
        const int row0 = bh * p.T;
        const int nsteps = nq - jt;
        // K, V of this item into buffer kb once the item that last used it has
        // finished its MMAs (kv_empty, committed after its last dQ)
        const int kb = item % KV_BUFS;
        if (item >= KV_BUFS && !mbar_wait(kv_empty(kb), uint32_t((item / KV_BUFS - 1) & 1), g, 16)) break;
        mbar_expect_tx(kv_full(kb), 2 * TB);
#pragma unroll
        for (int c = 0; c < Tile::NCHUNK; ++c) {
          tma_load_2d(sK(kb) + c * 128 * Tile::SWB, &maps.k, kv_full(kb), c * Tile::CHUNK_ELEMS, row0 + jt * 128);
          tma_load_2d(sV(kb) + c * 128 * Tile::SWB, &maps.v, kv_full(kb), c * Tile::CHUNK_ELEMS, row0 + jt * 128);
        }
        kv_par[kb] = (item / KV_BUFS) & 1;
        for (int n = 0; n < nsteps; ++n, ++gstep) {
          const int s = gstep % STAGES;
          const uint32_t ph = (gstep / STAGES) & 1;
          if (!mbar_wait(qdo_empty(s), ph ^ 1, g, 1)) break;
          const int qrow = row0 + (jt + n) * 128;
          const uint32_t fb = qdo_full(s);
          mbar_expect_tx(fb, 2 * TB + 1024);
#pragma unroll
          for (int c = 0; c < Tile::NCHUNK; ++c) {
            tma_load_2d(sQ(s) + c * 128 * Tile::SWB, &maps.q, fb, c * Tile::CHUNK_ELEMS, qrow);
            tma_load_2d(sdO(s) + c * 128 * Tile::SWB, &maps.dO, fb, c * Tile::CHUNK_ELEMS, qrow);
          }
          bulk_load(smem_u32(lse_s + s * 256), p.lse2 + qrow, 512, fb);
          bulk_load(smem_u32(lse_s + s * 256 + 128), p.delta + qrow, 512, fb);
          last_par[s] = int(ph);
        }
      }
      if (!g.ok) {
        for (int b = 0; b < 2; ++b)
          if (kv_par[b] >= 0) mbar_drain(kv_full(b), uint32_t(kv_par[b]));
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_drain(qdo_full(s), uint32_t(last_par[s]));
      } else {
        // Tail: wait for the MMA warp's release (tcgen05.commit) of every Q/dO
        // slot's and K/V buffer's last fill, so no asynchronous arrive targets
        // this CTA's shared memory after it exits.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(qdo_empty(s), uint32_t(last_par[s]), g, 15);
        for (int b = 0; b < 2; ++b)
          if (kv_par[b] >= 0) mbar_wait(kv_empty(b), uint32_t(kv_par[b]), g, 17);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      bool any = false;
      // S_g = Q_g K^T and dP_g = dO_g V^T (global step g, K/V buffer kb), committed together to st_full.
      auto issue_sdp = [&](int gs, int kb) -> bool {
        const int s = gs % STAGES;
        if (!mbar_wait(qdo_full(s), (gs / STAGES) & 1, g, 3)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_ss(tmem + Cfg::S_COL, Tile::kmajor(sQ(s), 128, kk), Tile::kmajor(sK(kb), 128, kk), IDESC_SS,
                 kk > 0 ? 1u : 0u);
        if (!OVERLAP && gs > 0) {  // dP's columns held dQ_{g-1}: wait for its read-out
          if (!mbar_wait(dq_empty, (gs - 1) & 1, g, 4)) return false;
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_ss(tmem + Cfg::DP_COL, Tile::kmajor(sdO(s), 128, kk), Tile::kmajor(sV(kb), 128, kk), IDESC_SS,
                 kk > 0 ? 1u : 0u);
        mma_commit(st_full);
        any = true;
        return true;
      };
      int gstep = 0, item = 0;
      bool first = true;
      for (PairItems it(nq, BH, blockIdx.x, gridDim.x); it.valid() && g.ok; it.next(), ++item) {
        int bh, jt;
        it.get(bh, jt);
        const int nsteps = nq - jt;
        const int kb = item % KV_BUFS;
        PairItems nx = it;
        nx.next();
        const bool has_next = nx.valid();
        const int nkb = (item + 1) % KV_BUFS;
        if (first) {  // later items' first scores are issued at the end of the previous item
          if (!mbar_wait(kv_full(kb), 0, g, 2) || !issue_sdp(gstep, kb)) break;
          first = false;
        }
        for (int n = 0; n < nsteps; ++n, ++gstep) {
          const int s = gstep % STAGES;
          const bool last = (n + 1 == nsteps);
          if (OVERLAP && (!last || has_next)) {  // S_g, dP_g read: issue the next scores now
            if (!mbar_wait(st_empty, gstep & 1, g, 12)) break;
            tc_fence_after();
            if (last && !mbar_wait(kv_full(nkb), ((item + 1) / KV_BUFS) & 1, g, 18)) break;
            if (!issue_sdp(gstep + 1, last ? nkb : kb)) break;
          }
          if (!mbar_wait(ds_full, gstep & 1, g, 5)) break;
          tc_fence_after();
          if (n == 0 && item > 0) {  // dK / dV of the previous item have been read out
            if (!mbar_wait(kvacc_empty, (item - 1) & 1, g, 19)) break;
            tc_fence_after();
          }
          // dV += P^T dO_g ; dK += dS^T Q_g  (A operands MN-major from shared memory)
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ss(tmem + Cfg::DV_COL, ptile_mn(sP, kc), Tile::mnmajor(sdO(s), 128, kc), IDESC_KV,
                   (n > 0 || kc > 0) ? 1u : 0u);
          if (OVERLAP) mma_commit(p_free);  // the next P may be stored once these have read the tile
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ss(tmem + Cfg::DK_COL, ptile_mn(sDS, kc), Tile::mnmajor(sQ(s), 128, kc), IDESC_KV,
                   (n > 0 || kc > 0) ? 1u : 0u);
          if (OVERLAP) mma_commit(ds_free);
          // Q_g and dO_g are last read by the dV and dK MMAs (dQ reads dS from TMEM
          // and K): their stage goes back to the producer before the dQ MMAs.
          mma_commit(qdo_empty(s));
          if (OVERLAP && gstep > 0) {
            if (!mbar_wait(dq_empty, (gstep - 1) & 1, g, 6)) break;
            tc_fence_after();
          }
          // dQ_g = dS K  (dS from TMEM, packed bf16)
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ts(tmem + Cfg::DQ_COL, tmem + Cfg::DS_COL + kc * 8, Tile::mnmajor(sK(kb), 128, kc), IDESC_DQ,
                   kc > 0 ? 1u : 0u);
          mma_commit(dq_full);
          if (last) mma_commit(kv_empty(kb));  // every MMA reading this K/V buffer is complete
          if (!OVERLAP && (!last || has_next)) {
            if (last && !mbar_wait(kv_full(nkb), ((item + 1) / KV_BUFS) & 1, g, 18)) break;
            if (!issue_sdp(gstep + 1, last ? nkb : kb)) break;
          }
        }
      }
      if (!g.ok && any) {
        mma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
    }
    finish();
    return;
  }
  if (warp < 12) {
    reg_alloc<Cfg::REG_SOFTMAX>();
    // ---------------- softmax warps 4..11 ----------------
    // Query row r = TMEM lane; warps 4..7 take key columns [0, 64), warps 8..11
    // [64, 128), so each sub-partition runs two softmax warps.
    const int quarter = warp & 3;
    const int hh = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int gstep = 0;
    for (PairItems it(nq, BH, blockIdx.x, gridDim.x); it.valid() && ok; it.next()) {
      int bh, jt;
      it.get(bh, jt);
      const int nsteps = nq - jt;
      for (int n = 0; n < nsteps; ++n, ++gstep) {
        const int s = gstep % STAGES;
        ok = mbar_wait(qdo_full(s), (gstep / STAGES) & 1, g, 7);
        ok = __all_sync(0xffffffffu, ok && mbar_wait(st_full, gstep & 1, g, 8));
        if (!ok) break;
        tc_fence_after();
        const float neg_lse = -lse_s[s * 256 + r];
        const float dl = lse_s[s * 256 + 128 + r];
        uint32_t pk[32], dsk[32];
        // N <= 64: the P tile is free once step g-1's dV MMAs have read it
        // (p_free), usually while this step's exponentials are still running, so
        // the first two P chunks go out mid-row and the rest right after; the dS
        // tile follows its dK MMAs (ds_free), the dS TMEM columns its dQ MMAs
        // (dq_full).  N = 128: everything after dq_full.
        auto store_p_front = [&]() {
          if (!OVERLAP) return;
          if (gstep > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(p_free, (gstep - 1) & 1, g, 23));
            if (!ok) return;
            tc_fence_after();
          }
          st_tile_row16(sP, r, 4 * hh + 0, pk);
          st_tile_row16(sP, r, 4 * hh + 1, pk + 8);
        };
        if (n == 0)  // the item's first query tile is the diagonal one
          bwd_half_row<true>(lane_base + Cfg::S_COL, lane_base + Cfg::DP_COL, hh, r, sl2, neg_lse, dl, pk, dsk,
                             store_p_front);
        else
          bwd_half_row<false>(lane_base + Cfg::S_COL, lane_base + Cfg::DP_COL, hh, r, sl2, neg_lse, dl, pk, dsk,
                              store_p_front);
        if (OVERLAP) {  // every TMEM load of S_g / dP_g has completed
          tc_fence_before();
          mbar_arrive(st_empty);
        }
        if (!ok) break;
        if (OVERLAP) {
          st_tile_row16(sP, r, 4 * hh + 2, pk + 16);
          st_tile_row16(sP, r, 4 * hh + 3, pk + 24);
          if (gstep > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(ds_free, (gstep - 1) & 1, g, 24));
            if (!ok) break;
            tc_fence_after();
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) st_tile_row16(sDS, r, 4 * hh + c, dsk + 8 * c);
        }
        if (gstep > 0) {  // the dS TMEM columns (and for N = 128 both tiles) are free once step g-1's MMAs are done
          ok = __all_sync(0xffffffffu, mbar_wait(dq_full, (gstep - 1) & 1, g, 10));
          if (!ok) break;
          tc_fence_after();
        }
        if (!OVERLAP) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            st_tile_row16(sP, r, 4 * hh + c, pk + 8 * c);
            st_tile_row16(sDS, r, 4 * hh + c, dsk + 8 * c);
          }
        }
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tmem_st16(lane_base + Cfg::DS_COL + 32 * hh + 16 * c, *reinterpret_cast<const uint32_t(*)[16]>(dsk + 16 * c));
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_full);
      }
    }
    // Tail: the last step's p_free / ds_free arrivals (tcgen05.commit) have landed
    // before the CTA exits.
    if (OVERLAP && ok && gstep > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(p_free, (gstep - 1) & 1, g, 25));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(ds_free, (gstep - 1) & 1, g, 26));
    }
    if (!ok) g.ok = false;
    finish();
    return;
  }
  {
    reg_dealloc<Cfg::REG_READOUT>();
    // ---------------- dQ / dK / dV read-out warps 12..15 ----------------
    // Row r of each finished dQ tile out of TMEM (dq_full), scaled, added into
    // the fp32 accumulator through the staging tile, DQ_COLS columns per round,
    // and one TMA reduce-add per 32-column box (the lead thread waits for all
    // 128 writers, stg_full, and the tile is reused once the previous
    // reduce-add has read it, stg_empty).  At the end of each work item the
    // same warps write its dK and dV (key row r) and hand their TMEM columns
    // to the next item's MMAs (kvacc_empty), off the softmax warps' path.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const bool lead = (warp == 12 && lane == 0);
    const uint32_t stg = base + Cfg::OFF_DQ;
    bool ok = true;
    // Staging-tile rounds (dQ column blocks, then each item's dK and dV): a round
    // starts once the previous round's TMA op has read the tile (stg_empty) and
    // its op is issued by the lead thread once all 128 writers are done (stg_full).
    int rnd = 0;
    auto stage_begin = [&]() -> bool {
      if (rnd > 0) {
        if (lead) {
          bulk_wait_read0();
          mbar_arrive(stg_empty);
        }
        return __all_sync(0xffffffffu, mbar_wait(stg_empty, (rnd - 1) & 1, g, 13));
      }
      return true;
    };
    auto stage_end = [&](auto&& issue) -> bool {
      fence_proxy_async_smem();
      mbar_arrive(stg_full);
      bool okk = true;
      if (lead) {
        okk = mbar_wait(stg_full, rnd & 1, g, 14);
        if (okk) {
          issue();
          bulk_commit();
        }
      }
      ++rnd;
      return __all_sync(0xffffffffu, okk);
    };
    // bf16 tile row r, columns [c, c+16) (packed pairs in w[0..7]) into the staging
    // tile in the swizzled layout of the dK / dV tensor maps (boxes of 64 columns).
    auto stage_bf16 = [&](int c, const uint32_t* w) {
      constexpr int BW = HD < 64 ? HD : 64;  // box width (elements)
      const uint32_t box = stg + (c / BW) * (128 * BW * 2);
#pragma unroll
      for (int u2 = 0; u2 < 2; ++u2) {
        const int u = ((c % BW) >> 3) + u2;
        const uint32_t addr = BW == 64 ? box + r * 128 + ((u ^ (r & 7)) << 4)
                                       : box + r * 64 + ((u ^ ((r >> 1) & 3)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[4 * u2]), "r"(w[4 * u2 + 1]),
                     "r"(w[4 * u2 + 2]), "r"(w[4 * u2 + 3])
                     : "memory");
      }
    };
    int gstep = 0;
    for (PairItems it(nq, BH, blockIdx.x, gridDim.x); it.valid() && ok; it.next()) {
      int bh, jt;
      it.get(bh, jt);
      const int nsteps = nq - jt;
      // This thread's dV row factor, loaded now so its latency is spent under the dQ rounds.
      const float dv_sc =
          p.dv_scale ? __ldg(p.dv_scale + size_t(bh / p.H) * p.T + jt * 128 + r) : 1.0f;
      for (int k = 0; k < nsteps && ok; ++k, ++gstep) {
        ok = __all_sync(0xffffffffu, mbar_wait(dq_full, gstep & 1, g, 9));
        if (!ok) break;
        tc_fence_after();
        constexpr int NC = Cfg::DQ_COLS, NR = Cfg::DQ_ROUNDS;
        const int qrow = bh * p.T + (jt + k) * 128;
        // N <= 64: the whole dQ tile goes to registers first, so its TMEM columns
        // return to the next dQ MMA (dq_empty) before the staging rounds.
        uint32_t v[OVERLAP ? HD / 16 : 1][16];
        if constexpr (OVERLAP) {
#pragma unroll
          for (int c = 0; c < HD / 16; ++c) tmem_ld16(lane_base + Cfg::DQ_COL + 16 * c, v[c]);
#pragma unroll
          for (int c = 0; c < HD / 16; c += 2) tmem_wait_ld_tied2(v[c], v[c + 1]);
          tc_fence_before();
          mbar_arrive(dq_empty);
        }
#pragma unroll
        for (int h = 0; h < NR && ok; ++h) {
          if (!(ok = stage_begin())) break;
          if constexpr (OVERLAP) {
#pragma unroll
            for (int c = 0; c < NC; c += 16) {
              const uint32_t* vv = v[(h * NC + c) / 16];
              const uint32_t row = stg + (c >> 5) * 16384 + r * 128;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int unit = ((c & 31) >> 2) + u;
                asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(row + ((unit ^ (r & 7)) << 4)),
                             "f"(__uint_as_float(vv[4 * u]) * p.scale), "f"(__uint_as_float(vv[4 * u + 1]) * p.scale),
                             "f"(__uint_as_float(vv[4 * u + 2]) * p.scale),
                             "f"(__uint_as_float(vv[4 * u + 3]) * p.scale)
                             : "memory");
              }
            }
          } else {
            dq_stage<NC>(lane_base + Cfg::DQ_COL, h * NC, r, stg, p.scale);
            if (h == NR - 1) {  // every TMEM load of the dQ tile has completed
              tc_fence_before();
              mbar_arrive(dq_empty);
            }
          }
          ok = stage_end([&] {
#pragma unroll
            for (int bx = 0; bx < NC / 32; ++bx)
              tma_reduce_add_2d(&maps.dq, stg + bx * 16384, h * NC + bx * 32, qrow);
          });
        }
      }
      if (!ok) break;
      // Item end: its last dq_full (waited above) completed every MMA of the item.
      // dK (scaled) and dV go out through the staging tile by TMA; their TMEM
      // columns go to the next item's MMAs (kvacc_empty) once read.
      const int b = bh / p.H, h = bh - b * p.H;
      constexpr int BW = HD < 64 ? HD : 64;
#pragma unroll 1
      for (int which = 0; which < 2 && ok; ++which) {
        if (!(ok = stage_begin())) break;
        const uint32_t col = which ? Cfg::DV_COL : Cfg::DK_COL;
        const float sc = which ? dv_sc : p.scale;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t a0[16], a1[16];
          tmem_ld16(lane_base + col + c, a0);
          tmem_ld16(lane_base + col + c + 16, a1);
          tmem_wait_ld_tied2(a0, a1);
          uint32_t w[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = pack_bf16(__uint_as_float(a0[2 * j]) * sc, __uint_as_float(a0[2 * j + 1]) * sc);
          stage_bf16(c, w);
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = pack_bf16(__uint_as_float(a1[2 * j]) * sc, __uint_as_float(a1[2 * j + 1]) * sc);
          stage_bf16(c + 16, w);
        }
        if (which) {
          tc_fence_before();
          mbar_arrive(kvacc_empty);
        }
        ok = stage_end([&] {
#pragma unroll
          for (int bx = 0; bx < HD / BW; ++bx) {
            if (which && p.dv_heads)
              tma_store_2d(&maps.dv, stg + bx * (128 * BW * 2), bx * BW, bh * p.T + jt * 128);
            else if (which)
              tma_store_2d(&maps.dv, stg + bx * (128 * BW * 2), h * HD + bx * BW, b * p.T + jt * 128);
            else
              tma_store_2d(&maps.dk, stg + bx * (128 * BW * 2), bx * BW, bh * p.T + jt * 128);
          }
        });
      }
    }
    if (lead) bulk_wait0();  // every reduce-add has landed before the CTA exits
    if (!ok) g.ok = false;
    finish();
  }
}

template <int HD>
static int launch_attn_bwd_t(const AttnBwdMaps& maps, const AttnBwdParams& p, cudaStream_t st) {
  using Cfg = AttnBwdCfg<HD>;
  static_assert(Cfg::SMEM <= 232448, "attention backward shared memory");
  auto kern = attn_bwd_kernel<HD>;
  if (!smem_attr_set(reinterpret_cast<const void*>(kern), int(Cfg::SMEM)))
    return set_error(MEA_ERR_CUDA, "cudaFuncSetAttribute(attn_bwd) failed");
  // Persistent: one CTA per SM, each striding over pairs of work items.
  const int pairs = p.B * p.H * ((p.T / 128 + 1) / 2);
  const int grid = pairs < num_sms() ? pairs : num_sms();
  kern<<<grid, 512, Cfg::SMEM, st>>>(maps, p);
  return check_launch("attn_bwd_kernel");
}

int check_attn_bwd_args(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* dO,
                        const float* lse2, const float* delta, const void* dk, const void* dv, long long ld_dv) {
  if (B <= 0 || H <= 0 || T <= 0)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "attention backward: dims must be positive (B=%d H=%d T=%d)", B, H, T);
  if (HD != 32 && HD != 64 && HD != 128)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention backward: head dim %d not in {32, 64, 128}", HD);
  if (T % 128 != 0)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention backward: T=%d must be a positive multiple of 128", T);
  if (uint64_t(B) * H * T * HD > (uint64_t(1) << 31))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention backward: B*H*T*N must stay below 2^31");
  if (!q || !k || !v || !dO || !lse2 || !delta || !dk || !dv)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "attention backward: NULL tensor pointer");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(dO)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "attention backward: q/k/v/dO must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(lse2) | reinterpret_cast<uintptr_t>(delta)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "attention backward: lse/delta must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15 || ld_dv % 8 || ld_dv < (long long)H * HD)
    return set_error(MEA_ERR_ALIGNMENT, "attention backward: dk/dv must be 16-byte aligned, ld_dv a multiple of 8 >= H*N");
  return MEA_OK;
}

int run_attn_bwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* dO,
                 const float* lse2, const float* delta, float* dq_acc, void* dk, void* dv, long long ld_dv, int* status,
                 cudaStream_t st, const float* dv_row_scale, bool dv_heads) {
  if (dv_heads) ld_dv = (long long)H * HD;
  const int rc0 = check_attn_bwd_args(B, H, T, HD, q, k, v, dO, lse2, delta, dk, dv, ld_dv);
  if (rc0 != MEA_OK) return rc0;
  if (!dq_acc || (reinterpret_cast<uintptr_t>(dq_acc) & 15))
    return set_error(MEA_ERR_ALIGNMENT, "attention backward: dq_acc must be non-NULL and 16-byte aligned");
  const uint64_t rows = uint64_t(B) * H * T;
  const int swb = HD * 2 >= 128 ? 128 : HD * 2;
  const int box_inner = swb / 2;
  const auto sw = swizzle_for(swb);
  AttnBwdMaps maps;
  int rc = make_tmap_2d(&maps.q, q, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.k, k, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.v, v, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.dO, dO, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.dq, dq_acc, HD, rows, uint64_t(HD) * 4, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
  const uint32_t bw = HD < 64 ? uint32_t(HD) : 64u;
  rc |= make_tmap_2d(&maps.dk, dk, HD, rows, uint64_t(HD) * 2, bw, 128, swizzle_for(bw * 2));
  if (dv_heads)
    rc |= make_tmap_2d(&maps.dv, dv, HD, rows, uint64_t(HD) * 2, bw, 128, swizzle_for(bw * 2));
  else
    rc |= make_tmap_2d(&maps.dv, dv, uint64_t(H) * HD, uint64_t(B) * T, uint64_t(ld_dv) * 2, bw, 128,
                       swizzle_for(bw * 2));
  if (rc) return set_error(MEA_ERR_CUDA, "attention backward: tensor map encode failed");
  AttnBwdParams p;
  p.B = B;
  p.H = H;
  p.T = T;
  p.scale = 1.0f / sqrtf(float(HD));
  p.scale_log2 = 1.4426950408889634f * p.scale;
  p.lse2 = lse2;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.ld_dv = ld_dv;
  p.dv_heads = dv_heads ? 1 : 0;
  p.dv_scale = dv_row_scale;
  p.status = status;
  switch (HD) {
    case 32: return launch_attn_bwd_t<32>(maps, p, st);
    case 64: return launch_attn_bwd_t<64>(maps, p, st);
    default: return launch_attn_bwd_t<128>(maps, p, st);
  }
}

}  // namespace mea
