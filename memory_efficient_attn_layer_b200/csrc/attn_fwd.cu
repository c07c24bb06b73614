// Causal softmax attention forward on tcgen05, with the sigmoid gate and the
// [B,H,T,N] -> [B,T,H*N] repack fused into the epilogue.
//
// Replaces the reference's ATen flash-attention call plus gate_repack_kernel
// (fast_triton_attn.py:425-457) and, in the backward, the recompute gate
// (fast_triton_attn.py:559-570).
//
// One CTA = one (b, h, 128-row query tile).  Warp 0 loads Q once and streams
// K/V tiles through a ring with TMA; warp 1 issues S_j = Q K_j^T into one of
// two TMEM score buffers and O += P_j V_j with P read straight from TMEM (the
// softmax warps overwrite S_j with bf16 P_j in place); warps 2..5 run the
// online softmax, one query row per thread.  The running max is refreshed
// lazily: O and the row sum are rescaled only when a row's max grows by more
// than 2^8, which keeps every P value <= 256.  Key tiles above the diagonal
// are never loaded (causal skipping); the diagonal tile is masked.
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
  float* lse2;              // [B,H,T]
  __nv_bfloat16* o_out;     // optional [B,H,T,N]
  int* status;
};

struct AttnFwdMaps {
  CUtensorMap q, k, v;
};

template <int HD>
struct AttnFwdCfg {
  static constexpr int STAGES = HD <= 64 ? 3 : 2;
  static constexpr uint32_t TILE_BYTES = 128 * HD * 2;
  static constexpr uint32_t O_COL = 256;  // TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+HD)
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr size_t SMEM_USED = 1024 + TILE_BYTES * (1 + 2 * STAGES) + 256;
  // All 512 TMEM columns are taken, so ask for enough shared memory that a
  // second CTA never lands on the same SM (it would only wait in tcgen05.alloc).
  static constexpr size_t SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
};

template <int HD>
__global__ void __launch_bounds__(192, 1) attn_fwd_kernel(const __grid_constant__ AttnFwdMaps maps, const AttnFwdParams p) {
  using Cfg = AttnFwdCfg<HD>;
  using Tile = HeadTile<HD>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t TB = Cfg::TILE_BYTES;
  constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0, 0);
  constexpr uint32_t IDESC_O = idesc_bf16(128, HD, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + TB;           // STAGES K tiles
  const uint32_t sV = sK + STAGES * TB;  // STAGES V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TB * (1 + 2 * STAGES));
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0;
  auto k_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto v_full = [&](int s) { return b0 + 8u * (1 + STAGES + s); };
  auto kv_empty = [&](int s) { return b0 + 8u * (1 + 2 * STAGES + s); };
  auto s_full = [&](int i) { return b0 + 8u * (1 + 3 * STAGES + i); };
  auto p_full = [&](int i) { return b0 + 8u * (3 + 3 * STAGES + i); };
  const uint32_t o_bar = b0 + 8u * (5 + 3 * STAGES);
  const uint32_t drain_bar = b0 + 8u * (6 + 3 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 3 * STAGES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int nq = p.T / 128;
  const int qt = nq - 1 - int(blockIdx.x) / BH;  // heaviest query tiles first
  const int bh = int(blockIdx.x) % BH;
  const int nkv = qt + 1;
  const int row0 = bh * p.T;  // first row of this (b,h) in the [B*H*T, HD] view

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i), 128);
    }
    mbar_init(o_bar, 1);
    mbar_init(drain_bar, 1);
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
      int last_par[STAGES];
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(kv_empty(s), ph ^ 1, g, 1)) break;
        mbar_expect_tx(k_full(s), TB);
#pragma unroll
        for (int c = 0; c < Tile::NCHUNK; ++c)
          tma_load_2d(sK + s * TB + c * 128 * Tile::SWB, &maps.k, k_full(s), c * Tile::CHUNK_ELEMS, row0 + j * 128);
        mbar_expect_tx(v_full(s), TB);
#pragma unroll
        for (int c = 0; c < Tile::NCHUNK; ++c)
          tma_load_2d(sV + s * TB + c * 128 * Tile::SWB, &maps.v, v_full(s), c * Tile::CHUNK_ELEMS, row0 + j * 128);
        last_par[s] = int(ph);
      }
      if (!g.ok) {
        mbar_drain(q_full, 0);
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) {
            mbar_drain(k_full(s), uint32_t(last_par[s]));
            mbar_drain(v_full(s), uint32_t(last_par[s]));
          }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      bool any = false;
      auto issue_pv = [&](int i) -> bool {
        const int s = i % STAGES;
        if (!mbar_wait(p_full(i & 1), (i >> 1) & 1, g, 3)) return false;
        if (!mbar_wait(v_full(s), (i / STAGES) & 1, g, 4)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + (i & 1) * 128;
#pragma unroll
        for (int kc = 0; kc < 8; ++kc)
          mma_ts(tmem + Cfg::O_COL, p_tmem + kc * 8, Tile::mnmajor(sV + s * TB, 128, kc), IDESC_O,
                 (i > 0 || kc > 0) ? 1u : 0u);
        mma_commit(kv_empty(s));
        mma_commit(o_bar);
        return true;
      };
      if (mbar_wait(q_full, 0, g, 5)) {
        for (int j = 0; j < nkv; ++j) {
          const int s = j % STAGES;
          if (!mbar_wait(k_full(s), (j / STAGES) & 1, g, 2)) break;
          tc_fence_after();
          const uint32_t s_tmem = tmem + (j & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(s_tmem, Tile::kmajor(sQ, 128, kk), Tile::kmajor(sK + s * TB, 128, kk), IDESC_S, kk > 0 ? 1u : 0u);
          mma_commit(s_full(j & 1));
          any = true;
          if (j > 0 && !issue_pv(j - 1)) break;
        }
        if (g.ok) issue_pv(nkv - 1);
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
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full(j & 1), (j >> 1) & 1, g, 6));
      if (!ok) break;
      tc_fence_after();
      const uint32_t sb = lane_base + (j & 1) * 128;
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(sb + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c]));
      tmem_ld_wait();
      float mx = -INFINITY;
      if (j == qt) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          float x = __uint_as_float(sv[c]) * p.scale_log2;
          x = c > r ? -INFINITY : x;
          sv[c] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const float x = __uint_as_float(sv[c]) * p.scale_log2;
          sv[c] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      }
      // Lazy rescale: refresh the reference max only when it grows by > 8 (log2 units).
      const bool need = mx > m_run + 8.0f;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_run;
        const float alpha = ex2(m_run - m_new);  // 0 when m_run = -inf
        if (j > 0) {
          // O holds sum_{i<j} P_i V_i: wait for PV_{j-1}, then rescale this warp's rows.
          ok = __all_sync(0xffffffffu, mbar_wait(o_bar, (j - 1) & 1, g, 7));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD; c += 16) {
            uint32_t ov[16];
            tmem_ld16(lane_base + Cfg::O_COL + c, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st16(lane_base + Cfg::O_COL + c, ov);
          }
        }
        l_run *= alpha;
        m_run = m_new;
      }
      // P = exp2(s - m), row sum, pack to bf16 pairs and store into the S buffer.
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2(__uint_as_float(sv[32 * c + 2 * e]) - m_run);
          const float p1 = ex2(__uint_as_float(sv[32 * c + 2 * e + 1]) - m_run);
          lsum += p0 + p1;
          pk[e] = pack_bf16(p0, p1);
        }
        tmem_st16(sb + 16 * c, pk);
      }
      l_run += lsum;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full(j & 1));
    }
    // ---- epilogue: O / l, gate, repack ----
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_bar, (nkv - 1) & 1, g, 8));
    if (ok) {
      tc_fence_after();
      const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
      const int t = qt * 128 + r;
      const size_t bht = size_t(bh) * p.T + t;
      const float inv_l = 1.0f / l_run;
      const __nv_bfloat16* gsrow = p.gs + bht * HD;
      __nv_bfloat16* grow = p.gated + (size_t(b) * p.T + t) * size_t(p.H * HD) + size_t(h) * HD;
      __nv_bfloat16* orow = p.o_out ? p.o_out + bht * HD : nullptr;
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        uint32_t ov[16];
        tmem_ld16(lane_base + Cfg::O_COL + c, ov);
        tmem_ld_wait();
        const uint4 g0 = *reinterpret_cast<const uint4*>(gsrow + c);
        const uint4 g1 = *reinterpret_cast<const uint4*>(gsrow + c + 8);
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
      p.lse2[bht] = m_run + __log2f(l_run);
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
  auto kern = attn_fwd_kernel<HD>;
  if (!smem_attr_set(reinterpret_cast<const void*>(kern), int(Cfg::SMEM)))
    return set_error(MEA_ERR_CUDA, "cudaFuncSetAttribute(attn_fwd) failed");
  const int grid = p.B * p.H * (p.T / 128);
  kern<<<grid, 192, Cfg::SMEM, st>>>(maps, p);
  return check_launch("attn_fwd_kernel");
}

int run_attn_fwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* gs, void* gated,
                 float* lse2, void* o_out, int* status, cudaStream_t st) {
  if (HD != 32 && HD != 64 && HD != 128)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention: head dim %d not in {32, 64, 128}", HD);
  if (T % 128 != 0 || T <= 0 || B <= 0 || H <= 0)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention: T=%d must be a positive multiple of 128", T);
  const uint64_t rows = uint64_t(B) * H * T;
  const int swb = HD * 2 >= 128 ? 128 : HD * 2;
  const int box_inner = swb / 2;
  AttnFwdMaps maps;
  const auto sw = swizzle_for(swb);
  int rc = make_tmap_2d(&maps.q, q, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.k, k, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.v, v, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  if (rc) return set_error(MEA_ERR_CUDA, "attention: tensor map encode failed");
  AttnFwdParams p;
  p.B = B;
  p.H = H;
  p.T = T;
  p.scale_log2 = 1.4426950408889634f / sqrtf(float(HD));
  p.gs = static_cast<const __nv_bfloat16*>(gs);
  p.gated = static_cast<__nv_bfloat16*>(gated);
  p.lse2 = lse2;
  p.o_out = static_cast<__nv_bfloat16*>(o_out);
  p.status = status;
  switch (HD) {
    case 32: return launch_attn_fwd_t<32>(maps, p, st);
    case 64: return launch_attn_fwd_t<64>(maps, p, st);
    default: return launch_attn_fwd_t<128>(maps, p, st);
  }
}

}  // namespace mea
