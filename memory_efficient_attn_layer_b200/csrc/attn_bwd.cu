// Causal softmax attention backward on tcgen05.
//
// Replaces the reference's ATen flash-attention backward
// (fast_triton_attn.py:586-596).  Inputs are the rotated q/k, v, dO, the
// saved row log-sum-exp (log2 units) and delta = rowsum(dO * O).
//
// One CTA = one (b, h, 128-row key tile); it walks the query tiles from the
// diagonal to the end (causal skipping).  Per query tile:
//   S^T  = K Q^T,  dP^T = V dO^T                     (tcgen05, TMEM)
//   P^T  = exp2(S^T*c - lse2),  dS^T = P^T (dP^T - delta)   (compute warps)
//   dV  += P^T dO      (P^T read from TMEM, written there over S^T)
//   dK  += dS^T Q      (dS^T staged once in swizzled shared memory ...)
//   dQ   = dS K        (... and read back as an MN-major operand)
// dK and dV stay in TMEM for the whole walk; each dQ tile is added into an
// fp32 accumulator in global memory ([B,H,T,N], zeroed by the caller).
//
// TMEM columns: S^T [0,128), dP^T [128,256), dK [256,256+N), dV [256+N,256+2N),
// dQ [256+2N, 256+3N) for N <= 64; for N = 128 dQ reuses the dP^T columns
// (dP^T is fully read before dQ is written; the next dP^T waits for the dQ
// read-out).
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
  float* dq_acc;           // [B,H,T,N] fp32, accumulated
  __nv_bfloat16* dk;       // [B,H,T,N]
  __nv_bfloat16* dv;       // dv[(b*T + t)*ld_dv + h*N + n]
  long long ld_dv;
  int* status;
};

struct AttnBwdMaps {
  CUtensorMap q, k, v, dO;
};

template <int HD>
struct AttnBwdCfg {
  static constexpr int STAGES = HD <= 64 ? 2 : 1;
  static constexpr bool DQ_ALIAS = HD > 64;
  static constexpr uint32_t TB = 128 * HD * 2;
  static constexpr uint32_t DS_BYTES = 128 * 128 * 2;
  static constexpr uint32_t DK_COL = 256, DV_COL = 256 + HD;
  static constexpr uint32_t DQ_COL = DQ_ALIAS ? 128 : 256 + 2 * HD;
  static constexpr uint32_t TMEM_COLS = 512;
  // K, V, STAGES x (Q, dO), dS^T, then STAGES x (lse, delta), barriers
  static constexpr uint32_t OFF_K = 0, OFF_V = TB, OFF_Q = 2 * TB, OFF_DO = OFF_Q + STAGES * TB;
  static constexpr uint32_t OFF_DS = OFF_DO + STAGES * TB;
  static constexpr uint32_t OFF_LSE = OFF_DS + DS_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_LSE + STAGES * 1024;
  static constexpr size_t SMEM_USED = 1024 + OFF_BAR + 256;
  // One CTA per SM: all 512 TMEM columns are allocated.
  static constexpr size_t SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
};

template <int HD>
__global__ void __launch_bounds__(192, 1) attn_bwd_kernel(const __grid_constant__ AttnBwdMaps maps, const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<HD>;
  using Tile = HeadTile<HD>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t TB = Cfg::TB;
  constexpr uint32_t IDESC_SS = idesc_bf16(128, 128, 0, 0);   // S^T, dP^T
  constexpr uint32_t IDESC_KV = idesc_bf16(128, HD, 0, 1);    // dV (A from TMEM), dK (A K-major)
  constexpr uint32_t IDESC_DQ = idesc_bf16(128, HD, 1, 1);    // dQ (A = dS, MN-major)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t base = smem_u32(smem);
  const uint32_t sK = base + Cfg::OFF_K, sV = base + Cfg::OFF_V;
  auto sQ = [&](int s) { return base + Cfg::OFF_Q + s * TB; };
  auto sdO = [&](int s) { return base + Cfg::OFF_DO + s * TB; };
  const uint32_t sdS = base + Cfg::OFF_DS;
  float* lse_s = reinterpret_cast<float*>(smem + Cfg::OFF_LSE);  // [STAGES][2][128]: lse2, delta
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t kv_full = b0;
  auto qdo_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto qdo_empty = [&](int s) { return b0 + 8u * (1 + STAGES + s); };
  const uint32_t st_full = b0 + 8u * (1 + 2 * STAGES);
  const uint32_t ds_full = st_full + 8;
  const uint32_t dq_full = st_full + 16;
  const uint32_t dq_empty = st_full + 24;
  const uint32_t drain_bar = st_full + 32;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6 + 2 * STAGES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int nq = p.T / 128;
  // Head-major order: the key tiles of one (b,h) run side by side, so their dQ
  // reductions land in the same L2-resident rows; the longest walks (small jt)
  // start first within a head.
  const int bh = int(blockIdx.x) / nq;
  const int jt = int(blockIdx.x) % nq;
  (void)BH;
  const int nsteps = nq - jt;
  const int row0 = bh * p.T;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(qdo_full(s), 1);
      mbar_init(qdo_empty(s), 1);
    }
    mbar_init(st_full, 1);
    mbar_init(ds_full, 128);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
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
  Guard g(p.status, KID_ATTN_BWD);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k);
      tma_prefetch_desc(&maps.v);
      tma_prefetch_desc(&maps.dO);
      mbar_expect_tx(kv_full, 2 * TB);
#pragma unroll
      for (int c = 0; c < Tile::NCHUNK; ++c) {
        tma_load_2d(sK + c * 128 * Tile::SWB, &maps.k, kv_full, c * Tile::CHUNK_ELEMS, row0 + jt * 128);
        tma_load_2d(sV + c * 128 * Tile::SWB, &maps.v, kv_full, c * Tile::CHUNK_ELEMS, row0 + jt * 128);
      }
      int last_par[STAGES];
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      for (int n = 0; n < nsteps; ++n) {
        const int s = n % STAGES;
        const uint32_t ph = (n / STAGES) & 1;
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
      if (!g.ok) {
        mbar_drain(kv_full, 0);
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_drain(qdo_full(s), uint32_t(last_par[s]));
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      bool any = false;
      if (mbar_wait(kv_full, 0, g, 2)) {
        for (int n = 0; n < nsteps; ++n) {
          const int s = n % STAGES;
          if (!mbar_wait(qdo_full(s), (n / STAGES) & 1, g, 3)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem, Tile::kmajor(sK, 128, kk), Tile::kmajor(sQ(s), 128, kk), IDESC_SS, kk > 0 ? 1u : 0u);
          any = true;
          if (Cfg::DQ_ALIAS && n > 0) {
            if (!mbar_wait(dq_empty, (n - 1) & 1, g, 4)) break;
            tc_fence_after();
          }
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem + 128, Tile::kmajor(sV, 128, kk), Tile::kmajor(sdO(s), 128, kk), IDESC_SS, kk > 0 ? 1u : 0u);
          mma_commit(st_full);
          if (!mbar_wait(ds_full, n & 1, g, 5)) break;
          tc_fence_after();
          // dV += P^T dO  (P^T from TMEM columns [0, 64) as packed bf16)
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ts(tmem + Cfg::DV_COL, tmem + kc * 8, Tile::mnmajor(sdO(s), 128, kc), IDESC_KV,
                   (n > 0 || kc > 0) ? 1u : 0u);
          // dK += dS^T Q  (dS^T K-major over the query index)
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ss(tmem + Cfg::DK_COL, smem_desc(sdS + (kc >> 2) * 16384 + (kc & 3) * 32, 16, 1024, SW_128B),
                   Tile::mnmajor(sQ(s), 128, kc), IDESC_KV, (n > 0 || kc > 0) ? 1u : 0u);
          if (!Cfg::DQ_ALIAS && n > 0) {
            if (!mbar_wait(dq_empty, (n - 1) & 1, g, 6)) break;
            tc_fence_after();
          }
          // dQ = dS K  (dS read MN-major from the same shared-memory tile)
#pragma unroll
          for (int kc = 0; kc < 8; ++kc)
            mma_ss(tmem + Cfg::DQ_COL, smem_desc(sdS + kc * 2048, 16384, 1024, SW_128B), Tile::mnmajor(sK, 128, kc),
                   IDESC_DQ, kc > 0 ? 1u : 0u);
          mma_commit(qdo_empty(s));
          mma_commit(dq_full);
        }
      }
      if (!g.ok && any) {
        mma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ---------------- compute warps 2..5 ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row (S^T, dK, dV) / query row (dQ)
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    bool ok = true;
    for (int n = 0; n < nsteps; ++n) {
      const int s = n % STAGES;
      const int qi = jt + n;
      ok = mbar_wait(qdo_full(s), (n / STAGES) & 1, g, 7);
      ok = __all_sync(0xffffffffu, ok && mbar_wait(st_full, n & 1, g, 8));
      if (!ok) break;
      tc_fence_after();
      const float* lse = lse_s + s * 256;
      const float* dl = lse + 128;
      const bool diag = (n == 0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32], dp[32];
        tmem_ld32(lane_base + 32 * c, sv);
        tmem_ld32(lane_base + 128 + 32 * c, dp);
        tmem_ld_wait();
        uint32_t pk[16], dsp[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float pv[2], dsv[2];
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int col = 32 * c + 2 * e + h2;
            float pr = ex2(__uint_as_float(sv[2 * e + h2]) * p.scale_log2 - lse[col]);
            if (diag && col < r) pr = 0.f;
            pv[h2] = pr;
            dsv[h2] = pr * (__uint_as_float(dp[2 * e + h2]) - dl[col]);
          }
          pk[e] = pack_bf16(pv[0], pv[1]);
          dsp[e] = pack_bf16(dsv[0], dsv[1]);
        }
        tmem_st16(lane_base + 16 * c, pk);
        // dS^T row r, query columns [32c, 32c+32): 4 16-byte units of chunk c/2, swizzled.
        const uint32_t row_addr = sdS + (c >> 1) * 16384 + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int lu = (c & 1) * 4 + u;
          const uint32_t addr = row_addr + ((lu ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(dsp[4 * u]), "r"(dsp[4 * u + 1]),
                       "r"(dsp[4 * u + 2]), "r"(dsp[4 * u + 3])
                       : "memory");
        }
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      // dQ read-out: this thread owns query row r of tile qi.
      ok = __all_sync(0xffffffffu, mbar_wait(dq_full, n & 1, g, 9));
      if (!ok) break;
      tc_fence_after();
      float* dqrow = p.dq_acc + (size_t(row0) + size_t(qi) * 128 + r) * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + Cfg::DQ_COL + c, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          red_add_v4_f32(dqrow + c + 4 * j, __uint_as_float(v[4 * j]) * p.scale, __uint_as_float(v[4 * j + 1]) * p.scale,
                         __uint_as_float(v[4 * j + 2]) * p.scale, __uint_as_float(v[4 * j + 3]) * p.scale);
      }
      tc_fence_before();
      mbar_arrive(dq_empty);
    }
    // ---- epilogue: dK (scaled) and dV for key row r ----
    if (ok) {
      const int b = bh / p.H, h = bh - b * p.H;
      const int t = jt * 128 + r;
      __nv_bfloat16* dkrow = p.dk + (size_t(row0) + t) * HD;
      __nv_bfloat16* dvrow = p.dv + (size_t(b) * p.T + t) * p.ld_dv + size_t(h) * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t a[32], v[32];
        tmem_ld32(lane_base + Cfg::DK_COL + c, a);
        tmem_ld32(lane_base + Cfg::DV_COL + c, v);
        tmem_ld_wait();
        uint32_t pa[16], pv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          pa[j] = pack_bf16(__uint_as_float(a[2 * j]) * p.scale, __uint_as_float(a[2 * j + 1]) * p.scale);
          pv[j] = pack_bf16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          st_global_v4(dkrow + c + 8 * j, pa[4 * j], pa[4 * j + 1], pa[4 * j + 2], pa[4 * j + 3]);
          st_global_v4(dvrow + c + 8 * j, pv[4 * j], pv[4 * j + 1], pv[4 * j + 2], pv[4 * j + 3]);
        }
      }
    } else {
      g.ok = false;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int HD>
static int launch_attn_bwd_t(const AttnBwdMaps& maps, const AttnBwdParams& p, cudaStream_t st) {
  using Cfg = AttnBwdCfg<HD>;
  static_assert(Cfg::SMEM <= 232448, "attention backward shared memory");
  auto kern = attn_bwd_kernel<HD>;
  if (!smem_attr_set(reinterpret_cast<const void*>(kern), int(Cfg::SMEM)))
    return set_error(MEA_ERR_CUDA, "cudaFuncSetAttribute(attn_bwd) failed");
  const int grid = p.B * p.H * (p.T / 128);
  kern<<<grid, 192, Cfg::SMEM, st>>>(maps, p);
  return check_launch("attn_bwd_kernel");
}

int run_attn_bwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* dO,
                 const float* lse2, const float* delta, float* dq_acc, void* dk, void* dv, long long ld_dv, int* status,
                 cudaStream_t st) {
  if (HD != 32 && HD != 64 && HD != 128)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention backward: head dim %d not in {32, 64, 128}", HD);
  if (T % 128 != 0 || T <= 0 || B <= 0 || H <= 0)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "attention backward: T=%d must be a positive multiple of 128", T);
  if ((reinterpret_cast<uintptr_t>(lse2) | reinterpret_cast<uintptr_t>(delta)) & 15)
    return set_error(MEA_ERR_ALIGNMENT, "attention backward: lse/delta must be 16-byte aligned");
  const uint64_t rows = uint64_t(B) * H * T;
  const int swb = HD * 2 >= 128 ? 128 : HD * 2;
  const int box_inner = swb / 2;
  const auto sw = swizzle_for(swb);
  AttnBwdMaps maps;
  int rc = make_tmap_2d(&maps.q, q, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.k, k, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.v, v, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
  rc |= make_tmap_2d(&maps.dO, dO, HD, rows, uint64_t(HD) * 2, box_inner, 128, sw);
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
  p.status = status;
  switch (HD) {
    case 32: return launch_attn_bwd_t<32>(maps, p, st);
    case 64: return launch_attn_bwd_t<64>(maps, p, st);
    default: return launch_attn_bwd_t<128>(maps, p, st);
  }
}

}  // namespace mea
