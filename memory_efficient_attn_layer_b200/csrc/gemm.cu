// Host-side set-up and dispatch of the CTA-pair tcgen05 GEMM (gemm.cuh).
#include <cstdio>

#include "gemm.cuh"
#include "launch.h"
#include "tma.h"

namespace mea {

// Persistent grid: one 2-CTA cluster per SM pair that can hold one, at most one
// per work unit.
template <int BN, int AM, int BMD, int EPI, int HD, bool E4M3 = false>
static int launch_gemm_t(const GemmMaps& maps, const GemmParams& p, cudaStream_t st) {
  using Cfg = GemmCfg<BN, EPI, HD>;
  auto kern = gemm_kernel<BN, AM, BMD, EPI, HD, E4M3>;
  if (!smem_attr_set(reinterpret_cast<const void*>(kern), int(Cfg::SMEM)))
    return set_error(MEA_ERR_CUDA, "cudaFuncSetAttribute(gemm) failed");
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_pairs[2][64] = {{0}};  // per instantiation kind and device
  int dev = 0;
  cudaGetDevice(&dev);
  int& mp = max_pairs[E4M3 ? 1 : 0][dev & 63];
  if (mp <= 0) {
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    mp = n;
  }
  const int units = p.m_pairs * p.n_tiles * p.k_splits;
  cfg.gridDim = dim3(2 * (units < mp ? units : mp));
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, p);
  char what[112];
  snprintf(what, sizeof(what), "gemm_kernel<%d,%d,%d,%d,%d%s> M=%d N=%d K=%d splits=%d", BN, AM, BMD, EPI, HD,
           E4M3 ? ",e4m3" : "", p.M, p.N, p.K, p.k_splits);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(MEA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return check_launch(what);
}

#define MEA_GEMM_CASE(BN_, AM_, BMD_, EPI_)                                   \
  if (bn == BN_ && am == AM_ && bmd == BMD_ && epi == EPI_)                   \
    return launch_gemm_t<BN_, AM_, BMD_, EPI_, 0>(maps, p, st);
// per-head epilogues: one instantiation per head dim
#define MEA_GEMM_CASE_HD(BN_, AM_, BMD_, EPI_)                                \
  if (bn == BN_ && am == AM_ && bmd == BMD_ && epi == EPI_) {                 \
    if (p.hd == 32) return launch_gemm_t<BN_, AM_, BMD_, EPI_, 32>(maps, p, st);   \
    if (p.hd == 64) return launch_gemm_t<BN_, AM_, BMD_, EPI_, 64>(maps, p, st);   \
    if (p.hd == 128) return launch_gemm_t<BN_, AM_, BMD_, EPI_, 128>(maps, p, st); \
  }

static int dispatch(int bn, int am, int bmd, int epi, bool e4m3, const GemmMaps& maps, const GemmParams& p,
                    cudaStream_t st) {
  if (e4m3) {  // e4m3 operands: K-major A and B, fp32 or bf16 output
    if (am == A_K && bmd == B_K && epi == EPI_F32)
      return bn == 256 ? launch_gemm_t<256, A_K, B_K, EPI_F32, 0, true>(maps, p, st)
                       : launch_gemm_t<128, A_K, B_K, EPI_F32, 0, true>(maps, p, st);
    if (am == A_K && bmd == B_K && epi == EPI_BF16)
      return bn == 256 ? launch_gemm_t<256, A_K, B_K, EPI_BF16, 0, true>(maps, p, st)
                       : launch_gemm_t<128, A_K, B_K, EPI_BF16, 0, true>(maps, p, st);
    return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: e4m3 operands need K-major A and B and an fp32/bf16 output");
  }
  // forward: fused projections, o_proj
  MEA_GEMM_CASE_HD(256, A_K, B_SLABS, EPI_QKVG)
  MEA_GEMM_CASE(256, A_K, B_K, EPI_BF16)
  MEA_GEMM_CASE(128, A_K, B_K, EPI_BF16)
  // backward: dGated (+ gate bwd), dx_normed, weight gradients
  MEA_GEMM_CASE_HD(256, A_K, B_MN, EPI_DGATE)
  MEA_GEMM_CASE_HD(128, A_K, B_MN, EPI_DGATE)
  MEA_GEMM_CASE(256, A_K, B_MN_KSPLIT4, EPI_BF16)
  MEA_GEMM_CASE(128, A_K, B_MN_KSPLIT4, EPI_BF16)
  MEA_GEMM_CASE(256, A_MN, B_MN, EPI_RED_F32)
  MEA_GEMM_CASE(128, A_MN, B_MN, EPI_RED_F32)
  // the same two with dAcc read from its per-head parts (head dim >= 64)
  MEA_GEMM_CASE(256, A_K_HEADS, B_MN_KSPLIT4, EPI_BF16)
  MEA_GEMM_CASE(128, A_K_HEADS, B_MN_KSPLIT4, EPI_BF16)
  MEA_GEMM_CASE(256, A_MN_HEADS, B_MN, EPI_RED_F32)
  MEA_GEMM_CASE(128, A_MN_HEADS, B_MN, EPI_RED_F32)
  // generic fp32-output GEMMs (unit tests of every operand layout)
  MEA_GEMM_CASE(256, A_K, B_K, EPI_F32)
  MEA_GEMM_CASE(128, A_K, B_K, EPI_F32)
  MEA_GEMM_CASE(256, A_MN, B_MN, EPI_F32)
  MEA_GEMM_CASE(128, A_MN, B_MN, EPI_F32)
  MEA_GEMM_CASE(256, A_K, B_MN, EPI_F32)
  MEA_GEMM_CASE(128, A_K, B_MN, EPI_F32)
  MEA_GEMM_CASE(256, A_MN, B_K, EPI_F32)
  MEA_GEMM_CASE(128, A_MN, B_K, EPI_F32)
  return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: no kernel for bn=%d amode=%d bmode=%d epi=%d hd=%d", bn, am, bmd,
                   epi, p.hd);
}
#undef MEA_GEMM_CASE
#undef MEA_GEMM_CASE_HD

// Map over a [rows, hd] bf16 tensor with boxes of 32 rows x min(hd, 64) columns,
// swizzled to match the epilogue's staging layout.
static int hd_map(CUtensorMap* m, const void* base, uint64_t rows, int hd, uint64_t pitch_elems, uint64_t cols) {
  const uint32_t box_w = hd < 64 ? uint32_t(hd) : 64u;
  return make_tmap_2d(m, base, cols, rows, pitch_elems * 2, box_w, 32, swizzle_for(box_w * 2));
}

int run_gemm(const GemmLaunch& L, GemmParams p, cudaStream_t st) {
  const int bn = L.bn;
  // K elements per 128-byte stage row: 64 bf16 or 128 e4m3
  const int kbe = L.e4m3 ? 2 * GEMM_BK : GEMM_BK;
  const int eb = L.e4m3 ? 1 : 2;  // operand element bytes
  if (bn != 128 && bn != 256) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: bn must be 128 or 256");
  if (L.M % GEMM_BM || L.N % bn || L.K % kbe || L.M <= 0 || L.N <= 0 || L.K <= 0)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gemm: M=%d N=%d K=%d must be multiples of 128/%d/%d", L.M, L.N, L.K,
                     bn, kbe);
  if (L.e4m3 && (L.amode != A_K || L.bmode != B_K))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: e4m3 operands must both be K-major");
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc;
  // A operand (this CTA's 128 rows): K-major [M rows, K] or MN-major [K rows, M],
  // or (per-head modes) four [tokens*H, hd] parts with 64-wide boxes of 128
  // (K-major) or 64 (MN-major) rows.
  const bool a_heads = L.amode == A_K_HEADS || L.amode == A_MN_HEADS;
  if (a_heads) {
    const int hd = p.hd;
    const long long tokens = L.amode == A_K_HEADS ? L.M : L.K;
    const long long hn4 = 4LL * p.H * hd;
    if (hd % 64 || hd <= 0 || p.H <= 0 || p.T % GEMM_BM || p.T <= 0 || tokens % p.T ||
        (L.amode == A_K_HEADS ? L.K : L.M) != hn4)
      return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gemm: per-head A needs hd %% 64 == 0, T %% 128 == 0, 4*H*hd = %s",
                       L.amode == A_K_HEADS ? "K" : "M");
    for (int i = 0; i < 4; ++i) {
      if (!L.a4[i]) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: A part %d is null", i);
      rc = make_tmap_2d(&maps.a[i], L.a4[i], uint64_t(hd), uint64_t(tokens) * p.H, uint64_t(hd) * 2, 64,
                        L.amode == A_K_HEADS ? 128 : 64, sw);
      if (rc) return set_error(MEA_ERR_CUDA, "gemm: A part map %d failed (%d)", i, rc);
    }
  } else {
    if (L.e4m3)
      rc = make_tmap_2d(&maps.a[0], L.a, L.K, L.M, uint64_t(L.lda) * eb, kbe, 128, sw, CU_TENSOR_MAP_DATA_TYPE_UINT8);
    else if (L.amode == A_K)
      rc = make_tmap_2d(&maps.a[0], L.a, L.K, L.M, uint64_t(L.lda) * 2, 64, 128, sw);
    else
      rc = make_tmap_2d(&maps.a[0], L.a, L.M, L.K, uint64_t(L.lda) * 2, 64, 64, sw);
    if (rc) return set_error(MEA_ERR_CUDA, "gemm: A tensor map failed (%d)", rc);
    for (int i = 1; i < 4; ++i) maps.a[i] = maps.a[0];
  }
  // B operand (this CTA's bn/2 columns)
  const int nb = (L.bmode == B_K || L.bmode == B_MN) ? 1 : 4;
  for (int i = 0; i < nb; ++i) {
    const void* src = L.b[i];
    if (!src) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: B tensor %d is null", i);
    if (L.e4m3)
      rc = make_tmap_2d(&maps.b[i], src, L.K, L.N, uint64_t(L.ldb) * eb, kbe, bn / 2, sw,
                        CU_TENSOR_MAP_DATA_TYPE_UINT8);
    else if (L.bmode == B_K)
      rc = make_tmap_2d(&maps.b[i], src, L.K, L.N, uint64_t(L.ldb) * 2, 64, bn / 2, sw);
    else if (L.bmode == B_MN)
      rc = make_tmap_2d(&maps.b[i], src, L.N, L.K, uint64_t(L.ldb) * 2, 64, 64, sw);
    else if (L.bmode == B_SLABS)
      rc = make_tmap_2d(&maps.b[i], src, L.K, L.b_rows, uint64_t(L.ldb) * 2, 64, L.slab_rows, sw);
    else
      rc = make_tmap_2d(&maps.b[i], src, L.N, L.b_rows, uint64_t(L.ldb) * 2, 64, 64, sw);
    if (rc) return set_error(MEA_ERR_CUDA, "gemm: B tensor map %d failed (%d)", i, rc);
  }
  for (int i = nb; i < 4; ++i) maps.b[i] = maps.b[0];

  // Epilogue maps
  if (L.epi == EPI_BF16 || L.epi == EPI_F32 || L.epi == EPI_RED_F32) {
    if (!L.out[0]) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: output is null");
    if (L.epi == EPI_BF16)
      rc = make_tmap_2d(&maps.out[0], L.out[0], L.N, L.M, uint64_t(L.ldo) * 2, 64, 32, sw);
    else
      rc = make_tmap_2d(&maps.out[0], L.out[0], L.N, L.M, uint64_t(L.ldo) * 4, 32, 32, sw,
                        CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    if (rc) return set_error(MEA_ERR_CUDA, "gemm: output tensor map failed (%d)", rc);
  } else {
    const int hd = p.hd;
    if (hd != 32 && hd != 64 && hd != 128) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: head dim %d", hd);
    const uint64_t bht = uint64_t(L.M) * p.H;  // B*H*T rows of a [B,H,T,N] tensor
    const int nout = L.epi == EPI_QKVG ? 4 : 1;
    for (int i = 0; i < nout; ++i) {
      if (!L.out[i]) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: epilogue output %d is null", i);
      if ((rc = hd_map(&maps.out[i], L.out[i], bht, hd, hd, hd)))
        return set_error(MEA_ERR_CUDA, "gemm: epilogue output map %d failed (%d)", i, rc);
    }
    if (L.epi == EPI_DGATE) {
      if (!L.out[1]) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: dg output is null");
      if (p.dg_heads)
        rc = hd_map(&maps.out[1], L.out[1], bht, hd, hd, hd);
      else
        rc = hd_map(&maps.out[1], L.out[1], uint64_t(L.M), hd, uint64_t(L.ldo), uint64_t(p.H) * hd);
      if (rc) return set_error(MEA_ERR_CUDA, "gemm: dg output map failed (%d)", rc);
    }
    for (int i = 0; i < 2; ++i) {
      if (!L.in[i]) return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: epilogue input %d is null", i);
      if (L.epi == EPI_QKVG)
        rc = hd_map(&maps.in[i], L.in[i], uint64_t(L.in_rows), hd, uint64_t(L.ldin), hd);
      else
        rc = hd_map(&maps.in[i], L.in[i], bht, hd, hd, hd);
      if (rc) return set_error(MEA_ERR_CUDA, "gemm: epilogue input map %d failed (%d)", i, rc);
    }
  }

  p.M = L.M;
  p.N = L.N;
  p.K = L.K;
  p.m_pairs = (L.M / GEMM_BM + 1) / 2;
  p.n_tiles = L.N / bn;
  p.kb_total = L.K / kbe;
  int splits = L.k_splits < 1 ? 1 : L.k_splits;
  if (splits > p.kb_total) splits = p.kb_total;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.k_splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;  // every split non-empty
  p.slab_rows = L.slab_rows;
  p.b_kb_per_src = L.b_rows / GEMM_BK;
  if (p.k_splits > 1 && L.epi != EPI_RED_F32)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "gemm: split-K needs the reducing epilogue");
  if (L.bmode == B_SLABS && (L.slab_rows % 8 || bn % (2 * L.slab_rows)))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gemm: slab rows %d must divide %d", L.slab_rows, bn / 2);
  if (L.bmode == B_MN_KSPLIT4 && (L.b_rows % GEMM_BK || 4 * L.b_rows != L.K))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gemm: K must be 4 x rows of each B tensor");
  if ((L.epi == EPI_QKVG || L.epi == EPI_DGATE) && (p.T % GEMM_BM || L.M % p.T))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "gemm: per-head epilogue needs T %% 128 == 0 and M %% T == 0");
  return dispatch(bn, L.amode, L.bmode, L.epi, L.e4m3, maps, p, st);
}

// Split count for a long-K GEMM with few output tiles.  Each CTA pair runs
// ceil(splits * tiles / pairs) work units of kb_total / splits k-blocks; a unit
// also costs about six k-blocks' time of its own (pipeline fill and its fp32
// reduce-add epilogue, overlapped only with a following unit).  The split
// count minimising that makespan wins; ties go to fewer splits (less
// reduce-add traffic).  `waves` caps the units per pair.
int auto_splits(int m_tiles, int n_tiles, int kb_total, int waves) {
  const int units = ((m_tiles + 1) / 2) * n_tiles;
  const int pairs = num_sms() / 2;
  int best_s = 1;
  double best = 1e30;
  for (int sp = 1; sp <= kb_total / 8; ++sp) {
    const int per_pair = (sp * units + pairs - 1) / pairs;
    if (per_pair > waves) break;
    const double cost = per_pair * (double(kb_total) / sp + 6.0);
    if (cost < best - 1e-6) {
      best = cost;
      best_s = sp;
    }
  }
  return best_s;
}

}  // namespace mea
