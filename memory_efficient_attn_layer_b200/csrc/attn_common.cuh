// Shared-memory tile geometry shared by the attention kernels.
//
// A [rows x HD] bf16 tile is stored as HD/64 column chunks (one chunk when
// HD <= 64), each chunk `rows` rows of SWB = min(128, 2*HD) bytes with the
// matching TMA/UMMA swizzle.  The same bytes serve as a K-major operand
// (reduction over HD) and as an MN-major operand (reduction over rows).
#pragma once
#include "ptx.cuh"

namespace mea {

// Pairs of each 16-score softmax chunk whose exp2 runs as a polynomial on the
// FMA pipe (bit e = pair e, exp2_poly2); the rest use MUFU ex2.  The forward's
// softmax does little else on the FMA pipe, the backward's also forms dS there,
// so each balances the two pipes with its own share.
#ifndef MEA_POLY_FWD
#define MEA_POLY_FWD 0x4A
#endif
#ifndef MEA_POLY_BWD
#define MEA_POLY_BWD 0x4A
#endif
constexpr uint32_t kPolyPairsFwd = MEA_POLY_FWD;
constexpr uint32_t kPolyPairsBwd = MEA_POLY_BWD;

// exp2 of a pair, on the FMA pipe when `poly` (argument clamped at -127, where
// the result is negligible next to the row's largest term) else on MUFU.
__device__ __forceinline__ float2 exp2_pair(float2 t, bool poly) {
  if (poly) return exp2_poly2(make_float2(fmaxf(t.x, -127.f), fmaxf(t.y, -127.f)));
  return make_float2(ex2(t.x), ex2(t.y));
}

// Work items of the persistent attention kernels: one (b,h) and one 128-row
// tile index, paired as (k, nq-1-k) within a head.  In the backward the index
// is a key tile walking the nq - k query tiles from the diagonal, in the
// forward a query tile walking its k + 1 key tiles up to the diagonal; either
// way a pair holds nq + 1 tile steps, so CTAs striding over pairs get equal
// work.  Consecutive pairs belong to the same head, so the CTAs running at one
// time share a few heads' rows in L2.  Every role of a CTA walks the same
// sequence.
struct PairItems {
  int nq, pairs_per_head, total_pairs, stride;
  int p, side;
  __device__ PairItems(int nq_, int bh_count, int start, int stride_)
      : nq(nq_), pairs_per_head((nq_ + 1) / 2), total_pairs(bh_count * ((nq_ + 1) / 2)), stride(stride_), p(start),
        side(0) {}
  __device__ bool valid() const { return p < total_pairs; }
  __device__ void get(int& bh, int& tile) const {
    bh = p / pairs_per_head;
    const int k = p - bh * pairs_per_head;
    tile = side ? nq - 1 - k : k;
  }
  __device__ void next() {
    const int k = p % pairs_per_head;
    if (side == 0 && nq - 1 - k != k) {
      side = 1;
    } else {
      side = 0;
      p += stride;
    }
  }
};

template <int HD>
struct HeadTile {
  static constexpr int SWB = HD * 2 >= 128 ? 128 : HD * 2;   // bytes per swizzled row
  static constexpr int CHUNK_ELEMS = SWB / 2;                  // elements per row chunk
  static constexpr int NCHUNK = HD / CHUNK_ELEMS;
  static constexpr uint32_t SWZ = SWB == 128 ? SW_128B : (SWB == 64 ? SW_64B : SW_32B);

  // K-major descriptor (reduce over HD), k-step of 16 elements.
  __device__ static __forceinline__ uint64_t kmajor(uint32_t base, int rows, int kk) {
    const int e = kk * 16;
    const int chunk = e / CHUNK_ELEMS;
    const int within = (e - chunk * CHUNK_ELEMS) * 2;
    return smem_desc(base + chunk * rows * SWB + within, 16, 8 * SWB, SWZ);
  }
  // MN-major descriptor (reduce over rows; HD is the N/M side), k-step of 16 rows.
  __device__ static __forceinline__ uint64_t mnmajor(uint32_t base, int rows, int kk) {
    return smem_desc(base + kk * 16 * SWB, rows * SWB, 8 * SWB, SWZ);
  }
};

}  // namespace mea
