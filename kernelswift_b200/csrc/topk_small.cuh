// Exact per-row top-k for short rows and small k: one warp per row.
//
// Same semantics and output as topk_rows_kernel (topk.cuh; baseline/indexer.py:
// 185-205 of KernelSwift): the valid prefix of each row, top min(k, T) by value
// descending with ties by lower index, -1 / offset post-processing.  Used when
// T <= TS_MAXT and k <= 256, e.g. the reference's own indexer shape (T = 650,
// k = 128 over 20 800 rows), where a 512-thread CTA per row spent most of its time
// in block-wide scans and barriers for a row of a few hundred keys.
//
// Per row (one warp, no block-wide barrier):
//   1. stage the valid prefix as 16-bit order keys in the warp's shared memory
//      (two per word, as the row kernel does) and find the smallest and largest;
//   2. threshold: the K-th largest key is the largest t with count(key >= t) >= K,
//      found bit by bit over [kmin, kmax]; each count is a pass over the staged
//      keys and one warp reduction (no atomics: score rows hold few distinct
//      values, which would serialise a histogram's atomics);
//   3. compaction in index order with ballots: every key above the threshold and
//      the lowest-index keys equal to it, as composites (0xFFFF - key) << 16 | index;
//   4. a warp bitonic sort of the composites (value descending, index ascending)
//      and the post-processed writes.
#pragma once
#include "topk.cuh"

namespace ks {

constexpr int TS_WARPS = 8;     // rows per CTA
constexpr int TS_MAXT = 2048;   // longest row this path takes (keys staged per warp)

template <int EPL>  // composites per lane: k <= 32 EPL
__global__ void __launch_bounds__(TS_WARPS * 32) topk_small_kernel(TopkParams p) {
  constexpr int KP = 32 * EPL;
  extern __shared__ __align__(16) uint8_t ts_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t* keys = reinterpret_cast<uint16_t*>(ts_smem) + warp * TS_MAXT;
  uint32_t* sel = reinterpret_cast<uint32_t*>(ts_smem + TS_WARPS * TS_MAXT * 2) + warp * KP;
  const int64_t row = (int64_t)blockIdx.x * TS_WARPS + warp;
  if (row >= p.rows) return;  // the whole warp: nothing below waits on other warps
  const int64_t s = row % p.S;
  int64_t lim64 = p.causal ? (p.pos0 + s + 1) / p.ratio : (int64_t)p.T;
  if (lim64 > p.T) lim64 = p.T;
  if (lim64 < 0) lim64 = 0;
  const int L = (int)lim64;
  const int K = p.k;
  const uint16_t* src = p.scores + row * p.row_stride;

  // ---- 1. order keys and their range
  uint32_t kmin = 0xFFFFu, kmax = 0u;
  uint32_t kmin2 = 0xFFFFFFFFu, kmax2 = 0u;
  for (int i0 = lane * 8; i0 < L; i0 += 256) {
    if (i0 + 8 <= L) {
      const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + i0));
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
      if (maybe_negzero2(w[0]) | maybe_negzero2(w[1]) | maybe_negzero2(w[2]) | maybe_negzero2(w[3])) {
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = fold_negzero2(w[q]);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w[q] = bf16_key2(w[q]);
        kmin2 = min_u16x2(kmin2, w[q]);
        kmax2 = max_u16x2(kmax2, w[q]);
      }
      *reinterpret_cast<uint4*>(keys + i0) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int q = 0; q < 8 && i0 + q < L; ++q) {
        const uint32_t k = bf16_key(src[i0 + q]);
        keys[i0 + q] = (uint16_t)k;
        kmin = min(kmin, k);
        kmax = max(kmax, k);
      }
    }
  }
  kmin = min(kmin, min(kmin2 & 0xFFFFu, kmin2 >> 16));
  kmax = max(kmax, max(kmax2 & 0xFFFFu, kmax2 >> 16));
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  __syncwarp();

  // keys >= t in the row (every lane gets the count)
  auto count_ge = [&](uint32_t t) -> uint32_t {
    uint32_t c = 0;
    for (int i = lane * 2; i < L; i += 64) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(keys + i);
      c += (w & 0xFFFFu) >= t ? 1u : 0u;
      c += (i + 1 < L && (w >> 16) >= t) ? 1u : 0u;
    }
    return __reduce_add_sync(0xFFFFFFFFu, c);
  };

  // ---- 2. threshold (rows longer than k)
  const bool need_select = L > K;
  uint32_t thr = 0, need_eq = 0;
  if (need_select) {
    const uint32_t range = kmax - kmin;
    uint32_t d = 0;  // largest d with count(key >= kmin + d) >= K (count is non-increasing in d)
    for (int bit = range ? 31 - __clz(range) : -1; bit >= 0; --bit) {
      const uint32_t cand = d + (1u << bit);
      if (cand <= range && count_ge(kmin + cand) >= (uint32_t)K) d = cand;
    }
    thr = kmin + d;
    need_eq = (uint32_t)K - (thr < 0xFFFFu ? count_ge(thr + 1) : 0u);
  }

  // ---- 3. compaction in index order
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t g = 0, e = 0;  // keys above / equal to thr before this step
  for (int base = 0; base < L; base += 32) {
    const int i = base + lane;
    const uint32_t k = i < L ? keys[i] : 0u;
    const bool gt = i < L && (!need_select || k > thr);
    const bool eq = i < L && need_select && k == thr;
    const uint32_t bg = __ballot_sync(0xFFFFFFFFu, gt), be = __ballot_sync(0xFFFFFFFFu, eq);
    const uint32_t rg = g + __popc(bg & lt), re = e + __popc(be & lt);
    int pos = -1;
    if (gt) pos = (int)(rg + (re < need_eq ? re : need_eq));
    else if (eq && re < need_eq) pos = (int)(rg + re);
    if (pos >= 0) sel[pos] = ((0xFFFFu - k) << 16) | (uint32_t)i;
    g += __popc(bg);
    e += __popc(be);
  }
  const int nsel = need_select ? K : L;
  __syncwarp();

  // ---- 4. bitonic sort of the KP composites, ascending; lane l owns l*EPL ..
  uint32_t v[EPL];
#pragma unroll
  for (int q = 0; q < EPL; ++q) {
    const int i = lane * EPL + q;
    v[q] = i < nsel ? sel[i] : 0xFFFFFFFFu;
  }
#pragma unroll
  for (int kk = 2; kk <= KP; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      if (j < EPL) {
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
          const int q2 = q ^ j;
          if (q2 > q) {
            const bool asc = ((lane * EPL + q) & kk) == 0;
            const uint32_t lo = min(v[q], v[q2]), hi = max(v[q], v[q2]);
            v[q] = asc ? lo : hi;
            v[q2] = asc ? hi : lo;
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
          const uint32_t w = __shfl_xor_sync(0xFFFFFFFFu, v[q], j / EPL);
          const int el = lane * EPL + q;
          const bool take_min = ((el & j) == 0) == ((el & kk) == 0);
          v[q] = take_min ? min(v[q], w) : max(v[q], w);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < EPL; ++q) {
    const int i = lane * EPL + q;
    if (i < K) {
      int64_t o = -1;
      if (i < nsel) {
        const int64_t idx = (int64_t)(v[q] & 0xFFFFu);
        o = (p.causal && idx >= lim64) ? -1 : idx + p.offset;
      }
      if (p.out_i64)
        reinterpret_cast<int64_t*>(p.out)[row * p.out_row_stride + i] = o;
      else
        reinterpret_cast<int32_t*>(p.out)[row * p.out_row_stride + i] = (int32_t)o;
    }
  }
}

}  // namespace ks
