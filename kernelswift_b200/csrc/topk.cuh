// Exact per-row top-k over bf16 score rows with the indexer's post-processing.
//
// Semantics follow baseline/indexer.py:185-205 of KernelSwift:
//   * causal prefill rows only have keys t < (s+1)//ratio; the rest are -inf;
//   * idx = topk(score, min(k, T)) sorted by value descending, ties by lower
//     index (the order torch.topk returns on CUDA);
//   * causal: idx >= (s+1)//ratio -> -1, else idx + offset; otherwise idx + offset.
// The reference NPU kernel (optimized/indexer_project/op_kernel/indexer_topk.asc:
// 155-248) is limited to k = 128 over 672 columns; here k <= 4096, T <= 65536.
//
// One CTA per row.  The valid prefix of the row is staged once in shared memory
// as 16-bit order keys (monotone in the bf16 value, -0.0 folded onto +0.0).
//   1. the staging pass also finds the row's smallest and largest key; a
//      histogram of (key - min) >> s over at most 1024 bins (shared atomics; s = 0
//      when the row spans at most 1024 distinct keys, as indexer score rows do)
//      and a descending block scan find the bin of the k-th largest key; when
//      s > 0 a second histogram over the low s bits, fed only by the keys of that
//      bin, finishes it.  The result is the exact threshold key `thr`, the count
//      of keys above it and how many keys equal to it are taken (lowest indices
//      first).  Bins sized to the row's key range matter: score rows hold a few
//      hundred distinct bf16 values that nearly all share one high byte, so a
//      fixed high-byte histogram sends every key of a warp to the same bin and
//      its atomics serialise;
//   2. one pass in index order compacts the selected (key, index) pairs with one
//      block-wide exclusive scan per 4096-element chunk (counts of keys above and
//      equal to `thr` packed into one word);
//   3. a stable counting sort when the selected keys span fewer than TK_CBINS values
//      (see below), else a bitonic sort of the 32-bit composites ((0xFFFF-key)<<16 | index) puts
//      them in (value desc, index asc) order; the composites are all distinct.
//      Each thread holds EPT consecutive composites in registers: strides below
//      EPT are exchanged in registers, strides within a warp by shuffles, and only
//      the strides across warps go through shared memory;
//   4. the post-processed indices are written as int64 or int32.
#pragma once
#include <type_traits>

#include "ks_device.cuh"

namespace ks {

constexpr int TK_THREADS = 512;
constexpr int TK_WARPS = TK_THREADS / 32;
constexpr int TK_PER_THREAD = 8;
constexpr int TK_CHUNK = TK_THREADS * TK_PER_THREAD;
constexpr int TK_HBITS = 10;                 // first-pass histogram: at most 1024 bins
constexpr int TK_HBINS = 1 << TK_HBITS;
constexpr int TK_HPER = TK_HBINS / TK_THREADS;
constexpr int TK_CBINS = 1024;               // counting sort: selection spans < 1024 key values

struct TopkParams {
  const uint16_t* scores;  // bf16 bits, row r at scores + r * row_stride
  int64_t row_stride;      // elements, multiple of 8
  int64_t rows;            // B * S
  int64_t S;               // rows per batch
  int64_t pos0;            // sequence position of row s = 0 (for the causal limit)
  int32_t causal, ratio, T, k;  // k = number of outputs per row = min(topk, T)
  int64_t offset;
  void* out;               // [rows, k] int64 or int32
  int32_t out_i64;
  int64_t out_row_stride;  // elements
  int32_t kpow2;           // power of two >= k
  int* status;
};

__device__ __forceinline__ uint32_t bf16_key(uint32_t u) {
  u &= 0xFFFFu;
  if (u == 0x8000u) u = 0;  // -0.0 == +0.0
  return (u & 0x8000u) ? ((~u) & 0xFFFFu) : (u | 0x8000u);
}
// bf16_key of both halves of a word: a negative half is inverted (xor 0xFFFF), a
// non-negative one gets its sign bit set (xor 0x8000).  m - (m >> 15) turns each
// half's sign bit into 0x7FFF without a borrow between the halves.  -0.0 halves
// must have been folded onto +0.0 first (fold_negzero2).
__device__ __forceinline__ uint32_t bf16_key2(uint32_t w) {
  const uint32_t m = w & 0x80008000u;
  return w ^ (0x80008000u | (m - (m >> 15)));
}
// Nonzero when some half of w may be 0x8000 (-0.0): the zero-half test on w ^ 0x8000
// per half (it can also fire for other words; fold_negzero2 then changes nothing).
__device__ __forceinline__ uint32_t maybe_negzero2(uint32_t w) {
  const uint32_t t = w ^ 0x80008000u;
  return (t - 0x00010001u) & ~t & 0x80008000u;
}
__device__ __forceinline__ uint32_t fold_negzero2(uint32_t w) {
  if ((w >> 16) == 0x8000u) w &= 0x0000FFFFu;
  if ((w & 0xFFFFu) == 0x8000u) w &= 0xFFFF0000u;
  return w;
}
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Exclusive scan of one value per thread over the block; also returns the total.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_tot,
                                                    uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < TK_WARPS ? warp_tot[lane] : 0;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t t = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < TK_WARPS) warp_tot[lane] = wi - w;  // exclusive warp offsets
    if (lane == TK_WARPS - 1) warp_tot[TK_WARPS] = wi;
  }
  __syncthreads();
  const uint32_t res = warp_tot[warp] + inc - v;
  total = warp_tot[TK_WARPS];
  __syncthreads();
  return res;
}

// Given a histogram of `nbins` (<= TK_HBINS) bins in ascending key order, find the
// bin holding the `need`-th largest element (1 <= need <= total count).  Writes
// (bin, count in the bins above it) to out2.  Thread t scans the bins of
// descending ranks t * TK_HPER ...; one block scan gives each thread its prefix.
__device__ __forceinline__ void find_bin_desc(const uint32_t* hist, int nbins, uint32_t need,
                                              uint32_t* warp_tot, uint32_t* out2) {
  uint32_t c[TK_HPER], sum = 0;
#pragma unroll
  for (int j = 0; j < TK_HPER; ++j) {
    const int r = threadIdx.x * TK_HPER + j;
    c[j] = r < nbins ? hist[nbins - 1 - r] : 0u;
    sum += c[j];
  }
  uint32_t tot;
  uint32_t run = block_excl_scan(sum, warp_tot, tot);
#pragma unroll
  for (int j = 0; j < TK_HPER; ++j) {
    if (run < need && run + c[j] >= need) {
      out2[0] = (uint32_t)(nbins - 1 - (int)(threadIdx.x * TK_HPER + j));
      out2[1] = run;
    }
    run += c[j];
  }
  __syncthreads();
}

template <int EPT>
__global__ void __launch_bounds__(TK_THREADS, 3) topk_rows_kernel(TopkParams p) {
  constexpr int NS = TK_THREADS * EPT;  // sorted composites, >= kpow2
  constexpr int NBUF = NS > TK_HBINS ? NS : TK_HBINS;
  extern __shared__ __align__(16) uint8_t tk_smem[];
  // layout: sortbuf[NBUF] u32 (the histograms before the compaction) |
  //         warp_tot[TK_WARPS+4] | misc[8] | red[2*TK_WARPS] | keys
  uint32_t* sortbuf = reinterpret_cast<uint32_t*>(tk_smem);
  uint32_t* hist = sortbuf;
  uint32_t* warp_tot = sortbuf + NBUF;
  uint32_t* misc = warp_tot + TK_WARPS + 4;
  uint32_t* red = misc + 8;
  uint16_t* keys = reinterpret_cast<uint16_t*>(red + 2 * TK_WARPS);

  const int tid = threadIdx.x;
  const int64_t row = p.rows - 1 - (int64_t)blockIdx.x;  // longest causal rows first
  const int64_t s = row % p.S;
  int64_t lim64 = p.causal ? (p.pos0 + s + 1) / p.ratio : (int64_t)p.T;
  if (lim64 > p.T) lim64 = p.T;
  if (lim64 < 0) lim64 = 0;
  const int L = (int)lim64;
  const int K = p.k;
  const uint16_t* src = p.scores + row * p.row_stride;

  // ---- stage the valid prefix as order keys; smallest and largest key
  const bool need_select = L > K;
  uint32_t kmin = 0xFFFFu, kmax = 0u;
  uint32_t kmin2 = 0xFFFFFFFFu, kmax2 = 0u;  // per half, full chunks (two keys per word)
  // the next chunk's 16 bytes are loaded while this chunk is converted, so the
  // loop does not wait out one memory latency per 8 keys
  uint4 nxt = make_uint4(0u, 0u, 0u, 0u);
  if (tid * TK_PER_THREAD + TK_PER_THREAD <= L)
    nxt = __ldcs(reinterpret_cast<const uint4*>(src + tid * TK_PER_THREAD));
  for (int base = 0; base < L; base += TK_CHUNK) {
    const int i0 = base + tid * TK_PER_THREAD;
    uint32_t kv[TK_PER_THREAD];
    const uint4 v = nxt;
    if (i0 + TK_CHUNK + TK_PER_THREAD <= L)
      nxt = __ldcs(reinterpret_cast<const uint4*>(src + i0 + TK_CHUNK));
    if (i0 + TK_PER_THREAD <= L) {
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
      // order keys two per word; -0.0 is rare, so one test covers the 8 values
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
#pragma unroll
      for (int q = 0; q < TK_PER_THREAD; ++q) {
        if (i0 + q < L) {
          kv[q] = bf16_key(src[i0 + q]);
          keys[i0 + q] = (uint16_t)kv[q];
          kmin = min(kmin, kv[q]);
          kmax = max(kmax, kv[q]);
        }
      }
    }
  }

  kmin = min(kmin, min(kmin2 & 0xFFFFu, kmin2 >> 16));
  kmax = max(kmax, max(kmax2 & 0xFFFFu, kmax2 >> 16));
  // the row's smallest and largest key (for the threshold bins and the counting sort)
  const int lane = tid & 31, warp = tid >> 5;
  if (need_select) {
#pragma unroll
    for (int j = 0; j < TK_HPER; ++j) hist[tid * TK_HPER + j] = 0u;
  }
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  if (lane == 0) {
    red[warp] = kmin;
    red[TK_WARPS + warp] = kmax;
  }
  __syncthreads();  // also publishes the staged keys and the cleared bins
#pragma unroll
  for (int w = 0; w < TK_WARPS; ++w) {
    kmin = min(kmin, red[w]);
    kmax = max(kmax, red[TK_WARPS + w]);
  }

  uint32_t thr = 0, need_eq = 0;
  if (need_select) {  // block-uniform
    // bins of width 2^sh cover [kmin, kmax] in at most TK_HBINS bins
    const uint32_t range = kmax - kmin;
    const int bits = range ? 32 - __clz(range) : 0;
    const int sh = bits > TK_HBITS ? bits - TK_HBITS : 0;
    const uint32_t kmin2w = kmin | (kmin << 16);
    for (int base = 0; base < L; base += TK_CHUNK) {
      const int i0 = base + tid * TK_PER_THREAD;
      if (i0 + TK_PER_THREAD <= L) {
        const uint4 v = *reinterpret_cast<const uint4*>(keys + i0);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t d = w[q] - kmin2w;  // both halves at once: no half is below kmin
          atomicAdd(hist + ((d & 0xFFFFu) >> sh), 1u);
          atomicAdd(hist + (d >> (16 + sh)), 1u);
        }
      } else {
        for (int q = 0; q < TK_PER_THREAD; ++q)
          if (i0 + q < L) atomicAdd(hist + (((uint32_t)keys[i0 + q] - kmin) >> sh), 1u);
      }
    }
    __syncthreads();
    find_bin_desc(hist, (int)(range >> sh) + 1, (uint32_t)K, warp_tot, misc);
    const uint32_t b1 = misc[0], above1 = misc[1];
    uint32_t b2 = 0, above2 = 0;
    if (sh > 0) {
      // the low sh bits of the keys in bin b1 only
      const uint32_t lmask = (1u << sh) - 1u;
      if (tid < (1 << sh)) hist[tid] = 0u;
      __syncthreads();
      for (int base = 0; base < L; base += TK_CHUNK) {
        const int i0 = base + tid * TK_PER_THREAD;
        if (i0 + TK_PER_THREAD <= L) {
          const uint4 v = *reinterpret_cast<const uint4*>(keys + i0);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t d0 = (w[q] & 0xFFFFu) - kmin, d1 = (w[q] >> 16) - kmin;
            if ((d0 >> sh) == b1) atomicAdd(hist + (d0 & lmask), 1u);
            if ((d1 >> sh) == b1) atomicAdd(hist + (d1 & lmask), 1u);
          }
        } else {
          for (int q = 0; q < TK_PER_THREAD; ++q) {
            if (i0 + q < L) {
              const uint32_t d = (uint32_t)keys[i0 + q] - kmin;
              if ((d >> sh) == b1) atomicAdd(hist + (d & lmask), 1u);
            }
          }
        }
      }
      __syncthreads();
      find_bin_desc(hist, 1 << sh, (uint32_t)K - above1, warp_tot, misc + 2);
      b2 = misc[2];
      above2 = misc[3];
    }
    thr = kmin + (b1 << sh) + b2;
    need_eq = (uint32_t)K - above1 - above2;
  }

  // ---- compaction in index order: one scan of (equal << 16 | above) counts per chunk
  const int nsel = need_select ? K : L;
  uint32_t gt_base = 0, eq_base = 0;
  for (int base = 0; base < L; base += TK_CHUNK) {
    const int i0 = base + tid * TK_PER_THREAD;
    uint32_t kq[TK_PER_THREAD];
    if (i0 + TK_PER_THREAD <= L) {
      const uint4 v = *reinterpret_cast<const uint4*>(keys + i0);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        kq[2 * q] = w[q] & 0xFFFFu;
        kq[2 * q + 1] = w[q] >> 16;
      }
    } else {
#pragma unroll
      for (int q = 0; q < TK_PER_THREAD; ++q) kq[q] = (i0 + q < L) ? keys[i0 + q] : 0u;
    }
    uint32_t n_gt = 0, n_eq = 0;
#pragma unroll
    for (int q = 0; q < TK_PER_THREAD; ++q) {
      const bool in = i0 + q < L;
      n_gt += (in && (!need_select || kq[q] > thr)) ? 1u : 0u;
      n_eq += (in && need_select && kq[q] == thr) ? 1u : 0u;
    }
    uint32_t tot;
    const uint32_t pre = block_excl_scan((n_eq << 16) | n_gt, warp_tot, tot);
    uint32_t g = gt_base + (pre & 0xFFFFu), e = eq_base + (pre >> 16);
#pragma unroll
    for (int q = 0; q < TK_PER_THREAD; ++q) {
      if (i0 + q < L) {
        int pos = -1;
        if (!need_select || kq[q] > thr) {
          pos = (int)(g + (e < need_eq ? e : need_eq));
          ++g;
        } else if (kq[q] == thr) {
          if (e < need_eq) pos = (int)(g + e);
          ++e;
        }
        if (pos >= 0 && pos < NS) sortbuf[pos] = ((0xFFFFu - kq[q]) << 16) | (uint32_t)(i0 + q);
      }
    }
    gt_base += tot & 0xFFFFu;
    eq_base += tot >> 16;
  }
  for (int i = nsel + tid; i < NS; i += TK_THREADS) sortbuf[i] = 0xFFFFFFFFu;
  __syncthreads();

  // output slot i: the selected element `comp` (valid) or -1
  auto write_out = [&](int i, bool valid, uint32_t comp) {
    int64_t o = -1;
    if (valid) {
      const int64_t idx = (int64_t)(comp & 0xFFFFu);
      o = (p.causal && idx >= lim64) ? -1 : idx + p.offset;
    }
    if (p.out_i64)
      reinterpret_cast<int64_t*>(p.out)[row * p.out_row_stride + i] = o;
    else
      reinterpret_cast<int32_t*>(p.out)[row * p.out_row_stride + i] = (int32_t)o;
  };

  // ---- stable counting sort when the selected keys span at most TK_CBINS values
  // (indexer score rows: a few dozen).  sortbuf holds the selection in index order;
  // warp w ranks its contiguous segment.  Equal keys of one 32-element step are
  // found with match_any and ranked by lane, so every element's output position is
  // (elements of larger keys) + (equal keys in earlier warps, steps and lanes): value
  // descending, index ascending, as the bitonic sort below gives.  The per-warp
  // counters live in the staged-key area, which the compaction has finished with.
  {
    const uint32_t lo = need_select ? thr : kmin;
    // CB key values (bins): 128 covers the selections of long score rows (a few
    // dozen values); up to TK_CBINS covers rows shorter than k, whose selection
    // is the whole row (a few hundred values).  The per-warp counters live in the
    // staged-key area, which the host sizes for TK_WARPS x TK_CBINS of them.
    auto count_sort = [&](auto cb_tag) {
      constexpr int CB = decltype(cb_tag)::value;
      constexpr int BPT = CB > TK_THREADS ? CB / TK_THREADS : 1;  // key values per thread
      uint16_t* cnt = keys;  // [TK_WARPS][CB]
      for (int i = tid; i < TK_WARPS * CB; i += TK_THREADS) cnt[i] = 0;
      __syncthreads();
      const int seg = (nsel + TK_THREADS - 1) / TK_THREADS * 32;
      const int s0 = warp * seg, s1 = min(nsel, s0 + seg);
      uint16_t* wc = cnt + warp * CB;
      for (int b = s0; b < s1; b += 32) {
        const int i = b + lane;
        const uint32_t d = i < s1 ? kmax - (0xFFFFu - (sortbuf[i] >> 16)) : 0xFFFFFFFFu;
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
        if (i < s1 && lane == __ffs(peers) - 1) wc[d] += (uint16_t)__popc(peers);
        __syncwarp();
      }
      __syncthreads();
      // exclusive prefix over warps per key, then over keys (descending key =
      // ascending d); thread t owns the key values t BPT .. t BPT + BPT - 1
      uint32_t tot_b[BPT], tsum = 0;
#pragma unroll
      for (int j = 0; j < BPT; ++j) {
        const int d = tid * BPT + j;
        tot_b[j] = 0;
        if (d < CB) {
          for (int w = 0; w < TK_WARPS; ++w) {
            const uint32_t c = cnt[w * CB + d];
            cnt[w * CB + d] = (uint16_t)tot_b[j];
            tot_b[j] += c;
          }
        }
        tsum += tot_b[j];
      }
      uint32_t total;
      uint32_t kbase = block_excl_scan(tsum, warp_tot, total);
#pragma unroll
      for (int j = 0; j < BPT; ++j) {
        const int d = tid * BPT + j;
        if (d < CB)
          for (int w = 0; w < TK_WARPS; ++w) cnt[w * CB + d] += (uint16_t)kbase;
        kbase += tot_b[j];
      }
      __syncthreads();
      const uint32_t lt = (1u << lane) - 1u;
      for (int b = s0; b < s1; b += 32) {
        const int i = b + lane;
        const uint32_t comp = i < s1 ? sortbuf[i] : 0u;
        const uint32_t d = i < s1 ? kmax - (0xFFFFu - (comp >> 16)) : 0xFFFFFFFFu;
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
        if (i < s1) write_out((int)wc[d] + __popc(peers & lt), true, comp);
        __syncwarp();
        if (i < s1 && lane == __ffs(peers) - 1) wc[d] += (uint16_t)__popc(peers);
        __syncwarp();
      }
      for (int i = nsel + tid; i < K; i += TK_THREADS) write_out(i, false, 0u);
    };
    if (nsel > 0 && kmax - lo < 128u) {  // block-uniform
      count_sort(std::integral_constant<int, 128>{});
      return;
    }
    if (nsel > 0 && kmax - lo < (uint32_t)TK_CBINS) {
      count_sort(std::integral_constant<int, TK_CBINS>{});
      return;
    }
  }

  // ---- bitonic sort of NS composites, ascending; thread t owns elements t*EPT ..
  uint32_t v[EPT];
#pragma unroll
  for (int q = 0; q < EPT; ++q) v[q] = sortbuf[tid * EPT + q];
#pragma unroll
  for (int kk = 2; kk <= NS; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      if (j < EPT) {
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const int q2 = q ^ j;
          if (q2 > q) {
            const bool asc = ((tid * EPT + q) & kk) == 0;
            const uint32_t lo = min(v[q], v[q2]), hi = max(v[q], v[q2]);
            v[q] = asc ? lo : hi;
            v[q2] = asc ? hi : lo;
          }
        }
      } else if (j < 32 * EPT) {
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const uint32_t w = __shfl_xor_sync(0xFFFFFFFFu, v[q], j / EPT);
          const int e = tid * EPT + q;
          const bool take_min = ((e & j) == 0) == ((e & kk) == 0);
          v[q] = take_min ? min(v[q], w) : max(v[q], w);
        }
      } else {
#pragma unroll
        for (int q = 0; q < EPT; ++q) sortbuf[tid * EPT + q] = v[q];
        __syncthreads();
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const int e = tid * EPT + q;
          const uint32_t w = sortbuf[e ^ j];
          const bool take_min = ((e & j) == 0) == ((e & kk) == 0);
          v[q] = take_min ? min(v[q], w) : max(v[q], w);
        }
        __syncthreads();
      }
    }
  }

  // ---- post-process and write
#pragma unroll
  for (int q = 0; q < EPT; ++q) {
    const int i = tid * EPT + q;
    if (i < K) write_out(i, i < nsel, v[q]);
  }
}

}  // namespace ks
