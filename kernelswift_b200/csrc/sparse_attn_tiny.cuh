// Top-k sparse attention for very short index rows (K <= 64) over many tokens:
// heads as the MMA's M dimension, several tokens packed into one 128-row tile.
//
// Semantics are those of sparse_attn_kernel (baseline/sparse_attention.py:5-42).
// At the reference's own default geometry (H = 64, D = 128, K = 16 over 20 800
// tokens) the work per token is tiny and the call is bound by reading q and
// writing the output (~0.68 GB); one CTA per token with keys as M (the few-heads
// kernel) spent ~24 K warp instructions per token on cross-lane reductions over
// 128 padded key lanes.  Here a tile is 128 query rows = TPT = 128 / H tokens x H
// heads (rows of q are consecutive), and the keys of those tokens sit side by
// side along N (KP slots per token, N_ = TPT x KP):
//   S[rows, N_] = Q[rows, D] . Kg^T                 M = 128, N = N_, K = D
//   O[rows, dv] = P[rows, N_] . Vg[N_, dv]          M = 128, N = dv, K = N_
// Row r (token r / H) keeps only its own token's KP columns: the softmax writes
// P = 0 elsewhere, so the one PV product gives every token its own output.  The
// reductions are then per thread (thread = TMEM lane = row).  The gathered rows
// are the K-major B operand of QK and, read MN-major (dims contiguous), the B
// operand of PV: nothing is gathered twice.  P is rounded to bf16 for PV and the
// normalisation applied in fp32 at the end, as in sparse_attn_kernel.
//
// One CTA of 128 threads per tile: all gather the key rows (cp.async, 16 bytes per
// copy, zeros for masked keys); the query tile comes by TMA (128-byte swizzle, rows
// past the last token read as zeros) and the output tile leaves by TMA (staged over
// P, rows past the last token clipped); one elected lane of warp 0 issues the MMAs;
// thread t runs the softmax and the epilogue of row t.  P overwrites the query tile
// (free once QK has completed) and O the score columns in TMEM (free once the
// softmax has read them).
#pragma once
#include "sparse_attn.cuh"

namespace ks {

constexpr int SAT_THREADS = 128;
constexpr int SAT_MAX_K = 64;    // longest index row this path takes
constexpr int SAT_MAX_N = 256;   // key columns per tile (TPT x KP)
constexpr int SAT_HDR = 2048;

struct SaTinyParams {
  const uint16_t* q;    // bf16 [B, M, H, D] = rows [B*M*H, D]
  const int32_t* idx;   // [B, M, K]
  const uint16_t* kv;   // bf16 [B, N, D]
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t B, M, H, D, N, K, dv_begin, dv;
  int32_t tpt, kp, ncol;  // tokens per tile, key slots per token, ncol = tpt * kp
  float inv_kp;           // 1 / kp
  int32_t nkb;            // 64-dim chunks of D
  uint32_t kg_off, q_off; // shared-memory regions (bytes from the aligned base)
  uint32_t tmem_cols;
  float scale_log2;
  int* status;
  uint64_t budget_ns;
};

struct SaTinyShared {
  uint64_t mma_bar;
  uint64_t q_bar;       // the query tile's TMA loads
  uint32_t tmem_base;
  int abort;
  int32_t idx[SAT_MAX_N];  // column c -> row of kv as [B N, D] (batch folded in; -1: masked slot)
  uint32_t vmask[SAT_MAX_N / 32];  // bit c % 32 of word c / 32: column c holds a valid row
};
static_assert(sizeof(SaTinyShared) <= SAT_HDR, "SaTinyShared exceeds its header");

__global__ void __launch_bounds__(SAT_THREADS)
    sparse_attn_tiny_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap omap, SaTinyParams p) {
  extern __shared__ uint8_t sat_raw[];
  const uint32_t raw = smem_u32(sat_raw);
  uint8_t* smem = sat_raw + (((raw + 1023u) & ~1023u) - raw);
  SaTinyShared* sh = reinterpret_cast<SaTinyShared*>(smem);
  uint8_t* kg = smem + p.kg_off;  // [nkb][ncol rows x 128 B], 128-byte swizzle
  uint8_t* qs = smem + p.q_off;   // [nkb][128 rows x 128 B]; later P [ncol / 64][128 rows x 128 B]
  const int warp = threadIdx.x >> 5;
  const int64_t n_tok = (int64_t)p.B * p.M;
  const int64_t tok0 = (int64_t)blockIdx.x * p.tpt;  // first token of the tile
  const int64_t row0 = tok0 * p.H;                   // first q / out row of the tile
  const uint32_t chunk = (uint32_t)p.ncol * 128u;    // bytes of one 64-dim chunk of kg
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  // the query tile first: it depends on nothing, and one thread issues it
  if (threadIdx.x == 0) {
    mbar_init(&sh->q_bar, 1);
    fence_barrier_init();
    mbar_expect_tx(&sh->q_bar, (uint32_t)p.nkb * 16384u);
    for (int kb = 0; kb < p.nkb; ++kb) tma_load_2d(&qmap, &sh->q_bar, qs + kb * 16384, kb * 64, (int32_t)row0);
  }
  // the index rows of the tile's tokens (-1 for slots past K and tokens past the
  // end), loaded before the set-up so their latency overlaps it; every copy then
  // reads its row from shared memory (ncol <= 2 x 128)
  // Column c is slot i of token j = c / kp: (c + 1/2) / kp in fp32 floors to j
  // exactly (c < 256, kp <= 64: the rounding error is far below 1 / (2 kp)).  The
  // token's batch comes from the tile's first token (one division) and carries.
  int32_t ix[2], bt[2];
  const int t0 = (int)tok0;  // tokens < B M < 2^30
  const int b0 = t0 / p.M, m0 = t0 - b0 * p.M;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int c = threadIdx.x + u * SAT_THREADS;
    const int j = (int)(((float)c + 0.5f) * p.inv_kp), i = c - j * p.kp;
    const int64_t tok = tok0 + j;
    const bool live = c < p.ncol && i < p.K && tok < n_tok;
    ix[u] = live ? __ldg(p.idx + tok * p.K + i) : -1;
    int bb = b0, mm = m0 + j;
    if (live)
      while (mm >= p.M) {  // at most tpt - 1 steps
        mm -= p.M;
        ++bb;
      }
    bt[u] = bb;
  }
  if (threadIdx.x == 0) {
    mbar_init(&sh->mma_bar, 1);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc<1>(&sh->tmem_base, p.tmem_cols);
    tmem_relinquish<1>();
  }
  // each column's row of kv seen as [B N, D] (its token's batch folded in, so no
  // copy below divides), the columns' validity bits, and whether any index is >= N
  bool oob = false;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int c = threadIdx.x + u * SAT_THREADS;
    const bool valid = ix[u] >= 0 && ix[u] < p.N;
    const uint32_t vb = __ballot_sync(0xFFFFFFFFu, valid);
    oob |= ix[u] >= p.N;
    if (c < p.ncol) {
      sh->idx[c] = valid ? bt[u] * p.N + ix[u] : -1;  // B N < 2^31
      if ((threadIdx.x & 31) == 0) sh->vmask[c >> 5] = vb;
    }
  }
  oob = __syncthreads_or(oob);

  // ---------------------------------------------------------------- gathers
  {
    // key rows: piece c (16 bytes) of column r lands in chunk c / 8, row r,
    // 16-byte unit (c % 8) ^ (r % 8); masked slots are zero-filled
    // (column r, piece c) of element e, advanced by the block size per step without
    // a division
    const int pieces = p.nkb * 8;
    const int dr = SAT_THREADS / pieces, dc = SAT_THREADS - dr * pieces;
    int r = threadIdx.x / pieces, c = threadIdx.x - r * pieces;
    for (int e = threadIdx.x; e < p.ncol * pieces; e += SAT_THREADS, r += dr, c += dc) {
      if (c >= pieces) {
        c -= pieces;
        ++r;
      }
      const int32_t v = sh->idx[r];
      const bool ok = v >= 0;
      const uint16_t* src = p.kv + (int64_t)(ok ? v : 0) * p.D + c * 8;
      uint8_t* dst = kg + (c >> 3) * chunk + r * 128 + (((c & 7) ^ (r & 7)) << 4);
      cp_async16(dst, ok ? src : p.kv, ok ? 16u : 0u);
    }
    cp_async_wait_all();
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  // ---------------------------------------------------------------- S = Q Kg^T
  if (warp == 0 && __all_sync(0xFFFFFFFFu, mbar_wait(&sh->q_bar, 0, wc))) {
    tc_fence_after();
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(128, p.ncol, false, false);
      for (int ks = 0; ks < p.D / 16; ++ks) {
        const uint32_t a = smem_u32(qs + (ks >> 2) * 16384) + (ks & 3) * 32;
        const uint32_t bk = smem_u32(kg + (ks >> 2) * chunk) + (ks & 3) * 32;
        umma_bf16_ss(tmem, sdesc_sw128(a, 16, 1024), sdesc_sw128(bk, 16, 1024), idesc, ks > 0 ? 1u : 0u);
      }
      umma_commit(&sh->mma_bar);
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- softmax of row r
  // (TMEM loads are warp-wide: every lane reads its warp's tokens' columns and keeps
  // those of its own token, c0 .. c0 + kp)
  const int r = threadIdx.x;
  const int j = r / p.H, h = r - j * p.H;
  const int c0 = j * p.kp;
  // the key columns of the warp's tokens (one token for H >= 32, two for H = 16):
  // the only ones its rows can keep, so the only ones it loads from TMEM
  const int cw0 = (warp * 32 / p.H) * p.kp;
  const int cw1 = min(p.ncol, ((warp * 32 + 31) / p.H + 1) * p.kp);
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const float sink2 = __ldg(p.sink + h) * 1.4426950408889634f;
  float m = sink2, lsum = 0.f;
  bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->mma_bar, 0, wc));
  if (ok) {
    tc_fence_after();
    for (int cc = cw0; cc < cw1; cc += 16) {
      uint32_t s[16];
      tmem_ld16(tmem + lane_off + cc, s);
      // valid columns of this 16-column group that belong to the row's token (kp
      // and c0 are multiples of 16: a group is wholly the row's token or not)
      const uint32_t gm = (cc >= c0 && cc < c0 + p.kp) ? (sh->vmask[cc >> 5] >> (cc & 31)) & 0xFFFFu : 0u;
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if ((gm >> i) & 1u) m = fmaxf(m, __uint_as_float(s[i]) * p.scale_log2);
    }
    // P row r (K-major, 64 columns per 128-byte row of a 16 KB chunk, swizzled),
    // written over the query tile, which the completed QK no longer reads
    for (int cc = 0; cc < p.ncol; cc += 16) {
      uint32_t pk[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};  // other tokens' columns: P = 0
      if (cc >= cw0 && cc < cw1) {
        uint32_t s[16];
        tmem_ld16(tmem + lane_off + cc, s);
        const uint32_t gm = (cc >= c0 && cc < c0 + p.kp) ? (sh->vmask[cc >> 5] >> (cc & 31)) & 0xFFFFu : 0u;
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float e[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            e[u] = ((gm >> (i + u)) & 1u) ? ex2f(fmaf(__uint_as_float(s[i + u]), p.scale_log2, -m)) : 0.f;
            lsum += e[u];
          }
          pk[i >> 1] = cvt_bf16x2(e[0], e[1]);
        }
      }
      uint8_t* prow = qs + (cc >> 6) * 16384 + r * 128;
      const int u0 = (cc & 63) >> 3;
      *reinterpret_cast<uint4*>(prow + ((u0 ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<uint4*>(prow + (((u0 + 1) ^ (r & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    fence_proxy_async_smem();  // P is read by the tensor cores next
  }
  tc_fence_before();
  __syncthreads();

  // ---------------------------------------------------------------- O = P Vg
  if (warp == 0 && ok) {
    if (elect_one()) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, p.dv, false, true);
      const uint32_t vb = smem_u32(kg + (p.dv_begin / 64) * chunk);
      for (int ks = 0; ks < p.ncol / 16; ++ks) {
        // A = P (K-major); B = the gathered rows read MN-major: dims [dv_begin, +dv)
        // of keys [16 ks, +16); their 64-dim chunks are `chunk` bytes apart (LBO)
        const uint32_t a = smem_u32(qs + (ks >> 2) * 16384) + (ks & 3) * 32;
        umma_bf16_ss(tmem, sdesc_sw128(a, 16, 1024), sdesc_sw128(vb + ks * 2048, chunk, 1024), idesc,
                     ks > 0 ? 1u : 0u);
      }
      umma_commit(&sh->mma_bar);
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- epilogue of row r
  // Row r's dv outputs go to shared memory (over P, which the completed PV no longer
  // reads) in 64-column chunks with the 128-byte swizzle; one thread then stores the
  // tile with TMA (rows past the last token are clipped by the tensor map).
  if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->mma_bar, 1, wc));
  if (ok) {
    tc_fence_after();
    const float inv = 1.f / (lsum + ex2f(sink2 - m));
    for (int cc = 0; cc < p.dv; cc += 16) {
      uint32_t o[16];
      tmem_ld16(tmem + lane_off + cc, o);
      tmem_wait_ld();
      uint32_t w[8];
#pragma unroll
      for (int t = 0; t < 8; ++t)
        w[t] = cvt_bf16x2(__uint_as_float(o[2 * t]) * inv, __uint_as_float(o[2 * t + 1]) * inv);
      uint8_t* orow = qs + (cc >> 6) * 16384 + r * 128;
      const int u0 = (cc & 63) >> 3;
      *reinterpret_cast<uint4*>(orow + ((u0 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4*>(orow + (((u0 + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
    fence_proxy_async_smem();  // read by the TMA store next
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sh->abort) {
    for (int kb = 0; kb < p.dv / 64; ++kb) tma_store_2d(&omap, qs + kb * 16384, kb * 64, (int32_t)row0);
    bulk_commit_group();
    bulk_wait_group_read<0>();  // the staging area may be released once read
  }
  if (threadIdx.x == 0 && oob) report_bounds(p.status, (int)tok0, p.N);
  // (no TMA write may be in flight when the CTA leaves, also after a timeout)
  if (threadIdx.x == 0) mbar_wait(&sh->q_bar, 0, wc, false, true);

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc<1>(tmem, p.tmem_cols);
}

}  // namespace ks
