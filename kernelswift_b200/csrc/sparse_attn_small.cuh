// Top-k sparse attention for few heads (H <= 64) and short index rows (K <= 512):
// one CTA per query token, keys as the MMA's M dimension.
//
// Semantics are those of sparse_attn_kernel (baseline/sparse_attention.py:5-42).
// With H = 16 (C2) or the reference's own default (H = 64, K = 16) the head
// count fills only a fraction of an M = 128 tile, so the product is transposed:
//   S^T[keys, heads] = K_g[keys, D] . Q^T          M = 128 keys, N = Hn (H rounded up)
//   O^T[dims, heads] = V^T[dims, keys] . P^T        M = 128 output dims, N = Hn
// The gathered rows are the A operand of both products: K-major (rows = keys) for
// QK and, read as MN-major (dims contiguous), V^T for PV, so nothing is gathered
// twice.  All K keys stay resident (K_pad x D_alloc x 2 bytes of shared memory),
// so the softmax sees every score at once: one exact max and sum per head, no
// rescaling.  P is rounded to bf16 for the PV product and the normalisation is
// applied in fp32 at the end, as in sparse_attn_kernel.
//
// One CTA of 128 G threads (G = 2 warp groups for index rows of at most 256 keys,
// 4 for longer ones): all warps gather (cp.async, 16 bytes per copy, zeros for
// masked keys); warp 4 issues the MMAs (one elected lane); every warp group runs
// the softmax over its own 128-key tiles of S^T (warp w reads TMEM lane quarter
// w % 4), so the tiles of one token are worked on side by side, and the groups
// share the epilogue's column blocks of O^T.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int SAS_MAX_G = 4;     // warp groups of the widest CTA
constexpr int SAS_MAX_K = 512;
constexpr int SAS_HDR = 7168;

struct SaSmallParams {
  const uint16_t* q;    // bf16 [B, M, H, D]
  const int32_t* idx;   // [B, M, K]
  const uint16_t* kv;   // bf16 [B, N, D]
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t B, M, H, D, N, K, dv_begin, dv;
  int32_t nt;           // 128-key tiles (K_pad / 128)
  int32_t nkb;          // 64-dim chunks held per key row (covers D and the PV columns)
  int32_t dv_tiles;     // 128-row M tiles of O^T
  uint32_t kg_off, q_off, p_off;  // shared-memory regions (bytes from the aligned base)
  uint32_t tmem_cols;
  float scale_log2;
  int* status;
  uint64_t budget_ns;
};

struct SaSmallShared {
  uint64_t mma_bar;
  uint32_t tmem_base;
  int abort;
  int oob;
  float red[4 * SAS_MAX_G][64];  // per-warp partial max / sum per head
  float head_m[64];     // max per head (base-2 scaled), sink included
  float head_inv[64];   // 1 / denominator per head
  int32_t idx[SAS_MAX_K];  // the token's index row, -1 past K
};
static_assert(sizeof(SaSmallShared) <= SAS_HDR, "SaSmallShared exceeds its header");

// Max (MX) or sum of v[i] over the warp's 32 lanes for 16 values i at once, by
// halving exchanges: at offset 16 a lane sends the half of its values that its
// partner keeps (8 shuffles), then 4, 2 and 1 at offsets 8, 4, 2, and a last
// shuffle at offset 1 -- 16 shuffles instead of 16 x 5.  Lane L ends with the
// result for i = (L >> 1) & 15.  Every value goes through the same pairwise tree
// as a butterfly per value (v[L] op v[L ^ 16], then with L ^ 8, ...), so results
// are bit-identical to it.
template <bool MX>
__device__ __forceinline__ float reduce16_lanes(const float (&v)[16], int lane) {
  auto op = [](float a, float b) { return MX ? fmaxf(a, b) : a + b; };
  float w[8], x[4], y[2];
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float keep = b4 ? v[j + 8] : v[j];
    w[j] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, b4 ? v[j] : v[j + 8], 16));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float keep = b3 ? w[j + 4] : w[j];
    x[j] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, b3 ? w[j] : w[j + 4], 8));
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float keep = b2 ? x[j + 2] : x[j];
    y[j] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, b2 ? x[j] : x[j + 2], 4));
  }
  const float z = op(b1 ? y[1] : y[0], __shfl_xor_sync(0xFFFFFFFFu, b1 ? y[0] : y[1], 2));
  return op(z, __shfl_xor_sync(0xFFFFFFFFu, z, 1));
}

template <int HN, int G>
__global__ void __launch_bounds__(128 * G)
    sparse_attn_small_kernel(SaSmallParams p) {
  constexpr int THREADS = 128 * G;
  extern __shared__ uint8_t sas_raw[];
  const uint32_t raw = smem_u32(sas_raw);
  uint8_t* smem = sas_raw + (((raw + 1023u) & ~1023u) - raw);
  SaSmallShared* sh = reinterpret_cast<SaSmallShared*>(smem);
  uint8_t* kg = smem + p.kg_off;  // [nt][nkb][128 keys x 128 B], 128-byte swizzle
  uint8_t* qs = smem + p.q_off;   // [nkb][HN rows x 128 B]
  uint8_t* ps = smem + p.p_off;   // P^T [K_pad / 64][HN rows x 128 B] (K-major: keys contiguous)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t token = blockIdx.x;
  const int b = (int)(token / p.M);
  const int K_pad = p.nt * 128;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    mbar_init(&sh->mma_bar, 1);
    sh->abort = 0;
    sh->oob = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc<1>(&sh->tmem_base, p.tmem_cols);
    tmem_relinquish<1>();
  }

  // ---------------------------------------------------------------- gathers
  // Key rows: piece c (16 bytes) of key k lands in tile k / 128, chunk c / 8, row
  // k % 128, 16-byte unit (c % 8) ^ (k % 8).  Masked keys (negative, >= N, or past
  // K) are zero-filled; the D columns past D (when nkb covers more) too.
  const int32_t* ip = p.idx + token * p.K;
  const uint16_t* kvb = p.kv + (int64_t)b * p.N * p.D;
  // the index row first (one coalesced pass), so no row copy waits on an index load
  for (int k = threadIdx.x; k < K_pad; k += THREADS) sh->idx[k] = k < p.K ? __ldg(ip + k) : -1;
  __syncthreads();
  {
    const int pieces_per_row = p.nkb * 8;
    const int total = K_pad * pieces_per_row;
    // (key, piece) of element e, advanced by THREADS elements per step without a division
    const int dk = THREADS / pieces_per_row, dc = THREADS - dk * pieces_per_row;
    int k = threadIdx.x / pieces_per_row, c = threadIdx.x - k * pieces_per_row;
    for (int e = threadIdx.x; e < total; e += THREADS, k += dk, c += dc) {
      if (c >= pieces_per_row) {
        c -= pieces_per_row;
        ++k;
      }
      const int32_t v = sh->idx[k];
      const bool ok = v >= 0 && v < p.N && c * 8 < p.D;
      if (k < p.K && v >= p.N) sh->oob = 1;
      uint8_t* dst = kg + ((k >> 7) * p.nkb + (c >> 3)) * 16384 + (k & 127) * 128 +
                     (((c & 7) ^ (k & 7)) << 4);
      cp_async16(dst, ok ? kvb + (int64_t)v * p.D + c * 8 : kvb, ok ? 16u : 0u);
    }
    // the query rows (heads) h < H of this token, zeros for the padding rows
    const uint16_t* qt = p.q + token * (int64_t)p.H * p.D;
    const int qpieces = HN * p.nkb * 8;
    for (int e = threadIdx.x; e < qpieces; e += THREADS) {
      const int h = e / (p.nkb * 8), c = e % (p.nkb * 8);
      const bool ok = h < p.H && c * 8 < p.D;
      uint8_t* dst = qs + (c >> 3) * (HN * 128) + h * 128 + (((c & 7) ^ (h & 7)) << 4);
      cp_async16(dst, ok ? qt + (int64_t)h * p.D + c * 8 : qt, ok ? 16u : 0u);
    }
    cp_async_wait_all();
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  const uint32_t s_col = 0, o_col = (uint32_t)(p.nt * HN);

  // ---------------------------------------------------------------- QK^T
  if (warp == 4) {
    const bool leader = elect_one();
    if (leader) {
      const uint32_t idesc = idesc_bf16_f32(128, HN, false, false);
      const int ksteps = (p.D + 15) / 16;
      for (int t = 0; t < p.nt; ++t)
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint32_t a = smem_u32(kg + (t * p.nkb + (ks >> 2)) * 16384) + (ks & 3) * 32;
          const uint32_t bq = smem_u32(qs + (ks >> 2) * (HN * 128)) + (ks & 3) * 32;
          umma_bf16_ss(tmem + s_col + t * HN, sdesc_sw128(a, 16, 1024), sdesc_sw128(bq, 16, 1024),
                       idesc, ks > 0 ? 1u : 0u);
        }
      umma_commit(&sh->mma_bar);
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- softmax (all warps)
  // Thread = key: warp w of group g = w / 4 takes keys 32 (w % 4) + lane of tiles
  // g, g + G, ...  Heads go in groups of 16 TMEM columns; each pass re-reads S^T
  // from TMEM, so registers do not grow with H or K.  Max and sum per head are
  // reduced over the warp by a shuffle butterfly and over the warps through shared
  // memory (warps without a tile contribute -inf / 0).
  const int quarter = warp & 3, grp = warp >> 2;
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->mma_bar, 0, wc));
  uint32_t vmask = 0;  // bit t: this thread's key of tile t is valid
  for (int t = grp; t < p.nt; t += G) {
    const int32_t v = sh->idx[t * 128 + quarter * 32 + lane];
    vmask |= (uint32_t)(v >= 0 && v < p.N) << t;
  }
  if (ok) {
    tc_fence_after();
#pragma unroll 1
    for (int hg = 0; hg < HN; hg += 16) {
      float mh[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) mh[i] = -INFINITY;
      for (int t = grp; t < p.nt; t += G) {
        uint32_t r[16];
        tmem_ld16(tmem + s_col + t * HN + hg + lane_off, r);
        tmem_wait_ld();
        if ((vmask >> t) & 1u) {
#pragma unroll
          for (int i = 0; i < 16; ++i) mh[i] = fmaxf(mh[i], __uint_as_float(r[i]) * p.scale_log2);
        }
      }
      const float rm = reduce16_lanes<true>(mh, lane);  // head hg + (lane >> 1)
      if ((lane & 1) == 0) sh->red[warp][hg + (lane >> 1)] = rm;
    }
  }
  __syncthreads();
  const float sink2 = threadIdx.x < p.H ? __ldg(p.sink + threadIdx.x) * 1.4426950408889634f : 0.f;
  if (ok && threadIdx.x < HN) {
    const int h = threadIdx.x;
    float m = sink2;
#pragma unroll
    for (int w = 0; w < 4 * G; ++w) m = fmaxf(m, sh->red[w][h]);
    sh->head_m[h] = m;
  }
  __syncthreads();
  if (ok) {
#pragma unroll 1
    for (int hg = 0; hg < HN; hg += 16) {
      float ls[16], hm[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        ls[i] = 0.f;
        hm[i] = sh->head_m[hg + i];
      }
      for (int t = grp; t < p.nt; t += G) {
        const int k = t * 128 + quarter * 32 + lane;  // key of this thread in tile t
        const bool valid = (vmask >> t) & 1u;
        uint32_t r[16];
        tmem_ld16(tmem + s_col + t * HN + hg + lane_off, r);
        tmem_wait_ld();
        const int kk = k & 63;
        uint8_t* chunk = ps + (k >> 6) * (HN * 128);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int h = hg + i;
          const float e = valid ? ex2f(fmaf(__uint_as_float(r[i]), p.scale_log2, -hm[i])) : 0.f;
          ls[i] += e;
          // P^T (K-major: row h holds the keys, 64 per 128-byte row): pairs of
          // keys (even lane, odd lane) go out as one 32-bit store by the even lane
          const float e_hi = __shfl_down_sync(0xFFFFFFFFu, e, 1);
          if ((lane & 1) == 0)
            *reinterpret_cast<uint32_t*>(chunk + h * 128 + (((kk >> 3) ^ (h & 7)) << 4) + (kk & 7) * 2) =
                cvt_bf16x2(e, e_hi);
        }
      }
      const float rs = reduce16_lanes<false>(ls, lane);
      if ((lane & 1) == 0) sh->red[warp][hg + (lane >> 1)] = rs;
    }
    fence_proxy_async_smem();  // P^T is read by the tensor cores next
  }
  __syncthreads();
  if (ok && threadIdx.x < HN) {
    const int h = threadIdx.x;
    float den = ex2f(sink2 - sh->head_m[h]);
#pragma unroll
    for (int w = 0; w < 4 * G; ++w) den += sh->red[w][h];
    sh->head_inv[h] = 1.f / den;
  }
  tc_fence_before();
  __syncthreads();

  // ---------------------------------------------------------------- P V
  if (warp == 4) {
    const bool leader = elect_one();
    if (leader) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, HN, true, false);
      const int ksteps = K_pad / 16;
      const int c0 = p.dv_begin / 64;
      for (int m = 0; m < p.dv_tiles; ++m)
        for (int ks = 0; ks < ksteps; ++ks) {
          // A = V^T: dims [dv_begin + 128 m, +128) of keys [16 ks, +16), MN-major;
          // its two 64-dim halves are chunks 16 KB apart (LBO)
          const int t = ks >> 3;
          const uint32_t a = smem_u32(kg + (t * p.nkb + c0 + 2 * m) * 16384) + (ks & 7) * 2048;
          const uint32_t bp = smem_u32(ps + (ks >> 2) * (HN * 128)) + (ks & 3) * 32;
          umma_bf16_ss(tmem + o_col + m * HN, sdesc_sw128(a, 16384, 1024), sdesc_sw128(bp, 16, 1024),
                       idesc, ks > 0 ? 1u : 0u);
        }
      umma_commit(&sh->mma_bar);
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- epilogue (all warps)
  // Thread = output dim (TMEM lane) of each 128-dim tile; out[token, h, dim] for h < H.
  // Block j = (tile m, 16 heads) goes to warp group j % G.
  if (__all_sync(0xFFFFFFFFu, mbar_wait(&sh->mma_bar, 1, wc))) {
    tc_fence_after();
    uint16_t* orow = p.out + token * (int64_t)p.H * p.dv;
    const int nblk = p.dv_tiles * (HN / 16);
    for (int j = grp; j < nblk; j += G) {
      const int m = j / (HN / 16), c = (j % (HN / 16)) * 16;
      const int d = m * 128 + quarter * 32 + lane;
      uint32_t r[16];
      tmem_ld16(tmem + o_col + m * HN + c + lane_off, r);
      tmem_wait_ld();
      if (d < p.dv) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c + i < p.H)
            orow[(int64_t)(c + i) * p.dv + d] =
                __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[i]) * sh->head_inv[c + i]));
      }
    }
  }
  if (threadIdx.x == 0 && sh->oob) report_bounds(p.status, (int)token, p.N);

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc<1>(tmem, p.tmem_cols);
}

}  // namespace ks
