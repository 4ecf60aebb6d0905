// Indexer scores on tcgen05: RoPE fused into the query-tile load, the q.k GEMM on
// the tensor cores with TMEM accumulators, and the bf16-exact epilogue.
//
// Semantics follow baseline/indexer.py:170-193 of KernelSwift (the NPU version is
// optimized/indexer_project/op_kernel/fused_indexer_qk_reduce.asc:368-428):
//   score[b,s,t] = bf16( sum_h bf16( relu(bf16(q[b,s,h,:] . k[b,t,:])) * w[b,s,h] ) )
// with the head sum in fp32 in head order, and t >= (s+1)//ratio masked to -inf
// for causal prefill rows.  RoPE rotates the last `rd` dims of q (interleaved
// pairs, fp32 products and sums rounded separately, result rounded to bf16),
// baseline/indexer.py:114-129,172.
//
// GEMM orientation: keys are the M dimension (128 per tile) and (token, head) is
// the N dimension (tok = 256/H tokens x H heads = 256).  The head reduction is
// therefore along TMEM columns, i.e. inside one thread: TMEM lane = key.
//
// Persistent CTAs, one per SM, 12 warps:
//   warp 0      TMA producer: query tiles (2 buffers) and key tiles (KST stages)
//   warp 1      TMEM owner and MMA issuer (one elected lane)
//   warps 2-3   RoPE on the query tile in shared memory (swizzled layout)
//   warps 4-11  epilogue: TMEM -> registers -> bf16 chain -> global scores
// Accumulators: 2 x 256 TMEM columns (double buffered), 512 columns in total.
// Work items (batch, token group) are handed out heaviest-first (causal cost
// grows with the position), strided over CTAs.
//
// FP8 variant (F8 = true; DeepSeek-style FP8 indexer keys and queries, the
// ModelArgs.dtype = "fp8" / scale_fmt = "ue8m0" option of baseline/indexer.py:14-17,
// which the bf16 baseline declares but does not use): q and k are e4m3 with one
// scale per (token, head) row of q and per key row of k; the GEMM runs as
// tcgen05 kind::f8f6f4 (K = 32 per instruction, 128-byte rows: D = 128 only, no
// RoPE in the kernel: q is rotated before it is quantised), and the epilogue is
//   score[b,s,t] = bf16( k_scale[b,t] * sum_h ( relu(q8[b,s,h,:] . k8[b,t,:]) * w[b,s,h] ) )
// in fp32 (each product and each partial sum rounded to nearest, heads in order),
// with w fp32 = head weight x the query row's scale.  The bf16 result feeds the
// same exact top-k as the bf16 path.
#pragma once
#include <type_traits>

#include "ks_device.cuh"

namespace ks {

constexpr int IX_THREADS = 384;
constexpr int IX_EPI_WARP0 = 4;
constexpr int IX_EPI_THREADS = 256;
constexpr int IX_ROPE_THREADS = 64;
constexpr int IX_TILE_KEYS = 128;
constexpr int IX_N = 256;
constexpr int IX_MAX_KST = 8;

struct IndexerScoreParams {
  const float* freqs;  // [S, rd/2, 2] (cos, sin) for the rows' positions
  const uint16_t* w;   // bf16 [B, S, H] (batch stride w_bs elements); bf16 path
  const float* wf;     // fp32 [B, S, H] (batch stride w_bs elements); FP8 path
  const float* k_scale;  // fp32 per key row, batch b key t at b * k_rows_per_batch + t; FP8 path
  int64_t w_bs;
  int32_t w_vec16;     // w and w_bs allow 16-byte loads
  uint16_t* scores;    // bf16 [B*S, score_ld]
  int64_t score_ld;
  int32_t B, S, H, D, T, rd;
  int64_t k_rows_per_batch;  // rows between batches in the key tensor map
  int64_t pos0;              // sequence position of row s = 0
  int32_t causal, ratio;
  int32_t tok, n_groups, n_items, kst;
  int* status;
  uint64_t budget_ns;
};

template <bool F8>
struct IxShared {
  uint64_t k_full[IX_MAX_KST], k_empty[IX_MAX_KST];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t q_tma[2], q_full[2], q_empty[2];
  uint64_t drain;
  uint64_t w_full, w_free;  // item weights staged / every epilogue warp done with them
  uint32_t tmem_base;
  int abort;
  // head weights of the current work item's tokens (token-major, IX_N = tok * H;
  // bf16, or fp32 on the FP8 path), staged once per item: read per tile from
  // shared memory rather than through the global-load path, whose traffic slowed
  // the MMAs
  alignas(16) typename std::conditional<F8, float, uint16_t>::type wbuf[IX_N];
};
// shared-memory header in front of the tiles (the bf16 path keeps 1 KB: one more
// would cost it a key stage)
template <bool F8>
__host__ __device__ constexpr uint32_t ix_hdr_bytes() { return F8 ? 2048u : 1024u; }
static_assert(sizeof(IxShared<false>) <= ix_hdr_bytes<false>(), "IxShared exceeds its header");
static_assert(sizeof(IxShared<true>) <= ix_hdr_bytes<true>(), "IxShared exceeds its header");

__device__ __forceinline__ int ix_item_tiles(const IndexerScoreParams& p, int item, int& b,
                                             int& g) {
  g = p.n_groups - 1 - item / p.B;
  b = item % p.B;
  int s_last = g * p.tok + p.tok - 1;
  if (s_last > p.S - 1) s_last = p.S - 1;
  int64_t kmax = p.T;
  if (p.causal) {
    const int64_t lim = (p.pos0 + s_last + 1) / p.ratio;
    kmax = lim < kmax ? lim : kmax;
  }
  if (kmax < 0) kmax = 0;
  return (int)((kmax + IX_TILE_KEYS - 1) / IX_TILE_KEYS);
}

template <int H, bool F8>
__global__ void __launch_bounds__(IX_THREADS, 1)
    indexer_score_kernel(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kmap, IndexerScoreParams p) {
  extern __shared__ uint8_t ix_raw[];
  const uint32_t raw_addr = smem_u32(ix_raw);
  uint8_t* smem = ix_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  // layout: [IxShared, padded to its header][2 query tiles][kst key stages], 1 KB aligned
  const int D = p.D;
  constexpr uint32_t ESZ = F8 ? 1 : 2;                        // bytes per element
  const uint32_t q_bytes = (uint32_t)IX_N * D * ESZ;          // one query tile
  const uint32_t k_bytes = (uint32_t)IX_TILE_KEYS * D * ESZ;  // one key stage
  const int nkb = D * (int)ESZ / 128;                         // 128-byte K blocks per row
  IxShared<F8>* sh = reinterpret_cast<IxShared<F8>*>(smem);
  uint8_t* qbuf = smem + ix_hdr_bytes<F8>();
  uint8_t* kbuf = qbuf + 2 * q_bytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.kst; ++i) {
      mbar_init(&sh->k_full[i], 1);
      mbar_init(&sh->k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->acc_full[i], 1);
      mbar_init(&sh->acc_empty[i], IX_EPI_THREADS / 32);
      mbar_init(&sh->q_tma[i], 1);
      mbar_init(&sh->q_full[i], IX_ROPE_THREADS);
      mbar_init(&sh->q_empty[i], 1);
    }
    mbar_init(&sh->drain, 1);
    mbar_init(&sh->w_full, 1);
    mbar_init(&sh->w_free, IX_EPI_THREADS / 32);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(&sh->tmem_base, 512);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      uint32_t kc = 0, qc = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x) {
        int b, g;
        const int nt = ix_item_tiles(p, item, b, g);
        if (nt == 0) continue;
        const int qs = qc & 1;
        if (!(ok = mbar_wait(&sh->q_empty[qs], ((qc >> 1) & 1) ^ 1, wc))) break;
        mbar_expect_tx(&sh->q_tma[qs], q_bytes);
        const int32_t qrow = (int32_t)(((int64_t)b * p.S + (int64_t)g * p.tok) * p.H);
        for (int kb = 0; kb < nkb; ++kb)
          tma_load_2d(&qmap, &sh->q_tma[qs], qbuf + qs * q_bytes + kb * (IX_N * 128),
                      kb * (int)(128 / ESZ), qrow);
        ++qc;
        for (int t = 0; t < nt; ++t) {
          const int st = kc % p.kst;
          if (!(ok = mbar_wait(&sh->k_empty[st], ((kc / p.kst) & 1) ^ 1, wc))) break;
          mbar_expect_tx(&sh->k_full[st], k_bytes);
          const int32_t krow = (int32_t)(b * p.k_rows_per_batch + t * IX_TILE_KEYS);
          for (int kb = 0; kb < nkb; ++kb)
            tma_load_2d(&kmap, &sh->k_full[st], kbuf + st * k_bytes + kb * (IX_TILE_KEYS * 128),
                        kb * (int)(128 / ESZ), krow);
          ++kc;
        }
      }
      // drain: wait for every load this thread issued (bounded)
      for (uint32_t i = (kc > (uint32_t)p.kst ? kc - p.kst : 0); i < kc; ++i)
        mbar_wait(&sh->k_full[i % p.kst], (i / p.kst) & 1, wc, false, true);
      for (uint32_t i = (qc > 2 ? qc - 2 : 0); i < qc; ++i)
        mbar_wait(&sh->q_tma[i & 1], (i >> 1) & 1, wc, false, true);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc =
          F8 ? idesc_e4m3_f32(IX_TILE_KEYS, IX_N) : idesc_bf16_f32(IX_TILE_KEYS, IX_N, false, false);
      uint32_t kc = 0, qc = 0, ac = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x) {
        int b, g;
        const int nt = ix_item_tiles(p, item, b, g);
        if (nt == 0) continue;
        const int qs = qc & 1;
        if (!(ok = mbar_wait(&sh->q_full[qs], (qc >> 1) & 1, wc))) break;
        const uint32_t qaddr = smem_u32(qbuf + qs * q_bytes);
        for (int t = 0; t < nt; ++t) {
          const int st = kc % p.kst, as = ac & 1;
          if (!(ok = mbar_wait_inl(&sh->acc_empty[as], ((ac >> 1) & 1) ^ 1, wc))) break;
          if (!(ok = mbar_wait_inl(&sh->k_full[st], (kc / p.kst) & 1, wc))) break;
          tc_fence_after();
          const uint32_t kaddr = smem_u32(kbuf + st * k_bytes);
          const uint32_t d_tmem = tmem + as * IX_N;
          // 32 bytes of K per instruction: 16 bf16 or 32 e4m3 elements
          for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sdesc_sw128(kaddr + kb * (IX_TILE_KEYS * 128) + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(qaddr + kb * (IX_N * 128) + kk * 32, 16, 1024);
              if constexpr (F8)
                umma_f8_ss(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
              else
                umma_bf16_ss(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
            }
          }
          umma_commit(&sh->k_empty[st]);
          umma_commit(&sh->acc_full[as]);
          ++kc;
          ++ac;
        }
        if (!ok) break;
        umma_commit(&sh->q_empty[qs]);
        ++qc;
      }
      umma_commit(&sh->drain);
      mbar_wait(&sh->drain, 0, wc, false, true);
    }
  } else if (warp < IX_EPI_WARP0) {
    // ------------------------------------------------------------ RoPE on the query tile
    const int t = threadIdx.x - 64;
    const int rd = p.rd;
    const int cpr = rd / 8;           // 16-byte chunks per row inside the rope segment
    const int c0 = (D - rd) / 8;      // first rope chunk of a row
    uint32_t qc = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
      int b, g;
      const int nt = ix_item_tiles(p, item, b, g);
      if (nt == 0) continue;
      const int qs = qc & 1;
      if (!mbar_wait(&sh->q_tma[qs], (qc >> 1) & 1, wc)) break;
      uint8_t* qt = qbuf + qs * q_bytes;
      for (int id = t; id < IX_N * cpr; id += IX_ROPE_THREADS) {
        const int n = id / cpr, cc = id % cpr;
        const int s = g * p.tok + n / p.H;
        if (s >= p.S) continue;
        const int cid = c0 + cc;
        uint8_t* a = qt + (cid >> 3) * (IX_N * 128) + n * 128 + (((cid & 7) ^ (n & 7)) << 4);
        uint4 v = *reinterpret_cast<uint4*>(a);
        const float4* f = reinterpret_cast<const float4*>(p.freqs + ((int64_t)s * (rd / 2) + cc * 4) * 2);
        const float4 f01 = __ldg(f), f23 = __ldg(f + 1);
        const float cs[4] = {f01.x, f01.z, f23.x, f23.z};
        const float sn[4] = {f01.y, f01.w, f23.y, f23.w};
        uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float xr = bf16lo_f32(w4[q]), xi = bf16hi_f32(w4[q]);
          const float re = __fsub_rn(__fmul_rn(xr, cs[q]), __fmul_rn(xi, sn[q]));
          const float im = __fadd_rn(__fmul_rn(xr, sn[q]), __fmul_rn(xi, cs[q]));
          w4[q] = cvt_bf16x2(re, im);
        }
        *reinterpret_cast<uint4*>(a) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&sh->q_full[qs]);
      ++qc;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Thread = key (TMEM lane); two tokens at a time, each summed in head order
    // with round-to-nearest fp32 adds (F8: the pair carried as one f32x2 value).
    const int e = warp - IX_EPI_WARP0;  // 0..7
    const int quarter = warp & 3;       // TMEM lanes [32*quarter, +32) belong to this warp
    const int half = e >> 2;            // which half of the item's tokens
    constexpr int TOK = IX_N / H;
    constexpr int TOK_HALF = TOK / 2;
    uint32_t ac = 0, ic = 0;  // tiles and (non-empty) items so far
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
      int b, g;
      const int nt = ix_item_tiles(p, item, b, g);
      if (nt == 0) continue;
      bool ok = true;
      // key limits of this warp's tokens (causal: (pos0 + s + 1) / ratio; else T),
      // fixed for the item, so the division is not repeated per tile
      int64_t lims[TOK_HALF];
#pragma unroll
      for (int u = 0; u < TOK_HALF; ++u) {
        const int s = g * TOK + half * TOK_HALF + u;
        int64_t lim = p.T;
        if (p.causal) {
          const int64_t l2 = (p.pos0 + s + 1) / p.ratio;
          lim = l2 < lim ? l2 : lim;
        }
        lims[u] = s < p.S ? lim : 0;  // rows past S are not stored
      }
      // stage the item's weights (epilogue warp 0), once every epilogue warp is
      // done with the previous item's; the others wait until they are in place
      if (e == 0) {
        if (ic > 0 && !(ok = mbar_wait(&sh->w_free, (ic - 1) & 1, wc))) break;
        const int n = lane * 8;  // 8 consecutive weights of token n / H
        const int u = n / H, h0 = n % H;
        const int su = g * TOK + u;
        const int64_t off = (int64_t)b * p.w_bs + (int64_t)(su < p.S ? su : p.S - 1) * H + h0;
        if constexpr (F8) {
          const float* src = p.wf + off;
          float4 v0, v1;
          if (p.w_vec16) {
            v0 = __ldg(reinterpret_cast<const float4*>(src));
            v1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
          } else {
            v0 = make_float4(__ldg(src), __ldg(src + 1), __ldg(src + 2), __ldg(src + 3));
            v1 = make_float4(__ldg(src + 4), __ldg(src + 5), __ldg(src + 6), __ldg(src + 7));
          }
          reinterpret_cast<float4*>(sh->wbuf + n)[0] = v0;
          reinterpret_cast<float4*>(sh->wbuf + n)[1] = v1;
        } else {
          const uint16_t* src = p.w + off;
          uint4 v;
          if (p.w_vec16) {
            v = __ldg(reinterpret_cast<const uint4*>(src));
          } else {
            uint32_t x[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = (uint32_t)__ldg(src + 2 * i) | ((uint32_t)__ldg(src + 2 * i + 1) << 16);
            v = make_uint4(x[0], x[1], x[2], x[3]);
          }
          *reinterpret_cast<uint4*>(sh->wbuf + n) = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->w_full);
      }
      if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->w_full, ic & 1, wc)))) break;
      for (int t = 0; t < nt; ++t) {
        const int as = ac & 1;
        if (!(ok = mbar_wait_inl(&sh->acc_full[as], (ac >> 1) & 1, wc))) break;
        tc_fence_after();
        const int key = t * IX_TILE_KEYS + quarter * 32 + lane;
        if constexpr (F8) {
          // per key: k_scale * sum_h relu(dot) * w, products and partial sums rounded
          // separately, two tokens at a time as one f32x2 pair
          const float ksc = key < p.T ? __ldg(p.k_scale + (int64_t)b * p.k_rows_per_batch + key) : 0.f;
#pragma unroll 1
          for (int jp = 0; jp < TOK_HALF; jp += 2) {
            const int j0 = half * TOK_HALF + jp;
            const int s0 = g * TOK + j0, s1 = s0 + 1;
            const float* wrow0 = sh->wbuf + j0 * H;
            const float* wrow1 = wrow0 + H;
            const uint32_t col0 = tmem + as * IX_N + j0 * H + ((uint32_t)(quarter * 32) << 16);
            uint64_t acc = 0;  // (token s0, token s1) partial sums, f32x2
#pragma unroll
            for (int c = 0; c < H; c += 16) {
              uint32_t r0[16], r1[16];
              tmem_ld16(col0 + c, r0);
              tmem_ld16(col0 + H + c, r1);
              float w0[16], w1[16];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 a = reinterpret_cast<const float4*>(wrow0 + c)[i];
                const float4 bq = reinterpret_cast<const float4*>(wrow1 + c)[i];
                w0[4 * i] = a.x; w0[4 * i + 1] = a.y; w0[4 * i + 2] = a.z; w0[4 * i + 3] = a.w;
                w1[4 * i] = bq.x; w1[4 * i + 1] = bq.y; w1[4 * i + 2] = bq.z; w1[4 * i + 3] = bq.w;
              }
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 16; ++h) {
                const float a0 = fmaxf(__uint_as_float(r0[h]), 0.f);
                const float a1 = fmaxf(__uint_as_float(r1[h]), 0.f);
                asm("{ .reg .b64 x, y, t; mov.b64 x, {%1, %2}; mov.b64 y, {%3, %4};"
                    " mul.rn.f32x2 t, x, y; add.rn.f32x2 %0, %0, t; }"
                    : "+l"(acc) : "f"(a0), "f"(a1), "f"(w0[h]), "f"(w1[h]));
              }
            }
            float acc0, acc1;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(acc0), "=f"(acc1) : "l"(acc));
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int s = u ? s1 : s0;
              uint16_t out = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(u ? acc1 : acc0, ksc)));
              if (key >= lims[jp + u]) out = 0xFF80;  // -inf
              if (s < p.S && key < p.T)
                p.scores[((int64_t)b * p.S + s) * p.score_ld + key] = out;
            }
          }
        } else {
#pragma unroll 1
        for (int jp = 0; jp < TOK_HALF; jp += 2) {
          const int j0 = half * TOK_HALF + jp;
          const int s0 = g * TOK + j0, s1 = s0 + 1;
          // head weights of the two tokens (shared memory, warp-uniform: broadcast)
          const uint16_t* wrow0 = sh->wbuf + j0 * H;
          const uint16_t* wrow1 = wrow0 + H;
          const uint32_t col0 = tmem + as * IX_N + j0 * H + ((uint32_t)(quarter * 32) << 16);
          float acc0 = 0.f, acc1 = 0.f;  // token s0, token s1 partial sums
#pragma unroll
          for (int c = 0; c < H; c += 16) {
            uint32_t r0[16], r1[16];
            tmem_ld16(col0 + c, r0);
            tmem_ld16(col0 + H + c, r1);
            uint32_t w0[8], w1[8];
            {
              const uint4 a0 = *reinterpret_cast<const uint4*>(wrow0 + c);
              const uint4 a1 = *reinterpret_cast<const uint4*>(wrow0 + c + 8);
              const uint4 b0 = *reinterpret_cast<const uint4*>(wrow1 + c);
              const uint4 b1 = *reinterpret_cast<const uint4*>(wrow1 + c + 8);
              w0[0] = a0.x; w0[1] = a0.y; w0[2] = a0.z; w0[3] = a0.w;
              w0[4] = a1.x; w0[5] = a1.y; w0[6] = a1.z; w0[7] = a1.w;
              w1[0] = b0.x; w1[1] = b0.y; w1[2] = b0.z; w1[3] = b0.w;
              w1[4] = b1.x; w1[5] = b1.y; w1[6] = b1.z; w1[7] = b1.w;
            }
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < 16; h += 2) {
              const uint32_t p0 = mul_bf16x2(cvt_relu_bf16x2(__uint_as_float(r0[h]), __uint_as_float(r0[h + 1])), w0[h >> 1]);
              const uint32_t p1 = mul_bf16x2(cvt_relu_bf16x2(__uint_as_float(r1[h]), __uint_as_float(r1[h + 1])), w1[h >> 1]);
              // head h (low halves), then head h + 1 (high halves): a mixed-precision
              // add takes the bf16 half as it is (exact widening, fp32 round-to-nearest
              // sum), with no separate unpacking of the pair
              asm("{ .reg .b16 l0, h0, l1, h1; mov.b32 {l0, h0}, %2; mov.b32 {l1, h1}, %3;"
                  " add.rn.f32.bf16 %0, l0, %0; add.rn.f32.bf16 %1, l1, %1;"
                  " add.rn.f32.bf16 %0, h0, %0; add.rn.f32.bf16 %1, h1, %1; }"
                  : "+f"(acc0), "+f"(acc1) : "r"(p0), "r"(p1));
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int s = u ? s1 : s0;
            uint16_t out = __bfloat16_as_ushort(__float2bfloat16_rn(u ? acc1 : acc0));
            if (key >= lims[jp + u]) out = 0xFF80;  // -inf
            if (s < p.S && key < p.T)
              p.scores[((int64_t)b * p.S + s) * p.score_ld + key] = out;
          }
        }
        }  // bf16 path
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->acc_empty[as]);
        ++ac;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->w_free);  // this warp is done with the item's weights
      ++ic;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<1>(tmem, 512);
}

}  // namespace ks
