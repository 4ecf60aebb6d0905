// Top-k sparse attention with a per-head sink on tcgen05, one CTA pair per query.
//
// Semantics follow baseline/sparse_attention.py:5-42 of KernelSwift:
//   s_t   = (q_h . kv[idx_t]) * scale, entries with idx_t < 0 masked out
//   z     = max(max_t s_t, sink_h)
//   out_h = sum_t exp(s_t - z) kv[idx_t] / (sum_t exp(s_t - z) + exp(sink_h - z))
// with repeated indices counted once per occurrence.  The reference NPU kernel
// (optimized/sparse_attention/op_kernel/fused_sparse_attn_basic_kernel.asc) runs a
// dense softmax over all N kv rows and is limited to H = 64, N = 32; here the K
// selected rows are gathered and processed online, any N.
//
// Shape of the work.  The 128 query heads of one token share the same gathered
// rows (MQA / MLA latent), and for H = 128, dv = 512 the fp32 output accumulator
// (128 x 512 x 4 B) is the whole TMEM of one SM.  So a cluster of two CTAs handles
// one token with cta_group::2 MMAs (M = 128 = 64 heads per CTA): each SM holds
// the accumulators of its 64 heads.
//   QK:  S[64 heads, 64 keys] per CTA, N = 64 keys per block; each CTA gathers
//        32 of the block's keys (all D dims) as its half of the B operand.
//   PV:  O[64 heads, dv] per CTA += P[64, 64 keys] . V[64 keys, dv]; each CTA
//        supplies its half of every PV instruction's N columns, for all 64 keys
//        (so its V rows include the peer's keys in those columns).
// Rows are gathered with 16-byte cp.async copies (the swizzle computed per copy)
// into the 128-byte-swizzled layout; the same rows serve as the K-major B
// operand of QK and the MN-major B operand of PV.  (TMA tile::gather4 moves only
// four 128-byte rows per instruction; issuing the ~136 instructions a block needs
// took ~5 us per block, so the gather is spread over 128 threads instead.)
//
// Roles per CTA (9 warps): warps 0-3 gather, warp 4 issues the MMAs in CTA 0 and
// relays CTA 1's "ready" events to CTA 0, warps 5-8 run the online softmax (base
// 2, lazy rescaling of O when the running max grows by more than 2^8) and the
// epilogue; P is double buffered so softmax(j) overlaps PV(j-1).  TMEM lane l holds head (l mod 64); lanes l and l+64
// hold the two halves of that head's keys (QK) and output columns (PV), and
// exchange their block maxima through shared memory.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int SA_THREADS = 288;
constexpr int SA_PRODUCERS = 128;  // warps 0-3
constexpr int SA_MMA_WARP = 4;
constexpr int SA_SMX_WARP0 = 5;
constexpr int SA_NB = 64;      // keys per block
constexpr int SA_HALF = 32;    // keys per CTA in the QK product
constexpr int SA_MAX_ST = 4;
constexpr int SA_HDR = 2048;   // shared header bytes

struct SaParams {
  const int32_t* idx;   // [B, M, K]
  const uint16_t* kv;   // bf16 [B, N, D]
  int32_t pv_col[2][4]; // first column (relative to dv_begin) of each 64-column V block, per CTA
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t B, M, H, D, N, K;
  int32_t dv_begin, dv, dv_pad;
  int32_t n_pv;         // PV instructions
  int32_t pv_n[2];      // N of each (128 or 256)
  int32_t n_pvblk;      // 64-column V blocks per CTA
  int32_t nst, nblk;
  int32_t idx_vec4;     // indices may be read as int4 (K % 4 == 0, 16-byte aligned)
  uint32_t q_off, p_off, st_off, st_bytes, sreg_bytes;
  float scale_log2;     // softmax_scale * log2(e)
  int* status;
  uint64_t budget_ns;
};

struct SaShared {
  uint64_t full[SA_MAX_ST], peer_full[SA_MAX_ST], empty[SA_MAX_ST];
  uint64_t s_full[2];
  // per P buffer: phase k of p_full[b] / peer_p_full[b] / p_free[b] is block b + 2k,
  // so none of them can run two phases ahead of its consumer
  uint64_t p_full[2], peer_p_full[2], p_free[2], o_full, q_full, peer_q, drain;
  uint64_t xchg[3];
  uint64_t mask[SA_MAX_ST];
  uint32_t tmem_base;
  int abort;
  float xslot[3][128];
};
static_assert(sizeof(SaShared) <= SA_HDR, "SaShared exceeds the header");

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(SA_THREADS, 1)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap qmap, SaParams p) {
  extern __shared__ uint8_t sa_raw[];
  const uint32_t raw = smem_u32(sa_raw);
  uint8_t* smem = sa_raw + (((raw + 1023u) & ~1023u) - raw);
  SaShared* sh = reinterpret_cast<SaShared*>(smem);
  uint8_t* qs = smem + p.q_off;
  uint8_t* ps = smem + p.p_off;
  uint8_t* stg = smem + p.st_off;

  const uint32_t cta = cluster_ctarank();
  const int64_t token = blockIdx.x >> 1;
  const int b = (int)(token / p.M);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.D / 64;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nst; ++i) {
      mbar_init(&sh->full[i], SA_PRODUCERS);
      mbar_init(&sh->peer_full[i], 1);
      mbar_init(&sh->empty[i], 1);
    }
    mbar_init(&sh->s_full[0], 1);
    mbar_init(&sh->s_full[1], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->p_full[i], 128);
      mbar_init(&sh->peer_p_full[i], 1);
    }
    mbar_init(&sh->p_free[0], 1);
    mbar_init(&sh->p_free[1], 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->q_full, 1);  // TMA of the query tile
    mbar_init(&sh->peer_q, 1);
    mbar_init(&sh->drain, 1);
    for (int i = 0; i < 3; ++i) mbar_init(&sh->xchg[i], 128);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == SA_MMA_WARP) {
    tmem_alloc<2>(&sh->tmem_base, 512);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp < SA_PRODUCERS / 32) {
    // ------------------------------------------------------------ gathers (cp.async)
    // Thread t copies 16-byte chunk (t % 8) of rows r = t/8 + 16 i (i < 4) of every
    // block: of all 64 keys for this CTA's V columns, and of its own 32 keys for
    // all D columns.  Indices are loaded one block ahead.
    const int t = threadIdx.x;
    const int c = t & 7, rg = t >> 3;
    if (t == 0) {
      tma_prefetch_desc(&qmap);
      mbar_expect_tx(&sh->q_full, (uint32_t)nkb * 8192u);
      const int32_t qrow = (int32_t)(token * p.H + cta * 64);
      for (int d = 0; d < nkb; ++d) tma_load_2d(&qmap, &sh->q_full, qs + d * 8192, d * 64, qrow);
    }
    const int32_t* ip = p.idx + token * p.K;
    const uint16_t* kvb = p.kv + (int64_t)b * p.N * p.D;
    int32_t cur[4], nxt[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = rg + 16 * i;
      cur[i] = k < p.K ? __ldg(ip + k) : -1;
    }
    for (int j = 0; j < p.nblk; ++j) {
      const int st = j % p.nst;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = (j + 1) * SA_NB + rg + 16 * i;
        nxt[i] = (j + 1 < p.nblk && k < p.K) ? __ldg(ip + k) : -1;
      }
      if (!mbar_wait(&sh->empty[st], ((j / p.nst) & 1) ^ 1, wc)) break;
      uint8_t* sreg = stg + st * p.st_bytes;
      uint8_t* pvreg = sreg + p.sreg_bytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rg + 16 * i;
        const bool ok = cur[i] >= 0 && cur[i] < p.N;
        const uint16_t* row = kvb + (int64_t)(ok ? cur[i] : 0) * p.D;
        const uint32_t sw = (uint32_t)((c ^ (r & 7)) << 4);
        for (int u = 0; u < p.n_pvblk; ++u) {
          const int col = p.dv_begin + p.pv_col[cta][u] + 8 * c;
          cp_async16(pvreg + u * 8192 + r * 128 + sw, row + (col < p.D ? col : 0), col < p.D ? 16u : 0u);
        }
        if ((r >> 5) == (int)cta) {
          const int rs = r & 31;
          for (int d = 0; d < nkb; ++d)
            cp_async16(sreg + d * 4096 + rs * 128 + sw, row + 64 * d + 8 * c);
        }
      }
      cp_async_arrive(&sh->full[st]);
#pragma unroll
      for (int i = 0; i < 4; ++i) cur[i] = nxt[i];
    }
    cp_async_wait_all();
    if (t == 0) mbar_wait(&sh->q_full, 0, wc, false, true);
  } else if (warp == SA_MMA_WARP) {
    if (lane == 0 && cta == 0) {
      // ---------------------------------------------------------- MMA issuer (leader CTA)
      // Issues S(j) and PV(j) in whichever order their inputs become ready:
      // S(j) needs both CTAs' gathers of block j and S buffer j%2 free (PV(j-2)
      // issued); PV(j) needs both CTAs' P(j).
      const uint32_t qaddr = smem_u32(qs), paddr = smem_u32(ps);
      const uint32_t idesc_s = idesc_bf16_f32(128, SA_NB, false, false);
      bool ok = mbar_wait(&sh->q_full, 0, wc) && mbar_wait(&sh->peer_q, 0, wc, true);
      int ns = 0, npv = 0;
      uint64_t t0 = clock64();
      const uint64_t lim = budget_cycles(p.budget_ns);
      while (ok && npv < p.nblk) {
        bool progress = false;
        if (npv < ns && mbar_poll(smem_u32(&sh->p_full[npv & 1]), (npv >> 1) & 1) &&
            mbar_poll_cluster(smem_u32(&sh->peer_p_full[npv & 1]), (npv >> 1) & 1)) {
          tc_fence_after();
          fence_proxy_async_smem();
          const int st = npv % p.nst;
          const uint32_t pvreg = smem_u32(stg + st * p.st_bytes) + p.sreg_bytes;
          uint32_t ocol = tmem + 64;
          int u = 0;
          for (int i = 0; i < p.n_pv; ++i) {
            const uint32_t idesc_pv = idesc_bf16_f32(128, p.pv_n[i], false, true);
#pragma unroll
            for (int kk = 0; kk < SA_NB / 16; ++kk) {
              const uint64_t ad = sdesc_sw128(paddr + (npv & 1) * 8192 + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(pvreg + u * 8192 + kk * 2048, 8192, 1024);
              umma_bf16_ss_cg2(ocol, ad, bd, idesc_pv, (npv > 0 || kk > 0) ? 1u : 0u);
            }
            ocol += p.pv_n[i] / 2;
            u += p.pv_n[i] / 128;
          }
          umma_commit_cg2(&sh->empty[st], 3);
          umma_commit_cg2(&sh->p_free[npv & 1], 3);
          ++npv;
          progress = true;
        }
        if (ns < p.nblk && ns <= npv + 1) {
          const int st = ns % p.nst;
          const uint32_t ph = (ns / p.nst) & 1;
          if (mbar_poll(smem_u32(&sh->full[st]), ph) &&
              mbar_poll_cluster(smem_u32(&sh->peer_full[st]), ph)) {
            tc_fence_after();
            fence_proxy_async_smem();
            const uint32_t sreg = smem_u32(stg + st * p.st_bytes);
            const uint32_t d_s = tmem + (ns & 1) * 32;
            for (int k = 0; k < p.D / 16; ++k) {
              const uint64_t ad = sdesc_sw128(qaddr + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(sreg + (k >> 2) * 4096 + (k & 3) * 32, 16, 1024);
              umma_bf16_ss_cg2(d_s, ad, bd, idesc_s, k > 0 ? 1u : 0u);
            }
            umma_commit_cg2(&sh->s_full[ns & 1], 3);
            ++ns;
            progress = true;
          }
        }
        if (progress) {
          t0 = clock64();
        } else if (*wc.abort) {
          ok = false;
        } else if ((uint64_t)clock64() - t0 > lim) {
          raise_error(wc, DEV_TIMEOUT);
          ok = false;
        }
      }
      if (ok) umma_commit_cg2(&sh->o_full, 3);
      umma_commit_cg2(&sh->drain, 1);
      mbar_wait(&sh->drain, 0, wc, false, true);
    } else if (lane == 0) {
      // ---------------------------------------------------------- relay (CTA 1)
      // Forwards "my gathers of block j landed" and "my P(j) is written" to the
      // leader CTA, each stream in order, whichever is ready first.
      bool ok = mbar_wait(&sh->q_full, 0, wc);
      if (ok) mbar_arrive_cluster(&sh->peer_q, 0);
      int nf = 0, np = 0;
      uint64_t t0 = clock64();
      const uint64_t lim = budget_cycles(p.budget_ns);
      while (ok && np < p.nblk) {
        bool progress = false;
        if (nf < p.nblk && mbar_poll(smem_u32(&sh->full[nf % p.nst]), (nf / p.nst) & 1)) {
          mbar_arrive_cluster(&sh->peer_full[nf % p.nst], 0);
          ++nf;
          progress = true;
        }
        if (np < nf && mbar_poll(smem_u32(&sh->p_full[np & 1]), (np >> 1) & 1)) {
          mbar_arrive_cluster(&sh->peer_p_full[np & 1], 0);
          ++np;
          progress = true;
        }
        if (progress) {
          t0 = clock64();
        } else if (*wc.abort) {
          ok = false;
        } else if ((uint64_t)clock64() - t0 > lim) {
          raise_error(wc, DEV_TIMEOUT);
          ok = false;
        }
      }
    }
  } else if (warp >= SA_SMX_WARP0) {
    // ------------------------------------------------------------ softmax + epilogue
    const int q4 = warp & 3;
    const int l = q4 * 32 + lane;  // TMEM lane of this thread
    const int m = l & 63, half = l >> 6;
    const int head = (int)cta * 64 + m;
    const bool real = head < p.H;
    const float sink2 = real ? __ldg(p.sink + head) * 1.4426950408889634f : 0.f;
    float m_used = sink2, lsum = 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const int o_cols = p.dv_pad / 2;
    const int32_t* ip = p.idx + token * p.K + 32 * half;  // this lane's 32 keys of a block
    // validity bits of this lane's 32 keys of block j (warp-uniform loads)
    auto valid_bits = [&](int j) -> uint32_t {
      uint32_t mk = 0;
      const int k0 = j * SA_NB + 32 * half;
      if (p.idx_vec4 && k0 + 32 <= p.K) {
        const int4* v4 = reinterpret_cast<const int4*>(ip + j * SA_NB);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int4 v = __ldg(v4 + q);
          mk |= (uint32_t)(v.x >= 0 && v.x < p.N) << (4 * q);
          mk |= (uint32_t)(v.y >= 0 && v.y < p.N) << (4 * q + 1);
          mk |= (uint32_t)(v.z >= 0 && v.z < p.N) << (4 * q + 2);
          mk |= (uint32_t)(v.w >= 0 && v.w < p.N) << (4 * q + 3);
        }
      } else {
        for (int i = 0; i < 32; ++i) {
          const int k = k0 + i;
          const int32_t v = k < p.K ? __ldg(ip + j * SA_NB + i) : -1;
          mk |= (uint32_t)(v >= 0 && v < p.N) << i;
        }
      }
      return mk;
    };
    uint32_t mk_next = valid_bits(0);
    bool ok = true;
    for (int j = 0; j < p.nblk; ++j) {
      const int sb = j & 1;
      const uint32_t mk = mk_next;
      if (j + 1 < p.nblk) mk_next = valid_bits(j + 1);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->s_full[sb], (j >> 1) & 1, wc));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(lane_base + sb * 32, r);
      tmem_wait_ld();
      float s2[32];
      float bmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        s2[i] = ((mk >> i) & 1u) ? __uint_as_float(r[i]) * p.scale_log2 : -INFINITY;
        bmax = fmaxf(bmax, s2[i]);
      }
      // block max of the head = max over this lane and its partner (lane l ^ 64)
      sh->xslot[j & 1][l] = bmax;
      mbar_arrive(&sh->xchg[j & 1]);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->xchg[j & 1], (j >> 1) & 1, wc));
      if (!ok) break;
      const float m_new = fmaxf(m_used, fmaxf(bmax, sh->xslot[j & 1][l ^ 64]));
      const bool resc = m_new > m_used + 8.f;
      float alpha = 1.f;
      if (resc) {
        alpha = ex2f(m_used - m_new);
        lsum *= alpha;
        m_used = m_new;
      }
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float e0 = ex2f(s2[2 * i] - m_used), e1 = ex2f(s2[2 * i + 1] - m_used);
        lsum += e0 + e1;
        pk[i] = cvt_bf16x2(e0, e1);
      }
      // P buffer j%2 is free once PV(j-2) is done
      if (j >= 2) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->p_free[sb], ((j >> 1) - 1) & 1, wc));
        if (!ok) break;
      }
      // rescaling O needs PV(j-1) done (rare: the running max rose by > 2^8)
      if (j >= 1 && __any_sync(0xFFFFFFFFu, resc)) {  // TMEM access is warp-wide; alpha = 1 elsewhere
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->p_free[sb ^ 1], ((j - 1) >> 1) & 1, wc));
        if (!ok) break;
        tc_fence_after();
        for (int c = 0; c < o_cols; c += 16) {
          uint32_t o[16];
          tmem_ld16(lane_base + 64 + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st16(lane_base + 64 + c, o);
        }
        tmem_wait_st();
      }
      // P row m, keys [32*half, 32*half + 32) -> 16-byte chunks 4*half .. 4*half+3
      uint8_t* prow = ps + sb * 8192 + m * 128;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = half * 4 + cc;
        *reinterpret_cast<uint4*>(prow + ((c ^ (m & 7)) << 4)) =
            make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sh->p_full[sb]);
    }
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->o_full, 0, wc));
    if (ok) {
      sh->xslot[2][l] = lsum;
      mbar_arrive(&sh->xchg[2]);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->xchg[2], 0, wc));
    }
    if (ok) {
      tc_fence_after();
      const float ltot = lsum + sh->xslot[2][l ^ 64];
      const float inv = 1.f / (ltot + ex2f(sink2 - m_used));
      uint16_t* orow = p.out + ((int64_t)token * p.H + (real ? head : 0)) * p.dv;
      int ocol = 0;
      for (int i = 0; i < p.n_pv; ++i) {
        const int hn = p.pv_n[i] / 2;
        const int d0 = 256 * i + half * hn;
        for (int c = 0; c < hn; c += 16) {
          uint32_t o[16];
          tmem_ld16(lane_base + 64 + ocol + c, o);
          tmem_wait_ld();
          if (real && d0 + c < p.dv) {
            uint32_t w[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              w[t] = cvt_bf16x2(__uint_as_float(o[2 * t]) * inv, __uint_as_float(o[2 * t + 1]) * inv);
            uint4* dst = reinterpret_cast<uint4*>(orow + d0 + c);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
        ocol += hn;
      }
    }
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == SA_MMA_WARP) tmem_dealloc<2>(tmem, 512);
}

}  // namespace ks
