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
// Rows are gathered from HBM/L2 with TMA tile::gather4 (4 rows x 128 bytes per
// instruction) into the 128-byte-swizzled layout; the same rows serve as the
// K-major B operand of QK and the MN-major B operand of PV.
//
// Roles per CTA (6 warps): warp 0 gathers (one lane), warp 1 issues the MMAs in
// CTA 0 and relays CTA 1's "ready" events to CTA 0, warps 2-5 run the online
// softmax (base 2, lazy rescaling of O when the running max grows by more than
// 2^8) and the epilogue.  TMEM lane l holds head (l mod 64); lanes l and l+64
// hold the two halves of that head's keys (QK) and output columns (PV), and
// exchange their block maxima through shared memory.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int SA_THREADS = 192;
constexpr int SA_NB = 64;      // keys per block
constexpr int SA_HALF = 32;    // keys per CTA in the QK product
constexpr int SA_MAX_ST = 4;
constexpr int SA_HDR = 2048;   // shared header bytes

struct SaParams {
  const int32_t* idx;   // [B, M, K]
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t B, M, H, D, N, K;
  int32_t dv_begin, dv, dv_pad;
  int32_t n_pv;         // PV instructions
  int32_t pv_n[2];      // N of each (128 or 256)
  int32_t n_pvblk;      // 64-column V blocks per CTA
  int32_t nst, nblk;
  uint32_t q_off, p_off, st_off, st_bytes, sreg_bytes;
  float scale_log2;     // softmax_scale * log2(e)
  int* status;
  uint64_t budget_ns;
};

struct SaShared {
  uint64_t full[SA_MAX_ST], peer_full[SA_MAX_ST], empty[SA_MAX_ST];
  uint64_t s_full[2];
  uint64_t p_full, peer_p_full, p_free, o_full, q_full, peer_q, drain;
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
    sparse_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kvmap, SaParams p) {
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
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->peer_full[i], 1);
      mbar_init(&sh->empty[i], 1);
    }
    mbar_init(&sh->s_full[0], 1);
    mbar_init(&sh->s_full[1], 1);
    mbar_init(&sh->p_full, 128);
    mbar_init(&sh->peer_p_full, 1);
    mbar_init(&sh->p_free, 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->q_full, 1);
    mbar_init(&sh->peer_q, 1);
    mbar_init(&sh->drain, 1);
    for (int i = 0; i < 3; ++i) mbar_init(&sh->xchg[i], 128);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(&sh->tmem_base, 512);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ gathers (TMA)
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kvmap);
      mbar_expect_tx(&sh->q_full, (uint32_t)nkb * 8192u);
      const int32_t qrow = (int32_t)(token * p.H + cta * 64);
      for (int d = 0; d < nkb; ++d) tma_load_2d(&qmap, &sh->q_full, qs + d * 8192, d * 64, qrow);
      const int32_t* ip = p.idx + token * p.K;
      const uint32_t stage_tx = (uint32_t)(nkb * SA_HALF + p.n_pvblk * SA_NB) * 128u;
      int issued = 0;
      for (int j = 0; j < p.nblk; ++j) {
        const int st = j % p.nst;
        if (!mbar_wait(&sh->empty[st], ((j / p.nst) & 1) ^ 1, wc)) break;
        int32_t rows[SA_NB];
        uint64_t mask = 0;
#pragma unroll
        for (int i = 0; i < SA_NB; ++i) {
          const int kk = j * SA_NB + i;
          const int32_t v = kk < p.K ? __ldg(ip + kk) : -1;
          const bool ok = v >= 0 && v < p.N;
          mask |= (uint64_t)ok << i;
          rows[i] = b * p.N + (ok ? v : 0);
        }
        sh->mask[st] = mask;
        mbar_expect_tx(&sh->full[st], stage_tx);
        uint8_t* sreg = stg + st * p.st_bytes;
        for (int d = 0; d < nkb; ++d) {
#pragma unroll
          for (int g = 0; g < SA_HALF / 4; ++g) {
            const int r = cta * SA_HALF + 4 * g;
            tma_gather4(&kvmap, &sh->full[st], sreg + d * 4096 + g * 512, d * 64, rows[r],
                        rows[r + 1], rows[r + 2], rows[r + 3]);
          }
        }
        uint8_t* pvreg = sreg + p.sreg_bytes;
        int u = 0;
        for (int i = 0; i < p.n_pv; ++i) {
          const int hn = p.pv_n[i] / 2;
          for (int v = 0; v < hn / 64; ++v, ++u) {
            const int col = p.dv_begin + 256 * i + (int)cta * hn + 64 * v;
#pragma unroll
            for (int g = 0; g < SA_NB / 4; ++g)
              tma_gather4(&kvmap, &sh->full[st], pvreg + u * 8192 + g * 512, col, rows[4 * g],
                          rows[4 * g + 1], rows[4 * g + 2], rows[4 * g + 3]);
          }
        }
        ++issued;
      }
      for (int i = issued > p.nst ? issued - p.nst : 0; i < issued; ++i)
        mbar_wait(&sh->full[i % p.nst], (i / p.nst) & 1, wc, false, true);
      mbar_wait(&sh->q_full, 0, wc, false, true);
    }
  } else if (warp == 1) {
    if (lane == 0 && cta == 0) {
      // ---------------------------------------------------------- MMA issuer (leader CTA)
      const uint32_t qaddr = smem_u32(qs), paddr = smem_u32(ps);
      const uint32_t idesc_s = idesc_bf16_f32(128, SA_NB, false, false);
      bool ok = mbar_wait(&sh->q_full, 0, wc) && mbar_wait(&sh->peer_q, 0, wc, true);
      for (int j = 0; ok && j <= p.nblk; ++j) {
        if (j < p.nblk) {
          const int st = j % p.nst;
          const uint32_t ph = (j / p.nst) & 1;
          if (!(ok = mbar_wait(&sh->full[st], ph, wc))) break;
          if (!(ok = mbar_wait(&sh->peer_full[st], ph, wc, true))) break;
          tc_fence_after();
          const uint32_t sreg = smem_u32(stg + st * p.st_bytes);
          const uint32_t d_s = tmem + (j & 1) * 32;
          for (int k = 0; k < p.D / 16; ++k) {
            const uint64_t ad = sdesc_sw128(qaddr + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(sreg + (k >> 2) * 4096 + (k & 3) * 32, 16, 1024);
            umma_bf16_ss_cg2(d_s, ad, bd, idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit_cg2(&sh->s_full[j & 1], 3);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj % p.nst;
          if (!(ok = mbar_wait(&sh->p_full, jj & 1, wc))) break;
          if (!(ok = mbar_wait(&sh->peer_p_full, jj & 1, wc, true))) break;
          tc_fence_after();
          const uint32_t pvreg = smem_u32(stg + st * p.st_bytes) + p.sreg_bytes;
          uint32_t ocol = tmem + 64;
          int u = 0;
          for (int i = 0; i < p.n_pv; ++i) {
            const uint32_t idesc_pv = idesc_bf16_f32(128, p.pv_n[i], false, true);
#pragma unroll
            for (int kk = 0; kk < SA_NB / 16; ++kk) {
              const uint64_t ad = sdesc_sw128(paddr + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(pvreg + u * 8192 + kk * 2048, 8192, 1024);
              umma_bf16_ss_cg2(ocol, ad, bd, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
            }
            ocol += p.pv_n[i] / 2;
            u += p.pv_n[i] / 128;
          }
          umma_commit_cg2(&sh->empty[st], 3);
          umma_commit_cg2(&sh->p_free, 3);
        }
      }
      if (ok) umma_commit_cg2(&sh->o_full, 3);
      umma_commit_cg2(&sh->drain, 1);
      mbar_wait(&sh->drain, 0, wc, false, true);
    } else if (lane == 0) {
      // ---------------------------------------------------------- relay (CTA 1)
      bool ok = mbar_wait(&sh->q_full, 0, wc);
      if (ok) mbar_arrive_cluster(&sh->peer_q, 0);
      for (int j = 0; ok && j <= p.nblk; ++j) {
        if (j < p.nblk) {
          const int st = j % p.nst;
          if (!(ok = mbar_wait(&sh->full[st], (j / p.nst) & 1, wc))) break;
          mbar_arrive_cluster(&sh->peer_full[st], 0);
        }
        if (j >= 1) {
          if (!(ok = mbar_wait(&sh->p_full, (j - 1) & 1, wc))) break;
          mbar_arrive_cluster(&sh->peer_p_full, 0);
        }
      }
    }
  } else {
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
    bool ok = true;
    for (int j = 0; j < p.nblk; ++j) {
      const int sb = j & 1, st = j % p.nst;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->s_full[sb], (j >> 1) & 1, wc));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(lane_base + sb * 32, r);
      tmem_wait_ld();
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->full[st], (j / p.nst) & 1, wc));
      if (!ok) break;
      const uint32_t mk = (uint32_t)(sh->mask[st] >> (half * 32));
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
      if (j >= 1) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->p_free, (j - 1) & 1, wc));
        if (!ok) break;
        if (__any_sync(0xFFFFFFFFu, resc)) {  // TMEM access is warp-wide; alpha = 1 elsewhere
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
      }
      // P row m, keys [32*half, 32*half + 32) -> 16-byte chunks 4*half .. 4*half+3
      uint8_t* prow = ps + m * 128;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = half * 4 + cc;
        *reinterpret_cast<uint4*>(prow + ((c ^ (m & 7)) << 4)) =
            make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sh->p_full);
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
  if (warp == 1) tmem_dealloc<2>(tmem, 512);
}

}  // namespace ks
