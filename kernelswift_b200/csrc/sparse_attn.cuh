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
// the accumulators of its 64 heads.  Keys are processed in blocks of 256:
//   QK:  S[64 heads, 256 keys] per CTA with N = 256 per instruction; each CTA
//        supplies 128 of the block's keys as its half of the B operand, streamed
//        through a ring of 64-dim chunks (128 keys x 64 dims = 16 KB).
//   PV:  O[64 heads, dv] per CTA += P[64, 256] . V[256, dv] in four 64-key chunks;
//        each CTA supplies its half of every PV instruction's N columns for the
//        64 keys of a chunk, streamed through a ring of V chunks.
// Rows are gathered by 256 threads with 16-byte loads into registers and 16-byte
// shared stores (the swizzle computed per store) into the 128-byte-swizzled
// layout the MMAs read (K-major for QK, MN-major for PV).  Random 128-byte rows
// need many loads in flight: measured per SM, cp.async from 128 threads stays near
// 50 GB/s whatever the ring depth, register-staged loads from 256 threads reach
// ~113 GB/s (8 loads in flight each).  Per 256 keys an SM runs 36 + 32 MMAs of 64
// tensor cycles each and gathers ~275 KB.
//
// Roles per CTA (13 warps): warps 0-7 gather, warp 8 issues the MMAs in CTA 0 and
// relays CTA 1's "ready" events to CTA 0 (both with suspending waits, in the
// order the gathers are produced), warps 9-12 run the online softmax (base
// 2, lazy rescaling of O when the running max grows by more than 2^8) and the
// epilogue.  TMEM lane l holds head (l mod 64); lanes l and l+64 hold the two
// halves of that head's keys (QK) and output columns (PV) and exchange their
// block maxima through shared memory.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int SA_THREADS = 416;
constexpr int SA_PRODUCERS = 256;   // warps 0-7
constexpr int SA_MMA_WARP = 8;
constexpr int SA_SMX_WARP0 = 9;
constexpr int SA_NB = 256;          // keys per block
constexpr int SA_HALF = 128;        // keys per CTA in the QK product
constexpr int SA_KC = 64;           // keys per PV chunk
constexpr int SA_NKC = SA_NB / SA_KC;
constexpr int SA_MAX_S = 4;         // QK chunk ring slots
constexpr int SA_MAX_V = 4;         // V chunk ring slots
constexpr int SA_HDR = 2048;        // shared header bytes
constexpr uint32_t SA_SCHUNK = SA_HALF * 128;  // 128 keys x 64 dims bf16
constexpr uint32_t SA_PBYTES = 64 * SA_NB * 2; // P: 64 heads x 256 keys bf16
constexpr int SA_SCOLS = SA_NB / 2;            // TMEM columns of one S buffer (2x2 layout)
constexpr int SA_OCOL = 2 * SA_SCOLS;          // first TMEM column of O

struct SaParams {
  const int32_t* idx;   // [B, M, K]
  const uint16_t* kv;   // bf16 [B, N, D]
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t pv_col[2][4]; // first column (relative to dv_begin) of each 64-column V block, per CTA
  int32_t B, M, H, D, N, K;
  int32_t dv_begin, dv, dv_pad;
  int32_t n_pv;         // PV instructions per 64-key chunk
  int32_t pv_n[2];      // N of each (128 or 256)
  int32_t n_pvblk;      // 64-column V blocks per CTA
  int32_t ns_slots, nv_slots, nblk;
  int32_t idx_vec4;     // indices may be read as int4 (K % 4 == 0, 16-byte aligned)
  uint32_t q_off, p_off, s_off, v_off, v_bytes;
  float scale_log2;     // softmax_scale * log2(e)
  int* status;
  uint64_t budget_ns;
};

struct SaShared {
  uint64_t s_full[SA_MAX_S], peer_s_full[SA_MAX_S], s_empty[SA_MAX_S];
  uint64_t v_full[SA_MAX_V], peer_v_full[SA_MAX_V], v_empty[SA_MAX_V];
  uint64_t acc_full[2];
  uint64_t p_full, peer_p_full, p_free, o_full, q_full, peer_q, drain;
  uint64_t xchg[3];
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

  const uint32_t cta = cluster_ctarank();
  const int64_t token = blockIdx.x >> 1;
  const int b = (int)(token / p.M);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.D / 64;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.ns_slots; ++i) {
      mbar_init(&sh->s_full[i], SA_PRODUCERS);
      mbar_init(&sh->peer_s_full[i], 1);
      mbar_init(&sh->s_empty[i], 1);
    }
    for (int i = 0; i < p.nv_slots; ++i) {
      mbar_init(&sh->v_full[i], SA_PRODUCERS);
      mbar_init(&sh->peer_v_full[i], 1);
      mbar_init(&sh->v_empty[i], 1);
    }
    mbar_init(&sh->acc_full[0], 1);
    mbar_init(&sh->acc_full[1], 1);
    mbar_init(&sh->p_full, 128);
    mbar_init(&sh->peer_p_full, 1);
    mbar_init(&sh->p_free, 1);
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
    // ------------------------------------------------------------ gathers
    // Thread t moves 16-byte piece (t % 8) of rows t/8 + 32 i.  Order: the QK
    // chunks of block j (this CTA's 128 keys, 64 dims each; two chunks per round so
    // eight loads are in flight), then the V chunks of block j-1 (64 keys, this
    // CTA's V columns) - the order the MMAs consume them.  Shared stores are
    // generic-proxy writes: each thread fences them for the tensor core before it
    // arrives on the slot's barrier.
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
    auto idx_at = [&](int key) -> int32_t { return key < p.K ? __ldg(ip + key) : -1; };
    auto row_of = [&](int32_t v) -> const uint16_t* {
      return kvb + (int64_t)((v >= 0 && v < p.N) ? v : 0) * p.D;
    };
    // indices of this thread's rows, loaded one block ahead:
    //   s_idx: QK rows of block j (this CTA's keys), v_idx: V rows of block j-1
    int32_t s_idx[4], v_idx[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) s_idx[i] = idx_at((int)cta * SA_HALF + rg + 32 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) v_idx[i] = -1;
    uint32_t sc = 0, vc = 0;
    bool ok = true;
    for (int j = 0; ok && j <= p.nblk; ++j) {
      int32_t s_nxt[4], v_nxt[8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        s_nxt[i] = j + 1 < p.nblk ? idx_at((j + 1) * SA_NB + (int)cta * SA_HALF + rg + 32 * i) : -1;
#pragma unroll
      for (int i = 0; i < 8; ++i)  // chunk i/2, row rg + 32 (i%2)
        v_nxt[i] = j < p.nblk ? idx_at(j * SA_NB + (i >> 1) * SA_KC + rg + 32 * (i & 1)) : -1;
      if (j < p.nblk) {
        const uint16_t* rows[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rows[i] = row_of(s_idx[i]) + 8 * c;
        for (int d = 0; d < nkb; d += 2) {
          const bool two = d + 1 < nkb;
          uint4 v[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[i] = __ldcg(reinterpret_cast<const uint4*>(rows[i] + 64 * d));
            if (two) v[4 + i] = __ldcg(reinterpret_cast<const uint4*>(rows[i] + 64 * (d + 1)));
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            const int slot = sc % p.ns_slots;
            if (!(ok = mbar_wait(&sh->s_empty[slot], ((sc / p.ns_slots) & 1) ^ 1, wc))) break;
            uint8_t* dst = smem + p.s_off + slot * SA_SCHUNK;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = rg + 32 * i;
              *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = v[4 * h + i];
            }
            fence_proxy_async_smem();
            mbar_arrive(&sh->s_full[slot]);
            ++sc;
          }
          if (!ok) break;
        }
      }
      if (ok && j >= 1) {
        for (int kc = 0; kc < SA_NKC; ++kc, ++vc) {
          uint4 v[8];
          const uint16_t* row0 = row_of(v_idx[2 * kc]);
          const uint16_t* row1 = row_of(v_idx[2 * kc + 1]);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (u < p.n_pvblk) {
              const int col = p.dv_begin + p.pv_col[cta][u] + 8 * c;
              const bool in = col < p.D;
              v[2 * u] = in ? __ldcg(reinterpret_cast<const uint4*>(row0 + col)) : make_uint4(0, 0, 0, 0);
              v[2 * u + 1] = in ? __ldcg(reinterpret_cast<const uint4*>(row1 + col)) : make_uint4(0, 0, 0, 0);
            }
          }
          const int slot = vc % p.nv_slots;
          if (!(ok = mbar_wait(&sh->v_empty[slot], ((vc / p.nv_slots) & 1) ^ 1, wc))) break;
          uint8_t* dst = smem + p.v_off + slot * p.v_bytes;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (u < p.n_pvblk) {
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int r = rg + 32 * i;
                *reinterpret_cast<uint4*>(dst + u * 8192 + r * 128 + ((c ^ (r & 7)) << 4)) = v[2 * u + i];
              }
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(&sh->v_full[slot]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) s_idx[i] = s_nxt[i];
#pragma unroll
      for (int i = 0; i < 8; ++i) v_idx[i] = v_nxt[i];
    }
    if (t == 0) mbar_wait(&sh->q_full, 0, wc, false, true);
  } else if (warp == SA_MMA_WARP) {
    if (lane == 0 && cta == 0) {
      // ---------------------------------------------------------- MMA issuer (leader CTA)
      // Consumption order = production order: the QK chunks of block j, then
      // P(j-1) and the V chunks of block j-1.  Blocking (suspending) waits.
      const uint32_t qaddr = smem_u32(qs), paddr = smem_u32(ps);
      const uint32_t idesc_s = idesc_bf16_f32(128, SA_NB, false, false);
      bool ok = mbar_wait(&sh->q_full, 0, wc) && mbar_wait(&sh->peer_q, 0, wc, true);
      uint32_t sc = 0, vc = 0;
      for (int j = 0; ok && j <= p.nblk; ++j) {
        if (j < p.nblk) {
          // S buffer j%2 was last read by softmax(j-2), whose P was consumed by PV(j-2)
          const uint32_t d_s = tmem + (j & 1) * SA_SCOLS;
          for (int d = 0; d < nkb; ++d, ++sc) {
            const int slot = sc % p.ns_slots;
            const uint32_t ph = (sc / p.ns_slots) & 1;
            if (!(ok = mbar_wait(&sh->s_full[slot], ph, wc) &&
                       mbar_wait(&sh->peer_s_full[slot], ph, wc, true)))
              break;
            tc_fence_after();
            fence_proxy_async_smem();
            const uint32_t saddr = smem_u32(smem + p.s_off + slot * SA_SCHUNK);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sdesc_sw128(qaddr + d * 8192 + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(saddr + kk * 32, 16, 1024);
              umma_bf16_ss_cg2(d_s, ad, bd, idesc_s, (d > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit_cg2(&sh->s_empty[slot], 3);
          }
          if (!ok) break;
          umma_commit_cg2(&sh->acc_full[j & 1], 3);
        }
        if (j >= 1) {
          const int jj = j - 1;
          if (!(ok = mbar_wait(&sh->p_full, jj & 1, wc) &&
                     mbar_wait(&sh->peer_p_full, jj & 1, wc, true)))
            break;
          for (int kc = 0; kc < SA_NKC; ++kc, ++vc) {
            const int slot = vc % p.nv_slots;
            const uint32_t ph = (vc / p.nv_slots) & 1;
            if (!(ok = mbar_wait(&sh->v_full[slot], ph, wc) &&
                       mbar_wait(&sh->peer_v_full[slot], ph, wc, true)))
              break;
            tc_fence_after();
            fence_proxy_async_smem();
            const uint32_t vaddr = smem_u32(smem + p.v_off + slot * p.v_bytes);
            uint32_t ocol = tmem + SA_OCOL;
            int u = 0;
            for (int i = 0; i < p.n_pv; ++i) {
              const uint32_t idesc_pv = idesc_bf16_f32(128, p.pv_n[i], false, true);
#pragma unroll
              for (int kk = 0; kk < SA_KC / 16; ++kk) {
                const uint64_t ad = sdesc_sw128(paddr + kc * 8192 + kk * 32, 16, 1024);
                const uint64_t bd = sdesc_sw128(vaddr + u * 8192 + kk * 2048, 8192, 1024);
                umma_bf16_ss_cg2(ocol, ad, bd, idesc_pv, (jj > 0 || kc > 0 || kk > 0) ? 1u : 0u);
              }
              ocol += p.pv_n[i] / 2;
              u += p.pv_n[i] / 128;
            }
            umma_commit_cg2(&sh->v_empty[slot], 3);
          }
          if (!ok) break;
          umma_commit_cg2(&sh->p_free, 3);
        }
      }
      if (ok) umma_commit_cg2(&sh->o_full, 3);
      umma_commit_cg2(&sh->drain, 1);
      mbar_wait(&sh->drain, 0, wc, false, true);
    } else if (lane == 0) {
      // ---------------------------------------------------------- relay (CTA 1)
      // Forwards "my QK chunk landed", "my P is written" and "my V chunk landed"
      // to the leader CTA, in the leader's consumption order.
      bool ok = mbar_wait(&sh->q_full, 0, wc);
      if (ok) mbar_arrive_cluster(&sh->peer_q, 0);
      uint32_t sc = 0, vc = 0;
      for (int j = 0; ok && j <= p.nblk; ++j) {
        if (j < p.nblk) {
          for (int d = 0; d < nkb; ++d, ++sc) {
            if (!(ok = mbar_wait(&sh->s_full[sc % p.ns_slots], (sc / p.ns_slots) & 1, wc))) break;
            mbar_arrive_cluster(&sh->peer_s_full[sc % p.ns_slots], 0);
          }
          if (!ok) break;
        }
        if (j >= 1) {
          if (!(ok = mbar_wait(&sh->p_full, (j - 1) & 1, wc))) break;
          mbar_arrive_cluster(&sh->peer_p_full, 0);
          for (int kc = 0; kc < SA_NKC; ++kc, ++vc) {
            if (!(ok = mbar_wait(&sh->v_full[vc % p.nv_slots], (vc / p.nv_slots) & 1, wc))) break;
            mbar_arrive_cluster(&sh->peer_v_full[vc % p.nv_slots], 0);
          }
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
    const int32_t* ip = p.idx + token * p.K;
    // validity bits of this lane's 128 keys of block j (warp-uniform loads)
    auto valid_bits = [&](int j, uint32_t* mk) {
      const int k0 = j * SA_NB + half * SA_HALF;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t bits = 0;
        const int kw = k0 + 32 * w;
        if (p.idx_vec4 && kw + 32 <= p.K) {
          const int4* v4 = reinterpret_cast<const int4*>(ip + kw);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int4 v = __ldg(v4 + q);
            bits |= (uint32_t)(v.x >= 0 && v.x < p.N) << (4 * q);
            bits |= (uint32_t)(v.y >= 0 && v.y < p.N) << (4 * q + 1);
            bits |= (uint32_t)(v.z >= 0 && v.z < p.N) << (4 * q + 2);
            bits |= (uint32_t)(v.w >= 0 && v.w < p.N) << (4 * q + 3);
          }
        } else {
          for (int i = 0; i < 32; ++i) {
            const int k = kw + i;
            const int32_t v = k < p.K ? __ldg(ip + k) : -1;
            bits |= (uint32_t)(v >= 0 && v < p.N) << i;
          }
        }
        mk[w] = bits;
      }
    };
    bool ok = true;
    for (int j = 0; j < p.nblk; ++j) {
      const int sb = j & 1;
      uint32_t mk[4];
      valid_bits(j, mk);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->acc_full[sb], (j >> 1) & 1, wc));
      if (!ok) break;
      tc_fence_after();
      const uint32_t sbase = lane_base + sb * SA_SCOLS;
      // pass 1: block max over this lane's 128 keys
      float bmax = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t r[32];
        tmem_ld32(sbase + 32 * w, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if ((mk[w] >> i) & 1u) bmax = fmaxf(bmax, __uint_as_float(r[i]) * p.scale_log2);
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
      if (j >= 1) {
        // P buffer free and O stable: PV of block j-1 done
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->p_free, (j - 1) & 1, wc));
        if (!ok) break;
        if (__any_sync(0xFFFFFFFFu, resc)) {  // TMEM access is warp-wide; alpha = 1 elsewhere
          tc_fence_after();
          for (int c = 0; c < o_cols; c += 16) {
            uint32_t o[16];
            tmem_ld16(lane_base + SA_OCOL + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st16(lane_base + SA_OCOL + c, o);
          }
          tmem_wait_st();
        }
      }
      // pass 2: probabilities as bf16, straight into P row m, keys [128*half, +128)
      // (64-key blocks 2*half and 2*half + 1; 32 keys = four 16-byte chunks per step)
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t r[32];
        tmem_ld32(sbase + 32 * w, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float s0 = ((mk[w] >> (2 * i)) & 1u) ? __uint_as_float(r[2 * i]) * p.scale_log2 : -INFINITY;
          const float s1 = ((mk[w] >> (2 * i + 1)) & 1u) ? __uint_as_float(r[2 * i + 1]) * p.scale_log2 : -INFINITY;
          const float e0 = ex2f(s0 - m_used), e1 = ex2f(s1 - m_used);
          lsum += e0 + e1;
          pk[i] = cvt_bf16x2(e0, e1);
        }
        uint8_t* prow = ps + (2 * half + (w >> 1)) * 8192 + m * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int cc = (w & 1) * 4 + q;
          *reinterpret_cast<uint4*>(prow + ((cc ^ (m & 7)) << 4)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
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
          tmem_ld16(lane_base + SA_OCOL + ocol + c, o);
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
