// Top-k sparse attention with a per-head sink on tcgen05, one CTA pair per query
// token at a time, persistent over the tokens.
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
//        supplies 128 of the block's keys as its half of the B operand, in
//        64-dim chunks (128 keys x 64 dims = 16 KB).
//   PV:  O[64 heads, dv] per CTA += P[64, 256] . V[256, dv] in eight 32-key
//        chunks; each CTA supplies its half of every PV instruction's N columns
//        for the 32 keys of a chunk (up to 16 KB).
// All chunks go through ONE ring of 16 KB slots in the order the MMAs consume
// them: S(0) | S(1) V(0) | S(2) V(1) | ... | V(nblk-1), where S(j) = the nkb QK
// chunks of block j and V(j) its 8 V chunks.  S(j+1) runs on the tensor cores
// while the softmax of block j works; V(j) follows once P(j) is written.
//
// Gathers.  Rows are random 128-byte pieces; they are moved with 16-byte loads
// into registers and 16-byte shared stores (the swizzle computed per store) into
// the 128-byte-swizzled layouts the MMAs read (K-major for QK, MN-major for PV).
// A thread's proxy fence and barrier arrive wait for every load it still has in
// flight, so one thread cannot overlap two chunks; instead five groups of two
// warps take turns (group g fills chunks g, g + 5, ...): each group loads a whole
// chunk into registers (16 loads per thread) before its slot is free, so up to
// 80 KB per SM are in flight while the slots turn over.  Measured per SM on
// random rows: register-staged loads reach ~120 GB/s with 32 KB in flight;
// cp.async saturates near 16 KB in flight (~55 GB/s) and TMA tile::gather4 near
// 48 GB/s with 16 issuing warps.  Per 256 keys an SM runs 36 + 32 MMAs of 64
// tensor cycles each and gathers ~272 KB.
//
// Persistent CTA pairs.  Each cluster takes tokens cid, cid + clusters, ... in
// turn; the ring, every barrier phase and the S/P buffers continue from one
// token to the next (global block index), so the next token's gathers, query
// tile and first QK blocks overlap the previous token's last PV and epilogue.
// The query tile is reloaded once the token's last QK MMAs have read it
// ("q_free", committed by the QK issuer to both CTAs); a token's first PV (which
// overwrites O) waits for its P, which the softmax warps write only after they
// have read the previous token's O out.
//
// Roles per CTA (16 warps; registers are granted per four warps, so 13 would
// cost the same):
//   warps 0-7   four gather groups (warps 2g, 2g + 1),
//   warps 8, 9  issue the MMAs in CTA 0: warp 8 the QK chunks (and loads the
//               leader's query tiles), warp 9 the V chunks; in CTA 1 warp 8
//               loads that CTA's query tiles and forwards "query tile landed",
//   warps 10-11 a fifth gather group,
//   warps 12-15 online softmax (base 2, lazy rescaling of O when the running max
//               grows by more than 2^8) and the epilogue.
// TMEM lane l holds head (l mod 64); lanes l and l+64 hold the two halves of that
// head's keys (QK) and output columns (PV) and exchange their block maxima
// through shared memory.
#pragma once
#include "ks_device.cuh"

namespace ks {

// Event timestamps of the first CTA pair for pipeline studies: a build that
// defines KS_SA_TRACE(ev, i) records them; normal builds compile them out.
#ifndef KS_SA_TRACE
#define KS_SA_TRACE(ev, i) do { } while (0)
#endif

constexpr int SA_THREADS = 512;
constexpr int SA_GROUPS = 5;        // gather groups (warps 0-7 and 10-11)
constexpr int SA_GROUP = 64;        // threads per gather group
constexpr int SA_MMA_WARP = 8;
constexpr int SA_SMX_WARP0 = 12;
constexpr int SA_SMX_WARPS = 4;
constexpr int SA_NB = 256;          // keys per block
constexpr int SA_HALF = 128;        // keys per CTA in the QK product
constexpr int SA_KC = 32;           // keys per V chunk
constexpr int SA_NKC = SA_NB / SA_KC;
constexpr int SA_MAX_SLOTS = 10;    // ring slots (a multiple of SA_GROUPS)
constexpr int SA_HDR = 2048;        // shared header bytes
constexpr uint32_t SA_SLOT = SA_HALF * 128;    // 16 KB: 128 keys x 64 dims bf16
constexpr uint32_t SA_VSEG = SA_KC * 128;      // one 64-column V segment of a chunk
constexpr uint32_t SA_PBYTES = 64 * SA_NB * 2; // P: 64 heads x 256 keys bf16
constexpr int SA_SCOLS = SA_NB / 2;            // TMEM columns of one S buffer (2x2 layout)
constexpr int SA_OCOL = 2 * SA_SCOLS;          // first TMEM column of O

struct SaParams {
  const int32_t* idx;   // [B, M, K]
  const uint16_t* kv;   // bf16 [B, N, D]
  const float* sink;    // [H]
  uint16_t* out;        // bf16 [B, M, H, dv]
  int32_t pv_col[2][4]; // first column (relative to dv_begin) of each 64-column V segment, per CTA
  int32_t B, M, H, D, N, K;
  int32_t dv_begin, dv, dv_pad;
  int32_t n_pv;         // PV instructions per 16-key step
  int32_t pv_n[2];      // N of each (128 or 256)
  int32_t n_pvblk;      // 64-column V segments per CTA
  int32_t n_slots, nblk;
  int32_t idx_vec4;     // indices may be read as int4 (K % 4 == 0, 16-byte aligned)
  uint32_t q_off, p_off, r_off;  // query tile, P, ring
  float scale_log2;     // softmax_scale * log2(e)
  int32_t out_v8;       // out is 32-byte aligned: 32-byte row stores
  int* status;
  uint64_t budget_ns;
};

struct SaShared {
  uint64_t full_s[SA_MAX_SLOTS], full_v[SA_MAX_SLOTS], empty[SA_MAX_SLOTS];
  uint64_t acc_full[2], s_free[2];
  // per P buffer: with two buffers the softmax can finish P(j + 1) before the V
  // issuer has seen P(j), so one barrier would run two phases ahead of its waiter
  uint64_t p_full[2], p_free[2], o_full, q_full, q_free, peer_q, drain_s, drain_v;
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

// One warp's "my part of this chunk is in shared memory" for the leader CTA's
// barrier: every lane fences its own stores for the tensor core (async proxy),
// then one lane arrives, locally in CTA 0 or remotely (release, cluster scope)
// from CTA 1.
__device__ __forceinline__ void sa_warp_ready(uint64_t* bar, uint32_t cta, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (cta == 0) mbar_arrive(bar);
    else mbar_arrive_cluster(bar, 0);
  }
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
  // this cluster's tokens: cid, cid + ncl, ... (n_it of them; the grid has at
  // most one cluster per token)
  const int64_t n_tok = (int64_t)p.B * p.M;
  const int64_t cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int n_it = (int)((n_tok - cid + ncl - 1) / ncl);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.D / 64;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.n_slots; ++i) {
      mbar_init(&sh->full_s[i], 2 * (SA_GROUP / 32));  // the filling group's warps, both CTAs
      mbar_init(&sh->full_v[i], 2 * (SA_GROUP / 32));
      mbar_init(&sh->empty[i], 1);
    }
    mbar_init(&sh->acc_full[0], 1);
    mbar_init(&sh->acc_full[1], 1);
    mbar_init(&sh->s_free[0], 2 * SA_SMX_WARPS);
    mbar_init(&sh->s_free[1], 2 * SA_SMX_WARPS);
    mbar_init(&sh->p_full[0], 2 * SA_SMX_WARPS);
    mbar_init(&sh->p_full[1], 2 * SA_SMX_WARPS);
    mbar_init(&sh->p_free[0], 1);
    mbar_init(&sh->p_free[1], 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->q_full, 1);  // TMA of the query tile
    mbar_init(&sh->q_free, 1);  // the token's last QK MMAs have read it (commit, both CTAs)
    mbar_init(&sh->peer_q, 1);
    mbar_init(&sh->drain_s, 1);
    mbar_init(&sh->drain_v, 1);
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
  // Indices are fetched raw (-1 past K) well before they are used and checked
  // only then, so no thread waits on an index load; a masked key (negative or
  // beyond N) is gathered as zeros.  Likewise the row loads are predicated loads
  // that nothing reads until the shared-memory store.
  auto idx_ok = [&](int32_t v) -> bool { return v >= 0 && v < p.N; };
  // query tile of token `tok` (this CTA's 64 heads) into qs, completing on q_full
  auto load_q = [&](int64_t tok) {
    mbar_expect_tx(&sh->q_full, (uint32_t)nkb * 8192u);
    const int32_t qrow = (int32_t)(tok * p.H + cta * 64);
    for (int d = 0; d < nkb; ++d) tma_load_2d(&qmap, &sh->q_full, qs + d * 8192, d * 64, qrow);
  };

  // Ring position n -> chunk: S(0) first, then per period p = 1..nblk the
  // chunks S(p) (p < nblk) followed by V(p - 1).  is_v: V chunk; blk: its block;
  // sub: dims chunk (QK) or 32-key chunk (V).
  const uint32_t period = (uint32_t)(nkb + SA_NKC);
  const uint32_t n_total = (uint32_t)p.nblk * period;  // ring positions per token
  const uint32_t n_all = (uint32_t)n_it * n_total;       // ... of all this cluster's tokens
  auto decode = [&](uint32_t n, bool& is_v, int& blk, int& sub) {
    if (n < (uint32_t)nkb) {
      is_v = false; blk = 0; sub = (int)n;
      return;
    }
    const uint32_t m = n - nkb;
    const int pp = 1 + (int)(m / period), r = (int)(m % period);
    if (pp < p.nblk && r < nkb) {
      is_v = false; blk = pp; sub = r;
    } else {
      is_v = true; blk = pp - 1; sub = pp < p.nblk ? r - nkb : r;
    }
  };

  if (warp < 8 || warp == 10 || warp == 11) {
    // ------------------------------------------------------------ gathers
    // Group g (warps 2g, 2g + 1) fills ring positions g, g + 5, ...  Thread u of
    // the group moves 16-byte piece c = u % 8 of keys rg + 8 i, rg = u / 8:
    //   QK chunk: i < 16 (the CTA's 128 keys of the block), dims 64 sub + 8 c;
    //   V chunk:  i < 4 (keys 32 sub + ..), each of the CTA's n_pvblk V segments.
    // Row r = rg + 8 i lands at r * 128 + 16 (c ^ rg) of its 1024-byte swizzle
    // atom.  The raw indices of the group's next chunk are fetched with the
    // current chunk's loads; the round's fence has waited for them by the time
    // they are used.
    const int g = warp < 8 ? warp >> 1 : 4;
    const int u = ((warp & 1) << 5) | lane;
    const int c = u & 7, rg = u >> 3;
    const uint32_t swz = (uint32_t)((c ^ rg) << 4);
    int colv[4];
    bool colin[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      colv[s] = s < p.n_pvblk ? p.dv_begin + p.pv_col[cta][s] + 8 * c : 0;
      colin[s] = s < p.n_pvblk && colv[s] < p.D;
    }
    // This group's chunks are ring positions ng = g, g + 5, ... of the cluster's
    // token sequence; (it, n) = (token iteration, position in that token) is
    // advanced alongside, without a division (n_total >= 9 > SA_GROUPS, so a
    // step crosses at most one token boundary).
    auto step = [&](uint32_t& n, int& it) {
      n += SA_GROUPS;
      if (n >= n_total) {
        n -= n_total;
        ++it;
      }
    };
    int32_t nidx[16];
    int ip_it = -1;  // token iteration ip belongs to
    const int32_t* ip = p.idx;
    // raw indices of chunk (it, n), fetched one round ahead of its loads
    auto fetch = [&](uint32_t n, int it) {
      if (it != ip_it) {
        ip_it = it;
        ip = p.idx + (cid + (int64_t)it * ncl) * p.K;
      }
      bool is_v;
      int blk, sub;
      decode(n, is_v, blk, sub);
      if (!is_v) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = blk * SA_NB + (int)cta * SA_HALF + rg + 8 * i;
          nidx[i] = ldg_s32_or(ip + key, key < p.K, -1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = blk * SA_NB + sub * SA_KC + rg + 8 * i;
          nidx[i] = ldg_s32_or(ip + key, key < p.K, -1);
        }
      }
    };
    uint32_t nc = (uint32_t)g, nf = (uint32_t)g;  // this chunk, the next fetch
    int ic = 0, ifc = 0;
    if ((uint32_t)g < n_all) fetch(nf, ifc);
    step(nf, ifc);
    int kv_it = -1;  // token iteration kvb belongs to
    const uint16_t* kvb = p.kv;
    bool ok = true;
    for (uint32_t ng = (uint32_t)g; ok && ng < n_all; ng += SA_GROUPS) {
      if (ic != kv_it) {
        kv_it = ic;
        kvb = p.kv + (int64_t)((int)(cid + (int64_t)ic * ncl) / p.M) * p.N * p.D;  // token < 2^31
      }
      bool is_v;
      int blk, sub;
      decode(nc, is_v, blk, sub);
      uint4 v[16];
      if (!is_v) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          v[i] = ldcg_or_zero(kvb + (int64_t)nidx[i] * p.D + 64 * sub + 8 * c, idx_ok(nidx[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool rok = idx_ok(nidx[i]);
          const uint16_t* row = kvb + (int64_t)nidx[i] * p.D;
#pragma unroll
          for (int s = 0; s < 4; ++s) v[4 * i + s] = ldcg_or_zero(row + colv[s], colin[s] && rok);
        }
      }
      step(nc, ic);
      if (ng + SA_GROUPS < n_all) fetch(nf, ifc);
      step(nf, ifc);
      // n_slots is a multiple of SA_GROUPS, so this group alone fills this slot
      // and its parity wait is never two phases ahead of the barrier.
      const int slot = (int)(ng % (uint32_t)p.n_slots);
      wc.tag = (int)ng;
      if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->empty[slot], ((ng / p.n_slots) & 1) ^ 1, wc))))
        break;
      if (u == 0) KS_SA_TRACE(g, ng / SA_GROUPS);
      uint8_t* dst = smem + p.r_off + slot * SA_SLOT;
      if (!is_v) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          *reinterpret_cast<uint4*>(dst + (rg + 8 * i) * 128 + swz) = v[i];
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int s = 0; s < 4; ++s)
            if (s < p.n_pvblk)
              *reinterpret_cast<uint4*>(dst + s * SA_VSEG + (rg + 8 * i) * 128 + swz) = v[4 * i + s];
      }
      sa_warp_ready(is_v ? &sh->full_v[slot] : &sh->full_s[slot], cta, lane);
      if (u == 0) KS_SA_TRACE(4 + g, ng / SA_GROUPS);
    }
    if (threadIdx.x == 0) {
      // Tail: the tensor cores signal "slot consumed" asynchronously, also into
      // this CTA from the leader's commits.  Wait until the last signal of every
      // slot has landed, so none can reach the barriers of the next CTA that
      // this SM runs.
      // (Skipped after an abort: the waits would only run out their budgets.)
      for (int sl = 0; sl < p.n_slots && !*wc.abort; ++sl) {
        const uint32_t uses = (n_all + (uint32_t)(p.n_slots - 1 - sl)) / (uint32_t)p.n_slots;
        if (uses > 0) mbar_wait(&sh->empty[sl], (uses - 1) & 1, wc, false, true);
      }
    }
  } else if (warp == SA_MMA_WARP || warp == SA_MMA_WARP + 1) {
    int q_loads = 0;  // query tile loads issued (lane 0 of warp 8)
    if (warp == SA_MMA_WARP && lane == 0) {
      tma_prefetch_desc(&qmap);
      load_q(cid);  // the first token's query tile (this CTA's heads)
      q_loads = 1;
    }
    __syncwarp();
    if (cta == 0) {
      // ---------------------------------------------------------- MMA issuers (leader CTA)
      // Two warps: warp 8 issues the QK chunks, warp 9 the V chunks, each in
      // ring order.  One issuing thread alone keeps the tensor cores about half
      // busy (its barrier waits and commits cannot overlap its own MMAs); two
      // interleave.  Each stream has its own "full" barrier per slot, so a barrier
      // phase is never awaited while an earlier phase of the other stream in that
      // slot is still open.  The whole warp runs the loop: every lane waits on the
      // same barrier phase and computes the same (warp-uniform) descriptors, and
      // one elected lane (always the same one: the commits track the MMAs of the
      // thread that issued them) issues the MMAs and commits.  The waits are
      // compiled in (a call here costs more than the four MMAs of a chunk) and
      // CTA-scoped: the data they publish is read by the tensor cores, not by
      // this warp.
      const bool v_issuer = warp != SA_MMA_WARP;
      const bool leader = elect_one();
      bool ok = true;
      // Descriptors are built once; a byte offset o moves the start address field by o / 16.
      const uint64_t rd0 = sdesc_sw128(smem_u32(smem + p.r_off), v_issuer ? SA_VSEG : 16, 1024);
      uint32_t ph = 0;  // bit k: parity of the next phase of slot k's full barrier for this stream
      // Ring position (rn) and slot (rs = rn mod n_slots) of this stream's next
      // chunk, advanced incrementally: the per-chunk work is a short dependent
      // chain, so it carries no division.  Per token the ring order is S(0) |
      // S(1) V(0) | S(2) V(1) | ... | V(nblk-1): the QK stream starts at the
      // token's first position and skips V(j-2) before S(j), j >= 2, and the last
      // two V blocks after S(nblk-1); the V stream starts after S(1) and skips
      // S(j+2) after V(j), and the next token's S(0) S(1) after V(nblk-1).
      const int ns = p.n_slots;
      const int s01 = nkb + (p.nblk > 1 ? nkb : 0);  // S(0) S(1)
      uint32_t rn = v_issuer ? (uint32_t)s01 : 0u;
      int rs = (int)(rn % (uint32_t)ns);
      auto adv = [&](int k) {  // k <= 2 nkb: a few subtractions, no division
        rn += (uint32_t)k;
        rs += k;
        while (rs >= ns) rs -= ns;
      };
      uint64_t* const fulls = v_issuer ? sh->full_v : sh->full_s;
      // One chunk at a time: its MMAs go out as soon as it has landed, so its slot
      // is released without waiting for the next chunk (the kernel is bound by how
      // fast slots turn over; taking chunks in pairs held each first chunk back).
      auto take1 = [&](uint32_t n, int s0) -> bool {
        wc.tag = (int)n;
        const uint32_t q0 = (ph >> s0) & 1u;
        bool r0 = mbar_poll(smem_u32(&fulls[s0]), q0);
        if (!r0) r0 = mbar_wait_inl(&fulls[s0], q0, wc);
        r0 = __all_sync(0xFFFFFFFFu, r0);
        ph ^= 1u << s0;
        tc_fence_after();
        return r0;
      };
      if (!v_issuer) {
        const uint64_t qd0 = sdesc_sw128(smem_u32(qs), 16, 1024);
        const uint32_t qlo = (uint32_t)qd0, qhi = (uint32_t)(qd0 >> 32);
        const uint32_t rlo = (uint32_t)rd0, rhi = (uint32_t)(rd0 >> 32);
        const uint32_t idesc_s = idesc_bf16_f32(128, SA_NB, false, false);
        for (int it = 0; ok && it < n_it; ++it) {
          // both CTAs' query tiles of this token have landed
          wc.tag = 4000 + it;
          if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->q_full, it & 1, wc) &&
                                                  mbar_wait(&sh->peer_q, it & 1, wc, true))))
            break;
          tc_fence_after();
          for (int j = 0; ok && j < p.nblk; ++j) {
            const int jg = it * p.nblk + j;  // global block index
            // S buffer jg % 2 was last read by softmax(jg - 2)
            wc.tag = 2000 + j;
            if (jg >= 2 && !(ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->s_free[jg & 1], ((jg - 2) >> 1) & 1, wc)))) break;
            const uint32_t d_s = tmem + (jg & 1) * SA_SCOLS;
            if (j >= 2) adv(SA_NKC);
            for (int d = 0; d < nkb; ++d) {
              const uint32_t n = rn;
              const int slh = rs;
              if (!(ok = take1(n, slh))) break;
              adv(1);
              const uint32_t blo = rlo + (uint32_t)(slh * (SA_SLOT >> 4));
              const uint32_t alo = qlo + (uint32_t)(d * 512);
              if (leader) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  umma_cg2_w(d_s, alo + kk * 2, qhi, blo + kk * 2, rhi, idesc_s, (d > 0 || kk > 0) ? 1u : 0u);
                umma_commit_cg2(&sh->empty[slh], 3);
              }
              __syncwarp();
              KS_SA_TRACE(12, n);
            }
            if (!ok) break;
            if (leader) umma_commit_cg2(&sh->acc_full[jg & 1], 3);
            __syncwarp();
          }
          if (!ok) break;
          adv(p.nblk >= 2 ? 2 * SA_NKC : SA_NKC);  // to the next token's S(0)
          if (it + 1 < n_it) {
            // the query tiles are free once this token's QK MMAs have completed;
            // both CTAs then load the next token's
            if (leader) umma_commit_cg2(&sh->q_free, 3);
            __syncwarp();
            if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->q_free, it & 1, wc)))) break;
            if (lane == 0) {
              load_q(cid + (int64_t)(it + 1) * ncl);
              ++q_loads;
            }
            __syncwarp();
          }
        }
        if (leader) umma_commit_cg2(&sh->drain_s, 1);
        __syncwarp();
        mbar_wait(&sh->drain_s, 0, wc, false, true);
      } else {
        const uint64_t pd0 = sdesc_sw128(smem_u32(ps), 16, 1024);
        const uint32_t plo = (uint32_t)pd0, phi = (uint32_t)(pd0 >> 32);
        const uint32_t rlo = (uint32_t)rd0, rhi = (uint32_t)(rd0 >> 32);
        // (scalars, not arrays: an array indexed in a loop would live in local memory)
        const uint32_t idesc_pv0 = idesc_bf16_f32(128, p.pv_n[0], false, true);
        const uint32_t idesc_pv1 = idesc_bf16_f32(128, p.n_pv > 1 ? p.pv_n[1] : 128, false, true);
        const int npv = p.n_pv, pvn0 = p.pv_n[0];
        for (int it = 0; ok && it < n_it; ++it) {
          for (int j = 0; ok && j < p.nblk; ++j) {
            const int jg = it * p.nblk + j;
            // P(jg) written (and O rescaled) by the softmax; for a token's first
            // block also the previous token's O read out by the epilogue
            wc.tag = 1000 + j;
            if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->p_full[jg & 1], (jg >> 1) & 1, wc)))) break;
            KS_SA_TRACE(8, j);
            for (int sp = 0; sp < SA_NKC; sp += 2) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int sub = sp + h;
                const uint32_t n = rn;
                const int slh = rs;
                if (!(ok = take1(n, slh))) break;
                adv(1);
                const uint32_t boff = (uint32_t)(slh * (SA_SLOT >> 4));
                const uint32_t alo = plo + (uint32_t)((jg & 1) * (SA_PBYTES >> 4) + (sub >> 1) * 512 + (sub & 1) * 4);
                if (leader) {
#pragma unroll
                  for (int i = 0; i < 2; ++i) {
                    if (i == 1 && npv < 2) break;
                    // instruction i: N = pv_n[i]; its columns start at segment 2 i (pv_n[0] = 256 when there are two)
                    const uint32_t ocol = tmem + SA_OCOL + (i ? pvn0 / 2 : 0);
                    const uint32_t blo = rlo + boff + (uint32_t)(i ? (pvn0 / 128) * (SA_VSEG >> 4) : 0);
#pragma unroll
                    for (int kk = 0; kk < SA_KC / 16; ++kk)
                      umma_cg2_w(ocol, alo + kk * 2, phi, blo + kk * 128, rhi, i ? idesc_pv1 : idesc_pv0,
                                 (j > 0 || sub > 0 || kk > 0) ? 1u : 0u);
                  }
                  umma_commit_cg2(&sh->empty[slh], 3);
                }
                __syncwarp();
                KS_SA_TRACE(12, n);
              }
              if (!ok) break;
            }
            if (!ok) break;
            if (leader) umma_commit_cg2(&sh->p_free[jg & 1], 3);
            __syncwarp();
            if (j + 2 < p.nblk) adv(nkb);
          }
          if (!ok) break;
          if (leader) umma_commit_cg2(&sh->o_full, 3);
          __syncwarp();
          adv(s01);  // past the next token's S(0) S(1)
        }
        if (leader) umma_commit_cg2(&sh->drain_v, 1);
        __syncwarp();
        mbar_wait(&sh->drain_v, 0, wc, false, true);
      }
    } else if (lane == 0 && warp == SA_MMA_WARP) {
      // CTA 1: tell the leader that this CTA's query tile has landed; reload it
      // for the next token once the leader's QK MMAs are done with it
      for (int it = 0; it < n_it; ++it) {
        wc.tag = 4000 + it;
        if (!mbar_wait(&sh->q_full, it & 1, wc)) break;
        mbar_arrive_cluster(&sh->peer_q, 0);
        if (it + 1 == n_it) break;
        if (!mbar_wait(&sh->q_free, it & 1, wc)) break;
        load_q(cid + (int64_t)(it + 1) * ncl);
        ++q_loads;
      }
    }
    // every query tile load issued has landed before the CTA exits
    if (warp == SA_MMA_WARP && lane == 0) mbar_wait(&sh->q_full, (q_loads - 1) & 1, wc, false, true);
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
    const int32_t* ip = p.idx;  // the current token's index row
    bool oob = false;  // an index >= N was seen (reported once per token, after its last block)
    // validity bits of this lane's 128 keys of block j (warp-uniform loads).  An
    // index >= N (which the reference's gather rejects) is masked like -1 and, in
    // CTA 0, reported as a bounds error; negative indices are masked silently.
    auto valid_bits = [&](int j, uint32_t* mk) {
      const int k0 = j * SA_NB + half * SA_HALF;
      // (0 <= v < N as one unsigned compare; v >= N as the OR of the signed ones)
      const uint32_t un = (uint32_t)p.N;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t bits = 0;
        const int kw = k0 + 32 * w;
        if (p.idx_vec4 && kw + 32 <= p.K) {
          const int4* v4 = reinterpret_cast<const int4*>(ip + kw);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int4 v = __ldg(v4 + q);
            bits |= (uint32_t)((uint32_t)v.x < un) << (4 * q);
            bits |= (uint32_t)((uint32_t)v.y < un) << (4 * q + 1);
            bits |= (uint32_t)((uint32_t)v.z < un) << (4 * q + 2);
            bits |= (uint32_t)((uint32_t)v.w < un) << (4 * q + 3);
            oob |= (v.x >= p.N) | (v.y >= p.N) | (v.z >= p.N) | (v.w >= p.N);
          }
        } else {
          for (int i = 0; i < 32; ++i) {
            const int k = kw + i;
            const int32_t v = k < p.K ? __ldg(ip + k) : -1;
            bits |= (uint32_t)((uint32_t)v < un) << i;
            oob |= v >= p.N;
          }
        }
        mk[w] = bits;
      }
    };
    bool ok = true;
    for (int it = 0; ok && it < n_it; ++it) {
    const int64_t token = cid + (int64_t)it * ncl;
    ip = p.idx + token * p.K;
    m_used = sink2;
    lsum = 0.f;
    oob = false;
    for (int j = 0; j < p.nblk; ++j) {
      const int jg = it * p.nblk + j;  // global block index (barrier phases, S and P buffers)
      const int sb = jg & 1;
      uint32_t mk[4];
      valid_bits(j, mk);
      wc.tag = 3000 + j;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->acc_full[sb], (jg >> 1) & 1, wc));
      if (!ok) break;
      tc_fence_after();
      if (l == 0) KS_SA_TRACE(9, j);
      const uint32_t sbase = lane_base + sb * SA_SCOLS;
      // pass 1: block max over this lane's 128 keys of s * scale, taken over the raw
      // scores s * sign(scale) and scaled once (rounding is monotonic)
      const float sgn = p.scale_log2 < 0.f ? -1.f : 1.f;
      float bmax = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t r[32];
        tmem_ld32(sbase + 32 * w, r);
        tmem_wait_ld();
        float m0 = -INFINITY, m1 = -INFINITY;
        if (mk[w] == 0xFFFFFFFFu) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            m0 = fmaxf(m0, sgn * __uint_as_float(r[i]));
            m1 = fmaxf(m1, sgn * __uint_as_float(r[i + 1]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            m0 = fmaxf(m0, ((mk[w] >> i) & 1u) ? sgn * __uint_as_float(r[i]) : -INFINITY);
            m1 = fmaxf(m1, ((mk[w] >> (i + 1)) & 1u) ? sgn * __uint_as_float(r[i + 1]) : -INFINITY);
          }
        }
        bmax = fmaxf(bmax, fmaxf(m0, m1));
      }
      bmax = (sgn * bmax) * p.scale_log2;  // -inf when no key is valid
      // block max of the head = max over this lane and its partner (lane l ^ 64)
      sh->xslot[sb][l] = bmax;
      mbar_arrive(&sh->xchg[sb]);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->xchg[sb], (jg >> 1) & 1, wc));
      if (!ok) break;
      const float m_new = fmaxf(m_used, fmaxf(bmax, sh->xslot[sb][l ^ 64]));
      const bool resc = m_new > m_used + 8.f;
      float alpha = 1.f;
      if (resc) {
        alpha = ex2f(m_used - m_new);
        lsum *= alpha;
        m_used = m_new;
      }
      // P is double buffered: P(jg) goes to buffer jg % 2, last read by PV(jg - 2)
      if (jg >= 2) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->p_free[sb], ((jg - 2) >> 1) & 1, wc));
        if (!ok) break;
      }
      // (a token's first PV overwrites O, so O holds nothing to rescale at j = 0)
      if (j >= 1 && __any_sync(0xFFFFFFFFu, resc)) {  // TMEM access is warp-wide; alpha = 1 elsewhere
        // O is rescaled once PV(jg - 1) has finished with it
        ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&sh->p_free[(jg - 1) & 1], ((jg - 1) >> 1) & 1, wc));
        if (!ok) break;
        {
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
      if (l == 0) KS_SA_TRACE(10, j);
      // pass 2: probabilities as bf16, straight into P row m, keys [128*half, +128)
      // (64-key blocks 2*half and 2*half + 1; 16 keys = two 16-byte chunks per step):
      // p = 2^(s * scale_log2 - m), one FFMA and one ex2 per score; masked keys -> 0.
      {
        const float neg_m = -m_used;
        float ls0 = 0.f, ls1 = 0.f;
        uint8_t* pbase = ps + sb * SA_PBYTES + (2 * half) * 8192 + m * 128;
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          uint32_t r[16];
          tmem_ld16(sbase + 16 * c16, r);
          tmem_wait_ld();
          const uint32_t bits = (mk[c16 >> 1] >> ((c16 & 1) * 16)) & 0xFFFFu;
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float e0 = ex2f(fmaf(__uint_as_float(r[2 * i]), p.scale_log2, neg_m));
            float e1 = ex2f(fmaf(__uint_as_float(r[2 * i + 1]), p.scale_log2, neg_m));
            if (bits != 0xFFFFu) {
              e0 = ((bits >> (2 * i)) & 1u) ? e0 : 0.f;
              e1 = ((bits >> (2 * i + 1)) & 1u) ? e1 : 0.f;
            }
            ls0 += e0;
            ls1 += e1;
            pk[i] = cvt_bf16x2(e0, e1);
          }
          // keys 16 c16 .. +16 of this half: 64-key block c16 / 4, 16-byte chunks 2 (c16 % 4) + {0, 1}
          uint8_t* prow = pbase + (c16 >> 2) * 8192;
          const int cc = (c16 & 3) * 2;
          *reinterpret_cast<uint4*>(prow + ((cc ^ (m & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(prow + (((cc + 1) ^ (m & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        lsum += ls0 + ls1;
      }
      tc_fence_before();
      sa_warp_ready(&sh->p_full[sb], cta, lane);
      if (lane == 0) {  // S buffer sb read out
        if (cta == 0) mbar_arrive(&sh->s_free[sb]);
        else mbar_arrive_cluster(&sh->s_free[sb], 0);
      }
      if (lane == 0) KS_SA_TRACE(11, 16 * q4 + j);
    }
    if (cta == 0 && __any_sync(0xFFFFFFFFu, oob) && oob) report_bounds(p.status, (int)token, p.N);
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->o_full, it & 1, wc));
    if (ok) {
      sh->xslot[2][l] = lsum;
      mbar_arrive(&sh->xchg[2]);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sh->xchg[2], it & 1, wc));
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
            if (p.out_v8) {  // one whole 32-byte sector per store
              asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(orow + d0 + c),
                           "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]),
                           "r"(w[7])
                           : "memory");
            } else {
              uint4* dst = reinterpret_cast<uint4*>(orow + d0 + c);
              dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
              dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            }
          }
        }
        ocol += hn;
      }
    }
    }  // tokens
    // tail: the last two "P free" signals land before the CTA exits (see the gathers)
    const int jtot = n_it * p.nblk;
    for (int jj = jtot - 2; ok && jj < jtot; ++jj)
      if (jj >= 0) mbar_wait(&sh->p_free[jj & 1], (jj >> 1) & 1, wc, false, true);
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == SA_MMA_WARP) tmem_dealloc<2>(tmem, 512);
}

}  // namespace ks
