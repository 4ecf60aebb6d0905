// The indexer's projections on tcgen05 with their follow-up arithmetic fused into
// the epilogue: the producer of the score kernel's inputs.
//
// Semantics follow baseline/indexer.py:170-175 (+ RoPE, :114-129,172):
//   y[m, n] = bf16( sum_k a[m, k] * w[n, k] )          F.linear, bf16 in, fp32 accumulate
//   rope:  the last `rd` of every `hd` columns are rotated as interleaved pairs
//          with freqs[m % S] (fp32 products and sums rounded separately, result
//          rounded to bf16), as apply_rotary_emb does to q[..., -rd:]
//   scale: y = bf16( float(y) * scale ), as weights_proj(x) * (D^-0.5 H^-0.5)
// so q = wq_b(qr) leaves this kernel already rotated (the score kernel then runs
// without RoPE) and the head weights leave it scaled.  Fusing the projection into
// the score kernel itself would make every 4-token work item stream all of w
// (16 MB for 64 heads x 128 dims x 1024) from L2; as its producer the GEMM reads
// each operand tile once per output tile.
//
// Persistent CTAs (one per SM; two for tiles at most 64 columns wide), 10 warps: warp 0 TMA producer (A tile 128 x 64 and
// B tile N_TILE x 64 per stage, 128-byte swizzle), warp 1 TMEM owner and MMA
// issuer (M = 128, N = N_TILE, K = 16 per instruction, fp32 accumulators double
// buffered in TMEM), warps 2-9 epilogue: thread = output row = TMEM lane, two
// warps per lane quarter splitting the tile's columns when the tile is wide
// enough (with one warp per scheduler, each TMEM load latency went unhidden).
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int PG_THREADS = 320;
constexpr int PG_THREADS_NARROW = 192;
constexpr int PG_EPI_WARP0 = 2;
constexpr int PG_EPI_WARPS = 8;
constexpr int PG_TILE_M = 128;
constexpr int PG_MAX_STAGES = 8;

struct ProjParams {
  uint16_t* out;        // bf16 [M, N]
  const float* freqs;   // [S, rd/2, 2] (cos, sin), row m uses freqs[m % S]
  int32_t M, N, K, S;
  int32_t n_tile;       // 16..256, multiple of 16, divides N
  int32_t hd, rd;       // head dim and rotated dims (rd = 0: no RoPE)
  float scale;          // applied after the bf16 rounding when apply_scale
  int32_t apply_scale;
  int32_t stages;
  int32_t tiles_m, tiles_n;
  uint32_t fr_off;      // shared-memory offset of the per-row RoPE factors (rd > 0)
  uint32_t st_off;      // shared-memory offset of the output staging boxes (tma_store)
  int32_t tma_store;    // write the output through TMA stores (n_tile >= 64)
  uint32_t acc_cols;    // TMEM columns per accumulator buffer (two buffers)
  uint32_t tmem_cols;   // TMEM columns allocated (2 acc_cols, a power of two >= 32)
  int* status;
  uint64_t budget_ns;
};

struct PgShared {
  uint64_t full[PG_MAX_STAGES], empty[PG_MAX_STAGES];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint64_t fr_full[4], fr_free[4];  // RoPE factor hand-over between the two warps of a quarter
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(PgShared) <= 1024, "PgShared exceeds its header");

// THREADS = PG_THREADS (one CTA per SM) or PG_THREADS_NARROW (tiles at most 64
// columns wide: four epilogue warps, two CTAs per SM within the register file)
template <int THREADS, int MIN_BLOCKS>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap amap,
                     const __grid_constant__ CUtensorMap bmap,
                     const __grid_constant__ CUtensorMap omap, ProjParams p) {
  extern __shared__ uint8_t pg_raw[];
  const uint32_t raw_addr = smem_u32(pg_raw);
  uint8_t* smem = pg_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  PgShared* sh = reinterpret_cast<PgShared*>(smem);
  const uint32_t a_bytes = PG_TILE_M * 128, b_bytes = (uint32_t)p.n_tile * 128;
  const uint32_t st_bytes = a_bytes + b_bytes;
  uint8_t* stage0 = smem + 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_k = (p.K + 63) / 64;
  const int n_tiles = p.tiles_m * p.tiles_n;
  WaitCtx wc{&sh->abort, p.status, p.budget_ns};
  // two epilogue warps per lane quarter, each converting half the tile's columns,
  // when a half is a whole number of 64-column store boxes (of 32-column steps
  // without TMA stores); otherwise warps 6-9 stay idle
  const bool split = p.tma_store ? p.n_tile >= 128 : p.n_tile >= 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->acc_full[i], 1);
      mbar_init(&sh->acc_empty[i], split ? PG_EPI_WARPS : 4);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&sh->fr_full[i], 32);
      mbar_init(&sh->fr_free[i], 32);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(&sh->tmem_base, p.tmem_cols);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      uint32_t c = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
        for (int kc = 0; kc < n_k; ++kc, ++c) {
          const int st = (int)(c % (uint32_t)p.stages);
          if (!(ok = mbar_wait(&sh->empty[st], ((c / p.stages) & 1) ^ 1, wc))) break;
          uint8_t* sa = stage0 + st * st_bytes;
          mbar_expect_tx(&sh->full[st], st_bytes);
          tma_load_2d(&amap, &sh->full[st], sa, kc * 64, tm * PG_TILE_M);
          tma_load_2d(&bmap, &sh->full[st], sa + a_bytes, kc * 64, tn * p.n_tile);
        }
      }
      // drain: every load issued has landed before the CTA exits
      for (uint32_t i = (c > (uint32_t)p.stages ? c - p.stages : 0); i < c; ++i)
        mbar_wait(&sh->full[i % p.stages], (i / p.stages) & 1, wc, false, true);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(PG_TILE_M, p.n_tile, false, false);
      uint32_t c = 0, ac = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++ac) {
        const int as = ac & 1;
        if (!(ok = mbar_wait(&sh->acc_empty[as], ((ac >> 1) & 1) ^ 1, wc))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + as * p.acc_cols;
        for (int kc = 0; kc < n_k; ++kc, ++c) {
          const int st = (int)(c % (uint32_t)p.stages);
          if (!(ok = mbar_wait_inl(&sh->full[st], (c / p.stages) & 1, wc))) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(stage0 + st * st_bytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(sa + a_bytes + kk * 32, 16, 1024);
            umma_bf16_ss(d_tmem, ad, bd, idesc, (kc | kk) ? 1u : 0u);
          }
          umma_commit(&sh->empty[st]);
        }
        if (!ok) break;
        umma_commit(&sh->acc_full[as]);
      }
      umma_commit(&sh->drain);
      mbar_wait(&sh->drain, 0, wc, false, true);
    }
  } else if (split || warp < PG_EPI_WARP0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, +32)
    const int row_in_tile = quarter * 32 + lane;
    const int ehalf = (warp - PG_EPI_WARP0) >> 2;
    const int c_begin = split ? ehalf * (p.n_tile / 2) : 0;
    const int c_end = split ? c_begin + p.n_tile / 2 : p.n_tile;
    const int rope0 = p.hd - p.rd;  // first rotated column of a head
    // this thread's row of RoPE factors (cos, sin pairs), staged once per tile by
    // the quarter's first warp: a load per rotated pair from global memory would
    // put one memory latency on every step.  Row stride rd + 2 words: a warp's
    // 8-byte reads of one pair index fall on distinct banks within each half-warp.
    // The second warp reads the same rows; fr_full / fr_free hand them over so
    // that the first warp never overwrites factors the second still reads.
    float* my_fr = reinterpret_cast<float*>(smem + p.fr_off) + row_in_tile * (p.rd + 2);
    // output staging (32 KB): 32-row x 64-column boxes (128-byte rows, swizzled like
    // the tensor map) written out by TMA stores, one per warp when split, else two
    // per warp so that one fills while the other is stored
    const int n_box = split ? 1 : 2;
    uint8_t* stage = smem + p.st_off + (split ? (warp - PG_EPI_WARP0) * 4096 : quarter * 8192);
    uint32_t nbox = 0;
    uint32_t ac = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++ac) {
      const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
      const int as = ac & 1;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sh->acc_full[as], (ac >> 1) & 1, wc))) break;
      tc_fence_after();
      const int m = tm * PG_TILE_M + row_in_tile;
      const bool row_ok = m < p.M;
      if (p.rd > 0) {
        if (ehalf == 0) {
          if (split && ac > 0 &&
              !__all_sync(0xFFFFFFFFu, mbar_wait(&sh->fr_free[quarter], (ac - 1) & 1, wc)))
            break;
          const float2* fr = reinterpret_cast<const float2*>(p.freqs + (int64_t)(row_ok ? m % p.S : 0) * p.rd);
          float2 f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < p.rd / 2) f[j] = __ldg(fr + j);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < p.rd / 2) reinterpret_cast<float2*>(my_fr)[j] = f[j];
          if (split) mbar_arrive(&sh->fr_full[quarter]);
        } else if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sh->fr_full[quarter], ac & 1, wc))) {
          break;
        }
      }
      uint16_t* orow = p.out + (int64_t)m * p.N + (int64_t)tn * p.n_tile;
      const uint32_t tbase = tmem + as * p.acc_cols + ((uint32_t)(quarter * 32) << 16);
      uint8_t* box = stage;
      // 32 columns per TMEM load where the range allows, one wait per load
      for (int c0 = c_begin; c0 < c_end; c0 += 32) {
        const int nsub = c0 + 16 < c_end ? 2 : 1;
        uint32_t r[32];
        if (nsub == 2) tmem_ld32(tbase + c0, r);
        else tmem_ld16(tbase + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h >= nsub) break;
          const int c = c0 + 16 * h;
          if (p.tma_store && (c & 63) == 0) {
            // the box this 64-column group fills was last stored n_box groups ago
            box = stage + (nbox % n_box) * 4096;
            if (lane == 0) {
              if (n_box == 1) bulk_wait_group_read<0>();
              else bulk_wait_group_read<1>();
            }
            __syncwarp();
          }
          uint32_t o[8];
          // head-local column of r[16 h]; a 16-column step never crosses a head (hd
          // and the tile's columns are multiples of 16), so it is wholly rotated or
          // not, unless rope0 falls inside it.  (Rows past M rotate with row 0's
          // factors; the TMA store clips them.)
          const int dc = tn * p.n_tile + c;
          const int d0 = (p.hd & (p.hd - 1)) == 0 ? dc & (p.hd - 1) : dc % p.hd;
          const bool all_rot = p.rd > 0 && d0 >= rope0;
          const bool some_rot = p.rd > 0 && d0 + 16 > rope0;
          auto rotate = [&](uint32_t v, int j) -> uint32_t {
            const float2 cs = reinterpret_cast<const float2*>(my_fr)[j];
            const float xr = bf16lo_f32(v), xi = bf16hi_f32(v);
            const float re = __fsub_rn(__fmul_rn(xr, cs.x), __fmul_rn(xi, cs.y));
            const float im = __fadd_rn(__fmul_rn(xr, cs.y), __fmul_rn(xi, cs.x));
            return cvt_bf16x2(re, im);
          };
#pragma unroll
          for (int i = 0; i < 8; ++i)  // bf16 rounding of the GEMM output (F.linear returns bf16)
            o[i] = cvt_bf16x2(__uint_as_float(r[16 * h + 2 * i]), __uint_as_float(r[16 * h + 2 * i + 1]));
          if (all_rot) {
            const int j0 = (d0 - rope0) >> 1;
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = rotate(o[i], j0 + i);
          } else if (some_rot) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (d0 + 2 * i >= rope0) o[i] = rotate(o[i], (d0 + 2 * i - rope0) >> 1);
          }
          if (p.apply_scale) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              o[i] = cvt_bf16x2(__fmul_rn(bf16lo_f32(o[i]), p.scale), __fmul_rn(bf16hi_f32(o[i]), p.scale));
          }
          if (p.tma_store) {
            // row `lane` of the box, 16-byte units 2 s and 2 s + 1 (s = the 16-column
            // step in the group), 128-byte swizzle: unit u at (u ^ (row % 8)) * 16
            const int s2 = ((c & 63) >> 4) * 2;
            uint8_t* brow = box + lane * 128;
            *reinterpret_cast<uint4*>(brow + (((s2) ^ (lane & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(brow + (((s2 + 1) ^ (lane & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            if ((c & 63) == 48) {  // box complete: one TMA store of 32 rows x 64 columns
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&omap, box, tn * p.n_tile + (c & ~63), tm * PG_TILE_M + quarter * 32);
                bulk_commit_group();
              }
              ++nbox;
            }
          } else if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
      tc_fence_before();
      if (p.rd > 0 && split && ehalf == 1) mbar_arrive(&sh->fr_free[quarter]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->acc_empty[as]);
    }
    if (lane == 0) bulk_wait_group<0>();  // stores done before the shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<1>(tmem, p.tmem_cols);
}

}  // namespace ks
