// Host side of libks_b200.so: argument validation, TMA descriptor encoding,
// launches and the device status word.  The extern "C" functions are declared in
// include/ks_b200.h.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "ks_b200.h"
#include "ks_device.cuh"
#include "indexer_score.cuh"
#include "proj_gemm.cuh"
#include "quant_fp8.cuh"
#include "sinkhorn.cuh"
#include "sparse_attn.cuh"
#include "sparse_attn_small.cuh"
#include "sparse_attn_tiny.cuh"
#include "topk.cuh"
#include "topk_small.cuh"

namespace ks {

// Per-device status written by kernels whose bounded waits ran out: [0] the code,
// [1], [2] where the first timeout happened (block; thread, barrier offset, parity).
__device__ int g_status_word[4];

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(KS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct Device {
  bool ready = false;
  int* status = nullptr;  // address of g_status_word on this device
  int num_sms = 0;
  // kernels whose dynamic shared-memory opt-in has been set on this device
  // (cudaFuncSetAttribute acts on the current device's context only)
  const void* smem_optin[64] = {};  // more than the library's kernel instances
  int n_smem_optin = 0;
  // co-resident CTA pairs of the persistent attention kernel, for the shared
  // memory size it was last asked for
  int sa_clusters = 0;
  size_t sa_clusters_smem = 0;
};
constexpr int kMaxDevices = 64;
std::mutex g_mu;
Device g_devices[kMaxDevices];

int device(Device** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(KS_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  Device& d = g_devices[dev];
  if (!d.ready) {
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_status_word);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    d.ready = true;
  }
  *out = &d;
  return KS_OK;
}

// Allow `func` the 227 KB shared-memory maximum on the device `d` describes (the
// current device), once per device and kernel.
int smem_optin(Device* d, const void* func, const char* what) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < d->n_smem_optin; ++i)
    if (d->smem_optin[i] == func) return KS_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
  if (e != cudaSuccess) return cuda_fail(e, what);
  // the table only saves repeating the call: when it is full the attribute is set anyway
  if (d->n_smem_optin < (int)(sizeof(d->smem_optin) / sizeof(d->smem_optin[0])))
    d->smem_optin[d->n_smem_optin++] = func;
  return KS_OK;
}

uint64_t wait_budget_ns() {
  static uint64_t budget = [] {
    const char* s = getenv("KS_WAIT_BUDGET_MS");
    long ms = s ? atol(s) : 2000;
    if (ms < 1) ms = 1;
    return (uint64_t)ms * 1000000ull;
  }();
  return budget;
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return KS_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 2D tensor map [rows, inner] with a row stride, 128-byte swizzle, box
// (box_inner x box_rows).  Rows beyond `rows` read as zero.
int make_map_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(KS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KS_OK;
}

// 8-bit 2D tensor map [rows, inner] (e4m3 bytes), 128-byte swizzle, box
// (box_inner x box_rows).
int make_map_u8(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(KS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KS_OK;
}

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// ------------------------------------------------------------------ indexer helpers
struct IndexerGeom {
  int tok, n_groups, n_items, kst;
  size_t smem;
};

int indexer_geom(int64_t B, int64_t S, int64_t H, int64_t D, bool f8, IndexerGeom* g) {
  g->tok = (int)(IX_N / H);
  g->n_groups = (int)((S + g->tok - 1) / g->tok);
  g->n_items = (int)(B * g->n_groups);
  const size_t esz = f8 ? 1 : 2;
  const size_t q_bytes = (size_t)IX_N * D * esz, k_bytes = (size_t)IX_TILE_KEYS * D * esz;
  const size_t fixed = 1024 /* alignment slack */ + 2 * q_bytes;
  const size_t limit = 232448;  // 227 KB opt-in maximum per CTA on sm_100
  const size_t hdr = f8 ? ix_hdr_bytes<true>() : ix_hdr_bytes<false>();  // IxShared, padded
  int kst = (int)((limit - fixed - hdr) / k_bytes);
  if (kst > (f8 ? 8 : 4)) kst = f8 ? 8 : 4;
  if (kst < 2) return fail(KS_ERR_UNSUPPORTED, "indexer: D=%lld leaves no room for key stages", (long long)D);
  g->kst = kst;
  g->smem = fixed + hdr + (size_t)kst * k_bytes;
  return KS_OK;
}

int indexer_check(const void* q, const void* k, const void* w, const float* freqs, int64_t B,
                  int64_t S, int64_t H, int64_t D, int64_t T, int32_t rope_dim, int32_t ratio,
                  int64_t k_batch_rows) {
  if (!q || !k || !w) return fail(KS_ERR_INVALID, "indexer: null input pointer");
  if (B < 1 || S < 1 || T < 0) return fail(KS_ERR_INVALID, "indexer: bad sizes B=%lld S=%lld T=%lld", (long long)B, (long long)S, (long long)T);
  if (!(H == 16 || H == 32 || H == 64)) return fail(KS_ERR_UNSUPPORTED, "indexer: H=%lld (supported: 16, 32, 64)", (long long)H);
  if (!(D == 64 || D == 128)) return fail(KS_ERR_UNSUPPORTED, "indexer: D=%lld (supported: 64, 128)", (long long)D);
  if (T > 65536) return fail(KS_ERR_UNSUPPORTED, "indexer: T=%lld > 65536", (long long)T);
  if (rope_dim < 0 || rope_dim > D || rope_dim % 8) return fail(KS_ERR_INVALID, "indexer: rope_dim=%d must be a multiple of 8 in [0, D]", rope_dim);
  if (rope_dim > 0 && !freqs) return fail(KS_ERR_INVALID, "indexer: freqs is null");
  if (ratio < 1) return fail(KS_ERR_INVALID, "indexer: ratio=%d", ratio);
  if (k_batch_rows < T) return fail(KS_ERR_INVALID, "indexer: k_batch_rows < T");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(w, 4) || (freqs && !aligned(freqs, 16)))
    return fail(KS_ERR_ALIGNMENT, "indexer: q, k, freqs must be 16-byte and w 4-byte aligned");
  if (B * S * H >= (1ll << 31) || B * k_batch_rows >= (1ll << 31))
    return fail(KS_ERR_UNSUPPORTED, "indexer: too many rows for 32-bit TMA coordinates");
  return KS_OK;
}

template <int H, bool F8>
int launch_indexer_scores(Device* dev, const CUtensorMap& qm, const CUtensorMap& km,
                          const IndexerScoreParams& p, const IndexerGeom& g, int grid,
                          cudaStream_t st) {
  if (int rc = smem_optin(dev, reinterpret_cast<const void*>(indexer_score_kernel<H, F8>),
                          "cudaFuncSetAttribute(indexer)"))
    return rc;
  indexer_score_kernel<H, F8><<<grid, IX_THREADS, g.smem, st>>>(qm, km, p);
  return launch_check("indexer_score_kernel launch");
}

// Score stage.  f8: q and k are e4m3 bytes, w is fp32 (head weight x query scale),
// k_scale fp32 per key row; else q, k, w are bf16 and k_scale is unused.
int indexer_scores_impl(const void* q, const void* k, int64_t k_batch_rows, const void* w,
                        const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D,
                        int64_t T, int32_t rope_dim, int64_t pos0, int32_t causal,
                        int32_t ratio, void* scores, int64_t score_ld, cudaStream_t st,
                        bool f8 = false, const float* k_scale = nullptr) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  IndexerGeom g;
  if (int rc = indexer_geom(B, S, H, D, f8, &g)) return rc;
  if (T == 0) return KS_OK;
  CUtensorMap qm, km;
  if (f8) {
    if (int rc = make_map_u8(&qm, q, D, (uint64_t)(B * S * H), D, 128, IX_N)) return rc;
    if (int rc = make_map_u8(&km, k, D, (uint64_t)(B * k_batch_rows), D, 128, IX_TILE_KEYS)) return rc;
  } else {
    if (int rc = make_map_bf16(&qm, q, D, (uint64_t)(B * S * H), D * 2, 64, IX_N)) return rc;
    if (int rc = make_map_bf16(&km, k, D, (uint64_t)(B * k_batch_rows), D * 2, 64, IX_TILE_KEYS)) return rc;
  }
  IndexerScoreParams p{};
  p.freqs = freqs;
  p.w = f8 ? nullptr : static_cast<const uint16_t*>(w);
  p.wf = f8 ? static_cast<const float*>(w) : nullptr;
  p.k_scale = k_scale;
  p.w_bs = S * H;
  p.w_vec16 = aligned(w, 16) ? 1 : 0;  // rows of H >= 16 elements are 16-byte multiples
  p.scores = static_cast<uint16_t*>(scores);
  p.score_ld = score_ld;
  p.B = (int)B; p.S = (int)S; p.H = (int)H; p.D = (int)D; p.T = (int)T; p.rd = rope_dim;
  p.k_rows_per_batch = k_batch_rows;
  p.pos0 = pos0;
  p.causal = causal ? 1 : 0;
  p.ratio = ratio;
  p.tok = g.tok; p.n_groups = g.n_groups; p.n_items = g.n_items; p.kst = g.kst;
  p.status = dev->status;
  p.budget_ns = wait_budget_ns();
  const int grid = g.n_items < dev->num_sms ? g.n_items : dev->num_sms;
  if (f8) {
    switch (H) {
      case 16: return launch_indexer_scores<16, true>(dev, qm, km, p, g, grid, st);
      case 32: return launch_indexer_scores<32, true>(dev, qm, km, p, g, grid, st);
      default: return launch_indexer_scores<64, true>(dev, qm, km, p, g, grid, st);
    }
  }
  switch (H) {
    case 16: return launch_indexer_scores<16, false>(dev, qm, km, p, g, grid, st);
    case 32: return launch_indexer_scores<32, false>(dev, qm, km, p, g, grid, st);
    default: return launch_indexer_scores<64, false>(dev, qm, km, p, g, grid, st);
  }
}

template <int EPT>
int launch_topk(Device* dev, const TopkParams& p, int64_t rows, size_t smem, cudaStream_t st) {
  if (int rc = smem_optin(dev, reinterpret_cast<const void*>(topk_rows_kernel<EPT>),
                          "cudaFuncSetAttribute(topk)"))
    return rc;
  topk_rows_kernel<EPT><<<(unsigned)rows, TK_THREADS, smem, st>>>(p);
  return launch_check("topk_rows_kernel launch");
}

int topk_impl(const void* scores, int64_t score_ld, int64_t B, int64_t S, int64_t T,
              int64_t pos0, int32_t causal, int32_t ratio, int32_t topk, int64_t offset,
              void* out, int32_t out_dtype, cudaStream_t st) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  if (!scores || !out) return fail(KS_ERR_INVALID, "topk: null pointer");
  if (B < 1 || S < 1 || T < 0 || topk < 0) return fail(KS_ERR_INVALID, "topk: bad sizes");
  if (T > 65536) return fail(KS_ERR_UNSUPPORTED, "topk: T=%lld > 65536", (long long)T);
  if (topk > 4096) return fail(KS_ERR_UNSUPPORTED, "topk: k=%d > 4096", topk);
  if (score_ld < T || score_ld % 8) return fail(KS_ERR_INVALID, "topk: score_ld must be >= T and a multiple of 8");
  if (!aligned(scores, 16)) return fail(KS_ERR_ALIGNMENT, "topk: scores must be 16-byte aligned");
  if (ratio < 1) return fail(KS_ERR_INVALID, "topk: ratio=%d", ratio);
  if (out_dtype != KS_INT32 && out_dtype != KS_INT64) return fail(KS_ERR_INVALID, "topk: out_dtype");
  const int K = (int)(topk < T ? topk : T);
  if (K == 0) return KS_OK;
  int kpow2 = 1;
  while (kpow2 < K) kpow2 <<= 1;
  TopkParams p{};
  p.scores = static_cast<const uint16_t*>(scores);
  p.row_stride = score_ld;
  p.rows = B * S;
  p.S = S;
  p.pos0 = pos0;
  p.causal = causal ? 1 : 0;
  p.ratio = ratio;
  p.T = (int)T;
  p.k = K;
  p.offset = offset;
  p.out = out;
  p.out_i64 = out_dtype == KS_INT64;
  p.out_row_stride = K;
  p.kpow2 = kpow2;
  p.status = dev->status;
  if (B * S > 0x7FFFFFFFll) return fail(KS_ERR_UNSUPPORTED, "topk: too many rows");
  // short rows and small k: one warp per row (topk_small.cuh)
  if (T <= TS_MAXT && kpow2 <= 256) {
    const int epl = kpow2 <= 32 ? 1 : kpow2 / 32;
    const size_t smem_s = (size_t)TS_WARPS * ((size_t)TS_MAXT * 2 + (size_t)32 * epl * 4);  // <= 40 KB
    const unsigned blocks = (unsigned)((B * S + TS_WARPS - 1) / TS_WARPS);
    switch (epl) {
      case 1: topk_small_kernel<1><<<blocks, TS_WARPS * 32, smem_s, st>>>(p); break;
      case 2: topk_small_kernel<2><<<blocks, TS_WARPS * 32, smem_s, st>>>(p); break;
      case 4: topk_small_kernel<4><<<blocks, TS_WARPS * 32, smem_s, st>>>(p); break;
      default: topk_small_kernel<8><<<blocks, TS_WARPS * 32, smem_s, st>>>(p); break;
    }
    return launch_check("topk_small_kernel launch");
  }
  // composites sorted per row: TK_THREADS * ept >= kpow2
  const int ept = kpow2 <= TK_THREADS ? 1 : kpow2 / TK_THREADS;
  const size_t nbuf = (size_t)TK_THREADS * ept > (size_t)TK_HBINS ? (size_t)TK_THREADS * ept : (size_t)TK_HBINS;
  // the staged keys, reused by the counting sort's per-warp counters
  const size_t key_bytes = std::max<size_t>((size_t)round_up(T, 8) * 2, (size_t)TK_WARPS * TK_CBINS * 2);
  const size_t smem = nbuf * 4 + (TK_WARPS + 4 + 8 + 2 * TK_WARPS) * 4 + key_bytes;
  switch (ept) {
    case 1: return launch_topk<1>(dev, p, B * S, smem, st);
    case 2: return launch_topk<2>(dev, p, B * S, smem, st);
    case 4: return launch_topk<4>(dev, p, B * S, smem, st);
    default: return launch_topk<8>(dev, p, B * S, smem, st);
  }
}

int sparse_attn_impl(const void* q, const void* kv, const float* sink, const int32_t* idx,
                     void* out, int64_t B, int64_t M, int64_t H, int64_t D, int64_t N, int64_t K,
                     int64_t dv_begin, int64_t dv, float scale, cudaStream_t st) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  if (!q || !kv || !sink || !idx || !out) return fail(KS_ERR_INVALID, "sparse_attn: null pointer");
  if (B < 1 || M < 0 || H < 1 || N < 1 || K < 1) return fail(KS_ERR_INVALID, "sparse_attn: bad sizes");
  if (H > 128) return fail(KS_ERR_UNSUPPORTED, "sparse_attn: H=%lld > 128", (long long)H);
  if (D % 64 || D < 64 || D > 576) return fail(KS_ERR_UNSUPPORTED, "sparse_attn: D=%lld (multiple of 64, <= 576)", (long long)D);
  if (dv < 64 || dv > 512 || dv % 64 || dv_begin < 0 || dv_begin % 64 || dv_begin + dv > D)
    return fail(KS_ERR_UNSUPPORTED, "sparse_attn: dv=%lld dv_begin=%lld (multiples of 64, dv <= 512, within D)", (long long)dv, (long long)dv_begin);
  if (!aligned(q, 16) || !aligned(kv, 16) || !aligned(out, 16) || !aligned(idx, 4) || !aligned(sink, 4))
    return fail(KS_ERR_ALIGNMENT, "sparse_attn: q, kv, out must be 16-byte aligned");
  if (B * M * H >= (1ll << 31) || B * N >= (1ll << 31) || 2 * B * M >= (1ll << 31))
    return fail(KS_ERR_UNSUPPORTED, "sparse_attn: too many rows");
  if (M == 0) return KS_OK;
  // Very short index rows: 128 / H tokens per 128-row tile, heads as the MMA's M
  // dimension (sparse_attn_tiny.cuh).
  if (H >= 16 && 128 % H == 0 && K <= SAT_MAX_K && D <= 256 && dv <= 256 && dv % 64 == 0) {
    const int tpt = (int)(128 / H);
    const int kp = (int)round_up(K, 16);
    const int ncol = tpt * kp;
    if (ncol <= SAT_MAX_N) {
      SaTinyParams tp{};
      tp.q = static_cast<const uint16_t*>(q);
      tp.idx = idx;
      tp.kv = static_cast<const uint16_t*>(kv);
      tp.sink = sink;
      tp.out = static_cast<uint16_t*>(out);
      tp.B = (int)B; tp.M = (int)M; tp.H = (int)H; tp.D = (int)D; tp.N = (int)N; tp.K = (int)K;
      tp.dv_begin = (int)dv_begin; tp.dv = (int)dv;
      tp.tpt = tpt; tp.kp = kp; tp.ncol = ncol;
      tp.inv_kp = 1.0f / (float)kp;
      tp.nkb = (int)(D / 64);
      const size_t kg_bytes = (size_t)tp.nkb * ncol * 128;          // a multiple of 1 KB
      const int q_chunks = std::max(tp.nkb, (ncol + 63) / 64);      // Q, then P
      tp.kg_off = SAT_HDR;
      tp.q_off = (uint32_t)(SAT_HDR + kg_bytes);
      int tcols = 32;
      while (tcols < std::max(ncol, (int)dv)) tcols <<= 1;
      tp.tmem_cols = (uint32_t)tcols;
      tp.scale_log2 = scale * 1.4426950408889634f;
      const size_t smem = 1024 + SAT_HDR + kg_bytes + (size_t)q_chunks * 16384;
      tp.status = dev->status;
      tp.budget_ns = wait_budget_ns();
      CUtensorMap qm;  // q as [B M H rows, D], boxes of 64 dims x 128 rows
      if (int rc = make_map_bf16(&qm, q, (uint64_t)D, (uint64_t)(B * M * H), (uint64_t)D * 2, 64, 128))
        return rc;
      CUtensorMap om;  // out as [B M H rows, dv], the same boxes
      if (int rc = make_map_bf16(&om, out, (uint64_t)dv, (uint64_t)(B * M * H), (uint64_t)dv * 2, 64, 128))
        return rc;
      if (int rc = smem_optin(dev, reinterpret_cast<const void*>(sparse_attn_tiny_kernel),
                              "cudaFuncSetAttribute(sparse_attn_tiny)"))
        return rc;
      const unsigned grid = (unsigned)((B * M + tpt - 1) / tpt);
      sparse_attn_tiny_kernel<<<grid, SAT_THREADS, smem, st>>>(qm, om, tp);
      return launch_check("sparse_attn_tiny_kernel launch");
    }
  }
  // Few heads and short index rows: one CTA per token, keys as the MMA's M
  // dimension (sparse_attn_small.cuh).
  {
    const int hn = H <= 16 ? 16 : H <= 32 ? 32 : H <= 64 ? 64 : 0;
    const int64_t k_pad = round_up(K, 128), nt = k_pad / 128;
    const int dv_tiles = (int)((dv + 127) / 128);
    const int nkb = (int)std::max<int64_t>(D / 64, dv_begin / 64 + 2 * dv_tiles);
    const size_t kg = (size_t)nt * nkb * 16384, qb = (size_t)nkb * hn * 128,
                 pb = (size_t)(k_pad / 64) * hn * 128;
    const size_t smem = 1024 + SAS_HDR + kg + qb + pb;
    int cols = (int)(nt * hn + dv_tiles * hn);
    int tcols = 32;
    while (tcols < cols) tcols <<= 1;
    if (hn > 0 && K <= SAS_MAX_K && dv <= 256 && smem <= 232448 && tcols <= 512) {
      SaSmallParams sp{};
      sp.q = static_cast<const uint16_t*>(q);
      sp.idx = idx;
      sp.kv = static_cast<const uint16_t*>(kv);
      sp.sink = sink;
      sp.out = static_cast<uint16_t*>(out);
      sp.B = (int)B; sp.M = (int)M; sp.H = (int)H; sp.D = (int)D; sp.N = (int)N; sp.K = (int)K;
      sp.dv_begin = (int)dv_begin; sp.dv = (int)dv;
      sp.nt = (int)nt; sp.nkb = nkb; sp.dv_tiles = dv_tiles;
      sp.kg_off = SAS_HDR;
      sp.q_off = (uint32_t)(SAS_HDR + kg);
      sp.p_off = (uint32_t)(SAS_HDR + kg + qb);
      sp.tmem_cols = (uint32_t)tcols;
      sp.scale_log2 = scale * 1.4426950408889634f;
      sp.status = dev->status;
      sp.budget_ns = wait_budget_ns();
      // two warp groups for up to two key tiles, four (one per tile) beyond
      const bool wide = nt > 2;
      const void* fn =
          wide ? (hn == 16 ? reinterpret_cast<const void*>(sparse_attn_small_kernel<16, 4>)
                  : hn == 32 ? reinterpret_cast<const void*>(sparse_attn_small_kernel<32, 4>)
                             : reinterpret_cast<const void*>(sparse_attn_small_kernel<64, 4>))
               : (hn == 16 ? reinterpret_cast<const void*>(sparse_attn_small_kernel<16, 2>)
                  : hn == 32 ? reinterpret_cast<const void*>(sparse_attn_small_kernel<32, 2>)
                             : reinterpret_cast<const void*>(sparse_attn_small_kernel<64, 2>));
      if (int rc = smem_optin(dev, fn, "cudaFuncSetAttribute(sparse_attn_small)")) return rc;
      const unsigned grid = (unsigned)(B * M);
      if (wide) {
        if (hn == 16) sparse_attn_small_kernel<16, 4><<<grid, 512, smem, st>>>(sp);
        else if (hn == 32) sparse_attn_small_kernel<32, 4><<<grid, 512, smem, st>>>(sp);
        else sparse_attn_small_kernel<64, 4><<<grid, 512, smem, st>>>(sp);
      } else {
        if (hn == 16) sparse_attn_small_kernel<16, 2><<<grid, 256, smem, st>>>(sp);
        else if (hn == 32) sparse_attn_small_kernel<32, 2><<<grid, 256, smem, st>>>(sp);
        else sparse_attn_small_kernel<64, 2><<<grid, 256, smem, st>>>(sp);
      }
      return launch_check("sparse_attn_small_kernel launch");
    }
  }
  SaParams p{};
  p.idx = idx;
  p.kv = static_cast<const uint16_t*>(kv);
  p.sink = sink;
  p.out = static_cast<uint16_t*>(out);
  p.B = (int)B; p.M = (int)M; p.H = (int)H; p.D = (int)D; p.N = (int)N; p.K = (int)K;
  p.dv_begin = (int)dv_begin;
  p.dv = (int)dv;
  p.dv_pad = (int)round_up(dv, 128);
  p.n_pv = (p.dv_pad + 255) / 256;
  p.n_pvblk = 0;
  for (int i = 0; i < p.n_pv; ++i) {
    p.pv_n[i] = p.dv_pad - 256 * i < 256 ? p.dv_pad - 256 * i : 256;
    // CTA c supplies columns [256 i + c * n/2, 256 i + (c + 1) * n/2) of instruction i
    for (int c = 0; c < 2; ++c)
      for (int v = 0; v < p.pv_n[i] / 128; ++v)
        p.pv_col[c][p.n_pvblk + v] = 256 * i + c * (p.pv_n[i] / 2) + 64 * v;
    p.n_pvblk += p.pv_n[i] / 128;
  }
  p.nblk = (int)((K + SA_NB - 1) / SA_NB);
  p.idx_vec4 = (K % 4 == 0) && aligned(idx, 16);
  const uint32_t nkb = (uint32_t)(D / 64);
  p.q_off = SA_HDR;
  p.p_off = p.q_off + nkb * 8192;
  p.r_off = p.p_off + 2 * SA_PBYTES;  // P double buffered
  // ring: as many 16 KB slots as fit in the 227 KB per-CTA limit
  const size_t limit = 232448 - 1024 /* alignment slack */;
  const size_t avail = limit > p.r_off ? limit - p.r_off : 0;
  int ns = (int)(avail / SA_SLOT);
  if (ns > SA_MAX_SLOTS) ns = SA_MAX_SLOTS;
  // A multiple of the gather groups, so every use of a slot falls to the same
  // group (position n: slot n mod ns, group n mod SA_GROUPS).  The "slot empty"
  // waits are parity waits, which only hold when the waiter is at most one phase
  // ahead of the barrier; a group that did not fill the slot's previous round
  // could be two ahead of it and would overwrite a chunk not yet consumed.
  ns -= ns % SA_GROUPS;
  if (ns < SA_GROUPS)
    return fail(KS_ERR_UNSUPPORTED, "sparse_attn: shared memory too small for D=%lld", (long long)D);
  p.n_slots = ns;
  const size_t smem = 1024 + p.r_off + (size_t)ns * SA_SLOT;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out_v8 = aligned(out, 32) ? 1 : 0;  // rows are dv * 2 bytes (a multiple of 128), steps 32
  p.status = dev->status;
  p.budget_ns = wait_budget_ns();
  CUtensorMap qm;
  if (int rc = make_map_bf16(&qm, q, D, (uint64_t)(B * M * H), D * 2, 64, 64)) return rc;
  if (int rc = smem_optin(dev, reinterpret_cast<const void*>(sparse_attn_kernel),
                          "cudaFuncSetAttribute(sparse_attn)"))
    return rc;
  // Persistent: as many CTA pairs as can be resident at once (pairs must sit in
  // one GPC, so this can be below num_sms / 2), at most one per token.
  if (dev->sa_clusters_smem != smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)dev->num_sms);
    cfg.blockDim = dim3(SA_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(sparse_attn_kernel), &cfg);
    if (e != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = dev->num_sms / 2;
    }
    dev->sa_clusters = n;
    dev->sa_clusters_smem = smem;
  }
  const int64_t clusters = std::min<int64_t>(B * M, dev->sa_clusters);
  sparse_attn_kernel<<<(unsigned)(2 * clusters), SA_THREADS, smem, st>>>(qm, p);
  return launch_check("sparse_attn_kernel launch");
}

__global__ void selftest_wait_kernel(int* status, uint64_t budget_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtx w{&abort_flag, status, budget_ns};
    mbar_wait(&bar, 0, w);  // nobody arrives: gives up after budget_ns
    mbar_arrive(&bar);      // complete the phase so the barrier is left consistent
  }
}

// ------------------------------------------------------------------ allocation-free indexer
// Scratch for ks_indexer_noalloc: the bf16 score rows between the score and top-k
// kernels live in this fixed array instead of caller-provided memory.  Every GPU
// that loads the library holds it until the process exits.  In host code the name
// is only a stand-in for the device array; its device address comes from
// cudaGetSymbolAddress, once per device.
constexpr size_t kNoallocScratchBytes = 32u << 20;  // 32 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device (set up on the first
// call on that device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(KS_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(indexer scratch)");
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return KS_OK;
}

}  // namespace
}  // namespace ks

using namespace ks;

extern "C" {

const char* ks_last_error(void) { return t_err.c_str(); }

int ks_version(void) { return 101; }

int ks_sinkhorn(const float* x, float* out, int64_t n_mats, int32_t n, int32_t repeat, float eps,
                void* stream) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  if (!x || !out) return fail(KS_ERR_INVALID, "sinkhorn: null pointer");
  if (n_mats < 0 || n < 1) return fail(KS_ERR_INVALID, "sinkhorn: bad sizes");
  if (n > 64) return fail(KS_ERR_UNSUPPORTED, "sinkhorn: n=%d > 64", n);
  if (!aligned(x, 16) || !aligned(out, 16)) return fail(KS_ERR_ALIGNMENT, "sinkhorn: pointers must be 16-byte aligned");
  if (n_mats == 0) return KS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t blocks_reg = (n_mats + SK_THREADS - 1) / SK_THREADS;
  auto launch_reg = [&](auto kern, int N) {
    const size_t smem = (size_t)SK_THREADS * (N * N + 1) * 4;
    kern<<<(unsigned)blocks_reg, SK_THREADS, smem, st>>>(x, out, n_mats, repeat, eps);
  };
  if (blocks_reg > 0x7FFFFFFFll / 2) return fail(KS_ERR_UNSUPPORTED, "sinkhorn: too many matrices");
  // even n <= 8: two threads per matrix (SK_THREADS / 2 matrices per block)
  auto launch_pair = [&](auto kern, int) {
    const int64_t blocks = (n_mats + SK_THREADS / 2 - 1) / (SK_THREADS / 2);
    kern<<<(unsigned)blocks, SK_THREADS, 0, st>>>(x, out, n_mats, repeat, eps);
  };

  switch (n) {
    case 1: launch_reg(sinkhorn_reg_kernel<1>, 1); break;
    case 2: launch_pair(sinkhorn_pair_kernel<2>, 2); break;
    case 3: launch_reg(sinkhorn_reg_kernel<3>, 3); break;
    case 4: launch_pair(sinkhorn_pair_kernel<4>, 4); break;
    case 5: launch_reg(sinkhorn_reg_kernel<5>, 5); break;
    case 6: launch_pair(sinkhorn_pair_kernel<6>, 6); break;
    case 7: launch_reg(sinkhorn_reg_kernel<7>, 7); break;
    case 8: launch_pair(sinkhorn_pair_kernel<8>, 8); break;
    default: {
      if (int rc = smem_optin(dev, reinterpret_cast<const void*>(sinkhorn_warp_kernel),
                              "cudaFuncSetAttribute(sinkhorn)"))
        return rc;
      const size_t smem = (size_t)SKW_WARPS * n * (n + 1) * 4;
      const int64_t blocks = (n_mats + SKW_WARPS - 1) / SKW_WARPS;
      sinkhorn_warp_kernel<<<(unsigned)blocks, SKW_WARPS * 32, smem, st>>>(x, out, n_mats, n, repeat, eps);
    }
  }
  return launch_check("sinkhorn kernel launch");
}

size_t ks_indexer_workspace_size(int64_t B, int64_t S, int64_t T) {
  if (B < 1 || S < 1 || T < 1) return 256;
  return (size_t)round_up(B * S * round_up(T, 8) * 2, 256);
}

int ks_indexer_scores(const void* q, const void* k, int64_t k_batch_rows, const void* w,
                      const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                      int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio,
                      void* scores, int64_t score_ld, void* stream) {
  if (int rc = indexer_check(q, k, w, freqs, B, S, H, D, T, rope_dim, ratio, k_batch_rows)) return rc;
  if (!scores || score_ld < T || score_ld % 8 || !aligned(scores, 16))
    return fail(KS_ERR_INVALID, "indexer_scores: scores must be 16-byte aligned with score_ld >= T, multiple of 8");
  return indexer_scores_impl(q, k, k_batch_rows, w, freqs, B, S, H, D, T, rope_dim, pos0, causal,
                             ratio, scores, score_ld, static_cast<cudaStream_t>(stream));
}

int ks_topk_rows(const void* scores, int64_t score_ld, int64_t B, int64_t S, int64_t T,
                 int64_t pos0, int32_t causal, int32_t ratio, int32_t topk, int64_t offset,
                 void* out, int32_t out_dtype, void* stream) {
  return topk_impl(scores, score_ld, B, S, T, pos0, causal, ratio, topk, offset, out, out_dtype,
                   static_cast<cudaStream_t>(stream));
}

int ks_indexer(const void* q, const void* k, int64_t k_batch_rows, const void* w,
               const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
               int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio, int32_t topk,
               int64_t offset, void* out, int32_t out_dtype, void* workspace,
               size_t workspace_bytes, void* stream) {
  if (int rc = indexer_check(q, k, w, freqs, B, S, H, D, T, rope_dim, ratio, k_batch_rows)) return rc;
  if (topk < 1 || topk > 4096) return fail(KS_ERR_UNSUPPORTED, "indexer: topk=%d (1..4096)", topk);
  if (!out) return fail(KS_ERR_INVALID, "indexer: out is null");
  if (T == 0) return KS_OK;
  const size_t need = ks_indexer_workspace_size(B, S, T);
  if (!workspace || workspace_bytes < need)
    return fail(KS_ERR_WORKSPACE, "indexer: workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(KS_ERR_ALIGNMENT, "indexer: workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ld = round_up(T, 8);
  if (int rc = indexer_scores_impl(q, k, k_batch_rows, w, freqs, B, S, H, D, T, rope_dim, pos0,
                                   causal, ratio, workspace, ld, st))
    return rc;
  return topk_impl(workspace, ld, B, S, T, pos0, causal, ratio, topk, offset, out, out_dtype, st);
}

int ks_sparse_attn(const void* q, const void* kv, const float* attn_sink,
                   const int32_t* topk_idxs, void* out, int64_t B, int64_t M, int64_t H,
                   int64_t D, int64_t N, int64_t K, int64_t dv_begin, int64_t dv,
                   float softmax_scale, void* stream) {
  return sparse_attn_impl(q, kv, attn_sink, topk_idxs, out, B, M, H, D, N, K, dv_begin, dv,
                          softmax_scale, static_cast<cudaStream_t>(stream));
}

int ks_dsa(const void* q_ix, const void* k_ix, int64_t k_batch_rows, const void* w,
           const float* freqs, int64_t B, int64_t S, int64_t H_ix, int64_t D_ix, int64_t T,
           int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio, int32_t topk,
           int64_t offset, const void* q_sa, const void* kv, int64_t N, const float* attn_sink,
           int64_t H_sa, int64_t D_sa, int64_t dv, float softmax_scale, int32_t* idx_out,
           void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = indexer_check(q_ix, k_ix, w, freqs, B, S, H_ix, D_ix, T, rope_dim, ratio, k_batch_rows))
    return rc;
  if (topk < 1 || topk > 4096) return fail(KS_ERR_UNSUPPORTED, "dsa: topk=%d (1..4096)", topk);
  if (!idx_out || !out) return fail(KS_ERR_INVALID, "dsa: idx_out and out must be set");
  if (T < 1) return fail(KS_ERR_INVALID, "dsa: T=%lld leaves no key to attend to", (long long)T);
  const size_t need = ks_indexer_workspace_size(B, S, T);
  if (!workspace || workspace_bytes < need)
    return fail(KS_ERR_WORKSPACE, "dsa: workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(KS_ERR_ALIGNMENT, "dsa: workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ld = round_up(T, 8);
  const int64_t K = topk < T ? topk : T;
  if (int rc = indexer_scores_impl(q_ix, k_ix, k_batch_rows, w, freqs, B, S, H_ix, D_ix, T,
                                   rope_dim, pos0, causal, ratio, workspace, ld, st))
    return rc;
  if (int rc = topk_impl(workspace, ld, B, S, T, pos0, causal, ratio, topk, offset, idx_out,
                         KS_INT32, st))
    return rc;
  return sparse_attn_impl(q_sa, kv, attn_sink, idx_out, out, B, S, H_sa, D_sa, N, K, 0, dv,
                          softmax_scale, st);
}

int ks_proj_rope(const void* a, const void* w, void* out, int64_t M, int64_t N, int64_t K,
                 int32_t head_dim, int32_t rope_dim, const float* freqs, int64_t S, float scale,
                 int32_t apply_scale, void* stream) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  if (!a || !w || !out) return fail(KS_ERR_INVALID, "proj_rope: null pointer");
  if (M < 0 || N < 16 || K < 8 || N % 16 || K % 8)
    return fail(KS_ERR_INVALID, "proj_rope: M=%lld N=%lld K=%lld (N a multiple of 16, K of 8)", (long long)M, (long long)N, (long long)K);
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return fail(KS_ERR_UNSUPPORTED, "proj_rope: too large");
  if (rope_dim < 0 || rope_dim % 2) return fail(KS_ERR_INVALID, "proj_rope: rope_dim=%d must be even", rope_dim);
  if (rope_dim > 0) {
    if (head_dim < rope_dim || head_dim % 16 || N % head_dim)
      return fail(KS_ERR_INVALID, "proj_rope: head_dim=%d must be a multiple of 16 that divides N and holds rope_dim", head_dim);
    if (!freqs || S < 1 || !aligned(freqs, 8)) return fail(KS_ERR_INVALID, "proj_rope: freqs [S, rope_dim/2, 2] (8-byte aligned) required");
  }
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16))
    return fail(KS_ERR_ALIGNMENT, "proj_rope: a, w, out must be 16-byte aligned");
  if (M == 0) return KS_OK;
  int n_tile = 256;
  while (N % n_tile) n_tile >>= 1;  // N % 16 == 0, so this stops at 16 or above
  ProjParams p{};
  p.out = static_cast<uint16_t*>(out);
  p.freqs = freqs;
  p.M = (int)M; p.N = (int)N; p.K = (int)K; p.S = (int)(S > 0 ? S : 1);
  p.n_tile = n_tile;
  p.hd = rope_dim > 0 ? head_dim : 16;
  p.rd = rope_dim;
  p.scale = scale;
  p.apply_scale = apply_scale ? 1 : 0;
  if (rope_dim > 64) return fail(KS_ERR_UNSUPPORTED, "proj_rope: rope_dim=%d > 64", rope_dim);
  const size_t st_bytes = (size_t)PG_TILE_M * 128 + (size_t)n_tile * 128;
  // per-row RoPE factors of the tile (epilogue), rows of rd + 2 words
  const size_t fr_bytes = rope_dim > 0 ? round_up((int64_t)PG_TILE_M * (rope_dim + 2) * 4, 1024) : 0;
  // output through TMA stores (boxes of 64 columns) when a tile is at least that wide
  p.tma_store = n_tile >= 64 ? 1 : 0;
  const size_t out_stage = p.tma_store ? 32768 : 0;
  // Tiles at most 64 columns wide need at most 2 x 64 TMEM columns: two CTAs share
  // an SM (half the shared memory each) when that still leaves three ring stages,
  // so a short grid (e.g. N = 16: 163 tiles on 148 SMs) runs in one wave.
  const size_t two_budget = 112 * 1024;
  const bool two_per_sm = n_tile <= 64 && (int)((two_budget - 2048 - fr_bytes - out_stage) / st_bytes) >= 3;
  const size_t budget = two_per_sm ? two_budget : 232448;
  p.acc_cols = n_tile >= 128 ? 256u : (n_tile < 32 ? 32u : (uint32_t)n_tile);
  p.tmem_cols = 2 * p.acc_cols;
  int stages = (int)((budget - 2048 - fr_bytes - out_stage) / st_bytes);
  if (stages > PG_MAX_STAGES) stages = PG_MAX_STAGES;
  if (stages < 2) return fail(KS_ERR_UNSUPPORTED, "proj_rope: shared memory too small");
  p.stages = stages;
  p.fr_off = (uint32_t)(1024 + (size_t)stages * st_bytes);
  p.st_off = (uint32_t)(p.fr_off + fr_bytes);
  p.tiles_m = (int)((M + PG_TILE_M - 1) / PG_TILE_M);
  p.tiles_n = (int)(N / n_tile);
  p.status = dev->status;
  p.budget_ns = wait_budget_ns();
  // one CTA per SM takes at least half of the shared memory, so two never share an
  // SM (each allocates all 512 TMEM columns)
  size_t smem = 1024 + 1024 + (size_t)stages * st_bytes + fr_bytes + out_stage;
  if (!two_per_sm && smem < 120 * 1024) smem = 120 * 1024;
  CUtensorMap am, bm, om;
  if (int rc = make_map_bf16(&am, a, K, (uint64_t)M, K * 2, 64, PG_TILE_M)) return rc;
  if (int rc = make_map_bf16(&bm, w, K, (uint64_t)N, K * 2, 64, n_tile)) return rc;
  if (p.tma_store) {
    if (int rc = make_map_bf16(&om, out, N, (uint64_t)M, N * 2, 64, 32)) return rc;
  } else {
    om = am;  // unused
  }
  const void* pfn = two_per_sm ? reinterpret_cast<const void*>(proj_gemm_kernel<PG_THREADS_NARROW, 2>)
                               : reinterpret_cast<const void*>(proj_gemm_kernel<PG_THREADS, 1>);
  if (int rc = smem_optin(dev, pfn, "cudaFuncSetAttribute(proj_gemm)")) return rc;
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  const int64_t slots = (int64_t)dev->num_sms * (two_per_sm ? 2 : 1);
  const int grid = (int)(tiles < slots ? tiles : slots);
  if (two_per_sm)
    proj_gemm_kernel<PG_THREADS_NARROW, 2><<<grid, PG_THREADS_NARROW, smem, static_cast<cudaStream_t>(stream)>>>(am, bm, om, p);
  else
    proj_gemm_kernel<PG_THREADS, 1><<<grid, PG_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(am, bm, om, p);
  return launch_check("proj_gemm_kernel launch");
}

int ks_quant_fp8_rows(const void* x, void* x8, float* scale, int64_t rows, int32_t D,
                      void* stream) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  if (!x || !x8 || !scale) return fail(KS_ERR_INVALID, "quant_fp8_rows: null pointer");
  if (rows < 0 || D < 4 || D % 4) return fail(KS_ERR_INVALID, "quant_fp8_rows: rows=%lld D=%d (D a multiple of 4)", (long long)rows, D);
  if (!aligned(x, 8) || !aligned(x8, 4) || !aligned(scale, 4))
    return fail(KS_ERR_ALIGNMENT, "quant_fp8_rows: x must be 8-byte and x8, scale 4-byte aligned");
  if (rows == 0) return KS_OK;
  const int64_t blocks = (rows + QF_WARPS - 1) / QF_WARPS;
  if (blocks > 0x7FFFFFFFll) return fail(KS_ERR_UNSUPPORTED, "quant_fp8_rows: too many rows");
  quant_fp8_rows_kernel<<<(unsigned)blocks, QF_WARPS * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<uint8_t*>(x8), scale, rows, D);
  return launch_check("quant_fp8_rows_kernel launch");
}

namespace {
int indexer_fp8_check(const void* q8, const void* k8, const float* w, const float* k_scale,
                      int64_t B, int64_t S, int64_t H, int64_t D, int64_t T, int32_t ratio,
                      int64_t k_batch_rows) {
  if (!q8 || !k8 || !w || !k_scale) return fail(KS_ERR_INVALID, "indexer_fp8: null input pointer");
  if (B < 1 || S < 1 || T < 0) return fail(KS_ERR_INVALID, "indexer_fp8: bad sizes B=%lld S=%lld T=%lld", (long long)B, (long long)S, (long long)T);
  if (!(H == 16 || H == 32 || H == 64)) return fail(KS_ERR_UNSUPPORTED, "indexer_fp8: H=%lld (supported: 16, 32, 64)", (long long)H);
  if (D != 128) return fail(KS_ERR_UNSUPPORTED, "indexer_fp8: D=%lld (supported: 128)", (long long)D);
  if (T > 65536) return fail(KS_ERR_UNSUPPORTED, "indexer_fp8: T=%lld > 65536", (long long)T);
  if (ratio < 1) return fail(KS_ERR_INVALID, "indexer_fp8: ratio=%d", ratio);
  if (k_batch_rows < T) return fail(KS_ERR_INVALID, "indexer_fp8: k_batch_rows < T");
  if (!aligned(q8, 16) || !aligned(k8, 16) || !aligned(w, 4) || !aligned(k_scale, 4))
    return fail(KS_ERR_ALIGNMENT, "indexer_fp8: q8, k8 must be 16-byte and w, k_scale 4-byte aligned");
  if (B * S * H >= (1ll << 31) || B * k_batch_rows >= (1ll << 31))
    return fail(KS_ERR_UNSUPPORTED, "indexer_fp8: too many rows for 32-bit TMA coordinates");
  return KS_OK;
}
}  // namespace

int ks_indexer_fp8_scores(const void* q8, const void* k8, int64_t k_batch_rows, const float* w,
                          const float* k_scale, int64_t B, int64_t S, int64_t H, int64_t D,
                          int64_t T, int64_t pos0, int32_t causal, int32_t ratio, void* scores,
                          int64_t score_ld, void* stream) {
  if (int rc = indexer_fp8_check(q8, k8, w, k_scale, B, S, H, D, T, ratio, k_batch_rows)) return rc;
  if (!scores || score_ld < T || score_ld % 8 || !aligned(scores, 16))
    return fail(KS_ERR_INVALID, "indexer_fp8_scores: scores must be 16-byte aligned with score_ld >= T, multiple of 8");
  return indexer_scores_impl(q8, k8, k_batch_rows, w, nullptr, B, S, H, D, T, 0, pos0, causal,
                             ratio, scores, score_ld, static_cast<cudaStream_t>(stream), true,
                             k_scale);
}

int ks_indexer_fp8(const void* q8, const void* k8, int64_t k_batch_rows, const float* w,
                   const float* k_scale, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                   int64_t pos0, int32_t causal, int32_t ratio, int32_t topk, int64_t offset,
                   void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (int rc = indexer_fp8_check(q8, k8, w, k_scale, B, S, H, D, T, ratio, k_batch_rows)) return rc;
  if (topk < 1 || topk > 4096) return fail(KS_ERR_UNSUPPORTED, "indexer_fp8: topk=%d (1..4096)", topk);
  if (!out) return fail(KS_ERR_INVALID, "indexer_fp8: out is null");
  if (T == 0) return KS_OK;
  const size_t need = ks_indexer_workspace_size(B, S, T);
  if (!workspace || workspace_bytes < need)
    return fail(KS_ERR_WORKSPACE, "indexer_fp8: workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(KS_ERR_ALIGNMENT, "indexer_fp8: workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ld = round_up(T, 8);
  if (int rc = indexer_scores_impl(q8, k8, k_batch_rows, w, nullptr, B, S, H, D, T, 0, pos0,
                                   causal, ratio, workspace, ld, st, true, k_scale))
    return rc;
  return topk_impl(workspace, ld, B, S, T, pos0, causal, ratio, topk, offset, out, out_dtype, st);
}

int ks_device_status(void* stream) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v[4] = {0, 0, 0, 0};
  e = cudaMemcpy(v, dev->status, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status word");
  if (v[0] != 0) {
    const int zero[4] = {0, 0, 0, 0};
    e = cudaMemcpy(dev->status, zero, sizeof(zero), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clear status word");
    if (v[0] == DEV_TIMEOUT)
      return fail(KS_ERR_DEVICE,
                  "device status %d (a bounded wait timed out: block %d, thread %d, barrier at "
                  "shared offset %d, parity %d, tag %d)",
                  v[0], v[1], (int)((unsigned)v[2] >> 20), (v[2] >> 1) & 0x7FFFF, v[2] & 1, v[3]);
    if (v[0] == DEV_BOUNDS)
      return fail(KS_ERR_DEVICE,
                  "device status %d (query row %d held an index >= its table size %d; the "
                  "access was skipped)",
                  v[0], v[1], v[3]);
    return fail(KS_ERR_DEVICE, "device status %d", v[0]);
  }
  return KS_OK;
}

int ks_indexer_noalloc(const void* q, const void* k, int64_t k_batch_rows, const void* w,
                       const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                       int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio,
                       int32_t topk, int64_t offset, void* out, int32_t out_dtype,
                       void* stream) {
  if (int rc = indexer_check(q, k, w, freqs, B, S, H, D, T, rope_dim, ratio, k_batch_rows)) return rc;
  if (topk < 1 || topk > 4096) return fail(KS_ERR_UNSUPPORTED, "indexer: topk=%d (1..4096)", topk);
  if (!out) return fail(KS_ERR_INVALID, "indexer: out is null");
  if (T == 0) return KS_OK;
  const size_t need = ks_indexer_workspace_size(B, S, T);
  if (need > kNoallocScratchBytes)
    return fail(KS_ERR_WORKSPACE,
                "indexer_noalloc: B*S*round_up(T,8)*2 = %zu bytes of scores exceeds the fixed "
                "%zu-byte scratch; split the rows into smaller calls or use ks_indexer",
                need, kNoallocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Nothing in the scratch has to start at zero: the score kernel writes every
  // element the top-k kernel reads (each row's causal prefix).
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ld = round_up(T, 8);
  if (int rc = indexer_scores_impl(q, k, k_batch_rows, w, freqs, B, S, H, D, T, rope_dim, pos0,
                                   causal, ratio, scratch, ld, st))
    return rc;
  return topk_impl(scratch, ld, B, S, T, pos0, causal, ratio, topk, offset, out, out_dtype, st);
}

int ks_selftest_wait_timeout(uint64_t budget_ns, void* stream) {
  Device* dev;
  if (int rc = device(&dev)) return rc;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status, budget_ns);
  return launch_check("selftest_wait_kernel launch");
}

}  // extern "C"
