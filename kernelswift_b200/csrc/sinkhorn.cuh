// Sinkhorn normalisation of a batch of n x n fp32 matrices, all iterations on chip.
//
// Semantics follow baseline/sinkhorn.py:13-19 of KernelSwift:
//   x = softmax(x, -1) + eps            (eps outside the softmax denominator)
//   x = x / (colsum(x) + eps)
//   repeat-1 times: x = x / (rowsum(x) + eps); x = x / (colsum(x) + eps)
// One HBM read and one HBM write per matrix.  The reference NPU kernel
// (optimized/sinkhorn_project/op_kernel/sinkhorn_kernel.asc:168-189) is limited
// to 4x4; here any n is accepted.
//
// Register path (n <= 8): one thread owns one matrix in registers.  A block of
// 128 threads stages its 128 contiguous matrices through shared memory so the
// HBM traffic is 128-bit coalesced; the per-thread copy uses an odd word stride
// (n*n + 1) so shared-memory reads are free of bank conflicts.
// Scaling path (even n <= 8): see sinkhorn_pair_kernel (two threads per matrix).
// Warp path (8 < n <= 64): one warp per matrix in shared memory.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int SK_THREADS = 128;

// 1/d from the hardware reciprocal (rcp.approx: within 1 ulp; d >= eps > 0 here).
__device__ __forceinline__ float sk_rcp(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}
// Two fp32 lanes in one 64-bit register: add/mul.rn.f32x2 do two IEEE operations
// per instruction.
__device__ __forceinline__ uint64_t sk_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void sk_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t sk_add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sk_mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sk_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

template <int N>
__global__ void __launch_bounds__(SK_THREADS)
    sinkhorn_reg_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n_mats,
                        int repeat, float eps) {
  constexpr int NN = N * N;
  constexpr int STRIDE = NN + 1;  // odd word stride: conflict-free per-thread access
  extern __shared__ float sk_smem[];
  const int tid = threadIdx.x;
  const int64_t mat0 = (int64_t)blockIdx.x * SK_THREADS;
  const int nm = (int)min((int64_t)SK_THREADS, n_mats - mat0);
  const float* src = x + mat0 * NN;
  float* dst = out + mat0 * NN;
  const int total = nm * NN;

  // coalesced load of the block's contiguous chunk into the padded layout
  if (nm == SK_THREADS && (NN % 4) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (int v = tid; v < total / 4; v += SK_THREADS) {
      float4 f = __ldcs(s4 + v);
      int e = v * 4;
      int m = e / NN, o = e % NN;
      float* d = sk_smem + m * STRIDE + o;
      d[0] = f.x; d[1] = f.y; d[2] = f.z; d[3] = f.w;
    }
  } else {
    for (int e = tid; e < total; e += SK_THREADS) {
      int m = e / NN, o = e % NN;
      sk_smem[m * STRIDE + o] = __ldcs(src + e);
    }
  }
  __syncthreads();

  if (tid < nm) {
    float a[N][N];
    const float* my = sk_smem + tid * STRIDE;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) a[i][j] = my[i * N + j];

    // softmax over the last dim, then + eps (exp through ex2 of x * log2(e))
    constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float m = a[i][0];
#pragma unroll
      for (int j = 1; j < N; ++j) m = fmaxf(m, a[i][j]);
      const float mb = m * kLog2e;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        a[i][j] = exp2f(fmaf(a[i][j], kLog2e, -mb));
        s += a[i][j];
      }
      const float r = sk_rcp(s);
#pragma unroll
      for (int j = 0; j < N; ++j) a[i][j] = fmaf(a[i][j], r, eps);
    }
    const int rounds = repeat < 1 ? 1 : repeat;
    if constexpr (N % 2 == 0) {
      // pairs of adjacent columns: p[i][c] = (a[i][2c], a[i][2c + 1])
      constexpr int C = N / 2;
      uint64_t pr[N][C];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < C; ++c) pr[i][c] = sk_pack(a[i][2 * c], a[i][2 * c + 1]);
      const uint64_t eps2 = sk_pack(eps, eps);
      // baseline/sinkhorn.py:15-18: one column pass, then repeat-1 (row, column) pairs
      for (int it = 0; it < rounds; ++it) {
        if (it > 0) {  // row normalisation (skipped in the first round)
#pragma unroll
          for (int i = 0; i < N; ++i) {
            uint64_t sp = pr[i][0];
#pragma unroll
            for (int c = 1; c < C; ++c) sp = sk_add2(sp, pr[i][c]);
            float lo, hi;
            sk_unpack(sp, lo, hi);
            const float r = sk_rcp(lo + hi + eps);
            const uint64_t r2 = sk_pack(r, r);
#pragma unroll
            for (int c = 0; c < C; ++c) pr[i][c] = sk_mul2(pr[i][c], r2);
          }
        }
        // column normalisation, two columns at a time
#pragma unroll
        for (int c = 0; c < C; ++c) {
          uint64_t sp = pr[0][c];
#pragma unroll
          for (int i = 1; i < N; ++i) sp = sk_add2(sp, pr[i][c]);
          sp = sk_add2(sp, eps2);
          float lo, hi;
          sk_unpack(sp, lo, hi);
          const uint64_t r2 = sk_pack(sk_rcp(lo), sk_rcp(hi));
#pragma unroll
          for (int i = 0; i < N; ++i) pr[i][c] = sk_mul2(pr[i][c], r2);
        }
      }
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < C; ++c) sk_unpack(pr[i][c], a[i][2 * c], a[i][2 * c + 1]);
    } else {
      // baseline/sinkhorn.py:15-18: one column pass, then repeat-1 (row, column) pairs
      for (int it = 0; it < rounds; ++it) {
        if (it > 0) {  // row normalisation (skipped in the first round)
#pragma unroll
          for (int i = 0; i < N; ++i) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) s += a[i][j];
            const float r = sk_rcp(s + eps);
#pragma unroll
            for (int j = 0; j < N; ++j) a[i][j] *= r;
          }
        }
        // column normalisation
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s += a[i][j];
          const float r = sk_rcp(s + eps);
#pragma unroll
          for (int i = 0; i < N; ++i) a[i][j] *= r;
        }
      }
    }
    float* myw = sk_smem + tid * STRIDE;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) myw[i * N + j] = a[i][j];
  }
  __syncthreads();

  if (nm == SK_THREADS && (NN % 4) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int v = tid; v < total / 4; v += SK_THREADS) {
      int e = v * 4;
      int m = e / NN, o = e % NN;
      const float* s = sk_smem + m * STRIDE + o;
      __stcs(d4 + v, make_float4(s[0], s[1], s[2], s[3]));
    }
  } else {
    for (int e = tid; e < total; e += SK_THREADS) {
      int m = e / NN, o = e % NN;
      __stcs(dst + e, sk_smem[m * STRIDE + o]);
    }
  }
}

// Scaling path (even n <= 8).  The iteration is carried as
//   x_ij = u_i K_ij v_j,  K = softmax(x) + eps,  u = v = 1,
// which is the reference's sequence of normalisations written with row and column
// scale vectors:
//   column pass:  v_j <- v_j / (v_j (u^T K)_j + eps)
//   row pass:     u_i <- u_i / (u_i (K v)_i + eps)
// so each pass is one matrix-vector product (n^2 FMAs, two columns at a time as
// f32x2) plus n reciprocals, instead of rewriting all n^2 entries (sums and
// products) every pass.  The result x_ij = u_i K_ij v_j is formed once at the end.
// Only the rounding differs from the reference's entry-wise updates.
// Two threads per matrix, so twice as many warps hide the latency of the
// per-matrix chain (one thread per matrix leaves a C5-sized batch at ~14 warps
// per SM).  Thread h of a pair (lanes 2k, 2k + 1) owns rows [h n/2, (h+1) n/2) of
// K and their u, and keeps all of v.  Each thread holds its columns rotated by
// h n/2, so local columns 0 .. n/2-1 are the ones whose v it updates and local
// column n/2 + k of one thread is local column k of its partner.  Row pass:
// local.  Column pass: each thread forms the partial column sums of its rows;
// one shuffle per column brings the partner's part of the columns this thread
// updates, and one more returns the new v.
// Reciprocals go in pairs (1/a = b r, 1/b = a r with r = 1/(a b)): the XU pipe
// (rcp, ex2) runs 16 operations per clock per SM against 128 FMAs, and at C5's
// size it bounded the kernel; the pairing trades half the reciprocals for three
// multiplies.  The denominators are sums plus eps, far from the fp32 range ends,
// so their products neither overflow nor underflow.
// No shared-memory staging: each thread loads its own rows (a contiguous half
// matrix, 16-byte loads when the half is a multiple of 16 bytes) and stores them
// back the same way, so every warp starts as soon as its own loads land (the C5
// batch is a single wave: a block-wide staging step made all its warps wait for
// the slowest load).
__device__ __forceinline__ void sk_rcp_pair(float a, float b, float& ra, float& rb) {
  const float r = sk_rcp(a * b);
  ra = b * r;
  rb = a * r;
}

template <int N>
__global__ void __launch_bounds__(SK_THREADS)
    sinkhorn_pair_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n_mats,
                         int repeat, float eps) {
  static_assert(N % 2 == 0 && N <= 8, "pair path: even n <= 8");
  constexpr int NN = N * N;
  constexpr int R = N / 2;         // rows per thread, and columns whose v it updates
  constexpr int C = N / 2;         // column pairs
  constexpr int HW = NN / 2;       // words per row half
  constexpr bool V4 = (HW % 4) == 0;
  const int tid = threadIdx.x;
  const int h = tid & 1;
  const int64_t mat = (int64_t)blockIdx.x * (SK_THREADS / 2) + (tid >> 1);
  const bool live = mat < n_mats;  // threads past the batch run the iteration (shuffles) on zeros
  const float* src = x + (live ? mat : 0) * NN + h * HW;
  float* dst = out + mat * NN + h * HW;

  {
    // Every thread runs the iteration (the shuffles need all lanes).
    float raw[HW];
    if (live) {
      if constexpr (V4) {
#pragma unroll
        for (int q = 0; q < HW / 4; ++q) {
          const float4 f = __ldcs(reinterpret_cast<const float4*>(src) + q);
          raw[4 * q] = f.x; raw[4 * q + 1] = f.y; raw[4 * q + 2] = f.z; raw[4 * q + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < HW; ++e) raw[e] = __ldcs(src + e);
      }
    } else {
#pragma unroll
      for (int e = 0; e < HW; ++e) raw[e] = 0.f;
    }
    // K = softmax(x) + eps for this thread's rows, as (local) column pairs
    uint64_t kp[R][C];
    constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      float r[N];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        // global column (j + rot) mod N; rot is 0 or R, selected without indexing
        const int j0 = j, j1 = j + R < N ? j + R : j + R - N;
        r[j] = h ? raw[i * N + j1] : raw[i * N + j0];
      }
      float m = r[0];
#pragma unroll
      for (int j = 1; j < N; ++j) m = fmaxf(m, r[j]);
      const float mb = m * kLog2e;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        r[j] = exp2f(fmaf(r[j], kLog2e, -mb));
        s += r[j];
      }
      const float rs = sk_rcp(s);
#pragma unroll
      for (int c = 0; c < C; ++c) kp[i][c] = sk_pack(fmaf(r[2 * c], rs, eps), fmaf(r[2 * c + 1], rs, eps));
    }
    float u[R], v[N];  // v in local column order
#pragma unroll
    for (int i = 0; i < R; ++i) u[i] = 1.f;
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = 1.f;
    const int rounds = repeat < 1 ? 1 : repeat;
    for (int it = 0; it < rounds; ++it) {
      if (it > 0) {  // row pass: u_i <- u_i / (u_i (K v)_i + eps)
        uint64_t vp[C];
#pragma unroll
        for (int c = 0; c < C; ++c) vp[c] = sk_pack(v[2 * c], v[2 * c + 1]);
        float d[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
          uint64_t acc = sk_mul2(kp[i][0], vp[0]);
#pragma unroll
          for (int c = 1; c < C; ++c) acc = sk_fma2(kp[i][c], vp[c], acc);
          float lo, hi;
          sk_unpack(acc, lo, hi);
          d[i] = fmaf(u[i], lo + hi, eps);
        }
#pragma unroll
        for (int i = 0; i + 1 < R; i += 2) {
          float r0, r1;
          sk_rcp_pair(d[i], d[i + 1], r0, r1);
          u[i] *= r0;
          u[i + 1] *= r1;
        }
        if constexpr (R % 2) u[R - 1] *= sk_rcp(d[R - 1]);
      }
      // column pass: partial sums of this thread's rows, then v_j <- v_j / (v_j t_j + eps)
      uint64_t t[C];
      {
        const uint64_t u0 = sk_pack(u[0], u[0]);
#pragma unroll
        for (int c = 0; c < C; ++c) t[c] = sk_mul2(kp[0][c], u0);
      }
#pragma unroll
      for (int i = 1; i < R; ++i) {
        const uint64_t ui = sk_pack(u[i], u[i]);
#pragma unroll
        for (int c = 0; c < C; ++c) t[c] = sk_fma2(kp[i][c], ui, t[c]);
      }
      float tf[N];
#pragma unroll
      for (int c = 0; c < C; ++c) sk_unpack(t[c], tf[2 * c], tf[2 * c + 1]);
      // this thread updates its local columns k < R; the partner sends its partial
      // sums of them (its local columns R + k) and gets back the new v
      float d[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const float theirs = __shfl_xor_sync(0xFFFFFFFFu, tf[R + k], 1);
        d[k] = fmaf(v[k], tf[k] + theirs, eps);
      }
#pragma unroll
      for (int k = 0; k + 1 < R; k += 2) {
        float r0, r1;
        sk_rcp_pair(d[k], d[k + 1], r0, r1);
        v[k] *= r0;
        v[k + 1] *= r1;
      }
      if constexpr (R % 2) v[R - 1] *= sk_rcp(d[R - 1]);
#pragma unroll
      for (int k = 0; k < R; ++k) v[R + k] = __shfl_xor_sync(0xFFFFFFFFu, v[k], 1);
    }
    // x_ij = u_i K_ij v_j for this thread's rows, back in global column order
    uint64_t vp[C];
#pragma unroll
    for (int c = 0; c < C; ++c) vp[c] = sk_pack(v[2 * c], v[2 * c + 1]);
    float res[HW];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const uint64_t ui = sk_pack(u[i], u[i]);
      float loc[N];
#pragma unroll
      for (int c = 0; c < C; ++c) sk_unpack(sk_mul2(sk_mul2(kp[i][c], ui), vp[c]), loc[2 * c], loc[2 * c + 1]);
#pragma unroll
      for (int g = 0; g < N; ++g) {
        // global column g is local column (g - rot) mod N
        const int l0 = g, l1 = g - R >= 0 ? g - R : g - R + N;
        res[i * N + g] = h ? loc[l1] : loc[l0];
      }
    }
    if (live) {
      if constexpr (V4) {
#pragma unroll
        for (int q = 0; q < HW / 4; ++q)
          __stcs(reinterpret_cast<float4*>(dst) + q,
                 make_float4(res[4 * q], res[4 * q + 1], res[4 * q + 2], res[4 * q + 3]));
      } else {
#pragma unroll
        for (int e = 0; e < HW; ++e) __stcs(dst + e, res[e]);
      }
    }
  }
}

// One warp per matrix, matrix in shared memory with row stride n+1.
constexpr int SKW_WARPS = 4;
__global__ void __launch_bounds__(SKW_WARPS * 32)
    sinkhorn_warp_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n_mats,
                         int n, int repeat, float eps) {
  extern __shared__ float skw_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = n + 1;
  float* a = skw_smem + warp * n * ld;
  const int64_t mat = (int64_t)blockIdx.x * SKW_WARPS + warp;
  if (mat >= n_mats) return;
  const float* src = x + mat * n * n;
  float* dst = out + mat * n * n;
  for (int e = lane; e < n * n; e += 32) a[(e / n) * ld + e % n] = src[e];
  __syncwarp();
  for (int i = lane; i < n; i += 32) {
    float* row = a + i * ld;
    float m = row[0];
    for (int j = 1; j < n; ++j) m = fmaxf(m, row[j]);
    float s = 0.f;
    for (int j = 0; j < n; ++j) {
      row[j] = expf(row[j] - m);
      s += row[j];
    }
    const float r = sk_rcp(s);
    for (int j = 0; j < n; ++j) row[j] = row[j] * r + eps;
  }
  __syncwarp();
  const int rounds = repeat < 1 ? 1 : repeat;
  for (int it = 0; it < rounds; ++it) {
    if (it > 0) {
      for (int i = lane; i < n; i += 32) {
        float* row = a + i * ld;
        float s = 0.f;
        for (int j = 0; j < n; ++j) s += row[j];
        const float r = sk_rcp(s + eps);
        for (int j = 0; j < n; ++j) row[j] *= r;
      }
      __syncwarp();
    }
    for (int j = lane; j < n; j += 32) {
      float s = 0.f;
      for (int i = 0; i < n; ++i) s += a[i * ld + j];
      const float r = sk_rcp(s + eps);
      for (int i = 0; i < n; ++i) a[i * ld + j] *= r;
    }
    __syncwarp();
  }
  for (int e = lane; e < n * n; e += 32) dst[e] = a[(e / n) * ld + e % n];
}

}  // namespace ks
