// Exact two-digit GEMM on CUDA cores (EX_ALGO_SIMT): int8 dp4a products, int32 accumulation, int64 combine.
//
// Same integer arithmetic as the reference's _exact_kernel (kernels.py:103-157): three (or four) digit dot products,
// tot = (hh << 16) + (md << 8) + ll, then the shared epilogue. It is the portable correctness baseline of this
// library and handles every shape and alignment (any leading dimension, any K); the tensor-core kernels must match
// it bit for bit.
//
// Mapping: one weight row n per thread (256 rows per CTA), the activation digits of up to 8 tokens for a K chunk
// staged in shared memory and read as broadcasts. Split-K partitions K over gridDim.y; partial totals are added into
// an int64 workspace with relaxed atomics (exact in any order) and the last CTA of each row block (counted with an
// atomic ticket) runs the epilogue and returns the workspace to zero.
#pragma once
#include "ex_common.cuh"

namespace ex {

constexpr int SIMT_THREADS = 256;
constexpr int SIMT_MT = 8;    // tokens per pass
constexpr int SIMT_KC = 256;  // K elements of activation digits staged per chunk

// Final step for one output element: F=15 offset correction over the call's K, then either the raw int64 total
// (partial mode) or the scaled, rounded output.
template <int F, int OUT_DTYPE, bool PARTIAL>
__device__ __forceinline__ void ex_finish(long long tot, int m, int n, int K, const int32_t* __restrict__ cx,
                                          const int32_t* __restrict__ cw, const int32_t* __restrict__ sx,
                                          const int32_t* __restrict__ sw, void* out, int64_t ldo) {
  if constexpr (F == 15) tot += 128ll * ((long long)cx[m] + (long long)cw[n]) + 16384ll * (long long)K;
  if constexpr (PARTIAL) {
    reinterpret_cast<long long*>(out)[(int64_t)m * ldo + n] = tot;
  } else {
    ex_store_out<OUT_DTYPE>(out, (int64_t)m * ldo + n, ex_scale_to_f32(tot, sx[m], sw[n]));
  }
}

__device__ __forceinline__ void load16_i8(const int8_t* p, int valid, bool vec, int (&w)[4]) {
  if (vec && valid >= 16) {
    int4 v = __ldg(reinterpret_cast<const int4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t u = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = 4 * i + j;
        const uint32_t b = idx < valid ? (uint32_t)(uint8_t)__ldg(p + idx) : 0u;
        u |= b << (8 * j);
      }
      w[i] = (int)u;
    }
  }
}

template <int F, bool TRUNC, int OUT_DTYPE, bool PARTIAL>
__global__ void __launch_bounds__(SIMT_THREADS) k_exact_simt(
    const int8_t* __restrict__ xh, const int8_t* __restrict__ xl, int64_t ldx, const int32_t* __restrict__ cx,
    const int32_t* __restrict__ sx, const int8_t* __restrict__ wh, const int8_t* __restrict__ wl, int64_t ldw,
    const int32_t* __restrict__ cw, const int32_t* __restrict__ sw, int M, int N, int K, int kchunk, bool vecw,
    void* out, int64_t ldo, long long* __restrict__ ws_acc, int* __restrict__ ws_cnt) {
  __shared__ __align__(16) int8_t xs_h[SIMT_MT][SIMT_KC];
  __shared__ __align__(16) int8_t xs_l[SIMT_MT][SIMT_KC];
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int n = blockIdx.x * SIMT_THREADS + tid;
  const int splits = gridDim.y;
  const int k0 = blockIdx.y * kchunk;
  const int k1 = min(K, k0 + kchunk);
  const int8_t* whr = wh + (int64_t)min(n, N - 1) * ldw;
  const int8_t* wlr = wl + (int64_t)min(n, N - 1) * ldw;

  for (int mt0 = 0; mt0 < M; mt0 += SIMT_MT) {
    int hh[SIMT_MT], md[SIMT_MT], ll[SIMT_MT];
#pragma unroll
    for (int t = 0; t < SIMT_MT; ++t) hh[t] = md[t] = ll[t] = 0;
    for (int kc = k0; kc < k1; kc += SIMT_KC) {
      __syncthreads();
      // stage activation digits [mt0, mt0+8) x [kc, kc+SIMT_KC) (zero outside M / outside this split's K range)
      for (int i = tid; i < SIMT_MT * SIMT_KC; i += SIMT_THREADS) {
        const int t = i / SIMT_KC, kk = i % SIMT_KC;
        const int m = mt0 + t, k = kc + kk;
        const bool ok = (m < M) && (k < k1);
        xs_h[t][kk] = ok ? xh[(int64_t)m * ldx + k] : (int8_t)0;
        xs_l[t][kk] = ok ? xl[(int64_t)m * ldx + k] : (int8_t)0;
      }
      __syncthreads();
      if (n < N) {
        const int kend = min(SIMT_KC, k1 - kc);
        for (int kk = 0; kk < kend; kk += 16) {
          int a_h[4], a_l[4];
          load16_i8(whr + kc + kk, kend - kk, vecw, a_h);
          load16_i8(wlr + kc + kk, kend - kk, vecw, a_l);
#pragma unroll
          for (int t = 0; t < SIMT_MT; ++t) {
            const int4 bh = *reinterpret_cast<const int4*>(&xs_h[t][kk]);
            const int4 bl = *reinterpret_cast<const int4*>(&xs_l[t][kk]);
            hh[t] = __dp4a(a_h[0], bh.x, hh[t]);
            hh[t] = __dp4a(a_h[1], bh.y, hh[t]);
            hh[t] = __dp4a(a_h[2], bh.z, hh[t]);
            hh[t] = __dp4a(a_h[3], bh.w, hh[t]);
            md[t] = __dp4a(a_h[0], bl.x, md[t]);
            md[t] = __dp4a(a_h[1], bl.y, md[t]);
            md[t] = __dp4a(a_h[2], bl.z, md[t]);
            md[t] = __dp4a(a_h[3], bl.w, md[t]);
            md[t] = __dp4a(a_l[0], bh.x, md[t]);
            md[t] = __dp4a(a_l[1], bh.y, md[t]);
            md[t] = __dp4a(a_l[2], bh.z, md[t]);
            md[t] = __dp4a(a_l[3], bh.w, md[t]);
            if constexpr (!TRUNC) {
              ll[t] = __dp4a(a_l[0], bl.x, ll[t]);
              ll[t] = __dp4a(a_l[1], bl.y, ll[t]);
              ll[t] = __dp4a(a_l[2], bl.z, ll[t]);
              ll[t] = __dp4a(a_l[3], bl.w, ll[t]);
            }
          }
        }
      }
    }
    if (n < N) {
#pragma unroll
      for (int t = 0; t < SIMT_MT; ++t) {
        const int m = mt0 + t;
        if (m < M) {
          const long long tot = ex_combine(hh[t], md[t], ll[t]);
          if (splits == 1)
            ex_finish<F, OUT_DTYPE, PARTIAL>(tot, m, n, K, cx, cw, sx, sw, out, ldo);
          else
            red_add_s64(ws_acc + (int64_t)m * N + n, tot);
        }
      }
    }
  }
  if (splits == 1) return;
  // split-K completion: the last CTA of this row block applies the epilogue and clears the workspace
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(ws_cnt + blockIdx.x, 1) == splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (n < N) {
#pragma unroll 4
    for (int m = 0; m < M; ++m) {
      long long* p = ws_acc + (int64_t)m * N + n;
      const long long tot = __ldcg(p);  // every other contribution is in L2; this CTA owns the row block now
      __stcg(p, 0ll);
      ex_finish<F, OUT_DTYPE, PARTIAL>(tot, m, n, K, cx, cw, sx, sw, out, ldo);
    }
  }
  if (tid == 0) ws_cnt[blockIdx.x] = 0;
}

// Scaling epilogue of an int64 total (ex_epilogue_i64).
template <int OUT_DTYPE>
__global__ void k_epilogue_i64(const long long* __restrict__ tot, int64_t ldt, const int32_t* __restrict__ sx,
                               const int32_t* __restrict__ sw, int M, int N, void* out, int64_t ldo) {
  const int64_t total = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    ex_store_out<OUT_DTYPE>(out, (int64_t)m * ldo + n, ex_scale_to_f32(tot[(int64_t)m * ldt + n], sx[m], sw[n]));
  }
}

}  // namespace ex
