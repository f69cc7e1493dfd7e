// Tensor parallelism of the exact linear layer over peer memory: the two exchange steps of a row-parallel (K-sharded)
// layer, each one kernel over NVLink with plain peer loads and stores (CUDA IPC mappings; no multicast object, no
// NCCL on the data path). The reference has no multi-GPU path; exactness rests on its kernels.py:25-29 (a row's
// fixed-point scale comes from the maximum over the whole row) and :144-146, :159-177 (int64 partial totals of
// disjoint K slices add up exactly to the total of the whole K range).
//
// k_tp_digitize: row maxima of this rank's K slice -> every rank -> whole-row maxima -> digits of the slice. Each
//   maximum travels as one 64-bit word (call epoch << 32 | float bits) stored with release semantics into slot
//   [rank][row] of every rank's exchange buffer; a reader polls its own buffer until the slot carries the current
//   epoch, so the value and its flag arrive together (one store per peer and row, no separate flag round trip).
//
// k_tp_allreduce_epilogue: reduce-scatter + exact epilogue + all-gather of the int64 partial totals. Rank r owns the
//   output columns [r N / p, (r + 1) N / p): it sums the p partials of its columns (peer loads; integer addition is
//   exact in any order), applies the epilogue once, and stores the finished values into every rank's output exchange
//   buffer (peer stores). Each rank reads (p - 1) / p of one partial over NVLink and sends 1 / p of the output to each
//   peer, instead of reading every peer's whole partial. Block b of every rank works on the same positions of its
//   rank's column range, so block b only ever waits for block b of the other ranks (its `done` flag), never for
//   another block of its own grid: no kernel relies on all of its blocks being resident at once. After that wait,
//   block b copies the values the ranks' blocks b wrote into this rank's `out`.
//
// Epochs live on the device (ctl words, advanced by the last block of each call), so calls can be captured in a CUDA
// graph and replayed. Every wait is bounded (EX_WAIT_TIMEOUT_NS): a wait that runs out records EX_DEVERR_WAIT_PEER
// and the kernel finishes without the missing data (wrong outputs, reported by ex_device_error).
// Buffer reuse: a rank starts call e + 1 of either kernel only after call e of k_tp_allreduce_epilogue, whose block b
// waited for block b of every rank to finish reading this rank's partial and writing into its output buffer; so a
// partial or an exchange slot is never overwritten while a peer may still read it.
#pragma once
#include "ex_common.cuh"
#include "ex_digitize.cuh"

namespace ex {

constexpr int TPF_THREADS = 256;
constexpr int TPF_MAX_BLOCKS = EX_TP_MAX_BLOCKS;  // blocks of k_tp_allreduce_epilogue (one done flag per block and rank)
constexpr int TPF_MAX_WORLD = EX_TP_MAX_WORLD;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// peer data written before the matching flag: relaxed system-scope loads (no stale L1 copy)
__device__ __forceinline__ longlong2 ld_relaxed_sys_v2s64(const long long* p) {
  longlong2 v;
  asm volatile("ld.relaxed.sys.global.v2.s64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}

// Bounded wait until f[0] >= e. Returns false (and records the error) on timeout.
__device__ __forceinline__ bool tpf_wait_flag(const int* f, int e) {
  if (ld_acquire_sys(f) >= e) return true;
  const uint64_t t0 = ex_globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire_sys(f) >= e) return true;
    if ((it & 63u) == 0) {
      const uint64_t dt = ex_globaltimer() - t0;
      if (dt > EX_WAIT_TIMEOUT_NS || (dt > 1000000ull && *(volatile int*)&g_ex_dev_error != 0)) {
        ex_set_error(EX_DEVERR_WAIT_PEER);
        return false;
      }
    }
  }
}

// Last block of a call (counter ctl[1] reaches gridDim.x): reset the counter and publish the epoch. Every block read
// the epoch from ctl[0] before incrementing the counter, so none can read the new value.
__device__ __forceinline__ void tpf_finish_call(int* ctl, int e) {
  __threadfence();
  if (atomicAdd(ctl + 1, 1) == (int)gridDim.x - 1) {
    ctl[1] = 0;
    __threadfence();
    *(volatile int*)ctl = e;
  }
}

// ------------------------------------------------------------------------------------------------------------------
// k_tp_digitize: grid-stride over rows (grid <= rows, all blocks small enough to be resident together)
// ------------------------------------------------------------------------------------------------------------------
template <typename T, int F>
__global__ void __launch_bounds__(DIG_THREADS) k_tp_digitize(const T* __restrict__ x, int64_t ldx, int rows, int K,
                                                             unsigned long long* const* __restrict__ xch, int* ctl,
                                                             int rank, int world, int max_rows,
                                                             int8_t* __restrict__ h, int8_t* __restrict__ l,
                                                             int64_t ldd, int32_t* __restrict__ cs,
                                                             int32_t* __restrict__ sh) {
  __shared__ float redf[DIG_THREADS / 32];
  __shared__ int redi[DIG_THREADS / 32];
  __shared__ int e_s;
  __shared__ float gmax_s;
  if (threadIdx.x == 0) e_s = *(volatile int*)ctl + 1;
  __syncthreads();
  const int e = e_s;
  // 1. maxima of this rank's slice of each row, to slot [rank][row] of every rank
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + (int64_t)row * ldx;
    float amax = 0.0f;
    for (int k = threadIdx.x; k < K; k += DIG_THREADS) amax = fmaxf(amax, fabsf(to_f32<T>(xr[k])));
    amax = block_max(amax, redf);
    if ((int)threadIdx.x < world) {
      const unsigned long long w = ((unsigned long long)(uint32_t)e << 32) | __float_as_uint(amax);
      st_release_sys_u64(xch[threadIdx.x] + (int64_t)rank * max_rows + row, w);
    }
    __syncthreads();  // redf is reused by the next row's reduction
  }
  // 2. whole-row maxima from this rank's exchange buffer, then the digits of the slice
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    if (threadIdx.x < 32) {
      float v = 0.0f;
      if ((int)threadIdx.x < world) {
        const unsigned long long* slot = xch[rank] + (int64_t)threadIdx.x * max_rows + row;
        unsigned long long w = ld_acquire_sys_u64(slot);
        if ((int)(w >> 32) != e) {
          const uint64_t t0 = ex_globaltimer();
          for (uint32_t it = 1; (int)(w >> 32) != e; ++it) {
            w = ld_acquire_sys_u64(slot);
            if ((it & 63u) == 0 && (int)(w >> 32) != e) {
              const uint64_t dt = ex_globaltimer() - t0;
              if (dt > EX_WAIT_TIMEOUT_NS || (dt > 1000000ull && *(volatile int*)&g_ex_dev_error != 0)) {
                ex_set_error(EX_DEVERR_WAIT_PEER);
                break;
              }
            }
          }
        }
        v = (int)(w >> 32) == e ? __uint_as_float((uint32_t)w) : 0.0f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (threadIdx.x == 0) gmax_s = v;
    }
    __syncthreads();
    const int s = F - frexp_exponent(gmax_s);
    const float scale = __uint_as_float(((uint32_t)(s + 127)) << 23);  // 2^s, int32 wrap-around as kernels.py:29
    const T* xr = x + (int64_t)row * ldx;
    int8_t* hr = h + (int64_t)row * ldd;
    int8_t* lr = l + (int64_t)row * ldd;
    int csum = 0;
    for (int k = threadIdx.x; k < K; k += DIG_THREADS) {
      const int q = __float2int_rz(__fmul_rn(to_f32<T>(xr[k]), scale));
      int dh, dl;
      digits_of<F>(q, dh, dl);
      if constexpr (F == 15) csum += 256 * dh + dl;
      hr[k] = (int8_t)dh;
      lr[k] = (int8_t)dl;
    }
    if constexpr (F == 15) csum = block_sum_i32(csum, redi);
    if (threadIdx.x == 0) {
      cs[row] = (F == 15) ? csum : 0;
      sh[row] = s;
    }
    __syncthreads();  // gmax_s / redi are reused by the next row
  }
  __syncthreads();
  if (threadIdx.x == 0) tpf_finish_call(ctl, e);
}

// ------------------------------------------------------------------------------------------------------------------
// k_tp_allreduce_epilogue
//   parts[p]  (M, N) int64 partial of rank p, leading dimension ldt
//   outs[p]   (M, N) output exchange buffer of rank p, element type OUT_DTYPE, leading dimension N
//   flags[p]  rank p's int32 flags: [0, world) partial ready from rank q; then done[q][b] at world + q * MAX_BLOCKS + b
//   ctl       this rank's int32 x 2 (epoch, block counter)
// Columns of rank r: [c0(r), c0(r + 1)), c0(r) = r * N / world rounded down to even; pairs of columns per thread.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ int tpf_col0(int r, int N, int world) { return (int)(((int64_t)r * N / world) & ~1ll); }

template <int OUT_DTYPE>
__device__ __forceinline__ void tpf_store2(void* base, int64_t idx, float a, float b) {
  if constexpr (OUT_DTYPE == EX_DTYPE_F32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + idx) = make_float2(a, b);
  } else if constexpr (OUT_DTYPE == EX_DTYPE_BF16) {
    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(base) + idx) =
        __halves2bfloat162(__float2bfloat16_rn(a), __float2bfloat16_rn(b));
  } else {
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + idx) =
        __halves2half2(__float2half_rn(a), __float2half_rn(b));
  }
}

template <int OUT_DTYPE>
__global__ void __launch_bounds__(TPF_THREADS) k_tp_allreduce_epilogue(
    const long long* const* __restrict__ parts, int64_t ldt, void* const* __restrict__ outs,
    int* const* __restrict__ flags, int* ctl, int rank, int world, const int32_t* __restrict__ sx,
    const int32_t* __restrict__ sw, int M, int N, void* __restrict__ out, int64_t ldo) {
  constexpr int ESZ = OUT_DTYPE == EX_DTYPE_F32 ? 4 : 2;
  __shared__ int e_s, ok_s;
  const int b = blockIdx.x, B = gridDim.x;
  if (threadIdx.x == 0) {
    const int e = *(volatile int*)ctl + 1;
    e_s = e;
    // this rank's partial was written by the preceding kernel on the stream (complete): announce it to every rank
    // (every block stores the same flag value), then wait for every rank's partial of this call
    for (int p = 0; p < world; ++p) st_release_sys(flags[p] + rank, e);
    int ok = 1;
    for (int p = 0; p < world && ok; ++p) ok = tpf_wait_flag(flags[rank] + p, e) ? 1 : 0;
    ok_s = ok;
  }
  __syncthreads();
  const int e = e_s;
  if (ok_s) {
    // 1. this rank's columns: block b takes pairs [b * P / B, (b + 1) * P / B) of the M x (c1 - c0) / 2 pairs
    const int c0 = tpf_col0(rank, N, world), c1 = tpf_col0(rank + 1, N, world);
    const int half = (c1 - c0) >> 1;
    const int64_t P = (int64_t)M * half;
    const int64_t p0 = P * b / B, p1 = P * (b + 1) / B;
    for (int64_t i = p0 + threadIdx.x; i < p1; i += TPF_THREADS) {
      const int m = (int)(i / half), n = c0 + 2 * (int)(i % half);
      const int64_t off = (int64_t)m * ldt + n;
      long long t0 = 0, t1 = 0;
      for (int p = 0; p < world; ++p) {
        const longlong2 v = ld_relaxed_sys_v2s64(parts[p] + off);
        t0 += v.x;
        t1 += v.y;
      }
      const int sxm = sx[m];
      const float f0 = ex_scale_to_f32(t0, sxm, sw[n]), f1 = ex_scale_to_f32(t1, sxm, sw[n + 1]);
      for (int p = 0; p < world; ++p) tpf_store2<OUT_DTYPE>(outs[p], (int64_t)m * N + n, f0, f1);
    }
  }
  // 2. block b's stores are visible system-wide -> done[rank][b] in every rank's flags; wait for block b of every rank
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < world; ++p) st_release_sys(flags[p] + world + rank * TPF_MAX_BLOCKS + b, e);
    int ok = 1;
    for (int p = 0; p < world && ok; ++p) ok = tpf_wait_flag(flags[rank] + world + p * TPF_MAX_BLOCKS + b, e) ? 1 : 0;
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s) {
    // 3. what block b of every rank wrote into this rank's exchange buffer -> out
    const char* src = reinterpret_cast<const char*>(outs[rank]);
    for (int p = 0; p < world; ++p) {
      const int c0 = tpf_col0(p, N, world), c1 = tpf_col0(p + 1, N, world);
      const int half = (c1 - c0) >> 1;
      const int64_t P = (int64_t)M * half;
      const int64_t p0 = P * b / B, p1 = P * (b + 1) / B;
      for (int64_t i = p0 + threadIdx.x; i < p1; i += TPF_THREADS) {
        const int m = (int)(i / half), n = c0 + 2 * (int)(i % half);
        char* dst = reinterpret_cast<char*>(out) + ((int64_t)m * ldo + n) * ESZ;
        const char* s = src + ((int64_t)m * N + n) * ESZ;
        if constexpr (ESZ == 4)
          *reinterpret_cast<float2*>(dst) = __ldcv(reinterpret_cast<const float2*>(s));
        else
          *reinterpret_cast<unsigned*>(dst) = __ldcv(reinterpret_cast<const unsigned*>(s));
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) tpf_finish_call(ctl, e);
}

}  // namespace ex
