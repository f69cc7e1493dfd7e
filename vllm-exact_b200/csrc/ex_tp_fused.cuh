// Tensor parallelism of the exact linear layer over peer memory: the two exchange steps of a row-parallel (K-sharded)
// layer, each one kernel over NVLink with plain peer loads and stores (CUDA IPC mappings; no multicast object, no
// NCCL on the data path). The reference has no multi-GPU path; exactness rests on its kernels.py:25-29 (a row's
// fixed-point scale comes from the maximum over the whole row) and :144-146, :159-177 (int64 partial totals of
// disjoint K slices add up exactly to the total of the whole K range).
//
// Both kernels move values as 64-bit words (call epoch << 32 | 32-bit payload) written with one relaxed system-scope
// store each: a reader polls its own copy until the word carries the current epoch, so a value and its "ready" signal
// arrive together and no fence or separate flag round trip is needed (a system-scope release or fence drains the
// writer's outstanding memory traffic; an earlier design with a release store per value and a system fence per block
// was slower than NCCL).
//
// k_tp_digitize: row maxima of this rank's K slice -> slot [epoch parity][rank][row] of every rank's exchange buffer
//   -> whole-row maxima -> digits of the slice. Safe for back-to-back calls on its own (two halves by epoch parity).
// k_tp_allreduce_epilogue: reduce-scatter + exact epilogue + all-gather of the int64 partial totals. Rank r owns the
//   output columns [r N / p, (r + 1) N / p) (rounded down to even): after one flag exchange saying every rank's
//   partial is complete, it sums the p partials of its columns (peer loads; integer addition is exact in any order),
//   applies the epilogue once, and stores the finished values as epoch words into every rank's output exchange buffer
//   (a bf16/fp16 column pair or one fp32 value per word). Each block then copies into `out` the words of its share of
//   every rank's columns, waiting for each word's epoch. Block b of every rank covers the same positions, so a block
//   only waits for the other ranks, never for another block of its own grid.
//
// Epochs live on the device (ctl words, advanced by the last block of each call), so calls can be captured in a CUDA
// graph and replayed. Every wait is bounded (EX_WAIT_TIMEOUT_NS): a wait that runs out records EX_DEVERR_WAIT_PEER
// and the kernel finishes without the missing data (wrong outputs, reported by ex_device_error).
// Buffer reuse: a peer writes epoch e + 1 words into this rank's buffers only after seeing this rank's "partial ready"
// flag of call e + 1, which this rank raises after its call e has read every epoch e word; and this rank's partial of
// call e is overwritten (by the GEMM of call e + 1) only after every rank's finished words of call e arrived, each of
// which a peer computed from the partials it had loaded.
#pragma once
#include "ex_common.cuh"
#include "ex_digitize.cuh"

namespace ex {

constexpr int TPF_THREADS = 256;
constexpr int TPF_MAX_BLOCKS = EX_TP_MAX_BLOCKS;  // blocks of k_tp_allreduce_epilogue
constexpr int TPF_MAX_WORLD = EX_TP_MAX_WORLD;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
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

// Bounded wait until the word at p carries epoch e; returns its payload (0 after a timeout, which is recorded).
__device__ __forceinline__ uint32_t tpf_wait_word(const unsigned long long* p, int e) {
  unsigned long long w = ld_relaxed_sys_u64(p);
  if ((int)(w >> 32) == e) return (uint32_t)w;
  const uint64_t t0 = ex_globaltimer();
  for (uint32_t it = 1;; ++it) {
    w = ld_relaxed_sys_u64(p);
    if ((int)(w >> 32) == e) return (uint32_t)w;
    if ((it & 63u) == 0) {
      const uint64_t dt = ex_globaltimer() - t0;
      if (dt > EX_WAIT_TIMEOUT_NS || (dt > 1000000ull && *(volatile int*)&g_ex_dev_error != 0)) {
        ex_set_error(EX_DEVERR_WAIT_PEER);
        return 0u;
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
  pdl_launch_dependents();  // the partial GEMM's prologue (and early weight loads) may start now
  pdl_wait();               // x comes from the previous kernel; ctl from this kernel's previous call
  if (threadIdx.x == 0) e_s = *(volatile int*)ctl + 1;
  __syncthreads();
  const int e = e_s;
  // Two halves of slots, by epoch parity: a rank can finish call e (it has every rank's call-e words) and write its
  // call e + 1 words before a slower rank has read call e's; they land in the other half. It cannot get to call
  // e + 2 (the same half again) before every rank has written its call e + 1 words, i.e. has finished call e.
  const int half = e & 1;
  // 1. maxima of this rank's slice of each row, to slot [rank][row] of every rank
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + (int64_t)row * ldx;
    float amax = 0.0f;
    for (int k = threadIdx.x; k < K; k += DIG_THREADS) amax = fmaxf(amax, fabsf(to_f32<T>(xr[k])));
    amax = block_max(amax, redf);
    if ((int)threadIdx.x < world) {
      const unsigned long long w = ((unsigned long long)(uint32_t)e << 32) | __float_as_uint(amax);
      st_relaxed_sys_u64(xch[threadIdx.x] + ((int64_t)half * world + rank) * max_rows + row, w);
    }
    __syncthreads();  // redf is reused by the next row's reduction
  }
  // 2. whole-row maxima from this rank's exchange buffer, then the digits of the slice
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    if (threadIdx.x < 32) {
      float v = 0.0f;
      if ((int)threadIdx.x < world)
        v = __uint_as_float(tpf_wait_word(xch[rank] + ((int64_t)half * world + threadIdx.x) * max_rows + row, e));
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
//   xch[p]    rank p's output exchange buffer of 64-bit words: word m * N / 2 + n / 2 holds the column pair (n, n + 1)
//             for 2-byte outputs, word m * N + n the column n for fp32 outputs
//   flags[p]  rank p's `world` int32 "partial ready" flags, entry q = last epoch in which rank q's partial was ready
//   ctl       this rank's int32 x 2 (epoch, block counter)
// Columns of rank r: [c0(r), c0(r + 1)), c0(r) = r * N / world rounded down to even; a thread takes a column pair.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ int tpf_col0(int r, int N, int world) { return (int)(((int64_t)r * N / world) & ~1ll); }

template <int OUT_DTYPE>
__device__ __forceinline__ uint32_t tpf_pack2(float a, float b) {
  if constexpr (OUT_DTYPE == EX_DTYPE_BF16) {
    const __nv_bfloat162 v = __halves2bfloat162(__float2bfloat16_rn(a), __float2bfloat16_rn(b));
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __halves2half2(__float2half_rn(a), __float2half_rn(b));
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <int OUT_DTYPE>
__global__ void __launch_bounds__(TPF_THREADS) k_tp_allreduce_epilogue(
    const long long* const* __restrict__ parts, int64_t ldt, unsigned long long* const* __restrict__ xch,
    int* const* __restrict__ flags, int* ctl, int rank, int world, const int32_t* __restrict__ sx,
    const int32_t* __restrict__ sw, int M, int N, void* __restrict__ out, int64_t ldo) {
  constexpr bool F32 = OUT_DTYPE == EX_DTYPE_F32;
  __shared__ int e_s, ok_s;
  const int b = blockIdx.x, B = gridDim.x;
  pdl_launch_dependents();
  pdl_wait();  // this rank's partial comes from the previous kernel (the partial GEMM)
  if (threadIdx.x == 0) {
    const int e = *(volatile int*)ctl + 1;
    e_s = e;
    // announce this rank's partial to every rank (every block stores the same value), then wait for every rank's
    for (int p = 0; p < world; ++p) st_release_sys(flags[p] + rank, e);
    int ok = 1;
    for (int p = 0; p < world && ok; ++p) ok = tpf_wait_flag(flags[rank] + p, e) ? 1 : 0;
    ok_s = ok;
  }
  __syncthreads();
  const int e = e_s;
  const unsigned long long tag = (unsigned long long)(uint32_t)e << 32;
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
      if constexpr (F32) {
        const int64_t w = (int64_t)m * N + n;
        for (int p = 0; p < world; ++p) {
          st_relaxed_sys_u64(xch[p] + w, tag | __float_as_uint(f0));
          st_relaxed_sys_u64(xch[p] + w + 1, tag | __float_as_uint(f1));
        }
      } else {
        const int64_t w = ((int64_t)m * N + n) >> 1;
        const unsigned long long word = tag | tpf_pack2<OUT_DTYPE>(f0, f1);
        for (int p = 0; p < world; ++p) st_relaxed_sys_u64(xch[p] + w, word);
      }
    }
    // 2. the words block b of every rank wrote into this rank's buffer (waiting for each) -> out
    for (int q = 0; q < world; ++q) {
      const int d0 = tpf_col0(q, N, world), d1 = tpf_col0(q + 1, N, world);
      const int qh = (d1 - d0) >> 1;
      const int64_t Q = (int64_t)M * qh;
      const int64_t q0 = Q * b / B, q1 = Q * (b + 1) / B;
      for (int64_t i = q0 + threadIdx.x; i < q1; i += TPF_THREADS) {
        const int m = (int)(i / qh), n = d0 + 2 * (int)(i % qh);
        if constexpr (F32) {
          const int64_t w = (int64_t)m * N + n;
          const uint32_t a0 = tpf_wait_word(xch[rank] + w, e), a1 = tpf_wait_word(xch[rank] + w + 1, e);
          *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + (int64_t)m * ldo + n) =
              make_float2(__uint_as_float(a0), __uint_as_float(a1));
        } else {
          const uint32_t v = tpf_wait_word(xch[rank] + (((int64_t)m * N + n) >> 1), e);
          *reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(out) + (int64_t)m * ldo + n) = v;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) tpf_finish_call(ctl, e);
}

}  // namespace ex
