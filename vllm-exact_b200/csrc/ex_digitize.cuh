// Per-row fixed-point digitization (replaces kernels.py:46-85; semantics of digitize_torch, kernels.py:22-39).
//
// One CTA per row: a max-|x| reduction over the row, then the digits. Rows of up to 16384 aligned elements are held
// in registers between the two steps (k_digitize_reg); longer or unaligned rows are read twice (k_digitize, the
// second pass hits L1/L2). HBM traffic per row: K * sizeof(x) read + 2K bytes of digits + 8 bytes of cs/sh written.
#pragma once
#include "ex_common.cuh"

namespace ex {

constexpr int DIG_THREADS = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// frexp exponent of a >= 0 (a = m * 2^e, m in [0.5, 1)), subnormals included; 0 for a == 0 and for inf / NaN
// (kernels.py:26-27: e is forced to 0 where a is not > 0; glibc frexp returns 0 for inf).
__device__ __forceinline__ int frexp_exponent(float a) {
  const uint32_t bits = __float_as_uint(a);
  const uint32_t ex = (bits >> 23) & 0xFFu;
  const uint32_t man = bits & 0x7FFFFFu;
  if (!(a > 0.0f) || ex == 0xFFu) return 0;
  if (ex != 0) return (int)ex - 126;
  return -117 - __clz((int)man);  // subnormal: a = man * 2^-149, highest set bit p -> e = p - 148
}

// Load 8 consecutive elements as float (vectorised when the caller guarantees 16-byte alignment for T=bf16/f16
// or 32-byte alignment for float via two 16-byte loads).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
  } else {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < DIG_THREADS / 32 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ int block_sum_i32(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < DIG_THREADS / 32 ? red[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  return v;
}

template <int F>
__device__ __forceinline__ void digits_of(int q, int& h, int& l) {
  if constexpr (F == 15) {
    l = (q & 255) - 128;
    h = (q - l - 128) >> 8;
  } else {
    l = ((q + 128) & 255) - 128;
    h = (q - l) >> 8;
  }
}

// Modes of the digitizer kernel:
//   DIG_LOCAL    row maximum of this row (the reference's digitize)
//   DIG_GIVEN    row maximum supplied by the caller (amax_io[row]), e.g. the maximum over all K shards of a row
//   DIG_ABSMAX   only the row maximum, written to amax_io[row] (no digits)
enum { DIG_LOCAL = 0, DIG_GIVEN = 1, DIG_ABSMAX = 2 };

// VEC: rows are 16-byte aligned (32 for float), K % 8 == 0 and ldd % 8 == 0, so 8 elements move per access.
template <typename T, int F, bool VEC, int MODE>
__global__ void __launch_bounds__(DIG_THREADS) k_digitize(const T* __restrict__ x, int64_t ldx, int K,
                                                          int8_t* __restrict__ h, int8_t* __restrict__ l, int64_t ldd,
                                                          int32_t* __restrict__ cs, int32_t* __restrict__ sh,
                                                          float* __restrict__ amax_io) {
  __shared__ float redf[DIG_THREADS / 32];
  __shared__ int redi[DIG_THREADS / 32];
  // Let the consumer (the exact GEMM) start its prologue now: everything a kernel of this library does before its
  // own pdl_wait() is safe to overlap with this kernel. Then wait: the input comes from the previous kernel.
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  float amax = 0.0f;
  if constexpr (MODE == DIG_GIVEN) {
    amax = amax_io[row];
  } else if constexpr (VEC) {
    for (int k = threadIdx.x * 8; k < K; k += DIG_THREADS * 8) {
      float v[8];
      load8<T>(xr + k, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
  } else {
    for (int k = threadIdx.x; k < K; k += DIG_THREADS) amax = fmaxf(amax, fabsf(to_f32<T>(xr[k])));
  }
  if constexpr (MODE != DIG_GIVEN) amax = block_max(amax, redf);
  if constexpr (MODE == DIG_ABSMAX) {
    if (threadIdx.x == 0) amax_io[row] = amax;
    return;
  }
  const int e = frexp_exponent(amax);
  const int s = F - e;
  // 2^s built from float32 bits with int32 wrap-around, exactly as kernels.py:29
  const float scale = __uint_as_float(((uint32_t)(s + 127)) << 23);
  int csum = 0;
  int8_t* hr = h + row * ldd;
  int8_t* lr = l + row * ldd;
  if constexpr (VEC) {
    for (int k = threadIdx.x * 8; k < K; k += DIG_THREADS * 8) {
      float v[8];
      load8<T>(xr + k, v);
      uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = __float2int_rz(__fmul_rn(v[i], scale));
        int dh, dl;
        digits_of<F>(q, dh, dl);
        if constexpr (F == 15) csum += 256 * dh + dl;
        hw[i >> 2] |= ((uint32_t)(dh & 0xFF)) << (8 * (i & 3));
        lw[i >> 2] |= ((uint32_t)(dl & 0xFF)) << (8 * (i & 3));
      }
      *reinterpret_cast<uint2*>(hr + k) = make_uint2(hw[0], hw[1]);
      *reinterpret_cast<uint2*>(lr + k) = make_uint2(lw[0], lw[1]);
    }
  } else {
    for (int k = threadIdx.x; k < K; k += DIG_THREADS) {
      const int q = __float2int_rz(__fmul_rn(to_f32<T>(xr[k]), scale));
      int dh, dl;
      digits_of<F>(q, dh, dl);
      if constexpr (F == 15) csum += 256 * dh + dl;
      hr[k] = (int8_t)dh;
      lr[k] = (int8_t)dl;
    }
  }
  if constexpr (F == 15) csum = block_sum_i32(csum, redi);
  if (threadIdx.x == 0) {
    cs[row] = (F == 15) ? csum : 0;
    sh[row] = s;
  }
}

// Register-resident variant for rows of at most NV * 8 * DIG_THREADS elements (aligned as for VEC): every thread
// issues all of its loads before using any, the row maximum is reduced once, and the digits are made from the
// registers, so a row costs one global round trip instead of one per loop iteration in each of two passes. The
// digitizer sits between two GEMMs on the critical path of a decode step, where this latency is what counts.
template <typename T, int F, int NV, int MODE>
__global__ void __launch_bounds__(DIG_THREADS) k_digitize_reg(const T* __restrict__ x, int64_t ldx, int K,
                                                              int8_t* __restrict__ h, int8_t* __restrict__ l,
                                                              int64_t ldd, int32_t* __restrict__ cs,
                                                              int32_t* __restrict__ sh, float* __restrict__ amax_io) {
  __shared__ float redf[DIG_THREADS / 32];
  __shared__ int redi[DIG_THREADS / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  float v[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = (i * DIG_THREADS + (int)threadIdx.x) * 8;
    if (k < K) {
      load8<T>(xr + k, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.0f;
    }
  }
  float amax = 0.0f;
  if constexpr (MODE == DIG_GIVEN) {
    amax = amax_io[row];
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[i][e]));
    amax = block_max(amax, redf);
  }
  if constexpr (MODE == DIG_ABSMAX) {
    if (threadIdx.x == 0) amax_io[row] = amax;
    return;
  }
  const int s = F - frexp_exponent(amax);
  const float scale = __uint_as_float(((uint32_t)(s + 127)) << 23);  // 2^s, int32 wrap-around as kernels.py:29
  int csum = 0;
  int8_t* hr = h + row * ldd;
  int8_t* lr = l + row * ldd;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = (i * DIG_THREADS + (int)threadIdx.x) * 8;
    if (k >= K) continue;
    uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int q = __float2int_rz(__fmul_rn(v[i][e], scale));
      int dh, dl;
      digits_of<F>(q, dh, dl);
      if constexpr (F == 15) csum += 256 * dh + dl;
      hw[e >> 2] |= ((uint32_t)(dh & 0xFF)) << (8 * (e & 3));
      lw[e >> 2] |= ((uint32_t)(dl & 0xFF)) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(hr + k) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lr + k) = make_uint2(lw[0], lw[1]);
  }
  if constexpr (F == 15) csum = block_sum_i32(csum, redi);
  if (threadIdx.x == 0) {
    cs[row] = (F == 15) ? csum : 0;
    sh[row] = s;
  }
}

template <typename T, int F, int MODE>
static cudaError_t launch_digitize_t(const void* x, int64_t ldx, int64_t rows, int64_t K, int8_t* h, int8_t* l,
                                     int64_t ldd, int32_t* cs, int32_t* sh, float* amax_io, cudaStream_t st) {
  const T* xp = reinterpret_cast<const T*>(x);
  const size_t valign = sizeof(T) == 2 ? 16 : 32;
  const bool vec = (K % 8 == 0) && ((ldx * (int64_t)sizeof(T)) % (int64_t)valign == 0) &&
                   (reinterpret_cast<uintptr_t>(x) % valign == 0) &&
                   (MODE == DIG_ABSMAX || ((ldd % 8 == 0) && (reinterpret_cast<uintptr_t>(h) % 8 == 0) &&
                                           (reinterpret_cast<uintptr_t>(l) % 8 == 0)));
  dim3 grid((unsigned)rows);
  constexpr int64_t PER_NV = 8 * DIG_THREADS;  // elements per register vector slot across the CTA
#define EX_DIG_REG(NV)                                                                                              \
  return ex_launch_pdl(k_digitize_reg<T, F, NV, MODE>, grid, dim3(DIG_THREADS), 0, st, xp, ldx, (int)K, h, l, ldd, \
                       cs, sh, amax_io)
  if (vec && K <= 1 * PER_NV) EX_DIG_REG(1);
  if (vec && K <= 2 * PER_NV) EX_DIG_REG(2);
  if (vec && K <= 4 * PER_NV) EX_DIG_REG(4);
  if (vec && K <= 8 * PER_NV) EX_DIG_REG(8);
#undef EX_DIG_REG
  if (vec)
    return ex_launch_pdl(k_digitize<T, F, true, MODE>, grid, dim3(DIG_THREADS), 0, st, xp, ldx, (int)K, h, l, ldd, cs,
                         sh, amax_io);
  return ex_launch_pdl(k_digitize<T, F, false, MODE>, grid, dim3(DIG_THREADS), 0, st, xp, ldx, (int)K, h, l, ldd, cs,
                       sh, amax_io);
}

template <typename T, int MODE>
static cudaError_t launch_digitize_f(int F, const void* x, int64_t ldx, int64_t rows, int64_t K, int8_t* h,
                                     int8_t* l, int64_t ldd, int32_t* cs, int32_t* sh, float* amax_io,
                                     cudaStream_t st) {
  return F == 15 ? launch_digitize_t<T, 15, MODE>(x, ldx, rows, K, h, l, ldd, cs, sh, amax_io, st)
                 : launch_digitize_t<T, 14, MODE>(x, ldx, rows, K, h, l, ldd, cs, sh, amax_io, st);
}

template <int MODE>
static cudaError_t launch_digitize(const void* x, int dtype, int64_t ldx, int64_t rows, int64_t K, int F, int8_t* h,
                                   int8_t* l, int64_t ldd, int32_t* cs, int32_t* sh, float* amax_io, cudaStream_t st) {
  if (dtype == EX_DTYPE_F32)
    return launch_digitize_f<float, MODE>(F, x, ldx, rows, K, h, l, ldd, cs, sh, amax_io, st);
  if (dtype == EX_DTYPE_BF16)
    return launch_digitize_f<__nv_bfloat16, MODE>(F, x, ldx, rows, K, h, l, ldd, cs, sh, amax_io, st);
  return launch_digitize_f<__half, MODE>(F, x, ldx, rows, K, h, l, ldd, cs, sh, amax_io, st);
}

}  // namespace ex
