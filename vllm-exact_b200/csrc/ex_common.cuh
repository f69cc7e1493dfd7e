// Common device helpers for the vllm-exact B200 library: status codes, the device error word, numeric helpers of
// the exact epilogue, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05 (sm_100a).
//
// Every spin-wait in this library is bounded: after EX_WAIT_TIMEOUT_NS of global time the waiting thread records
// an error in g_ex_dev_error and gives up, so a broken pipeline ends with an error status instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "vllm_exact_b200.h"

#define EX_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate in-kernel wait

// Device error word. 0 = fine; otherwise the code of the first failure (EX_DEVERR_*). Read and cleared by the host
// through ex_device_error().
__device__ int g_ex_dev_error;

enum {
  EX_DEVERR_NONE = 0,
  EX_DEVERR_WAIT_TMA = 1,      // a consumer gave up waiting for a TMA load
  EX_DEVERR_WAIT_SLOT = 2,     // the producer gave up waiting for a free pipeline slot
  EX_DEVERR_WAIT_MMA = 3,      // the epilogue gave up waiting for the accumulator
  EX_DEVERR_WAIT_TMEM = 4,     // the MMA warp gave up waiting for the epilogue to release TMEM
  EX_DEVERR_TMEM_ALLOC = 5,    // TMEM allocation returned an unexpected address
  EX_DEVERR_WAIT_PEER = 6,     // a rank of the fused tensor-parallel epilogue gave up waiting for a peer's partial
};

__device__ __forceinline__ void ex_set_error(int code) { atomicCAS(&g_ex_dev_error, 0, code); }

__device__ __forceinline__ uint64_t ex_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------------------------
// Exact epilogue numerics (reference kernels.py:98-100 and :154-157):
//   y = float32( float64(tot) * 2^-(sx+sw) ), the power of two built from float64 bits with int64 arithmetic.
// int64 -> float64 is exact (|tot| < 2^53), the product by a power of two is exact, float64 -> float32 rounds once
// to nearest even. A bf16/fp16 output then rounds once more from that float32 (the reference's double rounding).
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex_scale_to_f32(long long tot, int sx, int sw) {
  long long e = -((long long)sx + (long long)sw);
  unsigned long long bits = ((unsigned long long)(e + 1023)) << 52;
  double scale = __longlong_as_double((long long)bits);
  return __double2float_rn(__dmul_rn(__ll2double_rn(tot), scale));
}

template <int OUT_DTYPE>
__device__ __forceinline__ void ex_store_out(void* out, long long idx, float v) {
  if constexpr (OUT_DTYPE == EX_DTYPE_F32) {
    reinterpret_cast<float*>(out)[idx] = v;
  } else if constexpr (OUT_DTYPE == EX_DTYPE_BF16) {
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  }
}

// Integer total of the two-digit product plus the F=15 offset correction (reference kernels.py:93-97, :143, :148-151).
__device__ __forceinline__ long long ex_combine(int hh, int md, int ll) {
  return ((long long)hh << 16) + ((long long)md << 8) + (long long)ll;
}

// ------------------------------------------------------------------------------------------------------------------
// shared-memory address helpers
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ex_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(ex_smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(ex_smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   ex_smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(ex_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records `code`) if the phase did not complete within
// EX_WAIT_TIMEOUT_NS. Once any thread has recorded an error the others give up quickly too.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ex_globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      const uint64_t dt = ex_globaltimer() - t0;
      if (dt > EX_WAIT_TIMEOUT_NS) {
        ex_set_error(code);
        return false;
      }
      if (dt > 1000000ull && *(volatile int*)&g_ex_dev_error != 0) return false;  // someone else already failed
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), tiled 2D loads into this CTA's shared memory, completion counted on an mbarrier.
// Every tensor load of this library writes only the issuing CTA's shared memory (no multicast form is used).
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
      "[%2], %5;" ::"r"(ex_smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(ex_smem_u32(bar)), "r"(c0), "r"(c1), "l"(cache_hint)
      : "memory");
}

// Prefetch a tile into L2 only (no shared-memory write). L2 is coherent with every writer, so this is safe even
// before griddepcontrol.wait.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// Programmatic dependent launch: wait until the preceding kernel in the stream has completed and its memory is
// visible (no-op when launched without the attribute), and allow the next kernel to begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 cache-policy hints (createpolicy): weights are streamed once, activations are re-read by every CTA.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, tensor memory)
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ex_smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once all tcgen05.mma previously issued by this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(ex_smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, both operands K-major.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread (thread i of the warp reads TMEM lane base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile in the 128-byte swizzled layout written by TMA
// (CU_TENSOR_MAP_SWIZZLE_128B): rows of 128 bytes, 8-row atoms of 1024 bytes. Fields (sm_100 UMMA descriptor):
// start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30) (unused for swizzled K-major; 16 bytes),
// stride byte offset >> 4 in [32,46) (1024 bytes between 8-row atoms), version 1 in [46,48), base offset 0,
// layout type 2 (128-byte swizzle) in [61,64). The tile must start on a 1024-byte boundary; stepping along K inside
// the 128-byte row is done by adding the byte offset to the start address.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)(16 >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8 (sm_100): D format in bits [4,6) (2 = s32), A and B formats in
// [7,10) and [10,13) (1 = signed int8), A/B K-major (bits 15,16 = 0), N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t make_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred;
}

// ------------------------------------------------------------------------------------------------------------------
// thread-block clusters: rank, distributed shared memory, cluster-wide barrier
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address in the shared memory of cluster CTA `rank` of the variable at local shared address `addr`.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// (no memory clobber: these loads follow a cluster barrier, which orders them, and may overlap one another)
__device__ __forceinline__ long long dsmem_ld_s64(uint32_t addr) {
  long long v;
  asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void dsmem_ld_v2s64(uint32_t addr, long long& a, long long& b) {
  asm volatile("ld.shared::cluster.v2.s64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr) : "memory");
}

// Every thread of every CTA of the cluster arrives (release) and waits (acquire): shared-memory writes made before
// the barrier by any CTA of the cluster are visible to all of them after it. Not a software spin: the hardware
// completes it once all threads have arrived, so every thread must reach it exactly as often as the others.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// ------------------------------------------------------------------------------------------------------------------
// Launch with the programmatic-stream-serialization attribute: the kernel may start while the previous kernel in the
// stream is finishing; it must call pdl_wait() before touching memory that kernel produces or consumes.
// ------------------------------------------------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
static cudaError_t ex_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same launch as a grid of thread-block clusters of `cluster` CTAs along x (gridDim.x a multiple of it).
template <typename... KArgs, typename... Args>
static cudaError_t ex_launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster,
                                         cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------------------------------------------------------
// bulk (TMA-engine) reduce-add of a shared-memory buffer into global memory, tracked with bulk groups
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void bulk_reduce_add_u64(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.u64 [%0], [%1], %2;" ::"l"(gdst),
               "r"(ex_smem_u32(ssrc)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory source of all but the newest N bulk groups may be overwritten
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// every bulk group of this thread has completed (its global writes are performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ------------------------------------------------------------------------------------------------------------------
// int64 reduction into the split-K workspace: relaxed atomic add at L2. Integer addition is associative and
// commutative, so the final value does not depend on the order in which CTAs arrive.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void red_add_s64(long long* p, long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
