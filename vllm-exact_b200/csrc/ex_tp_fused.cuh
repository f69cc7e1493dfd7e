// Fused all-reduce + exact epilogue of K-sharded partial totals over peer memory (tensor parallelism without NCCL
// on the data path). Replaces, for row-parallel layers, the int64 SUM all-reduce followed by the epilogue kernel
// (the reference has no multi-GPU path; the exactness argument is that of kernels.py:144-146, :159-177: integer
// partial totals of disjoint K slices add up exactly to the total of the whole K range).
//
// Every rank runs this kernel after writing its (M, N) int64 partial into a buffer the other GPUs can read (CUDA IPC
// mapping, plain loads over NVLink; no multicast object). Per rank: ctl[0] = epoch of the last completed call,
// ctl[1] = blocks of the current call that have finished; flags (every rank's array of 2*world int32) hold, per
// source rank p, the last epoch in which p's partial was ready (entry p) and in which p finished reading
// (entry world + p). One call, epoch e = ctl[0] + 1:
//   1. every block, thread 0: release store of e into ready[rank] of every rank's flags
//      (idempotent: no block depends on another block of this grid being scheduled), then a bounded wait until every
//      ready[p] of this rank's flags is >= e;
//   2. every thread: sum the world partials of its outputs (exact integers), apply the epilogue, store;
//   3. the last block to finish: release store of e into done[rank] of every rank's flags, bounded wait until every
//      done[p] here is >= e (every rank has finished reading this rank's partial), then ctl = {e, 0}.
// So when the kernel completes, this rank's partial buffer may be overwritten by the next work on the stream, and
// the epoch lives on the device: the call can be captured in a CUDA graph and replayed. A wait that runs out records
// EX_DEVERR_WAIT_PEER and the kernel finishes without writing the outputs of the blocks concerned.
#pragma once
#include "ex_common.cuh"

namespace ex {

constexpr int TPF_THREADS = 256;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until flags[first + p] >= e for every p < world. Returns false (and records the error) on timeout.
__device__ __forceinline__ bool tpf_wait_all(const int* f, int first, int world, int e) {
  const uint64_t t0 = ex_globaltimer();
  for (int p = 0; p < world; ++p) {
    for (uint32_t it = 0;; ++it) {
      if (ld_acquire_sys(f + first + p) >= e) break;
      if ((it & 63u) == 63u) {
        const uint64_t dt = ex_globaltimer() - t0;
        if (dt > EX_WAIT_TIMEOUT_NS || (dt > 1000000ull && *(volatile int*)&g_ex_dev_error != 0)) {
          ex_set_error(EX_DEVERR_WAIT_PEER);
          return false;
        }
      }
    }
  }
  return true;
}

template <int OUT_DTYPE>
__global__ void __launch_bounds__(TPF_THREADS) k_allreduce_epilogue_i64(
    const long long* const* __restrict__ parts, int64_t ldt, int* const* __restrict__ flags, int* ctl, int rank,
    int world, const int32_t* __restrict__ sx, const int32_t* __restrict__ sw, int M, int N, void* __restrict__ out,
    int64_t ldo) {
  __shared__ int ok, ep;
  if (threadIdx.x == 0) {
    const int e = *(volatile int*)ctl + 1;
    ep = e;
    // This rank's partial was written by the preceding kernel on the stream, which has completed; peers read it
    // through this GPU's L2, so the release stores order it before the ready flags.
    for (int p = 0; p < world; ++p) st_release_sys(flags[p] + rank, e);
    ok = tpf_wait_all(flags[rank], 0, world, e) ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    const int64_t total = (int64_t)M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int m = (int)(i / N), n = (int)(i % N);
      const int64_t off = (int64_t)m * ldt + n;
      long long tot = 0;
      for (int p = 0; p < world; ++p) tot += __ldcv(parts[p] + off);  // volatile: peer memory, never stale
      ex_store_out<OUT_DTYPE>(out, (int64_t)m * ldo + n, ex_scale_to_f32(tot, sx[m], sw[n]));
    }
  }
  __syncthreads();  // every thread of this block has finished reading the partials
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctl + 1, 1) == (int)gridDim.x - 1) {  // last block of this rank's grid
      const int e = ep;
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(flags[p] + world + rank, e);
      tpf_wait_all(flags[rank], world, world, e);  // every rank has finished reading this rank's partial
      ctl[1] = 0;
      *(volatile int*)ctl = e;
    }
  }
}

}  // namespace ex
