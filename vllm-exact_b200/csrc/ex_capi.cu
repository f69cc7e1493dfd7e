// C ABI of the vllm-exact B200 library (declarations and contracts: include/vllm_exact_b200.h).
//
// The whole library is one translation unit (this file includes the kernel headers) so that every kernel shares the
// single device error word g_ex_dev_error. Every entry point validates its arguments before launching anything,
// never allocates device memory and never synchronizes the host.
#include <cstring>
#include <mutex>
#include <string>

#include "ex_common.cuh"
#include "ex_tp_fused.cuh"
#include "ex_digitize.cuh"
#include "ex_gemm_simt.cuh"
#include "ex_gemm_tc.cuh"
#include "ex_paged_decode.cuh"
#include "ex_paged_decode_tma.cuh"

// Split-K scratch of ex_linear_noalloc: a file-scope device array, so that entry point never allocates. Host code
// must not hand this symbol to a kernel (on the host it is only a stand-in); the device address is looked up once per
// device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_ex_noalloc_scratch[EX_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string g_last_error;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return EX_OK;
  g_last_error = cudaGetErrorString(e);
  return EX_ERR_CUDA;
}

bool dtype_ok(int d) { return d == EX_DTYPE_F32 || d == EX_DTYPE_BF16 || d == EX_DTYPE_F16; }
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = v;
    else
      sms = 148;
  }
  return sms;
}

// ---------------------------------------------------------------------------------------------------------------
// SIMT plan: row blocks of 256 weight rows, K split so that there are about two CTAs per SM.
// ---------------------------------------------------------------------------------------------------------------
struct SimtPlan {
  int splits;
  int kchunk;
  int nblocks;
  size_t ws_bytes;
};

SimtPlan simt_plan(int64_t M, int64_t N, int64_t K, int split_k) {
  SimtPlan p;
  p.nblocks = (int)cdiv(N, ex::SIMT_THREADS);
  int s = split_k;
  if (s <= 0) {
    const int target = 2 * num_sms();
    s = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(target, p.nblocks), K / 256));
  }
  s = (int)std::max<int64_t>(1, std::min<int64_t>(s, std::max<int64_t>(1, cdiv(K, 16))));
  p.kchunk = (int)std::max<int64_t>(16, align_up((size_t)cdiv(K, s), 16));
  p.splits = K > 0 ? (int)cdiv(K, p.kchunk) : 1;
  p.ws_bytes = p.splits > 1 ? align_up((size_t)p.nblocks * 4, 256) + (size_t)M * N * 8 : 0;
  return p;
}

template <int F, bool TRUNC, int OD, bool PARTIAL>
cudaError_t launch_simt_t(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
                          const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw,
                          int M, int N, int K, const SimtPlan& p, void* out, int64_t ldo, void* ws, cudaStream_t st) {
  const bool vecw = (ldw % 16 == 0) && (reinterpret_cast<uintptr_t>(wh) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(wl) % 16 == 0);
  int* cnt = reinterpret_cast<int*>(ws);
  long long* acc = p.splits > 1 ? reinterpret_cast<long long*>(reinterpret_cast<char*>(ws) +
                                                               align_up((size_t)p.nblocks * 4, 256))
                                 : nullptr;
  dim3 grid(p.nblocks, p.splits);
  ex::k_exact_simt<F, TRUNC, OD, PARTIAL><<<grid, ex::SIMT_THREADS, 0, st>>>(
      xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, M, N, K, p.kchunk, vecw, out, ldo, acc, cnt);
  return cudaGetLastError();
}

template <bool PARTIAL>
cudaError_t launch_simt(int F, int trunc, int od, const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx,
                        const int32_t* sx, const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw,
                        const int32_t* sw, int M, int N, int K, const SimtPlan& p, void* out, int64_t ldo, void* ws,
                        cudaStream_t st) {
#define EX_SIMT_CASE(FF, TT, OO)                                                                              \
  if (F == FF && (trunc != 0) == TT && (PARTIAL || od == OO))                                                 \
    return launch_simt_t<FF, TT, OO, PARTIAL>(xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, M, N, K, p, out, ldo, \
                                              ws, st);
  EX_SIMT_CASE(14, true, EX_DTYPE_BF16)
  EX_SIMT_CASE(14, true, EX_DTYPE_F32)
  EX_SIMT_CASE(14, true, EX_DTYPE_F16)
  EX_SIMT_CASE(14, false, EX_DTYPE_BF16)
  EX_SIMT_CASE(14, false, EX_DTYPE_F32)
  EX_SIMT_CASE(14, false, EX_DTYPE_F16)
  EX_SIMT_CASE(15, true, EX_DTYPE_BF16)
  EX_SIMT_CASE(15, true, EX_DTYPE_F32)
  EX_SIMT_CASE(15, true, EX_DTYPE_F16)
  EX_SIMT_CASE(15, false, EX_DTYPE_BF16)
  EX_SIMT_CASE(15, false, EX_DTYPE_F32)
  EX_SIMT_CASE(15, false, EX_DTYPE_F16)
#undef EX_SIMT_CASE
  return cudaErrorInvalidValue;
}

// Shared argument validation of ex_linear / ex_linear_partial_i64.
int check_linear_args(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int8_t* wh,
                      const int8_t* wl, int64_t ldw, const int32_t* cw, int64_t M, int64_t N, int64_t K, int F,
                      const void* out, int64_t ldo) {
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX) return EX_ERR_ARG;
  if (K > ex::EX_MAX_K) return EX_ERR_UNSUPPORTED;
  if (F != 14 && F != 15) return EX_ERR_ARG;
  if (M == 0 || N == 0) return EX_OK;
  if (!out || ldo < N) return EX_ERR_ARG;
  if (K > 0 && (!xh || !xl || !wh || !wl || ldx < K || ldw < K)) return EX_ERR_ARG;
  if (F == 15 && (!cx || !cw)) return EX_ERR_ARG;
  return EX_OK;
}

// Algorithm choice for EX_ALGO_AUTO: the tcgen05 int8 kernel whenever its TMA alignment rules hold, else SIMT.
int pick_algo(int algo, const int8_t* xh, const int8_t* xl, int64_t ldx, const int8_t* wh, const int8_t* wl,
              int64_t ldw, int64_t M, int64_t N, int64_t K) {
  if (algo != EX_ALGO_AUTO) return algo;
  if (ex::tc_supported(xh, xl, ldx, wh, wl, ldw, M, N, K)) return EX_ALGO_TC_I8;
  return EX_ALGO_SIMT;
}

template <bool PARTIAL>
int linear_impl(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
                const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw, int64_t M,
                int64_t N, int64_t K, int F, int trunc, void* out, int out_dtype, int64_t ldo, void* workspace,
                size_t workspace_bytes, int split_k, int algo, cudaStream_t st) {
  int rc = check_linear_args(xh, xl, ldx, cx, wh, wl, ldw, cw, M, N, K, F, out, ldo);
  if (rc != EX_OK || M == 0 || N == 0) return rc;
  if (!PARTIAL && (!sx || !sw)) return EX_ERR_ARG;
  if (!PARTIAL && !dtype_ok(out_dtype)) return EX_ERR_DTYPE;
  if (split_k < 0) return EX_ERR_ARG;
  const bool static_w = (algo & EX_LINEAR_STATIC_WEIGHTS) != 0;
  algo = pick_algo(algo & ~EX_LINEAR_STATIC_WEIGHTS, xh, xl, ldx, wh, wl, ldw, M, N, K);
  if (algo == EX_ALGO_SIMT) {
    const SimtPlan p = simt_plan(M, N, K, split_k);
    if (p.ws_bytes > 0 && (!workspace || workspace_bytes < p.ws_bytes)) return EX_ERR_WORKSPACE;
    if (p.ws_bytes > 0 && reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return EX_ERR_ALIGN;
    return cuda_status(launch_simt<PARTIAL>(F, trunc, out_dtype, xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, (int)M,
                                            (int)N, (int)K, p, out, ldo, workspace, st));
  }
  if (algo == EX_ALGO_TC_I8) {
    if (!ex::tc_supported(xh, xl, ldx, wh, wl, ldw, M, N, K)) return EX_ERR_ALIGN;
    const ex::TcPlan p = ex::tc_plan(M, N, K, split_k, num_sms(), ex::tc_cluster_cap());
    if (p.ws_bytes > 0 && (!workspace || workspace_bytes < p.ws_bytes)) return EX_ERR_WORKSPACE;
    if (p.ws_bytes > 0 && reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return EX_ERR_ALIGN;
    cudaError_t e = ex::launch_tc<PARTIAL>(p, F, trunc, out_dtype, xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, (int)M,
                                           (int)N, (int)K, out, ldo, workspace, static_w, st);
    if (e == cudaErrorNotSupported) return EX_ERR_UNSUPPORTED;
    return cuda_status(e);
  }
  return EX_ERR_ARG;
}

// Per-device address of g_ex_noalloc_scratch, looked up (and the array cleared) on the first call on each device.
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[128] = {};

int noalloc_scratch(cudaStream_t st, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 128) return EX_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ex_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaMemsetAsync(p, 0, EX_NOALLOC_SCRATCH_BYTES, st);  // split-K slots and tickets must start at zero
    if (e != cudaSuccess) return cuda_status(e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return EX_OK;
}

// Clears the scratch of every device that has used it (synchronously, each with its own device current). A call
// that stopped early on a timed-out wait can leave split-K partials and tickets behind; ex_device_error() calls this
// whenever it reports such an error, so later calls start from zero again.
int noalloc_clear_all() {
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_status(e);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  int rc = EX_OK;
  for (int d = 0; d < 128; ++d) {
    if (!g_noalloc_ptr[d]) continue;
    if ((e = cudaSetDevice(d)) == cudaSuccess) e = cudaMemset(g_noalloc_ptr[d], 0, EX_NOALLOC_SCRATCH_BYTES);
    if (e != cudaSuccess && rc == EX_OK) rc = cuda_status(e);
  }
  e = cudaSetDevice(cur);
  if (e != cudaSuccess && rc == EX_OK) rc = cuda_status(e);
  return rc;
}

// 4-D tensor map over a paged K or V cache: (head dim, KV head, offset in page, page), 16-token x 64-dim boxes.
bool encode_kv_map(CUtensorMap* map, const void* base, int D, int KV, int BS, int64_t num_blocks, int64_t s_head,
                   int64_t s_page, int64_t s_block) {
  ex::PFN_encodeTiled enc = ex::get_encode_fn();
  if (!enc || reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)KV, (cuuint64_t)BS, (cuuint64_t)num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)s_head * 2, (cuuint64_t)s_page * 2, (cuuint64_t)s_block * 2};
  cuuint32_t box[4] = {64, 1, 16, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_merge(const float* ws_m, const float* ws_l, const float* ws_acc, void* out, int64_t so_t, int64_t so_h,
                 int n, int H, int NS, int D, int out_dtype, const int32_t* seq_lens, int split, const int32_t* qsl,
                 cudaStream_t st) {
  const int mthreads = std::min(D, 256);
  const dim3 mg(n * H), mb(mthreads);
  cudaError_t e;
  if (out_dtype == EX_DTYPE_BF16)
    e = ex_launch_pdl(ex::k_paged_merge<EX_DTYPE_BF16>, mg, mb, 0, st, ws_m, ws_l, ws_acc, out, so_t, so_h, H, NS, D,
                      seq_lens, split, qsl);
  else if (out_dtype == EX_DTYPE_F16)
    e = ex_launch_pdl(ex::k_paged_merge<EX_DTYPE_F16>, mg, mb, 0, st, ws_m, ws_l, ws_acc, out, so_t, so_h, H, NS, D,
                      seq_lens, split, qsl);
  else
    e = ex_launch_pdl(ex::k_paged_merge<EX_DTYPE_F32>, mg, mb, 0, st, ws_m, ws_l, ws_acc, out, so_t, so_h, H, NS, D,
                      seq_lens, split, qsl);
  if (e != cudaSuccess) return cuda_status(e);
  return cuda_status(cudaGetLastError());
}

size_t linear_ws(int64_t M, int64_t N, int64_t K, int split_k, int algo) {
  if (M <= 0 || N <= 0) return 0;
  algo &= ~EX_LINEAR_STATIC_WEIGHTS;
  size_t a = simt_plan(M, N, K, split_k).ws_bytes;
  if (algo == EX_ALGO_SIMT) return a;
  const size_t b = ex::tc_plan(M, N, K, split_k, num_sms(), ex::tc_cluster_cap()).ws_bytes;
  if (algo == EX_ALGO_TC_I8) return b;
  return std::max(a, b);  // automatic choice: enough for either algorithm
}

}  // namespace

extern "C" {

const char* ex_version(void) { return "vllm-exact-b200 0.1.0 (sm_100a)"; }

const char* ex_status_string(int s) {
  switch (s) {
    case EX_OK: return "ok";
    case EX_ERR_ARG: return "invalid argument";
    case EX_ERR_ALIGN: return "misaligned pointer or leading dimension";
    case EX_ERR_WORKSPACE: return "workspace missing or too small";
    case EX_ERR_DTYPE: return "unsupported dtype";
    case EX_ERR_UNSUPPORTED: return "unsupported shape or algorithm";
    case EX_ERR_CUDA: return "CUDA error";
    case EX_ERR_DEVICE: return "device-side bounded wait timed out";
    default: return "unknown status";
  }
}

const char* ex_last_error_string(void) { return g_last_error.c_str(); }

int ex_device_error(int* code) {
  if (!code) return EX_ERR_ARG;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_ex_dev_error, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e);
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_ex_dev_error, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e);
  *code = v;
  if (v != 0) return noalloc_clear_all();  // a stopped call may have left the static split-K scratch dirty
  return EX_OK;
}

int ex_digitize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F, int8_t* h, int8_t* l,
                int64_t ldd, int32_t* cs, int32_t* sh, void* stream) {
  if (rows < 0 || K < 0 || rows > INT32_MAX || K > INT32_MAX) return EX_ERR_ARG;
  if (F != 14 && F != 15) return EX_ERR_ARG;
  if (!dtype_ok(x_dtype)) return EX_ERR_DTYPE;
  if (rows == 0) return EX_OK;
  if (!cs || !sh) return EX_ERR_ARG;
  if (K > 0 && (!x || !h || !l || ldx < K || ldd < K)) return EX_ERR_ARG;
  return cuda_status(
      ex::launch_digitize<ex::DIG_LOCAL>(x, x_dtype, ldx, rows, K, F, h, l, ldd, cs, sh, nullptr, (cudaStream_t)stream));
}

int ex_row_absmax(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, float* amax, void* stream) {
  if (rows < 0 || K < 0 || rows > INT32_MAX || K > INT32_MAX) return EX_ERR_ARG;
  if (!dtype_ok(x_dtype)) return EX_ERR_DTYPE;
  if (rows == 0) return EX_OK;
  if (!amax || (K > 0 && (!x || ldx < K))) return EX_ERR_ARG;
  return cuda_status(ex::launch_digitize<ex::DIG_ABSMAX>(x, x_dtype, ldx, rows, K, 14, nullptr, nullptr, K, nullptr,
                                                         nullptr, amax, (cudaStream_t)stream));
}

int ex_digitize_given_absmax(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F,
                             const float* amax, int8_t* h, int8_t* l, int64_t ldd, int32_t* cs, int32_t* sh,
                             void* stream) {
  if (rows < 0 || K < 0 || rows > INT32_MAX || K > INT32_MAX) return EX_ERR_ARG;
  if (F != 14 && F != 15) return EX_ERR_ARG;
  if (!dtype_ok(x_dtype)) return EX_ERR_DTYPE;
  if (rows == 0) return EX_OK;
  if (!cs || !sh || !amax) return EX_ERR_ARG;
  if (K > 0 && (!x || !h || !l || ldx < K || ldd < K)) return EX_ERR_ARG;
  return cuda_status(ex::launch_digitize<ex::DIG_GIVEN>(x, x_dtype, ldx, rows, K, F, h, l, ldd, cs, sh,
                                                        const_cast<float*>(amax), (cudaStream_t)stream));
}

size_t ex_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int split_k, int algo) {
  return linear_ws(M, N, K, split_k, algo);
}

int ex_linear(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
              const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw, int64_t M,
              int64_t N, int64_t K, int F, int trunc, void* out, int out_dtype, int64_t ldo, void* workspace,
              size_t workspace_bytes, int split_k, int algo, void* stream) {
  return linear_impl<false>(xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, M, N, K, F, trunc, out, out_dtype, ldo,
                            workspace, workspace_bytes, split_k, algo, (cudaStream_t)stream);
}

int ex_linear_noalloc(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
                      const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw,
                      int64_t M, int64_t N, int64_t K, int F, int trunc, void* out, int out_dtype, int64_t ldo,
                      int split_k, int algo, void* stream) {
  int rc = check_linear_args(xh, xl, ldx, cx, wh, wl, ldw, cw, M, N, K, F, out, ldo);
  if (rc != EX_OK || M == 0 || N == 0) return rc;
  if (split_k < 0) return EX_ERR_ARG;
  const int chosen = pick_algo(algo & ~EX_LINEAR_STATIC_WEIGHTS, xh, xl, ldx, wh, wl, ldw, M, N, K);
  size_t need = 0;
  if (chosen == EX_ALGO_SIMT)
    need = simt_plan(M, N, K, split_k).ws_bytes;
  else if (chosen == EX_ALGO_TC_I8 && ex::tc_supported(xh, xl, ldx, wh, wl, ldw, M, N, K))
    need = ex::tc_plan(M, N, K, split_k, num_sms(), ex::tc_cluster_cap()).ws_bytes;
  if (need > EX_NOALLOC_SCRATCH_BYTES) {
    g_last_error = "ex_linear_noalloc: this shape's split-K plan needs " + std::to_string(need) +
                   " bytes of scratch, more than the static EX_NOALLOC_SCRATCH_BYTES (" +
                   std::to_string((size_t)EX_NOALLOC_SCRATCH_BYTES) + ")";
    return EX_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  rc = noalloc_scratch((cudaStream_t)stream, &scratch);
  if (rc != EX_OK) return rc;
  return linear_impl<false>(xh, xl, ldx, cx, sx, wh, wl, ldw, cw, sw, M, N, K, F, trunc, out, out_dtype, ldo, scratch,
                            EX_NOALLOC_SCRATCH_BYTES, split_k, algo, (cudaStream_t)stream);
}

int ex_linear_noalloc_reset(void* stream) {
  void* scratch = nullptr;
  const int rc = noalloc_scratch((cudaStream_t)stream, &scratch);
  if (rc != EX_OK) return rc;
  return cuda_status(cudaMemsetAsync(scratch, 0, EX_NOALLOC_SCRATCH_BYTES, (cudaStream_t)stream));
}

int ex_linear_noalloc_fill_scratch(int byte_value, void* stream) {
  if (byte_value < 0 || byte_value > 255) return EX_ERR_ARG;
  void* scratch = nullptr;
  const int rc = noalloc_scratch((cudaStream_t)stream, &scratch);
  if (rc != EX_OK) return rc;
  return cuda_status(cudaMemsetAsync(scratch, byte_value, EX_NOALLOC_SCRATCH_BYTES, (cudaStream_t)stream));
}

int ex_linear_partial_i64(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int8_t* wh,
                          const int8_t* wl, int64_t ldw, const int32_t* cw, int64_t M, int64_t N, int64_t K, int F,
                          int trunc, int64_t* tot, int64_t ldt, void* workspace, size_t workspace_bytes, int split_k,
                          int algo, void* stream) {
  return linear_impl<true>(xh, xl, ldx, cx, nullptr, wh, wl, ldw, cw, nullptr, M, N, K, F, trunc, tot,
                           EX_DTYPE_F32, ldt, workspace, workspace_bytes, split_k, algo, (cudaStream_t)stream);
}

int ex_epilogue_i64(const int64_t* tot, int64_t ldt, const int32_t* sx, const int32_t* sw, int64_t M, int64_t N,
                    void* out, int out_dtype, int64_t ldo, void* stream) {
  if (M < 0 || N < 0 || M > INT32_MAX || N > INT32_MAX) return EX_ERR_ARG;
  if (!dtype_ok(out_dtype)) return EX_ERR_DTYPE;
  if (M == 0 || N == 0) return EX_OK;
  if (!tot || !sx || !sw || !out || ldt < N || ldo < N) return EX_ERR_ARG;
  const int64_t total = M * N;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>(cdiv(total, threads), 16 * (int64_t)num_sms());
  cudaStream_t st = (cudaStream_t)stream;
  const long long* t = reinterpret_cast<const long long*>(tot);
  if (out_dtype == EX_DTYPE_F32)
    ex::k_epilogue_i64<EX_DTYPE_F32><<<blocks, threads, 0, st>>>(t, ldt, sx, sw, (int)M, (int)N, out, ldo);
  else if (out_dtype == EX_DTYPE_BF16)
    ex::k_epilogue_i64<EX_DTYPE_BF16><<<blocks, threads, 0, st>>>(t, ldt, sx, sw, (int)M, (int)N, out, ldo);
  else
    ex::k_epilogue_i64<EX_DTYPE_F16><<<blocks, threads, 0, st>>>(t, ldt, sx, sw, (int)M, (int)N, out, ldo);
  return cuda_status(cudaGetLastError());
}

int ex_ipc_get_handle(const void* dev_ptr, unsigned char* handle, uint64_t* offset) {
  if (!dev_ptr || !handle || !offset) return EX_ERR_ARG;
  typedef CUresult (*PFN_range)(CUdeviceptr*, size_t*, CUdeviceptr);
  static PFN_range range_fn = nullptr;
  if (!range_fn) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fp, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return EX_ERR_UNSUPPORTED;
    range_fn = reinterpret_cast<PFN_range>(fp);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return EX_ERR_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_status(e);
  static_assert(sizeof(h) == EX_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return EX_OK;
}

int ex_ipc_open_handle(const unsigned char* handle, void** base) {
  if (!handle || !base) return EX_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
}

int ex_ipc_close_handle(void* base) {
  if (!base) return EX_ERR_ARG;
  return cuda_status(cudaIpcCloseMemHandle(base));
}

int ex_tp_digitize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F, const void* xch,
                   int64_t max_rows, int32_t* ctl, int rank, int world, int8_t* h, int8_t* l, int64_t ldd, int32_t* cs,
                   int32_t* sh, void* stream) {
  if (rows < 0 || K < 0 || rows > INT32_MAX || K > INT32_MAX || max_rows > INT32_MAX) return EX_ERR_ARG;
  if (F != 14 && F != 15) return EX_ERR_ARG;
  if (!dtype_ok(x_dtype)) return EX_ERR_DTYPE;
  if (world < 1 || world > ex::TPF_MAX_WORLD || rank < 0 || rank >= world) return EX_ERR_ARG;
  if (!xch || !ctl || rows > max_rows) return EX_ERR_ARG;
  if (rows == 0) return EX_OK;  // every rank makes the same call, so every rank skips it
  if (!cs || !sh || (K > 0 && (!x || !h || !l || ldx < K || ldd < K))) return EX_ERR_ARG;
  // all blocks resident together (256 threads, no dynamic shared memory): every wait is on other ranks only
  const int blocks = (int)std::min<int64_t>(rows, 4 * (int64_t)num_sms());
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long* const* xp = reinterpret_cast<unsigned long long* const*>(xch);
  cudaError_t e = cudaSuccess;
#define EX_TPD(T, FF)                                                                                              \
  e = ex_launch_pdl(ex::k_tp_digitize<T, FF>, dim3(blocks), dim3(ex::DIG_THREADS), 0, st,                          \
                    reinterpret_cast<const T*>(x), ldx, (int)rows, (int)K, xp, ctl, rank, world, (int)max_rows, h, l, \
                    ldd, cs, sh)
  if (x_dtype == EX_DTYPE_F32) {
    if (F == 15) EX_TPD(float, 15); else EX_TPD(float, 14);
  } else if (x_dtype == EX_DTYPE_BF16) {
    if (F == 15) EX_TPD(__nv_bfloat16, 15); else EX_TPD(__nv_bfloat16, 14);
  } else {
    if (F == 15) EX_TPD(__half, 15); else EX_TPD(__half, 14);
  }
#undef EX_TPD
  return cuda_status(e);
}

int ex_allreduce_epilogue_i64(const void* parts, int64_t ldt, const void* xch, const void* flags, int32_t* ctl,
                              int rank, int world, const int32_t* sx, const int32_t* sw, int64_t M, int64_t N,
                              void* out, int out_dtype, int64_t ldo, void* stream) {
  if (M < 0 || N < 0 || M > INT32_MAX || N > INT32_MAX) return EX_ERR_ARG;
  if (world < 1 || world > ex::TPF_MAX_WORLD || rank < 0 || rank >= world) return EX_ERR_ARG;
  if (!dtype_ok(out_dtype)) return EX_ERR_DTYPE;
  if (!parts || !xch || !flags || !ctl || !sx || !sw || !out || ldt < N || ldo < N) return EX_ERR_ARG;
  if (N % 2 != 0 || ldt % 2 != 0 || ldo % 2 != 0) return EX_ERR_ALIGN;  // column pairs: 16-byte partial loads
  // every rank takes part in every call, also for an empty output (one block then only exchanges the flags). The
  // block count depends on (M, N, world) only, so it is the same on every rank: block b pairs with block b of the
  // others; at most TPF_MAX_BLOCKS small blocks, all resident together.
  const int64_t pairs = M * cdiv(N, 2 * (int64_t)world);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(pairs, ex::TPF_THREADS), ex::TPF_MAX_BLOCKS));
  cudaStream_t st = (cudaStream_t)stream;
  const long long* const* pp = reinterpret_cast<const long long* const*>(parts);
  unsigned long long* const* xp = reinterpret_cast<unsigned long long* const*>(xch);
  int* const* fp = reinterpret_cast<int* const*>(flags);
  cudaError_t e;
#define EX_TPF_LAUNCH(OD)                                                                                        \
  e = ex_launch_pdl(ex::k_tp_allreduce_epilogue<OD>, dim3(blocks), dim3(ex::TPF_THREADS), 0, st, pp, ldt, xp, fp, \
                    ctl, rank, world, sx, sw, (int)M, (int)N, out, ldo)
  if (out_dtype == EX_DTYPE_F32)
    EX_TPF_LAUNCH(EX_DTYPE_F32);
  else if (out_dtype == EX_DTYPE_BF16)
    EX_TPF_LAUNCH(EX_DTYPE_BF16);
  else
    EX_TPF_LAUNCH(EX_DTYPE_F16);
#undef EX_TPF_LAUNCH
  return cuda_status(e);
}

size_t ex_paged_decode_workspace_bytes(int n, int H, int D, int max_len, int split) {
  if (n <= 0 || H <= 0 || D <= 0 || split <= 0) return 0;
  const int64_t NS = std::max<int64_t>(1, cdiv(max_len, split));
  const int64_t rows = (int64_t)n * H * NS;
  return align_up((size_t)rows * 4, 256) * 2 + (size_t)rows * D * 4;
}

int ex_paged_decode(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, const void* v_cache,
                    int64_t s_block, int64_t s_page, int64_t s_head, int64_t num_blocks, const int32_t* block_table,
                    int64_t sbt,
                    const int32_t* seq_lens, int n, int H, int KV, int D, int BS, float scale, int max_len, int split,
                    void* out, int64_t so_t, int64_t so_h, int out_dtype, void* workspace, size_t workspace_bytes,
                    void* stream) {
  return ex_paged_decode_leading(q, sq_t, sq_h, k_cache, v_cache, s_block, s_page, s_head, num_blocks, block_table,
                                 sbt, seq_lens, nullptr, n, H, KV, D, BS, scale, max_len, split, out, so_t, so_h,
                                 out_dtype, workspace, workspace_bytes, stream);
}

int ex_paged_decode_leading(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, const void* v_cache,
                            int64_t s_block, int64_t s_page, int64_t s_head, int64_t num_blocks,
                            const int32_t* block_table, int64_t sbt, const int32_t* seq_lens,
                            const int32_t* query_start_loc, int n, int H, int KV, int D, int BS, float scale,
                            int max_len, int split, void* out, int64_t so_t, int64_t so_h, int out_dtype,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0 || H <= 0 || KV <= 0 || H % KV != 0 || BS <= 0 || split <= 0 || max_len < 0) return EX_ERR_ARG;
  const int G = H / KV;
  if (G > 16) return EX_ERR_UNSUPPORTED;
  if (D != 64 && D != 128 && D != 256) return EX_ERR_UNSUPPORTED;
  if (!dtype_ok(out_dtype)) return EX_ERR_DTYPE;
  if (n == 0) return EX_OK;
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out) return EX_ERR_ARG;
  // 16-byte cp.async gathers and 4-byte query loads
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0 ||
      s_block % 8 != 0 || s_page % 8 != 0 || s_head % 8 != 0)
    return EX_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(q) % 4 != 0 || sq_t % 2 != 0 || sq_h % 2 != 0) return EX_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(query_start_loc) % 4 != 0) return EX_ERR_ALIGN;
  const size_t need = ex_paged_decode_workspace_bytes(n, H, D, max_len, split);
  if (!workspace || workspace_bytes < need) return EX_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return EX_ERR_ALIGN;
  const int NS = (int)std::max<int64_t>(1, cdiv(max_len, split));
  if (KV > 65535 || NS > 65535) return EX_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)n * H * NS;
  float* ws_m = reinterpret_cast<float*>(workspace);
  float* ws_l = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + align_up((size_t)rows * 4, 256));
  float* ws_acc = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + 2 * align_up((size_t)rows * 4, 256));
  cudaStream_t st = (cudaStream_t)stream;
  const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(q);
  const __nv_bfloat16* kp = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  const __nv_bfloat16* vp = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  dim3 grid(n, KV, NS);
  cudaError_t e = cudaSuccess;
  if (num_blocks <= 0) return EX_ERR_ARG;
  // TMA page-gather kernel for the common layouts; the cp.async kernel below handles everything else
  if ((D == 64 || D == 128) && G <= 8 && BS % 16 == 0 && split % ex::PT_BLK == 0 && ex::device_is_sm100()) {
    CUtensorMap mk, mv;
    if (encode_kv_map(&mk, k_cache, D, KV, BS, num_blocks, s_head, s_page, s_block) &&
        encode_kv_map(&mv, v_cache, D, KV, BS, num_blocks, s_head, s_page, s_block)) {
      const dim3 blk(ex::PT_THREADS);
#define EX_PT_LAUNCH(DD)                                                                                         \
  {                                                                                                              \
    const int smem = ex::PtCfg<DD>::SMEM;                                                                        \
    e = cudaFuncSetAttribute(ex::k_paged_tma<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);            \
    if (e == cudaSuccess)                                                                                        \
      e = ex_launch_pdl(ex::k_paged_tma<DD>, grid, blk, smem, st, mk, mv, qp, sq_t, sq_h, block_table, sbt,      \
                        seq_lens, query_start_loc, H, G, BS, scale, split, NS, ws_m, ws_l, ws_acc);              \
  }
      if (D == 64) EX_PT_LAUNCH(64)
      else EX_PT_LAUNCH(128)
#undef EX_PT_LAUNCH
      if (e != cudaSuccess) return cuda_status(e);
      return launch_merge(ws_m, ws_l, ws_acc, out, so_t, so_h, n, H, NS, D, out_dtype, seq_lens, split,
                        query_start_loc, st);
    }
  }
#define EX_PD_LAUNCH(DD)                                                                                         \
  {                                                                                                              \
    const int smem = ex::PdCfg<DD>::SMEM;                                                                        \
    e = cudaFuncSetAttribute(ex::k_paged_partial<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);        \
    if (e == cudaSuccess)                                                                                        \
      e = ex_launch_pdl(ex::k_paged_partial<DD>, grid, dim3(ex::PD_THREADS), smem, st, qp, sq_t, sq_h, kp, vp,   \
                        s_block, s_page, s_head, block_table, sbt, seq_lens, query_start_loc, H, G, BS, scale,   \
                        split, NS, ws_m, ws_l, ws_acc);                                                          \
  }
  if (D == 64) EX_PD_LAUNCH(64)
  else if (D == 128) EX_PD_LAUNCH(128)
  else EX_PD_LAUNCH(256)
#undef EX_PD_LAUNCH
  if (e != cudaSuccess) return cuda_status(e);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e);
  return launch_merge(ws_m, ws_l, ws_acc, out, so_t, so_h, n, H, NS, D, out_dtype, seq_lens, split,
                        query_start_loc, st);
}

}  // extern "C"
