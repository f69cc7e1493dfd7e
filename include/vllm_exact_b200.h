/*
 * vllm-exact B200 library: C ABI of the two hot paths of vllm-exact, built for sm_100a.
 *
 *   1. exact_int8 linear layer: fixed-point digitization + exact two-digit integer GEMM with fused epilogue;
 *   2. batch-invariant paged decode attention.
 *
 * Conventions (all entry points):
 *   - every pointer is caller-owned device memory; nothing here allocates device memory;
 *   - every call is asynchronous and stream-ordered on `stream` (a cudaStream_t; NULL = legacy default stream);
 *     no entry point synchronizes the host;
 *   - the return value is EX_OK or an EX_ERR_* status; bad arguments are reported before anything is launched;
 *   - strides / leading dimensions are in ELEMENTS of the tensor they describe;
 *   - split-K workspaces must be zero-filled once before first use; each call leaves them zero again.
 *     Calls that share a workspace must not overlap on the GPU (use one workspace per stream).
 *
 * Each entry point names the reference function it replaces (catoneone/vllm-exact, path:line).
 */
#ifndef VLLM_EXACT_B200_H
#define VLLM_EXACT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
enum {
  EX_OK = 0,
  EX_ERR_ARG = 1,         /* bad shape, mode or null pointer */
  EX_ERR_ALIGN = 2,       /* pointer or leading dimension not aligned as the chosen kernel requires */
  EX_ERR_WORKSPACE = 3,   /* workspace missing or smaller than the *_workspace_bytes() answer */
  EX_ERR_DTYPE = 4,       /* unsupported element type */
  EX_ERR_UNSUPPORTED = 5, /* requested algorithm cannot run this shape on this device */
  EX_ERR_CUDA = 6,        /* CUDA runtime error at launch; see ex_last_error_string() */
  EX_ERR_DEVICE = 7       /* a kernel reported a bounded wait that timed out (see ex_device_error) */
};

/* element types */
enum { EX_DTYPE_F32 = 0, EX_DTYPE_BF16 = 1, EX_DTYPE_F16 = 2 };

/* exact GEMM algorithms; all produce bit-identical results (other values are rejected with EX_ERR_ARG) */
enum {
  EX_ALGO_AUTO = 0,  /* pick by shape and alignment */
  EX_ALGO_SIMT = 1,  /* CUDA cores, int8 dp4a, int32 accumulation; any alignment */
  EX_ALGO_TC_I8 = 2  /* tcgen05 kind::i8 tensor cores, TMA-fed, int32 accumulators in tensor memory */
};

/* Flag OR-ed into the `algo` argument of ex_linear, ex_linear_partial_i64 and ex_linear_noalloc: the weight digits
 * (wh, wl) are static, i.e. written before `stream` was last synchronized. The tensor-core kernel then starts loading
 * its first weight tiles before the kernels ahead of it on the stream have finished (programmatic dependent launch),
 * instead of after. Same result bits. Do not set it while a kernel that writes the weight digits may still be running
 * on the stream (for instance right after digitizing the weights without a synchronization). No counterpart in the
 * reference (its Triton launches do not overlap). */
#define EX_LINEAR_STATIC_WEIGHTS 0x100

const char* ex_version(void);
const char* ex_status_string(int status);
/* Message of the last EX_ERR_CUDA on this host thread. */
const char* ex_last_error_string(void);

/* Synchronizes the current device, stores the device error word into *code (0 = none) and clears it. When the
 * code is non-zero it also clears the static scratch of ex_linear_noalloc on every device that has used it, since
 * a call stopped by a timed-out wait may have left partial sums there (caller-owned split-K workspaces of ex_linear
 * must then be re-zeroed by their owner). Returns EX_OK, or EX_ERR_CUDA if a CUDA call failed. For tests and
 * diagnostics, not for hot paths. */
int ex_device_error(int* code);

/*
 * Per-row fixed-point digitization.
 * Replaces kernels.digitize / _digitize_kernel (src/vllm_exact/kernels.py:74-85, :46-71), with the semantics of
 * digitize_torch (kernels.py:22-39): per row a = max|x|, e = frexp exponent of a (0 if a == 0), sh = F - e,
 * q = trunc(x * 2^sh); F = 14 balanced digits (cs = 0), F = 15 offset digits with row sum cs.
 *   x      rows x K, element type x_dtype (EX_DTYPE_F32/BF16/F16), leading dimension ldx
 *   h, l   rows x K int8 digits, leading dimension ldd (>= K)
 *   cs, sh rows int32
 */
int ex_digitize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F, int8_t* h, int8_t* l,
                int64_t ldd, int32_t* cs, int32_t* sh, void* stream);

/*
 * Row maxima for tensor-parallel digitization: amax[r] = max_k |x[r, k]| (float32; exact).
 * No reference counterpart: the reference runs on one GPU. A K-sharded (row-parallel) layer needs the row scale of
 * the WHOLE row (src/vllm_exact/kernels.py:25-29 computes it from the whole row), so each rank computes the maxima of
 * its K slice, the ranks take the elementwise MAX (an exact, order-free all-reduce), and the slice is digitized with
 * ex_digitize_given_absmax.
 */
int ex_row_absmax(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, float* amax, void* stream);

/*
 * ex_digitize with the per-row maximum supplied by the caller (amax[r] >= max_k |x[r, k]|, e.g. the all-reduced
 * maximum over all K shards): the digits of a K slice are then exactly the corresponding slice of the digits of the
 * whole row (semantics of digitize_torch, src/vllm_exact/kernels.py:22-39, with `a` taken from amax). For F = 15, cs
 * is the row sum over this slice only; slice sums add up to the whole row's sum.
 */
int ex_digitize_given_absmax(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F,
                             const float* amax, int8_t* h, int8_t* l, int64_t ldd, int32_t* cs, int32_t* sh,
                             void* stream);

/* Bytes of zero-initialised split-K workspace that ex_linear / ex_linear_partial_i64 need for this shape, split_k
 * (0 = automatic) and algorithm. 0 means no workspace is needed. */
size_t ex_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int split_k, int algo);

/*
 * Exact linear layer: out (M x N) = fp32(fp64(tot) * 2^-(sx+sw)) rounded to out_dtype, where
 * tot = 2^16 xh.wh + 2^8 (xh.wl + xl.wh) [+ xl.wl unless trunc] [+ 128 (cx + cw) + 2^14 K when F == 15].
 * Replaces kernels.exact_linear (src/vllm_exact/kernels.py:257-289) with its kernels _exact_kernel (:103-157),
 * _exact_bf16_kernel (:180-247) and _exact_fin (:159-177). Bit-identical to exact_linear_torch (:89-100) for every
 * algorithm and split_k.
 *   xh, xl (M x K, ld ldx) activation digits; cx, sx (M) int32;   wh, wl (N x K, ld ldw) weight digits; cw, sw (N)
 *   cx / cw are read only when F == 15 (may be NULL otherwise)
 *   split_k: 0 = automatic, >= 1 = number of K partitions (results are identical for every value)
 */
int ex_linear(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
              const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw, int64_t M,
              int64_t N, int64_t K, int F, int trunc, void* out, int out_dtype, int64_t ldo, void* workspace,
              size_t workspace_bytes, int split_k, int algo, void* stream);

/*
 * ex_linear for callers that cannot allocate device memory: same arguments and results as ex_linear, minus the
 * workspace. No counterpart in the reference (its split-K path allocates a fresh int64 workspace with torch.empty on
 * every call, kernels.py:273). Some callers cannot do that, or call cudaMalloc themselves: a serving engine that has
 * already reserved nearly all device memory for its KV cache (an extra allocation fails or fragments its pool), a
 * plugin host that owns every device allocation, or code running inside a region where allocation calls are not
 * allowed. This entry point allocates nothing: its split-K scratch is a static device array of
 * EX_NOALLOC_SCRATCH_BYTES inside this library, which every GPU that loads the library holds until the process exits.
 *   - The first call on a device looks up the array's device address and clears it on `stream`; make that first
 *     call before any stream capture.
 *   - Shapes whose split-K plan needs more scratch than EX_NOALLOC_SCRATCH_BYTES are rejected with EX_ERR_WORKSPACE
 *     (ex_last_error_string() says so) before anything is launched.
 *   - All calls share the one array and leave it zeroed; calls that overlap on the GPU (two streams, or two
 *     threads) race on it and must be serialized by the caller.
 */
#define EX_NOALLOC_SCRATCH_BYTES (24u << 20)
int ex_linear_noalloc(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int32_t* sx,
                      const int8_t* wh, const int8_t* wl, int64_t ldw, const int32_t* cw, const int32_t* sw,
                      int64_t M, int64_t N, int64_t K, int F, int trunc, void* out, int out_dtype, int64_t ldo,
                      int split_k, int algo, void* stream);

/* Clears the static scratch of ex_linear_noalloc on the current device, ordered on `stream`. Needed only after a
 * device error (a call stopped by a timed-out wait can leave partial sums in it); ex_device_error() already does
 * this when it reports an error. No counterpart in the reference. */
int ex_linear_noalloc_reset(void* stream);

/* Diagnostics for tests of the recovery path: fills the static scratch of the current device with `byte_value`
 * (0..255) on `stream`, which stands for what a stopped call can leave behind. Never needed in normal use. */
int ex_linear_noalloc_fill_scratch(int byte_value, void* stream);

/*
 * Integer part of ex_linear without the scaling epilogue: tot (M x N int64, ld ldt) = the exact integer total
 * of this K slice, including the F == 15 offset terms of the slice. Summing the tot of disjoint K slices (e.g. an
 * int64 all-reduce over K-sharded ranks) gives exactly the tot of the whole K range. This is the row-parallel
 * (K-sharded) building block; the reference has it only inside the split-K plumbing (kernels.py:144-146, :271-273).
 */
int ex_linear_partial_i64(const int8_t* xh, const int8_t* xl, int64_t ldx, const int32_t* cx, const int8_t* wh,
                          const int8_t* wl, int64_t ldw, const int32_t* cw, int64_t M, int64_t N, int64_t K, int F,
                          int trunc, int64_t* tot, int64_t ldt, void* workspace, size_t workspace_bytes, int split_k,
                          int algo, void* stream);

/*
 * Scaling epilogue of an int64 total: out = fp32(fp64(tot) * 2^-(sx+sw)) rounded to out_dtype.
 * Replaces the epilogue of _exact_fin (src/vllm_exact/kernels.py:172-177).
 */
int ex_epilogue_i64(const int64_t* tot, int64_t ldt, const int32_t* sx, const int32_t* sw, int64_t M, int64_t N,
                    void* out, int out_dtype, int64_t ldo, void* stream);

/*
 * Tensor parallelism over peer memory (no counterpart in the reference, which has no multi-GPU path; the exactness
 * argument is kernels.py:144-146, :159-177: int64 partial totals of disjoint K slices add up to the full total).
 *
 * CUDA IPC: ex_ipc_get_handle exports the device allocation that contains dev_ptr (handle of EX_IPC_HANDLE_BYTES
 * bytes) and the byte offset of dev_ptr inside it (allocators hand out pieces of larger allocations);
 * ex_ipc_open_handle maps an allocation exported by another process on this GPU (plain peer mapping, no multicast
 * object) and returns its base, to which the caller adds the exporter's offset; ex_ipc_close_handle unmaps a base.
 */
#define EX_IPC_HANDLE_BYTES 64
int ex_ipc_get_handle(const void* dev_ptr, unsigned char* handle, uint64_t* offset);
int ex_ipc_open_handle(const unsigned char* handle, void** base);
int ex_ipc_close_handle(void* base);

/*
 * The two exchange steps of a row-parallel (K-sharded) layer over peer memory, one kernel each (replacing the MAX
 * all-reduce of row maxima + ex_digitize_given_absmax, and the int64 SUM all-reduce of the partial totals +
 * ex_epilogue_i64). Every rank of the group makes the same calls in the same order; ranks run on different GPUs (the
 * kernels wait for one another), and on one rank calls sharing a ctl array must not overlap on the GPU (each reads
 * its call epoch from ctl). Buffers named "of every rank" are device arrays of `world` pointers, index p = rank
 * p's buffer as mapped on this GPU (e.g. with ex_ipc_open_handle), this rank's at index `rank`; all of them are
 * zero-filled once before the first call. Values cross GPUs as 64-bit words (call epoch << 32 | payload) that the
 * reader polls, so no fence is needed. Epochs live in the ctl words on the device, so calls can be captured in a CUDA
 * graph. Both kernels are launched with programmatic dependent launch. A wait that runs out (about 2 s) records a
 * device error (ex_device_error) and the call finishes with wrong outputs. Neither kernel depends on all of its own
 * blocks being resident at once.
 */
#define EX_TP_MAX_WORLD 16
#define EX_TP_MAX_BLOCKS 256
/* int32 flag words per rank of ex_allreduce_epilogue_i64 */
#define EX_TP_FLAG_WORDS(world) (world)

/* ex_tp_digitize: row maxima of this rank's K slice x (rows x K) sent to every rank, whole-row maxima taken, and the
 * slice digitized with them: bitwise the K slice of the digits of the whole rows (semantics of digitize_torch,
 * src/vllm_exact/kernels.py:22-39; for F = 15, cs is the slice's row sum).
 *   xch   of every rank: 64-bit exchange words [2][world][max_rows] (two halves by call parity, so back-to-back calls
 *         of this kernel alone are safe)
 *   ctl   this rank's two int32 words for this kernel (epoch, block counter) */
int ex_tp_digitize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t K, int F, const void* xch,
                   int64_t max_rows, int32_t* ctl, int rank, int world, int8_t* h, int8_t* l, int64_t ldd, int32_t* cs,
                   int32_t* sh, void* stream);

/* ex_allreduce_epilogue_i64: the (M, N) int64 partial totals of every rank summed (exact), scaled (exact epilogue of
 * ex_epilogue_i64) and written to this rank's `out`, as a reduce-scatter (rank r sums and finishes columns
 * [r N / world, (r + 1) N / world), rounded down to even) followed by an all-gather of the finished values.
 *   parts  of every rank: (M, N) int64 partial, leading dimension ldt
 *   xch    of every rank: output exchange buffer of 64-bit words, M * N / 2 of them for bf16/fp16 outputs, M * N for
 *          fp32 outputs
 *   flags  of every rank: EX_TP_FLAG_WORDS(world) int32 words
 *   ctl    this rank's two int32 words for this kernel
 * N, ldt and ldo must be even (EX_ERR_ALIGN otherwise). When the call completes on every rank, every rank has
 * finished reading this rank's partial, so it may be rewritten by the next work on the stream. */
int ex_allreduce_epilogue_i64(const void* parts, int64_t ldt, const void* xch, const void* flags, int32_t* ctl,
                              int rank, int world, const int32_t* sx, const int32_t* sw, int64_t M, int64_t N,
                              void* out, int out_dtype, int64_t ldo, void* stream);

/* Bytes of (uninitialised) partial-result workspace ex_paged_decode needs. */
size_t ex_paged_decode_workspace_bytes(int n, int H, int D, int max_len, int split);

/*
 * Batch-invariant paged decode attention over a paged KV cache.
 * Replaces paged_attn.paged_decode with _paged_partial / _paged_merge (src/vllm_exact/paged_attn.py:97-114,
 * :31-94). For each request b < n and query head h (KV head h / (H/KV)): softmax(scale * q.K^T) V over the first
 * seq_lens[b] tokens, token t at page block_table[b, t / BS], offset t % BS. Each request's keys are processed in
 * fixed segments of `split` keys (NS = ceil(max_len / split) segments) merged in fixed order, so a request's output
 * bits do not depend on n, on the other requests, or on where its pages are placed.
 *   q        (>= n) x H x D, strides (sq_t, sq_h, 1), bf16
 *   k_cache, v_cache: num_blocks x BS x KV x D with strides (s_block, s_page, s_head, 1), bf16; block-table entries
 *            must lie in [0, num_blocks) for every token below seq_lens
 *   block_table int32 (n x pages, row stride sbt); seq_lens int32 (n)
 *   out      (>= n) x H x D, strides (so_t, so_h, 1), out_dtype (bf16, fp16 or fp32)
 */
int ex_paged_decode(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, const void* v_cache,
                    int64_t s_block, int64_t s_page, int64_t s_head, int64_t num_blocks, const int32_t* block_table,
                    int64_t sbt,
                    const int32_t* seq_lens, int n, int H, int KV, int D, int BS, float scale, int max_len, int split,
                    void* out, int64_t so_t, int64_t so_h, int out_dtype, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * ex_paged_decode for the decode requests of a mixed prefill + decode step, without a host sync.
 * Replaces the host-side count in the patched FlashAttentionImpl.forward (src/vllm_exact/paged_attn.py:153-159:
 * ql = query_start_loc[1:] - query_start_loc[:-1]; nd = cumprod(ql == 1).sum(); paged_decode(..., nd)).
 * query_start_loc: int32 device array of at least n + 1 entries (n = number of requests described). Request b < n is
 * computed, exactly as by ex_paged_decode, iff query_start_loc[i + 1] - query_start_loc[i] == 1 for every i <= b;
 * the rows of `out` of every other request are left untouched. The count is made on the device, so the call can be
 * captured in a CUDA graph. query_start_loc == NULL: every request b < n is computed (ex_paged_decode).
 */
int ex_paged_decode_leading(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, const void* v_cache,
                            int64_t s_block, int64_t s_page, int64_t s_head, int64_t num_blocks,
                            const int32_t* block_table, int64_t sbt, const int32_t* seq_lens,
                            const int32_t* query_start_loc, int n, int H, int KV, int D, int BS, float scale,
                            int max_len, int split, void* out, int64_t so_t, int64_t so_h, int out_dtype,
                            void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VLLM_EXACT_B200_H */
