// Batch-invariant paged decode attention (replaces paged_attn.py:31-114).
//
// Kernel 1 (k_paged_partial), one CTA per (request b, KV head g, segment s): keys [s*split, min((s+1)*split, L_b)),
// gathered page by page through the block table with cp.async into a 3-stage shared-memory ring (16-byte chunks,
// XOR-swizzled rows so the ldmatrix reads below are bank-conflict free). Four warps; each warp owns a fixed group of
// 16 keys of every block (and, for D = 256, half of the value dimensions) and keeps its own online-softmax state.
//   S = q.K^T      one bf16 tensor-core product (mma.sync m16n8k16, fp32 accumulate; the G <= 16 query heads that
//                  share the KV head are the 16 MMA rows)
//   p = exp(S*scale - m), p_hi = bf16(p), p_lo = bf16(p - p_hi)
//   O = O*alpha + p_hi.V + p_lo.V    two bf16 tensor-core products, i.e. p is used to ~16 bits
// The warps are merged in fixed order and the segment's (m, l, acc) is written to the partial workspace.
// Kernel 2 (k_paged_merge), one CTA per (request, head): merges the request's non-empty segments in fixed order
// s = 0 .. min(NS, ceil(L / split)) - 1 (NS = ceil(max_len / split) segment CTAs per request are launched; those past
// the request's length exit at once without writing) and writes acc / l. Merging an empty segment at the end of the
// fixed order only adds +0 to acc and l, so stopping before the empty ones changes no bits (an exactly -0.0 output
// keeps its sign). The stopping point depends on the request's own length only, so invariance is unaffected.
// Nothing in either kernel depends on n, on other requests, or on where pages live, so a request's output is
// bitwise the same alone, in any batch, and under any page placement.
#pragma once
#include "ex_common.cuh"

namespace ex {

constexpr int PD_THREADS = 128;
constexpr int PD_STAGES = 3;

template <int D>
struct PdCfg {
  static constexpr int DSPLIT = D > 128 ? D / 128 : 1;  // warps sharing one key group, each owning DW value dims
  static constexpr int DW = D / DSPLIT;
  static constexpr int KG = 4 / DSPLIT;  // key groups (of 16 keys) per block
  static constexpr int BLK = 16 * KG;    // keys per block
  static constexpr int CH = D / 8;       // 16-byte chunks per K/V row
  static constexpr int TILE_BYTES = BLK * D * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int SMEM = PD_STAGES * STAGE_BYTES;
  static_assert(D == 64 || D == 128 || D == 256, "head size");
};

__device__ __forceinline__ uint32_t pd_swz(int row, int chunk, int D) {
  return (uint32_t)(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0: nothing is read, the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (lower 16 bits), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}

// Mixed prefill + decode steps: the reference counts on the host the leading requests whose query length is 1
// (paged_attn.py:153-159, nd = cumprod(ql == 1).sum(), a host sync) and decodes requests [0, nd). Here every block
// evaluates the same rule on the device: request b is decoded iff qsl[i + 1] - qsl[i] == 1 for every i <= b (qsl =
// query_start_loc, at least b + 2 entries). Block-wide vote: every thread of the block must call it.
__device__ __forceinline__ bool pd_in_leading_decodes(const int32_t* __restrict__ qsl, int b) {
  int ok = 1;
  for (int i = threadIdx.x; i <= b; i += blockDim.x) ok &= (qsl[i + 1] - qsl[i] == 1) ? 1 : 0;
  return __syncthreads_and(ok) != 0;
}

template <int D>
__global__ void __launch_bounds__(PD_THREADS, 2)
    k_paged_partial(const __nv_bfloat16* __restrict__ q, int64_t sq_t, int64_t sq_h,
                    const __nv_bfloat16* __restrict__ kc, const __nv_bfloat16* __restrict__ vc, int64_t s_block,
                    int64_t s_page, int64_t s_head, const int32_t* __restrict__ bt, int64_t sbt,
                    const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ qsl, int H, int G, int BS,
                    float scale, int split, int NS, float* __restrict__ ws_m, float* __restrict__ ws_l,
                    float* __restrict__ ws_acc) {
  using C = PdCfg<D>;
  extern __shared__ __align__(1024) uint8_t pd_smem[];
  pdl_launch_dependents();  // the merge kernel's prologue may start; it waits for this grid before reading
  pdl_wait();               // query / cache / block table come from earlier kernels
  if (qsl != nullptr && !pd_in_leading_decodes(qsl, blockIdx.x)) return;  // not a leading decode: nothing to do
  const int b = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kg = warp / C::DSPLIT, dh = warp % C::DSPLIT;
  const int L = seq_lens[b];
  const int start = s * split;
  const int end = min(start + split, L);
  const int64_t pbase = ((int64_t)b * H + (int64_t)g * G) * NS + s;  // partial index of row 0

  if (start >= end) return;  // empty segment (s >= ceil(L / split)): the merge stops before it, nothing to write

  const uint32_t smem0 = ex_smem_u32(pd_smem);
  const __nv_bfloat16* kbase = kc + (int64_t)g * s_head;
  const __nv_bfloat16* vbase = vc + (int64_t)g * s_head;
  const int32_t* btr = bt + (int64_t)b * sbt;
  const int nblk = (end - start + C::BLK - 1) / C::BLK;

  auto issue = [&](int blk, int stage) {
    const int kb = start + blk * C::BLK;
    const uint32_t ks = smem0 + stage * C::STAGE_BYTES;
    const uint32_t vs = ks + C::TILE_BYTES;
#pragma unroll
    for (int i = 0; i < (C::BLK * C::CH) / PD_THREADS; ++i) {
      const int c = tid + i * PD_THREADS;
      const int row = c / C::CH, ch = c % C::CH;
      const int key = kb + row;
      const bool ok = key < end;
      int64_t off = 0;
      if (ok) {
        const int page = btr[key / BS];
        off = (int64_t)page * s_block + (int64_t)(key % BS) * s_page + ch * 8;
      }
      const uint32_t d = pd_swz(row, ch, D);
      cp_async16(ks + d, ok ? (const void*)(kbase + off) : (const void*)kc, ok);
      cp_async16(vs + d, ok ? (const void*)(vbase + off) : (const void*)vc, ok);
    }
  };

  // query fragments (A operand, 16 rows = query heads g*G .. g*G+G-1, zero rows beyond G)
  uint32_t qa[D / 16][4];
  {
    const int r0 = lane >> 2, c0 = (lane & 3) * 2;
#pragma unroll
    for (int kt = 0; kt < D / 16; ++kt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r0 + ((j & 1) ? 8 : 0);
        const int col = kt * 16 + c0 + ((j & 2) ? 8 : 0);
        uint32_t v = 0;
        if (r < G) v = *reinterpret_cast<const uint32_t*>(q + (int64_t)b * sq_t + (int64_t)(g * G + r) * sq_h + col);
        qa[kt][j] = v;
      }
    }
  }

  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  float o[C::DW / 8][4];
#pragma unroll
  for (int i = 0; i < C::DW / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;

#pragma unroll
  for (int st = 0; st < PD_STAGES - 1; ++st) {
    if (st < nblk) issue(st, st);
    cp_async_commit();
  }

  for (int blk = 0; blk < nblk; ++blk) {
    cp_async_wait<PD_STAGES - 2>();
    __syncthreads();
    if (blk + PD_STAGES - 1 < nblk) issue(blk + PD_STAGES - 1, (blk + PD_STAGES - 1) % PD_STAGES);
    cp_async_commit();

    const uint32_t ks = smem0 + (blk % PD_STAGES) * C::STAGE_BYTES;
    const uint32_t vs = ks + C::TILE_BYTES;
    const int kb = start + blk * C::BLK;

    // S = Q K^T for this warp's 16 keys (two n-tiles of 8 keys)
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
      const int row = 16 * kg + 8 * j + (lane & 7);
#pragma unroll
      for (int kt = 0; kt < D / 16; kt += 2) {
        uint32_t bfr[4];
        ldsm_x4(ks + pd_swz(row, 2 * kt + (lane >> 3), D), bfr);
        mma_bf16_16816(sc[j], qa[kt], bfr[0], bfr[1]);
        mma_bf16_16816(sc[j], qa[kt + 1], bfr[2], bfr[3]);
      }
    }
    // online softmax (rows r0 = lane/4 -> elements 0,1; r0 + 8 -> elements 2,3)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb + 16 * kg + 8 * j + (lane & 3) * 2 + (e & 1);
        const float v = key < end ? sc[j][e] * scale : -INFINITY;
        sc[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2], msub[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_run[r], mx[r]);
      const bool none = (mnew == -INFINITY);
      alpha[r] = none ? 1.0f : expf(m_run[r] - mnew);
      msub[r] = none ? 0.0f : mnew;
      m_run[r] = mnew;
    }
    uint32_t ph[4], pl[4];
    float psum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float p[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[e] = expf(sc[j][e] - msub[e >> 1]);
        psum[e >> 1] += p[e];
      }
      ph[2 * j + 0] = pack_bf16(p[0], p[1]);
      ph[2 * j + 1] = pack_bf16(p[2], p[3]);
      const __nv_bfloat162 h01 = *reinterpret_cast<const __nv_bfloat162*>(&ph[2 * j + 0]);
      const __nv_bfloat162 h23 = *reinterpret_cast<const __nv_bfloat162*>(&ph[2 * j + 1]);
      lo[0] = p[0] - __low2float(h01);
      lo[1] = p[1] - __high2float(h01);
      lo[2] = p[2] - __low2float(h23);
      lo[3] = p[3] - __high2float(h23);
      pl[2 * j + 0] = pack_bf16(lo[0], lo[1]);
      pl[2 * j + 1] = pack_bf16(lo[2], lo[3]);
    }
    // A fragment of P (16 rows x 16 keys): a0a1 = (r0, keys 0-7), a2a3 = (r0+8, keys 0-7), a4a5 = (r0, keys 8-15),
    // a6a7 = (r0+8, keys 8-15)
    const uint32_t pah[4] = {ph[0], ph[1], ph[2], ph[3]};
    const uint32_t pal[4] = {pl[0], pl[1], pl[2], pl[3]};
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * alpha[r] + psum[r];
#pragma unroll
    for (int nt = 0; nt < C::DW / 8; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }
    {
      const int mi = lane >> 3;
      const int row = 16 * kg + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int nt = 0; nt < C::DW / 8; nt += 2) {
        uint32_t bfr[4];
        ldsm_x4_t(vs + pd_swz(row, (dh * C::DW) / 8 + nt + (mi >> 1), D), bfr);
        mma_bf16_16816(o[nt], pah, bfr[0], bfr[1]);
        mma_bf16_16816(o[nt], pal, bfr[0], bfr[1]);
        mma_bf16_16816(o[nt + 1], pah, bfr[2], bfr[3]);
        mma_bf16_16816(o[nt + 1], pal, bfr[2], bfr[3]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // merge the warps of this CTA in fixed key-group order
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  float* sm_m = reinterpret_cast<float*>(pd_smem);     // [4 warps][16 rows]
  float* sm_l = sm_m + 4 * 16;                         // [4][16]
  float* sm_o = sm_l + 4 * 16;                         // [4][16][DW]
  {
    const int r0 = lane >> 2;
    if ((lane & 3) == 0) {
      sm_m[warp * 16 + r0] = m_run[0];
      sm_m[warp * 16 + r0 + 8] = m_run[1];
      sm_l[warp * 16 + r0] = l_run[0];
      sm_l[warp * 16 + r0 + 8] = l_run[1];
    }
    float* ow = sm_o + warp * 16 * C::DW;
#pragma unroll
    for (int nt = 0; nt < C::DW / 8; ++nt) {
      const int c = nt * 8 + (lane & 3) * 2;
      ow[r0 * C::DW + c] = o[nt][0];
      ow[r0 * C::DW + c + 1] = o[nt][1];
      ow[(r0 + 8) * C::DW + c] = o[nt][2];
      ow[(r0 + 8) * C::DW + c + 1] = o[nt][3];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += PD_THREADS) {
    const int r = i / D, d = i % D;
    const int dhh = d / C::DW, dd = d % C::DW;
    float mxx = -INFINITY;
#pragma unroll
    for (int k = 0; k < C::KG; ++k) mxx = fmaxf(mxx, sm_m[(k * C::DSPLIT + dhh) * 16 + r]);
    float lsum = 0.0f, acc = 0.0f;
#pragma unroll
    for (int k = 0; k < C::KG; ++k) {
      const int w = k * C::DSPLIT + dhh;
      const float mw = sm_m[w * 16 + r];
      const float c = (mw == -INFINITY) ? 0.0f : expf(mw - mxx);
      lsum += sm_l[w * 16 + r] * c;
      acc += sm_o[(w * 16 + r) * C::DW + dd] * c;
    }
    const int64_t pi = pbase + (int64_t)r * NS;
    ws_acc[pi * D + d] = acc;
    if (d == 0) {
      ws_m[pi] = mxx;
      ws_l[pi] = lsum;
    }
  }
}

// Fixed-order merge of the NS segment partials of one (request, head) (paged_attn.py:75-94).
template <int OUT_DTYPE>
__global__ void k_paged_merge(const float* __restrict__ ws_m, const float* __restrict__ ws_l,
                              const float* __restrict__ ws_acc, void* out, int64_t so_t, int64_t so_h, int H, int NS,
                              int D, const int32_t* __restrict__ seq_lens, int split,
                              const int32_t* __restrict__ qsl) {
  pdl_launch_dependents();
  pdl_wait();
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  if (qsl != nullptr && !pd_in_leading_decodes(qsl, b)) return;  // row b belongs to a prefill: left untouched
  const int L = seq_lens[b];
  const int ns = L > 0 ? min(NS, (int)(((int64_t)L + split - 1) / split)) : 0;  // non-empty segments (L = 0: none)
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float m = -INFINITY, l = 0.0f, acc = 0.0f;
    for (int s = 0; s < ns; ++s) {
      const int64_t pi = (int64_t)bh * NS + s;
      const float ms = ws_m[pi];
      const float ls = ws_l[pi];
      const float as = ws_acc[pi * D + d];
      const float mn = fmaxf(m, ms);
      const float c_old = (m == -INFINITY) ? 0.0f : expf(m - mn);
      const float c_new = (ms == -INFINITY) ? 0.0f : expf(ms - mn);
      l = l * c_old + ls * c_new;
      acc = acc * c_old + as * c_new;
      m = mn;
    }
    ex_store_out<OUT_DTYPE>(out, (int64_t)b * so_t + (int64_t)h * so_h + d, acc / l);
  }
}

}  // namespace ex
