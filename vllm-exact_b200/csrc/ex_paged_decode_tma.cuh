// Batch-invariant paged decode attention, TMA page-gather variant (replaces paged_attn.py:31-72 for the common
// layouts: head size 64 or 128, at most 8 query heads per KV head, page size a multiple of 16).
//
// One CTA per (request b, KV head g, segment s) of `split` keys, 5 warps:
//   warp 4     producer: walks the segment in blocks of 64 keys; for every 16-key group it looks up the page in the
//              block table and issues TMA tiled loads of that group's K and V rows (a 4-D tensor map over the
//              cache's (head dim, KV head, page offset, page) strides, 128-byte swizzle) into a 3-stage mbarrier ring.
//   warps 0-3  consumers: warp w owns keys [16w, 16w+16) of every block and keeps its own online-softmax state.
//              Orientation is swapped so the keys fill the 16 MMA rows and the <= 8 query heads the 8 MMA columns:
//                S^T = K . Q^T                       mma.sync m16n8k16 bf16 -> fp32 (exact products)
//                p = exp(S*scale - m); p_hi = bf16(p); p_lo = bf16(p - p_hi)   (transposed in registers: movmatrix)
//                O^T = O^T*alpha + V^T . p_hi^T + V^T . p_lo^T
// Rows of a 16-key group past the sequence end are masked (-inf scores) and their V rows are zeroed in shared
// memory before use, so unwritten cache slots never reach the output. The four warps are merged in fixed order and
// the segment's (m, l, acc) goes to the same partial workspace as the cp.async kernel; k_paged_merge combines the
// segments. Nothing depends on the batch or on page placement, so results are batch invariant.
#pragma once
#include "ex_common.cuh"
#include "ex_paged_decode.cuh"

namespace ex {

constexpr int PT_THREADS = 160;
constexpr int PT_BLK = 64;        // keys per stage
constexpr int PT_GROUP = 16;      // keys per TMA box (one consumer warp)

template <int D>
struct PtCfg {
  static constexpr int NH = D / 64;                     // 64-dim (128-byte) column blocks
  static constexpr int HALF_BYTES = PT_BLK * 128;       // one column block of 64 keys
  static constexpr int TILE_BYTES = NH * HALF_BYTES;    // K or V of one stage
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int STAGES = 3;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(D == 64 || D == 128, "head size");
};

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::
          "r"(ex_smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(ex_smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// byte offset of (row, 16-byte chunk) inside a [rows][128 B] tile written by TMA with 128-byte swizzle
__device__ __forceinline__ uint32_t sw128(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

template <int D>
__global__ void __launch_bounds__(PT_THREADS, 2)
    k_paged_tma(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                const __nv_bfloat16* __restrict__ q, int64_t sq_t, int64_t sq_h, const int32_t* __restrict__ bt,
                int64_t sbt, const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ qsl, int H, int G,
                int BS, float scale, int split, int NS, float* __restrict__ ws_m, float* __restrict__ ws_l,
                float* __restrict__ ws_acc) {
  using C = PtCfg<D>;
  extern __shared__ uint8_t pt_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pt_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;

  pdl_launch_dependents();
  const int b = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  if (qsl != nullptr && !pd_in_leading_decodes(qsl, b)) return;  // not a leading decode (mixed step): nothing to do
  const int L = seq_lens[b];
  const int start = s * split;
  const int end = min(start + split, L);
  const int64_t pbase = ((int64_t)b * H + (int64_t)g * G) * NS + s;  // partial index of query head g*G

  if (start >= end) return;  // empty segment (s >= ceil(L / split)): the merge stops before it, nothing to write
  const int nblk = (end - start + PT_BLK - 1) / PT_BLK;
  if (tid == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(full_bar + i, 1);
      mbar_init(empty_bar + i, 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------------ producer
    const int32_t* btr = bt + (int64_t)b * sbt;
    for (int blk = 0; blk < nblk; ++blk) {
      const int st = blk % C::STAGES;
      const uint32_t ph = (uint32_t)(blk / C::STAGES) & 1u;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(empty_bar + st, ph ^ 1u, EX_DEVERR_WAIT_SLOT);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const int kb = start + blk * PT_BLK;
      const int ngroups = min(PT_BLK / PT_GROUP, (end - kb + PT_GROUP - 1) / PT_GROUP);
      if (lane == 0) mbar_arrive_expect_tx(full_bar + st, (uint32_t)(ngroups * 2 * C::TILE_BYTES / (PT_BLK / PT_GROUP)));
      __syncwarp();
      if (lane < ngroups) {  // one lane per 16-key group (groups never cross a page: BS and split are multiples of 16)
        const int key0 = kb + lane * PT_GROUP;
        const int page = btr[key0 / BS];
        const int off = key0 % BS;
        uint8_t* ks = smem + (size_t)st * C::STAGE_BYTES;
        uint8_t* vs = ks + C::TILE_BYTES;
#pragma unroll
        for (int h = 0; h < C::NH; ++h) {
          tma_load_4d(ks + h * C::HALF_BYTES + lane * PT_GROUP * 128, &tm_k, full_bar + st, h * 64, g, off, page);
          tma_load_4d(vs + h * C::HALF_BYTES + lane * PT_GROUP * 128, &tm_v, full_bar + st, h * 64, g, off, page);
        }
      }
      __syncwarp();
    }
    // every issued load must have landed before the CTA may exit (the consumers normally consumed them all; after a
    // timed-out wait this bounds the drain)
    if (lane == 0) {
      for (int blk = max(0, nblk - C::STAGES); blk < nblk; ++blk)
        mbar_wait(full_bar + blk % C::STAGES, (uint32_t)(blk / C::STAGES) & 1u, EX_DEVERR_WAIT_TMA);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ consumers (warps 0..3)
    const int w = warp;
    const int qr = lane >> 2, qc = (lane & 3) * 2;  // C-fragment row (key) / column pair (query head)
    // Q^T fragments (B operand, 16 dims x 8 heads per k-step): b0b1 = Q[head lane/4][dims 2(lane%4)..+1]
    uint32_t qb[D / 16][2];
#pragma unroll
    for (int kt = 0; kt < D / 16; ++kt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t v = 0;
        if (qr < G)
          v = *reinterpret_cast<const uint32_t*>(q + (int64_t)b * sq_t + (int64_t)(g * G + qr) * sq_h + kt * 16 + qc +
                                                 8 * j);
        qb[kt][j] = v;
      }
    }
    float m_run[2] = {-INFINITY, -INFINITY};  // query heads qc, qc+1
    float l_run[2] = {0.0f, 0.0f};
    float o[D / 16][4];  // O^T: rows = dims (mt*16 + qr (+8)), columns = heads (qc, qc+1)
#pragma unroll
    for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;

    for (int blk = 0; blk < nblk; ++blk) {
      const int st = blk % C::STAGES;
      const uint32_t ph = (uint32_t)(blk / C::STAGES) & 1u;
      if (!mbar_wait(full_bar + st, ph, EX_DEVERR_WAIT_TMA)) break;
      const int kb = start + blk * PT_BLK;
      const int key0 = kb + w * PT_GROUP;
      const uint8_t* ks = smem + (size_t)st * C::STAGE_BYTES;
      uint8_t* vs = smem + (size_t)st * C::STAGE_BYTES + C::TILE_BYTES;
      if (key0 < end) {
        if (key0 + PT_GROUP > end) {
          // partial group: zero the V rows past the end (unwritten cache slots may hold anything)
          const int r0 = w * PT_GROUP + (end - key0);
          const int nr = w * PT_GROUP + PT_GROUP - r0;
          for (int i = lane; i < nr * C::NH * 8; i += 32) {
            const int r = r0 + i / (C::NH * 8), h = (i / 8) % C::NH, c = i % 8;
            *reinterpret_cast<uint4*>(vs + h * C::HALF_BYTES + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
        }
        // S^T (16 keys x 8 heads) = K (16 keys x D) . Q^T
        float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int arow = w * PT_GROUP + (lane & 15);
#pragma unroll
        for (int kt = 0; kt < D / 16; ++kt) {
          const int chunk = (kt & 3) * 2 + (lane >> 4);
          uint32_t a[4];
          ldsm_x4(ex_smem_u32(ks + (kt >> 2) * C::HALF_BYTES + sw128(arow, chunk)), a);
          mma_bf16_16816(sc, a, qb[kt][0], qb[kt][1]);
        }
        // online softmax per query-head column
        float mx[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + qr + ((e & 2) ? 8 : 0);
          sc[e] = key < end ? sc[e] * scale : -INFINITY;
        }
        mx[0] = fmaxf(sc[0], sc[2]);
        mx[1] = fmaxf(sc[1], sc[3]);
        float alpha[2], msub[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
          const float mnew = fmaxf(m_run[j], mx[j]);
          const bool none = (mnew == -INFINITY);
          alpha[j] = none ? 1.0f : expf(m_run[j] - mnew);
          msub[j] = none ? 0.0f : mnew;
          m_run[j] = mnew;
        }
        float p[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = expf(sc[e] - msub[e & 1]);
        l_run[0] = l_run[0] * alpha[0] + p[0] + p[2];
        l_run[1] = l_run[1] * alpha[1] + p[1] + p[3];
        const uint32_t h01 = pack_bf16(p[0], p[1]), h23 = pack_bf16(p[2], p[3]);
        {
          const __nv_bfloat162 a01 = *reinterpret_cast<const __nv_bfloat162*>(&h01);
          const __nv_bfloat162 a23 = *reinterpret_cast<const __nv_bfloat162*>(&h23);
          lo[0] = p[0] - __low2float(a01);
          lo[1] = p[1] - __high2float(a01);
          lo[2] = p[2] - __low2float(a23);
          lo[3] = p[3] - __high2float(a23);
        }
        // P^T as the B operand (16 keys x 8 heads): transpose the 8x8 blocks of the C fragment
        const uint32_t bh0 = movmatrix_t(h01), bh1 = movmatrix_t(h23);
        const uint32_t bl0 = movmatrix_t(pack_bf16(lo[0], lo[1])), bl1 = movmatrix_t(pack_bf16(lo[2], lo[3]));
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          o[mt][0] *= alpha[0];
          o[mt][1] *= alpha[1];
          o[mt][2] *= alpha[0];
          o[mt][3] *= alpha[1];
        }
        // O^T (16 dims x 8 heads) += V^T (16 dims x 16 keys) . P^T
        const int mi = lane >> 3;
        const int vrow = w * PT_GROUP + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int cidx = mt * 2 + (mi & 1);  // 8-dim chunk index over the whole head dimension
          uint32_t a[4];
          ldsm_x4_t(ex_smem_u32(vs + (cidx >> 3) * C::HALF_BYTES + sw128(vrow, cidx & 7)), a);
          mma_bf16_16816(o[mt], a, bh0, bh1);
          mma_bf16_16816(o[mt], a, bl0, bl1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar + st);
    }
    // per-warp totals: l summed over the warp's keys (lanes with the same head column)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 4);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 8);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 16);
    }
    // stash (m, l, O) of this warp for the fixed-order merge (stage memory is free: every load was consumed)
    float* sm_m = reinterpret_cast<float*>(smem);  // [4 warps][8 heads]
    float* sm_l = sm_m + 4 * 8;                    // [4][8]
    float* sm_o = sm_l + 4 * 8;                    // [4][8 heads][D]
    // the four consumer warps must be done reading stage memory before it is reused for the merge
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (lane < 4) {
      sm_m[w * 8 + qc] = m_run[0];
      sm_m[w * 8 + qc + 1] = m_run[1];
      sm_l[w * 8 + qc] = l_run[0];
      sm_l[w * 8 + qc + 1] = l_run[1];
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int dim = mt * 16 + qr + ((e & 2) ? 8 : 0);
        const int head = qc + (e & 1);
        sm_o[(w * 8 + head) * D + dim] = o[mt][e];
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    for (int i = tid; i < G * D; i += 128) {
      const int r = i / D, d = i % D;
      float mxx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) mxx = fmaxf(mxx, sm_m[k * 8 + r]);
      float lsum = 0.0f, acc = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float mw = sm_m[k * 8 + r];
        const float c = (mw == -INFINITY) ? 0.0f : expf(mw - mxx);
        lsum += sm_l[k * 8 + r] * c;
        acc += sm_o[(k * 8 + r) * D + d] * c;
      }
      const int64_t pi = pbase + (int64_t)r * NS;
      ws_acc[pi * D + d] = acc;
      if (d == 0) {
        ws_m[pi] = mxx;
        ws_l[pi] = lsum;
      }
    }
  }
}

}  // namespace ex
