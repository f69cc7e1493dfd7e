// Exact two-digit GEMM on 5th-generation tensor cores (EX_ALGO_TC_I8), sm_100a.
//
// Same integers as the reference's _exact_kernel / _exact_bf16_kernel (kernels.py:103-157, :180-247), computed with
// tcgen05.mma kind::i8 (int8 x int8 -> int32, exact) from TMA-loaded digit tiles, int32 accumulators in tensor
// memory, int64 combine and the exact epilogue fused in.
//
// Orientation ("swap-AB"): the MMA's M dimension is 128 weight rows, its N dimension is the token tile (BT tokens),
// so decode batches (M <= 64) still fill the 128-row tensor-core datapath. Per K step of 128 bytes the CTA holds
//   Wh, Wl : 128 x 128 int8 (16 KB each)          A operands
//   X      : [xh rows 0..BT) ; [xl rows BT..2BT)   B operand (xh and xl stacked along N)
// and issues
//   MMA1  D[hh | md] (+)= Wh . [Xh ; Xl]^T     (N = 2 BT)  -> hh = Wh.Xh, md = Wh.Xl
//   MMA2  D[md]      +=  Wl . Xh^T             (N = BT)    -> md += Wl.Xh
//   MMA3  D[ll]      (+)= Wl . Xl^T            (N = BT, only without truncation)
// so md holds xh.wl + xl.wh directly. int32 is exact: |md| <= 2^15 K < 2^31 for K <= 65536.
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer, warps 2..9 = epilogue
// (TMEM -> registers -> int64 combine -> scale -> store), two warps per TMEM lane quarter. Two TMEM accumulator
// buffers let the epilogue of one segment overlap the MMAs of the next.
//
// Work partition: the (n-tile, k-iteration) space of one row of m-tiles is cut into `groups` equal contiguous
// ranges; a group is gs sibling CTAs that walk the same range on gs different m-tiles in lockstep, so each weight
// tile leaves HBM once and the siblings find it in L2. A CTA's walk is a list of segments (m-tile, n-tile, k_begin,
// k_end). A segment covering a whole tile is finished straight from TMEM. Split tiles are combined in one of two ways:
//   * cluster reduction (plans that cut every n-tile into ks equal K parts, one per CTA): the CTAs of one n-tile are a
//     thread-block cluster; each writes its int64 partial tile to its own shared memory, and after a cluster barrier
//     each adds a 1/ks share of the tile's elements over the ks CTAs through distributed shared memory and finishes
//     it. No global workspace, no atomics;
//   * workspace reduction (other plans): int64 totals are added with bulk reduce-adds (TMA engine) into the tile's
//     workspace slot (one slot per (group boundary, m-tile)) and a ticket counting k-iterations elects the CTA that
//     completes the tile, which applies the epilogue and zeroes the slot again.
// Integer addition is exact and order-free, so the result bits do not depend on the partition or on arrival order.
#pragma once
#include <mutex>

#include "ex_common.cuh"
#include "ex_tc_plan.h"

namespace ex {

// sxs / cxs: this tile's per-token scale words, already in shared memory; swn / cwn: this weight row's.
// All CW values are converted first with straight-line float64 code (ex_scale_to_f32: exact int64 -> float64, exact
// power-of-two scaling, one rounding to float32; on sm_100 this is about twice as fast as an int64 -> float32
// conversion, which is not a single hardware operation), then stored, predicated on the token count.
template <int CW>
__device__ __forceinline__ void tc_finish_chunk(const long long (&tot)[CW], int m0, int n, const int* sxs,
                                                const int* cxs, int swn, long long cwn, const TcArgs& a) {
  if (n >= a.N) return;
  const int jmax = min(CW, a.M - m0);
  long long v[CW];
  if (a.F == 15) {
    const long long kc = 16384ll * (long long)a.K + 128ll * cwn;
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = tot[j] + 128ll * (long long)cxs[j] + kc;
  } else {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = tot[j];
  }
  if (a.partial) {
    long long* op = reinterpret_cast<long long*>(a.out) + (int64_t)m0 * a.ldo + n;
#pragma unroll
    for (int j = 0; j < CW; ++j)
      if (j < jmax) op[(int64_t)j * a.ldo] = v[j];
    return;
  }
  float f[CW];
#pragma unroll
  for (int j = 0; j < CW; ++j) f[j] = ex_scale_to_f32(v[j], sxs[j], swn);
  if (a.out_dtype == EX_DTYPE_BF16) {
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)m0 * a.ldo + n;
#pragma unroll
    for (int j = 0; j < CW; ++j)
      if (j < jmax) op[(int64_t)j * a.ldo] = __float2bfloat16_rn(f[j]);
  } else if (a.out_dtype == EX_DTYPE_F32) {
    float* op = reinterpret_cast<float*>(a.out) + (int64_t)m0 * a.ldo + n;
#pragma unroll
    for (int j = 0; j < CW; ++j)
      if (j < jmax) op[(int64_t)j * a.ldo] = f[j];
  } else {
    __half* op = reinterpret_cast<__half*>(a.out) + (int64_t)m0 * a.ldo + n;
#pragma unroll
    for (int j = 0; j < CW; ++j)
      if (j < jmax) op[(int64_t)j * a.ldo] = __float2half_rn(f[j]);
  }
}

// One output element (token m, weight row n) from its int64 total and the scale words of its token (sxm, cxm) and
// weight row (swn, cwn): the same arithmetic as tc_finish_chunk.
__device__ __forceinline__ void tc_finish_one(long long tot, int m, int n, int sxm, int cxm, int swn, long long cwn,
                                              const TcArgs& a) {
  if (a.F == 15) tot += 128ll * ((long long)cxm + cwn) + 16384ll * (long long)a.K;
  const int64_t idx = (int64_t)m * a.ldo + n;
  if (a.partial) {
    reinterpret_cast<long long*>(a.out)[idx] = tot;
    return;
  }
  const float f = ex_scale_to_f32(tot, sxm, swn);
  if (a.out_dtype == EX_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(f);
  else if (a.out_dtype == EX_DTYPE_F32)
    reinterpret_cast<float*>(a.out)[idx] = f;
  else
    reinterpret_cast<__half*>(a.out)[idx] = __float2half_rn(f);
}

template <int CW>
__device__ __forceinline__ void tmem_ldc(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 16)
    tmem_ld16(taddr, r);
  else
    tmem_ld8(taddr, r);
}

template <int BT>
struct TcLayout {
  static constexpr int XH = BT * TC_BK;    // bytes of the tile's xh rows (its xl rows follow)
  static constexpr int XTILE = 2 * XH;     // bytes of the stacked activation tile
  static constexpr int STAGE = 2 * TC_WTILE + XTILE;
  static constexpr int WROWS = 128;        // weight rows of one n-tile
  static constexpr int CB_TRUNC = 2 * BT;  // TMEM columns per accumulator buffer
  static constexpr int CB_FULL = 3 * BT;
  static_assert(BT % 8 == 0 && BT >= 8 && BT <= 128, "token tile");
};

template <int BT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_exact_tc_i8(const __grid_constant__ CUtensorMap tm_wh, const __grid_constant__ CUtensorMap tm_wl,
                  const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                  const TcArgs a) {
  using Lay = TcLayout<BT>;
  extern __shared__ uint8_t tc_smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  // per epilogue warp, two 1 KB staging buffers (4 tokens x 32 rows of int64) for bulk reduce-adds of split tiles
  long long* stage_red = reinterpret_cast<long long*>(smem + (size_t)S * Lay::STAGE);
  // per epilogue warp: the current tile's per-token shifts and row sums (2 x BT int32)
  int* tok_words = reinterpret_cast<int*>(smem + (size_t)S * Lay::STAGE + TC_RED_STAGING);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + (size_t)S * Lay::STAGE + TC_RED_STAGING + TC_TOK_WORDS);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;  // [2]
  uint64_t* done_bar = tempty_bar + 2;   // MMA completion before teardown
  uint64_t* epi_bar = done_bar + 1;      // epilogue threads finished their atomic adds
  uint64_t* flag_bar = epi_bar + 1;      // ticket result published
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(flag_bar + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = a.trunc ? Lay::CB_TRUNC : Lay::CB_FULL;
  const int nbuf = (2 * cb <= TC_TMEM_COLS) ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full_bar + i, 1);
      mbar_init(empty_bar + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull_bar + i, 1);
      mbar_init(tempty_bar + i, 32 * TC_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    mbar_init(epi_bar, 32 * TC_EPI_WARPS);
    mbar_init(flag_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_wh);
    tma_prefetch_desc(&tm_wl);
    tma_prefetch_desc(&tm_xh);
    tma_prefetch_desc(&tm_xl);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Programmatic dependent launch: this prologue may overlap the kernels still running before it (typically the
  // activation digitizer and the previous GEMM). Before waiting, the producer touches only this CTA's first S weight
  // tiles: with a.w_early (the caller guarantees the weight digits are static, i.e. written before the stream was
  // last synchronized) it loads them into the first S pipeline stages, so the weight stream starts at once;
  // otherwise it only warms L2 with them (L2 is coherent with any writer, so that is safe even if a kernel still
  // running wrote them). Activation tiles, scales and every write wait for pdl_wait().
  int pre = 0;  // producer lane: pipeline stages whose weight tiles were loaded before pdl_wait()
  if (warp == 0 && lane == 0) {
    const uint64_t pol_w = l2_policy_evict_first();
    TcWalk walk(a, (int)blockIdx.x);
    TcSeg sg;
    while (pre < S && walk.next(sg)) {
      const int wr = sg.n_tile * Lay::WROWS;
      for (int kt = sg.kb; kt < sg.ke && pre < S; ++kt, ++pre) {
        if (a.w_early) {
          uint8_t* st = smem + (size_t)pre * Lay::STAGE;
          mbar_arrive_expect_tx(full_bar + pre, Lay::STAGE);  // this stage's activation tiles complete it later
          tma_load_2d(st, &tm_wh, full_bar + pre, kt * TC_BK, wr, pol_w);
          tma_load_2d(st + TC_WTILE, &tm_wl, full_bar + pre, kt * TC_BK, wr, pol_w);
        } else {
          tma_prefetch_l2_2d(&tm_wh, kt * TC_BK, wr);
          tma_prefetch_l2_2d(&tm_wl, kt * TC_BK, wr);
        }
      }
    }
    if (!a.w_early) pre = 0;
  }
  pdl_launch_dependents();
  pdl_wait();

  int fin_sw = 0;        // cluster reduction: scale words of the weight row this thread finishes
  long long fin_cw = 0;
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      TcWalk walk(a, (int)blockIdx.x);
      TcSeg sg;
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      while (ok && walk.next(sg)) {
        const int n_tile = sg.n_tile, m_tile = sg.m_tile;
        for (int kt = sg.kb; kt < sg.ke; ++kt) {
          const bool early = issued < pre;  // weights already loading into this stage since before pdl_wait()
          if (!early && !mbar_wait(empty_bar + stage, phase ^ 1, EX_DEVERR_WAIT_SLOT)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (size_t)stage * Lay::STAGE;
          const int kc = kt * TC_BK;
          const int wr = n_tile * Lay::WROWS, xr = m_tile * BT;
          if (!early) {
            mbar_arrive_expect_tx(full_bar + stage, Lay::STAGE);
            tma_load_2d(st, &tm_wh, full_bar + stage, kc, wr, pol_w);
            tma_load_2d(st + TC_WTILE, &tm_wl, full_bar + stage, kc, wr, pol_w);
          }
          tma_load_2d(st + 2 * TC_WTILE, &tm_xh, full_bar + stage, kc, xr, pol_x);
          tma_load_2d(st + 2 * TC_WTILE + Lay::XH, &tm_xl, full_bar + stage, kc, xr, pol_x);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // wait for every load still in flight before the CTA may exit (bounded)
      const int64_t pending = issued < S ? issued : S;
      for (int64_t i = 0; i < pending; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1;
        }
        mbar_wait(full_bar + stage, phase, EX_DEVERR_WAIT_TMA);
      }
    }
    __syncwarp();  // reconverge the warp before the CTA barrier below (lane 0 alone ran the producer)
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_2bt = make_idesc_i8(128, 2 * BT);
      const uint32_t idesc_bt = make_idesc_i8(128, BT);
      TcWalk walk(a, (int)blockIdx.x);
      TcSeg sg;
      int stage = 0;
      uint32_t phase = 0;
      int seg_i = 0;
      bool ok = true;
      while (ok && walk.next(sg)) {
        const int buf = nbuf == 2 ? (seg_i & 1) : 0;
        const uint32_t use = nbuf == 2 ? (uint32_t)(seg_i >> 1) : (uint32_t)seg_i;  // uses of this buffer so far
        if (!mbar_wait(tempty_bar + buf, (use & 1) ^ 1, EX_DEVERR_WAIT_TMEM)) break;
        tc_fence_after();
        const uint32_t d_hh = tmem_base + (uint32_t)(buf * cb);
        const uint32_t d_md = d_hh + BT;
        const uint32_t d_ll = d_hh + 2 * BT;
        for (int kt = sg.kb; kt < sg.ke; ++kt) {
          if (!mbar_wait(full_bar + stage, phase, EX_DEVERR_WAIT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = ex_smem_u32(smem + (size_t)stage * Lay::STAGE);
          const uint64_t dwh = make_sw128_desc(st);
          const uint64_t dwl = make_sw128_desc(st + TC_WTILE);
          const uint64_t dxh = make_sw128_desc(st + 2 * TC_WTILE);
          const uint64_t dxl = make_sw128_desc(st + 2 * TC_WTILE + Lay::XH);
#pragma unroll
          for (int j = 0; j < TC_BK / 32; ++j) {  // 32-byte K steps inside the swizzled row (+2 in 16-byte units)
            const uint64_t o = (uint64_t)(2 * j);
            const uint32_t acc = (kt > sg.kb || j > 0) ? 1u : 0u;
            tc_mma_i8(d_hh, dwh + o, dxh + o, idesc_2bt, acc);
            tc_mma_i8(d_md, dwl + o, dxh + o, idesc_bt, 1u);
            if (!a.trunc) tc_mma_i8(d_ll, dwl + o, dxl + o, idesc_bt, acc);
          }
          // frees this smem stage once the MMAs above have read it
          tc_commit(empty_bar + stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        // accumulator of this segment is complete
        tc_commit(tfull_bar + buf);
        ++seg_i;
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, EX_DEVERR_WAIT_MMA);
    }
    __syncwarp();  // reconverge the warp before the CTA barrier below (lane 0 alone issued the MMAs)
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    // Two warps per TMEM lane quarter; warp half h takes the token chunks c with (c / CW) % 2 == h.
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;     // 0 or 1
    const int row = 32 * q + lane;        // weight row inside the tile = TMEM lane
    const int et = threadIdx.x - 64;      // 0 .. 32 * TC_EPI_WARPS - 1
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    long long* my_stage = stage_red + (size_t)(warp - 2) * 2 * TC_RED_TOK * 32;  // this warp's two buffers
    int* my_sx = tok_words + (warp - 2) * 2 * 128;  // this warp's copy of the tile's token shifts / row sums
    int* my_cx = my_sx + 128;
    constexpr int CW = BT < 32 ? 8 : 16;  // TMEM columns per tcgen05.ld (and tokens per chunk)
    constexpr int NCH = BT / CW;          // chunks per tile; this warp takes chunks half, half + 2, ...
    uint32_t nbulk = 0;  // bulk reduce-adds issued by this warp (selects and recycles the staging buffers)
    TcWalk walk(a, (int)blockIdx.x);
    TcSeg sg = {0, 0, 0, 0};
    int seg_i = 0;
    uint32_t epi_phase = 0;
    if (a.ks > 1) {
      // Cluster reduction, first half: this CTA's only segment is one K part of its tile. Its int64 partial tile goes
      // to this CTA's shared memory as [token][128 rows], over the pipeline stages: once the accumulator is complete
      // every load has landed and every MMA has read its operands, so nothing touches that memory any more. The
      // cluster's CTAs add the parts after the cluster barrier that follows the role branches.
      long long* red = reinterpret_cast<long long*>(smem);
      if (walk.next(sg)) {
        // scale words the finishing step needs, fetched while the MMAs still run: the tile's token shifts and row
        // sums into shared memory (one copy per CTA), this thread's weight row's into registers
        const int m0 = sg.m_tile * BT;
        for (int j = et; j < BT; j += 32 * TC_EPI_WARPS) {
          const int t = min(m0 + j, a.M - 1);
          tok_words[j] = a.partial ? 0 : __ldg(a.sx + t);
          tok_words[128 + j] = a.F == 15 ? __ldg(a.cx + t) : 0;
        }
        const int part = (int)cluster_ctarank() / a.gs;
        const int E = min(BT, a.M - m0) * 128;
        const int nf = sg.n_tile * Lay::WROWS + (((int)(((int64_t)E * part) / a.ks) + et) & 127);
        if (nf < a.N) {
          fin_sw = a.partial ? 0 : __ldg(a.sw + nf);
          fin_cw = a.F == 15 ? (long long)__ldg(a.cw + nf) : 0ll;
        }
      }
      if (sg.kb < sg.ke && mbar_wait(tfull_bar, 0, EX_DEVERR_WAIT_MMA)) {
        tc_fence_after();
        const uint32_t t_hh = tmem_base + lane_off;
#pragma unroll 1
        for (int ci = half; ci < NCH; ci += 2) {
          const int c = ci * CW;
          uint32_t vh[CW], vm[CW], vl[CW];
          tmem_ldc<CW>(t_hh + c, vh);
          tmem_ldc<CW>(t_hh + BT + c, vm);
          if (!a.trunc) tmem_ldc<CW>(t_hh + 2 * BT + c, vl);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < CW; ++j)
            red[(c + j) * 128 + row] = ex_combine((int)vh[j], (int)vm[j], a.trunc ? 0 : (int)vl[j]);
        }
      }
    }
    while (a.ks <= 1 && walk.next(sg)) {
      const int buf = nbuf == 2 ? (seg_i & 1) : 0;
      const uint32_t use = nbuf == 2 ? (uint32_t)(seg_i >> 1) : (uint32_t)seg_i;
      const int n_tile = sg.n_tile, m_tile = sg.m_tile;
      const int n = n_tile * Lay::WROWS + row;
      const int m0 = m_tile * BT;
      // scale words of this tile, fetched while the MMAs still run (global latency is long under full HBM load)
      __syncwarp();  // the previous segment's reads of my_sx / my_cx are done
      for (int j = lane; j < BT; j += 32) {
        const int t = min(m0 + j, a.M - 1);
        my_sx[j] = a.partial ? 0 : __ldg(a.sx + t);  // partial mode has no scales (sx may be null)
        my_cx[j] = a.F == 15 ? __ldg(a.cx + t) : 0;
      }
      const int swn = (a.partial || n >= a.N) ? 0 : __ldg(a.sw + n);
      const long long cwn = (a.F == 15 && n < a.N) ? (long long)__ldg(a.cw + n) : 0ll;
      __syncwarp();
      if (!mbar_wait(tfull_bar + buf, use & 1, EX_DEVERR_WAIT_MMA)) break;
      tc_fence_after();
      const bool whole = (sg.kb == 0 && sg.ke == a.KI);
      // Slot layout: [lane quarter][token][32 rows].
      // A split tile (m, n) owns slot (b* - 1) * m_tiles + m, b* = the first group boundary strictly inside n's
      // k-range: every contributor computes the same slot and distinct split tiles get distinct slots.
      const int slot = whole ? 0 : tc_split_slot(a, n_tile, m_tile);
      long long* slot_q = a.ws_acc + ((int64_t)slot * 4 + q) * BT * 32;
      const uint32_t t_hh = tmem_base + lane_off + (uint32_t)(buf * cb);
      if (half >= NCH) {  // no chunk for this warp (BT = 8): release the accumulator right away
        tc_fence_before();
        mbar_arrive(tempty_bar + buf);
      }
#pragma unroll 1
      for (int ci = half; ci < NCH; ci += 2) {
        const int c = ci * CW;
        uint32_t vh[CW], vm[CW], vl[CW];
        tmem_ldc<CW>(t_hh + c, vh);
        tmem_ldc<CW>(t_hh + BT + c, vm);
        if (!a.trunc) tmem_ldc<CW>(t_hh + 2 * BT + c, vl);
        tmem_ld_wait();
        if (ci + 2 >= NCH) {  // this warp's TMEM reads of the buffer are done: hand it back to the MMA warp
          tc_fence_before();
          mbar_arrive(tempty_bar + buf);
        }
        if (whole) {
          long long tot[CW];
#pragma unroll
          for (int j = 0; j < CW; ++j) tot[j] = ex_combine((int)vh[j], (int)vm[j], a.trunc ? 0 : (int)vl[j]);
          tc_finish_chunk<CW>(tot, m0 + c, n, my_sx + c, my_cx + c, swn, cwn, a);
        } else {
          // Stage 4 tokens x 32 rows in shared memory, then one 1 KB bulk reduce-add into the slot (TMA engine).
          // Per-element atomics from registers measured slower on wide layers: the adds of a CTA's first split
          // segment then compete with the weight stream in L2, where the bulk engine's do not.
#pragma unroll
          for (int j0 = 0; j0 < CW; j0 += TC_RED_TOK) {
            long long* sb = my_stage + (size_t)(nbulk & 1) * TC_RED_TOK * 32;
            if (nbulk >= 2 && lane == 0) bulk_wait_read<1>();  // the reduce that last read this buffer is done
            __syncwarp();
#pragma unroll
            for (int j = 0; j < TC_RED_TOK; ++j)
              sb[j * 32 + lane] = ex_combine((int)vh[j0 + j], (int)vm[j0 + j], a.trunc ? 0 : (int)vl[j0 + j]);
            fence_proxy_async_shared();  // make the generic-proxy writes visible to the bulk copy
            __syncwarp();
            if (lane == 0) {
              bulk_reduce_add_u64(slot_q + (int64_t)(c + j0) * 32, sb, TC_RED_TOK * 32 * 8);
              bulk_commit();
            }
            ++nbulk;
          }
        }
      }
      ++seg_i;
      if (whole) continue;
      // split tile: wait until this warp's reduce-adds are performed, then take a ticket counting k-iterations;
      // the CTA that completes the tile finishes it
      if (lane == 0) {
        bulk_wait_all();
        fence_proxy_async_global();
      }
      __syncwarp();
      __threadfence();
      mbar_arrive(epi_bar);
      if (et == 0) {
        int flag = 0;
        if (mbar_wait(epi_bar, epi_phase, EX_DEVERR_WAIT_MMA)) {
          const int old = atomicAdd(a.ws_cnt + slot, sg.ke - sg.kb);
          flag = (old + (sg.ke - sg.kb) == a.KI) ? 1 : 0;
          if (flag) a.ws_cnt[slot] = 0;
        }
        *(volatile int*)last_flag = flag;
        mbar_arrive(flag_bar);
      }
      if (!mbar_wait(flag_bar, epi_phase, EX_DEVERR_WAIT_MMA)) break;
      epi_phase ^= 1;
      if (*(volatile int*)last_flag) {
        // This CTA completed the tile: every contribution is in L2. Read the slot back in batches of independent
        // L2 loads, finish, and zero it for the next call.
        __threadfence();
        if (n < a.N) {
          const int tmax = min(BT, a.M - m0);
          long long* sp = slot_q + lane;
#pragma unroll 1
          for (int ci = half; ci * CW < tmax; ci += 2) {
            const int j0 = ci * CW;
            long long v[CW];
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = (j0 + j < tmax) ? __ldcg(sp + (int64_t)(j0 + j) * 32) : 0ll;
#pragma unroll
            for (int j = 0; j < CW; ++j)
              if (j0 + j < tmax) __stcg(sp + (int64_t)(j0 + j) * 32, 0ll);
            tc_finish_chunk<CW>(v, m0 + j0, n, my_sx + j0, my_cx + j0, swn, cwn, a);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // no bulk copy may still read shared memory when the CTA exits
    __syncwarp();
  }

  if (a.ks > 1) {
    // Cluster reduction, second half. Every thread of the cluster passes both barriers exactly once, on every path.
    cluster_sync_all();  // all K parts of the tile are in their CTAs' shared memory
    if (warp >= 2) {
      // The ks CTAs of sibling m-tile j (cluster ranks p * gs + j) share the tile's valid elements (token-major,
      // tokens < M only) in ks equal ranges; this CTA adds the ks parts of its range from distributed shared memory
      // in a fixed order and finishes them. Consecutive threads take consecutive weight rows: coalesced stores.
      // The element stride (256) is a multiple of 128, so each thread keeps one weight row n (its scale words were
      // loaded before the barrier) and steps over tokens.
      const int rank = (int)cluster_ctarank();
      const int part = rank / a.gs, sib = rank % a.gs;
      const int n_tile = (int)blockIdx.x / (a.ks * a.gs);
      const int m0 = sib * BT;
      const int E = min(BT, a.M - m0) * 128;
      const int e0 = (int)(((int64_t)E * part) / a.ks), e1 = (int)(((int64_t)E * (part + 1)) / a.ks);
      const int et = threadIdx.x - 64;
      const int n = n_tile * 128 + ((e0 + et) & 127);
      if (n < a.N) {
        const uint32_t red_local = ex_smem_u32(smem);
        uint32_t peer[TC_MAX_CLUSTER];
#pragma unroll
        for (int p = 0; p < TC_MAX_CLUSTER; ++p)
          peer[p] = p < a.ks ? dsmem_map(red_local, (uint32_t)(p * a.gs + sib)) : 0u;
#pragma unroll 4
        for (int e = e0 + et; e < e1; e += 32 * TC_EPI_WARPS) {
          long long v = 0;
#pragma unroll
          for (int p = 0; p < TC_MAX_CLUSTER; ++p)
            if (p < a.ks) v += dsmem_ld_s64(peer[p] + (uint32_t)e * 8u);
          const int tok = e >> 7;
          tc_finish_one(v, m0 + tok, n, tok_words[tok], tok_words[128 + tok], fin_sw, fin_cw, a);
        }
      }
    }
    cluster_sync_all();  // no CTA leaves while another may still read its shared memory
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_TMEM_COLS);
  }
}

// --------------------------------------------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

static bool device_is_sm100() {
  static int cached = -1;
  if (cached < 0) {
    int dev = 0, major = 0, minor = 0;
    cached = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess)
      cached = (major == 10 && minor == 0) ? 1 : 0;
  }
  return cached == 1;
}

// How many thread-block clusters of c CTAs of the tensor-core kernel (full shared-memory budget, one CTA per SM) the
// current device holds at once, for c = 0 .. TC_MAX_CLUSTER (0 where clusters of c cannot run). Queried once per
// device; nullptr when the query is not possible (no device), in which case plans use no clusters.
static const int* tc_cluster_cap() {
  static int cap[16][TC_MAX_CLUSTER + 1];
  static int state[16] = {};  // 0 not queried, 1 ok, 2 failed
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (state[dev] == 0) {
    state[dev] = 2;
    if (cudaFuncSetAttribute(k_exact_tc_i8<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_BUDGET) ==
        cudaSuccess) {
      state[dev] = 1;
      for (int c = 0; c <= TC_MAX_CLUSTER; ++c) {
        cap[dev][c] = 0;
        if (c < 2) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c * 64);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = TC_SMEM_BUDGET;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)c;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_exact_tc_i8<8>, &cfg) == cudaSuccess) cap[dev][c] = n;
        else (void)cudaGetLastError();
      }
    } else {
      (void)cudaGetLastError();
    }
  }
  return state[dev] == 1 ? cap[dev] : nullptr;
}

// TMA rules: 16-byte aligned bases and leading dimensions (bytes); K within the int32-exact range.
static bool tc_supported(const int8_t* xh, const int8_t* xl, int64_t ldx, const int8_t* wh, const int8_t* wl,
                         int64_t ldw, int64_t M, int64_t N, int64_t K) {
  if (K <= 0 || K > EX_MAX_K || M <= 0 || N <= 0) return false;
  if (ldx % 16 != 0 || ldw % 16 != 0) return false;
  const uintptr_t o = reinterpret_cast<uintptr_t>(xh) | reinterpret_cast<uintptr_t>(xl) |
                      reinterpret_cast<uintptr_t>(wh) | reinterpret_cast<uintptr_t>(wl);
  if (o % 16 != 0) return false;
  return device_is_sm100();
}

static bool encode_2d_i8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_bytes,
                         uint32_t box_inner, uint32_t box_outer) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BT>
static cudaError_t launch_tc_bt(const TcPlan& p, const TcArgs& a, const CUtensorMap& mwh, const CUtensorMap& mwl,
                                const CUtensorMap& mxh, const CUtensorMap& mxl, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(k_exact_tc_i8<BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  if (p.cs > 1)
    return ex_launch_pdl_cluster(k_exact_tc_i8<BT>, dim3(p.G), dim3(TC_THREADS), p.smem, p.cs, st, mwh, mwl, mxh, mxl,
                                 a);
  return ex_launch_pdl(k_exact_tc_i8<BT>, dim3(p.G), dim3(TC_THREADS), p.smem, st, mwh, mwl, mxh, mxl, a);
}

template <bool PARTIAL>
static cudaError_t launch_tc(const TcPlan& p, int F, int trunc, int out_dtype, const int8_t* xh, const int8_t* xl,
                             int64_t ldx, const int32_t* cx, const int32_t* sx, const int8_t* wh, const int8_t* wl,
                             int64_t ldw, const int32_t* cw, const int32_t* sw, int M, int N, int K, void* out,
                             int64_t ldo, void* ws, bool static_weights, cudaStream_t st) {
  CUtensorMap mwh, mwl, mxh, mxl;
  if (!encode_2d_i8(&mwh, wh, K, N, ldw, TC_BK, 128) || !encode_2d_i8(&mwl, wl, K, N, ldw, TC_BK, 128) ||
      !encode_2d_i8(&mxh, xh, K, M, ldx, TC_BK, p.BT) || !encode_2d_i8(&mxl, xl, K, M, ldx, TC_BK, p.BT))
    return cudaErrorNotSupported;
  TcArgs a;
  a.cx = cx;
  a.sx = sx;
  a.cw = cw;
  a.sw = sw;
  a.out = out;
  a.ldo = ldo;
  a.ws_cnt = p.ws_bytes ? reinterpret_cast<int*>(ws) : nullptr;
  a.ws_acc = p.ws_bytes ? reinterpret_cast<long long*>(reinterpret_cast<char*>(ws) + p.cnt_bytes) : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.F = F;
  a.trunc = trunc ? 1 : 0;
  a.out_dtype = out_dtype;
  a.partial = PARTIAL ? 1 : 0;
  tc_plan_args(p, a);
  a.w_early = static_weights ? 1 : 0;
  switch (p.BT) {
    case 8: return launch_tc_bt<8>(p, a, mwh, mwl, mxh, mxl, st);
    case 16: return launch_tc_bt<16>(p, a, mwh, mwl, mxh, mxl, st);
    case 32: return launch_tc_bt<32>(p, a, mwh, mwl, mxh, mxl, st);
    case 64: return launch_tc_bt<64>(p, a, mwh, mwl, mxh, mxl, st);
    default: return launch_tc_bt<128>(p, a, mwh, mwl, mxh, mxl, st);
  }
}

}  // namespace ex
