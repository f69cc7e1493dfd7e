// Work plan of the tensor-core exact GEMM (k_exact_tc_i8): token tile, partition of the (n-tile, k-iteration) space
// into groups of sibling CTAs, each CTA's walk over its segments, and the workspace slot of every split tile.
//
// Host and device code share this file, and it compiles as plain C++ too: the launcher plans with tc_plan(), the
// kernel walks with TcWalk and tc_split_slot(), and a host test enumerates the same functions over many shapes and
// SM counts to check that every (m-tile, n-tile) has its K range covered exactly once. That coverage is what makes
// results bit-identical under any partition, because integer addition is exact and order-free.
//
// Split tiles are combined in one of two ways:
//   * cluster reduction (TcPlan::cs > 1): when every n-tile is cut into s equal K parts and each CTA owns exactly one
//     part of one tile, the s x gs CTAs of one n-tile form a thread-block cluster and add their int64 partial tiles
//     through distributed shared memory; no global workspace is used;
//   * workspace reduction (otherwise): bulk reduce-adds into a per-tile workspace slot in global memory, and a ticket
//     elects the CTA that finishes the tile.
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>

#include "vllm_exact_b200.h"

#ifdef __CUDACC__
#define EX_HD __host__ __device__ __forceinline__
#else
#define EX_HD inline
#endif

namespace ex {

constexpr int64_t EX_MAX_K = 65536;  // int32 accumulators: |md| <= 2^15 K must stay below 2^31
constexpr int TC_EPI_WARPS = 8;  // two epilogue warps per TMEM lane quarter, splitting the token chunks
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_BK = 128;               // K bytes (int8 elements) per pipeline stage = one 128-byte swizzle row
constexpr int TC_WTILE = 128 * TC_BK;    // bytes of one weight digit tile
constexpr int TC_SMEM_BUDGET = 220 * 1024;
constexpr int TC_TMEM_COLS = 512;
constexpr int TC_RED_TOK = 4;  // tokens per bulk reduce-add (1 KB per warp)
constexpr int TC_RED_STAGING = TC_EPI_WARPS * 2 * TC_RED_TOK * 32 * 8;  // per warp 2 buffers x 4 tokens x 32 rows x int64
constexpr int TC_TOK_WORDS = TC_EPI_WARPS * 2 * 128 * 4;                // per warp (sx, cx) x up to 128 tokens x int32

struct TcPlan {
  int BT;        // token tile
  int m_tiles, n_tiles, KI;
  int64_t T;     // k-iterations of one m-tile row of tiles = n_tiles * KI
  int gs;        // CTAs per group (one per m-tile of a chunk)
  int groups;    // groups; group g walks (n-tile, k) range [T*g/groups, T*(g+1)/groups)
  int chunks;    // passes over the range: m-tiles c*gs + j for c < chunks
  int G;         // CTAs = groups * gs
  int stages;
  int cs;        // CTAs per thread-block cluster (1: no cluster, split tiles reduced through the workspace)
  int ks;        // K parts per n-tile reduced inside a cluster (cluster plans only; cs = ks * gs)
  size_t smem;
  size_t ws_bytes;
  size_t cnt_bytes;
};

struct TcArgs {
  const int32_t* cx;
  const int32_t* sx;
  const int32_t* cw;
  const int32_t* sw;
  void* out;
  int64_t ldo;
  long long* ws_acc;
  int* ws_cnt;
  int M, N, K;
  int F, trunc, out_dtype, partial;
  int m_tiles, n_tiles, KI;
  int64_t T;  // n_tiles * KI
  int gs, groups, chunks;
  int stages;
  int ks;  // > 1: cluster reduction of the ks K parts of each tile (CTA rank in the cluster = part * gs + sibling)
  int w_early;  // 1: weight digits are static, so the first stages' weight tiles may load before griddepcontrol.wait
};

struct TcSeg {
  int m_tile, n_tile, kb, ke;
};

// Segment walker shared by all roles. CTAs form groups of gs siblings; sibling j of group g walks the (n-tile,
// k-iteration) range [T*g/groups, T*(g+1)/groups) once for each m-tile chunk c, on m-tile c*gs + j. Siblings run in
// lockstep over the same weight k-slices, so a weight tile leaves HBM once per chunk and the other siblings read it
// from L2 (one m-tile: the original one-range-per-CTA partition). 32-bit arithmetic whenever the products fit.
// `cta` is the CTA's index in the grid (blockIdx.x).
struct TcWalk {
  int64_t r0, r1, it;
  int KI, j, mc, chunks, gs, m_tiles;
  EX_HD TcWalk(const TcArgs& a, int cta) {
    const int g = cta / a.gs;
    j = cta % a.gs;
    if (a.T * (int64_t)a.groups < 2147483647ll) {
      const uint32_t T = (uint32_t)a.T, G = (uint32_t)a.groups, b = (uint32_t)g;
      r0 = (int64_t)((T * b) / G);
      r1 = (int64_t)((T * (b + 1)) / G);
    } else {
      r0 = (a.T * (int64_t)g) / a.groups;
      r1 = (a.T * (int64_t)(g + 1)) / a.groups;
    }
    it = r0;
    KI = a.KI;
    mc = 0;
    chunks = a.chunks;
    gs = a.gs;
    m_tiles = a.m_tiles;
  }
  EX_HD bool next(TcSeg& s) {
    while (mc < chunks) {
      const int m_tile = mc * gs + j;
      if (m_tile >= m_tiles || it >= r1) {
        ++mc;
        it = r0;
        continue;
      }
      if (it < 2147483647ll) {
        const uint32_t u = (uint32_t)it, k = (uint32_t)KI;
        s.n_tile = (int)(u / k);
        s.kb = (int)(u % k);
      } else {
        s.n_tile = (int)(it / KI);
        s.kb = (int)(it % KI);
      }
      s.m_tile = m_tile;
      const int64_t end = (int64_t)s.kb + (r1 - it);
      s.ke = (int)(end < (int64_t)KI ? end : (int64_t)KI);
      it += s.ke - s.kb;
      return true;
    }
    return false;
  }
};

// Workspace slot of a split tile (a segment with kb > 0 or ke < KI): slot (b* - 1) * m_tiles + m_tile, b* = the first
// group boundary strictly inside n_tile's k-range. Every contributor of the tile computes the same slot and distinct
// split tiles get distinct slots in [0, (groups - 1) * m_tiles).
EX_HD int tc_split_slot(const TcArgs& a, int n_tile, int m_tile) {
  const int64_t num = ((int64_t)n_tile * a.KI + 1) * a.groups + a.T - 1;
  const int bstar = num < 2147483647ll ? (int)((uint32_t)num / (uint32_t)a.T) : (int)(num / a.T);
  return (bstar - 1) * a.m_tiles + m_tile;
}

inline int tc_pick_bt(int64_t M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

inline size_t tc_stage_bytes(int BT) { return 2 * (size_t)TC_WTILE + 2 * (size_t)BT * TC_BK; }

constexpr int TC_MAX_CLUSTER = 8;  // portable cluster size limit

// Single CTAs on 128-row n-tiles with the token tile picked from M. `cluster_cap[c]` (c <= TC_MAX_CLUSTER), when
// given, is how many clusters of c CTAs of this kernel the device holds at once; a plan uses cluster reduction only
// if all of its clusters fit at once (one wave), so no cluster waits for another to finish.
inline TcPlan tc_plan_bt(int64_t M, int64_t N, int64_t K, int split_k, int sms, const int* cluster_cap, int BT) {
  TcPlan p;
  p.BT = BT;
  p.m_tiles = (int)((M + p.BT - 1) / p.BT);
  p.n_tiles = (int)((N + 127) / 128);
  p.KI = (int)((K + TC_BK - 1) / TC_BK);
  p.T = (int64_t)p.n_tiles * p.KI;
  p.gs = std::min(p.m_tiles, 8);
  p.chunks = (p.m_tiles + p.gs - 1) / p.gs;
  const int64_t fit = std::max<int64_t>(1, sms / p.gs);  // groups resident at once (one CTA per SM)
  int64_t groups = fit;  // automatic default: the balanced (n-tile, k-step) partition over every resident group
  if (split_k > 0) {
    groups = (int64_t)p.n_tiles * split_k;
  } else {
    // Tile-aligned partition when it keeps at least 60% of the groups busy: every n-tile split into s equal K ranges
    // (s = 1: whole tiles, no workspace). Fewer, aligned split tiles cost less in reduction and finishing than the
    // balanced partition's ragged ones; measured on B200 it wins for the narrow layers (o_proj M=64 17.5 -> 15.2 us,
    // qkv M=256 34.6 -> 26.6 us) and is not taken for wide ones (gate_up, lm_head), where it would not apply.
    const int64_t s = fit / p.n_tiles;
    if (s >= 1 && (int64_t)p.n_tiles * s * 10 >= fit * 6) groups = (int64_t)p.n_tiles * s;
    // More n-tiles than resident groups, with sibling m-tiles (tensor-bound sizes): whole tiles per group when a
    // divisor of n_tiles keeps >= 60 % of the groups busy with at most 3 tiles each, since the balanced partition
    // would split nearly every tile. Measured on B200: gate_up M = 256 78.1 -> 67.7 us, in_proj_qkvz (N = 12288)
    // M = 256 51.5 -> 47.8 us, o_proj M = 1024 59.5 -> 46.9 us, M = 4096 189 -> 164 us; with 6-12 tiles per group
    // (gate_up, in_proj_qkvz at M >= 1024) it was 2-10 % slower, so those keep the balanced partition.
    if (s == 0 && p.gs >= 2)
      for (int64_t g = fit; g * 10 >= fit * 6; --g)
        if (p.n_tiles % g == 0 && p.n_tiles / g <= 3) {
          groups = g;
          break;
        }
  }
  groups = std::max<int64_t>(1, std::min<int64_t>(groups, p.T));
  groups = std::min<int64_t>(groups, 2147483647 / p.gs);
  p.groups = (int)groups;
  p.G = p.groups * p.gs;
  const size_t stage = tc_stage_bytes(p.BT);
  const size_t overhead = 1024 + 256 + TC_RED_STAGING + TC_TOK_WORDS;  // alignment, barriers, staging, scale words
  p.stages = (int)std::min<size_t>(8, (TC_SMEM_BUDGET - overhead) / stage);
  p.smem = (size_t)p.stages * stage + overhead;
  const bool aligned = (groups <= p.n_tiles) && (p.n_tiles % groups == 0);  // every group covers whole n-tiles
  // cluster reduction: every n-tile cut into ks >= 2 K parts (one per group), one segment per CTA (one m-tile chunk)
  p.ks = 0;
  p.cs = 1;
  if (cluster_cap && !aligned && groups % p.n_tiles == 0 && p.chunks == 1) {
    const int64_t ks = groups / p.n_tiles;
    const int64_t cs = ks * p.gs;
    // the partial tile ([BT][128] int64) is written over the pipeline stages, so it must fit in them
    const size_t red = (size_t)p.BT * 128 * 8, stages_bytes = (size_t)std::min<size_t>(
        8, (TC_SMEM_BUDGET - (1024 + 256 + TC_RED_STAGING + TC_TOK_WORDS)) / tc_stage_bytes(p.BT)) * tc_stage_bytes(p.BT);
    if (ks >= 2 && ks <= p.KI && cs <= TC_MAX_CLUSTER && (int64_t)cluster_cap[cs] * cs >= (int64_t)p.G &&
        red <= stages_bytes) {
      p.ks = (int)ks;
      p.cs = (int)cs;
    }
  }
  const int64_t slots = (groups - 1) * (int64_t)p.m_tiles;  // one per (group boundary, m-tile)
  p.cnt_bytes = (size_t)((slots * 4 + 255) / 256 * 256);
  p.ws_bytes = (aligned || slots == 0 || p.cs > 1) ? 0 : p.cnt_bytes + (size_t)slots * p.BT * 128 * 8;
  // (slot layout [4 lane quarters][BT tokens][32 rows] per 128 rows: each epilogue warp reduces contiguous 1 KB)
  return p;
}

// The plan of an M x N x K call: the token tile picked from M, except that for 128 < M <= 256 an automatic plan takes
// 64-token tiles when the 128-token plan would cut K into parts of at most 16 steps per CTA and the 64-token plan
// covers whole tiles: such CTAs spend more on pipeline fill and split-tile reduction than on their MMAs (measured on
// B200 at M = 256: o_proj 28.0 -> 24.4 us; qkv, gate_up and down, whose plans do not qualify, are 26-42 % slower
// with 64-token tiles).
inline TcPlan tc_plan(int64_t M, int64_t N, int64_t K, int split_k, int sms, const int* cluster_cap = nullptr) {
  const TcPlan p = tc_plan_bt(M, N, K, split_k, sms, cluster_cap, tc_pick_bt(M));
  if (split_k == 0 && M > 128 && M <= 256 && p.groups > p.n_tiles && (int64_t)p.KI * p.n_tiles <= 16ll * p.groups) {
    const TcPlan q = tc_plan_bt(M, N, K, 0, sms, cluster_cap, 64);
    if (q.groups <= q.n_tiles && q.n_tiles % q.groups == 0) return q;
  }
  return p;
}

// The plan's fields as kernel arguments (the launcher adds pointers, shape and mode).
inline void tc_plan_args(const TcPlan& p, TcArgs& a) {
  a.m_tiles = p.m_tiles;
  a.n_tiles = p.n_tiles;
  a.KI = p.KI;
  a.T = p.T;
  a.gs = p.gs;
  a.groups = p.groups;
  a.chunks = p.chunks;
  a.stages = p.stages;
  a.ks = p.cs > 1 ? p.ks : 0;
}

}  // namespace ex
