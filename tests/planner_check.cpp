// Host check of the tensor-core exact GEMM's work plan (vllm-exact_b200/csrc/ex_tc_plan.h: tc_plan, TcWalk,
// tc_split_slot), compiled with g++ by tests/test_planner_host.py. No GPU is involved: the kernel's bit-exactness
// under every partition rests on these properties, checked here for every plan of the shape matrix below:
//   * the grid is groups x gs CTAs;
//   * every segment lies inside the tile grid, with 0 <= kb < ke <= KI;
//   * every (m-tile, n-tile) has its K iterations [0, KI) covered exactly once (so each ticket reaches KI once);
//   * a tile covered by more than one segment (a split tile) gets one workspace slot from all of its contributors,
//     distinct split tiles get distinct slots, and the slot's accumulator and ticket lie inside the planned workspace;
//   * a plan without workspace has no split tile, unless it is a cluster plan; shared memory fits the 227 KB limit
//     with at least two stages;
//   * a cluster plan (cs > 1) has clusters of cs = ks x gs <= 8 consecutive CTAs, all of which fit on the device at
//     once, one segment per CTA, and CTA rank p x gs + j of cluster t owns K part p (of ks equal parts) of n-tile t on
//     m-tile j, so the cluster holds every K part of its gs tiles; its partial tile fits in the pipeline stages.
// Plans are made for three device models: no cluster support, and two cluster capacity tables (every SM usable, and
// SMs in groups of 18 as in graphics processing clusters).
// Prints "OK <plans> <segments> <cluster plans>" or the first violation, and exits non-zero on a violation.
#include <algorithm>
#include <cstdio>
#include <string>
#include <vector>

#include "ex_tc_plan.h"

using namespace ex;

namespace {

struct Fail {
  char msg[512];
};

bool check_plan(int64_t M, int64_t N, int64_t K, int split_k, int sms, const int* cap, long long& nseg,
                long long& ncl, Fail& f) {
  const TcPlan p = tc_plan(M, N, K, split_k, sms, cap);
  auto bad = [&](const char* what) {
    std::snprintf(f.msg, sizeof f.msg, "M=%lld N=%lld K=%lld split=%d sms=%d: %s", (long long)M, (long long)N,
                  (long long)K, split_k, sms, what);
    return false;
  };
  TcArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  tc_plan_args(p, a);
  if (p.groups < 1 || p.gs < 1 || p.G != p.groups * p.gs) return bad("grid size");
  if (p.m_tiles != (int)((M + p.BT - 1) / p.BT) || (int64_t)p.m_tiles * p.BT < M) return bad("m-tiles");
  if ((int64_t)p.n_tiles * 128 < N || (int64_t)p.KI * TC_BK < K) return bad("n-tiles / KI");
  if (p.stages < 2 || p.smem > 227 * 1024) return bad("shared memory");
  if (p.cs > 1) {
    ++ncl;
    if (!cap) return bad("cluster plan without cluster support");
    if (p.cs != p.ks * p.gs || p.cs > TC_MAX_CLUSTER || p.ks < 2 || p.G % p.cs != 0) return bad("cluster shape");
    if ((int64_t)cap[p.cs] * p.cs < p.G) return bad("clusters do not fit at once");
    if (p.chunks != 1 || p.ws_bytes != 0 || a.ks != p.ks) return bad("cluster plan fields");
    if ((size_t)p.BT * 128 * 8 > (size_t)p.stages * tc_stage_bytes(p.BT)) return bad("partial tile exceeds stages");
    for (int cta = 0; cta < p.G; ++cta) {
      TcWalk w(a, cta);
      TcSeg s;
      if (!w.next(s)) return bad("cluster CTA without segment");
      const int t = cta / p.cs, r = cta % p.cs, part = r / p.gs, j = r % p.gs;
      if (s.n_tile != t || s.m_tile != j) return bad("cluster CTA on another tile");
      if (s.kb != (int)((int64_t)p.KI * part / p.ks) || s.ke != (int)((int64_t)p.KI * (part + 1) / p.ks))
        return bad("cluster CTA K part");
      if (w.next(s)) return bad("cluster CTA with two segments");
    }
  } else if (a.ks != 0) {
    return bad("cluster reduction flag outside a cluster plan");
  }
  const size_t tiles = (size_t)p.m_tiles * p.n_tiles;
  std::vector<std::vector<std::pair<int, int>>> cov(tiles);
  std::vector<long long> slot_of(tiles, -1);
  const long long slots = (long long)(p.groups - 1) * p.m_tiles;
  for (int cta = 0; cta < p.G; ++cta) {
    TcWalk w(a, cta);
    TcSeg s;
    while (w.next(s)) {
      ++nseg;
      if (s.m_tile < 0 || s.m_tile >= p.m_tiles || s.n_tile < 0 || s.n_tile >= p.n_tiles) return bad("tile range");
      if (s.kb < 0 || s.kb >= s.ke || s.ke > p.KI) return bad("k range");
      const size_t t = (size_t)s.m_tile * p.n_tiles + s.n_tile;
      cov[t].push_back({s.kb, s.ke});
      if (s.kb == 0 && s.ke == p.KI) continue;
      if (p.cs > 1) continue;  // reduced inside the cluster
      const long long sl = tc_split_slot(a, s.n_tile, s.m_tile);
      if (sl < 0 || sl >= slots) return bad("split slot out of range");
      if (slot_of[t] < 0) slot_of[t] = sl;
      else if (slot_of[t] != sl) return bad("contributors of a split tile disagree on its slot");
      if (p.ws_bytes == 0) return bad("split tile in a plan without workspace");
      const size_t acc_end = p.cnt_bytes + (size_t)(sl + 1) * p.BT * 128 * 8;
      if (acc_end > p.ws_bytes || (size_t)(sl + 1) * 4 > p.cnt_bytes) return bad("slot outside workspace");
    }
  }
  std::vector<long long> used;
  for (size_t t = 0; t < tiles; ++t) {
    auto& v = cov[t];
    std::sort(v.begin(), v.end());
    int k = 0;
    for (const auto& seg : v) {
      if (seg.first != k) return bad(seg.first < k ? "k iterations covered twice" : "k iterations not covered");
      k = seg.second;
    }
    if (k != p.KI) return bad("tile not covered to KI");
    if (v.size() > 1 && p.cs > 1) continue;
    if (v.size() > 1) {
      if (slot_of[t] < 0) return bad("split tile without slot");
      used.push_back(slot_of[t]);
    } else if (slot_of[t] >= 0) {
      return bad("whole tile given a slot");
    }
  }
  std::sort(used.begin(), used.end());
  if (std::adjacent_find(used.begin(), used.end()) != used.end()) return bad("two split tiles share a slot");
  return true;
}

}  // namespace

// `planner_check dump`: the automatic plans of the configs[1] shapes on 148 SMs whose clusters sit in groups of 18 SMs
// (one line each: M N K BT m_tiles n_tiles KI gs groups chunks G cs ks ws_bytes), for the plan-choice test.
int dump() {
  int cap[TC_MAX_CLUSTER + 1] = {};
  for (int c = 2; c <= TC_MAX_CLUSTER; ++c) cap[c] = (148 / 18) * (18 / c) + (148 % 18) / c;
  const int64_t shapes[][2] = {{4096, 6144}, {4096, 4096}, {4096, 24576}, {12288, 4096}, {4096, 151936}};
  for (int64_t M : {1, 16, 64, 256, 4096})
    for (const auto& kn : shapes) {
      const TcPlan p = tc_plan(M, kn[1], kn[0], 0, 148, cap);
      std::printf("%lld %lld %lld %d %d %d %d %d %d %d %d %d %d %zu\n", (long long)M, (long long)kn[1],
                  (long long)kn[0], p.BT, p.m_tiles, p.n_tiles, p.KI, p.gs, p.groups, p.chunks, p.G, p.cs, p.ks,
                  p.ws_bytes);
    }
  return 0;
}

int main(int argc, char** argv) {
  if (argc > 1 && std::string(argv[1]) == "dump") return dump();
  const int64_t Ms[] = {1, 8, 9, 16, 17, 33, 64, 65, 100, 128, 129, 256, 300, 1000, 4096};
  const int64_t Ns[] = {1, 100, 128, 129, 1024, 4096, 6144, 24576, 151936};
  const int64_t Ks[] = {1, 100, 128, 1024, 4096, 12288, 65536};
  const int splits[] = {0, 1, 2, 3, 4, 8};
  const int smss[] = {148, 132, 7, 2, 1};
  long long plans = 0, nseg = 0, ncl = 0;
  Fail f;
  for (int model = 0; model < 3; ++model)
    for (int sms : smss) {
      int cap[TC_MAX_CLUSTER + 1] = {};
      for (int c = 2; c <= TC_MAX_CLUSTER; ++c)
        cap[c] = model == 1 ? sms / c : (sms / 18) * (18 / c) + (sms % 18) / c;
      for (int64_t M : Ms)
        for (int64_t N : Ns)
          for (int64_t K : Ks)
            for (int sk : splits) {
              ++plans;
              if (!check_plan(M, N, K, sk, sms, model == 0 ? nullptr : cap, nseg, ncl, f)) {
                std::printf("FAIL %s\n", f.msg);
                return 1;
              }
            }
    }
  std::printf("OK %lld %lld %lld\n", plans, nseg, ncl);
  return 0;
}
