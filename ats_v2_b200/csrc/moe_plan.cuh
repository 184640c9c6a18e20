// Workspace layout of the MoE routing plan, shared by every MoE stage.
#pragma once

#include "common.cuh"

namespace ats {

constexpr int kRouteTokensPerBlock = 64;  // tokens per route/permute block (route: 8 warps x 8 tokens)
constexpr int kSegAlign = 128;             // expert segments padded to this many rows
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 16;

struct MoePlan {
  int64_t T;
  int E, k;
  int64_t C;         // capacity per expert
  int nb;            // route blocks
  int64_t max_rows;  // upper bound of permuted (padded) rows
  float* prob_partial;  // [nb][E]
  int* cnt_partial;     // [nb][E]
  int* blk_prefix;      // [nb][E] exclusive prefix over blocks
  int* counts;          // [E] pre-capacity counts
  int* kept;            // [E] min(count, C)
  int* seg_start;       // [E+1] padded segment starts; seg_start[E] = padded total
  float* frac;          // [E] count/T
  float* prob_mean;     // [E]
  int* row_token;       // [max_rows] token of a permuted row, -1 = padding
  float* row_gate;      // [max_rows] gate weight of the row
  int* tok_row;         // [T*k] permuted row of (token, slot), -1 = dropped
  int* dev_err;         // [1] device status: 0, or the code of a bounded wait that gave up
};

inline int64_t moe_cap_rows(int64_t T, int E, int k, int64_t C) {
  const int64_t per = C < T ? C : T;
  int64_t kept = T * k;
  if ((int64_t)E * per < kept) kept = (int64_t)E * per;
  return (int64_t)align_up((size_t)(kept + (int64_t)E * (kSegAlign - 1)), kSegAlign);
}

// Carves `ws` (or computes the size when ws == nullptr).  Every array starts
// on a 256-byte boundary.
inline size_t moe_plan_carve(void* ws, int64_t T, int E, int k, int64_t C, MoePlan* p) {
  const int nb = (int)((T + kRouteTokensPerBlock - 1) / kRouteTokensPerBlock);
  const int64_t mr = moe_cap_rows(T, E, k, C);
  size_t off = 0;
  char* base = static_cast<char*>(ws);
  auto take = [&](size_t bytes) -> void* {
    void* r = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return r;
  };
  MoePlan q;
  q.T = T; q.E = E; q.k = k; q.C = C; q.nb = nb; q.max_rows = mr;
  q.prob_partial = (float*)take((size_t)nb * E * 4);
  q.cnt_partial = (int*)take((size_t)nb * E * 4);
  q.blk_prefix = (int*)take((size_t)nb * E * 4);
  q.counts = (int*)take((size_t)E * 4);
  q.kept = (int*)take((size_t)E * 4);
  q.seg_start = (int*)take((size_t)(E + 1) * 4);
  q.frac = (float*)take((size_t)E * 4);
  q.prob_mean = (float*)take((size_t)E * 4);
  q.row_token = (int*)take((size_t)mr * 4);
  q.row_gate = (float*)take((size_t)mr * 4);
  q.tok_row = (int*)take((size_t)T * k * 4);
  q.dev_err = (int*)take(4);
  if (p) *p = q;
  return off;
}

inline int moe_check(int64_t T, int E, int k, int64_t C) {
  if (T < 0 || E < 1 || E > kMaxExperts || k < 1 || k > kMaxTopK || k > E || C < 1)
    return fail(ATS_EBADARG, "moe: bad sizes T=%lld E=%d k=%d capacity=%lld", (long long)T, E, k, (long long)C);
  if (T * k >= ((int64_t)1 << 31)) return fail(ATS_EUNSUPPORTED, "moe: T*k above 2^31");
  return ATS_OK;
}

inline int moe_plan_from_ws(const void* ws, size_t bytes, int64_t T, int E, int k, int64_t C, MoePlan* p) {
  ATS_TRY(moe_check(T, E, k, C));
  const size_t need = moe_plan_carve(nullptr, T, E, k, C, nullptr);
  if (ws == nullptr || bytes < need)
    return fail(ATS_EBADARG, "moe: workspace too small (%zu < %zu)", bytes, need);
  moe_plan_carve(const_cast<void*>(ws), T, E, k, C, p);
  return ATS_OK;
}

}  // namespace ats
