// Workspace layout of the MoE routing plan, shared by every MoE stage, and the
// segment table the grouped expert GEMMs walk.
#pragma once

#include "common.cuh"

namespace ats {

constexpr int kRouteTokensPerBlock = 64;  // tokens per route/permute block (route: 8 warps x 8 tokens)
constexpr int kSegAlign = 128;            // expert segments padded to this many rows
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 16;

// Layouts of the permuted row space.
//   ATS_MOE_PACKED: expert e's kept rows follow expert e-1's, each segment
//     padded to a multiple of 128 rows (the single-GPU layout).
//   ATS_MOE_SLOTS: expert e owns the fixed slots [e*Cp, (e+1)*Cp) with
//     Cp = capacity rounded up to 128, so the buffer is [rank][local expert][Cp]
//     for the expert-parallel exchange (equal splits).

// The grouped GEMMs' view of the permuted rows: segments of rows that share an
// expert's weights.  M-grouped GEMMs tile every segment; weight-gradient GEMMs
// reduce over all segments of an expert.
struct SegTable {
  const int* row0;    // [nseg] first permuted row of the segment
  const int* rows;    // [nseg] rows to compute: a multiple of 128, padding rows are zero
  const int* expert;  // [nseg] weight index of the segment
  const int* eseg;    // [E*spe] segments of expert e: eseg[e*spe + q]
  int nseg, spe, E;
  int64_t max_rows;      // rows of the permuted buffers
  int64_t max_seg_rows;  // upper bound of rows[s]
  int* err;              // device status word
  const int* kept = nullptr;  // [nseg] kept (non-padding) rows of the segment, or null: every row.  The
                              // K-grouped GEMMs reduce over them rounded up to 64 (one K block), not over
                              // the zero padding to 128
};

struct MoePlan {
  int64_t T;
  int E, k;
  int64_t C;         // capacity per expert
  int layout;        // ATS_MOE_PACKED or ATS_MOE_SLOTS
  int nb;            // route blocks
  int64_t max_rows;  // upper bound of permuted (padded) rows
  float* prob_partial;  // [nb][E]
  int* cnt_partial;     // [nb][E]
  int* blk_prefix;      // [nb][E] exclusive prefix over blocks
  int* counts;          // [E] pre-capacity counts
  int* kept;            // [E] min(count, C)
  int* seg_start;       // [E+1] segment starts; seg_start[E] = end of the row space
  int* seg_rows;        // [E] rows each segment computes (kept rounded up to 128)
  int* seg_expert;      // [E] identity map (segment e uses expert e)
  float* frac;          // [E] count/T
  float* prob_mean;     // [E]
  int* row_token;       // [max_rows] token of a permuted row, -1 = padding
  float* row_gate;      // [max_rows] gate weight of the row
  int* tok_row;         // [T*k] permuted row of (token, slot), -1 = dropped
  int* dev_err;         // [1] device status: 0, or the code of a bounded wait that gave up
};

__host__ __device__ inline int64_t slot_rows(int64_t C) { return (C + kSegAlign - 1) / kSegAlign * kSegAlign; }

// The kept permuted rows of token t, ascending (= ascending expert): the order the combine sums them in.
__device__ __forceinline__ int token_rows(const MoePlan& plan, int64_t t, int (&rows)[kMaxTopK]) {
  int n = 0;
  for (int s = 0; s < plan.k; ++s) {
    const int r = plan.tok_row[t * plan.k + s];
    if (r < 0) continue;
    int p = n++;
    while (p > 0 && rows[p - 1] > r) {
      rows[p] = rows[p - 1];
      --p;
    }
    rows[p] = r;
  }
  return n;
}

inline int64_t moe_cap_rows(int64_t T, int E, int k, int64_t C, int layout) {
  if (layout == ATS_MOE_SLOTS) return (int64_t)E * slot_rows(C);
  const int64_t per = C < T ? C : T;
  int64_t kept = T * k;
  if ((int64_t)E * per < kept) kept = (int64_t)E * per;
  return (int64_t)align_up((size_t)(kept + (int64_t)E * (kSegAlign - 1)), kSegAlign);
}

// Carves `ws` (or computes the size when ws == nullptr).  Every array starts
// on a 256-byte boundary.
inline size_t moe_plan_carve(void* ws, int64_t T, int E, int k, int64_t C, int layout, MoePlan* p) {
  const int nb = (int)((T + kRouteTokensPerBlock - 1) / kRouteTokensPerBlock);
  const int64_t mr = moe_cap_rows(T, E, k, C, layout);
  size_t off = 0;
  char* base = static_cast<char*>(ws);
  auto take = [&](size_t bytes) -> void* {
    void* r = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return r;
  };
  MoePlan q;
  q.T = T; q.E = E; q.k = k; q.C = C; q.layout = layout; q.nb = nb; q.max_rows = mr;
  q.prob_partial = (float*)take((size_t)nb * E * 4);
  q.cnt_partial = (int*)take((size_t)nb * E * 4);
  q.blk_prefix = (int*)take((size_t)nb * E * 4);
  q.counts = (int*)take((size_t)E * 4);
  q.kept = (int*)take((size_t)E * 4);
  q.seg_start = (int*)take((size_t)(E + 1) * 4);
  q.seg_rows = (int*)take((size_t)E * 4);
  q.seg_expert = (int*)take((size_t)E * 4);
  q.frac = (float*)take((size_t)E * 4);
  q.prob_mean = (float*)take((size_t)E * 4);
  q.row_token = (int*)take((size_t)mr * 4);
  q.row_gate = (float*)take((size_t)mr * 4);
  q.tok_row = (int*)take((size_t)T * k * 4);
  q.dev_err = (int*)take(4);
  if (p) *p = q;
  return off;
}

inline int moe_check(int64_t T, int E, int k, int64_t C, int layout) {
  if (T < 0 || E < 1 || E > kMaxExperts || k < 1 || k > kMaxTopK || k > E || C < 1)
    return fail(ATS_EBADARG, "moe: bad sizes T=%lld E=%d k=%d capacity=%lld", (long long)T, E, k, (long long)C);
  if (layout != ATS_MOE_PACKED && layout != ATS_MOE_SLOTS) return fail(ATS_EBADARG, "moe: unknown layout %d", layout);
  if (T * k >= ((int64_t)1 << 31)) return fail(ATS_EUNSUPPORTED, "moe: T*k above 2^31");
  if (moe_cap_rows(T, E, k, C, layout) >= ((int64_t)1 << 31)) return fail(ATS_EUNSUPPORTED, "moe: row space above 2^31");
  return ATS_OK;
}

inline int moe_plan_from_ws(const void* ws, size_t bytes, int64_t T, int E, int k, int64_t C, int layout,
                            MoePlan* p) {
  ATS_TRY(moe_check(T, E, k, C, layout));
  const size_t need = moe_plan_carve(nullptr, T, E, k, C, layout, nullptr);
  if (ws == nullptr || bytes < need)
    return fail(ATS_EBADARG, "moe: workspace too small (%zu < %zu)", bytes, need);
  moe_plan_carve(const_cast<void*>(ws), T, E, k, C, layout, p);
  return ATS_OK;
}

// The plan's own segment table: one segment per expert, identity expert map.
inline SegTable plan_segments(const MoePlan& p) {
  SegTable s;
  s.row0 = p.seg_start;
  s.rows = p.seg_rows;
  s.expert = p.seg_expert;
  s.eseg = p.seg_expert;  // identity: expert e's only segment is e
  s.nseg = p.E;
  s.spe = 1;
  s.E = p.E;
  s.max_rows = p.max_rows;
  const int64_t per = p.C < p.T ? p.C : p.T;
  s.max_seg_rows = (int64_t)align_up((size_t)(per > 0 ? per : 1), kSegAlign);
  s.err = p.dev_err;
  s.kept = p.kept;
  return s;
}

}  // namespace ats
