// Device-driven row exchange of the expert-parallel MoE layer.
//
// Every rank holds its kept rows in the packed layout: the segment of global
// expert e starts at seg[e] and is its kept count rounded up to 128 rows.  The
// expert side of rank d holds, for each part p of its local experts (experts
// [d*El + p*Ep, +Ep), Ep = El/parts), the segments every source rank keeps for
// them, source by source in rank order -- the layout ats_moe_ep_segments reads.
// So row r of rank s, in the segment of expert e = d*El + p*Ep + j, lives on
// rank d at part p, row
//   base(s, d, p) + (r - seg_s[d*El + p*Ep]),
//   base(s, d, p) = sum over sources q < s of the rounded kept rows q keeps for
//                   the experts of (d, p).
// The counts every rank all-gathered ([W][2E+3] int32: kept[E], Cp, R,
// seg[E+1]) are all the kernels need, so the split sizes never visit the host.
//
//   push: a warp per kept row stores it (16-byte stores) straight into the
//         expert rank's buffer through its mapped address (CUDA IPC); the rows
//         come from the tokens through the plan's row_token (no gathered copy)
//         or from a row buffer in the packed layout.
//   pull: the reverse: a warp per kept row loads it from the expert rank's
//         buffer into the local packed layout.
//   zero: the receiving rank zeroes the padding rows of its own buffer (the
//         K-grouped weight-gradient GEMMs sum over them); peers send only
//         kept rows.
//
// No kernel waits on another rank: the caller orders them with collectives
// (the counts all-gather before a push; a one-element all-reduce after it,
// before the expert GEMMs read the rows; another after the GEMMs, before a
// pull).  Each kernel ends with a system-scope fence.  Every index is checked
// against its buffer before the access; a row that would fall outside is
// skipped and recorded in the exchange status word (ats_device_status).
#include "moe_plan.cuh"

namespace ats {
namespace {

constexpr int kMaxRanks = 64;
constexpr int kXThreads = 256;
constexpr int kXWarps = kXThreads / 32;
constexpr int kUnroll = 8;

}  // namespace

// First failed check of an exchange kernel on this device since the status
// was last taken (0: none).
__device__ int g_ep_status;

namespace {

struct XArgs {
  const int* counts;  // [W][2E+3]
  int W, me, E, El, Ep, part_lo, part_hi;
  const uint64_t* peer;  // [W] part-0 addresses of each rank's expert-side buffer
  int64_t part_rows;     // rows of one part of an expert-side buffer
  int vec;               // 16-byte chunks per row
  int dest_self;         // push: -1 every row; 1 only the rows whose expert rank is this rank; 0 only the others
};

__device__ __forceinline__ int cnt_kept(const XArgs& a, int s, int e) { return a.counts[s * (2 * a.E + 3) + e]; }
__device__ __forceinline__ int cnt_cp(const XArgs& a, int s) { return a.counts[s * (2 * a.E + 3) + a.E]; }
__device__ __forceinline__ int cnt_seg(const XArgs& a, int s, int e) { return a.counts[s * (2 * a.E + 3) + a.E + 2 + e]; }

__device__ __forceinline__ int rounded(int kept, int cp) {
  kept = kept < 0 ? 0 : (kept > cp ? cp : kept);
  return (kept + 127) / 128 * 128;
}

__device__ __forceinline__ void flag(int code) { atomicCAS(&g_ep_status, 0, code); }

// Shared state of a push/pull block: this rank's segment starts and kept
// counts, and base(me, d, p) for every destination rank and part.
struct XShared {
  int seg[kMaxExperts + 1];
  int kept[kMaxExperts];
  int base[kMaxExperts];  // [d * parts + p]
  int ok;
};

__device__ void load_shared(const XArgs& a, XShared& sh) {
  const int parts = a.El / a.Ep;
  const int cp = cnt_cp(a, a.me);
  for (int e = threadIdx.x; e <= a.E; e += blockDim.x) {
    sh.seg[e] = cnt_seg(a, a.me, e);
    if (e < a.E) sh.kept[e] = cnt_kept(a, a.me, e);
  }
  for (int dp = threadIdx.x; dp < a.W * parts; dp += blockDim.x) {
    const int d = dp / parts, p = dp - d * parts;
    int b = 0;
    for (int q = 0; q < a.me; ++q) {
      const int cq = cnt_cp(a, q);
      for (int j = 0; j < a.Ep; ++j) b += rounded(cnt_kept(a, q, d * a.El + p * a.Ep + j), cq);
    }
    sh.base[dp] = b;
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int q = 0; q < a.W; ++q) ok &= cnt_cp(a, q) == cp;  // one capacity: one slot size everywhere
    sh.ok = ok;
    if (!ok) flag(1);
  }
  __syncthreads();
}

// The expert segment of row r (seg[e] <= r < seg[e+1]).
__device__ __forceinline__ int seg_of(const XShared& sh, int E, int r) {
  int lo = 0, hi = E;  // seg[lo] <= r < seg[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sh.seg[mid] <= r) lo = mid; else hi = mid;
  }
  return lo;
}

// Copies one row of `vec` 16-byte chunks with one warp, kUnroll chunks in flight per lane.
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int vec, int lane) {
  for (int c0 = 0; c0 < vec; c0 += 32 * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < vec) v[u] = src[c];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < vec) dst[c] = v[u];
    }
  }
}

// push (to_peer) or pull (!to_peer) of this rank's kept rows.
//   push: local source row = src[row_token[r]] (tokens) or src[r] (rows); remote destination.
//   pull: remote source; local destination dst[r].
__global__ void __launch_bounds__(kXThreads) ep_move_kernel(XArgs a, const uint4* __restrict__ src,
                                                            const int* __restrict__ row_token, int64_t src_rows,
                                                            uint4* __restrict__ dst, int64_t dst_rows, int to_peer) {
  __shared__ XShared sh;
  load_shared(a, sh);
  if (!sh.ok) return;
  const int parts = a.El / a.Ep;
  const int lane = threadIdx.x & 31;
  const int nrows = sh.seg[a.E];
  for (int r = blockIdx.x * kXWarps + (threadIdx.x >> 5); r < nrows; r += gridDim.x * kXWarps) {
    const int e = seg_of(sh, a.E, r);
    if (r - sh.seg[e] >= sh.kept[e]) continue;  // padding row: the receiver zeroes its own
    const int d = e / a.El, p = (e - d * a.El) / a.Ep;
    if (p < a.part_lo || p >= a.part_hi) continue;
    if (a.dest_self >= 0 && (d == a.me) != (a.dest_self == 1)) continue;
    const int64_t prow = (int64_t)sh.base[d * parts + p] + (r - sh.seg[d * a.El + p * a.Ep]);
    if (prow < 0 || prow >= a.part_rows) {
      if (lane == 0) flag(2);
      continue;
    }
    uint4* remote = reinterpret_cast<uint4*>(a.peer[d]) + ((int64_t)p * a.part_rows + prow) * a.vec;
    if (to_peer) {
      int64_t s = r;
      if (row_token != nullptr) s = row_token[r];
      if (s < 0 || s >= src_rows) {
        if (lane == 0) flag(3);
        continue;
      }
      copy_row(remote, src + s * a.vec, a.vec, lane);
    } else {
      if (r >= dst_rows) {
        if (lane == 0) flag(4);
        continue;
      }
      copy_row(dst + (int64_t)r * a.vec, remote, a.vec, lane);
    }
  }
  __threadfence_system();
}

// The pull fused with the combine: token t's output is the sum, in ascending row (= expert) order, of its
// kept rows' expert outputs times their gates, loaded straight from the expert ranks' buffers; every product
// and partial sum is rounded as ats_moe_combine rounds them, so the result is the pull followed by the
// combine, bit for bit.  Each kept row is also stored into the local packed layout `ys`, which the backward's
// combine reads.  A warp per token; the rows of a token are at most kMaxTopK.
template <typename T>
__global__ void __launch_bounds__(kXThreads) ep_combine_kernel(XArgs a, MoePlan plan, T* __restrict__ ys,
                                                               int64_t ys_rows, T* __restrict__ out) {
  __shared__ XShared sh;
  load_shared(a, sh);
  if (!sh.ok) return;
  constexpr int N = Chunk<T>::N;
  const int parts = a.El / a.Ep;
  const int lane = threadIdx.x & 31;
  const int64_t H = (int64_t)a.vec * N;
  for (int64_t t = (int64_t)blockIdx.x * kXWarps + (threadIdx.x >> 5); t < plan.T;
       t += (int64_t)gridDim.x * kXWarps) {
    int rows[kMaxTopK];
    const int n = token_rows(plan, t, rows);
    const uint4* src[kMaxTopK];
    float g[kMaxTopK];
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int r = rows[i];
      const int e = seg_of(sh, a.E, r);
      const int d = e / a.El, p = (e - d * a.El) / a.Ep;
      const int64_t prow = (int64_t)sh.base[d * parts + p] + (r - sh.seg[d * a.El + p * a.Ep]);
      if (r - sh.seg[e] >= sh.kept[e] || prow < 0 || prow >= a.part_rows || r >= ys_rows) {
        ok = false;
        break;
      }
      src[i] = reinterpret_cast<const uint4*>(a.peer[d]) + ((int64_t)p * a.part_rows + prow) * a.vec;
      g[i] = plan.row_gate[r];
    }
    if (!ok) {  // a row outside its buffer: the token is left alone
      if (lane == 0) flag(6);
      continue;
    }
    // kUnroll chunks of the first two rows in flight per lane (remote loads are latency-bound), then the sums
    for (int c0 = lane; c0 < a.vec; c0 += 32 * kUnroll) {
      uint4 w[2][kUnroll];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (i < n && c0 + 32 * u < a.vec) w[i][u] = src[i][c0 + 32 * u];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + 32 * u;
        if (c >= a.vec) break;
        float acc[N];
#pragma unroll
        for (int q = 0; q < N; ++q) acc[q] = 0.f;
        for (int i = 0; i < n; ++i) {
          const uint4 raw = i == 0 ? w[0][u] : (i == 1 ? w[1][u] : src[i][c]);
          reinterpret_cast<uint4*>(ys + (int64_t)rows[i] * H)[c] = raw;
          const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int q = 0; q < N; ++q)
            acc[q] = round_to<T>(__fadd_rn(acc[q], round_to<T>(__fmul_rn(Cvt<T>::to_f(v[q]), g[i]))));
        }
        store_chunk<T>(out + t * H + (int64_t)c * N, acc);
      }
    }
  }
}

// The receiving rank zeroes the padding rows of parts [part_lo, part_hi) of
// its expert-side buffer: one block per (part, source, local expert) segment.
__global__ void __launch_bounds__(kXThreads) ep_zero_kernel(XArgs a, uint4* __restrict__ buf) {
  const int nseg = a.W * a.Ep;  // segments of one part
  const int p = a.part_lo + blockIdx.x / nseg;
  const int sj = blockIdx.x - (p - a.part_lo) * nseg;
  const int s = sj / a.Ep, j = sj - s * a.Ep;
  const int e = a.me * a.El + p * a.Ep + j;
  __shared__ int start_s;
  if (threadIdx.x == 0) {
    int st = 0;
    for (int q = 0; q < s; ++q)
      for (int jj = 0; jj < a.Ep; ++jj) st += rounded(cnt_kept(a, q, a.me * a.El + p * a.Ep + jj), cnt_cp(a, q));
    for (int jj = 0; jj < j; ++jj) st += rounded(cnt_kept(a, s, a.me * a.El + p * a.Ep + jj), cnt_cp(a, s));
    start_s = st;
  }
  __syncthreads();
  const int cp = cnt_cp(a, s);
  int kept = cnt_kept(a, s, e);
  kept = kept < 0 ? 0 : (kept > cp ? cp : kept);
  const int64_t row0 = (int64_t)start_s + kept, row1 = (int64_t)start_s + rounded(kept, cp);
  if (row1 > a.part_rows) {
    if (threadIdx.x == 0) flag(5);
    return;
  }
  uint4* base = buf + (int64_t)p * a.part_rows * a.vec;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int64_t i = row0 * a.vec + threadIdx.x; i < row1 * a.vec; i += blockDim.x) base[i] = z;
}

int check_args(const int32_t* counts, int W, int me, int E_local, int parts, int part_lo, int part_hi,
               const uint64_t* peer, int64_t part_rows, int64_t hidden, ats_dtype dtype, XArgs* a) {
  if (counts == nullptr || peer == nullptr) return fail(ATS_EBADARG, "moe_ep exchange: null counts or addresses");
  if (W < 1 || W > kMaxRanks || me < 0 || me >= W || E_local < 1 || W * E_local > kMaxExperts)
    return fail(ATS_EBADARG, "moe_ep exchange: W=%d rank=%d E_local=%d", W, me, E_local);
  if (parts < 1 || E_local % parts != 0 || part_lo < 0 || part_hi > parts || part_lo >= part_hi)
    return fail(ATS_EBADARG, "moe_ep exchange: parts %d [%d, %d) of %d local experts", parts, part_lo, part_hi,
                E_local);
  if (dtype != ATS_BF16 && dtype != ATS_F32) return fail(ATS_EBADARG, "moe_ep exchange: dtype");
  const int64_t row_bytes = hidden * (dtype == ATS_BF16 ? 2 : 4);
  if (hidden <= 0 || row_bytes % 16 != 0 || row_bytes / 16 > (1 << 20))
    return fail(ATS_EUNSUPPORTED, "moe_ep exchange: rows of %lld bytes (need a multiple of 16)", (long long)row_bytes);
  if (part_rows < 0 || part_rows * (row_bytes / 16) * parts >= ((int64_t)1 << 40))
    return fail(ATS_EBADARG, "moe_ep exchange: part_rows %lld", (long long)part_rows);
  a->counts = counts;
  a->W = W;
  a->me = me;
  a->E = W * E_local;
  a->El = E_local;
  a->Ep = E_local / parts;
  a->part_lo = part_lo;
  a->part_hi = part_hi;
  a->peer = peer;
  a->part_rows = part_rows;
  a->vec = (int)(row_bytes / 16);
  a->dest_self = -1;
  return ATS_OK;
}

// CTAs of a move kernel: enough warps for the rows, at most 4 per SM, or 4 per SM of the `sms` SMs a caller
// leaves to the exchange beside a GEMM held to the others (ats_set_gemm_sm_limit).
int move_grid(int64_t max_rows, int sms) {
  const int64_t want = (max_rows + kXWarps - 1) / kXWarps;
  const int64_t cap = (int64_t)(sms > 0 && sms < num_sms() ? sms : num_sms()) * 4;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

int ep_take_status(int* code) {
  const int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(code, g_ep_status, sizeof(int));
  if (e == cudaSuccess && *code != 0) e = cudaMemcpyToSymbol(g_ep_status, &zero, sizeof(int));
  if (e != cudaSuccess) return fail(ATS_ECUDA, "device_status (exchange): %s", cudaGetErrorString(e));
  return ATS_OK;
}

}  // namespace ats

using namespace ats;

extern "C" {

size_t ats_moe_ep_counts_ints(int E) { return E > 0 ? (size_t)(2 * E + 3) : 0; }

int ats_moe_ep_push(const void* src, const int32_t* row_token, int64_t src_rows, const int32_t* counts, int W,
                    int me, int E_local, int parts, int part_lo, int part_hi, const uint64_t* peer_bufs,
                    int64_t part_rows, int64_t hidden, ats_dtype dtype, int sms, void* stream) {
  XArgs a;
  ATS_TRY(check_args(counts, W, me, E_local, parts, part_lo, part_hi, peer_bufs, part_rows, hidden, dtype, &a));
  if (src == nullptr || src_rows < 0) return fail(ATS_EBADARG, "moe_ep_push: null source");
  if (!aligned16(src)) return fail(ATS_EBADARG, "moe_ep_push: source not 16-byte aligned");
  // every kept row of this rank is < W*E_local*Cp <= the rows the sender's packed layout can hold
  ep_move_kernel<<<move_grid((int64_t)W * part_rows * parts, sms), kXThreads, 0, (cudaStream_t)stream>>>(
      a, static_cast<const uint4*>(src), row_token, src_rows, nullptr, 0, 1);
  return check_launch("moe_ep_push");
}

int ats_moe_ep_push_split(const void* src, const int32_t* row_token, int64_t src_rows, const int32_t* counts, int W,
                          int me, int E_local, int parts, int part_lo, int part_hi, const uint64_t* peer_bufs,
                          int64_t part_rows, int64_t hidden, ats_dtype dtype, int to_self, int sms, void* stream) {
  XArgs a;
  ATS_TRY(check_args(counts, W, me, E_local, parts, part_lo, part_hi, peer_bufs, part_rows, hidden, dtype, &a));
  if (src == nullptr || src_rows < 0) return fail(ATS_EBADARG, "moe_ep_push_split: null source");
  if (!aligned16(src)) return fail(ATS_EBADARG, "moe_ep_push_split: source not 16-byte aligned");
  a.dest_self = to_self ? 1 : 0;
  ep_move_kernel<<<move_grid((int64_t)W * part_rows * parts, sms), kXThreads, 0, (cudaStream_t)stream>>>(
      a, static_cast<const uint4*>(src), row_token, src_rows, nullptr, 0, 1);
  return check_launch("moe_ep_push_split");
}

int ats_moe_ep_pull(void* dst, int64_t dst_rows, const int32_t* counts, int W, int me, int E_local, int parts,
                    int part_lo, int part_hi, const uint64_t* peer_bufs, int64_t part_rows, int64_t hidden,
                    ats_dtype dtype, int sms, void* stream) {
  XArgs a;
  ATS_TRY(check_args(counts, W, me, E_local, parts, part_lo, part_hi, peer_bufs, part_rows, hidden, dtype, &a));
  if (dst == nullptr || dst_rows < 0) return fail(ATS_EBADARG, "moe_ep_pull: null destination");
  if (!aligned16(dst)) return fail(ATS_EBADARG, "moe_ep_pull: destination not 16-byte aligned");
  ep_move_kernel<<<move_grid(dst_rows, sms), kXThreads, 0, (cudaStream_t)stream>>>(a, nullptr, nullptr, 0,
                                                                              static_cast<uint4*>(dst), dst_rows, 0);
  return check_launch("moe_ep_pull");
}

int ats_moe_ep_combine(void* ys, int64_t ys_rows, void* out, int64_t T, int k, int64_t capacity,
                       const void* moe_workspace, size_t moe_workspace_bytes, const int32_t* counts, int W, int me,
                       int E_local, int parts, const uint64_t* peer_bufs, int64_t part_rows, int64_t hidden,
                       ats_dtype dtype, void* stream) {
  XArgs a;
  ATS_TRY(check_args(counts, W, me, E_local, parts, 0, parts, peer_bufs, part_rows, hidden, dtype, &a));
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(moe_workspace, moe_workspace_bytes, T, W * E_local, k, capacity, ATS_MOE_PACKED, &plan));
  if (T == 0) return ATS_OK;
  if (ys == nullptr || out == nullptr || ys_rows < 0 || !aligned16(ys) || !aligned16(out))
    return fail(ATS_EBADARG, "moe_ep_combine: bad output buffers");
  const int64_t want = (T + kXWarps - 1) / kXWarps, cap = (int64_t)num_sms() * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    ep_combine_kernel<bf16><<<grid, kXThreads, 0, st>>>(a, plan, static_cast<bf16*>(ys), ys_rows,
                                                        static_cast<bf16*>(out));
  else
    ep_combine_kernel<float><<<grid, kXThreads, 0, st>>>(a, plan, static_cast<float*>(ys), ys_rows,
                                                         static_cast<float*>(out));
  return check_launch("moe_ep_combine");
}

int ats_moe_ep_zero_padding(void* buf, const int32_t* counts, int W, int me, int E_local, int parts, int part_lo,
                            int part_hi, int64_t part_rows, int64_t hidden, ats_dtype dtype, void* stream) {
  XArgs a;
  const uint64_t dummy = 0;
  ATS_TRY(check_args(counts, W, me, E_local, parts, part_lo, part_hi, &dummy, part_rows, hidden, dtype, &a));
  a.peer = nullptr;
  if (buf == nullptr || !aligned16(buf)) return fail(ATS_EBADARG, "moe_ep_zero_padding: bad buffer");
  const int blocks = (part_hi - part_lo) * W * a.Ep;
  ep_zero_kernel<<<blocks, kXThreads, 0, (cudaStream_t)stream>>>(a, static_cast<uint4*>(buf));
  return check_launch("moe_ep_zero_padding");
}

}  // extern "C"
