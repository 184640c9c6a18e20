// MoE routing and token permutation without host synchronisation.
//
//   route    : one warp per token (blocks of 64 tokens, 8 warps).  Lane l holds logits l, l+32, ...; max and
//              sum are warp reductions, the softmax is float32, top-k is k
//              rounds of a warp arg-max on the logits (softmax is monotone, so
//              this is the probability order; exact ties go to the lower
//              expert index).  Per-block expert counts and probability sums go
//              to the workspace in a fixed order, so the plan is deterministic.
//   plan     : one block.  Block-prefix of the counts (gives every token its
//              stable rank inside its expert), capacity clamp, 128-row padded
//              segment starts, aux loss and utilisation.
//   permute  : same 256-token blocks as route.  A token's rank inside expert e
//              is the block prefix plus the number of earlier tokens of its
//              block that chose e -- the ascending-token order of
//              moe.py:109-116 -- and rank < capacity keeps it.
//   gather / combine / combine_bwd / scatter_grad / route_bwd: one warp per
//              permuted row or per token, 16-byte vector accesses.
#include "moe_plan.cuh"

namespace ats {
namespace {

constexpr int kWarps = 8;                                    // route block: 8 warps
constexpr int kTokPerWarp = kRouteTokensPerBlock / kWarps;  // tokens per route warp

// (value, index) arg-max across the warp: larger value wins, ties -> lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& i, float& pay) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    const float op = __shfl_xor_sync(0xffffffffu, pay, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
      pay = op;
    }
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Softmax pieces of one token for the lane's experts; shared by forward and backward
// so both see bit-identical probabilities.
template <int EPL>
__device__ __forceinline__ void token_softmax(const float* __restrict__ lrow, int E, int lane, float (&l)[EPL],
                                              float (&p)[EPL], float& m, float& s) {
  m = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    l[j] = e < E ? lrow[e] : -INFINITY;
    m = fmaxf(m, l[j]);
  }
  m = warp_max(m);
  float ls = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < E ? expf(l[j] - m) : 0.f;
    ls += p[j];
  }
  s = warp_sum(ls);
#pragma unroll
  for (int j = 0; j < EPL; ++j) p[j] = p[j] / s;
}

template <int EPL, bool PLAN>
__global__ void __launch_bounds__(32 * kWarps) route_kernel(const float* __restrict__ logits, int64_t T,
                                                                     int E, int k, float* __restrict__ gates,
                                                                     int64_t* __restrict__ idx,
                                                                     float* __restrict__ probs, MoePlan plan) {
  extern __shared__ unsigned char smem_raw[];
  int* wcnt = reinterpret_cast<int*>(smem_raw);                    // [kWarps][E]
  float* wprob = reinterpret_cast<float*>(smem_raw) + kWarps * E;  // [kWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (PLAN) {
    for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) wcnt[i] = 0;
    // padding rows of the permuted space are marked before permute fills the kept ones
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < plan.max_rows;
         r += (int64_t)gridDim.x * blockDim.x) {
      plan.row_token[r] = -1;
      plan.row_gate[r] = 0.f;
    }
    __syncthreads();
  }
  float psum[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) psum[j] = 0.f;
  const int64_t t0 = (int64_t)blockIdx.x * kRouteTokensPerBlock + warp * kTokPerWarp;
  for (int q = 0; q < kTokPerWarp; ++q) {
    const int64_t t = t0 + q;
    if (t >= T) break;
    float l[EPL], p[EPL], m, s;
    token_softmax<EPL>(logits + t * E, E, lane, l, p, m, s);
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (probs != nullptr && e < E) probs[t * E + e] = p[j];
      psum[j] += p[j];
    }
    unsigned taken = 0u;
    float sel_p[kMaxTopK];
    int sel_i[kMaxTopK];
    float S = 0.f;
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY, bp = 0.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        if (e < E && !((taken >> j) & 1u) && (l[j] > bv || (l[j] == bv && e < bi))) {
          bv = l[j];
          bi = e;
          bp = p[j];
        }
      }
      warp_argmax(bv, bi, bp);
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      sel_p[r] = bp;
      sel_i[r] = bi;
      S += bp;  // left-to-right sum of the selected probabilities
    }
    if (lane == 0) {
      for (int r = 0; r < k; ++r) {
        gates[t * k + r] = sel_p[r] / S;
        idx[t * k + r] = sel_i[r];
        if (PLAN) wcnt[warp * E + sel_i[r]] += 1;
      }
    }
  }
  if (PLAN) {
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E) wprob[warp * E + e] = psum[j];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int c = 0;
      float ps = 0.f;
      for (int w = 0; w < kWarps; ++w) {
        c += wcnt[w * E + e];
        ps += wprob[w * E + e];
      }
      plan.cnt_partial[(size_t)blockIdx.x * E + e] = c;
      plan.prob_partial[(size_t)blockIdx.x * E + e] = ps;
    }
  }
}

// Inclusive warp scan of v (lane order).
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

// Block-wide exclusive scan of one int per thread (thread order), with the block total, and a float sum over
// the block in a fixed tree (warp shuffles, then the warps in order); blockDim.x a multiple of 32, at most 1024.
__device__ __forceinline__ void block_scan_sum(int v, float f, int& excl, int& total, float& fsum) {
  __shared__ int ws[32];
  __shared__ float wf[32];
  __shared__ int wtotal;
  __shared__ float wfsum;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int incl = warp_incl_scan(v, lane);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) f += __shfl_down_sync(0xffffffffu, f, o);
  if (lane == 31) ws[warp] = incl;
  if (lane == 0) wf[warp] = f;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < nw ? ws[lane] : 0;
    const int wi = warp_incl_scan(w, lane);
    float a = lane < nw ? wf[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_down_sync(0xffffffffu, a, o);
    ws[lane] = wi - w;  // exclusive prefix of the warps
    if (lane == 0) wfsum = a;
    if (lane == 31) wtotal = wi;
  }
  __syncthreads();
  excl = ws[warp] + incl - v;
  total = wtotal;
  fsum = wfsum;
  __syncthreads();  // the shared words are reused by the next call
}

// Phase 1 of the plan, one block per expert: thread i owns a contiguous run of route blocks; the exclusive
// prefix of every (route block, expert) is the block scan of the run sums plus the running sum inside the
// run.  The probability sum goes the same fixed way (run sums, then the block tree): the plan is
// deterministic.
__global__ void __launch_bounds__(1024) plan_expert_kernel(MoePlan plan, int* __restrict__ counts_out) {
  const int e = blockIdx.x, E = plan.E, nb = plan.nb;
  const int per = (nb + (int)blockDim.x - 1) / (int)blockDim.x;
  const int b0 = (int)threadIdx.x * per, b1 = min(nb, b0 + per);
  int c = 0;
  float ps = 0.f;
  for (int b = b0; b < b1; ++b) {
    c += plan.cnt_partial[(size_t)b * E + e];
    ps += plan.prob_partial[(size_t)b * E + e];
  }
  int run, total;
  float psum;
  block_scan_sum(c, ps, run, total, psum);
  for (int b = b0; b < b1; ++b) {
    plan.blk_prefix[(size_t)b * E + e] = run;
    run += plan.cnt_partial[(size_t)b * E + e];
  }
  if (threadIdx.x == 0) {
    const int kept = (int64_t)total < plan.C ? total : (int)plan.C;
    plan.counts[e] = total;
    plan.kept[e] = kept;
    plan.seg_rows[e] = (kept + kSegAlign - 1) / kSegAlign * kSegAlign;
    plan.seg_expert[e] = e;
    const float Tf = (float)plan.T;
    plan.frac[e] = plan.T > 0 ? (float)total / Tf : 0.f;
    plan.prob_mean[e] = plan.T > 0 ? psum / Tf : 0.f;
    if (counts_out) counts_out[e] = total;
  }
}

// Phase 2, one block of 1024 threads: block scan of the padded segment sizes in expert order (the segment
// starts), the aux loss E * lbw * sum(prob_mean * frac) and the utilization frac / sum(frac), the sums in one
// fixed tree.
__global__ void __launch_bounds__(1024) plan_finish_kernel(MoePlan plan, float lbw, float* __restrict__ aux_loss,
                                                           float* __restrict__ util) {
  const int E = plan.E, e = threadIdx.x;
  const int pad = e < E ? (plan.layout == ATS_MOE_SLOTS ? (int)slot_rows(plan.C) : plan.seg_rows[e]) : 0;
  const float fr = e < E ? plan.frac[e] : 0.f;
  int excl, total, unused_excl, unused_total;
  float prod_sum, frac_sum;
  block_scan_sum(pad, e < E ? plan.prob_mean[e] * fr : 0.f, excl, total, prod_sum);
  block_scan_sum(0, fr, unused_excl, unused_total, frac_sum);
  if (e < E) plan.seg_start[e] = excl;
  if (e == 0) {
    plan.seg_start[E] = total;
    plan.dev_err[0] = 0;
    if (aux_loss) aux_loss[0] = (float)E * prod_sum * lbw;
  }
  const float fs = fmaxf(frac_sum, 1e-8f);
  if (util && e < E) util[e] = fr / fs;
}

__global__ void __launch_bounds__(kRouteTokensPerBlock) permute_kernel(const int64_t* __restrict__ idx,
                                                                       const float* __restrict__ gates,
                                                                       MoePlan plan) {
  extern __shared__ int sidx[];  // [256][k]
  const int k = plan.k, E = plan.E;
  const int64_t t = (int64_t)blockIdx.x * kRouteTokensPerBlock + threadIdx.x;
  for (int s = 0; s < k; ++s) sidx[threadIdx.x * k + s] = t < plan.T ? (int)idx[t * k + s] : -1;
  __syncthreads();
  if (t >= plan.T) return;
  for (int s = 0; s < k; ++s) {
    const int e = sidx[threadIdx.x * k + s];
    int local = 0;
    for (int u = 0; u < (int)threadIdx.x; ++u)
      for (int s2 = 0; s2 < k; ++s2) local += (sidx[u * k + s2] == e);
    const int64_t rank = (int64_t)plan.blk_prefix[(size_t)blockIdx.x * E + e] + local;
    int row = -1;
    if (rank < plan.C) {
      row = plan.seg_start[e] + (int)rank;
      plan.row_token[row] = (int)t;
      plan.row_gate[row] = gates[t * k + s];
    }
    plan.tok_row[t * k + s] = row;
  }
}

// Kept rows of a token in ascending expert order.  Segments are laid out in
// expert order, so ascending row index is ascending expert index.

// Rows the grouped GEMMs read: every row of the packed layout; in the slot
// layout only the first align128(kept) rows of each expert's slot (the rest
// of the slot is never read, so it is not written either).
__device__ __forceinline__ bool row_in_segment(const MoePlan& plan, int64_t row) {
  if (row >= plan.seg_start[plan.E]) return false;
  if (plan.layout != ATS_MOE_SLOTS) return true;
  const int64_t cp = slot_rows(plan.C);
  const int e = (int)(row / cp);
  return row - (int64_t)e * cp < plan.seg_rows[e];
}

template <typename T>
__global__ void __launch_bounds__(256) gather_kernel(const T* __restrict__ x, T* __restrict__ xp, int64_t H,
                                                     MoePlan plan, bool vec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (!row_in_segment(plan, row)) return;
  const int tok = plan.row_token[row];
  T* dst = xp + row * H;
  if (vec) {
    constexpr int N = Chunk<T>::N;
    const int64_t nch = H / N;
    for (int64_t c = lane; c < nch; c += 32) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (tok >= 0) v = *reinterpret_cast<const uint4*>(x + (int64_t)tok * H + c * N);
      *reinterpret_cast<uint4*>(dst + c * N) = v;
    }
  } else {
    for (int64_t i = lane; i < H; i += 32) dst[i] = tok >= 0 ? x[(int64_t)tok * H + i] : Cvt<T>::from_f(0.f);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) combine_kernel(const T* __restrict__ y, T* __restrict__ out, int64_t H,
                                                      MoePlan plan, bool vec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= plan.T) return;
  int rows[kMaxTopK];
  const int n = token_rows(plan, t, rows);
  float g[kMaxTopK];
  for (int i = 0; i < n; ++i) g[i] = plan.row_gate[rows[i]];
  if (vec) {
    // four chunks of the first two rows in flight per lane (the loads are latency-bound), then the sums in the
    // same order as one chunk at a time
    constexpr int N = Chunk<T>::N, U = 4;
    const int64_t nc = H / N;
    for (int64_t c0 = lane; c0 < nc; c0 += 32 * U) {
      uint4 w[2][U];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (i < n && c0 + 32 * u < nc)
            w[i][u] = *reinterpret_cast<const uint4*>(y + (int64_t)rows[i] * H + (c0 + 32 * u) * N);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + 32 * u;
        if (c >= nc) break;
        float acc[N];
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] = 0.f;
        for (int i = 0; i < n; ++i) {
          uint4 raw;
          if (i == 0)
            raw = w[0][u];
          else if (i == 1)
            raw = w[1][u];
          else
            raw = *reinterpret_cast<const uint4*>(y + (int64_t)rows[i] * H + c * N);
          const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int e = 0; e < N; ++e)
            acc[e] = round_to<T>(__fadd_rn(acc[e], round_to<T>(__fmul_rn(Cvt<T>::to_f(v[e]), g[i]))));
        }
        store_chunk<T>(out + t * H + c * N, acc);
      }
    }
  } else {
    for (int64_t h = lane; h < H; h += 32) {
      float acc = 0.f;
      for (int i = 0; i < n; ++i)
        acc = round_to<T>(__fadd_rn(acc, round_to<T>(__fmul_rn(Cvt<T>::to_f(y[(int64_t)rows[i] * H + h]), g[i]))));
      out[t * H + h] = Cvt<T>::from_f(acc);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) combine_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ y,
                                                          T* __restrict__ dy, float* __restrict__ dgate_row,
                                                          int64_t H, MoePlan plan, bool vec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (!row_in_segment(plan, row)) return;
  const int tok = plan.row_token[row];
  const float g = plan.row_gate[row];
  float dot = 0.f;
  if (vec) {
    constexpr int N = Chunk<T>::N;
    for (int64_t c = lane; c < H / N; c += 32) {
      float o[N];
      if (tok >= 0) {
        float d[N], yv[N];
        load_chunk<T>(dout + (int64_t)tok * H + c * N, d);
        load_chunk<T>(y + row * H + c * N, yv);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          o[e] = __fmul_rn(d[e], g);
          dot = fmaf(d[e], yv[e], dot);
        }
      } else {
#pragma unroll
        for (int e = 0; e < N; ++e) o[e] = 0.f;
      }
      store_chunk<T>(dy + row * H + c * N, o);
    }
  } else {
    for (int64_t h = lane; h < H; h += 32) {
      float o = 0.f;
      if (tok >= 0) {
        const float d = Cvt<T>::to_f(dout[(int64_t)tok * H + h]);
        o = __fmul_rn(d, g);
        dot = fmaf(d, Cvt<T>::to_f(y[row * H + h]), dot);
      }
      dy[row * H + h] = Cvt<T>::from_f(o);
    }
  }
  dot = warp_sum(dot);
  if (lane == 0) dgate_row[row] = tok >= 0 ? dot : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(256) scatter_grad_kernel(const T* __restrict__ dxp, T* __restrict__ dx, int64_t H,
                                                           MoePlan plan, bool vec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= plan.T) return;
  int rows[kMaxTopK];
  const int n = token_rows(plan, t, rows);
  if (vec) {
    constexpr int N = Chunk<T>::N;
    for (int64_t c = lane; c < H / N; c += 32) {
      float acc[N];
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] = 0.f;
      for (int i = 0; i < n; ++i) {
        float v[N];
        load_chunk<T>(dxp + (int64_t)rows[i] * H + c * N, v);
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] += v[e];
      }
      store_chunk<T>(dx + t * H + c * N, acc);
    }
  } else {
    for (int64_t h = lane; h < H; h += 32) {
      float acc = 0.f;
      for (int i = 0; i < n; ++i) acc += Cvt<T>::to_f(dxp[(int64_t)rows[i] * H + h]);
      dx[t * H + h] = Cvt<T>::from_f(acc);
    }
  }
}

template <int EPL>
__global__ void __launch_bounds__(256) route_bwd_kernel(const float* __restrict__ logits,
                                                        const float* __restrict__ gates,
                                                        const int64_t* __restrict__ idx,
                                                        const float* __restrict__ dgate_row, const float* __restrict__ daux, float lbw,
                                                        float* __restrict__ dlogits, MoePlan plan) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= plan.T) return;
  const int E = plan.E, k = plan.k;
  const float* lrow = logits + t * E;
  float l[EPL], p[EPL], m, s;
  token_softmax<EPL>(lrow, E, lane, l, p, m, s);
  // selected probabilities, recomputed exactly as the forward computed them
  float S = 0.f, Sg = 0.f;
  float dg[kMaxTopK];
  int ei[kMaxTopK];
  for (int r = 0; r < k; ++r) {
    ei[r] = (int)idx[t * k + r];
    const int row = plan.tok_row[t * k + r];
    dg[r] = row >= 0 ? dgate_row[row] : 0.f;
    S += expf(lrow[ei[r]] - m) / s;
    Sg += dg[r] * gates[t * k + r];
  }
  const float coef = (daux != nullptr ? daux[0] : 0.f) * lbw * (float)E / (float)plan.T;
  float dp[EPL];
  float inner = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    float v = 0.f;
    if (e < E) {
      v = coef * plan.frac[e];
      for (int r = 0; r < k; ++r)
        if (ei[r] == e) v += (dg[r] - Sg) / S;
    }
    dp[j] = v;
    inner = fmaf(p[j], v, inner);
  }
  inner = warp_sum(inner);
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    if (e < E) dlogits[t * E + e] = p[j] * (dp[j] - inner);
  }
}

int epl_for(int E) {
  const int need = (E + 31) / 32;
  int epl = 1;
  while (epl < need) epl <<= 1;
  return epl;
}

template <bool PLAN>
int launch_route(const float* logits, int64_t T, int E, int k, float* gates, int64_t* idx, float* probs,
                 const MoePlan& plan, cudaStream_t st) {
  const int nb = (int)((T + kRouteTokensPerBlock - 1) / kRouteTokensPerBlock);
  if (nb == 0) return ATS_OK;
  const size_t smem = PLAN ? (size_t)kWarps * E * 8 : 0;
  const int epl = epl_for(E);
#define ATS_ROUTE(EP)                                                                              \
  do {                                                                                             \
    auto kfn = route_kernel<EP, PLAN>;                                                             \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    kfn<<<nb, 32 * kWarps, smem, st>>>(logits, T, E, k, gates, idx, probs, plan);         \
  } while (0)
  switch (epl) {
    case 1: ATS_ROUTE(1); break;
    case 2: ATS_ROUTE(2); break;
    case 4: ATS_ROUTE(4); break;
    case 8: ATS_ROUTE(8); break;
    case 16: ATS_ROUTE(16); break;
    default: ATS_ROUTE(32); break;
  }
#undef ATS_ROUTE
  return check_launch("moe_route");
}

bool rows_vec(const void* a, const void* b, int64_t H, int N) {
  return aligned16(a) && aligned16(b) && (H % N) == 0;
}

}  // namespace
}  // namespace ats

using namespace ats;

extern "C" {

int64_t ats_moe_max_rows(int64_t T, int E, int k, int64_t capacity, int layout) {
  if (moe_check(T, E, k, capacity, layout) != ATS_OK) return -1;
  return moe_cap_rows(T, E, k, capacity, layout);
}

size_t ats_moe_workspace_bytes(int64_t T, int E, int k, int64_t capacity, int layout) {
  if (moe_check(T, E, k, capacity, layout) != ATS_OK) return 0;
  return moe_plan_carve(nullptr, T, E, k, capacity, layout, nullptr);
}

int ats_moe_status(const void* workspace, size_t workspace_bytes, int64_t T, int E, int k, int64_t capacity,
                   int layout, int* status) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (status == nullptr) return fail(ATS_EBADARG, "moe_status: null output");
  cudaError_t e = cudaMemcpy(status, plan.dev_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "moe_status: %s", cudaGetErrorString(e));
  return *status == 0 ? ATS_OK : fail(ATS_ETIMEOUT, "moe: a bounded device wait gave up (code %d)", *status);
}

int ats_moe_plan_export(const void* workspace, size_t workspace_bytes, int64_t T, int E, int k, int64_t capacity,
                        int layout, int32_t* seg_start, int32_t* row_token, int32_t* kept, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  cudaStream_t st = (cudaStream_t)stream;
  if (seg_start != nullptr &&
      cudaMemcpyAsync(seg_start, plan.seg_start, (size_t)(E + 1) * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return fail(ATS_ECUDA, "moe_plan_export: copy failed");
  if (row_token != nullptr &&
      cudaMemcpyAsync(row_token, plan.row_token, (size_t)plan.max_rows * 4, cudaMemcpyDeviceToDevice, st) !=
          cudaSuccess)
    return fail(ATS_ECUDA, "moe_plan_export: copy failed");
  if (kept != nullptr &&
      cudaMemcpyAsync(kept, plan.kept, (size_t)E * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return fail(ATS_ECUDA, "moe_plan_export: copy failed");
  return ATS_OK;
}

int ats_moe_topk(const float* logits, int64_t T, int E, int k, float* gates, int64_t* idx, float* probs,
                 void* stream) {
  ATS_TRY(moe_check(T, E, k, 1, ATS_MOE_PACKED));
  if (T == 0) return ATS_OK;
  if (logits == nullptr || gates == nullptr || idx == nullptr) return fail(ATS_EBADARG, "moe_topk: null pointer");
  MoePlan none{};
  return launch_route<false>(logits, T, E, k, gates, idx, probs, none, (cudaStream_t)stream);
}

int ats_moe_route_plan(const float* logits, int64_t T, int E, int k, int64_t capacity, int layout, float lbw,
                       float* gates,
                       int64_t* idx, float* aux_loss, float* utilization, int32_t* counts, void* workspace,
                       size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (T > 0 && (logits == nullptr || gates == nullptr || idx == nullptr))
    return fail(ATS_EBADARG, "moe_route_plan: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (T > 0) ATS_TRY(launch_route<true>(logits, T, E, k, gates, idx, nullptr, plan, st));
  else {
    if (cudaMemsetAsync(plan.row_token, 0xff, (size_t)plan.max_rows * 4, st) != cudaSuccess)
      return fail(ATS_ECUDA, "moe_route_plan: memset failed");
  }
  plan_expert_kernel<<<E, 1024, 0, st>>>(plan, counts);
  ATS_TRY(check_launch("moe_plan_experts"));
  plan_finish_kernel<<<1, 1024, 0, st>>>(plan, lbw, aux_loss, utilization);
  ATS_TRY(check_launch("moe_plan_finish"));
  if (T > 0) {
    permute_kernel<<<plan.nb, kRouteTokensPerBlock, (size_t)kRouteTokensPerBlock * k * 4, st>>>(idx, gates, plan);
    ATS_TRY(check_launch("moe_permute"));
  }
  return ATS_OK;
}

int ats_moe_gather(const void* x, void* xp, ats_dtype dtype, int64_t T, int64_t H, int E, int k, int64_t capacity,
                   int layout, const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (H <= 0 || xp == nullptr || (T > 0 && x == nullptr)) return fail(ATS_EBADARG, "moe_gather: bad arguments");
  const unsigned blocks = (unsigned)((plan.max_rows + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    gather_kernel<bf16><<<blocks, 256, 0, st>>>((const bf16*)x, (bf16*)xp, H, plan, rows_vec(x, xp, H, 8));
  else if (dtype == ATS_F32)
    gather_kernel<float><<<blocks, 256, 0, st>>>((const float*)x, (float*)xp, H, plan, rows_vec(x, xp, H, 4));
  else
    return fail(ATS_EBADARG, "moe_gather: dtype");
  return check_launch("moe_gather");
}

int ats_moe_combine(const void* y, void* out, ats_dtype dtype, int64_t T, int64_t H, int E, int k,
                    int64_t capacity, int layout, const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (T == 0) return ATS_OK;
  if (H <= 0 || y == nullptr || out == nullptr) return fail(ATS_EBADARG, "moe_combine: bad arguments");
  const unsigned blocks = (unsigned)((T + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    combine_kernel<bf16><<<blocks, 256, 0, st>>>((const bf16*)y, (bf16*)out, H, plan, rows_vec(y, out, H, 8));
  else if (dtype == ATS_F32)
    combine_kernel<float><<<blocks, 256, 0, st>>>((const float*)y, (float*)out, H, plan, rows_vec(y, out, H, 4));
  else
    return fail(ATS_EBADARG, "moe_combine: dtype");
  return check_launch("moe_combine");
}

int ats_moe_combine_bwd(const void* dout, const void* y, void* dy, float* dgate_row, ats_dtype dtype, int64_t T,
                        int64_t H, int E, int k, int64_t capacity, int layout, const void* workspace, size_t workspace_bytes,
                        void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (H <= 0 || y == nullptr || dy == nullptr || dgate_row == nullptr || (T > 0 && dout == nullptr))
    return fail(ATS_EBADARG, "moe_combine_bwd: bad arguments");
  const unsigned blocks = (unsigned)((plan.max_rows + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    combine_bwd_kernel<bf16><<<blocks, 256, 0, st>>>((const bf16*)dout, (const bf16*)y, (bf16*)dy, dgate_row, H,
                                                     plan, rows_vec(dout, y, H, 8) && aligned16(dy));
  else if (dtype == ATS_F32)
    combine_bwd_kernel<float><<<blocks, 256, 0, st>>>((const float*)dout, (const float*)y, (float*)dy, dgate_row,
                                                      H, plan, rows_vec(dout, y, H, 4) && aligned16(dy));
  else
    return fail(ATS_EBADARG, "moe_combine_bwd: dtype");
  return check_launch("moe_combine_bwd");
}

int ats_moe_scatter_grad(const void* dxp, void* dx, ats_dtype dtype, int64_t T, int64_t H, int E, int k,
                         int64_t capacity, int layout, const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (T == 0) return ATS_OK;
  if (H <= 0 || dxp == nullptr || dx == nullptr) return fail(ATS_EBADARG, "moe_scatter_grad: bad arguments");
  const unsigned blocks = (unsigned)((T + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    scatter_grad_kernel<bf16><<<blocks, 256, 0, st>>>((const bf16*)dxp, (bf16*)dx, H, plan, rows_vec(dxp, dx, H, 8));
  else if (dtype == ATS_F32)
    scatter_grad_kernel<float><<<blocks, 256, 0, st>>>((const float*)dxp, (float*)dx, H, plan,
                                                       rows_vec(dxp, dx, H, 4));
  else
    return fail(ATS_EBADARG, "moe_scatter_grad: dtype");
  return check_launch("moe_scatter_grad");
}

int ats_moe_route_bwd(const float* logits, const float* gates, const int64_t* idx, const float* dgate_row,
                      const float* daux, float* dlogits, int64_t T, int E, int k, int64_t capacity, int layout,
                      float lbw,
                      const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  if (T == 0) return ATS_OK;
  if (logits == nullptr || gates == nullptr || idx == nullptr || dgate_row == nullptr || dlogits == nullptr)
    return fail(ATS_EBADARG, "moe_route_bwd: null pointer");
  const unsigned blocks = (unsigned)((T + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
#define ATS_RB(EP) route_bwd_kernel<EP><<<blocks, 256, 0, st>>>(logits, gates, idx, dgate_row, daux, lbw, dlogits, plan)
  switch (epl_for(E)) {
    case 1: ATS_RB(1); break;
    case 2: ATS_RB(2); break;
    case 4: ATS_RB(4); break;
    case 8: ATS_RB(8); break;
    case 16: ATS_RB(16); break;
    default: ATS_RB(32); break;
  }
#undef ATS_RB
  return check_launch("moe_route_bwd");
}

}  // extern "C"
