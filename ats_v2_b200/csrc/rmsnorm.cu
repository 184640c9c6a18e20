// RMSNorm and RMSNorm+residual, forward and backward, for sm_100a.
//
// Forward: one warp per row.  A row is read once from HBM as 16-byte chunks
// (lane l owns chunks l, l+32, l+64, ...; consecutive lanes touch consecutive
// 16 B so every warp load is fully coalesced), kept in registers as raw
// chunks, reduced with warp shuffles, and written once: one HBM pass.
//
// Backward: persistent blocks of WARPS warps, one row per warp at a time.
// x and dy are read once into registers, dx is written once; the weight
// gradient of each warp accumulates in its own shared-memory slice (a lane
// owns fixed columns, so no atomics), the block folds its slices in a fixed
// order into one float32 partial row in the workspace, and a small second
// kernel sums the partial rows in block order.  dw is therefore
// deterministic.
//
// Rows longer than the register budget (more than 16 chunks per lane) take
// a streaming variant that reads the row twice (the second read is served
// from L1/L2).
//
// Plain RMSNorm on rows of at most 8 KB (bf16 hidden <= 4096, fp32 <= 2048)
// runs on the TMA ring kernels instead: a persistent CTA per SM in which one
// thread streams whole rows into a shared-memory ring with 1-D bulk copies
// (cp.async.bulk, completion on an mbarrier per slot) while four independent
// groups of two consumer warps each process a row.  The producer keeps 128 KB
// of rows in flight per SM whatever the consumers are doing, which is what
// saturates HBM; every consumer thread owns fixed columns, so (backward) the
// dw accumulators stay in registers.
#include "common.cuh"

#include <mutex>
#include <type_traits>

#include "tc_ptx.cuh"

namespace ats {
namespace {

constexpr int kMaxChunksPerLane = 16;

// Promotion of (x dtype, w dtype) for the residual variant's output.
template <typename A, typename B> struct Promote { typedef float type; };
template <> struct Promote<bf16, bf16> { typedef bf16 type; };

template <typename T>
__device__ __forceinline__ void unpack(const uint4& raw, float (&v)[Chunk<T>::N]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Chunk<T>::N; ++i) v[i] = Cvt<T>::to_f(e[i]);
}

// Unpack N values of T held in Q raw 16-byte chunks.
template <typename T, int N, int Q>
__device__ __forceinline__ void unpack_span(const uint4 (&raw)[Q], float (&v)[N]) {
  static_assert(Q * 16 == N * (int)sizeof(T), "unpack_span: size mismatch");
  const T* e = reinterpret_cast<const T*>(&raw[0]);
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = Cvt<T>::to_f(e[i]);
}

// Load n values of T at p as floats; vectorised when 16-byte aligned sizes allow.
template <typename T, int N>
__device__ __forceinline__ void load_vals(const T* p, float (&v)[N]) {
  if constexpr ((N * sizeof(T)) % 16 == 0) {
    load_n<T, N>(p, v);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = Cvt<T>::to_f(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_vals(T* p, const float (&v)[N]) {
  if constexpr ((N * sizeof(T)) % 16 == 0) {
    store_n<T, N>(p, v);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Cvt<T>::from_f(v[i]);
  }
}

// ----------------------------------------------------------------- forward
// RESID=false: y = round_X(x*r*w)                      (F.rms_norm composite)
// RESID=true : out = round_O(res + round_P(round_X(x*r) * w))  (norm_triton.py:95-98)
template <typename TX, typename TW, bool RESID, int NCH>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(
    const TX* __restrict__ x, int64_t xs, const TX* __restrict__ res, const TW* __restrict__ w,
    void* __restrict__ yv, int64_t ys, float* __restrict__ rstd, int64_t rows, int H, float eps) {
  typedef typename Promote<TX, TW>::type TO_RES;
  typedef typename std::conditional<RESID, TO_RES, TX>::type TO;
  constexpr int N = Chunk<TX>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nch = H / N;
  const TX* xr = x + row * xs;
  uint4 raw[NCH];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = j * 32 + lane;
    if (c < nch) {
      raw[j] = *reinterpret_cast<const uint4*>(xr + (int64_t)c * N);
      float v[N];
      unpack<TX>(raw[j], v);
#pragma unroll
      for (int i = 0; i < N; ++i) ss = fmaf(v[i], v[i], ss);
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
  if (rstd != nullptr && lane == 0) rstd[row] = r;
  TO* y = reinterpret_cast<TO*>(yv) + row * ys;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = j * 32 + lane;
    if (c < nch) {
      float v[N], wv[N], o[N];
      unpack<TX>(raw[j], v);
      load_vals<TW, N>(w + (int64_t)c * N, wv);
      if constexpr (!RESID) {
#pragma unroll
        for (int i = 0; i < N; ++i) o[i] = (v[i] * r) * wv[i];
      } else {
        float rv[N];
        load_vals<TX, N>(res + row * xs + (int64_t)c * N, rv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          const float n1 = round_to<TX>(v[i] * r);
          const float n2 = round_to<TO_RES>(n1 * wv[i]);
          o[i] = rv[i] + n2;
        }
      }
      store_vals<TO, N>(y + (int64_t)c * N, o);
    }
  }
}

// Streaming forward for long rows: pass 1 sums squares, pass 2 re-reads.
template <typename TX, typename TW, bool RESID>
__global__ void __launch_bounds__(256) rmsnorm_fwd_stream_kernel(
    const TX* __restrict__ x, int64_t xs, const TX* __restrict__ res, const TW* __restrict__ w,
    void* __restrict__ yv, int64_t ys, float* __restrict__ rstd, int64_t rows, int H, float eps) {
  typedef typename Promote<TX, TW>::type TO_RES;
  typedef typename std::conditional<RESID, TO_RES, TX>::type TO;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const TX* xr = x + row * xs;
  float ss = 0.f;
  for (int i = lane; i < H; i += 32) {
    const float v = Cvt<TX>::to_f(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
  if (rstd != nullptr && lane == 0) rstd[row] = r;
  TO* y = reinterpret_cast<TO*>(yv) + row * ys;
  for (int i = lane; i < H; i += 32) {
    const float v = Cvt<TX>::to_f(xr[i]);
    const float wv = Cvt<TW>::to_f(w[i]);
    float o;
    if constexpr (!RESID) {
      o = (v * r) * wv;
    } else {
      const float n1 = round_to<TX>(v * r);
      o = Cvt<TX>::to_f(res[row * xs + i]) + round_to<TO_RES>(n1 * wv);
    }
    y[i] = Cvt<TO>::from_f(o);
  }
}

// ---------------------------------------------------------------- backward
// RESID=false: TD = TX; g = dy*w; dx = r*g - x*r^3/H*sum(g*x); dw += dy*x*r.
// RESID=true : TD = promote(X,W); dres = round_X(dout); dn1 = round_X(dout*w);
//              dx = r*dn1 - x*r^3/H*sum(dn1*x); dw += dout*round_X(x*r).
// The per-warp dw slice is lane-interleaved: value i of the lane's j-th chunk
// lives at acc[(j*N + i)*32 + lane], so every shared-memory access of a warp
// touches 32 consecutive words (no bank conflicts).
template <typename TX, typename TW, bool RESID, int NCH>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const void* __restrict__ dyv, const TX* __restrict__ x, const TW* __restrict__ w,
    TX* __restrict__ dx, TX* __restrict__ dres, float* __restrict__ partial,
    int64_t rows, int H, float eps) {
  typedef typename std::conditional<RESID, typename Promote<TX, TW>::type, TX>::type TD;
  constexpr int N = Chunk<TX>::N;
  constexpr int SLICE = NCH * N * 32;
  extern __shared__ float acc_smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* acc = acc_smem + (size_t)warp * SLICE;
  for (int i = lane; i < SLICE; i += 32) acc[i] = 0.f;
  const int nch = H / N;
  const TD* dy = reinterpret_cast<const TD*>(dyv);
  const float invH = 1.0f / (float)H;
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows; row += (int64_t)gridDim.x * warps) {
    const TX* xr = x + row * H;
    const TD* dr = dy + row * H;
    // raw 16-byte chunks: x needs one per chunk, dy (dtype TD) needs DQ
    constexpr int DQ = (N * (int)sizeof(TD)) / 16;
    uint4 xraw[NCH];
    uint4 draw[NCH][DQ];
    float ss = 0.f, c = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int ch = j * 32 + lane;
      if (ch < nch) {
        xraw[j] = *reinterpret_cast<const uint4*>(xr + (int64_t)ch * N);
#pragma unroll
        for (int q = 0; q < DQ; ++q) draw[j][q] = reinterpret_cast<const uint4*>(dr + (int64_t)ch * N)[q];
      }
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int ch = j * 32 + lane;
      if (ch < nch) {
        float v[N], wv[N], d[N];
        unpack<TX>(xraw[j], v);
        unpack_span<TD, N, DQ>(draw[j], d);
        load_vals<TW, N>(w + (int64_t)ch * N, wv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          ss = fmaf(v[i], v[i], ss);
          float g;
          if constexpr (!RESID) g = d[i] * wv[i];
          else g = round_to<TX>(d[i] * wv[i]);
          c = fmaf(g, v[i], c);
        }
      }
    }
    ss = warp_sum(ss);
    c = warp_sum(c);
    const float r = 1.0f / sqrtf(ss * invH + eps);
    const float k2 = r * r * r * c * invH;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int ch = j * 32 + lane;
      if (ch < nch) {
        float v[N], wv[N], o[N], d[N];
        unpack<TX>(xraw[j], v);
        unpack_span<TD, N, DQ>(draw[j], d);
        load_vals<TW, N>(w + (int64_t)ch * N, wv);
        float* a = acc + (j * N) * 32 + lane;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float g;
          if constexpr (!RESID) {
            g = d[i] * wv[i];
            a[i * 32] = fmaf(d[i], v[i] * r, a[i * 32]);
          } else {
            g = round_to<TX>(d[i] * wv[i]);
            a[i * 32] = fmaf(d[i], round_to<TX>(v[i] * r), a[i * 32]);
          }
          o[i] = r * g - v[i] * k2;
        }
        store_vals<TX, N>(dx + row * H + (int64_t)ch * N, o);
        if constexpr (RESID) store_vals<TX, N>(dres + row * H + (int64_t)ch * N, d);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const int ch = c / N, i = c - ch * N;
    const int idx = ((ch >> 5) * N + i) * 32 + (ch & 31);
    float s = 0.f;
    for (int q = 0; q < warps; ++q) s += acc_smem[(size_t)q * SLICE + idx];
    partial[(size_t)blockIdx.x * H + c] = s;
  }
}

// Streaming backward (long rows): reads x and dy twice, dw partial in smem.
template <typename TX, typename TW, bool RESID>
__global__ void __launch_bounds__(256) rmsnorm_bwd_stream_kernel(
    const void* __restrict__ dyv, const TX* __restrict__ x, const TW* __restrict__ w,
    TX* __restrict__ dx, TX* __restrict__ dres, float* __restrict__ partial,
    int64_t rows, int H, float eps) {
  typedef typename std::conditional<RESID, typename Promote<TX, TW>::type, TX>::type TD;
  extern __shared__ float acc_smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* acc = acc_smem + (size_t)warp * H;
  for (int i = lane; i < H; i += 32) acc[i] = 0.f;
  const TD* dy = reinterpret_cast<const TD*>(dyv);
  const float invH = 1.0f / (float)H;
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows; row += (int64_t)gridDim.x * warps) {
    const TX* xr = x + row * H;
    const TD* dr = dy + row * H;
    float ss = 0.f, c = 0.f;
    for (int i = lane; i < H; i += 32) {
      const float v = Cvt<TX>::to_f(xr[i]);
      const float d = Cvt<TD>::to_f(dr[i]);
      const float wv = Cvt<TW>::to_f(w[i]);
      ss = fmaf(v, v, ss);
      const float g = RESID ? round_to<TX>(d * wv) : d * wv;
      c = fmaf(g, v, c);
    }
    ss = warp_sum(ss);
    c = warp_sum(c);
    const float r = 1.0f / sqrtf(ss * invH + eps);
    const float k2 = r * r * r * c * invH;
    for (int i = lane; i < H; i += 32) {
      const float v = Cvt<TX>::to_f(xr[i]);
      const float d = Cvt<TD>::to_f(dr[i]);
      const float wv = Cvt<TW>::to_f(w[i]);
      float g;
      if constexpr (!RESID) {
        g = d * wv;
        acc[i] = fmaf(d, v * r, acc[i]);
      } else {
        g = round_to<TX>(d * wv);
        acc[i] = fmaf(d, round_to<TX>(v * r), acc[i]);
        dres[row * H + i] = Cvt<TX>::from_f(d);
      }
      dx[row * H + i] = Cvt<TX>::from_f(r * g - v * k2);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < warps; ++q) s += acc_smem[(size_t)q * H + i];
    partial[(size_t)blockIdx.x * H + i] = s;
  }
}

// dw[i] = round_W(sum_b partial[b][i]).  A block of 1024 threads takes 32
// columns; thread (c, q) sums the partial rows b = q, q+32, ... of column c
// (a handful of independent loads, so the latency overlaps), and the 32 sums
// are added in q order: a fixed summation order, so dw is deterministic.
constexpr int kReduceLanes = 32;
template <typename TW>
__global__ void __launch_bounds__(32 * kReduceLanes) dw_reduce_kernel(const float* __restrict__ partial, int nblk,
                                                                      int H, TW* __restrict__ dw) {
  __shared__ float part[kReduceLanes][33];
  const int cx = threadIdx.x & 31, q = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + cx;
  float s = 0.f;
  if (col < H) {
#pragma unroll 4
    for (int b = q; b < nblk; b += kReduceLanes) s += partial[(size_t)b * H + col];
  }
  part[q][cx] = s;
  __syncthreads();
  if (q == 0 && col < H) {
    float t = 0.f;
#pragma unroll
    for (int r = 0; r < kReduceLanes; ++r) t += part[r][cx];
    dw[col] = Cvt<TW>::from_f(t);
  }
}

// ---------------------------------------------------------- TMA ring kernels
// One producer thread streams rows into a shared-memory ring with 1-D bulk
// copies.  Eight consumer warps form four independent groups of two warps;
// group g processes rows g, g+4, g+8, ... so four rows are in flight in the
// consumers at any time and their latency chains overlap.  Group thread gt
// owns the 16-byte chunks gt + 64*j of every row; the weight sits in shared
// memory interleaved by gt (conflict-free reads) and the backward's dw
// accumulators stay in registers.  A row's partial sums meet through a small
// shared buffer and one named barrier per group and row (bar.red.and, which
// also makes every member take the same decision when a bounded wait gives
// up, so none is left waiting at the barrier).
constexpr int kGroups = 4;
constexpr int kGroupWarps = 2;
constexpr int kGroupThreads = 32 * kGroupWarps;
constexpr int kConsumerThreads = kGroups * kGroupThreads;
constexpr int kRingThreads = 32 + kConsumerThreads;
constexpr int kSlotsFwd = 16, kSlotsBwd = 8;
constexpr long long kRingBudget = 4000000000LL;  // SM cycles, about 2 s

// Budget of the ring kernels' main-loop waits on this device, read once per
// CTA.  ats_set_wait_budget shortens it so a test can make a wait run out; the
// producer's final wait for its own copies in flight always keeps kRingBudget.
__device__ long long g_ring_wait_budget = kRingBudget;
constexpr int kRingMaxRowBytes = 8192;

// First bounded wait of a ring kernel that gave up (diagnostics; 0 = none).
__device__ int g_ring_status;

__device__ __forceinline__ void ring_fail(volatile int* abort, int code) {
  if (*abort == 0) {
    *abort = 1;
    atomicCAS(&g_ring_status, 0, code);
  }
}

// Named barrier `id` over `count` threads; true only if `ok` held in all of them.
__device__ __forceinline__ bool bar_and(bool ok, int id, int count) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// w staged as float32 in float4 units interleaved by group thread: values
// 4q..4q+3 of chunk gt+64*j form the float4 at ws4[(j*N/4 + q)*64 + gt], so a
// thread reads a chunk's weights with N/4 conflict-free 16-byte loads.
template <typename TW, int NPL, int N>
__device__ __forceinline__ void stage_weight(float* ws, const TW* __restrict__ w, int H, int tid, int nthreads) {
  for (int idx = tid; idx < NPL * N * kGroupThreads; idx += nthreads) {
    const int e4 = idx & 3, v = idx >> 2;
    const int gt = v % kGroupThreads, jq = v / kGroupThreads, q = jq % (N / 4), j = jq / (N / 4);
    const int col = (gt + kGroupThreads * j) * N + q * 4 + e4;
    ws[idx] = col < H ? Cvt<TW>::to_f(w[col]) : 0.f;
  }
}

template <int N>
__device__ __forceinline__ void weight_chunk(const float* ws, int j, int gt, float (&wv)[N]) {
  const float4* w4 = reinterpret_cast<const float4*>(ws);
#pragma unroll
  for (int q = 0; q < N / 4; ++q) {
    const float4 t = w4[(j * (N / 4) + q) * kGroupThreads + gt];
    wv[q * 4 + 0] = t.x;
    wv[q * 4 + 1] = t.y;
    wv[q * 4 + 2] = t.z;
    wv[q * 4 + 3] = t.w;
  }
}

// Rows of this CTA: interleaved (blockIdx.x + i*gridDim.x) or, with
// ATS_RING_CONTIG, one contiguous run per CTA.  Either way fixed per CTA, so
// the backward's per-CTA dw partial sums are deterministic.
#ifndef ATS_RING_CONTIG
#define ATS_RING_CONTIG 1
#endif
__device__ __forceinline__ int64_t ring_row(int64_t i, int64_t rows) {
#if ATS_RING_CONTIG
  return rows * blockIdx.x / gridDim.x + i;
#else
  (void)rows;
  return blockIdx.x + i * gridDim.x;
#endif
}
__device__ __forceinline__ int64_t ring_my_rows(int64_t rows) {
#if ATS_RING_CONTIG
  return rows * (blockIdx.x + 1) / gridDim.x - rows * blockIdx.x / gridDim.x;
#else
  return (rows - blockIdx.x + gridDim.x - 1) / gridDim.x;
#endif
}

// The producer: row ring_row(i) for i < my_rows, into slot i % S.
// `nbytes` per tensor; `second` (may be null) goes to the slot's second half.
template <int S>
__device__ __forceinline__ void ring_produce(uint8_t* ring, uint32_t slot_bytes, uint32_t half_bytes,
                                             const uint8_t* first, const uint8_t* second, int64_t row_stride_bytes,
                                             uint32_t nbytes, int64_t my_rows, int64_t rows, uint64_t* full_bar,
                                             uint64_t* empty_bar, volatile int* abort_flag, int code,
                                             long long budget) {
  int last_par[S];
#pragma unroll
  for (int q = 0; q < S; ++q) last_par[q] = -1;
  const uint32_t tx = second ? 2 * nbytes : nbytes;
  for (int64_t i = 0; i < my_rows && !*abort_flag; ++i) {
    const int slot = (int)(i % S);
    const uint32_t par = (uint32_t)((i / S) & 1);
    if (!tc::mbar_wait(&empty_bar[slot], par ^ 1u, abort_flag, budget)) {
      ring_fail(abort_flag, code);
      break;
    }
    const int64_t off = ring_row(i, rows) * row_stride_bytes;
    tc::mbar_arrive_expect_tx(&full_bar[slot], tx);
    tc::bulk_load(ring + slot * slot_bytes, first + off, nbytes, &full_bar[slot]);
    if (second) tc::bulk_load(ring + slot * slot_bytes + half_bytes, second + off, nbytes, &full_bar[slot]);
    last_par[slot] = (int)par;
  }
  for (int q = 0; q < S; ++q)  // every issued copy lands before the CTA exits
    if (last_par[q] >= 0 && !tc::mbar_wait(&full_bar[q], (uint32_t)last_par[q], nullptr, kRingBudget))
      atomicCAS(&g_ring_status, 0, code + 10);
}

template <typename TX, typename TW, int NPL>
__global__ void __launch_bounds__(kRingThreads, 1) rmsnorm_fwd_ring_kernel(
    const TX* __restrict__ x, int64_t xs, const TW* __restrict__ w, TX* __restrict__ y, int64_t ys,
    float* __restrict__ rstd, int64_t rows, int H, float eps) {
  constexpr int N = Chunk<TX>::N;
  constexpr int S = kSlotsFwd;
  constexpr int WSF = NPL * N * kGroupThreads;  // floats of the staged weight
  extern __shared__ __align__(128) uint8_t smem_ring[];
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S];
  __shared__ float red[kGroups][2][kGroupWarps];
  __shared__ volatile int abort_flag;
  const long long budget = g_ring_wait_budget;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = H / N;
  const uint32_t row_bytes = (uint32_t)H * sizeof(TX);
  const uint32_t slot_bytes = (row_bytes + 127u) & ~127u;
  float* ws = reinterpret_cast<float*>(smem_ring);
  uint8_t* ring = smem_ring + WSF * 4;
  if (threadIdx.x == 0) {
    for (int q = 0; q < S; ++q) {
      tc::mbar_init(&full_bar[q], 1);
      tc::mbar_init(&empty_bar[q], 1);
    }
    tc::fence_barrier_init();
    tc::fence_proxy_async_smem();
    abort_flag = 0;
  }
  stage_weight<TW, NPL, N>(ws, w, H, threadIdx.x, blockDim.x);
  __syncthreads();
  const int64_t my_rows = ring_my_rows(rows);
  if (warp == 0) {
    if (lane == 0)
      ring_produce<S>(ring, slot_bytes, 0, reinterpret_cast<const uint8_t*>(x), nullptr,
                      xs * (int64_t)sizeof(TX), row_bytes, my_rows, rows, full_bar, empty_bar, &abort_flag, 1, budget);
    return;
  }
  const int ct = threadIdx.x - 32;
  const int grp = ct / kGroupThreads, gt = ct % kGroupThreads, gw = gt >> 5;
  int held = -1;  // slot whose row is still being read by this group's bulk store
  for (int64_t i = grp; i < my_rows; i += kGroups) {
    const int slot = (int)(i % S);
    const bool ok = tc::mbar_wait(&full_bar[slot], (uint32_t)((i / S) & 1), &abort_flag, budget);
    const uint4* src = reinterpret_cast<const uint4*>(ring + slot * slot_bytes);
    uint4 raw[NPL];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int c = gt + kGroupThreads * j;
      if (ok && c < nch) {
        raw[j] = src[c];
        float v[N];
        unpack<TX>(raw[j], v);
#pragma unroll
        for (int e = 0; e < N; ++e) ss = fmaf(v[e], v[e], ss);
      }
    }
    ss = warp_sum(ss);
    const int rb = (int)((i / kGroups) & 1);
    if (lane == 0) red[grp][rb][gw] = ss;
    if (!bar_and(ok, 1 + grp, kGroupThreads)) {
      if (gt == 0) ring_fail(&abort_flag, 2);
      break;
    }
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < kGroupWarps; ++q) tot += red[grp][rb][q];
    const float r = 1.0f / sqrtf(tot / (float)H + eps);
    const int64_t row = ring_row(i, rows);
    if (rstd != nullptr && gt == 0) rstd[row] = r;
    TX* yr = y + row * ys;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int c = gt + kGroupThreads * j;
      if (c < nch) {
        float v[N], o[N], wv[N];
        unpack<TX>(raw[j], v);
        weight_chunk<N>(ws, j, gt, wv);
#pragma unroll
        for (int e = 0; e < N; ++e) o[e] = (v[e] * r) * wv[e];
        // y goes back into the slot, over x (already in registers); one bulk store sends the row
        uint4 packed;
        pack_chunk<TX>(o, packed);
        reinterpret_cast<uint4*>(ring + slot * slot_bytes)[c] = packed;
      }
    }
    tc::fence_proxy_async_smem();  // this thread's writes, visible to the bulk copy
    bar_and(true, 1 + grp, kGroupThreads);
    if (gt == 0) {
      tc::bulk_store(yr, ring + slot * slot_bytes, row_bytes);
      tc::bulk_commit();
      tc::bulk_wait_read<1>();  // the previous row's store has read its slot: release it
      if (held >= 0) tc::mbar_arrive(&empty_bar[held]);
    }
    held = slot;
  }
  if (gt == 0) tc::bulk_wait<0>();  // every store of this group complete before the CTA exits
}

template <typename TX, typename TW, int NPL>
__global__ void __launch_bounds__(kRingThreads, 1) rmsnorm_bwd_ring_kernel(
    const TX* __restrict__ dy, const TX* __restrict__ x, const TW* __restrict__ w, TX* __restrict__ dx,
    float* __restrict__ partial, int64_t rows, int H, float eps) {
  constexpr int N = Chunk<TX>::N;
  constexpr int S = kSlotsBwd;
  constexpr int WSF = NPL * N * kGroupThreads;  // floats of the staged weight / of one group's dw fold
  extern __shared__ __align__(128) uint8_t smem_ring[];
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S];
  __shared__ float2 red[kGroups][2][kGroupWarps];
  __shared__ volatile int abort_flag;
  const long long budget = g_ring_wait_budget;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = H / N;
  const uint32_t row_bytes = (uint32_t)H * sizeof(TX);
  const uint32_t half_bytes = (row_bytes + 127u) & ~127u;
  const uint32_t slot_bytes = 2 * half_bytes;  // x row, then dy row
  float* ws = reinterpret_cast<float*>(smem_ring);
  uint8_t* ring = smem_ring + WSF * 4;
  if (threadIdx.x == 0) {
    for (int q = 0; q < S; ++q) {
      tc::mbar_init(&full_bar[q], 1);
      tc::mbar_init(&empty_bar[q], 1);
    }
    tc::fence_barrier_init();
    tc::fence_proxy_async_smem();
    abort_flag = 0;
  }
  stage_weight<TW, NPL, N>(ws, w, H, threadIdx.x, blockDim.x);
  __syncthreads();
  const int64_t my_rows = ring_my_rows(rows);
  if (warp == 0) {
    if (lane == 0)
      ring_produce<S>(ring, slot_bytes, half_bytes, reinterpret_cast<const uint8_t*>(x),
                      reinterpret_cast<const uint8_t*>(dy), (int64_t)H * sizeof(TX), row_bytes, my_rows, rows,
                      full_bar, empty_bar, &abort_flag, 3, budget);
    return;
  }
  const int ct = threadIdx.x - 32;
  const int grp = ct / kGroupThreads, gt = ct % kGroupThreads, gw = gt >> 5;
  const float invH = 1.0f / (float)H;
  float acc[NPL][N];
#pragma unroll
  for (int j = 0; j < NPL; ++j)
#pragma unroll
    for (int e = 0; e < N; ++e) acc[j][e] = 0.f;
  for (int64_t i = grp; i < my_rows; i += kGroups) {
    const int slot = (int)(i % S);
    const bool ok = tc::mbar_wait(&full_bar[slot], (uint32_t)((i / S) & 1), &abort_flag, budget);
    const uint4* sx = reinterpret_cast<const uint4*>(ring + slot * slot_bytes);
    const uint4* sd = reinterpret_cast<const uint4*>(ring + slot * slot_bytes + half_bytes);
    uint4 xr[NPL], dr[NPL];
    float ss = 0.f, cc = 0.f;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int c = gt + kGroupThreads * j;
      if (ok && c < nch) {
        xr[j] = sx[c];
        dr[j] = sd[c];
        float v[N], d[N], wv[N];
        unpack<TX>(xr[j], v);
        unpack<TX>(dr[j], d);
        weight_chunk<N>(ws, j, gt, wv);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          ss = fmaf(v[e], v[e], ss);
          cc = fmaf(d[e] * wv[e], v[e], cc);
        }
      }
    }
    ss = warp_sum(ss);
    cc = warp_sum(cc);
    const int rb = (int)((i / kGroups) & 1);
    if (lane == 0) red[grp][rb][gw] = make_float2(ss, cc);
    if (!bar_and(ok, 1 + grp, kGroupThreads)) {
      if (gt == 0) ring_fail(&abort_flag, 4);
      break;
    }
    if (gt == 0) tc::mbar_arrive(&empty_bar[slot]);
    float tss = 0.f, tcc = 0.f;
#pragma unroll
    for (int q = 0; q < kGroupWarps; ++q) {
      const float2 t = red[grp][rb][q];
      tss += t.x;
      tcc += t.y;
    }
    const float r = 1.0f / sqrtf(tss * invH + eps);
    const float k2 = r * r * r * tcc * invH;
    TX* dxr = dx + ring_row(i, rows) * (int64_t)H;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int c = gt + kGroupThreads * j;
      if (c < nch) {
        float v[N], d[N], o[N], wv[N];
        unpack<TX>(xr[j], v);
        unpack<TX>(dr[j], d);
        weight_chunk<N>(ws, j, gt, wv);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float g = d[e] * wv[e];
          acc[j][e] = fmaf(d[e], v[e] * r, acc[j][e]);
          o[e] = r * g - v[e] * k2;
        }
        store_chunk<TX>(dxr + (int64_t)c * N, o);
      }
    }
  }
  // fold the four groups' dw in the (now idle) ring, then write this block's partial row
  bar_and(true, 5, kConsumerThreads);
  float* fold = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int j = 0; j < NPL; ++j)
#pragma unroll
    for (int e = 0; e < N; ++e) fold[(size_t)grp * WSF + (j * N + e) * kGroupThreads + gt] = acc[j][e];
  bar_and(true, 5, kConsumerThreads);
  for (int c = ct; c < H; c += kConsumerThreads) {
    const int ch = c / N, e = c - ch * N;
    const int idx = ((ch / kGroupThreads) * N + e) * kGroupThreads + (ch % kGroupThreads);
    float s2 = 0.f;
#pragma unroll
    for (int q = 0; q < kGroups; ++q) s2 += fold[(size_t)q * WSF + idx];
    partial[(size_t)blockIdx.x * H + c] = s2;
  }
}

template <typename TX>
bool ring_ok(const void* x, int64_t xs, const void* out, int64_t os, int64_t H, int64_t rows) {
  constexpr int N = Chunk<TX>::N;
  return rows > 0 && (H % N) == 0 && H * (int64_t)sizeof(TX) <= kRingMaxRowBytes && aligned16(x) && aligned16(out) &&
         (xs % N) == 0 && (os % N) == 0;
}

// 16-byte chunks per group thread (1..8 for rows of at most 8 KB).
int ring_npl(int64_t H, int N) {
  const int64_t per = (H / N + kGroupThreads - 1) / kGroupThreads;
  return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8;
}

// ----------------------------------------------------------------- launchers
constexpr int kBwdMaxBlocks = 160;  // upper bound on persistent blocks (>= B200's 148 SMs)
constexpr size_t kBwdSmemBudget = 160 * 1024;

int bwd_warps(int64_t H) {
  int w = (int)(kBwdSmemBudget / ((size_t)H * 4));
  return w < 1 ? 1 : (w > 8 ? 8 : w);
}

int bwd_blocks(int64_t rows, int64_t H) {
  const int warps = bwd_warps(H);
  int64_t need = (rows + warps - 1) / warps;
  int sms = num_sms();
  int b = sms < kBwdMaxBlocks ? sms : kBwdMaxBlocks;
  if (need < b) b = (int)need;
  return b < 1 ? 1 : b;
}

int chunks_per_lane(int64_t H, int N) {
  const int64_t nch = H / N;
  return (int)((nch + 31) / 32);
}

template <typename TX>
bool vec_ok(const void* x, int64_t xs, int64_t H) {
  constexpr int N = Chunk<TX>::N;
  return (H % N) == 0 && (xs % N) == 0 && aligned16(x);
}

template <typename TX, typename TW, bool RESID>
int launch_fwd(const void* x, int64_t xs, const void* res, const void* w, void* y, int64_t ys,
               float* rstd, int64_t rows, int64_t H, float eps, cudaStream_t st) {
  const int warps = 8;
  const dim3 grid((unsigned)((rows + warps - 1) / warps)), block(32 * warps);
  const TX* xp = static_cast<const TX*>(x);
  const TX* rp = static_cast<const TX*>(res);
  const TW* wp = static_cast<const TW*>(w);
  constexpr int N = Chunk<TX>::N;
  const bool vec = vec_ok<TX>(x, xs, H) && aligned16(y) && (ys % N) == 0 &&
                   (!RESID || aligned16(res)) && aligned16(w);
  const int nch = chunks_per_lane(H, N);
  if (!RESID && vec && ring_ok<TX>(x, xs, y, ys, H, rows)) {
    const int npl = ring_npl(H, N);
    const int slot = (int)((H * (int64_t)sizeof(TX) + 127) & ~(int64_t)127);
    const int smem = npl * N * kGroupThreads * 4 + kSlotsFwd * slot;
    int grid = num_sms();
    if (rows < grid) grid = (int)rows;
    TX* yo = static_cast<TX*>(y);
    auto kfn = npl == 1 ? rmsnorm_fwd_ring_kernel<TX, TW, 1>
             : npl == 2 ? rmsnorm_fwd_ring_kernel<TX, TW, 2>
             : npl == 4 ? rmsnorm_fwd_ring_kernel<TX, TW, 4>
                        : rmsnorm_fwd_ring_kernel<TX, TW, 8>;
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kfn<<<grid, kRingThreads, smem, st>>>(xp, xs, wp, yo, ys, rstd, rows, (int)H, eps);
    return check_launch("rmsnorm_fwd_ring");
  }
  if (vec && nch <= kMaxChunksPerLane) {
#define ATS_FWD(NC) rmsnorm_fwd_kernel<TX, TW, RESID, NC><<<grid, block, 0, st>>>(xp, xs, rp, wp, y, ys, rstd, rows, (int)H, eps)
    if (nch <= 1) ATS_FWD(1);
    else if (nch <= 2) ATS_FWD(2);
    else if (nch <= 4) ATS_FWD(4);
    else if (nch <= 8) ATS_FWD(8);
    else ATS_FWD(16);
#undef ATS_FWD
  } else {
    rmsnorm_fwd_stream_kernel<TX, TW, RESID><<<grid, block, 0, st>>>(xp, xs, rp, wp, y, ys, rstd, rows, (int)H, eps);
  }
  return check_launch("rmsnorm_fwd");
}

template <typename TX, typename TW, bool RESID>
int launch_bwd(const void* dy, const void* x, const void* w, void* dx, void* dres, void* dw,
               void* ws, int64_t rows, int64_t H, float eps, cudaStream_t st) {
  constexpr int N = Chunk<TX>::N;
  const int nch = chunks_per_lane(H, N);
  const int ncht = nch <= 1 ? 1 : nch <= 2 ? 2 : nch <= 4 ? 4 : nch <= 8 ? 8 : 16;
  const bool vec = vec_ok<TX>(x, H, H) && aligned16(dy) && aligned16(dx) && aligned16(w) &&
                   (!RESID || aligned16(dres)) && nch <= kMaxChunksPerLane;
  const int64_t slice = vec ? (int64_t)ncht * N * 32 : H;  // floats of one warp's dw slice
  const int warps = bwd_warps(slice);
  const int blocks = bwd_blocks(rows, slice);
  const size_t smem = (size_t)warps * slice * 4;
  float* partial = static_cast<float*>(ws);
  const TX* xp = static_cast<const TX*>(x);
  const TW* wp = static_cast<const TW*>(w);
  if (!RESID && vec && ring_ok<TX>(x, H, dx, H, H, rows) && aligned16(dy)) {
    const int npl = ring_npl(H, N);
    const int64_t half = (H * (int64_t)sizeof(TX) + 127) & ~(int64_t)127;
    // the ring region also holds the final dw fold of the four consumer groups
    const int64_t ring_bytes = kSlotsBwd * 2 * half;
    const int64_t fold_bytes = (int64_t)kGroups * npl * N * kGroupThreads * 4;
    const int smem = npl * N * kGroupThreads * 4 + (int)(ring_bytes > fold_bytes ? ring_bytes : fold_bytes);
    int grid = num_sms() < kBwdMaxBlocks ? num_sms() : kBwdMaxBlocks;
    if (rows < grid) grid = (int)rows;
    const TX* dyp = static_cast<const TX*>(dy);
    TX* dxo = static_cast<TX*>(dx);
    auto kfn = npl == 1 ? rmsnorm_bwd_ring_kernel<TX, TW, 1>
             : npl == 2 ? rmsnorm_bwd_ring_kernel<TX, TW, 2>
             : npl == 4 ? rmsnorm_bwd_ring_kernel<TX, TW, 4>
                        : rmsnorm_bwd_ring_kernel<TX, TW, 8>;
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kfn<<<grid, kRingThreads, smem, st>>>(dyp, xp, wp, dxo, partial, rows, (int)H, eps);
    ATS_TRY(check_launch("rmsnorm_bwd_ring"));
    dw_reduce_kernel<TW><<<(unsigned)((H + 31) / 32), 32 * kReduceLanes, 0, st>>>(partial, grid, (int)H, static_cast<TW*>(dw));
    return check_launch("rmsnorm_dw_reduce");
  }
  if (rows > 0) {
    if (vec) {
#define ATS_BWD(NC)                                                                                        \
  do {                                                                                                     \
    auto kfn = rmsnorm_bwd_kernel<TX, TW, RESID, NC>;                                                     \
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                    \
    kfn<<<blocks, 32 * warps, smem, st>>>(dy, xp, wp, static_cast<TX*>(dx), static_cast<TX*>(dres),      \
                                           partial, rows, (int)H, eps);                                    \
  } while (0)
      if (nch <= 1) ATS_BWD(1);
      else if (nch <= 2) ATS_BWD(2);
      else if (nch <= 4) ATS_BWD(4);
      else if (nch <= 8) ATS_BWD(8);
      else ATS_BWD(16);
#undef ATS_BWD
    } else {
      auto kfn = rmsnorm_bwd_stream_kernel<TX, TW, RESID>;
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kfn<<<blocks, 32 * warps, smem, st>>>(dy, xp, wp, static_cast<TX*>(dx), static_cast<TX*>(dres), partial,
                                             rows, (int)H, eps);
    }
    ATS_TRY(check_launch("rmsnorm_bwd"));
  }
  const int nblk = rows > 0 ? blocks : 0;
  dw_reduce_kernel<TW><<<(unsigned)((H + 31) / 32), 32 * kReduceLanes, 0, st>>>(partial, nblk, (int)H, static_cast<TW*>(dw));
  return check_launch("rmsnorm_dw_reduce");
}

// The backward keeps one float32 dw slice of `hidden` values per warp in shared memory.
constexpr int64_t kBwdMaxHidden = 48 * 1024;

int check_bwd_hidden(int64_t H) {
  if (H > kBwdMaxHidden) return fail(ATS_EUNSUPPORTED, "rmsnorm_bwd: hidden=%lld above %lld", (long long)H, (long long)kBwdMaxHidden);
  return ATS_OK;
}

int check_common(const void* x, ats_dtype xd, const void* w, ats_dtype wd, int64_t rows, int64_t H) {
  if (rows < 0 || H <= 0) return fail(ATS_EBADARG, "rmsnorm: bad shape rows=%lld hidden=%lld", (long long)rows, (long long)H);
  if (H > (1 << 20)) return fail(ATS_EUNSUPPORTED, "rmsnorm: hidden=%lld above 2^20", (long long)H);
  if ((xd != ATS_F32 && xd != ATS_BF16) || (wd != ATS_F32 && wd != ATS_BF16))
    return fail(ATS_EBADARG, "rmsnorm: unsupported dtype");
  if ((rows > 0 && x == nullptr) || w == nullptr) return fail(ATS_EBADARG, "rmsnorm: null pointer");
  return ATS_OK;
}

}  // namespace
}  // namespace ats

using namespace ats;

#define ATS_DISPATCH2(xd, wd, FN, R)                                                      \
  ((xd) == ATS_BF16 ? ((wd) == ATS_BF16 ? FN<bf16, bf16, R> : FN<bf16, float, R>)        \
                    : ((wd) == ATS_BF16 ? FN<float, bf16, R> : FN<float, float, R>))

namespace ats {

int ring_set_wait_budget(long long cycles) {
  const long long v = cycles > 0 ? cycles : kRingBudget;
  cudaError_t e = cudaMemcpyToSymbol(g_ring_wait_budget, &v, sizeof(v));
  if (e != cudaSuccess) return fail(ATS_ECUDA, "set_wait_budget (rmsnorm): %s", cudaGetErrorString(e));
  return ATS_OK;
}

int ring_take_status(int* code) {
  const int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(code, g_ring_status, sizeof(int));
  if (e == cudaSuccess && *code != 0) e = cudaMemcpyToSymbol(g_ring_status, &zero, sizeof(int));
  if (e != cudaSuccess) return fail(ATS_ECUDA, "rmsnorm_status: %s", cudaGetErrorString(e));
  return ATS_OK;
}

}  // namespace ats

extern "C" {

int ats_rmsnorm_status(int* status) {
  if (status == nullptr) return fail(ATS_EBADARG, "rmsnorm_status: null output");
  ATS_TRY(ring_take_status(status));
  return *status == 0 ? ATS_OK : fail(ATS_ETIMEOUT, "rmsnorm: a bounded device wait gave up (code %d)", *status);
}

size_t ats_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t hidden) {
  (void)rows;
  if (hidden <= 0) return 0;
  return (size_t)kBwdMaxBlocks * (size_t)hidden * sizeof(float);
}

int ats_rmsnorm_fwd(const void* x, int64_t x_row_stride, ats_dtype x_dtype, const void* w, ats_dtype w_dtype,
                    void* y, int64_t y_row_stride, float* rstd, int64_t rows, int64_t hidden, float eps,
                    void* stream) {
  ATS_TRY(check_common(x, x_dtype, w, w_dtype, rows, hidden));
  if (rows == 0) return ATS_OK;
  if (y == nullptr) return fail(ATS_EBADARG, "rmsnorm_fwd: null output");
  if (x_row_stride < hidden || y_row_stride < hidden) return fail(ATS_EBADARG, "rmsnorm_fwd: row stride < hidden");
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_fwd, false);
  return fn(x, x_row_stride, nullptr, w, y, y_row_stride, rstd, rows, hidden, eps, (cudaStream_t)stream);
}

int ats_rmsnorm_bwd(const void* dy, const void* x, ats_dtype x_dtype, const void* w, ats_dtype w_dtype, void* dx,
                    void* dw, void* workspace, size_t workspace_bytes, int64_t rows, int64_t hidden, float eps,
                    void* stream) {
  ATS_TRY(check_common(x, x_dtype, w, w_dtype, rows, hidden));
  ATS_TRY(check_bwd_hidden(hidden));
  if (dw == nullptr || (rows > 0 && (dy == nullptr || dx == nullptr)))
    return fail(ATS_EBADARG, "rmsnorm_bwd: null pointer");
  if (workspace == nullptr || workspace_bytes < ats_rmsnorm_bwd_workspace_bytes(rows, hidden))
    return fail(ATS_EBADARG, "rmsnorm_bwd: workspace too small (%zu < %zu)", workspace_bytes,
                ats_rmsnorm_bwd_workspace_bytes(rows, hidden));
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_bwd, false);
  return fn(dy, x, w, dx, nullptr, dw, workspace, rows, hidden, eps, (cudaStream_t)stream);
}

int ats_rmsnorm_residual_fwd(const void* x, const void* residual, ats_dtype x_dtype, const void* w,
                             ats_dtype w_dtype, void* out, int64_t rows, int64_t hidden, float eps,
                             void* stream) {
  ATS_TRY(check_common(x, x_dtype, w, w_dtype, rows, hidden));
  if (rows == 0) return ATS_OK;
  if (residual == nullptr || out == nullptr) return fail(ATS_EBADARG, "rmsnorm_residual_fwd: null pointer");
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_fwd, true);
  return fn(x, hidden, residual, w, out, hidden, nullptr, rows, hidden, eps, (cudaStream_t)stream);
}

int ats_rmsnorm_residual_bwd(const void* dout, const void* x, ats_dtype x_dtype, const void* w, ats_dtype w_dtype,
                             void* dx, void* dresidual, void* dw, void* workspace, size_t workspace_bytes,
                             int64_t rows, int64_t hidden, float eps, void* stream) {
  ATS_TRY(check_common(x, x_dtype, w, w_dtype, rows, hidden));
  ATS_TRY(check_bwd_hidden(hidden));
  if (dw == nullptr || (rows > 0 && (dout == nullptr || dx == nullptr || dresidual == nullptr)))
    return fail(ATS_EBADARG, "rmsnorm_residual_bwd: null pointer");
  if (workspace == nullptr || workspace_bytes < ats_rmsnorm_bwd_workspace_bytes(rows, hidden))
    return fail(ATS_EBADARG, "rmsnorm_residual_bwd: workspace too small");
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_bwd, true);
  return fn(dout, x, w, dx, dresidual, dw, workspace, rows, hidden, eps, (cudaStream_t)stream);
}

}  // extern "C"

// ------------------------------------------------------------ no-alloc variant
// ats_rmsnorm_bwd_noalloc: the same backward kernels, with the per-block dw
// partial sums kept in a fixed device array of this file instead of a
// caller-supplied workspace.  See include/ats_b200.h for the contract.
namespace ats {
namespace {
constexpr int64_t kNoAllocMaxHidden = 8192;
constexpr size_t kNoAllocScratchFloats = (size_t)kBwdMaxBlocks * (size_t)kNoAllocMaxHidden;  // 5 MiB
}  // namespace
}  // namespace ats

// One copy per GPU that loads this library, alive until the process exits.
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[ats::kNoAllocScratchFloats];

namespace ats {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_rmsnorm_bwd_scratch on the current device, looked up
// once per device (the host-side name of the array is not a device address).
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "rmsnorm_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(ATS_EUNSUPPORTED, "rmsnorm_bwd_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(ATS_ECUDA, "rmsnorm_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return ATS_OK;
}
}  // namespace
}  // namespace ats

extern "C" int ats_rmsnorm_bwd_noalloc(const void* dy, const void* x, ats_dtype x_dtype, const void* w,
                                       ats_dtype w_dtype, void* dx, void* dw, int64_t rows, int64_t hidden,
                                       float eps, void* stream) {
  ATS_TRY(check_common(x, x_dtype, w, w_dtype, rows, hidden));
  if (hidden > kNoAllocMaxHidden)
    return fail(ATS_EUNSUPPORTED,
                "rmsnorm_bwd_noalloc: hidden=%lld exceeds the fixed scratch limit of %lld; "
                "use ats_rmsnorm_bwd with a caller workspace",
                (long long)hidden, (long long)kNoAllocMaxHidden);
  if (dw == nullptr || (rows > 0 && (dy == nullptr || dx == nullptr)))
    return fail(ATS_EBADARG, "rmsnorm_bwd_noalloc: null pointer");
  float* scratch = nullptr;
  ATS_TRY(scratch_for_current_device(&scratch));
  // kBwdMaxBlocks partial rows of `hidden` floats fit: hidden <= kNoAllocMaxHidden.
  // Every block that runs writes its whole partial row before the reduce reads
  // it (a block whose bounded wait gave up writes one too), and the reduce
  // reads only those rows, so nothing needs clearing.  A call whose wait gave
  // up (ats_rmsnorm_status) leaves undefined dx and dw; the next call's rows
  // overwrite what it left.
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_bwd, false);
  return fn(dy, x, w, dx, nullptr, dw, scratch, rows, hidden, eps, (cudaStream_t)stream);
}
