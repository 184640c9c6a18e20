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
#include "common.cuh"

#include <mutex>
#include <type_traits>

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

// dw[i] = round_W(sum_b partial[b][i]), blocks summed in index order.
template <typename TW>
__global__ void dw_reduce_kernel(const float* __restrict__ partial, int nblk, int H, TW* __restrict__ dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H) return;
  float s = 0.f;
  for (int b = 0; b < nblk; ++b) s += partial[(size_t)b * H + i];
  dw[i] = Cvt<TW>::from_f(s);
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
  dw_reduce_kernel<TW><<<(unsigned)((H + 255) / 256), 256, 0, st>>>(partial, nblk, (int)H, static_cast<TW*>(dw));
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

extern "C" {

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
  // it, and the reduce reads only those rows, so nothing needs clearing.
  auto fn = ATS_DISPATCH2(x_dtype, w_dtype, launch_bwd, false);
  return fn(dy, x, w, dx, nullptr, dw, scratch, rows, hidden, eps, (cudaStream_t)stream);
}
