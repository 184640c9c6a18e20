// Residual add fused with the RMSNorm that follows it (TransformerBlock.forward,
// ats/model/transformer.py:208-212):
//
//   x = residual + attn_out; residual = x; h = post_attention_norm(x)
//
// Forward: s = round(a + b) is written (it is the block's next residual) and
// y = round((s * rstd(s)) * w) -- one pass that reads a and b and writes s and
// y, where the unfused pair reads a and b, writes s, reads s again and writes y.
// Backward: autograd sums two gradients into s, the one the next residual add
// hands back (ds_in) and the RMSNorm backward's; ds = round(round(dnorm) +
// ds_in) goes to both a and b.  One pass reads dy, s and ds_in and writes ds;
// the unfused pair reads dy and s, writes dnorm, then reads dnorm and ds_in and
// writes ds.  dw = sum over rows of dy * s * rstd (float32, per-block partial
// rows summed in a fixed order).
//
// A warp per row; each lane holds its 16-byte chunks of the row in registers.
#include "common.cuh"

namespace ats {
namespace {

constexpr int kFwdWarps = 8;
constexpr int kMaxChunks = 16;  // chunks per lane: rows of at most 512 16-byte chunks
constexpr int kReduceCols = 32, kReduceLanes = 32;

// N consecutive weights as floats: 16-byte loads when they span whole chunks, else one by one.
template <typename TW, int N>
__device__ __forceinline__ void load_w(const TW* p, float (&v)[N]) {
  if constexpr ((N * sizeof(TW)) % 16 == 0) {
    load_n<TW, N>(p, v);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = Cvt<TW>::to_f(p[i]);
  }
}

template <typename TX, typename TW, int NCH>
__global__ void __launch_bounds__(32 * kFwdWarps) add_rmsnorm_fwd_kernel(const TX* __restrict__ a,
                                                                        const TX* __restrict__ b,
                                                                        const TW* __restrict__ w, TX* __restrict__ s,
                                                                        TX* __restrict__ y, int64_t rows, int H,
                                                                        float eps) {
  constexpr int N = Chunk<TX>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kFwdWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nch = H / N;
  const int64_t base = row * H;
  uint4 sraw[NCH];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int ch = j * 32 + lane;
    if (ch < nch) {
      float va[N], vb[N], v[N];
      load_chunk<TX>(a + base + (int64_t)ch * N, va);
      load_chunk<TX>(b + base + (int64_t)ch * N, vb);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        v[i] = round_to<TX>(va[i] + vb[i]);
        ss = fmaf(v[i], v[i], ss);
      }
      pack_chunk<TX>(v, sraw[j]);
      *reinterpret_cast<uint4*>(s + base + (int64_t)ch * N) = sraw[j];
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)H + eps);
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int ch = j * 32 + lane;
    if (ch < nch) {
      float v[N], wv[N], o[N];
      const TX* e = reinterpret_cast<const TX*>(&sraw[j]);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = Cvt<TX>::to_f(e[i]);
      load_w<TW, N>(w + (int64_t)ch * N, wv);
#pragma unroll
      for (int i = 0; i < N; ++i) o[i] = (v[i] * r) * wv[i];
      store_chunk<TX>(y + base + (int64_t)ch * N, o);
    }
  }
}

// dw partial sums live in shared memory, one lane-interleaved slice per warp:
// value i of the lane's j-th chunk at acc[(j*N + i)*32 + lane] (conflict-free).
template <typename TX, typename TW, int NCH>
__global__ void __launch_bounds__(256) add_rmsnorm_bwd_kernel(const TX* __restrict__ dy, const TX* __restrict__ s,
                                                             const TX* __restrict__ ds_in, const TW* __restrict__ w,
                                                             TX* __restrict__ ds, float* __restrict__ partial,
                                                             int64_t rows, int H, float eps) {
  constexpr int N = Chunk<TX>::N;
  constexpr int SLICE = NCH * N * 32;
  extern __shared__ float acc_smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* acc = acc_smem + (size_t)warp * SLICE;
  for (int i = lane; i < SLICE; i += 32) acc[i] = 0.f;
  const int nch = H / N;
  const float invH = 1.0f / (float)H;
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows; row += (int64_t)gridDim.x * warps) {
    const int64_t base = row * H;
    uint4 sraw[NCH], draw[NCH];
    float ss = 0.f, c = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int ch = j * 32 + lane;
      if (ch < nch) {
        sraw[j] = *reinterpret_cast<const uint4*>(s + base + (int64_t)ch * N);
        draw[j] = *reinterpret_cast<const uint4*>(dy + base + (int64_t)ch * N);
      }
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int ch = j * 32 + lane;
      if (ch < nch) {
        float v[N], d[N], wv[N];
        const TX* ev = reinterpret_cast<const TX*>(&sraw[j]);
        const TX* ed = reinterpret_cast<const TX*>(&draw[j]);
        load_w<TW, N>(w + (int64_t)ch * N, wv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          v[i] = Cvt<TX>::to_f(ev[i]);
          d[i] = Cvt<TX>::to_f(ed[i]);
          ss = fmaf(v[i], v[i], ss);
          c = fmaf(d[i] * wv[i], v[i], c);
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
        float v[N], d[N], wv[N], o[N];
        const TX* ev = reinterpret_cast<const TX*>(&sraw[j]);
        const TX* ed = reinterpret_cast<const TX*>(&draw[j]);
        load_w<TW, N>(w + (int64_t)ch * N, wv);
        float add[N];
        if (ds_in != nullptr) {
          load_chunk<TX>(ds_in + base + (int64_t)ch * N, add);
        } else {
#pragma unroll
          for (int i = 0; i < N; ++i) add[i] = 0.f;
        }
        float* accp = acc + (j * N) * 32 + lane;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          v[i] = Cvt<TX>::to_f(ev[i]);
          d[i] = Cvt<TX>::to_f(ed[i]);
          accp[i * 32] = fmaf(d[i], v[i] * r, accp[i * 32]);
          // the RMSNorm gradient rounded to TX, then the other gradient of s added (one more rounding)
          o[i] = round_to<TX>(r * (d[i] * wv[i]) - v[i] * k2) + add[i];
        }
        store_chunk<TX>(ds + base + (int64_t)ch * N, o);
      }
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    const int ch = col / N, i = col - ch * N;
    const int idx = ((ch >> 5) * N + i) * 32 + (ch & 31);
    float t = 0.f;
    for (int q = 0; q < warps; ++q) t += acc_smem[(size_t)q * SLICE + idx];
    partial[(size_t)blockIdx.x * H + col] = t;
  }
}

// dw[c] = sum over the nblk partial rows in block order (32 row lanes, then the lanes in order).
template <typename TW>
__global__ void __launch_bounds__(kReduceCols* kReduceLanes) add_rmsnorm_dw_kernel(const float* __restrict__ partial,
                                                                                 int nblk, int H,
                                                                                 TW* __restrict__ dw) {
  __shared__ float red[kReduceLanes][kReduceCols + 1];
  const int cl = threadIdx.x % kReduceCols, rl = threadIdx.x / kReduceCols;
  const int col = blockIdx.x * kReduceCols + cl;
  float t = 0.f;
  if (col < H)
    for (int q = rl; q < nblk; q += kReduceLanes) t += partial[(size_t)q * H + col];
  red[rl][cl] = t;
  __syncthreads();
  if (rl == 0 && col < H) {
    float u = 0.f;
    for (int q = 0; q < kReduceLanes; ++q) u += red[q][cl];
    dw[col] = Cvt<TW>::from_f(u);
  }
}

int chunks_needed(int64_t H, int N) { return (int)((H / N + 31) / 32); }

int nch_bucket(int n) { return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : n <= 8 ? 8 : 16; }

int bwd_warps(int nchb, int N) {
  const int slice_bytes = nchb * N * 32 * 4;
  int warps = 8;
  while (warps > 1 && warps * slice_bytes > 96 * 1024) warps >>= 1;
  return warps;
}

int bwd_blocks(int64_t rows, int warps) {
  const int64_t want = (rows + warps - 1) / warps;
  const int64_t cap = (int64_t)num_sms() * 2;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

int check(const void* a, const void* b, ats_dtype dt, const void* w, ats_dtype wdt, int64_t rows, int64_t H,
          const char* what) {
  if (dt != ATS_BF16 && dt != ATS_F32) return fail(ATS_EBADARG, "%s: dtype", what);
  if (wdt != ATS_BF16 && wdt != ATS_F32) return fail(ATS_EBADARG, "%s: weight dtype", what);
  if (rows < 0 || H <= 0 || H >= (1 << 30)) return fail(ATS_EBADARG, "%s: rows=%lld hidden=%lld", what,
                                                        (long long)rows, (long long)H);
  if (a == nullptr || b == nullptr || w == nullptr) return fail(ATS_EBADARG, "%s: null input", what);
  const int N = dt == ATS_BF16 ? 8 : 4;
  if (H % N != 0 || chunks_needed(H, N) > kMaxChunks || !aligned16(a) || !aligned16(b) ||
      !aligned16(w))
    return fail(ATS_EUNSUPPORTED, "%s: hidden=%lld needs 16-byte rows of at most %d chunks, aligned", what,
                (long long)H, 32 * kMaxChunks);
  return ATS_OK;
}

template <typename TX, typename TW>
int fwd_t(const void* a, const void* b, const void* w, void* s, void* y, int64_t rows, int64_t H, float eps,
          cudaStream_t st) {
  constexpr int N = Chunk<TX>::N;
  const int nchb = nch_bucket(chunks_needed(H, N));
  const unsigned grid = (unsigned)((rows + kFwdWarps - 1) / kFwdWarps);
  auto* ap = static_cast<const TX*>(a);
  auto* bp = static_cast<const TX*>(b);
  auto* wp = static_cast<const TW*>(w);
  auto* sp = static_cast<TX*>(s);
  auto* yp = static_cast<TX*>(y);
#define ATS_ADD_FWD(NC) add_rmsnorm_fwd_kernel<TX, TW, NC><<<grid, 32 * kFwdWarps, 0, st>>>(ap, bp, wp, sp, yp, rows, (int)H, eps)
  if (nchb == 1) ATS_ADD_FWD(1);
  else if (nchb == 2) ATS_ADD_FWD(2);
  else if (nchb == 4) ATS_ADD_FWD(4);
  else if (nchb == 8) ATS_ADD_FWD(8);
  else ATS_ADD_FWD(16);
#undef ATS_ADD_FWD
  return check_launch("add_rmsnorm_fwd");
}

template <typename TX, typename TW>
int bwd_t(const void* dy, const void* s, const void* ds_in, const void* w, void* ds, void* dw, float* partial,
          int64_t rows, int64_t H, float eps, cudaStream_t st) {
  constexpr int N = Chunk<TX>::N;
  const int nchb = nch_bucket(chunks_needed(H, N));
  const int warps = bwd_warps(nchb, N);
  const int blocks = rows > 0 ? bwd_blocks(rows, warps) : 0;
  const size_t smem = (size_t)warps * nchb * N * 32 * 4;
  auto* dyp = static_cast<const TX*>(dy);
  auto* sp = static_cast<const TX*>(s);
  auto* dip = static_cast<const TX*>(ds_in);
  auto* wp = static_cast<const TW*>(w);
  auto* dsp = static_cast<TX*>(ds);
  if (blocks > 0) {
#define ATS_ADD_BWD(NC)                                                                                      \
  do {                                                                                                       \
    auto kfn = add_rmsnorm_bwd_kernel<TX, TW, NC>;                                                           \
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                      \
    kfn<<<blocks, 32 * warps, smem, st>>>(dyp, sp, dip, wp, dsp, partial, rows, (int)H, eps);              \
  } while (0)
    if (nchb == 1) ATS_ADD_BWD(1);
    else if (nchb == 2) ATS_ADD_BWD(2);
    else if (nchb == 4) ATS_ADD_BWD(4);
    else if (nchb == 8) ATS_ADD_BWD(8);
    else ATS_ADD_BWD(16);
#undef ATS_ADD_BWD
    ATS_TRY(check_launch("add_rmsnorm_bwd"));
  }
  add_rmsnorm_dw_kernel<TW><<<(unsigned)((H + kReduceCols - 1) / kReduceCols), kReduceCols * kReduceLanes, 0, st>>>(
      partial, blocks, (int)H, static_cast<TW*>(dw));
  return check_launch("add_rmsnorm_dw");
}

}  // namespace
}  // namespace ats

using namespace ats;

extern "C" {

int ats_add_rmsnorm_fwd(const void* a, const void* b, ats_dtype dtype, const void* w, ats_dtype w_dtype, void* sum,
                        void* y, int64_t rows, int64_t hidden, float eps, void* stream) {
  ATS_TRY(check(a, b, dtype, w, w_dtype, rows, hidden, "add_rmsnorm_fwd"));
  if (rows == 0) return ATS_OK;
  if (sum == nullptr || y == nullptr || !aligned16(sum) || !aligned16(y))
    return fail(ATS_EBADARG, "add_rmsnorm_fwd: outputs must be non-null and 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16)
    return w_dtype == ATS_BF16 ? fwd_t<bf16, bf16>(a, b, w, sum, y, rows, hidden, eps, st)
                               : fwd_t<bf16, float>(a, b, w, sum, y, rows, hidden, eps, st);
  return w_dtype == ATS_BF16 ? fwd_t<float, bf16>(a, b, w, sum, y, rows, hidden, eps, st)
                             : fwd_t<float, float>(a, b, w, sum, y, rows, hidden, eps, st);
}

size_t ats_add_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t hidden) {
  if (hidden <= 0 || rows < 0) return 0;
  return (size_t)num_sms() * 2 * (size_t)hidden * sizeof(float);
}

int ats_add_rmsnorm_bwd(const void* dy, const void* sum, const void* dsum_in, ats_dtype dtype, const void* w,
                        ats_dtype w_dtype, void* dsum, void* dw, void* workspace, size_t workspace_bytes,
                        int64_t rows, int64_t hidden, float eps, void* stream) {
  ATS_TRY(check(dy, sum, dtype, w, w_dtype, rows, hidden, "add_rmsnorm_bwd"));
  if (dw == nullptr || (rows > 0 && (dsum == nullptr || !aligned16(dsum))) ||
      (dsum_in != nullptr && !aligned16(dsum_in)))
    return fail(ATS_EBADARG, "add_rmsnorm_bwd: bad output or gradient pointer");
  if (workspace == nullptr || workspace_bytes < ats_add_rmsnorm_bwd_workspace_bytes(rows, hidden))
    return fail(ATS_EBADARG, "add_rmsnorm_bwd: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  float* part = static_cast<float*>(workspace);
  if (dtype == ATS_BF16)
    return w_dtype == ATS_BF16 ? bwd_t<bf16, bf16>(dy, sum, dsum_in, w, dsum, dw, part, rows, hidden, eps, st)
                               : bwd_t<bf16, float>(dy, sum, dsum_in, w, dsum, dw, part, rows, hidden, eps, st);
  return w_dtype == ATS_BF16 ? bwd_t<float, bf16>(dy, sum, dsum_in, w, dsum, dw, part, rows, hidden, eps, st)
                             : bwd_t<float, float>(dy, sum, dsum_in, w, dsum, dw, part, rows, hidden, eps, st);
}

}  // extern "C"
