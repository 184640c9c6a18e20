// MoE router GEMMs on the tensor cores, for bf16 tokens and a float32 router
// weight (the float32 router of moe.py:76-90 computed as x.float() @ w.T).
//
// A float32 operand v is split into three bf16 parts p0 = bf16(v),
// p1 = bf16(v - p0), p2 = bf16(v - p0 - p1); each difference is exact, and
// v - p0 - p1 - p2 is below 2^-24 |v|, so p0 + p1 + p2 carries the float32
// value.  A bf16 x bf16 product is exact in float32, so summing the part
// products in the float32 accumulator gives a float32 GEMM up to summation
// order:
//   forward   logits = x . (w0 + w1 + w2)^T (+ bias)                  3 parts
//   token     dx = dl . w over the part pairs (0,0) (0,1) (0,2) (1,0) (1,1) (2,0)
//             (the others are below 2^-24 of the leading term), fused
//             with the un-permute of the expert-row gradients, so the
//             token gradient is written once
//   weight    dw^T = x^T . (dl0 + dl1 + dl2), split over token chunks so
//             every SM has tiles, the chunks summed in a fixed order
// The bf16 tokens are exact in every part product, so no token part is needed.
#include "moe_gemm.cuh"

namespace ats {
namespace {

constexpr int kMaxChunks = 16;

struct RouterWs {
  int* tab;        // segment tables (see router_tables_kernel) and a status word
  bf16* wparts;    // [3][Ep][H]
  bf16* dlparts;   // [T][3][Ep]
  float* partial;  // [KS][H][Ep]
  int KS, Ep;
  int64_t chunk;   // token rows per weight-gradient chunk (multiple of 64)
};

int router_ep(int) { return kRouterEp; }

// Token chunks of the router weight gradient: the chunk count whose tiles (H/128 per chunk) fill `ctas` CTAs
// in the fewest, least ragged waves -- cost = waves x (K blocks of a chunk + 4, the fixed cost of a tile in K
// blocks); ties go to fewer chunks (fewer partial sums).  At 32768 tokens, hidden 4096 and 148 SMs: 9 chunks
// (288 tiles, 2 waves of 57 K blocks) where one chunk per 32 SMs gave 5 (160 tiles: 12 SMs ran a second
// 103-block tile while the others idled).
int router_chunks(int64_t T, int64_t H, int ctas) {
  const int64_t tiles = H / 128;
  const int64_t kb = (T + 63) / 64;
  const int64_t maxk = kb < kMaxChunks ? kb : kMaxChunks;
  int64_t best = 1, best_cost = -1;
  for (int64_t ks = 1; ks <= maxk; ++ks) {
    const int64_t waves = (ks * tiles + ctas - 1) / ctas;
    const int64_t cost = waves * ((kb + ks - 1) / ks + 4);
    if (best_cost < 0 || cost < best_cost) {
      best = ks;
      best_cost = cost;
    }
  }
  return (int)best;
}

bool router_supported(ats_dtype dt, int64_t T, int64_t H, int E) {
  return dt == ATS_BF16 && H % 128 == 0 && H >= 128 && H < (1 << 24) && T >= 128 && T < (1 << 30) && E >= 1 &&
         E <= kRouterEp;
}

size_t router_carve(void* ws, int64_t T, int64_t H, int E, RouterWs* o) {
  RouterWs q;
  q.Ep = router_ep(E);
  // the device's SM count, not a caller's SM limit: the chunks fix the summation order of the weight gradient,
  // which must not depend on what runs beside it
  q.KS = router_chunks(T, H, num_sms());
  const int64_t tk = (T + 63) / 64 * 64;
  q.chunk = ((tk + q.KS - 1) / q.KS + 63) / 64 * 64;
  size_t off = 0;
  char* base = static_cast<char*>(ws);
  auto take = [&](size_t bytes) -> void* {
    void* r = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return r;
  };
  q.tab = (int*)take((size_t)(5 + 4 * kMaxChunks) * 4);
  q.wparts = (bf16*)take((size_t)3 * q.Ep * H * 2);
  q.dlparts = (bf16*)take((size_t)T * 3 * q.Ep * 2);
  q.partial = (float*)take((size_t)q.KS * H * q.Ep * 4);
  if (o) *o = q;
  return off;
}

int router_ws(void* ws, size_t bytes, int64_t T, int64_t H, int E, RouterWs* o) {
  const size_t need = router_carve(nullptr, T, H, E, nullptr);
  if (ws == nullptr || bytes < need) return fail(ATS_EBADARG, "moe_router: workspace too small (%zu < %zu)", bytes, need);
  router_carve(ws, T, H, E, o);
  return ATS_OK;
}

// tab: [0..3] the one-segment table of the token GEMMs (row0, rows, expert, eseg);
//      [4 + c*kMaxChunks + g] column c of the chunk table (row0, rows, expert, eseg);
//      [4 + 4*kMaxChunks] status word.
__global__ void router_tables_kernel(int* tab, int T, int KS, int chunk) {
  const int tk = (T + 63) / 64 * 64;
  if (threadIdx.x == 0) {
    tab[0] = 0;
    tab[1] = (T + 127) / 128 * 128;
    tab[2] = 0;
    tab[3] = 0;
    tab[4 + 4 * kMaxChunks] = 0;
  }
  for (int g = threadIdx.x; g < KS; g += blockDim.x) {
    const int r0 = g * chunk;
    const int rows = r0 >= tk ? 0 : (tk - r0 < chunk ? tk - r0 : chunk);
    tab[4 + g] = r0 < tk ? r0 : 0;
    tab[4 + kMaxChunks + g] = rows;
    tab[4 + 2 * kMaxChunks + g] = g;
    tab[4 + 3 * kMaxChunks + g] = g;
  }
}

SegTable one_table(const RouterWs& q, int64_t T) {
  SegTable s;
  s.row0 = q.tab;
  s.rows = q.tab + 1;
  s.expert = q.tab + 2;
  s.eseg = q.tab + 3;
  s.nseg = 1;
  s.spe = 1;
  s.E = 1;
  s.max_rows = (T + 127) / 128 * 128;
  s.max_seg_rows = s.max_rows;
  s.err = q.tab + 4 + 4 * kMaxChunks;
  return s;
}

SegTable chunk_table(const RouterWs& q, int64_t T) {
  SegTable s;
  s.row0 = q.tab + 4;
  s.rows = q.tab + 4 + kMaxChunks;
  s.expert = q.tab + 4 + 2 * kMaxChunks;
  s.eseg = q.tab + 4 + 3 * kMaxChunks;
  s.nseg = q.KS;
  s.spe = 1;
  s.E = q.KS;
  s.max_rows = (T + 63) / 64 * 64;
  s.max_seg_rows = q.chunk;
  s.err = q.tab + 4 + 4 * kMaxChunks;
  return s;
}

__device__ __forceinline__ void split3(float v, bf16& p0, bf16& p1, bf16& p2) {
  p0 = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(p0);
  p1 = __float2bfloat16_rn(r1);
  p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
}

// w [E][H] float32 -> parts [3][Ep][H] bf16 (rows E..Ep-1 zero)
__global__ void __launch_bounds__(256) split_w_kernel(const float* __restrict__ w, int E, int64_t H, int Ep,
                                                      bf16* __restrict__ out) {
  const int64_t n = (int64_t)Ep * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i / H;
    const float v = e < E ? w[i] : 0.f;
    bf16 a, b, c;
    split3(v, a, b, c);
    out[i] = a;
    out[n + i] = b;
    out[2 * n + i] = c;
  }
}

// dl [T][E] float32 -> parts [T][3][Ep] bf16 (columns E..Ep-1 zero)
__global__ void __launch_bounds__(256) split_dl_kernel(const float* __restrict__ dl, int64_t T, int E, int Ep,
                                                       bf16* __restrict__ out) {
  const int64_t n = T * Ep;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / Ep;
    const int e = (int)(i - t * Ep);
    const float v = e < E ? dl[t * E + e] : 0.f;
    bf16 a, b, c;
    split3(v, a, b, c);
    bf16* o = out + t * 3 * Ep + e;
    o[0] = a;
    o[Ep] = b;
    o[2 * Ep] = c;
  }
}

// dw[e][h] = sum over chunks g (in order) of partial[g][h][e], through a 32 x 32 transpose tile
__global__ void __launch_bounds__(256) router_dw_reduce_kernel(const float* __restrict__ partial, int KS,
                                                               int64_t H, int E, int Ep, float* __restrict__ dw) {
  __shared__ float tile[32][33];
  const int64_t h0 = (int64_t)blockIdx.x * 32;
  const int e0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t h = h0 + r;
    const int e = e0 + threadIdx.x;
    float s = 0.f;
    if (h < H && e < Ep)
      for (int g = 0; g < KS; ++g) s += partial[((int64_t)g * H + h) * Ep + e];
    tile[r][threadIdx.x] = s;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int e = e0 + r;
    const int64_t h = h0 + threadIdx.x;
    if (e < E && h < H) dw[(int64_t)e * H + h] = tile[threadIdx.x][r];
  }
}

unsigned grid_for(int64_t n) {
  int64_t b = (n + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  return (unsigned)(b < 1 ? 1 : b > cap ? cap : b);
}

int prepare(RouterWs& q, const float* w, int64_t T, int64_t H, int E, cudaStream_t st) {
  router_tables_kernel<<<1, 32, 0, st>>>(q.tab, (int)T, q.KS, (int)q.chunk);
  ATS_TRY(check_launch("moe_router_tables"));
  split_w_kernel<<<grid_for((int64_t)q.Ep * H), 256, 0, st>>>(w, E, H, q.Ep, q.wparts);
  return check_launch("moe_router_split_w");
}

}  // namespace
}  // namespace ats

using namespace ats;

extern "C" {

int ats_moe_router_supported(ats_dtype x_dtype, int64_t T, int64_t H, int E) {
  return router_supported(x_dtype, T, H, E) ? 1 : 0;
}

size_t ats_moe_router_workspace_bytes(int64_t T, int64_t H, int E) {
  if (!router_supported(ATS_BF16, T, H, E)) return 0;
  return router_carve(nullptr, T, H, E, nullptr);
}

int ats_moe_router_fwd(const void* x, const float* w, const float* bias, float* logits, int64_t T, int64_t H, int E,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!router_supported(ATS_BF16, T, H, E))
    return fail(ATS_EUNSUPPORTED, "moe_router_fwd: needs bf16 tokens, T >= 128, hidden %% 128 == 0, E <= 256 "
                "(T=%lld hidden=%lld E=%d)", (long long)T, (long long)H, E);
  if (x == nullptr || w == nullptr || logits == nullptr) return fail(ATS_EBADARG, "moe_router_fwd: null pointer");
  RouterWs q;
  ATS_TRY(router_ws(workspace, workspace_bytes, T, H, E, &q));
  cudaStream_t st = (cudaStream_t)stream;
  ATS_TRY(prepare(q, w, T, H, E, st));
  return tc_router_logits(x, q.wparts, bias, logits, T, H, E, q.Ep, one_table(q, T), st);
}

int ats_moe_router_bwd(const float* dlogits, const void* x, const float* w, const void* dxp, const void* moe_workspace,
                       size_t moe_workspace_bytes, int k, int64_t capacity, int layout, void* dx, float* dw,
                       int64_t T, int64_t H, int E, void* workspace, size_t workspace_bytes, void* stream) {
  return ats_moe_router_bwd_staged(dlogits, x, w, dxp, moe_workspace, moe_workspace_bytes, k, capacity, layout, dx,
                                   dw, T, H, E, workspace, workspace_bytes, ATS_ROUTER_BWD_ALL, stream);
}

int ats_moe_router_bwd_staged(const float* dlogits, const void* x, const float* w, const void* dxp,
                              const void* moe_workspace, size_t moe_workspace_bytes, int k, int64_t capacity,
                              int layout, void* dx, float* dw, int64_t T, int64_t H, int E, void* workspace,
                              size_t workspace_bytes, int stages, void* stream) {
  if (stages < 1 || stages > ATS_ROUTER_BWD_ALL) return fail(ATS_EBADARG, "moe_router_bwd: stages %d", stages);
  if (!router_supported(ATS_BF16, T, H, E))
    return fail(ATS_EUNSUPPORTED, "moe_router_bwd: unsupported shape (T=%lld hidden=%lld E=%d)", (long long)T,
                (long long)H, E);
  RouterWs q;
  ATS_TRY(router_ws(workspace, workspace_bytes, T, H, E, &q));
  cudaStream_t st = (cudaStream_t)stream;
  if (stages & ATS_ROUTER_BWD_DW) {
    // the split weight and gradient parts stay in the workspace for the token-gradient stage
    if (dlogits == nullptr || x == nullptr || w == nullptr || dw == nullptr)
      return fail(ATS_EBADARG, "moe_router_bwd: null pointer");
    ATS_TRY(prepare(q, w, T, H, E, st));
    split_dl_kernel<<<grid_for(T * q.Ep), 256, 0, st>>>(dlogits, T, E, q.Ep, q.dlparts);
    ATS_TRY(check_launch("moe_router_split_dl"));
    ATS_TRY(tc_router_dw(x, q.dlparts, q.partial, T, H, q.Ep, chunk_table(q, T), st));
    router_dw_reduce_kernel<<<dim3((unsigned)((H + 31) / 32), (unsigned)(q.Ep / 32)), dim3(32, 8), 0, st>>>(
        q.partial, q.KS, H, E, q.Ep, dw);
    ATS_TRY(check_launch("moe_router_dw_reduce"));
  }
  if (stages & ATS_ROUTER_BWD_DX) {
    if (dx == nullptr) return fail(ATS_EBADARG, "moe_router_bwd: null token gradient");
    const int* tok_row = nullptr;
    if (dxp != nullptr) {
      MoePlan plan;
      ATS_TRY(moe_plan_from_ws(moe_workspace, moe_workspace_bytes, T, E, k, capacity, layout, &plan));
      tok_row = plan.tok_row;
    }
    ATS_TRY(tc_router_dx(q.dlparts, q.wparts, dxp, tok_row, k, dx, T, H, q.Ep, one_table(q, T), st));
  }
  return ATS_OK;
}

int ats_moe_router_status(const void* workspace, size_t workspace_bytes, int64_t T, int64_t H, int E, int* status) {
  RouterWs q;
  ATS_TRY(router_ws(const_cast<void*>(workspace), workspace_bytes, T, H, E, &q));
  if (status == nullptr) return fail(ATS_EBADARG, "moe_router_status: null output");
  cudaError_t e = cudaMemcpy(status, q.tab + 4 + 4 * kMaxChunks, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "moe_router_status: %s", cudaGetErrorString(e));
  return *status == 0 ? ATS_OK : fail(ATS_ETIMEOUT, "moe_router: a bounded device wait gave up (code %d)", *status);
}

}  // extern "C"
