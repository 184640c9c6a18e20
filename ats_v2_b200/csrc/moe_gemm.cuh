// Shared pieces of the expert GEMM paths.
#pragma once

#include "moe_plan.cuh"

namespace ats {

// a = round(round(silu(g)) * u): torch's silu (x / (1 + exp(-x)), float32 math,
// rounded to T) followed by the product rounded to T (ffn.py:44).
template <typename T>
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float s = round_to<T>(g / (1.0f + expf(-g)));
  return round_to<T>(s * u);
}

// Gradients of a = round(round(silu(g)) * u) for upstream da:
//   du = round(da * s), ds = round(da * u), dg = round(ds * sig * (1 + g * (1 - sig)))
// (torch's mul and silu_backward formulas, float32 math rounded to T).
template <typename T>
__device__ __forceinline__ void swiglu_grad(float g, float u, float da, float& dg, float& du) {
  const float e = expf(-g);
  const float s = round_to<T>(g / (1.0f + e));
  const float sig = 1.0f / (1.0f + e);
  du = round_to<T>(da * s);
  const float ds = round_to<T>(da * u);
  dg = round_to<T>((ds * sig) * (1.0f + g * (1.0f - sig)));
}

// Packed forms for the tensor-core epilogues, on pairs of columns.  A product of two bf16 values is exact
// in float32, so mul.rn.bf16x2 rounds the same product the float32 path rounds, once.  The sigmoid's
// reciprocal is rcp.approx (relative error below 2^-22, far under half a bf16 ulp): the rounded results
// equal those of a correctly rounded reciprocal except at rare exact ties.
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {  // round both to bf16, lo in the low half
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf2_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf2_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float sigmoid_fast(float g) { return rcp_approx(1.0f + __expf(-g)); }

// SwiGLU forward on a column pair: g2, u2 hold bf16 gate and up values; returns a = round(round(g*sig(g)) * u).
__device__ __forceinline__ uint32_t silu_mul_bf2(uint32_t g2, uint32_t u2) {
  const float gl = bf2_lo(g2), gh = bf2_hi(g2);
  return bf2_mul(bf2_pack(gl * sigmoid_fast(gl), gh * sigmoid_fast(gh)), u2);
}

// SwiGLU backward on a column pair (the formulas of swiglu_grad): g2, u2 the bf16 pre-activations, da2 the
// bf16 gradient of a; dg2, du2 the bf16 gradients of the gate and up columns.
__device__ __forceinline__ void swiglu_grad_bf2(uint32_t g2, uint32_t u2, uint32_t da2, uint32_t& dg2,
                                                uint32_t& du2) {
  const float gl = bf2_lo(g2), gh = bf2_hi(g2);
  const float sl = sigmoid_fast(gl), sh = sigmoid_fast(gh);
  du2 = bf2_mul(da2, bf2_pack(gl * sl, gh * sh));
  const uint32_t ds2 = bf2_mul(da2, u2);
  dg2 = bf2_pack((bf2_lo(ds2) * sl) * fmaf(gl, 1.0f - sl, 1.0f), (bf2_hi(ds2) * sh) * fmaf(gh, 1.0f - sh, 1.0f));
}

// Shapes the tcgen05 tiling covers: hidden and ffn multiples of 128.
inline bool tc_shape_supported(int64_t H, int64_t F) {
  return H % 128 == 0 && F % 128 == 0 && H >= 128 && F >= 128;
}

// tcgen05 tensor-core expert GEMMs (bf16).  Return ATS_EUNSUPPORTED for shapes
// the tensor-core tiling does not cover; the caller then uses the CUDA-core path.
// io_rows > 0: the token-side tensors (xp, y, dy, dxp) have only io_rows rows (TMA reads past them
// are zero and stores are clipped); h, a and dh always have sg.max_rows rows.
// C[M,N] = A[M,K] B[N,K]^T and its gradients on the same kernel (bf16; N, K multiples of 128; sg one
// segment of M rounded up to 128 rows; A, C, dC, dA have io_rows = M rows).
int tc_gemm_nt_fwd(const void* a, const void* b, void* c, int64_t N, int64_t K, const SegTable& sg, cudaStream_t st,
                   int64_t io_rows);
int tc_gemm_nt_bwd(const void* dc, const void* a, const void* b, void* da, void* db, int64_t N, int64_t K,
                   const SegTable& sg, cudaStream_t st, int64_t io_rows);
// C = A B^T with the rotary embedding of each 128-column head applied in the epilogue; C's row stride is ldc.
// cos/sin: [seq, 128] bf16; row r of C is position r % seq.
int tc_gemm_rope_fwd(const void* a, const void* b, void* c, int64_t ldc, int64_t N, int64_t K, const void* cos,
                     const void* sin, int64_t seq, const SegTable& sg, cudaStream_t st, int64_t io_rows);
int tc_experts_fwd(const void* xp, const void* wgu, const void* wd, void* h, void* a, void* y, int E, int64_t H,
                   int64_t F, const SegTable& sg, cudaStream_t st, int64_t io_rows = 0);
// Stages of the expert backward: the data gradient (dh through the SwiGLU backward, then dxp) and the
// weight gradients (dWd, dWgu, which need dh).  A caller may run them as two calls, data first, to send dxp
// on while the weight gradients compute.
constexpr int kBwdData = 1, kBwdWeights = 2, kBwdAll = 3;
int tc_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* wgu, const void* wd,
                   void* dh, void* dxp, void* dwgu, void* dwd, int E, int64_t H, int64_t F, const SegTable& sg,
                   cudaStream_t st, int64_t io_rows = 0, int stages = kBwdAll);

// Router GEMMs on the tensor cores (bf16 tokens, float32 router weight as three bf16 parts).
// The expert count is padded to kRouterEp (one 64-wide tile holds every expert).
constexpr int kRouterEp = 64;
//   logits[T,E] = x[T,H] . w^T (+ bias), float32;  wparts [3][Ep][H]
int tc_router_logits(const void* x, const void* wparts, const float* bias, float* logits, int64_t T, int64_t H,
                     int E, int Ep, const SegTable& one, cudaStream_t st);
//   dx[T,H] = bf16(dlogits . w) (+ the token's permuted-row gradients);  dlparts [T][3Ep]
int tc_router_dx(const void* dlparts, const void* wparts, const void* dxp, const int* tok_row, int k, void* dx,
                 int64_t T, int64_t H, int Ep, const SegTable& one, cudaStream_t st);
//   partial[g][H][Ep] = x[rows of chunk g]^T . dlogits[rows of chunk g]
int tc_router_dw(const void* x, const void* dlparts, float* partial, int64_t T, int64_t H, int Ep,
                 const SegTable& chunks, cudaStream_t st);

// Main-loop wait budget of the GEMM kernels on the current device (SM cycles;
// <= 0 restores the default of about 2 s), and the first code of a GEMM wait
// that gave up there since the last call (0: none), which this call clears.
int gemm_set_wait_budget(long long cycles);
int gemm_take_status(int* code);

}  // namespace ats
