// Grouped SwiGLU experts: entry points and the CUDA-core (SIMT) path.
//
// Expert e's tokens occupy the padded permuted rows [seg_start[e], seg_start[e+1]).
// Two kinds of grouped GEMM cover the forward and backward:
//   M-grouped : C[rows of e] = A[rows of e] * B_e          (forward, data grads)
//   K-grouped : C_e = sum over rows r of e of A(:, r) B(r, :) (weight grads)
// Padding rows are zero in every permuted operand, so they add nothing.
//
// bf16 experts run on the tcgen05 tensor-core kernels (moe_gemm_tc.cu);
// float32 experts run here on CUDA cores in float32, the dtype the reference
// computes them in.
#include "moe_gemm.cuh"

namespace ats {
namespace {

constexpr int kBM = 64, kBN = 64, kBK = 16;

// element (i, j) of an operand = p[g*sg + i*si + j*sj]
struct Opnd {
  const void* p;
  int64_t si, sj, sg;
};

template <typename TI, typename TO>
__global__ void __launch_bounds__(256) simt_gemm_kernel(Opnd A, Opnd B, TO* __restrict__ C, int64_t c_si,
                                                        int64_t c_sg, int M, int N, int K, bool kgrouped,
                                                        const int* __restrict__ seg_start) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  const int e = blockIdx.z;
  int m0, m1, k0, k1;
  if (!kgrouped) {  // rows of the group are global rows of A and C
    m0 = seg_start[e] + blockIdx.y * kBM;
    m1 = seg_start[e + 1];
    if (m0 >= m1) return;
    k0 = 0;
    k1 = K;
  } else {
    m0 = blockIdx.y * kBM;
    m1 = M;
    k0 = seg_start[e];
    k1 = seg_start[e + 1];
  }
  const int n0 = blockIdx.x * kBN;
  const TI* Ap = static_cast<const TI*>(A.p) + (kgrouped ? 0 : 0);
  const TI* Bp = static_cast<const TI*>(B.p) + (kgrouped ? 0 : (int64_t)e * B.sg);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  const bool a_kfast = A.sj == 1, b_nfast = B.sj == 1;
  for (int kb = k0; kb < k1; kb += kBK) {
    for (int q = threadIdx.x; q < kBM * kBK; q += 256) {
      int mm, kk;
      if (a_kfast) { mm = q / kBK; kk = q % kBK; } else { mm = q % kBM; kk = q / kBM; }
      const int gm = m0 + mm, gk = kb + kk;
      As[kk][mm] = (gm < m1 && gk < k1) ? Cvt<TI>::to_f(Ap[(int64_t)gm * A.si + (int64_t)gk * A.sj]) : 0.f;
    }
    for (int q = threadIdx.x; q < kBN * kBK; q += 256) {
      int nn, kk;
      if (b_nfast) { nn = q % kBN; kk = q / kBN; } else { nn = q / kBK; kk = q % kBK; }
      const int gn = n0 + nn, gk = kb + kk;
      Bs[kk][nn] = (gn < N && gk < k1) ? Cvt<TI>::to_f(Bp[(int64_t)gk * B.si + (int64_t)gn * B.sj]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  TO* Cp = C + (kgrouped ? (int64_t)e * c_sg : 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= m1) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn < N) Cp[(int64_t)gm * c_si + gn] = Cvt<TO>::from_f(acc[i][j]);
    }
  }
}

template <typename T>
int simt_gemm(Opnd A, Opnd B, T* C, int64_t c_si, int64_t c_sg, int M, int N, int K, bool kgrouped,
              const int* seg_start, int E, int64_t max_seg_rows, cudaStream_t st) {
  const int gy = kgrouped ? (M + kBM - 1) / kBM : (int)((max_seg_rows + kBM - 1) / kBM);
  if (gy == 0 || E == 0) return ATS_OK;
  dim3 grid((N + kBN - 1) / kBN, gy, E);
  simt_gemm_kernel<T, T><<<grid, 256, 0, st>>>(A, B, C, c_si, c_sg, M, N, K, kgrouped, seg_start);
  return check_launch("moe_simt_gemm");
}

// a = round(round(silu(g)) * u) over the padded rows (h = [g | u], row stride 2F)
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ h, T* __restrict__ a, int64_t F,
                                  const int* __restrict__ seg_start, int E) {
  const int64_t rows = seg_start[E];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * F;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, f = i - r * F;
    const float g = Cvt<T>::to_f(h[r * 2 * F + f]);
    const float u = Cvt<T>::to_f(h[r * 2 * F + F + f]);
    a[i] = Cvt<T>::from_f(silu_mul<T>(g, u));
  }
}

// In place on dh = [dg | du] whose du half holds da on entry.
template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ h, T* __restrict__ dh, int64_t F,
                                  const int* __restrict__ seg_start, int E) {
  const int64_t rows = seg_start[E];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * F;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, f = i - r * F;
    const float g = Cvt<T>::to_f(h[r * 2 * F + f]);
    const float u = Cvt<T>::to_f(h[r * 2 * F + F + f]);
    const float da = Cvt<T>::to_f(dh[r * 2 * F + F + f]);
    float dg, du;
    swiglu_grad<T>(g, u, da, dg, du);
    dh[r * 2 * F + f] = Cvt<T>::from_f(dg);
    dh[r * 2 * F + F + f] = Cvt<T>::from_f(du);
  }
}

template <typename T>
int simt_experts_fwd(const void* xp, const void* wgu, const void* wd, void* h, void* a, void* y, int E, int64_t H,
                     int64_t F, const MoePlan& plan, cudaStream_t st) {
  const int64_t msr = align_up((size_t)(plan.C < plan.T ? plan.C : plan.T), kSegAlign);
  const int* seg = plan.seg_start;
  // h = xp Wgu_e^T : A(m=row,k=h) = xp[row*H+h], B(k=h,n=j) = Wgu_e[j*H+h]
  ATS_TRY(simt_gemm<T>(Opnd{xp, H, 1, 0}, Opnd{wgu, 1, H, 2 * F * H}, static_cast<T*>(h), 2 * F, 0, 0, (int)(2 * F),
                       (int)H, false, seg, E, msr, st));
  swiglu_fwd_kernel<T><<<num_sms() * 8, 256, 0, st>>>(static_cast<const T*>(h), static_cast<T*>(a), F, seg, E);
  ATS_TRY(check_launch("moe_swiglu_fwd"));
  // y = a Wd_e^T : B(k=f,n=h) = Wd_e[h*F+f]
  return simt_gemm<T>(Opnd{a, F, 1, 0}, Opnd{wd, 1, F, H * F}, static_cast<T*>(y), H, 0, 0, (int)H, (int)F, false,
                      seg, E, msr, st);
}

template <typename T>
int simt_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* wgu, const void* wd,
                     void* dh, void* dxp, void* dwgu, void* dwd, int E, int64_t H, int64_t F, const MoePlan& plan,
                     cudaStream_t st) {
  const int64_t msr = align_up((size_t)(plan.C < plan.T ? plan.C : plan.T), kSegAlign);
  const int* seg = plan.seg_start;
  T* dhp = static_cast<T*>(dh);
  // da = dy Wd_e into the du half of dh : B(k=h,n=f) = Wd_e[h*F+f]
  ATS_TRY(simt_gemm<T>(Opnd{dy, H, 1, 0}, Opnd{wd, F, 1, H * F}, dhp + F, 2 * F, 0, 0, (int)F, (int)H, false, seg, E,
                       msr, st));
  swiglu_bwd_kernel<T><<<num_sms() * 8, 256, 0, st>>>(static_cast<const T*>(h), dhp, F, seg, E);
  ATS_TRY(check_launch("moe_swiglu_bwd"));
  // dWd_e[h,f] = sum_r dy[r,h] a[r,f]
  ATS_TRY(simt_gemm<T>(Opnd{dy, 1, H, 0}, Opnd{a, F, 1, 0}, static_cast<T*>(dwd), F, H * F, (int)H, (int)F, 0, true,
                       seg, E, msr, st));
  // dxp = dh Wgu_e : B(k=j,n=h) = Wgu_e[j*H+h]
  ATS_TRY(simt_gemm<T>(Opnd{dh, 2 * F, 1, 0}, Opnd{wgu, H, 1, 2 * F * H}, static_cast<T*>(dxp), H, 0, 0, (int)H,
                       (int)(2 * F), false, seg, E, msr, st));
  // dWgu_e[j,h] = sum_r dh[r,j] xp[r,h]
  return simt_gemm<T>(Opnd{dh, 1, 2 * F, 0}, Opnd{xp, H, 1, 0}, static_cast<T*>(dwgu), H, 2 * F * H, (int)(2 * F),
                      (int)H, 0, true, seg, E, msr, st);
}

int check_experts(const void* p0, const void* p1, int64_t H, int64_t F, ats_dtype dt) {
  if (H <= 0 || F <= 0 || p0 == nullptr || p1 == nullptr) return fail(ATS_EBADARG, "moe_experts: bad arguments");
  if (dt != ATS_BF16 && dt != ATS_F32) return fail(ATS_EBADARG, "moe_experts: dtype");
  if (H >= (1 << 30) || F >= (1 << 29)) return fail(ATS_EUNSUPPORTED, "moe_experts: dims too large");
  return ATS_OK;
}

}  // namespace
}  // namespace ats

using namespace ats;

extern "C" {

int ats_moe_uses_tensor_cores(ats_dtype dtype, int64_t H, int64_t F) {
  return dtype == ATS_BF16 && tc_shape_supported(H, F) ? 1 : 0;
}

int ats_moe_experts_fwd(const void* xp, const void* w_gate_up, const void* w_down, void* h, void* a, void* y,
                        ats_dtype dtype, int64_t T, int E, int k, int64_t capacity, int64_t H, int64_t F,
                        const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, &plan));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (xp == nullptr || h == nullptr || a == nullptr || y == nullptr) return fail(ATS_EBADARG, "moe_experts_fwd: null");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16) {
    const int r = tc_experts_fwd(xp, w_gate_up, w_down, h, a, y, E, H, F, plan, st);
    if (r != ATS_EUNSUPPORTED) return r;
    return simt_experts_fwd<bf16>(xp, w_gate_up, w_down, h, a, y, E, H, F, plan, st);
  }
  return simt_experts_fwd<float>(xp, w_gate_up, w_down, h, a, y, E, H, F, plan, st);
}

int ats_moe_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* w_gate_up,
                        const void* w_down, void* dh, void* dxp, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                        int64_t T, int E, int k, int64_t capacity, int64_t H, int64_t F, const void* workspace,
                        size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, &plan));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (dy == nullptr || xp == nullptr || h == nullptr || a == nullptr || dh == nullptr || dxp == nullptr ||
      dw_gate_up == nullptr || dw_down == nullptr)
    return fail(ATS_EBADARG, "moe_experts_bwd: null");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == ATS_BF16) {
    const int r = tc_experts_bwd(dy, xp, h, a, w_gate_up, w_down, dh, dxp, dw_gate_up, dw_down, E, H, F, plan, st);
    if (r != ATS_EUNSUPPORTED) return r;
    return simt_experts_bwd<bf16>(dy, xp, h, a, w_gate_up, w_down, dh, dxp, dw_gate_up, dw_down, E, H, F, plan, st);
  }
  return simt_experts_bwd<float>(dy, xp, h, a, w_gate_up, w_down, dh, dxp, dw_gate_up, dw_down, E, H, F, plan, st);
}

}  // extern "C"
