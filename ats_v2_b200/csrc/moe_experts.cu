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
                                                        SegTable sg) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  const int z = blockIdx.z;  // M-grouped: segment; K-grouped: expert
  int m0, m1, nranges;
  const TI* Bp = static_cast<const TI*>(B.p);
  if (!kgrouped) {  // rows of the segment are global rows of A and C
    m0 = sg.row0[z] + blockIdx.y * kBM;
    m1 = sg.row0[z] + sg.rows[z];
    if (m0 >= m1) return;
    Bp += (int64_t)sg.expert[z] * B.sg;
    nranges = 1;
  } else {
    m0 = blockIdx.y * kBM;
    m1 = M;
    nranges = sg.spe;
  }
  const TI* Ap = static_cast<const TI*>(A.p);
  const int n0 = blockIdx.x * kBN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  const bool a_kfast = A.sj == 1, b_nfast = B.sj == 1;
  for (int q = 0; q < nranges; ++q) {
    int k0 = 0, k1 = K;
    if (kgrouped) {  // the expert's q-th segment of rows
      const int s = sg.eseg[z * sg.spe + q];
      k0 = sg.row0[s];
      k1 = sg.row0[s] + sg.rows[s];
    }
    for (int kb = k0; kb < k1; kb += kBK) {
      for (int i = threadIdx.x; i < kBM * kBK; i += 256) {
        int mm, kk;
        if (a_kfast) { mm = i / kBK; kk = i % kBK; } else { mm = i % kBM; kk = i / kBM; }
        const int gm = m0 + mm, gk = kb + kk;
        As[kk][mm] = (gm < m1 && gk < k1) ? Cvt<TI>::to_f(Ap[(int64_t)gm * A.si + (int64_t)gk * A.sj]) : 0.f;
      }
      for (int i = threadIdx.x; i < kBN * kBK; i += 256) {
        int nn, kk;
        if (b_nfast) { nn = i % kBN; kk = i / kBN; } else { nn = i / kBK; kk = i % kBK; }
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
  }
  TO* Cp = C + (kgrouped ? (int64_t)z * c_sg : 0);
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
              const SegTable& sg, cudaStream_t st) {
  const int gy = kgrouped ? (M + kBM - 1) / kBM : (int)((sg.max_seg_rows + kBM - 1) / kBM);
  const int gz = kgrouped ? sg.E : sg.nseg;
  if (gy == 0 || gz == 0) return ATS_OK;
  dim3 grid((N + kBN - 1) / kBN, gy, gz);
  simt_gemm_kernel<T, T><<<grid, 256, 0, st>>>(A, B, C, c_si, c_sg, M, N, K, kgrouped, sg);
  return check_launch("moe_simt_gemm");
}

// a = round(round(silu(g)) * u) over every segment's rows (h = [g | u], row stride 2F)
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ h, T* __restrict__ a, int64_t F, SegTable sg) {
  const int s = blockIdx.y;
  const int64_t r0 = sg.row0[s], n = (int64_t)sg.rows[s] * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = r0 + i / F, f = i % F;
    const float g = Cvt<T>::to_f(h[r * 2 * F + f]);
    const float u = Cvt<T>::to_f(h[r * 2 * F + F + f]);
    a[r * F + f] = Cvt<T>::from_f(silu_mul<T>(g, u));
  }
}

// In place on dh = [dg | du] whose du half holds da on entry.
template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ h, T* __restrict__ dh, int64_t F, SegTable sg) {
  const int s = blockIdx.y;
  const int64_t r0 = sg.row0[s], n = (int64_t)sg.rows[s] * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = r0 + i / F, f = i % F;
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
int simt_experts_fwd(const void* xp, const void* wgu, const void* wd, void* h, void* a, void* y, int64_t H, int64_t F,
                     const SegTable& sg, cudaStream_t st) {
  // h = xp Wgu_e^T : A(m=row,k=h) = xp[row*H+h], B(k=h,n=j) = Wgu_e[j*H+h]
  ATS_TRY(simt_gemm<T>(Opnd{xp, H, 1, 0}, Opnd{wgu, 1, H, 2 * F * H}, static_cast<T*>(h), 2 * F, 0, 0, (int)(2 * F),
                       (int)H, false, sg, st));
  const dim3 eg((unsigned)(num_sms() * 2), (unsigned)sg.nseg);
  swiglu_fwd_kernel<T><<<eg, 256, 0, st>>>(static_cast<const T*>(h), static_cast<T*>(a), F, sg);
  ATS_TRY(check_launch("moe_swiglu_fwd"));
  // y = a Wd_e^T : B(k=f,n=h) = Wd_e[h*F+f]
  return simt_gemm<T>(Opnd{a, F, 1, 0}, Opnd{wd, 1, F, H * F}, static_cast<T*>(y), H, 0, 0, (int)H, (int)F, false,
                      sg, st);
}

template <typename T>
int simt_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* wgu, const void* wd,
                     void* dh, void* dxp, void* dwgu, void* dwd, int64_t H, int64_t F, const SegTable& sg,
                     cudaStream_t st, int stages) {
  T* dhp = static_cast<T*>(dh);
  if (stages & kBwdData) {
    // da = dy Wd_e into the du half of dh : B(k=h,n=f) = Wd_e[h*F+f]
    ATS_TRY(simt_gemm<T>(Opnd{dy, H, 1, 0}, Opnd{wd, F, 1, H * F}, dhp + F, 2 * F, 0, 0, (int)F, (int)H, false, sg,
                         st));
    const dim3 eg((unsigned)(num_sms() * 2), (unsigned)sg.nseg);
    swiglu_bwd_kernel<T><<<eg, 256, 0, st>>>(static_cast<const T*>(h), dhp, F, sg);
    ATS_TRY(check_launch("moe_swiglu_bwd"));
    // dxp = dh Wgu_e : B(k=j,n=h) = Wgu_e[j*H+h]
    ATS_TRY(simt_gemm<T>(Opnd{dh, 2 * F, 1, 0}, Opnd{wgu, H, 1, 2 * F * H}, static_cast<T*>(dxp), H, 0, 0, (int)H,
                         (int)(2 * F), false, sg, st));
  }
  if (!(stages & kBwdWeights)) return ATS_OK;
  // dWd_e[h,f] = sum over the expert's rows r of dy[r,h] a[r,f]
  ATS_TRY(simt_gemm<T>(Opnd{dy, 1, H, 0}, Opnd{a, F, 1, 0}, static_cast<T*>(dwd), F, H * F, (int)H, (int)F, 0, true,
                       sg, st));
  // dWgu_e[j,h] = sum over the expert's rows r of dh[r,j] xp[r,h]
  return simt_gemm<T>(Opnd{dh, 1, 2 * F, 0}, Opnd{xp, H, 1, 0}, static_cast<T*>(dwgu), H, 2 * F * H, (int)(2 * F),
                      (int)H, 0, true, sg, st);
}

int experts_fwd(const void* xp, const void* wgu, const void* wd, void* h, void* a, void* y, ats_dtype dtype, int E,
                int64_t H, int64_t F, const SegTable& sg, cudaStream_t st) {
  if (dtype == ATS_BF16) {
    const int r = tc_experts_fwd(xp, wgu, wd, h, a, y, E, H, F, sg, st);
    if (r != ATS_EUNSUPPORTED) return r;
    return simt_experts_fwd<bf16>(xp, wgu, wd, h, a, y, H, F, sg, st);
  }
  return simt_experts_fwd<float>(xp, wgu, wd, h, a, y, H, F, sg, st);
}

int experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* wgu, const void* wd,
                void* dh, void* dxp, void* dwgu, void* dwd, ats_dtype dtype, int E, int64_t H, int64_t F,
                const SegTable& sg, cudaStream_t st, int stages = kBwdAll) {
  if (dtype == ATS_BF16) {
    const int r = tc_experts_bwd(dy, xp, h, a, wgu, wd, dh, dxp, dwgu, dwd, E, H, F, sg, st, 0, stages);
    if (r != ATS_EUNSUPPORTED) return r;
    return simt_experts_bwd<bf16>(dy, xp, h, a, wgu, wd, dh, dxp, dwgu, dwd, H, F, sg, st, stages);
  }
  return simt_experts_bwd<float>(dy, xp, h, a, wgu, wd, dh, dxp, dwgu, dwd, H, F, sg, st, stages);
}

// ---------------------------------------------------------- EP segment table
struct EpSegs {
  int* row0;
  int* rows;
  int* expert;
  int* eseg;
  int* err;
  int* kept;
};

size_t ep_carve(void* ws, int W, int El, EpSegs* o) {
  const size_t n = (size_t)W * El;
  size_t off = 0;
  char* base = static_cast<char*>(ws);
  auto take = [&](size_t bytes) -> void* {
    void* r = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return r;
  };
  EpSegs q;
  q.row0 = (int*)take(n * 4);
  q.rows = (int*)take(n * 4);
  q.expert = (int*)take(n * 4);
  q.eseg = (int*)take(n * 4);
  q.err = (int*)take(4);
  q.kept = (int*)take(n * 4);
  if (o) *o = q;
  return off;
}

int ep_check(int W, int El, int64_t C) {
  if (W < 1 || El < 1 || (int64_t)W * El > kMaxExperts || C < 1)
    return fail(ATS_EBADARG, "moe_ep: bad sizes W=%d E_local=%d capacity=%lld", W, El, (long long)C);
  if ((int64_t)W * El * slot_rows(C) >= ((int64_t)1 << 31)) return fail(ATS_EUNSUPPORTED, "moe_ep: rows above 2^31");
  return ATS_OK;
}

int ep_table(const void* ws, size_t bytes, int W, int El, int64_t C, SegTable* sg) {
  ATS_TRY(ep_check(W, El, C));
  if (ws == nullptr || bytes < ep_carve(nullptr, W, El, nullptr))
    return fail(ATS_EBADARG, "moe_ep: segment workspace too small");
  EpSegs q;
  ep_carve(const_cast<void*>(ws), W, El, &q);
  sg->row0 = q.row0;
  sg->rows = q.rows;
  sg->expert = q.expert;
  sg->eseg = q.eseg;
  sg->nseg = W * El;
  sg->spe = W;
  sg->E = El;
  sg->max_rows = (int64_t)W * El * slot_rows(C);
  sg->max_seg_rows = slot_rows(C);
  sg->err = q.err;
  sg->kept = q.kept;
  return ATS_OK;
}

// Segment s = source rank * E_local + local expert.  ATS_MOE_SLOTS: at rows
// s*Cp.  ATS_MOE_PACKED: right after segment s-1 (the received rows are the
// sources' packed segments, each rounded up to 128 rows, in (source, expert) order).
__global__ void ep_segments_kernel(const int* __restrict__ recv_kept, int W, int El, int Cp, int layout,
                                   EpSegs q) {
  __shared__ int wsum[32];
  const int n = W * El;  // <= kMaxExperts = blockDim.x
  const int s = threadIdx.x, lane = s & 31, warp = s >> 5;
  int rows = 0, kept = 0;
  if (s < n) {
    kept = recv_kept[s];
    kept = kept < 0 ? 0 : (kept > Cp ? Cp : kept);
    rows = (kept + kSegAlign - 1) / kSegAlign * kSegAlign;
  }
  // exclusive block scan of rows in segment order
  int incl = rows;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = wsum[lane];
    int wi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    wsum[lane] = wi - v;
  }
  __syncthreads();
  if (s < n) {
    const int src = s / El, el = s - src * El;
    q.row0[s] = layout == ATS_MOE_SLOTS ? s * Cp : wsum[warp] + incl - rows;
    q.rows[s] = rows;
    q.expert[s] = el;
    q.eseg[el * W + src] = s;
    q.kept[s] = kept;
  }
  if (s == 0) q.err[0] = 0;
}

// ---- dense SwiGLU FFN: one expert over the T token rows, table [row0, rows, expert, eseg, status]
constexpr size_t kDenseWsBytes = 256;

int64_t dense_rows(int64_t T) { return (T + kSegAlign - 1) / kSegAlign * kSegAlign; }

bool dense_supported(ats_dtype dt, int64_t T, int64_t H, int64_t F) {
  return dt == ATS_BF16 && tc_shape_supported(H, F) && T >= kSegAlign && dense_rows(T) < ((int64_t)1 << 31);
}

__global__ void dense_table_kernel(int* tab, int rows) {
  tab[0] = 0;
  tab[1] = rows;
  tab[2] = 0;
  tab[3] = 0;
  tab[4] = 0;
}

int dense_table(void* ws, size_t bytes, int64_t T, SegTable* sg) {
  if (ws == nullptr || bytes < kDenseWsBytes) return fail(ATS_EBADARG, "swiglu: workspace too small");
  int* tab = static_cast<int*>(ws);
  sg->row0 = tab;
  sg->rows = tab + 1;
  sg->expert = tab + 2;
  sg->eseg = tab + 3;
  sg->nseg = 1;
  sg->spe = 1;
  sg->E = 1;
  sg->max_rows = dense_rows(T);
  sg->max_seg_rows = sg->max_rows;
  sg->err = tab + 4;
  return ATS_OK;
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

int ats_swiglu_supported(ats_dtype dtype, int64_t T, int64_t H, int64_t F) {
  return dense_supported(dtype, T, H, F) ? 1 : 0;
}

size_t ats_swiglu_workspace_bytes(void) { return kDenseWsBytes; }

int64_t ats_swiglu_rows(int64_t T) { return T > 0 ? dense_rows(T) : 0; }

int ats_swiglu_fwd(const void* x, const void* w_gate_up, const void* w_down, void* h, void* a, void* y,
                   ats_dtype dtype, int64_t T, int64_t H, int64_t F, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (!dense_supported(dtype, T, H, F))
    return fail(ATS_EUNSUPPORTED, "swiglu_fwd: needs bf16, T >= 128 and hidden, ffn multiples of 128 "
                "(T=%lld hidden=%lld ffn=%lld)", (long long)T, (long long)H, (long long)F);
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (x == nullptr || h == nullptr || a == nullptr || y == nullptr) return fail(ATS_EBADARG, "swiglu_fwd: null");
  SegTable sg;
  ATS_TRY(dense_table(workspace, workspace_bytes, T, &sg));
  cudaStream_t st = (cudaStream_t)stream;
  dense_table_kernel<<<1, 1, 0, st>>>(static_cast<int*>(workspace), (int)dense_rows(T));
  ATS_TRY(check_launch("swiglu_table"));
  return tc_experts_fwd(x, w_gate_up, w_down, h, a, y, 1, H, F, sg, st, T);
}

int ats_swiglu_bwd(const void* dy, const void* x, const void* h, const void* a, const void* w_gate_up,
                   const void* w_down, void* dh, void* dx, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                   int64_t T, int64_t H, int64_t F, void* workspace, size_t workspace_bytes, void* stream) {
  if (!dense_supported(dtype, T, H, F))
    return fail(ATS_EUNSUPPORTED, "swiglu_bwd: unsupported shape (T=%lld hidden=%lld ffn=%lld)", (long long)T,
                (long long)H, (long long)F);
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (dy == nullptr || x == nullptr || h == nullptr || a == nullptr || dh == nullptr || dx == nullptr ||
      dw_gate_up == nullptr || dw_down == nullptr)
    return fail(ATS_EBADARG, "swiglu_bwd: null");
  SegTable sg;
  ATS_TRY(dense_table(workspace, workspace_bytes, T, &sg));
  cudaStream_t st = (cudaStream_t)stream;
  dense_table_kernel<<<1, 1, 0, st>>>(static_cast<int*>(workspace), (int)dense_rows(T));
  ATS_TRY(check_launch("swiglu_table"));
  return tc_experts_bwd(dy, x, h, a, w_gate_up, w_down, dh, dx, dw_gate_up, dw_down, 1, H, F, sg, st, T);
}

int ats_gemm_supported(ats_dtype dtype, int64_t M, int64_t N, int64_t K) {
  return dense_supported(dtype, M, N, K) ? 1 : 0;
}

size_t ats_gemm_workspace_bytes(void) { return kDenseWsBytes; }

int ats_gemm_fwd(const void* a, const void* b, void* c, ats_dtype dtype, int64_t M, int64_t N, int64_t K,
                 void* workspace, size_t workspace_bytes, void* stream) {
  if (!ats_gemm_supported(dtype, M, N, K))
    return fail(ATS_EUNSUPPORTED, "gemm_fwd: needs bf16, M >= 128 and N, K multiples of 128 (M=%lld N=%lld K=%lld)",
                (long long)M, (long long)N, (long long)K);
  if (a == nullptr || b == nullptr || c == nullptr) return fail(ATS_EBADARG, "gemm_fwd: null");
  SegTable sg;
  ATS_TRY(dense_table(workspace, workspace_bytes, M, &sg));
  cudaStream_t st = (cudaStream_t)stream;
  dense_table_kernel<<<1, 1, 0, st>>>(static_cast<int*>(workspace), (int)dense_rows(M));
  ATS_TRY(check_launch("gemm_table"));
  return tc_gemm_nt_fwd(a, b, c, N, K, sg, st, M);
}

int ats_gemm_bwd(const void* dc, const void* a, const void* b, void* da, void* db, ats_dtype dtype, int64_t M,
                 int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ats_gemm_supported(dtype, M, N, K))
    return fail(ATS_EUNSUPPORTED, "gemm_bwd: unsupported shape (M=%lld N=%lld K=%lld)", (long long)M, (long long)N,
                (long long)K);
  if (dc == nullptr || (da != nullptr && b == nullptr) || (db != nullptr && a == nullptr))
    return fail(ATS_EBADARG, "gemm_bwd: null");
  SegTable sg;
  ATS_TRY(dense_table(workspace, workspace_bytes, M, &sg));
  cudaStream_t st = (cudaStream_t)stream;
  dense_table_kernel<<<1, 1, 0, st>>>(static_cast<int*>(workspace), (int)dense_rows(M));
  ATS_TRY(check_launch("gemm_table"));
  return tc_gemm_nt_bwd(dc, a, b, da, db, N, K, sg, st, M);
}

int ats_gemm_rope_fwd(const void* x, const void* w, void* out, int64_t ld_out, ats_dtype dtype, int64_t M, int64_t N,
                      int64_t K, const void* cos, const void* sin, int64_t seq_len, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!ats_gemm_supported(dtype, M, N, K))
    return fail(ATS_EUNSUPPORTED, "gemm_rope_fwd: needs bf16, M >= 128 and N, K multiples of 128 (M=%lld N=%lld "
                "K=%lld)", (long long)M, (long long)N, (long long)K);
  if (x == nullptr || w == nullptr || out == nullptr || cos == nullptr || sin == nullptr)
    return fail(ATS_EBADARG, "gemm_rope_fwd: null");
  if (seq_len < 1 || M % seq_len != 0 || ld_out < N || (ld_out * 2) % 16 != 0 || !aligned16(out) || !aligned16(cos) ||
      !aligned16(sin))
    return fail(ATS_EBADARG, "gemm_rope_fwd: seq_len %lld must divide M=%lld; output stride %lld >= N=%lld, "
                "16-byte aligned rows and tables", (long long)seq_len, (long long)M, (long long)ld_out, (long long)N);
  SegTable sg;
  ATS_TRY(dense_table(workspace, workspace_bytes, M, &sg));
  cudaStream_t st = (cudaStream_t)stream;
  dense_table_kernel<<<1, 1, 0, st>>>(static_cast<int*>(workspace), (int)dense_rows(M));
  ATS_TRY(check_launch("gemm_table"));
  return tc_gemm_rope_fwd(x, w, out, ld_out, N, K, cos, sin, seq_len, sg, st, M);
}

int ats_swiglu_status(const void* workspace, size_t workspace_bytes, int* status) {
  if (workspace == nullptr || workspace_bytes < kDenseWsBytes || status == nullptr)
    return fail(ATS_EBADARG, "swiglu_status: bad arguments");
  cudaError_t e = cudaMemcpy(status, static_cast<const int*>(workspace) + 4, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "swiglu_status: %s", cudaGetErrorString(e));
  return *status == 0 ? ATS_OK : fail(ATS_ETIMEOUT, "swiglu: a bounded device wait gave up (code %d)", *status);
}

int ats_moe_experts_fwd(const void* xp, const void* w_gate_up, const void* w_down, void* h, void* a, void* y,
                        ats_dtype dtype, int64_t T, int E, int k, int64_t capacity, int layout, int64_t H, int64_t F,
                        const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (xp == nullptr || h == nullptr || a == nullptr || y == nullptr) return fail(ATS_EBADARG, "moe_experts_fwd: null");
  return experts_fwd(xp, w_gate_up, w_down, h, a, y, dtype, E, H, F, plan_segments(plan), (cudaStream_t)stream);
}

int ats_moe_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* w_gate_up,
                        const void* w_down, void* dh, void* dxp, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                        int64_t T, int E, int k, int64_t capacity, int layout, int64_t H, int64_t F,
                        const void* workspace, size_t workspace_bytes, void* stream) {
  MoePlan plan;
  ATS_TRY(moe_plan_from_ws(workspace, workspace_bytes, T, E, k, capacity, layout, &plan));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (dy == nullptr || xp == nullptr || h == nullptr || a == nullptr || dh == nullptr || dxp == nullptr ||
      dw_gate_up == nullptr || dw_down == nullptr)
    return fail(ATS_EBADARG, "moe_experts_bwd: null");
  return experts_bwd(dy, xp, h, a, w_gate_up, w_down, dh, dxp, dw_gate_up, dw_down, dtype, E, H, F,
                     plan_segments(plan), (cudaStream_t)stream);
}

size_t ats_moe_ep_segments_bytes(int W, int E_local) {
  if (W < 1 || E_local < 1) return 0;
  return ep_carve(nullptr, W, E_local, nullptr);
}

int ats_moe_ep_segments(const int32_t* recv_kept, int W, int E_local, int64_t capacity, int layout, void* seg_workspace,
                        size_t seg_workspace_bytes, void* stream) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, capacity, &sg));
  if (recv_kept == nullptr) return fail(ATS_EBADARG, "moe_ep_segments: null counts");
  EpSegs q;
  ep_carve(seg_workspace, W, E_local, &q);
  if (layout != ATS_MOE_PACKED && layout != ATS_MOE_SLOTS) return fail(ATS_EBADARG, "moe_ep_segments: layout %d", layout);
  ep_segments_kernel<<<1, kMaxExperts, 0, (cudaStream_t)stream>>>(recv_kept, W, E_local, (int)slot_rows(capacity),
                                                                  layout, q);
  return check_launch("moe_ep_segments");
}

int ats_moe_ep_experts_fwd_sources(const void* xr, const void* w_gate_up, const void* w_down, void* h, void* a,
                                   void* y, ats_dtype dtype, int W, int E_local, int64_t capacity, int64_t H,
                                   int64_t F, const void* seg_workspace, size_t seg_workspace_bytes, int src_lo,
                                   int src_hi, void* stream) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, capacity, &sg));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (xr == nullptr || h == nullptr || a == nullptr || y == nullptr)
    return fail(ATS_EBADARG, "moe_ep_experts_fwd_sources: null");
  if (src_lo < 0 || src_hi > W || src_lo > src_hi)
    return fail(ATS_EBADARG, "moe_ep_experts_fwd_sources: sources [%d, %d) of %d", src_lo, src_hi, W);
  if (src_lo == src_hi) return ATS_OK;
  // segments are source-major (segment = source * E_local + expert): the sources' segments are one range
  sg.row0 += src_lo * E_local;
  sg.rows += src_lo * E_local;
  sg.expert += src_lo * E_local;
  sg.nseg = (src_hi - src_lo) * E_local;
  return experts_fwd(xr, w_gate_up, w_down, h, a, y, dtype, E_local, H, F, sg, (cudaStream_t)stream);
}

int ats_moe_ep_experts_fwd(const void* xr, const void* w_gate_up, const void* w_down, void* h, void* a, void* y,
                           ats_dtype dtype, int W, int E_local, int64_t capacity, int64_t H, int64_t F,
                           const void* seg_workspace, size_t seg_workspace_bytes, void* stream) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, capacity, &sg));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (xr == nullptr || h == nullptr || a == nullptr || y == nullptr) return fail(ATS_EBADARG, "moe_ep_experts_fwd: null");
  return experts_fwd(xr, w_gate_up, w_down, h, a, y, dtype, E_local, H, F, sg, (cudaStream_t)stream);
}

int ats_moe_ep_experts_bwd_staged(const void* dy, const void* xr, const void* h, const void* a,
                                  const void* w_gate_up, const void* w_down, void* dh, void* dxr, void* dw_gate_up,
                                  void* dw_down, ats_dtype dtype, int W, int E_local, int64_t capacity, int64_t H,
                                  int64_t F, const void* seg_workspace, size_t seg_workspace_bytes, int stages,
                                  void* stream) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, capacity, &sg));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (stages < 1 || stages > kBwdAll) return fail(ATS_EBADARG, "moe_ep_experts_bwd_staged: stages %d", stages);
  if (dy == nullptr || xr == nullptr || h == nullptr || a == nullptr || dh == nullptr ||
      ((stages & kBwdData) && dxr == nullptr) ||
      ((stages & kBwdWeights) && (dw_gate_up == nullptr || dw_down == nullptr)))
    return fail(ATS_EBADARG, "moe_ep_experts_bwd_staged: null");
  return experts_bwd(dy, xr, h, a, w_gate_up, w_down, dh, dxr, dw_gate_up, dw_down, dtype, E_local, H, F, sg,
                     (cudaStream_t)stream, stages);
}

int ats_moe_ep_experts_bwd(const void* dy, const void* xr, const void* h, const void* a, const void* w_gate_up,
                           const void* w_down, void* dh, void* dxr, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                           int W, int E_local, int64_t capacity, int64_t H, int64_t F, const void* seg_workspace,
                           size_t seg_workspace_bytes, void* stream) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, capacity, &sg));
  ATS_TRY(check_experts(w_gate_up, w_down, H, F, dtype));
  if (dy == nullptr || xr == nullptr || h == nullptr || a == nullptr || dh == nullptr || dxr == nullptr ||
      dw_gate_up == nullptr || dw_down == nullptr)
    return fail(ATS_EBADARG, "moe_ep_experts_bwd: null");
  return experts_bwd(dy, xr, h, a, w_gate_up, w_down, dh, dxr, dw_gate_up, dw_down, dtype, E_local, H, F, sg,
                     (cudaStream_t)stream);
}

int ats_moe_ep_status(const void* seg_workspace, size_t seg_workspace_bytes, int W, int E_local, int* status) {
  SegTable sg;
  ATS_TRY(ep_table(seg_workspace, seg_workspace_bytes, W, E_local, 1, &sg));
  if (status == nullptr) return fail(ATS_EBADARG, "moe_ep_status: null output");
  cudaError_t e = cudaMemcpy(status, sg.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "moe_ep_status: %s", cudaGetErrorString(e));
  return *status == 0 ? ATS_OK : fail(ATS_ETIMEOUT, "moe_ep: a bounded device wait gave up (code %d)", *status);
}

}  // extern "C"
