// Rotate-half rotary embedding for q and k in one launch, forward and adjoint.
//
// A thread owns one (token, group of up to 8 heads, 16-byte chunk pair):
// the chunk at column j of the first half of a head row and the matching
// chunk at j+D/2.  It loads the token's cos/sin chunks once, keeps them in
// registers, and rotates that chunk pair in every head of its group, several
// heads per step so many loads are in flight.  Consecutive threads take consecutive chunks of
// a head row, so for the attention layout (BSHD memory viewed as [B,H,S,D])
// every warp load is whole 128-byte lines.  q/k are read once and written
// once: one HBM pass in each direction.
//
// Rounding mirrors the reference's torch ops (rope.py:85-86), each of which
// rounds to the tensor dtype:
//   forward : o1 = R(R(x1*c1) - R(x2*s1)),   o2 = R(R(x2*c2) + R(x1*s2))
//   adjoint : d1 = R(R(g1*c1) + R(g2*s2)),   d2 = R(R(g2*c2) - R(g1*s1))
// with c1=cos[j], c2=cos[j+D/2], s1=sin[j], s2=sin[j+D/2].  Products and sums
// use explicitly rounded intrinsics so float32 results are not contracted
// into FMAs.
#include "common.cuh"

namespace ats {
namespace {

struct RopeTensor {
  const void* in;
  void* out;
  int64_t heads;
  int64_t is_b, is_h, is_s;  // input strides (elements)
  int64_t os_b, os_h, os_s;  // output strides (elements)
};

template <typename T>
__device__ __forceinline__ void rot_pair(float x1, float x2, float c1, float c2, float s1, float s2, bool adj,
                                         float& o1, float& o2) {
  if (!adj) {
    o1 = round_to<T>(__fsub_rn(round_to<T>(__fmul_rn(x1, c1)), round_to<T>(__fmul_rn(x2, s1))));
    o2 = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(x2, c2)), round_to<T>(__fmul_rn(x1, s2))));
  } else {
    o1 = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(x1, c1)), round_to<T>(__fmul_rn(x2, s2))));
    o2 = round_to<T>(__fsub_rn(round_to<T>(__fmul_rn(x2, c2)), round_to<T>(__fmul_rn(x1, s1))));
  }
}

// Packed bf16x2 arithmetic (sm_90+): each op rounds its exact result once
// to bf16, which is what torch's bf16 mul/add/sub produce (the float32
// intermediate of two bf16 operands cannot double-round differently).
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Rotate one 16-byte chunk pair (x1 at column j, x2 at j+D/2).
template <typename T, bool adj>
__device__ __forceinline__ void rot_chunk(const uint4& x1, const uint4& x2, const uint4& c1, const uint4& c2,
                                          const uint4& s1, const uint4& s2, uint4& o1, uint4& o2) {
  if constexpr (sizeof(T) == 2) {
    const uint32_t* a = &x1.x;
    const uint32_t* bq = &x2.x;
    const uint32_t* C1 = &c1.x;
    const uint32_t* C2 = &c2.x;
    const uint32_t* S1 = &s1.x;
    const uint32_t* S2 = &s2.x;
    uint32_t* p1 = &o1.x;
    uint32_t* p2 = &o2.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (!adj) {
        p1[q] = bsub2(bmul2(a[q], C1[q]), bmul2(bq[q], S1[q]));
        p2[q] = badd2(bmul2(bq[q], C2[q]), bmul2(a[q], S2[q]));
      } else {
        p1[q] = badd2(bmul2(a[q], C1[q]), bmul2(bq[q], S2[q]));
        p2[q] = bsub2(bmul2(bq[q], C2[q]), bmul2(a[q], S1[q]));
      }
    }
  } else {
    const float* a = reinterpret_cast<const float*>(&x1);
    const float* bq = reinterpret_cast<const float*>(&x2);
    const float* C1 = reinterpret_cast<const float*>(&c1);
    const float* C2 = reinterpret_cast<const float*>(&c2);
    const float* S1 = reinterpret_cast<const float*>(&s1);
    const float* S2 = reinterpret_cast<const float*>(&s2);
    float* p1 = reinterpret_cast<float*>(&o1);
    float* p2 = reinterpret_cast<float*>(&o2);
#pragma unroll
    for (int q = 0; q < 4; ++q) rot_pair<float>(a[q], bq[q], C1[q], C2[q], S1[q], S2[q], adj, p1[q], p2[q]);
  }
}

// Vectorised: one thread per (token, head group, 16-byte chunk pair).  The
// thread loads its four cos/sin chunks (L2-resident tables) and rotates that
// chunk pair in the kHG heads of its group, kUH heads per step so 2*kUH loads
// are in flight.  Groups of 8 heads give about six blocks per resident block
// slot on 148 SMs at the 7B shapes, so the last wave is short.
constexpr int kUH = 4;
constexpr int kHG = 8;

template <typename T, bool adj>
__global__ void __launch_bounds__(256, 3) rope_vec_kernel(RopeTensor q, RopeTensor k, const T* __restrict__ cosp,
                                                        const T* __restrict__ sinp, int64_t cs_stride, int S,
                                                        int half, int n_tokens, int gq, int gk) {
  constexpr int N = Chunk<T>::N;
  const unsigned cph = (unsigned)half / N;  // chunk pairs per head row
  const unsigned G = (unsigned)(gq + gk);
  // the launcher keeps every thread index below 2^31, so 32-bit index math is exact
  const unsigned idx = blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned rest = idx / cph;
  const unsigned tok = rest / G;
  if (tok >= (unsigned)n_tokens) return;
  const int j = (int)(idx - rest * cph) * N;
  const int g = (int)(rest - tok * G);
  const unsigned b = tok / (unsigned)S, s = tok - b * (unsigned)S;
  const T* cs = cosp + (int64_t)s * cs_stride + j;
  const T* sn = sinp + (int64_t)s * cs_stride + j;
  const uint4 c1 = *reinterpret_cast<const uint4*>(cs);
  const uint4 s1 = *reinterpret_cast<const uint4*>(sn);
  const uint4 c2 = *reinterpret_cast<const uint4*>(cs + half);
  const uint4 s2 = *reinterpret_cast<const uint4*>(sn + half);
  // field-wise selects keep the chosen tensor's description in registers
  const bool isq = g < gq;
  const int heads = (int)(isq ? q.heads : k.heads);
  const int64_t is_h = isq ? q.is_h : k.is_h, os_h = isq ? q.os_h : k.os_h;
  const int hb = (isq ? g : g - gq) * kHG;
  const int nh = heads - hb < kHG ? heads - hb : kHG;
  const T* src = static_cast<const T*>(isq ? q.in : k.in) + (int64_t)b * (isq ? q.is_b : k.is_b) +
                 (int64_t)s * (isq ? q.is_s : k.is_s) + (int64_t)hb * is_h + j;
  T* dst = static_cast<T*>(isq ? q.out : k.out) + (int64_t)b * (isq ? q.os_b : k.os_b) +
           (int64_t)s * (isq ? q.os_s : k.os_s) + (int64_t)hb * os_h + j;
#pragma unroll 1
  for (int h0 = 0; h0 < nh; h0 += kUH, src += kUH * is_h, dst += kUH * os_h) {
    uint4 x1[kUH], x2[kUH];
#pragma unroll
    for (int u = 0; u < kUH; ++u) {
      if (h0 + u < nh) {
        x1[u] = *reinterpret_cast<const uint4*>(src + u * is_h);
        x2[u] = *reinterpret_cast<const uint4*>(src + u * is_h + half);
      }
    }
#pragma unroll
    for (int u = 0; u < kUH; ++u) {
      if (h0 + u < nh) {
        uint4 o1, o2;
        rot_chunk<T, adj>(x1[u], x2[u], c1, c2, s1, s2, o1, o2);
        *reinterpret_cast<uint4*>(dst + u * os_h) = o1;
        *reinterpret_cast<uint4*>(dst + u * os_h + half) = o2;
      }
    }
  }
}

// Scalar fallback: one thread per element pair, any strides and D.
template <typename T>
__global__ void __launch_bounds__(256) rope_scalar_kernel(RopeTensor q, RopeTensor k, const T* __restrict__ cosp,
                                                           const T* __restrict__ sinp, int64_t cs_stride, int64_t S,
                                                           int64_t D, int64_t n_items, bool adj) {
  const int64_t half = D / 2;
  const int64_t heads = q.heads + k.heads;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < n_items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = it % half;
    const int64_t rest = it / half;
    const int64_t hh = rest % heads;
    const int64_t tok = rest / heads;
    const int64_t s = tok % S, b = tok / S;
    const bool isq = hh < q.heads;
    const RopeTensor& t = isq ? q : k;
    const int64_t h = isq ? hh : hh - q.heads;
    const T* src = static_cast<const T*>(t.in) + b * t.is_b + h * t.is_h + s * t.is_s;
    T* dst = static_cast<T*>(t.out) + b * t.os_b + h * t.os_h + s * t.os_s;
    const float x1 = Cvt<T>::to_f(src[j]), x2 = Cvt<T>::to_f(src[j + half]);
    const float c1 = Cvt<T>::to_f(cosp[s * cs_stride + j]), c2 = Cvt<T>::to_f(cosp[s * cs_stride + j + half]);
    const float s1 = Cvt<T>::to_f(sinp[s * cs_stride + j]), s2 = Cvt<T>::to_f(sinp[s * cs_stride + j + half]);
    float o1, o2;
    rot_pair<T>(x1, x2, c1, c2, s1, s2, adj, o1, o2);
    dst[j] = Cvt<T>::from_f(o1);
    dst[j + half] = Cvt<T>::from_f(o2);
  }
}

bool tensor_vec_ok(const RopeTensor& t, int N) {
  if (t.heads == 0) return true;
  return aligned16(t.in) && aligned16(t.out) && t.is_b % N == 0 && t.is_h % N == 0 && t.is_s % N == 0 &&
         t.os_b % N == 0 && t.os_h % N == 0 && t.os_s % N == 0;
}

template <typename T>
int launch(const RopeTensor& q, const RopeTensor& k, const void* cosp, const void* sinp, int64_t cs_stride,
           int64_t B, int64_t S, int64_t D, bool adj, cudaStream_t st) {
  constexpr int N = Chunk<T>::N;
  const int64_t heads = q.heads + k.heads;
  bool vec = ((D / 2) % N) == 0 && tensor_vec_ok(q, N) && tensor_vec_ok(k, N) && aligned16(cosp) &&
             aligned16(sinp) && (cs_stride % N) == 0;
  const int64_t n_tokens = B * S;
  if (n_tokens * heads == 0) return ATS_OK;
  if (vec) {
    const int64_t gq = (q.heads + kHG - 1) / kHG, gk = (k.heads + kHG - 1) / kHG;
    const int64_t threads = n_tokens * (gq + gk) * ((D / 2) / N);
    vec = threads + 255 < ((int64_t)1 << 31) && S < ((int64_t)1 << 31);
    if (vec) {
      const unsigned blocks = (unsigned)((threads + 255) / 256);
      if (adj)
        rope_vec_kernel<T, true><<<blocks, 256, 0, st>>>(q, k, static_cast<const T*>(cosp),
                                                         static_cast<const T*>(sinp), cs_stride, (int)S, (int)(D / 2),
                                                         (int)n_tokens, (int)gq, (int)gk);
      else
        rope_vec_kernel<T, false><<<blocks, 256, 0, st>>>(q, k, static_cast<const T*>(cosp),
                                                          static_cast<const T*>(sinp), cs_stride, (int)S, (int)(D / 2),
                                                          (int)n_tokens, (int)gq, (int)gk);
    }
  }
  if (!vec) {  // any strides or head size, or more work items than 32-bit indices cover
    const int64_t n_items = n_tokens * heads * (D / 2);
    const int64_t cap = (int64_t)num_sms() * 16;
    int64_t blocks = (n_items + 255) / 256;
    if (blocks > cap) blocks = cap;
    rope_scalar_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(q, k, static_cast<const T*>(cosp),
                                                              static_cast<const T*>(sinp), cs_stride, S, D, n_items,
                                                              adj);
  }
  return check_launch("rope_apply");
}

}  // namespace
}  // namespace ats

using namespace ats;

extern "C" int ats_rope_apply(const void* q_in, void* q_out, int64_t Hq, const int64_t q_in_strides[3],
                              const int64_t q_out_strides[3], const void* k_in, void* k_out, int64_t Hk,
                              const int64_t k_in_strides[3], const int64_t k_out_strides[3], const void* cosp,
                              const void* sinp, int64_t cs_row_stride, int64_t B, int64_t S, int64_t D,
                              ats_dtype x_dtype, int backward, void* stream) {
  if (B < 0 || S < 0 || D <= 0 || (D % 2) != 0 || Hq < 0)
    return fail(ATS_EBADARG, "rope_apply: bad shape B=%lld S=%lld D=%lld Hq=%lld", (long long)B, (long long)S,
                (long long)D, (long long)Hq);
  if (x_dtype != ATS_F32 && x_dtype != ATS_BF16) return fail(ATS_EBADARG, "rope_apply: unsupported dtype");
  if (q_in_strides == nullptr || q_out_strides == nullptr) return fail(ATS_EBADARG, "rope_apply: null strides");
  const bool has_k = k_in != nullptr;
  if (has_k && (k_out == nullptr || Hk < 0 || k_in_strides == nullptr || k_out_strides == nullptr))
    return fail(ATS_EBADARG, "rope_apply: incomplete k arguments");
  if (B * S * (Hq + (has_k ? Hk : 0)) == 0) return ATS_OK;
  if ((Hq > 0 && (q_in == nullptr || q_out == nullptr)) || cosp == nullptr || sinp == nullptr)
    return fail(ATS_EBADARG, "rope_apply: null pointer");
  if (cs_row_stride < D && cs_row_stride != 0)
    return fail(ATS_EBADARG, "rope_apply: cos/sin row stride must be 0 (one row for all positions) or >= D");
  RopeTensor q{q_in, q_out, Hq, q_in_strides[0], q_in_strides[1], q_in_strides[2],
               q_out_strides[0], q_out_strides[1], q_out_strides[2]};
  RopeTensor k{nullptr, nullptr, 0, 0, 0, 0, 0, 0, 0};
  if (has_k)
    k = RopeTensor{k_in, k_out, Hk, k_in_strides[0], k_in_strides[1], k_in_strides[2],
                   k_out_strides[0], k_out_strides[1], k_out_strides[2]};
  cudaStream_t st = (cudaStream_t)stream;
  if (x_dtype == ATS_BF16) return launch<bf16>(q, k, cosp, sinp, cs_row_stride, B, S, D, backward != 0, st);
  return launch<float>(q, k, cosp, sinp, cs_row_stride, B, S, D, backward != 0, st);
}
