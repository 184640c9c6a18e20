// Rotate-half rotary embedding for q and k in one launch, forward and adjoint.
//
// Work item = (token, head, chunk pair): a thread loads the 16-byte chunk at
// column j of the first half of a head row and the matching chunk at j+D/2,
// plus the cos/sin chunks of the token's position, and writes both output
// chunks.  Items are ordered token-major, then head, then chunk, so for the
// attention layout (BSHD memory viewed as [B,H,S,D]) consecutive threads
// stream consecutive memory, and the 4*D bytes of cos/sin for a position are
// reused from L1 by all Hq+Hk heads of that token.  q/k are read once and
// written once: one HBM pass in each direction.
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

// Vectorised: D/2 a multiple of the chunk size, strides and pointers aligned.
// Block b handles tokens [b*TPB, b*TPB+TPB); within it, item i decomposes
// (32-bit) into (token, head, chunk pair).
constexpr int kTokensPerBlock = 4;

template <typename T>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeTensor q, RopeTensor k, const T* __restrict__ cosp,
                                                        const T* __restrict__ sinp, int64_t cs_stride, int64_t S,
                                                        int64_t D, int64_t n_tokens, bool adj) {
  constexpr int N = Chunk<T>::N;
  const int half = (int)(D / 2);
  const int cph = half / N;  // chunk pairs per head row
  const int heads = (int)(q.heads + k.heads);
  const int per_tok = heads * cph;
  const int64_t tok0 = (int64_t)blockIdx.x * kTokensPerBlock;
  int64_t ntok = n_tokens - tok0;
  if (ntok > kTokensPerBlock) ntok = kTokensPerBlock;
  const int items = (int)ntok * per_tok;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int tl = i / per_tok;
    const int r = i - tl * per_tok;
    const int hh = r / cph;
    const int cp = r - hh * cph;
    const int64_t tok = tok0 + tl;
    const int64_t b = tok / S, s = tok - b * S;
    const bool isq = hh < q.heads;
    const RopeTensor& t = isq ? q : k;
    const int64_t h = isq ? hh : hh - q.heads;
    const int j = cp * N;
    const T* src = static_cast<const T*>(t.in) + b * t.is_b + h * t.is_h + s * t.is_s;
    T* dst = static_cast<T*>(t.out) + b * t.os_b + h * t.os_h + s * t.os_s;
    float x1[N], x2[N], c1[N], c2[N], s1[N], s2[N], o1[N], o2[N];
    load_chunk<T>(src + j, x1);
    load_chunk<T>(src + j + half, x2);
    const T* cr = cosp + s * cs_stride;
    const T* sr = sinp + s * cs_stride;
    load_chunk<T>(cr + j, c1);
    load_chunk<T>(cr + j + half, c2);
    load_chunk<T>(sr + j, s1);
    load_chunk<T>(sr + j + half, s2);
#pragma unroll
    for (int e = 0; e < N; ++e) rot_pair<T>(x1[e], x2[e], c1[e], c2[e], s1[e], s2[e], adj, o1[e], o2[e]);
    store_chunk<T>(dst + j, o1);
    store_chunk<T>(dst + j + half, o2);
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
  const bool vec = ((D / 2) % N) == 0 && tensor_vec_ok(q, N) && tensor_vec_ok(k, N) && aligned16(cosp) &&
                   aligned16(sinp) && (cs_stride % N) == 0;
  const int64_t n_tokens = B * S;
  if (n_tokens * heads == 0) return ATS_OK;
  if (vec && heads * (D / 2) / N < (int64_t)1 << 28) {
    const int64_t blocks = (n_tokens + kTokensPerBlock - 1) / kTokensPerBlock;
    if (blocks >= ((int64_t)1 << 31)) return fail(ATS_EUNSUPPORTED, "rope_apply: too many tokens");
    rope_vec_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(q, k, static_cast<const T*>(cosp),
                                                           static_cast<const T*>(sinp), cs_stride, S, D, n_tokens,
                                                           adj);
  } else {
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
