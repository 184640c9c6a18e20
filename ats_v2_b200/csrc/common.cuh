// Shared device/host helpers for the ats_b200 sm_100a library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/ats_b200.h"

namespace ats {

// ---------------------------------------------------------------------------
// error reporting: every C entry point returns an ats status; the detail text
// of the last failure on this host thread is kept for ats_last_error_message.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

void count_launch();  // process-wide count of this library's kernel launches

// Checks the launch just made (exactly one launch per call); returns ATS_OK or
// ATS_ECUDA with the CUDA text.
inline int check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ATS_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return ATS_OK;
}

#define ATS_TRY(expr)               \
  do {                              \
    int _st = (expr);               \
    if (_st != ATS_OK) return _st;  \
  } while (0)

int num_sms();  // SM count of the current device (cached per device)
// Main-loop wait budget of the RMSNorm ring kernels on the current device (SM
// cycles; <= 0 restores the default), and the first code of a ring wait that
// gave up there since the last call (0: none), which this call clears.
int ring_set_wait_budget(long long cycles);
int ring_take_status(int* code);
// The first failed check of a device-driven exchange kernel on the current
// device since the last call (0: none), which this call clears.
int ep_take_status(int* code);
int gemm_ctas();  // CTAs of a persistent GEMM: num_sms() or this thread's lower limit
bool gemm_pairs();  // expert / dense / MLA GEMMs on CTA pairs (ats_set_gemm_pairs)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
typedef __nv_bfloat16 bf16;

template <typename T> struct Cvt;
template <> struct Cvt<float> {
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <> struct Cvt<bf16> {
  __device__ __forceinline__ static float to_f(bf16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static bf16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Round a float to the precision of T (identity for float).
template <typename T>
__device__ __forceinline__ float round_to(float v) { return Cvt<T>::to_f(Cvt<T>::from_f(v)); }

// 16-byte chunk of T: 8 bf16 or 4 float.
template <typename T> struct Chunk { static constexpr int N = 16 / sizeof(T); };

template <typename T>
__device__ __forceinline__ void load_chunk(const T* p, float (&v)[Chunk<T>::N]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Chunk<T>::N; ++i) v[i] = Cvt<T>::to_f(e[i]);
}

template <typename T>
__device__ __forceinline__ void pack_chunk(const float (&v)[Chunk<T>::N], uint4& raw) {
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Chunk<T>::N; ++i) e[i] = Cvt<T>::from_f(v[i]);
}

template <typename T>
__device__ __forceinline__ void store_chunk(T* p, const float (&v)[Chunk<T>::N]) {
  uint4 raw;
  pack_chunk<T>(v, raw);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Load N consecutive values of T (N*sizeof(T) a multiple of 16) as floats.
template <typename T, int N>
__device__ __forceinline__ void load_n(const T* p, float (&v)[N]) {
  constexpr int C = Chunk<T>::N;
  static_assert(N % C == 0, "load_n: N must be a multiple of the chunk size");
#pragma unroll
  for (int c = 0; c < N / C; ++c) {
    float t[C];
    load_chunk<T>(p + c * C, t);
#pragma unroll
    for (int i = 0; i < C; ++i) v[c * C + i] = t[i];
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_n(T* p, const float (&v)[N]) {
  constexpr int C = Chunk<T>::N;
  static_assert(N % C == 0, "store_n: N must be a multiple of the chunk size");
#pragma unroll
  for (int c = 0; c < N / C; ++c) {
    float t[C];
#pragma unroll
    for (int i = 0; i < C; ++i) t[i] = v[c * C + i];
    store_chunk<T>(p + c * C, t);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace ats
