// Peer-memory pieces of the expert-parallel row exchange.
//
// A rank exports the device buffers its peers write into (CUDA IPC handles of
// their base allocations plus the buffer's offset in it); each peer maps them
// once and, every step, copies rows straight into them with the copy engines
// (cudaMemcpyAsync over NVLink).  The copy engines take no SMs, so the
// transfers run beside the expert GEMMs.  Ordering between ranks is the
// caller's: it issues the copies on a stream that waits for a collective every
// rank reaches only after its earlier reads of these buffers, and makes readers
// wait for a collective issued after the copies.
#include "common.cuh"

#include <cuda.h>
#include <string.h>

namespace ats {
namespace {

typedef CUresult (*PFN_addressRange)(CUdeviceptr* base, size_t* size, CUdeviceptr ptr);
PFN_addressRange g_range = nullptr;

int range_fn(PFN_addressRange* out) {
  if (g_range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_addressRange>(fn);
  }
  if (g_range == nullptr) return fail(ATS_ECUDA, "peer: cuMemGetAddressRange unavailable");
  *out = g_range;
  return ATS_OK;
}

}  // namespace
}  // namespace ats

extern "C" {

size_t ats_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int ats_ipc_export(const void* ptr, void* handle, uint64_t* offset, uint64_t* alloc_bytes) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return ats::fail(ATS_EBADARG, "ipc_export: null argument");
  ats::PFN_addressRange range;
  ATS_TRY(ats::range_fn(&range));
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return ats::fail(ATS_ECUDA, "ipc_export: address range lookup failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return ats::fail(ATS_ECUDA, "ipc_export: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  if (alloc_bytes != nullptr) *alloc_bytes = static_cast<uint64_t>(size);
  return ATS_OK;
}

int ats_ipc_open(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr) return ats::fail(ATS_EBADARG, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ats::fail(ATS_ECUDA, "ipc_open: %s", cudaGetErrorString(e));
  return ATS_OK;
}

int ats_ipc_close(void* base) {
  if (base == nullptr) return ats::fail(ATS_EBADARG, "ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return ats::fail(ATS_ECUDA, "ipc_close: %s", cudaGetErrorString(e));
  return ATS_OK;
}

int ats_peer_copies(int n, void* const* dst, const void* const* src, const uint64_t* bytes, void* stream) {
  if (n < 0 || (n > 0 && (dst == nullptr || src == nullptr || bytes == nullptr)))
    return ats::fail(ATS_EBADARG, "peer_copies: bad arguments");
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    if (dst[i] == nullptr || src[i] == nullptr) return ats::fail(ATS_EBADARG, "peer_copies: null pointer in copy %d", i);
    const cudaError_t e = cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyDefault, (cudaStream_t)stream);
    if (e != cudaSuccess) return ats::fail(ATS_ECUDA, "peer_copies: copy %d: %s", i, cudaGetErrorString(e));
  }
  return ATS_OK;
}

}  // extern "C"
