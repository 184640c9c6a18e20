// Library-wide C ABI pieces: version, status strings, last-error text, SM count.
#include "common.cuh"
#include "moe_gemm.cuh"

#include <atomic>
#include <string.h>

namespace ats {

static thread_local char g_last_error[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int num_sms() {
  // Per-device cache; device ordinals are small.  Written before first read
  // on each thread that asks, and the value never changes, so a benign race.
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// CTAs a persistent GEMM may launch with on this host thread: 0 = one per SM.
// A caller that runs a collective on another stream beside the GEMMs lowers it
// so that the collective's blocks find free SMs (a GEMM CTA fills its SM).
static thread_local int g_gemm_sm_limit = 0;

int gemm_ctas() {
  const int n = num_sms();
  return (g_gemm_sm_limit > 0 && g_gemm_sm_limit < n) ? g_gemm_sm_limit : n;
}

// Whether the expert, dense and MLA GEMMs run 256-row tiles on CTA pairs (cta_group::2) or 128-row tiles on
// single CTAs (the default: as fast on long-K GEMMs, faster on the short expert segments of an
// expert-parallel step).  Process-wide; each GEMM entry point reads it once.
static std::atomic<int> g_gemm_pairs{0};

bool gemm_pairs() { return g_gemm_pairs.load(std::memory_order_relaxed) != 0; }

}  // namespace ats

extern "C" {

int ats_abi_version(void) { return ATS_ABI_VERSION; }

const char* ats_strerror(int status) {
  switch (status) {
    case ATS_OK: return "ok";
    case ATS_EBADARG: return "invalid argument";
    case ATS_EUNSUPPORTED: return "unsupported configuration";
    case ATS_ECUDA: return "CUDA error";
    case ATS_ETIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* ats_last_error_message(void) { return ats::g_last_error; }

uint64_t ats_kernel_launches(void) { return ats::g_launches.load(std::memory_order_relaxed); }

int ats_set_gemm_sm_limit(int sms) {
  if (sms < 0) return ats::fail(ATS_EBADARG, "set_gemm_sm_limit: %d SMs", sms);
  ats::g_gemm_sm_limit = sms;
  return ATS_OK;
}

int ats_gemm_sm_limit(void) { return ats::g_gemm_sm_limit; }

int ats_set_gemm_pairs(int enable) {
  ats::g_gemm_pairs.store(enable != 0 ? 1 : 0, std::memory_order_relaxed);
  return ATS_OK;
}

int ats_gemm_pairs(void) { return ats::g_gemm_pairs.load(std::memory_order_relaxed); }

int ats_set_wait_budget(int64_t cycles) {
  ATS_TRY(ats::gemm_set_wait_budget((long long)cycles));
  return ats::ring_set_wait_budget((long long)cycles);
}

int ats_device_status(int* status) {
  if (status == nullptr) return ats::fail(ATS_EBADARG, "device_status: null output");
  int g = 0, r = 0, x = 0;
  ATS_TRY(ats::gemm_take_status(&g));
  ATS_TRY(ats::ring_take_status(&r));
  ATS_TRY(ats::ep_take_status(&x));
  *status = g != 0 ? g : r;
  if (*status != 0)
    return ats::fail(ATS_ETIMEOUT, "a bounded device wait gave up (%s code %d); the results of that call are undefined",
                     g != 0 ? "tensor-core GEMM" : "RMSNorm ring", *status);
  *status = x;
  if (x == 0) return ATS_OK;
  return ats::fail(ATS_EBADARG, "expert-parallel exchange: a row fell outside its buffer or the ranks' capacities "
                   "differ (code %d); the rows of that step are undefined", x);
}

}  // extern "C"
