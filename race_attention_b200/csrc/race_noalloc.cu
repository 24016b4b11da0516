// race_noalloc.cu -- race_fwd_probs_noalloc: the probability-level forward
// without any caller-provided workspace.
//
// Who needs this: code that hands us only its input and output buffers and
// cannot give us device memory for scratch.  Typical cases are a host
// application that has already carved the whole device into its own pool and
// forbids side allocations, a plugin callback whose contract is "enqueue work
// on this stream, allocate nothing", and a tight launch loop that cannot
// afford cudaMalloc/cudaFree (cudaFree waits for the whole device).  For them
// the chunk records of the scan live in one library-owned array, declared
// below as a file-scope static __device__ array of RACE_NOALLOC_SCRATCH_BYTES
// bytes.  The driver reserves it on each GPU when this file's module is first
// loaded there and keeps it until the process exits.
//
// Rules that follow from one shared array:
//  * Host code never uses the array's name as a device address; the address
//    is looked up once per device with cudaGetSymbolAddress (with that device
//    current) and passed to the kernels as an ordinary pointer.  The first
//    call on a device performs that lookup, so make the first call outside any
//    stream capture (a lookup that failed is not remembered: the next call
//    on that device tries again).
//  * Every call reuses the same bytes and they keep the previous call's
//    contents.  Nothing here relies on them being zero: the chunk-totals
//    kernel writes every record the scan and readout later read.
//  * Calls whose GPU work overlaps (different streams, or different host
//    threads without ordering between their streams) race on the array and
//    produce wrong results.  Serialise them.
//  * Problems whose chunk records do not fit are rejected with
//    RACE_ERR_WORKSPACE before any GPU work; streams are processed in groups
//    that fit.
#include "race_b200.h"

#include <mutex>
#include <stdio.h>

#include "generic.cuh"
#include "internal.h"

namespace {

namespace gen = race::gen;

static __device__ __align__(256) unsigned char g_noalloc_scratch[RACE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;

// Address of the array on each device, looked up on first use.  Only a
// successful lookup is kept: a lookup that failed (for example one attempted
// during a stream capture) is retried by the next call.
std::mutex g_dev_mu;
void *g_dev_ptr[kMaxDevices] = {};

int err(int code, const char *fmt, long long a = 0, long long b = 0) {
  char buf[256];
  snprintf(buf, sizeof(buf), fmt, a, b);
  return race::report_error(code, buf);
}

int scratch_for_current_device(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return err(RACE_ERR_CUDA, "cudaGetDevice failed (%lld)", (long long)e);
  if (dev < 0 || dev >= kMaxDevices) return err(RACE_ERR_UNSUPPORTED, "device ordinal %lld >= %lld", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (g_dev_ptr[dev] == nullptr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // the next call on this device tries again
      return err(RACE_ERR_CUDA, "cudaGetSymbolAddress of the scratch array failed (%lld)", (long long)e);
    }
    g_dev_ptr[dev] = p;
  }
  *out = g_dev_ptr[dev];
  return RACE_OK;
}

int launched(const char *what) {
  race::note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    return race::report_error(RACE_ERR_CUDA, buf);
  }
  return RACE_OK;
}

}  // namespace

extern "C" int race_fwd_probs_noalloc(const float *probsK, const float *probsQ, const float *V2, float *out,
                                      int64_t N, int64_t T, int64_t S, int64_t D, float eps, void *stream) {
  if (!probsK || !probsQ || !V2 || !out) return err(RACE_ERR_ARG, "probsK, probsQ, V2 and out must not be NULL");
  if (N < 1 || N > 65535) return err(RACE_ERR_SHAPE, "N=%lld out of range [1,65535]", N);
  if (T < 1 || T > (int64_t(1) << 31) - 1) return err(RACE_ERR_SHAPE, "T=%lld out of range [1,2^31)", T);
  if (S < 1 || S > 1024) return err(RACE_ERR_SHAPE, "S=%lld out of range [1,1024]", S);
  if (D < 1 || D > gen::MAX_D) return err(RACE_ERR_SHAPE, "D=%lld out of range [1,%lld]", D, gen::MAX_D);
  const int64_t G = (T + gen::GC - 1) / gen::GC;
  const size_t per_stream = sizeof(float) * (size_t)G * gen::state_elems((int)S, (int)D);
  if (per_stream > (size_t)RACE_NOALLOC_SCRATCH_BYTES)
    return err(RACE_ERR_WORKSPACE,
               "scratch for one stream needs %lld bytes, more than the %lld-byte static array; "
               "use race_fwd_probs with a workspace",
               (long long)per_stream, (long long)RACE_NOALLOC_SCRATCH_BYTES);
  void *scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != RACE_OK) return rc;
  float *St = static_cast<float *>(scratch);
  int64_t grp = (int64_t)(RACE_NOALLOC_SCRATCH_BYTES / per_stream);
  if (grp > N) grp = N;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  const size_t sm_tot = sizeof(float) * ((size_t)gen::GC * D + gen::GC * gen::GST);
  const size_t sm_ro = gen::fwd_readout_smem((int)D);
  cudaError_t ea = cudaFuncSetAttribute(gen::fwd_totals<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)sm_tot);
  if (ea == cudaSuccess)
    ea = cudaFuncSetAttribute(gen::fwd_readout<float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_ro);
  if (ea != cudaSuccess) return err(RACE_ERR_CUDA, "cudaFuncSetAttribute failed (%lld)", (long long)ea);

  for (int64_t n0 = 0; n0 < N; n0 += grp) {
    const int64_t nn = (N - n0) < grp ? (N - n0) : grp;
    gen::Dims p;
    p.N = (int)nn;
    p.T = (int)T;
    p.S = (int)S;
    p.D = (int)D;
    p.G = (int)G;
    p.eps = eps;
    const size_t po = (size_t)n0 * T * S, xo = (size_t)n0 * T * D;
    gen::fwd_totals<float><<<dim3(p.G, p.N), gen::NT, sm_tot, s>>>(probsK + po, V2 + xo, St, p);
    if ((rc = launched("fwd_totals")) != RACE_OK) return rc;
    const size_t E = gen::state_elems(p.S, p.D);
    gen::chunk_scan<<<dim3((unsigned)((E + 255) / 256), p.N), 256, 0, s>>>(St, nullptr, nullptr, nullptr, nullptr,
                                                                            p.N, p.G, p.S, p.D, 0);
    if ((rc = launched("chunk_scan")) != RACE_OK) return rc;
    gen::fwd_readout<float, float><<<dim3(p.G, p.N), gen::NT, sm_ro, s>>>(probsK + po, probsQ + po, V2 + xo, St,
                                                                           out + xo, p);
    if ((rc = launched("fwd_readout")) != RACE_OK) return rc;
  }
  race::clear_error();
  return RACE_OK;
}
