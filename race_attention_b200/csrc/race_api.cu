// race_api.cu -- extern "C" entry points of librace_b200.so (see include/race_b200.h).
//
// Host code only: argument validation, workspace carving and kernel dispatch.
// Nothing here allocates device memory; launches go on the caller's stream.
#include "race_b200.h"

// the generic path's layout for the gradient-totals half of the split backward
#define RACE_OP_BWD_TOTALS RACE_OP_BWD_SPLIT

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <algorithm>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <set>
#include <type_traits>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "common.cuh"
#include "decode.cuh"
#include "fast_host.cuh"
#include "generic.cuh"
#include "noncausal.cuh"

using race::align_up;
namespace gen = race::gen;

namespace {

thread_local char g_err[512] = {0};

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = 0;
  return RACE_OK;
}

std::atomic<unsigned long long> g_launches{0};

// Bounded-wait controls of the tcgen05 kernels (race_set_wait_limit,
// race_set_status_check, race_test_withhold_first_load): process-wide
// settings read when a call launches its kernels.
std::atomic<uint32_t> g_wait_limit{0};  // 0: tc::kDefaultWaitPolls
std::atomic<int> g_status_check{0};
std::atomic<int> g_withhold_first_load{0};

uint32_t wait_limit() {
  const uint32_t v = g_wait_limit.load(std::memory_order_relaxed);
  return v ? v : race::tc::kDefaultWaitPolls;
}

int check_launch(const char *what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

// Per-kernel device timing of the tcgen05 path (race_kernel_timing): an event
// pair recorded on the launch stream around each launch while enabled.
struct KernelTimer {
  std::mutex mu;
  bool on = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending[RACE_KT_COUNT];
  double ms[RACE_KT_COUNT] = {};
  long long launches[RACE_KT_COUNT] = {};
};

KernelTimer &ktimer() {
  static KernelTimer t;
  return t;
}

// NVTX range over a host-side phase (a profiler shows each tcgen05 launch and each
// forward / backward call by name; without a profiler attached these are no-ops).
class NvtxRange {
 public:
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

const char *kernel_range_name(int id) {
  static const char *names[RACE_KT_COUNT] = {"race fwd_totals_kernel", "race fwd_readout_kernel",
                                             "race bwd_rev_kernel", "race chunk_scan", "race bwd_fix_kernel",
                                             "race ace_tile_kernel"};
  return id >= 0 && id < RACE_KT_COUNT ? names[id] : "race kernel";
}

class KernelScope {
 public:
  KernelScope(int id, cudaStream_t s) : id_(id), s_(s), range_(kernel_range_name(id)) {
    KernelTimer &t = ktimer();
    std::lock_guard<std::mutex> g(t.mu);
    if (!t.on) return;
    if (cudaEventCreate(&e0_) != cudaSuccess || cudaEventCreate(&e1_) != cudaSuccess ||
        cudaEventRecord(e0_, s_) != cudaSuccess) {
      release();
      cudaGetLastError();
    }
  }
  ~KernelScope() { release(); }
  void stop() {
    if (!e0_) return;
    if (cudaEventRecord(e1_, s_) == cudaSuccess) {
      KernelTimer &t = ktimer();
      std::lock_guard<std::mutex> g(t.mu);
      t.pending[id_].push_back({e0_, e1_});
      e0_ = e1_ = nullptr;
    }
    release();
  }

 private:
  void release() {
    if (e0_) cudaEventDestroy(e0_);
    if (e1_) cudaEventDestroy(e1_);
    e0_ = e1_ = nullptr;
  }
  int id_;
  cudaStream_t s_;
  NvtxRange range_;
  cudaEvent_t e0_ = nullptr, e1_ = nullptr;
};

constexpr int64_t kMaxN = 65535;
constexpr int64_t kMaxS = 1024;
constexpr int64_t kMaxT = (int64_t(1) << 31) - 1;

int check_nts(int64_t N, int64_t T, int64_t S, int64_t D) {
  if (N < 1 || N > kMaxN) return fail(RACE_ERR_SHAPE, "N=%lld out of range [1,%lld]", (long long)N, (long long)kMaxN);
  if (T < 1 || T > kMaxT) return fail(RACE_ERR_SHAPE, "T=%lld out of range [1,2^31)", (long long)T);
  if (S < 1 || S > kMaxS) return fail(RACE_ERR_SHAPE, "S=%lld out of range [1,%lld]", (long long)S, (long long)kMaxS);
  if (D < 1 || D > gen::MAX_D) return fail(RACE_ERR_SHAPE, "D=%lld out of range [1,%d]", (long long)D, gen::MAX_D);
  return RACE_OK;
}

int check_lp(int64_t L, int64_t P, int64_t *S) {
  if (P < 1 || P > 10) return fail(RACE_ERR_SHAPE, "P=%lld out of range [1,10]", (long long)P);
  if (L < 1 || (L << P) > kMaxS)
    return fail(RACE_ERR_SHAPE, "L=%lld, P=%lld gives S=L*2^P outside [1,%lld]", (long long)L, (long long)P,
                (long long)kMaxS);
  *S = L << P;
  return RACE_OK;
}

int check_dtype(int dtype) {
  if (dtype != RACE_F32 && dtype != RACE_BF16) return fail(RACE_ERR_DTYPE, "dtype %d not supported", dtype);
  return RACE_OK;
}

#define RACE_TRY(...)                 \
  do {                                \
    int _rc = (__VA_ARGS__);          \
    if (_rc != RACE_OK) return _rc;   \
  } while (0)

#define RACE_NONNULL(p) \
  if ((p) == nullptr) return fail(RACE_ERR_ARG, "%s must not be NULL", #p)

// ---- workspace layout of the generic path ---------------------------------
// Streams are processed in groups of `grp` so the workspace stays bounded
// (kGroupBudget per group, at least one stream per group).
struct Layout {
  size_t pk = 0, pq = 0, dpk = 0, dpq = 0, st = 0, st2 = 0, total = 0;
  int64_t grp = 1;
};

constexpr size_t kAlign = 256;
constexpr size_t kGroupBudget = size_t(4) << 30;

Layout layout_for(int op, int64_t n, int64_t T, int64_t S, int64_t D) {
  const int64_t G = (T + gen::GC - 1) / gen::GC;
  const size_t probs = sizeof(float) * (size_t)n * T * S;
  const size_t states = sizeof(float) * (size_t)n * G * gen::state_elems((int)S, (int)D);
  Layout w;
  w.grp = n;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes, kAlign);
    return at;
  };
  const bool qkv = op == RACE_OP_FWD_QKV || op == RACE_OP_BWD_QKV || op == RACE_OP_STATE || op == RACE_OP_BWD_TOTALS;
  if (qkv) w.pk = take(probs);
  if (op == RACE_OP_FWD_QKV || op == RACE_OP_BWD_QKV || op == RACE_OP_BWD_TOTALS) w.pq = take(probs);
  if (op == RACE_OP_BWD_QKV) {
    w.dpk = take(probs);
    w.dpq = take(probs);
  }
  w.st = take(states);
  if (op == RACE_OP_BWD_PROBS || op == RACE_OP_BWD_QKV || op == RACE_OP_BWD_TOTALS) w.st2 = take(states);
  w.total = off;
  return w;
}

Layout generic_layout(int op, int64_t N, int64_t T, int64_t S, int64_t D) {
  const size_t per_stream = layout_for(op, 1, T, S, D).total;
  int64_t grp = (int64_t)(kGroupBudget / (per_stream ? per_stream : 1));
  if (grp < 1) grp = 1;
  if (grp > N) grp = N;
  return layout_for(op, grp, T, S, D);
}

int check_ws(void *ws, size_t have, size_t need) {
  if (need == 0) return RACE_OK;
  if (ws == nullptr) return fail(RACE_ERR_WORKSPACE, "workspace is NULL but %zu bytes are required", need);
  if (have < need) return fail(RACE_ERR_WORKSPACE, "workspace has %zu bytes, %zu required", have, need);
  if (reinterpret_cast<uintptr_t>(ws) % kAlign) return fail(RACE_ERR_ALIGN, "workspace must be %zu-byte aligned", kAlign);
  return RACE_OK;
}

template <typename T>
T *at(void *ws, size_t off) {
  return reinterpret_cast<T *>(static_cast<char *>(ws) + off);
}

// All of the unified L1/shared array as shared memory, so that as many CTAs fit as
// their shared-memory needs allow (the driver's default split can leave room for
// fewer).  Set once per kernel and device: the first launch happens outside any
// stream capture, later ones (possibly inside a capture) make no runtime call.
int set_carveout(const void *kernel) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(RACE_ERR_CUDA, "cudaGetDevice failed");
  static std::mutex mu;
  static std::set<std::pair<const void *, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return RACE_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "cudaFuncSetAttribute(carveout): %s", cudaGetErrorString(e));
  done.insert({kernel, dev});
  return RACE_OK;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "cudaFuncSetAttribute(%zu B smem): %s", bytes, cudaGetErrorString(e));
  }
  return RACE_OK;
}

gen::Dims make_dims(int64_t N, int64_t T, int64_t S, int64_t D, float eps) {
  gen::Dims p;
  p.N = (int)N;
  p.T = (int)T;
  p.S = (int)S;
  p.D = (int)D;
  p.G = (int)((T + gen::GC - 1) / gen::GC);
  p.eps = eps;
  return p;
}

// ---- generic building blocks ------------------------------------------------
template <typename VT>
int launch_totals(const float *pk, const VT *V, float *St, const gen::Dims &p, cudaStream_t s) {
  const size_t sm = sizeof(float) * ((size_t)gen::GC * p.D + gen::GC * gen::GST);
  RACE_TRY(set_smem(gen::fwd_totals<VT>, sm));
  gen::fwd_totals<VT><<<dim3(p.G, p.N), gen::NT, sm, s>>>(pk, V, St, p);
  return check_launch("fwd_totals");
}

int launch_scan(float *St, const float *initA, const float *initB, float *finA, float *finB, const gen::Dims &p,
                int reverse, cudaStream_t s) {
  const size_t E = gen::state_elems(p.S, p.D);
  gen::chunk_scan<<<dim3((unsigned)((E + 255) / 256), p.N), 256, 0, s>>>(St, initA, initB, finA, finB, p.N, p.G, p.S,
                                                                          p.D, reverse);
  return check_launch("chunk_scan");
}

template <typename VT, typename OT>
int launch_readout(const float *pk, const float *pq, const VT *V, const float *St, OT *out, const gen::Dims &p,
                   cudaStream_t s) {
  const size_t sm = gen::fwd_readout_smem(p.D);
  RACE_TRY(set_smem(gen::fwd_readout<VT, OT>, sm));
  gen::fwd_readout<VT, OT><<<dim3(p.G, p.N), gen::NT, sm, s>>>(pk, pq, V, St, out, p);
  return check_launch("fwd_readout");
}

template <typename VT>
int launch_bwd_totals(const float *pk, const float *pq, const VT *V, const VT *dO, const float *St, float *St2,
                      float *dpq, const gen::Dims &p, cudaStream_t s) {
  const size_t sm = sizeof(float) * gen::bwd_smem_floats(p.D, false);
  RACE_TRY(set_smem(gen::bwd_totals<VT>, sm));
  gen::bwd_totals<VT><<<dim3(p.G, p.N), gen::NT, sm, s>>>(pk, pq, V, dO, St, St2, dpq, p);
  return check_launch("bwd_totals");
}

template <typename VT, typename OT>
int launch_bwd_readout(const float *pk, const float *pq, const VT *V, const VT *dO, const float *St,
                       const float *St2, float *dpk, OT *dV, const gen::Dims &p, cudaStream_t s) {
  const size_t sm = sizeof(float) * gen::bwd_smem_floats(p.D, true);
  RACE_TRY(set_smem(gen::bwd_readout<VT, OT>, sm));
  gen::bwd_readout<VT, OT><<<dim3(p.G, p.N), gen::NT, sm, s>>>(pk, pq, V, dO, St, St2, dpk, dV, p);
  return check_launch("bwd_readout");
}

template <typename XT>
int launch_hash(const XT *X, const float *planes_T, float *probs, int64_t rows, int64_t D, int64_t L, int64_t P,
                float scale, cudaStream_t s) {
  const size_t sm = sizeof(float) * ((size_t)gen::HT * D + (size_t)gen::HT * L * P);
  RACE_TRY(set_smem(gen::soft_hash_fwd<XT>, sm));
  const unsigned grid = (unsigned)((rows + gen::HT - 1) / gen::HT);
  gen::soft_hash_fwd<XT><<<grid, gen::NT, sm, s>>>(X, planes_T, probs, rows, (int)D, (int)L, (int)P, scale);
  return check_launch("soft_hash_fwd");
}

template <typename XT>
int launch_hash_bwd(const XT *X, const float *planes_T, const float *dprobs, XT *dX, int64_t rows, int64_t D,
                    int64_t L, int64_t P, float scale, cudaStream_t s) {
  const size_t sm = sizeof(float) * ((size_t)gen::HT * D + 2 * (size_t)gen::HT * L * P);
  RACE_TRY(set_smem(gen::soft_hash_bwd<XT>, sm));
  const unsigned grid = (unsigned)((rows + gen::HT - 1) / gen::HT);
  gen::soft_hash_bwd<XT><<<grid, gen::NT, sm, s>>>(X, planes_T, dprobs, dX, rows, (int)D, (int)L, (int)P, scale);
  return check_launch("soft_hash_bwd");
}

// ---- composite operations (templated on the activation dtype) -------------
// Each loops over stream groups of w.grp streams (see generic_layout).
template <typename T>
T *off(T *p, size_t o) {
  return p ? p + o : nullptr;
}

template <typename XT>
int fwd_qkv_generic(const XT *Q, const XT *K, const XT *V, const float *planes_T, XT *out, const float *A0,
                    const float *B0, float *Af, float *Bf, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                    float eps, float scale, void *ws, cudaStream_t s) {
  const int64_t S = L << P;
  const Layout w = generic_layout(RACE_OP_FWD_QKV, N, T, S, D);
  float *pk = at<float>(ws, w.pk), *pq = at<float>(ws, w.pq), *St = at<float>(ws, w.st);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t xo = (size_t)n0 * T * D, so = (size_t)n0 * S, bo = (size_t)n0 * S * D;
    const gen::Dims p = make_dims(nn, T, S, D, eps);
    RACE_TRY(launch_hash<XT>(Q + xo, planes_T, pq, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_hash<XT>(K + xo, planes_T, pk, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_totals<XT>(pk, V + xo, St, p, s));
    RACE_TRY(launch_scan(St, off(A0, so), off(B0, bo), off(Af, so), off(Bf, bo), p, 0, s));
    RACE_TRY(launch_readout<XT, XT>(pk, pq, V + xo, St, out + xo, p, s));
  }
  return RACE_OK;
}

template <typename XT>
int bwd_qkv_generic(const XT *Q, const XT *K, const XT *V, const XT *dO, const float *planes_T, XT *dQ, XT *dK,
                    XT *dV, const float *A0, const float *B0, const float *gA, const float *gB, float *dA0,
                    float *dB0, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps, float scale,
                    void *ws, cudaStream_t s) {
  const int64_t S = L << P;
  const Layout w = generic_layout(RACE_OP_BWD_QKV, N, T, S, D);
  float *pk = at<float>(ws, w.pk), *pq = at<float>(ws, w.pq), *dpk = at<float>(ws, w.dpk),
        *dpq = at<float>(ws, w.dpq), *St = at<float>(ws, w.st), *St2 = at<float>(ws, w.st2);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t xo = (size_t)n0 * T * D, so = (size_t)n0 * S, bo = (size_t)n0 * S * D;
    const gen::Dims p = make_dims(nn, T, S, D, eps);
    RACE_TRY(launch_hash<XT>(Q + xo, planes_T, pq, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_hash<XT>(K + xo, planes_T, pk, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_totals<XT>(pk, V + xo, St, p, s));
    RACE_TRY(launch_scan(St, off(A0, so), off(B0, bo), nullptr, nullptr, p, 0, s));
    RACE_TRY(launch_bwd_totals<XT>(pk, pq, V + xo, dO + xo, St, St2, dpq, p, s));
    RACE_TRY(launch_scan(St2, off(gA, so), off(gB, bo), off(dA0, so), off(dB0, bo), p, 1, s));
    RACE_TRY(launch_bwd_readout<XT, XT>(pk, pq, V + xo, dO + xo, St, St2, dpk, dV + xo, p, s));
    RACE_TRY(launch_hash_bwd<XT>(Q + xo, planes_T, dpq, dQ + xo, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_hash_bwd<XT>(K + xo, planes_T, dpk, dK + xo, nn * T, D, L, P, scale, s));
  }
  return RACE_OK;
}

template <typename XT>
int state_generic(const XT *K, const XT *V, const float *planes_T, const float *A0, const float *B0, float *Ao,
                  float *Bo, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float scale, void *ws,
                  cudaStream_t s) {
  const int64_t S = L << P;
  const Layout w = generic_layout(RACE_OP_STATE, N, T, S, D);
  float *pk = at<float>(ws, w.pk), *St = at<float>(ws, w.st);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t xo = (size_t)n0 * T * D, so = (size_t)n0 * S, bo = (size_t)n0 * S * D;
    const gen::Dims p = make_dims(nn, T, S, D, 0.f);
    RACE_TRY(launch_hash<XT>(K + xo, planes_T, pk, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_totals<XT>(pk, V + xo, St, p, s));
    RACE_TRY(launch_scan(St, off(A0, so), off(B0, bo), Ao + so, Bo + bo, p, 0, s));
  }
  return RACE_OK;
}

template <typename XT>
int bwd_totals_generic(const XT *Q, const XT *K, const XT *V, const XT *dO, const float *planes_T, const float *A0,
                       const float *B0, float *gA, float *gB, int64_t N, int64_t T, int64_t D, int64_t L,
                       int64_t P, float eps, float scale, void *ws, cudaStream_t s) {
  const int64_t S = L << P;
  const Layout w = generic_layout(RACE_OP_BWD_TOTALS, N, T, S, D);
  float *pk = at<float>(ws, w.pk), *pq = at<float>(ws, w.pq), *St = at<float>(ws, w.st), *St2 = at<float>(ws, w.st2);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t xo = (size_t)n0 * T * D, so = (size_t)n0 * S, bo = (size_t)n0 * S * D;
    const gen::Dims p = make_dims(nn, T, S, D, eps);
    RACE_TRY(launch_hash<XT>(Q + xo, planes_T, pq, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_hash<XT>(K + xo, planes_T, pk, nn * T, D, L, P, scale, s));
    RACE_TRY(launch_totals<XT>(pk, V + xo, St, p, s));
    RACE_TRY(launch_scan(St, off(A0, so), off(B0, bo), nullptr, nullptr, p, 0, s));
    RACE_TRY(launch_bwd_totals<XT>(pk, pq, V + xo, dO + xo, St, St2, nullptr, p, s));
    RACE_TRY(launch_scan(St2, nullptr, nullptr, gA + so, gB + bo, p, 1, s));
  }
  return RACE_OK;
}

cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- tcgen05 path (bf16, D=64, P=4, L in {8,16}) -----------------------------
namespace fh = race::fasthost;
namespace fk = race::fast;

int fast_args(fk::FwdArgs &a, const fh::Plan &pl, int64_t N, int64_t T, int64_t L, float eps, float scale,
              const float *planes_T, void *ws) {
  a.N = (int)N;
  a.T = (int)T;
  a.H = 1;
  a.L = (int)L;
  a.LP = (int)(4 * L);
  a.S = (int)(16 * L);
  a.ngroups = a.S / fk::GB;
  a.nseg = pl.nseg;
  a.seg_chunks = pl.seg_chunks;
  a.nchunks = pl.nchunks;
  a.eps = eps;
  a.scale = scale;
  a.poly = 2.f * std::fabs(scale) <= 0.5f ? 1 : 0;
  a.batch_rcp = eps >= 1e-8f ? 1 : 0;
  a.planes = planes_T;
  a.seg_state = at<float>(ws, pl.rec_off);
  a.seg_tot = at<float>(ws, pl.rec_off);
  a.out = nullptr;
  a.chunkA = nullptr;
  a.chunkB = nullptr;
  a.seedA = a.seedB = nullptr;
  a.err = at<int>(ws, pl.status_off);
  a.wait_limit = wait_limit();
  a.withhold_first_load = g_withhold_first_load.load(std::memory_order_relaxed);
  return RACE_OK;
}

// Plan, kernel arguments and K/V tensor maps of the forward kernels.
int fast_prepare(const void *K, const void *V, const float *planes_T, int64_t N, int64_t T, int64_t L, float eps,
                 float scale, void *ws, fk::FwdArgs &a, CUtensorMap &mK, CUtensorMap &mV, fh::Plan &pl,
                 size_t rec_off = 0, int64_t H = 1) {
  const int64_t S = 16 * L;
  if (!fh::bind_current_context()) return fail(RACE_ERR_CUDA, "no current CUDA device/context on this thread");
  pl = fh::plan(N, T, S, fh::sm_count());
  if (rec_off) pl.rec_off = rec_off;
  fast_args(a, pl, N, T, L, eps, scale, planes_T, ws);
  a.H = (int)H;
  if (!fh::make_act_map(&mK, K, N, T, H))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled(K %p, N=%lld, T=%lld) failed: CUresult %d", K, (long long)N,
                (long long)T, fh::last_encode_status());
  if (!fh::make_act_map(&mV, V, N, T, H))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled(V %p, N=%lld, T=%lld) failed: CUresult %d", V, (long long)N,
                (long long)T, fh::last_encode_status());
  return RACE_OK;
}

int fast_totals_and_scan(const void *K, const void *V, const float *planes_T, const float *A0, const float *B0,
                         float *Af, float *Bf, int64_t N, int64_t T, int64_t L, float eps, float scale, void *ws,
                         cudaStream_t s, fk::FwdArgs &a, CUtensorMap &mK, CUtensorMap &mV, size_t rec_off = 0,
                         int64_t H = 1) {
  const int64_t S = 16 * L;
  fh::Plan pl;
  RACE_TRY(fast_prepare(K, V, planes_T, N, T, L, eps, scale, ws, a, mK, mV, pl, rec_off, H));
  cudaError_t e = cudaMemsetAsync(at<int>(ws, pl.status_off), 0, sizeof(int), s);
  if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  const fk::TotSmem ts = fk::tot_smem_plan(a.ngroups, a.LP);
  RACE_TRY(set_smem(fk::fwd_totals_kernel, ts.total));
  {
    KernelScope ks(RACE_KT_FWD_TOTALS, s);
    fk::fwd_totals_kernel<<<(unsigned)(N * pl.nseg), fk::NTHR, ts.total, s>>>(mK, mV, a);
    ks.stop();
  }
  RACE_TRY(check_launch("fast fwd_totals"));
  gen::Dims p = make_dims(N, T, S, fk::HD, eps);
  p.G = pl.nseg;
  KernelScope ks(RACE_KT_SCAN, s);
  const int rc = launch_scan(at<float>(ws, pl.rec_off), A0, B0, Af, Bf, p, 0, s);
  ks.stop();
  return rc;
}

// finish: the readout half of a sequence shard's split forward.  The workspace
// holds the segment prefixes race_fwd_local left (unseeded); A0/B0, the
// earlier shards' state, are added to each as the readout loads it.
int fast_forward(const void *Q, const void *K, const void *V, const float *planes_T, void *out, const float *A0,
                 const float *B0, float *Af, float *Bf, int64_t N, int64_t T, int64_t L, float eps, float scale,
                 void *ws, cudaStream_t s, void *saved = nullptr, bool finish = false, int64_t H = 1) {
  NvtxRange range(finish ? "race forward (finish)" : "race forward");
  fk::FwdArgs a;
  CUtensorMap mQ, mK, mV;
  if (finish) {
    fh::Plan pl;
    RACE_TRY(fast_prepare(K, V, planes_T, N, T, L, eps, scale, ws, a, mK, mV, pl, 0, H));
    a.seedA = A0;
    a.seedB = B0;
  } else {
    RACE_TRY(fast_totals_and_scan(K, V, planes_T, A0, B0, Af, Bf, N, T, L, eps, scale, ws, s, a, mK, mV, 0, H));
  }
  if (!fh::make_act_map(&mQ, Q, N, T, H))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled(Q) failed: CUresult %d", fh::last_encode_status());
  a.out = static_cast<__nv_bfloat16 *>(out);
  if (saved != nullptr) {
    const fh::SavedPlan sp = fh::saved_plan(N, T, 16 * L);
    a.chunkA = at<float>(saved, sp.chunkA);
    a.chunkB = at<__nv_bfloat16>(saved, sp.chunkB);
  }
  const fk::FwdSmem fs = fk::fwd_smem_plan(a.ngroups, a.LP);
  RACE_TRY(set_smem(fk::fwd_readout_kernel, fs.total));
  KernelScope ks(RACE_KT_FWD_READOUT, s);
  fk::fwd_readout_kernel<<<(unsigned)(N * a.nseg), fk::NTHR, fs.total, s>>>(mQ, mK, mV, a);
  ks.stop();
  return check_launch("fast fwd_readout");
}

// Backward of the tcgen05 path.  FULL: everything in one call.  LOCAL (first half of
// the split backward of a sequence shard): the walk and the suffix scan over this
// shard's segments; dA0/dB0 receive the shard's gradient totals and the workspace
// keeps the rest.  FINISH: the fix-up with the later shards' suffix (seedA/seedB)
// added to every segment's, on the workspace LOCAL left.
enum BwdMode { BWD_FULL = 0, BWD_LOCAL, BWD_FINISH };

int fast_backward(const void *Q, const void *K, const void *V, const void *dO, const float *planes_T, void *dQ,
                  void *dK, void *dV, const float *A0, const float *B0, const float *gA, const float *gB, float *dA0,
                  float *dB0, int64_t N, int64_t T, int64_t L, float eps, float scale, void *ws, cudaStream_t s,
                  BwdMode mode, const void *saved = nullptr, int64_t H = 1) {
  NvtxRange range(mode == BWD_FULL ? "race backward" : mode == BWD_LOCAL ? "race backward (local)"
                                                                          : "race backward (finish)");
  const int64_t S = 16 * L;
  const fh::BwdPlan bp = fh::bwd_plan(N, T, S, fh::sm_count(), mode != BWD_FULL);
  fk::FwdArgs fa;
  CUtensorMap mQ, mK, mV, mO, mB, mP;
  // chunk-start states: saved by the forward, or rebuilt below
  const fh::SavedPlan sp = fh::saved_plan(N, T, S);
  float *chunkA = saved ? at<float>(const_cast<void *>(saved), sp.chunkA) : at<float>(ws, bp.chunkA);
  __nv_bfloat16 *chunkB =
      saved ? at<__nv_bfloat16>(const_cast<void *>(saved), sp.chunkB) : at<__nv_bfloat16>(ws, bp.chunkB);
  const bool rebuild = saved == nullptr && mode != BWD_FINISH;
  if (rebuild) {
    // forward segment prefixes (exclusive, seeded with the carried-in state)
    RACE_TRY(fast_totals_and_scan(K, V, planes_T, A0, B0, nullptr, nullptr, N, T, L, eps, scale, ws, s, fa, mK, mV,
                                  bp.fwd_rec, H));
  } else {
    if (!fh::bind_current_context()) return fail(RACE_ERR_CUDA, "no current CUDA device/context on this thread");
    if (!fh::make_act_map(&mK, K, N, T, H) || !fh::make_act_map(&mV, V, N, T, H))
      return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled(K/V) failed: CUresult %d", fh::last_encode_status());
    if (mode != BWD_FINISH) {
      cudaError_t e = cudaMemsetAsync(at<int>(ws, 0), 0, sizeof(int), s);
      if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
  }
  if (!fh::make_map(&mP, at<void>(ws, bp.dprojQ), N, T) ||
      (mode != BWD_FINISH && (!fh::make_act_map(&mQ, Q, N, T, H) || !fh::make_act_map(&mO, dO, N, T, H) ||
                              !fh::make_rows_map(&mB, chunkB, N * (int64_t)bp.p.nchunks * S))))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled failed in the backward: CUresult %d",
                fh::last_encode_status());
  fk::BwdArgs b;
  b.N = (int)N;
  b.T = (int)T;
  b.H = (int)H;
  b.L = (int)L;
  b.LP = (int)(4 * L);
  b.S = (int)S;
  b.ngroups = (int)(S / fk::GW);
  b.nseg = bp.p.nseg;
  b.seg_chunks = bp.p.seg_chunks;
  b.nchunks = bp.p.nchunks;
  b.eps = eps;
  b.scale = scale;
  b.poly = 2.f * std::fabs(scale) <= 0.5f ? 1 : 0;
  b.batch_rcp = eps >= 1e-8f ? 1 : 0;
  b.planes = planes_T;
  b.fwd_state = at<float>(ws, bp.fwd_rec);
  b.tot = at<float>(ws, bp.bwd_rec);
  b.suf_state = nullptr;
  b.chunkA = chunkA;
  b.chunkB = chunkB;
  b.dQ = nullptr;
  b.dK = static_cast<__nv_bfloat16 *>(dK);
  b.dV = mode == BWD_FULL ? static_cast<__nv_bfloat16 *>(dV) : at<__nv_bfloat16>(ws, bp.dVloc);
  b.dprojQ = at<__nv_bfloat16>(ws, bp.dprojQ);
  b.dprojK = at<float>(ws, bp.dprojK);
  b.seedA = b.seedB = nullptr;
  b.dVloc = nullptr;
  b.err = at<int>(ws, 0);
  b.wait_limit = wait_limit();
  const unsigned grid = (unsigned)(N * bp.p.nseg);
  gen::Dims p = make_dims(N, T, S, fk::HD, eps);
  p.G = bp.p.nseg;
  if (mode != BWD_FINISH) {
    // 1. chunk-start forward states (A + eps, bf16 B) from the segment prefixes, unless saved
    if (rebuild) {
      fa.chunkA = b.chunkA;
      fa.chunkB = b.chunkB;
      fa.seg_state = b.fwd_state;
      {
        const fk::TotSmem ts = fk::tot_smem_plan(fa.ngroups, fa.LP);
        KernelScope ks(RACE_KT_FWD_TOTALS, s);
        fk::fwd_totals_kernel<<<grid, fk::NTHR, ts.total, s>>>(mK, mV, fa);
        ks.stop();
      }
      RACE_TRY(check_launch("fast chunk states"));
    }
    // 2. segment-local reverse walk: dV and d proj_K without the later segments' suffix,
    //    d proj_Q, the segments' local totals
    const fk::BwdSmem rs = fk::bwd_smem_plan(b.LP, b.S);
    RACE_TRY(set_smem(fk::bwd_rev_kernel<fk::REV_TPW>, rs.total));
    {
      KernelScope ks(RACE_KT_BWD_REV, s);
      fk::bwd_rev_kernel<fk::REV_TPW><<<grid, fk::rev_block_threads<fk::REV_TPW>(), rs.total, s>>>(mQ, mK, mV, mO, mB, b);
      ks.stop();
    }
    RACE_TRY(check_launch("fast bwd_rev"));
    // 3. suffix over segments (seeded with the carried-in gradient state); its totals are dA0, dB0
    {
      KernelScope ks(RACE_KT_SCAN, s);
      const int rc = launch_scan(at<float>(ws, bp.bwd_rec), mode == BWD_FULL ? gA : nullptr,
                                 mode == BWD_FULL ? gB : nullptr, dA0, dB0, p, 1, s);
      ks.stop();
      RACE_TRY(rc);
    }
    if (mode == BWD_LOCAL) return RACE_OK;
  }
  // 4. fix-up: the suffix's linear share of dV and d proj_K; dK, dQ from d proj_K, d proj_Q
  b.suf_state = at<float>(ws, bp.bwd_rec);
  b.dQ = static_cast<__nv_bfloat16 *>(dQ);
  b.dV = static_cast<__nv_bfloat16 *>(dV);
  if (mode == BWD_FINISH) {
    b.seedA = gA;
    b.seedB = gB;
    b.dVloc = at<__nv_bfloat16>(ws, bp.dVloc);
  }
  // tile maps of the walk's dV (read) and of the outputs (written by TMA tile stores)
  CUtensorMap mVL, mOK, mOV, mOQ;
  if (!fh::make_act_map(&mVL, b.dVloc ? (void *)b.dVloc : dV, N, T, H) || !fh::make_act_map(&mOK, dK, N, T, H) ||
      !fh::make_act_map(&mOV, dV, N, T, H) || !fh::make_act_map(&mOQ, dQ, N, T, H))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the fix-up's dV/dK/dQ: CUresult %d",
                fh::last_encode_status());
  const fk::FixSmem xs = fk::fix_smem_plan(b.LP, b.S);
  RACE_TRY(set_smem(fk::bwd_fix_kernel, xs.total));
  KernelScope ks(RACE_KT_BWD_FIX, s);
  fk::bwd_fix_kernel<<<grid, fk::NTHR, xs.total, s>>>(mK, mV, mP, mVL, mOK, mOV, mOQ, b);
  ks.stop();
  return check_launch("fast bwd_fix");
}

// End of a tcgen05-path call: with race_set_status_check(1), wait for the stream
// and turn a non-zero status word (a bounded device-side wait gave up) into
// RACE_ERR_TIMEOUT; otherwise the word stays at the head of the workspace for
// race_read_status.
int fast_status(const void *ws, cudaStream_t s, const char *what) {
  if (!g_status_check.load(std::memory_order_relaxed)) return ok();
  int st = 0;
  cudaError_t e = cudaMemcpyAsync(&st, ws, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "%s: status read: %s", what, cudaGetErrorString(e));
  if (st != 0)
    return fail(RACE_ERR_TIMEOUT, "%s: a bounded device-side wait gave up (status %d); outputs are invalid", what,
                st);
  return ok();
}

// Non-causal RACE: the per-token tile kernel (noncausal.cuh) in one of its modes.  X, Y: the
// input activations (Y unused by ACE_OUT); O1, O2: the outputs (O2 only for ACE_KV); totA /
// totB: the (K, V) totals A, b; totG: the (Q, dO) totals dE (ACE_KV).
int ace_tiles(int mode, const void *X, const void *Y, void *O1, void *O2, const float *planes_T, const float *totA,
              const float *totB, const float *totG, int64_t N, int64_t T, int64_t L, float eps, float scale, void *ws,
              cudaStream_t s) {
  const int64_t S = 16 * L;
  if (!fh::bind_current_context()) return fail(RACE_ERR_CUDA, "no current CUDA device/context on this thread");
  const fh::Plan pl = fh::plan(N, T, S, fh::sm_count());
  fk::AceArgs a;
  a.N = (int)N;
  a.T = (int)T;
  a.L = (int)L;
  a.LP = (int)(4 * L);
  a.S = (int)S;
  a.H = 1;
  a.nseg = pl.nseg;
  a.seg_chunks = pl.seg_chunks;
  a.nchunks = pl.nchunks;
  a.eps = eps;
  a.scale = scale;
  a.poly = 2.f * std::fabs(scale) <= 0.5f ? 1 : 0;
  a.planes = planes_T;
  a.totA = totA;
  a.totB = totB;
  a.totG = totG;
  a.err = at<int>(ws, 0);
  a.wait_limit = wait_limit();
  CUtensorMap mX, mY, mO1, mO2;
  if (!fh::make_act_map(&mX, X, N, T, 1) || !fh::make_act_map(&mO1, O1, N, T, 1) ||
      (Y && !fh::make_act_map(&mY, Y, N, T, 1)) || (O2 && !fh::make_act_map(&mO2, O2, N, T, 1)))
    return fail(RACE_ERR_CUDA, "cuTensorMapEncodeTiled failed in the non-causal kernel: CUresult %d",
                fh::last_encode_status());
  if (!Y) mY = mX;    // unused by the kernel
  if (!O2) mO2 = mO1;  // unused by the kernel
  const fk::AceSmem sp = fk::ace_smem_plan(a.LP, a.S);
  const unsigned grid = (unsigned)(N * pl.nseg);
  KernelScope ks(RACE_KT_ACE_TILE, s);
  switch (mode) {
    case fk::ACE_OUT:
      RACE_TRY(set_smem(fk::ace_tile_kernel<fk::ACE_OUT>, sp.total));
      fk::ace_tile_kernel<fk::ACE_OUT><<<grid, fk::NTHR, sp.total, s>>>(mX, mY, mO1, mO2, a);
      break;
    case fk::ACE_KV:
      RACE_TRY(set_smem(fk::ace_tile_kernel<fk::ACE_KV>, sp.total));
      fk::ace_tile_kernel<fk::ACE_KV><<<grid, fk::NTHR, sp.total, s>>>(mX, mY, mO1, mO2, a);
      break;
    default:
      RACE_TRY(set_smem(fk::ace_tile_kernel<fk::ACE_Q>, sp.total));
      fk::ace_tile_kernel<fk::ACE_Q><<<grid, fk::NTHR, sp.total, s>>>(mX, mY, mO1, mO2, a);
      break;
  }
  ks.stop();
  return check_launch("ace_tile_kernel");
}

// Workspace of the non-causal backward: the totals kernel's status word and segment records,
// then the (Q, dO) totals dE [N, S, 64] fp32.
size_t ace_bwd_dE_offset(int64_t N, int64_t T, int64_t S) { return fh::fwd_workspace_bytes(N, T, S); }
size_t ace_bwd_workspace_bytes(int64_t N, int64_t T, int64_t S) {
  return ace_bwd_dE_offset(N, T, S) + align_up(sizeof(float) * (size_t)N * S * fk::HD, 256);
}

int check_fast_ptrs(std::initializer_list<const void *> ptrs) {
  for (const void *p : ptrs)
    if (p && !fh::aligned16(p)) return fail(RACE_ERR_ALIGN, "bf16 activations must be 16-byte aligned");
  return RACE_OK;
}


}  // namespace

// Shared with the other translation units of the library (csrc/internal.h).
namespace race {
int report_error(int code, const char *msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}
void clear_error() { g_err[0] = 0; }
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace race

// ============================================================================
extern "C" {

int race_abi_version(void) { return 1; }

const char *race_status_string(int status) {
  switch (status) {
    case RACE_OK: return "ok";
    case RACE_ERR_ARG: return "invalid argument";
    case RACE_ERR_SHAPE: return "invalid or unsupported shape";
    case RACE_ERR_DTYPE: return "unsupported dtype";
    case RACE_ERR_ALIGN: return "misaligned pointer";
    case RACE_ERR_WORKSPACE: return "workspace missing or too small";
    case RACE_ERR_CUDA: return "CUDA error";
    case RACE_ERR_TIMEOUT: return "device-side wait timed out";
    case RACE_ERR_UNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

const char *race_last_error(void) { return g_err; }

unsigned long long race_launch_counter(void) { return g_launches.load(std::memory_order_relaxed); }

int race_kernel_timing(int enable) {
  KernelTimer &t = ktimer();
  std::lock_guard<std::mutex> g(t.mu);
  for (int k = 0; k < RACE_KT_COUNT; ++k) {
    for (auto &ev : t.pending[k]) {
      cudaEventDestroy(ev.first);
      cudaEventDestroy(ev.second);
    }
    t.pending[k].clear();
    t.ms[k] = 0;
    t.launches[k] = 0;
  }
  t.on = enable != 0;
  return ok();
}

int race_kernel_time(int kernel, double *total_ms, long long *launches) {
  RACE_NONNULL(total_ms);
  RACE_NONNULL(launches);
  if (kernel < 0 || kernel >= RACE_KT_COUNT) return fail(RACE_ERR_ARG, "kernel id %d out of range", kernel);
  KernelTimer &t = ktimer();
  std::lock_guard<std::mutex> g(t.mu);
  for (auto &ev : t.pending[kernel]) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(ev.second);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev.first, ev.second);
    cudaEventDestroy(ev.first);
    cudaEventDestroy(ev.second);
    if (e != cudaSuccess) {
      t.pending[kernel].clear();
      return fail(RACE_ERR_CUDA, "kernel timing events: %s", cudaGetErrorString(e));
    }
    t.ms[kernel] += ms;
    t.launches[kernel] += 1;
  }
  t.pending[kernel].clear();
  *total_ms = t.ms[kernel];
  *launches = t.launches[kernel];
  return ok();
}

int race_set_wait_limit(unsigned int polls) {
  g_wait_limit.store(polls, std::memory_order_relaxed);
  return ok();
}

int race_set_status_check(int synchronous) {
  g_status_check.store(synchronous ? 1 : 0, std::memory_order_relaxed);
  return ok();
}

int race_read_status(const void *workspace, void *stream, int *status) {
  RACE_NONNULL(workspace);
  RACE_NONNULL(status);
  cudaStream_t s = as_stream(stream);
  int st = 0;
  cudaError_t e = cudaMemcpyAsync(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(RACE_ERR_CUDA, "race_read_status: %s", cudaGetErrorString(e));
  *status = st;
  return ok();
}

int race_test_withhold_first_load(int on) {
  g_withhold_first_load.store(on ? 1 : 0, std::memory_order_relaxed);
  return ok();
}

int race_plan_segments(int64_t N, int64_t T, int64_t S, int sms, int *nseg, int *seg_chunks, int *max_nseg) {
  RACE_NONNULL(nseg);
  RACE_NONNULL(seg_chunks);
  RACE_NONNULL(max_nseg);
  if (N < 1 || T < 1 || S < 1) return fail(RACE_ERR_SHAPE, "N, T, S must be >= 1");
  if (sms < 1 || sms > 65536) return fail(RACE_ERR_ARG, "sms=%d not in [1, 65536]", sms);
  const fh::Plan p = fh::plan(N, T, S, sms);
  *nseg = p.nseg;
  *seg_chunks = p.seg_chunks;
  *max_nseg = fh::plan(N, T, S, 256).nseg;
  return ok();
}

int race_workspace_bytes(int op, int64_t N, int64_t T, int64_t S, int64_t D, int64_t L, int64_t P, int dtype,
                         int64_t chunk, size_t *bytes) {
  (void)chunk;
  RACE_NONNULL(bytes);
  *bytes = 0;
  if (op == RACE_OP_ACE_FWD || op == RACE_OP_ACE_BWD) {
    RACE_TRY(check_dtype(dtype));
    RACE_TRY(check_lp(L, P, &S));
    RACE_TRY(check_nts(N, T, S, D));
    if (!fh::eligible(dtype, D, L, P))
      return fail(RACE_ERR_UNSUPPORTED, "non-causal kernels: bf16, D=64, P=4, L in {8,16} only");
    *bytes = op == RACE_OP_ACE_FWD ? fh::fwd_workspace_bytes(N, T, S) : ace_bwd_workspace_bytes(N, T, S);
    return ok();
  }
  if (op == RACE_OP_FWD_QKV || op == RACE_OP_BWD_QKV || op == RACE_OP_STATE || op == RACE_OP_BWD_SPLIT ||
      op == RACE_OP_FWD_SPLIT) {
    RACE_TRY(check_dtype(dtype));
    RACE_TRY(check_lp(L, P, &S));
  } else if (op != RACE_OP_FWD_PROBS && op != RACE_OP_BWD_PROBS) {
    return fail(RACE_ERR_ARG, "unknown op %d", op);
  }
  RACE_TRY(check_nts(N, T, S, D));
  if ((op == RACE_OP_FWD_QKV || op == RACE_OP_STATE) && fh::eligible(dtype, D, L, P))
    *bytes = fh::fwd_workspace_bytes(N, T, S);
  else if (op == RACE_OP_BWD_QKV && fh::eligible(dtype, D, L, P))
    *bytes = fh::bwd_workspace_bytes(N, T, S);
  else if (op == RACE_OP_BWD_SPLIT && fh::eligible(dtype, D, L, P))
    *bytes = fh::bwd_workspace_bytes(N, T, S, true);
  else if (op == RACE_OP_BWD_SPLIT)
    *bytes = std::max(generic_layout(RACE_OP_BWD_TOTALS, N, T, S, D).total,
                      generic_layout(RACE_OP_BWD_QKV, N, T, S, D).total);
  else if (op == RACE_OP_FWD_SPLIT && fh::eligible(dtype, D, L, P))
    *bytes = fh::fwd_workspace_bytes(N, T, S);
  else if (op == RACE_OP_FWD_SPLIT)
    *bytes = std::max(generic_layout(RACE_OP_STATE, N, T, S, D).total,
                      generic_layout(RACE_OP_FWD_QKV, N, T, S, D).total);
  else
    *bytes = generic_layout(op, N, T, S, D).total;
  return ok();
}

int race_fwd_probs(const float *probsK, const float *probsQ, const float *V2, float *out, float *A_final,
                   float *B_final, int64_t N, int64_t T, int64_t S, int64_t D, float eps, int64_t chunk,
                   void *workspace, size_t workspace_bytes, void *stream) {
  (void)chunk;
  RACE_NONNULL(probsK);
  RACE_NONNULL(probsQ);
  RACE_NONNULL(V2);
  RACE_NONNULL(out);
  RACE_TRY(check_nts(N, T, S, D));
  const Layout w = generic_layout(RACE_OP_FWD_PROBS, N, T, S, D);
  RACE_TRY(check_ws(workspace, workspace_bytes, w.total));
  cudaStream_t s = as_stream(stream);
  float *St = at<float>(workspace, w.st);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t po = (size_t)n0 * T * S, xo = (size_t)n0 * T * D, so = (size_t)n0 * S, bo = (size_t)n0 * S * D;
    const gen::Dims p = make_dims(nn, T, S, D, eps);
    RACE_TRY(launch_totals<float>(probsK + po, V2 + xo, St, p, s));
    RACE_TRY(launch_scan(St, nullptr, nullptr, off(A_final, so), off(B_final, bo), p, 0, s));
    RACE_TRY(launch_readout<float, float>(probsK + po, probsQ + po, V2 + xo, St, out + xo, p, s));
  }
  return ok();
}

int race_bwd_probs(const float *probsK, const float *probsQ, const float *V2, const float *grad_out,
                   float *grad_probsK, float *grad_probsQ, float *grad_V2, int64_t N, int64_t T, int64_t S, int64_t D,
                   float eps, int64_t chunk, void *workspace, size_t workspace_bytes, void *stream) {
  (void)chunk;
  RACE_NONNULL(probsK);
  RACE_NONNULL(probsQ);
  RACE_NONNULL(V2);
  RACE_NONNULL(grad_out);
  RACE_NONNULL(grad_probsK);
  RACE_NONNULL(grad_probsQ);
  RACE_NONNULL(grad_V2);
  RACE_TRY(check_nts(N, T, S, D));
  const Layout w = generic_layout(RACE_OP_BWD_PROBS, N, T, S, D);
  RACE_TRY(check_ws(workspace, workspace_bytes, w.total));
  cudaStream_t s = as_stream(stream);
  float *St = at<float>(workspace, w.st), *St2 = at<float>(workspace, w.st2);
  for (int64_t n0 = 0; n0 < N; n0 += w.grp) {
    const int64_t nn = std::min(w.grp, N - n0);
    const size_t po = (size_t)n0 * T * S, xo = (size_t)n0 * T * D;
    const gen::Dims p = make_dims(nn, T, S, D, eps);
    RACE_TRY(launch_totals<float>(probsK + po, V2 + xo, St, p, s));
    RACE_TRY(launch_scan(St, nullptr, nullptr, nullptr, nullptr, p, 0, s));
    RACE_TRY(launch_bwd_totals<float>(probsK + po, probsQ + po, V2 + xo, grad_out + xo, St, St2, grad_probsQ + po,
                                      p, s));
    RACE_TRY(launch_scan(St2, nullptr, nullptr, nullptr, nullptr, p, 1, s));
    RACE_TRY(launch_bwd_readout<float, float>(probsK + po, probsQ + po, V2 + xo, grad_out + xo, St, St2,
                                              grad_probsK + po, grad_V2 + xo, p, s));
  }
  return ok();
}

int race_soft_hash(const void *X, int dtype, const float *planes_T, float *probs, int64_t N, int64_t T, int64_t D,
                   int64_t L, int64_t P, float logit_scale, void *stream) {
  RACE_NONNULL(X);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(probs);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (dtype == RACE_F32)
    RACE_TRY(launch_hash<float>((const float *)X, planes_T, probs, N * T, D, L, P, logit_scale, s));
  else
    RACE_TRY(launch_hash<__nv_bfloat16>((const __nv_bfloat16 *)X, planes_T, probs, N * T, D, L, P, logit_scale, s));
  return ok();
}

int race_soft_hash_bwd(const void *X, int dtype, const float *planes_T, const float *dprobs, void *dX, int64_t N,
                       int64_t T, int64_t D, int64_t L, int64_t P, float logit_scale, void *stream) {
  RACE_NONNULL(X);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(dprobs);
  RACE_NONNULL(dX);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (dtype == RACE_F32)
    RACE_TRY(launch_hash_bwd<float>((const float *)X, planes_T, dprobs, (float *)dX, N * T, D, L, P, logit_scale, s));
  else
    RACE_TRY(launch_hash_bwd<__nv_bfloat16>((const __nv_bfloat16 *)X, planes_T, dprobs, (__nv_bfloat16 *)dX, N * T,
                                            D, L, P, logit_scale, s));
  return ok();
}

static int fwd_qkv_impl(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out,
                        const float *A0, const float *B0, float *A_final, float *B_final, void *saved,
                        size_t saved_bytes, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                        float logit_scale, void *workspace, size_t workspace_bytes, void *stream, int64_t H = 1) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(out);
  if (H > 1 && !fh::eligible(dtype, D, L, P))
    return fail(RACE_ERR_UNSUPPORTED, "the [B, T, H, D] layout needs the tcgen05 path (bf16, D=64, P=4, L in {8,16})");
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::fwd_workspace_bytes(N, T, S)));
    RACE_TRY(check_fast_ptrs({Q, K, V, out}));
    if (saved != nullptr) {
      if (saved_bytes < fh::saved_plan(N, T, S).total)
        return fail(RACE_ERR_WORKSPACE, "saved-state buffer too small: %zu < %zu bytes", saved_bytes,
                    fh::saved_plan(N, T, S).total);
      if (!fh::aligned16(saved)) return fail(RACE_ERR_ALIGN, "saved-state buffer must be 16-byte aligned");
    }
    RACE_TRY(fast_forward(Q, K, V, planes_T, out, A0, B0, A_final, B_final, N, T, L, eps, logit_scale, workspace, s,
                          saved, false, H));
    return fast_status(workspace, s, "forward");
  }
  RACE_TRY(check_ws(workspace, workspace_bytes, generic_layout(RACE_OP_FWD_QKV, N, T, S, D).total));
  if (dtype == RACE_F32)
    RACE_TRY(fwd_qkv_generic<float>((const float *)Q, (const float *)K, (const float *)V, planes_T, (float *)out, A0,
                                    B0, A_final, B_final, N, T, D, L, P, eps, logit_scale, workspace, s));
  else
    RACE_TRY(fwd_qkv_generic<__nv_bfloat16>((const __nv_bfloat16 *)Q, (const __nv_bfloat16 *)K,
                                            (const __nv_bfloat16 *)V, planes_T, (__nv_bfloat16 *)out, A0, B0,
                                            A_final, B_final, N, T, D, L, P, eps, logit_scale, workspace, s));
  return ok();
}

static int bwd_qkv_impl(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                        const float *planes_T, const void *saved, size_t saved_bytes, void *dQ, void *dK, void *dV,
                        const float *A0, const float *B0, const float *gA_in, const float *gB_in, float *dA0,
                        float *dB0, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                        float logit_scale, void *workspace, size_t workspace_bytes, void *stream, int64_t H = 1) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(dO);
  if (H > 1 && !fh::eligible(dtype, D, L, P))
    return fail(RACE_ERR_UNSUPPORTED, "the [B, T, H, D] layout needs the tcgen05 path (bf16, D=64, P=4, L in {8,16})");
  RACE_NONNULL(planes_T);
  RACE_NONNULL(dQ);
  RACE_NONNULL(dK);
  RACE_NONNULL(dV);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::bwd_workspace_bytes(N, T, S)));
    RACE_TRY(check_fast_ptrs({Q, K, V, dO, dQ, dK, dV}));
    if (saved != nullptr) {
      if (saved_bytes < fh::saved_plan(N, T, S).total)
        return fail(RACE_ERR_WORKSPACE, "saved-state buffer too small: %zu < %zu bytes", saved_bytes,
                    fh::saved_plan(N, T, S).total);
      if (!fh::aligned16(saved)) return fail(RACE_ERR_ALIGN, "saved-state buffer must be 16-byte aligned");
    }
    RACE_TRY(fast_backward(Q, K, V, dO, planes_T, dQ, dK, dV, A0, B0, gA_in, gB_in, dA0, dB0, N, T, L, eps,
                           logit_scale, workspace, s, BWD_FULL, saved, H));
    return fast_status(workspace, s, "backward");
  }
  RACE_TRY(check_ws(workspace, workspace_bytes, generic_layout(RACE_OP_BWD_QKV, N, T, S, D).total));
  if (dtype == RACE_F32)
    RACE_TRY(bwd_qkv_generic<float>((const float *)Q, (const float *)K, (const float *)V, (const float *)dO, planes_T,
                                    (float *)dQ, (float *)dK, (float *)dV, A0, B0, gA_in, gB_in, dA0, dB0, N, T, D,
                                    L, P, eps, logit_scale, workspace, s));
  else
    RACE_TRY(bwd_qkv_generic<__nv_bfloat16>(
        (const __nv_bfloat16 *)Q, (const __nv_bfloat16 *)K, (const __nv_bfloat16 *)V, (const __nv_bfloat16 *)dO,
        planes_T, (__nv_bfloat16 *)dQ, (__nv_bfloat16 *)dK, (__nv_bfloat16 *)dV, A0, B0, gA_in, gB_in, dA0, dB0, N,
        T, D, L, P, eps, logit_scale, workspace, s));
  return ok();
}

int race_fwd_qkv(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out,
                 const float *A0, const float *B0, float *A_final, float *B_final, int64_t N, int64_t T, int64_t D,
                 int64_t L, int64_t P, float eps, float logit_scale, void *workspace, size_t workspace_bytes,
                 void *stream) {
  return fwd_qkv_impl(Q, K, V, dtype, planes_T, out, A0, B0, A_final, B_final, nullptr, 0, N, T, D, L, P, eps,
                      logit_scale, workspace, workspace_bytes, stream);
}

int race_bwd_qkv(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                 void *dQ, void *dK, void *dV, const float *A0, const float *B0, const float *gA_in,
                 const float *gB_in, float *dA0, float *dB0, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                 float eps, float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  return bwd_qkv_impl(Q, K, V, dO, dtype, planes_T, nullptr, 0, dQ, dK, dV, A0, B0, gA_in, gB_in, dA0, dB0, N, T, D,
                      L, P, eps, logit_scale, workspace, workspace_bytes, stream);
}

int race_fwd_bthd(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out,
                  void *saved, size_t saved_bytes, int64_t B, int64_t T, int64_t H, int64_t D, int64_t L, int64_t P,
                  float eps, float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  if (B < 1 || H < 1) return fail(RACE_ERR_SHAPE, "B and H must be >= 1");
  return fwd_qkv_impl(Q, K, V, dtype, planes_T, out, nullptr, nullptr, nullptr, nullptr, saved, saved_bytes, B * H, T,
                      D, L, P, eps, logit_scale, workspace, workspace_bytes, stream, H);
}

int race_bwd_bthd(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                  const void *saved, size_t saved_bytes, void *dQ, void *dK, void *dV, int64_t B, int64_t T,
                  int64_t H, int64_t D, int64_t L, int64_t P, float eps, float logit_scale, void *workspace,
                  size_t workspace_bytes, void *stream) {
  if (B < 1 || H < 1) return fail(RACE_ERR_SHAPE, "B and H must be >= 1");
  return bwd_qkv_impl(Q, K, V, dO, dtype, planes_T, saved, saved_bytes, dQ, dK, dV, nullptr, nullptr, nullptr,
                      nullptr, nullptr, nullptr, B * H, T, D, L, P, eps, logit_scale, workspace, workspace_bytes,
                      stream, H);
}

int race_saved_bytes(int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, int dtype, size_t *bytes) {
  RACE_NONNULL(bytes);
  *bytes = 0;
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  if (fh::eligible(dtype, D, L, P)) *bytes = fh::saved_plan(N, T, S).total;
  return ok();
}

int race_fwd_qkv_save(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out,
                      const float *A0, const float *B0, float *A_final, float *B_final, void *saved,
                      size_t saved_bytes, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                      float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  return fwd_qkv_impl(Q, K, V, dtype, planes_T, out, A0, B0, A_final, B_final, saved_bytes ? saved : nullptr,
                      saved_bytes, N, T, D, L, P, eps, logit_scale, workspace, workspace_bytes, stream);
}

int race_bwd_qkv_saved(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                       const void *saved, size_t saved_bytes, void *dQ, void *dK, void *dV, const float *A0,
                       const float *B0, const float *gA_in, const float *gB_in, float *dA0, float *dB0, int64_t N,
                       int64_t T, int64_t D, int64_t L, int64_t P, float eps, float logit_scale, void *workspace,
                       size_t workspace_bytes, void *stream) {
  return bwd_qkv_impl(Q, K, V, dO, dtype, planes_T, saved_bytes ? saved : nullptr, saved_bytes, dQ, dK, dV, A0, B0,
                      gA_in, gB_in, dA0, dB0, N, T, D, L, P, eps, logit_scale, workspace, workspace_bytes, stream);
}

int race_state_from_prefill(const void *K, const void *V, int dtype, const float *planes_T, const float *A0,
                            const float *B0, float *A_out, float *B_out, int64_t N, int64_t T, int64_t D, int64_t L,
                            int64_t P, float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(A_out);
  RACE_NONNULL(B_out);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::fwd_workspace_bytes(N, T, S)));
    RACE_TRY(check_fast_ptrs({K, V}));
    fk::FwdArgs a;
    CUtensorMap mK, mV;
    RACE_TRY(fast_totals_and_scan(K, V, planes_T, A0, B0, A_out, B_out, N, T, L, 0.f, logit_scale, workspace, s, a,
                                  mK, mV));
    return fast_status(workspace, s, "state from prefill");
  }
  RACE_TRY(check_ws(workspace, workspace_bytes, generic_layout(RACE_OP_STATE, N, T, S, D).total));
  if (dtype == RACE_F32)
    RACE_TRY(state_generic<float>((const float *)K, (const float *)V, planes_T, A0, B0, A_out, B_out, N, T, D, L, P,
                                  logit_scale, workspace, s));
  else
    RACE_TRY(state_generic<__nv_bfloat16>((const __nv_bfloat16 *)K, (const __nv_bfloat16 *)V, planes_T, A0, B0,
                                          A_out, B_out, N, T, D, L, P, logit_scale, workspace, s));
  return ok();
}

int race_fwd_local(const void *K, const void *V, int dtype, const float *planes_T, float *A_tot, float *B_tot,
                   int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float logit_scale, void *workspace,
                   size_t workspace_bytes, void *stream) {
  // the tcgen05 path keeps its (unseeded) segment prefixes in the workspace for
  // race_fwd_finish; the generic path recomputes everything there
  return race_state_from_prefill(K, V, dtype, planes_T, nullptr, nullptr, A_tot, B_tot, N, T, D, L, P, logit_scale,
                                 workspace, workspace_bytes, stream);
}

int race_fwd_finish(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out,
                    void *saved, size_t saved_bytes, const float *A0, const float *B0, int64_t N, int64_t T,
                    int64_t D, int64_t L, int64_t P, float eps, float logit_scale, void *workspace,
                    size_t workspace_bytes, void *stream) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(out);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::fwd_workspace_bytes(N, T, S)));
    RACE_TRY(check_fast_ptrs({Q, K, V, out}));
    if (saved_bytes && saved_bytes < fh::saved_plan(N, T, S).total)
      return fail(RACE_ERR_WORKSPACE, "saved-state buffer too small");
    RACE_TRY(fast_forward(Q, K, V, planes_T, out, A0, B0, nullptr, nullptr, N, T, L, eps, logit_scale, workspace,
                          as_stream(stream), saved_bytes ? saved : nullptr, true));
    return fast_status(workspace, as_stream(stream), "forward finish");
  }
  if (saved_bytes) return fail(RACE_ERR_UNSUPPORTED, "saved chunk states need the tcgen05 path");
  return race_fwd_qkv(Q, K, V, dtype, planes_T, out, A0, B0, nullptr, nullptr, N, T, D, L, P, eps, logit_scale,
                      workspace, workspace_bytes, stream);
}

int race_bwd_local(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                   const void *saved, size_t saved_bytes, const float *A0, const float *B0, float *gA_tot,
                   float *gB_tot, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                   float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(dO);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(gA_tot);
  RACE_NONNULL(gB_tot);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::bwd_workspace_bytes(N, T, S, true)));
    RACE_TRY(check_fast_ptrs({Q, K, V, dO}));
    if (saved_bytes && saved_bytes < fh::saved_plan(N, T, S).total)
      return fail(RACE_ERR_WORKSPACE, "saved-state buffer too small");
    RACE_TRY(fast_backward(Q, K, V, dO, planes_T, nullptr, nullptr, nullptr, A0, B0, nullptr, nullptr, gA_tot,
                           gB_tot, N, T, L, eps, logit_scale, workspace, s, BWD_LOCAL,
                           saved_bytes ? saved : nullptr));
    return fast_status(workspace, s, "backward local");
  }
  RACE_TRY(check_ws(workspace, workspace_bytes, generic_layout(RACE_OP_BWD_TOTALS, N, T, S, D).total));
  if (dtype == RACE_F32)
    RACE_TRY(bwd_totals_generic<float>((const float *)Q, (const float *)K, (const float *)V, (const float *)dO,
                                       planes_T, A0, B0, gA_tot, gB_tot, N, T, D, L, P, eps, logit_scale, workspace,
                                       s));
  else
    RACE_TRY(bwd_totals_generic<__nv_bfloat16>((const __nv_bfloat16 *)Q, (const __nv_bfloat16 *)K,
                                               (const __nv_bfloat16 *)V, (const __nv_bfloat16 *)dO, planes_T, A0, B0,
                                               gA_tot, gB_tot, N, T, D, L, P, eps, logit_scale, workspace, s));
  return ok();
}

int race_bwd_finish(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                    const void *saved, size_t saved_bytes, const float *A0, const float *B0, const float *gA_in,
                    const float *gB_in, void *dQ, void *dK, void *dV, int64_t N, int64_t T, int64_t D, int64_t L,
                    int64_t P, float eps, float logit_scale, void *workspace, size_t workspace_bytes, void *stream) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(dO);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(dQ);
  RACE_NONNULL(dK);
  RACE_NONNULL(dV);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  cudaStream_t s = as_stream(stream);
  if (fh::eligible(dtype, D, L, P)) {
    RACE_TRY(check_ws(workspace, workspace_bytes, fh::bwd_workspace_bytes(N, T, S, true)));
    RACE_TRY(check_fast_ptrs({K, V, dQ, dK, dV}));
    RACE_TRY(fast_backward(Q, K, V, dO, planes_T, dQ, dK, dV, A0, B0, gA_in, gB_in, nullptr, nullptr, N, T, L, eps,
                           logit_scale, workspace, s, BWD_FINISH, saved_bytes ? saved : nullptr));
    return fast_status(workspace, s, "backward finish");
  }
  // generic path: the whole backward again, with the later shards' suffix
  return race_bwd_qkv(Q, K, V, dO, dtype, planes_T, dQ, dK, dV, A0, B0, gA_in, gB_in, nullptr, nullptr, N, T, D, L,
                      P, eps, logit_scale, workspace, workspace_bytes, stream);
}

int race_ace_fwd(const void *Q, const void *K, const void *V, int dtype, const float *planes_T, void *out, float *A,
                 float *B, int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps, float logit_scale,
                 void *workspace, size_t workspace_bytes, void *stream) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(out);
  RACE_NONNULL(A);
  RACE_NONNULL(B);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  if (!fh::eligible(dtype, D, L, P))
    return fail(RACE_ERR_UNSUPPORTED, "non-causal kernels: bf16, D=64, P=4, L in {8,16} only");
  RACE_TRY(check_ws(workspace, workspace_bytes, fh::fwd_workspace_bytes(N, T, S)));
  RACE_TRY(check_fast_ptrs({Q, K, V, out}));
  cudaStream_t s = as_stream(stream);
  NvtxRange range("race non-causal forward");
  fk::FwdArgs a;
  CUtensorMap mK, mV;
  // A = sum_t pk, b = sum_t pk^T V (the totals kernel and the segment scan's finals)
  RACE_TRY(fast_totals_and_scan(K, V, planes_T, nullptr, nullptr, A, B, N, T, L, 0.f, logit_scale, workspace, s, a,
                                mK, mV));
  RACE_TRY(ace_tiles(fk::ACE_OUT, Q, nullptr, out, nullptr, planes_T, A, B, nullptr, N, T, L, eps, logit_scale,
                     workspace, s));
  return fast_status(workspace, s, "non-causal forward");
}

int race_ace_bwd(const void *Q, const void *K, const void *V, const void *dO, int dtype, const float *planes_T,
                 const float *A, const float *B, void *dQ, void *dK, void *dV, int64_t N, int64_t T, int64_t D,
                 int64_t L, int64_t P, float eps, float logit_scale, void *workspace, size_t workspace_bytes,
                 void *stream) {
  RACE_NONNULL(Q);
  RACE_NONNULL(K);
  RACE_NONNULL(V);
  RACE_NONNULL(dO);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(A);
  RACE_NONNULL(B);
  RACE_NONNULL(dQ);
  RACE_NONNULL(dK);
  RACE_NONNULL(dV);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  RACE_TRY(check_nts(N, T, S, D));
  if (!fh::eligible(dtype, D, L, P))
    return fail(RACE_ERR_UNSUPPORTED, "non-causal kernels: bf16, D=64, P=4, L in {8,16} only");
  RACE_TRY(check_ws(workspace, workspace_bytes, ace_bwd_workspace_bytes(N, T, S)));
  RACE_TRY(check_fast_ptrs({Q, K, V, dO, dQ, dK, dV}));
  cudaStream_t s = as_stream(stream);
  NvtxRange range("race non-causal backward");
  float *dE = at<float>(workspace, ace_bwd_dE_offset(N, T, S));
  fk::FwdArgs a;
  CUtensorMap mQ, mO;
  // dE = sum_t pq^T dO: the same totals kernel over (Q, dO)
  RACE_TRY(fast_totals_and_scan(Q, dO, planes_T, nullptr, nullptr, nullptr, dE, N, T, L, 0.f, logit_scale, workspace,
                                s, a, mQ, mO));
  RACE_TRY(ace_tiles(fk::ACE_KV, K, V, dK, dV, planes_T, A, B, dE, N, T, L, eps, logit_scale, workspace, s));
  RACE_TRY(ace_tiles(fk::ACE_Q, Q, dO, dQ, nullptr, planes_T, A, B, nullptr, N, T, L, eps, logit_scale, workspace,
                     s));
  return fast_status(workspace, s, "non-causal backward");
}

int race_decode_step(const void *q, const void *k, const void *v, int dtype, const float *planes_T, float *A,
                     float *B, void *out, int64_t Nq, int64_t Nkv, int64_t D, int64_t L, int64_t P, float eps,
                     float logit_scale, void *stream) {
  RACE_NONNULL(q);
  RACE_NONNULL(k);
  RACE_NONNULL(v);
  RACE_NONNULL(planes_T);
  RACE_NONNULL(A);
  RACE_NONNULL(B);
  RACE_NONNULL(out);
  RACE_TRY(check_dtype(dtype));
  int64_t S = 0;
  RACE_TRY(check_lp(L, P, &S));
  if (Nkv < 1 || Nkv > (int64_t(1) << 31) - 1) return fail(RACE_ERR_SHAPE, "Nkv=%lld out of range", (long long)Nkv);
  if (Nq < Nkv || Nq % Nkv) return fail(RACE_ERR_SHAPE, "Nq=%lld must be a positive multiple of Nkv=%lld",
                                        (long long)Nq, (long long)Nkv);
  const int64_t group = Nq / Nkv;
  if (group > race::dec::MAX_GROUP)
    return fail(RACE_ERR_UNSUPPORTED, "query group %lld > %d", (long long)group, race::dec::MAX_GROUP);
  if (D < 1 || D > race::dec::NT) return fail(RACE_ERR_SHAPE, "D=%lld out of range [1,%d]", (long long)D, race::dec::NT);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  // both kernels copy the state rows 16 bytes at a time
  if (!al16(A) || !al16(B)) return fail(RACE_ERR_ALIGN, "decode state A and B must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  using bf = __nv_bfloat16;
  constexpr int MAXG = race::dec::MAX_GROUP;
  if (race::dec::d64_eligible((int)D, (int)L, (int)P, (int)group) && al16(q) && al16(k) && al16(v) && al16(out) &&
      al16(planes_T) && al16(A) && al16(B)) {
    // head_dim 64, 4 planes per table: the compile-time-shaped kernel (one CTA per kv stream)
    namespace d6 = race::dec::d64;
    auto launch64 = [&](auto kernel, auto lay, auto *qq, auto *kk, auto *vv, auto *oo) -> int {
      const size_t smb = sizeof(float) * (size_t)decltype(lay)::TOTAL;
      RACE_TRY(set_smem(kernel, smb));
      RACE_TRY(set_carveout(reinterpret_cast<const void *>(kernel)));
      kernel<<<(unsigned)Nkv, d6::NT, smb, s>>>(qq, kk, vv, planes_T, A, B, oo, (int)group, eps, logit_scale);
      return RACE_OK;
    };
    auto by_group = [&](auto tag, auto *qq, auto *kk, auto *vv, auto *oo) -> int {
      using X = std::remove_const_t<std::remove_pointer_t<decltype(qq)>>;
      constexpr int Lc = decltype(tag)::value;
      if (group == 1) return launch64(d6::decode_step_d64<X, Lc, 1>, d6::Layout<Lc, 1>{}, qq, kk, vv, oo);
      if (group == 2) return launch64(d6::decode_step_d64<X, Lc, 2>, d6::Layout<Lc, 2>{}, qq, kk, vv, oo);
      if (group <= 4) return launch64(d6::decode_step_d64<X, Lc, 4>, d6::Layout<Lc, 4>{}, qq, kk, vv, oo);
      return launch64(d6::decode_step_d64<X, Lc, 8>, d6::Layout<Lc, 8>{}, qq, kk, vv, oo);
    };
    auto by_l = [&](auto *qq, auto *kk, auto *vv, auto *oo) -> int {
      return L == 8 ? by_group(std::integral_constant<int, 8>{}, qq, kk, vv, oo)
                    : by_group(std::integral_constant<int, 16>{}, qq, kk, vv, oo);
    };
    if (dtype == RACE_F32)
      RACE_TRY(by_l((const float *)q, (const float *)k, (const float *)v, (float *)out));
    else
      RACE_TRY(by_l((const bf *)q, (const bf *)k, (const bf *)v, (bf *)out));
    RACE_TRY(check_launch("decode_step_d64"));
    return ok();
  }
  const size_t sm = sizeof(float) * race::dec::smem_floats((int)D, (int)S, (int)(L * P), (int)group);
  auto launch = [&](auto kernel, auto *qq, auto *kk, auto *vv, auto *oo) -> int {
    RACE_TRY(set_smem(kernel, sm));
    RACE_TRY(set_carveout(reinterpret_cast<const void *>(kernel)));  // 4 CTAs per SM
    kernel<<<(unsigned)Nkv, race::dec::NT, sm, s>>>(qq, kk, vv, planes_T, A, B, oo, (int)group, (int)D, (int)L,
                                                    (int)P, eps, logit_scale);
    return RACE_OK;
  };
  if (dtype == RACE_F32) {
    RACE_TRY(group <= 4 ? launch(race::dec::decode_step<float, 4>, (const float *)q, (const float *)k,
                                 (const float *)v, (float *)out)
                        : launch(race::dec::decode_step<float, MAXG>, (const float *)q, (const float *)k,
                                 (const float *)v, (float *)out));
  } else {
    RACE_TRY(group <= 4 ? launch(race::dec::decode_step<bf, 4>, (const bf *)q, (const bf *)k, (const bf *)v,
                                 (bf *)out)
                        : launch(race::dec::decode_step<bf, MAXG>, (const bf *)q, (const bf *)k, (const bf *)v,
                                 (bf *)out));
  }
  RACE_TRY(check_launch("decode_step"));
  return ok();
}

}  // extern "C"
