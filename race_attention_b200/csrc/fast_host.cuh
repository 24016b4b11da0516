// fast_host.cuh -- host side of the tcgen05 path: eligibility, planning,
// tensor maps and launches.  Included once, by race_api.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "fast_bwd.cuh"
#include "fast_fwd.cuh"
#include "generic.cuh"

namespace race {
namespace fasthost {

namespace fk = race::fast;

// The tcgen05 path covers bf16 activations with D = 64, P = 4 and S = 128 or
// 256 (L = 8 or 16): the BASELINE configurations.  Everything else runs on
// the generic kernels.
inline bool eligible(int dtype, int64_t D, int64_t L, int64_t P) {
  return dtype == RACE_BF16 && D == fk::HD && P == 4 && (L == 8 || L == 16);
}

struct Plan {
  int nchunks, nseg, seg_chunks;
  size_t status_off, rec_off, total;
};

inline int sm_count() {
  static int cached[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

// Largest segment count a plan may use: four waves at 256 SMs (the workspace bound).
inline int64_t max_segments(int64_t N, int64_t nchunks) {
  int64_t m = (4 * (int64_t)256) / N;
  if (m < 1) m = 1;
  return m < nchunks ? m : nchunks;
}

// One CTA (one SM) per (stream, segment), from about four waves of CTAs: among the
// segment counts between that and the workspace bound, the one with the smallest
// waves x (chunks per segment + 2), the 2 standing for a segment's fixed start and end
// work (the last wave of a launch is otherwise partly idle: 32 streams on 148 SMs give
// 576 CTAs = 3.89 waves at 18 segments, 736 = 4.97 at 23).
inline Plan plan(int64_t N, int64_t T, int64_t S, int sms) {
  Plan p;
  p.nchunks = (int)((T + fk::C - 1) / fk::C);
  // (a device with more than 256 SMs plans within the same workspace bound: the
  // segment count never exceeds max_segments, which the workspace is sized for)
  const int64_t cap = max_segments(N, p.nchunks);
  int64_t want = (4 * (int64_t)sms) / N;
  if (want < 1) want = 1;
  if (want > cap) want = cap;
  auto cost = [&](int64_t cand, int64_t *nseg) {
    const int64_t sc = (p.nchunks + cand - 1) / cand;
    *nseg = (p.nchunks + sc - 1) / sc;
    return ((N * *nseg + sms - 1) / sms) * (sc + 2);
  };
  int64_t best_seg = 0, best = cost(want, &best_seg);
  for (int64_t cand = want + 1; cand <= cap; ++cand) {
    int64_t ns = 0;
    const int64_t c = cost(cand, &ns);
    if (c < best) {
      best = c;
      best_seg = ns;
    }
  }
  p.seg_chunks = (int)((p.nchunks + best_seg - 1) / best_seg);
  p.nseg = (p.nchunks + p.seg_chunks - 1) / p.seg_chunks;
  const size_t E = (size_t)S + (size_t)S * fk::HD;
  p.status_off = 0;
  p.rec_off = 256;
  p.total = p.rec_off + align_up(sizeof(float) * (size_t)N * p.nseg * E, 256);
  return p;
}

// Workspace of the fast forward (planned for the worst case of the SM count
// so the size does not depend on the device: 4 waves at up to 256 SMs).
inline size_t fwd_workspace_bytes(int64_t N, int64_t T, int64_t S) { return plan(N, T, S, 256).total; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor-map encoding is a driver-API call and needs a current context on the
// calling thread; a thread that has only queried the runtime (e.g. torch's
// autograd worker) may not have one yet.  Binding the current device's primary
// context is a no-op when it is already current.
inline bool bind_current_context() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess;
}

// result of the last failed encode on this thread (for error messages)
inline int &last_encode_status() {
  static thread_local int st = 0;
  return st;
}

// 3-D map over a [N][T][64] bf16 tensor, box [1][128][64], 128-byte swizzle.
inline bool make_map(CUtensorMap *m, const void *base, int64_t N, int64_t T) {
  EncodeTiledFn enc = encoder();
  if (!enc) {
    last_encode_status() = -1;
    return false;
  }
  cuuint64_t dims[3] = {(cuuint64_t)fk::HD, (cuuint64_t)T, (cuuint64_t)N};
  cuuint64_t strides[2] = {(cuuint64_t)fk::HD * 2, (cuuint64_t)T * fk::HD * 2};
  cuuint32_t box[3] = {(cuuint32_t)fk::HD, (cuuint32_t)fk::C, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  last_encode_status() = (int)r;
  return r == CUDA_SUCCESS;
}

// Activation tensor [B, T, H, 64] bf16 (N = B H streams; H = 1: [N, T, 64]) as a 4-D map
// (64, H, T, B), box (64, 1, 128, 1): one stream's 128-token tile per copy, rows past T read
// as zero (loads) or are not written (stores).
inline bool make_act_map(CUtensorMap *m, const void *base, int64_t N, int64_t T, int64_t H) {
  EncodeTiledFn enc = encoder();
  if (!enc || H < 1 || N % H != 0) {
    last_encode_status() = -1;
    return false;
  }
  cuuint64_t dims[4] = {(cuuint64_t)fk::HD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)(N / H)};
  cuuint64_t strides[3] = {(cuuint64_t)fk::HD * 2, (cuuint64_t)H * fk::HD * 2, (cuuint64_t)T * H * fk::HD * 2};
  cuuint32_t box[4] = {(cuuint32_t)fk::HD, 1, (cuuint32_t)fk::C, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  last_encode_status() = (int)r;
  return r == CUDA_SUCCESS;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Backward workspace: status | forward segment records | backward segment
// records | per-chunk start state (A + eps fp32, B bf16) | d proj_Q [N, T, 64] bf16
// and segment-local d proj_K [N, T, 64] fp32 (reverse walk -> fix-up) | for the
// split backward, the walk's dV [N, T, 64] bf16.
struct BwdPlan {
  Plan p;
  size_t fwd_rec, bwd_rec, chunkA, chunkB, dprojQ, dprojK, dVloc, total;
};

// split: room for the walk's dV between race_bwd_local and race_bwd_finish
inline BwdPlan bwd_plan(int64_t N, int64_t T, int64_t S, int sms, bool split = false) {
  BwdPlan b;
  b.p = plan(N, T, S, sms);
  const size_t E = (size_t)S + (size_t)S * fk::HD;
  const size_t rec = align_up(sizeof(float) * (size_t)N * b.p.nseg * E, 256);
  b.fwd_rec = 256;
  b.bwd_rec = b.fwd_rec + rec;
  b.chunkA = b.bwd_rec + rec;
  b.chunkB = b.chunkA + align_up(sizeof(float) * (size_t)N * b.p.nchunks * S, 256);
  b.dprojQ = b.chunkB + align_up(sizeof(uint16_t) * (size_t)N * b.p.nchunks * S * fk::HD, 256);
  b.dprojK = b.dprojQ + align_up(sizeof(uint16_t) * (size_t)N * T * fk::HD, 256);
  // d proj_K table-major per chunk: [N, nchunks, LP/4 tables, 128 tokens, 4] fp32
  b.dVloc = b.dprojK + align_up(sizeof(float) * (size_t)N * b.p.nchunks * fk::C * (S / 4), 256);
  b.total = b.dVloc + (split ? align_up(sizeof(uint16_t) * (size_t)N * T * fk::HD, 256) : 0);
  return b;
}

inline size_t bwd_workspace_bytes(int64_t N, int64_t T, int64_t S, bool split = false) {
  return bwd_plan(N, T, S, 256, split).total;
}

// What a saving forward keeps for the backward: A + eps [N, nchunks, S] fp32 and
// B [N, nchunks, S, 64] bf16 at every 128-token chunk start (independent of the segment plan).
struct SavedPlan {
  size_t chunkA, chunkB, total;
};

inline SavedPlan saved_plan(int64_t N, int64_t T, int64_t S) {
  SavedPlan v;
  const int64_t nchunks = (T + fk::C - 1) / fk::C;
  v.chunkA = 0;
  v.chunkB = align_up(sizeof(float) * (size_t)N * nchunks * S, 256);
  v.total = v.chunkB + align_up(sizeof(uint16_t) * (size_t)N * nchunks * S * fk::HD, 256);
  return v;
}

// 2-D map over the per-chunk B states viewed as [rows][64] bf16, box [64 x 64].
inline bool make_rows_map(CUtensorMap *m, const void *base, int64_t rows) {
  EncodeTiledFn enc = encoder();
  if (!enc) {
    last_encode_status() = -1;
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)fk::HD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)fk::HD * 2};
  cuuint32_t box[2] = {(cuuint32_t)fk::HD, (cuuint32_t)fk::GW};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  last_encode_status() = (int)r;
  return r == CUDA_SUCCESS;
}

}  // namespace fasthost
}  // namespace race
