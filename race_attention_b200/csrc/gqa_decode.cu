// gqa_decode.cu -- softmax grouped-query attention for one decode token over a
// KV cache, with the token's own key/value appended to the cache in the same
// launch.
//
// This is not a RACE operator.  It is the softmax half of a hybrid decoder in
// which some layers are RACE (the fused decode step of decode.cuh) and the
// others are ordinary softmax attention over a KV cache (the Llama-3.2-1B
// hybrid decode configuration).  It exists so that a whole decode step can be
// captured once as a CUDA graph: the cache length is read from device memory
// instead of being a launch parameter, so the same launch serves every step.
//
// Semantics, per batch row b and kv head g (query heads g*G .. g*G+G-1,
// G = Hq / Hkv <= 8, the repeat-interleave grouping of grouped-query attention):
//   n = *len (tokens already in the cache);  cache[b, g, n] <- (k_new, v_new)
//   out[b, g*G+h] = softmax_j(scale * q[b, g*G+h] . K[b, g, j]) V[b, g, j],  j = 0 .. n
//
// Parallel layout (split-KV): grid (n_splits, B*Hkv); split s of a stream takes
// an equal share of the n+1 keys, computes a partial softmax (running max m,
// sum l, unnormalised output o per head) and writes it to the workspace; the
// last split to finish (an atomic ticket per stream, no waiting) merges the
// partials and writes the output.  Inside a CTA each of 4 warps streams its
// own contiguous run of 16-key blocks through a 4-stage shared-memory ring
// (cp.async, 16 bytes per lane, rows XOR-swizzled by 16-byte chunk so the
// fragment loads are conflict-free).  Per block the warp runs the two products
// on the bf16 tensor cores with mma.sync m16n8k16: S = Q K^T with the group's
// query heads as the rows of a 16-row tile (rows >= G are zero), then O += P V
// with P (the block's softmax weights, rounded to bf16) taken straight from
// the score fragments.  The work is an HBM stream of the cache, 4*D bytes per
// key (K and V rows in bf16), about 6 warp instructions per key.
#include "race_b200.h"

#include <atomic>
#include <stdio.h>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kD = 64;          // head dim
constexpr int kWarps = 4;       // warps per CTA
constexpr int kNT = 32 * kWarps;
constexpr int kBlk = 16;        // keys per block
constexpr int kStages = 4;      // ring depth per warp
constexpr int kMaxG = 8;
constexpr int kMaxSplits = 64;
constexpr int kMaxDevices = 128;
constexpr int kRowBytes = kD * 2;                      // one K or V row
constexpr int kStageBytes = 2 * kBlk * kRowBytes;      // K block + V block
constexpr int kWarpSmem = kStages * kStageBytes;       // 16 KB
constexpr int kSmem = kWarps * kWarpSmem;              // 64 KB

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous copy; src_bytes == 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulators.  Rows 8..15
// of A are always zero here (at most 8 query heads), so a1 = a3 = 0.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};\n"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// byte offset of 16-byte chunk c of row r inside a [16 rows][8 chunks] block
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * kRowBytes + ((c ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(kNT)
gqa_decode_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k_new,
                  const __nv_bfloat16 *__restrict__ v_new, __nv_bfloat16 *__restrict__ k_cache,
                  __nv_bfloat16 *__restrict__ v_cache, const int32_t *__restrict__ len_p,
                  __nv_bfloat16 *__restrict__ out, float *__restrict__ ws_o, float *__restrict__ ws_ml,
                  unsigned *__restrict__ tickets, int *__restrict__ status, long long Tmax, int G, int n_splits,
                  float qscale) {
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ float red_o[kWarps][kMaxG][kD];
  __shared__ float red_ml[kWarps][kMaxG][2];
  __shared__ int last_flag;

  const int split = blockIdx.x;
  const long long n = blockIdx.y;  // stream b*Hkv + g
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = lane >> 2, quad = lane & 3;  // fragment row (query head) and column pair

  const long long len = *len_p;
  if (len < 0 || len >= Tmax) {  // no room for the new token: report, touch nothing
    if (split == 0 && n == 0 && tid == 0) *status = 1;
    return;
  }
  const long long total = len + 1;
  long long chunk = (total + n_splits - 1) / n_splits;
  chunk = (chunk + kBlk - 1) / kBlk * kBlk;
  const long long k0 = (long long)split * chunk;
  const long long k1 = k0 + chunk < total ? k0 + chunk : total;

  const __nv_bfloat16 *kc = k_cache + n * Tmax * kD;
  const __nv_bfloat16 *vc = v_cache + n * Tmax * kD;
  const __nv_bfloat16 *kn = k_new + n * kD;
  const __nv_bfloat16 *vn = v_new + n * kD;

  // The split that owns position len appends the new key/value; reads of that
  // position inside this launch come from k_new / v_new, so no ordering is needed.
  if (k0 <= len && len < k1 && tid < 16) {
    const int which = tid >> 3, part = tid & 7;
    const __nv_bfloat16 *src = (which ? vn : kn) + part * 8;
    __nv_bfloat16 *dst = (which ? v_cache : k_cache) + (n * Tmax + len) * kD + part * 8;
    *reinterpret_cast<uint4 *>(dst) = __ldg(reinterpret_cast<const uint4 *>(src));
  }

  // this warp's blocks: a contiguous quarter of the split's blocks
  const int nblk_cta = k1 > k0 ? (int)((k1 - k0 + kBlk - 1) / kBlk) : 0;
  const int b_begin = nblk_cta * warp / kWarps, b_end = nblk_cta * (warp + 1) / kWarps;
  const int nblk = b_end - b_begin;

  // Q fragments (A operand, row = query head, k = dim), zero for rows >= G
  uint32_t qa0[4], qa2[4];
  {
    const bool live = row < G;
    const __nv_bfloat16 *qr = q + (n * G + (live ? row : 0)) * kD;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t x0 = __ldg(reinterpret_cast<const uint32_t *>(qr + 16 * s + 2 * quad));
      const uint32_t x2 = __ldg(reinterpret_cast<const uint32_t *>(qr + 16 * s + 8 + 2 * quad));
      qa0[s] = live ? x0 : 0u;
      qa2[s] = live ? x2 : 0u;
    }
  }

  const uint32_t wring = smem_u32(ring) + warp * kWarpSmem;
  // lane l copies chunks (l & 7) of rows (l >> 3) + 4i, i = 0..3, of the K and V blocks
  auto issue = [&](int bi) {
    const uint32_t st = wring + (uint32_t)((bi % kStages) * kStageBytes);
    if (bi < nblk) {
      const long long kb = k0 + (long long)(b_begin + bi) * kBlk;
      const int c = lane & 7;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (lane >> 3) + 4 * i;
        const long long j = kb + r;
        const bool in = j < k1;
        const bool fresh = j == len;
        const __nv_bfloat16 *ks = fresh ? kn : kc + (in ? j : k0) * kD;
        const __nv_bfloat16 *vs = fresh ? vn : vc + (in ? j : k0) * kD;
        cp_async16(st + swz(r, c), ks + c * 8, in ? 16 : 0);
        cp_async16(st + kBlk * kRowBytes + swz(r, c), vs + c * 8, in ? 16 : 0);
      }
    }
    cp_async_commit();  // an empty group past the end keeps the wait count uniform
  };

  float m_run = -INFINITY, l_run = 0.f;  // row `row`, this lane's share of the sum
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) issue(i);
  for (int bi = 0; bi < nblk; ++bi) {
    issue(bi + kStages - 1);
    cp_async_wait<kStages - 1>();
    __syncwarp();
    const uint32_t kst = wring + (uint32_t)((bi % kStages) * kStageBytes);
    const uint32_t vst = kst + kBlk * kRowBytes;

    // S = Q K^T for keys [0,8) and [8,16) of the block
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {  // dims [32*s2, 32*s2+32): two k-steps per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        const int r = nt * 8 + (lane & 7);
        ldsm_x4(kst + swz(r, 4 * s2 + (lane >> 3)), b0, b1, b2, b3);
        mma_bf16(sc[nt], qa0[2 * s2], qa2[2 * s2], b0, b1);
        mma_bf16(sc[nt], qa0[2 * s2 + 1], qa2[2 * s2 + 1], b2, b3);
      }
    }
    // scores of row `row` for keys 2q, 2q+1 (tile 0) and 8+2q, 9+2q (tile 1), in log2 units
    const long long kb = k0 + (long long)(b_begin + bi) * kBlk;
    float x[4] = {sc[0][0] * qscale, sc[0][1] * qscale, sc[1][0] * qscale, sc[1][1] * qscale};
    const int kk[4] = {2 * quad, 2 * quad + 1, 8 + 2 * quad, 9 + 2 * quad};
    float bm = -INFINITY;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (kb + kk[e] >= k1) x[e] = -INFINITY;
      bm = fmaxf(bm, x[e]);
    }
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    const float m_new = fmaxf(m_run, bm);
    const float mr = m_new == -INFINITY ? 0.f : m_new;
    const float corr = exp2f(m_run - mr);
    m_run = m_new;
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = exp2f(x[e] - mr);
    l_run = l_run * corr + ((p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= corr;
      o[j][1] *= corr;
    }
    const uint32_t pa0 = pack_bf16(p[0], p[1]), pa2 = pack_bf16(p[2], p[3]);
    // O += P V: dims [16*jj, 16*jj+16) per ldmatrix.x4.trans
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t b0, b1, b2, b3;
      const int r = ((lane >> 3) & 1) * 8 + (lane & 7);
      ldsm_x4_t(vst + swz(r, 2 * jj + (lane >> 4)), b0, b1, b2, b3);
      mma_bf16(o[2 * jj], pa0, pa2, b0, b1);
      mma_bf16(o[2 * jj + 1], pa0, pa2, b2, b3);
    }
    __syncwarp();  // the stage is refilled by the next iteration's issue
  }
  cp_async_wait<0>();

  // row sums across the quad; the quad already shares m_run
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (row < G) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      red_o[warp][row][8 * j + 2 * quad] = o[j][0];
      red_o[warp][row][8 * j + 2 * quad + 1] = o[j][1];
    }
    if (quad == 0) {
      red_ml[warp][row][0] = m_run;
      red_ml[warp][row][1] = l_run;
    }
  }
  __syncthreads();

  // merge the CTA's warps: one (head, dim) per thread
  const long long part = n * n_splits + split;
  for (int e = tid; e < G * kD; e += kNT) {
    const int h = e / kD, d = e % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_ml[w][h][0]);
    const float Mr = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = exp2f(red_ml[w][h][0] - Mr);
      L = fmaf(red_ml[w][h][1], c, L);
      O = fmaf(red_o[w][h][d], c, O);
    }
    if (n_splits == 1) {
      out[(n * G + h) * kD + d] = __float2bfloat16_rn(O / L);
    } else {
      ws_o[(part * G + h) * kD + d] = O;
      if (d == 0) {
        ws_ml[(part * G + h) * 2 + 0] = M;
        ws_ml[(part * G + h) * 2 + 1] = L;
      }
    }
  }
  if (n_splits == 1) return;

  // the last split of this stream merges all partials
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = atomicAdd(&tickets[n], 1u) == (unsigned)(n_splits - 1);
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  for (int e = tid; e < G * kD; e += kNT) {
    const int h = e / kD, d = e % kD;
    float M = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(ws_ml + ((n * n_splits + sp) * G + h) * 2));
    const float Mr = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const long long pp = (n * n_splits + sp) * G + h;
      const float c = exp2f(__ldcg(ws_ml + pp * 2) - Mr);
      L = fmaf(__ldcg(ws_ml + pp * 2 + 1), c, L);
      O = fmaf(__ldcg(ws_o + pp * kD + d), c, O);
    }
    out[(n * G + h) * kD + d] = __float2bfloat16_rn(O / L);
  }
  if (tid == 0) tickets[n] = 0u;  // every split has taken its ticket: ready for the next call
}

int err(int code, const char *fmt, long long a = 0, long long b = 0) {
  char buf[256];
  snprintf(buf, sizeof(buf), fmt, a, b);
  return race::report_error(code, buf);
}

int launch(const void *q, const void *k_new, const void *v_new, void *k_cache, void *v_cache, const int32_t *len,
           void *out, float *ws, long long streams, int G, long long Tmax, int n_splits, float qscale,
           cudaStream_t s) {
  // The first call on a device (make it outside any stream capture) raises the
  // kernel's dynamic shared-memory limit there.
  static std::atomic<bool> smem_set[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return err(RACE_ERR_CUDA, "no usable current device (%lld)", dev);
  if (!smem_set[dev].load()) {
    const cudaError_t e = cudaFuncSetAttribute(gqa_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return err(RACE_ERR_CUDA, "cudaFuncSetAttribute failed (%lld)", (long long)e);
    smem_set[dev].store(true);
  }
  float *ws_o = ws;
  float *ws_ml = ws_o + (size_t)streams * n_splits * G * kD;
  unsigned *tickets = reinterpret_cast<unsigned *>(ws_ml + (size_t)streams * n_splits * G * 2);
  int *status = reinterpret_cast<int *>(tickets + streams);
  dim3 grid((unsigned)n_splits, (unsigned)streams);
  gqa_decode_kernel<<<grid, kNT, kSmem, s>>>(
      (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_new, (const __nv_bfloat16 *)v_new,
      (__nv_bfloat16 *)k_cache, (__nv_bfloat16 *)v_cache, len, (__nv_bfloat16 *)out, ws_o, ws_ml, tickets, status,
      Tmax, G, n_splits, qscale);
  race::note_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "gqa_decode_kernel: %s", cudaGetErrorString(e));
    return race::report_error(RACE_ERR_CUDA, buf);
  }
  race::clear_error();
  return RACE_OK;
}

}  // namespace

extern "C" {

size_t race_gqa_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int n_splits) {
  if (B < 1 || Hq < 1 || Hkv < 1 || n_splits < 1) return 0;
  const size_t streams = (size_t)B * Hkv;
  return sizeof(float) * (size_t)B * Hq * n_splits * (kD + 2) + sizeof(unsigned) * streams + sizeof(int);
}

int race_gqa_decode_attn(const void *q, const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                         const int32_t *len, void *out, void *workspace, int64_t B, int64_t Hq, int64_t Hkv,
                         int64_t Tmax, int64_t D, int n_splits, float softmax_scale, void *stream) {
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !len || !out || !workspace)
    return err(RACE_ERR_ARG, "race_gqa_decode_attn: null pointer");
  if (D != kD) return err(RACE_ERR_UNSUPPORTED, "head dim %lld (only %lld)", (long long)D, (long long)kD);
  if (B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv) return err(RACE_ERR_SHAPE, "Hq=%lld must be a multiple of Hkv=%lld",
                                                           (long long)Hq, (long long)Hkv);
  if (B * Hkv > 65535) return err(RACE_ERR_SHAPE, "B*Hkv=%lld > 65535", (long long)(B * Hkv));
  if (Tmax < 1) return err(RACE_ERR_SHAPE, "cache capacity %lld < 1", (long long)Tmax);
  if (n_splits < 1 || n_splits > kMaxSplits) return err(RACE_ERR_SHAPE, "n_splits=%lld not in [1,%lld]", n_splits,
                                                        kMaxSplits);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
       reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return err(RACE_ERR_ALIGN, "q, k_new, v_new, caches and workspace must be 16-byte aligned");
  const long long G = Hq / Hkv, streams = B * Hkv;
  const float qscale = softmax_scale * 1.4426950408889634f;  // exp(x) = exp2(x log2 e)
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float *ws = reinterpret_cast<float *>(workspace);
  if (G > kMaxG) return err(RACE_ERR_UNSUPPORTED, "query group %lld > %lld", G, kMaxG);
  return launch(q, k_new, v_new, k_cache, v_cache, len, out, ws, streams, (int)G, Tmax, n_splits, qscale, s);
}

}  // extern "C"
