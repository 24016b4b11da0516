// decode.cuh -- fused single-token decode step over a persistent RACE state.
//
// The reference has no decode path (chat/nanochat/gpt.py:143-146 raises); the
// math is one step of the causal scan of scaling/race_common.py:76-90 with the
// state (A, B) carried across calls -- exactly race_prefix_ref's
// A_final/B_final (scaling/race_common.py:88-90).  Grouped-query sharing: q
// head i reads kv stream i / group; the state is kept once per kv stream.
#pragma once

#include "common.cuh"

namespace race {
namespace dec {

constexpr int NT = 256;
constexpr int MAX_GROUP = 16;

__host__ __device__ __forceinline__ size_t smem_floats(int D, int S, int LP, int group) {
  const int nsg = NT / D;
  return (size_t)(1 + group) * D + D + (size_t)(1 + group) * LP + (size_t)(1 + group) * S + S +
         (size_t)nsg * group * D;
}

// grid Nkv, block NT (requires D <= NT, group <= MAX_GROUP)
template <typename XT>
__global__ void __launch_bounds__(NT) decode_step(const XT *__restrict__ q, const XT *__restrict__ k,
                                                  const XT *__restrict__ v, const float *__restrict__ planes_T,
                                                  float *__restrict__ A, float *__restrict__ B,
                                                  XT *__restrict__ out, int group, int D, int L, int P,
                                                  float eps, float scale) {
  extern __shared__ float sm[];
  const int LP = L * P, R = 1 << P, S = L * R;
  const int n = blockIdx.x, tid = threadIdx.x;
  const int rows = 1 + group;          // row 0 = key, rows 1.. = query heads of this group
  float *sX = sm;                      // [rows][D]
  float *sv = sX + rows * D;           // [D]
  float *sa = sv + D;                  // [rows][LP]
  float *sp = sa + rows * LP;          // [rows][S]  row 0 = pk, rows 1.. = pq
  float *sAn = sp + rows * S;          // [S]  updated A + eps
  float *red = sAn + S;                // [nsg][group][D]
  for (int i = tid; i < rows * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[i] = r == 0 ? to_f(k[(size_t)n * D + d]) : to_f(q[((size_t)n * group + r - 1) * D + d]);
  }
  for (int d = tid; d < D; d += NT) sv[d] = to_f(v[(size_t)n * D + d]);
  __syncthreads();
  for (int i = tid; i < rows * LP; i += NT) {
    const int r = i / LP, j = i % LP;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(sX[r * D + d], planes_T[(size_t)d * LP + j], acc);
    sa[i] = tanhf(acc) * scale;
  }
  __syncthreads();
  for (int i = tid; i < rows * L; i += NT) {
    const int r = i / L, l = i % L;
    const float *a = sa + r * LP + l * P;
    float mx = -INFINITY;
    for (int c = 0; c < R; ++c) {
      float x = 0.f;
      for (int p = 0; p < P; ++p) x = fmaf(a[p], corner_sign(c, p, P), x);
      mx = fmaxf(mx, x);
    }
    float z = 0.f;
    for (int c = 0; c < R; ++c) {
      float x = 0.f;
      for (int p = 0; p < P; ++p) x = fmaf(a[p], corner_sign(c, p, P), x);
      z += expf(x - mx);
    }
    const float iz = 1.f / z;
    for (int c = 0; c < R; ++c) {
      float x = 0.f;
      for (int p = 0; p < P; ++p) x = fmaf(a[p], corner_sign(c, p, P), x);
      sp[r * S + l * R + c] = expf(x - mx) * iz;
    }
  }
  __syncthreads();
  for (int s = tid; s < S; s += NT) {
    const float an = A[(size_t)n * S + s] + sp[s];
    A[(size_t)n * S + s] = an;
    sAn[s] = an + eps;
  }
  __syncthreads();
  const int nsg = NT / D;
  const int d = tid % D, sg = tid / D;
  float acc[MAX_GROUP];
#pragma unroll
  for (int h = 0; h < MAX_GROUP; ++h) acc[h] = 0.f;
  if (sg < nsg) {
    const float vd = sv[d];
    float *bn = B + (size_t)n * S * D;
    for (int s = sg; s < S; s += nsg) {
      const float b = fmaf(sp[s], vd, bn[(size_t)s * D + d]);
      bn[(size_t)s * D + d] = b;
      const float e = b / sAn[s];
#pragma unroll
      for (int h = 0; h < MAX_GROUP; ++h)
        if (h < group) acc[h] = fmaf(sp[(1 + h) * S + s], e, acc[h]);
    }
#pragma unroll
    for (int h = 0; h < MAX_GROUP; ++h)
      if (h < group) red[((size_t)sg * group + h) * D + d] = acc[h];
  }
  __syncthreads();
  for (int i = tid; i < group * D; i += NT) {
    const int h = i / D, dd = i % D;
    float o = 0.f;
    for (int g2 = 0; g2 < nsg; ++g2) o += red[((size_t)g2 * group + h) * D + dd];
    out[((size_t)n * group + h) * D + dd] = from_f<XT>(o);
  }
}

}  // namespace dec
}  // namespace race
