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

// Bucket slots of the state pass: with D % 4 == 0 a thread owns 4 consecutive dims
// (float4 rows of B), otherwise one dim.
__host__ __device__ __forceinline__ int bucket_slots(int D) { return (D % 4 == 0) ? NT / (D / 4) : NT / D; }

// The planes are staged in shared memory when they take at most this many floats, and
// the stream's B state (S x D fp32) when D % 4 == 0 and it takes at most this many.
constexpr int PLANES_SMEM_MAX = 16384;
constexpr int STATE_SMEM_MAX = 16384;

__host__ __device__ __forceinline__ bool planes_in_smem(int D, int LP) { return D * LP <= PLANES_SMEM_MAX; }
__host__ __device__ __forceinline__ bool state_in_smem(int D, int S) {
  return D % 4 == 0 && S % 4 == 0 && S * D <= STATE_SMEM_MAX;
}

// shared-memory plan, in floats
struct DecLayout {
  size_t x, v, a, p, an, a0, red, pl, b, total;
};

__host__ __device__ __forceinline__ DecLayout dec_layout(int D, int S, int LP, int group) {
  const size_t rows = 1 + group;
  DecLayout m;
  size_t o = 0;
  m.x = o; o += rows * D;          // [rows][D]   row 0 = key, rows 1.. = query heads of the group
  m.v = o; o += D;                 // [D]
  m.a = o; o += rows * LP * 2;     // [rows][LP][2]  per plane: sigma(-2a), sigma(+2a)
  m.p = o; o += rows * S;          // [rows][S]   row 0 = pk, rows 1.. = pq
  m.an = o; o += S;                // [S]         1 / (updated A + eps)
  o = (o + 3) & ~(size_t)3;
  m.a0 = o; if (state_in_smem(D, S)) o += S;  // [S] the stream's A, prefetched
  m.pl = o; if (planes_in_smem(D, LP)) o += (size_t)D * LP;  // [D][LP]
  o = (o + 3) & ~(size_t)3;
  m.b = o; if (state_in_smem(D, S)) o += (size_t)S * D;      // [S][D] the stream's B, prefetched
  // [slots][group][D] partial outputs; they reuse the prefetched B once it has been consumed
  const size_t nred = (size_t)bucket_slots(D) * group * D;
  if (state_in_smem(D, S) && nred <= (size_t)S * D) {
    m.red = m.b;
  } else {
    m.red = o;
    o += nred;
  }
  m.total = o;
  return m;
}

__host__ __device__ __forceinline__ size_t smem_floats(int D, int S, int LP, int group) {
  return dec_layout(D, S, LP, group).total;
}

__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// grid Nkv, block NT (requires D <= NT, group <= MG <= MAX_GROUP; MG sizes the accumulators)
template <typename XT, int MG>
__global__ void __launch_bounds__(NT, MG <= 4 ? 4 : 1) decode_step(const XT *__restrict__ q, const XT *__restrict__ k,
                                                  const XT *__restrict__ v, const float *__restrict__ planes_T,
                                                  float *__restrict__ A, float *__restrict__ B,
                                                  XT *__restrict__ out, int group, int D, int L, int P,
                                                  float eps, float scale) {
  extern __shared__ __align__(16) float sm[];
  const int LP = L * P, R = 1 << P, S = L * R;
  const int n = blockIdx.x, tid = threadIdx.x;
  const int rows = 1 + group;
  const DecLayout lay = dec_layout(D, S, LP, group);
  float *sX = sm + lay.x, *sv = sm + lay.v, *sa = sm + lay.a, *sp = sm + lay.p, *sAn = sm + lay.an;
  float *red = sm + lay.red, *spl = sm + lay.pl, *sB = sm + lay.b, *sA = sm + lay.a0;
  const bool pl_smem = planes_in_smem(D, LP), b_smem = state_in_smem(D, S);
  // the stream's state (A, B) starts streaming in now and lands while the token is hashed
  if (b_smem) {
    const float *src = B + (size_t)n * S * D;
    for (int i = tid; i < S * D / 4; i += NT) cp_async16(sB + 4 * i, src + 4 * i);
    for (int i = tid; i < S / 4; i += NT) cp_async16(sA + 4 * i, A + (size_t)n * S + 4 * i);
  }
  for (int i = tid; i < rows * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[i] = r == 0 ? to_f(k[(size_t)n * D + d]) : to_f(q[((size_t)n * group + r - 1) * D + d]);
  }
  for (int d = tid; d < D; d += NT) sv[d] = to_f(v[(size_t)n * D + d]);
  if (pl_smem)
    for (int i = tid; i < D * LP; i += NT) spl[i] = planes_T[i];
  __syncthreads();
  // a = scale tanh(x . plane); the softmax over a table's 2^P corners (logit of corner c:
  // sum_p sign_p(c) a_p) is the product over its planes of two-way softmaxes, so each
  // plane keeps sigma(-2a) and sigma(+2a), computed without overflow for either sign
  const float *pl = pl_smem ? spl : planes_T;
  for (int i = tid; i < rows * LP; i += NT) {
    const int r = i / LP, j = i % LP;
    float acc0 = 0.f, acc1 = 0.f;  // two independent chains
    int d = 0;
#pragma unroll 4
    for (; d + 1 < D; d += 2) {
      acc0 = fmaf(sX[r * D + d], pl[(size_t)d * LP + j], acc0);
      acc1 = fmaf(sX[r * D + d + 1], pl[(size_t)(d + 1) * LP + j], acc1);
    }
    if (d < D) acc0 = fmaf(sX[r * D + d], pl[(size_t)d * LP + j], acc0);
    const float a2 = 2.f * tanhf(acc0 + acc1) * scale;
    const float e = expf(-fabsf(a2)), big = 1.f / (1.f + e), small = e * big;
    sa[2 * i] = a2 >= 0.f ? small : big;      // sigma(-2a)
    sa[2 * i + 1] = a2 >= 0.f ? big : small;  // sigma(+2a)
  }
  __syncthreads();
  // corner c of table l: prod_p sigma(sign_p(c) 2 a_p), sign_p(c) = + iff bit P-1-p of c is set
  for (int i = tid; i < rows * S; i += NT) {
    const int r = i / S, si = i % S, l = si / R, c = si % R;
    const float *f = sa + 2 * (r * LP + l * P);
    float pr = 1.f;
    for (int p = 0; p < P; ++p) pr *= f[2 * p + ((c >> (P - 1 - p)) & 1)];
    sp[i] = pr;
  }
  __syncthreads();
  if (b_smem) {
    cp_async_wait_all();
    __syncthreads();
  }
  for (int s = tid; s < S; s += NT) {
    const float an = (b_smem ? sA[s] : A[(size_t)n * S + s]) + sp[s];
    A[(size_t)n * S + s] = an;
    sAn[s] = 1.f / (an + eps);
  }
  __syncthreads();
  // B[s,:] += pk[s] v ;  acc_h += pq_h[s] B[s,:] / (A[s] + eps), bucket slots over s
  const int nsg = bucket_slots(D);
  if (D % 4 == 0) {
    const int D4 = D / 4, c4 = tid % D4, sg = tid / D4;
    float4 acc[MG];
#pragma unroll
    for (int h = 0; h < MG; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (sg < nsg) {
      const float4 vd = reinterpret_cast<const float4 *>(sv)[c4];
      float4 *bn = reinterpret_cast<float4 *>(B + (size_t)n * S * D) + c4;
      const float4 *bsrc = b_smem ? reinterpret_cast<const float4 *>(sB) + c4 : bn;
      auto step = [&](int s, float4 b) {
        const float ps = sp[s], r = sAn[s];
        b.x = fmaf(ps, vd.x, b.x);
        b.y = fmaf(ps, vd.y, b.y);
        b.z = fmaf(ps, vd.z, b.z);
        b.w = fmaf(ps, vd.w, b.w);
        bn[(size_t)s * D4] = b;
#pragma unroll
        for (int h = 0; h < MG; ++h)
          if (h < group) {
            const float w = sp[(1 + h) * S + s] * r;
            acc[h].x = fmaf(w, b.x, acc[h].x);
            acc[h].y = fmaf(w, b.y, acc[h].y);
            acc[h].z = fmaf(w, b.z, acc[h].z);
            acc[h].w = fmaf(w, b.w, acc[h].w);
          }
      };
      int s = sg;
      for (; s + 3 * nsg < S; s += 4 * nsg) {  // four rows in flight
        const float4 b0 = bsrc[(size_t)s * D4], b1 = bsrc[(size_t)(s + nsg) * D4];
        const float4 b2 = bsrc[(size_t)(s + 2 * nsg) * D4], b3 = bsrc[(size_t)(s + 3 * nsg) * D4];
        step(s, b0);
        step(s + nsg, b1);
        step(s + 2 * nsg, b2);
        step(s + 3 * nsg, b3);
      }
      for (; s < S; s += nsg) step(s, bsrc[(size_t)s * D4]);
    }
    __syncthreads();  // red may overlay the prefetched B
    if (sg < nsg) {
#pragma unroll
      for (int h = 0; h < MG; ++h)
        if (h < group) reinterpret_cast<float4 *>(red + ((size_t)sg * group + h) * D)[c4] = acc[h];
    }
  } else {
    const int d = tid % D, sg = tid / D;
    float acc[MG];
#pragma unroll
    for (int h = 0; h < MG; ++h) acc[h] = 0.f;
    if (sg < nsg) {
      const float vd = sv[d];
      float *bn = B + (size_t)n * S * D;
      for (int s = sg; s < S; s += nsg) {
        const float b = fmaf(sp[s], vd, bn[(size_t)s * D + d]);
        bn[(size_t)s * D + d] = b;
        const float e = b * sAn[s];
#pragma unroll
        for (int h = 0; h < MG; ++h)
          if (h < group) acc[h] = fmaf(sp[(1 + h) * S + s], e, acc[h]);
      }
#pragma unroll
      for (int h = 0; h < MG; ++h)
        if (h < group) red[((size_t)sg * group + h) * D + d] = acc[h];
    }
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
