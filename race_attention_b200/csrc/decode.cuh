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

__device__ __forceinline__ void fma4(float4 &acc, float w, const float4 &b) {
  acc.x = fmaf(w, b.x, acc.x);
  acc.y = fmaf(w, b.y, acc.y);
  acc.z = fmaf(w, b.z, acc.z);
  acc.w = fmaf(w, b.w, acc.w);
}

template <typename XT>
__device__ __forceinline__ void store4(XT *dst, const float4 &v);
template <>
__device__ __forceinline__ void store4<float>(float *dst, const float4 &v) {
  *reinterpret_cast<float4 *>(dst) = v;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *dst, const float4 &v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t *>(&lo);
  w.y = *reinterpret_cast<const uint32_t *>(&hi);
  *reinterpret_cast<uint2 *>(dst) = w;
}

// ---------------------------------------------------------------------------
// Decode step for head_dim 64 and 4 planes per table (the hybrid decoder's shape),
// with every size a compile-time constant.  The general kernel above is bound by
// instruction issue (about 16 K warp instructions per kv stream, most of them index
// arithmetic with run-time divisors and per-element reloads); this one keeps to the
// work itself:
//   * all global reads at kernel start: planes and A by cp.async (group 0); the
//     stream's B state by cp.async, each thread copying exactly the row chunks it
//     updates, in four groups awaited one by one during the update (the first rows are
//     updated and stored while the later ones arrive); the key / query rows and v
//     through registers;
//   * projections: thread (plane j, dim range) over all 1 + group rows, x read as
//     float4 broadcasts; partial sums combined in shared memory;
//   * one pass per bucket s (thread s): pk[s], the queries' corner probabilities,
//     A[s] += pk[s] (written back here: the CTA owns the stream), and
//     W_h[s] = pq_h[s] / (A[s] + eps) stored next to pk[s];
//   * update and readout: warp w owns bucket rows [w S/8, (w+1) S/8), half-warp
//     (row parity) x float4 column c4; per row one vector load of the B row chunk,
//     one of pk / W, B += pk v stored straight to global, acc_h += W_h B;
//   * reduction: the two half-warps by one shuffle, the 8 warps in shared memory.
// L in {8, 16} (S = 128, 256), group <= MG in {1, 2, 4, 8}.
namespace d64 {
constexpr int D = 64, P = 4, R = 16, NT = 256, NW = NT / 32;

// cp.async.wait_group with the count as an immediate
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// the same for a count known only after unrolling (0 <= pending < MAXN)
template <int MAXN>
__device__ __forceinline__ void cp_async_wait_dyn(int pending) {
  if constexpr (MAXN > 0) {
    if (pending == MAXN - 1) {
      cp_async_wait<MAXN - 1>();
      return;
    }
    cp_async_wait_dyn<MAXN - 1>(pending);
  }
}

template <int L, int MG>
struct Layout {
  static constexpr int S = L * R, LP = L * P, ROWS = 1 + MG, NPARTS = NT / LP, WS = MG < 4 ? 4 : MG;
  static constexpr int B0 = 0;                        // [S][64]  the stream's B
  static constexpr int PL = B0 + S * D;               // [64][LP] planes
  static constexpr int X = PL + D * LP;               // [ROWS][64] key, then queries (fp32)
  static constexpr int PART = X + ROWS * D;           // [NPARTS][ROWS][LP] partial projections
  static constexpr int SIG = PART + NPARTS * ROWS * LP;  // [ROWS][LP][2] sigma(-2a), sigma(+2a)
  static constexpr int A0 = SIG + ROWS * LP * 2;      // [S] A as loaded
  static constexpr int PK = A0 + S;                   // [S] pk
  static constexpr int W = PK + S;                    // [S][WS] W_h (WS >= 4: float4 rows)
  static constexpr int TOTAL = W + S * WS;           // floats
  // [NW][MG][64] per-warp partial outputs, over the planes, rows, partial projections and
  // plane softmaxes (all dead once W is written; pk and W stay live)
  static constexpr int RED = PL;
  static_assert(RED + NW * MG * D <= A0, "partial outputs overlap live data");
};

// (L = 8: four CTAs per SM, 50 KB of shared memory each; L = 16: two, 95 KB)
template <typename XT, int L, int MG>
__global__ void __launch_bounds__(NT, L == 8 ? 4 : 2) decode_step_d64(const XT *__restrict__ q, const XT *__restrict__ k,
                                                         const XT *__restrict__ v, const float *__restrict__ planes_T,
                                                         float *__restrict__ A, float *__restrict__ B,
                                                         XT *__restrict__ out, int group, float eps, float scale) {
  using Ly = Layout<L, MG>;
  constexpr int S = Ly::S, LP = Ly::LP, NPARTS = Ly::NPARTS, WS = Ly::WS;
  extern __shared__ __align__(16) float sm[];
  const int n = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = 1 + group;
  // ---- loads: planes, A (group 0) ; B (group 1) ; key / query rows and v through registers
  for (int i = tid; i < D * LP / 4; i += NT) cp_async16(sm + Ly::PL + 4 * i, planes_T + 4 * i);
  if (tid < S / 4) cp_async16(sm + Ly::A0 + 4 * tid, A + (size_t)n * S + 4 * tid);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  // B: each thread copies exactly the row chunks it updates below (so waiting for its own
  // copies is enough), in NB groups in the order it consumes them: the first rows are
  // updated and stored while the later ones are still arriving
  constexpr int RPW = S / NW, NB = 4, RPB = RPW / 2 / NB;  // rows per warp; row pairs per group
  const int half = lane >> 4, c4 = lane & 15;
  {
    const float *src = B + (size_t)n * S * D;
#pragma unroll
    for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
      for (int i = 0; i < RPB; ++i) {
        const int s = warp * RPW + 2 * (blk * RPB + i) + half;
        cp_async16(sm + Ly::B0 + s * D + 4 * c4, src + s * D + 4 * c4);
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
  }
  float xr[(Ly::ROWS * D + NT - 1) / NT];
#pragma unroll
  for (int i = 0; i < (Ly::ROWS * D + NT - 1) / NT; ++i) {
    const int e = tid + i * NT, r = e / D, d = e % D;  // constant divisor
    xr[i] = 0.f;
    if (r < rows) xr[i] = r == 0 ? to_f(k[(size_t)n * D + d]) : to_f(q[((size_t)n * group + r - 1) * D + d]);
  }
  float4 vv;
  vv.x = to_f(v[(size_t)n * D + 4 * c4]);
  vv.y = to_f(v[(size_t)n * D + 4 * c4 + 1]);
  vv.z = to_f(v[(size_t)n * D + 4 * c4 + 2]);
  vv.w = to_f(v[(size_t)n * D + 4 * c4 + 3]);
#pragma unroll
  for (int i = 0; i < (Ly::ROWS * D + NT - 1) / NT; ++i) {
    const int e = tid + i * NT;
    if (e < Ly::ROWS * D) sm[Ly::X + e] = xr[i];
  }
  cp_async_wait<NB>();  // planes and A (every group but the NB of B)
  __syncthreads();
  // ---- partial projections: thread (j, part) over dims [part 64 / NPARTS, ...), all rows
  {
    const int j = tid % LP, part = tid / LP;
    constexpr int DR = D / NPARTS;
    float acc[Ly::ROWS];
#pragma unroll
    for (int r = 0; r < Ly::ROWS; ++r) acc[r] = 0.f;
#pragma unroll
    for (int d4 = 0; d4 < DR; d4 += 4) {
      const int d = part * DR + d4;
      const float p0 = sm[Ly::PL + (d + 0) * LP + j], p1 = sm[Ly::PL + (d + 1) * LP + j];
      const float p2 = sm[Ly::PL + (d + 2) * LP + j], p3 = sm[Ly::PL + (d + 3) * LP + j];
#pragma unroll
      for (int r = 0; r < Ly::ROWS; ++r) {
        if (r < rows) {
          const float4 x = *reinterpret_cast<const float4 *>(sm + Ly::X + r * D + d);
          acc[r] = fmaf(x.x, p0, fmaf(x.y, p1, fmaf(x.z, p2, fmaf(x.w, p3, acc[r]))));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < Ly::ROWS; ++r)
      if (r < rows) sm[Ly::PART + (part * Ly::ROWS + r) * LP + j] = acc[r];
  }
  __syncthreads();
  // ---- a = scale tanh(x . plane) -> the plane's two-way softmax pair (see decode_step)
  for (int i = tid; i < Ly::ROWS * LP; i += NT) {
    if (i < rows * LP) {
      float x = 0.f;
#pragma unroll
      for (int p = 0; p < NPARTS; ++p) x += sm[Ly::PART + p * Ly::ROWS * LP + i];
      const float a2 = 2.f * tanhf(x) * scale;
      const float e = expf(-fabsf(a2)), big = 1.f / (1.f + e), small = e * big;
      sm[Ly::SIG + 2 * i] = a2 >= 0.f ? small : big;
      sm[Ly::SIG + 2 * i + 1] = a2 >= 0.f ? big : small;
    }
  }
  __syncthreads();
  // ---- bucket s: pk, A += pk (written back), W_h = pq_h / (A + eps)
  if (tid < S) {
    const int s = tid, l = s >> 4, c = s & 15;
    auto corner = [&](int r) {
      const float *f = sm + Ly::SIG + 2 * (r * LP + P * l);
      return f[(c >> 3) & 1] * f[2 + ((c >> 2) & 1)] * f[4 + ((c >> 1) & 1)] * f[6 + (c & 1)];
    };
    const float pk = corner(0);
    const float an = sm[Ly::A0 + s] + pk;
    A[(size_t)n * S + s] = an;
    const float inv = 1.f / (an + eps);
    sm[Ly::PK + s] = pk;
#pragma unroll
    for (int h = 0; h < WS; ++h) sm[Ly::W + s * WS + h] = h < group ? corner(1 + h) * inv : 0.f;
  }
  __syncthreads();
  // ---- B[s] += pk[s] v (to global) ; acc_h += W_h[s] B[s], row-chunk group by group
  float4 acc[MG];
#pragma unroll
  for (int h = 0; h < MG; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  {
    float4 *bout = reinterpret_cast<float4 *>(B + (size_t)n * S * D);
#pragma unroll
    for (int i = 0; i < RPW / 2; ++i) {
      if (i % RPB == 0) cp_async_wait_dyn<NB>(NB - 1 - i / RPB);  // this thread's copies of group i / RPB
      const int s = warp * RPW + 2 * i + half;
      float4 b = *reinterpret_cast<const float4 *>(sm + Ly::B0 + s * D + 4 * c4);
      const float pk = sm[Ly::PK + s];
      fma4(b, pk, vv);
      bout[s * (D / 4) + c4] = b;
#pragma unroll
      for (int h4 = 0; h4 < MG; h4 += 4) {
        const float4 w = *reinterpret_cast<const float4 *>(sm + Ly::W + s * WS + h4);
        const float ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4 && h4 + e < MG; ++e) fma4(acc[h4 + e], ws[e], b);
      }
    }
  }
  // ---- the two row parities (lane bit 4), then the warps
#pragma unroll
  for (int h = 0; h < MG; ++h) {
    if (h < group) {
      acc[h].x += __shfl_xor_sync(0xffffffffu, acc[h].x, 16);
      acc[h].y += __shfl_xor_sync(0xffffffffu, acc[h].y, 16);
      acc[h].z += __shfl_xor_sync(0xffffffffu, acc[h].z, 16);
      acc[h].w += __shfl_xor_sync(0xffffffffu, acc[h].w, 16);
      if (half == 0) *reinterpret_cast<float4 *>(sm + Ly::RED + (warp * MG + h) * D + 4 * c4) = acc[h];
    }
  }
  __syncthreads();
  for (int i = tid; i < MG * (D / 4); i += NT) {
    const int h = i / (D / 4), cc = i % (D / 4);
    if (h < group) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float4 pw = *reinterpret_cast<const float4 *>(sm + Ly::RED + (w * MG + h) * D + 4 * cc);
        o.x += pw.x;
        o.y += pw.y;
        o.z += pw.z;
        o.w += pw.w;
      }
      store4<XT>(out + ((size_t)n * group + h) * D + 4 * cc, o);
    }
  }
}
}  // namespace d64

__host__ __device__ __forceinline__ bool d64_eligible(int D, int L, int P, int group) {
  return D == 64 && P == 4 && (L == 8 || L == 16) && group >= 1 && group <= 8;
}

}  // namespace dec
}  // namespace race
