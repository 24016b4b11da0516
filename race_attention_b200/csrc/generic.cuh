// generic.cuh -- all-shapes SIMT path of the causal RACE operator.
//
// Covers every shape the reference accepts up to D <= 256 and S <= 1024, in
// fp32 arithmetic (it is the fp32 path, rel 1e-4 parity).  Structure: the time
// axis is cut into chunks of GC tokens; every chunk runs in parallel.
//
//   forward : totals (per chunk  A_c = sum pk,  B_c = sum pk (x) V)
//             -> exclusive scan over chunks (double accumulation, optional
//                carried-in state)  -> readout per chunk:
//                out = W @ B_start + tril(W @ Pk^T) @ V,
//                W[t,s] = pq[t,s] / (A_start[s] + cumsum_t pk[.,s] + eps)
//   backward: forward totals/scan again -> per chunk G = dO.B_t, dpq, dA and
//             chunk totals of (sum dA, sum W^T dO) -> reverse exclusive scan ->
//             per chunk dpk = gA + V.gB,  dV = Pk gB  (gA/gB = suffix states).
//
// State buffer layout, one record per (stream n, chunk g):
//   St[(n*G + g)*E + s]           = A part (s < S)
//   St[(n*G + g)*E + S + s*D + d] = B part
// with E = S + S*D.  The chunk-level scan is dictated by the math (prefix sums
// with a nonlinear per-bucket normaliser); the reference does the same at
// kernels/gpu/forward_kernel.cu:8-14 and kernels/gpu/backward_kernels.cu:4-21,
// but here each CTA owns a whole chunk x all buckets, reads every input once
// per chunk, never materialises [N,T,S] temporaries and writes each output
// element exactly once (no atomics, bitwise run-to-run deterministic).
#pragma once

#include "common.cuh"

namespace race {
namespace gen {

constexpr int GC = 32;   // tokens per chunk
constexpr int GST = 32;  // bucket tile
constexpr int NT = 256;  // threads per CTA
constexpr int MAX_D = 256;
constexpr int HT = 16;   // tokens per soft-hash CTA

struct Dims {
  int N, T, S, D, G;
  float eps;
};

__host__ __device__ __forceinline__ size_t state_elems(int S, int D) { return (size_t)S + (size_t)S * D; }

// ---------------------------------------------------------------------------
// chunk totals:  St[n,g] = ( sum_{t in g} pk[t,:],  sum_{t in g} pk[t,:] (x) V[t,:] )
// grid (G, N), dynamic smem: (GC*D + GC*GST) floats
template <typename VT>
__global__ void __launch_bounds__(NT) fwd_totals(const float *__restrict__ pk, const VT *__restrict__ V,
                                                 float *__restrict__ St, Dims p) {
  extern __shared__ float sm[];
  float *sV = sm;                 // [GC][D]
  float *sK = sV + GC * p.D;      // [GC][GST]
  const int g = blockIdx.x, n = blockIdx.y, tid = threadIdx.x;
  const int t0 = g * GC, nt = min(GC, p.T - t0);
  const size_t E = state_elems(p.S, p.D);
  float *st = St + ((size_t)n * p.G + g) * E;
  for (int i = tid; i < GC * p.D; i += NT) {
    const int t = i / p.D, d = i % p.D;
    sV[i] = t < nt ? to_f(V[((size_t)n * p.T + t0 + t) * p.D + d]) : 0.f;
  }
  for (int s0 = 0; s0 < p.S; s0 += GST) {
    const int ns = min(GST, p.S - s0);
    __syncthreads();
    for (int i = tid; i < GC * GST; i += NT) {
      const int t = i / GST, s = i % GST;
      sK[i] = (t < nt && s < ns) ? pk[((size_t)n * p.T + t0 + t) * p.S + s0 + s] : 0.f;
    }
    __syncthreads();
    for (int i = tid; i < ns * p.D; i += NT) {
      const int s = i / p.D, d = i % p.D;
      float acc = 0.f;
#pragma unroll 8
      for (int t = 0; t < GC; ++t) acc = fmaf(sK[t * GST + s], sV[t * p.D + d], acc);
      st[p.S + (size_t)(s0 + s) * p.D + d] = acc;
    }
    if (tid < ns) {
      float a = 0.f;
      for (int t = 0; t < GC; ++t) a += sK[t * GST + tid];
      st[s0 + tid] = a;
    }
  }
}

// ---------------------------------------------------------------------------
// in-place exclusive scan of the chunk records over g (forward or reverse),
// seeded with init (may be NULL), inclusive total written to fin (may be NULL).
// grid (ceil(E/256), N), block 256.  Running sums are kept in double.
static __global__ void chunk_scan(float *__restrict__ St, const float *__restrict__ initA,
                           const float *__restrict__ initB, float *__restrict__ finA,
                           float *__restrict__ finB, int N, int G, int S, int D, int reverse) {
  const size_t E = state_elems(S, D);
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int n = blockIdx.y;
  if (e >= E) return;
  double run = 0.0;
  const bool isA = e < (size_t)S;
  if (isA) {
    if (initA) run = initA[(size_t)n * S + e];
  } else if (initB) {
    run = initB[(size_t)n * S * D + (e - S)];
  }
  float *col = St + (size_t)n * G * E + e;
  if (!reverse) {
    for (int g = 0; g < G; ++g) {
      const float v = col[(size_t)g * E];
      col[(size_t)g * E] = (float)run;
      run += v;
    }
  } else {
    for (int g = G - 1; g >= 0; --g) {
      const float v = col[(size_t)g * E];
      col[(size_t)g * E] = (float)run;
      run += v;
    }
  }
  if (isA) {
    if (finA) finA[(size_t)n * S + e] = (float)run;
  } else if (finB) {
    finB[(size_t)n * S * D + (e - S)] = (float)run;
  }
}

// ---------------------------------------------------------------------------
// forward readout of one chunk from its exclusive-prefix state.
// grid (G, N), dynamic smem: see fwd_readout_smem()
__host__ __device__ __forceinline__ size_t fwd_readout_smem(int D) {
  return sizeof(float) * ((size_t)GC * D * 2 + (size_t)GST * D + 2 * GC * GST + GC * GC + GST);
}

template <typename VT, typename OT>
__global__ void __launch_bounds__(NT) fwd_readout(const float *__restrict__ pk, const float *__restrict__ pq,
                                                  const VT *__restrict__ V, const float *__restrict__ St,
                                                  OT *__restrict__ out, Dims p) {
  extern __shared__ float sm[];
  float *sV = sm;                    // [GC][D]
  float *sO = sV + GC * p.D;         // [GC][D]
  float *sB = sO + GC * p.D;         // [GST][D]
  float *sK = sB + GST * p.D;        // [GC][GST]
  float *sW = sK + GC * GST;         // [GC][GST]  pq, then W
  float *sSm = sW + GC * GST;        // [GC][GC]
  float *sA = sSm + GC * GC;         // [GST]
  const int g = blockIdx.x, n = blockIdx.y, tid = threadIdx.x;
  const int t0 = g * GC, nt = min(GC, p.T - t0);
  const size_t E = state_elems(p.S, p.D);
  const float *st = St + ((size_t)n * p.G + g) * E;
  for (int i = tid; i < GC * p.D; i += NT) {
    const int t = i / p.D, d = i % p.D;
    sV[i] = t < nt ? to_f(V[((size_t)n * p.T + t0 + t) * p.D + d]) : 0.f;
    sO[i] = 0.f;
  }
  for (int i = tid; i < GC * GC; i += NT) sSm[i] = 0.f;
  for (int s0 = 0; s0 < p.S; s0 += GST) {
    const int ns = min(GST, p.S - s0);
    __syncthreads();
    for (int i = tid; i < GC * GST; i += NT) {
      const int t = i / GST, s = i % GST;
      const bool ok = t < nt && s < ns;
      const size_t idx = ((size_t)n * p.T + t0 + t) * p.S + s0 + s;
      sK[i] = ok ? pk[idx] : 0.f;
      sW[i] = ok ? pq[idx] : 0.f;
    }
    for (int i = tid; i < GST * p.D; i += NT) {
      const int s = i / p.D;
      sB[i] = s < ns ? st[p.S + (size_t)s0 * p.D + i] : 0.f;
    }
    if (tid < GST) sA[tid] = tid < ns ? st[s0 + tid] : 0.f;
    __syncthreads();
    if (tid < ns) {
      float A = sA[tid];
      for (int t = 0; t < GC; ++t) {
        A += sK[t * GST + tid];
        sW[t * GST + tid] = sW[t * GST + tid] / (A + p.eps);
      }
    }
    __syncthreads();
    for (int i = tid; i < GC * GC; i += NT) {
      const int t = i / GC, tau = i % GC;
      if (tau <= t) {
        float acc = 0.f;
#pragma unroll 8
        for (int s = 0; s < GST; ++s) acc = fmaf(sW[t * GST + s], sK[tau * GST + s], acc);
        sSm[i] += acc;
      }
    }
    for (int i = tid; i < GC * p.D; i += NT) {
      const int t = i / p.D, d = i % p.D;
      float acc = 0.f;
#pragma unroll 8
      for (int s = 0; s < GST; ++s) acc = fmaf(sW[t * GST + s], sB[s * p.D + d], acc);
      sO[i] += acc;
    }
  }
  __syncthreads();
  for (int i = tid; i < nt * p.D; i += NT) {
    const int t = i / p.D, d = i % p.D;
    float acc = sO[i];
    for (int tau = 0; tau <= t; ++tau) acc = fmaf(sSm[t * GC + tau], sV[tau * p.D + d], acc);
    out[((size_t)n * p.T + t0 + t) * p.D + d] = from_f<OT>(acc);
  }
}

// ---------------------------------------------------------------------------
// backward, shared per-chunk front half: W, 1/(A+eps), G, dA for one bucket
// tile.  Writes sW (W), sInv, sG (= dA) for tile s0.
struct BwdSmem {
  float *sV, *sdO, *sB, *sP, *sK, *sW, *sInv, *sG, *sA;
};

__host__ __device__ __forceinline__ size_t bwd_smem_floats(int D, bool readout) {
  size_t f = (size_t)GC * D * 2 + (size_t)GST * D + GC * GC + 4 * GC * GST + GST;
  if (readout) f += (size_t)GC * GC + (size_t)GC * D + GST;
  return f;
}

__device__ __forceinline__ void bwd_tile_front(const BwdSmem &m, const float *__restrict__ pk,
                                               const float *__restrict__ pq, const float *st, int n,
                                               int t0, int nt, int s0, int ns, const Dims &p,
                                               float *__restrict__ dpq) {
  const int tid = threadIdx.x;
  __syncthreads();
  for (int i = tid; i < GC * GST; i += NT) {
    const int t = i / GST, s = i % GST;
    const bool ok = t < nt && s < ns;
    const size_t idx = ((size_t)n * p.T + t0 + t) * p.S + s0 + s;
    m.sK[i] = ok ? pk[idx] : 0.f;
    m.sW[i] = ok ? pq[idx] : 0.f;
  }
  for (int i = tid; i < GST * p.D; i += NT) {
    const int s = i / p.D;
    m.sB[i] = s < ns ? st[p.S + (size_t)s0 * p.D + i] : 0.f;
  }
  if (tid < GST) m.sA[tid] = tid < ns ? st[s0 + tid] : 0.f;
  __syncthreads();
  if (tid < GST) {
    float A = m.sA[tid];
    for (int t = 0; t < GC; ++t) {
      A += m.sK[t * GST + tid];
      const float inv = 1.f / (A + p.eps);
      m.sInv[t * GST + tid] = inv;
      m.sW[t * GST + tid] *= inv;
    }
  }
  __syncthreads();
  for (int i = tid; i < GC * GST; i += NT) {
    const int t = i / GST, s = i % GST;
    float gsum = 0.f;
    for (int tau = 0; tau <= t; ++tau) gsum = fmaf(m.sP[t * GC + tau], m.sK[tau * GST + s], gsum);
#pragma unroll 8
    for (int d = 0; d < p.D; ++d) gsum = fmaf(m.sdO[t * p.D + d], m.sB[s * p.D + d], gsum);
    const float inv = m.sInv[i];
    if (dpq && t < nt && s < ns) dpq[((size_t)n * p.T + t0 + t) * p.S + s0 + s] = gsum * inv;
    m.sG[i] = -m.sW[i] * inv * gsum;
  }
  __syncthreads();
}

template <typename VT>
__device__ __forceinline__ void bwd_load_chunk(const BwdSmem &m, const VT *__restrict__ V,
                                               const VT *__restrict__ dO, int n, int t0, int nt,
                                               const Dims &p) {
  const int tid = threadIdx.x;
  for (int i = tid; i < GC * p.D; i += NT) {
    const int t = i / p.D, d = i % p.D;
    const size_t idx = ((size_t)n * p.T + t0 + t) * p.D + d;
    m.sV[i] = t < nt ? to_f(V[idx]) : 0.f;
    m.sdO[i] = t < nt ? to_f(dO[idx]) : 0.f;
  }
  __syncthreads();
  // P[t][tau] = dO_t . V_tau  (full square; masks applied by the users)
  for (int i = tid; i < GC * GC; i += NT) {
    const int t = i / GC, tau = i % GC;
    float acc = 0.f;
#pragma unroll 8
    for (int d = 0; d < p.D; ++d) acc = fmaf(m.sdO[t * p.D + d], m.sV[tau * p.D + d], acc);
    m.sP[i] = acc;
  }
}

__device__ __forceinline__ BwdSmem bwd_carve(float *sm, int D) {
  BwdSmem m;
  m.sV = sm;
  m.sdO = m.sV + GC * D;
  m.sB = m.sdO + GC * D;
  m.sP = m.sB + GST * D;
  m.sK = m.sP + GC * GC;
  m.sW = m.sK + GC * GST;
  m.sInv = m.sW + GC * GST;
  m.sG = m.sInv + GC * GST;
  m.sA = m.sG + GC * GST;
  return m;
}

// per chunk: dpq (optional) and the chunk totals of (sum_t dA_t, sum_t W_t (x) dO_t)
// grid (G, N), dynamic smem bwd_smem_floats(D,false)*4
template <typename VT>
__global__ void __launch_bounds__(NT) bwd_totals(const float *__restrict__ pk, const float *__restrict__ pq,
                                                 const VT *__restrict__ V, const VT *__restrict__ dO,
                                                 const float *__restrict__ St, float *__restrict__ St2,
                                                 float *__restrict__ dpq, Dims p) {
  extern __shared__ float sm[];
  const BwdSmem m = bwd_carve(sm, p.D);
  const int g = blockIdx.x, n = blockIdx.y, tid = threadIdx.x;
  const int t0 = g * GC, nt = min(GC, p.T - t0);
  const size_t E = state_elems(p.S, p.D);
  const float *st = St + ((size_t)n * p.G + g) * E;
  float *st2 = St2 + ((size_t)n * p.G + g) * E;
  bwd_load_chunk(m, V, dO, n, t0, nt, p);
  for (int s0 = 0; s0 < p.S; s0 += GST) {
    const int ns = min(GST, p.S - s0);
    bwd_tile_front(m, pk, pq, st, n, t0, nt, s0, ns, p, dpq);
    if (tid < ns) {
      float a = 0.f;
      for (int t = 0; t < GC; ++t) a += m.sG[t * GST + tid];
      st2[s0 + tid] = a;
    }
    for (int i = tid; i < ns * p.D; i += NT) {
      const int s = i / p.D, d = i % p.D;
      float acc = 0.f;
#pragma unroll 8
      for (int t = 0; t < GC; ++t) acc = fmaf(m.sW[t * GST + s], m.sdO[t * p.D + d], acc);
      st2[p.S + (size_t)(s0 + s) * p.D + d] = acc;
    }
  }
}

// per chunk: dpk and dV from forward prefix states St and backward suffix states St2.
// grid (G, N), dynamic smem bwd_smem_floats(D,true)*4
template <typename VT, typename OT>
__global__ void __launch_bounds__(NT) bwd_readout(const float *__restrict__ pk, const float *__restrict__ pq,
                                                  const VT *__restrict__ V, const VT *__restrict__ dO,
                                                  const float *__restrict__ St, const float *__restrict__ St2,
                                                  float *__restrict__ dpk, OT *__restrict__ dV, Dims p) {
  extern __shared__ float sm[];
  const BwdSmem m = bwd_carve(sm, p.D);
  float *sQ2 = m.sA + GST;            // [GC][GC]  sum_s pk[tau,s] W[t,s]
  float *sdV = sQ2 + GC * GC;         // [GC][D]
  float *sgA = sdV + GC * p.D;        // [GST]
  const int g = blockIdx.x, n = blockIdx.y, tid = threadIdx.x;
  const int t0 = g * GC, nt = min(GC, p.T - t0);
  const size_t E = state_elems(p.S, p.D);
  const float *st = St + ((size_t)n * p.G + g) * E;
  const float *st2 = St2 + ((size_t)n * p.G + g) * E;
  for (int i = tid; i < GC * GC; i += NT) sQ2[i] = 0.f;
  for (int i = tid; i < GC * p.D; i += NT) sdV[i] = 0.f;
  bwd_load_chunk(m, V, dO, n, t0, nt, p);
  for (int s0 = 0; s0 < p.S; s0 += GST) {
    const int ns = min(GST, p.S - s0);
    bwd_tile_front(m, pk, pq, st, n, t0, nt, s0, ns, p, nullptr);
    // suffix state of this tile replaces the forward state in sB
    for (int i = tid; i < GST * p.D; i += NT) {
      const int s = i / p.D;
      m.sB[i] = s < ns ? st2[p.S + (size_t)s0 * p.D + i] : 0.f;
    }
    if (tid < GST) sgA[tid] = tid < ns ? st2[s0 + tid] : 0.f;
    __syncthreads();
    if (tid < GST) {  // gA_tau = gA_suffix + sum_{t >= tau} dA_t   (in place over sG)
      float ga = sgA[tid];
      for (int t = GC - 1; t >= 0; --t) {
        ga += m.sG[t * GST + tid];
        m.sG[t * GST + tid] = ga;
      }
    }
    __syncthreads();
    for (int i = tid; i < GC * GST; i += NT) {
      const int tau = i / GST, s = i % GST;
      float v = m.sG[i];
#pragma unroll 8
      for (int d = 0; d < p.D; ++d) v = fmaf(m.sV[tau * p.D + d], m.sB[s * p.D + d], v);
      for (int t = tau; t < GC; ++t) v = fmaf(m.sP[t * GC + tau], m.sW[t * GST + s], v);
      if (tau < nt && s < ns) dpk[((size_t)n * p.T + t0 + tau) * p.S + s0 + s] = v;
    }
    for (int i = tid; i < GC * GC; i += NT) {
      const int tau = i / GC, t = i % GC;
      if (t >= tau) {
        float acc = 0.f;
#pragma unroll 8
        for (int s = 0; s < GST; ++s) acc = fmaf(m.sK[tau * GST + s], m.sW[t * GST + s], acc);
        sQ2[i] += acc;
      }
    }
    for (int i = tid; i < GC * p.D; i += NT) {
      const int tau = i / p.D, d = i % p.D;
      float acc = 0.f;
#pragma unroll 8
      for (int s = 0; s < GST; ++s) acc = fmaf(m.sK[tau * GST + s], m.sB[s * p.D + d], acc);
      sdV[i] += acc;
    }
  }
  __syncthreads();
  for (int i = tid; i < nt * p.D; i += NT) {
    const int tau = i / p.D, d = i % p.D;
    float acc = sdV[i];
    for (int t = tau; t < GC; ++t) acc = fmaf(sQ2[tau * GC + t], m.sdO[t * p.D + d], acc);
    dV[((size_t)n * p.T + t0 + tau) * p.D + d] = from_f<OT>(acc);
  }
}

// ---------------------------------------------------------------------------
// soft hash: probs[row, l*R+r] = softmax_r( sum_p tanh(x.planes[:,l*P+p]) * scale * sign(p,r) )
// grid ceil(rows/HT), dynamic smem (HT*D + HT*LP) floats
template <typename XT>
__global__ void __launch_bounds__(NT) soft_hash_fwd(const XT *__restrict__ X, const float *__restrict__ planes_T,
                                                    float *__restrict__ probs, long rows, int D, int L,
                                                    int P, float scale) {
  extern __shared__ float sm[];
  const int LP = L * P, R = 1 << P, S = L * R;
  float *sX = sm;             // [HT][D]
  float *sA = sX + HT * D;    // [HT][LP]
  const long r0 = (long)blockIdx.x * HT;
  const int nr = (int)min((long)HT, rows - r0);
  const int tid = threadIdx.x;
  for (int i = tid; i < HT * D; i += NT) {
    const int r = i / D;
    sX[i] = r < nr ? to_f(X[(r0 + r) * D + (i % D)]) : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < HT * LP; i += NT) {
    const int r = i / LP, j = i % LP;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(sX[r * D + d], planes_T[(size_t)d * LP + j], acc);
    sA[i] = tanhf(acc) * scale;
  }
  __syncthreads();
  for (int i = tid; i < HT * L; i += NT) {
    const int r = i / L, l = i % L;
    if (r >= nr) continue;
    const float *a = sA + r * LP + l * P;
    float mx = -INFINITY;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(a[q], corner_sign(c, q, P), v);
      mx = fmaxf(mx, v);
    }
    float z = 0.f;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(a[q], corner_sign(c, q, P), v);
      z += expf(v - mx);
    }
    const float iz = 1.f / z;
    float *out = probs + (r0 + r) * (long)S + l * R;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(a[q], corner_sign(c, q, P), v);
      out[c] = expf(v - mx) * iz;
    }
  }
}

// dX = d<dprobs, soft_hash(X)>/dX.  dynamic smem (HT*D + 2*HT*LP) floats
template <typename XT>
__global__ void __launch_bounds__(NT) soft_hash_bwd(const XT *__restrict__ X, const float *__restrict__ planes_T,
                                                    const float *__restrict__ dprobs, XT *__restrict__ dX,
                                                    long rows, int D, int L, int P, float scale) {
  extern __shared__ float sm[];
  const int LP = L * P, R = 1 << P, S = L * R;
  float *sX = sm;              // [HT][D]
  float *sT = sX + HT * D;     // [HT][LP]  tanh(proj)
  float *sG = sT + HT * LP;    // [HT][LP]  d proj
  const long r0 = (long)blockIdx.x * HT;
  const int nr = (int)min((long)HT, rows - r0);
  const int tid = threadIdx.x;
  for (int i = tid; i < HT * D; i += NT) {
    const int r = i / D;
    sX[i] = r < nr ? to_f(X[(r0 + r) * D + (i % D)]) : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < HT * LP; i += NT) {
    const int r = i / LP, j = i % LP;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(sX[r * D + d], planes_T[(size_t)d * LP + j], acc);
    sT[i] = tanhf(acc);
  }
  __syncthreads();
  for (int i = tid; i < HT * L; i += NT) {
    const int r = i / L, l = i % L;
    float *gp = sG + r * LP + l * P;
    if (r >= nr) {
      for (int q = 0; q < P; ++q) gp[q] = 0.f;
      continue;
    }
    const float *th = sT + r * LP + l * P;
    const float *g = dprobs + (r0 + r) * (long)S + l * R;
    float mx = -INFINITY;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(th[q] * scale, corner_sign(c, q, P), v);
      mx = fmaxf(mx, v);
    }
    float z = 0.f, cz = 0.f;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(th[q] * scale, corner_sign(c, q, P), v);
      const float e = expf(v - mx);
      z += e;
      cz += e * g[c];
    }
    const float iz = 1.f / z, c0 = cz * iz;
    float da[16];
    for (int q = 0; q < P; ++q) da[q] = 0.f;
    for (int c = 0; c < R; ++c) {
      float v = 0.f;
      for (int q = 0; q < P; ++q) v = fmaf(th[q] * scale, corner_sign(c, q, P), v);
      const float dl = expf(v - mx) * iz * (g[c] - c0);
      for (int q = 0; q < P; ++q) da[q] = fmaf(dl, corner_sign(c, q, P), da[q]);
    }
    for (int q = 0; q < P; ++q) gp[q] = da[q] * scale * (1.f - th[q] * th[q]);
  }
  __syncthreads();
  for (int i = tid; i < nr * D; i += NT) {
    const int r = i / D, d = i % D;
    float acc = 0.f;
    for (int j = 0; j < LP; ++j) acc = fmaf(sG[r * LP + j], planes_T[(size_t)d * LP + j], acc);
    dX[(r0 + r) * D + d] = from_f<XT>(acc);
  }
}

}  // namespace gen
}  // namespace race
