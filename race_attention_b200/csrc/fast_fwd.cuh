// fast_fwd.cuh -- fused tcgen05 forward for bf16, D = 64, P = 4, S in {128, 256}.
//
// One CTA walks one (stream n, segment) -- a contiguous run of 128-token
// chunks -- carrying the bucket state on chip:
//   Bstate[s, :]  fp32 in TMEM (lanes = buckets of a 128-bucket group),
//   A_start[s]    fp32 in shared memory.
// Per chunk (all MMAs tcgen05 kind::f16, bf16 operands, fp32 accumulation):
//   projK/projQ  = K/Q tile [128 x 64] x planes^T [64 x L*P]          (TMEM)
//   per bucket group g (128 buckets = 8 tables):
//     Pk_g       = soft hash of projK (epilogue warps, factorised: the
//                  softmax over the 16 corners of a table is the product of
//                  4 per-plane sigmoids)                                (smem bf16)
//     Apref_g    = tril(1) x Pk_g      -> A_t = A_start + Apref         (TMEM)
//     W_g        = pq / (A_t + eps)                                     (smem bf16)
//     Smat_g     = W_g x Pk_g^T ;  out (+)= W_g x bf16(Bstate_g)        (TMEM)
//     Smask_g    = tril(Smat_g)                                         (smem bf16)
//     out       += Smask_g x V ;  Bstate_g += Pk_g^T x V                (TMEM)
//   out -> bf16 -> HBM.
// The segment-start state comes from fast_totals (one pass over K, V) and the
// chunk_scan over segments.  Q, K, V tiles arrive by TMA (3-D maps [N][T][64],
// 128B swizzle; rows past T read as zero).  Every wait on an mbarrier is
// bounded: on expiry the CTA raises *err, skips the rest of its work, frees its
// TMEM and returns.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace race {
namespace fast {

constexpr int C = 128;             // tokens per chunk (MMA M)
constexpr int HD = 64;             // head dim
constexpr int GB = 128;            // buckets per group
constexpr int NEPI = 16;           // epilogue warps (4 per TMEM lane quarter, one column quarter each)
constexpr int NTHR = (NEPI + 1) * 32;
constexpr int NARR = NEPI;        // arrivals that complete an epilogue barrier (one per warp)
constexpr int NEPI_T = NEPI * 32;
constexpr uint32_t TILE = C * 128;  // one [128 x 64] bf16 tile = 16 KB

// TMEM column map of the forward kernel (512 columns allocated)
constexpr uint32_t T_PK = 0, T_PQ = 64, T_G = 128, T_OUT = 256, T_B = 320;

// Activations (Q, K, V, out; dO, dQ, dK, dV) are [B, T, H, 64] bf16 with N = B H streams,
// stream n = b H + h: H = 1 is the [N, T, 64] layout, H = heads the [B, T, H, 64] layout
// attention modules produce.  TMA reads and writes them through 4-D maps (64, H, T, B),
// box (64, 1, 128, 1); act_row gives the element offset of token t of stream (b, h) for
// plain loads/stores.
__host__ __device__ __forceinline__ size_t act_row(int b, int h, int t, int T, int H) {
  return ((size_t)b * T + t) * H * 64 + (size_t)h * 64;
}

struct FwdArgs {
  int N, T, L, LP, S, ngroups;
  int H;                  // heads of the activation layout (see act_row)
  int nseg, seg_chunks, nchunks;  // chunks per segment; total chunks per stream
  float eps, scale;
  int poly;               // plane sigmoids by series (2|scale| <= 1/2)
  int batch_rcp;          // reciprocals of A + eps four at a time (eps >= 1e-8)
  const float *planes;    // [64, LP] fp32
  const float *seg_state;  // [N, nseg, S + S*64]  (A part, then B part) exclusive segment prefixes
  float *seg_tot;          // totals kernel output, same layout
  __nv_bfloat16 *out;      // [N, T, 64]
  float *chunkA;           // states pass of the totals kernel, or a forward that saves them for the
  __nv_bfloat16 *chunkB;   // backward: [N, nchunks, S] A + eps and [N, nchunks, S, 64] bf16 B at each
                           // chunk start (nullptr: not wanted)
  const float *seedA;      // readout of a sequence shard: the earlier shards' state ([N,S], [N,S,64])
  const float *seedB;      // added to every segment's prefix (nullptr: none)
  int *err;
  uint32_t wait_limit;     // polls before a bounded wait gives up (tc::kDefaultWaitPolls unless set)
  int withhold_first_load;  // test hook: issue no tile load for the first chunk, so the first waits
                            // expire with nothing in flight (the call then reports a timeout)
};

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs: sm_100 issues one FFMA2 / FMUL2 / FADD2 for two independent
// lanes of element-wise work, halving the epilogues' arithmetic instruction count
// (round-to-nearest on each lane: bit-identical to the scalar operations)
__device__ __forceinline__ float2 ld2(const float *v, int i) { return make_float2(v[i], v[i + 1]); }
__device__ __forceinline__ void st2(float *v, int i, float2 x) {
  v[i] = x.x;
  v[i + 1] = x.y;
}
__device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }
// a[i] += b[i], a[i] *= b[i] for n (even) values
template <int n>
__device__ __forceinline__ void vadd(float *a, const float *b) {
#pragma unroll
  for (int i = 0; i < n; i += 2) st2(a, i, __fadd2_rn(ld2(a, i), ld2(b, i)));
}
template <int n>
__device__ __forceinline__ void vmul(float *a, const float *b) {
#pragma unroll
  for (int i = 0; i < n; i += 2) st2(a, i, __fmul2_rn(ld2(a, i), ld2(b, i)));
}

// q_p = sigma(z_p), z_p = 2 * scale * tanh(proj_p), of one table's 4 planes, from
// th = tanh(proj).  `poly` (host-chosen: 2|scale| <= 1/2, which bounds |z| since
// |tanh| <= 1) selects sigma(z) = (1 + tanh(z/2)) / 2 with the odd Taylor series
// tanh(w) = w - w^3/3 + 2w^5/15 - 17w^7/315 + 62w^9/2835 - ... truncated after w^9
// (|w| <= 1/4: truncation error < 3e-9): FMA-pipe operations on pairs of planes
// instead of an exponential and a reciprocal on the SFU; otherwise the SFU exponential.
__device__ __forceinline__ void plane_sigmoids(const float *th4, float scale, bool poly, float *q4) {
  if (poly) {
    const float2 c9 = dup2(62.f / 2835.f), c7 = dup2(-17.f / 315.f), c5 = dup2(2.f / 15.f), c3 = dup2(-1.f / 3.f);
    const float2 one = dup2(1.f), half = dup2(0.5f), sc = dup2(scale);
#pragma unroll
    for (int p = 0; p < 4; p += 2) {
      const float2 w = __fmul2_rn(sc, ld2(th4, p)), w2 = __fmul2_rn(w, w);
      float2 q = __ffma2_rn(w2, c9, c7);
      q = __ffma2_rn(q, w2, c5);
      q = __ffma2_rn(q, w2, c3);
      q = __ffma2_rn(q, w2, one);
      st2(q4, p, __ffma2_rn(__fmul2_rn(half, w), q, half));
    }
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) q4[p] = __fdividef(1.f, 1.f + __expf(-2.f * scale * th4[p]));
  }
}

// probabilities of the 16 corners of one table from its 4 plane sigmoids
// (corner r: bit (3-p) of r selects sigma(+2a_p) vs sigma(-2a_p))
__device__ __forceinline__ void corner_probs(const float *q, float *p16) {
  float x[4], y[8];
#pragma unroll
  for (int b0 = 0; b0 < 2; ++b0)
#pragma unroll
    for (int b1 = 0; b1 < 2; ++b1) x[b0 * 2 + b1] = (b0 ? q[0] : 1.f - q[0]) * (b1 ? q[1] : 1.f - q[1]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    y[2 * i] = x[i] * (1.f - q[2]);
    y[2 * i + 1] = x[i] * q[2];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    p16[2 * i] = y[i] * (1.f - q[3]);
    p16[2 * i + 1] = y[i] * q[3];
  }
}

// corner_probs of two tables at once, table a in the low lane and table b in the high
// lane of each packed pair (the same products in the same order: bit-identical)
__device__ __forceinline__ void corner_probs2(const float *qa, const float *qb, float *pa, float *pb) {
  float2 q[4], nq[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    q[p] = make_float2(qa[p], qb[p]);
    nq[p] = __ffma2_rn(q[p], dup2(-1.f), dup2(1.f));  // 1 - q
  }
  float2 x[4], y[8];
#pragma unroll
  for (int b0 = 0; b0 < 2; ++b0)
#pragma unroll
    for (int b1 = 0; b1 < 2; ++b1) x[b0 * 2 + b1] = __fmul2_rn(b0 ? q[0] : nq[0], b1 ? q[1] : nq[1]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    y[2 * i] = __fmul2_rn(x[i], nq[2]);
    y[2 * i + 1] = __fmul2_rn(x[i], q[2]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 lo = __fmul2_rn(y[i], nq[3]), hi = __fmul2_rn(y[i], q[3]);
    pa[2 * i] = lo.x;
    pb[2 * i] = lo.y;
    pa[2 * i + 1] = hi.x;
    pb[2 * i + 1] = hi.y;
  }
}

// corner probabilities of one table straight from its 4 raw projections
__device__ __forceinline__ void table_probs(const float *proj4, float scale, bool poly, float *p16) {
  float th[4], q[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) th[p] = tanh_fast(proj4[p]);
  plane_sigmoids(th, scale, poly, q);
  corner_probs(q, p16);
}

// table_probs of two tables (4 projections each), paired as in corner_probs2
__device__ __forceinline__ void table_probs2(const float *proj_a, const float *proj_b, float scale, bool poly,
                                             float *pa, float *pb) {
  float th[8], q[8];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    th[p] = tanh_fast(proj_a[p]);
    th[4 + p] = tanh_fast(proj_b[p]);
  }
  plane_sigmoids(th, scale, poly, q);
  plane_sigmoids(th + 4, scale, poly, q + 4);
  corner_probs2(q, q + 4, pa, pb);
}

// Reciprocals of 4 values with one SFU operation (Montgomery's simultaneous
// inversion: 1/x_i from 1/(x0 x1 x2 x3) and the partial products).  Needs the
// product to be a normal float: callers use it for x = A + eps with
// eps >= 1e-8 and A < 2^31 (host flag `batch_rcp`), else one reciprocal each.
__device__ __forceinline__ void rcp4(const float *x, float *r) {  // r may alias x
  const float x0 = x[0], x1 = x[1], x2 = x[2], x3 = x[3];
  const float x01 = x0 * x1, x012 = x01 * x2;
  float inv = __fdividef(1.f, x012 * x3);
  r[3] = inv * x012;
  inv *= x3;
  r[2] = inv * x01;
  inv *= x2;
  r[1] = inv * x0;
  r[0] = inv * x1;
}

// r[i] = 1 / x[i] for n (a multiple of 4) values
template <int n>
__device__ __forceinline__ void rcp_n(const float *x, float *r, bool batch) {
  if (batch) {
#pragma unroll
    for (int i = 0; i < n; i += 4) rcp4(x + i, r + i);
  } else {
#pragma unroll
    for (int i = 0; i < n; ++i) r[i] = __fdividef(1.f, x[i]);
  }
}

// den[i] += A[i] for n (a multiple of 4) consecutive floats of a shared array
template <int n>
__device__ __forceinline__ void add_shared_row(uint32_t addr, float *den) {
#pragma unroll
  for (int i = 0; i < n; i += 4) {
    const float4 v = tc::ld_shared_f4(addr + 4 * i);
    st2(den, i, __fadd2_rn(ld2(den, i), make_float2(v.x, v.y)));
    st2(den, i + 2, __fadd2_rn(ld2(den, i + 2), make_float2(v.z, v.w)));
  }
}

// v[i] = A[i] for n (a multiple of 4) consecutive floats of a shared array
template <int n>
__device__ __forceinline__ void load_shared_row(uint32_t addr, float *v) {
#pragma unroll
  for (int i = 0; i < n; i += 4) {
    const float4 x = tc::ld_shared_f4(addr + 4 * i);
    v[i] = x.x;
    v[i + 1] = x.y;
    v[i + 2] = x.z;
    v[i + 3] = x.w;
  }
}

template <int n>
__device__ __forceinline__ void store_shared_row(uint32_t addr, const float *v) {
#pragma unroll
  for (int i = 0; i < n; i += 4) tc::st_shared_f4(addr + 4 * i, make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
}

// --------------------------------------------------------------------------
// shared-memory plan (byte offsets from a 1024-aligned base)
struct FwdSmem {
  uint32_t q, k, v, pk, w, bst, tril, planes, a0, a1, bars, total;  // v: 2 stages of TILE bytes
};

__host__ __device__ __forceinline__ FwdSmem fwd_smem_plan(int ngroups, int LP) {
  FwdSmem m;
  uint32_t o = 0;
  m.q = o; o += TILE;
  m.k = o; o += TILE;
  m.v = o; o += 2 * TILE;
  m.pk = o; o += 2 * TILE;
  m.w = o; o += 2 * TILE;
  m.bst = o; o += (uint32_t)ngroups * TILE;
  m.tril = o; o += 2 * TILE;
  m.planes = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.a0 = o; o += 1024;
  m.a1 = o; o += 1024;
  m.bars = o; o += 256;
  m.total = o + 1024;  // + alignment slack
  return m;
}

// mbarrier slots (TMA and MMA completions) and named barriers (epilogue -> MMA issuer)
enum { B_QK = 0, B_V0, B_V1, B_PROJ, B_APREF, B_SMAT, B_GDONE, B_FINAL, B_COUNT };
enum { NB_INIT = 1, NB_PK, NB_W, NB_SMASK, NB_ESYNC };

// Schedule (u = chunk * ngroups + group).  The control warp issues, per group,
//   {PK}    Apref = tril Pk          -> APREF ;  Bstate_g += Pk^T V
//   {W}     Smat = W Pk^T ; out (+)= W bf16(Bstate_g at chunk start) -> SMAT
//           (after the chunk's last W: proj of the next chunk -> PROJ)
//   {SMASK} out += Smask V           -> GDONE
// while the epilogue warps, per group, do
//   Pk {PK} ; pq (overlaps Apref) ; [APREF] W {W} ;
//   bf16 refresh of the previous group's Bstate (overlaps Smat) ;
//   [SMAT] Smask {SMASK} ; (next group's Pk overlaps Smask V)
// and read out after the chunk's last GDONE.  {X}: the epilogue warps arrive
// on named barrier X (bar.arrive), the control warp waits on it (bar.sync);
// [X]: mbarrier signalled by tcgen05.commit.  A Bstate refresh and the out
// readout precede the epilogue's next {W} arrival, which is what orders them
// before the MMAs that overwrite their sources.  Q/K are single-buffered (the
// next chunk's tiles load while this chunk's groups run), V double-buffered.
// Abort: a bounded wait that gives up raises *abort; from then on no thread
// waits or works, but every thread still takes every named-barrier step, so
// no bar.sync can be left without its arrivals.
__global__ void __launch_bounds__(NTHR, 1) fwd_readout_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                              const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = (unsigned char *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  const FwdSmem P = fwd_smem_plan(a.ngroups, a.LP);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bars);
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort[2];  // wait control: abort flag, poll limit
  const uint32_t sbase = tc::smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x / a.nseg, seg = blockIdx.x % a.nseg;
  const int hn = n % a.H, bn = n / a.H;  // head and batch of stream n in the activation layout
  const int c_begin = seg * a.seg_chunks;
  const int c_end = min(a.nchunks, c_begin + a.seg_chunks);
  const int nch = c_end - c_begin;
  const int S = a.S, NG = a.ngroups;
  const size_t E = (size_t)S + (size_t)S * HD;
  const float *state0 = a.seg_state + ((size_t)n * a.nseg + seg) * E;

  if (threadIdx.x == 0) {
    s_abort[0] = 0;
    s_abort[1] = (int)a.wait_limit;
    for (int i = 0; i < B_COUNT; ++i) tc::mbar_init(&bars[i], 1);
    tc::fence_mbar_init();
  }
  if (warp == NEPI) tc::tmem_alloc(&s_tmem, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int *abort = s_abort;

  if (warp == NEPI) {
    // ===================== control warp: named-barrier steps as a warp, TMA + MMA issue by lane 0
    const bool leader = lane == 0;
    const uint32_t oq = P.q, ok_ = P.k, ov = P.v;
    auto load_qk = [=, &tmQ, &tmK](int c) {
      const int t0 = (c_begin + c) * C;
      tc::mbar_arrive_expect_tx(&bars[B_QK], 2 * TILE);
      tc::tma_load_4d(sm + oq, &tmQ, &bars[B_QK], 0, hn, t0, bn);
      tc::tma_load_4d(sm + ok_, &tmK, &bars[B_QK], 0, hn, t0, bn);
    };
    auto load_v = [=, &tmV](int c) {
      const int st = c & 1;
      tc::mbar_arrive_expect_tx(&bars[B_V0 + st], TILE);
      tc::tma_load_4d(sm + ov + st * TILE, &tmV, &bars[B_V0 + st], 0, hn, (c_begin + c) * C, bn);
    };
    const uint32_t id_proj = tc::idesc_bf16(C, a.LP, false, false);
    const uint32_t id_apref = tc::idesc_bf16(C, GB, false, true);
    const uint32_t id_smat = tc::idesc_bf16(C, C, false, false);
    const uint32_t id_out = tc::idesc_bf16(C, HD, false, true);
    const uint32_t id_bupd = tc::idesc_bf16(GB, HD, true, true);
    auto issue_proj = [=]() {
#pragma unroll
      for (int k0 = 0; k0 < HD; k0 += 16) {
        const uint64_t bp = tc::desc_kmajor(sbase + P.planes, k0, 0);
        tc::mma_bf16(tmem + T_PK, tc::desc_kmajor(sbase + P.k, k0, 0), bp, id_proj, k0 > 0);
        tc::mma_bf16(tmem + T_PQ, tc::desc_kmajor(sbase + P.q, k0, 0), bp, id_proj, k0 > 0);
      }
      tc::mma_commit(&bars[B_PROJ]);
    };
    bool ok = true;
    if (leader && nch > 0 && !a.withhold_first_load) {
      tc::prefetch_tmap(&tmQ);
      tc::prefetch_tmap(&tmK);
      tc::prefetch_tmap(&tmV);
      load_qk(0);
      load_v(0);
    }
    // the epilogue prologue (planes, tril, A/B state) is in smem past this point
    tc::named_bar_sync(NB_INIT, NTHR);
    if (leader && nch > 0) {
      ok = tc::mbar_wait(&bars[B_QK], 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_proj();
      }
    }
    for (int c = 0; c < nch; ++c) {
      const uint32_t vt = sbase + P.v + (uint32_t)(c & 1) * TILE;
      for (int g = 0; g < NG; ++g) {
        tc::named_bar_sync(NB_PK, NTHR);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + T_G, tc::desc_kmajor(sbase + P.tril, k0, TILE),
                         tc::desc_mnmajor(sbase + P.pk, k0, TILE), id_apref, k0 > 0);
          tc::mma_commit(&bars[B_APREF]);
          if (g == 0) {
            // Pk(0) implies the epilogue saw this chunk's proj complete and the
            // previous chunk's last MMA done: refill Q/K and the other V stage
            if (c + 1 < nch) {
              load_qk(c + 1);
              load_v(c + 1);
            }
            ok = tc::mbar_wait(&bars[B_V0 + (c & 1)], (c >> 1) & 1, abort);
          }
          if (ok) {
            tc::tc_fence_after();
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16)
              tc::mma_bf16(tmem + T_B + 64 * g, tc::desc_mnmajor(sbase + P.pk, k0, TILE),
                           tc::desc_mnmajor(vt, k0, TILE), id_bupd, true);
          }
        }
        tc::named_bar_sync(NB_W, NTHR);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
          const uint32_t bst = sbase + P.bst + (uint32_t)g * TILE;
#pragma unroll
          for (int k0 = 0; k0 < GB; k0 += 16) {
            const uint64_t aw = tc::desc_kmajor(sbase + P.w, k0, TILE);
            tc::mma_bf16(tmem + T_G, aw, tc::desc_kmajor(sbase + P.pk, k0, TILE), id_smat, k0 > 0);
            tc::mma_bf16(tmem + T_OUT, aw, tc::desc_mnmajor(bst, k0, TILE), id_out, g > 0 || k0 > 0);
          }
          tc::mma_commit(&bars[B_SMAT]);
          if (g == NG - 1 && c + 1 < nch) {
            // every reader of proj (Pk and W phases) is done: next chunk's proj
            ok = tc::mbar_wait(&bars[B_QK], (c + 1) & 1, abort);
            if (ok) {
              tc::tc_fence_after();
              issue_proj();
            }
          }
        }
        tc::named_bar_sync(NB_SMASK, NTHR);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + T_OUT, tc::desc_kmajor(sbase + P.w, k0, TILE), tc::desc_mnmajor(vt, k0, TILE), id_out,
                         true);
          tc::mma_commit(&bars[B_GDONE]);
        }
      }
    }
    if (leader && nch > 0) {
      // drain: every MMA this thread issued has completed before TMEM is freed
      tc::mma_commit(&bars[B_FINAL]);
      if (!tc::mbar_wait_drain(&bars[B_FINAL], 0)) atomicExch(a.err, 2);
    }
    __syncwarp();
  } else {
    // ===================== epilogue warps: row t of the chunk, column quarter hq
    const int q4 = warp & 3, hq = warp >> 2;
    const int t = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t blk = (uint32_t)(hq >> 1) * TILE;  // 64-column block holding this quarter's 32 columns
    const int ch0 = (hq & 1) * 4;                      // its first 16-byte chunk inside that block
    float *const sA0 = reinterpret_cast<float *>(sm + P.a0);
    // chunk-start state for the backward (when saving): B of group gr at chunk cc, this
    // thread's bucket row and d in [16hq, 16hq+16), bf16
    auto save_b = [=](int cc, int gr, const float *v16) {
      __nv_bfloat16 *dst = a.chunkB + (((size_t)n * a.nchunks + cc) * S + gr * GB + t) * HD + 16 * hq;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint4 w4;
        w4.x = tc::pack_bf16(v16[8 * ch + 0], v16[8 * ch + 1]);
        w4.y = tc::pack_bf16(v16[8 * ch + 2], v16[8 * ch + 3]);
        w4.z = tc::pack_bf16(v16[8 * ch + 4], v16[8 * ch + 5]);
        w4.w = tc::pack_bf16(v16[8 * ch + 6], v16[8 * ch + 7]);
        reinterpret_cast<uint4 *>(dst)[ch] = w4;
      }
    };
    // ---- prologue: planes (bf16, K-major rows j), tril, A_start, Bstate
    for (int i = threadIdx.x; i < a.LP * HD; i += NEPI_T) {
      const int j = i / HD, d = i % HD;
      const uint32_t off = P.planes + tc::sw128_off(j, d >> 3) + (d & 7) * 2;
      *reinterpret_cast<__nv_bfloat16 *>(sm + off) = __float2bfloat16(a.planes[(size_t)d * a.LP + j]);
    }
    {
      // tril[t][tau] = tau <= t; this thread writes row t, columns [32hq, 32hq+32)
      float v[8];
      for (int ch = 0; ch < 4; ++ch) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = (32 * hq + ch * 8 + e) <= t ? 1.f : 0.f;
        tc::st_row_chunk(sbase + P.tril + blk, t, ch0 + ch, v);
      }
    }
    // the A arrays hold A + eps (the chunk recurrence adds counts, so the offset carries)
    for (int s = threadIdx.x; s < S; s += NEPI_T)
      sA0[s] = state0[s] + a.eps + (a.seedA != nullptr ? a.seedA[(size_t)n * S + s] : 0.f);
    for (int g = 0; g < NG; ++g) {
      float v[16];
      const float *src = state0 + S + (size_t)(g * GB + t) * HD + 16 * hq;
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = src[i];
      if (a.seedB != nullptr) {
        const float *sd = a.seedB + ((size_t)n * S + g * GB + t) * HD + 16 * hq;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] += sd[i];
      }
      tc::tmem_st16(tmem + lane_off + T_B + 64 * g + 16 * hq, v);
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) tc::st_row_chunk(sbase + P.bst + g * TILE, t, 2 * hq + ch, v + 8 * ch);
      if (a.chunkB != nullptr && nch > 0) save_b(c_begin, g, v);
    }
    tc::tmem_wait_st();
    tc::fence_async_smem();
    tc::tc_fence_before();
    tc::named_bar_sync(NB_INIT, NTHR);

    // bf16 copy of Bstate_gr (lane t = bucket t), d in [16hq, 16hq+16), for the
    // next chunk's W x Bstate
    // (cc: the chunk this is the start state of; saved for the backward when asked)
    auto refresh = [=](int gr, int cc) {
      float bv[16];
      tc::tmem_ld16(tmem + lane_off + T_B + 64 * gr + 16 * hq, bv);
      tc::tmem_wait_ld();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) tc::st_row_chunk(sbase + P.bst + gr * TILE, t, 2 * hq + ch, bv + 8 * ch);
      if (a.chunkB != nullptr && cc < nch) save_b(c_begin + cc, gr, bv);
      tc::fence_async_smem();
      tc::tc_fence_before();
    };

    bool ok = true;
    for (int c = 0; c < nch; ++c) {
      const int tok0 = (c_begin + c) * C;
      const int nt = min(C, a.T - tok0);
      const uint32_t aCur = sbase + ((c & 1) ? P.a1 : P.a0), aNxt = sbase + ((c & 1) ? P.a0 : P.a1);
      // the row-127 threads wrote this chunk's A during the previous one
      tc::named_bar_sync(NB_ESYNC, NEPI_T);
      if (a.chunkA != nullptr) {  // A + eps at chunk start, for the backward
        const float *ac = reinterpret_cast<const float *>(sm + ((c & 1) ? P.a1 : P.a0));
        for (int s = threadIdx.x; s < S; s += NEPI_T) a.chunkA[((size_t)n * a.nchunks + c_begin + c) * S + s] = ac[s];
      }
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[B_PROJ], c & 1, abort));
      tc::tc_fence_after();
      for (int g = 0; g < NG; ++g) {
        const int u = c * NG + g;
        const int j0 = (g * 8 + hq * 2) * 4;  // first projection column of this thread's 2 tables
        // ---- Pk (row t, buckets [32hq, 32hq+32) of group g)
        if (ok) {
          float pj[8], pr[32];
          tc::tmem_ld8(tmem + lane_off + T_PK + j0, pj);
          tc::tmem_wait_ld();
          // (one table at a time: the two-table packed form measured slower in this kernel)
#pragma unroll
          for (int i = 0; i < 2; ++i) table_probs(pj + 4 * i, a.scale, a.poly, pr + 16 * i);
          if (t >= nt) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pr[i] = 0.f;
          }
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tc::st_row_chunk(sbase + P.pk + blk, t, ch0 + ch, pr + 8 * ch);
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(NB_PK, NTHR);
        // ---- pq while Apref runs, then W = pq / (A_start + Apref + eps)
        float pq[32];
        if (ok) {
          float pj[8];
          tc::tmem_ld8(tmem + lane_off + T_PQ + j0, pj);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) table_probs(pj + 4 * i, a.scale, a.poly, pq + 16 * i);
          ok = tc::warp_all(tc::mbar_wait(&bars[B_APREF], u & 1, abort));
        }
        tc::tc_fence_after();
        if (ok) {
          float ap[32];
          tc::tmem_ld32(tmem + lane_off + T_G + 32 * hq, ap);
          tc::tmem_wait_ld();
          const int sb = g * GB + 32 * hq;
          // den = A_start + eps + Apref; the row-127 thread's den is the next chunk's A + eps
          add_shared_row<32>(aCur + 4 * sb, ap);
          if (t == C - 1) store_shared_row<32>(aNxt + 4 * sb, ap);
          rcp_n<32>(ap, ap, a.batch_rcp);
          vmul<32>(pq, ap);
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tc::st_row_chunk(sbase + P.w + blk, t, ch0 + ch, pq + 8 * ch);
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(NB_W, NTHR);
        // ---- previous group's state refresh while Smat runs (with one group per
        // chunk the refresh follows Smask instead: the next Bupd is this group's)
        if (ok && NG > 1 && u > 0) refresh(g > 0 ? g - 1 : NG - 1, g > 0 ? c + 1 : c);
        // ---- Smask = tril(Smat), columns tau in [32hq, 32hq+32)
        if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[B_SMAT], u & 1, abort));
        tc::tc_fence_after();
        if (ok) {
          // warps above the diagonal (hq > q4) store zeros without reading TMEM
          float sv[32];
          if (hq <= q4) {
            tc::tmem_ld32(tmem + lane_off + T_G + 32 * hq, sv);
            tc::tmem_wait_ld();
            if (hq == q4) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (32 * hq + i > t) sv[i] = 0.f;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[i] = 0.f;
          }
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tc::st_row_chunk(sbase + P.w + blk, t, ch0 + ch, sv + 8 * ch);
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(NB_SMASK, NTHR);
        if (ok && NG == 1) refresh(0, c + 1);
      }
      // ---- out rows, d in [16hq, 16hq+16), after the chunk's last Smask V
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[B_GDONE], (c * NG + NG - 1) & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        float ov[16];
        tc::tmem_ld16(tmem + lane_off + T_OUT + 16 * hq, ov);
        tc::tmem_wait_ld();
        if (t < nt) {
          uint4 *dst = reinterpret_cast<uint4 *>(a.out + act_row(bn, hn, tok0 + t, a.T, a.H) + 16 * hq);
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint4 w4;
            w4.x = tc::pack_bf16(ov[8 * ch + 0], ov[8 * ch + 1]);
            w4.y = tc::pack_bf16(ov[8 * ch + 2], ov[8 * ch + 3]);
            w4.z = tc::pack_bf16(ov[8 * ch + 4], ov[8 * ch + 5]);
            w4.w = tc::pack_bf16(ov[8 * ch + 6], ov[8 * ch + 7]);
            dst[ch] = w4;
          }
        }
      }
      tc::tc_fence_before();
    }
    if (!ok && lane == 0) atomicExch(a.err, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NEPI) {
    if (s_abort[0] && lane == 0) atomicExch(a.err, 1);
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------------------
// Segment totals: A_tot[s] = sum_t pk[t,s], B_tot[s,:] = sum_t pk[t,s] V[t,:]
// over one (stream, segment), written as a record of the chunk_scan layout.
// Same warp roles; A_tot comes from an MMA against a ones column.
// States pass (a.chunkA != nullptr): the same walk started from the segment's
// exclusive prefix (a.seg_state) stores the state at every chunk start --
// A + eps in fp32 and B in bf16, the operands of the backward's reverse walk --
// and writes no record.
struct TotSmem {
  uint32_t k, v, pk, planes, bars, total;  // k: 2 stages of TILE bytes; v: 2 stages of [V | ones]
};

__host__ __device__ __forceinline__ TotSmem tot_smem_plan(int ngroups, int LP) {
  TotSmem m;
  uint32_t o = 0;
  m.k = o; o += 2 * TILE;
  m.v = o; o += 4 * TILE;  // stage st: V tile at v + 2 st TILE, a ones block right after it
  m.pk = o; o += (uint32_t)ngroups * 2 * TILE;
  m.planes = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.bars = o; o += 256;
  m.total = o + 1024;
  return m;
}

// TMEM map of the totals kernel (256 columns): projK 0..63; group g's sums at 64 + 80 g: Bstate
// (64 columns) then A (16 identical columns), one N = 80 accumulator: the B operand is the V
// stage and the ones block after it (MN-major 64-column blocks), so Pk^T [V | 1] gives both
// sums with one MMA per K step
enum { TB_FULL0 = 0, TB_FULL1, TB_PROJ, TB_PK, TB_DONE, TB_FINAL, TB_INIT, TB_COUNT };

__global__ void __launch_bounds__(NTHR, 1) fwd_totals_kernel(const __grid_constant__ CUtensorMap tmK,
                                                             const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = (unsigned char *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  const TotSmem P = tot_smem_plan(a.ngroups, a.LP);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bars);
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort[2];  // wait control: abort flag, poll limit
  const uint32_t sbase = tc::smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x / a.nseg, seg = blockIdx.x % a.nseg;
  const int hn = n % a.H, bn = n / a.H;  // head and batch of stream n in the activation layout
  const int c_begin = seg * a.seg_chunks;
  const int c_end = min(a.nchunks, c_begin + a.seg_chunks);
  const int nch = c_end - c_begin;
  const int S = a.S;
  const size_t E = (size_t)S + (size_t)S * HD;
  float *rec = a.seg_tot + ((size_t)n * a.nseg + seg) * E;
  const bool states = a.chunkA != nullptr;

  if (threadIdx.x == 0) {
    s_abort[0] = 0;
    s_abort[1] = (int)a.wait_limit;
    tc::mbar_init(&bars[TB_FULL0], 1);
    tc::mbar_init(&bars[TB_FULL1], 1);
    tc::mbar_init(&bars[TB_PROJ], 1);
    tc::mbar_init(&bars[TB_PK], NARR);
    tc::mbar_init(&bars[TB_DONE], 1);
    tc::mbar_init(&bars[TB_FINAL], 1);
    tc::mbar_init(&bars[TB_INIT], NARR);
    tc::fence_mbar_init();
  }
  if (warp == NEPI) tc::tmem_alloc(&s_tmem, 256);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int *abort = s_abort;

  if (warp == NEPI) {
    if (lane == 0 && nch > 0) {
      tc::prefetch_tmap(&tmK);
      tc::prefetch_tmap(&tmV);
      for (int c = a.withhold_first_load ? 2 : 0; c < 2 && c < nch; ++c) {
        tc::mbar_arrive_expect_tx(&bars[TB_FULL0 + c], 2 * TILE);
        tc::tma_load_4d(sm + P.k + c * TILE, &tmK, &bars[TB_FULL0 + c], 0, hn, (c_begin + c) * C, bn);
        tc::tma_load_4d(sm + P.v + 2 * c * TILE, &tmV, &bars[TB_FULL0 + c], 0, hn, (c_begin + c) * C, bn);
      }
      const uint32_t id_proj = tc::idesc_bf16(C, a.LP, false, false);
      const uint32_t id_sums = tc::idesc_bf16(GB, HD + 16, true, true);
      auto issue_proj = [&](int st) {
        for (int k0 = 0; k0 < HD; k0 += 16)
          tc::mma_bf16(tmem + 0, tc::desc_kmajor(sbase + P.k + st * TILE, k0, TILE),
                       tc::desc_kmajor(sbase + P.planes, k0, 0), id_proj, k0 > 0);
        tc::mma_commit(&bars[TB_PROJ]);
      };
      bool ok = tc::mbar_wait(&bars[TB_INIT], 0, abort);  // planes + ones column written
      if (ok) ok = tc::mbar_wait(&bars[TB_FULL0], 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_proj(0);
      }
      // Per chunk c: [PK c] the next chunk's projection first (its K tile is in the other
      // stage; the epilogue has read proj c), then the sums for c.  MMAs complete in issue
      // order, so proj c+1 is ready while the sums of c run and the epilogue's soft hash of
      // c+1 overlaps them; the stage of c refills once the sums complete.
      for (int c = 0; c < nch && ok; ++c) {
        const int st = c & 1;
        ok = tc::mbar_wait(&bars[TB_PK], c & 1, abort);
        if (!ok) break;
        tc::tc_fence_after();
        if (c + 1 < nch) {
          ok = tc::mbar_wait(&bars[TB_FULL0 + (st ^ 1)], ((c + 1) >> 1) & 1, abort);
          if (!ok) break;
          tc::tc_fence_after();
          issue_proj(st ^ 1);
        }
        for (int g = 0; g < a.ngroups; ++g) {
          const uint32_t pk = sbase + P.pk + (uint32_t)g * 2 * TILE;
          for (int k0 = 0; k0 < C; k0 += 16) {
            const uint64_t ap = tc::desc_mnmajor(pk, k0, TILE);
            tc::mma_bf16(tmem + 64 + 80 * g, ap, tc::desc_mnmajor(sbase + P.v + 2 * st * TILE, k0, TILE), id_sums,
                         states || c > 0 || k0 > 0);
          }
        }
        tc::mma_commit(&bars[TB_DONE]);
        if (c + 2 < nch) {
          ok = tc::mbar_wait(&bars[TB_DONE], c & 1, abort);
          if (!ok) break;
          tc::mbar_arrive_expect_tx(&bars[TB_FULL0 + st], 2 * TILE);
          tc::tma_load_4d(sm + P.k + st * TILE, &tmK, &bars[TB_FULL0 + st], 0, hn, (c_begin + c + 2) * C,
                          bn);
          tc::tma_load_4d(sm + P.v + 2 * st * TILE, &tmV, &bars[TB_FULL0 + st], 0, hn, (c_begin + c + 2) * C,
                          bn);
        }
      }
      tc::mma_commit(&bars[TB_FINAL]);
      if (!tc::mbar_wait_drain(&bars[TB_FINAL], 0)) atomicExch(a.err, 2);
    }
    __syncwarp();
  } else {
    const int q4 = warp & 3, hq = warp >> 2;
    const int t = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    for (int i = threadIdx.x; i < a.LP * HD; i += NEPI_T) {
      const int j = i / HD, d = i % HD;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.planes + tc::sw128_off(j, d >> 3) + (d & 7) * 2) =
          __float2bfloat16(a.planes[(size_t)d * a.LP + j]);
    }
    {
      float v[8];
      for (int ch = 2 * hq; ch < 2 * hq + 2; ++ch) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = (ch * 8 + e) < 16 ? 1.f : 0.f;
        tc::st_row_chunk(sbase + P.v + TILE, t, ch, v);      // after V stage 0
        tc::st_row_chunk(sbase + P.v + 3 * TILE, t, ch, v);  // after V stage 1
      }
    }
    if (states) {  // segment-start state into the accumulators (lane t = bucket t of group g)
      const float *st0 = a.seg_state + ((size_t)n * a.nseg + seg) * E;
      for (int g = 0; g < a.ngroups; ++g) {
        float v[16];
        const float *src = st0 + S + (size_t)(g * GB + t) * HD + 16 * hq;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = src[i];
        tc::tmem_st16(tmem + lane_off + 64 + 80 * g + 16 * hq, v);
        if (hq == 0) tc::tmem_st1(tmem + lane_off + 128 + 80 * g, st0[g * GB + t]);
      }
      tc::tmem_wait_st();
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    tc::warp_arrive(&bars[TB_INIT]);
    bool ok = true;
    for (int c = 0; c < nch && ok; ++c) {
      const int nt = min(C, a.T - (c_begin + c) * C);
      ok = tc::warp_wait(&bars[TB_PROJ], c & 1, abort);
      // the states pass reads the accumulators, which hold this chunk's start state once the
      // previous chunk's sums are complete
      if (ok && c > 0 && states) ok = tc::warp_wait(&bars[TB_DONE], (c - 1) & 1, abort);
      if (!ok) break;
      __syncwarp();
      tc::tc_fence_after();
      if (states) {  // the accumulators hold this chunk's start state until its MMAs are issued
        const int cg = c_begin + c;
        for (int g = 0; g < a.ngroups; ++g) {
          float bv[16], av;
          tc::tmem_ld16(tmem + lane_off + 64 + 80 * g + 16 * hq, bv);
          tc::tmem_ld1(tmem + lane_off + 128 + 80 * g, av);
          tc::tmem_wait_ld();
          const size_t row = ((size_t)n * a.nchunks + cg) * S + g * GB + t;
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint4 w4;
            w4.x = tc::pack_bf16(bv[8 * ch + 0], bv[8 * ch + 1]);
            w4.y = tc::pack_bf16(bv[8 * ch + 2], bv[8 * ch + 3]);
            w4.z = tc::pack_bf16(bv[8 * ch + 4], bv[8 * ch + 5]);
            w4.w = tc::pack_bf16(bv[8 * ch + 6], bv[8 * ch + 7]);
            *reinterpret_cast<uint4 *>(a.chunkB + row * HD + 16 * hq + 8 * ch) = w4;
          }
          if (hq == 0) a.chunkA[row] = av + a.eps;
        }
      }
      // Pk of this row for every group in registers (overlapping the previous chunk's sums),
      // then into the shared tiles once those sums, their readers, are complete
      float pr[2][32];  // ngroups <= 2 (S <= 256)
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        if (g < a.ngroups) {
          const int j0 = (g * 8 + hq * 2) * 4;
          float pj[8];
          tc::tmem_ld8(tmem + lane_off + j0, pj);
          tc::tmem_wait_ld();
          table_probs2(pj, pj + 4, a.scale, a.poly, pr[g], pr[g] + 16);
          if (t >= nt) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pr[g][i] = 0.f;
          }
        }
      }
      if (c > 0 && !states) {
        ok = tc::warp_wait(&bars[TB_DONE], (c - 1) & 1, abort);
        if (!ok) break;
        __syncwarp();
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        if (g < a.ngroups) {
#pragma unroll
          for (int ch = 0; ch < 4; ++ch)
            tc::st_row_chunk(sbase + P.pk + (g * 2 + (hq >> 1)) * TILE, t, (hq & 1) * 4 + ch, pr[g] + 8 * ch);
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::warp_arrive(&bars[TB_PK]);
    }
    // write the totals record
    if (ok && nch > 0) ok = tc::warp_wait(&bars[TB_DONE], (nch - 1) & 1, abort);
    __syncwarp();
    tc::tc_fence_after();
    if (ok && !states) {
      for (int g = 0; g < a.ngroups; ++g) {
        float bv[16], av;
        tc::tmem_ld16(tmem + lane_off + 64 + 80 * g + 16 * hq, bv);
        tc::tmem_ld1(tmem + lane_off + 128 + 80 * g, av);
        tc::tmem_wait_ld();
        float *dst = rec + S + (size_t)(g * GB + t) * HD + 16 * hq;
#pragma unroll
        for (int i = 0; i < 16; ++i) dst[i] = bv[i];
        if (hq == 0) rec[g * GB + t] = av;
      }
    }
    if (nch == 0 && !states) {  // empty segment: zero record
      for (int i = threadIdx.x; i < (int)E; i += NEPI_T) rec[i] = 0.f;
    }
    if (!ok && lane == 0) atomicExch(a.err, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NEPI) {
    if (s_abort[0] && lane == 0) atomicExch(a.err, 1);
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

}  // namespace fast
}  // namespace race
