// noncausal.cuh -- fused tcgen05 per-token kernel of non-causal RACE (the
// reference's BatchedACE with shared planes: scaling/benchmark_time.py:77-166,
// misc/classification.py:257-308) for bf16, D = 64, P = 4, S in {128, 256}.
//
// Non-causal RACE reads one [S, D] summary per stream instead of a running
// state:
//   b = sum_t pk_t^T V_t,  A = sum_t pk_t,  E = b / (A + eps),  out_t = pq_t E
// with the exact gradients
//   dE = sum_t pq_t^T dO_t,  db = dE / (A + eps),
//   dA_s = -sum_d dE[s,d] b[s,d] / (A_s + eps)^2,
//   dpq_t = dO_t E^T,  dpk_t = dA + V_t db^T,  dV_t = pk_t db.
// The sums over tokens (b and A from (K, V); dE from (Q, dO)) are the causal
// path's totals kernel and segment scan.  Every per-token product is
// ace_tile_kernel, one CTA per (stream, segment of 128-token tiles); tiles do
// not depend on one another:
//   ACE_OUT (X = Q)         proj, pq -> P tile ; O = P E                -> out
//   ACE_KV  (X = K, Y = V)  proj, pk -> P tile ; O = P db               -> dV
//                           Dfix = V db^T ; dproj = softmax bwd of (Dfix + dA)
//                           dX = dproj planes                          -> dK
//   ACE_Q   (X = Q, Y = dO) proj, pq ; Dfix = dO E^T ;
//                           dproj = softmax bwd of Dfix ; dX = dproj planes -> dQ
// Each CTA forms its summary (E or db, bf16, the MMA operand) and dA in its
// prologue from the fp32 totals; no [N, T, S] tensor exists anywhere.  The
// projections and dproj use bf16 hi + lo pairs of the planes and of dproj
// (exact to ~2^-17 once summed), as in the causal fix-up kernel.
//
// Schedule per tile c ({X}: the epilogue warps arrive on named barrier X, the
// control warp waits; [X]: mbarrier completed by tcgen05.commit):
//   control: proj -> [PROJ] ; Dfix -> [DFIX] ; -> [TFREE] (X, Y tiles read)
//            {PK} next tile's loads after [TFREE] ; O = P M
//            {DP} dX = dproj planes ; (the previous tile's stores have read the
//                 staging tiles) -> [OUT] ; next tile's proj, Dfix
//            {OUTFREE} TMA tile stores of this tile's outputs
//   epilogue: [PROJ] tanh, plane sigmoids, P tile {PK} ;
//             [DFIX] dproj hi/lo tiles {DP} ; [OUT] output rows into the
//             staging tiles {OUTFREE}
// The next tile's loads overlap this tile's products and epilogue.  All waits
// are bounded (see fast_fwd.cuh).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"
#include "fast_bwd.cuh"
#include "fast_fwd.cuh"
#include "tc_ptx.cuh"

namespace race {
namespace fast {

enum { ACE_OUT = 0, ACE_KV = 1, ACE_Q = 2 };

struct AceArgs {
  int N, T, L, LP, S, H;
  int nseg, seg_chunks, nchunks;
  float eps, scale;
  int poly;             // plane sigmoids by series (2|scale| <= 1/2)
  const float *planes;  // [64, LP]
  const float *totA;    // [N, S]      A = sum_t pk
  const float *totB;    // [N, S, 64]  b = sum_t pk^T V
  const float *totG;    // [N, S, 64]  dE = sum_t pq^T dO (ACE_KV only)
  int *err;
  uint32_t wait_limit;
};

struct AceSmem {
  uint32_t x, y, pk, m, dp, dplo, s1, s2, planes, plo, bias, bars, total;
};

// x, y: input tiles ; pk: [128 t x S] bf16 probabilities, 64-column K-major blocks ;
// m: the summary [S rows x 64] bf16 ; dp, dplo: dproj hi / lo [128 x LP] ;
// s1, s2: output staging tiles (TMA stores) ; planes, plo: planes hi / lo [LP x 64]
__host__ __device__ __forceinline__ AceSmem ace_smem_plan(int LP, int S) {
  AceSmem m;
  uint32_t o = 0;
  m.x = o; o += TILE;
  m.y = o; o += TILE;
  m.pk = o; o += (uint32_t)(S / 64) * TILE;
  m.m = o; o += (uint32_t)S * 128;
  m.dp = o; o += TILE;
  m.dplo = o; o += TILE;
  m.s1 = o; o += TILE;
  m.s2 = o; o += TILE;
  m.planes = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.plo = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.bias = o; o += (uint32_t)align_up((size_t)S * 4, 128);
  m.bars = o; o += 256;
  m.total = o + 1024;
  return m;
}

enum { AB_XY = 0, AB_PROJ, AB_DFIX, AB_TFREE, AB_OUT, AB_FINAL, AB_COUNT };
enum { AN_INIT = 1, AN_PK, AN_DP, AN_OUTFREE };

// tmX: Q (ACE_OUT, ACE_Q) or K (ACE_KV); tmY: V (ACE_KV) or dO (ACE_Q), unused by ACE_OUT;
// tmO1: out (ACE_OUT), dK (ACE_KV) or dQ (ACE_Q); tmO2: dV (ACE_KV), unused otherwise.
template <int MODE>
__global__ void __launch_bounds__(NTHR, 1) ace_tile_kernel(const __grid_constant__ CUtensorMap tmX,
                                                           const __grid_constant__ CUtensorMap tmY,
                                                           const __grid_constant__ CUtensorMap tmO1,
                                                           const __grid_constant__ CUtensorMap tmO2, AceArgs a) {
  constexpr bool kP = MODE != ACE_Q;    // the P tile and O = P M
  constexpr bool kD = MODE != ACE_OUT;  // Dfix, dproj and dX = dproj planes
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = (unsigned char *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  const AceSmem P = ace_smem_plan(a.LP, a.S);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bars);
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort[2];  // wait control: abort flag, poll limit
  const uint32_t sbase = tc::smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x / a.nseg, seg = blockIdx.x % a.nseg;
  const int hn = n % a.H, bn = n / a.H;
  const int c_begin = seg * a.seg_chunks;
  const int nch = min(a.nchunks, c_begin + a.seg_chunks) - c_begin;
  const int S = a.S, LP = a.LP;
  // TMEM: proj [0, 64) ; Dfix [64, 64 + S) ; O and dX 64 columns each after it
  const uint32_t T_PJ = 0, T_D = 64, T_O = 64 + S, T_DX = T_O + 64;

  if (threadIdx.x == 0) {
    s_abort[0] = 0;
    s_abort[1] = (int)a.wait_limit;
    for (int i = 0; i < AB_COUNT; ++i) tc::mbar_init(&bars[i], 1);
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
    const uint32_t id_proj = tc::idesc_bf16(C, LP, false, false);
    const uint32_t id_d = tc::idesc_bf16(C, S, false, false);
    const uint32_t id_o = tc::idesc_bf16(C, HD, false, true);
    const uint32_t ox = P.x, oy = P.y;
    auto load = [=, &tmX, &tmY](int c) {
      const int t0 = (c_begin + c) * C;
      tc::mbar_arrive_expect_tx(&bars[AB_XY], (kD ? 2u : 1u) * TILE);
      tc::tma_load_4d(sm + ox, &tmX, &bars[AB_XY], 0, hn, t0, bn);
      if (kD) tc::tma_load_4d(sm + oy, &tmY, &bars[AB_XY], 0, hn, t0, bn);
    };
    // proj = X (planes_hi + planes_lo) -> [PROJ] ; Dfix = Y M^T -> [DFIX] ; then [TFREE]
    auto issue_front = [=]() {
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int k0 = 0; k0 < HD; k0 += 16)
          tc::mma_bf16(tmem + T_PJ, tc::desc_kmajor(sbase + P.x, k0, 0),
                       tc::desc_kmajor(sbase + (part ? P.plo : P.planes), k0, 0), id_proj, part > 0 || k0 > 0);
      tc::mma_commit(&bars[AB_PROJ]);
      if (kD) {
#pragma unroll
        for (int k0 = 0; k0 < HD; k0 += 16)
          tc::mma_bf16(tmem + T_D, tc::desc_kmajor(sbase + P.y, k0, 0), tc::desc_kmajor(sbase + P.m, k0, 0), id_d,
                       k0 > 0);
        tc::mma_commit(&bars[AB_DFIX]);
      }
      tc::mma_commit(&bars[AB_TFREE]);
    };
    auto store_out = [=, &tmO1, &tmO2](int c) {
      const int t0 = (c_begin + c) * C;
      tc::tma_store_4d(&tmO1, sm + P.s1, 0, hn, t0, bn);
      if (MODE == ACE_KV) tc::tma_store_4d(&tmO2, sm + P.s2, 0, hn, t0, bn);
      tc::bulk_commit();
    };
    bool ok = true;
    if (leader && nch > 0) {
      tc::prefetch_tmap(&tmX);
      if (kD) tc::prefetch_tmap(&tmY);
      load(0);
    }
    tc::named_bar_sync(AN_INIT, NTHR);  // planes, summary and dA are in shared memory
    if (leader && nch > 0) {
      ok = tc::mbar_wait(&bars[AB_XY], 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_front();
      }
    }
    for (int c = 0; c < nch; ++c) {
      tc::named_bar_sync(AN_PK, NTHR);
      ok = ok && !*abort;
      if (leader && ok) {
        tc::tc_fence_after();
        ok = tc::mbar_wait(&bars[AB_TFREE], c & 1, abort);  // every reader of the X, Y tiles completed
        if (ok && c + 1 < nch) load(c + 1);
        if (ok && kP) {
#pragma unroll 4
          for (int k0 = 0; k0 < S; k0 += 16)
            tc::mma_bf16(tmem + T_O, tc::desc_kmajor(sbase + P.pk, k0, TILE), tc::desc_mnmajor(sbase + P.m, k0, 0),
                         id_o, k0 > 0);
        }
        if (ok && !kD) {
          if (c > 0) tc::bulk_wait_read();  // the previous tile's store has read the staging tile
          tc::mma_commit(&bars[AB_OUT]);
        }
      }
      if (kD) {
        tc::named_bar_sync(AN_DP, NTHR);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
          // dX = dproj (planes_hi + planes_lo) + dproj_lo planes_hi
#pragma unroll
          for (int part = 0; part < 3; ++part)
            for (int k0 = 0; k0 < LP; k0 += 16)
              tc::mma_bf16(tmem + T_DX, tc::desc_kmajor(sbase + (part == 2 ? P.dplo : P.dp), k0, 0),
                           tc::desc_mnmajor(sbase + (part == 1 ? P.plo : P.planes), k0, 0), id_o, part > 0 || k0 > 0);
          if (c > 0) tc::bulk_wait_read();  // the previous tile's stores have read the staging tiles
          tc::mma_commit(&bars[AB_OUT]);
        }
      }
      if (leader && ok && c + 1 < nch) {
        // the epilogue has read this tile's proj and Dfix: the next tile's go into the same columns
        ok = tc::mbar_wait(&bars[AB_XY], (c + 1) & 1, abort);
        if (ok) {
          tc::tc_fence_after();
          issue_front();
        }
      }
      tc::named_bar_sync(AN_OUTFREE, NTHR);  // this tile's output rows are in the staging tiles
      ok = ok && !*abort;
      if (leader && ok) store_out(c);
    }
    if (leader && nch > 0) {
      tc::bulk_wait();  // stores complete (and shared memory read) before the CTA exits
      tc::mma_commit(&bars[AB_FINAL]);
      if (!tc::mbar_wait_drain(&bars[AB_FINAL], 0)) atomicExch(a.err, 2);
    }
    __syncwarp();
  } else {
    // ============================== epilogue warps: row t, column quarter hq
    // (quarter hq owns tables [tq hq, tq hq + tq), tq = L / 4: buckets [16 tq hq, +16 tq),
    // projection columns [4 tq hq, +4 tq), output columns [16 hq, +16))
    const int q4 = warp & 3, hq = warp >> 2;
    const int t = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int tq = a.L / 4;
    for (int i = threadIdx.x; i < LP * HD; i += NEPI_T) {  // planes = hi + lo, both bf16
      const int j = i / HD, d = i % HD;
      const float pv = a.planes[(size_t)d * LP + j];
      const __nv_bfloat16 hi = __float2bfloat16(pv);
      const uint32_t off = tc::sw128_off(j, d >> 3) + (d & 7) * 2;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.planes + off) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.plo + off) = __float2bfloat16(pv - __bfloat162float(hi));
    }
    // the summary M (bf16 rows s): E = b / (A + eps), or db = dE / (A + eps) for ACE_KV;
    // and for ACE_KV, dA_s = -sum_d dE[s,d] b[s,d] / (A_s + eps)^2
    const float *tA = a.totA + (size_t)n * S;
    const float *tB = a.totB + (size_t)n * S * HD;
    const float *src = MODE == ACE_KV ? a.totG + (size_t)n * S * HD : tB;
    for (int i = threadIdx.x; i < S * 8; i += NEPI_T) {
      const int sr = i >> 3, ch = i & 7;
      const float inv = 1.f / (tA[sr] + a.eps);
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = src[(size_t)sr * HD + ch * 8 + e] * inv;
      tc::st_row_chunk(sbase + P.m, sr, ch, v);
    }
    float *sBias = reinterpret_cast<float *>(sm + P.bias);
    if (MODE == ACE_KV) {
      for (int s = threadIdx.x; s < S; s += NEPI_T) {
        float acc = 0.f;
        for (int d = 0; d < HD; ++d) acc = fmaf(src[(size_t)s * HD + d], tB[(size_t)s * HD + d], acc);
        const float inv = 1.f / (tA[s] + a.eps);
        sBias[s] = -acc * inv * inv;
      }
    }
    tc::fence_async_smem();
    tc::named_bar_sync(AN_INIT, NTHR);

    bool ok = true;
    for (int c = 0; c < nch; ++c) {
      float th[16], q[16];  // tanh and plane sigmoids of this quarter's tables (up to 4)
      // ---- soft hash of X ; the P tile
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[AB_PROJ], c & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        if (tq == 4) {
          float pj[16];
          tc::tmem_ld16(tmem + lane_off + T_PJ + 16 * hq, pj);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) th[i] = tanh_fast(pj[i]);
        } else {
          float pj[8];
          tc::tmem_ld8(tmem + lane_off + T_PJ + 8 * hq, pj);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) th[i] = tanh_fast(pj[i]);
#pragma unroll
          for (int i = 8; i < 16; ++i) th[i] = 0.f;
        }
#pragma unroll
        for (int tb = 0; tb < 4; tb += 2) {  // tables in pairs (tq is 2 or 4)
          if (tb < tq) {
            plane_sigmoids(th + 4 * tb, a.scale, a.poly, q + 4 * tb);
            plane_sigmoids(th + 4 * tb + 4, a.scale, a.poly, q + 4 * tb + 4);
            if (kP) {
              float pr[32];
              corner_probs2(q + 4 * tb, q + 4 * tb + 4, pr, pr + 16);
              const int b0 = 16 * (tq * hq + tb);  // first bucket of the table pair
#pragma unroll
              for (int ch = 0; ch < 4; ++ch)
                tc::st_row_chunk(sbase + P.pk + (uint32_t)(b0 >> 6) * TILE, t, ((b0 & 63) >> 3) + ch, pr + 8 * ch);
            }
          }
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(AN_PK, NTHR);
      // ---- dproj = softmax bwd of (Dfix + dA), as hi + lo bf16
      if (kD) {
        if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[AB_DFIX], c & 1, abort));
        tc::tc_fence_after();
        if (ok) {
#pragma unroll
          for (int tb = 0; tb < 4; ++tb) {
            if (tb < tq) {
              const int b0 = 16 * (tq * hq + tb);
              float g16[16], p16[16], dp[4], lo[4];
              tc::tmem_ld16(tmem + lane_off + T_D + b0, g16);
              tc::tmem_wait_ld();
              if (MODE == ACE_KV) add_shared_row<16>(sbase + P.bias + 4 * b0, g16);
              corner_probs(q + 4 * tb, p16);
              table_probs_bwd(p16, g16, q + 4 * tb, th + 4 * tb, a.scale, dp);
              bf16r2(dp[0], dp[1], lo[0], lo[1]);
              bf16r2(dp[2], dp[3], lo[2], lo[3]);
#pragma unroll
              for (int i = 0; i < 4; ++i) lo[i] = dp[i] - lo[i];
              const int j = 4 * (tq * hq + tb);  // first projection column of the table
              tc::st_row_half(sbase + P.dp, t, j >> 3, (j >> 2) & 1, dp);
              tc::st_row_half(sbase + P.dplo, t, j >> 3, (j >> 2) & 1, lo);
            }
          }
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(AN_DP, NTHR);
      }
      // ---- output rows (d in [16 hq, 16 hq + 16)) into the staging tiles
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[AB_OUT], c & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        float vx[16], vo[16];
        if (kD) tc::tmem_ld16(tmem + lane_off + T_DX + 16 * hq, vx);
        if (kP) tc::tmem_ld16(tmem + lane_off + T_O + 16 * hq, vo);
        tc::tmem_wait_ld();
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          if (kD) tc::st_row_chunk(sbase + P.s1, t, 2 * hq + ch, vx + 8 * ch);
          if (MODE == ACE_OUT) tc::st_row_chunk(sbase + P.s1, t, 2 * hq + ch, vo + 8 * ch);
          if (MODE == ACE_KV) tc::st_row_chunk(sbase + P.s2, t, 2 * hq + ch, vo + 8 * ch);
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(AN_OUTFREE, NTHR);
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

}  // namespace fast
}  // namespace race
