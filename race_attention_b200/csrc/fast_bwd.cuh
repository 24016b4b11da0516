// fast_bwd.cuh -- fused tcgen05 backward for bf16, D = 64, P = 4, S in {128, 256}.
//
// Exact gradients of the causal RACE layer (scaling/race_common.py:76-90 with
// the soft hash of :36-73), per stream n, with W = pq/(A_t+eps):
//   G_t[s]  = dO_t . B_t[s]                    dpq = G/(A_t+eps)
//   dA_t[s] = -W_t[s] G_t[s] / (A_t[s]+eps)
//   gA_t    = sum_{t'>=t} dA_t'   gB_t = sum_{t'>=t} W_t' (x) dO_t'   (suffix states)
//   dpk     = gA_t + V_t . gB_t   dV_t = sum_s pk[t,s] gB_t[s]
// Per (stream, segment) of 128-token chunks, with buckets in groups of 64
// (4 tables); per-bucket state accumulators are M=64 tcgen05 tiles, two groups
// sharing a TMEM column block (lane offsets 0 and 16):
//
//   bwd_rev_kernel (reverse walk from a zero suffix state at the segment end,
//     i.e. segment-local gradient states, forward state from the stored chunk
//     starts): per group Pk, Apref = tril Pk, W, G = dO Bst^T + P1m Pk, dA,
//     dpq -> d proj_Q ; dpk = tril^T dA + V gBst^T + P1m^T W + gA -> d proj_K ;
//     Q2 = Pk W^T (masked t' >= tau) ; dV = Pk gBst + Q2m dO ; gB += W^T dO,
//     gA += dA^T 1 ; the segment's local totals at the end.
//   chunk_scan (reverse): the suffix of later segments for each segment.
//   bwd_fix_kernel (chunks independent): that suffix's linear share of dpk and
//     dV, dK = d proj_K planes, dQ = d proj_Q planes.
// All waits are bounded (see fast_fwd.cuh).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"
#include "fast_fwd.cuh"
#include "tc_ptx.cuh"

namespace race {
namespace fast {

constexpr int GW = 64;  // buckets per backward group

struct BwdArgs {
  int N, T, L, LP, S, ngroups;  // ngroups = S / 64
  int H;                        // heads of the activation layout (act_row); dVloc follows it too
  int nseg, seg_chunks, nchunks;
  float eps, scale;
  int poly;                 // plane sigmoids by series (2|scale| <= 1/2)
  int batch_rcp;            // reciprocals of A + eps four at a time (eps >= 1e-8)
  const float *planes;      // [64, LP]
  const float *fwd_state;   // [N, nseg, E]  forward exclusive segment prefixes
  float *tot;               // [N, nseg, E]  first walk: segment gradient totals
  const float *suf_state;   // [N, nseg, E]  reverse-scanned totals (suffix at segment end)
  float *chunkA;            // [N, nchunks, S]        fp32 A at chunk start
  __nv_bfloat16 *chunkB;    // [N, nchunks, S, 64]    bf16 B at chunk start
  __nv_bfloat16 *dQ, *dK, *dV;  // [N, T, 64]
  __nv_bfloat16 *dprojQ;        // [N, T, 64] d proj_Q (columns >= LP unused), reverse walk -> fix-up
  float *dprojK;                // segment-local d proj_K (fp32), reverse walk -> fix-up, table-major per
                                //   chunk: [N, nchunks, LP/4 tables, 128 tokens, 4] (one 16-byte row
                                //   per token and table: a warp's rows are one contiguous 512 bytes)
  const float *seedA, *seedB;   // fix-up: suffix of later shards added to every segment's ([N,S], [N,S,64])
  const __nv_bfloat16 *dVloc;   // fix-up: the walk's dV when it is not in dV itself (split backward)
  int *err;
  uint32_t wait_limit;          // polls before a bounded wait gives up (tc::kDefaultWaitPolls unless set)
};

// d proj of one table from the gradient g16 of its 16 corner probabilities.
// p_r = prod_b f_b(r) with f_b = q_b or 1 - q_b by bit (3-b) of r, so
//   dL/dz_b = q_b (1 - q_b) dL/dq_b = sum_{r: bit set} g_r p_r - q_b sum_r g_r p_r
// (the softmax backward over the corner logits, sum_r sign_b(r) p_r (g_r - c),
// written with sum_{bit set} p_r = q_b), then z_b = 2 scale tanh(proj_b).
// The bit-set sums come from one pairwise-sum tree.
__device__ __forceinline__ void table_probs_bwd(const float *p16, const float *g16, const float *q4, const float *th4,
                                                float scale, float *out4) {
  float gp[16];
#pragma unroll
  for (int r = 0; r < 16; r += 2) st2(gp, r, __fmul2_rn(ld2(p16, r), ld2(g16, r)));
  float a[8], s3 = 0.f;  // plane 3: bit 0
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a[i] = gp[2 * i] + gp[2 * i + 1];
    s3 += gp[2 * i + 1];
  }
  float b[4], s2 = 0.f;  // plane 2: bit 1
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    b[j] = a[2 * j] + a[2 * j + 1];
    s2 += a[2 * j + 1];
  }
  const float s1 = b[1] + b[3];  // plane 1: bit 2
  const float s0 = b[2] + b[3];  // plane 0: bit 3
  const float c = (b[0] + b[1]) + s0;
  const float set[4] = {s0, s1, s2, s3};
  const float2 nc = dup2(-c), s2s = dup2(2.f * scale), one = dup2(1.f);
#pragma unroll
  for (int p = 0; p < 4; p += 2) {
    const float2 th = ld2(th4, p);
    const float2 d = __ffma2_rn(ld2(q4, p), nc, ld2(set, p));               // set_p - q_p c
    const float2 sech2 = __ffma2_rn(make_float2(-th.x, -th.y), th, one);   // 1 - tanh^2
    st2(out4, p, __fmul2_rn(__fmul2_rn(d, s2s), sech2));
  }
}


// bf16 roundings (to nearest even, as the MMA operands are stored) of two values
// with one packed conversion
__device__ __forceinline__ void bf16r2(float a, float b, float &ra, float &rb) {
  const uint32_t p = tc::pack_bf16(a, b);
  ra = __uint_as_float(p << 16);
  rb = __uint_as_float(p & 0xffff0000u);
}

__device__ __forceinline__ void st_bf16x8_global(__nv_bfloat16 *dst, const float *v) {
  uint4 w;
  w.x = tc::pack_bf16(v[0], v[1]);
  w.y = tc::pack_bf16(v[2], v[3]);
  w.z = tc::pack_bf16(v[4], v[5]);
  w.w = tc::pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4 *>(dst) = w;
}

// --------------------------------------------------------------------------
struct BwdSmem {
  uint32_t q, k, v, o, p1m, tril, planes, pk, w, da, bst, gbst, ones, diag, a0, ga, bars, total;
};

// planes: per 64-bucket group g, 32 K-major rows: the group's 16 bf16 planes (rows 32g..)
// then their residuals planes - bf16(planes) (rows 32g+16..), so one N = 32 MMA gives
// both halves of the projections (exact to ~2^-17 once summed); tril and p1m: strictly lower triangles (tau < t),
// the diagonal terms being added in fp32 by the epilogue from diag, the fp32
// diagonal of P1 = dO V^T; ones: the B operand of the gA column sums.
__host__ __device__ __forceinline__ BwdSmem bwd_smem_plan(int LP, int S) {
  BwdSmem m;
  uint32_t o = 0;
  m.q = o; o += TILE;
  m.k = o; o += TILE;
  m.v = o; o += TILE;
  m.o = o; o += TILE;
  m.p1m = o; o += 2 * TILE;
  m.tril = o; o += 2 * TILE;
  m.planes = o; o += (uint32_t)align_up((size_t)2 * LP * 128, 1024);
  m.pk = o; o += TILE;
  m.w = o; o += TILE;
  m.da = o; o += TILE;  // must follow w: [w | da] is the 2-block Q2m tile
  m.bst = o; o += GW * 128;
  m.gbst = o; o += GW * 128;
  m.ones = o; o += 16 * C * 2;  // K-major [16 x 128] of ones: the B of gA += dA^T 1
  m.diag = o; o += C * 4;
  m.a0 = o; o += (uint32_t)align_up((size_t)S * 4, 128);
  m.ga = o; o += 2 * GW * 4;  // two buffers (group parity)
  m.bars = o; o += 256;
  m.total = o + 1024;
  return m;
}

// TMEM loads / stores of n consecutive columns of this thread's lane
template <int n>
__device__ __forceinline__ void tmem_ldn(uint32_t addr, float *v) {
  if constexpr (n == 4) {
    tc::tmem_ld4(addr, *reinterpret_cast<float(*)[4]>(v));
  } else if constexpr (n == 8) {
    tc::tmem_ld8(addr, *reinterpret_cast<float(*)[8]>(v));
  } else if constexpr (n == 16) {
    tc::tmem_ld16(addr, *reinterpret_cast<float(*)[16]>(v));
  } else {
    static_assert(n % 32 == 0, "tmem_ldn: 4, 8, 16 or a multiple of 32 columns");
#pragma unroll
    for (int i = 0; i < n / 32; ++i) tc::tmem_ld32(addr + 32 * i, *reinterpret_cast<float(*)[32]>(v + 32 * i));
  }
}
template <int n>
__device__ __forceinline__ void tmem_stn(uint32_t addr, const float *v) {
  if constexpr (n == 16) {
    tc::tmem_st16(addr, *reinterpret_cast<const float(*)[16]>(v));
  } else {
    static_assert(n % 32 == 0, "tmem_stn: 16 or a multiple of 32 columns");
#pragma unroll
    for (int i = 0; i < n / 32; ++i)
      tc::tmem_st32(addr + 32 * i, *reinterpret_cast<const float(*)[32]>(v + 32 * i));
  }
}

// row of an M=64 accumulator held by this thread's TMEM lane (lane quarter q, lane i):
// group parity (i >= 16) and row 16q + (i & 15)
__device__ __forceinline__ int m64_row(int q4, int lane) { return 16 * q4 + (lane & 15); }

__device__ __forceinline__ uint32_t m64_addr(uint32_t tmem, uint32_t col0, int g, uint32_t width) {
  return tmem + col0 + (uint32_t)(g >> 1) * width + ((uint32_t)((g & 1) * 16) << 16);
}

// ===========================================================================
// reverse walk of the backward pass
//
// TMEM: X [0,128) = P1 at chunk start, then Q2 summed over the chunk's groups;
// R [128,192) = Apref, then dpk; GD [192,256) = proj of the group (K and Q x hi | lo
// planes), then G; then GB, GA (M=64 suffix-state blocks) and DV [.., +64).
// Schedule per group g ({X} named barrier, [X] mbarrier):
//   control: {PK} Apref -> [APREF] ; {P1M, first group} ; G = P1m Pk, [BST] + dO Bst^T
//            -> [G] ; {W} dpk = V gBst^T + P1m^T W (in R) ;
//            {DA} dpk += tril^T dA -> [DPK] ; next group's Bst load and proj -> [PROJ] ;
//            Q2 += Pk W^T ; dV (+)= Pk gBst -> [PKFREE] (the last readers of the Pk
//            tile) ; gB += W^T dO ; gA += dA^T 1 (last group: -> [D2]) ;
// (critical MMAs first in each handoff: the tensor pipe runs them in order; the
// next group's Pk phase waits only for [PKFREE], not for the state updates)
//            chunk end: {Q2} dV += Q2m dO -> [OUT] ; next chunk's proj(0) ;
//            V/dO/Bst refill once every reader completed.
// P1m and tril are strictly lower triangular: the tau = t terms of Apref, G and
// dpk (pk_t, P1[t][t] pk_t, dA_t + P1[t][t] W_t) are added by the epilogue in fp32.
//   epilogue: [PROJ] Pk, plane sigmoids, [PKFREE] {PK} ;
//            [APREF] gB suffix copy (bf16 gBst), W {W} ; [G] gA suffix copy, dA {DA} ;
//            [DPK] dprojK ;
//            chunk end: [D2] Q2m {Q2} ; [OUT] dV rows {OUTFREE}.
enum { V3_QK = 0, V3_VO, V3_BST, V3_P1, V3_PROJ, V3_APREF, V3_G, V3_DPK, V3_PKFREE, V3_D2, V3_OUT, V3_TFREE,
       V3_FINAL, V3_COUNT };
// the reverse walk's epilogue layout (see bwd_rev_kernel): 8 warps of two tables each (fewer
// warps beside the MMA issuer, each phase's TMEM loads batched over both tables) measured 2 %
// faster than 16 warps of one table once the element-wise work ran on packed pairs
constexpr int REV_TPW = 2;
enum { N3_INIT = 1, N3_PK, N3_P1M, N3_W, N3_DA, N3_Q2, N3_OUTFREE, N3_ESYNC, N3_GSYNC, N3_GASYNC };
constexpr uint32_t B3_X = 0, B3_R = 128, B3_GD = 192, B3_ST = 256;

// TPW: tables per epilogue thread per 64-bucket group (1: 16 epilogue warps, 2: 8 epilogue warps
// and twice the registers per thread -- two warps beside the MMA issuer on its SM
// sub-partition instead of four, and each thread's work twice as wide).
// With TPW = 2 the block is three warpgroups: two of epilogue warps and a control warpgroup
// (the MMA / TMA issuer and three warps that only take the block's first and last barriers).
// Launched at 168 registers a thread (the limit of 384 threads on one SM), the control
// warpgroup drops to REV_CTL_REGS and the epilogue warps rise to REV_EPI_REGS:
// 4 x 128 + 8 x 184 = 1984 <= 12 x 168 = 2016 registers a lane for the block, and on each SM
// sub-partition (two epilogue warps, one control warp) 2 x 184 + 128 = 496 <= 512.
constexpr int REV_CTL_REGS = 128, REV_EPI_REGS = 184;
template <int TPW>
constexpr int rev_block_threads() { return TPW == 2 ? 32 * (16 / TPW + 4) : 32 * (16 / TPW + 1); }
static_assert(4 * REV_CTL_REGS + 8 * REV_EPI_REGS <= 12 * 168 && 2 * REV_EPI_REGS + REV_CTL_REGS <= 512,
              "reverse walk register split exceeds the block's launch registers");
template <int TPW>
__global__ void __launch_bounds__(rev_block_threads<TPW>(), 1) __maxnreg__(TPW == 1 ? 96 : 168) bwd_rev_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                        const __grid_constant__ CUtensorMap tmK,
                                                                        const __grid_constant__ CUtensorMap tmV,
                                                                        const __grid_constant__ CUtensorMap tmO,
                                                                        const __grid_constant__ CUtensorMap tmB,
                                                                        BwdArgs a) {
  // epilogue warps; threads of the named barriers (epilogue + issuer), of the epilogue
  constexpr int NE = 16 / TPW, NT = 32 * (NE + 1), NET = 32 * NE;
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = (unsigned char *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  const BwdSmem P = bwd_smem_plan(a.LP, a.S);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bars);
  // no static shared memory (it would cost a 1 KB aligned block): the TMEM base
  // and the wait control (abort flag, poll limit) live after the barriers
  uint32_t &s_tmem = *reinterpret_cast<uint32_t *>(sm + P.bars + 8 * V3_COUNT);
  int *s_abort = reinterpret_cast<int *>(sm + P.bars + 8 * V3_COUNT + 8);
  const uint32_t sbase = tc::smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x / a.nseg, seg = blockIdx.x % a.nseg;
  const int hn = n % a.H, bn = n / a.H;  // head and batch of stream n in the activation layout
  const int c_begin = seg * a.seg_chunks;
  const int nch = min(a.nchunks, c_begin + a.seg_chunks) - c_begin;
  const int S = a.S, NG = a.ngroups, nblk = (NG + 1) / 2;
  const size_t E = (size_t)S + (size_t)S * HD;
  const uint32_t T_GB = B3_ST, T_GA = B3_ST + 64 * nblk, T_DV = B3_ST + 80 * nblk;

  if (threadIdx.x == 0) {
    s_abort[0] = 0;
    s_abort[1] = (int)a.wait_limit;
    for (int i = 0; i < V3_COUNT; ++i) tc::mbar_init(&bars[i], 1);
    tc::fence_mbar_init();
  }
  if (warp == NE) tc::tmem_alloc(&s_tmem, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int *abort = s_abort;
  if constexpr (TPW == 2) {  // whole warpgroups: warps 0-7 epilogue, 8-11 control
    if (warp < NE)
      tc::setmaxnreg_inc<REV_EPI_REGS>();
    else
      tc::setmaxnreg_dec<REV_CTL_REGS>();
  }

  if (warp == NE) {
    // ===================== control warp: named-barrier steps as a warp, TMA + MMA issue by lane 0
    const bool leader = lane == 0;
    const uint32_t id_p1 = tc::idesc_bf16(C, C, false, false);
    const uint32_t id_proj = tc::idesc_bf16(C, 32, false, false);
    const uint32_t id_apref = tc::idesc_bf16(C, GW, false, true);
    const uint32_t id_gk = tc::idesc_bf16(C, GW, false, false);
    const uint32_t id_gm = tc::idesc_bf16(C, GW, false, true);
    const uint32_t id_mm = tc::idesc_bf16(C, GW, true, true);
    const uint32_t id_q2 = tc::idesc_bf16(C, C, false, false);
    const uint32_t id_st = tc::idesc_bf16(GW, HD, true, true);
    const uint32_t id_cs = tc::idesc_bf16(GW, 16, true, false);
    const uint32_t id_dv = tc::idesc_bf16(C, HD, false, true);
    const uint32_t oq = P.q, ok_ = P.k, ov = P.v, oo = P.o, obst = P.bst;
    const int nchunks = a.nchunks;
    auto load_qk = [=, &tmQ, &tmK](int c) {
      const int t0 = (c_begin + c) * C;
      tc::mbar_arrive_expect_tx(&bars[V3_QK], 2 * TILE);
      tc::tma_load_4d(sm + oq, &tmQ, &bars[V3_QK], 0, hn, t0, bn);
      tc::tma_load_4d(sm + ok_, &tmK, &bars[V3_QK], 0, hn, t0, bn);
    };
    auto load_vo = [=, &tmV, &tmO](int c) {
      const int t0 = (c_begin + c) * C;
      tc::mbar_arrive_expect_tx(&bars[V3_VO], 2 * TILE);
      tc::tma_load_4d(sm + ov, &tmV, &bars[V3_VO], 0, hn, t0, bn);
      tc::tma_load_4d(sm + oo, &tmO, &bars[V3_VO], 0, hn, t0, bn);
    };
    auto load_bst = [=, &tmB](int c, int g) {
      const int row = (int)(((size_t)n * nchunks + c_begin + c) * S + g * GW);
      tc::mbar_arrive_expect_tx(&bars[V3_BST], GW * 128);
      tc::tma_load_2d(sm + obst, &tmB, &bars[V3_BST], 0, row);
    };
    // proj of group g into GD (free between the epilogue's G read and the next G):
    // K x [planes_hi | planes_lo] in GD[0, 32), Q x the same in GD[32, 64)
    auto issue_proj = [=](int g) {
      const uint32_t pl = sbase + P.planes + (uint32_t)g * 32 * 128;
#pragma unroll
      for (int k0 = 0; k0 < HD; k0 += 16) {
        const uint64_t bp = tc::desc_kmajor(pl, k0, 0);
        tc::mma_bf16(tmem + B3_GD, tc::desc_kmajor(sbase + P.k, k0, 0), bp, id_proj, k0 > 0);
        tc::mma_bf16(tmem + B3_GD + 32, tc::desc_kmajor(sbase + P.q, k0, 0), bp, id_proj, k0 > 0);
      }
      tc::mma_commit(&bars[V3_PROJ]);
    };
    bool ok = true;
    if (leader && nch > 0) {
      load_qk(nch - 1);
      load_vo(nch - 1);
      load_bst(nch - 1, 0);
    }
    tc::named_bar_sync(N3_INIT, NT);  // planes, tril and suffix state are in place
    if (leader && nch > 0) {
      ok = tc::mbar_wait_sleep(&bars[V3_QK], 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_proj(0);
      }
    }
    for (int k = 0; k < nch; ++k) {
      const int c = nch - 1 - k;
      if (k > 0) tc::named_bar_sync(N3_OUTFREE, NT);  // dK and dV of the previous chunk are out
      ok = ok && !*abort;
      if (leader && ok) {
        ok = tc::mbar_wait_sleep(&bars[V3_VO], k & 1, abort);
        if (ok) {
          tc::tc_fence_after();
#pragma unroll
          for (int k0 = 0; k0 < HD; k0 += 16)
            tc::mma_bf16(tmem + B3_X, tc::desc_kmajor(sbase + P.o, k0, 0), tc::desc_kmajor(sbase + P.v, k0, 0), id_p1,
                         k0 > 0);
          tc::mma_commit(&bars[V3_P1]);
        }
      }
      for (int g = 0; g < NG; ++g) {
        const int u = k * NG + g;
        tc::named_bar_sync(N3_PK, NT);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + B3_R, tc::desc_kmajor(sbase + P.tril, k0, TILE),
                         tc::desc_mnmajor(sbase + P.pk, k0, 0), id_apref, k0 > 0);
          tc::mma_commit(&bars[V3_APREF]);
        }
        if (g == 0) {
          tc::named_bar_sync(N3_P1M, NT);
          ok = ok && !*abort;
        }
        if (leader && ok) {
          tc::tc_fence_after();
          // G = P1m Pk (needs only this group's Pk) + dO Bst^T once the state tile is in (the
          // load, issued at the previous group's {DA} step, is waited for only here, after
          // Apref and P1m Pk are queued: waiting for it before {PK} held the next Apref back)
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + B3_GD, tc::desc_kmajor(sbase + P.p1m, k0, TILE),
                         tc::desc_mnmajor(sbase + P.pk, k0, 0), id_gm, k0 > 0);
          ok = tc::mbar_wait_sleep(&bars[V3_BST], u & 1, abort);
          if (ok) {
            tc::tc_fence_after();
#pragma unroll
            for (int k0 = 0; k0 < HD; k0 += 16)
              tc::mma_bf16(tmem + B3_GD, tc::desc_kmajor(sbase + P.o, k0, 0), tc::desc_kmajor(sbase + P.bst, k0, 0),
                           id_gk, true);
            tc::mma_commit(&bars[V3_G]);
            if (g + 1 == NG && k + 1 < nch) load_qk(c - 1);  // the chunk's last proj was consumed before {PK}
          }
        }
        tc::named_bar_sync(N3_W, NT);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
          // dpk (in R, Apref consumed) = V gBst^T + P1m^T W: the W-dependent MMAs on the way to {DA}
#pragma unroll
          for (int k0 = 0; k0 < HD; k0 += 16)
            tc::mma_bf16(tmem + B3_R, tc::desc_kmajor(sbase + P.v, k0, 0), tc::desc_kmajor(sbase + P.gbst, k0, 0),
                         id_gk, k0 > 0);
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + B3_R, tc::desc_mnmajor(sbase + P.p1m, k0, TILE), tc::desc_mnmajor(sbase + P.w, k0, 0),
                         id_mm, true);
        }
        tc::named_bar_sync(N3_DA, NT);
        ok = ok && !*abort;
        if (leader && ok) {
          tc::tc_fence_after();
          // dpk += tril^T dA -> [DPK] ; the next group's chunk-start state (every epilogue
          // thread saw G complete before {DA}, so the Bst tile is free) ; next group's proj ->
          // [PROJ] ; Q2 (in X, summed over the chunk's groups) += Pk W^T and dV (+)= Pk gBst,
          // the last readers of the Pk tile -> [PKFREE] (the next group's Pk phase waits only
          // for these) ; then suffix gB += W^T dO and gA += dA^T 1 (the epilogue copies group
          // g+1's gB state after [APREF] and its gA state after [G] of g+1, by when these have
          // completed) ; last group: -> [D2] (every reader of W and dA: the epilogue then
          // overwrites them with Q2m)
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(tmem + B3_R, tc::desc_mnmajor(sbase + P.tril, k0, TILE),
                         tc::desc_mnmajor(sbase + P.da, k0, 0), id_mm, true);
          tc::mma_commit(&bars[V3_DPK]);
          if (g + 1 < NG) {
            load_bst(c, g + 1);
            issue_proj(g + 1);
          }
#pragma unroll
          for (int k0 = 0; k0 < GW; k0 += 16)
            tc::mma_bf16(tmem + B3_X, tc::desc_kmajor(sbase + P.pk, k0, 0), tc::desc_kmajor(sbase + P.w, k0, 0),
                         id_q2, g > 0 || k0 > 0);
#pragma unroll
          for (int k0 = 0; k0 < GW; k0 += 16)
            tc::mma_bf16(tmem + T_DV, tc::desc_kmajor(sbase + P.pk, k0, 0), tc::desc_mnmajor(sbase + P.gbst, k0, 0),
                         id_dv, g > 0 || k0 > 0);
          tc::mma_commit(&bars[V3_PKFREE]);
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(m64_addr(tmem, T_GB, g, 64), tc::desc_mnmajor(sbase + P.w, k0, 0),
                         tc::desc_mnmajor(sbase + P.o, k0, 0), id_st, true);
#pragma unroll
          for (int k0 = 0; k0 < C; k0 += 16)
            tc::mma_bf16(m64_addr(tmem, T_GA, g, 16), tc::desc_mnmajor(sbase + P.da, k0, 0),
                         tc::desc_kmajor(sbase + P.ones, k0, 16 * 128), id_cs, true);
          if (g + 1 == NG) tc::mma_commit(&bars[V3_D2]);
        }
      }
      tc::named_bar_sync(N3_Q2, NT);
      ok = ok && !*abort;
      if (leader && ok) {
        tc::tc_fence_after();
        // dV += Q2m dO (Q2m is the two-block tile [w | da])
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16)
          tc::mma_bf16(tmem + T_DV, tc::desc_kmajor(sbase + P.w, k0, TILE), tc::desc_mnmajor(sbase + P.o, k0, 0),
                       id_dv, true);
      }
      if (leader && ok) {
        tc::mma_commit(&bars[V3_OUT]);  // dV of the chunk complete
        if (k + 1 < nch) {
          ok = tc::mbar_wait_sleep(&bars[V3_QK], (k + 1) & 1, abort);
          if (ok) {
            tc::tc_fence_after();
            issue_proj(0);
            // V, dO and the Bst tile are free once every MMA issued so far has completed
            tc::mma_commit(&bars[V3_TFREE]);
            ok = tc::mbar_wait_sleep(&bars[V3_TFREE], k & 1, abort);
            if (ok) {
              load_vo(c - 1);
              load_bst(c - 1, 0);
            }
          }
        }
      }
    }
    if (leader && nch > 0) {
      tc::mma_commit(&bars[V3_FINAL]);
      if (!tc::mbar_wait_drain(&bars[V3_FINAL], 0)) atomicExch(a.err, 2);
    }
    __syncwarp();
  } else if (warp < NE) {
    // ============================== epilogue warps: row t, column slot hq
    // (NE = 16/TPW warps, four per TMEM lane quarter; in a 64-bucket group slot hq owns
    // tables 4g + TPW hq + [0, TPW): buckets and d columns [TB hq, TB hq + TB), TB = 16 TPW;
    // in a 128-column token tile, columns [CW hq, CW hq + CW), CW = 32 TPW)
    constexpr int TB = 16 * TPW, CW = 32 * TPW;
    const int q4 = warp & 3, hq = warp >> 2;
    const int t = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t blk = (uint32_t)((CW * hq) >> 6) * TILE;  // 64-column block holding this slot's columns
    const int ch0 = ((CW * hq) & 63) >> 3;                    // its first 16-byte chunk inside that block
    const int mrow = m64_row(q4, lane), mpar = lane >> 4;
    float *sA = reinterpret_cast<float *>(sm + P.a0);
    float *sGA = reinterpret_cast<float *>(sm + P.ga);
    float *sDiag = reinterpret_cast<float *>(sm + P.diag);
    const float *sst = a.suf_state ? a.suf_state + ((size_t)n * a.nseg + seg) * E : nullptr;
    for (int i = threadIdx.x; i < a.LP * HD; i += NET) {  // planes = hi + lo, both bf16
      const int j = i / HD, d = i % HD;
      const float pv = a.planes[(size_t)d * a.LP + j];
      const __nv_bfloat16 hi = __float2bfloat16(pv);
      const int row = 32 * (j >> 4) + (j & 15);  // hi row of plane j; its residual 16 rows on
      const uint32_t cb = (uint32_t)(d & 7) * 2;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.planes + tc::sw128_off(row, d >> 3) + cb) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.planes + tc::sw128_off(row + 16, d >> 3) + cb) =
          __float2bfloat16(pv - __bfloat162float(hi));
    }
    {
      // strictly lower triangle: tril[t][tau] = tau < t (the diagonal terms are added in fp32)
      float v[8];
      for (int ch = 0; ch < CW / 8; ++ch) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = (CW * hq + ch * 8 + e) < t ? 1.f : 0.f;
        tc::st_row_chunk(sbase + P.tril + blk, t, ch0 + ch, v);
      }
    }
    for (int i = threadIdx.x; i < 16 * C / 2; i += NET)  // bf16 ones, any layout
      *reinterpret_cast<uint32_t *>(sm + P.ones + 4 * i) = 0x3F803F80u;
    for (int b = 0; b < nblk; ++b) {  // suffix state at the segment end (zero: segment-local walk) -> TMEM
      const int g = 2 * b + mpar;
      float v[TB];
      if (g < NG && sst != nullptr) {
        const float *src = sst + S + (size_t)(g * GW + mrow) * HD + TB * hq;
#pragma unroll
        for (int i = 0; i < TB; ++i) v[i] = src[i];
      } else {
#pragma unroll
        for (int i = 0; i < TB; ++i) v[i] = 0.f;
      }
      tmem_stn<TB>(tmem + lane_off + T_GB + 64 * b + TB * hq, v);
      if (hq == 0) tc::tmem_st1(tmem + lane_off + T_GA + 16 * b, g < NG && sst != nullptr ? sst[g * GW + mrow] : 0.f);
    }
    tc::tmem_wait_st();
    tc::fence_async_smem();
    tc::tc_fence_before();
    tc::named_bar_sync(N3_INIT, NT);

    bool ok = true;
    for (int k = 0; k < nch; ++k) {
      const int c = nch - 1 - k, cg = c_begin + c, tok0 = cg * C;
      const int nt = min(C, a.T - tok0);
      // chunk-start A + eps (stored by the forward walk)
      for (int s = threadIdx.x; s < S; s += NET) sA[s] = a.chunkA[((size_t)n * a.nchunks + cg) * S + s];
      tc::named_bar_sync(N3_ESYNC, NET);  // sA visible to all epilogue threads
      for (int g = 0; g < NG; ++g) {
        const int u = k * NG + g;
        // tanh, plane sigmoids of the slot's tables ; 1/(A + eps), then dpq, then the diagonal terms ;
        // the K-side corner probabilities (unmasked), computed once and used by every phase
        float thK[4 * TPW], thQ[4 * TPW], qK[4 * TPW], qQ[4 * TPW], inv[TB], pkc[TB];
        // ---- Pk (once [PKFREE] of the previous group says the Pk tile is read)
        if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_PROJ], u & 1, abort));
        tc::tc_fence_after();
        if (ok) {
          float loK[4 * TPW], loQ[4 * TPW];  // the residual-plane halves
          tmem_ldn<4 * TPW>(tmem + lane_off + B3_GD + 4 * TPW * hq, thK);
          tmem_ldn<4 * TPW>(tmem + lane_off + B3_GD + 16 + 4 * TPW * hq, loK);
          tmem_ldn<4 * TPW>(tmem + lane_off + B3_GD + 32 + 4 * TPW * hq, thQ);
          tmem_ldn<4 * TPW>(tmem + lane_off + B3_GD + 48 + 4 * TPW * hq, loQ);
          tc::tmem_wait_ld();
          vadd<4 * TPW>(thK, loK);
          vadd<4 * TPW>(thQ, loQ);
#pragma unroll
          for (int i = 0; i < 4 * TPW; ++i) {
            thK[i] = tanh_fast(thK[i]);
            thQ[i] = tanh_fast(thQ[i]);
          }
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) {
            plane_sigmoids(thK + 4 * tb, a.scale, a.poly, qK + 4 * tb);
            plane_sigmoids(thQ + 4 * tb, a.scale, a.poly, qQ + 4 * tb);
            corner_probs(qK + 4 * tb, pkc + 16 * tb);
          }
        }
        if (ok && u > 0) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_PKFREE], (u - 1) & 1, abort));
        tc::tc_fence_after();
        if (ok) {
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) {  // one table at a time (registers)
            float pr[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) pr[i] = t < nt ? pkc[16 * tb + i] : 0.f;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
              tc::st_row_chunk(sbase + P.pk, t, 2 * (TPW * hq + tb) + ch, pr + 8 * ch);
          }
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(N3_PK, NT);
        if (g == 0) {
          // P1m after the first group's Pk: the Pk work overlaps the chunk's V / dO loads and
          // the dO V^T MMA (the control warp takes {PK} before {P1M})
          // ---- P1m = tril-masked dO V^T
          if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_P1], k & 1, abort));
          tc::tc_fence_after();
          if (ok) {
            // 32 columns at a time; column runs all at or above the diagonal store zeros without
            // reading TMEM
#pragma unroll
            for (int h = 0; h < CW / 32; ++h) {
              const int col0 = CW * hq + 32 * h;  // first token column of this run
              float v[32];
              if (col0 < 32 * q4 + 32) {
                tc::tmem_ld32(tmem + lane_off + B3_X + col0, v);
                tc::tmem_wait_ld();
                if (col0 + 32 > 32 * q4) {  // the run holds this row's diagonal (col0 == 32 q4)
                  float dg = 0.f;
#pragma unroll
                  for (int i = 0; i < 32; ++i) dg = i == lane ? v[i] : dg;
                  sDiag[t] = dg;  // fp32 diagonal P1[t][t] (the exact-diagonal terms below)
#pragma unroll
                  for (int i = 0; i < 32; ++i)  // strictly lower: the diagonal term is added in fp32
                    if (i >= lane) v[i] = 0.f;
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
              }
#pragma unroll
              for (int ch = 0; ch < 4; ++ch) tc::st_row_chunk(sbase + P.p1m + blk, t, ch0 + 4 * h + ch, v + 8 * ch);
            }
          }
          tc::fence_async_smem();
          tc::tc_fence_before();
          tc::named_bar_arrive(N3_P1M, NT);
        }
        // at the first group: the fp32 diagonal complete before any read
        if (g == 0) tc::named_bar_sync(N3_GSYNC, NET);
        // ---- suffix gB copy of group g (bf16 gBst: the previous group's MMAs, the last readers
        // of the gBst tile and writers of the gB blocks, completed before Apref) ; W = pq / (A + eps)
        if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_APREF], u & 1, abort));
        tc::tc_fence_after();
        if (ok) {
          // both TMEM loads first, the Q-side corner probabilities while they are in flight
          float bv[TB], ap[TB], w[TB];
          tmem_ldn<TB>(tmem + lane_off + T_GB + 64 * (g >> 1) + TB * hq, bv);
          tmem_ldn<TB>(tmem + lane_off + B3_R + TB * hq, ap);
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) corner_probs(qQ + 4 * tb, w + 16 * tb);
          tc::tmem_wait_ld();
          if (mpar == (g & 1)) {
#pragma unroll
            for (int ch = 0; ch < 2 * TPW; ++ch) tc::st_row_chunk(sbase + P.gbst, mrow, 2 * TPW * hq + ch, bv + 8 * ch);
          }
          if (t < nt) vadd<TB>(ap, pkc);  // the MMA summed tau < t: the diagonal pk_t in fp32
          add_shared_row<TB>(sbase + P.a0 + 4 * (g * GW + TB * hq), ap);  // + (A + eps) at chunk start
          rcp_n<TB>(ap, inv, a.batch_rcp);
          if (t >= nt) {  // rows past the end: W, dpq, dA and the diagonal terms below all vanish
#pragma unroll
            for (int i = 0; i < TB; ++i) inv[i] = 0.f;
          }
          vmul<TB>(w, inv);
#pragma unroll
          for (int ch = 0; ch < 2 * TPW; ++ch) tc::st_row_chunk(sbase + P.w, t, 2 * TPW * hq + ch, w + 8 * ch);
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(N3_W, NT);
        // ---- suffix gA copy of group g ; dA = -W G / (A + eps)
        if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_G], u & 1, abort));
        tc::tc_fence_after();
        if (ok) {
          const bool live = t < nt;
          // Exact diagonal (tau = t), in fp32: the MMAs with P1m and tril cover tau < t only.
          // G gets P1[t][t] pk_t ; dpk gets dA_t + P1[t][t] W_t = W_t (P1[t][t] - dpq_t), which
          // cancels exactly at the first tokens (carried to the dpk phase in inv).
          // (rows past the end have inv = 0, so W, dpq, dA and these terms are zero there)
          // TMEM loads first (G; the gA suffix copy: G of this group completed after the
          // previous group's gA update, so the block is settled), pq while they are in flight
          float G[TB], pq[TB], av = 0.f;
          tmem_ldn<TB>(tmem + lane_off + B3_GD + TB * hq, G);
          if (hq == 0) tc::tmem_ld1(tmem + lane_off + T_GA + 16 * (g >> 1), av);
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) corner_probs(qQ + 4 * tb, pq + 16 * tb);
          tc::tmem_wait_ld();
          if (hq == 0 && mpar == (g & 1)) sGA[(g & 1) * GW + mrow] = av;
          const float p1 = sDiag[t];
          const float2 p12 = dup2(p1);
          uint32_t pw[2 * TPW];  // d proj_Q of the slot's tables, bf16 pairs
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) {  // one table at a time (registers)
            float dpq[16];
            float *Gt = G + 16 * tb, *pqt = pq + 16 * tb, *iv = inv + 16 * tb;
            const float *pk = pkc + 16 * tb;
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float2 v = ld2(iv, i);
              const float2 w = __fmul2_rn(ld2(pqt, i), v);
              const float2 dq = __fmul2_rn(__ffma2_rn(p12, ld2(pk, i), ld2(Gt, i)), v);
              const float2 da = __fmul2_rn(make_float2(-w.x, -w.y), dq);
              st2(dpq, i, dq);
              st2(Gt, i, da);
              st2(iv, i, __ffma2_rn(p12, w, da));  // the diagonal term, carried to the dpk phase
            }
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
              tc::st_row_chunk(sbase + P.da, t, 2 * (TPW * hq + tb) + ch, Gt + 8 * ch);
            float dp[4];
            table_probs_bwd(pqt, dpq, qQ + 4 * tb, thQ + 4 * tb, a.scale, dp);
            pw[2 * tb] = tc::pack_bf16(dp[0], dp[1]);
            pw[2 * tb + 1] = tc::pack_bf16(dp[2], dp[3]);
          }
          if (a.dprojQ != nullptr && live) {  // d proj_Q of the slot's tables -> the fix-up's dQ
            __nv_bfloat16 *dst = a.dprojQ + ((size_t)n * a.T + tok0 + t) * HD + 16 * g + 4 * TPW * hq;
            if constexpr (TPW == 1)
              *reinterpret_cast<uint2 *>(dst) = make_uint2(pw[0], pw[1]);
            else
              *reinterpret_cast<uint4 *>(dst) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
          }
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        tc::named_bar_arrive(N3_DA, NT);
        // sGA (double-buffered by group parity: a warp may write the next group's copy while
        // a slower one still reads this one) complete before any read
        tc::named_bar_sync(N3_GASYNC, NET);
        // ---- dpk -> d proj_K
        if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_DPK], u & 1, abort));
        tc::tc_fence_after();
        if (ok) {
          // the TMEM load first, the suffix gA row from shared memory while it is in flight
          float dpk[TB], ga[TB];
          tmem_ldn<TB>(tmem + lane_off + B3_R + TB * hq, dpk);
          load_shared_row<TB>(sbase + P.ga + 4 * ((g & 1) * GW + TB * hq), ga);
          tc::tmem_wait_ld();
          vadd<TB>(dpk, ga);   // + suffix gA
          vadd<TB>(dpk, inv);  // + the fp32 diagonal term
#pragma unroll
          for (int tb = 0; tb < TPW; ++tb) {
            float dp[4];
            table_probs_bwd(pkc + 16 * tb, dpk + 16 * tb, qK + 4 * tb, thK + 4 * tb, a.scale, dp);
            // segment-local d proj_K of table 4g + TPW hq + tb, fp32, to the fix-up (rows past
            // the end too: the chunk's block is read whole)
            *reinterpret_cast<float4 *>(a.dprojK +
                                        (((size_t)n * a.nchunks + cg) * (a.LP / 4) + 4 * g + TPW * hq + tb) * (C * 4) +
                                        4 * t) = make_float4(dp[0], dp[1], dp[2], dp[3]);
          }
        }
      }
      // ---- Q2m[tau = t][t'] = Q2 (summed over the groups) for t' >= tau ; blocks: w (t' < 64),
      // da (t' >= 64), once Q2 and every reader of w and dA completed
      // (32-column runs all below the diagonal store zeros without reading TMEM)
      if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_D2], k & 1, abort));
      tc::tc_fence_after();
      if (ok) {
#pragma unroll
        for (int h = 0; h < CW / 32; ++h) {
          const int col0 = CW * hq + 32 * h;  // first token column of this run
          float v[32];
          if (col0 + 32 > 32 * q4) {
            tc::tmem_ld32(tmem + lane_off + B3_X + col0, v);
            tc::tmem_wait_ld();
            if (col0 < 32 * q4 + 32) {  // the run holds this row's diagonal
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < lane) v[i] = 0.f;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tc::st_row_chunk(sbase + P.w + blk, t, ch0 + 4 * h + ch, v + 8 * ch);
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(N3_Q2, NT);
      // ---- dV rows
      if (ok) ok = tc::warp_all(tc::mbar_wait_sleep(&bars[V3_OUT], k & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        float vv[TB];
        tmem_ldn<TB>(tmem + lane_off + T_DV + TB * hq, vv);
        tc::tmem_wait_ld();
        if (t < nt) {
          __nv_bfloat16 *dv = a.dV + act_row(bn, hn, tok0 + t, a.T, a.H) + TB * hq;
#pragma unroll
          for (int ch = 0; ch < TB / 8; ++ch) st_bf16x8_global(dv + 8 * ch, vv + 8 * ch);
        }
      }
      tc::tc_fence_before();
      if (k + 1 < nch) tc::named_bar_arrive(N3_OUTFREE, NT);
    }
    // ---- segment-local gradient totals (suffix state at the segment start; OUT of the last
    // chunk covers every accumulation)
    if (a.tot != nullptr) {
      float *rec = a.tot + ((size_t)n * a.nseg + seg) * E;
      if (ok && nch > 0) {
        for (int b = 0; b < nblk; ++b) {
          const int g = 2 * b + mpar;
          float bv[TB], av;
          tmem_ldn<TB>(tmem + lane_off + T_GB + 64 * b + TB * hq, bv);
          tc::tmem_ld1(tmem + lane_off + T_GA + 16 * b, av);
          tc::tmem_wait_ld();
          if (g < NG) {
            float *dst = rec + S + (size_t)(g * GW + mrow) * HD + TB * hq;
#pragma unroll
            for (int i = 0; i < TB; ++i) dst[i] = bv[i];
            if (hq == 0) rec[g * GW + mrow] = av;
          }
        }
      } else if (nch == 0) {
        for (int i = threadIdx.x; i < (int)E; i += NET) rec[i] = 0.f;
      }
    }
    if (!ok && lane == 0) atomicExch(a.err, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NE) {
    if (s_abort[0] && lane == 0) atomicExch(a.err, 1);
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Suffix fix-up of the backward.  The reverse walk runs each segment with a
// zero suffix state at its end (segment-local gradient states); the true
// suffix of a segment, gA_in / gB_in (later segments + the carried-in state,
// from the reverse chunk_scan of the walks' totals), enters the gradients
// linearly:
//   dpk_t[s] += gA_in[s] + V_t . gB_in[s]   (d proj_K: softmax backward of it, plus
//                                            the walk's local d proj_K, fp32)
//   dV_t     += sum_s pk_t[s] gB_in[s]
// then dK = d proj_K planes, dQ = d proj_Q planes (planes and d proj_K as
// bf16 hi + lo pairs).  No chunk depends on
// another, so one CTA per (stream, segment) loops over its chunks with the
// segment's gB_in held in shared memory (bf16, the MMA operand for both
// products).
// The outputs leave through shared memory and TMA tile stores (dK and dQ rows staged in
// the d proj tiles, dV rows in the tile the walk's dV came in through), not per-thread
// 16-byte stores that split every warp instruction into 32 row transactions.
//   control: [KV] proj = K (planes_hi + planes_lo) -> [PROJ] ;
//            {OUTFREE} store the previous chunk's dK, dV, dQ tiles ; Dfix = V gB_in^T -> [DPK] ;
//            dQ = dprojQ planes -> [TFREE] ; once the stores have read the tiles: this chunk's
//            dV tile -> [DVL] and the walk's fp32 d proj_K tile into the d proj tiles -> [DPL] ;
//            {PK} dV = Pk gB_in ; {DP} dK = dproj planes -> [OUT]
//   epilogue: [PROJ] Pk {PK} ; [DPK] [DPL] dproj = softmax bwd of (Dfix + gA_in) + the walk's,
//             as hi + lo bf16 into the d proj tiles once every thread read its fp32 values {DP} ;
//             [OUT] [DVL] dK, dV += , dQ rows into the tiles {OUTFREE}
enum { VF_KV = 0, VF_DVL, VF_PROJ, VF_DPK, VF_OUT, VF_TFREE, VF_DPL, VF_FINAL, VF_COUNT };
enum { NF_ESYNC = 5 };  // epilogue-only barrier
enum { NF_INIT = 1, NF_PK, NF_DP, NF_OUTFREE };

struct FixSmem {
  uint32_t k, v, dq, dvl, pk, gb, dp, dplo, planes, plo, ga, bars, total;
};

__host__ __device__ __forceinline__ FixSmem fix_smem_plan(int LP, int S) {
  FixSmem m;
  uint32_t o = 0;
  m.k = o; o += TILE;
  m.v = o; o += TILE;
  m.dq = o; o += TILE;
  m.dvl = o; o += TILE;                      // the walk's dV rows in, dV rows out
  m.pk = o; o += (uint32_t)(S / 64) * TILE;  // [128 t x S] K-major, 64-column blocks
  m.gb = o; o += (uint32_t)S * 128;          // [S rows x 64 d] bf16
  m.dp = o; o += TILE;                       // d proj_K = hi + lo, bf16 tiles; then dK, dQ rows out
  m.dplo = o; o += TILE;
  m.planes = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.plo = o; o += (uint32_t)align_up((size_t)LP * 128, 1024);
  m.ga = o; o += (uint32_t)align_up((size_t)S * 4, 128);
  m.bars = o; o += 256;
  m.total = o + 1024;
  return m;
}

// TMEM: projK [0,64) ; Dfix [64, 64+S) ; dQ, dK, dV 64 columns each after it
constexpr uint32_t FX_PJ = 0, FX_D = 64;

__global__ void __launch_bounds__(NTHR, 1) bwd_fix_kernel(const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV,
                                                          const __grid_constant__ CUtensorMap tmDQ,
                                                          const __grid_constant__ CUtensorMap tmVL,
                                                          const __grid_constant__ CUtensorMap tmOK,
                                                          const __grid_constant__ CUtensorMap tmOV,
                                                          const __grid_constant__ CUtensorMap tmOQ, BwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char *sm = (unsigned char *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  const FixSmem P = fix_smem_plan(a.LP, a.S);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bars);
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort[2];  // wait control: abort flag, poll limit
  const uint32_t sbase = tc::smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x / a.nseg, seg = blockIdx.x % a.nseg;
  const int hn = n % a.H, bn = n / a.H;  // head and batch of stream n in the activation layout
  const int c_begin = seg * a.seg_chunks;
  const int nch = min(a.nchunks, c_begin + a.seg_chunks) - c_begin;
  const int S = a.S, LP = a.LP;
  const size_t E = (size_t)S + (size_t)S * HD;
  const uint32_t T_DQ = FX_D + S, T_DK = T_DQ + 64, T_DV = T_DK + 64;

  if (threadIdx.x == 0) {
    s_abort[0] = 0;
    s_abort[1] = (int)a.wait_limit;
    for (int i = 0; i < VF_COUNT; ++i) tc::mbar_init(&bars[i], 1);
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
    const uint32_t id_vg = tc::idesc_bf16(C, S, false, false);
    const uint32_t id_d = tc::idesc_bf16(C, HD, false, true);
    const uint32_t ok_ = P.k, ov = P.v, oq = P.dq;
    auto load = [=, &tmK, &tmV, &tmDQ](int c) {
      const int t0 = (c_begin + c) * C;
      tc::mbar_arrive_expect_tx(&bars[VF_KV], 3 * TILE);
      tc::tma_load_4d(sm + ok_, &tmK, &bars[VF_KV], 0, hn, t0, bn);
      tc::tma_load_4d(sm + ov, &tmV, &bars[VF_KV], 0, hn, t0, bn);
      tc::tma_load_3d(sm + oq, &tmDQ, &bars[VF_KV], 0, t0, n);  // d proj_Q: [N, T, 64] workspace
    };
    auto load_dvl = [=, &tmVL](int c) {
      tc::mbar_arrive_expect_tx(&bars[VF_DVL], TILE);
      tc::tma_load_4d(sm + P.dvl, &tmVL, &bars[VF_DVL], 0, hn, (c_begin + c) * C, bn);
    };
    // the walk's fp32 d proj_K block of chunk c (LP/4 tables x 128 tokens x 16 bytes, contiguous)
    // into the (free, adjacent) d proj tiles
    auto load_dpl = [=](int c) {
      const uint32_t bytes = (uint32_t)LP * C * 4;
      tc::mbar_arrive_expect_tx(&bars[VF_DPL], bytes);
      tc::bulk_load(sm + P.dp, a.dprojK + ((size_t)n * a.nchunks + c_begin + c) * LP * C, bytes, &bars[VF_DPL]);
    };
    auto store_out = [=, &tmOK, &tmOV, &tmOQ](int c) {
      const int t0 = (c_begin + c) * C;
      tc::tma_store_4d(&tmOK, sm + P.dp, 0, hn, t0, bn);
      tc::tma_store_4d(&tmOV, sm + P.dvl, 0, hn, t0, bn);
      tc::tma_store_4d(&tmOQ, sm + P.dplo, 0, hn, t0, bn);
      tc::bulk_commit();
    };
    auto issue_proj = [=]() {  // proj = K planes for the chunk in the tiles
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int k0 = 0; k0 < HD; k0 += 16)
          tc::mma_bf16(tmem + FX_PJ, tc::desc_kmajor(sbase + P.k, k0, 0),
                       tc::desc_kmajor(sbase + (part ? P.plo : P.planes), k0, 0), id_proj, part > 0 || k0 > 0);
      tc::mma_commit(&bars[VF_PROJ]);
    };
    auto issue_dfix = [=]() {  // Dfix = V gB_in^T
#pragma unroll
      for (int k0 = 0; k0 < HD; k0 += 16)
        tc::mma_bf16(tmem + FX_D, tc::desc_kmajor(sbase + P.v, k0, 0), tc::desc_kmajor(sbase + P.gb, k0, 0), id_vg,
                     k0 > 0);
      tc::mma_commit(&bars[VF_DPK]);
    };
    // D = A (planes_hi + planes_lo) [+ A_lo planes_hi]
    auto issue_planes = [=](uint32_t d_col, uint32_t a_tile, uint32_t a_lo) {
      for (int part = 0; part < 3; ++part) {
        if (part == 2 && a_lo == 0) break;
        for (int k0 = 0; k0 < LP; k0 += 16)
          tc::mma_bf16(tmem + d_col, tc::desc_kmajor(sbase + (part == 2 ? a_lo : a_tile), k0, 0),
                       tc::desc_mnmajor(sbase + (part == 1 ? P.plo : P.planes), k0, 0), id_d, part > 0 || k0 > 0);
      }
    };
    bool ok = true;
    if (leader && nch > 0) {
      load(0);
      load_dvl(0);
      load_dpl(0);
    }
    tc::named_bar_sync(NF_INIT, NTHR);  // planes, gB_in, gA_in in shared memory
    if (leader && nch > 0) {
      ok = tc::mbar_wait(&bars[VF_KV], 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_proj();
        issue_dfix();
      }
    }
    for (int c = 0; c < nch; ++c) {
      if (c > 0) {
        tc::named_bar_sync(NF_OUTFREE, NTHR);  // the previous chunk's dK, dV, dQ rows are in the tiles
        ok = ok && !*abort;
        if (leader && ok) {
          store_out(c - 1);
          tc::tc_fence_after();
          issue_dfix();
        }
      }
      if (leader && ok) {
        tc::tc_fence_after();
        issue_planes(T_DQ, P.dq, 0);
        tc::mma_commit(&bars[VF_TFREE]);  // every reader of the K, V, dprojQ tiles issued
        if (c > 0) {
          // the stores have read the tiles: this chunk's dV rows and d proj_K tile may come in
          tc::bulk_wait_read();
          load_dvl(c);
          load_dpl(c);
        }
      }
      tc::named_bar_sync(NF_PK, NTHR);
      ok = ok && !*abort;
      if (leader && ok) {
        ok = tc::mbar_wait(&bars[VF_TFREE], c & 1, abort);
        if (ok && c + 1 < nch) load(c + 1);
        tc::tc_fence_after();
        for (int k0 = 0; k0 < S; k0 += 16)
          tc::mma_bf16(tmem + T_DV, tc::desc_kmajor(sbase + P.pk, k0, TILE), tc::desc_mnmajor(sbase + P.gb, k0, 0),
                       id_d, k0 > 0);
      }
      tc::named_bar_sync(NF_DP, NTHR);
      ok = ok && !*abort;
      if (leader && ok) {
        tc::tc_fence_after();
        issue_planes(T_DK, P.dp, P.dplo);
        tc::mma_commit(&bars[VF_OUT]);
        if (c + 1 < nch) {
          ok = tc::mbar_wait(&bars[VF_KV], (c + 1) & 1, abort);
          if (ok) {
            tc::tc_fence_after();
            issue_proj();
          }
        }
      }
    }
    if (nch > 0) {
      tc::named_bar_sync(NF_OUTFREE, NTHR);  // the last chunk's rows are in the tiles
      ok = ok && !*abort;
      if (leader && ok) store_out(nch - 1);
    }
    if (leader && nch > 0) {
      tc::bulk_wait();  // stores complete (and shared memory read) before the CTA exits
      tc::mma_commit(&bars[VF_FINAL]);
      if (!tc::mbar_wait_drain(&bars[VF_FINAL], 0)) atomicExch(a.err, 2);
    }
    __syncwarp();
  } else {
    // ============================== epilogue warps: row t, column quarter hq
    // (quarter hq owns the tables [tq*hq, tq*hq + tq), tq = L/4: buckets [16 tq hq, +16 tq))
    const int q4 = warp & 3, hq = warp >> 2;
    const int t = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int tq = a.L / 4;
    const float *sin = a.suf_state + ((size_t)n * a.nseg + seg) * E;
    float *sGA = reinterpret_cast<float *>(sm + P.ga);
    for (int i = threadIdx.x; i < LP * HD; i += NEPI_T) {  // planes = hi + lo, both bf16
      const int j = i / HD, d = i % HD;
      const float pv = a.planes[(size_t)d * LP + j];
      const __nv_bfloat16 hi = __float2bfloat16(pv);
      const uint32_t off = tc::sw128_off(j, d >> 3) + (d & 7) * 2;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.planes + off) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(sm + P.plo + off) = __float2bfloat16(pv - __bfloat162float(hi));
    }
    const float *seedB = a.seedB ? a.seedB + (size_t)n * S * HD : nullptr;
    const float *seedA = a.seedA ? a.seedA + (size_t)n * S : nullptr;
    for (int i = threadIdx.x; i < S * 8; i += NEPI_T) {  // gB_in (bf16 rows s), 8 values per step
      const int sr = i >> 3, ch = i & 7;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[e] = sin[S + (size_t)sr * HD + ch * 8 + e] + (seedB ? seedB[(size_t)sr * HD + ch * 8 + e] : 0.f);
      tc::st_row_chunk(sbase + P.gb, sr, ch, v);
    }
    for (int s = threadIdx.x; s < S; s += NEPI_T) sGA[s] = sin[s] + (seedA ? seedA[s] : 0.f);
    tc::fence_async_smem();
    tc::named_bar_sync(NF_INIT, NTHR);

    bool ok = true;
    for (int c = 0; c < nch; ++c) {
      const int tok0 = (c_begin + c) * C;
      const int nt = min(C, a.T - tok0);
      float thK[16], qK[16];  // tanh and plane sigmoids of this quarter's tables (up to 4)
      // ---- Pk of this quarter's buckets
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[VF_PROJ], c & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        if (tq == 4) {
          float pj[16];
          tc::tmem_ld16(tmem + lane_off + FX_PJ + 16 * hq, pj);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) thK[i] = tanh_fast(pj[i]);
        } else {
          float pj[8];
          tc::tmem_ld8(tmem + lane_off + FX_PJ + 8 * hq, pj);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) thK[i] = tanh_fast(pj[i]);
#pragma unroll
          for (int i = 8; i < 16; ++i) thK[i] = 0.f;
        }
#pragma unroll
        for (int tb = 0; tb < 4; tb += 2) {  // tables in pairs (tq is 2 or 4)
          if (tb < tq) {
            plane_sigmoids(thK + 4 * tb, a.scale, a.poly, qK + 4 * tb);
            plane_sigmoids(thK + 4 * tb + 4, a.scale, a.poly, qK + 4 * tb + 4);
            float pr[32];
            corner_probs2(qK + 4 * tb, qK + 4 * tb + 4, pr, pr + 16);
            if (t >= nt) {
#pragma unroll
              for (int i = 0; i < 32; ++i) pr[i] = 0.f;
            }
            const int b0 = 16 * (tq * hq + tb);  // first bucket of the table pair
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
              tc::st_row_chunk(sbase + P.pk + (uint32_t)(b0 >> 6) * TILE, t, ((b0 & 63) >> 3) + ch, pr + 8 * ch);
          }
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(NF_PK, NTHR);
      // ---- dproj_fix = softmax bwd of (V gB_in^T + gA_in) + the walk's segment-local d proj_K
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[VF_DPK], c & 1, abort));
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[VF_DPL], c & 1, abort));
      tc::tc_fence_after();
      float4 loc[4];  // the walk's d proj_K of this slot's tables (table-major block, 16 B per row)
#pragma unroll
      for (int tb = 0; tb < 4; ++tb)
        loc[tb] = ok && tb < tq ? tc::ld_shared_f4(sbase + P.dp + (uint32_t)((tq * hq + tb) * C + t) * 16)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      tc::named_bar_sync(NF_ESYNC, NEPI_T);  // every fp32 value read before the tiles are rewritten
      if (ok) {
#pragma unroll
        for (int tb = 0; tb < 4; ++tb) {
          if (tb < tq) {
            const int b0 = 16 * (tq * hq + tb);
            float g16[16], p16[16], dp[4];
            tc::tmem_ld16(tmem + lane_off + FX_D + b0, g16);
            tc::tmem_wait_ld();
            add_shared_row<16>(sbase + P.ga + 4 * b0, g16);
            corner_probs(qK + 4 * tb, p16);
            table_probs_bwd(p16, g16, qK + 4 * tb, thK + 4 * tb, a.scale, dp);
            const int j = 4 * (tq * hq + tb);  // first projection column of the table
            // then hi + lo bf16 for the dK MMA
            dp[0] += loc[tb].x;
            dp[1] += loc[tb].y;
            dp[2] += loc[tb].z;
            dp[3] += loc[tb].w;
            float lo[4];
            bf16r2(dp[0], dp[1], lo[0], lo[1]);
            bf16r2(dp[2], dp[3], lo[2], lo[3]);
#pragma unroll
            for (int i = 0; i < 4; ++i) lo[i] = dp[i] - lo[i];
            tc::st_row_half(sbase + P.dp, t, j >> 3, (j >> 2) & 1, dp);
            tc::st_row_half(sbase + P.dplo, t, j >> 3, (j >> 2) & 1, lo);
          }
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(NF_DP, NTHR);
      // ---- dK, dV += dV_fix, dQ rows (row t, d in [16hq, 16hq+16)) into the output tiles:
      // dK into the d proj_K hi tile and dQ into its lo tile (both read by the dK MMAs, complete
      // at [OUT]), dV in place in the tile holding the walk's dV rows
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[VF_OUT], c & 1, abort));
      if (ok) ok = tc::warp_all(tc::mbar_wait(&bars[VF_DVL], c & 1, abort));
      tc::tc_fence_after();
      if (ok) {
        float vq[16], vk[16], vv[16];
        tc::tmem_ld16(tmem + lane_off + T_DQ + 16 * hq, vq);
        tc::tmem_ld16(tmem + lane_off + T_DK + 16 * hq, vk);
        tc::tmem_ld16(tmem + lane_off + T_DV + 16 * hq, vv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          const uint32_t off = tc::sw128_off(t, 2 * hq + ch);
          const uint4 v4 = *reinterpret_cast<const uint4 *>(sm + P.dvl + off);
          const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            vv[8 * ch + 2 * e] += __uint_as_float(vw[e] << 16);
            vv[8 * ch + 2 * e + 1] += __uint_as_float(vw[e] & 0xFFFF0000u);
          }
          tc::st_row_chunk(sbase + P.dvl, t, 2 * hq + ch, vv + 8 * ch);
          tc::st_row_chunk(sbase + P.dp, t, 2 * hq + ch, vk + 8 * ch);
          tc::st_row_chunk(sbase + P.dplo, t, 2 * hq + ch, vq + 8 * ch);
        }
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::named_bar_arrive(NF_OUTFREE, NTHR);
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

