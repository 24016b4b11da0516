// tc_ptx.cuh -- thin inline-PTX layer for sm_100a: TMEM, tcgen05 MMA, TMA,
// mbarriers with bounded waits, and the 128-byte-swizzled smem layout the MMA
// descriptors describe.  Written against the PTX ISA (tcgen05 / cp.async.bulk
// chapters); descriptor bit layouts as documented there.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace race {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Longest time (ns) one sleeping poll may keep its thread suspended before it
// looks again: the thread sleeps until the phase completes (or this hint runs
// out) instead of spinning, so it takes no issue slots from the warps it waits
// for (the MMA-issuing lane shares an SM sub-partition with four epilogue warps).
constexpr uint32_t kSuspendNs = 1000;

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Default poll limit of a bounded wait (about a second of polling on a B200); a
// launch may carry another limit (race_set_wait_limit).  A sleeping wait counts
// each of its polls, which last up to kSuspendNs, as kSleepPollWeight polls.
constexpr uint32_t kDefaultWaitPolls = 1u << 26;
constexpr uint32_t kSleepPollWeight = 32;

// Bounded wait: returns false (and raises the abort flag) after abort[1]
// polls, or as soon as another thread has raised the flag.  `abort` points at
// the CTA's wait-control pair in shared memory, {abort flag, poll limit},
// which the kernel initialises from its launch arguments before any wait.
// Never spins forever.  Short waits: polls without sleeping.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
  const uint32_t limit = (uint32_t)abort[1];
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort) return false;
  }
  *abort = 1;
  return false;
}

// The same bound, sleeping between polls: for waits that are long next to the
// work of the warps they wait for (measured faster in the backward reverse
// walk, slower in the kernels whose waits are short).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, volatile int *abort) {
  const uint32_t limit = max((uint32_t)abort[1] / kSleepPollWeight, 1u);
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 15) == 15 && *abort) return false;
  }
  *abort = 1;
  return false;
}

// Bounded barrier among the threads an mbarrier was initialised for: arrive,
// then wait for the phase with the given parity (callers count the uses).
__device__ __forceinline__ bool mbar_sync(uint64_t *bar, uint32_t parity, volatile int *abort) {
  mbar_arrive(bar);
  return mbar_wait(bar, parity, abort);
}

// Warp-level forms for barriers counted in warps: one elected arrival per warp
// after __syncwarp (which orders every lane's prior writes before it).  Every
// lane still polls the wait itself: electing one poller and broadcasting the
// result measured ~25% slower on the epilogue warps of the tcgen05 kernels.
// The whole warp must call them.
__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
  return mbar_wait(bar, parity, abort);
}

__device__ __forceinline__ bool warp_sync(uint64_t *bar, uint32_t parity, volatile int *abort) {
  warp_arrive(bar);
  return warp_wait(bar, parity, abort);
}

// Bounded wait that ignores the abort flag: used to drain this thread's own
// in-flight MMAs before TMEM is released (at most about two seconds).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity, uint32_t limit = (1u << 21)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait_sleep(bar, parity)) return true;
  return false;
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_async_smem() {  // generic-proxy smem writes -> async proxy (MMA/TMA)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Per-thread register limit of a whole warpgroup (all four warps execute the same
// instruction).  A decrease returns registers to the block's pool, an increase takes them
// from it and waits until they are there: the increases a block makes must never exceed
// what it was launched with (threads x registers per thread) less what stays in use.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg: 24..256, a multiple of 8");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg: 24..256, a multiple of 8");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Non-blocking arrival on a named barrier (producer side of a bar.sync).
// Arrivals count whole warps; the warp must be converged.
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// warp-uniform success flag: a lane whose bounded wait gave up fails the warp
__device__ __forceinline__ bool warp_all(bool ok) { return __all_sync(0xffffffffu, ok); }

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous global -> shared copy of `bytes` (multiple of 16; both addresses 16-byte aligned)
// completing on an mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

// Tile store shared -> global through a tensor map (rows past the map's extent are
// not written), tracked by bulk groups of the issuing thread.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the committed stores have finished reading shared memory (the tiles may be rewritten)
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the committed stores are complete
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- TMEM
// Allocate `ncols` (power of two >= 32) TMEM columns; whole warp must call.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 consecutive columns: thread i of the warp gets lane (base lane + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, float &v) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  v = __uint_as_float(r);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v)) : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- MMA
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
//   start: smem byte address; lbo/sbo: byte offsets (multiples of 16).
//   Built as its two 32-bit words: lo = start >> 4 (bits 0-13) | lbo >> 4 (bits 16-29);
//   hi = sbo >> 4 (bits 32-45) | version 1 (bit 46) | SWIZZLE_128B (bits 61-63), a constant
//   for a given sbo.
__host__ __device__ constexpr uint32_t sdesc_hi(uint32_t sbo) {
  return ((sbo >> 4) & 0x3FFF) | (1u << 14) | (2u << 29);
}
__device__ __forceinline__ uint64_t sdesc(uint32_t start, uint32_t lbo, uint32_t sbo) {
  const uint32_t lo = ((start >> 4) & 0x3FFF) | (((lbo >> 4) & 0x3FFF) << 16);
  return ((uint64_t)sdesc_hi(sbo) << 32) | lo;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation.
//   a_mn / b_mn: operand is MN-major (transposed) instead of K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | ((a_mn ? 1u : 0u) << 15)      // A major
         | ((b_mn ? 1u : 0u) << 16)      // B major
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; single thread issues.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

// mbarrier arrives once all previously issued tcgen05.mma of this thread completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- swizzled tiles
// A "tile" is R rows x 64 bf16 (128 bytes per row), 1024-byte aligned, stored
// in 8-row atoms of 1024 bytes with the 16-byte chunks of row r XOR-ed by
// (r % 8) -- the canonical 128B-swizzle layout (what TMA SWIZZLE_128B writes).
// Wider matrices are stored as consecutive column blocks of 64, each a tile.
__host__ __device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk16 ^ (row & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void st_shared_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Store 8 consecutive values of row `row`, chunk `chunk16` (columns 8*chunk16..+7 of a tile) as bf16.
__device__ __forceinline__ void st_row_chunk(uint32_t tile, int row, int chunk16, const float *v) {
  st_shared_v4(tile + sw128_off(row, chunk16), pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
               pack_bf16(v[6], v[7]));
}

__device__ __forceinline__ void ld_row_chunk(uint32_t tile, int row, int chunk16, float *v) {
  uint32_t a, b, c, d;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(tile + sw128_off(row, chunk16)));
  const uint32_t w[4] = {a, b, c, d};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Store 4 values as bf16 (8 bytes) at columns 8*chunk16 + 4*half .. +3 of row `row`.
__device__ __forceinline__ void st_row_half(uint32_t tile, int row, int chunk16, int half, const float *v) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(tile + sw128_off(row, chunk16) + 8 * half),
               "r"(pack_bf16(v[0], v[1])), "r"(pack_bf16(v[2], v[3]))
               : "memory");
}

// Operand descriptors for the layouts above.
// The start-address field is the low 14 bits, address >> 4, and shared addresses
// stay below 2^18 (tile bases and offsets are multiples of 16): a byte offset from
// `base` enters as offset >> 4 added to the low word, which never carries out of the
// field.  The high word is a compile-time constant and the low word's base part is
// loop-invariant, so with k0 a compile-time constant each K step costs the issuing
// thread one 32-bit add.  (That thread issues every MMA of the CTA alone: each
// dependent integer instruction in front of an MMA delays it, and a 64-bit rebuild of
// the descriptor per MMA measured about 3x slower issue than precomputed words.)
//   K-major (rows = M or N, 64-wide column blocks along K), K step k0 (multiple of 16):
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int k0, uint32_t block_bytes) {
  const uint32_t lo = ((base >> 4) | (1u << 16)) + (((uint32_t)(k0 >> 6) * block_bytes + (uint32_t)(k0 & 63) * 2) >> 4);
  return ((uint64_t)sdesc_hi(1024) << 32) | lo;
}
//   MN-major (rows = K, 64-wide column blocks along M/N), K step k0 (multiple of 16):
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int k0, uint32_t block_bytes) {
  const uint32_t lo = ((base >> 4) | ((block_bytes >> 4) << 16)) + (uint32_t)k0 * 8;
  return ((uint64_t)sdesc_hi(1024) << 32) | lo;
}

}  // namespace tc
}  // namespace race
