// tc_ptx.cuh -- inline-PTX building blocks of the sm_100a tensor-core
// kernels (gemm_tc.cu, head_tc.cu): mbarriers with bounded waits, TMA tile
// loads and stores, tcgen05 MMA / commit / TMEM loads, shared-memory matrix
// and instruction descriptors, and the epilogue's small numeric helpers.
// Every wait is bounded: it gives up after a wall-time limit (or
// kWaitLimit polls), records a code in an error flag and returns false.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace zrl {
namespace {

// a second bound on a wait, on the number of polls, should the global timer
// not advance; the wall-time bound (a launch parameter) is the one that normally ends
// a wait that never completes
constexpr uint32_t kWaitLimit = 1u << 24;

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps until the
// phase completes (or ~1 ms passes) instead of spinning and taking issue
// slots from the producer / MMA threads.
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: the single-thread producer and MMA roles spin on it
// (a suspended try_wait wakes up too late for a per-k-block handshake).
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: true when the phase completed, false (and *err set) when
// limit_ns of wall time passed without it (however long each poll slept).
// The limit is a launch parameter (the context's wait limit, 20 s unless
// set otherwise).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int *err,
                                          int code, uint64_t limit_ns) {
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try(b, parity)) return true;
    if (global_ns() - t0 > limit_ns) break;
  }
  atomicExch(err, code);
  return false;
}

// Bounded spin for the latency-critical single-thread roles.
__device__ __forceinline__ bool mbar_spin(uint64_t *b, uint32_t parity, int *err, int code,
                                          uint64_t limit_ns) {
  if (mbar_test(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_test(b, parity)) return true;
    if ((i & 255) == 255 && global_ns() - t0 > limit_ns) break;
  }
  atomicExch(err, code);
  return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"((uint64_t)map),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src,
                                             int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          (uint64_t)map),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void st_shared4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}
// Eight 16-byte shared loads in one statement: all eight are in flight
// before the first result is used (separate volatile loads would each be
// waited for in turn).
__device__ __forceinline__ void ld_shared4x8(const uint32_t (&a)[8], float (&v)[32]) {
  asm volatile(
      "ld.shared.v4.f32 {%0, %1, %2, %3}, [%32];\n\t"
      "ld.shared.v4.f32 {%4, %5, %6, %7}, [%33];\n\t"
      "ld.shared.v4.f32 {%8, %9, %10, %11}, [%34];\n\t"
      "ld.shared.v4.f32 {%12, %13, %14, %15}, [%35];\n\t"
      "ld.shared.v4.f32 {%16, %17, %18, %19}, [%36];\n\t"
      "ld.shared.v4.f32 {%20, %21, %22, %23}, [%37];\n\t"
      "ld.shared.v4.f32 {%24, %25, %26, %27}, [%38];\n\t"
      "ld.shared.v4.f32 {%28, %29, %30, %31}, [%39];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7]), "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]),
        "=f"(v[14]), "=f"(v[15]), "=f"(v[16]), "=f"(v[17]), "=f"(v[18]), "=f"(v[19]),
        "=f"(v[20]), "=f"(v[21]), "=f"(v[22]), "=f"(v[23]), "=f"(v[24]), "=f"(v[25]),
        "=f"(v[26]), "=f"(v[27]), "=f"(v[28]), "=f"(v[29]), "=f"(v[30]), "=f"(v[31])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7])
      : "memory");
}
// Eight 4-byte shared loads in one statement.
__device__ __forceinline__ void ld_shared1x8(const uint32_t (&a)[8], float (&v)[8]) {
  asm volatile(
      "ld.shared.f32 %0, [%8];\n\t"
      "ld.shared.f32 %1, [%9];\n\t"
      "ld.shared.f32 %2, [%10];\n\t"
      "ld.shared.f32 %3, [%11];\n\t"
      "ld.shared.f32 %4, [%12];\n\t"
      "ld.shared.f32 %5, [%13];\n\t"
      "ld.shared.f32 %6, [%14];\n\t"
      "ld.shared.f32 %7, [%15];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7])
      : "memory");
}
// Column sum of one 32 x 32 fp32 chunk staged with the 128-byte swizzle
// (row r's 16-byte piece q at q ^ (r & 7)): lane j adds column j over the
// rows in row order, the loads batched eight rows at a time.
__device__ __forceinline__ float colsum_staged(uint32_t base, int lane) {
  const uint32_t q = (uint32_t)lane >> 2, w = ((uint32_t)lane & 3u) * 4u;
  float cs = 0.0f;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += 8) {
    uint32_t a[8];
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      a[i] = base + (uint32_t)(r0 + i) * 128u + ((q ^ (uint32_t)i) << 4) + w;
    ld_shared1x8(a, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) cs += x[i];
  }
  return cs;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}


__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)m) : "memory");
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptors (sm_100 format: start address, leading /
// stride byte offsets in 16-byte units, version 1 at bit 46, layout type at
// bits 61-63).
//  K-major (layout 2, 128-byte swizzle of 16-byte chunks): 8-row x 128-byte
//    atoms stacked along M/N every 1024 bytes (sbo); lbo unused.
//  MN-major (layout 1, 128-byte swizzle of 32-byte chunks -- the only
//    MN-major layout tf32 operands support): 128 bytes (32 elements) of
//    M/N per K-row, 4 K-rows per atom; K-row groups every 512 bytes (sbo),
//    32-element M/N chunks every `lbo` bytes.
__device__ __forceinline__ uint64_t make_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= (uint64_t)layout << 61;
  return d;
}
constexpr uint32_t kLayoutSw128 = 2, kLayoutSw128Base32 = 1;
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  return make_desc(addr, 16, 1024, kLayoutSw128);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
  return make_desc(addr, 4096, 512, kLayoutSw128Base32);
}
//  MN-major bf16 (layout 2, the plain 128-byte swizzle): 64 elements of
//    M/N per K-row, 8 K-rows per 1 KB atom (sbo); 64-element M/N atom
//    columns (one TMA box of 64 K-rows each) every 8 KB (lbo).
__device__ __forceinline__ uint64_t desc_mnmajor_bf16(uint32_t addr) {
  return make_desc(addr, 8192, 1024, kLayoutSw128);
}

// Instruction descriptor for kind::tf32 with an f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                      // D format f32
         | (2u << 7)                    // A format tf32
         | (2u << 10)                   // B format tf32
         | ((a_mn ? 1u : 0u) << 15)     // A major
         | ((b_mn ? 1u : 0u) << 16)     // B major
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// Instruction descriptor for kind::f16 with bf16 inputs and an f32
// accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | ((a_mn ? 1u : 0u) << 15)     // A major
         | ((b_mn ? 1u : 0u) << 16)     // B major
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The CTA pair (cta_group::2): a cluster of two CTAs on two SMs whose
// tensor cores act as one, with M = 256 rows -- 128 in each CTA's TMEM --
// and the B tile split by columns between the two CTAs' shared memory.
// The even CTA issues the MMAs.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of this CTA's shared-memory offset `addr` in
// the CTA of rank `rank`.
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the
// mbarrier at cluster address `bar` (the even CTA's, for the pair).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Completion of the pair's MMAs arrives on the mbarrier at this offset in
// both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// tcgen05.ld of 32 columns without the wait: r is undefined until
// tmem_ld_wait(r), which takes r as an operand so that no use of r can be
// scheduled before it.  Nothing may come between the two but other such
// loads: registers of a load in flight must not be live across other code.
__device__ __forceinline__ void tmem_ld32_start(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// min(a, b) that returns NaN when either input is NaN
__device__ __forceinline__ float fmin_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Round to the tf32 grid (10 mantissa bits), to nearest with ties away
// from zero, as cvt.rna.tf32.f32 does for every non-NaN input: add half a
// tf32 ulp to the magnitude bits, then clear the 13 low bits (a carry into
// the exponent is the correct round-up, to infinity past the largest value).
__device__ __forceinline__ float round_tf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// e^x = 2^(x log2 e) with one ex2.approx: relative error about 2^-22 plus
// |x| 2^-24 from rounding the product; 0 below x = -87 (flush to zero)
__device__ __forceinline__ float exp_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.44269504088896341f));
  return y;
}

}  // namespace
}  // namespace zrl
