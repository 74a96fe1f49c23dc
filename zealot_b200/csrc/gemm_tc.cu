// gemm_tc.cu -- tcgen05 tensor-core GEMMs for the MLP (sm_100a).
//
// One persistent, warp-specialised kernel serves the three GEMM shapes of
// the update, all on sample-major activations [rows, features]:
//
//   forward  Z[rows,out] = X[rows,in] W^T        A K-major,  B K-major
//   dgrad    D[rows,in]  = Delta[rows,out] W     A K-major,  B MN-major
//   wgrad    dW[out,in]  = Delta^T X  (split-K)  A MN-major, B MN-major
//
// One CTA per SM walks the 128 x BN output tiles (m fastest, so CTAs that
// run together share the B tile in L2).  Ten warps:
//   warp 0, one lane: TMA producer -- streams A/B k-blocks of 128 bytes
//     (32 tf32) into a ring of shared-memory stages;
//   warp 1, one lane: MMA issuer -- tcgen05.mma kind::tf32 (M=128, N=BN,
//     K=8, four per k-block) into one of two TMEM accumulators, committing
//     each stage back to the producer and each finished tile to the
//     epilogue;
//   warps 2-9: epilogue -- two warps per TMEM lane quarter (warp w reads
//     lanes 32*(w%4).. = tile rows), taking alternate 32-column chunks:
//     tcgen05.ld of the chunk (the accumulator goes back to the MMA warp
//     after the tile's last load), bias + ELU (forward) or ELU' from the
//     stored post-activation (dgrad; that box arrives by TMA into the
//     warp's staging slot one chunk ahead) or nothing (wgrad), optional
//     per-tile column sums (the bias gradient, taken before rounding, by a
//     shuffle butterfly), rounding to tf32 for outputs that feed later
//     GEMMs, then the 128B-swizzled staging slot and one TMA tensor store
//     per 32 x 32 chunk.
// With two accumulators the epilogue of tile i overlaps the MMAs of tile
// i+1, and the TMA engine does all bulk global reads and writes.
//
// Every mbarrier wait is bounded; a timeout sets *err and the waiting role
// leaves its loop.  No TMA multicast is used.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "zrl_gemm.h"

namespace zrl {
namespace {

constexpr int BM = 128;          // UMMA M (cta_group::1)
constexpr int BKB = 128;         // bytes of K per k-block (one swizzle row)
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;
// a second bound on a wait, on the number of polls, should the global timer
// not advance; the wall-time bound (kWaitNs) is the one that normally ends
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
// kWaitNs of wall time passed without it (however long each poll slept).
constexpr uint64_t kWaitNs = 20ull * 1000 * 1000 * 1000;
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int *err,
                                          int code) {
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try(b, parity)) return true;
    if (global_ns() - t0 > kWaitNs) break;
  }
  atomicExch(err, code);
  return false;
}

// Bounded spin for the latency-critical single-thread roles.
__device__ __forceinline__ bool mbar_spin(uint64_t *b, uint32_t parity, int *err, int code) {
  if (mbar_test(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_test(b, parity)) return true;
    if ((i & 255) == 255 && global_ns() - t0 > kWaitNs) break;
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

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
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

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
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

__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// e^x = 2^(x log2 e) with one ex2.approx: relative error about 2^-22 plus
// |x| 2^-24 from rounding the product; 0 below x = -87 (flush to zero)
__device__ __forceinline__ float exp_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.44269504088896341f));
  return y;
}

// Column sums of a [32 x 32] chunk held one row per lane: five butterfly
// steps, each exchanging half of the remaining columns with the partner
// lane, leave the sum of column `lane` in lane `lane` (a fixed summation
// tree, so the same bits every run).
__device__ __forceinline__ float colsum32(const float (&v)[32], int lane) {
  float w[16];
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float send = up ? v[i] : v[i + 16];
      const float keep = up ? v[i + 16] : v[i];
      w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
#pragma unroll
  for (int h = 8; h >= 1; h >>= 1) {
    const bool up = lane & h;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? w[i] : w[i + h];
      const float keep = up ? w[i + h] : w[i];
      w[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  return w[0];
}

// One GEMM of a grouped launch.  A launch runs up to kMaxProbs GEMMs of
// one kind and epilogue (e.g. the same layer of the actor and the critic,
// or every weight gradient of both nets) as one flat tile space, problem
// after problem.
constexpr int kMaxProbs = 8;
struct TcProb {
  int M, N, K;
  int kc;          // K per split (multiple of 32); split z covers [z*kc, ...)
  int splits;
  int tiles_m, tiles_n;
  int tile0;       // first flat tile index of this problem
  const float *bias;
  int round_out;
  float *colsum;   // optional per-m-tile column sums [tiles_m][N] (no split-K)
};
struct TcGroup {
  TcProb p[kMaxProbs];
  int n;       // problems
  int tiles;   // total tiles
  int *err;
};
// Tensor maps per problem: A and B operands, the output C (3-D, split
// index outermost) and the dgrad epilogue's post-activation X.
struct TcMaps {
  CUtensorMap a[kMaxProbs], b[kMaxProbs], c[kMaxProbs], x[kMaxProbs];
};

// Staging slots per epilogue warp, each one [32 x 32] fp32 box: one for the
// output; two for the dgrad epilogue, whose slots also receive the
// TMA-loaded post-activation one chunk ahead.
constexpr int slots_for(int epi) { return epi == EPI_ELU_GRAD ? 2 : 1; }

template <int BN, int STAGES, int EPI>
struct Smem {
  static constexpr int kA = BM * BKB;                 // 16 KB
  static constexpr int kB = BN * BKB;                 // BN * 128 B
  static constexpr int kStage = kA + kB;
  static constexpr int kStageBytes = STAGES * kStage;
  static constexpr int kSlots = slots_for(EPI);
  static constexpr int kStaging = kEpiWarps * kSlots * 4096;
  static constexpr int kRed = 4 * BN * 4;             // column sums per lane quarter
  static constexpr int kBarOff = kStageBytes + kStaging + kRed;
  // full, empty, acc_full x2, acc_empty x2, one aux barrier per staging slot
  static constexpr int kBars = 2 * STAGES + 4 + kEpiWarps * kSlots;
  static constexpr int kBytes = 1024 /*align*/ + kBarOff + kBars * 8 + 16;
};

struct Tile {
  int p, m0, n0, z, kbeg, nk;
};

// Flat tile t -> problem, then m fastest, n, split.
template <int BN>
__device__ __forceinline__ Tile decode_tile(int t, const TcGroup &g) {
  Tile tl;
  int p = 0;
  while (p + 1 < g.n && t >= g.p[p + 1].tile0) ++p;
  const TcProb &pr = g.p[p];
  const int lt = t - pr.tile0;
  tl.p = p;
  const int mt = lt % pr.tiles_m;
  const int rest = lt / pr.tiles_m;
  tl.m0 = mt * BM;
  tl.n0 = (rest % pr.tiles_n) * BN;
  tl.z = rest / pr.tiles_n;
  tl.kbeg = tl.z * pr.kc;
  const int kend = min(pr.K, tl.kbeg + pr.kc);
  tl.nk = kend > tl.kbeg ? (kend - tl.kbeg + 31) / 32 : 0;
  return tl;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcGroup g) {
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "BN");
  using S = Smem<BN, STAGES, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + S::kBarOff);
  uint64_t *empty = full + STAGES;
  uint64_t *accf = empty + STAGES;  // [2]
  uint64_t *acce = accf + 2;        // [2]
  uint64_t *xbar = acce + 2;        // [kEpiWarps][kSlots]
  uint32_t *tmem_slot = (uint32_t *)(xbar + kEpiWarps * S::kSlots);
  float *red = (float *)(smem + S::kStageBytes + S::kStaging);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = g.tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kEpiWarps);
    }
    for (int b = 0; b < kEpiWarps * S::kSlots; ++b) mbar_init(&xbar[b], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    if (lane < g.n) {
      prefetch_tmap(&maps.a[lane]);
      prefetch_tmap(&maps.b[lane]);
      prefetch_tmap(&maps.c[lane]);
      if (EPI == EPI_ELU_GRAD) prefetch_tmap(&maps.x[lane]);
    }
    __syncwarp();
    // TMEM: two BN-column fp32 accumulators of 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)(2 * BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: the set-up above overlapped the previous
  // kernel's tail; every global access below waits for that kernel to have
  // completed, and the next kernel may start its own set-up from here
  grid_dependency_wait();
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0) {
      int kbg = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const Tile tl = decode_tile<BN>(t, g);
        for (int kb = 0; kb < tl.nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (uint32_t)(kbg / STAGES) & 1u;
          if (kbg >= STAGES && !(ok = mbar_spin(&empty[s], ph ^ 1u, g.err, 1))) break;
          uint8_t *a_s = smem + s * S::kStage;
          uint8_t *b_s = a_s + S::kA;
          const int k0 = tl.kbeg + kb * 32;
          mbar_expect_tx(&full[s], S::kStage);
          if (A_MN) {  // Delta [K rows, M cols]: four 32-column boxes of 32 rows
#pragma unroll
            for (int c = 0; c < BM / 32; ++c)
              tma_load_2d(a_s + c * 4096, &maps.a[tl.p], &full[s], tl.m0 + 32 * c, k0);
          } else {     // [M rows, K cols]: one box of 128 rows x 32
            tma_load_2d(a_s, &maps.a[tl.p], &full[s], k0, tl.m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
              tma_load_2d(b_s + c * 4096, &maps.b[tl.p], &full[s], tl.n0 + 32 * c, k0);
          } else {
            tma_load_2d(b_s, &maps.b[tl.p], &full[s], k0, tl.n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      int kbg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        const Tile tl = decode_tile<BN>(t, g);
        const int ab = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        // the epilogue must have drained this accumulator (tile it-2)
        if (it >= 2 && !(ok = mbar_spin(&acce[ab], aph ^ 1u, g.err, 4))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        for (int kb = 0; kb < tl.nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (uint32_t)(kbg / STAGES) & 1u;
          if (!(ok = mbar_spin(&full[s], ph, g.err, 2))) break;
          tc_fence_after();
          const uint32_t a_s = smem_u32(smem + s * S::kStage);
          const uint32_t b_s = a_s + S::kA;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // K-major: 32 bytes further in the swizzle row; MN-major: 8
            // K-rows (1024 bytes) further
            const uint64_t da = A_MN ? desc_mnmajor(a_s + 1024 * j) : desc_kmajor(a_s + 32 * j);
            const uint64_t db = B_MN ? desc_mnmajor(b_s + 1024 * j) : desc_kmajor(b_s + 32 * j);
            mma_tf32(d, da, db, idesc, (kb > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        // completes when every MMA above has finished (at once for an empty
        // K range, whose accumulator the epilogue does not read)
        mma_commit(&accf[ab]);
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    // two warps per TMEM lane quarter (warp w may only read lanes
    // 32*(w%4)..+31), taking alternate 32-column chunks.  A warp's chunks,
    // numbered j = 0, 1, ... over its tiles, cycle through its kSlots
    // staging slots.
    constexpr int NS = S::kSlots;
    const int ew = warp - 2;       // 0..kEpiWarps-1
    const int quarter = warp & 3;  // TMEM lane quarter = rows of this warp
    const int half = ew >> 2;      // chunks c with c % 2 == half
    const int cpt = (BN / 32 - half + 1) / 2;  // chunks per tile of this warp
    uint8_t *slots = smem + S::kStageBytes + ew * (NS * 4096);
    uint64_t *wbar = xbar + ew * NS;
    uint32_t xph = 0;  // phase bit per slot of the aux barriers
    // dgrad: TMA load of the stored post-activation box of chunk j into its
    // slot (the slot's previous store must be done reading it)
    auto issue_aux = [&](int j) {
      if (cpt == 0) return;
      const int t = blockIdx.x + (j / cpt) * gridDim.x;
      if (t >= tiles) return;
      const Tile tl = decode_tile<BN>(t, g);
      const TcProb &pr = g.p[tl.p];
      const int n = tl.n0 + (half + 2 * (j % cpt)) * 32, r0 = tl.m0 + quarter * 32;
      if (n >= pr.N || r0 >= pr.M) return;
      const int sl = j % NS;
      mbar_expect_tx(&wbar[sl], 4096);
      tma_load_2d(slots + sl * 4096, &maps.x[tl.p], &wbar[sl], n, r0);
    };
    if (EPI == EPI_ELU_GRAD && lane == 0)
      for (int p = 0; p < NS - 1; ++p) issue_aux(p);
    int it = 0, j = 0;
    bool ok = true, prev_store = false;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const Tile tl = decode_tile<BN>(t, g);
      const TcProb &pr = g.p[tl.p];
      const int ab = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      if (ok) ok = mbar_wait(&accf[ab], aph, g.err, 3);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is collective
      tc_fence_after();
      const int row0 = tl.m0 + quarter * 32;
      const int row = row0 + lane;
      const bool row_ok = row < pr.M;
      const uint32_t taddr = tmem + (uint32_t)(ab * BN) + ((uint32_t)(quarter * 32) << 16);
      const bool have = ok && tl.nk > 0;
      bool released = false;
#pragma unroll 1
      for (int k = 0; k < cpt; ++k, ++j) {
        const int c = half + 2 * k;
        const int n = tl.n0 + c * 32;
        const int sl = j % NS;
        float *buf = (float *)(slots + sl * 4096);
        const bool live = n < pr.N && row0 < pr.M;  // uniform over the warp
        float v[32];
        if (live && have) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.0f;
        }
        if (k == cpt - 1) {
          // last read of this accumulator: hand it back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[ab]);
          released = true;
        }
        bool stored = false;
        if (live) {
          const bool full_chunk = n + 32 <= pr.N;
          float4 *rowp = reinterpret_cast<float4 *>(buf + lane * 32);
          if (EPI == EPI_BIAS || EPI == EPI_BIAS_ELU) {
            if (full_chunk) {
              const float4 *bp = reinterpret_cast<const float4 *>(pr.bias + n);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 b = __ldg(bp + q);
                v[4 * q + 0] += b.x;
                v[4 * q + 1] += b.y;
                v[4 * q + 2] += b.z;
                v[4 * q + 3] += b.w;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (n + i < pr.N) v[i] += __ldg(&pr.bias[n + i]);
            }
          }
          if (EPI == EPI_BIAS_ELU) {
            // ELU (net.rs:13-16); exp on the special-function unit, whose
            // error is far below the tf32 rounding applied next
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = v[i] > 0.0f ? v[i] : exp_sfu(v[i]) - 1.0f;
          }
          if (EPI == EPI_ELU_GRAD) {
            // ELU' from the stored post-activation y (net.rs:19-22), whose
            // box the TMA has put in this slot (zero-filled out of range)
            if (!mbar_wait(&wbar[sl], (xph >> sl) & 1u, g.err, 5)) ok = false;
            xph ^= 1u << sl;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 y = rowp[q ^ (lane & 7)];
              v[4 * q + 0] *= y.x > 0.0f ? 1.0f : y.x + 1.0f;
              v[4 * q + 1] *= y.y > 0.0f ? 1.0f : y.y + 1.0f;
              v[4 * q + 2] *= y.z > 0.0f ? 1.0f : y.z + 1.0f;
              v[4 * q + 3] *= y.w > 0.0f ? 1.0f : y.w + 1.0f;
            }
          }
          // invalid rows and columns hold 0 (column sums, clipped stores)
          if (!row_ok) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.0f;
          }
          if (!full_chunk) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n + i >= pr.N) v[i] = 0.0f;
          }
          if (pr.colsum) {
            // bias gradient: column sums of the unrounded chunk over its 32
            // rows (lane = row), a butterfly that leaves column `lane` in
            // lane `lane`
            red[quarter * BN + c * 32 + lane] = colsum32(v, lane);
          }
          if (pr.round_out) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = round_tf32(v[i]);
          }
          if (EPI != EPI_ELU_GRAD) {
            // the store that last used this slot (NS chunks back) must be
            // done reading it
            if (lane == 0) {
              if (prev_store) bulk_wait_read<NS - 1>();
              else bulk_wait_read<0>();
            }
            __syncwarp();
          }
          // stage in the 128B-swizzled layout (16-byte chunk q of row r at
          // position q ^ (r & 7): conflict-free) for one TMA store; the
          // store clips rows >= M and columns >= N
#pragma unroll
          for (int q = 0; q < 8; ++q)
            rowp[q ^ (lane & 7)] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&maps.c[tl.p], buf, n, row0, tl.z);
            bulk_commit();
          }
          stored = true;
        }
        if (!live && pr.colsum && n < pr.N) red[quarter * BN + c * 32 + lane] = 0.0f;  // no rows
        if (EPI == EPI_ELU_GRAD && lane == 0) {
          // refill the slot of chunk j-1 with the aux box of chunk j+NS-1
          if (stored) bulk_wait_read<1>();
          else bulk_wait_read<0>();
          issue_aux(j + NS - 1);
        }
        prev_store = stored;
      }
      if (!released) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[ab]);
      }
      if (pr.colsum) {
        named_bar_sync(1, 32 * kEpiWarps);
        for (int i = ew * 32 + lane; i < BN; i += 32 * kEpiWarps) {
          const int n = tl.n0 + i;
          if (n < pr.N)
            pr.colsum[(int64_t)(tl.m0 / BM) * pr.N + n] =
                red[i] + red[BN + i] + red[2 * BN + i] + red[3 * BN + i];
        }
        named_bar_sync(1, 32 * kEpiWarps);
      }
    }
    if (lane == 0) bulk_wait_all();  // stores done before shared memory goes away
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)(2 * BN))
                 : "memory");
  }
}

// ================================================================== host

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn g_encode = nullptr;
std::mutex g_mu;
int g_sms = 148;

// Row-major fp32 matrix [rows, cols] with row pitch ld (elements), read in
// boxes of [box_rows, 32].  K-major operands use the 128-byte swizzle of
// 16-byte chunks; MN-major ones the 128-byte swizzle of 32-byte chunks
// (the layout the MN-major tf32 descriptor expects).
bool make_map(CUtensorMap *m, const float *base, int64_t rows, int64_t cols, int64_t ld,
              int box_rows, bool mn_major, std::string *err) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw =
      mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

// Output [splits][rows][cols] (row pitch ld) written in [32 x 32] boxes with
// the 128-byte swizzle; the split index is the third coordinate so a box
// never spills rows into the next split's partial.
bool make_out_map(CUtensorMap *m, float *base, int64_t rows, int64_t cols, int64_t ld,
                  int64_t splits, std::string *err) {
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)splits};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(rows * ld * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled (output) failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

// The deepest stage ring (at most 6) that fits next to the epilogue
// staging slots: more k-blocks in flight hide the TMA -> MMA -> release
// round trip.
template <int BN, int EPI>
constexpr int stages_for() {
  constexpr int avail = 227 * 1024 - 1024 - kEpiWarps * slots_for(EPI) * 4096 - 4 * BN * 4 -
                        (8 + kEpiWarps * slots_for(EPI)) * 8 - 64;
  constexpr int st = avail / (BM * BKB + BN * BKB);
  return st > 6 ? 6 : st;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
cudaError_t launch_one(const TcMaps &maps, const TcGroup &grp, cudaStream_t s) {
  constexpr int ST = stages_for<BN, EPI>();
  static_assert(ST >= 2, "stage ring");
  using S = Smem<BN, ST, EPI>;
  static_assert(S::kBytes <= 227 * 1024, "shared memory");
  auto kfn = tc_gemm_kernel<BN, A_MN, B_MN, EPI, ST>;
  static bool attr = false;  // set once per instantiation (same value on every device)
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::kBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grp.tiles < g_sms ? grp.tiles : g_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::kBytes;
  cfg.stream = s;
  // may start (set-up only) while the previous kernel in the stream ends
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kfn, maps, grp);
}

template <int BN>
cudaError_t dispatch_bn(int kind, int epi, const TcMaps &maps, const TcGroup &grp,
                        cudaStream_t s) {
  if (kind == 0) {  // forward
    if (epi == EPI_BIAS_ELU) return launch_one<BN, false, false, EPI_BIAS_ELU>(maps, grp, s);
    if (epi == EPI_BIAS) return launch_one<BN, false, false, EPI_BIAS>(maps, grp, s);
    return launch_one<BN, false, false, EPI_STORE>(maps, grp, s);
  }
  if (kind == 1) {  // dgrad
    if (epi == EPI_ELU_GRAD) return launch_one<BN, false, true, EPI_ELU_GRAD>(maps, grp, s);
    return launch_one<BN, false, true, EPI_STORE>(maps, grp, s);
  }
  return launch_one<BN, true, true, EPI_STORE>(maps, grp, s);  // wgrad
}

}  // namespace

struct TcCache {
  std::map<std::tuple<const void *, int64_t, int64_t, int64_t, int, int>, CUtensorMap> maps;
};

// kind: 0 K-major operand, 1 MN-major operand, 2 output
static const CUtensorMap *cached_map(GemmEngine *eng, const float *base, int64_t rows,
                                     int64_t cols, int64_t ld, int box_or_splits, int kind,
                                     std::string *err) {
  TcCache *c = static_cast<TcCache *>(eng->cache);
  auto key = std::make_tuple((const void *)base, rows, cols, ld, box_or_splits, kind);
  auto it = c->maps.find(key);
  if (it != c->maps.end()) return &it->second;
  CUtensorMap m;
  const bool ok = kind == 2 ? make_out_map(&m, (float *)base, rows, cols, ld, box_or_splits, err)
                            : make_map(&m, base, rows, cols, ld, box_or_splits, kind == 1, err);
  if (!ok) return nullptr;
  if (c->maps.size() > 4096) c->maps.clear();
  return &(c->maps[key] = m);
}

zrl_status gemm_tc_init(int device, std::string *err) {
  std::lock_guard<std::mutex> lk(g_mu);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess &&
      sms > 0)
    g_sms = sms;
  if (g_encode) return ZRL_OK;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || !fn || q != cudaDriverEntryPointSuccess) {
    *err = "cuTensorMapEncodeTiled unavailable from the driver";
    return ZRL_CUDA_ERROR;
  }
  g_encode = (EncodeTiledFn)fn;
  return ZRL_OK;
}

zrl_status GemmEngine::init(int device, std::string *err) {
  (void)device;
  cache = new TcCache();
  cudaError_t e = cudaMalloc((void **)&err_dev, sizeof(int));
  if (e != cudaSuccess) {
    *err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
    return ZRL_CUDA_ERROR;
  }
  cudaMemset(err_dev, 0, sizeof(int));
  return ZRL_OK;
}

void GemmEngine::destroy() {
  delete static_cast<TcCache *>(cache);
  cache = nullptr;
  if (err_dev) cudaFree(err_dev);
  err_dev = nullptr;
}

static int layout_kind(const GemmArgs &g) {
  if (!g.trans_a && g.trans_b) return 0;   // forward
  if (!g.trans_a && !g.trans_b) return 1;  // dgrad
  if (g.trans_a && !g.trans_b) return 2;   // wgrad
  return -1;
}

zrl_status gemm_tc_group(GemmEngine *eng, const GemmArgs *gs, int n, int precision,
                         cudaStream_t s, int *launched, std::string *err) {
  *launched = 0;
  if (precision != ZRL_GEMM_TF32) {
    *err = "bf16 tensor-core GEMMs are not built in this library";
    return ZRL_NOT_SUPPORTED;
  }
  if (n < 1 || n > kMaxProbs) {
    *err = "a grouped tensor-core GEMM takes 1 to 8 problems";
    return ZRL_INVALID_ARG;
  }
  const int kind = layout_kind(gs[0]);
  if (kind < 0) {
    *err = "unsupported operand layout for the tensor-core GEMM";
    return ZRL_NOT_SUPPORTED;
  }
  int maxN = 0;
  for (int i = 0; i < n; ++i) {
    const GemmArgs &g = gs[i];
    if (layout_kind(g) != kind || g.epi != gs[0].epi) {
      *err = "the GEMMs of one group share operand layout and epilogue";
      return ZRL_INVALID_ARG;
    }
    // TMA needs 16-byte aligned bases and row pitches.  Ragged M, N and K
    // are handled (out-of-range TMA reads are zero-filled, stores clipped).
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (g.lda % 4 || g.ldb % 4 || g.ldc % 4 || (g.aux && g.ldaux % 4) || !a16(g.A) ||
        !a16(g.B) || !a16(g.C) || (g.aux && !a16(g.aux))) {
      *err = "tensor-core GEMM needs 16-byte aligned operands and row pitches (multiples of 4)";
      return ZRL_INVALID_ARG;
    }
    if (g.M <= 0 || g.N <= 0 || g.K <= 0) {
      *err = "tensor-core GEMM with an empty dimension";
      return ZRL_INVALID_ARG;
    }
    if (g.colsum && g.split_k > 1) {
      *err = "column sums are taken on unsplit GEMMs only";
      return ZRL_INVALID_ARG;
    }
    if (kind == 1 && g.epi == EPI_ELU_GRAD && !g.aux) {
      *err = "the ELU' epilogue needs the post-activation";
      return ZRL_INVALID_ARG;
    }
    maxN = std::max(maxN, g.N);
  }
  // 128-column tiles from N = 128 up: at M = 24,576 rows that gives 2.6 to
  // 5.2 tiles per SM per GEMM, a better balance than 256-column tiles
  const int BN = maxN <= 32 ? 32 : (maxN <= 64 ? 64 : 128);
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  TcGroup grp;
  memset(&grp, 0, sizeof(grp));
  int tiles = 0;
  for (int i = 0; i < n; ++i) {
    const GemmArgs &g = gs[i];
    const int split = g.split_k < 1 ? 1 : g.split_k;
    // A: [M rows, K cols] K-major, or [K rows, M cols] MN-major (wgrad)
    const CUtensorMap *ta = kind == 2 ? cached_map(eng, g.A, g.K, g.M, g.lda, 32, 1, err)
                                      : cached_map(eng, g.A, g.M, g.K, g.lda, BM, 0, err);
    // B: [N rows, K cols] K-major (forward) or [K rows, N cols] MN-major
    const CUtensorMap *tb = kind == 0 ? cached_map(eng, g.B, g.N, g.K, g.ldb, BN, 0, err)
                                      : cached_map(eng, g.B, g.K, g.N, g.ldb, 32, 1, err);
    const CUtensorMap *tc = cached_map(eng, g.C, g.M, g.N, g.ldc, split, 2, err);
    if (!ta || !tb || !tc) return ZRL_CUDA_ERROR;
    maps.a[i] = *ta;
    maps.b[i] = *tb;
    maps.c[i] = *tc;
    if (kind == 1 && g.epi == EPI_ELU_GRAD) {
      // the post-activation read by the dgrad epilogue in [32 x 32] boxes
      const CUtensorMap *tx = cached_map(eng, g.aux, g.M, g.N, g.ldaux, 32, 0, err);
      if (!tx) return ZRL_CUDA_ERROR;
      maps.x[i] = *tx;
    }
    TcProb &pr = grp.p[i];
    pr.M = g.M;
    pr.N = g.N;
    pr.K = g.K;
    pr.kc = ((g.K + split - 1) / split + 31) / 32 * 32;
    pr.splits = split;
    pr.tiles_m = (g.M + BM - 1) / BM;
    pr.tiles_n = (g.N + BN - 1) / BN;
    pr.tile0 = tiles;
    pr.bias = g.bias;
    pr.round_out = g.round_out;
    pr.colsum = g.colsum;
    tiles += pr.tiles_m * pr.tiles_n * split;
  }
  grp.n = n;
  grp.tiles = tiles;
  grp.err = eng->err_dev;
  cudaError_t e;
  if (BN == 32) e = dispatch_bn<32>(kind, gs[0].epi, maps, grp, s);
  else if (BN == 64) e = dispatch_bn<64>(kind, gs[0].epi, maps, grp, s);
  else e = dispatch_bn<128>(kind, gs[0].epi, maps, grp, s);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core GEMM launch: ") + cudaGetErrorString(e);
    return ZRL_CUDA_ERROR;
  }
  *launched = 1;
  return ZRL_OK;
}

zrl_status gemm_tc(GemmEngine *eng, const GemmArgs &g, int precision, cudaStream_t s,
                   int *launched, std::string *err) {
  return gemm_tc_group(eng, &g, 1, precision, s, launched, err);
}

}  // namespace zrl
