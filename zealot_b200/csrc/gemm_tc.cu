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
#include <climits>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "tc_ptx.cuh"
#include "zrl_gemm.h"

namespace zrl {
namespace {

constexpr int BM = 128;          // UMMA M (cta_group::1)
constexpr int BKB = 128;         // bytes of K per k-block (one swizzle row)
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;

// One GEMM of a grouped launch.  A launch runs up to kMaxProbs GEMMs of
// one kind and epilogue (e.g. the same layer of the actor and the critic,
// or every weight gradient of both nets) as one flat tile space, problem
// after problem.
constexpr int kMaxProbs = 8;
constexpr bool kLongKOneSlot = true;  // see dispatch_bn
constexpr int kMaxStages = 8;
// n / d for 0 <= n < 2^31 as (umulhi(n, mul) + n) >> shift (Granlund and
// Montgomery's division by invariant integers; the host picks mul, shift).
struct FastDiv {
  uint32_t d, mul, shift;
};
__device__ __forceinline__ int fdiv(int n, const FastDiv &f) {
  return (int)((__umulhi((uint32_t)n, f.mul) + (uint32_t)n) >> f.shift);
}

struct TcProb {
  int M, N, K;
  int kc;          // K per split (multiple of 32); split z covers [z*kc, ...)
  int splits;
  int tiles_m, tiles_n;
  FastDiv div_m, div_n;  // by tiles_m, by tiles_n
  int bn;          // this problem's tile width: the launch's BN or BN / 2
  int tile0;       // first flat tile index of this problem
  const float *bias;
  int round_out;
  float *colsum;   // optional column sums per 32-row quarter of each 128-row
                   // block: [ceil(M / 128) * 4][N] (no split-K)
};
struct TcGroup {
  TcProb p[kMaxProbs];
  int n;       // problems
  int tiles;   // total tiles
  int reverse; // walk the tiles last to first (L2 reuse of the previous launch's last tiles)
  int *err;
  uint64_t wait_ns;  // bound of every mbarrier wait
  int stall;         // test hook: the MMA issuer waits on a barrier nothing completes
};
// Tensor maps per problem: A and B operands, the output C (3-D, split
// index outermost) and the dgrad epilogue's post-activation X.
struct TcMaps {
  CUtensorMap a[kMaxProbs], b[kMaxProbs], c[kMaxProbs], x[kMaxProbs];
};

// Staging slots per epilogue warp, each one [32 x 32] fp32 box: two, so a
// chunk is staged while the previous chunk's store still reads its slot;
// three in the dgrad epilogue, where a slot first receives the chunk's
// TMA-loaded post-activation, two chunks ahead.
// The per-warp bias of the current tile (the epilogues that add a bias).
constexpr int bias_bytes(int bn, int epi) {
  return (epi == EPI_BIAS || epi == EPI_BIAS_ELU) ? kEpiWarps * (bn / 2 > 64 ? bn / 2 : 64) * 4 : 0;
}

// A plain store epilogue (the weight gradients' split-K partials: about one
// tile per CTA and launch) takes one slot, which leaves room for one more
// stage of the operand stream.
constexpr int slots_for(int epi) {
  return epi == EPI_ELU_GRAD ? 3 : (epi == EPI_STORE ? 1 : 2);
}

template <int BN, int STAGES, int EPI, int CG, int NSL>
struct Smem {
  static constexpr int kA = BM * BKB;                 // 16 KB
  static constexpr int kB = BN / CG * BKB;            // this CTA's B columns * 128 B
  static constexpr int kStage = kA + kB;
  static constexpr int kStageBytes = STAGES * kStage;
  static constexpr int kSlots = NSL;
  static constexpr int kStaging = kEpiWarps * kSlots * 4096;
  // the bias of a warp's chunks in the current tile
  static constexpr int kBiasPerWarp = BN / 2 > 64 ? BN / 2 : 64;  // floats
  static constexpr int kBias = bias_bytes(BN, EPI);
  static constexpr int kBarOff = kStageBytes + kStaging + kBias;
  // full, empty, acc_full x2, acc_empty x2, one aux barrier per staging
  // slot, and one that nothing completes (the stall test hook)
  static constexpr int kBars = 2 * STAGES + 4 + kEpiWarps * kSlots + 1;
  static constexpr int kBytes = 1024 /*align*/ + kBarOff + kBars * 8 + 16;
};

struct Tile {
  int p, m0, n0, z, kbeg, nk, bn;
};

// Flat tile t -> problem, then m fastest, n, split.  Tiles are BM * CG
// rows (the CTA pair's tile: 256 rows).
template <int BN, int CG, int KE>
__device__ __forceinline__ Tile decode_tile(int t, const TcGroup &g) {
  Tile tl;
  if (g.reverse) t = g.tiles - 1 - t;
  int p = 0;
  while (p + 1 < g.n && t >= g.p[p + 1].tile0) ++p;
  const TcProb &pr = g.p[p];
  const int lt = t - pr.tile0;
  tl.p = p;
  // n fastest: the tiles of one row block run side by side and share its
  // A rows through L2
  const int rest = fdiv(lt, pr.div_n);
  const int nt = lt - rest * pr.tiles_n;
  const int z = fdiv(rest, pr.div_m);
  tl.m0 = (rest - z * pr.tiles_m) * BM * CG;
  tl.bn = pr.bn;
  tl.n0 = nt * pr.bn;
  tl.z = z;
  tl.kbeg = tl.z * pr.kc;
  const int kend = min(pr.K, tl.kbeg + pr.kc);
  tl.nk = kend > tl.kbeg ? (kend - tl.kbeg + KE - 1) / KE : 0;
  return tl;
}

// One 32 x 32 chunk of the epilogue for one warp (lane = row): TMEM ->
// registers, the epilogue function, the optional column sums, rounding,
// and the 128B-swizzled staging for the TMA store.
struct EpiChunk {
  uint32_t taddr;    // TMEM address of the chunk (0xFFFFFFFF: accumulator not written)
  uint32_t slot;     // shared address of this lane's row in the staging slot
  uint32_t sw;       // swizzle phase of the row (lane & 7)
  uint32_t bias;     // shared address of the chunk's 32 bias values
  int round;         // round the stored values to tf32
  float *colsum;     // this quarter's partial row at the chunk's first column
};

template <int EPI, bool FULL, typename Release>
__device__ __forceinline__ void epi_chunk(const EpiChunk &e, int lane, bool last,
                                          Release release, bool row_ok, int valid_cols) {
  float v[32];
  if (!FULL && e.taddr == 0xFFFFFFFFu) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
  } else {
    uint32_t r[32];
    tmem_ld32(e.taddr, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    // last read of this accumulator: hand it back to the MMA warp
    if (last) release();
  }
  if (EPI == EPI_BIAS || EPI == EPI_BIAS_ELU) {
    uint32_t a[8];
    float b[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = e.bias + 16u * q;  // broadcast
    ld_shared4x8(a, b);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += b[i];
  }
  if (EPI == EPI_BIAS_ELU) {
    // ELU (net.rs:13-16); exp on the special-function unit, whose error is
    // far below the tf32 rounding applied next.  Both sides are computed
    // and selected (no per-element branch).
    float ex[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) ex[i] = exp_sfu(v[i]);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] > 0.0f ? v[i] : ex[i] - 1.0f;
  }
  if (EPI == EPI_ELU_GRAD) {
    // ELU' from the stored post-activation y in the slot (net.rs:19-22):
    // 1 for y > 0, else y + 1 = min(y + 1, 1) (NaN kept)
    uint32_t a[8];
    float y[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = e.slot + ((q ^ e.sw) << 4);
    ld_shared4x8(a, y);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= fmin_nan(y[i] + 1.0f, 1.0f);
  }
  if (!FULL) {
    // invalid rows and columns hold 0 (column sums; the store clips them)
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (!row_ok || i >= valid_cols) v[i] = 0.0f;
  }
  if (e.colsum) {
    // bias gradient: column sums of the unrounded chunk, staged first;
    // lane j then adds column j over the 32 rows in row order
    // (conflict-free: row r's 16-byte piece q sits at q ^ (r & 7))
#pragma unroll
    for (int q = 0; q < 8; ++q)
      st_shared4(e.slot + ((q ^ e.sw) << 4), v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
    const float cs = colsum_staged(e.slot - (uint32_t)lane * 128u, lane);
    if (lane < valid_cols) e.colsum[lane] = cs;
    __syncwarp();
  }
  if (e.round) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = round_tf32(v[i]);
  }
  // stage for the TMA store
#pragma unroll
  for (int q = 0; q < 8; ++q)
    st_shared4(e.slot + ((q ^ e.sw) << 4), v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// Two 32 x 32 chunks of the forward bias + ELU epilogue (fp32 output, every
// row and column valid, no column sums) in lockstep: the same operations as
// epi_chunk<EPI_BIAS_ELU, true> on each, as two independent chains the
// scheduler can interleave.
__device__ __forceinline__ void epi_pair_bias_elu(float (&va)[32], float (&vb)[32],
                                                  uint32_t bias_a, uint32_t bias_b,
                                                  uint32_t slot_a, uint32_t slot_b, uint32_t sw,
                                                  int round) {
  {
    uint32_t a[8], b[8];
    float x[32], y[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      a[q] = bias_a + 16u * q;  // broadcast
      b[q] = bias_b + 16u * q;
    }
    ld_shared4x8(a, x);
    ld_shared4x8(b, y);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      va[i] += x[i];
      vb[i] += y[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float ea = exp_sfu(va[i]), eb = exp_sfu(vb[i]);
    va[i] = va[i] > 0.0f ? va[i] : ea - 1.0f;
    vb[i] = vb[i] > 0.0f ? vb[i] : eb - 1.0f;
  }
  if (round) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      va[i] = round_tf32(va[i]);
      vb[i] = round_tf32(vb[i]);
    }
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    st_shared4(slot_a + ((q ^ sw) << 4), va[4 * q], va[4 * q + 1], va[4 * q + 2], va[4 * q + 3]);
    st_shared4(slot_b + ((q ^ sw) << 4), vb[4 * q], vb[4 * q + 1], vb[4 * q + 2], vb[4 * q + 3]);
  }
}

// The 64-column chunk of the bf16-output epilogues (forward hidden layers,
// dgrad): one row of 64 bf16 is 128 bytes, so the staging slot keeps the
// 128-byte swizzle.  fp32 math as in epi_chunk; the column sums are taken
// in two 32-column halves; the stored values are rounded to bf16 (nearest
// even) by the conversion.
template <int EPI, bool FULL, typename Release>
__device__ __forceinline__ void epi_chunk_bf16(const EpiChunk &e, int lane, bool last,
                                               Release release, bool row_ok, int valid_cols) {
  float v[64];
  if (!FULL && e.taddr == 0xFFFFFFFFu) {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = 0.0f;
  } else {
    uint32_t r[32];
    tmem_ld32(e.taddr, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    tmem_ld32(e.taddr + 32, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(r[i]);
    if (last) release();
  }
  if (EPI == EPI_BIAS_ELU) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t a[8];
      float b[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) a[q] = e.bias + 128u * h + 16u * q;  // broadcast
      ld_shared4x8(a, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[32 * h + i] += b[i];
    }
    float ex[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) ex[i] = exp_sfu(v[i]);
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = v[i] > 0.0f ? v[i] : ex[i] - 1.0f;
  }
  if (EPI == EPI_ELU_GRAD) {
    // the bf16 post-activation row in the slot: 16-byte piece q holds
    // columns 8q..8q+7
    uint32_t a[8];
    float raw[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) a[q] = e.slot + ((q ^ e.sw) << 4);
    ld_shared4x8(a, raw);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t w = __float_as_uint(raw[i]);
      const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xFFFF0000u);
      v[2 * i] *= fmin_nan(lo + 1.0f, 1.0f);
      v[2 * i + 1] *= fmin_nan(hi + 1.0f, 1.0f);
    }
  }
  if (!FULL) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (!row_ok || i >= valid_cols) v[i] = 0.0f;
  }
  if (e.colsum) {
    const uint32_t base = e.slot - (uint32_t)lane * 128u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k)
        st_shared4(e.slot + ((k ^ e.sw) << 4), v[32 * h + 4 * k], v[32 * h + 4 * k + 1],
                   v[32 * h + 4 * k + 2], v[32 * h + 4 * k + 3]);
      __syncwarp();
      const float cs = colsum_staged(base, lane);
      if (32 * h + lane < valid_cols) e.colsum[32 * h + lane] = cs;
    }
    __syncwarp();
  }
  // bf16 pairs (round to nearest even), staged for the TMA store
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
          : "=r"(pk[i])
          : "f"(v[8 * q + 2 * i + 1]), "f"(v[8 * q + 2 * i]));
    st_shared4(e.slot + ((q ^ e.sw) << 4), __uint_as_float(pk[0]), __uint_as_float(pk[1]),
               __uint_as_float(pk[2]), __uint_as_float(pk[3]));
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI, int STAGES, int CG, bool BF, int NSL>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcGroup g) {
  // K elements of one 128-byte k-block, and the M/N width of one MN-major
  // TMA box (one 128-byte row): 32 tf32 or 64 bf16
  constexpr int KE = BF ? 64 : 32;
  constexpr int MNB = BF ? 64 : 32;   // MN-major box width (elements)
  constexpr int MNBB = BF ? 8192 : 4096;  // bytes of one MN-major box
  static_assert(!BF || !B_MN || BN / CG >= 64, "bf16 MN-major B needs 64-column boxes");
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "BN");
  static_assert(CG == 1 || (CG == 2 && BN >= 64), "a CTA pair splits B in 32-column boxes");
  using S = Smem<BN, STAGES, EPI, CG, NSL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + S::kBarOff);
  uint64_t *empty = full + STAGES;
  uint64_t *accf = empty + STAGES;  // [2]
  uint64_t *acce = accf + 2;        // [2]
  uint64_t *xbar = acce + 2;        // [kEpiWarps][kSlots]
  uint64_t *never = xbar + kEpiWarps * S::kSlots;
  uint32_t *tmem_slot = (uint32_t *)(never + 1);
  float *bias_sh = (float *)(smem + S::kStageBytes + S::kStaging);  // [kEpiWarps][kCptMax][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = g.tiles;
  // CTA pairs walk the tiles together: pair index, pair count, rank
  const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
  const int unit = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      // this CTA's epilogue warps, and on the even CTA of a pair one more
      // arrival: the odd CTA's, forwarded once all its warps arrived
      mbar_init(&acce[b], kEpiWarps + (CG == 2 && rank == 0 ? 1 : 0));
    }
    for (int b = 0; b < kEpiWarps * S::kSlots; ++b) mbar_init(&xbar[b], 1);
    mbar_init(never, 1);
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
    // TMEM: two BN-column fp32 accumulators of 128 lanes (per CTA; for the
    // pair one warp of each CTA allocates jointly)
    if (CG == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"((uint32_t)(2 * BN))
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"((uint32_t)(2 * BN))
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if (CG == 2)
    cluster_sync();  // both CTAs' barriers initialised before any remote arrive
  else
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
      for (int t = unit; t < tiles && ok; t += units) {
        const Tile tl = decode_tile<BN, CG, KE>(t, g);
        // this CTA's rows of A and columns of B
        const int am = tl.m0 + BM * (int)rank;
        const int bn = tl.n0 + tl.bn / CG * (int)rank;
        // bytes of one stage in each CTA: A, and this CTA's tl.bn / CG
        // columns of B
        const uint32_t stage_bytes = (uint32_t)(S::kA + tl.bn / CG * BKB);
        for (int kb = 0; kb < tl.nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (uint32_t)(kbg / STAGES) & 1u;
          if (kbg >= STAGES && !(ok = mbar_spin(&empty[s], ph ^ 1u, g.err, 1, g.wait_ns))) break;
          uint8_t *a_s = smem + s * S::kStage;
          uint8_t *b_s = a_s + S::kA;
          const int k0 = tl.kbeg + kb * KE;
          if (CG == 2) {
            // both CTAs' boxes count on the even CTA's full barrier
            const uint32_t fb = peer_addr(smem_u32(&full[s]), 0);
            if (rank == 0) mbar_expect_tx(&full[s], 2 * stage_bytes);
            if (A_MN) {
#pragma unroll
              for (int c = 0; c < BM / MNB; ++c)
                tma_load_2d_pair(a_s + c * MNBB, &maps.a[tl.p], fb, am + MNB * c, k0);
            } else {
              tma_load_2d_pair(a_s, &maps.a[tl.p], fb, k0, am);
            }
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / CG / MNB; ++c)
                if (c < tl.bn / CG / MNB)
                  tma_load_2d_pair(b_s + c * MNBB, &maps.b[tl.p], fb, bn + MNB * c, k0);
            } else {
              tma_load_2d_pair(b_s, &maps.b[tl.p], fb, k0, bn);
            }
          } else {
            mbar_expect_tx(&full[s], stage_bytes);
            if (A_MN) {  // Delta [K rows, M cols]: MN-major boxes of one k-block
#pragma unroll
              for (int c = 0; c < BM / MNB; ++c)
                tma_load_2d(a_s + c * MNBB, &maps.a[tl.p], &full[s], am + MNB * c, k0);
            } else {     // [M rows, K cols]: one box of 128 rows x 32
              tma_load_2d(a_s, &maps.a[tl.p], &full[s], k0, am);
            }
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / MNB; ++c)
                if (c < tl.bn / MNB)
                  tma_load_2d(b_s + c * MNBB, &maps.b[tl.p], &full[s], bn + MNB * c, k0);
            } else {
              tma_load_2d(b_s, &maps.b[tl.p], &full[s], k0, bn);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_full = BF ? idesc_bf16(BM * CG, BN, A_MN, B_MN)
                                         : idesc_tf32(BM * CG, BN, A_MN, B_MN);
      constexpr uint32_t idesc_half = BF ? idesc_bf16(BM * CG, BN / 2, A_MN, B_MN)
                                         : idesc_tf32(BM * CG, BN / 2, A_MN, B_MN);
      int kbg = 0, it = 0;
      // the stall test hook: a wait that runs out (nothing completes the
      // barrier), after which every role of the kernel gives up in turn
      bool ok = !g.stall || mbar_spin(never, 0, g.err, 7, g.wait_ns);
      for (int t = unit; t < tiles && ok; t += units, ++it) {
        const Tile tl = decode_tile<BN, CG, KE>(t, g);
        const int ab = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        // the epilogue must have drained this accumulator (tile it-2)
        if (it >= 2 && !(ok = mbar_spin(&acce[ab], aph ^ 1u, g.err, 4, g.wait_ns))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        const uint32_t idesc = tl.bn == BN ? idesc_full : idesc_half;
        for (int kb = 0; kb < tl.nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (uint32_t)(kbg / STAGES) & 1u;
          if (!(ok = mbar_spin(&full[s], ph, g.err, 2, g.wait_ns))) break;
          tc_fence_after();
          const uint32_t a_s = smem_u32(smem + s * S::kStage);
          const uint32_t b_s = a_s + S::kA;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // one MMA takes 32 bytes of K: K-major, 32 bytes further in the
            // swizzle row; MN-major, 8 (tf32) or 16 (bf16) K-rows further
            const uint32_t step = BF ? 2048 : 1024;
            const uint64_t da = A_MN ? (BF ? desc_mnmajor_bf16(a_s + step * j)
                                           : desc_mnmajor(a_s + step * j))
                                     : desc_kmajor(a_s + 32 * j);
            const uint64_t db = B_MN ? (BF ? desc_mnmajor_bf16(b_s + step * j)
                                           : desc_mnmajor(b_s + step * j))
                                     : desc_kmajor(b_s + 32 * j);
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            if (CG == 2) {
              if (BF)
                mma_bf16_pair(d, da, db, idesc, acc);
              else
                mma_tf32_pair(d, da, db, idesc, acc);
            } else {
              if (BF)
                mma_bf16(d, da, db, idesc, acc);
              else
                mma_tf32(d, da, db, idesc, acc);
            }
          }
          if (CG == 2)
            mma_commit_pair(&empty[s]);
          else
            mma_commit(&empty[s]);
        }
        // completes when every MMA above has finished (at once for an empty
        // K range, whose accumulator the epilogue does not read)
        if (CG == 2)
          mma_commit_pair(&accf[ab]);
        else
          mma_commit(&accf[ab]);
      }
    } else if (CG == 2 && lane == 0) {
      // the odd CTA of a pair: forward its epilogue's release of each
      // accumulator to the even CTA's barrier, where the MMA issuer waits
      // (one cluster-scope arrival per tile instead of one per warp, off
      // the epilogue warps' path)
      const uint32_t acce_peer = peer_addr(smem_u32(acce), 0);
      int it = 0;
      for (int t = unit; t < tiles; t += units, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_spin(&acce[ab], aph, g.err, 6, g.wait_ns)) break;
        mbar_arrive_cluster(acce_peer + 8u * ab);
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    // two warps per TMEM lane quarter (warp w may only read lanes
    // 32*(w%4)..+31), taking alternate 32-column chunks (CPT per tile; for
    // BN = 32 the second warp of a quarter has none).  A warp's chunks,
    // numbered j = 0, 1, ... over its tiles, cycle through its NS staging
    // slots.
    constexpr int NS = S::kSlots;
    // chunk width: 32 fp32 columns, or 64 for bf16 outputs (128-byte rows)
    constexpr bool OB = BF && (EPI == EPI_BIAS_ELU || EPI == EPI_ELU_GRAD);
    constexpr int CW = OB ? 64 : 32;
    constexpr int CPT = BN >= 2 * CW ? BN / (2 * CW) : 1;
    const int ew = warp - 2;       // 0..kEpiWarps-1
    const int quarter = warp & 3;  // TMEM lane quarter = rows of this warp
    const int half = ew >> 2;      // chunks c with c % 2 == half
    const bool idle = BN < 2 * CW && half == 1;
    const uint32_t slots = smem_u32(smem + S::kStageBytes + ew * (NS * 4096));
    uint64_t *wbar = xbar + ew * NS;
    const uint32_t row_addr = (uint32_t)lane * 128u;  // this lane's row in a slot
    const uint32_t sw = (uint32_t)(lane & 7);         // its 128B-swizzle phase
    uint32_t xph = 0;  // phase bit per slot of the aux barriers
    // dgrad: TMA load of the stored post-activation box of chunk j into its
    // slot (the slot's previous store must be done reading it)
    auto issue_aux = [&](int j) {
      const int t = unit + (j / CPT) * units;
      if (idle || t >= tiles) return;
      const Tile tl = decode_tile<BN, CG, KE>(t, g);
      const TcProb &pr = g.p[tl.p];
      const int c = half + 2 * (j % CPT);
      const int n = tl.n0 + c * CW;
      const int r0 = tl.m0 + BM * (int)rank + quarter * 32;
      if (c * CW >= tl.bn || n >= pr.N || r0 >= pr.M) return;
      const int sl = j % NS;
      mbar_expect_tx(&wbar[sl], 4096);
      tma_load_2d(smem + S::kStageBytes + ew * (NS * 4096) + sl * 4096, &maps.x[tl.p], &wbar[sl],
                  n, r0);
    };
    if (EPI == EPI_ELU_GRAD && lane == 0)
      for (int p = 0; p < NS - 1; ++p) issue_aux(p);
    int it = 0, j = 0;
    bool ok = true, prev_store = false;
    // the pair's MMA warp waits on the even CTA's acc_empty barriers
    const uint32_t wbias = smem_u32(bias_sh + ew * S::kBiasPerWarp);
    for (int t = unit; t < tiles; t += units, ++it) {
      const Tile tl = decode_tile<BN, CG, KE>(t, g);
      const TcProb &pr = g.p[tl.p];
      const int ab = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      const int row0 = tl.m0 + BM * (int)rank + quarter * 32;
      if ((EPI == EPI_BIAS || EPI == EPI_BIAS_ELU) && !idle) {
        // this tile's bias for the warp's chunks, one coalesced load per
        // chunk before the accumulator wait (0 past N)
#pragma unroll
        for (int k = 0; k < CPT; ++k)
#pragma unroll
          for (int h = 0; h < CW / 32; ++h) {
            const int n = tl.n0 + (half + 2 * k) * CW + 32 * h + lane;
            const float b = n < pr.N ? __ldg(pr.bias + n) : 0.0f;
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(wbias + (uint32_t)(k * CW + 32 * h + lane) *
                                                              4u),
                         "f"(b)
                         : "memory");
          }
        __syncwarp();
      }
      if (EPI == EPI_ELU_GRAD && lane == 0 && !idle && t + units < tiles) {
        // the next tile's post-activation boxes of this warp into L2
        const Tile nt = decode_tile<BN, CG, KE>(t + units, g);
        const TcProb &np = g.p[nt.p];
        const int r0 = nt.m0 + BM * (int)rank + quarter * 32;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
          const int n = nt.n0 + (half + 2 * k) * CW;
          if ((half + 2 * k) * CW < nt.bn && n < np.N && r0 < np.M)
            tma_prefetch_2d(&maps.x[nt.p], n, r0);
        }
      }
      if (ok) ok = mbar_wait(&accf[ab], aph, g.err, 3, g.wait_ns);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is collective
      tc_fence_after();
      const bool rows_full = row0 + 32 <= pr.M;  // uniform
      const bool row_ok = row0 + lane < pr.M;
      const uint32_t taddr = tmem + (uint32_t)(ab * BN) + ((uint32_t)(quarter * 32) << 16);
      const bool have = ok && tl.nk > 0;
      if constexpr (EPI == EPI_BIAS_ELU && !OB && CPT % 2 == 0 && NS == 2) {
        // full forward tiles with a short K (at most 4 k-blocks: the
        // epilogue, not the main loop, sets their pace): the warp's chunks
        // two at a time -- both accumulator loads, one wait, both chunks'
        // math, both stores (measured at C2: level 0, K = 96, 36.5 -> 32.5
        // us; levels 1-2, K = 512 and 256, 4 % slower, so they stay single)
        if (!idle && have && tl.nk <= 4 && rows_full && tl.bn == BN && tl.n0 + BN <= pr.N &&
            !pr.colsum) {
#pragma unroll 1
          for (int k = 0; k < CPT; k += 2, j += 2) {
            // both staging slots free: the previous stores have read them
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
            uint32_t ra[32], rb[32];
            tmem_ld32_start(taddr + (half + 2 * k) * CW, ra);
            tmem_ld32_start(taddr + (half + 2 * k + 2) * CW, rb);
            tmem_ld_wait(ra);
            tmem_ld_wait(rb);
            if (k + 2 == CPT) {
              // the accumulator's last columns are in registers
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acce[ab]);
            }
            float va[32], vb[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              va[i] = __uint_as_float(ra[i]);
              vb[i] = __uint_as_float(rb[i]);
            }
            const uint32_t sa = slots + (uint32_t)(j % NS) * 4096u;
            const uint32_t sb = slots + (uint32_t)((j + 1) % NS) * 4096u;
            epi_pair_bias_elu(va, vb, wbias + (uint32_t)(k * CW) * 4u,
                              wbias + (uint32_t)((k + 1) * CW) * 4u, sa + row_addr,
                              sb + row_addr, sw, pr.round_out);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&maps.c[tl.p], smem + (sa - smem_u32(smem)),
                           tl.n0 + (half + 2 * k) * CW, row0, tl.z);
              tma_store_3d(&maps.c[tl.p], smem + (sb - smem_u32(smem)),
                           tl.n0 + (half + 2 * k + 2) * CW, row0, tl.z);
              bulk_commit();
            }
          }
          prev_store = true;
          continue;
        }
      }
#pragma unroll 1
      for (int k = 0; k < CPT; ++k, ++j) {
        const int c = half + 2 * k;
        const int n = tl.n0 + c * CW;
        const int sl = j % NS;
        const uint32_t slot = slots + (uint32_t)sl * 4096u;
        const bool live = !idle && c * CW < tl.bn && n < pr.N && row0 < pr.M;  // warp-uniform
        if (k == CPT - 1 && !(live && have)) {
          // (no TMEM read in this chunk) hand the accumulator back now
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[ab]);
        }
        if (EPI == EPI_ELU_GRAD && lane == 0 && j >= 1) {
          // the aux box of chunk j+NS-2 into the slot of chunk j-2, whose
          // store (issued two chunks back) must be done reading it; the
          // prologue issued chunks 0..NS-2
          if (prev_store) bulk_wait_read<1>();
          else bulk_wait_read<0>();
          issue_aux(j + NS - 2);
        }
        bool stored = false;
        if (live) {
          if (EPI == EPI_ELU_GRAD) {
            // the post-activation box of this chunk (TMA, one chunk ahead)
            if (!mbar_wait(&wbar[sl], (xph >> sl) & 1u, g.err, 5, g.wait_ns)) ok = false;
            xph ^= 1u << sl;
          }
          if (EPI != EPI_ELU_GRAD) {
            // the store that last used this slot (NS chunks back) must be
            // done reading it
            if (lane == 0) {
              if (prev_store && NS > 1) bulk_wait_read<1>();
              else bulk_wait_read<0>();
            }
            __syncwarp();
          }
          EpiChunk ec;
          ec.taddr = have ? taddr + c * CW : 0xFFFFFFFFu;
          ec.slot = slot + row_addr;
          ec.sw = sw;
          ec.bias = wbias + (uint32_t)(k * CW) * 4u;
          ec.round = pr.round_out;
          ec.colsum = pr.colsum
                          ? pr.colsum + ((int64_t)(tl.m0 / BM + rank) * 4 + quarter) * pr.N + n
                          : nullptr;
          // the common case (every row and column valid, accumulator
          // written) has its own code path, free of per-element predicates
          const int valid_cols = pr.N - n < CW ? pr.N - n : CW;
          auto release = [&] {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[ab]);
          };
          if (have && rows_full && valid_cols == CW) {
            if (OB)
              epi_chunk_bf16<EPI, true>(ec, lane, k == CPT - 1, release, true, CW);
            else
              epi_chunk<EPI, true>(ec, lane, k == CPT - 1, release, true, CW);
          } else {
            if (OB)
              epi_chunk_bf16<EPI, false>(ec, lane, k == CPT - 1 && have, release, row_ok,
                                         valid_cols);
            else
              epi_chunk<EPI, false>(ec, lane, k == CPT - 1 && have, release, row_ok, valid_cols);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&maps.c[tl.p], smem + (slot - smem_u32(smem)), n, row0, tl.z);
            bulk_commit();
          }
          stored = true;
        } else if (!idle && pr.colsum && c * CW < tl.bn && n < pr.N &&
                   tl.m0 + BM * (int)rank < pr.M) {
          // a quarter past the last row: its partial row is 0
#pragma unroll
          for (int h = 0; h < CW / 32; ++h)
            if (n + 32 * h + lane < pr.N)
              pr.colsum[((int64_t)(tl.m0 / BM + rank) * 4 + quarter) * pr.N + n + 32 * h + lane] =
                  0.0f;
        }
        prev_store = stored;
      }
    }
    if (lane == 0) bulk_wait_all();  // stores done before shared memory goes away
  }
  tc_fence_before();
  // neither CTA of a pair leaves while the other may still signal its
  // barriers
  if (CG == 2)
    cluster_sync();
  else
    __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    if (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"((uint32_t)(2 * BN))
                   : "memory");
    else
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
//
// bf16 operands: boxes of [box_rows, 64] elements (still 128-byte rows),
// the plain 128-byte swizzle for both majors.
bool make_map(CUtensorMap *m, const float *base, int64_t rows, int64_t cols, int64_t ld,
              int box_rows, bool mn_major, std::string *err, bool bf16 = false) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * (bf16 ? 2 : 4)};
  cuuint32_t box[2] = {bf16 ? 64u : 32u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = (mn_major && !bf16) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                    : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        2, (void *)base, dims, strides, box,
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
                  int64_t splits, std::string *err, bool bf16 = false) {
  // bf16 outputs: [32 x 64] boxes, still 128-byte rows
  const int es = bf16 ? 2 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)splits};
  cuuint64_t strides[2] = {(cuuint64_t)ld * es, (cuuint64_t)(rows * ld * es)};
  cuuint32_t box[3] = {bf16 ? 64u : 32u, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        3, (void *)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled (output) failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

// The deepest stage ring (at most kMaxStages) that fits next to the epilogue
// staging slots: more k-blocks in flight hide the TMA -> MMA -> release
// round trip.
template <int BN, int EPI, int CG, int NSL>
constexpr int stages_for() {
  constexpr int avail = 227 * 1024 - 1024 - kEpiWarps * NSL * 4096 - bias_bytes(BN, EPI) -
                        (8 + kEpiWarps * NSL) * 8 - 64;
  constexpr int st = avail / (BM * BKB + BN / CG * BKB);
  return st > kMaxStages ? kMaxStages : st;
}

// Co-resident CTA pairs of one instantiation (its shared memory and the
// GPCs decide).
template <typename K>
int max_pairs(K kfn, int smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = g_sms / 2;
  }
  return n;
}

// With units_out set, only reports the persistent grid's size in tiles
// processed at once (CTA pairs or CTAs) and launches nothing.
template <int BN, bool A_MN, bool B_MN, int EPI, int CG, bool BF, int NSL = slots_for(EPI)>
cudaError_t launch_one(const TcMaps &maps, const TcGroup &grp, cudaStream_t s, int *units_out) {
  constexpr int ST = stages_for<BN, EPI, CG, NSL>();
  static_assert(ST >= 2, "stage ring");
  using S = Smem<BN, ST, EPI, CG, NSL>;
  static_assert(S::kBytes <= 227 * 1024, "shared memory");
  auto kfn = tc_gemm_kernel<BN, A_MN, B_MN, EPI, ST, CG, BF, NSL>;
  // the shared-memory opt-in belongs to the current device's context: set
  // once per instantiation and device
  constexpr int kMaxDevices = 64;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::kBytes);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  // cached per instantiation (every instantiation has the same function
  // type, so the cache cannot live in max_pairs)
  static int pairs = 0;
  if (CG == 2 && pairs == 0) pairs = max_pairs(kfn, S::kBytes);
  int units = CG == 2 ? pairs : g_sms;
  if (units_out) {
    *units_out = units;
    return cudaSuccess;
  }
  cudaLaunchConfig_t cfg = {};
  if (grp.tiles < units) units = grp.tiles;
  cfg.gridDim = dim3(CG * units);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  // may start (set-up only) while the previous kernel in the stream ends
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = CG;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = CG == 2 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kfn, maps, grp);
}

// epi | kOneSlot: a long-K forward (its main loop, not its epilogue, sets
// the pace) with one staging slot per epilogue warp, whose room goes to
// one more operand stage
constexpr int kOneSlot = 0x100;

template <int BN, int CG, bool BF>
cudaError_t dispatch_bn(int kind, int epi, const TcMaps &maps, const TcGroup &grp,
                        cudaStream_t s, int *u) {
  const bool one = (epi & kOneSlot) != 0;
  epi &= ~kOneSlot;
  if (kind == 0) {  // forward
    if constexpr (BN >= 128 && CG == 2) {
      if (epi == EPI_BIAS_ELU && one)
        return launch_one<BN, false, false, EPI_BIAS_ELU, CG, BF, 1>(maps, grp, s, u);
    }
    if (epi == EPI_BIAS_ELU)
      return launch_one<BN, false, false, EPI_BIAS_ELU, CG, BF>(maps, grp, s, u);
    if (epi == EPI_BIAS) return launch_one<BN, false, false, EPI_BIAS, CG, BF>(maps, grp, s, u);
    return launch_one<BN, false, false, EPI_STORE, CG, BF>(maps, grp, s, u);
  }
  if constexpr (!BF || BN / CG >= 64) {
    if (kind == 1) {  // dgrad
      if (epi == EPI_ELU_GRAD)
        return launch_one<BN, false, true, EPI_ELU_GRAD, CG, BF>(maps, grp, s, u);
      return launch_one<BN, false, true, EPI_STORE, CG, BF>(maps, grp, s, u);
    }
    return launch_one<BN, true, true, EPI_STORE, CG, BF>(maps, grp, s, u);  // wgrad
  }
  return cudaErrorInvalidValue;
}

template <bool BF>
cudaError_t dispatch(int CG, int BN, int kind, int epi, const TcMaps &maps, const TcGroup &grp,
                     cudaStream_t s, int *units_out = nullptr) {
  if (CG == 1) {
    if (BN == 32) return dispatch_bn<32, 1, BF>(kind, epi, maps, grp, s, units_out);
    if (BN == 64) return dispatch_bn<64, 1, BF>(kind, epi, maps, grp, s, units_out);
    return dispatch_bn<128, 1, BF>(kind, epi, maps, grp, s, units_out);
  }
  if (BN == 64) return dispatch_bn<64, 2, BF>(kind, epi, maps, grp, s, units_out);
  if (BN == 128) return dispatch_bn<128, 2, BF>(kind, epi, maps, grp, s, units_out);
  return dispatch_bn<256, 2, BF>(kind, epi, maps, grp, s, units_out);
}

}  // namespace

struct TcCache {
  std::map<std::tuple<const void *, int64_t, int64_t, int64_t, int, int>, CUtensorMap> maps;
};

// kind: 0 K-major operand, 1 MN-major operand, 2 output, 3 K-major bf16
// operand, 4 MN-major bf16 operand, 5 bf16 output.  The map is copied out:
// the cache may be emptied by a later call (shapes that change from call
// to call, e.g. each rank's share of a minibatch, keep adding keys), so no
// pointer into it may be held across calls.
static bool cached_map(GemmEngine *eng, CUtensorMap *out, const float *base, int64_t rows,
                       int64_t cols, int64_t ld, int box_or_splits, int kind, std::string *err) {
  TcCache *c = static_cast<TcCache *>(eng->cache);
  auto key = std::make_tuple((const void *)base, rows, cols, ld, box_or_splits, kind);
  auto it = c->maps.find(key);
  if (it != c->maps.end()) {
    *out = it->second;
    return true;
  }
  CUtensorMap m;
  const bool ok = (kind == 2 || kind == 5)
                      ? make_out_map(&m, (float *)base, rows, cols, ld, box_or_splits, err,
                                     kind == 5)
                      : make_map(&m, base, rows, cols, ld, box_or_splits, kind == 1 || kind == 4,
                                 err, kind >= 3);
  if (!ok) return false;
  if (c->maps.size() > 4096) c->maps.clear();
  c->maps[key] = m;
  *out = m;
  return true;
}

bool tc_tensor_map(GemmEngine *eng, CUtensorMap *out, const float *base, int64_t rows,
                   int64_t cols, int64_t ld, int box_or_splits, int kind, std::string *err) {
  if (kind < 0 || kind > 2) {
    *err = "tc_tensor_map: unknown kind";
    return false;
  }
  return cached_map(eng, out, base, rows, cols, ld, box_or_splits, kind, err);
}

int tc_sm_count() { return g_sms; }

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

// Multiplier and shift for fdiv by d >= 1 (n < 2^31): shift = ceil(log2 d),
// mul = floor(2^32 (2^shift - d) / d) + 1.
static FastDiv fast_div(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  FastDiv f;
  f.d = d;
  f.shift = l;
  f.mul = (uint32_t)((((1ull << l) - d) << 32) / d + 1);
  return f;
}

static int layout_kind(const GemmArgs &g) {
  if (!g.trans_a && g.trans_b) return 0;   // forward
  if (!g.trans_a && !g.trans_b) return 1;  // dgrad
  if (g.trans_a && !g.trans_b) return 2;   // wgrad
  return -1;
}

// Tall GEMMs (every M >= 256) run on CTA pairs with 256 x BN tiles, BN up
// to 256: each SM then stages half of the B tile, which halves the
// shared-memory and L2 bytes per flop.  Others run on single CTAs with
// 128 x BN tiles, BN up to 128.  bf16 MN-major B is loaded in 64-column
// boxes: each CTA's share of a tile is a whole number of them.
static void tile_shape(int minM, int maxN, bool bf, int kind, int *CG, int *BN) {
  *CG = (minM >= 256 && maxN > 32) ? 2 : 1;
  *BN = maxN <= 32 ? 32 : (maxN <= 64 ? 64 : (maxN <= 128 || *CG == 1 ? 128 : 256));
  if (bf && kind != 0 && *BN / *CG < 64) *BN = 64 * *CG;
  // input gradients: 256 x 128 pair tiles (measured at C2: dgrad level 1,
  // N = 512, 61.9 -> 57.5 us; level 2, N = 256, 36.1 -> 35.3 us), twice
  // the tiles to even out the persistent grid's last round; the forward
  // keeps 256-wide tiles (level 1, N = 256, is 24 % slower at 128)
  if (*CG == 2 && *BN == 256 && kind == 1) *BN = 128;
}

// A problem at most half as wide as the launch's tiles takes half-width
// tiles (while each CTA's share of B stays whole 32-column boxes, 64 for
// bf16 MN-major).
static int tile_width(int N, int BN, int CG, bool bf, int kind) {
  const int min_share = (bf && kind != 0) ? 64 : 32;
  return (BN / 2 / CG >= min_share && N <= BN / 2) ? BN / 2 : BN;
}

int gemm_tc_split(GemmEngine *eng, const GemmArgs *gs, int n, int precision, int max_split,
                  int *splits) {
  (void)eng;
  const bool bf = precision == ZRL_GEMM_BF16;
  if (n < 1 || n > kMaxProbs || max_split < 1) return 0;
  const int kind = layout_kind(gs[0]);
  if (kind < 0) return 0;
  int maxN = 0, minM = INT32_MAX;
  for (int i = 0; i < n; ++i) {
    maxN = std::max(maxN, gs[i].N);
    minM = std::min(minM, gs[i].M);
  }
  int CG, BN;
  tile_shape(minM, maxN, bf, kind, &CG, &BN);
  int bn[kMaxProbs];
  int64_t tiles1[kMaxProbs];  // output tiles of one split
  for (int i = 0; i < n; ++i) {
    bn[i] = tile_width(gs[i].N, BN, CG, bf, kind);
    tiles1[i] = (int64_t)((gs[i].M + BM * CG - 1) / (BM * CG)) * ((gs[i].N + bn[i] - 1) / bn[i]);
  }
  int units = 0;
  TcMaps maps{};  // not read: the dispatch only reports the grid's units
  TcGroup grp{};
  const cudaError_t e = bf ? dispatch<true>(CG, BN, kind, gs[0].epi, maps, grp, nullptr, &units)
                           : dispatch<false>(CG, BN, kind, gs[0].epi, maps, grp, nullptr, &units);
  if (e != cudaSuccess || units < 1) return 0;
  // These tiles stream both operands (K = samples) and are bound by the
  // operand bytes of a k-block, which grow with the tile's rows + columns:
  // a problem with narrower tiles takes proportionally fewer splits, so
  // every tile of the launch moves about the same bytes (the persistent grid
  // deals tiles round-robin, so equal tiles keep its units equally busy).
  // Measured at C2, layer 1 (256 x 256 tiles) and layer 0 (256 x 128): equal
  // splits 61.5 us, splits in the ratio of the MMA work (2 : 1) 74 us.
  const int wmax = BM * CG + BN;
  auto split_of = [&](int S, int i) {
    const int s = (int)(((int64_t)S * (BM * CG + bn[i]) * 2 + wmax) / (2 * wmax));  // rounded
    return s < 1 ? 1 : s;
  };
  // estimated time: rounds of the persistent grid x the largest tile's
  // bytes -- its k-blocks of (rows + columns) x 128 B, plus its fp32
  // partial tile, written here and read back by the segment reduce; the
  // fewest splits within 3 % of the best
  const int ke = bf ? 64 : 32;
  auto cost = [&](int S) {
    int64_t tiles = 0, big = 0;
    for (int i = 0; i < n; ++i) {
      const int si = split_of(S, i);
      tiles += tiles1[i] * si;
      const int64_t kc = ((gs[i].K + si - 1) / si + ke - 1) / ke;
      big = std::max<int64_t>(big, kc * (BM * CG + bn[i]) + (int64_t)BM * CG * bn[i] / 16);
    }
    return (tiles + units - 1) / units * big;
  };
  int64_t best = INT64_MAX;
  for (int S = 1; S <= max_split; ++S) best = std::min(best, cost(S));
  int pick = 1;
  for (int S = 1; S <= max_split; ++S)
    if (cost(S) * 100 <= best * 103) {
      pick = S;
      break;
    }
  for (int i = 0; i < n; ++i) splits[i] = split_of(pick, i);
  return pick;
}

zrl_status gemm_tc_group(GemmEngine *eng, const GemmArgs *gs, int n, int precision,
                         cudaStream_t s, int *launched, std::string *err) {
  *launched = 0;
  if (precision != ZRL_GEMM_TF32 && precision != ZRL_GEMM_BF16) {
    *err = "the tensor-core GEMM takes tf32 or bf16 operands";
    return ZRL_NOT_SUPPORTED;
  }
  const bool bf = precision == ZRL_GEMM_BF16;
  if (n < 1 || n > kMaxProbs) {
    *err = "a grouped tensor-core GEMM takes 1 to 8 problems";
    return ZRL_INVALID_ARG;
  }
  const int kind = layout_kind(gs[0]);
  if (kind < 0) {
    *err = "unsupported operand layout for the tensor-core GEMM";
    return ZRL_NOT_SUPPORTED;
  }
  int maxN = 0, minM = INT32_MAX;
  for (int i = 0; i < n; ++i) {
    const GemmArgs &g = gs[i];
    if (layout_kind(g) != kind || g.epi != gs[0].epi) {
      *err = "the GEMMs of one group share operand layout and epilogue";
      return ZRL_INVALID_ARG;
    }
    // TMA needs 16-byte aligned bases and row pitches (operand pitches in
    // elements: multiples of 4 for fp32, 8 for bf16).  Ragged M, N and K are
    // handled (out-of-range TMA reads are zero-filled, stores clipped).
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    const int op_align = bf ? 8 : 4;
    const int out_align = (bf && (g.epi == EPI_BIAS_ELU || g.epi == EPI_ELU_GRAD)) ? 8 : 4;
    if (g.lda % op_align || g.ldb % op_align || g.ldc % out_align || (g.aux && g.ldaux % op_align) ||
        !a16(g.A) || !a16(g.B) || !a16(g.C) || (g.aux && !a16(g.aux))) {
      *err = "tensor-core GEMM needs 16-byte aligned operands and row pitches";
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
    minM = std::min(minM, g.M);
  }
  int CG, BN;
  tile_shape(minM, maxN, bf, kind, &CG, &BN);
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  TcGroup grp;
  memset(&grp, 0, sizeof(grp));
  int tiles = 0;
  for (int i = 0; i < n; ++i) {
    const GemmArgs &g = gs[i];
    const int split = g.split_k < 1 ? 1 : g.split_k;
    // A: [M rows, K cols] K-major, or [K rows, M cols] MN-major (wgrad)
    const bool ta = kind == 2 ? cached_map(eng, &maps.a[i], g.A, g.K, g.M, g.lda, bf ? 64 : 32,
                                           bf ? 4 : 1, err)
                              : cached_map(eng, &maps.a[i], g.A, g.M, g.K, g.lda, BM, bf ? 3 : 0,
                                           err);
    // B: [N rows, K cols] K-major (forward) or [K rows, N cols] MN-major
    // a problem at most half as wide as the launch's tiles takes half-width
    // tiles (while each CTA's share of B stays whole 32-column boxes)
    const int bn = tile_width(g.N, BN, CG, bf, kind);
    const int kmaj = bf ? 3 : 0, mnmaj = bf ? 4 : 1, ke = bf ? 64 : 32;
    const bool tb = kind == 0
                        ? cached_map(eng, &maps.b[i], g.B, g.N, g.K, g.ldb, bn / CG, kmaj, err)
                        : cached_map(eng, &maps.b[i], g.B, g.K, g.N, g.ldb, ke, mnmaj, err);
    // bf16 contexts store the forward hidden activations and the dgrad
    // deltas in bf16 (the operands of later GEMMs)
    const bool out_bf = bf && (g.epi == EPI_BIAS_ELU || g.epi == EPI_ELU_GRAD);
    const bool tc =
        cached_map(eng, &maps.c[i], g.C, g.M, g.N, g.ldc, split, out_bf ? 5 : 2, err);
    if (!ta || !tb || !tc) return ZRL_CUDA_ERROR;
    if (kind == 1 && g.epi == EPI_ELU_GRAD) {
      // the post-activation read by the dgrad epilogue in [32 x 32] boxes
      // ([32 x 64] bf16 boxes in bf16 contexts)
      if (!cached_map(eng, &maps.x[i], g.aux, g.M, g.N, g.ldaux, 32, bf ? 3 : 0, err))
        return ZRL_CUDA_ERROR;
    }
    TcProb &pr = grp.p[i];
    pr.M = g.M;
    pr.N = g.N;
    pr.K = g.K;
    pr.kc = ((g.K + split - 1) / split + ke - 1) / ke * ke;
    pr.splits = split;
    pr.tiles_m = (g.M + BM * CG - 1) / (BM * CG);
    pr.div_m = fast_div((uint32_t)pr.tiles_m);
    pr.bn = bn;
    pr.tiles_n = (g.N + bn - 1) / bn;
    pr.div_n = fast_div((uint32_t)pr.tiles_n);
    pr.tile0 = tiles;
    pr.bias = g.bias;
    pr.round_out = g.round_out;
    pr.colsum = g.colsum;
    tiles += pr.tiles_m * pr.tiles_n * split;
  }
  grp.n = n;
  grp.tiles = tiles;
  grp.reverse = gs[0].reverse_tiles;
  grp.err = eng->err_dev;
  grp.wait_ns = eng->wait_ns;
  grp.stall = eng->stall_next;
  eng->stall_next = 0;
  // a forward whose every problem has K >= 256 (8 k-blocks or more)
  int minK = INT32_MAX;
  for (int i = 0; i < n; ++i) minK = std::min(minK, gs[i].K);
  const int epi_sel =
      gs[0].epi | ((kLongKOneSlot && kind == 0 && gs[0].epi == EPI_BIAS_ELU && minK >= 256)
                       ? kOneSlot
                       : 0);
  const cudaError_t e = bf ? dispatch<true>(CG, BN, kind, epi_sel, maps, grp, s)
                           : dispatch<false>(CG, BN, kind, epi_sel, maps, grp, s);
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
