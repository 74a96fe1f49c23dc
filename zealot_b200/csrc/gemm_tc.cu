// gemm_tc.cu -- tcgen05 tensor-core GEMMs for the MLP (sm_100a).
//
// One warp-specialised kernel serves the three GEMM shapes of the update,
// all on sample-major activations [rows, features]:
//
//   forward  Z[rows,out] = X[rows,in] W^T        A K-major,  B K-major
//   dgrad    D[rows,in]  = Delta[rows,out] W     A K-major,  B MN-major
//   wgrad    dW[out,in]  = Delta^T X  (split-K)  A MN-major, B MN-major
//
// Per CTA one 128 x BN output tile: warp 0 (one lane) streams A/B k-blocks
// of 128 bytes (32 tf32) into a ring of shared-memory stages with TMA (128B
// swizzle), warp 1 (one lane) issues tcgen05.mma kind::tf32 into a TMEM
// accumulator (M=128, N=BN, K=8 per instruction, 4 per k-block) and commits
// each stage back to the producer; then all four warps drain TMEM with
// tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = tile rows) and apply the
// epilogue: bias + ELU (forward), ELU' from the stored post-activation
// (dgrad) or a plain store of the split-K partial (wgrad).  Outputs that
// feed later GEMMs are rounded to tf32 (round-to-nearest) in the epilogue,
// so the tensor core's tf32 read of them is exact.
//
// Every mbarrier wait is bounded; a timeout sets *err and the CTA leaves
// its loops (it still frees its TMEM).  No TMA multicast is used.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <tuple>

#include "zrl_gemm.h"

namespace zrl {
namespace {

constexpr int BM = 128;          // UMMA M (cta_group::1)
constexpr int BKB = 128;         // bytes of K per k-block (one swizzle row)
constexpr int kThreads = 128;
constexpr uint32_t kWaitLimit = 1u << 26;  // try_wait polls before giving up

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

__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed, false (and *err set) when
// the poll budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int *err,
                                          int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try(b, parity)) return true;
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

struct TcArgs {
  int M, N, K;
  int kc;              // K per split (multiple of 32); split z covers [z*kc, ...)
  float *C;
  int ldc;
  int64_t split_stride;  // elements between split partial outputs
  const float *bias;
  const float *aux;
  int ldaux;
  int round_out;
  float *colsum;  // optional per-tile column sums [grid.y][N] (no split-K)
  int *err;
};

template <int BN, int STAGES>
struct Smem {
  static constexpr int kA = BM * BKB;          // 16 KB
  static constexpr int kB = BN * BKB;          // BN * 128 B
  static constexpr int kStage = kA + kB;
  static constexpr int kBars = 2 * STAGES + 1;
  static constexpr int kBytes = 1024 /*align*/ + STAGES * kStage + kBars * 8 + 16;
};

template <int BN, bool A_MN, bool B_MN, int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
               const __grid_constant__ CUtensorMap tmB, TcArgs g) {
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "BN");
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + STAGES * S::kStage);
  uint64_t *empty = full + STAGES;
  uint64_t *accf = empty + STAGES;
  uint32_t *tmem_slot = (uint32_t *)(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int kbeg = blockIdx.z * g.kc;
  const int kend = min(g.K, kbeg + g.kc);
  const int nk = kend > kbeg ? (kend - kbeg + 31) / 32 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
  }
  if (warp == 0) {  // TMEM: BN fp32 columns for the 128 x BN accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0 && nk > 0) {
    // ---------------------------------------------------- TMA producer
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (kb >= STAGES) ok = mbar_wait(&empty[s], ph ^ 1u, g.err, 1);
      if (!ok) break;
      uint8_t *a_s = smem + s * S::kStage;
      uint8_t *b_s = a_s + S::kA;
      const int k0 = kbeg + kb * 32;
      mbar_expect_tx(&full[s], S::kStage);
      if (A_MN) {  // Delta [K rows, M cols]: four 32-column boxes of 32 rows
#pragma unroll
        for (int c = 0; c < BM / 32; ++c) tma_load_2d(a_s + c * 4096, &tmA, &full[s], m0 + 32 * c, k0);
      } else {     // X [M rows, K cols]: one box of 128 rows x 32
        tma_load_2d(a_s, &tmA, &full[s], k0, m0);
      }
      if (B_MN) {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tma_load_2d(b_s + c * 4096, &tmB, &full[s], n0 + 32 * c, k0);
      } else {
        tma_load_2d(b_s, &tmB, &full[s], k0, n0);
      }
    }
  } else if (warp == 1 && lane == 0 && nk > 0) {
    // ---------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      ok = mbar_wait(&full[s], ph, g.err, 2);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a_s = smem_u32(smem + s * S::kStage);
      const uint32_t b_s = a_s + S::kA;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // K-major: advance 32 bytes inside the swizzle row; MN-major:
        // advance 8 K-rows = 1024 bytes
        const uint64_t da = A_MN ? desc_mnmajor(a_s + 1024 * j) : desc_kmajor(a_s + 32 * j);
        const uint64_t db = B_MN ? desc_mnmajor(b_s + 1024 * j) : desc_kmajor(b_s + 32 * j);
        mma_tf32(tmem, da, db, idesc, (kb > 0 || j > 0) ? 1u : 0u);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(accf);  // fires once every MMA issued above has completed
  }
  __syncwarp();

  // -------------------------------------------------------- epilogue
  const int row = m0 + warp * 32 + lane;
  const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);
  float *Cz = g.C + (int64_t)blockIdx.z * g.split_stride;
  if (nk == 0) {
    // an empty K range (a trailing split): the partial is zero
    if (row < g.M)
      for (int n = n0; n < min(g.N, n0 + BN); n += 4)
        *reinterpret_cast<float4 *>(Cz + (int64_t)row * g.ldc + n) = make_float4(0, 0, 0, 0);
  }
  // warp-uniform go/no-go: tcgen05.ld below is warp-collective
  const bool acc_ok = nk > 0 && mbar_wait(accf, 0, g.err, 3);
  tc_fence_after();
  const bool go = __all_sync(0xffffffffu, acc_ok) &&
                  __shfl_sync(0xffffffffu, lane == 0 ? *(volatile int *)g.err : 0, 0) == 0;
  // column-sum scratch [4 warps][BN] in stage 0 (free: every TMA write has
  // been consumed by the MMAs that the accumulator barrier waited for)
  float *red = reinterpret_cast<float *>(smem);
  const bool row_ok = row < g.M;
  if (go) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(t_row + c * 32, r);  // warp-collective: every lane runs it
      const int n = n0 + c * 32;
      if (n >= g.N) continue;        // uniform across the warp
      const bool full_chunk = n + 32 <= g.N;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (row_ok) {
        if (EPI == EPI_BIAS || EPI == EPI_BIAS_ELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (full_chunk || n + i < g.N) v[i] += __ldg(&g.bias[n + i]);
        }
        if (EPI == EPI_BIAS_ELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = v[i] > 0.0f ? v[i] : expf(v[i]) - 1.0f;
        }
        if (EPI == EPI_ELU_GRAD) {
          const float *ap = g.aux + (int64_t)row * g.ldaux + n;
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 y = __ldg(reinterpret_cast<const float4 *>(ap) + q);
              v[4 * q + 0] *= y.x > 0.0f ? 1.0f : y.x + 1.0f;
              v[4 * q + 1] *= y.y > 0.0f ? 1.0f : y.y + 1.0f;
              v[4 * q + 2] *= y.z > 0.0f ? 1.0f : y.z + 1.0f;
              v[4 * q + 3] *= y.w > 0.0f ? 1.0f : y.w + 1.0f;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n + i < g.N) {
                const float y = __ldg(ap + i);
                v[i] *= y > 0.0f ? 1.0f : y + 1.0f;
              }
          }
        }
      }
      if (g.colsum) {
        // per-column sums over this warp's 32 rows, taken before rounding:
        // a butterfly reduce-scatter (31 shuffles) leaves column c*32+lane
        // in s[0] of lane `lane`
        float s[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = (row_ok && (full_chunk || n + i < g.N)) ? v[i] : 0.0f;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          const bool upper = (lane & o) != 0;
#pragma unroll
          for (int i = 0; i < o; ++i) {
            const float send = upper ? s[i] : s[i + o];
            const float keep = upper ? s[i + o] : s[i];
            s[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        red[warp * BN + c * 32 + lane] = s[0];
      }
      if (!row_ok) continue;
      if (g.round_out) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = round_tf32(v[i]);
      }
      float *cp = Cz + (int64_t)row * g.ldc + n;
      if (full_chunk) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          reinterpret_cast<float4 *>(cp)[q] =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < g.N) cp[i] = v[i];
      }
    }
  } else if (g.colsum) {
    for (int c = 0; c < BN / 32; ++c) red[warp * BN + c * 32 + lane] = 0.0f;
  }
  tc_fence_before();
  __syncthreads();
  if (g.colsum && threadIdx.x < BN) {
    const int n = n0 + threadIdx.x;
    if (n < g.N)
      g.colsum[(int64_t)blockIdx.y * g.N + n] =
          red[threadIdx.x] + red[BN + threadIdx.x] + red[2 * BN + threadIdx.x] +
          red[3 * BN + threadIdx.x];
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)BN)
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

template <int BN, bool A_MN, bool B_MN, int EPI, int STAGES>
cudaError_t launch_one(const CUtensorMap &ta, const CUtensorMap &tb, const TcArgs &a,
                       dim3 grid, cudaStream_t s) {
  using S = Smem<BN, STAGES>;
  auto kfn = tc_gemm_kernel<BN, A_MN, B_MN, EPI, STAGES>;
  static bool attr = false;  // set once per instantiation (same value on every device)
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::kBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kfn<<<grid, kThreads, S::kBytes, s>>>(ta, tb, a);
  return cudaGetLastError();
}

template <int BN>
cudaError_t dispatch_bn(int kind, int epi, const CUtensorMap &ta, const CUtensorMap &tb,
                        const TcArgs &a, dim3 grid, cudaStream_t s) {
  // two CTAs per SM (one's epilogue overlaps the other's main loop):
  // 3 x 32 KB stages at BN=128, 4 x <=24 KB below
  constexpr int ST = BN >= 128 ? 3 : 4;
  if (kind == 0) {  // forward
    if (epi == EPI_BIAS_ELU) return launch_one<BN, false, false, EPI_BIAS_ELU, ST>(ta, tb, a, grid, s);
    if (epi == EPI_BIAS) return launch_one<BN, false, false, EPI_BIAS, ST>(ta, tb, a, grid, s);
    return launch_one<BN, false, false, EPI_STORE, ST>(ta, tb, a, grid, s);
  }
  if (kind == 1) {  // dgrad
    if (epi == EPI_ELU_GRAD) return launch_one<BN, false, true, EPI_ELU_GRAD, ST>(ta, tb, a, grid, s);
    return launch_one<BN, false, true, EPI_STORE, ST>(ta, tb, a, grid, s);
  }
  return launch_one<BN, true, true, EPI_STORE, ST>(ta, tb, a, grid, s);  // wgrad
}

}  // namespace

struct TcCache {
  std::map<std::tuple<const void *, int64_t, int64_t, int64_t, int, bool>, CUtensorMap> maps;
};

static const CUtensorMap *cached_map(GemmEngine *eng, const float *base, int64_t rows,
                                     int64_t cols, int64_t ld, int box_rows, bool mn_major,
                                     std::string *err) {
  TcCache *c = static_cast<TcCache *>(eng->cache);
  auto key = std::make_tuple((const void *)base, rows, cols, ld, box_rows, mn_major);
  auto it = c->maps.find(key);
  if (it != c->maps.end()) return &it->second;
  CUtensorMap m;
  if (!make_map(&m, base, rows, cols, ld, box_rows, mn_major, err)) return nullptr;
  if (c->maps.size() > 4096) c->maps.clear();
  return &(c->maps[key] = m);
}

zrl_status gemm_tc_init(int device, std::string *err) {
  (void)device;
  std::lock_guard<std::mutex> lk(g_mu);
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

zrl_status gemm_tc(GemmEngine *eng, const GemmArgs &g, int precision, cudaStream_t s,
                   int *launched, std::string *err) {
  *launched = 0;
  if (precision != ZRL_GEMM_TF32) {
    *err = "bf16 tensor-core GEMMs are not built in this library";
    return ZRL_NOT_SUPPORTED;
  }
  int kind;
  if (!g.trans_a && g.trans_b) kind = 0;
  else if (!g.trans_a && !g.trans_b) kind = 1;
  else if (g.trans_a && !g.trans_b) kind = 2;
  else {
    *err = "unsupported operand layout for the tensor-core GEMM";
    return ZRL_NOT_SUPPORTED;
  }
  // TMA needs 16-byte aligned bases and row pitches; the vector epilogue
  // needs 16-byte aligned output/aux rows.  Ragged M, N and K are handled
  // (out-of-range TMA reads are zero-filled, ragged columns are masked).
  auto a16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  if (g.lda % 4 || g.ldb % 4 || g.ldc % 4 || (g.aux && g.ldaux % 4) || !a16(g.A) ||
      !a16(g.B) || !a16(g.C) || (g.aux && !a16(g.aux))) {
    *err = "tensor-core GEMM needs 16-byte aligned operands and row pitches (multiples of 4)";
    return ZRL_INVALID_ARG;
  }
  if (g.K <= 0) {
    *err = "tensor-core GEMM with K = 0";
    return ZRL_INVALID_ARG;
  }
  const int BN = g.N <= 32 ? 32 : (g.N <= 64 ? 64 : 128);
  // A: [M rows, K cols] K-major, or [K rows, M cols] MN-major (wgrad)
  const CUtensorMap *ta = kind == 2 ? cached_map(eng, g.A, g.K, g.M, g.lda, 32, true, err)
                                    : cached_map(eng, g.A, g.M, g.K, g.lda, BM, false, err);
  // B: [N rows, K cols] K-major (forward) or [K rows, N cols] MN-major
  const CUtensorMap *tb = kind == 0 ? cached_map(eng, g.B, g.N, g.K, g.ldb, BN, false, err)
                                    : cached_map(eng, g.B, g.K, g.N, g.ldb, 32, true, err);
  if (!ta || !tb) return ZRL_CUDA_ERROR;
  int split = g.split_k < 1 ? 1 : g.split_k;
  int kc = (g.K + split - 1) / split;
  kc = (kc + 31) / 32 * 32;
  TcArgs a{};
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.kc = kc;
  a.C = g.C;
  a.ldc = g.ldc;
  a.split_stride = (int64_t)g.M * g.ldc;
  a.bias = g.bias;
  a.aux = g.aux;
  a.ldaux = g.ldaux;
  a.round_out = g.round_out;
  a.colsum = g.colsum;
  if (g.colsum && split != 1) {
    *err = "column sums are taken on unsplit GEMMs only";
    return ZRL_INVALID_ARG;
  }
  a.err = eng->err_dev;
  dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, split);
  cudaError_t e;
  if (BN == 32) e = dispatch_bn<32>(kind, g.epi, *ta, *tb, a, grid, s);
  else if (BN == 64) e = dispatch_bn<64>(kind, g.epi, *ta, *tb, a, grid, s);
  else e = dispatch_bn<128>(kind, g.epi, *ta, *tb, a, grid, s);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core GEMM launch: ") + cudaGetErrorString(e);
    return ZRL_CUDA_ERROR;
  }
  *launched = 1;
  return ZRL_OK;
}

}  // namespace zrl
