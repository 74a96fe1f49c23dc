// head_tc.cu -- the fused output head of the PPO update (sm_100a).
//
// Per minibatch the update's backward starts at the two output layers
// (ppo.rs:410-452, net.rs:113-140): Z = A W^T + b (the action mean or the
// value), the PPO losses of every row on Z, the output-layer delta D, then
// the last hidden layer's delta D' = (D W) * ELU'(A).  Here one persistent
// kernel does all of it, a 128-row block of one net per tile:
//
//   warp 0, one lane: TMA producer -- both nets' output weights once (in the
//     K-major layout of the forward and the MN-major one of the input
//     gradient), then per tile the 128 x k activation block A into one of
//     two shared-memory buffers (k / 32 boxes of 128 rows x 32 columns);
//   warp 1, one lane: MMA issuer -- tcgen05.mma kind::tf32 M = 128: the
//     forward Z (N = 32, K = k) into TMEM columns 0-31, one tile ahead, and
//     once the loss warps have written D, D W (N = k, K = 32) into columns
//     128-255;
//   warps 2-5, the loss warps, one per TMEM lane quarter (lane = row): the
//     row's 32 outputs + bias, its losses and gradients (the loss kernel's
//     arithmetic, kernels.cu), D rounded to tf32 into the shared operand
//     tile and to memory (the output layer's weight-gradient input);
//   warps 6-9, the input-gradient warps, one per lane quarter: per 32-column
//     chunk of D W, ELU' from the row's activations still in the A buffer,
//     the bias-gradient column sums of the unrounded delta, and D' rounded
//     to tf32 -- staged in place of the activations it replaces and stored
//     by TMA.
// The two epilogue groups work on consecutive tiles at once (the losses of
// tile i + 1 while the input gradient of tile i drains).
//
// Column sums (the log_std gradient, both output biases, the last hidden
// bias) and the statistic sums accumulate per warp over the CTA's tiles in
// a fixed order and leave as one partial row per warp.  Every mbarrier wait
// is bounded (an error code in *err, then the role stops).  No TMA
// multicast.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "tc_ptx.cuh"
#include "zrl_gemm.h"

namespace zrl {
namespace {

constexpr int kHeadRows = 128;             // rows of a tile (UMMA M)
constexpr int kHeadMaxK = 128;             // widest last hidden layer taken
constexpr int kHeadEpi = 4;                // warps per epilogue group, one per lane quarter
constexpr int kHeadThreads = 64 + 2 * 32 * kHeadEpi;
constexpr int kKBlock = kHeadRows * 128;   // one 128-row k-block: 16 KB
constexpr int kABuf = kHeadMaxK / 32 * kKBlock;  // 64 KB
constexpr int kWBox = 32 * 128;            // 32 rows x 32 fp32 columns
constexpr int kWNet = 2 * (kHeadMaxK / 32) * kWBox;  // K-major + MN-major: 32 KB
constexpr uint32_t kColOut = 0, kColDin = 128, kTmemCols = 256;
constexpr float kLogSqrt2PiH = 0.9189385f;  // ppo.rs:18

struct HeadMaps {
  CUtensorMap a[2], wk[2], wn[2], dout[2], din[2];
};

struct HeadParams {
  int k[2];
  const float *b[2];
  float *colsum[2];
  const float *action, *mean_old, *logp_old, *value_old, *adv, *ret, *log_std;
  int A;
  int rows;
  int blocks;  // 128-row blocks per net
  float scale, clip, entropy_coef, value_coef;
  float *part;
  int *err;
  uint64_t wait_ns;  // bound of every mbarrier wait
};

// shared memory: two activation buffers, both nets' weights, the delta
// operand tile, per-dimension constants, output biases, barriers
struct HeadSmem {
  static constexpr int kA0 = 0;
  static constexpr int kW = 2 * kABuf;                 // 128 KB
  static constexpr int kD = kW + 2 * kWNet;            // 192 KB
  static constexpr int kConst = kD + kKBlock;          // 208 KB
  static constexpr int kBias = kConst + 5 * 32 * 4;
  // per input-gradient warp: its running column sums [net][chunk][32]
  static constexpr int kHb = kBias + 2 * 32 * 4;
  static constexpr int kBar = kHb + kHeadEpi * 2 * (kHeadMaxK / 32) * 32 * 4;
  // w_full, a_full x2, a_empty x2, out_full, out_empty, d_full, din_full, din_empty
  static constexpr int kBars = 10;
  static constexpr int kBytes = 1024 + kBar + kBars * 8 + 16;
};
static_assert(HeadSmem::kBytes <= 227 * 1024, "head shared memory");

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// the two epilogue groups (warps 2-9)
__device__ __forceinline__ void named_sync_epi() {
  asm volatile("bar.sync 1, %0;" ::"n"(2 * 32 * kHeadEpi) : "memory");
}

// a / b correctly rounded (to nearest even), given y = RN(1 / b), by
// Markstein's correction (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34,
// 1990): q = RN(a y) is within an ulp of a / b, the remainder
// r = a - b q is exact in one fused multiply-add, and RN(q + r y) is the
// correctly rounded quotient -- for operands far from overflow and
// underflow, as here (b = exp(log_std) in [0.2, 2.72], |a| a difference of
// actions and means).  Straight-line code: the 29 divisions of a row
// interleave instead of each taking the general division's branches.
__device__ __forceinline__ float div_rn(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, y, q);
}

// 32 values of this lane's row into its 128-byte row of a 32 x 32 block
// staged with the 128-byte swizzle (16-byte piece c at c ^ (row & 7))
__device__ __forceinline__ void stage_row(uint32_t row_addr, uint32_t sw, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared4(row_addr + ((c ^ sw) << 4), v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

__global__ void __launch_bounds__(kHeadThreads, 1)
head_kernel(const __grid_constant__ HeadMaps maps, const __grid_constant__ HeadParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(smem + HeadSmem::kBar);
  uint64_t *w_full = bars + 0, *a_full = bars + 1, *a_empty = bars + 3;
  uint64_t *out_full = bars + 5, *out_empty = bars + 6, *d_full = bars + 7;
  uint64_t *din_full = bars + 8, *din_empty = bars + 9;
  uint32_t *tmem_slot = (uint32_t *)(bars + HeadSmem::kBars);
  // [5][32]: log_std, sd, exp(-log_std), 1/var, RN(1/sd)
  float *kconst = (float *)(smem + HeadSmem::kConst);
  float *bias = (float *)(smem + HeadSmem::kBias);     // [2][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = 2 * p.blocks;
  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a_full[b], 1);
      mbar_init(&a_empty[b], kHeadEpi);
    }
    mbar_init(out_full, 1);
    mbar_init(out_empty, kHeadEpi);
    mbar_init(d_full, kHeadEpi);
    mbar_init(din_full, 1);
    mbar_init(din_empty, kHeadEpi);
    fence_barrier_init();
  }
  if (warp == 0) {
    if (lane < 2) {
      prefetch_tmap(&maps.a[lane]);
      prefetch_tmap(&maps.wk[lane]);
      prefetch_tmap(&maps.wn[lane]);
      prefetch_tmap(&maps.dout[lane]);
      prefetch_tmap(&maps.din[lane]);
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      uint32_t wbytes = 0;
      for (int k = 0; k < 2; ++k) wbytes += 2u * (uint32_t)(p.k[k] / 32) * kWBox;
      mbar_expect_tx(w_full, wbytes);
      for (int k = 0; k < 2; ++k) {
        uint8_t *wk = smem + HeadSmem::kW + k * kWNet;
        uint8_t *wn = wk + kWNet / 2;
        for (int c = 0; c < p.k[k] / 32; ++c) {
          tma_load_2d(wk + c * kWBox, &maps.wk[k], w_full, 32 * c, 0);  // K-major k-block c
          tma_load_2d(wn + c * kWBox, &maps.wn[k], w_full, 32 * c, 0);  // MN-major columns c
        }
      }
      int i = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int net = t >= p.blocks ? 1 : 0;
        const int m0 = (t - net * p.blocks) * kHeadRows;
        const int b = i & 1;
        if (i >= 2 && !(ok = mbar_wait(&a_empty[b], ((i >> 1) & 1) ^ 1u, p.err, 11, p.wait_ns))) break;
        const int nk = p.k[net] / 32;
        mbar_expect_tx(&a_full[b], (uint32_t)(nk * kKBlock));
        uint8_t *abuf = smem + HeadSmem::kA0 + b * kABuf;
        for (int c = 0; c < nk; ++c)
          tma_load_2d(abuf + c * kKBlock, &maps.a[net], &a_full[b], 32 * c, m0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    // (its waits are per tile and long: suspended polls, which leave the
    // sub-partition's issue slots to the epilogue warp that shares it)
    if (lane == 0) {
      bool ok = mbar_wait(w_full, 0, p.err, 12, p.wait_ns);
      // the forward of tile i (its A buffer loaded, the previous output read)
      auto fwd = [&](int i, int t) -> bool {
        const int net = t >= p.blocks ? 1 : 0;
        const int nk = p.k[net] / 32;
        const int b = i & 1;
        if (!mbar_wait(&a_full[b], (i >> 1) & 1, p.err, 13, p.wait_ns)) return false;
        if (i >= 1 && !mbar_wait(out_empty, ((uint32_t)i & 1u) ^ 1u, p.err, 14, p.wait_ns)) return false;
        tc_fence_after();
        // Z[128 x 32] = A[128 x k] W^T
        const uint32_t a_s = smem_u32(smem + HeadSmem::kA0 + b * kABuf);
        const uint32_t wk = smem_u32(smem + HeadSmem::kW + net * kWNet);
        constexpr uint32_t id_out = idesc_tf32(kHeadRows, 32, false, false);
        for (int c = 0; c < nk; ++c)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_tf32(tmem + kColOut, desc_kmajor(a_s + c * kKBlock + 32 * j),
                     desc_kmajor(wk + c * kWBox + 32 * j), id_out, (c > 0 || j > 0) ? 1u : 0u);
        mma_commit(out_full);
        return true;
      };
      int i = 0;
      if (ok && (int)blockIdx.x < tiles) ok = fwd(0, blockIdx.x);
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int net = t >= p.blocks ? 1 : 0;
        const uint32_t ph = (uint32_t)i & 1u;
        // the next tile's forward first: the loss warps read it while this
        // tile's input gradient drains
        if (t + (int)gridDim.x < tiles && !(ok = fwd(i + 1, t + gridDim.x))) break;
        // (D W)[128 x k] = D[128 x 32] W[32 x k]
        if (!(ok = mbar_wait(d_full, ph, p.err, 15, p.wait_ns))) break;
        if (i >= 1 && !(ok = mbar_wait(din_empty, ph ^ 1u, p.err, 16, p.wait_ns))) break;
        tc_fence_after();
        const uint32_t d_s = smem_u32(smem + HeadSmem::kD);
        const uint32_t wn = smem_u32(smem + HeadSmem::kW + net * kWNet) + kWNet / 2;
        const uint32_t id_in = idesc_tf32(kHeadRows, p.k[net], false, true);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_tf32(tmem + kColDin, desc_kmajor(d_s + 32 * j), desc_mnmajor(wn + 1024 * j), id_in,
                   j > 0 ? 1u : 0u);
        mma_commit(din_full);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter: rows 32q..32q+31 of a tile
    const bool loss_group = warp < 2 + kHeadEpi;
    if (warp == 2) {
      // per-dimension constants of the log-likelihood (loss kernel)
      const int k = lane;
      const float l = k < p.A ? p.log_std[k] : 0.0f;
      kconst[k] = l;
      kconst[32 + k] = expf(l);
      kconst[64 + k] = expf(-l);
      kconst[96 + k] = expf(-2.0f * l);
      kconst[128 + k] = __frcp_rn(kconst[32 + k]);
    } else if (warp == 3) {
      bias[lane] = p.b[0][lane];
      bias[32 + lane] = p.b[1][lane];
    }
    named_sync_epi();
    const uint32_t row_off = (uint32_t)lane * 128u, sw = (uint32_t)(lane & 7);
    const int pr = blockIdx.x * kHeadEpi + q;  // this quarter's partial row
    bool ok = true;
    if (loss_group) {
      // ---------------------------------------------------- loss warps
      const float lo = 1.0f - p.clip, hi = 1.0f + p.clip;
      const float ent_term = -p.entropy_coef * p.scale;
      const int A = p.A;
      // running sums over this warp's rows of every tile: lane j holds
      // column j of the log_std gradient and of each output bias gradient
      float acc_gl = 0.0f, acc_gb0 = 0.0f, acc_gb1 = 0.0f;
      float acc_surr = 0.0f, acc_vloss = 0.0f, acc_kl = 0.0f;
      const uint32_t dreg = smem_u32(smem + HeadSmem::kD) + (uint32_t)(q * 32 * 128);
      float *sm = reinterpret_cast<float *>(smem + HeadSmem::kD + q * 32 * 128);
      int i = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        const int net = t >= p.blocks ? 1 : 0;
        const int m0 = (t - net * p.blocks) * kHeadRows;
        const uint32_t ph = (uint32_t)i & 1u;
        const int row0 = m0 + 32 * q;
        const int64_t s = (int64_t)row0 + lane;
        const bool live = s < p.rows;
        // the row's loss inputs.  The warp's 32 action (and mean_old) rows
        // are one contiguous run of 32 A floats: loaded coalesced, staged in
        // the warp's 4 KB of the delta tile and read back a row per lane (A
        // odd: no bank conflicts).
        float ac[32], mo[32];
        float lpo = 0.0f, adv = 0.0f, vo = 0.0f, R = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; ++k) ac[k] = mo[k] = 0.0f;
        const int nf = net == 0 ? (row0 < p.rows ? min(32, p.rows - row0) : 0) * A : 0;
        float x[32], y[32];
        {
          const float *ga = p.action + (int64_t)row0 * A, *gm = p.mean_old + (int64_t)row0 * A;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int e = lane + 32 * j;
            x[j] = e < nf ? __ldg(ga + e) : 0.0f;
            y[j] = e < nf ? __ldg(gm + e) : 0.0f;
          }
        }
        if (live) {
          if (net == 0) {
            lpo = __ldg(p.logp_old + s);
            adv = __ldg(p.adv + s);
          } else {
            vo = __ldg(p.value_old + s);
            R = __ldg(p.ret + s);
          }
        }
        // the delta tile is free once the previous tile's D W has read it
        // and this warp's previous store out of it is done reading
        if (i >= 1) {
          if (ok) ok = mbar_wait(din_full, ph ^ 1u, p.err, 19, p.wait_ns);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if (net == 0) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (lane + 32 * j < nf) sm[lane + 32 * j] = x[j];
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (live && k < A) ac[k] = sm[lane * A + k];
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (lane + 32 * j < nf) sm[lane + 32 * j] = y[j];
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (live && k < A) mo[k] = sm[lane * A + k];
          __syncwarp();
        }
        // ---- the forward output of the row
        if (ok) ok = mbar_wait(out_full, ph, p.err, 17, p.wait_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem + kColOut + ((uint32_t)(q * 32) << 16), r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(out_empty);
        float g[32], gl[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) g[k] = gl[k] = 0.0f;
        if (net == 0) {
          // ---- actor: logp, ratio, clipped surrogate, KL, gradients
          // (ppo.rs:297-305, 327-334, 410-433; the loss kernel's operations)
          float d[32], lp = 0.0f, kl = 0.0f;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            d[k] = 0.0f;
            if (live && k < A) {
              const float mu = __uint_as_float(r[k]) + bias[k];
              d[k] = __fsub_rn(ac[k], mu);
              const float z = div_rn(d[k], kconst[32 + k], kconst[128 + k]);
              const float tk = __fsub_rn(
                  __fsub_rn(__fmul_rn(__fmul_rn(-0.5f, z), z), kconst[k]), kLogSqrt2PiH);
              lp = __fadd_rn(lp, tk);
              const float dk = (mu - mo[k]) * kconst[64 + k];
              kl += 0.5f * (dk * dk);
            }
          }
          if (live) {
            const float ratio = expf(lp - lpo);
            const float rc = fminf(fmaxf(ratio, lo), hi);
            const bool clipped = (adv >= 0.0f && ratio > hi) || (adv < 0.0f && ratio < lo);
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              if (k < A) {
                float gls = 0.0f;
                if (!clipped) {
                  g[k] = -(adv * ratio * d[k] * kconst[96 + k]) * p.scale;
                  const float dls = adv * ratio * ((d[k] * d[k]) * kconst[96 + k] - 1.0f);
                  gls = -dls * p.scale;
                }
                gl[k] = gls + ent_term;
              }
            }
            acc_surr += fminf(ratio * adv, rc * adv) * p.scale;
            acc_kl += kl * p.scale;
          }
        } else if (live) {
          // ---- critic: clipped value loss (ppo.rs:435-450)
          const float v = __uint_as_float(r[0]) + bias[32];
          const float vc = vo + fminf(fmaxf(v - vo, -p.clip), p.clip);
          const float eu = v - R, ec = vc - R;
          const float lu = eu * eu, lc = ec * ec;
          float vloss, dv;
          if (lc > lu) {
            vloss = lc;
            dv = 2.0f * ec;
          } else {
            vloss = lu;
            dv = 2.0f * eu;
          }
          acc_vloss += vloss * p.scale;
          g[0] = p.value_coef * dv * p.scale;
        }
        // ---- column sums of this warp's rows, staged in its 4 KB
        if (net == 0) {
          stage_row(dreg + row_off, sw, gl);
          __syncwarp();
          acc_gl += colsum_staged(dreg, lane);
          __syncwarp();
        }
        stage_row(dreg + row_off, sw, g);
        __syncwarp();
        {
          const float cs = colsum_staged(dreg, lane);
          if (net == 0)
            acc_gb0 += cs;
          else
            acc_gb1 += cs;
        }
        __syncwarp();
        // the delta, rounded to tf32: the operand of D W, and the output
        // layer's weight-gradient input in memory (a quarter wholly past the
        // last row stores nothing)
#pragma unroll
        for (int k = 0; k < 32; ++k) g[k] = round_tf32(g[k]);
        stage_row(dreg + row_off, sw, g);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < p.rows) {
            tma_store_3d(&maps.dout[net], smem + (dreg - smem_u32(smem)), 0, row0, 0);
            bulk_commit();
          }
          mbar_arrive(d_full);
        }
      }
      acc_surr = warp_sum_f(acc_surr);
      acc_vloss = warp_sum_f(acc_vloss);
      acc_kl = warp_sum_f(acc_kl);
      float *row = p.part + (int64_t)pr * kHeadWidth;
      row[lane] = lane < A ? acc_gl : 0.0f;
      row[32 + lane] = lane < A ? acc_gb0 : 0.0f;
      if (lane < 4)
        row[64 + lane] = lane == 0 ? acc_surr : (lane == 1 ? acc_vloss : (lane == 2 ? acc_kl : 0.0f));
      row[68 + lane] = lane == 0 ? acc_gb1 : 0.0f;
    } else {
      // ------------------------------------------ input-gradient warps
      // running sums in shared memory: lane j holds column 32c + j of the
      // last hidden bias gradient of each net (the chunk loop stays rolled:
      // one copy of its code)
      float *hb = (float *)(smem + HeadSmem::kHb) + q * 2 * (kHeadMaxK / 32) * 32;
      for (int e = lane; e < 2 * (kHeadMaxK / 32) * 32; e += 32) hb[e] = 0.0f;
      int i = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        const int net = t >= p.blocks ? 1 : 0;
        const int m0 = (t - net * p.blocks) * kHeadRows;
        const int nk = p.k[net] / 32;
        const int b = i & 1;
        const int row0 = m0 + 32 * q;
        const bool live = (int64_t)row0 + lane < p.rows;
        if (ok) ok = mbar_wait(din_full, (uint32_t)i & 1u, p.err, 18, p.wait_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t abuf = smem_u32(smem + HeadSmem::kA0 + b * kABuf) + (uint32_t)(q * 32 * 128);
#pragma unroll 1
        for (int c = 0; c < nk; ++c) {
          uint32_t v32[32];
          tmem_ld32(tmem + kColDin + 32u * c + ((uint32_t)(q * 32) << 16), v32);
          if (c == nk - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(din_empty);
          }
          const uint32_t reg = abuf + (uint32_t)c * kKBlock;
          float y[32], v[32];
          {
            uint32_t a8[8];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) a8[cc] = reg + row_off + ((cc ^ sw) << 4);
            ld_shared4x8(a8, y);
          }
          // ELU' from the stored activation (net.rs:19-22): 1 above 0, else
          // a + 1 = min(a + 1, 1); rows past the end hold 0
#pragma unroll
          for (int k = 0; k < 32; ++k)
            v[k] = live ? __uint_as_float(v32[k]) * fmin_nan(y[k] + 1.0f, 1.0f) : 0.0f;
          // (each lane reads and overwrites only its own row; the column
          // sum then reads every row)
          stage_row(reg + row_off, sw, v);
          __syncwarp();
          hb[(net * (kHeadMaxK / 32) + c) * 32 + lane] += colsum_staged(reg, lane);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = round_tf32(v[k]);
          stage_row(reg + row_off, sw, v);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < p.rows) {
            tma_store_3d(&maps.din[net], smem + (reg - smem_u32(smem)), 32 * c, row0, 0);
            bulk_commit();
          }
        }
        // the activation buffer goes back to the producer once this warp's
        // stores out of it are done reading
        if (lane == 0) {
          bulk_wait_read<0>();
          mbar_arrive(&a_empty[b]);
        }
        __syncwarp();
      }
      for (int k = 0; k < 2; ++k)
        for (int c = 0; c < p.k[k] / 32; ++c)
          p.colsum[k][(int64_t)pr * p.k[k] + 32 * c + lane] =
              hb[(k * (kHeadMaxK / 32) + c) * 32 + lane];
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

int head_grid(int64_t rows) {
  const int64_t tiles = 2 * ((rows + kHeadRows - 1) / kHeadRows);
  return (int)std::max<int64_t>(1, std::min<int64_t>(tiles, tc_sm_count()));
}

}  // namespace

int head_partial_rows(int64_t rows) { return head_grid(rows) * kHeadEpi; }

zrl_status head_tc(GemmEngine *eng, const HeadArgs &a, cudaStream_t s, std::string *err) {
  if (a.rows <= 0) return ZRL_OK;
  if (a.A < 1 || a.A > 32 || a.rows > INT32_MAX) {
    *err = "head: action dimension must be 1..32";
    return ZRL_INVALID_ARG;
  }
  HeadMaps maps;
  HeadParams p{};
  for (int k = 0; k < 2; ++k) {
    const HeadNet &n = a.net[k];
    if (n.k < 32 || n.k > kHeadMaxK || n.k % 32) {
      *err = "head: the last hidden layer must be 32..128 wide (padded)";
      return ZRL_INVALID_ARG;
    }
    if (!tc_tensor_map(eng, &maps.a[k], n.a, a.rows, n.k, n.k, kHeadRows, 0, err) ||
        !tc_tensor_map(eng, &maps.wk[k], n.w, 32, n.k, n.k, 32, 0, err) ||
        !tc_tensor_map(eng, &maps.wn[k], n.w, 32, n.k, n.k, 32, 1, err) ||
        !tc_tensor_map(eng, &maps.dout[k], n.d_out, a.rows, 32, 32, 1, 2, err) ||
        !tc_tensor_map(eng, &maps.din[k], n.d_in, a.rows, n.k, n.k, 1, 2, err))
      return ZRL_CUDA_ERROR;
    p.k[k] = n.k;
    p.b[k] = n.b;
    p.colsum[k] = n.colsum;
  }
  p.action = a.action;
  p.mean_old = a.mean_old;
  p.logp_old = a.logp_old;
  p.value_old = a.value_old;
  p.adv = a.adv;
  p.ret = a.ret;
  p.log_std = a.log_std;
  p.A = a.A;
  p.rows = (int)a.rows;
  p.blocks = (int)((a.rows + kHeadRows - 1) / kHeadRows);
  p.scale = a.scale;
  p.clip = a.clip;
  p.entropy_coef = a.entropy_coef;
  p.value_coef = a.value_coef;
  p.part = a.part;
  p.err = a.err;
  p.wait_ns = eng->wait_ns;
  // the shared-memory opt-in belongs to the current device's context: set
  // once per device
  constexpr int kMaxDevices = 64;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = "head: no usable current device";
    return ZRL_CUDA_ERROR;
  }
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         HeadSmem::kBytes);
    if (e != cudaSuccess) {
      *err = std::string("head: ") + cudaGetErrorString(e);
      return ZRL_CUDA_ERROR;
    }
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(head_grid(a.rows));
  cfg.blockDim = dim3(kHeadThreads);
  cfg.dynamicSmemBytes = HeadSmem::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, head_kernel, maps, p);
  if (e != cudaSuccess) {
    *err = std::string("head launch: ") + cudaGetErrorString(e);
    return ZRL_CUDA_ERROR;
  }
  return ZRL_OK;
}

}  // namespace zrl
