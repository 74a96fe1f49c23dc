// kernels.cu -- the bandwidth-bound kernels of the PPO update.
//
// Arithmetic that the reference does in plain f32 and that has to match it
// bit for bit (GAE, the normalizers, Adam) uses the explicitly rounded
// intrinsics (__fadd_rn, __fmul_rn, ...) so that the compiler cannot fuse a
// multiply and an add into one FMA.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "zrl_internal.h"

namespace zrl {

namespace {

// Programmatic dependent launch.  A kernel launched with launch_pdl may
// start while the previous kernel in the stream is still running: it must
// call pdl_wait() before touching global memory, after which that kernel
// has completed and its writes are visible.  pdl_trigger() lets the next
// kernel begin its own launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... K, typename... A>
void launch_pdl(void (*kfn)(K...), unsigned grid, unsigned block, cudaStream_t s, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kfn, args...);
}


constexpr float kLogSqrt2Pi = 0.9189385f;  // ppo.rs:18

// tf32 with round-to-nearest (ties away): the tensor-core GEMMs then read
// these operands exactly instead of truncating them.
// GEMM-operand storage modes (OperandMode): 0 fp32 as is, 1 fp32 rounded to
// tf32 (RN), 2 bf16 (RN-even).  `p` points at element 0 of the row; for
// bf16 the row holds 2-byte elements.
__device__ __forceinline__ void store_operand(float *p, int64_t i, float x, int mode) {
  if (mode == 2) {
    reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(x);
  } else {
    uint32_t r;
    if (mode == 1) {
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
      x = __uint_as_float(r);
    }
    p[i] = x;
  }
}

__device__ __forceinline__ float rna_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum in a fixed order (warp shuffles, then warp 0 over warps).
template <typename T>
__device__ T block_sum(T v, T *sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if constexpr (sizeof(T) == 8)
    v = warp_sum_d(v);
  else
    v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  T r = 0;
  if (w == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    r = lane < nw ? sh[lane] : T(0);
    if constexpr (sizeof(T) == 8)
      r = warp_sum_d(r);
    else
      r = warp_sum(r);
  }
  return r;  // valid in thread 0
}

// ---------------------------------------------------------------- GAE

// One block handles kEnvs consecutive environments: their [kEnvs*T] slices
// of rewards/values/dones are contiguous, so they are staged through shared
// memory with coalesced loads; one thread per env runs the reverse scan
// (ppo.rs:689-702); results go back through shared memory.
constexpr int kGaeEnvs = 32;
constexpr int kGaeThreads = 128;

// Shared memory per block when staged: kGaeEnvs * T * (4 floats + 1 byte).
// Longer horizons read global memory directly (same arithmetic).
constexpr int kGaeMaxStagedT = 48 * 1024 / (kGaeEnvs * 17);

template <bool STAGED>
__global__ void __launch_bounds__(kGaeThreads)
gae_kernel(GaeArgs a, double *partials) {
  extern __shared__ float sm[];
  const int64_t e0 = (int64_t)blockIdx.x * kGaeEnvs;
  const int ne = (int)(a.n_envs - e0 < kGaeEnvs ? a.n_envs - e0 : kGaeEnvs);
  const int T = (int)a.T;
  const int cnt = ne * T;
  const int64_t base = e0 * T;
  const float *r_ = a.rewards + base;
  const float *v_ = a.values + base;
  const uint8_t *d_ = a.dones + base;
  float *adv_ = a.adv + base;
  float *ret_ = a.ret + base;
  if (STAGED) {
    float *s_r = sm;
    float *s_v = s_r + kGaeEnvs * T;
    float *s_adv = s_v + kGaeEnvs * T;
    float *s_ret = s_adv + kGaeEnvs * T;
    uint8_t *s_d = reinterpret_cast<uint8_t *>(s_ret + kGaeEnvs * T);
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
      s_r[i] = r_[i];
      s_v[i] = v_[i];
      s_d[i] = d_[i];
    }
    __syncthreads();
    r_ = s_r;
    v_ = s_v;
    d_ = s_d;
    adv_ = s_adv;
    ret_ = s_ret;
  }
  if (threadIdx.x < ne) {
    const int e = threadIdx.x;
    const float gl = __fmul_rn(a.gamma, a.lam);
    float acc = 0.0f;
    float next_v = a.last_values[e0 + e];
    for (int t = T - 1; t >= 0; --t) {
      const int i = e * T + t;
      const float nt = d_[i] ? 0.0f : 1.0f;
      // delta = r + gamma * next_v * nt - v   (left to right, ppo.rs:696)
      const float delta =
          __fsub_rn(__fadd_rn(r_[i], __fmul_rn(__fmul_rn(a.gamma, next_v), nt)), v_[i]);
      // gae = delta + gamma * lam * nt * gae   (ppo.rs:697)
      acc = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nt), acc));
      adv_[i] = acc;
      ret_[i] = __fadd_rn(acc, v_[i]);
      next_v = v_[i];
    }
  }
  __syncthreads();
  double part = 0.0;
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
    const float av = adv_[i];  // shared (staged) or global, written above
    if (STAGED) {
      a.adv[base + i] = av;
      a.ret[base + i] = ret_[i];
    }
    part += (double)av;
  }
  __shared__ double sh[32];
  double tot = block_sum(part, sh);
  if (threadIdx.x == 0 && partials) partials[blockIdx.x] = tot;
}

// ------------------------------------------------------- advantage moments

constexpr int kAdvThreads = 256;

__global__ void adv_sum_kernel(const float *adv, int64_t n, double *partials) {
  double s = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    s += (double)adv[i];
  __shared__ double sh[32];
  double t = block_sum(s, sh);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// One block: moments[slot] = sum of partials (fixed order).
__global__ void reduce_partials_kernel(const double *partials, int nblk,
                                       double *moments, int slot) {
  double s = 0.0;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) s += partials[i];
  __shared__ double sh[32];
  double t = block_sum(s, sh);
  if (threadIdx.x == 0) moments[slot] = t;
}

__device__ __forceinline__ float adv_mean_from(const double *moments,
                                               int64_t n_global) {
  return (float)(moments[0] / (double)n_global);
}

__global__ void adv_sqdev_kernel(const float *adv, int64_t n,
                                 const double *moments, int64_t n_global,
                                 double *partials) {
  const float mean = adv_mean_from(moments, n_global);
  double s = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float d = __fsub_rn(adv[i], mean);
    s += (double)d * (double)d;
  }
  __shared__ double sh[32];
  double t = block_sum(s, sh);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

__global__ void adv_finalize_kernel(const double *moments, int64_t n_global,
                                    DevState *st) {
  const float mean = adv_mean_from(moments, n_global);
  const float var = (float)(moments[1] / (double)n_global);
  float sd = __fsqrt_rn(var);
  if (sd < 1e-6f) sd = 1e-6f;  // ppo.rs:345
  st->adv_mean = mean;
  st->adv_sd = sd;
}

// ------------------------------------------------------------ gather

// One warp per output position: copies row order[p] of every batch array --
// the observation rows already normalized (normalize_rows_kernel, once per
// update) as 16-byte pieces -- and applies the advantage normalization
// (ppo.rs:346-348) to adv.  With the mirror augmentation a virtual row
// r < n_base takes base row r's mirrored normalized rows and its action and
// mean_old through the action space's signed permutation.
__global__ void gather_kernel(GatherArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int R = 2;  // rows per warp and pass, their loads all in flight together
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float am = a.st->adv_mean, asd = a.st->adv_sd;
  // 16-byte pieces per padded observation row
  const int qa = a.odp * a.x_bytes / 16, qc = a.cdp * a.x_bytes / 16;
  const bool small = qa <= 32 && qc <= 32 && a.A <= 32;
  const bool al = lane < a.A;
  const int ai = al && a.n_base > 0 ? a.m_aperm[lane] : lane;
  const float asg = al && a.n_base > 0 ? a.m_asign[lane] : 1.0f;
  for (int64_t p0 = warp * R; p0 < a.n_used; p0 += nwarps * R) {
    int64_t src[R];
    bool mir[R], live[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      live[u] = p0 + u < a.n_used;
      const int64_t r = live[u] ? a.order[p0 + u] : 0;
      mir[u] = a.n_base > 0 && r < a.n_base;
      src[u] = a.n_base > 0 ? (mir[u] ? r : r - a.n_base) : r;
    }
    if (small) {
      // every load of both rows first, then every store
      float4 va[R], vc[R];
      float act[R], mo[R], sc[R];
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const float4 *xa = reinterpret_cast<const float4 *>(mir[u] ? a.xm_a : a.xn_a) + src[u] * qa;
        const float4 *xc = reinterpret_cast<const float4 *>(mir[u] ? a.xm_c : a.xn_c) + src[u] * qc;
        va[u] = live[u] && lane < qa ? xa[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        vc[u] = live[u] && lane < qc ? xc[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        act[u] = mo[u] = sc[u] = 0.0f;
        if (live[u] && al) {
          const int kk = mir[u] ? ai : lane;
          act[u] = a.action[src[u] * a.A + kk];
          mo[u] = a.mean_old[src[u] * a.A + kk];
        }
        if (live[u] && lane < 4) {
          const float *col = lane == 0 ? a.logp_old : lane == 1 ? a.value_old
                           : lane == 2 ? a.adv : a.ret;
          sc[u] = col[src[u]];
        }
      }
#pragma unroll
      for (int u = 0; u < R; ++u) {
        if (!live[u]) break;
        const int64_t p = p0 + u;
        if (lane < qa) reinterpret_cast<float4 *>(a.x_a)[p * qa + lane] = va[u];
        if (lane < qc) reinterpret_cast<float4 *>(a.x_c)[p * qc + lane] = vc[u];
        if (al) {
          a.g_action[p * a.A + lane] = mir[u] ? act[u] * asg : act[u];
          a.g_mean_old[p * a.A + lane] = mir[u] ? mo[u] * asg : mo[u];
        }
        if (lane == 0) a.g_logp_old[p] = sc[u];
        else if (lane == 1) a.g_value_old[p] = sc[u];
        else if (lane == 2)
          a.g_adv[p] = a.apply_adv_norm ? __fdiv_rn(__fsub_rn(sc[u], am), asd) : sc[u];
        else if (lane == 3) a.g_ret[p] = sc[u];
      }
      continue;
    }
    // wide rows (more than 512 bytes, or more than 32 action dimensions)
    for (int u = 0; u < R; ++u) {
      if (!live[u]) break;
      const int64_t p = p0 + u;
      const float4 *xa = reinterpret_cast<const float4 *>(mir[u] ? a.xm_a : a.xn_a) + src[u] * qa;
      const float4 *xc = reinterpret_cast<const float4 *>(mir[u] ? a.xm_c : a.xn_c) + src[u] * qc;
      for (int i = lane; i < qa; i += 32) reinterpret_cast<float4 *>(a.x_a)[p * qa + i] = xa[i];
      for (int i = lane; i < qc; i += 32) reinterpret_cast<float4 *>(a.x_c)[p * qc + i] = xc[i];
      for (int k = lane; k < a.A; k += 32) {
        const int kk = mir[u] ? a.m_aperm[k] : k;
        const float sg = mir[u] ? a.m_asign[k] : 1.0f;
        a.g_action[p * a.A + k] = a.action[src[u] * a.A + kk] * sg;
        a.g_mean_old[p * a.A + k] = a.mean_old[src[u] * a.A + kk] * sg;
      }
      if (lane == 0) {
        a.g_logp_old[p] = a.logp_old[src[u]];
        a.g_value_old[p] = a.value_old[src[u]];
        const float v = a.adv[src[u]];
        a.g_adv[p] = a.apply_adv_norm ? __fdiv_rn(__fsub_rn(v, am), asd) : v;
        a.g_ret[p] = a.ret[src[u]];
      }
    }
  }
}

// sd[i] = sqrt(max(m2[i]/count, 1e-8)) in f32, the divisor of
// Normalizer::normalize.
__global__ void norm_prepare_kernel(const float *m2, float count, int dim,
                                    float *sd) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dim) {
    float var = __fdiv_rn(m2[i], count);
    if (var < 1e-8f) var = 1e-8f;
    sd[i] = __fsqrt_rn(var);
  }
}

// One warp per row (rows strided over the grid): lane i takes columns
// i, i+32, ... of the padded row, so the index math has no division.
// With perm/sign (the mirror augmentation) row r is first mapped by the
// signed permutation: x'[i] = sign[i] * x[perm[i]].
// One thread per padded column (blockDim = pitch, at most 256), a block per
// group of kNormRows rows: every row's load is issued before the first
// division, so each warp keeps kNormRows 128-byte loads in flight.
constexpr int kNormRows = 8;

__global__ void normalize_rows_kernel(const float *__restrict__ x, int64_t n, int dim,
                                      int pitch, const float *__restrict__ mean,
                                      const float *__restrict__ sd, float *__restrict__ out,
                                      int mode, const int32_t *__restrict__ perm,
                                      const float *__restrict__ sign) {
  const int i = threadIdx.x;
  const bool col = i < dim;
  const int src = col ? (perm ? perm[i] : i) : 0;
  const float sg = col && perm ? sign[i] : 1.0f;
  const float mu = col ? mean[i] : 0.0f, s = col ? sd[i] : 1.0f;
  for (int64_t r0 = (int64_t)blockIdx.x * kNormRows; r0 < n; r0 += (int64_t)gridDim.x * kNormRows) {
    float v[kNormRows];
#pragma unroll
    for (int u = 0; u < kNormRows; ++u)
      v[u] = col && r0 + u < n ? x[(r0 + u) * dim + src] : 0.0f;
#pragma unroll
    for (int u = 0; u < kNormRows; ++u) {
      if (r0 + u >= n) break;
      float y = 0.0f;
      if (col) {
        const float vv = perm ? v[u] * sg : v[u];
        y = __fdiv_rn(__fsub_rn(vv, mu), s);
        y = fminf(fmaxf(y, -5.0f), 5.0f);
      }
      store_operand(out, (r0 + u) * pitch + i, y, mode);
    }
  }
}

__global__ void round_copy_kernel(const float *src, float *dst, int64_t n, int mode) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_operand(dst, i, src[i], mode);
}

// ------------------------------------------------------------ PPO loss

constexpr int kLossThreads = 256;
constexpr int kLossMaxA = 128;  // 4 action dims per lane

// One warp per sample (ppo.rs:410-452).  Lane k holds action dims k,
// k+32, ...; log-prob and KL are warp sums.  Per-block partials of the
// log_std gradient and of the three statistics are written to scratch; the
// last block to finish adds the partials in block order (deterministic).
__global__ void __launch_bounds__(kLossThreads)
loss_kernel(LossArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nwb = blockDim.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * nwb + wid;
  const int64_t nw = (int64_t)gridDim.x * nwb;
  const int A = a.A;
  float ls[4], sd[4], inv_var[4], inv_sd[4], gls[4], gmu[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = lane + 32 * j;
    ls[j] = k < A ? a.log_std[k] : 0.0f;
    sd[j] = expf(ls[j]);
    inv_var[j] = expf(-2.0f * ls[j]);
    inv_sd[j] = expf(-ls[j]);
    gls[j] = 0.0f;
    gmu[j] = 0.0f;
  }
  float acc_surr = 0.0f, acc_vloss = 0.0f, acc_kl = 0.0f, acc_gv = 0.0f;
  const float lo = 1.0f - a.clip, hi = 1.0f + a.clip;
  const float ent_term = -a.entropy_coef * a.scale;
  // The loads of one sample: its action-dimension rows by lane (4 per lane
  // for A <= 128) and the five per-sample scalars by lanes 0-4.  The warp
  // walks its samples with the next sample's loads in flight while the
  // current one is computed.
  struct Row {
    float mu[4], ac[4], mo[4], scal;
  };
  auto fetch = [&](int64_t s, Row &r) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = lane + 32 * j;
      r.mu[j] = r.ac[j] = r.mo[j] = 0.0f;
      if (k < A) {
        r.mu[j] = a.mean[s * a.Ap + k];
        r.ac[j] = a.action[s * A + k];
        r.mo[j] = a.mean_old[s * A + k];
      }
    }
    r.scal = 0.0f;
    if (lane == 0) r.scal = a.logp_old[s];
    else if (lane == 1) r.scal = a.adv[s];
    else if (lane == 2) r.scal = a.value[s * a.cp];
    else if (lane == 3) r.scal = a.value_old[s];
    else if (lane == 4) r.scal = a.ret[s];
  };
  Row nxt;
  if (gw < a.mb) fetch(gw, nxt);
  for (int64_t s = gw; s < a.mb; s += nw) {
    const Row cur = nxt;
    if (s + nw < a.mb) fetch(s + nw, nxt);
    float d_r[4];
    float lp = 0.0f, kl = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = lane + 32 * j;
      d_r[j] = 0.0f;
      if (k < A) {
        d_r[j] = cur.ac[j] - cur.mu[j];
        const float z = d_r[j] / sd[j];
        lp += -0.5f * z * z - ls[j] - kLogSqrt2Pi;
        const float dk = (cur.mu[j] - cur.mo[j]) * inv_sd[j];
        kl += 0.5f * (dk * dk);
      }
    }
    lp = warp_sum(lp);
    kl = warp_sum(kl);
    const float ratio = expf(lp - __shfl_sync(0xffffffffu, cur.scal, 0));
    const float adv = __shfl_sync(0xffffffffu, cur.scal, 1);
    const float v = __shfl_sync(0xffffffffu, cur.scal, 2);
    const float vo = __shfl_sync(0xffffffffu, cur.scal, 3);
    const float R = __shfl_sync(0xffffffffu, cur.scal, 4);
    const float rc = fminf(fmaxf(ratio, lo), hi);
    const float surr = fminf(ratio * adv, rc * adv);
    const bool clipped = (adv >= 0.0f && ratio > hi) || (adv < 0.0f && ratio < lo);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = lane + 32 * j;
      float g = 0.0f;
      if (k < A) {
        if (!clipped) {
          const float d = d_r[j];
          g = -(adv * ratio * d * inv_var[j]) * a.scale;
          const float dls = adv * ratio * ((d * d) * inv_var[j] - 1.0f);
          gls[j] += -dls * a.scale;
        }
        gls[j] += ent_term;
        gmu[j] += g;
      }
      if (k < a.Ap) store_operand(a.d_actor, s * a.Ap + k, g, a.out_mode);
    }
    if (lane == 0) {
      acc_surr += surr * a.scale;
      acc_kl += kl * a.scale;
      // clipped value loss, ppo.rs:439-449
      const float vc = vo + fminf(fmaxf(v - vo, -a.clip), a.clip);
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
      acc_vloss += vloss * a.scale;
      const float gv = a.value_coef * dv * a.scale;
      acc_gv += gv;
      store_operand(a.d_critic, s * a.cp, gv, a.out_mode);
    }
  }
  // ---- the block's partial row, its warps summed in warp order:
  // [g_logstd (Ap) | db_actor (Ap) | surr vloss kl 0 | db_critic (cp)],
  // zero in the padding; the segment reduce adds the rows of all blocks
  __shared__ float sh[kLossThreads / 32][2 * kLossMaxA + 4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = lane + 32 * j;
    if (k < A) {
      sh[wid][k] = gls[j];
      sh[wid][A + k] = gmu[j];
    }
  }
  if (lane == 0) {
    sh[wid][2 * A] = acc_surr;
    sh[wid][2 * A + 1] = acc_vloss;
    sh[wid][2 * A + 2] = acc_kl;
    sh[wid][2 * A + 3] = acc_gv;
  }
  __syncthreads();
  float *row = a.part + (int64_t)blockIdx.x * a.width;
  for (int c = threadIdx.x; c < a.width; c += blockDim.x) {
    // column c of the row -> column of the warp sums (or padding)
    int src = -1;
    if (c < a.Ap) src = c < A ? c : -1;
    else if (c < 2 * a.Ap) src = c - a.Ap < A ? A + (c - a.Ap) : -1;
    else if (c < 2 * a.Ap + 4) src = c - 2 * a.Ap < 3 ? 2 * A + (c - 2 * a.Ap) : -1;
    else src = c == 2 * a.Ap + 4 ? 2 * A + 3 : -1;
    float t = 0.0f;
    if (src >= 0)
      for (int w = 0; w < nwb; ++w) t += sh[w][src];
    row[c] = t;
  }
}

// Quad-per-sample form of the same loss for A <= 32 and Ap == 32 (the
// per-sample arithmetic of loss_kernel).  Four lanes take one sample, lane
// q of the quad dimensions 8q .. 8q+7, so a warp covers 8 samples: their
// mean rows load as two float4 per lane (coalesced), the log-prob and KL
// sums are two shuffle steps inside the quad, and each lane keeps the
// per-dimension sums of its 8 dimensions across the samples it visits.
// At the end the warp folds its 8 sample slots (3 shuffle steps), and the
// block's warps are summed in warp order into the block's partial row
// (the layout of loss_kernel's).
constexpr int kLossQuadThreads = 256;

// three blocks per SM (registers kept under 85): the sample groups of a
// C2 minibatch then run in one wave
__global__ void __launch_bounds__(kLossQuadThreads, 3)
loss_quad_kernel(LossArgs a) {
  constexpr int NW = kLossQuadThreads / 32;
  __shared__ float wrow[NW][2 * 32 + 4];
  __shared__ float kp[4][32];  // per dimension: log_std, sd, 1 / sd, 1 / var
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int q = lane & 3, slot = lane >> 2;
  const int A = a.A;
  if (threadIdx.x < 32) {
    const int k = threadIdx.x;
    const float l = k < A ? a.log_std[k] : 0.0f;
    kp[0][k] = l;
    kp[1][k] = expf(l);
    kp[2][k] = expf(-l);
    kp[3][k] = expf(-2.0f * l);
  }
  __syncthreads();
  const float *ls = kp[0] + 8 * q, *sd = kp[1] + 8 * q, *inv_sd = kp[2] + 8 * q,
              *inv_var = kp[3] + 8 * q;
  float gl[8], gm[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) gl[i] = gm[i] = 0.0f;
  const float lo = 1.0f - a.clip, hi = 1.0f + a.clip;
  const float ent_term = -a.entropy_coef * a.scale;
  float acc_surr = 0.0f, acc_vloss = 0.0f, acc_kl = 0.0f, acc_gv = 0.0f;
  // the warp walks groups of 8 samples; every lane runs every iteration
  // (the quad shuffles take the full warp), lanes past the end as dead
  const int64_t stride = (int64_t)gridDim.x * kLossQuadThreads / 4;
  for (int64_t s8 = ((int64_t)blockIdx.x * kLossQuadThreads + wid * 32) / 4; s8 < a.mb;
       s8 += stride) {
    const int64_t s = s8 + slot;
    const bool live = s < a.mb;
    float mu[8], ac[8], mo[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mu[i] = ac[i] = mo[i] = 0.0f;
    float lpo = 0.0f, adv = 0.0f;
    if (live) {
      const float4 *m4 = reinterpret_cast<const float4 *>(a.mean + s * 32 + 8 * q);
      const float4 x0 = m4[0], x1 = m4[1];
      mu[0] = x0.x, mu[1] = x0.y, mu[2] = x0.z, mu[3] = x0.w;
      mu[4] = x1.x, mu[5] = x1.y, mu[6] = x1.z, mu[7] = x1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = 8 * q + i;
        if (k < A) {
          ac[i] = a.action[s * A + k];
          mo[i] = a.mean_old[s * A + k];
        }
      }
      lpo = a.logp_old[s];
      adv = a.adv[s];
    }
    float v = 0.0f, vo = 0.0f, R = 0.0f;
    if (q == 0 && live) {
      v = a.value[s * a.cp];
      vo = a.value_old[s];
      R = a.ret[s];
    }
    float d[8], t[8], kl = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      d[i] = t[i] = 0.0f;
      if (live && 8 * q + i < A) {
        d[i] = __fsub_rn(ac[i], mu[i]);
        const float z = __fdiv_rn(d[i], sd[i]);
        t[i] = __fsub_rn(__fsub_rn(__fmul_rn(__fmul_rn(-0.5f, z), z), ls[i]), kLogSqrt2Pi);
        const float dk = (mu[i] - mo[i]) * inv_sd[i];
        kl += 0.5f * (dk * dk);
      }
    }
    // log-prob summed over k = 0, 1, ... in order, as ActorCritic::logp
    // (ppo.rs:297-305) and the rollout that recorded logp_old do: the
    // running sum passes through the quad's lanes in turn, so the ratio at
    // an unchanged policy is exactly 1
    float lp = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float prev = __shfl_up_sync(0xffffffffu, lp, 1);
      if (q == r) {
        if (r > 0) lp = prev;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (8 * q + i < A) lp = __fadd_rn(lp, t[i]);
      }
    }
    lp = __shfl_sync(0xffffffffu, lp, lane | 3);
    kl += __shfl_xor_sync(0xffffffffu, kl, 1);
    kl += __shfl_xor_sync(0xffffffffu, kl, 2);
    const float ratio = expf(lp - lpo);
    const float rc = fminf(fmaxf(ratio, lo), hi);
    const bool clipped = (adv >= 0.0f && ratio > hi) || (adv < 0.0f && ratio < lo);
    float g[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      g[i] = 0.0f;
      if (live && 8 * q + i < A) {
        float gls = 0.0f;  // this sample's log_std gradient term
        if (!clipped) {
          g[i] = -(adv * ratio * d[i] * inv_var[i]) * a.scale;
          const float dls = adv * ratio * ((d[i] * d[i]) * inv_var[i] - 1.0f);
          gls = -dls * a.scale;
        }
        gl[i] += gls + ent_term;
        gm[i] += g[i];
      }
    }
    if (live && a.out_mode == 0) {
      float4 *o = reinterpret_cast<float4 *>(a.d_actor + s * 32 + 8 * q);
      o[0] = make_float4(g[0], g[1], g[2], g[3]);
      o[1] = make_float4(g[4], g[5], g[6], g[7]);
    } else if (live) {
#pragma unroll
      for (int i = 0; i < 8; ++i) store_operand(a.d_actor, s * 32 + 8 * q + i, g[i], a.out_mode);
    }
    if (q == 0 && live) {
      acc_surr += fminf(ratio * adv, rc * adv) * a.scale;
      acc_kl += kl * a.scale;
      // clipped value loss, ppo.rs:439-449
      const float vc = vo + fminf(fmaxf(v - vo, -a.clip), a.clip);
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
      acc_vloss += vloss * a.scale;
      const float gv = a.value_coef * dv * a.scale;
      acc_gv += gv;
      store_operand(a.d_critic, s * a.cp, gv, a.out_mode);
    }
  }
  // fold the warp's 8 sample slots: lane q of slot 0 ends with dimensions
  // 8q .. 8q+7 summed over the warp
#pragma unroll
  for (int off = 4; off < 32; off *= 2)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      gl[i] += __shfl_xor_sync(0xffffffffu, gl[i], off);
      gm[i] += __shfl_xor_sync(0xffffffffu, gm[i], off);
    }
  acc_surr = warp_sum(acc_surr);
  acc_vloss = warp_sum(acc_vloss);
  acc_kl = warp_sum(acc_kl);
  acc_gv = warp_sum(acc_gv);
  if (slot == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wrow[wid][8 * q + i] = gl[i];
      wrow[wid][32 + 8 * q + i] = gm[i];
    }
  }
  if (lane == 0) {
    wrow[wid][64] = acc_surr;
    wrow[wid][65] = acc_vloss;
    wrow[wid][66] = acc_kl;
    wrow[wid][67] = acc_gv;
  }
  __syncthreads();
  // [g_logstd (Ap) | db_actor (Ap) | surr vloss kl 0 | db_critic (cp)]
  const int Ap = a.Ap;
  float *row = a.part + (int64_t)blockIdx.x * a.width;
  for (int c = threadIdx.x; c < a.width; c += blockDim.x) {
    int src = -1;
    if (c < Ap) src = c < A ? c : -1;
    else if (c < 2 * Ap) src = c - Ap < A ? 32 + (c - Ap) : -1;
    else if (c < 2 * Ap + 4) src = c - 2 * Ap < 3 ? 64 + (c - 2 * Ap) : -1;
    else src = c == 2 * Ap + 4 ? 67 : -1;
    float t = 0.0f;
    if (src >= 0)
      for (int w = 0; w < NW; ++w) t += wrow[w][src];
    row[c] = t;
  }
}

// ------------------------------------------------------------ colsum

__global__ void colsum_kernel(const float *x, int64_t rows, int cols, int ld,
                              float *partials, int splits) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int z = blockIdx.y;
  if (c >= cols) return;
  const int64_t chunk = (rows + splits - 1) / splits;
  const int64_t r0 = z * chunk, r1 = (rows < r0 + chunk ? rows : r0 + chunk);
  float s = 0.0f;
  for (int64_t r = r0; r < r1; ++r) s += x[r * ld + c];
  partials[(int64_t)z * cols + c] = s;
}

// ------------------------------------------------------ segment reduce

// Sum of split partials.  A segment with `splits` partial rows is cut into
// G = clamp(splits / 8, 1, 64) split groups (a power of two); a block of
// 512 threads covers 512 / G float4 columns x G groups, consecutive threads
// on consecutive columns (coalesced).  Group j sums splits j, j+G, j+2G,
// ... in split order, loading eight rows at a time before adding them, and
// the G group sums are then added pairwise in a fixed tree -- a fixed
// order, so every run gives the same bits.  Every segment count and stride is a multiple of
// 4 floats and every pointer 16-byte aligned (the padded layout guarantees
// both).
constexpr int kRsThreads = 512;

__host__ __device__ __forceinline__ int rs_groups(int splits) {
  int g = 1;
  while (g < 64 && g * 8 < splits) g *= 2;
  return g;
}
__host__ __device__ __forceinline__ int64_t rs_blocks(int64_t count, int splits) {
  const int64_t cols4 = kRsThreads / rs_groups(splits);
  return (count / 4 + cols4 - 1) / cols4;
}

__device__ void prestep_finish(const PrestepArgs &a, double na, double nc);
template <typename T>
__device__ T block_sum(T v, T *sh);

__global__ void __launch_bounds__(kRsThreads, 2)
reduce_segments_kernel(ReduceSegs segs, PrestepArgs pa, double *partials, unsigned int *ticket,
                       int fuse) {
  pdl_wait();
  pdl_trigger();
  int si = 0;
  while (si + 1 < segs.n && (int)blockIdx.x >= segs.first_block[si + 1]) ++si;
  const int b = (int)blockIdx.x - segs.first_block[si];
  const float *src0 = segs.seg[si].src;
  float *dst = segs.seg[si].dst;
  const int64_t count4 = segs.seg[si].count / 4;
  const int splits = segs.seg[si].splits;
  const int64_t stride4 = segs.seg[si].stride / 4;
  const int G = segs.groups[si];
  const int cols4 = kRsThreads / G;
  const int c = threadIdx.x & (cols4 - 1), grp = threadIdx.x / cols4;
  const int64_t i4 = (int64_t)b * cols4 + c;
  const bool live = i4 < count4;
  const float4 *src = reinterpret_cast<const float4 *>(src0) + i4;
  float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (live) {
    for (int z0 = grp; z0 < splits; z0 += 8 * G) {
      float4 x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int z = z0 + u * G;
        x[u] = z < splits ? __ldcs(src + (int64_t)z * stride4)  // read once: streaming
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        t.x += x[u].x;
        t.y += x[u].y;
        t.z += x[u].z;
        t.w += x[u].w;
      }
    }
  }
  // the G group sums of each column, pairwise in a fixed tree
  __shared__ float4 part[kRsThreads];
  part[threadIdx.x] = t;
  __syncthreads();
  for (int h = G >> 1; h >= 1; h >>= 1) {
    if (grp < h) {
      const float4 x = part[threadIdx.x + h * cols4];
      t.x += x.x;
      t.y += x.y;
      t.z += x.z;
      t.w += x.w;
      part[threadIdx.x] = t;
    }
    __syncthreads();
  }
  double sq = 0.0;
  if (grp == 0 && live) {
    const float4 s4 = t;
    reinterpret_cast<float4 *>(dst)[i4] = s4;
    sq = (double)s4.x * s4.x + (double)s4.y * s4.y + (double)s4.z * s4.z +
         (double)s4.w * s4.w;
  }
  if (!fuse) return;
  // the fused pre-step: squared norms of this block's outputs (one net per
  // segment), block partials, the last block finishes in block order
  __shared__ double sh[32];
  const double tot = block_sum(sq, sh);
  const int net = segs.net[si];
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = net == 0 ? tot : 0.0;
    partials[2 * blockIdx.x + 1] = net == 1 ? tot : 0.0;
  }
  __threadfence();
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  double na = 0.0, nc = 0.0;
  for (int bb = threadIdx.x; bb < (int)gridDim.x; bb += blockDim.x) {
    na += __ldcg(&partials[2 * bb]);
    nc += __ldcg(&partials[2 * bb + 1]);
  }
  na = block_sum(na, sh);
  nc = block_sum(nc, sh);
  if (threadIdx.x != 0) return;
  *ticket = 0u;
  prestep_finish(pa, na, nc);
}

// ------------------------------------------------------------ pre-step

__device__ float powi_f(float a, int b) {
  // square-and-multiply, the f32::powi lowering with a runtime exponent
  const bool recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r = __fmul_rn(r, a);
    b /= 2;
    if (b == 0) break;
    a = __fmul_rn(a, a);
  }
  return recip ? __fdiv_rn(1.0f, r) : r;
}

// The scalar half of the pre-step, given the two squared gradient norms:
// statistics, adaptive LR, per-net clip scales, Adam step counters and
// bias corrections (one thread).
__device__ void prestep_finish(const PrestepArgs &a, double na, double nc) {
  DevState *st = a.st;
  st->sumsq[0] = (float)na;
  st->sumsq[1] = (float)nc;
  const float kl = a.sums3[2];
  // entropy of the pre-step log_std (ppo.rs:308-311, 473)
  const float c = __fadd_rn(0.5f, kLogSqrt2Pi);
  float ent = 0.0f;
  for (int k = 0; k < a.A; ++k) ent = __fadd_rn(ent, __fadd_rn(a.log_std[k], c));
  if (a.count_stats) {
    st->ep_acc[0] += kl;
    st->ep_acc[1] += a.sums3[0];
    st->ep_acc[2] += a.sums3[1];
    st->ep_acc[3] += ent;
  }
  // adaptive LR (ppo.rs:476-482)
  float lr = st->lr;
  if (a.adaptive_lr) {
    if (kl > a.desired_kl * 2.0f)
      lr = fmaxf(__fdiv_rn(lr, 1.5f), a.lr_min);
    else if (kl > 0.0f && kl < a.desired_kl / 2.0f)
      lr = fminf(__fmul_rn(lr, 1.5f), a.lr_max);
  }
  st->lr = lr;
  st->step_lr = lr;
  // per-net clip (net.rs:197-202)
  const float norms[2] = {__fsqrt_rn((float)na), __fsqrt_rn((float)nc)};
  for (int j = 0; j < 2; ++j) {
    const float n = norms[j];
    st->clip_scale[j] =
        (n > a.max_grad_norm && n > 0.0f) ? __fdiv_rn(a.max_grad_norm, n) : 1.0f;
  }
  // Adam steps and bias corrections (net.rs:235-238, ppo.rs:497-500)
  for (int j = 0; j < 3; ++j) {
    const int t = st->t[j] + 1;
    st->t[j] = t;
    st->bc1[j] = __fsub_rn(1.0f, powi_f(0.9f, t));
    st->bc2[j] = __fsub_rn(1.0f, powi_f(0.999f, t));
  }
  if (a.count_stats && a.last_of_epoch) {
    const float inv = __fdiv_rn(1.0f, (float)a.minibatches);
    st->stats[0] = st->ep_acc[0] * inv;
    st->stats[1] = st->ep_acc[1] * inv;
    st->stats[2] = st->ep_acc[2] * inv;
    st->stats[3] = st->ep_acc[3] * inv;
    st->stats[4] = lr;
    for (int j = 0; j < 4; ++j) st->ep_acc[j] = 0.0f;
  }
}

constexpr int kPrestepThreads = 256;

__global__ void __launch_bounds__(kPrestepThreads)
prestep_kernel(PrestepArgs a, double *partials, unsigned int *ticket) {
  pdl_wait();
  pdl_trigger();
  double sa = 0.0, sc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
#pragma unroll 4
  for (int64_t i = a.actor_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
       i < a.actor_end; i += stride) {
    const double g = a.grads[i];
    sa += g * g;
  }
#pragma unroll 4
  for (int64_t i = a.critic_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
       i < a.critic_end; i += stride) {
    const double g = a.grads[i];
    sc += g * g;
  }
  __shared__ double sh[32];
  double ta = block_sum(sa, sh);
  double tc = block_sum(sc, sh);
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = ta;
    partials[2 * blockIdx.x + 1] = tc;
  }
  __threadfence();
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the whole last block: thread b takes block partials b, b + blockDim,
  // ..., then the fixed-order block sum
  double na = 0.0, nc = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    na += __ldcg(&partials[2 * b]);
    nc += __ldcg(&partials[2 * b + 1]);
  }
  na = block_sum(na, sh);
  nc = block_sum(nc, sh);
  if (threadIdx.x != 0) return;
  *ticket = 0u;
  prestep_finish(a, na, nc);
}

// ------------------------------------------------------------ Adam

__device__ __forceinline__ void adam_one(float &p, float &m, float &v, float g,
                                         float lr, float bc1, float bc2,
                                         bool clamp_ls) {
  const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;  // folded in f32
  m = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(omb1, g));
  v = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(omb2, g), g));
  const float step = __fdiv_rn(__fmul_rn(lr, __fdiv_rn(m, bc1)),
                               __fadd_rn(__fsqrt_rn(__fdiv_rn(v, bc2)), eps));
  float y = __fsub_rn(p, step);
  if (clamp_ls) y = fminf(fmaxf(y, -1.6f), 1.0f);
  p = y;
}

__global__ void adam_kernel(AdamArgs a) {
  pdl_wait();
  pdl_trigger();
  const DevState *st = a.st;
  const float lr = st->step_lr;
  const int64_t n4 = a.n / 4;
  float4 *p4 = reinterpret_cast<float4 *>(a.p);
  float4 *m4 = reinterpret_cast<float4 *>(a.m);
  float4 *v4 = reinterpret_cast<float4 *>(a.v);
  const float4 *g4 = reinterpret_cast<const float4 *>(a.g);
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = q * 4;  // segment boundaries are multiples of 32
    const int j = i < a.actor_end ? 0 : (i < a.critic_end ? 1 : 2);
    const float cs = j < 2 ? st->clip_scale[j] : 1.0f;
    float4 p = p4[q], m = m4[q], v = v4[q], g = g4[q];
    if (cs != 1.0f) {
      g.x = __fmul_rn(g.x, cs);
      g.y = __fmul_rn(g.y, cs);
      g.z = __fmul_rn(g.z, cs);
      g.w = __fmul_rn(g.w, cs);
    }
    const float b1c = st->bc1[j], b2c = st->bc2[j];
    const bool cl = j == 2;
    adam_one(p.x, m.x, v.x, g.x, lr, b1c, b2c, cl);
    adam_one(p.y, m.y, v.y, g.y, lr, b1c, b2c, cl);
    adam_one(p.z, m.z, v.z, g.z, lr, b1c, b2c, cl);
    adam_one(p.w, m.w, v.w, g.w, lr, b1c, b2c, cl);
    p4[q] = p;
    if (a.p_round) {
      if (a.p_mode == 2) {
        __nv_bfloat162 *o = reinterpret_cast<__nv_bfloat162 *>(a.p_round) + 2 * q;
        o[0] = __floats2bfloat162_rn(p.x, p.y);
        o[1] = __floats2bfloat162_rn(p.z, p.w);
      } else {
        reinterpret_cast<float4 *>(a.p_round)[q] =
            make_float4(rna_tf32(p.x), rna_tf32(p.y), rna_tf32(p.z), rna_tf32(p.w));
      }
    }
    m4[q] = m;
    v4[q] = v;
  }
}

// ------------------------------------------------ reduce + pre-step + Adam

// The stepping half of a minibatch (ppo.rs:462-489) in one cooperative
// launch, every block resident at once:
//  A. one rank: the segment reduce (the work of reduce_segments_kernel's
//     blocks, taken in turn by this grid's blocks), with each block's
//     squared norms of what it wrote, per net; several ranks (from_grads,
//     no segments): the squared norms of the allreduced gradient;
//  B. a grid barrier, then every block folds the block norms in block
//     order (the same bits in every block) and computes the pre-step's
//     scalars from the state it read before the barrier -- block 0 alone
//     writes them back (statistics, adaptive LR, clip scales, Adam steps);
//  C. Adam over the parameter buffer with those scalars.
// The barrier is a counter that only grows: this launch waits for it to
// reach `target` (the host adds the grid size per launch); its wait is
// bounded (error code 8 in *err, then the block goes on).
struct PreScalars {
  float lr, clip[2], bc1[3], bc2[3];
  int32_t t[3];
};

__device__ PreScalars prestep_scalars(const PrestepArgs &a, float lr, const int32_t *t_old,
                                      float kl, double na, double nc) {
  PreScalars o;
  if (a.adaptive_lr) {
    if (kl > a.desired_kl * 2.0f)
      lr = fmaxf(__fdiv_rn(lr, 1.5f), a.lr_min);
    else if (kl > 0.0f && kl < a.desired_kl / 2.0f)
      lr = fminf(__fmul_rn(lr, 1.5f), a.lr_max);
  }
  o.lr = lr;
  const float norms[2] = {__fsqrt_rn((float)na), __fsqrt_rn((float)nc)};
  for (int j = 0; j < 2; ++j)
    o.clip[j] = (norms[j] > a.max_grad_norm && norms[j] > 0.0f)
                    ? __fdiv_rn(a.max_grad_norm, norms[j]) : 1.0f;
  for (int j = 0; j < 3; ++j) {
    o.t[j] = t_old[j] + 1;
    o.bc1[j] = __fsub_rn(1.0f, powi_f(0.9f, o.t[j]));
    o.bc2[j] = __fsub_rn(1.0f, powi_f(0.999f, o.t[j]));
  }
  return o;
}

__global__ void __launch_bounds__(kRsThreads, 2)
reduce_step_kernel(ReduceSegs segs, PrestepArgs pa, AdamArgs aa, double *partials,
                   unsigned int *bar, unsigned int target, int *err, int items, int from_grads) {
  pdl_wait();
  pdl_trigger();
  __shared__ double sh[32];
  __shared__ float4 part[kRsThreads];
  DevState *st = pa.st;
  // the pre-step's inputs, read before the barrier: after it block 0
  // overwrites the state and every block's Adam writes log_std
  const float lr_old = st->lr;
  const int32_t t_old[3] = {st->t[0], st->t[1], st->t[2]};
  float ent = 0.0f;  // entropy of the pre-step log_std (ppo.rs:308-311, 473)
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const float c0 = __fadd_rn(0.5f, kLogSqrt2Pi);
    for (int k = 0; k < pa.A; ++k) ent = __fadd_rn(ent, __fadd_rn(pa.log_std[k], c0));
  }
  // ---- A: the reduce
  double sq[2] = {0.0, 0.0};
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    int si = 0;
    while (si + 1 < segs.n && item >= segs.first_block[si + 1]) ++si;
    const int b = item - segs.first_block[si];
    const int64_t count4 = segs.seg[si].count / 4;
    const int splits = segs.seg[si].splits;
    const int64_t stride4 = segs.seg[si].stride / 4;
    const int G = segs.groups[si];
    const int cols4 = kRsThreads / G;
    const int c = threadIdx.x & (cols4 - 1), grp = threadIdx.x / cols4;
    const int64_t i4 = (int64_t)b * cols4 + c;
    const bool live = i4 < count4;
    const float4 *src = reinterpret_cast<const float4 *>(segs.seg[si].src) + i4;
    float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (live) {
      for (int z0 = grp; z0 < splits; z0 += 8 * G) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int z = z0 + u * G;
          x[u] = z < splits ? __ldcs(src + (int64_t)z * stride4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          t.x += x[u].x;
          t.y += x[u].y;
          t.z += x[u].z;
          t.w += x[u].w;
        }
      }
    }
    __syncthreads();  // part[] of the previous item is no longer read
    part[threadIdx.x] = t;
    __syncthreads();
    for (int h = G >> 1; h >= 1; h >>= 1) {
      if (grp < h) {
        const float4 x = part[threadIdx.x + h * cols4];
        t.x += x.x;
        t.y += x.y;
        t.z += x.z;
        t.w += x.w;
        part[threadIdx.x] = t;
      }
      __syncthreads();
    }
    if (grp == 0 && live) {
      reinterpret_cast<float4 *>(segs.seg[si].dst)[i4] = t;
      const int net = segs.net[si];
      if (net >= 0)
        sq[net] += (double)t.x * t.x + (double)t.y * t.y + (double)t.z * t.z + (double)t.w * t.w;
    }
  }
  if (from_grads) {
    // several ranks: the norms of the allreduced gradient itself (the
    // per-net ranges start and end on 16-byte boundaries)
    const float4 *g4 = reinterpret_cast<const float4 *>(pa.grads);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t i = pa.actor_begin / 4 + t0; i < pa.actor_end / 4; i += stride) {
      const float4 x = __ldcg(g4 + i);
      sq[0] += (double)x.x * x.x + (double)x.y * x.y + (double)x.z * x.z + (double)x.w * x.w;
    }
    for (int64_t i = pa.critic_begin / 4 + t0; i < pa.critic_end / 4; i += stride) {
      const float4 x = __ldcg(g4 + i);
      sq[1] += (double)x.x * x.x + (double)x.y * x.y + (double)x.z * x.z + (double)x.w * x.w;
    }
  }
  const double ba = block_sum(sq[0], sh);
  const double bc = block_sum(sq[1], sh);
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = ba;
    partials[2 * blockIdx.x + 1] = bc;
  }
  // ---- B: grid barrier, norms, pre-step scalars
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicAdd(bar, 1u);
    unsigned int seen = 0;
    for (uint32_t i = 0;; ++i) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(bar) : "memory");
      if ((int)(seen - target) >= 0) break;
      if (i > (1u << 22)) {  // about a second of 256 ns naps: give up
        atomicExch(err, 8);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncthreads();
  double na = 0.0, nc = 0.0;
  for (int bb = threadIdx.x; bb < (int)gridDim.x; bb += blockDim.x) {
    na += __ldcg(&partials[2 * bb]);
    nc += __ldcg(&partials[2 * bb + 1]);
  }
  na = block_sum(na, sh);
  nc = block_sum(nc, sh);
  __shared__ PreScalars ps;
  if (threadIdx.x == 0) {
    const float kl = __ldcg(pa.sums3 + 2);
    ps = prestep_scalars(pa, lr_old, t_old, kl, na, nc);
    if (blockIdx.x == 0) {
      // what prestep_finish writes: statistics, lr, clip scales, steps
      st->sumsq[0] = (float)na;
      st->sumsq[1] = (float)nc;
      if (pa.count_stats) {
        st->ep_acc[0] += kl;
        st->ep_acc[1] += __ldcg(pa.sums3 + 0);
        st->ep_acc[2] += __ldcg(pa.sums3 + 1);
        st->ep_acc[3] += ent;
      }
      st->lr = ps.lr;
      st->step_lr = ps.lr;
      for (int j = 0; j < 2; ++j) st->clip_scale[j] = ps.clip[j];
      for (int j = 0; j < 3; ++j) {
        st->t[j] = ps.t[j];
        st->bc1[j] = ps.bc1[j];
        st->bc2[j] = ps.bc2[j];
      }
      if (pa.count_stats && pa.last_of_epoch) {
        const float inv = __fdiv_rn(1.0f, (float)pa.minibatches);
        for (int j = 0; j < 4; ++j) st->stats[j] = st->ep_acc[j] * inv;
        st->stats[4] = ps.lr;
        for (int j = 0; j < 4; ++j) st->ep_acc[j] = 0.0f;
      }
    }
  }
  __syncthreads();
  // ---- C: Adam (adam_kernel's arithmetic, these scalars)
  const int64_t n4 = aa.n / 4;
  float4 *p4 = reinterpret_cast<float4 *>(aa.p);
  float4 *m4 = reinterpret_cast<float4 *>(aa.m);
  float4 *v4 = reinterpret_cast<float4 *>(aa.v);
  const float4 *g4 = reinterpret_cast<const float4 *>(aa.g);
  for (int64_t qd = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; qd < n4;
       qd += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = qd * 4;
    const int j = i < aa.actor_end ? 0 : (i < aa.critic_end ? 1 : 2);
    const float cs = j < 2 ? ps.clip[j] : 1.0f;
    float4 pp = p4[qd], mm = m4[qd], vv = v4[qd], gg = __ldcg(g4 + qd);
    if (cs != 1.0f) {
      gg.x = __fmul_rn(gg.x, cs);
      gg.y = __fmul_rn(gg.y, cs);
      gg.z = __fmul_rn(gg.z, cs);
      gg.w = __fmul_rn(gg.w, cs);
    }
    const bool cl = j == 2;
    adam_one(pp.x, mm.x, vv.x, gg.x, ps.lr, ps.bc1[j], ps.bc2[j], cl);
    adam_one(pp.y, mm.y, vv.y, gg.y, ps.lr, ps.bc1[j], ps.bc2[j], cl);
    adam_one(pp.z, mm.z, vv.z, gg.z, ps.lr, ps.bc1[j], ps.bc2[j], cl);
    adam_one(pp.w, mm.w, vv.w, gg.w, ps.lr, ps.bc1[j], ps.bc2[j], cl);
    p4[qd] = pp;
    if (aa.p_round) {
      if (aa.p_mode == 2) {
        __nv_bfloat162 *o = reinterpret_cast<__nv_bfloat162 *>(aa.p_round) + 2 * qd;
        o[0] = __floats2bfloat162_rn(pp.x, pp.y);
        o[1] = __floats2bfloat162_rn(pp.z, pp.w);
      } else {
        reinterpret_cast<float4 *>(aa.p_round)[qd] =
            make_float4(rna_tf32(pp.x), rna_tf32(pp.y), rna_tf32(pp.z), rna_tf32(pp.w));
      }
    }
    m4[qd] = mm;
    v4[qd] = vv;
  }
}

// ------------------------------------------------------------ misc

__global__ void unpad_rows_kernel(const float *src, int64_t rows, int pitch,
                                  int cols, float *dst) {
  const int64_t total = rows * cols;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / cols;
    const int c = (int)(e - r * cols);
    dst[e] = src[r * pitch + c];
  }
}

// ------------------------------------------------------ Welford update

// Normalizer::update (ppo.rs:161-168) for n rows in order: one thread per
// feature runs the sequential recurrence, so the result is bit-identical
// to folding the rows one by one.
__global__ void record_obs_kernel(const float *x, int64_t n, int dim,
                                  float *mean, float *m2, float count0) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim) return;
  float c = count0, mu = mean[i], s = m2[i];
  for (int64_t r = 0; r < n; ++r) {
    c = __fadd_rn(c, 1.0f);
    const float xi = x[r * dim + i];
    const float d = __fsub_rn(xi, mu);
    mu = __fadd_rn(mu, __fdiv_rn(d, c));
    s = __fadd_rn(s, __fmul_rn(d, __fsub_rn(xi, mu)));
  }
  mean[i] = mu;
  m2[i] = s;
}

// ------------------------------------------------------ rollout sampling

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11): 10 rounds of the 4x32 S-box with the published
// multipliers and Weyl key increments.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// uniform in (0, 1): the top 24 bits, offset by half a step
__device__ __forceinline__ float u01(uint32_t x) {
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// One thread per (row, group of 4 action dims): Philox counter
// (group, row_lo, counter_lo, counter_hi ^ row_hi) under key (seed_lo,
// seed_hi) gives 4 uniforms -> 2 Box-Muller pairs -> 4 standard normals.
// action = mean + exp(log_std) * eps; logp (ppo.rs:297-305) is a warp-free
// second pass per row.
__global__ void policy_sample_kernel(const float *mean, int pitch,
                                     const float *log_std, int A, int64_t n,
                                     uint64_t seed, uint64_t counter,
                                     float *action, float *mean_out, int64_t row0) {
  const int groups = (A + 3) / 4;
  const int64_t total = n * groups;
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / groups;
    const int gidx = (int)(e - row * groups);
    const int64_t grow = row + row0;  // global row number: the draw is per row
    const uint4 ctr = make_uint4((uint32_t)gidx, (uint32_t)grow, (uint32_t)counter,
                                 (uint32_t)(counter >> 32) ^ (uint32_t)(grow >> 32));
    const uint4 r = philox4x32_10(ctr, key);
    const float ra = sqrtf(-2.0f * logf(u01(r.x)));
    const float rb = sqrtf(-2.0f * logf(u01(r.z)));
    const float ta = 6.28318548202514648f * u01(r.y);
    const float tb = 6.28318548202514648f * u01(r.w);
    const float z[4] = {ra * cosf(ta), ra * sinf(ta), rb * cosf(tb), rb * sinf(tb)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = gidx * 4 + j;
      if (k < A) {
        const float mu = mean[row * pitch + k];
        action[row * A + k] = mu + expf(log_std[k]) * z[j];
        if (mean_out) mean_out[row * A + k] = mu;
      }
    }
  }
}

__global__ void logp_rows_kernel(const float *action, const float *mean, int pitch,
                                 const float *log_std, int A, int64_t n, float *logp) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < n;
       row += (int64_t)gridDim.x * blockDim.x) {
    float lp = 0.0f;
    for (int k = 0; k < A; ++k) {
      const float d = (action[row * A + k] - mean[row * pitch + k]) / expf(log_std[k]);
      lp += -0.5f * d * d - log_std[k] - kLogSqrt2Pi;
    }
    logp[row] = lp;
  }
}

int grid_for(int64_t work, int threads, int cap = 148 * 16) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

}  // namespace

// ================================================================ wrappers

int gae_blocks(int64_t n_envs) { return (int)((n_envs + kGaeEnvs - 1) / kGaeEnvs); }

void launch_gae(const GaeArgs &a, double *partials, int nblk, cudaStream_t s) {
  if (a.T <= kGaeMaxStagedT) {
    const size_t smem = (size_t)kGaeEnvs * a.T * (4 * sizeof(float) + 1);
    gae_kernel<true><<<nblk, kGaeThreads, smem, s>>>(a, partials);
  } else {
    gae_kernel<false><<<nblk, kGaeThreads, 0, s>>>(a, partials);
  }
}

int adv_blocks(int64_t n) { return grid_for(n, kAdvThreads, 296); }

void launch_adv_sum(const float *adv, int64_t n, double *partials, int nblk,
                    cudaStream_t s) {
  adv_sum_kernel<<<nblk, kAdvThreads, 0, s>>>(adv, n, partials);
}

void launch_reduce_moment(const double *partials, int nblk, double *moments,
                          int slot, cudaStream_t s) {
  reduce_partials_kernel<<<1, 1024, 0, s>>>(partials, nblk, moments, slot);
}

void launch_adv_sqdev(const float *adv, int64_t n, const double *moments,
                      int64_t n_global, double *partials, int nblk,
                      cudaStream_t s) {
  adv_sqdev_kernel<<<nblk, kAdvThreads, 0, s>>>(adv, n, moments, n_global,
                                                 partials);
}

void launch_adv_finalize(const double *moments, int64_t n_global, DevState *st,
                         cudaStream_t s) {
  adv_finalize_kernel<<<1, 1, 0, s>>>(moments, n_global, st);
}

void launch_gather(const GatherArgs &a, cudaStream_t s) {
  const int threads = 256;
  launch_pdl(gather_kernel, grid_for(a.n_used * 32, threads), threads, s, a);
}

void launch_norm_prepare(const float *m2, float count, int dim, float *sd,
                         cudaStream_t s) {
  norm_prepare_kernel<<<(dim + 127) / 128, 128, 0, s>>>(m2, count, dim, sd);
}

void launch_normalize_rows(const float *x, int64_t n, int dim, int pitch,
                           const float *mean, const float *sd, float *out,
                           int mode, cudaStream_t s, const int32_t *perm, const float *sign) {
  // pitch is a multiple of 32 and at most 256 (zrl_create's limit)
  const int blocks = grid_for((n + kNormRows - 1) / kNormRows, 1, 148 * 32);
  normalize_rows_kernel<<<blocks, pitch, 0, s>>>(x, n, dim, pitch, mean, sd, out, mode, perm,
                                                 sign);
}

void launch_round_copy(const float *src, float *dst, int64_t n, int mode, cudaStream_t s) {
  round_copy_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, dst, n, mode);
}

// the quad form needs 16-byte aligned 32-float mean rows
static bool loss_by_quads(const LossArgs &a) {
  return a.A <= 32 && a.Ap == 32 && ((uintptr_t)a.mean & 15) == 0 &&
         ((uintptr_t)a.d_actor & 15) == 0;
}

int loss_blocks(const LossArgs &a) {
  if (loss_by_quads(a))  // a sample per quad, at most 4 blocks per SM
    return grid_for(a.mb * 4, kLossQuadThreads, 4 * 148);
  return grid_for(a.mb * 32, kLossThreads, 4 * 148);
}

void launch_loss(const LossArgs &a, cudaStream_t s) {
  // the block rows are summed by the segment reduce that follows the
  // backward pass
  const int blocks = loss_blocks(a);
  if (loss_by_quads(a))
    launch_pdl(loss_quad_kernel, blocks, kLossQuadThreads, s, a);
  else  // four blocks per SM, a warp per sample with the next sample's loads in flight
    launch_pdl(loss_kernel, blocks, kLossThreads, s, a);
}

void launch_colsum(const float *x, int64_t rows, int cols, int ld,
                   float *partials, int splits, cudaStream_t s) {
  dim3 grid((cols + 127) / 128, splits);
  colsum_kernel<<<grid, 128, 0, s>>>(x, rows, cols, ld, partials, splits);
}

// Segments with the most splits first (their blocks run longest, so they
// start in the first wave), then each segment's first block, split groups
// and net (with `fuse`: 0 actor, 1 critic, -1 neither).
static bool plan_segments(ReduceSegs &segs, const PrestepArgs *fuse, int *blocks_out) {
  for (int i = 1; i < segs.n; ++i)
    for (int j = i; j > 0 && segs.seg[j].splits > segs.seg[j - 1].splits; --j) {
      const ReduceSeg t = segs.seg[j];
      segs.seg[j] = segs.seg[j - 1];
      segs.seg[j - 1] = t;
    }
  int64_t blocks = 0;
  for (int i = 0; i < segs.n; ++i) {
    segs.first_block[i] = (int)blocks;
    segs.groups[i] = rs_groups(segs.seg[i].splits);
    blocks += rs_blocks(segs.seg[i].count, segs.seg[i].splits);
    segs.net[i] = -1;
    if (fuse) {
      const int64_t off = segs.seg[i].dst - fuse->grads;
      if (off >= fuse->actor_begin && off < fuse->actor_end) segs.net[i] = 0;
      else if (off >= fuse->critic_begin && off < fuse->critic_end) segs.net[i] = 1;
    }
  }
  segs.first_block[segs.n] = (int)blocks;
  if (blocks > INT32_MAX / 2) return false;
  *blocks_out = (int)blocks;
  return true;
}

int launch_reduce_segments(const ReduceSegs &segs_in, cudaStream_t s, const PrestepArgs *fuse,
                           ReduceScratch *rs) {
  // segments with the most splits first: their blocks run longest, so they
  // start in the first wave
  ReduceSegs segs = segs_in;
  int blocks = 0;
  if (!plan_segments(segs, fuse, &blocks)) return 0;
  if (blocks == 0) return 0;
  if (fuse && blocks > rs->max_blocks) fuse = nullptr;  // partials too small: not fused
  PrestepArgs pa{};
  if (fuse) pa = *fuse;
  launch_pdl(reduce_segments_kernel, (unsigned)blocks, kRsThreads, s, segs, pa,
             fuse ? rs->dpart : (double *)nullptr, fuse ? rs->ticket + 1 : (unsigned int *)nullptr,
             fuse ? 1 : 0);
  return fuse ? 1 : 0;
}

bool launch_reduce_step(const ReduceSegs &segs_in, const PrestepArgs &pa, const AdamArgs &aa,
                        ReduceScratch &rs, int *err, cudaStream_t s, bool from_grads) {
  if (rs.coop_blocks < 0) return false;
  if (rs.coop_blocks == 0) {
    // every block resident at once: the occupancy of this kernel on every SM
    int dev = 0, sms = 0, per_sm = 0, coop = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reduce_step_kernel, kRsThreads,
                                                      0) != cudaSuccess ||
        !coop || per_sm < 1) {
      cudaGetLastError();
      rs.coop_blocks = -1;
      return false;
    }
    rs.coop_blocks = sms * per_sm;
    if (rs.coop_blocks > rs.max_blocks) rs.coop_blocks = rs.max_blocks;
  }
  ReduceSegs segs = segs_in;
  int items = 0;
  if (!plan_segments(segs, from_grads ? nullptr : &pa, &items)) return false;
  if (items == 0 && !from_grads) return false;
  if (from_grads && ((pa.actor_begin | pa.actor_end | pa.critic_begin | pa.critic_end) & 3))
    return false;
  unsigned grid = (unsigned)rs.coop_blocks;
  if (aa.n % 4 != 0) return false;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRsThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const unsigned int target = rs.bar_count + grid;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, reduce_step_kernel, segs, pa, aa, rs.dpart,
                                           rs.ticket + 2, target, err, items, from_grads ? 1 : 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    rs.coop_blocks = -1;  // refused: the separate kernels from now on
    return false;
  }
  rs.bar_count = target;
  return true;
}

void launch_prestep(const PrestepArgs &a, ReduceScratch &rs, cudaStream_t s) {
  const int64_t work = (a.actor_end - a.actor_begin);
  int blocks = grid_for(work, kPrestepThreads, 148);
  if (blocks > rs.max_blocks) blocks = rs.max_blocks;
  launch_pdl(prestep_kernel, blocks, kPrestepThreads, s, a, rs.dpart, rs.ticket + 1);
}

void launch_adam(const AdamArgs &a, cudaStream_t s) {
  launch_pdl(adam_kernel, grid_for(a.n / 4, 256, 148 * 8), 256, s, a);
}

void launch_unpad_rows(const float *src, int64_t rows, int pitch, int cols,
                       float *dst, cudaStream_t s) {
  unpad_rows_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(src, rows, pitch,
                                                               cols, dst);
}

void launch_record_obs(const float *x, int64_t n, int dim, float *mean, float *m2,
                       float count0, cudaStream_t s) {
  record_obs_kernel<<<(dim + 127) / 128, 128, 0, s>>>(x, n, dim, mean, m2, count0);
}

void launch_policy_sample(const float *mean, int pitch, const float *log_std, int A,
                          int64_t n, uint64_t seed, uint64_t counter, float *action,
                          float *logp, float *mean_out, cudaStream_t s, int64_t row0) {
  const int64_t work = n * ((A + 3) / 4);
  policy_sample_kernel<<<grid_for(work, 256), 256, 0, s>>>(mean, pitch, log_std, A, n,
                                                            seed, counter, action,
                                                            mean_out, row0);
  if (logp)
    logp_rows_kernel<<<grid_for(n, 256), 256, 0, s>>>(action, mean, pitch, log_std, A,
                                                       n, logp);
}

void launch_logp_rows(const float *action, const float *mean, int pitch, const float *log_std,
                      int A, int64_t n, float *logp, cudaStream_t s) {
  logp_rows_kernel<<<grid_for(n, 256), 256, 0, s>>>(action, mean, pitch, log_std, A, n, logp);
}

}  // namespace zrl
