// welford.cu -- the observation normalizers' statistics on the device
// (zealot-rl/src/ppo.rs:104-195).
//
// Normalizer::update and PendingNorm::push fold rows one at a time
// (Welford); Normalizer::commit merges a pending state into the live one
// with Chan et al.'s pairwise formula.  Here:
//  * the sequential fold (record_obs_kernel in kernels.cu, one thread per
//    feature over every row in order) is bit-identical to the reference;
//  * the parallel fold splits the rows into chunks of kWelfordChunkRows (256),
//    folds each chunk from an empty state (a fresh PendingNorm::push per chunk: one
//    thread per chunk and feature, reading whole rows, so a warp's loads are
//    coalesced), then merges the chunk states into the destination in chunk
//    order with the commit formula -- the same statistics up to rounding
//    (relative 1e-5), at N / 256 times the parallelism;
//  * commit is the reference's merge, operation for operation.
#include <cuda_runtime.h>
#include <stdint.h>

#include "zrl_internal.h"

namespace zrl {
namespace {

constexpr int kThreads = 256;

// Chan et al. merge of (n2, pm, ps) into (n1, mu, s), in the f32 operation
// order of Normalizer::commit (ppo.rs:185-191):
//   mean += d * n2 / tot;  m2 += pm2 + d * d * n1 * n2 / tot
__device__ __forceinline__ void chan_merge(float n1, float n2, float &mu, float &s, float pm,
                                           float ps) {
  const float tot = __fadd_rn(n1, n2);
  const float d = __fsub_rn(pm, mu);
  mu = __fadd_rn(mu, __fdiv_rn(__fmul_rn(d, n2), tot));
  s = __fadd_rn(s, __fadd_rn(ps, __fdiv_rn(__fmul_rn(__fmul_rn(__fmul_rn(d, d), n1), n2), tot)));
}

// One thread per (chunk, feature): Welford over the chunk's rows from an
// empty state (ppo.rs:126-136), the chunk's mean and m2 into the partials.
__global__ void welford_chunks_kernel(const float *x, int64_t n, int dim, int chunk_rows,
                                      float *pmean, float *pm2) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nch = (n + chunk_rows - 1) / chunk_rows;
  if (t >= nch * dim) return;
  const int64_t ch = t / dim;
  const int i = (int)(t - ch * dim);
  const int64_t r0 = ch * chunk_rows;
  const int64_t r1 = n < r0 + chunk_rows ? n : r0 + chunk_rows;
  float c = 0.0f, mu = 0.0f, s = 0.0f;
  for (int64_t r = r0; r < r1; ++r) {
    c = __fadd_rn(c, 1.0f);
    const float xi = x[r * dim + i];
    const float d = __fsub_rn(xi, mu);
    mu = __fadd_rn(mu, __fdiv_rn(d, c));
    s = __fadd_rn(s, __fmul_rn(d, __fsub_rn(xi, mu)));
  }
  pmean[ch * dim + i] = mu;
  pm2[ch * dim + i] = s;
}

// One thread per feature: the chunk states merged into (count0, mean, m2)
// in chunk order; an empty destination (count0 = 0) takes the first chunk
// as it is.
__global__ void welford_merge_kernel(const float *pmean, const float *pm2, int64_t n,
                                     int chunk_rows, int dim, float count0, float *mean,
                                     float *m2) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim) return;
  const int64_t nch = (n + chunk_rows - 1) / chunk_rows;
  float c = count0, mu = mean[i], s = m2[i];
  for (int64_t ch = 0; ch < nch; ++ch) {
    const int64_t left = n - ch * chunk_rows;
    const float n2 = (float)(left < chunk_rows ? left : (int64_t)chunk_rows);
    const float pm = pmean[ch * dim + i], ps = pm2[ch * dim + i];
    if (c == 0.0f) {
      mu = pm;
      s = ps;
      c = n2;
      continue;
    }
    chan_merge(c, n2, mu, s, pm, ps);
    c = __fadd_rn(c, n2);
  }
  mean[i] = mu;
  m2[i] = s;
}

// Normalizer::commit (ppo.rs:179-195) per feature, then the pending state
// reset to empty.
__global__ void norm_commit_kernel(float *mean, float *m2, float count, float *p_mean,
                                   float *p_m2, float p_count, int dim) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim) return;
  float mu = mean[i], s = m2[i];
  chan_merge(count, p_count, mu, s, p_mean[i], p_m2[i]);
  mean[i] = mu;
  m2[i] = s;
  p_mean[i] = 0.0f;
  p_m2[i] = 0.0f;
}

}  // namespace

int64_t welford_partial_floats(int64_t n, int dim) {
  return 2 * ((n + kWelfordChunkRows - 1) / kWelfordChunkRows) * (int64_t)dim;
}

void launch_welford_parallel(const float *x, int64_t n, int dim, float count0, float *mean,
                             float *m2, float *scratch, cudaStream_t s) {
  if (n <= 0) return;
  const int64_t nch = (n + kWelfordChunkRows - 1) / kWelfordChunkRows;
  float *pmean = scratch, *pm2 = scratch + nch * dim;
  const int64_t work = nch * dim;
  welford_chunks_kernel<<<(unsigned)((work + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      x, n, dim, kWelfordChunkRows, pmean, pm2);
  welford_merge_kernel<<<(dim + 127) / 128, 128, 0, s>>>(pmean, pm2, n, kWelfordChunkRows, dim,
                                                          count0, mean, m2);
}

void launch_norm_commit(float *mean, float *m2, float count, float *p_mean, float *p_m2,
                        float p_count, int dim, cudaStream_t s) {
  norm_commit_kernel<<<(dim + 127) / 128, 128, 0, s>>>(mean, m2, count, p_mean, p_m2, p_count,
                                                       dim);
}

}  // namespace zrl
