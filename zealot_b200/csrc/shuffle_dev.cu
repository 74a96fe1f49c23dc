// shuffle_dev.cu -- the epoch permutation of ppo.rs:357-363 computed on the
// device, equal index for index to the sequential Fisher-Yates loop
// (host_rng.cpp zrl_shuffle).
//
// Step i (i = n-1 down to 1) swaps positions i and j_i = min(trunc(u_d *
// (i + 1)), i), where u_d is the d-th Lcg draw and d = n - i.  The draws
// depend on the seed alone, so every j_i is computed at once: the Lcg step
// is the affine map s -> a s + c (mod 2^64), and the state after d draws is
// the d-th power of that map applied to Lcg::new(seed), built by squaring.
//
// Position i is final after step i and receives what position j_i held
// just before step i.  Just before step t, a position p holds what the most
// recent earlier step that targeted it wrote there -- that is the step with
// the smallest k > t and j_k = p, which wrote what position k held just
// before step k -- or p itself when no such step exists.  Every output
// element walks that chain (each hop strictly increases k, so it ends) over
// per-position lists of the steps that targeted the position.
#include <cstdint>

#include "zrl_internal.h"

namespace zrl {
namespace {

constexpr uint64_t kLcgA = 6364136223846793005ull;  // rng.rs:21
constexpr uint64_t kLcgC = 1442695040888963407ull;

// The Lcg state after d steps from s0.
__device__ __forceinline__ uint64_t lcg_jump(uint64_t s0, uint64_t d) {
  uint64_t a = 1, c = 0;              // the composed map so far (identity)
  uint64_t pa = kLcgA, pc = kLcgC;    // the map of 2^b steps
  while (d) {
    if (d & 1) {
      c = pa * c + pc;
      a = pa * a;
    }
    pc = pa * pc + pc;
    pa = pa * pa;
    d >>= 1;
  }
  return a * s0 + c;
}

// ActorCritic::sample's draws (ppo.rs:313-323; the GPU trainer's host loop,
// biped_train_gpu.rs:913-919) from one sequential Lcg stream over (row, k):
// the g-th gauss (g = row * A + k) is Box-Muller (rng.rs:28-32) of the
// stream's draws 2g and 2g + 1 after s0, reached by jump-ahead -- the
// uniforms are the reference's bit for bit.
__global__ void lcg_sample_kernel(const float *mean, int pitch, const float *log_std, int A,
                                  int64_t n, uint64_t s0, int64_t row0, float *action,
                                  float *mean_out) {
  const int64_t total = n * A;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / A;
    const int k = (int)(e - row * A);
    const uint64_t g = (uint64_t)(row0 + row) * (uint64_t)A + (uint64_t)k;
    uint64_t st = lcg_jump(s0, 2 * g);
    st = st * kLcgA + kLcgC;
    const float u1 = (float)(st >> 40) / 16777216.0f;
    st = st * kLcgA + kLcgC;
    const float u2 = (float)(st >> 40) / 16777216.0f;
    const float z = sqrtf(-2.0f * logf(fmaxf(u1, 1e-7f))) * cosf(6.28318548202514648f * u2);
    const float mu = mean[row * pitch + k];
    action[row * A + k] = mu + expf(log_std[k]) * z;
    if (mean_out) mean_out[row * A + k] = mu;
  }
}

// j_i for every step, and the per-position lists of the steps that
// targeted it (head[p] -> next[k] -> ... -> -1, in any order).
__global__ void fy_link_kernel(uint64_t s0, int32_t n, int32_t *jt, int32_t *head,
                               int32_t *next) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x + 1; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t s = lcg_jump(s0, (uint64_t)(n - i));
    // Lcg::unit (rng.rs:19-26): the top 24 bits over 2^24 (exact)
    const float u = __fmul_rn((float)(s >> 40), 5.9604644775390625e-08f);
    const float prod = __fmul_rn(u, (float)(i + 1));
    int64_t j = (int64_t)prod;
    if (j > i) j = i;
    jt[i] = (int32_t)j;
    next[i] = atomicExch(&head[j], (int32_t)i);
  }
}

__global__ void fy_walk_kernel(int32_t n, const int32_t *jt, const int32_t *head,
                               const int32_t *next, int32_t *order) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int32_t p = i == 0 ? 0 : jt[i];
    int32_t t = (int32_t)i;
    for (;;) {
      int32_t best = INT32_MAX;
      for (int32_t e = head[p]; e >= 0; e = next[e])
        if (e > t && e < best) best = e;
      if (best == INT32_MAX) break;
      p = best;
      t = best;
    }
    order[i] = p;
  }
}

}  // namespace

void launch_shuffle_device(uint64_t seed, int32_t n, int32_t *order, int32_t *scratch,
                           cudaStream_t s) {
  if (n <= 0) return;
  int32_t *jt = scratch, *head = scratch + n, *next = scratch + 2 * (int64_t)n;
  cudaMemsetAsync(head, 0xFF, sizeof(int32_t) * (size_t)n, s);  // -1: empty lists
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>(((int64_t)n + threads - 1) / threads, 148 * 16);
  const uint64_t s0 = seed | 1ull;  // Lcg::new (rng.rs:14-16)
  fy_link_kernel<<<blocks, threads, 0, s>>>(s0, n, jt, head, next);
  fy_walk_kernel<<<blocks, threads, 0, s>>>(n, jt, head, next, order);
}

}  // namespace zrl

// ------------------------------------------------- one rank's share, on device

namespace zrl {
namespace {

constexpr int kScanThreads = 1024;

// flag of permutation position p: inside the used slices (p < used) and
// holding one of this rank's rows
__device__ __forceinline__ int rank_flag(const int32_t *perm, int64_t p, int64_t used,
                                         int64_t row_offset, int64_t n_local) {
  if (p >= used) return 0;
  const int64_t r = (int64_t)perm[p] - row_offset;
  return r >= 0 && r < n_local;
}

// exclusive prefix of v over the block (kScanThreads threads, every thread
// calls it), and the block's total
__device__ __forceinline__ int block_excl_scan(int v, int *total) {
  __shared__ int warp_tot[kScanThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int before = wid > 0 ? warp_tot[wid - 1] : 0;
  *total = warp_tot[kScanThreads / 32 - 1];
  __syncthreads();  // warp_tot is reused by the next call
  return before + x - v;
}

// pass 1: the number of flagged positions of each block
__global__ void rank_count_kernel(const int32_t *perm, int64_t used, int64_t row_offset,
                                  int64_t n_local, int32_t *block_sums) {
  const int64_t p = (int64_t)blockIdx.x * kScanThreads + threadIdx.x;
  int total;
  block_excl_scan(rank_flag(perm, p, used, row_offset, n_local), &total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// pass 2 (one block): exclusive prefix of the block sums, in place
__global__ void rank_offsets_kernel(int32_t *block_sums, int nblk) {
  int carry = 0;
  for (int b0 = 0; b0 < nblk; b0 += kScanThreads) {
    const int b = b0 + threadIdx.x;
    const int v = b < nblk ? block_sums[b] : 0;
    int total;
    const int e = block_excl_scan(v, &total);
    if (b < nblk) block_sums[b] = carry + e;
    carry += total;
  }
}

// pass 3: scatter this rank's rows in permutation order; the prefix at
// every slice boundary gives the per-slice counts: counts[m] receives
// -prefix(start of slice m), counts[mbs] the prefix at the end
__global__ void rank_scatter_kernel(const int32_t *perm, int64_t used, int64_t row_offset,
                                    int64_t n_local, const int32_t *block_offs, int64_t mb,
                                    int mbs, int32_t *order, int64_t *counts) {
  const int64_t p = (int64_t)blockIdx.x * kScanThreads + threadIdx.x;
  const int f = rank_flag(perm, p, used, row_offset, n_local);
  int total;
  const int64_t pos = block_offs[blockIdx.x] + block_excl_scan(f, &total);
  if (f) order[pos] = (int32_t)((int64_t)perm[p] - row_offset);
  if (p < used && p % mb == 0) counts[p / mb] = -pos;
  if (p == used - 1) counts[mbs] = pos + f;
}

// counts[m] = prefix(start of m+1) - prefix(start of m)
__global__ void rank_counts_kernel(int64_t *counts, int mbs) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int64_t end = counts[mbs];
  for (int m = mbs - 1; m >= 0; --m) {
    const int64_t start = -counts[m];
    counts[m] = end - start;
    end = start;
  }
}

}  // namespace

void launch_rank_orders(const int32_t *perm, int64_t n_global, int64_t n_local,
                        int64_t row_offset, int mbs, int32_t *order, int64_t *counts,
                        int32_t *scratch, cudaStream_t s) {
  const int64_t mb = n_global / mbs;
  const int64_t used = mb * mbs;
  const int nblk = (int)((n_global + kScanThreads - 1) / kScanThreads);
  cudaMemsetAsync(counts, 0, sizeof(int64_t) * (size_t)(mbs + 1), s);
  if (used <= 0 || nblk <= 0) return;
  rank_count_kernel<<<nblk, kScanThreads, 0, s>>>(perm, used, row_offset, n_local, scratch);
  rank_offsets_kernel<<<1, kScanThreads, 0, s>>>(scratch, nblk);
  rank_scatter_kernel<<<nblk, kScanThreads, 0, s>>>(perm, used, row_offset, n_local, scratch,
                                                    mb, mbs, order, counts);
  rank_counts_kernel<<<1, 32, 0, s>>>(counts, mbs);
}

void launch_lcg_sample(const float *mean, int pitch, const float *log_std, int A, int64_t n,
                       uint64_t s0, int64_t row0, float *action, float *mean_out,
                       cudaStream_t s) {
  const int64_t work = n * A;
  const int blocks = (int)std::min<int64_t>((work + 255) / 256, 148 * 16);
  lcg_sample_kernel<<<blocks, 256, 0, s>>>(mean, pitch, log_std, A, n, s0, row0, action,
                                            mean_out);
}

}  // namespace zrl
