// zrl_internal.h -- shared definitions of libzealot_rl.so (not part of the
// ABI).  Device layouts:
//
//  * Parameters live in one padded device buffer: for each net (actor, then
//    critic) and each layer l, W_l [dp_{l+1} x dp_l] row-major followed by
//    b_l [dp_{l+1}], then log_std padded to 32.  dp = dim rounded up to 32,
//    so every tensor starts on a 128-byte boundary (TMA-legal) and every
//    GEMM dimension is a multiple of 32.  Padding entries are zero and stay
//    zero (their gradients are zero).  Gradients, Adam m and v share the
//    layout, so the optimizer is one pass over one flat buffer.
//  * Samples are stored sample-major: row = sample, columns = features, so a
//    minibatch gather is a row gather and every activation is [rows x dp].
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/zealot_rl.h"

namespace zrl {

constexpr int kPad = 32;
inline int64_t pad_to(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

struct NetLayout {
  int L = 0;                  // layers
  int d[ZRL_MAX_LAYERS + 1];  // true dims
  int dp[ZRL_MAX_LAYERS + 1]; // padded dims
  int64_t w_off[ZRL_MAX_LAYERS], b_off[ZRL_MAX_LAYERS];   // device (padded)
  int64_t fw_off[ZRL_MAX_LAYERS], fb_off[ZRL_MAX_LAYERS]; // flat save order
  int64_t dev_begin = 0, dev_end = 0;
  int64_t flat_begin = 0, flat_end = 0;
};

// Per-minibatch scalar state that lives on the device (so a whole update
// can run without host round trips).
struct DevState {
  float lr;
  int32_t t[3];          // Adam steps: actor, critic, log_std
  float ep_acc[4];       // epoch accumulators: kl, surrogate, value_loss, entropy
  float stats[5];        // last finished epoch: kl, surr, vloss, entropy, lr
  // written by the pre-step for the Adam pass of the same minibatch
  float step_lr;
  float clip_scale[2];   // actor, critic
  float bc1[3], bc2[3];
  float sumsq[2];        // squared grad norms (actor, critic), diagnostics
  float adv_mean, adv_sd;
  int32_t err;           // device-side error flags
};

// Reduction scratch used by the "last block finishes" kernels: block
// partials, and one arrival counter per kernel kind (reset to 0 by the last
// block, so the scratch is reusable by the next launch on the stream).
struct ReduceScratch {
  float *fpart;          // [max_blocks * fwidth]
  double *dpart;         // [max_blocks * 2]
  unsigned int *ticket;  // [4]: [1] last-block ticket, [2] grid-barrier counter
  int max_blocks;
  int fwidth;
  unsigned int bar_count;  // the grid-barrier counter's value after the launches so far
  int coop_blocks;         // reduce_step grid: 0 not yet sized, -1 unavailable
};

// ---- kernel launch wrappers (kernels.cu) ------------------------------

struct GaeArgs {
  const float *rewards, *values, *last_values;
  const uint8_t *dones;
  float *adv, *ret;
  int64_t n_envs, T;
  float gamma, lam;
};
void launch_gae(const GaeArgs &a, double *adv_sum_partials, int nblk,
                cudaStream_t s);
int gae_blocks(int64_t n_envs);

// Advantage moments (ppo.rs:342-345) in two passes over the batch: the sum
// (GAE produces its block partials directly), then the squared deviations
// from the global mean.  moments[0] = sum, moments[1] = sum of squares of
// deviations, both in double; a data-parallel group allreduces each slot
// before the next pass reads it.  finalize writes adv_mean / adv_sd.
int adv_blocks(int64_t n);
void launch_adv_sum(const float *adv, int64_t n, double *partials, int nblk,
                    cudaStream_t s);
void launch_reduce_moment(const double *partials, int nblk, double *moments,
                          int slot, cudaStream_t s);
void launch_adv_sqdev(const float *adv, int64_t n, const double *moments,
                      int64_t n_global, double *partials, int nblk,
                      cudaStream_t s);
void launch_adv_finalize(const double *moments, int64_t n_global, DevState *st,
                         cudaStream_t s);

// Epoch gather: rows order[p] of the batch -> position p: the observation
// rows from their normalized copies (Normalizer::normalize applied once per
// update, ppo.rs:196-205), the advantage normalization (ppo.rs:346-348)
// applied to adv.  With the mirror augmentation on (n_base > 0) the batch
// is 2 n_base virtual rows: row r < n_base is the L/R mirror of base row r
// (biped_train_gpu.rs:89-185: its observation rows from the normalized
// mirrored copies xm_a / xm_c, its action and mean_old through the action
// space's signed permutation), row r >= n_base is base row r - n_base.
struct GatherArgs {
  const int32_t *order;  // [n_used] local (virtual) row indices
  int64_t n_used;
  const float *xn_a, *xn_c;  // normalized observation rows, pitch odp / cdp
  const float *xm_a, *xm_c;  // the same of the mirrored rows (mirror on)
  const float *action, *mean_old, *logp_old, *value_old, *adv, *ret;
  int A;
  int odp, cdp;           // padded row pitch (multiples of 32 elements)
  int x_bytes;            // bytes per observation element (4, or 2 for bf16)
  const DevState *st;   // adv_mean / adv_sd
  float *x_a, *x_c;     // [n_used, odp], [n_used, cdp]
  float *g_action, *g_mean_old;         // [n_used, A]
  float *g_logp_old, *g_value_old, *g_adv, *g_ret;
  int apply_adv_norm;
  int64_t n_base;       // mirror augmentation: base rows (0 = off)
  const int32_t *m_aperm;  // action space: (P a)[k] = sign[k] * a[perm[k]]
  const float *m_asign;
};
void launch_gather(const GatherArgs &a, cudaStream_t s);
// Normalizer divisors: sd = sqrt(max(m2/count, 1e-8)) (ppo.rs:201-202).
void launch_norm_prepare(const float *m2, float count, int dim, float *sd,
                         cudaStream_t s);
// perm/sign (optional): rows mapped by a signed permutation first.
void launch_normalize_rows(const float *x, int64_t n, int dim, int pitch,
                           const float *mean, const float *sd, float *out,
                           int mode, cudaStream_t s, const int32_t *perm = nullptr,
                           const float *sign = nullptr);
// dst = tf32(src) (round to nearest) over n floats.
// dst[i] = src[i] stored as `mode` says (1 tf32-rounded fp32, 2 bf16).
void launch_round_copy(const float *src, float *dst, int64_t n, int mode, cudaStream_t s);
// The epoch permutation of ppo.rs:357-363 (Fisher-Yates driven by
// Lcg::new(seed)) into order[n] on the device (shuffle_dev.cu); scratch
// holds 3 n int32.
void launch_shuffle_device(uint64_t seed, int32_t n, int32_t *order, int32_t *scratch,
                           cudaStream_t s);
// One rank's share of a device permutation perm[n_global] (shuffle_dev.cu):
// per slice of n_global / mbs positions, the positions whose sample lies in
// [row_offset, row_offset + n_local), as local rows, in permutation order,
// into order[]; counts[0..mbs] (device, mbs + 1 entries) ends with the
// per-slice counts in counts[0..mbs-1].  scratch holds n_global / 1024 + 1
// int32.
void launch_rank_orders(const int32_t *perm, int64_t n_global, int64_t n_local,
                        int64_t row_offset, int mbs, int32_t *order, int64_t *counts,
                        int32_t *scratch, cudaStream_t s);

// PPO losses (ppo.rs:410-452) over one minibatch.
struct LossArgs {
  const float *mean;      // actor output [mb, Ap]
  const float *value;     // critic output [mb, cp] (column 0)
  int Ap, cp;
  const float *action, *mean_old;       // [mb, A]
  const float *logp_old, *value_old, *adv, *ret;  // [mb]
  const float *log_std;   // [A]
  int A;
  int64_t mb;
  float scale;            // 1 / global minibatch size
  float clip, entropy_coef, value_coef;
  float *d_actor;         // [mb, Ap] delta of the actor output layer
  float *d_critic;        // [mb, cp] delta of the critic output layer
  // one partial row per block, width = 2 Ap + 4 + cp floats:
  // [g_logstd | db_actor | surr vloss kl 0 | db_critic], the log_std
  // gradient, the output-layer bias gradients (column sums of the two
  // deltas, taken in fp32 before any rounding) and the statistic sums
  float *part;
  int width;
  int out_mode;           // storage of the two output deltas (OperandMode)
};
void launch_loss(const LossArgs &a, cudaStream_t s);
int loss_blocks(const LossArgs &a);  // the partial rows launch_loss writes

// Column sums of a [rows, cols] matrix, split over row chunks into
// partials [splits, cols].
void launch_colsum(const float *x, int64_t rows, int cols, int ld,
                   float *partials, int splits, cudaStream_t s);

// Sum `splits` partial buffers into dst for a list of segments.
struct ReduceSeg {
  float *dst;
  const float *src;      // splits partial rows of count floats, stride apart
  int64_t count;
  int splits;
  int64_t stride;        // floats between partial rows (>= count)
};
constexpr int kMaxSegs = 2 * ZRL_MAX_LAYERS * 2 + 4;
struct ReduceSegs {
  ReduceSeg seg[kMaxSegs];
  int n;
  // filled by launch_reduce_segments: first block and split groups of
  // each segment
  int first_block[kMaxSegs + 1];
  int groups[kMaxSegs];
  int net[kMaxSegs];  // with a fused pre-step: 0 actor, 1 critic, -1 neither
};
struct PrestepArgs;
struct ReduceScratch;
// With `fuse` (one rank: no allreduce between the two), the reduce also
// takes the per-net squared norms of what it writes and its last block
// runs the pre-step; returns 1 when it did (launch_prestep is then
// skipped), 0 otherwise.
int launch_reduce_segments(const ReduceSegs &segs, cudaStream_t s,
                           const PrestepArgs *fuse = nullptr, ReduceScratch *rs = nullptr);

// Squared norms of the actor/critic gradient segments, then the pre-step
// scalars (ppo.rs:473-482, net.rs:197-202, net.rs:235-238, ppo.rs:497-500)
// computed by the last block.
struct PrestepArgs {
  const float *grads;
  int64_t actor_begin, actor_end, critic_begin, critic_end;
  const float *log_std;
  int A;
  const float *sums3;
  float max_grad_norm, desired_kl, lr_min, lr_max;
  int adaptive_lr;
  int minibatches;
  int last_of_epoch;
  int count_stats;
  DevState *st;
};
void launch_prestep(const PrestepArgs &a, ReduceScratch &rs, cudaStream_t s);

// Adam over the whole padded parameter buffer (net.rs:233-251,
// ppo.rs:496-510), with the per-net clip scale folded in.
struct AdamArgs {
  float *p, *m, *v;
  const float *g;
  int64_t n;
  int64_t actor_end, critic_end;  // [0,actor_end) actor, [.., critic_end) critic, rest log_std
  const DevState *st;
  float *p_round;  // optional: copy of p for the tensor-core GEMMs, stored
                   // as p_mode says (1 tf32-rounded fp32, 2 bf16)
  int p_mode;
};
void launch_adam(const AdamArgs &a, cudaStream_t s);

// One rank: the segment reduce, the pre-step and Adam in one cooperative
// launch (a grid barrier between the reduce and the step).  Several ranks
// (from_grads, segs empty): the pre-step's norms of the allreduced gradient
// and Adam, likewise.  Returns false, having launched nothing, where the
// device refuses a cooperative launch; the caller then runs the separate
// kernels.  A barrier wait that runs out leaves code 8 in *err.
bool launch_reduce_step(const ReduceSegs &segs, const PrestepArgs &pa, const AdamArgs &aa,
                        ReduceScratch &rs, int *err, cudaStream_t s, bool from_grads = false);

// Copy an n-element slice of a padded [rows, pitch] buffer into a dense
// [rows, cols] one (and back).
void launch_unpad_rows(const float *src, int64_t rows, int pitch, int cols,
                       float *dst, cudaStream_t s);
// Rollout sampling: action = mean + exp(log_std) * eps, eps from
// Philox4x32-10 keyed by (seed, counter); logp per row (may be null).
void launch_policy_sample(const float *mean, int pitch, const float *log_std,
                          int A, int64_t n, uint64_t seed, uint64_t counter,
                          float *action, float *logp, float *mean_out,
                          cudaStream_t s, int64_t row0 = 0);
// The reference's sampling stream (shuffle_dev.cu): action = mean +
// exp(log_std) * Lcg::gauss() with the gauss of (row, k) the (row * A + k)-th
// of one Lcg stream that starts at state s0 (rows numbered from row0).
void launch_lcg_sample(const float *mean, int pitch, const float *log_std, int A, int64_t n,
                       uint64_t s0, int64_t row0, float *action, float *mean_out,
                       cudaStream_t s);
// logp of n action rows (ppo.rs:297-305).
void launch_logp_rows(const float *action, const float *mean, int pitch, const float *log_std,
                      int A, int64_t n, float *logp, cudaStream_t s);
// Normalizer::update over n rows in order (bit-exact Welford).
void launch_record_obs(const float *x, int64_t n, int dim, float *mean,
                       float *m2, float count0, cudaStream_t s);
// The parallel Welford fold (welford.cu): rows in chunks of
// kWelfordChunkRows folded from empty states, merged into (count0, mean,
// m2) in chunk order by Normalizer::commit's formula; scratch holds
// welford_partial_floats(n, dim) floats.
constexpr int kWelfordChunkRows = 256;
int64_t welford_partial_floats(int64_t n, int dim);
void launch_welford_parallel(const float *x, int64_t n, int dim, float count0, float *mean,
                             float *m2, float *scratch, cudaStream_t s);
// Normalizer::commit (ppo.rs:179-195): the pending state merged into the
// live one, then reset (the counts are kept on the host).
void launch_norm_commit(float *mean, float *m2, float count, float *p_mean, float *p_m2,
                        float p_count, int dim, cudaStream_t s);

// ---- GEMMs (gemm_simt.cu / gemm_tc.cu) ---------------------------------

enum Epilogue {
  EPI_STORE = 0,      // C = acc
  EPI_BIAS = 1,       // C = acc + bias[n]
  EPI_BIAS_ELU = 2,   // C = elu(acc + bias[n])
  EPI_ELU_GRAD = 3    // C = acc * elu'(aux[m][n]) from the post-activation
};

// C[M,N] = op(A)[M,K] * op(B)[K,N] with fp32 FMA on CUDA cores.
//   trans_a: A is stored [K, M] (lda = its row pitch)
//   trans_b: B is stored [N, K]
// split_k > 1 writes partial sums to C + z*ldc*M for z < split_k.
struct GemmArgs {
  int M, N, K;
  const float *A; int lda; bool trans_a;
  const float *B; int ldb; bool trans_b;
  float *C; int ldc;
  int epi;
  const float *bias;
  const float *aux; int ldaux;
  int split_k;
  int round_out;  // tensor-core path: round the outputs to tf32 (RN)
  // tensor-core dgrad: column sums of the (unrounded) outputs, one row of N
  // partials per 128-row tile: colsum[tile_m * N + n]
  float *colsum;
  // tensor-core launches: walk the output tiles last to first (a launch
  // that reads what the previous one wrote meets its most recent tiles
  // first, while they are still in L2); no effect on the results
  int reverse_tiles;
};
void gemm_simt(const GemmArgs &g, cudaStream_t s);

}  // namespace zrl

#define ZRL_CUDA_CHECK_LAUNCH() (cudaGetLastError())
