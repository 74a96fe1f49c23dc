/*
 * zealot_rl.h -- C ABI of libzealot_rl.so, the B200 (sm_100a) backend for
 * zealot-rl's PPO update.
 *
 * Every entry point replaces one piece of the zealot-rl Rust API
 * (zealot-rl/src/lib.rs:27-28 re-exports); the reference item is cited
 * beside each declaration.  Conventions:
 *
 *  - Every call returns zrl_status; nothing aborts or throws across the ABI.
 *    zrl_last_error() gives the message of the last failure on a context.
 *  - Host pointers are borrowed for the duration of the call only.  Entry
 *    points that accept device pointers say so; "on_device" selects.
 *  - One context = one CUDA device + one stream.  A context is not
 *    thread-safe; use one context per thread.
 *  - Parameter vectors ("flat") use the tensor order of ActorCritic::save
 *    (zealot-rl/src/ppo.rs:539-571): actor.w_0 [out,in], actor.b_0 [out],
 *    ..., critic.w_0, critic.b_0, ..., log_std [act_dim].
 *  - Batches are structure-of-arrays, one row per zealot-rl Sample
 *    (ppo.rs:67-87), row index = env * T + t (env-major, as
 *    src/bin/biped_train_gpu.rs:982-987 flattens a rollout).
 */
#ifndef ZEALOT_RL_H
#define ZEALOT_RL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZRL_ABI_VERSION 1
#define ZRL_MAX_LAYERS 8

typedef enum {
  ZRL_OK = 0,
  ZRL_INVALID_ARG = 1,
  ZRL_CUDA_ERROR = 2,
  ZRL_NCCL_ERROR = 3,
  ZRL_TIMEOUT = 4,
  ZRL_NOT_SUPPORTED = 5,
  ZRL_OUT_OF_MEMORY = 6,
  ZRL_IO_ERROR = 7
} zrl_status;

/* GEMM arithmetic of the MLP forward/backward. */
typedef enum {
  ZRL_GEMM_TF32 = 0, /* tcgen05 kind::tf32, fp32 accumulate (default)   */
  ZRL_GEMM_FP32 = 1, /* CUDA-core fp32 FMA: the exact-parity mode       */
  ZRL_GEMM_BF16 = 2  /* tcgen05 kind::f16 with bf16 inputs, fp32 master */
} zrl_gemm_precision;

/* PpoConfig (zealot-rl/src/ppo.rs:22-65); lr_bounds split in two. */
typedef struct {
  float gamma, lam, clip, entropy_coef, value_coef;
  int32_t epochs, minibatches;
  float max_grad_norm, desired_kl, lr_min, lr_max;
  int32_t adaptive_lr;
} zrl_ppo_config;

/* PpoStats (ppo.rs:89-102). */
typedef struct {
  float kl, surrogate, value_loss, entropy, lr;
} zrl_stats;

/* Network shapes and capacity.  actor_dims[0] = obs dim,
 * actor_dims[n_actor_dims-1] = action dim (at most 128); critic_dims ends in
 * 1; both observation widths at most 256 (ZRL_NOT_SUPPORTED beyond)
 * (ActorCritic::new, ppo.rs:235-247). */
typedef struct {
  int32_t n_actor_dims;
  int32_t actor_dims[ZRL_MAX_LAYERS + 1];
  int32_t n_critic_dims;
  int32_t critic_dims[ZRL_MAX_LAYERS + 1];
  int64_t max_samples;  /* largest batch (rows) update() will be given   */
  int32_t precision;    /* zrl_gemm_precision                            */
} zrl_model_config;

/* Data-parallel group.  world_size == 1 (or a NULL zrl_comm) runs alone.
 * nccl_id is the 128-byte ncclUniqueId made by rank 0 and shared by the
 * caller (the reference is single-GPU: this has no counterpart there). */
typedef struct {
  int32_t rank;
  int32_t world_size;
  uint8_t nccl_id[128];
  int32_t timeout_ms; /* bound on each collective wait; <=0 means 60000 */
} zrl_comm;

/* One batch of samples (SoA).  For a data-parallel group, each rank passes
 * the rows it owns: global rows [row_offset, row_offset + n) of a global
 * batch of n_global rows. */
typedef struct {
  const float *obs;        /* [n, obs_dim]        */
  const float *critic_obs; /* [n, critic_obs_dim] */
  const float *action;     /* [n, act_dim]        */
  const float *mean_old;   /* [n, act_dim]        */
  const float *logp_old;   /* [n] */
  const float *value_old;  /* [n] */
  float *adv;              /* [n]  (advantages, normalized in place when
                                    write_back_adv is set)               */
  const float *ret;        /* [n] */
  int64_t n;
  int64_t n_global;        /* 0 means n (single rank)                    */
  int64_t row_offset;
  int32_t on_device;       /* pointers are CUDA device pointers          */
  int32_t write_back_adv;  /* store normalized advantages back into adv  */
} zrl_batch;

/* A rollout for the fused GAE + update entry point: env-major [n_envs, T]
 * rewards/values/dones plus the bootstrap values [n_envs]. */
typedef struct {
  const float *rewards;
  const float *values;
  const uint8_t *dones;
  const float *last_values;
  int64_t n_envs;
  int64_t T;
} zrl_rollout;

typedef struct zrl_ctx zrl_ctx;

/* Fills out[128] with a fresh ncclUniqueId (rank 0 calls it, the caller
 * distributes the bytes to the other ranks' zrl_comm.nccl_id).  No
 * counterpart in the reference, which trains on one device. */
zrl_status zrl_nccl_unique_id(uint8_t *out);

/* ---- lifetime ------------------------------------------------------- */

/* Creates a context on `device`.  comm may be NULL.
 * Replaces: ActorCritic::new's allocation half (ppo.rs:235-266); the
 * initialisation half is zrl_init_reference / zrl_set_params. */
zrl_status zrl_create(const zrl_model_config *cfg, int device,
                      const zrl_comm *comm, zrl_ctx **out);
/* Frees the context (the reference's ActorCritic is freed by Drop). */
zrl_status zrl_destroy(zrl_ctx *ctx);
/* The message of the last failure on ctx (where the reference panics, this
 * library returns a status and keeps the message here). */
const char *zrl_last_error(const zrl_ctx *ctx);
/* ZRL_ABI_VERSION of the loaded library.  No counterpart in the reference. */
int32_t zrl_abi_version(void);
/* Blocks until the context's stream is idle.  No counterpart in the
 * reference (its update returns when the work is done). */
zrl_status zrl_synchronize(zrl_ctx *ctx);
/* The context's cudaStream_t, for callers that order their own work.  No
 * counterpart in the reference. */
void *zrl_stream(zrl_ctx *ctx);

/* ---- parameters and state -------------------------------------------- */

/* Length of the flat parameter vector: the element count of the tensors
 * ActorCritic::save writes (ppo.rs:539-571). */
int64_t zrl_param_count(const zrl_ctx *ctx);
/* ActorCritic::new initialisation (ppo.rs:235-266, net.rs:61-78) from an
 * Lcg state (rng.rs); *lcg_state is advanced exactly as the reference. */
zrl_status zrl_init_reference(zrl_ctx *ctx, float init_noise_std,
                              float init_lr, uint64_t *lcg_state);
/* Replace/read all parameters (flat, save order).  Setting parameters
 * resets the Adam state, as ActorCritic::load does (ppo.rs:633-647). */
zrl_status zrl_set_params(zrl_ctx *ctx, const float *flat, int64_t count);
zrl_status zrl_get_params(zrl_ctx *ctx, float *flat, int64_t count);
/* Adam state (t for actor, critic, log_std; m and v flat in param order):
 * the reference's private opt_actor / opt_critic / m_logstd, v_logstd,
 * t_logstd fields (ppo.rs:221-226, net.rs:207-216), which it neither
 * exposes nor saves; here for checkpoints that keep them and for tests. */
zrl_status zrl_set_adam_state(zrl_ctx *ctx, const int32_t *t3,
                              const float *m, const float *v, int64_t count);
zrl_status zrl_get_adam_state(zrl_ctx *ctx, int32_t *t3, float *m, float *v,
                              int64_t count);
/* Normalizer state (ppo.rs:104-206): mean, m2, count for each net. */
zrl_status zrl_set_normalizers(zrl_ctx *ctx, const float *obs_mean,
                               const float *obs_m2, float obs_count,
                               const float *crit_mean, const float *crit_m2,
                               float crit_count);
zrl_status zrl_get_normalizers(zrl_ctx *ctx, float *obs_mean, float *obs_m2,
                               float *obs_count, float *crit_mean,
                               float *crit_m2, float *crit_count);
/* Normalizer::update for n rows of obs and critic obs (ActorCritic::
 * record_obs, ppo.rs:276-279), rows folded in order. */
zrl_status zrl_record_obs(zrl_ctx *ctx, const float *obs,
                          const float *critic_obs, int64_t n);
/* zrl_record_obs with device rows (on_device = 1) and a choice of fold:
 * mode 0 folds the rows in order (bit-identical to the reference), mode 1
 * folds chunks of 256 rows in parallel and merges them pairwise with
 * Normalizer::commit's formula (ppo.rs:185-191): the same statistics up to
 * f32 rounding, for large row counts. */
zrl_status zrl_record_obs_ex(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                             int64_t n, int32_t on_device, int32_t mode);
/* PendingNorm::push (ppo.rs:126-136) of n rows into the context's pending
 * statistics of each normalizer (the trainer's pn_obs / pn_cobs pair,
 * biped_train_gpu.rs:800-801, 904-905); modes as zrl_record_obs_ex. */
zrl_status zrl_pending_push(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                            int64_t n, int32_t on_device, int32_t mode);
/* Normalizer::commit (ppo.rs:179-195) of both pending states into the live
 * normalizers (biped_train_gpu.rs:1050-1051), which resets them; an empty
 * pending state leaves its normalizer as it is. */
zrl_status zrl_commit_pending(zrl_ctx *ctx);
/* The pending statistics (counts on the host): the fields of the two
 * PendingNorm values (ppo.rs:118-122). */
zrl_status zrl_get_pending(zrl_ctx *ctx, float *obs_mean, float *obs_m2,
                           float *obs_count, float *crit_mean, float *crit_m2,
                           float *crit_count);
/* ActorCritic::lr (ppo.rs:228). */
zrl_status zrl_set_lr(zrl_ctx *ctx, float lr);
zrl_status zrl_get_lr(zrl_ctx *ctx, float *lr);

/* ---- the hot path ----------------------------------------------------- */

/* gae (ppo.rs:681-703) for n_envs env-major trajectories of length T. */
zrl_status zrl_gae(zrl_ctx *ctx, const float *rewards, const float *values,
                   const uint8_t *dones, const float *last_values,
                   int64_t n_envs, int64_t T, float gamma, float lam,
                   float *adv_out, float *ret_out, int32_t on_device);

/* ActorCritic::update (ppo.rs:338-384): advantage normalization, then
 * epochs x minibatches of shuffled minibatch steps (ppo.rs:388-510).
 * Returns the last epoch's mean stats. */
zrl_status zrl_update(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                      zrl_batch *batch, zrl_stats *out);

/* gae for every env of the rollout, then update() on the batch whose adv
 * and ret are the GAE outputs (biped_train_gpu.rs:970-1553 in one call:
 * the batch's adv/ret fields are ignored).  rollout and batch must agree
 * on on_device. */
zrl_status zrl_gae_update(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                          const zrl_rollout *rollout, zrl_batch *batch,
                          zrl_stats *out);

/* ActorCritic::mean / value for n rows (ppo.rs:282-294). mean_out
 * [n, act_dim] and/or value_out [n] may be NULL. */
zrl_status zrl_forward(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                       int64_t n, float *mean_out, float *value_out,
                       int32_t on_device);

/* Rollout step: mean, value, a sampled action a = mean + exp(log_std)*eps
 * with eps ~ N(0,1) from a Philox4x32-10 counter stream keyed by
 * (seed, counter), and logp(a) (ActorCritic::sample, ppo.rs:313-323, and
 * GpuPolicy::forward, src/biped/gpu_policy.rs:210-248).  Outputs may be
 * NULL except action. */
zrl_status zrl_policy_step(zrl_ctx *ctx, const float *obs,
                           const float *critic_obs, int64_t n, uint64_t seed,
                           uint64_t counter, float *action, float *logp,
                           float *mean, float *value, int32_t on_device);
/* zrl_policy_step with the reference's sampler: the actions of row r draw
 * Lcg::gauss (rng.rs:28-32) from one sequential stream in (row, k) order, as
 * ActorCritic::sample (ppo.rs:313-323) and the GPU trainer's host loop
 * (biped_train_gpu.rs:913-919) do, starting at *lcg_state; on return
 * *lcg_state has advanced past the 2 n A uniforms used.  The uniforms are
 * the reference's bit for bit (jump-ahead on the device). */
zrl_status zrl_policy_step_lcg(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                               int64_t n, uint64_t *lcg_state, float *action, float *logp,
                               float *mean, float *value, int32_t on_device);

/* ---- parity hooks ------------------------------------------------------ */

/* The gradient half of minibatch_step (ppo.rs:388-462) on rows idx[0..n_idx)
 * of the batch: flat gradient sums (save order, before clipping) and
 * sums3 = {surrogate, value_loss, kl}.  Parameters are not changed. */
zrl_status zrl_minibatch_grads(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                               const zrl_batch *batch, const int64_t *idx,
                               int64_t n_idx, float *grads_out,
                               float *sums3_out);
/* The epoch permutation of ppo.rs:357-363 (the same indices as zrl_shuffle)
 * computed on the context's device into order[n] (device pointer, int32,
 * n < 2^31): the Lcg draws by jump-ahead, then each position's value from
 * the chain of steps that last wrote it.  Replaces the host loop of
 * ppo.rs:357-363 for callers that want the order on the device. */
zrl_status zrl_shuffle_device(zrl_ctx *ctx, uint64_t seed, int64_t n,
                              int32_t *order);
/* zrl_rank_orders computed on the context's device (the permutation by
 * zrl_shuffle_device, then an order-keeping compaction of the rank's rows):
 * order is a device pointer (at most n_local int32), counts a host array of
 * minibatches entries.  Returns the total, or -1 (zrl_last_error says
 * why). */
int64_t zrl_rank_orders_device(zrl_ctx *ctx, uint64_t seed, int64_t n_global,
                               int64_t n_local, int64_t row_offset,
                               int32_t minibatches, int32_t *order,
                               int64_t *counts);
/* One MLP GEMM through the context's GEMM engine (the precision it was
 * created with), on device pointers, row-major; C is fp32, A and B are fp32
 * (fp32 and tf32 contexts) or bf16 (bf16 contexts: 2-byte elements, lda and
 * ldb in elements, multiples of 8):
 *   layout 0: C[M,N] = A[M,K] * B[N,K]^T   (forward:  X W^T)
 *   layout 1: C[M,N] = A[M,K] * B[K,N]     (dgrad:    Delta W)
 *   layout 2: C[M,N] = A[K,M]^T * B[K,N]   (wgrad:    Delta^T X)
 * split_k > 1 writes split_k partial products at C + z*M*ldc.  The
 * counterpart of the cuTile GEMM self-test (src/biped/cutile_gemm.rs:
 * 695-828), which checks the same three layouts. */
zrl_status zrl_gemm(zrl_ctx *ctx, int32_t layout, int32_t M, int32_t N,
                    int32_t K, const float *A, int32_t lda, const float *B,
                    int32_t ldb, float *C, int32_t ldc, int32_t split_k);
/* The stepping half of minibatch_step (ppo.rs:475-489): adaptive LR from
 * kl, per-net gradient clip, Adam for actor and critic, step_log_std. */
zrl_status zrl_apply_grads(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                           const float *grads, float kl);

/* GAE for n_envs env-major trajectories plus the normalized advantages,
 * allocating nothing: for callers that cannot call cudaMalloc where they
 * need advantages (GPU memory owned by another runtime's pool, a real-time
 * loop that forbids allocation).  All
 * pointers are caller-owned device buffers; `stream` is a cudaStream_t (NULL
 * for the legacy default stream).  Outputs: adv_out/ret_out as zrl_gae,
 * adv_norm_out = (adv - mean) / max(population sd, 1e-6).  Reduction
 * scratch is a fixed array inside the library (about 67 KB on every GPU
 * that loads it), so n_envs is limited to 262,144 (ZRL_INVALID_ARG above)
 * and T to 4096; the first call on a device looks up that array's address
 * (cudaGetSymbolAddress) and caches it, so make that first call before any
 * stream capture begins on the device; that address does not survive a
 * cudaDeviceReset of that device; calls that overlap on the GPU
 * race on the shared array.  It has no counterpart in the reference, which computes
 * GAE on the host. */
zrl_status zrl_gae_normalize_noalloc(const float *rewards, const float *values,
                                     const uint8_t *dones,
                                     const float *last_values, int64_t n_envs,
                                     int64_t T, float gamma, float lam,
                                     float *adv_out, float *ret_out,
                                     float *adv_norm_out, void *stream);

/* ---- checkpoint --------------------------------------------------------- */

/* ActorCritic::save / load / load_from_bytes (ppo.rs:529-650): safetensors,
 * F32, the reference's tensor names and shapes.  Adam state is not saved;
 * load resets it.  Load requires the file's dims to match the context. */
zrl_status zrl_save(zrl_ctx *ctx, const char *path);
zrl_status zrl_load(zrl_ctx *ctx, const char *path);
zrl_status zrl_load_from_bytes(zrl_ctx *ctx, const uint8_t *bytes,
                               size_t len);

/* ---- host helpers (no device work) ------------------------------------ */

/* Lcg (rng.rs:9-33). */
uint64_t zrl_lcg_new(uint64_t seed);
float zrl_lcg_unit(uint64_t *state);
float zrl_lcg_gauss(uint64_t *state);
/* The epoch permutation of ppo.rs:357-363: Fisher-Yates over n driven by
 * Lcg::new(seed).  order receives n indices. */
void zrl_shuffle(uint64_t seed, int64_t n, int64_t *order);
/* One rank's share of the epoch permutation (data parallel over rows): the
 * permutation of n_global samples (zrl_shuffle(seed)) cut into minibatches
 * slices of n_global / minibatches positions; per slice, the positions
 * whose sample lies in [row_offset, row_offset + n_local), as local rows, in
 * permutation order.  order receives them (at most n_local), counts[m] the
 * number in slice m; returns the total, or -1 on invalid arguments.  The
 * host logic the several-rank update runs. */
int64_t zrl_rank_orders(uint64_t seed, int64_t n_global, int64_t n_local,
                        int64_t row_offset, int32_t minibatches, int32_t *order,
                        int64_t *counts);

/* L/R mirror augmentation of the GPU trainer (biped_train_gpu.rs:89-185,
 * 988-1003): when set, zrl_update / zrl_gae_update train on 2 n samples,
 * the n mirrored copies first, then the batch itself.  A mirrored sample
 * has obs, critic_obs, action and mean_old mapped by signed permutations,
 * (P x)[i] = sign[i] * x[perm[i]] (each perm a permutation of its space,
 * each sign +-1), and logp_old, value_old, adv, ret unchanged.  The mirror
 * is applied once per update, where the observations are normalized: the
 * mirrored raw observations are normalized with the same statistics, as
 * the trainer normalizes each mirrored Sample, and written beside the
 * originals; action and mean_old are mapped as the epoch gather copies
 * them.  cfg->minibatches counts minibatches of the 2 n samples: the GPU
 * trainer keeps its minibatch size and doubles the count
 * (biped_train_gpu.rs:639-643, 1005), so pass twice its minibatches to
 * train as it does.  obs_perm = NULL turns it off.  One rank only
 * (ZRL_NOT_SUPPORTED with several). */
zrl_status zrl_set_mirror(zrl_ctx *ctx, const int32_t *obs_perm, const float *obs_sign,
                          const int32_t *cobs_perm, const float *cobs_sign,
                          const int32_t *act_perm, const float *act_sign);

/* ---- failure handling ---------------------------------------------------- */

/* Bound (ns, at least 1 ms) of every wait inside the tensor-core kernels'
 * pipelines (default 20 s): a wait that runs out records a code in the
 * context's device error flag, every role of the kernel gives up in turn,
 * and the call that finishes the work returns ZRL_TIMEOUT (the flag is then
 * cleared, so the context stays usable).  No counterpart in the reference,
 * which has no device pipelines. */
zrl_status zrl_set_wait_limit(zrl_ctx *ctx, uint64_t ns);
/* Test hook: the next tensor-core GEMM launch of this context makes its MMA
 * issuer wait on a barrier that nothing completes, so the wait runs out
 * after the wait limit (the failure path above, without a GPU fault).  No
 * counterpart in the reference. */
zrl_status zrl_test_stall_next_gemm(zrl_ctx *ctx);
/* Test hook: the bounded stream wait of the several-rank path (the poll of
 * the stream and of NCCL's asynchronous error that aborts the communicator
 * on a timeout or an error) run on fakes, no GPU needed: scenario 0 the
 * stream completes, 1 it never does (ZRL_TIMEOUT after timeout_ms), 2 the
 * communicator reports an error (ZRL_NCCL_ERROR), 3 the stream reports a
 * failed kernel (ZRL_CUDA_ERROR).  *aborted: whether the communicator was
 * aborted.  No counterpart in the reference. */
zrl_status zrl_test_comm_wait(int32_t scenario, int32_t timeout_ms, int32_t *aborted);

/* ---- instrumentation ---------------------------------------------------- */

/* Number of kernels this context launched since it was created.  No
 * counterpart in the reference (instrumentation). */
int64_t zrl_kernel_launches(const zrl_ctx *ctx);
/* Device time (ms) of the GEMM kernels of the last update, measured with
 * CUDA events on the context's stream when profiling is enabled.  No
 * counterpart in the reference (instrumentation). */
zrl_status zrl_set_profiling(zrl_ctx *ctx, int32_t enabled);
zrl_status zrl_get_profile(zrl_ctx *ctx, float *gemm_ms, float *update_ms,
                           int64_t *gemm_launches);
/* Per launch site of the last profiled update (forward layer, input-
 * gradient level, weight-gradient group, loss, segment reduce, Adam,
 * gather, ...): entry i's name, summed device time (ms) and number of
 * bracketed launches.  Returns 0 past the last entry.  Instrumentation with
 * no counterpart in the reference; the events that bracket each site keep
 * consecutive kernels from overlapping, so the sum exceeds an unprofiled
 * update's time slightly. */
int32_t zrl_profile_site(const zrl_ctx *ctx, int32_t i, const char **name, float *ms,
                         int64_t *spans);

#ifdef __cplusplus
}
#endif
#endif
