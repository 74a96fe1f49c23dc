/*
 * zrl_oracle.h -- CPU restatement of zealot-rl's PPO update path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * library (libzealot_rl.so) is compared against.  Only tests/, the smoke()
 * entry and bench.py's CPU-baseline leg may load it; no product code path
 * links, imports or calls it.
 *
 * Each function restates one piece of zealot-rl (Rust, zealot-rl/src/{rng,net,ppo}.rs)
 * in plain C with the same f32 operation order, so the sequential mode
 * reproduces the reference's single-threaded results:
 *
 *   rng.rs        Lcg::new / unit / gauss                 -> orc_lcg_*
 *   ppo.rs:356-363 per-epoch Fisher-Yates shuffle          -> orc_shuffle
 *   ppo.rs:681-703 gae                                     -> orc_gae
 *   net.rs:61-140  Mlp::new / forward / backward           -> orc_mlp_*
 *   net.rs:181-202 MlpGrad::l2_norm / clip                 -> orc_grad_*
 *   net.rs:233-251 Adam::step                              -> orc_adam_step
 *   ppo.rs:104-205 Normalizer                              -> orc_norm_*
 *   ppo.rs:338-510 ActorCritic::update / minibatch_step /
 *                  step_log_std                            -> orc_ac_*
 *
 * The parameter layout of every flat buffer here is the order in which
 * ActorCritic::save pushes tensors (ppo.rs:539-571):
 *   actor.w_0 [out,in], actor.b_0 [out], ..., critic.w_0, critic.b_0, ...,
 *   log_std [act_dim].
 */
#ifndef ZRL_ORACLE_H
#define ZRL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MAX_LAYERS 8

/* ---- rng.rs ---- */
uint64_t orc_lcg_new(uint64_t seed);
float orc_lcg_unit(uint64_t *state);
float orc_lcg_gauss(uint64_t *state);
void orc_lcg_fill_unit(uint64_t *state, float *out, int64_t n);
void orc_lcg_fill_gauss(uint64_t *state, float *out, int64_t n);

/* ---- ppo.rs:356-363: order[] after Fisher-Yates with Lcg::new(seed) ---- */
void orc_shuffle(uint64_t seed, int64_t n, int64_t *order);

/* ---- ppo.rs:681-703 (one trajectory of length T) ---- */
void orc_gae(const float *rewards, const float *values, const uint8_t *dones,
             float last_value, int64_t T, float gamma, float lam,
             float *adv, float *ret);
/* Many env-major trajectories: arrays are [n_envs][T]. */
void orc_gae_batch(const float *rewards, const float *values,
                   const uint8_t *dones, const float *last_values,
                   int64_t n_envs, int64_t T, float gamma, float lam,
                   float *adv, float *ret);

/* ---- net.rs ---- */
int64_t orc_mlp_param_count(const int32_t *dims, int32_t n_dims);
/* Mlp::new: w ~ N(0, 1/fan_in) via Lcg::gauss, last layer * out_scale, b=0.
 * params layout: w_0, b_0, w_1, b_1, ... */
void orc_mlp_init(const int32_t *dims, int32_t n_dims, float out_scale,
                  uint64_t *rng, float *params);
/* Activations layout: a_0 (dims[0]) | a_1 (dims[1]) | ... | a_L. */
int64_t orc_mlp_act_count(const int32_t *dims, int32_t n_dims);
void orc_mlp_forward(const int32_t *dims, int32_t n_dims, const float *params,
                     const float *x, float *acts);
/* Accumulates into grads (same layout as params); writes the input gradient
 * to g_in when it is non-NULL. */
void orc_mlp_backward(const int32_t *dims, int32_t n_dims, const float *params,
                      const float *acts, const float *g_out, float *grads,
                      float *g_in);
float orc_grad_l2_norm(const float *g, int64_t n);
void orc_grad_clip(float *g, int64_t n, float max_norm);
/* Adam::step over one flat tensor list; *t is incremented first. */
void orc_adam_step(float *p, const float *g, float *m, float *v, int64_t n,
                   int32_t *t, float lr);
float orc_powi(float a, int32_t b);

/* ---- ppo.rs:104-205 Normalizer ---- */
void orc_norm_normalize(const float *mean, const float *m2, float count,
                        const float *x, int64_t dim, float *out);
void orc_norm_update(float *mean, float *m2, float *count, const float *x,
                     int64_t dim);
/* ppo.rs:179-195 Normalizer::commit of a PendingNorm (ppo.rs:126-136, whose
 * push is orc_norm_update from count 0): Chan merge, then pending reset. */
void orc_norm_commit(float *mean, float *m2, float *count, float *p_mean,
                     float *p_m2, float *p_count, int64_t dim);

/* ---- ppo.rs ActorCritic ---- */
typedef struct {
  float gamma, lam, clip, entropy_coef, value_coef;
  int32_t epochs, minibatches;
  float max_grad_norm, desired_kl, lr_min, lr_max;
  int32_t adaptive_lr;
} orc_ppo_config;

typedef struct {
  float kl, surrogate, value_loss, entropy, lr;
} orc_stats;

/* Structure-of-arrays batch (one row per Sample, ppo.rs:67-87). */
typedef struct {
  const float *obs;        /* [n, obs_dim]        */
  const float *critic_obs; /* [n, critic_obs_dim] */
  const float *action;     /* [n, act_dim]        */
  const float *mean_old;   /* [n, act_dim]        */
  const float *logp_old;   /* [n] */
  const float *value_old;  /* [n] */
  float *adv;              /* [n], normalized in place by update */
  const float *ret;        /* [n] */
  int64_t n;
} orc_batch;

typedef struct orc_ac orc_ac;

orc_ac *orc_ac_new(const int32_t *actor_dims, int32_t n_actor_dims,
                   const int32_t *critic_dims, int32_t n_critic_dims);
void orc_ac_free(orc_ac *ac);
/* ActorCritic::new's initialisation (ppo.rs:235-266) from an Lcg state. */
void orc_ac_init_reference(orc_ac *ac, float init_noise_std, float init_lr,
                           uint64_t *rng);
int64_t orc_ac_param_count(const orc_ac *ac);
void orc_ac_set_params(orc_ac *ac, const float *flat);
void orc_ac_get_params(const orc_ac *ac, float *flat);
void orc_ac_set_normalizers(orc_ac *ac, const float *obs_mean,
                            const float *obs_m2, float obs_count,
                            const float *crit_mean, const float *crit_m2,
                            float crit_count);
void orc_ac_set_lr(orc_ac *ac, float lr);
float orc_ac_get_lr(const orc_ac *ac);
/* 0 (default): the reference's f32 arithmetic.  1: additionally round every
 * GEMM operand to tf32 where a tensor-core backend stores it (inputs,
 * weights, hidden activations, the deltas entering the weight- and
 * input-gradient products), which isolates the tf32 rounding a tf32 GEMM
 * backend adds from everything else. */
void orc_ac_set_operand_rounding(orc_ac *ac, int32_t mode);
/* Adam state: t values for actor, critic, log_std; m/v flat in param order. */
void orc_ac_get_adam(const orc_ac *ac, int32_t *t3, float *m, float *v);
void orc_ac_set_adam(orc_ac *ac, const int32_t *t3, const float *m,
                     const float *v);

/* mean (act_dim) and value for n observations (ActorCritic::mean / value). */
void orc_ac_forward(const orc_ac *ac, const float *obs, const float *cobs,
                    int64_t n, float *mean_out, float *value_out);
float orc_ac_logp(const orc_ac *ac, const float *action, const float *mean);
float orc_ac_entropy(const orc_ac *ac);

/* The accumulation half of minibatch_step (ppo.rs:388-462): gradient sums
 * (flat param order, log_std segment included) and the three stat sums
 * {surrogate, value_loss, kl}.  n_threads <= 1 is the sequential fold. */
void orc_ac_minibatch_grads(const orc_ac *ac, const orc_batch *b,
                            const int64_t *idx, int64_t n_idx,
                            const orc_ppo_config *cfg, float *grads,
                            float *sums3, int32_t n_threads);
/* The stepping half of minibatch_step (ppo.rs:475-489): adaptive LR from kl,
 * per-net clip, Adam x2, step_log_std.  grads is consumed (clipped in place
 * in a copy). */
void orc_ac_apply(orc_ac *ac, const orc_ppo_config *cfg, const float *grads,
                  float kl);
/* ActorCritic::update (ppo.rs:338-384).  Normalizes b->adv in place. */
int orc_ac_update(orc_ac *ac, orc_batch *b, const orc_ppo_config *cfg,
                  orc_stats *out, int32_t n_threads);

#ifdef __cplusplus
}
#endif
#endif
