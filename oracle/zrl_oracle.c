/*
 * zrl_oracle.c -- CPU restatement of zealot-rl's PPO update (TEST ONLY).
 *
 * This is the checker for the CUDA library, never part of it.  Compile with
 * -ffp-contract=off (no fused multiply-add) and without fast-math, so every
 * f32 expression rounds exactly like the reference Rust, which LLVM does not
 * contract by default.  Every function names the reference lines it
 * follows; operation order inside expressions is kept as written there.
 */
#include "zrl_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ppo.rs:18 */
#define LOG_SQRT_2PI 0.9189385f
/* std::f32::consts::TAU */
#define TAU_F32 6.28318548202514648f

/* ------------------------------------------------------------------ rng.rs */

/* rng.rs:14-16 */
uint64_t orc_lcg_new(uint64_t seed) { return seed | 1ull; }

/* rng.rs:19-26 */
float orc_lcg_unit(uint64_t *s) {
  *s = *s * 6364136223846793005ull + 1442695040888963407ull;
  return (float)(*s >> 40) / (float)(1ull << 24);
}

/* rng.rs:28-32 */
float orc_lcg_gauss(uint64_t *s) {
  float u1 = orc_lcg_unit(s);
  if (u1 < 1e-7f) u1 = 1e-7f; /* f32::max(1e-7) */
  float r = sqrtf(-2.0f * logf(u1));
  return r * cosf(TAU_F32 * orc_lcg_unit(s));
}

void orc_lcg_fill_unit(uint64_t *s, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_lcg_unit(s);
}

void orc_lcg_fill_gauss(uint64_t *s, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_lcg_gauss(s);
}

/* -------------------------------------------------------- ppo.rs:356-363 */

void orc_shuffle(uint64_t seed, int64_t n, int64_t *order) {
  for (int64_t i = 0; i < n; ++i) order[i] = i;
  uint64_t sh = orc_lcg_new(seed);
  for (int64_t i = n - 1; i >= 1; --i) {
    float u = orc_lcg_unit(&sh);
    float prod = u * (float)(i + 1);
    int64_t j = (int64_t)prod; /* `as usize` truncation; prod >= 0 */
    if (j > i) j = i;          /* j.min(i) */
    int64_t tmp = order[i];
    order[i] = order[j];
    order[j] = tmp;
  }
}

/* -------------------------------------------------------- ppo.rs:681-703 */

void orc_gae(const float *rewards, const float *values, const uint8_t *dones,
             float last_value, int64_t T, float gamma, float lam, float *adv,
             float *ret) {
  float gae_acc = 0.0f;
  float next_v = last_value;
  for (int64_t i = T - 1; i >= 0; --i) {
    float nonterminal = dones[i] ? 0.0f : 1.0f;
    float delta = rewards[i] + gamma * next_v * nonterminal - values[i];
    gae_acc = delta + gamma * lam * nonterminal * gae_acc;
    adv[i] = gae_acc;
    ret[i] = gae_acc + values[i];
    next_v = values[i];
  }
}

/* gae per env of an env-major [n_envs, T] rollout, as the GPU trainer calls
 * it per env (biped_train_gpu.rs:974-981). */
void orc_gae_batch(const float *rewards, const float *values,
                   const uint8_t *dones, const float *last_values,
                   int64_t n_envs, int64_t T, float gamma, float lam,
                   float *adv, float *ret) {
  for (int64_t e = 0; e < n_envs; ++e)
    orc_gae(rewards + e * T, values + e * T, dones + e * T, last_values[e], T,
            gamma, lam, adv + e * T, ret + e * T);
}

/* ------------------------------------------------------------------ net.rs */

/* net.rs:13-16 */
static inline float elu(float x) { return x > 0.0f ? x : expf(x) - 1.0f; }
/* net.rs:21-23 */
static inline float elu_grad_from_act(float a) {
  return a > 0.0f ? 1.0f : a + 1.0f;
}

/* Parameters of Mlp::new(dims) (net.rs:61-78): w [out, in] and b [out] per
 * layer. */
int64_t orc_mlp_param_count(const int32_t *dims, int32_t n_dims) {
  int64_t c = 0;
  for (int32_t l = 0; l + 1 < n_dims; ++l)
    c += (int64_t)dims[l + 1] * dims[l] + dims[l + 1];
  return c;
}

int64_t orc_mlp_act_count(const int32_t *dims, int32_t n_dims) {
  int64_t c = 0;
  for (int32_t l = 0; l < n_dims; ++l) c += dims[l];
  return c;
}

/* net.rs:61-78 */
void orc_mlp_init(const int32_t *dims, int32_t n_dims, float out_scale,
                  uint64_t *rng, float *params) {
  int32_t layers = n_dims - 1;
  float *p = params;
  for (int32_t l = 0; l < layers; ++l) {
    int32_t fan_in = dims[l], fan_out = dims[l + 1];
    int last = l == layers - 1;
    float s = sqrtf(1.0f / (float)fan_in) * (last ? out_scale : 1.0f);
    for (int64_t k = 0; k < (int64_t)fan_out * fan_in; ++k)
      p[k] = orc_lcg_gauss(rng) * s;
    p += (int64_t)fan_out * fan_in;
    for (int32_t o = 0; o < fan_out; ++o) p[o] = 0.0f;
    p += fan_out;
  }
}

/* Operand rounding of a tf32 tensor-core GEMM, emulated: the value on the
 * tf32 grid (10 mantissa bits), nearest, ties away from zero.  The product
 * of two tf32 values is exact in f32, so a GEMM on rounded operands with
 * f32 accumulation differs from this emulation only in summation order. */
static inline float rtf32(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
  memcpy(&x, &u, 4);
  return x;
}

/* The same for a bf16 tensor-core GEMM: 8 significant bits, nearest, ties
 * to even (the conversion the bf16 backend stores with); a product of two
 * bf16 values is exact in f32 too. */
static inline float rbf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&x, &u, 4);
  return x;
}

/* The operand rounding of mode rnd: 0 none (f32), 1 tf32, 2 bf16. */
static inline float rop(float x, int rnd) {
  return rnd == 1 ? rtf32(x) : (rnd == 2 ? rbf16(x) : x);
}

/* net.rs:88-108.  rnd = 1 (2) rounds every GEMM operand to tf32 (bf16) where a
 * tensor-core backend stores it: the input row, the weights and each hidden
 * activation (after ELU); the output layer stays f32. */
static void mlp_forward_r(const int32_t *dims, int32_t n_dims, const float *params,
                          const float *x, float *acts, int rnd) {
  int32_t layers = n_dims - 1;
  memcpy(acts, x, sizeof(float) * (size_t)dims[0]);
  if (rnd)
    for (int32_t i = 0; i < dims[0]; ++i) acts[i] = rop(acts[i], rnd);
  const float *prev = acts;
  float *out = acts + dims[0];
  const float *p = params;
  for (int32_t l = 0; l < layers; ++l) {
    int32_t fan_in = dims[l], fan_out = dims[l + 1];
    const float *w = p;
    const float *b = p + (int64_t)fan_out * fan_in;
    int last = l == layers - 1;
    for (int32_t o = 0; o < fan_out; ++o) {
      float z = b[o];
      const float *row = w + (int64_t)o * fan_in;
      if (rnd)
        for (int32_t i = 0; i < fan_in; ++i) z += rop(row[i], rnd) * prev[i];
      else
        for (int32_t i = 0; i < fan_in; ++i) z += row[i] * prev[i];
      out[o] = last ? z : (rnd ? rop(elu(z), rnd) : elu(z));
    }
    p += (int64_t)fan_out * fan_in + fan_out;
    prev = out;
    out += fan_out;
  }
}

/* Mlp::forward (net.rs:88-108) with the reference's f32 arithmetic. */
void orc_mlp_forward(const int32_t *dims, int32_t n_dims, const float *params,
                     const float *x, float *acts) {
  mlp_forward_r(dims, n_dims, params, x, acts, 0);
}

/* net.rs:113-140.  rnd = 1: each layer's delta enters the weight- and
 * input-gradient products rounded to tf32 (as a tensor-core backend stores
 * it), the bias gradient sums the unrounded delta, the weights are read
 * rounded; acts are the (rounded) activations of mlp_forward_r. */
static void mlp_backward_r(const int32_t *dims, int32_t n_dims, const float *params,
                           const float *acts, const float *g_out, float *grads,
                           float *g_in, int rnd);

/* Mlp::backward (net.rs:113-140) with the reference's f32 arithmetic. */
void orc_mlp_backward(const int32_t *dims, int32_t n_dims, const float *params,
                      const float *acts, const float *g_out, float *grads,
                      float *g_in) {
  mlp_backward_r(dims, n_dims, params, acts, g_out, grads, g_in, 0);
}

static void mlp_backward_r(const int32_t *dims, int32_t n_dims, const float *params,
                           const float *acts, const float *g_out, float *grads,
                           float *g_in, int rnd) {
  int32_t layers = n_dims - 1;
  int32_t maxd = 0;
  for (int32_t l = 0; l < n_dims; ++l)
    if (dims[l] > maxd) maxd = dims[l];
  float *delta = (float *)malloc(sizeof(float) * (size_t)maxd);
  float *g_prev = (float *)malloc(sizeof(float) * (size_t)maxd);
  memcpy(delta, g_out, sizeof(float) * (size_t)dims[layers]);
  /* offsets of each layer's params and activations */
  int64_t poff[ORC_MAX_LAYERS + 1], aoff[ORC_MAX_LAYERS + 2];
  poff[0] = 0;
  aoff[0] = 0;
  for (int32_t l = 0; l < layers; ++l)
    poff[l + 1] = poff[l] + (int64_t)dims[l + 1] * dims[l] + dims[l + 1];
  for (int32_t l = 0; l < n_dims; ++l) aoff[l + 1] = aoff[l] + dims[l];
  for (int32_t l = layers - 1; l >= 0; --l) {
    int32_t fan_in = dims[l], fan_out = dims[l + 1];
    const float *prev = acts + aoff[l];
    const float *cur = acts + aoff[l + 1];
    const float *w = params + poff[l];
    float *gw = grads + poff[l];
    float *gb = gw + (int64_t)fan_out * fan_in;
    if (l != layers - 1)
      for (int32_t o = 0; o < fan_out; ++o) delta[o] *= elu_grad_from_act(cur[o]);
    for (int32_t i = 0; i < fan_in; ++i) g_prev[i] = 0.0f;
    for (int32_t o = 0; o < fan_out; ++o) {
      float d = delta[o];
      gb[o] += d;
      const float *wrow = w + (int64_t)o * fan_in;
      float *grow = gw + (int64_t)o * fan_in;
      if (rnd) {
        d = rop(d, rnd);
        for (int32_t i = 0; i < fan_in; ++i) {
          grow[i] += d * prev[i];
          g_prev[i] += d * rop(wrow[i], rnd);
        }
      } else {
        for (int32_t i = 0; i < fan_in; ++i) {
          grow[i] += d * prev[i];
          g_prev[i] += d * wrow[i];
        }
      }
    }
    float *t = delta;
    delta = g_prev;
    g_prev = t;
  }
  if (g_in) memcpy(g_in, delta, sizeof(float) * (size_t)dims[0]);
  free(delta);
  free(g_prev);
}

/* net.rs:181-194 (the w tensors then the b tensors; the f32 running sum is
 * order-dependent, so visit in that order when given an Mlp layout). */
float orc_grad_l2_norm(const float *g, int64_t n) {
  float s = 0.0f;
  for (int64_t i = 0; i < n; ++i) s += g[i] * g[i];
  return sqrtf(s);
}

static float mlp_grad_l2_norm(const int32_t *dims, int32_t n_dims,
                              const float *g) {
  float s = 0.0f;
  const float *p = g;
  for (int32_t l = 0; l + 1 < n_dims; ++l) {
    int64_t nw = (int64_t)dims[l + 1] * dims[l];
    for (int64_t i = 0; i < nw; ++i) s += p[i] * p[i];
    p += nw + dims[l + 1];
  }
  p = g;
  for (int32_t l = 0; l + 1 < n_dims; ++l) {
    int64_t nw = (int64_t)dims[l + 1] * dims[l];
    const float *b = p + nw;
    for (int32_t i = 0; i < dims[l + 1]; ++i) s += b[i] * b[i];
    p += nw + dims[l + 1];
  }
  return sqrtf(s);
}

/* net.rs:197-202 */
void orc_grad_clip(float *g, int64_t n, float max_norm) {
  float nrm = orc_grad_l2_norm(g, n);
  if (nrm > max_norm && nrm > 0.0f) {
    float s = max_norm / nrm;
    for (int64_t i = 0; i < n; ++i) g[i] *= s;
  }
}

static void mlp_grad_clip(const int32_t *dims, int32_t n_dims, float *g,
                          int64_t n, float max_norm) {
  float nrm = mlp_grad_l2_norm(dims, n_dims, g);
  if (nrm > max_norm && nrm > 0.0f) {
    float s = max_norm / nrm;
    for (int64_t i = 0; i < n; ++i) g[i] *= s;
  }
}

/* f32::powi with a runtime exponent lowers to a call of the runtime helper
 * that does binary exponentiation (square-and-multiply, result starting at
 * 1, reciprocal for negative exponents); restated here. */
float orc_powi(float a, int32_t b) {
  int recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

/* net.rs:233-251 */
void orc_adam_step(float *p, const float *g, float *m, float *v, int64_t n,
                   int32_t *t, float lr) {
  *t += 1;
  const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
  float bc1 = 1.0f - orc_powi(b1, *t);
  float bc2 = 1.0f - orc_powi(b2, *t);
  for (int64_t i = 0; i < n; ++i) {
    m[i] = b1 * m[i] + (1.0f - b1) * g[i];
    v[i] = b2 * v[i] + (1.0f - b2) * g[i] * g[i];
    p[i] -= lr * (m[i] / bc1) / (sqrtf(v[i] / bc2) + eps);
  }
}

/* ---------------------------------------------------------- Normalizer */

/* ppo.rs:198-205 */
void orc_norm_normalize(const float *mean, const float *m2, float count,
                        const float *x, int64_t dim, float *out) {
  for (int64_t i = 0; i < dim; ++i) {
    float var = m2[i] / count;
    if (var < 1e-8f) var = 1e-8f; /* f32::max(1e-8) */
    float y = (x[i] - mean[i]) / sqrtf(var);
    if (y < -5.0f) y = -5.0f; /* f32::clamp(-5, 5) */
    if (y > 5.0f) y = 5.0f;
    out[i] = y;
  }
}

/* ppo.rs:161-168 */
void orc_norm_update(float *mean, float *m2, float *count, const float *x,
                     int64_t dim) {
  *count += 1.0f;
  for (int64_t i = 0; i < dim; ++i) {
    float d = x[i] - mean[i];
    mean[i] += d / *count;
    m2[i] += d * (x[i] - mean[i]);
  }
}

/* ppo.rs:126-136: PendingNorm::push is the same recurrence as
 * Normalizer::update (orc_norm_update) on a state that starts at count 0,
 * mean 0, m2 0. */

/* ppo.rs:179-195: Normalizer::commit, the Chan et al. parallel-Welford
 * merge of a pending state into the live one, then the pending state is
 * reset.  A pending count of 0 leaves both untouched. */
void orc_norm_commit(float *mean, float *m2, float *count, float *p_mean,
                     float *p_m2, float *p_count, int64_t dim) {
  if (*p_count == 0.0f) return;
  float n1 = *count, n2 = *p_count;
  float tot = n1 + n2;
  for (int64_t i = 0; i < dim; ++i) {
    float d = p_mean[i] - mean[i];
    mean[i] += d * n2 / tot;
    m2[i] += p_m2[i] + d * d * n1 * n2 / tot;
  }
  *count = tot;
  *p_count = 0.0f;
  for (int64_t i = 0; i < dim; ++i) p_mean[i] = p_m2[i] = 0.0f;
}

/* ------------------------------------------------------- ActorCritic */

struct orc_ac {
  int32_t adims[ORC_MAX_LAYERS + 1], an;
  int32_t cdims[ORC_MAX_LAYERS + 1], cn;
  int32_t act_dim, obs_dim, cobs_dim;
  int64_t np_a, np_c, np; /* actor params, critic params, total (+log_std) */
  float *params;          /* actor | critic | log_std */
  float *m, *v;           /* Adam moments in the same layout */
  int32_t t_actor, t_critic, t_logstd;
  float *obs_mean, *obs_m2, obs_count;
  float *crit_mean, *crit_m2, crit_count;
  float lr;
  int32_t rnd; /* operand rounding emulated (mlp_forward_r): 1 tf32, 2 bf16 */
};

/* The ActorCritic state (ppo.rs:208-229, 235-266): two Mlps, log_std, one
 * Adam per net plus log_std's Adam state, both normalizers (identity
 * prior, ppo.rs:142-148). */
orc_ac *orc_ac_new(const int32_t *adims, int32_t an, const int32_t *cdims,
                   int32_t cn) {
  if (an < 2 || cn < 2 || an > ORC_MAX_LAYERS + 1 || cn > ORC_MAX_LAYERS + 1)
    return NULL;
  if (cdims[cn - 1] != 1) return NULL; /* ppo.rs:242-246 */
  orc_ac *ac = (orc_ac *)calloc(1, sizeof(orc_ac));
  memcpy(ac->adims, adims, sizeof(int32_t) * (size_t)an);
  memcpy(ac->cdims, cdims, sizeof(int32_t) * (size_t)cn);
  ac->an = an;
  ac->cn = cn;
  ac->act_dim = adims[an - 1];
  ac->obs_dim = adims[0];
  ac->cobs_dim = cdims[0];
  ac->np_a = orc_mlp_param_count(adims, an);
  ac->np_c = orc_mlp_param_count(cdims, cn);
  ac->np = ac->np_a + ac->np_c + ac->act_dim;
  ac->params = (float *)calloc((size_t)ac->np, sizeof(float));
  ac->m = (float *)calloc((size_t)ac->np, sizeof(float));
  ac->v = (float *)calloc((size_t)ac->np, sizeof(float));
  /* Normalizer::new (ppo.rs:142-148): mean 0, m2 1, count 1 */
  ac->obs_mean = (float *)calloc((size_t)ac->obs_dim, sizeof(float));
  ac->obs_m2 = (float *)malloc(sizeof(float) * (size_t)ac->obs_dim);
  for (int32_t i = 0; i < ac->obs_dim; ++i) ac->obs_m2[i] = 1.0f;
  ac->obs_count = 1.0f;
  ac->crit_mean = (float *)calloc((size_t)ac->cobs_dim, sizeof(float));
  ac->crit_m2 = (float *)malloc(sizeof(float) * (size_t)ac->cobs_dim);
  for (int32_t i = 0; i < ac->cobs_dim; ++i) ac->crit_m2[i] = 1.0f;
  ac->crit_count = 1.0f;
  ac->lr = 1e-3f;
  return ac;
}

void orc_ac_free(orc_ac *ac) {
  if (!ac) return;
  free(ac->params);
  free(ac->m);
  free(ac->v);
  free(ac->obs_mean);
  free(ac->obs_m2);
  free(ac->crit_mean);
  free(ac->crit_m2);
  free(ac);
}

/* ppo.rs:235-266 */
void orc_ac_init_reference(orc_ac *ac, float init_noise_std, float init_lr,
                           uint64_t *rng) {
  orc_mlp_init(ac->adims, ac->an, 0.01f, rng, ac->params);
  orc_mlp_init(ac->cdims, ac->cn, 1.0f, rng, ac->params + ac->np_a);
  float ls = logf(init_noise_std);
  for (int32_t k = 0; k < ac->act_dim; ++k)
    ac->params[ac->np_a + ac->np_c + k] = ls;
  memset(ac->m, 0, sizeof(float) * (size_t)ac->np);
  memset(ac->v, 0, sizeof(float) * (size_t)ac->np);
  ac->t_actor = ac->t_critic = ac->t_logstd = 0;
  ac->lr = init_lr;
}

int64_t orc_ac_param_count(const orc_ac *ac) { return ac->np; }

void orc_ac_set_params(orc_ac *ac, const float *flat) {
  memcpy(ac->params, flat, sizeof(float) * (size_t)ac->np);
}

void orc_ac_get_params(const orc_ac *ac, float *flat) {
  memcpy(flat, ac->params, sizeof(float) * (size_t)ac->np);
}

void orc_ac_set_normalizers(orc_ac *ac, const float *obs_mean,
                            const float *obs_m2, float obs_count,
                            const float *crit_mean, const float *crit_m2,
                            float crit_count) {
  memcpy(ac->obs_mean, obs_mean, sizeof(float) * (size_t)ac->obs_dim);
  memcpy(ac->obs_m2, obs_m2, sizeof(float) * (size_t)ac->obs_dim);
  ac->obs_count = obs_count;
  memcpy(ac->crit_mean, crit_mean, sizeof(float) * (size_t)ac->cobs_dim);
  memcpy(ac->crit_m2, crit_m2, sizeof(float) * (size_t)ac->cobs_dim);
  ac->crit_count = crit_count;
}

void orc_ac_set_lr(orc_ac *ac, float lr) { ac->lr = lr; }
void orc_ac_set_operand_rounding(orc_ac *ac, int32_t mode) {
  ac->rnd = (mode == 1 || mode == 2) ? mode : 0;
}
float orc_ac_get_lr(const orc_ac *ac) { return ac->lr; }

void orc_ac_get_adam(const orc_ac *ac, int32_t *t3, float *m, float *v) {
  t3[0] = ac->t_actor;
  t3[1] = ac->t_critic;
  t3[2] = ac->t_logstd;
  if (m) memcpy(m, ac->m, sizeof(float) * (size_t)ac->np);
  if (v) memcpy(v, ac->v, sizeof(float) * (size_t)ac->np);
}

void orc_ac_set_adam(orc_ac *ac, const int32_t *t3, const float *m,
                     const float *v) {
  ac->t_actor = t3[0];
  ac->t_critic = t3[1];
  ac->t_logstd = t3[2];
  if (m) memcpy(ac->m, m, sizeof(float) * (size_t)ac->np);
  if (v) memcpy(ac->v, v, sizeof(float) * (size_t)ac->np);
}

static const float *ac_log_std(const orc_ac *ac) {
  return ac->params + ac->np_a + ac->np_c;
}

/* ppo.rs:297-305 */
float orc_ac_logp(const orc_ac *ac, const float *action, const float *mean) {
  const float *ls = ac_log_std(ac);
  float lp = 0.0f;
  for (int32_t k = 0; k < ac->act_dim; ++k) {
    float sd = expf(ls[k]);
    float d = (action[k] - mean[k]) / sd;
    lp += -0.5f * d * d - ls[k] - LOG_SQRT_2PI;
  }
  return lp;
}

/* ppo.rs:308-311 */
float orc_ac_entropy(const orc_ac *ac) {
  const float *ls = ac_log_std(ac);
  float c = 0.5f + LOG_SQRT_2PI;
  float s = 0.0f;
  for (int32_t k = 0; k < ac->act_dim; ++k) s += ls[k] + c;
  return s;
}

/* ppo.rs:327-334 */
static float ac_kl(const orc_ac *ac, const float *mean_new,
                   const float *mean_old) {
  const float *ls = ac_log_std(ac);
  float kl = 0.0f;
  for (int32_t k = 0; k < ac->act_dim; ++k) {
    float inv = expf(-ls[k]);
    float d = (mean_new[k] - mean_old[k]) * inv;
    kl += 0.5f * (d * d);
  }
  return kl;
}

/* ActorCritic::mean / value (ppo.rs:282-294) for n rows. */
void orc_ac_forward(const orc_ac *ac, const float *obs, const float *cobs,
                    int64_t n, float *mean_out, float *value_out) {
  int64_t na = orc_mlp_act_count(ac->adims, ac->an);
  int64_t nc = orc_mlp_act_count(ac->cdims, ac->cn);
  float *xa = (float *)malloc(sizeof(float) * (size_t)ac->obs_dim);
  float *xc = (float *)malloc(sizeof(float) * (size_t)ac->cobs_dim);
  float *acts = (float *)malloc(sizeof(float) * (size_t)(na > nc ? na : nc));
  for (int64_t r = 0; r < n; ++r) {
    if (mean_out) {
      orc_norm_normalize(ac->obs_mean, ac->obs_m2, ac->obs_count,
                         obs + r * ac->obs_dim, ac->obs_dim, xa);
      mlp_forward_r(ac->adims, ac->an, ac->params, xa, acts, ac->rnd);
      memcpy(mean_out + r * ac->act_dim, acts + na - ac->act_dim,
             sizeof(float) * (size_t)ac->act_dim);
    }
    if (value_out) {
      orc_norm_normalize(ac->crit_mean, ac->crit_m2, ac->crit_count,
                         cobs + r * ac->cobs_dim, ac->cobs_dim, xc);
      mlp_forward_r(ac->cdims, ac->cn, ac->params + ac->np_a, xc, acts, ac->rnd);
      value_out[r] = acts[nc - 1];
    }
  }
  free(xa);
  free(xc);
  free(acts);
}

/* Per-sample body of the fold in ppo.rs:408-453; accumulates into acc,
 * laid out as [params (np) | surr | vloss | kl]. */
static void ac_sample_accumulate(const orc_ac *ac, const orc_batch *b,
                                 int64_t i, const orc_ppo_config *cfg,
                                 float scale, float *acc, float *work) {
  const int32_t A = ac->act_dim;
  int64_t na = orc_mlp_act_count(ac->adims, ac->an);
  int64_t nc = orc_mlp_act_count(ac->cdims, ac->cn);
  float *x = work;                                /* max(obs, cobs)       */
  float *acts = x + (ac->obs_dim > ac->cobs_dim ? ac->obs_dim : ac->cobs_dim);
  float *cacts = acts + na;
  float *g_mean = cacts + nc;
  const float *ls = ac_log_std(ac);
  float *g_actor = acc;
  float *g_critic = acc + ac->np_a;
  float *g_logstd = acc + ac->np_a + ac->np_c;
  float *sums = acc + ac->np;

  /* --- actor (normalized obs), ppo.rs:410-433 --- */
  orc_norm_normalize(ac->obs_mean, ac->obs_m2, ac->obs_count,
                     b->obs + i * ac->obs_dim, ac->obs_dim, x);
  mlp_forward_r(ac->adims, ac->an, ac->params, x, acts, ac->rnd);
  const float *mean = acts + na - A;
  const float *action = b->action + i * A;
  float logp = orc_ac_logp(ac, action, mean);
  float ratio = expf(logp - b->logp_old[i]);
  float a = b->adv[i];
  float lo = 1.0f - cfg->clip, hi = 1.0f + cfg->clip;
  float rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
  float s1 = ratio * a, s2 = rc * a;
  float surr = s1 < s2 ? s1 : s2; /* f32::min (no NaNs on this path) */
  sums[0] += surr * scale;
  int clipped = (a >= 0.0f && ratio > 1.0f + cfg->clip) ||
                (a < 0.0f && ratio < 1.0f - cfg->clip);
  for (int32_t k = 0; k < A; ++k) {
    float inv_var = expf(-2.0f * ls[k]);
    g_mean[k] = 0.0f;
    if (!clipped) {
      float d = action[k] - mean[k];
      g_mean[k] = -(a * ratio * d * inv_var) * scale;
      float dls = a * ratio * ((d * d) * inv_var - 1.0f);
      g_logstd[k] += -dls * scale;
    }
    g_logstd[k] += -cfg->entropy_coef * scale;
  }
  mlp_backward_r(ac->adims, ac->an, ac->params, acts, g_mean, g_actor, NULL, ac->rnd);

  /* --- critic (clipped value loss), ppo.rs:435-450 --- */
  orc_norm_normalize(ac->crit_mean, ac->crit_m2, ac->crit_count,
                     b->critic_obs + i * ac->cobs_dim, ac->cobs_dim, x);
  const float *cparams = ac->params + ac->np_a;
  mlp_forward_r(ac->cdims, ac->cn, cparams, x, cacts, ac->rnd);
  float v = cacts[nc - 1];
  float vo = b->value_old[i];
  float dvc = v - vo;
  if (dvc < -cfg->clip) dvc = -cfg->clip;
  if (dvc > cfg->clip) dvc = cfg->clip;
  float v_clipped = vo + dvc;
  float eu = v - b->ret[i], ec = v_clipped - b->ret[i];
  float l_unclipped = eu * eu, l_clipped = ec * ec;
  float vloss, dv;
  if (l_clipped > l_unclipped) {
    vloss = l_clipped;
    dv = 2.0f * ec;
  } else {
    vloss = l_unclipped;
    dv = 2.0f * eu;
  }
  sums[1] += vloss * scale;
  float gv = cfg->value_coef * dv * scale;
  mlp_backward_r(ac->cdims, ac->cn, cparams, cacts, &gv, g_critic, NULL, ac->rnd);

  /* ppo.rs:452 */
  sums[2] += ac_kl(ac, mean, b->mean_old + i * A) * scale;
}

static int64_t ac_work_floats(const orc_ac *ac) {
  return (ac->obs_dim > ac->cobs_dim ? ac->obs_dim : ac->cobs_dim) +
         orc_mlp_act_count(ac->adims, ac->an) +
         orc_mlp_act_count(ac->cdims, ac->cn) + ac->act_dim;
}

/* ppo.rs:388-462 (the fold/reduce).  With one thread the fold is
 * sequential in idx order, which is what the reference computes when rayon
 * runs on a single worker; with several threads each thread folds one
 * contiguous chunk and the chunk accumulators are added in chunk order
 * (MlpGrad::add, net.rs:153-164). */
void orc_ac_minibatch_grads(const orc_ac *ac, const orc_batch *b,
                            const int64_t *idx, int64_t n_idx,
                            const orc_ppo_config *cfg, float *grads,
                            float *sums3, int32_t n_threads) {
  const int64_t acc_n = ac->np + 3;
  float scale = 1.0f / (float)n_idx;
  if (n_threads < 1) n_threads = 1;
  float *accs = (float *)calloc((size_t)acc_n * (size_t)n_threads, sizeof(float));
  int64_t wn = ac_work_floats(ac);
#ifdef _OPENMP
#pragma omp parallel num_threads(n_threads)
#endif
  {
    int tid = 0, nt = 1;
#ifdef _OPENMP
    tid = omp_get_thread_num();
    nt = omp_get_num_threads();
#endif
    float *work = (float *)malloc(sizeof(float) * (size_t)wn);
    int64_t lo = n_idx * tid / nt, hi = n_idx * (tid + 1) / nt;
    float *acc = accs + (int64_t)tid * acc_n;
    for (int64_t s = lo; s < hi; ++s)
      ac_sample_accumulate(ac, b, idx[s], cfg, scale, acc, work);
    free(work);
  }
  /* reduce in chunk order */
  for (int64_t k = 0; k < acc_n; ++k) {
    float s = accs[k];
    for (int32_t t = 1; t < n_threads; ++t) s += accs[(int64_t)t * acc_n + k];
    if (k < ac->np)
      grads[k] = s;
    else
      sums3[k - ac->np] = s;
  }
  free(accs);
}

/* ppo.rs:496-510 */
static void ac_step_log_std(orc_ac *ac, const float *g) {
  ac->t_logstd += 1;
  const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
  float bc1 = 1.0f - orc_powi(b1, ac->t_logstd);
  float bc2 = 1.0f - orc_powi(b2, ac->t_logstd);
  float *ls = ac->params + ac->np_a + ac->np_c;
  float *m = ac->m + ac->np_a + ac->np_c;
  float *v = ac->v + ac->np_a + ac->np_c;
  for (int32_t k = 0; k < ac->act_dim; ++k) {
    m[k] = b1 * m[k] + (1.0f - b1) * g[k];
    v[k] = b2 * v[k] + (1.0f - b2) * g[k] * g[k];
    float step = ac->lr * (m[k] / bc1) / (sqrtf(v[k] / bc2) + eps);
    float y = ls[k] - step;
    if (y < -1.6f) y = -1.6f;
    if (y > 1.0f) y = 1.0f;
    ls[k] = y;
  }
}

/* ppo.rs:475-489 */
void orc_ac_apply(orc_ac *ac, const orc_ppo_config *cfg, const float *grads,
                  float kl) {
  if (cfg->adaptive_lr) {
    if (kl > cfg->desired_kl * 2.0f) {
      float l = ac->lr / 1.5f;
      ac->lr = l > cfg->lr_min ? l : cfg->lr_min;
    } else if (kl > 0.0f && kl < cfg->desired_kl / 2.0f) {
      float l = ac->lr * 1.5f;
      ac->lr = l < cfg->lr_max ? l : cfg->lr_max;
    }
  }
  float *g = (float *)malloc(sizeof(float) * (size_t)ac->np);
  memcpy(g, grads, sizeof(float) * (size_t)ac->np);
  mlp_grad_clip(ac->adims, ac->an, g, ac->np_a, cfg->max_grad_norm);
  mlp_grad_clip(ac->cdims, ac->cn, g + ac->np_a, ac->np_c, cfg->max_grad_norm);
  orc_adam_step(ac->params, g, ac->m, ac->v, ac->np_a, &ac->t_actor, ac->lr);
  orc_adam_step(ac->params + ac->np_a, g + ac->np_a, ac->m + ac->np_a,
                ac->v + ac->np_a, ac->np_c, &ac->t_critic, ac->lr);
  ac_step_log_std(ac, g + ac->np_a + ac->np_c);
  free(g);
}

/* ppo.rs:338-384 */
int orc_ac_update(orc_ac *ac, orc_batch *b, const orc_ppo_config *cfg,
                  orc_stats *out, int32_t n_threads) {
  int64_t n = b->n;
  if (cfg->minibatches < 1 || n < cfg->minibatches) return -1;
  /* advantage normalization, sequential f32 sums (ppo.rs:342-348) */
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum += b->adv[i];
  float mean = sum / (float)n;
  float sq = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float d = b->adv[i] - mean;
    sq += d * d;
  }
  float var = sq / (float)n;
  float sd = sqrtf(var);
  if (sd < 1e-6f) sd = 1e-6f;
  for (int64_t i = 0; i < n; ++i) b->adv[i] = (b->adv[i] - mean) / sd;

  int64_t mb = n / cfg->minibatches;
  orc_stats stats = {0};
  stats.lr = ac->lr;
  int64_t *order = (int64_t *)malloc(sizeof(int64_t) * (size_t)n);
  float *grads = (float *)malloc(sizeof(float) * (size_t)ac->np);
  for (int32_t e = 0; e < cfg->epochs; ++e) {
    orc_shuffle((uint64_t)ac->t_logstd + 1ull, n, order);
    orc_stats ep = {0};
    for (int32_t m = 0; m < cfg->minibatches; ++m) {
      float sums[3];
      orc_ac_minibatch_grads(ac, b, order + (int64_t)m * mb, mb, cfg, grads,
                             sums, n_threads);
      float entropy = orc_ac_entropy(ac);
      orc_ac_apply(ac, cfg, grads, sums[2]);
      ep.kl += sums[2];
      ep.surrogate += sums[0];
      ep.value_loss += sums[1];
      ep.entropy += entropy;
    }
    float inv = 1.0f / (float)cfg->minibatches;
    stats.kl = ep.kl * inv;
    stats.surrogate = ep.surrogate * inv;
    stats.value_loss = ep.value_loss * inv;
    stats.entropy = ep.entropy * inv;
    stats.lr = ac->lr;
  }
  free(order);
  free(grads);
  *out = stats;
  return 0;
}
