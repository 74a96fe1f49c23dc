// host_rng.cpp -- the reference's Lcg and epoch shuffle on the host.
//
// The minibatch permutation has to be bit-exact with zealot-rl, and it is
// data-independent (it depends only on the Adam step counter and n), so it
// is computed on the host while the GPU works and uploaded per epoch.
// Compiled with -ffp-contract=off so f32 arithmetic rounds like the
// reference Rust.
#include <math.h>
#include <stdint.h>

#include "../../include/zealot_rl.h"

namespace zrl {
void shuffle_i32(uint64_t seed, int64_t n, int32_t *order);
int64_t rank_slices(const int32_t *perm, int64_t n_global, int64_t n_local, int64_t row_offset,
                    int minibatches, int32_t *order, int64_t *counts, int64_t *offs);
}  // namespace zrl

extern "C" {

// rng.rs:14-16
uint64_t zrl_lcg_new(uint64_t seed) { return seed | 1ull; }

// rng.rs:19-26
float zrl_lcg_unit(uint64_t *s) {
  *s = *s * 6364136223846793005ull + 1442695040888963407ull;
  return (float)(*s >> 40) / (float)(1ull << 24);
}

// rng.rs:28-32 (TAU as f32 = 6.2831855)
float zrl_lcg_gauss(uint64_t *s) {
  float u1 = zrl_lcg_unit(s);
  if (u1 < 1e-7f) u1 = 1e-7f;
  // built with -ffp-contract=off: every f32 operation rounds separately
  float r = sqrtf(-2.0f * logf(u1));
  float ang = 6.28318548202514648f * zrl_lcg_unit(s);
  return r * cosf(ang);
}

int64_t zrl_rank_orders(uint64_t seed, int64_t n_global, int64_t n_local,
                        int64_t row_offset, int32_t minibatches, int32_t *order,
                        int64_t *counts) {
  if (n_global <= 0 || minibatches <= 0 || n_local < 0 || !order || !counts) return -1;
  int32_t *perm = new int32_t[(size_t)n_global];
  int64_t *offs = new int64_t[(size_t)minibatches];
  zrl::shuffle_i32(seed, n_global, perm);
  const int64_t n = zrl::rank_slices(perm, n_global, n_local, row_offset, minibatches, order,
                                     counts, offs);
  delete[] perm;
  delete[] offs;
  return n;
}

void zrl_shuffle(uint64_t seed, int64_t n, int64_t *order) {
  for (int64_t i = 0; i < n; ++i) order[i] = i;
  uint64_t sh = zrl_lcg_new(seed);
  for (int64_t i = n - 1; i >= 1; --i) {
    const float u = zrl_lcg_unit(&sh);
    const float prod = u * (float)(i + 1);
    int64_t j = (int64_t)prod;
    if (j > i) j = i;
    const int64_t t = order[i];
    order[i] = order[j];
    order[j] = t;
  }
}

}  // extern "C"

namespace zrl {

// ppo.rs:357-363 into 32-bit indices (the device gather format).
void shuffle_i32(uint64_t seed, int64_t n, int32_t *order) {
  for (int64_t i = 0; i < n; ++i) order[i] = (int32_t)i;
  uint64_t sh = zrl_lcg_new(seed);
  for (int64_t i = n - 1; i >= 1; --i) {
    const float u = zrl_lcg_unit(&sh);
    const float prod = u * (float)(i + 1);
    int64_t j = (int64_t)prod;
    if (j > i) j = i;
    const int32_t t = order[i];
    order[i] = order[j];
    order[j] = t;
  }
}

// One rank's share of an epoch (data parallel over rows): the global
// permutation perm[n_global] cut into `minibatches` slices of
// n_global / minibatches positions (ppo.rs:364-367); per slice, the
// positions whose sample lies in [row_offset, row_offset + n_local), as
// local rows, in permutation order.  Writes order[] (at most n_local
// entries) and the per-minibatch counts and offsets; returns the total.
int64_t rank_slices(const int32_t *perm, int64_t n_global, int64_t n_local, int64_t row_offset,
                    int minibatches, int32_t *order, int64_t *counts, int64_t *offs) {
  const int64_t mb = n_global / minibatches;
  int64_t n = 0;
  for (int m = 0; m < minibatches; ++m) {
    offs[m] = n;
    for (int64_t p = (int64_t)m * mb; p < (int64_t)(m + 1) * mb; ++p) {
      const int64_t r = perm[p] - row_offset;
      if (r >= 0 && r < n_local) order[n++] = (int32_t)r;
    }
    counts[m] = n - offs[m];
  }
  return n;
}

// Mlp::new (net.rs:61-78) into a flat [w_0, b_0, ...] buffer.
void mlp_init_reference(const int32_t *dims, int n_dims, float out_scale,
                        uint64_t *rng, float *params) {
  const int layers = n_dims - 1;
  float *p = params;
  for (int l = 0; l < layers; ++l) {
    const int fi = dims[l], fo = dims[l + 1];
    const bool last = l == layers - 1;
    const float s = sqrtf(1.0f / (float)fi) * (last ? out_scale : 1.0f);
    for (int64_t k = 0; k < (int64_t)fo * fi; ++k) p[k] = zrl_lcg_gauss(rng) * s;
    p += (int64_t)fo * fi;
    for (int o = 0; o < fo; ++o) p[o] = 0.0f;
    p += fo;
  }
}

}  // namespace zrl
