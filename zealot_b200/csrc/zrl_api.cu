// zrl_api.cu -- the C ABI of libzealot_rl.so: context, parameter layout and
// the PPO update orchestration (zealot-rl/src/ppo.rs:338-510).
//
// One update is one stream of kernels with no host synchronisation until
// the statistics are read back at the end: advantage moments -> per epoch
// (permutation upload, gather) -> per minibatch (forward x2 nets, loss,
// backward x2 nets, gradient reduce, [allreduce], pre-step, Adam).  The
// epoch permutations are computed on the host while the GPU runs the
// previous epoch.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>
#include <sys/resource.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <future>
#include <map>
#include <string>
#include <vector>

#include "zrl_comm.h"
#include "zrl_gemm.h"
#include "zrl_internal.h"

using namespace zrl;

namespace zrl {
struct StTensor {
  std::vector<int64_t> shape;
  std::vector<float> data;
};
std::vector<uint8_t> st_serialize(const std::map<std::string, StTensor> &ts);
bool st_parse(const uint8_t *buf, size_t len, std::map<std::string, StTensor> *out,
              std::string *err);
void shuffle_i32(uint64_t seed, int64_t n, int32_t *order);
int64_t rank_slices(const int32_t *perm, int64_t n_global, int64_t n_local, int64_t row_offset,
                    int minibatches, int32_t *order, int64_t *counts, int64_t *offs);
void mlp_init_reference(const int32_t *dims, int n_dims, float out_scale,
                        uint64_t *rng, float *params);
}

// The sample orders of one update (ppo.rs:360-366): per epoch the
// permutation of the global sample indices (Lcg seed = step + e * mbs + 1),
// cut into minibatches; with several ranks each rank keeps, per minibatch,
// the positions of the rows it holds, in order.  Each epoch's order is
// computed on its own worker thread into pinned memory, so the sequential
// shuffles run in parallel with each other and with the enqueueing of GPU
// work -- and, speculatively, during the previous update.
struct OrderPlan {
  int32_t *buf = nullptr;  // pinned [epochs][n_global]
  int64_t cap = 0;
  bool valid = false;
  uint64_t seed0 = 0;
  int64_t n_global = 0, n_local = 0, row_offset = 0;
  int epochs = 0, mbs = 0, world = 1;
  std::vector<int64_t> counts, offs, rows;  // [epochs * mbs], [epochs * mbs], [epochs]
  std::vector<std::vector<int32_t>> perm;   // [epochs][n_global] (several ranks), reused
  std::vector<std::future<void>> jobs;

  bool matches(uint64_t s0, int64_t ng, int64_t nl, int64_t ro, int ep, int mb, int w) const {
    return valid && seed0 == s0 && n_global == ng && n_local == nl && row_offset == ro &&
           epochs == ep && mbs == mb && world == w;
  }
  void wait_all() {
    for (auto &j : jobs)
      if (j.valid()) j.wait();
    jobs.clear();
  }
  void compute(int e) {
    const uint64_t seed = seed0 + (uint64_t)e * (uint64_t)mbs + 1ull;
    int32_t *ord = buf + (int64_t)e * n_global;
    const int64_t mb = n_global / mbs;
    if (world == 1) {
      zrl::shuffle_i32(seed, n_global, ord);
      rows[e] = mb * mbs;
      for (int m = 0; m < mbs; ++m) {
        counts[e * mbs + m] = mb;
        offs[e * mbs + m] = (int64_t)m * mb;
      }
      return;
    }
    std::vector<int32_t> &pe = perm[e];
    if ((int64_t)pe.size() < n_global) pe.resize(n_global);
    zrl::shuffle_i32(seed, n_global, pe.data());
    rows[e] = zrl::rank_slices(pe.data(), n_global, n_local, row_offset, mbs, ord,
                               counts.data() + (int64_t)e * mbs, offs.data() + (int64_t)e * mbs);
  }
};

// Several ranks: every epoch's orders computed on the device (the global
// permutation by zrl_shuffle_device's kernels, then the compaction of the
// rank's rows), the per-minibatch counts copied to pinned host memory.  The
// next update's orders are computed at the end of an update, so the stream
// synchronization that ends it also delivers the counts.
struct DevPlan {
  bool valid = false;
  // the counts have reached cnt_host: set by the successful synchronization
  // that ends an update (or the one right after queueing), cleared whenever
  // orders are queued, so a failed update's plan is queued again
  bool delivered = false;
  uint64_t seed0 = 0;
  int64_t n_global = 0, n_local = 0, row_offset = 0;
  int epochs = 0, mbs = 0;
  int32_t *order = nullptr;   // device [epochs][n_local]
  int32_t *scratch = nullptr; // device: perm [n_global] | shuffle [3 n_global] | block sums
  int64_t *cnt = nullptr;     // device [epochs][mbs + 1]
  int64_t *cnt_host = nullptr;  // pinned [epochs][mbs]
  int64_t cap_order = 0, cap_scratch = 0, cap_cnt = 0;
  bool matches(uint64_t s0, int64_t ng, int64_t nl, int64_t ro, int ep, int mb) const {
    return valid && delivered && seed0 == s0 && n_global == ng && n_local == nl &&
           row_offset == ro && epochs == ep && mbs == mb;
  }
};

struct zrl_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  zrl_model_config mcfg{};
  NetLayout net[2];
  int A = 0, Ap = 0;
  int64_t ls_off = 0;       // device offset of log_std
  int64_t dev_params = 0;   // padded parameter count (multiple of 32)
  int64_t grad_len = 0;     // dev_params + 32 (sums3 slot after the grads)
  int64_t flat_params = 0;
  int precision = ZRL_GEMM_TF32;

  float *P = nullptr, *G = nullptr, *M = nullptr, *V = nullptr;
  // tf32 mode: the weights rounded to tf32 (RN), the tensor-core GEMMs'
  // operand copy; P stays the fp32 master copy (bias reads, Adam)
  float *Ptc = nullptr;
  bool tc() const { return precision == ZRL_GEMM_TF32; }
  bool bf() const { return precision == ZRL_GEMM_BF16; }
  // the tensor-core path (tf32 or bf16 operands)
  bool tcore() const { return precision != ZRL_GEMM_FP32; }
  // storage of GEMM operands written by the non-GEMM kernels: 0 fp32, 1
  // tf32-rounded fp32, 2 bf16
  int opmode() const { return bf() ? 2 : (tc() ? 1 : 0); }
  int opbytes() const { return bf() ? 2 : 4; }
  // the weights the GEMMs read: a tf32-rounded or bf16 copy on the tensor
  // cores, the fp32 master otherwise
  const float *Wgemm() const { return tcore() ? Ptc : P; }
  // layer weights at element offset `off` of the GEMM copy
  const float *Wgemm_at(int64_t off) const {
    return reinterpret_cast<const float *>(reinterpret_cast<const char *>(Wgemm()) +
                                           off * (tcore() ? opbytes() : 4));
  }
  float *sums3 = nullptr;   // = G + dev_params
  DevState *st = nullptr;
  DevState *st_host = nullptr;  // pinned

  // normalizers (device) and host copies of the counts
  float *obs_mean = nullptr, *obs_m2 = nullptr, *obs_sd = nullptr;
  float *crit_mean = nullptr, *crit_m2 = nullptr, *crit_sd = nullptr;
  float obs_count = 1.0f, crit_count = 1.0f;
  // PendingNorm (ppo.rs:118-136) of each normalizer: folded by
  // zrl_pending_push, merged into the live statistics by zrl_commit_pending
  float *pend_obs_mean = nullptr, *pend_obs_m2 = nullptr;
  float *pend_crit_mean = nullptr, *pend_crit_m2 = nullptr;
  float pend_obs_count = 0.0f, pend_crit_count = 0.0f;
  float *welford_scratch = nullptr;  // chunk partials of the parallel fold
  int64_t welford_cap = 0;

  // batch capacity
  int64_t n_cap = 0;
  float *b_obs = nullptr, *b_cobs = nullptr, *b_act = nullptr, *b_mo = nullptr;
  float *b_lpo = nullptr, *b_vo = nullptr, *b_adv = nullptr, *b_ret = nullptr;
  float *r_rew = nullptr, *r_val = nullptr, *r_lv = nullptr;
  uint8_t *r_done = nullptr;
  int64_t env_cap = 0, r_cap = 0;
  // normalized observations of the whole batch, padded rows (computed once
  // per update; the epochs permute rows of these), and with the mirror
  // augmentation those of the mirrored rows (xm)
  float *n_xa = nullptr, *n_xc = nullptr, *n_xma = nullptr, *n_xmc = nullptr;
  int64_t n_xm_cap = 0;
  // L/R mirror augmentation (biped_train_gpu.rs:89-185, 988-1003): signed
  // permutations of the observation, critic observation and action spaces
  bool mirror = false;
  int32_t *mir_operm = nullptr, *mir_cperm = nullptr, *mir_aperm = nullptr;
  float *mir_osign = nullptr, *mir_csign = nullptr, *mir_asign = nullptr;
  float *e_xa = nullptr, *e_xc = nullptr, *e_act = nullptr, *e_mo = nullptr;
  float *e_lpo = nullptr, *e_vo = nullptr, *e_adv = nullptr, *e_ret = nullptr;
  int32_t *order_dev = nullptr;
  int32_t *order_pinned = nullptr;
  int64_t order_pinned_cap = 0;
  OrderPlan plan[2];  // this update's and (speculatively) the next one's
  DevPlan dplan;      // several ranks: orders on the device

  // minibatch activations / deltas
  int64_t mb_cap = 0;
  float *act[2][ZRL_MAX_LAYERS + 1] = {};
  float *dlt[2][ZRL_MAX_LAYERS] = {};

  // wgrad split-K partials
  float *wpart = nullptr;
  int64_t wpart_cap = 0;
  float *bpart = nullptr;
  int64_t bpart_cap = 0;

  ReduceScratch rs{};
  double *adv_part = nullptr;
  double *moments = nullptr;  // [2]
  int adv_part_cap = 0;

  int32_t t_logstd_host = 0;
  float lr_host = 1e-3f;
  int64_t launches = 0;

  bool profiling = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  float prof_gemm_ms = 0.0f, prof_update_ms = 0.0f;
  int64_t prof_gemm_launches = 0;
  // profiling: (site, start event, stop event, is a GEMM) per launch site
  // of the last update, and their per-site sums
  struct Span {
    const char *site;
    cudaEvent_t e0, e1;
    bool gemm;
  };
  std::vector<Span> spans;
  std::vector<std::pair<std::string, std::pair<float, int64_t>>> sites;

  Comm comm;
  GemmEngine gemm;
};

// ---------------------------------------------------------------- errors

#define CK(call)                                                          \
  do {                                                                    \
    cudaError_t e_ = (call);                                              \
    if (e_ != cudaSuccess) {                                              \
      ctx->err = std::string(#call) + ": " + cudaGetErrorString(e_);      \
      return ZRL_CUDA_ERROR;                                              \
    }                                                                     \
  } while (0)

#define CHECK_LAUNCH()                                                    \
  do {                                                                    \
    cudaError_t e_ = cudaGetLastError();                                  \
    if (e_ != cudaSuccess) {                                              \
      ctx->err = std::string("kernel launch: ") + cudaGetErrorString(e_); \
      return ZRL_CUDA_ERROR;                                              \
    }                                                                     \
  } while (0)

#define TRY(expr)                          \
  do {                                     \
    zrl_status s_ = (expr);                \
    if (s_ != ZRL_OK) return s_;           \
  } while (0)

static zrl_status bad(zrl_ctx *ctx, const char *msg) {
  if (ctx) ctx->err = msg;
  return ZRL_INVALID_ARG;
}


template <typename T>
static zrl_status dalloc(zrl_ctx *ctx, T **p, int64_t count) {
  if (*p) cudaFree(*p);
  *p = nullptr;
  if (count <= 0) return ZRL_OK;
  cudaError_t e = cudaMalloc((void **)p, sizeof(T) * (size_t)count);
  if (e != cudaSuccess) {
    ctx->err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
    *p = nullptr;
    return e == cudaErrorMemoryAllocation ? ZRL_OUT_OF_MEMORY : ZRL_CUDA_ERROR;
  }
  cudaMemsetAsync(*p, 0, sizeof(T) * (size_t)count, ctx->stream);
  return ZRL_OK;
}

// ---------------------------------------------------------------- layout

static void build_layout(zrl_ctx *ctx) {
  int64_t dev = 0, flat = 0;
  const int32_t *dims[2] = {ctx->mcfg.actor_dims, ctx->mcfg.critic_dims};
  const int nd[2] = {ctx->mcfg.n_actor_dims, ctx->mcfg.n_critic_dims};
  for (int k = 0; k < 2; ++k) {
    NetLayout &L = ctx->net[k];
    L.L = nd[k] - 1;
    for (int l = 0; l < nd[k]; ++l) {
      L.d[l] = dims[k][l];
      L.dp[l] = (int)pad_to(dims[k][l], kPad);
    }
    L.dev_begin = dev;
    L.flat_begin = flat;
    for (int l = 0; l < L.L; ++l) {
      L.w_off[l] = dev;
      dev += (int64_t)L.dp[l + 1] * L.dp[l];
      L.b_off[l] = dev;
      dev += L.dp[l + 1];
      L.fw_off[l] = flat;
      flat += (int64_t)L.d[l + 1] * L.d[l];
      L.fb_off[l] = flat;
      flat += L.d[l + 1];
    }
    L.dev_end = dev;
    L.flat_end = flat;
  }
  ctx->A = ctx->mcfg.actor_dims[ctx->mcfg.n_actor_dims - 1];
  ctx->Ap = (int)pad_to(ctx->A, kPad);
  ctx->ls_off = dev;
  dev += ctx->Ap;
  flat += ctx->A;
  ctx->dev_params = dev;
  ctx->grad_len = dev + 32;
  ctx->flat_params = flat;
}

// flat (save order) -> padded device layout, on the host
static void flat_to_padded(const zrl_ctx *ctx, const float *flat, float *pad) {
  memset(pad, 0, sizeof(float) * (size_t)ctx->dev_params);
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = 0; l < L.L; ++l) {
      for (int o = 0; o < L.d[l + 1]; ++o) {
        memcpy(pad + L.w_off[l] + (int64_t)o * L.dp[l],
               flat + L.fw_off[l] + (int64_t)o * L.d[l], sizeof(float) * L.d[l]);
        pad[L.b_off[l] + o] = flat[L.fb_off[l] + o];
      }
    }
  }
  memcpy(pad + ctx->ls_off, flat + ctx->net[1].flat_end, sizeof(float) * ctx->A);
}

static void padded_to_flat(const zrl_ctx *ctx, const float *pad, float *flat) {
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = 0; l < L.L; ++l) {
      for (int o = 0; o < L.d[l + 1]; ++o) {
        memcpy(flat + L.fw_off[l] + (int64_t)o * L.d[l],
               pad + L.w_off[l] + (int64_t)o * L.dp[l], sizeof(float) * L.d[l]);
        flat[L.fb_off[l] + o] = pad[L.b_off[l] + o];
      }
    }
  }
  memcpy(flat + ctx->net[1].flat_end, pad + ctx->ls_off, sizeof(float) * ctx->A);
}

// ------------------------------------------------------------- capacity

static zrl_status ensure_batch(zrl_ctx *ctx, int64_t n) {
  if (n <= ctx->n_cap) return ZRL_OK;
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  const int odp = ctx->net[0].dp[0], cdp = ctx->net[1].dp[0];
  const int A = ctx->A;
  TRY(dalloc(ctx, &ctx->b_obs, n * od));
  TRY(dalloc(ctx, &ctx->b_cobs, n * cd));
  TRY(dalloc(ctx, &ctx->b_act, n * A));
  TRY(dalloc(ctx, &ctx->b_mo, n * A));
  TRY(dalloc(ctx, &ctx->b_lpo, n));
  TRY(dalloc(ctx, &ctx->b_vo, n));
  TRY(dalloc(ctx, &ctx->b_adv, n));
  TRY(dalloc(ctx, &ctx->b_ret, n));
  TRY(dalloc(ctx, &ctx->n_xa, n * odp));
  TRY(dalloc(ctx, &ctx->n_xc, n * cdp));
  TRY(dalloc(ctx, &ctx->e_xa, n * odp));
  TRY(dalloc(ctx, &ctx->e_xc, n * cdp));
  TRY(dalloc(ctx, &ctx->e_act, n * A));
  TRY(dalloc(ctx, &ctx->e_mo, n * A));
  TRY(dalloc(ctx, &ctx->e_lpo, n));
  TRY(dalloc(ctx, &ctx->e_vo, n));
  TRY(dalloc(ctx, &ctx->e_adv, n));
  TRY(dalloc(ctx, &ctx->e_ret, n));
  TRY(dalloc(ctx, &ctx->order_dev, n));
  const int nb = adv_blocks(n) + gae_blocks(n) + 8;
  TRY(dalloc(ctx, &ctx->adv_part, nb));
  ctx->adv_part_cap = nb;
  ctx->n_cap = n;
  return ZRL_OK;
}

static zrl_status ensure_envs(zrl_ctx *ctx, int64_t n_envs, int64_t T) {
  TRY(ensure_batch(ctx, n_envs * T));
  // rewards/values/dones are sized by the batch capacity, bootstrap values
  // by the env count
  if (!ctx->r_rew || ctx->env_cap < n_envs || ctx->r_cap < ctx->n_cap) {
    TRY(dalloc(ctx, &ctx->r_rew, ctx->n_cap));
    TRY(dalloc(ctx, &ctx->r_val, ctx->n_cap));
    TRY(dalloc(ctx, &ctx->r_done, ctx->n_cap));
    TRY(dalloc(ctx, &ctx->r_lv, n_envs));
    ctx->env_cap = n_envs;
    ctx->r_cap = ctx->n_cap;
  }
  const int nb = gae_blocks(n_envs) + 8;
  if (nb > ctx->adv_part_cap) {
    TRY(dalloc(ctx, &ctx->adv_part, nb));
    ctx->adv_part_cap = nb;
  }
  return ZRL_OK;
}

static zrl_status ensure_pinned_orders(zrl_ctx *ctx, int64_t count) {
  if (count <= ctx->order_pinned_cap) return ZRL_OK;
  if (ctx->order_pinned) cudaFreeHost(ctx->order_pinned);
  ctx->order_pinned = nullptr;
  CK(cudaMallocHost((void **)&ctx->order_pinned, sizeof(int32_t) * (size_t)count));
  ctx->order_pinned_cap = count;
  return ZRL_OK;
}

static zrl_status start_plan(zrl_ctx *ctx, OrderPlan &P, uint64_t seed0, int64_t n_global,
                             int64_t n_local, int64_t row_offset, int epochs, int mbs) {
  P.wait_all();
  P.valid = false;
  const int64_t need = (int64_t)std::max(epochs, 1) * n_global;
  if (need > P.cap) {
    if (P.buf) cudaFreeHost(P.buf);
    P.buf = nullptr;
    P.cap = 0;
    CK(cudaMallocHost((void **)&P.buf, sizeof(int32_t) * (size_t)need));
    P.cap = need;
  }
  P.seed0 = seed0;
  P.n_global = n_global;
  P.n_local = n_local;
  P.row_offset = row_offset;
  P.epochs = epochs;
  P.mbs = mbs;
  P.world = ctx->comm.world;
  P.counts.assign((size_t)epochs * mbs, 0);
  P.offs.assign((size_t)epochs * mbs, 0);
  P.rows.assign((size_t)epochs, 0);
  if (P.world > 1 && (int)P.perm.size() < epochs) P.perm.resize(epochs);
  for (int e = 0; e < epochs; ++e)
    P.jobs.push_back(std::async(std::launch::async, [&P, e] {
      // below the submitting thread: with several ranks on one host these
      // workers (the global Fisher-Yates per rank and epoch) can outnumber
      // the cores, and a rank whose submitting thread waits for a core
      // delays every rank at the next allreduce
      setpriority(PRIO_PROCESS, (id_t)syscall(SYS_gettid), 10);
      P.compute(e);
    }));
  P.valid = true;
  return ZRL_OK;
}

constexpr int kMaxWSplit = 32;  // split-K partial rows the scratch holds per weight

static int wsplit_for(int64_t mb) {
  // enough row chunks to fill the machine on the small output tiles, each
  // chunk at least 512 rows
  int s = (int)std::min<int64_t>(32, std::max<int64_t>(1, mb / 512));
  return s;
}

static zrl_status ensure_mb(zrl_ctx *ctx, int64_t mb) {
  if (mb <= ctx->mb_cap) return ZRL_OK;
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = 1; l <= L.L; ++l) TRY(dalloc(ctx, &ctx->act[k][l], mb * L.dp[l]));
    for (int l = 0; l < L.L; ++l) TRY(dalloc(ctx, &ctx->dlt[k][l], mb * L.dp[l + 1]));
  }
  const int S = std::max(wsplit_for(mb), kMaxWSplit);
  int64_t wp = 0, bp = 0;
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = 0; l < L.L; ++l) {
      wp += (int64_t)S * L.dp[l + 1] * L.dp[l];
      // bias-gradient partials: S row chunks (CUDA-core colsum) or one row
      // per 32-row quarter of each 128-row block (tensor-core dgrad epilogue)
      // (or, for the fused head's level, one row per epilogue warp of each
      // CTA: at most 8 per 128-row block)
      bp += (int64_t)std::max<int64_t>(S, 8 * ((mb + 127) / 128)) * L.dp[l + 1];
    }
  }
  TRY(dalloc(ctx, &ctx->wpart, wp));
  TRY(dalloc(ctx, &ctx->bpart, bp));
  ctx->wpart_cap = wp;
  ctx->bpart_cap = bp;
  // loss-kernel partials: blocks of 8 warps, one sample per warp per pass
  ctx->mb_cap = mb;
  return ZRL_OK;
}

// ---------------------------------------------------------------- events

static cudaEvent_t next_event(zrl_ctx *ctx) {
  if (ctx->ev_used == ctx->ev_pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    ctx->ev_pool.push_back(e);
  }
  return ctx->ev_pool[ctx->ev_used++];
}

// Profiling (zrl_set_profiling): events on the stream around one launch
// site.  They separate the kernels they bracket (programmatic dependent
// launch cannot overlap across an event), so the profiled update runs a
// little slower than an unprofiled one; the per-site times say where the
// time goes.
struct ProfSpan {
  zrl_ctx *ctx;
  const char *site;
  cudaEvent_t e0 = nullptr;
  bool gemm;
  ProfSpan(zrl_ctx *c, const char *s, bool is_gemm = false) : ctx(c), site(s), gemm(is_gemm) {
    if (!ctx->profiling) return;
    e0 = next_event(ctx);
    cudaEventRecord(e0, ctx->stream);
  }
  ~ProfSpan() {
    if (!ctx->profiling || !e0) return;
    cudaEvent_t e1 = next_event(ctx);
    cudaEventRecord(e1, ctx->stream);
    ctx->spans.push_back(zrl_ctx::Span{site, e0, e1, gemm});
  }
};

// ------------------------------------------------------------------ GEMM

static zrl_status run_gemm(zrl_ctx *ctx, const GemmArgs &g, const char *site = "gemm") {
  ProfSpan ps(ctx, site, true);
  int launched = 0;
  zrl_status s = ctx->gemm.run(g, ctx->precision, ctx->stream, &launched, &ctx->err);
  if (s != ZRL_OK) return s;
  ctx->launches += launched;
  if (ctx->profiling) ctx->prof_gemm_launches += launched;
  CHECK_LAUNCH();
  return ZRL_OK;
}

static GemmArgs fwd_args(zrl_ctx *ctx, int k, int l, const float *in, int64_t rows) {
  const NetLayout &L = ctx->net[k];
  GemmArgs g{};
  g.M = (int)rows;
  g.N = L.dp[l + 1];
  g.K = L.dp[l];
  g.A = in;
  g.lda = L.dp[l];
  g.trans_a = false;
  g.B = ctx->Wgemm_at(L.w_off[l]);
  g.ldb = L.dp[l];
  g.trans_b = true;
  g.C = ctx->act[k][l + 1];
  g.ldc = L.dp[l + 1];
  g.epi = l < L.L - 1 ? EPI_BIAS_ELU : EPI_BIAS;
  // hidden activations feed later GEMMs: store them tf32-rounded; the
  // output layer (action mean / value) feeds the loss and stays fp32
  g.round_out = ctx->tc() && l < L.L - 1;
  g.bias = ctx->P + L.b_off[l];
  g.split_k = 1;
  return g;
}

static zrl_status run_group(zrl_ctx *ctx, const GemmArgs *gs, int n,
                            const char *site = "gemm") {
  if (n <= 0) return ZRL_OK;
  ProfSpan ps(ctx, site, true);
  int launched = 0;
  zrl_status s = ctx->gemm.run_group(gs, n, ctx->precision, ctx->stream, &launched, &ctx->err);
  if (s != ZRL_OK) return s;
  ctx->launches += launched;
  if (ctx->profiling) ctx->prof_gemm_launches += launched;
  CHECK_LAUNCH();
  return ZRL_OK;
}

// Forward of both nets over `rows` rows (inputs xa, xc with pitch dp[0]):
// layer l of the actor and of the critic run as one grouped launch when
// they share the epilogue.  Odd layers walk their tiles last to first, so
// each layer first reads the rows the layer before wrote last (still in
// L2).
static zrl_status forward_both(zrl_ctx *ctx, const float *xa, const float *xc, int64_t rows,
                               int layers = -1) {
  const int maxL = std::max(ctx->net[0].L, ctx->net[1].L);
  const int lim = layers < 0 ? maxL : std::min(layers, maxL);
  for (int l = 0; l < lim; ++l) {
    GemmArgs g[2];
    int n = 0;
    for (int k = 0; k < 2; ++k) {
      if (l >= ctx->net[k].L) continue;
      const float *in = l == 0 ? (k == 0 ? xa : xc) : ctx->act[k][l];
      g[n] = fwd_args(ctx, k, l, in, rows);
      g[n++].reverse_tiles = l & 1;
    }
    static const char *kFwd[ZRL_MAX_LAYERS] = {"gemm fwd L0", "gemm fwd L1", "gemm fwd L2",
                                                "gemm fwd L3", "gemm fwd L4", "gemm fwd L5",
                                                "gemm fwd L6", "gemm fwd L7"};
    const char *site = kFwd[std::min(l, ZRL_MAX_LAYERS - 1)];
    if (n == 2 && g[0].epi != g[1].epi) {
      TRY(run_group(ctx, &g[0], 1, site));
      TRY(run_group(ctx, &g[1], 1, site));
    } else {
      TRY(run_group(ctx, g, n, site));
    }
  }
  return ZRL_OK;
}

// Forward one net over `rows` rows of input x (pitch dp[0]); activations go
// to ctx->act[k][1..L].
static zrl_status forward_net(zrl_ctx *ctx, int k, const float *x, int64_t rows) {
  const NetLayout &L = ctx->net[k];
  for (int l = 0; l < L.L; ++l) {
    const GemmArgs g = fwd_args(ctx, k, l, l == 0 ? x : ctx->act[k][l], rows);
    TRY(run_group(ctx, &g, 1));
  }
  return ZRL_OK;
}

// Backward of both nets (net.rs:113-140 batched).  The dgrad chain runs
// level by level, actor and critic layer l in one launch, each with the
// ELU' epilogue; the weight gradients (split-K partials) of both nets run
// as grouped launches inside the chain.  Bias gradients are column sums of the
// deltas taken in fp32 where each delta is produced: the output layer's in
// the loss kernel, a hidden layer's in the epilogue of the tensor-core
// dgrad that produces it (a separate column-sum pass in the CUDA-core
// mode).
// top: the highest input-gradient level to run (maxL - 1 by default; the
// fused head computes that level itself and passes maxL - 2).
static zrl_status backward_both(zrl_ctx *ctx, const float *xa, const float *xc, int64_t rows,
                                float **wp, float **bp, ReduceSegs &segs, int top = -1) {
  const int m_tiles = (int)((rows + 127) / 128);
  const int maxL = std::max(ctx->net[0].L, ctx->net[1].L);
  if (top < 0) top = maxL - 1;
  const int S = wsplit_for(rows);
  // dW_l = delta_l^T a_l for every layer of both nets, split-K partials.
  // Tall ones (dp[l+1] >= 256 rows) go to CTA-pair tiles, the rest to
  // single-CTA tiles: a grouped launch (of at most 8) each, issued right
  // after the dgrad level that reads the same delta_l and a_l (level 1 for
  // layer 0), so those reads meet L2.  Each group takes the split counts
  // that fill the grid with the fewest partial rows (per problem: one with
  // half-width tiles takes half the splits, so the launch's tiles hold equal
  // work).
  GemmArgs tall[2 * ZRL_MAX_LAYERS], flat[2 * ZRL_MAX_LAYERS];
  int64_t tall_dst[2 * ZRL_MAX_LAYERS], flat_dst[2 * ZRL_MAX_LAYERS];
  int nt = 0, nf = 0, tall_lvl = 1, flat_lvl = 1;
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = L.L - 1; l >= 0; --l) {
      GemmArgs g{};
      g.M = L.dp[l + 1];
      g.N = L.dp[l];
      g.K = (int)rows;
      g.A = ctx->dlt[k][l];
      g.lda = L.dp[l + 1];
      g.trans_a = true;
      g.B = l == 0 ? (k == 0 ? xa : xc) : ctx->act[k][l];
      g.ldb = L.dp[l];
      g.trans_b = false;
      g.ldc = L.dp[l];
      g.epi = EPI_STORE;
      if (g.M >= 256) {
        tall_dst[nt] = L.w_off[l];
        tall[nt++] = g;
        tall_lvl = nt == 1 ? l : std::min(tall_lvl, l);
      } else {
        flat_dst[nf] = L.w_off[l];
        flat[nf++] = g;
        flat_lvl = nf == 1 ? l : std::min(flat_lvl, l);
      }
    }
  }
  auto place = [&](GemmArgs *w, const int64_t *dst, int nw) {
    int sp[2 * ZRL_MAX_LAYERS];
    for (int i0 = 0; i0 < nw; i0 += 8) {
      const int m = std::min(nw - i0, 8);
      if (ctx->gemm.split_for(w + i0, m, ctx->precision, kMaxWSplit, sp + i0, &ctx->err) < 1)
        for (int i = i0; i < i0 + m; ++i) sp[i] = S;
    }
    for (int i = 0; i < nw; ++i) {
      const int sg = sp[i];
      w[i].split_k = sg;
      w[i].C = *wp;
      const int64_t sz = (int64_t)w[i].M * w[i].N;
      segs.seg[segs.n++] = ReduceSeg{ctx->G + dst[i], *wp, sz, sg, sz};
      *wp += (int64_t)sg * sz;
    }
  };
  place(tall, tall_dst, nt);
  place(flat, flat_dst, nf);
  tall_lvl = std::max(tall_lvl, 1);
  flat_lvl = std::max(flat_lvl, 1);
  // successive launches alternate their tile order, starting opposite to
  // the forward's last layer (last to first when its index is odd)
  bool rev = !((maxL - 1) & 1);
  auto run_w = [&](GemmArgs *w, int nw, const char *site) -> zrl_status {
    for (int i = 0; i < nw; i += 8) {
      for (int j = i; j < std::min(nw, i + 8); ++j) w[j].reverse_tiles = rev;
      TRY(run_group(ctx, w + i, std::min(8, nw - i), site));
    }
    rev = !rev;
    return ZRL_OK;
  };
  for (int l = top; l >= 1; --l) {
    GemmArgs d[2];
    int n = 0;
    for (int k = 0; k < 2; ++k) {
      const NetLayout &L = ctx->net[k];
      if (l >= L.L) continue;
      // delta_{l-1} = (delta_l W_l) * elu'(a_l)
      GemmArgs &g = d[n++];
      g = GemmArgs{};
      g.M = (int)rows;
      g.N = L.dp[l];
      g.K = L.dp[l + 1];
      g.A = ctx->dlt[k][l];
      g.lda = L.dp[l + 1];
      g.trans_a = false;
      g.B = ctx->Wgemm_at(L.w_off[l]);
      g.round_out = ctx->tc();
      g.ldb = L.dp[l];
      g.trans_b = false;
      g.C = ctx->dlt[k][l - 1];
      g.ldc = L.dp[l];
      g.epi = EPI_ELU_GRAD;
      g.aux = ctx->act[k][l];
      g.ldaux = L.dp[l];
      g.split_k = 1;
      g.reverse_tiles = rev;
      if (ctx->tcore()) {
        // db_{l-1}: column sums of delta_{l-1} from the epilogue, one
        // partial row per 32-row quarter of each 128-row block
        g.colsum = *bp;
        ReduceSeg sb{ctx->G + L.b_off[l - 1], *bp, (int64_t)L.dp[l], 4 * m_tiles,
                     (int64_t)L.dp[l]};
        segs.seg[segs.n++] = sb;
        *bp += (int64_t)4 * m_tiles * L.dp[l];
      }
    }
    static const char *kDgrad[ZRL_MAX_LAYERS] = {"gemm dgrad L0", "gemm dgrad L1",
                                                  "gemm dgrad L2", "gemm dgrad L3",
                                                  "gemm dgrad L4", "gemm dgrad L5",
                                                  "gemm dgrad L6", "gemm dgrad L7"};
    TRY(run_group(ctx, d, n, kDgrad[std::min(l, ZRL_MAX_LAYERS - 1)]));
    rev = !rev;
    if (nf && flat_lvl == l) TRY(run_w(flat, nf, "gemm wgrad flat"));
    if (nt && tall_lvl == l) TRY(run_w(tall, nt, "gemm wgrad tall"));
  }
  if (!ctx->tcore()) {
    // db_l = column sums of delta_l for the hidden layers (CUDA-core mode)
    for (int k = 0; k < 2; ++k) {
      const NetLayout &L = ctx->net[k];
      for (int l = 0; l < L.L - 1; ++l) {
        launch_colsum(ctx->dlt[k][l], rows, L.dp[l + 1], L.dp[l + 1], *bp, S, ctx->stream);
        ctx->launches++;
        CHECK_LAUNCH();
        ReduceSeg sb{ctx->G + L.b_off[l], *bp, (int64_t)L.dp[l + 1], S, (int64_t)L.dp[l + 1]};
        segs.seg[segs.n++] = sb;
        *bp += (int64_t)S * L.dp[l + 1];
      }
    }
  }
  // single-layer nets: no dgrad chain, the weight gradients run here
  if (maxL == 1) {
    if (nt) TRY(run_w(tall, nt, "gemm wgrad tall"));
    if (nf) TRY(run_w(flat, nf, "gemm wgrad flat"));
  }
  return ZRL_OK;
}

struct MbView {
  const float *xa, *xc, *act, *mo, *lpo, *vo, *adv, *ret;
  int64_t rows;
};

// The fused output head (head_tc.cu) takes the tf32 update whenever both
// nets have the same depth (at least two layers), 32-wide (padded) output
// layers fed by hidden layers at most 128 wide, and at most 32 actions --
// the MLPs of the C1-C4 workloads.  Other shapes keep the separate
// output-layer forward, loss and input-gradient launches.
static bool head_applies(const zrl_ctx *ctx) {
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  if (!ctx->tc() || La.L != Lc.L || La.L < 2 || ctx->A > 32) return false;
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    if (L.dp[L.L] != 32 || L.dp[L.L - 1] > 128) return false;
  }
  return true;
}

// Adam over the whole parameter buffer (net.rs:233-251, ppo.rs:496-510).
static AdamArgs adam_args(zrl_ctx *ctx) {
  AdamArgs a{};
  a.p = ctx->P;
  a.m = ctx->M;
  a.v = ctx->V;
  a.g = ctx->G;
  a.n = ctx->dev_params;
  a.actor_end = ctx->net[0].dev_end;
  a.critic_end = ctx->net[1].dev_end;
  a.st = ctx->st;
  a.p_round = ctx->tcore() ? ctx->Ptc : nullptr;
  a.p_mode = ctx->opmode();
  return a;
}

// The segment reduce of a minibatch's partial sums.  One rank (`fuse` set):
// with the pre-step in the same launch (*fused = 1), and where the device
// takes a cooperative launch with the Adam step as well (*fused = 2).
static zrl_status reduce_grads(zrl_ctx *ctx, const ReduceSegs &segs, const PrestepArgs *fuse,
                               int *fused) {
  if (fuse && ctx->gemm.err_dev && ctx->rs.coop_blocks >= 0) {
    ProfSpan ps(ctx, "segment reduce + pre-step + adam");
    if (launch_reduce_step(segs, *fuse, adam_args(ctx), ctx->rs, ctx->gemm.err_dev,
                           ctx->stream)) {
      if (fused) *fused = 2;
      ctx->launches++;
      CHECK_LAUNCH();
      return ZRL_OK;
    }
  }
  ProfSpan ps(ctx, "segment reduce (+pre-step)");
  const int f = launch_reduce_segments(segs, ctx->stream, fuse, &ctx->rs);
  if (fused) *fused = f;
  ctx->launches++;
  CHECK_LAUNCH();
  return ZRL_OK;
}

// minibatch_grads with the fused head: forward of the hidden layers, the
// head (output layers, losses, last hidden layer's delta), then the rest of
// the backward and the segment reduce.
static zrl_status minibatch_grads_head(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                                       const MbView &v, float scale, const PrestepArgs *fuse,
                                       int *fused) {
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  const int L = La.L;
  TRY(forward_both(ctx, v.xa, v.xc, v.rows, L - 1));
  HeadArgs h{};
  float *wp = ctx->wpart, *bp = ctx->bpart;
  const int hr = head_partial_rows(v.rows);
  if (hr > ctx->rs.max_blocks || kHeadWidth > ctx->rs.fwidth) return bad(ctx, "head scratch too small");
  ReduceSegs segs{};
  for (int k = 0; k < 2; ++k) {
    const NetLayout &N = ctx->net[k];
    HeadNet &n = h.net[k];
    n.a = ctx->act[k][L - 1];
    n.k = N.dp[L - 1];
    n.w = ctx->Wgemm_at(N.w_off[L - 1]);
    n.b = ctx->P + N.b_off[L - 1];
    n.d_out = ctx->dlt[k][L - 1];
    n.d_in = ctx->dlt[k][L - 2];
    n.colsum = bp;
    segs.seg[segs.n++] = ReduceSeg{ctx->G + N.b_off[L - 2], bp, (int64_t)n.k, hr, (int64_t)n.k};
    bp += (int64_t)hr * n.k;
  }
  h.action = v.act;
  h.mean_old = v.mo;
  h.logp_old = v.lpo;
  h.value_old = v.vo;
  h.adv = v.adv;
  h.ret = v.ret;
  h.log_std = ctx->P + ctx->ls_off;
  h.A = ctx->A;
  h.rows = v.rows;
  h.scale = scale;
  h.clip = cfg->clip;
  h.entropy_coef = cfg->entropy_coef;
  h.value_coef = cfg->value_coef;
  h.part = ctx->rs.fpart;
  h.err = ctx->gemm.err_dev;
  {
    // its partial rows: log_std gradient, output-layer bias gradients of
    // both nets, statistic sums (the loss kernel's layout, 32-wide)
    const int64_t w = kHeadWidth;
    float *fp = ctx->rs.fpart;
    segs.seg[segs.n++] = ReduceSeg{ctx->G + ctx->ls_off, fp, 32, hr, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->G + La.b_off[L - 1], fp + 32, 32, hr, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->sums3, fp + 64, 4, hr, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->G + Lc.b_off[L - 1], fp + 68, 32, hr, w};
  }
  {
    ProfSpan ps(ctx, "head (fwd out + loss + dgrad out)", true);
    TRY(ctx->gemm.head(h, ctx->stream, &ctx->err));
    ctx->launches++;
    CHECK_LAUNCH();
  }
  TRY(backward_both(ctx, v.xa, v.xc, v.rows, &wp, &bp, segs, L - 2));
  return reduce_grads(ctx, segs, fuse, fused);
}

// Gradient accumulation of one minibatch (ppo.rs:388-462): leaves the
// summed gradient in G (padded layout, log_std included) and the three
// statistic sums in sums3.
static zrl_status minibatch_grads(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                                  const MbView &v, float scale,
                                  const PrestepArgs *fuse = nullptr, int *fused = nullptr) {
  if (fused) *fused = 0;
  TRY(ensure_mb(ctx, std::max<int64_t>(v.rows, 1)));
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  if (v.rows > 0 && head_applies(ctx)) return minibatch_grads_head(ctx, cfg, v, scale, fuse, fused);
  if (v.rows > 0) TRY(forward_both(ctx, v.xa, v.xc, v.rows));
  LossArgs la{};
  la.mean = ctx->act[0][La.L];
  la.value = ctx->act[1][Lc.L];
  la.Ap = La.dp[La.L];
  la.cp = Lc.dp[Lc.L];
  la.action = v.act;
  la.mean_old = v.mo;
  la.logp_old = v.lpo;
  la.value_old = v.vo;
  la.adv = v.adv;
  la.ret = v.ret;
  la.log_std = ctx->P + ctx->ls_off;
  la.A = ctx->A;
  la.mb = v.rows;
  la.scale = scale;
  la.clip = cfg->clip;
  la.entropy_coef = cfg->entropy_coef;
  la.value_coef = cfg->value_coef;
  la.out_mode = ctx->opmode();
  la.d_actor = ctx->dlt[0][La.L - 1];
  la.d_critic = ctx->dlt[1][Lc.L - 1];
  la.part = ctx->rs.fpart;
  la.width = 2 * la.Ap + 4 + la.cp;
  if (v.rows <= 0) {
    // a rank with no rows this minibatch contributes zeros (the entropy
    // term of the log_std gradient is per sample, so zero as well)
    CK(cudaMemsetAsync(ctx->G, 0, sizeof(float) * ctx->grad_len, ctx->stream));
    return ZRL_OK;
  }
  const int lb = loss_blocks(la);
  if (la.width > ctx->rs.fwidth || lb > ctx->rs.max_blocks) return bad(ctx, "loss scratch too small");
  {
    ProfSpan ps(ctx, "loss");
    launch_loss(la, ctx->stream);
    ctx->launches++;
    CHECK_LAUNCH();
  }
  float *wp = ctx->wpart, *bp = ctx->bpart;
  ReduceSegs segs{};
  {
    // the loss kernel's block rows: log_std gradient, output-layer bias
    // gradients of both nets, statistic sums
    const int64_t w = la.width;
    float *fp = ctx->rs.fpart;
    segs.seg[segs.n++] = ReduceSeg{ctx->G + ctx->ls_off, fp, (int64_t)la.Ap, lb, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->G + La.b_off[La.L - 1], fp + la.Ap, (int64_t)la.Ap, lb, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->sums3, fp + 2 * la.Ap, 4, lb, w};
    segs.seg[segs.n++] = ReduceSeg{ctx->G + Lc.b_off[Lc.L - 1], fp + 2 * la.Ap + 4, (int64_t)la.cp, lb, w};
  }
  TRY(backward_both(ctx, v.xa, v.xc, v.rows, &wp, &bp, segs));
  return reduce_grads(ctx, segs, fuse, fused);
}

static zrl_status allreduce_grads(zrl_ctx *ctx) {
  if (ctx->comm.world <= 1) return ZRL_OK;
  ProfSpan ps(ctx, "allreduce");
  return ctx->comm.allreduce_f32(ctx->G, ctx->grad_len, ctx->stream, &ctx->err);
}

// Stepping half of minibatch_step (ppo.rs:475-489).
static PrestepArgs prestep_args(zrl_ctx *ctx, const zrl_ppo_config *cfg, int minibatches,
                                bool last_of_epoch, bool count_stats) {
  PrestepArgs p{};
  p.grads = ctx->G;
  p.actor_begin = ctx->net[0].dev_begin;
  p.actor_end = ctx->net[0].dev_end;
  p.critic_begin = ctx->net[1].dev_begin;
  p.critic_end = ctx->net[1].dev_end;
  p.log_std = ctx->P + ctx->ls_off;
  p.A = ctx->A;
  p.sums3 = ctx->sums3;
  p.max_grad_norm = cfg->max_grad_norm;
  p.desired_kl = cfg->desired_kl;
  p.lr_min = cfg->lr_min;
  p.lr_max = cfg->lr_max;
  p.adaptive_lr = cfg->adaptive_lr;
  p.minibatches = minibatches;
  p.last_of_epoch = last_of_epoch;
  p.count_stats = count_stats;
  p.st = ctx->st;
  return p;
}

// done: what the segment reduce already ran (one rank): 1 the pre-step,
// 2 the pre-step and Adam.
static zrl_status step(zrl_ctx *ctx, const zrl_ppo_config *cfg, int minibatches,
                       bool last_of_epoch, bool count_stats, int done = 0) {
  if (done >= 2) return ZRL_OK;
  const PrestepArgs p = prestep_args(ctx, cfg, minibatches, last_of_epoch, count_stats);
  if (!done && ctx->gemm.err_dev && ctx->rs.coop_blocks >= 0) {
    // the pre-step and Adam in one cooperative launch
    ProfSpan ps(ctx, "pre-step + adam");
    const ReduceSegs none{};
    if (launch_reduce_step(none, p, adam_args(ctx), ctx->rs, ctx->gemm.err_dev, ctx->stream,
                           true)) {
      ctx->launches++;
      CHECK_LAUNCH();
      return ZRL_OK;
    }
  }
  if (!done) {
    ProfSpan ps(ctx, "pre-step");
    launch_prestep(p, ctx->rs, ctx->stream);
    ctx->launches++;
    CHECK_LAUNCH();
  }
  ProfSpan ps(ctx, "adam");
  launch_adam(adam_args(ctx), ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  return ZRL_OK;
}

// Advantage mean and population sd over the (global) batch, ppo.rs:342-345.
static zrl_status adv_moments(zrl_ctx *ctx, const float *adv, int64_t n,
                              int64_t n_global, bool partials_ready,
                              int partial_blocks) {
  ProfSpan ps(ctx, "advantage moments");
  int nb = partial_blocks;
  if (!partials_ready) {
    nb = adv_blocks(n);
    if (n > 0) {
      launch_adv_sum(adv, n, ctx->adv_part, nb, ctx->stream);
      ctx->launches++;
    } else {
      CK(cudaMemsetAsync(ctx->adv_part, 0, sizeof(double), ctx->stream));
      nb = 1;
    }
  }
  launch_reduce_moment(ctx->adv_part, nb, ctx->moments, 0, ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  if (ctx->comm.world > 1)
    TRY(ctx->comm.allreduce_f64(ctx->moments, 1, ctx->stream, &ctx->err));
  int nb2 = adv_blocks(std::max<int64_t>(n, 1));
  if (n > 0) {
    launch_adv_sqdev(adv, n, ctx->moments, n_global, ctx->adv_part, nb2, ctx->stream);
    ctx->launches++;
  } else {
    CK(cudaMemsetAsync(ctx->adv_part, 0, sizeof(double), ctx->stream));
    nb2 = 1;
  }
  launch_reduce_moment(ctx->adv_part, nb2, ctx->moments, 1, ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  if (ctx->comm.world > 1)
    TRY(ctx->comm.allreduce_f64(ctx->moments + 1, 1, ctx->stream, &ctx->err));
  launch_adv_finalize(ctx->moments, n_global, ctx->st, ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  return ZRL_OK;
}

struct DevBatch {
  const float *obs, *cobs, *act, *mo, *lpo, *vo, *adv, *ret;
};

// Normalized, clamped (tf32-rounded in the tensor-core modes) observation
// rows of the whole batch, padded to the GEMM pitch: Normalizer::normalize
// (ppo.rs:196-205) applied once per update, since the normalizers do not
// change during it -- and, with the mirror augmentation, the same of the
// mirrored rows (the normalizers apply to the mirrored raw observations,
// as the reference normalizes mirror_sample's output).
static zrl_status normalize_batch(zrl_ctx *ctx, const float *obs, const float *cobs,
                                  int64_t n) {
  if (n <= 0) return ZRL_OK;
  ProfSpan ps(ctx, "normalize");
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  launch_normalize_rows(obs, n, La.d[0], La.dp[0], ctx->obs_mean, ctx->obs_sd, ctx->n_xa,
                        ctx->opmode(), ctx->stream);
  launch_normalize_rows(cobs, n, Lc.d[0], Lc.dp[0], ctx->crit_mean, ctx->crit_sd, ctx->n_xc,
                        ctx->opmode(), ctx->stream);
  ctx->launches += 2;
  if (ctx->mirror) {
    if (n > ctx->n_xm_cap) {
      TRY(dalloc(ctx, &ctx->n_xma, n * La.dp[0]));
      TRY(dalloc(ctx, &ctx->n_xmc, n * Lc.dp[0]));
      ctx->n_xm_cap = n;
    }
    launch_normalize_rows(obs, n, La.d[0], La.dp[0], ctx->obs_mean, ctx->obs_sd, ctx->n_xma,
                          ctx->opmode(), ctx->stream, ctx->mir_operm, ctx->mir_osign);
    launch_normalize_rows(cobs, n, Lc.d[0], Lc.dp[0], ctx->crit_mean, ctx->crit_sd, ctx->n_xmc,
                          ctx->opmode(), ctx->stream, ctx->mir_cperm, ctx->mir_csign);
    ctx->launches += 2;
  }
  CHECK_LAUNCH();
  return ZRL_OK;
}

// The epoch gather's arguments (virtual rows [0, n_base) are the mirrored
// copies of the n_base base rows when n_base > 0).
static GatherArgs gather_args(zrl_ctx *ctx, const DevBatch &d, int64_t n_base) {
  GatherArgs g{};
  g.order = ctx->order_dev;
  g.xn_a = ctx->n_xa;
  g.xn_c = ctx->n_xc;
  g.action = d.act;
  g.mean_old = d.mo;
  g.logp_old = d.lpo;
  g.value_old = d.vo;
  g.adv = d.adv;
  g.ret = d.ret;
  g.A = ctx->A;
  g.odp = ctx->net[0].dp[0];
  g.cdp = ctx->net[1].dp[0];
  g.x_bytes = ctx->opbytes();
  g.st = ctx->st;
  g.x_a = ctx->e_xa;
  g.x_c = ctx->e_xc;
  g.g_action = ctx->e_act;
  g.g_mean_old = ctx->e_mo;
  g.g_logp_old = ctx->e_lpo;
  g.g_value_old = ctx->e_vo;
  g.g_adv = ctx->e_adv;
  g.g_ret = ctx->e_ret;
  if (n_base > 0) {
    g.n_base = n_base;
    g.xm_a = ctx->n_xma;
    g.xm_c = ctx->n_xmc;
    g.m_aperm = ctx->mir_aperm;
    g.m_asign = ctx->mir_asign;
  }
  return g;
}

static MbView epoch_view(zrl_ctx *ctx, int64_t off, int64_t rows) {
  MbView v{};
  // (bf16 rows are half as many bytes: offsets in the operand element size)
  v.xa = reinterpret_cast<const float *>(reinterpret_cast<const char *>(ctx->e_xa) +
                                         off * ctx->net[0].dp[0] * ctx->opbytes());
  v.xc = reinterpret_cast<const float *>(reinterpret_cast<const char *>(ctx->e_xc) +
                                         off * ctx->net[1].dp[0] * ctx->opbytes());
  v.act = ctx->e_act + off * ctx->A;
  v.mo = ctx->e_mo + off * ctx->A;
  v.lpo = ctx->e_lpo + off;
  v.vo = ctx->e_vo + off;
  v.adv = ctx->e_adv + off;
  v.ret = ctx->e_ret + off;
  v.rows = rows;
  return v;
}

static zrl_status stage_batch(zrl_ctx *ctx, const zrl_batch *b, DevBatch *d,
                              bool need_adv_ret) {
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0], A = ctx->A;
  const int64_t n = b->n;
  TRY(ensure_batch(ctx, n));  // the epoch buffers, for device batches too
  if (b->on_device) {
    *d = DevBatch{b->obs, b->critic_obs, b->action, b->mean_old,
                  b->logp_old, b->value_old, b->adv, b->ret};
    return ZRL_OK;
  }
  auto up = [&](float *dst, const float *src, int64_t cnt) -> zrl_status {
    if (cnt <= 0) return ZRL_OK;
    CK(cudaMemcpyAsync(dst, src, sizeof(float) * cnt, cudaMemcpyHostToDevice,
                       ctx->stream));
    return ZRL_OK;
  };
  TRY(up(ctx->b_obs, b->obs, n * od));
  TRY(up(ctx->b_cobs, b->critic_obs, n * cd));
  TRY(up(ctx->b_act, b->action, n * A));
  TRY(up(ctx->b_mo, b->mean_old, n * A));
  TRY(up(ctx->b_lpo, b->logp_old, n));
  TRY(up(ctx->b_vo, b->value_old, n));
  if (need_adv_ret) {
    TRY(up(ctx->b_adv, b->adv, n));
    TRY(up(ctx->b_ret, b->ret, n));
  }
  *d = DevBatch{ctx->b_obs, ctx->b_cobs, ctx->b_act, ctx->b_mo,
                ctx->b_lpo, ctx->b_vo, ctx->b_adv, ctx->b_ret};
  return ZRL_OK;
}

static zrl_status check_cfg(zrl_ctx *ctx, const zrl_ppo_config *cfg) {
  if (!cfg) return bad(ctx, "null config");
  if (cfg->epochs < 0 || cfg->minibatches < 1)
    return bad(ctx, "epochs must be >= 0 and minibatches >= 1");
  return ZRL_OK;
}

// The epoch/minibatch loop of ActorCritic::update (ppo.rs:350-383) once the
// batch is on the device and the advantage moments are in ctx->st.
// Queue the device orders of an update (several ranks) on the context's
// stream: per epoch the global permutation (seed0 + e * mbs + 1, the seed
// order of ppo.rs:360) and this rank's compacted rows; the counts reach
// cnt_host once the stream has passed this point.
static zrl_status queue_device_orders(zrl_ctx *ctx, uint64_t seed0, int64_t n_global,
                                      int64_t n_local, int64_t row_offset, int epochs,
                                      int mbs) {
  DevPlan &D = ctx->dplan;
  D.valid = false;
  D.delivered = false;
  if (n_global > INT32_MAX) return bad(ctx, "n_global beyond 2^31 samples");
  const int64_t nblk = (n_global + 1023) / 1024;
  const int64_t need_order = std::max<int64_t>((int64_t)epochs * n_local, 1);
  const int64_t need_scratch = 4 * n_global + nblk + 1;
  const int64_t need_cnt = (int64_t)epochs * (mbs + 1);
  if (need_order > D.cap_order) {
    if (D.order) cudaFree(D.order);
    D.order = nullptr;
    D.cap_order = 0;
    CK(cudaMalloc((void **)&D.order, sizeof(int32_t) * (size_t)need_order));
    D.cap_order = need_order;
  }
  if (need_scratch > D.cap_scratch) {
    if (D.scratch) cudaFree(D.scratch);
    D.scratch = nullptr;
    D.cap_scratch = 0;
    CK(cudaMalloc((void **)&D.scratch, sizeof(int32_t) * (size_t)need_scratch));
    D.cap_scratch = need_scratch;
  }
  if (need_cnt > D.cap_cnt) {
    if (D.cnt) cudaFree(D.cnt);
    if (D.cnt_host) cudaFreeHost(D.cnt_host);
    D.cnt = nullptr;
    D.cnt_host = nullptr;
    D.cap_cnt = 0;
    CK(cudaMalloc((void **)&D.cnt, sizeof(int64_t) * (size_t)need_cnt));
    CK(cudaMallocHost((void **)&D.cnt_host, sizeof(int64_t) * (size_t)need_cnt));
    D.cap_cnt = need_cnt;
  }
  int32_t *perm = D.scratch, *sh = D.scratch + n_global, *bs = D.scratch + 4 * n_global;
  for (int e = 0; e < epochs; ++e) {
    const uint64_t seed = seed0 + (uint64_t)e * (uint64_t)mbs + 1ull;
    launch_shuffle_device(seed, (int32_t)n_global, perm, sh, ctx->stream);
    launch_rank_orders(perm, n_global, n_local, row_offset, mbs, D.order + e * n_local,
                       D.cnt + (int64_t)e * (mbs + 1), bs, ctx->stream);
    ctx->launches += 6;
    CK(cudaMemcpyAsync(D.cnt_host + (int64_t)e * mbs, D.cnt + (int64_t)e * (mbs + 1),
                       sizeof(int64_t) * mbs, cudaMemcpyDeviceToHost, ctx->stream));
  }
  CHECK_LAUNCH();
  D.seed0 = seed0;
  D.n_global = n_global;
  D.n_local = n_local;
  D.row_offset = row_offset;
  D.epochs = epochs;
  D.mbs = mbs;
  D.valid = true;
  return ZRL_OK;
}

static zrl_status run_epochs(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                             const DevBatch &d, int64_t n_local,
                             int64_t n_global, int64_t row_offset) {
  // the mirror augmentation doubles the batch: virtual rows [0, n) are the
  // mirrored copies, [n, 2n) the samples themselves (biped_train_gpu.rs:
  // 988-1003 puts the mirrored copies first); one rank only
  const int64_t n_base = ctx->mirror ? n_local : 0;
  if (ctx->mirror) {
    n_local *= 2;
    n_global *= 2;
  }
  const int64_t mbs = cfg->minibatches;
  const int64_t mb = n_global / mbs;
  const float scale = 1.0f / (float)mb;
  // stats start as {0, 0, 0, 0, lr} (ppo.rs:351-354); lr and the Adam
  // steps stay on the device
  CK(cudaMemsetAsync(&ctx->st->ep_acc, 0, sizeof(float) * 4, ctx->stream));
  CK(cudaMemsetAsync(&ctx->st->stats, 0, sizeof(float) * 4, ctx->stream));
  CK(cudaMemcpyAsync(&ctx->st->stats[4], &ctx->st->lr, sizeof(float),
                     cudaMemcpyDeviceToDevice, ctx->stream));
  const bool multi = ctx->comm.world > 1;
  TRY(ensure_mb(ctx, std::max<int64_t>(multi ? std::min<int64_t>(mb, n_local) : mb, 1)));
  const uint64_t seed0 = (uint64_t)ctx->t_logstd_host;
  const int epochs = std::max(cfg->epochs, 0);
  OrderPlan *P = nullptr;
  // several ranks: per epoch and minibatch, the rank's row count and offset
  std::vector<int64_t> dcounts, doffs, drows;
  if (multi) {
    // this update's orders on the device: queued at the end of the previous
    // update (its closing synchronization delivered the counts), or now
    DevPlan &D = ctx->dplan;
    if (epochs > 0 && !D.matches(seed0, n_global, n_local, row_offset, epochs, (int)mbs)) {
      TRY(queue_device_orders(ctx, seed0, n_global, n_local, row_offset, epochs, (int)mbs));
      // the counts size this update's launches; the stream also holds the
      // advantage-moment allreduces, so the wait is the bounded one that
      // aborts the communicator when a peer is gone
      TRY(ctx->comm.wait(ctx->stream, &ctx->err));
      D.delivered = true;
    }
    dcounts.assign(D.cnt_host, D.cnt_host + (int64_t)epochs * mbs);
    doffs.assign((size_t)epochs * mbs, 0);
    drows.assign((size_t)epochs, 0);
    for (int e = 0; e < epochs; ++e) {
      int64_t o = 0;
      for (int64_t m = 0; m < mbs; ++m) {
        doffs[e * mbs + m] = o;
        o += dcounts[e * mbs + m];
      }
      drows[e] = o;
    }
  } else {
    // this update's orders: a speculative plan that matches, or start now
    for (auto &q : ctx->plan)
      if (q.matches(seed0, n_global, n_local, row_offset, epochs, (int)mbs, ctx->comm.world))
        P = &q;
    if (!P) {
      P = &ctx->plan[0];
      TRY(start_plan(ctx, *P, seed0, n_global, n_local, row_offset, epochs, (int)mbs));
    }
    // the next update's orders, computed while this one runs (in the other
    // plan, which the previous update -- complete by now -- used); started
    // here so the workers have the whole update to finish
    OrderPlan &Q = P == &ctx->plan[0] ? ctx->plan[1] : ctx->plan[0];
    if (epochs > 0)
      TRY(start_plan(ctx, Q, seed0 + (uint64_t)epochs * (uint64_t)mbs, n_global, n_local,
                     row_offset, epochs, (int)mbs));
  }
  if (epochs > 0) TRY(normalize_batch(ctx, d.obs, d.cobs, n_base > 0 ? n_base : n_local));
  for (int e = 0; e < epochs; ++e) {
    if (!multi) P->jobs[e].wait();
    const int64_t n_rows = multi ? drows[e] : P->rows[e];
    if (n_rows > 0) {
      GatherArgs g = gather_args(ctx, d, n_base);
      if (multi) {
        g.order = ctx->dplan.order + (int64_t)e * n_local;
      } else {
        CK(cudaMemcpyAsync(ctx->order_dev, P->buf + (int64_t)e * n_global,
                           sizeof(int32_t) * n_rows, cudaMemcpyHostToDevice, ctx->stream));
      }
      g.n_used = n_rows;
      g.apply_adv_norm = 1;
      ProfSpan ps(ctx, "gather");
      launch_gather(g, ctx->stream);
      ctx->launches++;
      CHECK_LAUNCH();
    }
    for (int64_t m = 0; m < mbs; ++m) {
      const int64_t off = multi ? doffs[e * mbs + m] : P->offs[e * mbs + m];
      const int64_t cnt = multi ? dcounts[e * mbs + m] : P->counts[e * mbs + m];
      MbView v = epoch_view(ctx, off, cnt);
      // one rank: the segment reduce also runs the pre-step
      const PrestepArgs pf = prestep_args(ctx, cfg, (int)mbs, m == mbs - 1, true);
      int fused = 0;
      TRY(minibatch_grads(ctx, cfg, v, scale, multi ? nullptr : &pf, &fused));
      TRY(allreduce_grads(ctx));
      TRY(step(ctx, cfg, (int)mbs, m == mbs - 1, true, fused));
    }
  }
  // several ranks: the next update's orders, behind this update's work (its
  // gathers have read the current ones)
  if (multi && epochs > 0)
    TRY(queue_device_orders(ctx, seed0 + (uint64_t)epochs * (uint64_t)mbs, n_global, n_local,
                            row_offset, epochs, (int)mbs));
  ctx->t_logstd_host += cfg->epochs * (int32_t)mbs;
  return ZRL_OK;
}

// A device wait that ran out leaves a code in the engine's device flag
// (tensor-core pipelines: 1 producer, 2 MMA issuer, 3 epilogue, ...;
// 8 the grid barrier of the fused reduce + step).
static zrl_status check_device_error(zrl_ctx *ctx) {
  if (!ctx->gemm.err_dev) return ZRL_OK;
  int code = 0;
  CK(cudaMemcpy(&code, ctx->gemm.err_dev, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    cudaMemset(ctx->gemm.err_dev, 0, sizeof(int));
    ctx->err = code == 8 ? std::string("reduce + step grid barrier wait timed out (code 8)")
                         : "tensor-core GEMM pipeline wait timed out (code " +
                               std::to_string(code) + ")";
    return ZRL_TIMEOUT;
  }
  return ZRL_OK;
}

static zrl_status finish_update(zrl_ctx *ctx, zrl_stats *out) {
  CK(cudaMemcpyAsync(ctx->st_host, ctx->st, sizeof(DevState),
                     cudaMemcpyDeviceToHost, ctx->stream));
  if (ctx->comm.world > 1)
    TRY(ctx->comm.wait(ctx->stream, &ctx->err));  // bounded: peers may be gone
  CK(cudaStreamSynchronize(ctx->stream));
  TRY(check_device_error(ctx));
  // the next update's device orders (queued at the end of this one) and
  // their counts are now in place; after a device error they are queued
  // again by the next update
  if (ctx->dplan.valid) ctx->dplan.delivered = true;
  ctx->lr_host = ctx->st_host->lr;
  if (ctx->st_host->t[2] != ctx->t_logstd_host) {
    ctx->err = "internal: Adam step counter mismatch";
    return ZRL_CUDA_ERROR;
  }
  if (out) {
    out->kl = ctx->st_host->stats[0];
    out->surrogate = ctx->st_host->stats[1];
    out->value_loss = ctx->st_host->stats[2];
    out->entropy = ctx->st_host->stats[3];
    out->lr = ctx->st_host->stats[4];
  }
  return ZRL_OK;
}

static zrl_status refresh_norm(zrl_ctx *ctx) {
  launch_norm_prepare(ctx->obs_m2, ctx->obs_count, ctx->net[0].d[0], ctx->obs_sd,
                      ctx->stream);
  launch_norm_prepare(ctx->crit_m2, ctx->crit_count, ctx->net[1].d[0], ctx->crit_sd,
                      ctx->stream);
  ctx->launches += 2;
  CHECK_LAUNCH();
  return ZRL_OK;
}

static void prof_begin(zrl_ctx *ctx, cudaEvent_t *u0) {
  if (!ctx->profiling) return;
  ctx->ev_used = 0;
  ctx->prof_gemm_launches = 0;
  ctx->spans.clear();
  *u0 = next_event(ctx);
  cudaEventRecord(*u0, ctx->stream);
}

static zrl_status prof_end(zrl_ctx *ctx, cudaEvent_t u0) {
  if (!ctx->profiling) return ZRL_OK;
  cudaEvent_t u1 = next_event(ctx);
  cudaEventRecord(u1, ctx->stream);
  // with several ranks the stream holds collectives: wait with the bounded
  // poll that aborts the communicator when a peer is gone
  if (ctx->comm.world > 1)
    TRY(ctx->comm.wait(ctx->stream, &ctx->err));
  else
    CK(cudaEventSynchronize(u1));
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, u0, u1);
  ctx->prof_update_ms = ms;
  float g = 0.0f;
  ctx->sites.clear();
  for (const auto &sp : ctx->spans) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, sp.e0, sp.e1);
    if (sp.gemm) g += t;
    bool found = false;
    for (auto &kv : ctx->sites)
      if (kv.first == sp.site) {
        kv.second.first += t;
        kv.second.second += 1;
        found = true;
        break;
      }
    if (!found) ctx->sites.push_back({std::string(sp.site), {t, 1}});
  }
  ctx->prof_gemm_ms = g;
  return ZRL_OK;
}

// =================================================================== ABI

extern "C" {

int32_t zrl_abi_version(void) { return ZRL_ABI_VERSION; }

zrl_status zrl_nccl_unique_id(uint8_t *out) {
  if (!out) return ZRL_INVALID_ARG;
  std::string err;
  zrl_status s = nccl_unique_id(out, &err);
  if (s != ZRL_OK) fprintf(stderr, "zrl_nccl_unique_id: %s\n", err.c_str());
  return s;
}

const char *zrl_last_error(const zrl_ctx *ctx) {
  return ctx ? ctx->err.c_str() : "null context";
}

zrl_status zrl_create(const zrl_model_config *cfg, int device,
                      const zrl_comm *comm, zrl_ctx **out) {
  if (!cfg || !out) return ZRL_INVALID_ARG;
  *out = nullptr;
  if (cfg->n_actor_dims < 2 || cfg->n_critic_dims < 2 ||
      cfg->n_actor_dims > ZRL_MAX_LAYERS + 1 || cfg->n_critic_dims > ZRL_MAX_LAYERS + 1)
    return ZRL_INVALID_ARG;
  if (cfg->critic_dims[cfg->n_critic_dims - 1] != 1) return ZRL_INVALID_ARG;
  for (int i = 0; i < cfg->n_actor_dims; ++i)
    if (cfg->actor_dims[i] < 1) return ZRL_INVALID_ARG;
  for (int i = 0; i < cfg->n_critic_dims; ++i)
    if (cfg->critic_dims[i] < 1) return ZRL_INVALID_ARG;
  if (cfg->actor_dims[cfg->n_actor_dims - 1] > 128) return ZRL_NOT_SUPPORTED;
  // the epoch gather normalizes observation rows up to 256 wide per warp
  if (cfg->actor_dims[0] > 256 || cfg->critic_dims[0] > 256) return ZRL_NOT_SUPPORTED;
  if (cfg->precision < 0 || cfg->precision > 2) return ZRL_INVALID_ARG;
  zrl_ctx *ctx = new zrl_ctx();
  ctx->mcfg = *cfg;
  ctx->device = device;
  ctx->precision = cfg->precision;
  auto fail = [&](zrl_status s) {
    zrl_destroy(ctx);
    return s;
  };
  if (cudaSetDevice(device) != cudaSuccess) return fail(ZRL_CUDA_ERROR);
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess)
    return fail(ZRL_CUDA_ERROR);
  build_layout(ctx);
  zrl_status s;
  if ((s = dalloc(ctx, &ctx->P, ctx->dev_params)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->G, ctx->grad_len)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->M, ctx->dev_params)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->V, ctx->dev_params)) != ZRL_OK) return fail(s);
  if (ctx->tcore() && (s = dalloc(ctx, &ctx->Ptc, ctx->dev_params)) != ZRL_OK) return fail(s);
  ctx->sums3 = ctx->G + ctx->dev_params;
  if ((s = dalloc(ctx, &ctx->st, 1)) != ZRL_OK) return fail(s);
  if (cudaMallocHost((void **)&ctx->st_host, sizeof(DevState)) != cudaSuccess)
    return fail(ZRL_CUDA_ERROR);
  memset(ctx->st_host, 0, sizeof(DevState));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  if ((s = dalloc(ctx, &ctx->obs_mean, od)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->obs_m2, od)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->obs_sd, od)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->crit_mean, cd)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->crit_m2, cd)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->crit_sd, cd)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->pend_obs_mean, od)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->pend_obs_m2, od)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->pend_crit_mean, cd)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->pend_crit_m2, cd)) != ZRL_OK) return fail(s);
  if ((s = dalloc(ctx, &ctx->moments, 2)) != ZRL_OK) return fail(s);
  ctx->rs.max_blocks = 148 * 16;
  ctx->rs.fwidth = 2 * 128 + 4 + 128;  // loss-kernel partial row for Ap, cp <= 128
  if ((s = dalloc(ctx, &ctx->rs.fpart, (int64_t)ctx->rs.max_blocks * ctx->rs.fwidth)) != ZRL_OK)
    return fail(s);
  if ((s = dalloc(ctx, &ctx->rs.dpart, (int64_t)ctx->rs.max_blocks * 2)) != ZRL_OK)
    return fail(s);
  if ((s = dalloc(ctx, &ctx->rs.ticket, 4)) != ZRL_OK) return fail(s);
  ctx->rs.bar_count = 0;
  ctx->rs.coop_blocks = 0;
  // identity normalizers (Normalizer::new: mean 0, m2 1, count 1)
  {
    std::vector<float> ones(std::max(od, cd), 1.0f);
    cudaMemcpyAsync(ctx->obs_m2, ones.data(), sizeof(float) * od,
                    cudaMemcpyHostToDevice, ctx->stream);
    cudaMemcpyAsync(ctx->crit_m2, ones.data(), sizeof(float) * cd,
                    cudaMemcpyHostToDevice, ctx->stream);
    if (refresh_norm(ctx) != ZRL_OK) return fail(ZRL_CUDA_ERROR);
  }
  ctx->st_host->lr = ctx->lr_host;
  cudaMemcpyAsync(ctx->st, ctx->st_host, sizeof(DevState), cudaMemcpyHostToDevice,
                  ctx->stream);
  if ((s = ctx->gemm.init(ctx->device, &ctx->err)) != ZRL_OK) return fail(s);
  if (comm && comm->world_size > 1) {
    if ((s = ctx->comm.init(*comm, &ctx->err)) != ZRL_OK) return fail(s);
  }
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return fail(ZRL_CUDA_ERROR);
  *out = ctx;
  return ZRL_OK;
}

zrl_status zrl_destroy(zrl_ctx *ctx) {
  if (!ctx) return ZRL_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  ctx->comm.destroy();
  ctx->gemm.destroy();
  float **bufs[] = {&ctx->P, &ctx->G, &ctx->M, &ctx->V, &ctx->obs_mean, &ctx->obs_m2,
                    &ctx->obs_sd, &ctx->crit_mean, &ctx->crit_m2, &ctx->crit_sd,
                    &ctx->b_obs, &ctx->b_cobs, &ctx->b_act, &ctx->b_mo, &ctx->b_lpo,
                    &ctx->b_vo, &ctx->b_adv, &ctx->b_ret, &ctx->r_rew, &ctx->r_val,
                    &ctx->r_lv, &ctx->n_xa, &ctx->n_xc, &ctx->n_xma, &ctx->n_xmc, &ctx->e_xa, &ctx->e_xc, &ctx->e_act, &ctx->e_mo,
                    &ctx->e_lpo, &ctx->e_vo, &ctx->e_adv, &ctx->e_ret, &ctx->wpart,
                    &ctx->bpart, &ctx->rs.fpart, &ctx->Ptc, &ctx->pend_obs_mean,
                    &ctx->pend_obs_m2, &ctx->pend_crit_mean, &ctx->pend_crit_m2,
                    &ctx->welford_scratch, &ctx->mir_osign, &ctx->mir_csign,
                    &ctx->mir_asign};
  for (float **b : bufs)
    if (*b) cudaFree(*b);
  for (int k = 0; k < 2; ++k) {
    for (auto *p : ctx->act[k])
      if (p) cudaFree(p);
    for (auto *p : ctx->dlt[k])
      if (p) cudaFree(p);
  }
  if (ctx->r_done) cudaFree(ctx->r_done);
  if (ctx->order_dev) cudaFree(ctx->order_dev);
  for (int32_t *m : {ctx->mir_operm, ctx->mir_cperm, ctx->mir_aperm})
    if (m) cudaFree(m);
  if (ctx->st) cudaFree(ctx->st);
  if (ctx->adv_part) cudaFree(ctx->adv_part);
  if (ctx->moments) cudaFree(ctx->moments);
  if (ctx->rs.dpart) cudaFree(ctx->rs.dpart);
  if (ctx->rs.ticket) cudaFree(ctx->rs.ticket);
  if (ctx->st_host) cudaFreeHost(ctx->st_host);
  if (ctx->dplan.order) cudaFree(ctx->dplan.order);
  if (ctx->dplan.scratch) cudaFree(ctx->dplan.scratch);
  if (ctx->dplan.cnt) cudaFree(ctx->dplan.cnt);
  if (ctx->dplan.cnt_host) cudaFreeHost(ctx->dplan.cnt_host);
  for (auto &q : ctx->plan) {
    q.wait_all();
    if (q.buf) cudaFreeHost(q.buf);
    q.buf = nullptr;
  }
  if (ctx->order_pinned) cudaFreeHost(ctx->order_pinned);
  for (auto e : ctx->ev_pool) cudaEventDestroy(e);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return ZRL_OK;
}

zrl_status zrl_synchronize(zrl_ctx *ctx) {
  if (!ctx) return ZRL_INVALID_ARG;
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

void *zrl_stream(zrl_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int64_t zrl_param_count(const zrl_ctx *ctx) { return ctx ? ctx->flat_params : 0; }

int64_t zrl_kernel_launches(const zrl_ctx *ctx) { return ctx ? ctx->launches : 0; }

static zrl_status reset_adam(zrl_ctx *ctx) {
  CK(cudaMemsetAsync(ctx->M, 0, sizeof(float) * ctx->dev_params, ctx->stream));
  CK(cudaMemsetAsync(ctx->V, 0, sizeof(float) * ctx->dev_params, ctx->stream));
  CK(cudaMemsetAsync(ctx->st->t, 0, sizeof(int32_t) * 3, ctx->stream));
  ctx->t_logstd_host = 0;
  return ZRL_OK;
}

zrl_status zrl_set_params(zrl_ctx *ctx, const float *flat, int64_t count) {
  if (!ctx || !flat) return ZRL_INVALID_ARG;
  if (count != ctx->flat_params) return bad(ctx, "parameter count mismatch");
  CK(cudaSetDevice(ctx->device));
  std::vector<float> pad(ctx->dev_params);
  flat_to_padded(ctx, flat, pad.data());
  CK(cudaMemcpyAsync(ctx->P, pad.data(), sizeof(float) * ctx->dev_params,
                     cudaMemcpyHostToDevice, ctx->stream));
  if (ctx->tcore()) {
    launch_round_copy(ctx->P, ctx->Ptc, ctx->dev_params, ctx->opmode(), ctx->stream);
    ctx->launches++;
    CHECK_LAUNCH();
  }
  TRY(reset_adam(ctx));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_get_params(zrl_ctx *ctx, float *flat, int64_t count) {
  if (!ctx || !flat) return ZRL_INVALID_ARG;
  if (count != ctx->flat_params) return bad(ctx, "parameter count mismatch");
  CK(cudaSetDevice(ctx->device));
  std::vector<float> pad(ctx->dev_params);
  CK(cudaMemcpyAsync(pad.data(), ctx->P, sizeof(float) * ctx->dev_params,
                     cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  padded_to_flat(ctx, pad.data(), flat);
  return ZRL_OK;
}

zrl_status zrl_init_reference(zrl_ctx *ctx, float init_noise_std, float init_lr,
                              uint64_t *lcg_state) {
  if (!ctx || !lcg_state || !(init_noise_std > 0.0f)) return ZRL_INVALID_ARG;
  std::vector<float> flat(ctx->flat_params);
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  mlp_init_reference(ctx->mcfg.actor_dims, ctx->mcfg.n_actor_dims, 0.01f, lcg_state,
                     flat.data() + La.flat_begin);
  mlp_init_reference(ctx->mcfg.critic_dims, ctx->mcfg.n_critic_dims, 1.0f, lcg_state,
                     flat.data() + Lc.flat_begin);
  const float ls = logf(init_noise_std);
  for (int k = 0; k < ctx->A; ++k) flat[Lc.flat_end + k] = ls;
  TRY(zrl_set_params(ctx, flat.data(), ctx->flat_params));
  return zrl_set_lr(ctx, init_lr);
}

zrl_status zrl_set_adam_state(zrl_ctx *ctx, const int32_t *t3, const float *m,
                              const float *v, int64_t count) {
  if (!ctx || !t3) return ZRL_INVALID_ARG;
  if ((m || v) && count != ctx->flat_params) return bad(ctx, "parameter count mismatch");
  CK(cudaSetDevice(ctx->device));
  std::vector<float> pad(ctx->dev_params);
  if (m) {
    flat_to_padded(ctx, m, pad.data());
    CK(cudaMemcpy(ctx->M, pad.data(), sizeof(float) * ctx->dev_params,
                  cudaMemcpyHostToDevice));
  }
  if (v) {
    flat_to_padded(ctx, v, pad.data());
    CK(cudaMemcpy(ctx->V, pad.data(), sizeof(float) * ctx->dev_params,
                  cudaMemcpyHostToDevice));
  }
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMemcpy(ctx->st->t, t3, sizeof(int32_t) * 3, cudaMemcpyHostToDevice));
  ctx->t_logstd_host = t3[2];
  return ZRL_OK;
}

zrl_status zrl_get_adam_state(zrl_ctx *ctx, int32_t *t3, float *m, float *v,
                              int64_t count) {
  if (!ctx || !t3) return ZRL_INVALID_ARG;
  if ((m || v) && count != ctx->flat_params) return bad(ctx, "parameter count mismatch");
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMemcpy(t3, ctx->st->t, sizeof(int32_t) * 3, cudaMemcpyDeviceToHost));
  std::vector<float> pad(ctx->dev_params);
  if (m) {
    CK(cudaMemcpy(pad.data(), ctx->M, sizeof(float) * ctx->dev_params,
                  cudaMemcpyDeviceToHost));
    padded_to_flat(ctx, pad.data(), m);
  }
  if (v) {
    CK(cudaMemcpy(pad.data(), ctx->V, sizeof(float) * ctx->dev_params,
                  cudaMemcpyDeviceToHost));
    padded_to_flat(ctx, pad.data(), v);
  }
  return ZRL_OK;
}

zrl_status zrl_set_normalizers(zrl_ctx *ctx, const float *obs_mean,
                               const float *obs_m2, float obs_count,
                               const float *crit_mean, const float *crit_m2,
                               float crit_count) {
  if (!ctx || !obs_mean || !obs_m2 || !crit_mean || !crit_m2) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  CK(cudaMemcpyAsync(ctx->obs_mean, obs_mean, sizeof(float) * od, cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->obs_m2, obs_m2, sizeof(float) * od, cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->crit_mean, crit_mean, sizeof(float) * cd, cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->crit_m2, crit_m2, sizeof(float) * cd, cudaMemcpyHostToDevice, ctx->stream));
  ctx->obs_count = obs_count;
  ctx->crit_count = crit_count;
  TRY(refresh_norm(ctx));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_get_normalizers(zrl_ctx *ctx, float *obs_mean, float *obs_m2,
                               float *obs_count, float *crit_mean, float *crit_m2,
                               float *crit_count) {
  if (!ctx) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  if (obs_mean) CK(cudaMemcpy(obs_mean, ctx->obs_mean, sizeof(float) * od, cudaMemcpyDeviceToHost));
  if (obs_m2) CK(cudaMemcpy(obs_m2, ctx->obs_m2, sizeof(float) * od, cudaMemcpyDeviceToHost));
  if (crit_mean) CK(cudaMemcpy(crit_mean, ctx->crit_mean, sizeof(float) * cd, cudaMemcpyDeviceToHost));
  if (crit_m2) CK(cudaMemcpy(crit_m2, ctx->crit_m2, sizeof(float) * cd, cudaMemcpyDeviceToHost));
  if (obs_count) *obs_count = ctx->obs_count;
  if (crit_count) *crit_count = ctx->crit_count;
  return ZRL_OK;
}

zrl_status zrl_set_lr(zrl_ctx *ctx, float lr) {
  if (!ctx) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  ctx->lr_host = lr;
  CK(cudaMemcpyAsync(&ctx->st->lr, &ctx->lr_host, sizeof(float), cudaMemcpyHostToDevice,
                     ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_get_lr(zrl_ctx *ctx, float *lr) {
  if (!ctx || !lr) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMemcpy(lr, &ctx->st->lr, sizeof(float), cudaMemcpyDeviceToHost));
  ctx->lr_host = *lr;
  return ZRL_OK;
}

zrl_status zrl_gae(zrl_ctx *ctx, const float *rewards, const float *values,
                   const uint8_t *dones, const float *last_values, int64_t n_envs,
                   int64_t T, float gamma, float lam, float *adv_out, float *ret_out,
                   int32_t on_device) {
  if (!ctx || !rewards || !values || !dones || !last_values || !adv_out || !ret_out)
    return ZRL_INVALID_ARG;
  if (n_envs < 0 || T < 0) return bad(ctx, "negative size");
  if (T > 4096) return bad(ctx, "T larger than 4096 is not supported");
  if (n_envs == 0 || T == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  TRY(ensure_envs(ctx, n_envs, T));
  GaeArgs a{};
  a.n_envs = n_envs;
  a.T = T;
  a.gamma = gamma;
  a.lam = lam;
  const int64_t n = n_envs * T;
  if (on_device) {
    a.rewards = rewards;
    a.values = values;
    a.dones = dones;
    a.last_values = last_values;
    a.adv = adv_out;
    a.ret = ret_out;
  } else {
    CK(cudaMemcpyAsync(ctx->r_rew, rewards, 4 * n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_val, values, 4 * n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_done, dones, n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_lv, last_values, 4 * n_envs, cudaMemcpyHostToDevice, ctx->stream));
    a.rewards = ctx->r_rew;
    a.values = ctx->r_val;
    a.dones = ctx->r_done;
    a.last_values = ctx->r_lv;
    a.adv = ctx->b_adv;
    a.ret = ctx->b_ret;
  }
  launch_gae(a, nullptr, gae_blocks(n_envs), ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  if (!on_device) {
    CK(cudaMemcpyAsync(adv_out, ctx->b_adv, 4 * n, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaMemcpyAsync(ret_out, ctx->b_ret, 4 * n, cudaMemcpyDeviceToHost, ctx->stream));
  }
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

static zrl_status check_batch(zrl_ctx *ctx, const zrl_batch *b, int64_t *n_global) {
  if (!b) return bad(ctx, "null batch");
  if (b->n < 0) return bad(ctx, "negative batch size");
  *n_global = b->n_global > 0 ? b->n_global : b->n;
  if (ctx->comm.world <= 1 && *n_global != b->n)
    return bad(ctx, "n_global != n without a data-parallel group");
  if (b->row_offset < 0 || b->row_offset + b->n > *n_global)
    return bad(ctx, "rows outside the global batch");
  if (*n_global > INT32_MAX) return bad(ctx, "batch larger than 2^31 rows");
  if (b->n > 0 && (!b->obs || !b->critic_obs || !b->action || !b->mean_old ||
                   !b->logp_old || !b->value_old))
    return bad(ctx, "null batch array");
  return ZRL_OK;
}

// The update's sample count check (ppo.rs:340), on the mirrored batch's
// doubled count when the augmentation is on (one rank only).
static zrl_status check_mirror(zrl_ctx *ctx, const zrl_batch *b, const zrl_ppo_config *cfg,
                               int64_t n_global) {
  if (ctx->mirror && ctx->comm.world > 1) {
    ctx->err = "the mirror augmentation runs on one rank";
    return ZRL_NOT_SUPPORTED;
  }
  const int64_t n = ctx->mirror ? 2 * n_global : n_global;
  if (n < cfg->minibatches) return bad(ctx, "fewer samples than minibatches");
  (void)b;
  return ZRL_OK;
}

static zrl_status write_back_adv(zrl_ctx *ctx, zrl_batch *b, const float *adv_dev) {
  if (!b->write_back_adv || b->n == 0) return ZRL_OK;
  // normalized advantages in the batch's own row order (ppo.rs:346-348):
  // (adv - mean) / sd with the device moments, applied to a host copy so the
  // caller's device buffer is only written once
  std::vector<float> tmp;
  CK(cudaStreamSynchronize(ctx->stream));
  DevState st;
  CK(cudaMemcpy(&st, ctx->st, sizeof(DevState), cudaMemcpyDeviceToHost));
  tmp.resize(b->n);
  CK(cudaMemcpy(tmp.data(), adv_dev, 4 * b->n, cudaMemcpyDeviceToHost));
  for (auto &x : tmp) x = (x - st.adv_mean) / st.adv_sd;
  if (b->on_device)
    CK(cudaMemcpy(b->adv, tmp.data(), 4 * b->n, cudaMemcpyHostToDevice));
  else
    memcpy(b->adv, tmp.data(), 4 * b->n);
  return ZRL_OK;
}

zrl_status zrl_update(zrl_ctx *ctx, const zrl_ppo_config *cfg, zrl_batch *batch,
                      zrl_stats *out) {
  if (!ctx) return ZRL_INVALID_ARG;
  TRY(check_cfg(ctx, cfg));
  int64_t n_global = 0;
  TRY(check_batch(ctx, batch, &n_global));
  if (batch->n > 0 && (!batch->adv || !batch->ret)) return bad(ctx, "null adv/ret");
  TRY(check_mirror(ctx, batch, cfg, n_global));
  CK(cudaSetDevice(ctx->device));
  cudaEvent_t u0 = nullptr;
  prof_begin(ctx, &u0);
  TRY(ensure_batch(ctx, ctx->mirror ? 2 * batch->n : batch->n));  // the doubled epoch rows
  DevBatch d{};
  TRY(stage_batch(ctx, batch, &d, true));
  TRY(adv_moments(ctx, d.adv, batch->n, n_global, false, 0));
  TRY(run_epochs(ctx, cfg, d, batch->n, n_global, batch->row_offset));
  TRY(prof_end(ctx, u0));
  TRY(write_back_adv(ctx, batch, d.adv));
  return finish_update(ctx, out);
}

zrl_status zrl_gae_update(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                          const zrl_rollout *ro, zrl_batch *batch, zrl_stats *out) {
  if (!ctx || !ro) return ZRL_INVALID_ARG;
  TRY(check_cfg(ctx, cfg));
  int64_t n_global = 0;
  TRY(check_batch(ctx, batch, &n_global));
  if (ro->n_envs * ro->T != batch->n) return bad(ctx, "rollout and batch disagree on n");
  if (ro->T > 4096) return bad(ctx, "T larger than 4096 is not supported");
  TRY(check_mirror(ctx, batch, cfg, n_global));
  CK(cudaSetDevice(ctx->device));
  cudaEvent_t u0 = nullptr;
  prof_begin(ctx, &u0);
  TRY(ensure_batch(ctx, ctx->mirror ? 2 * batch->n : batch->n));  // the doubled epoch rows
  DevBatch d{};
  TRY(stage_batch(ctx, batch, &d, false));
  TRY(ensure_envs(ctx, ro->n_envs, ro->T));
  const int64_t n = batch->n;
  GaeArgs a{};
  a.n_envs = ro->n_envs;
  a.T = ro->T;
  a.gamma = cfg->gamma;
  a.lam = cfg->lam;
  if (batch->on_device) {
    a.rewards = ro->rewards;
    a.values = ro->values;
    a.dones = ro->dones;
    a.last_values = ro->last_values;
  } else {
    CK(cudaMemcpyAsync(ctx->r_rew, ro->rewards, 4 * n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_val, ro->values, 4 * n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_done, ro->dones, n, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->r_lv, ro->last_values, 4 * ro->n_envs, cudaMemcpyHostToDevice,
                       ctx->stream));
    a.rewards = ctx->r_rew;
    a.values = ctx->r_val;
    a.dones = ctx->r_done;
    a.last_values = ctx->r_lv;
  }
  a.adv = ctx->b_adv;
  a.ret = ctx->b_ret;
  const int gb = gae_blocks(ro->n_envs);
  if (n > 0) {
    launch_gae(a, ctx->adv_part, gb, ctx->stream);
    ctx->launches++;
    CHECK_LAUNCH();
  }
  d.adv = ctx->b_adv;
  d.ret = ctx->b_ret;
  TRY(adv_moments(ctx, d.adv, n, n_global, n > 0, n > 0 ? gb : 0));
  TRY(run_epochs(ctx, cfg, d, n, n_global, batch->row_offset));
  TRY(prof_end(ctx, u0));
  return finish_update(ctx, out);
}

zrl_status zrl_forward(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                       int64_t n, float *mean_out, float *value_out, int32_t on_device) {
  if (!ctx) return ZRL_INVALID_ARG;
  if (n < 0) return bad(ctx, "negative n");
  if ((mean_out && !obs) || (value_out && !critic_obs)) return bad(ctx, "null input");
  if (n == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  const int odp = ctx->net[0].dp[0], cdp = ctx->net[1].dp[0];
  const int64_t chunk = std::min<int64_t>(n, 65536);
  TRY(ensure_batch(ctx, chunk));
  TRY(ensure_mb(ctx, chunk));
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t rows = std::min(chunk, n - r0);
    for (int k = 0; k < 2; ++k) {
      float *outp = k == 0 ? mean_out : value_out;
      if (!outp) continue;
      const float *src = k == 0 ? obs : critic_obs;
      const int dim = k == 0 ? od : cd;
      const int pitch = k == 0 ? odp : cdp;
      const float *x = src + r0 * dim;
      float *raw = k == 0 ? ctx->b_obs : ctx->b_cobs;
      if (!on_device) {
        CK(cudaMemcpyAsync(raw, x, sizeof(float) * rows * dim, cudaMemcpyHostToDevice,
                           ctx->stream));
        x = raw;
      }
      float *xn = k == 0 ? ctx->e_xa : ctx->e_xc;
      launch_normalize_rows(x, rows, dim, pitch, k == 0 ? ctx->obs_mean : ctx->crit_mean,
                            k == 0 ? ctx->obs_sd : ctx->crit_sd, xn, ctx->opmode(),
                            ctx->stream);
      ctx->launches++;
      CHECK_LAUNCH();
      TRY(forward_net(ctx, k, xn, rows));
      const NetLayout &L = ctx->net[k];
      const int cols = k == 0 ? ctx->A : 1;
      float *dst = outp + r0 * cols;
      float *tmp = k == 0 ? ctx->e_act : ctx->e_vo;
      launch_unpad_rows(ctx->act[k][L.L], rows, L.dp[L.L], cols,
                        on_device ? dst : tmp, ctx->stream);
      ctx->launches++;
      CHECK_LAUNCH();
      if (!on_device)
        CK(cudaMemcpyAsync(dst, tmp, sizeof(float) * rows * cols, cudaMemcpyDeviceToHost,
                           ctx->stream));
    }
  }
  CK(cudaStreamSynchronize(ctx->stream));
  return check_device_error(ctx);
}

zrl_status zrl_shuffle_device(zrl_ctx *ctx, uint64_t seed, int64_t n, int32_t *order) {
  if (!ctx || n < 0 || n > INT32_MAX || (n > 0 && !order)) return ZRL_INVALID_ARG;
  if (n == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  int32_t *scratch = nullptr;
  CK(cudaMallocAsync((void **)&scratch, sizeof(int32_t) * 3 * (size_t)n, ctx->stream));
  launch_shuffle_device(seed, (int32_t)n, order, scratch, ctx->stream);
  ctx->launches += 2;
  const cudaError_t e = cudaGetLastError();
  cudaFreeAsync(scratch, ctx->stream);
  if (e != cudaSuccess) {
    ctx->err = std::string("zrl_shuffle_device: ") + cudaGetErrorString(e);
    return ZRL_CUDA_ERROR;
  }
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

int64_t zrl_rank_orders_device(zrl_ctx *ctx, uint64_t seed, int64_t n_global, int64_t n_local,
                               int64_t row_offset, int32_t minibatches, int32_t *order,
                               int64_t *counts) {
  if (!ctx || n_global <= 0 || n_global > INT32_MAX || minibatches <= 0 || n_local < 0 ||
      !order || !counts)
    return -1;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return -1;
  const size_t nblk = (size_t)(n_global + 1023) / 1024;
  // perm [n_global] | shuffle scratch [3 n_global] | block sums [nblk + 1],
  // then the counts [minibatches + 1] on the next 8-byte boundary
  const size_t ints = (size_t)n_global * 4 + nblk + 1;
  int32_t *buf = nullptr;
  if (cudaMallocAsync((void **)&buf,
                      sizeof(int32_t) * ints + sizeof(int64_t) * (minibatches + 1) + 8,
                      ctx->stream) != cudaSuccess) {
    ctx->err = "zrl_rank_orders_device: allocation failed";
    return -1;
  }
  int32_t *perm = buf, *sh = buf + n_global, *bs = buf + 4 * (size_t)n_global;
  int64_t *cnt = reinterpret_cast<int64_t *>(
      (reinterpret_cast<uintptr_t>(buf + ints) + 7) & ~(uintptr_t)7);
  launch_shuffle_device(seed, (int32_t)n_global, perm, sh, ctx->stream);
  launch_rank_orders(perm, n_global, n_local, row_offset, minibatches, order, cnt, bs,
                     ctx->stream);
  ctx->launches += 6;
  cudaMemcpyAsync(counts, cnt, sizeof(int64_t) * minibatches, cudaMemcpyDeviceToHost,
                  ctx->stream);
  cudaFreeAsync(buf, ctx->stream);
  const cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    ctx->err = std::string("zrl_rank_orders_device: ") + cudaGetErrorString(e);
    return -1;
  }
  int64_t n = 0;
  for (int m = 0; m < minibatches; ++m) n += counts[m];
  return n;
}

zrl_status zrl_gemm(zrl_ctx *ctx, int32_t layout, int32_t M, int32_t N, int32_t K,
                    const float *A, int32_t lda, const float *B, int32_t ldb, float *C,
                    int32_t ldc, int32_t split_k) {
  if (!ctx || !A || !B || !C) return ZRL_INVALID_ARG;
  if (layout < 0 || layout > 2 || M < 0 || N < 0 || K < 0 || split_k < 1 || split_k > 64)
    return bad(ctx, "invalid GEMM arguments");
  CK(cudaSetDevice(ctx->device));
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = A;
  g.lda = lda;
  g.trans_a = layout == 2;
  g.B = B;
  g.ldb = ldb;
  g.trans_b = layout == 0;
  g.C = C;
  g.ldc = ldc;
  g.epi = EPI_STORE;
  g.split_k = split_k;
  TRY(run_gemm(ctx, g));
  CK(cudaStreamSynchronize(ctx->stream));
  return check_device_error(ctx);
}

zrl_status zrl_minibatch_grads(zrl_ctx *ctx, const zrl_ppo_config *cfg,
                               const zrl_batch *batch, const int64_t *idx,
                               int64_t n_idx, float *grads_out, float *sums3_out) {
  if (!ctx || !idx || !grads_out) return ZRL_INVALID_ARG;
  TRY(check_cfg(ctx, cfg));
  int64_t n_global = 0;
  TRY(check_batch(ctx, batch, &n_global));
  if (ctx->comm.world > 1) return bad(ctx, "minibatch_grads is a single-rank hook");
  if (n_idx < 1) return bad(ctx, "empty index set");
  for (int64_t i = 0; i < n_idx; ++i)
    if (idx[i] < 0 || idx[i] >= batch->n) return bad(ctx, "index out of range");
  CK(cudaSetDevice(ctx->device));
  DevBatch d{};
  TRY(stage_batch(ctx, batch, &d, true));
  TRY(ensure_batch(ctx, std::max(n_idx, batch->n)));
  TRY(ensure_pinned_orders(ctx, n_idx));
  for (int64_t i = 0; i < n_idx; ++i) ctx->order_pinned[i] = (int32_t)idx[i];
  CK(cudaMemcpyAsync(ctx->order_dev, ctx->order_pinned, sizeof(int32_t) * n_idx,
                     cudaMemcpyHostToDevice, ctx->stream));
  TRY(normalize_batch(ctx, d.obs, d.cobs, batch->n));
  GatherArgs g = gather_args(ctx, d, 0);
  g.n_used = n_idx;
  g.apply_adv_norm = 0;  // the hook takes advantages as given
  launch_gather(g, ctx->stream);
  ctx->launches++;
  CHECK_LAUNCH();
  TRY(minibatch_grads(ctx, cfg, epoch_view(ctx, 0, n_idx), 1.0f / (float)n_idx));
  std::vector<float> pad(ctx->grad_len);
  CK(cudaMemcpyAsync(pad.data(), ctx->G, sizeof(float) * ctx->grad_len,
                     cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  TRY(check_device_error(ctx));
  padded_to_flat(ctx, pad.data(), grads_out);
  if (sums3_out) memcpy(sums3_out, pad.data() + ctx->dev_params, sizeof(float) * 3);
  return ZRL_OK;
}

zrl_status zrl_apply_grads(zrl_ctx *ctx, const zrl_ppo_config *cfg, const float *grads,
                           float kl) {
  if (!ctx || !grads) return ZRL_INVALID_ARG;
  TRY(check_cfg(ctx, cfg));
  CK(cudaSetDevice(ctx->device));
  std::vector<float> pad(ctx->grad_len, 0.0f);
  flat_to_padded(ctx, grads, pad.data());
  pad[ctx->dev_params + 2] = kl;
  CK(cudaMemcpyAsync(ctx->G, pad.data(), sizeof(float) * ctx->grad_len,
                     cudaMemcpyHostToDevice, ctx->stream));
  TRY(step(ctx, cfg, cfg->minibatches, false, false));
  CK(cudaStreamSynchronize(ctx->stream));
  ctx->t_logstd_host += 1;
  float lr = 0.0f;
  return zrl_get_lr(ctx, &lr);
}

zrl_status zrl_set_mirror(zrl_ctx *ctx, const int32_t *obs_perm, const float *obs_sign,
                          const int32_t *cobs_perm, const float *cobs_sign,
                          const int32_t *act_perm, const float *act_sign) {
  if (!ctx) return ZRL_INVALID_ARG;
  if (!obs_perm) {
    ctx->mirror = false;
    return ZRL_OK;
  }
  if (!obs_sign || !cobs_perm || !cobs_sign || !act_perm || !act_sign)
    return bad(ctx, "the mirror needs all six arrays");
  // each a signed permutation: perm a permutation of 0..d-1, sign +-1
  auto valid = [](const int32_t *perm, const float *sign, int d) {
    std::vector<char> seen(d, 0);
    for (int i = 0; i < d; ++i) {
      if (perm[i] < 0 || perm[i] >= d || seen[perm[i]]) return false;
      seen[perm[i]] = 1;
      if (sign[i] != 1.0f && sign[i] != -1.0f) return false;
    }
    return true;
  };
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0], A = ctx->A;
  if (!valid(obs_perm, obs_sign, od) || !valid(cobs_perm, cobs_sign, cd) ||
      !valid(act_perm, act_sign, A))
    return bad(ctx, "mirror: perm must be a permutation and sign +-1");
  CK(cudaSetDevice(ctx->device));
  if (!ctx->mir_operm) {
    TRY(dalloc(ctx, &ctx->mir_operm, od));
    TRY(dalloc(ctx, &ctx->mir_cperm, cd));
    TRY(dalloc(ctx, &ctx->mir_aperm, A));
    TRY(dalloc(ctx, &ctx->mir_osign, od));
    TRY(dalloc(ctx, &ctx->mir_csign, cd));
    TRY(dalloc(ctx, &ctx->mir_asign, A));
  }
  CK(cudaMemcpy(ctx->mir_operm, obs_perm, 4 * od, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ctx->mir_cperm, cobs_perm, 4 * cd, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ctx->mir_aperm, act_perm, 4 * A, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ctx->mir_osign, obs_sign, 4 * od, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ctx->mir_csign, cobs_sign, 4 * cd, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ctx->mir_asign, act_sign, 4 * A, cudaMemcpyHostToDevice));
  ctx->mirror = true;
  return ZRL_OK;
}

zrl_status zrl_set_wait_limit(zrl_ctx *ctx, uint64_t ns) {
  if (!ctx) return ZRL_INVALID_ARG;
  if (ns < 1000000ull) return bad(ctx, "wait limit below 1 ms");
  ctx->gemm.wait_ns = ns;
  return ZRL_OK;
}

zrl_status zrl_test_comm_wait(int32_t scenario, int32_t timeout_ms, int32_t *aborted) {
  if (!aborted || scenario < 0 || scenario > 3 || timeout_ms < 0) return ZRL_INVALID_ARG;
  std::string err;
  int ab = 0;
  const zrl_status st = comm_wait_fake(scenario, timeout_ms, &ab, &err);
  *aborted = ab;
  return st;
}

zrl_status zrl_test_stall_next_gemm(zrl_ctx *ctx) {
  if (!ctx) return ZRL_INVALID_ARG;
  if (!ctx->tcore()) return bad(ctx, "the stall hook is in the tensor-core GEMM");
  ctx->gemm.stall_next = 1;
  return ZRL_OK;
}

zrl_status zrl_set_profiling(zrl_ctx *ctx, int32_t enabled) {
  if (!ctx) return ZRL_INVALID_ARG;
  ctx->profiling = enabled != 0;
  return ZRL_OK;
}

int32_t zrl_profile_site(const zrl_ctx *ctx, int32_t i, const char **name, float *ms,
                         int64_t *spans) {
  if (!ctx || i < 0 || i >= (int32_t)ctx->sites.size()) return 0;
  if (name) *name = ctx->sites[i].first.c_str();
  if (ms) *ms = ctx->sites[i].second.first;
  if (spans) *spans = ctx->sites[i].second.second;
  return 1;
}

zrl_status zrl_get_profile(zrl_ctx *ctx, float *gemm_ms, float *update_ms,
                           int64_t *gemm_launches) {
  if (!ctx) return ZRL_INVALID_ARG;
  if (gemm_ms) *gemm_ms = ctx->prof_gemm_ms;
  if (update_ms) *update_ms = ctx->prof_update_ms;
  if (gemm_launches) *gemm_launches = ctx->prof_gemm_launches;
  return ZRL_OK;
}

// Rows of both observation kinds on the device (host rows are copied to
// the batch staging buffers).
static zrl_status stage_obs(zrl_ctx *ctx, const float *obs, const float *critic_obs, int64_t n,
                            int32_t on_device, const float **xo, const float **xc) {
  if (on_device) {
    *xo = obs;
    *xc = critic_obs;
    return ZRL_OK;
  }
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  TRY(ensure_batch(ctx, n));
  CK(cudaMemcpyAsync(ctx->b_obs, obs, sizeof(float) * n * od, cudaMemcpyHostToDevice,
                     ctx->stream));
  CK(cudaMemcpyAsync(ctx->b_cobs, critic_obs, sizeof(float) * n * cd, cudaMemcpyHostToDevice,
                     ctx->stream));
  *xo = ctx->b_obs;
  *xc = ctx->b_cobs;
  return ZRL_OK;
}

// n rows folded into (count, mean, m2) of one normalizer: in order, one
// row at a time (mode 0, the reference's arithmetic), or in row chunks
// merged pairwise (mode 1, the parallel fold of welford.cu).
static zrl_status fold_rows(zrl_ctx *ctx, const float *x, int64_t n, int dim, float *count,
                            float *mean, float *m2, int32_t mode) {
  if (mode == 1) {
    const int64_t need = welford_partial_floats(n, dim);
    if (need > ctx->welford_cap) {
      TRY(dalloc(ctx, &ctx->welford_scratch, need));
      ctx->welford_cap = need;
    }
    launch_welford_parallel(x, n, dim, *count, mean, m2, ctx->welford_scratch, ctx->stream);
    ctx->launches += 2;
  } else {
    launch_record_obs(x, n, dim, mean, m2, *count, ctx->stream);
    ctx->launches++;
  }
  CHECK_LAUNCH();
  for (int64_t r = 0; r < n; ++r) *count += 1.0f;  // the f32 count recurrence
  return ZRL_OK;
}

static zrl_status record_obs_impl(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                                  int64_t n, int32_t on_device, int32_t mode) {
  if (!ctx || (n > 0 && (!obs || !critic_obs))) return ZRL_INVALID_ARG;
  if (n < 0) return bad(ctx, "negative n");
  if (mode != 0 && mode != 1) return bad(ctx, "mode must be 0 (sequential) or 1 (parallel)");
  if (n == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  const float *xo = nullptr, *xc = nullptr;
  TRY(stage_obs(ctx, obs, critic_obs, n, on_device, &xo, &xc));
  TRY(fold_rows(ctx, xo, n, ctx->net[0].d[0], &ctx->obs_count, ctx->obs_mean, ctx->obs_m2, mode));
  TRY(fold_rows(ctx, xc, n, ctx->net[1].d[0], &ctx->crit_count, ctx->crit_mean, ctx->crit_m2,
                mode));
  TRY(refresh_norm(ctx));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_record_obs(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                          int64_t n) {
  return record_obs_impl(ctx, obs, critic_obs, n, 0, 0);
}

zrl_status zrl_record_obs_ex(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                             int64_t n, int32_t on_device, int32_t mode) {
  return record_obs_impl(ctx, obs, critic_obs, n, on_device, mode);
}

zrl_status zrl_pending_push(zrl_ctx *ctx, const float *obs, const float *critic_obs, int64_t n,
                            int32_t on_device, int32_t mode) {
  if (!ctx || (n > 0 && (!obs || !critic_obs))) return ZRL_INVALID_ARG;
  if (n < 0) return bad(ctx, "negative n");
  if (mode != 0 && mode != 1) return bad(ctx, "mode must be 0 (sequential) or 1 (parallel)");
  if (n == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  const float *xo = nullptr, *xc = nullptr;
  TRY(stage_obs(ctx, obs, critic_obs, n, on_device, &xo, &xc));
  TRY(fold_rows(ctx, xo, n, ctx->net[0].d[0], &ctx->pend_obs_count, ctx->pend_obs_mean,
                ctx->pend_obs_m2, mode));
  TRY(fold_rows(ctx, xc, n, ctx->net[1].d[0], &ctx->pend_crit_count, ctx->pend_crit_mean,
                ctx->pend_crit_m2, mode));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_commit_pending(zrl_ctx *ctx) {
  if (!ctx) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  // a normalizer whose pending state is empty is left as it is (ppo.rs:180)
  if (ctx->pend_obs_count != 0.0f) {
    launch_norm_commit(ctx->obs_mean, ctx->obs_m2, ctx->obs_count, ctx->pend_obs_mean,
                       ctx->pend_obs_m2, ctx->pend_obs_count, ctx->net[0].d[0], ctx->stream);
    ctx->launches++;
    ctx->obs_count = ctx->obs_count + ctx->pend_obs_count;
    ctx->pend_obs_count = 0.0f;
  }
  if (ctx->pend_crit_count != 0.0f) {
    launch_norm_commit(ctx->crit_mean, ctx->crit_m2, ctx->crit_count, ctx->pend_crit_mean,
                       ctx->pend_crit_m2, ctx->pend_crit_count, ctx->net[1].d[0], ctx->stream);
    ctx->launches++;
    ctx->crit_count = ctx->crit_count + ctx->pend_crit_count;
    ctx->pend_crit_count = 0.0f;
  }
  CHECK_LAUNCH();
  TRY(refresh_norm(ctx));
  CK(cudaStreamSynchronize(ctx->stream));
  return ZRL_OK;
}

zrl_status zrl_get_pending(zrl_ctx *ctx, float *obs_mean, float *obs_m2, float *obs_count,
                           float *crit_mean, float *crit_m2, float *crit_count) {
  if (!ctx) return ZRL_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  if (obs_mean) CK(cudaMemcpy(obs_mean, ctx->pend_obs_mean, 4 * od, cudaMemcpyDeviceToHost));
  if (obs_m2) CK(cudaMemcpy(obs_m2, ctx->pend_obs_m2, 4 * od, cudaMemcpyDeviceToHost));
  if (crit_mean) CK(cudaMemcpy(crit_mean, ctx->pend_crit_mean, 4 * cd, cudaMemcpyDeviceToHost));
  if (crit_m2) CK(cudaMemcpy(crit_m2, ctx->pend_crit_m2, 4 * cd, cudaMemcpyDeviceToHost));
  if (obs_count) *obs_count = ctx->pend_obs_count;
  if (crit_count) *crit_count = ctx->pend_crit_count;
  return ZRL_OK;
}

// The Lcg state after d draws from s (the affine step of rng.rs:21-23
// raised to the d-th power by squaring).
static uint64_t lcg_jump_host(uint64_t s, uint64_t d) {
  uint64_t a = 1, c = 0, pa = 6364136223846793005ull, pc = 1442695040888963407ull;
  while (d) {
    if (d & 1) {
      c = pa * c + pc;
      a = pa * a;
    }
    pc = pa * pc + pc;
    pa = pa * pa;
    d >>= 1;
  }
  return a * s + c;
}

// The rollout policy step with either sampler: Philox (seed, counter) or
// the reference's sequential Lcg stream (*lcg, advanced by 2 n A draws).
static zrl_status policy_step_impl(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                                   int64_t n, uint64_t seed, uint64_t counter, uint64_t *lcg,
                                   float *action, float *logp, float *mean, float *value,
                                   int32_t on_device) {
  if (!ctx || !obs || !action) return ZRL_INVALID_ARG;
  if (value && !critic_obs) return bad(ctx, "value requested without critic_obs");
  if (n < 0) return bad(ctx, "negative n");
  if (n == 0) return ZRL_OK;
  CK(cudaSetDevice(ctx->device));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  const int odp = ctx->net[0].dp[0], cdp = ctx->net[1].dp[0];
  const int A = ctx->A;
  const int64_t chunk = std::min<int64_t>(n, 65536);
  TRY(ensure_batch(ctx, chunk));
  TRY(ensure_mb(ctx, chunk));
  const NetLayout &La = ctx->net[0], &Lc = ctx->net[1];
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t rows = std::min(chunk, n - r0);
    const float *x = obs + r0 * od;
    if (!on_device) {
      CK(cudaMemcpyAsync(ctx->b_obs, x, sizeof(float) * rows * od, cudaMemcpyHostToDevice,
                         ctx->stream));
      x = ctx->b_obs;
    }
    launch_normalize_rows(x, rows, od, odp, ctx->obs_mean, ctx->obs_sd, ctx->e_xa,
                          ctx->opmode(), ctx->stream);
    ctx->launches++;
    TRY(forward_net(ctx, 0, ctx->e_xa, rows));
    float *act_d = on_device ? action + r0 * A : ctx->e_act;
    float *lp_d = logp ? (on_device ? logp + r0 : ctx->e_lpo) : nullptr;
    float *mean_d = mean ? (on_device ? mean + r0 * A : ctx->e_mo) : nullptr;
    // rows are numbered globally so a chunked call draws the same numbers
    if (lcg) {
      launch_lcg_sample(ctx->act[0][La.L], La.dp[La.L], ctx->P + ctx->ls_off, A, rows, *lcg, r0,
                        act_d, mean_d, ctx->stream);
      if (lp_d)
        launch_logp_rows(act_d, ctx->act[0][La.L], La.dp[La.L], ctx->P + ctx->ls_off, A, rows,
                         lp_d, ctx->stream);
    } else {
      launch_policy_sample(ctx->act[0][La.L], La.dp[La.L], ctx->P + ctx->ls_off, A, rows,
                           seed, counter, act_d, lp_d, mean_d, ctx->stream, r0);
    }
    ctx->launches += logp ? 2 : 1;
    CHECK_LAUNCH();
    if (value) {
      const float *c = critic_obs + r0 * cd;
      if (!on_device) {
        CK(cudaMemcpyAsync(ctx->b_cobs, c, sizeof(float) * rows * cd,
                           cudaMemcpyHostToDevice, ctx->stream));
        c = ctx->b_cobs;
      }
      launch_normalize_rows(c, rows, cd, cdp, ctx->crit_mean, ctx->crit_sd, ctx->e_xc,
                            ctx->opmode(), ctx->stream);
      ctx->launches++;
      TRY(forward_net(ctx, 1, ctx->e_xc, rows));
      float *v_d = on_device ? value + r0 : ctx->e_vo;
      launch_unpad_rows(ctx->act[1][Lc.L], rows, Lc.dp[Lc.L], 1, v_d, ctx->stream);
      ctx->launches++;
      CHECK_LAUNCH();
      if (!on_device)
        CK(cudaMemcpyAsync(value + r0, v_d, sizeof(float) * rows, cudaMemcpyDeviceToHost,
                           ctx->stream));
    }
    if (!on_device) {
      CK(cudaMemcpyAsync(action + r0 * A, act_d, sizeof(float) * rows * A,
                         cudaMemcpyDeviceToHost, ctx->stream));
      if (logp)
        CK(cudaMemcpyAsync(logp + r0, lp_d, sizeof(float) * rows, cudaMemcpyDeviceToHost,
                           ctx->stream));
      if (mean)
        CK(cudaMemcpyAsync(mean + r0 * A, mean_d, sizeof(float) * rows * A,
                           cudaMemcpyDeviceToHost, ctx->stream));
    }
    // keep the staging buffers alive until the copies drain
    CK(cudaStreamSynchronize(ctx->stream));
  }
  if (lcg) *lcg = lcg_jump_host(*lcg, 2ull * (uint64_t)n * (uint64_t)A);
  return check_device_error(ctx);
}

zrl_status zrl_policy_step(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                           int64_t n, uint64_t seed, uint64_t counter, float *action,
                           float *logp, float *mean, float *value, int32_t on_device) {
  return policy_step_impl(ctx, obs, critic_obs, n, seed, counter, nullptr, action, logp, mean,
                          value, on_device);
}

zrl_status zrl_policy_step_lcg(zrl_ctx *ctx, const float *obs, const float *critic_obs,
                               int64_t n, uint64_t *lcg_state, float *action, float *logp,
                               float *mean, float *value, int32_t on_device) {
  if (!lcg_state) return bad(ctx, "null Lcg state");
  return policy_step_impl(ctx, obs, critic_obs, n, 0, 0, lcg_state, action, logp, mean, value,
                          on_device);
}

// ---------------------------------------------------------------- I/O

static zrl_status build_checkpoint(zrl_ctx *ctx, std::vector<uint8_t> *out) {
  std::vector<float> flat(ctx->flat_params);
  TRY(zrl_get_params(ctx, flat.data(), ctx->flat_params));
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  std::vector<float> om(od), om2(od), cm(cd), cm2(cd);
  float oc = 0, cc = 0, lr = 0;
  TRY(zrl_get_normalizers(ctx, om.data(), om2.data(), &oc, cm.data(), cm2.data(), &cc));
  TRY(zrl_get_lr(ctx, &lr));
  std::map<std::string, StTensor> ts;
  const char *prefix[2] = {"actor", "critic"};
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    for (int l = 0; l < L.L; ++l) {
      StTensor w, b;
      w.shape = {L.d[l + 1], L.d[l]};
      w.data.assign(flat.begin() + L.fw_off[l],
                    flat.begin() + L.fw_off[l] + (int64_t)L.d[l + 1] * L.d[l]);
      b.shape = {L.d[l + 1]};
      b.data.assign(flat.begin() + L.fb_off[l], flat.begin() + L.fb_off[l] + L.d[l + 1]);
      ts[std::string(prefix[k]) + ".w_" + std::to_string(l)] = w;
      ts[std::string(prefix[k]) + ".b_" + std::to_string(l)] = b;
    }
  }
  auto vec = [](std::vector<float> v) {
    StTensor t;
    t.shape = {(int64_t)v.size()};
    t.data = std::move(v);
    return t;
  };
  ts["log_std"] = vec(std::vector<float>(flat.begin() + ctx->net[1].flat_end, flat.end()));
  ts["obs_norm.mean"] = vec(om);
  ts["obs_norm.m2"] = vec(om2);
  ts["obs_norm.count"] = vec({oc});
  ts["critic_norm.mean"] = vec(cm);
  ts["critic_norm.m2"] = vec(cm2);
  ts["critic_norm.count"] = vec({cc});
  ts["lr"] = vec({lr});
  *out = st_serialize(ts);
  return ZRL_OK;
}

zrl_status zrl_save(zrl_ctx *ctx, const char *path) {
  if (!ctx || !path) return ZRL_INVALID_ARG;
  std::vector<uint8_t> bytes;
  TRY(build_checkpoint(ctx, &bytes));
  FILE *f = fopen(path, "wb");
  if (!f) {
    ctx->err = std::string("cannot open ") + path + " for writing";
    return ZRL_IO_ERROR;
  }
  const size_t w = fwrite(bytes.data(), 1, bytes.size(), f);
  const int c = fclose(f);
  if (w != bytes.size() || c != 0) {
    ctx->err = std::string("short write to ") + path;
    return ZRL_IO_ERROR;
  }
  return ZRL_OK;
}

zrl_status zrl_load_from_bytes(zrl_ctx *ctx, const uint8_t *bytes, size_t len) {
  if (!ctx || !bytes) return ZRL_INVALID_ARG;
  std::map<std::string, StTensor> ts;
  if (!st_parse(bytes, len, &ts, &ctx->err)) return ZRL_IO_ERROR;
  std::vector<float> flat(ctx->flat_params);
  const char *prefix[2] = {"actor", "critic"};
  for (int k = 0; k < 2; ++k) {
    const NetLayout &L = ctx->net[k];
    // layers are the contiguous w_{l} from 0 (ppo.rs:594-609)
    int layers = 0;
    while (ts.count(std::string(prefix[k]) + ".w_" + std::to_string(layers))) ++layers;
    if (layers != L.L) {
      ctx->err = std::string("checkpoint ") + prefix[k] + " has " + std::to_string(layers) +
                 " layers, context has " + std::to_string(L.L);
      return ZRL_INVALID_ARG;
    }
    for (int l = 0; l < L.L; ++l) {
      const std::string wn = std::string(prefix[k]) + ".w_" + std::to_string(l);
      const std::string bn = std::string(prefix[k]) + ".b_" + std::to_string(l);
      if (!ts.count(bn)) {
        ctx->err = "checkpoint lacks " + bn;
        return ZRL_IO_ERROR;
      }
      const StTensor &w = ts[wn], &b = ts[bn];
      if (w.shape.size() != 2) {
        ctx->err = wn + ": expected 2D";
        return ZRL_IO_ERROR;
      }
      if (w.shape[0] != L.d[l + 1] || w.shape[1] != L.d[l] ||
          (int64_t)b.data.size() != L.d[l + 1]) {
        ctx->err = wn + ": shape does not match the context";
        return ZRL_INVALID_ARG;
      }
      std::copy(w.data.begin(), w.data.end(), flat.begin() + L.fw_off[l]);
      std::copy(b.data.begin(), b.data.end(), flat.begin() + L.fb_off[l]);
    }
  }
  const char *need[] = {"log_std", "obs_norm.mean", "obs_norm.m2", "obs_norm.count",
                        "critic_norm.mean", "critic_norm.m2", "critic_norm.count", "lr"};
  for (const char *nm : need)
    if (!ts.count(nm) || ts[nm].data.empty()) {
      ctx->err = std::string("checkpoint lacks ") + nm;
      return ZRL_IO_ERROR;
    }
  const int od = ctx->net[0].d[0], cd = ctx->net[1].d[0];
  if ((int)ts["log_std"].data.size() != ctx->A || (int)ts["obs_norm.mean"].data.size() != od ||
      (int)ts["obs_norm.m2"].data.size() != od || (int)ts["critic_norm.mean"].data.size() != cd ||
      (int)ts["critic_norm.m2"].data.size() != cd) {
    ctx->err = "checkpoint vector sizes do not match the context";
    return ZRL_INVALID_ARG;
  }
  std::copy(ts["log_std"].data.begin(), ts["log_std"].data.end(),
            flat.begin() + ctx->net[1].flat_end);
  TRY(zrl_set_params(ctx, flat.data(), ctx->flat_params));  // resets Adam
  TRY(zrl_set_normalizers(ctx, ts["obs_norm.mean"].data.data(), ts["obs_norm.m2"].data.data(),
                          ts["obs_norm.count"].data[0], ts["critic_norm.mean"].data.data(),
                          ts["critic_norm.m2"].data.data(), ts["critic_norm.count"].data[0]));
  return zrl_set_lr(ctx, ts["lr"].data[0]);
}

zrl_status zrl_load(zrl_ctx *ctx, const char *path) {
  if (!ctx || !path) return ZRL_INVALID_ARG;
  FILE *f = fopen(path, "rb");
  if (!f) {
    ctx->err = std::string("cannot open ") + path;
    return ZRL_IO_ERROR;
  }
  std::vector<uint8_t> bytes;
  uint8_t buf[1 << 16];
  size_t r;
  while ((r = fread(buf, 1, sizeof(buf), f)) > 0) bytes.insert(bytes.end(), buf, buf + r);
  fclose(f);
  return zrl_load_from_bytes(ctx, bytes.data(), bytes.size());
}

}  // extern "C"
