// zrl_gemm.h -- GEMM dispatch for the MLP forward/backward.
//
// ZRL_GEMM_FP32 runs the CUDA-core kernel (gemm_simt.cu); ZRL_GEMM_TF32
// runs the tcgen05 tensor-core kernels (gemm_tc.cu).  There is no silent
// substitution: a shape the tensor-core kernel does not take is an error,
// not a fallback.
#pragma once

#include <cuda.h>

#include <string>

#include "zrl_internal.h"

namespace zrl {

struct GemmEngine;

// A TMA tensor map from the engine's cache (gemm_tc.cu): kind 0 a K-major
// fp32 operand [rows, cols] (pitch ld) in boxes of 32 columns x box rows,
// 128-byte swizzle; kind 1 the MN-major form (32-byte-atom swizzle); kind 2
// an fp32 output [splits][rows][cols] written in 32 x 32 boxes.
bool tc_tensor_map(GemmEngine *eng, CUtensorMap *out, const float *base, int64_t rows,
                   int64_t cols, int64_t ld, int box_or_splits, int kind, std::string *err);
// SMs of the device the tensor-core kernels were initialised on.
int tc_sm_count();

// The fused output head (head_tc.cu) of both nets over one minibatch: the
// output layer's forward Z = A W^T + b on the tensor cores, the PPO losses
// of each row (ppo.rs:410-452) giving the output-layer delta D (the loss
// kernel's math), and the last hidden layer's input gradient
// D' = (D W) * ELU'(A) on the tensor cores with its bias-gradient column
// sums -- one launch in place of the output-layer forward, the loss and the
// output-layer input-gradient launches.  tf32 operands; both nets' output
// layers 32 wide (padded), their inputs 32..128 wide.
struct HeadNet {
  const float *a;   // [rows, k] the last hidden activation (tf32-rounded)
  int k;            // its padded width (32..128, a multiple of 32)
  const float *w;   // output-layer weights [32, k] (tf32 copy)
  const float *b;   // output-layer bias [32] (fp32 master)
  float *d_out;     // out: the output-layer delta [rows, 32] (tf32-rounded)
  float *d_in;      // out: the last hidden layer's delta [rows, k] (tf32-rounded)
  float *colsum;    // out: [head_partial_rows, k] partial column sums of d_in (fp32)
};
struct HeadArgs {
  HeadNet net[2];  // actor, critic
  const float *action, *mean_old;                 // [rows, A]
  const float *logp_old, *value_old, *adv, *ret;  // [rows]
  const float *log_std;                           // [A]
  int A;
  int64_t rows;
  float scale, clip, entropy_coef, value_coef;
  // [head_partial_rows, 100]: [g_logstd (32) | db_actor (32) | surr vloss kl 0 |
  // db_critic (32)], the layout of the loss kernel's rows (LossArgs)
  float *part;
  int *err;
};
constexpr int kHeadWidth = 2 * 32 + 4 + 32;
// Partial rows the head writes for `rows` rows (four per CTA).
int head_partial_rows(int64_t rows);
zrl_status head_tc(GemmEngine *eng, const HeadArgs &a, cudaStream_t s, std::string *err);

// Tensor-core GEMM (gemm_tc.cu).  *launched receives the kernel count.
zrl_status gemm_tc(GemmEngine *eng, const GemmArgs &g, int precision, cudaStream_t s,
                   int *launched, std::string *err);
// n GEMMs (1..8) of one operand layout and epilogue in one launch.
zrl_status gemm_tc_group(GemmEngine *eng, const GemmArgs *gs, int n, int precision,
                         cudaStream_t s, int *launched, std::string *err);
zrl_status gemm_tc_init(int device, std::string *err);
// Split-K count (1..max_split) for a group of weight-gradient GEMMs sharing
// K: the fewest splits whose output tiles fill the persistent grid about as
// well as any (gemm_tc.cu).
int gemm_tc_split(GemmEngine *eng, const GemmArgs *gs, int n, int precision, int max_split,
                  int *splits);

struct GemmEngine {
  bool tc_ready = false;
  void *cache = nullptr;  // tensor-map cache (gemm_tc.cu)
  int *err_dev = nullptr; // device flag set by a timed-out pipeline wait
  uint64_t wait_ns = 20ull * 1000 * 1000 * 1000;  // bound of every pipeline wait
  int stall_next = 0;     // test hook: the next tensor-core GEMM launch stalls

  zrl_status init(int device, std::string *err);
  void destroy();

  zrl_status run(const GemmArgs &g, int precision, cudaStream_t s, int *launched,
                 std::string *err) {
    *launched = 0;
    if (g.M <= 0 || g.N <= 0) return ZRL_OK;
    if (precision == ZRL_GEMM_FP32) {
      gemm_simt(g, s);
      *launched = 1;
      return ZRL_OK;
    }
    if (!tc_ready) {
      zrl_status st = gemm_tc_init(0, err);
      if (st != ZRL_OK) return st;
      tc_ready = true;
    }
    return gemm_tc(this, g, precision, s, launched, err);
  }

  // Split-K counts for a weight-gradient group, one per problem, into
  // splits[0..n) (see gemm_tc_split); returns 0 on the CUDA cores, where
  // the caller keeps its own split.
  int split_for(const GemmArgs *gs, int n, int precision, int max_split, int *splits,
                std::string *err) {
    if (precision == ZRL_GEMM_FP32) return 0;
    if (!tc_ready) {
      if (gemm_tc_init(0, err) != ZRL_OK) return 0;
      tc_ready = true;
    }
    return gemm_tc_split(this, gs, n, precision, max_split, splits);
  }

  // The fused output head (tensor cores only).
  zrl_status head(const HeadArgs &a, cudaStream_t s, std::string *err) {
    if (!tc_ready) {
      zrl_status st = gemm_tc_init(0, err);
      if (st != ZRL_OK) return st;
      tc_ready = true;
    }
    return head_tc(this, a, s, err);
  }

  // Several GEMMs of one layout and epilogue: one grouped launch on the
  // tensor cores, one launch each on the CUDA cores.
  zrl_status run_group(const GemmArgs *gs, int n, int precision, cudaStream_t s,
                       int *launched, std::string *err) {
    *launched = 0;
    if (precision == ZRL_GEMM_FP32) {
      for (int i = 0; i < n; ++i) {
        if (gs[i].M <= 0 || gs[i].N <= 0) continue;
        gemm_simt(gs[i], s);
        ++*launched;
      }
      return ZRL_OK;
    }
    if (!tc_ready) {
      zrl_status st = gemm_tc_init(0, err);
      if (st != ZRL_OK) return st;
      tc_ready = true;
    }
    return gemm_tc_group(this, gs, n, precision, s, launched, err);
  }
};

}  // namespace zrl
