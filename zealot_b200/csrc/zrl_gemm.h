// zrl_gemm.h -- GEMM dispatch for the MLP forward/backward.
//
// ZRL_GEMM_FP32 runs the CUDA-core kernel (gemm_simt.cu); ZRL_GEMM_TF32
// runs the tcgen05 tensor-core kernels (gemm_tc.cu).  There is no silent
// substitution: a shape the tensor-core kernel does not take is an error,
// not a fallback.
#pragma once

#include <string>

#include "zrl_internal.h"

namespace zrl {

struct GemmEngine;

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
int gemm_tc_split(GemmEngine *eng, const GemmArgs *gs, int n, int precision, int max_split);

struct GemmEngine {
  bool tc_ready = false;
  void *cache = nullptr;  // tensor-map cache (gemm_tc.cu)
  int *err_dev = nullptr; // device flag set by a timed-out pipeline wait

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

  // Split-K count for a weight-gradient group (see gemm_tc_split); 0 on
  // the CUDA cores, where the caller keeps its own split.
  int split_for(const GemmArgs *gs, int n, int precision, int max_split, std::string *err) {
    if (precision == ZRL_GEMM_FP32) return 0;
    if (!tc_ready) {
      if (gemm_tc_init(0, err) != ZRL_OK) return 0;
      tc_ready = true;
    }
    return gemm_tc_split(this, gs, n, precision, max_split);
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
