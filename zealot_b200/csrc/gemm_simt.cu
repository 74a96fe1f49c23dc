// gemm_simt.cu -- fp32 CUDA-core GEMM with the MLP epilogues.
//
// This is the exact-arithmetic mode (ZRL_GEMM_FP32): every product is an
// fp32 FMA, so results differ from the reference's sequential dot products
// (net.rs:97-104, 127-136) only by summation order.  The tensor-core tf32
// kernels (gemm_tc.cu) are the fast path.
//
// Shapes used by the PPO update (sample-major activations, W [out, in]):
//   forward  Z[mb, out] = X[mb, in] * W^T        A=X,          B=W (trans_b)
//   dgrad    D[mb, in]  = Delta[mb, out] * W     A=Delta,      B=W
//   wgrad    dW[out,in] = Delta^T * X            A=Delta (trans_a), B=X
#include <cuda_runtime.h>

#include "zrl_internal.h"

namespace zrl {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;
constexpr int kThreads = (BM / TM) * (BN / TN);  // 256

template <bool TA, bool TB, int EPI>
__global__ void __launch_bounds__(kThreads)
sgemm_kernel(GemmArgs g) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int t = threadIdx.x;
  const int tx = t % (BN / TN), ty = t / (BN / TN);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  int kc = (g.K + g.split_k - 1) / g.split_k;
  kc = (kc + BK - 1) / BK * BK;
  const int kb = blockIdx.z * kc;
  const int ke = min(g.K, kb + kc);
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  for (int k0 = kb; k0 < ke; k0 += BK) {
#pragma unroll
    for (int r = 0; r < (BM * BK) / kThreads; ++r) {
      const int idx = t + r * kThreads;
      int ml, kl;
      if (TA) {
        kl = idx / BM;
        ml = idx % BM;
      } else {
        ml = idx / BK;
        kl = idx % BK;
      }
      const int m = m0 + ml, k = k0 + kl;
      float v = 0.0f;
      if (m < g.M && k < ke)
        v = TA ? g.A[(int64_t)k * g.lda + m] : g.A[(int64_t)m * g.lda + k];
      As[kl][ml] = v;
    }
#pragma unroll
    for (int r = 0; r < (BN * BK) / kThreads; ++r) {
      const int idx = t + r * kThreads;
      int nl, kl;
      if (TB) {
        nl = idx / BK;
        kl = idx % BK;
      } else {
        kl = idx / BN;
        nl = idx % BN;
      }
      const int n = n0 + nl, k = k0 + kl;
      float v = 0.0f;
      if (n < g.N && k < ke)
        v = TB ? g.B[(int64_t)n * g.ldb + k] : g.B[(int64_t)k * g.ldb + n];
      Bs[kl][nl] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

  float *C = g.C + (int64_t)blockIdx.z * g.M * g.ldc;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty * TM + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx * TN + j;
      if (n >= g.N) continue;
      float v = acc[i][j];
      if (EPI == EPI_BIAS || EPI == EPI_BIAS_ELU) v += g.bias[n];
      if (EPI == EPI_BIAS_ELU) v = v > 0.0f ? v : expf(v) - 1.0f;
      if (EPI == EPI_ELU_GRAD) {
        const float y = g.aux[(int64_t)m * g.ldaux + n];
        v *= y > 0.0f ? 1.0f : y + 1.0f;  // net.rs:21-23
      }
      C[(int64_t)m * g.ldc + n] = v;
    }
  }
}

template <bool TA, bool TB>
void dispatch_epi(const GemmArgs &g, dim3 grid, cudaStream_t s) {
  switch (g.epi) {
    case EPI_BIAS: sgemm_kernel<TA, TB, EPI_BIAS><<<grid, kThreads, 0, s>>>(g); break;
    case EPI_BIAS_ELU: sgemm_kernel<TA, TB, EPI_BIAS_ELU><<<grid, kThreads, 0, s>>>(g); break;
    case EPI_ELU_GRAD: sgemm_kernel<TA, TB, EPI_ELU_GRAD><<<grid, kThreads, 0, s>>>(g); break;
    default: sgemm_kernel<TA, TB, EPI_STORE><<<grid, kThreads, 0, s>>>(g); break;
  }
}

}  // namespace

void gemm_simt(const GemmArgs &g, cudaStream_t s) {
  const int split = g.split_k < 1 ? 1 : g.split_k;
  dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, split);
  GemmArgs a = g;
  a.split_k = split;
  if (a.trans_a && a.trans_b) dispatch_epi<true, true>(a, grid, s);
  else if (a.trans_a) dispatch_epi<true, false>(a, grid, s);
  else if (a.trans_b) dispatch_epi<false, true>(a, grid, s);
  else dispatch_epi<false, false>(a, grid, s);
}

}  // namespace zrl
