// noalloc.cu -- GAE plus advantage normalization without any allocation.
//
// Some callers cannot allocate device memory at the point where they need
// advantages: a trainer whose GPU memory is owned by another runtime's
// pooled allocator, or a host that forbids allocation inside its real-time
// loop.  zrl_gae_normalize_noalloc serves them: it
// takes only caller-owned device buffers and keeps its reduction scratch
// (per-block partial sums, the two advantage moments, mean and standard
// deviation) in the file-scope array below.
//
// Properties a caller must know:
//  * The array lives on every GPU that loads this library, for the life of
//    the process: kScratchDoubles doubles (about 67 KB).
//  * It bounds the problem size: n_envs <= kMaxEnvs (one partial per 32
//    envs); larger calls are rejected with ZRL_INVALID_ARG.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make
//    that first call before any stream capture begins on the device.  The
//    cached address belongs
//    to the device's current context: after cudaDeviceReset on that device
//    it is stale, so a process that resets a device must not call this entry
//    point on it again.
//  * All calls share the one array.  Every slot a call reads is written
//    earlier in the same call, so nothing has to start at zero, but two
//    calls that overlap on the GPU (different streams, or different host
//    threads, without ordering between them) race on the array.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "zrl_internal.h"

namespace zrl {
namespace {

constexpr int kGaeEnvsPerBlock = 32;   // must match the GAE kernel's block
constexpr int kMaxGaeBlocks = 8192;
constexpr int64_t kMaxEnvs = (int64_t)kMaxGaeBlocks * kGaeEnvsPerBlock;
constexpr int kMaxSqdevBlocks = 512;
// [GAE partials | sq-dev partials | moments (2) | DevState]
constexpr int kMomentsAt = kMaxGaeBlocks + kMaxSqdevBlocks;
constexpr int kStateAt = kMomentsAt + 2;
constexpr int kStateDoubles = (int)((sizeof(DevState) + sizeof(double) - 1) / sizeof(double));
constexpr int kScratchDoubles = kStateAt + kStateDoubles;

static __device__ __align__(256) double g_noalloc_scratch[kScratchDoubles];

__global__ void normalize_adv_kernel(const float *adv, int64_t n, const DevState *st,
                                     float *out) {
  const float mean = st->adv_mean, sd = st->adv_sd;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fdiv_rn(__fsub_rn(adv[i], mean), sd);  // ppo.rs:346-348
}

std::mutex g_mu;
double *g_addr[64] = {};

// Device address of the scratch array on the current device (looked up
// once per device).
zrl_status scratch_address(double **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ZRL_CUDA_ERROR;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p)
      return ZRL_CUDA_ERROR;
    g_addr[dev] = static_cast<double *>(p);
  }
  *out = g_addr[dev];
  return ZRL_OK;
}

}  // namespace
}  // namespace zrl

using namespace zrl;

extern "C" zrl_status zrl_gae_normalize_noalloc(
    const float *rewards, const float *values, const uint8_t *dones,
    const float *last_values, int64_t n_envs, int64_t T, float gamma, float lam,
    float *adv_out, float *ret_out, float *adv_norm_out, void *stream) {
  if (!rewards || !values || !dones || !last_values || !adv_out || !ret_out || !adv_norm_out)
    return ZRL_INVALID_ARG;
  if (n_envs < 0 || T < 0) return ZRL_INVALID_ARG;
  if (n_envs > kMaxEnvs) return ZRL_INVALID_ARG;  // scratch holds kMaxEnvs/32 partials
  if (T > 4096) return ZRL_INVALID_ARG;
  if (n_envs == 0 || T == 0) return ZRL_OK;
  double *scratch = nullptr;
  zrl_status s = scratch_address(&scratch);
  if (s != ZRL_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  double *gae_part = scratch;
  double *sq_part = scratch + kMaxGaeBlocks;
  double *moments = scratch + kMomentsAt;
  DevState *state = reinterpret_cast<DevState *>(scratch + kStateAt);
  const int64_t n = n_envs * T;
  GaeArgs a{};
  a.rewards = rewards;
  a.values = values;
  a.dones = dones;
  a.last_values = last_values;
  a.adv = adv_out;
  a.ret = ret_out;
  a.n_envs = n_envs;
  a.T = T;
  a.gamma = gamma;
  a.lam = lam;
  const int gb = gae_blocks(n_envs);  // one partial per GAE block
  if (gb > kMaxGaeBlocks) return ZRL_INVALID_ARG;
  launch_gae(a, gae_part, gb, st);
  launch_reduce_moment(gae_part, gb, moments, 0, st);
  int sb = adv_blocks(n);
  if (sb > kMaxSqdevBlocks) sb = kMaxSqdevBlocks;
  launch_adv_sqdev(adv_out, n, moments, n, sq_part, sb, st);
  launch_reduce_moment(sq_part, sb, moments, 1, st);
  launch_adv_finalize(moments, n, state, st);
  normalize_adv_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 1184), 256, 0, st>>>(
      adv_out, n, state, adv_norm_out);
  if (cudaGetLastError() != cudaSuccess) return ZRL_CUDA_ERROR;
  return ZRL_OK;
}
