// zrl_comm.cpp -- NCCL through dlopen, with bounded waits.
#include "zrl_comm.h"

#include <dlfcn.h>
#include <string.h>

#include <chrono>
#include <thread>

namespace zrl {
namespace {

// The subset of the NCCL C API used here (nccl.h, stable since 2.x).
typedef int nccl_result_t;
typedef struct {
  char internal[128];
} nccl_unique_id_t;
enum { kNcclSum = 0 };
enum { kNcclFloat32 = 7, kNcclFloat64 = 8 };  // ncclFloat, ncclDouble (nccl.h)
enum { kNcclInProgress = 7 };

struct NcclApi {
  nccl_result_t (*get_unique_id)(nccl_unique_id_t *) = nullptr;
  nccl_result_t (*comm_init_rank)(void **, int, nccl_unique_id_t, int) = nullptr;
  nccl_result_t (*all_reduce)(const void *, void *, size_t, int, int, void *,
                              cudaStream_t) = nullptr;
  nccl_result_t (*comm_destroy)(void *) = nullptr;
  nccl_result_t (*comm_abort)(void *) = nullptr;
  nccl_result_t (*async_error)(void *, nccl_result_t *) = nullptr;
  const char *(*error_string)(nccl_result_t) = nullptr;
};

NcclApi g_api;

bool load(void **lib, std::string *err) {
  if (*lib) return true;
  const char *names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char *n : names) {
    *lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (*lib) break;
  }
  if (!*lib) {
    *err = "NCCL not found (dlopen libnccl.so.2 failed)";
    return false;
  }
  auto sym = [&](const char *name) { return dlsym(*lib, name); };
  g_api.get_unique_id = (decltype(g_api.get_unique_id))sym("ncclGetUniqueId");
  g_api.comm_init_rank = (decltype(g_api.comm_init_rank))sym("ncclCommInitRank");
  g_api.all_reduce = (decltype(g_api.all_reduce))sym("ncclAllReduce");
  g_api.comm_destroy = (decltype(g_api.comm_destroy))sym("ncclCommDestroy");
  g_api.comm_abort = (decltype(g_api.comm_abort))sym("ncclCommAbort");
  g_api.async_error = (decltype(g_api.async_error))sym("ncclCommGetAsyncError");
  g_api.error_string = (decltype(g_api.error_string))sym("ncclGetErrorString");
  if (!g_api.get_unique_id || !g_api.comm_init_rank || !g_api.all_reduce || !g_api.comm_destroy ||
      !g_api.comm_abort || !g_api.async_error) {
    *err = "NCCL library lacks required symbols";
    return false;
  }
  return true;
}

std::string nccl_msg(const char *what, nccl_result_t r) {
  std::string m = std::string(what) + " failed: NCCL error " + std::to_string(r);
  if (g_api.error_string) m += std::string(" (") + g_api.error_string(r) + ")";
  return m;
}

}  // namespace

static void *g_lib = nullptr;

zrl_status nccl_unique_id(uint8_t *out, std::string *err) {
  if (!load(&g_lib, err)) return ZRL_NCCL_ERROR;
  nccl_unique_id_t id;
  nccl_result_t r = g_api.get_unique_id(&id);
  if (r != 0) {
    *err = nccl_msg("ncclGetUniqueId", r);
    return ZRL_NCCL_ERROR;
  }
  memcpy(out, id.internal, 128);
  return ZRL_OK;
}

zrl_status Comm::init(const zrl_comm &c, std::string *err) {
  if (c.world_size < 1 || c.rank < 0 || c.rank >= c.world_size) {
    *err = "invalid rank/world_size";
    return ZRL_INVALID_ARG;
  }
  rank = c.rank;
  world = c.world_size;
  timeout_ms = c.timeout_ms > 0 ? c.timeout_ms : 60000;
  if (world == 1) return ZRL_OK;
  if (!load(&lib, err)) return ZRL_NCCL_ERROR;
  nccl_unique_id_t id;
  memcpy(id.internal, c.nccl_id, 128);
  nccl_result_t r = g_api.comm_init_rank(&comm, world, id, rank);
  if (r != 0) {
    *err = nccl_msg("ncclCommInitRank", r);
    comm = nullptr;
    return ZRL_NCCL_ERROR;
  }
  return ZRL_OK;
}

static zrl_status do_allreduce(Comm *c, void *buf, int64_t count, int dtype,
                               cudaStream_t s, std::string *err) {
  if (c->world <= 1 || count <= 0) return ZRL_OK;
  if (!c->comm || c->aborted) {
    *err = "communicator unavailable";
    return ZRL_NCCL_ERROR;
  }
  nccl_result_t r = g_api.all_reduce(buf, buf, (size_t)count, dtype, kNcclSum,
                                     c->comm, s);
  if (r != 0) {
    *err = nccl_msg("ncclAllReduce", r);
    return ZRL_NCCL_ERROR;
  }
  return ZRL_OK;
}

zrl_status Comm::allreduce_f32(float *buf, int64_t count, cudaStream_t s,
                               std::string *err) {
  return do_allreduce(this, buf, count, kNcclFloat32, s, err);
}

zrl_status Comm::allreduce_f64(double *buf, int64_t count, cudaStream_t s,
                               std::string *err) {
  return do_allreduce(this, buf, count, kNcclFloat64, s, err);
}

// The bounded wait of Comm::wait over its three effects, so the failure
// paths can be driven by fakes: query() is cudaStreamQuery of the stream,
// async_err() the communicator's asynchronous error (0 or in progress:
// none), abort() aborts the communicator.
template <typename Query, typename AsyncErr, typename Abort>
static zrl_status wait_loop(int timeout_ms, Query query, AsyncErr async_err, Abort abort,
                            std::string *err) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = query();
    if (q == cudaSuccess) return ZRL_OK;
    if (q != cudaErrorNotReady) {
      *err = std::string("stream: ") + cudaGetErrorString(q);
      return ZRL_CUDA_ERROR;
    }
    const nccl_result_t ae = async_err();
    if (ae != 0 && ae != kNcclInProgress) {
      *err = nccl_msg("NCCL async", ae);
      abort();
      return ZRL_NCCL_ERROR;
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > timeout_ms) {
      *err = "timed out waiting for the stream (a peer rank may be gone)";
      abort();
      return ZRL_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

zrl_status Comm::wait(cudaStream_t s, std::string *err) {
  return wait_loop(
      timeout_ms, [&] { return cudaStreamQuery(s); },
      [&]() -> nccl_result_t {
        nccl_result_t ae = 0;
        if (world > 1 && comm) g_api.async_error(comm, &ae);
        return ae;
      },
      [&] {
        if (world > 1 && comm) {
          g_api.comm_abort(comm);
          aborted = true;
        }
      },
      err);
}

// Comm::wait's failure paths on fakes (no GPU, no NCCL): scenario 0 the
// stream completes on the fifth poll; 1 it never completes; 2 the
// communicator reports an asynchronous error on the third poll; 3 the
// stream reports a failed kernel.  *aborted receives whether the
// communicator would have been aborted.
zrl_status comm_wait_fake(int scenario, int timeout_ms, int *aborted, std::string *err) {
  int polls = 0;
  *aborted = 0;
  return wait_loop(
      timeout_ms,
      [&]() -> cudaError_t {
        ++polls;
        if (scenario == 0 && polls >= 5) return cudaSuccess;
        if (scenario == 3) return cudaErrorLaunchFailure;
        return cudaErrorNotReady;
      },
      [&]() -> nccl_result_t { return scenario == 2 && polls >= 3 ? 3 /* internal error */ : 0; },
      [&] { *aborted = 1; }, err);
}

void Comm::destroy() {
  if (comm) {
    if (aborted)
      ;  // ncclCommAbort already released it
    else
      g_api.comm_destroy(comm);
  }
  comm = nullptr;
}

}  // namespace zrl
