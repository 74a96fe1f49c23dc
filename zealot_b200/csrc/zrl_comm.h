// zrl_comm.h -- data-parallel gradient exchange over NCCL.
//
// The reference trains on one GPU and has no collective; here the rollout's
// envs are sharded over ranks and the flat gradient (plus the three loss
// sums) is summed with one ncclAllReduce per minibatch, on the compute
// stream.  NCCL is loaded with dlopen so the library has no link-time NCCL
// dependency (a process that already loaded libnccl.so.2, e.g. through
// torch, shares that copy).  Waits on the stream are bounded: a host-side
// poll of the stream and of ncclCommGetAsyncError gives up after the
// configured timeout and aborts the communicator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/zealot_rl.h"

namespace zrl {

zrl_status nccl_unique_id(uint8_t *out, std::string *err);

struct Comm {
  int rank = 0;
  int world = 1;
  int timeout_ms = 60000;
  void *comm = nullptr;  // ncclComm_t
  void *lib = nullptr;
  bool aborted = false;

  zrl_status init(const zrl_comm &c, std::string *err);
  zrl_status allreduce_f32(float *buf, int64_t count, cudaStream_t s,
                           std::string *err);
  zrl_status allreduce_f64(double *buf, int64_t count, cudaStream_t s,
                           std::string *err);
  // Waits for the stream with a deadline; polls the communicator's async
  // error while waiting.  Aborts the communicator on error or timeout.
  zrl_status wait(cudaStream_t s, std::string *err);
  void destroy();
};

// Comm::wait's bounded loop driven by fakes (zrl_comm.cpp), for tests.
zrl_status comm_wait_fake(int scenario, int timeout_ms, int *aborted, std::string *err);

}  // namespace zrl
