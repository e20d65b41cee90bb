// Data parallelism: one process per GPU, NCCL over NVLink/NVSwitch.
//
// The reference has no multi-device layer (docs/milestones/v5-plan.md:66
// defers it).  The nanoGPT workload shards by batch, so each rank runs the
// full replica on its own token slice and the only exchange is a sum
// all-reduce of the fused gradient buffer, issued on a dedicated stream so it
// overlaps the rest of the backward pass; the optimizer then applies 1/world.
//
// The communicator is created non-blocking; every wait on it is bounded
// (the caller's timeout) and ends in ncclCommAbort + an error return instead
// of a hang, so a rank that never joins is detected on the host.
#include "common.cuh"

#include <nccl.h>
#include <chrono>
#include <thread>

namespace malus {
namespace {
ncclComm_t g_comm = nullptr;
cudaStream_t g_dp_stream = nullptr;
cudaEvent_t g_ev_ready = nullptr, g_ev_done = nullptr;
int g_rank = 0, g_world = 1;
int g_timeout_ms = 60000;

int wait_comm(int timeout_ms) {
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st;
    ncclResult_t r = ncclCommGetAsyncError(g_comm, &st);
    if (r != ncclSuccess) return -2;
    if (st == ncclSuccess) return 0;
    if (st != ncclInProgress) {
      fprintf(stderr, "malus: NCCL error: %s\n", ncclGetErrorString(st));
      return -3;
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms) return -4;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void abort_comm() {
  if (g_comm) ncclCommAbort(g_comm);
  g_comm = nullptr;
  g_world = 1;
  g_rank = 0;
}
}  // namespace

cudaStream_t dp_stream() { return g_dp_stream; }
int dp_world() { return g_world; }

// Sum-allreduce `count` floats at `ptr` on the DP stream after all work
// already queued on the main stream; the main stream does not wait here.
int dp_allreduce_async(float* ptr, size_t count) {
  if (g_world <= 1 || !g_comm) return 0;
  MALUS_CUDA(cudaEventRecord(g_ev_ready, stream()));
  MALUS_CUDA(cudaStreamWaitEvent(g_dp_stream, g_ev_ready, 0));
  ncclResult_t r = ncclAllReduce(ptr, ptr, count, ncclFloat, ncclSum, g_comm, g_dp_stream);
  if (r != ncclSuccess && r != ncclInProgress) {
    fprintf(stderr, "malus: ncclAllReduce failed: %s\n", ncclGetErrorString(r));
    return -5;
  }
  if (r == ncclInProgress && wait_comm(g_timeout_ms) != 0) {
    abort_comm();
    return -4;
  }
  return 0;
}

// Make the main stream wait for every collective queued so far.
void dp_join() {
  if (g_world <= 1 || !g_comm) return;
  MALUS_CUDA(cudaEventRecord(g_ev_done, g_dp_stream));
  MALUS_CUDA(cudaStreamWaitEvent(stream(), g_ev_done, 0));
}

}  // namespace malus

using namespace malus;

extern "C" {

int32_t malus_dp_unique_id(uint8_t* out128) {
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return -1;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out128, &id, 128);
  return 0;
}

int32_t malus_dp_init(int32_t rank, int32_t world, const uint8_t* nccl_id, int32_t timeout_ms) {
  if (world <= 1) {
    g_world = 1;
    g_rank = 0;
    return 0;
  }
  stream();  // bind the device first
  if (timeout_ms > 0) g_timeout_ms = timeout_ms;
  ncclUniqueId id;
  memcpy(&id, nccl_id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&g_comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    fprintf(stderr, "malus: ncclCommInitRankConfig failed: %s\n", ncclGetErrorString(r));
    g_comm = nullptr;
    return -1;
  }
  int w = wait_comm(g_timeout_ms);
  if (w != 0) {
    fprintf(stderr, "malus: NCCL communicator init did not complete (%d); aborting it\n", w);
    abort_comm();
    return w;
  }
  if (!g_dp_stream) {
    MALUS_CUDA(cudaStreamCreateWithFlags(&g_dp_stream, cudaStreamNonBlocking));
    MALUS_CUDA(cudaEventCreateWithFlags(&g_ev_ready, cudaEventDisableTiming));
    MALUS_CUDA(cudaEventCreateWithFlags(&g_ev_done, cudaEventDisableTiming));
  }
  g_rank = rank;
  g_world = world;
  return 0;
}

int32_t malus_dp_allreduce_f32(void* dev_ptr, size_t count) {
  int r = dp_allreduce_async((float*)dev_ptr, count);
  if (r) return r;
  dp_join();
  return 0;
}

int32_t malus_dp_finish(void) {
  if (g_world <= 1 || !g_comm) return 0;
  dp_join();
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    // collectives run on the DP stream, or on the main stream inside a
    // replayed CUDA graph of the step: wait (bounded) for both
    cudaError_t q = cudaStreamQuery(g_dp_stream);
    if (q == cudaSuccess) q = cudaStreamQuery(stream());
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return -6;
    ncclResult_t st;
    ncclCommGetAsyncError(g_comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      abort_comm();
      return -3;
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0).count();
    if (ms > g_timeout_ms) {
      abort_comm();
      return -4;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int32_t malus_dp_destroy(void) {
  if (!g_comm) return 0;
  int r = malus_dp_finish();
  if (g_comm) {
    ncclCommFinalize(g_comm);
    wait_comm(g_timeout_ms);
    ncclCommDestroy(g_comm);
  }
  g_comm = nullptr;
  g_world = 1;
  g_rank = 0;
  return r;
}

int32_t malus_dp_world(void) { return g_world; }

// Local teardown after a peer is known to be gone: ncclCommAbort needs no peer.
int32_t malus_dp_abort(void) {
  abort_comm();
  return 0;
}

}  // extern "C"
