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
#include <unordered_map>
#include <vector>

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
  const int pid = prof_begin_on(3, 0.0, 4.0 * (double)count, g_dp_stream);
  ncclResult_t r = ncclAllReduce(ptr, ptr, count, ncclFloat, ncclSum, g_comm, g_dp_stream);
  if (r != ncclSuccess && r != ncclInProgress) {
    fprintf(stderr, "malus: ncclAllReduce failed: %s\n", ncclGetErrorString(r));
    return -5;
  }
  if (r == ncclInProgress && wait_comm(g_timeout_ms) != 0) {
    abort_comm();
    return -4;
  }
  // a non-blocking communicator enqueues the collective's kernel only when the
  // operation has left ncclInProgress: the closing event goes after that
  prof_end_on(pid, g_dp_stream);
  return 0;
}

// Make the main stream wait for every collective queued so far.
void dp_join() {
  if (g_world <= 1 || !g_comm) return;
  MALUS_CUDA(cudaEventRecord(g_ev_done, g_dp_stream));
  const int pid = prof_begin(4, 0.0, 0.0);   // from here to the end of the wait: exposed communication
  MALUS_CUDA(cudaStreamWaitEvent(stream(), g_ev_done, 0));
  prof_end(pid);
}

// ---- per-leaf readiness (malus_dp_register_leaves / malus_dp_grad_ready) ----
// Registered leaves are grouped, in registration order, into buckets of at
// least `bucket_bytes`.  A leaf becomes ready when its gradient is final; when
// the last leaf of a bucket is ready, the bucket's gradients are averaged in
// place across ranks by one grouped NCCL all-reduce on the DP stream, after
// everything already queued on the main stream (the gradients' producers).
// Every rank reports the same leaves in the same order (the tape walk is
// deterministic), so every rank launches the same buckets in the same order.
namespace {
struct DpLeafReg {
  std::unordered_map<int64_t, int> bucket_of;      // leaf -> bucket
  std::vector<int> need;                           // leaves per bucket
  std::vector<int> have;                           // reported in this backward pass
  std::vector<std::vector<std::pair<float*, size_t>>> pending;   // gradients per bucket
  std::vector<int64_t> held;                       // gradient handles retained until dp_leaves_join
  std::vector<int64_t> first_leaf;                 // one leaf of each bucket
};
DpLeafReg g_reg;
}  // namespace

bool dp_leaves_registered() { return g_world > 1 && g_comm && !g_reg.bucket_of.empty(); }
bool dp_is_leaf(int64_t h) { return g_reg.bucket_of.count(h) > 0; }

int dp_leaf_ready(int64_t leaf, int64_t grad) {
  if (g_world <= 1 || !g_comm) return 0;
  auto it = g_reg.bucket_of.find(leaf);
  if (it == g_reg.bucket_of.end()) return -7;
  const int b = it->second;
  if (grad) {
    tensor_retain(grad);
    g_reg.held.push_back(grad);
    g_reg.pending[(size_t)b].emplace_back(fptr(grad), tb(grad)->len);
  }
  if (++g_reg.have[(size_t)b] < g_reg.need[(size_t)b]) return 0;
  // the bucket is complete: one grouped all-reduce of its gradients
  auto& items = g_reg.pending[(size_t)b];
  g_reg.have[(size_t)b] = 0;
  if (items.empty()) return 0;
  MALUS_CUDA(cudaEventRecord(g_ev_ready, stream()));
  MALUS_CUDA(cudaStreamWaitEvent(g_dp_stream, g_ev_ready, 0));
  double bytes = 0.0;
  for (auto& pc : items) bytes += 4.0 * (double)pc.second;
  const int pid = prof_begin_on(3, 0.0, bytes, g_dp_stream);
  ncclResult_t r = ncclGroupStart();
  for (auto& pc : items)
    if (r == ncclSuccess || r == ncclInProgress)
      r = ncclAllReduce(pc.first, pc.first, pc.second, ncclFloat, ncclAvg, g_comm, g_dp_stream);
  ncclResult_t e = ncclGroupEnd();
  items.clear();
  if ((r != ncclSuccess && r != ncclInProgress) || (e != ncclSuccess && e != ncclInProgress)) {
    fprintf(stderr, "malus: bucket all-reduce failed: %s\n", ncclGetErrorString(r != ncclSuccess ? r : e));
    return -5;
  }
  if ((r == ncclInProgress || e == ncclInProgress) && wait_comm(g_timeout_ms) != 0) {
    abort_comm();
    return -4;
  }
  prof_end_on(pid, g_dp_stream);
  return 0;
}

// Launch every bucket that was only partly reported in this backward pass (its other
// leaves received no gradient), make the main stream wait for all the
// bucket reductions, and drop the gradients' extra references.
int dp_leaves_join() {
  if (!dp_leaves_registered()) return 0;
  int rc = 0;
  for (size_t b = 0; b < g_reg.need.size() && rc == 0; ++b)
    if (g_reg.have[b] != 0) {
      g_reg.have[b] = g_reg.need[b] - 1;
      rc = dp_leaf_ready(g_reg.first_leaf[b], 0);
    }
  dp_join();
  for (int64_t h : g_reg.held) tensor_release(h);
  g_reg.held.clear();
  return rc;
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

int32_t malus_dp_register_leaves(const int64_t* leaves, size_t n, size_t bucket_bytes) {
  g_reg = DpLeafReg();
  size_t acc = 0;
  int b = -1;
  for (size_t i = 0; i < n; ++i) {
    if (b < 0 || acc >= bucket_bytes) {
      ++b;
      acc = 0;
      g_reg.need.push_back(0);
      g_reg.have.push_back(0);
      g_reg.pending.emplace_back();
      g_reg.first_leaf.push_back(leaves[i]);
    }
    if (!g_reg.bucket_of.emplace(leaves[i], b).second) {
      g_reg = DpLeafReg();
      return -1;   // a leaf listed twice
    }
    g_reg.need[(size_t)b]++;
    acc += tb(leaves[i])->len * 4;
  }
  return b + 1;   // number of buckets
}

int32_t malus_dp_grad_ready(int64_t leaf, int64_t grad) { return dp_leaf_ready(leaf, grad); }

// Local teardown after a peer is known to be gone: ncclCommAbort needs no peer.
int32_t malus_dp_abort(void) {
  abort_comm();
  return 0;
}

}  // extern "C"
