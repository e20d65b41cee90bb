// Embedding backward that allocates nothing.
//
// Some callers cannot call cudaMalloc at the point where they need this op:
// code running inside a CUDA stream capture of a training step that must not
// add memory nodes, an allocator-less embedding of the runtime in another
// framework's memory arena, or a caller holding a memory budget that is
// already fully committed.  For them this entry point computes the same
// deterministic sort-then-segmented-sum embedding gradient as
// __embedding_bwd, but all of its scratch lives in one file-scope device
// array of fixed size; the caller passes the inputs, the output and the
// stream.  It calls no cudaMalloc/cudaFree and no allocating library routine,
// and it does not touch the runtime's own context (pool, error word, stream).
// Because of that, an id outside [0, vocab) is skipped without a report: its
// row of dout contributes to no gradient row, and the call still returns 0
// (the allocating __embedding_bwd reports such ids through the runtime's
// error word).
//
// The array exists on every GPU that loads this library, for the life of the
// process.  All calls share it: two calls that overlap on the GPU (different
// streams, no ordering between them) race on it.  What must start at zero (the
// per-bucket counts) is cleared by each call on the caller's stream.
#include "common.cuh"

#include <mutex>

namespace malus {
namespace {

// Limits: at most kMaxTokens ids per call, and vocab * ceil(n / 1024) at most
// kMaxBuckets (the per-chunk run counts and their offsets).
constexpr size_t kMaxTokens = 65536;
constexpr size_t kMaxBuckets = 524288;
constexpr size_t kA256(size_t b) { return (b + 255) & ~size_t(255); }
constexpr size_t kScratchBytes =
    256 + kA256((kMaxTokens / 1024) * 1024 * 8) + kA256(kMaxBuckets * 4) +
    kA256((kMaxBuckets + 1) * 4) + kA256(kMaxTokens * 4) + kA256((kMaxBuckets / 4096 + 1) * 4);

__device__ __align__(256) unsigned char g_emb_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[64] = {nullptr};  // device address of the array, per device ordinal

// Set-up, once per device, with that device current: the host-side name of a
// __device__ array is not a device address, so fetch the real one.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    fprintf(stderr, "malus: embedding_bwd_noalloc: cudaGetDevice failed\n");
    return -7;
  }
  if (dev < 0 || dev >= 64) {
    fprintf(stderr, "malus: embedding_bwd_noalloc: device ordinal %d is outside 0..63\n", dev);
    return -7;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_emb_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "malus: embedding_bwd_noalloc: cudaGetSymbolAddress failed: %s\n",
              cudaGetErrorString(e));
      return -7;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return 0;
}

}  // namespace
}  // namespace malus

extern "C" int32_t malus_embedding_bwd_noalloc(const float* dout, const void* indices,
                                               int32_t index_dtype, size_t n, size_t vocab,
                                               size_t dim, float* dweight, void* stream) {
  using namespace malus;
  if (index_dtype != MALUS_I32 && index_dtype != MALUS_I64) {
    fprintf(stderr, "malus: embedding_bwd_noalloc: index dtype %d is not i32 (5) or i64 (6)\n",
            index_dtype);
    return -1;
  }
  if (n > kMaxTokens) {
    fprintf(stderr, "malus: embedding_bwd_noalloc: %zu ids exceed the maximum of %zu per call\n",
            n, kMaxTokens);
    return -2;
  }
  size_t buckets = vocab * ((n + 1023) / 1024);
  if (buckets > kMaxBuckets) {
    fprintf(stderr,
            "malus: embedding_bwd_noalloc: vocab %zu x %zu id chunks = %zu buckets exceed the "
            "maximum of %zu\n", vocab, (n + 1023) / 1024, buckets, kMaxBuckets);
    return -3;
  }
  if (embedding_bwd_ws_bytes(n, vocab) > kScratchBytes) return -3;
  void* ws = nullptr;
  int r = scratch_address(&ws);
  if (r) return r;
  return embedding_bwd_ws(dout, indices, index_dtype, dweight, n, vocab, dim, ws,
                          (cudaStream_t)stream, nullptr);
}
