// Runtime core: device selection, the stream, the buffer pool, tensor handle
// lifetime, host access, RNG, host staging buffers, counters and the bench
// timer.  Semantics follow crates/malus-runtime/src/metal.rs (allocation,
// refcounting, reshape aliasing, Philox RNG, causal mask), buffer.rs,
// bench.rs and lib.rs; the mechanisms are CUDA-native:
//  - one non-blocking stream per process (process-per-GPU, so the
//    reference's single-consumer context, ADR-0033, holds);
//  - a stream-ordered exact-size free-list pool: a buffer released on the
//    host can be handed out again at once, because every later use is
//    queued behind every earlier use on the same stream (this replaces the
//    generation gating of metal.rs:364-456);
//  - host reads synchronise the stream (replaces flush_if_pending).
#include "common.cuh"

#include <chrono>

#include <cmath>
#include <cstdarg>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace malus {

void panic(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  fprintf(stderr, "malus: ");
  vfprintf(stderr, fmt, ap);
  fprintf(stderr, "\n");
  va_end(ap);
  fflush(stderr);
  abort();
}

size_t dtype_size(int32_t dtype) {
  switch (dtype) {
    case 0: case 5: case 9: return 4;
    case 1: case 2: case 4: case 8: return 2;
    case 3: case 7: return 1;
    case 6: case 10: return 8;
    default: panic("unknown dtype tag %d", dtype);
  }
}

// ------------------------------------------------------------------ context
namespace {
struct Context {
  bool init = false;
  int device = 0;
  cudaStream_t stream = nullptr;
  int32_t* d_error = nullptr;  // device error word (bounded waits)
  std::mutex mu;
};
Context g_ctx;

std::atomic<int64_t> g_launches{0};
std::atomic<int64_t> g_retains{0}, g_releases{0}, g_allocs{0};
bool g_sync_dispatch = false;

void ensure_init() {
  if (g_ctx.init) return;
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (g_ctx.init) return;
  int dev = 0;
  if (const char* s = getenv("MALUS_DEVICE")) dev = atoi(s);
  else if (const char* s = getenv("LOCAL_RANK")) dev = atoi(s);
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
    panic("no CUDA device available (this runtime has no CPU fallback)");
  if (dev >= n) dev = dev % n;
  MALUS_CUDA(cudaSetDevice(dev));
  MALUS_CUDA(cudaStreamCreateWithFlags(&g_ctx.stream, cudaStreamNonBlocking));
  MALUS_CUDA(cudaMalloc(&g_ctx.d_error, 256));
  MALUS_CUDA(cudaMemset(g_ctx.d_error, 0, 256));
  const char* sd = getenv("MALUS_SYNC_DISPATCH");
  g_sync_dispatch = sd && sd[0] == '1';
  g_ctx.device = dev;
  g_ctx.init = true;
}
}  // namespace

cudaStream_t stream() {
  ensure_init();
  return g_ctx.stream;
}
int32_t* device_error_word() { ensure_init(); return g_ctx.d_error; }
bool sync_dispatch() { return g_sync_dispatch; }
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void after_launch(const char* what) {
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) panic("kernel launch failed (%s): %s", what, cudaGetErrorString(e));
  if (g_sync_dispatch) {
    e = cudaStreamSynchronize(g_ctx.stream);
    if (e != cudaSuccess) panic("kernel %s failed: %s", what, cudaGetErrorString(e));
  }
}

// --------------------------------------------------------------------- pool
namespace {
struct Pool {
  std::mutex mu;
  std::unordered_map<size_t, std::vector<void*>> free_lists;
  int64_t hits = 0, misses = 0, pooled = 0, live = 0, peak = 0;
  int64_t budget = -1;
};
Pool g_pool;

size_t bucket_of(size_t bytes) {
  if (bytes == 0) bytes = 1;  // metal.rs:389-392: 1-byte placeholder for empty tensors
  return (bytes + 511) & ~size_t(511);
}

int64_t budget_bytes() {
  if (g_pool.budget < 0) {
    const char* s = getenv("MALUS_MEM_BUDGET_MB");
    g_pool.budget = s ? (int64_t)atoll(s) << 20 : 0;  // 0 = unlimited
  }
  return g_pool.budget;
}

bool capturing() {
  cudaStreamCaptureStatus st;
  if (cudaStreamIsCapturing(g_ctx.stream, &st) != cudaSuccess) return false;
  return st != cudaStreamCaptureStatusNone;
}

// Graph capture (malus_graph_begin .. malus_graph_end).  While the runtime
// stream is being captured, buffers freed go to the session's own free lists
// (reusable by later allocations of the same capture: one stream, so the
// graph runs them in capture order) instead of the pool, and every buffer
// handed out is recorded.  At the end the graph keeps all of them: a buffer
// the graph touches is never given to another tensor while the graph exists
// (a release of such a buffer is deferred to malus_graph_destroy).
struct GraphRec;
struct CaptureSession {
  bool active = false;
  int64_t launches_at_begin = 0;   // launch counter when the capture opened
  std::unordered_map<size_t, std::vector<void*>> free_lists;
  std::vector<std::pair<void*, size_t>> touched;
};
CaptureSession g_cap;                           // guarded by g_pool.mu
std::unordered_map<void*, GraphRec*> g_pinned;  // buffer -> graph that uses it (g_pool.mu)

struct GraphRec {
  cudaGraphExec_t exec = nullptr;
  int64_t launches = 0;    // kernels the graph holds (counted per replay)
  std::vector<std::pair<void*, size_t>> held;   // buffers returned to the pool at destroy
  std::vector<void*> pinned;
};

void trim_pool_locked() {
  if (capturing()) return;
  MALUS_CUDA(cudaStreamSynchronize(g_ctx.stream));
  for (auto& kv : g_pool.free_lists)
    for (void* p : kv.second) {
      MALUS_CUDA(cudaFree(p));
      g_pool.pooled -= (int64_t)kv.first;
    }
  g_pool.free_lists.clear();
}

void* pool_get(size_t bytes, size_t* bucket_out) {
  ensure_init();
  size_t b = bucket_of(bytes);
  *bucket_out = b;
  std::lock_guard<std::mutex> lk(g_pool.mu);
  if (g_cap.active) {
    auto ct = g_cap.free_lists.find(b);
    if (ct != g_cap.free_lists.end() && !ct->second.empty()) {
      void* p = ct->second.back();
      ct->second.pop_back();
      g_pool.hits++;
      g_pool.live += (int64_t)b;
      return p;
    }
  }
  auto it = g_pool.free_lists.find(b);
  if (it != g_pool.free_lists.end() && !it->second.empty()) {
    void* p = it->second.back();
    it->second.pop_back();
    g_pool.hits++;
    g_pool.pooled -= (int64_t)b;
    g_pool.live += (int64_t)b;
    if (g_cap.active) g_cap.touched.emplace_back(p, b);
    return p;
  }
  g_pool.misses++;
  int64_t bud = budget_bytes();
  if (bud > 0 && g_pool.live + g_pool.pooled + (int64_t)b > bud) trim_pool_locked();
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, b);
  if (e != cudaSuccess) {
    cudaGetLastError();
    trim_pool_locked();
    e = cudaMalloc(&p, b);
    if (e != cudaSuccess) panic("out of device memory allocating %zu bytes", b);
  }
  g_pool.live += (int64_t)b;
  if (g_pool.live + g_pool.pooled > g_pool.peak) g_pool.peak = g_pool.live + g_pool.pooled;
  if (g_cap.active) g_cap.touched.emplace_back(p, b);
  return p;
}

void pool_put(void* p, size_t bucket) {
  std::lock_guard<std::mutex> lk(g_pool.mu);
  auto pin = g_pinned.find(p);
  if (pin != g_pinned.end()) {          // a captured graph still uses it
    pin->second->held.emplace_back(p, bucket);
    g_pinned.erase(pin);
    g_pool.live -= (int64_t)bucket;
    return;
  }
  if (g_cap.active) {                   // reusable within the capture only
    g_cap.free_lists[bucket].push_back(p);
    g_pool.live -= (int64_t)bucket;
    return;
  }
  g_pool.free_lists[bucket].push_back(p);
  g_pool.live -= (int64_t)bucket;
  g_pool.pooled += (int64_t)bucket;
}
}  // namespace

// Raw pooled workspace for kernels (split operands, sort keys, partial sums).
// Freed back to the pool right after the launches that use it are queued:
// the stream order protects it exactly like a tensor buffer.
static std::mutex g_scratch_mu;
static std::unordered_map<void*, size_t>& scratch_map() {
  static auto* m = new std::unordered_map<void*, size_t>();
  return *m;
}
void* scratch_alloc(size_t bytes) {
  size_t b;
  void* p = pool_get(bytes, &b);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  scratch_map()[p] = b;
  return p;
}
void scratch_free(void* p) {
  if (!p) return;
  size_t b;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto it = scratch_map().find(p);
    if (it == scratch_map().end()) panic("scratch_free of an unknown pointer");
    b = it->second;
    scratch_map().erase(it);
  }
  pool_put(p, b);
}

// ----------------------------------------------------------- tensor handles
static int64_t make_handle(int32_t dtype, const size_t* shape, int ndim, Storage* st, size_t len) {
  auto* t = new TensorBuffer();
  t->st = st;
  t->dtype = dtype;
  t->ndim = ndim;
  t->len = len;
  for (int i = 0; i < ndim; ++i) t->shape[i] = shape[i];
  t->rc.store(1, std::memory_order_relaxed);
  g_allocs.fetch_add(1, std::memory_order_relaxed);
  return reinterpret_cast<int64_t>(t);
}

static std::atomic<uint64_t> g_storage_ids{1};

int64_t alloc(int32_t dtype, const size_t* shape, int ndim) {
  if (dtype != MALUS_F32 && dtype != MALUS_I32 && dtype != MALUS_I64)
    panic("unsupported dtype tag %d; supported: f32, i32, i64", dtype);
  if (ndim > kMaxRank) panic("rank %d exceeds the maximum of %d", ndim, kMaxRank);
  size_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= shape[i];
  size_t bytes = n * dtype_size(dtype);
  auto* st = new Storage();
  st->ptr = pool_get(bytes, &st->bytes);
  st->aliases = 1;
  st->owned = true;
  st->id = g_storage_ids.fetch_add(1, std::memory_order_relaxed);
  return make_handle(dtype, shape, ndim, st, n);
}

int64_t alloc_like(int64_t h) {
  auto* t = tb(h);
  return alloc(MALUS_F32, t->shape, t->ndim);
}

int64_t alloc_f32(std::initializer_list<size_t> shape) {
  size_t s[kMaxRank];
  int n = 0;
  for (size_t d : shape) s[n++] = d;
  return alloc(MALUS_F32, s, n);
}

bool same_shape(int64_t a, int64_t b) {
  auto *x = tb(a), *y = tb(b);
  if (x->ndim != y->ndim) return false;
  for (int i = 0; i < x->ndim; ++i)
    if (x->shape[i] != y->shape[i]) return false;
  return true;
}

int normalize_axis(int64_t axis, int ndim) {
  int64_t a = axis < 0 ? axis + ndim : axis;
  if (a < 0 || a >= ndim) panic("axis %lld is out of range for tensor with %d dimensions",
                                (long long)axis, ndim);
  return (int)a;
}

void split_axis(const Shape& s, int axis, size_t* outer, size_t* axis_sz, size_t* inner) {
  size_t o = 1, in = 1;
  for (int i = 0; i < axis; ++i) o *= s.d[i];
  for (int i = axis + 1; i < s.ndim; ++i) in *= s.d[i];
  *outer = o;
  *axis_sz = s.d[axis];
  *inner = in;
}

static void release_storage(Storage* st) {
  if (--st->aliases > 0) return;
  plane_cache_drop(st->id);
  if (st->owned) pool_put(st->ptr, st->bytes);
  delete st;
}

// ------------------------------------------------------------------- views
static bool reshape_view(const size_t* shape, int ndim, const View& view, const size_t* dims, size_t nd,
                         View* out);

bool view_as(int64_t h, const size_t* dims, size_t nd, View* out) {
  auto* t = tb(h);
  if (t->lazy) materialize(h);
  return t->len && reshape_view(t->shape, t->ndim, view_of(h), dims, nd, out);
}

View view_of(int64_t h) {
  auto* t = tb(h);
  if (t->view) return *t->view;
  View v;
  int64_t stride = 1;
  for (int d = t->ndim - 1; d >= 0; --d) {
    v.d[d] = ViewDim{0, 0, stride};
    stride *= (int64_t)t->shape[d];
  }
  return v;
}

static bool is_row_major(const size_t* shape, int ndim, const View& v) {
  int64_t stride = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (shape[d] != 1 && (v.d[d].div != 0 || v.d[d].lo != stride)) return false;
    stride *= (int64_t)shape[d];
  }
  return true;
}

int64_t make_view(int64_t h, const size_t* shape, int ndim, const View& v) {
  auto* t = tb(h);
  if (t->lazy) materialize(h);
  t->st->aliases++;
  int64_t out = make_handle(t->dtype, shape, ndim, t->st, t->len);
  if (!is_row_major(shape, ndim, v)) tb(out)->view = new View(v);
  return out;
}

struct ViewMeta {
  int ndim;
  int64_t size[kMaxRank];
  ViewDim d[kMaxRank];
};

// out[f] = src[offset of logical element f] (row-major over the logical shape)
template <typename T>
__global__ void k_view_gather(const T* __restrict__ src, T* __restrict__ out, size_t n, ViewMeta m) {
  for (size_t f = blockIdx.x * (size_t)blockDim.x + threadIdx.x; f < n; f += (size_t)gridDim.x * blockDim.x) {
    int64_t rem = (int64_t)f, off = 0;
    for (int d = m.ndim - 1; d >= 0; --d) {
      int64_t i = rem % m.size[d];
      rem /= m.size[d];
      off += m.d[d].at(i);
    }
    out[f] = src[off];
  }
}

// out = src * scale[0] (+ addend[f % add_len]), or src * colscale[f % cs_len],
// the eager ops' roundings
__global__ void k_lazy_eval(const float* __restrict__ src, const float* __restrict__ scale,
                            const float* __restrict__ add, size_t add_len, const float* __restrict__ cs,
                            size_t cs_len, float* __restrict__ out, size_t n) {
  const float sc = scale ? *scale : 1.0f;
  for (size_t f = blockIdx.x * (size_t)blockDim.x + threadIdx.x; f < n; f += (size_t)gridDim.x * blockDim.x) {
    float v = src[f];
    if (scale) v = __fmul_rn(v, sc);
    if (cs) v = __fmul_rn(v, cs[f % cs_len]);
    if (add) v = __fadd_rn(v, add[f % add_len]);
    out[f] = v;
  }
}

int64_t make_lazy(const size_t* shape, int ndim, int64_t src, int64_t scale, int64_t addend,
                  int64_t colscale) {
  size_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= shape[i];
  if (n != tb(src)->len) panic("make_lazy: %zu elements over a %zu-element source", n, tb(src)->len);
  int64_t h = make_handle(MALUS_F32, shape, ndim, nullptr, n);
  tensor_retain(src);
  if (scale) tensor_retain(scale);
  if (addend) tensor_retain(addend);
  if (colscale) tensor_retain(colscale);
  tb(h)->lazy = new Lazy{src, scale, addend, colscale};
  return h;
}

int64_t alias_of(int64_t h) {
  auto* t = tb(h);
  int64_t out;
  if (t->lazy)
    out = make_lazy(t->shape, t->ndim, t->lazy->src, t->lazy->scale, t->lazy->addend, t->lazy->colscale);
  else if (t->view)
    out = make_view(h, t->shape, t->ndim, *t->view);
  else {
    t->st->aliases++;
    out = make_handle(t->dtype, t->shape, t->ndim, t->st, t->len);
  }
  tb(out)->causal_zero = t->causal_zero;
  tb(out)->causal_mask = t->causal_mask;
  return out;
}

static void release_lazy(Lazy* z) {
  tensor_release(z->src);
  if (z->scale) tensor_release(z->scale);
  if (z->addend) tensor_release(z->addend);
  if (z->colscale) tensor_release(z->colscale);
  delete z;
}

void materialize(int64_t h) {
  auto* t = tb(h);
  if (t->lazy) {
    Lazy* z = t->lazy;
    auto* st = new Storage();
    st->ptr = pool_get(t->len * 4, &st->bytes);
    st->aliases = 1;
    st->owned = true;
    st->id = g_storage_ids.fetch_add(1, std::memory_order_relaxed);
    if (t->len) {
      const float* add = z->addend ? fptr(z->addend) : nullptr;
      const float* cs = z->colscale ? fptr(z->colscale) : nullptr;
      k_lazy_eval<<<grid_for(t->len, 256), 256, 0, stream()>>>(
          fptr(z->src), z->scale ? fptr(z->scale) : nullptr, add, add ? tb(z->addend)->len : 1, cs,
          cs ? tb(z->colscale)->len : 1, (float*)st->ptr, t->len);
      count_launch();
      after_launch("k_lazy_eval");
    }
    t->st = st;
    t->lazy = nullptr;
    release_lazy(z);
    return;
  }
  if (!t->view) return;
  ViewMeta m;
  m.ndim = t->ndim;
  for (int d = 0; d < t->ndim; ++d) {
    m.size[d] = (int64_t)t->shape[d];
    m.d[d] = t->view->d[d];
  }
  const size_t es = dtype_size(t->dtype);
  auto* st = new Storage();
  st->ptr = pool_get(t->len * es, &st->bytes);
  st->aliases = 1;
  st->owned = true;
  st->id = g_storage_ids.fetch_add(1, std::memory_order_relaxed);
  if (t->len) {
    if (es == 8)
      k_view_gather<int64_t><<<grid_for(t->len, 256), 256, 0, stream()>>>(
          (const int64_t*)t->st->ptr, (int64_t*)st->ptr, t->len, m);
    else
      k_view_gather<int32_t><<<grid_for(t->len, 256), 256, 0, stream()>>>(
          (const int32_t*)t->st->ptr, (int32_t*)st->ptr, t->len, m);
    count_launch();
    after_launch("k_view_gather");
  }
  release_storage(t->st);
  t->st = st;
  delete t->view;
  t->view = nullptr;
}

// The view of a reshape of a strided view, when the new shape can be read
// from the same memory.  The view's dims are flattened into atoms (extent,
// stride) in row-major order (a two-radix dim gives two), size-1 atoms are
// dropped and adjacent atoms that are contiguous with each other merged; each
// new dim must then be made of at most two consecutive atoms (an atom may be
// split: its leading part strides over the trailing one).  False: not
// expressible (the caller materialises).
static bool reshape_view(const size_t* shape, int ndim, const View& view, const size_t* dims, size_t nd,
                         View* out) {
  std::vector<std::pair<int64_t, int64_t>> at;   // (extent, stride)
  for (int d = 0; d < ndim; ++d) {
    const int64_t n = (int64_t)shape[d];
    if (n == 0) return false;
    const ViewDim vd = view.d[d];
    if (vd.div) {
      if (n % vd.div) return false;
      at.push_back({n / vd.div, vd.hi});
      at.push_back({vd.div, vd.lo});
    } else {
      at.push_back({n, vd.lo});
    }
  }
  std::vector<std::pair<int64_t, int64_t>> a;
  for (auto& x : at) {
    if (x.first == 1) continue;
    if (!a.empty() && a.back().second == x.first * x.second) {
      a.back().first *= x.first;
      a.back().second = x.second;
    } else {
      a.push_back(x);
    }
  }
  size_t ai = 0;
  int64_t rem = a.empty() ? 1 : a[0].first;
  for (size_t k = 0; k < nd; ++k) {
    int64_t need = (int64_t)dims[k];
    if (need == 1) { out->d[k] = ViewDim{0, 0, 0}; continue; }
    int np = 0;
    int64_t pn[2] = {0, 0}, ps[2] = {0, 0};
    while (need > 1) {
      if (ai >= a.size() || np == 2) return false;
      const int64_t st = a[ai].second;
      if (rem <= need) {
        if (need % rem) return false;
        pn[np] = rem; ps[np] = st; ++np;
        need /= rem;
        ++ai;
        rem = ai < a.size() ? a[ai].first : 1;
      } else {
        if (rem % need) return false;
        pn[np] = need; ps[np] = st * (rem / need); ++np;
        rem /= need;
        need = 1;
      }
    }
    if (np == 1 || ps[0] == pn[1] * ps[1]) out->d[k] = ViewDim{0, 0, np == 1 ? ps[0] : ps[1]};
    else out->d[k] = ViewDim{pn[1], ps[0], ps[1]};
  }
  return ai >= a.size();
}

}  // namespace malus

using namespace malus;

// ============================================================ C ABI: section 1
extern "C" {

int64_t tensor_alloc_gpu(int32_t dtype, const size_t* shape, size_t ndims, const float* data) {
  if (data && capturing())
    panic("tensor_alloc_gpu with host data during graph capture: upload into an existing tensor "
          "(malus_tensor_write) before malus_graph_replay instead");
  int64_t h = alloc(dtype, shape, (int)ndims);
  auto* t = tb(h);
  if (data && t->len > 0) {
    MALUS_CUDA(cudaMemcpyAsync(t->st->ptr, data, t->len * dtype_size(dtype),
                               cudaMemcpyHostToDevice, stream()));
    // The source is caller-owned pageable memory that may die right after
    // this call; the copy above is staged before it returns, which is what
    // the reference's immediate memcpy into a shared buffer guarantees.
  }
  return h;
}

int64_t tensor_alloc_zeros_gpu(const size_t* shape, size_t ndims) {
  int64_t h = alloc(MALUS_F32, shape, (int)ndims);
  auto* t = tb(h);
  MALUS_CUDA(cudaMemsetAsync(t->st->ptr, 0, std::max<size_t>(t->len * 4, 1), stream()));
  return h;
}

int64_t tensor_alloc_ones_gpu(const size_t* shape, size_t ndims) {
  int64_t h = alloc(MALUS_F32, shape, (int)ndims);
  auto* t = tb(h);
  if (t->len) scalar_op_imm(kSFill, nullptr, 1.0f, fptr(h), t->len);
  return h;
}

void tensor_retain(int64_t h) {
  if (h == 0) return;
  g_retains.fetch_add(1, std::memory_order_relaxed);
  tb(h)->rc.fetch_add(1, std::memory_order_relaxed);
}

void tensor_release(int64_t h) {
  if (h == 0) return;
  g_releases.fetch_add(1, std::memory_order_relaxed);
  auto* t = tb(h);
  int64_t prev = t->rc.fetch_sub(1, std::memory_order_acq_rel);
  if (prev <= 0)
    panic("over-release of tensor handle %#llx (refcount already zero) — likely a "
          "borrow-inference or tape-retain bug", (unsigned long long)h);
  if (prev == 1) {
    tape_on_release(h);
    if (t->lazy) release_lazy(t->lazy);
    else release_storage(t->st);
    delete t->view;
    delete t;
  }
}

void tensor_free(int64_t h) { tensor_release(h); }

int64_t tensor_len(int64_t h) { return (int64_t)tb(h)->len; }
int64_t tensor_ndim(int64_t h) { return (int64_t)tb(h)->ndim; }
int64_t tensor_dim(int64_t h, int64_t i) {
  auto* t = tb(h);
  int64_t idx = i < 0 ? i + t->ndim : i;
  if (idx < 0 || idx >= t->ndim)
    panic("tensor_dim index %lld out of range for rank-%d tensor", (long long)i, t->ndim);
  return (int64_t)t->shape[idx];
}

static void print_rec(const void* data, int32_t dtype, const size_t* shape, int ndim, size_t off) {
  auto pv = [&](size_t i) {
    if (dtype == MALUS_I32) printf("%d", ((const int32_t*)data)[i]);
    else if (dtype == MALUS_I64) printf("%lld", (long long)((const int64_t*)data)[i]);
    else printf("%g", (double)((const float*)data)[i]);
  };
  if (ndim == 0) { pv(off); return; }
  size_t stride = 1;
  for (int i = 1; i < ndim; ++i) stride *= shape[i];
  printf("[");
  for (size_t i = 0; i < shape[0]; ++i) {
    if (i) printf(", ");
    if (ndim == 1) pv(off + i);
    else print_rec(data, dtype, shape + 1, ndim - 1, off + i * stride);
  }
  printf("]");
}

void tensor_print(int64_t h) {
  if (h == 0) { printf("[]"); return; }
  auto* t = tb(h);
  std::vector<char> buf(std::max<size_t>(t->len * dtype_size(t->dtype), 1));
  malus_tensor_read(h, buf.data(), t->len * dtype_size(t->dtype));
  print_rec(buf.data(), t->dtype, t->shape, t->ndim, 0);
  fflush(stdout);
}

void gpu_barrier(void) {
  if (capturing())
    panic("host read or synchronisation during graph capture (between malus_graph_begin and "
          "malus_graph_end): read results after malus_graph_replay instead");
  cudaError_t e = cudaStreamSynchronize(stream());
  if (e != cudaSuccess)
    panic("GPU stream failed: %s (set MALUS_SYNC_DISPATCH=1 to attribute the failing op)",
          cudaGetErrorString(e));
}

float malus_tensor_get_f32(int64_t h, int64_t idx) {
  auto* t = tb(h);
  if (idx < 0 || (size_t)idx >= t->len)
    panic("tensor_get_f32 index %lld out of range for length %zu", (long long)idx, t->len);
  float v;
  MALUS_CUDA(cudaMemcpyAsync(&v, fptr(h) + idx, 4, cudaMemcpyDeviceToHost, stream()));
  gpu_barrier();
  return v;
}

int64_t tensor_reshape(int64_t h, const size_t* dims, size_t ndims) {
  auto* t = tb(h);
  size_t n = 1;
  for (size_t i = 0; i < ndims; ++i) n *= dims[i];
  if (n != t->len)
    panic("reshape element count mismatch: input has %zu elements, target would have %zu",
          t->len, n);
  if (ndims > (size_t)kMaxRank) panic("reshape rank %zu exceeds %d", ndims, kMaxRank);
  const bool keep_tail = t->ndim >= 2 && ndims >= 2 && dims[ndims - 1] == t->shape[t->ndim - 1] &&
                         dims[ndims - 2] == t->shape[t->ndim - 2];
  if (t->lazy) {   // same element order: a deferred result of the new shape
    int64_t out = make_lazy(dims, (int)ndims, t->lazy->src, t->lazy->scale, t->lazy->addend, t->lazy->colscale);
    tb(out)->causal_zero = t->causal_zero && keep_tail;
    return out;
  }
  if (t->view) {   // a strided view: a view again where the memory allows, else copied once
    View v;
    if (t->len && reshape_view(t->shape, t->ndim, *t->view, dims, ndims, &v)) return make_view(h, dims, (int)ndims, v);
    materialize(h);
  }
  t->st->aliases++;
  int64_t out = make_handle(t->dtype, dims, (int)ndims, t->st, t->len);
  tb(out)->causal_zero = t->causal_zero && keep_tail;
  return out;
}

// metal.rs:1601-1612 fills the [T,T] additive mask on the host (0 on and
// below the diagonal, -1e9 above); the same values are written by a kernel
// here, so the mask costs no host work or synchronisation (and can be
// captured in a graph).
__global__ void k_causal_mask(float* d, size_t T) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < T * T) d[i] = (i % T) > (i / T) ? -1e9f : 0.0f;
}

int64_t tensor_causal_mask(int64_t tsz) {
  size_t T = (size_t)tsz;
  size_t shape[2] = {T, T};
  int64_t h = alloc(MALUS_F32, shape, 2);
  if (T) {
    k_causal_mask<<<(unsigned)((T * T + 255) / 256), 256, 0, stream()>>>(fptr(h), T);
    count_launch();
    after_launch("k_causal_mask");
  }
  tb(h)->causal_mask = true;
  return h;
}

}  // extern "C"

// -------------------------------------------------------------------- RNG
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC'11), keyed by a per-call counter, followed by the
// Box-Muller transform in double precision — the generator of
// metal.rs:1692-1737 so that seeded weights are reproducible bit for bit.
namespace {
thread_local uint64_t t_rng_counter = 0;

struct Philox {
  static constexpr uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
  static constexpr uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
  static void run(uint32_t c[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
      uint64_t p0 = (uint64_t)c[0] * kMul0;
      uint64_t p1 = (uint64_t)c[2] * kMul1;
      uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
      uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
      uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
      c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
      k0 += kWeyl0;
      k1 += kWeyl1;
    }
  }
};

void randn_fill(float* out, size_t n, uint64_t call_idx) {
  uint32_t k0 = (uint32_t)call_idx, k1 = (uint32_t)(call_idx >> 32);
  size_t pairs = (n + 1) / 2;
  auto work = [&](size_t lo, size_t hi) {
    for (size_t k = lo; k < hi; ++k) {
      uint32_t c[4] = {(uint32_t)k, (uint32_t)((uint64_t)k >> 32), 0u, 0u};
      Philox::run(c, k0, k1);
      double u1 = ((double)c[0] + 0.5) / 4294967296.0;
      double u2 = ((double)c[1] + 0.5) / 4294967296.0;
      double mag = std::sqrt(-2.0 * std::log(u1));
      double ang = 2.0 * M_PI * u2;
      out[2 * k] = (float)(mag * std::cos(ang));
      if (2 * k + 1 < n) out[2 * k + 1] = (float)(mag * std::sin(ang));
    }
  };
  unsigned nt = pairs > (1u << 20) ? std::min(16u, std::max(1u, std::thread::hardware_concurrency())) : 1;
  if (nt <= 1) { work(0, pairs); return; }
  std::vector<std::thread> th;
  size_t chunk = (pairs + nt - 1) / nt;
  for (unsigned i = 0; i < nt; ++i) {
    size_t lo = i * chunk, hi = std::min(pairs, lo + chunk);
    if (lo < hi) th.emplace_back(work, lo, hi);
  }
  for (auto& t : th) t.join();
}
}  // namespace

extern "C" {

int64_t tensor_randn(const size_t* shape, size_t ndims) {
  size_t n = 1;
  for (size_t i = 0; i < ndims; ++i) n *= shape[i];
  uint64_t call_idx = t_rng_counter++;
  std::vector<float> d(std::max<size_t>(n, 1));
  randn_fill(d.data(), n, call_idx);
  int64_t h = tensor_alloc_gpu(MALUS_F32, shape, ndims, d.data());
  gpu_barrier();
  return h;
}

float malus_rand_uniform(void) {
  uint64_t call_idx = t_rng_counter++;
  uint32_t c[4] = {0, 0, 0, 0};
  Philox::run(c, (uint32_t)call_idx, (uint32_t)(call_idx >> 32));
  return (float)((double)c[0] / 4294967296.0);
}

int64_t malus_rand_int(int64_t n) {
  uint64_t call_idx = t_rng_counter++;
  uint32_t c[4] = {1, 0, 0, 0};
  Philox::run(c, (uint32_t)call_idx, (uint32_t)(call_idx >> 32));
  return (int64_t)((uint64_t)c[0] % (uint64_t)n);
}

void malus_rng_reset(uint64_t counter) { t_rng_counter = counter; }

void malus_philox4x32_10(uint32_t ctr[4], const uint32_t key[2]) { Philox::run(ctr, key[0], key[1]); }

// ------------------------------------------------------ host i32 buffers
// buffer.rs:11-50: a host Vec<i32>; freeze copies it into an i32 tensor.
struct HostBuf { std::vector<int32_t> v; };

int64_t malus_buffer_i32(int64_t len) {
  auto* b = new HostBuf();
  b->v.assign((size_t)len, 0);
  return reinterpret_cast<int64_t>(b);
}
int64_t malus_buffer_get_i32(int64_t buf, int64_t idx) {
  auto* b = reinterpret_cast<HostBuf*>(buf);
  if (idx < 0 || (size_t)idx >= b->v.size()) panic("buffer index %lld out of range", (long long)idx);
  return b->v[(size_t)idx];
}
void malus_buffer_set_i32(int64_t buf, int64_t idx, int64_t val) {
  auto* b = reinterpret_cast<HostBuf*>(buf);
  if (idx < 0 || (size_t)idx >= b->v.size()) panic("buffer index %lld out of range", (long long)idx);
  b->v[(size_t)idx] = (int32_t)val;
}
void malus_buffer_free(int64_t buf) { delete reinterpret_cast<HostBuf*>(buf); }
int64_t malus_buffer_freeze_i32(int64_t buf) {
  auto* b = reinterpret_cast<HostBuf*>(buf);
  size_t shape[1] = {b->v.size()};
  int64_t h = tensor_alloc_gpu(MALUS_I32, shape, 1, reinterpret_cast<const float*>(b->v.data()));
  return h;
}

// ------------------------------------------------------------ strings
// strio.rs: boxed host byte strings (not on the training hot path).
struct StrBox { std::string s; };
int64_t malus_str_box(const uint8_t* bytes, size_t len) {
  auto* s = new StrBox();
  s->s.assign(reinterpret_cast<const char*>(bytes), len);
  return reinterpret_cast<int64_t>(s);
}
int64_t malus_read_file(int64_t path_box) {
  auto* p = reinterpret_cast<StrBox*>(path_box);
  FILE* f = fopen(p->s.c_str(), "rb");
  if (!f) panic("read_file: cannot open '%s'", p->s.c_str());
  auto* s = new StrBox();
  char buf[65536];
  size_t r;
  while ((r = fread(buf, 1, sizeof buf, f)) > 0) s->s.append(buf, r);
  fclose(f);
  return reinterpret_cast<int64_t>(s);
}
int64_t malus_str_len(int64_t s) { return (int64_t)reinterpret_cast<StrBox*>(s)->s.size(); }
int64_t malus_str_char_at(int64_t s, int64_t i) {
  auto* b = reinterpret_cast<StrBox*>(s);
  if (i < 0 || (size_t)i >= b->s.size()) panic("str_char_at index %lld out of range", (long long)i);
  return (int64_t)(uint8_t)b->s[(size_t)i];
}
int64_t malus_str_from_char(int64_t c) {
  auto* s = new StrBox();
  s->s.assign(1, (char)c);
  return reinterpret_cast<int64_t>(s);
}

// -------------------------------------------------------- counters etc.
static int64_t g_cpu_compute = 0;   // lib.rs:1-21: this runtime never computes on the CPU
int64_t malus_cpu_compute_count(void) { return g_cpu_compute; }
void malus_cpu_compute_reset(void) { g_cpu_compute = 0; }

static float g_gradcheck_max = 0.0f;
void malus_record_diff(float v) {
  float a = std::fabs(v);
  if (a > g_gradcheck_max || std::isnan(a)) g_gradcheck_max = a;
}
float malus_gradcheck_max_diff(void) { return g_gradcheck_max; }
void malus_gradcheck_reset(void) { g_gradcheck_max = 0.0f; }

void malus_rc_counts(int64_t* r, int64_t* rel, int64_t* a) {
  if (r) *r = g_retains.load();
  if (rel) *rel = g_releases.load();
  if (a) *a = g_allocs.load();
}
void malus_rc_reset(void) { g_retains = 0; g_releases = 0; g_allocs = 0; }

void malus_pool_stats(int64_t* hits, int64_t* misses, int64_t* pooled, int64_t* peak) {
  std::lock_guard<std::mutex> lk(g_pool.mu);
  if (hits) *hits = g_pool.hits;
  if (misses) *misses = g_pool.misses;
  if (pooled) *pooled = g_pool.pooled;
  if (peak) *peak = g_pool.peak;
}
void malus_pool_reset(void) {
  ensure_init();
  std::lock_guard<std::mutex> lk(g_pool.mu);
  trim_pool_locked();
  g_pool.hits = g_pool.misses = 0;
  g_pool.peak = g_pool.live;
}
void malus_set_mem_budget(int64_t bytes) {
  std::lock_guard<std::mutex> lk(g_pool.mu);
  g_pool.budget = bytes < 0 ? -1 : bytes;
}

void* malus_tensor_data(int64_t h) {
  auto* t = tb(h);
  t->causal_zero = t->causal_mask = false;   // the caller may write through the pointer
  return vptr(h);
}
int32_t malus_tensor_dtype(int64_t h) { return tb(h)->dtype; }
void malus_tensor_read(int64_t h, void* dst, size_t bytes) {
  auto* t = tb(h);
  size_t have = t->len * dtype_size(t->dtype);
  if (bytes > have) panic("tensor_read of %zu bytes from a %zu-byte tensor", bytes, have);
  if (bytes) MALUS_CUDA(cudaMemcpyAsync(dst, vptr(h), bytes, cudaMemcpyDeviceToHost, stream()));
  gpu_barrier();
}
void malus_tensor_write(int64_t h, const void* src, size_t bytes) {
  auto* t = tb(h);
  size_t have = t->len * dtype_size(t->dtype);
  if (bytes > have) panic("tensor_write of %zu bytes into a %zu-byte tensor", bytes, have);
  plane_cache_clear();   // the data changes in place
  t->causal_zero = t->causal_mask = false;
  if (bytes) MALUS_CUDA(cudaMemcpyAsync(vptr(h), src, bytes, cudaMemcpyHostToDevice, stream()));
  gpu_barrier();
}
int64_t malus_tensor_wrap(int32_t dtype, void* dev_ptr, const size_t* shape, size_t ndims) {
  auto* st = new Storage();
  st->ptr = dev_ptr;
  st->bytes = 0;
  st->aliases = 1;
  st->owned = false;
  st->id = g_storage_ids.fetch_add(1, std::memory_order_relaxed);
  size_t n = 1;
  for (size_t i = 0; i < ndims; ++i) n *= shape[i];
  return make_handle(dtype, shape, (int)ndims, st, n);
}
void malus_set_device(int32_t dev) {
  if (g_ctx.init) {
    if (dev != g_ctx.device) panic("malus_set_device(%d) after the runtime bound device %d", dev, g_ctx.device);
    return;
  }
  char buf[16];
  snprintf(buf, sizeof buf, "%d", dev);
  setenv("MALUS_DEVICE", buf, 1);
  ensure_init();
}
int64_t malus_launch_count(void) { return g_launches.load(); }
void malus_launch_count_reset(void) { g_launches = 0; }
void* malus_stream(void) { return (void*)stream(); }

int32_t malus_device_error(void) {
  int32_t v = 0;
  MALUS_CUDA(cudaMemcpyAsync(&v, device_error_word(), 4, cudaMemcpyDeviceToHost, stream()));
  gpu_barrier();
  if (v) MALUS_CUDA(cudaMemsetAsync(device_error_word(), 0, 4, stream()));
  return v;
}

// ------------------------------------------------------------ graph capture
// Capture a sequence of runtime calls on the runtime stream into a CUDA graph
// and replay it (the caller side of the boundary: one training step becomes one
// launch).  Replays run on the same buffers as the capture, so a replayed
// step must update its state in place (malus_adamw_multi, malus_tensor_write
// of the next inputs) and its inputs must stay alive while the graph exists;
// host reads are not allowed inside the capture.  Run the sequence once
// before capturing it so that grow-on-demand workspaces are sized.
namespace {
std::unordered_map<int64_t, GraphRec*> g_graphs;
int64_t g_graph_next = 1;
}  // namespace

int32_t malus_graph_begin(void) {
  ensure_init();
  plane_cache_clear();
  {
    std::lock_guard<std::mutex> lk(g_pool.mu);
    if (g_cap.active) panic("malus_graph_begin: a capture is already open");
    g_cap.active = true;
    g_cap.launches_at_begin = g_launches.load();
  }
  MALUS_CUDA(cudaStreamBeginCapture(stream(), cudaStreamCaptureModeRelaxed));
  return 0;
}

int64_t malus_graph_end(void) {
  plane_cache_clear();
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(stream(), &graph);
  auto* rec = new GraphRec();
  {
    std::lock_guard<std::mutex> lk(g_pool.mu);
    if (!g_cap.active) panic("malus_graph_end without malus_graph_begin");
    rec->launches = g_launches.load() - g_cap.launches_at_begin;
    std::unordered_set<void*> freed;
    for (auto& kv : g_cap.free_lists)
      for (void* p : kv.second) {
        rec->held.emplace_back(p, kv.first);
        freed.insert(p);
      }
    for (auto& pb : g_cap.touched) {
      if (!freed.count(pb.first)) {      // still live in a tensor: pinned until destroy
        g_pinned[pb.first] = rec;
        rec->pinned.push_back(pb.first);
      }
    }
    g_cap = CaptureSession();
  }
  if (e != cudaSuccess || graph == nullptr)
    panic("graph capture failed: %s (an operation in the captured sequence cannot be captured)",
          cudaGetErrorString(e));
  MALUS_CUDA(cudaGraphInstantiate(&rec->exec, graph, 0));
  MALUS_CUDA(cudaGraphDestroy(graph));
  count_launch(-(int)rec->launches);   // captured, not launched: counted at each replay
  const int64_t id = g_graph_next++;
  g_graphs[id] = rec;
  return id;
}

int32_t malus_graph_replay(int64_t id) {
  auto it = g_graphs.find(id);
  if (it == g_graphs.end()) return -1;
  plane_cache_clear();   // the replay rewrites tensors in place
  MALUS_CUDA(cudaGraphLaunch(it->second->exec, stream()));
  count_launch((int)it->second->launches);
  return 0;
}

int32_t malus_graph_destroy(int64_t id) {
  auto it = g_graphs.find(id);
  if (it == g_graphs.end()) return -1;
  GraphRec* rec = it->second;
  g_graphs.erase(it);
  MALUS_CUDA(cudaStreamSynchronize(stream()));   // replays in flight still use the buffers
  MALUS_CUDA(cudaGraphExecDestroy(rec->exec));
  std::vector<std::pair<void*, size_t>> back;
  {
    std::lock_guard<std::mutex> lk(g_pool.mu);
    for (void* p : rec->pinned) {
      auto pin = g_pinned.find(p);
      if (pin != g_pinned.end() && pin->second == rec) g_pinned.erase(pin);
    }
    back.swap(rec->held);
  }
  for (auto& pb : back) {   // the pool takes back what the graph held
    std::lock_guard<std::mutex> lk(g_pool.mu);
    g_pool.free_lists[pb.second].push_back(pb.first);
    g_pool.pooled += (int64_t)pb.second;
  }
  delete rec;
  return 0;
}

// ------------------------------------------------------------- bench timer
// bench.rs:12-70: dormant unless enabled; a step is timed on the host clock
// from bench_step_begin to bench_step_end, whose wait for the GPU (gpu_barrier)
// lies inside the timed region; an end without a begin records nothing; the
// report is the median of the steps after the first 3 (warm-up); reset
// disables the timer and forgets the steps.
static bool g_bench_on = false;
static bool g_bench_started = false;
static std::chrono::steady_clock::time_point g_bench_t0;
static std::vector<double> g_bench_ms;
void bench_enable(void) { g_bench_on = true; }
void bench_step_begin(void) {
  if (!g_bench_on) return;
  g_bench_t0 = std::chrono::steady_clock::now();
  g_bench_started = true;
}
void bench_step_end(void) {
  if (!g_bench_on) return;
  gpu_barrier();
  if (!g_bench_started) return;
  g_bench_started = false;
  g_bench_ms.push_back(
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - g_bench_t0).count());
}
static std::vector<double> bench_warm_sorted() {
  const size_t warm = 3;
  if (g_bench_ms.size() <= warm) return {};
  std::vector<double> v(g_bench_ms.begin() + warm, g_bench_ms.end());
  std::sort(v.begin(), v.end());
  return v;
}
double bench_report(int64_t* n_steps) {
  std::vector<double> v = bench_warm_sorted();
  if (n_steps) *n_steps = (int64_t)v.size();
  if (v.empty()) return -1.0;
  size_t n = v.size();
  return n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}
void bench_report_range(double* min_ms, double* max_ms) {
  std::vector<double> v = bench_warm_sorted();
  if (min_ms) *min_ms = v.empty() ? -1.0 : v.front();
  if (max_ms) *max_ms = v.empty() ? -1.0 : v.back();
}
void bench_reset(void) {
  g_bench_on = false;
  g_bench_started = false;
  g_bench_ms.clear();
}

}  // extern "C"

// ------------------------------------------------------ live kernel timing
// Optional per-kernel-class timing for the bench's roofline figure: when
// enabled, launches of a class are bracketed by CUDA events on the runtime
// stream; the report sums the event durations and the algorithmic work the
// launcher declared.  Classes: 0 = tcgen05 GEMM, 1 = split of GEMM operands,
// 2 = SIMT GEMM, 3 = data-parallel all-reduce (on the collective stream;
// bytes = payload), 4 = the main stream's wait for the all-reduces at the
// join (the communication the backward pass does not hide).
namespace malus {
namespace {
struct ProfRec { cudaEvent_t a, b; int cls; double flops, bytes; const char* name; };
bool g_prof_on = false;
std::vector<ProfRec> g_prof;
std::vector<cudaEvent_t> g_ev_free;
cudaEvent_t ev_get() {
  if (!g_ev_free.empty()) { cudaEvent_t e = g_ev_free.back(); g_ev_free.pop_back(); return e; }
  cudaEvent_t e;
  MALUS_CUDA(cudaEventCreate(&e));
  return e;
}
}  // namespace
bool prof_on() { return g_prof_on; }
int prof_begin_on(int cls, double flops, double bytes, cudaStream_t s) {
  if (!g_prof_on) return -1;
  ProfRec r{ev_get(), ev_get(), cls, flops, bytes, nullptr};
  MALUS_CUDA(cudaEventRecord(r.a, s));
  g_prof.push_back(r);
  return (int)g_prof.size() - 1;
}
void prof_end_on(int id, cudaStream_t s) {
  if (id < 0) return;
  MALUS_CUDA(cudaEventRecord(g_prof[id].b, s));
}
int prof_begin(int cls, double flops, double bytes) { return prof_begin_on(cls, flops, bytes, stream()); }
int prof_begin_named(const char* name, double bytes) {
  const int id = prof_begin_on(5, 0.0, bytes, stream());
  if (id >= 0) g_prof[(size_t)id].name = name;
  return id;
}
void prof_end(int id) { prof_end_on(id, stream()); }
}  // namespace malus

extern "C" {
void malus_prof_enable(int32_t on) {
  using namespace malus;
  gpu_barrier();
  for (auto& r : g_prof) { g_ev_free.push_back(r.a); g_ev_free.push_back(r.b); }
  g_prof.clear();
  g_prof_on = on != 0;
}
// Per kernel label of class 5 (non-GEMM kernels of the compiled step, each with
// its algorithmic bytes): one line "label<TAB>launches<TAB>ms<TAB>bytes" per
// label, in first-launch order, written into buf (NUL-terminated, truncated
// at cap); returns the length the whole text needs.
int32_t malus_prof_kernels(char* buf, int32_t cap) {
  using namespace malus;
  gpu_barrier();
  std::vector<std::string> order;
  std::unordered_map<std::string, std::tuple<int64_t, double, double>> agg;
  for (auto& r : g_prof) {
    if (r.cls != 5 || !r.name) continue;
    float x = 0;
    MALUS_CUDA(cudaEventElapsedTime(&x, r.a, r.b));
    auto it = agg.find(r.name);
    if (it == agg.end()) {
      order.push_back(r.name);
      it = agg.emplace(r.name, std::make_tuple((int64_t)0, 0.0, 0.0)).first;
    }
    std::get<0>(it->second) += 1;
    std::get<1>(it->second) += x;
    std::get<2>(it->second) += r.bytes;
  }
  std::string text;
  char line[256];
  for (auto& n : order) {
    auto& a = agg[n];
    snprintf(line, sizeof line, "%s\t%lld\t%.6f\t%.0f\n", n.c_str(), (long long)std::get<0>(a), std::get<1>(a),
             std::get<2>(a));
    text += line;
  }
  if (buf && cap > 0) {
    const size_t k = std::min(text.size(), (size_t)cap - 1);
    memcpy(buf, text.data(), k);
    buf[k] = 0;
  }
  return (int32_t)text.size();
}

// Sum over recorded launches of class `cls`: count, total ms, flops, bytes.
void malus_prof_report(int32_t cls, int64_t* count, double* ms, double* flops, double* bytes) {
  using namespace malus;
  gpu_barrier();
  int64_t n = 0;
  double t = 0, f = 0, b = 0;
  for (auto& r : g_prof) {
    if (r.cls != cls) continue;
    float x = 0;
    MALUS_CUDA(cudaEventElapsedTime(&x, r.a, r.b));
    ++n; t += x; f += r.flops; b += r.bytes;
  }
  if (count) *count = n;
  if (ms) *ms = t;
  if (flops) *flops = f;
  if (bytes) *bytes = b;
}
}  // extern "C"
