// Internal definitions shared by the runtime's translation units.
//
// A tensor handle is a pointer to TensorBuffer (the handle layout of the
// reference is opaque too: crates/malus-runtime/src/metal.rs:280-296).  Data
// always lives in HBM, row-major and contiguous; reshape aliases share one
// Storage (metal.rs:1388-1403).  All device work is ordered on one CUDA
// stream, which is what makes the pool's immediate reuse of a freed buffer
// safe: a later kernel on the same stream cannot start before the kernels
// that last touched the buffer.
#pragma once
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <initializer_list>
#include <vector>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/malus_runtime.h"

namespace malus {

[[noreturn]] void panic(const char* fmt, ...);

#define MALUS_CUDA(call)                                                      \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess)                                                    \
      ::malus::panic("CUDA error %s at %s:%d: %s", cudaGetErrorName(e_),      \
                     __FILE__, __LINE__, cudaGetErrorString(e_));             \
  } while (0)

constexpr int kMaxRank = 8;

struct Storage {
  void* ptr;
  size_t bytes;      // allocated (pool bucket) size
  int aliases;       // number of TensorBuffers sharing this storage
  bool owned;        // false for malus_tensor_wrap'd memory
  uint64_t id;       // unique per storage for the process (never reused)
};

// One logical dimension of a strided view: index i lies at element offset
// (i / div) * hi + (i % div) * lo from the storage base (div == 0: i * lo).
// Two radices let a reshape merge two dimensions that are not adjacent in
// memory (the attention head fold [B, T, H, hs] -> [B*H, T, hs] after a permute).
struct ViewDim {
  int64_t div = 0, hi = 0, lo = 0;
  __host__ __device__ int64_t at(int64_t i) const { return div ? (i / div) * hi + (i % div) * lo : i * lo; }
};
struct View { ViewDim d[kMaxRank]; };

// A deferred elementwise result: value = src * scale[0] (+ addend, broadcast
// over src's leading dims: its shape is src's trailing dims), or src * colscale
// (a vector along the last dim), with the roundings of the eager multiply and
// add.  A multiply by a one-element tensor makes the first kind (the attention
// score scaling, and its VJP), an add of such a product and a tensor of its
// trailing shape extends it (the causal mask); a multiply by a vector of the
// last dim's length makes the second (the layernorm gain, and its VJP).  The
// softmax, the layernorm VJP and the GEMM operand split read them fused; any
// raw access materialises them.  They hold references to their operands and
// no storage.
struct Lazy { int64_t src, scale, addend, colscale; };

// A tensor is either contiguous row-major over its storage (view == nullptr)
// or a strided view of a storage shared with the tensor it was made from
// (permute, and reshapes of such views).  Raw pointers (fptr / vptr) always
// see contiguous row-major data: they materialise a view first.
struct TensorBuffer {
  Storage* st;
  int32_t dtype;
  int32_t ndim;
  size_t len;
  size_t shape[kMaxRank];
  std::atomic<int64_t> rc;
  View* view = nullptr;
  Lazy* lazy = nullptr;    // st == nullptr while set
  // Facts about the values the runtime knows from how it made them:
  //  causal_mask: the [T, T] additive mask of tensor_causal_mask (0 on and below
  //    the diagonal, -1e9 above);
  //  causal_zero: every [T, T] slice of the last two dims is exactly 0 above
  //    the diagonal (a softmax over scores plus that mask, and its VJP).
  // Both are dropped by writes the runtime cannot see into (host writes, raw
  // pointers handed out).
  bool causal_mask = false;
  bool causal_zero = false;
  // made by tensor_matmul: an activation of such a product (the MLP's GELU)
  // is read by the next GEMM, so its kernel writes the tf32 planes too
  bool gemm_out = false;
};

inline TensorBuffer* tb(int64_t h) {
  if (h == 0) panic("null tensor handle");
  return reinterpret_cast<TensorBuffer*>(h);
}
// A view or a deferred result becomes a contiguous tensor with storage of its own.
void materialize(int64_t h);
inline float* fptr(int64_t h) {
  auto* t = tb(h);
  if (t->view || t->lazy) materialize(h);
  return static_cast<float*>(t->st->ptr);
}
inline void* vptr(int64_t h) {
  auto* t = tb(h);
  if (t->view || t->lazy) materialize(h);
  return t->st->ptr;
}
// A deferred src * scale (+ addend), or src * colscale, of the given shape
// (src's element count); retains the operands.
int64_t make_lazy(const size_t* shape, int ndim, int64_t src, int64_t scale, int64_t addend,
                  int64_t colscale = 0);
// A new handle for the same values (same storage, view or deferred result).
int64_t alias_of(int64_t h);
// The view of tensor h's dims (row-major strides when it is contiguous).
View view_of(int64_t h);
// h's data read as the shape `dims` (same element count) through one view of
// its storage, when its memory allows that (false: it does not).
bool view_as(int64_t h, const size_t* dims, size_t nd, View* out);
// A new handle over h's storage with the given shape and view (no copy).
int64_t make_view(int64_t h, const size_t* shape, int ndim, const View& v);
size_t dtype_size(int32_t dtype);

// ---- runtime core (runtime.cu) ----
cudaStream_t stream();
int64_t alloc(int32_t dtype, const size_t* shape, int ndim);       // uninitialised
int64_t alloc_like(int64_t h);                                     // same shape, f32
int64_t alloc_f32(std::initializer_list<size_t> shape);
void* scratch_alloc(size_t bytes);                                 // pooled raw device memory
void scratch_free(void* p);
void count_launch(int n = 1);
void after_launch(const char* what);
bool sync_dispatch();
int32_t* device_error_word();
bool prof_on();
int prof_begin(int cls, double flops, double bytes);
void prof_end(int id);
int prof_begin_on(int cls, double flops, double bytes, cudaStream_t s);   // on another stream
int prof_begin_named(const char* name, double bytes);   // class 5: a labelled kernel (static label)
void prof_end_on(int id, cudaStream_t s);

// Shape helpers
struct Shape {
  int ndim = 0;
  size_t d[kMaxRank] = {0};
  size_t numel() const { size_t n = 1; for (int i = 0; i < ndim; ++i) n *= d[i]; return n; }
};
inline Shape shape_of(int64_t h) {
  Shape s; auto* t = tb(h); s.ndim = t->ndim;
  for (int i = 0; i < t->ndim; ++i) s.d[i] = t->shape[i];
  return s;
}
inline int64_t alloc_shape(const Shape& s, int32_t dtype = MALUS_F32) {
  return alloc(dtype, s.d, s.ndim);
}
bool same_shape(int64_t a, int64_t b);
int normalize_axis(int64_t axis, int ndim);
// outer / axis / inner decomposition (softmax.ml:1-7 convention)
void split_axis(const Shape& s, int axis, size_t* outer, size_t* axis_sz, size_t* inner);

// ---- launch geometry ----
constexpr int kNumSMs = 148;
inline unsigned grid_for(size_t work_items, int threads, int max_blocks_per_sm = 8) {
  size_t b = (work_items + threads - 1) / threads;
  size_t cap = (size_t)kNumSMs * max_blocks_per_sm;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

// ---- elementwise (elementwise.cu) ----
enum BinOp : int { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3 };
int64_t binary_broadcast(int op, int64_t a, int64_t b);          // NumPy broadcast result
void binary_same(int op, const float* a, const float* b, float* out, size_t n);
enum ScalarOp : int { kSAdd, kSSub, kSRSub, kSMul, kSDiv, kSRDiv, kSFill };
void scalar_op_dev(int op, const float* a, const float* s_dev, float* out, size_t n);
void scalar_op_imm(int op, const float* a, float s, float* out, size_t n);
enum UnaryOp : int { kRelu, kSigmoid, kTanh, kExp, kLog, kSqrt, kAbs, kGelu, kRsqrtEps, kNeg };
void unary_op(int op, const float* a, float* out, size_t n, float param = 0.f);
enum UnaryBwdOp : int { kSigmoidBwd, kReluBwd, kTanhBwd, kSqrtBwd, kAbsBwd, kGeluBwd, kEq };
void unary_bwd(int op, const float* x, const float* dout, float* out, size_t n);
void fill_from_dev_scalar(float* out, const float* s_dev, size_t n);
void expand_axis(const float* small, float* out, size_t outer, size_t axis_sz, size_t inner);
// the XOR user kernel `sigmoid_backward` (examples/xor.ml:1-2)
void sigmoid_backward_user(const float* g, const float* s, float* out, size_t n);

// ---- reductions (reduce.cu) ----
enum RedOp : int { kRSum = 0, kRMean = 1, kRMax = 2, kRVar = 3 };
void reduce_axis(int op, const float* x, float* out, size_t outer, size_t axis_sz, size_t inner);
// Sum over the axis of x[i] * x2[i] (each product rounded to f32), with the
// same partition and order as reduce_axis(kRSum) of the materialised product,
// so the result is bit-identical to it; inner > 1 (column sums) only.
void reduce_axis_sum_product(const float* x, const float* x2, float* out, size_t outer, size_t axis_sz,
                             size_t inner);

// ---- row kernels (rows.cu) ----
// x (optionally): each element times scale[0], plus addend[(row % add_rows) * axis + i]
// (same roundings as the eager multiply and add; rows along the last axis only).
// causal_T > 0: the addend is the causal mask of [causal_T, causal_T] scores
// (-1e9 above the diagonal), so in row r the elements past r % causal_T give
// exactly 0 and need not be read (the same bits as reading them, for scores
// below ~1e8 in magnitude).
// p_hi / p_lo: with causal_T, also the result's tf32 planes (row pitch
// axis_sz) up to each 128-row tile's diagonal block; only the row kernel
// (softmax_rows_path) writes them.
void softmax_fwd(const float* x, float* y, size_t outer, size_t axis_sz, size_t inner,
                 const float* scale = nullptr, const float* addend = nullptr, size_t add_rows = 1,
                 int causal_T = 0, float* p_hi = nullptr, float* p_lo = nullptr);
bool softmax_rows_path(const float* x, const float* y, const float* addend, size_t outer, size_t axis_sz,
                       size_t inner);
// GELU (g null) or its VJP (dout g) over n elements, also writing the result's
// tf32 planes hi / lo (n % 4 == 0, 16-byte-aligned arrays)
void gelu_planes(const float* x, const float* g, float* out, float* hi, float* lo, size_t n);
// causal_T > 0: s is zero past the diagonal of [causal_T, causal_T] blocks, so
// dx is zero there and those elements of s and dout are not read (the same
// values; a zero may differ in sign)
void softmax_bwd(const float* s, const float* dout, float* dx, size_t outer, size_t axis_sz,
                 size_t inner, int causal_T = 0);
void layernorm_fwd(const float* x, float* y, float* var, size_t outer, size_t axis_sz,
                   size_t inner, float eps);
// dout_colscale (optional, last axis only): dout is read as dout[i] * dout_colscale[i % axis]
void layernorm_bwd(const float* y, const float* var, const float* dout, float* dx, size_t outer,
                   size_t axis_sz, size_t inner, float eps, const float* dout_colscale = nullptr);
// probs [N,V] written; loss[0] = mean nll
void xent_fwd(const float* logits, const void* targets, int tgt_dtype, float* probs, float* loss,
              size_t n, size_t v);
void xent_bwd(const float* probs, const void* targets, int tgt_dtype, const float* dout_dev,
              float* dx, size_t n, size_t v);
// the same with a host scale in place of dout[0] / n
void xent_bwd_scaled(const float* probs, const void* targets, int tgt_dtype, float scale, float* dx,
                     size_t n, size_t v);
void xent_nll_gather(const float* probs, const void* targets, int tgt_dtype, float* out, size_t n,
                     size_t v);
void embedding_fwd(const float* w, const void* idx, int idx_dtype, float* out, size_t n,
                   size_t vocab, size_t dim);
void embedding_bwd(const float* dout, const void* idx, int idx_dtype, float* dw, size_t n,
                   size_t vocab, size_t dim);
void permute_nd(const float* x, float* out, const Shape& in_shape, const int* perm);
size_t embedding_bwd_ws_bytes(size_t n, size_t vocab);
// err: device word set to 4 when an id lies outside [0, vocab) (nullptr: a
// word in the workspace, cleared per call and never read)
int embedding_bwd_ws(const float* dout, const void* idx, int idx_dtype, float* dw, size_t n,
                     size_t vocab, size_t dim, void* workspace, cudaStream_t st, int32_t* err);

// ---- GEMM (gemm.cu) ----
// C[b] (MxN) = alpha * op(A[b]) * op(B[b]) + beta * C[b], f32 semantics via
// 3xTF32 on tcgen05 (large shapes) or exact-f32 SIMT (small shapes).
// Each operand is the stored matrix as the call sees it, a [nz][rows][cols]
// stack read through a strided view of a tensor's storage (element (z, r, c)
// at base + z.at(z) + r.at(r) + c.at(c)); nz is 1 (shared by every batch
// entry) or the batch.  A is MxK: a_trans = false -> stored {rows M, cols K};
// true -> stored {rows K, cols M} (A^T).  B is KxN: b_trans = false -> stored
// {rows K, cols N}; true -> {rows N, cols K}.  scale_dev (optional): the
// values are those of the view times *scale_dev (one f32 multiply).
// key: the storage's id for the operand-plane cache (0: not cached).
struct GemmOperand {
  const float* base = nullptr;
  int64_t nz = 1, rows = 0, cols = 0;
  ViewDim z, r, c;
  const float* scale_dev = nullptr;
  const float* colscale_dev = nullptr;   // optional: column c (of cols) times colscale_dev[c]
  uint64_t key = 0;
};
// A contiguous row-major stack: nz slices of rows x cols, row pitch ld, slice stride sstride.
GemmOperand plain_operand(const float* p, int64_t nz, int64_t rows, int64_t cols, int64_t ld,
                          int64_t sstride);
struct GemmArgs {
  int M, N, K, batch;
  GemmOperand A; bool a_trans;
  GemmOperand B; bool b_trans;
  float* C; int64_t ldc; int64_t strideC;
  float alpha = 1.f, beta = 0.f;
  // A[m][k] is exactly 0 for k > m (kCausalALower) or k < m (kCausalAUpper):
  // the GEMM clips its K ranges there (the skipped products are exact zeros)
  int a_zero = 0;
};
// Operand planes split from tensors during a step are kept per storage and
// view and reused by later GEMMs that read the same data (a weight in the
// forward and in both backward products, an activation saved for backward).
// The cache is dropped whenever tensor data may change in place (step
// boundaries: tape_zero_grad, the end of backward; AdamW; host writes;
// user-kernel dispatch; graph capture and replay) and entry by entry when a
// storage is freed.  MALUS_PLANE_CACHE=0 disables it.
void plane_cache_clear();
void plane_cache_drop(uint64_t storage_id);
// Planes for an operand that the kernel producing it writes as it stores the
// f32 values (hi = tf32_rn(x), lo = tf32_rn(x - hi), the split's own
// expressions): registers a cache entry for `o` (a plain row-major stack, no
// deferred scale) and returns its memory (hi, then lo after nz*rows*cols
// floats, row pitch = cols), or null when the cache is off, the layout is not
// plain, or an entry exists.  causal_T > 0: only the part a causally clipped
// GEMM reads need be written, and only such GEMMs use the entry.
float* plane_cache_prime(const GemmOperand& o, int64_t causal_T);
// x rounded to tf32 (round to nearest, ties away from zero), as the operand
// split does for the hi plane
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
void gemm(const GemmArgs& g);

// Low-level tcgen05 GEMM on pre-split tf32 planes (hi/lo), for callers that
// produce their operands already split.  Each operand is a stack of nz
// row-major slices (rows x cols, row pitch in floats, slice stride zstride);
// a K-major operand is stored {rows = M or N, cols = K}, an MN-major one
// {rows = K, cols = M or N}.  zmode selects what the third TMA coordinate
// follows: nothing, the problem batch index, k / seg (K segments spread over
// slices) or mn / seg (M or N segments spread over slices).
enum TcZMode : int { kZNone = 0, kZBatch = 1, kZKSeg = 2, kZMNSeg = 3 };
struct TcOperand {
  const float* hi;
  const float* lo;
  int64_t rows, cols, pitch;
  int nz;
  int64_t zstride;
  bool mn_major;
  int zmode;
  int seg;
};
// out offset = Z(z) + R(m) + Cc(n); each term maps an index i through two
// optional divisions: q1 = i / d1, r1 = i % d1 (d1 = 0: q1 = 0, r1 = i);
// q2 = r1 / d2, r2 = r1 % d2 (d2 = 0: q2 = 0, r2 = r1); term = q1*s1 + q2*s2 + r2*s3.
struct TcLayout { int64_t d1, s1, d2, s2, s3; };
enum TcEpi : int { kEpiStore = 0, kEpiResid = 1, kEpiGelu = 2, kEpiGeluBwd = 3, kEpiSoftmaxBwd = 4 };
struct TcProblem {
  int M, N, K, batch;
  TcOperand a, b;
  int epi;
  TcLayout oz, om, on;
  float* out;       // f32 output (Store/Resid: result; Gelu: pre-activation; GeluBwd: optional)
  float* out_hi;    // optional tf32 planes of the result (Gelu/GeluBwd: of the activation/derivative)
  float* out_lo;
  const float* aux; // Resid: residual input; GeluBwd: pre-activation
  float alpha = 1.f, beta = 0.f;
  int causal = 0;   // kCausal*: skip work on the zero side of an attention mask
  const float* aux_lo = nullptr;  // SoftmaxBwd: lo plane of P (aux = hi plane)
  const float* rowv = nullptr;    // SoftmaxBwd: D[z * M + m] = sum_j P dP of the row
};
enum { kCausalNone = 0, kCausalOut = 1, kCausalALower = 2, kCausalAUpper = 3 };
void gemm_tc_planes(const TcProblem& p);
// hi/lo planes of a stack of `batch` row-major slices (rows x cols, ld, sstride)
void tf32_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t batch,
                int64_t sstride, float* hi, float* lo, int64_t pitch);
void gemm_simt(const GemmArgs& g);        // contiguous (plain) operands only
int gemm_backend_for(const GemmArgs& g);   // 0 = SIMT, 1 = tcgen05
void gemm_force_backend(int b);            // -1 = auto (tests)

// ---- optimizer (adamw.cu) ----
struct AdamSeg { float* p; const float* g; float* m; float* v; int64_t n; };
void step_advance(int64_t* step_dev);
// data parallelism: per-leaf gradient readiness (dp.cu)
bool dp_leaves_registered();
bool dp_is_leaf(int64_t h);
int dp_leaf_ready(int64_t leaf, int64_t grad);
int dp_leaves_join();
std::vector<float> adam_bc_table(float b1, float b2, int64_t cap);
void adamw_flat(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
                float b2, float eps, float wd, float grad_scale, const float* bc_tab,
                const int64_t* step_dev, float* hi, float* lo);
void adamw_multi_tab(const AdamSeg* segs, int nseg, float lr, float b1, float b2, float eps,
                     float wd, float bc1, float bc2, float grad_scale, const float* bc_tab,
                     const int64_t* step_dev);
void adamw_multi(const AdamSeg* segs, int nseg, float lr, float b1, float b2, float eps, float wd,
                 float bc1, float bc2, float grad_scale);

// ---- tape (tape.cpp) ----
void tape_on_release(int64_t h);

// nanoGPT fused-buffer layout and its data-parallel all-reduce buckets (gpt.cu)
size_t gpt_layout(const malus_gpt_config& c, std::vector<std::vector<size_t>>& shapes,
                  std::vector<size_t>& offs, std::vector<size_t>& sizes);
std::vector<std::pair<size_t, size_t>> gpt_dp_buckets(int n_layer, const std::vector<size_t>& offs,
                                                      const std::vector<size_t>& sizes);

}  // namespace malus
