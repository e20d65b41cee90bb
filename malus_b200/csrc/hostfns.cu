// Native replacements for the stdlib host functions of
// crates/malus-stdlib/stdlib/*.ml (same names and signatures, so the BwdSlot
// table of crates/malus-codegen-cpu/src/lib.rs:189-220 can point at them), and
// the tensor ops of metal.rs (tensor_matmul, tensor_permute).  Each returns a
// new handle with refcount 1; inputs are borrowed.
//
// Shape semantics follow the host-side (CPU twin) evaluation of
// crates/malus-runtime/src/metal.rs where the GPU .ml path is ill-defined:
//  * broadcast binops compute a op b with the full NumPy result shape
//    (metal.rs:1024-1072); the .ml path instead keeps the higher-rank
//    operand's shape and swaps operands for sub/div when a.ndim < b.ndim
//    (broadcast_binop.ml:82-112) — both agree whenever that operand already
//    has the result shape, which is every call on the nanoGPT path;
//  * layernorm saves a per-group variance with keepdim at the axis
//    (metal.rs:1524-1530); the .ml kernel writes a full-size variance that
//    its VJP then indexes per element (layernorm.ml:40-58 with
//    reduce_bwd.ml:10-18), which mixes rows — the host twin is the oracle.
#include "common.cuh"

#include <vector>

using namespace malus;

namespace malus {
void binary_project_into_a(int op, int64_t ha, int64_t hb, float* out);
}

namespace {

int64_t tuple2(int64_t a, int64_t b) {
  // codegen-cpu lib.rs:58-86: 8-byte refcount header, fields at +8, +16.
  auto* box = static_cast<int64_t*>(calloc(1, 24));
  if (!box) panic("tuple allocation failed");
  box[0] = 1;
  box[1] = a;
  box[2] = b;
  return reinterpret_cast<int64_t>(box);
}

int64_t copy_of(int64_t h) {
  int64_t out = alloc_like(h);
  size_t n = tb(h)->len;
  if (n) MALUS_CUDA(cudaMemcpyAsync(fptr(out), fptr(h), n * 4, cudaMemcpyDeviceToDevice, stream()));
  return out;
}

int64_t reduce_impl(int op, int64_t x, int64_t axis, int64_t keepdim) {
  Shape s = shape_of(x);
  if (s.ndim == 0) panic("reduce on a rank-0 tensor");
  int ax = normalize_axis(axis, s.ndim);
  size_t outer, asz, inner;
  split_axis(s, ax, &outer, &asz, &inner);
  Shape o;
  if (s.ndim == 1) {
    o.ndim = 1;
    o.d[0] = 1;  // reduce_sum.ml:29-30: rank-1 input -> shape [1]
  } else if (keepdim) {
    o = s;
    o.d[ax] = 1;
  } else {
    for (int i = 0; i < s.ndim; ++i)
      if (i != ax) o.d[o.ndim++] = s.d[i];
  }
  int64_t out = alloc_shape(o);
  reduce_axis(op, fptr(x), fptr(out), outer, asz, inner);
  return out;
}

// Sum `g` down to the shape of `target` (the dual of broadcasting), the
// sequence of elementwise_bwd.ml:8-22: collapse extra leading dims, then
// reduce (keepdim) every axis where target has size 1 and g does not.
int64_t sum_to_shape(int64_t g, const Shape& target) {
  Shape s = shape_of(g);
  bool same = s.ndim == target.ndim;
  for (int i = 0; same && i < s.ndim; ++i) same = s.d[i] == target.d[i];
  if (same) return copy_of(g);
  if (s.ndim < target.ndim) panic("sum_to_shape: gradient rank %d below target rank %d", s.ndim, target.ndim);
  const float* src = fptr(g);
  int64_t cur = 0;  // owned intermediate (0 = still reading g)
  Shape cs = s;
  int extra = s.ndim - target.ndim;
  if (extra > 0) {
    size_t lead = 1, rest = 1;
    for (int i = 0; i < extra; ++i) lead *= s.d[i];
    for (int i = extra; i < s.ndim; ++i) rest *= s.d[i];
    Shape ns;
    ns.ndim = target.ndim;
    for (int i = 0; i < target.ndim; ++i) ns.d[i] = s.d[extra + i];
    if (ns.ndim == 0) { ns.ndim = 1; ns.d[0] = 1; }
    int64_t r = alloc_shape(ns);
    reduce_axis(kRSum, src, fptr(r), 1, lead, rest);
    cur = r;
    cs = ns;
    src = fptr(r);
  }
  for (int ax = 0; ax < target.ndim; ++ax) {
    if (target.d[ax] == 1 && cs.d[ax] > 1) {
      size_t outer, asz, inner;
      split_axis(cs, ax, &outer, &asz, &inner);
      Shape ns = cs;
      ns.d[ax] = 1;
      int64_t r = alloc_shape(ns);
      reduce_axis(kRSum, src, fptr(r), outer, asz, inner);
      if (cur) tensor_release(cur);
      cur = r;
      cs = ns;
      src = fptr(r);
    }
  }
  if (!cur) return copy_of(g);
  return cur;
}

// Deferred products are made only for large tensors (where the pass they
// save matters) whose consumers can read them fused.
constexpr size_t kLazyMin = (size_t)1 << 16;

bool one_element_f32(int64_t h) { return tb(h)->len == 1 && tb(h)->dtype == MALUS_F32; }

// a * b for a one-element b, deferred (the result has a's shape when b's rank
// does not exceed a's); 0 when not applicable.
int64_t lazy_scale(int64_t a, int64_t b) {
  auto *ta = tb(a), *tb_ = tb(b);
  if (ta->dtype != MALUS_F32 || ta->len < kLazyMin || !one_element_f32(b) || tb_->ndim > ta->ndim) return 0;
  int64_t z = make_lazy(ta->shape, ta->ndim, a, b, 0);
  tb(z)->causal_zero = ta->causal_zero;   // 0 * s stays 0 (the multiplier is taken to be finite)
  return z;
}

// a * w for a vector w along a's last dim (b of shape [C], a [..., C]),
// deferred; 0 when not applicable.
int64_t lazy_colscale(int64_t a, int64_t b) {
  auto *ta = tb(a), *tw = tb(b);
  if (ta->dtype != MALUS_F32 || ta->len < kLazyMin || ta->lazy || ta->ndim < 1 || tw->dtype != MALUS_F32 ||
      tw->ndim != 1 || tw->len < 2 || tw->len != ta->shape[ta->ndim - 1])
    return 0;
  return make_lazy(ta->shape, ta->ndim, a, 0, 0, b);
}

// (x * s) + m for a deferred x * s and an m of its trailing shape, deferred; 0
// when not applicable.
int64_t lazy_add(int64_t a, int64_t b) {
  auto *ta = tb(a), *tm = tb(b);
  if (!ta->lazy || !ta->lazy->scale || ta->lazy->addend || ta->lazy->colscale || tm->dtype != MALUS_F32 ||
      tm->ndim > ta->ndim ||
      tm->len == 0)
    return 0;
  for (int i = 0; i < tm->ndim; ++i)
    if (tm->shape[i] != ta->shape[ta->ndim - tm->ndim + i]) return 0;
  return make_lazy(ta->shape, ta->ndim, ta->lazy->src, ta->lazy->scale, b);
}

// The gradient of a same-shape operand is the incoming gradient itself: a new
// handle on the same data (gradients are never written in place); otherwise
// summed down to the target shape.
int64_t sum_to_shape_alias(int64_t g, const Shape& target) {
  Shape s = shape_of(g);
  bool same = s.ndim == target.ndim;
  for (int i = 0; same && i < s.ndim; ++i) same = s.d[i] == target.d[i];
  return same ? alias_of(g) : sum_to_shape(g, target);
}

int64_t scaled_copy(int64_t x, float c) {
  int64_t out = alloc_like(x);
  scalar_op_imm(kSMul, fptr(x), c, fptr(out), tb(x)->len);
  return out;
}

int64_t expand_impl(int64_t small, int64_t tmpl, int64_t axis) {
  Shape s = shape_of(tmpl);
  int ax = normalize_axis(axis, s.ndim);
  size_t outer, asz, inner;
  split_axis(s, ax, &outer, &asz, &inner);
  if (tb(small)->len < outer * inner)
    panic("expand_axis: source has %zu elements, needs %zu", tb(small)->len, outer * inner);
  int64_t out = alloc_shape(s);
  expand_axis(fptr(small), fptr(out), outer, asz, inner);
  return out;
}

std::vector<int> normalize_perm(const size_t* raw, size_t n, int rank) {
  std::vector<int> p;
  if (n == 0) {
    if (rank != 2) panic("transpose() with no dim args requires a 2-D tensor, got rank %d", rank);
    return {1, 0};
  }
  if (n == 2) {  // metal.rs:1303-1312: two args always mean "swap these axes"
    size_t i = raw[0], j = raw[1];
    if ((int)i >= rank || (int)j >= rank)
      panic("transpose axis %zu or %zu out of range for rank-%d tensor", i, j, rank);
    for (int k = 0; k < rank; ++k) p.push_back(k);
    std::swap(p[i], p[j]);
    return p;
  }
  if ((int)n == rank) {
    std::vector<bool> seen(rank, false);
    for (size_t k = 0; k < n; ++k) {
      if ((int)raw[k] >= rank) panic("permute dim %zu out of range for rank-%d tensor", raw[k], rank);
      if (seen[raw[k]]) panic("permute has duplicate dim %zu", raw[k]);
      seen[raw[k]] = true;
      p.push_back((int)raw[k]);
    }
    return p;
  }
  panic("permute/transpose got %zu dim args for rank-%d tensor; expected 0, 2, or %d", n, rank, rank);
}

// A permute is a view of the input's storage with its dims reordered (no
// copy): a GEMM reads it through its strides when it splits its operands, and
// any other consumer's raw-pointer access materialises it once.
int64_t permute_impl(int64_t x, const std::vector<int>& perm) {
  Shape s = shape_of(x);
  const View in = view_of(x);
  View v;
  size_t shape[kMaxRank];
  for (int d = 0; d < s.ndim; ++d) {
    shape[d] = s.d[perm[d]];
    v.d[d] = in.d[perm[d]];
  }
  return make_view(x, shape, s.ndim, v);
}

// Tensor h read as a GEMM operand [nz][rows][cols] (a view of its storage;
// a tensor whose memory cannot be read so is materialised first).
GemmOperand operand_of(int64_t h, size_t nz, size_t rows, size_t cols) {
  auto* t = tb(h);
  if (t->lazy && t->lazy->scale && !t->lazy->addend && !t->lazy->colscale && !tb(t->lazy->src)->lazy) {
    // x * s read straight from x: the split applies the multiply
    GemmOperand o = operand_of(t->lazy->src, nz, rows, cols);
    o.scale_dev = fptr(t->lazy->scale);
    return o;
  }
  if (t->lazy && t->lazy->colscale && !t->lazy->scale && !t->lazy->addend && !tb(t->lazy->src)->lazy &&
      t->ndim > 0 && cols == t->shape[t->ndim - 1]) {
    // x * w along the last dim (the operand's columns): the split applies it
    GemmOperand o = operand_of(t->lazy->src, nz, rows, cols);
    o.colscale_dev = fptr(t->lazy->colscale);
    return o;
  }
  const size_t dims[3] = {nz, rows, cols};
  View v;
  if (!view_as(h, dims, 3, &v)) {
    materialize(h);
    if (!view_as(h, dims, 3, &v)) panic("matmul operand of %zu elements read as [%zu][%zu][%zu]", t->len, nz, rows, cols);
  }
  GemmOperand o;
  o.base = static_cast<const float*>(t->st->ptr);
  o.nz = (int64_t)nz;
  o.rows = (int64_t)rows;
  o.cols = (int64_t)cols;
  o.z = v.d[0];
  o.r = v.d[1];
  o.c = v.d[2];
  o.key = t->st->id;
  return o;
}

// tf32 planes of `out` ([rows, C], C its last dim) primed in the GEMM operand
// cache, for a result that a GEMM reads next (the MLP activation and its VJP);
// null when it is small, 1-D, or not 16-byte friendly.
float* prime_row_planes(int64_t out, const float* src, const float* src2) {
  const TensorBuffer* t = tb(out);
  if (t->len < kLazyMin || t->ndim < 2 || t->len % 4) return nullptr;
  const size_t C = t->shape[t->ndim - 1];
  if (C % 4 || ((uintptr_t)src | (uintptr_t)src2 | (uintptr_t)fptr(out)) & 15) return nullptr;
  return plane_cache_prime(operand_of(out, 1, t->len / C, C), 0);
}

void check_f32(int64_t h, const char* what) {
  if (tb(h)->dtype != MALUS_F32) panic("%s expects an f32 tensor, got dtype %d", what, tb(h)->dtype);
}

}  // namespace

extern "C" {

// ------------------------------------------------------------ tensor ops
int64_t tensor_matmul(int64_t ha, int64_t hb) {
  Shape a = shape_of(ha), b = shape_of(hb);
  check_f32(ha, "matmul");
  check_f32(hb, "matmul");
  GemmArgs g{};
  g.a_trans = false;
  g.b_trans = false;
  Shape o;
  if (a.ndim == 2 && b.ndim == 2) {
    if (a.d[1] != b.d[0])
      panic("matmul shape mismatch: [%zux%zu] @ [%zux%zu] — inner dims %zu != %zu", a.d[0], a.d[1],
            b.d[0], b.d[1], a.d[1], b.d[0]);
    g.M = (int)a.d[0]; g.K = (int)a.d[1]; g.N = (int)b.d[1]; g.batch = 1;
    o.ndim = 2; o.d[0] = a.d[0]; o.d[1] = b.d[1];
  } else if (a.ndim == 3 && b.ndim == 3) {
    if (a.d[0] != b.d[0]) panic("batched matmul batch dims must match: %zu vs %zu", a.d[0], b.d[0]);
    if (a.d[2] != b.d[1]) panic("batched matmul inner dims must match: %zu vs %zu", a.d[2], b.d[1]);
    g.batch = (int)a.d[0]; g.M = (int)a.d[1]; g.K = (int)a.d[2]; g.N = (int)b.d[2];
    o.ndim = 3; o.d[0] = a.d[0]; o.d[1] = a.d[1]; o.d[2] = b.d[2];
  } else if (a.ndim == 3 && b.ndim == 2) {
    if (a.d[2] != b.d[0]) panic("matmul shape mismatch: inner dims %zu != %zu", a.d[2], b.d[0]);
    // (B, M, K) @ (K, N) is one (B*M, K) @ (K, N) GEMM
    g.batch = 1; g.M = (int)(a.d[0] * a.d[1]); g.K = (int)a.d[2]; g.N = (int)b.d[1];
    o.ndim = 3; o.d[0] = a.d[0]; o.d[1] = a.d[1]; o.d[2] = b.d[1];
  } else {
    panic("tensor_matmul requires both inputs to be 2-D, both 3-D, or (3-D, 2-D); got rank %d and %d",
          a.ndim, b.ndim);
  }
  int64_t out = alloc_shape(o);
  tb(out)->gemm_out = true;
  g.C = fptr(out);
  g.ldc = g.N;
  g.strideC = g.batch > 1 ? (int64_t)g.M * g.N : 0;
  if (o.numel() == 0) return out;
  if (g.K == 0) {
    MALUS_CUDA(cudaMemsetAsync(g.C, 0, o.numel() * 4, stream()));
    return out;
  }
  if (a.ndim == 3 && tb(ha)->causal_zero && g.M == g.K) g.a_zero = kCausalALower;
  g.A = operand_of(ha, (size_t)g.batch, (size_t)g.M, (size_t)g.K);
  g.B = operand_of(hb, b.ndim == 3 ? (size_t)g.batch : 1, (size_t)g.K, (size_t)g.N);
  gemm(g);
  return out;
}

int64_t tensor_permute(int64_t h, const size_t* perm, size_t ndims) {
  auto p = normalize_perm(perm, perm ? ndims : 0, tb(h)->ndim);
  return permute_impl(h, p);
}

// ------------------------------------------------------------ forward fns
int64_t __broadcast_add_fwd(int64_t a, int64_t b) {
  if (int64_t z = lazy_add(a, b)) return z;
  return binary_broadcast(kAdd, a, b);
}
int64_t __broadcast_sub_fwd(int64_t a, int64_t b) { return binary_broadcast(kSub, a, b); }
int64_t __broadcast_mul_fwd(int64_t a, int64_t b) {
  if (int64_t z = lazy_scale(a, b)) return z;
  if (int64_t z = lazy_colscale(a, b)) return z;
  return binary_broadcast(kMul, a, b);
}
int64_t __broadcast_div_fwd(int64_t a, int64_t b) { return binary_broadcast(kDiv, a, b); }

int64_t __softmax_fwd(int64_t x, int64_t axis) {
  check_f32(x, "softmax");
  Shape s = shape_of(x);
  int ax = normalize_axis(axis, s.ndim);
  size_t outer, asz, inner;
  split_axis(s, ax, &outer, &asz, &inner);
  int64_t out = alloc_shape(s);
  const Lazy* z = tb(x)->lazy;
  if (z && inner == 1 && !tb(z->src)->lazy && (!z->addend || tb(z->addend)->len % asz == 0)) {
    // softmax(src * s + m): one pass over src (the scaled and masked scores
    // are never written).  Over scores plus the causal mask (-1e9 above the
    // diagonal) the probabilities there underflow to exactly 0 (for scores
    // below ~1e8 in magnitude): those elements are not read, and the result
    // is tagged so that the GEMMs reading it clip their K ranges.
    const TensorBuffer* m = z->addend ? tb(z->addend) : nullptr;
    const bool causal = m && m->causal_mask && m->ndim == 2 && m->shape[0] == asz && m->shape[1] == asz &&
                        s.ndim >= 2 && s.d[s.ndim - 2] == asz;
    const float* src = fptr(z->src);
    const float* add = z->addend ? fptr(z->addend) : nullptr;
    // the probabilities feed P V (and P^T dO in the backward), which read
    // them as tf32 planes: the kernel writes those as it goes, for the part
    // the causally clipped GEMMs read, instead of a later split re-reading P
    float* planes = nullptr;
    if (causal && asz % 128 == 0 && tb(out)->len >= kLazyMin &&
        softmax_rows_path(src, fptr(out), add, outer, asz, inner))
      planes = plane_cache_prime(operand_of(out, outer / asz, asz, asz), (int64_t)asz);
    softmax_fwd(src, fptr(out), outer, asz, inner, z->scale ? fptr(z->scale) : nullptr, add,
                z->addend ? tb(z->addend)->len / asz : 1, causal ? (int)asz : 0, planes,
                planes ? planes + tb(out)->len : nullptr);
    tb(out)->causal_zero = causal;
    return out;
  }
  softmax_fwd(fptr(x), fptr(out), outer, asz, inner);
  return out;
}

int64_t __layernorm_fwd(int64_t x, int64_t axis) {
  check_f32(x, "layernorm");
  Shape s = shape_of(x);
  int ax = normalize_axis(axis, s.ndim);
  size_t outer, asz, inner;
  split_axis(s, ax, &outer, &asz, &inner);
  int64_t y = alloc_shape(s);
  Shape vs = s;
  vs.d[ax] = 1;
  int64_t var = alloc_shape(vs);
  layernorm_fwd(fptr(x), fptr(y), fptr(var), outer, asz, inner, 1e-5f);
  return tuple2(y, var);
}

int64_t __cross_entropy_fwd(int64_t logits, int64_t targets) {
  Shape s = shape_of(logits), t = shape_of(targets);
  if (s.ndim != 2) panic("cross_entropy logits must be rank-2 [N, C], got rank %d", s.ndim);
  if (t.ndim != 1) panic("cross_entropy targets must be rank-1 [N], got rank %d", t.ndim);
  if (t.d[0] != s.d[0]) panic("cross_entropy logits N=%zu but targets has %zu elements", s.d[0], t.d[0]);
  int tdt = tb(targets)->dtype;
  if (tdt != MALUS_I32 && tdt != MALUS_I64) panic("cross_entropy targets must be Tensor<i32> or Tensor<i64>");
  int64_t probs = alloc_shape(s);
  int64_t loss = alloc_f32({1});
  xent_fwd(fptr(logits), vptr(targets), tdt, fptr(probs), fptr(loss), s.d[0], s.d[1]);
  return tuple2(loss, probs);
}

int64_t __embedding_fwd(int64_t weight, int64_t indices) {
  Shape w = shape_of(weight);
  if (w.ndim != 2) panic("embedding weight must be rank-2 [V, D], got rank %d", w.ndim);
  int idt = tb(indices)->dtype;
  if (idt != MALUS_I32 && idt != MALUS_I64)
    panic("integer index tensor must be Tensor<i32> or Tensor<i64>, got dtype %d", idt);
  size_t n = tb(indices)->len;
  int64_t out = alloc_f32({n, w.d[1]});
  embedding_fwd(fptr(weight), vptr(indices), idt, fptr(out), n, w.d[0], w.d[1]);
  return out;
}

int64_t __gelu_fwd(int64_t x) {
  int64_t out = alloc_like(x);
  const float* a = fptr(x);
  // the MLP's activation (GELU of a GEMM's output) feeds the down product
  if (float* pl = tb(x)->gemm_out ? prime_row_planes(out, a, a) : nullptr) gelu_planes(a, nullptr, fptr(out), pl, pl + tb(out)->len, tb(out)->len);
  else unary_op(kGelu, a, fptr(out), tb(x)->len);
  return out;
}

int64_t __reduce_sum_fwd(int64_t x, int64_t axis, int64_t keepdim) { return reduce_impl(kRSum, x, axis, keepdim); }
int64_t __reduce_mean_fwd(int64_t x, int64_t axis, int64_t keepdim) { return reduce_impl(kRMean, x, axis, keepdim); }
int64_t __reduce_max_fwd(int64_t x, int64_t axis, int64_t keepdim) { return reduce_impl(kRMax, x, axis, keepdim); }
int64_t __reduce_var_fwd(int64_t x, int64_t axis, int64_t keepdim) { return reduce_impl(kRVar, x, axis, keepdim); }

int64_t __reduce_all_sum_fwd(int64_t x) {
  int64_t out = alloc_f32({1});
  size_t n = tb(x)->len;
  if (n == 0) scalar_op_imm(kSFill, nullptr, 0.0f, fptr(out), 1);
  else reduce_axis(kRSum, fptr(x), fptr(out), 1, n, 1);
  return out;
}

int64_t __permute_nd_fwd(int64_t x, int64_t p0, int64_t p1, int64_t p2, int64_t p3, int64_t p4,
                         int64_t p5, int64_t p6, int64_t p7) {
  int r = tb(x)->ndim;
  int64_t all[8] = {p0, p1, p2, p3, p4, p5, p6, p7};
  std::vector<int> perm(all, all + r);
  return permute_impl(x, perm);
}

int64_t __transpose_2d_fwd(int64_t x) {
  if (tb(x)->ndim != 2) panic("transpose_2d expects a 2-D tensor");
  return permute_impl(x, {1, 0});
}

int64_t __scale_fwd(int64_t x, float c) { return scaled_copy(x, c); }

int64_t __fill_like_fwd(int64_t x, float c) {
  int64_t out = alloc_like(x);
  scalar_op_imm(kSFill, nullptr, c, fptr(out), tb(x)->len);
  return out;
}

int64_t __eq_fwd(int64_t a, int64_t b) {
  int64_t out = alloc_like(a);
  unary_bwd(kEq, fptr(a), fptr(b), fptr(out), tb(a)->len);
  return out;
}

int64_t __expand_axis_fwd(int64_t small, int64_t x_template, int64_t axis) {
  return expand_impl(small, x_template, axis);
}

int64_t __sum_to_shape_bwd(int64_t dout, int64_t target) { return sum_to_shape(dout, shape_of(target)); }

int64_t __rsqrt_eps_fwd(int64_t v, float eps) {
  int64_t out = alloc_like(v);
  unary_op(kRsqrtEps, fptr(v), fptr(out), tb(v)->len, eps);
  return out;
}

// ------------------------------------------------------------ BwdSlot fns
int64_t __add_bwd_a(int64_t dout, int64_t a) { return sum_to_shape_alias(dout, shape_of(a)); }
int64_t __add_bwd_b(int64_t dout, int64_t b) { return sum_to_shape_alias(dout, shape_of(b)); }
int64_t __sub_bwd_a(int64_t dout, int64_t a) { return sum_to_shape_alias(dout, shape_of(a)); }
int64_t __sub_bwd_b(int64_t dout, int64_t b) {
  Shape sb = shape_of(b), sd = shape_of(dout);
  bool same = sb.ndim == sd.ndim;
  for (int i = 0; same && i < sb.ndim; ++i) same = sb.d[i] == sd.d[i];
  if (same) {   // -g in one pass
    int64_t r = alloc_shape(sb);
    unary_op(kNeg, fptr(dout), fptr(r), tb(r)->len);
    return r;
  }
  int64_t r = sum_to_shape(dout, sb);
  unary_op(kNeg, fptr(r), fptr(r), tb(r)->len);  // -(sum g) == sum(-g) exactly
  return r;
}
int64_t __mul_bwd_a(int64_t dout, int64_t a, int64_t b) {
  int64_t full = lazy_scale(dout, b);   // dout * s for a one-element b, dout * w for a vector: deferred
  if (!full) full = lazy_colscale(dout, b);
  if (!full) full = binary_broadcast(kMul, dout, b);
  int64_t r = sum_to_shape_alias(full, shape_of(a));
  tensor_release(full);
  return r;
}
int64_t __mul_bwd_b(int64_t dout, int64_t a, int64_t b) {
  auto *td = tb(dout), *tw = tb(b);
  if (tw->ndim == 1 && tw->len > 1 && td->ndim >= 2 && tw->len == td->shape[td->ndim - 1] && same_shape(dout, a) &&
      tb(a)->dtype == MALUS_F32 && tw->dtype == MALUS_F32) {
    // the gradient of a gain vector: column sums of dout * a in one pass (the
    // products are not written), same partition and order as summing the
    // materialised product down to [C]
    int64_t r = alloc_shape(shape_of(b));
    const size_t C = tw->len;
    reduce_axis_sum_product(fptr(dout), fptr(a), fptr(r), 1, td->len / C, C);
    return r;
  }
  int64_t full = binary_broadcast(kMul, dout, a);
  int64_t r = sum_to_shape(full, shape_of(b));
  tensor_release(full);
  return r;
}
int64_t __div_bwd_a(int64_t dout, int64_t a, int64_t b) {
  int64_t full = binary_broadcast(kDiv, dout, b);
  int64_t r = sum_to_shape(full, shape_of(a));
  tensor_release(full);
  return r;
}
int64_t __div_bwd_b(int64_t dout, int64_t a, int64_t b) {
  int64_t t1 = binary_broadcast(kMul, dout, a);
  unary_op(kNeg, fptr(t1), fptr(t1), tb(t1)->len);
  int64_t bsq = binary_broadcast(kMul, b, b);
  int64_t full = binary_broadcast(kDiv, t1, bsq);
  tensor_release(t1);
  tensor_release(bsq);
  int64_t r = sum_to_shape(full, shape_of(b));
  tensor_release(full);
  return r;
}

#define UBWD(NAME, OP)                                        \
  int64_t NAME(int64_t x, int64_t dout) {                     \
    int64_t out = alloc_like(x);                              \
    unary_bwd(OP, fptr(x), fptr(dout), fptr(out), tb(x)->len); \
    return out;                                               \
  }
UBWD(__sigmoid_bwd, kSigmoidBwd)
UBWD(__relu_bwd, kReluBwd)
UBWD(__tanh_bwd, kTanhBwd)
UBWD(__sqrt_bwd, kSqrtBwd)
UBWD(__abs_bwd, kAbsBwd)
#undef UBWD

int64_t __gelu_bwd(int64_t x, int64_t dout) {
  int64_t out = alloc_like(x);
  const float* a = fptr(x);
  const float* g = fptr(dout);
  // its VJP at a GEMM's output feeds both VJPs of that GEMM
  if (float* pl = tb(x)->gemm_out ? prime_row_planes(out, a, g) : nullptr) gelu_planes(a, g, fptr(out), pl, pl + tb(out)->len, tb(out)->len);
  else unary_bwd(kGeluBwd, a, g, fptr(out), tb(x)->len);
  return out;
}

int64_t __sum_bwd(int64_t x, int64_t dout) {
  int64_t out = alloc_like(x);
  fill_from_dev_scalar(fptr(out), fptr(dout), tb(x)->len);
  return out;
}

int64_t __reduce_sum_axis_bwd(int64_t x, int64_t dout, int64_t axis) { return expand_impl(dout, x, axis); }

int64_t __reduce_mean_axis_bwd(int64_t x, int64_t dout, int64_t axis) {
  int ax = normalize_axis(axis, tb(x)->ndim);
  float n = (float)tb(x)->shape[ax];
  int64_t sc = scaled_copy(dout, 1.0f / n);
  int64_t r = expand_impl(sc, x, axis);
  tensor_release(sc);
  return r;
}

int64_t __reduce_max_axis_bwd(int64_t x, int64_t y, int64_t dout, int64_t axis) {
  int64_t ybc = expand_impl(y, x, axis);
  int64_t mask = __eq_fwd(x, ybc);
  int64_t dbc = expand_impl(dout, x, axis);
  int64_t r = binary_broadcast(kMul, dbc, mask);
  tensor_release(ybc);
  tensor_release(mask);
  tensor_release(dbc);
  return r;
}

int64_t __reduce_var_axis_bwd(int64_t x, int64_t dout, int64_t axis) {
  int ax = normalize_axis(axis, tb(x)->ndim);
  float n = (float)tb(x)->shape[ax];
  int64_t mean = reduce_impl(kRMean, x, axis, 1);
  int64_t mbc = expand_impl(mean, x, axis);
  int64_t xm = binary_broadcast(kSub, x, mbc);
  scalar_op_imm(kSMul, fptr(xm), 2.0f / n, fptr(xm), tb(xm)->len);
  int64_t dbc = expand_impl(dout, x, axis);
  int64_t r = binary_broadcast(kMul, dbc, xm);
  tensor_release(mean);
  tensor_release(mbc);
  tensor_release(xm);
  tensor_release(dbc);
  return r;
}

int64_t __softmax_bwd(int64_t s, int64_t dout, int64_t axis) {
  Shape sh = shape_of(s);
  int ax = normalize_axis(axis, sh.ndim);
  size_t outer, asz, inner;
  split_axis(sh, ax, &outer, &asz, &inner);
  int64_t dx = alloc_shape(sh);
  // s (dout - sum) is 0 where s is: past the diagonal of a causal-zero s,
  // which is then not read (nor dout there)
  const bool causal = tb(s)->causal_zero && inner == 1 && sh.ndim >= 2 && sh.d[sh.ndim - 2] == asz;
  softmax_bwd(fptr(s), fptr(dout), fptr(dx), outer, asz, inner, causal ? (int)asz : 0);
  tb(dx)->causal_zero = causal;
  return dx;
}

int64_t __layernorm_bwd(int64_t y, int64_t var_h, int64_t dout, int64_t axis) {
  Shape sh = shape_of(y);
  int ax = normalize_axis(axis, sh.ndim);
  size_t outer, asz, inner;
  split_axis(sh, ax, &outer, &asz, &inner);
  if (tb(var_h)->len != outer * inner)
    panic("layernorm_bwd: variance has %zu elements, expected %zu (keepdim at axis)",
          tb(var_h)->len, outer * inner);
  int64_t dx = alloc_shape(sh);
  const Lazy* z = tb(dout)->lazy;
  if (z && z->colscale && !z->scale && !z->addend && !tb(z->src)->lazy && inner == 1 &&
      tb(z->colscale)->len == asz && same_shape(dout, y)) {
    // dout = g * w (the deferred gain VJP): read fused
    layernorm_bwd(fptr(y), fptr(var_h), fptr(z->src), fptr(dx), outer, asz, inner, 1e-5f, fptr(z->colscale));
    return dx;
  }
  layernorm_bwd(fptr(y), fptr(var_h), fptr(dout), fptr(dx), outer, asz, inner, 1e-5f);
  return dx;
}

int64_t __cross_entropy_bwd(int64_t probs, int64_t targets, int64_t dout) {
  Shape s = shape_of(probs);
  int64_t dx = alloc_shape(s);
  xent_bwd(fptr(probs), vptr(targets), tb(targets)->dtype, fptr(dout), fptr(dx), s.d[0], s.d[1]);
  return dx;
}

int64_t __embedding_bwd(int64_t weight, int64_t indices, int64_t dout) {
  Shape w = shape_of(weight);
  int64_t dw = alloc_shape(w);
  embedding_bwd(fptr(dout), vptr(indices), tb(indices)->dtype, fptr(dw), tb(indices)->len, w.d[0], w.d[1]);
  return dw;
}

int64_t __matmul_bwd_a(int64_t a, int64_t b, int64_t dout) {
  Shape sa = shape_of(a), sb = shape_of(b);
  int64_t da = alloc_shape(sa);
  GemmArgs g{};
  if (sb.ndim == 3) {
    // dA[b] = dC[b] @ B[b]^T : (M=m, N=k, K=n)
    g.batch = (int)sb.d[0]; g.M = (int)(tb(dout)->len / (sb.d[0] * sb.d[2])); g.N = (int)sb.d[1];
    g.K = (int)sb.d[2];
    g.a_trans = false;
    g.b_trans = true;
    g.strideC = (int64_t)g.M * g.N;
  } else {
    // (2,2) and (3,2): dA = dC @ B^T over all leading rows
    g.batch = 1; g.M = (int)(tb(dout)->len / sb.d[1]); g.N = (int)sb.d[0]; g.K = (int)sb.d[1];
    g.a_trans = false;
    g.b_trans = true;
    g.strideC = 0;
  }
  g.C = fptr(da);
  g.ldc = g.N;
  if (sa.numel()) {
    if (g.K == 0) {
      MALUS_CUDA(cudaMemsetAsync(fptr(da), 0, sa.numel() * 4, stream()));
    } else {
      if (sb.ndim == 3 && tb(dout)->causal_zero && g.M == g.K) g.a_zero = kCausalALower;
      g.A = operand_of(dout, (size_t)g.batch, (size_t)g.M, (size_t)g.K);
      g.B = operand_of(b, (size_t)g.batch, (size_t)g.N, (size_t)g.K);   // stored [N][K]
      gemm(g);
    }
  }
  return da;
}

int64_t __matmul_bwd_b(int64_t a, int64_t b, int64_t dout) {
  Shape sa = shape_of(a), sb = shape_of(b);
  int64_t db = alloc_shape(sb);
  GemmArgs g{};
  if (sa.ndim == 3 && sb.ndim == 3) {
    // dB[b] = A[b]^T @ dC[b] : (M=k, N=n, K=m)
    g.batch = (int)sa.d[0]; g.M = (int)sa.d[2]; g.N = (int)sb.d[2]; g.K = (int)sa.d[1];
    g.strideC = (int64_t)g.M * g.N;
  } else {
    // (2,2): A^T @ dC ; (3,2): sum_b A[b]^T @ dC[b] == A'^T @ dC' with K = B*m
    size_t kdim = sa.d[sa.ndim - 1];
    g.batch = 1; g.M = (int)kdim; g.N = (int)sb.d[1]; g.K = (int)(tb(a)->len / kdim);
    g.strideC = 0;
  }
  g.a_trans = true;
  g.b_trans = false;
  g.C = fptr(db);
  g.ldc = g.N;
  if (sb.numel()) {
    if (g.K == 0) {
      MALUS_CUDA(cudaMemsetAsync(fptr(db), 0, sb.numel() * 4, stream()));
    } else {
      // A = a^T: zero below the diagonal when a is zero above it
      if (sa.ndim == 3 && sb.ndim == 3 && tb(a)->causal_zero && g.M == g.K) g.a_zero = kCausalAUpper;
      g.A = operand_of(a, (size_t)g.batch, (size_t)g.K, (size_t)g.M);      // stored [K][M]
      g.B = operand_of(dout, (size_t)g.batch, (size_t)g.K, (size_t)g.N);
      gemm(g);
    }
  }
  return db;
}

}  // extern "C"
