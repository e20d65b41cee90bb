// Elementwise kernels: NumPy-broadcast binops, scalar-broadcast builtins,
// unary builtins and their VJPs.  All are HBM-bound, so every kernel is a
// grid-stride loop sized to a multiple of the SM count, with 16-byte (float4)
// loads/stores on the contiguous fast paths.
//
// Math follows the reference's device code:
//   broadcast binops   crates/malus-stdlib/stdlib/broadcast_binop.ml:10-80
//   scalar builtins    crates/malus-codegen-gpu/src/lib.rs:403-418
//   unary builtins     crates/malus-codegen-gpu/src/lib.rs:373-390
//   gelu / gelu bwd    stdlib/gelu.ml:5-10, stdlib/backward/transformer_bwd.ml:40-48
//   unary VJPs         stdlib/backward/unary_bwd.ml:6-91
#include "common.cuh"

namespace malus {

namespace {

constexpr int kThreads = 256;
constexpr float kGeluC0 = 0.7978845608028654f;
constexpr float kGeluC1 = 0.044715f;

__device__ __forceinline__ float bin(int op, float a, float b) {
  switch (op) {
    case kAdd: return a + b;
    case kSub: return a - b;
    case kMul: return a * b;
    default: return a / b;
  }
}

template <int OP>
__device__ __forceinline__ float binT(float a, float b) {
  if (OP == kAdd) return a + b;
  if (OP == kSub) return a - b;
  if (OP == kMul) return a * b;
  return a / b;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// ---- same-shape binary (also the reference's synthesized malus_add...) ----
template <int OP>
__global__ void k_binary_same(const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ out, size_t n, bool vec) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    size_t n4 = n >> 2;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (size_t i = tid; i < n4; i += stride) {
      float4 x = a4[i], y = b4[i];
      o4[i] = make_float4(binT<OP>(x.x, y.x), binT<OP>(x.y, y.y), binT<OP>(x.z, y.z),
                          binT<OP>(x.w, y.w));
    }
    for (size_t i = (n4 << 2) + tid; i < n; i += stride) out[i] = binT<OP>(a[i], b[i]);
  } else {
    for (size_t i = tid; i < n; i += stride) out[i] = binT<OP>(a[i], b[i]);
  }
}

// ---- row broadcast: the smaller operand repeats with period P ----
// out[i] = full[i] op row[i % P]   (row_on_right) or row[i % P] op full[i]
template <int OP, bool ROW_RIGHT>
__global__ void k_binary_row(const float* __restrict__ full, const float* __restrict__ row,
                             float* __restrict__ out, size_t n, size_t P, bool vec) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {  // P % 4 == 0
    size_t n4 = n >> 2, P4 = P >> 2;
    const float4* f4 = reinterpret_cast<const float4*>(full);
    const float4* r4 = reinterpret_cast<const float4*>(row);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (size_t i = tid; i < n4; i += stride) {
      float4 x = f4[i], y = r4[i % P4];
      if (ROW_RIGHT)
        o4[i] = make_float4(binT<OP>(x.x, y.x), binT<OP>(x.y, y.y), binT<OP>(x.z, y.z),
                            binT<OP>(x.w, y.w));
      else
        o4[i] = make_float4(binT<OP>(y.x, x.x), binT<OP>(y.y, x.y), binT<OP>(y.z, x.z),
                            binT<OP>(y.w, x.w));
    }
  } else {
    for (size_t i = tid; i < n; i += stride) {
      float x = full[i], y = row[i % P];
      out[i] = ROW_RIGHT ? binT<OP>(x, y) : binT<OP>(y, x);
    }
  }
}

// ---- general strided broadcast ----
struct BcastMeta {
  int ndim;
  int64_t out_shape[kMaxRank];
  int64_t sa[kMaxRank];  // 0 on broadcast dims
  int64_t sb[kMaxRank];
};

__global__ void k_binary_general(int op, const float* __restrict__ a, const float* __restrict__ b,
                                 float* __restrict__ out, size_t n, BcastMeta m) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    size_t rem = i;
    int64_t ia = 0, ib = 0;
    for (int d = m.ndim - 1; d >= 0; --d) {
      int64_t idx = (int64_t)(rem % (size_t)m.out_shape[d]);
      rem /= (size_t)m.out_shape[d];
      ia += idx * m.sa[d];
      ib += idx * m.sb[d];
    }
    out[i] = bin(op, a[ia], b[ib]);
  }
}

// ---- scalar ops; the scalar comes from device memory or an immediate ----
template <int OP>
__device__ __forceinline__ float sop(float x, float s) {
  if (OP == kSAdd) return x + s;
  if (OP == kSSub) return x - s;
  if (OP == kSRSub) return s - x;
  if (OP == kSMul) return x * s;
  if (OP == kSDiv) return x / s;
  if (OP == kSRDiv) return s / x;
  return s;  // kSFill
}

template <int OP>
__global__ void k_scalar(const float* __restrict__ a, const float* __restrict__ s_dev, float s_imm,
                         float* __restrict__ out, size_t n, bool vec) {
  float s = s_dev ? *s_dev : s_imm;
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    size_t n4 = n >> 2;
    float4* o4 = reinterpret_cast<float4*>(out);
    const float4* a4 = reinterpret_cast<const float4*>(a);
    for (size_t i = tid; i < n4; i += 2 * stride) {   // two chunks' loads in flight
      const size_t i2 = i + stride;
      const float4 x = OP == kSFill ? make_float4(0, 0, 0, 0) : a4[i];
      const float4 x2 = OP == kSFill || i2 >= n4 ? x : a4[i2];
      o4[i] = make_float4(sop<OP>(x.x, s), sop<OP>(x.y, s), sop<OP>(x.z, s), sop<OP>(x.w, s));
      if (i2 < n4) o4[i2] = make_float4(sop<OP>(x2.x, s), sop<OP>(x2.y, s), sop<OP>(x2.z, s), sop<OP>(x2.w, s));
    }
    for (size_t i = (n4 << 2) + tid; i < n; i += stride)
      out[i] = sop<OP>(OP == kSFill ? 0.f : a[i], s);
  } else {
    for (size_t i = tid; i < n; i += stride) out[i] = sop<OP>(OP == kSFill ? 0.f : a[i], s);
  }
}

// ---- unary ----
template <int OP>
__device__ __forceinline__ float uop(float x, float p) {
  if (OP == kRelu) return fmaxf(0.0f, x);
  if (OP == kSigmoid) return 1.0f / (1.0f + expf(-x));
  if (OP == kTanh) return tanhf(x);
  if (OP == kExp) return expf(x);
  if (OP == kLog) return logf(x);
  if (OP == kSqrt) return sqrtf(x);
  if (OP == kAbs) return fabsf(x);
  if (OP == kGelu) {
    float x3 = x * x * x;
    float inner = kGeluC0 * (x + kGeluC1 * x3);
    return 0.5f * x * (1.0f + tanhf(inner));
  }
  if (OP == kRsqrtEps) return rsqrtf(x + p);
  return -x;  // kNeg
}

template <int OP>
__global__ void k_unary(const float* __restrict__ a, float* __restrict__ out, size_t n, float p,
                        bool vec) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    size_t n4 = n >> 2;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    float4* o4 = reinterpret_cast<float4*>(out);
    if (OP == kGelu) {   // compute-heavy: one chunk per iteration measured faster
      for (size_t i = tid; i < n4; i += stride) {
        const float4 x = a4[i];
        o4[i] = make_float4(uop<OP>(x.x, p), uop<OP>(x.y, p), uop<OP>(x.z, p), uop<OP>(x.w, p));
      }
    } else {
      // two chunks per iteration, both loads issued before either is computed
      for (size_t i = tid; i < n4; i += 2 * stride) {
        const size_t i2 = i + stride;
        const float4 x = a4[i];
        const float4 x2 = i2 < n4 ? a4[i2] : x;
        o4[i] = make_float4(uop<OP>(x.x, p), uop<OP>(x.y, p), uop<OP>(x.z, p), uop<OP>(x.w, p));
        if (i2 < n4) o4[i2] = make_float4(uop<OP>(x2.x, p), uop<OP>(x2.y, p), uop<OP>(x2.z, p), uop<OP>(x2.w, p));
      }
    }
    for (size_t i = (n4 << 2) + tid; i < n; i += stride) out[i] = uop<OP>(a[i], p);
  } else {
    for (size_t i = tid; i < n; i += stride) out[i] = uop<OP>(a[i], p);
  }
}

// The same, also writing the result's tf32 planes (hi, lo; the operand
// split's expressions) for a GEMM that reads it next; 16-byte-aligned arrays
// of a multiple of 4 elements.
template <int OP>
__global__ void k_unary_planes(const float* __restrict__ a, float* __restrict__ out, float* __restrict__ hi,
                               float* __restrict__ lo, size_t n4) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 x = reinterpret_cast<const float4*>(a)[i];
    const float4 y = make_float4(uop<OP>(x.x, 0.f), uop<OP>(x.y, 0.f), uop<OP>(x.z, 0.f), uop<OP>(x.w, 0.f));
    const float4 h = make_float4(tf32_round(y.x), tf32_round(y.y), tf32_round(y.z), tf32_round(y.w));
    reinterpret_cast<float4*>(out)[i] = y;
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] =
        make_float4(tf32_round(y.x - h.x), tf32_round(y.y - h.y), tf32_round(y.z - h.z), tf32_round(y.w - h.w));
  }
}

// ---- unary VJPs: out = f(x or y, dout) ----
template <int OP>
__device__ __forceinline__ float ubwd(float x, float g) {
  if (OP == kSigmoidBwd) return g * x * (1.0f - x);           // x = s
  if (OP == kReluBwd) return x > 0.0f ? g : 0.0f;
  if (OP == kTanhBwd) return g * (1.0f - x * x);              // x = t
  if (OP == kSqrtBwd) return g / (2.0f * x);                  // x = s
  if (OP == kAbsBwd) return x > 0.0f ? g : (x < 0.0f ? -g : 0.0f);
  if (OP == kGeluBwd) {
    float x3 = x * x * x;
    float gg = kGeluC0 * (x + kGeluC1 * x3);
    float t = tanhf(gg);
    float gp = kGeluC0 * (1.0f + 3.0f * kGeluC1 * x * x);
    float deriv = 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * gp;
    return g * deriv;
  }
  return x == g ? 1.0f : 0.0f;  // kEq (a, b)
}

template <int OP>
__global__ void k_unary_bwd(const float* __restrict__ x, const float* __restrict__ g,
                            float* __restrict__ out, size_t n, bool vec) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    size_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (size_t i = tid; i < n4; i += stride) {
      float4 a = x4[i], b = g4[i];
      o4[i] = make_float4(ubwd<OP>(a.x, b.x), ubwd<OP>(a.y, b.y), ubwd<OP>(a.z, b.z),
                          ubwd<OP>(a.w, b.w));
    }
    for (size_t i = (n4 << 2) + tid; i < n; i += stride) out[i] = ubwd<OP>(x[i], g[i]);
  } else {
    for (size_t i = tid; i < n; i += stride) out[i] = ubwd<OP>(x[i], g[i]);
  }
}

// examples/xor.ml:1-2 — kernel sigmoid_backward(grad_out, sig_z) = g*s*(1-s)
__global__ void k_sigmoid_backward_user(const float* __restrict__ g, const float* __restrict__ s,
                                        float* __restrict__ out, size_t n) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    float sv = s[i];
    out[i] = g[i] * sv * (1.0f - sv);
  }
}

// reduce_bwd.ml:10-18: replicate [outer, inner] back to [outer, axis, inner]
__global__ void k_expand_axis(const float* __restrict__ small, float* __restrict__ out,
                              size_t n, size_t axis_sz, size_t inner) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t s1 = axis_sz * inner;
  for (size_t i = tid; i < n; i += stride) {
    size_t o = i / s1;
    size_t iv = (i - o * s1) % inner;
    out[i] = small[o * inner + iv];
  }
}

}  // namespace

#define LAUNCH(kern, n, ...)                                                      \
  do {                                                                            \
    if ((n) == 0) break;                                                          \
    kern<<<grid_for(((n) + 3) / 4, kThreads), kThreads, 0, stream()>>>(__VA_ARGS__); \
    count_launch();                                                               \
    after_launch(#kern);                                                          \
  } while (0)

void binary_same(int op, const float* a, const float* b, float* out, size_t n) {
  bool vec = aligned16(a) && aligned16(b) && aligned16(out);
  switch (op) {
    case kAdd: LAUNCH(k_binary_same<kAdd>, n, a, b, out, n, vec); break;
    case kSub: LAUNCH(k_binary_same<kSub>, n, a, b, out, n, vec); break;
    case kMul: LAUNCH(k_binary_same<kMul>, n, a, b, out, n, vec); break;
    default: LAUNCH(k_binary_same<kDiv>, n, a, b, out, n, vec); break;
  }
}

static void binary_row(int op, bool row_right, const float* full, const float* row, float* out,
                       size_t n, size_t P) {
  bool vec = (P % 4 == 0) && aligned16(full) && aligned16(row) && aligned16(out);
#define ROWCASE(OPV)                                                             \
  case OPV:                                                                      \
    if (row_right) LAUNCH((k_binary_row<OPV, true>), n, full, row, out, n, P, vec); \
    else LAUNCH((k_binary_row<OPV, false>), n, full, row, out, n, P, vec);       \
    break;
  switch (op) { ROWCASE(kAdd) ROWCASE(kSub) ROWCASE(kMul) ROWCASE(kDiv) }
#undef ROWCASE
}

// NumPy right-aligned broadcast of a op b.  Result shape follows
// broadcast_result_shape (metal.rs:1024-1043); the operand order is always
// a op b (the host-side semantics of metal.rs:1045-1072).
int64_t binary_broadcast(int op, int64_t ha, int64_t hb) {
  Shape sa = shape_of(ha), sb = shape_of(hb);
  if (same_shape(ha, hb)) {
    int64_t out = alloc_shape(sa);
    binary_same(op, fptr(ha), fptr(hb), fptr(out), sa.numel());
    return out;
  }
  int n = std::max(sa.ndim, sb.ndim);
  Shape so;
  so.ndim = n;
  size_t pa[kMaxRank], pb[kMaxRank];
  for (int i = 0; i < n; ++i) {
    int ia = i - (n - sa.ndim), ib = i - (n - sb.ndim);
    pa[i] = ia >= 0 ? sa.d[ia] : 1;
    pb[i] = ib >= 0 ? sb.d[ib] : 1;
    if (pa[i] == pb[i] || pb[i] == 1) so.d[i] = pa[i];
    else if (pa[i] == 1) so.d[i] = pb[i];
    else panic("broadcast shape mismatch at dim %d: %zu vs %zu", i, pa[i], pb[i]);
  }
  int64_t out = alloc_shape(so);
  size_t total = so.numel();
  if (total == 0) return out;
  const float* A = fptr(ha);
  const float* B = fptr(hb);
  size_t la = sa.numel(), lb = sb.numel();
  // Fast path: one operand is the full output and the other repeats with a
  // period equal to its own length (its shape is the trailing dims of the
  // output, with leading 1s) — e.g. the layernorm gain [M,C] * [C].
  auto is_trailing = [&](const size_t* p, size_t len) {
    size_t prod = 1;
    int d = n - 1;
    for (; d >= 0 && prod < len; --d) {
      if (p[d] != so.d[d]) return false;
      prod *= p[d];
    }
    for (; d >= 0; --d) if (p[d] != 1) return false;
    return prod == len;
  };
  if (la == total && is_trailing(pb, lb)) {
    binary_row(op, true, A, B, fptr(out), total, lb);
    return out;
  }
  if (lb == total && is_trailing(pa, la)) {
    binary_row(op, false, B, A, fptr(out), total, la);
    return out;
  }
  BcastMeta m;
  m.ndim = n;
  int64_t sta = 1, stb = 1;
  for (int d = n - 1; d >= 0; --d) {
    m.out_shape[d] = (int64_t)so.d[d];
    m.sa[d] = pa[d] == 1 ? 0 : sta;
    m.sb[d] = pb[d] == 1 ? 0 : stb;
    sta *= (int64_t)pa[d];
    stb *= (int64_t)pb[d];
  }
  k_binary_general<<<grid_for(total, kThreads), kThreads, 0, stream()>>>(op, A, B, fptr(out),
                                                                          total, m);
  count_launch();
  after_launch("k_binary_general");
  return out;
}

// kernel_dispatch_v2 form of __broadcast_*_kernel: out has a's shape and b is
// projected through its own strides on dims > 1 (broadcast_binop.ml:10-27).
void binary_project_into_a(int op, int64_t ha, int64_t hb, float* out) {
  Shape sa = shape_of(ha), sb = shape_of(hb);
  size_t total = sa.numel();
  if (!total) return;
  BcastMeta m;
  m.ndim = sa.ndim;
  int off = sa.ndim - sb.ndim;
  int64_t sta = 1;
  int64_t bst[kMaxRank];
  int64_t s = 1;
  for (int d = sb.ndim - 1; d >= 0; --d) { bst[d] = s; s *= (int64_t)sb.d[d]; }
  for (int d = sa.ndim - 1; d >= 0; --d) {
    m.out_shape[d] = (int64_t)sa.d[d];
    m.sa[d] = sta;
    sta *= (int64_t)sa.d[d];
    int db = d - off;
    m.sb[d] = (db >= 0 && sb.d[db] > 1) ? bst[db] : 0;
  }
  k_binary_general<<<grid_for(total, kThreads), kThreads, 0, stream()>>>(op, fptr(ha), fptr(hb),
                                                                          out, total, m);
  count_launch();
  after_launch("k_binary_general");
}

void scalar_op_dev(int op, const float* a, const float* s_dev, float* out, size_t n) {
  bool vec = (a == nullptr || aligned16(a)) && aligned16(out);
  switch (op) {
    case kSAdd: LAUNCH(k_scalar<kSAdd>, n, a, s_dev, 0.f, out, n, vec); break;
    case kSSub: LAUNCH(k_scalar<kSSub>, n, a, s_dev, 0.f, out, n, vec); break;
    case kSRSub: LAUNCH(k_scalar<kSRSub>, n, a, s_dev, 0.f, out, n, vec); break;
    case kSMul: LAUNCH(k_scalar<kSMul>, n, a, s_dev, 0.f, out, n, vec); break;
    case kSDiv: LAUNCH(k_scalar<kSDiv>, n, a, s_dev, 0.f, out, n, vec); break;
    case kSRDiv: LAUNCH(k_scalar<kSRDiv>, n, a, s_dev, 0.f, out, n, vec); break;
    default: LAUNCH(k_scalar<kSFill>, n, a, s_dev, 0.f, out, n, vec); break;
  }
}

void scalar_op_imm(int op, const float* a, float s, float* out, size_t n) {
  bool vec = (a == nullptr || aligned16(a)) && aligned16(out);
  switch (op) {
    case kSAdd: LAUNCH(k_scalar<kSAdd>, n, a, nullptr, s, out, n, vec); break;
    case kSSub: LAUNCH(k_scalar<kSSub>, n, a, nullptr, s, out, n, vec); break;
    case kSRSub: LAUNCH(k_scalar<kSRSub>, n, a, nullptr, s, out, n, vec); break;
    case kSMul: LAUNCH(k_scalar<kSMul>, n, a, nullptr, s, out, n, vec); break;
    case kSDiv: LAUNCH(k_scalar<kSDiv>, n, a, nullptr, s, out, n, vec); break;
    case kSRDiv: LAUNCH(k_scalar<kSRDiv>, n, a, nullptr, s, out, n, vec); break;
    default: LAUNCH(k_scalar<kSFill>, n, a, nullptr, s, out, n, vec); break;
  }
}

void fill_from_dev_scalar(float* out, const float* s_dev, size_t n) {
  scalar_op_dev(kSFill, nullptr, s_dev, out, n);
}

template <int OP>
__global__ void k_unary_bwd_planes(const float* __restrict__ x, const float* __restrict__ g,
                                   float* __restrict__ out, float* __restrict__ hi, float* __restrict__ lo,
                                   size_t n4) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 xv = reinterpret_cast<const float4*>(x)[i];
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    const float4 y = make_float4(ubwd<OP>(xv.x, gv.x), ubwd<OP>(xv.y, gv.y), ubwd<OP>(xv.z, gv.z),
                                 ubwd<OP>(xv.w, gv.w));
    const float4 h = make_float4(tf32_round(y.x), tf32_round(y.y), tf32_round(y.z), tf32_round(y.w));
    reinterpret_cast<float4*>(out)[i] = y;
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] =
        make_float4(tf32_round(y.x - h.x), tf32_round(y.y - h.y), tf32_round(y.z - h.z), tf32_round(y.w - h.w));
  }
}

// GELU and its VJP with the result's tf32 planes (see k_unary_planes); n % 4
// == 0 and every array 16-byte aligned.
void gelu_planes(const float* x, const float* g, float* out, float* hi, float* lo, size_t n) {
  if (!n) return;
  if (n % 4 || !aligned16(x) || (g && !aligned16(g)) || !aligned16(out) || !aligned16(hi) || !aligned16(lo))
    panic("gelu_planes: needs 16-byte-aligned arrays of a multiple of 4 elements");
  const size_t n4 = n / 4;
  if (g) {
    k_unary_bwd_planes<kGeluBwd><<<grid_for(n4, kThreads), kThreads, 0, stream()>>>(x, g, out, hi, lo, n4);
    count_launch();
    after_launch("k_unary_bwd_planes");
  } else {
    k_unary_planes<kGelu><<<grid_for(n4, kThreads), kThreads, 0, stream()>>>(x, out, hi, lo, n4);
    count_launch();
    after_launch("k_unary_planes");
  }
}

void unary_op(int op, const float* a, float* out, size_t n, float p) {
  bool vec = aligned16(a) && aligned16(out);
  switch (op) {
    case kRelu: LAUNCH(k_unary<kRelu>, n, a, out, n, p, vec); break;
    case kSigmoid: LAUNCH(k_unary<kSigmoid>, n, a, out, n, p, vec); break;
    case kTanh: LAUNCH(k_unary<kTanh>, n, a, out, n, p, vec); break;
    case kExp: LAUNCH(k_unary<kExp>, n, a, out, n, p, vec); break;
    case kLog: LAUNCH(k_unary<kLog>, n, a, out, n, p, vec); break;
    case kSqrt: LAUNCH(k_unary<kSqrt>, n, a, out, n, p, vec); break;
    case kAbs: LAUNCH(k_unary<kAbs>, n, a, out, n, p, vec); break;
    case kGelu: LAUNCH(k_unary<kGelu>, n, a, out, n, p, vec); break;
    case kRsqrtEps: LAUNCH(k_unary<kRsqrtEps>, n, a, out, n, p, vec); break;
    default: LAUNCH(k_unary<kNeg>, n, a, out, n, p, vec); break;
  }
}

void unary_bwd(int op, const float* x, const float* g, float* out, size_t n) {
  bool vec = aligned16(x) && aligned16(g) && aligned16(out);
  switch (op) {
    case kSigmoidBwd: LAUNCH(k_unary_bwd<kSigmoidBwd>, n, x, g, out, n, vec); break;
    case kReluBwd: LAUNCH(k_unary_bwd<kReluBwd>, n, x, g, out, n, vec); break;
    case kTanhBwd: LAUNCH(k_unary_bwd<kTanhBwd>, n, x, g, out, n, vec); break;
    case kSqrtBwd: LAUNCH(k_unary_bwd<kSqrtBwd>, n, x, g, out, n, vec); break;
    case kAbsBwd: LAUNCH(k_unary_bwd<kAbsBwd>, n, x, g, out, n, vec); break;
    case kGeluBwd: LAUNCH(k_unary_bwd<kGeluBwd>, n, x, g, out, n, vec); break;
    default: LAUNCH(k_unary_bwd<kEq>, n, x, g, out, n, vec); break;
  }
}

void sigmoid_backward_user(const float* g, const float* s, float* out, size_t n) {
  if (!n) return;
  k_sigmoid_backward_user<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(g, s, out, n);
  count_launch();
  after_launch("k_sigmoid_backward_user");
}

void expand_axis(const float* small, float* out, size_t outer, size_t axis_sz, size_t inner) {
  size_t n = outer * axis_sz * inner;
  if (!n) return;
  k_expand_axis<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(small, out, n, axis_sz, inner);
  count_launch();
  after_launch("k_expand_axis");
}

}  // namespace malus
