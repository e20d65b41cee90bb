// ORACLE — test infrastructure only.
//
// A plain C++ CPU restatement of the reference's (wintermute-motherbrain/malus)
// semantics for the nanoGPT training hot path.  It is the checker for the
// CUDA runtime in malus_b200/ and the timed CPU baseline of bench.py; nothing
// in the product links or calls it.  Only tests/, __graft_entry__.smoke() and
// bench.py's CPU leg load liboracle.so.
//
// The reference is Rust + Metal and cannot be built here (no cargo/rustc, no
// Metal), so every function below restates, loop for loop, the host-side
// evaluation the reference keeps as its own ground truth (the `cpu_fallback`
// code of crates/malus-runtime/src/metal.rs and tape.rs), or — where there is
// none — the per-thread math of the stdlib .ml kernels.  Each function cites
// the file:line it follows.  Floating-point order is the reference's
// (sequential, f32, separate multiply and add: build with -ffp-contract=off).
// Pinned against the reference's own golden vectors (crates/malus-runtime/src/
// tests.rs, README.md:66-67) by tests/test_oracle_golden.py.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

static int g_threads = 1;
void or_set_threads(int n) {
  g_threads = n < 1 ? 1 : n;
#ifdef _OPENMP
  omp_set_num_threads(g_threads);
#endif
}
int or_get_threads(void) { return g_threads; }

// ---------------------------------------------------------------- matmul
// metal.rs:699-800 tensor_matmul_cpu: out[i,j] += a[i,k]*b[k,j] for k in
// order.  Loop i-k-j keeps each out[i,j]'s k order, so the result is
// bit-identical to i-j-k.
void or_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N,
               int64_t batch, int64_t sA, int64_t sB) {
  for (int64_t b = 0; b < batch; ++b) {
    const float* a = A + b * sA;
    const float* bb = B + b * sB;
    float* c = C + b * M * N;
#pragma omp parallel for schedule(static) if (g_threads > 1 && M * N * K > 100000)
    for (int64_t i = 0; i < M; ++i) {
      float* ci = c + i * N;
      for (int64_t j = 0; j < N; ++j) ci[j] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        float av = a[i * K + k];
        const float* bk = bb + k * N;
        for (int64_t j = 0; j < N; ++j) ci[j] += av * bk[j];
      }
    }
  }
}

// C = A^T-aware general form used by the GPT backward: op(A)[MxK] op(B)[KxN]
static void mm(const float* A, bool at, const float* B, bool bt, float* C, int64_t M, int64_t K,
               int64_t N, bool accumulate) {
#pragma omp parallel for schedule(static) if (g_threads > 1 && M * N * K > 100000)
  for (int64_t i = 0; i < M; ++i) {
    float* ci = C + i * N;
    std::vector<float> acc(N, 0.0f);
    for (int64_t k = 0; k < K; ++k) {
      float av = at ? A[k * M + i] : A[i * K + k];
      if (bt) {
        for (int64_t j = 0; j < N; ++j) acc[j] += av * B[j * K + k];
      } else {
        const float* bk = B + k * N;
        for (int64_t j = 0; j < N; ++j) acc[j] += av * bk[j];
      }
    }
    for (int64_t j = 0; j < N; ++j) ci[j] = accumulate ? ci[j] + acc[j] : acc[j];
  }
}

// ----------------------------------------------------------- broadcast
// metal.rs:1024-1072 broadcast_result_shape + broadcast_cpu_loop.
static float binop(int op, float x, float y) {
  switch (op) {
    case 0: return x + y;
    case 1: return x - y;
    case 2: return x * y;
    default: return x / y;
  }
}

int or_broadcast_shape(const int64_t* as, int an, const int64_t* bs, int bn, int64_t* out) {
  int n = an > bn ? an : bn;
  for (int i = 0; i < n; ++i) {
    int64_t da = i + an >= n ? as[i + an - n] : 1;
    int64_t db = i + bn >= n ? bs[i + bn - n] : 1;
    if (da == db || db == 1) out[i] = da;
    else if (da == 1) out[i] = db;
    else return -1;
  }
  return n;
}

void or_broadcast(int op, const float* a, const int64_t* as, int an, const float* b,
                  const int64_t* bs, int bn, float* out) {
  int64_t os[8];
  int n = or_broadcast_shape(as, an, bs, bn, os);
  if (n < 0) return;
  int64_t pa[8], pb[8];
  for (int i = 0; i < n; ++i) {
    pa[i] = i + an >= n ? as[i + an - n] : 1;
    pb[i] = i + bn >= n ? bs[i + bn - n] : 1;
  }
  int64_t total = 1;
  for (int i = 0; i < n; ++i) total *= os[i];
  for (int64_t flat = 0; flat < total; ++flat) {
    int64_t rem = flat, idx[8];
    for (int d = n - 1; d >= 0; --d) { idx[d] = rem % os[d]; rem /= os[d]; }
    int64_t fa = 0, fb = 0;
    for (int d = 0; d < n; ++d) {
      fa = fa * pa[d] + idx[d] % pa[d];
      fb = fb * pb[d] + idx[d] % pb[d];
    }
    out[flat] = binop(op, a[fa], b[fb]);
  }
}

// ----------------------------------------------------------- reductions
// metal.rs:1165-1271 (reduce_elements: sequential in flat input order) and
// the stdlib kernels' serial per-group loops (reduce_sum.ml:16-20,
// reduce_var.ml:16-25).  op: 0 sum, 1 mean, 2 max, 3 var (population).
void or_reduce(int op, const float* x, int64_t outer, int64_t axis, int64_t inner, float* out) {
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t i = 0; i < inner; ++i) {
      const float* base = x + o * axis * inner + i;
      float r;
      if (op == 2) {
        r = axis ? base[0] : -INFINITY;
        for (int64_t a = 1; a < axis; ++a) r = fmaxf(r, base[a * inner]);
      } else {
        float s = 0.0f;
        for (int64_t a = 0; a < axis; ++a) s += base[a * inner];
        if (op == 0) r = s;
        else {
          float mean = s / (float)axis;
          if (op == 1) r = mean;
          else {
            float v = 0.0f;
            for (int64_t a = 0; a < axis; ++a) {
              float d = base[a * inner] - mean;
              v += d * d;
            }
            r = v / (float)axis;
          }
        }
      }
      out[o * inner + i] = r;
    }
}

// --------------------------------------------------------------- softmax
// metal.rs:1442-1470 softmax_axis_cpu
void or_softmax(const float* x, int64_t outer, int64_t axis, int64_t inner, float* y) {
#pragma omp parallel for schedule(static) if (g_threads > 1 && outer * axis * inner > 100000)
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t i = 0; i < inner; ++i) {
      const float* b = x + o * axis * inner + i;
      float* yb = y + o * axis * inner + i;
      float m = -INFINITY;
      for (int64_t a = 0; a < axis; ++a) if (b[a * inner] > m) m = b[a * inner];
      float s = 0.0f;
      for (int64_t a = 0; a < axis; ++a) {
        float e = expf(b[a * inner] - m);
        yb[a * inner] = e;
        s += e;
      }
      for (int64_t a = 0; a < axis; ++a) yb[a * inner] /= s;
    }
}

// tape.rs softmax_bwd (cpu_fallback): dx = s * (dout - sum(dout*s, axis))
void or_softmax_bwd(const float* s, const float* g, int64_t outer, int64_t axis, int64_t inner,
                    float* dx) {
#pragma omp parallel for schedule(static) if (g_threads > 1 && outer * axis * inner > 100000)
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t i = 0; i < inner; ++i) {
      int64_t base = o * axis * inner + i;
      float dot = 0.0f;
      for (int64_t a = 0; a < axis; ++a) dot += g[base + a * inner] * s[base + a * inner];
      for (int64_t a = 0; a < axis; ++a) {
        int64_t k = base + a * inner;
        dx[k] = s[k] * (g[k] - dot);
      }
    }
}

// ------------------------------------------------------------- layernorm
// metal.rs:1487-1533 tensor_layernorm_axis (var keepdim at the axis)
void or_layernorm(const float* x, int64_t outer, int64_t axis, int64_t inner, float eps, float* y,
                  float* var) {
#pragma omp parallel for schedule(static) if (g_threads > 1 && outer * axis * inner > 100000)
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t i = 0; i < inner; ++i) {
      int64_t base = o * axis * inner + i;
      float mu = 0.0f;
      for (int64_t a = 0; a < axis; ++a) mu += x[base + a * inner];
      mu /= (float)axis;
      float va = 0.0f;
      for (int64_t a = 0; a < axis; ++a) {
        float d = x[base + a * inner] - mu;
        va += d * d;
      }
      va /= (float)axis;
      float sigma = sqrtf(va + eps);
      if (var) var[o * inner + i] = va;
      for (int64_t a = 0; a < axis; ++a) y[base + a * inner] = (x[base + a * inner] - mu) / sigma;
    }
}

// tape.rs:1162-1186 layernorm_bwd (cpu_fallback):
//   inv = 1/sqrt(var+eps); dx = ((dout - mean(dout)) - y*mean(dout*y)) * inv
void or_layernorm_bwd(const float* y, const float* var, const float* g, int64_t outer,
                      int64_t axis, int64_t inner, float eps, float* dx) {
#pragma omp parallel for schedule(static) if (g_threads > 1 && outer * axis * inner > 100000)
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t i = 0; i < inner; ++i) {
      int64_t base = o * axis * inner + i;
      float inv = 1.0f / sqrtf(var[o * inner + i] + eps);
      float sg = 0.0f, sgy = 0.0f;
      for (int64_t a = 0; a < axis; ++a) sg += g[base + a * inner];
      for (int64_t a = 0; a < axis; ++a) sgy += g[base + a * inner] * y[base + a * inner];
      float mg = sg / (float)axis, mgy = sgy / (float)axis;
      for (int64_t a = 0; a < axis; ++a) {
        int64_t k = base + a * inner;
        dx[k] = ((g[k] - mg) - y[k] * mgy) * inv;
      }
    }
}

// ----------------------------------------------------------------- unary
// codegen-gpu lib.rs:373-390; gelu.ml:5-10 (c0 = 0.7978845608028654)
static const float kC0 = 0.7978845608028654f, kC1 = 0.044715f;
static float gelu1(float x) {
  float x3 = x * x * x;
  float inner = kC0 * (x + kC1 * x3);
  return 0.5f * x * (1.0f + tanhf(inner));
}
// op: 0 relu 1 sigmoid 2 tanh 3 exp 4 log 5 sqrt 6 abs 7 gelu 8 rsqrt_eps 9 neg
void or_unary(int op, const float* x, float* y, int64_t n, float p) {
  for (int64_t i = 0; i < n; ++i) {
    float v = x[i];
    switch (op) {
      case 0: y[i] = fmaxf(0.0f, v); break;
      case 1: y[i] = 1.0f / (1.0f + expf(-v)); break;
      case 2: y[i] = tanhf(v); break;
      case 3: y[i] = expf(v); break;
      case 4: y[i] = logf(v); break;
      case 5: y[i] = sqrtf(v); break;
      case 6: y[i] = fabsf(v); break;
      case 7: y[i] = gelu1(v); break;
      case 8: y[i] = 1.0f / sqrtf(v + p); break;
      default: y[i] = -v; break;
    }
  }
}
// unary_bwd.ml:6-91, transformer_bwd.ml:40-48
// op: 0 sigmoid(s) 1 relu(x) 2 tanh(t) 3 sqrt(s) 4 abs(x) 5 gelu(x) 6 eq(a,b)
void or_unary_bwd(int op, const float* x, const float* g, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float v = x[i], d = g[i];
    switch (op) {
      case 0: y[i] = d * v * (1.0f - v); break;
      case 1: y[i] = v > 0.0f ? d : 0.0f; break;
      case 2: y[i] = d * (1.0f - v * v); break;
      case 3: y[i] = d / (2.0f * v); break;
      case 4: y[i] = v > 0.0f ? d : (v < 0.0f ? -d : 0.0f); break;
      case 5: {
        float x3 = v * v * v;
        float gg = kC0 * (v + kC1 * x3);
        float t = tanhf(gg);
        float gp = kC0 * (1.0f + 3.0f * kC1 * v * v);
        float deriv = 0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * gp;
        y[i] = d * deriv;
        break;
      }
      default: y[i] = v == d ? 1.0f : 0.0f; break;
    }
  }
}

// --------------------------------------------------------- cross-entropy
// metal.rs:1555-1598 tensor_cross_entropy; tape.rs:1200-1215 bwd:
// (p - onehot) * dout[0] / N
void or_xent(const float* logits, const int32_t* t, int64_t n, int64_t v, float* probs,
             float* loss) {
  or_softmax(logits, n, v, 1, probs);
  float l = 0.0f;
  for (int64_t i = 0; i < n; ++i) l -= logf(probs[i * v + t[i]]);
  *loss = l / (float)n;
}
void or_xent_bwd(const float* probs, const int32_t* t, float dout0, int64_t n, int64_t v,
                 float* dx) {
  float scale = dout0 / (float)n;
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < v; ++j) {
      float g = probs[i * v + j];
      if (j == t[i]) g = g - 1.0f;
      dx[i * v + j] = g * scale;
    }
}

// -------------------------------------------------------------- embedding
// metal.rs:1629-1688 tensor_embedding / tensor_scatter_add (token order)
void or_embedding(const float* w, const int32_t* idx, int64_t n, int64_t V, int64_t D, float* out) {
  for (int64_t t = 0; t < n; ++t) memcpy(out + t * D, w + (int64_t)idx[t] * D, D * 4);
  (void)V;
}
void or_embedding_bwd(const float* dout, const int32_t* idx, int64_t n, int64_t V, int64_t D,
                      float* dw) {
  memset(dw, 0, V * D * 4);
  for (int64_t t = 0; t < n; ++t) {
    float* row = dw + (int64_t)idx[t] * D;
    for (int64_t d = 0; d < D; ++d) row[d] += dout[t * D + d];
  }
}

// --------------------------------------------------------------- permute
// metal.rs:1347-1383 permute_by_perm
void or_permute(const float* x, const int64_t* shape, int nd, const int* perm, float* out) {
  int64_t st[8], os[8];
  st[nd - 1] = 1;
  for (int d = nd - 2; d >= 0; --d) st[d] = st[d + 1] * shape[d + 1];
  int64_t total = 1;
  for (int d = 0; d < nd; ++d) { os[d] = shape[perm[d]]; total *= os[d]; }
  for (int64_t f = 0; f < total; ++f) {
    int64_t rem = f, src = 0;
    for (int d = nd - 1; d >= 0; --d) {
      int64_t i = rem % os[d];
      rem /= os[d];
      src += i * st[perm[d]];
    }
    out[f] = x[src];
  }
}

// ------------------------------------------------------------------- RNG
// metal.rs:1692-1759: Philox4x32-10 (Salmon et al., SC'11) keyed by a per-call
// counter; randn = Box-Muller in f64; rand_int = r[0] % n with ctr [1,0,0,0];
// rand_uniform = r[0] / 2^32 with ctr [0,0,0,0].
static void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)c[0] * 0xD2511F53u, p1 = (uint64_t)c[2] * 0xCD9E8D57u;
    uint32_t h0 = (uint32_t)(p0 >> 32), l0 = (uint32_t)p0, h1 = (uint32_t)(p1 >> 32), l1 = (uint32_t)p1;
    uint32_t n0 = h1 ^ c[1] ^ k0, n2 = h0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = l1; c[2] = n2; c[3] = l0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}
void or_philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) { philox(c, k0, k1); }
void or_randn(float* out, int64_t n, uint64_t call_idx) {
  uint32_t k0 = (uint32_t)call_idx, k1 = (uint32_t)(call_idx >> 32);
  for (int64_t k = 0; k < (n + 1) / 2; ++k) {
    uint32_t c[4] = {(uint32_t)k, (uint32_t)((uint64_t)k >> 32), 0, 0};
    philox(c, k0, k1);
    double u1 = ((double)c[0] + 0.5) / 4294967296.0, u2 = ((double)c[1] + 0.5) / 4294967296.0;
    double mag = sqrt(-2.0 * log(u1));
    out[2 * k] = (float)(mag * cos(2.0 * M_PI * u2));
    if (2 * k + 1 < n) out[2 * k + 1] = (float)(mag * sin(2.0 * M_PI * u2));
  }
}
int64_t or_rand_int(int64_t n, uint64_t call_idx) {
  uint32_t c[4] = {1, 0, 0, 0};
  philox(c, (uint32_t)call_idx, (uint32_t)(call_idx >> 32));
  return (int64_t)((uint64_t)c[0] % (uint64_t)n);
}
float or_rand_uniform(uint64_t call_idx) {
  uint32_t c[4] = {0, 0, 0, 0};
  philox(c, (uint32_t)call_idx, (uint32_t)(call_idx >> 32));
  return (float)((double)c[0] / 4294967296.0);
}

// ----------------------------------------------------------------- AdamW
// examples/nanogpt.ml:80-91 composed elementwise, f32, left to right
void or_adamw(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
              float b2, float eps, float wd, int64_t step, float gscale) {
  float bc1 = 1.0f - powf(b1, (float)step), bc2 = 1.0f - powf(b2, (float)step);
  float c1 = 1.0f - b1, c2 = 1.0f - b2;
  for (int64_t i = 0; i < n; ++i) {
    float gi = g ? g[i] : 0.0f;
    if (gscale != 1.0f) gi = gi * gscale;
    float gg = gi + wd * p[i];
    m[i] = b1 * m[i] + c1 * gg;
    v[i] = b2 * v[i] + (c2 * gg) * gg;
    float mh = m[i] / bc1, vh = v[i] / bc2;
    p[i] = p[i] - (lr * mh) / (sqrtf(vh) + eps);
  }
}

// ------------------------------------------------------------------- XOR
// examples/xor.ml: 2->8->1 MLP, sigmoid, hand-written backward, SGD lr=1.5.
void or_xor_train(int steps, float lr, float* loss_out, float* preds_out) {
  float x[8] = {0, 0, 0, 1, 1, 0, 1, 1}, tgt[4] = {0, 1, 1, 0}, ones[4] = {1, 1, 1, 1};
  float w1[16] = {0.5f, -0.6f, 0.7f, -0.4f, 0.3f, -0.5f, 0.6f, -0.3f,
                  -0.4f, 0.5f, -0.6f, 0.7f, -0.3f, 0.4f, -0.5f, 0.6f};
  float b1[8] = {0.1f, -0.1f, 0.1f, -0.1f, 0.1f, -0.1f, 0.1f, -0.1f};
  float w2[8] = {0.6f, -0.5f, 0.4f, -0.6f, 0.5f, -0.4f, 0.6f, -0.5f};
  float b2[1] = {0.0f};
  float loss = 0.0f, out[4];
  for (int step = 0; step < steps; ++step) {
    float z1a[32], z1b[32], z1[32], h[32], z2a[4], z2b[4], z2[4];
    or_matmul(x, w1, z1a, 4, 2, 8, 1, 0, 0);
    or_matmul(ones, b1, z1b, 4, 1, 8, 1, 0, 0);
    for (int i = 0; i < 32; ++i) z1[i] = z1a[i] + z1b[i];
    or_unary(1, z1, h, 32, 0);
    or_matmul(h, w2, z2a, 4, 8, 1, 1, 0, 0);
    or_matmul(ones, b2, z2b, 4, 1, 1, 1, 0, 0);
    for (int i = 0; i < 4; ++i) z2[i] = z2a[i] + z2b[i];
    or_unary(1, z2, out, 4, 0);
    float diff[4], sq[4];
    for (int i = 0; i < 4; ++i) { diff[i] = out[i] - tgt[i]; sq[i] = diff[i] * diff[i]; }
    loss = 0.0f;
    for (int i = 0; i < 4; ++i) loss += sq[i];
    float dout[4], dz2[4];
    for (int i = 0; i < 4; ++i) dout[i] = diff[i] * 2.0f;
    for (int i = 0; i < 4; ++i) dz2[i] = dout[i] * out[i] * (1.0f - out[i]);
    float hT[32], dw2[8], db2[1], w2T[8], dh[32], dz1[32], xT[8], dw1[16], db1[8];
    for (int i = 0; i < 4; ++i) for (int j = 0; j < 8; ++j) hT[j * 4 + i] = h[i * 8 + j];
    or_matmul(hT, dz2, dw2, 8, 4, 1, 1, 0, 0);
    or_matmul(ones, dz2, db2, 1, 4, 1, 1, 0, 0);
    for (int j = 0; j < 8; ++j) w2T[j] = w2[j];
    or_matmul(dz2, w2T, dh, 4, 1, 8, 1, 0, 0);
    for (int i = 0; i < 32; ++i) dz1[i] = dh[i] * h[i] * (1.0f - h[i]);
    for (int i = 0; i < 4; ++i) for (int j = 0; j < 2; ++j) xT[j * 4 + i] = x[i * 2 + j];
    or_matmul(xT, dz1, dw1, 2, 4, 8, 1, 0, 0);
    or_matmul(ones, dz1, db1, 1, 4, 8, 1, 0, 0);
    for (int i = 0; i < 16; ++i) w1[i] = w1[i] - dw1[i] * lr;
    for (int i = 0; i < 8; ++i) b1[i] = b1[i] - db1[i] * lr;
    for (int i = 0; i < 8; ++i) w2[i] = w2[i] - dw2[i] * lr;
    b2[0] = b2[0] - db2[0] * lr;
  }
  *loss_out = loss;
  for (int i = 0; i < 4; ++i) preds_out[i] = out[i];
}

// ------------------------------------------------------------- nanoGPT
// The training step of examples/nanogpt_modular.ml generalised to n_layer /
// n_head (scale 1/sqrt(head_size)); forward ops follow the call sequence the
// JIT emits, and the backward pass applies the tape's VJP rules
// (tape.rs:421-729 with the cpu_fallback VJPs of tape.rs:971-1260) to this
// graph in reverse order, summing each tensor's incoming gradients.
struct OrCfg {
  int32_t vocab, n_layer, n_head, n_embd, block_size, batch;
  int32_t tied;
  float lr, beta1, beta2, eps, wd, init_std;
  int32_t mode, use_graph;
  uint64_t seed;
};

struct OrGpt {
  OrCfg c;
  int64_t C, H, hs, T, B, V, L, C4, M;
  std::vector<std::vector<float>> p, m, v, g;
  std::vector<std::vector<int64_t>> shape;
  int64_t step = 0;
};

static void add_param(OrGpt* o, std::vector<int64_t> s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  o->p.emplace_back(n, 0.0f);
  o->m.emplace_back(n, 0.0f);
  o->v.emplace_back(n, 0.0f);
  o->g.emplace_back(n, 0.0f);
  o->shape.push_back(s);
}

int64_t or_gpt_create(const OrCfg* cfg) {
  auto* o = new OrGpt();
  o->c = *cfg;
  o->C = cfg->n_embd; o->H = cfg->n_head; o->hs = o->C / o->H; o->T = cfg->block_size;
  o->B = cfg->batch; o->V = cfg->vocab; o->L = cfg->n_layer; o->C4 = 4 * o->C; o->M = o->B * o->T;
  int64_t C = o->C, C4 = o->C4, V = o->V, T = o->T;
  for (int l = 0; l < o->L; ++l) {
    add_param(o, {C});
    for (int j = 0; j < 4; ++j) add_param(o, {C, C});
    add_param(o, {C});
    add_param(o, {C, C4});
    add_param(o, {C4, C});
  }
  add_param(o, {V, C});
  add_param(o, {T, C});
  add_param(o, {C});
  if (!cfg->tied) add_param(o, {C, V});
  uint64_t call = cfg->seed;
  auto randn = [&](int64_t i) {
    or_randn(o->p[i].data(), (int64_t)o->p[i].size(), call++);
    for (auto& x : o->p[i]) x = x * cfg->init_std;
  };
  auto ones = [&](int64_t i) { for (auto& x : o->p[i]) x = 1.0f; };
  for (int l = 0; l < o->L; ++l) {
    int64_t b = l * 8;
    ones(b);
    for (int j = 1; j <= 4; ++j) randn(b + j);
    ones(b + 5);
    randn(b + 6);
    randn(b + 7);
  }
  int64_t top = o->L * 8;
  randn(top);
  randn(top + 1);
  ones(top + 2);
  if (!cfg->tied) randn(top + 3);
  return (int64_t)o;
}

void or_gpt_destroy(int64_t h) { delete (OrGpt*)h; }
int32_t or_gpt_num_params(int64_t h) { return (int32_t)((OrGpt*)h)->p.size(); }
int64_t or_gpt_param_size(int64_t h, int32_t i) { return (int64_t)((OrGpt*)h)->p[i].size(); }
void or_gpt_get_param(int64_t h, int32_t i, float* out) {
  auto& v = ((OrGpt*)h)->p[i];
  memcpy(out, v.data(), v.size() * 4);
}
void or_gpt_set_param(int64_t h, int32_t i, const float* in) {
  auto& v = ((OrGpt*)h)->p[i];
  memcpy(v.data(), in, v.size() * 4);
}
void or_gpt_get_grad(int64_t h, int32_t i, float* out) {
  auto& v = ((OrGpt*)h)->g[i];
  memcpy(out, v.data(), v.size() * 4);
}

using Vec = std::vector<float>;

static void gain_mul(const Vec& y, const Vec& w, Vec& out, int64_t M, int64_t C) {
  out.resize(M * C);
  for (int64_t r = 0; r < M; ++r)
    for (int64_t c = 0; c < C; ++c) out[r * C + c] = y[r * C + c] * w[c];
}
// head fold [B*T, C] -> [B*H, T, hs] (reshape, permute(0,2,1,3), reshape)
static void fold(const Vec& x, Vec& out, int64_t B, int64_t T, int64_t H, int64_t hs) {
  out.resize(B * T * H * hs);
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t h = 0; h < H; ++h)
        memcpy(&out[((b * H + h) * T + t) * hs], &x[(b * T + t) * H * hs + h * hs], hs * 4);
}
static void unfold(const Vec& x, Vec& out, int64_t B, int64_t T, int64_t H, int64_t hs) {
  out.resize(B * T * H * hs);
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t h = 0; h < H; ++h)
        memcpy(&out[(b * T + t) * H * hs + h * hs], &x[((b * H + h) * T + t) * hs], hs * 4);
}

struct BlockAct {
  Vec x, y1, var1, xn1, q, k, v, Q, K, Vh, qk, attn, av, ao, x2, y2, var2, xn2, hpre, hid;
};

// forward; returns loss; keeps activations for backward
float or_gpt_step(int64_t h, const int32_t* xt, const int32_t* yt) {
  OrGpt* o = (OrGpt*)h;
  const int64_t C = o->C, H = o->H, hs = o->hs, T = o->T, B = o->B, V = o->V, L = o->L,
                C4 = o->C4, M = o->M, BH = B * H;
  const float scale = 1.0f / sqrtf((float)hs);
  auto P = [&](int64_t i) -> Vec& { return o->p[i]; };
  int64_t top = L * 8;
  std::vector<int32_t> pos(M);
  for (int64_t i = 0; i < M; ++i) pos[i] = (int32_t)(i % T);
  Vec te(M * C), pe(M * C), x(M * C);
  or_embedding(P(top).data(), xt, M, V, C, te.data());
  or_embedding(P(top + 1).data(), pos.data(), M, T, C, pe.data());
  for (int64_t i = 0; i < M * C; ++i) x[i] = te[i] + pe[i];
  std::vector<BlockAct> acts(L);
  for (int64_t l = 0; l < L; ++l) {
    BlockAct& a = acts[l];
    int64_t b = l * 8;
    a.x = x;
    a.y1.resize(M * C); a.var1.resize(M);
    or_layernorm(a.x.data(), M, C, 1, 1e-5f, a.y1.data(), a.var1.data());
    gain_mul(a.y1, P(b), a.xn1, M, C);
    a.q.resize(M * C); a.k.resize(M * C); a.v.resize(M * C);
    mm(a.xn1.data(), false, P(b + 1).data(), false, a.q.data(), M, C, C, false);
    mm(a.xn1.data(), false, P(b + 2).data(), false, a.k.data(), M, C, C, false);
    mm(a.xn1.data(), false, P(b + 3).data(), false, a.v.data(), M, C, C, false);
    fold(a.q, a.Q, B, T, H, hs);
    fold(a.k, a.K, B, T, H, hs);
    fold(a.v, a.Vh, B, T, H, hs);
    a.qk.resize(BH * T * T);
    for (int64_t z = 0; z < BH; ++z)  // Q @ Kt
      mm(&a.Q[z * T * hs], false, &a.K[z * T * hs], true, &a.qk[z * T * T], T, hs, T, false);
    Vec masked(BH * T * T);
    for (int64_t z = 0; z < BH; ++z)
      for (int64_t i = 0; i < T; ++i)
        for (int64_t j = 0; j < T; ++j) {
          int64_t k = (z * T + i) * T + j;
          float s = a.qk[k] * scale;
          masked[k] = s + (j > i ? -1e9f : 0.0f);
        }
    a.attn.resize(BH * T * T);
    or_softmax(masked.data(), BH * T, T, 1, a.attn.data());
    a.av.resize(BH * T * hs);
    for (int64_t z = 0; z < BH; ++z)
      mm(&a.attn[z * T * T], false, &a.Vh[z * T * hs], false, &a.av[z * T * hs], T, T, hs, false);
    unfold(a.av, a.ao, B, T, H, hs);
    Vec proj(M * C);
    mm(a.ao.data(), false, P(b + 4).data(), false, proj.data(), M, C, C, false);
    a.x2.resize(M * C);
    for (int64_t i = 0; i < M * C; ++i) a.x2[i] = a.x[i] + proj[i];
    a.y2.resize(M * C); a.var2.resize(M);
    or_layernorm(a.x2.data(), M, C, 1, 1e-5f, a.y2.data(), a.var2.data());
    gain_mul(a.y2, P(b + 5), a.xn2, M, C);
    a.hpre.resize(M * C4); a.hid.resize(M * C4);
    mm(a.xn2.data(), false, P(b + 6).data(), false, a.hpre.data(), M, C, C4, false);
    or_unary(7, a.hpre.data(), a.hid.data(), M * C4, 0);
    Vec mlp(M * C);
    mm(a.hid.data(), false, P(b + 7).data(), false, mlp.data(), M, C4, C, false);
    for (int64_t i = 0; i < M * C; ++i) x[i] = a.x2[i] + mlp[i];
  }
  Vec yf(M * C), varf(M), xf;
  or_layernorm(x.data(), M, C, 1, 1e-5f, yf.data(), varf.data());
  gain_mul(yf, P(top + 2), xf, M, C);
  Vec logits(M * V), probs(M * V);
  if (o->c.tied) mm(xf.data(), false, P(top).data(), true, logits.data(), M, C, V, false);
  else mm(xf.data(), false, P(top + 3).data(), false, logits.data(), M, C, V, false);
  float loss;
  or_xent(logits.data(), yt, M, V, probs.data(), &loss);

  // ---------------- backward ----------------
  for (auto& gg : o->g) std::fill(gg.begin(), gg.end(), 0.0f);
  Vec dlogits(M * V);
  or_xent_bwd(probs.data(), yt, 1.0f, M, V, dlogits.data());
  Vec dxf(M * C);
  if (o->c.tied) {
    mm(dlogits.data(), false, P(top).data(), false, dxf.data(), M, V, C, false);      // dC @ (wte^T)^T
    Vec dwT(C * V);                                                                   // xf^T @ dC -> [C,V]
    mm(xf.data(), true, dlogits.data(), false, dwT.data(), C, M, V, false);
    for (int64_t vv = 0; vv < V; ++vv)
      for (int64_t c = 0; c < C; ++c) o->g[top][vv * C + c] += dwT[c * V + vv];
  } else {
    mm(dlogits.data(), false, P(top + 3).data(), true, dxf.data(), M, V, C, false);
    mm(xf.data(), true, dlogits.data(), false, o->g[top + 3].data(), C, M, V, false);
  }
  // xf = yf * lnf
  Vec dyf(M * C);
  for (int64_t r = 0; r < M; ++r)
    for (int64_t c = 0; c < C; ++c) {
      dyf[r * C + c] = dxf[r * C + c] * P(top + 2)[c];
      o->g[top + 2][c] += dxf[r * C + c] * yf[r * C + c];
    }
  Vec dx(M * C);
  or_layernorm_bwd(yf.data(), varf.data(), dyf.data(), M, C, 1, 1e-5f, dx.data());
  for (int64_t l = L - 1; l >= 0; --l) {
    BlockAct& a = acts[l];
    int64_t b = l * 8;
    // x3 = x2 + mlp
    Vec& dx2 = dx;  // gradient of x2 (accumulates both paths below)
    Vec dmlp = dx;
    Vec dhid(M * C4);
    mm(dmlp.data(), false, P(b + 7).data(), true, dhid.data(), M, C, C4, false);
    mm(a.hid.data(), true, dmlp.data(), false, o->g[b + 7].data(), C4, M, C, true);
    Vec dhpre(M * C4);
    or_unary_bwd(5, a.hpre.data(), dhid.data(), dhpre.data(), M * C4);
    Vec dxn2(M * C);
    mm(dhpre.data(), false, P(b + 6).data(), true, dxn2.data(), M, C4, C, false);
    mm(a.xn2.data(), true, dhpre.data(), false, o->g[b + 6].data(), C, M, C4, true);
    Vec dy2(M * C);
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = 0; c < C; ++c) {
        dy2[r * C + c] = dxn2[r * C + c] * P(b + 5)[c];
        o->g[b + 5][c] += dxn2[r * C + c] * a.y2[r * C + c];
      }
    Vec dln2(M * C);
    or_layernorm_bwd(a.y2.data(), a.var2.data(), dy2.data(), M, C, 1, 1e-5f, dln2.data());
    Vec dx2t(M * C);
    for (int64_t i = 0; i < M * C; ++i) dx2t[i] = dx2[i] + dln2[i];
    // x2 = x + proj
    Vec dao(M * C);
    mm(dx2t.data(), false, P(b + 4).data(), true, dao.data(), M, C, C, false);
    mm(a.ao.data(), true, dx2t.data(), false, o->g[b + 4].data(), C, M, C, true);
    Vec dav;
    fold(dao, dav, B, T, H, hs);  // inverse of the unfold permute
    Vec dattn(BH * T * T), dVh(BH * T * hs);
    for (int64_t z = 0; z < BH; ++z) {
      mm(&dav[z * T * hs], false, &a.Vh[z * T * hs], true, &dattn[z * T * T], T, hs, T, false);
      mm(&a.attn[z * T * T], true, &dav[z * T * hs], false, &dVh[z * T * hs], T, T, hs, false);
    }
    Vec dmasked(BH * T * T);
    or_softmax_bwd(a.attn.data(), dattn.data(), BH * T, T, 1, dmasked.data());
    Vec dqk(BH * T * T);
    for (int64_t i = 0; i < BH * T * T; ++i) dqk[i] = dmasked[i] * scale;
    Vec dQ(BH * T * hs), dK(BH * T * hs);
    for (int64_t z = 0; z < BH; ++z) {
      mm(&dqk[z * T * T], false, &a.K[z * T * hs], false, &dQ[z * T * hs], T, T, hs, false);
      mm(&dqk[z * T * T], true, &a.Q[z * T * hs], false, &dK[z * T * hs], T, T, hs, false);
    }
    Vec dq, dk, dv;
    unfold(dQ, dq, B, T, H, hs);
    unfold(dK, dk, B, T, H, hs);
    unfold(dVh, dv, B, T, H, hs);
    Vec dxn1(M * C, 0.0f), tmp(M * C);
    const Vec* dqkv[3] = {&dq, &dk, &dv};
    for (int j = 2; j >= 0; --j) {  // reverse walk order: V, K, Q consumers of xn1
      mm(dqkv[j]->data(), false, P(b + 1 + j).data(), true, tmp.data(), M, C, C, false);
      for (int64_t i = 0; i < M * C; ++i) dxn1[i] = j == 2 ? tmp[i] : dxn1[i] + tmp[i];
      mm(a.xn1.data(), true, dqkv[j]->data(), false, o->g[b + 1 + j].data(), C, M, C, true);
    }
    Vec dy1(M * C);
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = 0; c < C; ++c) {
        dy1[r * C + c] = dxn1[r * C + c] * P(b)[c];
        o->g[b][c] += dxn1[r * C + c] * a.y1[r * C + c];
      }
    Vec dln1(M * C);
    or_layernorm_bwd(a.y1.data(), a.var1.data(), dy1.data(), M, C, 1, 1e-5f, dln1.data());
    for (int64_t i = 0; i < M * C; ++i) dx[i] = dx2t[i] + dln1[i];
  }
  // x = te + pe
  Vec dwte(V * C), dwpe(T * C);
  or_embedding_bwd(dx.data(), xt, M, V, C, dwte.data());
  or_embedding_bwd(dx.data(), pos.data(), M, T, C, dwpe.data());
  for (int64_t i = 0; i < V * C; ++i) o->g[top][i] += dwte[i];
  for (int64_t i = 0; i < T * C; ++i) o->g[top + 1][i] += dwpe[i];

  // ---------------- AdamW ----------------
  o->step++;
  for (size_t i = 0; i < o->p.size(); ++i)
    or_adamw(o->p[i].data(), o->g[i].data(), o->m[i].data(), o->v[i].data(), (int64_t)o->p[i].size(),
             o->c.lr, o->c.beta1, o->c.beta2, o->c.eps, o->c.wd, o->step, 1.0f);
  return loss;
}

}  // extern "C"
