// Fused multi-tensor AdamW: one launch updates every parameter.
//
// The reference composes the update from ~14 elementwise launches per
// parameter (examples/nanogpt.ml:80-91):
//   g  = grad + wd * p                      (L2-coupled weight decay)
//   m  = beta1 * m + (1 - beta1) * g
//   v  = beta2 * v + (1 - beta2) * g * g    (left to right: ((1-b2)*g)*g)
//   p' = p - lr * (m / bc1) / (sqrt(v / bc2) + eps)
// with bc = 1 - beta**t computed on the host in f32.  This kernel performs the
// same f32 operations in the same order with explicit round-to-nearest
// intrinsics (no FMA contraction), so its result is bit-identical to the
// composed sequence.  The data-parallel 1/world average is one more multiply
// applied to the raw gradient first (exact when world is a power of two).
#include "common.cuh"

#include <vector>

namespace malus {
namespace {

struct SegTable {
  AdamSeg seg[64];
  int64_t start[65];  // prefix of float4-chunk counts
};

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, float lr, float b1,
                                         float b2, float eps, float wd, float c1, float c2,
                                         float bc1, float bc2, float gs) {
  if (gs != 1.0f) g = __fmul_rn(g, gs);
  float gg = __fadd_rn(g, __fmul_rn(wd, p));
  m = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(c1, gg));
  v = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(c2, gg), gg));
  float mh = __fdiv_rn(m, bc1);
  float vh = __fdiv_rn(v, bc2);
  float upd = __fdiv_rn(__fmul_rn(lr, mh), __fadd_rn(__fsqrt_rn(vh), eps));
  p = __fsub_rn(p, upd);
}

// bc_tab (optional): host-computed bias corrections per step, [2*(t-1)] = 1 - b1**t,
// [2*(t-1)+1] = 1 - b2**t, indexed by the device step counter *step_dev, so a
// captured CUDA graph replays with the current step's values.
__global__ void k_adamw(SegTable t, int nseg, int64_t total4, float lr, float b1, float b2,
                        float eps, float wd, float c1, float c2, float bc1, float bc2, float gs,
                        const float* __restrict__ bc_tab, const int64_t* __restrict__ step_dev) {
  if (bc_tab) {
    const int64_t st = *step_dev;
    bc1 = bc_tab[2 * (st - 1)];
    bc2 = bc_tab[2 * (st - 1) + 1];
  }
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  int s = 0;
  for (int64_t q = tid; q < total4; q += step) {
    while (s + 1 < nseg && q >= t.start[s + 1]) ++s;
    while (s > 0 && q < t.start[s]) --s;
    const AdamSeg& sg = t.seg[s];
    int64_t e0 = (q - t.start[s]) * 4;
    const bool aligned = (((uintptr_t)sg.p | (uintptr_t)sg.m | (uintptr_t)sg.v | (uintptr_t)sg.g) & 15) == 0;
    const bool vec = e0 + 4 <= sg.n && aligned;
    // this thread's next chunk in the same segment: both chunks' loads are
    // issued before either is computed (the same per-element arithmetic)
    const int64_t q2 = q + step, e2 = e0 + 4 * step;
    if (vec && q2 < total4 && (s + 1 >= nseg || q2 < t.start[s + 1]) && e2 + 4 <= sg.n) {
      float4 pp = *reinterpret_cast<const float4*>(sg.p + e0), p2 = *reinterpret_cast<const float4*>(sg.p + e2);
      float4 mm = *reinterpret_cast<const float4*>(sg.m + e0), m2 = *reinterpret_cast<const float4*>(sg.m + e2);
      float4 vv = *reinterpret_cast<const float4*>(sg.v + e0), v2 = *reinterpret_cast<const float4*>(sg.v + e2);
      const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 gg = sg.g ? *reinterpret_cast<const float4*>(sg.g + e0) : z4;
      const float4 g2 = sg.g ? *reinterpret_cast<const float4*>(sg.g + e2) : z4;
      adam_one(pp.x, gg.x, mm.x, vv.x, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.y, gg.y, mm.y, vv.y, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.z, gg.z, mm.z, vv.z, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.w, gg.w, mm.w, vv.w, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(p2.x, g2.x, m2.x, v2.x, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(p2.y, g2.y, m2.y, v2.y, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(p2.z, g2.z, m2.z, v2.z, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(p2.w, g2.w, m2.w, v2.w, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      *reinterpret_cast<float4*>(sg.p + e0) = pp;
      *reinterpret_cast<float4*>(sg.m + e0) = mm;
      *reinterpret_cast<float4*>(sg.v + e0) = vv;
      *reinterpret_cast<float4*>(sg.p + e2) = p2;
      *reinterpret_cast<float4*>(sg.m + e2) = m2;
      *reinterpret_cast<float4*>(sg.v + e2) = v2;
      q = q2;   // the loop's increment then moves past both
      continue;
    }
    if (vec) {   // one 16-byte access per array (same per-element arithmetic)
      float4 pp = *reinterpret_cast<const float4*>(sg.p + e0);
      float4 mm = *reinterpret_cast<const float4*>(sg.m + e0);
      float4 vv = *reinterpret_cast<const float4*>(sg.v + e0);
      const float4 gg = sg.g ? *reinterpret_cast<const float4*>(sg.g + e0) : make_float4(0.f, 0.f, 0.f, 0.f);
      adam_one(pp.x, gg.x, mm.x, vv.x, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.y, gg.y, mm.y, vv.y, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.z, gg.z, mm.z, vv.z, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      adam_one(pp.w, gg.w, mm.w, vv.w, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      *reinterpret_cast<float4*>(sg.p + e0) = pp;
      *reinterpret_cast<float4*>(sg.m + e0) = mm;
      *reinterpret_cast<float4*>(sg.v + e0) = vv;
      continue;
    }
    for (int u = 0; u < 4; ++u) {
      int64_t e = e0 + u;
      if (e >= sg.n) break;
      float p = sg.p[e], m = sg.m[e], v = sg.v[e];
      float g = sg.g ? sg.g[e] : 0.0f;
      adam_one(p, g, m, v, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
      sg.p[e] = p;
      sg.m[e] = m;
      sg.v[e] = v;
    }
  }
}

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// One flat buffer (n a multiple of 4, 16-byte aligned): float4 loads and
// stores; optionally also the tf32 hi/lo planes of the updated parameters (the
// GEMM operands of the next step), so no separate split pass is needed.
__global__ void k_adamw_flat(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, int64_t n4, float lr,
                             float b1, float b2, float eps, float wd, float c1, float c2, float gs,
                             const float* __restrict__ bc_tab, const int64_t* __restrict__ step_dev,
                             float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t st = *step_dev;
  const float bc1 = bc_tab[2 * (st - 1)], bc2 = bc_tab[2 * (st - 1) + 1];
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n4;
       q += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[q];
    const float4 gg = reinterpret_cast<const float4*>(g)[q];
    float4 mm = reinterpret_cast<float4*>(m)[q];
    float4 vv = reinterpret_cast<float4*>(v)[q];
    adam_one(pp.x, gg.x, mm.x, vv.x, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
    adam_one(pp.y, gg.y, mm.y, vv.y, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
    adam_one(pp.z, gg.z, mm.z, vv.z, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
    adam_one(pp.w, gg.w, mm.w, vv.w, lr, b1, b2, eps, wd, c1, c2, bc1, bc2, gs);
    reinterpret_cast<float4*>(p)[q] = pp;
    reinterpret_cast<float4*>(m)[q] = mm;
    reinterpret_cast<float4*>(v)[q] = vv;
    if (hi) {
      const float4 h = make_float4(tf32_rn(pp.x), tf32_rn(pp.y), tf32_rn(pp.z), tf32_rn(pp.w));
      reinterpret_cast<float4*>(hi)[q] = h;
      reinterpret_cast<float4*>(lo)[q] = make_float4(tf32_rn(pp.x - h.x), tf32_rn(pp.y - h.y),
                                                     tf32_rn(pp.z - h.z), tf32_rn(pp.w - h.w));
    }
  }
}

}  // namespace

void adamw_flat(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
                float b2, float eps, float wd, float grad_scale, const float* bc_tab,
                const int64_t* step_dev, float* hi, float* lo) {
  if (n % 4 || ((uintptr_t)p | (uintptr_t)g | (uintptr_t)m | (uintptr_t)v) & 15 ||
      (hi && (((uintptr_t)hi | (uintptr_t)lo) & 15)))
    panic("adamw_flat: buffers must be 16-byte aligned with a multiple of 4 elements");
  const float c1 = 1.0f - b1, c2 = 1.0f - b2;
  k_adamw_flat<<<grid_for((size_t)n / 4, 256), 256, 0, stream()>>>(
      p, g, m, v, n / 4, lr, b1, b2, eps, wd, c1, c2, grad_scale, bc_tab, step_dev, hi, lo);
  count_launch();
  after_launch("k_adamw_flat");
}

namespace {
__global__ void k_step_advance(int64_t* step) { *step += 1; }
}  // namespace

// One more optimizer step on the device counter the table-driven AdamW reads
// (a captured step replays it, so every replay is a new step).
void step_advance(int64_t* step_dev) {
  k_step_advance<<<1, 1, 0, stream()>>>(step_dev);
  count_launch();
  after_launch("k_step_advance");
}

// Bias corrections 1 - beta**t for t = 1..cap, as the host path computes them
// (f32 powf), laid out [2*(t-1)] = bc1, [2*(t-1)+1] = bc2.
std::vector<float> adam_bc_table(float b1, float b2, int64_t cap) {
  std::vector<float> h((size_t)cap * 2);
  for (int64_t t = 1; t <= cap; ++t) {
    h[2 * (t - 1)] = 1.0f - powf(b1, (float)t);
    h[2 * (t - 1) + 1] = 1.0f - powf(b2, (float)t);
  }
  return h;
}

void adamw_multi(const AdamSeg* segs, int nseg, float lr, float b1, float b2, float eps, float wd,
                 float bc1, float bc2, float grad_scale) {
  adamw_multi_tab(segs, nseg, lr, b1, b2, eps, wd, bc1, bc2, grad_scale, nullptr, nullptr);
}

void adamw_multi_tab(const AdamSeg* segs, int nseg, float lr, float b1, float b2, float eps,
                     float wd, float bc1, float bc2, float grad_scale, const float* bc_tab,
                     const int64_t* step_dev) {
  plane_cache_clear();   // parameters and moments change in place
  float c1 = 1.0f - b1, c2 = 1.0f - b2;  // the host-side (1.0 - beta) literals
  for (int base = 0; base < nseg; base += 64) {
    int n = std::min(64, nseg - base);
    SegTable t;
    int64_t acc = 0;
    for (int i = 0; i < n; ++i) {
      t.seg[i] = segs[base + i];
      t.start[i] = acc;
      acc += (segs[base + i].n + 3) / 4;
    }
    t.start[n] = acc;
    if (acc == 0) continue;
    k_adamw<<<grid_for((size_t)acc, 256), 256, 0, stream()>>>(t, n, acc, lr, b1, b2, eps, wd, c1,
                                                              c2, bc1, bc2, grad_scale, bc_tab,
                                                              step_dev);
    count_launch();
    after_launch("k_adamw");
  }
}

}  // namespace malus

extern "C" void malus_adamw_multi(const int64_t* params, const int64_t* grads, const int64_t* ms,
                                  const int64_t* vs, size_t n, float lr, float beta1, float beta2,
                                  float eps, float wd, int64_t step, float grad_scale) {
  using namespace malus;
  std::vector<AdamSeg> segs;
  segs.reserve(n);
  for (size_t i = 0; i < n; ++i) {
    auto* p = tb(params[i]);
    if (tb(ms[i])->len != p->len || tb(vs[i])->len != p->len)
      panic("adamw: moment %zu has %zu/%zu elements, parameter has %zu", i, tb(ms[i])->len,
            tb(vs[i])->len, p->len);
    if (grads[i] && tb(grads[i])->len != p->len)
      panic("adamw: grad %zu has %zu elements, parameter has %zu", i, tb(grads[i])->len, p->len);
    segs.push_back(AdamSeg{fptr(params[i]), grads[i] ? fptr(grads[i]) : nullptr, fptr(ms[i]),
                           fptr(vs[i]), (int64_t)p->len});
  }
  float bc1 = 1.0f - powf(beta1, (float)step);
  float bc2 = 1.0f - powf(beta2, (float)step);
  adamw_multi(segs.data(), (int)segs.size(), lr, beta1, beta2, eps, wd, bc1, bc2, grad_scale);
}
