// The fused B200 nanoGPT step (mode 1).
//
// The same math as the tape replay of examples/nanogpt_modular.ml (pre-LN
// blocks, head-folded causal attention with scale 1/sqrt(hs) and a -1e9 mask,
// tanh-GELU MLP, cross-entropy, L2-coupled AdamW), organised for B200:
//  * every GEMM operand is produced already split into tf32 hi/lo planes by
//    the kernel that computes it (layernorm, softmax, GEMM epilogues, the
//    cross-entropy kernel), so no GEMM pays a separate split pass;
//  * GEMM epilogues write the attention head fold/unfold layouts directly
//    (no permute copies), fuse the residual adds, GELU and its derivative;
//  * Q, K, V come from one GEMM over the three contiguous weight slices
//    (N-segmented operand) and the Q/K/V input gradient is one K-segmented
//    GEMM; transposed operands use MN-major descriptors, never copies;
//  * cross-entropy forward and backward are one kernel (dL/dloss = 1);
//  * activations live in buffers allocated once per model.
// Gradient bookkeeping follows the tape's VJP rules; results agree with the
// tape replay and the CPU oracle within the parity tolerances.
#include "common.cuh"

#include <cmath>
#include <vector>

namespace malus {

int dp_allreduce_async(float* ptr, size_t count);
bool attn_fwd_supported(int T, int hs);
void attn_fwd(const float* qkv_hi, const float* qkv_lo, int B, int H, int T, int hs, float scale,
              float* p_hi, float* p_lo, float* o_hi, float* o_lo, float* stats);
void attn_bwd(const float* qkv_hi, const float* qkv_lo, const float* do_hi, const float* do_lo,
              const float* o_hi, const float* o_lo, const float* stats, float* D, int B, int H, int T, int hs,
              float scale, float* dqkv_hi, float* dqkv_lo);
void dp_join();
int dp_world();

namespace {

constexpr float kEps = 1e-5f;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void split_store(float* hi, float* lo, size_t o, float v) {
  float h = tf32_rn(v);
  hi[o] = h;
  lo[o] = tf32_rn(v - h);
}

// x0[m, :] = wte[tok[m], :] + wpe[m % T, :]
__global__ void k_embed2(const float* __restrict__ wte, const float* __restrict__ wpe,
                         const int32_t* __restrict__ tok, float* __restrict__ x, int M, int T,
                         int C, int V, int32_t* err) {
  int lane = threadIdx.x & 31;
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int nw = (gridDim.x * blockDim.x) >> 5;
  for (int m = warp; m < M; m += nw) {
    int t = tok[m];
    if (t < 0 || t >= V) {
      if (lane == 0) atomicExch(err, 4);
      t = 0;
    }
    const float4* a = reinterpret_cast<const float4*>(wte + (size_t)t * C);
    const float4* b = reinterpret_cast<const float4*>(wpe + (size_t)(m % T) * C);
    float4* o = reinterpret_cast<float4*>(x + (size_t)m * C);
    for (int c = lane; c < C / 4; c += 32) {
      float4 p = a[c], q = b[c];
      o[c] = make_float4(p.x + q.x, p.y + q.y, p.z + q.z, p.w + q.w);
    }
  }
}

__device__ __forceinline__ float4 f4(const float* p, int i4) { return reinterpret_cast<const float4*>(p)[i4]; }
__device__ __forceinline__ void split_store4(float* hi, float* lo, size_t o4, float4 v) {
  const float4 h = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
  reinterpret_cast<float4*>(hi)[o4] = h;
  reinterpret_cast<float4*>(lo)[o4] = make_float4(tf32_rn(v.x - h.x), tf32_rn(v.y - h.y),
                                                  tf32_rn(v.z - h.z), tf32_rn(v.w - h.w));
}

// Layernorm (no affine, population variance, eps) times gain, written as tf32
// planes; saves per-row mean and variance.  One warp per row, the row in
// registers as float4 groups (lane l owns groups l + 32k; C % 4 == 0).
template <int P4>
__global__ void k_ln_fwd_split(const float* __restrict__ x, const float* __restrict__ g,
                               float* __restrict__ out_hi, float* __restrict__ out_lo,
                               float* __restrict__ mean_out, float* __restrict__ var_out, int M,
                               int C) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int C4 = C >> 2;
  float4 gk[P4];
#pragma unroll
  for (int k = 0; k < P4; ++k) {
    const int i4 = lane + 32 * k;
    gk[k] = i4 < C4 ? f4(g, i4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r = warp; r < M; r += nw) {
    const float* xr = x + (size_t)r * C;
    float4 v[P4];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int i4 = lane + 32 * k;
      v[k] = i4 < C4 ? f4(xr, i4) : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    const float mean = wsum(s) / (float)C;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      if (lane + 32 * k < C4) {
        const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
      }
    }
    const float var = wsum(q) / (float)C;
    const float sigma = sqrtf(var + kEps);
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int i4 = lane + 32 * k;
      if (i4 < C4)
        split_store4(out_hi, out_lo, (size_t)r * C4 + i4,
                     make_float4(((v[k].x - mean) / sigma) * gk[k].x, ((v[k].y - mean) / sigma) * gk[k].y,
                                 ((v[k].z - mean) / sigma) * gk[k].z, ((v[k].w - mean) / sigma) * gk[k].w));
    }
    if (lane == 0) {
      mean_out[r] = mean;
      var_out[r] = var;
    }
  }
}

// Layernorm backward through the gain, plus the residual stream:
//   dy = dz * g ; y = (x - mean)/sigma ; dx = ((dy - mean(dy)) - y*mean(dy*y)) / sqrt(var+eps)
//   gout = resid + dx (f32 and optional tf32 planes); gain partials part[blk][c] = sum dz*y.
// One warp per row as float4 groups; lane l owns groups l + 32k, so each lane
// keeps its gain partials in registers across rows; a row's loads are issued
// before use.
template <int P4>
__global__ void k_ln_bwd_fused(const float* __restrict__ x, const float* __restrict__ mean_in,
                               const float* __restrict__ var_in, const float* __restrict__ g,
                               const float* __restrict__ dz, const float* __restrict__ resid,
                               float* __restrict__ gout, float* __restrict__ gout_hi,
                               float* __restrict__ gout_lo, float* __restrict__ part, int M,
                               int C) {
  extern __shared__ float sacc[];  // [warps][C]
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int nwb = blockDim.x >> 5;
  const int warp = blockIdx.x * nwb + wib;
  const int nw = gridDim.x * nwb;
  const int C4 = C >> 2;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 gk[P4], gacc[P4];
#pragma unroll
  for (int k = 0; k < P4; ++k) {
    const int i4 = lane + 32 * k;
    gk[k] = i4 < C4 ? f4(g, i4) : z4;
    gacc[k] = z4;
  }
  for (int r = warp; r < M; r += nw) {
    const size_t ro4 = (size_t)r * C4;
    float4 xv[P4], dv[P4], rv[P4];
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int i4 = lane + 32 * k;
      const bool in = i4 < C4;
      xv[k] = in ? f4(x, ro4 + i4) : z4;
      dv[k] = in ? f4(dz, ro4 + i4) : z4;
      rv[k] = (resid && in) ? f4(resid, ro4 + i4) : z4;
    }
    const float mean = mean_in[r], var = var_in[r];
    const float sigma = sqrtf(var + kEps);
    const float inv = 1.0f / sigma;
    float sg = 0.0f, sgy = 0.0f;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      if (lane + 32 * k < C4) {
        float4 y = make_float4((xv[k].x - mean) / sigma, (xv[k].y - mean) / sigma,
                               (xv[k].z - mean) / sigma, (xv[k].w - mean) / sigma);
        gacc[k].x += dv[k].x * y.x; gacc[k].y += dv[k].y * y.y;
        gacc[k].z += dv[k].z * y.z; gacc[k].w += dv[k].w * y.w;
        xv[k] = y;                                             // y from here on
        dv[k] = make_float4(dv[k].x * gk[k].x, dv[k].y * gk[k].y, dv[k].z * gk[k].z,
                            dv[k].w * gk[k].w);                // dy from here on
        sg += (dv[k].x + dv[k].y) + (dv[k].z + dv[k].w);
        sgy += (dv[k].x * y.x + dv[k].y * y.y) + (dv[k].z * y.z + dv[k].w * y.w);
      }
    }
    const float mg = wsum(sg) / (float)C, mgy = wsum(sgy) / (float)C;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int i4 = lane + 32 * k;
      if (i4 < C4) {
        float4 o = make_float4(((dv[k].x - mg) - xv[k].x * mgy) * inv, ((dv[k].y - mg) - xv[k].y * mgy) * inv,
                               ((dv[k].z - mg) - xv[k].z * mgy) * inv, ((dv[k].w - mg) - xv[k].w * mgy) * inv);
        if (resid) o = make_float4(rv[k].x + o.x, rv[k].y + o.y, rv[k].z + o.z, rv[k].w + o.w);
        reinterpret_cast<float4*>(gout)[ro4 + i4] = o;
        if (gout_hi) split_store4(gout_hi, gout_lo, ro4 + i4, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < P4; ++k) {
    const int i4 = lane + 32 * k;
    if (i4 < C4) reinterpret_cast<float4*>(sacc + (size_t)wib * C)[i4] = gacc[k];
  }
  __syncthreads();
  // block partial = sum over its warps (fixed order)
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    float s = 0.0f;
    for (int w = 0; w < nwb; ++w) s += sacc[(size_t)w * C + i];
    part[(size_t)blockIdx.x * C + i] = s;
  }
}

// out[c] = sum_b part[b][c] in a fixed order: 32 row groups per column (group
// g sums rows g, g + 32, ...), then the 32 group sums in order.  Block = 32
// columns x 32 row groups: the column count is small (C / 32 blocks), so the
// rows are spread over as many warps as a block holds to keep the serial
// chains short (the kernel is latency-bound).
constexpr int kColGroups = 32;
__global__ void __launch_bounds__(32 * kColGroups)
k_colsum(const float* __restrict__ part, float* __restrict__ out, int nblk, int C) {
  __shared__ float sh[kColGroups][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.0f;
  if (c < C) {
#pragma unroll 4
    for (int b = ty; b < nblk; b += kColGroups) s += part[(size_t)b * C + c];
  }
  sh[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < C) {
    float t = sh[0][tx];
#pragma unroll
    for (int q = 1; q < kColGroups; ++q) t += sh[q][tx];
    out[c] = t;
  }
}

// Causal softmax of one row of S (already scaled): P planes.  -1e9 above the
// diagonal as the reference's additive mask (metal.rs:1601-1612).  One warp per
// row as float4 groups (T % 4 == 0); only the groups that reach the diagonal
// are read (the causal S GEMM does not compute the rest).
template <int P4>
__global__ void k_softmax_causal_split(const float* __restrict__ S, float* __restrict__ p_hi,
                                       float* __restrict__ p_lo, int rows, int T) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int T4 = T >> 2;
  for (int r = warp; r < rows; r += nw) {
    const int i = r % T;
    const float* sr = S + (size_t)r * T;
    float4 v[P4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int j4 = lane + 32 * k, j = 4 * j4;
      // masked scores (j > i) would be s - 1e9, whose exp underflows to exactly
      // 0: -inf gives the same 0
      if (j4 < T4 && j <= i) {
        float4 t = f4(sr, j4);
        v[k] = make_float4(t.x, j + 1 <= i ? t.y : -INFINITY, j + 2 <= i ? t.z : -INFINITY,
                           j + 3 <= i ? t.w : -INFINITY);
      } else {
        v[k] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
      m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    }
    m = wmax(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int j = 4 * (lane + 32 * k);
      v[k] = make_float4(j <= i ? expf(v[k].x - m) : 0.0f, j + 1 <= i ? expf(v[k].y - m) : 0.0f,
                         j + 2 <= i ? expf(v[k].z - m) : 0.0f, j + 3 <= i ? expf(v[k].w - m) : 0.0f);
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    s = wsum(s);
    // keys past the query's 128-wide tile are never read by the causal GEMMs
    const int jend4 = min(T, (i / 128 + 1) * 128) >> 2;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int j4 = lane + 32 * k;
      if (j4 < jend4)
        split_store4(p_hi, p_lo, (size_t)r * T4 + j4,
                     make_float4(v[k].x / s, v[k].y / s, v[k].z / s, v[k].w / s));
    }
  }
}

// dS = scale * P * (dP - sum_j dP*P) as planes (softmax VJP, transformer_bwd.ml:15-20,
// then the scores = qk * scale VJP).  dP above the diagonal is not computed and
// P is 0 there, so neither is read.
template <int P4>
__global__ void k_softmax_bwd_split(const float* __restrict__ p_hi, const float* __restrict__ p_lo,
                                    const float* __restrict__ dP, float* __restrict__ ds_hi,
                                    float* __restrict__ ds_lo, int rows, int T, float scale) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int T4 = T >> 2;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = warp; r < rows; r += nw) {
    const size_t b4 = (size_t)r * T4;
    const int i = r % T;
    float4 pv[P4], gv[P4];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int j4 = lane + 32 * k, j = 4 * j4;
      if (j4 < T4 && j <= i) {
        const float4 h = f4(p_hi, b4 + j4), l = f4(p_lo, b4 + j4), d = f4(dP, b4 + j4);
        pv[k] = make_float4(h.x + l.x, j + 1 <= i ? h.y + l.y : 0.0f, j + 2 <= i ? h.z + l.z : 0.0f,
                            j + 3 <= i ? h.w + l.w : 0.0f);
        gv[k] = make_float4(d.x, j + 1 <= i ? d.y : 0.0f, j + 2 <= i ? d.z : 0.0f, j + 3 <= i ? d.w : 0.0f);
      } else {
        pv[k] = z4;
        gv[k] = z4;
      }
      dot += (gv[k].x * pv[k].x + gv[k].y * pv[k].y) + (gv[k].z * pv[k].z + gv[k].w * pv[k].w);
    }
    dot = wsum(dot);
    const int jend4 = min(T, (i / 128 + 1) * 128) >> 2;   // as in the forward: later tiles are never read
#pragma unroll
    for (int k = 0; k < P4; ++k) {
      const int j4 = lane + 32 * k;
      if (j4 < jend4)
        split_store4(ds_hi, ds_lo, b4 + j4,
                     make_float4((pv[k].x * (gv[k].x - dot)) * scale, (pv[k].y * (gv[k].y - dot)) * scale,
                                 (pv[k].z * (gv[k].z - dot)) * scale, (pv[k].w * (gv[k].w - dot)) * scale));
    }
  }
}

// Cross-entropy forward + backward in one pass per row: probs, nll[r], and
// dlogits = (p - onehot) / M as planes (pitch ldp).
template <int PER>
__global__ void k_xent_fused(const float* __restrict__ logits, const int32_t* __restrict__ tgt,
                             float* __restrict__ nll, float* __restrict__ d_hi,
                             float* __restrict__ d_lo, int M, int V, int ldp, int32_t* err) {
  int lane = threadIdx.x & 31;
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int nw = (gridDim.x * blockDim.x) >> 5;
  const float scale = 1.0f / (float)M;   // dout[0] / N with dout = ones_like(loss)
  for (int r = warp; r < M; r += nw) {
    const float* xr = logits + (size_t)r * V;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int j = lane + 32 * k;
      v[k] = j < V ? xr[j] : -INFINITY;
      m = fmaxf(m, v[k]);
    }
    m = wmax(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int j = lane + 32 * k;
      v[k] = j < V ? expf(v[k] - m) : 0.0f;
      s += v[k];
    }
    s = wsum(s);
    int t = tgt[r];
    bool bad = t < 0 || t >= V;
    float pt = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int j = lane + 32 * k;
      if (j < ldp) {
        float p = j < V ? v[k] / s : 0.0f;
        if (j == t) pt = p;
        float gr = j < V ? (j == t ? p - 1.0f : p) * scale : 0.0f;
        split_store(d_hi, d_lo, (size_t)r * ldp + j, gr);
      }
    }
    pt = wsum(pt);
    if (lane == 0) {
      if (bad) { atomicExch(err, 3); nll[r] = 0.0f; }
      else nll[r] = -logf(pt);
    }
  }
}

// The same cross-entropy for wide rows (vocab > 1024): one 512-thread block
// per row, three passes over the row (max, sum of exp, probabilities and
// dlogits planes); block reductions in a fixed order.
__device__ __forceinline__ float block_reduce(float v, float* sh, bool is_max) {
  v = is_max ? wmax(v) : wsum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = l < nw ? sh[l] : (is_max ? -INFINITY : 0.0f);
  t = is_max ? wmax(t) : wsum(t);
  return t;   // every thread of warp 0..nw-1 holds the result
}

__global__ void k_xent_fused_wide(const float* __restrict__ logits, const int32_t* __restrict__ tgt,
                                  float* __restrict__ nll, float* __restrict__ d_hi,
                                  float* __restrict__ d_lo, int M, int V, int ldp, int32_t* err) {
  __shared__ float sh[32];
  __shared__ float pt_sh;
  const float scale = 1.0f / (float)M;
  for (int r = blockIdx.x; r < M; r += gridDim.x) {
    const float* xr = logits + (size_t)r * V;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < V; j += blockDim.x) m = fmaxf(m, xr[j]);
    m = block_reduce(m, sh, true);
    float s = 0.0f;
    for (int j = threadIdx.x; j < V; j += blockDim.x) s += expf(xr[j] - m);
    s = block_reduce(s, sh, false);
    const int t = tgt[r];
    const bool bad = t < 0 || t >= V;
    if (threadIdx.x == 0) pt_sh = 0.0f;
    __syncthreads();
    for (int j = threadIdx.x; j < ldp; j += blockDim.x) {
      const float p = j < V ? expf(xr[j] - m) / s : 0.0f;
      if (j == t) pt_sh = p;
      const float gr = j < V ? (j == t ? p - 1.0f : p) * scale : 0.0f;
      split_store(d_hi, d_lo, (size_t)r * ldp + j, gr);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      if (bad) { atomicExch(err, 3); nll[r] = 0.0f; }
      else nll[r] = -logf(pt_sh);
    }
    __syncthreads();
  }
}

__global__ void k_mean_nll(const float* __restrict__ v, float* __restrict__ out, int n) {
  __shared__ float sh[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
  s = wsum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
    t = wsum(t);
    if (threadIdx.x == 0) out[0] = t / (float)n;
  }
}

__global__ void k_add_inplace(float* __restrict__ a, const float* __restrict__ b, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t st = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += st) a[i] = a[i] + b[i];
}

__global__ void k_step_inc(int64_t* step) { *step += 1; }

// dwpe[t][c] = sum over b = 0..B-1 (in that order) of g[b][t][c]: the order in
// which the embedding VJP scatters the position ids b*T + t.
__global__ void k_dwpe(const float* __restrict__ g, float* __restrict__ out, int B, size_t TC) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t st = (size_t)gridDim.x * blockDim.x;
  for (; i < TC; i += st) {
    float s = 0.0f;
    for (int b = 0; b < B; ++b) s += g[(size_t)b * TC + i];
    out[i] = s;
  }
}

TcLayout L(int64_t d1 = 0, int64_t s1 = 0, int64_t d2 = 0, int64_t s2 = 0, int64_t s3 = 0) {
  return TcLayout{d1, s1, d2, s2, s3};
}

struct Planes {
  float* hi = nullptr;
  float* lo = nullptr;
};

}  // namespace

struct FusedStep {
  malus_gpt_config cfg;
  int V, L, H, C, T, B, M, hs, C4, BH, Vp;
  float scale;
  std::vector<float*> params;
  std::vector<size_t> sizes, goff;
  std::vector<std::pair<size_t, size_t>> buckets;   // DP all-reduce ranges, issue order
  float* gbuf;
  std::vector<float*> allocs;
  // weight planes (mirror of the parameter layout) and the padded LM head planes
  Planes wpl;
  std::vector<size_t> poff;   // offsets into wpl (== parameter offsets)
  Planes lmpl;                // [C][Vp] (untied only)
  // activations
  std::vector<float*> x;      // L+1 residual stream tensors [M][C]
  std::vector<float*> mean1, var1, mean2, var2, x2, h;  // per layer
  std::vector<Planes> xn1, qkv, P, O, xn2, gel;
  bool fused_attn = false;     // attention forward by attn_fwd
  bool fused_attn_bwd = false; // ... and backward by attn_bwd (no [T][T] tensor at all)
  std::vector<float*> astats;  // per layer [B*H*T][2] row statistics of the fused forward
  float* arow = nullptr;       // [B*H*T] rowsum(dO * O) workspace of the fused backward
  Planes xf;
  float *meanf, *varf, *logits, *nll;
  Planes dlog;
  // backward scratch
  float *S, *dP, *dxf, *dxn, *g_a, *g_b, *part, *emb_tmp;
  Planes g_a_pl, g_b_pl, dh, dO, dqkv, dS;
  int part_blocks;
  void* emb_ws = nullptr;      // embedding-VJP workspace (no allocation inside a step)
  // optimizer state (the model's fused buffers) and the device step counter
  float *pbuf = nullptr, *mbuf = nullptr, *vbuf = nullptr;
  size_t total = 0;
  int64_t* step_dev = nullptr;
  float* bc_tab = nullptr;     // [2 * bc_cap] host-computed 1 - beta**t
  int64_t bc_cap = 0;
  int64_t host_step = 0;
  // CUDA graph of one whole training step (captured after the first eager step)
  cudaGraphExec_t exec = nullptr;
  int64_t graph_launches = 0;
};

namespace {

float* dalloc(FusedStep* f, size_t n) {
  float* p = nullptr;
  MALUS_CUDA(cudaMalloc(&p, std::max<size_t>(n, 64) * sizeof(float)));
  f->allocs.push_back(p);
  return p;
}
Planes palloc(FusedStep* f, size_t n) { return Planes{dalloc(f, n), dalloc(f, n)}; }

TcOperand op(const Planes& p, int64_t rows, int64_t cols, int64_t pitch, bool mn, int nz = 1,
             int64_t zstride = 0, int zmode = kZNone, int seg = 0, int64_t offset = 0) {
  return TcOperand{p.hi + offset, p.lo + offset, rows, cols, pitch, nz, zstride, mn, zmode, seg};
}

void gemm(int M, int N, int K, int batch, const TcOperand& a, const TcOperand& b, int epi,
          TcLayout oz, TcLayout om, TcLayout on, float* out, Planes outp, const float* aux,
          float alpha = 1.0f, int causal = kCausalNone, const float* aux_lo = nullptr,
          const float* rowv = nullptr) {
  TcProblem p{};
  p.M = M; p.N = N; p.K = K; p.batch = batch;
  p.a = a; p.b = b;
  p.epi = epi;
  p.oz = oz; p.om = om; p.on = on;
  p.out = out; p.out_hi = outp.hi; p.out_lo = outp.lo; p.aux = aux;
  p.alpha = alpha; p.beta = 0.0f;
  p.causal = causal;
  p.aux_lo = aux_lo;
  p.rowv = rowv;
  gemm_tc_planes(p);
}

unsigned rows_grid(int rows) { return grid_for((size_t)rows * 32, 256); }

// CUDA-event timing of one labelled launch (or launch group) with its
// algorithmic bytes (one read of each input, one write of each output), while
// the bench's profiled pass has kernel timing on; free otherwise.
struct KTimer {
  int id;
  KTimer(const char* label, double bytes) : id(prof_begin_named(label, bytes)) {}
  ~KTimer() { prof_end(id); }
};

// bytes of the causal tiles' rows of a [T][T] head: row i spans the 128-wide
// tiles up to its own (what the attention kernels read and write)
double causal_tile_elems(int T) {
  double e = 0.0;
  for (int i = 0; i < T; ++i) e += std::min(T, (i / 128 + 1) * 128);
  return e;
}

// float4 groups per lane for a row of LEN floats (LEN % 4 == 0, LEN <= 1024)
#define P4_DISPATCH(LEN, CALL)                                        \
  do {                                                                \
    const int l4_ = (LEN) / 4;                                        \
    if (l4_ <= 32) { constexpr int P_ = 1; CALL; }                    \
    else if (l4_ <= 64) { constexpr int P_ = 2; CALL; }               \
    else if (l4_ <= 96) { constexpr int P_ = 3; CALL; }               \
    else if (l4_ <= 128) { constexpr int P_ = 4; CALL; }              \
    else if (l4_ <= 192) { constexpr int P_ = 6; CALL; }              \
    else if (l4_ <= 256) { constexpr int P_ = 8; CALL; }              \
    else panic("fused step: row length %d exceeds 1024", (int)(LEN)); \
  } while (0)

#define PER_DISPATCH(LEN, CALL)                      \
  do {                                               \
    if ((LEN) <= 32) { constexpr int P_ = 1; CALL; } \
    else if ((LEN) <= 128) { constexpr int P_ = 4; CALL; } \
    else if ((LEN) <= 256) { constexpr int P_ = 8; CALL; } \
    else if ((LEN) <= 512) { constexpr int P_ = 16; CALL; } \
    else if ((LEN) <= 1024) { constexpr int P_ = 32; CALL; } \
    else panic("fused step: row length %d exceeds 1024", (int)(LEN)); \
  } while (0)

void ln_fwd(FusedStep* f, const float* x, const float* g, Planes out, float* mean, float* var) {
  const double MC = (double)f->M * f->C;
  KTimer kt("k_ln_fwd_split", 4.0 * (3.0 * MC + f->C + 2.0 * f->M));
  P4_DISPATCH(f->C, (k_ln_fwd_split<P_><<<rows_grid(f->M), 256, 0, stream()>>>(
                          x, g, out.hi, out.lo, mean, var, f->M, f->C)));
  count_launch();
  after_launch("k_ln_fwd_split");
}

void ln_bwd(FusedStep* f, const float* x, const float* mean, const float* var, const float* g,
            const float* dz, const float* resid, float* gout, Planes gpl, float* dgain) {
  int threads = 256;
  size_t smem = (size_t)(threads / 32) * f->C * sizeof(float);
  const double MC = (double)f->M * f->C, part = (double)f->part_blocks * f->C;
  {
    KTimer kt("k_ln_bwd_fused", 4.0 * (MC + 2.0 * f->M + f->C + MC + (resid ? MC : 0.0) + (gout ? MC : 0.0) +
                                       (gpl.hi ? 2.0 * MC : 0.0) + part));
    P4_DISPATCH(f->C, (k_ln_bwd_fused<P_><<<f->part_blocks, threads, smem, stream()>>>(
                            x, mean, var, g, dz, resid, gout, gpl.hi, gpl.lo, f->part, f->M, f->C)));
  }
  {
    KTimer kt("k_colsum", 4.0 * (part + f->C));
    k_colsum<<<(f->C + 31) / 32, 32 * kColGroups, 0, stream()>>>(f->part, dgain, f->part_blocks, f->C);
  }
  count_launch(2);
  after_launch("k_ln_bwd_fused");
}

void split_weights(FusedStep* f) {
  // the weight matrices that feed GEMMs: per layer Wq|Wk|Wv, Wo, W1, W2; wte (tied head)
  for (int l = 0; l < f->L; ++l) {
    size_t b = (size_t)l * 8;
    const float* src = f->params[b + 1];
    size_t n = 4 * (size_t)f->C * f->C;        // Wq, Wk, Wv, Wo are contiguous
    tf32_split(src, 1, (int64_t)n, (int64_t)n, 1, 0, f->wpl.hi + f->poff[b + 1],
               f->wpl.lo + f->poff[b + 1], (int64_t)n);
    tf32_split(f->params[b + 6], f->C, f->C4, f->C4, 1, 0, f->wpl.hi + f->poff[b + 6],
               f->wpl.lo + f->poff[b + 6], f->C4);
    tf32_split(f->params[b + 7], f->C4, f->C, f->C, 1, 0, f->wpl.hi + f->poff[b + 7],
               f->wpl.lo + f->poff[b + 7], f->C);
  }
  size_t top = (size_t)f->L * 8;
  if (f->cfg.tied)
    tf32_split(f->params[top], f->V, f->C, f->C, 1, 0, f->wpl.hi + f->poff[top],
               f->wpl.lo + f->poff[top], f->C);
  else
    tf32_split(f->params[top + 3], f->C, f->V, f->V, 1, 0, f->lmpl.hi, f->lmpl.lo, f->Vp);
}

}  // namespace

namespace {

// Bias-correction table for steps 1..cap: the same f32 powf the host computes.
void fill_bc_table(FusedStep* f, int64_t cap) {
  std::vector<float> h((size_t)cap * 2);
  for (int64_t t = 1; t <= cap; ++t) {
    h[2 * (t - 1)] = 1.0f - powf(f->cfg.beta1, (float)t);
    h[2 * (t - 1) + 1] = 1.0f - powf(f->cfg.beta2, (float)t);
  }
  if (f->bc_tab) {
    MALUS_CUDA(cudaStreamSynchronize(stream()));
    MALUS_CUDA(cudaFree(f->bc_tab));
  }
  MALUS_CUDA(cudaMalloc(&f->bc_tab, h.size() * sizeof(float)));
  MALUS_CUDA(cudaMemcpy(f->bc_tab, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
  f->bc_cap = cap;
}

}  // namespace

FusedStep* fused_create(const malus_gpt_config& cfg, const std::vector<float*>& params,
                        const std::vector<size_t>& sizes, float* gbuf,
                        const std::vector<size_t>& goff, float* pbuf, float* mbuf, float* vbuf,
                        size_t total_elems) {
  auto* f = new FusedStep();
  f->pbuf = pbuf;
  f->mbuf = mbuf;
  f->vbuf = vbuf;
  f->total = total_elems;
  f->cfg = cfg;
  f->V = cfg.vocab; f->L = cfg.n_layer; f->H = cfg.n_head; f->C = cfg.n_embd;
  f->T = cfg.block_size; f->B = cfg.batch;
  f->M = f->B * f->T; f->hs = f->C / f->H; f->C4 = 4 * f->C; f->BH = f->B * f->H;
  f->Vp = (f->V + 3) & ~3;
  f->scale = 1.0f / sqrtf((float)f->hs);
  // MALUS_ATTN_FUSED=0 keeps the GEMM + softmax attention where the fused kernels
  // apply.  The backward goes through the fused kernels (no [B*H][T][T]
  // tensor) from T = 512 on, where those tensors dominate (C5, T = 1024:
  // 47.5 vs 49.0 ms per step, 9.7 GB of P planes saved), and through the
  // GEMMs below (C4, T = 256: the GEMM backward is faster);
  // MALUS_ATTN_BWD=1 / 0 forces either
  const char* fa = getenv("MALUS_ATTN_FUSED");
  const char* fb = getenv("MALUS_ATTN_BWD");
  f->fused_attn = attn_fwd_supported(f->T, f->hs) && !(fa && fa[0] == '0');
  f->fused_attn_bwd = f->fused_attn && (fb ? fb[0] == '1' : f->T >= 512);
  if (f->C % 32 || f->hs % 4 || f->T % 4 || f->T > 1024 || f->C > 1024)
    panic("fused step needs n_embd %% 32 == 0, head size %% 4 == 0, T %% 4 == 0, T, C <= 1024 "
          "(got C=%d hs=%d T=%d)", f->C, f->hs, f->T);
  f->params = params;
  f->sizes = sizes;
  f->gbuf = gbuf;
  f->goff = goff;
  f->poff = goff;   // parameters and gradients share the slice layout
  f->buckets = gpt_dp_buckets(f->L, goff, sizes);
  size_t total = goff.back() + ((sizes.back() + 63) & ~size_t(63));
  f->wpl = palloc(f, total);
  if (!cfg.tied) f->lmpl = palloc(f, (size_t)f->C * f->Vp);
  size_t M = f->M, C = f->C, C4 = f->C4, TT = (size_t)f->BH * f->T * f->T;
  for (int l = 0; l <= f->L; ++l) f->x.push_back(dalloc(f, M * C));
  for (int l = 0; l < f->L; ++l) {
    f->mean1.push_back(dalloc(f, M));
    f->var1.push_back(dalloc(f, M));
    f->mean2.push_back(dalloc(f, M));
    f->var2.push_back(dalloc(f, M));
    f->x2.push_back(dalloc(f, M * C));
    f->h.push_back(dalloc(f, M * C4));
    f->xn1.push_back(palloc(f, M * C));
    f->qkv.push_back(palloc(f, 3 * M * C));
    if (f->fused_attn_bwd) f->astats.push_back(dalloc(f, 2 * (size_t)f->BH * f->T));
    else f->P.push_back(palloc(f, TT));
    f->O.push_back(palloc(f, M * C));
    f->xn2.push_back(palloc(f, M * C));
    f->gel.push_back(palloc(f, M * C4));
  }
  f->xf = palloc(f, M * C);
  f->meanf = dalloc(f, M);
  f->varf = dalloc(f, M);
  f->logits = dalloc(f, M * f->V);
  f->nll = dalloc(f, M);
  f->dlog = palloc(f, M * f->Vp);
  if (!f->fused_attn) f->S = dalloc(f, TT);
  if (f->fused_attn_bwd) {
    f->arow = dalloc(f, (size_t)f->BH * f->T);
  } else {
    f->dP = dalloc(f, TT);
    f->dS = palloc(f, TT);
  }
  f->dxf = dalloc(f, M * C);
  f->dxn = dalloc(f, M * C);
  f->g_a = dalloc(f, M * C);
  f->g_b = dalloc(f, M * C);
  f->g_a_pl = palloc(f, M * C);
  f->g_b_pl = palloc(f, M * C);
  f->dh = palloc(f, M * C4);
  f->dO = palloc(f, M * C);
  f->dqkv = palloc(f, 3 * M * C);
  f->part_blocks = kNumSMs * 2;
  f->part = dalloc(f, (size_t)f->part_blocks * C);
  f->emb_tmp = dalloc(f, (size_t)f->V * C);
  f->emb_ws = dalloc(f, (embedding_bwd_ws_bytes(M, f->V) + 3) / 4);
  MALUS_CUDA(cudaMalloc(&f->step_dev, sizeof(int64_t)));
  MALUS_CUDA(cudaMemset(f->step_dev, 0, sizeof(int64_t)));
  fill_bc_table(f, 1 << 16);

  split_weights(f);
  return f;
}

void fused_destroy(FusedStep* f) {
  cudaStreamSynchronize(stream());
  if (f->exec) cudaGraphExecDestroy(f->exec);
  for (float* p : f->allocs) cudaFree(p);
  cudaFree(f->step_dev);
  cudaFree(f->bc_tab);
  delete f;
}

void fused_step(FusedStep* f, const int32_t* xt, const int32_t* yt, float* loss_dev) {
  const int M = f->M, C = f->C, C4 = f->C4, T = f->T, H = f->H, hs = f->hs, BH = f->BH,
            B = f->B, V = f->V, Vp = f->Vp, Lc = f->L;
  const size_t MC = (size_t)M * C, TT = (size_t)T * T;
  const size_t top = (size_t)Lc * 8;
  auto P = [&](size_t i) { return f->params[i]; };
  auto G = [&](size_t i) { return f->gbuf + f->goff[i]; };
  auto W = [&](size_t i) { return Planes{f->wpl.hi + f->poff[i], f->wpl.lo + f->poff[i]}; };
  const TcLayout none = L();
  const TcLayout rowC = L(0, 0, 0, 0, C), rowC4 = L(0, 0, 0, 0, C4), unit = L(0, 0, 0, 0, 1);

  // ------------------------------------------------------------ forward
  {
    KTimer kt("k_embed2", 4.0 * ((double)MC + (double)(V + T) * C + M));
    k_embed2<<<grid_for((size_t)M * 32, 256), 256, 0, stream()>>>(P(top), P(top + 1), xt, f->x[0], M, T,
                                                                 C, V, device_error_word());
    count_launch();
    after_launch("k_embed2");
  }
  const double attn_elems = (double)BH * causal_tile_elems(T);   // causal-tile P / dS elements per layer
  const double qkv_elems = 3.0 * MC;
  for (int l = 0; l < Lc; ++l) {
    size_t b = (size_t)l * 8;
    ln_fwd(f, f->x[l], P(b), f->xn1[l], f->mean1[l], f->var1[l]);
    // Q|K|V = xn1 @ [Wq|Wk|Wv] written as [3][B][H][T][hs]
    gemm(M, 3 * C, C, 1, op(f->xn1[l], M, C, C, false),
         op(W(b + 1), C, C, C, true, 3, (int64_t)C * C, kZMNSeg, C), kEpiStore, none,
         L(T, (int64_t)H * T * hs, 0, 0, hs), L(C, (int64_t)B * H * T * hs, hs, (int64_t)T * hs, 1),
         nullptr, f->qkv[l], nullptr);
    if (f->fused_attn_bwd) {
      // S, causal softmax and O = P V in one kernel; the row statistics let the
      // backward recompute P
      KTimer kt("k_attn_fwd", 4.0 * (2.0 * qkv_elems + 2.0 * MC + 2.0 * BH * T));
      attn_fwd(f->qkv[l].hi, f->qkv[l].lo, B, H, T, hs, f->scale, nullptr, nullptr, f->O[l].hi, f->O[l].lo,
               f->astats[l]);
    } else if (f->fused_attn) {
      // the same kernel, keeping the P planes for the GEMM backward
      KTimer kt("k_attn_fwd", 4.0 * (2.0 * qkv_elems + 2.0 * MC + 2.0 * attn_elems));
      attn_fwd(f->qkv[l].hi, f->qkv[l].lo, B, H, T, hs, f->scale, f->P[l].hi, f->P[l].lo, f->O[l].hi,
               f->O[l].lo, nullptr);
    } else {
    // S = Q K^T * scale
    gemm(T, T, hs, BH, op(f->qkv[l], T, hs, hs, false, BH, (int64_t)T * hs, kZBatch),
         op(f->qkv[l], T, hs, hs, false, BH, (int64_t)T * hs, kZBatch, 0, MC), kEpiStore,
         L(0, 0, 0, 0, (int64_t)TT), L(0, 0, 0, 0, T), unit, f->S, Planes{}, nullptr, f->scale,
         kCausalOut);
    P4_DISPATCH(T, (k_softmax_causal_split<P_><<<rows_grid(BH * T), 256, 0, stream()>>>(
                        f->S, f->P[l].hi, f->P[l].lo, BH * T, T)));
    count_launch();
    after_launch("k_softmax_causal_split");
    // O = P V, written unfolded to [M][C]
    gemm(T, hs, T, BH, op(f->P[l], T, T, T, false, BH, (int64_t)TT, kZBatch),
         op(f->qkv[l], T, hs, hs, true, BH, (int64_t)T * hs, kZBatch, 0, 2 * MC), kEpiStore,
         L(H, (int64_t)T * C, 0, 0, hs), rowC, unit, nullptr, f->O[l], nullptr, 1.0f, kCausalALower);
    }
    // x2 = x + O Wo
    gemm(M, C, C, 1, op(f->O[l], M, C, C, false), op(W(b + 4), C, C, C, true), kEpiResid, none,
         rowC, unit, f->x2[l], Planes{}, f->x[l]);
    ln_fwd(f, f->x2[l], P(b + 5), f->xn2[l], f->mean2[l], f->var2[l]);
    // h = xn2 W1 ; gelu(h) planes
    gemm(M, C4, C, 1, op(f->xn2[l], M, C, C, false), op(W(b + 6), C, C4, C4, true), kEpiGelu, none,
         rowC4, unit, f->h[l], f->gel[l], nullptr);
    // x_{l+1} = x2 + gelu W2
    gemm(M, C, C4, 1, op(f->gel[l], M, C4, C4, false), op(W(b + 7), C4, C, C, true), kEpiResid, none,
         rowC, unit, f->x[l + 1], Planes{}, f->x2[l]);
  }
  ln_fwd(f, f->x[Lc], P(top + 2), f->xf, f->meanf, f->varf);
  if (f->cfg.tied)
    gemm(M, V, C, 1, op(f->xf, M, C, C, false), op(W(top), V, C, C, false), kEpiStore, none,
         L(0, 0, 0, 0, V), unit, f->logits, Planes{}, nullptr);
  else
    gemm(M, V, C, 1, op(f->xf, M, C, C, false), op(f->lmpl, C, V, Vp, true), kEpiStore, none,
         L(0, 0, 0, 0, V), unit, f->logits, Planes{}, nullptr);
  {
    KTimer kt("k_xent_fused + k_mean_nll", 4.0 * ((double)M * V + M + 2.0 * M * Vp + M + 1));
    if (Vp <= 1024) {
      PER_DISPATCH(Vp, (k_xent_fused<P_><<<rows_grid(M), 256, 0, stream()>>>(
                           f->logits, yt, f->nll, f->dlog.hi, f->dlog.lo, M, V, Vp, device_error_word())));
    } else {
      k_xent_fused_wide<<<std::min(M, kNumSMs * 4), 512, 0, stream()>>>(f->logits, yt, f->nll, f->dlog.hi,
                                                                        f->dlog.lo, M, V, Vp, device_error_word());
    }
    k_mean_nll<<<1, 1024, 0, stream()>>>(f->nll, loss_dev, M);
    count_launch(2);
    after_launch("k_xent_fused");
  }

  // ------------------------------------------------------------ backward
  // LM head
  if (f->cfg.tied) {
    gemm(M, C, V, 1, op(f->dlog, M, V, Vp, false), op(W(top), V, C, C, true), kEpiStore, none, rowC,
         unit, f->dxf, Planes{}, nullptr);
    gemm(V, C, M, 1, op(f->dlog, M, V, Vp, true), op(f->xf, M, C, C, true), kEpiStore, none, rowC,
         unit, G(top), Planes{}, nullptr);
  } else {
    gemm(M, C, V, 1, op(f->dlog, M, V, Vp, false), op(f->lmpl, C, V, Vp, false), kEpiStore, none,
         rowC, unit, f->dxf, Planes{}, nullptr);
    gemm(C, V, M, 1, op(f->xf, M, C, C, true), op(f->dlog, M, V, Vp, true), kEpiStore, none,
         L(0, 0, 0, 0, V), unit, G(top + 3), Planes{}, nullptr);
  }
  // g3 (grad of the last residual) = LN_f backward
  float* g3 = f->g_a;
  Planes g3p = f->g_a_pl;
  float* g2 = f->g_b;
  Planes g2p = f->g_b_pl;
  ln_bwd(f, f->x[Lc], f->meanf, f->varf, P(top + 2), f->dxf, nullptr, g3, g3p, G(top + 2));
  for (int l = Lc - 1; l >= 0; --l) {
    size_t b = (size_t)l * 8;
    // MLP: d(gelu) = g3 W2^T -> dh = d(gelu) * gelu'(h)
    gemm(M, C4, C, 1, op(g3p, M, C, C, false), op(W(b + 7), C4, C, C, false), kEpiGeluBwd, none,
         rowC4, unit, nullptr, f->dh, f->h[l]);
    gemm(C4, C, M, 1, op(f->gel[l], M, C4, C4, true), op(g3p, M, C, C, true), kEpiStore, none, rowC,
         unit, G(b + 7), Planes{}, nullptr);
    gemm(M, C, C4, 1, op(f->dh, M, C4, C4, false), op(W(b + 6), C, C4, C4, false), kEpiStore, none,
         rowC, unit, f->dxn, Planes{}, nullptr);
    gemm(C, C4, M, 1, op(f->xn2[l], M, C, C, true), op(f->dh, M, C4, C4, true), kEpiStore, none,
         rowC4, unit, G(b + 6), Planes{}, nullptr);
    ln_bwd(f, f->x2[l], f->mean2[l], f->var2[l], P(b + 5), f->dxn, g3, g2, g2p, G(b + 5));
    // attention output projection
    gemm(M, C, C, 1, op(g2p, M, C, C, false), op(W(b + 4), C, C, C, false), kEpiStore, none,
         L(T, (int64_t)H * T * hs, 0, 0, hs), L(hs, (int64_t)T * hs, 0, 0, 1), nullptr, f->dO, nullptr);
    gemm(C, C, M, 1, op(f->O[l], M, C, C, true), op(g2p, M, C, C, true), kEpiStore, none, rowC, unit,
         G(b + 4), Planes{}, nullptr);
    if (f->fused_attn_bwd) {
      // dq | dk | dv planes (head-unfolded into dqkv) with P recomputed
      KTimer kt("k_attn_bwd (dq, dkdv)", 4.0 * (2.0 * qkv_elems + 2.0 * MC + 2.0 * MC + 2.0 * BH * T + 2.0 * qkv_elems));
      attn_bwd(f->qkv[l].hi, f->qkv[l].lo, f->dO.hi, f->dO.lo, f->O[l].hi, f->O[l].lo, f->astats[l], f->arow,
               B, H, T, hs, f->scale, f->dqkv.hi, f->dqkv.lo);
    } else {
    // dP = dO V^T ; dV = P^T dO
    gemm(T, T, hs, BH, op(f->dO, T, hs, hs, false, BH, (int64_t)T * hs, kZBatch),
         op(f->qkv[l], T, hs, hs, false, BH, (int64_t)T * hs, kZBatch, 0, 2 * MC), kEpiStore,
         L(0, 0, 0, 0, (int64_t)TT), L(0, 0, 0, 0, T), unit, f->dP, Planes{}, nullptr, 1.0f, kCausalOut);
    Planes dqkv2{f->dqkv.hi + 2 * MC, f->dqkv.lo + 2 * MC};
    gemm(T, hs, T, BH, op(f->P[l], T, T, T, true, BH, (int64_t)TT, kZBatch),
         op(f->dO, T, hs, hs, true, BH, (int64_t)T * hs, kZBatch), kEpiStore,
         L(H, (int64_t)T * C, 0, 0, hs), rowC, unit, nullptr, dqkv2, nullptr, 1.0f, kCausalAUpper);
    {
      KTimer kt("k_softmax_bwd_split", 12.0 * BH * ((double)T * (T + 1) / 2) + 8.0 * attn_elems);
      P4_DISPATCH(T, (k_softmax_bwd_split<P_><<<rows_grid(BH * T), 256, 0, stream()>>>(
                          f->P[l].hi, f->P[l].lo, f->dP, f->dS.hi, f->dS.lo, BH * T, T, f->scale)));
    }
    count_launch();
    after_launch("k_softmax_bwd_split");
    // dQ = dS K ; dK = dS^T Q  (unfolded into dqkv [3][M][C])
    Planes dqkv1{f->dqkv.hi + MC, f->dqkv.lo + MC};
    gemm(T, hs, T, BH, op(f->dS, T, T, T, false, BH, (int64_t)TT, kZBatch),
         op(f->qkv[l], T, hs, hs, true, BH, (int64_t)T * hs, kZBatch, 0, MC), kEpiStore,
         L(H, (int64_t)T * C, 0, 0, hs), rowC, unit, nullptr, f->dqkv, nullptr, 1.0f, kCausalALower);
    gemm(T, hs, T, BH, op(f->dS, T, T, T, true, BH, (int64_t)TT, kZBatch),
         op(f->qkv[l], T, hs, hs, true, BH, (int64_t)T * hs, kZBatch), kEpiStore,
         L(H, (int64_t)T * C, 0, 0, hs), rowC, unit, nullptr, dqkv1, nullptr, 1.0f, kCausalAUpper);
    }
    // dxn1 = sum_j dqkv_j W_j^T (K segments) ; dW_j = xn1^T dqkv_j (N segments)
    gemm(M, C, 3 * C, 1, op(f->dqkv, M, C, C, false, 3, (int64_t)MC, kZKSeg, C),
         op(W(b + 1), C, C, C, false, 3, (int64_t)C * C, kZKSeg, C), kEpiStore, none, rowC, unit,
         f->dxn, Planes{}, nullptr);
    gemm(C, 3 * C, M, 1, op(f->xn1[l], M, C, C, true),
         op(f->dqkv, M, C, C, true, 3, (int64_t)MC, kZMNSeg, C), kEpiStore, none, rowC,
         L(C, (int64_t)C * C, 0, 0, 1), G(b + 1), Planes{}, nullptr);
    ln_bwd(f, f->x[l], f->mean1[l], f->var1[l], P(b), f->dxn, g2, g3, g3p, G(b));
    if (dp_world() > 1) {
      // this layer's gradients are final: reduce them while earlier layers run
      const auto& bk = f->buckets[(size_t)(Lc - 1 - l)];
      if (dp_allreduce_async(f->gbuf + bk.first, bk.second - bk.first) != 0)
        panic("data-parallel all-reduce failed (peer lost or timed out)");
    }
  }
  // embeddings: x0 = wte[tok] + wpe[pos]
  float* dwte = f->cfg.tied ? f->emb_tmp : G(top);
  // a token id outside [0, V) is reported through the runtime's error word,
  // as in __embedding_bwd
  int er;
  {
    KTimer kt("embedding VJP (sort, scan, segmented sum)", 4.0 * ((double)MC + M + (double)V * C));
    er = embedding_bwd_ws(g3, xt, MALUS_I32, dwte, M, V, C, f->emb_ws, stream(), device_error_word());
  }
  if (er != 0) panic("fused step: embedding backward failed (%d)", er);
  if (f->cfg.tied) {
    k_add_inplace<<<grid_for((size_t)V * C, 256), 256, 0, stream()>>>(G(top), f->emb_tmp, (size_t)V * C);
    count_launch();
    after_launch("k_add_inplace");
  }
  {
    KTimer kt("k_dwpe", 4.0 * ((double)MC + (double)T * C));
    k_dwpe<<<grid_for((size_t)T * C, 256), 256, 0, stream()>>>(g3, G(top + 1), B, (size_t)T * C);
    count_launch();
    after_launch("k_dwpe");
  }
  if (dp_world() > 1) {
    const auto& bk = f->buckets.back();
    if (dp_allreduce_async(f->gbuf + bk.first, bk.second - bk.first) != 0)
      panic("data-parallel all-reduce failed (peer lost or timed out)");
    dp_join();
  }
}

// Called after AdamW updates the parameters: refresh the weight planes.
void fused_after_update(FusedStep* f) { split_weights(f); }

namespace {

// One whole training step on the runtime stream: step counter, forward,
// backward (with the data-parallel all-reduces), AdamW, weight re-split.
// Nothing in here allocates or reads the host, so it can be captured.
void fused_body(FusedStep* f, const int32_t* x, const int32_t* y, float* loss) {
  k_step_inc<<<1, 1, 0, stream()>>>(f->step_dev);
  count_launch();
  after_launch("k_step_inc");
  fused_step(f, x, y, loss);
  float gscale = dp_world() > 1 ? 1.0f / (float)dp_world() : 1.0f;
  // AdamW over the whole fused buffer, writing the tf32 planes of every updated
  // parameter (the weight planes share the parameter layout); only the padded
  // untied LM head is re-split separately
  {
    KTimer kt("k_adamw_flat", 4.0 * 9.0 * (double)f->total);   // p, g, m, v in; p, m, v, hi, lo out
    adamw_flat(f->pbuf, f->gbuf, f->mbuf, f->vbuf, (int64_t)f->total, f->cfg.lr, f->cfg.beta1,
               f->cfg.beta2, f->cfg.eps, f->cfg.wd, gscale, f->bc_tab, f->step_dev, f->wpl.hi, f->wpl.lo);
  }
  if (!f->cfg.tied) {
    size_t top = (size_t)f->L * 8;
    tf32_split(f->params[top + 3], f->C, f->V, f->V, 1, 0, f->lmpl.hi, f->lmpl.lo, f->Vp);
  }
}

}  // namespace

// The training step of mode 1.  With cfg.use_graph the first step runs eagerly
// (it sizes the workspaces and sets kernel attributes); the second is captured
// into a CUDA graph that every later step replays.  Kernel timing (prof) and
// synchronous dispatch force the eager path.
void fused_train_step(FusedStep* f, const int32_t* x, const int32_t* y, float* loss) {
  f->host_step++;
  if (f->host_step > f->bc_cap) {
    if (f->exec) {                  // the table moves: the graph must be captured again
      MALUS_CUDA(cudaStreamSynchronize(stream()));
      MALUS_CUDA(cudaGraphExecDestroy(f->exec));
      f->exec = nullptr;
    }
    fill_bc_table(f, f->bc_cap * 4);
  }
  const bool graph = f->cfg.use_graph && !prof_on() && !sync_dispatch() && f->host_step > 1;
  if (!graph) {
    fused_body(f, x, y, loss);
    return;
  }
  if (!f->exec) {
    cudaGraph_t g = nullptr;
    int64_t before = malus_launch_count();
    MALUS_CUDA(cudaStreamBeginCapture(stream(), cudaStreamCaptureModeThreadLocal));
    fused_body(f, x, y, loss);
    MALUS_CUDA(cudaStreamEndCapture(stream(), &g));
    f->graph_launches = malus_launch_count() - before;
    count_launch(-(int)f->graph_launches);     // captured, not launched
    MALUS_CUDA(cudaGraphInstantiate(&f->exec, g, 0));
    MALUS_CUDA(cudaGraphDestroy(g));
  }
  MALUS_CUDA(cudaGraphLaunch(f->exec, stream()));
  count_launch((int)f->graph_launches);
}

}  // namespace malus
