// Row kernels: softmax, layernorm, cross-entropy, embedding and permute.
//
// Reference semantics:
//   softmax      stdlib/softmax.ml:9-28        (max, exp(x-max), sum, divide)
//   softmax VJP  stdlib/backward/transformer_bwd.ml:15-20  s*(dout - sum(dout*s))
//   layernorm    metal.rs:1487-1533 (host twin) / layernorm.ml:8-34 (no affine,
//                population variance, eps 1e-5); the saved variance is per
//                group with keepdim at the axis
//   layernorm VJP tape.rs:1162-1186 (host twin): (1/sigma)(dy - mean(dy) - y*mean(dy*y))
//   cross-entropy cross_entropy.ml:13-28 / metal.rs:1555-1598: probs = softmax,
//                nll = -log(probs[t]), loss = mean(nll)
//   CE VJP       transformer_bwd.ml:57-75: (p - onehot) * dout[0] / N
//   embedding    embedding.ml:11-23 gather; VJP transformer_bwd.ml:83-98
//   permute      permute.ml (materialising N-D permute)
//
// The reference launches one thread per element (or one threadgroup of
// `axis` threads per row, with O(axis^2) work).  Here rows are owned by a warp
// (short rows, held in registers) or a block (long rows), reductions use warp
// shuffles, and every pass is a coalesced stream over HBM.
#include "common.cuh"

#include <unordered_map>

namespace malus {
namespace {

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

// block-wide reduction helpers (blockDim multiple of 32, <= 1024)
__device__ float bsum(float v, float* sh) {
  v = wsum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.0f;
  r = wsum(r);
  return r;
}
__device__ float bmax(float v, float* sh) {
  v = wmax(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = (l < (int)(blockDim.x >> 5)) ? sh[l] : -INFINITY;
  r = wmax(r);
  return r;
}

// ------------------------------------------------------------------ softmax
// The row values a softmax reads: x, or the deferred x * scale[0] + addend
// (addend rows repeat every add_rows rows), rounded like the eager ops.
struct RowSrc {
  const float* x;
  const float* scale;
  const float* add;
  size_t add_rows;
  uint32_t causal_T;   // > 0: elements past row % causal_T are masked (read by k_softmax_rows only)
  __device__ __forceinline__ float at(size_t r, size_t i, size_t len, float sc) const {
    float v = x[r * len + i];
    if (scale) v = __fmul_rn(v, sc);
    if (add) v = __fadd_rn(v, add[(r % add_rows) * len + i]);
    return v;
  }
};

// One warp per contiguous row; the row is kept in registers (<= 32*PER).
template <int PER>
__global__ void k_softmax_warp(RowSrc x, float* __restrict__ y, size_t rows, int len) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  const float sc = x.scale ? *x.scale : 1.0f;
  for (size_t r = warp; r < rows; r += nw) {
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      v[k] = i < len ? x.at(r, i, len, sc) : -INFINITY;
      m = fmaxf(m, v[k]);
    }
    m = wmax(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      v[k] = i < len ? expf(v[k] - m) : 0.0f;
      s += v[k];
    }
    s = wsum(s);
    float* yr = y + r * (size_t)len;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      if (i < len) yr[i] = v[k] / s;
    }
  }
}

// Rows of 128..1024 elements (a multiple of 4, 16-byte aligned sources):
// LPR lanes per row, so a warp works on 32 / LPR rows at once and each lane
// has eight 16-byte loads in flight.  Lane j of a row holds chunks j, j + LPR,
// ... of four elements; max and sum combine the lane's values in chunk order,
// then across the row's lanes by a fixed xor tree; p = e * (1 / sum).  A
// deferred x * s + m reads through RowSrc with the eager roundings, and plain
// and deferred rows take this same kernel, so they give the same bits.
// With CAUSAL and phi (the result's tf32 planes, registered in the operand
// cache for the P V product that follows), each row also writes hi / lo of
// its values up to the end of its 128-row tile's diagonal block, the part that
// the causally clipped GEMMs read.
template <int LPR, bool CAUSAL>
__global__ void __launch_bounds__(256) k_softmax_rows(RowSrc x, float* __restrict__ y, uint32_t rows, int len,
                                                      float* __restrict__ phi, float* __restrict__ plo) {
  constexpr int PER4 = 8, RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, sub = lane % LPR;
  const uint32_t gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  const float sc = x.scale ? *x.scale : 1.0f;
  const int n4 = len >> 2;
  for (uint32_t base = gwarp * RPW; base < rows; base += nwarps * RPW) {
    const uint32_t r = base + (uint32_t)(lane / LPR);
    const bool live = r < rows;
    const float4* xr = reinterpret_cast<const float4*>(x.x + (size_t)r * len);
    const float4* ar = x.add ? reinterpret_cast<const float4*>(x.add + (size_t)(r % (uint32_t)x.add_rows) * len) : nullptr;
    // chunks wholly past the diagonal of a causal mask: exp gives exactly 0 there
    const uint32_t last = CAUSAL ? r % x.causal_T : 0xffffffffu;
    float4 v[PER4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      const int c = sub + LPR * k;
      if (live && c < n4 && (!CAUSAL || (uint32_t)(4 * c) <= last)) {
        float4 t = xr[c];
        if (x.scale) { t.x = __fmul_rn(t.x, sc); t.y = __fmul_rn(t.y, sc); t.z = __fmul_rn(t.z, sc); t.w = __fmul_rn(t.w, sc); }
        if (ar) {
          const float4 a = ar[c];
          t.x = __fadd_rn(t.x, a.x); t.y = __fadd_rn(t.y, a.y); t.z = __fadd_rn(t.z, a.z); t.w = __fadd_rn(t.w, a.w);
        }
        v[k] = t;
        m = fmaxf(m, fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)));
      } else {
        v[k] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      const int c = sub + LPR * k;
      if (live && c < n4 && (!CAUSAL || (uint32_t)(4 * c) <= last)) {
        v[k].x = expf(v[k].x - m); v[k].y = expf(v[k].y - m); v[k].z = expf(v[k].z - m); v[k].w = expf(v[k].w - m);
        sum += v[k].x; sum += v[k].y; sum += v[k].z; sum += v[k].w;
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    float4* yr = reinterpret_cast<float4*>(y + (size_t)r * len);
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      const int c = sub + LPR * k;
      if (live && c < n4) {
        const float4 pv = !CAUSAL || (uint32_t)(4 * c) <= last
                              ? make_float4(v[k].x * inv, v[k].y * inv, v[k].z * inv, v[k].w * inv)
                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        yr[c] = pv;
        if (CAUSAL && phi && (uint32_t)(4 * c) < ((last >> 7) + 1) * 128) {
          const float4 h = make_float4(tf32_round(pv.x), tf32_round(pv.y), tf32_round(pv.z), tf32_round(pv.w));
          const size_t at = (size_t)r * (len >> 2) + c;
          reinterpret_cast<float4*>(phi)[at] = h;
          reinterpret_cast<float4*>(plo)[at] = make_float4(tf32_round(pv.x - h.x), tf32_round(pv.y - h.y),
                                                           tf32_round(pv.z - h.z), tf32_round(pv.w - h.w));
        }
      }
    }
  }
}

// Blocks of 256 threads that stay resident together: the SM count times what
// the occupancy calculator allows for `kern` (once per kernel), at most `need`.
template <typename K>
unsigned resident_blocks(K kern, size_t need) {
  static std::unordered_map<const void*, int> per_sm;
  int& n = per_sm[(const void*)kern];
  if (!n) {
    MALUS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 256, 0));
    if (n < 1) n = 1;
  }
  return (unsigned)std::max<size_t>(1, std::min<size_t>(need, (size_t)kNumSMs * n));
}

// Long rows: one block per row, three passes (max, sum, write).
__global__ void k_softmax_block(RowSrc x, float* __restrict__ y, size_t rows, size_t len) {
  __shared__ float sh[32];
  const float sc = x.scale ? *x.scale : 1.0f;
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float m = -INFINITY;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) m = fmaxf(m, x.at(r, i, len, sc));
    m = bmax(m, sh);
    float s = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) s += expf(x.at(r, i, len, sc) - m);
    s = bsum(s, sh);
    float* yr = y + r * len;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) yr[i] = expf(x.at(r, i, len, sc) - m) / s;
    __syncthreads();
  }
}

// Strided softmax (axis not innermost): thread per (outer, inner) group.
__global__ void k_softmax_strided(const float* __restrict__ x, float* __restrict__ y, size_t outer,
                                  size_t axis_sz, size_t inner) {
  size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (g >= outer * inner) return;
  size_t o = g / inner, i = g % inner;
  const float* b = x + o * axis_sz * inner + i;
  float* yb = y + o * axis_sz * inner + i;
  float m = -INFINITY;
  for (size_t a = 0; a < axis_sz; ++a) m = fmaxf(m, b[a * inner]);
  float s = 0.0f;
  for (size_t a = 0; a < axis_sz; ++a) s += expf(b[a * inner] - m);
  for (size_t a = 0; a < axis_sz; ++a) yb[a * inner] = expf(b[a * inner] - m) / s;
}

// causal_T > 0: s is zero past column r % causal_T of row r; those terms add
// (signed) zeros to the dot product and give zero gradients, so they are not read.
template <int PER>
__global__ void k_softmax_bwd_warp(const float* __restrict__ s, const float* __restrict__ g,
                                   float* __restrict__ dx, size_t rows, int len, int causal_T) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t r = warp; r < rows; r += nw) {
    const float* sr = s + r * (size_t)len;
    const float* gr = g + r * (size_t)len;
    const int last = causal_T ? (int)(r % (size_t)causal_T) : len;
    float sv[PER], gv[PER];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      const bool rd = i < len && i <= last;
      sv[k] = rd ? sr[i] : 0.0f;
      gv[k] = rd ? gr[i] : 0.0f;
      dot += gv[k] * sv[k];
    }
    dot = wsum(dot);
    float* dr = dx + r * (size_t)len;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      if (i < len) dr[i] = i <= last ? sv[k] * (gv[k] - dot) : 0.0f;
    }
  }
}

__global__ void k_softmax_bwd_block(const float* __restrict__ s, const float* __restrict__ g,
                                    float* __restrict__ dx, size_t rows, size_t len) {
  __shared__ float sh[32];
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* sr = s + r * len;
    const float* gr = g + r * len;
    float dot = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) dot += gr[i] * sr[i];
    dot = bsum(dot, sh);
    float* dr = dx + r * len;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) dr[i] = sr[i] * (gr[i] - dot);
    __syncthreads();
  }
}

__global__ void k_softmax_bwd_strided(const float* __restrict__ s, const float* __restrict__ g,
                                      float* __restrict__ dx, size_t outer, size_t axis_sz,
                                      size_t inner) {
  size_t gi = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (gi >= outer * inner) return;
  size_t o = gi / inner, i = gi % inner;
  size_t base = o * axis_sz * inner + i;
  float dot = 0.0f;
  for (size_t a = 0; a < axis_sz; ++a) dot += g[base + a * inner] * s[base + a * inner];
  for (size_t a = 0; a < axis_sz; ++a) {
    size_t k = base + a * inner;
    dx[k] = s[k] * (g[k] - dot);
  }
}

// ---------------------------------------------------------------- layernorm
template <int PER>
__global__ void k_layernorm_warp(const float* __restrict__ x, float* __restrict__ y,
                                 float* __restrict__ var_out, size_t rows, int len, float eps) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t r = warp; r < rows; r += nw) {
    const float* xr = x + r * (size_t)len;
    float v[PER];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      v[k] = i < len ? xr[i] : 0.0f;
      s += v[k];
    }
    float mean = wsum(s) / (float)len;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      float d = i < len ? v[k] - mean : 0.0f;
      q += d * d;
    }
    float var = wsum(q) / (float)len;
    float sigma = sqrtf(var + eps);
    float* yr = y + r * (size_t)len;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      if (i < len) yr[i] = (v[k] - mean) / sigma;
    }
    if (lane == 0 && var_out) var_out[r] = var;
  }
}

// The same with 16-byte accesses (rows of a multiple of 4 elements, 16-byte
// aligned; lane l holds chunks l, l + 32, ...).
template <int PER4>
__global__ void k_layernorm_warp4(const float* __restrict__ x, float* __restrict__ y,
                                  float* __restrict__ var_out, size_t rows, int len, float eps) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int n4 = len >> 2;
  for (size_t r = warp; r < rows; r += nw) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * (size_t)len);
    float4 v[PER4];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      const int c = lane + 32 * k;
      v[k] = c < n4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      s += v[k].x; s += v[k].y; s += v[k].z; s += v[k].w;
    }
    float mean = wsum(s) / (float)len;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      if (lane + 32 * k < n4) {
        float d0 = v[k].x - mean, d1 = v[k].y - mean, d2 = v[k].z - mean, d3 = v[k].w - mean;
        q += d0 * d0; q += d1 * d1; q += d2 * d2; q += d3 * d3;
      }
    }
    float var = wsum(q) / (float)len;
    float sigma = sqrtf(var + eps);
    float4* yr = reinterpret_cast<float4*>(y + r * (size_t)len);
#pragma unroll
    for (int k = 0; k < PER4; ++k) {
      const int c = lane + 32 * k;
      if (c < n4)
        yr[c] = make_float4((v[k].x - mean) / sigma, (v[k].y - mean) / sigma, (v[k].z - mean) / sigma,
                            (v[k].w - mean) / sigma);
    }
    if (lane == 0 && var_out) var_out[r] = var;
  }
}

__global__ void k_layernorm_block(const float* __restrict__ x, float* __restrict__ y,
                                  float* __restrict__ var_out, size_t rows, size_t len, float eps) {
  __shared__ float sh[32];
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * len;
    float s = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) s += xr[i];
    float mean = bsum(s, sh) / (float)len;
    float q = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
      float d = xr[i] - mean;
      q += d * d;
    }
    float var = bsum(q, sh) / (float)len;
    float sigma = sqrtf(var + eps);
    float* yr = y + r * len;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) yr[i] = (xr[i] - mean) / sigma;
    if (threadIdx.x == 0 && var_out) var_out[r] = var;
    __syncthreads();
  }
}

__global__ void k_layernorm_strided(const float* __restrict__ x, float* __restrict__ y,
                                    float* __restrict__ var_out, size_t outer, size_t axis_sz,
                                    size_t inner, float eps) {
  size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (g >= outer * inner) return;
  size_t o = g / inner, i = g % inner;
  size_t base = o * axis_sz * inner + i;
  float s = 0.0f;
  for (size_t a = 0; a < axis_sz; ++a) s += x[base + a * inner];
  float mean = s / (float)axis_sz;
  float q = 0.0f;
  for (size_t a = 0; a < axis_sz; ++a) {
    float d = x[base + a * inner] - mean;
    q += d * d;
  }
  float var = q / (float)axis_sz;
  float sigma = sqrtf(var + eps);
  for (size_t a = 0; a < axis_sz; ++a) y[base + a * inner] = (x[base + a * inner] - mean) / sigma;
  if (var_out) var_out[g] = var;
}

// gs (optional): the incoming gradient is read as g[i] * gs[i] (the deferred
// gain VJP), rounded like the eager multiply.  The choice is a template
// parameter so that each variant issues its row loads as one straight run.
template <int PER, bool SCALED>
__device__ __forceinline__ void ln_bwd_warp_rows(const float* __restrict__ y, const float* __restrict__ var,
                                                 const float* __restrict__ g, float* __restrict__ dx,
                                                 size_t rows, int len, float eps, const float* __restrict__ gs) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t r = warp; r < rows; r += nw) {
    const float* yr = y + r * (size_t)len;
    const float* gr = g + r * (size_t)len;
    float yv[PER], gv[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      yv[k] = i < len ? yr[i] : 0.0f;
      gv[k] = i < len ? gr[i] : 0.0f;
    }
    if (SCALED) {
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        int i = lane + 32 * k;
        if (i < len) gv[k] = __fmul_rn(gv[k], gs[i]);
      }
    }
    float sg = 0.0f, sgy = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      sg += gv[k];
      sgy += gv[k] * yv[k];
    }
    float mg = wsum(sg) / (float)len;
    float mgy = wsum(sgy) / (float)len;
    float inv = 1.0f / sqrtf(var[r] + eps);
    float* dr = dx + r * (size_t)len;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      if (i < len) dr[i] = ((gv[k] - mg) - yv[k] * mgy) * inv;
    }
  }
}

template <int PER>
__global__ void k_layernorm_bwd_warp(const float* __restrict__ y, const float* __restrict__ var,
                                     const float* __restrict__ g, float* __restrict__ dx,
                                     size_t rows, int len, float eps, const float* __restrict__ gs) {
  if (gs) ln_bwd_warp_rows<PER, true>(y, var, g, dx, rows, len, eps, gs);
  else ln_bwd_warp_rows<PER, false>(y, var, g, dx, rows, len, eps, nullptr);
}

__global__ void k_layernorm_bwd_block(const float* __restrict__ y, const float* __restrict__ var,
                                      const float* __restrict__ g, float* __restrict__ dx,
                                      size_t rows, size_t len, float eps, const float* __restrict__ gs) {
  __shared__ float sh[32];
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* yr = y + r * len;
    const float* gr = g + r * len;
    auto gat = [&](size_t i) { return gs ? __fmul_rn(gr[i], gs[i]) : gr[i]; };
    float sg = 0.0f, sgy = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
      const float gv = gat(i);
      sg += gv;
      sgy += gv * yr[i];
    }
    float mg = bsum(sg, sh) / (float)len;
    float mgy = bsum(sgy, sh) / (float)len;
    float inv = 1.0f / sqrtf(var[r] + eps);
    float* dr = dx + r * len;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x)
      dr[i] = ((gat(i) - mg) - yr[i] * mgy) * inv;
    __syncthreads();
  }
}

__global__ void k_layernorm_bwd_strided(const float* __restrict__ y, const float* __restrict__ var,
                                        const float* __restrict__ g, float* __restrict__ dx,
                                        size_t outer, size_t axis_sz, size_t inner, float eps) {
  size_t gi = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (gi >= outer * inner) return;
  size_t o = gi / inner, i = gi % inner;
  size_t base = o * axis_sz * inner + i;
  float sg = 0.0f, sgy = 0.0f;
  for (size_t a = 0; a < axis_sz; ++a) {
    size_t k = base + a * inner;
    sg += g[k];
    sgy += g[k] * y[k];
  }
  float mg = sg / (float)axis_sz, mgy = sgy / (float)axis_sz;
  float inv = 1.0f / sqrtf(var[gi] + eps);
  for (size_t a = 0; a < axis_sz; ++a) {
    size_t k = base + a * inner;
    dx[k] = ((g[k] - mg) - y[k] * mgy) * inv;
  }
}

// ------------------------------------------------------------ cross-entropy
__device__ __forceinline__ int64_t load_index(const void* p, int dtype, size_t i) {
  return dtype == MALUS_I64 ? ((const int64_t*)p)[i] : (int64_t)((const int32_t*)p)[i];
}

template <int PER>
// part[blockIdx.x]: this block's sum of nll (each warp adds its rows in row
// order, the block adds its warps in warp order: a fixed order for a given grid)
__global__ void k_xent_fwd_warp(const float* __restrict__ logits, const void* __restrict__ tgt,
                                int tdt, float* __restrict__ probs, float* __restrict__ part,
                                size_t rows, int V, int32_t* err) {
  __shared__ float wpart[32];
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  float wacc = 0.0f;
  for (size_t r = warp; r < rows; r += nw) {
    const float* xr = logits + r * (size_t)V;
    const int64_t t = load_index(tgt, tdt, r);   // issued with the row's loads, used after the reductions
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      v[k] = i < V ? xr[i] : -INFINITY;
      m = fmaxf(m, v[k]);
    }
    m = wmax(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      v[k] = i < V ? expf(v[k] - m) : 0.0f;
      s += v[k];
    }
    s = wsum(s);
    bool bad = t < 0 || t >= V;
    float pt = 0.0f;
    float* pr = probs + r * (size_t)V;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = lane + 32 * k;
      if (i < V) {
        float p = v[k] / s;
        pr[i] = p;
        if (i == t) pt = p;
      }
    }
    pt = wsum(pt);
    if (lane == 0) {
      if (bad) atomicExch(err, 3);
      else wacc += -logf(pt);
    }
  }
  if (lane == 0) wpart[threadIdx.x >> 5] = wacc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b += wpart[w];
    part[blockIdx.x] = b;
  }
}

// Short rows (V <= 12 * LPR): LPR lanes per row, 32 / LPR rows per warp at
// once (k_xent_fwd_warp keeps one row per warp and leaves most of each row's
// latency exposed).  Lane j of a row holds elements j, j + LPR, ...; max, sum
// and the target's probability combine across the row's lanes by a fixed xor
// tree; each row group's first lane adds its rows' -log p in row order, and a
// block's partial is its warps' group sums in a fixed order.
template <int LPR>
__global__ void k_xent_fwd_rows(const float* __restrict__ logits, const void* __restrict__ tgt,
                                int tdt, float* __restrict__ probs, float* __restrict__ part,
                                size_t rows, int V, int32_t* err) {
  constexpr int PER = 12, RPW = 32 / LPR;
  __shared__ float wpart[32];
  const int lane = threadIdx.x & 31, sub = lane % LPR, grp = lane / LPR;
  const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  float wacc = 0.0f;
  for (size_t base = warp * RPW; base < rows; base += nw * RPW) {
    const size_t r = base + (size_t)grp;
    const bool live = r < rows;
    const float* xr = logits + r * (size_t)V;
    const int64_t t = live ? load_index(tgt, tdt, r) : 0;   // issued with the row's loads
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = sub + LPR * k;
      v[k] = live && i < V ? xr[i] : -INFINITY;
      m = fmaxf(m, v[k]);
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = sub + LPR * k;
      v[k] = live && i < V ? expf(v[k] - m) : 0.0f;
      s += v[k];
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float pt = 0.0f;
    float* pr = probs + r * (size_t)V;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = sub + LPR * k;
      if (live && i < V) {
        const float pv = v[k] / s;
        pr[i] = pv;
        if (i == t) pt = pv;
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) pt += __shfl_xor_sync(0xffffffffu, pt, o);
    if (sub == 0 && live) {
      if (t < 0 || t >= V) atomicExch(err, 3);
      else wacc += -logf(pt);
    }
  }
  float w = 0.0f;
#pragma unroll
  for (int g = 0; g < RPW; ++g) w += __shfl_sync(0xffffffffu, wacc, g * LPR);
  if (lane == 0) wpart[threadIdx.x >> 5] = w;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) b += wpart[i];
    part[blockIdx.x] = b;
  }
}

__global__ void k_xent_fwd_block(const float* __restrict__ logits, const void* __restrict__ tgt,
                                 int tdt, float* __restrict__ probs, float* __restrict__ part,
                                 size_t rows, size_t V, int32_t* err) {
  __shared__ float sh[32];
  __shared__ float pt_sh;
  float bacc = 0.0f;   // thread 0: this block's rows' nll in row order
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * V;
    float m = -INFINITY;
    for (size_t i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, xr[i]);
    m = bmax(m, sh);
    float s = 0.0f;
    for (size_t i = threadIdx.x; i < V; i += blockDim.x) s += expf(xr[i] - m);
    s = bsum(s, sh);
    int64_t t = load_index(tgt, tdt, r);
    bool bad = t < 0 || (size_t)t >= V;
    float* pr = probs + r * V;
    for (size_t i = threadIdx.x; i < V; i += blockDim.x) {
      float p = expf(xr[i] - m) / s;
      pr[i] = p;
      if ((int64_t)i == t) pt_sh = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      if (bad) atomicExch(err, 3);
      else bacc += -logf(pt_sh);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = bacc;
}

// out[0] = (sum of the n partials, in a fixed order) / rows
__global__ void k_mean_partials(const float* __restrict__ part, int n, float* __restrict__ out, size_t rows) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += 32) s += part[i];
  s = wsum(s);
  if (threadIdx.x == 0) out[0] = s / (float)rows;
}

// cross_entropy.ml:13-16: out[i] = -log(probs[i*V + t_i])
__global__ void k_xent_nll_gather(const float* __restrict__ probs, const void* __restrict__ tgt,
                                  int tdt, float* __restrict__ out, size_t n, size_t V,
                                  int32_t* err) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  int64_t t = load_index(tgt, tdt, i);
  if (t < 0 || (size_t)t >= V) { atomicExch(err, 3); out[i] = 0.0f; return; }
  out[i] = -logf(probs[i * V + (size_t)t]);
}

// dx = (p - onehot(t)) * scale, scale = dout[0] / rows (the tape's VJP) or a
// host value (the stdlib kernel's uniform, transformer_bwd.ml:56-75).  With
// 32-bit flat indices and aligned buffers each thread handles four
// consecutive elements (one float4), walking row boundaries incrementally
// instead of dividing per element.
__global__ void k_xent_bwd(const float* __restrict__ probs, const void* __restrict__ tgt, int tdt,
                           const float* __restrict__ dout, float hscale, float* __restrict__ dx,
                           size_t rows, size_t V, bool vec) {
  const float scale = dout ? dout[0] / (float)rows : hscale;
  const size_t n = rows * V;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    const uint32_t n4 = (uint32_t)(n / 4), V32 = (uint32_t)V;
    for (uint32_t q = (uint32_t)tid; q < n4; q += (uint32_t)stride) {
      const float4 p = reinterpret_cast<const float4*>(probs)[q];
      float r[4] = {p.x, p.y, p.z, p.w};
      uint32_t i = (q * 4) / V32, j = q * 4 - i * V32;
      int64_t t = load_index(tgt, tdt, i);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j == V32) { ++i; j = 0; t = load_index(tgt, tdt, i); }
        float g = r[u];
        if ((int64_t)j == t) g = g - 1.0f;
        r[u] = g * scale;
        ++j;
      }
      reinterpret_cast<float4*>(dx)[q] = make_float4(r[0], r[1], r[2], r[3]);
    }
    for (size_t f = (size_t)n4 * 4 + tid; f < n; f += stride) {
      size_t i = f / V, j = f - i * V;
      float g = probs[f];
      if ((int64_t)j == load_index(tgt, tdt, i)) g = g - 1.0f;
      dx[f] = g * scale;
    }
    return;
  }
  for (size_t f = tid; f < n; f += stride) {
    size_t i = f / V, j = f - i * V;
    float g = probs[f];
    if ((int64_t)j == load_index(tgt, tdt, i)) g = g - 1.0f;
    dx[f] = g * scale;
  }
}

// ---------------------------------------------------------------- embedding
// out[t, :] = w[idx[t], :]  — one warp per row, 16-byte copies when aligned.
__global__ void k_embedding_fwd(const float* __restrict__ w, const void* __restrict__ idx, int idt,
                                float* __restrict__ out, size_t n, size_t V, size_t D,
                                int32_t* err) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  bool vec = (D % 4 == 0) && (((uintptr_t)w & 15) == 0) && (((uintptr_t)out & 15) == 0);
  for (size_t t = warp; t < n; t += nw) {
    int64_t row = load_index(idx, idt, t);
    float* o = out + t * D;
    if (row < 0 || (size_t)row >= V) {
      if (lane == 0) atomicExch(err, 4);
      for (size_t c = lane; c < D; c += 32) o[c] = 0.0f;
      continue;
    }
    const float* src = w + (size_t)row * D;
    if (vec) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* o4 = reinterpret_cast<float4*>(o);
      for (size_t c = lane; c < D / 4; c += 32) o4[c] = s4[c];
    } else {
      for (size_t c = lane; c < D; c += 32) o[c] = src[c];
    }
  }
}

// Embedding VJP, deterministic sort-then-segmented-sum.
// K1: each block sorts a chunk of CH token keys (id<<32 | t) in shared memory
//     (bitonic), stores them, and writes the run length of each id present in
//     the chunk to counts[id * nch + chunk].
constexpr int kEmbChunk = 1024;

__global__ void k_emb_chunk_sort(const void* __restrict__ idx, int idt, size_t n, size_t V,
                                 int nch, unsigned long long* __restrict__ keys,
                                 int* __restrict__ counts, int32_t* err) {
  __shared__ unsigned long long sk[kEmbChunk];
  int c = blockIdx.x;
  size_t base = (size_t)c * kEmbChunk;
  for (int j = threadIdx.x; j < kEmbChunk; j += blockDim.x) {
    size_t t = base + j;
    unsigned long long key = ~0ull;
    if (t < n) {
      int64_t id = load_index(idx, idt, t);
      if (id < 0 || (size_t)id >= V) atomicExch(err, 4);
      else key = ((unsigned long long)id << 32) | (unsigned long long)(uint32_t)t;
    }
    sk[j] = key;
  }
  __syncthreads();
  for (int k = 2; k <= kEmbChunk; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < kEmbChunk; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          unsigned long long a = sk[i], b = sk[ixj];
          bool up = (i & k) == 0;
          if ((a > b) == up) { sk[i] = b; sk[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
  for (int j = threadIdx.x; j < kEmbChunk; j += blockDim.x) {
    unsigned long long key = sk[j];
    keys[base + j] = key;
    if (key == ~0ull) continue;
    uint32_t id = (uint32_t)(key >> 32);
    bool start = j == 0 || (uint32_t)(sk[j - 1] >> 32) != id;
    if (start) {
      int lo = j, hi = kEmbChunk;  // first index with id' > id
      while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (sk[mid] != ~0ull && (uint32_t)(sk[mid] >> 32) <= id) lo = mid + 1;
        else hi = mid;
      }
      counts[(size_t)id * nch + c] = lo - j;
    }
  }
}

// K2: exclusive scan of counts (length m) -> offs (length m+1); 3 phases.
constexpr int kScanTile = 4096;
__global__ void k_scan_tile_sums(const int* __restrict__ in, size_t m, int* __restrict__ sums) {
  __shared__ float sh[32];
  size_t base = (size_t)blockIdx.x * kScanTile;
  int s = 0;
  for (int j = threadIdx.x; j < kScanTile; j += blockDim.x) {
    size_t k = base + j;
    if (k < m) s += in[k];
  }
  // integer block sum via float-free path
  __shared__ int shi[32];
  (void)sh;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) shi[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = threadIdx.x < (blockDim.x >> 5) ? shi[threadIdx.x] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) sums[blockIdx.x] = v;
  }
}

__global__ void k_scan_sums_serial(int* __restrict__ sums, int nt, int* __restrict__ total_out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < nt; ++i) { int v = sums[i]; sums[i] = run; run += v; }
    *total_out = run;
  }
}

__global__ void k_scan_tile_apply(const int* __restrict__ in, size_t m, const int* __restrict__ sums,
                                  int* __restrict__ out) {
  // each block scans its tile: 1024 threads x 4 items
  __shared__ int warp_tot[32];
  size_t base = (size_t)blockIdx.x * kScanTile;
  int t = threadIdx.x;
  int v[4];
  int local = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    size_t k = base + (size_t)t * 4 + q;
    v[q] = k < m ? in[k] : 0;
    local += v[q];
  }
  int lane = t & 31, w = t >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    int x = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
    int xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += y;
    }
    warp_tot[lane] = xi - x;  // exclusive
  }
  __syncthreads();
  int run = sums[blockIdx.x] + warp_tot[w] + (incl - local);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    size_t k = base + (size_t)t * 4 + q;
    if (k < m) out[k] = run;
    run += v[q];
  }
}

// K3: place each chunk's sorted tokens at their global positions.
__global__ void k_emb_scatter(const unsigned long long* __restrict__ keys, size_t n, int nch,
                              const int* __restrict__ offs, int* __restrict__ order) {
  __shared__ unsigned long long sk[kEmbChunk];
  int c = blockIdx.x;
  size_t base = (size_t)c * kEmbChunk;
  for (int j = threadIdx.x; j < kEmbChunk; j += blockDim.x) sk[j] = keys[base + j];
  __syncthreads();
  for (int j = threadIdx.x; j < kEmbChunk; j += blockDim.x) {
    unsigned long long key = sk[j];
    if (key == ~0ull) continue;
    uint32_t id = (uint32_t)(key >> 32);
    int lo = 0, hi = j;  // first index with id' >= id
    while (lo < hi) {
      int mid = (lo + hi) >> 1;
      if ((uint32_t)(sk[mid] >> 32) < id) lo = mid + 1;
      else hi = mid;
    }
    order[offs[(size_t)id * nch + c] + (j - lo)] = (int)(uint32_t)key;
  }
}

// K4: dw[v, :] = sum over the run of v (token order) of dout[t, :].
// One thread per column of one vocabulary row, so every output element is a
// single chain of additions in token order (the order of the reference's
// per-row gather, embedding_bwd.ml via transformer_bwd.ml:83-98).  The run's
// token indices are staged in shared memory kSegIdx at a time; each thread
// loads the next kSegPipe rows while it adds the current ones (two register
// buffers), so the chains, which are few (vocab x dim), keep memory busy.
constexpr int kSegIdx = 1024;
constexpr int kSegPipe = 16;
constexpr int kSegThreads = 128;
__global__ void __launch_bounds__(kSegThreads)
k_emb_segsum(const float* __restrict__ dout, const int* __restrict__ order, const int* __restrict__ offs,
             int nch, size_t V, size_t D, float* __restrict__ dw) {
  __shared__ int sidx[kSegIdx];
  const size_t v = blockIdx.x;
  const size_t d = blockIdx.y * (size_t)blockDim.x + threadIdx.x;
  const int beg = offs[v * nch], end = offs[(v + 1) * nch];
  const float* col = dout + (d < D ? d : 0);
  float acc = 0.0f;
  for (int k0 = beg; k0 < end; k0 += kSegIdx) {
    const int cnt = min(kSegIdx, end - k0);
    __syncthreads();
    for (int j = threadIdx.x; j < cnt; j += blockDim.x) sidx[j] = order[k0 + j];
    __syncthreads();
    if (d >= D) continue;
    const int full = cnt / kSegPipe;   // whole batches
    float xa[kSegPipe], xb[kSegPipe];
    if (full > 0) {
#pragma unroll
      for (int u = 0; u < kSegPipe; ++u) xa[u] = col[(size_t)sidx[u] * D];
    }
    for (int b = 0; b < full; ++b) {
      const bool more = b + 1 < full;
      if (more) {
#pragma unroll
        for (int u = 0; u < kSegPipe; ++u) xb[u] = col[(size_t)sidx[(b + 1) * kSegPipe + u] * D];
      }
#pragma unroll
      for (int u = 0; u < kSegPipe; ++u) acc += xa[u];
      if (more) {
#pragma unroll
        for (int u = 0; u < kSegPipe; ++u) xa[u] = xb[u];
      }
    }
    for (int j = full * kSegPipe; j < cnt; ++j) acc += col[(size_t)sidx[j] * D];
  }
  if (d < D) dw[v * D + d] = acc;
}

// ------------------------------------------------------------------ permute
struct PermMeta {
  int ndim;
  int64_t out_shape[kMaxRank];
  int64_t in_stride_for_out_dim[kMaxRank];  // input stride of the input dim perm[d]
};

// Innermost dim preserved: copy contiguous rows of length L (warp per row).
__global__ void k_permute_rows(const float* __restrict__ x, float* __restrict__ out, size_t nrows,
                               size_t L, PermMeta m) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nw = ((size_t)gridDim.x * blockDim.x) >> 5;
  bool vec = (L % 4 == 0) && (((uintptr_t)x & 15) == 0) && (((uintptr_t)out & 15) == 0);
  for (size_t r = warp; r < nrows; r += nw) {
    size_t rem = r;
    int64_t src = 0;
    for (int d = m.ndim - 2; d >= 0; --d) {
      int64_t i = (int64_t)(rem % (size_t)m.out_shape[d]);
      rem /= (size_t)m.out_shape[d];
      src += i * m.in_stride_for_out_dim[d];
    }
    const float* s = x + src;
    float* o = out + r * L;
    if (vec) {
      for (size_t c = lane; c < L / 4; c += 32)
        reinterpret_cast<float4*>(o)[c] = reinterpret_cast<const float4*>(s)[c];
    } else {
      for (size_t c = lane; c < L; c += 32) o[c] = s[c];
    }
  }
}

// Batched transpose of the last two dims: in [B, R, C] -> out [B, C, R].
__global__ void k_transpose_tiled(const float* __restrict__ x, float* __restrict__ out, size_t R,
                                  size_t C) {
  __shared__ float tile[32][33];
  size_t b = blockIdx.z;
  size_t r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* xb = x + b * R * C;
  float* ob = out + b * R * C;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    size_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[k][threadIdx.x] = xb[r * C + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    size_t c = c0 + k, r = r0 + threadIdx.x;
    if (r < R && c < C) ob[c * R + r] = tile[threadIdx.x][k];
  }
}

__global__ void k_permute_general(const float* __restrict__ x, float* __restrict__ out, size_t n,
                                  PermMeta m) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t f = tid; f < n; f += stride) {
    size_t rem = f;
    int64_t src = 0;
    for (int d = m.ndim - 1; d >= 0; --d) {
      int64_t i = (int64_t)(rem % (size_t)m.out_shape[d]);
      rem /= (size_t)m.out_shape[d];
      src += i * m.in_stride_for_out_dim[d];
    }
    out[f] = x[src];
  }
}

}  // namespace

#define LAUNCH_ROWS_WARP(KERN, LEN, ROWS, ...)                                   \
  do {                                                                           \
    unsigned blocks_ = grid_for((ROWS) * 32, 256);                               \
    if ((LEN) <= 32) KERN<1><<<blocks_, 256, 0, stream()>>>(__VA_ARGS__);        \
    else if ((LEN) <= 128) KERN<4><<<blocks_, 256, 0, stream()>>>(__VA_ARGS__);  \
    else if ((LEN) <= 256) KERN<8><<<blocks_, 256, 0, stream()>>>(__VA_ARGS__);  \
    else if ((LEN) <= 512) KERN<16><<<blocks_, 256, 0, stream()>>>(__VA_ARGS__); \
    else KERN<32><<<blocks_, 256, 0, stream()>>>(__VA_ARGS__);                   \
    count_launch();                                                              \
    after_launch(#KERN);                                                         \
  } while (0)

static unsigned row_blocks(size_t rows) {
  return (unsigned)std::max<size_t>(1, std::min<size_t>(rows, (size_t)kNumSMs * 8));
}

bool softmax_rows_path(const float* x, const float* y, const float* addend, size_t outer, size_t axis_sz,
                       size_t inner) {
  const bool vec4 = axis_sz % 4 == 0 && ((((uintptr_t)x) | ((uintptr_t)y) | ((uintptr_t)addend)) & 15) == 0;
  return inner == 1 && axis_sz <= 1024 && vec4 && axis_sz >= 128 && outer < ((size_t)1 << 31);
}

void softmax_fwd(const float* x, float* y, size_t outer, size_t axis_sz, size_t inner,
                 const float* scale, const float* addend, size_t add_rows, int causal_T, float* p_hi,
                 float* p_lo) {
  if (!outer || !axis_sz || !inner) return;
  if (p_hi && (!causal_T || !p_lo || !softmax_rows_path(x, y, addend, outer, axis_sz, inner)))
    panic("softmax_fwd: planes are written only by the row kernel over a causal mask");
  if ((scale || addend) && inner != 1) panic("softmax_fwd: a deferred input needs the last axis");
  if (causal_T && (!addend || inner != 1 || (size_t)causal_T != axis_sz))
    panic("softmax_fwd: causal skipping needs the [T, T] mask as the addend");
  const RowSrc src{x, scale, addend, std::max<size_t>(add_rows, 1), (uint32_t)causal_T};
  // 16-byte rows whenever the row and every source are 16-byte aligned: a
  // deferred x * s + m must take the same kernel as its materialised value
  // (the row sum's grouping follows the kernel), so both give the same bits
  if (softmax_rows_path(x, y, addend, outer, axis_sz, inner)) {
    const uint32_t rows = (uint32_t)outer;
    const int len = (int)axis_sz;
    auto go = [&](auto kern, int rpw) {
      kern<<<resident_blocks(kern, (outer + 8 * rpw - 1) / (8 * rpw)), 256, 0, stream()>>>(src, y, rows, len,
                                                                                          p_hi, p_lo);
    };
    // the causal variant skips the chunks past the diagonal; its results are
    // those of the plain one (the skipped terms are exact zeros)
    if (causal_T) {
      if (axis_sz <= 128) go(k_softmax_rows<4, true>, 8);
      else if (axis_sz <= 256) go(k_softmax_rows<8, true>, 4);
      else if (axis_sz <= 512) go(k_softmax_rows<16, true>, 2);
      else go(k_softmax_rows<32, true>, 1);
    } else {
      if (axis_sz <= 128) go(k_softmax_rows<4, false>, 8);
      else if (axis_sz <= 256) go(k_softmax_rows<8, false>, 4);
      else if (axis_sz <= 512) go(k_softmax_rows<16, false>, 2);
      else go(k_softmax_rows<32, false>, 1);
    }
    count_launch();
    after_launch("k_softmax_rows");
  } else if (inner == 1 && axis_sz <= 1024) {
    LAUNCH_ROWS_WARP(k_softmax_warp, axis_sz, outer, src, y, outer, (int)axis_sz);
  } else if (inner == 1) {
    k_softmax_block<<<row_blocks(outer), 512, 0, stream()>>>(src, y, outer, axis_sz);
    count_launch();
    after_launch("k_softmax_block");
  } else {
    size_t g = outer * inner;
    k_softmax_strided<<<(unsigned)((g + 255) / 256), 256, 0, stream()>>>(x, y, outer, axis_sz, inner);
    count_launch();
    after_launch("k_softmax_strided");
  }
}

void softmax_bwd(const float* s, const float* g, float* dx, size_t outer, size_t axis_sz,
                 size_t inner, int causal_T) {
  if (!outer || !axis_sz || !inner) return;
  if (inner == 1 && axis_sz <= 1024) {
    LAUNCH_ROWS_WARP(k_softmax_bwd_warp, axis_sz, outer, s, g, dx, outer, (int)axis_sz, causal_T);
  } else if (inner == 1) {
    k_softmax_bwd_block<<<row_blocks(outer), 512, 0, stream()>>>(s, g, dx, outer, axis_sz);
    count_launch();
    after_launch("k_softmax_bwd_block");
  } else {
    size_t gg = outer * inner;
    k_softmax_bwd_strided<<<(unsigned)((gg + 255) / 256), 256, 0, stream()>>>(s, g, dx, outer,
                                                                             axis_sz, inner);
    count_launch();
    after_launch("k_softmax_bwd_strided");
  }
}

void layernorm_fwd(const float* x, float* y, float* var, size_t outer, size_t axis_sz,
                   size_t inner, float eps) {
  if (!outer || !axis_sz || !inner) return;
  const bool vec4 = axis_sz % 4 == 0 && ((((uintptr_t)x) | ((uintptr_t)y)) & 15) == 0;
  if (inner == 1 && axis_sz <= 1024 && axis_sz >= 128 && vec4) {
    const unsigned blocks = grid_for(outer * 32, 256);
    if (axis_sz <= 128) k_layernorm_warp4<1><<<blocks, 256, 0, stream()>>>(x, y, var, outer, (int)axis_sz, eps);
    else if (axis_sz <= 256) k_layernorm_warp4<2><<<blocks, 256, 0, stream()>>>(x, y, var, outer, (int)axis_sz, eps);
    else if (axis_sz <= 512) k_layernorm_warp4<4><<<blocks, 256, 0, stream()>>>(x, y, var, outer, (int)axis_sz, eps);
    else k_layernorm_warp4<8><<<blocks, 256, 0, stream()>>>(x, y, var, outer, (int)axis_sz, eps);
    count_launch();
    after_launch("k_layernorm_warp4");
  } else if (inner == 1 && axis_sz <= 1024) {
    LAUNCH_ROWS_WARP(k_layernorm_warp, axis_sz, outer, x, y, var, outer, (int)axis_sz, eps);
  } else if (inner == 1) {
    k_layernorm_block<<<row_blocks(outer), 512, 0, stream()>>>(x, y, var, outer, axis_sz, eps);
    count_launch();
    after_launch("k_layernorm_block");
  } else {
    size_t g = outer * inner;
    k_layernorm_strided<<<(unsigned)((g + 255) / 256), 256, 0, stream()>>>(x, y, var, outer,
                                                                           axis_sz, inner, eps);
    count_launch();
    after_launch("k_layernorm_strided");
  }
}

void layernorm_bwd(const float* y, const float* var, const float* g, float* dx, size_t outer,
                   size_t axis_sz, size_t inner, float eps, const float* gs) {
  if (!outer || !axis_sz || !inner) return;
  if (gs && inner != 1) panic("layernorm_bwd: a column-scaled gradient needs the last axis");
  if (inner == 1 && axis_sz <= 1024) {
    LAUNCH_ROWS_WARP(k_layernorm_bwd_warp, axis_sz, outer, y, var, g, dx, outer, (int)axis_sz, eps, gs);
  } else if (inner == 1) {
    k_layernorm_bwd_block<<<row_blocks(outer), 512, 0, stream()>>>(y, var, g, dx, outer, axis_sz, eps, gs);
    count_launch();
    after_launch("k_layernorm_bwd_block");
  } else {
    size_t gg = outer * inner;
    k_layernorm_bwd_strided<<<(unsigned)((gg + 255) / 256), 256, 0, stream()>>>(
        y, var, g, dx, outer, axis_sz, inner, eps);
    count_launch();
    after_launch("k_layernorm_bwd_strided");
  }
}

void xent_fwd(const float* logits, const void* tgt, int tdt, float* probs, float* loss, size_t n,
              size_t v) {
  if (!n) {
    scalar_op_imm(kSFill, nullptr, NAN, loss, 1);
    return;
  }
  const int lpr = v <= 96 ? 8 : v <= 192 ? 16 : 0;   // lanes per row of k_xent_fwd_rows
  const unsigned blocks = lpr ? grid_for((n + 32 / lpr - 1) / (32 / lpr) * 32, 256)
                              : v <= 1024 ? grid_for(n * 32, 256) : row_blocks(n);
  float* part = (float*)scratch_alloc(blocks * sizeof(float));
  if (lpr == 8) {
    k_xent_fwd_rows<8><<<blocks, 256, 0, stream()>>>(logits, tgt, tdt, probs, part, n, (int)v, device_error_word());
    count_launch();
    after_launch("k_xent_fwd_rows");
  } else if (lpr == 16) {
    k_xent_fwd_rows<16><<<blocks, 256, 0, stream()>>>(logits, tgt, tdt, probs, part, n, (int)v, device_error_word());
    count_launch();
    after_launch("k_xent_fwd_rows");
  } else if (v <= 1024) {
    LAUNCH_ROWS_WARP(k_xent_fwd_warp, v, n, logits, tgt, tdt, probs, part, n, (int)v,
                     device_error_word());
  } else {
    k_xent_fwd_block<<<blocks, 512, 0, stream()>>>(logits, tgt, tdt, probs, part, n, v,
                                                   device_error_word());
    count_launch();
    after_launch("k_xent_fwd_block");
  }
  k_mean_partials<<<1, 32, 0, stream()>>>(part, (int)blocks, loss, n);
  count_launch();
  after_launch("k_mean_partials");
  scratch_free(part);
}

void xent_nll_gather(const float* probs, const void* tgt, int tdt, float* out, size_t n, size_t v) {
  if (!n) return;
  k_xent_nll_gather<<<(unsigned)((n + 255) / 256), 256, 0, stream()>>>(probs, tgt, tdt, out, n, v,
                                                                      device_error_word());
  count_launch();
  after_launch("k_xent_nll_gather");
}

static void xent_bwd_launch(const float* probs, const void* tgt, int tdt, const float* dout_dev,
                            float hscale, float* dx, size_t n, size_t v) {
  size_t total = n * v;
  if (!total) return;
  const bool vec = total < (1ull << 32) && ((((uintptr_t)probs) | ((uintptr_t)dx)) & 15) == 0;
  k_xent_bwd<<<grid_for(vec ? (total + 3) / 4 : total, 256), 256, 0, stream()>>>(probs, tgt, tdt, dout_dev,
                                                                                  hscale, dx, n, v, vec);
  count_launch();
  after_launch("k_xent_bwd");
}

void xent_bwd(const float* probs, const void* tgt, int tdt, const float* dout_dev, float* dx,
              size_t n, size_t v) {
  xent_bwd_launch(probs, tgt, tdt, dout_dev, 0.0f, dx, n, v);
}

void xent_bwd_scaled(const float* probs, const void* tgt, int tdt, float scale, float* dx, size_t n,
                     size_t v) {
  xent_bwd_launch(probs, tgt, tdt, nullptr, scale, dx, n, v);
}

void embedding_fwd(const float* w, const void* idx, int idt, float* out, size_t n, size_t vocab,
                   size_t dim) {
  if (!n || !dim) return;
  k_embedding_fwd<<<grid_for(n * 32, 256), 256, 0, stream()>>>(w, idx, idt, out, n, vocab, dim,
                                                              device_error_word());
  count_launch();
  after_launch("k_embedding_fwd");
}

// Exclusive scan of m ints: out[0..m] (out[m] = total).
static void exclusive_scan_int(const int* in, int* out, size_t m) {
  int nt = (int)((m + kScanTile - 1) / kScanTile);
  if (nt == 0) nt = 1;
  int* sums = (int*)scratch_alloc((size_t)nt * sizeof(int));
  k_scan_tile_sums<<<nt, 1024, 0, stream()>>>(in, m, sums);
  k_scan_sums_serial<<<1, 32, 0, stream()>>>(sums, nt, out + m);
  k_scan_tile_apply<<<nt, 1024, 0, stream()>>>(in, m, sums, out);
  count_launch(3);
  after_launch("exclusive_scan_int");
  scratch_free(sums);
}

void embedding_bwd(const float* dout, const void* idx, int idt, float* dw, size_t n, size_t V,
                   size_t D) {
  if (!V || !D) return;
  if (!n) {
    MALUS_CUDA(cudaMemsetAsync(dw, 0, V * D * sizeof(float), stream()));
    return;
  }
  int nch = (int)((n + kEmbChunk - 1) / kEmbChunk);
  size_t m = V * (size_t)nch;
  auto* keys = (unsigned long long*)scratch_alloc((size_t)nch * kEmbChunk * 8);
  int* counts = (int*)scratch_alloc(m * sizeof(int));
  int* offs = (int*)scratch_alloc((m + 1) * sizeof(int));
  int* order = (int*)scratch_alloc(n * sizeof(int));
  MALUS_CUDA(cudaMemsetAsync(counts, 0, m * sizeof(int), stream()));
  k_emb_chunk_sort<<<nch, 512, 0, stream()>>>(idx, idt, n, V, nch, keys, counts,
                                              device_error_word());
  count_launch();
  after_launch("k_emb_chunk_sort");
  exclusive_scan_int(counts, offs, m);
  k_emb_scatter<<<nch, 512, 0, stream()>>>(keys, n, nch, offs, order);
  count_launch();
  after_launch("k_emb_scatter");
  dim3 grid((unsigned)V, (unsigned)((D + kSegThreads - 1) / kSegThreads));
  const unsigned threads = kSegThreads;
  k_emb_segsum<<<grid, threads, 0, stream()>>>(dout, order, offs, nch, V, D, dw);
  count_launch();
  after_launch("k_emb_segsum");
  scratch_free(keys);
  scratch_free(counts);
  scratch_free(offs);
  scratch_free(order);
}

void permute_nd(const float* x, float* out, const Shape& s, const int* perm) {
  size_t n = s.numel();
  if (!n) return;
  int r = s.ndim;
  int64_t in_stride[kMaxRank];
  int64_t st = 1;
  for (int d = r - 1; d >= 0; --d) { in_stride[d] = st; st *= (int64_t)s.d[d]; }
  PermMeta m;
  m.ndim = r;
  for (int d = 0; d < r; ++d) {
    m.out_shape[d] = (int64_t)s.d[perm[d]];
    m.in_stride_for_out_dim[d] = in_stride[perm[d]];
  }
  bool identity = true;
  for (int d = 0; d < r; ++d) identity &= perm[d] == d;
  if (identity) {
    MALUS_CUDA(cudaMemcpyAsync(out, x, n * 4, cudaMemcpyDeviceToDevice, stream()));
    return;
  }
  if (perm[r - 1] == r - 1) {
    size_t L = s.d[r - 1];
    size_t nrows = n / L;
    k_permute_rows<<<grid_for(nrows * 32, 256), 256, 0, stream()>>>(x, out, nrows, L, m);
    count_launch();
    after_launch("k_permute_rows");
    return;
  }
  // last two dims swapped, leading dims in order: batched tiled transpose
  bool lead_identity = r >= 2 && perm[r - 1] == r - 2 && perm[r - 2] == r - 1;
  for (int d = 0; d < r - 2 && lead_identity; ++d) lead_identity &= perm[d] == d;
  if (lead_identity) {
    size_t R = s.d[r - 2], C = s.d[r - 1];
    size_t B = n / (R * C);
    dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32), (unsigned)B);
    k_transpose_tiled<<<grid, dim3(32, 8), 0, stream()>>>(x, out, R, C);
    count_launch();
    after_launch("k_transpose_tiled");
    return;
  }
  k_permute_general<<<grid_for(n, 256), 256, 0, stream()>>>(x, out, n, m);
  count_launch();
  after_launch("k_permute_general");
}

}  // namespace malus

// ---------------------------------------------------------------------------
// Embedding VJP on caller-provided workspace and stream (used by the fused
// step and by the entry point that allocates nothing).  Same kernels and order
// as embedding_bwd, so results are bit-identical; errors are returned instead
// of raised.  An id outside [0, V) contributes nothing and sets *err to 4
// (err = nullptr: a word at the head of the workspace, cleared by every call
// and never read, so such ids are skipped without a report).
namespace malus {

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

size_t embedding_bwd_ws_bytes(size_t n, size_t V) {
  size_t nch = (n + kEmbChunk - 1) / kEmbChunk;
  size_t m = V * nch;
  size_t nt = (m + kScanTile - 1) / kScanTile;
  if (nt == 0) nt = 1;
  return 256 + align256(nch * kEmbChunk * 8) + align256(m * 4) + align256((m + 1) * 4) +
         align256(n * 4) + align256(nt * 4);
}

int embedding_bwd_ws(const float* dout, const void* idx, int idt, float* dw, size_t n, size_t V,
                     size_t D, void* ws, cudaStream_t st, int32_t* err) {
  if (!V || !D) return 0;
  if (!n) return cudaMemsetAsync(dw, 0, V * D * sizeof(float), st) == cudaSuccess ? 0 : -5;
  int nch = (int)((n + kEmbChunk - 1) / kEmbChunk);
  size_t m = V * (size_t)nch;
  int nt = (int)((m + kScanTile - 1) / kScanTile);
  if (nt == 0) nt = 1;
  char* p = (char*)ws;
  int32_t* own_err = (int32_t*)p;             p += 256;
  auto* keys = (unsigned long long*)p;        p += align256((size_t)nch * kEmbChunk * 8);
  int* counts = (int*)p;                      p += align256(m * 4);
  int* offs = (int*)p;                        p += align256((m + 1) * 4);
  int* order = (int*)p;                       p += align256(n * 4);
  int* sums = (int*)p;
  if (!err) {
    err = own_err;
    if (cudaMemsetAsync(err, 0, sizeof(int32_t), st) != cudaSuccess) return -5;
  }
  if (cudaMemsetAsync(counts, 0, m * sizeof(int), st) != cudaSuccess) return -5;
  // each launch is checked right after it (cudaGetLastError), so an error
  // left by some earlier, unrelated launch is not reported as this call's
  int bad = 0;
  auto check = [&] { if (cudaGetLastError() != cudaSuccess) bad = 1; };
  k_emb_chunk_sort<<<nch, 512, 0, st>>>(idx, idt, n, V, nch, keys, counts, err);
  check();
  k_scan_tile_sums<<<nt, 1024, 0, st>>>(counts, m, sums);
  check();
  k_scan_sums_serial<<<1, 32, 0, st>>>(sums, nt, offs + m);
  check();
  k_scan_tile_apply<<<nt, 1024, 0, st>>>(counts, m, sums, offs);
  check();
  k_emb_scatter<<<nch, 512, 0, st>>>(keys, n, nch, offs, order);
  check();
  dim3 grid((unsigned)V, (unsigned)((D + kSegThreads - 1) / kSegThreads));
  const unsigned threads = kSegThreads;
  k_emb_segsum<<<grid, threads, 0, st>>>(dout, order, offs, nch, V, D, dw);
  check();
  count_launch(6);
  return bad ? -6 : 0;
}

}  // namespace malus
