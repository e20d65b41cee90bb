// Axis reductions over the (outer, axis, inner) decomposition of
// crates/malus-stdlib/stdlib/reduce_{sum,mean,max,var}.ml.  The reference
// gives each (outer, inner) group one threadgroup of `axis` threads and lets
// thread 0 loop serially (so axis <= 1024).  Here:
//  - inner == 1 (contiguous rows): one warp per row (block per row for long
//    rows), 16-byte loads, shuffle reduction;
//  - inner > 1 (column reduction): threads walk consecutive `inner` indices
//    (coalesced), the axis is cut into a fixed number of chunks when the
//    output is too small to fill 148 SMs, and a second pass sums the chunk
//    partials in chunk order.  Both passes are deterministic (no atomics).
// Variance is population variance with the two-pass formula of
// reduce_var.ml:16-25 (mean first, then the mean of squared deviations).
#include "common.cuh"

namespace malus {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- contiguous rows: one warp per row ----
template <int OP>
__global__ void k_reduce_rows_warp(const float* __restrict__ x, float* __restrict__ out,
                                   size_t rows, int len) {
  int lane = threadIdx.x & 31;
  size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t r = warp; r < rows; r += nwarps) {
    const float* row = x + r * (size_t)len;
    float acc = OP == kRMax ? -INFINITY : 0.0f;
    for (int i = lane; i < len; i += 32) {
      float v = row[i];
      acc = OP == kRMax ? fmaxf(acc, v) : acc + v;
    }
    acc = OP == kRMax ? warp_max(acc) : warp_sum(acc);
    if (OP == kRVar) {
      float mean = acc / (float)len;
      float sq = 0.0f;
      for (int i = lane; i < len; i += 32) {
        float d = row[i] - mean;
        sq += d * d;
      }
      acc = warp_sum(sq) / (float)len;
    } else if (OP == kRMean) {
      acc = acc / (float)len;
    }
    if (lane == 0) out[r] = acc;
  }
}

// ---- long contiguous rows: one block (256 threads) per row, float4 ----
template <int OP>
__global__ void k_reduce_rows_block(const float* __restrict__ x, float* __restrict__ out,
                                    size_t rows, size_t len) {
  __shared__ float red[32];
  __shared__ float bcast;
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * len;
    bool vec = ((len & 3) == 0) && (((uintptr_t)row & 15) == 0);
    float acc = OP == kRMax ? -INFINITY : 0.0f;
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (size_t i = threadIdx.x; i < len / 4; i += blockDim.x) {
        float4 v = r4[i];
        if (OP == kRMax) acc = fmaxf(fmaxf(acc, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
        else acc += (v.x + v.y) + (v.z + v.w);
      }
    } else {
      for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
        float v = row[i];
        acc = OP == kRMax ? fmaxf(acc, v) : acc + v;
      }
    }
    acc = OP == kRMax ? warp_max(acc) : warp_sum(acc);
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[w] = acc;
    __syncthreads();
    if (w == 0) {
      float v = lane < (int)(blockDim.x >> 5) ? red[lane] : (OP == kRMax ? -INFINITY : 0.0f);
      v = OP == kRMax ? warp_max(v) : warp_sum(v);
      if (lane == 0) bcast = v;
    }
    __syncthreads();
    float total = bcast;
    if (OP == kRVar) {
      float mean = total / (float)len;
      float sq = 0.0f;
      for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
        float d = row[i] - mean;
        sq += d * d;
      }
      sq = warp_sum(sq);
      __syncthreads();
      if (lane == 0) red[w] = sq;
      __syncthreads();
      if (w == 0) {
        float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        v = warp_sum(v);
        if (lane == 0) bcast = v / (float)len;
      }
      __syncthreads();
      total = bcast;
    } else if (OP == kRMean) {
      total = total / (float)len;
    }
    if (threadIdx.x == 0) out[r] = total;
    __syncthreads();
  }
}

// ---- column reduction partials: part[c][o*inner+i] over axis chunk c ----
// mode 0: sum, 1: max, 2: sum of squared deviation from center[o*inner+i]
// x2 (mode 0 only, optional): the values summed are x[i] * x2[i], each rounded
__global__ void k_reduce_cols(const float* __restrict__ x, float* __restrict__ part,
                              const float* __restrict__ center, int mode, size_t outer,
                              size_t axis_sz, size_t inner, size_t chunk,
                              const float* __restrict__ x2 = nullptr) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t o = blockIdx.y;
  size_t c = blockIdx.z;
  if (i >= inner) return;
  size_t a0 = c * chunk, a1 = a0 + chunk < axis_sz ? a0 + chunk : axis_sz;
  const float* base = x + o * axis_sz * inner + i;
  const float* base2 = x2 ? x2 + o * axis_sz * inner + i : nullptr;
  float ctr = mode == 2 ? center[o * inner + i] : 0.0f;
  float acc0 = mode == 1 ? -INFINITY : 0.0f, acc1 = acc0, acc2 = acc0, acc3 = acc0;
  size_t a = a0;
  // eight rows' loads in flight per step; accumulator k still adds rows
  // a = k (mod 4) in increasing order (the same sums as four rows per step)
  for (; a + 8 <= a1; a += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = base[(a + u) * inner];
    if (base2) {
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __fmul_rn(v[u], base2[(a + u) * inner]);
    }
#pragma unroll
    for (int h = 0; h < 8; h += 4) {
      float v0 = v[h], v1 = v[h + 1], v2 = v[h + 2], v3 = v[h + 3];
      if (mode == 1) {
        acc0 = fmaxf(acc0, v0); acc1 = fmaxf(acc1, v1); acc2 = fmaxf(acc2, v2); acc3 = fmaxf(acc3, v3);
      } else if (mode == 2) {
        v0 -= ctr; v1 -= ctr; v2 -= ctr; v3 -= ctr;
        acc0 += v0 * v0; acc1 += v1 * v1; acc2 += v2 * v2; acc3 += v3 * v3;
      } else {
        acc0 += v0; acc1 += v1; acc2 += v2; acc3 += v3;
      }
    }
  }
  for (; a + 4 <= a1; a += 4) {
    float v0 = base[a * inner], v1 = base[(a + 1) * inner];
    float v2 = base[(a + 2) * inner], v3 = base[(a + 3) * inner];
    if (base2) {
      v0 = __fmul_rn(v0, base2[a * inner]); v1 = __fmul_rn(v1, base2[(a + 1) * inner]);
      v2 = __fmul_rn(v2, base2[(a + 2) * inner]); v3 = __fmul_rn(v3, base2[(a + 3) * inner]);
    }
    if (mode == 1) {
      acc0 = fmaxf(acc0, v0); acc1 = fmaxf(acc1, v1); acc2 = fmaxf(acc2, v2); acc3 = fmaxf(acc3, v3);
    } else if (mode == 2) {
      v0 -= ctr; v1 -= ctr; v2 -= ctr; v3 -= ctr;
      acc0 += v0 * v0; acc1 += v1 * v1; acc2 += v2 * v2; acc3 += v3 * v3;
    } else {
      acc0 += v0; acc1 += v1; acc2 += v2; acc3 += v3;
    }
  }
  for (; a < a1; ++a) {
    float v = base[a * inner];
    if (base2) v = __fmul_rn(v, base2[a * inner]);
    if (mode == 1) acc0 = fmaxf(acc0, v);
    else if (mode == 2) { v -= ctr; acc0 += v * v; }
    else acc0 += v;
  }
  float r = mode == 1 ? fmaxf(fmaxf(acc0, acc1), fmaxf(acc2, acc3)) : (acc0 + acc1) + (acc2 + acc3);
  part[c * outer * inner + o * inner + i] = r;
}

// out[j] = combine over chunks of part[c][j]; then /n for mean/var.
// One warp per output: lane l combines chunks l, l + 32, ... in order, then a
// fixed shuffle tree combines the lanes (the same order on every run).
__global__ void k_reduce_combine(const float* __restrict__ part, float* __restrict__ out,
                                 size_t m, int nchunks, int mode, float inv_n) {
  const size_t j = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= m) return;
  float acc = mode == 1 ? -INFINITY : 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    const float v = part[(size_t)c * m + j];
    acc = mode == 1 ? fmaxf(acc, v) : acc + v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, acc, o);
    acc = mode == 1 ? fmaxf(acc, w) : acc + w;
  }
  if (lane == 0) out[j] = inv_n != 0.0f ? acc * inv_n : acc;
}

// out[j] = part_sum[j] / n, computed with a true division to match s / n_f
__global__ void k_div_n(float* __restrict__ v, size_t m, float n) {
  size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (j < m) v[j] = v[j] / n;
}

void column_pass(const float* x, float* out, const float* center, int mode, size_t outer,
                 size_t axis_sz, size_t inner, bool divide, const float* x2 = nullptr) {
  size_t m = outer * inner;
  size_t target = (size_t)kNumSMs * 2048;
  size_t nchunks = 1;
  if (m < target) {
    nchunks = (target + m - 1) / m;
    size_t maxc = (axis_sz + 31) / 32;  // at least 32 rows per chunk
    if (nchunks > maxc) nchunks = maxc;
    if (nchunks < 1) nchunks = 1;
  }
  size_t chunk = (axis_sz + nchunks - 1) / nchunks;
  nchunks = (axis_sz + chunk - 1) / chunk;
  if (nchunks == 0) nchunks = 1;
  float* part = nchunks == 1 ? out : (float*)scratch_alloc(nchunks * m * sizeof(float));
  dim3 grid((unsigned)((inner + 255) / 256), (unsigned)outer, (unsigned)nchunks);
  k_reduce_cols<<<grid, 256, 0, stream()>>>(x, part, center, mode, outer, axis_sz, inner, chunk, x2);
  count_launch();
  after_launch("k_reduce_cols");
  if (nchunks > 1) {
    k_reduce_combine<<<(unsigned)((m * 32 + 255) / 256), 256, 0, stream()>>>(part, out, m, (int)nchunks,
                                                                            mode, 0.0f);
    count_launch();
    after_launch("k_reduce_combine");
    scratch_free(part);
  }
  if (divide) {
    k_div_n<<<(unsigned)((m + 255) / 256), 256, 0, stream()>>>(out, m, (float)axis_sz);
    count_launch();
    after_launch("k_div_n");
  }
}

}  // namespace

void reduce_axis(int op, const float* x, float* out, size_t outer, size_t axis_sz, size_t inner) {
  size_t m = outer * inner;
  if (m == 0) return;
  if (axis_sz == 0) {
    // empty reduction: sum 0, max -inf, mean/var NaN (0/0), as the serial loop gives
    float v = op == kRSum ? 0.0f : (op == kRMax ? -INFINITY : NAN);
    scalar_op_imm(kSFill, nullptr, v, out, m);
    return;
  }
  if (inner == 1) {
    if (axis_sz <= 2048) {
      unsigned blocks = grid_for(outer * 32, 256);
      switch (op) {
        case kRSum: k_reduce_rows_warp<kRSum><<<blocks, 256, 0, stream()>>>(x, out, outer, (int)axis_sz); break;
        case kRMean: k_reduce_rows_warp<kRMean><<<blocks, 256, 0, stream()>>>(x, out, outer, (int)axis_sz); break;
        case kRMax: k_reduce_rows_warp<kRMax><<<blocks, 256, 0, stream()>>>(x, out, outer, (int)axis_sz); break;
        default: k_reduce_rows_warp<kRVar><<<blocks, 256, 0, stream()>>>(x, out, outer, (int)axis_sz); break;
      }
      count_launch();
      after_launch("k_reduce_rows_warp");
      return;
    }
    if (outer >= (size_t)kNumSMs) {
      unsigned blocks = (unsigned)std::min<size_t>(outer, (size_t)kNumSMs * 8);
      switch (op) {
        case kRSum: k_reduce_rows_block<kRSum><<<blocks, 256, 0, stream()>>>(x, out, outer, axis_sz); break;
        case kRMean: k_reduce_rows_block<kRMean><<<blocks, 256, 0, stream()>>>(x, out, outer, axis_sz); break;
        case kRMax: k_reduce_rows_block<kRMax><<<blocks, 256, 0, stream()>>>(x, out, outer, axis_sz); break;
        default: k_reduce_rows_block<kRVar><<<blocks, 256, 0, stream()>>>(x, out, outer, axis_sz); break;
      }
      count_launch();
      after_launch("k_reduce_rows_block");
      return;
    }
    // few very long rows (e.g. a whole-tensor sum): treat the row as a column
    // of length axis_sz with inner = 1 and chunk it across the GPU.
  }
  if (op == kRVar) {
    float* mean = (float*)scratch_alloc(m * sizeof(float));
    column_pass(x, mean, nullptr, 0, outer, axis_sz, inner, true);
    column_pass(x, out, mean, 2, outer, axis_sz, inner, true);
    scratch_free(mean);
    return;
  }
  column_pass(x, out, nullptr, op == kRMax ? 1 : 0, outer, axis_sz, inner, op == kRMean);
}

void reduce_axis_sum_product(const float* x, const float* x2, float* out, size_t outer, size_t axis_sz,
                             size_t inner) {
  if (inner <= 1) panic("reduce_axis_sum_product: column sums only (inner %zu)", inner);
  const size_t m = outer * inner;
  if (m == 0) return;
  if (axis_sz == 0) {
    scalar_op_imm(kSFill, nullptr, 0.0f, out, m);
    return;
  }
  column_pass(x, out, nullptr, 0, outer, axis_sz, inner, false, x2);
}

}  // namespace malus
