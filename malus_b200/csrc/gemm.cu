// f32 GEMM for tensor_matmul and its VJPs (metal.rs:820-962 and
// stdlib/backward/matmul_bwd.ml:15-29).
//
// Two backends, both bound to f32 semantics:
//  * tcgen05 3xTF32 (large shapes).  Each operand x is split once into
//    x_hi = tf32_rn(x) and x_lo = tf32_rn(x - x_hi) (planes in the operand's
//    own layout); the tensor core accumulates A_hi*B_hi + A_hi*B_lo +
//    A_lo*B_hi in f32 in TMEM, which keeps ~22 bits of each product — well
//    inside the 1e-4 relative matmul tolerance.  Operands reach shared memory
//    by TMA (128-byte swizzle, no multicast); transposed operands use the
//    MN-major UMMA descriptor, so matmul VJPs never materialise a transpose.
//    One elected thread issues tcgen05.mma; four epilogue warps drain TMEM
//    with tcgen05.ld.  Every mbarrier wait is bounded: on timeout the kernel
//    records an error word, drains its own in-flight copies/MMAs (bounded),
//    frees TMEM and returns.
//  * SIMT (tiny shapes: XOR, N=65 heads of toy configs, degenerate dims):
//    exact f32, products added in k order with separate multiply and add,
//    which is bit-identical to the reference's CPU loop
//    (tensor_matmul_cpu, metal.rs:699-800).
#include "common.cuh"
#include "tc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace malus {

// ================================================================== SIMT
namespace {
constexpr int ST = 64, SK = 16;

__global__ void __launch_bounds__(256)
k_gemm_simt(int M, int N, int K, const float* __restrict__ A, int64_t lda, int64_t sA, bool at,
            const float* __restrict__ B, int64_t ldb, int64_t sB, bool bt, float* __restrict__ C,
            int64_t ldc, int64_t sC, float alpha, float beta) {
  __shared__ float As[SK][ST + 1];
  __shared__ float Bs[SK][ST + 1];
  int b = blockIdx.z;
  A += b * sA;
  B += b * sB;
  C += b * sC;
  int m0 = blockIdx.y * ST, n0 = blockIdx.x * ST;
  int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += SK) {
    for (int e = threadIdx.x; e < ST * SK; e += 256) {
      int r = e / SK, kk = e % SK;  // A tile: row r, col kk
      int m = m0 + r, k = k0 + kk;
      float v = 0.0f;
      if (m < M && k < K) v = at ? A[(int64_t)k * lda + m] : A[(int64_t)m * lda + k];
      As[kk][r] = v;
      int c = e % ST, kb = e / ST;   // B tile: row kb, col c
      int n = n0 + c, k2 = k0 + kb;
      float w = 0.0f;
      if (n < N && k2 < K) w = bt ? B[(int64_t)n * ldb + k2] : B[(int64_t)k2 * ldb + n];
      Bs[kb][c] = w;
    }
    __syncthreads();
    int kmax = min(SK, K - k0);
    for (int kk = 0; kk < kmax; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float* c = C + (int64_t)m * ldc + n;
      float r = alpha == 1.0f ? acc[i][j] : alpha * acc[i][j];
      if (beta != 0.0f) r = r + beta * *c;
      *c = r;
    }
  }
}
}  // namespace

void gemm_simt(const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return;
  if (g.K <= 0) {
    // empty reduction: C = beta*C (alpha*0)
    for (int b = 0; b < g.batch; ++b) {
      if (g.beta == 0.0f) {
        MALUS_CUDA(cudaMemset2DAsync(g.C + b * g.strideC, g.ldc * 4, 0, (size_t)g.N * 4, g.M, stream()));
      } else if (g.beta != 1.0f) {
        panic("gemm with K=0 and beta not in {0,1} is unsupported");
      }
    }
    return;
  }
  dim3 grid((g.N + ST - 1) / ST, (g.M + ST - 1) / ST, g.batch);
  int pid = prof_begin(2, 2.0 * g.M * (double)g.N * g.K * g.batch, 0.0);
  k_gemm_simt<<<grid, 256, 0, stream()>>>(g.M, g.N, g.K, g.A.base, g.A.r.lo, g.A.nz > 1 ? g.A.z.lo : 0,
                                          g.a_trans, g.B.base, g.B.r.lo, g.B.nz > 1 ? g.B.z.lo : 0,
                                          g.b_trans, g.C, g.ldc, g.strideC, g.alpha, g.beta);
  count_launch();
  after_launch("k_gemm_simt");
  prof_end(pid);
}

// =============================================================== tcgen05
//
// Persistent 3xTF32 GEMM.  One CTA per SM walks a static list of 128 x BN
// output tiles (BN 64-256), or one 2-CTA cluster per TPC walks 256 x BN tiles
// (CTA pairs, cta_group::2).  Warp 0 streams operand tiles with TMA into a
// shared-memory ring of up to six stages, warp 1 issues tcgen05.mma into one of
// two TMEM accumulators (2 x BN columns), and the epilogue warps (4 or 8) drain
// the other accumulator (tcgen05.ld -> registers -> global) while the next
// tile is being computed.
// Each f32 operand arrives as two tf32 planes (hi = rn(x), lo = rn(x - hi));
// the accumulator receives lo*hi + hi*lo + hi*hi per k-step.
//
// The epilogue writes through a mixed-radix address map out(z, m, n) =
// Z(z) + Mr(m) + Nc(n), each term (i / div) * hi + (i % div) * lo, which
// expresses plain row-major outputs, batched outputs, the attention head
// fold/unfold and N-segmented outputs without extra copies; and it can fuse a
// residual add, GELU (storing the pre-activation), the GELU derivative, and
// the tf32 split of its own output (so the next GEMM reads ready planes).
namespace {
using namespace malus::tc;

constexpr int BM = 128;
constexpr int kEpiWarpFloats = 32 * 32;   // per-warp 32x32 staging block (XOR-swizzled granules)
// Tile shape: width BN (64, 128, 192 or 256) and k-block depth BK (32 or 16).  A wider
// tile reads each A k-block once for more columns (less shared-memory and L2
// traffic per FLOP); a shallower k-block makes stages smaller, so more of them
// fit and the TMA latency is covered further ahead.  K-major tiles use the
// 128-byte swizzle (BK 32) or the 64-byte swizzle (BK 16); MN-major tiles the
// 32-byte-granule 128-byte swizzle with BK rows per 32-column chunk.
// With PAIR_ the tile is one of a CTA pair's (256 rows): this CTA loads its
// 128 rows of A and BN / 2 rows of B (see the pair notes at k_gemm_tc).
template <int BN_, int BK_, bool PAIR_ = false>
struct TileCfg {
  static constexpr int BN = BN_, BK = BK_;
  static constexpr int BNL = PAIR_ ? BN_ / 2 : BN_;   // B rows (tile columns) loaded by this CTA
  static constexpr int kTileBytesA = BM * BK * 4;
  static constexpr int kTileBytesB = BNL * BK * 4;
  static constexpr int kStageBytes = 2 * kTileBytesA + 2 * kTileBytesB;
  static constexpr int kFixed = 1024 /*align*/ + 256 /*barriers*/ + 8 * kEpiWarpFloats * 4 /*staging*/;
  static constexpr int kMaxStages = 6;   // barrier area: 2 x 6 stage barriers + 6 more + 2 words
  static constexpr int STAGES = (232448 - kFixed) / kStageBytes > kMaxStages ? kMaxStages
                                                                             : (232448 - kFixed) / kStageBytes;
  static constexpr int kSmemBytes = STAGES * kStageBytes + kFixed;
  static constexpr uint32_t kTmemCols = BN <= 64 ? 128 : (BN <= 128 ? 256 : 512);   // two accumulators, power of 2
  static constexpr int kChunkBytes = BK * 128;   // one 32-wide MN chunk (or 32-row K-major box)
  static_assert(STAGES >= 2 && kSmemBytes <= 232448, "shared memory");
};

// Shared-memory descriptors for a k-block of depth BK.
template <int BK>
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, int kk) {
  return BK == 32 ? umma_desc(tile + kk * 32, 16, 1024, 2)    // 128-B swizzle, 8-row atoms 1 KB
                  : umma_desc(tile + kk * 32, 16, 512, 4);    // 64-B swizzle, 8-row atoms 512 B
}
template <int BK>
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kk) {
  return umma_desc(tile + kk * 1024, BK * 128, 512, 1);       // chunks BK rows x 128 B apart
}
// Epilogue warps: 8 (two per TMEM lane quarter, half the columns each) when the
// epilogue reads an auxiliary input, whose load latency the extra warps hide;
// 4 otherwise, leaving L2 bandwidth to the operand loads.
__host__ __device__ constexpr int epi_warps(int epi) { return epi == 0 ? 4 : 8; }
// Epilogues with math per element or an auxiliary input, and stores that write
// tf32 planes, go through the transposing smem stage (coalesced loads and
// stores); a plain f32 store writes each lane's row directly.
__host__ __device__ constexpr int threads_tc(int epi) { return 64 + 32 * epi_warps(epi); }
constexpr float kGeluC0 = 0.7978845608028654f, kGeluC1 = 0.044715f;



// Indices (z < batch, m < M, n < N: all int) and radices fit 32 bits: 32-bit division.
__device__ __forceinline__ int64_t lay(const TcLayout& L, int64_t idx) {
  uint32_t i = (uint32_t)idx;
  int64_t off = 0;
  if (L.d1) { uint32_t d = (uint32_t)L.d1, q = i / d; off = (int64_t)q * L.s1; i -= q * d; }
  if (L.d2) { uint32_t d = (uint32_t)L.d2, q = i / d; off += (int64_t)q * L.s2; i -= q * d; }
  return off + (int64_t)i * L.s3;
}

struct TcKernelParams {
  TcProblem pr;
  int tiles_m, tiles_n, nk;
  int splits;      // K slices per tile (split-K); > 1 writes raw partial tiles to ws
  float* ws;       // [tile][split][BM][bn] partial accumulators when splits > 1
  int bn;          // tile width (the kernel's BN)
  int bk;          // k-block depth (the kernel's BK)
  int bm;          // tile height: 128, or 256 for a CTA pair
  int a_chunked, b_chunked;   // MN-major operand loaded as one {32, 32 K, 4 chunks} box per plane
  int a_pair, b_pair;         // both planes of a stage's tile in one box (a plane dimension)
  int a_swap, b_swap;         // ... whose plane 0 is the lo plane (it is the lower address)
  int staged;                 // epilogue through the smem transpose (see epi_warps)
  int32_t* err;
};

// Work unit -> tile and K-block range, honouring split-K and the causal modes.
// Returns false for output tiles wholly above the diagonal (kCausalOut).
struct Unit {
  int z, m0, n0, kb_lo, kb_hi;
};
__device__ __forceinline__ bool unit_of(const TcKernelParams& kp, int unit, Unit& u) {
  const TcProblem& p = kp.pr;
  const int per_batch = kp.tiles_m * kp.tiles_n;
  const int tile = unit / kp.splits, sl = unit % kp.splits;
  u.z = tile / per_batch;
  const int rem = tile % per_batch;
  u.m0 = (rem / kp.tiles_n) * kp.bm;
  u.n0 = (rem % kp.tiles_n) * kp.bn;
  if (p.causal == kCausalOut && u.n0 > u.m0 + BM - 1) return false;
  int lo = 0, hi = kp.nk;
  if (p.causal == kCausalALower) hi = min(kp.nk, (u.m0 + BM + kp.bk - 1) / kp.bk);
  if (p.causal == kCausalAUpper) lo = u.m0 / kp.bk;
  const int len = hi - lo;
  u.kb_lo = lo + sl * len / kp.splits;
  u.kb_hi = lo + (sl + 1) * len / kp.splits;
  return u.kb_hi > u.kb_lo;
}

// Operand coordinates for k-block k0 of tile (z, m0/n0).
__device__ __forceinline__ void operand_coords(int zmode, int seg, int z, int k0, int mn0,
                                               int* kc, int* mnc, int* zc) {
  *kc = k0;
  *mnc = mn0;
  *zc = 0;
  if (zmode == kZBatch) *zc = z;
  else if (zmode == kZKSeg) { *zc = k0 / seg; *kc = k0 % seg; }
  else if (zmode == kZMNSeg) { *zc = mn0 / seg; *mnc = mn0 % seg; }
}


__device__ __forceinline__ float gelu_f(float v) {
  float x3 = v * v * v;
  return 0.5f * v * (1.0f + tanhf(kGeluC0 * (v + kGeluC1 * x3)));
}
__device__ __forceinline__ float gelu_grad(float x) {
  float x3 = x * x * x;
  float t = tanhf(kGeluC0 * (x + kGeluC1 * x3));
  float gp = kGeluC0 * (1.0f + 3.0f * kGeluC1 * x * x);
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * gp;
}

// One output element: value v (the accumulator) at offset o.
template <int EPI>
__device__ __forceinline__ void epi_store1(const TcProblem& p, int64_t o, float v, float rv = 0.0f) {
  if (EPI != kEpiSoftmaxBwd && p.alpha != 1.0f) v *= p.alpha;
  float split_src;
  if (EPI == kEpiSoftmaxBwd) {    // dS = (P * (dP - D)) * scale
    const float pv = p.aux[o] + p.aux_lo[o];
    split_src = (pv * (v - rv)) * p.alpha;
    if (p.out) p.out[o] = split_src;
  } else if (EPI == kEpiStore) {
    if (p.out) {                  // the f32 output is optional: planes-only callers pass none
      if (p.beta != 0.0f) v += p.beta * p.out[o];
      p.out[o] = v;
    }
    split_src = v;
  } else if (EPI == kEpiResid) {
    v = p.aux[o] + v;
    if (p.out) p.out[o] = v;
    split_src = v;
  } else if (EPI == kEpiGelu) {
    if (p.out) p.out[o] = v;      // pre-activation, kept for the GELU derivative
    split_src = gelu_f(v);
  } else {                        // kEpiGeluBwd: v = dL/d(gelu out); aux = pre-activation
    split_src = v * gelu_grad(p.aux[o]);
    if (p.out) p.out[o] = split_src;
  }
  if (p.out_hi) {
    float h = tf32_rn(split_src);
    p.out_hi[o] = h;
    p.out_lo[o] = tf32_rn(split_src - h);
  }
}

// Four consecutive output elements at 16-byte aligned offset o.
template <int EPI>
__device__ __forceinline__ void epi_store4(const TcProblem& p, int64_t o, float4 v, float4 aux4,
                                           float4 auxlo4 = float4{}, float rv = 0.0f) {
  if (EPI != kEpiSoftmaxBwd && p.alpha != 1.0f) { v.x *= p.alpha; v.y *= p.alpha; v.z *= p.alpha; v.w *= p.alpha; }
  float4 s;
  if (EPI == kEpiSoftmaxBwd) {
    const float a = p.alpha;
    s = make_float4(((aux4.x + auxlo4.x) * (v.x - rv)) * a, ((aux4.y + auxlo4.y) * (v.y - rv)) * a,
                    ((aux4.z + auxlo4.z) * (v.z - rv)) * a, ((aux4.w + auxlo4.w) * (v.w - rv)) * a);
    if (p.out) *reinterpret_cast<float4*>(p.out + o) = s;
  } else if (EPI == kEpiStore) {
    if (p.out) {
      if (p.beta != 0.0f) {
        float4 q = *reinterpret_cast<const float4*>(p.out + o);
        v.x += p.beta * q.x; v.y += p.beta * q.y; v.z += p.beta * q.z; v.w += p.beta * q.w;
      }
      *reinterpret_cast<float4*>(p.out + o) = v;
    }
    s = v;
  } else if (EPI == kEpiResid) {
    const float4 q = aux4;
    v.x = q.x + v.x; v.y = q.y + v.y; v.z = q.z + v.z; v.w = q.w + v.w;
    if (p.out) *reinterpret_cast<float4*>(p.out + o) = v;
    s = v;
  } else if (EPI == kEpiGelu) {
    if (p.out) *reinterpret_cast<float4*>(p.out + o) = v;
    s = make_float4(gelu_f(v.x), gelu_f(v.y), gelu_f(v.z), gelu_f(v.w));
  } else {
    const float4 x = aux4;
    s = make_float4(v.x * gelu_grad(x.x), v.y * gelu_grad(x.y), v.z * gelu_grad(x.z),
                    v.w * gelu_grad(x.w));
    if (p.out) *reinterpret_cast<float4*>(p.out + o) = s;
  }
  if (p.out_hi) {
    float4 h = make_float4(tf32_rn(s.x), tf32_rn(s.y), tf32_rn(s.z), tf32_rn(s.w));
    float4 l = make_float4(tf32_rn(s.x - h.x), tf32_rn(s.y - h.y), tf32_rn(s.z - h.z),
                           tf32_rn(s.w - h.w));
    *reinterpret_cast<float4*>(p.out_hi + o) = h;
    *reinterpret_cast<float4*>(p.out_lo + o) = l;
  }
}

// PAIR: the kernel runs as 2-CTA clusters and each work unit is a 256 x BN
// tile computed by one M = 256 tcgen05.mma (cta_group::2) per k-step.  Both
// CTAs load their own 128 rows of A and BN / 2 rows of B into their own ring;
// the transaction bytes of both count on rank 0's full barrier (rank 0 expects
// the pair's bytes), rank 0 issues the MMAs, and its commits arrive on the
// empty and accumulator-full barriers of both CTAs.  Each CTA's epilogue
// drains its own 128 accumulator rows and arrives on rank 0's
// accumulator-empty barrier.  Per SM a k-step then moves A (128 rows) and half
// of B instead of all of B, which bounded the single-CTA mainloop (its TMA
// traffic per MMA).
template <int EPI, int BNT, int BKT, bool PAIR>
__global__ void __launch_bounds__(threads_tc(EPI), 1)
k_gemm_tc(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
          const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl,
          const TcKernelParams kp) {
  using CF = TileCfg<BNT, BKT, PAIR>;
  constexpr int BN = CF::BN, BK = CF::BK, STAGES = CF::STAGES, kStageBytes = CF::kStageBytes;
  constexpr int BNL = CF::BNL;
  constexpr int kTileBytesA = CF::kTileBytesA, kTileBytesB = CF::kTileBytesB, kChunk = CF::kChunkBytes;
  constexpr uint32_t kTmemCols = CF::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  const TcProblem& p = kp.pr;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* bar_area = smem + STAGES * kStageBytes;
  uint64_t* full = (uint64_t*)bar_area;
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint64_t* done = drain + 1;   // every epilogue warp finished reading TMEM
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  static_assert(CF::kMaxStages * 2 * 8 + 6 * 8 + 8 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_batch = kp.tiles_m * kp.tiles_n;
  const int splits = kp.splits;
  const int total = per_batch * p.batch * splits;   // work units: (tile, K slice)
  const int nk = kp.nk;
  // A pair walks the unit list as one: position = cluster index.
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int grp = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ngrp = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&accf[b]), 1);
      mbar_init(smem_u32(&acce[b]), epi_warps(EPI) * (PAIR ? 2 : 1));   // a pair: both CTAs' epilogues
    }
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(done), epi_warps(EPI));
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {   // the same columns in both CTAs' tensor memory
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();   // a CTA barrier needs converged warps (thread 0 initialised the barriers)
  __syncthreads();
  if (PAIR) cluster_sync_all();   // both CTAs' barriers exist before either signals the other
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // a pair's loads count on rank 0's full barrier
      auto ld3 = [&](uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2) {
        if constexpr (PAIR) tma_load_3d_pair(dst, m, bar, c0, c1, c2);
        else tma_load_3d(dst, m, bar, c0, c1, c2);
      };
      auto ld4 = [&](uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2, int c3) {
        if constexpr (PAIR) tma_load_4d_pair(dst, m, bar, c0, c1, c2, c3);
        else tma_load_4d(dst, m, bar, c0, c1, c2, c3);
      };
      uint32_t it = 0;
      bool ok = true;
      for (int unit = grp; unit < total && ok; unit += ngrp) {
        Unit un;
        if (!unit_of(kp, unit, un)) continue;
        // this CTA's rows of A and of B (a pair: rank 1 takes the second halves)
        const int z = un.z, m0 = un.m0 + (int)rank * BM, n0 = un.n0 + (int)rank * BNL;
        for (int kb = un.kb_lo; kb < un.kb_hi; ++kb, ++it) {
          int s = it % STAGES;
          uint32_t ph = (it / STAGES) & 1;
          if (it >= STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag, kp.err, 11)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          uint32_t fb = smem_u32(&full[s]);
          if (PAIR) {
            if (rank == 0) mbar_expect_tx(fb, 2 * kStageBytes);   // this CTA's and rank 1's copies
            fb = cluster_addr(fb, 0);
          } else {
            mbar_expect_tx(fb, kStageBytes);
          }
          int k0 = kb * BK, kc, mnc, zc;
          // A 128-wide M/N tile may straddle segments (segment width a multiple
          // of 32): MN-major tiles and K-major tiles of an MN-segmented operand
          // are loaded as four 32-wide boxes, each with its own segment.
          if (kp.a_chunked) {
            operand_coords(p.a.zmode, p.a.seg, z, k0, m0, &kc, &mnc, &zc);
            ld4(smem_u32(st), &mAh, fb, 0, kc, mnc >> 5, zc);
            ld4(smem_u32(st + kTileBytesA), &mAl, fb, 0, kc, mnc >> 5, zc);
          } else if (!p.a.mn_major && p.a.zmode != kZMNSeg) {
            operand_coords(p.a.zmode, p.a.seg, z, k0, m0, &kc, &mnc, &zc);
            if (kp.a_pair) {
              ld3(smem_u32(st), &mAh, fb, kc, mnc, 0);   // unbatched: the third coordinate is the plane
            } else {
              ld3(smem_u32(st), &mAh, fb, kc, mnc, zc);
              ld3(smem_u32(st + kTileBytesA), &mAl, fb, kc, mnc, zc);
            }
          } else {
            for (int j = 0; j < BM / 32; ++j) {
              operand_coords(p.a.zmode, p.a.seg, z, k0, m0 + 32 * j, &kc, &mnc, &zc);
              int x = p.a.mn_major ? mnc : kc, y = p.a.mn_major ? kc : mnc;
              ld3(smem_u32(st + j * kChunk), &mAh, fb, x, y, zc);
              ld3(smem_u32(st + kTileBytesA + j * kChunk), &mAl, fb, x, y, zc);
            }
          }
          uint8_t* sb = st + 2 * kTileBytesA;
          if (kp.b_chunked) {
            operand_coords(p.b.zmode, p.b.seg, z, k0, n0, &kc, &mnc, &zc);
            ld4(smem_u32(sb), &mBh, fb, 0, kc, mnc >> 5, zc);
            ld4(smem_u32(sb + kTileBytesB), &mBl, fb, 0, kc, mnc >> 5, zc);
          } else if (!p.b.mn_major && p.b.zmode != kZMNSeg && kp.b_pair) {
            operand_coords(p.b.zmode, p.b.seg, z, k0, n0, &kc, &mnc, &zc);
            ld3(smem_u32(sb), &mBh, fb, kc, mnc, 0);   // unbatched: the third coordinate is the plane
          } else if (!p.b.mn_major && p.b.zmode != kZMNSeg) {
            operand_coords(p.b.zmode, p.b.seg, z, k0, n0, &kc, &mnc, &zc);
            ld3(smem_u32(sb), &mBh, fb, kc, mnc, zc);
            ld3(smem_u32(sb + kTileBytesB), &mBl, fb, kc, mnc, zc);
          } else {
            for (int j = 0; j < BNL / 32; ++j) {
              operand_coords(p.b.zmode, p.b.seg, z, k0, n0 + 32 * j, &kc, &mnc, &zc);
              int x = p.b.mn_major ? mnc : kc, y = p.b.mn_major ? kc : mnc;
              ld3(smem_u32(sb + j * kChunk), &mBh, fb, x, y, zc);
              ld3(smem_u32(sb + kTileBytesB + j * kChunk), &mBl, fb, x, y, zc);
            }
          }
        }
      }
      if (*abort_flag) {
        // every issued stage must land before the CTA exits.  A pair's copies
        // count on rank 0's barrier only: rank 0 waits for its stages (both
        // CTAs' bytes, bounded as a whole), rank 1, which cannot observe its
        // own copies, waits a fixed 200 us (a copy takes microseconds).
        uint32_t lo = it > (uint32_t)STAGES ? it - STAGES : 0;
        if (PAIR && rank != 0) {
          const uint64_t t0 = gtimer();
          while (gtimer() - t0 < 200000ull) {}
        } else {
          const uint64_t t0 = gtimer();
          for (uint32_t q = lo; q < it; ++q)
            while (!mbar_try(smem_u32(&full[q % STAGES]), (q / STAGES) & 1) && gtimer() - t0 < kWaitNs) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (a pair: rank 0) ----------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_tf32(p.a.mn_major, p.b.mn_major, BN, PAIR ? 2 * BM : BM);
      // Descriptors of stage 0's tiles, built once.  A descriptor's address
      // field is (byte address / 16) in its low 14 bits and every shared
      // address here is below 256 KB, so a stage or k-step is a plain add of
      // (byte offset / 16): the issue loop spends no instructions on building
      // descriptors, and one thread keeps the tensor pipe fed.
      const uint32_t s0 = smem_u32(smem);
      const uint64_t da0 = p.a.mn_major ? desc_mn<BK>(s0, 0) : desc_k<BK>(s0, 0);
      const uint64_t db0 = p.b.mn_major ? desc_mn<BK>(s0 + 2 * kTileBytesA, 0)
                                        : desc_k<BK>(s0 + 2 * kTileBytesA, 0);
      const uint32_t ka = p.a.mn_major ? 1024 / 16 : 32 / 16;   // k-step of 8: 8 rows (MN) or 32 B (K)
      const uint32_t kbs = p.b.mn_major ? 1024 / 16 : 32 / 16;
      constexpr uint32_t kLoA = kTileBytesA / 16, kLoB = kTileBytesB / 16, kStage16 = kStageBytes / 16;
      // which tile of a stage holds which plane (a paired box puts the lower
      // address first, which may be the lo plane)
      const uint64_t a_hi = kp.a_swap ? kLoA : 0, a_lo = kp.a_swap ? 0 : kLoA;
      const uint64_t b_hi = kp.b_swap ? kLoB : 0, b_lo = kp.b_swap ? 0 : kLoB;
      uint32_t it = 0, local = 0;
      bool ok = true, issued = false;
      for (int unit = grp; unit < total && ok; unit += ngrp) {
        Unit un;
        if (!unit_of(kp, unit, un)) continue;
        uint32_t b = local & 1, u = local >> 1;
        ++local;
        if (u >= 1 && !(PAIR ? mbar_wait_cluster(smem_u32(&acce[b]), (u - 1) & 1, abort_flag, kp.err, 14)
                             : mbar_wait(smem_u32(&acce[b]), (u - 1) & 1, abort_flag, kp.err, 14))) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dacc = tmem + b * BN;
        const int kb_lo = un.kb_lo, kb_hi = un.kb_hi;
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, kp.err, 12)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t sa = da0 + (uint64_t)(s * kStage16), sbb = db0 + (uint64_t)(s * kStage16);
          const uint64_t dah = sa + a_hi, dal = sa + a_lo, dbh = sbb + b_hi, dbl = sbb + b_lo;
          auto mma = [&](uint64_t da, uint64_t db, uint32_t acc) {
            if constexpr (PAIR) mma_tf32_pair(dacc, da, db, idesc, acc);
            else mma_tf32(dacc, da, db, idesc, acc);
          };
          mma(dal, dbh, kb > kb_lo ? 1u : 0u);   // small terms first
          mma(dah, dbl, 1u);
          mma(dah, dbh, 1u);
#pragma unroll
          for (int kk = 1; kk < BK / 8; ++kk) {
            const uint64_t oa = (uint64_t)(kk * ka), ob = (uint64_t)(kk * kbs);
            mma(dal + oa, dbh + ob, 1u);
            mma(dah + oa, dbl + ob, 1u);
            mma(dah + oa, dbh + ob, 1u);
          }
          issued = true;
          // frees the stage (in both CTAs of a pair) when these MMAs finish
          if constexpr (PAIR) mma_commit_pair_both(smem_u32(&empty[s]));
          else mma_commit(smem_u32(&empty[s]));
        }
        if (ok) {
          if constexpr (PAIR) mma_commit_pair_both(smem_u32(&accf[b]));
          else mma_commit(smem_u32(&accf[b]));
        }
      }
      if ((PAIR || !ok) && issued) {
        // no MMA may be in flight when TMEM is freed; a pair always drains, so
        // that no MMA or commit touches rank 1 after the closing cluster barrier
        if constexpr (PAIR) mma_commit_pair(smem_u32(drain));
        else mma_commit(smem_u32(drain));
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(drain), 0) && gtimer() - t0 < kWaitNs) {}
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> global ----------------
    // Warp w reads TMEM lane quarter (w % 4) (its 32 tile rows, one per lane)
    // and, with 8 epilogue warps, column half (w - 2) / 4.  Auxiliary inputs of a 32-column
    // chunk are loaded before any of its stores so the loads overlap.
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    constexpr int kCols = BN * 4 / epi_warps(EPI);      // columns per epilogue warp
    const int chalf = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const bool contig = (p.on.d1 % 32 == 0) && (p.on.d2 % 32 == 0) && p.on.s3 == 1;
    const int rsub = lane >> 3, cgr = lane & 7, csub = cgr * 4;   // staged layout: lane's row group / columns
    uint32_t local = 0;
    for (int unit = grp; unit < total; unit += ngrp) {
      Unit un;
      if (!unit_of(kp, unit, un)) continue;
      uint32_t b = local & 1, u = local >> 1;
      ++local;
      if (!mbar_wait(smem_u32(&accf[b]), u & 1, abort_flag, kp.err, 13)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int z = un.z, m0 = un.m0 + (int)rank * BM, n0 = un.n0;   // this CTA's 128 rows
      const int m = m0 + row;
      const int64_t zm_z = lay(p.oz, z);
      const int64_t zm_off = zm_z + lay(p.om, m);
      int64_t zm[8];                  // staged path: output offsets of rows quarter*32 + 4t + rsub
      float rvs[8];
      if (kp.staged && splits == 1) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int mm = m0 + quarter * 32 + 4 * t + rsub;
          zm[t] = mm < p.M ? zm_z + lay(p.om, mm) : -1;
          rvs[t] = (EPI == kEpiSoftmaxBwd && mm < p.M) ? p.rowv[(int64_t)z * p.M + mm] : 0.0f;
        }
      }
#pragma unroll 1
      for (int c0 = chalf * kCols; c0 < (chalf + 1) * kCols; c0 += 32) {
        uint32_t r[32];
        uint32_t taddr = tmem + b * BN + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
              "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
              "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
              "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
              "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (splits > 1) {
          // raw partial tile, row-major [BM][BN]; k_splitk_reduce applies the epilogue
          float4* dst = reinterpret_cast<float4*>(kp.ws + (size_t)unit * (BM * BN) + row * BN + c0);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            dst[j / 4] = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                     __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          continue;
        }
        if (kp.staged) {
          // transpose the 32x32 chunk through smem: granule g of row r sits at
          // g ^ (r & 7) (conflict-free float4 both ways); each lane then owns 4
          // consecutive columns of rows 4t + rsub, so loads and stores are
          // 4 rows x 128 contiguous bytes per instruction
          float* wst = reinterpret_cast<float*>(bar_area + 256) + (warp - 2) * kEpiWarpFloats;
          float4* wrow = reinterpret_cast<float4*>(wst + lane * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            wrow[j ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          __syncwarp();
          const int nb = n0 + c0 + csub;
          const int64_t n_off = lay(p.on, nb);
          const bool vec = nb + 4 <= p.N;
          float4 ax[8], axl[8];
          if (EPI == kEpiResid || EPI == kEpiGeluBwd || EPI == kEpiSoftmaxBwd) {
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (zm[t] >= 0 && vec && ((zm[t] + n_off) & 3) == 0)
                ax[t] = __ldg(reinterpret_cast<const float4*>(p.aux + zm[t] + n_off));
          }
          if (EPI == kEpiSoftmaxBwd) {
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (zm[t] >= 0 && vec && ((zm[t] + n_off) & 3) == 0)
                axl[t] = __ldg(reinterpret_cast<const float4*>(p.aux_lo + zm[t] + n_off));
          }
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const int rr = 4 * t + rsub;
            const float4 v = *reinterpret_cast<const float4*>(wst + rr * 32 + ((cgr ^ (rr & 7)) << 2));
            if (zm[t] < 0) continue;
            const int64_t base = zm[t] + n_off;
            const float rv = EPI == kEpiSoftmaxBwd ? rvs[t] : 0.0f;
            if (vec && (base & 3) == 0) {
              epi_store4<EPI>(p, base, v, ax[t], axl[t], rv);
            } else {
              const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (nb + j < p.N) epi_store1<EPI>(p, base + j, vv[j], rv);
            }
          }
          __syncwarp();   // the staging block is rewritten by the next chunk
          continue;
        }
        if (m >= p.M) continue;
        const int nb = n0 + c0;
        const int64_t base = zm_off + lay(p.on, nb);
        const float rv = EPI == kEpiSoftmaxBwd ? p.rowv[(int64_t)z * p.M + m] : 0.0f;
        if (contig && nb + 32 <= p.N && (base & 3) == 0) {
          float4 ax[8], axl[8];
          if (EPI == kEpiResid || EPI == kEpiGeluBwd || EPI == kEpiSoftmaxBwd) {
#pragma unroll
            for (int j = 0; j < 8; ++j) ax[j] = __ldg(reinterpret_cast<const float4*>(p.aux + base) + j);
          }
          if (EPI == kEpiSoftmaxBwd) {
#pragma unroll
            for (int j = 0; j < 8; ++j) axl[j] = __ldg(reinterpret_cast<const float4*>(p.aux_lo + base) + j);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            epi_store4<EPI>(p, base + 4 * j,
                            make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                        __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])),
                            ax[j], axl[j], rv);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < p.N)
              epi_store1<EPI>(p, contig ? base + j : zm_off + lay(p.on, nb + j), __uint_as_float(r[j]), rv);
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(cluster_addr(smem_u32(&acce[b]), 0));   // rank 0 reuses the columns
        else mbar_arrive(smem_u32(&acce[b]));
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(done));
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  // lane 0 of the producer and MMA warps ran the role loops alone: the warps
  // reconverge before the CTA barrier
  __syncwarp();
  __syncthreads();
  // a pair: rank 0 has drained its MMAs and both CTAs' epilogues and copies
  // are done before either CTA frees its tensor memory or exits
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    // TMEM is freed only after every epilogue warp said it finished reading it
    // (an explicit barrier: the CTA barrier alone was seen to release early)
    mbar_wait_bounded(smem_u32(done), 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(kTmemCols));
  }
}

// ---- split-K: sum the K slices of each tile in slice order (deterministic),
// then the same epilogue as the GEMM.  One thread per 4 columns of a tile row.
template <int EPI>
__global__ void k_splitk_reduce(const TcKernelParams kp) {
  const TcProblem& p = kp.pr;
  const int per_batch = kp.tiles_m * kp.tiles_n;
  const int bn = kp.bn, tsz = BM * bn;
  const int64_t chunks = (int64_t)per_batch * p.batch * (tsz / 4);
  const bool contig4 = (p.on.d1 % 4 == 0) && (p.on.d2 % 4 == 0) && p.on.s3 == 1;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < chunks;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int tile = (int)(q / (tsz / 4));
    const int e = (int)(q % (tsz / 4)) * 4;    // element offset inside the tile
    const int r = e / bn, c = e % bn;
    const int z = tile / per_batch, rem = tile % per_batch;
    const int m = (rem / kp.tiles_n) * BM + r, n = (rem % kp.tiles_n) * bn + c;
    if (m >= p.M || n >= p.N) continue;
    const float4* src = reinterpret_cast<const float4*>(kp.ws + (size_t)tile * kp.splits * tsz + e);
    const size_t sstep = (size_t)(tsz / 4);
    float4 v = src[0];
    int sl = 1;
    // eight slices' loads in flight at a time, added in slice order (the same
    // sums, bit for bit, as one slice at a time)
    for (; sl + 8 <= kp.splits; sl += 8) {
      float4 t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = src[(size_t)(sl + j) * sstep];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v.x += t[j].x; v.y += t[j].y; v.z += t[j].z; v.w += t[j].w;
      }
    }
    for (; sl < kp.splits; ++sl) {
      const float4 t = src[(size_t)sl * sstep];
      v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
    }
    const int64_t zm = lay(p.oz, z) + lay(p.om, m);
    const int64_t base = zm + lay(p.on, n);
    const float rv = EPI == kEpiSoftmaxBwd ? p.rowv[(int64_t)z * p.M + m] : 0.0f;
    if (contig4 && n + 4 <= p.N && (base & 3) == 0) {
      float4 ax = make_float4(0.f, 0.f, 0.f, 0.f), axl = ax;
      if (EPI == kEpiResid || EPI == kEpiGeluBwd || EPI == kEpiSoftmaxBwd)
        ax = *reinterpret_cast<const float4*>(p.aux + base);
      if (EPI == kEpiSoftmaxBwd) axl = *reinterpret_cast<const float4*>(p.aux_lo + base);
      epi_store4<EPI>(p, base, v, ax, axl, rv);
    } else {
      const float vv[4] = {v.x, v.y, v.z, v.w};
      for (int j = 0; j < 4 && n + j < p.N; ++j)
        epi_store1<EPI>(p, contig4 ? base + j : zm + lay(p.on, n + j), vv[j], rv);
    }
  }
}

// ---- operand split: hi = tf32_rn(x), lo = tf32_rn(x - hi); one block per
// row chunk of 1024 columns, pitch padded to a multiple of 4 (zero-filled) ----
__global__ void k_split_tf32(const float* __restrict__ src, int64_t rows, int64_t cols, int64_t ld,
                             int64_t sstride, float* __restrict__ hi, float* __restrict__ lo,
                             int64_t pitch, bool vec) {
  int64_t row = blockIdx.x;                 // batch * rows + r
  int64_t c = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (c >= pitch) return;
  int64_t b = row / rows, r = row - b * rows;
  const float* s = src + b * sstride + r * ld;
  float x[4];
  if (vec && c + 4 <= cols) {
    float4 v = *reinterpret_cast<const float4*>(s + c);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) x[q] = c + q < cols ? s[c + q] : 0.0f;
  }
  float h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    h[q] = tf32_rn(x[q]);
    l[q] = tf32_rn(x[q] - h[q]);
  }
  *reinterpret_cast<float4*>(hi + row * pitch + c) = make_float4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<float4*>(lo + row * pitch + c) = make_float4(l[0], l[1], l[2], l[3]);
}

// ---- operand split through a strided view: planes [nz][n_outer][pitch],
// element (z, o, i) read at base + z.at(z) + outer.at(o) + inner.at(i) and
// multiplied by *scale, or by colscale[operand column], when given (one f32
// multiply, as the materialised product would be); pitch padding is
// zero-filled.  One block row per plane row, 1024 inner elements per block
// (four per thread).
struct SplitGeom {
  const float* base;
  const float* scale;
  const float* colscale;
  bool cs_inner;   // the operand's columns are the planes' inner index (else the outer)
  int64_t n_outer, n_inner, pitch;
  ViewDim z, outer, inner;
  bool vec;   // inner runs of 4 are contiguous and 16-byte aligned
};

// Division of 32-bit indices by a divisor fixed at launch, by multiply and
// shift (Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994, the round-up variant): with s = ceil(log2 d) and
// m = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s for all
// n, d < 2^31.  A 64-bit division costs dozens of instructions; the split of a
// viewed operand does three or four per four elements.
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t dv) : d(dv) {
    while (s < 32 && (1ull << s) < dv) ++s;
    m = (uint32_t)(((1ull << 32) * ((1ull << s) - dv)) / dv + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> s; }
};
struct ViewDim32 {
  FastDiv fd;
  bool has_div = false;
  int64_t hi = 0, lo = 0;
  ViewDim32() = default;
  explicit ViewDim32(const ViewDim& v) : fd(v.div ? (uint32_t)v.div : 1u), has_div(v.div != 0), hi(v.hi), lo(v.lo) {}
  __device__ __forceinline__ int64_t at(uint32_t i) const {
    if (!has_div) return (int64_t)i * lo;
    const uint32_t q = fd.div(i);
    return (int64_t)q * hi + (int64_t)(i - q * fd.d) * lo;
  }
};
struct SplitGeom32 {
  const float* base;
  const float* scale;
  const float* colscale;
  bool cs_inner;
  uint32_t n_inner, pitch;
  FastDiv cpr, n_outer;
  ViewDim32 z, outer, inner;
  bool vec;
};

// k_split_view with every index below 2^31: the same elements, values and
// plane layout, indexed by FastDiv.  causal_T > 0 (the operand is a [T, T]
// causal-zero block read by a GEMM that clips its K ranges to 128-row tiles):
// row o's columns from (o / 128 + 1) * 128 on are never read and not written.
__global__ void k_split_view32(SplitGeom32 g, float* __restrict__ hi, float* __restrict__ lo, uint32_t total,
                               uint32_t causal_T) {
  for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < total; q += gridDim.x * blockDim.x) {
    const uint32_t row = g.cpr.div(q), c = (q - row * g.cpr.d) * 4;
    const uint32_t zi = g.n_outer.div(row), o = row - zi * g.n_outer.d;
    if (causal_T && c >= ((o >> 7) + 1) * 128) continue;
    const float* s = g.base + g.z.at(zi) + g.outer.at(o);
    float x[4];
    if (g.vec && c + 4 <= g.n_inner) {
      const float4 v = *reinterpret_cast<const float4*>(s + g.inner.at(c));
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = c + k < g.n_inner ? s[g.inner.at(c + k)] : 0.0f;
    }
    if (g.scale) {
      const float sc = *g.scale;
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(x[k], sc);
    }
    if (g.colscale) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (c + k < g.n_inner) x[k] = __fmul_rn(x[k], g.colscale[g.cs_inner ? c + k : o]);
    }
    float h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h[k] = tf32_rn(x[k]);
      l[k] = tf32_rn(x[k] - h[k]);
    }
    const size_t at = (size_t)row * g.pitch + c;
    *reinterpret_cast<float4*>(hi + at) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + at) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

__global__ void k_split_view(SplitGeom g, float* __restrict__ hi, float* __restrict__ lo, int64_t rows_total) {
  // one thread per four consecutive plane elements, over all rows (a row of
  // a narrow operand is only a few chunks wide)
  const int64_t cpr = g.pitch >> 2;   // chunks per plane row
  const int64_t total = rows_total * cpr;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = q / cpr, c = (q - row * cpr) * 4;
    const int64_t zi = row / g.n_outer, o = row - zi * g.n_outer;
    const float* s = g.base + g.z.at(zi) + g.outer.at(o);
    float x[4];
    if (g.vec && c + 4 <= g.n_inner) {
      const float4 v = *reinterpret_cast<const float4*>(s + g.inner.at(c));
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = c + k < g.n_inner ? s[g.inner.at(c + k)] : 0.0f;
    }
    if (g.scale) {
      const float sc = *g.scale;
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(x[k], sc);
    }
    if (g.colscale) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (c + k < g.n_inner) x[k] = __fmul_rn(x[k], g.colscale[g.cs_inner ? c + k : o]);
    }
    float h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h[k] = tf32_rn(x[k]);
      l[k] = tf32_rn(x[k] - h[k]);
    }
    *reinterpret_cast<float4*>(hi + row * g.pitch + c) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + row * g.pitch + c) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// ---- operand gather into a contiguous [nz][rows][cols] stack (the SIMT path
// reads plain row-major operands), scaled like k_split_view
__global__ void k_operand_gather(GemmOperand o, float* __restrict__ out, int64_t n) {
  for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n; f += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = f % o.cols, rz = f / o.cols, r = rz % o.rows, zi = rz / o.rows;
    float x = o.base[o.z.at(zi) + o.r.at(r) + o.c.at(c)];
    if (o.scale_dev) x = __fmul_rn(x, *o.scale_dev);
    if (o.colscale_dev) x = __fmul_rn(x, o.colscale_dev[c]);
    out[f] = x;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

void load_encoder() {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    MALUS_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) panic("cuTensorMapEncodeTiled unavailable");
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  });
}

}  // namespace

// Generic f32 tensor map (rank 2..5; strides in bytes for dims 1..rank-1).
CUtensorMap encode_f32_map(int rank, const void* base, const uint64_t* dims, const uint64_t* strides,
                           const uint32_t* box, int swizzle) {
  load_encoder();
  CUtensorMap m;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) { d[i] = dims[i]; b[i] = box[i]; es[i] = 1; }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, (void*)base, d, st, b, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) panic("cuTensorMapEncodeTiled (rank %d) failed (%d)", rank, (int)r);
  return m;
}

namespace {

// 3-D f32 map {d0 (contiguous), d1, d2}, box {b0, b1, 1}: K-major tiles use the
// 128-byte (b0 = 32) or 64-byte (b0 = 16) swizzle with 16-byte granules,
// MN-major tiles the 128-byte swizzle with 32-byte granules.
CUtensorMap make_map(const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t pitch_bytes,
                     uint64_t plane_bytes, uint32_t b0, uint32_t b1, bool mn_major) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {pitch_bytes, plane_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                 : (b0 == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B),
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) panic("cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

// Map of one operand plane.  Stored matrix: nz slices of rows x cols with the
// given pitch; K-major operands are {cols=K, rows=MN}, MN-major {cols=MN, rows=K}.
// An MN-major operand whose columns are whole 32-element chunks (and whose
// segments, if any, are whole tiles of width tile_mn) is read as one box per
// plane: a 4-D view {32 columns, K rows, column chunks, slices} with box
// {32, 32, tile_mn / 32, 1} lands in shared memory as [chunk][k][32], the same
// swizzled layout that separate 32-wide boxes produce.  The view never
// addresses past a row's columns.
bool mn_chunked(const TcOperand& o, int tile_mn) {
  return o.mn_major && o.cols % 32 == 0 && (o.zmode != kZMNSeg || o.seg % tile_mn == 0);
}

CUtensorMap chunked_map(const TcOperand& o, const float* plane, uint64_t pitch_bytes,
                        uint64_t plane_bytes, int tile_mn, int bk) {
  CUtensorMap m;
  cuuint64_t dims[4] = {32, (cuuint64_t)o.rows, (cuuint64_t)(o.cols / 32),
                        (cuuint64_t)std::max(1, o.nz)};
  cuuint64_t strides[3] = {pitch_bytes, 128, plane_bytes};
  cuuint32_t box[4] = {32, (cuuint32_t)bk, (cuuint32_t)(tile_mn / 32), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)plane, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) panic("cuTensorMapEncodeTiled (chunked MN-major view) failed (%d)", (int)r);
  return m;
}

// Both planes of an operand in one tensor map: one more (outermost) dimension,
// the plane, whose stride is the distance between the planes and whose base
// is the lower one; a stage's hi and lo tiles then arrive in one box (half the
// TMA requests: each box carries a fixed issue cost on top of its bytes).
// Used only for K-major, unsegmented operands whose every box lies inside the
// tensor (rows a multiple of the tile, K a multiple of the k-block), with the
// distance a multiple of 16 bytes below 2^40.  The MN-major chunked view is
// never paired: a paired 5-D box reaching past a batched operand's columns
// made an illegal memory access.
bool pair_planes(const TcOperand& o, int tile_mn, int bk, bool* swap, uint64_t* delta) {
  const bool whole = !o.mn_major && o.zmode == kZNone && o.rows % tile_mn == 0 && o.cols % bk == 0;
  const uint64_t h = (uint64_t)(uintptr_t)o.hi, l = (uint64_t)(uintptr_t)o.lo;
  const uint64_t d = h > l ? h - l : l - h;
  if (!whole || d == 0 || d % 16 || d >= (1ull << 40)) return false;
  *swap = l < h;
  *delta = d;
  return true;
}

CUtensorMap paired_map(const TcOperand& o, int tile_mn, int bk, uint64_t delta) {
  const uint64_t pb = (uint64_t)o.pitch * 4;
  const void* base = std::min(o.hi, o.lo);
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)o.cols, (cuuint64_t)o.rows, 2};
  cuuint64_t strides[2] = {pb, delta};
  cuuint32_t box[3] = {(cuuint32_t)bk, (cuuint32_t)tile_mn, 2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, bk == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) panic("cuTensorMapEncodeTiled (paired planes) failed (%d)", (int)r);
  return m;
}

// tile_mn: the operand's tile extent along M (A: BM) or N (B: the tile width);
// bk: the k-block depth.
CUtensorMap operand_map(const TcOperand& o, const float* plane, int tile_mn, int bk) {
  uint64_t pb = (uint64_t)o.pitch * 4;
  uint64_t zb = (uint64_t)o.zstride * 4;
  if (o.nz > 1 && (zb % 16 != 0)) panic("gemm operand slice stride %lld is not 16-byte aligned", (long long)o.zstride);
  if (o.nz <= 1) zb = pb * (uint64_t)o.rows;
  if (mn_chunked(o, tile_mn)) return chunked_map(o, plane, pb, std::max<uint64_t>(zb, 16), tile_mn, bk);
  // K-major boxes are bk (K) x tile_mn rows, or bk x 32 rows when the rows are
  // segmented; MN-major boxes 32 columns x bk rows
  if (o.mn_major)
    return make_map(plane, (uint64_t)o.cols, (uint64_t)o.rows, (uint64_t)std::max(1, o.nz), pb,
                    std::max<uint64_t>(zb, 16), 32, (uint32_t)bk, true);
  uint32_t box_rows = o.zmode == kZMNSeg ? 32 : (uint32_t)tile_mn;
  return make_map(plane, (uint64_t)o.cols, (uint64_t)o.rows, (uint64_t)std::max(1, o.nz), pb,
                  std::max<uint64_t>(zb, 16), (uint32_t)bk, box_rows, false);
}

int g_force_backend = -1;

// K slices for a problem of `tiles` output tiles and nk k-blocks: split only
// when the tiles fill less than half the SMs and every slice keeps >= 8 k-blocks
// (the weight gradients dW = X^T dY, whose K is the token count).
int splitk_for(int tiles, int nk) {
  if (tiles * 2 > kNumSMs || nk < 16) return 1;
  return std::max(1, std::min({kNumSMs / tiles, nk / 8, 64}));
}

// Tile shape (measured on the C4 GEMMs): width 256 when N is a whole number of
// 256-wide tiles and the problem splits along K (the N = 1536 weight gradient;
// for full grids such as MLP up it measured no faster and the GELU backward
// slower), else 192 when N is a whole number of 192-wide tiles and the grid is
// either full or split along K (N = 384, 1152, 1536), else 128.  k-block depth 16 with the 192- and 256-wide tiles
// (four stages instead of two) except for stores of tf32 planes, which measured
// faster at 32; 32 with the 128-wide tile.  MALUS_GEMM_BN / _BK override for
// tuning (192 also keeps N % 256 == 0 problems at 192).
struct TileShape { int bn, bk; };
TileShape tile_shape_for(const TcProblem& pr) {
  static int forced_bn = [] { const char* e = getenv("MALUS_GEMM_BN"); return e ? atoi(e) : 0; }();
  static int forced_bk = [] { const char* e = getenv("MALUS_GEMM_BK"); return e ? atoi(e) : 0; }();
  int bn = 128;
  auto fills = [&](int w) {   // w-wide tiles fill the SMs, or the problem splits along K
    long tiles = (long)((pr.M + BM - 1) / BM) * (pr.N / w) * pr.batch;
    return tiles >= kNumSMs || splitk_for((int)tiles, (pr.K + 15) / 16) > 1;
  };
  if (forced_bn == 128 || forced_bn == 192) {
    bn = forced_bn;
  } else if (pr.N <= 64) {
    bn = 64;                       // attention outputs (N = head size): no idle half tile
  } else if (!pr.causal && pr.N % 256 == 0 && forced_bn != 192 &&
             splitk_for((int)((pr.M + BM - 1) / BM * (pr.N / 256) * pr.batch), (pr.K + 15) / 16) > 1) {
    bn = 256;   // split-K (weight gradients): measured 11 % faster than 192 at C4's dW1
  } else if (!pr.causal && pr.N % 192 == 0 && fills(192)) {
    bn = 192;
  }
  int bk = (bn >= 192 && !(pr.epi == kEpiStore && pr.out_hi)) ? 16 : 32;
  // the 64-wide tile exists with depth 32 only: an override must not give it
  // tensor maps of another depth than the kernel's stages expect
  if ((forced_bk == 16 || forced_bk == 32) && bn != 64) bk = forced_bk;
  return {bn, bk};
}

// Device workspace for split-K partials, grown on demand (never shrinks).
float* splitk_workspace(size_t floats) {
  static float* buf[16] = {};
  static size_t cap[16] = {};
  int dev = 0;
  MALUS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) panic("split-K workspace: device index %d out of range", dev);
  if (floats > cap[dev]) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    MALUS_CUDA(cudaStreamIsCapturing(stream(), &cs));
    if (cs != cudaStreamCaptureStatusNone)
      panic("split-K workspace must grow during graph capture: run the sequence once before capturing it");
    MALUS_CUDA(cudaStreamSynchronize(stream()));   // the old buffer may still be in use
    if (buf[dev]) MALUS_CUDA(cudaFree(buf[dev]));
    MALUS_CUDA(cudaMalloc(&buf[dev], floats * sizeof(float)));
    cap[dev] = floats;
  }
  return buf[dev];
}

template <int EPI, int BNT, int BKT, bool PAIR>
void tc_smem_attr() {
  static bool attr = false;
  if (!attr) {
    MALUS_CUDA(cudaFuncSetAttribute(k_gemm_tc<EPI, BNT, BKT, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    TileCfg<BNT, BKT, PAIR>::kSmemBytes));
    attr = true;
  }
}

cudaLaunchConfig_t pair_config(dim3 grid, int threads, int smem, cudaLaunchAttribute* at) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream();
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cfg;
}

std::atomic<int> g_pair_mode{[] {
  const char* e = getenv("MALUS_GEMM_CTA2");
  return e ? (atoi(e) == 0 ? 0 : (atoi(e) == 1 ? 1 : -1)) : -1;
}()};

// CTA pairs that can be resident at once (one CTA per SM, both SMs of a TPC).
// Every pair instantiation has the same footprint class (one CTA per SM), so
// one query stands for all; 0 disables pairs.
int pair_clusters() {
  static int n = -1;
  if (n < 0) {
    using CF = TileCfg<192, 16, true>;
    tc_smem_attr<kEpiStore, 192, 16, true>();
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pair_config(dim3(2 * (kNumSMs / 2)), threads_tc(kEpiStore), CF::kSmemBytes, at);
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, k_gemm_tc<kEpiStore, 192, 16, true>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      c = 0;
    }
    n = std::min(c, kNumSMs / 2);
  }
  return n;
}

template <int EPI, int BNT, int BKT, bool PAIR>
void launch_tc(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh,
               const CUtensorMap& bl, const TcKernelParams& kp, int grid) {
  constexpr int smem = TileCfg<BNT, BKT, PAIR>::kSmemBytes;
  tc_smem_attr<EPI, BNT, BKT, PAIR>();
  if (PAIR) {   // grid = 2 x pairs, launched as 2-CTA clusters
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = pair_config(dim3(grid), threads_tc(EPI), smem, at);
    MALUS_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc<EPI, BNT, BKT, PAIR>, ah, al, bh, bl, kp));
  } else {
    k_gemm_tc<EPI, BNT, BKT, PAIR><<<grid, threads_tc(EPI), smem, stream()>>>(ah, al, bh, bl, kp);
  }
  if (kp.splits > 1) {
    int64_t chunks = (int64_t)kp.tiles_m * kp.tiles_n * kp.pr.batch * (BM * kp.bn / 4);
    unsigned g = (unsigned)std::min<int64_t>((chunks + 255) / 256, (int64_t)kNumSMs * 8);
    // algorithmic bytes: every partial tile read once, the result (f32 and/or
    // tf32 planes) written once, an auxiliary input read once
    const TcProblem& p = kp.pr;
    const double mn = (double)p.M * p.N * p.batch;
    const double bytes = 4.0 * (double)chunks * 4.0 * kp.splits + (p.out ? 4.0 * mn : 0.0) +
                         (p.out_hi ? 8.0 * mn : 0.0) + (p.aux ? 4.0 * mn : 0.0) + (p.aux_lo ? 4.0 * mn : 0.0);
    const int pid = prof_begin_named("k_splitk_reduce (within the GEMM time)", bytes);
    k_splitk_reduce<EPI><<<g, 256, 0, stream()>>>(kp);
    prof_end(pid);
  }
}

}  // namespace

void gemm_force_backend(int b) { g_force_backend = b; }

int gemm_backend_for(const GemmArgs& g) {
  static int env_force = [] {
    const char* e = getenv("MALUS_GEMM_BACKEND");  // "simt" or "tc"
    if (!e) return -1;
    return strcmp(e, "simt") == 0 ? 0 : (strcmp(e, "tc") == 0 ? 1 : -1);
  }();
  if (g_force_backend >= 0) return g_force_backend;
  if (env_force >= 0) return env_force;
  if (g.M < 64 || g.N < 16 || g.K < 16) return 0;
  double work = (double)g.M * g.N * g.K * g.batch;
  if (work < 4.0e6) return 0;
  return 1;
}

void tf32_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t batch,
                int64_t sstride, float* hi, float* lo, int64_t pitch) {
  int64_t nrow = rows * batch;
  if (!nrow || !pitch) return;
  bool vec = (ld % 4 == 0) && (sstride % 4 == 0) && (((uintptr_t)src & 15) == 0);
  dim3 grid((unsigned)nrow, (unsigned)((pitch + 1023) / 1024));
  k_split_tf32<<<grid, 256, 0, stream()>>>(src, rows, cols, ld, sstride, hi, lo, pitch, vec);
  count_launch();
  after_launch("k_split_tf32");
}

void gemm_tc_planes(const TcProblem& pr) {
  if (pr.M <= 0 || pr.N <= 0 || pr.batch <= 0) return;
  if (pr.K <= 0) panic("gemm_tc_planes with K=0");
  if (!pr.out && !pr.out_hi) panic("gemm_tc_planes: no output (out and out_hi are both null)");
  if ((pr.out_hi == nullptr) != (pr.out_lo == nullptr)) panic("gemm_tc_planes: out_hi/out_lo must come together");
  if ((pr.epi == kEpiResid || pr.epi == kEpiGeluBwd) && !pr.aux) panic("gemm_tc_planes: epilogue %d needs aux", pr.epi);
  if ((pr.epi == kEpiGelu || pr.epi == kEpiGeluBwd) && !pr.out_hi) panic("gemm_tc_planes: GELU epilogues write planes");
  if (pr.epi < kEpiStore || pr.epi > kEpiSoftmaxBwd) panic("gemm_tc_planes: epilogue %d", pr.epi);
  if (pr.epi == kEpiSoftmaxBwd && (!pr.aux || !pr.aux_lo || !pr.rowv))
    panic("gemm_tc_planes: softmax-backward epilogue needs P planes (aux, aux_lo) and rowv");
  if (!pr.a.hi || !pr.a.lo || !pr.b.hi || !pr.b.lo) panic("gemm_tc_planes: missing operand plane");
  if (pr.causal < 0 || pr.causal > kCausalAUpper) panic("gemm_tc_planes: causal mode %d", pr.causal);
  for (const TcOperand* o : {&pr.a, &pr.b})
    if ((o->zmode == kZKSeg || o->zmode == kZMNSeg) && (o->seg <= 0 || o->seg % 32 != 0))
      panic("gemm_tc_planes: segment width %d must be a positive multiple of 32", o->seg);
  load_encoder();
  const TileShape ts = tile_shape_for(pr);
  const int BN = ts.bn, BK = ts.bk;
  static const bool no_pair = [] { const char* e = getenv("MALUS_GEMM_PAIR"); return e && e[0] == '0'; }();
  bool a_swap = false, b_swap = false;
  uint64_t a_d = 0, b_d = 0;
  // CTA pairs (256 x BN tiles, one M = 256 MMA per k-step): unsplit,
  // non-causal problems whose M is whole 256-row tiles, with the 192-wide
  // tiles or the 128-wide ones of depth 32, K >= 256 and an epilogue without
  // an auxiliary input (plain store, GELU).  Measured on the C4 GEMMs: Q|K|V
  // 14 % and MLP up + GELU 7 % faster as pairs; the residual and
  // GELU-derivative epilogues (whose aux reads make the two coupled CTAs wait
  // on the slower one) 5-9 % slower, a K = 64 batched product 26 % slower.
  // Mode (malus_gemm_pair_mode, initially MALUS_GEMM_CTA2): -1 this rule,
  // 0 no pairs, 1 pairs for every problem of an eligible shape.
  const int mode = g_pair_mode.load(std::memory_order_relaxed);
  const int tiles128 = ((pr.M + BM - 1) / BM) * ((pr.N + BN - 1) / BN) * pr.batch;
  const bool measured_ok = (pr.epi == kEpiStore || pr.epi == kEpiGelu) && pr.K >= 256;
  const bool cta2 = mode != 0 && (mode == 1 || measured_ok) && !pr.causal && pr.M % (2 * BM) == 0 &&
                    (BN == 192 || (BN == 128 && BK == 32)) && splitk_for(tiles128, (pr.K + BK - 1) / BK) == 1 &&
                    pair_clusters() > 0;
  const int BNL = cta2 ? BN / 2 : BN;   // B rows each CTA loads
  const bool a_pair = !no_pair && pair_planes(pr.a, BM, BK, &a_swap, &a_d);
  const bool b_pair = !no_pair && pair_planes(pr.b, BNL, BK, &b_swap, &b_d);
  CUtensorMap ah = a_pair ? paired_map(pr.a, BM, BK, a_d) : operand_map(pr.a, pr.a.hi, BM, BK);
  CUtensorMap al = a_pair ? ah : operand_map(pr.a, pr.a.lo, BM, BK);
  CUtensorMap bh = b_pair ? paired_map(pr.b, BNL, BK, b_d) : operand_map(pr.b, pr.b.hi, BNL, BK);
  CUtensorMap bl = b_pair ? bh : operand_map(pr.b, pr.b.lo, BNL, BK);
  TcKernelParams kp;
  kp.a_pair = a_pair ? 1 : 0;
  kp.b_pair = b_pair ? 1 : 0;
  kp.a_swap = a_swap ? 1 : 0;
  kp.b_swap = b_swap ? 1 : 0;
  kp.pr = pr;
  kp.bn = BN;
  kp.bk = BK;
  kp.bm = cta2 ? 2 * BM : BM;
  kp.tiles_m = (pr.M + kp.bm - 1) / kp.bm;
  kp.tiles_n = (pr.N + BN - 1) / BN;
  kp.nk = (pr.K + BK - 1) / BK;
  kp.err = device_error_word();
  int tiles = kp.tiles_m * kp.tiles_n * pr.batch;
  kp.splits = pr.causal || cta2 ? 1 : splitk_for(tiles, kp.nk);
  {
    const bool contig = (pr.on.d1 % 32 == 0) && (pr.on.d2 % 32 == 0) && pr.on.s3 == 1;
    kp.staged = contig && (pr.epi != kEpiStore || pr.out_hi != nullptr) ? 1 : 0;
  }
  kp.a_chunked = mn_chunked(pr.a, BM) ? 1 : 0;
  kp.b_chunked = mn_chunked(pr.b, BNL) ? 1 : 0;
  kp.ws = kp.splits > 1 ? splitk_workspace((size_t)tiles * kp.splits * BM * BN) : nullptr;
  int total = tiles * kp.splits;
  // Static round-robin over units: for causal problems the per-batch pattern of
  // skipped tiles / short K ranges has period 2 or 4, so an odd grid (147)
  // spreads the light and heavy units evenly over the CTAs.
  int grid = cta2 ? 2 * std::min(total, pair_clusters()) : std::min(total, pr.causal ? kNumSMs - 1 : kNumSMs);
  double flops = 2.0 * pr.M * (double)pr.N * pr.K * pr.batch;
  if (pr.causal) {   // the work actually done: tiles and K ranges the mask leaves
    double f = 0.0;
    for (int tm = 0; tm < kp.tiles_m; ++tm)
      for (int tn = 0; tn < kp.tiles_n; ++tn) {
        int m0 = tm * BM, n0 = tn * BN;
        if (pr.causal == kCausalOut && n0 > m0 + BM - 1) continue;
        int lo = 0, hi = kp.nk;
        if (pr.causal == kCausalALower) hi = std::min(kp.nk, (m0 + BM + BK - 1) / BK);
        if (pr.causal == kCausalAUpper) lo = m0 / BK;
        double k = std::min(hi * BK, pr.K) - lo * BK;
        f += 2.0 * std::min(BM, pr.M - m0) * std::min(BN, pr.N - n0) * std::max(0.0, k);
      }
    flops = f * pr.batch;
  }
  // algorithmic bytes: both operands' hi/lo planes once, each output array and aux once
  const double mn = (double)pr.M * pr.N * pr.batch;
  const int arrays = (pr.out ? 1 : 0) + (pr.out_hi ? 2 : 0) + (pr.aux ? 1 : 0);
  int pid = prof_begin(0, flops, 8.0 * ((double)pr.M * pr.K + (double)pr.N * pr.K) * pr.batch +
                                     4.0 * mn * arrays);
  // the maps above were built for (BN, BK): the kernel launched must have the same stages
  if ((BN == 64 && BK != 32) || (cta2 && BN == 128 && BK != 32) || (BK != 16 && BK != 32))
    panic("gemm_tc_planes: no kernel for tile width %d with k-block depth %d%s", BN, BK, cta2 ? " (pairs)" : "");
#define MALUS_TC_EPI_SWITCH(BN_, BK_, P_)                                                 \
  switch (pr.epi) {                                                                      \
    case kEpiStore: launch_tc<kEpiStore, BN_, BK_, P_>(ah, al, bh, bl, kp, grid); break;     \
    case kEpiResid: launch_tc<kEpiResid, BN_, BK_, P_>(ah, al, bh, bl, kp, grid); break;     \
    case kEpiGelu: launch_tc<kEpiGelu, BN_, BK_, P_>(ah, al, bh, bl, kp, grid); break;       \
    case kEpiGeluBwd: launch_tc<kEpiGeluBwd, BN_, BK_, P_>(ah, al, bh, bl, kp, grid); break; \
    default: launch_tc<kEpiSoftmaxBwd, BN_, BK_, P_>(ah, al, bh, bl, kp, grid); break;       \
  }
  if (cta2) {
    if (BN == 192 && BK == 16) { MALUS_TC_EPI_SWITCH(192, 16, true) }
    else if (BN == 192) { MALUS_TC_EPI_SWITCH(192, 32, true) }
    else { MALUS_TC_EPI_SWITCH(128, 32, true) }
  }
  else if (BN == 64) { MALUS_TC_EPI_SWITCH(64, 32, false) }
  else if (BN == 256 && BK == 16) { MALUS_TC_EPI_SWITCH(256, 16, false) }
  else if (BN == 256) { MALUS_TC_EPI_SWITCH(256, 32, false) }
  else if (BN == 192 && BK == 16) { MALUS_TC_EPI_SWITCH(192, 16, false) }
  else if (BN == 192) { MALUS_TC_EPI_SWITCH(192, 32, false) }
  else if (BK == 16) { MALUS_TC_EPI_SWITCH(128, 16, false) }
  else { MALUS_TC_EPI_SWITCH(128, 32, false) }
#undef MALUS_TC_EPI_SWITCH
  count_launch(kp.splits > 1 ? 2 : 1);
  after_launch("k_gemm_tc");
  prof_end(pid);
}

GemmOperand plain_operand(const float* p, int64_t nz, int64_t rows, int64_t cols, int64_t ld,
                          int64_t sstride) {
  GemmOperand o;
  o.base = p;
  o.nz = nz;
  o.rows = rows;
  o.cols = cols;
  o.z = ViewDim{0, 0, nz > 1 ? sstride : 0};
  o.r = ViewDim{0, 0, ld};
  o.c = ViewDim{0, 0, 1};
  return o;
}

namespace {

bool is_plain(const GemmOperand& o) {
  return !o.scale_dev && !o.colscale_dev && o.z.div == 0 && o.r.div == 0 && o.c.div == 0 && o.c.lo == 1;
}

// ---------------------------------------------------------- plane cache
struct PlaneEntry {
  int64_t nz, rows, cols;
  ViewDim z, r, c;
  const float* scale;
  const float* colscale;
  float* mem;          // hi then lo, each nz * n_outer * pitch floats
  int64_t pitch;
  bool transposed;     // planes hold the operand's columns as rows
  int64_t causal_T;    // > 0: only the part a causally clipped GEMM reads was written
};
std::mutex g_pc_mu;
std::unordered_map<uint64_t, std::vector<PlaneEntry>> g_pc;

bool plane_cache_on() {
  static const bool on = [] { const char* e = getenv("MALUS_PLANE_CACHE"); return !(e && e[0] == '0'); }();
  return on;
}

bool same_dim(const ViewDim& a, const ViewDim& b) { return a.div == b.div && a.hi == b.hi && a.lo == b.lo; }

// A cached entry of the same operand; partially written planes serve only a
// consumer that clips its K ranges the same way (causal_T equal).
const PlaneEntry* pc_find(const GemmOperand& o, int64_t causal_T) {
  auto it = g_pc.find(o.key);
  if (it == g_pc.end()) return nullptr;
  for (const PlaneEntry& e : it->second)
    if (e.nz == o.nz && e.rows == o.rows && e.cols == o.cols && same_dim(e.z, o.z) && same_dim(e.r, o.r) &&
        same_dim(e.c, o.c) && e.scale == o.scale_dev && e.colscale == o.colscale_dev &&
        (e.causal_T == 0 || e.causal_T == causal_T))
      return &e;
  return nullptr;
}

// The tf32 planes of one operand.  They hold the operand's inner dimension
// contiguously: its columns, or its rows when only those are contiguous in
// memory (then *trans flips: the GEMM reads them with the other major-ness).
struct Planes {
  const float* hi;
  const float* lo;
  int64_t rows, cols, pitch;   // as stored in the planes
  void* tmp;                   // scratch to free after the GEMM (null: cached)
};

// causal_T > 0: the operand is the A of a GEMM clipped to the causal
// triangle of [causal_T, causal_T] blocks (128-row tiles); when the planes hold
// it as (query row, key column), the part past each tile's diagonal block is
// skipped.
Planes operand_planes(const GemmOperand& o, bool* trans, int64_t causal_T = 0) {
  const bool flip = o.c.lo != 1 && o.r.lo == 1;
  const int64_t n_outer = flip ? o.cols : o.rows, n_inner = flip ? o.rows : o.cols;
  const ViewDim outer = flip ? o.c : o.r, inner = flip ? o.r : o.c;
  const int64_t pitch = (n_inner + 3) & ~int64_t(3);
  if (flip) *trans = !*trans;
  // rows of the planes are the T queries, each with its T keys contiguous
  if (!(causal_T > 0 && n_outer == causal_T && n_inner == causal_T && inner.div == 0 && inner.lo == 1 &&
        outer.div == 0 && outer.lo == causal_T && causal_T % 128 == 0))
    causal_T = 0;
  std::lock_guard<std::mutex> lk(g_pc_mu);
  const bool cache = o.key != 0 && plane_cache_on();
  if (cache)
    if (const PlaneEntry* e = pc_find(o, causal_T)) {
      const int64_t n = o.nz * n_outer * e->pitch;
      return Planes{e->mem, e->mem + n, n_outer, n_inner, e->pitch, nullptr};
    }
  const int64_t n = o.nz * n_outer * pitch;
  float* mem = (float*)scratch_alloc((size_t)(2 * n) * sizeof(float) + 256);
  SplitGeom g;
  g.base = o.base;
  g.scale = o.scale_dev;
  g.colscale = o.colscale_dev;
  g.cs_inner = !flip;
  g.n_outer = n_outer;
  g.n_inner = n_inner;
  g.pitch = pitch;
  g.z = o.z;
  g.outer = outer;
  g.inner = inner;
  auto m4 = [](int64_t v) { return v % 4 == 0; };
  g.vec = inner.lo == 1 && (inner.div == 0 || (m4(inner.div) && m4(inner.hi))) && m4(outer.lo) &&
          (outer.div == 0 || m4(outer.hi)) && m4(o.z.lo) && (o.z.div == 0 || m4(o.z.hi)) &&
          ((uintptr_t)o.base & 15) == 0;
  if (o.nz * n_outer > 0 && pitch > 0) {
    const int64_t rows_total = o.nz * n_outer;
    const int64_t total = rows_total * (pitch / 4);
    constexpr int64_t k31 = (int64_t)1 << 31;
    auto fits = [&](const ViewDim& v) { return v.div >= 0 && v.div < k31; };
    if (rows_total * pitch < k31 && n_outer < k31 && fits(o.z) && fits(outer) && fits(inner)) {
      SplitGeom32 h;
      h.base = g.base;
      h.scale = g.scale;
      h.colscale = g.colscale;
      h.cs_inner = g.cs_inner;
      h.n_inner = (uint32_t)n_inner;
      h.pitch = (uint32_t)pitch;
      h.cpr = FastDiv((uint32_t)(pitch / 4));
      h.n_outer = FastDiv((uint32_t)n_outer);
      h.z = ViewDim32(o.z);
      h.outer = ViewDim32(outer);
      h.inner = ViewDim32(inner);
      h.vec = g.vec;
      k_split_view32<<<grid_for((size_t)total, 256), 256, 0, stream()>>>(h, mem, mem + n, (uint32_t)total,
                                                                           (uint32_t)causal_T);
      count_launch();
      after_launch("k_split_view32");
    } else {
      causal_T = 0;   // the 64-bit-index split writes every element
      k_split_view<<<grid_for((size_t)total, 256), 256, 0, stream()>>>(g, mem, mem + n, rows_total);
      count_launch();
      after_launch("k_split_view");
    }
  }
  if (cache) {
    g_pc[o.key].push_back(PlaneEntry{o.nz, o.rows, o.cols, o.z, o.r, o.c, o.scale_dev, o.colscale_dev, mem, pitch,
                                     flip, causal_T});
    return Planes{mem, mem + n, n_outer, n_inner, pitch, nullptr};
  }
  return Planes{mem, mem + n, n_outer, n_inner, pitch, mem};
}

// tensor_matmul / VJP path: the operands' planes (cached, or split now from
// their views), then one persistent GEMM with a plain row-major (batched) output.
void gemm_tc(const GemmArgs& g) {
  bool at = g.a_trans, bt = g.b_trans;
  const int causal = (g.a_zero == kCausalALower || g.a_zero == kCausalAUpper) && g.M == g.K ? g.a_zero : kCausalNone;
  int pid = prof_begin(1, 0.0, 12.0 * (double)(g.A.nz * g.A.rows * g.A.cols + g.B.nz * g.B.rows * g.B.cols));
  // A partial split serves clipped consumers only.  The probabilities P are
  // read only so (their planes come from the softmax itself); the scaled
  // score gradient dS * s is also the B operand of d(K^T) = Q^T (dS * s),
  // which reads it whole, so it is split whole once for both.
  const bool partial = causal != kCausalNone && !g.A.scale_dev;
  const Planes pa = operand_planes(g.A, &at, partial ? g.M : 0);
  const Planes pb = operand_planes(g.B, &bt);
  prof_end(pid);
  TcProblem pr{};
  pr.M = g.M; pr.N = g.N; pr.K = g.K; pr.batch = g.batch;
  pr.a = TcOperand{pa.hi, pa.lo, pa.rows, pa.cols, pa.pitch, (int)g.A.nz, pa.rows * pa.pitch, at,
                   g.A.nz > 1 ? kZBatch : kZNone, 0};
  pr.b = TcOperand{pb.hi, pb.lo, pb.rows, pb.cols, pb.pitch, (int)g.B.nz, pb.rows * pb.pitch, !bt,
                   g.B.nz > 1 ? kZBatch : kZNone, 0};
  pr.epi = kEpiStore;
  pr.oz = TcLayout{0, 0, 0, 0, g.batch > 1 ? g.strideC : 0};
  pr.om = TcLayout{0, 0, 0, 0, g.ldc};
  pr.on = TcLayout{0, 0, 0, 0, 1};
  pr.out = g.C;
  pr.alpha = g.alpha;
  pr.beta = g.beta;
  pr.causal = causal;
  gemm_tc_planes(pr);
  if (pa.tmp) scratch_free(pa.tmp);
  if (pb.tmp) scratch_free(pb.tmp);
}

// A contiguous copy of a non-plain operand for the SIMT path.
GemmOperand gathered(const GemmOperand& o, void** tmp) {
  const int64_t n = o.nz * o.rows * o.cols;
  float* buf = (float*)scratch_alloc((size_t)std::max<int64_t>(n, 1) * sizeof(float));
  if (n) {
    k_operand_gather<<<grid_for((size_t)n, 256), 256, 0, stream()>>>(o, buf, n);
    count_launch();
    after_launch("k_operand_gather");
  }
  *tmp = buf;
  return plain_operand(buf, o.nz, o.rows, o.cols, o.cols, o.rows * o.cols);
}

}  // namespace

void plane_cache_clear() {
  std::vector<float*> mem;
  {
    std::lock_guard<std::mutex> lk(g_pc_mu);
    for (auto& kv : g_pc)
      for (auto& e : kv.second) mem.push_back(e.mem);
    g_pc.clear();
  }
  for (float* m : mem) scratch_free(m);
}

float* plane_cache_prime(const GemmOperand& o, int64_t causal_T) {
  if (!plane_cache_on() || o.key == 0 || o.scale_dev || o.colscale_dev || o.cols % 4 != 0) return nullptr;
  const bool plain = o.c.div == 0 && o.c.lo == 1 && o.r.div == 0 && o.r.lo == o.cols &&
                     (o.nz == 1 || (o.z.div == 0 && o.z.lo == o.rows * o.cols));
  if (!plain) return nullptr;
  std::lock_guard<std::mutex> lk(g_pc_mu);
  if (pc_find(o, causal_T)) return nullptr;
  const int64_t n = o.nz * o.rows * o.cols;
  float* mem = (float*)scratch_alloc((size_t)(2 * n) * sizeof(float) + 256);
  g_pc[o.key].push_back(PlaneEntry{o.nz, o.rows, o.cols, o.z, o.r, o.c, nullptr, nullptr, mem, o.cols, false,
                                   causal_T});
  return mem;
}

void plane_cache_drop(uint64_t sid) {
  std::vector<float*> mem;
  {
    std::lock_guard<std::mutex> lk(g_pc_mu);
    auto it = g_pc.find(sid);
    if (it == g_pc.end()) return;
    for (auto& e : it->second) mem.push_back(e.mem);
    g_pc.erase(it);
  }
  for (float* m : mem) scratch_free(m);
}

void gemm(const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return;
  if (gemm_backend_for(g) == 1 && g.K > 0) {
    gemm_tc(g);
    return;
  }
  GemmArgs s = g;
  void *ta = nullptr, *tb_ = nullptr;
  if (!is_plain(s.A)) s.A = gathered(s.A, &ta);
  if (!is_plain(s.B)) s.B = gathered(s.B, &tb_);
  gemm_simt(s);
  if (ta) scratch_free(ta);
  if (tb_) scratch_free(tb_);
}

}  // namespace malus

extern "C" void malus_tc_gemm(const malus_tc_problem* q) {
  using namespace malus;
  auto op = [](const malus_tc_operand& o) {
    return TcOperand{o.hi, o.lo, o.rows, o.cols, o.pitch, o.nz, o.zstride, o.mn_major != 0,
                     o.zmode, o.seg};
  };
  TcProblem p{};
  p.M = q->M; p.N = q->N; p.K = q->K; p.batch = q->batch;
  p.a = op(q->a);
  p.b = op(q->b);
  p.epi = q->epi;
  auto L = [](const malus_tc_layout& l) { return TcLayout{l.d1, l.s1, l.d2, l.s2, l.s3}; };
  p.oz = L(q->oz);
  p.om = L(q->om);
  p.on = L(q->on);
  p.out = q->out; p.out_hi = q->out_hi; p.out_lo = q->out_lo; p.aux = q->aux;
  p.alpha = q->alpha; p.beta = q->beta;
  p.causal = q->causal;
  p.aux_lo = q->aux_lo;
  p.rowv = q->rowv;
  gemm_tc_planes(p);
}

extern "C" int32_t malus_gemm_pair_clusters(void) {
  if (malus::g_pair_mode.load() == 0) return 0;
  return malus::pair_clusters();
}

extern "C" int32_t malus_gemm_pair_mode(int32_t mode) {
  const int m = mode == 0 ? 0 : (mode == 1 ? 1 : -1);
  return malus::g_pair_mode.exchange(m);
}

extern "C" void malus_tf32_split(const float* src, int64_t rows, int64_t cols, int64_t ld,
                                 int64_t batch, int64_t sstride, float* hi, float* lo,
                                 int64_t pitch) {
  malus::tf32_split(src, rows, cols, ld, batch, sstride, hi, lo, pitch);
}
