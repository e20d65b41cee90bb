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

#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

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
  k_gemm_simt<<<grid, 256, 0, stream()>>>(g.M, g.N, g.K, g.A, g.lda, g.strideA, g.a_trans, g.B,
                                          g.ldb, g.strideB, g.b_trans, g.C, g.ldc, g.strideC,
                                          g.alpha, g.beta);
  count_launch();
  after_launch("k_gemm_simt");
  prof_end(pid);
}

// =============================================================== tcgen05
namespace {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int kTileBytesA = BM * BK * 4;  // 16 KB
constexpr int kTileBytesB = BN * BK * 4;  // 16 KB
constexpr int kStageBytes = 2 * kTileBytesA + 2 * kTileBytesB;
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
constexpr int kThreadsTC = 192;   // warp0 TMA, warp1 MMA+TMEM, warps2-5 epilogue
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s bound on every wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false (and records `code`) when the bound runs out
// or another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag,
                                          int32_t* err, int code) {
  if (mbar_try(a, parity)) return true;
  uint64_t t0 = gtimer();
  while (true) {
    if (mbar_try(a, parity)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > kWaitNs) {
      *abort_flag = 1;
      atomicExch(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t mbar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"((uint64_t)map), "r"(mbar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// UMMA shared-memory descriptor (version 1).  Layout type 2 is the 128-byte
// swizzle with 16-byte granules used for K-major tiles; layout type 1 is the
// 128-byte swizzle with 32-byte granules (4-row atom) that 32-bit (tf32)
// MN-major tiles require.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}
// K-major tile: rows of 128 B (32 tf32 along K), 8-row atoms 1 KB apart.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk) {
  return umma_desc(tile + kk * 32, 16, 1024, 2);
}
// MN-major tile: 32-element (128 B) MN chunks 4 KB apart (one TMA box each),
// K rows 128 B apart in 4-row (512 B) atoms; one MMA consumes 8 K rows.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int kk) {
  return umma_desc(tile + kk * 1024, 4096, 512, 1);
}

// Instruction descriptor: f32 accumulate, tf32 A/B, M=128, N=BN.
__host__ __device__ constexpr uint32_t idesc_tf32(bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
      : "memory");
}

struct TcParams {
  int M, N, K;
  bool a_mn, b_mn;          // operand is MN-major (stored transposed)
  bool a_batched, b_batched;
  float* C;
  int64_t ldc, strideC;
  float alpha, beta;
  int32_t* err;
};

// A map: K-major -> dims {K, M, batch}, box {32, 128, 1}
//        MN-major -> dims {M, K, batch}, box {32, 32, 1} issued BM/32 times
__global__ void __launch_bounds__(kThreadsTC, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
          const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl,
          TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* bar_area = smem + STAGES * kStageBytes;
  uint64_t* full = (uint64_t*)bar_area;
  uint64_t* empty = full + STAGES;
  uint64_t* accb = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(accb + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, bz = blockIdx.z;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accb), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        int s = kb % STAGES;
        uint32_t ph = (uint32_t)((kb / STAGES) & 1);
        if (kb >= STAGES) {
          if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag, p.err, 11)) break;
        }
        uint8_t* st = smem + s * kStageBytes;
        uint32_t fb = smem_u32(&full[s]);
        mbar_expect_tx(fb, kStageBytes);
        int k0 = kb * BK;
        int za = p.a_batched ? bz : 0, zb = p.b_batched ? bz : 0;
        if (!p.a_mn) {
          tma_load_3d(smem_u32(st), &mAh, fb, k0, m0, za);
          tma_load_3d(smem_u32(st + kTileBytesA), &mAl, fb, k0, m0, za);
        } else {
          for (int j = 0; j < BM / 32; ++j) {
            tma_load_3d(smem_u32(st + j * 4096), &mAh, fb, m0 + 32 * j, k0, za);
            tma_load_3d(smem_u32(st + kTileBytesA + j * 4096), &mAl, fb, m0 + 32 * j, k0, za);
          }
        }
        uint8_t* sb = st + 2 * kTileBytesA;
        if (!p.b_mn) {
          tma_load_3d(smem_u32(sb), &mBh, fb, k0, n0, zb);
          tma_load_3d(smem_u32(sb + kTileBytesB), &mBl, fb, k0, n0, zb);
        } else {
          for (int j = 0; j < BN / 32; ++j) {
            tma_load_3d(smem_u32(sb + j * 4096), &mBh, fb, n0 + 32 * j, k0, zb);
            tma_load_3d(smem_u32(sb + kTileBytesB + j * 4096), &mBl, fb, n0 + 32 * j, k0, zb);
          }
        }
        issued = kb + 1;
      }
      // Drain: every stage that was filled must have landed before exit.
      if (*abort_flag) {
        for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb) {
          int s = kb % STAGES;
          uint32_t ph = (uint32_t)((kb / STAGES) & 1);
          uint64_t t0 = gtimer();
          while (!mbar_try(smem_u32(&full[s]), ph) && gtimer() - t0 < kWaitNs) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(p.a_mn, p.b_mn);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        int s = kb % STAGES;
        uint32_t ph = (uint32_t)((kb / STAGES) & 1);
        if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, p.err, 12)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint8_t* st = smem + s * kStageBytes;
        uint32_t ah = smem_u32(st), al = smem_u32(st + kTileBytesA);
        uint32_t bh = smem_u32(st + 2 * kTileBytesA), bl = bh + kTileBytesB;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          uint64_t dah = p.a_mn ? desc_mnmajor(ah, kk) : desc_kmajor(ah, kk);
          uint64_t dal = p.a_mn ? desc_mnmajor(al, kk) : desc_kmajor(al, kk);
          uint64_t dbh = p.b_mn ? desc_mnmajor(bh, kk) : desc_kmajor(bh, kk);
          uint64_t dbl = p.b_mn ? desc_mnmajor(bl, kk) : desc_kmajor(bl, kk);
          uint32_t acc0 = (kb > 0 || kk > 0) ? 1u : 0u;
          mma_tf32(tmem, dal, dbh, idesc, acc0);   // small terms first
          mma_tf32(tmem, dah, dbl, idesc, 1u);
          mma_tf32(tmem, dah, dbh, idesc, 1u);
        }
        mma_commit(smem_u32(&empty[s]));   // frees the stage when these MMAs finish
      }
      // Signal the epilogue (also on abort, so no MMA is in flight at exit).
      mma_commit(smem_u32(accb));
      if (!ok) {
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(accb), 0) && gtimer() - t0 < kWaitNs) {}
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> global ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    bool ok = mbar_wait(smem_u32(accb), 0, abort_flag, p.err, 13);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && !*abort_flag) {
      const int m = m0 + row;
      float* crow = p.C + (int64_t)bz * p.strideC + (int64_t)m * p.ldc;
      const bool vec = (p.ldc % 4 == 0) && ((((uintptr_t)p.C) & 15) == 0) && (p.strideC % 4 == 0);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
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
        if (m < p.M) {
          const int nb = n0 + c0;
          if (vec && nb + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                     __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
              float4* dst = reinterpret_cast<float4*>(crow + nb + j);
              if (p.alpha != 1.0f) { v.x *= p.alpha; v.y *= p.alpha; v.z *= p.alpha; v.w *= p.alpha; }
              if (p.beta != 0.0f) {
                float4 o = *dst;
                v.x += p.beta * o.x; v.y += p.beta * o.y; v.z += p.beta * o.z; v.w += p.beta * o.w;
              }
              *dst = v;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              int n = nb + j;
              if (n < p.N) {
                float v = __uint_as_float(r[j]);
                if (p.alpha != 1.0f) v *= p.alpha;
                if (p.beta != 0.0f) v += p.beta * crow[n];
                crow[n] = v;
              }
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)BN));
  }
}

// ---- operand split: hi = tf32_rn(x), lo = tf32_rn(x - hi), padded pitch ----
__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void k_split_tf32(const float* __restrict__ src, int64_t rows, int64_t cols,
                             int64_t ld, int64_t sstride, float* __restrict__ hi,
                             float* __restrict__ lo, int64_t pitch, int64_t total) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t f = tid; f < total; f += step) {
    int64_t c = f % pitch;
    int64_t rb = f / pitch;        // batch*rows + r
    int64_t r = rb % rows, b = rb / rows;
    float x = c < cols ? src[b * sstride + r * ld + c] : 0.0f;
    float h = tf32_rn(x);
    hi[f] = h;
    lo[f] = tf32_rn(x - h);
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

// 3-D f32 map {d0 (contiguous), d1, d2}, box {b0, b1, 1}, 128-B swizzle with
// 16-byte granules (K-major tiles) or 32-byte granules (MN-major tiles).
CUtensorMap make_map(const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t pitch_bytes,
                     uint64_t plane_bytes, uint32_t b0, uint32_t b1, bool mn_major) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {pitch_bytes, plane_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) panic("cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

int g_force_backend = -1;

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

static void gemm_tc(const GemmArgs& g) {
  load_encoder();
  static bool attr_set = false;
  if (!attr_set) {
    MALUS_CUDA(cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set = true;
  }
  // Operand A as stored: rows x cols = (a_trans ? K x M : M x K)
  int64_t ar = g.a_trans ? g.K : g.M, ac = g.a_trans ? g.M : g.K;
  int64_t br = g.b_trans ? g.N : g.K, bc = g.b_trans ? g.K : g.N;
  int64_t ap = (ac + 3) & ~int64_t(3), bp = (bc + 3) & ~int64_t(3);
  int64_t abatch = g.strideA ? g.batch : 1, bbatch = g.strideB ? g.batch : 1;
  int64_t an = abatch * ar * ap, bn = bbatch * br * bp;
  float* ws = (float*)scratch_alloc((size_t)(2 * an + 2 * bn) * sizeof(float) + 256);
  float *ah = ws, *al = ws + an, *bh = ws + 2 * an, *bl = bh + bn;
  int pid = prof_begin(1, 0.0, 12.0 * (double)(an + bn));
  k_split_tf32<<<grid_for((size_t)an, 256), 256, 0, stream()>>>(g.A, ar, ac, g.lda, g.strideA, ah, al,
                                                               ap, an);
  k_split_tf32<<<grid_for((size_t)bn, 256), 256, 0, stream()>>>(g.B, br, bc, g.ldb, g.strideB, bh, bl,
                                                               bp, bn);
  count_launch(2);
  after_launch("k_split_tf32");
  prof_end(pid);
  // A: K-major (not transposed) -> {K, M, batch} box {32, 128}; MN-major -> {M, K, batch} box {32, 32}
  bool a_mn = g.a_trans, b_mn = !g.b_trans;
  CUtensorMap mah, mal, mbh, mbl;
  uint64_t apb = (uint64_t)ap * 4, bpb = (uint64_t)bp * 4;
  if (!a_mn) {
    mah = make_map(ah, ac, ar, abatch, apb, apb * ar, 32, BM, false);
    mal = make_map(al, ac, ar, abatch, apb, apb * ar, 32, BM, false);
  } else {
    mah = make_map(ah, ac, ar, abatch, apb, apb * ar, 32, 32, true);
    mal = make_map(al, ac, ar, abatch, apb, apb * ar, 32, 32, true);
  }
  if (!b_mn) {
    mbh = make_map(bh, bc, br, bbatch, bpb, bpb * br, 32, BN, false);
    mbl = make_map(bl, bc, br, bbatch, bpb, bpb * br, 32, BN, false);
  } else {
    mbh = make_map(bh, bc, br, bbatch, bpb, bpb * br, 32, 32, true);
    mbl = make_map(bl, bc, br, bbatch, bpb, bpb * br, 32, 32, true);
  }
  TcParams p;
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.a_mn = a_mn; p.b_mn = b_mn;
  p.a_batched = g.strideA != 0; p.b_batched = g.strideB != 0;
  p.C = g.C; p.ldc = g.ldc; p.strideC = g.strideC;
  p.alpha = g.alpha; p.beta = g.beta;
  p.err = device_error_word();
  dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.batch);
  pid = prof_begin(0, 2.0 * g.M * (double)g.N * g.K * g.batch,
                   4.0 * ((double)g.M * g.N * g.batch * (g.beta != 0.0f ? 2 : 1)) +
                       8.0 * (double)(an + bn));
  k_gemm_tc<<<grid, kThreadsTC, kSmemBytes, stream()>>>(mah, mal, mbh, mbl, p);
  count_launch();
  after_launch("k_gemm_tc");
  prof_end(pid);
  scratch_free(ws);
}

void gemm(const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return;
  if (gemm_backend_for(g) == 1 && g.K > 0) gemm_tc(g);
  else gemm_simt(g);
}

}  // namespace malus
