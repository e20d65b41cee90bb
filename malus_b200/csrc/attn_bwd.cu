// Fused causal attention backward on tcgen05 (3xTF32), two kernels that
// recompute the probabilities from the forward's row statistics, so no [T][T]
// tensor is read or written.
//
// Reference semantics: the VJP chain of the attention block of
// examples/nanogpt_modular.ml (bmm, scale, mask, softmax, bmm), with the bmm
// rules of tape.rs (matmul VJP) and the softmax rule of
// crates/malus-stdlib/stdlib/nn/softmax.ml (dS = P * (dP - rowsum(dP * P))):
//   P  = softmax(Q K^T * scale + mask)      recomputed as 2^(s*scale*log2 e - m2) * (1/l)
//   dP = dO V^T
//   D  = rowsum(dP * P) = rowsum(dO * O)    (O = P V, the forward's output)
//   dS = P * (dP - D) * scale               (the scale VJP folded in)
//   dQ = dS K,   dK = dS^T Q,   dV = P^T dO
//
// Both kernels: 352 threads — warps 0 and 10 TMA producers (independent
// rings), warp 1 TMEM owner and MMA issuer, warps 2-9 two groups of four row
// warps: one thread per stationary row (its TMEM lane), group g taking columns
// 32g..32g+31 of every 64-wide block.  Blocks are 64 wide so that each MMA
// (M = 128, N = 64, K = 8) carries enough work for its issue cost.  One
// stationary operand lives in tensor memory (the row threads load their own
// rows and store them with tcgen05.st; the MMA reads A from TMEM), which frees
// shared memory for the streamed blocks; the operands the threads compute
// (dS, P^T, dS^T) are written to TMEM as tf32 hi/lo planes over the scores they
// were computed from.
//
// k_attn_bwd_dq   (one CTA = one head x 128 queries): Q in TMEM, dO in shared
//   memory; 64-key blocks up to the diagonal stream K and V (K-major, two
//   stages) and K (MN-major).  S = Q K^T and dP = dO V^T go to two TMEM buffers
//   (one block ahead); the threads overwrite them with dS; dQ += dS K
//   accumulates in TMEM.  The threads also compute D for their rows and store it
//   for:
// k_attn_bwd_dkdv (one CTA = one head x 128 keys): K in TMEM, V in shared
//   memory; 64-query blocks from the diagonal on stream Q and dO in both majors.
//   S^T = K Q^T and dP^T = V dO^T; the threads overwrite them with P^T and
//   write dS^T; dV += P^T dO and dK += dS^T Q accumulate in TMEM.
// Every mbarrier wait is bounded; on timeout the CTA records an error, drains
// its copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "tc_common.cuh"

namespace malus {
namespace {
using namespace malus::tc;

constexpr int RB = 128;   // stationary rows per CTA: queries (dq) or keys (dk, dv)
constexpr int SB = 64;    // streamed rows per block: keys (dq) or queries (dk, dv)
constexpr int kBwdThreads = 352;   // producer, MMA, 8 row warps (two column groups), second producer
constexpr int kProd2 = 10;         // warp of the second producer

template <int HS>
struct BwdCfg {
  static constexpr int kRowBytes = RB * HS * 4;   // one plane of a stationary tile
  static constexpr int kBlkBytes = SB * HS * 4;   // one plane of a streamed block (either major)
  // dq: dO (hi, lo) | two stages of {K, V} (K-major) x (hi, lo) | K (MN-major) x (hi, lo)
  static constexpr int kDqKv = 4 * kBlkBytes;
  static constexpr int kOffDqKv = 2 * kRowBytes;
  static constexpr int kOffDqMn = kOffDqKv + 2 * kDqKv;
  static constexpr int kDqBar = kOffDqMn + 2 * kBlkBytes;
  static constexpr int kOffDpart = kDqBar + 256;   // [2 groups][128 rows] partial rowsum(dO * O)
  static constexpr int kSmemDq = kOffDpart + 2 * RB * 4 + 1024;
  // dk/dv: V (hi, lo) | {Q, dO} (K-major) x (hi, lo) | {Q, dO} (MN-major) x (hi, lo)
  static constexpr int kOffKvQk = 2 * kRowBytes;
  static constexpr int kOffKvMn = kOffKvQk + 4 * kBlkBytes;
  static constexpr int kKvBar = kOffKvMn + 4 * kBlkBytes;
  static constexpr int kSmemKv = kKvBar + 256 + 1024;
  static_assert(kSmemDq <= 232448 && kSmemKv <= 232448, "shared memory");
  // tensor memory (512 columns).  dq: S[b] at 64b, dP[b] at 128 + 64b (then the
  // dS planes: hi over S, lo over dP), dQ at 256, Q hi at 320, Q lo at 320 + HS.
  static constexpr uint32_t kQS = 0, kQDP = 128, kQG = 256, kQQ = 320;
  // dkdv: K hi at 0, K lo at HS; S^T at 128 and dP^T at 192 (then the P^T
  // planes: hi over S^T, lo over dP^T); dS^T hi at 256, lo at 320; dV at 384,
  // dK at 384 + HS.
  static constexpr uint32_t kKK = 0, kKS = 128, kKDP = 192, kKDS = 256, kKG = 384;
};

struct BwdArgs {
  int H, T;
  float scale;
  const float2* stats;   // [B*H*T] (row max of the scaled scores in base-2 units, 1 / row sum) from the forward
  float* D;              // [B*H*T] rowsum(dO * O): written by dq, read by dkdv
  const float* qkv_hi;   // q|k|v planes, head-folded [3][B*H][T][hs]
  const float* qkv_lo;
  const float* o_hi;     // O planes, head-unfolded [B*T][H*hs]
  const float* o_lo;
  float* g_hi;           // dq (dq kernel) / dk (dkdv kernel) planes, head-unfolded [B*T][H*hs]
  float* g_lo;
  float* g2_hi;          // dv planes (dkdv kernel)
  float* g2_lo;
  int32_t* err;
};

// 128 rows x hs of a K-major tile: hs/32 slabs of [128 rows][128 B], two 64-row boxes each
template <int HS>
__device__ __forceinline__ void load_rows(uint8_t* dst, const CUtensorMap* m, uint32_t bar, int row, int z) {
#pragma unroll
  for (int sl = 0; sl < HS / 32; ++sl)
#pragma unroll
    for (int r2 = 0; r2 < RB / SB; ++r2)
      tma_load_3d(smem_u32(dst + sl * (RB * 128) + r2 * (SB * 128)), m, bar, sl * 32, row + r2 * SB, z);
}
// 64 rows x hs, K-major: hs/32 slabs of [64 rows][128 B]
template <int HS>
__device__ __forceinline__ void load_blk_k(uint8_t* dst, const CUtensorMap* m, uint32_t bar, int row, int z) {
#pragma unroll
  for (int sl = 0; sl < HS / 32; ++sl) tma_load_3d(smem_u32(dst + sl * (SB * 128)), m, bar, sl * 32, row, z);
}
// 64 rows x hs, MN-major: hs/32 chunks of [64 rows][32 columns], one 4-D box
__device__ __forceinline__ void load_blk_mn(uint8_t* dst, const CUtensorMap* m, uint32_t bar, int row, int z) {
  tma_load_4d(smem_u32(dst), m, bar, 0, row, 0, z);
}
// MN-major descriptor of a 64-row block: 32-column chunks 8 KB apart
__device__ __forceinline__ uint64_t desc_mn64(uint32_t tile) { return umma_desc(tile, SB * 128, 512, 1); }

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
}
__device__ __forceinline__ void tmem_alloc512(uint32_t* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(512));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_free512(uint32_t tmem) {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void wait_bounded(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = gtimer();
  while (!mbar_try(bar, parity) && gtimer() - t0 < kWaitNs) {}
}

// this thread's row segment (HS/2 columns of the hi and lo planes) into TMEM
// columns at hi_addr / lo_addr of its lane
template <int HS>
__device__ __forceinline__ void row_to_tmem(const float* src_hi, const float* src_lo, uint32_t hi_addr,
                                            uint32_t lo_addr) {
  constexpr int HC = HS / 2;
  uint32_t h[HC], l[HC];
#pragma unroll
  for (int j = 0; j < HC; j += 4) {
    const float4 x = *reinterpret_cast<const float4*>(src_hi + j);
    const float4 y = *reinterpret_cast<const float4*>(src_lo + j);
    h[j] = __float_as_uint(x.x);
    h[j + 1] = __float_as_uint(x.y);
    h[j + 2] = __float_as_uint(x.z);
    h[j + 3] = __float_as_uint(x.w);
    l[j] = __float_as_uint(y.x);
    l[j + 1] = __float_as_uint(y.y);
    l[j + 2] = __float_as_uint(y.z);
    l[j + 3] = __float_as_uint(y.w);
  }
  if constexpr (HC == 32) {
    tmem_st32(hi_addr, h);
    tmem_st32(lo_addr, l);
  } else {
    tmem_st16(hi_addr, h);
    tmem_st16(lo_addr, l);
  }
}

// columns [g*HS/2, (g+1)*HS/2) of this thread's TMEM row (accumulator at
// taddr) as tf32 planes at hi / lo (the row's first column)
template <int HS>
__device__ __forceinline__ void store_half(uint32_t taddr, int g, float* hi, float* lo) {
  constexpr int HC = HS / 2;
  uint32_t r[HC];
  if constexpr (HC == 32) tmem_ld32(taddr + g * HC, r);
  else tmem_ld16(taddr + g * HC, r);
#pragma unroll
  for (int j = 0; j < HC; j += 4) {
    const float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                 __uint_as_float(r[j + 3]));
    const float4 h4 = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
    *reinterpret_cast<float4*>(hi + g * HC + j) = h4;
    *reinterpret_cast<float4*>(lo + g * HC + j) =
        make_float4(tf32_rn(v.x - h4.x), tf32_rn(v.y - h4.y), tf32_rn(v.z - h4.z), tf32_rn(v.w - h4.w));
  }
}

// 32 values -> tf32 hi and lo planes into TMEM columns of this thread's lane
__device__ __forceinline__ void store_planes32(const float* v, uint32_t hi_addr, uint32_t lo_addr) {
  uint32_t t[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) t[c] = __float_as_uint(tf32_rn(v[c]));
  tmem_st32(hi_addr, t);
#pragma unroll
  for (int c = 0; c < 32; ++c) t[c] = __float_as_uint(tf32_rn(v[c] - __uint_as_float(t[c])));
  tmem_st32(lo_addr, t);
}

// ============================ dQ (query-major) ============================
template <int HS>
__global__ void __launch_bounds__(kBwdThreads, 1)
k_attn_bwd_dq(const __grid_constant__ CUtensorMap mRh, const __grid_constant__ CUtensorMap mRl,
              const __grid_constant__ CUtensorMap mOh, const __grid_constant__ CUtensorMap mOl,
              const __grid_constant__ CUtensorMap mNh, const __grid_constant__ CUtensorMap mNl,
              const BwdArgs a) {
  using CF = BwdCfg<HS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = (uint64_t*)(smem + CF::kDqBar);
  uint64_t* o_full = bar;         // dO landed
  uint64_t* q_tm = bar + 1;       // Q written to TMEM by the eight row warps
  uint64_t* k_full = bar + 2;     // [2] K-major K, V block landed
  uint64_t* k_empty = bar + 4;    // [2] its S, dP MMAs done
  uint64_t* n_full = bar + 6;     // MN-major K block landed
  uint64_t* n_empty = bar + 7;    // its dQ MMAs done
  uint64_t* s_full = bar + 8;     // [2] S and dP in TMEM buffer b
  uint64_t* d_full = bar + 10;    // [2] dS planes written over buffer b by the eight row warps
  uint64_t* d_done = bar + 12;    // [2] dQ MMAs reading buffer b done
  uint64_t* g_full = bar + 14;    // dQ complete
  uint64_t* drain = bar + 15;
  uint64_t* done = bar + 16;      // the eight row warps finished reading TMEM
  uint32_t* tmem_slot = (uint32_t*)(bar + 17);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.T / RB;
  const int qb = nq - 1 - (int)(blockIdx.x % nq);   // heavy (late) query tiles first
  const int z = (int)(blockIdx.x / nq);
  const int q0 = qb * RB;
  const int nkb = (q0 + RB) / SB;                    // key blocks up to the diagonal
  const int row_base = z * a.T;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(q_tm), 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&d_full[i]), 8);
      mbar_init(smem_u32(&d_done[i]), 1);
    }
    mbar_init(smem_u32(n_full), 1);
    mbar_init(smem_u32(n_empty), 1);
    mbar_init(smem_u32(g_full), 1);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(done), 8);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc512(tmem_slot);
  fence_before();
  __syncwarp();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  uint8_t* o_h = smem;
  uint8_t* o_l = smem + CF::kRowBytes;
  auto kstage = [&](int s) { return smem + CF::kOffDqKv + s * CF::kDqKv; };   // Kh Kl Vh Vl
  uint8_t* nst = smem + CF::kOffDqMn;                                          // Kh Kl (MN-major)

  if (warp == 0) {
    // ---------------- TMA producer: dO, then the K-major K, V ring ----------------
    if (lane == 0) {
      const uint32_t of = smem_u32(o_full);
      mbar_expect_tx(of, 2 * CF::kRowBytes);
      load_rows<HS>(o_h, &mOh, of, row_base + q0, 0);
      load_rows<HS>(o_l, &mOl, of, row_base + q0, 0);
      int it = 0;
      for (; it < nkb; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (it >= 2 && !mbar_wait(smem_u32(&k_empty[s]), ph ^ 1, abort_flag, a.err, 51)) break;
        uint8_t* st = kstage(s);
        const uint32_t fb = smem_u32(&k_full[s]);
        const int r = row_base + it * SB;
        mbar_expect_tx(fb, 4 * CF::kBlkBytes);
        load_blk_k<HS>(st, &mRh, fb, r, 1);
        load_blk_k<HS>(st + CF::kBlkBytes, &mRl, fb, r, 1);
        load_blk_k<HS>(st + 2 * CF::kBlkBytes, &mRh, fb, r, 2);
        load_blk_k<HS>(st + 3 * CF::kBlkBytes, &mRl, fb, r, 2);
      }
      if (*abort_flag) {
        // every issued load must land before the CTA exits
        wait_bounded(of, 0);
        for (int qi = it > 2 ? it - 2 : 0; qi < it; ++qi) wait_bounded(smem_u32(&k_full[qi & 1]), (qi >> 1) & 1);
      }
    }
  } else if (warp == kProd2) {
    // ---------------- TMA producer: the MN-major K buffer ----------------
    if (lane == 0) {
      int it = 0;
      for (; it < nkb; ++it) {
        if (it >= 1 && !mbar_wait(smem_u32(n_empty), (it - 1) & 1, abort_flag, a.err, 59)) break;
        const uint32_t fb = smem_u32(n_full);
        mbar_expect_tx(fb, 2 * CF::kBlkBytes);
        load_blk_mn(nst, &mNh, fb, row_base + it * SB, 1);
        load_blk_mn(nst + CF::kBlkBytes, &mNl, fb, row_base + it * SB, 1);
      }
      if (*abort_flag && it > 0) wait_bounded(smem_u32(n_full), (it - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc_tf32(false, false, SB);
      const uint32_t id_g = idesc_tf32(false, true, HS);
      bool ok = mbar_wait(smem_u32(o_full), 0, abort_flag, a.err, 52) &&
                mbar_wait(smem_u32(q_tm), 0, abort_flag, a.err, 48);
      bool issued = false;
      // descriptors built once; a stage or k-step adds (byte offset / 16) (the
      // address field is the low 14 bits, every address is below 256 KB)
      const uint64_t doh = desc_kmajor(smem_u32(o_h), 0), dol = doh + CF::kRowBytes / 16;
      const uint64_t dk0 = desc_kmajor(smem_u32(kstage(0)), 0);
      const uint64_t dnh = desc_mn64(smem_u32(nst)), dnl = dnh + CF::kBlkBytes / 16;
      const uint32_t qh = tmem + CF::kQQ, ql = tmem + CF::kQQ + HS;
      // S = Q K^T and dP = dO V^T of key block `it` into TMEM buffer it & 1
      auto issue_sd = [&](int it) -> bool {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&k_full[s]), ph, abort_flag, a.err, 53)) return false;
        // the buffer's previous block (it - 2) has been read by its dQ MMAs
        if (it >= 2 && !mbar_wait(smem_u32(&d_done[s]), ph ^ 1, abort_flag, a.err, 54)) return false;
        fence_after();
        const uint64_t kh = dk0 + (uint64_t)(s * (CF::kDqKv / 16)), kl = kh + CF::kBlkBytes / 16;
        const uint64_t vh = kh + 2 * (CF::kBlkBytes / 16), vl = kh + 3 * (CF::kBlkBytes / 16);
        const uint32_t dS = tmem + CF::kQS + s * SB, dP = tmem + CF::kQDP + s * SB;
#pragma unroll
        for (int kk = 0; kk < HS / 8; ++kk) {
          const uint32_t acc = kk > 0 ? 1u : 0u;
          const uint64_t oa = (uint64_t)((kk >> 2) * (RB * 128 / 16) + (kk & 3) * 2);   // 128-row tile
          const uint64_t ob = (uint64_t)((kk >> 2) * (SB * 128 / 16) + (kk & 3) * 2);   // 64-row block
          mma_tf32_ta(dS, ql + kk * 8, kh + ob, id_s, acc);
          mma_tf32_ta(dS, qh + kk * 8, kl + ob, id_s, 1u);
          mma_tf32_ta(dS, qh + kk * 8, kh + ob, id_s, 1u);
          mma_tf32(dP, dol + oa, vh + ob, id_s, acc);
          mma_tf32(dP, doh + oa, vl + ob, id_s, 1u);
          mma_tf32(dP, doh + oa, vh + ob, id_s, 1u);
        }
        issued = true;
        mma_commit(smem_u32(&s_full[s]));
        mma_commit(smem_u32(&k_empty[s]));   // K, V of this stage are consumed once these finish
        return true;
      };
      ok = ok && issue_sd(0);
      if (nkb > 1) ok = ok && issue_sd(1);
      for (int it = 0; it < nkb && ok; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&d_full[s]), ph, abort_flag, a.err, 55)) { ok = false; break; }
        if (!mbar_wait(smem_u32(n_full), it & 1, abort_flag, a.err, 50)) { ok = false; break; }
        fence_after();
        // dQ += dS K: A = the dS planes over buffer s (hi over S, lo over dP)
        const uint32_t ah = tmem + CF::kQS + s * SB, al = tmem + CF::kQDP + s * SB;
#pragma unroll
        for (int kk = 0; kk < SB / 8; ++kk) {
          const uint64_t bh = dnh + (uint64_t)(kk * 64), bl = dnl + (uint64_t)(kk * 64);   // 8 K rows = 1 KB
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          mma_tf32_ta(tmem + CF::kQG, al + kk * 8, bh, id_g, acc);
          mma_tf32_ta(tmem + CF::kQG, ah + kk * 8, bl, id_g, 1u);
          mma_tf32_ta(tmem + CF::kQG, ah + kk * 8, bh, id_g, 1u);
        }
        mma_commit(smem_u32(&d_done[s]));
        mma_commit(smem_u32(n_empty));
        if (it + 2 < nkb && !issue_sd(it + 2)) { ok = false; break; }
      }
      if (ok) mma_commit(smem_u32(g_full));
      if (!ok && issued) {
        mma_commit(smem_u32(drain));
        wait_bounded(smem_u32(drain), 0);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- row warps: one query row per thread, group g owns keys 32g..32g+31 of each block
    const int quarter = warp & 3;
    const int g = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int b = z / a.H, h = z % a.H;
    const size_t C = (size_t)a.H * HS;
    constexpr int HC = HS / 2;   // columns per group
    // Q (this group's half of the row) into TMEM: the A operand of S = Q K^T
    {
      const size_t qo = (size_t)(row_base + q) * HS + g * HC;
      row_to_tmem<HS>(a.qkv_hi + qo, a.qkv_lo + qo, tmem + CF::kQQ + g * HC + lane_off,
                      tmem + CF::kQQ + HS + g * HC + lane_off);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(q_tm));
    }
    const float2 st2 = a.stats[row_base + q];
    const float m2 = st2.x, inv_l = st2.y;   // row max in base-2 units, 1 / row sum
    const float sl2e = a.scale * kLog2e;
    // D = rowsum(dO * O), each group over half of the head's columns: O from its
    // planes in global memory, dO from the stationary tile once it has landed
    float* dpart = reinterpret_cast<float*>(smem + CF::kOffDpart);
    {
      const size_t oo = ((size_t)b * a.T + q) * C + (size_t)h * HS + g * HC;
      const float4* oh = reinterpret_cast<const float4*>(a.o_hi + oo);
      const float4* ol = reinterpret_cast<const float4*>(a.o_lo + oo);
      float4 ov[HC / 4];
#pragma unroll
      for (int j = 0; j < HC / 4; ++j) {
        const float4 x = oh[j], y = ol[j];
        ov[j] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
      }
      float part = 0.0f;
      if (mbar_wait(smem_u32(o_full), 0, abort_flag, a.err, 49)) {
        // row `row` of the 128-byte-swizzled K-major tile: slab j/8, granule (j%8) ^ (row%8)
#pragma unroll
        for (int jj = 0; jj < HC / 4; ++jj) {
          const int j = g * (HC / 4) + jj;
          const int off = (j >> 3) * (RB * 128) + row * 128 + (((j & 7) ^ (row & 7)) << 4);
          const float4 x = *reinterpret_cast<const float4*>(o_h + off);
          const float4 y = *reinterpret_cast<const float4*>(o_l + off);
          part += (x.x + y.x) * ov[jj].x;
          part += (x.y + y.y) * ov[jj].y;
          part += (x.z + y.z) * ov[jj].z;
          part += (x.w + y.w) * ov[jj].w;
        }
      }
      dpart[g * RB + row] = part;
    }
    __syncwarp();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float D = dpart[row] + dpart[RB + row];
    if (g == 0) a.D[row_base + q] = D;
    bool ok = true;
    for (int it = 0; it < nkb && ok; ++it) {
      const int s = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const bool failed = !mbar_wait(smem_u32(&s_full[s]), ph, abort_flag, a.err, 56);
      if (bar_any(1, 256, failed)) { ok = false; break; }
      fence_after();
      const uint32_t cs = tmem + CF::kQS + s * SB + 32 * g + lane_off;
      const uint32_t cp = tmem + CF::kQDP + s * SB + 32 * g + lane_off;
      uint32_t rs[32], rp[32];
      tmem_ld32(cs, rs);
      tmem_ld32(cp, rp);
      float ds[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int key = it * SB + 32 * g + c;   // keys past the query are masked (P = 0)
        ds[c] = 0.0f;
        if (key <= q) {
          const float p = exp2_hw(fmaf(__uint_as_float(rs[c]), sl2e, -m2)) * inv_l;
          ds[c] = p * (__uint_as_float(rp[c]) - D) * a.scale;
        }
      }
      // dS planes over the scores just read: hi over S, lo over dP
      store_planes32(ds, cs, cp);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&d_full[s]));
    }
    if (ok && mbar_wait(smem_u32(g_full), 0, abort_flag, a.err, 58)) {
      fence_after();
      const size_t go = ((size_t)b * a.T + q) * C + (size_t)h * HS;
      store_half<HS>(tmem + CF::kQG + lane_off, g, a.g_hi + go, a.g_lo + go);
    }
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(done));
  }
  fence_before();
  __syncwarp();   // lane 0 of the producer / MMA warps may arrive alone: reconverge first
  __syncthreads();
  if (warp == 1) {
    mbar_wait_bounded(smem_u32(done), 0);   // every TMEM reader finished: explicit, not the CTA barrier alone
    tmem_free512(tmem);
  }
}

// ============================ dK, dV (key-major) ============================
template <int HS>
__global__ void __launch_bounds__(kBwdThreads, 1)
k_attn_bwd_dkdv(const __grid_constant__ CUtensorMap mRh, const __grid_constant__ CUtensorMap mRl,
                const __grid_constant__ CUtensorMap mOh, const __grid_constant__ CUtensorMap mOl,
                const __grid_constant__ CUtensorMap mNh, const __grid_constant__ CUtensorMap mNl,
                const __grid_constant__ CUtensorMap mONh, const __grid_constant__ CUtensorMap mONl,
                const BwdArgs a) {
  using CF = BwdCfg<HS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = (uint64_t*)(smem + CF::kKvBar);
  uint64_t* v_full = bar;         // V landed
  uint64_t* k_tm = bar + 1;       // K written to TMEM by the eight row warps
  uint64_t* qk_full = bar + 2;    // K-major Q, dO block landed
  uint64_t* qk_empty = bar + 3;   // its S^T, dP^T MMAs done
  uint64_t* mn_full = bar + 4;    // MN-major Q, dO block landed
  uint64_t* mn_empty = bar + 5;   // its dV, dK MMAs done
  uint64_t* s_full = bar + 6;     // S^T and dP^T in TMEM
  uint64_t* pd_full = bar + 7;    // P^T and dS^T planes written by the eight row warps
  uint64_t* pd_done = bar + 8;    // dV, dK MMAs reading them done
  uint64_t* g_full = bar + 9;     // dV, dK complete
  uint64_t* drain = bar + 10;
  uint64_t* done = bar + 11;      // the eight row warps finished reading TMEM
  uint32_t* tmem_slot = (uint32_t*)(bar + 12);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = a.T / RB;
  const int kb = (int)(blockIdx.x % nk);            // heavy (early) key tiles first
  const int z = (int)(blockIdx.x / nk);
  const int k0 = kb * RB;
  const int nqb = (a.T - k0) / SB;                  // query blocks from the diagonal on
  const int row_base = z * a.T;
  const size_t BHT = (size_t)(gridDim.x / nk) * a.T;   // rows of one q / k / v plane

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(v_full), 1);
    mbar_init(smem_u32(k_tm), 8);
    mbar_init(smem_u32(qk_full), 1);
    mbar_init(smem_u32(qk_empty), 1);
    mbar_init(smem_u32(mn_full), 1);
    mbar_init(smem_u32(mn_empty), 1);
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(pd_full), 8);
    mbar_init(smem_u32(pd_done), 1);
    mbar_init(smem_u32(g_full), 1);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(done), 8);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc512(tmem_slot);
  fence_before();
  __syncwarp();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  uint8_t* v_h = smem;
  uint8_t* v_l = smem + CF::kRowBytes;
  uint8_t* qk = smem + CF::kOffKvQk;   // Qh Ql dOh dOl (K-major)
  uint8_t* mn = smem + CF::kOffKvMn;   // Qh Ql dOh dOl (MN-major)

  if (warp == 0) {
    // ---------------- TMA producer: V, then the K-major Q, dO buffer ----------------
    if (lane == 0) {
      const uint32_t vf = smem_u32(v_full);
      mbar_expect_tx(vf, 2 * CF::kRowBytes);
      load_rows<HS>(v_h, &mRh, vf, row_base + k0, 2);
      load_rows<HS>(v_l, &mRl, vf, row_base + k0, 2);
      int it = 0;
      for (; it < nqb; ++it) {
        if (it >= 1 && !mbar_wait(smem_u32(qk_empty), (it - 1) & 1, abort_flag, a.err, 61)) break;
        const uint32_t fb = smem_u32(qk_full);
        const int r = row_base + k0 + it * SB;
        mbar_expect_tx(fb, 4 * CF::kBlkBytes);
        load_blk_k<HS>(qk, &mRh, fb, r, 0);
        load_blk_k<HS>(qk + CF::kBlkBytes, &mRl, fb, r, 0);
        load_blk_k<HS>(qk + 2 * CF::kBlkBytes, &mOh, fb, r, 0);
        load_blk_k<HS>(qk + 3 * CF::kBlkBytes, &mOl, fb, r, 0);
      }
      if (*abort_flag) {
        wait_bounded(vf, 0);
        if (it > 0) wait_bounded(smem_u32(qk_full), (it - 1) & 1);
      }
    }
  } else if (warp == kProd2) {
    // ---------------- TMA producer: the MN-major Q, dO buffer ----------------
    if (lane == 0) {
      int it = 0;
      for (; it < nqb; ++it) {
        if (it >= 1 && !mbar_wait(smem_u32(mn_empty), (it - 1) & 1, abort_flag, a.err, 62)) break;
        const uint32_t mb = smem_u32(mn_full);
        const int r = row_base + k0 + it * SB;
        mbar_expect_tx(mb, 4 * CF::kBlkBytes);
        load_blk_mn(mn, &mNh, mb, r, 0);
        load_blk_mn(mn + CF::kBlkBytes, &mNl, mb, r, 0);
        load_blk_mn(mn + 2 * CF::kBlkBytes, &mONh, mb, r, 0);
        load_blk_mn(mn + 3 * CF::kBlkBytes, &mONl, mb, r, 0);
      }
      if (*abort_flag && it > 0) wait_bounded(smem_u32(mn_full), (it - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc_tf32(false, false, SB);
      const uint32_t id_g = idesc_tf32(false, true, HS);
      bool ok = mbar_wait(smem_u32(v_full), 0, abort_flag, a.err, 63) &&
                mbar_wait(smem_u32(k_tm), 0, abort_flag, a.err, 60);
      bool issued = false;
      // descriptors built once; a k-step adds (byte offset / 16)
      const uint64_t dvh = desc_kmajor(smem_u32(v_h), 0), dvl = dvh + CF::kRowBytes / 16;
      const uint64_t dqh = desc_kmajor(smem_u32(qk), 0), dql = dqh + CF::kBlkBytes / 16;
      const uint64_t doh = dqh + 2 * (CF::kBlkBytes / 16), dol = dqh + 3 * (CF::kBlkBytes / 16);
      const uint64_t nqh = desc_mn64(smem_u32(mn)), nql = nqh + CF::kBlkBytes / 16;
      const uint64_t noh = nqh + 2 * (CF::kBlkBytes / 16), nol = nqh + 3 * (CF::kBlkBytes / 16);
      const uint32_t kh = tmem + CF::kKK, kl = tmem + CF::kKK + HS;
      const uint32_t dS = tmem + CF::kKS, dP = tmem + CF::kKDP;
      const uint32_t dV = tmem + CF::kKG, dK = tmem + CF::kKG + HS;
      for (int it = 0; it < nqb && ok; ++it) {
        // S^T = K Q^T and dP^T = V dO^T of query block `it`
        if (!mbar_wait(smem_u32(qk_full), it & 1, abort_flag, a.err, 64)) { ok = false; break; }
        // the previous block's P^T (over these columns) and dS^T have been read
        if (it >= 1 && !mbar_wait(smem_u32(pd_done), (it - 1) & 1, abort_flag, a.err, 65)) { ok = false; break; }
        fence_after();
#pragma unroll
        for (int kk = 0; kk < HS / 8; ++kk) {
          const uint32_t acc = kk > 0 ? 1u : 0u;
          const uint64_t oa = (uint64_t)((kk >> 2) * (RB * 128 / 16) + (kk & 3) * 2);
          const uint64_t ob = (uint64_t)((kk >> 2) * (SB * 128 / 16) + (kk & 3) * 2);
          mma_tf32_ta(dS, kl + kk * 8, dqh + ob, id_s, acc);
          mma_tf32_ta(dS, kh + kk * 8, dql + ob, id_s, 1u);
          mma_tf32_ta(dS, kh + kk * 8, dqh + ob, id_s, 1u);
          mma_tf32(dP, dvl + oa, doh + ob, id_s, acc);
          mma_tf32(dP, dvh + oa, dol + ob, id_s, 1u);
          mma_tf32(dP, dvh + oa, doh + ob, id_s, 1u);
        }
        issued = true;
        mma_commit(smem_u32(s_full));
        mma_commit(smem_u32(qk_empty));
        // dV += P^T dO, dK += dS^T Q once the row warps wrote P^T and dS^T
        if (!mbar_wait(smem_u32(pd_full), it & 1, abort_flag, a.err, 66)) { ok = false; break; }
        if (!mbar_wait(smem_u32(mn_full), it & 1, abort_flag, a.err, 67)) { ok = false; break; }
        fence_after();
        const uint32_t ph_ = tmem + CF::kKS, pl_ = tmem + CF::kKDP;            // P^T planes
        const uint32_t sh_ = tmem + CF::kKDS, sl_ = tmem + CF::kKDS + SB;      // dS^T planes
#pragma unroll
        for (int kk = 0; kk < SB / 8; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          const uint64_t boh = noh + (uint64_t)(kk * 64), bol = nol + (uint64_t)(kk * 64);
          mma_tf32_ta(dV, pl_ + kk * 8, boh, id_g, acc);
          mma_tf32_ta(dV, ph_ + kk * 8, bol, id_g, 1u);
          mma_tf32_ta(dV, ph_ + kk * 8, boh, id_g, 1u);
          const uint64_t bqh = nqh + (uint64_t)(kk * 64), bql = nql + (uint64_t)(kk * 64);
          mma_tf32_ta(dK, sl_ + kk * 8, bqh, id_g, acc);
          mma_tf32_ta(dK, sh_ + kk * 8, bql, id_g, 1u);
          mma_tf32_ta(dK, sh_ + kk * 8, bqh, id_g, 1u);
        }
        mma_commit(smem_u32(pd_done));
        mma_commit(smem_u32(mn_empty));
      }
      if (ok) mma_commit(smem_u32(g_full));
      if (!ok && issued) {
        mma_commit(smem_u32(drain));
        wait_bounded(smem_u32(drain), 0);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- row warps: one key row per thread, group g owns queries 32g..32g+31 of each block
    const int quarter = warp & 3;
    const int g = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    constexpr int HC = HS / 2;
    // K (this group's half of the row) into TMEM: the A operand of S^T = K Q^T
    {
      const size_t ko = (BHT + (size_t)(row_base + key)) * HS + g * HC;
      row_to_tmem<HS>(a.qkv_hi + ko, a.qkv_lo + ko, tmem + CF::kKK + g * HC + lane_off,
                      tmem + CF::kKK + HS + g * HC + lane_off);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(k_tm));
    }
    const float sl2e = a.scale * kLog2e;
    // per-query statistics of the next block: lane c loads query c's of this
    // group's 32 (coalesced) and the values reach every lane by shuffles
    float2 nst = a.stats[row_base + k0 + 32 * g + lane];
    float nD = a.D[row_base + k0 + 32 * g + lane];
    bool ok = true;
    for (int it = 0; it < nqb && ok; ++it) {
      const int qbase = k0 + it * SB + 32 * g;   // first query of this group's columns
      const float qm = nst.x, qi = nst.y, qD = nD;
      if (it + 1 < nqb) {
        nst = a.stats[row_base + qbase + SB + lane];
        nD = a.D[row_base + qbase + SB + lane];
      }
      const bool failed = !mbar_wait(smem_u32(s_full), it & 1, abort_flag, a.err, 68);
      if (bar_any(1, 256, failed)) { ok = false; break; }
      fence_after();
      const uint32_t cs = tmem + CF::kKS + 32 * g + lane_off;
      const uint32_t cp = tmem + CF::kKDP + 32 * g + lane_off;
      uint32_t rs[32], rp[32];
      tmem_ld32(cs, rs);
      tmem_ld32(cp, rp);
      float p[32], ds[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float cm = __shfl_sync(0xffffffffu, qm, c);
        const float ci = __shfl_sync(0xffffffffu, qi, c);
        const float cD = __shfl_sync(0xffffffffu, qD, c);
        p[c] = 0.0f;
        ds[c] = 0.0f;
        if (key <= qbase + c) {   // the query sees this key
          p[c] = exp2_hw(fmaf(__uint_as_float(rs[c]), sl2e, -cm)) * ci;
          ds[c] = p[c] * (__uint_as_float(rp[c]) - cD) * a.scale;
        }
      }
      // P^T planes over the scores just read (hi over S^T, lo over dP^T); dS^T
      // planes into their region (free: the previous block's dK MMAs finished
      // before these scores were computed)
      store_planes32(p, cs, cp);
      store_planes32(ds, tmem + CF::kKDS + 32 * g + lane_off, tmem + CF::kKDS + SB + 32 * g + lane_off);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(pd_full));
    }
    if (ok && mbar_wait(smem_u32(g_full), 0, abort_flag, a.err, 70)) {
      fence_after();
      const int b = z / a.H, h = z % a.H;
      const size_t C = (size_t)a.H * HS;
      const size_t go = ((size_t)b * a.T + key) * C + (size_t)h * HS;
      store_half<HS>(tmem + CF::kKG + lane_off, g, a.g2_hi + go, a.g2_lo + go);
      store_half<HS>(tmem + CF::kKG + HS + lane_off, g, a.g_hi + go, a.g_lo + go);
    }
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(done));
  }
  fence_before();
  __syncwarp();   // lane 0 of the producer / MMA warps may arrive alone: reconverge first
  __syncthreads();
  if (warp == 1) {
    mbar_wait_bounded(smem_u32(done), 0);   // every TMEM reader finished: explicit, not the CTA barrier alone
    tmem_free512(tmem);
  }
}

template <int HS>
void launch_attn_bwd(const float* qkv_hi, const float* qkv_lo, const float* do_hi, const float* do_lo,
                     const float* o_hi, const float* o_lo, const float* stats, float* D, int B, int H, int T,
                     float scale, float* dqkv_hi, float* dqkv_lo) {
  using CF = BwdCfg<HS>;
  const uint64_t BHT = (uint64_t)B * H * T;
  const uint64_t plane = BHT * HS * 4;   // bytes of one of q, k, v (and of dO)
  // K-major rows: {hs, B*H*T, z}, box {32, 64 rows, 1}, 128-B swizzle
  const uint64_t dr[3] = {(uint64_t)HS, BHT, 3}, dro[3] = {(uint64_t)HS, BHT, 1};
  const uint64_t sr[2] = {(uint64_t)HS * 4, plane};
  const uint32_t br[3] = {32, (uint32_t)SB, 1};
  // MN-major blocks: {32, rows, hs/32 chunks, z}, box {32, 64 rows, hs/32, 1}, 32-B-granule swizzle
  const uint64_t dn[4] = {32, BHT, (uint64_t)HS / 32, 3}, dno[4] = {32, BHT, (uint64_t)HS / 32, 1};
  const uint64_t sn[3] = {(uint64_t)HS * 4, 128, plane};
  const uint32_t bn[4] = {32, (uint32_t)SB, (uint32_t)HS / 32, 1};
  const CUtensorMap rh = encode_f32_map(3, qkv_hi, dr, sr, br, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap rl = encode_f32_map(3, qkv_lo, dr, sr, br, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap oh = encode_f32_map(3, do_hi, dro, sr, br, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap ol = encode_f32_map(3, do_lo, dro, sr, br, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap nh = encode_f32_map(4, qkv_hi, dn, sn, bn, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const CUtensorMap nl = encode_f32_map(4, qkv_lo, dn, sn, bn, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const CUtensorMap onh = encode_f32_map(4, do_hi, dno, sn, bn, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const CUtensorMap onl = encode_f32_map(4, do_lo, dno, sn, bn, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const size_t MC = (size_t)BHT * HS;
  static bool attr = false;
  if (!attr) {
    MALUS_CUDA(cudaFuncSetAttribute(k_attn_bwd_dq<HS>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmemDq));
    MALUS_CUDA(cudaFuncSetAttribute(k_attn_bwd_dkdv<HS>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmemKv));
    attr = true;
  }
  const unsigned grid = (unsigned)(B * H * (T / RB));
  BwdArgs aq{H, T, scale, reinterpret_cast<const float2*>(stats), D, qkv_hi, qkv_lo, o_hi, o_lo,
             dqkv_hi, dqkv_lo, nullptr, nullptr, device_error_word()};
  k_attn_bwd_dq<HS><<<grid, kBwdThreads, CF::kSmemDq, stream()>>>(rh, rl, oh, ol, nh, nl, aq);
  count_launch();
  after_launch("k_attn_bwd_dq");
  BwdArgs ak{H, T, scale, reinterpret_cast<const float2*>(stats), D, qkv_hi, qkv_lo, o_hi, o_lo,
             dqkv_hi + MC, dqkv_lo + MC, dqkv_hi + 2 * MC, dqkv_lo + 2 * MC, device_error_word()};
  k_attn_bwd_dkdv<HS><<<grid, kBwdThreads, CF::kSmemKv, stream()>>>(rh, rl, oh, ol, nh, nl, onh, onl, ak);
  count_launch();
  after_launch("k_attn_bwd_dkdv");
}

}  // namespace

// qkv planes [3][B][H][T][hs]; dO planes [B][H][T][hs]; O planes [B*T][H*hs];
// stats [B*H*T] pairs from attn_fwd; D workspace [B*H*T] floats; outputs the
// planes of dq | dk | dv head-unfolded into dqkv [3][B*T][H*hs].
void attn_bwd(const float* qkv_hi, const float* qkv_lo, const float* do_hi, const float* do_lo,
              const float* o_hi, const float* o_lo, const float* stats, float* D, int B, int H, int T, int hs,
              float scale, float* dqkv_hi, float* dqkv_lo) {
  if (T % RB != 0 || (hs != 32 && hs != 64))
    panic("attn_bwd: needs T %% 128 == 0 and hs in {32, 64} (T=%d hs=%d)", T, hs);
  for (const void* p : {(const void*)qkv_hi, (const void*)qkv_lo, (const void*)do_hi, (const void*)do_lo,
                        (const void*)o_hi, (const void*)o_lo, (const void*)stats, (const void*)D,
                        (const void*)dqkv_hi, (const void*)dqkv_lo})
    if (p == nullptr || ((uintptr_t)p & 15)) panic("attn_bwd: buffers must be non-null and 16-byte aligned");
  if (hs == 64) launch_attn_bwd<64>(qkv_hi, qkv_lo, do_hi, do_lo, o_hi, o_lo, stats, D, B, H, T, scale, dqkv_hi, dqkv_lo);
  else launch_attn_bwd<32>(qkv_hi, qkv_lo, do_hi, do_lo, o_hi, o_lo, stats, D, B, H, T, scale, dqkv_hi, dqkv_lo);
}

}  // namespace malus

extern "C" int32_t malus_attn_bwd(const float* qkv_hi, const float* qkv_lo, const float* do_hi,
                                  const float* do_lo, const float* o_hi, const float* o_lo,
                                  const float* stats, float* D, int32_t B, int32_t H, int32_t T,
                                  int32_t hs, float scale, float* dqkv_hi, float* dqkv_lo) {
  if (T % 128 != 0 || (hs != 32 && hs != 64)) return -1;
  malus::attn_bwd(qkv_hi, qkv_lo, do_hi, do_lo, o_hi, o_lo, stats, D, B, H, T, hs, scale, dqkv_hi, dqkv_lo);
  return 0;
}
