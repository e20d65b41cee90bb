// Fused causal attention forward on tcgen05 (3xTF32): S = Q K^T * scale,
// causal softmax, O = P V in one kernel, without an f32 score tensor.
//
// Reference semantics (examples/nanogpt_modular.ml attention block; the mask of
// metal.rs:1601-1612): scores = (Q K^T) * 1/sqrt(hs) + mask(-1e9 above the
// diagonal), P = softmax(scores, axis -1), O = P V.  Masked scores underflow to
// exactly 0 after the exponential, so keys past the diagonal are skipped.
//
// One CTA = one head (z = b*H + h) x 128 query rows; 192 threads:
//   warp 0     TMA producer: Q once (tf32 hi/lo planes), then key blocks of 64
//              keys through two K/V stages (K only in pass 1, K and V in pass 2);
//   warp 1     TMEM owner and MMA issuer: S_b = Q K^T into two 64-column TMEM
//              buffers, O += P V into a third region;
//   warps 2-5  softmax: one thread per query row (its TMEM lane).
//              Pass 1: row max m and sum l over the key blocks (online).
//              Pass 2: S recomputed, p = exp(s*scale - m) * (1/l) written in 32-key
//              halves into a swizzled shared stage that is both the A operand of
//              the P V MMA and the source of a TMA store of the P planes (the
//              backward reads them); finally O is read from TMEM and written as
//              head-unfolded tf32 planes [B*T][H*hs].
// Every mbarrier wait is bounded; on timeout the CTA records an error, drains
// its MMAs and returns.
#include "common.cuh"
#include "tc_common.cuh"

namespace malus {
namespace {
using namespace malus::tc;

// OR of `v` over the 128 softmax threads (named barrier 1): every exit
// decision in those warps is collective, so no thread is left at a barrier.
__device__ __forceinline__ bool any128(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

constexpr int AQ = 128;  // query rows per CTA
constexpr int AK = 64;   // keys per block

template <int HS>
struct AttnCfg {
  static constexpr int kQBytes = AQ * HS * 4;              // one plane of the Q tile
  static constexpr int kKBytes = AK * HS * 4;              // one plane of a K (or V) block
  static constexpr int kStageBytes = 4 * kKBytes;          // K hi, K lo, V hi, V lo
  static constexpr int kPBytes = AQ * 32 * 4;              // one plane of a 32-key P half
  static constexpr int kOffStage = 2 * kQBytes;
  static constexpr int kOffP = kOffStage + 2 * kStageBytes;
  static constexpr int kOffBar = kOffP + 2 * kPBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;
  static_assert(kSmem <= 232448, "shared memory");
};

struct AttnArgs {
  int H, T, hs;
  float scale;
  float* o_hi;
  float* o_lo;
  int32_t* err;
};

template <int HS>
__global__ void __launch_bounds__(192, 1)
k_attn_fwd(const __grid_constant__ CUtensorMap mQKh, const __grid_constant__ CUtensorMap mQKl,
           const __grid_constant__ CUtensorMap mVh, const __grid_constant__ CUtensorMap mVl,
           const __grid_constant__ CUtensorMap mPh, const __grid_constant__ CUtensorMap mPl,
           const AttnArgs a) {
  using CF = AttnCfg<HS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(smem + CF::kOffBar);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;    // [2]
  uint64_t* s_empty = bar + 7;   // [2]
  uint64_t* p_full = bar + 9;
  uint64_t* p_empty = bar + 10;
  uint64_t* o_full = bar + 11;
  uint64_t* drain = bar + 12;
  uint32_t* tmem_slot = (uint32_t*)(bar + 13);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.T / AQ;
  const int qb = nq - 1 - (int)(blockIdx.x % nq);   // heavy (late) query blocks first
  const int z = (int)(blockIdx.x / nq);
  const int q0 = qb * AQ;
  const int nkb = (q0 + AQ) / AK;                     // key blocks up to the diagonal
  const int iters = 2 * nkb;                          // pass 1 + pass 2
  const int row_base = z * a.T;                       // first row of this head in the [BH*T] views

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&kv_full[i]), 1);
      mbar_init(smem_u32(&kv_empty[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_empty[i]), 4);
    }
    mbar_init(smem_u32(p_full), 1);
    mbar_init(smem_u32(p_empty), 1);
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)), "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;   // S buffers at columns 0 and 64, O at 128

  uint8_t* q_h = smem;
  uint8_t* q_l = smem + CF::kQBytes;
  uint8_t* p_h = smem + CF::kOffP;
  uint8_t* p_l = p_h + CF::kPBytes;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(smem_u32(q_full), 2 * CF::kQBytes);
      for (int sl = 0; sl < HS / 32; ++sl)
        for (int rh = 0; rh < 2; ++rh) {
          const uint32_t off = sl * (AQ * 128) + rh * (64 * 128);
          tma_load_3d(smem_u32(q_h + off), &mQKh, smem_u32(q_full), sl * 32, row_base + q0 + rh * 64, 0);
          tma_load_3d(smem_u32(q_l + off), &mQKl, smem_u32(q_full), sl * 32, row_base + q0 + rh * 64, 0);
        }
      int it = 0;
      for (; it < iters; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (it >= 2 && !mbar_wait(smem_u32(&kv_empty[s]), ph ^ 1, abort_flag, a.err, 31)) break;
        const bool pass2 = it >= nkb;
        const int kb = pass2 ? it - nkb : it;
        uint8_t* st = smem + CF::kOffStage + s * CF::kStageBytes;
        const uint32_t fb = smem_u32(&kv_full[s]);
        mbar_expect_tx(fb, pass2 ? CF::kStageBytes : 2 * CF::kKBytes);
        for (int sl = 0; sl < HS / 32; ++sl) {
          tma_load_3d(smem_u32(st + sl * (AK * 128)), &mQKh, fb, sl * 32, row_base + kb * AK, 1);
          tma_load_3d(smem_u32(st + CF::kKBytes + sl * (AK * 128)), &mQKl, fb, sl * 32, row_base + kb * AK, 1);
        }
        if (pass2) {
          for (int half = 0; half < 2; ++half) {
            const uint32_t voff = 2 * CF::kKBytes + half * (HS / 32) * 4096;
            tma_load_4d(smem_u32(st + voff), &mVh, fb, 0, row_base + kb * AK + 32 * half, 0, 2);
            tma_load_4d(smem_u32(st + CF::kKBytes + voff), &mVl, fb, 0, row_base + kb * AK + 32 * half, 0, 2);
          }
        }
      }
      if (*abort_flag) {
        // every issued load must land before the CTA exits
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(q_full), 0) && gtimer() - t0 < kWaitNs) {}
        for (int qi = it > 2 ? it - 2 : 0; qi < it; ++qi) {
          t0 = gtimer();
          while (!mbar_try(smem_u32(&kv_full[qi & 1]), (qi >> 1) & 1) && gtimer() - t0 < kWaitNs) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc_tf32(false, false, AK);
      const uint32_t id_o = idesc_tf32(false, true, HS);
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, a.err, 32);
      bool issued = false;
      int pcount = 0;
      const uint32_t qh = smem_u32(q_h), ql = smem_u32(q_l);
      // S_it = Q K_it^T into TMEM buffer it & 1
      auto issue_s = [&](int it) -> bool {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&kv_full[s]), ph, abort_flag, a.err, 33)) return false;
        if (it >= 2 && !mbar_wait(smem_u32(&s_empty[s]), ph ^ 1, abort_flag, a.err, 34)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t kh = smem_u32(smem + CF::kOffStage + s * CF::kStageBytes), kl = kh + CF::kKBytes;
        const uint32_t dS = tmem + s * AK;
#pragma unroll
        for (int kk = 0; kk < HS / 8; ++kk) {
          const int sl = kk >> 2, sub = kk & 3;
          const uint64_t dqh = desc_kmajor(qh + sl * (AQ * 128), sub), dql = desc_kmajor(ql + sl * (AQ * 128), sub);
          const uint64_t dkh = desc_kmajor(kh + sl * (AK * 128), sub), dkl = desc_kmajor(kl + sl * (AK * 128), sub);
          mma_tf32(dS, dql, dkh, id_s, kk > 0 ? 1u : 0u);
          mma_tf32(dS, dqh, dkl, id_s, 1u);
          mma_tf32(dS, dqh, dkh, id_s, 1u);
        }
        issued = true;
        mma_commit(smem_u32(&s_full[s]));
        return true;
      };
      ok = ok && issue_s(0);
      for (int it = 0; it < iters && ok; ++it) {
        // the next block's scores first, so the softmax warps never wait for them
        if (it + 1 < iters && !issue_s(it + 1)) { ok = false; break; }
        const int s = it & 1;
        if (it >= nkb) {
          // O += P V for the two 32-key halves of this block
          const uint32_t vh = smem_u32(smem + CF::kOffStage + s * CF::kStageBytes) + 2 * CF::kKBytes;
          const uint32_t vl = vh + CF::kKBytes;
          for (int half = 0; half < 2; ++half, ++pcount) {
            if (!mbar_wait(smem_u32(p_full), pcount & 1, abort_flag, a.err, 35)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t pvh = vh + half * (HS / 32) * 4096, pvl = vl + half * (HS / 32) * 4096;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t dph = desc_kmajor(smem_u32(p_h), kk), dpl = desc_kmajor(smem_u32(p_l), kk);
              const uint64_t dvh = desc_mnmajor(pvh, kk), dvl = desc_mnmajor(pvl, kk);
              const uint32_t acc0 = (pcount > 0 || kk > 0) ? 1u : 0u;
              mma_tf32(tmem + 128, dpl, dvh, id_o, acc0);
              mma_tf32(tmem + 128, dph, dvl, id_o, 1u);
              mma_tf32(tmem + 128, dph, dvh, id_o, 1u);
            }
            mma_commit(smem_u32(p_empty));
          }
          if (!ok) break;
        }
        mma_commit(smem_u32(&kv_empty[s]));   // K (and V) of this stage are consumed
      }
      if (ok) mma_commit(smem_u32(o_full));
      if (!ok && issued) {
        mma_commit(smem_u32(drain));
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(drain), 0) && gtimer() - t0 < kWaitNs) {}
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax warps ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;      // TMEM lane == tile row
    const int q = q0 + row;                   // query index in the head
    const bool issuer = (warp == 2 && lane == 0);
    float m = -INFINITY, l = 0.0f;
    int pcount = 0;
    bool ok = true;
    for (int it = 0; it < iters && ok; ++it) {
      const int s = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const bool failed = !mbar_wait(smem_u32(&s_full[s]), ph, abort_flag, a.err, 36);
      if (any128(failed)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const bool pass2 = it >= nkb;
      const int kb = pass2 ? it - nkb : it;
      uint32_t r[64];
      const uint32_t taddr = tmem + s * AK + ((uint32_t)(quarter * 32) << 16);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
            "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
            "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
            "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr));
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]),
            "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]),
            "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]),
            "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]),
            "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
          : "r"(taddr + 32));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      // scores of this block; keys past the query are masked (exp -> 0)
      float sv[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int key = kb * AK + c;
        sv[c] = key <= q ? __uint_as_float(r[c]) * a.scale : -INFINITY;
      }
      if (!pass2) {
        float bm = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) bm = fmaxf(bm, sv[c]);
        const float mn = fmaxf(m, bm);
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < 64; ++c) sum += expf(sv[c] - mn);
        l = (m == -INFINITY ? 0.0f : l * expf(m - mn)) + sum;
        m = mn;
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&s_empty[s]));
        continue;
      }
      // pass 2: S has been read into registers: release the TMEM buffer, then
      // p = exp(s - m) / l for the whole block before touching the stage
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_empty[s]));
      const float inv_l = 1.0f / l;
#pragma unroll
      for (int c = 0; c < 64; ++c) sv[c] = expf(sv[c] - m) * inv_l;
#pragma unroll
      for (int half = 0; half < 2; ++half, ++pcount) {
        // the stage is free once the previous P V MMAs and the previous TMA
        // store have finished reading it
        bool failed2 = false;
        if (issuer) {
          if (pcount > 0) failed2 = !mbar_wait(smem_u32(p_empty), (pcount - 1) & 1, abort_flag, a.err, 37);
          bulk_wait_read<0>();
        }
        if (any128(failed2)) { ok = false; break; }   // also the barrier before the stage is rewritten
        float4* rh = reinterpret_cast<float4*>(p_h + row * 128);
        float4* rl = reinterpret_cast<float4*>(p_l + row * 128);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float pv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) pv[e] = sv[32 * half + 4 * g + e];
          const float4 h4 = make_float4(tf32_rn(pv[0]), tf32_rn(pv[1]), tf32_rn(pv[2]), tf32_rn(pv[3]));
          rh[g ^ (row & 7)] = h4;
          rl[g ^ (row & 7)] = make_float4(tf32_rn(pv[0] - h4.x), tf32_rn(pv[1] - h4.y),
                                          tf32_rn(pv[2] - h4.z), tf32_rn(pv[3] - h4.w));
        }
        fence_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (issuer) {
          mbar_arrive(smem_u32(p_full));
          tma_store_2d(&mPh, smem_u32(p_h), kb * AK + 32 * half, row_base + q0);
          tma_store_2d(&mPl, smem_u32(p_l), kb * AK + 32 * half, row_base + q0);
          bulk_commit();
        }
      }
    }
    // O = P V: read the accumulator and write head-unfolded tf32 planes
    if (ok && mbar_wait(smem_u32(o_full), 0, abort_flag, a.err, 38)) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int b = z / a.H, h = z % a.H;
      const size_t C = (size_t)a.H * HS;
      float* oh = a.o_hi + ((size_t)b * a.T + q) * C + (size_t)h * HS;
      float* ol = a.o_lo + ((size_t)b * a.T + q) * C + (size_t)h * HS;
#pragma unroll
      for (int c0 = 0; c0 < HS; c0 += 32) {
        uint32_t o[32];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]), "=r"(o[4]), "=r"(o[5]), "=r"(o[6]),
              "=r"(o[7]), "=r"(o[8]), "=r"(o[9]), "=r"(o[10]), "=r"(o[11]), "=r"(o[12]), "=r"(o[13]),
              "=r"(o[14]), "=r"(o[15]), "=r"(o[16]), "=r"(o[17]), "=r"(o[18]), "=r"(o[19]),
              "=r"(o[20]), "=r"(o[21]), "=r"(o[22]), "=r"(o[23]), "=r"(o[24]), "=r"(o[25]),
              "=r"(o[26]), "=r"(o[27]), "=r"(o[28]), "=r"(o[29]), "=r"(o[30]), "=r"(o[31])
            : "r"(tmem + 128 + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 v = make_float4(__uint_as_float(o[j]), __uint_as_float(o[j + 1]),
                                       __uint_as_float(o[j + 2]), __uint_as_float(o[j + 3]));
          const float4 h4 = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
          *reinterpret_cast<float4*>(oh + c0 + j) = h4;
          *reinterpret_cast<float4*>(ol + c0 + j) =
              make_float4(tf32_rn(v.x - h4.x), tf32_rn(v.y - h4.y), tf32_rn(v.z - h4.z), tf32_rn(v.w - h4.w));
        }
      }
    }
    if (issuer) bulk_wait<0>();   // the P stores have landed before the CTA exits
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

template <int HS>
void launch_attn(const float* qkv_hi, const float* qkv_lo, int B, int H, int T, float scale,
                 float* p_hi, float* p_lo, float* o_hi, float* o_lo) {
  using CF = AttnCfg<HS>;
  const uint64_t BHT = (uint64_t)B * H * T;
  const uint64_t plane = BHT * HS * 4;           // bytes of one of q, k, v
  // Q / K: {hs, B*H*T rows, 3 (q,k,v)}, box {32, 64, 1}, 128-B swizzle (K-major tiles)
  const uint64_t d3[3] = {(uint64_t)HS, BHT, 3}, s3[2] = {(uint64_t)HS * 4, plane};
  const uint32_t b3[3] = {32, 64, 1};
  // V: {32, rows, hs/32 chunks, 3}, box {32, 32 keys, hs/32, 1}, 32-B-granule swizzle (MN-major)
  const uint64_t d4[4] = {32, BHT, (uint64_t)HS / 32, 3}, s4[3] = {(uint64_t)HS * 4, 128, plane};
  const uint32_t b4[4] = {32, 32, (uint32_t)HS / 32, 1};
  // P: {T, B*H*T rows}, box {32 keys, 128 rows}, 128-B swizzle (the shared stage's layout)
  const uint64_t d2[2] = {(uint64_t)T, BHT}, s2[1] = {(uint64_t)T * 4};
  const uint32_t b2[2] = {32, 128};
  CUtensorMap qh = encode_f32_map(3, qkv_hi, d3, s3, b3, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ql = encode_f32_map(3, qkv_lo, d3, s3, b3, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap vh = encode_f32_map(4, qkv_hi, d4, s4, b4, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  CUtensorMap vl = encode_f32_map(4, qkv_lo, d4, s4, b4, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  CUtensorMap ph = encode_f32_map(2, p_hi, d2, s2, b2, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap pl = encode_f32_map(2, p_lo, d2, s2, b2, CU_TENSOR_MAP_SWIZZLE_128B);
  AttnArgs args{H, T, HS, scale, o_hi, o_lo, device_error_word()};
  static bool attr = false;
  if (!attr) {
    MALUS_CUDA(cudaFuncSetAttribute(k_attn_fwd<HS>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr = true;
  }
  const unsigned grid = (unsigned)(B * H * (T / AQ));
  k_attn_fwd<HS><<<grid, 192, CF::kSmem, stream()>>>(qh, ql, vh, vl, ph, pl, args);
  count_launch();
  after_launch("k_attn_fwd");
}

}  // namespace

bool attn_fwd_supported(int T, int hs) { return T % AQ == 0 && (hs == 32 || hs == 64); }

// qkv planes: [3][B][H][T][hs] (q, k, v); P planes [B*H][T][T] (keys up to each
// query's 128-wide tile written); O planes [B*T][H*hs].
void attn_fwd(const float* qkv_hi, const float* qkv_lo, int B, int H, int T, int hs, float scale,
              float* p_hi, float* p_lo, float* o_hi, float* o_lo) {
  if (!attn_fwd_supported(T, hs)) panic("attn_fwd: needs T %% 128 == 0 and hs in {32, 64} (T=%d hs=%d)", T, hs);
  for (const void* p : {(const void*)qkv_hi, (const void*)qkv_lo, (const void*)p_hi, (const void*)p_lo,
                        (const void*)o_hi, (const void*)o_lo})
    if ((uintptr_t)p & 15) panic("attn_fwd: buffers must be 16-byte aligned");
  if (hs == 64) launch_attn<64>(qkv_hi, qkv_lo, B, H, T, scale, p_hi, p_lo, o_hi, o_lo);
  else launch_attn<32>(qkv_hi, qkv_lo, B, H, T, scale, p_hi, p_lo, o_hi, o_lo);
}

}  // namespace malus

extern "C" int32_t malus_attn_fwd(const float* qkv_hi, const float* qkv_lo, int32_t B, int32_t H,
                                  int32_t T, int32_t hs, float scale, float* p_hi, float* p_lo,
                                  float* o_hi, float* o_lo) {
  if (!malus::attn_fwd_supported(T, hs)) return -1;
  malus::attn_fwd(qkv_hi, qkv_lo, B, H, T, hs, scale, p_hi, p_lo, o_hi, o_lo);
  return 0;
}
