// Fused causal attention forward on tcgen05 (3xTF32): S = Q K^T * scale,
// causal softmax, O = P V in one kernel, without an f32 score tensor.
//
// Reference semantics (examples/nanogpt_modular.ml attention block; the mask of
// metal.rs:1601-1612): scores = (Q K^T) * 1/sqrt(hs) + mask(-1e9 above the
// diagonal), P = softmax(scores, axis -1), O = P V.  Masked scores underflow to
// exactly 0 after the exponential, so keys past the diagonal are skipped.
//
// One CTA = one head (z = b*H + h) x 128 query rows; 320 threads:
//   warp 0     TMA producer: Q once (tf32 hi/lo planes), then key blocks of 64
//              keys: K through two stages (both passes), V into one buffer
//              (pass 2, after the previous block's P V);
//   warp 1     TMEM owner and MMA issuer: S_b = Q K^T into two 64-column TMEM
//              buffers (one block ahead), O += P V into a third region;
//   warps 2-9  softmax, two groups of four warps: group g owns keys 32g..32g+31
//              of every block, one thread per query row (its TMEM lane).
//              Pass 1: each group's row max and sum (online), combined once.
//              Pass 2: S recomputed, p = 2^(s*scale*log2 e - m2) * (1/l) written into
//              the group's own swizzled shared stage, which is both the A
//              operand of that half's P V MMA and the source of a TMA store of
//              the P planes (the backward reads them); finally O is read from
//              TMEM and written as head-unfolded tf32 planes [B*T][H*hs].
// Every mbarrier wait is bounded; on timeout the CTA records an error, drains
// its MMAs and returns.
#include "common.cuh"
#include "tc_common.cuh"

namespace malus {
namespace {
using namespace malus::tc;

// OR of `v` over the 256 softmax threads (named barrier 1): every exit
// decision in those warps is collective, so no thread is left at a barrier.
__device__ __forceinline__ bool any256(bool v) {
  __syncwarp();   // the barrier needs the warp converged (lane 0 may have waited alone)
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}
// barrier among the 128 threads of softmax group g (named barriers 2 and 3)
__device__ __forceinline__ void group_sync(int g) {
  __syncwarp();
  asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory");
}

constexpr int AQ = 128;  // query rows per CTA
constexpr int AK = 64;   // keys per block
constexpr int kAttnThreads = 64 + 256;   // producer, MMA, 8 softmax warps

// The resident-score kernel (k_attn_fwd_rs) serves T <= 384 unless switched
// off (MALUS_ATTN_RS=0, or malus_attn_set_resident(0)); both kernels give the
// same bits.
int g_attn_rs = -1;
bool attn_resident_on() {
  if (g_attn_rs < 0) {
    const char* e = getenv("MALUS_ATTN_RS");
    g_attn_rs = (e && e[0] == '0') ? 0 : 1;
  }
  return g_attn_rs != 0;
}

template <int HS>
struct AttnCfg {
  static constexpr int kQBytes = AQ * HS * 4;              // one plane of the Q tile
  static constexpr int kKBytes = AK * HS * 4;              // one plane of a K (or V) block
  static constexpr int kPBytes = AQ * 32 * 4;              // one plane of a 32-key P half
  static constexpr int kOffK = 2 * kQBytes;                // two K stages (hi, lo)
  static constexpr int kOffV = kOffK + 2 * 2 * kKBytes;    // one V buffer (hi, lo)
  static constexpr int kOffP = kOffV + 2 * kKBytes;        // two P stages (hi, lo), one per half
  // [2 groups][128 rows] (m, l) at the end of pass 1.  Aliases P stage 0: every
  // thread reads the other group's statistics before the first collective
  // any256() of pass 2, and no P stage is written before that.
  static constexpr int kOffStats = kOffP;
  static constexpr int kOffBar = kOffP + 2 * 2 * kPBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;
  static_assert(kSmem <= 232448, "shared memory");
};

struct AttnArgs {
  int H, T, hs;
  float scale;
  float* o_hi;
  float* o_lo;
  float2* stats;   // optional [B*H*T] (row max of the scores in base-2 units, 1 / row sum)
  int store_p;     // write the P planes
  int32_t* err;
};

template <int HS>
__global__ void __launch_bounds__(kAttnThreads, 1)
k_attn_fwd(const __grid_constant__ CUtensorMap mQKh, const __grid_constant__ CUtensorMap mQKl,
           const __grid_constant__ CUtensorMap mVh, const __grid_constant__ CUtensorMap mVl,
           const __grid_constant__ CUtensorMap mPh, const __grid_constant__ CUtensorMap mPl,
           const AttnArgs a) {
  using CF = AttnCfg<HS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(smem + CF::kOffBar);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* k_empty = bar + 3;   // [2]
  uint64_t* s_full = bar + 5;    // [2]
  uint64_t* s_empty = bar + 7;   // [2]
  uint64_t* p_full = bar + 9;    // [2] one per P half
  uint64_t* p_empty = bar + 11;  // [2]
  uint64_t* v_full = bar + 13;
  uint64_t* v_empty = bar + 14;
  uint64_t* o_full = bar + 15;
  uint64_t* drain = bar + 16;
  uint64_t* done = bar + 17;   // the eight softmax warps finished reading TMEM
  uint32_t* tmem_slot = (uint32_t*)(bar + 18);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float2* stats = (float2*)(smem + CF::kOffStats);

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
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_empty[i]), 8);
      mbar_init(smem_u32(&p_full[i]), 1);
      mbar_init(smem_u32(&p_empty[i]), 1);
    }
    mbar_init(smem_u32(v_full), 1);
    mbar_init(smem_u32(v_empty), 1);
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(done), 8);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)), "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();   // lane 0 of the producer / MMA warps may arrive alone: reconverge first
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;   // S buffers at columns 0 and 64, O at 128

  uint8_t* q_h = smem;
  uint8_t* q_l = smem + CF::kQBytes;
  uint8_t* v_h = smem + CF::kOffV;
  uint8_t* v_l = v_h + CF::kKBytes;

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
      int it = 0, vcount = 0;
      bool ok = true;
      for (; it < iters && ok; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (it >= 2 && !mbar_wait(smem_u32(&k_empty[s]), ph ^ 1, abort_flag, a.err, 31)) { ok = false; break; }
        const bool pass2 = it >= nkb;
        const int kb = pass2 ? it - nkb : it;
        uint8_t* kst = smem + CF::kOffK + s * 2 * CF::kKBytes;
        const uint32_t fb = smem_u32(&k_full[s]);
        mbar_expect_tx(fb, 2 * CF::kKBytes);
        for (int sl = 0; sl < HS / 32; ++sl) {
          tma_load_3d(smem_u32(kst + sl * (AK * 128)), &mQKh, fb, sl * 32, row_base + kb * AK, 1);
          tma_load_3d(smem_u32(kst + CF::kKBytes + sl * (AK * 128)), &mQKl, fb, sl * 32, row_base + kb * AK, 1);
        }
        if (pass2) {
          // the V buffer is free once the previous block's P V MMAs are done
          if (vcount > 0 && !mbar_wait(smem_u32(v_empty), (vcount - 1) & 1, abort_flag, a.err, 39)) {
            ok = false;
            ++it;   // K of this block is in flight and must be drained
            break;
          }
          const uint32_t vb = smem_u32(v_full);
          mbar_expect_tx(vb, 2 * CF::kKBytes);
          for (int half = 0; half < 2; ++half) {
            const uint32_t voff = half * (HS / 32) * 4096;
            tma_load_4d(smem_u32(v_h + voff), &mVh, vb, 0, row_base + kb * AK + 32 * half, 0, 2);
            tma_load_4d(smem_u32(v_l + voff), &mVl, vb, 0, row_base + kb * AK + 32 * half, 0, 2);
          }
          ++vcount;
        }
      }
      if (*abort_flag) {
        // every issued load must land before the CTA exits
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(q_full), 0) && gtimer() - t0 < kWaitNs) {}
        for (int qi = it > 2 ? it - 2 : 0; qi < it; ++qi) {
          t0 = gtimer();
          while (!mbar_try(smem_u32(&k_full[qi & 1]), (qi >> 1) & 1) && gtimer() - t0 < kWaitNs) {}
        }
        if (vcount > 0) {
          t0 = gtimer();
          while (!mbar_try(smem_u32(v_full), (vcount - 1) & 1) && gtimer() - t0 < kWaitNs) {}
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
      // descriptors built once; a stage or k-step adds (byte offset / 16) (the
      // address field is the low 14 bits, every address is below 256 KB)
      const uint64_t dqh = desc_kmajor(smem_u32(q_h), 0), dql = desc_kmajor(smem_u32(q_l), 0);
      const uint64_t dk0 = desc_kmajor(smem_u32(smem + CF::kOffK), 0);
      const uint64_t dp0 = desc_kmajor(smem_u32(smem + CF::kOffP), 0);
      const uint64_t dv0 = desc_mnmajor(smem_u32(v_h), 0);
      // S_it = Q K_it^T into TMEM buffer it & 1
      auto issue_s = [&](int it) -> bool {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&k_full[s]), ph, abort_flag, a.err, 33)) return false;
        if (it >= 2 && !mbar_wait(smem_u32(&s_empty[s]), ph ^ 1, abort_flag, a.err, 34)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t kh = dk0 + (uint64_t)(s * (2 * CF::kKBytes / 16)), kl = kh + CF::kKBytes / 16;
        const uint32_t dS = tmem + s * AK;
#pragma unroll
        for (int kk = 0; kk < HS / 8; ++kk) {
          const uint64_t oa = (uint64_t)((kk >> 2) * (AQ * 128 / 16) + (kk & 3) * 2);
          const uint64_t ob = (uint64_t)((kk >> 2) * (AK * 128 / 16) + (kk & 3) * 2);
          mma_tf32(dS, dql + oa, kh + ob, id_s, kk > 0 ? 1u : 0u);
          mma_tf32(dS, dqh + oa, kl + ob, id_s, 1u);
          mma_tf32(dS, dqh + oa, kh + ob, id_s, 1u);
        }
        issued = true;
        mma_commit(smem_u32(&s_full[s]));
        mma_commit(smem_u32(&k_empty[s]));   // K of this stage is consumed once these finish
        return true;
      };
      ok = ok && issue_s(0);
      int vcount = 0;
      for (int it = 0; it < iters && ok; ++it) {
        // the next block's scores first, so the softmax warps never wait for them
        if (it + 1 < iters && !issue_s(it + 1)) { ok = false; break; }
        if (it < nkb) continue;
        // O += P V, half g from P stage g
        if (!mbar_wait(smem_u32(v_full), vcount & 1, abort_flag, a.err, 40)) { ok = false; break; }
        for (int g = 0; g < 2; ++g) {
          const int pc = vcount;   // uses of each P stage so far
          if (!mbar_wait(smem_u32(&p_full[g]), pc & 1, abort_flag, a.err, 35)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ph0 = dp0 + (uint64_t)(g * (2 * CF::kPBytes / 16)), pl0 = ph0 + CF::kPBytes / 16;
          const uint64_t vh0 = dv0 + (uint64_t)(g * (HS / 32) * (4096 / 16)), vl0 = vh0 + CF::kKBytes / 16;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dph = ph0 + (uint64_t)(kk * 2), dpl = pl0 + (uint64_t)(kk * 2);
            const uint64_t dvh = vh0 + (uint64_t)(kk * 64), dvl = vl0 + (uint64_t)(kk * 64);
            const uint32_t acc0 = (vcount > 0 || g > 0 || kk > 0) ? 1u : 0u;
            mma_tf32(tmem + 128, dpl, dvh, id_o, acc0);
            mma_tf32(tmem + 128, dph, dvl, id_o, 1u);
            mma_tf32(tmem + 128, dph, dvh, id_o, 1u);
          }
          mma_commit(smem_u32(&p_empty[g]));
        }
        if (!ok) break;
        mma_commit(smem_u32(v_empty));
        ++vcount;
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
    // ---------------- softmax warps: group g owns keys 32g..32g+31 of each block ----------------
    const int quarter = warp & 3;
    const int g = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;      // TMEM lane == tile row
    const int q = q0 + row;                   // query index in the head
    const bool issuer = (warp == 2 + 4 * g) && lane == 0;
    uint8_t* p_h = smem + CF::kOffP + g * 2 * CF::kPBytes;
    uint8_t* p_l = p_h + CF::kPBytes;
    float m = -INFINITY, l = 0.0f, inv_l = 0.0f;   // row max (base-2 units) and sum
    const float sl2e = a.scale * kLog2e;
    int pcount = 0;
    bool ok = true;
    for (int it = 0; it < iters && ok; ++it) {
      const int s = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const bool failed = !mbar_wait(smem_u32(&s_full[s]), ph, abort_flag, a.err, 36);
      if (any256(failed)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const bool pass2 = it >= nkb;
      const int kb = pass2 ? it - nkb : it;
      if (it == nkb) {
        // end of pass 1: combine the two groups' row statistics
        stats[g * AQ + row] = make_float2(m, l);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const float2 o = stats[(1 - g) * AQ + row];
        const float mm = fmaxf(m, o.x);
        l = (m == -INFINITY ? 0.0f : l * exp2_hw(m - mm)) + (o.x == -INFINITY ? 0.0f : o.y * exp2_hw(o.x - mm));
        m = mm;
        inv_l = 1.0f / l;
        if (g == 0 && a.stats) a.stats[row_base + q] = make_float2(m, inv_l);
      }
      uint32_t r[32];
      tmem_ld32(tmem + s * AK + 32 * g + ((uint32_t)(quarter * 32) << 16), r);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_empty[s]));   // S is in registers
      // scores in base-2 units: exp(s*scale - m) = 2^(s*scale*log2 e - m2)
      const int key0 = kb * AK + 32 * g;   // keys past the query are masked (P = 0)
      float sv[32];
      if (!pass2) {
        float bm = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (key0 + c <= q) bm = fmaxf(bm, __uint_as_float(r[c]) * sl2e);
        const float mn = fmaxf(m, bm);
        if (mn != -INFINITY) {
          float sum = 0.0f;
#pragma unroll
          for (int c = 0; c < 32; ++c)
            sum += key0 + c <= q ? exp2_hw(fmaf(__uint_as_float(r[c]), sl2e, -mn)) : 0.0f;
          l = (m == -INFINITY ? 0.0f : l * exp2_hw(m - mn)) + sum;
          m = mn;
        }
        continue;
      }
      // pass 2: p = 2^(s2 - m2) / l for this group's 32 keys, then the P stage
#pragma unroll
      for (int c = 0; c < 32; ++c)
        sv[c] = key0 + c <= q ? exp2_hw(fmaf(__uint_as_float(r[c]), sl2e, -m)) * inv_l : 0.0f;
      bool failed2 = false;
      if (issuer) {
        if (pcount > 0) failed2 = !mbar_wait(smem_u32(&p_empty[g]), (pcount - 1) & 1, abort_flag, a.err, 37);
        bulk_wait_read<0>();
      }
      if (any256(failed2)) { ok = false; break; }   // also: the stage is free for the whole group
      float4* rh = reinterpret_cast<float4*>(p_h + row * 128);
      float4* rl = reinterpret_cast<float4*>(p_l + row * 128);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = make_float4(sv[4 * j], sv[4 * j + 1], sv[4 * j + 2], sv[4 * j + 3]);
        const float4 h4 = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
        rh[j ^ (row & 7)] = h4;
        rl[j ^ (row & 7)] = make_float4(tf32_rn(v.x - h4.x), tf32_rn(v.y - h4.y), tf32_rn(v.z - h4.z),
                                        tf32_rn(v.w - h4.w));
      }
      fence_async_smem();
      group_sync(g);
      if (issuer) {
        mbar_arrive(smem_u32(&p_full[g]));
        if (a.store_p) {
          tma_store_2d(&mPh, smem_u32(p_h), kb * AK + 32 * g, row_base + q0);
          tma_store_2d(&mPl, smem_u32(p_l), kb * AK + 32 * g, row_base + q0);
          bulk_commit();
        }
      }
      ++pcount;
    }
    // O = P V: group g reads and writes columns [g*HS/2, (g+1)*HS/2) as head-unfolded tf32 planes
    if (ok && mbar_wait(smem_u32(o_full), 0, abort_flag, a.err, 38)) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int b = z / a.H, h = z % a.H;
      const size_t C = (size_t)a.H * HS;
      float* oh = a.o_hi + ((size_t)b * a.T + q) * C + (size_t)h * HS;
      float* ol = a.o_lo + ((size_t)b * a.T + q) * C + (size_t)h * HS;
#pragma unroll
      for (int c0 = g * 32; c0 < HS; c0 += 64) {
        uint32_t o[32];
        tmem_ld32(tmem + 128 + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, o);
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
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(done));
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();   // lane 0 of the producer / MMA warps may arrive alone: reconverge first
  __syncthreads();
  if (warp == 1) {
    // TMEM is freed only after every softmax warp said it finished reading it
    mbar_wait_bounded(smem_u32(done), 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

// ---------------------------------------------------------------------------
// Resident-score variant (T <= 384).  A 128-query tile has at most 384 keys up
// to its diagonal, so all its score blocks fit in tensor memory at once (64
// columns per 64-key block) beside O.  S = Q K^T is then computed once: pass 1
// reads the resident blocks for the row max and sum, pass 2 reads them again
// for P.  K blocks and then V blocks stream through one three-stage ring, so V
// is prefetched while pass 1 runs, and each softmax group has two P stages
// (the second one in Q's shared memory once every S product is done, for
// hs = 64), so a block's P is written while the previous block's P V runs and
// its TMA store drains.  The products and their order (S per block with the
// same three tf32 MMAs per k-step; O accumulated over blocks, halves and
// k-steps in the same order) and the softmax expressions are those of
// k_attn_fwd, so both kernels give the same bits.
constexpr int kRsMaxBlocks = 6;   // 384 keys
constexpr int kRsRing = 3;
constexpr int kRsOCol = kRsMaxBlocks * AK;   // O after the score columns

template <int HS>
struct AttnRsCfg {
  static constexpr int kQBytes = AQ * HS * 4;
  static constexpr int kKBytes = AK * HS * 4;              // one plane of a K or V block
  static constexpr int kStage = 2 * kKBytes;               // hi + lo
  static constexpr int kPBytes = AQ * 32 * 4;              // one plane of a 32-key P half
  static constexpr int kPStage = 2 * kPBytes;              // hi + lo
  static constexpr int kOffRing = 2 * kQBytes;
  static constexpr int kOffP0 = kOffRing + kRsRing * kStage;          // P buffer 0 of both groups
  static constexpr bool kP1InQ = 2 * kQBytes >= 2 * kPStage;         // buffer 1 reuses Q (hs = 64)
  static constexpr int kOffP1 = kP1InQ ? 0 : kOffP0 + 2 * kPStage;
  static constexpr int kOffStats = kOffP0;                 // as in k_attn_fwd: read before any P write
  static constexpr int kOffBar = (kP1InQ ? kOffP0 + 2 * kPStage : kOffP1 + 2 * kPStage);
  static constexpr int kSmem = kOffBar + 512 + 1024;
  static_assert(kSmem <= 232448, "shared memory");
};

template <int HS>
__global__ void __launch_bounds__(kAttnThreads, 1)
k_attn_fwd_rs(const __grid_constant__ CUtensorMap mQKh, const __grid_constant__ CUtensorMap mQKl,
              const __grid_constant__ CUtensorMap mVh, const __grid_constant__ CUtensorMap mVl,
              const __grid_constant__ CUtensorMap mPh, const __grid_constant__ CUtensorMap mPl,
              const __grid_constant__ CUtensorMap mOh, const __grid_constant__ CUtensorMap mOl,
              const AttnArgs a) {
  using CF = AttnRsCfg<HS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(smem + CF::kOffBar);
  uint64_t* q_full = bar;
  uint64_t* r_full = bar + 1;                    // [kRsRing]
  uint64_t* r_empty = bar + 1 + kRsRing;         // [kRsRing]
  uint64_t* s_full = bar + 1 + 2 * kRsRing;      // [kRsMaxBlocks], one use each
  uint64_t* p_full = s_full + kRsMaxBlocks;      // [2 groups][2 buffers]
  uint64_t* p_empty = p_full + 4;                // [2][2]
  uint64_t* o_full = p_empty + 4;
  uint64_t* drain = o_full + 1;
  uint64_t* done = drain + 1;
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float2* stats = (float2*)(smem + CF::kOffStats);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.T / AQ;
  const int qb = nq - 1 - (int)(blockIdx.x % nq);   // heavy (late) query blocks first
  const int z = (int)(blockIdx.x / nq);
  const int q0 = qb * AQ;
  const int nkb = (q0 + AQ) / AK;                     // key blocks up to the diagonal (<= 6)
  const int items = 2 * nkb;                          // ring items: K blocks, then V blocks
  const int row_base = z * a.T;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int i = 0; i < kRsRing; ++i) {
      mbar_init(smem_u32(&r_full[i]), 1);
      mbar_init(smem_u32(&r_empty[i]), 1);
    }
    for (int i = 0; i < kRsMaxBlocks; ++i) mbar_init(smem_u32(&s_full[i]), 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(smem_u32(&p_full[i]), 1);
      mbar_init(smem_u32(&p_empty[i]), 1);
    }
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(done), 8);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)), "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;   // S block b at columns 64 b, O at kRsOCol

  uint8_t* q_h = smem;
  uint8_t* q_l = smem + CF::kQBytes;

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
      for (; it < items; ++it) {
        const int st = it % kRsRing, use = it / kRsRing;
        if (use > 0 && !mbar_wait(smem_u32(&r_empty[st]), (use - 1) & 1, abort_flag, a.err, 41)) break;
        uint8_t* base = smem + CF::kOffRing + st * CF::kStage;
        const uint32_t fb = smem_u32(&r_full[st]);
        mbar_expect_tx(fb, CF::kStage);
        if (it < nkb) {
          const int kb = it;
          for (int sl = 0; sl < HS / 32; ++sl) {
            tma_load_3d(smem_u32(base + sl * (AK * 128)), &mQKh, fb, sl * 32, row_base + kb * AK, 1);
            tma_load_3d(smem_u32(base + CF::kKBytes + sl * (AK * 128)), &mQKl, fb, sl * 32, row_base + kb * AK, 1);
          }
        } else {
          const int kb = it - nkb;
          for (int half = 0; half < 2; ++half) {
            const uint32_t voff = half * (HS / 32) * 4096;
            tma_load_4d(smem_u32(base + voff), &mVh, fb, 0, row_base + kb * AK + 32 * half, 0, 2);
            tma_load_4d(smem_u32(base + CF::kKBytes + voff), &mVl, fb, 0, row_base + kb * AK + 32 * half, 0, 2);
          }
        }
      }
      if (*abort_flag) {
        // every issued load must land before the CTA exits (the last kRsRing
        // items are in distinct stages, each at its latest phase)
        uint64_t t0 = gtimer();
        while (!mbar_try(smem_u32(q_full), 0) && gtimer() - t0 < kWaitNs) {}
        for (int qi = it > kRsRing ? it - kRsRing : 0; qi < it; ++qi) {
          t0 = gtimer();
          while (!mbar_try(smem_u32(&r_full[qi % kRsRing]), (qi / kRsRing) & 1) && gtimer() - t0 < kWaitNs) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc_tf32(false, false, AK);
      const uint32_t id_o = idesc_tf32(false, true, HS);
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, a.err, 42);
      bool issued = false;
      const uint64_t dqh = desc_kmajor(smem_u32(q_h), 0), dql = desc_kmajor(smem_u32(q_l), 0);
      const uint64_t dr0 = desc_kmajor(smem_u32(smem + CF::kOffRing), 0);
      const uint64_t dv0 = desc_mnmajor(smem_u32(smem + CF::kOffRing), 0);
      // S_b = Q K_b^T for every block, as the K blocks land
      for (int b = 0; b < nkb && ok; ++b) {
        const int st = b % kRsRing;
        if (!mbar_wait(smem_u32(&r_full[st]), (b / kRsRing) & 1, abort_flag, a.err, 43)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t kh = dr0 + (uint64_t)(st * (CF::kStage / 16)), kl = kh + CF::kKBytes / 16;
        const uint32_t dS = tmem + b * AK;
#pragma unroll
        for (int kk = 0; kk < HS / 8; ++kk) {
          const uint64_t oa = (uint64_t)((kk >> 2) * (AQ * 128 / 16) + (kk & 3) * 2);
          const uint64_t ob = (uint64_t)((kk >> 2) * (AK * 128 / 16) + (kk & 3) * 2);
          mma_tf32(dS, dql + oa, kh + ob, id_s, kk > 0 ? 1u : 0u);
          mma_tf32(dS, dqh + oa, kl + ob, id_s, 1u);
          mma_tf32(dS, dqh + oa, kh + ob, id_s, 1u);
        }
        issued = true;
        mma_commit(smem_u32(&s_full[b]));
        mma_commit(smem_u32(&r_empty[st]));
      }
      // O += P_b V_b, half g from group g's P buffer b & 1
      for (int b = 0; b < nkb && ok; ++b) {
        const int it = nkb + b, st = it % kRsRing;
        if (!mbar_wait(smem_u32(&r_full[st]), (it / kRsRing) & 1, abort_flag, a.err, 44)) { ok = false; break; }
        const int buf = b & 1, use = b >> 1;
        for (int g = 0; g < 2; ++g) {
          if (!mbar_wait(smem_u32(&p_full[g * 2 + buf]), use & 1, abort_flag, a.err, 45)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t poff = (buf ? CF::kOffP1 : CF::kOffP0) + g * CF::kPStage;
          const uint64_t ph0 = desc_kmajor(smem_u32(smem + poff), 0), pl0 = ph0 + CF::kPBytes / 16;
          const uint64_t vh0 = dv0 + (uint64_t)(st * (CF::kStage / 16)) + (uint64_t)(g * (HS / 32) * (4096 / 16));
          const uint64_t vl0 = vh0 + CF::kKBytes / 16;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dph = ph0 + (uint64_t)(kk * 2), dpl = pl0 + (uint64_t)(kk * 2);
            const uint64_t dvh = vh0 + (uint64_t)(kk * 64), dvl = vl0 + (uint64_t)(kk * 64);
            const uint32_t acc0 = (b > 0 || g > 0 || kk > 0) ? 1u : 0u;
            mma_tf32(tmem + kRsOCol, dpl, dvh, id_o, acc0);
            mma_tf32(tmem + kRsOCol, dph, dvl, id_o, 1u);
            mma_tf32(tmem + kRsOCol, dph, dvh, id_o, 1u);
          }
          mma_commit(smem_u32(&p_empty[g * 2 + buf]));
        }
        if (!ok) break;
        mma_commit(smem_u32(&r_empty[st]));
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

    // ---------------- softmax warps: group g owns keys 32g..32g+31 of each block ----------------
    const int quarter = warp & 3;
    const int g = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;      // TMEM lane == tile row
    const int q = q0 + row;
    const bool issuer = (warp == 2 + 4 * g) && lane == 0;
    float m = -INFINITY, l = 0.0f, inv_l = 0.0f;
    const float sl2e = a.scale * kLog2e;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    // pass 1: row max and sum of this group's keys, block by block as S lands
    for (int b = 0; b < nkb && ok; ++b) {
      const bool failed = !mbar_wait(smem_u32(&s_full[b]), 0, abort_flag, a.err, 46);
      if (any256(failed)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t r[32];
      tmem_ld32(tmem + b * AK + 32 * g + lane_off, r);
      const int key0 = b * AK + 32 * g;
      float bm = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (key0 + c <= q) bm = fmaxf(bm, __uint_as_float(r[c]) * sl2e);
      const float mn = fmaxf(m, bm);
      if (mn != -INFINITY) {
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          sum += key0 + c <= q ? exp2_hw(fmaf(__uint_as_float(r[c]), sl2e, -mn)) : 0.0f;
        l = (m == -INFINITY ? 0.0f : l * exp2_hw(m - mn)) + sum;
        m = mn;
      }
    }
    if (ok) {
      // combine the two groups' row statistics
      stats[g * AQ + row] = make_float2(m, l);
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float2 o = stats[(1 - g) * AQ + row];
      const float mm = fmaxf(m, o.x);
      l = (m == -INFINITY ? 0.0f : l * exp2_hw(m - mm)) + (o.x == -INFINITY ? 0.0f : o.y * exp2_hw(o.x - mm));
      m = mm;
      inv_l = 1.0f / l;
      if (g == 0 && a.stats) a.stats[row_base + q] = make_float2(m, inv_l);
    }
    // pass 2: P from the resident scores, into buffer b & 1 of this group
    for (int b = 0; b < nkb && ok; ++b) {
      uint32_t r[32];
      tmem_ld32(tmem + b * AK + 32 * g + lane_off, r);
      const int key0 = b * AK + 32 * g;
      float sv[32];
#pragma unroll
      for (int c = 0; c < 32; ++c)
        sv[c] = key0 + c <= q ? exp2_hw(fmaf(__uint_as_float(r[c]), sl2e, -m)) * inv_l : 0.0f;
      const int buf = b & 1, use = b >> 1;
      bool failed2 = false;
      if (issuer) {
        if (use > 0) failed2 = !mbar_wait(smem_u32(&p_empty[g * 2 + buf]), (use - 1) & 1, abort_flag, a.err, 47);
        bulk_wait_read<1>();   // the store of this buffer's previous block has read it
      }
      if (any256(failed2)) { ok = false; break; }
      uint8_t* p_h = smem + (buf ? CF::kOffP1 : CF::kOffP0) + g * CF::kPStage;
      uint8_t* p_l = p_h + CF::kPBytes;
      float4* rh = reinterpret_cast<float4*>(p_h + row * 128);
      float4* rl = reinterpret_cast<float4*>(p_l + row * 128);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = make_float4(sv[4 * j], sv[4 * j + 1], sv[4 * j + 2], sv[4 * j + 3]);
        const float4 h4 = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
        rh[j ^ (row & 7)] = h4;
        rl[j ^ (row & 7)] = make_float4(tf32_rn(v.x - h4.x), tf32_rn(v.y - h4.y), tf32_rn(v.z - h4.z),
                                        tf32_rn(v.w - h4.w));
      }
      fence_async_smem();
      group_sync(g);
      if (issuer) {
        mbar_arrive(smem_u32(&p_full[g * 2 + buf]));
        if (a.store_p) {
          tma_store_2d(&mPh, smem_u32(p_h), key0, row_base + q0);
          tma_store_2d(&mPl, smem_u32(p_l), key0, row_base + q0);
        }
        bulk_commit();
      }
    }
    // O = P V: group g takes columns [32g, 32g + 32) of each 64 (hs = 32: group
    // 0 only) and stores them as head-unfolded tf32 planes [B*T][H*hs] by TMA,
    // staged in its P buffer 0 (every MMA and P store has read it by then)
    if (ok) {
      const bool failed = !mbar_wait(smem_u32(o_full), 0, abort_flag, a.err, 48);
      ok = !any256(failed);
    }
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int bb = z / a.H, h = z % a.H;
      uint8_t* o_h = smem + CF::kOffP0 + g * CF::kPStage;
      uint8_t* o_l = o_h + CF::kPBytes;
#pragma unroll
      for (int c0 = g * 32; c0 < HS; c0 += 64) {
        uint32_t o[32];
        tmem_ld32(tmem + kRsOCol + lane_off + (uint32_t)c0, o);
        if (issuer) bulk_wait_read<0>();
        group_sync(g);
        float4* rh = reinterpret_cast<float4*>(o_h + row * 128);
        float4* rl = reinterpret_cast<float4*>(o_l + row * 128);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 v = make_float4(__uint_as_float(o[4 * j]), __uint_as_float(o[4 * j + 1]),
                                       __uint_as_float(o[4 * j + 2]), __uint_as_float(o[4 * j + 3]));
          const float4 h4 = make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
          rh[j ^ (row & 7)] = h4;
          rl[j ^ (row & 7)] = make_float4(tf32_rn(v.x - h4.x), tf32_rn(v.y - h4.y), tf32_rn(v.z - h4.z),
                                          tf32_rn(v.w - h4.w));
        }
        fence_async_smem();
        group_sync(g);
        if (issuer) {
          tma_store_2d(&mOh, smem_u32(o_h), h * HS + c0, bb * a.T + q0);
          tma_store_2d(&mOl, smem_u32(o_l), h * HS + c0, bb * a.T + q0);
          bulk_commit();
        }
      }
    }
    if (issuer) bulk_wait<0>();   // the P and O stores have landed before the CTA exits
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(done));
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    mbar_wait_bounded(smem_u32(done), 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

template <int HS>
void launch_attn(const float* qkv_hi, const float* qkv_lo, int B, int H, int T, float scale,
                 float* p_hi, float* p_lo, float* o_hi, float* o_lo, float* stats) {
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
  // without P planes the P maps are never used; they describe a valid range anyway
  const bool store_p = p_hi != nullptr;
  CUtensorMap ph = store_p ? encode_f32_map(2, p_hi, d2, s2, b2, CU_TENSOR_MAP_SWIZZLE_128B) : qh;
  CUtensorMap pl = store_p ? encode_f32_map(2, p_lo, d2, s2, b2, CU_TENSOR_MAP_SWIZZLE_128B) : ql;
  AttnArgs args{H, T, HS, scale, o_hi, o_lo, reinterpret_cast<float2*>(stats), store_p ? 1 : 0,
                device_error_word()};
  const unsigned grid = (unsigned)(B * H * (T / AQ));
  if (attn_resident_on() && T <= kRsMaxBlocks * AK) {
    using RF = AttnRsCfg<HS>;
    static bool attr_rs = false;
    if (!attr_rs) {
      MALUS_CUDA(cudaFuncSetAttribute(k_attn_fwd_rs<HS>, cudaFuncAttributeMaxDynamicSharedMemorySize, RF::kSmem));
      attr_rs = true;
    }
    // O planes [B*T][H*hs], box {32 columns, 128 rows}: the layout of a P stage
    const uint64_t dO[2] = {(uint64_t)H * HS, (uint64_t)B * T}, sO[1] = {(uint64_t)H * HS * 4};
    const uint32_t bO[2] = {32, 128};
    CUtensorMap oh = encode_f32_map(2, o_hi, dO, sO, bO, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap ol = encode_f32_map(2, o_lo, dO, sO, bO, CU_TENSOR_MAP_SWIZZLE_128B);
    k_attn_fwd_rs<HS><<<grid, kAttnThreads, RF::kSmem, stream()>>>(qh, ql, vh, vl, ph, pl, oh, ol, args);
    count_launch();
    after_launch("k_attn_fwd_rs");
    return;
  }
  static bool attr = false;
  if (!attr) {
    MALUS_CUDA(cudaFuncSetAttribute(k_attn_fwd<HS>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr = true;
  }
  k_attn_fwd<HS><<<grid, kAttnThreads, CF::kSmem, stream()>>>(qh, ql, vh, vl, ph, pl, args);
  count_launch();
  after_launch("k_attn_fwd");
}

}  // namespace

bool attn_fwd_supported(int T, int hs) { return T % AQ == 0 && (hs == 32 || hs == 64); }

// qkv planes: [3][B][H][T][hs] (q, k, v); P planes [B*H][T][T] (keys up to each
// query's 128-wide tile written; optional: null skips them); O planes
// [B*T][H*hs]; stats (optional) [B*H*T] pairs (row max of the scaled scores
// in base-2 units, i.e. times log2 e; 1 / row sum), which the fused backward
// recomputes P from.
void attn_fwd(const float* qkv_hi, const float* qkv_lo, int B, int H, int T, int hs, float scale,
              float* p_hi, float* p_lo, float* o_hi, float* o_lo, float* stats) {
  if (!attn_fwd_supported(T, hs)) panic("attn_fwd: needs T %% 128 == 0 and hs in {32, 64} (T=%d hs=%d)", T, hs);
  if ((p_hi == nullptr) != (p_lo == nullptr)) panic("attn_fwd: P planes come in pairs");
  for (const void* p : {(const void*)qkv_hi, (const void*)qkv_lo, (const void*)p_hi, (const void*)p_lo,
                        (const void*)o_hi, (const void*)o_lo, (const void*)stats})
    if ((uintptr_t)p & 15) panic("attn_fwd: buffers must be 16-byte aligned");
  if (hs == 64) launch_attn<64>(qkv_hi, qkv_lo, B, H, T, scale, p_hi, p_lo, o_hi, o_lo, stats);
  else launch_attn<32>(qkv_hi, qkv_lo, B, H, T, scale, p_hi, p_lo, o_hi, o_lo, stats);
}

}  // namespace malus

// Select the fused attention forward for T <= 384: 1 = resident scores
// (default), 0 = scores recomputed per pass.  Returns the previous setting.
extern "C" int32_t malus_attn_set_resident(int32_t on) {
  const int32_t prev = malus::attn_resident_on() ? 1 : 0;
  malus::g_attn_rs = on ? 1 : 0;
  return prev;
}

extern "C" int32_t malus_attn_fwd(const float* qkv_hi, const float* qkv_lo, int32_t B, int32_t H,
                                  int32_t T, int32_t hs, float scale, float* p_hi, float* p_lo,
                                  float* o_hi, float* o_lo, float* stats) {
  if (!malus::attn_fwd_supported(T, hs)) return -1;
  malus::attn_fwd(qkv_hi, qkv_lo, B, H, T, hs, scale, p_hi, p_lo, o_hi, o_lo, stats);
  return 0;
}
