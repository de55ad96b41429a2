// Non-causal flash attention, head_dim 128, on the 5th-generation tensor cores (replaces the cuDNN SDPA local
// attention of the Ulysses forward, upstream Attention._run_local_attention called at
// h3_tp2/ulysses_exact.py:495-496).
//
// One CTA per (pair of 128-row query tiles, head).  TMEM (512 columns): S0 | S1 | O0 | O1, 128 f32 columns each.
//   warps 0-3 : softmax for query tile 0 (thread = query row = TMEM lane), warps 4-7: query tile 1
//   warp 8    : TMA producer (Q once; K and V tiles of 128 keys through 2-stage rings)
//   warp 9    : TMEM allocator + single-thread MMA issuer
// Per key tile j and query tile q:
//   S_q = Q_q K_j^T            tcgen05.mma kind::f16 bf16 x bf16 -> f32, both operands K-major in shared memory
//   softmax: one row per thread, exp2 on the MUFU, running max with lazy rescaling of O (only when the max grows by
//            more than 2^8), P written back into TMEM (columns 0..63 of S_q as packed 16-bit pairs)
//   O_q += P_q V_j             tcgen05.mma kind::f16 with A = P from TMEM, B = V (MN-major in shared memory)
// The MMA for S_q(j+1) is issued after O_q += P_q V_j, so the in-order tensor pipe never overwrites P before it is
// consumed, and the commit that publishes S_q(j+1) also covers that P.V (the softmax may rescale O right away).
// P.V runs in f16 when V is given in f16 (P in [0, 256], V exact in f16's normal range): the P rounding error is 8x
// below bf16's, which keeps the output within rel-L2 2e-3 of fp32 SDPA.  Every wait is bounded; no multicast.
#include <stdlib.h>

#include <mutex>

#include "common.cuh"

namespace h3b {
namespace attn {

constexpr int BQ = 128, BKV = 128, D = 128;
constexpr int TILE_BYTES = BQ * D * 2;  // 32 KB
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int KST = 2, VST = 2;
constexpr int THREADS = 320;
constexpr int SMEM_BYTES = (2 + KST + VST) * TILE_BYTES + 1024 + 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr int kDefaultPoly = 2;             // FMA-pipe exponential pairs per 8 (see poly_pairs)

struct Params {
  int64_t s_q, s_kv, valid_kv;
  int heads;
  float scale_log2;  // softmax scale * log2(e)
  uint16_t* o;
  int64_t o_tok, o_head;
  int nkv;
  const int32_t* range_flag;
  int range_mode;  // 0: flag set -> record H3B_ERANGE, skip; 1: flag set -> skip; 2: run only when the flag is set
  // the scaled fallback for a v beyond f16's range: per (head, column) the bits of max |v| (finite values); the f16 v
  // given holds v * 2^-e and the output column is multiplied by 2^e, e = colscale_exp(colmax[head * 128 + c])
  const uint32_t* colmax;
  // m_rows > 0: output row t goes to rank t / m_rows, row (rank * m_rows + t % m_rows) of peer_o[t / m_rows]
  int64_t m_rows;
  int rank;
  uint16_t* peer_o[H3B_MAX_RANKS];
  WaitCtl wc;
};

// Exponent e >= 0 of the power of two that brings a column of bf16 values whose largest magnitude has the bits
// `amax_bits` into f16's range: amax * 2^-e <= 65504.  A bf16 magnitude m * 2^E has m <= 1.9921875 < 65504 / 2^15,
// so e = max(0, E - 15) suffices (and is the smallest such e).
__host__ __device__ __forceinline__ int colscale_exp(uint32_t amax_bits) {
  const int e = static_cast<int>((amax_bits >> 23) & 0xFFu) - 127 - 15;
  return e > 0 ? e : 0;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe (relieves the MUFU): Cody-Waite style range reduction x = n + f, n = round(x), f in
// [-1/2, 1/2], then a degree-3 polynomial fitted here for minimum relative error on that interval (max 7.5e-5,
// far below the f16 rounding of P), and the exponent of the result moved by n with an integer add.  x is clamped at
// -126 first (masked scores are -inf): results below 2^-126 only need to be tiny and non-negative.
__device__ __forceinline__ float ex2_poly(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound has round(x) in its low mantissa bits
  x = fmaxf(x, -126.0f);
  const float j = x + kRound;
  const float f = x - (j - kRound);
  float p = fmaf(0.055170949548482895f, f, 0.2426096349954605f);
  p = fmaf(p, f, 0.6932609677314758f);
  p = fmaf(p, f, 0.9999281764030457f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

// packed fp32 pair arithmetic (one instruction for two lanes of work on sm_100a)
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// ex2_poly on a pair with the packed instructions
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& e0, float& e1) {
  constexpr float kRound = 12582912.0f;
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  float j0, j1, n0, n1, f0, f1, p0, p1;
  fadd2(j0, j1, x0, x1, kRound, kRound);
  fadd2(n0, n1, j0, j1, -kRound, -kRound);
  ffma2(f0, f1, n0, n1, -1.0f, -1.0f, x0, x1);
  ffma2(p0, p1, 0.055170949548482895f, 0.055170949548482895f, f0, f1, 0.2426096349954605f, 0.2426096349954605f);
  ffma2(p0, p1, p0, p1, f0, f1, 0.6932609677314758f, 0.6932609677314758f);
  ffma2(p0, p1, p0, p1, f0, f1, 0.9999281764030457f, 0.9999281764030457f);
  e0 = __int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23));
  e1 = __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23));
}

template <bool F16>
__device__ __forceinline__ uint32_t pack_p(float lo, float hi) {
  if (F16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// POLY = how many of every 8 exponential pairs run on the FMA pipe (ex2_poly2) instead of the MUFU
template <bool F16, int POLY = 0>
__global__ void __launch_bounds__(THREADS, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ Params p) {
  constexpr uint32_t IDESC_QK = idesc_make(FMT_BF16, FMT_BF16, 0, BQ, BKV);
  constexpr uint32_t IDESC_PV = idesc_make(F16 ? FMT_F16 : FMT_BF16, F16 ? FMT_F16 : FMT_BF16, 1, BQ, D);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);                   // 2 tiles
  const uint32_t sK = sQ + 2 * TILE_BYTES;              // KST tiles
  const uint32_t sV = sK + KST * TILE_BYTES;            // VST tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (2 + KST + VST) * TILE_BYTES);
  const uint32_t b0 = smem_u32(bars);
  // q_full | k_full[2] | k_empty[2] | v_full[2] | v_empty[2] | s_full[2] | p_full[2] | o_full[2] | done
  const uint32_t q_full = b0;
  auto k_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return b0 + 8u * (3 + s); };
  auto v_full = [&](int s) { return b0 + 8u * (5 + s); };
  auto v_empty = [&](int s) { return b0 + 8u * (7 + s); };
  auto s_full = [&](int q) { return b0 + 8u * (9 + q); };
  auto p_full = [&](int q) { return b0 + 8u * (11 + q); };
  auto o_full = [&](int q) { return b0 + 8u * (13 + q); };
  const uint32_t done_bar = b0 + 8u * 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 2 * BQ;
  // The range flag was written by an earlier launch on this stream, so every thread reads the same value and the
  // whole CTA leaves together, before it touches barriers or TMEM: a launch that is skipped costs almost nothing.
  if (p.range_flag != nullptr) {
    const bool raised = *reinterpret_cast<const volatile int32_t*>(p.range_flag) != 0;
    if (p.range_mode == 0 && raised) {
      if (threadIdx.x == 0) record_status(p.wc, H3B_ERANGE);
      return;
    }
    if ((p.range_mode == 1 && raised) || (p.range_mode == 2 && !raised)) return;
  }
  const bool aborted_at_entry = status_bad(p.wc);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
      mbar_init(s_full(s), 1);
      mbar_init(p_full(s), 4);  // one arrival per softmax warp (128 per-thread arrivals serialise on the word)
      mbar_init(o_full(s), 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkv = p.nkv;

  if (!aborted_at_entry) {
    if (warp == 8) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d(sQ + t * TILE_BYTES + hf * HALF_BYTES, &tmQ, q_full, hf * 64, static_cast<int32_t>(q0 + t * BQ),
                        head);
        int kn[KST] = {0, 0}, vn[VST] = {0, 0};
        for (int j = 0; j < nkv; ++j) {
          const int ks = j % KST, vs = j % VST;
          const uint32_t kph = static_cast<uint32_t>(j / KST) & 1u, vph = static_cast<uint32_t>(j / VST) & 1u;
          if (!mbar_wait(k_empty(ks), kph ^ 1u, p.wc)) break;
          mbar_arrive_expect_tx(k_full(ks), TILE_BYTES);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d(sK + ks * TILE_BYTES + hf * HALF_BYTES, &tmK, k_full(ks), hf * 64, j * BKV, head);
          kn[ks]++;
          if (!mbar_wait(v_empty(vs), vph ^ 1u, p.wc)) break;
          mbar_arrive_expect_tx(v_full(vs), TILE_BYTES);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d(sV + vs * TILE_BYTES + hf * HALF_BYTES, &tmV, v_full(vs), hf * 64, j * BKV, head);
          vn[vs]++;
        }
        // drain outstanding loads before the CTA can exit
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(q_full, 0) && globaltimer() - t0 < p.wc.timeout) {
        }
        for (int s = 0; s < 2; ++s) {
          if (kn[s] > 0)
            while (!mbar_try_wait(k_full(s), static_cast<uint32_t>(kn[s] - 1) & 1u) && globaltimer() - t0 < p.wc.timeout) {
            }
          if (vn[s] > 0)
            while (!mbar_try_wait(v_full(s), static_cast<uint32_t>(vn[s] - 1) & 1u) && globaltimer() - t0 < p.wc.timeout) {
            }
        }
      }
    } else if (warp == 9) {
      if (lane == 0) {
        // ---------------- MMA issuer ----------------
        bool ok = mbar_wait(q_full, 0, p.wc);
        tc_fence_after();
        auto issue_qk = [&](int q, int ks) {
          const uint32_t d_tmem = tmem + static_cast<uint32_t>(q * BKV);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
            umma_f16_ss(d_tmem, sdesc_sw128(sQ + q * TILE_BYTES + off, 16, 1024),
                        sdesc_sw128(sK + ks * TILE_BYTES + off, 16, 1024), IDESC_QK, kk != 0);
          }
        };
        auto issue_pv = [&](int q, int vs, bool accumulate) {
          const uint32_t d_tmem = tmem + static_cast<uint32_t>(2 * BKV + q * D);
          const uint32_t p_tmem = tmem + static_cast<uint32_t>(q * BKV);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16_ts(d_tmem, p_tmem + 8u * kk, sdesc_sw128(sV + vs * TILE_BYTES + kk * 2048, HALF_BYTES, 1024),
                        IDESC_PV, accumulate || kk != 0);
        };
        for (int j = 0; j < nkv && ok; ++j) {
          const int ks = j % KST;
          if (!mbar_wait(k_full(ks), static_cast<uint32_t>(j / KST) & 1u, p.wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int vprev = (j - 1) % VST;
          for (int q = 0; q < 2 && ok; ++q) {
            if (j > 0) {
              if (!mbar_wait(p_full(q), static_cast<uint32_t>(j - 1) & 1u, p.wc)) {
                ok = false;
                break;
              }
              if (q == 0 && !mbar_wait(v_full(vprev), static_cast<uint32_t>((j - 1) / VST) & 1u, p.wc)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_pv(q, vprev, j > 1);
              if (q == 1) umma_commit(v_empty(vprev));
            }
            issue_qk(q, ks);
            umma_commit(s_full(q));
          }
          if (!ok) break;
          umma_commit(k_empty(ks));
        }
        if (ok) {
          const int j = nkv;
          const int vprev = (j - 1) % VST;
          for (int q = 0; q < 2; ++q) {
            if (!mbar_wait(p_full(q), static_cast<uint32_t>(j - 1) & 1u, p.wc)) break;
            if (q == 0 && !mbar_wait(v_full(vprev), static_cast<uint32_t>((j - 1) / VST) & 1u, p.wc)) break;
            tc_fence_after();
            issue_pv(q, vprev, j > 1);
            umma_commit(o_full(q));
          }
        }
        umma_commit(done_bar);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(done_bar, 0) && globaltimer() - t0 < p.wc.timeout) {
        }
      }
    } else {
      // ---------------- softmax + epilogue (warps 0-7) ----------------
      const int q = warp >> 2;
      const int sub = warp & 3;
      const uint32_t lane_addr = static_cast<uint32_t>(sub * 32) << 16;
      const uint32_t s_tmem = tmem + lane_addr + static_cast<uint32_t>(q * BKV);
      const uint32_t o_tmem = tmem + lane_addr + static_cast<uint32_t>(2 * BKV + q * D);
      const float c = p.scale_log2;
      float m_run = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        if (!mbar_wait(s_full(q), static_cast<uint32_t>(j) & 1u, p.wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[128];
        tmem_ld32_at<0>(s_tmem + 0, s);
        tmem_ld32_at<32>(s_tmem + 32, s);
        tmem_ld32_at<64>(s_tmem + 64, s);
        tmem_ld32_at<96>(s_tmem + 96, s);
        tmem_ld_wait();
        reg_fence(s);
        const int64_t kv_left = p.valid_kv - static_cast<int64_t>(j) * BKV;
        if (kv_left < BKV) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= kv_left) s[i] = __float_as_uint(-INFINITY);
        }
        // row max: 8 independent chains of 3-input max (the softmax warps have no other warps to hide latency)
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]));
#pragma unroll
        for (int i = 16; i < 128; i += 2)
          m8[(i >> 1) & 7] = fmax3(m8[(i >> 1) & 7], __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
        const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        const float m_new = fmaxf(m_run, mx * c);
        const bool need = j > 0 && (m_new - m_run > RESCALE_THRESHOLD);
        if (j == 0) {
          m_run = m_new;
        } else if (__any_sync(0xffffffffu, need)) {
          // rescale this warp's rows of O (warp-collective TMEM access; rows that need none use alpha = 1)
          const float alpha = need ? ex2(m_run - m_new) : 1.0f;
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
#pragma unroll 1
          for (int cc = 0; cc < D; cc += 8) {
            uint32_t o[8];
            tmem_ld8(o_tmem + cc, o);
            tmem_ld_wait();
            asm volatile("" : "+r"(o[0]), "+r"(o[1]), "+r"(o[2]), "+r"(o[3]), "+r"(o[4]), "+r"(o[5]), "+r"(o[6]), "+r"(o[7]));
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st8(o_tmem + cc, o);
          }
          tmem_st_wait();
        }
        const float neg_m = -m_run;
        float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // P (16-bit pairs) goes to columns [0, 64) of S_q: chunk cc covers keys [32cc, 32cc+32) -> columns
        // [16cc, 16cc+16), all of which were read into registers above
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1, e0, e1;
            ffma2(x0, x1, __uint_as_float(s[32 * cc + 2 * i]), __uint_as_float(s[32 * cc + 2 * i + 1]), c, c, neg_m,
                  neg_m);
            if ((i & 7) >= 8 - POLY) {
              ex2_poly2(x0, x1, e0, e1);
            } else {
              e0 = ex2(x0);
              e1 = ex2(x1);
            }
            s[32 * cc + 2 * i] = __float_as_uint(e0);  // kept for the row sum, taken after P is handed over
            s[32 * cc + 2 * i + 1] = __float_as_uint(e1);
            pk[i] = pack_p<F16>(e0, e1);
          }
          tmem_st16(s_tmem + 16 * cc, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(q));
        // the row sum is off the MMA warp's critical path: same pairs, same order as summing during the exponentials
#pragma unroll
        for (int i = 0; i < 128; i += 2) {
          const int a = i & 7;
          fadd2(l8[a], l8[a + 1], l8[a], l8[a + 1], __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
        }
        l_run += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
      }
      if (ok && mbar_wait(o_full(q), 0, p.wc)) {
        tc_fence_after();
        const int64_t row = q0 + q * BQ + sub * 32 + lane;
        const float inv_l = 1.0f / l_run;
        uint16_t* orow = p.o + row * p.o_tok + static_cast<int64_t>(head) * p.o_head;
        // peer stores: this warp's 32 output rows are staged in the (now idle) K tiles and leave as 2 rows x 256 B per
        // store instruction; every QK^T MMA completed before o_full, so nothing reads K any more
        uint4* srow = reinterpret_cast<uint4*>(smem + 2 * TILE_BYTES) + (warp * 32 + lane) * 16;
#pragma unroll
        for (int cc = 0; cc < D; cc += 32) {
          uint32_t o[32];
          tmem_ld32(o_tmem + cc, o);
          tmem_ld_wait();
          reg_fence(o);
          // per-column factor: 1 / l, times 2^e on the scaled fallback (a power of two: the product is exact)
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = inv_l;
          if (p.colmax != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              f[i] = inv_l * __int_as_float((127 + colscale_exp(__ldg(p.colmax + head * D + cc + i))) << 23);
          }
          if (p.m_rows > 0) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 8 * v + 2 * e;
                __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(o[i]) * f[i], __uint_as_float(o[i + 1]) * f[i + 1]);
                w[e] = *reinterpret_cast<uint32_t*>(&b);
              }
              srow[((cc >> 3) + v) ^ (lane & 15)] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else if (row < p.s_q) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 8 * v + 2 * e;
                __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(o[i]) * f[i], __uint_as_float(o[i + 1]) * f[i + 1]);
                w[e] = *reinterpret_cast<uint32_t*>(&b);
              }
              *reinterpret_cast<uint4*>(orow + cc + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
        if (p.m_rows > 0) {  // Ulysses reverse exchange: row t goes to rank t / m_rows, slot `rank` there
          __syncwarp();
          const int64_t r0 = q0 + q * BQ + sub * 32;
          const uint4* wst = reinterpret_cast<const uint4*>(smem + 2 * TILE_BYTES) + warp * 32 * 16;
#pragma unroll 4
          for (int it = 0; it < 16; ++it) {
            const int idx = it * 32 + lane, r = idx >> 4, part = idx & 15;
            const int64_t t = r0 + r;
            if (t < p.s_q) {
              const int64_t owner = t / p.m_rows;
              uint16_t* dst = p.peer_o[owner < H3B_MAX_RANKS ? owner : 0] +
                              (p.rank * p.m_rows + (t - owner * p.m_rows)) * p.o_tok +
                              static_cast<int64_t>(head) * p.o_head + part * 8;
              *reinterpret_cast<uint4*>(dst) = wst[r * 16 + (part ^ (r & 15))];
            }
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}


// ------------------------------------------------------------------------------------------------------------------
// The CTA-pair kernel.  A cluster of two CTAs on two SMs computes 256 query rows of one head: CTA r holds rows
// [128 r, 128 r + 128) of Q, keys [64 r, 64 r + 64) of each 128-key K tile and columns [64 r, 64 r + 64) of each V tile
// in its shared memory (every tile is loaded once for the pair, no multicast), and its 128 rows of S, O and P in its
// TMEM.  The even CTA's single MMA thread issues 2-SM MMAs (tcgen05.mma.cta_group::2, M = 256): S = Q K^T (N = 128
// keys) and O += P V (N = 128 = d, P from TMEM).  Per CTA, TMEM columns: S0 | S1 | O | P0 | P1 (128, 128, 128, 64,
// 64).  S is double buffered and P has columns of its own, so the MMA for S(j+1) runs while the softmax of step j
// does; each step the tensor pipe does S(j+2) and P(j) V(j).
//   warps 0-7 : softmax + epilogue.  Warp w serves TMEM lanes [32 (w % 4), +32) (query rows) and the key / O column
//               half w / 4: every thread reads its row's 128 scores (the row maximum needs all of them) and
//               exponentiates its 64, so the two halves never wait for each other during the key loop.  Their
//               partial row sums are added once, at the end.
//   warp 8    : TMA producer of this CTA's tiles; every load completes on the even CTA's barrier, armed with the
//               pair's bytes by the even CTA's producer
//   warp 9    : TMEM allocator of the pair; in the even CTA the MMA issuer, whose commits arrive on both CTAs'
//               barriers (one multicast commit per event)
// The handoffs into the even CTA's barriers from the odd CTA's softmax warps are relaxed cluster arrivals (tensor
// memory is ordered by tcgen05.wait and the tcgen05 fences): a release at cluster scope stalls a warp ~1,000 cycles.
// Every wait is bounded; the two CTAs leave together (cluster barrier) after all MMAs completed.
namespace pair {
constexpr int QROWS = 128;                     // query rows per CTA
constexpr int KH = 64;                         // keys of each 128-key tile per CTA
constexpr int Q_BYTES = QROWS * D * 2;         // 32 KB
constexpr int Q_HALF = Q_BYTES / 2;            // 64 of the 128 dims of the 128 rows (one 128-byte swizzle column)
constexpr int K_BYTES = KH * D * 2;            // 16 KB
constexpr int K_HALF = K_BYTES / 2;
constexpr int V_BYTES = BKV * 64 * 2;          // 16 KB: 128 keys x this CTA's 64 columns
constexpr int STAGE_BYTES = K_BYTES + V_BYTES; // stage n: K tile n and V tile n - 2 (what the MMAs of step n read)
constexpr int STAGES = 5;
constexpr int THREADS = 320;
constexpr int STAGE_AREA = Q_BYTES + STAGES * STAGE_BYTES;
constexpr int NBARS = 1 + 2 * STAGES + 2 + 2 + 2 + 2 + 2;   // q, full/empty per stage, s_full, p_full, pv_done,
                                                            // s_free, done + l_ready
constexpr int SMEM_BYTES = STAGE_AREA + 1024 + 256 + 2 * QROWS * 4;
constexpr uint32_t S_COL0 = 0, O_COL = 256, P_COL0 = 384;  // S buffer b at 128 b, P buffer b at 384 + 64 b
static_assert(8 * (NBARS + 1) <= 256, "barrier area");
static_assert(SMEM_BYTES <= 232448, "shared memory");
}  // namespace pair

// exp2(s * c - m) of the 64 scores s[OFF, OFF + 64) as 32 packed 16-bit pairs, their sum added into l8
template <bool F16, int POLY, int OFF>
__device__ __forceinline__ void exp_half(const uint32_t (&s)[128], float c, float neg_m, float (&l8)[8],
                                         uint32_t (&pk)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float x0, x1, e0, e1;
    ffma2(x0, x1, __uint_as_float(s[OFF + 2 * i]), __uint_as_float(s[OFF + 2 * i + 1]), c, c, neg_m, neg_m);
    if ((i & 7) >= 8 - POLY) {
      ex2_poly2(x0, x1, e0, e1);
    } else {
      e0 = ex2(x0);
      e1 = ex2(x1);
    }
    const int a = (2 * i) & 7;
    fadd2(l8[a], l8[a + 1], l8[a], l8[a + 1], e0, e1);
    pk[i] = pack_p<F16>(e0, e1);
  }
}

template <bool F16, int POLY = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::THREADS, 1)
    flash_attn_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ Params p) {
  using namespace pair;
  constexpr uint32_t IDESC_QK = idesc_make(FMT_BF16, FMT_BF16, 0, 2 * QROWS, BKV);
  constexpr uint32_t IDESC_PV = idesc_make(F16 ? FMT_F16 : FMT_BF16, F16 ? FMT_F16 : FMT_BF16, 1, 2 * QROWS, D);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sS = sQ + Q_BYTES;  // stage n % STAGES: K half (K_BYTES), then V half (V_BYTES)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGE_AREA);
  const uint32_t b0 = smem_u32(bars);
  // q_full | full[STAGES] | empty[STAGES] | s_full[2] | p_full[2] | pv_done[2] | s_free[2] | done | l_ready
  const uint32_t q_full = b0;
  auto st_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto st_empty = [&](int s) { return b0 + 8u * (1 + STAGES + s); };
  auto s_full = [&](int b) { return b0 + 8u * (1 + 2 * STAGES + b); };
  auto p_full = [&](int b) { return b0 + 8u * (3 + 2 * STAGES + b); };
  auto pv_done = [&](int b) { return b0 + 8u * (5 + 2 * STAGES + b); };
  auto s_free = [&](int b) { return b0 + 8u * (7 + 2 * STAGES + b); };
  const uint32_t done_bar = b0 + 8u * (9 + 2 * STAGES);
  const uint32_t l_ready = b0 + 8u * (10 + 2 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  float* lred = reinterpret_cast<float*>(smem + STAGE_AREA + 256);  // [2][QROWS] partial row sums of the two halves

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();  // 0: the pair's leader (issues the MMAs)
  const int head = blockIdx.y;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x >> 1) * 2 * QROWS + crank * QROWS;  // this CTA's first row
  // the range flag comes from an earlier launch: every CTA of the grid reads the same value and leaves together
  if (p.range_flag != nullptr) {
    const bool raised = *reinterpret_cast<const volatile int32_t*>(p.range_flag) != 0;
    if (p.range_mode == 0 && raised) {
      if (threadIdx.x == 0) record_status(p.wc, H3B_ERANGE);
      return;
    }
    if ((p.range_mode == 1 && raised) || (p.range_mode == 2 && !raised)) return;
  }
  const bool aborted_at_entry = status_bad(p.wc);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(st_full(s), 1);
      mbar_init(st_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(p_full(b), 16);  // one arrival per softmax warp of both CTAs (counted on the leader's)
      mbar_init(s_free(b), 16);  // likewise, once the warp has read its scores
      mbar_init(pv_done(b), 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(l_ready, 8);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkv = p.nkv;
  const int nsteps = nkv + 2;  // stage n carries K(n) (n < nkv) and V(n - 2) (n >= 2)

  if (!aborted_at_entry) {
    if (warp == 8) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        const uint32_t lead_b0 = mapa_shared(b0, 0);
        auto lead = [&](uint32_t bar) { return bar - b0 + lead_b0; };
        if (crank == 0) mbar_arrive_expect_tx(q_full, 2 * Q_BYTES);
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d_pair(sQ + hf * Q_HALF, &tmQ, lead(q_full), hf * 64, static_cast<int32_t>(q0), head);
        int issued[STAGES];
        for (int s = 0; s < STAGES; ++s) issued[s] = 0;
        for (int n = 0; n < nsteps; ++n) {
          const int st = n % STAGES;
          if (!mbar_wait(st_empty(st), (static_cast<uint32_t>(n / STAGES) & 1u) ^ 1u, p.wc)) break;
          const bool k_now = n < nkv, v_now = n >= 2;
          if (crank == 0) mbar_arrive_expect_tx(st_full(st), 2u * ((k_now ? K_BYTES : 0) + (v_now ? V_BYTES : 0)));
          const uint32_t base = sS + st * STAGE_BYTES;
          if (k_now)
            for (int hf = 0; hf < 2; ++hf)
              tma_load_3d_pair(base + hf * K_HALF, &tmK, lead(st_full(st)), hf * 64,
                               n * BKV + static_cast<int>(crank) * KH, head);
          if (v_now)
            tma_load_3d_pair(base + K_BYTES, &tmV, lead(st_full(st)), static_cast<int>(crank) * 64, (n - 2) * BKV,
                             head);
          issued[st]++;
        }
        // drain: no TMA write may be in flight into shared memory the CTA is about to release.  The leader sees the
        // pair's bytes on its full barriers; the partner's loads of a stage have landed once the MMAs that read
        // them completed (its empty barriers), and its Q once the first S MMA did (stage 0's empty barrier)
        const uint64_t t0 = globaltimer();
        if (crank == 0)
          while (!mbar_try_wait(q_full, 0) && globaltimer() - t0 < p.wc.timeout) {
          }
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0) {
            const uint32_t bar = crank == 0 ? st_full(s) : st_empty(s);
            while (!mbar_try_wait(bar, static_cast<uint32_t>(issued[s] - 1) & 1u) && globaltimer() - t0 < p.wc.timeout) {
            }
          }
      }
    } else if (warp == 9) {
      if (lane == 0 && crank == 0) {
        // ---------------- MMA issuer (the leader only) ----------------
        // Step n: S(n) = Q K(n)^T into S buffer n & 1 (once every softmax warp has read S(n - 2) out of it), then
        // O += P(n - 2) V(n - 2) (once the softmax of step n - 2 wrote P).  So S(n) is computed while the softmax of
        // step n - 1 runs.  Each completion event is one multicast commit that arrives on the barrier of both CTAs.
        constexpr uint16_t kBoth = 3;
        bool ok = mbar_wait(q_full, 0, p.wc);
        tc_fence_after();
        for (int n = 0; n < nsteps && ok; ++n) {
          const int st = n % STAGES;
          const uint32_t base = sS + st * STAGE_BYTES;
          if (!mbar_wait(st_full(st), static_cast<uint32_t>(n / STAGES) & 1u, p.wc)) {
            ok = false;
            break;
          }
          if (n < nkv) {
            if (n >= 2 && !mbar_wait(s_free(n & 1), static_cast<uint32_t>((n - 2) >> 1) & 1u, p.wc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem + S_COL0 + 128u * static_cast<uint32_t>(n & 1);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t cq = (kk >> 2) * Q_HALF + (kk & 3) * 32, ck = (kk >> 2) * K_HALF + (kk & 3) * 32;
              umma_f16_ss_pair(d, sdesc_sw128(sQ + cq, 16, 1024), sdesc_sw128(base + ck, 16, 1024), IDESC_QK, kk != 0);
            }
            umma_commit_pair_mc(s_full(n & 1), kBoth);
          }
          if (n >= 2) {
            const int j = n - 2;
            if (!mbar_wait(p_full(j & 1), static_cast<uint32_t>(j >> 1) & 1u, p.wc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a = tmem + P_COL0 + 64u * static_cast<uint32_t>(j & 1);
#pragma unroll
            for (int kk = 0; kk < BKV / 16; ++kk)
              umma_f16_ts_pair(tmem + O_COL, a + 8u * kk, sdesc_sw128(base + K_BYTES + kk * 2048, V_BYTES, 1024),
                               IDESC_PV, j > 0 || kk != 0);
            umma_commit_pair_mc(pv_done(j & 1), kBoth);
          }
          umma_commit_pair_mc(st_empty(st), kBoth);  // K(n) and V(n - 2) are read once these MMAs complete
        }
        // every issued MMA completes before the pair's TMEM is released
        umma_commit_pair(done_bar);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(done_bar, 0) && globaltimer() - t0 < p.wc.timeout) {
        }
      }
    } else {
      // ---------------- softmax + epilogue (warps 0-7) ----------------
      const int g = warp >> 2;    // key / O column half
      const int sub = warp & 3;   // TMEM lanes [32 sub, 32 sub + 32)
      const int row = sub * 32 + lane;
      const uint32_t lane_addr = static_cast<uint32_t>(sub * 32) << 16;
      const uint32_t o_tmem = tmem + lane_addr + O_COL + 64u * static_cast<uint32_t>(g);
      const uint32_t lead_b0 = mapa_shared(b0, 0);
      const float c = p.scale_log2;
      float m_run = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const int b = j & 1;
        if (!mbar_wait(s_full(b), static_cast<uint32_t>(j >> 1) & 1u, p.wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[128];
        const uint32_t s_tmem = tmem + lane_addr + S_COL0 + 128u * static_cast<uint32_t>(b);
        tmem_ld32_at<0>(s_tmem + 0, s);
        tmem_ld32_at<32>(s_tmem + 32, s);
        tmem_ld32_at<64>(s_tmem + 64, s);
        tmem_ld32_at<96>(s_tmem + 96, s);
        tmem_ld_wait();
        reg_fence(s);
        // the scores are in registers: S buffer b may take S(j + 2)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(s_free(b) - b0 + lead_b0);
        const int64_t kv_left = p.valid_kv - static_cast<int64_t>(j) * BKV;
        if (kv_left < BKV) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= kv_left) s[i] = __float_as_uint(-INFINITY);
        }
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]));
#pragma unroll
        for (int i = 16; i < 128; i += 2)
          m8[(i >> 1) & 7] = fmax3(m8[(i >> 1) & 7], __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
        const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        const float m_new = fmaxf(m_run, mx * c);
        const bool need = j > 0 && (m_new - m_run > RESCALE_THRESHOLD);
        if (j == 0) {
          m_run = m_new;
        } else if (__any_sync(0xffffffffu, need)) {
          // O holds P(j-1) V(j-1) once that MMA completed; rescale this warp's rows of this half
          if (!mbar_wait(pv_done((j - 1) & 1), static_cast<uint32_t>((j - 1) >> 1) & 1u, p.wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = need ? ex2(m_run - m_new) : 1.0f;
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
#pragma unroll 1
          for (int cc = 0; cc < 64; cc += 8) {
            uint32_t o[8];
            tmem_ld8(o_tmem + cc, o);
            tmem_ld_wait();
            asm volatile("" : "+r"(o[0]), "+r"(o[1]), "+r"(o[2]), "+r"(o[3]), "+r"(o[4]), "+r"(o[5]), "+r"(o[6]), "+r"(o[7]));
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st8(o_tmem + cc, o);
          }
          tmem_st_wait();
        }
        // P buffer b is free again once P(j-2) V(j-2) completed
        if (j >= 2) {
          if (!mbar_wait(pv_done(b), static_cast<uint32_t>((j - 2) >> 1) & 1u, p.wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t pk[32];
        if (g == 0)   // the half is warp-uniform; the register indices stay compile-time constants
          exp_half<F16, POLY, 0>(s, c, -m_run, l8, pk);
        else
          exp_half<F16, POLY, 64>(s, c, -m_run, l8, pk);
        // keys [64 g, 64 g + 64) of the tile as 16-bit pairs: P columns [32 g, 32 g + 32)
        tmem_st32(tmem + lane_addr + P_COL0 + 64u * static_cast<uint32_t>(b) + 32u * static_cast<uint32_t>(g), pk);
        l_run += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(p_full(b) - b0 + lead_b0);
      }
      const int jl = nkv - 1;
      if (ok && mbar_wait(pv_done(jl & 1), static_cast<uint32_t>(jl >> 1) & 1u, p.wc)) {
        tc_fence_after();
        // the row's sum: the two halves' partial sums, added in the same order by both
        lred[g * QROWS + row] = l_run;
        __syncwarp();
        if (lane == 0) mbar_arrive(l_ready);
        if (mbar_wait(l_ready, 0, p.wc)) {
          const float inv_l = 1.0f / (lred[row] + lred[QROWS + row]);
          const int64_t t = q0 + row;
          uint16_t* orow = p.o + t * p.o_tok + static_cast<int64_t>(head) * p.o_head + 64 * g;
          // peer stores: the warp's 32 rows x 128 B are staged in the stage area (every load was consumed by MMAs
          // that completed before the last pv_done) and leave as 4 rows per store instruction
          uint4* stg = reinterpret_cast<uint4*>(smem + Q_BYTES) + warp * 32 * 8;
#pragma unroll
          for (int cc = 0; cc < 64; cc += 32) {
            uint32_t o[32];
            tmem_ld32(o_tmem + cc, o);
            tmem_ld_wait();
            reg_fence(o);
            float f[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = inv_l;
            if (p.colmax != nullptr) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                f[i] = inv_l * __int_as_float((127 + colscale_exp(__ldg(p.colmax + head * D + 64 * g + cc + i))) << 23);
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 8 * v + 2 * e;
                __nv_bfloat162 bb = __floats2bfloat162_rn(__uint_as_float(o[i]) * f[i], __uint_as_float(o[i + 1]) * f[i + 1]);
                w[e] = *reinterpret_cast<uint32_t*>(&bb);
              }
              const uint4 val = make_uint4(w[0], w[1], w[2], w[3]);
              const int gi = (cc >> 3) + v;  // 16-byte granule of the row's 128 bytes
              if (p.m_rows > 0)
                stg[lane * 8 + (gi ^ (lane & 7))] = val;
              else if (t < p.s_q)
                *reinterpret_cast<uint4*>(orow + 8 * gi) = val;
            }
          }
          if (p.m_rows > 0) {  // Ulysses reverse exchange: row t goes to rank t / m_rows, slot `rank` there
            __syncwarp();
            const int64_t r0 = q0 + sub * 32;
#pragma unroll 4
            for (int it = 0; it < 8; ++it) {
              const int idx = it * 32 + lane, r = idx >> 3, part = idx & 7;
              const int64_t tt = r0 + r;
              if (tt < p.s_q) {
                const int64_t owner = tt / p.m_rows;
                uint16_t* dst = p.peer_o[owner < H3B_MAX_RANKS ? owner : 0] +
                                (p.rank * p.m_rows + (tt - owner * p.m_rows)) * p.o_tok +
                                static_cast<int64_t>(head) * p.o_head + 64 * g + part * 8;
                *reinterpret_cast<uint4*>(dst) = stg[r * 8 + (part ^ (r & 7))];
              }
            }
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves (or frees the pair's TMEM) while the other may still signal it
  tc_fence_after();
  if (warp == 9) tmem_dealloc_pair(tmem, 512);
}

}  // namespace attn
}  // namespace h3b

using namespace h3b;

static int make_qkv_map(CUtensorMap* m, const void* base, int64_t tokens, int heads, int64_t tok_stride,
                        int64_t head_stride, uint32_t box_rows) {
  const uint64_t dims[3] = {128, static_cast<uint64_t>(tokens), static_cast<uint64_t>(heads)};
  const uint64_t strides[2] = {static_cast<uint64_t>(tok_stride) * 2, static_cast<uint64_t>(head_stride) * 2};
  const uint32_t box[3] = {64, box_rows, 1};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// How many of every 8 softmax exponential pairs run on the FMA pipe: kDefaultPoly, or H3B_ATTN_EXP2_POLY in
// {0, 2, 3, 4} (a tuning switch; every setting computes the same softmax within the kernel's tolerance)
static int poly_pairs() {
  static const int n = [] {
    const char* v = getenv("H3B_ATTN_EXP2_POLY");
    if (v == nullptr || v[0] == '\0') return h3b::attn::kDefaultPoly;
    const int x = atoi(v);
    return (x == 0 || x == 2 || x == 3 || x == 4) ? x : h3b::attn::kDefaultPoly;
  }();
  return n;
}

template <typename K>
static cudaError_t set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Which attention kernel runs: the one-CTA kernel (default) or the CTA-pair kernel (H3B_ATTN_PAIR=1; both compute
// the same softmax within the kernels' tolerance)
static bool use_pair() {
  static const bool on = [] {
    const char* v = getenv("H3B_ATTN_PAIR");
    return v != nullptr && v[0] != '\0' && atoi(v) != 0;
  }();
  return on;
}

// once per device: the shared-memory opt-in of every kernel variant (first calls from several threads serialise
// on the mutex; a device is marked done only after every attribute was set)
static int attn_attrs() {
  using namespace h3b::attn;
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "flash_attn: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(H3B_EUNSUPPORTED, "flash_attn: device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return H3B_OK;
  e = set_smem(flash_attn_kernel<true, 0>, SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_kernel<true, 2>, SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_kernel<true, 3>, SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_kernel<true, 4>, SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_kernel<false, kDefaultPoly>, SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_pair_kernel<true, 0>, pair::SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_pair_kernel<true, 2>, pair::SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_pair_kernel<true, 3>, pair::SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_pair_kernel<true, 4>, pair::SMEM_BYTES);
  if (e == cudaSuccess) e = set_smem(flash_attn_pair_kernel<false, kDefaultPoly>, pair::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "flash_attn: smem attribute");
  done[dev] = true;
  return H3B_OK;
}

// Builds the tensor maps and launches one attention kernel.  p carries everything but nkv.
static int launch_attention(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                            int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, bool v_f16,
                            h3b::attn::Params p, cudaStream_t st) {
  using namespace h3b::attn;
  int rc = attn_attrs();
  if (rc) return rc;
  CUtensorMap tq, tk, tv;
  // K and V maps end at valid_kv: the last key tile's rows beyond it come from the TMA's zero fill, never from
  // memory (padding rows may hold anything, even values whose product with a zero P would not be zero)
  rc = make_qkv_map(&tq, q, p.s_q, p.heads, q_tok, q_head, BQ);
  const bool pr = use_pair();
  if (!rc) rc = make_qkv_map(&tk, k, p.valid_kv, p.heads, k_tok, k_head, pr ? pair::KH : BKV);
  if (!rc) rc = make_qkv_map(&tv, v, p.valid_kv, p.heads, v_tok, v_head, BKV);
  if (rc) return rc;
  p.nkv = static_cast<int>((p.valid_kv + BKV - 1) / BKV);
  const int poly = poly_pairs();
  if (pr) {  // clusters of two CTAs over 256-row query tiles
    dim3 grid(2 * static_cast<unsigned>((p.s_q + 2 * pair::QROWS - 1) / (2 * pair::QROWS)),
              static_cast<unsigned>(p.heads));
    const int sm = pair::SMEM_BYTES;
    if (!v_f16)
      flash_attn_pair_kernel<false, kDefaultPoly><<<grid, pair::THREADS, sm, st>>>(tq, tk, tv, p);
    else if (poly == 0)
      flash_attn_pair_kernel<true, 0><<<grid, pair::THREADS, sm, st>>>(tq, tk, tv, p);
    else if (poly == 2)
      flash_attn_pair_kernel<true, 2><<<grid, pair::THREADS, sm, st>>>(tq, tk, tv, p);
    else if (poly == 3)
      flash_attn_pair_kernel<true, 3><<<grid, pair::THREADS, sm, st>>>(tq, tk, tv, p);
    else
      flash_attn_pair_kernel<true, 4><<<grid, pair::THREADS, sm, st>>>(tq, tk, tv, p);
    H3B_CHECK_LAUNCH("flash_attn launch");
    return H3B_OK;
  }
  dim3 grid(static_cast<unsigned>((p.s_q + 2 * BQ - 1) / (2 * BQ)), static_cast<unsigned>(p.heads));
  if (!v_f16)
    flash_attn_kernel<false, kDefaultPoly><<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
  else if (poly == 0)
    flash_attn_kernel<true, 0><<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
  else if (poly == 2)
    flash_attn_kernel<true, 2><<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
  else if (poly == 3)
    flash_attn_kernel<true, 3><<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
  else
    flash_attn_kernel<true, 4><<<grid, THREADS, SMEM_BYTES, st>>>(tq, tk, tv, p);
  H3B_CHECK_LAUNCH("flash_attn launch");
  return H3B_OK;
}

namespace h3b {
namespace attn {

// v [rows, heads, 128] bf16 (token stride v_tok, head stride v_head) -> out [rows, heads, 128] f16 contiguous;
// *flag = 1 when a finite value overflows f16.  Only the rows the attention reads are converted (rows = valid_kv),
// so padding rows beyond them can hold anything.
__global__ void v_to_f16_kernel(const uint16_t* __restrict__ v, int64_t rows, int heads, int64_t v_tok,
                                int64_t v_head, uint16_t* __restrict__ out, int32_t* flag) {
  const int64_t total = rows * heads * 16;  // 16-byte granules of 8 elements
  bool bad = false;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t & 15, th = t >> 4;
    const int64_t h = th % heads, tok = th / heads;
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(v + tok * v_tok + h * v_head) + c);
    uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = __uint_as_float(w[i] << 16), b = __uint_as_float(w[i] & 0xFFFF0000u);
      bad |= (fabsf(a) > 65504.0f && isfinite(a)) || (fabsf(b) > 65504.0f && isfinite(b));
      __half2 hv = __floats2half2_rn(a, b);
      w[i] = *reinterpret_cast<uint32_t*>(&hv);
    }
    reinterpret_cast<uint4*>(out)[t] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicExch(flag, 1);
}

// Only when *flag is set (a v beyond f16's range): colmax[h * 128 + c] = bits of max |v[t, h, c]| over the finite
// values of rows t < rows (non-negative floats order as their bits).  Grid (x, heads), 256 threads: thread i keeps
// the maxima of the 8 columns of granule i % 16 over its tokens, the CTA merges them in shared memory and adds them
// to the global maxima with one atomic per column.
__global__ void v_colmax_kernel(const uint16_t* __restrict__ v, int64_t rows, int64_t v_tok, int64_t v_head,
                                const int32_t* flag, uint32_t* colmax) {
  if (*reinterpret_cast<const volatile int32_t*>(flag) == 0) return;
  __shared__ uint32_t cm[D];
  if (threadIdx.x < D) cm[threadIdx.x] = 0;
  __syncthreads();
  const int h = blockIdx.y, c = threadIdx.x & 15;
  uint32_t m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t tok = blockIdx.x * static_cast<int64_t>(blockDim.x / 16) + (threadIdx.x >> 4); tok < rows;
       tok += static_cast<int64_t>(gridDim.x) * (blockDim.x / 16)) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(v + tok * v_tok + h * v_head) + c);
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = (w[i] << 16) & 0x7FFFFFFFu, b = w[i] & 0x7FFF0000u;
      if (a < 0x7F800000u) m[2 * i] = max(m[2 * i], a);  // finite magnitudes only
      if (b < 0x7F800000u) m[2 * i + 1] = max(m[2 * i + 1], b);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) atomicMax(&cm[c * 8 + i], m[i]);
  __syncthreads();
  if (threadIdx.x < D) atomicMax(colmax + h * D + threadIdx.x, cm[threadIdx.x]);
}

// Only when *flag is set: out[t, h, c] = f16(v[t, h, c] * 2^-e), e = colscale_exp(colmax[h * 128 + c]); every
// finite value then fits f16, and the power-of-two scale is exact (the attention multiplies the output column back).
__global__ void v_to_f16_scaled_kernel(const uint16_t* __restrict__ v, int64_t rows, int heads, int64_t v_tok,
                                       int64_t v_head, uint16_t* __restrict__ out, const int32_t* flag,
                                       const uint32_t* __restrict__ colmax) {
  if (*reinterpret_cast<const volatile int32_t*>(flag) == 0) return;
  const int64_t total = rows * heads * 16;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t & 15, th = t >> 4;
    const int64_t h = th % heads, tok = th / heads;
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(v + tok * v_tok + h * v_head) + c);
    uint32_t w[4] = {x.x, x.y, x.z, x.w};
    const uint32_t* cmx = colmax + h * D + c * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float sa = __int_as_float((127 - colscale_exp(__ldg(cmx + 2 * i))) << 23);
      const float sb = __int_as_float((127 - colscale_exp(__ldg(cmx + 2 * i + 1))) << 23);
      __half2 hv = __floats2half2_rn(__uint_as_float(w[i] << 16) * sa, __uint_as_float(w[i] & 0xFFFF0000u) * sb);
      w[i] = *reinterpret_cast<uint32_t*>(&hv);
    }
    reinterpret_cast<uint4*>(out)[t] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace attn
}  // namespace h3b

// The attention of a bf16 v of any range, decided on the device (no host read).  ctl (H3B_ATTN_CTL_BYTES(heads),
// 16-byte aligned): int32 range flag at byte 0, bytes 4-15 untouched, colmax [heads * 128] uint32 from byte 16.
//   1. clear the flag and colmax; convert the valid rows of v to f16 into v16 (flag = 1 on a finite overflow)
//   2. the f16 P.V kernel, unless the flag is set                                   (the path of every v that fits)
//   3. only if the flag is set: colmax, then v16 = f16(v * 2^-e) per (head, column)
//   4. only if the flag is set: the f16 P.V kernel on that v16, the output columns multiplied by 2^e
// Launches whose condition does not hold leave at once.  p carries everything but the range fields and nkv; p.wc says
// where a wait failure is recorded.
static int attention_bf16v(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok, int64_t k_head,
                           const void* v, int64_t v_tok, int64_t v_head, void* v16, void* ctl, h3b::attn::Params p,
                           cudaStream_t st) {
  using namespace h3b::attn;
  int32_t* flag = static_cast<int32_t*>(ctl);
  uint32_t* colmax = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(ctl) + 16);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(colmax, 0, static_cast<size_t>(p.heads) * D * sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "flash_attn: clearing the range flag");
  const int64_t granules = p.valid_kv * p.heads * 16;
  int64_t blocks = (granules + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  const uint16_t* v_in = static_cast<const uint16_t*>(v);
  uint16_t* v_out = static_cast<uint16_t*>(v16);
  v_to_f16_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(v_in, p.valid_kv, p.heads, v_tok, v_head, v_out, flag);
  H3B_CHECK_LAUNCH("flash_attn: v conversion launch");
  p.range_flag = flag;
  p.range_mode = 1;  // f16 P.V unless v overflowed f16
  int rc = launch_attention(q, q_tok, q_head, k, k_tok, k_head, v16, static_cast<int64_t>(p.heads) * 128, 128, true,
                            p, st);
  if (rc) return rc;
  // the scaled fallback: every launch below reads the flag first and leaves when v fitted
  int64_t gx = (static_cast<int64_t>(num_sms()) * 4 + p.heads - 1) / p.heads;
  const int64_t gx_max = (p.valid_kv + 15) / 16;
  if (gx > gx_max) gx = gx_max;
  if (gx > 65535) gx = 65535;
  v_colmax_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(p.heads)), 256, 0, st>>>(
      v_in, p.valid_kv, v_tok, v_head, flag, colmax);
  H3B_CHECK_LAUNCH("flash_attn: v column maxima launch");
  v_to_f16_scaled_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(v_in, p.valid_kv, p.heads, v_tok, v_head, v_out,
                                                                     flag, colmax);
  H3B_CHECK_LAUNCH("flash_attn: scaled v conversion launch");
  p.range_mode = 2;  // only if v overflowed: f16 P.V on the scaled copy
  p.colmax = colmax;
  return launch_attention(q, q_tok, q_head, k, k_tok, k_head, v16, static_cast<int64_t>(p.heads) * 128, 128, true, p,
                          st);
}

// Argument checks shared by the local entry points (ABI names in messages); on success *p holds everything but the
// range fields, nkv and the wait control.
static int local_params(const char* who, const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                        int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o, int64_t o_tok,
                        int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim,
                        float scale, h3b::attn::Params* p) {
  if (s_q < 0 || s_kv <= 0 || heads <= 0)
    return fail(H3B_EINVAL, "%s: s_q %lld s_kv %lld heads %d", who, (long long)s_q, (long long)s_kv, heads);
  if (head_dim != 128) return fail(H3B_EUNSUPPORTED, "%s: head_dim %d (only 128)", who, head_dim);
  if (heads > 65535 || s_q > (1ll << 31) - 1 || s_kv > (1ll << 31) - 1)
    return fail(H3B_EUNSUPPORTED, "%s: size limits (heads <= 65535, s_q and s_kv < 2^31)", who);
  if (valid_kv < 0) valid_kv = s_kv;
  if (valid_kv == 0 || valid_kv > s_kv)
    return fail(H3B_EINVAL, "%s: valid_kv %lld of %lld", who, (long long)valid_kv, (long long)s_kv);
  *p = h3b::attn::Params{};
  p->s_q = s_q;
  p->valid_kv = valid_kv;
  if (s_q == 0) return H3B_OK;  // nothing to compute: the callers return before any launch
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return fail(H3B_EINVAL, "%s: null pointer", who);
  const int64_t strides[8] = {q_tok, q_head, k_tok, k_head, v_tok, v_head, o_tok, o_head};
  for (int64_t st : strides)
    if (st <= 0 || st % 8) return fail(H3B_EALIGN, "%s: token/head strides must be positive multiples of 8", who);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return fail(H3B_EALIGN, "%s: q, k, v, o must be 16-byte aligned", who);
  p->s_kv = s_kv;
  p->heads = heads;
  p->scale_log2 = scale * 1.4426950408889634f;
  p->o = static_cast<uint16_t*>(o);
  p->o_tok = o_tok;
  p->o_head = o_head;
  return H3B_OK;
}

// the same for the peer-memory entry points: output row t of this rank's heads goes to rank t / m_rows
static int p2p_params(const char* who, const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                      int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* const* peer_back,
                      int32_t ws, int32_t rank, int64_t m_rows, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                      int32_t heads, int32_t head_dim, float scale, h3b::attn::Params* p) {
  if (peer_back == nullptr || ws < 1 || ws > H3B_MAX_RANKS || rank < 0 || rank >= ws)
    return fail(H3B_EINVAL, "%s: ws %d rank %d", who, ws, rank);
  if (m_rows <= 0 || s_q != m_rows * ws)
    return fail(H3B_EINVAL, "%s: s_q %lld must be ws * m_rows (%d * %lld)", who, (long long)s_q, ws, (long long)m_rows);
  for (int r = 0; r < ws; ++r)
    if (peer_back[r] == nullptr || (reinterpret_cast<uintptr_t>(peer_back[r]) & 15u))
      return fail(H3B_EALIGN, "%s: peer buffer %d null or not 16-byte aligned", who, r);
  // receive buffers [P, m_rows, heads, 128]: the own buffer stands in for o in the checks
  const int64_t o_tok = static_cast<int64_t>(heads) * 128;
  int rc = local_params(who, q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, peer_back[rank], o_tok, 128, s_q,
                        s_kv, valid_kv, heads, head_dim, scale, p);
  if (rc) return rc;
  for (int r = 0; r < ws; ++r) p->peer_o[r] = static_cast<uint16_t*>(peer_back[r]);
  p->m_rows = m_rows;
  p->rank = rank;
  return H3B_OK;
}

static int library_wait(const char* who, h3b::attn::Params* p) {
  p->wc.status = device_status_word();
  p->wc.timeout = wait_timeout_ns();
  if (p->wc.status == nullptr) return fail(H3B_ECUDA, "%s: device status word", who);
  return H3B_OK;
}

namespace h3b {
namespace attn {

// The bf16-v attention for a caller that brings its own scratch (the allocation-free entry point): the checks of
// h3b_flash_attn_fwd_bf16v, a limit on the f16 copy of v (valid_kv * heads * 128 <= max_v16 elements) and on heads
// (the control words: H3B_NOALLOC_MAX_HEADS), then, unless there is nothing to compute, `scratch` supplies the f16
// buffer, the control words (as attention_bf16v lays them out) and the status word for the waits.
int bf16v_with_scratch(const char* who, const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                       int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o, int64_t o_tok,
                       int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim,
                       float scale, int64_t max_v16, int (*scratch)(void** v16, void** ctl, int** status),
                       cudaStream_t st) {
  Params p;
  // heads <= 65535 and s_kv < 2^31 are checked first, so valid_kv * heads * 128 below cannot wrap
  int rc = local_params(who, q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, o, o_tok, o_head, s_q, s_kv,
                        valid_kv, heads, head_dim, scale, &p);
  if (rc) return rc;
  if (heads > H3B_NOALLOC_MAX_HEADS)
    return fail(H3B_EUNSUPPORTED, "%s: %d heads (at most %d with the fixed scratch); use h3b_flash_attn_fwd_bf16v",
                who, heads, H3B_NOALLOC_MAX_HEADS);
  if (p.valid_kv > max_v16 / (static_cast<int64_t>(heads) * 128))
    return fail(H3B_EUNSUPPORTED,
                "%s: valid_kv * heads * 128 = %lld exceeds the fixed scratch of %lld f16 elements (valid_kv * heads "
                "<= %lld); use h3b_flash_attn_fwd_bf16v",
                who, (long long)(p.valid_kv * heads * 128), (long long)max_v16, (long long)(max_v16 / 128));
  if (s_q == 0) return H3B_OK;
  void* v16 = nullptr;
  void* ctl = nullptr;
  rc = scratch(&v16, &ctl, &p.wc.status);
  if (rc) return rc;
  p.wc.timeout = wait_timeout_ns();
  return attention_bf16v(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, v16, ctl, p, st);
}

}  // namespace attn
}  // namespace h3b

extern "C" int h3b_flash_attn_fwd(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                  int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o, int64_t o_tok,
                                  int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads,
                                  int32_t head_dim, float scale, int32_t v_f16, const int32_t* range_flag,
                                  h3b_stream_t stream) {
  h3b::attn::Params p;
  int rc = local_params("flash_attn", q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, o, o_tok, o_head, s_q,
                        s_kv, valid_kv, heads, head_dim, scale, &p);
  if (!rc) rc = library_wait("flash_attn", &p);
  if (rc || s_q == 0) return rc;
  p.range_flag = v_f16 ? range_flag : nullptr;
  return launch_attention(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, v_f16 != 0, p,
                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_flash_attn_fwd_bf16v(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                        int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o,
                                        int64_t o_tok, int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                        int32_t heads, int32_t head_dim, float scale, void* v16, void* ctl,
                                        h3b_stream_t stream) {
  h3b::attn::Params p;
  int rc = local_params("flash_attn_bf16v", q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, o, o_tok, o_head,
                        s_q, s_kv, valid_kv, heads, head_dim, scale, &p);
  if (!rc) rc = library_wait("flash_attn_bf16v", &p);
  if (rc || s_q == 0) return rc;
  if (v16 == nullptr || ctl == nullptr || ((reinterpret_cast<uintptr_t>(v16) | reinterpret_cast<uintptr_t>(ctl)) & 15u))
    return fail(H3B_EINVAL, "flash_attn_bf16v: v16 and ctl are required, 16-byte aligned");
  return attention_bf16v(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, v16, ctl, p,
                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_flash_attn_fwd_p2p(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                      int64_t k_head, const void* v, int64_t v_tok, int64_t v_head,
                                      void* const* peer_back, int32_t ws, int32_t rank, int64_t m_rows, int64_t s_q,
                                      int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim, float scale,
                                      int32_t v_f16, const int32_t* range_flag, h3b_stream_t stream) {
  h3b::attn::Params p;
  int rc = p2p_params("flash_attn_p2p", q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, peer_back, ws, rank,
                      m_rows, s_q, s_kv, valid_kv, heads, head_dim, scale, &p);
  if (!rc) rc = library_wait("flash_attn_p2p", &p);
  if (rc) return rc;
  p.range_flag = v_f16 ? range_flag : nullptr;
  return launch_attention(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, v_f16 != 0, p,
                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_flash_attn_fwd_p2p_bf16v(const void* q, int64_t q_tok, int64_t q_head, const void* k,
                                            int64_t k_tok, int64_t k_head, const void* v, int64_t v_tok,
                                            int64_t v_head, void* const* peer_back, int32_t ws, int32_t rank,
                                            int64_t m_rows, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                            int32_t heads, int32_t head_dim, float scale, void* v16, void* ctl,
                                            h3b_stream_t stream) {
  h3b::attn::Params p;
  int rc = p2p_params("flash_attn_p2p_bf16v", q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, peer_back, ws,
                      rank, m_rows, s_q, s_kv, valid_kv, heads, head_dim, scale, &p);
  if (!rc) rc = library_wait("flash_attn_p2p_bf16v", &p);
  if (rc) return rc;
  if (v16 == nullptr || ctl == nullptr || ((reinterpret_cast<uintptr_t>(v16) | reinterpret_cast<uintptr_t>(ctl)) & 15u))
    return fail(H3B_EINVAL, "flash_attn_p2p_bf16v: v16 and ctl are required, 16-byte aligned");
  return attention_bf16v(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, v16, ctl, p,
                         reinterpret_cast<cudaStream_t>(stream));
}

