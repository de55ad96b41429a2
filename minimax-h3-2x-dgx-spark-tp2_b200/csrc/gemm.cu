// FP8 (e4m3 x e4m3 -> f32) GEMM on the 5th-generation tensor cores with the per-token x per-channel scaled epilogue
// fused: y = out(sa[m] * (sb[n] * acc)) (bias by fma), the arithmetic of fp8_gemm._scale_bias_cast
// (h3_tp2/fp8_gemm.py:38-54) and of the CuTe-DSL kernel's epilogue (h3_tp2/fp8_cutlass_kernel.py), with no fp32
// product in memory.
//
// Design (one CTA per SM, persistent over output tiles):
//   tile 128 x 256 (M x N), K step 128 (one 128-byte swizzle row of e4m3), 4-stage TMA ring (48 KB per stage).
//   warp 0      : TMA producer (one elected thread), A box 128x128 B and two B boxes 128x128 B per stage
//   warp 1      : TMEM allocator + single-thread tcgen05.mma issuer (kind::f8f6f4, M=128 N=256 K=32)
//   warps 2..5  : epilogue; thread t of the 128 owns accumulator row t (TMEM lane), reads 32-column slices with
//                 tcgen05.ld, applies the scales and stores bf16/f16 (or scatters into the Ulysses send layout, or
//                 applies SwiGLU to the gate/up halves).
//   The accumulator is double buffered in TMEM (2 x 256 of the 512 columns) so the epilogue of tile i overlaps the
//   main loop of tile i+1.  Every wait is bounded (common.cuh).  No TMA multicast, no clusters.
#include "common.cuh"

namespace h3b {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK;   // 16 KB
constexpr int B_BYTES = BN * BK;   // 32 KB (two 128-row boxes)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;
constexpr int EPI_GATE = 3;  // internal epilogue kind of h3b_fp8_gemm_gate
// peer-store staging: per epilogue warp 32 rows x 128 B (64 columns), so the stores to another GPU leave as whole
// 128-byte lines instead of 16-byte pieces of 32 different rows
// (only the PEER instantiation of the kernel has it; the other keeps its registers and shared memory as without)
constexpr int STAGING_BYTES = 4 * 32 * 128;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int SMEM_BYTES_PEER = SMEM_BYTES + STAGING_BYTES;
constexpr uint32_t IDESC = idesc_make(FMT_E4M3, FMT_E4M3, 0, BM, BN);

struct Params {
  int64_t M, N, K;
  int num_mb, num_nb, num_kb;
  const float* sa;
  const float* sb;
  const __nv_bfloat16* bias;
  void* y;
  int64_t ldy;
  int out_f16;
  int epi;
  int64_t half;  // SWIGLU: N / 2
  void* send[3];
  int hd;        // QKV_SEND: heads * 128
  int hl;        // heads per rank and group (hgl)
  int rsh;       // QKV_SEND: heads per send row (hl, or 3 * hl when q, k, v are interleaved)
  int64_t qkv_step;  // QKV_SEND interleaved: elements between the q, k and v slots of a row
  int hg;        // heads per group
  int ws;        // Ulysses degree P
  int v_f16;
  int32_t* range_flag;
  const __nv_bfloat16* norm_w[2];  // q, k RMSNorm weights (nullptr: no norm + RoPE)
  const float* rope;
  int64_t rope_stride;
  int rot;
  float eps;
  const uint16_t* gx;                    // GATE: residual x, gate rows, token -> gate row
  int64_t ldx;
  const uint16_t* gate;
  int64_t ldg, gate_rows;
  const int64_t* gidx;
  int p2p;                               // QKV_SEND into the peers' receive buffers
  int rank;
  void* peer[H3B_MAX_RANKS][3];
  int32_t* peer_rf[H3B_MAX_RANKS];
  WaitCtl wc;
};

// QKV_SEND destination of (which, group g, destination rank): the slab base and its slot index in that buffer
__device__ __forceinline__ uint16_t* send_slab(const Params& p, int which, int g, int dst_rank, int64_t& slot) {
  if (p.p2p) {
    slot = p.rank;  // the peer's receive buffer [P, M, hl, d], indexed by the source rank
    return static_cast<uint16_t*>(p.peer[dst_rank][which]);
  }
  slot = static_cast<int64_t>(g) * p.ws + dst_rank;  // (group, destination) slab of this rank's send buffer
  if (p.qkv_step) return static_cast<uint16_t*>(p.send[0]) + which * p.qkv_step;
  return static_cast<uint16_t*>(p.send[which]);
}

__device__ __forceinline__ float rbf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& mb, int& nb) {
  const int in_group = GROUP_M * p.num_nb;
  const int group = t / in_group;
  const int first = group * GROUP_M;
  const int gsize = min(p.num_mb - first, GROUP_M);
  const int r = t - group * in_group;
  mb = first + r % gsize;
  nb = r / gsize;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, int f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}
// bf16 rounding first, then an exact conversion to f16 (the v slab for the f16 P.V attention)
__device__ __forceinline__ uint32_t pack2_bf16_as_f16(float lo, float hi) {
  const float a = __bfloat162float(__float2bfloat16_rn(lo));
  const float b = __bfloat162float(__float2bfloat16_rn(hi));
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float silu_mul_bf16(float g, float u) {
  g = __bfloat162float(__float2bfloat16_rn(g));
  u = __bfloat162float(__float2bfloat16_rn(u));
  u = (u == 0.0f) ? fabsf(u) : u;
  const float s = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(g, 1.0f + expf(-g))));
  return s * u;
}

// PEER: the QKV_SEND epilogue stores into other GPUs' receive buffers (Params::p2p set)
template <bool PEER>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  uint4* staging = reinterpret_cast<uint4*>(smem + STAGES * STAGE_BYTES + 256);
  const uint32_t smem0 = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool aborted_at_entry = status_bad(p.wc);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 128);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_mb * p.num_nb;
  if (!aborted_at_entry) {
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        int issued[STAGES] = {0, 0, 0, 0};
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
          int mb, nb;
          tile_coords(t, p, mb, nb);
          const int n0 = p.epi == H3B_EPI_SWIGLU ? nb * 128 : nb * BN;
          const int n1 = p.epi == H3B_EPI_SWIGLU ? static_cast<int>(p.half) + nb * 128 : nb * BN + 128;
          for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.wc)) {
              ok = false;
              break;
            }
            const uint32_t sA = smem0 + stage * STAGE_BYTES;
            const uint32_t sB = sA + A_BYTES;
            mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
            tma_load_2d(sA, &tmA, full_bar(stage), kb * BK, mb * BM);
            tma_load_2d(sB, &tmB, full_bar(stage), kb * BK, n0);
            tma_load_2d(sB + 16384, &tmB, full_bar(stage), kb * BK, n1);
            issued[stage]++;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        // drain: never leave a TMA write in flight into shared memory the CTA is about to release
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0) {
            const uint32_t par = static_cast<uint32_t>(issued[s] - 1) & 1u;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(full_bar(s), par) && globaltimer() - t0 < p.wc.timeout) {
            }
          }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ---------------- MMA issuer ----------------
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
          if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.wc)) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
          for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait(full_bar(stage), phase, p.wc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sA = smem0 + stage * STAGE_BYTES;
            const uint32_t sB = sA + A_BYTES;
            const uint64_t adesc = sdesc_sw128(sA, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(sB, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk)
              umma_f8_ss(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, IDESC, (kb | kk) != 0);
            umma_commit(empty_bar(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(tfull_bar(acc));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        // all issued MMAs complete before TMEM is released
        umma_commit(done_bar);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(done_bar, 0) && globaltimer() - t0 < p.wc.timeout) {
        }
      }
    } else {
      // ---------------- epilogue (warps 2..5) ----------------
      const int sub = warp & 3;
      const int row_in_tile = sub * 32 + lane;
      const uint32_t lane_addr = static_cast<uint32_t>(sub * 32) << 16;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        if (!mbar_wait(tfull_bar(acc), acc_phase, p.wc)) break;
        tc_fence_after();
        const int64_t m = static_cast<int64_t>(mb) * BM + row_in_tile;
        const bool row_ok = m < p.M;
        const float sam = row_ok ? __ldg(p.sa + m) : 0.0f;
        const uint32_t tacc = tmem_base + lane_addr + static_cast<uint32_t>(acc * BN);
        if (p.epi == H3B_EPI_SWIGLU) {
          for (int c0 = 0; c0 < 128; c0 += 32) {
            uint32_t g[32], u[32];
            tmem_ld32(tacc + c0, g);
            tmem_ld32(tacc + 128 + c0, u);
            tmem_ld_wait();
            reg_fence(g);
            reg_fence(u);
            const int64_t ng = static_cast<int64_t>(nb) * 128 + c0;  // output / gate column
            const int64_t nu = p.half + ng;                           // up column of W
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float gv[2], uv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float tg = __ldg(p.sb + ng + i + e) * __uint_as_float(g[i + e]);
                const float tu = __ldg(p.sb + nu + i + e) * __uint_as_float(u[i + e]);
                if (p.bias != nullptr) {
                  gv[e] = fmaf(sam, tg, __bfloat162float(p.bias[ng + i + e]));
                  uv[e] = fmaf(sam, tu, __bfloat162float(p.bias[nu + i + e]));
                } else {
                  gv[e] = sam * tg;
                  uv[e] = sam * tu;
                }
              }
              o[i / 2] = pack2(silu_mul_bf16(gv[0], uv[0]), silu_mul_bf16(gv[1], uv[1]), 0);
            }
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.y) + m * p.ldy + ng);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            }
          }
        } else {
          for (int c0 = 0; c0 < BN; c0 += 32) {
            const int64_t n0 = static_cast<int64_t>(nb) * BN + c0;
            if (n0 >= p.N) break;  // warp-uniform
            if (p.epi == H3B_EPI_QKV_SEND && p.norm_w[0] != nullptr && n0 < 2ll * p.hd) {
              // q or k head with RMSNorm + partial RoPE: handled a whole head (128 columns) at a time
              if ((c0 & 127) == 0) {
                const int which = static_cast<int>(n0 / p.hd);
                const int hcol = static_cast<int>(n0 - static_cast<int64_t>(which) * p.hd);
                const int h = hcol >> 7;
                const int g = h / p.hg, hh = h - g * p.hg;
                const int dst_rank = hh / p.hl, j = hh - dst_rank * p.hl;
                int64_t seg;
                uint16_t* dst = send_slab(p, which, g, dst_rank, seg);
                dst += ((seg * p.M + m) * p.rsh + j) * 128;
                const __nv_bfloat16* wn = p.norm_w[which];
                const uint32_t hbase = tacc + c0;
                // pass 1: the bf16 head values (the GEMM output the reference normalises) and their sum of squares
                float ss = 0.0f;
#pragma unroll 1
                for (int cc = 0; cc < 128; cc += 32) {
                  uint32_t r[32];
                  tmem_ld32(hbase + cc, r);
                  tmem_ld_wait();
                  reg_fence(r);
                  const float4* sb4 = reinterpret_cast<const float4*>(p.sb + n0 + cc);
#pragma unroll
                  for (int i4 = 0; i4 < 8; ++i4) {
                    const float4 sv = __ldg(sb4 + i4);
                    const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const float y = rbf16(sam * (s4[e] * __uint_as_float(r[4 * i4 + e])));
                      ss = __fadd_rn(ss, __fmul_rn(y, y));
                    }
                  }
                }
                const float inv = rsqrtf(__fadd_rn(ss * (1.0f / 128.0f), p.eps));
                const int half = p.rot >> 1;
                const float* trow = p.rope + (row_ok ? m : 0) * p.rope_stride;  // rows past M read row 0
                // pass 2: 16-column blocks; block b < half/16 rotates with block b + half/16
#pragma unroll 1
                for (int b = 0; b < 8; ++b) {
                  const int e0 = 16 * b;
                  if (e0 >= half && e0 < p.rot) continue;  // written with its partner below
                  uint32_t ra[16], rb[16];
                  tmem_ld16(hbase + e0, ra);
                  const bool rotate = e0 < half;
                  if (rotate) tmem_ld16(hbase + e0 + half, rb);
                  tmem_ld_wait();
                  reg_fence16<0>(ra);
                  reg_fence16<0>(rb);
                  // 16 normalised values of columns [c, c + 16): bf16 GEMM output, * rsqrt, * weight, rounded to bf16
                  auto normed = [&](const uint32_t (&rr)[16], int c, float (&nn)[16]) {
                    const float4* sb4 = reinterpret_cast<const float4*>(p.sb + n0 + c);
                    const uint4* w8 = reinterpret_cast<const uint4*>(wn + c);
#pragma unroll
                    for (int h8 = 0; h8 < 2; ++h8) {
                      const uint4 wq = __ldg(w8 + h8);
                      const uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
                      const float4 s0 = __ldg(sb4 + 2 * h8), s1 = __ldg(sb4 + 2 * h8 + 1);
                      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                      for (int e = 0; e < 8; ++e) {
                        const int i = 8 * h8 + e;
                        const float wf = __uint_as_float((e & 1) ? (ww[e >> 1] & 0xFFFF0000u) : (ww[e >> 1] << 16));
                        const float y = rbf16(sam * (sv[e] * __uint_as_float(rr[i])));
                        nn[i] = rbf16(__fmul_rn(__fmul_rn(y, inv), wf));
                      }
                    }
                  };
                  float na[16], nb2[16];
                  normed(ra, e0, na);
                  if (rotate) {
                    normed(rb, e0 + half, nb2);
                    float oa[16], ob[16];
                    const float4* cs4 = reinterpret_cast<const float4*>(trow + e0);
                    const float4* sn4 = reinterpret_cast<const float4*>(trow + half + e0);
#pragma unroll
                    for (int i4 = 0; i4 < 4; ++i4) {
                      const float4 cv = __ldg(cs4 + i4), sv = __ldg(sn4 + i4);
                      const float c4[4] = {cv.x, cv.y, cv.z, cv.w}, s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                      for (int e = 0; e < 4; ++e) {
                        const int i = 4 * i4 + e;
                        oa[i] = __fsub_rn(__fmul_rn(na[i], c4[e]), __fmul_rn(nb2[i], s4[e]));
                        ob[i] = __fadd_rn(__fmul_rn(nb2[i], c4[e]), __fmul_rn(na[i], s4[e]));
                      }
                    }
                    if (row_ok) {
                      uint4* da = reinterpret_cast<uint4*>(dst + e0);
                      uint4* db = reinterpret_cast<uint4*>(dst + e0 + half);
#pragma unroll
                      for (int q = 0; q < 2; ++q) {
                        da[q] = make_uint4(pack2(oa[8 * q], oa[8 * q + 1], 0), pack2(oa[8 * q + 2], oa[8 * q + 3], 0),
                                           pack2(oa[8 * q + 4], oa[8 * q + 5], 0), pack2(oa[8 * q + 6], oa[8 * q + 7], 0));
                        db[q] = make_uint4(pack2(ob[8 * q], ob[8 * q + 1], 0), pack2(ob[8 * q + 2], ob[8 * q + 3], 0),
                                           pack2(ob[8 * q + 4], ob[8 * q + 5], 0), pack2(ob[8 * q + 6], ob[8 * q + 7], 0));
                      }
                    }
                  } else if (row_ok) {
                    uint4* da = reinterpret_cast<uint4*>(dst + e0);
#pragma unroll
                    for (int q = 0; q < 2; ++q)
                      da[q] = make_uint4(pack2(na[8 * q], na[8 * q + 1], 0), pack2(na[8 * q + 2], na[8 * q + 3], 0),
                                         pack2(na[8 * q + 4], na[8 * q + 5], 0), pack2(na[8 * q + 6], na[8 * q + 7], 0));
                  }
                }
              }
              continue;
            }
            uint32_t r[32];
            tmem_ld32(tacc + c0, r);
            tmem_ld_wait();
            reg_fence(r);
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 sbv = make_float4(0.f, 0.f, 0.f, 0.f);
              if (n0 + i < p.N) sbv = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + i));
              const float s4[4] = {sbv.x, sbv.y, sbv.z, sbv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float tv = s4[e] * __uint_as_float(r[i + e]);
                if (p.bias != nullptr && n0 + i + e < p.N)
                  v[i + e] = fmaf(sam, tv, __bfloat162float(p.bias[n0 + i + e]));
                else
                  v[i + e] = sam * tv;
              }
            }
            if (PEER && p.epi == H3B_EPI_QKV_SEND) {
              // peer stores (warp-uniform branch): the warp's 32 rows of this 64-column block go through shared
              // memory and leave as 4 rows x 128 B per store instruction
              const int which = static_cast<int>(n0 / p.hd);
              const int hcol = static_cast<int>(n0 - static_cast<int64_t>(which) * p.hd);
              const int h = hcol >> 7, c = hcol & 127;
              const int dst_rank = h / p.hl, j = h - dst_rank * p.hl;
              const bool as_f16 = which == 2 && p.v_f16;
              int32_t* rf = p.peer_rf[dst_rank];
              if (row_ok && as_f16 && rf != nullptr) {
                bool bad = false;
#pragma unroll
                for (int i = 0; i < 32; ++i) bad |= fabsf(v[i]) > 65504.0f && isfinite(v[i]);
                if (bad) atomicExch(rf, 1);
              }
              uint4* srow = staging + (sub * 32 + lane) * 8;
              const int hb = (c >> 5) & 1;  // which 32-column half of the 64-column block
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = as_f16 ? pack2_bf16_as_f16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1])
                                : pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], 0);
                srow[(hb * 4 + q) ^ (lane & 7)] = make_uint4(w[0], w[1], w[2], w[3]);
              }
              if (hb == 1) {
                __syncwarp();
                const int64_t m0 = static_cast<int64_t>(mb) * BM + sub * 32;
                uint16_t* base = static_cast<uint16_t*>(p.peer[dst_rank][which]) +
                                 ((static_cast<int64_t>(p.rank) * p.M + m0) * p.hl + j) * 128 + (c & 64);
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                  const int idx = it * 32 + lane, r = idx >> 3, part = idx & 7;
                  if (m0 + r < p.M)
                    *reinterpret_cast<uint4*>(base + static_cast<int64_t>(r) * p.hl * 128 + part * 8) =
                        staging[(sub * 32 + r) * 8 + (part ^ (r & 7))];
                }
                __syncwarp();
              }
              continue;
            }
            if (!row_ok) continue;
            if (p.epi == H3B_EPI_QKV_SEND) {
              // 32 columns inside one head: which tensor, which destination rank, which local head
              const int which = static_cast<int>(n0 / p.hd);
              const int hcol = static_cast<int>(n0 - static_cast<int64_t>(which) * p.hd);
              const int h = hcol >> 7, c = hcol & 127;
              const int g = h / p.hg, hh = h - g * p.hg;
              const int dst_rank = hh / p.hl, j = hh - dst_rank * p.hl;
              int64_t seg;
              uint16_t* slab = send_slab(p, which, g, dst_rank, seg);
              const int64_t off = ((seg * p.M + m) * p.rsh + j) * 128 + c;
              const bool as_f16 = which == 2 && p.v_f16;
              int32_t* rf = p.range_flag;
              if (as_f16 && rf != nullptr) {
                bool bad = false;
#pragma unroll
                for (int i = 0; i < 32; ++i) bad |= fabsf(v[i]) > 65504.0f && isfinite(v[i]);
                if (bad) atomicExch(rf, 1);
              }
              uint4* dst = reinterpret_cast<uint4*>(slab + off);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = as_f16 ? pack2_bf16_as_f16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1])
                                : pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], 0);
                dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
              }
            } else if (p.epi == EPI_GATE) {
              // y = x + gate[idx[m]] * bf16(o): fp32, product and sum rounded separately (the eager mirror's order)
              const int64_t gi = __ldg(p.gidx + m);
              if (gi < 0 || gi >= p.gate_rows) {
                record_status(p.wc, H3B_EINVAL);
                continue;
              }
              const uint4* xrow = reinterpret_cast<const uint4*>(p.gx + m * p.ldx + n0);
              const uint4* grow = reinterpret_cast<const uint4*>(p.gate + gi * p.ldg + n0);
              uint16_t* yrow = static_cast<uint16_t*>(p.y) + m * p.ldy;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (n0 + 8 * q >= p.N) break;
                const uint4 xv = __ldg(xrow + q), gv = __ldg(grow + q);
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float r[2];
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const float xf = __uint_as_float(h ? (xw[e] & 0xFFFF0000u) : (xw[e] << 16));
                    const float gf = __uint_as_float(h ? (gw[e] & 0xFFFF0000u) : (gw[e] << 16));
                    r[h] = __fadd_rn(xf, __fmul_rn(gf, rbf16(v[8 * q + 2 * e + h])));
                  }
                  w[e] = pack2(r[0], r[1], 0);
                }
                *reinterpret_cast<uint4*>(yrow + n0 + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            } else {
              uint16_t* yrow = static_cast<uint16_t*>(p.y) + m * p.ldy;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (n0 + 8 * q >= p.N) break;
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) w[e] = pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], p.out_f16);
                *reinterpret_cast<uint4*>(yrow + n0 + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(tempty_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace gemm
}  // namespace h3b

using namespace h3b;

namespace {
struct GateArgs {
  const void* x;
  int64_t ldx;
  const void* gate;
  int64_t ldg;
  int64_t gate_rows;
  const int64_t* indices;
};

int fp8_gemm_impl(const void* a, int64_t lda, const void* w, int64_t ldw, const float* sa, const float* sb,
                  const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int32_t out_dtype,
                  int32_t epilogue, const h3b_qkv_send* send, const GateArgs* ga, h3b_stream_t stream) {
  using namespace h3b::gemm;
  if (M < 0 || N <= 0 || K <= 0) return fail(H3B_EINVAL, "fp8_gemm: M %lld N %lld K %lld", (long long)M, (long long)N, (long long)K);
  if (out_dtype != H3B_OUT_BF16 && out_dtype != H3B_OUT_F16) return fail(H3B_EINVAL, "fp8_gemm: out dtype %d", out_dtype);
  if (M == 0) return H3B_OK;
  if (a == nullptr || w == nullptr || sa == nullptr || sb == nullptr) return fail(H3B_EINVAL, "fp8_gemm: null operand");
  if (K % 16 || N % 16) return fail(H3B_EUNSUPPORTED, "fp8_gemm: K and N must be multiples of 16");
  if (lda < K || ldw < K || lda % 16 || ldw % 16) return fail(H3B_EALIGN, "fp8_gemm: lda/ldw must be >= K and multiples of 16");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(sb)) & 15u)
    return fail(H3B_EALIGN, "fp8_gemm: a, w and sb must be 16-byte aligned");
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1) return fail(H3B_EUNSUPPORTED, "fp8_gemm: dims above 2^31");

  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sa = sa;
  p.sb = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = y;
  p.ldy = ldy;
  p.out_f16 = out_dtype == H3B_OUT_F16;
  p.epi = epilogue;
  p.num_mb = static_cast<int>((M + BM - 1) / BM);
  p.num_kb = static_cast<int>((K + BK - 1) / BK);
  if (epilogue == H3B_EPI_SWIGLU) {
    if (N % 256) return fail(H3B_EUNSUPPORTED, "fp8_gemm swiglu: N/2 must be a multiple of 128");
    if (out_dtype != H3B_OUT_BF16) return fail(H3B_EUNSUPPORTED, "fp8_gemm swiglu: bf16 output only");
    if (y == nullptr || ldy < N / 2 || ldy % 8) return fail(H3B_EINVAL, "fp8_gemm swiglu: y / ldy");
    p.half = N / 2;
    p.num_nb = static_cast<int>(p.half / 128);
  } else if (epilogue == H3B_EPI_QKV_SEND) {
    if (send == nullptr) return fail(H3B_EINVAL, "fp8_gemm qkv_send: send descriptor");
    if (send->head_dim != 128) return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: head_dim must be 128");
    if (send->heads <= 0 || send->ws <= 0 || send->heads % send->ws) return fail(H3B_EINVAL, "fp8_gemm qkv_send: heads % ws");
    if (N != 3ll * send->heads * 128) return fail(H3B_EINVAL, "fp8_gemm qkv_send: N must be 3 * heads * 128");
    if (out_dtype != H3B_OUT_BF16) return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: bf16 output only");
    const int groups = send->groups > 1 ? send->groups : 1;
    if (send->p2p) {
      if (groups != 1) return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: p2p with head groups");
      if (send->ws > H3B_MAX_RANKS || send->rank < 0 || send->rank >= send->ws)
        return fail(H3B_EINVAL, "fp8_gemm qkv_send: p2p ws %d rank %d", send->ws, send->rank);
      p.p2p = 1;
      p.rank = send->rank;
      for (int r = 0; r < send->ws; ++r) {
        for (int i = 0; i < 3; ++i) {
          if (send->peer_recv[r][i] == nullptr || (reinterpret_cast<uintptr_t>(send->peer_recv[r][i]) & 15u))
            return fail(H3B_EALIGN, "fp8_gemm qkv_send: peer buffer %d/%d null or not 16-byte aligned", r, i);
          p.peer[r][i] = send->peer_recv[r][i];
        }
        p.peer_rf[r] = send->v_f16 ? send->peer_range_flag[r] : nullptr;
      }
    } else if (send->qkv_interleaved) {
      if (send->send[0] == nullptr || (reinterpret_cast<uintptr_t>(send->send[0]) & 15u))
        return fail(H3B_EALIGN, "fp8_gemm qkv_send: send buffer null or not 16-byte aligned");
      p.send[0] = send->send[0];
    } else {
      for (int i = 0; i < 3; ++i) {
        if (send->send[i] == nullptr || (reinterpret_cast<uintptr_t>(send->send[i]) & 15u))
          return fail(H3B_EALIGN, "fp8_gemm qkv_send: send buffer %d null or not 16-byte aligned", i);
        p.send[i] = send->send[i];
      }
    }
    if (send->heads % (groups * send->ws)) return fail(H3B_EINVAL, "fp8_gemm qkv_send: heads %% (groups * ws) != 0");
    if ((send->q_norm_weight == nullptr) != (send->k_norm_weight == nullptr))
      return fail(H3B_EINVAL, "fp8_gemm qkv_send: q and k norm weights go together");
    if (send->q_norm_weight != nullptr) {
      if (send->rot < 0 || send->rot > 128 || send->rot % 32)
        return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: rot %d (0, 32, 64, 96 or 128)", send->rot);
      if (send->rot > 0 && send->rope_table == nullptr) return fail(H3B_EINVAL, "fp8_gemm qkv_send: rope table");
      if (((reinterpret_cast<uintptr_t>(send->q_norm_weight) | reinterpret_cast<uintptr_t>(send->k_norm_weight) |
            reinterpret_cast<uintptr_t>(send->rope_table)) & 15u) || (send->rot > 0 && send->rope_stride % 4))
        return fail(H3B_EALIGN, "fp8_gemm qkv_send: norm weights and rope table 16-byte aligned, rope_stride % 4 == 0");
      p.norm_w[0] = static_cast<const __nv_bfloat16*>(send->q_norm_weight);
      p.norm_w[1] = static_cast<const __nv_bfloat16*>(send->k_norm_weight);
      p.rope = send->rope_table;
      p.rope_stride = send->rope_stride;
      p.rot = send->rot;
      p.eps = send->eps;
    }
    p.hd = send->heads * 128;
    p.hg = send->heads / groups;
    p.hl = p.hg / send->ws;
    if (send->qkv_interleaved && send->p2p) return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: interleaved with p2p");
    p.rsh = send->qkv_interleaved ? 3 * p.hl : p.hl;
    p.qkv_step = send->qkv_interleaved ? static_cast<int64_t>(p.hl) * 128 : 0;
    p.ws = send->ws;
    p.v_f16 = send->v_f16 != 0;
    p.range_flag = send->range_flag;
    p.num_nb = static_cast<int>((N + BN - 1) / BN);
  } else {
    if (y == nullptr || ldy < N || ldy % 8 || (reinterpret_cast<uintptr_t>(y) & 15u))
      return fail(H3B_EALIGN, "fp8_gemm: y must be 16-byte aligned with ldy >= N, ldy % 8 == 0");
    if (epilogue == EPI_GATE) {
      if (ga == nullptr || ga->x == nullptr || ga->gate == nullptr || ga->indices == nullptr || ga->gate_rows <= 0)
        return fail(H3B_EINVAL, "fp8_gemm_gate: x, gate (>= 1 row) and indices are required");
      if (out_dtype != H3B_OUT_BF16) return fail(H3B_EUNSUPPORTED, "fp8_gemm_gate: bf16 output only");
      if (ga->ldx < N || ga->ldx % 8 || ga->ldg < N || ga->ldg % 8 ||
          ((reinterpret_cast<uintptr_t>(ga->x) | reinterpret_cast<uintptr_t>(ga->gate)) & 15u))
        return fail(H3B_EALIGN, "fp8_gemm_gate: x and gate must be 16-byte aligned with leading dimensions >= N, % 8 == 0");
      p.gx = static_cast<const uint16_t*>(ga->x);
      p.ldx = ga->ldx;
      p.gate = static_cast<const uint16_t*>(ga->gate);
      p.ldg = ga->ldg;
      p.gate_rows = ga->gate_rows;
      p.gidx = ga->indices;
    }
    p.num_nb = static_cast<int>((N + BN - 1) / BN);
  }
  p.wc.status = device_status_word();
  p.wc.timeout = wait_timeout_ns();
  if (p.wc.status == nullptr) return fail(H3B_ECUDA, "fp8_gemm: device status word");

  CUtensorMap tmA, tmB;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda)};
    const uint32_t box[2] = {BK, BM};
    int rc = encode_tmap(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw)};
    const uint32_t box[2] = {BK, 128};
    int rc = encode_tmap(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fp8_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES_PEER);
    if (e != cudaSuccess) return cuda_fail(e, "fp8_gemm: smem attribute");
    attr_set[dev] = true;
  }
  const int tiles = p.num_mb * p.num_nb;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (p.p2p)
    fp8_gemm_kernel<true><<<grid, THREADS, SMEM_BYTES_PEER, reinterpret_cast<cudaStream_t>(stream)>>>(tmA, tmB, p);
  else
    fp8_gemm_kernel<false><<<grid, THREADS, SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(tmA, tmB, p);
  H3B_CHECK_LAUNCH("fp8_gemm launch");
  return H3B_OK;
}
}  // namespace

extern "C" int h3b_fp8_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, const float* sa, const float* sb,
                            const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int32_t out_dtype,
                            int32_t epilogue, const h3b_qkv_send* send, h3b_stream_t stream) {
  if (epilogue < H3B_EPI_PLAIN || epilogue > H3B_EPI_SWIGLU) return fail(H3B_EINVAL, "fp8_gemm: epilogue %d", epilogue);
  return fp8_gemm_impl(a, lda, w, ldw, sa, sb, bias, y, ldy, M, N, K, out_dtype, epilogue, send, nullptr, stream);
}

extern "C" int h3b_fp8_gemm_gate(const void* a, int64_t lda, const void* w, int64_t ldw, const float* sa,
                                 const float* sb, const void* bias, const void* x, int64_t ldx, const void* gate,
                                 int64_t ld_gate, int64_t gate_rows, const int64_t* indices, void* y, int64_t ldy,
                                 int64_t M, int64_t N, int64_t K, h3b_stream_t stream) {
  const GateArgs ga{x, ldx, gate, ld_gate, gate_rows, indices};
  return fp8_gemm_impl(a, lda, w, ldw, sa, sb, bias, y, ldy, M, N, K, H3B_OUT_BF16, h3b::gemm::EPI_GATE, nullptr, &ga,
                       stream);
}
