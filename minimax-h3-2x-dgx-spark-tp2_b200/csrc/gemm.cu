// FP8 (e4m3 x e4m3 -> f32) GEMM on the 5th-generation tensor cores with the per-token x per-channel scaled epilogue
// fused: y = out(sa[m] * (sb[n] * acc)) (bias by fma), the arithmetic of fp8_gemm._scale_bias_cast
// (h3_tp2/fp8_gemm.py:38-54) and of the CuTe-DSL kernel's epilogue (h3_tp2/fp8_cutlass_kernel.py), with no fp32
// product in memory.
//
// Design (CTA pairs: clusters of two CTAs on two SMs, persistent over 256 x 256 output tiles):
//   The pair computes a 256 x 256 tile with 2-SM MMAs (tcgen05.mma.cta_group::2, M = 256, N = 256, K = 32): CTA r
//   of the pair holds rows [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128) of the B tile in its
//   shared memory, and rows [128 r, 128 r + 128) x all 256 columns of the accumulator in its TMEM.  Each SM thus
//   stages 32 KB per 128-deep K step instead of the 48 KB a one-CTA 128 x 256 tile needs for the same MMA work, and
//   the 6-stage ring (192 KB) covers 1.5x the L2 latency of the one-CTA ring.
//   warp 0      : TMA producer (one elected thread per CTA): A box 128x128 B and one B box 128x128 B per stage, both
//                 counted on the even (leader) CTA's full barrier, which expects the pair's 64 KB
//   warp 1      : TMEM allocator of the pair; in the leader, the single-thread tcgen05.mma issuer, whose commits
//                 arrive on both CTAs' barriers
//   warps 2..5  : epilogue; thread t of the 128 owns accumulator row t of its CTA (TMEM lane), reads 32-column
//                 slices with tcgen05.ld, applies the scales (and SwiGLU to the gate/up halves, or the gated
//                 residual), stages each 128-column block of its warp's 32 rows in shared memory and stores it as two
//                 whole rows per instruction or as TMA boxes (into y, or scattered into the Ulysses send layout); each
//                 warp arrives on the leader's accumulator-empty barrier once its TMEM reads of a tile are done (8
//                 arrivals per tile, 4 of them from the other CTA).
//   Two epilogue forms run 8 warps (2..9; the template MODE): SwiGLU (MODE_SWIGLU8, each warp 64 of a tile's 128
//   output columns of its 32 rows) and the q/k/v send layout with qk RMSNorm + RoPE (MODE_QKV8, each warp one of the
//   tile's two 128-column heads, with 64 KB of staging and a 5-stage ring); the accumulator-empty barrier then counts
//   16 arrivals.
//   The accumulator is double buffered in TMEM (2 x 256 of the 512 columns) so the epilogue of tile i overlaps the
//   main loop of tile i+1.  Every wait is bounded (common.cuh).  No TMA multicast.
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace h3b {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 6;  // BM: rows per CTA (the pair's tile is 2 x BM rows)
constexpr int A_BYTES = BM * BK;   // 16 KB
constexpr int B_BYTES = 128 * BK;  // 16 KB: this CTA's half of the 256 B rows
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;  // producer, MMA issuer, 4 epilogue warps (the 8-warp forms: THREADS + 128)
// pair row blocks (256 rows each) sharing one column block's W tile in L2: 16 measured 2-4 % faster than 8 on the
// qkv GEMM and the FFN at 15,624-124,992 rows (interleaved runs on one GPU), 12, 24 and 32 slower
constexpr int GROUP_M = 16;
constexpr int EPI_GATE = 3;  // internal epilogue kind of h3b_fp8_gemm_gate
// epilogue staging: per epilogue warp 32 rows x 256 B (one 128-column block of its rows); 64 KB for the 8-warp q/k/v
// form, which holds one block per warp and runs a 5-stage ring to make room
constexpr int STAGING_BYTES = 4 * 32 * 256;
// epilogue forms: 0 four warps (every epilogue), 1 eight warps for SwiGLU, 2 eight warps for the q/k/v send layout
constexpr int MODE_STD = 0, MODE_SWIGLU8 = 1, MODE_QKV8 = 2;
__host__ __device__ constexpr int mode_stages(int mode) { return mode == MODE_QKV8 ? 5 : STAGES; }
__host__ __device__ constexpr int mode_staging(int mode) { return mode == MODE_QKV8 ? 2 * STAGING_BYTES : STAGING_BYTES; }
// ring, alignment slack, barriers (1 KB, so that the staging starts 1024-byte aligned as the 128-byte swizzle of the
// TMA stores needs), staging: 231,424 B of the 232,448 a CTA may have in every form
__host__ __device__ constexpr int mode_smem(int mode) {
  return mode_stages(mode) * (16384 + 16384) + 1024 + 1024 + mode_staging(mode);
}
static_assert(mode_smem(MODE_STD) <= 232448 && mode_smem(MODE_QKV8) <= 232448, "shared memory");
constexpr uint32_t IDESC = idesc_make(FMT_E4M3, FMT_E4M3, 0, 2 * BM, BN);

struct Params {
  int64_t M, N, K;
  int num_mb, num_nb, num_kb;  // num_mb: 256-row blocks of the CTA pairs
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
  int tma_out;                           // 1: staged blocks leave through TMA stores (tmY, below)
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

// pair tile t -> (256-row block, column block): GROUP_M row blocks in a row share each column block's W tile in L2
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

// With Params::p2p the QKV_SEND epilogue stores into the other GPUs' receive buffers (send_slab).
// MODE: the epilogue form.  MODE_STD: 4 epilogue warps, every epilogue.  MODE_SWIGLU8: 8 warps for the SwiGLU
// epilogue (with TMA stores), whose per-element arithmetic (silu with expf and an IEEE division, three bf16 roundings)
// makes four warps a bottleneck: each of the 8 takes 64 of a tile's 128 output columns for its 32 rows and stores
// them as one TMA box.  MODE_QKV8: 8 warps for the local q/k/v send epilogue with the qk-norm (and TMA stores),
// each taking one of the tile's two 128-column head blocks for its 32 rows (the qk-norm needs a head's 128 columns
// in one thread), with 64 KB of staging and a 5-stage ring.
template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(MODE == MODE_STD ? THREADS : THREADS + 128, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmY0, const __grid_constant__ CUtensorMap tmY1,
                    const __grid_constant__ CUtensorMap tmY2, const __grid_constant__ Params p) {
  constexpr int EW = MODE == MODE_STD ? 4 : 8;
  constexpr int NST = mode_stages(MODE);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NST * STAGE_BYTES);
  // bars: full[NST], empty[NST], tfull[2], tempty[2], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NST + 5);
  uint4* staging = reinterpret_cast<uint4*>(smem + NST * STAGE_BYTES + 1024);
  const uint32_t smem0 = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (NST + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * NST + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * NST + 2 + a); };
  const uint32_t done_bar = bar0 + 8u * (2 * NST + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();  // 0: the pair's leader (issues the MMAs), 1: its partner
  const uint32_t peer = crank ^ 1u;
  const bool aborted_at_entry = status_bad(p.wc);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * EW);  // one arrival per epilogue warp of both CTAs (counted on the leader's)
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_mb * p.num_nb;
  const int first_tile = static_cast<int>(cluster_id_x());
  const int tile_step = static_cast<int>(cluster_count_x());
  if (!aborted_at_entry) {
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer (both CTAs; stage completion counted on the leader's full barrier) -------
        const uint32_t lead_full0 = mapa_shared(full_bar(0), 0);
        int stage = 0;
        uint32_t phase = 0;
        int issued[NST];
        for (int s = 0; s < NST; ++s) issued[s] = 0;
        bool ok = true;
        for (int t = first_tile; t < num_tiles && ok; t += tile_step) {
          int mb, nb;
          tile_coords(t, p, mb, nb);
          const int arow = (2 * mb + static_cast<int>(crank)) * BM;
          // this CTA's 128 B rows: SWIGLU gate rows (leader) / up rows (partner); else columns [256 nb + 128 r, +128)
          const int brow = p.epi == H3B_EPI_SWIGLU ? (crank ? static_cast<int>(p.half) : 0) + nb * 128
                                                   : nb * BN + 128 * static_cast<int>(crank);
          for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.wc)) {
              ok = false;
              break;
            }
            const uint32_t sA = smem0 + stage * STAGE_BYTES;
            const uint32_t sB = sA + A_BYTES;
            const uint32_t fb = lead_full0 + 8u * stage;
            if (crank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * STAGE_BYTES);
            tma_load_2d_pair(sA, &tmA, fb, kb * BK, arow);
            tma_load_2d_pair(sB, &tmB, fb, kb * BK, brow);
            issued[stage]++;
            if (++stage == NST) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        // drain: never leave a TMA write in flight into shared memory the CTA is about to release.  The leader
        // sees both CTAs' bytes on its full barriers; the partner's last load of a stage has landed once the
        // leader's MMAs consumed it (its empty barrier).
        for (int s = 0; s < NST; ++s)
          if (issued[s] > 0) {
            const uint32_t par = static_cast<uint32_t>(issued[s] - 1) & 1u;
            const uint32_t bar = crank == 0 ? full_bar(s) : empty_bar(s);
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(bar, par) && globaltimer() - t0 < p.wc.timeout) {
            }
          }
      }
    } else if (warp == 1) {
      if (lane == 0 && crank == 0) {
        // ---------------- MMA issuer (the leader only) ----------------
        const uint32_t peer_bar0 = mapa_shared(bar0, peer);  // the partner's barrier array
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = first_tile; t < num_tiles && ok; t += tile_step) {
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
              umma_f8_ss_pair(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, IDESC, (kb | kk) != 0);
            umma_commit_pair(empty_bar(stage));
            umma_commit_pair(peer_bar0 + 8u * (NST + stage));
            if (++stage == NST) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit_pair(tfull_bar(acc));
          umma_commit_pair(peer_bar0 + 8u * (2 * NST + acc));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        // all issued MMAs complete before TMEM is released
        umma_commit_pair(done_bar);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(done_bar, 0) && globaltimer() - t0 < p.wc.timeout) {
        }
      }
    } else {
      // ---------------- epilogue (warps 2..5) ----------------
      // Each warp turns its 32 accumulator rows into output 128 columns at a time: the values go through shared
      // memory (32 rows x 256 B per warp; 16-byte granule g of row r at r * 16 + (g ^ (r & 15))), and every store
      // instruction then writes two whole 256-byte rows (four full lines) instead of 16 bytes of 32 different rows,
      // which keeps the load/store path free for the TMA fills of the main loop.
      const int sub = warp & 3;
      const int hw = (warp - 2) >> 2;  // EW = 8: which 64 of the block's 128 output columns
      const int row_in_tile = sub * 32 + lane;
      const uint32_t lane_addr = static_cast<uint32_t>(sub * 32) << 16;
      uint4* stg = MODE == MODE_STD ? staging + sub * 32 * 16
                   : (MODE == MODE_SWIGLU8 ? staging + (warp - 2) * 32 * 8 : staging + (warp - 2) * 32 * 16);
      // With TMA stores the block is staged as the two 64-column boxes the stores read: 32 rows x 128 B each, in
      // the 128-byte swizzle (granule c of row r at r * 8 + (c ^ (r & 7))); otherwise as 32 rows x 256 B.
      const bool tma = p.tma_out != 0;
      auto stage = [&](int g, uint4 val) {
        if (tma)
          stg[(g >> 3) * 256 + lane * 8 + ((g & 7) ^ (lane & 7))] = val;
        else
          stg[lane * 16 + (g ^ (lane & 15))] = val;
      };
      // before the block's values are staged: the previous TMA stores of this warp have read the staging
      auto staging_free = [&]() {
        if (tma) {
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
        }
      };
      // the staged block leaves as two TMA stores (box 64 columns x 32 rows); rows at or beyond M and columns at or
      // beyond the map's extent are clipped by the TMA unit
      auto store_tma = [&](const CUtensorMap* map, int rank, int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t src = smem_u32(stg);
          if (rank == 2) {
            tma_store_2d(map, src, c0, c1);
            tma_store_2d(map, src + 4096, c0 + 64, c1);
          } else {
            tma_store_4d(map, src, c0, c1, c2, c3);
            tma_store_4d(map, src + 4096, c0 + 64, c1, c2, c3);
          }
          bulk_commit();
        }
      };
      // the warp's rows m0 + r (r < 32) of one 128-column block: row r to base + (m0 + r) * rstride, granules
      // below `granules`
      auto store_rows = [&](uint16_t* base, int64_t rstride, int64_t m0, int granules) {
        __syncwarp();
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
          const int r = 2 * it + (lane >> 4), g = lane & 15;
          if (m0 + r < p.M && g < granules)
            *reinterpret_cast<uint4*>(base + (m0 + r) * rstride + g * 8) = stg[r * 16 + (g ^ (r & 15))];
        }
        __syncwarp();
      };
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t lead_tempty0 = mapa_shared(tempty_bar(0), 0);
      // one arrival per warp on the leader's accumulator-empty barrier once this warp's TMEM reads of the tile are
      // complete (tcgen05.wait::ld is warp-wide); the stores of the last block follow it
      auto release_acc = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead_tempty0 + 8u * acc);
      };
      for (int t = first_tile; t < num_tiles; t += tile_step) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        mb = 2 * mb + static_cast<int>(crank);  // this CTA's 128-row block
        if (!mbar_wait(tfull_bar(acc), acc_phase, p.wc)) break;
        tc_fence_after();
        const int64_t m = static_cast<int64_t>(mb) * BM + row_in_tile;
        const int64_t m0 = static_cast<int64_t>(mb) * BM + sub * 32;  // the warp's first row
        const bool row_ok = m < p.M;
        const float sam = row_ok ? __ldg(p.sa + m) : 0.0f;
        const uint32_t tacc = tmem_base + lane_addr + static_cast<uint32_t>(acc * BN);
        if (MODE == MODE_SWIGLU8 || (MODE == MODE_STD && p.epi == H3B_EPI_SWIGLU)) {
          staging_free();
          for (int c0 = MODE == MODE_SWIGLU8 ? 64 * hw : 0; c0 < (MODE == MODE_SWIGLU8 ? 64 * hw + 64 : 128); c0 += 32) {
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
              // column scales of the gate and up halves, two at a time (ng and nu are multiples of 32)
              const float2 sg = __ldg(reinterpret_cast<const float2*>(p.sb + ng + i));
              const float2 su = __ldg(reinterpret_cast<const float2*>(p.sb + nu + i));
              const float sgv[2] = {sg.x, sg.y}, suv[2] = {su.x, su.y};
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float tg = sgv[e] * __uint_as_float(g[i + e]);
                const float tu = suv[e] * __uint_as_float(u[i + e]);
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
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const uint4 val = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
              if (MODE == MODE_SWIGLU8) {
                const int g = (c0 - 64 * hw) / 8 + v;  // granule of the warp's own 64-column box
                stg[lane * 8 + (g ^ (lane & 7))] = val;
              } else {
                stage(c0 / 8 + v, val);
              }
            }
          }
          release_acc();
          if (MODE == MODE_SWIGLU8) {  // one box: the warp's 32 rows x its 64 columns
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmY0, smem_u32(stg), nb * 128 + 64 * hw, static_cast<int32_t>(m0));
              bulk_commit();
            }
          } else if (tma) {
            store_tma(&tmY0, 2, nb * 128, static_cast<int32_t>(m0), 0, 0);
          } else {
            store_rows(static_cast<uint16_t*>(p.y) + static_cast<int64_t>(nb) * 128, p.ldy, m0, 16);
          }
        } else if constexpr (MODE != MODE_SWIGLU8) {
          // MODE_QKV8: this warp's one block (hw); every warp still releases the accumulator once per tile
          for (int b0 = MODE == MODE_QKV8 ? 128 * hw : 0; b0 < (MODE == MODE_QKV8 ? 128 * hw + 128 : BN); b0 += 128) {
            const int64_t nbk = static_cast<int64_t>(nb) * BN + b0;  // first column of the block
            const bool last_block = MODE == MODE_QKV8 || b0 + 128 >= BN || nbk + 128 >= p.N;
            if (nbk >= p.N) {  // warp-uniform
              if (MODE == MODE_QKV8) release_acc();
              break;
            }
            // QKV_SEND: the block is one head of q, k or v; its destination rows are 256 B apart from the slab base
            int which = 0, dst_rank = 0, j = 0;
            uint16_t* qbase = nullptr;
            int64_t qstride = 0;
            if (p.epi == H3B_EPI_QKV_SEND) {
              which = static_cast<int>(nbk / p.hd);
              const int h = static_cast<int>(nbk - static_cast<int64_t>(which) * p.hd) >> 7;
              const int g = h / p.hg, hh = h - g * p.hg;
              dst_rank = hh / p.hl;
              j = hh - dst_rank * p.hl;
              int64_t seg;
              uint16_t* slab = send_slab(p, which, g, dst_rank, seg);
              qbase = slab + (seg * p.M * p.rsh + j) * 128;
              qstride = static_cast<int64_t>(p.rsh) * 128;
            }
            if (p.epi == H3B_EPI_QKV_SEND && p.norm_w[0] != nullptr && which < 2) {
              // q or k head with RMSNorm + partial RoPE: with TMA stores the head is staged and leaves as whole lines
              // like the other blocks; without them each thread stores its row's values (staging for plain stores
              // measured 3 % slower here)
              const __nv_bfloat16* wn = p.norm_w[which];
              staging_free();
              uint16_t* dst = qbase + m * qstride;
              const uint32_t hbase = tacc + b0;
              // pass 1: the bf16 head values (the GEMM output the reference normalises) and their sum of squares
              float ss = 0.0f;
#pragma unroll 1
              for (int cc = 0; cc < 128; cc += 32) {
                uint32_t r[32];
                tmem_ld32(hbase + cc, r);
                tmem_ld_wait();
                reg_fence(r);
                const float4* sb4 = reinterpret_cast<const float4*>(p.sb + nbk + cc);
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
                  const float4* sb4 = reinterpret_cast<const float4*>(p.sb + nbk + c);
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
                  if (tma) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                      stage((e0 >> 3) + q, make_uint4(pack2(oa[8 * q], oa[8 * q + 1], 0), pack2(oa[8 * q + 2], oa[8 * q + 3], 0),
                                                      pack2(oa[8 * q + 4], oa[8 * q + 5], 0), pack2(oa[8 * q + 6], oa[8 * q + 7], 0)));
                      stage(((e0 + half) >> 3) + q,
                            make_uint4(pack2(ob[8 * q], ob[8 * q + 1], 0), pack2(ob[8 * q + 2], ob[8 * q + 3], 0),
                                       pack2(ob[8 * q + 4], ob[8 * q + 5], 0), pack2(ob[8 * q + 6], ob[8 * q + 7], 0)));
                    }
                  } else if (row_ok) {
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
                } else if (tma) {
#pragma unroll
                  for (int q = 0; q < 2; ++q)
                    stage((e0 >> 3) + q, make_uint4(pack2(na[8 * q], na[8 * q + 1], 0), pack2(na[8 * q + 2], na[8 * q + 3], 0),
                                                    pack2(na[8 * q + 4], na[8 * q + 5], 0), pack2(na[8 * q + 6], na[8 * q + 7], 0)));
                } else if (row_ok) {
                  uint4* da = reinterpret_cast<uint4*>(dst + e0);
#pragma unroll
                  for (int q = 0; q < 2; ++q)
                    da[q] = make_uint4(pack2(na[8 * q], na[8 * q + 1], 0), pack2(na[8 * q + 2], na[8 * q + 3], 0),
                                       pack2(na[8 * q + 4], na[8 * q + 5], 0), pack2(na[8 * q + 6], na[8 * q + 7], 0));
                }
              }
              if (last_block) release_acc();
              if (tma) {
                const int h = static_cast<int>(nbk - static_cast<int64_t>(which) * p.hd) >> 7;
                store_tma(which == 0 ? &tmY0 : &tmY1, 4, 0, j, static_cast<int32_t>(m0), (h / p.hg) * p.ws + dst_rank);
              }
              continue;
            }
            // scaled accumulator of the block, 32 columns at a time, staged as the output's 16-bit values
            staging_free();
            const bool as_f16 = p.epi == H3B_EPI_QKV_SEND && which == 2 && p.v_f16;
            int32_t* rf = p.epi == H3B_EPI_QKV_SEND ? (p.p2p ? p.peer_rf[dst_rank] : p.range_flag) : nullptr;
            for (int c = 0; c < 128; c += 32) {
              const int64_t n0 = nbk + c;
              if (n0 >= p.N) break;  // warp-uniform
              uint32_t r[32];
              tmem_ld32(tacc + b0 + c, r);
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
              if (row_ok && as_f16 && rf != nullptr) {
                bool bad = false;
#pragma unroll
                for (int i = 0; i < 32; ++i) bad |= fabsf(v[i]) > 65504.0f && isfinite(v[i]);
                if (bad && p.p2p) {
                  // every rank's flag, not only the destination's: after the epoch barrier that follows this GEMM
                  // all ranks then see the same flag and take the same decision
                  for (int r = 0; r < p.ws; ++r)
                    if (p.peer_rf[r] != nullptr) atomicExch(p.peer_rf[r], 1);
                } else if (bad) {
                  atomicExch(rf, 1);
                }
              }
              const int f16 = p.epi == H3B_EPI_PLAIN ? p.out_f16 : 0;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = as_f16 ? pack2_bf16_as_f16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1])
                                : pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], f16);
                stage(c / 8 + q, make_uint4(w[0], w[1], w[2], w[3]));
              }
            }
            if (last_block) release_acc();
            const int granules = p.N - nbk >= 128 ? 16 : static_cast<int>((p.N - nbk) / 8);
            if (p.epi == H3B_EPI_QKV_SEND && tma) {
              // map of q, k or v: (d, head in the send row, token, group-major slab), box (64, 1, 32, 1)
              const int h = static_cast<int>(nbk - static_cast<int64_t>(which) * p.hd) >> 7;
              const int g = h / p.hg;
              store_tma(which == 0 ? &tmY0 : (which == 1 ? &tmY1 : &tmY2), 4, 0, j, static_cast<int32_t>(m0),
                        g * p.ws + dst_rank);
            } else if (p.epi == H3B_EPI_QKV_SEND) {
              store_rows(qbase, qstride, m0, 16);  // with p2p: the destination rank's receive buffer
            } else if (p.epi == EPI_GATE) {
              // y = x + gate[idx[m]] * o with o the staged bf16 output: fp32, product and sum rounded separately
              // (the eager mirror's order); two rows per instruction, 16 bytes of x, gate and y per lane
              __syncwarp();
#pragma unroll 2
              for (int it = 0; it < 16; ++it) {
                const int r = 2 * it + (lane >> 4), g = lane & 15;
                const int64_t mr = m0 + r;
                if (mr >= p.M || g >= granules) continue;
                const int64_t gi = __ldg(p.gidx + mr);
                if (gi < 0 || gi >= p.gate_rows) {
                  record_status(p.wc, H3B_EINVAL);
                  continue;
                }
                const int64_t col = nbk + g * 8;
                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(p.gx + mr * p.ldx + col));
                const uint4 gv = __ldg(reinterpret_cast<const uint4*>(p.gate + gi * p.ldg + col));
                const uint4 ov = stg[r * 16 + (g ^ (r & 15))];
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
                const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float rr[2];
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const float xf = __uint_as_float(h ? (xw[e] & 0xFFFF0000u) : (xw[e] << 16));
                    const float gf = __uint_as_float(h ? (gw[e] & 0xFFFF0000u) : (gw[e] << 16));
                    const float of = __uint_as_float(h ? (ow[e] & 0xFFFF0000u) : (ow[e] << 16));
                    rr[h] = __fadd_rn(xf, __fmul_rn(gf, of));
                  }
                  w[e] = pack2(rr[0], rr[1], 0);
                }
                *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + mr * p.ldy + col) = make_uint4(w[0], w[1], w[2], w[3]);
              }
              __syncwarp();
            } else if (tma) {
              store_tma(&tmY0, 2, static_cast<int32_t>(nbk), static_cast<int32_t>(m0), 0, 0);
            } else {
              store_rows(static_cast<uint16_t*>(p.y) + nbk, p.ldy, m0, granules);
            }
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (tma && lane == 0) bulk_wait_all0();  // this warp's TMA stores are complete before the CTA leaves
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves (or frees the pair's TMEM) while the other may still signal it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
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
  p.num_mb = static_cast<int>((M + 2 * BM - 1) / (2 * BM));
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
      if (bias != nullptr) return fail(H3B_EUNSUPPORTED, "fp8_gemm qkv_send: the norm + RoPE epilogue has no bias term");
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
  // output maps of the TMA-store epilogue: plain and SwiGLU outputs, and the local (not peer) q/k/v send buffers;
  // H3B_GEMM_TMA_STORE=0 keeps the staged blocks on plain stores (a tuning switch: both write the same bytes)
  CUtensorMap tmY[3];
  memset(tmY, 0, sizeof(tmY));
  static const bool tma_store_on = [] {
    const char* v = getenv("H3B_GEMM_TMA_STORE");
    return v == nullptr || v[0] == '\0' || atoi(v) != 0;
  }();
  if (tma_store_on) {
    if (epilogue == H3B_EPI_PLAIN || (epilogue == H3B_EPI_SWIGLU && (reinterpret_cast<uintptr_t>(y) & 15u) == 0)) {
      const uint64_t cols = static_cast<uint64_t>(epilogue == H3B_EPI_SWIGLU ? p.half : N);
      const uint64_t dims[2] = {cols, static_cast<uint64_t>(M)};
      const uint64_t strides[1] = {static_cast<uint64_t>(ldy) * 2};
      const uint32_t box[2] = {64, 32};
      int rc = encode_tmap(&tmY[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, y, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      p.tma_out = 1;
    } else if (epilogue == H3B_EPI_QKV_SEND && !p.p2p) {
      const int groups = send->groups > 1 ? send->groups : 1;
      const uint64_t row = static_cast<uint64_t>(p.rsh) * 256;  // bytes between a slab's token rows
      const uint64_t dims[4] = {128, static_cast<uint64_t>(p.hl), static_cast<uint64_t>(M),
                                static_cast<uint64_t>(groups) * static_cast<uint64_t>(p.ws)};
      const uint64_t strides[3] = {256, row, row * static_cast<uint64_t>(M)};
      const uint32_t box[4] = {64, 1, 32, 1};
      for (int i = 0; i < 3; ++i) {
        const void* base = p.qkv_step ? static_cast<const void*>(static_cast<const uint16_t*>(p.send[0]) + i * p.qkv_step)
                                      : p.send[i];
        int rc = encode_tmap(&tmY[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, base, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
      }
      p.tma_out = 1;
    }
  }
  // per device and kernel form: the shared-memory limit and how many CTA pairs fit at once (a pair needs two SMs of
  // one GPC; the grid is that many pairs, or fewer when there are fewer tiles).  The SwiGLU epilogue with TMA stores
  // runs the 8-epilogue-warp form (H3B_GEMM_SWIGLU_WARPS=4, a tuning switch, keeps 4: both write the same bytes);
  static const bool swiglu8_on = [] {
    const char* v = getenv("H3B_GEMM_SWIGLU_WARPS");
    return v == nullptr || v[0] == '\0' || atoi(v) != 4;
  }();
  // the local q/k/v send epilogue with the qk-norm + RoPE and TMA stores runs the 8-warp form (4.90 against 5.01-5.14
  // ms at 62,496 rows; without the norm the 5-stage ring costs more than the extra warps give back: 4.11-4.17 against
  // 4.08-4.13, so that one keeps 4).  H3B_GEMM_QKV_WARPS=4 keeps 4 for the norm form too (same bytes).
  static const bool qkv8_on = [] {
    const char* v = getenv("H3B_GEMM_QKV_WARPS");
    return v == nullptr || v[0] == '\0' || atoi(v) != 4;
  }();
  int mode = MODE_STD;
  if (swiglu8_on && epilogue == H3B_EPI_SWIGLU && p.tma_out) mode = MODE_SWIGLU8;
  if (qkv8_on && epilogue == H3B_EPI_QKV_SEND && p.tma_out && p.norm_w[0] != nullptr) mode = MODE_QKV8;
  static int pairs_fit[3][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(H3B_EUNSUPPORTED, "fp8_gemm: device ordinal %d", dev);
  const int threads = mode == MODE_STD ? THREADS : THREADS + 128;
  const int smem = mode_smem(mode);
  static std::mutex fit_mu;  // first calls from several threads compute the entry once
  std::unique_lock<std::mutex> fit_lock(fit_mu);
  int& fit_dev = pairs_fit[mode][dev];
  if (fit_dev == 0) {
    auto kern = mode == MODE_SWIGLU8 ? fp8_gemm_kernel<MODE_SWIGLU8>
                                     : (mode == MODE_QKV8 ? fp8_gemm_kernel<MODE_QKV8> : fp8_gemm_kernel<MODE_STD>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int fit = 0;
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(num_sms() & ~1), 1, 1);
      cfg.blockDim = dim3(threads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      e = cudaOccupancyMaxActiveClusters(&fit, kern, &cfg);
    }
    if (e != cudaSuccess) return cuda_fail(e, "fp8_gemm: smem attribute / cluster occupancy");
    if (fit < 1) return fail(H3B_EUNSUPPORTED, "fp8_gemm: no CTA pair fits on this device");
    fit_dev = fit;
  }
  const int fit_now = fit_dev;
  fit_lock.unlock();
  const int tiles = p.num_mb * p.num_nb;
  const int grid = 2 * (tiles < fit_now ? tiles : fit_now);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (mode == MODE_SWIGLU8)
    fp8_gemm_kernel<MODE_SWIGLU8><<<grid, threads, smem, st>>>(tmA, tmB, tmY[0], tmY[1], tmY[2], p);
  else if (mode == MODE_QKV8)
    fp8_gemm_kernel<MODE_QKV8><<<grid, threads, smem, st>>>(tmA, tmB, tmY[0], tmY[1], tmY[2], p);
  else
    fp8_gemm_kernel<MODE_STD><<<grid, threads, smem, st>>>(tmA, tmB, tmY[0], tmY[1], tmY[2], p);
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
