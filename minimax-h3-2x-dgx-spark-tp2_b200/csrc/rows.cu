// Row kernels of the hot path (HBM bound): the per-token dynamic FP8 quant and the producers fused with it
// (RMSNorm + modulation, gated residual + RMSNorm, SiLU-mul, the SwiGLU scale pass), the two-pass scale epilogue and
// the Ulysses layout kernels.
//
// One CTA per row.  The row is read once with 16-byte loads and kept in registers as packed bf16 (the value the
// stock producer would store), reduced for its abs-max across the CTA, and written once as e4m3 with 8-byte stores.
// Quant arithmetic (fp8_quant_fuse.py:4-13, ulysses_outq.py:15-26):
//   amax  = max |h| (NaN propagates)
//   scale = max(amax / 448, 1/(448*512))        division: IEEE (eager torch) or div.full (Triton `/`)
//   q     = e4m3_rn(clamp(h * (1 / scale), -448, 448))
#include <stdio.h>

#include "common.cuh"

namespace h3b {

static constexpr float kFp8Max = 448.0f;
static constexpr float kMinScale = 1.0f / (448.0f * 512.0f);

__device__ __forceinline__ float qdiv(float a, float b, int mode) {
  return mode == H3B_DIV_FULL ? div_full(a, b) : __fdiv_rn(a, b);
}

// abs-max of non-negative bf16 bit patterns as unsigned integers: for |x| the bit order is the value order, and every
// NaN pattern (0x7F81..0x7FFF) sorts above +inf (0x7F80), so the integer max propagates NaN like the reference's max
template <int THREADS>
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t* red) {
  v = __reduce_max_sync(0xffffffffu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < THREADS / 32 ? red[lane] : 0u;
    w = __reduce_max_sync(0xffffffffu, w);
    if (lane == 0) red[32] = w;
  }
  __syncthreads();
  return red[32];
}

template <int THREADS>
__device__ __forceinline__ float block_max_nan(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < THREADS / 32 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = nan_max(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) red[32] = w;
  }
  __syncthreads();
  return red[32];
}

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < THREADS / 32 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) red[32] = w;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// running abs-max of 8 bf16 values, kept as two packed 16-bit unsigned maxima
__device__ __forceinline__ uint32_t absmax8(const uint4& v, uint32_t m2) {
  m2 = __vmaxu2(m2, v.x & 0x7FFF7FFFu);
  m2 = __vmaxu2(m2, v.y & 0x7FFF7FFFu);
  m2 = __vmaxu2(m2, v.z & 0x7FFF7FFFu);
  m2 = __vmaxu2(m2, v.w & 0x7FFF7FFFu);
  return m2;
}
__device__ __forceinline__ uint32_t fold16(uint32_t m2) { return max(m2 & 0xFFFFu, m2 >> 16); }

// 8 bf16 -> 8 e4m3 (one 8-byte word): x * inv, round to nearest even; satfinite clamps to +-448 exactly as the
// reference's clamp does for every finite or infinite product, and keeps NaN
__device__ __forceinline__ uint2 quant8(const uint4& v, float inv) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint16_t a = f32x2_to_e4m3x2(lo_bf16(w[2 * i]) * inv, hi_bf16(w[2 * i]) * inv);
    const uint16_t b = f32x2_to_e4m3x2(lo_bf16(w[2 * i + 1]) * inv, hi_bf16(w[2 * i + 1]) * inv);
    o[i] = static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
  }
  return make_uint2(o[0], o[1]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// the quant tail shared by every row kernel: row held as VPT x 8 bf16 per thread (vector i = tid + k*THREADS),
// m2 = this thread's packed abs-max bits
template <int THREADS, int VPT>
__device__ __forceinline__ void quant_tail(const uint4 (&h)[VPT], uint32_t m2, int64_t nvec, uint8_t* qrow,
                                           float* srow, int div_mode, uint32_t* red) {
  const float amax = __uint_as_float(block_max_u32<THREADS>(fold16(m2), red) << 16);
  const float scale = nan_max(qdiv(amax, kFp8Max, div_mode), kMinScale);
  const float inv = qdiv(1.0f, scale, div_mode);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * THREADS;
    if (i < nvec) *reinterpret_cast<uint2*>(qrow + i * 8) = quant8(h[k], inv);
  }
  if (threadIdx.x == 0) *srow = scale;
}

// ---------------------------------------------------------------------------------------------------------------
// K6 / K10: quant of segmented rows (ulysses_outq._quant_rows_kernel, fp8_quant_fuse._quant_kernel/_unpack_quant)
// ---------------------------------------------------------------------------------------------------------------
template <int THREADS, int VPT, bool SEGMENTED>
__global__ void __launch_bounds__(THREADS) quant_rows_vec_kernel(const __nv_bfloat16* __restrict__ base, int64_t m,
                                                                 int64_t segv, int64_t stride_p, int64_t stride_m,
                                                                 int64_t nvec, uint8_t* __restrict__ q,
                                                                 float* __restrict__ s, int div_mode) {
  __shared__ uint32_t red[33];
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    uint4 h[VPT];
    uint32_t m2 = 0;
    const __nv_bfloat16* rbase = base + row * stride_m;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const uint32_t i = threadIdx.x + static_cast<uint32_t>(k) * THREADS;
      if (i < nvec) {
        const __nv_bfloat16* src;
        if (SEGMENTED) {
          const uint32_t sg = i / static_cast<uint32_t>(segv);
          src = rbase + sg * stride_p + static_cast<int64_t>(i - sg * static_cast<uint32_t>(segv)) * 8;
        } else {
          src = rbase + static_cast<int64_t>(i) * 8;
        }
        h[k] = __ldg(reinterpret_cast<const uint4*>(src));
        m2 = absmax8(h[k], m2);
      } else {
        h[k] = make_uint4(0, 0, 0, 0);
      }
    }
    quant_tail<THREADS, VPT>(h, m2, nvec, q + row * nvec * 8, s + row, div_mode, red);
  }
}

// any alignment / width: two passes over global memory (second pass hits L1/L2)
__global__ void __launch_bounds__(256) quant_rows_scalar_kernel(const __nv_bfloat16* __restrict__ base, int64_t m,
                                                                int64_t seg, int64_t p, int64_t stride_p,
                                                                int64_t stride_m, uint8_t* __restrict__ q,
                                                                float* __restrict__ s, int div_mode) {
  __shared__ float red[33];
  const int64_t K = p * seg;
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    float amax = 0.0f;
    for (int64_t j = threadIdx.x; j < K; j += 256) {
      const int64_t sg = j / seg, c = j - sg * seg;
      amax = nan_max(amax, fabsf(__bfloat162float(base[sg * stride_p + row * stride_m + c])));
    }
    amax = block_max_nan<256>(amax, red);
    const float scale = nan_max(qdiv(amax, kFp8Max, div_mode), kMinScale);
    const float inv = qdiv(1.0f, scale, div_mode);
    for (int64_t j = threadIdx.x; j < K; j += 256) {
      const int64_t sg = j / seg, c = j - sg * seg;
      const float y = __bfloat162float(base[sg * stride_p + row * stride_m + c]) * inv;
      q[row * K + j] = static_cast<uint8_t>(f32x2_to_e4m3x2(y, 0.0f) & 0xFF);
    }
    if (threadIdx.x == 0) s[row] = scale;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------------------------
// K7: RMSNorm (+ AdaLN modulation) + quant      (fp8_quant_fuse._rms_norm_indexed_scale_shift_quant_kernel)
// K8: gated residual + RMSNorm + modulation + quant (_indexed_gate_rms_norm_scale_shift_quant_kernel)
// ---------------------------------------------------------------------------------------------------------------
struct RmsArgs {
  const __nv_bfloat16* x;  // K7: x; K8: residual
  int64_t stride_x;
  const __nv_bfloat16* gate;  // K8 only
  int64_t stride_gate;
  const __nv_bfloat16* branch;  // K8 only
  int64_t stride_branch;
  const __nv_bfloat16* weight;
  const __nv_bfloat16* shift;
  int64_t stride_shift;
  const __nv_bfloat16* scale;
  int64_t stride_scale;
  const int64_t* indices;
  int64_t rows, hidden;
  float eps;
  __nv_bfloat16* ph;            // optional bf16 copy of the modulated row
  __nv_bfloat16* residual_out;  // K8
  uint8_t* q;
  float* s;
  int div_mode;
};

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = lo_bf16(w[i]);
    f[2 * i + 1] = hi_bf16(w[i]);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

template <int THREADS, int VPT, bool GATED>
__global__ void __launch_bounds__(THREADS) rms_quant_kernel(RmsArgs a) {
  __shared__ float red[33];
  __shared__ uint32_t redu[33];
  const int64_t nvec = a.hidden / 8;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t idx = a.indices != nullptr ? a.indices[row] : 0;
    uint4 xv[VPT];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * THREADS;
      xv[k] = make_uint4(0, 0, 0, 0);
      if (i < nvec) {
        float x[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.x + row * a.stride_x) + i), x);
        if (GATED) {
          float g[8], b[8];
          unpack8(__ldg(reinterpret_cast<const uint4*>(a.gate + idx * a.stride_gate) + i), g);
          unpack8(__ldg(reinterpret_cast<const uint4*>(a.branch + row * a.stride_branch) + i), b);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = fmaf(g[e], b[e], x[e]);
          xv[k] = pack8(x);  // the bf16 residual value
          *reinterpret_cast<uint4*>(a.residual_out + row * a.hidden + i * 8) = xv[k];
          unpack8(xv[k], x);
        } else {
          xv[k] = __ldg(reinterpret_cast<const uint4*>(a.x + row * a.stride_x) + i);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
      }
    }
    const float var = __fdiv_rn(block_sum<THREADS>(ss, red), static_cast<float>(a.hidden));
    const float rstd = rsqrtf(var + a.eps);
    uint32_t m2 = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * THREADS;
      if (i < nvec) {
        float x[8], w[8];
        unpack8(xv[k], x);
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.weight) + i), w);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = x[e] * rstd * w[e];
        if (a.shift != nullptr) {
          float sh[8], sc[8];
          unpack8(__ldg(reinterpret_cast<const uint4*>(a.shift + idx * a.stride_shift) + i), sh);
          unpack8(__ldg(reinterpret_cast<const uint4*>(a.scale + idx * a.stride_scale) + i), sc);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = fmaf(x[e], 1.0f + sc[e], sh[e]);
        }
        xv[k] = pack8(x);
        if (a.ph != nullptr) *reinterpret_cast<uint4*>(a.ph + row * a.hidden + i * 8) = xv[k];
        m2 = absmax8(xv[k], m2);
      }
    }
    quant_tail<THREADS, VPT>(xv, m2, nvec, a.q + row * a.hidden, a.s + row, a.div_mode, redu);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// K11: SiLU-mul + quant (fp8_quant_fuse._silu_mul_quant_kernel; vLLM act_and_mul arithmetic)
// K5 : SwiGLU scale pass (+ quant) over the fp32 fc1 product (fp8_swiglu._scale_swiglu / _scale_swiglu_quant)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// silu(g) rounded to bf16, times u (-0 -> +0), rounded to bf16: the bf16 silu_and_mul output as fp32
__device__ __forceinline__ float silu_mul(float g, float u) {
  u = (u == 0.0f) ? fabsf(u) : u;
  const float s = round_bf16(__fdiv_rn(g, 1.0f + expf(-g)));
  return s * u;
}

template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                                 int64_t d, int64_t stride_x, uint8_t* __restrict__ q,
                                                                 float* __restrict__ s, int div_mode) {
  __shared__ uint32_t red[33];
  const int64_t nvec = d / 8;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    uint4 h[VPT];
    uint32_t m2 = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * THREADS;
      h[k] = make_uint4(0, 0, 0, 0);
      if (i < nvec) {
        float g[8], u[8], y[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(x + row * stride_x) + i), g);
        unpack8(__ldg(reinterpret_cast<const uint4*>(x + row * stride_x + d) + i), u);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = silu_mul(g[e], u[e]);
        h[k] = pack8(y);
        m2 = absmax8(h[k], m2);
      }
    }
    quant_tail<THREADS, VPT>(h, m2, nvec, q + row * d, s + row, div_mode, red);
  }
}

// fp32 product -> bf16 gate/up (fp8_gemm epilogue arithmetic, then bf16 rounding) -> silu * up.  VEC: sb (and bias)
// are 16-byte aligned and read as vectors; otherwise element by element (same values, same arithmetic)
template <bool VEC>
__device__ __forceinline__ void swiglu8(const float* xr, int64_t half, int64_t c, float sa, const float* sb,
                                        const __nv_bfloat16* bias, float (&y)[8]) {
  const float4 g0 = __ldcs(reinterpret_cast<const float4*>(xr + c));
  const float4 g1 = __ldcs(reinterpret_cast<const float4*>(xr + c + 4));
  const float4 u0 = __ldcs(reinterpret_cast<const float4*>(xr + half + c));
  const float4 u1 = __ldcs(reinterpret_cast<const float4*>(xr + half + c + 4));
  const float ga[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float ua[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  float sg[8], su[8], bg[8], bu[8];
  if (VEC) {
    const float4 a0 = __ldg(reinterpret_cast<const float4*>(sb + c));
    const float4 a1 = __ldg(reinterpret_cast<const float4*>(sb + c + 4));
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(sb + half + c));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(sb + half + c + 4));
    const float sgv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float suv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sg[e] = sgv[e];
      su[e] = suv[e];
    }
    if (bias != nullptr) {
      unpack8(__ldg(reinterpret_cast<const uint4*>(bias + c)), bg);
      unpack8(__ldg(reinterpret_cast<const uint4*>(bias + half + c)), bu);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sg[e] = __ldg(sb + c + e);
      su[e] = __ldg(sb + half + c + e);
      if (bias != nullptr) {
        bg[e] = __bfloat162float(bias[c + e]);
        bu[e] = __bfloat162float(bias[half + c + e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float g = sg[e] * ga[e];
    float u = su[e] * ua[e];
    if (bias != nullptr) {
      g = fmaf(sa, g, bg[e]);
      u = fmaf(sa, u, bu[e]);
    } else {
      g = sa * g;
      u = sa * u;
    }
    y[e] = silu_mul(round_bf16(g), round_bf16(u));
  }
}

template <int THREADS, int VPT, bool VEC>
__global__ void __launch_bounds__(THREADS) scale_swiglu_quant_kernel(const float* __restrict__ x,
                                                                     const float* __restrict__ sa,
                                                                     const float* __restrict__ sb,
                                                                     const __nv_bfloat16* __restrict__ bias, int64_t M,
                                                                     int64_t half, uint8_t* __restrict__ q,
                                                                     float* __restrict__ s, int div_mode) {
  __shared__ uint32_t red[33];
  const int64_t nvec = half / 8;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const float sar = sa[row];
    uint4 h[VPT];
    uint32_t m2 = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * THREADS;
      h[k] = make_uint4(0, 0, 0, 0);
      if (i < nvec) {
        float y[8];
        swiglu8<VEC>(x + row * 2 * half, half, i * 8, sar, sb, bias, y);
        h[k] = pack8(y);
        m2 = absmax8(h[k], m2);
      }
    }
    quant_tail<THREADS, VPT>(h, m2, nvec, q + row * half, s + row, div_mode, red);
  }
}

template <bool VEC>
__global__ void scale_swiglu_kernel(const float* __restrict__ x, const float* __restrict__ sa,
                                    const float* __restrict__ sb, const __nv_bfloat16* __restrict__ bias, int64_t M,
                                    int64_t half, __nv_bfloat16* __restrict__ y) {
  const int64_t nvec = half / 8;
  const int64_t total = M * nvec;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = t / nvec, i = t - row * nvec;
    float o[8];
    swiglu8<VEC>(x + row * 2 * half, half, i * 8, sa[row], sb, bias, o);
    *reinterpret_cast<uint4*>(y + row * half + i * 8) = pack8(o);
  }
}

// K2: two-pass scale epilogue y = out(sa * (sb * x)) (+ bias by fma)
template <bool BF16_OUT>
__global__ void scale_bias_cast_kernel(const float* __restrict__ x, const float* __restrict__ sa,
                                       const float* __restrict__ sb, const __nv_bfloat16* __restrict__ bias,
                                       void* __restrict__ y, int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = t / N, col = t - row * N;
    const float tv = __ldg(sb + col) * x[t];
    const float v = bias != nullptr ? fmaf(sa[row], tv, __bfloat162float(bias[col])) : sa[row] * tv;
    if (BF16_OUT)
      reinterpret_cast<__nv_bfloat16*>(y)[t] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<__half*>(y)[t] = __float2half_rn(v);
  }
}

// the same arithmetic 8 columns at a time: x read as two streaming 16-byte loads, sb and bias as 16-byte loads,
// y written as one 16-byte store (N % 8 == 0, every pointer 16-byte aligned)
template <bool BF16_OUT>
__global__ void scale_bias_cast_vec_kernel(const float* __restrict__ x, const float* __restrict__ sa,
                                           const float* __restrict__ sb, const __nv_bfloat16* __restrict__ bias,
                                           void* __restrict__ y, int64_t M, int64_t nvec) {
  const int64_t total = M * nvec;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = t / nvec, i = t - row * nvec;
    const float4 x0 = __ldcs(reinterpret_cast<const float4*>(x) + 2 * t);
    const float4 x1 = __ldcs(reinterpret_cast<const float4*>(x) + 2 * t + 1);
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(sb) + 2 * i);
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(sb) + 2 * i + 1);
    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const float sar = __ldg(sa + row);
    float bb[8];
    if (bias != nullptr) unpack8(__ldg(reinterpret_cast<const uint4*>(bias) + i), bb);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float tv = bv[e] * xv[e];
      v[e] = bias != nullptr ? fmaf(sar, tv, bb[e]) : sar * tv;
    }
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (BF16_OUT) {
        w[k] = pack_bf16x2(v[2 * k], v[2 * k + 1]);
      } else {
        __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    __stcs(reinterpret_cast<uint4*>(y) + t, make_uint4(w[0], w[1], w[2], w[3]));
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Ulysses layout kernels (16-byte granules)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v, int32_t* range_flag) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = lo_bf16(w[i]), b = hi_bf16(w[i]);
    bad |= (fabsf(a) > 65504.0f && isfinite(a)) || (fabsf(b) > 65504.0f && isfinite(b));
    __half2 h = __floats2half2_rn(a, b);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  if (bad && range_flag != nullptr) atomicExch(range_flag, 1);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void pack_by_dest_kernel(const uint16_t* __restrict__ x, int64_t m, int32_t hl, int32_t dv,
                                    int64_t stride_m, int64_t stride_h, int32_t ws, uint16_t* __restrict__ send,
                                    int to_f16, int32_t* range_flag) {
  // send [P, M, hl, d] in 8-element granules; dv = d / 8
  const int64_t total = static_cast<int64_t>(ws) * m * hl * dv;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = t;
    const int64_t cv = r % dv;
    r /= dv;
    const int64_t j = r % hl;
    r /= hl;
    const int64_t mm = r % m;
    const int64_t p = r / m;
    uint4 v = __ldg(reinterpret_cast<const uint4*>(x + mm * stride_m + (p * hl + j) * stride_h + cv * 8));
    if (to_f16) v = bf16x8_to_f16x8(v, range_flag);
    reinterpret_cast<uint4*>(send)[t] = v;
  }
}

__global__ void unpack_recv_kernel(const uint16_t* __restrict__ recv, int32_t ws, int64_t m, int32_t hl, int32_t dv,
                                   uint16_t* __restrict__ out) {
  // out [M, P, hl, d] granule t -> recv [P, M, hl, d]
  const int64_t total = static_cast<int64_t>(ws) * m * hl * dv;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = t;
    const int64_t cv = r % dv;
    r /= dv;
    const int64_t j = r % hl;
    r /= hl;
    const int64_t p = r % ws;
    const int64_t mm = r / ws;
    reinterpret_cast<uint4*>(out)[t] = __ldg(reinterpret_cast<const uint4*>(recv) + ((p * m + mm) * hl + j) * dv + cv);
  }
}

__global__ void bf16_to_f16_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, int64_t nvec,
                                   int32_t* range_flag) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < nvec;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[t] = bf16x8_to_f16x8(__ldg(x + t), range_flag);
}


// ---------------------------------------------------------------------------------------------------------------
// qk RMSNorm + partial RoPE per (token, head) row, written into the Ulysses send layout (rope_into_send producer)
// ---------------------------------------------------------------------------------------------------------------
__global__ void norm_rope_send_kernel(const uint16_t* __restrict__ x, int64_t m, int heads, int64_t stride_m,
                                      int64_t stride_h, const __nv_bfloat16* __restrict__ w,
                                      const float* __restrict__ table, int64_t tstride, int rot, float eps, int hl,
                                      uint16_t* __restrict__ send) {
  // a warp per token: the RoPE factors of the lane's 4 elements are read once and reused for every head; the heads
  // go 4 at a time so that their loads are in flight together
  constexpr int HU = 4;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int half = rot >> 1;
  const int e0 = 4 * lane;  // this lane's 4 elements of the 128
  const bool first = e0 < half, second = e0 >= half && e0 < rot;
  const int src = first ? lane + (half >> 2) : (second ? lane - (half >> 2) : lane);
  float wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = __bfloat162float(w[e0 + i]);
  for (int64_t mm = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; mm < m; mm += warps) {
    float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    const float* trow = table + mm * tstride;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (first) {
        cs[i] = __ldg(trow + e0 + i);
        sn[i] = __ldg(trow + half + e0 + i);
      } else if (second) {
        cs[i] = __ldg(trow + e0 - half + i);
        sn[i] = __ldg(trow + e0 + i);
      }
    }
    const uint16_t* xrow = x + mm * stride_m + e0;
    for (int h0 = 0; h0 < heads; h0 += HU) {
      uint2 raw[HU];
#pragma unroll
      for (int u = 0; u < HU; ++u)
        raw[u] = (h0 + u < heads) ? __ldg(reinterpret_cast<const uint2*>(xrow + (h0 + u) * stride_h)) : make_uint2(0, 0);
#pragma unroll
      for (int u = 0; u < HU; ++u) {
        const int h = h0 + u;
        if (h >= heads) break;  // warp-uniform
        float f[4] = {lo_bf16(raw[u].x), hi_bf16(raw[u].x), lo_bf16(raw[u].y), hi_bf16(raw[u].y)};
        float ss = __fmul_rn(f[0], f[0]);
#pragma unroll
        for (int i = 1; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(f[i], f[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(__fadd_rn(ss * (1.0f / 128.0f), eps));
        float n[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) n[i] = round_bf16(__fmul_rn(__fmul_rn(f[i], inv), wv[i]));
        // rotation partner: element e pairs with e + half (first half) or e - half (second half of the rotated dims)
        float pn[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pn[i] = __shfl_sync(0xffffffffu, n[i], src);
        float out[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (first)
            out[i] = __fsub_rn(__fmul_rn(n[i], cs[i]), __fmul_rn(pn[i], sn[i]));  // a cos - b sin
          else if (second)
            out[i] = __fadd_rn(__fmul_rn(n[i], cs[i]), __fmul_rn(pn[i], sn[i]));  // b cos + a sin
          else
            out[i] = n[i];
        }
        const int p = h / hl, j = h - p * hl;
        uint2 o;
        o.x = pack_bf16x2(out[0], out[1]);
        o.y = pack_bf16x2(out[2], out[3]);
        *reinterpret_cast<uint2*>(send + ((static_cast<int64_t>(p) * m + mm) * hl + j) * 128 + e0) = o;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------------------------------
static inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static inline int grid_rows(int64_t rows) {
  return static_cast<int>(rows < (1ll << 30) ? rows : (1ll << 30));
}
static inline int grid_elems(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

// VPT choices for 256-thread CTAs: widths up to 256 * 8 * 16 = 32768 elements
// the same for CTAs of 128 threads, with every VPT up to 6 and 10 (a row of 5120 is 128 x 5 vectors exactly)
#define H3B_VPT128_DISPATCH(NVEC, LAUNCH)     \
  do {                                        \
    const int64_t per_ = ((NVEC) + 127) / 128; \
    if (per_ <= 1) { LAUNCH(1); }             \
    else if (per_ <= 2) { LAUNCH(2); }        \
    else if (per_ <= 3) { LAUNCH(3); }        \
    else if (per_ <= 4) { LAUNCH(4); }        \
    else if (per_ <= 5) { LAUNCH(5); }        \
    else if (per_ <= 6) { LAUNCH(6); }        \
    else if (per_ <= 8) { LAUNCH(8); }        \
    else if (per_ <= 10) { LAUNCH(10); }      \
    else if (per_ <= 12) { LAUNCH(12); }      \
    else { LAUNCH(16); }                      \
  } while (0)

#define H3B_VPT_DISPATCH(NVEC, LAUNCH)        \
  do {                                        \
    const int64_t per_ = ((NVEC) + 255) / 256; \
    if (per_ <= 1) { LAUNCH(1); }             \
    else if (per_ <= 2) { LAUNCH(2); }        \
    else if (per_ <= 3) { LAUNCH(3); }        \
    else if (per_ <= 4) { LAUNCH(4); }        \
    else if (per_ <= 6) { LAUNCH(6); }        \
    else if (per_ <= 8) { LAUNCH(8); }        \
    else if (per_ <= 12) { LAUNCH(12); }      \
    else { LAUNCH(16); }                      \
  } while (0)

}  // namespace h3b

using namespace h3b;

extern "C" {

int h3b_quant_rows_e4m3(const void* base, int64_t m, int32_t p, int64_t seg, int64_t stride_p, int64_t stride_m,
                        void* q, float* scale, int32_t div_mode, h3b_stream_t stream) {
  if (m < 0 || p < 1 || seg < 0) return fail(H3B_EINVAL, "quant_rows: m %lld p %d seg %lld", (long long)m, p, (long long)seg);
  if (div_mode != H3B_DIV_IEEE && div_mode != H3B_DIV_FULL) return fail(H3B_EINVAL, "quant_rows: div_mode %d", div_mode);
  if (m == 0 || seg == 0) return H3B_OK;
  if (base == nullptr || q == nullptr || scale == nullptr) return fail(H3B_EINVAL, "quant_rows: null pointer");
  const int64_t K = static_cast<int64_t>(p) * seg;
  const auto* b = static_cast<const __nv_bfloat16*>(base);
  auto* qq = static_cast<uint8_t*>(q);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = seg % 8 == 0 && stride_p % 8 == 0 && stride_m % 8 == 0 && al16(base) && al16(q) &&
                   K <= 256 * 8 * 16;
  if (vec) {
    const int64_t nvec = K / 8, segv = seg / 8;
    if (p == 1) {
#define L(V) quant_rows_vec_kernel<256, V, false><<<grid_rows(m), 256, 0, st>>>(b, m, segv, stride_p, stride_m, nvec, qq, scale, div_mode)
      H3B_VPT_DISPATCH(nvec, L);
#undef L
    } else {
#define L(V) quant_rows_vec_kernel<256, V, true><<<grid_rows(m), 256, 0, st>>>(b, m, segv, stride_p, stride_m, nvec, qq, scale, div_mode)
      H3B_VPT_DISPATCH(nvec, L);
#undef L
    }
  } else {
    quant_rows_scalar_kernel<<<grid_rows(m), 256, 0, st>>>(b, m, seg, p, stride_p, stride_m, qq, scale, div_mode);
  }
  H3B_CHECK_LAUNCH("quant_rows launch");
  return H3B_OK;
}

static int rms_common(RmsArgs& a, bool gated, cudaStream_t st) {
  if (a.rows < 0 || a.hidden <= 0) return fail(H3B_EINVAL, "rms_quant: rows %lld hidden %lld", (long long)a.rows, (long long)a.hidden);
  if (a.div_mode != H3B_DIV_IEEE && a.div_mode != H3B_DIV_FULL) return fail(H3B_EINVAL, "rms_quant: div_mode");
  if (a.rows == 0) return H3B_OK;
  if (a.x == nullptr || a.weight == nullptr || a.q == nullptr || a.s == nullptr) return fail(H3B_EINVAL, "rms_quant: null pointer");
  if ((a.shift == nullptr) != (a.scale == nullptr)) return fail(H3B_EINVAL, "rms_quant: shift and scale go together");
  if (gated && (a.gate == nullptr || a.branch == nullptr || a.residual_out == nullptr))
    return fail(H3B_EINVAL, "gate_rms_quant: null pointer");
  if (a.hidden % 8 || a.stride_x % 8 || (gated && (a.stride_gate % 8 || a.stride_branch % 8)) ||
      (a.shift && (a.stride_shift % 8 || a.stride_scale % 8)) || !al16(a.x) || !al16(a.weight) || !al16(a.q) ||
      (a.shift && (!al16(a.shift) || !al16(a.scale))) || (a.ph && !al16(a.ph)) ||
      (gated && (!al16(a.gate) || !al16(a.branch) || !al16(a.residual_out))))
    return fail(H3B_EALIGN, "rms_quant: rows, strides and pointers must be 16-byte granular");
  const int64_t nvec = a.hidden / 8;
  if (nvec > 256 * 16) return fail(H3B_EUNSUPPORTED, "rms_quant: hidden %lld above 32768", (long long)a.hidden);
  // A CTA of 128 threads per row (rows up to 16,384 wide): measured against 256 threads at 62,496 x 5120, 0.240 against
  // 0.304 ms (K7) and 0.407 against 0.473 ms (K8, then a persistent kernel streaming rows through shared memory); 512
  // threads and one warp per row were slower.  More, smaller CTAs keep more rows in flight per SM and shorten each
  // row's two block reductions.
  if (nvec <= 128 * 16) {
    if (gated) {
#define L(V) rms_quant_kernel<128, V, true><<<grid_rows(a.rows), 128, 0, st>>>(a)
      H3B_VPT128_DISPATCH(nvec, L);
#undef L
    } else {
#define L(V) rms_quant_kernel<128, V, false><<<grid_rows(a.rows), 128, 0, st>>>(a)
      H3B_VPT128_DISPATCH(nvec, L);
#undef L
    }
  } else if (gated) {
#define L(V) rms_quant_kernel<256, V, true><<<grid_rows(a.rows), 256, 0, st>>>(a)
    H3B_VPT_DISPATCH(nvec, L);
#undef L
  } else {
#define L(V) rms_quant_kernel<256, V, false><<<grid_rows(a.rows), 256, 0, st>>>(a)
    H3B_VPT_DISPATCH(nvec, L);
#undef L
  }
  H3B_CHECK_LAUNCH("rms_quant launch");
  return H3B_OK;
}

int h3b_rms_quant_e4m3(const void* x, int64_t rows, int64_t hidden, int64_t stride_x, const void* weight,
                       const void* shift, int64_t stride_shift, const void* scale, int64_t stride_scale,
                       const int64_t* indices, float eps, void* ph, void* q, float* s, int32_t div_mode,
                       h3b_stream_t stream) {
  RmsArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.stride_x = stride_x;
  a.weight = static_cast<const __nv_bfloat16*>(weight);
  a.shift = static_cast<const __nv_bfloat16*>(shift);
  a.stride_shift = stride_shift;
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.stride_scale = stride_scale;
  a.indices = indices;
  a.rows = rows;
  a.hidden = hidden;
  a.eps = eps;
  a.ph = static_cast<__nv_bfloat16*>(ph);
  a.q = static_cast<uint8_t*>(q);
  a.s = s;
  a.div_mode = div_mode;
  return rms_common(a, false, reinterpret_cast<cudaStream_t>(stream));
}

int h3b_gate_rms_quant_e4m3(const void* residual, int64_t stride_residual, const void* gate, int64_t stride_gate,
                            const void* branch, int64_t stride_branch, const void* weight, const void* shift,
                            int64_t stride_shift, const void* scale, int64_t stride_scale, const int64_t* indices,
                            int64_t rows, int64_t hidden, float eps, void* residual_out, void* q, float* s,
                            int32_t div_mode, h3b_stream_t stream) {
  RmsArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(residual);
  a.stride_x = stride_residual;
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.stride_gate = stride_gate;
  a.branch = static_cast<const __nv_bfloat16*>(branch);
  a.stride_branch = stride_branch;
  a.weight = static_cast<const __nv_bfloat16*>(weight);
  a.shift = static_cast<const __nv_bfloat16*>(shift);
  a.stride_shift = stride_shift;
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.stride_scale = stride_scale;
  a.indices = indices;
  a.rows = rows;
  a.hidden = hidden;
  a.eps = eps;
  a.residual_out = static_cast<__nv_bfloat16*>(residual_out);
  a.q = static_cast<uint8_t*>(q);
  a.s = s;
  a.div_mode = div_mode;
  return rms_common(a, true, reinterpret_cast<cudaStream_t>(stream));
}

int h3b_silu_mul_quant_e4m3(const void* x, int64_t rows, int64_t d, int64_t stride_x, void* q, float* s,
                            int32_t div_mode, h3b_stream_t stream) {
  if (rows < 0 || d <= 0) return fail(H3B_EINVAL, "silu_mul_quant: rows %lld d %lld", (long long)rows, (long long)d);
  if (div_mode != H3B_DIV_IEEE && div_mode != H3B_DIV_FULL) return fail(H3B_EINVAL, "silu_mul_quant: div_mode");
  if (rows == 0) return H3B_OK;
  if (x == nullptr || q == nullptr || s == nullptr) return fail(H3B_EINVAL, "silu_mul_quant: null pointer");
  if (d % 8 || stride_x % 8 || !al16(x) || !al16(q)) return fail(H3B_EALIGN, "silu_mul_quant: 16-byte granules needed");
  const int64_t nvec = d / 8;
  if (nvec > 256 * 16) return fail(H3B_EUNSUPPORTED, "silu_mul_quant: d above 32768");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qq = static_cast<uint8_t*>(q);
  if (nvec == 288 * 6) {
    // the DiT FFN width (13,824): 288 threads x 6 vectors cover the row exactly (0.288 against 0.308 ms with 256 x 8
    // at 15,624 rows; 192 x 9 and 576 x 3 were slower)
    silu_mul_quant_kernel<288, 6><<<grid_rows(rows), 288, 0, st>>>(xb, rows, d, stride_x, qq, s, div_mode);
  } else {
#define L(V) silu_mul_quant_kernel<256, V><<<grid_rows(rows), 256, 0, st>>>(xb, rows, d, stride_x, qq, s, div_mode)
    H3B_VPT_DISPATCH(nvec, L);
#undef L
  }
  H3B_CHECK_LAUNCH("silu_mul_quant launch");
  return H3B_OK;
}

int h3b_scale_bias_cast(const float* x, const float* sa, const float* sb, const void* bias, void* y, int64_t M,
                        int64_t N, int32_t out_dtype, h3b_stream_t stream) {
  if (M < 0 || N < 0) return fail(H3B_EINVAL, "scale_bias_cast: M %lld N %lld", (long long)M, (long long)N);
  if (out_dtype != H3B_OUT_BF16 && out_dtype != H3B_OUT_F16) return fail(H3B_EINVAL, "scale_bias_cast: out dtype");
  if (M == 0 || N == 0) return H3B_OK;
  if (x == nullptr || sa == nullptr || sb == nullptr || y == nullptr) return fail(H3B_EINVAL, "scale_bias_cast: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* bb = static_cast<const __nv_bfloat16*>(bias);
  const bool vec = N % 8 == 0 && al16(x) && al16(sb) && al16(y) && (bias == nullptr || al16(bias));
  if (vec && out_dtype == H3B_OUT_BF16)
    scale_bias_cast_vec_kernel<true><<<grid_elems(M * (N / 8), 256), 256, 0, st>>>(x, sa, sb, bb, y, M, N / 8);
  else if (vec)
    scale_bias_cast_vec_kernel<false><<<grid_elems(M * (N / 8), 256), 256, 0, st>>>(x, sa, sb, bb, y, M, N / 8);
  else if (out_dtype == H3B_OUT_BF16)
    scale_bias_cast_kernel<true><<<grid_elems(M * N, 256), 256, 0, st>>>(x, sa, sb, bb, y, M, N);
  else
    scale_bias_cast_kernel<false><<<grid_elems(M * N, 256), 256, 0, st>>>(x, sa, sb, bb, y, M, N);
  H3B_CHECK_LAUNCH("scale_bias_cast launch");
  return H3B_OK;
}

int h3b_scale_swiglu(const float* x, const float* sa, const float* sb, const void* bias, void* y, int64_t M,
                     int64_t half, h3b_stream_t stream) {
  if (M < 0 || half < 0) return fail(H3B_EINVAL, "scale_swiglu: M %lld half %lld", (long long)M, (long long)half);
  if (M == 0 || half == 0) return H3B_OK;
  if (x == nullptr || sa == nullptr || sb == nullptr || y == nullptr) return fail(H3B_EINVAL, "scale_swiglu: null pointer");
  if (half % 8 || !al16(x) || !al16(y)) return fail(H3B_EALIGN, "scale_swiglu: half must be a multiple of 8, 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* bb = static_cast<const __nv_bfloat16*>(bias);
  auto* yy = static_cast<__nv_bfloat16*>(y);
  if (al16(sb) && (bias == nullptr || al16(bias)))
    scale_swiglu_kernel<true><<<grid_elems(M * (half / 8), 256), 256, 0, st>>>(x, sa, sb, bb, M, half, yy);
  else
    scale_swiglu_kernel<false><<<grid_elems(M * (half / 8), 256), 256, 0, st>>>(x, sa, sb, bb, M, half, yy);
  H3B_CHECK_LAUNCH("scale_swiglu launch");
  return H3B_OK;
}

int h3b_scale_swiglu_quant(const float* x, const float* sa, const float* sb, const void* bias, void* q, float* s,
                           int64_t M, int64_t half, int32_t div_mode, h3b_stream_t stream) {
  if (M < 0 || half < 0) return fail(H3B_EINVAL, "scale_swiglu_quant: M %lld half %lld", (long long)M, (long long)half);
  if (div_mode != H3B_DIV_IEEE && div_mode != H3B_DIV_FULL) return fail(H3B_EINVAL, "scale_swiglu_quant: div_mode");
  if (M == 0 || half == 0) return H3B_OK;
  if (x == nullptr || sa == nullptr || sb == nullptr || q == nullptr || s == nullptr)
    return fail(H3B_EINVAL, "scale_swiglu_quant: null pointer");
  if (half % 8 || !al16(x) || !al16(q)) return fail(H3B_EALIGN, "scale_swiglu_quant: half % 8 and 16-byte alignment");
  const int64_t nvec = half / 8;
  if (nvec > 256 * 16) return fail(H3B_EUNSUPPORTED, "scale_swiglu_quant: half above 32768");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* bb = static_cast<const __nv_bfloat16*>(bias);
  auto* qq = static_cast<uint8_t*>(q);
  if (al16(sb) && (bias == nullptr || al16(bias))) {
    if (nvec == 288 * 6) {  // the DiT FFN width: 288 x 6 covers it exactly (0.560 against 0.594 ms)
      scale_swiglu_quant_kernel<288, 6, true><<<grid_rows(M), 288, 0, st>>>(x, sa, sb, bb, M, half, qq, s, div_mode);
    } else {
#define L(V) scale_swiglu_quant_kernel<256, V, true><<<grid_rows(M), 256, 0, st>>>(x, sa, sb, bb, M, half, qq, s, div_mode)
      H3B_VPT_DISPATCH(nvec, L);
#undef L
    }
  } else {
#define L(V) scale_swiglu_quant_kernel<256, V, false><<<grid_rows(M), 256, 0, st>>>(x, sa, sb, bb, M, half, qq, s, div_mode)
    H3B_VPT_DISPATCH(nvec, L);
#undef L
  }
  H3B_CHECK_LAUNCH("scale_swiglu_quant launch");
  return H3B_OK;
}

int h3b_pack_by_dest(const void* x, int64_t m, int32_t heads, int32_t d, int64_t stride_m, int64_t stride_h,
                     int32_t ws, void* send, int32_t to_f16, int32_t* range_flag, h3b_stream_t stream) {
  if (m < 0 || heads <= 0 || d <= 0 || ws <= 0 || heads % ws) return fail(H3B_EINVAL, "pack_by_dest: bad shape");
  if (m == 0) return H3B_OK;
  if (x == nullptr || send == nullptr) return fail(H3B_EINVAL, "pack_by_dest: null pointer");
  if (d % 8 || stride_m % 8 || stride_h % 8 || !al16(x) || !al16(send)) return fail(H3B_EALIGN, "pack_by_dest: 16-byte granules");
  const int64_t total = static_cast<int64_t>(ws) * m * (heads / ws) * (d / 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pack_by_dest_kernel<<<grid_elems(total, 256), 256, 0, st>>>(static_cast<const uint16_t*>(x), m, heads / ws, d / 8,
                                                              stride_m, stride_h, ws, static_cast<uint16_t*>(send),
                                                              to_f16, range_flag);
  H3B_CHECK_LAUNCH("pack_by_dest launch");
  return H3B_OK;
}

int h3b_norm_rope_send(const void* x, int64_t m, int32_t heads, int64_t stride_m, int64_t stride_h,
                       const void* weight, const float* table, int64_t table_stride, int32_t rot, float eps,
                       int32_t ws, void* send, h3b_stream_t stream) {
  if (m < 0 || heads <= 0 || ws <= 0 || heads % ws) return fail(H3B_EINVAL, "norm_rope_send: bad shape");
  if (rot < 0 || rot > 128 || rot % 8) return fail(H3B_EUNSUPPORTED, "norm_rope_send: rot %d (multiple of 8, <= 128)", rot);
  if (m == 0) return H3B_OK;
  if (x == nullptr || weight == nullptr || send == nullptr || (rot > 0 && table == nullptr))
    return fail(H3B_EINVAL, "norm_rope_send: null pointer");
  if (stride_m % 4 || stride_h % 4 || (reinterpret_cast<uintptr_t>(x) & 7u) || (reinterpret_cast<uintptr_t>(send) & 7u))
    return fail(H3B_EALIGN, "norm_rope_send: 8-byte granules needed");
  const int64_t warps = m;  // a warp per token
  const int threads = 256;
  int64_t blocks = (warps * 32 + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  norm_rope_send_kernel<<<static_cast<int>(blocks), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), m, heads, stride_m, stride_h, static_cast<const __nv_bfloat16*>(weight), table,
      table_stride, rot, eps, heads / ws, static_cast<uint16_t*>(send));
  H3B_CHECK_LAUNCH("norm_rope_send launch");
  return H3B_OK;
}

int h3b_unpack_recv(const void* recv, int32_t ws, int64_t m, int32_t hl, int32_t d, void* out, h3b_stream_t stream) {
  if (m < 0 || hl <= 0 || d <= 0 || ws <= 0) return fail(H3B_EINVAL, "unpack_recv: bad shape");
  if (m == 0) return H3B_OK;
  if (recv == nullptr || out == nullptr) return fail(H3B_EINVAL, "unpack_recv: null pointer");
  if (d % 8 || !al16(recv) || !al16(out)) return fail(H3B_EALIGN, "unpack_recv: 16-byte granules");
  const int64_t total = static_cast<int64_t>(ws) * m * hl * (d / 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unpack_recv_kernel<<<grid_elems(total, 256), 256, 0, st>>>(static_cast<const uint16_t*>(recv), ws, m, hl, d / 8,
                                                             static_cast<uint16_t*>(out));
  H3B_CHECK_LAUNCH("unpack_recv launch");
  return H3B_OK;
}

int h3b_bf16_to_f16(const void* x, void* y, int64_t n, int32_t* range_flag, h3b_stream_t stream) {
  if (n < 0) return fail(H3B_EINVAL, "bf16_to_f16: n < 0");
  if (n == 0) return H3B_OK;
  if (x == nullptr || y == nullptr) return fail(H3B_EINVAL, "bf16_to_f16: null pointer");
  if (n % 8 || !al16(x) || !al16(y)) return fail(H3B_EALIGN, "bf16_to_f16: n % 8 and 16-byte alignment");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bf16_to_f16_kernel<<<grid_elems(n / 8, 256), 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<uint4*>(y),
                                                             n / 8, range_flag);
  H3B_CHECK_LAUNCH("bf16_to_f16 launch");
  return H3B_OK;
}

}  // extern "C"
