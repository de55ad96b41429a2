/*
 * h3b.h -- C ABI of the B200-native (sm_100a) DiT attention-block hot path.
 *
 * The hot path is Ulysses sequence-parallel self-attention wrapped in online-FP8 projections, as served by the
 * h3_tp2 vLLM plugin.  Every entry point below replaces one kernel or op of that plugin; the comment above each names
 * the reference interface it stands in for (paths inside the knapcio/MiniMax-H3-2x-DGX-Spark-TP2 project).
 *
 * Conventions
 *  - Plain pointers and sizes only.  Element types are fixed per argument and written in the comment:
 *    bf16 = IEEE bfloat16, f16 = IEEE half, e4m3 = OCP FP8 E4M3 (torch.float8_e4m3fn), f32 = float.
 *  - Sizes and strides are in ELEMENTS unless the name ends in _bytes.  Row-major unless stated.
 *  - The caller owns and allocates every buffer (inputs, outputs, scratch).  No entry point allocates device memory
 *    except the one-time per-device status word (h3b_device_status) and cached TMA descriptors (host memory).
 *  - All work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).  Nothing synchronises.
 *  - Return value: 0 (H3B_OK) or a negative h3b_status.  h3b_last_error() gives a one-line reason for the last
 *    failure of the calling thread.  Argument errors are detected on the host before anything is enqueued.
 *  - Device-side waits are bounded: a kernel whose pipeline stalls past H3B_WAIT_TIMEOUT_NS records
 *    H3B_ETIMEOUT in the per-device status word and returns; h3b_device_status() reads and clears it.
 */
#ifndef H3B_H_
#define H3B_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define H3B_API __attribute__((visibility("default")))
#else
#define H3B_API
#endif

typedef struct CUstream_st* h3b_stream_t; /* == cudaStream_t */

#define H3B_MAX_RANKS 8 /* Ulysses ranks of one NVSwitch box */

enum h3b_status {
  H3B_OK = 0,
  H3B_EINVAL = -1,       /* bad shape, null pointer, negative size */
  H3B_EALIGN = -2,       /* pointer or stride alignment not supported by the kernel */
  H3B_EUNSUPPORTED = -3, /* valid request outside what the kernels implement (e.g. head_dim != 128) */
  H3B_ECUDA = -4,        /* a CUDA runtime/driver call failed (launch, descriptor encode, ...) */
  H3B_ETIMEOUT = -5,     /* a device-side bounded wait expired (pipeline stall, peer never signalled) */
  H3B_ERANGE = -6        /* input values outside the range the requested fast path handles exactly */
};

enum h3b_div_mode {
  H3B_DIV_IEEE = 0, /* correctly rounded fp32 division: the eager torch path (fp8_quant_fuse.quant_torch) */
  H3B_DIV_FULL = 1  /* PTX div.full.f32: the instruction Triton emits for `/` in the Inductor QuantFP8 kernel */
};

enum h3b_out_dtype { H3B_OUT_BF16 = 0, H3B_OUT_F16 = 1 };

/* FP8 GEMM epilogue kinds (h3b_fp8_gemm `epilogue`) */
enum h3b_epilogue_kind {
  H3B_EPI_PLAIN = 0,    /* y[m, n] = out(sa[m] * (sb[n] * acc)), bias by fma */
  H3B_EPI_QKV_SEND = 1, /* plain epilogue, stored straight into three Ulysses send buffers [P, M, H/P, d] */
  H3B_EPI_SWIGLU = 2    /* fc1: gate columns [0, F) and up columns [F, 2F) of W -> bf16 silu(gate) * up, y [M, F] */
};

/* Extra arguments of H3B_EPI_QKV_SEND.  Column n of the [M, 3*H*d] product is (which = n / (H*d), head
 * h = (n % (H*d)) / d, c = n % d).  With G head groups (groups <= 1: one group) of hg = H/G heads and
 * hgl = hg/P heads per rank and group, head h = g*hg + p*hgl + j is written to send[which][g][p][m][j][c]
 * (each send buffer [G, P, M, hgl, d]; G = 1 is stock's input_t [P, M, H/P, d]), so each group's all-to-all is one
 * contiguous equal-split exchange (the reference's head-group overlap, h3_tp2/ulysses_overlap.py:116-159).
 * v_f16 != 0 stores the v slab as f16 (bf16-rounded first, then converted exactly) for the f16 P.V attention. */
typedef struct h3b_qkv_send {
  void* send[3]; /* q, k, v send buffers, each [P, M, H/P, d] contiguous, bf16 (v: f16 if v_f16) */
  int32_t heads; /* H */
  int32_t head_dim; /* d, must be 128 */
  int32_t ws;    /* P (Ulysses degree), H % P == 0 */
  int32_t v_f16;
  int32_t* range_flag; /* device int or NULL: set to 1 when a finite v value overflows f16 (v_f16 only) */
  int32_t groups;      /* head groups G (0 or 1: none); H % (G * P) == 0 */
  /* optional qk RMSNorm + partial RoPE on q and k before the store (the upstream norm+RoPE producer fused, see
   * h3b_norm_rope_send): per (token, head) n = bf16(y * rsqrt(mean(y^2) + eps) * w) of the bf16 GEMM output y, then
   * the first `rot` dims rotate with rope_table[m] = cos | sin.  NULL weights: no norm (v is never normed).  The norm
   * epilogue has no bias term: a bias with norm weights returns H3B_EUNSUPPORTED. */
  const void* q_norm_weight; /* bf16 [128] */
  const void* k_norm_weight; /* bf16 [128] */
  const float* rope_table;   /* [M, rot] f32, row stride rope_stride */
  int64_t rope_stride;
  int32_t rot;               /* 0, 32, 64, 96 or 128 */
  float eps;
  /* optional peer-memory exchange (p2p != 0; groups must be 1; send[] and range_flag unused): destination rank p's
   * slab is stored straight into rank p's receive buffer peer_recv[p][which] ([P, M, H/P, d], slot `rank`), so the
   * forward all-to-all (h3_tp2/ulysses_exact.py:94 dist.all_to_all_single) never runs.  No reference counterpart. */
  int32_t p2p;
  int32_t rank;
  void* peer_recv[H3B_MAX_RANKS][3];
  int32_t* peer_range_flag[H3B_MAX_RANKS]; /* v_f16 overflow flag of each rank (replaces range_flag); an overflow
                                            * in any slab raises all of them, so every rank sees the same flag */
  /* qkv_interleaved != 0 (not with p2p): one send buffer send[0] = [G, P, M, 3, hgl, d] holding q, k, v of a token
   * side by side (the combined-exchange layout of h3_tp2/ulysses_nocopy.py:74-90; send[1], send[2] unused) */
  int32_t qkv_interleaved;
} h3b_qkv_send;

/* ---------------------------------------------------------------------------------------------------------------
 * library information
 * ------------------------------------------------------------------------------------------------------------- */
H3B_API int h3b_abi_version(void); /* 3: h3b_qkv_send gained the peer-memory fields (2) and qkv_interleaved (3); 4: the *_bf16v attention entry points and h3b_noalloc_status */
H3B_API const char* h3b_status_string(int status);
H3B_API const char* h3b_last_error(void);
/* Reads and clears the sticky device status word of the current device (0 or a negative h3b_status). Synchronises
 * the current device first. */
H3B_API int h3b_device_status(void);
/* Sets the device-side wait bound (nanoseconds, default 4e9). */
H3B_API int h3b_set_wait_timeout_ns(uint64_t ns);

/* ---------------------------------------------------------------------------------------------------------------
 * per-token dynamic FP8 quant (row kernels, HBM bound)
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces ulysses_outq.quant_rows (h3_tp2/ulysses_outq.py:109) and its Triton kernel _quant_rows_kernel (:74-93);
 * also serves fp8_quant_fuse.quant (h3_tp2/fp8_quant_fuse.py:318) with p = 1 and unpack_quant (:379) with the receive
 * buffer's strides.  Row m (0 <= m < M) is the concatenation over s < p of the `seg` bf16 elements at
 * base + s*stride_p + m*stride_m.  Writes q [M, p*seg] e4m3 contiguous and scale [M] f32:
 *   amax = max |x| (NaN propagates), scale = max(amax / 448, 1/(448*512)), q = e4m3_rn(clamp(x * (1/scale), +-448)). */
H3B_API int h3b_quant_rows_e4m3(const void* base, int64_t m, int32_t p, int64_t seg, int64_t stride_p, int64_t stride_m,
                        void* q, float* scale, int32_t div_mode, h3b_stream_t stream);

/* Replaces fp8_quant_fuse.rms_quant + _rms_norm_indexed_scale_shift_quant_kernel (h3_tp2/fp8_quant_fuse.py:144-188,
 * :330): RMSNorm (fp32) * weight, then AdaLN modulation `* (1 + scale[idx]) + shift[idx]` when shift/scale are
 * non-NULL (indices NULL = row i uses modulation row 0), rounded to bf16, then the per-token quant.  x [rows, hidden]
 * bf16 (row stride stride_x), weight [hidden] bf16, shift/scale bf16 rows.  If ph != NULL the bf16 row is also
 * stored there ([rows, hidden] contiguous). */
H3B_API int h3b_rms_quant_e4m3(const void* x, int64_t rows, int64_t hidden, int64_t stride_x, const void* weight,
                       const void* shift, int64_t stride_shift, const void* scale, int64_t stride_scale,
                       const int64_t* indices, float eps, void* ph, void* q, float* s, int32_t div_mode,
                       h3b_stream_t stream);

/* Replaces fp8_quant_fuse.gate_rms_quant + _indexed_gate_rms_norm_scale_shift_quant_kernel
 * (h3_tp2/fp8_quant_fuse.py:191-243, :350): residual_out = bf16(residual + gate[idx] * branch), then RMSNorm,
 * modulation and the per-token quant of the result.  All row tensors bf16 with the given row strides;
 * residual_out [rows, hidden] contiguous. */
H3B_API int h3b_gate_rms_quant_e4m3(const void* residual, int64_t stride_residual, const void* gate, int64_t stride_gate,
                            const void* branch, int64_t stride_branch, const void* weight, const void* shift,
                            int64_t stride_shift, const void* scale, int64_t stride_scale, const int64_t* indices,
                            int64_t rows, int64_t hidden, float eps, void* residual_out, void* q, float* s,
                            int32_t div_mode, h3b_stream_t stream);

/* Replaces fp8_quant_fuse.silu_mul_quant + _silu_mul_quant_kernel (h3_tp2/fp8_quant_fuse.py:263-278, :392):
 * x [rows, 2d] bf16 (row stride stride_x) -> silu_and_mul (vLLM arithmetic: silu rounded to bf16, bf16 product)
 * -> per-token quant: q [rows, d] e4m3, s [rows] f32. */
H3B_API int h3b_silu_mul_quant_e4m3(const void* x, int64_t rows, int64_t d, int64_t stride_x, void* q, float* s,
                            int32_t div_mode, h3b_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * scale passes over an fp32 GEMM product (the two-pass path's second pass)
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces fp8_gemm._scale_bias_cast (h3_tp2/fp8_gemm.py:38-54): y[m,n] = out(sa[m] * (sb[n] * x[m,n])) or
 * out(fma(sa[m], sb[n]*x[m,n], bias[n])).  x [M, N] f32, bias bf16 [N] or NULL, y [M, N] (out_dtype). */
H3B_API int h3b_scale_bias_cast(const float* x, const float* sa, const float* sb, const void* bias, void* y, int64_t M,
                        int64_t N, int32_t out_dtype, h3b_stream_t stream);

/* Replaces fp8_swiglu._scale_swiglu (h3_tp2/fp8_swiglu.py:48-70): x [M, 2*half] f32 product of fc1 ->
 * y [M, half] bf16 = bf16(bf16(g / (1 + exp(-g))) * u) with g, u the bf16-rounded epilogue of the gate/up halves. */
H3B_API int h3b_scale_swiglu(const float* x, const float* sa, const float* sb, const void* bias, void* y, int64_t M,
                     int64_t half, h3b_stream_t stream);

/* Replaces fp8_swiglu._scale_swiglu_quant (h3_tp2/fp8_swiglu.py:73-103): as h3b_scale_swiglu, then the per-token
 * quant of each SwiGLU row for fc2: q [M, half] e4m3, s [M] f32. */
H3B_API int h3b_scale_swiglu_quant(const float* x, const float* sa, const float* sb, const void* bias, void* q, float* s,
                           int64_t M, int64_t half, int32_t div_mode, h3b_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * FP8 GEMM (tcgen05 + TMEM + TMA), scaled epilogue fused
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces ops.cutlass_scaled_mm as routed by fp8_gemm._mm / route (h3_tp2/fp8_gemm.py:328-386) for per-token x
 * per-channel scales: scaled_mm_tensor32 (:149), the CuTe-DSL kernel fp8_cutlass.scaled_mm (h3_tp2/fp8_cutlass.py:115,
 * h3_tp2/fp8_cutlass_kernel.py:52) and, with H3B_EPI_SWIGLU, fp8_swiglu.gemm_swiglu (h3_tp2/fp8_swiglu.py:230).
 *   a [M, K] e4m3 (row stride lda), w [N, K] e4m3 (row stride ldw; the reference's b = w.t()),
 *   sa [M] f32, sb [N] f32, bias [N] bf16 or NULL, y [M, N] (row stride ldy; H3B_EPI_SWIGLU: [M, N/2]).
 * Epilogue arithmetic: t = sb[n] * acc; y = sa[m] * t (or fma(sa[m], t, bias[n])); one rounding to out_dtype.
 * Requirements: K % 16 == 0, N % 16 == 0 (SWIGLU: (N/2) % 128 == 0), lda/ldw multiples of 16, ldy multiple of 8,
 * a/w 16-byte aligned. */
H3B_API int h3b_fp8_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, const float* sa, const float* sb,
                 const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int32_t out_dtype,
                 int32_t epilogue, const h3b_qkv_send* send, h3b_stream_t stream);

/* fc2 with the indexed gated residual in its epilogue.  Replaces the fc2 consumer pair the reference fuses at the
 * tensor32 level: the scale pass + indexed_gate (h3_tp2/fp8_consumers.py:203-239 _scale_indexed_gate_kernel, its
 * eager mirror _gate_torch :367-371): o = bf16(sa[m] * (sb[n] * acc)) (bias by fma), then
 * y[m, n] = bf16(x[m, n] + gate[indices[m], n] * o) in fp32 with separate rounding of the product and the sum.
 * x, gate, y: bf16 row-major with leading dimensions ldx, ld_gate, ldy (multiples of 8, 16-byte aligned);
 * indices: int64 [M] (row of gate for each token, in [0, gate_rows); a row whose index is outside leaves y
 * untouched and records H3B_EINVAL in the device status word). */
H3B_API int h3b_fp8_gemm_gate(const void* a, int64_t lda, const void* w, int64_t ldw, const float* sa,
                              const float* sb, const void* bias, const void* x, int64_t ldx, const void* gate,
                              int64_t ld_gate, int64_t gate_rows, const int64_t* indices, void* y, int64_t ldy,
                              int64_t M, int64_t N, int64_t K, h3b_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * attention (tcgen05 flash attention, non-causal, head_dim 128)
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces the local attention of the Ulysses forward (upstream Attention._run_local_attention -> cuDNN SDPA, called
 * at h3_tp2/ulysses_exact.py:495-496).  o[t, h, :] = softmax(q[t, h, :] . k[:valid_kv, h, :]^T * scale) v[:valid_kv].
 *   q [s_q, heads, 128] bf16, k [s_kv, heads, 128] bf16, v [s_kv, heads, 128] bf16 or f16 (v_f16 != 0), o [s_q, heads,
 *   128] bf16; token strides q_tok/k_tok/v_tok/o_tok and head strides q_head/k_head/v_head/o_head (elements, multiples
 *   of 8, innermost stride 1).  valid_kv <= s_kv (< 0: s_kv).
 * With v_f16 the P.V product runs in f16 (P in [0, 256] after the online max, V exactly representable when |v| lies
 * in f16's normal range); with bf16 V it runs in bf16.  range_flag (device int or NULL) is the flag that the f16
 * conversion of v raised; when it holds 1 the kernel writes nothing and records H3B_ERANGE in the device status word
 * (the caller then reruns with bf16 v).  h3b_flash_attn_fwd_bf16v makes that choice on the device instead. */
H3B_API int h3b_flash_attn_fwd(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok, int64_t k_head,
                       const void* v, int64_t v_tok, int64_t v_head, void* o, int64_t o_tok, int64_t o_head,
                       int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim, float scale,
                       int32_t v_f16, const int32_t* range_flag, h3b_stream_t stream);

/* The drop-in local attention for a bf16 v of any range, as the reference's cuDNN SDPA takes it
 * (h3_tp2/ulysses_exact.py:495-496): same arguments and result as h3b_flash_attn_fwd with a bf16 v, plus two
 * caller-allocated scratch buffers, both 16-byte aligned: v16 [valid_kv, heads, 128] f16 (contiguous) and ctl of
 * H3B_ATTN_CTL_BYTES(heads) bytes (int32 range flag at byte 0, bytes 4-15 left alone, per (head, column) maxima from
 * byte 16).  Enqueued on `stream`: the flag and maxima are cleared; v16 = f16(v[:valid_kv]), the flag set to 1 if a
 * finite value overflows f16; the f16 P.V kernel computes o unless the flag is set; only if it is set, v16 is
 * rewritten as f16(v * 2^-e) with e >= 0 the smallest exponent that brings each (head, column) of v into f16's range,
 * and the f16 P.V kernel computes o with each output column multiplied back by 2^e (exact power-of-two scaling).  The
 * choice is made on the device (no host read), so o is always written; the flag afterwards says which pass ran.
 * Rows of v and k at or beyond valid_kv are never read. */
#define H3B_ATTN_CTL_BYTES(heads) (16ll + 512ll * (long long)(heads))
H3B_API int h3b_flash_attn_fwd_bf16v(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                     int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o,
                                     int64_t o_tok, int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                     int32_t heads, int32_t head_dim, float scale, void* v16, void* ctl,
                                     h3b_stream_t stream);

/* No counterpart in the reference: an attention entry point for callers that cannot allocate device memory (plugins
 * whose host framework owns all device memory and exposes no allocator to them; processes that must not allocate
 * after start-up, such as real-time services with a fixed memory plan).  Same arguments and result as
 * h3b_flash_attn_fwd_bf16v (a bf16 v of any range), but it allocates nothing: the f16 copy of v, the control words
 * and a status word live in a fixed file-scope device array of H3B_NOALLOC_SCRATCH_BYTES (32 MiB + 128.25 KiB)
 * that every GPU loading the library holds until exit.
 * Limits: valid_kv * heads * 128 <= H3B_NOALLOC_MAX_V_ELEMS (valid_kv * heads <= 131072) and heads <=
 * H3B_NOALLOC_MAX_HEADS, else H3B_EUNSUPPORTED.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) and sets the kernels'
 * shared-memory limit; make that first call before any stream capture.  All calls share the array: calls that
 * overlap on the GPU (other streams, other threads) race and must be serialised by the caller.  A device-side wait
 * that gives up is recorded in the array's own status word (not in h3b_device_status()); it stays set, and later
 * calls on that device skip their work, until h3b_noalloc_status() reads and clears it. */
#define H3B_NOALLOC_MAX_V_ELEMS (16ll << 20)
#define H3B_NOALLOC_MAX_HEADS 256
#define H3B_NOALLOC_CTL_BYTES (256ll * ((H3B_ATTN_CTL_BYTES(H3B_NOALLOC_MAX_HEADS) + 255ll) / 256ll))
#define H3B_NOALLOC_SCRATCH_BYTES (H3B_NOALLOC_CTL_BYTES + 2ll * H3B_NOALLOC_MAX_V_ELEMS)
H3B_API int h3b_flash_attn_fwd_noalloc(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                       int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o,
                                       int64_t o_tok, int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                       int32_t heads, int32_t head_dim, float scale, h3b_stream_t stream);

/* No counterpart in the reference: the status word of h3b_flash_attn_fwd_noalloc on the current device.  Waits for
 * the device (cudaDeviceSynchronize), returns 0 or the h3b_status a call recorded since the last read, and clears
 * it.  Allocates nothing. */
H3B_API int h3b_noalloc_status(void);

/* Peer-memory variant of h3b_flash_attn_fwd for the Ulysses reverse exchange (no reference counterpart: it replaces
 * the head->seq dist.all_to_all_single of h3_tp2/ulysses_exact.py:94): instead of o, each output row t of this
 * rank's heads goes to its owner rank t / m_rows, into that rank's reverse receive buffer peer_back[owner]
 * ([P, m_rows, heads, 128] bf16, this rank's slot `rank`), so the head->seq all-to-all never runs.
 * peer_back: host array of ws device pointers (this rank's own buffer at index rank). */
H3B_API int h3b_flash_attn_fwd_p2p(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                   int64_t k_head, const void* v, int64_t v_tok, int64_t v_head,
                                   void* const* peer_back, int32_t ws, int32_t rank, int64_t m_rows, int64_t s_q,
                                   int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim, float scale,
                                   int32_t v_f16, const int32_t* range_flag, h3b_stream_t stream);

/* Peer-memory variant of h3b_flash_attn_fwd_bf16v (bf16 v of any range, chosen on the device; v16 and ctl as there),
 * with the output rows stored as h3b_flash_attn_fwd_p2p stores them. */
H3B_API int h3b_flash_attn_fwd_p2p_bf16v(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                         int64_t k_head, const void* v, int64_t v_tok, int64_t v_head,
                                         void* const* peer_back, int32_t ws, int32_t rank, int64_t m_rows,
                                         int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim,
                                         float scale, void* v16, void* ctl, h3b_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * peer memory (CUDA IPC over NVLink; no multicast) for the Ulysses P2P exchange.  No reference counterpart: the
 * reference exchanges through NCCL only (h3_tp2/ulysses_exact.py:94, h3_tp2/ulysses_overlap.py:34,45).
 * ------------------------------------------------------------------------------------------------------------- */
typedef struct h3b_ipc_handle {
  unsigned char bytes[64];
} h3b_ipc_handle;

/* cudaMalloc + zero fill + IPC handle of `bytes` on the current device. */
H3B_API int h3b_p2p_alloc(size_t bytes, void** ptr, h3b_ipc_handle* handle);
/* Maps a peer's allocation into this process (peer access enabled lazily); *ptr is its device address here. */
H3B_API int h3b_p2p_open(const h3b_ipc_handle* handle, void** ptr);
H3B_API int h3b_p2p_close(void* peer_ptr);
H3B_API int h3b_p2p_free(void* ptr);
/* One kernel on `stream`: this rank stores `epoch` (system-scope release, after a system fence) into slot `rank` of every
 * rank's flag array (peer_flags[p], an int32[ws] on rank p), then waits until its own flags (my_flags) hold at least
 * `epoch` in every slot (acquire loads, bounded: H3B_ETIMEOUT in the device status word).  Work enqueued before it on
 * this stream is visible to the peers' work enqueued after their matching call. */
H3B_API int h3b_p2p_signal_wait(int32_t* const* peer_flags, int32_t* my_flags, int32_t ws, int32_t rank,
                                int32_t epoch, h3b_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Ulysses layout kernels
 * ------------------------------------------------------------------------------------------------------------- */

/* Replaces ulysses_exact.pack_into (h3_tp2/ulysses_exact.py:119, stock comm.py:44's pack copy): x [M, H, d] with
 * strides (stride_m, stride_h, 1) -> send [P, M, H/P, d] contiguous.  elem_bytes 2 (bf16/f16); to_f16 != 0 converts
 * bf16 -> f16 on the way (and sets *range_flag to 1 when a finite value overflows f16). */
H3B_API int h3b_pack_by_dest(const void* x, int64_t m, int32_t heads, int32_t d, int64_t stride_m, int64_t stride_h,
                     int32_t ws, void* send, int32_t to_f16, int32_t* range_flag, h3b_stream_t stream);

/* Replaces the upstream norm+RoPE producer launched per destination by ulysses_exact.rope_into_send
 * (h3_tp2/ulysses_exact.py:264-271; arithmetic of the reference's eager stand-in, tests/test_ulysses_exact.py:107-116):
 * x [M, H, 128] bf16 (strides stride_m, stride_h, 1), per (token, head) row n = bf16(x * rsqrt(mean(x^2) + eps) * w),
 * then the first `rot` dims rotate in half-split pairs with table[m] = cos[rot/2] | sin[rot/2] (f32, row stride
 * table_stride): (a, b) = (n[i], n[i + rot/2]) -> (a cos_i - b sin_i, b cos_i + a sin_i); written as bf16 into
 * send [P, M, H/P, 128] (head h -> rank h / (H/P)).  rot % 8 == 0, rot <= 128. */
H3B_API int h3b_norm_rope_send(const void* x, int64_t m, int32_t heads, int64_t stride_m, int64_t stride_h,
                               const void* weight, const float* table, int64_t table_stride, int32_t rot, float eps,
                               int32_t ws, void* send, h3b_stream_t stream);

/* Replaces ulysses_exact.exchange_back's unpack (copy 5, h3_tp2/ulysses_exact.py:181-183) and unpack
 * (:124): recv [P, M, hl, d] contiguous -> out [M, P*hl, d] contiguous.  2-byte elements. */
H3B_API int h3b_unpack_recv(const void* recv, int32_t ws, int64_t m, int32_t hl, int32_t d, void* out, h3b_stream_t stream);

/* bf16 -> f16 conversion of n elements (exact for values in f16's normal range); *range_flag (device int, may be
 * NULL) is set to 1 if any finite value overflows f16.  Used to feed the f16 P.V attention from a bf16 v. */
H3B_API int h3b_bf16_to_f16(const void* x, void* y, int64_t n, int32_t* range_flag, h3b_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
