/*
 * dsv41q.h -- C ABI of the B200 (sm_100a) quantized-weight hot path of the
 * DeepSeek-V4.1-Flash runtime (thedracle/deepseek-v41-mlx).
 *
 * Conventions
 *   - Every entry point returns 0 (DSV41_OK) or one of the DSV41_ERR_* codes
 *     below; dsv41_get_last_error() gives a one-line reason (thread-local).
 *   - Pointers are raw DEVICE pointers unless the name says host; sizes are
 *     element counts (int64).  The caller owns all memory.  Outputs are
 *     written, inputs are never modified, except the engram id cache, which
 *     dsv41_engram_hash updates in place exactly as the reference does.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL means
 *     the legacy default stream) and is asynchronous with respect to the host.
 *     Calls on distinct streams may run concurrently if their workspaces do
 *     not alias.
 *   - Entry points that need scratch memory take (workspace, workspace_bytes)
 *     and have a *_workspace_size() query.  The library never calls cudaMalloc
 *     on a compute path.
 *   - Shapes, dtypes and alignment are validated on the host; no device
 *     assert exists in these kernels.  Device-side waits are bounded; a wait
 *     that runs out sets a device flag read by dsv41_device_status().
 *
 * Citations name the reference interface each entry point replaces, as
 * path:line inside the reference repository.
 */
#ifndef DSV41Q_H
#define DSV41Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define DSV41_OK 0
#define DSV41_ERR_BAD_SHAPE 1
#define DSV41_ERR_BAD_DTYPE 2
#define DSV41_ERR_MISALIGNED 3
#define DSV41_ERR_CUDA 4
#define DSV41_ERR_NCCL 5
#define DSV41_ERR_TIMEOUT 6
#define DSV41_ERR_BAD_ARG 7
#define DSV41_ERR_UNSUPPORTED 8
#define DSV41_ERR_WORKSPACE 9

/* ---- dtype codes (outputs / bf16-or-f32 scale operands) ---------------- */
#define DSV41_F32 0
#define DSV41_BF16 1
#define DSV41_F16 2
#define DSV41_U8 3

/* ---- router score functions (ModelArgs.score_func) ---------------------- */
#define DSV41_SCORE_SQRTSOFTPLUS 0
#define DSV41_SCORE_SIGMOID 1
#define DSV41_SCORE_SOFTMAX 2

/* ---- MoE numerics flags -------------------------------------------------- */
/* Round the gate/up projection outputs and the shared-expert intermediates to
 * bf16 where the MLX port's SwitchGLU / SharedExpert produce bf16 arrays
 * (deepseek_v41_mlx/moe.py:37-43, :85-93).  Without it every intermediate is
 * kept in fp32 ("exact" mode, used for the 1e-5 fp32 comparison). */
#define DSV41_MOE_ROUND_BF16 1
/* Skip the shared expert (output = routed experts only). */
#define DSV41_MOE_NO_SHARED 2
/* dsv41_moe_prefill only: the shared expert alone (no routing, no routed experts) -- the
 * source-rank half of expert-parallel prefill. */
#define DSV41_MOE_SHARED_ONLY 4
/* Decode entries (dsv41_moe_decode, dsv41_moe_experts): w->s1, s3, s2 point into the
 * decode-packed scales written by dsv41_moe_decode_pack (s1 at offset 0, s3 at
 * E*I*(D/32), s2 at 2*E*I*(D/32) bytes) instead of the release layout.  Needs dim and inter
 * multiples of 256 and 16-byte aligned pointers.  Rejected by the prefill entries. */
#define DSV41_MOE_PACKED_SCALES 8
/* With packed scales, dim % 128 == 0 and enough routed work to fill a wave of CTAs, the
 * routed down projection runs two 64-row tiles of one expert per work item (shared
 * activation fragments, two MMA chains per warp).  This flag keeps it on single 64-row
 * tiles; both give the same bits whenever they pick the same K split. */
#define DSV41_MOE_NO_ROWPAIR 16

/* ---- library ------------------------------------------------------------ */
const char *dsv41_get_last_error(void);
int dsv41_abi_version(void);
/* Reads and clears the device-side status flags of the current device
 * (bit 0: a bounded wait ran out).  Synchronises `stream`. */
int dsv41_device_status(void *stream, uint32_t *flags_out);
/* Wall-time limit of every bounded device wait (mbarrier waits of the pipelined
 * kernels, waits on peers' flags in expert-parallel decode) on the current device, in
 * nanoseconds; 0 restores the default of 2 s.  A wait that runs out raises bit 0 of
 * dsv41_device_status and its kernel returns.  Set it while no kernel of this library
 * runs on the device.  No counterpart in the reference (MLX has no bounded device waits;
 * its own failure handling is the Metal-timeout retry of deepseek_v41_mlx/generate.py:47-67). */
int dsv41_set_wait_limit_ns(uint64_t ns);

/* ---- launch timing (no reference counterpart; the reference times with
 * ad-hoc time.time(), scripts/ppl_large.py:81-84).  When enabled, every hot
 * kernel launch is bracketed by CUDA events on its stream; report() waits for
 * them and writes one line per kernel name: "<name> <launches> <total_ms>". */
int dsv41_prof_enable(int on);
int dsv41_prof_reset(void);
int dsv41_prof_report(char *buf, size_t cap);
/* Time only the kernels named in the comma-separated list (NULL or "" = all), so that a
 * timed region carries events around its dominant kernel alone; every launch is still
 * counted (dsv41_prof_launches, since the last reset). */
int dsv41_prof_select(const char *names);
long long dsv41_prof_launches(void);

/* ---- a1..a7: release-format decode (bit-exact) --------------------------
 * e8m0_to_float    replaces deepseek_v41_mlx/dequant.py:33-36
 * dequant_fp8      replaces deepseek_v41_mlx/dequant.py:45-50 (+ _expand_blocks :39-42)
 * unpack_fp4       replaces deepseek_v41_mlx/dequant.py:53-60
 * dequant_fp4      replaces deepseek_v41_mlx/dequant.py:63-68
 * dequant_fp8_rows replaces deepseek_v41_mlx/dequant.py:71-79                */
int dsv41_e8m0_to_float(const uint8_t *scale, int64_t n, float *out, void *stream);
/* w u8 [rows, cols] e4m3 + s u8 [ceil(rows/32), ceil(cols/32)] -> out [rows, cols] */
int dsv41_dequant_fp8_block(const uint8_t *w, const uint8_t *s, int64_t rows, int64_t cols,
                            int out_dtype, void *out, void *stream);
/* packed u8 [rows, cols/2] -> f32 [rows, cols]; low nibble = even column */
int dsv41_unpack_fp4(const uint8_t *packed, int64_t rows, int64_t cols, float *out,
                     void *stream);
/* packed u8 [rows, cols/2] + s u8 [rows, ceil(cols/32)] -> out [rows, cols] */
int dsv41_dequant_fp4(const uint8_t *packed, const uint8_t *s, int64_t rows, int64_t cols,
                      int out_dtype, void *out, void *stream);
/* w u8 [rows, d] + s u8 [rows, d/block] -> f32 [rows, d] */
int dsv41_dequant_fp8_rows(const uint8_t *w, const uint8_t *s, int64_t rows, int64_t d,
                           int64_t block, float *out, void *stream);

/* ---- a14/a17: MLX affine group quantization -----------------------------
 * Replaces mx.dequantize as called at deepseek_v41_mlx/engram.py:219-223 and
 * the weight layout written by deepseek_v41_mlx/convert.py:156-175.
 * wq u32 [rows, cols*bits/32] (little-endian bit stream per row, element j at
 * bits [bits*j, bits*j+bits)), scales/biases [rows, cols/group] of
 * sb_dtype (BF16, F16 or F32); out = round(fma_f32(s, q, b)) to out_dtype. */
int dsv41_dequant_affine(const uint32_t *wq, const void *scales, const void *biases,
                         int sb_dtype, int64_t rows, int64_t cols, int bits, int group,
                         int out_dtype, void *out, void *stream);
/* The inverse direction, mx.quantize as called by the converter
 * (deepseek_v41_mlx/convert.py:169 quantize_tree, :188 quantize_engram_table): w
 * [rows, cols] of dtype (BF16 or F32), cols % group == 0, group in {32, 64, 128},
 * bits in {2, 4, 8} -> wq u32 [rows, cols*bits/32] in the layout above, scales and biases
 * [rows, cols/group] of the same dtype.  Per group, in fp32: scale = max((max - min) /
 * (2^bits - 1), 1e-7), signed toward the edge of larger magnitude; q0 = round(edge / scale);
 * if q0 != 0 then scale = edge / q0 and bias = edge, else bias = 0; code = clamp(round((w -
 * bias) / scale), 0, 2^bits - 1) (round half away from zero).  MLX's own numerics are not
 * pinned by any reference test. */
int dsv41_quantize_affine(const void *w, int dtype, int64_t rows, int64_t cols, int group,
                          int bits, uint32_t *wq, void *scales, void *biases, void *stream);

/* ---- a12: upstream act_quant (docs/reference/kernel.py:40-124,
 * mirrored by tests/kernel_stub.py:47-63).  x bf16 [M, K] (K % block == 0).
 * round_scale=1: s = 2^ceil(log2(amax/448)) (ue8m0, "scale_fmt" set),
 * round_scale=0: s = amax/448.  q u8 [M, K] e4m3 codes; s of s_dtype
 * (F32, or U8 = ue8m0 byte, which needs round_scale=1) [M, K/block].
 * If deq_out != NULL it also receives q*s as bf16 (the inplace=True form). */
int dsv41_act_quant_fp8(const void *x, int64_t M, int64_t K, int block, int round_scale,
                        uint8_t *q, void *s, int s_dtype, void *deq_out, void *stream);

/* ---- a3+a13 / a5+a13 / a14: weight-decode fused into the product --------
 * y[M, N] = x[M, K] . W^T with x bf16 and W in a release / MLX format.
 * Replaces the dequant-then-matmul of deepseek_v41_mlx/convert.py:119-127 +
 * nn.Linear, upstream linear() docs/reference/model.py:181-207 (a16 form:
 * activations are NOT quantized) and mx.quantized_matmul behind
 * nn.QuantizedLinear (deepseek_v41_mlx/load.py:124-131).
 * Requires K % 32 == 0 (fp8/fp4) or K % group == 0 (affine); N arbitrary.
 * out_dtype F32 or BF16.  A single activation row (M == 1) of dsv41_gemv_fp8_block or
 * dsv41_gemv_affine with K <= 16384 and 16-byte aligned x and weights runs as one
 * CUDA-core launch and leaves the workspace untouched (pass it all the same). */
size_t dsv41_gemv_workspace_size(int64_t M, int64_t N, int64_t K);
int dsv41_gemv_fp8_block(const void *x, int64_t M, int64_t K, const uint8_t *w,
                         const uint8_t *s, int64_t N, int out_dtype, void *y, void *workspace,
                         size_t workspace_bytes, void *stream);
int dsv41_gemv_fp4(const void *x, int64_t M, int64_t K, const uint8_t *w, const uint8_t *s,
                   int64_t N, int out_dtype, void *y, void *workspace, size_t workspace_bytes,
                   void *stream);
/* The same fp8 GEMV for callers that cannot give the library device memory and
 * must not have it allocate: hosts whose GPU memory is owned up front by their own
 * pool, and FFI callers with no device allocator for a workspace.  No counterpart
 * in the reference (it has no allocation-free entry point).  Scratch is a 4 MiB
 * array inside the library, held by every GPU that loads it until exit; limits
 * 1 <= M <= 32, M*K <= 262144, N <= 16384 (else DSV41_ERR_UNSUPPORTED).  The first
 * call on a device looks up that array's address and should come before any
 * stream capture; calls that overlap on the GPU race on the shared array. */
int dsv41_gemv_fp8_block_noalloc(const void *x, int64_t M, int64_t K, const uint8_t *w,
                                 const uint8_t *s, int64_t N, int out_dtype, void *y,
                                 void *stream);
/* affine: bits 4 or 8, group 64; scales/biases bf16 [N, K/64] */
int dsv41_gemv_affine(const void *x, int64_t M, int64_t K, const uint32_t *wq,
                      const void *scales, const void *biases, int bits, int64_t N,
                      int out_dtype, void *y, void *workspace, size_t workspace_bytes,
                      void *stream);

/* ---- a8: router (deepseek_v41_mlx/moe.py:58-74; upstream
 * docs/reference/model.py:809-827).  x bf16 [T, D], w bf16 [E, D], bias f32
 * [E] (may be NULL) -> weights f32 [T, topk], indices int32 [T, topk], in
 * descending biased-score order (ties: lower expert id first). */
size_t dsv41_moe_route_workspace_size(int64_t T, int64_t D, int64_t E);
int dsv41_moe_route(const void *x, int64_t T, int64_t D, const void *gate_w, const float *bias,
                    int64_t E, int topk, int score_func, float gate_temp, int norm_topk_prob,
                    float route_scale, float *weights, int32_t *indices, void *workspace,
                    size_t workspace_bytes, void *stream);

/* ---- a9..a11: MoE layer at decode (deepseek_v41_mlx/moe.py:105-112 with
 * SwitchGLU :101-102, ClampedSwiGLU :30-43, SharedExpert :77-93).
 * Routed experts fp4 e2m1 stacked per expert:
 *   w1 (gate) u8 [E, I, D/2] + s u8 [E, I, D/32];  w3 (up) same;
 *   w2 (down) u8 [E, D, I/2] + s u8 [E, D, I/32].
 * Shared expert fp8 e4m3 with 32x32 ue8m0 blocks:
 *   sw1, sw3 u8 [I, D] + s u8 [I/32, D/32];  sw2 u8 [D, I] + s u8 [D/32, I/32].
 * Routing weights are applied after w2 and summed in fp32 in top-k order,
 * then the shared expert is added and the sum rounded to out_dtype.
 * 0 < swiglu_limit <= 255.  flags: DSV41_MOE_*.  weights_out/indices_out may
 * be NULL. */
typedef struct dsv41_moe_weights {
  const void *gate_w;      /* bf16 [E, D] */
  const float *gate_bias;  /* f32 [E] or NULL */
  const uint8_t *w1, *s1;  /* fp4 experts */
  const uint8_t *w3, *s3;
  const uint8_t *w2, *s2;
  const uint8_t *sw1, *ss1; /* fp8 shared expert */
  const uint8_t *sw3, *ss3;
  const uint8_t *sw2, *ss2;
} dsv41_moe_weights;

typedef struct dsv41_moe_config {
  int64_t dim;        /* D */
  int64_t inter;      /* I (moe_inter_dim) */
  int64_t n_experts;  /* E */
  int topk;
  int score_func;
  float gate_temp;
  int norm_topk_prob;
  float route_scale;
  float swiglu_limit;
  int flags;
} dsv41_moe_config;

/* Decode-packed expert scales (no reference counterpart; the release layout is kept as the
 * input): for each of s1, s3 ([E*I, D/32]) and s2 ([E*D, I/32]) the bytes one decode stage of
 * one 64-row tile reads -- 64 rows x 8 groups of 32 -- become one contiguous 512-byte block
 * ([rows/64][K/256][64][8]), fetched by a single bulk copy instead of an 8-byte request per row.
 * packed: dsv41_moe_decode_pack_size(cfg) bytes, 16-byte aligned; valid while the scales are
 * unchanged. */
size_t dsv41_moe_decode_pack_size(const dsv41_moe_config *cfg);
int dsv41_moe_decode_pack(const dsv41_moe_config *cfg, const dsv41_moe_weights *w, void *packed,
                          size_t packed_bytes, void *stream);
size_t dsv41_moe_decode_workspace_size(const dsv41_moe_config *cfg, int64_t T);
/* The routed experts alone for given routing (mlx_lm SwitchGLU as called at
 * deepseek_v41_mlx/moe.py:109, i.e. MoE.experts(xf, indices)): indices int32
 * [T, topk] -> y f32 [T, topk, D], unweighted.  Same workspace size query. */
int dsv41_moe_experts(const dsv41_moe_config *cfg, const dsv41_moe_weights *w, const void *x,
                      int64_t T, const int32_t *indices, float *y, void *workspace,
                      size_t workspace_bytes, void *stream);
int dsv41_moe_decode(const dsv41_moe_config *cfg, const dsv41_moe_weights *w, const void *x,
                     int64_t T, int out_dtype, void *y, float *weights_out,
                     int32_t *indices_out, void *workspace, size_t workspace_bytes,
                     void *stream);

/* ---- a14 at prefill sizes: MLX affine quantized matmul (mx.quantized_matmul behind
 * nn.QuantizedLinear, deepseek_v41_mlx/load.py:124-131) on tcgen05 kind::f16.
 * y[M, N] = x[M, K] . W^T, W = bf16(fma_f32(scale, q, bias)) per group of 64 -- the weights
 * dequantized to the activation dtype as MLX's quantized matmul does for bf16 inputs.
 * x bf16 [M, K]; wq u32 [N, K*bits/32] (little-endian row bit stream); scales, biases bf16
 * [N, K/64]; bits 4 or 8; K % 64 == 0, N % 128 == 0; out F32 or BF16.  For decode sizes use
 * dsv41_gemv_affine (exact affine arithmetic, no weight rounding). */
int dsv41_qmm_affine(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                     const void *biases, int bits, int64_t N, int out_dtype, void *y,
                     void *stream);

/* ---- a13: upstream fp8_gemm / fp4_gemm (docs/reference/kernel.py:277-308 and
 * :562-591) on tcgen05 block-scaled MMA (kind::mxf8f6f4, fp32
 * accumulation in TMEM).  C[M, N] = A[M, K] . B[N, K]^T with
 *   a   fp8 e4m3 [M, K], a_s ue8m0 bytes [M, K / block] (act_quant output);
 *   b   fp8_gemm: fp8 e4m3 [N, K], b_s ue8m0 [ceil(N/block), K/block] (block 32 or 128);
 *       fp4_gemm: fp4 e2m1 packed two per byte [N, K/2] (low nibble = even k),
 *                 b_s ue8m0 [N, K/32]; act_block_size 32 or 128 for a_s;
 *   c   [M, N] F32 or BF16 (upstream returns torch's default dtype).
 * N and K must be multiples of 128; a and c 16-byte aligned, scales 4-byte aligned.
 * Only ue8m0 scales: upstream's float32-scale variant has no block-scaled MMA form. */
int dsv41_fp8_gemm(const uint8_t *a, const uint8_t *a_s, const uint8_t *b, const uint8_t *b_s,
                   int64_t M, int64_t N, int64_t K, int block_size, void *c, int c_dtype,
                   void *stream);
int dsv41_fp4_gemm(const uint8_t *a, const uint8_t *a_s, const uint8_t *b, const uint8_t *b_s,
                   int64_t M, int64_t N, int64_t K, int act_block_size, void *c, int c_dtype,
                   void *stream);

/* ---- MoE prefill, a8 numerics (docs/reference/model.py:889-904 with Expert.forward
 * :841-851 and linear() :181-207): act_quant(x, 32, ue8m0), per-expert fp4 gate/up on the
 * block-scaled grouped GEMM, clamped SwiGLU x routing weight -> bf16 -> act_quant, fp4
 * down -> bf16 per (token, expert), summed in ascending expert order, + the fp8 shared
 * expert (same a8 form).  Routing is either given (route_weights f32 [T, topk],
 * route_indices int32 [T, topk]) or computed with the router of dsv41_moe_route when
 * route_indices is NULL.  dim and inter must be multiples of 128, topk <= 8.
 *
 * packed_scales: the expert scales rearranged once by dsv41_moe_prefill_pack into the
 * layout the tensor cores read (dsv41_moe_prefill_pack_size bytes, 16-byte aligned); valid
 * while the expert scales are unchanged.  NULL: they are packed into the workspace on
 * every call.  No reference counterpart (the reference dequantizes per call).
 * Workspace query: with_routing = 1 when routing is passed, with_packed = 1 when
 * packed_scales is passed. */
size_t dsv41_moe_prefill_pack_size(const dsv41_moe_config *cfg);
int dsv41_moe_prefill_pack(const dsv41_moe_config *cfg, const dsv41_moe_weights *w, void *packed,
                           size_t packed_bytes, void *stream);
size_t dsv41_moe_prefill_workspace_size(const dsv41_moe_config *cfg, int64_t T, int with_routing,
                                        int with_packed);
int dsv41_moe_prefill(const dsv41_moe_config *cfg, const dsv41_moe_weights *w,
                      const void *packed_scales, const void *x, int64_t T,
                      const float *route_weights, const int32_t *route_indices, int out_dtype,
                      void *y, void *workspace, size_t workspace_bytes, void *stream);

/* ---- a10 + a13 at prefill sizes in the port's numerics ("a16"): the MoE layer of
 * deepseek_v41_mlx/moe.py:96-112 (SwitchGLU over the release's fp4 experts decoded exactly to
 * bf16, dequant.py:63-68; the fp8 shared expert, moe.py:77-93) with bf16 activations as they
 * are, on tcgen05 kind::f16 tensor cores: routed gate/up -> clamped SwiGLU in fp32 -> down on
 * that fp32 h (as bf16 hi + lo halves) -> expert outputs weighted and summed in top-k order,
 * fp32, + the shared expert.  cfg->flags: DSV41_MOE_ROUND_BF16 = the port's bf16 rounding of
 * the gate/up outputs and of the shared expert's intermediates (else every intermediate stays
 * fp32); DSV41_MOE_NO_SHARED / DSV41_MOE_SHARED_ONLY as for dsv41_moe_prefill.  Routing is
 * computed (route_indices NULL) or given (weights f32 [T, topk], indices int32 [T, topk]).
 * dim % 128 == 0, moe_inter_dim % 128 == 0, topk <= 8; x bf16 [T, dim], y F32 or BF16
 * [T, dim], both 16-byte aligned. */
size_t dsv41_moe_prefill_a16_workspace_size(const dsv41_moe_config *cfg, int64_t T,
                                            int with_routing);
int dsv41_moe_prefill_a16(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, const void *x,
                          int64_t T, const float *route_weights, const int32_t *route_indices,
                          int out_dtype, void *y, void *workspace, size_t workspace_bytes,
                          void *stream);

/* ---- (e) expert-parallel prefill (replaces upstream's replicate + fp32 all_reduce,
 * docs/reference/model.py:854-904).  Source rank: dsv41_moe_ep_pack quantizes its tokens
 * (act_quant), sorts the (token, slot) pairs by global expert (hence by owner rank) and packs
 * each pair as one row of dsv41_moe_ep_row_bytes(dim) bytes -- fp8 codes, ue8m0 scales,
 * owner-local expert id (int32), routing weight (f32) -- plus int64 send_counts[world] and
 * int32 slot_pos[T*topk] (row of pair (t, j)).  The caller exchanges the rows (all-to-all);
 * the owner runs dsv41_moe_ep_experts (cfg with its local expert count) -> bf16 [R, dim]
 * in arrival order; after the mirror exchange, dsv41_moe_ep_combine sums each token's rows
 * in ascending expert order and adds the shared expert (bf16 [T, dim], may be NULL). */
size_t dsv41_moe_ep_row_bytes(int64_t dim);
size_t dsv41_moe_ep_pack_workspace_size(const dsv41_moe_config *cfg, int64_t T);
int dsv41_moe_ep_pack(const dsv41_moe_config *cfg, const void *x, int64_t T,
                      const float *route_weights, const int32_t *route_indices, int world,
                      void *send_rows, int64_t *send_counts, int32_t *slot_pos, void *workspace,
                      size_t workspace_bytes, void *stream);
size_t dsv41_moe_ep_experts_workspace_size(const dsv41_moe_config *cfg, int64_t R, int with_packed);
int dsv41_moe_ep_experts(const dsv41_moe_config *cfg, const dsv41_moe_weights *w,
                         const void *packed_scales, const void *recv_rows, int64_t R, void *y,
                         void *workspace, size_t workspace_bytes, void *stream);
int dsv41_moe_ep_combine(const void *back, const int32_t *slot_pos, const int32_t *route_indices,
                         const void *shared, int64_t T, int topk, int64_t dim, int out_dtype,
                         void *y, void *stream);

/* ---- (e) expert-parallel decode over NVLink peer memory (replaces upstream's replicate +
 * fp32 all_reduce, docs/reference/model.py:854-904, at decode).  One context per rank:
 * dsv41_ep_create allocates this rank's exchange buffer (rows it receives, outputs it gets
 * back, step flags); every rank exports its IPC handle (dsv41_ep_handle,
 * dsv41_ep_handle_bytes() bytes), the caller gathers them in rank order (e.g. an
 * all_gather) and each rank maps its peers' buffers with dsv41_ep_connect.  One MoE decode
 * step is then dsv41_moe_ep_decode on every rank (a collective: all ranks call it the same
 * number of times, T may differ per rank): route the rank's own tokens with the replicated
 * router, write each (token, expert) row into the owning rank's buffer, run this rank's
 * experts (cfg->n_experts / world of them, w holding only those, renumbered from 0) on the
 * rows it received, write the fp32 outputs back into the sources' buffers, and sum each
 * token's outputs in top-k order with the shared expert -- the same fp32 operations as
 * dsv41_moe_decode on one GPU.  No host synchronisation; waits for peers are bounded (on
 * expiry the device status bit 0 is raised).  cfg->n_experts is the total expert count. */
typedef struct dsv41_ep_ctx dsv41_ep_ctx;
int dsv41_ep_create(int world, int rank, int64_t max_tokens, int topk, int64_t dim,
                    dsv41_ep_ctx **out);
size_t dsv41_ep_handle_bytes(void);
int dsv41_ep_handle(const dsv41_ep_ctx *ctx, void *handle_out);
int dsv41_ep_connect(dsv41_ep_ctx *ctx, const void *handles);
int dsv41_ep_destroy(dsv41_ep_ctx *ctx);
/* The bounded wait of one exchange direction of dsv41_moe_ep_decode, on its own: until
 * every rank has published the current step's flag (which = 0: its rows arrived in this
 * rank's buffer; which = 1: its outputs arrived back), or the wait limit runs out (bit 0 of
 * dsv41_device_status).  Stream-ordered; does not advance the step.  Part of the
 * exchange that replaces upstream's fp32 all_reduce (docs/reference/model.py:895-902). */
int dsv41_ep_wait(const dsv41_ep_ctx *ctx, int which, void *stream);
size_t dsv41_moe_ep_decode_workspace_size(const dsv41_moe_config *cfg, const dsv41_ep_ctx *ctx,
                                          int64_t T);
int dsv41_moe_ep_decode(const dsv41_moe_config *cfg, const dsv41_moe_weights *w,
                        dsv41_ep_ctx *ctx, const void *x, int64_t T, int out_dtype, void *y,
                        float *weights_out, int32_t *indices_out, void *workspace,
                        size_t workspace_bytes, void *stream);

/* ---- a15: engram hasher (deepseek_v41_mlx/engram.py:154-180; upstream
 * docs/reference/engram.py NgramHashState.forward).  input_ids int64 [B, L];
 * token_map int64 [V]; ids_cache int64 [B, max_seq], positions
 * [start_pos, start_pos+L) are written in place; multipliers int64 [nL, G];
 * primes int64 [nL, G-1, H]; offsets int64 [nL, (G-1)*H].
 * out int64 [B, L, nL, (G-1)*H].  Input ids outside [0, V) are an error
 * reported through dsv41_device_status bit 1 and hash to row 0. */
int dsv41_engram_hash(const int64_t *input_ids, int64_t B, int64_t L, int64_t start_pos,
                      const int64_t *token_map, int64_t vocab, int64_t *ids_cache,
                      int64_t max_seq, const int64_t *multipliers, const int64_t *primes,
                      const int64_t *offsets, int n_layers, int max_ngram, int n_heads,
                      int64_t pad_id, int64_t *out, void *stream);

/* ---- a15 + a16 in one launch: hash layer `layer` of the dsv41_engram_hash layout and sum
 * its (G-1)*H <= 32 rows a position from a packed table -- EngramHasher.__call__
 * (deepseek_v41_mlx/engram.py:154-180) followed by EngramEmbedding.__call__ (:197-203) and
 * the sum over the hashed rows (upstream Engram.forward's embedding sum,
 * docs/reference/model.py:344-365), without writing the ids.  The id cache is updated as
 * dsv41_engram_hash updates it.  packed: [n_rows, dsv41_engram_row_bytes(d, block)] rows
 * (dsv41_engram_pack_rows with idx = NULL), holding table rows [row_lo, row_lo + n_rows);
 * other ids read as zero rows.  reciprocals: NULL, or uint64 [nL, G-1, H] =
 * floor((2^64 - 1) / prime) (0 where prime <= 1), computed once with the layout, which spares
 * every launch a 64-bit division per prime.  Needs (G-1)*H <= 32 and G <= 8.
 * out f32/bf16 [B, L, d], the same bits as dsv41_engram_hash then dsv41_engram_sum_rows. */
int dsv41_engram_lookup_sum(const int64_t *input_ids, int64_t B, int64_t L, int64_t start_pos,
                            const int64_t *token_map, int64_t vocab, int64_t *ids_cache,
                            int64_t max_seq, const int64_t *multipliers, const int64_t *primes,
                            const int64_t *offsets, const uint64_t *reciprocals, int n_layers,
                            int layer, int max_ngram, int n_heads, int64_t pad_id,
                            const void *packed, int64_t n_rows,
                            int64_t row_lo, int64_t d, int64_t block, int out_dtype, void *out,
                            void *stream);

/* ---- a16: engram row gather (deepseek_v41_mlx/engram.py:197-203; upstream
 * ParallelEngramEmbedding.forward docs/reference/model.py:312-325).
 * table u8 [rows, d] e4m3 + scale u8 [rows, d/block]; idx int64 [n_idx]
 * (row ids; rows outside [row_lo, row_lo + rows) read as zero rows, which is
 * the row-sharded form with row_lo = rank * rows_per_rank).
 *   gather_rows: out f32/bf16 [n_idx, d]  (= EngramEmbedding output)
 *   gather_sum : out f32/bf16 [n_tok, d], out[t] = fp32 sum over the
 *                n_per_tok rows idx[t*n_per_tok + h] in h order. */
int dsv41_engram_gather_rows(const uint8_t *table, const uint8_t *scale, int64_t rows,
                             int64_t row_lo, int64_t d, int64_t block, const int64_t *idx,
                             int64_t n_idx, int out_dtype, void *out, void *stream);
int dsv41_engram_gather_sum(const uint8_t *table, const uint8_t *scale, int64_t rows,
                            int64_t row_lo, int64_t d, int64_t block, const int64_t *idx,
                            int64_t n_tok, int n_per_tok, int out_dtype, void *out,
                            void *stream);

/* ---- (e) row-sharded engram table (replaces upstream ParallelEngramEmbedding.forward,
 * docs/reference/model.py:312-325: zero-masked local lookup + all_reduce of the rows).
 * Rank r owns rows [r*part, (r+1)*part) of the table; the hashes are known on every rank.
 * Each rank sums the rows of one slice of the tokens: the owners copy the raw rows that
 * slice needs (dsv41_engram_pack_rows, packed rows of dsv41_engram_row_bytes(d, block)
 * bytes: d e4m3 codes, d/block ue8m0 bytes, zero padding to 16), the caller exchanges
 * them (all-to-all), and the slice's rank sums them per token in head order
 * (dsv41_engram_sum_rows, = dsv41_engram_gather_sum on the received rows; pos[t*n + h] is
 * the received row of (t, h), negative = skipped) or dequantizes them one by one
 * (dsv41_engram_dequant_rows, = dsv41_engram_gather_rows).  Bit-identical to one GPU.
 * dsv41_engram_pack_rows with idx = NULL repacks rows 0 .. n-1 of a table in order: a
 * table stored that way (1040 bytes a row at d = 1024) is read with dsv41_engram_sum_rows /
 * dsv41_engram_dequant_rows with pos = the row ids -- one contiguous read a row. */
size_t dsv41_engram_row_bytes(int64_t d, int64_t block);
int dsv41_engram_pack_rows(const uint8_t *table, const uint8_t *scale, int64_t rows,
                           int64_t row_lo, int64_t d, int64_t block, const int64_t *idx, int64_t n,
                           void *out_rows, void *stream);
int dsv41_engram_sum_rows(const void *packed, int64_t n_rows, int64_t d, int64_t block,
                          const int64_t *pos, int64_t n_tok, int n_per_tok, int out_dtype,
                          void *out, void *stream);
int dsv41_engram_dequant_rows(const void *packed, int64_t n_rows, int64_t d, int64_t block,
                              const int64_t *pos, int64_t n, int out_dtype, void *out,
                              void *stream);

/* ---- Engram gate (deepseek_v41_mlx/engram.py:245-264; upstream Engram.forward,
 * docs/reference/model.py:344-365), applied after kv = wkv(rows):
 * x, out [T, hc, D] of x_dtype (F32 or BF16; out takes x's type); kv [T, (hc+1)*D] of kv_dtype
 * (hc keys, then the shared value); q_weight, k_weight f32 [hc, D]; token_mask u8 [T] or NULL
 * (upstream's mask: 0 closes the gate).  Per (token, hc copy): rstd = rsqrt(mean(h^2)+eps) *
 * rsqrt(mean(key^2)+eps), dot = sum(h*q*k*key)*rstd/sqrt(D), gate = sigmoid(sign(dot) *
 * sqrt(max(|dot|, clamp))), out = h + gate*value.  fp32 arithmetic. */
int dsv41_engram_gate(const void *x, int x_dtype, const void *kv, int kv_dtype,
                      const float *q_weight, const float *k_weight, const uint8_t *token_mask,
                      int64_t T, int hc, int64_t D, float eps, float clamp, void *out,
                      void *stream);

/* ---- (e) row-sharded engram table read in place through NVLink peer memory: every rank maps
 * the other ranks' shards (CUDA IPC) once, then sums the rows of its own slice of the tokens
 * reading each row from the GPU that holds it -- no row packing, no exchange of rows, no
 * host synchronisation (the callers all-gather the slices).  tables / scales: device arrays
 * of nsh pointers (uint64) to shard s's codes u8 [rows, d] and scales u8 [rows, d/block]
 * (shard s holds global rows [s*rows, (s+1)*rows), the last one possibly fewer: ids at or past
 * total, the table's row count, read as zero rows); otherwise as dsv41_engram_gather_sum.
 * dsv41_ipc_export gives the IPC handle (dsv41_ep_handle_bytes() bytes) of the allocation
 * holding ptr and ptr's offset in it; dsv41_ipc_import maps a peer's allocation (its base;
 * add the offset), dsv41_ipc_close unmaps it.  Each allocation is imported once per process. */
int dsv41_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out);
int dsv41_ipc_import(const void *handle, void **base_out);
int dsv41_ipc_close(void *base);
int dsv41_engram_gather_sum_peers(const uint64_t *tables, const uint64_t *scales, int nsh,
                                  int64_t rows, int64_t total, int64_t d, int64_t block,
                                  const int64_t *idx,
                                  int64_t n_tok, int n_per_tok, int out_dtype, void *out,
                                  void *stream);
/* dsv41_engram_lookup_sum over the row shards: the hashing of dsv41_engram_lookup_sum (id
 * cache updated the same way), the rows read from the shards as dsv41_engram_gather_sum_peers
 * reads them.  The same bits as dsv41_engram_hash then dsv41_engram_gather_sum_peers. */
int dsv41_engram_lookup_sum_peers(const int64_t *input_ids, int64_t B, int64_t L,
                                  int64_t start_pos, const int64_t *token_map, int64_t vocab,
                                  int64_t *ids_cache, int64_t max_seq,
                                  const int64_t *multipliers, const int64_t *primes,
                                  const int64_t *offsets, const uint64_t *reciprocals,
                                  int n_layers, int layer, int max_ngram, int n_heads,
                                  int64_t pad_id, const uint64_t *tables, const uint64_t *scales,
                                  int nsh, int64_t rows, int64_t total, int64_t d, int64_t block,
                                  int out_dtype, void *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DSV41Q_H */
