/* mingmoe — C-ABI of the B200 (sm_100a) kernels for ming-voice's Ling-style MoE block.
 *
 * Every entry point takes raw device pointers, sizes, element strides, dtype codes and a cudaStream_t
 * (passed as void*), enqueues its kernels on that stream without synchronising the host, and returns an
 * int status (MV_OK = 0). On failure the message is available from mv_last_error() (thread-local). No entry
 * point allocates device memory: callers pass a zero-initialised workspace where one is needed and query its
 * size with the matching *_workspace_bytes function. A workspace may be reused by every call on one stream
 * (the kernels leave it zeroed again), but two calls that can run at the same time need two workspaces.
 *
 * The Python modules fused_moe.py / fused_ops.py / fastlinear.py of the `ming-voice_b200` directory wrap
 * these entry points behind the reference's own signatures; each declaration names the reference function
 * it replaces (file:line in ming-voice).
 */
#ifndef MINGMOE_H
#define MINGMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MV_API __attribute__((visibility("default")))
#else
#define MV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define MV_OK 0
#define MV_ERR_INVALID 1     /* bad shape, size or argument */
#define MV_ERR_ALIGN 2       /* pointer / stride alignment requirement not met */
#define MV_ERR_CUDA 3        /* CUDA runtime error while launching */
#define MV_ERR_UNSUPPORTED 4 /* dtype or option combination not implemented */
#define MV_ERR_WORKSPACE 5   /* workspace missing or too small */

/* ---- dtype codes ---- */
#define MV_BF16 0
#define MV_F16 1
#define MV_F32 2
#define MV_I8 3
#define MV_I32 4
#define MV_I64 5

/* ---- router modes ---- */
#define MV_ROUTE_SOFTMAX 0       /* softmax(logits [+ bias]) -> top-k -> renormalise (Ling v1 style) */
#define MV_ROUTE_SIGMOID_GROUP 1 /* sigmoid + bias, group-limited top-k, renormalise, x scale (ming-voice) */

/* Library version (major * 10000 + minor * 100 + patch). */
MV_API int mv_version(void);

/* Message of the last failed call on this host thread ("" if none). */
MV_API const char* mv_last_error(void);

/* Reads (synchronously, on `stream`) the device-side error word of a workspace: 0 = none, 1 = a bounded
 * wait timed out, 2 = an expert id outside [0, E1) was skipped, 3 = a capacity was exceeded. `info` (may be
 * NULL) receives where it was raised. With clear != 0 the word is reset. Host-synchronising; not for use
 * inside stream capture. */
MV_API int mv_workspace_status(void* workspace, int clear, unsigned int* code, unsigned int* info, void* stream);

/* RMSNorm over the last dimension: replaces fused_ops.rms_norm (fused_ops.py:28-37, kernel :16-25).
 * y[r] = cast(w * cast(x[r] / sqrt(mean(x[r]^2) + eps), x_dtype), y_dtype); fp32 statistics.
 * x: rows x n (row stride x_stride elements, inner stride 1), dtype bf16/f16/f32; w: [n] bf16/f16/f32;
 * y: rows x n contiguous. */
MV_API int mv_rmsnorm(const void* x, int x_dtype, long long x_stride, const void* w, int w_dtype, void* y, int y_dtype,
               int rows, int n, float eps, void* stream);

/* Router for n_tokens tokens: replaces fused_ops.moe_route (fused_ops.py:96-103; kernels :40-93) in mode
 * MV_ROUTE_SIGMOID_GROUP, and is the BASELINE softmax-top-k router in mode MV_ROUTE_SOFTMAX.
 *  x        [n_tokens, H] bf16 (row stride x_stride), the normalised hidden states;
 *  w        [E, H] router weight, dtype w_dtype in {f32 (the reference's w32 copy), bf16, i8};
 *  w_scale  [E] per-row scale when w is i8 (dtype scale_dtype f32/bf16), else NULL;
 *  bias     [E] f32 or NULL: added to the sigmoid scores (sigmoid mode) / to the logits (softmax mode);
 *  logits_out [n_tokens, E] f32 (may be NULL);
 *  ids_out  [n_tokens, top_k + n_shared] (i32 or i64); wts_out same shape f32: the top_k experts, largest
 *           first, ties to the lower id, then the shared slots shared_id .. shared_id + n_shared - 1 with
 *           weight 1.0 (fused_ops.py:89-93).
 * Sigmoid mode: n_group groups, keep topk_group groups by their top-2 sum, weights renormalised with +1e-20
 * and multiplied by `scale`. Softmax mode ignores n_group / topk_group / scale.
 * Logits are accumulated in fp64 and rounded once to fp32 (order-independent selection).
 * workspace: mv_route_workspace_bytes(n_tokens, E) bytes, zero-initialised. */
MV_API int mv_route(int mode, const void* x, long long x_stride, const void* w, int w_dtype, const void* w_scale,
             int scale_dtype, const float* bias, int n_tokens, int H, int E, int top_k, int n_group,
             int topk_group, double scale, int n_shared, int shared_id, float* logits_out, void* ids_out,
             int ids_dtype, float* wts_out, void* workspace, size_t workspace_bytes, void* stream);
MV_API size_t mv_route_workspace_bytes(int n_tokens, int E);

/* Symmetric per-row int8 quantisation: replaces fused_moe.quantize_rows_int8 (fused_moe.py:199-204).
 * w: rows x K (row stride w_stride elements), bf16/f16/f32. q: rows x K int8 contiguous;
 * scale: [rows], dtype scale_dtype (f32 = the reference's layout; bf16 = scale rounded to bf16 first and q
 * computed against the rounded scale). amax = max|w| clamped to >= 1e-8, scale = amax / 127,
 * q = round_half_even(w / scale) clamped to [-127, 127]; bit-exact with torch. */
MV_API int mv_quantize_rows_int8(const void* w, int w_dtype, long long w_stride, long long rows, int K, int8_t* q,
                          void* scale, int scale_dtype, void* stream);

/* Quantise-on-load into a stacked slot: replaces the loader hook of ming-voice's _int8_expert_loaders
 * (engine.py:126-147: quantize_rows_int8 on the device, then copies into q[e, off:off + n] and s[e, off:off + n]),
 * which the loader threads call per checkpoint tensor (direct_load.py:109-135). The `rows` x K matrix w (row
 * stride w_stride elements; bf16/f16/f32; device memory or pinned host memory the device can read) is quantised
 * as mv_quantize_rows_int8 does and written directly to rows [row_off, row_off + rows) of slot e of the
 * contiguous int8 stack q_stack [E1, rows_per_expert, K] and of the scale stack s_stack [E1, rows_per_expert]
 * (s_dtype f32 or bf16). Nothing is allocated; calls on different streams for different slots may run at the
 * same time (each loader thread on its own stream). */
MV_API int mv_quantize_into_stack(const void* w, int w_dtype, long long w_stride, int rows, int K, int8_t* q_stack,
                                  void* s_stack, int s_dtype, int E1, int rows_per_expert, int e, int row_off,
                                  void* stream);

/* Dequantisation exactly as the int8 kernels perform it in registers: out = float(q) * float(scale[row]),
 * one correctly rounded fp32 multiply (== torch q.float() * s.float()). Exported so the in-kernel
 * dequantisation can be checked bit for bit. q: rows x K contiguous; out: rows x K f32. */
MV_API int mv_dequant_rows_int8(const int8_t* q, const void* scale, int scale_dtype, long long rows, int K,
                         float* out, void* stream);

/* Small-M linear layer: replaces fastlinear.small_linear's kernel path (fastlinear.py:142-174, kernel
 * _small_m_linear :20-62). y[m] = bf16( act(norm?(x[m]) @ W^T + bias) [+ residual[m]] ) for M <= 16 rows.
 * x [M, K] bf16 (row stride x_stride), W [N, K] bf16 (row stride w_stride), bias [N] bf16 or NULL,
 * residual [M, N] bf16 (row stride residual_stride) or NULL, norm_w [K] bf16 or NULL (RMSNorm prologue with
 * eps, as mv_rmsnorm), act 0 none / 1 gelu-tanh / 2 silu (on the bf16-rounded pre-activation; with a
 * residual the activation is rounded to bf16 before the add), y [M, N] bf16 (row stride y_stride).
 * Requirements: K a multiple of 8, M * K * 2 <= 200 KB, 16-byte aligned x / W / norm_w and row strides. */
MV_API int mv_small_linear(const void* x, long long x_stride, const void* w, long long w_stride, const void* bias,
                           const void* residual, long long residual_stride, const void* norm_w, float eps, int act,
                           void* y, long long y_stride, int M, int N, int K, void* stream);

/* Stacked expert weights in the reference layout (engine.py:150-188, fused_moe.py:3-6):
 * w_gu [E1, 2I, H] (gate rows [0, I), up rows [I, 2I)), w_d [E1, H, I]; inner stride 1; strides in elements.
 * w_dtype MV_BF16 or MV_I8; int8 weights carry per-output-row scales s_gu [E1, 2I] and s_d [E1, H]
 * (s_dtype MV_F32 or MV_BF16, inner stride 1). */
typedef struct mv_moe_weights {
  const void* w_gu;
  const void* w_d;
  const void* s_gu;
  const void* s_d;
  int w_dtype;
  int s_dtype;
  int E1;
  int H;
  int I;
  int pad0;
  long long gu_se, gu_sr; /* w_gu strides: expert, row */
  long long d_se, d_sr;   /* w_d strides: expert, row */
  long long sgu_se;       /* s_gu expert stride */
  long long sd_se;        /* s_d expert stride */
} mv_moe_weights;

/* Decode MoE (M <= 16 tokens): replaces fused_moe.fused_moe_decode (fused_moe.py:67-83; kernels :14-61)
 * and the M = 2..16 use of fused_moe_prefill (engine.py:381-382).
 *   out[m] = cast_bf16( residual[m] + sum_k wts[m,k] * down_e(silu(gate_e(xn_m)) * up_e(xn_m)) ),  e = ids[m,k]
 * x [M, H] bf16 (row stride x_stride). If norm_w (bf16 [H]) is non-NULL, xn = RMSNorm(x) with eps, computed
 * as mv_rmsnorm does; otherwise xn = x. ids [M, NK] (i32 or i64, row stride NK), wts [M, NK] f32. ids outside
 * [0, E1) are skipped and flagged in the workspace. residual [M, H] bf16 or NULL. out [M, H] bf16.
 * Intermediates stay fp32 (no bf16 rounding of gate/up/act/per-expert outputs).
 * One cooperative kernel (one CTA per SM): each CTA streams an equal share of the selected experts' gate/up
 * rows, then (after one grid barrier) an equal share of output rows of their down projections.
 * workspace: mv_moe_decode_workspace_bytes(M, NK, I, 0) bytes, zero-initialised (left zeroed).
 * Requirements: M <= 16, NK <= 32, E1 <= 4096, H and I multiples of 8 (bf16) / 16 (i8), H <= 8192,
 * 8 rows of w_d within 32 KB (I <= 2048 bf16 / 4096 i8), 16-byte aligned pointers and row strides. */
MV_API int mv_moe_decode(const mv_moe_weights* w, const void* x, long long x_stride, const void* norm_w, float eps,
                         const void* ids, int ids_dtype, const float* wts, int M, int NK, const void* residual,
                         void* out, void* workspace, size_t workspace_bytes, void* stream);
MV_API size_t mv_moe_decode_workspace_bytes(int M, int NK, int I, int E);

/* Sort of (token, slot) pairs by expert for the grouped GEMMs: replaces fused_moe._align_blocks
 * (fused_moe.py:154-173), same outputs. ids [P] (i32/i64, the flattened [N, NK] expert ids). Each expert's
 * pairs keep their index order (stable) and its run is padded to a multiple of BM rows.
 *   sorted_out [nb_max * BM] i32: pair index, P for padding;  bexp_out [nb_max] i32: expert of each block,
 *   -1 for unused blocks;  nb_used_out [1] i32: blocks in use;  nb_max = (P + E1 * (BM - 1) + BM - 1) / BM.
 * ids outside [0, E1) are dropped and flagged in the workspace (mv_moe_align_workspace_bytes(P, E1) bytes,
 * header zero-initialised). Requirements: E1 <= 512, 1 <= BM <= 4096. */
MV_API int mv_moe_align(const void* ids, int ids_dtype, int P, int E1, int BM, int* sorted_out, int* bexp_out,
                        int* nb_used_out, void* workspace, size_t workspace_bytes, void* stream);
MV_API size_t mv_moe_align_workspace_bytes(int P, int E1);

/* Prefill MoE for N tokens on the tensor cores (tcgen05): replaces fused_moe.fused_moe_prefill
 * (fused_moe.py:176-196; kernels _moe_gu_grouped :93-121, _moe_down_grouped :125-148).
 *   out[t] = bf16( residual[t] + sum_k wts[t,k] * down_e(bf16(silu(gate_e(x_t)) * up_e(x_t))) ), e = ids[t,k]
 * x [N, H] bf16 (row stride x_stride), ids [N, NK] i32/i64, wts [N, NK] f32, residual [N, H] bf16 (row stride
 * residual_stride) or NULL, out [N, H] bf16 contiguous. Gate/up accumulate in fp32; the activation is rounded
 * to bf16 once (the tensor-core operand of the down projection); the per-pair outputs are weighted and summed
 * in fp32 (reduction order not fixed). Weights bf16, or int8 with row scales: the experts in use are widened to
 * bf16 (exact) in the workspace and the scales multiply the fp32 products, as the reference's int8 kernels do.
 * workspace: mv_moe_prefill_workspace_bytes(N, NK, H, I, E1, w_dtype) bytes, 256-byte aligned, header zeroed
 * (int8 adds bf16 copies of the stacks: E1 * 3 * I * H * 2 bytes).
 * An id of -1 marks "no pair" (an expert held by another rank in expert-parallel prefill): the pair is skipped;
 * any other id outside [0, E1) is an error (recorded in the workspace, the pair skipped).
 * Requirements: H a multiple of 256, I a multiple of 128, E1 <= 512, 16-byte aligned pointers/strides. */
MV_API int mv_moe_prefill(const mv_moe_weights* w, const void* x, long long x_stride, const void* ids, int ids_dtype,
                          const float* wts, int N, int NK, const void* residual, long long residual_stride, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);
MV_API size_t mv_moe_prefill_workspace_bytes(int N, int NK, int H, int I, int E1, int w_dtype);

/* mv_moe_prefill with fp32 outputs: out32 [N, H] f32 (contiguous) receives residual + sum_k wts * expert outputs,
 * accumulated in fp32 and not rounded. For expert-parallel prefill, whose partial sums from several ranks are
 * added before the one rounding to bf16 (ming-voice has no counterpart: it is single-GPU, engine.py:34). Rows
 * [0, n_x) are read from x (row stride x_stride), rows [n_x, N) from x2 (row stride x2_stride; NULL when
 * n_x == N): a rank's own rows and the rows it received, each where it lies. max_ctas > 0 limits the persistent
 * GEMM to that many SMs; 0 = all SMs. */
MV_API int mv_moe_prefill_f32(const mv_moe_weights* w, const void* x, long long x_stride, int n_x, const void* x2,
                              long long x2_stride, const void* ids, int ids_dtype, const float* wts, int N, int NK,
                              const void* residual, long long residual_stride, float* out32, int max_ctas,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Expert-parallel prefill, the device side of one rank's dispatch and combine (ming-voice is single-GPU,
 * engine.py:34, so these have no counterpart there; they implement the exchange of an expert-parallel block whose
 * experts are placed by owner[E] (the rank holding routed expert e, or -1 when every rank holds it) and slot[E]
 * (its index in the holding rank's stacks). Pair ids / weights are [N, NK] int32 / f32 with the K routed pairs
 * first and the shared slots after them. Capacity `cap` pairs per peer; send_meta / recv_meta are
 * [world][cap + 1][2] int32: (slot, weight bits) per place and the place count in entry cap. None of them
 * synchronises the host.
 *  mv_ep_plan     one CTA: ids_local / wts_local [N, NK] (local slot, or -1 for a pair held by another rank),
 *                 pos [N, K] (d * cap + j for a pair sent to place j of peer d, else -1), send_src [world * cap]
 *                 (source row of each place), send_meta. Places follow token order per peer. More than cap pairs
 *                 for one peer: the excess pairs are dropped and workspace error 3 (capacity) is raised.
 *                 workspace: mv_ep_workspace_bytes() bytes, header zeroed.
 *  mv_ep_pack     send_rows [world * cap, H + 8] bf16 wire rows: row send_src of xn (row stride x_stride) and a
 *                 16-byte tail (slot, weight bits, in-use flag 1, 0) for every place in use; the other places get a
 *                 zero tail only. Rows and metadata then cross in one all-to-all.
 *  mv_ep_unpack   ids / wts [world * cap, NK] of the received wire rows recv_rows [world * cap, H + 8]: column 0 =
 *                 (slot, weight) of a place in use, the rest -1 / 0.
 *  mv_ep_narrow   out[i] = bf16(y[i]) for n values (n % 8 == 0): the received rows' fp32 outputs (one weighted
 *                 pair each) rounded once for the return exchange, halving its bytes.
 *  mv_ep_combine  out [N, H] bf16 = x + y_local + the returned outputs back[pos[n, k]] of n's remote pairs
 *                 (k order; back_dtype MV_F32 or MV_BF16, added in fp32), rounded once. */
MV_API size_t mv_ep_workspace_bytes(void);
MV_API int mv_ep_plan(const int* ids, const float* wts, int N, int NK, int K, const int* owner, const int* slot, int E,
                      int rank, int world, int cap, int* ids_local, float* wts_local, int* pos, int* send_src,
                      int* send_meta, void* workspace, size_t workspace_bytes, void* stream);
MV_API int mv_ep_pack(const void* xn, long long x_stride, int H, const int* send_src, const int* send_meta, int world,
                      int cap, void* send_rows, void* stream);
MV_API int mv_ep_unpack(const void* recv_rows, int H, int world, int cap, int NK, int* ids, float* wts, void* stream);
MV_API int mv_ep_narrow(const float* y, long long n, void* out, void* stream);
MV_API int mv_ep_combine(const void* x, long long x_stride, const float* y_local, const void* back, int back_dtype,
                         const int* pos, int N, int K, int H, void* out, void* stream);

/* Workspace for the fastest decode path (the tensor-core kernel, bf16 weights, H and I multiples of 128,
 * H <= 2048): larger than mv_moe_decode_workspace_bytes, which is the minimum (with the minimum the CUDA-core
 * kernel runs). Sized for M tokens with NK experts each from E1 stacked slots. */
MV_API size_t mv_moe_decode_workspace_bytes_tc(int M, int NK, int H, int I, int E1);

/* One MoE block: RMSNorm -> router -> routed + shared experts -> residual. */
typedef struct mv_block {
  mv_moe_weights experts;   /* stacked routed experts and the shared-expert slot(s) */
  const void* norm_w;       /* bf16 [H] post-attention RMSNorm weight (NULL: x is already normalised) */
  const void* router_w;     /* [E, H] router weight, f32 / bf16 / i8 */
  const void* router_scale; /* [E] row scales for an i8 router (f32 / bf16), else NULL */
  const float* router_bias; /* [E] f32 or NULL (sigmoid mode: added to the scores; softmax: to the logits) */
  float eps;
  int router_dtype;
  int router_scale_dtype;
  int E;                    /* routed experts (ids 0..E-1 of the stacks) */
  int top_k;
  int route_mode;           /* MV_ROUTE_SOFTMAX or MV_ROUTE_SIGMOID_GROUP */
  int n_group, topk_group;  /* sigmoid mode */
  int n_shared;             /* shared-expert slots appended to every token with weight 1 */
  int shared_id;            /* first shared slot (E in ming-voice's stacks) */
  int residual_from_x;      /* 1: out = x + MoE(norm(x)) (the decoder layer's residual); 0: out = MoE(...) */
  int pad0;
  double route_scale;       /* sigmoid mode: routed_scaling_factor */
  const struct mv_block* next; /* the block decoded after this one, or NULL. Decode only reads its router weight
                                  and RMSNorm weight pointers: they are prefetched into L2 while this block runs,
                                  so the next block's routing starts from L2 (a layer stack links block l to l+1). */
} mv_block;

/* Decode step of one block for M <= 16 tokens, each kernel cooperative and fused end to end: replaces the patched
 * single-token MoE forward (engine.py:371-386: fused_ops.moe_route followed by fused_moe.fused_moe_decode),
 * including the RMSNorm before it (engine.py:229) and the decoder layer's residual. One launch, except that the
 * one-token kernel runs once per token for bf16 M = 2 and int8 M >= 2 (the block is per-token work, and there
 * that is faster). x [M, H] bf16 contiguous, out [M, H] bf16.
 * Optional router outputs (each may be NULL): logits_out [M, E] f32, ids_out [M, top_k + n_shared]
 * (i32/i64), wts_out [M, top_k + n_shared] f32 -- the aux the reference block returns.
 * workspace: mv_block_decode_workspace_bytes(M, top_k + n_shared, I, E) bytes, zero-initialised. */
MV_API int mv_block_decode(const mv_block* b, const void* x, int M, void* out, float* logits_out, void* ids_out,
                           int ids_dtype, float* wts_out, void* workspace, size_t workspace_bytes, void* stream);
MV_API size_t mv_block_decode_workspace_bytes(int M, int n_experts_per_token, int I, int E);
/* Workspace for the fastest mv_block_decode path for up to M tokens (see mv_moe_decode_workspace_bytes_tc). */
MV_API size_t mv_block_decode_workspace_bytes_tc(const mv_block* b, int M);

/* Padded-bucket prefill: sets ids[r, k] = -1 ("no pair", skipped by mv_moe_prefill) for every row
 * r >= *n_valid of the [N, NK] expert ids (i32 or i64). n_valid is a device int read by the kernel, so a CUDA
 * graph captured once for a padded length N serves every prompt length up to N: ming-voice pads short prompts
 * to 32 / 64 / 128 tokens and replays one graph per length (engine.py:716-757, :950-961), where the padded rows
 * also run through the experts; here they are dropped from the expert sort. */
MV_API int mv_mask_pad_rows(void* ids, int ids_dtype, int N, int NK, const int* n_valid, void* stream);

/* mv_block_decode without a caller workspace: no counterpart in the reference (its Triton launches take
 * torch-allocated buffers). For callers that cannot allocate device memory or keep a workspace -- a C/FFI
 * host without a device allocator, or code that must not call cudaMalloc while a stream is captured.
 * The scratch is a static 1 MiB device array per device; the first call on a device (with it current)
 * looks its address up, so make that call before any stream capture. Calls whose scratch need
 * (mv_block_decode_workspace_bytes) exceeds 1 MiB are rejected with MV_ERR_WORKSPACE. Every call runs the
 * CUDA-core decode kernels (the one-token kernel, once per token where mv_block_decode would, or the general
 * one): the tensor-core kernel's layout (3.4 MB at M = 1 up to 50 MB at M = 16 for H=2048, I=1408, 64 + 2
 * slots) does not fit the static scratch. Each call clears the
 * scratch's 256-byte header (barrier counters, error word) on `stream` before its launch.
 * status_out (device or pinned host memory, 2 x u32, may be NULL) receives the call's device-side error
 * code and location, as mv_workspace_status reports them. One scratch per device: calls that can run
 * concurrently on one device race; keep them on one stream or order them with events. Allocates nothing. */
MV_API int mv_block_decode_noalloc(const mv_block* b, const void* x, int M, void* out, float* logits_out,
                                   void* ids_out, int ids_dtype, float* wts_out, unsigned int* status_out,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINGMOE_H */
