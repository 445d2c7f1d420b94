/*
 * fnx_gemv.h — C ABI of the B200 (sm_100a) weight-only quantized GEMV library.
 *
 * Drop-in boundary for the reference's decode/verify GEMV operators.  Every entry point
 * takes raw device pointers, element strides and sizes, plus the CUDA stream to launch
 * on; nothing here allocates device memory.  Scratch buffers are owned by the caller
 * and described by fnx_workspace / fnx_moe_workspace (sizes from the *_bytes queries).
 *
 * Return codes: FNX_OK on success; FNX_EINVAL for an argument the reference would
 * reject (its `assert`s and `ValueError`s); FNX_EUNSUPPORTED for a shape this build does
 * not tile (the caller keeps its fallback, as the reference's `apply_into` returning
 * None does); FNX_ECUDA when the launch itself failed.  fnx_last_error() describes the
 * last failure of the calling thread.
 *
 * Reference interfaces replaced (paths inside the reference repository):
 *   fnx_w8a16_gemv           kernels/sglang/srt/layers/quantization/w8a16_gemv.py:642-666
 *                            (w8a16_gemv) and :826-847 (bf16_gemv, w_dtype FNX_W_BF16)
 *   fnx_w8a16_gemv_silu_mul  w8a16_gemv.py:1009-1061 (w8a16_gemv_silu_mul)
 *   fnx_w8a16_gemv_norm_gated  w8a16_gemv.py:780-823 (w8a16_gemv_norm_gated; the norm
 *                            prologue of the kernel at :186-190, :220-233, :246-255)
 *   fnx_router_gemv_topk     kernels/sglang/srt/layers/moe/router_gemv.py:10-93 (router_gemv,
 *                            topk = 0) fused with the softmax top-k below (topk > 0)
 *   fnx_softmax_topk         route_softmax_fast, patches/sglang/series/0110-moe-router-packed-
 *                            key-softmax-top-k-SGLANG_ROUTER_FA.patch:27-184 as changed by 0111
 *   fnx_draft_topk1          draft_topk1_postprocess (patches/sglang/series/0016-spec-remove-
 *                            per-draft-step-glue-in-the-topk-1-chain-.patch:46-73: argmax,
 *                            hot-vocabulary map, draft_tokens column, positions + 1)
 *   fnx_draft_head_topk1     the draft head GEMV with the same step fused into its argmax
 *   fnx_w8a16_gemv_vocab_sharded  the vocab-sharded lm_head with the greedy token's MAX
 *                            reduction over ranks fused into the GEMV (the NCCL all-reduce
 *                            of argmax keys it replaces has no counterpart in the reference,
 *                            which serves one GPU); fnx_peer_* / fnx_ipc_* set its buffers up
 *   fnx_w4a16_nvfp4_gemv     kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:342-401
 *   fnx_nvfp4_quantize / fnx_nvfp4_dequantize  w4a16_nvfp4_gemv.py:426-510 (quantize_nvfp4,
 *                            dequantize_nvfp4; the load-time codec)
 *   fnx_moe_gemv             patches/sglang/series/0112-DG1-one-token-draft-MoE-as-a-W4A16-
 *                            NVFP4-Triton-GEMV.patch:328-386 (draft_moe_gemv), generalised
 *                            from one token to M <= 16
 *   fnx_argmax_decode        greedy top-1 over the logits buffer (the consumer of
 *                            patches/sglang/series/0032-...patch:188-215's lm_head output)
 *   fnx_*_workspace_bytes    w8a16_gemv.py:325-395 (split-K scratch, prealloc) and
 *                            0112-...patch:307-325 (make_workspace)
 */
#ifndef FNX_GEMV_H_
#define FNX_GEMV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t; kept opaque so the header needs no CUDA include. */
typedef void* fnx_stream_t;

#define FNX_OK 0
#define FNX_EINVAL 1
#define FNX_ECUDA 2
#define FNX_EUNSUPPORTED 3

/* Weight element formats. */
#define FNX_W_INT8 0      /* int8, exact in the fp16 A operand                  */
#define FNX_W_FP8_E4M3 1  /* float8_e4m3fn (the reference's W8A16 weights)      */
#define FNX_W_BF16 2      /* bf16 (bf16_gemv)                                   */
#define FNX_W_NVFP4 3     /* packed e2m1 pairs + e4m3 block-16 scales           */

/* Output scale formats: applied per output row after the k reduction. */
#define FNX_SCALE_NONE 0
#define FNX_SCALE_F32_SCALAR 1
#define FNX_SCALE_F32_ROW 2
#define FNX_SCALE_BF16_SCALAR 3
#define FNX_SCALE_BF16_ROW 4

/* Maximum tokens per call (the reference asserts M <= 16, w8a16_gemv.py:658). */
#define FNX_MAX_M 16

/* Device error codes.  A device-side wait that runs out of time (2 s unless stated
 * otherwise) records the first such code of a call in the workspace's error_flag, leaves
 * its loop, and the launch completes with wrong results; the host reads the flag (after
 * the work has finished) and clears it.  Nothing on the device clears it. */
#define FNX_DEVERR_WAIT_FULL 1     /* a consumer waited for a weight stage          */
#define FNX_DEVERR_WAIT_EMPTY 2    /* the producer waited for a free stage          */
#define FNX_DEVERR_WAIT_RED 3      /* an epilogue waited for consumer partials      */
#define FNX_DEVERR_WAIT_RFREE 4    /* a consumer waited for a free reduction slot   */
#define FNX_DEVERR_DRAIN 5         /* in-flight copies did not land before exit     */
#define FNX_DEVERR_WAIT_X 6        /* the activation rows did not arrive            */
#define FNX_DEVERR_WAIT_PEER 7     /* another rank did not publish its greedy key   */
#define FNX_DEVERR_PEER_DESYNC 8   /* another rank is two or more calls ahead       */
#define FNX_DEVERR_ROUTES 9        /* a routing table the kernel cannot hold        */
#define FNX_DEVERR_WAIT_EXPERT 10  /* a down projection waited for its expert's act */
#define FNX_DEVERR_RING 11         /* a launch whose ring stages the waits cannot order */

/* Split-K and argmax scratch of the dense GEMVs.  Counters and keys must be zero when
 * first used; every launch leaves them zero again (self-resetting, graph-replay safe).
 * Two launches that share one workspace must not run concurrently (the reference's
 * scratch_slot rule, w8a16_gemv.py:337-345). */
typedef struct fnx_workspace {
  float* partials;                 /* split-K fp32 partials                       */
  int64_t partial_floats;          /* capacity of `partials`                      */
  unsigned int* counters;          /* split-K per-tile arrival counters            */
  int64_t n_counters;
  unsigned long long* argmax_keys; /* FNX_MAX_M keys                              */
  unsigned int* argmax_count;      /* one CTA arrival counter                     */
  int* error_flag;                 /* device error code (0 = none), or NULL: a wait
                                      that exceeded its time limit records its code */
} fnx_workspace;

/* Optional launch geometry override (NULL = built-in planner).  A work unit is
 * `groups` 16-row tiles x (K / ksplit).  warps: consumer warps per CTA (<= 16);
 * chunks_per_warp: 64-byte row chunks each consumer streams per unit (1, 2, 4 or 8);
 * groups: 16-row tiles per unit (1..4, dividing warps); ksplit: k splits (separate
 * units, summed by the last split); grid: CTAs (0 = one persistent wave).
 * (warps / groups) * chunks_per_warp * ksplit must equal K / chunk, chunk = 64 B of a row
 * (64 k for int8/fp8, 32 for bf16, 128 for NVFP4). */
typedef struct fnx_gemv_cfg {
  int warps;
  int chunks_per_warp;
  int groups;
  int ksplit;
  int grid;
} fnx_gemv_cfg;

/* Which contraction the dense GEMV entry points use when cfg is NULL (process-wide):
 *  FNX_DENSE_PATH_AUTO     tcgen05 tensor-core form (A dequantised into tensor memory,
 *                          stream-K over 128-row blocks) for int8 / fp8 weights at M > 8,
 *                          mma.sync elsewhere (the default);
 *  FNX_DENSE_PATH_MMA      mma.sync form only;
 *  FNX_DENSE_PATH_TCGEN05  tcgen05 form wherever it applies, at every M.
 * The tcgen05 form needs K a multiple of 128 and a workspace of >= 4096 * SMs partial
 * floats and >= 4 * SMs counters; it is skipped (mma.sync form) for the fused SiLU,
 * gated-norm and draft-chain variants and when a cfg is given.  *previous (may be
 * NULL) receives the earlier setting.  No counterpart in the reference (its GEMV is one
 * Triton kernel). */
#define FNX_DENSE_PATH_AUTO 0
#define FNX_DENSE_PATH_MMA 1
#define FNX_DENSE_PATH_TCGEN05 2
int fnx_set_dense_path(int path, int* previous);

/* Planner used when cfg is NULL (exposed for tests and workspace sizing). */
int fnx_plan_gemv(int M, int N, int K, int w_dtype, int fused_silu, int argmax,
                  fnx_gemv_cfg* out);

/* Workspace floats / counters a call with this plan needs. */
int fnx_gemv_workspace_need(int M, int N, int K, int w_dtype, int fused_silu,
                            const fnx_gemv_cfg* cfg, int64_t* partial_floats,
                            int64_t* n_counters);

/*
 * y[m, n] = bf16( (sum_k w[n, k] * x[m, k]) * scale[n] )      m < M <= 16, n < N
 *
 * x: bf16 [M, K], row stride ldx elements (16-byte aligned rows).
 * w: [N, K] of w_dtype (FNX_W_INT8 / FNX_W_FP8_E4M3 / FNX_W_BF16), row stride ldw BYTES.
 * scale: per-row or scalar scale (scale_kind), bf16 scales are widened exactly.
 * y: [M, N] (or columns [0, split_n) when y2 != NULL), row stride ldy elements;
 *    out_f32 != 0 stores the bf16-rounded value widened to fp32 (bit-identical to a bf16
 *    result followed by a copy into an fp32 buffer, w8a16_gemv.py:599-618).
 * y2: columns [split_n, N) at column n - split_n (two-destination store), or NULL.
 * argmax_out: int64 [M] greedy top-1 row of the bf16-rounded logits (lowest row on
 *    ties), or NULL.  row_offset is added to the row ids (vocab shards);
 *    argmax_key_out (uint64 [M], may be NULL) receives the raw keys for a cross-shard
 *    MAX reduction followed by fnx_argmax_decode.
 */
int fnx_w8a16_gemv(const void* x, int64_t ldx, const void* w, int64_t ldw, int w_dtype,
                   const void* scale, int scale_kind, void* y, int64_t ldy, void* y2,
                   int64_t ldy2, int64_t split_n, int out_f32, int64_t* argmax_out,
                   unsigned long long* argmax_key_out, int64_t row_offset, int M, int N,
                   int K, const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                   fnx_stream_t stream);

/*
 * y[m, j] = bf16( silu(g) * u ),  g = x_m . w[j] * scale[j],  u = x_m . w[H + j] * scale[H + j]
 * w: [2H, K] with the gate half first (MergedColumnParallelLinear [gate|up]); scale per
 * row (2H entries).  y: bf16 [M, H].
 */
int fnx_w8a16_gemv_silu_mul(const void* x, int64_t ldx, const void* w, int64_t ldw,
                            int w_dtype, const void* scale, int scale_kind, void* y,
                            int64_t ldy, int M, int H, int K, const fnx_gemv_cfg* cfg,
                            const fnx_workspace* ws, int pdl, fnx_stream_t stream);

/*
 * y = (gated_rms_norm(x, z) @ w^T) * scale in one launch.  x, z: bf16 [M, K], rows
 * 16-byte aligned (strides ldx, ldz elements).  Each contiguous group_size slice of a
 * row is its own RMS group (RMSNormGated(group_size, norm_before_gate=True)):
 *   xn[m, k] = bf16( x[m, k] * rsqrt(mean_group(x^2) + eps) * norm_weight[k % G] * gate )
 *   gate = z * sigmoid(z) (sigmoid_gate == 0, silu) or sigmoid(z) (sigmoid_gate != 0)
 * norm_weight: [group_size] bf16 (norm_weight_f32 == 0) or fp32, 16-byte aligned.
 * group_size: a power of two in [8, 256] dividing K (FNX_EUNSUPPORTED otherwise).
 * y: bf16, or fp32 holding bf16-rounded values (out_f32), [M, ldy].  Remaining
 * arguments as fnx_w8a16_gemv; the split-K workspace need is fnx_gemv_workspace_need's
 * for the same M, N, K and w_dtype.
 */
int fnx_w8a16_gemv_norm_gated(const void* x, int64_t ldx, const void* z, int64_t ldz,
                              const void* norm_weight, int norm_weight_f32, int group_size,
                              float eps, int sigmoid_gate, const void* w, int64_t ldw,
                              int w_dtype, const void* scale, int scale_kind, void* y,
                              int64_t ldy, int out_f32, int M, int N, int K,
                              const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                              fnx_stream_t stream);

/*
 * MoE router.  logits[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]) in fp32 (bf16 inputs,
 * no rounding of the result): x [M, K] and w [N, K] bf16 with 16-byte aligned rows
 * (strides ldx, ldw in elements), bias bf16 [N] or NULL, 1 <= M <= 16, K % 128 == 0,
 * N % 32 == 0.  With topk > 0 (<= 32, N <= 512) the same launch also writes the softmax
 * top-k routing table (fnx_softmax_topk's rule) to topk_weights (fp32) and topk_ids
 * (int32), both [M, ldk]; it then uses ws->counters[0] (zero between calls, left at zero)
 * and, when logits is NULL, ws->partials as the logits buffer.
 */
int fnx_router_gemv_topk(const void* x, int64_t ldx, const void* w, int64_t ldw,
                         const void* bias, float* logits, int64_t ldl, float* topk_weights,
                         int32_t* topk_ids, int64_t ldk, int M, int N, int K, int topk,
                         int renormalize, const fnx_workspace* ws, int pdl,
                         fnx_stream_t stream);

/*
 * Softmax top-k routing of given logits (bf16, or fp32 with scores_f32) plus an optional
 * fp32 bias [N]: per row, weight[n] = exp(l[n] - max) / sum_n' exp(l[n'] - max); the topk
 * largest l (NaN ranks as -1e30, -0.0 as +0.0; the lowest expert id wins ties) in
 * descending order; with renormalize the picked weights are divided by their sum when it
 * is positive.  N <= 512, topk <= min(N, 32).
 */
int fnx_softmax_topk(const void* scores, int64_t lds, int scores_f32, const float* bias,
                     float* topk_weights, int32_t* topk_ids, int64_t ldk, int M, int N,
                     int topk, int renormalize, int pdl, fnx_stream_t stream);

/*
 * Greedy draft step on draft logits (fp32, or bf16 with logits_f32 == 0) [M, ldl], V
 * columns, M <= 16: per row the argmax column (lowest on ties), mapped through
 * hot_token_id (int64 [V], NULL: the column itself) to a token that is written to
 * topk_index[m] and draft_tokens[m * ld_draft + draft_col]; topk_p[m] = 1 and
 * positions[m] += 1.  Any of the four outputs may be NULL (not all).  Uses the workspace's
 * argmax keys and counter (zero between calls, left at zero).
 */
int fnx_draft_topk1(const void* logits, int64_t ldl, int logits_f32, int M, int V,
                    const int64_t* hot_token_id, int64_t* positions, int64_t* draft_tokens,
                    int64_t ld_draft, int draft_col, int64_t* topk_index, float* topk_p,
                    const fnx_workspace* ws, int pdl, fnx_stream_t stream);

/*
 * The draft head in one launch: logits = fnx_w8a16_gemv(x, w, scale) (bf16, or fp32
 * holding bf16 values with out_f32) and fnx_draft_topk1's step on their bf16-rounded
 * values, done by the GEMV's last CTA.  Arguments as those two entry points.
 */
int fnx_draft_head_topk1(const void* x, int64_t ldx, const void* w, int64_t ldw, int w_dtype,
                         const void* scale, int scale_kind, void* logits, int64_t ldl,
                         int out_f32, int M, int N, int K, const int64_t* hot_token_id,
                         int64_t* positions, int64_t* draft_tokens, int64_t ld_draft,
                         int draft_col, int64_t* topk_index, float* topk_p,
                         const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                         fnx_stream_t stream);

/*
 * Vocab-sharded lm_head, one process per GPU on one node.  Each rank allocates one
 * FNX_PEER_BUFFER_BYTES device buffer (fnx_peer_alloc, zeroed), exports it
 * (fnx_ipc_get_handle, FNX_IPC_HANDLE_BYTES), opens the other ranks' handles
 * (fnx_ipc_open) and records all of them (fnx_peer_setup, bufs[r] = rank r's buffer as
 * mapped in this process, bufs[rank] = its own).  fnx_w8a16_gemv_vocab_sharded then
 * computes its shard's logits like fnx_w8a16_gemv (rows row_offset + n) and, in the same
 * launch, exchanges the greedy keys with every rank over NVLink and writes the global
 * greedy row to argmax_out on every rank.  All ranks must make the same sequence of calls;
 * a rank that waits more than 2 s for the others records an error code in ws->error_flag
 * and returns its own shard's token.  Calls on one rank are ordered on one stream.
 * At most FNX_MAX_PEERS ranks, M <= 16.
 */
#define FNX_PEER_BUFFER_BYTES 4096
#define FNX_IPC_HANDLE_BYTES 64
#define FNX_MAX_PEERS 8
int fnx_peer_alloc(void** buf);
int fnx_peer_free(void* buf);
int fnx_ipc_get_handle(void* buf, void* handle);
int fnx_ipc_open(const void* handle, void** buf);
int fnx_ipc_close(void* buf);
int fnx_peer_setup(void* local, void* const* bufs, int world, int rank);
/* Limit of the in-kernel wait for the other ranks' keys, in nanoseconds (0 = the 2 s
 * default); set after fnx_peer_setup, between calls.  An expired wait records
 * FNX_DEVERR_WAIT_PEER and the rank keeps its own shard's token; a rank that finds
 * another two or more calls ahead records FNX_DEVERR_PEER_DESYNC and does the same. */
int fnx_peer_set_wait_limit(void* local, int64_t wait_ns);
int fnx_w8a16_gemv_vocab_sharded(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                 int w_dtype, const void* scale, int scale_kind, void* y,
                                 int64_t ldy, int out_f32, int64_t* argmax_out,
                                 int64_t row_offset, int M, int N, int K, void* peer_buf,
                                 const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                                 fnx_stream_t stream);

/*
 * y[m, n] = bf16( (sum_k e2m1(wq[n, k]) * e4m3(bs[n, k / 16]) * x[m, k]) * gscale )
 * wq: uint8 [N, K/2], low nibble = even k, row stride ldwq bytes.
 * bs: e4m3 bytes [N, K/16] (linear layout), row stride ldbs bytes.
 * gscale: fp32 scalar (gscale_per_row == 0) or [N]; the plain global scale (no 2^14
 * factor: this library decodes e2m1 natively).
 * Remaining arguments as fnx_w8a16_gemv.
 */
int fnx_w4a16_nvfp4_gemv(const void* x, int64_t ldx, const void* wq, int64_t ldwq,
                         const void* bs, int64_t ldbs, const float* gscale,
                         int gscale_per_row, void* y, int64_t ldy, void* y2, int64_t ldy2,
                         int64_t split_n, int out_f32, int64_t* argmax_out,
                         unsigned long long* argmax_key_out, int64_t row_offset, int M,
                         int N, int K, const fnx_gemv_cfg* cfg, const fnx_workspace* ws,
                         int pdl, fnx_stream_t stream);

/*
 * NVFP4 load-time codec on the GPU (quantize_nvfp4 / dequantize_nvfp4,
 * kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:426-510).
 * fnx_nvfp4_quantize: w [N, K] bf16 (w_f32 == 0) or fp32, row stride ldw elements ->
 *   wq uint8 [N, K/2] (low nibble = even k), bs e4m3 bytes [N, K/16], gscale[0] =
 *   max(amax|w| / 2688, 1e-30); the codes equal the reference's bit for bit.  scratch: one
 *   u32 of device memory (cleared by the call).  K % 16 == 0.
 * fnx_nvfp4_dequantize: -> out [N, K] fp32 (out_f32) or bf16, value = e2m1(code) *
 *   (e4m3(bs) * gscale), gscale scalar or [N] (gscale_per_row).
 */
int fnx_nvfp4_quantize(const void* w, int64_t ldw, int w_f32, int N, int K, void* wq,
                       int64_t ldwq, void* bs, int64_t ldbs, float* gscale,
                       unsigned int* scratch, fnx_stream_t stream);
int fnx_nvfp4_dequantize(const void* wq, int64_t ldwq, const void* bs, int64_t ldbs,
                         const float* gscale, int gscale_per_row, void* out, int64_t ldo,
                         int out_f32, int N, int K, fnx_stream_t stream);

/* NVFP4 expert bank in the server layout (ModelOptNvFp4FusedMoEMethod after
 * process_weights_after_loading, 0112-...patch:68-76). */
typedef struct fnx_moe_weights {
  const void* w13;          /* uint8 [E, 2I, H/2]: rows [up(I); gate(I)]               */
  const void* w13_scale;    /* e4m3 [E, 2I, H/16], 128x4 swizzled if scales_swizzled    */
  const float* w13_gscale;  /* global scale of expert e at w13_gscale[e * stride]      */
  int64_t w13_gscale_stride;
  const void* w2;           /* uint8 [E, H, I/2]                                        */
  const void* w2_scale;     /* e4m3 [E, H, I/16]                                        */
  const float* w2_gscale;
  int64_t w2_gscale_stride;
  int num_experts;          /* experts held by these tensors                           */
  int expert_offset;        /* global id of local expert 0 (expert-parallel shards)    */
  int hidden;               /* H */
  int inter;                /* I */
  int scales_swizzled;
} fnx_moe_weights;

typedef struct fnx_moe_workspace {
  void* act;                     /* bf16 act rows of the routes (bytes: sizes.act)      */
  float* partials;               /* fp32 [max_m * (max_routes + 1), H]                  */
  int* error_flag;               /* device error code, or NULL                          */
  int max_m;                     /* capacity the buffers were sized for                 */
  int max_routes;
  unsigned int* counters;        /* sizes.counters u32, zero when first used (every call */
                                 /* leaves them zero), or NULL: the three-launch form    */
  int64_t n_counters;
} fnx_moe_workspace;

/* Sizes of the fnx_moe_workspace buffers for (max_m, max_routes, E, H, I): act and
 * partials in bytes, counters in u32 entries; also checks that the library tiles these
 * shapes (FNX_EUNSUPPORTED otherwise).  num_experts is the largest expert count the
 * workspace will serve. */
typedef struct fnx_moe_workspace_sizes {
  int64_t act, partials, counters;
} fnx_moe_workspace_sizes;

int fnx_moe_workspace_bytes(int max_m, int max_routes, int num_experts, int H, int I,
                            fnx_moe_workspace_sizes* out);

/* The form fnx_moe_gemv takes for (M, R, E, H, I) with a workspace that has counters:
 * *fused = 2 for the decode-width one-launch layer and 1 for the general one, with its
 * weight-ring stages, consumer groups and dynamic shared memory; *fused = 0 (and zeros)
 * for the three-launch layer.  Exposed for tests and launch accounting. */
int fnx_plan_moe(int M, int R, int E, int H, int I, int* fused, int* stages, int* groups,
                 int64_t* smem_bytes);

/* Which one-launch MoE layer fnx_moe_gemv uses (process-wide), given a workspace with
 * counters:
 *  FNX_MOE_PATH_AUTO   the decode-width layer (moe_lean_kernel: every SM one CTA, each
 *                      CTA's share of the layer's weight bytes in flight at once, the route
 *                      sum done by the CTA that owns the output rows) for M = 1 with
 *                      swizzled, 16-byte aligned block scales, H and I multiples of 256,
 *                      I <= 512, H <= 2048; the general one-launch layer otherwise (the
 *                      default);
 *  FNX_MOE_PATH_FUSED  the general one-launch layer at every M.
 * fnx_plan_moe reports *fused = 2 for the decode-width layer (assuming swizzled scales).
 * *previous (may be NULL) receives the earlier setting.  No counterpart in the reference
 * (its one-token MoE is two Triton launches). */
#define FNX_MOE_PATH_AUTO 0
#define FNX_MOE_PATH_FUSED 1
int fnx_set_moe_path(int path, int* previous);

/*
 * out[t, :] = sum_r topk_weights[t, r] * expert(topk_ids[t, r])(x[t]) [+ shared(x[t])]
 * expert(x) = w2 @ (silu(gate(x)) * up(x)); act rounded to bf16 between the GEMVs; the
 * route sum in route order, then the shared expert (deterministic, no float atomics).
 * With ws->counters (and H, I among the fused tilings: 2048 x 512, 2560 x 640,
 * 1024 x 256, 2048 x 1024) the layer runs as ONE launch whose CTAs all run at once, one
 * per SM; otherwise as three launches (gate/up, down, route sum).  Any routing is
 * served: repeated ids and any number of routes per expert (the fused form; the
 * three-launch form holds at most 8 routes per expert at M <= 8, 16 above, and records
 * FNX_DEVERR_ROUTES for more).
 * x: bf16 [M, H] (row stride ldx); topk_ids int32 [M, R] (ids < 0 skipped);
 * topk_weights fp32 [M, R]; shared: an always-on expert with weight 1.0 (num_experts 1),
 * or NULL.  out: bf16 [M, H] (row stride ldo), or the fp32 partial sum of this expert
 * slice when out_f32 != 0 (for a cross-rank SUM).
 */
int fnx_moe_gemv(const void* x, int64_t ldx, const int32_t* topk_ids,
                 const float* topk_weights, int M, int R, const fnx_moe_weights* experts,
                 const fnx_moe_weights* shared, void* out, int64_t ldo, int out_f32,
                 const fnx_moe_workspace* ws, int pdl, fnx_stream_t stream);

/* out[t] = row id encoded in keys[t] (after a cross-shard MAX reduction of the keys). */
int fnx_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                      fnx_stream_t stream);

/*
 * fnx_w8a16_gemv without a caller workspace: the argmax keys, split-K partials and
 * counters live in one static device array of the library (FNX_STATIC_SCRATCH_BYTES
 * per device), so the call allocates no device memory.  No counterpart in the
 * reference, whose Triton launches allocate their scratch through torch.
 *
 * - Arguments and results are those of fnx_w8a16_gemv (ws omitted).
 * - A plan whose split-K scratch exceeds FNX_STATIC_PARTIAL_FLOATS partial floats or
 *   FNX_STATIC_COUNTERS counters is rejected with FNX_EUNSUPPORTED.
 * - The first call on a device resolves the array's address (one-time setup with
 *   that device current); make that first call before capturing a stream.
 * - All calls on a device share the array, which keeps the previous call's contents:
 *   calls that may run at the same time (different streams without ordering) race on
 *   it.  The argmax keys, the argmax counter and the split-K counters must be zero when
 *   the kernel starts; each call clears them with a memset on its stream first.
 * - A device-side wait that gives up records its code in the array's error word.  Each
 *   call clears the word before its launch (with the keys and counters), so after the
 *   call has finished fnx_static_ws_error reports whether that call's waits all ended.
 */
#define FNX_STATIC_PARTIAL_FLOATS (256 * 1024)
#define FNX_STATIC_COUNTERS 2048
#define FNX_STATIC_SCRATCH_BYTES (4096 + 4 * FNX_STATIC_COUNTERS + 4 * FNX_STATIC_PARTIAL_FLOATS)
int fnx_w8a16_gemv_static_ws(const void* x, int64_t ldx, const void* w, int64_t ldw,
                             int w_dtype, const void* scale, int scale_kind, void* y,
                             int64_t ldy, void* y2, int64_t ldy2, int64_t split_n, int out_f32,
                             int64_t* argmax_out, unsigned long long* argmax_key_out,
                             int64_t row_offset, int M, int N, int K, const fnx_gemv_cfg* cfg,
                             int pdl, fnx_stream_t stream);
/* The error word of fnx_w8a16_gemv_static_ws's array on the current device, read after
 * the work on `stream` has finished (this call synchronises the stream); clear != 0 sets
 * it back to zero.  *code receives an FNX_DEVERR_* value, or 0. */
int fnx_static_ws_error(int clear, fnx_stream_t stream, int* code);

/* Description of the last error of the calling thread ("" if none). */
const char* fnx_last_error(void);

/* Library version string. */
const char* fnx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FNX_GEMV_H_ */
