/*
 * dsm.h -- C ABI of libdsm, a B200 (sm_100a) implementation of the DeepSeek-V4 DSpark
 * draft-layer Mixture-of-Experts block (router, token permutation, grouped quantised
 * expert SwiGLU products, weighted combine and shared expert).
 *
 * Conventions
 *   - Every pointer argument is a device pointer unless stated otherwise; all buffers are
 *     owned by the caller. No entry point allocates device memory: scratch space comes
 *     from a caller-provided workspace whose size a *_workspace_bytes query returns.
 *   - Every call is ordered on the given CUDA stream (passed as void*, a cudaStream_t;
 *     NULL is the legacy default stream) and returns immediately.
 *   - Return value: DSM_OK (0) or a nonzero dsm status. No C++ exception crosses the ABI.
 *     dsm_last_error_message() gives a description of the last failure on this thread.
 *   - Data-dependent faults that can only be seen on the device (an expert id outside
 *     [0, n_experts), a token id outside the hash table, a pipeline wait that ran out of
 *     its time budget) are recorded in a device-side error word that
 *     dsm_device_error() reads; the kernel skips the offending access instead of faulting.
 *
 * Reference interface each entry point replaces (dspark_mlx, file:line):
 *   dsm_router          Gate.__call__                       model/moe.py:62-79
 *   dsm_permute         (implicit in gather_mm rhs_indices)  model/moe.py:145-148
 *   dsm_stage_rows      gather_mm lhs broadcast x[N,1,1,dim]  model/moe.py:158
 *   dsm_expert_gate_up  gather_mm / gather_qmm w1, w3 + _swiglu  model/moe.py:37-44,138-147
 *   dsm_expert_down     gather_mm / gather_qmm w2             model/moe.py:143,148
 *   dsm_combine         sum_k o * weights + shared, cast      model/moe.py:159-161
 *   dsm_moe_forward     MoE.__call__                          model/moe.py:151-161
 *   dsm_affine_quantize mx.quantize in MoE.quantize           model/moe.py:124-130
 *   dsm_pack_weights    stacked [E,out,in] expert weights      loading.py:88-100 (+103-114)
 *   dsm_hc_pre_norm     hc_pre + ffn_norm before the MoE       model/hyper.py:24-42, kernels.py:60-85,
 *                       (DSparkBlock.__call__, block.py:84-85) model/norm_rope.py:22-39
 *   dsm_hc_post         hc_post after the MoE (block.py:86)    model/hyper.py:45-51
 *   dsm_dense_mlp       Qwen3MLP.__call__ / Expert.__call__    arch/qwen3.py:146-154, model/moe.py:82-97
 *   dsm_linear          nn.Linear over packed weights (the LM head, drafter.py:29, block.py:112)
 *   dsm_hc_head_norm    hc_head + the head's RMSNorm            model/hyper.py:52-67, block.py:111-112
 *   dsm_markov_head     DSparkMarkovHead.__call__              model/heads.py:26-30
 *   dsm_draft_head      DSparkBlock.forward_head + LM head      model/block.py:103-116, recipe.py:21-63,
 *                       (Markov walk, sampler, confidence)     model/heads.py:11-49
 *   dsm_rows_norm_rope, dsm_q_head_norm_rope, dsm_kv_window_write, dsm_sparse_attn, dsm_round_rows:
 *                       DSparkAttention.__call__ / advance_window around dsm_linear
 *                       (model/attention.py:27-142, kernels.py:20-57, norm_rope.py:22-77)
 *   dsm_qkv_norm_rope, dsm_gqa_attn: Qwen3DSparkAttention.__call__ / context_kv /
 *                       attend_cached around dsm_linear (arch/qwen3.py:64-143)
 *   dsm_add_rms_norm    the residual adds and RMSNorms of Qwen3DSparkLayer (arch/qwen3.py:157-176)
 *   dsm_gather_rows     the draft block's embedding rows (block.py:97-101)
 *   dsm_ep_*            expert parallelism over peer stores; the reference runs on one device
 *                       (tests/reference_model.py:55-56 forces world_size 1) and has no
 *                       counterpart.
 */
#ifndef DSM_H_
#define DSM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSM_ABI_VERSION 1

/* status codes */
#define DSM_OK 0
#define DSM_ERR_INVALID_ARGUMENT 1
#define DSM_ERR_UNSUPPORTED 2
#define DSM_ERR_WORKSPACE 3
#define DSM_ERR_CUDA 4
/* device-side error word values */
#define DSM_DEV_ERR_EXPERT_RANGE 0x10
#define DSM_DEV_ERR_TOKEN_RANGE 0x11
#define DSM_DEV_ERR_PIPELINE_TIMEOUT 0x12
#define DSM_DEV_ERR_PEER_TIMEOUT 0x13   /* an expert-parallel peer did not signal within ~2 s */
#define DSM_DEV_ERR_CAPACITY 0x14       /* more expert-parallel rows than the exchange buffer holds */

/* element types */
#define DSM_DT_F32 0
#define DSM_DT_BF16 1
#define DSM_DT_F16 2
#define DSM_DT_I32 3
#define DSM_DT_I64 4

/* Gate.score_func (model/config.py:33) */
#define DSM_SCORE_SOFTMAX 0
#define DSM_SCORE_SIGMOID 1
#define DSM_SCORE_SQRTSOFTPLUS 2

/* expert weight storage formats */
#define DSM_WFMT_F16 0      /* bf16/fp32 weights held as f16 with a per-expert power-of-two scale */
#define DSM_WFMT_FP8_B128 1 /* e4m3 codes, fp32 scale per 128x128 block (loading.py:103-107) */
#define DSM_WFMT_FP4_G32 2  /* e2m1 codes, e4m3 scale per 32 along K, fp32 per expert (loading.py:110-114) */
#define DSM_WFMT_AFFINE8 3  /* MLX affine 8-bit: q*scale+bias per group (moe.py:124-130) */
#define DSM_WFMT_AFFINE4 4  /* MLX affine 4-bit */

/* activation applied between the gate/up and down products */
#define DSM_ACT_SWIGLU_CLAMP 0 /* _swiglu, fp32, asymmetric clamp at swiglu_limit (moe.py:37-44) */
#define DSM_ACT_SILU_MUL_BF16 1 /* silu(g)*u with every op rounded to bf16 (arch/qwen3.py:153-154) */

int dsm_abi_version(void);
const char* dsm_status_string(int status);
const char* dsm_last_error_message(void);

/* Read (and optionally clear) the device-side error word of the current device.
 * Synchronises the stream. *code receives 0 or a DSM_DEV_ERR_* value. */
int dsm_device_error(int* code, int clear, void* stream);

/* ---- router: Gate.__call__ (model/moe.py:62-79) ---------------------------------------
 * x [n_tokens, dim] (x_dtype F32 or BF16); gate_weight [n_experts, dim] fp32.
 * Score mode: gate_bias [n_experts] fp32, tid2eid = NULL. Hash mode: gate_bias = NULL,
 * tid2eid [vocab, topk] int32 and input_ids (I32 or I64) of length n_ids == n_tokens or 1.
 * workspace: dsm_router_workspace_bytes() of scratch (fp64 logit partial sums). Outputs
 * weights [n_tokens, topk] fp32 and indices [n_tokens, topk] int32 (ascending by biased
 * score: best expert in the last slot). Logits are accumulated in fp64 and rounded once. */
size_t dsm_router_workspace_bytes(int64_t n_tokens, int dim, int n_experts);
int dsm_router(const void* x, int x_dtype, int64_t n_tokens, int dim, const float* gate_weight,
               int n_experts, const float* gate_bias, const int32_t* tid2eid, int64_t vocab,
               const void* input_ids, int ids_dtype, int64_t n_ids, int topk, int score_func,
               float route_scale, void* workspace, float* weights_out, int32_t* indices_out,
               void* stream);

/* ---- router without a workspace ---------------------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device memory -- an
 * engine whose memory arena owns the whole GPU and cannot grant per-call buffers, or a
 * latency-critical loop that must not touch an allocator. Same arguments and results as
 * dsm_router minus the workspace: the scratch is a fixed array of
 * DSM_ROUTER_NOALLOC_MAX_SCRATCH_BYTES inside the library, held on every GPU that loads it
 * until exit. Calls needing more (dsm_router_workspace_bytes) fail with DSM_ERR_WORKSPACE.
 * The first call on a device resolves the array's address there: make it before any stream
 * capture. After cudaDeviceReset the first call resolves it again (the address is cached per
 * CUDA context), so make that call before any capture too. All calls share the array: calls
 * that can overlap on the GPU race on it. */
#define DSM_ROUTER_NOALLOC_MAX_SCRATCH_BYTES (8u << 20)
int dsm_router_noalloc(const void* x, int x_dtype, int64_t n_tokens, int dim, const float* gate_weight,
                       int n_experts, const float* gate_bias, const int32_t* tid2eid, int64_t vocab,
                       const void* input_ids, int ids_dtype, int64_t n_ids, int topk, int score_func,
                       float route_scale, float* weights_out, int32_t* indices_out, void* stream);

/* ---- permutation (defines per-expert token lists) ------------------------------------
 * indices [n_pairs] int32 (the flattened [n_tokens, topk] routing). Outputs counts [E],
 * offsets [E+1], perm [n_pairs] (sorted position -> pair id, stable), inv [n_pairs]. */
size_t dsm_permute_workspace_bytes(int64_t n_pairs, int n_experts);
int dsm_permute(const int32_t* indices, int64_t n_pairs, int n_experts, int32_t* counts,
                int32_t* offsets, int32_t* perm, int32_t* inv, void* workspace,
                size_t workspace_bytes, void* stream);

/* ---- activation staging ---------------------------------------------------------------
 * Writes rows of x (row r = token perm[r] / topk, or token r when perm is NULL) into the
 * K-chunked f16 layout the expert kernels stream: chunk c holds columns [128c, 128c+128)
 * of every row, rows_cap rows of DSM_STAGE_PITCH halves each. Each row is scaled by a
 * power of two so its largest magnitude lies in [2^14, 2^15); row_scale[r] receives the
 * inverse (exact) factor. Columns past k_dim are written as zeros. */
#define DSM_STAGE_PITCH 160
size_t dsm_stage_bytes(int64_t rows_cap, int k_dim);
int64_t dsm_stage_rows_cap(int64_t n_rows);
int dsm_stage_rows(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                   int64_t n_rows, int topk, void* staged, int64_t rows_cap, float* row_scale,
                   void* stream);
/* stage_rows_count: as stage_rows over rows r < *n_valid (a device count, <= max_rows); the
 * expert-parallel receiver stages the rows that arrived without reading their count back. */
int dsm_stage_rows_count(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                         int64_t max_rows, int topk, void* staged, int64_t rows_cap, float* row_scale,
                         const int32_t* n_valid, void* stream);
/* fp32 rows x [n_rows, dim] staged as 2 * n_rows f16 rows: row r as dsm_stage_rows stages it
 * (hi), row n_rows + r the residual x - hi with its own scale (lo); a product over all rows
 * then adds up, hi + lo, to the fp32 row's product within ~2^-22 relative.
 * rows_cap >= dsm_stage_rows_cap(2 * n_rows). */
int dsm_stage_rows_hilo(const float* x, int64_t n_rows, int dim, void* staged, int64_t rows_cap, float* row_scale,
                        void* stream);

/* ---- expert weight packing (load time) ------------------------------------------------
 * Converts stacked expert weights [n_experts, rows, cols] (nn.Linear [out, in] layout)
 * into the tile stream the expert kernels read. Source arrays per format:
 *   F16:      codes = weights (src_dtype F32 or BF16)
 *   FP8_B128: codes uint8 e4m3 [E,rows,cols]; scales fp32 [E,ceil(rows/128),ceil(cols/128)]
 *   FP4_G32:  codes uint8 [E,rows,cols/2] (element 2j low nibble); scales uint8 e4m3
 *             [E,rows,cols/32]; tensor_scale fp32 [E]
 *   AFFINE8/4: codes uint8 [E,rows,cols*bits/8] (byte view of MLX's uint32 packing);
 *             scales, biases bf16 [E,rows,cols/group_size]
 * The packed buffer must not alias the sources. */
size_t dsm_packed_bytes(int wfmt, int n_experts, int rows, int cols, int group_size);
int dsm_pack_weights(int wfmt, int n_experts, int rows, int cols, int group_size, int src_dtype,
                     const void* codes, const void* scales, const void* biases,
                     const float* tensor_scale, void* packed, void* stream);

/* ---- affine quantisation (mx.quantize restated) ---------------------------------------
 * w [n_rows, cols] (F32 or BF16) -> codes uint8 [n_rows, cols*bits/8], scales and biases
 * [n_rows, cols/group_size] in w's dtype. bits 4 or 8; group_size 32, 64 or 128. */
int dsm_affine_quantize(const void* w, int w_dtype, int64_t n_rows, int cols, int group_size,
                        int bits, uint8_t* codes, void* scales, void* biases, void* stream);

/* ---- grouped expert products ----------------------------------------------------------
 * Rows of expert e are the staged rows [offsets[e], offsets[e+1]); offsets may be NULL when
 * n_experts == 1 (one group holding rows [0, n_rows), e.g. the shared expert).
 * gate_up: h = act(x W1^T, x W3^T) for every row, written to the staged layout of h
 *   (k_dim = inter) scaled by h_scale (power of two). round_gu bit 0: round the two
 *   products to bf16 before the activation (the reference's products are bf16 for bf16 or
 *   affine weights with bf16 x); bit 1: round h to bf16 (the reference casts h to x's dtype).
 * down: o = h W2^T (h read with scale 1/h_scale), fp32 rows [n_rows, ldo];
 *   round_o: round o to bf16 first; o_row_map (NULL = identity) sends staged row r to
 *   output row o_row_map[r] (e.g. back to the order the rows arrived in). */
int dsm_expert_gate_up(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int dim,
                       const int32_t* offsets, int n_experts, int wfmt, int group_size,
                       const void* w1_packed, const void* w3_packed, int inter, int act,
                       float swiglu_limit, int round_gu, void* h_staged, float h_scale,
                       int64_t n_rows, void* stream);
int dsm_expert_down(const void* h_staged, float h_scale, int64_t rows_cap, int inter,
                    const int32_t* offsets, int n_experts, int wfmt, int group_size,
                    const void* w2_packed, int dim, int round_o, float* o_rows, int ldo,
                    const int32_t* o_row_map, int64_t n_rows, void* stream);

/* ---- dense SwiGLU MLP: y = down(act(gate(x), up(x))) for every token ---------------------
 * One expert over all rows (arch/qwen3.py:146-154, model/moe.py:82-97): staging, gate/up with
 * the activation, down, and the cast to y_dtype (F32 or BF16) in one call. w1/w3/w2 packed
 * by dsm_pack_weights with n_experts = 1 (w1, w3 [inter, dim], w2 [dim, inter]); act,
 * swiglu_limit and round_gu as for dsm_expert_gate_up; round_o rounds y to bf16 values
 * first. dim % 4 == 0. The fp4 and affine down product is split along K into partial sums
 * added in a fixed order when the row tiles alone would leave SMs idle. Workspace from
 * dsm_dense_mlp_workspace_bytes. */
size_t dsm_dense_mlp_workspace_bytes(int64_t n_tokens, int dim, int inter);
int dsm_dense_mlp(const void* x, int x_dtype, int64_t n_tokens, int dim, int inter, int wfmt, int group_size,
                  const void* w1_packed, const void* w3_packed, const void* w2_packed, int act, float swiglu_limit,
                  int round_gu, int round_o, void* y, int y_dtype, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ---- plain linear layer over packed weights -------------------------------------------------
 * o[r, :out_dim] = x[r] W^T (fp32 rows, row stride ldo) for rows staged by dsm_stage_rows
 * (their row scales in x_row_scale); W [out_dim, k_dim] packed by dsm_pack_weights with
 * n_experts = 1. */
int dsm_linear(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim, int wfmt, int group_size,
               const void* w_packed, int out_dim, float* o_rows, int ldo, int64_t n_rows, void* stream);
/* grouped_linear: dsm_linear over n_groups weight matrices in one launch. Staged rows
 * [offsets[g], offsets[g+1]) (device offsets, n_groups + 1 entries) are multiplied by group g's
 * matrix of w_packed (dsm_pack_weights with n_experts = n_groups); row r of the product goes
 * to output row o_row_map[r] (NULL: r) with row stride ldo. The grouped low-rank output
 * projection of the draft attention (model/attention.py:124-128: o [b, s, groups, d] x wo_a
 * [groups, rank, d]) is one call: group-major rows, o_row_map[g * n + t] = t * groups + g,
 * ldo = rank. */
int dsm_grouped_linear(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim, int wfmt,
                       int group_size, const void* w_packed, int n_groups, const int32_t* offsets, int out_dim,
                       float* o_rows, int ldo, const int32_t* o_row_map, int64_t n_rows, void* stream);
/* grouped_linear_splitk: dsm_grouped_linear with K split as dsm_linear_splitk splits it, for
 * the streaming formats (f16, fp8); workspace dsm_linear_splitk_workspace_bytes(n_rows,
 * out_dim), the partial rows summed in range order into o_rows through o_row_map. Other
 * formats, one-range products and unaligned pointers run dsm_grouped_linear. Same product as
 * grouped_linear (model/attention.py:124-128), with no reference counterpart of its own. */
int dsm_grouped_linear_splitk(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                              int wfmt, int group_size, const void* w_packed, int n_groups, const int32_t* offsets,
                              int out_dim, float* o_rows, int ldo, const int32_t* o_row_map, int64_t n_rows,
                              void* ws, size_t ws_bytes, void* stream);
/* dsm_linear with K split across the GPU, where a product's row tiles alone would leave most
 * SMs idle: the tensor-memory formats (fp4, affine; units of up to 128 rows), and the
 * streaming formats (f16, fp8) below the tcgen05 row count, whose units then hold a whole
 * draft step's rows (up to 64) so that each weight tile is streamed once per K range. fp32
 * partial slabs per K range go to the workspace (dsm_linear_splitk_workspace_bytes) and are
 * summed in range order into o_rows. One-range products, out_dim or ldo not a multiple of 4,
 * or pointers off 16 bytes run dsm_linear. */
size_t dsm_linear_splitk_workspace_bytes(int64_t n_rows, int out_dim);
int dsm_linear_splitk(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim, int wfmt,
                      int group_size, const void* w_packed, int out_dim, float* o_rows, int ldo, int64_t n_rows,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- the draft head ---------------------------------------------------------------------------
 * hc_head_norm: x [n, hc, dim] -> y [n, dim] = hc_head(x) (x dtype), x_norm [n, dim] =
 *   RMSNorm(y) * norm_weight (x dtype), conf_out[t] = y[t] . conf_w[:dim] when conf_w is given.
 * markov_head: logits [n, vocab] = w1[ids] . w2^T in fp32 and embed [n, rank] = w1[ids]
 *   (w dtype; NULL to skip). rank % 8 == 0, w2 16-byte aligned.
 * draft_head: for x [batch, block, hc, dim] and anchor [batch], the hc_head, the final
 *   RMSNorm, the LM head in fp32, then the block walk: at position i the Markov bias of the
 *   previous token is added to the base logits (written to biased_logits [batch, block,
 *   vocab]) and the next token is taken by argmax (temperature 0, lowest index on ties) or by
 *   Gumbel-max over softmax(logits / temperature) with uniforms [block, batch, vocab];
 *   out_ids [batch, block + 1] starts with the anchor; confidence [batch, block] =
 *   [y || w1[token]] . conf_w + conf_bias. An F32 x is staged as two f16 rows (hi + lo) for
 *   the LM head. batch <= 32. The walk is one cooperative launch (one CTA per SM, grid
 *   barriers bounded by ~2 s: a stalled wait sets the device error and ends the kernel). */
typedef struct dsm_head_desc {
  int64_t batch;
  int block, hc_mult, dim, vocab, rank;
  float norm_eps, hc_eps;
  const float* hc_fn;       /* [hc, hc * dim] */
  const float* hc_scale;    /* [1] */
  const float* hc_base;     /* [hc] */
  const float* norm_weight; /* [dim] or NULL */
  int head_wfmt, head_group_size;
  const void* head_w; /* packed LM head [vocab, dim] */
  int markov_dtype;   /* DSM_DT_F32 or DSM_DT_BF16 */
  const void* markov_w1; /* [vocab, rank] */
  const void* markov_w2; /* [vocab, rank] */
  const float* conf_w;   /* [dim + rank] or NULL (no confidence) */
  float conf_bias;
} dsm_head_desc;
int dsm_hc_head_norm(const void* x, int x_dtype, int64_t n_tokens, int hc_mult, int dim, const float* hc_fn,
                     const float* hc_scale, const float* hc_base, float norm_eps, float hc_eps,
                     const float* norm_weight, const float* conf_w, void* y_out, void* x_norm_out, float* conf_out,
                     void* stream);
int dsm_markov_head(const void* ids, int ids_dtype, int64_t n, int vocab, int rank, const void* w1, const void* w2,
                    int w_dtype, float* logits, void* embed, void* stream);
size_t dsm_draft_head_workspace_bytes(const dsm_head_desc* d, int x_dtype);
int dsm_draft_head(const dsm_head_desc* d, const void* x, int x_dtype, const void* anchor, int anchor_dtype,
                   float temperature, const float* uniforms, int32_t* out_ids, float* biased_logits, float* confidence,
                   void* y_out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- the draft attention (compress_ratio == 0 MLA) --------------------------------------------
 * The projections run on dsm_linear (fp32 rows; an F32 activation staged hi + lo gives a second
 * block of rows, passed as *_lo). cos_t / sin_t are [positions, rope_dim / 2] fp32 tables.
 * rows_norm_rope: out[r] = RoPE(T(RMSNorm(T(in[r] + in_lo[r])) * weight)), the RoPE on the last
 *   rope_dim columns at position pos0 + r % period (rope_dim 0: none). cols <= 49152.
 * q_head_norm_rope: each head of in [n_rows, n_heads * head_dim] scaled by rsqrt(mean(q^2) + eps)
 *   with every elementwise op rounded to T, then RoPE as above.
 * kv_window_write: window[b, (pos0 + j) % window] = rows[b, j] for j < n <= window.
 * sparse_attn: for token (b, m) and head h, attention over the window's first n_win slots and the
 *   block's rows [b, block] of the shared KV head, with a denominator sink exp(sink[h] - max),
 *   then the inverse RoPE at position pos0 + m; out is group-major [n_groups][b * block]
 *   [(n_heads / n_groups) * head_dim]. scratch: dsm_sparse_attn_scratch_bytes.
 * round_rows: out = T(in + in_lo). */
int dsm_rows_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int cols, const float* weight, float eps,
                       int rope_dim, const float* cos_t, const float* sin_t, int pos0, int period, void* out,
                       int out_dtype, void* stream);
int dsm_q_head_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int n_heads, int head_dim, float eps,
                         int rope_dim, const float* cos_t, const float* sin_t, int pos0, int period, void* out,
                         int out_dtype, void* stream);
int dsm_kv_window_write(const void* rows, int dtype, int batch, int n, int dim, int pos0, int window, void* win,
                        void* stream);
size_t dsm_sparse_attn_scratch_bytes(int batch, int block, int n_heads, int n_win);
int dsm_sparse_attn(const void* q, const void* window_kv, const void* block_kv, int dtype, const float* sink, int batch,
                    int block, int n_heads, int head_dim, int window, int n_win, float scale, int rope_dim,
                    const float* cos_t, const float* sin_t, int pos0, int n_groups, void* out, float* scratch,
                    void* stream);
int dsm_round_rows(const float* in, const float* in_lo, int64_t n, void* out, int out_dtype, void* stream);

/* ---- the Qwen3 draft attention (grouped-query) ------------------------------------------------
 * Qwen3DSparkAttention (arch/qwen3.py:84-143) around dsm_linear. cos_t / sin_t are the
 * caller's [tab_rows, head_dim] fp32 tables (rope_tables, qwen3.py:76-81).
 * qkv_norm_rope: in [n_rows, (n_q + 2 n_kv) * head_dim] fp32 (+ in_lo) holds q, k, v heads in
 *   that order. Row r is token t = r % period of sequence b = r / period. Every head is
 *   rounded to T; q and k heads get RMSNorm with q_norm_w / k_norm_w (head_dim fp32) and NeoX
 *   RoPE with table row tab0 + t (x * T(cos) + rotate_half(x) * T(sin), each op rounded to T).
 *   q heads -> q_out [n_rows, n_q, head_dim] (n_q may be 0); k and v heads -> k_out / v_out
 *   [n_rows / period, n_kv, kv_cap, head_dim] at row row0 + t. head_dim even, <= 256.
 * gqa_attn: out [batch, block, n_heads, head_dim] (T) = softmax(q k^T * scale) v per head h
 *   over KV head h / (n_heads / n_kv): the n_ctx context rows ctx_k / ctx_v (element offset
 *   b * ctx_batch_stride + g * ctx_head_stride + row * head_dim) and then the block's rows
 *   blk_k / blk_v [batch, n_kv, block, head_dim]; q is [batch, block, n_heads, head_dim].
 *   head_dim 32, 64, 128 or 256. workspace: dsm_gqa_attn_workspace_bytes (fp32 partials of
 *   the key ranges), 16-byte aligned.
 * set_attn_kernel: 0 (the default) runs bf16 attention on the tensor-core kernels (mma.m16n8k16) where
 *   they apply: dsm_gqa_attn with head_dim 64 / 128, every pointer 16-byte aligned and the
 *   context strides multiples of 8; dsm_sparse_attn with head_dim 64..512 (a multiple of 64),
 *   at most 256 keys, q / window / block rows 16-byte aligned. Elsewhere the CUDA-core kernels
 *   run. 1 runs the CUDA-core kernels everywhere. The choice holds for the
 *   calling host thread only (thread-local): other threads keep their own. */
int dsm_qkv_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int n_q, int n_kv, int head_dim,
                      const float* q_norm_w, const float* k_norm_w, float eps, const float* cos_t, const float* sin_t,
                      int tab_rows, int tab0, int period, void* q_out, void* k_out, void* v_out, int kv_cap, int row0,
                      int dtype, void* stream);
size_t dsm_gqa_attn_workspace_bytes(int batch, int block, int n_heads, int n_kv, int head_dim, int n_ctx);
int dsm_gqa_attn(const void* q, const void* ctx_k, const void* ctx_v, int64_t ctx_batch_stride,
                 int64_t ctx_head_stride, int n_ctx, const void* blk_k, const void* blk_v, int dtype, int batch,
                 int block, int n_heads, int n_kv, int head_dim, float scale, void* out, void* workspace,
                 size_t workspace_bytes, void* stream);
int dsm_set_attn_kernel(int kernel);

/* ---- the Qwen3 draft layer's glue --------------------------------------------------------------
 * add_rms_norm (Qwen3DSparkLayer.__call__ / forward_cached, arch/qwen3.py:165-176): for each of
 * n_rows rows of dim values, s = T(x + delta) (delta NULL: s = x) and y = T(RMSNorm(s) * weight)
 * with the norm in fp32 (norm_rope.py:22-39). sum_out (s) and norm_out (y) are each optional,
 * not both NULL. dim <= 49152. */
int dsm_add_rms_norm(const void* x, const void* delta, int dtype, int64_t n_rows, int dim, const float* weight,
                     float eps, void* sum_out, void* norm_out, void* stream);

/* Kernel regime of the grouped expert products: 0 (default) picks by rows per busy
 * expert -- the mma.sync weight-streaming kernel at decode sizes, the tcgen05/TMEM kernel
 * (fp8 block-scaled experts) from ~64 rows per expert; 1 forces the streaming kernel;
 * 2 forces tcgen05 wherever the format supports it. The choice holds for the calling host
 * thread only (thread-local): other threads keep their own. */
int dsm_set_expert_regime(int regime);

/* ---- row gather and expert parallelism ---------------------------------------------------
 * gather_rows: out[r] = x[perm[r] / topk] (perm NULL: x[r]), same dtype (F32/BF16).
 *
 * Expert parallelism: no counterpart in the reference, which runs the MoE on one device
 * (tests/reference_model.py:55-56 forces world_size 1). Rank `rank` of `world` owns experts
 * [rank * e_local, (rank + 1) * e_local) and routes its own tokens. Each rank allocates one
 * exchange buffer of dsm_ep_buffer_bytes (zero-filled once) that every peer maps (CUDA IPC);
 * peer_base [world] (device memory) holds the peers' mapped addresses, peer_base[rank] this
 * rank's own buffer. A step, all stream-ordered, no host synchronisation:
 *   dsm_ep_dispatch      the sender's expert-sorted (token, slot) rows (dsm_permute's perm,
 *                        offsets, counts over all experts; indices = the routing [n*topk]) go
 *                        into their owners' buffers; row_map[pair] = owner * capacity + slot
 *                        for the combine; raises this rank's flag in every peer.
 *   dsm_ep_receive       waits (bounded) for every sender, whose rows then sit at own_buffer +
 *                        dsm_ep_rows_offset(epoch) ([world * capacity, dim], sender-major),
 *                        and writes offsets [e_local + 1] of the
 *                        arrived rows by local expert, lperm (staged position -> arrival row
 *                        sender * capacity + slot, for dsm_stage_rows_count and as the down
 *                        product's o_row_map) and n_valid [1 + world] (rows arrived, rows per
 *                        sender).
 *   dsm_ep_return        result rows [world * capacity, dim] fp32 (arrival order) go back to
 *                        their senders; raises this rank's result flag in every peer.
 *   dsm_ep_wait_results  waits (bounded) for every owner; dsm_combine then reads the results at
 *                        own_buffer + dsm_ep_results_offset(epoch) through row_map.
 * epoch: 1, 2, 3 ... one per step, the same on every rank (two buffer sets alternate by its
 * parity). done: one zero-initialised uint32 per kernel (dispatch, return), reset by the kernel.
 * capacity: rows per (sender, owner) block >= n_tokens * min(topk, e_local) of any rank.
 * Waits give up after ~2 s with DSM_DEV_ERR_PEER_TIMEOUT. enable_peer_access: lets this
 * device's kernels store into peer_device's memory. */
typedef struct dsm_ep_desc {
  int world;
  int rank;
  int e_local;
  int dim;
  int x_dtype; /* BF16 or F32: the rows the dispatch sends */
  int64_t capacity;
} dsm_ep_desc;
int dsm_gather_rows(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                    int64_t n_rows, int topk, void* out, void* stream);
size_t dsm_ep_buffer_bytes(const dsm_ep_desc* d);
int64_t dsm_ep_rows_offset(const dsm_ep_desc* d, uint32_t epoch);
int64_t dsm_ep_results_offset(const dsm_ep_desc* d, uint32_t epoch);
int dsm_ep_dispatch(const dsm_ep_desc* d, const void* x, int64_t n_tokens, const int32_t* indices,
                    const int32_t* perm, const int32_t* offsets, const int32_t* counts, int topk,
                    const uint64_t* peer_base, int32_t* row_map, uint32_t* done, uint32_t epoch,
                    void* stream);
int dsm_ep_receive(const dsm_ep_desc* d, const void* own_buffer, uint32_t epoch, int32_t* offsets,
                   int32_t* lperm, int32_t* n_valid, void* stream);
int dsm_ep_return(const dsm_ep_desc* d, const float* o_rows, const int32_t* n_valid,
                  const uint64_t* peer_base, uint32_t* done, uint32_t epoch, void* stream);
int dsm_ep_wait_results(const dsm_ep_desc* d, const void* own_buffer, uint32_t epoch, void* stream);
int dsm_enable_peer_access(int peer_device);
/* The exchange buffers across processes: ipc_get_handle gives the 64-byte CUDA IPC handle of
 * the allocation holding ptr and ptr's offset in it; ipc_open maps a peer's handle into the
 * current device's address space (peer access enabled as needed) and returns the base, to
 * which the peer's offset is added; ipc_close unmaps it. */
int dsm_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
int dsm_ipc_open(const void* handle, uint64_t* base);
int dsm_ipc_close(uint64_t base);

/* ---- combine: y = sum_s o[inv[t*k+s]] * w[t,s] (+ shared[t]) -> y_dtype --------------- */
int dsm_combine(const float* o_sorted, const int32_t* inv, const float* route_weights,
                int64_t n_tokens, int topk, int dim, const float* shared_rows, void* y,
                int y_dtype, void* stream);

/* ---- the MoE's neighbours in the draft block (DSparkBlock.__call__, block.py:83-86) ----
 * x [n_tokens, hc_mult, dim] (F32 or BF16; the hyper-connection copies of each token).
 * dsm_hc_pre_norm writes the MoE input x_norm [n_tokens, dim] (x's dtype) =
 * RMSNorm(sum_c pre[c] * x[c]) * norm_weight (norm_weight may be NULL: no scale), and the
 * mixing weights post [n_tokens, hc_mult], comb [n_tokens, hc_mult, hc_mult] (fp32) that
 * dsm_hc_post uses to re-expand the MoE output h [n_tokens, dim] against the residual x:
 * out[t, c] = post[t, c] * h[t] + sum_a comb[t, a, c] * x[t, a]. hc_fn is
 * [(2 + hc_mult) * hc_mult, hc_mult * dim] fp32, hc_scale [3], hc_base [(2 + hc_mult) * hc_mult].
 * hc_mult must be 1, 2 or 4. */
int dsm_hc_pre_norm(const void* x, int x_dtype, int64_t n_tokens, int hc_mult, int dim,
                    const float* hc_fn, const float* hc_scale, const float* hc_base,
                    int sinkhorn_iters, float norm_eps, float hc_eps, const float* norm_weight,
                    void* x_norm_out, float* post_out, float* comb_out, void* stream);
int dsm_hc_post(const void* h, const void* residual, int dtype, int64_t n_tokens, int hc_mult,
                int dim, const float* post, const float* comb, void* out, void* stream);

/* ---- whole MoE.__call__ -----------------------------------------------------------------*/
typedef struct dsm_moe_desc {
  int64_t n_tokens; /* tokens of x (after flattening) */
  int dim, inter, n_experts, topk;
  int score_func;
  float route_scale, swiglu_limit;
  const float* gate_weight; /* [E, dim] */
  const float* gate_bias;   /* [E] (score mode) or NULL */
  const int32_t* tid2eid;   /* [vocab, topk] (hash mode) or NULL */
  int64_t vocab;
  int wfmt, group_size;     /* routed experts */
  const void *w1, *w3, *w2; /* packed */
  int round_gu, round_o;
  int shared_wfmt, shared_group_size; /* shared expert; s1 == NULL: none */
  const void *s1, *s3, *s2;
  int shared_inter, shared_round_gu, shared_round_o;
  int act;
} dsm_moe_desc;

size_t dsm_moe_workspace_bytes(const dsm_moe_desc* d);
int dsm_moe_forward(const dsm_moe_desc* d, const void* x, int x_dtype, const void* input_ids,
                    int ids_dtype, int64_t n_ids, void* y, float* route_weights_out,
                    int32_t* route_indices_out, void* workspace, size_t workspace_bytes,
                    void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DSM_H_ */
