/*
 * kq.h -- C ABI of the B200 quantized routed-expert engine (libkq.so).
 *
 * Two families of entry points live here.
 *
 * 1. Reference-compatible symbols (bakan_cpu_expert_*).  Same names, argument
 *    meaning, host-pointer I/O and return convention (0 = OK, -1 = error with a
 *    "[kandiga] ..." line on stderr) as the reference's native expert library,
 *    so the reference's own ctypes binding (_CPUExpertLib) can load libkq.so
 *    unchanged.  Expert weights are read once from the BKEX layer files at init
 *    and kept resident in HBM; each call copies x to the device, runs the
 *    sm_100a kernels and copies the result back (synchronous, like the
 *    reference).
 *
 * 2. Device-pointer entry points (kq_*).  All pointers are device pointers
 *    unless stated otherwise, every call takes a cudaStream_t (passed as void*)
 *    and is asynchronous.  Return value: 0 OK, >0 argument/setup error
 *    (KQ_ERR_*); kernel-side conditions (bad expert id, wait timeout) are
 *    latched in a device status word read with kq_status_read().  No call on
 *    the hot path allocates memory: scratch comes from a caller-provided
 *    workspace whose size is queried up front.
 *
 * Reference interfaces replaced (paths relative to the kandiga project root)
 * are cited beside each declaration.
 */
#ifndef KQ_H
#define KQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- codes ----------------------------------------------------------------- */
#define KQ_OK 0
#define KQ_ERR_ARG 1
#define KQ_ERR_CUDA 2
#define KQ_ERR_ALLOC 3
#define KQ_ERR_IO 4
#define KQ_ERR_FORMAT 5
#define KQ_ERR_UNSUPPORTED 6
#define KQ_ERR_WORKSPACE 7

/* device status bits (kq_status_read) */
#define KQ_DEV_BAD_EXPERT 1u  /* an expert id outside [0, num_experts): output rows zeroed */
#define KQ_DEV_WAIT_TIMEOUT 2u /* a bounded device-side wait gave up */
#define KQ_DEV_BAD_INDEX 4u   /* a token/slot index outside its range */
#define KQ_DEV_RANGE 16u      /* kq_moe_prefill: a dequantised weight |q*s + b| does not fit fp16 */

/* element types */
#define KQ_DT_F16 0
#define KQ_DT_BF16 1
#define KQ_DT_F32 2

/* activations */
#define KQ_ACT_SILU 0      /* silu(g) * u  (kandiga/metal/kandiga_cpu_expert.m:384-394) */
#define KQ_ACT_GELU_TANH 1 /* gelu_tanh(g) * u (kandiga/metal/kandiga_cpu_expert_lg.m:237-250) */

/* ---- 1. reference-compatible ABI ------------------------------------------- */

/* replaces kandiga/metal/kandiga_cpu_expert.h:40 (bakan_cpu_expert_init).
 * Reads packed_dir/layer_XX.bin (BKEX, kandiga/_pack_experts.py:95-132) for
 * XX in [0, num_layers), takes hidden/inter/bits from the header the way
 * kandiga/metal/kandiga_cpu_expert_lg.m:67-117 does, repacks every expert into
 * the HBM table.  Returns NULL on failure. */
void* bakan_cpu_expert_init(const char* packed_dir, int num_layers);

/* replaces kandiga/metal/kandiga_cpu_expert.h:51 (fp32 host in/out).
 * output_f32 [num_experts][hidden], unweighted per-expert outputs. */
int bakan_cpu_expert_mlp(void* engine, int layer_idx, const float* x_f32,
                         const int32_t* expert_indices, int num_experts, float* output_f32);

/* replaces kandiga/metal/kandiga_cpu_expert.h:65 (fp16 host in/out). */
int bakan_cpu_expert_mlp_f16(void* engine, int layer_idx, const void* x_f16,
                             const int32_t* expert_indices, int num_experts, void* output_f16);

/* replaces kandiga/metal/kandiga_cpu_expert.h:79 (bf16 host in, fp16 host out). */
int bakan_cpu_expert_mlp_bf16(void* engine, int layer_idx, const void* x_bf16,
                              const int32_t* expert_indices, int num_experts, void* output_f16);

/* replaces kandiga/metal/kandiga_cpu_expert.m:564 (bakan_cpu_expert_mlp_batch_f16):
 * x [num_tokens][hidden] fp16, indices [num_tokens][K], output [num_tokens][K][hidden] fp16. */
int bakan_cpu_expert_mlp_batch_f16(void* engine, int layer_idx, const void* x_f16_batch,
                                   const int32_t* indices_batch, int num_tokens, int K,
                                   void* output_f16_batch);

/* replaces kandiga/metal/kandiga_cpu_expert.m:773 (bakan_cpu_expert_mlp_prefill_f16).
 * CSR-grouped prefill: the groups describe which (token, k) pairs use which
 * expert; output [num_tokens][K][hidden] fp16 at (token, k_pos). */
int bakan_cpu_expert_mlp_prefill_f16(void* engine, int layer_idx, const void* x_f16,
                                     int num_tokens, int K, int hidden_size,
                                     const int32_t* sorted_token_indices,
                                     const int32_t* sorted_expert_indices,
                                     const int32_t* sorted_k_positions,
                                     const int32_t* group_starts, const int32_t* unique_experts,
                                     int num_unique_experts, void* output_f16);

/* replaces kandiga/metal/kandiga_cpu_expert.m:847 (bakan_cpu_expert_pread_batch):
 * copies the raw BKEX bytes of the listed experts into a caller host buffer
 * (num_experts_to_read * expert_size bytes), reconstructed from the HBM table. */
int bakan_cpu_expert_pread_batch(void* engine, int layer_idx, const int32_t* expert_ids,
                                 int num_experts_to_read, void* output_buffer);

/* replaces kandiga/metal/kandiga_cpu_expert.h:91 */
void bakan_cpu_expert_destroy(void* engine);

/* replaces kandiga/metal/kandiga_cpu_expert.h:96 */
int bakan_cpu_expert_num_layers(void* engine);

/* ---- 1b. MoE block engine (kandiga/metal/bakan_forward.h) -----------------------
 * The reference declares this ABI (bakan_forward.h:55-151) without an
 * implementation; here it runs the arithmetic of kandiga/metal/moe_block.metal
 * on the GPU.  Host pointers, synchronous, not re-entrant per engine; 0 / -1
 * with a "[kandiga] ERROR" line on stderr.  The routed experts come from the
 * BKEX layer files; the other tensors of a layer from set_weight. */

/* replaces kandiga/metal/bakan_forward.h:64 */
void* bakan_forward_init(const char* packed_expert_dir, int num_layers);

/* replaces kandiga/metal/bakan_forward.h:83.  weight_type: WT_* of
 * bakan_forward.h:35-53 (0 post-attention norm [H]; 1-3 router weight /
 * scales / biases; 4-6 shared-expert gate row; 7-9 shared up_proj; 10-12
 * shared gate_proj; 13-15 shared down_proj), MLX layout; dtype 0 fp16,
 * 1 uint32 (packed 3- or 4-bit codes), 2 bf16; size = rows * cols * element
 * bytes.  A matrix is repacked into HBM once its weight, scales and biases
 * are all set. */
int bakan_forward_set_weight(void* engine, int layer_idx, int weight_type, const void* data, size_t size, int rows,
                             int cols, int dtype);

/* replaces kandiga/metal/bakan_forward.h:110: output = h + MoE(rmsnorm(h)),
 * h and output fp16 [hidden]. */
int bakan_forward_moe_block(void* engine, int layer_idx, const void* h_f16, void* output_f16);

/* replaces kandiga/metal/bakan_forward.h:135: output = MoE(x), x already normed. */
int bakan_forward_moe_block_normed(void* engine, int layer_idx, const void* x_f16, void* output_f16);

/* replaces kandiga/metal/bakan_forward.h:145 */
void bakan_forward_destroy(void* engine);

/* replaces kandiga/metal/bakan_forward.h:150 */
int bakan_forward_num_layers(void* engine);

/* Block parameters the reference fixes in MoeBlockParams
 * (kandiga/metal/moe_block.metal:114-121): top-K (default 8) and the RMSNorm
 * epsilon (default 1e-6).  KQ_OK or KQ_ERR_ARG. */
int kq_forward_set_params(void* engine, int top_k, float rms_norm_eps);

/* Whole-model single-token decode step (kandiga/metal/full_forward.h:43-220,
 * the reference's bakan_full_* ABI; its implementation full_forward_lg.m
 * hard-codes one model).  The model shape comes from `packed_expert_dir`/config.json
 * (hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
 * num_key_value_heads, head_dim, vocab_size, rms_norm_eps, rope_theta,
 * partial_rotary_factor; max_cache_len, default 4096, sizes the KV cache).
 * Token mixers: full attention -- input RMSNorm, q|k|v (separate
 * q_proj/k_proj/v_proj or the reference's fused self_attn.combined_proj; a
 * q_proj of 2 x heads x head_dim rows carries the per-head output gate),
 * optional q_norm/k_norm, RoPE, GQA decode attention over the fp16 cache,
 * o_proj + residual -- or GatedDeltaNet (layer_types "linear_attention", or
 * all but every full_attention_interval-th layer when linear_num_value_heads
 * is set; linear_num_key_heads, linear_key_head_dim (64/128/256),
 * linear_value_head_dim, linear_conv_kernel_dim): in_proj_qkv|z|b|a (or
 * linear_attn.combined_proj), conv1d + SiLU over a ring buffer, q/k RMSNorm
 * and scaling, the gated delta rule on an fp32 state [v heads][v dim][k dim],
 * RMSNormGated, out_proj + residual.  MLP: post-attention RMSNorm + gate/up
 * SwiGLU + down, or, when num_experts > 0, the MoE block of the
 * bakan_forward_* engine (experts from packed_expert_dir/layer_XX.bin; router
 * mlp.gate, mlp.shared_expert.*, mlp.shared_expert_gate; num_experts_per_tok).
 * Then norm and lm_head (or the tied quantized embedding).  Linears are MLX-affine 3/4-bit (weight uint32, scales
 * and biases fp16/bf16); head_dim 64/128/256, 1/2/4/8 q heads per kv head,
 * vocab_size a multiple of 16.  Names may carry the "language_model.model." /
 * "model." prefixes.  Weight dtype codes: 0 fp16, 1 bf16, 2 fp32, 3 packed uint32.
 * Host pointers throughout; calls are synchronous; 0 / -1 with a
 * "[kandiga] ERROR" line, as the reference. */
void* bakan_full_init(const char* packed_expert_dir, int num_layers);          /* full_forward.h:43 */
int bakan_full_set_weight(void* engine, const char* name, const void* data, size_t size, int ndim,
                          const int64_t* shape, int dtype);                     /* full_forward.h:61 */
int bakan_full_build(void* engine);                                              /* full_forward.h:73 */
int bakan_full_forward(void* engine, int token_id, int position, float* logits_out,
                       int* vocab_size_out);                                     /* full_forward.h:90 */
int bakan_full_prefill(void* engine, const int32_t* token_ids, int num_tokens, float* logits_out,
                       int* vocab_size_out);                                     /* full_forward.h:114 */
void bakan_full_reset_cache(void* engine);                                       /* full_forward.h:121 */
void bakan_full_destroy(void* engine);                                           /* full_forward.h:126 */
int bakan_full_num_layers(void* engine);                                         /* full_forward.h:131 */
int bakan_full_vocab_size(void* engine);                                         /* full_forward.h:132 */
void bakan_full_set_debug(void* engine, int enable);                             /* full_forward.h:138 */
int bakan_full_set_kv_cache(void* engine, int attn_layer_idx, const void* keys_data, const void* values_data,
                            int seq_len, int num_kv_heads, int head_dim);        /* full_forward.h:157 */
int bakan_full_set_linear_state(void* engine, int lin_layer_idx, const void* state_data,
                                int state_bytes);                                /* full_forward.h:174 */
int bakan_full_set_conv_state(void* engine, int lin_layer_idx, const void* conv_data,
                              int conv_bytes);                                   /* full_forward.h:193 */
int bakan_full_set_position(void* engine, int position);                         /* full_forward.h:214 */
/* bakan_full_init with the config given as JSON text (no file). */
void* kq_full_init_json(const char* config_json, const char* packed_dir, int num_layers);
/* next position the engine expects (one past the last token run) */
int kq_full_position(void* engine);
/* `steps` decode steps of token_id at positions position.. (device-resident
 * logits, no host copies but the 12-byte token/position upload per step),
 * timed with CUDA events on the engine's stream: *device_ms.  For benchmarks;
 * no counterpart in the reference. */
int kq_full_time_steps(void* engine, int token_id, int position, int steps, float* device_ms);

/* ---- 2. device ABI ------------------------------------------------------------ */

typedef struct kq_table kq_table; /* HBM-resident routed-expert table (all layers) */
typedef struct kq_qmat kq_qmat;   /* HBM-resident dense quantized matrix */

typedef struct {
    int32_t num_layers;
    int32_t num_experts;
    int32_t hidden;     /* H: gate/up input, down output */
    int32_t inter;      /* I: moe_intermediate */
    int32_t bits;       /* 3 or 4 */
    int32_t group_size; /* 64 */
    int32_t sb_dtype;   /* KQ_DT_F16 or KQ_DT_BF16: per-group scale/bias storage */
    int32_t activation; /* KQ_ACT_* */
} kq_table_desc;

/* One MLX-layout quantized matrix, optionally stacked over experts.
 * weight: 3-bit -> bytes [rows][cols*3/8] (== MLX uint32 [rows][cols*3/32]),
 *         4-bit -> uint32 [rows][cols/8]; nibble / 3-bit field j at bit bits*j,
 *         LSB first (kandiga/metal/kandiga_cpu_expert.m:194-201,285-291).
 * scales, biases: 16-bit [rows][cols/group_size].
 * *_stride: bytes between consecutive experts (0 for a single matrix). */
typedef struct {
    const void* weight;
    const void* scales;
    const void* biases;
    int64_t weight_stride;
    int64_t sb_stride;
} kq_mlx_matrix;

/* Table lifetime.  The table owns its HBM; size = layers * experts * expert bytes. */
int kq_table_create(const kq_table_desc* desc, kq_table** out);
int kq_table_destroy(kq_table* t);
int kq_table_desc_get(const kq_table* t, kq_table_desc* desc);
size_t kq_table_bytes(const kq_table* t);
/* bytes one expert occupies in HBM (equal to the MLX/BKEX expert size) */
size_t kq_table_expert_bytes(const kq_table* t);

/* Repack experts [expert_begin, expert_begin + num_experts) of `layer` from
 * device MLX-layout arrays into the table (replaces the pread path of
 * kandiga/metal/kandiga_cpu_expert.m:495-515: weights are made resident once). */
int kq_table_load_mlx(kq_table* t, int layer, int expert_begin, int num_experts,
                      const kq_mlx_matrix* gate, const kq_mlx_matrix* up,
                      const kq_mlx_matrix* down, void* stream);

/* Load one BKEX layer file image (header + payload) that the caller has in
 * host memory into experts [0, file's count) of `layer`.  The header must
 * match the table's desc, which may hold more experts than the file. */
int kq_table_load_bkex(kq_table* t, int layer, const void* file_bytes, size_t nbytes, void* stream);

/* Unpack one matrix (0 gate, 1 up, 2 down) of one expert back to MLX layout
 * (device buffers sized as for kq_mlx_matrix).  Bit-exact inverse of the load. */
int kq_table_unpack_mlx(const kq_table* t, int layer, int expert, int matrix, void* weight,
                        void* scales, void* biases, void* stream);

/* Scratch for kq_moe_*: query, allocate (device), zero once with kq_workspace_init. */
size_t kq_moe_workspace_size(const kq_table* t, int max_tokens, int top_k);
int kq_workspace_init(void* workspace, size_t bytes, void* stream);

/* Router: softmax over E logits, top-K (strict '>', lowest index wins ties),
 * renormalised weights.  replaces kandiga/metal/moe_block.metal:419-505.
 * logits [T][E] fp32 -> idx [T][K] int32, weights [T][K] fp32. */
int kq_router_topk(const float* logits, int T, int E, int K, int32_t* idx, float* weights,
                   void* stream);

/* Routed-expert MLP for T tokens (decode-shaped: every (token, k) pair runs
 * its own expert).  replaces _CPUSwitchGLU.__call__ (kandiga/engine.py:670-739)
 * and bakan_cpu_expert_mlp_f16/bf16 (kandiga/metal/kandiga_cpu_expert.m:662-719).
 *   x          [T][H] in x_dtype (f16, bf16 or f32)
 *   logits     [T][E] fp32 or NULL.  If given, routing runs first and idx /
 *              weights are OUTPUTS; if NULL they are INPUTS.
 *   idx        [T][K] int32;  weights [T][K] fp32 (may be NULL when out is NULL).
 *              An id of -1 is an empty slot: its output is zero and nothing
 *              is latched; other ids outside [0, E) latch KQ_DEV_BAD_EXPERT.
 *   out_per_k  [T][K][H] out_dtype, unweighted per-expert outputs, or NULL
 *   out        [T][H] out_dtype: residual + sum_k w_k y_k
 *              (kandiga/metal/moe_block.metal:515-584), or NULL
 *   residual   [T][H] out_dtype or NULL */
int kq_moe_decode(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                  const float* logits, int32_t* idx, float* weights, int K, void* out_per_k,
                  void* out, int out_dtype, const void* residual, void* workspace,
                  size_t workspace_bytes, void* stream);

/* kq_moe_decode without a caller workspace, for callers that cannot allocate
 * device memory (a runtime that hands a plugin only its input and output
 * buffers; an FFI host with no device allocator).  No counterpart in the
 * reference.  Scratch is one fixed 8 MiB array inside libkq.so, held by every
 * GPU that loads the library until exit; calls needing more are rejected with
 * KQ_ERR_WORKSPACE.  The first call on a device resolves the array's device
 * address (cudaGetSymbolAddress) and must come before any stream capture; the
 * stream must belong to the current device (KQ_ERR_ARG otherwise), and a
 * context reset (cudaDeviceReset) invalidates the cached address.  All calls
 * share the array: overlapping calls on the GPU race.  Allocates nothing.
 * Arguments as kq_moe_decode. */
int kq_moe_decode_static(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                         const float* logits, int32_t* idx, float* weights, int K, void* out_per_k,
                         void* out, int out_dtype, const void* residual, void* stream);
/* Device status bits (KQ_DEV_*) left by the last kq_moe_decode_static call on
 * the current device; reads and clears the word (synchronises `stream`). */
int kq_moe_decode_static_status(uint32_t* status_out, void* stream);

/* Routed-expert decode of n independent single-token items in one persistent
 * launch: item j is row j of x, routed by row j of logits (or idx/weights as
 * inputs when logits is NULL, exactly as kq_moe_decode), through layer
 * layers[j] (device int32 [n]; NULL: every item uses `layer`); out [n][H],
 * out_per_k [n][K][H], residual [n][H], optional RMSNorm of x (norm_w [H] in
 * the x dtype, fp16/bf16 x).  Each item is the reference's per-token expert
 * path (kandiga/metal/kandiga_cpu_expert.m:471-552 with the routing of
 * kandiga/metal/moe_block.metal:419-505 and the blend of :556-584), so with
 * layers == NULL this equals kq_moe_decode for T = n tokens.  The items'
 * weight tiles are one stream of equal work units spread over all SMs, so
 * weights of later items are read from HBM while earlier items' gate/up ->
 * down dependencies resolve; items must not depend on one another's outputs.
 * One CTA per SM, launched cooperatively; the workspace (size independent of
 * n) holds small rings of activations and counters, which the call zeroes on
 * the stream before its launch.  K <= 32. */
size_t kq_moe_decode_batch_workspace_size(const kq_table* t, int top_k);
int kq_moe_decode_batch(const kq_table* t, int n, const int32_t* layers, int layer, const void* x,
                        int x_dtype, const float* logits, int32_t* idx, float* weights, int K,
                        void* out_per_k, void* out, int out_dtype, const void* residual,
                        const void* norm_w, float eps, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Routed-expert MLP for many tokens (prefill), same arguments and outputs as
 * kq_moe_decode.  The T*K assignments are grouped by expert (stable, token
 * order inside an expert, as kandiga/engine.py:407-418) and every expert runs
 * once over its tokens on the tensor cores (tcgen05): weights dequantised to
 * fp16 in shared memory, the expert's tokens as the MMA's N dimension, fp32
 * accumulators in tensor memory.  replaces _gpu_prefill_experts
 * (kandiga/engine.py:386-516) and bakan_cpu_expert_mlp_prefill_f16
 * (kandiga/metal/kandiga_cpu_expert.m:773-838).  Requires hidden and inter to
 * be multiples of 512.  Range: each weight is dequantised as W = q*s + b in
 * fp16 with one rounding (a weight that does not fit fp16 latches
 * KQ_DEV_RANGE); inputs of any magnitude are scaled by powers of two per
 * token, and SwiGLU activations by powers of two per (token, expert) where
 * they reach 2^15, so no fp16 intermediate overflows. */
size_t kq_moe_prefill_workspace_size(const kq_table* t, int max_tokens, int top_k);
int kq_moe_prefill(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                   const float* logits, int32_t* idx, float* weights, int K, void* out_per_k,
                   void* out, int out_dtype, const void* residual, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Shared expert gate of a MoE block (kandiga/metal/moe_block.metal:335-404):
 * gate[t] = sigmoid(w_gate . x[t]), w_gate one MLX-layout row of H weights
 * (bits 3/4, fp16/bf16 scales and biases).  The shared expert itself is stored
 * as expert `shared_id` of the layer's table; this call writes the routed
 * assignments extended by it, idx_out / weights_out [T][K+1] = (idx[t], shared_id)
 * / (weights[t], gate[t]), so kq_moe_decode / kq_moe_prefill with K+1 compute
 * [res] + sum_k w_k y_k + gate * y_shared, the reference's blend
 * (moe_block.metal:515-584), in their own combine.  gate_out [T] may be NULL. */
int kq_shared_gate(const void* x, int x_dtype, int T, int H, const void* gate_weight, const void* gate_scales,
                   const void* gate_biases, int bits, int sb_dtype, const int32_t* idx, const float* weights, int K,
                   int shared_id, int32_t* idx_out, float* weights_out, float* gate_out, void* stream);

/* Blend of a MoE block from per-expert outputs (kandiga/metal/moe_block.metal:515-584):
 * out[t] = [res[t]] + sum_k w[t][k] y[t][k] + [gate[t] * shared[t]] (gate NULL = 1).
 * y [T][K][H] in y_dtype, residual [T][H] in out_dtype, shared [T][H] in shared_dtype;
 * residual / shared may be NULL.  The last step of the expert-parallel path,
 * where the per-expert rows come back from other GPUs. */
int kq_combine(const void* y, int y_dtype, const float* weights, int T, int K, int H, const void* residual,
               const void* shared, int shared_dtype, const float* gate, void* out, int out_dtype, void* stream);

/* Read and clear the device status word of a workspace (synchronises `stream`). */
int kq_status_read(void* workspace, uint32_t* status, void* stream);

/* ---- expert spill: tables larger than HBM ------------------------------------
 * The reference streams experts that do not fit in memory from the SSD and
 * warms the page cache ahead of use with a cross-layer predictor
 * (kandiga/engine.py:577-668: the next layer's router applied to this layer's
 * input, top-K per token, union over tokens).  Here the whole table
 * (layers x experts, in the HBM tile layout) sits in pinned, device-mapped host
 * memory, and every layer keeps `slots` experts in an HBM pool.  The pool is
 * an ordinary kq_table with `slots` experts per layer, so kq_moe_decode /
 * kq_moe_prefill run on it unchanged, given slot ids in place of expert ids.
 * kq_spill_fetch turns expert ids into slot ids on the device and copies the
 * experts that are not resident over the host link into the least recently
 * used slots, with no host round trip (stream-ordered, graph-capturable).
 * Calls for one layer must be ordered (one stream, or events); calls for
 * different layers may overlap (each layer has its own slots and state). */
typedef struct kq_spill kq_spill;
#define KQ_DEV_CAPACITY 8u /* kq_spill_fetch: more distinct experts than slots; the rest got slot id -1 */
/* slots <= 1024 and <= num_experts, num_experts <= 16384.  Allocates the host
 * store (pinned, mapped) and the pool; residency starts empty. */
int kq_spill_create(const kq_table_desc* desc, int slots, kq_spill** out);
int kq_spill_destroy(kq_spill* s);
/* The HBM pool: a kq_table of desc.num_layers layers x `slots` experts. */
const kq_table* kq_spill_pool(const kq_spill* s);
size_t kq_spill_host_bytes(const kq_spill* s);
/* Copy layer `src_layer` of a device table of the same shape (experts,
 * hidden, inter, bits, scale dtype, activation) into layer `layer` of the
 * host store, and empty that layer's residency. */
int kq_spill_store_layer(kq_spill* s, int layer, const kq_table* src, int src_layer, void* stream);
/* ids [n]: expert ids of `layer` (any order, repeats allowed).  Writes
 * slot_ids [n] (may be NULL) and makes every named expert resident: hits
 * refresh the slot's use stamp, misses (in expert-id order) take the least
 * recently used slots not named by this call (ties: lowest slot) and are
 * copied from host memory.  An id outside [0, num_experts) gets slot -1 and
 * latches KQ_DEV_BAD_EXPERT; more distinct ids than slots latches
 * KQ_DEV_CAPACITY (the experts that did not fit get -1).  Two kernels. */
int kq_spill_fetch(kq_spill* s, int layer, const int32_t* ids, int n, int32_t* slot_ids, void* stream);
/* kq_spill_fetch without slot ids and without KQ_DEV_CAPACITY: brings
 * predicted experts in ahead of use and stops when every slot holds an
 * expert of this call (the background prefetch of kandiga/engine.py:577-616,
 * issued on a second stream while the current layer computes). */
int kq_spill_prefetch(kq_spill* s, int layer, const int32_t* ids, int n, void* stream);
/* counters since the last reset: [0] hits (distinct resident experts named),
 * [1] misses (experts copied), [2] bytes copied, [3] status bits.  Host
 * array; synchronises `stream`; reset != 0 clears them. */
int kq_spill_stats(kq_spill* s, uint64_t out[4], int reset, void* stream);
/* Residency of `layer` (host arrays, synchronises `stream`):
 * slot_of [num_experts] (slot or -1), owner [slots] (expert or -1). */
int kq_spill_residency(const kq_spill* s, int layer, int32_t* slot_of, int32_t* owner, void* stream);

/* ---- dense quantized GEMV (tq3 / shared-layer path) -------------------------- */

/* Dense MLX-affine matrix [rows][cols].  With `pair` set, two matrices of the
 * same shape (gate, up) are interleaved so one pass yields act(gate x) * (up x). */
int kq_qmat_create(int rows, int cols, int bits, int sb_dtype, int pair, kq_qmat** out);
int kq_qmat_destroy(kq_qmat* m);
int kq_qmat_load_mlx(kq_qmat* m, const kq_mlx_matrix* a, const kq_mlx_matrix* b, void* stream);
/* Unpack matrix `which` (0 = a / gate, 1 = b / up) back to MLX layout, bit-exact. */
int kq_qmat_unpack_mlx(const kq_qmat* m, int which, void* weight, void* scales, void* biases,
                       void* stream);

/* y[t] = W x[t] (pair: y = act(Wg x) * (Wu x), activation KQ_ACT_*).
 * Optional RMSNorm prologue: x <- x * rsqrt(mean(x^2) + eps) * norm_w
 * (kandiga/metal/attention.metal:530-675), norm_w in x_dtype or NULL.
 * replaces the MLX QuantizedLinear(bits=3) path loaded at kandiga/engine.py:928-989. */
int kq_dense_gemv(const kq_qmat* m, const void* x, int x_dtype, int T, const void* norm_w,
                  float eps, int activation, void* y, int y_dtype, void* stream);

/* Re-quantize an MLX-layout affine matrix (rows x cols, group 64; weight
 * bytes [rows][cols*src_bits/8], 16-bit scales/biases [rows][cols/64] in
 * sb_dtype; device) to dst_bits: dequantize each element to the scale dtype,
 * then quantize each group as MLX's affine quantizer does (fp32: the edge of
 * larger magnitude made exactly representable, scale = edge / round(edge /
 * ((max - min) / (2^bits - 1))), bias = edge; codes from those values; scale
 * and bias then rounded to sb_dtype; scales may be negative).  The
 * 4-bit -> 3-bit expert repack of scripts/repack_experts_3bit.py:76-103. */
int kq_requantize_mlx(const void* weight, const void* scales, const void* biases, long rows, int cols, int src_bits,
                      int dst_bits, int sb_dtype, void* weight_out, void* scales_out, void* biases_out,
                      void* stream);

/* ---- TQ3_1S dense GEMV --------------------------------------------------------- */

/* A TQ3_1S matrix [rows][cols] (cols % 32 == 0): the reference's block stream
 * (kandiga/tq3/quantize.py:122-145, 390-461) uploaded unchanged, 20-byte
 * blocks (fp16 d0 d1 m0 m1 + 12 bytes of 3-bit indices) or the 16-byte
 * variant without means (kandiga/tq3/quantize.py:483-516). */
typedef struct kq_tq3_mat kq_tq3_mat;
int kq_tq3_create(int rows, int cols, int block_bytes, const void* host_blocks, size_t nbytes, kq_tq3_mat** out);
int kq_tq3_destroy(kq_tq3_mat* m);
size_t kq_tq3_bytes(const kq_tq3_mat* m);
/* y[t] = W x[t] (+ bias, fp32 [rows] or NULL) for T tokens: x [T][cols], y [T][rows].
 * Scores the codes against the Walsh-Hadamard-rotated input (w . x = r . WHT(x)).
 * replaces tq3_gemv (kandiga/tq3/fused_kernel.py:289-341) and TQ3Linear.forward
 * (kandiga/tq3/engine.py:61-73). */
int kq_tq3_gemv(const kq_tq3_mat* m, const void* x, int x_dtype, int T, const float* bias, void* y, int y_dtype,
                void* stream);
/* Reconstructed weights, fp32 [rows][cols] (kandiga/tq3/quantize.py:483-516). */
int kq_tq3_dequant(const kq_tq3_mat* m, float* w, void* stream);

/* ---- TurboQuant KV cache (PolarQuant 3-bit + 1-bit QJL) ----------------------- */

/* A compressed K/V cache of `batch` x `num_heads` x capacity vectors of
 * head_dim elements (1..128; KQ_ERR_UNSUPPORTED above).  replaces TurboQuantCache
 * (kandiga/kv_compress.py:22-57): `rotation` (R, x_rot = x R) and `qjl`
 * (P) are the caller's head_dim x head_dim fp32 host matrices, built as in
 * kandiga/kv_compress.py:34-44.  Per vector the cache holds, for K and for V,
 * one nibble per element (3-bit code << 1 | QJL sign) and fp32 scale and zero
 * (the reference's int8 codes, int8 signs, fp32 scales/zeros, packed). */
typedef struct kq_tq_cache kq_tq_cache;
#define KQ_ERR_CAPACITY 8

int kq_tq_create(int head_dim, int num_heads, int batch, int capacity, const float* rotation, const float* qjl,
                 kq_tq_cache** out);
int kq_tq_destroy(kq_tq_cache* c);
int kq_tq_seq_len(const kq_tq_cache* c);
/* Width at which vectors are stored: head_dim rounded up to 64 or 128 (the
 * packed rows of kq_tq_save / kq_tq_restore hold storage_dim / 2 bytes). */
int kq_tq_storage_dim(const kq_tq_cache* c);
int kq_tq_capacity(const kq_tq_cache* c);
/* Grow the capacity to at least `capacity` vectors per head, keeping the contents. */
int kq_tq_reserve(kq_tq_cache* c, int capacity, void* stream);
/* Compress T new tokens of keys and values ([batch][heads][T][head_dim] in
 * dtype KQ_DT_*, device) onto the end of the cache: rotate, uniform 3-bit
 * quantize per vector, residual, QJL sign sketch (kandiga/kv_compress.py:59-92,
 * 120-150).  KQ_ERR_CAPACITY if the tokens do not fit.  Storage width 128 (head_dim
 * 65..128): the two D x D products run on the tensor cores (tcgen05, fp16 with
 * two limbs per operand, ~22 bits); width 64: fp32 FMA chains. */
int kq_tq_append(kq_tq_cache* c, const void* keys, const void* values, int dtype, int T, void* stream);
/* Device status bits (KQ_DEV_WAIT_TIMEOUT) latched by the cache's append
 * kernels (synchronises `stream`). */
int kq_tq_status(const kq_tq_cache* c, uint32_t* status_out, void* stream);
/* Reconstruct all cached keys (which = 0) or values (1) as fp16
 * [batch][heads][seq_len][head_dim] (kandiga/kv_compress.py:94-118, 152-168). */
int kq_tq_dequant(const kq_tq_cache* c, int which, void* out_f16, void* stream);
/* Unpacked codes/signs (int8 [batch][heads][seq_len][head_dim]) and fp32
 * scales/zeros ([batch][heads][seq_len]) of K (0) or V (1), the reference's
 * storage layout; any pointer may be NULL. */
int kq_tq_export(const kq_tq_cache* c, int which, int8_t* codes, int8_t* signs, float* scales, float* zeros,
                 void* stream);
/* Session persistence of the compressed cache (kandiga/engine.py:1342-1479
 * saves and restores a session's caches).  kq_tq_save copies keys' (which = 0)
 * or values' (1) packed storage, compact: packed [batch][heads][seq_len][storage_dim/2]
 * bytes (two nibbles a byte), scales and zeros fp32 [batch][heads][seq_len]
 * (device).  kq_tq_restore sets the cache to `len` vectors per head from
 * arrays in that layout, growing the capacity if needed. */
int kq_tq_save(const kq_tq_cache* c, int which, uint8_t* packed, float* scales, float* zeros, void* stream);
int kq_tq_restore(kq_tq_cache* c, int len, const uint8_t* k_packed, const float* k_scales, const float* k_zeros,
                  const uint8_t* v_packed, const float* v_scales, const float* v_zeros, void* stream);
/* Single-query attention over the compressed cache: q [batch][q_heads][head_dim]
 * (q_heads a multiple of num_heads, grouped-query), out fp32 [batch][q_heads][head_dim]
 * = softmax(q K^T / sqrt(D)) V with K, V the reconstructions.  Scores are taken
 * on the codes in the rotated domain, values are accumulated there and
 * un-rotated once.  `scores` (fp32 [batch][q_heads][seq_len], the scaled
 * logits) may be NULL.  No counterpart in the reference, which dequantizes
 * the whole cache for MLX attention. */
size_t kq_tq_attend_workspace_size(const kq_tq_cache* c, int q_heads);
int kq_tq_attend(const kq_tq_cache* c, const void* q, int q_dtype, int q_heads, float* out, float* scores,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- tensor-core building block ---------------------------------------------- */

/* C[M][N] (fp32) = A[M][K] * B[N][K]^T with fp16 A, B (K contiguous), on the
 * 5th-generation tensor cores (tcgen05, TMEM accumulator).  M % 128 == 0,
 * 16 <= N <= 256 with N % 16 == 0, K % 64 == 0.  The operand staging and MMA
 * path of the prefill expert GEMM, exposed for direct checks.  No counterpart
 * in the reference (its prefill matmuls run in Metal / MLX). */
int kq_gemm_f16_tc(const void* A, const void* B, float* C, int M, int N, int K, void* stream);

/* ---- expert parallelism across the GPUs of one node ---------------------------
 * The routed experts of a layer are partitioned over `world` ranks (one process,
 * or one context, per GPU); tokens are data-parallel.  The reference has no
 * cross-device code: the parallelism this replaces is its per-token loop over
 * the K experts (kandiga/metal/kandiga_cpu_expert.m:522-543).  Each rank owns an
 * exchange buffer of the same layout; peers map it (CUDA IPC) and every
 * transfer is a store into the destination's buffer (no loads from a peer).
 * A token row travels once to every rank owning one of its experts; that rank
 * runs the grouped MLP of its experts on all rows it received and writes the
 * weighted partial sum straight into the owner's buffer; the owner adds
 * residual + partials (+ shared).  A shared expert replicated on every rank
 * can ride along as one more slot of the owner's own segment (top_k of the
 * context = routed K + 1), so it runs inside the same grouped MLP.
 * No host synchronisation: counts live on the device and the bounded waits
 * (default 2 s, kq_ep_set_wait_ns) poll flags that only grow, so a layer's
 * calls can be captured in a CUDA graph.  Every rank must make the same calls
 * in the same order.  A wait that gives up latches KQ_DEV_WAIT_TIMEOUT
 * (kq_ep_status); the ranks stay out of step until every rank's status is
 * cleared and the buffers are recreated. */
#define KQ_EP_MAX_RANKS 8
#define KQ_EP_HANDLE_BYTES 64
typedef struct kq_ep kq_ep;

/* Bytes of one rank's exchange buffer. */
size_t kq_ep_buffer_bytes(int world, int max_tokens, int hidden, int top_k);
/* Allocate this rank's buffer on the current device (the only allocation; all
 * later calls allocate nothing).  max_tokens: most tokens any rank passes in one
 * call; top_k: slots per row (routed K, + 1 with a shared-expert slot);
 * x_dtype f16 or bf16 (rows travel and partial sums return in it). */
int kq_ep_create(int rank, int world, int max_tokens, int hidden, int top_k, int x_dtype, kq_ep** out);
/* KQ_EP_HANDLE_BYTES describing this rank's buffer to the other processes. */
int kq_ep_ipc_handle(const kq_ep* ep, void* handle_out);
/* Map the peers' buffers: handles = world * KQ_EP_HANDLE_BYTES in rank order
 * (this rank's entry is ignored).  All ranks must connect before any dispatch. */
int kq_ep_connect(kq_ep* ep, const void* handles);
/* n contexts of one process on one device, ranks 0..n-1, joined by plain
 * pointers.  For emulating n ranks on one GPU: issue every rank's dispatch
 * before any receive, and every return before any combine, on one stream, so
 * that no wait is ever pending while another launch would satisfy it. */
int kq_ep_connect_local(kq_ep* const* eps, int n);
void kq_ep_destroy(kq_ep* ep);
int kq_ep_set_wait_ns(kq_ep* ep, uint64_t ns);

/* The steps of one layer, in this order, on one stream:
 *   kq_ep_dispatch  route plan + push rows: x [T][H] (16-byte aligned), idx /
 *                   weights [T][k_route] (global expert ids, -1 = empty),
 *                   owner[E] / local[E] int32 (rank of expert e, its index in
 *                   that rank's table); T <= max_tokens.  shared_id >= 0:
 *                   a shared expert (that local id on every rank) runs as
 *                   slot k_route of each token's row on its own rank, weighted
 *                   by shared_w [T] (then k_route + 1 == the context's top_k);
 *                   shared_id -1: no such slot
 *   kq_ep_receive   wait for every source; the received rows as a batch of
 *                   world * max_tokens rows [rows][H] with ids [rows][K] local to
 *                   this rank (-1 for empty slots) and weights [rows][K]
 *   kq_ep_compute   kq_moe_prefill of the local table on that batch, its
 *                   weighted sums written into the owners' buffers (below 16
 *                   rows: kq_moe_decode into kq_ep_partials())
 *   kq_ep_return    release the owners' return flags (below 16 rows: push
 *                   each partial row back first)
 *   kq_ep_combine   wait for every destination; out [T][H] = residual +
 *                   sum of partials + gate[t] * shared[t] (gate NULL: 1)
 * kq_ep_moe issues all five. */
int kq_ep_dispatch(kq_ep* ep, const void* x, const int32_t* idx, const float* weights, int T, int k_route,
                   const int32_t* owner, const int32_t* local, int num_experts, int shared_id,
                   const float* shared_w, void* stream);
int kq_ep_receive(kq_ep* ep, void** recv_x, int32_t** recv_idx, float** recv_w, int* rows, void* stream);
size_t kq_ep_moe_workspace_size(const kq_ep* ep, const kq_table* t);
int kq_ep_compute(kq_ep* ep, const kq_table* t, int layer, void* workspace, size_t workspace_bytes, void* stream);
void* kq_ep_partials(kq_ep* ep);
int kq_ep_return(kq_ep* ep, void* stream);
int kq_ep_combine(kq_ep* ep, int T, const void* residual, int res_dtype, const void* shared, int shared_dtype,
                  const float* gate, void* out, int out_dtype, void* stream);
int kq_ep_moe(kq_ep* ep, const kq_table* t, int layer, const void* x, int T, const int32_t* idx,
              const float* weights, int k_route, int num_experts, const int32_t* owner, const int32_t* local,
              int shared_id, const float* shared_w, const void* residual, int res_dtype, const void* shared,
              int shared_dtype, const float* gate, void* out, int out_dtype, void* workspace,
              size_t workspace_bytes, void* stream);
/* Status bits (KQ_DEV_*) of this rank's exchange kernels and, in site[4], the
 * first wait that gave up: (1 receive | 2 combine, source rank, flag value
 * seen, CTA).  Synchronises the stream. */
int kq_ep_status(kq_ep* ep, uint32_t* status_out, uint32_t* site_out, void* stream);
int kq_ep_clear_status(kq_ep* ep, void* stream);
/* Layer calls issued so far (synchronous read). */
int kq_ep_calls(kq_ep* ep, uint32_t* calls_out);

#ifdef __cplusplus
}
#endif

#endif /* KQ_H */
