/*
 * anelm_b200 -- C ABI of the B200 (sm_100a) attention core for Qwen3.5-style
 * hybrid models: gated full attention + Gated DeltaNet.
 *
 * This library replaces the CPU attention core that ANE-LM runs between its
 * Neural Engine projection chunks:
 *   - core/cpu_ops.h:16-58              (the op entry points),
 *   - models/llm/qwen3_5.cpp:849-1002   (forward_deltanet_from_proj /
 *                                        forward_full_attn_from_proj glue),
 *   - scripts/serve_hybrid.py:85-132    (cpu_attention, the Python route).
 * (Paths are relative to the ANE-LM project root.)
 *
 * Conventions
 *   - Every entry point returns an int status (anelm_status); 0 is success.
 *     anelm_last_error() gives a message for the calling thread.
 *   - Tensors passed to anelm_* compute calls are DEVICE pointers unless the
 *     name says _host; weights given to the setters are host fp32.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls are
 *     asynchronous on that stream unless documented otherwise.
 *   - An anelm_ctx owns the device KV rings and DeltaNet state for up to
 *     max_seqs sequences (the KVCache / DeltaNetState structs of
 *     models/llm/qwen3_5.h:158-171, one per layer and sequence).
 *   - There is no CPU fallback: without a usable sm_100 device every compute
 *     entry point fails with ANELM_ERR_CUDA.
 */
#ifndef ANELM_B200_H
#define ANELM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ANELM_API __attribute__((visibility("default")))

typedef struct anelm_ctx anelm_ctx;
typedef struct anelm_plan anelm_plan;

typedef enum anelm_status {
    ANELM_OK = 0,
    ANELM_ERR_INVALID_ARG = 1,   /* bad pointer, index or shape */
    ANELM_ERR_CAPACITY = 2,      /* position / length beyond a ring's capacity */
    ANELM_ERR_CUDA = 3,          /* CUDA runtime error (message has the detail) */
    ANELM_ERR_TIMEOUT = 4,       /* a bounded device-side wait gave up */
    ANELM_ERR_UNSUPPORTED = 5,   /* shape or mode this build has no kernel for */
    ANELM_ERR_STATE = 6,         /* weights not set / wrong layer type */
    ANELM_ERR_NOMEM = 7          /* device allocation failed */
} anelm_status;

typedef enum anelm_dtype { ANELM_F32 = 0, ANELM_F16 = 1, ANELM_BF16 = 2 } anelm_dtype;

/* LayerType, models/llm/qwen3_5.h:13-16 */
typedef enum anelm_layer_type { ANELM_LAYER_LINEAR_ATTN = 0, ANELM_LAYER_FULL_ATTN = 1 } anelm_layer_type;

/* RoPE pairing: interleaved (v[i], v[i+1]) as core/cpu_ops.cpp:40-63, or
 * rotate-half (v[j], v[j+R/2]) as scripts/serve_hybrid.py:94-103. */
typedef enum anelm_rope_mode { ANELM_ROPE_INTERLEAVED = 0, ANELM_ROPE_HALF = 1 } anelm_rope_mode;

/* Delta rule order: core/cpu_ops.cpp:131-146 (S^T k from the undecayed state)
 * or scripts/export_hybrid_chunks.py:142-147 (decay first, beta on delta). */
typedef enum anelm_delta_mode { ANELM_DELTA_CPUOPS = 0, ANELM_DELTA_HF = 1 } anelm_delta_mode;

/* KV placement: ring (models/llm/qwen3_5.cpp:973-983) or linear slot = pos
 * (scripts/serve_hybrid.py:105-108). */
typedef enum anelm_kv_mode { ANELM_KV_RING = 0, ANELM_KV_LINEAR = 1 } anelm_kv_mode;

/* Shape and variant configuration.  Fields follow Qwen35Args
 * (models/llm/qwen3_5.h:51-80); anelm_config_default() fills the
 * Qwen3.5-0.8B values used there. */
typedef struct anelm_config {
    int num_layers;
    const int* layer_types;       /* [num_layers] anelm_layer_type; NULL => every
                                     full_attention_interval-th layer is full attention */
    int full_attention_interval;  /* qwen3_5.h:59 (used when layer_types == NULL) */
    /* full attention */
    int num_q_heads, num_kv_heads, head_dim, rot_dim;
    float rope_theta, rms_eps;
    int attn_output_gate;
    /* Gated DeltaNet */
    int lin_num_key_heads, lin_num_val_heads, lin_key_dim, lin_val_dim, conv_kernel;
    /* sequences */
    int max_seqs;
    int kv_capacity;              /* ring slots per sequence (reference: 2048, qwen3_5.h:126) */
    const int* seq_kv_capacity;   /* optional [max_seqs] per-sequence capacity (overrides) */
    int rope_table_len;           /* positions with a host-built cos/sin row (reference: 4096) */
    /* variants */
    int rope_mode;                /* anelm_rope_mode */
    int delta_mode;               /* anelm_delta_mode */
    float l2_eps;                 /* added inside the sqrt of the q/k L2 norm; 1e-12 (cpu_ops.cpp:85) */
    int qk_norm_in_core;          /* 1: per-head RMSNorm of q/k inside the core (qwen3_5.cpp:952-959) */
    int kv_mode;                  /* anelm_kv_mode */
} anelm_config;

/* Fills *cfg with the Qwen3.5-0.8B defaults of models/llm/qwen3_5.h:51-80
 * (24 layers, 8/2 heads, d=256, R=64, theta 1e7; DeltaNet 16/16 heads of 128)
 * and the reference's C++ core variants.  Replaces: Qwen35Args defaults. */
ANELM_API int anelm_config_default(anelm_config* cfg);

/* Creates a context on CUDA device `device`: allocates the KV rings (fp16,
 * slot-major [capacity][Hkv][d] per layer and sequence), the DeltaNet states
 * (fp32 [Hv][dk][dv]) and conv rings, and uploads the RoPE table built on the
 * host exactly as qwen3_5.cpp:309-324.  Everything starts zeroed.
 * Replaces: the allocation part of Qwen35Model::load, qwen3_5.cpp:280-347. */
ANELM_API int anelm_create(const anelm_config* cfg, int device, anelm_ctx** out);
ANELM_API int anelm_destroy(anelm_ctx* ctx);

/* Status text / last error message of the calling thread. */
ANELM_API const char* anelm_status_string(int status);
ANELM_API const char* anelm_last_error(void);

/* Full-attention per-head norm weights (host fp32 [head_dim], already with the
 * +1 of load_norm_weight, core/safetensors.cpp:302-308).
 * Replaces: FullAttnWeights, qwen3_5.cpp:437-446. */
ANELM_API int anelm_set_full_attn_weights(anelm_ctx* ctx, int layer, const float* q_norm_host,
                                          const float* k_norm_host);

/* DeltaNet weights (host fp32): conv1d_w [C][conv_kernel], A [Hv] = exp(A_log),
 * dt_bias [Hv], norm_w [dv] (no +1).  Replaces: DeltaNetWeights, qwen3_5.cpp:404-433. */
ANELM_API int anelm_set_deltanet_weights(anelm_ctx* ctx, int layer, const float* conv1d_w_host,
                                         const float* A_host, const float* dt_bias_host,
                                         const float* norm_w_host);

/* Zeroes KV rings, DeltaNet state and conv rings of sequence `seq` (-1: all).
 * Synchronous.  Replaces: Qwen35Model::reset, qwen3_5.cpp:159-182. */
ANELM_API int anelm_reset(anelm_ctx* ctx, int seq);

/* Copies one sequence's ring of one full-attention layer to/from the host in
 * the reference layout: fp32 [capacity][Hkv][d], plus len/start
 * (KVCache, qwen3_5.h:165-171).  Synchronous.  Import rounds K/V to fp16. */
ANELM_API int anelm_kv_export(anelm_ctx* ctx, int layer, int seq, float* k_host, float* v_host,
                              int* len, int* start);
ANELM_API int anelm_kv_import(anelm_ctx* ctx, int layer, int seq, const float* k_host,
                              const float* v_host, int len, int start);

/* Copies one sequence's DeltaNet state of one linear-attention layer to/from
 * the host in the reference layout: ssm [Hv][dk][dv] fp32, conv ring
 * [C][conv_kernel-1] fp32 and conv_pos (DeltaNetState, qwen3_5.h:158-162).
 * Synchronous. */
ANELM_API int anelm_deltanet_state_export(anelm_ctx* ctx, int layer, int seq, float* ssm_host,
                                          float* conv_host, int* conv_pos);
ANELM_API int anelm_deltanet_state_import(anelm_ctx* ctx, int layer, int seq, const float* ssm_host,
                                          const float* conv_host, int conv_pos);

/* Device-side bulk import: writes n_slots consecutive ring slots
 * [slot0, slot0+n_slots) of sequence `seq` from device fp16 arrays
 * [n_slots][Hkv][d] (either may be NULL), asynchronously on `stream`; then
 * anelm_kv_set_meta sets len/start.  For loading KV produced elsewhere (an
 * external prefill).  Replaces: the memcpy of qwen3_5.cpp:984-986, in bulk. */
ANELM_API int anelm_kv_write(anelm_ctx* ctx, int layer, int seq, int slot0, int n_slots, const void* k_src,
                             const void* v_src, void* stream);
ANELM_API int anelm_kv_set_meta(anelm_ctx* ctx, int layer, int seq, int len, int start);

/* Device-side import of one sequence's DeltaNet state S (fp32 [Hv][dk][dv]
 * device array), asynchronous on `stream`. */
ANELM_API int anelm_deltanet_state_write(anelm_ctx* ctx, int layer, int seq, const float* ssm_src, void* stream);

/* Synchronises the context's device and returns (and clears) the first status
 * a kernel recorded (e.g. ANELM_ERR_CAPACITY for a device-side position beyond
 * a linear cache).  0 if none. */
ANELM_API int anelm_get_device_error(anelm_ctx* ctx, int* code);

/* ---- single-sequence decode (the glue functions) ---- */

/* One decode token of a full-attention layer for sequence `seq` at absolute
 * position `pos`: per-head QK RMSNorm, RoPE, KV-ring append, GQA softmax
 * attention over the ring (split-K flash decoding) and the sigmoid output gate.
 * proj: [q_gate (Hq*2d) | k (Hkv*d) | v (Hkv*d)] of proj_dtype (not modified).
 * out: [Hq*d] of out_dtype.
 * Replaces: forward_full_attn_from_proj, models/llm/qwen3_5.cpp:944-1002. */
ANELM_API int anelm_full_attn_from_proj(anelm_ctx* ctx, int layer, int seq, const void* proj,
                                        int proj_dtype, int pos, void* out, int out_dtype,
                                        void* stream);

/* One decode token of a Gated DeltaNet layer for sequence `seq`: conv1d ring +
 * SiLU, q/k L2 norm and q scale, beta/decay gating, delta-rule state update,
 * y = S^T q and the gated RMSNorm.
 * proj: [mixed_qkv (C) | z (Hv*dv) | a (Hv) | b (Hv)] of proj_dtype.
 * out: [Hv*dv] of out_dtype.
 * Replaces: forward_deltanet_from_proj, models/llm/qwen3_5.cpp:849-910. */
ANELM_API int anelm_deltanet_from_proj(anelm_ctx* ctx, int layer, int seq, const void* proj,
                                       int proj_dtype, void* out, int out_dtype, void* stream);

/* ---- batched (ragged) decode: one token for each of n sequences ---- */

/* A plan fixes the batch (host list of n distinct sequence ids) and owns the
 * split-K work tables and scratch for it.  Reuse it across steps and layers.
 * Replaces: nothing in the reference (it decodes one sequence); batching is
 * the serving form of the per-token loop of qwen3_5.cpp:1205-1217. */
ANELM_API int anelm_plan_create(anelm_ctx* ctx, int n, const int* seq_ids_host, anelm_plan** out);
ANELM_API int anelm_plan_destroy(anelm_plan* plan);

/* Tokens per split-K work unit and number of CTAs per kv head the plan launches. */
ANELM_API int anelm_plan_info(const anelm_plan* plan, int* split_tokens, int* n_blocks);

/* Batched forward_full_attn_from_proj: proj [n][proj_dim], pos [n] (device
 * int32, absolute positions), out [n][Hq*d].  Row i belongs to seq_ids[i]. */
ANELM_API int anelm_full_attn_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer,
                                     const void* proj, int proj_dtype, const int* pos,
                                     void* out, int out_dtype, void* stream);

/* Batched forward_deltanet_from_proj: proj [n][proj_dim], out [n][Hv*dv]. */
ANELM_API int anelm_deltanet_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer,
                                    const void* proj, int proj_dtype, void* out, int out_dtype,
                                    void* stream);

/* ---- layer steps: projections on the device around the core ----
 * The reference runs first_proj and o_proj on the ANE and hands the core host fp32
 * projection rows (models/llm/qwen3_5.cpp:912-1012, core/ane_runtime.cpp:279-361).  With the
 * projection weights in the context, one call runs a decode layer's in-projection (tcgen05
 * GEMM), its core (anelm_full_attn_decode / anelm_deltanet_decode) and its out-projection
 * without leaving the device.
 * w_in: bf16 [proj_dim][hidden] (attention: Hq*2d + 2*Hkv*d rows in the q|gate, k, v order of
 * qwen3_5.cpp:948-950; DeltaNet: 2*Hk*dk + 2*Hv*dv + 2*Hv rows, qkv | z | a | b of
 * qwen3_5.cpp:853-860); w_out: bf16 [hidden][core out] (Hq*d or Hv*dv).  Host or device
 * pointers; hidden a multiple of 8. */
ANELM_API int anelm_set_layer_projections(anelm_ctx* ctx, int layer, int hidden, const void* w_in,
                                          const void* w_out);
/* x [n][hidden] bf16 -> y [n][hidden] bf16 for the plan's n rows; pos [n] (attention layers). */
ANELM_API int anelm_layer_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* x,
                                 const int* pos, void* y, void* stream);

/* ---- prefill ---- */

/* Causal prefill of the plan's sequences, each of n_tokens prompt tokens, on top
 * of whatever their rings already hold.  Equivalent to n_tokens successive
 * forward_full_attn_from_proj calls at positions start_pos, start_pos+1, ... (the
 * per-token loop of qwen3_5.cpp:1205-1217 / serve_hybrid.py:368-370, and the
 * chunks of forward_batch, qwen3_5.cpp:1164-1217, that generate.cpp:57-73 feeds at
 * a running start_pos), computed as one causal attention on the tcgen05 tensor
 * cores: token t attends to the ring's old tokens and the new tokens 0..t, at most
 * `capacity` tokens in all, and is appended as the reference's ring update does
 * (qwen3_5.cpp:974-983), so a prompt may continue an earlier turn and may be
 * longer than the ring (the ring slides).  Afterwards len / start are what the
 * per-token loop leaves and decode continues from there.  One start_pos for all
 * the plan's sequences.  proj: [n_seqs][n_tokens][proj_dim] of proj_dtype; out:
 * [n_seqs][n_tokens][Hq*d].  head_dim 256 only.  A linear cache (kv_mode
 * ANELM_KV_LINEAR) is filled only from position 0 of an empty cache, n_tokens <=
 * capacity.  Uses a context-owned staging buffer sized for the old tokens the
 * first new token sees (min(len, capacity - 1) per sequence): prefill calls on
 * one context must not overlap on the GPU. */
ANELM_API int anelm_full_attn_prefill(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                      const void* proj, int proj_dtype, int start_pos, void* out, int out_dtype,
                                      void* stream);

/* Head-sharded prefill with the all-gather fused into the attention kernel.  A long prompt split
 * over GPUs by head (each rank's context holds its share of the query heads and their KV heads)
 * ends in an all-gather of the gated outputs; here each rank's attention epilogue stores its
 * output tiles by TMA straight into every rank's output buffer (over NVLink for the peers), so the
 * transfer overlaps the attention tile by tile and no separate collective moves the data.  outs:
 * n_outs (<= 8) device addresses usable on this context's device -- this rank's own buffer and the
 * peers' buffers mapped with anelm_ipc_open -- each [n_seqs][n_tokens][out_cols] of out_dtype
 * (bf16 or fp16, 16-byte aligned); this context's Hq heads fill columns [col0, col0 + Hq*d) (col0 a
 * multiple of 64) of every one.  Otherwise as anelm_full_attn_prefill.  The stores have completed
 * when this call's kernels have; a rank may read its buffer once every rank's call has completed
 * (order that with a collective on the same stream, e.g. a one-element all-reduce), and may start
 * the next call into the same buffers only after every rank has finished reading.
 * Replaces: the prefill loop of qwen3_5.cpp:1205-1217 for one sequence spread over GPUs (the
 * reference has no multi-device path). */
ANELM_API int anelm_full_attn_prefill_gather(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                             const void* proj, int proj_dtype, int start_pos, void* const* outs,
                                             int n_outs, int col0, int out_cols, int out_dtype, void* stream);

/* CUDA IPC plumbing for the peer buffers above (one process per GPU): anelm_ipc_handle gives the
 * 64-byte handle of the allocation holding dev_ptr and dev_ptr's offset in it; another process
 * maps it with anelm_ipc_open (peer access enabled on `device`) and unmaps it with anelm_ipc_close.
 * No counterpart in the reference. */
ANELM_API int anelm_ipc_handle(const void* dev_ptr, void* handle_out, size_t* offset_out);
ANELM_API int anelm_ipc_open(const void* handle, size_t offset, int device, void** ptr_out);
ANELM_API int anelm_ipc_close(void* ptr);

/* Prefill of the plan's sequences through a Gated DeltaNet layer: equivalent to n_tokens
 * successive forward_deltanet_from_proj calls (qwen3_5.cpp:849-909, the per-token loop
 * of qwen3_5.cpp:1205-1217), computed chunkwise (64-token chunks, WY form).  Continues
 * from each sequence's current state, conv ring and ring position, and leaves them as
 * the token loop would.  proj: [n_seqs][n_tokens][proj_dim]; out: [n_seqs][n_tokens][Hv*dv].
 * key/value head dims 128 only.  Uses a context-owned staging buffer: prefill calls on
 * one context must not overlap on the GPU. */
ANELM_API int anelm_deltanet_prefill(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                     const void* proj, int proj_dtype, void* out, int out_dtype, void* stream);

/* The chunked gated delta rule alone (no conv, norms or gates): for each of B sequences
 * and value head h (key head h / (Hv/Hk)), over tokens t = 0..T-1,
 *   ANELM_DELTA_CPUOPS (ssm_step, cpu_ops.cpp:131-146): S = g S + beta k (v - S^T k)^T
 *   ANELM_DELTA_HF (export_hybrid_chunks.py:142-147):    S = g S; S += beta k (v - S^T k)^T
 * then y = S^T q, with g = exp(log_decay).  q, k [B][T][Hk][dk], v [B][T][Hv][dv] of
 * qkv_dtype (device); log_decay, beta [B][T][Hv] fp32; state [B][Hv][dk][dv] fp32, read
 * and written in place; y [B][T][Hv][dv] of y_dtype.  dk = dv = 128.  workspace: device
 * memory of at least anelm_gated_delta_chunked_workspace_bytes(B, T, Hk, Hv) bytes (the
 * call allocates nothing). */
ANELM_API size_t anelm_gated_delta_chunked_workspace_bytes(int B, int T, int Hk, int Hv);
ANELM_API int anelm_gated_delta_chunked(const void* q, const void* k, const void* v, int qkv_dtype,
                                        const float* log_decay, const float* beta, float* state, int B, int T,
                                        int Hk, int Hv, int dk, int dv, int delta_mode, void* y, int y_dtype,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* ---- Python route: scripts/serve_hybrid.py cpu_attention ---- */

/* Drop-in for cpu_attention(q_gate_fp16, k_fp16, v_fp16, pos, kv_caches, layer_idx)
 * (scripts/serve_hybrid.py:85-132): HOST fp16 buffers q_gate [Hq][2d], k [Hkv][d],
 * v [Hkv][d]; out [Hq*d] fp16.  KV lives in the context (sequence `seq`);
 * the context must be created with rope_mode = ANELM_ROPE_HALF,
 * qk_norm_in_core = 0 and kv_mode = ANELM_KV_LINEAR.  Synchronous on `stream`. */
ANELM_API int anelm_py_cpu_attention(anelm_ctx* ctx, int layer, int seq, const uint16_t* q_gate_host,
                                     const uint16_t* k_host, const uint16_t* v_host, int pos,
                                     uint16_t* out_host, void* stream);

/* ---- op-level entry points (core/cpu_ops.h), device pointers, fp32 ---- */

/* gqa_attention (core/cpu_ops.cpp:148-204) over a caller-owned ring in the
 * reference layout: q [n_heads][q_head_stride], k/v cache
 * [cache_capacity][n_kv_heads][head_dim] of kv_dtype (F32 or F16), out
 * [n_heads][head_dim] fp32.  cache_len <= 0 writes zeros (cpu_ops.cpp:152-155). */
ANELM_API int anelm_gqa_attention(float* out, const float* q, const void* k_cache,
                                  const void* v_cache, int kv_dtype, int n_heads, int n_kv_heads,
                                  int head_dim, int q_head_stride, int cache_start, int cache_len,
                                  int cache_capacity, void* stream);

/* Dense projection on the tensor cores: C[M][N] = A[M][K] * B[N][K]^T with bf16 A, B
 * (nn.Linear layout: A = activations [rows][in], B = weights [out][in]), fp32 accumulation,
 * C of c_dtype (ANELM_BF16 / ANELM_F16 / ANELM_F32) with row stride ldc.  The reference runs
 * these projections on the ANE around the CPU core: first_proj and o_proj,
 * models/llm/qwen3_5.cpp:912-1012, core/ane_runtime.cpp:279-361.  Device pointers; A and B
 * 16-byte aligned, lda and ldb multiples of 8 (ANELM_ERR_UNSUPPORTED otherwise). */
ANELM_API int anelm_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc,
                              int c_dtype, int M, int N, int K, void* stream);

/* LM head with in-model top-k: the k (<= 32) largest logits of each row of h [n][hidden] times
 * W [vocab][hidden]^T (bf16, nn.Linear layout), values (fp32) and vocabulary indices sorted
 * descending — LMHeadArgmax of scripts/export_hybrid_chunks.py:409-421 (torch.topk(32) on the
 * ANE so that 2 x 32 values instead of the vocabulary's logits leave it), read by
 * serve_hybrid.py:283-307.  The logits are never written: each CTA keeps, per row, a running
 * top-32 over the vocabulary tiles it streams (candidate lists in `workspace`, at least
 * anelm_lm_head_topk_workspace_bytes(n, vocab) bytes, 16-byte aligned; the size depends on n)
 * and a second kernel merges them.  Ties between equal logits may order differently than torch.topk. */
ANELM_API size_t anelm_lm_head_topk_workspace_bytes(int n, int vocab);
ANELM_API int anelm_lm_head_topk(const void* h, long long ldh, const void* W, long long ldw, int n, int vocab,
                                 int hidden, int k, float* top_vals, int* top_idx, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Allocation-free variant of anelm_gqa_attention for fp16 caches.  No
 * counterpart in the reference.  For callers that cannot allocate device memory
 * where attention runs: a server whose own pool already holds all free HBM (a
 * cudaMalloc / cudaMallocAsync there would fail or fragment it) or a plugin host
 * that owns the allocator.  anelm_gqa_attention draws its split-K scratch from
 * the stream-ordered pool on each call; this one uses a fixed device array of
 * ANELM_GQA_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads
 * the library holds until the process exits.  It calls no cudaMalloc / cudaFree
 * and no allocating library routine.  Arguments as anelm_gqa_attention with
 * kv_dtype = ANELM_F16 implied.  Limit: the scratch holds partial results of
 * (ANELM_GQA_NOALLOC_SCRATCH_BYTES - 16 KiB) / (n_kv_heads * (4*head_dim + 8) * 4)
 * splits; longer caches get longer splits, and a configuration whose single
 * split does not fit is rejected with ANELM_ERR_CAPACITY.  All calls on a device
 * share the array and it keeps the last call's contents (the call clears what
 * must start at zero): calls whose executions overlap on the GPU race on it.
 * The first call on each device looks the array's device address up
 * (cudaGetSymbolAddress, with that device current); make it before any stream
 * capture. */
#define ANELM_GQA_NOALLOC_SCRATCH_BYTES (4u << 20)
ANELM_API int anelm_gqa_attention_noalloc(float* out, const float* q, const void* k_cache, const void* v_cache,
                                          int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                                          int cache_start, int cache_len, int cache_capacity, void* stream);

/* ssm_step (core/cpu_ops.cpp:131-146): state [key_dim][value_dim] updated in place. */
ANELM_API int anelm_ssm_step(float* y, float* state, const float* q, const float* k, const float* v,
                             float decay, float beta, int key_dim, int value_dim, void* stream);

/* conv1d_update (core/cpu_ops.cpp:89-129): conv_state [channels][kernel_size-1],
 * *state_pos is a HOST int advanced by this call. */
ANELM_API int anelm_conv1d_update(float* y, float* conv_state, int* state_pos_host, const float* x,
                                  const float* w, int channels, int kernel_size, void* stream);

/* rmsnorm / rmsnorm_gated (core/cpu_ops.cpp:24-38), over `rows` vectors of dim
 * (the reference calls them once per head). */
ANELM_API int anelm_rmsnorm(float* out, const float* x, const float* weight, int dim, float eps,
                            int rows, void* stream);
ANELM_API int anelm_rmsnorm_gated(float* out, const float* x, const float* z, const float* weight,
                                  int dim, int rows, void* stream);

/* apply_rope_cached (core/cpu_ops.cpp:40-63).  cos_row/sin_row are device
 * [rot_dim/2] or NULL (then computed from pos and theta). */
ANELM_API int anelm_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                                      int head_dim, int q_head_stride, int k_head_stride,
                                      int rot_dim, int pos, float theta, const float* cos_row,
                                      const float* sin_row, void* stream);

/* l2_normalize (82-87), silu_vec_inplace (6-13), mul_sigmoid_inplace (15-22),
 * softmax (65-75), each over `rows` contiguous vectors of n. */
ANELM_API int anelm_l2_normalize(float* x, int dim, int rows, void* stream);
ANELM_API int anelm_silu_vec_inplace(float* x, int n, void* stream);
ANELM_API int anelm_mul_sigmoid_inplace(float* y, const float* z, int n, void* stream);
ANELM_API int anelm_softmax(float* x, int n, int rows, void* stream);

/* matvec (core/cpu_ops.cpp:77-80): y = W x, W row-major [out_dim][in_dim]. */
ANELM_API int anelm_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim,
                           void* stream);

/* Self-test of the failure path every tensor-core kernel here shares: one thread waits on an
 * mbarrier that nothing ever arrives on, with the kernels' bounded wait, gives up after `polls`
 * polls (1 .. 2^22) and records ANELM_ERR_TIMEOUT in the context's device error word, which
 * anelm_get_device_error then returns (and clears); the context stays usable.  No counterpart in
 * the reference (its CPU core has no waits).  Asynchronous on `stream`. */
ANELM_API int anelm_selftest_wait_timeout(anelm_ctx* ctx, unsigned polls, void* stream);

/* Library / device introspection (no GPU needed for the version). */
ANELM_API const char* anelm_version(void);
ANELM_API int anelm_device_check(int device);

#ifdef __cplusplus
}
#endif

#endif /* ANELM_B200_H */
