/*
 * anelm oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement, in plain C, of the attention core that ANE-LM runs on the
 * host between its Neural Engine projection chunks.  It exists to check the
 * CUDA library; nothing in the product links, loads or calls it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg may use it.
 *
 * Parity pin: the same glue (oracle/glue_impl.h) is also compiled against the
 * reference's own core/cpu_ops.cpp (built unmodified by oracle/Makefile into
 * oracle/_ref/), and the golden fixtures in tests/golden/ are outputs of that
 * reference build on seeded inputs.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the ANE-LM project root).
 */
#ifndef ANELM_ORACLE_H
#define ANELM_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ops: core/cpu_ops.h:16-58 / core/cpu_ops.cpp ---- */
void orc_silu_vec_inplace(float* x, int n, float* tmp);                       /* cpu_ops.cpp:6-13 */
void orc_mul_sigmoid_inplace(float* y, const float* z, int n, float* tmp);    /* cpu_ops.cpp:15-22 */
void orc_rmsnorm(float* out, const float* x, const float* weight, int dim, float eps); /* 24-30 */
void orc_rmsnorm_gated(float* out, const float* x, const float* z,
                       const float* weight, int dim);                          /* cpu_ops.cpp:32-38 */
void orc_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                           int head_dim, int q_head_stride, int k_head_stride,
                           int rot_dim, int pos, float theta,
                           const float* cos_row, const float* sin_row);        /* cpu_ops.cpp:40-63 */
void orc_softmax(float* x, int n);                                             /* cpu_ops.cpp:65-75 */
void orc_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim); /* 77-80 */
void orc_l2_normalize(float* x, int dim);                                      /* cpu_ops.cpp:82-87 */
void orc_conv1d_update(float* y, float* conv_state, int* state_pos, const float* x,
                       const float* w, int channels, int kernel_size);         /* cpu_ops.cpp:89-129 */
void orc_ssm_step(float* y, float* state, const float* q, const float* k,
                  const float* v, float decay, float beta, int key_dim, int value_dim); /* 131-146 */
void orc_gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                       int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                       int cache_start, int cache_len, int cache_capacity);    /* cpu_ops.cpp:148-204 */

/* ---- layer glue: models/llm/qwen3_5.cpp:849-1002 (see glue_impl.h) ---- */

/* Shape parameters; field meaning follows Qwen35Args (models/llm/qwen3_5.h:51-80). */
typedef struct {
    int num_q_heads, num_kv_heads, head_dim, rot_dim;
    float rope_theta, rms_eps;
    int attn_output_gate;
    int lin_num_key_heads, lin_num_val_heads, lin_key_dim, lin_val_dim, conv_kernel;
} orc_shape;

/* Variant switches.  All zero = the C++ cpu_ops path (the default oracle). */
typedef struct {
    int rope_half;        /* 1: rotate-half pairing (scripts/serve_hybrid.py:94-103) */
    int no_qk_norm;       /* 1: QK-norm done before the core (export_hybrid_chunks.py:193-197) */
    int kv_linear;        /* 1: linear KV, slot = pos, len = pos+1 (serve_hybrid.py:105-108) */
    int kv_round_f16;     /* 1: K/V rounded to fp16 when written (models fp16 KV storage) */
    int delta_hf;         /* 1: decay-first delta rule (export_hybrid_chunks.py:142-147) */
    float l2_eps;         /* 0 => 1e-12 inside sqrt (cpu_ops.cpp:85); HF uses 1e-6 */
} orc_variant;

/* RoPE cos/sin table [n_pos][rot_dim/2] as built by qwen3_5.cpp:309-324. */
void orc_rope_table(float* cos_tab, float* sin_tab, int n_pos, int rot_dim, float theta);

/* One token of forward_full_attn_from_proj (qwen3_5.cpp:944-1002).  proj is
 * [q_gate (Hq*2d) | k (Hkv*d) | v (Hkv*d)] and is modified in place exactly as the
 * reference does.  KV cache is slot-major [capacity][Hkv][d] fp32.  rope tables
 * may be NULL (then the on-the-fly formula of cpu_ops.cpp:51-56 is used).
 * tmp must hold head_dim floats.  Returns 0 on success. */
int orc_full_attn_from_proj(const orc_shape* s, const orc_variant* var,
                            const float* q_norm, const float* k_norm,
                            float* k_cache, float* v_cache, int* len, int* start, int capacity,
                            const float* rope_cos, const float* rope_sin, int rope_table_len,
                            float* proj, int pos, float* out, float* tmp);

/* One token of forward_deltanet_from_proj (qwen3_5.cpp:849-910), norm-fused
 * layout: proj = [mixed_qkv (C) | z (Hv*dv) | a (Hv) | b (Hv)].  A holds exp(A_log)
 * (qwen3_5.cpp:417-421).  conv_state is [C][K-1] with ring index *conv_pos.
 * scratch must hold 2*C + Hv*dv floats.  Returns 0 on success. */
int orc_deltanet_from_proj(const orc_shape* s, const orc_variant* var,
                           const float* conv_w, const float* A, const float* dt_bias,
                           const float* norm_w, float* ssm_state, float* conv_state,
                           int* conv_pos, const float* proj, float* out, float* scratch);

/* Convenience: n_tokens successive DeltaNet steps (the per-token loop of
 * qwen3_5.cpp:1205-1217).  proj is [n_tokens][proj_dim] (copied, not modified),
 * out is [n_tokens][Hv*dv]. */
int orc_gated_delta_tokens(int T, int Hk, int Hv, int dk, int dv, int delta_hf, const float* q,
                           const float* k, const float* v, const float* log_decay,
                           const float* beta, float* state, float* y);
int orc_deltanet_tokens(const orc_shape* s, const orc_variant* var,
                        const float* conv_w, const float* A, const float* dt_bias,
                        const float* norm_w, float* ssm_state, float* conv_state,
                        int* conv_pos, const float* proj, int n_tokens, float* out);

/* Convenience: n_tokens successive full-attention steps at positions
 * start_pos, start_pos+1, ... (qwen3_5.cpp:1205-1217).  proj is copied. */
int orc_full_attn_tokens(const orc_shape* s, const orc_variant* var,
                         const float* q_norm, const float* k_norm,
                         float* k_cache, float* v_cache, int* len, int* start, int capacity,
                         const float* rope_cos, const float* rope_sin, int rope_table_len,
                         const float* proj, int start_pos, int n_tokens, float* out);

#ifdef __cplusplus
}
#endif

#endif /* ANELM_ORACLE_H */
