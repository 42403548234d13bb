/*
 * anelm oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * Restatement of the Qwen3.5 layer glue around the CPU attention core,
 * models/llm/qwen3_5.cpp:849-1002 (forward_deltanet_from_proj and
 * forward_full_attn_from_proj), calling the cpu_ops in the same order.
 *
 * This file is included twice:
 *   - by anelm_oracle.c with OP(x) = orc_x       (our C restatement of cpu_ops), and
 *   - by ref_glue.cpp  with OP(x) = ane_lm::x    (the reference's own cpu_ops.cpp),
 * so the two oracle builds differ only in which cpu_ops they call.
 * The caller defines OP(name) and GLUE(name) before including it.
 *
 * The variant switches (orc_variant) add the Python / Hugging Face forms of the
 * same math that the reference uses elsewhere; with all switches zero the code
 * below is the qwen3_5.cpp path.
 */

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float glue_sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }   /* cpu_ops.h:13 */
static inline float glue_softplus_f(float x) { return logf(1.0f + expf(x)); }      /* cpu_ops.h:14 */

static inline float glue_round_f16(float x) { return (float)(_Float16)x; }

/* Rotate-half RoPE on dims [0, R/2) and [R/2, R): scripts/serve_hybrid.py:94-103
 * (also scripts/export_fused_attention.py:113-122).  Frequencies are those of
 * the table in qwen3_5.cpp:309-324 (inv_freq[j] = theta^(-2j/R)). */
static void glue_rope_half(float* v, int rot_dim, int pos, float theta,
                           const float* cos_row, const float* sin_row) {
    int half = rot_dim / 2;
    for (int j = 0; j < half; j++) {
        float c, s;
        if (cos_row && sin_row) {
            c = cos_row[j];
            s = sin_row[j];
        } else {
            float freq = 1.0f / powf(theta, (float)(2 * j) / (float)rot_dim);
            float angle = pos * freq;
            c = cosf(angle);
            s = sinf(angle);
        }
        float x1 = v[j], x2 = v[j + half];
        v[j] = x1 * c - x2 * s;
        v[j + half] = x2 * c + x1 * s;
    }
}

/* L2 normalisation with an explicit eps: x * 1/sqrt(sum x^2 + eps)
 * (HF form, transformers qwen3_5 l2norm; validate_deltanet.py:48-51). */
static void glue_l2_eps(float* x, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss + eps);
    for (int i = 0; i < dim; i++) x[i] = x[i] * inv;
}

/* Decay-first delta rule, scripts/export_hybrid_chunks.py:142-147:
 * S = g*S; Sk = S^T k; delta = (v - Sk)*beta; S += k delta^T; y = S^T q. */
static void glue_ssm_step_hf(float* y, float* state, const float* q, const float* k,
                             const float* v, float decay, float beta, int key_dim, int value_dim) {
    float* delta = (float*)malloc((size_t)value_dim * sizeof(float));
    for (int n = 0; n < key_dim * value_dim; n++) state[n] *= decay;
    for (int j = 0; j < value_dim; j++) {
        float s = 0.0f;
        for (int i = 0; i < key_dim; i++) s += state[(size_t)i * value_dim + j] * k[i];
        delta[j] = (v[j] - s) * beta;
    }
    for (int i = 0; i < key_dim; i++)
        for (int j = 0; j < value_dim; j++) state[(size_t)i * value_dim + j] += k[i] * delta[j];
    for (int j = 0; j < value_dim; j++) {
        float s = 0.0f;
        for (int i = 0; i < key_dim; i++) s += state[(size_t)i * value_dim + j] * q[i];
        y[j] = s;
    }
    free(delta);
}

/* qwen3_5.cpp:944-1002 */
int GLUE(full_attn_from_proj)(const orc_shape* s, const orc_variant* var,
                              const float* q_norm, const float* k_norm,
                              float* k_cache, float* v_cache, int* len, int* start, int capacity,
                              const float* rope_cos, const float* rope_sin, int rope_table_len,
                              float* proj, int pos, float* out, float* tmp) {
    static const orc_variant zero_var = {0, 0, 0, 0, 0, 0.0f};
    if (!var) var = &zero_var;
    const int Hq = s->num_q_heads, Hkv = s->num_kv_heads, d = s->head_dim, R = s->rot_dim;
    if (Hq <= 0 || Hkv <= 0 || Hq % Hkv || capacity <= 0) return -1;
    float* q_gate = proj;                              /* 948 */
    float* k_raw = proj + (size_t)Hq * d * 2;          /* 949 */
    float* v_raw = k_raw + (size_t)Hkv * d;            /* 950 */

    if (!var->no_qk_norm) {                            /* 952-959 */
        for (int h = 0; h < Hq; h++) {
            float* qh = q_gate + (size_t)h * d * 2;
            OP(rmsnorm)(qh, qh, q_norm, d, s->rms_eps);
        }
        for (int h = 0; h < Hkv; h++)
            OP(rmsnorm)(k_raw + (size_t)h * d, k_raw + (size_t)h * d, k_norm, d, s->rms_eps);
    }

    const float* cos_row = NULL;                       /* 961-968 */
    const float* sin_row = NULL;
    if (pos >= 0 && pos < rope_table_len && rope_cos && rope_sin) {
        cos_row = rope_cos + (size_t)pos * (R / 2);
        sin_row = rope_sin + (size_t)pos * (R / 2);
    }
    if (!var->rope_half) {                             /* 969-971 */
        OP(apply_rope_cached)(q_gate, k_raw, Hq, Hkv, d, d * 2, d, R, pos, s->rope_theta,
                              cos_row, sin_row);
    } else {
        for (int h = 0; h < Hq; h++)
            glue_rope_half(q_gate + (size_t)h * d * 2, R, pos, s->rope_theta, cos_row, sin_row);
        for (int h = 0; h < Hkv; h++)
            glue_rope_half(k_raw + (size_t)h * d, R, pos, s->rope_theta, cos_row, sin_row);
    }

    int slot;                                          /* 973-983 */
    if (var->kv_linear) {                              /* serve_hybrid.py:105-108 */
        if (pos < 0 || pos >= capacity) return -2;
        slot = pos;
        *len = pos + 1;
        *start = 0;
    } else if (*len < capacity) {
        slot = *start + *len;
        if (slot >= capacity) slot -= capacity;
        (*len)++;
    } else {
        slot = *start;
        (*start)++;
        if (*start >= capacity) *start = 0;
    }
    size_t kv_stride = (size_t)Hkv * d;                /* 984-986 */
    if (var->kv_round_f16) {
        for (size_t i = 0; i < kv_stride; i++) {
            k_cache[(size_t)slot * kv_stride + i] = glue_round_f16(k_raw[i]);
            v_cache[(size_t)slot * kv_stride + i] = glue_round_f16(v_raw[i]);
        }
    } else {
        memcpy(k_cache + (size_t)slot * kv_stride, k_raw, kv_stride * sizeof(float));
        memcpy(v_cache + (size_t)slot * kv_stride, v_raw, kv_stride * sizeof(float));
    }

    OP(gqa_attention)(out, q_gate, k_cache, v_cache, Hq, Hkv, d, d * 2,  /* 988-991 */
                      *start, *len, capacity);

    if (s->attn_output_gate) {                         /* 993-1000 */
        for (int h = 0; h < Hq; h++) {
            float* oh = out + (size_t)h * d;
            const float* gh = q_gate + (size_t)h * d * 2 + d;
            OP(mul_sigmoid_inplace)(oh, gh, d, tmp);
        }
    }
    return 0;
}

/* qwen3_5.cpp:849-910 (norm_fused layout) */
int GLUE(deltanet_from_proj)(const orc_shape* s, const orc_variant* var,
                             const float* conv_w, const float* A, const float* dt_bias,
                             const float* norm_w, float* ssm_state, float* conv_state,
                             int* conv_pos, const float* proj, float* out, float* scratch) {
    static const orc_variant zero_var = {0, 0, 0, 0, 0, 0.0f};
    if (!var) var = &zero_var;
    const int Hk = s->lin_num_key_heads, Hv = s->lin_num_val_heads;
    const int dk = s->lin_key_dim, dv = s->lin_val_dim;
    if (Hk <= 0 || Hv <= 0 || Hv % Hk) return -1;
    const int key_total = Hk * dk, val_total = Hv * dv;
    const int C = 2 * key_total + val_total;

    const float* mixed_qkv = proj;                     /* 853 */
    const float* z = proj + C;                         /* 854 */
    const float* a_vec = proj + C + val_total;         /* 859 */
    const float* b_vec = a_vec + Hv;                   /* 860 */

    float* conv_out = scratch;
    float* silu_tmp = scratch + C;
    float* y = scratch + 2 * C;

    OP(conv1d_update)(conv_out, conv_state, conv_pos, mixed_qkv, conv_w, C, s->conv_kernel); /* 869 */
    OP(silu_vec_inplace)(conv_out, C, silu_tmp);                                             /* 870 */

    float* Q = conv_out;                               /* 873-875 */
    float* K = conv_out + key_total;
    float* V = conv_out + 2 * key_total;

    float q_scale = 1.0f / sqrtf((float)dk);           /* 879 */
    int kv_group = Hv / Hk;                            /* 880 */
    for (int kh = 0; kh < Hk; kh++) {                  /* 882-887 */
        if (var->l2_eps == 0.0f) {
            OP(l2_normalize)(Q + (size_t)kh * dk, dk);
            OP(l2_normalize)(K + (size_t)kh * dk, dk);
        } else {
            glue_l2_eps(Q + (size_t)kh * dk, dk, var->l2_eps);
            glue_l2_eps(K + (size_t)kh * dk, dk, var->l2_eps);
        }
        for (int i = 0; i < dk; i++) Q[(size_t)kh * dk + i] = Q[(size_t)kh * dk + i] * q_scale;
    }

    for (int h = 0; h < Hv; h++) {                     /* 889-900 */
        int kh_idx = (kv_group > 1) ? (h / kv_group) : h;
        float* qh = Q + (size_t)kh_idx * dk;
        float* kh_ptr = K + (size_t)kh_idx * dk;
        float* vh = V + (size_t)h * dv;
        float* yh = y + (size_t)h * dv;
        float* state = ssm_state + (size_t)h * dk * dv;
        float beta = glue_sigmoid_f(b_vec[h]);
        float decay = expf(-A[h] * glue_softplus_f(a_vec[h] + dt_bias[h]));
        if (!var->delta_hf)
            OP(ssm_step)(yh, state, qh, kh_ptr, vh, decay, beta, dk, dv);
        else
            glue_ssm_step_hf(yh, state, qh, kh_ptr, vh, decay, beta, dk, dv);
    }

    for (int h = 0; h < Hv; h++)                       /* 902-908 */
        OP(rmsnorm_gated)(out + (size_t)h * dv, y + (size_t)h * dv, z + (size_t)h * dv, norm_w, dv);
    return 0;
}

/* The delta-rule core alone over T tokens (the per-head step of qwen3_5.cpp:889-900 without
 * conv, norms and gates): q, k [T][Hk][dk], v [T][Hv][dv], log_decay, beta [T][Hv],
 * state [Hv][dk][dv] (updated in place), y [T][Hv][dv].  Value head h reads key head
 * h / (Hv / Hk) (qwen3_5.cpp:891).  delta_hf selects the decay-first order. */
int GLUE(gated_delta_tokens)(int T, int Hk, int Hv, int dk, int dv, int delta_hf, const float* q,
                             const float* k, const float* v, const float* log_decay,
                             const float* beta, float* state, float* y) {
    if (Hk <= 0 || Hv <= 0 || Hv % Hk) return -1;
    const int group = Hv / Hk;
    for (int t = 0; t < T; t++)
        for (int h = 0; h < Hv; h++) {
            const int kh = h / group;
            const float* qh = q + ((size_t)t * Hk + kh) * dk;
            const float* kp = k + ((size_t)t * Hk + kh) * dk;
            const float* vh = v + ((size_t)t * Hv + h) * dv;
            float* yh = y + ((size_t)t * Hv + h) * dv;
            float* st = state + (size_t)h * dk * dv;
            const float decay = expf(log_decay[(size_t)t * Hv + h]);
            const float b = beta[(size_t)t * Hv + h];
            if (!delta_hf)
                OP(ssm_step)(yh, st, qh, kp, vh, decay, b, dk, dv);
            else
                glue_ssm_step_hf(yh, st, qh, kp, vh, decay, b, dk, dv);
        }
    return 0;
}

/* Per-token loop of qwen3_5.cpp:1205-1217 for the DeltaNet layer. */
int GLUE(deltanet_tokens)(const orc_shape* s, const orc_variant* var,
                          const float* conv_w, const float* A, const float* dt_bias,
                          const float* norm_w, float* ssm_state, float* conv_state,
                          int* conv_pos, const float* proj, int n_tokens, float* out) {
    const int C = 2 * s->lin_num_key_heads * s->lin_key_dim + s->lin_num_val_heads * s->lin_val_dim;
    const int val_total = s->lin_num_val_heads * s->lin_val_dim;
    const int proj_dim = C + val_total + 2 * s->lin_num_val_heads;
    float* scratch = (float*)malloc(((size_t)2 * C + val_total) * sizeof(float));
    int rc = 0;
    for (int t = 0; t < n_tokens && rc == 0; t++)
        rc = GLUE(deltanet_from_proj)(s, var, conv_w, A, dt_bias, norm_w, ssm_state, conv_state,
                                      conv_pos, proj + (size_t)t * proj_dim,
                                      out + (size_t)t * val_total, scratch);
    free(scratch);
    return rc;
}

/* Per-token loop of qwen3_5.cpp:1205-1217 for the full-attention layer. */
int GLUE(full_attn_tokens)(const orc_shape* s, const orc_variant* var,
                           const float* q_norm, const float* k_norm,
                           float* k_cache, float* v_cache, int* len, int* start, int capacity,
                           const float* rope_cos, const float* rope_sin, int rope_table_len,
                           const float* proj, int start_pos, int n_tokens, float* out) {
    const int Hq = s->num_q_heads, Hkv = s->num_kv_heads, d = s->head_dim;
    const size_t proj_dim = (size_t)Hq * 2 * d + (size_t)2 * Hkv * d;
    float* pbuf = (float*)malloc(proj_dim * sizeof(float));
    float* tmp = (float*)malloc((size_t)d * sizeof(float));
    int rc = 0;
    for (int t = 0; t < n_tokens && rc == 0; t++) {
        memcpy(pbuf, proj + (size_t)t * proj_dim, proj_dim * sizeof(float));
        rc = GLUE(full_attn_from_proj)(s, var, q_norm, k_norm, k_cache, v_cache, len, start,
                                       capacity, rope_cos, rope_sin, rope_table_len, pbuf,
                                       start_pos + t, out + (size_t)t * Hq * d, tmp);
    }
    free(pbuf);
    free(tmp);
    return rc;
}
