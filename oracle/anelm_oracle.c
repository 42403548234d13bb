/*
 * anelm oracle -- TEST INFRASTRUCTURE ONLY (see anelm_oracle.h).
 *
 * Plain-C restatement of the reference's core/cpu_ops.cpp.  Each Accelerate call
 * the reference makes is written as the loop that Accelerate documents, in the
 * same order as oracle/shim/Accelerate/Accelerate.h, so that this file and the
 * reference compiled against that shim agree bit for bit (-ffp-contract=off).
 */
#include "anelm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float orc_sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); } /* cpu_ops.h:13 */
static inline float orc_softplus_f(float x) { return logf(1.0f + expf(x)); }    /* cpu_ops.h:14 */

/* cpu_ops.cpp:6-13: tmp=-x; tmp=exp(tmp); tmp+=1; x=x/tmp */
void orc_silu_vec_inplace(float* x, int n, float* tmp) {
    for (int i = 0; i < n; i++) tmp[i] = -x[i];
    for (int i = 0; i < n; i++) tmp[i] = expf(tmp[i]);
    for (int i = 0; i < n; i++) tmp[i] = tmp[i] + 1.0f;
    for (int i = 0; i < n; i++) x[i] = x[i] / tmp[i];
}

/* cpu_ops.cpp:15-22: y = y / (1 + exp(-z)) */
void orc_mul_sigmoid_inplace(float* y, const float* z, int n, float* tmp) {
    for (int i = 0; i < n; i++) tmp[i] = -z[i];
    for (int i = 0; i < n; i++) tmp[i] = expf(tmp[i]);
    for (int i = 0; i < n; i++) tmp[i] = tmp[i] + 1.0f;
    for (int i = 0; i < n; i++) y[i] = y[i] / tmp[i];
}

/* cpu_ops.cpp:24-30 */
void orc_rmsnorm(float* out, const float* x, const float* weight, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / dim + eps);
    for (int i = 0; i < dim; i++) out[i] = x[i] * ss;
    for (int i = 0; i < dim; i++) out[i] = out[i] * weight[i];
}

/* cpu_ops.cpp:32-38: rmsnorm (eps 1e-6), then * sigmoid(z), then * z */
void orc_rmsnorm_gated(float* out, const float* x, const float* z, const float* weight, int dim) {
    orc_rmsnorm(out, x, weight, dim, 1e-6f);
    float* tmp = (float*)malloc((size_t)dim * sizeof(float));
    orc_mul_sigmoid_inplace(out, z, dim, tmp);
    free(tmp);
    for (int i = 0; i < dim; i++) out[i] = out[i] * z[i];
}

/* cpu_ops.cpp:40-63: interleaved pairs (v[i], v[i+1]) for i < rot_dim */
void orc_apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                           int head_dim, int q_head_stride, int k_head_stride,
                           int rot_dim, int pos, float theta,
                           const float* cos_row, const float* sin_row) {
    (void)head_dim;
    for (int h = 0; h < n_q_heads + n_kv_heads; h++) {
        float* v = (h < n_q_heads) ? q + (size_t)h * q_head_stride
                                   : k + (size_t)(h - n_q_heads) * k_head_stride;
        for (int i = 0, j = 0; i < rot_dim; i += 2, j++) {
            float cos_a, sin_a;
            if (cos_row && sin_row) {
                cos_a = cos_row[j];
                sin_a = sin_row[j];
            } else {
                float freq = 1.0f / powf(theta, (float)i / (float)rot_dim);
                float angle = pos * freq;
                cos_a = cosf(angle);
                sin_a = sinf(angle);
            }
            float v0 = v[i];
            float v1 = v[i + 1];
            v[i] = v0 * cos_a - v1 * sin_a;
            v[i + 1] = v0 * sin_a + v1 * cos_a;
        }
    }
}

/* cpu_ops.cpp:65-75 */
void orc_softmax(float* x, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

/* cpu_ops.cpp:77-80: y = W x, W row-major [out_dim][in_dim] */
void orc_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim) {
    for (int o = 0; o < out_dim; o++) {
        float s = 0.0f;
        for (int i = 0; i < in_dim; i++) s += W[(size_t)o * in_dim + i] * x[i];
        y[o] = s;
    }
}

/* cpu_ops.cpp:82-87 */
void orc_l2_normalize(float* x, int dim) {
    float norm = 0.0f;
    for (int i = 0; i < dim; i++) norm += x[i] * x[i];
    norm = 1.0f / sqrtf(norm + 1e-12f);
    for (int i = 0; i < dim; i++) x[i] = x[i] * norm;
}

/* cpu_ops.cpp:89-129: depthwise causal conv over a ring of kernel_size-1 inputs */
void orc_conv1d_update(float* y, float* conv_state, int* state_pos, const float* x,
                       const float* w, int channels, int kernel_size) {
    int state_len = kernel_size - 1;
    int pos = *state_pos;
    if (kernel_size == 4) {
        int p0 = pos;
        int p1 = pos + 1;
        if (p1 == 3) p1 = 0;
        int p2 = p1 + 1;
        if (p2 == 3) p2 = 0;
        for (int c = 0; c < channels; c++) {
            const int sb = c * 3, wb = c * 4;
            float s0 = conv_state[sb + p0], s1 = conv_state[sb + p1], s2 = conv_state[sb + p2];
            float xc = x[c];
            y[c] = s0 * w[wb] + s1 * w[wb + 1] + s2 * w[wb + 2] + xc * w[wb + 3];
            conv_state[sb + p0] = xc;
        }
    } else {
        for (int c = 0; c < channels; c++) {
            float sum = 0.0f;
            int base = c * state_len;
            for (int j = 0; j < state_len; j++) {
                int idx = pos + j;
                if (idx >= state_len) idx -= state_len;
                sum += conv_state[base + idx] * w[c * kernel_size + j];
            }
            float xc = x[c];
            y[c] = sum + xc * w[c * kernel_size + state_len];
            conv_state[base + pos] = xc;
        }
    }
    pos++;
    if (pos == state_len) pos = 0;
    *state_pos = pos;
}

/* cpu_ops.cpp:131-146: Sk = S^T k (undecayed); delta = v - Sk; S *= decay;
 * S += beta * k delta^T; y = S^T q.  S row-major [key_dim][value_dim]. */
void orc_ssm_step(float* y, float* state, const float* q, const float* k,
                  const float* v, float decay, float beta, int key_dim, int value_dim) {
    float* Sk = (float*)malloc((size_t)value_dim * sizeof(float));
    float* delta = (float*)malloc((size_t)value_dim * sizeof(float));
    for (int j = 0; j < value_dim; j++) {
        float s = 0.0f;
        for (int i = 0; i < key_dim; i++) s += state[(size_t)i * value_dim + j] * k[i];
        Sk[j] = 1.0f * s;
    }
    for (int j = 0; j < value_dim; j++) delta[j] = v[j] - Sk[j];
    for (int n = 0; n < key_dim * value_dim; n++) state[n] *= decay;
    for (int i = 0; i < key_dim; i++) {
        const float ax = beta * k[i];
        for (int j = 0; j < value_dim; j++) state[(size_t)i * value_dim + j] += ax * delta[j];
    }
    for (int j = 0; j < value_dim; j++) {
        float s = 0.0f;
        for (int i = 0; i < key_dim; i++) s += state[(size_t)i * value_dim + j] * q[i];
        y[j] = 1.0f * s;
    }
    free(Sk);
    free(delta);
}

/* cpu_ops.cpp:148-204: per q head, two passes over the ring in logical order
 * [cache_start, capacity) then [0, ...). */
void orc_gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                       int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                       int cache_start, int cache_len, int cache_capacity) {
    if (cache_len <= 0) {
        memset(out, 0, (size_t)n_heads * head_dim * sizeof(float));
        return;
    }
    int groups = n_heads / n_kv_heads;
    float scale = 1.0f / sqrtf((float)head_dim);
    size_t kv_step = (size_t)n_kv_heads * head_dim;
    int first_span = cache_capacity - cache_start;
    if (first_span > cache_len) first_span = cache_len;
    int second_span = cache_len - first_span;
    float* scores = (float*)malloc((size_t)cache_len * sizeof(float));
    for (int h = 0; h < n_heads; h++) {
        int kv_h = h / groups;
        const float* qh = q + (size_t)h * q_head_stride;
        float* oh = out + (size_t)h * head_dim;
        size_t kv_off = (size_t)kv_h * head_dim;
        int t = 0;
        for (int s = 0; s < cache_len; s++, t++) {
            size_t slot = (s < first_span) ? (size_t)(cache_start + s) : (size_t)(s - first_span);
            const float* kh = k_cache + slot * kv_step + kv_off;
            float dot = 0.0f;
            for (int i = 0; i < head_dim; i++) dot += qh[i] * kh[i];
            scores[t] = dot * scale;
        }
        orc_softmax(scores, cache_len);
        memset(oh, 0, (size_t)head_dim * sizeof(float));
        (void)second_span;
        for (int s = 0; s < cache_len; s++) {
            size_t slot = (s < first_span) ? (size_t)(cache_start + s) : (size_t)(s - first_span);
            const float* vh = v_cache + slot * kv_step + kv_off;
            const float sv = scores[s];
            for (int i = 0; i < head_dim; i++) oh[i] += sv * vh[i];
        }
    }
    free(scores);
}

/* qwen3_5.cpp:309-324 */
void orc_rope_table(float* cos_tab, float* sin_tab, int n_pos, int rot_dim, float theta) {
    int half_rot = rot_dim / 2;
    float* inv_freq = (float*)malloc((size_t)half_rot * sizeof(float));
    for (int j = 0, i = 0; i < rot_dim; i += 2, j++)
        inv_freq[j] = 1.0f / powf(theta, (float)i / (float)rot_dim);
    for (int pos = 0; pos < n_pos; pos++) {
        for (int j = 0; j < half_rot; j++) {
            float angle = pos * inv_freq[j];
            cos_tab[(size_t)pos * half_rot + j] = cosf(angle);
            sin_tab[(size_t)pos * half_rot + j] = sinf(angle);
        }
    }
    free(inv_freq);
}

/* The layer glue, built on the ops above. */
#define OP(name) orc_##name
#define GLUE(name) orc_##name
#include "glue_impl.h"
