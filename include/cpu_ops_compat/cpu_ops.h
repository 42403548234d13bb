/*
 * Link-compatible replacement for ANE-LM's core/cpu_ops.h (namespace ane_lm), backed by the
 * B200 kernels of libanelm_b200.so.
 *
 * Put this directory ahead of the reference's core/ on the include path and link
 * libanelm_b200.so instead of compiling core/cpu_ops.cpp: the reference's callers
 * (models/llm/qwen3_5.cpp) then run unchanged, every op on the GPU.  Each function has the
 * reference's exact signature (core/cpu_ops.h:16-58) and semantics: HOST pointers in and out,
 * synchronous.  Each call copies its inputs to device scratch owned by the calling thread, runs
 * the matching anelm_* op and copies the results back, so this route is for drop-in
 * compatibility, not speed; the fast path is the context API of anelm_b200.h, whose state
 * stays on the device.  A CUDA failure prints the library's last error and aborts (the
 * reference's functions cannot report errors).
 */
#pragma once

#include <cmath>

namespace ane_lm {

/* core/cpu_ops.h:12-14 */
inline float silu_f(float x) { return x / (1.0f + std::exp(-x)); }
inline float sigmoid_f(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float softplus_f(float x) { return std::log(1.0f + std::exp(x)); }

/* core/cpu_ops.h:16-17 (tmp: n floats of caller scratch, unused here) */
void silu_vec_inplace(float* x, int n, float* tmp);
void mul_sigmoid_inplace(float* y, const float* z, int n, float* tmp);

/* core/cpu_ops.h:21-22 */
void rmsnorm(float* out, const float* x, const float* weight, int dim, float eps = 1e-6f);
void rmsnorm_gated(float* out, const float* x, const float* z, const float* weight, int dim);

/* core/cpu_ops.h:26-29 (cos_row / sin_row: host [rot_dim/2] or null) */
void apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads,
                       int head_dim, int q_head_stride, int k_head_stride,
                       int rot_dim, int pos, float theta,
                       const float* cos_row, const float* sin_row);

/* core/cpu_ops.h:33, 37, 41 */
void softmax(float* x, int n);
void matvec(float* y, const float* W, const float* x, int out_dim, int in_dim);
void l2_normalize(float* x, int dim);

/* core/cpu_ops.h:45-46: conv_state [channels][kernel_size-1], *state_pos advanced */
void conv1d_update(float* y, float* conv_state, int* state_pos, const float* x,
                   const float* w, int channels, int kernel_size);

/* core/cpu_ops.h:50-51: state [key_dim][value_dim] updated in place */
void ssm_step(float* y, float* state, const float* q, const float* k,
              const float* v, float decay, float beta, int key_dim, int value_dim);

/* core/cpu_ops.h:55-58: fp32 ring [cache_capacity][n_kv_heads][head_dim] */
void gqa_attention(float* out, const float* q,
                   const float* k_cache, const float* v_cache,
                   int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                   int cache_start, int cache_len, int cache_capacity);

}  // namespace ane_lm
