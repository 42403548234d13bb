// Host-pointer ane_lm:: ops (include/cpu_ops_compat/cpu_ops.h) over the anelm_* op entries:
// the link-compatible drop-in for ANE-LM's core/cpu_ops.cpp.  Every call uploads its inputs to
// device scratch owned by the calling thread, runs the op on the default stream and downloads
// the results; the device work is synchronous with the call, as the reference's is.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include <cstddef>

#include "anelm_b200.h"
#include "cpu_ops_compat/cpu_ops.h"

#define SHIM_API __attribute__((visibility("default")))

namespace {

// Grown-on-demand device buffer (one set per thread, released when the thread exits).
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
    void* get(size_t need) {
        if (need > bytes) {
            if (ptr) cudaFree(ptr);
            ptr = nullptr;
            bytes = 0;
            if (cudaMalloc(&ptr, need) != cudaSuccess) {
                fprintf(stderr, "anelm cpu_ops shim: cudaMalloc of %zu bytes failed\n", need);
                abort();
            }
            bytes = need;
        }
        return ptr;
    }
    ~Scratch() {
        if (ptr) cudaFree(ptr);
    }
};
thread_local Scratch g_buf[8];

void check(int rc, const char* what) {
    if (rc != ANELM_OK) {
        fprintf(stderr, "anelm cpu_ops shim: %s: %s\n", what, anelm_last_error());
        abort();
    }
}
void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        fprintf(stderr, "anelm cpu_ops shim: %s: %s\n", what, cudaGetErrorString(e));
        abort();
    }
}

template <class T>
T* up(int slot, const T* host, size_t n) {
    T* d = static_cast<T*>(g_buf[slot].get(n * sizeof(T) > 0 ? n * sizeof(T) : 16));
    if (host && n) check_cuda(cudaMemcpy(d, host, n * sizeof(T), cudaMemcpyHostToDevice), "upload");
    return d;
}
template <class T>
void down(T* host, const T* dev, size_t n) {
    if (n) check_cuda(cudaMemcpy(host, dev, n * sizeof(T), cudaMemcpyDeviceToHost), "download");
}

}  // namespace

namespace ane_lm {

SHIM_API void silu_vec_inplace(float* x, int n, float*) {
    float* d = up(0, x, n);
    check(anelm_silu_vec_inplace(d, n, nullptr), "silu_vec_inplace");
    down(x, d, n);
}

SHIM_API void mul_sigmoid_inplace(float* y, const float* z, int n, float*) {
    float* dy = up(0, y, n);
    const float* dz = up(1, z, n);
    check(anelm_mul_sigmoid_inplace(dy, dz, n, nullptr), "mul_sigmoid_inplace");
    down(y, dy, n);
}

SHIM_API void rmsnorm(float* out, const float* x, const float* weight, int dim, float eps) {
    const float* dx = up(1, x, dim);
    const float* dw = up(2, weight, dim);
    float* dout = up<float>(0, nullptr, dim);
    check(anelm_rmsnorm(dout, dx, dw, dim, eps, 1, nullptr), "rmsnorm");
    down(out, dout, dim);
}

SHIM_API void rmsnorm_gated(float* out, const float* x, const float* z, const float* weight, int dim) {
    const float* dx = up(1, x, dim);
    const float* dz = up(2, z, dim);
    const float* dw = up(3, weight, dim);
    float* dout = up<float>(0, nullptr, dim);
    check(anelm_rmsnorm_gated(dout, dx, dz, dw, dim, 1, nullptr), "rmsnorm_gated");
    down(out, dout, dim);
}

SHIM_API void apply_rope_cached(float* q, float* k, int n_q_heads, int n_kv_heads, int head_dim, int q_head_stride,
                                int k_head_stride, int rot_dim, int pos, float theta, const float* cos_row,
                                const float* sin_row) {
    const size_t nq = (size_t)(n_q_heads - 1) * q_head_stride + head_dim;
    const size_t nk = (size_t)(n_kv_heads - 1) * k_head_stride + head_dim;
    float* dq = up(0, q, nq);
    float* dk = up(1, k, nk);
    const float* dc = cos_row ? up(2, cos_row, (size_t)rot_dim / 2) : nullptr;
    const float* ds = sin_row ? up(3, sin_row, (size_t)rot_dim / 2) : nullptr;
    check(anelm_apply_rope_cached(dq, dk, n_q_heads, n_kv_heads, head_dim, q_head_stride, k_head_stride, rot_dim,
                                  pos, theta, dc, ds, nullptr),
          "apply_rope_cached");
    down(q, dq, nq);
    down(k, dk, nk);
}

SHIM_API void softmax(float* x, int n) {
    float* d = up(0, x, n);
    check(anelm_softmax(d, n, 1, nullptr), "softmax");
    down(x, d, n);
}

SHIM_API void matvec(float* y, const float* W, const float* x, int out_dim, int in_dim) {
    const float* dW = up(1, W, (size_t)out_dim * in_dim);
    const float* dx = up(2, x, in_dim);
    float* dy = up<float>(0, nullptr, out_dim);
    check(anelm_matvec(dy, dW, dx, out_dim, in_dim, nullptr), "matvec");
    down(y, dy, out_dim);
}

SHIM_API void l2_normalize(float* x, int dim) {
    float* d = up(0, x, dim);
    check(anelm_l2_normalize(d, dim, 1, nullptr), "l2_normalize");
    down(x, d, dim);
}

SHIM_API void conv1d_update(float* y, float* conv_state, int* state_pos, const float* x, const float* w,
                            int channels, int kernel_size) {
    const size_t ns = (size_t)channels * (kernel_size - 1);
    float* ds = up(1, conv_state, ns);
    const float* dx = up(2, x, channels);
    const float* dw = up(3, w, (size_t)channels * kernel_size);
    float* dy = up<float>(0, nullptr, channels);
    check(anelm_conv1d_update(dy, ds, state_pos, dx, dw, channels, kernel_size, nullptr), "conv1d_update");
    down(y, dy, channels);
    down(conv_state, ds, ns);
}

SHIM_API void ssm_step(float* y, float* state, const float* q, const float* k, const float* v, float decay, float beta,
                       int key_dim, int value_dim) {
    const size_t ns = (size_t)key_dim * value_dim;
    float* dS = up(1, state, ns);
    const float* dq = up(2, q, key_dim);
    const float* dk = up(3, k, key_dim);
    const float* dv = up(4, v, value_dim);
    float* dy = up<float>(0, nullptr, value_dim);
    check(anelm_ssm_step(dy, dS, dq, dk, dv, decay, beta, key_dim, value_dim, nullptr), "ssm_step");
    down(y, dy, value_dim);
    down(state, dS, ns);
}

SHIM_API void gqa_attention(float* out, const float* q, const float* k_cache, const float* v_cache, int n_heads,
                            int n_kv_heads, int head_dim, int q_head_stride, int cache_start, int cache_len,
                            int cache_capacity) {
    const size_t nq = (size_t)(n_heads - 1) * q_head_stride + head_dim;
    const size_t nkv = (size_t)cache_capacity * n_kv_heads * head_dim;
    const float* dq = up(1, q, nq);
    const float* dk = up(2, k_cache, cache_len > 0 ? nkv : 0);
    const float* dv = up(3, v_cache, cache_len > 0 ? nkv : 0);
    float* dout = up<float>(0, nullptr, (size_t)n_heads * head_dim);
    check(anelm_gqa_attention(dout, dq, dk, dv, ANELM_F32, n_heads, n_kv_heads, head_dim, q_head_stride, cache_start,
                              cache_len, cache_capacity, nullptr),
          "gqa_attention");
    down(out, dout, (size_t)n_heads * head_dim);
}

}  // namespace ane_lm
