// Launchers for the op-level kernels of ops.cu (core/cpu_ops.h mirror).
#pragma once

#include <cuda_runtime.h>

namespace anelm {

constexpr int kMaxLenF32 = 49152;  // fp32-cache gqa_attention: scores kept in shared memory

int op_rmsnorm(float* out, const float* x, const float* w, int dim, float eps, int rows, int gated, const float* z,
               cudaStream_t st);
int op_l2(float* x, int dim, int rows, cudaStream_t st);
int op_softmax(float* x, int n, int rows, cudaStream_t st);
int op_sigmoid_mul(float* y, const float* z, long long n, cudaStream_t st);
int op_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim, cudaStream_t st);
int op_rope(float* q, float* k, int nq, int nkv, int qs, int ks, int rot, int pos, float theta, const float* c,
            const float* s, cudaStream_t st);
int op_conv1d(float* y, float* stt, int pos, const float* x, const float* w, int channels, int K, cudaStream_t st);
int op_ssm_step(float* y, float* S, const float* q, const float* k, const float* v, float decay, float beta, int kd,
                int vd, cudaStream_t st);
int op_gqa_f32(float* out, const float* q, const float* kc, const float* vc, int nh, int nkv, int hd, int qs,
               int start, int len, int cap, cudaStream_t st);

}  // namespace anelm
