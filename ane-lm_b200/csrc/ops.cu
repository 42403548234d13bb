// Op-level kernels: one per core/cpu_ops.h entry point, on device fp32 buffers.
//
// These mirror the reference's individual ops (core/cpu_ops.cpp) for callers
// that link against the cpu_ops.h interface op by op.  The fused layer kernels
// (fa_decode.cu, gdn_decode.cu) are the fast path; these are sized for
// correctness and modest speed.
#include <math.h>

#include "common.cuh"
#include "ops.h"

namespace anelm {

namespace {

__device__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    const int nw = (blockDim.x + 31) >> 5;
    for (int w = 0; w < nw; w++) t += red[w];
    return t;
}

__device__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    const int nw = (blockDim.x + 31) >> 5;
    for (int w = 0; w < nw; w++) t = fmaxf(t, red[w]);
    return t;
}

// rmsnorm, cpu_ops.cpp:24-30 (one block per row)
__global__ void rmsnorm_kernel(float* out, const float* x, const float* w, int dim, float eps, int gated,
                               const float* z) {
    __shared__ float red[32];
    const float* xr = x + (long long)blockIdx.x * dim;
    float* orow = out + (long long)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)dim + eps);
    const float* zr = gated ? z + (long long)blockIdx.x * dim : nullptr;
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float o = __fmul_rn(__fmul_rn(xr[i], r), w[i]);
        if (gated) {  // rmsnorm_gated, cpu_ops.cpp:32-38
            o = o / (1.0f + expf(-zr[i]));
            o = __fmul_rn(o, zr[i]);
        }
        orow[i] = o;
    }
}

// l2_normalize, cpu_ops.cpp:82-87
__global__ void l2_kernel(float* x, int dim) {
    __shared__ float red[32];
    float* xr = x + (long long)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss + 1e-12f);
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = __fmul_rn(xr[i], inv);
}

// softmax, cpu_ops.cpp:65-75
__global__ void softmax_kernel(float* x, int n) {
    __shared__ float red[32];
    float* xr = x + (long long)blockIdx.x * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, xr[i]);
    m = block_max(m, red);
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(xr[i] - m);
        xr[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xr[i] = __fmul_rn(xr[i], inv);
}

// silu_vec_inplace (z == nullptr) / mul_sigmoid_inplace, cpu_ops.cpp:6-22
__global__ void sigmoid_mul_kernel(float* y, const float* z, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float g = z ? z[i] : y[i];
        y[i] = y[i] / (1.0f + expf(-g));
    }
}

// matvec, cpu_ops.cpp:77-80 (one warp per output row)
__global__ void matvec_kernel(float* y, const float* W, const float* x, int out_dim, int in_dim) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= out_dim) return;
    const float* wr = W + (long long)row * in_dim;
    float s = 0.f;
    for (int i = lane; i < in_dim; i += 32) s += wr[i] * x[i];
    s = warp_sum(s);
    if (lane == 0) y[row] = s;
}

// apply_rope_cached, cpu_ops.cpp:40-63 (one thread per rotated pair)
__global__ void rope_kernel(float* q, float* k, int nq, int nkv, int qs, int ks, int rot, int pos, float theta,
                            const float* cos_row, const float* sin_row) {
    const int half = rot >> 1;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (nq + nkv) * half) return;
    const int h = idx / half, j = idx - h * half;
    float* v = h < nq ? q + (long long)h * qs : k + (long long)(h - nq) * ks;
    float c, s;
    if (cos_row && sin_row) {
        c = cos_row[j];
        s = sin_row[j];
    } else {
        const float freq = 1.0f / powf(theta, (float)(2 * j) / (float)rot);
        const float angle = (float)pos * freq;
        c = cosf(angle);
        s = sinf(angle);
    }
    const float v0 = v[2 * j], v1 = v[2 * j + 1];
    v[2 * j] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    v[2 * j + 1] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
}

// conv1d_update, cpu_ops.cpp:89-129 (reference ring layout [C][K-1], position passed in)
__global__ void conv1d_kernel(float* y, float* st, int pos, const float* x, const float* w, int channels, int K) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    const int sl = K - 1;
    float sum;
    if (K == 4) {
        int p1 = pos + 1;
        if (p1 == 3) p1 = 0;
        int p2 = p1 + 1;
        if (p2 == 3) p2 = 0;
        const float s0 = st[c * 3 + pos], s1 = st[c * 3 + p1], s2 = st[c * 3 + p2];
        sum = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s0, w[c * 4]), __fmul_rn(s1, w[c * 4 + 1])),
                                  __fmul_rn(s2, w[c * 4 + 2])),
                        __fmul_rn(x[c], w[c * 4 + 3]));
    } else {
        float acc = 0.f;
        for (int j = 0; j < sl; j++) {
            int idx = pos + j;
            if (idx >= sl) idx -= sl;
            acc = __fadd_rn(acc, __fmul_rn(st[c * sl + idx], w[c * K + j]));
        }
        sum = __fadd_rn(acc, __fmul_rn(x[c], w[c * K + sl]));
    }
    y[c] = sum;
    st[c * sl + pos] = x[c];
}

// ssm_step, cpu_ops.cpp:131-146 (one thread per value column; coalesced across j)
__global__ void ssm_step_kernel(float* y, float* S, const float* q, const float* k, const float* v, float decay,
                                float beta, int kd, int vd) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= vd) return;
    float sk = 0.f;
    for (int i = 0; i < kd; i++) sk += S[(long long)i * vd + j] * k[i];
    const float delta = v[j] - sk;
    float yy = 0.f;
    for (int i = 0; i < kd; i++) {
        float s = S[(long long)i * vd + j];
        s = __fadd_rn(__fmul_rn(s, decay), __fmul_rn(beta * k[i], delta));
        S[(long long)i * vd + j] = s;
        yy += s * q[i];
    }
    y[j] = yy;
}

// gqa_attention over an fp32 ring, cpu_ops.cpp:148-204: one block per query head,
// scores in shared memory (len <= kMaxLenF32).
__global__ void gqa_f32_kernel(float* out, const float* q, const float* kc, const float* vc, int nh, int nkv,
                               int hd, int qs, int start, int len, int cap) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    const int h = blockIdx.x;
    const int kvh = h / (nh / nkv);
    const float* qh = q + (long long)h * qs;
    const float scale = 1.0f / sqrtf((float)hd);
    int first = cap - start;
    if (first > len) first = len;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int t = warp; t < len; t += nw) {
        const long long slot = t < first ? (long long)start + t : (long long)(t - first);
        const float* kr = kc + (slot * nkv + kvh) * hd;
        float d = 0.f;
        for (int i = lane; i < hd; i += 32) d += qh[i] * kr[i];
        d = warp_sum(d);
        if (lane == 0) sc[t] = d * scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = threadIdx.x; t < len; t += blockDim.x) m = fmaxf(m, sc[t]);
    m = block_max(m, red);
    float s = 0.f;
    for (int t = threadIdx.x; t < len; t += blockDim.x) {
        const float e = expf(sc[t] - m);
        sc[t] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float o = 0.f;
        for (int t = 0; t < len; t++) {
            const long long slot = t < first ? (long long)start + t : (long long)(t - first);
            o += (sc[t] * inv) * vc[(slot * nkv + kvh) * hd + i];
        }
        out[(long long)h * hd + i] = o;
    }
}

}  // namespace

int op_rmsnorm(float* out, const float* x, const float* w, int dim, float eps, int rows, int gated, const float* z,
               cudaStream_t st) {
    rmsnorm_kernel<<<rows, 256, 0, st>>>(out, x, w, dim, eps, gated, z);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_l2(float* x, int dim, int rows, cudaStream_t st) {
    l2_kernel<<<rows, 128, 0, st>>>(x, dim);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_softmax(float* x, int n, int rows, cudaStream_t st) {
    softmax_kernel<<<rows, 256, 0, st>>>(x, n);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_sigmoid_mul(float* y, const float* z, long long n, cudaStream_t st) {
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    sigmoid_mul_kernel<<<(unsigned)blocks, 256, 0, st>>>(y, z, n);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim, cudaStream_t st) {
    matvec_kernel<<<(out_dim + 7) / 8, 256, 0, st>>>(y, W, x, out_dim, in_dim);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_rope(float* q, float* k, int nq, int nkv, int qs, int ks, int rot, int pos, float theta, const float* c,
            const float* s, cudaStream_t st) {
    const int n = (nq + nkv) * (rot / 2);
    if (n == 0) return 0;
    rope_kernel<<<(n + 127) / 128, 128, 0, st>>>(q, k, nq, nkv, qs, ks, rot, pos, theta, c, s);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_conv1d(float* y, float* stt, int pos, const float* x, const float* w, int channels, int K, cudaStream_t st) {
    conv1d_kernel<<<(channels + 127) / 128, 128, 0, st>>>(y, stt, pos, x, w, channels, K);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_ssm_step(float* y, float* S, const float* q, const float* k, const float* v, float decay, float beta, int kd,
                int vd, cudaStream_t st) {
    ssm_step_kernel<<<(vd + 127) / 128, 128, 0, st>>>(y, S, q, k, v, decay, beta, kd, vd);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}
int op_gqa_f32(float* out, const float* q, const float* kc, const float* vc, int nh, int nkv, int hd, int qs,
               int start, int len, int cap, cudaStream_t st) {
    const size_t sm = (size_t)len * sizeof(float);
    cudaFuncSetAttribute(gqa_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxLenF32 * 4);
    gqa_f32_kernel<<<nh, 256, sm, st>>>(out, q, kc, vc, nh, nkv, hd, qs, start, len, cap);
    return cudaGetLastError() == cudaSuccess ? 0 : ANELM_ERR_CUDA;
}

}  // namespace anelm
