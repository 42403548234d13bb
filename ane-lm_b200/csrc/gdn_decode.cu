// Gated DeltaNet decode step (sm_100a).
//
// Replaces, for one token per sequence:
//   forward_deltanet_from_proj  models/llm/qwen3_5.cpp:849-910
//     conv1d_update + silu_vec_inplace  (core/cpu_ops.cpp:89-129, 6-13)
//     l2_normalize of q/k + q scale     (cpu_ops.cpp:82-87, qwen3_5.cpp:879-887)
//     beta / decay gating               (qwen3_5.cpp:897-898)
//     ssm_step                          (cpu_ops.cpp:131-146)
//     rmsnorm_gated                     (cpu_ops.cpp:32-38)
//
// Work decomposition: a thread-block cluster of NSPLIT CTAs per (batch row,
// value head).  The 128x128 fp32 state S[k][v] of the head is split by value
// columns: CTA r of the cluster owns columns [r*W, r*W+W), W = 128/NSPLIT.
// The delta rule is column-separable (each column j needs only k, q, v[j] and
// its own column of S), so each CTA streams its 128 x W block of S from HBM
// into registers exactly once, updates it and writes it back once.  The only
// cross-CTA dependency, the RMS of y over all 128 value columns for the gated
// norm, is exchanged through distributed shared memory (DSMEM) inside the
// cluster.  The S loads are issued before the conv / L2 prologue so HBM latency
// overlaps that work.
//
// Conv state: the reference keeps the last K-1 = 3 inputs per channel in a
// 3-slot ring plus conv_pos (cpu_ops.cpp:89-129).  Every CTA that shares a key
// head must read the same three old q/k inputs while one of them stores the
// new one, so here the ring has 4 slots: input x_t lives in slot t mod 4, the
// three old inputs are slots (n+1..n+3) mod 4 and the new one goes to slot
// n mod 4, which nobody reads in the same step.  The token counter n is kept
// mod 12 (so n mod 3 and n mod 4 are both recoverable); state export/import in
// anelm_abi.cu converts to and from the reference [C][3] + conv_pos layout.
#include <cooperative_groups.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace anelm {

namespace {

constexpr int kThreads = 128;
constexpr int kDk = 128;
constexpr int kDv = 128;

__device__ __forceinline__ float pick4(const float4& v, int k) {
    return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

template <int NSPLIT>
__global__ void __launch_bounds__(kThreads) gdn_decode_kernel(const GdnDecodeParams p) {
    constexpr int W = kDv / NSPLIT;       // value columns per CTA
    constexpr int QPR = W / 4;            // float4 quads per row segment
    constexpr int RPP = kThreads / QPR;   // rows per pass
    constexpr int NR = kDk / RPP;         // rows per thread
    constexpr int NQK = 2 * kDk / NSPLIT; // q/k conv channels whose ring this CTA stores

    __shared__ __align__(16) float q_s[kDk];
    __shared__ __align__(16) float k_s[kDk];
    __shared__ __align__(16) float v_s[W];
    __shared__ __align__(16) float z_s[W];
    __shared__ __align__(16) float y_s[W];
    __shared__ __align__(16) float red[kThreads / 32][W];
    __shared__ float scal[8];
    __shared__ float ss_part;
    __shared__ int s_last;

    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = (int)cluster.block_rank();
    const int hb = blockIdx.x / NSPLIT;
    const int h = hb % p.Hv;
    const int b = hb / p.Hv;
    const int seq = p.seq_ids ? p.seq_ids[b] : p.seq_scalar;
    const int ratio = p.Hv / p.Hk;
    const int kh = h / ratio;             // qwen3_5.cpp:890
    const int C = p.C;
    const int key_total = p.Hk * kDk;
    const int j0 = r * W;

    // ---- issue the state loads first (HBM latency overlaps the prologue) ----
    const int cq = tid % QPR, rg = tid / QPR;
    float* Sbase = p.ssm + (((long long)seq * p.Hv + h) * kDk) * kDv + j0 + 4 * cq;
    float4 S[NR];
#pragma unroll
    for (int i = 0; i < NR; i++) S[i] = __ldcs(reinterpret_cast<const float4*>(Sbase + (long long)(rg + RPP * i) * kDv));

    const char* proj_row = reinterpret_cast<const char*>(p.proj) +
                           (long long)b * p.proj_stride * dtype_bytes(p.proj_dtype);
    const int n = p.conv_cnt[seq];
    const int s_new = n & 3;
    float* conv_seq = p.conv4 + (long long)seq * C * 4;

    // ---- conv1d (K=4) + SiLU for the 256 q/k channels of key head kh and this CTA's W v channels ----
    // core/cpu_ops.cpp:101-110 (y = s0*w0 + s1*w1 + s2*w2 + x*w3) and 6-13 (x / (1 + exp(-x)))
    auto conv_ch = [&](int c, bool store) -> float {
        const float4 ring = *reinterpret_cast<const float4*>(conv_seq + (long long)c * 4);
        const float4 w = *reinterpret_cast<const float4*>(p.conv_w + (long long)c * 4);
        const float x = load_as_float(proj_row, p.proj_dtype, c);
        const float s0 = pick4(ring, (n + 1) & 3), s1 = pick4(ring, (n + 2) & 3), s2 = pick4(ring, (n + 3) & 3);
        float y = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s0, w.x), __fmul_rn(s1, w.y)), __fmul_rn(s2, w.z)),
                            __fmul_rn(x, w.w));
        if (store) conv_seq[(long long)c * 4 + s_new] = x;
        return y / (1.0f + expf(-y));
    };
    const bool qk_owner = (h % ratio) == 0;
    for (int i = tid; i < 2 * kDk; i += kThreads) {
        const int c = (i < kDk) ? kh * kDk + i : key_total + kh * kDk + (i - kDk);
        const bool store = qk_owner && (i / NQK == r);
        const float y = conv_ch(c, store);
        if (i < kDk) q_s[i] = y; else k_s[i - kDk] = y;
    }
    for (int i = tid; i < W; i += kThreads) {
        v_s[i] = conv_ch(2 * key_total + h * kDv + j0 + i, true);
        z_s[i] = load_as_float(proj_row, p.proj_dtype, C + (long long)h * kDv + j0 + i);
    }
    __syncthreads();
    // ---- L2 normalise q and k (warps 0 / 1), then q *= 1/sqrt(dk) ----
    if (warp < 2) {
        float* x = warp == 0 ? q_s : k_s;
        float ss = 0.f;
        for (int i = lane; i < kDk; i += 32) ss += x[i] * x[i];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + p.l2_eps);   // cpu_ops.cpp:85
        const float qscale = 1.0f / sqrtf((float)kDk);   // qwen3_5.cpp:879
        for (int i = lane; i < kDk; i += 32) {
            float v = __fmul_rn(x[i], inv);
            if (warp == 0) v = __fmul_rn(v, qscale);
            x[i] = v;
        }
    } else if (warp == 2 && lane == 0) {
        // gating, qwen3_5.cpp:897-898
        const float a = load_as_float(proj_row, p.proj_dtype, C + (long long)p.Hv * kDv + h);
        const float bb = load_as_float(proj_row, p.proj_dtype, C + (long long)p.Hv * kDv + p.Hv + h);
        scal[0] = sigmoid_ref(bb);
        scal[1] = expf(-p.A[h] * softplus_ref(a + p.dt_bias[h]));
    }
    __syncthreads();
    const float beta = scal[0], decay = scal[1];

    float kr[NR], qr[NR];
#pragma unroll
    for (int i = 0; i < NR; i++) {
        kr[i] = k_s[rg + RPP * i];
        qr[i] = q_s[rg + RPP * i];
    }

    // column reduction over the 128 key rows: within the warp across row groups, then across warps
    auto colsum = [&](float4 v) -> float4 {
#pragma unroll
        for (int o = QPR; o < 32; o <<= 1) {
            v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
            v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
            v.z += __shfl_xor_sync(0xffffffffu, v.z, o);
            v.w += __shfl_xor_sync(0xffffffffu, v.w, o);
        }
        if (lane < QPR) *reinterpret_cast<float4*>(&red[warp][4 * lane]) = v;
        __syncthreads();
        float4 t = *reinterpret_cast<const float4*>(&red[0][4 * cq]);
#pragma unroll
        for (int w = 1; w < kThreads / 32; w++) {
            const float4 u = *reinterpret_cast<const float4*>(&red[w][4 * cq]);
            t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
        }
        __syncthreads();
        return t;
    };

    float4 delta;
    if (p.delta_mode == ANELM_DELTA_CPUOPS) {
        // cpu_ops.cpp:134-142: Sk = S^T k (undecayed), delta = v - Sk, S = decay*S + beta*k*delta^T
        float4 sk = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            sk.x += S[i].x * kr[i]; sk.y += S[i].y * kr[i]; sk.z += S[i].z * kr[i]; sk.w += S[i].w * kr[i];
        }
        sk = colsum(sk);
        const float* vv = &v_s[4 * cq];
        delta = make_float4(vv[0] - sk.x, vv[1] - sk.y, vv[2] - sk.z, vv[3] - sk.w);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            const float ax = beta * kr[i];
            S[i].x = __fadd_rn(__fmul_rn(S[i].x, decay), __fmul_rn(ax, delta.x));
            S[i].y = __fadd_rn(__fmul_rn(S[i].y, decay), __fmul_rn(ax, delta.y));
            S[i].z = __fadd_rn(__fmul_rn(S[i].z, decay), __fmul_rn(ax, delta.z));
            S[i].w = __fadd_rn(__fmul_rn(S[i].w, decay), __fmul_rn(ax, delta.w));
        }
    } else {
        // export_hybrid_chunks.py:142-147: S = g*S; Sk = S^T k; delta = (v - Sk)*beta; S += k delta^T
#pragma unroll
        for (int i = 0; i < NR; i++) {
            S[i].x = __fmul_rn(S[i].x, decay); S[i].y = __fmul_rn(S[i].y, decay);
            S[i].z = __fmul_rn(S[i].z, decay); S[i].w = __fmul_rn(S[i].w, decay);
        }
        float4 sk = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            sk.x += S[i].x * kr[i]; sk.y += S[i].y * kr[i]; sk.z += S[i].z * kr[i]; sk.w += S[i].w * kr[i];
        }
        sk = colsum(sk);
        const float* vv = &v_s[4 * cq];
        delta = make_float4((vv[0] - sk.x) * beta, (vv[1] - sk.y) * beta, (vv[2] - sk.z) * beta,
                            (vv[3] - sk.w) * beta);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            S[i].x = __fadd_rn(S[i].x, __fmul_rn(kr[i], delta.x));
            S[i].y = __fadd_rn(S[i].y, __fmul_rn(kr[i], delta.y));
            S[i].z = __fadd_rn(S[i].z, __fmul_rn(kr[i], delta.z));
            S[i].w = __fadd_rn(S[i].w, __fmul_rn(kr[i], delta.w));
        }
    }
    // y = S^T q (cpu_ops.cpp:144-145), and write S back
    float4 yv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NR; i++) {
        yv.x += S[i].x * qr[i]; yv.y += S[i].y * qr[i]; yv.z += S[i].z * qr[i]; yv.w += S[i].w * qr[i];
        __stcs(reinterpret_cast<float4*>(Sbase + (long long)(rg + RPP * i) * kDv), S[i]);
    }
    yv = colsum(yv);
    if (rg == 0) *reinterpret_cast<float4*>(&y_s[4 * cq]) = yv;
    __syncthreads();

    // ---- gated RMSNorm over all 128 value columns (cluster-wide sum of y^2) ----
    if (warp == 0) {
        float ss = 0.f;
        for (int i = lane; i < W; i += 32) ss += y_s[i] * y_s[i];
        ss = warp_sum(ss);
        if (lane == 0) ss_part = ss;
    }
    cluster.sync();
    if (tid == 0) {
        float tot = 0.f;
        for (int q = 0; q < NSPLIT; q++) tot += *cluster.map_shared_rank(&ss_part, q);
        scal[2] = 1.0f / sqrtf(tot / (float)kDv + 1e-6f);  // rmsnorm eps 1e-6, cpu_ops.cpp:34
    }
    cluster.sync();  // peers have read ss_part; safe to exit afterwards
    const float rinv = scal[2];
    const long long orow = (long long)b * p.out_stride + (long long)h * kDv + j0;
    for (int i = tid; i < W; i += kThreads) {
        const float z = z_s[i];
        float o = __fmul_rn(__fmul_rn(y_s[i], rinv), p.norm_w[j0 + i]);
        o = o / (1.0f + expf(-z));
        o = __fmul_rn(o, z);
        store_from_float(p.out, p.out_dtype, orow + i, o);
    }

    // ---- the last CTA of this row advances the conv ring counter ----
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(&p.cnt_seq[b], 1);
        s_last = (prev == p.Hv * NSPLIT - 1);
    }
    __syncthreads();
    if (s_last && tid == 0) {
        p.conv_cnt[seq] = (n + 1) % 12;
        p.cnt_seq[b] = 0;
    }
}

template <int NSPLIT>
int launch(const GdnDecodeParams& p, int n_rows, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n_rows * p.Hv * NSPLIT));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = NSPLIT;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_decode_kernel<NSPLIT>, p);
    return e == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

}  // namespace

int launch_gdn_decode(const GdnDecodeParams& p, int n_rows, int key_dim, int val_dim, cudaStream_t stream) {
    if (key_dim != kDk || val_dim != kDv) return ANELM_ERR_UNSUPPORTED;
    // Small batches: 8 CTAs per head to fill the 148 SMs; large batches: 4 (less redundant q/k work).
    if ((long long)n_rows * p.Hv * 4 < 2 * 148) return launch<8>(p, n_rows, stream);
    return launch<4>(p, n_rows, stream);
}

}  // namespace anelm
