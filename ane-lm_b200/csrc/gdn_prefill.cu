// Chunkwise Gated DeltaNet prefill (sm_100a).
//
// Replaces the per-token prefill loop of the reference for the linear-attention layers
// (qwen3_5.cpp:1205-1217 calling forward_deltanet_from_proj, qwen3_5.cpp:849-909, once per
// prompt token; serve_hybrid.py runs the same recurrence inside its CoreML chunks).  Per token:
// conv1d_update over the q|k|v channels (cpu_ops.cpp:89-129), SiLU, per-head L2 norm of q and k,
// q *= 1/sqrt(dk), beta = sigmoid(b), g = exp(-A softplus(a + dt_bias)), one delta-rule step
// (cpu_ops.cpp:131-146, or the decay-first order of export_hybrid_chunks.py:142-147), and the
// gated RMSNorm of the output (cpu_ops.cpp:32-38).
//
// The recurrence over a chunk of C = 64 tokens is solved in closed form.  Both orders are
//     S_t = (g_t I - b_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T,    y_t = S_t^T q_t
// with b_t = beta_t (cpu_ops: Sk from the undecayed state) or g_t beta_t (decay first).  With
// the in-chunk cumulative log decay lc_t = sum_{i<=t} log g_i and lt_t = lc_{t-1} (cpu_ops) or
// lc_t (decay first), the corrected values D (rows delta_t) of a chunk starting from state S0 are
//     (I + A) D = diag(beta) V - diag(beta e^{lt}) K S0,    A_ti = beta_t e^{lt_t - lc_i} k_t.k_i  (i < t)
// so with T = (I + A)^{-1}:  D = U - W S0,  U = T diag(beta) V,  W = T diag(beta e^{lt}) K, and
//     Y   = diag(e^{lc}) Q S0 + M D,           M_ti = e^{lc_t - lc_i} q_t.k_i  (i <= t)
//     S_C = e^{lc_C} S0 + K^T diag(e^{lc_C - lc}) D.
// Only ratios of decays appear (no 1/g), so small g is harmless.  The columns of S are
// independent, so the sequential part runs one chain per (sequence, value head, 32 state columns).
//
// Launches:
//   gdn_pf_snapshot_kernel  copy of the conv rings / positions of the plan's sequences (the
//                           prep kernel reads the old ring while the last tokens overwrite it)
//   gdn_pf_prep_kernel      per token: conv + SiLU + L2 / scale, gates; q, k, v in chunk
//                           layout, log g and beta; the last 3 inputs into the ring, new position
//   gdn_pf_pack_kernel      (core op only) token-major q, k, v, log g, beta -> chunk layout
//   gdn_pf_chunk_kernel     per (chunk, value head): K K^T, Q K^T, T by forward substitution,
//                           W, U, M
//   gdn_pf_chain_kernel     per (sequence, value head, 32 columns): the chunk recurrence over
//                           the state block; each operand buffer is refilled with the next
//                           chunk's data (cp.async) as soon as this chunk's last reader is done
//   gdn_pf_out_kernel       gated RMSNorm of y with z (layer path)
// Products run on the tensor cores (mma.sync m16n8k16) with every operand split into an fp16
// hi + lo pair (three MMAs per product), so they carry ~2^-22 relative error like the fp32
// reference arithmetic; operands are kept in fp32 in memory.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace anelm {

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kDk = 128;   // key head dim of these kernels
constexpr int kDv = 128;   // value head dim
constexpr int kDvb = 32;   // state columns per chain CTA
constexpr int kLd = kDk + 4;  // fp32 row pitch of the 64 x 128 tiles in shared memory (bank spread)

// ---------------------------------------------------------------- mma.sync fragments
// m16n8k16, fp16 operands, fp32 accumulate.  g = lane / 4, c = lane % 4:
//   A (16 x 16, row):  a0 = A[g][2c..2c+1], a1 = A[g+8][2c..], a2 = A[g][2c+8..], a3 = A[g+8][2c+8..]
//   B (16 x 8, col):   b0 = B[2c..2c+1][g], b1 = B[2c+8..2c+9][g]
//   C (16 x 8):        c0 = C[g][2c], c1 = C[g][2c+1], c2 = C[g+8][2c], c3 = C[g+8][2c+1]
__device__ __forceinline__ uint32_t h2(float lo, float hi) {
    const __half2 t = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&t);
}
// fp32 pair -> (hi, lo) fp16 pairs with hi + lo = x to ~2^-22 relative
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
    hi = pack_half2(h0, h1);
    lo = h2(x0 - __half2float(h0), x1 - __half2float(h1));
}

// acc[MT][NT] += A[r0 .. r0 + 16 MT) x B[.. , n0 .. n0 + 8 NT) over k in [0, K).
// fa(r, k), fb(k, n) return fp32 values; SA / SB: split that operand into hi + lo fp16 parts
// (two extra MMAs per step: hi*hi + lo*hi + hi*lo).
template <bool SA, bool SB, int MT, int NT, class FA, class FB>
__device__ __forceinline__ void warp_gemm(float (&acc)[MT][NT][4], int r0, int n0, int K, int lane, FA fa, FB fb) {
    const int g = lane >> 2, c = lane & 3;
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t ah[MT][4], al[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            const int r = r0 + mt * 16 + g;
            const int k = k0 + 2 * c;
            if (SA) {
                split2(fa(r, k), fa(r, k + 1), ah[mt][0], al[mt][0]);
                split2(fa(r + 8, k), fa(r + 8, k + 1), ah[mt][1], al[mt][1]);
                split2(fa(r, k + 8), fa(r, k + 9), ah[mt][2], al[mt][2]);
                split2(fa(r + 8, k + 8), fa(r + 8, k + 9), ah[mt][3], al[mt][3]);
            } else {
                ah[mt][0] = h2(fa(r, k), fa(r, k + 1));
                ah[mt][1] = h2(fa(r + 8, k), fa(r + 8, k + 1));
                ah[mt][2] = h2(fa(r, k + 8), fa(r, k + 9));
                ah[mt][3] = h2(fa(r + 8, k + 8), fa(r + 8, k + 9));
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int n = n0 + nt * 8 + g;
            const int k = k0 + 2 * c;
            uint32_t bh0, bh1, bl0 = 0, bl1 = 0;
            if (SB) {
                split2(fb(k, n), fb(k + 1, n), bh0, bl0);
                split2(fb(k + 8, n), fb(k + 9, n), bh1, bl1);
            } else {
                bh0 = h2(fb(k, n), fb(k + 1, n));
                bh1 = h2(fb(k + 8, n), fb(k + 9, n));
            }
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                mma_16816(acc[mt][nt], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], bh0, bh1);
                if (SA) mma_16816(acc[mt][nt], al[mt][0], al[mt][1], al[mt][2], al[mt][3], bh0, bh1);
                if (SB) mma_16816(acc[mt][nt], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], bl0, bl1);
            }
        }
    }
}

// ---------------------------------------------------------------- snapshot

__global__ void gdn_pf_snapshot_kernel(const GdnPrefillParams p) {
    const int b = blockIdx.y;
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    const long long nring = (long long)p.C * 3;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nring; i += (long long)gridDim.x * blockDim.x)
        p.ring_snap[b * nring + i] = p.conv[seq * nring + i];
    if (blockIdx.x == 0 && threadIdx.x < p.Hk) p.pos_snap[b * p.Hk + threadIdx.x] = p.conv_pos[seq * p.Hk + threadIdx.x];
}

// ---------------------------------------------------------------- prep (one CTA per token)

__global__ void __launch_bounds__(256) gdn_pf_prep_kernel(const GdnPrefillParams p) {
    extern __shared__ float ys[];  // [C] conv + SiLU outputs of this token
    const int t = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Hk = p.Hk, Hv = p.Hv, C = p.C;
    const int key_total = Hk * kDk;
    const int ratio = Hv / Hk;
    const long long qrow = ((long long)b * Hk) * p.T_pad + t;  // + kh * T_pad
    const long long vrow = ((long long)b * Hv) * p.T_pad + t;
    if (t >= p.n) {  // padding tokens of the last chunk: no effect on the state (beta = 0, g = 1, k = v = 0)
        for (int i = tid; i < Hk * kDk; i += 256) {
            const long long o = (qrow + (long long)(i / kDk) * p.T_pad) * kDk + i % kDk;
            p.qb[o] = 0.f;
            p.kb[o] = 0.f;
        }
        for (int i = tid; i < Hv * kDv; i += 256) p.vb[(vrow + (long long)(i / kDv) * p.T_pad) * kDv + i % kDv] = 0.f;
        for (int h = tid; h < Hv; h += 256) {
            p.lg[vrow + (long long)h * p.T_pad] = 0.f;
            p.beta[vrow + (long long)h * p.T_pad] = 0.f;
        }
        return;
    }
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    const long long rb = (long long)p.proj_stride * dtype_bytes(p.proj_dtype);
    const char* base = reinterpret_cast<const char*>(p.proj) + (long long)b * p.n * rb;
    const float* snap = p.ring_snap + (long long)b * C * 3;
    float* ring = p.conv + (long long)seq * C * 3;
    // conv1d_update (cpu_ops.cpp:95-110) + SiLU (cpu_ops.cpp:6-13) over the sequence: inputs
    // before the first token come from the ring (slot (pos0 + tau + 3) % 3 holds input tau < 0)
    for (int c = tid; c < C; c += 256) {
        const int kh = c < key_total ? c / kDk : c < 2 * key_total ? (c - key_total) / kDk
                                                                   : (c - 2 * key_total) / kDv / ratio;
        const int pos0 = p.pos_snap[b * Hk + kh];
        float s[3];
#pragma unroll
        for (int m = 0; m < 3; m++) {
            const int tau = t - 3 + m;
            s[m] = tau >= 0 ? load_as_float(base + tau * rb, p.proj_dtype, c) : snap[c * 3 + (pos0 + tau + 3) % 3];
        }
        const float x = load_as_float(base + t * rb, p.proj_dtype, c);
        const float4 w = *reinterpret_cast<const float4*>(p.conv_w + (long long)c * 4);
        const float y = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s[0], w.x), __fmul_rn(s[1], w.y)), __fmul_rn(s[2], w.z)),
                                  __fmul_rn(x, w.w));
        ys[c] = y / (1.0f + expf(-y));
        if (t >= p.n - 3) ring[c * 3 + (pos0 + t) % 3] = x;  // cpu_ops.cpp:109: the last 3 inputs stay
    }
    if (t == 0 && tid < Hk) p.conv_pos[seq * Hk + tid] = (p.pos_snap[b * Hk + tid] + p.n) % 3;
    if (tid < Hv) {
        const int h = tid;
        const float a = load_as_float(base + t * rb, p.proj_dtype, C + (long long)Hv * kDv + h);
        const float bb = load_as_float(base + t * rb, p.proj_dtype, C + (long long)Hv * kDv + Hv + h);
        p.beta[vrow + (long long)h * p.T_pad] = sigmoid_ref(bb);                      // qwen3_5.cpp:897
        p.lg[vrow + (long long)h * p.T_pad] = -p.A[h] * softplus_ref(a + p.dt_bias[h]);  // log of qwen3_5.cpp:898
    }
    __syncthreads();
    // L2-normalise q and k per key head (cpu_ops.cpp:82-87), q *= 1/sqrt(dk) (qwen3_5.cpp:879-887)
    const float qscale = 1.0f / sqrtf((float)kDk);
    for (int sgm = warp; sgm < 2 * Hk; sgm += 8) {
        const bool isq = sgm < Hk;
        const int kh = isq ? sgm : sgm - Hk;
        const float* x = ys + (isq ? 0 : key_total) + kh * kDk;
        float ss = 0.f;
        for (int i = lane; i < kDk; i += 32) ss += x[i] * x[i];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + p.l2_eps);
        float* dst = (isq ? p.qb : p.kb) + (qrow + (long long)kh * p.T_pad) * kDk;
        for (int i = lane; i < kDk; i += 32) {
            float v = __fmul_rn(x[i], inv);
            if (isq) v = __fmul_rn(v, qscale);
            dst[i] = v;
        }
    }
    for (int i = tid; i < Hv * kDv; i += 256) p.vb[(vrow + (long long)(i / kDv) * p.T_pad) * kDv + i % kDv] = ys[2 * key_total + i];
}

// ---------------------------------------------------------------- pack (core op: token-major inputs)

__global__ void __launch_bounds__(256) gdn_pf_pack_kernel(const GdnPrefillParams p) {
    const int t = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int Hk = p.Hk, Hv = p.Hv;
    const bool live = t < p.n;
    const long long tok = (long long)b * p.n + t;
    for (int i = tid; i < Hk * kDk; i += 256) {
        const long long o = (((long long)b * Hk + i / kDk) * p.T_pad + t) * kDk + i % kDk;
        p.qb[o] = live ? load_as_float(p.q_in, p.in_dtype, tok * Hk * kDk + i) : 0.f;
        p.kb[o] = live ? load_as_float(p.k_in, p.in_dtype, tok * Hk * kDk + i) : 0.f;
    }
    for (int i = tid; i < Hv * kDv; i += 256) {
        const long long o = (((long long)b * Hv + i / kDv) * p.T_pad + t) * kDv + i % kDv;
        p.vb[o] = live ? load_as_float(p.v_in, p.in_dtype, tok * Hv * kDv + i) : 0.f;
    }
    for (int h = tid; h < Hv; h += 256) {
        const long long o = ((long long)b * Hv + h) * p.T_pad + t;
        p.lg[o] = live ? p.lg_in[tok * Hv + h] : 0.f;
        p.beta[o] = live ? p.beta_in[tok * Hv + h] : 0.f;
    }
}

// ---------------------------------------------------------------- per-chunk quantities

struct ChunkSmem {
    float k[kC][kLd];
    float qv[kC][kLd];        // Q, then V
    float a[kC][kC + 1];      // A, then T = (I + A)^{-1} in place
    float lc[kC], lt[kC], bt[kC];
};

__device__ __forceinline__ void load_tile(float (*dst)[kLd], const float* src, int tid) {
    for (int i = tid; i < kC * (kDk / 4); i += 256) {
        const int r = i / (kDk / 4), cv = i % (kDk / 4);
        *reinterpret_cast<float4*>(&dst[r][cv * 4]) = *reinterpret_cast<const float4*>(src + (long long)r * kDk + cv * 4);
    }
}

__global__ void __launch_bounds__(256) gdn_pf_chunk_kernel(const GdnPrefillParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(smem_raw);
    const int ci = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int kh = h / (p.Hv / p.Hk);
    const int t0 = ci * kC;
    const long long krow = ((long long)b * p.Hk + kh) * p.T_pad + t0;
    const long long vrow = ((long long)b * p.Hv + h) * p.T_pad + t0;
    load_tile(sm.k, p.kb + krow * kDk, tid);
    load_tile(sm.qv, p.qb + krow * kDk, tid);
    if (warp == 0) {  // inclusive prefix sum of log g over the chunk (two tokens per lane)
        const float g0 = p.lg[vrow + 2 * lane], g1 = p.lg[vrow + 2 * lane + 1];
        float s = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        const float excl = s - (g0 + g1);
        sm.lc[2 * lane] = excl + g0;
        sm.lc[2 * lane + 1] = s;
        // lt = lc_{t-1} (Sk from the undecayed state) or lc_t (decay first)
        sm.lt[2 * lane] = p.delta_mode == ANELM_DELTA_CPUOPS ? excl : excl + g0;
        sm.lt[2 * lane + 1] = p.delta_mode == ANELM_DELTA_CPUOPS ? excl + g0 : s;
        sm.bt[2 * lane] = p.beta[vrow + 2 * lane];
        sm.bt[2 * lane + 1] = p.beta[vrow + 2 * lane + 1];
    }
    __syncthreads();
    // K K^T -> A (strictly lower), Q K^T -> M (lower incl. diagonal): warp -> 16 rows x 32 columns
    {
        const int r0 = 16 * (warp & 3), n0 = 32 * (warp >> 2);
        float kk[1][4][4] = {}, qk[1][4][4] = {};
        warp_gemm<true, true, 1, 4>(kk, r0, n0, kDk, lane, [&](int r, int k) { return sm.k[r][k]; },
                                    [&](int k, int n) { return sm.k[n][k]; });
        warp_gemm<true, true, 1, 4>(qk, r0, n0, kDk, lane, [&](int r, int k) { return sm.qv[r][k]; },
                                    [&](int k, int n) { return sm.k[n][k]; });
        float* mrow = p.Mb + vrow * kC;
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int r = r0 + g + (e >> 1) * 8, i = n0 + nt * 8 + 2 * c + (e & 1);
                sm.a[r][i] = i < r ? sm.bt[r] * expf(sm.lt[r] - sm.lc[i]) * kk[0][nt][e] : 0.f;
                mrow[r * kC + i] = i <= r ? expf(sm.lc[r] - sm.lc[i]) * qk[0][nt][e] : 0.f;
            }
    }
    if (tid < kC) p.lcb[vrow + tid] = sm.lc[tid];
    __syncthreads();  // Q no longer needed
    load_tile(sm.qv, p.vb + vrow * kDv, tid);
    // T = (I + A)^{-1} by forward substitution, one column per 4 threads: x_t = [t == j] - sum_{i<t} A_ti x_i.
    // Thread part pt keeps x_i for i = 4m + pt in registers; each row's sum is reduced over the 4 threads.
    {
        const int j = tid >> 2, pt = tid & 3;
        float xs[kC / 4];
#pragma unroll
        for (int m = 0; m < kC / 4; m++) xs[m] = 0.f;
#pragma unroll
        for (int t = 0; t < kC; t++) {
            float s = 0.f;
#pragma unroll
            for (int m = 0; m < kC / 4; m++)
                if (4 * m + pt < t) s = fmaf(sm.a[t][4 * m + pt], xs[m], s);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            const float x = (t == j ? 1.0f : 0.0f) - s;
            if (pt == (t & 3)) xs[t >> 2] = x;
        }
        __syncthreads();  // every thread has read A (and V has landed)
#pragma unroll
        for (int m = 0; m < kC / 4; m++) sm.a[4 * m + pt][j] = xs[m];
    }
    __syncthreads();
    // W = T diag(beta e^{lt}) K,  U = T diag(beta) V: warp -> 16 rows x 64 columns
    {
        const int r0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
        float w[1][8][4] = {}, u[1][8][4] = {};
        warp_gemm<true, true, 1, 8>(w, r0, n0, kC, lane, [&](int r, int k) { return sm.a[r][k] * sm.bt[k] * expf(sm.lt[k]); },
                                    [&](int k, int n) { return sm.k[k][n]; });
        warp_gemm<true, true, 1, 8>(u, r0, n0, kC, lane, [&](int r, int k) { return sm.a[r][k] * sm.bt[k]; },
                                    [&](int k, int n) { return sm.qv[k][n]; });
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const int r = r0 + g + (e >> 1) * 8, n = n0 + nt * 8 + 2 * c;
                *reinterpret_cast<float2*>(p.Wb + (vrow + r) * kDk + n) = make_float2(w[0][nt][e], w[0][nt][e + 1]);
                *reinterpret_cast<float2*>(p.Ub + (vrow + r) * kDv + n) = make_float2(u[0][nt][e], u[0][nt][e + 1]);
            }
    }
}

// ---------------------------------------------------------------- the recurrence over chunks

struct ChainSmem {
    float w[kC][kLd], q[kC][kLd], k[kC][kLd];  // this chunk's W, Q, K
    float u[kC][kDvb + 4];                     // U columns of this block
    float m[kC][kC + 4];                       // M
    float lc[2][kC];                           // in-chunk cumulative log decay, by chunk parity
    float s[kDk][kDvb + 1];                    // state block (fp32 master)
    float d[kC][kDvb + 1];                     // corrected values D of the chunk
};

// cp.async of this chunk's W, Q, U columns and lc (read by the [W; Q] S product and D = U - W S)
__device__ __forceinline__ void chain_load_wqu(ChainSmem& sm, const GdnPrefillParams& p, long long krow, long long vrow,
                                               int j0, int par, int tid) {
    for (int i = tid; i < kC * (kDk / 4); i += 256) {
        const int r = i / (kDk / 4), cv = i % (kDk / 4);
        cp_async_16(smem_u32(&sm.w[r][cv * 4]), p.Wb + (vrow + r) * kDk + cv * 4, 16);
        cp_async_16(smem_u32(&sm.q[r][cv * 4]), p.qb + (krow + r) * kDk + cv * 4, 16);
    }
    for (int i = tid; i < kC * (kDvb / 4); i += 256) {
        const int r = i / (kDvb / 4), cv = i % (kDvb / 4);
        cp_async_16(smem_u32(&sm.u[r][cv * 4]), p.Ub + (vrow + r) * kDv + j0 + cv * 4, 16);
    }
    if (tid < kC / 4) cp_async_16(smem_u32(&sm.lc[par][tid * 4]), p.lcb + vrow + tid * 4, 16);
    cp_async_commit();
}
// cp.async of this chunk's M and K (read by Y = ... + M D and the state update)
__device__ __forceinline__ void chain_load_mk(ChainSmem& sm, const GdnPrefillParams& p, long long krow, long long vrow,
                                              int tid) {
    for (int i = tid; i < kC * (kDk / 4); i += 256) {
        const int r = i / (kDk / 4), cv = i % (kDk / 4);
        cp_async_16(smem_u32(&sm.k[r][cv * 4]), p.kb + (krow + r) * kDk + cv * 4, 16);
    }
    for (int i = tid; i < kC * (kC / 4); i += 256) {
        const int r = i / (kC / 4), cv = i % (kC / 4);
        cp_async_16(smem_u32(&sm.m[r][cv * 4]), p.Mb + (vrow + r) * kC + cv * 4, 16);
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(256) gdn_pf_chain_kernel(const GdnPrefillParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChainSmem& sm = *reinterpret_cast<ChainSmem*>(smem_raw);
    const int nblk = kDv / kDvb;
    const int h = blockIdx.x / nblk, j0 = (blockIdx.x % nblk) * kDvb, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int kh = h / (p.Hv / p.Hk);
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    float* S = p.state + ((long long)seq * p.Hv + h) * kDk * kDv;
    for (int i = tid; i < kDk * kDvb; i += 256) sm.s[i / kDvb][i % kDvb] = S[(long long)(i / kDvb) * kDv + j0 + i % kDvb];
    const int nC = p.T_pad / kC;
    const long long krow0 = ((long long)b * p.Hk + kh) * p.T_pad;
    const long long vrow0 = ((long long)b * p.Hv + h) * p.T_pad;
    // cp.async groups in flight at the top of chunk ci: [WQU(ci), MK(ci)]
    chain_load_wqu(sm, p, krow0, vrow0, j0, 0, tid);
    chain_load_mk(sm, p, krow0, vrow0, tid);
    const int r16 = 16 * (warp & 3);  // this warp's 16 rows of W (warps 0-3) or Q (warps 4-7)
    for (int ci = 0; ci < nC; ci++) {
        const int par = ci & 1;
        const bool more = ci + 1 < nC;
        cp_async_wait<1>();
        __syncthreads();  // W, Q, U, lc of this chunk (and the state block) are in shared memory
        // [W; Q] S: warps 0-3 the W rows (-> D = U - W S), warps 4-7 the Q rows (kept for Y)
        float ws[1][4][4] = {};
        warp_gemm<true, true, 1, 4>(ws, r16, 0, kDk, lane,
                                    [&](int r, int k) { return warp < 4 ? sm.w[r][k] : sm.q[r][k]; },
                                    [&](int k, int n) { return sm.s[k][n]; });
        if (warp < 4) {
#pragma unroll
            for (int nt = 0; nt < 4; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int r = r16 + g + (e >> 1) * 8, n = nt * 8 + 2 * c + (e & 1);
                    sm.d[r][n] = sm.u[r][n] - ws[0][nt][e];
                }
        }
        __syncthreads();  // D complete; W, Q, U free
        if (more) {
            chain_load_wqu(sm, p, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, j0, par ^ 1, tid);
            cp_async_wait<1>();  // MK(ci) done, WQU(ci + 1) in flight
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // M, K of this chunk are in shared memory
        const float* lc = sm.lc[par];
        const float lcC = lc[kC - 1];
        if (warp >= 4) {
            // Y = diag(e^lc) Q S + M D for this warp's 16 rows
            float md[1][4][4] = {};
            warp_gemm<true, true, 1, 4>(md, r16, 0, kC, lane, [&](int r, int k) { return sm.m[r][k]; },
                                        [&](int k, int n) { return sm.d[k][n]; });
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int r = r16 + g + (e >> 1) * 8;
                const int t = ci * kC + r;
                if (t >= p.n) continue;
                const float gam = expf(lc[r]);
                const long long o = ((long long)b * p.n + t) * p.y_stride + (long long)h * kDv + j0;
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    const int n = nt * 8 + 2 * c + (e & 1);
                    store_from_float(p.y, p.y_dtype, o + n, fmaf(gam, ws[0][nt][e], md[0][nt][e]));
                }
            }
        }
        // S = e^{lc_C} S + K^T diag(e^{lc_C - lc}) D: warp -> 16 rows of d
        {
            float kd[1][4][4] = {};
            const int d0 = 16 * warp;
            warp_gemm<true, true, 1, 4>(kd, d0, 0, kC, lane, [&](int r, int k) { return sm.k[k][r]; },
                                        [&](int k, int n) { return expf(lcC - lc[k]) * sm.d[k][n]; });
            const float gC = expf(lcC);
#pragma unroll
            for (int nt = 0; nt < 4; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int r = d0 + g + (e >> 1) * 8, n = nt * 8 + 2 * c + (e & 1);
                    sm.s[r][n] = fmaf(gC, sm.s[r][n], kd[0][nt][e]);
                }
        }
        __syncthreads();  // S updated; M, K, D free
        if (more) chain_load_mk(sm, p, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, tid);
    }
    for (int i = tid; i < kDk * kDvb; i += 256) S[(long long)(i / kDvb) * kDv + j0 + i % kDvb] = sm.s[i / kDvb][i % kDvb];
}

// ---------------------------------------------------------------- gated RMSNorm (layer path)

__global__ void __launch_bounds__(256) gdn_pf_out_kernel(const GdnPrefillParams p) {
    const int t = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long rb = (long long)p.proj_stride * dtype_bytes(p.proj_dtype);
    const char* row = reinterpret_cast<const char*>(p.proj) + ((long long)b * p.n + t) * rb;
    const float* y = reinterpret_cast<const float*>(p.y) + ((long long)b * p.n + t) * p.y_stride;
    for (int h = warp; h < p.Hv; h += 8) {
        float v[kDv / 32];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < kDv / 32; e++) {
            v[e] = y[h * kDv + e * 32 + lane];
            ss += v[e] * v[e];
        }
        ss = warp_sum(ss);
        const float rinv = 1.0f / sqrtf(ss / (float)kDv + 1e-6f);  // rmsnorm_gated, cpu_ops.cpp:32-38
        const long long orow = ((long long)b * p.n + t) * p.out_stride + (long long)h * kDv;
#pragma unroll
        for (int e = 0; e < kDv / 32; e++) {
            const int j = e * 32 + lane;
            const float z = load_as_float(row, p.proj_dtype, p.C + (long long)h * kDv + j);
            float o = __fmul_rn(__fmul_rn(v[e], rinv), p.norm_w[j]);
            o = o / (1.0f + expf(-z));
            o = __fmul_rn(o, z);
            store_from_float(p.out, p.out_dtype, orow + j, o);
        }
    }
}

}  // namespace

// ---------------------------------------------------------------- host side

size_t gdn_prefill_workspace_bytes(int B, int n, int Hk, int Hv, int C, bool layer) {
    const long long Tp = (long long)(n + kC - 1) / kC * kC;
    size_t s = 0;
    auto add = [&](size_t bytes) { s += (bytes + 255) / 256 * 256; };
    add((size_t)B * Hk * Tp * kDk * 4);  // qb
    add((size_t)B * Hk * Tp * kDk * 4);  // kb
    add((size_t)B * Hv * Tp * kDv * 4);  // vb
    add((size_t)B * Hv * Tp * 4);        // lg
    add((size_t)B * Hv * Tp * 4);        // beta
    add((size_t)B * Hv * Tp * kDk * 4);  // W
    add((size_t)B * Hv * Tp * kDv * 4);  // U
    add((size_t)B * Hv * Tp * kC * 4);   // M
    add((size_t)B * Hv * Tp * 4);        // lc
    if (layer) {
        add((size_t)B * n * Hv * kDv * 4);  // y
        add((size_t)B * C * 3 * 4);          // ring snapshot
        add((size_t)B * Hk * 4);             // position snapshot
    }
    return s;
}

static void carve(GdnPrefillParams& p, void* ws, bool layer) {
    char* c = static_cast<char*>(ws);
    const long long Tp = p.T_pad;
    auto take = [&](size_t bytes) {
        char* r = c;
        c += (bytes + 255) / 256 * 256;
        return r;
    };
    p.qb = reinterpret_cast<float*>(take((size_t)p.B * p.Hk * Tp * kDk * 4));
    p.kb = reinterpret_cast<float*>(take((size_t)p.B * p.Hk * Tp * kDk * 4));
    p.vb = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * kDv * 4));
    p.lg = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * 4));
    p.beta = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * 4));
    p.Wb = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * kDk * 4));
    p.Ub = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * kDv * 4));
    p.Mb = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * kC * 4));
    p.lcb = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * 4));
    if (layer) {
        p.y = take((size_t)p.B * p.n * p.Hv * kDv * 4);
        p.ring_snap = reinterpret_cast<float*>(take((size_t)p.B * p.C * 3 * 4));
        p.pos_snap = reinterpret_cast<int*>(take((size_t)p.B * p.Hk * 4));
    }
}

static int launch_chunks_and_chain(const GdnPrefillParams& p, cudaStream_t stream) {
    const int nC = p.T_pad / kC;
    const size_t chunk_smem = sizeof(ChunkSmem), chain_smem = sizeof(ChainSmem);
    cudaFuncSetAttribute(gdn_pf_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk_smem);
    cudaFuncSetAttribute(gdn_pf_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chain_smem);
    gdn_pf_chunk_kernel<<<dim3(nC, p.Hv, p.B), 256, chunk_smem, stream>>>(p);
    gdn_pf_chain_kernel<<<dim3(p.Hv * (kDv / kDvb), p.B), 256, chain_smem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

int launch_gdn_prefill(GdnPrefillParams p, void* workspace, cudaStream_t stream) {
    if (p.dk != kDk || p.dv != kDv || p.Hv % p.Hk) return ANELM_ERR_UNSUPPORTED;
    p.T_pad = (p.n + kC - 1) / kC * kC;
    carve(p, workspace, true);
    p.y_dtype = ANELM_F32;
    p.y_stride = (long long)p.Hv * kDv;
    gdn_pf_snapshot_kernel<<<dim3((p.C * 3 + 255) / 256, p.B), 256, 0, stream>>>(p);
    const size_t prep_smem = (size_t)p.C * sizeof(float);
    if (prep_smem > 48 * 1024)
        cudaFuncSetAttribute(gdn_pf_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem);
    gdn_pf_prep_kernel<<<dim3(p.T_pad, p.B), 256, prep_smem, stream>>>(p);
    if (int rc = launch_chunks_and_chain(p, stream)) return rc;
    gdn_pf_out_kernel<<<dim3(p.n, p.B), 256, 0, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

int launch_gated_delta_chunked(GdnPrefillParams p, void* workspace, cudaStream_t stream) {
    if (p.dk != kDk || p.dv != kDv || p.Hv % p.Hk) return ANELM_ERR_UNSUPPORTED;
    p.T_pad = (p.n + kC - 1) / kC * kC;
    carve(p, workspace, false);
    gdn_pf_pack_kernel<<<dim3(p.T_pad, p.B), 256, 0, stream>>>(p);
    return launch_chunks_and_chain(p, stream);
}

}  // namespace anelm
