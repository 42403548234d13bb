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
// Precision: every tensor-core operand is held as an fp16 hi + lo pair (x = hi + lo to ~2^-22
// relative) and each product is three mma.sync m16n8k16 (hi*hi + lo*hi + hi*lo) with fp32
// accumulation, so the products match fp32 arithmetic; plain fp16 operands would let the gated
// RMSNorm amplify their 2^-12 rounding past the tolerance.  Operands live in memory as a hi
// plane followed by a lo plane and reach the MMAs through ldmatrix.
//
// Launches:
//   gdn_pf_snapshot_kernel  copy of the conv rings / positions of the plan's sequences (the
//                           prep kernel reads the old ring while the last tokens overwrite it)
//   gdn_pf_prep_kernel      per token: conv + SiLU + L2 / scale, gates; q, k, v (hi / lo) in
//                           chunk layout, log g and beta; the last 3 inputs into the ring
//   gdn_pf_pack_kernel      (core op only) token-major q, k, v, log g, beta -> chunk layout
//   gdn_pf_chunk_kernel     per (chunk, value head): K K^T, Q K^T, T by forward substitution,
//                           W, U, M
//   gdn_pf_chain_kernel     per (sequence, value head, 32 columns): the chunk recurrence over
//                           the state block; each operand buffer is refilled with the next
//                           chunk's data (cp.async) as soon as this chunk's last reader is done
//   gdn_pf_out_kernel       gated RMSNorm of y with z (layer path)
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace anelm {

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kDk = 128;   // key head dim of these kernels
constexpr int kDv = 128;   // value head dim
constexpr int kDvb = 32;   // state columns per chain CTA
constexpr int kP = kDk + 8;   // fp16 pitch of 128-wide tiles (272 B: ldmatrix rows hit distinct banks)
constexpr int kPc = kC + 8;   // fp16 pitch of 64-wide tiles (144 B)

// ---------------------------------------------------------------- fragments (mma.sync m16n8k16)

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float x) {
    const __half h = __float2half_rn(x);
    *hi = h;
    *lo = __float2half_rn(x - __half2float(h));
}

// A (16 x 16) at (r0, k0) of a row-major tile base[r][k]
__device__ __forceinline__ void lda(uint32_t (&a)[4], const __half* base, int pitch, int r0, int k0, int lane) {
    ldmatrix_x4(smem_u32(base + (r0 + (lane & 15)) * pitch + k0 + (lane >> 4) * 8), a[0], a[1], a[2], a[3]);
}
// A (16 x 16) at (r0, k0) of A[r][k] = base[k][r] (the tile is stored transposed)
__device__ __forceinline__ void lda_t(uint32_t (&a)[4], const __half* base, int pitch, int r0, int k0, int lane) {
    const int mat = lane >> 3, i = lane & 7;
    ldmatrix_x4_trans(smem_u32(base + (k0 + i + (mat >> 1) * 8) * pitch + r0 + (mat & 1) * 8), a[0], a[1], a[2], a[3]);
}
// B (16 x 8) fragments of two n-tiles n0, n0 + 8 at k0, with B[k][n] = base[n][k]
__device__ __forceinline__ void ldb2(uint32_t (&b)[4], const __half* base, int pitch, int n0, int k0, int lane) {
    const int mat = lane >> 3, i = lane & 7;
    ldmatrix_x4(smem_u32(base + (n0 + i + (mat >> 1) * 8) * pitch + k0 + (mat & 1) * 8), b[0], b[1], b[2], b[3]);
}
// the same with B[k][n] = base[k][n]
__device__ __forceinline__ void ldb2_t(uint32_t (&b)[4], const __half* base, int pitch, int n0, int k0, int lane) {
    const int mat = lane >> 3, i = lane & 7;
    ldmatrix_x4_trans(smem_u32(base + (k0 + i + (mat & 1) * 8) * pitch + n0 + (mat >> 1) * 8), b[0], b[1], b[2], b[3]);
}
// acc[NT] (16 rows x 8 NT columns) += A[r0.., 0..K) B[0..K, n0..); A and B as hi / lo tiles.
// TA: A stored transposed; TB: B stored [k][n] (else [n][k]).  Per k-step all fragments are
// loaded first and each of the three product terms is issued across the NT accumulators in
// turn, so consecutive MMAs into one accumulator are NT instructions apart.
template <bool TA, bool TB, int NT>
__device__ __forceinline__ void gemm16(float (&acc)[NT][4], const __half* ahi, const __half* alo, int pa,
                                       const __half* bhi, const __half* blo, int pb, int r0, int n0, int K, int lane) {
    static_assert(NT % 2 == 0, "n-tiles come in pairs");
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t ah[4], al[4], bh[NT / 2][4], bl[NT / 2][4];
        if (TA) {
            lda_t(ah, ahi, pa, r0, k0, lane);
            lda_t(al, alo, pa, r0, k0, lane);
        } else {
            lda(ah, ahi, pa, r0, k0, lane);
            lda(al, alo, pa, r0, k0, lane);
        }
#pragma unroll
        for (int np = 0; np < NT / 2; np++) {
            if (TB) {
                ldb2_t(bh[np], bhi, pb, n0 + 16 * np, k0, lane);
                ldb2_t(bl[np], blo, pb, n0 + 16 * np, k0, lane);
            } else {
                ldb2(bh[np], bhi, pb, n0 + 16 * np, k0, lane);
                ldb2(bl[np], blo, pb, n0 + 16 * np, k0, lane);
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
            mma_16816(acc[nt], ah[0], ah[1], ah[2], ah[3], bh[nt / 2][2 * (nt & 1)], bh[nt / 2][2 * (nt & 1) + 1]);
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
            mma_16816(acc[nt], al[0], al[1], al[2], al[3], bh[nt / 2][2 * (nt & 1)], bh[nt / 2][2 * (nt & 1) + 1]);
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
            mma_16816(acc[nt], ah[0], ah[1], ah[2], ah[3], bl[nt / 2][2 * (nt & 1)], bl[nt / 2][2 * (nt & 1) + 1]);
    }
}

// Named barrier over `count` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_bar_sync_cta(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// 16-byte cp.async copies of `rows` rows of `cols` fp16 (hi and lo planes) into a pitched tile pair
__device__ __forceinline__ void cp_tile_hl(__half* dhi, __half* dlo, int pitch, const __half* src, long long plane,
                                           int rows, int cols, int tid, int nthreads) {
    const int vpr = cols / 8;
    for (int i = tid; i < rows * vpr; i += nthreads) {
        const int r = i / vpr, cv = i % vpr;
        cp_async_16(smem_u32(dhi + r * pitch + cv * 8), src + (long long)r * cols + cv * 8, 16);
        cp_async_16(smem_u32(dlo + r * pitch + cv * 8), src + plane + (long long)r * cols + cv * 8, 16);
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

__device__ __forceinline__ void put_hl(__half* hi, long long plane, long long i, float x) {
    split_store(hi + i, hi + plane + i, x);
}

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
            put_hl(p.qh, p.q_plane, o, 0.f);
            put_hl(p.kh, p.q_plane, o, 0.f);
        }
        for (int i = tid; i < Hv * kDv; i += 256) put_hl(p.vh, p.v_plane, (vrow + (long long)(i / kDv) * p.T_pad) * kDv + i % kDv, 0.f);
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
        const long long o = (qrow + (long long)kh * p.T_pad) * kDk;
        for (int i = lane; i < kDk; i += 32) {
            float v = __fmul_rn(x[i], inv);
            if (isq) v = __fmul_rn(v, qscale);
            put_hl(isq ? p.qh : p.kh, p.q_plane, o + i, v);
        }
    }
    for (int i = tid; i < Hv * kDv; i += 256)
        put_hl(p.vh, p.v_plane, (vrow + (long long)(i / kDv) * p.T_pad) * kDv + i % kDv, ys[2 * key_total + i]);
}

// ---------------------------------------------------------------- pack (core op: token-major inputs)

// 8 consecutive values (i a multiple of 8) as hi / lo planes, 16-byte stores
__device__ __forceinline__ void put_hl8(__half* hi, long long plane, long long i, const float (&x)[8]) {
    float h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const __half q = __float2half_rn(x[e]);
        h[e] = __half2float(q);
        l[e] = x[e] - h[e];
    }
    *reinterpret_cast<uint4*>(hi + i) = pack8(h, false);
    *reinterpret_cast<uint4*>(hi + plane + i) = pack8(l, false);
}

__global__ void __launch_bounds__(256) gdn_pf_pack_kernel(const GdnPrefillParams p) {
    const int t = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int Hk = p.Hk, Hv = p.Hv;
    const bool live = t < p.n;
    const long long tok = (long long)b * p.n + t;
    if (p.in_vec) {  // 16-byte aligned rows: 8 values per thread and step
        const int nq = Hk * kDk / 8, nv = Hv * kDv / 8;
        const int eb = dtype_bytes(p.in_dtype);
        for (int gi = tid; gi < 2 * nq + nv; gi += 256) {
            float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (gi < 2 * nq) {
                const bool isk = gi >= nq;
                const int e = (isk ? gi - nq : gi) * 8;
                if (live)
                    load8(reinterpret_cast<const char*>(isk ? p.k_in : p.q_in) + tok * Hk * kDk * eb, p.in_dtype, e, x);
                const long long o = (((long long)b * Hk + e / kDk) * p.T_pad + t) * kDk + e % kDk;
                put_hl8(isk ? p.kh : p.qh, p.q_plane, o, x);
            } else {
                const int e = (gi - 2 * nq) * 8;
                if (live) load8(reinterpret_cast<const char*>(p.v_in) + tok * Hv * kDv * eb, p.in_dtype, e, x);
                const long long o = (((long long)b * Hv + e / kDv) * p.T_pad + t) * kDv + e % kDv;
                put_hl8(p.vh, p.v_plane, o, x);
            }
        }
    } else {
        for (int i = tid; i < Hk * kDk; i += 256) {
            const long long o = (((long long)b * Hk + i / kDk) * p.T_pad + t) * kDk + i % kDk;
            put_hl(p.qh, p.q_plane, o, live ? load_as_float(p.q_in, p.in_dtype, tok * Hk * kDk + i) : 0.f);
            put_hl(p.kh, p.q_plane, o, live ? load_as_float(p.k_in, p.in_dtype, tok * Hk * kDk + i) : 0.f);
        }
        for (int i = tid; i < Hv * kDv; i += 256) {
            const long long o = (((long long)b * Hv + i / kDv) * p.T_pad + t) * kDv + i % kDv;
            put_hl(p.vh, p.v_plane, o, live ? load_as_float(p.v_in, p.in_dtype, tok * Hv * kDv + i) : 0.f);
        }
    }
    for (int h = tid; h < Hv; h += 256) {
        const long long o = ((long long)b * Hv + h) * p.T_pad + t;
        p.lg[o] = live ? p.lg_in[tok * Hv + h] : 0.f;
        p.beta[o] = live ? p.beta_in[tok * Hv + h] : 0.f;
    }
}

// ---------------------------------------------------------------- per-chunk quantities

struct ChunkSmem {
    __half khi[kC][kP], klo[kC][kP];
    __half qhi[kC][kP], qlo[kC][kP];    // Q, then V
    float at[kC][kC];                   // A^T, rows interleaved: at[i][16 (t % 4) + t / 4] = A[t][i]
    __half thi[kC][kPc], tlo[kC][kPc];  // T scaled by columns (W's, then U's factors)
    float lc[kC], lt[kC], bt[kC];
};

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
    cp_tile_hl(&sm.khi[0][0], &sm.klo[0][0], kP, p.kh + krow * kDk, p.q_plane, kC, kDk, tid, 256);
    cp_tile_hl(&sm.qhi[0][0], &sm.qlo[0][0], kP, p.qh + krow * kDk, p.q_plane, kC, kDk, tid, 256);
    cp_async_commit();
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
    cp_async_wait<0>();
    __syncthreads();
    // K K^T -> A (strictly lower), Q K^T -> M (lower incl. diagonal): warp -> 16 rows x 32 columns
    {
        const int r0 = 16 * (warp & 3), n0 = 32 * (warp >> 2);
        float kk[4][4] = {}, qk[4][4] = {};
        gemm16<false, false, 4>(kk, &sm.khi[0][0], &sm.klo[0][0], kP, &sm.khi[0][0], &sm.klo[0][0], kP, r0, n0, kDk, lane);
        gemm16<false, false, 4>(qk, &sm.qhi[0][0], &sm.qlo[0][0], kP, &sm.khi[0][0], &sm.klo[0][0], kP, r0, n0, kDk, lane);
        __half* mhi = p.mh + vrow * kC;
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int r = r0 + g + (e >> 1) * 8, i = n0 + nt * 8 + 2 * c + (e & 1);
                sm.at[i][16 * (r & 3) + (r >> 2)] = i < r ? sm.bt[r] * expf(sm.lt[r] - sm.lc[i]) * kk[nt][e] : 0.f;
                put_hl(mhi, p.m_plane, r * kC + i, i <= r ? expf(sm.lc[r] - sm.lc[i]) * qk[nt][e] : 0.f);
            }
    }
    if (tid < kC) p.lcb[vrow + tid] = sm.lc[tid];
    __syncthreads();  // Q no longer needed: V into its buffers
    cp_tile_hl(&sm.qhi[0][0], &sm.qlo[0][0], kP, p.vh + vrow * kDv, p.v_plane, kC, kDv, tid, 256);
    cp_async_commit();
    // T = (I + A)^{-1} by forward substitution, one column j per 4 threads: x_t = [t == j] - sum_{i<t} A_ti x_i,
    // right-looking: thread part pt keeps the running sums r of rows t = 4m + pt; once x_t is final (in the
    // thread owning row t) it is broadcast to the 4 threads, which add A[4m + pt][t] x_t to their rows'
    // sums (column t of A read as four 16-byte words).  A is strictly lower, so rows <= t add zeros.
    const int j = tid >> 2, pt = tid & 3;
    float xs[kC / 4], rs[kC / 4];
#pragma unroll
    for (int m = 0; m < kC / 4; m++) xs[m] = rs[m] = 0.f;
#pragma unroll
    for (int t = 0; t < kC; t++) {
        const float x = __shfl_sync(0xffffffffu, (t == j ? 1.0f : 0.0f) - rs[t >> 2], (lane & ~3) | (t & 3));
        if (pt == (t & 3)) xs[t >> 2] = x;
        const float4* col = reinterpret_cast<const float4*>(&sm.at[t][16 * pt]);
#pragma unroll
        for (int q = 0; q < kC / 16; q++) {
            if (16 * q + 15 <= t) continue;  // rows 4m + pt <= 4m + 3 <= t of this word are final
            const float4 a4 = col[q];
            rs[4 * q] = fmaf(a4.x, x, rs[4 * q]);
            rs[4 * q + 1] = fmaf(a4.y, x, rs[4 * q + 1]);
            rs[4 * q + 2] = fmaf(a4.z, x, rs[4 * q + 2]);
            rs[4 * q + 3] = fmaf(a4.w, x, rs[4 * q + 3]);
        }
    }
    {  // T' = T diag(beta e^{lt}) (W's factor) as hi / lo; column j belongs to this thread group
        const float fw = sm.bt[j] * expf(sm.lt[j]);
#pragma unroll
        for (int m = 0; m < kC / 4; m++) split_store(&sm.thi[4 * m + pt][j], &sm.tlo[4 * m + pt][j], xs[m] * fw);
    }
    cp_async_wait<0>();
    __syncthreads();
    const int r0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);  // warp -> 16 rows x 64 columns of W / U
    {  // W = T diag(beta e^{lt}) K
        float w[8][4] = {};
        gemm16<false, true, 8>(w, &sm.thi[0][0], &sm.tlo[0][0], kPc, &sm.khi[0][0], &sm.klo[0][0], kP, r0, n0, kC, lane);
        __half* whi = p.wh + vrow * kDk;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int r = r0 + g + (e >> 1) * 8, n = n0 + nt * 8 + 2 * c + (e & 1);
                put_hl(whi, p.v_plane, r * kDk + n, w[nt][e]);
            }
    }
    __syncthreads();  // T' read by every warp
    {  // T'' = T diag(beta) (U's factor)
        const float fu = sm.bt[j];
#pragma unroll
        for (int m = 0; m < kC / 4; m++) split_store(&sm.thi[4 * m + pt][j], &sm.tlo[4 * m + pt][j], xs[m] * fu);
    }
    __syncthreads();
    {  // U = T diag(beta) V
        float u[8][4] = {};
        gemm16<false, true, 8>(u, &sm.thi[0][0], &sm.tlo[0][0], kPc, &sm.qhi[0][0], &sm.qlo[0][0], kP, r0, n0, kC, lane);
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const int r = r0 + g + (e >> 1) * 8, n = n0 + nt * 8 + 2 * c;
                *reinterpret_cast<float2*>(p.Ub + (vrow + r) * kDv + n) = make_float2(u[nt][e], u[nt][e + 1]);
            }
    }
}

// ---------------------------------------------------------------- the recurrence over chunks

// One chain CTA per (sequence, value head, 32 state columns j0 .. j0 + 32), four warps: warp
// (jg, dh) = (warp / 2, warp % 2) keeps S^T rows j0 + 16 jg .. + 16 (state columns) times key dims
// d in [64 dh, 64 dh + 64) in registers, in the accumulator layout of mma.m16n8k16, which is also
// the A-operand layout: S^T feeds W S and Q S directly (as hi / lo pairs), and the state update
// S^T += E^T K accumulates into the same registers.  The two warps of a column group hold the two
// halves of d, so their partial W S and Q S sums meet in shared memory.  Per chunk and warp:
//   [W; Q] S over its d half -> exchange -> D = U - W S (all 64 rows t), Y = e^lc Q S + M D for
//   its 32 rows t, S = e^{lc_C} S + K^T (e^{lc_C - lc} D) for its d half.
constexpr int kChainThreads = 128;
struct ChainSmem {
    __half whi[kC][kP], wlo[kC][kP];   // W[t][d]
    __half qhi[kC][kP], qlo[kC][kP];   // Q[t][d]
    __half khi[kC][kP], klo[kC][kP];   // K[t][d]
    __half mhi[kC][kPc], mlo[kC][kPc]; // M[t][i]
    float u[kC][kDvb + 4];             // U columns of this block
    float lc[2][kC];                   // in-chunk cumulative log decay, by chunk parity
    float xd[4][32][32];               // partial W S of each warp, [warp][register][lane]
    float xy[4][32][32];               // partial Q S
};

__device__ __forceinline__ uint32_t h2u(const __half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
// x0, x1 as an fp16 hi pair and the fp16 pair of the remainders
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}
// A fragments (hi / lo) of k-step ks from accumulator tiles acc[2 ks] (k 0-7) and acc[2 ks + 1]
// (k 8-15), each column scaled by sc (sc[nt][0 / 1]: columns 8 nt + 2 c, + 1)
template <int NT>
__device__ __forceinline__ void afrag(const float (&acc)[NT][4], const float (&sc)[NT][2], int ks, uint32_t (&ah)[4],
                                      uint32_t (&al)[4]) {
    const int t0 = 2 * ks, t1 = 2 * ks + 1;
    split2(acc[t0][0] * sc[t0][0], acc[t0][1] * sc[t0][1], ah[0], al[0]);
    split2(acc[t0][2] * sc[t0][0], acc[t0][3] * sc[t0][1], ah[1], al[1]);
    split2(acc[t1][0] * sc[t1][0], acc[t1][1] * sc[t1][1], ah[2], al[2]);
    split2(acc[t1][2] * sc[t1][0], acc[t1][3] * sc[t1][1], ah[3], al[3]);
}
template <int NT>
__device__ __forceinline__ void afrag(const float (&acc)[NT][4], int ks, uint32_t (&ah)[4], uint32_t (&al)[4]) {
    const int t0 = 2 * ks, t1 = 2 * ks + 1;
    split2(acc[t0][0], acc[t0][1], ah[0], al[0]);
    split2(acc[t0][2], acc[t0][3], ah[1], al[1]);
    split2(acc[t1][0], acc[t1][1], ah[2], al[2]);
    split2(acc[t1][2], acc[t1][3], ah[3], al[3]);
}
// acc[0 / 1] += A B for the n-tile pair of b (hi / lo fragments from ldb2 / ldb2_t): three terms
__device__ __forceinline__ void mma3x2(float (&a0)[4], float (&a1)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                       const uint32_t (&bh)[4], const uint32_t (&bl)[4]) {
    mma_16816(a0, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
    mma_16816(a1, ah[0], ah[1], ah[2], ah[3], bh[2], bh[3]);
    mma_16816(a0, al[0], al[1], al[2], al[3], bh[0], bh[1]);
    mma_16816(a1, al[0], al[1], al[2], al[3], bh[2], bh[3]);
    mma_16816(a0, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
    mma_16816(a1, ah[0], ah[1], ah[2], ah[3], bl[2], bl[3]);
}

// cp.async of a chunk's W and Q (read by [W; Q] S)
__device__ __forceinline__ void chain_load_wq(ChainSmem& sm, const GdnPrefillParams& p, long long krow, long long vrow,
                                              int tid) {
    cp_tile_hl(&sm.whi[0][0], &sm.wlo[0][0], kP, p.wh + vrow * kDk, p.v_plane, kC, kDk, tid, kChainThreads);
    cp_tile_hl(&sm.qhi[0][0], &sm.qlo[0][0], kP, p.qh + krow * kDk, p.q_plane, kC, kDk, tid, kChainThreads);
    cp_async_commit();
}
// cp.async of a chunk's U columns and lc (read by D = U - W S and the decay factors)
__device__ __forceinline__ void chain_load_u(ChainSmem& sm, const GdnPrefillParams& p, long long vrow, int j0, int par,
                                             int tid) {
    for (int i = tid; i < kC * (kDvb / 4); i += kChainThreads) {
        const int r = i / (kDvb / 4), cv = i % (kDvb / 4);
        cp_async_16(smem_u32(&sm.u[r][cv * 4]), p.Ub + (vrow + r) * kDv + j0 + cv * 4, 16);
    }
    if (tid < kC / 4) cp_async_16(smem_u32(&sm.lc[par][tid * 4]), p.lcb + vrow + tid * 4, 16);
    cp_async_commit();
}
// cp.async of a chunk's M and K (read by M D and the state update)
__device__ __forceinline__ void chain_load_mk(ChainSmem& sm, const GdnPrefillParams& p, long long krow, long long vrow,
                                              int tid) {
    cp_tile_hl(&sm.khi[0][0], &sm.klo[0][0], kP, p.kh + krow * kDk, p.q_plane, kC, kDk, tid, kChainThreads);
    cp_tile_hl(&sm.mhi[0][0], &sm.mlo[0][0], kPc, p.mh + vrow * kC, p.m_plane, kC, kC, tid, kChainThreads);
    cp_async_commit();
}

__global__ void __launch_bounds__(kChainThreads, 1) gdn_pf_chain_kernel(const GdnPrefillParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    ChainSmem& sm = *reinterpret_cast<ChainSmem*>(smem_raw);
    const int nblk = kDv / kDvb;
    const int h = blockIdx.x / nblk, j0 = (blockIdx.x % nblk) * kDvb, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int jg = warp >> 1, dh = warp & 1;
    const int jr = 16 * jg;      // this warp's state columns j0 + jr .. + 16
    const int dbase = 64 * dh;   // and key dims dbase .. + 64
    const int kh = h / (p.Hv / p.Hk);
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    float* S = p.state + ((long long)seq * p.Hv + h) * kDk * kDv;
    // s[nt][e] = S[d][j0 + j], j = jr + g + 8 (e / 2), d = dbase + 8 nt + 2 c + (e % 2)
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++)
            s[nt][e] = S[(long long)(dbase + 8 * nt + 2 * c + (e & 1)) * kDv + j0 + jr + g + 8 * (e >> 1)];
    const int nC = p.T_pad / kC;
    const long long krow0 = ((long long)b * p.Hk + kh) * p.T_pad;
    const long long vrow0 = ((long long)b * p.Hv + h) * p.T_pad;
    // cp.async groups in flight at the top of chunk ci: [WQ(ci), U(ci), MK(ci)]
    chain_load_wq(sm, p, krow0, vrow0, tid);
    chain_load_u(sm, p, vrow0, j0, 0, tid);
    chain_load_mk(sm, p, krow0, vrow0, tid);
    for (int ci = 0; ci < nC; ci++) {
        const int par = ci & 1;
        const bool more = ci + 1 < nC;
        cp_async_wait<2>();
        __syncthreads();  // W and Q of this chunk are in shared memory
        // ---- [W; Q] S over this warp's half of d: D part and Y part, all 64 rows t ----
        float ad[8][4], ay[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) ad[nt][e] = ay[nt][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            uint32_t ah[4], al[4];
            afrag(s, ks, ah, al);
            const int k0 = dbase + 16 * ks;
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t bh[4], bl[4];
                ldb2(bh, &sm.whi[0][0], kP, 16 * np, k0, lane);
                ldb2(bl, &sm.wlo[0][0], kP, 16 * np, k0, lane);
                mma3x2(ad[2 * np], ad[2 * np + 1], ah, al, bh, bl);
                ldb2(bh, &sm.qhi[0][0], kP, 16 * np, k0, lane);
                ldb2(bl, &sm.qlo[0][0], kP, 16 * np, k0, lane);
                mma3x2(ay[2 * np], ay[2 * np + 1], ah, al, bh, bl);
            }
        }
        __syncthreads();  // W, Q free
        if (more) chain_load_wq(sm, p, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, tid);
        // ---- the two d halves of this column group meet ----
#pragma unroll
        for (int r = 0; r < 32; r++) {
            sm.xd[warp][r][lane] = ad[r >> 2][r & 3];
            sm.xy[warp][r][lane] = ay[r >> 2][r & 3];
        }
        named_bar_sync_cta(1 + jg, 64);
        // Q S of this warp's rows t in [32 dh, 32 dh + 32) (the other half is the partner's)
        float y[4][4];
#pragma unroll
        for (int n4 = 0; n4 < 4; n4++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                y[n4][e] = (dh ? ay[4 + n4][e] : ay[n4][e]) + sm.xy[warp ^ 1][4 * (4 * dh + n4) + e][lane];
#pragma unroll
        for (int r = 0; r < 32; r++) ad[r >> 2][r & 3] += sm.xd[warp ^ 1][r][lane];
        if (more) cp_async_wait<2>();
        else cp_async_wait<1>();
        __syncthreads();  // U and lc of this chunk are in shared memory
        const float* lc = sm.lc[par];
        const float lcC = lc[kC - 1];
        // D = U - W S (in place of ad)
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                ad[nt][e] = sm.u[8 * nt + 2 * c + (e & 1)][jr + g + 8 * (e >> 1)] - ad[nt][e];
        if (more) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();  // M and K of this chunk are in shared memory; U read by every warp
        if (more) chain_load_u(sm, p, vrow0 + (ci + 1) * kC, j0, par ^ 1, tid);
        // ---- Y = e^lc Q S + M D for rows t in [32 dh, 32 dh + 32) ----
        {
            const int tt = 32 * dh;
#pragma unroll
            for (int n4 = 0; n4 < 4; n4++)
#pragma unroll
                for (int e = 0; e < 4; e++) y[n4][e] *= expf(lc[tt + 8 * n4 + 2 * c + (e & 1)]);
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                if (16 * ks >= tt + 32) break;  // M[t][i] = 0 for i > t
                uint32_t ah[4], al[4];
                afrag(ad, ks, ah, al);
#pragma unroll
                for (int np = 0; np < 2; np++) {
                    uint32_t bh[4], bl[4];
                    ldb2(bh, &sm.mhi[0][0], kPc, tt + 16 * np, 16 * ks, lane);
                    ldb2(bl, &sm.mlo[0][0], kPc, tt + 16 * np, 16 * ks, lane);
                    mma3x2(y[2 * np], y[2 * np + 1], ah, al, bh, bl);
                }
            }
#pragma unroll
            for (int n4 = 0; n4 < 4; n4++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int t = ci * kC + tt + 8 * n4 + 2 * c + (e & 1);
                    if (t < p.n)
                        store_from_float(p.y, p.y_dtype,
                                         ((long long)b * p.n + t) * p.y_stride + (long long)h * kDv + j0 + jr + g +
                                             8 * (e >> 1),
                                         y[n4][e]);
                }
        }
        // ---- S = e^{lc_C} S + K^T diag(e^{lc_C - lc}) D over this warp's half of d ----
        {
            const float gC = expf(lcC);
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) s[nt][e] *= gC;
            float fs[8][2];  // e^{lc_C - lc_t}, t = 8 nt + 2 c + e
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 2; e++) fs[nt][e] = expf(lcC - lc[8 * nt + 2 * c + e]);
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                uint32_t ah[4], al[4];
                afrag(ad, fs, ks, ah, al);
#pragma unroll
                for (int np = 0; np < 4; np++) {
                    uint32_t bh[4], bl[4];
                    ldb2_t(bh, &sm.khi[0][0], kP, dbase + 16 * np, 16 * ks, lane);
                    ldb2_t(bl, &sm.klo[0][0], kP, dbase + 16 * np, 16 * ks, lane);
                    mma3x2(s[2 * np], s[2 * np + 1], ah, al, bh, bl);
                }
            }
        }
        __syncthreads();  // M, K free
        if (more) chain_load_mk(sm, p, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, tid);
    }
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++)
            S[(long long)(dbase + 8 * nt + 2 * c + (e & 1)) * kDv + j0 + jr + g + 8 * (e >> 1)] = s[nt][e];
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
            const int jj = e * 32 + lane;
            const float z = load_as_float(row, p.proj_dtype, p.C + (long long)h * kDv + jj);
            float o = __fmul_rn(__fmul_rn(v[e], rinv), p.norm_w[jj]);
            o = o / (1.0f + expf(-z));
            o = __fmul_rn(o, z);
            store_from_float(p.out, p.out_dtype, orow + jj, o);
        }
    }
}

}  // namespace

// ---------------------------------------------------------------- host side

size_t gdn_prefill_workspace_bytes(int B, int n, int Hk, int Hv, int C, bool layer) {
    const long long Tp = (long long)(n + kC - 1) / kC * kC;
    size_t s = 0;
    auto add = [&](size_t bytes) { s += (bytes + 255) / 256 * 256; };
    add((size_t)B * Hk * Tp * kDk * 4);  // q hi + lo
    add((size_t)B * Hk * Tp * kDk * 4);  // k hi + lo
    add((size_t)B * Hv * Tp * kDv * 4);  // v hi + lo
    add((size_t)B * Hv * Tp * 4);        // lg
    add((size_t)B * Hv * Tp * 4);        // beta
    add((size_t)B * Hv * Tp * kDk * 4);  // W hi + lo
    add((size_t)B * Hv * Tp * kDv * 4);  // U
    add((size_t)B * Hv * Tp * kC * 4);   // M hi + lo
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
    p.q_plane = (long long)p.B * p.Hk * Tp * kDk;
    p.v_plane = (long long)p.B * p.Hv * Tp * kDv;
    p.m_plane = (long long)p.B * p.Hv * Tp * kC;
    p.qh = reinterpret_cast<__half*>(take((size_t)p.q_plane * 4));
    p.kh = reinterpret_cast<__half*>(take((size_t)p.q_plane * 4));
    p.vh = reinterpret_cast<__half*>(take((size_t)p.v_plane * 4));
    p.lg = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * 4));
    p.beta = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * 4));
    p.wh = reinterpret_cast<__half*>(take((size_t)p.v_plane * 4));
    p.Ub = reinterpret_cast<float*>(take((size_t)p.B * p.Hv * Tp * kDv * 4));
    p.mh = reinterpret_cast<__half*>(take((size_t)p.m_plane * 4));
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
    gdn_pf_chain_kernel<<<dim3(p.Hv * (kDv / kDvb), p.B), kChainThreads, chain_smem, stream>>>(p);
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
    p.in_vec = (uintptr_t)p.q_in % 16 == 0 && (uintptr_t)p.k_in % 16 == 0 && (uintptr_t)p.v_in % 16 == 0;
    gdn_pf_pack_kernel<<<dim3(p.T_pad, p.B), 256, 0, stream>>>(p);
    return launch_chunks_and_chain(p, stream);
}

}  // namespace anelm
