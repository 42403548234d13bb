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
// relative) and each product is three tcgen05 MMAs (hi*hi + lo*hi + hi*lo) with fp32 accumulation
// in TMEM, so the products match fp32 arithmetic; plain fp16 operands would let the gated RMSNorm
// amplify their 2^-12 rounding past the tolerance.  Operands live in memory as a hi plane followed
// by a lo plane and reach shared memory by TMA.  When the bare core op gets 16-bit q / k / v they
// are exact, so they need no lo plane: K K^T / Q K^T take one term and the products with K, Q or V
// on one side take two; [Q; W] S takes two as well, W meeting S by its hi plane alone (the state
// and U keep their pairs: their lo planes carry the accuracy).  On 16-byte boundaries they are read in place (4D tensor maps over the
// caller's [B][n][heads][128] arrays, no pack), and with bf16 inputs the operands that meet them in
// an MMA are bf16 hi / lo pairs (16 significant bits, ~1e-5 relative per product).
//
// Launches:
//   gdn_pf_snapshot_kernel  copy of the conv rings / positions of the plan's sequences (the
//                           prep kernel reads the old ring while the last tokens overwrite it)
//   gdn_pf_prep_kernel      per token: conv + SiLU + L2 / scale, gates; q, k, v (hi / lo) in
//                           chunk layout, log g and beta; the last 3 inputs into the ring
//   gdn_pf_pack_kernel      (core op, 32-bit or unaligned inputs) token-major q, k, v, log g, beta ->
//                           chunk layout
//   gdn_pf_chunk_kernel     per (chunk, value head): K K^T, Q K^T, T by forward substitution,
//                           W, U, M
//   gdn_pf_chain_tc_kernel  per (sequence, value head, 32 columns): the chunk recurrence over
//                           the state block on tcgen05, warp-specialised; each operand buffer is
//                           refilled with the next chunk's data (TMA) as soon as this chunk's
//                           last reader is done
//   gdn_pf_out_kernel       gated RMSNorm of y with z (layer path)
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

namespace anelm {

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kDk = 128;   // key head dim of these kernels
constexpr int kDv = 128;   // value head dim
constexpr int kUBox = 32;  // fp32 columns of one U tile box (128 bytes)

// ---------------------------------------------------------------- hi / lo operand planes

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float x) {
    const __half h = __float2half_rn(x);
    *hi = h;
    *lo = __float2half_rn(x - __half2float(h));
}

__device__ __forceinline__ uint32_t h2u(const __half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
// x0, x1 as an fp16 hi pair and the fp16 pair of the remainders
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}
// the same split in bf16 (8 + 8 significant bits): the operands that meet bf16 inputs in an MMA
__device__ __forceinline__ void split2_bf(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// hi / lo planes (fp16, or bf16 with BF) of 8 consecutive values as two 16-byte words
template <bool BF = false>
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (BF) split2_bf(v[2 * i], v[2 * i + 1], h[i], l[i]);
        else split2(v[2 * i], v[2 * i + 1], h[i], l[i]);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
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

// 8 consecutive values (i a multiple of 8) as hi / lo planes, 16-byte stores (hi only: values exact in fp16)
__device__ __forceinline__ void put_hl8(__half* hi, long long plane, long long i, const float (&x)[8],
                                        bool hi_only = false) {
    float h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const __half q = __float2half_rn(x[e]);
        h[e] = __half2float(q);
        l[e] = x[e] - h[e];
    }
    *reinterpret_cast<uint4*>(hi + i) = pack8(h, false);
    if (!hi_only) *reinterpret_cast<uint4*>(hi + plane + i) = pack8(l, false);
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
                put_hl8(isk ? p.kh : p.qh, p.q_plane, o, x, p.qkv_exact);
            } else {
                const int e = (gi - 2 * nq) * 8;
                if (live) load8(reinterpret_cast<const char*>(p.v_in) + tok * Hv * kDv * eb, p.in_dtype, e, x);
                const long long o = (((long long)b * Hv + e / kDv) * p.T_pad + t) * kDv + e % kDv;
                put_hl8(p.vh, p.v_plane, o, x, p.qkv_exact);
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

// One CTA per (chunk, value head, sequence), 256 threads, two tcgen05 GEMMs (fp32 accumulators in
// TMEM, fp16 operands staged by TMA with the 128-byte swizzle, each product as three MMAs over the
// hi / lo planes: hi*hi + lo*hi + hi*lo):
//   GEMM 1  [K; Q] K^T  (M 128 = 64 K rows + 64 Q rows, N 64, K 128): K K^T -> A, Q K^T -> M;
//   GEMM 2  [T'; T''] [K | V]  (M 128, K 64) with T' = T diag(beta e^{lt}), T'' = T diag(beta), in two
//           N = 128 halves through the same 128 TMEM columns: [T'; T''] [K0 K1], whose rows 0-63 are
//           W = T' K, then [T'; T''] [V0 V1], whose rows 64-127 are U = T'' V (the other rows unused).
// The operand buffer of each plane is [K d0-63 | Q d0-63 | K d64-127 | Q d64-127] (8 KB boxes of
// 64 rows x 128 bytes): read as the K-major A of GEMM 1 (two 16 KB boxes of 128 rows), as its
// K-major B (the K rows), and, once V has replaced Q, as the MN-major B of GEMM 2 (N boxes K0, K1 or
// V0, V1, 16 KB apart).  T = (I + A)^{-1} by forward substitution on the CUDA cores in between.  With
// exact inputs the lo plane is not allocated: 71 KB of shared memory and 128 TMEM columns admit three
// CTAs per SM.
constexpr int kChunkThreads = 256;
constexpr int kOpPlane = 32768;            // bytes of one plane of the operand buffer
constexpr int kTPlane = 16384;             // bytes of one plane of [T'; T''] (128 rows x 128 bytes)
constexpr int kTs = kC + 4;                // fp32 pitch of A and T in the inversion
constexpr uint32_t kChunkTmemCols = 128;
struct ChunkSmem {
    uint8_t op[kOpPlane];                  // hi plane of the operand buffer (1024-byte aligned)
    union {
        uint8_t t[2][kTPlane];             // [T'; T''] hi, lo (K-major, 128-byte swizzle)
        struct {
            float a[kC][kTs];              // A (strictly lower)
            float tm[kC][kTs];             // T = (I + A)^{-1}
            float z[3][16][17];            // block products of one level
        } inv;
        uint8_t ustage[4 * 8192];          // U staged for its tile stores once GEMM 2 is done
    };
    float lc[kC], lt[kC], bt[kC];
    uint64_t bar[5];                       // K+Q loaded, GEMM 1 done, V loaded, GEMM 2 K half done, V half done
    uint32_t tmem_slot;
    int abort;
    alignas(1024) uint8_t op_lo[kOpPlane];  // lo plane: allocated and read only for inputs that are not exact
};
// shared memory of a chunk-kernel CTA (with the slack that aligns its base to 1024 bytes)
inline size_t chunk_smem_bytes(bool exact) { return (exact ? offsetof(ChunkSmem, op_lo) : sizeof(ChunkSmem)) + 1024; }


// byte offset of element (row, col) (fp16, 64 columns per 128-byte row) in a 128B-swizzled tile
__device__ __forceinline__ int sw128_off(int row, int col) {
    return row * 128 + ((((col >> 3) ^ row) & 7) << 4) + (col & 7) * 2;
}

template <bool BF>
__global__ void __launch_bounds__(kChunkThreads, 3) gdn_pf_chunk_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                      const __grid_constant__ CUtensorMap tmQ,
                                                                      const __grid_constant__ CUtensorMap tmV,
                                                                      const __grid_constant__ CUtensorMap tmW,
                                                                      const __grid_constant__ CUtensorMap tmU,
                                                                      const GdnPrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ci = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kh = h / (p.Hv / p.Hk);
    const int t0 = ci * kC;
    const long long krow = ((long long)b * p.Hk + kh) * p.T_pad + t0;
    const long long vrow = ((long long)b * p.Hv + h) * p.T_pad + t0;
    volatile int* abort = &sm.abort;
    uint64_t* bar = sm.bar;
    if (tid == 0) {
        sm.abort = 0;
        for (int i = 0; i < 5; i++) tc::mbar_init(&bar[i], 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&sm.tmem_slot, kChunkTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;
    const uint32_t aop = (uint32_t)__cvta_generic_to_shared(&sm.op[0]);
    const uint32_t aop_lo = (uint32_t)__cvta_generic_to_shared(&sm.op_lo[0]);  // not inside the launch when exact
    const uint32_t at_ = (uint32_t)__cvta_generic_to_shared(&sm.t[0][0]);
    auto opl = [&](int pl) { return pl ? sm.op_lo : sm.op; };  // a plane of the operand buffer
    if (tid == 0) {  // K and Q, both planes, into the operand buffers
        tc::prefetch_tmap(&tmK);
        tc::prefetch_tmap(&tmQ);
        const bool lo = !p.qkv_exact;  // exact 16-bit inputs: the lo plane is zero, not loaded
        tc::mbar_arrive_expect_tx(&bar[0], (lo ? 2 : 1) * kOpPlane);
#pragma unroll
        for (int pl = 0; pl < 2; pl++)
            if (pl == 0 || lo)
#pragma unroll
                for (int kb = 0; kb < 2; kb++) {
                    if (p.direct) {  // the caller's token-major q / k: [b][token][head][d]
                        tc::tma_load_4d(opl(pl) + kb * 16384, &tmK, &bar[0], kb * 64, kh, t0, b);
                        tc::tma_load_4d(opl(pl) + kb * 16384 + 8192, &tmQ, &bar[0], kb * 64, kh, t0, b);
                    } else {
                        tc::tma_load_3d(opl(pl) + kb * 16384, &tmK, &bar[0], kb * 64, (int)krow, pl);
                        tc::tma_load_3d(opl(pl) + kb * 16384 + 8192, &tmQ, &bar[0], kb * 64, (int)krow, pl);
                    }
                }
    }
    if (warp == 1) {  // inclusive prefix sum of log g over the chunk (two tokens per lane)
        // log g and beta of tokens t0 + 2 lane, + 1 (direct: the caller's [b][token][head] arrays, zero
        // past the prompt)
        float g0, g1, b0, b1;
        if (p.direct) {
            const int ta = t0 + 2 * lane, tb = ta + 1;
            const long long ia = ((long long)b * p.n + ta) * p.Hv + h, ib = ia + p.Hv;
            g0 = ta < p.n ? p.lg_in[ia] : 0.f;
            g1 = tb < p.n ? p.lg_in[ib] : 0.f;
            b0 = ta < p.n ? p.beta_in[ia] : 0.f;
            b1 = tb < p.n ? p.beta_in[ib] : 0.f;
        } else {
            g0 = p.lg[vrow + 2 * lane];
            g1 = p.lg[vrow + 2 * lane + 1];
            b0 = p.beta[vrow + 2 * lane];
            b1 = p.beta[vrow + 2 * lane + 1];
        }
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
        sm.bt[2 * lane] = b0;
        sm.bt[2 * lane + 1] = b1;
    }
    if (tid == 0) {  // GEMM 1: [K; Q] K^T -> TMEM columns [0, 64)
        if (tc::mbar_wait(&bar[0], 0, p.err, ANELM_ERR_TIMEOUT, abort)) {
            tc::tc_fence_after();
            constexpr uint32_t id1 = BF ? tc::idesc_as_bf16(tc::idesc_f16_f32(128, kC)) : tc::idesc_f16_f32(128, kC);
            // exact inputs: K and Q are exact in fp16, so hi * hi is the whole product
            const bool lo_terms = !p.qkv_exact;
#pragma unroll
            for (int term = 0; term < 3; term++) {
                const uint32_t pa = term == 1 ? aop_lo : aop, pb = term == 2 ? aop_lo : aop;
                if (term == 0 || lo_terms)
#pragma unroll
                    for (int kb = 0; kb < 2; kb++)
#pragma unroll
                        for (int ks = 0; ks < 4; ks++)
                            tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(pa + kb * 16384 + ks * 32),
                                           tc::desc_kmajor_sw128(pb + kb * 16384 + ks * 32), id1, (term | kb | ks) != 0);
            }
            tc::mma_commit(&bar[1]);
        }
    }
    // ---- epilogue 1: A (rows 0-63) into shared memory, M (rows 64-127) to global ----
    const bool ok1 = tc::mbar_wait(&bar[1], 0, p.err, ANELM_ERR_TIMEOUT, abort);
    tc::tc_fence_after();
    __syncthreads();  // lc / lt / bt visible; every thread past GEMM 1 (Q no longer read)
    if (tid == 0 && ok1) {  // V replaces Q in the operand buffers
        tc::prefetch_tmap(&tmV);
        const bool lo = !p.qkv_exact;
        tc::mbar_arrive_expect_tx(&bar[2], (lo ? 2 : 1) * (kOpPlane / 2));
#pragma unroll
        for (int pl = 0; pl < 2; pl++)
            if (pl == 0 || lo)
#pragma unroll
                for (int kb = 0; kb < 2; kb++)
                    if (p.direct) tc::tma_load_4d(opl(pl) + kb * 16384 + 8192, &tmV, &bar[2], kb * 64, h, t0, b);
                    else tc::tma_load_3d(opl(pl) + kb * 16384 + 8192, &tmV, &bar[2], kb * 64, (int)vrow, pl);
    }
    {
        const int q = warp & 3, hc = warp >> 2;
        const int r = 32 * q + lane;
        uint32_t x[32];
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 32 * hc, x);
        tc::tmem_ld_wait();
        if (r < kC) {  // A_ti = beta_t e^{lt_t - lc_i} k_t.k_i (i < t)
            const int t = r;
            const float bt = sm.bt[t], lt = sm.lt[t];
            float4* dst = reinterpret_cast<float4*>(&sm.inv.a[t][32 * hc]);
#pragma unroll
            for (int c4 = 0; c4 < 8; c4++) {
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int i = 32 * hc + 4 * c4 + e;
                    v[e] = i < t ? bt * __expf(lt - sm.lc[i]) * __uint_as_float(x[4 * c4 + e]) : 0.f;
                }
                dst[c4] = make_float4(v[0], v[1], v[2], v[3]);
            }
        } else {  // M_ti = e^{lc_t - lc_i} q_t.k_i (i <= t), hi / lo planes
            const int t = r - kC;
            const float lct = sm.lc[t];
            __half* mhi = p.mh + (vrow + t) * kC + 32 * hc;
#pragma unroll
            for (int c8 = 0; c8 < 4; c8++) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int i = 32 * hc + 8 * c8 + e;
                    v[e] = i <= t ? __expf(lct - sm.lc[i]) * __uint_as_float(x[8 * c8 + e]) : 0.f;
                }
                put_hl8(mhi, p.m_plane, 8 * c8, v);
            }
        }
    }
    if (tid < kC) p.lcb[vrow + tid] = sm.lc[tid];
    __syncthreads();  // A complete
    // ---- T = (I + A)^{-1}, blocked by 16: the four diagonal blocks T_ii = (I + A_ii)^{-1} by forward
    // substitution (one column per thread), then the sub-diagonals d = 1, 2, 3 in turn:
    //   Z_ij = sum_{k=j}^{i-1} A_ik T_kj,  T_ij = -T_ii Z_ij   (i - j = d), 16 x 16 blocks ----
    if (tid < kC) {
        const int o = 16 * (tid >> 4), jj = tid & 15;
        float rsum[16], xv[16];
#pragma unroll
        for (int t = 0; t < 16; t++) rsum[t] = 0.f;
#pragma unroll
        for (int t = 0; t < 16; t++) {
            xv[t] = (t == jj ? 1.0f : 0.0f) - rsum[t];
#pragma unroll
            for (int u = t + 1; u < 16; u++) rsum[u] = fmaf(sm.inv.a[o + u][o + t], xv[t], rsum[u]);
        }
#pragma unroll
        for (int t = 0; t < 16; t++) sm.inv.tm[o + t][o + jj] = xv[t];
    } else {  // blocks above the diagonal are zero
        for (int e = tid - kC; e < 6 * 256; e += kChunkThreads - kC) {
            const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
            const int bi = blk < 3 ? 0 : blk < 5 ? 1 : 2, bj = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
            sm.inv.tm[16 * bi + r][16 * bj + c] = 0.f;
        }
    }
    __syncthreads();
    // d and the block index j unrolled: every trip count is a constant, so each thread's shared-memory
    // loads of a phase issue together instead of one dependent round trip per k-step
#pragma unroll
    for (int d = 1; d < 4; d++) {
        const int nb = 4 - d;  // blocks (j + d, j), j = 0 .. nb - 1
#pragma unroll
        for (int jb = 0; jb < nb; jb++) {
            const int e = jb * 256 + tid;
            const int j = e >> 8, i = j + d, r = (e >> 4) & 15, c = e & 15;
            const float* arow = &sm.inv.a[16 * i + r][16 * j];
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int k = 0; k < 16 * d; k += 4) {
                const float4 a4 = *reinterpret_cast<const float4*>(arow + k);
                s0 = fmaf(a4.x, sm.inv.tm[16 * j + k][16 * j + c], s0);
                s1 = fmaf(a4.y, sm.inv.tm[16 * j + k + 1][16 * j + c], s1);
                s0 = fmaf(a4.z, sm.inv.tm[16 * j + k + 2][16 * j + c], s0);
                s1 = fmaf(a4.w, sm.inv.tm[16 * j + k + 3][16 * j + c], s1);
            }
            sm.inv.z[j][r][c] = s0 + s1;
        }
        __syncthreads();
#pragma unroll
        for (int jb = 0; jb < nb; jb++) {
            const int e = jb * 256 + tid;
            const int j = e >> 8, i = j + d, r = (e >> 4) & 15, c = e & 15;
            const float* trow = &sm.inv.tm[16 * i + r][16 * i];
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int k = 0; k < 16; k += 4) {
                const float4 t4 = *reinterpret_cast<const float4*>(trow + k);
                s0 = fmaf(t4.x, sm.inv.z[j][k][c], s0);
                s1 = fmaf(t4.y, sm.inv.z[j][k + 1][c], s1);
                s0 = fmaf(t4.z, sm.inv.z[j][k + 2][c], s0);
                s1 = fmaf(t4.w, sm.inv.z[j][k + 3][c], s1);
            }
            sm.inv.tm[16 * i + r][16 * j + c] = -(s0 + s1);
        }
        __syncthreads();
    }
    const int j = tid >> 2, pt = tid & 3;  // column j, rows 4 m + pt of T into registers
    float xs[kC / 4];
#pragma unroll
    for (int m = 0; m < kC / 4; m++) xs[m] = sm.inv.tm[4 * m + pt][j];
    __syncthreads();  // A^T no longer read: its space becomes [T'; T'']
    {  // T' = T diag(beta e^{lt}) in rows 0-63, T'' = T diag(beta) in rows 64-127, column j
        const float fw = sm.bt[j] * expf(sm.lt[j]), fu = sm.bt[j];
#pragma unroll
        for (int m = 0; m < kC / 4; m++) {
            const int t = 4 * m + pt;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const float v = xs[m] * (half ? fu : fw);
                const int off = sw128_off(half * kC + t, j);
                if (BF) {  // hi / lo in bf16, the type of the K / V operands they meet
                    const __nv_bfloat16 hv = __float2bfloat16_rn(v);
                    *reinterpret_cast<__nv_bfloat16*>(&sm.t[0][off]) = hv;
                    *reinterpret_cast<__nv_bfloat16*>(&sm.t[1][off]) = __float2bfloat16_rn(v - __bfloat162float(hv));
                } else {
                    const __half hv = __float2half_rn(v);
                    *reinterpret_cast<__half*>(&sm.t[0][off]) = hv;
                    *reinterpret_cast<__half*>(&sm.t[1][off]) = __float2half_rn(v - __half2float(hv));
                }
            }
        }
    }
    tc::fence_proxy_async_smem();
    __syncthreads();  // [T'; T''] visible to the tensor core
    // ---- GEMM 2 in two N = 128 halves through TMEM columns [0, 128): [T'; T''] [K0 K1] (rows 0-63 are W),
    // then, once the W rows are read, [T'; T''] [V0 V1] (rows 64-127 are U) ----
    constexpr uint32_t id2 = BF ? tc::idesc_as_bf16(tc::idesc_f16_f32_bmn(128, 128)) : tc::idesc_f16_f32_bmn(128, 128);
    const bool b_lo = !p.qkv_exact;  // exact inputs: K and V have no lo plane (hi * lo vanishes)
    auto gemm2 = [&](uint32_t boff) {  // B = the two 64-column boxes at boff, boff + 16 KB of each plane
#pragma unroll
        for (int term = 0; term < 3; term++) {
            const uint32_t pa = at_ + (term == 1 ? kTPlane : 0), pb = (term == 2 ? aop_lo : aop) + boff;
            if (term < 2 || b_lo)
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                    tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(pa + ks * 32), tc::desc_sw128(pb + ks * 16 * 128, 16384, 1024),
                                   id2, (term | ks) != 0);
        }
    };
    if (tid == 0 && ok1) {
        if (tc::mbar_wait(&bar[2], 0, p.err, ANELM_ERR_TIMEOUT, abort)) {  // V landed too (read by the second half)
            tc::tc_fence_after();
            gemm2(0);
            tc::mma_commit(&bar[3]);
        }
    }
    const int q = warp & 3, hc = warp >> 2;  // hc: key / value dims [64 hc, 64 hc + 64)
    const int r = 32 * q + lane;
    const bool is_w = r < kC;                // warps of TMEM lanes 0-63: W; 64-127: U
    const int t = is_w ? r : r - kC;
    uint32_t xx[2][32];  // this thread's 64 values of W or U, both 32-column loads in flight before one wait
    const bool okw = tc::mbar_wait(&bar[3], 0, p.err, ANELM_ERR_TIMEOUT, abort);
    if (okw && is_w) {
        tc::tc_fence_after();
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64 * hc, xx[0]);
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64 * hc + 32, xx[1]);
        tc::tmem_ld_wait();
    }
    tc::tc_fence_before();
    __syncthreads();  // the W rows are read: the second half may overwrite the columns
    if (tid == 0 && okw) {
        tc::tc_fence_after();
        gemm2(8192);
        tc::mma_commit(&bar[4]);
    }
    const bool oku = okw && tc::mbar_wait(&bar[4], 0, p.err, ANELM_ERR_TIMEOUT, abort);
    if (oku) {
        tc::tc_fence_after();
        if (!is_w) {
            tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64 * hc, xx[0]);
            tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64 * hc + 32, xx[1]);
            tc::tmem_ld_wait();
        }
        // GEMM 2 is done with the operand buffer and [T'; T'']: W (hi / lo) is staged in the former as
        // four 64-column boxes (128-byte rows, 128B swizzle), U (fp32) in the latter as four 32-column
        // boxes, in the tiles' TMA layouts, and both are written by eight tile stores
#pragma unroll
        for (int h32 = 0; h32 < 2; h32++) {
            const uint32_t (&x)[32] = xx[h32];
            if (is_w) {
#pragma unroll
                for (int c8 = 0; c8 < 4; c8++) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = __uint_as_float(x[8 * c8 + e]);
                    uint4 whi, wlo;
                    split8<BF>(v, whi, wlo);
                    const int off = t * 128 + ((((4 * h32 + c8) ^ t) & 7) << 4);
                    *reinterpret_cast<uint4*>(&sm.op[hc * 8192 + off]) = whi;
                    *reinterpret_cast<uint4*>(&sm.op[16384 + hc * 8192 + off]) = wlo;
                }
            } else {
                uint8_t* ub = &sm.ustage[(2 * hc + h32) * 8192 + t * 128];
#pragma unroll
                for (int c4 = 0; c4 < 8; c4++)
                    *reinterpret_cast<float4*>(ub + (((c4 ^ t) & 7) << 4)) =
                        make_float4(__uint_as_float(x[4 * c4]), __uint_as_float(x[4 * c4 + 1]),
                                    __uint_as_float(x[4 * c4 + 2]), __uint_as_float(x[4 * c4 + 3]));
            }
        }
        tc::fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0 && oku && !*abort) {
#pragma unroll
        for (int pl = 0; pl < (p.qkv_exact ? 1 : 2); pl++)  // exact inputs: the chain reads W hi only
#pragma unroll
            for (int kb = 0; kb < 2; kb++) tc::tma_store_3d(&tmW, &sm.op[pl * 16384 + kb * 8192], 64 * kb, (int)vrow, pl);
#pragma unroll
        for (int bx = 0; bx < 4; bx++) tc::tma_store_2d(&tmU, &sm.ustage[bx * 8192], 32 * bx, (int)vrow);
        tc::bulk_commit_group();
        tc::bulk_wait_group_read0();  // the shared-memory sources stay valid until the copies read them
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) {  // nothing of this CTA's may still be in flight when its TMEM is released
            for (int i = 0; i < 5; i++)
                for (uint32_t n = 0; n < tc::kWaitPolls && !tc::mbar_try_wait(&bar[i], 0); n++) {
                    if (i == 2 && !ok1) break;  // V was never requested
                    if ((i == 1 || i >= 3) && *abort) break;
                }
        }
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kChunkTmemCols);
    }
}

// ---------------------------------------------------------------- the recurrence on tcgen05

// A chunk's operand tiles, fetched by TMA tile copies (64 rows x 128 bytes, 128B swizzle): W, Q, K
// and M hi / lo planes, U (fp32, 32-column boxes)
struct ChainMaps {
    CUtensorMap w, q, k, m, u;
};

// One CTA per (sequence, value head, NB state columns); the three products of a chunk step run on
// the tensor core with fp32 accumulators in TMEM (hi / lo operand planes, three MMAs per product as
// above, two where one side is an exact 16-bit input):
//   A:  [Q; W] S        M 128 (64 Q rows over 64 W rows), N NB, K 128   -> Q S and W S
//   C:  K^T (Gamma D)   M 128 (key dims), N NB, K 64 (tokens)            -> the state update
//   B:  M D             M 128 (64 M rows, 64 zero rows), N NB, K 64      -> the intra-chunk output
// with D = U - W S and Gamma = diag(e^{lc_C - lc}).  Warp roles (a warp reads the TMEM lanes of its
// index mod 4, 32 each):
//   0-7         state: thread (lane quadrant q, half hf) holds S[32 q + lane][NB/2 hf .. + NB/2] in
//               registers and, once C is done, applies S = e^{lc_C} S + K^T Gamma D and writes its
//               part of the next S operand;
//   10, 11, 14, 15  D = U - W S and Gamma D from the W S rows (lanes 64-127), NB/2 columns each;
//   8, 9        Y = e^{lc} Q S + M D from lanes 0-63, stored to global;
//   12          issues the MMAs; 13: issues the TMA loads of the next chunk as soon as the tensor
//               core or the D warps are done with a buffer (both run converged and elect one lane
//               for each tcgen05 / TMA instruction).
// A step's critical path is A -> D -> C -> S; B is issued after C and runs while the state warps
// work, and the outputs follow it (the A / B accumulators and D are double-buffered, so the output
// warps may lag a step).  Every hand-over is an mbarrier (thread arrivals or tcgen05.commit), every
// wait bounded.  A traced step spends about as long in the epilogues as in the MMAs
// (~47 cycles per M=128 MMA issued, for N = 32 or 64), so narrow column blocks on many SMs pay:
// NB 32 gives 4 x 32 x B CTAs.
constexpr int kChainTcThreads = 512;
template <int NB>
struct ChainTcSmem {
    static constexpr int kRowB = NB * 2;  // bytes of one fp16 row of an N = NB operand
    uint8_t qw[2][32768];          // [Q; W] hi, lo: per key-dim box of 64 (16 KB) 64 Q rows, then 64 W rows
    uint8_t m[2][16384];           // M hi, lo as a 128-row K-major A: rows 64-127 stay zero
    uint8_t k[2][16384];           // K[t][d] hi, lo: two 8 KB key-dim boxes (MN-major A of the update)
    uint8_t s[2][kDk * kRowB];     // S[d][j] hi, lo: swizzled rows of NB fp16 (MN-major B)
    uint8_t d[2][2][kC * kRowB];   // D[t][j] hi, lo (MN-major B of M D), by chunk parity
    uint8_t gd[2][kC * kRowB];     // (Gamma D)[t][j] hi, lo (MN-major B of the update)
    uint8_t u[kC * NB * 4];        // U[t][j0 .. j0 + NB] fp32 in 32-column 128B-swizzled boxes
    float lc[4][kC];               // in-chunk cumulative log decay, ring by chunk index
    // one phase per chunk each: 0 S written (256 arrivals) and [Q; W] landed, 1 A done and U + lc
    // landed, 2 D written (128 arrivals) and K landed, 3 C done, 4-5 B done (by accumulator buffer),
    // 6-7 Y read (by buffer, 64 arrivals), 8 all MMAs done, 9 M landed
    uint64_t bar[10];
    uint32_t tmem_slot;
    int abort;
};

// Operands with rows of NB fp16 (K index = row, N = column, N contiguous): 128-byte rows with the
// 128-byte swizzle (NB 64: 16-byte word c of row r at ((c ^ r) & 7)) or 64-byte rows with the
// 64-byte swizzle (NB 32: word c at ((c ^ (r >> 1)) & 3)); 8-row groups of 8 NB * 2 bytes.
template <int NB>
__device__ __forceinline__ uint32_t nb_word(int r, int c) {
    if (NB == 64) return (uint32_t)(r * 128 + (((c ^ r) & 7) << 4));
    return (uint32_t)(r * 64 + (((c ^ (r >> 1)) & 3) << 4));
}
// MN-major operand descriptor of such a tile (one N atom, so the leading offset is unused)
template <int NB>
__device__ __forceinline__ uint64_t nb_desc(uint32_t smem_addr) {
    uint64_t d = (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                           // LBO (unused: one atom along N)
    d |= (uint64_t)((8 * NB * 2) >> 4) << 32;         // SBO: 8 rows
    d |= (uint64_t)1 << 46;                           // descriptor version (sm100)
    d |= (uint64_t)(NB == 64 ? 2 : 4) << 61;          // SWIZZLE_128B / SWIZZLE_64B
    return d;
}
// 16 consecutive fp32 columns of U[t][..] from its 32-column 128B-swizzled boxes
__device__ __forceinline__ void u_row16(const uint8_t* u, int t, int j, float (&x)[16]) {
    const uint8_t* row = u + (j >> 5) * 8192 + t * 128;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float4 v = *reinterpret_cast<const float4*>(row + ((((((j & 31) >> 2) + q) ^ t) & 7) << 4));
        x[4 * q] = v.x;
        x[4 * q + 1] = v.y;
        x[4 * q + 2] = v.z;
        x[4 * q + 3] = v.w;
    }
}

template <int NB, bool BF>
__global__ void __launch_bounds__(kChainTcThreads, 1) gdn_pf_chain_tc_kernel(const __grid_constant__ ChainMaps mp,
                                                                             const GdnPrefillParams p) {
    static_assert(NB == 32 || NB == 64, "operand rows of 64 or 128 bytes");
    extern __shared__ uint8_t smem_raw[];
    using Smem = ChainTcSmem<NB>;
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int nblk = kDv / NB;
    constexpr int kRowB = Smem::kRowB, kSPlane = kDk * kRowB, kDPlane = kC * kRowB;
    constexpr int kHalf = NB / 2;               // columns per state / D thread
    constexpr uint32_t kTmemCols = NB == 64 ? 512 : 256;
    const int h = blockIdx.x / nblk, j0 = (blockIdx.x % nblk) * NB, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kh = h / (p.Hv / p.Hk);
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    float* S = p.state + ((long long)seq * p.Hv + h) * kDk * kDv;
    const int nC = p.T_pad / kC;
    const int krow0 = (int)(((long long)b * p.Hk + kh) * p.T_pad);
    const int vrow0 = (int)(((long long)b * p.Hv + h) * p.T_pad);
    const bool exact = p.qkv_exact != 0;
    uint64_t* bar = sm.bar;
    volatile int* abort = &sm.abort;
    if (tid == 0) {
        sm.abort = 0;
        const uint32_t count[10] = {257, 2, 129, 1, 1, 1, 64, 64, 1, 1};
        for (int i = 0; i < 10; i++) tc::mbar_init(&bar[i], count[i]);
        tc::fence_barrier_init();
    }
    {  // zero rows of the A tiles that no load fills: M rows 64-127
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        for (int i = tid; i < 2 * 512; i += kChainTcThreads)
            *reinterpret_cast<uint4*>(&sm.m[i >> 9][8192 + (i & 511) * 16]) = z;
    }
    if (warp == 12) {
        tc::tmem_alloc(&sm.tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    // TMEM columns: A accumulators [0, 2 NB) by buffer, B accumulators [2 NB, 4 NB), C at 4 NB
    constexpr uint32_t kColB = 2 * NB, kColC = 4 * NB;
    static_assert(5 * NB <= kTmemCols, "TMEM columns");
    int* const err = p.err;
    auto wait = [=](int i, uint32_t parity) { return tc::mbar_wait(&bar[i], parity, err, ANELM_ERR_TIMEOUT, abort); };
    // the same for the converged issuing warps: every lane polls (the lanes see the same barrier and
    // stay converged), one plain bounded loop.  Measured on cfg 4: polling in lane 0 alone with the
    // other lanes parked at a shuffle 1.03 ms per call; every lane through the shared bounded wait
    // and a shuffle 0.600 ms; this loop 0.587 ms.
    auto wait_w = [=](int i, uint32_t parity) {
        for (uint32_t n = 0; n < tc::kWaitPolls; n++) {
            if (tc::mbar_try_wait(&bar[i], parity)) return true;
            if ((n & 1023) == 1023 && *abort) return false;
        }
        *abort = 1;
        if (err) atomicCAS(err, 0, ANELM_ERR_TIMEOUT);
        return false;
    };

    if (warp == 13) {
        // ---------------------------------------------------------------- TMA loads
        int loaded[4] = {0, 0, 0, 0};  // chunks whose loads are issued on bars 0-2 and 9 (one phase each)
        auto load_qw = [&](int ci) {
            if (tc::elect_one()) {
                // exact inputs: the hi plane alone (A drops its [Q; W] lo term, below)
                tc::mbar_arrive_expect_tx(&bar[0], (exact ? 2 : 4) * 2 * 8192);
                for (int pl = 0; pl < (exact ? 1 : 2); pl++)
                    for (int kb = 0; kb < 2; kb++) {
                        tc::tma_load_3d(&sm.qw[pl][kb * 16384 + 8192], &mp.w, &bar[0], 64 * kb, vrow0 + ci * kC, pl);
                        if (p.direct)  // the caller's token-major q: [b][token][head][d]
                            tc::tma_load_4d(&sm.qw[pl][kb * 16384], &mp.q, &bar[0], 64 * kb, kh, ci * kC, b);
                        else
                            tc::tma_load_3d(&sm.qw[pl][kb * 16384], &mp.q, &bar[0], 64 * kb, krow0 + ci * kC, pl);
                    }
            }
            loaded[0] = ci + 1;
        };
        auto load_u = [&](int ci) {
            if (tc::elect_one()) {
                tc::mbar_arrive_expect_tx(&bar[1], kC * NB * 4 + kC * 4);
                for (int c32 = 0; c32 < NB / 32; c32++)
                    tc::tma_load_2d(&sm.u[c32 * 8192], &mp.u, &bar[1], j0 + 32 * c32, vrow0 + ci * kC);
                tc::bulk_load(sm.lc[ci & 3], p.lcb + vrow0 + (long long)ci * kC, kC * 4, &bar[1]);
            }
            loaded[1] = ci + 1;
        };
        auto load_k = [&](int ci) {
            if (tc::elect_one()) {
                tc::mbar_arrive_expect_tx(&bar[2], (exact ? 1 : 2) * 2 * 8192);
                for (int pl = 0; pl < (exact ? 1 : 2); pl++)
                    for (int kb = 0; kb < 2; kb++)
                        if (p.direct) tc::tma_load_4d(&sm.k[pl][kb * 8192], &mp.k, &bar[2], 64 * kb, kh, ci * kC, b);
                        else tc::tma_load_3d(&sm.k[pl][kb * 8192], &mp.k, &bar[2], 64 * kb, krow0 + ci * kC, pl);
            }
            loaded[2] = ci + 1;
        };
        auto load_m = [&](int ci) {
            if (tc::elect_one()) {
                tc::mbar_arrive_expect_tx(&bar[9], 2 * 8192);
                for (int pl = 0; pl < 2; pl++) tc::tma_load_3d(&sm.m[pl][0], &mp.m, &bar[9], 0, vrow0 + ci * kC, pl);
            }
            loaded[3] = ci + 1;
        };
        if (nC > 0) {
            if (tc::elect_one()) {
                tc::prefetch_tmap(&mp.w);
                tc::prefetch_tmap(&mp.q);
                tc::prefetch_tmap(&mp.k);
                tc::prefetch_tmap(&mp.m);
                tc::prefetch_tmap(&mp.u);
            }
            load_qw(0);
            load_u(0);
            load_k(0);
            load_m(0);
            // each buffer is refilled once its readers of chunk ci are done; none of these barriers can
            // run a phase ahead of this warp, since their next phase needs the load issued here
            for (int ci = 0; ci + 1 < nC; ci++) {
                if (!wait_w(1, ci & 1)) break;  // A read [Q; W]
                load_qw(ci + 1);
                if (!wait_w(2, ci & 1)) break;  // the D warps read U and lc
                load_u(ci + 1);
                if (!wait_w(3, ci & 1)) break;  // C read K
                load_k(ci + 1);
                if (!wait_w(4 + (ci & 1), (ci >> 1) & 1)) break;  // B read M
                load_m(ci + 1);
            }
            // nothing may still be in flight when the CTA leaves; a load is issued only once the
            // previous phase of its barrier has completed, so waiting for the parity of the last one
            // is exact (after an abort the phase may never complete: the wait is bounded)
            if (lane == 0)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    for (uint32_t n = 0; n < tc::kWaitPolls && !tc::mbar_try_wait(&bar[i < 3 ? i : 9], (loaded[i] - 1) & 1);
                         n++) {
                    }
        }
        __syncwarp();
    } else if (warp == 12) {
        // ---------------------------------------------------------------- MMAs
        // A and C meet q / k: their operands are bf16 when those are (BF); B (M D) stays fp16
        constexpr uint32_t idB = tc::idesc_f16_f32_bmn(128, NB);
        constexpr uint32_t idA = BF ? tc::idesc_as_bf16(idB) : idB;
        constexpr uint32_t idC = idA | (1u << 15);  // A (K^T) MN-major too
        // descriptors of the tiles' first bytes; later k-steps add their byte offset >> 4 to the
        // start-address field (shared-memory addresses stay below 2^18, so it never carries out)
        const uint64_t dqw = tc::desc_kmajor_sw128(smem_u32(sm.qw)), dm = tc::desc_kmajor_sw128(smem_u32(sm.m));
        const uint64_t dk = tc::desc_sw128(smem_u32(sm.k), 8192, 1024);
        const uint64_t ds = nb_desc<NB>(smem_u32(sm.s)), dd = nb_desc<NB>(smem_u32(sm.d));
        const uint64_t dgd = nb_desc<NB>(smem_u32(sm.gd));
        // B of chunk c: M D -> columns [2 NB + NB (c & 1), ...), D from its parity buffer
        auto issue_b = [&](int c) {
            const uint32_t cb = c & 1;
            if (!wait_w(9, c & 1)) return false;  // M of chunk c landed
            tc::tc_fence_after();
#pragma unroll
            for (int term = 0; term < 3; term++)
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                    if (tc::elect_one())
                        tc::mma_f16_ss(tmem + kColB + NB * cb, dm + (((term == 1 ? 16384 : 0) + ks * 32) >> 4),
                                       dd + ((cb * 2 * kDPlane + (term == 2 ? kDPlane : 0) + ks * 16 * kRowB) >> 4), idB,
                                       (term | ks) != 0);
            if (tc::elect_one()) tc::mma_commit(&bar[4 + cb]);
            return true;
        };
        for (int ci = 0; ci < nC; ci++) {
            const uint32_t ph = ci & 1, bb = ci & 1;
            if (!wait_w(0, ph)) break;  // S of this step written, [Q; W] landed
            if (ci >= 2 && !wait_w(6 + bb, ((ci >> 1) + 1) & 1)) break;  // outputs of step ci - 2 read
            tc::tc_fence_after();
            // A: [Q; W] S -> columns [NB bb, NB bb + NB).  Exact inputs: Q has no lo plane, and W enters
            // by its hi plane alone (16 MMAs instead of 24 on the step's critical path); over 128 chunk
            // steps that moves y and the state by ~2e-6 (fp16) / ~2e-5 (bf16), 1 % of the tolerance
#pragma unroll
            for (int term = 0; term < 3; term++) {
                if (term == 1 && exact) continue;
#pragma unroll
                for (int kb = 0; kb < 2; kb++)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        if (tc::elect_one())
                            tc::mma_f16_ss(tmem + NB * bb, dqw + (((term == 1 ? 32768 : 0) + kb * 16384 + ks * 32) >> 4),
                                           ds + (((term == 2 ? kSPlane : 0) + (kb * 4 + ks) * 16 * kRowB) >> 4), idA,
                                           (term | kb | ks) != 0);
            }
            if (tc::elect_one()) tc::mma_commit(&bar[1]);
            if (!wait_w(2, ph)) break;  // D, Gamma D written; K landed
            tc::tc_fence_after();
            // C: K^T (Gamma D) -> columns [4 NB, 5 NB)
#pragma unroll
            for (int term = 0; term < 3; term++) {
                if (term == 2 && exact) break;  // K exact: no K lo plane
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                    if (tc::elect_one())
                        tc::mma_f16_ss(tmem + kColC, dk + (((term == 2 ? 16384 : 0) + ks * 2048) >> 4),
                                       dgd + (((term == 1 ? kDPlane : 0) + ks * 16 * kRowB) >> 4), idC, (term | ks) != 0);
            }
            if (tc::elect_one()) tc::mma_commit(&bar[3]);
            if (!issue_b(ci)) break;  // overlaps the state warps' epilogue
        }
        // one commit tracks every MMA issued above: none may run once TMEM is released
        if (tc::elect_one()) tc::mma_commit(&bar[8]);
        if (lane == 0)
            for (uint32_t n = 0; n < tc::kWaitPolls && !tc::mbar_try_wait(&bar[8], 0); n++) {
            }
        __syncwarp();
    } else if (warp < 8) {
        // ---------------------------------------------------------------- state: S[i][j0 + kHalf hf ..]
        const int i = 32 * (warp & 3) + lane, hf = warp >> 2;
        float s[kHalf];
        const float4* src = reinterpret_cast<const float4*>(S + (long long)i * kDv + j0 + kHalf * hf);
#pragma unroll
        for (int c4 = 0; c4 < kHalf / 4; c4++) {
            const float4 v = src[c4];
            s[4 * c4] = v.x;
            s[4 * c4 + 1] = v.y;
            s[4 * c4 + 2] = v.z;
            s[4 * c4 + 3] = v.w;
        }
        auto write_s = [&]() {  // row i, this thread's columns of the S operand, hi / lo
#pragma unroll
            for (int c = 0; c < kHalf / 8; c++) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = s[8 * c + e];
                uint4 hi, lo;
                split8<BF>(v, hi, lo);  // S meets [Q; W] in A
                const uint32_t o = nb_word<NB>(i, hf * (kHalf / 8) + c);
                *reinterpret_cast<uint4*>(&sm.s[0][o]) = hi;
                *reinterpret_cast<uint4*>(&sm.s[1][o]) = lo;
            }
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&bar[0]);
        };
        if (nC > 0) write_s();
        for (int ci = 0; ci < nC; ci++) {
            if (!wait(3, ci & 1)) break;
            tc::tc_fence_after();
            const float gC = expf(sm.lc[ci & 3][kC - 1]);
#pragma unroll
            for (int q = 0; q < kHalf / 16; q++) {
                uint32_t x[16];
                tc::tmem_ld16(tmem + lane_base + kColC + kHalf * hf + 16 * q, x);
                tc::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; j++) s[16 * q + j] = fmaf(gC, s[16 * q + j], __uint_as_float(x[j]));
            }
            tc::tc_fence_before();
            if (ci + 1 < nC) write_s();
        }
        float4* dst = reinterpret_cast<float4*>(S + (long long)i * kDv + j0 + kHalf * hf);
#pragma unroll
        for (int c4 = 0; c4 < kHalf / 4; c4++)
            dst[c4] = make_float4(s[4 * c4], s[4 * c4 + 1], s[4 * c4 + 2], s[4 * c4 + 3]);
    } else if ((warp & 3) >= 2) {
        // ---------------------------------------------------------------- D = U - W S, Gamma D
        const int t = 32 * ((warp & 3) - 2) + lane;  // token row of the chunk; TMEM lane 64 + t
        const int hf = warp >= 14;                    // columns kHalf hf .. + kHalf
        for (int ci = 0; ci < nC; ci++) {
            const uint32_t bb = ci & 1;
            if (!wait(1, ci & 1)) break;  // A done, U and lc landed
            tc::tc_fence_after();
            const float* lc = sm.lc[ci & 3];
            const float gam = expf(lc[kC - 1] - lc[t]);
#pragma unroll
            for (int q = 0; q < kHalf / 16; q++) {
                uint32_t x[16];
                tc::tmem_ld16(tmem + lane_base + NB * bb + kHalf * hf + 16 * q, x);
                float u[16];
                u_row16(sm.u, t, kHalf * hf + 16 * q, u);
                tc::tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = u[8 * c + e] - __uint_as_float(x[8 * c + e]);
                    uint4 hi, lo;
                    split8(v, hi, lo);
                    const uint32_t o = nb_word<NB>(t, (kHalf * hf + 16 * q) / 8 + c);
                    *reinterpret_cast<uint4*>(&sm.d[bb][0][o]) = hi;
                    *reinterpret_cast<uint4*>(&sm.d[bb][1][o]) = lo;
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] *= gam;
                    split8<BF>(v, hi, lo);  // Gamma D meets K in C; D (for B) stays fp16
                    *reinterpret_cast<uint4*>(&sm.gd[0][o]) = hi;
                    *reinterpret_cast<uint4*>(&sm.gd[1][o]) = lo;
                }
            }
            tc::fence_proxy_async_smem();
            tc::tc_fence_before();
            tc::mbar_arrive(&bar[2]);
        }
    } else {
        // ---------------------------------------------------------------- Y = e^{lc} Q S + M D
        const int t = 32 * (warp & 3) + lane;  // token row of the chunk; TMEM lane t
        const bool vec = p.y_vec != 0;
        for (int ci = 0; ci < nC; ci++) {
            const uint32_t bb = ci & 1;
            if (!wait(4 + bb, (ci >> 1) & 1)) break;
            tc::tc_fence_after();
            const float eg = expf(sm.lc[ci & 3][t]);
            const int tok = ci * kC + t;
            const long long o = ((long long)b * p.n + tok) * p.y_stride + (long long)h * kDv + j0;
#pragma unroll
            for (int q = 0; q < NB / 16; q++) {  // 16 columns at a time
                uint32_t qs[16], md[16];
                tc::tmem_ld16(tmem + lane_base + NB * bb + 16 * q, qs);
                tc::tmem_ld16(tmem + lane_base + kColB + NB * bb + 16 * q, md);
                tc::tmem_ld_wait();
                if (tok >= p.n) continue;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = fmaf(eg, __uint_as_float(qs[8 * c + e]), __uint_as_float(md[8 * c + e]));
                    const long long oc = o + 16 * q + 8 * c;
                    if (!vec) {
#pragma unroll
                        for (int e = 0; e < 8; e++) store_from_float(p.y, p.y_dtype, oc + e, v[e]);
                    } else if (p.y_dtype == ANELM_F32) {
                        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.y) + oc);
                        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
                    } else {
                        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.y) + oc) = pack8(v, p.y_dtype == ANELM_BF16);
                    }
                }
            }
            // the accumulators and this step's lc slot are read: release them
            tc::tc_fence_before();
            tc::mbar_arrive(&bar[6 + bb]);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 12) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
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

// 3D fp16 tensor map over the hi / lo planes of a [rows][cols] operand: box {64, 64, 1}, 128B swizzle
static bool make_plane_map(CUtensorMap* m, const __half* base, uint64_t rows, long long plane, uint64_t cols = 128) {
    auto fn = tc::tmap_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {cols, rows, 2};
    cuuint64_t strides[2] = {cols * 2, (cuuint64_t)plane * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)kC, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4D map over the caller's token-major 16-bit [B][n][heads][128] q, k or v: box {64 d, 1 head, 64 tokens,
// 1 sequence}, 128B swizzle (the same tile as a plane box); tokens past n read as zeros
static bool make_direct_map(CUtensorMap* m, const void* base, int dtype, uint64_t heads, uint64_t n, uint64_t B) {
    auto fn = tc::tmap_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {128, heads, n, B};
    cuuint64_t strides[3] = {256, heads * 256, n * heads * 256};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)kC, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, dtype == ANELM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int launch_chunks_and_chain(const GdnPrefillParams& p, cudaStream_t stream) {
    const int nC = p.T_pad / kC;
    const size_t chunk_smem = chunk_smem_bytes(p.qkv_exact != 0);
    const uint64_t krows = (uint64_t)p.B * p.Hk * p.T_pad, vrows = (uint64_t)p.B * p.Hv * p.T_pad;
    CUtensorMap mK, mQ, mV;
    ChainMaps cm;
    if (p.direct) {
        if (!make_direct_map(&mK, p.k_in, p.in_dtype, p.Hk, p.n, p.B) ||
            !make_direct_map(&mQ, p.q_in, p.in_dtype, p.Hk, p.n, p.B) ||
            !make_direct_map(&mV, p.v_in, p.in_dtype, p.Hv, p.n, p.B))
            return ANELM_ERR_CUDA;
    } else if (!make_plane_map(&mK, p.kh, krows, p.q_plane) || !make_plane_map(&mQ, p.qh, krows, p.q_plane) ||
               !make_plane_map(&mV, p.vh, vrows, p.v_plane)) {
        return ANELM_ERR_CUDA;
    }
    cm.k = mK;
    cm.q = mQ;
    {  // W (hi / lo like V), M (64 columns), U (fp32, 32-column boxes of this block's state columns)
        auto fn = tc::tmap_encode_fn();
        cuuint64_t dims[2] = {(cuuint64_t)kDv, vrows};
        cuuint64_t strides[1] = {(cuuint64_t)kDv * 4};
        cuuint32_t box[2] = {(cuuint32_t)kUBox, (cuuint32_t)kC};
        cuuint32_t estr[2] = {1, 1};
        if (!make_plane_map(&cm.w, p.wh, vrows, p.v_plane) || !make_plane_map(&cm.m, p.mh, vrows, p.m_plane, kC) ||
            fn(&cm.u, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.Ub, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return ANELM_ERR_CUDA;
    }
    constexpr int NB = 32;
    const size_t chain_smem = sizeof(ChainTcSmem<NB>) + 1024;
    const dim3 chunk_grid(nC, p.Hv, p.B), chain_grid(p.Hv * (kDv / NB), p.B);
    if (p.direct && p.op_bf16) {  // bf16 inputs read in place: the operands that meet them are bf16 too
        cudaFuncSetAttribute(gdn_pf_chunk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chunk_smem_bytes(false));
        gdn_pf_chunk_kernel<true><<<chunk_grid, kChunkThreads, chunk_smem, stream>>>(mK, mQ, mV, cm.w, cm.u, p);
        cudaFuncSetAttribute(gdn_pf_chain_tc_kernel<NB, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chain_smem);
        gdn_pf_chain_tc_kernel<NB, true><<<chain_grid, kChainTcThreads, chain_smem, stream>>>(cm, p);
    } else {
        cudaFuncSetAttribute(gdn_pf_chunk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chunk_smem_bytes(false));
        gdn_pf_chunk_kernel<false><<<chunk_grid, kChunkThreads, chunk_smem, stream>>>(mK, mQ, mV, cm.w, cm.u, p);
        cudaFuncSetAttribute(gdn_pf_chain_tc_kernel<NB, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)chain_smem);
        gdn_pf_chain_tc_kernel<NB, false><<<chain_grid, kChainTcThreads, chain_smem, stream>>>(cm, p);
    }
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

int launch_gdn_prefill(GdnPrefillParams p, void* workspace, cudaStream_t stream) {
    if (p.dk != kDk || p.dv != kDv || p.Hv % p.Hk) return ANELM_ERR_UNSUPPORTED;
    p.T_pad = (p.n + kC - 1) / kC * kC;
    carve(p, workspace, true);
    p.qkv_exact = 0;  // q, k, v come out of the conv / SiLU / L2 norm in fp32: both planes carry them
    p.direct = 0;
    p.op_bf16 = 0;
    p.y_dtype = ANELM_F32;
    p.y_stride = (long long)p.Hv * kDv;
    p.y_vec = 1;      // workspace rows: 256-byte aligned base, 16-byte aligned rows
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
    // 16-bit inputs are exact in fp16 (bf16 normal values have 8 significant bits): lo planes are zero
    p.qkv_exact = p.in_dtype == ANELM_F16 || p.in_dtype == ANELM_BF16;
    p.y_vec = (uintptr_t)p.y % 16 == 0 && p.y_stride % 8 == 0;  // 16-byte stores of 8 outputs
    // 16-bit inputs on 16-byte boundaries are read in place by TMA (no pack); their products then use
    // their own type (bf16 inputs: bf16 hi / lo partners, 16 significant bits)
    p.direct = p.qkv_exact && p.in_vec;
    p.op_bf16 = p.direct && p.in_dtype == ANELM_BF16;
    if (!p.direct) gdn_pf_pack_kernel<<<dim3(p.T_pad, p.B), 256, 0, stream>>>(p);
    return launch_chunks_and_chain(p, stream);
}

}  // namespace anelm
