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
// plane followed by a lo plane and reach the MMAs through ldmatrix.  When the bare core op gets
// 16-bit q / k / v (bf16 values have 8 significant bits, so they are exact in fp16), their lo
// planes are zero: they are neither written nor loaded, K K^T / Q K^T take one term, and the
// products with K, Q or V on one side take two.
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
#include "tc100.cuh"

namespace anelm {

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kDk = 128;   // key head dim of these kernels
constexpr int kDv = 128;   // value head dim
constexpr int kDvb = 32;   // state columns per chain CTA

// ---------------------------------------------------------------- fragments (mma.sync m16n8k16)

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float x) {
    const __half h = __float2half_rn(x);
    *hi = h;
    *lo = __float2half_rn(x - __half2float(h));
}

// B (16 x 8) fragments of two n-tiles n0, n0 + 8 at k0 (ldmatrix), with B[k][n] = T[n][k] (ldb2_sw)
// or B[k][n] = T[k][n] (ldb2_t_sw) for a tile T in shared memory.
// Tiles are in the TMA's 128B-swizzled layout of 64-column boxes: element (row, col) of a tile at shared
// address `tile` lives in box col / 64, 8192 bytes per box of 64 rows.
__device__ __forceinline__ uint32_t sw_addr(uint32_t tile, int row, int col) {
    return tile + (uint32_t)((col >> 6) * 8192 + row * 128 + ((((col & 63) >> 3) ^ row) & 7) * 16 + (col & 7) * 2);
}
__device__ __forceinline__ void ldb2_sw(uint32_t (&b)[4], uint32_t tile, int n0, int k0, int lane) {
    const int mat = lane >> 3, i = lane & 7;
    ldmatrix_x4(sw_addr(tile, n0 + i + (mat >> 1) * 8, k0 + (mat & 1) * 8), b[0], b[1], b[2], b[3]);
}
__device__ __forceinline__ void ldb2_t_sw(uint32_t (&b)[4], uint32_t tile, int n0, int k0, int lane) {
    const int mat = lane >> 3, i = lane & 7;
    ldmatrix_x4_trans(sw_addr(tile, k0 + i + (mat & 1) * 8, n0 + (mat >> 1) * 8), b[0], b[1], b[2], b[3]);
}
// Named barrier over `count` threads (a multiple of 32) of this CTA: wait, or arrive without waiting.
__device__ __forceinline__ void named_bar_sync_cta(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive_cta(uint32_t id, uint32_t count) {
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(count) : "memory");
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
//   GEMM 2  [T'; T''] [K | V]  (M 128, N 256, K 64) with T' = T diag(beta e^{lt}), T'' = T diag(beta):
//           its diagonal blocks are W = T' K and U = T'' V (the off-diagonal ones are not used).
// The operand buffer of each plane is [K d0-63 | Q d0-63 | K d64-127 | Q d64-127] (8 KB boxes of
// 64 rows x 128 bytes): read as the K-major A of GEMM 1 (two 16 KB boxes of 128 rows), as its
// K-major B (the K rows), and, once V has replaced Q, as the MN-major B of GEMM 2 (N boxes K0, V0,
// K1, V1, 8 KB apart).  T = (I + A)^{-1} by forward substitution on the CUDA cores in between.
constexpr int kChunkThreads = 256;
constexpr int kOpPlane = 32768;            // bytes of one plane of the operand buffer
constexpr int kTPlane = 16384;             // bytes of one plane of [T'; T''] (128 rows x 128 bytes)
constexpr int kTs = kC + 4;                // fp32 pitch of A and T in the inversion
constexpr uint32_t kChunkTmemCols = 256;
struct ChunkSmem {
    uint8_t op[2][kOpPlane];               // hi, lo planes (1024-byte aligned)
    union {
        uint8_t t[2][kTPlane];             // [T'; T''] hi, lo (K-major, 128-byte swizzle)
        struct {
            float a[kC][kTs];              // A (strictly lower)
            float tm[kC][kTs];             // T = (I + A)^{-1}
            float z[3][16][17];            // block products of one level
        } inv;
    };
    float lc[kC], lt[kC], bt[kC];
    uint64_t bar[4];                       // K+Q loaded, GEMM 1 done, V loaded, GEMM 2 done
    uint32_t tmem_slot;
    int abort;
};


// byte offset of element (row, col) (fp16, 64 columns per 128-byte row) in a 128B-swizzled tile
__device__ __forceinline__ int sw128_off(int row, int col) {
    return row * 128 + ((((col >> 3) ^ row) & 7) << 4) + (col & 7) * 2;
}

__global__ void __launch_bounds__(kChunkThreads) gdn_pf_chunk_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                      const __grid_constant__ CUtensorMap tmQ,
                                                                      const __grid_constant__ CUtensorMap tmV,
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
        for (int i = 0; i < 4; i++) tc::mbar_init(&bar[i], 1);
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
    const uint32_t aop = (uint32_t)__cvta_generic_to_shared(&sm.op[0][0]);
    const uint32_t at_ = (uint32_t)__cvta_generic_to_shared(&sm.t[0][0]);
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
                    tc::tma_load_3d(&sm.op[pl][kb * 16384], &tmK, &bar[0], kb * 64, (int)krow, pl);
                    tc::tma_load_3d(&sm.op[pl][kb * 16384 + 8192], &tmQ, &bar[0], kb * 64, (int)krow, pl);
                }
    }
    if (warp == 1) {  // inclusive prefix sum of log g over the chunk (two tokens per lane)
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
    if (tid == 0) {  // GEMM 1: [K; Q] K^T -> TMEM columns [0, 64)
        if (tc::mbar_wait(&bar[0], 0, p.err, ANELM_ERR_TIMEOUT, abort)) {
            tc::tc_fence_after();
            constexpr uint32_t id1 = tc::idesc_f16_f32(128, kC);
            // exact inputs: K and Q are exact in fp16, so hi * hi is the whole product
            const bool lo_terms = !p.qkv_exact;
#pragma unroll
            for (int term = 0; term < 3; term++) {
                const uint32_t pa = aop + (term == 1 ? kOpPlane : 0), pb = aop + (term == 2 ? kOpPlane : 0);
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
                    tc::tma_load_3d(&sm.op[pl][kb * 16384 + 8192], &tmV, &bar[2], kb * 64, (int)vrow, pl);
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
                const __half hv = __float2half_rn(v);
                const int off = sw128_off(half * kC + t, j);
                *reinterpret_cast<__half*>(&sm.t[0][off]) = hv;
                *reinterpret_cast<__half*>(&sm.t[1][off]) = __float2half_rn(v - __half2float(hv));
            }
        }
    }
    tc::fence_proxy_async_smem();
    __syncthreads();  // [T'; T''] visible to the tensor core
    if (tid == 0 && ok1) {  // GEMM 2: [T'; T''] [K0 V0 K1 V1] -> TMEM columns [0, 256)
        if (tc::mbar_wait(&bar[2], 0, p.err, ANELM_ERR_TIMEOUT, abort)) {
            tc::tc_fence_after();
            constexpr uint32_t id2 = tc::idesc_f16_f32_bmn(128, 256);
            const bool b_lo = !p.qkv_exact;  // exact inputs: K and V have no lo plane (hi * lo vanishes)
#pragma unroll
            for (int term = 0; term < 3; term++) {
                const uint32_t pa = at_ + (term == 1 ? kTPlane : 0), pb = aop + (term == 2 ? kOpPlane : 0);
                if (term < 2 || b_lo)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(pa + ks * 32),
                                       tc::desc_sw128(pb + ks * 16 * 128, 8192, 1024), id2, (term | ks) != 0);
            }
            tc::mma_commit(&bar[3]);
        }
    }
    // ---- epilogue 2: W = T' K (rows 0-63) hi / lo, U = T'' V (rows 64-127) fp32 ----
    if (tc::mbar_wait(&bar[3], 0, p.err, ANELM_ERR_TIMEOUT, abort)) {
        tc::tc_fence_after();
        const int q = warp & 3, hc = warp >> 2;  // hc: key / value dims [64 hc, 64 hc + 64)
        const int r = 32 * q + lane;
        const bool is_w = r < kC;
        const int t = is_w ? r : r - kC;
        const uint32_t col0 = (is_w ? 0 : 64) + 128 * hc;
        uint32_t xx[2][32];  // both 32-column loads in flight before the one wait
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + col0, xx[0]);
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + col0 + 32, xx[1]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int h32 = 0; h32 < 2; h32++) {
            const uint32_t (&x)[32] = xx[h32];
            const int d0 = 64 * hc + 32 * h32;
            if (is_w) {
                __half* whi = p.wh + (vrow + t) * kDk + d0;
#pragma unroll
                for (int c8 = 0; c8 < 4; c8++) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = __uint_as_float(x[8 * c8 + e]);
                    put_hl8(whi, p.v_plane, 8 * c8, v);
                }
            } else {
                float4* u = reinterpret_cast<float4*>(p.Ub + (vrow + t) * kDv + d0);
#pragma unroll
                for (int c4 = 0; c4 < 8; c4++)
                    u[c4] = make_float4(__uint_as_float(x[4 * c4]), __uint_as_float(x[4 * c4 + 1]),
                                        __uint_as_float(x[4 * c4 + 2]), __uint_as_float(x[4 * c4 + 3]));
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) {  // nothing of this CTA's may still be in flight when its TMEM is released
            for (int i = 0; i < 4; i++)
                for (uint32_t n = 0; n < tc::kWaitPolls && !tc::mbar_try_wait(&bar[i], 0); n++) {
                    if (i == 2 && !ok1) break;  // V was never requested
                    if ((i == 1 || i == 3) && *abort) break;
                }
        }
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kChunkTmemCols);
    }
}

// ---------------------------------------------------------------- the recurrence over chunks

// One chain CTA per (sequence, value head, 32 state columns j0 .. j0 + 32), eight warps.  State warp
// w < 4, (jg, dh) = (w / 2, w % 2), keeps S^T rows j0 + 16 jg .. + 16 (state columns) times key dims
// d in [64 dh, 64 dh + 64) in registers, in the accumulator layout of mma.m16n8k16, which is also
// the A-operand layout: S^T feeds W S directly (as hi / lo pairs), and the state update
// S^T += E^T K accumulates into the same registers.  The two state warps of a column group hold the
// two halves of d, so their partial W S sums meet in shared memory.  Output warp 4 + w computes,
// beside state warp w, Q S over the same d half from the state warp's S^T fragments (handed over
// in shared memory) and then Y = e^lc Q S + M D for 32 rows t from the group's D fragments, so
// only W S, D and the state update are on the recurrence's critical path.  Per chunk:
//   state:  S^T fragments -> W S -> exchange -> D = U - W S -> D fragments -> S = e^{lc_C} S + K^T E
//   output:                  Q S -> exchange ->                 e^lc Q S + M D -> Y
constexpr int kChainThreads = 256;
struct ChainSmem {
    // operand tiles in the TMA's 128B-swizzled layout (1024-byte aligned): [plane][box][64 rows][128 B]
    uint8_t w[2][2][8192];             // W[t][d], d in boxes of 64
    uint8_t q[2][2][8192];             // Q[t][d]
    uint8_t k[2][2][8192];             // K[t][d]
    uint8_t m[2][8192];                // M[t][i]
    uint8_t u[8192];                   // U[t][j0 .. j0 + 32] fp32, 128-byte rows
    float lc[2][kC];                   // in-chunk cumulative log decay, by chunk parity
    float eg[kC], ef[kC];              // e^{lc_t}, e^{lc_C - lc_t} of the current chunk
    float xd[4][32][32];               // partial W S of each state warp, [warp][register][lane]
    float xy[4][32][32];               // partial Q S of each output warp
    uint32_t sa[4][4][8][32];          // S^T fragments of each state warp: [warp][k-step][hi 0-3, lo 0-3][lane]
    uint32_t sdf[2][4][8][32];         // D fragments of each column group: [jg][k-step][8][lane]
    uint64_t bar[3];                   // W+Q, U+lc, M+K of the chunk landed (one phase per chunk)
    int abort;
};
// U[t][j] (fp32, j < 32) in its 128B-swizzled tile
__device__ __forceinline__ float u_at(const ChainSmem& sm, int t, int j) {
    return *reinterpret_cast<const float*>(&sm.u[t * 128 + ((((j >> 2) ^ t) & 7) << 4) + (j & 3) * 4]);
}

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
// acc[2 np], acc[2 np + 1] += A B over NP n-tile pairs (fragments bh[np], bl[np]), issued term by
// term across all 2 NP accumulators so dependent MMAs are 2 NP instructions apart
template <int NP>
__device__ __forceinline__ void mma3_tm(float (*acc)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                        const uint32_t (&bh)[NP][4], const uint32_t (&bl)[NP][4], bool b_lo = true) {
#pragma unroll
    for (int np = 0; np < NP; np++) {
        mma_16816(acc[2 * np], ah[0], ah[1], ah[2], ah[3], bh[np][0], bh[np][1]);
        mma_16816(acc[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bh[np][2], bh[np][3]);
    }
#pragma unroll
    for (int np = 0; np < NP; np++) {
        mma_16816(acc[2 * np], al[0], al[1], al[2], al[3], bh[np][0], bh[np][1]);
        mma_16816(acc[2 * np + 1], al[0], al[1], al[2], al[3], bh[np][2], bh[np][3]);
    }
    if (!b_lo) return;  // B exact in fp16 (its lo plane is zero)
#pragma unroll
    for (int np = 0; np < NP; np++) {
        mma_16816(acc[2 * np], ah[0], ah[1], ah[2], ah[3], bl[np][0], bl[np][1]);
        mma_16816(acc[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bl[np][2], bl[np][3]);
    }
}

// A chunk's operand tiles are fetched by one thread as TMA tile copies (64 rows x 128 bytes, 128B
// swizzle; the fragment loads undo the swizzle), completing on one mbarrier per group.
struct ChainMaps {
    CUtensorMap w, q, k, m, u;
};
// W and Q, hi and lo planes (read by W S and Q S)
__device__ __forceinline__ void chain_load_wq(ChainSmem& sm, const ChainMaps& mp, long long krow, long long vrow,
                                              bool exact) {
    tc::mbar_arrive_expect_tx(&sm.bar[0], (exact ? 3 : 4) * 2 * 8192);  // exact: no Q lo plane
    for (int pl = 0; pl < 2; pl++)
        for (int bx = 0; bx < 2; bx++) {
            tc::tma_load_3d(sm.w[pl][bx], &mp.w, &sm.bar[0], 64 * bx, (int)vrow, pl);
            if (pl == 0 || !exact) tc::tma_load_3d(sm.q[pl][bx], &mp.q, &sm.bar[0], 64 * bx, (int)krow, pl);
        }
}
// this block's U columns and lc (read by D = U - W S and the decay factors)
__device__ __forceinline__ void chain_load_u(ChainSmem& sm, const ChainMaps& mp, const GdnPrefillParams& p,
                                             long long vrow, int j0, int par) {
    tc::mbar_arrive_expect_tx(&sm.bar[1], 8192 + kC * 4);
    tc::tma_load_2d(sm.u, &mp.u, &sm.bar[1], j0, (int)vrow);
    tc::bulk_load(sm.lc[par], p.lcb + vrow, kC * 4, &sm.bar[1]);
}
// K and M, hi and lo planes (read by the state update and M D)
__device__ __forceinline__ void chain_load_mk(ChainSmem& sm, const ChainMaps& mp, long long krow, long long vrow,
                                              bool exact) {
    tc::mbar_arrive_expect_tx(&sm.bar[2], (exact ? 1 : 2) * 2 * 8192 + 2 * 8192);  // exact: no K lo plane
    for (int pl = 0; pl < 2; pl++) {
        if (pl == 0 || !exact)
            for (int bx = 0; bx < 2; bx++) tc::tma_load_3d(sm.k[pl][bx], &mp.k, &sm.bar[2], 64 * bx, (int)krow, pl);
        tc::tma_load_3d(sm.m[pl], &mp.m, &sm.bar[2], 0, (int)vrow, pl);
    }
}

__global__ void __launch_bounds__(kChainThreads, 1) gdn_pf_chain_kernel(const __grid_constant__ ChainMaps mp,
                                                                        const GdnPrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    ChainSmem& sm = *reinterpret_cast<ChainSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nblk = kDv / kDvb;
    const int h = blockIdx.x / nblk, j0 = (blockIdx.x % nblk) * kDvb, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const bool state = warp < 4;
    const int w4 = warp & 3, jg = w4 >> 1, dh = w4 & 1;
    const int jr = 16 * jg;      // this warp's state columns j0 + jr .. + 16
    const int dbase = 64 * dh;   // and key dims dbase .. + 64
    const int kh = h / (p.Hv / p.Hk);
    const int seq = p.seq_ids ? p.seq_ids[b] : b;
    float* S = p.state + ((long long)seq * p.Hv + h) * kDk * kDv;
    // state warps: s[nt][e] = S[d][j0 + j], j = jr + g + 8 (e / 2), d = dbase + 8 nt + 2 c + (e % 2)
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++)
            s[nt][e] = state ? S[(long long)(dbase + 8 * nt + 2 * c + (e & 1)) * kDv + j0 + jr + g + 8 * (e >> 1)] : 0.f;
    const int nC = p.T_pad / kC;
    const long long krow0 = ((long long)b * p.Hk + kh) * p.T_pad;
    const long long vrow0 = ((long long)b * p.Hv + h) * p.T_pad;
    // the loads of chunk ci complete phase ci of bar[0] (W, Q), bar[1] (U, lc), bar[2] (M, K); output
    // warps 4, 5, 6 issue them once the previous chunk's readers are done
    if (tid == 0) {
        for (int i = 0; i < 3; i++) tc::mbar_init(&sm.bar[i], 1);
        sm.abort = 0;
        tc::fence_barrier_init();
    }
    __syncthreads();
    volatile int* abort = &sm.abort;
    const bool loader = tid == 4 * 32;  // lane 0 of output warp 4 issues every copy
    const bool exact = p.qkv_exact != 0;  // Q and K exact in fp16: their lo planes are neither loaded nor used
    if (loader) {
        chain_load_wq(sm, mp, krow0, vrow0, exact);
        chain_load_u(sm, mp, p, vrow0, j0, 0);
        chain_load_mk(sm, mp, krow0, vrow0, exact);
    }
    const uint32_t a_w = smem_u32(sm.w), a_q = smem_u32(sm.q), a_k = smem_u32(sm.k), a_m = smem_u32(sm.m);
    // named barriers: 1 + jg state pair, 3 + jg output pair (64 threads); 5 + jg S^T fragments and
    // 7 + jg D fragments, state warps arrive, output warps wait (128 threads)
    for (int ci = 0; ci < nC; ci++) {
        const int par = ci & 1;
        const bool more = ci + 1 < nC;
        tc::mbar_wait(&sm.bar[0], par, p.err, ANELM_ERR_TIMEOUT, abort);
        __syncthreads();  // W and Q of this chunk are in shared memory
        // ---- W S (state warps) and Q S (output warps) over this warp's half of d, all 64 rows t ----
        float acc[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[nt][e] = 0.f;
        {
            const uint32_t bhi = state ? a_w : a_q, blo = bhi + 16384;
            uint32_t fa[4][4], fl[4][4];
            if (state) {
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    afrag(s, ks, fa[ks], fl[ks]);
#pragma unroll
                    for (int r = 0; r < 4; r++) {
                        sm.sa[w4][ks][r][lane] = fa[ks][r];
                        sm.sa[w4][ks][4 + r][lane] = fl[ks][r];
                    }
                }
                named_bar_arrive_cta(5 + jg, 128);
            } else {
                named_bar_sync_cta(5 + jg, 128);
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
#pragma unroll
                    for (int r = 0; r < 4; r++) {
                        fa[ks][r] = sm.sa[w4][ks][r][lane];
                        fl[ks][r] = sm.sa[w4][ks][4 + r][lane];
                    }
            }
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const int k0 = dbase + 16 * ks;
#pragma unroll
                for (int n2 = 0; n2 < 2; n2++) {
                    uint32_t bh[2][4], bl[2][4];
                    const bool b_lo = state || !exact;  // W always has a lo plane, Q only when not exact
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        ldb2_sw(bh[q], bhi, 32 * n2 + 16 * q, k0, lane);
                        if (b_lo) ldb2_sw(bl[q], blo, 32 * n2 + 16 * q, k0, lane);
                    }
                    mma3_tm<2>(&acc[4 * n2], fa[ks], fl[ks], bh, bl, b_lo);
                }
            }
        }
        __syncthreads();  // W, Q free
        if (more && loader) chain_load_wq(sm, mp, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, exact);
        // ---- the two d halves of a column group meet ----
        float (*xb)[32][32] = state ? sm.xd : sm.xy;
#pragma unroll
        for (int r = 0; r < 32; r++) xb[w4][r][lane] = acc[r >> 2][r & 3];
        named_bar_sync_cta((state ? 1 : 3) + jg, 64);
        float y[4][4];  // output warps: Q S for rows t in [32 dh, 32 dh + 32)
        if (state) {
#pragma unroll
            for (int r = 0; r < 32; r++) acc[r >> 2][r & 3] += xb[w4 ^ 1][r][lane];
        } else {
#pragma unroll
            for (int n4 = 0; n4 < 4; n4++)
#pragma unroll
                for (int e = 0; e < 4; e++)
                    y[n4][e] = (dh ? acc[4 + n4][e] : acc[n4][e]) + xb[w4 ^ 1][4 * (4 * dh + n4) + e][lane];
        }
        tc::mbar_wait(&sm.bar[1], par, p.err, ANELM_ERR_TIMEOUT, abort);
        __syncthreads();  // U and lc of this chunk are in shared memory
        const float* lc = sm.lc[par];
        const float lcC = lc[kC - 1];
        if (tid < kC) {  // published by the barrier before M D
            sm.eg[tid] = expf(lc[tid]);
            sm.ef[tid] = expf(lcC - lc[tid]);
        }
        if (state) {
            // D = U - W S (in place of acc); its fragments (k-steps 2 dh, 2 dh + 1) for the output warps
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++)
                    acc[nt][e] = u_at(sm, 8 * nt + 2 * c + (e & 1), jr + g + 8 * (e >> 1)) - acc[nt][e];
#pragma unroll
            for (int k2 = 0; k2 < 2; k2++) {
                uint32_t ah[4], al[4];
                if (dh) afrag(acc, 2 + k2, ah, al);
                else afrag(acc, k2, ah, al);
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    sm.sdf[jg][2 * dh + k2][r][lane] = ah[r];
                    sm.sdf[jg][2 * dh + k2][4 + r][lane] = al[r];
                }
            }
            named_bar_arrive_cta(7 + jg, 128);
        }
        tc::mbar_wait(&sm.bar[2], par, p.err, ANELM_ERR_TIMEOUT, abort);
        __syncthreads();  // M and K of this chunk are in shared memory; U read; e^lc factors visible
        if (more && loader) chain_load_u(sm, mp, p, vrow0 + (ci + 1) * kC, j0, par ^ 1);
        if (!state) {
            // ---- Y = e^lc Q S + M D for rows t in [32 dh, 32 dh + 32) ----
            const int tt = 32 * dh;
#pragma unroll
            for (int n4 = 0; n4 < 4; n4++)
#pragma unroll
                for (int e = 0; e < 4; e++) y[n4][e] *= sm.eg[tt + 8 * n4 + 2 * c + (e & 1)];
            named_bar_sync_cta(7 + jg, 128);
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                if (16 * ks >= tt + 32) break;  // M[t][i] = 0 for i > t
                uint32_t ah[4], al[4];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    ah[r] = sm.sdf[jg][ks][r][lane];
                    al[r] = sm.sdf[jg][ks][4 + r][lane];
                }
                uint32_t bh[2][4], bl[2][4];
#pragma unroll
                for (int np = 0; np < 2; np++) {
                    ldb2_sw(bh[np], a_m, tt + 16 * np, 16 * ks, lane);
                    ldb2_sw(bl[np], a_m + 8192, tt + 16 * np, 16 * ks, lane);
                }
                mma3_tm<2>(y, ah, al, bh, bl);
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
        } else {
            // ---- S = e^{lc_C} S + K^T diag(e^{lc_C - lc}) D over this warp's half of d ----
            const float gC = expf(lcC);
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) s[nt][e] *= gC;
            float fs[8][2];  // e^{lc_C - lc_t}, t = 8 nt + 2 c + e
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 2; e++) fs[nt][e] = sm.ef[8 * nt + 2 * c + e];
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                uint32_t ah[4], al[4];
                afrag(acc, fs, ks, ah, al);
                uint32_t bh[4][4], bl[4][4];
#pragma unroll
                for (int np = 0; np < 4; np++) {
                    ldb2_t_sw(bh[np], a_k, dbase + 16 * np, 16 * ks, lane);
                    if (!exact) ldb2_t_sw(bl[np], a_k + 16384, dbase + 16 * np, 16 * ks, lane);
                }
                mma3_tm<4>(s, ah, al, bh, bl, !exact);
            }
        }
        __syncthreads();  // M, K free
        if (more && loader) chain_load_mk(sm, mp, krow0 + (ci + 1) * kC, vrow0 + (ci + 1) * kC, exact);
    }
    if (state) {
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                S[(long long)(dbase + 8 * nt + 2 * c + (e & 1)) * kDv + j0 + jr + g + 8 * (e >> 1)] = s[nt][e];
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

static int launch_chunks_and_chain(const GdnPrefillParams& p, cudaStream_t stream) {
    const int nC = p.T_pad / kC;
    const size_t chunk_smem = sizeof(ChunkSmem) + 1024, chain_smem = sizeof(ChainSmem) + 1024;
    const uint64_t krows = (uint64_t)p.B * p.Hk * p.T_pad, vrows = (uint64_t)p.B * p.Hv * p.T_pad;
    CUtensorMap mK, mQ, mV;
    ChainMaps cm;
    if (!make_plane_map(&mK, p.kh, krows, p.q_plane) || !make_plane_map(&mQ, p.qh, krows, p.q_plane) ||
        !make_plane_map(&mV, p.vh, vrows, p.v_plane))
        return ANELM_ERR_CUDA;
    cm.k = mK;
    cm.q = mQ;
    {  // W (hi / lo like V), M (64 columns), U (fp32, 32-column boxes of this block's state columns)
        auto fn = tc::tmap_encode_fn();
        cuuint64_t dims[2] = {(cuuint64_t)kDv, vrows};
        cuuint64_t strides[1] = {(cuuint64_t)kDv * 4};
        cuuint32_t box[2] = {(cuuint32_t)kDvb, (cuuint32_t)kC};
        cuuint32_t estr[2] = {1, 1};
        if (!make_plane_map(&cm.w, p.wh, vrows, p.v_plane) || !make_plane_map(&cm.m, p.mh, vrows, p.m_plane, kC) ||
            fn(&cm.u, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.Ub, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return ANELM_ERR_CUDA;
    }
    cudaFuncSetAttribute(gdn_pf_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk_smem);
    cudaFuncSetAttribute(gdn_pf_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chain_smem);
    gdn_pf_chunk_kernel<<<dim3(nC, p.Hv, p.B), kChunkThreads, chunk_smem, stream>>>(mK, mQ, mV, p);
    gdn_pf_chain_kernel<<<dim3(p.Hv * (kDv / kDvb), p.B), kChainThreads, chain_smem, stream>>>(cm, p);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

int launch_gdn_prefill(GdnPrefillParams p, void* workspace, cudaStream_t stream) {
    if (p.dk != kDk || p.dv != kDv || p.Hv % p.Hk) return ANELM_ERR_UNSUPPORTED;
    p.T_pad = (p.n + kC - 1) / kC * kC;
    carve(p, workspace, true);
    p.qkv_exact = 0;  // q, k, v come out of the conv / SiLU / L2 norm in fp32: both planes carry them
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
    // 16-bit inputs are exact in fp16 (bf16 normal values have 8 significant bits): lo planes are zero
    p.qkv_exact = p.in_dtype == ANELM_F16 || p.in_dtype == ANELM_BF16;
    gdn_pf_pack_kernel<<<dim3(p.T_pad, p.B), 256, 0, stream>>>(p);
    return launch_chunks_and_chain(p, stream);
}

}  // namespace anelm
