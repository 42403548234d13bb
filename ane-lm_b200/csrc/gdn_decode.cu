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
// Work decomposition.  One thread-block cluster per (batch row, key head kh).
// The cluster holds RATIO x NSPLIT CTAs: the RATIO value heads that share kh
// (GQA, qwen3_5.cpp:880-890) times NSPLIT column blocks of each head's 128x128
// fp32 state S[k][v].  The delta rule is column-separable (column j of S needs
// only k, q and v[j]), so every CTA streams its 128 x W block of S (W = 128 /
// NSPLIT) from HBM into registers once, updates it and writes it back once; the
// block's loads are issued right after the conv inputs', so the conv, the q/k
// exchange and the norms overlap its transfer.
//
// Conv ring ownership.  Each conv channel of the row belongs to exactly one CTA
// of exactly one cluster: the cluster of kh owns the 256 q/k channels of kh
// (split evenly over its CTAs) and the v channels of its value heads (each CTA
// its W columns).  So the reference's own ring layout [C][K-1] is updated in
// place without races, and the ring position is kept per (sequence, key head):
// every CTA of the cluster reads it before the first cluster barrier and rank 0
// advances it once the whole cluster's q/k slices (pushed after each CTA read
// the position) have arrived.  No atomics, no memory fences.
//
// Exchanges (distributed shared memory, no cluster barriers).  Each CTA convolves
// its slice of the q/k channels and pushes the SiLU outputs into every peer's q/k
// buffer with st.async, whose arrival is counted in bytes on the peer's
// mbarrier; the gated RMSNorm's sum(y^2) partials travel the same way to the
// CTAs of the same head.  Each CTA waits only on its own barriers, so no
// cluster-wide release has to wait for the state loads or stores in flight.  A
// single relaxed cluster arrive/wait publishes the barrier initialisation.
#include <cooperative_groups.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

namespace cg = cooperative_groups;

namespace anelm {

namespace {

constexpr int kDk = 128;
constexpr int kDv = 128;
constexpr int kPrefetchItems = 192;  // ~ the (row, key head) items resident at once (5 CTAs per SM)

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory"); }

// Shared-memory address of `p` inside CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_rank(const void* p, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// Asynchronous 4-byte store into another CTA's shared memory; its arrival is
// counted (as 4 transaction bytes) on that CTA's mbarrier `bar`.
__device__ __forceinline__ void st_async_f32(uint32_t dst, float v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];\n" ::"r"(dst),
                 "r"(__float_as_uint(v)), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void mbar_init1(uint64_t* bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(bar)));
}
__device__ __forceinline__ void mbar_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// Bounded wait for phase 0 of a single-use barrier; false (and *err set) if it never completes.
__device__ __forceinline__ bool mbar_wait0(uint64_t* bar, int* err) {
    for (uint32_t i = 0; i < (1u << 22); i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(smem_u32(bar))
            : "memory");
        if (ok) return true;
    }
    if (err) atomicCAS(err, 0, ANELM_ERR_TIMEOUT);
    return false;
}

// STAGED: the CTA's 128 x W state block comes in by one TMA tile load into shared memory, issued at
// entry (before the conv inputs), and goes back by one TMA tile store; the delta rule runs in two
// passes over shared memory, so no registers hold the block and more CTAs fit an SM.  Otherwise the
// block streams into registers (float4 per thread and row) and back.
template <int RATIO, int NSPLIT, int THREADS, bool STAGED>
// 128-thread CTAs are held to 96 registers: at 102 the per-warp allocation rounds to 3,328 and
// only four CTAs fit an SM, at 96 five do (a 20-byte spill).  Staged CTAs: six per SM (shared memory).
__global__ void __launch_bounds__(THREADS, STAGED ? 6 : (THREADS == 128 ? 5 : 1))
    gdn_decode_kernel(const GdnDecodeParams p, const __grid_constant__ CUtensorMap tmS) {
    constexpr int CS = RATIO * NSPLIT;     // CTAs per cluster
    constexpr int W = kDv / NSPLIT;        // value columns per CTA
    constexpr int QPR = W / 4;             // float4 quads per row segment
    constexpr int RPP = THREADS / QPR;     // rows per pass
    constexpr int NR = kDk / RPP;          // rows per thread
    constexpr int QKP = 2 * kDk / CS;      // q/k conv channels convolved by this CTA
    constexpr int NW = THREADS / 32;
    constexpr int NU = (QKP + THREADS - 1) / THREADS;
    static_assert(RPP * NR == kDk, "row split");
    static_assert(QKP * CS == 2 * kDk, "q/k split");

    __shared__ __align__(16) float qk_s[2 * kDk];  // [0,128) q, [128,256) k (filled by the whole cluster)
    __shared__ __align__(16) float v_s[W];
    __shared__ __align__(16) float z_s[W];
    __shared__ __align__(16) float y_s[W];
    __shared__ __align__(16) float w_s[W];
    __shared__ __align__(16) float red[2][NW][W];
    __shared__ __align__(16) float ss_s[NSPLIT];
    __shared__ float scal[4];
    __shared__ __align__(8) uint64_t bar_qk, bar_ss, bar_s;
    __shared__ __align__(128) float s_blk[STAGED ? kDk * W : 4];  // staged state block [128 rows][W]

    cg::cluster_group cluster = cg::this_cluster();
    if (threadIdx.x == 0) {
        mbar_init1(&bar_qk);
        mbar_init1(&bar_ss);
        // expected bytes are posted before this CTA arrives on the cluster barrier, so no
        // peer can deliver before the expectation exists
        mbar_expect(&bar_qk, 2 * kDk * 4);   // the whole q | k vector arrives from the cluster
        mbar_expect(&bar_ss, NSPLIT * 4);    // one partial sum of y^2 per column block of this head
        if (STAGED) mbar_init1(&bar_s);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    cluster_arrive_relaxed();  // matched below, before the first store into a peer

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = (int)cluster.block_rank();
    const int hl = rank / NSPLIT, cb = rank % NSPLIT;
    const int item = blockIdx.x / CS;          // = b * Hk + kh
    const int kh = item % p.Hk;
    const int b = item / p.Hk;
    const int h = kh * RATIO + hl;              // value head, qwen3_5.cpp:890
    const int seq = p.seq_ids ? p.seq_ids[b] : p.seq_scalar;
    const int C = p.C;
    const int key_total = p.Hk * kDk;
    const int j0 = cb * W;
    const int s_row0 = (int)(((long long)seq * p.Hv + h) * kDk);  // first row of this head's state (TMA view)
    if (STAGED && threadIdx.x == 0) {  // the state block, first of all loads
        mbar_expect(&bar_s, kDk * W * 4);
        tc::tma_load_2d(s_blk, &tmS, &bar_s, j0, s_row0);
    }

    // ---- 1. loads: the small inputs of the conv / gates first, then the 32 KB state block ----
    // Requests are served roughly in issue order, so small loads issued after the state block
    // would wait for it; issued first, the conv, the q/k exchange and the norms run while the
    // state block streams in, and only the delta rule waits for it.
    const int cq = tid % QPR, rg = tid / QPR;
    float* Sbase = p.ssm + (((long long)seq * p.Hv + h) * kDk) * kDv + j0 + 4 * cq;
    const char* proj_row = reinterpret_cast<const char*>(p.proj) +
                           (long long)b * p.proj_stride * dtype_bytes(p.proj_dtype);
    int* pos_ptr = p.conv_pos + (long long)seq * p.Hk + kh;
    float* ring = p.conv + (long long)seq * C * 3;
    const int n = *pos_ptr;                     // ring position (reference conv_pos)
    // all three ring slots are loaded (the position selects among them once it arrives)
    struct ConvIn { float4 w; float r0, r1, r2, x; };
    auto conv_load = [&](int c) -> ConvIn {
        ConvIn ci;
        ci.w = *reinterpret_cast<const float4*>(p.conv_w + (long long)c * 4);
        ci.r0 = ring[c * 3];
        ci.r1 = ring[c * 3 + 1];
        ci.r2 = ring[c * 3 + 2];
        ci.x = load_as_float(proj_row, p.proj_dtype, c);
        return ci;
    };
    constexpr int NV = (W + THREADS - 1) / THREADS;
    ConvIn vin[NV], qkin[NU];
    float zin[NV], nwin[NV];
#pragma unroll
    for (int u = 0; u < NV; u++) {
        const int i = tid + u * THREADS;
        if (i < W) {
            vin[u] = conv_load(2 * key_total + h * kDv + j0 + i);
            zin[u] = load_as_float(proj_row, p.proj_dtype, C + (long long)h * kDv + j0 + i);
            nwin[u] = p.norm_w[j0 + i];
        }
    }
#pragma unroll
    for (int u = 0; u < NU; u++) {
        const int i = tid + u * THREADS;
        if (i < QKP) {
            const int ci = rank * QKP + i;  // 0..255 within (q | k) of key head kh
            qkin[u] = conv_load((ci < kDk) ? kh * kDk + ci : key_total + kh * kDk + (ci - kDk));
        }
    }
    float ga = 0.f, gb = 0.f;
    if (tid == 0) {
        ga = load_as_float(proj_row, p.proj_dtype, C + (long long)p.Hv * kDv + h);
        gb = load_as_float(proj_row, p.proj_dtype, C + (long long)p.Hv * kDv + p.Hv + h);
    }
    float4 S[STAGED ? 1 : NR];
    if constexpr (!STAGED) {
#pragma unroll
        for (int i = 0; i < NR; i++) S[i] = __ldcs(reinterpret_cast<const float4*>(Sbase + (long long)(rg + RPP * i) * kDv));
    }
    // L2 prefetch of the state head that the CTA about one resident wave later (kPrefetchItems
    // (row, key head) items on) will stream: its 64 KB are in L2 when it starts, which adds bytes
    // in flight beyond what the register-resident blocks hold
    if (cb == 0 && tid == 0) {
        const int item2 = item + kPrefetchItems;
        if (item2 < (int)(gridDim.x / CS)) {
            const int b2 = item2 / p.Hk, kh2 = item2 % p.Hk;
            const int seq2 = p.seq_ids ? p.seq_ids[b2] : p.seq_scalar;
            const float* S2 = p.ssm + ((long long)seq2 * p.Hv + kh2 * RATIO + hl) * kDk * kDv;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(S2), "r"(kDk * kDv * 4) : "memory");
        }
    }

    int p1 = n + 1;
    if (p1 == 3) p1 = 0;
    int p2 = p1 + 1;
    if (p2 == 3) p2 = 0;
    // conv1d_update (cpu_ops.cpp:95-110) + SiLU (cpu_ops.cpp:6-13) of one channel.  The new input x
    // goes into ring slot n only after the exchanges (a barrier's release would otherwise wait for
    // that global store to be acknowledged).
    auto conv_ch = [&](const ConvIn& ci) -> float {
        const float s0 = n == 0 ? ci.r0 : n == 1 ? ci.r1 : ci.r2;
        const float s1 = p1 == 0 ? ci.r0 : p1 == 1 ? ci.r1 : ci.r2;
        const float s2 = p2 == 0 ? ci.r0 : p2 == 1 ? ci.r1 : ci.r2;
        const float y = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s0, ci.w.x), __fmul_rn(s1, ci.w.y)), __fmul_rn(s2, ci.w.z)),
                                  __fmul_rn(ci.x, ci.w.w));
        return y / (1.0f + expf(-y));
    };

    // ---- 2. this CTA's v / z columns and its slice of the q/k channels ----
    float xv[NV], xqk[NU];
#pragma unroll
    for (int u = 0; u < NV; u++) {
        const int i = tid + u * THREADS;
        xv[u] = 0.f;
        if (i < W) {
            v_s[i] = conv_ch(vin[u]);
            xv[u] = vin[u].x;
            z_s[i] = zin[u];
            w_s[i] = nwin[u];
        }
    }
    float qk_mine[NU];
#pragma unroll
    for (int u = 0; u < NU; u++) {
        const int i = tid + u * THREADS;
        qk_mine[u] = 0.f;
        xqk[u] = 0.f;
        if (i < QKP) {
            qk_mine[u] = conv_ch(qkin[u]);
            xqk[u] = qkin[u].x;
        }
    }
    if (tid == 0) {
        scal[0] = sigmoid_ref(gb);                                     // qwen3_5.cpp:897
        scal[1] = expf(-p.A[h] * softplus_ref(ga + p.dt_bias[h]));     // qwen3_5.cpp:898
    }
    cluster_wait();  // every CTA of the cluster has initialised its barriers
#pragma unroll
    for (int u = 0; u < NU; u++) {
        const int i = tid + u * THREADS;
        if (i < QKP) {
#pragma unroll
            for (int q = 0; q < CS; q++)
                st_async_f32(map_rank(&qk_s[rank * QKP + i], q), qk_mine[u], map_rank(&bar_qk, q));
        }
    }
    // q | k of this key head complete.  Every CTA of the cluster read the ring position before
    // pushing its slice, so once rank 0 has every slice the position may advance.
    mbar_wait0(&bar_qk, p.err);
    if (rank == 0 && tid == 0) *pos_ptr = p1;  // cpu_ops.cpp:126-128

    // ---- 3. L2-normalise q and k (cpu_ops.cpp:82-87), q *= 1/sqrt(dk) (qwen3_5.cpp:879-887) ----
    if (warp < 2) {
        float* x = qk_s + warp * kDk;
        float ss = 0.f;
        for (int i = lane; i < kDk; i += 32) ss += x[i] * x[i];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + p.l2_eps);
        const float qscale = 1.0f / sqrtf((float)kDk);
        for (int i = lane; i < kDk; i += 32) {
            float v = __fmul_rn(x[i], inv);
            if (warp == 0) v = __fmul_rn(v, qscale);
            x[i] = v;
        }
    }
    __syncthreads();
    const float beta = scal[0], decay = scal[1];

    // column sums over the 128 key rows: shuffles across row groups, then across warps
    // (each of the two uses has its own buffer, so one barrier per reduction suffices)
    auto colsum = [&](float4 v, int buf) -> float4 {
#pragma unroll
        for (int o = QPR; o < 32; o <<= 1) {
            v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
            v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
            v.z += __shfl_xor_sync(0xffffffffu, v.z, o);
            v.w += __shfl_xor_sync(0xffffffffu, v.w, o);
        }
        if (lane < QPR) *reinterpret_cast<float4*>(&red[buf][warp][4 * lane]) = v;
        __syncthreads();
        float4 t = *reinterpret_cast<const float4*>(&red[buf][0][4 * cq]);
#pragma unroll
        for (int w = 1; w < NW; w++) {
            const float4 u = *reinterpret_cast<const float4*>(&red[buf][w][4 * cq]);
            t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
        }
        return t;
    };

    // ---- 4. delta rule on the register block (or, staged, on the shared-memory block) ----
    const float* q_s = qk_s;
    const float* k_s = qk_s + kDk;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 yv = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (STAGED) {
        if (!mbar_wait0(&bar_s, p.err)) {  // the block never arrived: wait once more (bounded), then leave
            mbar_wait0(&bar_s, nullptr);
            return;
        }
        float* blk = s_blk + 4 * cq;
        auto at = [&](int i) -> float4* { return reinterpret_cast<float4*>(blk + (rg + RPP * i) * W); };
        const bool hf = p.delta_mode != ANELM_DELTA_CPUOPS;
        // pass 1: Sk = S^T k (cpu_ops.cpp:134-135), or (g S)^T k when the decay comes first
#pragma unroll
        for (int i = 0; i < NR; i++) {
            float4 v = *at(i);
            if (hf) {
                v.x = __fmul_rn(v.x, decay); v.y = __fmul_rn(v.y, decay);
                v.z = __fmul_rn(v.z, decay); v.w = __fmul_rn(v.w, decay);
            }
            const float kr = k_s[rg + RPP * i];
            sk.x += v.x * kr; sk.y += v.y * kr; sk.z += v.z * kr; sk.w += v.w * kr;
        }
        sk = colsum(sk, 0);
        float4 d = make_float4(v_s[4 * cq] - sk.x, v_s[4 * cq + 1] - sk.y, v_s[4 * cq + 2] - sk.z,
                               v_s[4 * cq + 3] - sk.w);
        if (hf) { d.x *= beta; d.y *= beta; d.z *= beta; d.w *= beta; }
        // pass 2: the update (cpu_ops.cpp:140-142 / export_hybrid_chunks.py:142-147) and y = S^T q (144-145)
#pragma unroll
        for (int i = 0; i < NR; i++) {
            float4 v = *at(i);
            const float kr = k_s[rg + RPP * i];
            if (hf) {
                v.x = __fadd_rn(__fmul_rn(v.x, decay), __fmul_rn(kr, d.x));
                v.y = __fadd_rn(__fmul_rn(v.y, decay), __fmul_rn(kr, d.y));
                v.z = __fadd_rn(__fmul_rn(v.z, decay), __fmul_rn(kr, d.z));
                v.w = __fadd_rn(__fmul_rn(v.w, decay), __fmul_rn(kr, d.w));
            } else {
                const float ax = beta * kr;
                v.x = __fadd_rn(__fmul_rn(v.x, decay), __fmul_rn(ax, d.x));
                v.y = __fadd_rn(__fmul_rn(v.y, decay), __fmul_rn(ax, d.y));
                v.z = __fadd_rn(__fmul_rn(v.z, decay), __fmul_rn(ax, d.z));
                v.w = __fadd_rn(__fmul_rn(v.w, decay), __fmul_rn(ax, d.w));
            }
            *at(i) = v;
            const float qr = q_s[rg + RPP * i];
            yv.x += v.x * qr; yv.y += v.y * qr; yv.z += v.z * qr; yv.w += v.w * qr;
        }
        tc::fence_proxy_async_smem();  // this thread's block writes, for the TMA store
    } else if (p.delta_mode == ANELM_DELTA_CPUOPS) {
        // cpu_ops.cpp:134-142: Sk = S^T k (undecayed); delta = v - Sk; S = decay*S + (beta*k) delta^T
#pragma unroll
        for (int i = 0; i < NR; i++) {
            const float kr = k_s[rg + RPP * i];
            sk.x += S[i].x * kr; sk.y += S[i].y * kr; sk.z += S[i].z * kr; sk.w += S[i].w * kr;
        }
        sk = colsum(sk, 0);
        const float4 d = make_float4(v_s[4 * cq] - sk.x, v_s[4 * cq + 1] - sk.y, v_s[4 * cq + 2] - sk.z,
                                     v_s[4 * cq + 3] - sk.w);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            const float ax = beta * k_s[rg + RPP * i];
            S[i].x = __fadd_rn(__fmul_rn(S[i].x, decay), __fmul_rn(ax, d.x));
            S[i].y = __fadd_rn(__fmul_rn(S[i].y, decay), __fmul_rn(ax, d.y));
            S[i].z = __fadd_rn(__fmul_rn(S[i].z, decay), __fmul_rn(ax, d.z));
            S[i].w = __fadd_rn(__fmul_rn(S[i].w, decay), __fmul_rn(ax, d.w));
        }
    } else {
        // export_hybrid_chunks.py:142-147: S = g*S; Sk = S^T k; delta = (v - Sk)*beta; S += k delta^T
#pragma unroll
        for (int i = 0; i < NR; i++) {
            S[i].x = __fmul_rn(S[i].x, decay); S[i].y = __fmul_rn(S[i].y, decay);
            S[i].z = __fmul_rn(S[i].z, decay); S[i].w = __fmul_rn(S[i].w, decay);
            const float kr = k_s[rg + RPP * i];
            sk.x += S[i].x * kr; sk.y += S[i].y * kr; sk.z += S[i].z * kr; sk.w += S[i].w * kr;
        }
        sk = colsum(sk, 0);
        const float4 d = make_float4((v_s[4 * cq] - sk.x) * beta, (v_s[4 * cq + 1] - sk.y) * beta,
                                     (v_s[4 * cq + 2] - sk.z) * beta, (v_s[4 * cq + 3] - sk.w) * beta);
#pragma unroll
        for (int i = 0; i < NR; i++) {
            const float kr = k_s[rg + RPP * i];
            S[i].x = __fadd_rn(S[i].x, __fmul_rn(kr, d.x));
            S[i].y = __fadd_rn(S[i].y, __fmul_rn(kr, d.y));
            S[i].z = __fadd_rn(S[i].z, __fmul_rn(kr, d.z));
            S[i].w = __fadd_rn(S[i].w, __fmul_rn(kr, d.w));
        }
    }
    if constexpr (!STAGED) {  // y = S^T q (cpu_ops.cpp:144-145)
#pragma unroll
        for (int i = 0; i < NR; i++) {
            const float qr = q_s[rg + RPP * i];
            yv.x += S[i].x * qr; yv.y += S[i].y * qr; yv.z += S[i].z * qr; yv.w += S[i].w * qr;
        }
    }
    yv = colsum(yv, 1);
    if (rg == 0) *reinterpret_cast<float4*>(&y_s[4 * cq]) = yv;
    __syncthreads();
    if (STAGED && tid == 0) {  // the updated block back to HBM (every thread's writes are fenced and past the barrier)
        tc::tma_store_2d(&tmS, s_blk, j0, s_row0);
        tc::bulk_commit_group();
    }

    // ---- 5. gated RMSNorm over the head's 128 columns (rmsnorm_gated, cpu_ops.cpp:32-38) ----
    if (warp == 0) {
        float ss = 0.f;
        for (int i = lane; i < W; i += 32) ss += y_s[i] * y_s[i];
        ss = warp_sum(ss);
        if (lane < NSPLIT) st_async_f32(map_rank(&ss_s[cb], hl * NSPLIT + lane), ss, map_rank(&bar_ss, hl * NSPLIT + lane));
    }
    // global stores: the state block (unless staged) and the new inputs into ring slot n (cpu_ops.cpp:109)
    if constexpr (!STAGED) {
#pragma unroll
        for (int i = 0; i < NR; i++) __stcs(reinterpret_cast<float4*>(Sbase + (long long)(rg + RPP * i) * kDv), S[i]);
    }
#pragma unroll
    for (int u = 0; u < NV; u++) {
        const int i = tid + u * THREADS;
        if (i < W) ring[(2 * key_total + h * kDv + j0 + i) * 3 + n] = xv[u];
    }
#pragma unroll
    for (int u = 0; u < NU; u++) {
        const int i = tid + u * THREADS;
        if (i < QKP) {
            const int ci = rank * QKP + i;
            const int c = (ci < kDk) ? kh * kDk + ci : key_total + kh * kDk + (ci - kDk);
            ring[c * 3 + n] = xqk[u];
        }
    }
    mbar_wait0(&bar_ss, p.err);  // the head's partial sums have arrived
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < NSPLIT; q++) tot += ss_s[q];
    const float rinv = 1.0f / sqrtf(tot / (float)kDv + 1e-6f);
    const long long orow = (long long)b * p.out_stride + (long long)h * kDv + j0;
    for (int i = tid; i < W; i += THREADS) {
        const float z = z_s[i];
        float o = __fmul_rn(__fmul_rn(y_s[i], rinv), w_s[i]);
        o = o / (1.0f + expf(-z));
        o = __fmul_rn(o, z);
        store_from_float(p.out, p.out_dtype, orow + i, o);
    }
    if (STAGED && tid == 0) tc::bulk_wait_group_read0();  // the block's store has read shared memory
}


template <int RATIO, int NSPLIT, int THREADS, bool STAGED>
int launch_cfg(const GdnDecodeParams& p, int n_rows, cudaStream_t stream) {
    constexpr int CS = RATIO * NSPLIT;
    CUtensorMap tmS;
    memset(&tmS, 0, sizeof(tmS));
    if (STAGED) {  // ssm as a [rows][128] fp32 matrix, box {W, 128} (one state block), no swizzle
        auto enc = tc::tmap_encode_fn();
        const cuuint64_t dims[2] = {(cuuint64_t)kDv, (cuuint64_t)p.ssm_rows};
        const cuuint64_t strides[1] = {(cuuint64_t)kDv * 4};
        const cuuint32_t box[2] = {(cuuint32_t)(kDv / NSPLIT), (cuuint32_t)kDk};
        const cuuint32_t estr[2] = {1, 1};
        if (!enc || (uintptr_t)p.ssm % 16 ||
            enc(&tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.ssm, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
                CUDA_SUCCESS)
            return ANELM_ERR_CUDA;
        cudaFuncSetAttribute(gdn_decode_kernel<RATIO, NSPLIT, THREADS, STAGED>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((long long)n_rows * p.Hk * CS));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_decode_kernel<RATIO, NSPLIT, THREADS, STAGED>, p, tmS);
    return e == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

}  // namespace

int launch_gdn_decode(const GdnDecodeParams& p, int n_rows, int key_dim, int val_dim, cudaStream_t stream) {
    if (key_dim != kDk || val_dim != kDv) return ANELM_ERR_UNSUPPORTED;
    const int ratio = p.Hv / p.Hk;
    // Column blocks per value head and threads per CTA.  Few rows: narrow blocks to spread
    // the state over more SMs; many rows: wide blocks so each CTA's serial chain (conv,
    // norms, two reductions, two cluster barriers) covers more bytes.
    int nsplit = 0, threads = 0;
    if (const char* e = getenv("ANELM_GDN_SPLIT")) {  // tuning override "nsplit,threads"
        if (sscanf(e, "%d,%d", &nsplit, &threads) != 2) nsplit = threads = 0;
    }
    const bool small = (long long)n_rows * p.Hv * 4 < 2 * 148;
    if (!nsplit) {  // measured on B200: 2 x 128 is fastest for 256 rows (60% of HBM peak vs 52% for 2 x 256)
        nsplit = small ? (ratio == 1 ? 8 : 4) : 2;
        threads = 128;
        if (ratio == 4) nsplit = 2;
    }
    // staged state blocks (TMA in / out through shared memory) for wide batches: measured on B200 for the
    // 4B shape (32 value heads), one layer: 256 rows 0.190 vs 0.217 ms, 128 rows 0.103 vs 0.113; at 64
    // rows (4,096 CTAs) and fewer the register form is slightly ahead (32 rows 0.0276 vs 0.0294 ms).
    // Override with ANELM_GDN_STAGED=0 / 1
    bool staged = !small && nsplit == 2 && threads == 128 && (long long)n_rows * p.Hv * nsplit >= 6144;
    if (const char* e = getenv("ANELM_GDN_STAGED"))
        staged = atoi(e) != 0 && !small && nsplit == 2 && threads == 128;
    if (staged && ratio == 2) return launch_cfg<2, 2, 128, true>(p, n_rows, stream);
    if (staged && ratio == 1) return launch_cfg<1, 2, 128, true>(p, n_rows, stream);
#define GDN_CASE(R, NS, T) \
    if (ratio == R && nsplit == NS && threads == T) return launch_cfg<R, NS, T, false>(p, n_rows, stream);
    GDN_CASE(1, 8, 128) GDN_CASE(1, 4, 128) GDN_CASE(1, 4, 256) GDN_CASE(1, 2, 256) GDN_CASE(1, 2, 128)
    GDN_CASE(2, 4, 128) GDN_CASE(2, 4, 256) GDN_CASE(2, 2, 128) GDN_CASE(2, 2, 256)
    GDN_CASE(4, 2, 128) GDN_CASE(4, 2, 256)
#undef GDN_CASE
    return ANELM_ERR_UNSUPPORTED;
}

}  // namespace anelm
