// bf16 GEMM C = A B^T on tcgen05 (sm_100a): the projections on either side of the attention core.
//
// In the reference the Apple Neural Engine runs them: first_proj (hidden -> the q|gate|k|v or
// qkv|z|a|b projection rows the core consumes) and o_proj (core output -> hidden),
// models/llm/qwen3_5.cpp:912-1012 with core/ane_runtime.cpp:279-361 running the compiled
// chunks.  Here they are plain dense GEMMs in the nn.Linear layout, A [M][K] (activations,
// rows = tokens or sequences) times B [N][K] (weights, [out][in]), fp32 accumulation, so the
// projections never leave the device around the core.
//
// One CTA per 128 x 256 output tile, 192 threads: warp 4 streams 128 x 64 tiles of A and 256 x 64
// tiles of B (TMA, 128B swizzle, zero fill past M / N / K) through a 4-stage ring, one thread of
// warp 5 issues tcgen05.mma (M = 128, N = 256, K = 16, both operands K-major from shared memory)
// into a 256-column fp32 accumulator in TMEM and frees each stage with tcgen05.commit, warps 0-3
// read the accumulator (one row per thread) and store it as bf16 / fp16 / fp32.  N = 256 halves the
// operand bytes per FLOP against 128 x 128 tiles (whose loads ran at the L2-to-SM limit).
// Grids of few tiles (decode-size M with a small N) split K over a thread-block cluster of up to
// 8 CTAs per tile: each CTA accumulates its K range in TMEM, parks the fp32 partial in its (now
// idle) stage buffers, and after a cluster barrier each CTA sums its share of the tile's rows over
// all partials through distributed shared memory and stores them.
//
// The LM head with in-model top-k (export_hybrid_chunks.py:409-421, LMHeadArgmax: logits =
// x W^T over the vocabulary, then torch.topk(32), read by serve_hybrid.py:283-307) reuses the
// same tiles in a persistent kernel: each CTA walks a strided set of 256-column vocabulary tiles
// for its 128 rows, with two TMEM accumulators so that the MMAs of tile i+1 run while the
// epilogue folds tile i into each row's running top-32 (kept sorted in registers); it writes one
// candidate list per row, and lm_topk_merge_kernel reduces the CTAs' lists to the row's top-k.
// The vocabulary logits never reach memory.  Every mbarrier wait
// is bounded and reports ANELM_ERR_TIMEOUT.
#include <algorithm>
#include <climits>
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

namespace anelm {

namespace {

constexpr int kGBM = 128, kGBN = 256, kGBK = 64, kGStages = 4;
constexpr int kGThreads = 192;
constexpr int kGTileA = kGBM * kGBK * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int kGTileB = kGBN * kGBK * 2;  // 32 KB: 256 rows x 128 bytes
constexpr int kGroupM = 16;          // row tiles per raster band of a multi-wave GEMM
constexpr int kGMaxStages = 8;         // projection GEMM: stages in flight for narrow B tiles
constexpr int kGSmemMax = 227 * 1024;  // dynamic shared memory per CTA
constexpr int kGPartPitch = kGBN + 4;  // fp32 words per row of a parked split-K partial
// LM head: stage ring, barriers, and a buffer of (value, index) entries per row for the epilogue
// (32 entries + 1 of padding, so rows whose counts agree write different banks)
constexpr int kLmBufPitch = 33;
constexpr int kLmSmem = kGStages * (kGTileA + kGTileB) + 256 + 128 * kLmBufPitch * 8 + 128 * 4 + 1024;
constexpr unsigned long long kLmTauWaitNs = 20000;  // longest wait for the other CTAs' first-tile maxima
static_assert(kLmSmem <= kGSmemMax, "LM-head stages and row buffers fit in shared memory");
static_assert(kGBM * kGPartPitch * 4 <= kGStages * (kGTileA + kGTileB), "partial fits the stage buffers");

// kind::f16 instruction descriptor with bf16 A and B (formats 1), fp32 D, both K-major
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return tc::idesc_f16_f32(M, N) | (1u << 7) | (1u << 10);
}

// Every top-k with k <= 32 is the head of the top-32, so the running lists always hold 32.
constexpr int kTopK = 32;

// kNarrow: tile width bn and stage count nst as given (one partial wave of narrower tiles);
// otherwise the compile-time 256 columns and kGStages stages.
template <bool kNarrow>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* C,
                        long long ldc, int c_dtype, int M, int N, int K, int ks, int bn_arg, int nst_arg, int* err) {
    // nst stages of [A 128 x 64 | B bn x 64] (narrower B tiles leave room for more stages in flight)
    const int bn = kNarrow ? bn_arg : kGBN;
    const int nst = kNarrow ? nst_arg : kGStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tileB = bn * kGBK * 2;
    uint8_t* sA = smem;
    uint8_t* sB = smem + nst * kGTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + nst * tileB);
    uint64_t* empty = full + kGMaxStages;
    uint64_t* done = empty + kGMaxStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // ks > 1: blockIdx.x = tile * ks + split, the ks CTAs of a tile form one cluster
    const int split = blockIdx.x % ks;
    const int n0 = (blockIdx.x / ks) * bn, m0 = blockIdx.y * kGBM;
    const int nk_all = (K + kGBK - 1) / kGBK;
    const int per = (nk_all + ks - 1) / ks;
    const int kt0 = split * per;
    const int nk = max(0, min(nk_all, kt0 + per) - kt0);  // this CTA's k-tiles
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < nst; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(done, 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kGBN);  // bn <= 256 columns used
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {  // TMA producer
            tc::prefetch_tmap(&tmA);
            tc::prefetch_tmap(&tmB);
            // stage s and its use count u (kt = u * nst + s), stepped without division
            for (int kt = 0, s = 0, u = 0; kt < nk; kt++) {
                if (u > 0 && !tc::mbar_wait(&empty[s], (uint32_t)(u - 1) & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
                tc::mbar_arrive_expect_tx(&full[s], kGTileA + tileB);
                tc::tma_load_2d(sA + s * kGTileA, &tmA, &full[s], (kt0 + kt) * kGBK, m0);
                tc::tma_load_2d(sB + s * tileB, &tmB, &full[s], (kt0 + kt) * kGBK, n0);
                if (++s == nst) {
                    s = 0;
                    u++;
                }
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = idesc_bf16_f32(kGBM, bn);
            const uint32_t aA = (uint32_t)__cvta_generic_to_shared(sA), aB = (uint32_t)__cvta_generic_to_shared(sB);
            for (int kt = 0, s = 0, u = 0; kt < nk; kt++) {
                if (!tc::mbar_wait(&full[s], (uint32_t)u & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
                tc::tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < kGBK / 16; ks++)
                    tc::mma_f16_ss(tmem, tc::desc_kmajor_sw128(aA + s * kGTileA + ks * 32),
                                   tc::desc_kmajor_sw128(aB + s * tileB + ks * 32), idesc, (kt | ks) != 0);
                tc::mma_commit(&empty[s]);
                if (++s == nst) {
                    s = 0;
                    u++;
                }
            }
            tc::mma_commit(done);  // all MMAs issued (an aborted loop still completes `done`)
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: thread = accumulator row m0 + 32 warp + lane ----------------
        const bool ok = tc::mbar_wait(done, 0, err, ANELM_ERR_TIMEOUT, abort);
        tc::tc_fence_after();
        const int m = m0 + 32 * warp + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        if (ks > 1) {  // park this split's partial (zeros for an empty K range) in the stage buffers
            float* part = reinterpret_cast<float*>(smem) + (32 * warp + lane) * kGPartPitch;
#pragma unroll 1
            for (int c0 = 0; c0 < bn; c0 += 32) {
                uint32_t x[32];
                const int w = kNarrow ? min(32, bn - c0) : 32;  // 32, or 16 for the last chunk of a bn = 16 (mod 32)
                if (w == 32) tc::tmem_ld32(trow + c0, x); else tc::tmem_ld16(trow + c0, x);
                tc::tmem_ld_wait();
#pragma unroll
                for (int c4 = 0; c4 < 8; c4++)
                    if (c4 < w / 4)
                    *reinterpret_cast<float4*>(part + c0 + 4 * c4) =
                        nk > 0 ? make_float4(__uint_as_float(x[4 * c4]), __uint_as_float(x[4 * c4 + 1]),
                                             __uint_as_float(x[4 * c4 + 2]), __uint_as_float(x[4 * c4 + 3]))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll 1
        for (int c0 = 0; c0 < (ks > 1 ? 0 : bn); c0 += 32) {
            uint32_t x[32];
            const int w = kNarrow ? min(32, bn - c0) : 32;
            if (w == 32) tc::tmem_ld32(trow + c0, x); else tc::tmem_ld16(trow + c0, x);
            tc::tmem_ld_wait();
            if (!ok || m >= M) continue;
            const int nb = n0 + c0;
            if (nb + w <= N && c_dtype != ANELM_F32 && (ldc % 8) == 0 && ((uintptr_t)C % 16) == 0) {
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(C) + (long long)m * ldc + nb);
#pragma unroll
                for (int c8 = 0; c8 < 4; c8++) {
                    if (c8 >= w / 8) break;
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = __uint_as_float(x[8 * c8 + e]);
                    dst[c8] = pack8(v, c_dtype == ANELM_BF16);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; c++)
                    if (c < w && nb + c < N) store_from_float(C, c_dtype, (long long)m * ldc + nb + c, __uint_as_float(x[c]));
            }
        }
    }
    if (ks > 1) {
        // ---------------- split-K: rows [split R, split R + R) summed over the cluster's partials ----------------
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();  // every split's partial is parked
        const int R = (kGBM + ks - 1) / ks;
        const int r0 = split * R, r1 = min(kGBM, r0 + R);
        const float* part0 = reinterpret_cast<const float*>(smem);
        for (int i = tid; i < (r1 - r0) * (bn / 4); i += kGThreads) {
            const int r = r0 + i / (bn / 4), c = 4 * (i % (bn / 4));
            const int m = m0 + r, n = n0 + c;
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < ks; q++) {
                const float4 v = *reinterpret_cast<const float4*>(cl.map_shared_rank(part0 + r * kGPartPitch + c, q));
                s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
            }
            if (m >= M) continue;
            const float o[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (n + e < N) store_from_float(C, c_dtype, (long long)m * ldc + n + e, o[e]);
        }
        cl.sync();  // peers are done reading this CTA's partial
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kGBN);
    }
}

// Persistent form for several waves of 256-wide tiles: one CTA per SM walks tiles c, c + G, ...
// (G = gridDim.x) in the banded order (16 row tiles, column by column).  Warp 4: TMA ring over
// (tile, k-step); warp 5: MMAs of tile i into TMEM accumulator i & 1 once the epilogue released
// it; warps 0-3: drain accumulator i & 1 (row = thread) and store, while the MMAs of tile i + 1
// run into the other accumulator.
__device__ __forceinline__ void banded_tile(int t, int ntn, int mtn, int& mt, int& nt) {
    const int grp = t / (kGroupM * ntn), first_m = grp * kGroupM;
    const int gm = min(mtn - first_m, kGroupM);
    const int r = t - grp * kGroupM * ntn;
    mt = first_m + r % gm;
    nt = r / gm;
}

__global__ void __launch_bounds__(kGThreads, 1)
    gemm_bf16_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                void* C, long long ldc, int c_dtype, int M, int N, int K, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kGStages * kGTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + kGStages * kGTileB);
    uint64_t* empty = full + kGStages;
    uint64_t* tfull = empty + kGStages;  // [2] accumulator b holds a finished tile
    uint64_t* tfree = tfull + 2;         // [2] the epilogue has read accumulator b
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfree + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, g = blockIdx.x;
    const int ntn = (N + kGBN - 1) / kGBN, mtn = (M + kGBM - 1) / kGBM;
    const int ntile = ntn * mtn;
    const int my_tiles = g < ntile ? (ntile - 1 - g) / G + 1 : 0;
    const int nk = (K + kGBK - 1) / kGBK;
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < kGStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tfree[b], 128);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 2 * kGBN);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {  // TMA producer over (tile, k-step), one continuous ring
            tc::prefetch_tmap(&tmA);
            tc::prefetch_tmap(&tmB);
            int s = 0, u = 0;
            for (int i = 0; i < my_tiles && !*abort; i++) {
                int mt, nt;
                banded_tile(g + i * G, ntn, mtn, mt, nt);
                for (int kt = 0; kt < nk; kt++) {
                    if (u > 0 && !tc::mbar_wait(&empty[s], (uint32_t)(u - 1) & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
                    tc::mbar_arrive_expect_tx(&full[s], kGTileA + kGTileB);
                    tc::tma_load_2d(sA + s * kGTileA, &tmA, &full[s], kt * kGBK, mt * kGBM);
                    tc::tma_load_2d(sB + s * kGTileB, &tmB, &full[s], kt * kGBK, nt * kGBN);
                    if (++s == kGStages) {
                        s = 0;
                        u++;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_bf16_f32(kGBM, kGBN);
            const uint32_t aA = (uint32_t)__cvta_generic_to_shared(sA), aB = (uint32_t)__cvta_generic_to_shared(sB);
            int s = 0, u = 0;
            for (int i = 0; i < my_tiles; i++) {
                const int b = i & 1;
                if (i >= 2 && !tc::mbar_wait(&tfree[b], (uint32_t)((i >> 1) - 1) & 1, err, ANELM_ERR_TIMEOUT, abort))
                    break;
                tc::tc_fence_after();
                bool ok = true;
                for (int kt = 0; kt < nk; kt++) {
                    if (!tc::mbar_wait(&full[s], (uint32_t)u & 1, err, ANELM_ERR_TIMEOUT, abort)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kGBK / 16; ks++)
                        tc::mma_f16_ss(tmem + b * kGBN, tc::desc_kmajor_sw128(aA + s * kGTileA + ks * 32),
                                       tc::desc_kmajor_sw128(aB + s * kGTileB + ks * 32), idesc, (kt | ks) != 0);
                    tc::mma_commit(&empty[s]);
                    if (++s == kGStages) {
                        s = 0;
                        u++;
                    }
                }
                tc::mma_commit(&tfull[b]);  // an aborted loop still completes the tile's barrier
                if (!ok) break;
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: thread = row 32 warp + lane of each tile ----------------
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        const bool vec = c_dtype != ANELM_F32 && (ldc % 8) == 0 && ((uintptr_t)C % 16) == 0;
        for (int i = 0; i < my_tiles; i++) {
            const int b = i & 1;
            int mt, nt;
            banded_tile(g + i * G, ntn, mtn, mt, nt);
            const int m = mt * kGBM + 32 * warp + lane;
            if (!tc::mbar_wait(&tfull[b], (uint32_t)(i >> 1) & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
            tc::tc_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < kGBN; c0 += 32) {
                uint32_t x[32];
                tc::tmem_ld32(trow + b * kGBN + c0, x);
                tc::tmem_ld_wait();
                if (c0 == kGBN - 32) {  // every column of accumulator b is read: the MMAs may reuse it
                    tc::tc_fence_before();
                    tc::mbar_arrive(&tfree[b]);
                }
                if (m >= M) continue;
                const int nb = nt * kGBN + c0;
                if (nb + 32 <= N && vec) {
                    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(C) + (long long)m * ldc + nb);
#pragma unroll
                    for (int c8 = 0; c8 < 4; c8++) {
                        float v[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) v[e] = __uint_as_float(x[8 * c8 + e]);
                        dst[c8] = pack8(v, c_dtype == ANELM_BF16);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c++)
                        if (nb + c < N) store_from_float(C, c_dtype, (long long)m * ldc + nb + c, __uint_as_float(x[c]));
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * kGBN);
    }
}

// Few-row products (M <= kGvMaxM): C[m][n] = sum_k A[m][k] B[n][k] on the CUDA cores.  A 128-row
// tensor-core tile would be almost all padding; the cost is streaming B (the weights) from HBM.
// The M rows of A are staged in shared memory (bf16); each warp walks groups of kGvRows rows of B
// (grid-stride over all warps of a grid sized to the resident capacity, so no partial last
// wave), kGvUnroll 16-byte loads per row in flight, fp32 accumulation, one warp reduction per output.
constexpr int kGvRows = 2, kGvUnroll = 4, kGvThreads = 256, kGvMaxM = 4;
constexpr int kGvBlocksPerSm = 2;  // few-row LM head: CTAs per SM (128 registers a thread)
constexpr int kLmGvRows = 4, kLmGvUnroll = 4;  // its vocabulary rows per warp, loads in flight per row
constexpr int kLmGemvRows = 1;      // LM head rows that take the CUDA-core path (at 4 rows the
                                    // tensor-core path is faster: 380 vs 464 us at 248,320 x 2560)

__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__global__ void __launch_bounds__(kGvThreads) gemv_bf16_kernel(const __nv_bfloat16* A, long long lda,
                                                               const __nv_bfloat16* B, long long ldb, void* C,
                                                               long long ldc, int c_dtype, int M, int N, int K) {
    extern __shared__ uint4 xs[];  // [M][K / 8]
    const int kc = K / 8;
    for (int i = threadIdx.x; i < M * kc; i += kGvThreads) {
        const int m = i / kc, c = i - m * kc;
        xs[i] = *reinterpret_cast<const uint4*>(A + (long long)m * lda + (long long)c * 8);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * (kGvThreads / 32);
    for (int n0 = (blockIdx.x * (kGvThreads / 32) + warp) * kGvRows; n0 < N; n0 += nwarps * kGvRows) {
    const uint4* brow[kGvRows];
#pragma unroll
    for (int r = 0; r < kGvRows; r++)
        brow[r] = reinterpret_cast<const uint4*>(B + (long long)min(n0 + r, N - 1) * ldb);
    float acc[kGvRows][kGvMaxM];
#pragma unroll
    for (int r = 0; r < kGvRows; r++)
#pragma unroll
        for (int m = 0; m < kGvMaxM; m++) acc[r][m] = 0.f;
    for (int c0 = lane; c0 < kc; c0 += 32 * kGvUnroll) {
        uint4 w[kGvRows][kGvUnroll];
#pragma unroll
        for (int u = 0; u < kGvUnroll; u++)
#pragma unroll
            for (int r = 0; r < kGvRows; r++)
                w[r][u] = (c0 + 32 * u < kc) ? ld_stream16(brow[r] + c0 + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < kGvUnroll; u++) {
            const int c = c0 + 32 * u;
            if (c >= kc) break;
            float wf[kGvRows][8];
#pragma unroll
            for (int r = 0; r < kGvRows; r++) unpack8(w[r][u], true, wf[r]);
#pragma unroll
            for (int m = 0; m < kGvMaxM; m++) {
                if (m >= M) break;
                float xf[8];
                unpack8(xs[m * kc + c], true, xf);
#pragma unroll
                for (int r = 0; r < kGvRows; r++)
#pragma unroll
                    for (int e = 0; e < 8; e++) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kGvRows; r++)
#pragma unroll
        for (int m = 0; m < kGvMaxM; m++) {
            if (m >= M) break;
            const float s = warp_sum(acc[r][m]);
            if (lane == 0 && n0 + r < N) store_from_float(C, c_dtype, (long long)m * ldc + n0 + r, s);
        }
    }
}

// 2D bf16 tensor map over a row-major [rows][cols] matrix (row stride ld elements), box {64, box_rows}
bool make_bf16_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    auto fn = tc::tmap_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kGBK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_gemm_bf16_tn(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int c_dtype,
                        int M, int N, int K, int* err, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0) return ANELM_ERR_INVALID_ARG;
    if ((uintptr_t)A % 16 || (uintptr_t)B % 16 || (lda * 2) % 16 || (ldb * 2) % 16 || lda < K || ldb < K || ldc < N)
        return ANELM_ERR_UNSUPPORTED;
    if (M <= kGvMaxM && K % 8 == 0 && (size_t)M * K * 2 <= 160 * 1024) {
        // few rows: stream the weights on the CUDA cores
        const int smem = M * K * 2;
        if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        const int rows_per_block = kGvRows * (kGvThreads / 32);
        int dev = 0, sms = 148, per_sm = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_bf16_kernel, kGvThreads, smem) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        const int blocks = std::min((N + rows_per_block - 1) / rows_per_block, sms * per_sm);
        gemv_bf16_kernel<<<blocks, kGvThreads, smem, stream>>>(
            static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(B), ldb, C, ldc, c_dtype, M,
            N, K);
        return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
    }
    const int mt = (M + kGBM - 1) / kGBM;
    const int tiles = ((N + kGBN - 1) / kGBN) * mt;
    const int nk = (K + kGBK - 1) / kGBK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // tile width: when the 256-wide tiles make one partial wave (half the SMs to all of them), the
    // width in [128, 256] (step 16) with the fewest columns per SM (waves x width): e.g. M = 256,
    // N = 10240 takes 144 tiles of 144 columns instead of 80 tiles of 256; fewer tiles than that
    // split K instead (below); several waves keep 256
    int bn = kGBN;
    if (2 * tiles >= sms && tiles <= sms) {
        long long best = -1;
        for (int b = kGBN; b >= 128; b -= 16) {
            const long long t = (long long)mt * ((N + b - 1) / b);
            const long long cost = ((t + sms - 1) / sms) * b;
            if (best < 0 || cost < best) {
                best = cost;
                bn = b;
            }
        }
    }
    // narrower tiles: as many stages as shared memory holds (at most kGMaxStages)
    const int nst = bn == kGBN ? kGStages
                               : std::min(kGMaxStages, (kGSmemMax - 1280) / (kGTileA + bn * kGBK * 2));
    const int smem = nst * (kGTileA + bn * kGBK * 2) + 256 + 1024;  // + barriers, alignment
    auto kern = bn == kGBN ? gemm_bf16_tn_kernel<false> : gemm_bf16_tn_kernel<true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    CUtensorMap mA, mB;
    if (!make_bf16_map(&mA, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, kGBM) ||
        !make_bf16_map(&mB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, (uint32_t)bn))
        return ANELM_ERR_CUDA;
    if (tiles > sms) {  // several waves of 256-wide tiles: one persistent CTA per SM
        constexpr int psmem = kGStages * (kGTileA + kGTileB) + 256 + 1024;
        cudaFuncSetAttribute(gemm_bf16_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, psmem);
        gemm_bf16_persistent_kernel<<<sms, kGThreads, psmem, stream>>>(mA, mB, C, ldc, c_dtype, M, N, K, err);
        return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
    }
    // split K over a cluster when the tiles fill less than half of the SMs: the largest cluster
    // size (<= 8) of which the GPU can hold one cluster per tile at once (GPC packing caps it below
    // the SM count / tiles), measured once per device and size
    int ks = 1;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (2 * tiles < sms) {
        static int active[16][9];  // [device][cluster size]: clusters resident at once (0 = not measured)
        for (int c = std::min(8, std::min(nk, sms / tiles)); c >= 2 && ks == 1; c--) {
            int& a = active[dev & 15][c];
            if (a == 0) {
                cfg.gridDim = dim3(c, 1);
                attr[0].val.clusterDim.x = c;
                if (cudaOccupancyMaxActiveClusters(&a, (void*)kern, &cfg) != cudaSuccess || a <= 0) {
                    cudaGetLastError();
                    a = -1;
                }
            }
            if (a >= tiles) ks = c;
        }
        if (ks > 1) ks = (nk + ((nk + ks - 1) / ks) - 1) / ((nk + ks - 1) / ks);  // no empty K range
    }
    if (ks > 1) {
        cfg.gridDim = dim3(((N + kGBN - 1) / kGBN) * ks, (M + kGBM - 1) / kGBM);
        attr[0].val.clusterDim.x = ks;
        if (cudaLaunchKernelEx(&cfg, kern, mA, mB, C, ldc, c_dtype, M, N, K, ks, bn, nst, err) == cudaSuccess)
            return ANELM_OK;
        cudaGetLastError();  // a cluster that cannot be placed: one CTA per tile instead
    }
    dim3 grid((N + bn - 1) / bn, mt);
    kern<<<grid, kGThreads, smem, stream>>>(mA, mB, C, ldc, c_dtype, M, N, K, 1, bn, nst, err);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

namespace {

// Running top-32 of one row spread over a warp: lane j holds the j-th largest (value, index).
// Branch-free form: every lane runs every shuffle whatever `valid` is (valid, v, id warp-uniform).
__device__ __forceinline__ void warp_topk_insert_if(float& tv, int& ti, bool valid, float v, int id, int lane) {
    const bool ok = valid && v > __shfl_sync(0xffffffffu, tv, 31);
    const unsigned lt = __ballot_sync(0xffffffffu, tv < v);
    const int pos = lt ? __ffs(lt) - 1 : 32;
    const float up_v = __shfl_up_sync(0xffffffffu, tv, 1);
    const int up_i = __shfl_up_sync(0xffffffffu, ti, 1);
    const float nv = lane > pos ? up_v : (lane == pos ? v : tv);
    const int ni = lane > pos ? up_i : (lane == pos ? id : ti);
    tv = ok ? nv : tv;
    ti = ok ? ni : ti;
}
// Order of the running lists: a before b when a's value is larger, or equal with the smaller index.
// Folding columns in ascending order by insertion (ties kept behind the earlier entry) and taking the
// top 32 of a union under this order give the same list.
__device__ __forceinline__ bool key_gt(float av, int ai, float bv, int bi) {
    return av > bv || (av == bv && ai < bi);
}

// Bitonic sort of four rows at once, one element per lane, ascending under key_gt (lane 0 smallest);
// the rows' shuffle chains interleave.
__device__ __forceinline__ void warp_sort4_asc(float (&v)[4], int (&s)[4], int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const bool keep_min = ((lane & j) == 0) == ((lane & k) == 0);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float pv = __shfl_xor_sync(0xffffffffu, v[q], j);
                const int ps = __shfl_xor_sync(0xffffffffu, s[q], j);
                const bool take = keep_min != key_gt(pv, ps, v[q], s[q]);
                v[q] = take ? pv : v[q];
                s[q] = take ? ps : s[q];
            }
        }
    }
}

// Merge of 32 candidates sorted ascending (cv, ci) into the descending list (tv, ti): the larger of
// list entry j and candidate j is the top 32 of the union as a bitonic sequence, which five
// half-cleaner steps sort descending.
__device__ __forceinline__ void warp_merge_sorted(float& tv, int& ti, float cv, int ci, int lane) {
    const bool c = key_gt(cv, ci, tv, ti);
    float v = c ? cv : tv;
    int i = c ? ci : ti;
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const float pv = __shfl_xor_sync(0xffffffffu, v, j);
        const int pi = __shfl_xor_sync(0xffffffffu, i, j);
        const bool take = ((lane & j) == 0) == key_gt(pv, pi, v, i);
        v = take ? pv : v;
        i = take ? pi : i;
    }
    tv = v;
    ti = i;
}

__device__ __forceinline__ void warp_topk_insert(float& tv, int& ti, float v, int id, int lane) {
    // v and id are the same in every lane; the list is sorted descending across lanes
    if (!(v > __shfl_sync(0xffffffffu, tv, 31))) return;
    const int pos = __ffs(__ballot_sync(0xffffffffu, tv < v)) - 1;  // first lane below v (a suffix)
    const float up_v = __shfl_up_sync(0xffffffffu, tv, 1);
    const int up_i = __shfl_up_sync(0xffffffffu, ti, 1);
    if (lane > pos) {
        tv = up_v;
        ti = up_i;
    } else if (lane == pos) {
        tv = v;
        ti = id;
    }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// Persistent LM-head kernel: CTA (g, mt) handles vocabulary tiles g, g + G, ... (G = gridDim.x)
// for rows [128 mt, 128 mt + 128).  Warp 4: TMA ring (A rows, B vocabulary rows); warp 5: MMAs
// of each tile into TMEM buffer (i & 1) once the epilogue released it; warps 0-3: per row, the
// running top-32 over all its tiles (spread over a warp's lanes), then candidate lists
// [M][G rep][32] (values, then indices).  With rep > 1 (one row tile of at most 128 / rep rows; the
// launcher takes rep = 4 for 9-24 rows) the A tile holds rep copies of the rr = 128 / rep row block
// (one TMA box each, tmA's box is rr rows), so every epilogue warp has rows: the warps reading copy
// cp take columns [cp 256 / rep, (cp + 1) 256 / rep) of each tile and keep their own list (copy cp's
// list of CTA g is candidate list g rep + cp).
//
// Before any list is fed, every CTA publishes each row's largest logit of its first tile (pmax
// [M][gpitch], slot g; NaN = not yet published, set by the launcher) and waits, at most
// kLmTauWaitNs, for the other CTAs' maxima (arrive counts the publishing warps).  For a row, the
// maxima in slots j, j + 32, ... (j = 0..31) form 32 disjoint groups of columns; the smallest of the
// 32 group maxima is the 32nd largest of 32 distinct logits, so no logit below it can be among the
// row's top 32.  The lists then only take logits at or above that bound (ties kept), and being
// the top 32 under key_gt of those, they still merge to the exact top 32.  A CTA that stops
// waiting uses what is published by then: a weaker bound, the same result.
__global__ void __launch_bounds__(kGThreads, 1)
    lm_head_topk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, float* cand,
                        float* pmax, int gpitch, unsigned* arrive, int M, int N, int K, int rep, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kGStages * kGTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + kGStages * kGTileB);
    uint64_t* empty = full + kGStages;
    uint64_t* tfull = empty + kGStages;  // [2] accumulator b holds a finished tile
    uint64_t* tfree = tfull + 2;         // [2] the epilogue has read accumulator b
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfree + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* rows = reinterpret_cast<float*>(tmem_slot + 4);  // [128 rows][kLmBufPitch] (value, index) buffers
    float* pub = rows + 128 * kLmBufPitch * 2;              // [4 warps][32] first-tile maxima
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, g = blockIdx.x, m0 = blockIdx.y * kGBM;
    const int ntile = (N + kGBN - 1) / kGBN;
    const int my_tiles = g < ntile ? (ntile - 1 - g) / G + 1 : 0;
    const int nk = (K + kGBK - 1) / kGBK;
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < kGStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tfree[b], 128);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 2 * kGBN);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {  // TMA producer over (tile, k-step), one continuous ring
            tc::prefetch_tmap(&tmA);
            tc::prefetch_tmap(&tmB);
            long long q = 0;
            for (int i = 0; i < my_tiles && !*abort; i++) {
                const int n0 = (g + i * G) * kGBN;
                for (int kt = 0; kt < nk; kt++, q++) {
                    const int s = (int)(q % kGStages);
                    if (q >= kGStages &&
                        !tc::mbar_wait(&empty[s], (uint32_t)((q / kGStages) - 1) & 1, err, ANELM_ERR_TIMEOUT, abort))
                        break;
                    tc::mbar_arrive_expect_tx(&full[s], kGTileA + kGTileB);
                    for (int c = 0; c < rep; c++)  // rep boxes of kGBM / rep rows (whole 8-row swizzle atoms)
                        tc::tma_load_2d(sA + s * kGTileA + c * (kGBM / rep) * 128, &tmA, &full[s], kt * kGBK, m0);
                    tc::tma_load_2d(sB + s * kGTileB, &tmB, &full[s], kt * kGBK, n0);
                }
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_bf16_f32(kGBM, kGBN);
            const uint32_t aA = (uint32_t)__cvta_generic_to_shared(sA), aB = (uint32_t)__cvta_generic_to_shared(sB);
            long long q = 0;
            for (int i = 0; i < my_tiles; i++) {
                const int b = i & 1;
                if (i >= 2 && !tc::mbar_wait(&tfree[b], (uint32_t)((i >> 1) - 1) & 1, err, ANELM_ERR_TIMEOUT, abort))
                    break;
                tc::tc_fence_after();
                bool ok = true;
                for (int kt = 0; kt < nk; kt++, q++) {
                    const int s = (int)(q % kGStages);
                    if (!tc::mbar_wait(&full[s], (uint32_t)(q / kGStages) & 1, err, ANELM_ERR_TIMEOUT, abort)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kGBK / 16; ks++)
                        tc::mma_f16_ss(tmem + b * kGBN, tc::desc_kmajor_sw128(aA + s * kGTileA + ks * 32),
                                       tc::desc_kmajor_sw128(aB + s * kGTileB + ks * 32), idesc, (kt | ks) != 0);
                    tc::mma_commit(&empty[s]);
                }
                tc::mma_commit(&tfull[b]);
                if (!ok) break;
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: running top-32 of rows 32 warp + r, spread over the warp's lanes ----------------
        // Thread r holds row r's logits of each 16-column half chunk (tcgen05.ld, thread = row) and
        // appends those above its row's 32nd value to the row's buffer in shared memory.  A row
        // whose buffer passes 16 entries (so the next half always fits) has it sorted (bitonic,
        // four rows at a time) and merged into the list in one step, which refreshes the row's
        // threshold; the buffers left at the end are merged the same way.  The list of a row is the
        // top 32 under key_gt of every column it saw, the same as inserting them one by one.
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        float2* buf = reinterpret_cast<float2*>(rows) + warp * 32 * kLmBufPitch;  // [32 rows][pitch] (value, index)
        const int rr = kGBM / rep;                    // rows per copy of the A block
        const int cp = (32 * warp) / rr;              // the copy this warp's TMEM lanes hold
        const int rbase = (32 * warp) % rr;           // its first row within the copy
        const int cbeg = cp * (kGBN / rep), cend = cbeg + kGBN / rep;  // its columns of every tile
        const int nrow = M - (m0 + rbase);            // rows of this warp inside the matrix
        float lv[32];
        int li[32];
#pragma unroll
        for (int r = 0; r < 32; r++) {
            lv[r] = -INFINITY;
            li[r] = -1;
        }
        // ---- the rows' lower bounds from every CTA's first-tile maxima ----
        float my_max = -INFINITY;  // row `lane`'s largest logit among this warp's columns of the first tile
        if (tc::mbar_wait(&tfull[0], 0, err, ANELM_ERR_TIMEOUT, abort)) {
            tc::tc_fence_after();
            const int n0 = g * kGBN;
#pragma unroll 1
            for (int c = cbeg; c < cend; c += 16) {
                uint32_t x[16];
                tc::tmem_ld16(trow + c, x);
                tc::tmem_ld_wait();
                const int lim = N - (n0 + c);
#pragma unroll
                for (int k = 0; k < 16; k++)
                    if (k < lim) my_max = fmaxf(my_max, __uint_as_float(x[k]));
            }
        }
        pub[warp * 32 + lane] = my_max;
        tc::named_bar_sync(1, 128);
        if (cp == 0) {  // the warps of copy 0 publish their rows' maxima over the rep copies
#pragma unroll 1
            for (int k = 1; k < rep; k++) my_max = fmaxf(my_max, pub[(warp + k * (rr / 32)) * 32 + lane]);
            if (lane < nrow) pmax[(long long)(m0 + rbase + lane) * gpitch + g] = my_max;
            __syncwarp();
            if (lane == 0) {
                __threadfence();
                atomicAdd(arrive, 1u);
            }
        }
        if (lane == 0) {
            const unsigned total = gridDim.x * gridDim.y * (4 / rep);
            const unsigned long long t0 = globaltimer_ns();
            while (ld_acquire_gpu(arrive) < total && globaltimer_ns() - t0 < kLmTauWaitNs) __nanosleep(128);
        }
        __syncwarp();
        float my_tau = -INFINITY;  // row `lane`'s bound: min over groups j of max(pmax[row][j + 32 t])
        if (lane < nrow) {
            const float* prow = pmax + (long long)(m0 + rbase + lane) * gpitch;
            float grp[32];
#pragma unroll
            for (int j = 0; j < 32; j++) grp[j] = -INFINITY;
#pragma unroll 1
            for (int t0 = 0; t0 < G; t0 += 32) {  // 32 slots (8 float4) a batch, slot t in group t % 32
                float4 q[8];
#pragma unroll
                for (int u = 0; u < 8; u++)
                    q[u] = t0 + 4 * u < G ? __ldcg(reinterpret_cast<const float4*>(prow + t0) + u)
                                          : make_float4(NAN, NAN, NAN, NAN);
#pragma unroll
                for (int u = 0; u < 8; u++) {  // slots past G (padding of the row pitch) hold NaN
                    grp[4 * u] = fmaxf(grp[4 * u], q[u].x);
                    grp[4 * u + 1] = fmaxf(grp[4 * u + 1], q[u].y);
                    grp[4 * u + 2] = fmaxf(grp[4 * u + 2], q[u].z);
                    grp[4 * u + 3] = fmaxf(grp[4 * u + 3], q[u].w);
                }
            }
            my_tau = grp[0];
#pragma unroll
            for (int j = 1; j < 32; j++) my_tau = fminf(my_tau, grp[j]);
        }
        // v >= tau as one strict compare: the float just below tau (-inf stays -inf)
        const float tau_lo = my_tau > -INFINITY ? nextafterf(my_tau, -INFINITY) : -INFINITY;
        float my_thr = lane < nrow ? tau_lo : INFINITY;  // row `lane`'s admission bound (+inf: no such row)
        int my_cnt = 0;                                  // entries in row `lane`'s buffer
        float2* my_buf = buf + lane * kLmBufPitch;
        const float2 pad = make_float2(-INFINITY, __int_as_float(INT_MAX));
        int i = 0, c0 = cbeg;  // the next tile and half chunk
        for (;;) {
            const bool last = i >= my_tiles;  // every tile read: merge what the buffers still hold
            unsigned need;
            if (!last) {
                const int b = i & 1, n0 = (g + i * G) * kGBN;
                if (c0 == cbeg) {
                    if (!tc::mbar_wait(&tfull[b], (uint32_t)(i >> 1) & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
                    tc::tc_fence_after();
                }
                uint32_t x[16];
                tc::tmem_ld16(trow + b * kGBN + c0, x);
                tc::tmem_ld_wait();
                if (c0 + 16 == cend) {  // this warp's last read of accumulator b: the MMAs may reuse it
                    tc::tc_fence_before();
                    tc::mbar_arrive(&tfree[b]);
                }
                const int lim = N - (n0 + c0);  // columns of this half inside the vocabulary
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const float v = __uint_as_float(x[c]);
                    if (c < lim && v > my_thr) {
                        my_buf[my_cnt] = make_float2(v, __int_as_float(n0 + c0 + c));
                        my_cnt++;
                    }
                }
                need = __ballot_sync(0xffffffffu, my_cnt > 16);
                c0 += 16;
                if (c0 == cend) {
                    c0 = cbeg;
                    i++;
                }
            } else {
                need = __ballot_sync(0xffffffffu, my_cnt > 0);
            }
            if (need) {
                __syncwarp();  // the rows' appends are visible to the whole warp
                // sort each chosen row's buffer ascending (the unused slots as padding), four rows at
                // a time, in place
                unsigned pend = need;
                while (pend) {
                    int rs[4];
                    float cv[4];
                    int ci[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        rs[q] = pend ? __ffs(pend) - 1 : 32;
                        pend &= pend - 1;
                        const int cnt = __shfl_sync(0xffffffffu, my_cnt, rs[q] & 31);
                        const float2 e = rs[q] < 32 && lane < cnt ? buf[rs[q] * kLmBufPitch + lane] : pad;
                        cv[q] = e.x;
                        ci[q] = __float_as_int(e.y);
                    }
                    warp_sort4_asc(cv, ci, lane);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (rs[q] < 32) buf[rs[q] * kLmBufPitch + lane] = make_float2(cv[q], __int_as_float(ci[q]));
                }
                __syncwarp();
                // merge them into the lists, four rows' shuffle chains together, and refresh the thresholds
#pragma unroll
                for (int r0 = 0; r0 < 32; r0 += 4) {
                    if (!((need >> r0) & 0xFu)) continue;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float2 e = (need >> (r0 + q)) & 1u ? buf[(r0 + q) * kLmBufPitch + lane] : pad;
                        warp_merge_sorted(lv[r0 + q], li[r0 + q], e.x, __float_as_int(e.y), lane);
                    }
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float t = __shfl_sync(0xffffffffu, lv[r0 + q], 31);
                        my_thr = lane == r0 + q && ((need >> (r0 + q)) & 1u) ? fmaxf(t, tau_lo) : my_thr;
                    }
                }
                my_cnt = (need >> lane) & 1u ? 0 : my_cnt;
                __syncwarp();  // the merged buffers are read before they are refilled
            }
            if (last) break;
        }
#pragma unroll
        for (int r = 0; r < 32; r++) {
            const int m = m0 + rbase + r;
            if (r < nrow) {
                const long long slot = ((long long)m * G + g) * rep + cp;
                cand[slot * kTopK + lane] = lv[r];
                reinterpret_cast<int*>(cand + (long long)M * G * rep * kTopK)[slot * kTopK + lane] = li[r];
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * kGBN);
    }
}

// LM head for a few rows (up to 16; the launcher takes it for 2-8) with the roles swapped:
// D^T [128 vocabulary rows][16] = W_tile . h^T, so the
// streamed weights are the M = 128 operand (16 KB a k-step, kLsStages of them in flight) and the
// rows of h the N = 16 operand, loaded once for the whole K and kept in shared memory.  TMEM lane =
// vocabulary row, column = row of h: epilogue warp w reads its 32 vocabulary rows of a tile with
// one tcgen05.ld and keeps, per row of h, a running top-32 spread over its lanes (a ballot over the
// 32 logits, survivors inserted); its lists are candidate lists g 4 + w.  Warp 4: TMA (h once, then
// the weight ring); warp 5: MMAs into one of kLsBufs 16-column accumulators per tile.
constexpr int kLsN = 16, kLsBM = 128, kLsStages = 8, kLsBufs = 4;
constexpr int kLsTileW = kLsBM * kGBK * 2;  // 16 KB
constexpr int kLsTileH = kLsN * kGBK * 2;   // 2 KB: 16 rows x 128 bytes (two swizzle atoms)
static size_t lm_swap_smem(int K) { return (size_t)kLsStages * kLsTileW + (size_t)((K + kGBK - 1) / kGBK) * kLsTileH + 256 + 1024; }

__global__ void __launch_bounds__(kGThreads, 1)
    lm_head_swap_topk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmH,
                             float* cand, int M, int N, int K, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nk = (K + kGBK - 1) / kGBK;
    uint8_t* sW = smem;
    uint8_t* sH = smem + kLsStages * kLsTileW;
    uint64_t* full = reinterpret_cast<uint64_t*>(sH + nk * kLsTileH);
    uint64_t* empty = full + kLsStages;
    uint64_t* tfull = empty + kLsStages;  // [kLsBufs]
    uint64_t* tfree = tfull + kLsBufs;    // [kLsBufs]
    uint64_t* hfull = tfree + kLsBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(hfull + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, g = blockIdx.x;
    const int ntile = (N + kLsBM - 1) / kLsBM;
    const int my_tiles = g < ntile ? (ntile - 1 - g) / G + 1 : 0;
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < kLsStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kLsBufs; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tfree[b], 128);
        }
        tc::mbar_init(hfull, 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kLsBufs * kLsN);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {  // TMA: the rows of h for every k-step (rows >= M zero-filled), then the weight ring
            tc::prefetch_tmap(&tmW);
            tc::prefetch_tmap(&tmH);
            tc::mbar_arrive_expect_tx(hfull, (uint32_t)(nk * kLsTileH));
            for (int kt = 0; kt < nk; kt++) tc::tma_load_2d(sH + kt * kLsTileH, &tmH, hfull, kt * kGBK, 0);
            int s = 0;
            uint32_t ph = 0;
            long long q = 0;
            for (int i = 0; i < my_tiles && !*abort; i++) {
                const int r0 = (g + i * G) * kLsBM;
                for (int kt = 0; kt < nk; kt++, q++) {
                    if (q >= kLsStages && !tc::mbar_wait(&empty[s], ph ^ 1u, err, ANELM_ERR_TIMEOUT, abort)) break;
                    tc::mbar_arrive_expect_tx(&full[s], kLsTileW);
                    tc::tma_load_2d(sW + s * kLsTileW, &tmW, &full[s], kt * kGBK, r0);
                    if (++s == kLsStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_bf16_f32(kLsBM, kLsN);
            const uint32_t aW = (uint32_t)__cvta_generic_to_shared(sW), aH = (uint32_t)__cvta_generic_to_shared(sH);
            bool ok = tc::mbar_wait(hfull, 0, err, ANELM_ERR_TIMEOUT, abort);
            int s = 0;
            uint32_t ph = 0;
            for (int i = 0; i < my_tiles && ok; i++) {
                const int b = i % kLsBufs;
                if (i >= kLsBufs &&
                    !tc::mbar_wait(&tfree[b], (uint32_t)((i / kLsBufs) - 1) & 1, err, ANELM_ERR_TIMEOUT, abort))
                    break;
                tc::tc_fence_after();
                for (int kt = 0; kt < nk; kt++) {
                    if (!tc::mbar_wait(&full[s], ph, err, ANELM_ERR_TIMEOUT, abort)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kGBK / 16; ks++)
                        tc::mma_f16_ss(tmem + b * kLsN, tc::desc_kmajor_sw128(aW + s * kLsTileW + ks * 32),
                                       tc::desc_kmajor_sw128(aH + kt * kLsTileH + ks * 32), idesc, (kt | ks) != 0);
                    tc::mma_commit(&empty[s]);
                    if (++s == kLsStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                tc::mma_commit(&tfull[b]);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warp w's 32 vocabulary rows of each tile (TMEM lanes 32 w + lane) ----------------
        float lv[kLsN];
        int li[kLsN];
#pragma unroll
        for (int j = 0; j < kLsN; j++) {
            lv[j] = -INFINITY;
            li[j] = -1;
        }
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        for (int i = 0; i < my_tiles; i++) {
            const int b = i % kLsBufs;
            if (!tc::mbar_wait(&tfull[b], (uint32_t)(i / kLsBufs) & 1, err, ANELM_ERR_TIMEOUT, abort)) break;
            tc::tc_fence_after();
            uint32_t x[kLsN];
            tc::tmem_ld16(trow + b * kLsN, x);
            tc::tmem_ld_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&tfree[b]);  // accumulator b read: the MMAs may reuse it
            const int v0 = (g + i * G) * kLsBM + 32 * warp;  // this warp's first vocabulary row
            const bool in = v0 + lane < N;
#pragma unroll
            for (int j = 0; j < kLsN; j++) {
                if (j < M) {  // warp-uniform
                    const float v = __uint_as_float(x[j]);
                    const float thr = __shfl_sync(0xffffffffu, lv[j], 31);
                    unsigned mk = __ballot_sync(0xffffffffu, in && v > thr);
                    while (mk) {
                        const int src = __ffs(mk) - 1;
                        mk &= mk - 1;
                        const float xv = __shfl_sync(0xffffffffu, v, src);
                        warp_topk_insert_if(lv[j], li[j], true, xv, v0 + src, lane);
                    }
                }
            }
        }
        const long long lists = (long long)G * 4;
#pragma unroll
        for (int j = 0; j < kLsN; j++) {
            if (j < M) {
                const long long slot = (long long)j * lists + (long long)g * 4 + warp;
                cand[slot * kTopK + lane] = lv[j];
                reinterpret_cast<int*>(cand + (long long)M * lists * kTopK)[slot * kTopK + lane] = li[j];
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kLsBufs * kLsN);
    }
}

}  // namespace

namespace {

// LM head for a few rows (n <= kLmGemvRows <= kGvMaxM): the weight read is the cost, so the CUDA cores stream the
// vocabulary rows as gemv_bf16_kernel does (rows of h staged in shared memory, four vocabulary rows
// per warp, 16-byte loads) and each warp keeps, per row of h, a running top-32 spread across its
// lanes (lane j holds the j-th largest; a ballot places a new logit, a shuffle shifts the tail).
// The CTA's eight lists per row are merged by warp 0 into one candidate list [M][G][32] (values,
// then indices) for lm_topk_merge_kernel.  Logits are never written.
__global__ void __launch_bounds__(kGvThreads) lm_head_gemv_topk_kernel(const __nv_bfloat16* A, long long lda,
                                                                       const __nv_bfloat16* B, long long ldb, float* cand,
                                                                       int M, int N, int K) {
    extern __shared__ uint4 xs[];  // [M][K / 8]
    __shared__ float s_v[kGvThreads / 32][kGvMaxM][32];
    __shared__ int s_i[kGvThreads / 32][kGvMaxM][32];
    const int kc = K / 8;
    for (int i = threadIdx.x; i < M * kc; i += kGvThreads) {
        const int m = i / kc, c = i - m * kc;
        xs[i] = *reinterpret_cast<const uint4*>(A + (long long)m * lda + (long long)c * 8);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * (kGvThreads / 32);
    float tv[kGvMaxM];
    int ti[kGvMaxM];
#pragma unroll
    for (int m = 0; m < kGvMaxM; m++) {
        tv[m] = -INFINITY;
        ti[m] = -1;
    }
    for (int n0 = (blockIdx.x * (kGvThreads / 32) + warp) * kLmGvRows; n0 < N; n0 += nwarps * kLmGvRows) {
        const uint4* brow[kLmGvRows];
#pragma unroll
        for (int r = 0; r < kLmGvRows; r++)
            brow[r] = reinterpret_cast<const uint4*>(B + (long long)min(n0 + r, N - 1) * ldb);
        float acc[kLmGvRows][kGvMaxM];
#pragma unroll
        for (int r = 0; r < kLmGvRows; r++)
#pragma unroll
            for (int m = 0; m < kGvMaxM; m++) acc[r][m] = 0.f;
        for (int c0 = lane; c0 < kc; c0 += 32 * kLmGvUnroll) {
            uint4 w[kLmGvRows][kLmGvUnroll];
#pragma unroll
            for (int u = 0; u < kLmGvUnroll; u++)
#pragma unroll
                for (int r = 0; r < kLmGvRows; r++)
                    w[r][u] = (c0 + 32 * u < kc) ? ld_stream16(brow[r] + c0 + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < kLmGvUnroll; u++) {
                const int c = c0 + 32 * u;
                if (c >= kc) break;
                float wf[kLmGvRows][8];
#pragma unroll
                for (int r = 0; r < kLmGvRows; r++) unpack8(w[r][u], true, wf[r]);
#pragma unroll
                for (int m = 0; m < kGvMaxM; m++) {
                    if (m >= M) break;
                    float xf[8];
                    unpack8(xs[m * kc + c], true, xf);
#pragma unroll
                    for (int r = 0; r < kLmGvRows; r++)
#pragma unroll
                        for (int e = 0; e < 8; e++) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kLmGvRows; r++)
#pragma unroll
            for (int m = 0; m < kGvMaxM; m++) {
                if (m >= M) break;
                // lane 0's sum for every lane: the butterfly's lanes can differ in the last bit
                const float s = __shfl_sync(0xffffffffu, warp_sum(acc[r][m]), 0);
                if (n0 + r < N) warp_topk_insert(tv[m], ti[m], s, n0 + r, lane);
            }
    }
#pragma unroll
    for (int m = 0; m < kGvMaxM; m++) {
        s_v[warp][m][lane] = tv[m];
        s_i[warp][m][lane] = ti[m];
    }
    __syncthreads();
    if (warp == 0) {
        const long long G = gridDim.x;
#pragma unroll
        for (int m = 0; m < kGvMaxM; m++) {
            if (m >= M) break;
            for (int w = 1; w < kGvThreads / 32; w++)
                for (int j = 0; j < 32; j++) {
                    const float v = s_v[w][m][j];
                    if (!(v > __shfl_sync(0xffffffffu, tv[m], 31))) break;  // sorted: the rest cannot enter
                    warp_topk_insert(tv[m], ti[m], v, s_i[w][m][j], lane);
                }
            cand[((long long)m * G + blockIdx.x) * kTopK + lane] = tv[m];
            reinterpret_cast<int*>(cand + (long long)M * G * kTopK)[((long long)m * G + blockIdx.x) * kTopK + lane] =
                ti[m];
        }
    }
}

constexpr int kMergeWarps = 8;
constexpr int kMergeBatch = 8;  // candidate lists whose loads a warp keeps in flight together
// One CTA per row.  Every candidate list arrives sorted descending (lane j of the writing warp held
// its j-th largest), so a warp folds a whole list in one step: read reversed (ascending), merged
// into a running top-32 spread over its lanes by warp_merge_sorted.  Each warp keeps two running
// lists so two merges' shuffle chains overlap, folds a strided share of the row's lists, then
// merges its two lists; warp 0 merges the other warps' lists the same way.  Ties among equal
// values keep the smaller vocabulary index first.  Every trip count is warp-uniform.
__global__ void __launch_bounds__(32 * kMergeWarps) lm_topk_merge_kernel(const float* cand, int M, int ntile, int k,
                                                                         float* top_vals, int* top_idx) {
    __shared__ float sv[kMergeWarps][kTopK];
    __shared__ int si[kMergeWarps][kTopK];
    const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long nc = (long long)ntile * kTopK;
    const float* cv = cand + (long long)m * nc;
    const int* ci = reinterpret_cast<const int*>(cand + (long long)M * nc) + (long long)m * nc;
    float tv[2] = {-INFINITY, -INFINITY};  // lane j: the j-th largest so far, two independent lists
    int ti[2] = {-1, -1};
    // list t = base + kMergeWarps u for round u of a batch; the loads of a batch are issued together
    for (int base = warp; base < ntile; base += kMergeWarps * kMergeBatch) {
        float v[kMergeBatch];
        int id[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; u++) {
            const int t = base + kMergeWarps * u;
            const long long i = (long long)t * kTopK + (kTopK - 1 - lane);  // reversed: ascending
            v[u] = t < ntile ? cv[i] : -INFINITY;
            id[u] = t < ntile ? ci[i] : INT_MAX;
        }
#pragma unroll
        for (int u = 0; u < kMergeBatch; u++) warp_merge_sorted(tv[u & 1], ti[u & 1], v[u], id[u], lane);
    }
    warp_merge_sorted(tv[0], ti[0], __shfl_sync(0xffffffffu, tv[1], 31 - lane),
                      __shfl_sync(0xffffffffu, ti[1], 31 - lane), lane);
    sv[warp][lane] = tv[0];
    si[warp][lane] = ti[0];
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < kMergeWarps; w++)
            warp_merge_sorted(tv[0], ti[0], sv[w][kTopK - 1 - lane], si[w][kTopK - 1 - lane], lane);
        if (lane < k) {
            top_vals[(long long)m * k + lane] = tv[0];
            top_idx[(long long)m * k + lane] = ti[0];
        }
    }
}

}  // namespace

// CTAs over the vocabulary per 128-row tile (about one CTA per SM overall, at most one per tile)
static int lm_groups(int n, int vocab) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int mt = (n + kGBM - 1) / kGBM, ntile = (vocab + kGBN - 1) / kGBN;
    return std::max(1, std::min(ntile, sms / mt));
}

// CTAs of the few-row path: at most kGvBlocksPerSm per SM, at most one per 32 vocabulary rows
static int lm_gemv_groups(int vocab) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int rows_per_block = kLmGvRows * (kGvThreads / 32);
    return std::max(1, std::min((vocab + rows_per_block - 1) / rows_per_block, sms * kGvBlocksPerSm));
}

// copies of the row block in the tensor-core path's A tile, so every epilogue warp has rows: with
// 9-24 rows four copies (graph-timed, 16 rows 241 -> 228 us, 24 rows 241 -> 217 us); from 25 rows
// one copy does as well or better (32 rows 220 -> 210 us), since the epilogue takes few logits
static int lm_rep(int n) { return n > 8 && n <= 24 ? 4 : 1; }
// rows up to which the swapped kernel is taken (16 rows: 240 us there against 228 in the tile kernel)
constexpr int kLmSwapRows = 8;
static_assert(kLmSwapRows <= kLsN, "the swapped kernel's N covers its rows");

// CTAs of the swapped few-row path: one per SM, at most one per 128 vocabulary rows
static int lm_swap_groups(int vocab) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return std::max(1, std::min((vocab + kLsBM - 1) / kLsBM, sms));
}

// the tensor-core path's first-tile maxima [n][pitch] (pitch: CTAs over the vocabulary, rounded up to
// whole 16-byte rows) and its arrival counter follow its candidate lists
static int lm_max_pitch(int n, int vocab) { return (lm_groups(n, vocab) + 3) & ~3; }

size_t lm_head_topk_workspace_bytes(int n, int vocab) {
    int g = lm_groups(n, vocab) * lm_rep(n);                      // tensor-core path
    if (n <= kLmGemvRows) g = std::max(g, lm_gemv_groups(vocab));  // CUDA-core path
    if (n <= kLmSwapRows) g = std::max(g, lm_swap_groups(vocab) * 4);  // swapped path
    const size_t tc_extra = (size_t)n * lm_max_pitch(n, vocab) * 4 + 16;
    return (size_t)n * g * kTopK * 8 + tc_extra;
}

int launch_lm_head_topk(const void* h, long long ldh, const void* W, long long ldw, int n, int vocab, int hidden, int k,
                        float* top_vals, int* top_idx, void* workspace, size_t workspace_bytes, int* err,
                        cudaStream_t stream) {
    if (n <= 0 || vocab <= 0 || hidden <= 0 || k < 1 || k > 32 || k > vocab) return ANELM_ERR_INVALID_ARG;
    if (workspace_bytes < lm_head_topk_workspace_bytes(n, vocab)) return ANELM_ERR_CAPACITY;
    if ((uintptr_t)h % 16 || (uintptr_t)W % 16 || (ldh * 2) % 16 || (ldw * 2) % 16 || ldh < hidden || ldw < hidden ||
        (uintptr_t)workspace % 16)
        return ANELM_ERR_UNSUPPORTED;
    if (n <= kLmGemvRows && hidden % 8 == 0 && (size_t)n * hidden * 2 <= 48 * 1024) {
        // one row (single-sequence decode): stream the weights on the CUDA cores, top-32 kept per warp
        const int G = lm_gemv_groups(vocab);
        lm_head_gemv_topk_kernel<<<G, kGvThreads, n * hidden * 2, stream>>>(
            static_cast<const __nv_bfloat16*>(h), ldh, static_cast<const __nv_bfloat16*>(W), ldw,
            static_cast<float*>(workspace), n, vocab, hidden);
        lm_topk_merge_kernel<<<n, 32 * kMergeWarps, 0, stream>>>(static_cast<const float*>(workspace), n, G, k, top_vals,
                                                              top_idx);
        return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
    }
    if (n <= kLmSwapRows && lm_swap_smem(hidden) <= (size_t)kGSmemMax) {
        // 2-8 rows: weights as the M operand, h resident in shared memory (see lm_head_swap_topk_kernel)
        CUtensorMap mW, mH;
        if (!make_bf16_map(&mW, W, (uint64_t)vocab, (uint64_t)hidden, (uint64_t)ldw, kLsBM) ||
            !make_bf16_map(&mH, h, (uint64_t)n, (uint64_t)hidden, (uint64_t)ldh, kLsN))
            return ANELM_ERR_CUDA;
        const int smem = (int)lm_swap_smem(hidden);
        cudaFuncSetAttribute(lm_head_swap_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        const int G = lm_swap_groups(vocab);
        lm_head_swap_topk_kernel<<<G, kGThreads, smem, stream>>>(mW, mH, static_cast<float*>(workspace), n, vocab,
                                                                hidden, err);
        lm_topk_merge_kernel<<<n, 32 * kMergeWarps, 0, stream>>>(static_cast<const float*>(workspace), n, G * 4, k,
                                                              top_vals, top_idx);
        return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
    }
    const int rep = lm_rep(n);
    CUtensorMap mA, mB;
    if (!make_bf16_map(&mA, h, (uint64_t)n, (uint64_t)hidden, (uint64_t)ldh, kGBM / rep) ||
        !make_bf16_map(&mB, W, (uint64_t)vocab, (uint64_t)hidden, (uint64_t)ldw, kGBN))
        return ANELM_ERR_CUDA;
    constexpr int smem = kLmSmem;
    cudaFuncSetAttribute(lm_head_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const int G = lm_groups(n, vocab), gpitch = lm_max_pitch(n, vocab);
    float* pmax = static_cast<float*>(workspace) + (size_t)n * G * rep * kTopK * 2;
    unsigned* arrive = reinterpret_cast<unsigned*>(pmax + (size_t)n * gpitch);
    if (cudaMemsetAsync(pmax, 0xFF, (size_t)n * gpitch * 4, stream) != cudaSuccess ||  // NaN: not published
        cudaMemsetAsync(arrive, 0, 4, stream) != cudaSuccess)
        return ANELM_ERR_CUDA;
    dim3 grid(G, (n + kGBM - 1) / kGBM);
    lm_head_topk_kernel<<<grid, kGThreads, smem, stream>>>(mA, mB, static_cast<float*>(workspace), pmax, gpitch, arrive,
                                                           n, vocab, hidden, rep, err);
    lm_topk_merge_kernel<<<n, 32 * kMergeWarps, 0, stream>>>(static_cast<const float*>(workspace), n, G * rep, k,
                                                          top_vals, top_idx);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

}  // namespace anelm
