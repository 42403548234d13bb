// Split-K flash-decoding for the Qwen3.5 gated full-attention core (sm_100a).
//
// Replaces, for one decode token per sequence:
//   forward_full_attn_from_proj  models/llm/qwen3_5.cpp:944-1002
//     (QK RMSNorm 952-959, RoPE 961-971, ring append 973-986, gqa_attention
//      988-991, sigmoid gate 993-1000), and
//   gqa_attention                core/cpu_ops.cpp:148-204.
//
// Work decomposition: one CTA per (batch row, split of the ring's logical
// range, kv head).  A CTA
//   1. rebuilds the group's G query heads from the projection row (RMSNorm,
//      RoPE, 1/sqrt(d)), and the new token's k/v; split 0 appends k/v to the
//      ring slot (fp16);
//   2. streams its range of K and V rows (64-token tiles, 16-byte cp.async into
//      XOR-swizzled shared memory, 3-stage pipeline) -- each KV byte is read
//      from HBM once and serves all G query heads;
//   3. computes Q K^T and P V on the tensor cores with fp32 accumulation.  The
//      fp32 queries and probabilities are split into fp16 hi + lo halves that
//      sit side by side in the 8 columns of an m16n8k16 MMA (G <= 4), so the
//      products carry ~22 significant bits while K/V stay in their fp16
//      storage format;
//   4. keeps an online softmax (running max / sum per head) across tiles and
//      writes an unnormalised partial (O, m, l).
// The last CTA of a (row, kv head) -- found with an atomic counter, no waiting
// -- merges the partials, applies the sigmoid gate and writes the output; the
// last of those updates the ring's len/start.  For a single row with at most 16
// splits the splits of a kv head instead form one thread-block cluster: each CTA
// keeps its partial in shared memory and, after a cluster barrier, merges a
// slice of the output columns from all of them through distributed shared
// memory (no global round trip, no serial merging CTA).
//
// New-token handling: the slot being written is never one of the old tokens the
// other CTAs read (it is either empty or the evicted oldest slot), so the
// append and the reads of the same launch do not race.  The CTA whose tile
// holds the new token patches that row in shared memory with the fp16 k/v.
#include <cooperative_groups.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace anelm {

namespace {

constexpr int kTile = 64;      // tokens per pipeline tile
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 3;
constexpr int kGP = 4;         // padded query heads per kv head (hi+lo fill n=8)
constexpr int kPRow = kTile + 8;  // halves per P row (padding breaks bank conflicts)

template <int D>
struct Smem {
    static constexpr size_t tiles = 0;
    static constexpr size_t tile_bytes = size_t(kTile) * D * 2;
    static constexpr size_t q = tiles + kStages * tile_bytes;     // float [kGP][D]
    static constexpr size_t kf = q + size_t(kGP) * D * 4;          // float [D]
    static constexpr size_t vf = kf + size_t(D) * 4;               // float [D]
    static constexpr size_t kh = vf + size_t(D) * 4;               // half  [D]
    static constexpr size_t vh = kh + size_t(D) * 2;               // half  [D]
    static constexpr size_t sc = vh + size_t(D) * 2;               // float [kGP][kTile]
    static constexpr size_t P = sc + size_t(kGP) * kTile * 4;      // half  [2*kGP][kPRow]
    static constexpr size_t misc = P + size_t(2 * kGP) * kPRow * 2;  // float [32]
    static constexpr size_t total = misc + 32 * 4;
};

__device__ __forceinline__ void rope_cs(const FaDecodeParams& p, int pos, int j, float& c, float& s) {
    const int half = p.rot_dim >> 1;
    if (pos >= 0 && pos < p.rope_len && p.rope_cos) {
        c = p.rope_cos[(long long)pos * half + j];
        s = p.rope_sin[(long long)pos * half + j];
    } else {  // core/cpu_ops.cpp:51-56
        float freq = 1.0f / powf(p.rope_theta, (float)(2 * j) / (float)p.rot_dim);
        float angle = (float)pos * freq;
        c = cosf(angle);
        s = sinf(angle);
    }
}

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Merge of one row's splits inside a thread-block cluster (one CTA per split of kv head kvh): every
// CTA holds its unnormalised partial O [kGP][D] and (m, l) [kGP][2] in shared memory at `po`.  After a
// cluster barrier, warp g < G of each CTA turns the heads' (m, l) of all splits into merge weights,
// and each CTA merges its slice of the G * D / 4 float4 output columns (8 lanes per column, each
// over every eighth split) from its peers' shared memory, then gates and stores them.  A second
// cluster barrier keeps every CTA resident until its peers have read it.
template <int D>
__device__ __forceinline__ void cluster_merge(const FaDecodeParams& p, uint8_t* smem, const float* po, int b, int kvh,
                                              int G, int seq, const char* proj_row, int len1, int start1,
                                              const float (&gate4)[4]) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = (int)cl.block_rank(), ns = (int)cl.num_blocks();
    __shared__ float s_w[16][kGP];  // merge weight of split r for head g
    __shared__ float s_L[kGP];
    cl.sync();  // every split's partial is in its shared memory
    // every CTA of this kv head is past its reads of the ring metadata: count the kv head now (the
    // last of the row's kv heads updates len / start), overlapping the merge below
    if (rank == 0 && tid == 0) {
        __threadfence();  // this CTA's ring append is visible before it is counted
        const int prev = atomicAdd(&p.cnt_seq[b], 1);
        if (prev == p.Hkv - 1) {
            if (p.append && p.kv_len) {
                p.kv_len[seq] = len1;
                p.kv_start[seq] = start1;
            }
            p.cnt_seq[b] = 0;
        }
    }
    if (warp < G) {
        const int g = warp;
        float m = -INFINITY, l = 0.f;
        if (lane < ns) {
            const float* ml = cl.map_shared_rank(po + kGP * D, lane);
            m = ml[2 * g];
            l = ml[2 * g + 1];
        }
        const float M = warp_max(m);
        const float w = (m == -INFINITY) ? 0.f : expf(m - M);
        const float L = warp_sum(w * l);
        if (lane < ns) s_w[lane][g] = w;
        if (lane == 0) s_L[g] = L;
    }
    __syncthreads();
    const int nitem = G * D / 4;
    const int per = (nitem + ns - 1) / ns;
    const int i0 = rank * per, i1 = min(nitem, i0 + per);
    const int sub = tid & 7;
    for (int base = i0; base < i1; base += kThreads / 8) {  // uniform trip count: whole warps shuffle
        const int it = base + (tid >> 3);
        const bool valid = it < i1;
        const int g = valid ? (it * 4) / D : 0, col = valid ? it * 4 - g * D : 0;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = sub; r < ns && valid; r += 8) {
            const float4 v = *reinterpret_cast<const float4*>(cl.map_shared_rank(po + g * D + col, r));
            const float w = s_w[r][g];
            o.x += w * v.x; o.y += w * v.y; o.z += w * v.z; o.w += w * v.w;
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            o.x += __shfl_xor_sync(0xffffffffu, o.x, off);
            o.y += __shfl_xor_sync(0xffffffffu, o.y, off);
            o.z += __shfl_xor_sync(0xffffffffu, o.z, off);
            o.w += __shfl_xor_sync(0xffffffffu, o.w, off);
        }
        if (sub == 0 && valid) {
            const float L = s_L[g];
            const float ov[4] = {o.x, o.y, o.z, o.w};
            const int h = kvh * G + g;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float O = (L > 0.f) ? ov[e] / L : 0.f;
                if (p.gate) {  // mul_sigmoid_inplace, core/cpu_ops.cpp:15-22 (first item: prefetched)
                    const float z = base == i0 ? gate4[e]
                                               : load_as_float(proj_row, p.proj_dtype,
                                                               p.gate_off + (long long)h * p.q_head_stride + col + e);
                    O = O / (1.0f + expf(-z));
                }
                store_from_float(p.out, p.out_dtype, (long long)b * p.out_stride + (long long)h * D + col + e, O);
            }
        }
    }
    cl.sync();  // peers are done reading this CTA's partial
}

template <int D, bool CM>
__global__ void __launch_bounds__(kThreads, 2) fa_decode_kernel(const FaDecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using S = Smem<D>;
    constexpr int CPR = D / 8;             // 16-byte chunks per row
    constexpr int DW = D / kWarps;         // d columns per warp in P V
    constexpr int MT = DW / 16;            // m16 tiles per warp in P V

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int blk = blockIdx.x, kvh = blockIdx.y;
    // Programmatic dependent launch (the one-row cluster form is launched as one): a following
    // launch may start once every CTA of this grid is resident; before griddepcontrol.wait this
    // CTA reads only the QK-norm weights (never written by a kernel), after it everything else
    // (the projection row, ring metadata, positions, K / V pools).  Both are no-ops without PDL.
    asm volatile("griddepcontrol.launch_dependents;");
    if (CM && tid == 0) {
        // Before the dependency wait, an L2 prefetch of this CTA's share (1 / Hkv of the rows, for K and
        // for V) of the ring slots its split will stream, so the tiles hit L2 once the wait is over.  A
        // prefetch is only a hint -- L2 stays coherent with whatever the previous kernel writes -- so the
        // ring metadata it is sized from may be read here, before that kernel has finished.
        const int sq = p.seq_ids ? p.seq_ids[0] : 0;
        const int cap_ = p.kv_len ? p.kv_cap[sq] : p.cap_s;
        const int len_ = p.kv_len ? p.kv_len[sq] : p.len_s;
        const int st_ = p.kv_len ? p.kv_start[sq] : p.start_s;
        const long long base_ = p.kv_len ? p.kv_base[sq] : 0;
        const int t0 = blk * p.CH, t1 = min(t0 + p.CH, len_);
        if (cap_ > 0 && t1 > t0 && st_ >= 0 && st_ < cap_) {
            const long long row_bytes = (long long)p.Hkv * D * 2;  // one slot: every kv head
            int s0 = st_ + t0;
            if (s0 >= cap_) s0 -= cap_;
            int n = t1 - t0;
            const int share = (n + p.Hkv - 1) / p.Hkv;  // this CTA's rows of each contiguous run
            while (n > 0) {
                const int run = min(n, cap_ - s0);          // up to the end of the ring, then from slot 0
                const int r0 = min(run, kvh * share), r1 = min(run, r0 + share);
                if (r1 > r0) {
                    const long long off = (base_ + s0 + r0) * row_bytes;
                    const uint32_t bytes = (uint32_t)((r1 - r0) * row_bytes);
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(
                                     reinterpret_cast<const char*>(p.k_pool) + off), "r"(bytes) : "memory");
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(
                                     reinterpret_cast<const char*>(p.v_pool) + off), "r"(bytes) : "memory");
                }
                n -= run;
                s0 = 0;
            }
        }
    }
    constexpr int NW = D / 32;
    float wq[NW], wk[NW];
    if (p.qk_norm) {
#pragma unroll
        for (int m = 0; m < NW; m++) {
            wq[m] = p.q_norm[lane + 32 * m];
            wk[m] = p.k_norm[lane + 32 * m];
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the cluster-merge form serves a one-row plan with one CTA per split: no table lookup
    const int b = CM ? 0 : p.blk_b[blk], split = CM ? blk : p.blk_split[blk];
    const int Hkv = p.Hkv;
    const int G = p.Hq / Hkv;
    const int seq = p.seq_ids ? p.seq_ids[b] : 0;
    const char* proj_row = reinterpret_cast<const char*>(p.proj) +
                           (long long)b * p.proj_stride * dtype_bytes(p.proj_dtype);

    // ---- the projection values this CTA needs, first: one 16-byte q chunk per thread (head
    // tid / CPR of the group) and, for the append, one k or v chunk; issued ahead of the ring
    // metadata and the K / V tiles, so they do not queue behind the tile loads ----
    const int qg = tid / CPR, qc = tid % CPR;
    const bool has_q = p.proj_vec && tid < kGP * CPR && qg < G;
    const bool has_k = p.proj_vec && p.append && tid < CPR;
    const bool has_v = p.proj_vec && p.append && tid >= CPR && tid < 2 * CPR;
    float q8[8], kv8[8];
    if (has_q) load8(proj_row, p.proj_dtype, (long long)(kvh * G + qg) * p.q_head_stride + qc * 8, q8);
    if (has_k) load8(proj_row, p.proj_dtype, p.k_off + (long long)kvh * D + tid * 8, kv8);
    if (has_v) load8(proj_row, p.proj_dtype, p.v_off + (long long)kvh * D + (tid - CPR) * 8, kv8);

    // ---- per-thread constants of the prologue and the merge, loaded now so their latency overlaps
    // the projection loads (the QK-norm weights came before the dependency wait): the RoPE angle of the pair
    // this thread rotates (the same pair index for every vector when the thread count is a
    // multiple of the half rotary width), and, for the cluster merge, the gate values of the first
    // output columns this thread merges ----
    const int pos = p.pos_arr ? p.pos_arr[b] : p.pos_scalar;
    const int rhalf = p.rot_dim >> 1;
    const bool rope_pre = rhalf > 0 && kThreads % rhalf == 0;
    float rc = 1.f, rs = 0.f;
    if (rope_pre) rope_cs(p, pos, tid % rhalf, rc, rs);
    float gate4[4] = {0.f, 0.f, 0.f, 0.f};
    if (CM && p.gate && (tid & 7) == 0) {
        const int ns = p.cluster_ns, nitem = G * D / 4, per = (nitem + ns - 1) / ns;
        const int it = blk * per + (tid >> 3);
        if (it < min(nitem, blk * per + per)) {
            const int g = (it * 4) / D, col = it * 4 - g * D;
#pragma unroll
            for (int e = 0; e < 4; e++)
                gate4[e] = load_as_float(proj_row, p.proj_dtype,
                                         p.gate_off + (long long)(kvh * G + g) * p.q_head_stride + col + e);
        }
    }

    // ---- ring metadata (models/llm/qwen3_5.cpp:973-983) ----
    int cap, len0, start0;
    long long base;
    if (p.kv_len) {
        cap = p.kv_cap[seq];
        len0 = p.kv_len[seq];
        start0 = p.kv_start[seq];
        base = p.kv_base[seq];
    } else {
        cap = p.cap_s;
        len0 = p.len_s;
        start0 = p.start_s;
        base = 0;
    }
    int len1 = len0, start1 = start0, slot = -1;
    if (p.append) {
        if (p.kv_mode == ANELM_KV_LINEAR) {  // scripts/serve_hybrid.py:105-108
            if (pos < 0 || pos >= cap) {
                set_err(p.err, ANELM_ERR_CAPACITY);
                return;  // uniform for every CTA of this row: counters stay untouched
            }
            slot = pos;
            len1 = pos + 1;
            start1 = 0;
        } else if (len0 < cap) {
            slot = start0 + len0;
            if (slot >= cap) slot -= cap;
            len1 = len0 + 1;
        } else {
            slot = start0;
            start1 = start0 + 1;
            if (start1 >= cap) start1 = 0;
        }
    }
    const int n_old = p.append ? len1 - 1 : len1;  // tokens read from the ring
    const int t_begin = split * p.CH;
    const int t_end = min(t_begin + p.CH, len1);
    const int n_tok = max(0, t_end - t_begin);
    const int n_tiles = (n_tok + kTile - 1) / kTile;

    float* q_s = reinterpret_cast<float*>(smem + S::q);
    float* kf_s = reinterpret_cast<float*>(smem + S::kf);
    float* vf_s = reinterpret_cast<float*>(smem + S::vf);
    __half* kh_s = reinterpret_cast<__half*>(smem + S::kh);
    __half* vh_s = reinterpret_cast<__half*>(smem + S::vh);
    float* sc_s = reinterpret_cast<float*>(smem + S::sc);
    __half* P_s = reinterpret_cast<__half*>(smem + S::P);
    float* misc = reinterpret_cast<float*>(smem + S::misc);
    // misc: [0..3] m_run, [4..7] l_run, [8..11] alpha, [12..15] score scale

    float acc[MT][4];
#pragma unroll
    for (int i = 0; i < MT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    // ---- 0. the first K / V tiles start loading now: they depend only on the ring metadata, so
    // their latency overlaps the prologue (projection loads, norms, RoPE) ----
    const int t_new = p.append ? len1 - 1 : -1;  // logical index of the new token
    const __half* kpool = p.k_pool;
    const __half* vpool = p.v_pool;
    auto issue = [&](int j) {
        const int stage = j % kStages;
        const int tile = j >> 1;
        const __half* pool = (j & 1) ? vpool : kpool;
        const uint32_t sbase = smem_u32(smem + S::tiles + stage * S::tile_bytes);
        for (int idx = tid; idx < kTile * CPR; idx += kThreads) {
            const int r = idx / CPR, ch = idx - r * CPR;
            const int t = t_begin + tile * kTile + r;
            const bool valid = (t < t_end) && (t < n_old);
            int s = start1 + t;
            if (s >= cap) s -= cap;
            const __half* src = pool + ((base + (valid ? s : 0)) * Hkv + kvh) * (long long)D + ch * 8;
            const uint32_t dst = sbase + (uint32_t)(r * D + ((ch ^ (r & 7)) * 8)) * 2u;
            cp_async_16(dst, src, valid ? 16 : 0);
        }
    };
    const int n_jobs = 2 * n_tiles;
    if (n_tok > 0) {
#pragma unroll
        for (int j = 0; j < kStages - 1; j++) {
            if (j < n_jobs) issue(j);
            cp_async_commit();
        }
    }

    if (n_tok > 0) {
        // ---- 1. prologue: queries, new k/v ----
        if (p.proj_vec) {
            if (tid < kGP * CPR) {
#pragma unroll
                for (int e = 0; e < 8; e++) q_s[qg * D + qc * 8 + e] = has_q ? q8[e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (has_k) kf_s[tid * 8 + e] = kv8[e];
                if (has_v) vf_s[(tid - CPR) * 8 + e] = kv8[e];
            }
        } else {
            for (int idx = tid; idx < kGP * D; idx += kThreads) {
                int g = idx / D, i = idx - g * D;
                q_s[idx] = (g < G) ? load_as_float(proj_row, p.proj_dtype,
                                                   (long long)(kvh * G + g) * p.q_head_stride + i)
                                   : 0.f;
            }
            if (p.append) {
                for (int i = tid; i < D; i += kThreads) {
                    kf_s[i] = load_as_float(proj_row, p.proj_dtype, p.k_off + (long long)kvh * D + i);
                    vf_s[i] = load_as_float(proj_row, p.proj_dtype, p.v_off + (long long)kvh * D + i);
                }
            }
        }
        __syncthreads();
        const int nvec = G + (p.append ? 1 : 0);
        if (p.qk_norm) {  // rmsnorm, core/cpu_ops.cpp:24-30
            for (int vec = warp; vec < nvec; vec += kWarps) {
                float* x = vec < G ? q_s + vec * D : kf_s;
                float ss = 0.f;
                for (int i = lane; i < D; i += 32) ss += x[i] * x[i];
                ss = warp_sum(ss);
                const float r = 1.0f / sqrtf(ss / (float)D + p.rms_eps);
#pragma unroll
                for (int m = 0; m < NW; m++)
                    x[lane + 32 * m] = __fmul_rn(__fmul_rn(x[lane + 32 * m], r), vec < G ? wq[m] : wk[m]);
            }
            __syncthreads();
        }
        if (p.rot_dim > 0) {  // apply_rope_cached, core/cpu_ops.cpp:40-63 (or rotate-half)
            const int half = p.rot_dim >> 1;
            for (int idx = tid; idx < nvec * half; idx += kThreads) {
                int vec = idx / half, j = idx - vec * half;
                float* x = vec < G ? q_s + vec * D : kf_s;
                float c = rc, s = rs;
                if (!rope_pre) rope_cs(p, pos, j, c, s);
                int i0, i1;
                if (p.rope_mode == ANELM_ROPE_INTERLEAVED) {
                    i0 = 2 * j;
                    i1 = 2 * j + 1;
                } else {
                    i0 = j;
                    i1 = j + half;
                }
                float v0 = x[i0], v1 = x[i1];
                if (p.rope_mode == ANELM_ROPE_INTERLEAVED) {
                    x[i0] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
                    x[i1] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
                } else {  // serve_hybrid.py:98-99: q1*cos - q2*sin, q2*cos + q1*sin
                    x[i0] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
                    x[i1] = __fadd_rn(__fmul_rn(v1, c), __fmul_rn(v0, s));
                }
            }
            __syncthreads();
        }
        if (p.append) {
            for (int i = tid; i < D; i += kThreads) {
                kh_s[i] = __float2half_rn(kf_s[i]);
                vh_s[i] = __float2half_rn(vf_s[i]);
            }
        }
        // per-head power-of-two prescale so the fp16 hi/lo split keeps full range
        if (warp < kGP) {
            float mx = 0.f;
            for (int i = lane; i < D; i += 32) mx = fmaxf(mx, fabsf(q_s[warp * D + i]));
            mx = warp_max(mx);
            int e = 0;
            if (mx > 0.f) frexpf(mx, &e);
            const int sh = 10 - e;  // max |q| * 2^sh in [2^9, 2^10)
            if (lane == 0) {
                misc[12 + warp] = ldexpf(p.scale, -sh);
                misc[16 + warp] = ldexpf(1.0f, sh);
            }
        }
        __syncthreads();
        if (p.append && split == 0 && slot >= 0) {  // ring append, qwen3_5.cpp:984-986
            const long long row = ((base + slot) * Hkv + kvh) * (long long)D;
            for (int ch = tid; ch < CPR; ch += kThreads) {
                reinterpret_cast<uint4*>(p.k_pool + row)[ch] = reinterpret_cast<const uint4*>(kh_s)[ch];
                reinterpret_cast<uint4*>(p.v_pool + row)[ch] = reinterpret_cast<const uint4*>(vh_s)[ch];
            }
        }
    }

    if (n_tok > 0) {
        // B fragments of Q (k = d, n = [4 hi heads | 4 lo heads]) kept in registers.
        uint32_t qb[D / 16][2];
        {
            const int n = lane >> 2, c = lane & 3, h = n & 3;
            const bool lo = n >= 4;
            const float up = misc[16 + h];
#pragma unroll
            for (int ks = 0; ks < D / 16; ks++) {
#pragma unroll
                for (int part = 0; part < 2; part++) {
                    const int i = 16 * ks + 8 * part + 2 * c;
                    float x0 = q_s[h * D + i] * up, x1 = q_s[h * D + i + 1] * up;
                    __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
                    if (lo) {
                        h0 = __float2half_rn(x0 - __half2float(h0));
                        h1 = __float2half_rn(x1 - __half2float(h1));
                    }
                    qb[ks][part] = pack_half2(h0, h1);
                }
            }
        }
        if (tid < kGP) {
            misc[tid] = -INFINITY;
            misc[4 + tid] = 0.f;
            misc[8 + tid] = 1.f;
        }
        for (int idx = tid; idx < 2 * kGP * kPRow; idx += kThreads) P_s[idx] = __float2half_rn(0.f);

        for (int j = 0; j < n_jobs; j++) {
            cp_async_wait<kStages - 2>();
            __syncthreads();
            if (j + kStages - 1 < n_jobs) issue(j + kStages - 1);
            cp_async_commit();
            const int stage = j % kStages;
            const int tile = j >> 1;
            const bool isV = j & 1;
            uint8_t* tbuf = smem + S::tiles + stage * S::tile_bytes;
            const int tile_t0 = t_begin + tile * kTile;
            if (t_new >= tile_t0 && t_new < tile_t0 + kTile && t_new < t_end) {
                const int r = t_new - tile_t0;
                const __half* src = isV ? vh_s : kh_s;
                for (int ch = tid; ch < CPR; ch += kThreads)
                    *reinterpret_cast<uint4*>(tbuf + (r * D + ((ch ^ (r & 7)) * 8)) * 2) =
                        reinterpret_cast<const uint4*>(src)[ch];
                __syncthreads();
            }
            const uint32_t tb = smem_u32(tbuf);
            if (!isV) {
                // ---- scores for tokens [16*warp, 16*warp+16) of this tile ----
                float c4[4] = {0.f, 0.f, 0.f, 0.f};
                const int r = 16 * warp + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
                for (int ks = 0; ks < D / 16; ks++) {
                    const int ch = 2 * ks + (lane >> 4);
                    uint32_t a0, a1, a2, a3;
                    ldmatrix_x4(tb + (uint32_t)(r * D + ((ch ^ (r & 7)) * 8)) * 2u, a0, a1, a2, a3);
                    mma_16816(c4, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
                }
                float o0 = __shfl_xor_sync(0xffffffffu, c4[0], 2);
                float o1 = __shfl_xor_sync(0xffffffffu, c4[1], 2);
                float o2 = __shfl_xor_sync(0xffffffffu, c4[2], 2);
                float o3 = __shfl_xor_sync(0xffffffffu, c4[3], 2);
                if ((lane & 3) < 2) {
                    const int h0 = 2 * (lane & 3), h1 = h0 + 1;
                    const int tl = 16 * warp + (lane >> 2);
                    const bool v0 = tile_t0 + tl < t_end, v1 = tile_t0 + tl + 8 < t_end;
                    sc_s[h0 * kTile + tl] = v0 ? (c4[0] + o0) * misc[12 + h0] : -INFINITY;
                    sc_s[h1 * kTile + tl] = v0 ? (c4[1] + o1) * misc[12 + h1] : -INFINITY;
                    sc_s[h0 * kTile + tl + 8] = v1 ? (c4[2] + o2) * misc[12 + h0] : -INFINITY;
                    sc_s[h1 * kTile + tl + 8] = v1 ? (c4[3] + o3) * misc[12 + h1] : -INFINITY;
                }
                __syncthreads();
                // ---- online softmax update, one warp per query head ----
                if (warp < G) {
                    const int h = warp;
                    const float s0 = sc_s[h * kTile + lane], s1 = sc_s[h * kTile + lane + 32];
                    const float m_old = misc[h];
                    const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
                    float alpha = 1.f, p0 = 0.f, p1 = 0.f;
                    if (m_new != -INFINITY) {
                        alpha = expf(m_old - m_new);
                        p0 = expf(s0 - m_new);
                        p1 = expf(s1 - m_new);
                    }
                    const float ps = warp_sum(p0 + p1);
                    const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
                    P_s[h * kPRow + lane] = h0;
                    P_s[h * kPRow + lane + 32] = h1;
                    P_s[(kGP + h) * kPRow + lane] = __float2half_rn(p0 - __half2float(h0));
                    P_s[(kGP + h) * kPRow + lane + 32] = __float2half_rn(p1 - __half2float(h1));
                    if (lane == 0) {
                        misc[h] = m_new;
                        misc[4 + h] = misc[4 + h] * alpha + ps;
                        misc[8 + h] = alpha;
                    }
                }
            } else {
                // ---- O^T[d][n] += V^T P^T for d in this warp's columns ----
                const int c = lane & 3;
                const float al0 = misc[8 + ((2 * c) & 3)], al1 = misc[8 + ((2 * c + 1) & 3)];
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    acc[mt][0] *= al0;
                    acc[mt][1] *= al1;
                    acc[mt][2] *= al0;
                    acc[mt][3] *= al1;
                }
                const int n = lane >> 2;
                const int jm = lane >> 3;
#pragma unroll
                for (int kk = 0; kk < kTile / 16; kk++) {
                    const int tl = 16 * kk + 2 * c;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(P_s + n * kPRow + tl);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(P_s + n * kPRow + tl + 8);
                    const int r = 16 * kk + (lane & 7) + ((jm >> 1) << 3);
#pragma unroll
                    for (int mt = 0; mt < MT; mt++) {
                        const int ch = ((warp * DW + 16 * mt) >> 3) + (jm & 1);
                        uint32_t a0, a1, a2, a3;
                        ldmatrix_x4_trans(tb + (uint32_t)(r * D + ((ch ^ (r & 7)) * 8)) * 2u, a0, a1, a2, a3);
                        mma_16816(acc[mt], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
        }
        cp_async_wait<0>();
        __syncthreads();
    }

    // ---- 4. partial (O unnormalised, m, l): to global memory, or to this CTA's shared memory
    // for the cluster merge (the tile buffers are free now) ----
    const long long pidx = (p.part_off[b] + split) * Hkv + kvh;
    float* po = CM ? reinterpret_cast<float*>(smem + S::tiles) : p.part_o + pidx * kGP * D;
    float* pml = CM ? po + kGP * D : p.part_ml + pidx * kGP * 2;
    {
        const int c = lane & 3;
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            float o0 = __shfl_xor_sync(0xffffffffu, acc[mt][0], 2);
            float o1 = __shfl_xor_sync(0xffffffffu, acc[mt][1], 2);
            float o2 = __shfl_xor_sync(0xffffffffu, acc[mt][2], 2);
            float o3 = __shfl_xor_sync(0xffffffffu, acc[mt][3], 2);
            if (c < 2) {
                const int d0 = warp * DW + 16 * mt + (lane >> 2);
                const int h0 = 2 * c, h1 = h0 + 1;
                po[h0 * D + d0] = acc[mt][0] + o0;
                po[h1 * D + d0] = acc[mt][1] + o1;
                po[h0 * D + d0 + 8] = acc[mt][2] + o2;
                po[h1 * D + d0 + 8] = acc[mt][3] + o3;
            }
        }
        if (tid < kGP) {
            pml[2 * tid] = (n_tok > 0) ? misc[tid] : -INFINITY;
            pml[2 * tid + 1] = (n_tok > 0) ? misc[4 + tid] : 0.f;
        }
    }
    if constexpr (CM) {
        cluster_merge<D>(p, smem, po, b, kvh, G, seq, proj_row, len1, start1, gate4);
        return;
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) {
        const int prev = atomicAdd(&p.cnt_head[b * Hkv + kvh], 1);
        s_last = (prev == p.nsplit[b] - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- 5. merge splits, gate, write (last CTA of this row / kv head) ----
    const int ns = p.nsplit[b];
    const long long p0 = p.part_off[b];
    float* wts = reinterpret_cast<float*>(smem + S::tiles);  // [ns][kGP] (tiles are free now)
    __shared__ float s_L[kGP];
    if (warp < G) {
        const int h = warp;
        float M = -INFINITY;
        for (int s = lane; s < ns; s += 32)
            M = fmaxf(M, ld_cg(p.part_ml + ((p0 + s) * Hkv + kvh) * kGP * 2 + 2 * h));
        M = warp_max(M);
        float L = 0.f;
        for (int s = lane; s < ns; s += 32) {
            const float* ml = p.part_ml + ((p0 + s) * Hkv + kvh) * kGP * 2 + 2 * h;
            const float m = ld_cg(ml);
            const float w = (m == -INFINITY) ? 0.f : expf(m - M);
            wts[s * kGP + h] = w;
            L += w * ld_cg(ml + 1);
        }
        L = warp_sum(L);
        if (lane == 0) s_L[h] = L;
    }
    __syncthreads();
    // Each thread merges two float4 columns (G * D / 4 <= 2 * kThreads) and keeps the loads of eight
    // splits of both in flight at once: the merge is bound by L2 latency, not bandwidth.
    constexpr int kMB = 8;
    static_assert(kGP * D / 4 <= 2 * kThreads, "two float4 columns per thread");
    const int nitem = (G * D) / 4;
    const int ia = tid, ib = tid + kThreads;
    const int ga = (ia * 4) / D, gb = (ib * 4) / D;
    const float* pa = p.part_o + (p0 * Hkv + kvh) * kGP * D + (long long)ia * 4;
    const float* pb = p.part_o + (p0 * Hkv + kvh) * kGP * D + (long long)ib * 4;
    const long long sstride = (long long)Hkv * kGP * D;
    float4 oa = make_float4(0.f, 0.f, 0.f, 0.f), ob = oa;
    for (int s0 = 0; s0 < ns; s0 += kMB) {
        float4 va[kMB], vb[kMB];
#pragma unroll
        for (int j = 0; j < kMB; j++) {
            const bool ok = s0 + j < ns;
            va[j] = (ok && ia < nitem) ? __ldcg(reinterpret_cast<const float4*>(pa + (s0 + j) * sstride)) : make_float4(0.f, 0.f, 0.f, 0.f);
            vb[j] = (ok && ib < nitem) ? __ldcg(reinterpret_cast<const float4*>(pb + (s0 + j) * sstride)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < kMB; j++) {
            if (s0 + j >= ns) break;
            const float wa = ia < nitem ? wts[(s0 + j) * kGP + ga] : 0.f;
            const float wb = ib < nitem ? wts[(s0 + j) * kGP + gb] : 0.f;
            oa.x += wa * va[j].x; oa.y += wa * va[j].y; oa.z += wa * va[j].z; oa.w += wa * va[j].w;
            ob.x += wb * vb[j].x; ob.y += wb * vb[j].y; ob.z += wb * vb[j].z; ob.w += wb * vb[j].w;
        }
    }
    for (int which = 0; which < 2; which++) {
        const int idx4 = which ? ib : ia;
        if (idx4 >= nitem) continue;
        const int g = (idx4 * 4) / D, i = idx4 * 4 - g * D;
        const float4 o = which ? ob : oa;
        const float L = s_L[g];
        float ov[4] = {o.x, o.y, o.z, o.w};
        const int h = kvh * G + g;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float O = (L > 0.f) ? ov[e] / L : 0.f;
            if (p.gate) {  // mul_sigmoid_inplace, core/cpu_ops.cpp:15-22
                const float z = load_as_float(proj_row, p.proj_dtype,
                                              p.gate_off + (long long)h * p.q_head_stride + i + e);
                O = O / (1.0f + expf(-z));
            }
            store_from_float(p.out, p.out_dtype, (long long)b * p.out_stride + (long long)h * D + i + e, O);
        }
    }
    if (tid == 0) {
        p.cnt_head[b * Hkv + kvh] = 0;
        __threadfence();
        const int prev = atomicAdd(&p.cnt_seq[b], 1);
        if (prev == Hkv - 1) {
            if (p.append && p.kv_len) {
                p.kv_len[seq] = len1;
                p.kv_start[seq] = start1;
            }
            p.cnt_seq[b] = 0;
        }
    }
}

}  // namespace

int fa_decode_max_splits(int head_dim) {
    const size_t tiles = size_t(kStages) * kTile * head_dim * 2;
    return (int)(tiles / (kGP * sizeof(float)));
}

size_t fa_decode_smem_bytes(int head_dim) {
    return head_dim == 256 ? Smem<256>::total : Smem<128>::total;
}

int launch_fa_decode(const FaDecodeParams& p0, int head_dim, int n_blocks, cudaStream_t stream) {
    FaDecodeParams p = p0;
    const int eb = dtype_bytes(p.proj_dtype);
    p.proj_vec = (uintptr_t)p.proj % 16 == 0 && (p.proj_stride * eb) % 16 == 0 && ((long long)p.q_head_stride * eb) % 16 == 0 &&
                 (p.k_off * eb) % 16 == 0 && (p.v_off * eb) % 16 == 0 && head_dim % 8 == 0;
    dim3 grid(n_blocks, p.Hkv);
    if (head_dim != 256 && head_dim != 128) return ANELM_ERR_UNSUPPORTED;
    const size_t sm = head_dim == 256 ? Smem<256>::total : Smem<128>::total;
    if (p.cluster_ns >= 2 && p.cluster_ns <= 16 && n_blocks == p.cluster_ns) {
        // one row: its splits of each kv head form a cluster and merge through shared memory
        auto kern = head_dim == 256 ? fa_decode_kernel<256, true> : fa_decode_kernel<128, true>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (p.cluster_ns > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = sm;
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = p.cluster_ns;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // prologue overlaps the previous kernel
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        if (cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess) return ANELM_OK;
        cudaGetLastError();  // a cluster that cannot be placed: merge through global memory instead
    }
    auto kern = head_dim == 256 ? fa_decode_kernel<256, false> : fa_decode_kernel<128, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    kern<<<grid, kThreads, sm, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

}  // namespace anelm
