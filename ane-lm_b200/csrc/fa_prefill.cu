// Causal prefill for the Qwen3.5 gated full-attention core (sm_100a, tcgen05 + TMA).
//
// Replaces the per-token prefill loop of the reference (qwen3_5.cpp:1205-1217,
// serve_hybrid.py:368-370; the chunks of forward_batch, qwen3_5.cpp:1164-1217, called by
// generate.cpp:57-73 at a running start_pos), which runs forward_full_attn_from_proj
// (qwen3_5.cpp:944-1002) once per prompt token: for each token t, QK RMSNorm, RoPE at
// position start_pos + t, ring append (qwen3_5.cpp:974-986: slot start + len, or the
// oldest slot once the ring is full), softmax attention over the ring, sigmoid gate.  The
// result is the same set of outputs, computed as one causal attention over [old | new]
// keys: new token t sees the ring's old tokens and the new tokens 0..t, at most `capacity`
// tokens in all (the ring's window), so prompts may continue a non-empty ring and may be
// longer than the ring.
//
// Three launches:
//   fa_prefill_gather_kernel  per sequence: snapshot of the ring's len / start / capacity and
//                           copy of the old tokens the first new token still sees (the last
//                           min(len, capacity - 1), in the ring's logical order) into the key
//                           rows ahead of the new tokens;
//   fa_prefill_prep_vec_kernel  per token: RMSNorm + RoPE of the q and k heads (same arithmetic
//                           as the decode prologue), fp16 Q [B][Hq][n_pad][D], K and V
//                           [B][Hkv][P + n_pad][D] (new token t at row P + t), sigmoid(gate) for
//                           the epilogue, and the ring append (slot (start + len + t) mod
//                           capacity for the tokens that stay in the ring; final len / start as
//                           the per-token updates leave them).  Warp per 256-element segment,
//                           16-byte lanes (fa_prefill_prep_kernel: same work for any shape);
//   fa_prefill_kernel       one CTA per (q head, 128-row query tile, sequence); within a sequence
//                           all heads' longest causal tiles are dispatched first; 11 warps:
//     warps 0-7  softmax: warps w and w+4 share TMEM lanes [32(w%4), +32) and take keys
//             [0, 64) / [64, 128) of each 128-key S tile; tcgen05.ld of the S row, causal mask,
//             row max exchanged through shared memory (pairwise named barriers), lazy rescale
//             of O (only when the max grows by more than 2^8), P = exp2(...) as fp16 pairs
//             written over the first 64 columns of the S buffer (tcgen05.st);
//     warp 8  TMA producer: Q (4 boxes), then one 64 KB K tile per key tile, then the
//             sigmoid(gate) tile into the K buffer once the last Q K^T has read it;
//     warp 9  MMA issuer (one thread): S = Q K^T (M=128, N=128, K=256) into one of two
//             128-column TMEM S buffers, O += P V with A = P from TMEM and B = V read
//             MN-major from its natural [key][d] layout (M=128, N=256, K=128) into the
//             256-column O accumulator, so Q K^T of tile j+1 overlaps the softmax of tile j;
//     warp 10 TMA producer: one 64 KB V tile per key tile.
//   Epilogue: O / l * sigmoid(gate) into 128B-swizzled tiles in the idle Q buffer and four TMA
//   tile stores (a 3D tensor map clips rows past the sequence end); other output dtypes /
//   alignments store rows from a staged fp32 copy.  All MMAs are kind::f16 (fp16 operands,
//   fp32 accumulation in TMEM).  Every mbarrier wait is bounded and records ANELM_ERR_TIMEOUT
//   instead of hanging.
#include <cuda.h>
#include <algorithm>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

namespace anelm {

namespace {

constexpr int kBM = 128;   // query rows per CTA
constexpr int kBN = 128;   // keys per tile (Q K^T at N = 128: a tcgen05.mma costs ~100 cycles even at
                           // N = 64, so narrower tiles leave the tensor core two-thirds idle)
constexpr int kD = 256;    // head dim of this kernel
constexpr int kQBytes = kBM * kD * 2;        // 64 KB: 4 boxes of 128 rows x 64 d
constexpr int kKBytes = kBN * kD * 2;        // 64 KB: 4 boxes of 128 keys x 64 d
constexpr int kVBytes = kD * kBN * 2;        // 64 KB: V, 4 boxes of 128 keys x 64 d (MN-major B of P V)
constexpr int kSmemTiles = kQBytes + kKBytes + kVBytes;
constexpr int kSmemBytes = kSmemTiles + 256 + 6 * 128 * 4 + 1024;  // barriers, softmax exchange, alignment
constexpr int kSoftmaxWarps = 8;             // two per TMEM lane quadrant, 64 keys of each tile each
constexpr int kWarpK = kSoftmaxWarps, kWarpMma = kSoftmaxWarps + 1, kWarpV = kSoftmaxWarps + 2;
constexpr int kThreads = 32 * (kSoftmaxWarps + 3);
constexpr uint32_t kTmemCols = 512;          // S0 [0,128), S1 [128,256) (P over the first 64 of each), O [256,512)
constexpr uint32_t kOCol = 2 * kBN;
constexpr int kORow = kD + 4;                // fp32 words per staged output row (padding: no bank conflicts)
static_assert(kBM * kORow * 4 <= kSmemTiles, "output staging fits the Q/K/V buffers");

// 2^x by the hardware approximation (PTX ex2.approx.ftz: relative error ~2^-22, -inf -> +0)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1/x by the hardware approximation (PTX rcp.approx.ftz: relative error ~2^-23, 1/inf -> 0)
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


// ---- the ring of one sequence as it was before this call (written by the gather kernel) ----
struct RingSnap {
    int len, start, cap, Pb;  // Pb: old tokens in key rows [P - Pb, P)
};

__device__ __forceinline__ RingSnap ring_snap(const FaPrefillParams& p, int b) {
    const int4 m = *reinterpret_cast<const int4*>(p.meta + 4 * b);
    return {m.x, m.y, m.z, m.w};
}

// Ring slot of new token t: the update of qwen3_5.cpp:974-983 applied once per token puts token t
// at slot start + len + t modulo the capacity; -1 if a later token of this call takes that slot.
__device__ __forceinline__ int ring_slot(const RingSnap& r, int n, int t) {
    if (t < n - r.cap) return -1;
    return (int)(((long long)r.start + r.len + t) % r.cap);
}

// len / start after the n appends of this call (the same per-token updates).
__device__ __forceinline__ void ring_finish(const FaPrefillParams& p, const RingSnap& r, int seq) {
    const long long total = (long long)r.len + p.n;
    p.kv_len[seq] = (int)(total < r.cap ? total : r.cap);
    p.kv_start[seq] = (int)(((long long)r.start + (total > r.cap ? total - r.cap : 0)) % r.cap);
}

// One CTA per 64 key rows (at least one per sequence).  Takes the snapshot of sequence b's ring
// and copies its last Pb tokens, oldest first from `start` as gqa_attention reads them
// (cpu_ops.cpp:161-163), into key rows [P - Pb, P); rows of the first key tile below P - Pb are
// zeroed (an attention tile reads them, masked, and P V needs them finite).  Runs before the
// prep appends to the ring, so it reads the old tokens only.
__global__ void __launch_bounds__(256) fa_prefill_gather_kernel(const FaPrefillParams p) {
    // the prep may start now (programmatic dependent launch): it waits for this grid before it reads
    // the snapshots or appends to a ring
    asm volatile("griddepcontrol.launch_dependents;");
    const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = p.seq_ids ? p.seq_ids[b] : 0;
    const int len = p.kv_len[seq], start = p.kv_start[seq], cap = p.kv_cap[seq];
    int Pb = min(len, cap - 1);
    if (Pb > p.P) {  // the host sizes P from its record of every ring's length; that record was wrong
        if (blockIdx.x == 0 && threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, ANELM_ERR_STATE);
        Pb = p.P;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<int4*>(p.meta + 4 * b) = make_int4(len, start, cap, Pb);
    const int first = (p.P - Pb) / kBN * kBN;
    const int r1 = min(p.P, ((int)blockIdx.x + 1) * 64);
    const long long base = p.kv_base[seq];
    const int vecs = p.Hkv * (kD / 8);  // 16-byte vectors per slot row [Hkv][kD]
    for (int r = (int)blockIdx.x * 64 + warp; r < r1; r += 8) {
        if (r < first) continue;
        const bool old = r >= p.P - Pb;
        long long src = 0;
        if (old) {
            const int j = len - (p.P - r);  // logical index, 0 = oldest
            src = (base + (long long)(((long long)start + j) % cap)) * p.Hkv * kD;
        }
        for (int e = lane; e < vecs; e += 32) {
            const int kh = e / (kD / 8), c = e % (kD / 8);
            const long long dst = (((long long)b * p.Hkv + kh) * p.n_tot + r) * kD + 8 * c;
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
            if (old) {
                kv = *reinterpret_cast<const uint4*>(p.k_pool + src + (long long)e * 8);
                vv = *reinterpret_cast<const uint4*>(p.v_pool + src + (long long)e * 8);
            }
            *reinterpret_cast<uint4*>(p.Kh + dst) = kv;
            *reinterpret_cast<uint4*>(p.Vh + dst) = vv;
        }
    }
}

// Single-stage K and V buffers: a 64 KB load (~0.4 us) hides behind the other operand's
// MMAs (~1.4 us per tile).  Each barrier is used once per tile (K, V) or once per use of
// a TMEM buffer (S_FULL, P_FULL, PV_DONE), so no barrier runs two phases ahead of a waiter.
// PV_DONE[s] frees TMEM buffer s (its P was read) and says O is stable for rescaling.
// Destinations of the output tiles: this context's own output, or, for a head-sharded prefill, the
// output buffer of every rank (peer buffers mapped into this process), each a [B][n][cols] tensor
// of which this launch's heads fill columns [col0, col0 + Hq D).  wait_full: the storing thread
// waits until the stores have completed, not just until their shared-memory source was read.
constexpr int kMaxOuts = 8;
struct OutMaps {
    CUtensorMap m[kMaxOuts];
    int n, col0, wait_full;
};

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 2, V_FULL = 3, V_EMPTY = 4, S_FULL = 5, P_FULL = 7, PV_DONE = 9,
           G_FULL = 11, N_BARS = 12 };

__device__ __forceinline__ void rope_cs_pf(const FaPrefillParams& p, int pos, int j, float& c, float& s) {
    const int half = p.rot_dim >> 1;
    if (pos >= 0 && pos < p.rope_len && p.rope_cos) {
        c = p.rope_cos[(long long)pos * half + j];
        s = p.rope_sin[(long long)pos * half + j];
    } else {  // core/cpu_ops.cpp:51-56
        const float freq = 1.0f / powf(p.rope_theta, (float)(2 * j) / (float)p.rot_dim);
        const float angle = (float)pos * freq;
        c = cosf(angle);
        s = sinf(angle);
    }
}

// One token of one sequence per CTA (256 threads).
__global__ void __launch_bounds__(256) fa_prefill_prep_kernel(const FaPrefillParams p) {
    extern __shared__ float xs[];  // [(Hq + Hkv) vectors][kD], then v [Hkv][kD]
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the gather kernel's snapshots (a no-op for a plain launch)
    const int t = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Hq = p.Hq, Hkv = p.Hkv;
    const int nvec = Hq + Hkv;
    const long long qrow = ((long long)b * Hq) * p.n_pad + t;
    const long long krow = ((long long)b * Hkv) * p.n_tot + p.P + t;
    if (t >= p.n) {  // padding rows: finite zeros
        for (int idx = tid; idx < Hq * kD; idx += 256)
            p.Qh[(qrow + (long long)(idx / kD) * p.n_pad) * kD + idx % kD] = __float2half_rn(0.f);
        for (int idx = tid; idx < Hkv * kD; idx += 256) {
            const long long o = (krow + (long long)(idx / kD) * p.n_tot) * kD + idx % kD;
            p.Kh[o] = __float2half_rn(0.f);
            p.Vh[o] = __float2half_rn(0.f);
        }
        return;
    }
    const char* row = reinterpret_cast<const char*>(p.proj) +
                      ((long long)b * p.n + t) * p.proj_stride * dtype_bytes(p.proj_dtype);
    float* vs = xs + nvec * kD;
    for (int idx = tid; idx < nvec * kD; idx += 256) {
        const int v = idx / kD, i = idx % kD;
        const long long off = v < Hq ? (long long)v * 2 * kD + i : (long long)Hq * 2 * kD + (long long)(v - Hq) * kD + i;
        xs[idx] = load_as_float(row, p.proj_dtype, off);
    }
    for (int idx = tid; idx < Hkv * kD; idx += 256)
        vs[idx] = load_as_float(row, p.proj_dtype, (long long)Hq * 2 * kD + (long long)Hkv * kD + idx);
    __syncthreads();
    if (p.qk_norm) {  // rmsnorm, cpu_ops.cpp:24-30 (qwen3_5.cpp:952-959)
        for (int v = warp; v < nvec; v += 8) {
            float* x = xs + v * kD;
            const float* w = v < Hq ? p.q_norm : p.k_norm;
            float ss = 0.f;
            for (int i = lane; i < kD; i += 32) ss += x[i] * x[i];
            ss = warp_sum(ss);
            const float r = 1.0f / sqrtf(ss / (float)kD + p.rms_eps);
            for (int i = lane; i < kD; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
        }
        __syncthreads();
    }
    const int pos = p.start_pos + t;
    if (p.rot_dim > 0) {  // apply_rope_cached, cpu_ops.cpp:40-63 (or rotate-half)
        const int half = p.rot_dim >> 1;
        for (int idx = tid; idx < nvec * half; idx += 256) {
            const int v = idx / half, j = idx % half;
            float* x = xs + v * kD;
            float c, s;
            rope_cs_pf(p, pos, j, c, s);
            const int i0 = p.rope_mode == ANELM_ROPE_INTERLEAVED ? 2 * j : j;
            const int i1 = p.rope_mode == ANELM_ROPE_INTERLEAVED ? 2 * j + 1 : j + half;
            const float v0 = x[i0], v1 = x[i1];
            x[i0] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
            x[i1] = p.rope_mode == ANELM_ROPE_INTERLEAVED ? __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c))
                                                          : __fadd_rn(__fmul_rn(v1, c), __fmul_rn(v0, s));
        }
        __syncthreads();
    }
    const int seq = p.seq_ids ? p.seq_ids[b] : 0;
    const RingSnap rs = ring_snap(p, b);
    const int slot = ring_slot(rs, p.n, t);
    const long long slot_row = slot >= 0 ? (p.kv_base[seq] + slot) * Hkv : -1;
    for (int idx = tid; idx < Hq * kD; idx += 256)
        p.Qh[(qrow + (long long)(idx / kD) * p.n_pad) * kD + idx % kD] = __float2half_rn(xs[idx]);
    for (int idx = tid; idx < Hkv * kD; idx += 256) {
        const int v = idx / kD, i = idx % kD;
        const __half kh = __float2half_rn(xs[(Hq + v) * kD + i]);
        const __half vh = __float2half_rn(vs[idx]);
        const long long o = (krow + (long long)v * p.n_tot) * kD + i;
        p.Kh[o] = kh;
        p.Vh[o] = vh;
        if (slot_row >= 0) {  // ring append (qwen3_5.cpp:984-986)
            p.k_pool[(slot_row + v) * kD + i] = kh;
            p.v_pool[(slot_row + v) * kD + i] = vh;
        }
    }
    if (p.SG) {  // sigmoid of the gate columns for the TMA epilogue (mul_sigmoid_inplace, cpu_ops.cpp:15-22)
        __half* sg = p.SG + ((long long)b * p.n + t) * Hq * kD;
        for (int idx = tid; idx < Hq * kD; idx += 256) {
            const float g = load_as_float(row, p.proj_dtype, (long long)(idx / kD) * 2 * kD + kD + idx % kD);
            sg[idx] = __float2half_rn(1.0f / (1.0f + expf(-g)));
        }
    }
    if (t == 0 && tid == 0) ring_finish(p, rs, seq);
}

// Same work as fa_prefill_prep_kernel, organised for bandwidth: one CTA per token, each warp owns
// whole 256-element segments of the token's projection row (segment s = q head s/2 or its gate for
// s < 2 Hq, then the k heads, then the v heads; it starts at element 256 s), one 16-byte vector of
// 8 elements per lane.  A warp issues the loads of up to four segments before using any, RMSNorm is a
// warp reduction and rotate-half RoPE pairs lanes by shuffle, so no shared memory or block barrier is
// involved.  Needs a 16-byte aligned projection row and rot_dim % 16 == 0.
constexpr int kPrepBatch = 4;  // segments whose loads a warp issues together (more registers per thread
                               // cost occupancy: 5 at 3 CTAs per SM ran slower than 4 at 4)
__device__ __forceinline__ uint4 half8(const float (&x)[8]) { return pack8(x, false); }

// The prep arithmetic of one 16-byte lane (elements e0 = 8 lane .. +8) of segment s of a token's
// projection row [q_0 | gate_0 | ... | q_{Hq-1} | gate_{Hq-1} | k_0 .. k_{Hkv-1} | v_0 .. v_{Hkv-1}]:
// RMSNorm + RoPE of q / k, sigmoid of the gate, and the fp16 stores (Q, K, V, SG, ring pools).
// `qn` / `kn` hold this lane's 8 norm weights; `cs(j, c, s)` gives the RoPE cos / sin of pair j.
template <class CS>
__device__ __forceinline__ void prep_segment(const FaPrefillParams& p, float (&v)[8], int s, int lane, int b, int t,
                                             long long slot_row, const float* qn, const float* kn, CS cs) {
    const int Hq = p.Hq, Hkv = p.Hkv;
    const int e0 = 8 * lane, half = p.rot_dim >> 1;
    const bool is_q = s < 2 * Hq && !(s & 1), is_gate = s < 2 * Hq && (s & 1);
    const bool is_k = s >= 2 * Hq && s < 2 * Hq + Hkv;
    if (is_q || is_k) {
        if (p.qk_norm) {  // rmsnorm, cpu_ops.cpp:24-30 (qwen3_5.cpp:952-959)
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 8; e++) ss += v[e] * v[e];
            ss = warp_sum(ss);
            const float r = 1.0f / sqrtf(ss / (float)kD + p.rms_eps);
            const float* w = is_q ? qn : kn;
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fmul_rn(v[e], r), w[e]);
        }
        if (p.rot_dim > 0) {  // apply_rope_cached, cpu_ops.cpp:40-63 (or rotate-half)
            if (p.rope_mode == ANELM_ROPE_INTERLEAVED) {
                if (e0 < p.rot_dim) {
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        float c, sn;
                        cs((e0 + e) >> 1, c, sn);
                        const float v0 = v[e], v1 = v[e + 1];
                        v[e] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
                        v[e + 1] = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c));
                    }
                }
            } else {
                const int hl = half >> 3;  // lanes per rotary half
                float o[8];
#pragma unroll
                for (int e = 0; e < 8; e++) o[e] = __shfl_sync(0xffffffffu, v[e], lane < hl ? lane + hl : lane - hl);
                if (e0 < p.rot_dim) {
                    const bool first = lane < hl;
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        float c, sn;
                        cs((first ? e0 : e0 - half) + e, c, sn);
                        v[e] = first ? __fsub_rn(__fmul_rn(v[e], c), __fmul_rn(o[e], sn))
                                     : __fadd_rn(__fmul_rn(v[e], c), __fmul_rn(o[e], sn));
                    }
                }
            }
        }
    }
    if (is_q) {
        const int h = s >> 1;
        *reinterpret_cast<uint4*>(p.Qh + (((long long)b * Hq + h) * p.n_pad + t) * kD + e0) = half8(v);
    } else if (is_gate) {
        if (p.SG) {  // sigmoid of the gate for the TMA epilogue (mul_sigmoid_inplace, cpu_ops.cpp:15-22);
                     // stored as fp16, so the hardware exp2 and reciprocal are exact enough
            float g[8];
#pragma unroll
            for (int e = 0; e < 8; e++) g[e] = rcp_approx(1.0f + ex2_approx(-1.4426950408889634f * v[e]));
            *reinterpret_cast<uint4*>(p.SG + (((long long)b * p.n + t) * Hq + (s >> 1)) * kD + e0) = half8(g);
        }
    } else {
        const int kh = is_k ? s - 2 * Hq : s - 2 * Hq - Hkv;
        const uint4 hv = half8(v);
        const long long o = (((long long)b * Hkv + kh) * p.n_tot + p.P + t) * kD + e0;
        *reinterpret_cast<uint4*>((is_k ? p.Kh : p.Vh) + o) = hv;
        if (slot_row >= 0)  // ring append (qwen3_5.cpp:984-986)
            *reinterpret_cast<uint4*>((is_k ? p.k_pool : p.v_pool) + (slot_row + kh) * kD + e0) = hv;
    }
}

// Padding rows t >= n of token (b, t): finite zeros in Q, K and V (this warp's heads).
__device__ __forceinline__ void prep_zero_row(const FaPrefillParams& p, int b, int t, int warp, int nwarps, int e0) {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int h = warp; h < p.Hq; h += nwarps)
        *reinterpret_cast<uint4*>(p.Qh + (((long long)b * p.Hq + h) * p.n_pad + t) * kD + e0) = z;
    for (int h = warp; h < p.Hkv; h += nwarps) {
        const long long o = (((long long)b * p.Hkv + h) * p.n_tot + p.P + t) * kD + e0;
        *reinterpret_cast<uint4*>(p.Kh + o) = z;
        *reinterpret_cast<uint4*>(p.Vh + o) = z;
    }
}

__global__ void __launch_bounds__(256, 4) fa_prefill_prep_vec_kernel(const FaPrefillParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the gather kernel's snapshots (a no-op for a plain launch)
    const int t = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int Hq = p.Hq, Hkv = p.Hkv;
    const int nseg = 2 * Hq + 2 * Hkv;
    const int e0 = 8 * lane;  // this lane's first element within a 256-element segment
    if (t >= p.n) {
        prep_zero_row(p, b, t, warp, 8, e0);
        return;
    }
    const char* row = reinterpret_cast<const char*>(p.proj) +
                      ((long long)b * p.n + t) * p.proj_stride * dtype_bytes(p.proj_dtype);
    const int pos = p.start_pos + t;
    const int seq = p.seq_ids ? p.seq_ids[b] : 0;
    const RingSnap rs = ring_snap(p, b);
    const int slot = ring_slot(rs, p.n, t);
    const long long slot_row = slot >= 0 ? (p.kv_base[seq] + slot) * Hkv : -1;
    const auto cs = [&](int j, float& c, float& sn) { rope_cs_pf(p, pos, j, c, sn); };
    for (int s0 = warp; s0 < nseg; s0 += 8 * kPrepBatch) {
        float x[kPrepBatch][8];
#pragma unroll
        for (int i = 0; i < kPrepBatch; i++)
            if (s0 + 8 * i < nseg) load8(row, p.proj_dtype, (long long)(s0 + 8 * i) * kD + e0, x[i]);
#pragma unroll
        for (int i = 0; i < kPrepBatch; i++) {
            const int s = s0 + 8 * i;
            if (s >= nseg) break;
            prep_segment(p, x[i], s, lane, b, t, slot_row, p.q_norm + e0, p.k_norm + e0, cs);
        }
    }
    if (t == 0 && threadIdx.x == 0) ring_finish(p, rs, seq);
}

// Streaming form of the prep for 16-bit projections: a persistent CTA walks the tokens
// u = blockIdx.x, blockIdx.x + gridDim.x, ... of the [B][n_pad] grid.  Warp 8 copies each
// token's whole projection row (and its RoPE table rows) into one of kPrepStages shared-memory
// stages with untiled bulk copies, kPrepStages - 1 tokens ahead; warps 0-7 take the staged row's
// segments.  The arithmetic is prep_segment's (same roundings, same results); the work is laid
// out for instruction count, which bounds this kernel once the copies stream: a lane's RoPE
// cos / sin (8 pairs) are read once per token as 16-byte words, a segment's role is a
// warp-uniform branch, lanes past rot_dim select their unrotated value instead of branching,
// and token / stage indices advance incrementally (no 64-bit division per token).
constexpr int kPrepStages = 3;
constexpr int kPrepWarps = 8;  // consumer warps; warp kPrepWarps is the copy producer
constexpr int kPrepCtas = 3;   // CTAs per SM: the consumers' latency (warp reductions) needs the warps
constexpr int kPrepStageMax = 24 * 1024;  // stage bytes that still let kPrepCtas CTAs share an SM

// RoPE coefficients of lane elements e0 + e (e0 = 8 lane) at one position.  Rotate-half: element
// e0 + e rotates with element e0 + e -+ half by angle index (e0 mod half) + e, and `sg` carries
// the sign of the partner term (-sin in the first half, +sin in the second).  Interleaved: pair
// (e0 + e, e0 + e + 1), e even, uses angle index (e0 + e) / 2.  Lanes past rot_dim keep (1, 0).
template <bool kHalf>
__device__ __forceinline__ void prep_rope_lane(const FaPrefillParams& p, bool tab, const float* tcos, int pos,
                                               int lane, float (&c)[8], float (&sg)[8]) {
    const int e0 = 8 * lane, half = p.rot_dim >> 1;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        c[e] = 1.f;
        sg[e] = 0.f;
    }
    if (e0 >= p.rot_dim) return;
    if (kHalf) {
        const bool first = e0 < half;
        const int j0 = first ? e0 : e0 - half;
        if (tab) {
            const float4 c0 = *reinterpret_cast<const float4*>(tcos + j0);
            const float4 c1 = *reinterpret_cast<const float4*>(tcos + j0 + 4);
            const float4 s0 = *reinterpret_cast<const float4*>(tcos + half + j0);
            const float4 s1 = *reinterpret_cast<const float4*>(tcos + half + j0 + 4);
            const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                c[e] = cc[e];
                sg[e] = first ? -ss[e] : ss[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                float s;
                rope_cs_pf(p, pos, j0 + e, c[e], s);
                sg[e] = first ? -s : s;
            }
        }
    } else {
        const int j0 = e0 >> 1;
        if (tab) {
            const float4 c0 = *reinterpret_cast<const float4*>(tcos + j0);
            const float4 s0 = *reinterpret_cast<const float4*>(tcos + half + j0);
            const float cc[4] = {c0.x, c0.y, c0.z, c0.w}, ss[4] = {s0.x, s0.y, s0.z, s0.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                c[2 * i] = c[2 * i + 1] = cc[i];
                sg[2 * i] = sg[2 * i + 1] = ss[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                rope_cs_pf(p, pos, j0 + i, c[2 * i], sg[2 * i]);
                c[2 * i + 1] = c[2 * i];
                sg[2 * i + 1] = sg[2 * i];
            }
        }
    }
}

// RMSNorm (cpu_ops.cpp:24-30) and RoPE (cpu_ops.cpp:40-63, or rotate-half) of one q / k segment,
// with prep_segment's roundings; `rot` is false for lanes past rot_dim.
template <bool kHalf>
__device__ __forceinline__ void prep_qk_lane(const FaPrefillParams& p, float (&v)[8], const float (&w)[8],
                                             const float (&c)[8], const float (&sg)[8], bool rot, int partner) {
    if (p.qk_norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss += v[e] * v[e];
        ss = warp_sum(ss);
        const float r = 1.0f / sqrtf(ss / (float)kD + p.rms_eps);
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fmul_rn(v[e], r), w[e]);
    }
    if (p.rot_dim > 0) {
        if (kHalf) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float o = __shfl_sync(0xffffffffu, v[e], partner);
                const float y = __fadd_rn(__fmul_rn(v[e], c[e]), __fmul_rn(o, sg[e]));
                v[e] = rot ? y : v[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const float v0 = v[e], v1 = v[e + 1];
                const float y0 = __fsub_rn(__fmul_rn(v0, c[e]), __fmul_rn(v1, sg[e]));
                const float y1 = __fadd_rn(__fmul_rn(v0, sg[e]), __fmul_rn(v1, c[e]));
                v[e] = rot ? y0 : v0;
                v[e + 1] = rot ? y1 : v1;
            }
        }
    }
}

template <bool kHalf, bool kBf>
__global__ void __launch_bounds__(32 * (kPrepWarps + 1), kPrepCtas)
    fa_prefill_prep_bulk_kernel(const FaPrefillParams p, int stage_bytes, int rope_off) {
    extern __shared__ __align__(128) uint8_t prep_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(prep_smem);
    uint64_t* empty = full + kPrepStages;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + kPrepStages);
    uint8_t* stage0 = prep_smem + 128;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int Hq = p.Hq, Hkv = p.Hkv, n = p.n, n_pad = p.n_pad;
    const int nseg = 2 * Hq + 2 * Hkv;
    const uint32_t row_bytes = (uint32_t)nseg * kD * 2;
    const int half = p.rot_dim >> 1;
    const int G = gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPrepStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], kPrepWarps);
        }
        *abort = 0;
        tc::fence_barrier_init();
        // the attention launch that follows may start its prologue now: every CTA of this persistent
        // grid is resident, so its CTAs only take SMs this grid has left (they wait for its results
        // at griddepcontrol.wait)
        asm volatile("griddepcontrol.launch_dependents;");
    }
    __syncthreads();
    // token u = b n_pad + t, advanced by G per step (the host keeps B n_pad + G below 2^31)
    if (warp == kPrepWarps) {  // producer: one thread issues every copy
        if (lane != 0) return;
        int last_ph[kPrepStages];
#pragma unroll
        for (int s = 0; s < kPrepStages; s++) last_ph[s] = -1;
        int b = blockIdx.x / n_pad, t = blockIdx.x % n_pad, s = 0;
        uint32_t ph = 0;  // this pass's phase of stage s (flips each time s wraps)
        for (int k = 0; b < p.B; k++) {
            if (k >= kPrepStages && !tc::mbar_wait(&empty[s], ph ^ 1u, p.err, ANELM_ERR_TIMEOUT, abort)) break;
            last_ph[s] = (int)ph;
            if (t >= n) {  // padding row: nothing to copy
                tc::mbar_arrive(&full[s]);
            } else {
                uint8_t* st = stage0 + (size_t)s * stage_bytes;
                const int pos = p.start_pos + t;
                const bool tab = p.rot_dim > 0 && p.rope_cos && pos >= 0 && pos < p.rope_len;
                tc::mbar_arrive_expect_tx(&full[s], row_bytes + (tab ? 8u * half : 0u));
                tc::bulk_load(st, reinterpret_cast<const char*>(p.proj) + ((long long)b * n + t) * p.proj_stride * 2,
                              row_bytes, &full[s]);
                if (tab) {
                    tc::bulk_load(st + rope_off, p.rope_cos + (long long)pos * half, 4u * half, &full[s]);
                    tc::bulk_load(st + rope_off + 4 * half, p.rope_sin + (long long)pos * half, 4u * half, &full[s]);
                }
            }
            t += G;
            while (t >= n_pad) {
                t -= n_pad;
                b++;
            }
            if (++s == kPrepStages) {
                s = 0;
                ph ^= 1u;
            }
        }
        // every issued copy has landed before the CTA can exit (normally the consumers already
        // waited for them; after a timeout this bounds the wait for the ones still in flight)
#pragma unroll
        for (int s2 = 0; s2 < kPrepStages; s2++)
            if (last_ph[s2] >= 0)
                for (uint32_t i = 0; i < tc::kWaitPolls; i++)
                    if (tc::mbar_try_wait(&full[s2], (uint32_t)last_ph[s2])) break;
        return;
    }
    const int e0 = 8 * lane;
    float qn[8], kn[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        qn[e] = p.qk_norm ? p.q_norm[e0 + e] : 0.f;
        kn[e] = p.qk_norm ? p.k_norm[e0 + e] : 0.f;
    }
    const bool rot = e0 < p.rot_dim;
    const int hl = half >> 3;  // lanes per rotary half (rotate-half partner lane = lane +- hl)
    const int partner = lane < hl ? lane + hl : lane - hl;
    const long long q_hstride = (long long)n_pad * kD;    // Q: [B][Hq][n_pad][kD]
    const long long k_hstride = (long long)p.n_tot * kD;  // K / V: [B][Hkv][P + n_pad][kD]
    // job j of the token -> segment: with Hq a multiple of 8, blocks of 8 jobs alternate q heads and
    // gates (q 0-7, gate 0-7, q 8-15, ...), so each warp gets the same number of RMSNorm + RoPE
    // segments (the warps' slowest bounds the stage's release); k and v heads follow
    const bool mix = (Hq & 7) == 0;
    // consumers read the gather kernel's ring snapshots and append to the rings it read: wait for that
    // grid (the producer's projection copies do not depend on it and run ahead)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    int cur_b = -1, seq = 0;  // the sequence of row b, its pool base and ring snapshot, reloaded when b changes
    long long kv0 = 0;
    RingSnap rs{0, 0, 1, 0};
    int b = blockIdx.x / n_pad, t = blockIdx.x % n_pad, s = 0;
    uint32_t ph = 0;
    while (b < p.B) {
        if (!tc::mbar_wait(&full[s], ph, p.err, ANELM_ERR_TIMEOUT, abort)) break;
        if (t >= n) {
            prep_zero_row(p, b, t, warp, kPrepWarps, e0);
        } else {
            const uint8_t* st = stage0 + (size_t)s * stage_bytes;
            const int pos = p.start_pos + t;
            if (b != cur_b) {
                cur_b = b;
                seq = p.seq_ids ? p.seq_ids[b] : 0;
                kv0 = p.kv_base[seq];
                rs = ring_snap(p, b);
            }
            const bool tab = p.rot_dim > 0 && p.rope_cos && pos >= 0 && pos < p.rope_len;
            float c[8], sg[8];
            prep_rope_lane<kHalf>(p, tab, reinterpret_cast<const float*>(st + rope_off), pos, lane, c, sg);
            __half* qrow = p.Qh + ((long long)b * Hq * n_pad + t) * kD + e0;
            __half* krow = p.Kh + ((long long)b * Hkv * p.n_tot + p.P + t) * kD + e0;
            __half* vrow = p.Vh + ((long long)b * Hkv * p.n_tot + p.P + t) * kD + e0;
            __half* grow = p.SG ? p.SG + ((long long)b * n + t) * Hq * kD + e0 : nullptr;
            const int slot = ring_slot(rs, n, t);  // ring append (qwen3_5.cpp:984-986), if the token stays
            const long long pool = slot >= 0 ? (kv0 + slot) * Hkv * kD + e0 : -1;
            for (int j = warp; j < nseg; j += kPrepWarps) {
                int sgm = j;
                if (mix && j < 2 * Hq) {
                    const int bk = j >> 3;
                    sgm = 2 * ((bk >> 1) * 8 + (j & 7)) + (bk & 1);
                }
                float x[8];
                unpack8(*reinterpret_cast<const uint4*>(st + (size_t)sgm * kD * 2 + 16 * lane), kBf, x);
                if (sgm < 2 * Hq) {
                    const int h = sgm >> 1;
                    if (!(sgm & 1)) {  // q head h
                        prep_qk_lane<kHalf>(p, x, qn, c, sg, rot, partner);
                        *reinterpret_cast<uint4*>(qrow + h * q_hstride) = half8(x);
                    } else if (grow) {  // sigmoid(gate) (mul_sigmoid_inplace, cpu_ops.cpp:15-22), fp16
                        float g[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) g[e] = rcp_approx(1.0f + ex2_approx(-1.4426950408889634f * x[e]));
                        *reinterpret_cast<uint4*>(grow + h * kD) = half8(g);
                    }
                } else if (sgm < 2 * Hq + Hkv) {  // k head
                    const int kh = sgm - 2 * Hq;
                    prep_qk_lane<kHalf>(p, x, kn, c, sg, rot, partner);
                    const uint4 hv = half8(x);
                    *reinterpret_cast<uint4*>(krow + kh * k_hstride) = hv;
                    if (pool >= 0) *reinterpret_cast<uint4*>(p.k_pool + pool + kh * kD) = hv;  // ring append
                } else {  // v head
                    const int vh = sgm - 2 * Hq - Hkv;
                    const uint4 hv = half8(x);
                    *reinterpret_cast<uint4*>(vrow + vh * k_hstride) = hv;
                    if (pool >= 0) *reinterpret_cast<uint4*>(p.v_pool + pool + vh * kD) = hv;
                }
            }
            if (t == 0 && warp == 0 && lane == 0) ring_finish(p, rs, seq);
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
        t += G;
        while (t >= n_pad) {
            t -= n_pad;
            b++;
        }
        if (++s == kPrepStages) {
            s = 0;
            ph ^= 1u;
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmG,
                      const __grid_constant__ OutMaps om, const FaPrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + kQBytes;
    uint8_t* sV = sK + kKBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(sV + kVBytes + 256);  // [6][128]: row max (2 tiles x 2 halves), row sum

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_qt = p.n_pad / kBM;
    // CTAs are dispatched in blockIdx order (x fastest): within a sequence, every head's longest
    // causal tile goes out before any shorter one (longest-processing-time-first packing onto the SMs)
    const int qt = n_qt - 1 - (int)blockIdx.y;
    const int h = blockIdx.x, b = blockIdx.z;
    const int G = p.Hq / p.Hkv;
    const int kvh = h / G;
    const int q0 = qt * kBM;
    const int P = p.P;

    if (tid == 0) {
        *abort = 0;
        for (int i = 0; i < N_BARS; i++) tc::mbar_init(&bars[i], (i == P_FULL || i == P_FULL + 1) ? 2 * kBM : 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // launched as a programmatic dependent of the prep: Q, K, V and sigmoid(gate) are read only
    // after the prep grid has completed and its writes are visible (a no-op for a plain launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Keys of query row q (new token q) among the [old | new] key rows: [lo(q), P + q] with
    // lo(q) = max(P - Pb, P + q + 1 - capacity) -- the old tokens still in the ring and, once
    // more than `capacity` tokens precede it, only the last `capacity` (qwen3_5.cpp:974-983).
    const RingSnap rs = ring_snap(p, b);
    const int lo_base = P - rs.Pb, lo_win = P + 1 - rs.cap;
    const int lo_max = max(lo_base, lo_win + q0 + kBM - 1);  // largest lower bound of the tile's rows
    const int kt0 = max(lo_base, lo_win + q0) / kBN;         // first key tile (row q0 has the smallest bound)
    const int nT = (P + min(q0 + kBM, p.n) + kBN - 1) / kBN - kt0;

    if (warp == kWarpK || warp == kWarpV) {
        // ---------------- TMA producers: one warp streams Q then K (then the gate tile), one streams V ----------------
        // (each runs converged, polls its barriers with every lane and elects one lane per copy)
        if (nT > 0) {
            const int krow0 = (b * p.Hkv + kvh) * p.n_tot + kt0 * kBN;
            if (warp == kWarpK) {
                const int qrow0 = (b * p.Hq + h) * p.n_pad + q0;
                if (tc::elect_one()) {
                    tc::prefetch_tmap(&tmQ);
                    tc::prefetch_tmap(&tmK);
                    tc::mbar_arrive_expect_tx(&bars[Q_FULL], kQBytes);
                    for (int kb = 0; kb < 4; kb++) tc::tma_load_2d(sQ + kb * (kBM * 128), &tmQ, &bars[Q_FULL], kb * 64, qrow0);
                }
                for (int j = 0; j < nT; j++) {
                    if (j >= 1) tc::mbar_wait(&bars[K_EMPTY], (j - 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                    if (tc::elect_one()) {
                        tc::mbar_arrive_expect_tx(&bars[K_FULL], kKBytes);
                        for (int kb = 0; kb < 4; kb++)
                            tc::tma_load_2d(sK + kb * (kBN * 128), &tmK, &bars[K_FULL], kb * 64, krow0 + j * kBN);
                    }
                }
                if (p.tma_epilogue && p.gate) {
                    // sigmoid(gate) of this tile's 128 rows into the K buffer once the last Q K^T has
                    // read it (rows past the sequence end are zero-filled), hidden behind the last tiles
                    tc::mbar_wait(&bars[K_EMPTY], (nT - 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                    if (tc::elect_one()) {
                        tc::prefetch_tmap(&tmG);
                        tc::mbar_arrive_expect_tx(&bars[G_FULL], kBM * kD * 2);
                        for (int kb = 0; kb < 4; kb++)
                            tc::tma_load_3d(sK + kb * (kBM * 128), &tmG, &bars[G_FULL], h * kD + kb * 64, q0, b);
                    }
                }
            } else {
                if (tc::elect_one()) tc::prefetch_tmap(&tmV);
                for (int j = 0; j < nT; j++) {
                    if (j >= 1) tc::mbar_wait(&bars[V_EMPTY], (j - 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                    if (tc::elect_one()) {
                        tc::mbar_arrive_expect_tx(&bars[V_FULL], kVBytes);
                        for (int kb = 0; kb < 4; kb++)
                            tc::tma_load_2d(sV + kb * (kBN * 128), &tmV, &bars[V_FULL], kb * 64, krow0 + j * kBN);
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == kWarpMma) {
        // ---------------- MMA issuer (converged warp, one elected lane per tcgen05 instruction) ----------------
        if (nT > 0) {
            constexpr uint32_t id_qk = tc::idesc_f16_f32(kBM, kBN);
            constexpr uint32_t id_pv = tc::idesc_f16_f32_bmn(kBM, kD);  // V[key][d]: d contiguous
            // descriptors of the tiles' first bytes; a k-step adds its byte offset >> 4 to the start
            // address field (shared-memory addresses stay below 2^18, so it never carries out)
            const uint64_t dQ = tc::desc_kmajor_sw128((uint32_t)__cvta_generic_to_shared(sQ));
            const uint64_t dK = tc::desc_kmajor_sw128((uint32_t)__cvta_generic_to_shared(sK));
            const uint64_t dV = tc::desc_sw128((uint32_t)__cvta_generic_to_shared(sV), kBN * 128, 1024);
            tc::mbar_wait(&bars[Q_FULL], 0, p.err, ANELM_ERR_TIMEOUT, abort);
            auto qk = [&](int j) {
                const int s = j & 1, u = j >> 1;
                tc::mbar_wait(&bars[K_FULL], j & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                // TMEM buffer s is free once P V of tile j-2 (which read P from it) completed
                if (j >= 2) tc::mbar_wait(&bars[PV_DONE + s], (u - 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                tc::tc_fence_after();
#pragma unroll
                for (int kb = 0; kb < 4; kb++)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        if (tc::elect_one())
                            tc::mma_f16_ss(tmem + s * kBN, dQ + ((kb * (kBM * 128) + ks * 32) >> 4),
                                           dK + ((kb * (kBN * 128) + ks * 32) >> 4), id_qk, (kb | ks) != 0);
                if (tc::elect_one()) {
                    tc::mma_commit(&bars[S_FULL + s]);
                    tc::mma_commit(&bars[K_EMPTY]);
                }
            };
            auto pv = [&](int j) {
                const int s = j & 1, u = j >> 1;
                tc::mbar_wait(&bars[P_FULL + s], u & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                tc::mbar_wait(&bars[V_FULL], j & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                tc::tc_fence_after();
                // A = P from TMEM (16 keys = 8 columns per step); B = V, MN-major: 16 key rows of the
                // four 64-d boxes (boxes kBN * 128 bytes apart, 8-row groups 1024 bytes apart)
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ks++)
                    if (tc::elect_one())
                        tc::mma_f16_ts(tmem + kOCol, tmem + s * kBN + ks * 8, dV + ((ks * 16 * 128) >> 4), id_pv,
                                       (j > 0) || (ks > 0));
                if (tc::elect_one()) {
                    tc::mma_commit(&bars[PV_DONE + s]);
                    tc::mma_commit(&bars[V_EMPTY]);
                }
            };
            qk(0);
            for (int j = 0; j < nT; j++) {
                if (j + 1 < nT) qk(j + 1);
                pv(j);
            }
        }
        __syncwarp();
    } else {
        // ---------------- softmax: thread (r, hf) owns keys [64 hf, 64 hf + 64) of query row q0 + r ----------------
        const int r = tid & (kBM - 1), hf = tid >> 7;  // TMEM lane; key half of each S tile
        const int qpos = q0 + r;
        const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t pair_bar = 1 + (warp & 3);  // warps w and w + 4 share TMEM lanes [32w, 32w + 32)
        const float sl2 = 1.4426950408889634f / sqrtf((float)kD);  // log2(e) / sqrt(d)
        float m_used = -INFINITY, l = 0.f;
        float x[64];
        for (int j = 0; j < nT; j++) {
            const int s = j & 1, u = j >> 1;
            tc::mbar_wait(&bars[S_FULL + s], u & 1, p.err, ANELM_ERR_TIMEOUT, abort);
            tc::tc_fence_after();
            const int k0 = (kt0 + j) * kBN + hf * 64;  // key row of x[0]
            tc::tmem_ld64(trow + s * kBN + hf * 64, x);
            tc::tmem_ld_wait();
            if ((k0 + 63 > P + q0) || (k0 + 64 > P + p.n) || (k0 < lo_max)) {
                // diagonal, ragged end or window edge: masked scores become -inf (exp2 -> 0)
                const int lo_r = max(lo_base, lo_win + qpos);
#pragma unroll
                for (int c = 0; c < 64; c++)
                    if (k0 + c > P + qpos || k0 + c >= P + p.n || k0 + c < lo_r) x[c] = -INFINITY;
            }
            float m4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
            for (int c = 4; c < 64; c++) m4[c & 3] = fmaxf(m4[c & 3], x[c]);
            float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            // row max over both halves; the exchange slots alternate by tile so a slot is only
            // rewritten after the partner has passed the next pair barrier (and so read it)
            red[((j & 1) * 2 + hf) * kBM + r] = mx;
            tc::named_bar_sync(pair_bar, 64);
            mx = fmaxf(mx, red[((j & 1) * 2 + (hf ^ 1)) * kBM + r]);
            const float m_new = fmaxf(m_used, mx);
            // lazy rescaling: keep the old max unless it grew by more than 2^8 in probability units
            // (both halves see the same maxima, so they take the same branch)
            const bool grow = (m_used == -INFINITY) || ((m_new - m_used) * sl2 > 8.0f);
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                // O is stable once P V of the previous tile completed; this half rescales O columns
                // [128 hf, 128 hf + 128).  A row with no visible key yet (max still -inf) has O = 0.
                tc::mbar_wait(&bars[PV_DONE + ((j - 1) & 1)], ((j - 1) >> 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
                tc::tc_fence_after();
                const float alpha = (grow && m_new != -INFINITY) ? exp2f((m_used - m_new) * sl2) : 1.0f;
#pragma unroll 1
                for (int ch = 0; ch < 4; ch++) {  // 32 columns at a time: the S row stays in registers
                    uint32_t o[32];
                    tc::tmem_ld32(trow + kOCol + hf * 128 + ch * 32, o);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tc::tmem_st32(trow + kOCol + hf * 128 + ch * 32, o);
                }
                tc::tmem_st_wait();
                l *= alpha;
            }
            if (grow) m_used = m_new;
            const float nm = m_used == -INFINITY ? 0.f : -m_used * sl2;  // all -inf: exp2 gives P = 0
            // P = exp2((s - m) * log2(e)/sqrt(d)) as fp16 pairs: half hf fills columns [32 hf, 32 hf + 32) of
            // the S buffer (both halves read their S columns before the pair barrier above)
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t w[32];
#pragma unroll
            for (int e = 0; e < 32; e++) {
                const float a = ex2_approx(fmaf(x[2 * e], sl2, nm));
                const float b2 = ex2_approx(fmaf(x[2 * e + 1], sl2, nm));
                s4[e & 3] += a + b2;
                const __half2 hp = __floats2half2_rn(a, b2);
                w[e] = *reinterpret_cast<const uint32_t*>(&hp);
            }
            tc::tmem_st32(trow + s * kBN + hf * 32, w);
            l += (s4[0] + s4[1]) + (s4[2] + s4[3]);
            tc::tmem_st_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bars[P_FULL + s]);
        }
        // row sum over both halves (own slots: the max exchange slots may still be read)
        red[4 * kBM + hf * kBM + r] = l;
        tc::named_bar_sync(pair_bar, 64);
        l += red[4 * kBM + (hf ^ 1) * kBM + r];
        if (p.tma_epilogue) {
            // ---------------- epilogue: O / l * sigmoid(gate) -> swizzled tiles -> TMA store ----------------
            // Thread (r, hf) reads O row r, columns [128 hf, 128 hf + 128), from TMEM and the matching gate
            // values from the K buffer (128B-swizzled boxes of 64 columns, the TMA layout) and writes the
            // 16-bit output into the Q buffer in the same layout; one thread then stores the four boxes
            // (rows past the sequence end are clipped).
            tc::mbar_wait(&bars[PV_DONE + ((nT - 1) & 1)], ((nT - 1) >> 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
            tc::tc_fence_after();
            if (p.gate) tc::mbar_wait(&bars[G_FULL], 0, p.err, ANELM_ERR_TIMEOUT, abort);
            const float inv = (l > 0.f) ? 1.0f / l : 0.f;
            const bool out_bf = p.out_dtype == ANELM_BF16;
#pragma unroll 1
            for (int ch = 2 * hf; ch < 2 * hf + 2; ch++) {
                float o[64];
                tc::tmem_ld64(trow + kOCol + ch * 64, o);
                tc::tmem_ld_wait();
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int off = ch * (kBM * 128) + r * 128 + ((u ^ (r & 7)) << 4);
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = o[u * 8 + e] * inv;
                    if (p.gate) {  // sigmoid(gate) was computed by the prep kernel
                        float g[8];
                        unpack8(*reinterpret_cast<const uint4*>(sK + off), false, g);
#pragma unroll
                        for (int e = 0; e < 8; e++) v[e] *= g[e];
                    }
                    *reinterpret_cast<uint4*>(sQ + off) = pack8(v, out_bf);
                }
            }
            tc::fence_proxy_async_smem();
            tc::named_bar_sync(5, 2 * kBM);
            if (tid == 0) {
                for (int r = 0; r < om.n; r++) {
                    tc::prefetch_tmap(&om.m[r]);
                    for (int ch = 0; ch < 4; ch++)
                        tc::tma_store_3d(&om.m[r], sQ + ch * (kBM * 128), om.col0 + h * kD + ch * 64, q0, b);
                }
                tc::bulk_commit_group();
                if (om.wait_full) tc::bulk_wait_group0();
                else tc::bulk_wait_group_read0();
            }
        } else if (nT > 0) {
            // ---------------- epilogue part 1: O / l into shared memory ----------------
            // (Q / K / V buffers are idle once the last P V completed)
            tc::mbar_wait(&bars[PV_DONE + ((nT - 1) & 1)], ((nT - 1) >> 1) & 1, p.err, ANELM_ERR_TIMEOUT, abort);
            tc::tc_fence_after();
            const float inv = (l > 0.f) ? 1.0f / l : 0.f;
            float* orow = reinterpret_cast<float*>(sQ) + r * kORow;
#pragma unroll 1
            for (int ch = 2 * hf; ch < 2 * hf + 2; ch++) {
                float o[64];
                tc::tmem_ld64(trow + kOCol + ch * 64, o);
                tc::tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 64; c += 4)
                    *reinterpret_cast<float4*>(orow + ch * 64 + c) =
                        make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
            }
        }
    }
    // ---------------- epilogue part 2: gate and store, one warp per row ----------------
    if (!p.tma_epilogue) __syncthreads();
    if (!p.tma_epilogue && warp < kSoftmaxWarps && nT > 0) {
        // four rows per pass: all gate loads of the pass are issued before any store
        for (int r0 = warp * 4; r0 < kBM; r0 += 4 * kSoftmaxWarps) {
            float z[4][kD / 32];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int qpos = min(q0 + r0 + i, p.n - 1);
                const char* prow = reinterpret_cast<const char*>(p.proj) +
                                   ((long long)b * p.n + qpos) * p.proj_stride * dtype_bytes(p.proj_dtype);
#pragma unroll
                for (int e = 0; e < kD / 32; e++)
                    z[i][e] = p.gate ? load_as_float(prow, p.proj_dtype, (long long)h * 2 * kD + kD + e * 32 + lane)
                                     : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int rr = r0 + i;
                const int qpos = q0 + rr;
                if (qpos >= p.n) break;
                const float* orow = reinterpret_cast<const float*>(sQ) + rr * kORow;
                const long long obase = ((long long)b * p.n + qpos) * p.out_stride + (long long)h * kD;
#pragma unroll
                for (int e = 0; e < kD / 32; e++) {
                    const int c = e * 32 + lane;
                    float v = orow[c];
                    if (p.gate) v = v / (1.0f + expf(-z[i][e]));  // mul_sigmoid_inplace, cpu_ops.cpp:15-22
                    store_from_float(p.out, p.out_dtype, obase + c, v);
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tc::tmap_encode_fn(); }

// 2D fp16 tensor map, inner dimension `cols` (contiguous), 128B swizzle, box {64, box_rows}.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3D map over a [B][n][row_stride] tensor of a 16-bit type, inner extent `cols`, box {64, 128, 1}, 128B
// swizzle: rows past n fall outside the map (loads zero-fill them, stores skip them).
bool make_map_rows(CUtensorMap* m, int dtype, const void* base, uint64_t cols, uint64_t n, uint64_t B,
                   uint64_t row_stride) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {cols, n, B};
    cuuint64_t strides[2] = {row_stride * 2, n * row_stride * 2};
    cuuint32_t box[3] = {64, kBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, dtype == ANELM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

// Launches `kern` as a programmatic dependent of the previous kernel on the stream (its prologue may
// overlap that kernel; it reads that kernel's results only after griddepcontrol.wait).  Returns
// nonzero (error cleared) if the launch was refused, so the caller can launch it plainly.
template <class... KArgs, class... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess) return 0;
    cudaGetLastError();
    return 1;
}

size_t fa_prefill_workspace_bytes(int B, int n, int P, int Hq, int Hkv, int head_dim) {
    const long long n_pad = (n + kBM - 1) / kBM * kBM;
    // fp16 Q [B][Hq][n_pad][D], K and V [B][Hkv][P + n_pad][D], sigmoid(gate) [B][n][Hq][D]; the
    // ring snapshots [B][4] ints
    return (size_t)B * head_dim * 2 * (2 * (size_t)Hq * n_pad + 2 * (size_t)Hkv * (P + n_pad)) + (size_t)B * 16;
}

int launch_fa_prefill(FaPrefillParams p, void* workspace, int head_dim, cudaStream_t stream, const PrefillDests* dests) {
    if (head_dim != kD || p.P < 0 || p.P % kBN || !p.kv_len || !p.kv_start || !p.kv_cap || !p.kv_base ||
        !p.k_pool || !p.v_pool)
        return ANELM_ERR_UNSUPPORTED;
    p.n_pad = (p.n + kBM - 1) / kBM * kBM;
    p.n_tot = p.P + p.n_pad;
    const long long nq = (long long)p.B * p.Hq * p.n_pad * kD, nk = (long long)p.B * p.Hkv * p.n_tot * kD;
    __half* ws = static_cast<__half*>(workspace);
    p.Qh = ws;
    p.Kh = ws + nq;
    p.Vh = p.Kh + nk;
    p.SG = nullptr;
    p.meta = reinterpret_cast<int*>(p.Vh + nk + nq);  // after sigmoid(gate) (<= nq halves), 16-byte aligned
    CUtensorMap mQ, mK, mV;
    if (!make_map(&mQ, p.Qh, (uint64_t)p.B * p.Hq * p.n_pad, kD, kBM) ||
        !make_map(&mK, p.Kh, (uint64_t)p.B * p.Hkv * p.n_tot, kD, kBN) ||
        !make_map(&mV, p.Vh, (uint64_t)p.B * p.Hkv * p.n_tot, kD, kBN))
        return ANELM_ERR_CUDA;
    // ring snapshots and the old tokens still visible, before the prep appends to the rings
    fa_prefill_gather_kernel<<<dim3(std::max(1, (p.P + 63) / 64), p.B), 256, 0, stream>>>(p);
    // TMA epilogue: 16-bit output with a 16-byte aligned base and row stride; sigmoid(gate) as fp16
    // [B][n][Hq * D] after V in the workspace
    CUtensorMap mG = mQ;
    OutMaps om{};
    __half* sg = p.Vh + nk;
    const bool out16 = p.out_dtype == ANELM_BF16 || p.out_dtype == ANELM_F16;
    if (dests && dests->n > 0) {
        // every destination by TMA tile stores (the only epilogue that writes them all)
        if (!out16 || dests->n > kMaxOuts || p.out_stride % 8 || dests->col0 < 0 || dests->col0 % 64 ||
            dests->col0 + (long long)p.Hq * kD > p.out_stride)
            return ANELM_ERR_UNSUPPORTED;
        for (int r = 0; r < dests->n; r++)
            if ((uintptr_t)dests->ptrs[r] % 16 ||
                !make_map_rows(&om.m[r], p.out_dtype, dests->ptrs[r], (uint64_t)p.out_stride, p.n, p.B, p.out_stride))
                return ANELM_ERR_UNSUPPORTED;
        om.n = dests->n;
        om.col0 = dests->col0;
        om.wait_full = 1;
        p.tma_epilogue = !p.gate || make_map_rows(&mG, ANELM_F16, sg, (uint64_t)p.Hq * kD, p.n, p.B,
                                                  (uint64_t)p.Hq * kD);
        if (!p.tma_epilogue) return ANELM_ERR_UNSUPPORTED;
    } else {
        om.n = 1;
        p.tma_epilogue = out16 && ((uintptr_t)p.out % 16 == 0) && (p.out_stride % 8 == 0) &&
                         make_map_rows(&om.m[0], p.out_dtype, p.out, (uint64_t)p.Hq * kD, p.n, p.B, p.out_stride) &&
                         (!p.gate || make_map_rows(&mG, ANELM_F16, sg, (uint64_t)p.Hq * kD, p.n, p.B,
                                                   (uint64_t)p.Hq * kD));
    }
    if (p.tma_epilogue && p.gate) p.SG = sg;
    const long long row_bytes = p.proj_stride * dtype_bytes(p.proj_dtype);
    const bool vec = (uintptr_t)p.proj % 16 == 0 && row_bytes % 16 == 0 && p.rot_dim % 16 == 0;
    // streaming prep: 16-bit projection, 16-byte aligned RoPE table rows, two CTAs per SM
    const int nseg = 2 * p.Hq + 2 * p.Hkv;
    const int rope_off = nseg * kD * 2;
    const int stage_bytes = (rope_off + 8 * (p.rot_dim >> 1) + 127) / 128 * 128;
    const bool bulk = vec && dtype_bytes(p.proj_dtype) == 2 && stage_bytes <= kPrepStageMax &&
                      (long long)p.B * p.n_pad + 4LL * kPrepCtas * 1024 < (1LL << 31) &&
                      (!p.rope_cos || ((uintptr_t)p.rope_cos % 16 == 0 && (uintptr_t)p.rope_sin % 16 == 0));
    if (bulk) {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const long long total = (long long)p.B * p.n_pad;
        const int grid = (int)std::min<long long>(total, (long long)kPrepCtas * sms);
        const int smem = 128 + kPrepStages * stage_bytes;
        const bool half = p.rope_mode != ANELM_ROPE_INTERLEAVED, bf = p.proj_dtype == ANELM_BF16;
        auto kern = half ? (bf ? fa_prefill_prep_bulk_kernel<true, true> : fa_prefill_prep_bulk_kernel<true, false>)
                         : (bf ? fa_prefill_prep_bulk_kernel<false, true> : fa_prefill_prep_bulk_kernel<false, false>);
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (launch_pdl(kern, dim3(grid), dim3(32 * (kPrepWarps + 1)), smem, stream, p, stage_bytes, rope_off))
            kern<<<grid, 32 * (kPrepWarps + 1), smem, stream>>>(p, stage_bytes, rope_off);
    } else if (vec) {
        if (launch_pdl(fa_prefill_prep_vec_kernel, dim3(p.n_pad, p.B), dim3(256), 0, stream, p))
            fa_prefill_prep_vec_kernel<<<dim3(p.n_pad, p.B), 256, 0, stream>>>(p);
    } else {
        const size_t prep_smem = (size_t)(p.Hq + 2 * p.Hkv) * kD * sizeof(float);
        if (prep_smem > 48 * 1024)
            cudaFuncSetAttribute(fa_prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem);
        if (launch_pdl(fa_prefill_prep_kernel, dim3(p.n_pad, p.B), dim3(256), prep_smem, stream, p))
            fa_prefill_prep_kernel<<<dim3(p.n_pad, p.B), 256, prep_smem, stream>>>(p);
    }
    cudaFuncSetAttribute(fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    // programmatic dependent launch: the prologue (barriers, TMEM allocation) overlaps the prep's
    // tail; the kernel reads the prep's outputs only after griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.Hq, p.n_pad / kBM, p.B);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, fa_prefill_kernel, mQ, mK, mV, mG, om, p) != cudaSuccess) {
        cudaGetLastError();  // clear, then the plain launch
        fa_prefill_kernel<<<cfg.gridDim, kThreads, kSmemBytes, stream>>>(mQ, mK, mV, mG, om, p);
    }
    return cudaGetLastError() == cudaSuccess ? ANELM_OK : ANELM_ERR_CUDA;
}

}  // namespace anelm
