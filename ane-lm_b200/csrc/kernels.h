// Kernel parameter blocks and launchers shared between the host ABI (anelm_abi.cu)
// and the kernel translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace anelm {

// Split-K flash-decoding over slot-major fp16 KV rings [slots][Hkv][D].
// One CTA per (batch row b, ring split, kv head).
struct FaDecodeParams {
    int Hq, Hkv, rot_dim;
    float rope_theta, rms_eps, scale;
    int gate, qk_norm, rope_mode, kv_mode, append;
    const float* q_norm;
    const float* k_norm;
    const float* rope_cos;
    const float* rope_sin;
    int rope_len;
    // KV pool of this layer
    __half* k_pool;
    __half* v_pool;
    const long long* kv_base;  // [seq] first slot of the sequence's ring in the pool
    const int* kv_cap;         // [seq]
    int* kv_len;               // [seq] (this layer); nullptr => scalar metadata below
    int* kv_start;             // [seq]
    int cap_s, len_s, start_s;
    // batch
    const int* seq_ids;        // [n] or nullptr (=> seq 0)
    const int* pos_arr;        // [n] device positions or nullptr
    int pos_scalar;
    const void* proj;          // [n][proj_stride] elements of proj_dtype
    int proj_dtype;
    long long proj_stride;
    int q_head_stride;         // elements between q heads inside a proj row (2*D in the glue)
    long long k_off, v_off;    // element offsets of the new k / v inside a proj row
    long long gate_off;        // element offset of head 0's gate inside a proj row (q_head_stride apart)
    int proj_vec;              // proj rows and the q / k / v offsets are 16-byte aligned (vector loads)
    int cluster_ns;            // >= 2: one row whose ns splits form a thread-block cluster and merge
                               // through distributed shared memory (0: partials through global memory)
    void* out;
    int out_dtype;
    long long out_stride;
    // split plan
    const int* blk_b;
    const int* blk_split;
    const int* nsplit;         // [n]
    const long long* part_off; // [n] first split index of row b in the partial arrays
    int CH;                    // tokens per split (multiple of 64)
    float* part_o;             // [total_splits][Hkv][4][D]
    float* part_ml;            // [total_splits][Hkv][4][2]
    int* cnt_head;             // [n][Hkv] zero between launches
    int* cnt_seq;              // [n]      zero between launches
    int* err;                  // device error word (first error code wins), may be nullptr
};

// Gated DeltaNet decode step; one cluster per (batch row, key head): the value heads
// sharing that key head times column blocks of their fp32 state.
struct GdnDecodeParams {
    int Hk, Hv, C;
    float l2_eps;
    int delta_mode;
    const float* conv_w;   // [C][4]
    const float* A;        // [Hv] = exp(A_log)
    const float* dt_bias;  // [Hv]
    const float* norm_w;   // [dv]
    float* ssm;            // [seqs][Hv][128][128]
    long long ssm_rows;    // seqs * Hv * 128: rows of ssm seen as a [rows][128] fp32 matrix (the TMA view)
    float* conv;           // [seqs][C][3] ring of the last 3 inputs (reference layout)
    int* conv_pos;         // [seqs][Hk] ring position, one copy per key-head cluster
    const int* seq_ids;    // [n] or nullptr
    int seq_scalar;
    const void* proj;
    int proj_dtype;
    long long proj_stride;
    void* out;
    int out_dtype;
    long long out_stride;
    int* err;              // device error word (first error code wins), may be nullptr
};

// Causal prefill of a fresh ring: B sequences of n tokens each.
struct FaPrefillParams {
    // n new tokens per sequence (n_pad: rounded up to the 128-row tile).  The attention keys of
    // sequence b are [old | new]: the last P_b <= P tokens its ring held before the call (the ones
    // the first new token still sees: P_b = min(len, capacity - 1)), right-aligned in rows
    // [P - P_b, P), then the n new tokens in rows [P, P + n); P is a multiple of 128 and
    // n_tot = P + n_pad rows per (sequence, kv head).
    int B, n, n_pad, Hq, Hkv, rot_dim, P, n_tot;
    float rope_theta, rms_eps;
    int qk_norm, rope_mode, gate, start_pos;
    const float* q_norm;
    const float* k_norm;
    const float* rope_cos;
    const float* rope_sin;
    int rope_len;
    const void* proj;      // [B][n][proj_stride] elements of proj_dtype
    int proj_dtype;
    long long proj_stride;
    __half* Qh;            // [B][Hq][n_pad][D]   (workspace)
    __half* Kh;            // [B][Hkv][n_pad][D]
    __half* Vh;            // [B][Hkv][n_pad][D]
    __half* SG;            // [B][n][Hq * D] sigmoid(gate), written by the prep kernel for the TMA epilogue
    __half* k_pool;        // ring pools of the layer (nullptr: no append)
    __half* v_pool;
    const long long* kv_base;
    const int* seq_ids;    // [B]
    int* kv_len;
    int* kv_start;
    const int* kv_cap;     // [max_seqs] ring capacity per sequence
    int* meta;             // [B][4] (workspace): len, start, capacity, P_b of each ring before the call
    void* out;             // [B][n][out_stride]
    int out_dtype;
    long long out_stride;
    int* err;
    int tma_epilogue;      // set by launch_fa_prefill: gate tile loaded and output stored by TMA
};

// Chunkwise Gated DeltaNet prefill (layer path: from projections) and the bare chunked
// delta rule (core op: from q, k, v, log g, beta).
struct GdnPrefillParams {
    int B, n, T_pad, Hk, Hv, dk, dv, C, delta_mode;
    float l2_eps;
    // layer path
    const float* conv_w;
    const float* A;
    const float* dt_bias;
    const float* norm_w;
    float* conv;           // [max_seqs][C][3]
    int* conv_pos;         // [max_seqs][Hk]
    const void* proj;      // [B][n][proj_stride]
    int proj_dtype;
    long long proj_stride;
    void* out;             // [B][n][out_stride]
    int out_dtype;
    long long out_stride;
    // core op inputs (token-major)
    const void* q_in;
    const void* k_in;
    const void* v_in;
    int in_dtype;
    int in_vec;            // set by the launcher: q_in, k_in, v_in 16-byte aligned
    int qkv_exact;        // q, k, v arrive as 16-bit values: exact in fp16, their lo planes are zero and
                          // are neither written nor read; products against them take two of the three terms
    int direct;           // set by the launcher: 16-bit q, k, v (and log g, beta) read in place by the chunk
                          // and chain kernels (no pack), every product with them in their own type
    int op_bf16;          // with direct: the inputs (and so the hi / lo operands meeting them) are bf16
    const float* lg_in;
    const float* beta_in;
    // state [seq][Hv][dk][dv], row b uses seq_ids[b] (or b)
    float* state;
    const int* seq_ids;
    // y = S^T q per token: [B][n][y_stride]
    void* y;
    int y_dtype;
    long long y_stride;
    int y_vec;             // set by the launcher: y and y_stride allow 16-byte stores of 8 outputs
    // workspace (carved by the launcher); tensor-core operands as an fp16 hi plane followed by a
    // lo plane (x = hi + lo)
    __half* qh;            // [B][Hk][T_pad][dk], lo plane at + q_plane
    __half* kh;
    __half* vh;            // [B][Hv][T_pad][dv], lo plane at + v_plane
    long long q_plane, v_plane, m_plane;
    float* lg;             // [B][Hv][T_pad]
    float* beta;
    __half* wh;            // [B][Hv][T_pad][dk], lo plane at + v_plane
    float* Ub;             // [B][Hv][T_pad][dv]
    __half* mh;            // [B][Hv][T_pad][64], lo plane at + m_plane
    float* lcb;            // [B][Hv][T_pad]
    float* ring_snap;      // [B][C][3]
    int* pos_snap;         // [B][Hk]
    int* err;
};
size_t gdn_prefill_workspace_bytes(int B, int n, int Hk, int Hv, int C, bool layer);
int launch_gdn_prefill(GdnPrefillParams p, void* workspace, cudaStream_t stream);
int launch_gated_delta_chunked(GdnPrefillParams p, void* workspace, cudaStream_t stream);

size_t fa_prefill_workspace_bytes(int B, int n, int P, int Hq, int Hkv, int head_dim);
// Extra destinations of a prefill's output: n device addresses (this device's memory or a peer's
// mapped into this process) of [B][n_tokens][out_stride] 16-bit buffers; the launch's heads fill
// columns [col0, col0 + Hq D) of each, by TMA tile stores that complete before the CTA exits.
struct PrefillDests {
    const void* const* ptrs;
    int n, col0;
};
int launch_fa_prefill(FaPrefillParams p, void* workspace, int head_dim, cudaStream_t stream,
                      const PrefillDests* dests = nullptr);

int launch_fa_decode(const FaDecodeParams& p, int head_dim, int n_blocks, cudaStream_t stream);
size_t fa_decode_smem_bytes(int head_dim);
// Largest split count one row may use: the merge keeps [splits][4] weights in the tile buffers.
int fa_decode_max_splits(int head_dim);
// Sets the message anelm_last_error() returns on the calling thread.
void set_last_error(const char* msg);

int launch_gdn_decode(const GdnDecodeParams& p, int n_rows, int key_dim, int val_dim, cudaStream_t stream);

// bf16 GEMM C[M][N] = A[M][K] B[N][K]^T (nn.Linear layout), fp32 accumulation, C of c_dtype.
// A, B 16-byte aligned with row strides lda, ldb (elements) multiples of 8.
int launch_gemm_bf16_tn(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int c_dtype,
                        int M, int N, int K, int* err, cudaStream_t stream);
// LM head with in-model top-k (k <= 32): top_vals / top_idx [n][k] of h [n][hidden] W [vocab][hidden]^T,
// sorted descending; workspace of lm_head_topk_workspace_bytes(n, vocab) bytes (16-byte aligned).
size_t lm_head_topk_workspace_bytes(int n, int vocab);
int launch_lm_head_topk(const void* h, long long ldh, const void* W, long long ldw, int n, int vocab, int hidden, int k,
                        float* top_vals, int* top_idx, void* workspace, size_t workspace_bytes, int* err,
                        cudaStream_t stream);

}  // namespace anelm
