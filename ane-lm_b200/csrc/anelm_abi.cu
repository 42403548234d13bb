// Host side of the anelm_b200 C ABI (include/anelm_b200.h).
//
// Owns the device state that models/llm/qwen3_5.{h,cpp} keeps on the host
// (KVCache / DeltaNetState per layer, qwen3_5.h:158-171; allocation
// qwen3_5.cpp:280-347; reset 159-182), validates every call's arguments before
// anything is launched, and turns the reference's per-token glue calls
// (qwen3_5.cpp:849-1002) into launches of the fused kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "anelm_b200.h"
#include "kernels.h"
#include "ops.h"
#include "tc100.cuh"  // (also brings cuda.h: CUresult / CUdeviceptr for the IPC helpers)

using namespace anelm;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CUDA_TRY(x)                                                                              \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) return fail(ANELM_ERR_CUDA, "%s: %s", #x, cudaGetErrorString(e_)); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            ok = false;
            return;
        }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int launch_status(int rc, const char* what) {
    if (rc == ANELM_OK) return ANELM_OK;
    if (rc == ANELM_ERR_CUDA) {
        cudaError_t e = cudaGetLastError();
        return fail(ANELM_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    }
    return fail(rc, "%s: unsupported configuration", what);
}

}  // namespace

namespace anelm {
void set_last_error(const char* msg) { g_err = msg; }
}  // namespace anelm

struct anelm_plan {
    anelm_ctx* ctx = nullptr;
    int n = 0;
    std::vector<int> seq_h;
    int* seq_d = nullptr;
    int CH = 64;
    int n_blocks = 0;
    int ns0 = 0;  // splits of the single row of a one-row plan (0 otherwise)
    int* blk_b = nullptr;
    int* blk_split = nullptr;
    int* nsplit = nullptr;
    long long* part_off = nullptr;
    float* part_o = nullptr;
    float* part_ml = nullptr;
    int* cnt_head = nullptr;
    int* cnt_seq = nullptr;
    std::vector<void*> allocs;
};

struct anelm_ctx {
    anelm_config cfg{};
    std::vector<int> layer_types;
    int device = 0;
    std::vector<int> fa_idx, gdn_idx;
    int n_fa = 0, n_gdn = 0;
    int C = 0, fa_proj = 0, gdn_proj = 0;
    std::vector<int> cap_h;
    std::vector<long long> base_h;
    long long total_slots = 0;
    long long* kv_base = nullptr;
    int* kv_cap = nullptr;
    int* kv_len = nullptr;    // [n_fa][max_seqs]
    int* kv_start = nullptr;  // [n_fa][max_seqs]
    std::vector<__half*> k_pool, v_pool;
    std::vector<float*> q_norm, k_norm;
    std::vector<char> fa_w_set;
    std::vector<float*> ssm, conv;
    int* conv_pos = nullptr;  // [n_gdn][max_seqs][Hk]
    std::vector<float*> conv_w, A, dt_bias, norm_w;
    std::vector<char> gdn_w_set;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    int* err = nullptr;
    // [n_fa][max_seqs]: host record of each ring's len, kept by every call that changes it (reset,
    // import / set_meta, decode: one append per row, prefill: n appends, each capped at the
    // capacity).  Prefill sizes its old-token rows from it; the device's len / start stay the truth.
    std::vector<int> len_h;
    void* prefill_ws = nullptr;  // prefill staging (Q, K, V, V^T, sigmoid(gate)), grown on demand
    size_t prefill_ws_bytes = 0;
    void* gdn_prefill_ws = nullptr;  // DeltaNet prefill staging (chunk operands), grown on demand
    size_t gdn_prefill_ws_bytes = 0;
    std::vector<void*> w_in, w_out;  // per layer, bf16: [proj_dim][hidden], [hidden][core out] (or null)
    std::vector<int> hidden;         // per layer hidden size of the projections (0: not set)
    void* layer_ws = nullptr;        // layer-step staging (projection rows, core output), grown on demand
    size_t layer_ws_bytes = 0;
    __half* py_proj = nullptr;  // staging for anelm_py_cpu_attention
    __half* py_out = nullptr;
    std::vector<void*> allocs;
    std::mutex mu;
    std::map<int, anelm_plan*> single;  // per-sequence batch-1 plans
};

namespace {

template <class T>
int dev_alloc(std::vector<void*>& list, T** p, size_t count) {
    void* q = nullptr;
    const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
    cudaError_t e = cudaMalloc(&q, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ANELM_ERR_NOMEM, "cudaMalloc(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    }
    e = cudaMemset(q, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(q);
        return fail(ANELM_ERR_CUDA, "cudaMemset failed: %s", cudaGetErrorString(e));
    }
    list.push_back(q);
    *p = static_cast<T*>(q);
    return ANELM_OK;
}

#define ALLOC(list, ptr, count)                      \
    do {                                             \
        int rc_ = dev_alloc((list), &(ptr), (count)); \
        if (rc_) return rc_;                         \
    } while (0)

int check_dtype(int dt) {
    if (dt != ANELM_F32 && dt != ANELM_F16 && dt != ANELM_BF16) return fail(ANELM_ERR_INVALID_ARG, "bad dtype %d", dt);
    return ANELM_OK;
}

int check_layer(anelm_ctx* ctx, int layer, int type) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers)
        return fail(ANELM_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, ctx->cfg.num_layers);
    if (ctx->layer_types[layer] != type)
        return fail(ANELM_ERR_STATE, "layer %d is not a %s layer", layer,
                    type == ANELM_LAYER_FULL_ATTN ? "full-attention" : "linear-attention");
    return ANELM_OK;
}

int check_seq(anelm_ctx* ctx, int seq) {
    if (seq < 0 || seq >= ctx->cfg.max_seqs)
        return fail(ANELM_ERR_INVALID_ARG, "sequence %d out of range [0,%d)", seq, ctx->cfg.max_seqs);
    return ANELM_OK;
}

int choose_split_tokens(const anelm_ctx* ctx, const std::vector<int>& seqs) {
    if (const char* e = getenv("ANELM_SPLIT_TOKENS")) {
        int v = atoi(e);
        if (v >= 64) return (v / 64) * 64;
    }
    long long total = 0;
    for (int s : seqs) total += ctx->cap_h[s];
    total *= ctx->cfg.num_kv_heads;
    const long long target = 148LL * 2 * 8;  // about eight waves of two CTAs per SM
    long long ch = (total + target - 1) / target;
    ch = ((ch + 63) / 64) * 64;
    if (ch < 64) ch = 64;
    if (ch > 4096) ch = 4096;
    return (int)ch;
}

int build_plan(anelm_ctx* ctx, int n, const int* seqs, anelm_plan** out) {
    if (n <= 0 || !seqs) return fail(ANELM_ERR_INVALID_ARG, "plan needs n > 0 sequence ids");
    std::vector<char> seen(ctx->cfg.max_seqs, 0);
    for (int i = 0; i < n; i++) {
        if (int rc = check_seq(ctx, seqs[i])) return rc;
        if (seen[seqs[i]]) return fail(ANELM_ERR_INVALID_ARG, "sequence %d appears twice in a plan", seqs[i]);
        seen[seqs[i]] = 1;
    }
    auto* p = new anelm_plan();
    p->ctx = ctx;
    p->n = n;
    p->seq_h.assign(seqs, seqs + n);
    auto cleanup = [&](int rc) {
        for (void* a : p->allocs) cudaFree(a);
        delete p;
        return rc;
    };
    int rc;
#define PALLOC(ptr, count)                                   \
    do {                                                     \
        if ((rc = dev_alloc(p->allocs, &(ptr), (count)))) return cleanup(rc); \
    } while (0)
    PALLOC(p->seq_d, n);
    if (cudaMemcpy(p->seq_d, seqs, n * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
        return cleanup(fail(ANELM_ERR_CUDA, "plan upload failed"));
    if (ctx->n_fa > 0) {
        p->CH = choose_split_tokens(ctx, p->seq_h);
        if (n == 1) {  // one row: at most 16 splits, so they can merge inside one thread-block cluster
            const int cap = ctx->cap_h[seqs[0]];
            p->CH = std::max(p->CH, ((cap + 15) / 16 + 63) / 64 * 64);
        }
        std::vector<int> bb, bs, ns(n);
        std::vector<long long> off(n);
        long long tot = 0;
        for (int i = 0; i < n; i++) {
            const int cap = ctx->cap_h[seqs[i]];
            ns[i] = std::max(1, (cap + p->CH - 1) / p->CH);
            if (ns[i] > fa_decode_max_splits(ctx->cfg.head_dim))
                return cleanup(fail(ANELM_ERR_UNSUPPORTED, "too many splits (%d)", ns[i]));
            off[i] = tot;
            tot += ns[i];
            for (int s = 0; s < ns[i]; s++) {
                bb.push_back(i);
                bs.push_back(s);
            }
        }
        p->n_blocks = (int)bb.size();
        p->ns0 = n == 1 ? ns[0] : 0;
        const int Hkv = ctx->cfg.num_kv_heads, D = ctx->cfg.head_dim;
        PALLOC(p->blk_b, bb.size());
        PALLOC(p->blk_split, bs.size());
        PALLOC(p->nsplit, n);
        PALLOC(p->part_off, n);
        PALLOC(p->part_o, (size_t)tot * Hkv * 4 * D);
        PALLOC(p->part_ml, (size_t)tot * Hkv * 4 * 2);
        PALLOC(p->cnt_head, (size_t)n * Hkv);
        PALLOC(p->cnt_seq, n);
        if (cudaMemcpy(p->blk_b, bb.data(), bb.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(p->blk_split, bs.data(), bs.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(p->nsplit, ns.data(), n * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(p->part_off, off.data(), n * sizeof(long long), cudaMemcpyHostToDevice) != cudaSuccess)
            return cleanup(fail(ANELM_ERR_CUDA, "plan upload failed"));
    }
#undef PALLOC
    *out = p;
    return ANELM_OK;
}

void free_plan(anelm_plan* p) {
    if (!p) return;
    for (void* a : p->allocs) cudaFree(a);
    delete p;
}

FaDecodeParams fa_params(anelm_ctx* ctx, int layer, const anelm_plan* plan, const void* proj, int proj_dtype,
                         const int* pos_arr, int pos_scalar, void* out, int out_dtype) {
    const anelm_config& c = ctx->cfg;
    const int fi = ctx->fa_idx[layer];
    const int D = c.head_dim;
    FaDecodeParams p{};
    p.Hq = c.num_q_heads;
    p.Hkv = c.num_kv_heads;
    p.rot_dim = c.rot_dim;
    p.rope_theta = c.rope_theta;
    p.rms_eps = c.rms_eps;
    p.scale = 1.0f / sqrtf((float)D);
    p.gate = c.attn_output_gate;
    p.qk_norm = c.qk_norm_in_core;
    p.rope_mode = c.rope_mode;
    p.kv_mode = c.kv_mode;
    p.append = 1;
    p.q_norm = ctx->q_norm[fi];
    p.k_norm = ctx->k_norm[fi];
    p.rope_cos = ctx->rope_cos;
    p.rope_sin = ctx->rope_sin;
    p.rope_len = c.rope_table_len;
    p.k_pool = ctx->k_pool[fi];
    p.v_pool = ctx->v_pool[fi];
    p.kv_base = ctx->kv_base;
    p.kv_cap = ctx->kv_cap;
    p.kv_len = ctx->kv_len + (long long)fi * c.max_seqs;
    p.kv_start = ctx->kv_start + (long long)fi * c.max_seqs;
    p.seq_ids = plan->seq_d;
    p.pos_arr = pos_arr;
    p.pos_scalar = pos_scalar;
    p.proj = proj;
    p.proj_dtype = proj_dtype;
    p.proj_stride = ctx->fa_proj;
    p.q_head_stride = 2 * D;
    p.k_off = (long long)c.num_q_heads * 2 * D;
    p.v_off = p.k_off + (long long)c.num_kv_heads * D;
    p.gate_off = D;
    p.out = out;
    p.out_dtype = out_dtype;
    p.out_stride = (long long)c.num_q_heads * D;
    p.blk_b = plan->blk_b;
    p.blk_split = plan->blk_split;
    p.nsplit = plan->nsplit;
    p.part_off = plan->part_off;
    p.CH = plan->CH;
    p.cluster_ns = plan->ns0;
    p.part_o = plan->part_o;
    p.part_ml = plan->part_ml;
    p.cnt_head = plan->cnt_head;
    p.cnt_seq = plan->cnt_seq;
    p.err = ctx->err;
    return p;
}

GdnDecodeParams gdn_params(anelm_ctx* ctx, int layer, const anelm_plan* plan, const void* proj, int proj_dtype,
                           void* out, int out_dtype) {
    const anelm_config& c = ctx->cfg;
    const int gi = ctx->gdn_idx[layer];
    GdnDecodeParams p{};
    p.Hk = c.lin_num_key_heads;
    p.Hv = c.lin_num_val_heads;
    p.C = ctx->C;
    p.l2_eps = c.l2_eps;
    p.delta_mode = c.delta_mode;
    p.conv_w = ctx->conv_w[gi];
    p.A = ctx->A[gi];
    p.dt_bias = ctx->dt_bias[gi];
    p.norm_w = ctx->norm_w[gi];
    p.ssm = ctx->ssm[gi];
    p.ssm_rows = (long long)c.max_seqs * c.lin_num_val_heads * c.lin_key_dim;
    p.conv = ctx->conv[gi];
    p.conv_pos = ctx->conv_pos + (long long)gi * c.max_seqs * c.lin_num_key_heads;
    p.seq_ids = plan->seq_d;
    p.proj = proj;
    p.proj_dtype = proj_dtype;
    p.proj_stride = ctx->gdn_proj;
    p.out = out;
    p.out_dtype = out_dtype;
    p.out_stride = (long long)c.lin_num_val_heads * c.lin_val_dim;
    p.err = ctx->err;
    return p;
}

anelm_plan* single_plan(anelm_ctx* ctx, int seq, int* rc) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = ctx->single.find(seq);
    if (it != ctx->single.end()) {
        *rc = ANELM_OK;
        return it->second;
    }
    anelm_plan* p = nullptr;
    *rc = build_plan(ctx, 1, &seq, &p);
    if (*rc) return nullptr;
    ctx->single[seq] = p;
    return p;
}

}  // namespace

extern "C" {

ANELM_API const char* anelm_version(void) { return "anelm_b200 0.1 (sm_100a)"; }

ANELM_API const char* anelm_status_string(int s) {
    switch (s) {
        case ANELM_OK: return "ok";
        case ANELM_ERR_INVALID_ARG: return "invalid argument";
        case ANELM_ERR_CAPACITY: return "capacity exceeded";
        case ANELM_ERR_CUDA: return "CUDA error";
        case ANELM_ERR_TIMEOUT: return "device wait timed out";
        case ANELM_ERR_UNSUPPORTED: return "unsupported configuration";
        case ANELM_ERR_STATE: return "invalid state";
        case ANELM_ERR_NOMEM: return "out of device memory";
        default: return "unknown status";
    }
}

ANELM_API const char* anelm_last_error(void) { return g_err.c_str(); }

ANELM_API int anelm_device_check(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return fail(ANELM_ERR_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
    if (device < 0 || device >= n) return fail(ANELM_ERR_INVALID_ARG, "device %d of %d", device, n);
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(ANELM_ERR_UNSUPPORTED, "device %d is sm_%d%d, this build is sm_100a", device,
                                      prop.major, prop.minor);
    return ANELM_OK;
}

ANELM_API int anelm_config_default(anelm_config* c) {
    if (!c) return fail(ANELM_ERR_INVALID_ARG, "null config");
    memset(c, 0, sizeof(*c));
    c->num_layers = 24;  // qwen3_5.h:52-80
    c->layer_types = nullptr;
    c->full_attention_interval = 4;
    c->num_q_heads = 8;
    c->num_kv_heads = 2;
    c->head_dim = 256;
    c->rot_dim = 64;  // 256 * 0.25
    c->rope_theta = 10000000.0f;
    c->rms_eps = 1e-6f;
    c->attn_output_gate = 1;
    c->lin_num_key_heads = 16;
    c->lin_num_val_heads = 16;
    c->lin_key_dim = 128;
    c->lin_val_dim = 128;
    c->conv_kernel = 4;
    c->max_seqs = 1;
    c->kv_capacity = 2048;  // KV_CACHE_CAPACITY, qwen3_5.h:126
    c->seq_kv_capacity = nullptr;
    c->rope_table_len = 4096;  // MAX_SEQ_LEN, qwen3_5.h:125
    c->rope_mode = ANELM_ROPE_INTERLEAVED;
    c->delta_mode = ANELM_DELTA_CPUOPS;
    c->l2_eps = 1e-12f;
    c->qk_norm_in_core = 1;
    c->kv_mode = ANELM_KV_RING;
    return ANELM_OK;
}

ANELM_API int anelm_create(const anelm_config* cfg, int device, anelm_ctx** out) {
    if (!cfg || !out) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const anelm_config& c = *cfg;
    if (c.num_layers <= 0 || c.max_seqs <= 0) return fail(ANELM_ERR_INVALID_ARG, "num_layers/max_seqs must be > 0");
    if (c.num_q_heads <= 0 || c.num_kv_heads <= 0 || c.num_q_heads % c.num_kv_heads)
        return fail(ANELM_ERR_INVALID_ARG, "num_q_heads must be a positive multiple of num_kv_heads");
    if (c.num_q_heads / c.num_kv_heads > 4)
        return fail(ANELM_ERR_UNSUPPORTED, "more than 4 query heads per kv head is not built");
    if (c.head_dim != 128 && c.head_dim != 256) return fail(ANELM_ERR_UNSUPPORTED, "head_dim must be 128 or 256");
    if (c.rot_dim < 0 || c.rot_dim > c.head_dim || (c.rot_dim & 1))
        return fail(ANELM_ERR_INVALID_ARG, "rot_dim must be even and <= head_dim");
    if (c.lin_key_dim != 128 || c.lin_val_dim != 128)
        return fail(ANELM_ERR_UNSUPPORTED, "DeltaNet head dims must be 128");
    if (c.lin_num_key_heads <= 0 || c.lin_num_val_heads <= 0 || c.lin_num_val_heads % c.lin_num_key_heads)
        return fail(ANELM_ERR_INVALID_ARG, "lin_num_val_heads must be a positive multiple of lin_num_key_heads");
    if (c.conv_kernel != 4) return fail(ANELM_ERR_UNSUPPORTED, "conv_kernel must be 4");
    if (c.kv_capacity <= 0 && !c.seq_kv_capacity) return fail(ANELM_ERR_INVALID_ARG, "kv_capacity must be > 0");
    if (c.rope_table_len < 0) return fail(ANELM_ERR_INVALID_ARG, "rope_table_len < 0");
    if (int rc = anelm_device_check(device)) return rc;
    DeviceGuard dg(device);
    if (!dg.ok) return fail(ANELM_ERR_CUDA, "cannot select device %d", device);

    auto* ctx = new anelm_ctx();
    ctx->cfg = c;
    ctx->device = device;
    ctx->layer_types.resize(c.num_layers);
    ctx->w_in.assign(c.num_layers, nullptr);
    ctx->w_out.assign(c.num_layers, nullptr);
    ctx->hidden.assign(c.num_layers, 0);
    for (int l = 0; l < c.num_layers; l++) {
        if (c.layer_types) {
            ctx->layer_types[l] = c.layer_types[l];
        } else {  // qwen3_5.cpp:64-72: every interval-th layer is full attention
            const int iv = c.full_attention_interval > 0 ? c.full_attention_interval : 4;
            ctx->layer_types[l] = ((l + 1) % iv == 0) ? ANELM_LAYER_FULL_ATTN : ANELM_LAYER_LINEAR_ATTN;
        }
    }
    ctx->cfg.layer_types = nullptr;
    ctx->cfg.seq_kv_capacity = nullptr;
    ctx->fa_idx.assign(c.num_layers, -1);
    ctx->gdn_idx.assign(c.num_layers, -1);
    for (int l = 0; l < c.num_layers; l++) {
        if (ctx->layer_types[l] == ANELM_LAYER_FULL_ATTN) ctx->fa_idx[l] = ctx->n_fa++;
        else ctx->gdn_idx[l] = ctx->n_gdn++;
    }
    const int Hv = c.lin_num_val_heads, dk = c.lin_key_dim, dv = c.lin_val_dim;
    ctx->C = 2 * c.lin_num_key_heads * dk + Hv * dv;
    ctx->gdn_proj = ctx->C + Hv * dv + 2 * Hv;
    ctx->fa_proj = c.num_q_heads * 2 * c.head_dim + 2 * c.num_kv_heads * c.head_dim;
    ctx->cap_h.resize(c.max_seqs);
    ctx->base_h.resize(c.max_seqs);
    for (int s = 0; s < c.max_seqs; s++) {
        const int cap = c.seq_kv_capacity ? c.seq_kv_capacity[s] : c.kv_capacity;
        if (cap <= 0) {
            delete ctx;
            return fail(ANELM_ERR_INVALID_ARG, "sequence %d capacity %d", s, cap);
        }
        ctx->cap_h[s] = cap;
        ctx->base_h[s] = ctx->total_slots;
        ctx->total_slots += cap;
    }
    auto bail = [&](int rc) {
        for (void* a : ctx->allocs) cudaFree(a);
        delete ctx;
        return rc;
    };
    int rc;
#define CALLOC(ptr, count)                                              \
    do {                                                                \
        if ((rc = dev_alloc(ctx->allocs, &(ptr), (count)))) return bail(rc); \
    } while (0)
    CALLOC(ctx->err, 1);
    CALLOC(ctx->kv_base, c.max_seqs);
    CALLOC(ctx->kv_cap, c.max_seqs);
    if (cudaMemcpy(ctx->kv_base, ctx->base_h.data(), c.max_seqs * sizeof(long long), cudaMemcpyHostToDevice) ||
        cudaMemcpy(ctx->kv_cap, ctx->cap_h.data(), c.max_seqs * sizeof(int), cudaMemcpyHostToDevice))
        return bail(fail(ANELM_ERR_CUDA, "metadata upload failed"));
    if (ctx->n_fa > 0) {
        ctx->len_h.assign((size_t)ctx->n_fa * c.max_seqs, 0);
        CALLOC(ctx->kv_len, (size_t)ctx->n_fa * c.max_seqs);
        CALLOC(ctx->kv_start, (size_t)ctx->n_fa * c.max_seqs);
        const size_t row = (size_t)c.num_kv_heads * c.head_dim;
        ctx->k_pool.resize(ctx->n_fa);
        ctx->v_pool.resize(ctx->n_fa);
        ctx->q_norm.resize(ctx->n_fa);
        ctx->k_norm.resize(ctx->n_fa);
        ctx->fa_w_set.assign(ctx->n_fa, 0);
        for (int f = 0; f < ctx->n_fa; f++) {
            CALLOC(ctx->k_pool[f], (size_t)ctx->total_slots * row);
            CALLOC(ctx->v_pool[f], (size_t)ctx->total_slots * row);
            CALLOC(ctx->q_norm[f], c.head_dim);
            CALLOC(ctx->k_norm[f], c.head_dim);
        }
        if (c.rot_dim > 0 && c.rope_table_len > 0) {
            // qwen3_5.cpp:309-324, built on the host with the same libm calls
            const int half = c.rot_dim / 2;
            std::vector<float> inv(half), cs((size_t)c.rope_table_len * half), sn((size_t)c.rope_table_len * half);
            for (int j = 0, i = 0; i < c.rot_dim; i += 2, j++) inv[j] = 1.0f / powf(c.rope_theta, (float)i / (float)c.rot_dim);
            for (int pos = 0; pos < c.rope_table_len; pos++)
                for (int j = 0; j < half; j++) {
                    float angle = pos * inv[j];
                    cs[(size_t)pos * half + j] = cosf(angle);
                    sn[(size_t)pos * half + j] = sinf(angle);
                }
            CALLOC(ctx->rope_cos, cs.size());
            CALLOC(ctx->rope_sin, sn.size());
            if (cudaMemcpy(ctx->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) ||
                cudaMemcpy(ctx->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice))
                return bail(fail(ANELM_ERR_CUDA, "rope table upload failed"));
        } else {
            ctx->cfg.rope_table_len = 0;
        }
        CALLOC(ctx->py_proj, (size_t)ctx->fa_proj);
        CALLOC(ctx->py_out, (size_t)c.num_q_heads * c.head_dim);
    }
    if (ctx->n_gdn > 0) {
        CALLOC(ctx->conv_pos, (size_t)ctx->n_gdn * c.max_seqs * c.lin_num_key_heads);
        ctx->ssm.resize(ctx->n_gdn);
        ctx->conv.resize(ctx->n_gdn);
        ctx->conv_w.resize(ctx->n_gdn);
        ctx->A.resize(ctx->n_gdn);
        ctx->dt_bias.resize(ctx->n_gdn);
        ctx->norm_w.resize(ctx->n_gdn);
        ctx->gdn_w_set.assign(ctx->n_gdn, 0);
        for (int g = 0; g < ctx->n_gdn; g++) {
            CALLOC(ctx->ssm[g], (size_t)c.max_seqs * Hv * dk * dv);
            CALLOC(ctx->conv[g], (size_t)c.max_seqs * ctx->C * 3);
            CALLOC(ctx->conv_w[g], (size_t)ctx->C * 4);
            CALLOC(ctx->A[g], Hv);
            CALLOC(ctx->dt_bias[g], Hv);
            CALLOC(ctx->norm_w[g], dv);
        }
    }
#undef CALLOC
    *out = ctx;
    return ANELM_OK;
}

ANELM_API int anelm_destroy(anelm_ctx* ctx) {
    if (!ctx) return ANELM_OK;
    DeviceGuard dg(ctx->device);
    cudaDeviceSynchronize();
    for (auto& kv : ctx->single) free_plan(kv.second);
    if (ctx->prefill_ws) cudaFree(ctx->prefill_ws);
    if (ctx->gdn_prefill_ws) cudaFree(ctx->gdn_prefill_ws);
    if (ctx->layer_ws) cudaFree(ctx->layer_ws);
    for (void* w : ctx->w_in) if (w) cudaFree(w);
    for (void* w : ctx->w_out) if (w) cudaFree(w);
    for (void* a : ctx->allocs) cudaFree(a);
    delete ctx;
    return ANELM_OK;
}

ANELM_API int anelm_set_full_attn_weights(anelm_ctx* ctx, int layer, const float* qn, const float* kn) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (!qn || !kn) return fail(ANELM_ERR_INVALID_ARG, "null weight");
    DeviceGuard dg(ctx->device);
    const int f = ctx->fa_idx[layer];
    CUDA_TRY(cudaMemcpy(ctx->q_norm[f], qn, ctx->cfg.head_dim * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->k_norm[f], kn, ctx->cfg.head_dim * 4, cudaMemcpyHostToDevice));
    ctx->fa_w_set[f] = 1;
    return ANELM_OK;
}

ANELM_API int anelm_set_deltanet_weights(anelm_ctx* ctx, int layer, const float* conv_w, const float* A,
                                         const float* dt_bias, const float* norm_w) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (!conv_w || !A || !dt_bias || !norm_w) return fail(ANELM_ERR_INVALID_ARG, "null weight");
    DeviceGuard dg(ctx->device);
    const int g = ctx->gdn_idx[layer];
    const int Hv = ctx->cfg.lin_num_val_heads;
    CUDA_TRY(cudaMemcpy(ctx->conv_w[g], conv_w, (size_t)ctx->C * 4 * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->A[g], A, Hv * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->dt_bias[g], dt_bias, Hv * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->norm_w[g], norm_w, ctx->cfg.lin_val_dim * 4, cudaMemcpyHostToDevice));
    ctx->gdn_w_set[g] = 1;
    return ANELM_OK;
}

ANELM_API int anelm_reset(anelm_ctx* ctx, int seq) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (seq != -1)
        if (int rc = check_seq(ctx, seq)) return rc;
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int s0 = seq < 0 ? 0 : seq, s1 = seq < 0 ? c.max_seqs : seq + 1;
    const size_t row = (size_t)c.num_kv_heads * c.head_dim;
    for (int f = 0; f < ctx->n_fa; f++) {
        const long long a = ctx->base_h[s0], e = (s1 < c.max_seqs) ? ctx->base_h[s1] : ctx->total_slots;
        CUDA_TRY(cudaMemset(ctx->k_pool[f] + a * row, 0, (e - a) * row * 2));
        CUDA_TRY(cudaMemset(ctx->v_pool[f] + a * row, 0, (e - a) * row * 2));
        CUDA_TRY(cudaMemset(ctx->kv_len + (size_t)f * c.max_seqs + s0, 0, (s1 - s0) * 4));
        CUDA_TRY(cudaMemset(ctx->kv_start + (size_t)f * c.max_seqs + s0, 0, (s1 - s0) * 4));
        for (int s = s0; s < s1; s++) ctx->len_h[(size_t)f * c.max_seqs + s] = 0;
    }
    const size_t st = (size_t)c.lin_num_val_heads * c.lin_key_dim * c.lin_val_dim;
    for (int g = 0; g < ctx->n_gdn; g++) {
        CUDA_TRY(cudaMemset(ctx->ssm[g] + s0 * st, 0, (s1 - s0) * st * 4));
        CUDA_TRY(cudaMemset(ctx->conv[g] + (size_t)s0 * ctx->C * 3, 0, (size_t)(s1 - s0) * ctx->C * 12));
        const size_t hk = c.lin_num_key_heads;
        CUDA_TRY(cudaMemset(ctx->conv_pos + ((size_t)g * c.max_seqs + s0) * hk, 0, (s1 - s0) * hk * 4));
    }
    CUDA_TRY(cudaDeviceSynchronize());
    return ANELM_OK;
}

ANELM_API int anelm_kv_export(anelm_ctx* ctx, int layer, int seq, float* k_host, float* v_host, int* len,
                              int* start) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int f = ctx->fa_idx[layer];
    const size_t n = (size_t)ctx->cap_h[seq] * c.num_kv_heads * c.head_dim;
    const size_t off = (size_t)ctx->base_h[seq] * c.num_kv_heads * c.head_dim;
    std::vector<__half> tmp(n);
    CUDA_TRY(cudaDeviceSynchronize());
    if (k_host) {
        CUDA_TRY(cudaMemcpy(tmp.data(), ctx->k_pool[f] + off, n * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; i++) k_host[i] = __half2float(tmp[i]);
    }
    if (v_host) {
        CUDA_TRY(cudaMemcpy(tmp.data(), ctx->v_pool[f] + off, n * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; i++) v_host[i] = __half2float(tmp[i]);
    }
    if (len) CUDA_TRY(cudaMemcpy(len, ctx->kv_len + (size_t)f * c.max_seqs + seq, 4, cudaMemcpyDeviceToHost));
    if (start) CUDA_TRY(cudaMemcpy(start, ctx->kv_start + (size_t)f * c.max_seqs + seq, 4, cudaMemcpyDeviceToHost));
    return ANELM_OK;
}

ANELM_API int anelm_kv_import(anelm_ctx* ctx, int layer, int seq, const float* k_host, const float* v_host, int len,
                              int start) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    const int cap = ctx->cap_h[seq];
    if (len < 0 || len > cap || start < 0 || start >= cap)
        return fail(ANELM_ERR_CAPACITY, "len %d / start %d outside capacity %d", len, start, cap);
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int f = ctx->fa_idx[layer];
    const size_t n = (size_t)cap * c.num_kv_heads * c.head_dim;
    const size_t off = (size_t)ctx->base_h[seq] * c.num_kv_heads * c.head_dim;
    std::vector<__half> tmp(n);
    CUDA_TRY(cudaDeviceSynchronize());
    if (k_host) {
        for (size_t i = 0; i < n; i++) tmp[i] = __float2half_rn(k_host[i]);
        CUDA_TRY(cudaMemcpy(ctx->k_pool[f] + off, tmp.data(), n * 2, cudaMemcpyHostToDevice));
    }
    if (v_host) {
        for (size_t i = 0; i < n; i++) tmp[i] = __float2half_rn(v_host[i]);
        CUDA_TRY(cudaMemcpy(ctx->v_pool[f] + off, tmp.data(), n * 2, cudaMemcpyHostToDevice));
    }
    CUDA_TRY(cudaMemcpy(ctx->kv_len + (size_t)f * c.max_seqs + seq, &len, 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->kv_start + (size_t)f * c.max_seqs + seq, &start, 4, cudaMemcpyHostToDevice));
    ctx->len_h[(size_t)f * c.max_seqs + seq] = len;
    return ANELM_OK;
}

ANELM_API int anelm_kv_write(anelm_ctx* ctx, int layer, int seq, int slot0, int n_slots, const void* k_src,
                             const void* v_src, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    const int cap = ctx->cap_h[seq];
    if (slot0 < 0 || n_slots < 0 || slot0 + n_slots > cap)
        return fail(ANELM_ERR_CAPACITY, "slots [%d,%d) outside capacity %d", slot0, slot0 + n_slots, cap);
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int f = ctx->fa_idx[layer];
    const size_t row = (size_t)c.num_kv_heads * c.head_dim;
    const size_t off = ((size_t)ctx->base_h[seq] + slot0) * row;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (k_src) CUDA_TRY(cudaMemcpyAsync(ctx->k_pool[f] + off, k_src, n_slots * row * 2, cudaMemcpyDeviceToDevice, st));
    if (v_src) CUDA_TRY(cudaMemcpyAsync(ctx->v_pool[f] + off, v_src, n_slots * row * 2, cudaMemcpyDeviceToDevice, st));
    return ANELM_OK;
}

ANELM_API int anelm_kv_set_meta(anelm_ctx* ctx, int layer, int seq, int len, int start) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    const int cap = ctx->cap_h[seq];
    if (len < 0 || len > cap || start < 0 || start >= cap)
        return fail(ANELM_ERR_CAPACITY, "len %d / start %d outside capacity %d", len, start, cap);
    DeviceGuard dg(ctx->device);
    const int f = ctx->fa_idx[layer];
    CUDA_TRY(cudaMemcpy(ctx->kv_len + (size_t)f * ctx->cfg.max_seqs + seq, &len, 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(ctx->kv_start + (size_t)f * ctx->cfg.max_seqs + seq, &start, 4, cudaMemcpyHostToDevice));
    ctx->len_h[(size_t)f * ctx->cfg.max_seqs + seq] = len;
    return ANELM_OK;
}

ANELM_API int anelm_deltanet_state_export(anelm_ctx* ctx, int layer, int seq, float* ssm_host, float* conv_host,
                                          int* conv_pos) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int g = ctx->gdn_idx[layer];
    const size_t st = (size_t)c.lin_num_val_heads * c.lin_key_dim * c.lin_val_dim;
    CUDA_TRY(cudaDeviceSynchronize());
    if (ssm_host) CUDA_TRY(cudaMemcpy(ssm_host, ctx->ssm[g] + seq * st, st * 4, cudaMemcpyDeviceToHost));
    // the ring is kept in the reference layout [C][3]; every key-head copy of the position is equal
    const size_t hk = c.lin_num_key_heads;
    std::vector<int> pos(hk);
    CUDA_TRY(cudaMemcpy(pos.data(), ctx->conv_pos + ((size_t)g * c.max_seqs + seq) * hk, hk * 4,
                        cudaMemcpyDeviceToHost));
    for (size_t i = 1; i < hk; i++)
        if (pos[i] != pos[0]) return fail(ANELM_ERR_STATE, "conv ring positions disagree across key heads");
    if (conv_host)
        CUDA_TRY(cudaMemcpy(conv_host, ctx->conv[g] + (size_t)seq * ctx->C * 3, (size_t)ctx->C * 12,
                            cudaMemcpyDeviceToHost));
    if (conv_pos) *conv_pos = pos[0];
    return ANELM_OK;
}

ANELM_API int anelm_deltanet_state_import(anelm_ctx* ctx, int layer, int seq, const float* ssm_host,
                                          const float* conv_host, int conv_pos) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    if (conv_pos < 0 || conv_pos > 2) return fail(ANELM_ERR_INVALID_ARG, "conv_pos %d not in [0,3)", conv_pos);
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const int g = ctx->gdn_idx[layer];
    const size_t st = (size_t)c.lin_num_val_heads * c.lin_key_dim * c.lin_val_dim;
    CUDA_TRY(cudaDeviceSynchronize());
    if (ssm_host) CUDA_TRY(cudaMemcpy(ctx->ssm[g] + seq * st, ssm_host, st * 4, cudaMemcpyHostToDevice));
    if (conv_host)
        CUDA_TRY(cudaMemcpy(ctx->conv[g] + (size_t)seq * ctx->C * 3, conv_host, (size_t)ctx->C * 12,
                            cudaMemcpyHostToDevice));
    const size_t hk = c.lin_num_key_heads;
    std::vector<int> pos(hk, conv_pos);
    CUDA_TRY(cudaMemcpy(ctx->conv_pos + ((size_t)g * c.max_seqs + seq) * hk, pos.data(), hk * 4,
                        cudaMemcpyHostToDevice));
    return ANELM_OK;
}

ANELM_API int anelm_deltanet_state_write(anelm_ctx* ctx, int layer, int seq, const float* ssm_src, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    if (!ssm_src) return fail(ANELM_ERR_INVALID_ARG, "null source");
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    const size_t st = (size_t)c.lin_num_val_heads * c.lin_key_dim * c.lin_val_dim;
    CUDA_TRY(cudaMemcpyAsync(ctx->ssm[ctx->gdn_idx[layer]] + seq * st, ssm_src, st * 4, cudaMemcpyDeviceToDevice,
                             static_cast<cudaStream_t>(stream)));
    return ANELM_OK;
}

ANELM_API int anelm_get_device_error(anelm_ctx* ctx, int* code) {
    if (!ctx || !code) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(code, ctx->err, 4, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemset(ctx->err, 0, 4));
    return ANELM_OK;
}

ANELM_API int anelm_plan_create(anelm_ctx* ctx, int n, const int* seq_ids, anelm_plan** out) {
    if (!ctx || !out) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(ctx->device);
    return build_plan(ctx, n, seq_ids, out);
}

ANELM_API int anelm_plan_destroy(anelm_plan* plan) {
    if (!plan) return ANELM_OK;
    DeviceGuard dg(plan->ctx->device);
    cudaDeviceSynchronize();
    free_plan(plan);
    return ANELM_OK;
}

ANELM_API int anelm_plan_info(const anelm_plan* plan, int* split_tokens, int* n_blocks) {
    if (!plan) return fail(ANELM_ERR_INVALID_ARG, "null plan");
    if (split_tokens) *split_tokens = plan->CH;
    if (n_blocks) *n_blocks = plan->n_blocks;
    return ANELM_OK;
}

static int fa_launch(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* proj, int proj_dtype,
                     const int* pos_arr, int pos_scalar, void* out, int out_dtype, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (!plan || plan->ctx != ctx) return fail(ANELM_ERR_INVALID_ARG, "plan belongs to another context");
    if (!proj || !out) return fail(ANELM_ERR_INVALID_ARG, "null tensor");
    if (int rc = check_dtype(proj_dtype)) return rc;
    if (int rc = check_dtype(out_dtype)) return rc;
    if (ctx->cfg.qk_norm_in_core && !ctx->fa_w_set[ctx->fa_idx[layer]])
        return fail(ANELM_ERR_STATE, "full-attention weights of layer %d not set", layer);
    DeviceGuard dg(ctx->device);
    for (int s : plan->seq_h) {  // one append per row (a linear cache's length follows the position: unknown here)
        int& len = ctx->len_h[(size_t)ctx->fa_idx[layer] * ctx->cfg.max_seqs + s];
        len = ctx->cfg.kv_mode == ANELM_KV_LINEAR ? ctx->cap_h[s] : std::min(len + 1, ctx->cap_h[s]);
    }
    FaDecodeParams p = fa_params(ctx, layer, plan, proj, proj_dtype, pos_arr, pos_scalar, out, out_dtype);
    return launch_status(launch_fa_decode(p, ctx->cfg.head_dim, plan->n_blocks, static_cast<cudaStream_t>(stream)),
                         "fa_decode");
}

ANELM_API int anelm_full_attn_from_proj(anelm_ctx* ctx, int layer, int seq, const void* proj, int proj_dtype, int pos,
                                        void* out, int out_dtype, void* stream) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (int rc = check_seq(ctx, seq)) return rc;
    if (ctx->cfg.kv_mode == ANELM_KV_LINEAR && (pos < 0 || pos >= ctx->cap_h[seq]))
        return fail(ANELM_ERR_CAPACITY, "position %d outside linear cache of %d", pos, ctx->cap_h[seq]);
    int rc = 0;
    anelm_plan* plan;
    {
        DeviceGuard dg(ctx->device);
        plan = single_plan(ctx, seq, &rc);
    }
    if (rc) return rc;
    return fa_launch(ctx, plan, layer, proj, proj_dtype, nullptr, pos, out, out_dtype, stream);
}

ANELM_API int anelm_full_attn_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* proj,
                                     int proj_dtype, const int* pos, void* out, int out_dtype, void* stream) {
    if (!pos) return fail(ANELM_ERR_INVALID_ARG, "null positions");
    return fa_launch(ctx, plan, layer, proj, proj_dtype, pos, 0, out, out_dtype, stream);
}

static int gdn_launch(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* proj, int proj_dtype, void* out,
                      int out_dtype, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (!plan || plan->ctx != ctx) return fail(ANELM_ERR_INVALID_ARG, "plan belongs to another context");
    if (!proj || !out) return fail(ANELM_ERR_INVALID_ARG, "null tensor");
    if (int rc = check_dtype(proj_dtype)) return rc;
    if (int rc = check_dtype(out_dtype)) return rc;
    if (!ctx->gdn_w_set[ctx->gdn_idx[layer]]) return fail(ANELM_ERR_STATE, "DeltaNet weights of layer %d not set", layer);
    DeviceGuard dg(ctx->device);
    GdnDecodeParams p = gdn_params(ctx, layer, plan, proj, proj_dtype, out, out_dtype);
    return launch_status(launch_gdn_decode(p, plan->n, ctx->cfg.lin_key_dim, ctx->cfg.lin_val_dim,
                                           static_cast<cudaStream_t>(stream)),
                         "gdn_decode");
}

ANELM_API int anelm_deltanet_from_proj(anelm_ctx* ctx, int layer, int seq, const void* proj, int proj_dtype,
                                       void* out, int out_dtype, void* stream) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (int rc = check_seq(ctx, seq)) return rc;
    int rc = 0;
    anelm_plan* plan;
    {
        DeviceGuard dg(ctx->device);
        plan = single_plan(ctx, seq, &rc);
    }
    if (rc) return rc;
    return gdn_launch(ctx, plan, layer, proj, proj_dtype, out, out_dtype, stream);
}

ANELM_API int anelm_deltanet_prefill(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                     const void* proj, int proj_dtype, void* out, int out_dtype, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_LINEAR_ATTN)) return rc;
    if (!plan || plan->ctx != ctx) return fail(ANELM_ERR_INVALID_ARG, "plan belongs to another context");
    if (!proj || !out || n_tokens <= 0) return fail(ANELM_ERR_INVALID_ARG, "null tensor or no tokens");
    if (int rc = check_dtype(proj_dtype)) return rc;
    if (int rc = check_dtype(out_dtype)) return rc;
    const anelm_config& c = ctx->cfg;
    if (c.lin_key_dim != 128 || c.lin_val_dim != 128)
        return fail(ANELM_ERR_UNSUPPORTED, "DeltaNet prefill is built for key/value head dims 128");
    if (c.conv_kernel != 4) return fail(ANELM_ERR_UNSUPPORTED, "DeltaNet prefill is built for conv kernel 4");
    const int gi = ctx->gdn_idx[layer];
    if (!ctx->gdn_w_set[gi]) return fail(ANELM_ERR_STATE, "DeltaNet weights of layer %d not set", layer);
    DeviceGuard dg(ctx->device);
    const size_t need = gdn_prefill_workspace_bytes(plan->n, n_tokens, c.lin_num_key_heads, c.lin_num_val_heads,
                                                    ctx->C, true);
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (need > ctx->gdn_prefill_ws_bytes) {
            if (ctx->gdn_prefill_ws) cudaFree(ctx->gdn_prefill_ws);
            ctx->gdn_prefill_ws = nullptr;
            ctx->gdn_prefill_ws_bytes = 0;
            cudaError_t e = cudaMalloc(&ctx->gdn_prefill_ws, need);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(ANELM_ERR_NOMEM, "DeltaNet prefill workspace of %zu bytes: %s", need, cudaGetErrorString(e));
            }
            ctx->gdn_prefill_ws_bytes = need;
        }
    }
    GdnPrefillParams p{};
    p.B = plan->n;
    p.n = n_tokens;
    p.Hk = c.lin_num_key_heads;
    p.Hv = c.lin_num_val_heads;
    p.dk = c.lin_key_dim;
    p.dv = c.lin_val_dim;
    p.C = ctx->C;
    p.delta_mode = c.delta_mode;
    p.l2_eps = c.l2_eps;
    p.conv_w = ctx->conv_w[gi];
    p.A = ctx->A[gi];
    p.dt_bias = ctx->dt_bias[gi];
    p.norm_w = ctx->norm_w[gi];
    p.conv = ctx->conv[gi];
    p.conv_pos = ctx->conv_pos + (long long)gi * c.max_seqs * c.lin_num_key_heads;
    p.proj = proj;
    p.proj_dtype = proj_dtype;
    p.proj_stride = ctx->gdn_proj;
    p.out = out;
    p.out_dtype = out_dtype;
    p.out_stride = (long long)c.lin_num_val_heads * c.lin_val_dim;
    p.state = ctx->ssm[gi];
    p.seq_ids = plan->seq_d;
    p.err = ctx->err;
    return launch_status(launch_gdn_prefill(p, ctx->gdn_prefill_ws, static_cast<cudaStream_t>(stream)),
                         "deltanet_prefill");
}

ANELM_API size_t anelm_gated_delta_chunked_workspace_bytes(int B, int T, int Hk, int Hv) {
    if (B <= 0 || T <= 0 || Hk <= 0 || Hv <= 0) return 0;
    return gdn_prefill_workspace_bytes(B, T, Hk, Hv, 0, false);
}

ANELM_API int anelm_gated_delta_chunked(const void* q, const void* k, const void* v, int qkv_dtype,
                                        const float* log_decay, const float* beta, float* state, int B, int T,
                                        int Hk, int Hv, int dk, int dv, int delta_mode, void* y, int y_dtype,
                                        void* workspace, size_t workspace_bytes, void* stream) {
    if (!q || !k || !v || !log_decay || !beta || !state || !y || !workspace)
        return fail(ANELM_ERR_INVALID_ARG, "null pointer");
    if (B <= 0 || T <= 0 || Hk <= 0 || Hv <= 0 || Hv % Hk)
        return fail(ANELM_ERR_INVALID_ARG, "bad sizes B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
    if (dk != 128 || dv != 128) return fail(ANELM_ERR_UNSUPPORTED, "chunked delta rule is built for dk = dv = 128");
    if (delta_mode != ANELM_DELTA_CPUOPS && delta_mode != ANELM_DELTA_HF)
        return fail(ANELM_ERR_INVALID_ARG, "unknown delta mode %d", delta_mode);
    if (int rc = check_dtype(qkv_dtype)) return rc;
    if (int rc = check_dtype(y_dtype)) return rc;
    const size_t need = gdn_prefill_workspace_bytes(B, T, Hk, Hv, 0, false);
    if (workspace_bytes < need)
        return fail(ANELM_ERR_CAPACITY, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
    GdnPrefillParams p{};
    p.B = B;
    p.n = T;
    p.Hk = Hk;
    p.Hv = Hv;
    p.dk = dk;
    p.dv = dv;
    p.delta_mode = delta_mode;
    p.q_in = q;
    p.k_in = k;
    p.v_in = v;
    p.in_dtype = qkv_dtype;
    p.lg_in = log_decay;
    p.beta_in = beta;
    p.state = state;
    p.y = y;
    p.y_dtype = y_dtype;
    p.y_stride = (long long)Hv * dv;
    return launch_status(launch_gated_delta_chunked(p, workspace, static_cast<cudaStream_t>(stream)),
                         "gated_delta_chunked");
}

ANELM_API int anelm_deltanet_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* proj,
                                    int proj_dtype, void* out, int out_dtype, void* stream) {
    return gdn_launch(ctx, plan, layer, proj, proj_dtype, out, out_dtype, stream);
}

// Projection widths around the core of a layer: rows in (the projections the core reads) and
// the core's output row.
static void layer_widths(const anelm_ctx* ctx, int layer, int* proj_dim, int* out_dim) {
    const anelm_config& c = ctx->cfg;
    if (ctx->layer_types[layer] == ANELM_LAYER_FULL_ATTN) {
        *proj_dim = ctx->fa_proj;
        *out_dim = c.num_q_heads * c.head_dim;
    } else {
        *proj_dim = ctx->gdn_proj;
        *out_dim = c.lin_num_val_heads * c.lin_val_dim;
    }
}

ANELM_API int anelm_set_layer_projections(anelm_ctx* ctx, int layer, int hidden, const void* w_in,
                                          const void* w_out) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers)
        return fail(ANELM_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, ctx->cfg.num_layers);
    if (!w_in || !w_out || hidden <= 0 || hidden % 8)
        return fail(ANELM_ERR_INVALID_ARG, "projection weights need hidden > 0, a multiple of 8");
    int pd = 0, od = 0;
    layer_widths(ctx, layer, &pd, &od);
    if (pd % 8 || od % 8) return fail(ANELM_ERR_UNSUPPORTED, "projection widths %d / %d not multiples of 8", pd, od);
    DeviceGuard dg(ctx->device);
    for (void** w : {&ctx->w_in[layer], &ctx->w_out[layer]}) {
        if (*w) cudaFree(*w);
        *w = nullptr;
    }
    ctx->hidden[layer] = 0;
    const size_t bi = (size_t)pd * hidden * 2, bo = (size_t)hidden * od * 2;
    if (cudaMalloc(&ctx->w_in[layer], bi) != cudaSuccess || cudaMalloc(&ctx->w_out[layer], bo) != cudaSuccess) {
        cudaGetLastError();
        return fail(ANELM_ERR_NOMEM, "projection weights of layer %d", layer);
    }
    CUDA_TRY(cudaMemcpy(ctx->w_in[layer], w_in, bi, cudaMemcpyDefault));
    CUDA_TRY(cudaMemcpy(ctx->w_out[layer], w_out, bo, cudaMemcpyDefault));
    ctx->hidden[layer] = hidden;
    return ANELM_OK;
}

ANELM_API int anelm_layer_decode(anelm_ctx* ctx, const anelm_plan* plan, int layer, const void* x, const int* pos,
                                 void* y, void* stream) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (layer < 0 || layer >= ctx->cfg.num_layers)
        return fail(ANELM_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, ctx->cfg.num_layers);
    if (!plan || plan->ctx != ctx) return fail(ANELM_ERR_INVALID_ARG, "plan belongs to another context");
    if (!x || !y) return fail(ANELM_ERR_INVALID_ARG, "null tensor");
    const int H = ctx->hidden[layer];
    if (!H) return fail(ANELM_ERR_STATE, "projections of layer %d not set", layer);
    const bool fa = ctx->layer_types[layer] == ANELM_LAYER_FULL_ATTN;
    if (fa && !pos) return fail(ANELM_ERR_INVALID_ARG, "null positions");
    int pd = 0, od = 0;
    layer_widths(ctx, layer, &pd, &od);
    const int n = plan->n;
    DeviceGuard dg(ctx->device);
    const size_t need = (size_t)n * (pd + od) * 2 + 256;
    if (need > ctx->layer_ws_bytes) {
        if (ctx->layer_ws) cudaFree(ctx->layer_ws);
        ctx->layer_ws = nullptr;
        ctx->layer_ws_bytes = 0;
        if (cudaMalloc(&ctx->layer_ws, need) != cudaSuccess) {
            cudaGetLastError();
            return fail(ANELM_ERR_NOMEM, "layer-step staging of %zu bytes", need);
        }
        ctx->layer_ws_bytes = need;
    }
    __nv_bfloat16* proj = static_cast<__nv_bfloat16*>(ctx->layer_ws);
    __nv_bfloat16* core = proj + ((size_t)n * pd + 127) / 128 * 128;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // first_proj on the device: [n][hidden] x [proj_dim][hidden]^T -> projection rows
    if (int rc = launch_status(launch_gemm_bf16_tn(x, H, ctx->w_in[layer], H, proj, pd, ANELM_BF16, n, pd, H, ctx->err, st),
                               "layer in-projection"))
        return rc;
    const int rc = fa ? fa_launch(ctx, plan, layer, proj, ANELM_BF16, pos, 0, core, ANELM_BF16, stream)
                      : gdn_launch(ctx, plan, layer, proj, ANELM_BF16, core, ANELM_BF16, stream);
    if (rc) return rc;
    // o_proj: [n][core out] x [hidden][core out]^T -> hidden rows
    return launch_status(launch_gemm_bf16_tn(core, od, ctx->w_out[layer], od, y, H, ANELM_BF16, n, H, od, ctx->err, st),
                         "layer out-projection");
}

static int full_attn_prefill_impl(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens, const void* proj,
                                  int proj_dtype, int start_pos, void* out, int out_dtype, long long out_stride,
                                  const PrefillDests* dests, void* stream) {
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (!plan || plan->ctx != ctx) return fail(ANELM_ERR_INVALID_ARG, "plan belongs to another context");
    if (!proj || !out || n_tokens <= 0) return fail(ANELM_ERR_INVALID_ARG, "null tensor or no tokens");
    if (int rc = check_dtype(proj_dtype)) return rc;
    if (int rc = check_dtype(out_dtype)) return rc;
    const anelm_config& c = ctx->cfg;
    if (c.head_dim != 256) return fail(ANELM_ERR_UNSUPPORTED, "prefill kernel is built for head_dim 256");
    if (c.kv_mode == ANELM_KV_LINEAR && start_pos != 0)
        return fail(ANELM_ERR_UNSUPPORTED, "linear-cache prefill starts at position 0");
    if (c.qk_norm_in_core && !ctx->fa_w_set[ctx->fa_idx[layer]])
        return fail(ANELM_ERR_STATE, "full-attention weights of layer %d not set", layer);
    const int f = ctx->fa_idx[layer];
    // old-token rows: the first new token of a sequence sees min(len, capacity - 1) old tokens
    int P = 0;
    for (int s : plan->seq_h) {
        const int len = ctx->len_h[(size_t)f * c.max_seqs + s];
        if (c.kv_mode == ANELM_KV_LINEAR && (len != 0 || n_tokens > ctx->cap_h[s]))
            return fail(ANELM_ERR_CAPACITY, "linear-cache prefill fills an empty cache of %d positions (sequence %d)",
                        ctx->cap_h[s], s);
        P = std::max(P, std::min(len, ctx->cap_h[s] - 1));
    }
    P = (P + 127) / 128 * 128;
    DeviceGuard dg(ctx->device);
    const size_t need = fa_prefill_workspace_bytes(plan->n, n_tokens, P, c.num_q_heads, c.num_kv_heads, c.head_dim);
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (need > ctx->prefill_ws_bytes) {
            if (ctx->prefill_ws) cudaFree(ctx->prefill_ws);
            ctx->prefill_ws = nullptr;
            ctx->prefill_ws_bytes = 0;
            cudaError_t e = cudaMalloc(&ctx->prefill_ws, need);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(ANELM_ERR_NOMEM, "prefill workspace of %zu bytes: %s", need, cudaGetErrorString(e));
            }
            ctx->prefill_ws_bytes = need;
        }
    }
    FaPrefillParams p{};
    p.B = plan->n;
    p.n = n_tokens;
    p.Hq = c.num_q_heads;
    p.Hkv = c.num_kv_heads;
    p.rot_dim = c.rot_dim;
    p.rope_theta = c.rope_theta;
    p.rms_eps = c.rms_eps;
    p.qk_norm = c.qk_norm_in_core;
    p.rope_mode = c.rope_mode;
    p.gate = c.attn_output_gate;
    p.start_pos = start_pos;
    p.P = P;
    p.q_norm = ctx->q_norm[f];
    p.k_norm = ctx->k_norm[f];
    p.rope_cos = ctx->rope_cos;
    p.rope_sin = ctx->rope_sin;
    p.rope_len = c.rope_table_len;
    p.proj = proj;
    p.proj_dtype = proj_dtype;
    p.proj_stride = ctx->fa_proj;
    p.k_pool = ctx->k_pool[f];
    p.v_pool = ctx->v_pool[f];
    p.kv_base = ctx->kv_base;
    p.seq_ids = plan->seq_d;
    p.kv_len = ctx->kv_len + (size_t)f * c.max_seqs;
    p.kv_start = ctx->kv_start + (size_t)f * c.max_seqs;
    p.kv_cap = ctx->kv_cap;
    p.out = out;
    p.out_dtype = out_dtype;
    p.out_stride = out_stride;
    p.err = ctx->err;
    const int rc = launch_fa_prefill(p, ctx->prefill_ws, c.head_dim, static_cast<cudaStream_t>(stream), dests);
    if (rc) return launch_status(rc, "fa_prefill");
    for (int s : plan->seq_h) {
        int& len = ctx->len_h[(size_t)f * c.max_seqs + s];
        len = (int)std::min<long long>((long long)len + n_tokens, ctx->cap_h[s]);
    }
    return ANELM_OK;
}

ANELM_API int anelm_full_attn_prefill(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                      const void* proj, int proj_dtype, int start_pos, void* out, int out_dtype,
                                      void* stream) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    return full_attn_prefill_impl(ctx, plan, layer, n_tokens, proj, proj_dtype, start_pos, out, out_dtype,
                                  (long long)ctx->cfg.num_q_heads * ctx->cfg.head_dim, nullptr, stream);
}

ANELM_API int anelm_full_attn_prefill_gather(anelm_ctx* ctx, const anelm_plan* plan, int layer, int n_tokens,
                                             const void* proj, int proj_dtype, int start_pos, void* const* outs,
                                             int n_outs, int col0, int out_cols, int out_dtype, void* stream) {
    if (!ctx || !outs) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    if (n_outs < 1 || n_outs > 8) return fail(ANELM_ERR_INVALID_ARG, "1 to 8 output buffers");
    for (int r = 0; r < n_outs; r++)
        if (!outs[r] || (uintptr_t)outs[r] % 16) return fail(ANELM_ERR_INVALID_ARG, "output %d null or not 16-byte aligned", r);
    if (out_dtype != ANELM_BF16 && out_dtype != ANELM_F16) return fail(ANELM_ERR_UNSUPPORTED, "16-bit outputs only");
    const long long cols = (long long)ctx->cfg.num_q_heads * ctx->cfg.head_dim;
    if (col0 < 0 || col0 % 64 || out_cols % 8 || col0 + cols > out_cols)
        return fail(ANELM_ERR_INVALID_ARG, "columns [%d, %lld) outside a row of %d (or not 64-aligned)", col0, col0 + cols,
                    out_cols);
    PrefillDests d{outs, n_outs, col0};
    return full_attn_prefill_impl(ctx, plan, layer, n_tokens, proj, proj_dtype, start_pos, outs[0], out_dtype,
                                  out_cols, &d, stream);
}

// ---- CUDA IPC: map another process's device buffer (peer outputs of a sharded prefill) ----

namespace {
typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
    static AddrRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<AddrRangeFn>(f);
    }();
    return fn;
}
std::mutex g_ipc_mu;
std::map<void*, void*> g_ipc_base;  // pointer handed out by anelm_ipc_open -> mapping base
}  // namespace

ANELM_API int anelm_ipc_handle(const void* dev_ptr, void* handle_out, size_t* offset_out) {
    if (!dev_ptr || !handle_out || !offset_out) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    AddrRangeFn range = addr_range_fn();
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!range || range(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS)
        return fail(ANELM_ERR_CUDA, "cuMemGetAddressRange failed for %p", dev_ptr);
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    memcpy(handle_out, &h, sizeof(h));
    *offset_out = (size_t)((CUdeviceptr)dev_ptr - base);
    return ANELM_OK;
}

ANELM_API int anelm_ipc_open(const void* handle, size_t offset, int device, void** ptr_out) {
    if (!handle || !ptr_out) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    DeviceGuard dg(device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    void* p = static_cast<char*>(base) + offset;
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    g_ipc_base[p] = base;
    *ptr_out = p;
    return ANELM_OK;
}

ANELM_API int anelm_ipc_close(void* ptr) {
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_ipc_mu);
        auto it = g_ipc_base.find(ptr);
        if (it == g_ipc_base.end()) return fail(ANELM_ERR_INVALID_ARG, "%p was not opened by anelm_ipc_open", ptr);
        base = it->second;
        g_ipc_base.erase(it);
    }
    CUDA_TRY(cudaIpcCloseMemHandle(base));
    return ANELM_OK;
}

ANELM_API int anelm_py_cpu_attention(anelm_ctx* ctx, int layer, int seq, const uint16_t* q_gate, const uint16_t* k,
                                     const uint16_t* v, int pos, uint16_t* out, void* stream) {
    if (!ctx || !q_gate || !k || !v || !out) return fail(ANELM_ERR_INVALID_ARG, "null argument");
    if (ctx->cfg.rope_mode != ANELM_ROPE_HALF || ctx->cfg.qk_norm_in_core || ctx->cfg.kv_mode != ANELM_KV_LINEAR)
        return fail(ANELM_ERR_STATE, "context is not configured for the serve_hybrid route");
    if (int rc = check_layer(ctx, layer, ANELM_LAYER_FULL_ATTN)) return rc;
    if (int rc = check_seq(ctx, seq)) return rc;
    DeviceGuard dg(ctx->device);
    const anelm_config& c = ctx->cfg;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t nq = (size_t)c.num_q_heads * 2 * c.head_dim, nk = (size_t)c.num_kv_heads * c.head_dim;
    CUDA_TRY(cudaMemcpyAsync(ctx->py_proj, q_gate, nq * 2, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(ctx->py_proj + nq, k, nk * 2, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(ctx->py_proj + nq + nk, v, nk * 2, cudaMemcpyHostToDevice, st));
    if (int rc = anelm_full_attn_from_proj(ctx, layer, seq, ctx->py_proj, ANELM_F16, pos, ctx->py_out, ANELM_F16, stream))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(out, ctx->py_out, (size_t)c.num_q_heads * c.head_dim * 2, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    int code = 0;
    CUDA_TRY(cudaMemcpy(&code, ctx->err, 4, cudaMemcpyDeviceToHost));
    if (code) {
        cudaMemset(ctx->err, 0, 4);
        return fail(code, "device reported status %d", code);
    }
    return ANELM_OK;
}

// ---- bounded-wait self-test ----

namespace {
// One thread waits on an mbarrier that nothing arrives on, with the same bounded wait every
// tensor-core kernel uses; after `polls` polls it records ANELM_ERR_TIMEOUT in the context's error
// word and returns.  No copy or MMA is in flight, so the give-up path leaves nothing behind.
__global__ void bounded_wait_probe_kernel(int* err, uint32_t polls) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        abort = 0;
        tc::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) tc::mbar_wait_polls(&bar, 0, err, ANELM_ERR_TIMEOUT, &abort, polls);
}
}  // namespace

ANELM_API int anelm_selftest_wait_timeout(anelm_ctx* ctx, unsigned polls, void* stream) {
    if (!ctx) return fail(ANELM_ERR_INVALID_ARG, "null context");
    if (polls == 0 || polls > tc::kWaitPolls) return fail(ANELM_ERR_INVALID_ARG, "polls must be in [1, %u]", tc::kWaitPolls);
    DeviceGuard dg(ctx->device);
    bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(ctx->err, polls);
    CUDA_TRY(cudaGetLastError());
    return ANELM_OK;
}

// ---- op level (core/cpu_ops.h) ----

ANELM_API int anelm_gqa_attention(float* out, const float* q, const void* k_cache, const void* v_cache, int kv_dtype,
                                  int n_heads, int n_kv_heads, int head_dim, int q_head_stride, int cache_start,
                                  int cache_len, int cache_capacity, void* stream) {
    if (!out || !q || !k_cache || !v_cache) return fail(ANELM_ERR_INVALID_ARG, "null tensor");
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || q_head_stride < head_dim)
        return fail(ANELM_ERR_INVALID_ARG, "bad head configuration");
    if (cache_capacity <= 0 || cache_len > cache_capacity || cache_start < 0 || cache_start >= cache_capacity)
        return fail(ANELM_ERR_CAPACITY, "start %d / len %d outside capacity %d", cache_start, cache_len, cache_capacity);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cache_len <= 0) {  // cpu_ops.cpp:152-155
        CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)n_heads * head_dim * 4, st));
        return ANELM_OK;
    }
    if (kv_dtype == ANELM_F32) {
        if (cache_len > kMaxLenF32) return fail(ANELM_ERR_UNSUPPORTED, "fp32 cache longer than %d", kMaxLenF32);
        return launch_status(op_gqa_f32(out, q, (const float*)k_cache, (const float*)v_cache, n_heads, n_kv_heads,
                                        head_dim, q_head_stride, cache_start, cache_len, cache_capacity, st),
                             "gqa_attention");
    }
    if (kv_dtype != ANELM_F16) return fail(ANELM_ERR_UNSUPPORTED, "kv dtype %d", kv_dtype);
    if ((head_dim != 128 && head_dim != 256) || n_heads / n_kv_heads > 4)
        return fail(ANELM_ERR_UNSUPPORTED, "fp16 cache needs head_dim 128/256 and <= 4 heads per kv head");
    // Split plan for a single sequence; scratch comes from the stream-ordered pool
    // (the reference mallocs its score buffer per call, cpu_ops.cpp:165).
    const int CH = std::max(64, std::min(4096, ((cache_len * n_kv_heads / (148 * 2) + 63) / 64) * 64));
    const int ns = (cache_len + CH - 1) / CH;
    if (ns > fa_decode_max_splits(head_dim)) return fail(ANELM_ERR_UNSUPPORTED, "too many splits (%d)", ns);
    const size_t words = (size_t)2 * ns + 2 + (size_t)n_kv_heads + 1;
    const size_t part_o = (size_t)ns * n_kv_heads * 4 * head_dim, part_ml = (size_t)ns * n_kv_heads * 8;
    void* ws = nullptr;
    const size_t bytes = (part_o + part_ml) * 4 + words * 8;
    CUDA_TRY(cudaMallocAsync(&ws, bytes, st));
    float* po = static_cast<float*>(ws);
    float* pml = po + part_o;
    int* iw = reinterpret_cast<int*>(pml + part_ml);
    std::vector<int> host((size_t)2 * ns + 2 + n_kv_heads + 1, 0);
    for (int s = 0; s < ns; s++) {
        host[s] = 0;        // blk_b
        host[ns + s] = s;   // blk_split
    }
    host[2 * ns] = ns;      // nsplit
    // part_off (long long) needs 8-byte alignment: place it after the ints
    long long* ploff = reinterpret_cast<long long*>(iw + ((2 * ns + 2 + n_kv_heads + 1 + 1) & ~1));
    cudaError_t e = cudaMemcpyAsync(iw, host.data(), host.size() * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ploff, 0, 8, st);
    if (e != cudaSuccess) {
        cudaFreeAsync(ws, st);
        return fail(ANELM_ERR_CUDA, "workspace setup: %s", cudaGetErrorString(e));
    }
    FaDecodeParams p{};
    p.Hq = n_heads;
    p.Hkv = n_kv_heads;
    p.rot_dim = 0;
    p.scale = 1.0f / sqrtf((float)head_dim);
    p.append = 0;
    p.k_pool = (__half*)k_cache;
    p.v_pool = (__half*)v_cache;
    p.cap_s = cache_capacity;
    p.len_s = cache_len;
    p.start_s = cache_start;
    p.proj = q;
    p.proj_dtype = ANELM_F32;
    p.proj_stride = 0;
    p.q_head_stride = q_head_stride;
    p.out = out;
    p.out_dtype = ANELM_F32;
    p.out_stride = 0;
    p.blk_b = iw;
    p.blk_split = iw + ns;
    p.nsplit = iw + 2 * ns;
    p.cnt_head = iw + 2 * ns + 2;
    p.cnt_seq = iw + 2 * ns + 2 + n_kv_heads;
    p.part_off = ploff;
    p.CH = CH;
    p.part_o = po;
    p.part_ml = pml;
    int rc = launch_fa_decode(p, head_dim, ns, st);
    cudaFreeAsync(ws, st);
    return launch_status(rc, "gqa_attention");
}

ANELM_API int anelm_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc,
                              int c_dtype, int M, int N, int K, void* stream) {
    if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || c_dtype < ANELM_F32 || c_dtype > ANELM_BF16)
        return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(launch_gemm_bf16_tn(A, lda, B, ldb, C, ldc, c_dtype, M, N, K, nullptr,
                                             static_cast<cudaStream_t>(stream)),
                         "gemm_bf16");
}

ANELM_API size_t anelm_lm_head_topk_workspace_bytes(int n, int vocab) {
    return (n > 0 && vocab > 0) ? lm_head_topk_workspace_bytes(n, vocab) : 0;
}

ANELM_API int anelm_lm_head_topk(const void* h, long long ldh, const void* W, long long ldw, int n, int vocab,
                                 int hidden, int k, float* top_vals, int* top_idx, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (!h || !W || !top_vals || !top_idx || !workspace || n <= 0 || vocab <= 0 || hidden <= 0 || k < 1 || k > 32 ||
        k > vocab)
        return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    if (workspace_bytes < lm_head_topk_workspace_bytes(n, vocab))
        return fail(ANELM_ERR_CAPACITY, "workspace of %zu bytes, %zu needed", workspace_bytes,
                    lm_head_topk_workspace_bytes(n, vocab));
    return launch_status(launch_lm_head_topk(h, ldh, W, ldw, n, vocab, hidden, k, top_vals, top_idx, workspace,
                                             workspace_bytes, nullptr, static_cast<cudaStream_t>(stream)),
                         "lm_head_topk");
}

ANELM_API int anelm_ssm_step(float* y, float* state, const float* q, const float* k, const float* v, float decay,
                             float beta, int key_dim, int value_dim, void* stream) {
    if (!y || !state || !q || !k || !v || key_dim <= 0 || value_dim <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_ssm_step(y, state, q, k, v, decay, beta, key_dim, value_dim, (cudaStream_t)stream), "ssm_step");
}

ANELM_API int anelm_conv1d_update(float* y, float* conv_state, int* state_pos, const float* x, const float* w,
                                  int channels, int kernel_size, void* stream) {
    if (!y || !conv_state || !state_pos || !x || !w || channels <= 0 || kernel_size < 2)
        return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    if (*state_pos < 0 || *state_pos >= kernel_size - 1)
        return fail(ANELM_ERR_INVALID_ARG, "state_pos %d outside [0,%d)", *state_pos, kernel_size - 1);
    int rc = op_conv1d(y, conv_state, *state_pos, x, w, channels, kernel_size, (cudaStream_t)stream);
    if (rc) return launch_status(rc, "conv1d_update");
    int pos = *state_pos + 1;  // cpu_ops.cpp:126-128
    if (pos == kernel_size - 1) pos = 0;
    *state_pos = pos;
    return ANELM_OK;
}

ANELM_API int anelm_rmsnorm(float* out, const float* x, const float* w, int dim, float eps, int rows, void* stream) {
    if (!out || !x || !w || dim <= 0 || rows <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_rmsnorm(out, x, w, dim, eps, rows, 0, nullptr, (cudaStream_t)stream), "rmsnorm");
}

ANELM_API int anelm_rmsnorm_gated(float* out, const float* x, const float* z, const float* w, int dim, int rows,
                                  void* stream) {
    if (!out || !x || !z || !w || dim <= 0 || rows <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_rmsnorm(out, x, w, dim, 1e-6f, rows, 1, z, (cudaStream_t)stream), "rmsnorm_gated");
}

ANELM_API int anelm_apply_rope_cached(float* q, float* k, int nq, int nkv, int head_dim, int qs, int ks, int rot,
                                      int pos, float theta, const float* c, const float* s, void* stream) {
    if ((!q && nq > 0) || (!k && nkv > 0) || rot < 0 || rot > head_dim || (rot & 1))
        return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_rope(q, k, nq, nkv, qs, ks, rot, pos, theta, c, s, (cudaStream_t)stream), "apply_rope_cached");
}

ANELM_API int anelm_l2_normalize(float* x, int dim, int rows, void* stream) {
    if (!x || dim <= 0 || rows <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_l2(x, dim, rows, (cudaStream_t)stream), "l2_normalize");
}

ANELM_API int anelm_silu_vec_inplace(float* x, int n, void* stream) {
    if (!x || n < 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    if (n == 0) return ANELM_OK;
    return launch_status(op_sigmoid_mul(x, nullptr, n, (cudaStream_t)stream), "silu_vec_inplace");
}

ANELM_API int anelm_mul_sigmoid_inplace(float* y, const float* z, int n, void* stream) {
    if (!y || !z || n < 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    if (n == 0) return ANELM_OK;
    return launch_status(op_sigmoid_mul(y, z, n, (cudaStream_t)stream), "mul_sigmoid_inplace");
}

ANELM_API int anelm_softmax(float* x, int n, int rows, void* stream) {
    if (!x || n <= 0 || rows <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_softmax(x, n, rows, (cudaStream_t)stream), "softmax");
}

ANELM_API int anelm_matvec(float* y, const float* W, const float* x, int out_dim, int in_dim, void* stream) {
    if (!y || !W || !x || out_dim <= 0 || in_dim <= 0) return fail(ANELM_ERR_INVALID_ARG, "bad argument");
    return launch_status(op_matvec(y, W, x, out_dim, in_dim, (cudaStream_t)stream), "matvec");
}

}  // extern "C"
