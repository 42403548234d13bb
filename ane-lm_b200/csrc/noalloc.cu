// anelm_gqa_attention_noalloc: the fp16-cache gqa_attention entry point without
// any device allocation.
//
// Who needs it: hosts that cannot call cudaMalloc / cudaMallocAsync at the point
// where attention runs -- for example an inference server that hands all free
// HBM to its own KV-block pool at start-up (a later allocation fails or
// fragments that pool), or a plugin host that owns the device allocator and
// forbids plugins from allocating on their own.  anelm_gqa_attention takes its
// split-K scratch from the stream-ordered pool on every call; this variant uses
// the file-scope device array below instead.
//
// The array is part of the library image: every GPU that loads the library
// keeps ANELM_GQA_NOALLOC_SCRATCH_BYTES of device memory for it until the
// process exits.  All calls on a device share it and it keeps the previous
// call's contents, so the counters that must start at zero are cleared on every
// call, and calls whose executions overlap on the GPU (different streams,
// nothing ordering them) race on it.
//
// Host code must not pass the array's name to a kernel: on the host it is only
// a stand-in symbol.  The device address is fetched with cudaGetSymbolAddress on
// the first call made while a device is current; make that first call before any
// stream capture.  The address is cached per device together with the CUDA
// context that was current: after a device reset (a new primary context, in which
// the library's module and the array are loaded again) the next call looks the
// address up again instead of writing through a stale pointer.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "anelm_b200.h"
#include "kernels.h"

using namespace anelm;

namespace {

static __device__ __align__(256) unsigned char g_gqa_scratch[ANELM_GQA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_dev[kMaxDevices] = {nullptr};
CUcontext g_scratch_ctx[kMaxDevices] = {nullptr};

// cuCtxGetCurrent through the runtime's driver entry point (the library links no libcuda).
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(f);
    }();
    return fn;
}

int noalloc_fail(int code, const char* msg) {
    set_last_error(msg);
    return code;
}

// Writes the single-sequence split table and zeroes the merge counters inside the scratch.
__global__ void noalloc_tables_kernel(int* blk_b, int* blk_split, int* nsplit, long long* part_off, int* counters,
                                      int ns, int n_counters) {
    for (int i = threadIdx.x; i < ns; i += blockDim.x) {
        blk_b[i] = 0;
        blk_split[i] = i;
    }
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;
    if (threadIdx.x == 0) {
        nsplit[0] = ns;
        part_off[0] = 0;
    }
}

int scratch_for_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return noalloc_fail(ANELM_ERR_CUDA, "no current CUDA device");
    // A cached address is used only while the context it was taken in is still the current one.
    CUcontext cur = nullptr;
    CtxGetCurrentFn get = ctx_get_current();
    std::lock_guard<std::mutex> lk(g_mu);
    if (get && g_scratch_dev[dev] && (get(&cur) != CUDA_SUCCESS || cur != g_scratch_ctx[dev]))
        g_scratch_dev[dev] = nullptr;  // another context than the one the address was taken in
    if (!g_scratch_dev[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_gqa_scratch);
        if (e != cudaSuccess || !p) {
            set_last_error((std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e)).c_str());
            return ANELM_ERR_CUDA;
        }
        cur = nullptr;
        if (get && get(&cur) != CUDA_SUCCESS) cur = nullptr;
        g_scratch_dev[dev] = p;
        g_scratch_ctx[dev] = cur;
    }
    *out = g_scratch_dev[dev];
    return ANELM_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

extern "C" {

ANELM_API int anelm_gqa_attention_noalloc(float* out, const float* q, const void* k_cache, const void* v_cache,
                                          int n_heads, int n_kv_heads, int head_dim, int q_head_stride,
                                          int cache_start, int cache_len, int cache_capacity, void* stream) {
    if (!out || !q || !k_cache || !v_cache) return noalloc_fail(ANELM_ERR_INVALID_ARG, "null tensor");
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || q_head_stride < head_dim)
        return noalloc_fail(ANELM_ERR_INVALID_ARG, "bad head configuration");
    if ((head_dim != 128 && head_dim != 256) || n_heads / n_kv_heads > 4)
        return noalloc_fail(ANELM_ERR_UNSUPPORTED, "needs head_dim 128/256 and <= 4 heads per kv head");
    if (cache_capacity <= 0 || cache_len > cache_capacity || cache_start < 0 || cache_start >= cache_capacity)
        return noalloc_fail(ANELM_ERR_CAPACITY, "start / len outside the cache capacity");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cache_len <= 0) {  // core/cpu_ops.cpp:152-155
        if (cudaMemsetAsync(out, 0, (size_t)n_heads * head_dim * sizeof(float), st) != cudaSuccess)
            return noalloc_fail(ANELM_ERR_CUDA, "cudaMemsetAsync failed");
        return ANELM_OK;
    }
    // Split plan: as many splits as the scratch holds, but never fewer than 64 tokens each.
    const size_t per_split = (size_t)n_kv_heads * (4 * head_dim + 8) * sizeof(float);
    const size_t fixed = 16384;  // tables and counters region, see layout below
    const size_t budget = ANELM_GQA_NOALLOC_SCRATCH_BYTES - fixed;
    const int max_ns = (int)std::min<size_t>(budget / per_split, (size_t)fa_decode_max_splits(head_dim));
    if (max_ns < 1)
        return noalloc_fail(ANELM_ERR_CAPACITY, "one split of this head configuration exceeds the static scratch");
    int CH = (int)std::max(64LL, std::min(4096LL, (((long long)cache_len * n_kv_heads / (148 * 2) + 63) / 64) * 64));
    int ns = (cache_len + CH - 1) / CH;
    if (ns > max_ns) {
        CH = (int)((((long long)cache_len + max_ns - 1) / max_ns + 63) / 64 * 64);
        ns = (cache_len + CH - 1) / CH;
    }
    const int n_counters = n_kv_heads + 1;
    if (ns > max_ns || (size_t)(2 * ns + 2 + n_counters) * sizeof(int) + 16 > fixed)
        return noalloc_fail(ANELM_ERR_CAPACITY, "cache too long for the static scratch of this entry point");

    void* base = nullptr;
    if (int rc = scratch_for_current_device(&base)) return rc;
    // layout: [fixed: part_off (8 B) | blk_b | blk_split | nsplit | counters] [part_o] [part_ml]
    char* b = static_cast<char*>(base);
    long long* part_off = reinterpret_cast<long long*>(b);
    int* blk_b = reinterpret_cast<int*>(b + 16);
    int* blk_split = blk_b + ns;
    int* nsplit = blk_split + ns;
    int* counters = nsplit + 1;
    float* part_o = reinterpret_cast<float*>(b + fixed);
    float* part_ml = part_o + (size_t)ns * n_kv_heads * 4 * head_dim;
    if (align_up((size_t)((char*)(part_ml + (size_t)ns * n_kv_heads * 8) - b), 16) > ANELM_GQA_NOALLOC_SCRATCH_BYTES)
        return noalloc_fail(ANELM_ERR_CAPACITY, "static scratch overflow");

    noalloc_tables_kernel<<<1, 256, 0, st>>>(blk_b, blk_split, nsplit, part_off, counters, ns, n_counters);
    if (cudaGetLastError() != cudaSuccess) return noalloc_fail(ANELM_ERR_CUDA, "table kernel launch failed");

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
    p.q_head_stride = q_head_stride;
    p.out = out;
    p.out_dtype = ANELM_F32;
    p.blk_b = blk_b;
    p.blk_split = blk_split;
    p.nsplit = nsplit;
    p.part_off = part_off;
    p.CH = CH;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.cnt_head = counters;
    p.cnt_seq = counters + n_kv_heads;
    const int rc = launch_fa_decode(p, head_dim, ns, st);
    if (rc != ANELM_OK) return noalloc_fail(rc, "attention kernel launch failed");
    return ANELM_OK;
}

}  // extern "C"
