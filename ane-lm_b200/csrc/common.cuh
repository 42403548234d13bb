// Shared device helpers for the anelm_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "anelm_b200.h"

namespace anelm {

// ---- dtype-generic scalar access -------------------------------------------

__device__ __forceinline__ float load_as_float(const void* p, int dtype, long long i) {
    if (dtype == ANELM_F32) return reinterpret_cast<const float*>(p)[i];
    if (dtype == ANELM_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_float(void* p, int dtype, long long i, float v) {
    if (dtype == ANELM_F32) {
        reinterpret_cast<float*>(p)[i] = v;
    } else if (dtype == ANELM_F16) {
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    } else {
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    }
}

__host__ __device__ __forceinline__ int dtype_bytes(int dtype) { return dtype == ANELM_F32 ? 4 : 2; }

// ---- reductions -------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- reference scalar functions (core/cpu_ops.h:12-14) ------------------------

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_ref(float x) { return logf(1.0f + expf(x)); }

// ---- async copies / tensor-core fragments -----------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte cp.async (L2 only); src_bytes == 0 zero-fills the destination.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
    return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

// 8 consecutive 16-bit values (bf16 or fp16) <-> fp32
__device__ __forceinline__ void unpack8(const uint4 v, bool bf, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 t;
        if (bf) t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        else t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8], bool bf) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (bf) {
            const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&t);
        } else {
            const __half2 t = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&t);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}
// 8 consecutive elements of a dtype row (16-byte aligned: row + e0 * dtype bytes) as fp32
__device__ __forceinline__ void load8(const char* row, int dtype, long long e0, float (&x)[8]) {
    if (dtype == ANELM_F32) {
        const float4 a = *reinterpret_cast<const float4*>(row + e0 * 4);
        const float4 c = *reinterpret_cast<const float4*>(row + e0 * 4 + 16);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
    } else {
        unpack8(*reinterpret_cast<const uint4*>(row + e0 * 2), dtype == ANELM_BF16, x);
    }
}

// Loads that bypass L1 (data written by other CTAs of the same launch).
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

}  // namespace anelm
