// kcommon.cuh -- device helpers shared by the sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace s2b {

typedef __nv_bfloat16 bf16;
typedef __half f16;

template <typename T> struct Cvt;
template <> struct Cvt<float> {
    static __device__ __forceinline__ float to_f(float x) { return x; }
    static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Cvt<bf16> {
    static __device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ bf16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Cvt<f16> {
    static __device__ __forceinline__ float to_f(f16 x) { return __half2float(x); }
    static __device__ __forceinline__ f16 from_f(float x) { return __float2half_rn(x); }
};

// Load 4 consecutive elements as floats (16-byte / 8-byte aligned rows).
__device__ __forceinline__ void load4(const float* p, float v[4]) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
__device__ __forceinline__ void load4(const bf16* p, float v[4]) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
    const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
__device__ __forceinline__ void load4(const f16* p, float v[4]) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
    v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
__device__ __forceinline__ void store4(float* p, const float v[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(bf16* p, const float v[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
}

__device__ __forceinline__ void store4(f16* p, const float v[4]) {
    __half2 a = __floats2half2_rn(v[0], v[1]);
    __half2 b = __floats2half2_rn(v[2], v[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
}

__device__ __forceinline__ float warp_sum(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// x / (1 + exp(-x)), the reference's SiLU (src/dit_vk.cpp:53).
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.f, expf(-x))); }

}  // namespace s2b
