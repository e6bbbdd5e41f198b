// f32x2.cuh -- packed fp32 pairs (sm_100 f32x2 arithmetic) and 16-byte units of bf16 / f32 as pairs.
// Shared by the RMSNorm and tensor-parallel AllReduce+RMSNorm kernels.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

namespace dsb2 {

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction per two lanes of math, IEEE fp32 rounding
// per element, so results equal the scalar fp32 ones).
using f2x = unsigned long long;
__device__ __forceinline__ f2x f2_make(float lo, float hi) {
    f2x d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ float2 f2_split(f2x v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ f2x f2_mul(f2x a, f2x b) {
    f2x d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2x f2_fma(f2x a, f2x b, f2x c) {
    f2x d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f2x f2_add(f2x a, f2x b) {
    f2x d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// A 16-byte unit of elements as kPairs fp32 pairs.
template <typename T>
struct RmsElem;
template <>
struct RmsElem<__nv_bfloat16> {
    static constexpr int kPairs = 4;
    static __device__ __forceinline__ void unpack(uint4 p, f2x* f) {   // bf16 -> f32 is a 16-bit shift
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) f[k] = f2_make(__uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xffff0000u));
    }
    static __device__ __forceinline__ uint4 pack(const f2x* f) {   // round to nearest even, two per cvt
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = f2_split(f[k]);
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w[k]) : "f"(v.y), "f"(v.x));
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct RmsElem<float> {
    static constexpr int kPairs = 2;
    static __device__ __forceinline__ void unpack(uint4 p, f2x* f) {
        f[0] = f2_make(__uint_as_float(p.x), __uint_as_float(p.y));
        f[1] = f2_make(__uint_as_float(p.z), __uint_as_float(p.w));
    }
    static __device__ __forceinline__ uint4 pack(const f2x* f) {
        const float2 a = f2_split(f[0]), b = f2_split(f[1]);
        return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x), __float_as_uint(b.y));
    }
};

}  // namespace dsb2
