// Packed fp32 pairs for the bit-exact SIMT kernels.
#pragma once

#include <cstdint>

namespace eb {

// Packed pairs of fp32 (element 0 in the low half): sm_100's f32x2 add and
// sub round each element exactly as the scalar .rn instructions do, so a pair
// of independent sequential chains advances with one instruction per step
// instead of two. Products are NOT formed with the packed multiply: the
// compiler contracts a packed mul.rn followed by a packed add.rn into a fused
// multiply-add (measured: the sums then differ in the last bit), whereas a
// scalar mul.rn is never contracted. f2_prod therefore multiplies each
// element with scalar mul.rn and packs the two products.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_prod(unsigned long long a, unsigned long long b) {
    float a0, a1, b0, b1;
    f2_unpack(a, a0, a1);
    f2_unpack(b, b0, b1);
    return f2_pack(__fmul_rn(a0, b0), __fmul_rn(a1, b1));
}

}  // namespace eb
