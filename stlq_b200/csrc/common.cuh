// Shared device helpers for the stlq_b200 kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "types.h"

namespace stlq_b200 {

// Monotone map from float to uint32 so that unsigned order equals float order (-inf < ... < +inf).
// Codes are stored as uint8 or, for codebooks above 256 codewords, uint16.
__device__ __forceinline__ int LoadCode(const void* B, int64_t i, int wide) {
    return wide ? static_cast<const uint16_t*>(B)[i] : static_cast<const uint8_t*>(B)[i];
}
__device__ __forceinline__ void StoreCode(void* B, int64_t i, int code, int wide) {
    if (wide) static_cast<uint16_t*>(B)[i] = static_cast<uint16_t>(code);
    else static_cast<uint8_t*>(B)[i] = static_cast<uint8_t>(code);
}

__device__ __forceinline__ uint32_t OrderKey(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float KeyToFloat(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// Round-to-nearest float ops that nvcc may not contract into FMA: the reference's host code is
// built for the x86-64 baseline ISA, so every a*b+c there rounds twice.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }

}  // namespace stlq_b200
