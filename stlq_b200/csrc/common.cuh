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

// K-block split of the reference's CPU BLAS (OpenBLAS 0.3.15 SkylakeX SGEMM, single thread): blocks
// of 448, a remainder in (448, 896) halved and rounded up to 16.  Every block length is a multiple
// of 4 when d is.
__host__ __device__ __forceinline__ int NextKBlock(int rem) {
    const int Q = 448, U = 16;
    if (rem >= 2 * Q) return Q;
    if (rem > Q) return ((rem / 2) + U - 1) & ~(U - 1);
    return rem;
}

// One xC entry c . x exactly as the exact GEMM (XcGemmExactKernel) computes it: per K block an
// FMA chain from zero, folded as t = fma(1, chain, t) from t = 0 in block order.  d % 4 == 0 and
// the codeword row 16-byte aligned.  x is float or uint8 (converted exactly); with kVecX it is read
// four at a time (a 16-byte aligned float row: the beam kernels' staged copy), otherwise one
// element at a time (a caller's row, whatever its alignment).
template <bool kVecX>
__device__ __forceinline__ float4 Load4(const float* p) {
    if constexpr (kVecX) return *reinterpret_cast<const float4*>(p);
    else return make_float4(p[0], p[1], p[2], p[3]);
}
template <bool kVecX>
__device__ __forceinline__ float4 Load4(const uint8_t* p) {
    return make_float4(p[0], p[1], p[2], p[3]);
}
template <typename TX, bool kVecX = false>
__device__ __noinline__ float ExactDot(const float* __restrict__ c, const TX* __restrict__ x, int d) {
    float t = 0.0f;
    for (int k0 = 0; k0 < d;) {
        const int kb = NextKBlock(d - k0);
        float acc = 0.0f;
#pragma unroll 8
        for (int i = k0; i < k0 + kb; i += 4) {
            const float4 cv = __ldg(reinterpret_cast<const float4*>(c + i));
            const float4 xv = Load4<kVecX>(x + i);
            acc = __fmaf_rn(cv.x, xv.x, acc);
            acc = __fmaf_rn(cv.y, xv.y, acc);
            acc = __fmaf_rn(cv.z, xv.z, acc);
            acc = __fmaf_rn(cv.w, xv.w, acc);
        }
        t = __fmaf_rn(1.0f, acc, t);
        k0 += kb;
    }
    return t;
}

// ExactDot for R codeword rows at once (rows[r], results out[r]): R independent chains advanced
// together, each exactly ExactDot's sequence.  x read one element at a time (any alignment).
template <int R, typename TX>
__device__ __noinline__ void ExactDotRows(const float* const (&rows)[R], const TX* __restrict__ x, int d, float (&out)[R]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
        for (int i = 0; i < d; i += 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(rows[r] + i));
    float t[R];
#pragma unroll
    for (int r = 0; r < R; ++r) t[r] = 0.0f;
    for (int k0 = 0; k0 < d;) {
        const int kb = NextKBlock(d - k0);
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll 2
        for (int i = k0; i < k0 + kb; i += 4) {
            const float4 xv = Load4<false>(x + i);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float4 cv = __ldg(reinterpret_cast<const float4*>(rows[r] + i));
                acc[r] = __fmaf_rn(cv.x, xv.x, acc[r]);
                acc[r] = __fmaf_rn(cv.y, xv.y, acc[r]);
                acc[r] = __fmaf_rn(cv.z, xv.z, acc[r]);
                acc[r] = __fmaf_rn(cv.w, xv.w, acc[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) t[r] = __fmaf_rn(1.0f, acc[r], t[r]);
        k0 += kb;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = t[r];
}

// STRICT mode: xC comes from the tensor cores (3xTF32), which differ from the exact GEMM's entries
// by at most kappa * ||c_h|| * ||x||.  Decisions are bounded from the tensor-core values and every
// value a decision or an output depends on is recomputed with ExactDot, so codes, coefficients and
// costs equal the exact mode's.  The bound is checked on every entry computed exactly:
// CheckTcBound sets kErrTcBound when |g - ga| exceeds dg (both values finite).
__device__ __forceinline__ void CheckTcBound(float g, float ga, float dg, unsigned int* err) {
    if (isfinite(g) && isfinite(ga) && !(fabsf(g - ga) <= dg)) atomicOr(err, kErrTcBound);
}

// Per vector, in the beam kernels: x staged as float in shared memory.
struct ExactCtx {
    const float* C;      // codeword rows (H x d)
    const float* cn;     // upper bounds of ||c_h||
    const float* xc;     // the vector's tensor-core xC row
    const float* xs;     // the vector, float, 16-byte aligned (shared memory)
    int d;
    float kx;            // kappa * (upper bound of ||x||)
    unsigned int* err;
    __device__ float Bound(int flat) const { return kx * __ldg(cn + flat); }
    __device__ float Gamma(int flat) const {
        const float g = ExactDot<float, true>(C + static_cast<size_t>(flat) * d, xs, d);
        CheckTcBound(g, xc[flat], Bound(flat), err);
        return g;
    }
};

// kx for a vector with float ||x||^2 = nx2 (its square root, rounded up by far more than its
// rounding error).
__device__ __forceinline__ float StrictKx(float kappa, float nx2) { return kappa * sqrtf(fmaxf(nx2, 0.0f)) * 1.0001f; }

}  // namespace stlq_b200
