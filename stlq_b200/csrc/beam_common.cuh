// Device code shared by the two beam-search kernels of beam.cu.
//
// Reference: BeamSearchPrefixLS, src/quantizer/beam_search.cpp:196-422.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace stlq_b200 {
namespace beam {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kCpt = kMaxK / kThreads;  // codewords per thread
constexpr unsigned kFull = 0xffffffffu;
// A slot whose last pivot satisfies R_LL^2 < kIllCond * G(c,c) (its codeword nearly in the span
// of the earlier ones) evaluates all its candidates exactly; so does a candidate whose cheap
// denominator falls below kDenomGuard * alpha.
constexpr float kIllCond = 1e-4f;
constexpr float kDenomGuard = 1e-3f;

__device__ __forceinline__ float PosInf() { return __int_as_float(0x7f800000); }

// Beam slots in dynamic shared memory, sized by the runtime beam width.
template <int MAXM>
struct SlotView {
    float* R;     // [beam][MAXM*MAXM] upper Cholesky factor, row-major R[r*MAXM + c], r <= c
    float* rinv;  // [beam][MAXM] 1/R_ii (cheap bound only)
    float* a;     // [beam][MAXM]
    float* E;     // [beam]
    int* code;    // [beam][MAXM]
    int* ill;     // [beam] 1 when any pivot was ill-conditioned
    __device__ float* Rh(int h) const { return R + h * MAXM * MAXM; }
    __device__ float* rinvh(int h) const { return rinv + h * MAXM; }
    __device__ float* ah(int h) const { return a + h * MAXM; }
    __device__ int* codeh(int h) const { return code + h * MAXM; }
    __host__ __device__ static constexpr size_t Bytes(int beam) {
        return sizeof(float) * static_cast<size_t>(beam) * (MAXM * MAXM + 2 * MAXM + 1) +
               sizeof(int) * static_cast<size_t>(beam) * (MAXM + 1);
    }
    __device__ static SlotView At(unsigned char* p, int beam) {
        SlotView v;
        v.R = reinterpret_cast<float*>(p);
        v.rinv = v.R + beam * MAXM * MAXM;
        v.a = v.rinv + beam * MAXM;
        v.E = v.a + beam * MAXM;
        v.code = reinterpret_cast<int*>(v.E + beam);
        v.ill = v.code + beam * MAXM;
        return v;
    }
};

// Flat codeword indices of slot h's prefix (passed by value so they stay in registers).
template <int MAXM>
struct FlatArr {
    int v[MAXM];
};

template <int MAXM, int L>
__device__ __forceinline__ FlatArr<MAXM> FlatOf(const Dims& dims, const SlotView<MAXM>& cur, int h) {
    FlatArr<MAXM> f;
#pragma unroll
    for (int t = 0; t < MAXM; ++t) f.v[t] = t < L ? dims.off[t] + cur.codeh(h)[t] : 0;
    return f;
}

// Exact candidate evaluation for slot h at layer L, in the reference's float operation sequence
// (SolveCholUpperRawFixed forward and back substitution, beam_search.cpp:127-162; delta = A.v and
// eta = A.a_old, :299-305; denom, a_last, e with the clamp at 0, :307-318).  Returns the error,
// +inf for a candidate the reference skips (denom == 0) or that can never enter the beam
// (e >= +inf or NaN, :320).  Optionally returns y, v, denom and a_last for materialisation.
// Kept out of line: several call sites share one copy, which keeps the kernels' code small.
template <int MAXM, int L>
__device__ __noinline__ float EvalExact(const SlotView<MAXM> cur, int h, const FlatArr<MAXM> flat,
                                        const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                        float* y_out, float* v_out, float* denom_out, float* alast_out) {
    const float* Rh = cur.Rh(h);
    const float* ah = cur.ah(h);
    float A[L], y[L], v[L];
#pragma unroll
    for (int t = 0; t < L; ++t) A[t] = __ldg(Grow + static_cast<size_t>(flat.v[t]) * H + col);
#pragma unroll
    for (int i = 0; i < L; ++i) {
        float s = A[i];
#pragma unroll
        for (int k = 0; k < i; ++k) s = sub_rn(s, mul_rn(Rh[k * MAXM + i], y[k]));
        y[i] = div_rn(s, Rh[i * MAXM + i]);
    }
#pragma unroll
    for (int i = L - 1; i >= 0; --i) {
        float s = y[i];
#pragma unroll
        for (int k = i + 1; k < L; ++k) s = sub_rn(s, mul_rn(Rh[i * MAXM + k], v[k]));
        v[i] = div_rn(s, Rh[i * MAXM + i]);
    }
    float delta = 0.0f, eta = 0.0f;
#pragma unroll
    for (int t = 0; t < L; ++t) {
        delta = add_rn(delta, mul_rn(A[t], v[t]));
        eta = add_rn(eta, mul_rn(A[t], ah[t]));
    }
    const float denom = sub_rn(alpha, delta);
    const float diff = sub_rn(gamma, eta);
    const float a_last = div_rn(diff, denom);
    float e = sub_rn(cur.E[h], mul_rn(diff, a_last));
    if (e < 0.0f) e = 0.0f;
    if (y_out) {
#pragma unroll
        for (int t = 0; t < L; ++t) {
            y_out[t] = y[t];
            v_out[t] = v[t];
        }
        *denom_out = denom;
        *alast_out = a_last;
    }
    return (denom != 0.0f && e < PosInf()) ? e : PosInf();
}

// Cheap bounds [lo, hi] on a candidate's exact error.
// e' = E_old - diff^2/denom with y from FMA forward substitution, delta = |y|^2, eta = A.a.  The
// half-width covers the rounding of both this and the exact sequence: relative errors of order
// L ulp in diff (scale |gamma| + sum|A_t a_t|) and in denom (scale alpha + delta), propagated
// through r = diff^2/denom, plus the final subtraction; kept with a factor 16.  A candidate
// whose cheap value is unreliable (ill-conditioned slot, denom <= kDenomGuard * alpha, NaN)
// gets [-inf, +inf].
template <int MAXM, int L>
__device__ __forceinline__ void CheapBounds(const SlotView<MAXM>& cur, int h, const FlatArr<MAXM>& flat,
                                            const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                            float* lo, float* hi) {
    const float* Rh = cur.Rh(h);
    const float* rinv = cur.rinvh(h);
    const float* ah = cur.ah(h);
    float A[L], y[L];
#pragma unroll
    for (int t = 0; t < L; ++t) A[t] = __ldg(Grow + static_cast<size_t>(flat.v[t]) * H + col);
    float delta = 0.0f, eta = 0.0f, seta = fabsf(gamma);
#pragma unroll
    for (int i = 0; i < L; ++i) {
        float s = A[i];
#pragma unroll
        for (int k = 0; k < i; ++k) s = fmaf(-Rh[k * MAXM + i], y[k], s);
        y[i] = s * rinv[i];
        delta = fmaf(y[i], y[i], delta);
        const float p = A[i] * ah[i];
        eta += p;
        seta += fabsf(p);
    }
    const float denom = alpha - delta;
    const float diff = gamma - eta;
    const float rden = __fdividef(1.0f, denom);  // approximate: only bounds depend on it
    const float r = diff * diff * rden;
    const float Eo = cur.E[h];
    const float ep = fmaxf(Eo - r, 0.0f);
    constexpr float u = 1.2e-7f * (L + 2);
    const float de = (2.0f * fabsf(diff) * (u * seta) + fabsf(r) * (u * (alpha + delta))) * fabsf(rden) +
                     1.2e-7f * (Eo + fabsf(r));
    const float w = 16.0f * de;
    const bool force = cur.ill[h] || !(denom > kDenomGuard * alpha) || !(w < PosInf()) || !(ep < PosInf());
    *lo = force ? -PosInf() : ep - w;
    *hi = force ? PosInf() : ep + w;
}

}  // namespace beam
}  // namespace stlq_b200
