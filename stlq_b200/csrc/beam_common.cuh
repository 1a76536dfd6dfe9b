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

// The beam's diagonal marks a codeword of codebooks 1..m-1 whose Gram column is exactly zero
// (a zero codeword) with alpha = -0.0f.  Every prefix then has A = 0, so y, v and delta are 0 and
// denom = alpha - delta == 0: the reference skips the candidate (beam_search.cpp:309), in every
// slot.  -0.0f and +0.0f take the same branch in every comparison the reference makes.
__device__ __forceinline__ bool IsZeroColumn(float alpha) { return __float_as_uint(alpha) == 0x80000000u; }

// Beam slots in dynamic shared memory, sized by the runtime beam width.
template <int MAXM>
struct SlotView {
    float* R;     // [beam][MAXM*MAXM] upper Cholesky factor by columns: R(r, c) at [c*MAXM + r], r <= c
    float* rinv;  // [beam][MAXM] 1/R_ii (cheap bound only)
    float* a;     // [beam][MAXM]
    float* E;     // [beam]
    int* row;     // [beam][MAXM] row of each prefix codeword in Grow: (layer offset + code) * H
    int* ill;     // [beam] 1 when any pivot was ill-conditioned
    __device__ float* Rh(int h) const { return R + h * MAXM * MAXM; }
    __device__ float* rinvh(int h) const { return rinv + h * MAXM; }
    __device__ float* ah(int h) const { return a + h * MAXM; }
    __device__ int* rowh(int h) const { return row + h * MAXM; }
    // Rounded to 16 bytes: a second buffer placed after the first stays 16-byte aligned.
    __host__ __device__ static constexpr size_t Bytes(int beam) {
        return (sizeof(float) * static_cast<size_t>(beam) * (MAXM * MAXM + 2 * MAXM + 1) +
                sizeof(int) * static_cast<size_t>(beam) * (MAXM + 1) + 15) &
               ~static_cast<size_t>(15);
    }
    __device__ static SlotView At(unsigned char* p, int beam) {
        SlotView v;
        v.R = reinterpret_cast<float*>(p);
        v.rinv = v.R + beam * MAXM * MAXM;
        v.a = v.rinv + beam * MAXM;
        v.row = reinterpret_cast<int*>(v.a + beam * MAXM);  // 16-byte aligned per slot (int4 loads)
        v.E = reinterpret_cast<float*>(v.row + beam * MAXM);
        v.ill = reinterpret_cast<int*>(v.E + beam);
        return v;
    }
};

// The kernels take the layer index L (1 <= L < m <= MAXM) at run time: one copy of each routine
// serves every layer.  Per-layer copies (L as a template parameter) made the kernels several times
// larger than the instruction cache, and instruction fetch became their main stall.  Loops run to
// the compile-time bound NL = MAXM - 1 with warp-uniform guards on L.

// Grow row offsets of slot h's prefix codewords (passed by value so they stay in registers).
template <int MAXM>
struct RowArr {
    int v[MAXM];
};

template <int MAXM>
__device__ __forceinline__ RowArr<MAXM> RowsOf(const SlotView<MAXM>& cur, int h, int L) {
    RowArr<MAXM> f;
#pragma unroll
    for (int t = 0; t < MAXM; ++t) {
        if (t >= L) break;
        f.v[t] = cur.rowh(h)[t];
    }
    return f;
}

// Exact candidate evaluation for slot h at layer L, in the reference's float operation sequence
// (SolveCholUpperRawFixed forward and back substitution, beam_search.cpp:127-162; delta = A.v and
// eta = A.a_old, :299-305; denom, a_last, e with the clamp at 0, :307-318).  Returns the error,
// +inf for a candidate the reference skips (denom == 0) or that can never enter the beam
// (e >= +inf or NaN, :320).  Optionally returns y, v, denom and a_last for materialisation.
// NL bounds L; with kFixed the layer is NL itself (a per-layer copy).  With `recip` (large-root
// encoders) both substitutions multiply by the float reciprocal 1/R_ii, held in the slot as rinv,
// as BeamSearchPrefixLSLargeRoot's SolveCholUpperRawBatched does (beam_search.cpp:517-575).
template <int MAXM, int NL, bool kFixed>
__device__ __noinline__ float EvalExact(const SlotView<MAXM> cur, int h, int Lrt, const RowArr<MAXM> flat,
                                        const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                        float* y_out, float* v_out, float* denom_out, float* alast_out, bool recip) {
    const int L = kFixed ? NL : Lrt;
    const float* Rh = cur.Rh(h);
    const float* rinv = cur.rinvh(h);
    const float* ah = cur.ah(h);
    float A[NL], y[NL], v[NL];
#pragma unroll
    for (int t = 0; t < NL; ++t) {
        if (t >= L) break;
        A[t] = __ldg(Grow + flat.v[t] + col);
    }
#pragma unroll
    for (int i = 0; i < NL; ++i) {
        if (i >= L) break;
        float s = A[i];
#pragma unroll
        for (int k = 0; k < i; ++k) s = sub_rn(s, mul_rn(Rh[i * MAXM + k], y[k]));
        y[i] = recip ? mul_rn(s, rinv[i]) : div_rn(s, Rh[i * MAXM + i]);
    }
#pragma unroll
    for (int i = NL - 1; i >= 0; --i) {
        if (i >= L) continue;
        float s = y[i];
#pragma unroll
        for (int k = i + 1; k < NL; ++k) {
            if (k >= L) break;
            s = sub_rn(s, mul_rn(Rh[k * MAXM + i], v[k]));
        }
        v[i] = recip ? mul_rn(s, rinv[i]) : div_rn(s, Rh[i * MAXM + i]);
    }
    float delta = 0.0f, eta = 0.0f;
#pragma unroll
    for (int t = 0; t < NL; ++t) {
        if (t >= L) break;
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
        for (int t = 0; t < NL; ++t) {
            if (t >= L) break;
            y_out[t] = y[t];
            v_out[t] = v[t];
        }
        *denom_out = denom;
        *alast_out = a_last;
    }
    return (denom != 0.0f && e < PosInf()) ? e : PosInf();
}

// EvalExact for layer L: one out-of-line copy per layer (each a short dependent chain, fastest with
// its loops fully unrolled; they are called, not inlined, so they stay small next to the cheap
// pass).  In the 16-layer kernel this measured 1.3% faster than two copies with run-time bounds.
template <int MAXM>
__device__ __forceinline__ float EvalExactL(const SlotView<MAXM>& cur, int h, int L, const RowArr<MAXM>& flat,
                                            const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                            float* y_out, float* v_out, float* denom_out, float* alast_out,
                                            bool recip) {
#define STLQ_B200_EXACT(NL) \
    EvalExact<MAXM, NL, true>(cur, h, L, flat, Grow, H, col, alpha, gamma, y_out, v_out, denom_out, alast_out, recip)
#define STLQ_B200_EXACT_CASE(LL)                                     \
    case LL:                                                         \
        if constexpr (LL < MAXM - 1) return STLQ_B200_EXACT(LL);     \
        break;
    switch (L) {
        STLQ_B200_EXACT_CASE(1) STLQ_B200_EXACT_CASE(2) STLQ_B200_EXACT_CASE(3) STLQ_B200_EXACT_CASE(4)
        STLQ_B200_EXACT_CASE(5) STLQ_B200_EXACT_CASE(6) STLQ_B200_EXACT_CASE(7) STLQ_B200_EXACT_CASE(8)
        STLQ_B200_EXACT_CASE(9) STLQ_B200_EXACT_CASE(10) STLQ_B200_EXACT_CASE(11) STLQ_B200_EXACT_CASE(12)
        STLQ_B200_EXACT_CASE(13) STLQ_B200_EXACT_CASE(14)
        default: break;
    }
    return STLQ_B200_EXACT(MAXM - 1);
#undef STLQ_B200_EXACT_CASE
#undef STLQ_B200_EXACT
}

// The error bounds of one candidate from its cheap delta, eta and seta (see CheapBounds).
// lof: the lower bound of a forced candidate: -inf, or +inf for a zero codeword, which is always
// forced (its cheap denominator is -0 - 0) and which the reference always skips.
// kStrict: gamma is a tensor-core value within dg of the exact one, so the exact diff lies within
// dg of this one and e' = E_old - diff^2/denom moves by at most (2|diff| + dg) dg / denom.
template <bool kStrict>
__device__ __forceinline__ void BoundsTail(int L, float alpha, float gamma, float delta, float eta, float seta, float Eo,
                                           bool ill, float dg, float& lo, float& hi) {
    const float lof = IsZeroColumn(alpha) ? PosInf() : -PosInf();  // derived here: one register less per codeword
    // Half-width w = 16 * de with de as documented at CheapBounds; the factor 16 is folded into the
    // constants.
    const float u16 = 16.0f * 1.2e-7f * static_cast<float>(L + 2);
    constexpr float e16 = 16.0f * 1.2e-7f;
    const float denom = alpha - delta;
    const float diff = gamma - eta;
    const float rden = __fdividef(1.0f, denom);  // approximate: only bounds depend on it
    const float r = diff * diff * rden;
    const float ep = fmaxf(Eo - r, 0.0f);
    float w = fmaf(2.0f * fabsf(diff) * seta + fabsf(r) * (alpha + delta), u16 * fabsf(rden), e16 * (Eo + fabsf(r)));
    if constexpr (kStrict) w = fmaf((2.0f * fabsf(diff) + dg) * dg, 1.001f * fabsf(rden), w);
    // One test for both ep and w: their sum is +inf or NaN when either is (ep is never NaN, being a
    // fmaxf); a finite pair whose sum overflows is forced too, which only costs an exact evaluation.
    const float hw = ep + w;
    const bool force = ill || !(denom > kDenomGuard * alpha) || !(hw < PosInf());
    lo = force ? lof : ep - w;
    hi = force ? PosInf() : hw;
}

// Cheap bounds [lo, hi] on the exact errors of slot h's candidates at layer L for this thread's
// kCpt codewords (Gram column pointers gq[q] = Grow + col[q]; the values of a codeword with !ok[q]
// are meaningless and unused).  This is the hot loop (see CheapPass in beam.cu).
// e' = E_old - diff^2/denom with y from FMA forward substitution, delta = |y|^2, eta = A.a.  The
// half-width covers the rounding of both this and the exact sequence: relative errors of order
// L ulp in diff (scale |gamma| + sum|A_t a_t|) and in denom (scale alpha + delta), propagated
// through r = diff^2/denom, plus the final subtraction; kept with a factor 16.  A candidate
// whose cheap value is unreliable (ill-conditioned slot, denom <= kDenomGuard * alpha, NaN)
// gets [-inf, +inf].  A codeword whose whole Gram column is zero (alpha is -0.0f in the beam's
// diagonal, see IsZeroColumn) gets [+inf, +inf]: the reference always skips it.
// The layer L is a run-time value (loops run to NL = MAXM - 1 with uniform guards): one copy of
// this code serves every layer, which keeps the kernel's hot code within the instruction cache.
template <int MAXM, bool kStrict>
__device__ __forceinline__ void CheapBounds(const SlotView<MAXM>& cur, int h, int L, const float* const (&gq)[kCpt],
                                            const bool (&ok)[kCpt],
                                            const float (&alpha)[kCpt], const float (&gamma)[kCpt],
                                            const float (&dg)[kCpt], float (&lo)[kCpt], float (&hi)[kCpt]) {
    const float* Rh = cur.Rh(h);
    const float* rinv = cur.rinvh(h);
    const float* ah = cur.ah(h);
    const int* rw = cur.rowh(h);
    // Slot values are warp-uniform shared-memory broadcasts, loaded where they are used (loading
    // them ahead into registers costs more in spills than it saves in load instructions).
    constexpr int NL = MAXM - 1;
    float A[kCpt][NL], y[kCpt][NL];
#pragma unroll
    for (int i = 0; i < NL; ++i) {
        if (i >= L) break;
        const int r = rw[i];
#pragma unroll
        for (int q = 0; q < kCpt; ++q) A[q][i] = ok[q] ? __ldg(gq[q] + r) : 0.0f;
    }
    float delta[kCpt], eta[kCpt], seta[kCpt];
#pragma unroll
    for (int q = 0; q < kCpt; ++q) {
        delta[q] = 0.0f;
        eta[q] = 0.0f;
        seta[q] = fabsf(gamma[q]);
    }
#pragma unroll
    for (int i = 0; i < NL; ++i) {
        if (i >= L) break;
        const float ri = rinv[i], ai = ah[i];
#pragma unroll
        for (int q = 0; q < kCpt; ++q) {
            float s = A[q][i];
#pragma unroll
            for (int k = 0; k < i; ++k) s = fmaf(-Rh[i * MAXM + k], y[q][k], s);
            y[q][i] = s * ri;
            delta[q] = fmaf(y[q][i], y[q][i], delta[q]);
            eta[q] = fmaf(A[q][i], ai, eta[q]);
            seta[q] = fmaf(fabsf(A[q][i]), fabsf(ai), seta[q]);
        }
    }
    const float Eo = cur.E[h];
    const bool ill = cur.ill[h] != 0;
#pragma unroll
    for (int q = 0; q < kCpt; ++q)
        BoundsTail<kStrict>(L, alpha[q], gamma[q], delta[q], eta[q], seta[q], Eo, ill, dg[q], lo[q], hi[q]);
}

}  // namespace beam
}  // namespace stlq_b200
