// Beam search with prefix least squares (BeamSearchPrefixLS, reference
// src/quantizer/beam_search.cpp:196-422) for sm_100a.
//
// One CTA of 128 threads encodes one vector at a time (persistent grid-stride loop).  Thread t
// owns codewords k = t, t+128, ... of the layer being expanded, for every live beam slot, so the
// per-code values (alpha = G(k,k), gamma = xC(k)) stay in registers and the per-slot values (the
// Cholesky factor R, coefficients, error) are warp-uniform shared-memory broadcasts.
//
// Candidate arithmetic follows the reference's float operation sequence exactly (forward and back
// substitution of SolveCholUpperRawFixed, delta = A.v, eta = A.a_old, IEEE division and square
// root, no fused multiply-add), so every candidate error is bit-identical to the reference's
// given the same xC, G and ||x||^2.
//
// Selection reproduces the reference's beam exactly, slot order included.  The reference scans
// candidates slot-major, code-minor; a candidate enters when its error is strictly below the
// current worst slot error and replaces the first slot holding that worst error
// (beam_search.cpp:101-113, 252-260, 320-333).  Here every candidate error of the layer is first
// written to shared memory by all threads; warp 0 then replays the scan 32 candidates at a time:
// one ballot finds the candidates below the current worst, and only those are replayed one by one
// (the slots live one per lane, so finding the first worst slot is a max-reduce plus a ballot).
// The next layer scans the slots in the resulting order, exactly like the reference, so ties
// between equal errors resolve identically.
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kThreads = 128;
constexpr int kCpt = kMaxK / kThreads;  // codewords per thread
constexpr unsigned kFull = 0xffffffffu;

template <int MAXM>
struct BeamSlots {
    float R[kMaxBeam][MAXM * MAXM];  // upper Cholesky factor, row-major R[r*MAXM + c], r <= c
    float a[kMaxBeam][MAXM];
    float E[kMaxBeam];
    int code[kMaxBeam][MAXM];
};

struct SlotTable {
    int cand[kMaxBeam];  // scan index of the candidate that holds each slot
    int n_finite;        // slots with a finite error (they form a prefix)
};

__device__ __forceinline__ float PosInf() { return __int_as_float(0x7f800000); }

// Exact candidate evaluation for slot h at layer L (compile-time L so the substitutions unroll).
// Returns the error; +inf for a candidate the reference skips (denom == 0, :309-311) or that can
// never enter the beam (e >= +inf or NaN, :320).  Optionally returns y, v, denom and a_last.
template <int MAXM, int L>
__device__ __forceinline__ float EvalCandidate(const BeamSlots<MAXM>& cur, int h, const int (&flat)[MAXM],
                                               const float* __restrict__ Grow, int H, int col, float alpha,
                                               float gamma, float* y_out, float* v_out, float* denom_out,
                                               float* alast_out) {
    const float* Rh = cur.R[h];
    float A[L], y[L], v[L];
#pragma unroll
    for (int t = 0; t < L; ++t) A[t] = __ldg(Grow + static_cast<size_t>(flat[t]) * H + col);
    // Forward solve R^T y = A (beam_search.cpp:138-147).
#pragma unroll
    for (int i = 0; i < L; ++i) {
        float s = A[i];
#pragma unroll
        for (int k = 0; k < i; ++k) s = sub_rn(s, mul_rn(Rh[k * MAXM + i], y[k]));
        y[i] = div_rn(s, Rh[i * MAXM + i]);
    }
    // Back solve R v = y (beam_search.cpp:152-161).
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
        eta = add_rn(eta, mul_rn(A[t], cur.a[h][t]));
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

// Warp 0 replays the reference's replace-worst scan over errs[0..n) (scan order) for `beam`
// slots.  Lane s < beam holds slot s.  Writes the slot table; returns nothing (call from warp 0).
__device__ void ReplayBeam(const float* errs, int n, int beam, SlotTable& st) {
    const int lane = threadIdx.x & 31;
    float es = lane < beam ? PosInf() : -PosInf();  // lanes >= beam never hold the worst
    int cs = -1;
    uint32_t wkey = __reduce_max_sync(kFull, OrderKey(es));
    int widx = __ffs(__ballot_sync(kFull, OrderKey(es) == wkey)) - 1;
    float worst = KeyToFloat(wkey);
    for (int base = 0; base < n; base += 32) {
        const int j = base + lane;
        const float e = j < n ? errs[j] : PosInf();
        unsigned mask = __ballot_sync(kFull, e < worst);
        while (mask) {
            const int l = __ffs(mask) - 1;
            mask &= mask - 1;
            const float el = __shfl_sync(kFull, e, l);
            if (el < worst) {  // the worst only decreases: re-test against the current one
                if (lane == widx) {
                    es = el;
                    cs = base + l;
                }
                wkey = __reduce_max_sync(kFull, OrderKey(es));
                widx = __ffs(__ballot_sync(kFull, OrderKey(es) == wkey)) - 1;
                worst = KeyToFloat(wkey);
            }
        }
    }
    if (lane < beam) st.cand[lane] = cs;
    const unsigned fin = __ballot_sync(kFull, lane < beam && es < PosInf());
    if (lane == 0) st.n_finite = __popc(fin);
}

template <int MAXM, int L>
__device__ void ExpandLayer(const Dims& dims, BeamSlots<MAXM>& cur, BeamSlots<MAXM>& nxt, int& curH,
                            const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                            const float* __restrict__ xc, int beam, float* errs, SlotTable& st) {
    const int tid = threadIdx.x;
    const int H = dims.H;
    const int K = dims.h_vec[L];
    const int offL = dims.off[L];
    float alpha[kCpt], gamma[kCpt];
#pragma unroll
    for (int c = 0; c < kCpt; ++c) {
        const int k = tid + c * kThreads;
        alpha[c] = k < K ? __ldg(Gdiag + offL + k) : 0.0f;
        gamma[c] = k < K ? __ldg(xc + offL + k) : 0.0f;
    }
    for (int h = 0; h < curH; ++h) {
        int flat[MAXM];
#pragma unroll
        for (int t = 0; t < MAXM; ++t) flat[t] = t < L ? dims.off[t] + cur.code[h][t] : 0;
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K)
                errs[h * K + k] = EvalCandidate<MAXM, L>(cur, h, flat, Grow, H, offL + k, alpha[c], gamma[c], nullptr,
                                                         nullptr, nullptr, nullptr);
        }
    }
    __syncthreads();
    if (tid < 32) ReplayBeam(errs, curH * K, beam, st);
    __syncthreads();
    const int newH = st.n_finite;
    if (newH == 0) {
        // No finite candidate (beam_search.cpp:385-400): keep the previous slots.  The code of
        // this layer is written as 0; the reference copies a stale buffer value there.
        const int keep = min(curH, beam);
        for (int e = tid; e < keep * MAXM * MAXM; e += kThreads)
            nxt.R[e / (MAXM * MAXM)][e % (MAXM * MAXM)] = cur.R[e / (MAXM * MAXM)][e % (MAXM * MAXM)];
        for (int e = tid; e < keep * MAXM; e += kThreads) {
            const int h = e / MAXM, t = e % MAXM;
            nxt.code[h][t] = t < L ? cur.code[h][t] : 0;
            nxt.a[h][t] = t < L ? cur.a[h][t] : 0.0f;
        }
        for (int h = tid; h < keep; h += kThreads) nxt.E[h] = cur.E[h];
        __syncthreads();
        curH = max(1, keep);
        return;
    }
    // Materialise the winners (beam_search.cpp:337-383): copy the parent's prefix, then the
    // winner's own column of R, coefficients and code.
    for (int e = tid; e < newH * L * L; e += kThreads) {
        const int o = e / (L * L), rc = e % (L * L), r = rc / L, c = rc % L;
        if (r <= c) nxt.R[o][r * MAXM + c] = cur.R[st.cand[o] / K][r * MAXM + c];
    }
    if (tid < newH) {
        const int o = tid;
        const int idx = st.cand[o];
        const int h = idx / K, k = idx % K;
        int flat[MAXM];
#pragma unroll
        for (int t = 0; t < MAXM; ++t) flat[t] = t < L ? dims.off[t] + cur.code[h][t] : 0;
        float y[L], v[L], denom, a_last;
        const float e = EvalCandidate<MAXM, L>(cur, h, flat, Grow, H, offL + k, __ldg(Gdiag + offL + k),
                                               __ldg(xc + offL + k), y, v, &denom, &a_last);
#pragma unroll
        for (int t = 0; t < L; ++t) {
            nxt.code[o][t] = cur.code[h][t];
            nxt.a[o][t] = sub_rn(cur.a[h][t], mul_rn(v[t], a_last));
            nxt.R[o][t * MAXM + L] = y[t];
        }
        nxt.code[o][L] = k;
        nxt.a[o][L] = a_last;
        nxt.R[o][L * MAXM + L] = __fsqrt_rn(denom);
        nxt.E[o] = e;
    }
    __syncthreads();
    curH = newH;
}

template <int MAXM>
__device__ void ExpandLayerDispatch(int L, const Dims& dims, BeamSlots<MAXM>& cur, BeamSlots<MAXM>& nxt, int& curH,
                                    const float* Grow, const float* Gdiag, const float* xc, int beam, float* errs,
                                    SlotTable& st) {
#define STLQ_B200_EXPAND(LL)                                                              \
    case LL:                                                                              \
        if constexpr (LL < MAXM)                                                          \
            ExpandLayer<MAXM, LL>(dims, cur, nxt, curH, Grow, Gdiag, xc, beam, errs, st); \
        break;
    switch (L) {
        STLQ_B200_EXPAND(1) STLQ_B200_EXPAND(2) STLQ_B200_EXPAND(3) STLQ_B200_EXPAND(4) STLQ_B200_EXPAND(5)
        STLQ_B200_EXPAND(6) STLQ_B200_EXPAND(7) STLQ_B200_EXPAND(8) STLQ_B200_EXPAND(9) STLQ_B200_EXPAND(10)
        STLQ_B200_EXPAND(11) STLQ_B200_EXPAND(12) STLQ_B200_EXPAND(13) STLQ_B200_EXPAND(14) STLQ_B200_EXPAND(15)
        default: break;
    }
#undef STLQ_B200_EXPAND
}

template <int MAXM>
__global__ void __launch_bounds__(kThreads) BeamSearchKernel(Dims dims, const float* __restrict__ Grow,
                                                             const float* __restrict__ Gdiag,
                                                             const float* __restrict__ xnorm2,
                                                             const float* __restrict__ xC, int64_t n, int beam,
                                                             uint8_t* __restrict__ Bout) {
    extern __shared__ __align__(16) unsigned char smem[];
    BeamSlots<MAXM>* slots = reinterpret_cast<BeamSlots<MAXM>*>(smem);
    SlotTable& st = *reinterpret_cast<SlotTable*>(smem + 2 * sizeof(BeamSlots<MAXM>));
    float* errs = reinterpret_cast<float*>(smem + 2 * sizeof(BeamSlots<MAXM>) + sizeof(SlotTable));
    const int tid = threadIdx.x;
    const int m = dims.m;
    const int K0 = dims.h_vec[0];

    for (int64_t vec = blockIdx.x; vec < n; vec += gridDim.x) {
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        BeamSlots<MAXM>* cur = &slots[0];
        BeamSlots<MAXM>* nxt = &slots[1];
        // Layer 0 (beam_search.cpp:238-263): a1 = gamma/alpha, e1 = ||x||^2 - gamma*a1 (no
        // clamp); a zero codeword (alpha == 0) is skipped.
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K0) {
                const float alpha = __ldg(Gdiag + k);
                const float gamma = __ldg(xc + k);
                const float a1 = div_rn(gamma, alpha);
                const float e1 = sub_rn(nx2, mul_rn(gamma, a1));
                errs[k] = (alpha != 0.0f && e1 < PosInf()) ? e1 : PosInf();
            }
        }
        __syncthreads();
        if (tid < 32) ReplayBeam(errs, K0, beam, st);
        __syncthreads();
        int curH = st.n_finite;
        if (tid < curH) {
            const int k = st.cand[tid];
            const float alpha = __ldg(Gdiag + k);
            const float gamma = __ldg(xc + k);
            const float a1 = div_rn(gamma, alpha);
            cur->code[tid][0] = k;
            cur->a[tid][0] = a1;
            cur->E[tid] = sub_rn(nx2, mul_rn(gamma, a1));
            cur->R[tid][0] = __fsqrt_rn(alpha);
        }
        if (curH == 0) {
            // No finite layer-0 candidate (every codeword zero): the reference carries one slot
            // with error +inf through every layer (every later candidate is then non-finite and
            // the fallback keeps the slot), ending with code 0 in every layer.
            if (tid < MAXM) {
                cur->code[0][tid] = 0;
                cur->a[0][tid] = 0.0f;
            }
            for (int e = tid; e < MAXM * MAXM; e += kThreads) cur->R[0][e] = 0.0f;
            if (tid == 0) cur->E[0] = PosInf();
            curH = 1;
        }
        __syncthreads();
        for (int L = 1; L < m; ++L) {
            ExpandLayerDispatch<MAXM>(L, dims, *cur, *nxt, curH, Grow, Gdiag, xc, beam, errs, st);
            BeamSlots<MAXM>* t = cur;
            cur = nxt;
            nxt = t;
        }
        // Final pick: the first slot holding the smallest error (beam_search.cpp:409-416).
        if (tid < 32) {
            const uint32_t key = tid < curH ? OrderKey(cur->E[tid]) : 0xffffffffu;
            const uint32_t kmin = __reduce_min_sync(kFull, key);
            const int best = __ffs(__ballot_sync(kFull, key == kmin)) - 1;
            if (tid < m) Bout[vec * m + tid] = static_cast<uint8_t>(cur->code[best][tid]);
        }
        __syncthreads();
    }
}

template <int MAXM>
size_t BeamSmemBytes(int beam, int maxK) {
    return 2 * sizeof(BeamSlots<MAXM>) + sizeof(SlotTable) + sizeof(float) * beam * maxK + 16;
}

template <int MAXM>
cudaError_t LaunchBeamT(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2, const float* xC,
                        int64_t n, int beam, uint8_t* Bout, int num_sms, cudaStream_t stream) {
    const size_t smem = BeamSmemBytes<MAXM>(beam, dims.maxK);
    cudaError_t e = cudaFuncSetAttribute(BeamSearchKernel<MAXM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, BeamSearchKernel<MAXM>, kThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1));
    BeamSearchKernel<MAXM><<<static_cast<int>(grid), kThreads, smem, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam,
                                                                               Bout);
    return cudaGetLastError();
}

}  // namespace

cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, uint8_t* Bout, unsigned int* err_flag,
                             int num_sms, cudaStream_t stream) {
    (void)err_flag;
    if (n <= 0) return cudaSuccess;
    if (dims.m <= 8) return LaunchBeamT<8>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, num_sms, stream);
    return LaunchBeamT<16>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, num_sms, stream);
}

}  // namespace stlq_b200
