// Beam search with prefix least squares (BeamSearchPrefixLS, reference
// src/quantizer/beam_search.cpp:196-422) for sm_100a.
//
// One CTA of 128 threads encodes one vector at a time (persistent grid-stride loop).  Thread t
// owns codewords k = t, t+128, ... of the layer being expanded, for every live beam entry, so the
// per-code values (alpha = G(k,k), gamma = xC(k)) stay in registers and the per-beam values (the
// Cholesky factor R, coefficients, error) are warp-uniform shared-memory broadcasts.
//
// Candidate arithmetic follows the reference's float operation sequence exactly (forward and back
// substitution of SolveCholUpperRawFixed, delta = A.v, eta = A.a_old, IEEE division and square
// root, no fused multiply-add), so every candidate error is bit-identical to the reference's
// given the same xC, G and ||x||^2.
//
// Selection.  The reference keeps B slots and lets a candidate replace the first worst slot when
// its error is strictly smaller (beam_search.cpp:101-113, 320-333).  The set it ends with is the B
// smallest errors; among equal errors at the boundary the earlier-scanned candidate wins.  Here
// every candidate gets the composite key (error, scan index) and the B smallest composites are
// selected exactly:
//   1. each thread keeps the minimum composite of its own candidates;
//   2. tau = the B-th smallest of the 128 per-thread minima (composites are unique, so exactly
//      B threads have a minimum <= tau, and tau bounds the B-th smallest candidate from above);
//   3. candidates <= tau survive; only those B threads can hold one, so the survivor list holds
//      at most B * (candidates per thread) entries;
//   4. survivors are ranked by counting and written to slot = rank (slots sorted by composite).
// The reference's slot order is its replacement history; here slots are sorted.  The two differ
// only when two candidates have bit-equal errors (scan order inside a layer, and the final pick
// among equal errors).
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kThreads = 128;
constexpr uint32_t kInvalidKey = 0xffffffffu;

template <int MAXM>
struct BeamSlots {
    float R[kMaxBeam][MAXM * MAXM];  // upper Cholesky factor, row-major R[r*MAXM + c], r <= c
    float a[kMaxBeam][MAXM];
    float E[kMaxBeam];
    int code[kMaxBeam][MAXM];
};

__device__ __forceinline__ uint64_t Composite(uint32_t key, uint32_t idx) {
    return (static_cast<uint64_t>(key) << 32) | idx;
}

// Exact candidate evaluation for beam entry h at layer L (compile-time L so the substitutions
// unroll).  Returns the key (kInvalidKey for a skipped candidate) and optionally y, v, denom,
// a_last, e for materialisation.
template <int MAXM, int L>
__device__ __forceinline__ uint32_t EvalCandidate(const BeamSlots<MAXM>& cur, int h, const int (&flat)[MAXM],
                                                  const float* __restrict__ Grow, int H, int col, float alpha,
                                                  float gamma, float* y_out, float* v_out, float* denom_out,
                                                  float* alast_out, float* e_out) {
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
        *e_out = e;
    }
    // Skipped: denom == 0 (beam_search.cpp:309-311); never entering: e >= +inf or NaN (:320).
    const bool valid = (denom != 0.0f) && (e < __int_as_float(0x7f800000));
    return valid ? OrderKey(e) : kInvalidKey;
}

struct SelectShared {
    uint64_t mins[kThreads];
    uint64_t tau;
    int n_surv;
    int n_valid;
    int slot_idx[kMaxBeam];
};

// Steps 2-4 of the selection (see file comment).  keys[idx] holds every candidate's key;
// my_min is this thread's minimum composite.  Returns the number of filled slots
// (slot_idx[0..ret) sorted by composite); all threads get the same value.
// This thread's candidates are idx = h*K + tid + c*kThreads for h < n_h, c < kCpt (code < K).
__device__ int SelectTopB(const uint32_t* keys, int n_h, int K, uint64_t my_min, int beam, SelectShared& ss,
                          uint16_t* surv, int surv_cap, unsigned int* err_flag) {
    constexpr int kCpt = kMaxK / kThreads;
    const int tid = threadIdx.x;
    ss.mins[tid] = my_min;
    if (tid == 0) {
        ss.tau = ~0ull;
        ss.n_surv = 0;
    }
    __syncthreads();
    int rank = 0;
    for (int s = 0; s < kThreads; ++s) rank += (ss.mins[s] < my_min);
    if (rank == beam - 1) ss.tau = my_min;  // unique: composites of distinct candidates differ
    __syncthreads();
    const uint64_t tau = ss.tau;
    for (int h = 0; h < n_h; ++h) {
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k >= K) continue;
            const int idx = h * K + k;
            const uint32_t key = keys[idx];
            if (key != kInvalidKey && Composite(key, idx) <= tau) {
                const int pos = atomicAdd(&ss.n_surv, 1);
                if (pos < surv_cap) surv[pos] = static_cast<uint16_t>(idx);
                else atomicOr(err_flag, kErrSurvivorOverflow);
            }
        }
    }
    __syncthreads();
    const int S = min(ss.n_surv, surv_cap);
    for (int s = tid; s < S; s += kThreads) {
        const int idx = surv[s];
        const uint64_t cs = Composite(keys[idx], idx);
        int r = 0;
        for (int q = 0; q < S; ++q) {
            const int iq = surv[q];
            r += (Composite(keys[iq], iq) < cs);
        }
        if (r < beam) ss.slot_idx[r] = idx;
    }
    __syncthreads();
    return min(S, beam);
}

template <int MAXM, int L>
__device__ void ExpandLayer(const Dims& dims, BeamSlots<MAXM>& cur, BeamSlots<MAXM>& nxt, int& curH,
                            const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                            const float* __restrict__ xc, int beam, uint32_t* keys, SelectShared& ss,
                            uint16_t* surv, int surv_cap, unsigned int* err_flag) {
    const int tid = threadIdx.x;
    const int H = dims.H;
    const int K = dims.h_vec[L];
    const int offL = dims.off[L];
    constexpr int kCpt = kMaxK / kThreads;
    float alpha[kCpt], gamma[kCpt];
#pragma unroll
    for (int c = 0; c < kCpt; ++c) {
        const int k = tid + c * kThreads;
        alpha[c] = k < K ? __ldg(Gdiag + offL + k) : 0.0f;
        gamma[c] = k < K ? __ldg(xc + offL + k) : 0.0f;
    }
    uint64_t my_min = ~0ull;
    for (int h = 0; h < curH; ++h) {
        int flat[MAXM];
#pragma unroll
        for (int t = 0; t < MAXM; ++t) flat[t] = t < L ? dims.off[t] + cur.code[h][t] : 0;
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K) {
                const uint32_t key = EvalCandidate<MAXM, L>(cur, h, flat, Grow, H, offL + k, alpha[c], gamma[c],
                                                            nullptr, nullptr, nullptr, nullptr, nullptr);
                const int idx = h * K + k;
                keys[idx] = key;
                const uint64_t comp = Composite(key, idx);
                my_min = comp < my_min ? comp : my_min;
            }
        }
    }
    const int newH = SelectTopB(keys, curH, K, my_min, beam, ss, surv, surv_cap, err_flag);
    if (newH == 0) {
        // No finite candidate (beam_search.cpp:385-400): keep the previous entries; the code of
        // this layer is written as 0 (the reference copies a stale buffer value there).
        const int keep = min(curH, beam);
        for (int e = tid; e < keep * MAXM * MAXM; e += kThreads) nxt.R[e / (MAXM * MAXM)][e % (MAXM * MAXM)] =
            cur.R[e / (MAXM * MAXM)][e % (MAXM * MAXM)];
        for (int e = tid; e < keep * MAXM; e += kThreads) {
            const int h = e / MAXM, t = e % MAXM;
            nxt.code[h][t] = t < L ? cur.code[h][t] : 0;
            nxt.a[h][t] = t < L ? cur.a[h][t] : 0.0f;
        }
        for (int h = tid; h < keep; h += kThreads) nxt.E[h] = cur.E[h];
        __syncthreads();
        curH = keep;
        return;
    }
    // Materialise the winners (beam_search.cpp:337-383): copy the parent's prefix, then the
    // winner's own column of R, coefficients and code.
    for (int e = tid; e < newH * L * L; e += kThreads) {
        const int o = e / (L * L), rc = e % (L * L), r = rc / L, c = rc % L;
        if (r <= c) nxt.R[o][r * MAXM + c] = cur.R[ss.slot_idx[o] / K][r * MAXM + c];
    }
    if (tid < newH) {
        const int o = tid;
        const int idx = ss.slot_idx[o];
        const int h = idx / K, k = idx % K;
        int flat[MAXM];
#pragma unroll
        for (int t = 0; t < MAXM; ++t) flat[t] = t < L ? dims.off[t] + cur.code[h][t] : 0;
        float y[L], v[L], denom, a_last, e;
        EvalCandidate<MAXM, L>(cur, h, flat, Grow, H, offL + k, __ldg(Gdiag + offL + k), __ldg(xc + offL + k), y, v,
                               &denom, &a_last, &e);
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
                                    const float* Grow, const float* Gdiag, const float* xc, int beam, uint32_t* keys,
                                    SelectShared& ss, uint16_t* surv, int surv_cap, unsigned int* err) {
#define STLQ_B200_EXPAND(LL)                                                                                  \
    case LL:                                                                                                  \
        if constexpr (LL < MAXM)                                                                              \
            ExpandLayer<MAXM, LL>(dims, cur, nxt, curH, Grow, Gdiag, xc, beam, keys, ss, surv, surv_cap, err); \
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
                                                             uint8_t* __restrict__ Bout, unsigned int* err_flag) {
    extern __shared__ __align__(16) unsigned char smem[];
    BeamSlots<MAXM>* slots = reinterpret_cast<BeamSlots<MAXM>*>(smem);
    SelectShared& ss = *reinterpret_cast<SelectShared*>(smem + 2 * sizeof(BeamSlots<MAXM>));
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem + 2 * sizeof(BeamSlots<MAXM>) + sizeof(SelectShared));
    uint16_t* surv = reinterpret_cast<uint16_t*>(keys + beam * dims.maxK);
    const int surv_cap = beam * beam * (kMaxK / kThreads);
    const int tid = threadIdx.x;
    const int m = dims.m;
    const int K0 = dims.h_vec[0];
    constexpr int kCpt = kMaxK / kThreads;

    for (int64_t vec = blockIdx.x; vec < n; vec += gridDim.x) {
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        BeamSlots<MAXM>* cur = &slots[0];
        BeamSlots<MAXM>* nxt = &slots[1];
        // Layer 0 (beam_search.cpp:238-263): a1 = gamma/alpha, e1 = ||x||^2 - gamma*a1 (no clamp).
        uint64_t my_min = ~0ull;
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K0) {
                const float alpha = __ldg(Gdiag + k);
                const float gamma = __ldg(xc + k);
                const float a1 = div_rn(gamma, alpha);
                const float e1 = sub_rn(nx2, mul_rn(gamma, a1));
                const bool valid = (alpha != 0.0f) && (e1 < __int_as_float(0x7f800000));
                const uint32_t key = valid ? OrderKey(e1) : kInvalidKey;
                keys[k] = key;
                const uint64_t comp = Composite(key, k);
                my_min = comp < my_min ? comp : my_min;
            }
        }
        int curH = SelectTopB(keys, 1, K0, my_min, beam, ss, surv, surv_cap, err_flag);
        if (tid < curH) {
            const int k = ss.slot_idx[tid];
            const float alpha = __ldg(Gdiag + k);
            const float gamma = __ldg(xc + k);
            const float a1 = div_rn(gamma, alpha);
            cur->code[tid][0] = k;
            cur->a[tid][0] = a1;
            cur->E[tid] = sub_rn(nx2, mul_rn(gamma, a1));
            cur->R[tid][0] = __fsqrt_rn(alpha);
        }
        __syncthreads();
        if (curH == 0) {
            // No finite layer-0 candidate (every codeword zero): the reference carries one slot
            // with error +inf through every layer (each later candidate is then non-finite and
            // the fallback keeps the slot), ending with code 0 in every layer.
            if (tid < MAXM) {
                cur->code[0][tid] = 0;
                cur->a[0][tid] = 0.0f;
            }
            for (int e = tid; e < MAXM * MAXM; e += kThreads) cur->R[0][e] = 0.0f;
            if (tid == 0) cur->E[0] = __int_as_float(0x7f800000);
            __syncthreads();
            curH = 1;
        }
        for (int L = 1; L < m; ++L) {
            ExpandLayerDispatch<MAXM>(L, dims, *cur, *nxt, curH, Grow, Gdiag, xc, beam, keys, ss, surv, surv_cap,
                                      err_flag);
            BeamSlots<MAXM>* t = cur;
            cur = nxt;
            nxt = t;
        }
        // Slot 0 holds the smallest (error, scan index): the reference's final pick (:409-416).
        if (tid < m) Bout[vec * m + tid] = static_cast<uint8_t>(cur->code[0][tid]);
        __syncthreads();
    }
}

template <int MAXM>
size_t BeamSmemBytes(int beam, int maxK) {
    const size_t base = 2 * sizeof(BeamSlots<MAXM>) + sizeof(SelectShared);
    return base + sizeof(uint32_t) * beam * maxK + sizeof(uint16_t) * beam * beam * (kMaxK / kThreads) + 16;
}

}  // namespace

// Host launcher.  Returns a cudaError_t.
cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, uint8_t* Bout, unsigned int* err_flag,
                             int num_sms, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (dims.m <= 8) {
        const size_t smem = BeamSmemBytes<8>(beam, dims.maxK);
        cudaError_t e = cudaFuncSetAttribute(BeamSearchKernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, BeamSearchKernel<8>, kThreads, smem);
        const int64_t grid = std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1));
        BeamSearchKernel<8><<<static_cast<int>(grid), kThreads, smem, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam,
                                                                                 Bout, err_flag);
    } else {
        const size_t smem = BeamSmemBytes<16>(beam, dims.maxK);
        cudaError_t e = cudaFuncSetAttribute(BeamSearchKernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, BeamSearchKernel<16>, kThreads, smem);
        const int64_t grid = std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1));
        BeamSearchKernel<16><<<static_cast<int>(grid), kThreads, smem, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n,
                                                                                  beam, Bout, err_flag);
    }
    return cudaGetLastError();
}

}  // namespace stlq_b200
