// Beam search with prefix least squares (BeamSearchPrefixLS, reference
// src/quantizer/beam_search.cpp:196-422) for sm_100a.
//
// One CTA of 128 threads encodes one vector at a time (persistent grid-stride loop).  Thread t
// owns codewords k = t, t+128 of the layer being expanded, for every live beam slot, so the
// per-code values (alpha = G(k,k), gamma = xC(k)) stay in registers and the per-slot values (the
// Cholesky factor R, coefficients, error) are warp-uniform shared-memory broadcasts.
//
// Exactness.  Every candidate error that can influence the result is computed with the
// reference's float operation sequence (forward and back substitution of SolveCholUpperRawFixed,
// delta = A.v, eta = A.a_old, IEEE division and square root, no fused multiply-add), so it is
// bit-identical to the reference's given the same xC, G and ||x||^2.
//
// Selection reproduces the reference's beam, slot order included.  The reference scans
// candidates slot-major, code-minor; a candidate enters when its error is strictly below the
// current worst slot error and replaces the first slot holding that worst error
// (beam_search.cpp:101-113, 252-260, 320-333).  Warp 0 replays that scan (slots one per lane;
// the first worst slot is a max-reduce plus a ballot).
//
// Work saving without changing any decision.  A layer runs in four phases:
//   A. slot 0's candidates are evaluated exactly and replayed; tau = the worst slot error after
//      them.  The worst error never increases during the scan, so no later candidate with an
//      exact error >= tau can enter the beam;
//   B. every other candidate is evaluated with a cheap FMA/reciprocal formula (forward
//      substitution only, delta = |y|^2) together with a bound on its rounding error relative to
//      the exact sequence; a candidate is kept when its cheap error minus the bound is below tau
//      (and always when the slot or the candidate is ill-conditioned or the value is not finite);
//   C. the kept candidates are compacted in scan order and evaluated exactly by all threads;
//   D. warp 0 continues the replay over the kept candidates only.
// Dropped candidates provably cannot enter the beam, so the replay sees the same sequence of
// entering candidates as the reference.  With STLQ_B200_CHECK_FILTER set, the kernel evaluates
// every candidate exactly as well and raises an error flag if a dropped one would have entered.
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kCpt = kMaxK / kThreads;  // codewords per thread
constexpr unsigned kFull = 0xffffffffu;
// A slot whose last pivot satisfies R_LL^2 < kIllCond * G(c,c) (its codeword nearly in the span of
// the earlier ones) evaluates all its candidates exactly; so does a candidate whose cheap denom
// falls below kDenomGuard * alpha.
constexpr float kIllCond = 1e-4f;
constexpr float kDenomGuard = 1e-3f;

// Beam slots in dynamic shared memory, sized by the runtime beam width.
template <int MAXM>
struct SlotView {
    float* R;     // [beam][MAXM*MAXM] upper Cholesky factor, row-major R[r*MAXM + c], r <= c
    float* rinv;  // [beam][MAXM] 1/R_ii (cheap path only)
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

// Shared state of the layer loop.
struct LayerShared {
    int cand[kMaxBeam];     // scan index of the candidate held by each slot
    int n_finite;           // slots with a finite error (a prefix)
    float tau;              // worst slot error after slot 0's candidates
    int n_kept;             // compacted candidates of phase C
    int chunk_off[kMaxBeam * kCpt * kWarps + 1];
    unsigned chunk_mask[kMaxBeam * kCpt * kWarps];
};

__device__ __forceinline__ float PosInf() { return __int_as_float(0x7f800000); }

// Exact candidate evaluation for slot h at layer L (compile-time L so the substitutions unroll).
// Returns the error; +inf for a candidate the reference skips (denom == 0, :309-311) or that can
// never enter the beam (e >= +inf or NaN, :320).  Optionally returns y, v, denom and a_last.
template <int MAXM, int L>
__device__ __forceinline__ float EvalExact(const SlotView<MAXM>& cur, int h, const int (&flat)[MAXM],
                                           const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                           float* y_out, float* v_out, float* denom_out, float* alast_out) {
    const float* Rh = cur.Rh(h);
    const float* ah = cur.ah(h);
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

// Cheap evaluation: true when the candidate may have an exact error below tau.
// e' = E_old - diff^2/denom with y from FMA forward substitution, delta = |y|^2, eta = A.a.  The
// bound de covers the rounding of both this and the exact sequence: relative errors of order
// L ulp in diff (scale |gamma| + sum|A_t a_t|) and in denom (scale alpha + delta), propagated
// through r = diff^2/denom, plus the final subtraction; kept with a factor 16.
template <int MAXM, int L>
__device__ __forceinline__ bool MayEnter(const SlotView<MAXM>& cur, int h, const int (&flat)[MAXM],
                                         const float* __restrict__ Grow, int H, int col, float alpha, float gamma,
                                         float tau) {
    const float* Rh = cur.Rh(h);
    const float* rinv = cur.rinvh(h);
    const float* ah = cur.ah(h);
    float A[L], y[L];
#pragma unroll
    for (int t = 0; t < L; ++t) A[t] = __ldg(Grow + static_cast<size_t>(flat[t]) * H + col);
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
    const float r = __fdividef(diff * diff, denom);
    const float ep = cur.E[h] - r;
    constexpr float u = 1.2e-7f * (L + 2);
    const float de = 2.0f * fabsf(diff) * (u * seta) / denom + fabsf(r) * (u * (alpha + delta)) / denom +
                     1.2e-7f * (cur.E[h] + fabsf(r));
    const bool force = cur.ill[h] || !(denom > kDenomGuard * alpha);
    return force || !(ep - 16.0f * de >= tau);
}

// Warp-0 state of the replay of the reference's replace-worst scan: lane s < beam holds slot s.
struct Replay {
    float es;
    int cs;
    float worst;
    int widx;
    __device__ void Init(int beam) {
        const int lane = threadIdx.x & 31;
        es = lane < beam ? PosInf() : -PosInf();  // lanes >= beam never hold the worst
        cs = -1;
        Refresh();
    }
    __device__ void Refresh() {
        const uint32_t key = OrderKey(es);
        const uint32_t wkey = __reduce_max_sync(kFull, key);
        widx = __ffs(__ballot_sync(kFull, key == wkey)) - 1;
        worst = KeyToFloat(wkey);
    }
    // Offers 32 candidates (lane l holds candidate id ids and error e; invalid lanes +inf).
    __device__ void Offer(float e, int id) {
        const int lane = threadIdx.x & 31;
        unsigned mask = __ballot_sync(kFull, e < worst);
        while (mask) {
            const int l = __ffs(mask) - 1;
            mask &= mask - 1;
            const float el = __shfl_sync(kFull, e, l);
            const int il = __shfl_sync(kFull, id, l);
            if (el < worst) {  // the worst only decreases: re-test against the current one
                if (lane == widx) {
                    es = el;
                    cs = il;
                }
                Refresh();
            }
        }
    }
    __device__ void Publish(int beam, LayerShared& ls) {
        const int lane = threadIdx.x & 31;
        if (lane < beam) ls.cand[lane] = cs;
        const unsigned fin = __ballot_sync(kFull, lane < beam && es < PosInf());
        if (lane == 0) ls.n_finite = __popc(fin);
    }
};

template <int MAXM, int L>
__device__ __forceinline__ void FlatOf(const Dims& dims, const SlotView<MAXM>& cur, int h, int (&flat)[MAXM]) {
#pragma unroll
    for (int t = 0; t < MAXM; ++t) flat[t] = t < L ? dims.off[t] + cur.codeh(h)[t] : 0;
}

template <int MAXM, int L>
__device__ void ExpandLayer(const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int& curH,
                            const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                            const float* __restrict__ xc, int beam, float* errs, uint16_t* list, LayerShared& ls,
                            int check, unsigned int* err_flag) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
    // Phase A: slot 0 exactly, then its replay; tau bounds every later entering error.
    {
        int flat[MAXM];
        FlatOf<MAXM, L>(dims, cur, 0, flat);
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K)
                errs[k] = EvalExact<MAXM, L>(cur, 0, flat, Grow, H, offL + k, alpha[c], gamma[c], nullptr, nullptr,
                                             nullptr, nullptr);
        }
    }
    __syncthreads();
    Replay rp;
    if (warp == 0) {
        rp.Init(beam);
        for (int base = 0; base < K; base += 32) {
            const int j = base + lane;
            rp.Offer(j < K ? errs[j] : PosInf(), j);
        }
        if (lane == 0) ls.tau = rp.worst;
    }
    __syncthreads();
    const float tau = ls.tau;
    // Phase B: cheap evaluation of the other slots -> one keep-mask per 32 candidates.
    for (int h = 1; h < curH; ++h) {
        int flat[MAXM];
        FlatOf<MAXM, L>(dims, cur, h, flat);
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            bool keep = false;
            if (k < K) {
                keep = MayEnter<MAXM, L>(cur, h, flat, Grow, H, offL + k, alpha[c], gamma[c], tau);
                if (check && !keep) {
                    const float e = EvalExact<MAXM, L>(cur, h, flat, Grow, H, offL + k, alpha[c], gamma[c], nullptr,
                                                       nullptr, nullptr, nullptr);
                    if (e < tau) atomicOr(err_flag, kErrFilterMiss);
                }
            }
            const unsigned mask = __ballot_sync(kFull, keep);
            if (lane == 0) ls.chunk_mask[((h - 1) * kCpt + c) * kWarps + warp] = mask;
        }
    }
    __syncthreads();
    // Phase C: compact the kept candidates in scan order, then evaluate them exactly.
    const int nq = (curH - 1) * kCpt * kWarps;
    if (warp == 0) {
        const int per = (nq + 31) / 32;
        const int q0 = lane * per;
        int s = 0;
        for (int q = q0; q < min(q0 + per, nq); ++q) s += __popc(ls.chunk_mask[q]);
        int incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - s;
        for (int q = q0; q < min(q0 + per, nq); ++q) {
            ls.chunk_off[q] = run;
            run += __popc(ls.chunk_mask[q]);
        }
        if (lane == 31) ls.n_kept = incl;
    }
    __syncthreads();
    for (int h = 1; h < curH; ++h) {
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int q = ((h - 1) * kCpt + c) * kWarps + warp;
            const unsigned mask = ls.chunk_mask[q];
            if ((mask >> lane) & 1u)
                list[ls.chunk_off[q] + __popc(mask & ((1u << lane) - 1u))] =
                    static_cast<uint16_t>(h * K + tid + c * kThreads);
        }
    }
    __syncthreads();
    const int n_kept = ls.n_kept;
    for (int p = tid; p < n_kept; p += kThreads) {
        const int idx = list[p];
        const int h = idx / K, k = idx - h * K;
        int flat[MAXM];
        FlatOf<MAXM, L>(dims, cur, h, flat);
        errs[idx] = EvalExact<MAXM, L>(cur, h, flat, Grow, H, offL + k, __ldg(Gdiag + offL + k), __ldg(xc + offL + k),
                                       nullptr, nullptr, nullptr, nullptr);
    }
    __syncthreads();
    // Phase D: the replay continues over the kept candidates only.
    if (warp == 0) {
        for (int base = 0; base < n_kept; base += 32) {
            const int p = base + lane;
            const int id = p < n_kept ? list[p] : -1;
            rp.Offer(p < n_kept ? errs[id] : PosInf(), id);
        }
        rp.Publish(beam, ls);
    }
    __syncthreads();
    const int newH = ls.n_finite;
    if (newH == 0) {
        // No finite candidate (beam_search.cpp:385-400): keep the previous slots.  The code of
        // this layer is written as 0; the reference copies a stale buffer value there.
        const int keep = min(curH, beam);
        for (int e = tid; e < keep * MAXM * MAXM; e += kThreads) nxt.R[e] = cur.R[e];
        for (int e = tid; e < keep * MAXM; e += kThreads) {
            const int t = e % MAXM;
            nxt.code[e] = t < L ? cur.code[e] : 0;
            nxt.a[e] = t < L ? cur.a[e] : 0.0f;
            nxt.rinv[e] = cur.rinv[e];
        }
        for (int h = tid; h < keep; h += kThreads) {
            nxt.E[h] = cur.E[h];
            nxt.ill[h] = cur.ill[h];
        }
        __syncthreads();
        curH = max(1, keep);
        return;
    }
    // Materialise the winners (beam_search.cpp:337-383): copy the parent's prefix, then the
    // winner's own column of R, coefficients and code.
    for (int e = tid; e < newH * L * L; e += kThreads) {
        const int o = e / (L * L), rc = e % (L * L), r = rc / L, c = rc % L;
        if (r <= c) nxt.Rh(o)[r * MAXM + c] = cur.Rh(ls.cand[o] / K)[r * MAXM + c];
    }
    if (tid < newH) {
        const int o = tid;
        const int idx = ls.cand[o];
        const int h = idx / K, k = idx - h * K;
        int flat[MAXM];
        FlatOf<MAXM, L>(dims, cur, h, flat);
        float y[L], v[L], denom, a_last;
        const float ak = __ldg(Gdiag + offL + k);
        const float e = EvalExact<MAXM, L>(cur, h, flat, Grow, H, offL + k, ak, __ldg(xc + offL + k), y, v, &denom,
                                           &a_last);
#pragma unroll
        for (int t = 0; t < L; ++t) {
            nxt.codeh(o)[t] = cur.codeh(h)[t];
            nxt.ah(o)[t] = sub_rn(cur.ah(h)[t], mul_rn(v[t], a_last));
            nxt.Rh(o)[t * MAXM + L] = y[t];
            nxt.rinvh(o)[t] = cur.rinvh(h)[t];
        }
        const float rll = __fsqrt_rn(denom);
        nxt.codeh(o)[L] = k;
        nxt.ah(o)[L] = a_last;
        nxt.Rh(o)[L * MAXM + L] = rll;
        nxt.rinvh(o)[L] = __frcp_rn(rll);
        nxt.E[o] = e;
        nxt.ill[o] = cur.ill[h] | !(denom >= kIllCond * ak);
    }
    __syncthreads();
    curH = newH;
}

template <int MAXM>
__device__ void ExpandLayerDispatch(int L, const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt,
                                    int& curH, const float* Grow, const float* Gdiag, const float* xc, int beam,
                                    float* errs, uint16_t* list, LayerShared& ls, int check, unsigned int* err) {
#define STLQ_B200_EXPAND(LL)                                                                                   \
    case LL:                                                                                                   \
        if constexpr (LL < MAXM)                                                                               \
            ExpandLayer<MAXM, LL>(dims, cur, nxt, curH, Grow, Gdiag, xc, beam, errs, list, ls, check, err);   \
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
struct BeamSmem {
    static size_t Bytes(int beam, int maxK) {
        size_t b = 2 * SlotView<MAXM>::Bytes(beam);
        b = (b + 15) & ~size_t(15);
        b += sizeof(LayerShared);
        b = (b + 15) & ~size_t(15);
        b += sizeof(float) * beam * maxK;      // errs
        b += sizeof(uint16_t) * beam * maxK;   // list
        return b + 16;
    }
};

template <int MAXM>
__global__ void __launch_bounds__(kThreads, MAXM <= 8 ? 5 : 1) BeamSearchKernel(Dims dims, const float* __restrict__ Grow,
                                                             const float* __restrict__ Gdiag,
                                                             const float* __restrict__ xnorm2,
                                                             const float* __restrict__ xC, int64_t n, int beam,
                                                             uint8_t* __restrict__ Bout, int check,
                                                             unsigned int* err_flag) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t sv = SlotView<MAXM>::Bytes(beam);
    size_t off = (2 * sv + 15) & ~size_t(15);
    LayerShared& ls = *reinterpret_cast<LayerShared*>(smem + off);
    off = (off + sizeof(LayerShared) + 15) & ~size_t(15);
    float* errs = reinterpret_cast<float*>(smem + off);
    uint16_t* list = reinterpret_cast<uint16_t*>(errs + beam * dims.maxK);
    const int tid = threadIdx.x;
    const int m = dims.m;
    const int K0 = dims.h_vec[0];

    for (int64_t vec = blockIdx.x; vec < n; vec += gridDim.x) {
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        int ci = 0;  // index of the current slot buffer
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
        if (tid < 32) {
            Replay rp;
            rp.Init(beam);
            for (int base = 0; base < K0; base += 32) {
                const int j = base + tid;
                rp.Offer(j < K0 ? errs[j] : PosInf(), j);
            }
            rp.Publish(beam, ls);
        }
        __syncthreads();
        int curH = ls.n_finite;
        const SlotView<MAXM> s0 = SlotView<MAXM>::At(smem, beam);
        if (tid < curH) {
            const int k = ls.cand[tid];
            const float alpha = __ldg(Gdiag + k);
            const float gamma = __ldg(xc + k);
            const float a1 = div_rn(gamma, alpha);
            const float r00 = __fsqrt_rn(alpha);
            s0.codeh(tid)[0] = k;
            s0.ah(tid)[0] = a1;
            s0.E[tid] = sub_rn(nx2, mul_rn(gamma, a1));
            s0.Rh(tid)[0] = r00;
            s0.rinvh(tid)[0] = __frcp_rn(r00);
            s0.ill[tid] = 0;
        }
        if (curH == 0) {
            // No finite layer-0 candidate (every codeword zero): the reference carries one slot
            // with error +inf through every layer (every later candidate is then non-finite and
            // the fallback keeps the slot), ending with code 0 in every layer.
            if (tid < MAXM) {
                s0.codeh(0)[tid] = 0;
                s0.ah(0)[tid] = 0.0f;
                s0.rinvh(0)[tid] = 0.0f;
            }
            for (int e = tid; e < MAXM * MAXM; e += kThreads) s0.Rh(0)[e] = 0.0f;
            if (tid == 0) {
                s0.E[0] = PosInf();
                s0.ill[0] = 1;
            }
            curH = 1;
        }
        __syncthreads();
        for (int L = 1; L < m; ++L) {
            ExpandLayerDispatch<MAXM>(L, dims, SlotView<MAXM>::At(smem + ci * sv, beam),
                                      SlotView<MAXM>::At(smem + (ci ^ 1) * sv, beam), curH, Grow, Gdiag, xc, beam, errs,
                                      list, ls, check, err_flag);
            ci ^= 1;
        }
        // Final pick: the first slot holding the smallest error (beam_search.cpp:409-416).
        if (tid < 32) {
            const SlotView<MAXM> cur = SlotView<MAXM>::At(smem + ci * sv, beam);
            const uint32_t key = tid < curH ? OrderKey(cur.E[tid]) : 0xffffffffu;
            const uint32_t kmin = __reduce_min_sync(kFull, key);
            const int best = __ffs(__ballot_sync(kFull, key == kmin)) - 1;
            if (tid < m) Bout[vec * m + tid] = static_cast<uint8_t>(cur.codeh(best)[tid]);
        }
        __syncthreads();
    }
}

template <int MAXM>
cudaError_t LaunchBeamT(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2, const float* xC,
                        int64_t n, int beam, uint8_t* Bout, int check, unsigned int* err_flag, int num_sms,
                        cudaStream_t stream) {
    const size_t smem = BeamSmem<MAXM>::Bytes(beam, dims.maxK);
    cudaError_t e = cudaFuncSetAttribute(BeamSearchKernel<MAXM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, BeamSearchKernel<MAXM>, kThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1));
    BeamSearchKernel<MAXM><<<static_cast<int>(grid), kThreads, smem, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam,
                                                                               Bout, check, err_flag);
    return cudaGetLastError();
}

}  // namespace

cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, uint8_t* Bout, int check, unsigned int* err_flag,
                             int num_sms, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (dims.m <= 8)
        return LaunchBeamT<8>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, check, err_flag, num_sms, stream);
    return LaunchBeamT<16>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, check, err_flag, num_sms, stream);
}

}  // namespace stlq_b200
