// Beam search with prefix least squares (BeamSearchPrefixLS, reference
// src/quantizer/beam_search.cpp:196-422) for sm_100a: two kernels with identical results.
//
// Both: one CTA of 128 threads encodes one vector at a time.  Thread t owns codewords t, t+128 of
// the layer being expanded, for every live beam slot; per-code values (alpha = G(k,k),
// gamma = xC(k)) stay in registers, per-slot values (Cholesky factor R, coefficients, error) are
// warp-uniform shared-memory broadcasts.  Every error that decides anything is computed in the
// reference's float operation sequence (beam::EvalExact), so it is bit-identical to the
// reference's given the same xC, G and ||x||^2.
//
// The reference's beam keeps B slots; a candidate (scanned slot-major, code-minor) enters when its
// error is strictly below the current worst slot error and replaces the first slot holding it
// (beam_search.cpp:101-113, 252-260, 320-333); the final pick is the first slot with the
// smallest error (:409-416).  What ends in the slots is the B smallest errors; the slot ORDER (its
// replacement history, which is also the next layer's scan order) and the final pick can only
// matter when two candidates have bit-equal errors at the selection boundary or at the minimum.
//
// BeamFastKernel uses that: per layer it bounds every candidate's exact error from a cheap
// evaluation (beam::CheapBounds), takes tau = a value below which B candidates provably lie,
// evaluates exactly only the candidates whose lower bound is <= tau, and selects the B smallest
// exact errors.  When an exact tie sits at the boundary (or at the final minimum), or the survivor
// list would overflow, the vector is handed to BeamReplayKernel.
//
// BeamReplayKernel evaluates every candidate exactly and replays the reference's replacement
// scan itself (warp 0, slots one per lane), so ties resolve exactly as in the reference.
#include <cstdint>

#include "beam_common.cuh"
#include "launch.h"

namespace stlq_b200 {

using namespace beam;

namespace {

constexpr int kSurvCap = 512;  // exactly evaluated survivors per layer in the fast kernel

struct LayerTable {
    int cand[kMaxBeam];  // candidate (scan index) held by each slot, slot order
    int n_slots;         // slots filled
    int redo;            // fast kernel: hand the vector to the replay kernel
    uint32_t tau_key[kWarps];
    uint32_t mins[kWarps * kMaxBeam];  // each warp's B smallest per-thread upper bounds, sorted
    int n_surv;
    uint32_t key_b;
};

// Copies the winners' state into the next slot buffer (beam_search.cpp:337-383): parent prefix of
// R, then each winner's own R column (y, sqrt(denom)), coefficients a_t - v_t a_last, a_last, code.
template <int MAXM, int L>
__device__ void Materialize(const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt,
                            const LayerTable& lt, int newH, const float* __restrict__ Grow,
                            const float* __restrict__ Gdiag, const float* __restrict__ xc) {
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L], H = dims.H;
    for (int e = tid; e < newH * L * L; e += kThreads) {
        const int o = e / (L * L), rc = e % (L * L), r = rc / L, c = rc % L;
        if (r <= c) nxt.Rh(o)[r * MAXM + c] = cur.Rh(lt.cand[o] / K)[r * MAXM + c];
    }
    if (tid < newH) {
        const int o = tid;
        const int idx = lt.cand[o];
        const int h = idx / K, k = idx - h * K;
        const FlatArr<MAXM> flat = FlatOf<MAXM, L>(dims, cur, h);
        float y[L], v[L], denom, a_last;
        const float ak = __ldg(Gdiag + offL + k);
        const float e =
            EvalExact<MAXM, L>(cur, h, flat, Grow, H, offL + k, ak, __ldg(xc + offL + k), y, v, &denom, &a_last);
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
}

// No finite candidate in a layer (beam_search.cpp:385-400): the previous slots are kept.  The code
// of this layer is written as 0; the reference copies a stale buffer value there.
template <int MAXM, int L>
__device__ int KeepPrevious(const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int curH, int beam) {
    const int tid = threadIdx.x;
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
    return max(1, keep);
}

// Layer 0 state of slot o holding codeword k (beam_search.cpp:248-258).
template <int MAXM>
__device__ void InitSlot0(const SlotView<MAXM>& s, int o, int k, const float* Gdiag, const float* xc, float nx2) {
    const float alpha = __ldg(Gdiag + k);
    const float gamma = __ldg(xc + k);
    const float a1 = div_rn(gamma, alpha);
    const float r00 = __fsqrt_rn(alpha);
    s.codeh(o)[0] = k;
    s.ah(o)[0] = a1;
    s.E[o] = sub_rn(nx2, mul_rn(gamma, a1));
    s.Rh(o)[0] = r00;
    s.rinvh(o)[0] = __frcp_rn(r00);
    s.ill[o] = 0;
}

// Every layer-0 codeword is zero: the reference carries one slot with error +inf through every
// layer (each later candidate is then non-finite and the fallback keeps the slot), ending with
// code 0 in every layer.
template <int MAXM>
__device__ void DeadSlot0(const SlotView<MAXM>& s) {
    const int tid = threadIdx.x;
    if (tid < MAXM) {
        s.codeh(0)[tid] = 0;
        s.ah(0)[tid] = 0.0f;
        s.rinvh(0)[tid] = 0.0f;
    }
    for (int e = tid; e < MAXM * MAXM; e += kThreads) s.Rh(0)[e] = 0.0f;
    if (tid == 0) {
        s.E[0] = PosInf();
        s.ill[0] = 1;
    }
}

// Layer-0 error of codeword k: a1 = gamma/alpha, e1 = ||x||^2 - gamma*a1, not clamped; a zero
// codeword (alpha == 0) is skipped (beam_search.cpp:240-252).
__device__ __forceinline__ float Layer0Error(const float* Gdiag, const float* xc, float nx2, int k) {
    const float alpha = __ldg(Gdiag + k);
    const float gamma = __ldg(xc + k);
    const float e1 = sub_rn(nx2, mul_rn(gamma, div_rn(gamma, alpha)));
    return (alpha != 0.0f && e1 < PosInf()) ? e1 : PosInf();
}

// ---------------------------------------------------------------------------------------------
// Replay kernel: exact errors for every candidate and the reference's replacement scan.

// Warp-0 replay state: lane s < beam holds slot s.
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
    // Scans errs[0..n) in order: one ballot per 32 candidates, entering ones replayed in order.
    __device__ void Scan(const float* errs, int n) {
        const int lane = threadIdx.x & 31;
        for (int base = 0; base < n; base += 32) {
            const float e = base + lane < n ? errs[base + lane] : PosInf();
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
                    Refresh();
                }
            }
        }
    }
    __device__ void Publish(int beam, LayerTable& lt) {
        const int lane = threadIdx.x & 31;
        if (lane < beam) lt.cand[lane] = cs;
        const unsigned fin = __ballot_sync(kFull, lane < beam && es < PosInf());
        if (lane == 0) lt.n_slots = __popc(fin);
    }
};

template <int MAXM, int L>
__device__ void ReplayLayer(const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int& curH,
                            const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                            const float* __restrict__ xc, int beam, float* errs, LayerTable& lt) {
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L];
    float alpha[kCpt], gamma[kCpt];
#pragma unroll
    for (int c = 0; c < kCpt; ++c) {
        const int k = tid + c * kThreads;
        alpha[c] = k < K ? __ldg(Gdiag + offL + k) : 0.0f;
        gamma[c] = k < K ? __ldg(xc + offL + k) : 0.0f;
    }
    for (int h = 0; h < curH; ++h) {
        const FlatArr<MAXM> flat = FlatOf<MAXM, L>(dims, cur, h);
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K)
                errs[h * K + k] = EvalExact<MAXM, L>(cur, h, flat, Grow, dims.H, offL + k, alpha[c], gamma[c],
                                                     nullptr, nullptr, nullptr, nullptr);
        }
    }
    __syncthreads();
    if (tid < 32) {
        Replay rp;
        rp.Init(beam);
        rp.Scan(errs, curH * K);
        rp.Publish(beam, lt);
    }
    __syncthreads();
    const int newH = lt.n_slots;
    if (newH == 0) {
        curH = KeepPrevious<MAXM, L>(cur, nxt, curH, beam);
    } else {
        Materialize<MAXM, L>(dims, cur, nxt, lt, newH, Grow, Gdiag, xc);
        curH = newH;
    }
    __syncthreads();
}

template <int MAXM>
__device__ void ReplayDispatch(int L, const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int& curH,
                               const float* Grow, const float* Gdiag, const float* xc, int beam, float* errs,
                               LayerTable& lt) {
#define STLQ_B200_REPLAY(LL)                                                                    \
    case LL:                                                                                    \
        if constexpr (LL < MAXM) ReplayLayer<MAXM, LL>(dims, cur, nxt, curH, Grow, Gdiag, xc, beam, errs, lt); \
        break;
    switch (L) {
        STLQ_B200_REPLAY(1) STLQ_B200_REPLAY(2) STLQ_B200_REPLAY(3) STLQ_B200_REPLAY(4) STLQ_B200_REPLAY(5)
        STLQ_B200_REPLAY(6) STLQ_B200_REPLAY(7) STLQ_B200_REPLAY(8) STLQ_B200_REPLAY(9) STLQ_B200_REPLAY(10)
        STLQ_B200_REPLAY(11) STLQ_B200_REPLAY(12) STLQ_B200_REPLAY(13) STLQ_B200_REPLAY(14) STLQ_B200_REPLAY(15)
        default: break;
    }
#undef STLQ_B200_REPLAY
}

// Encodes the vectors listed in vec_list[0 .. *count) (or 0 .. n when vec_list is null).
template <int MAXM>
__global__ void __launch_bounds__(kThreads) BeamReplayKernel(Dims dims, const float* __restrict__ Grow,
                                                             const float* __restrict__ Gdiag,
                                                             const float* __restrict__ xnorm2,
                                                             const float* __restrict__ xC, int64_t n, int beam,
                                                             uint8_t* __restrict__ Bout, const int* vec_list,
                                                             const int* count) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t sv = SlotView<MAXM>::Bytes(beam);
    size_t off = (2 * sv + 15) & ~size_t(15);
    LayerTable& lt = *reinterpret_cast<LayerTable*>(smem + off);
    float* errs = reinterpret_cast<float*>(smem + ((off + sizeof(LayerTable) + 15) & ~size_t(15)));
    const int tid = threadIdx.x;
    const int m = dims.m, K0 = dims.h_vec[0];
    const int64_t total = vec_list ? static_cast<int64_t>(*count) : n;
    for (int64_t i = blockIdx.x; i < total; i += gridDim.x) {
        const int64_t vec = vec_list ? vec_list[i] : i;
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        for (int k = tid; k < K0; k += kThreads) errs[k] = Layer0Error(Gdiag, xc, nx2, k);
        __syncthreads();
        if (tid < 32) {
            Replay rp;
            rp.Init(beam);
            rp.Scan(errs, K0);
            rp.Publish(beam, lt);
        }
        __syncthreads();
        int curH = lt.n_slots;
        const SlotView<MAXM> s0 = SlotView<MAXM>::At(smem, beam);
        if (tid < curH) InitSlot0<MAXM>(s0, tid, lt.cand[tid], Gdiag, xc, nx2);
        if (curH == 0) {
            DeadSlot0<MAXM>(s0);
            curH = 1;
        }
        __syncthreads();
        int ci = 0;
        for (int L = 1; L < m; ++L) {
            ReplayDispatch<MAXM>(L, dims, SlotView<MAXM>::At(smem + ci * sv, beam),
                                 SlotView<MAXM>::At(smem + (ci ^ 1) * sv, beam), curH, Grow, Gdiag, xc, beam, errs, lt);
            ci ^= 1;
        }
        if (tid < 32) {  // first slot with the smallest error (beam_search.cpp:409-416)
            const SlotView<MAXM> cur = SlotView<MAXM>::At(smem + ci * sv, beam);
            const uint32_t key = tid < curH ? OrderKey(cur.E[tid]) : 0xffffffffu;
            const uint32_t kmin = __reduce_min_sync(kFull, key);
            const int best = __ffs(__ballot_sync(kFull, key == kmin)) - 1;
            if (tid < m) Bout[vec * m + tid] = static_cast<uint8_t>(cur.codeh(best)[tid]);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------------------
// Fast kernel: exact B smallest errors of each layer; ties handed to the replay kernel.

// Ascending bitonic sort of one key per lane across the warp; returns this lane's sorted key.
__device__ __forceinline__ uint32_t WarpSortAsc(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint32_t o = __shfl_xor_sync(kFull, v, j);
            const bool up = (lane & k) == 0, lower = (lane & j) == 0;
            v = (lower == up) ? min(v, o) : max(v, o);
        }
    }
    return v;
}

// Selection shared by every layer of the fast kernel, out of line so that one copy serves every
// layer.  Inputs: lo[idx] (a lower bound of each candidate's exact error; the exact error itself
// in layer 0) and this thread's smallest upper bound `hmin`.  The 128 per-thread minima belong to
// distinct candidates, so their B-th smallest, tau, bounds the B-th smallest exact error from
// above; every candidate with lo <= tau is a survivor (all others are provably larger than the
// B-th smallest exact error).  Returns the survivor count, or -1 when the list overflows.
__device__ __noinline__ int SelectSurvivors(const float* lo, int n_cand, uint32_t hmin, int beam, LayerTable& lt,
                                            uint16_t* surv) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Each warp sorts its 32 minima; only a warp's B smallest can be among the B smallest of all
    // 128, so warp 0 ranks those 4B values (binary search into the other sorted lists).
    const uint32_t sorted = WarpSortAsc(hmin);
    if (lane < beam) lt.mins[warp * kMaxBeam + lane] = sorted;
    if (tid == 0) {
        lt.n_surv = 0;
        lt.n_slots = 0;
        lt.key_b = 0u;
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t tb = 0xffffffffu;
        for (int i = lane; i < kWarps * beam; i += 32) {
            const int w = i / beam, j = i % beam;
            const uint32_t v = lt.mins[w * kMaxBeam + j];
            int r = j;
            for (int w2 = 0; w2 < kWarps; ++w2) {
                if (w2 == w) continue;
                int a = 0, b = beam;
                while (a < b) {
                    const int mid = (a + b) >> 1;
                    const uint32_t u = lt.mins[w2 * kMaxBeam + mid];
                    if (u < v || (u == v && w2 < w)) a = mid + 1;
                    else b = mid;
                }
                r += a;
            }
            if (r == beam - 1) tb = v;
        }
        tb = __reduce_min_sync(kFull, tb);
        if (lane == 0) lt.tau_key[0] = tb;
    }
    __syncthreads();
    const uint32_t tk = lt.tau_key[0];
    const float tau = tk >= OrderKey(PosInf()) ? PosInf() : KeyToFloat(tk);  // < B finite bounds: keep all
    for (int idx = tid; idx < n_cand; idx += kThreads) {
        if (lo[idx] <= tau) {
            const int p = atomicAdd(&lt.n_surv, 1);
            if (p < kSurvCap) surv[p] = static_cast<uint16_t>(idx);
        }
    }
    __syncthreads();
    const int S = lt.n_surv;
    return S > kSurvCap ? -1 : S;
}

// Ranks the S survivors by (exact error, scan index), fills lt.cand with the B smallest and returns
// the slot count, or -1 when an exact tie sits at the selection boundary.
__device__ __noinline__ int RankSurvivors(const float* ex, const uint16_t* surv, int S, int beam, LayerTable& lt,
                                          int* rank) {
    const int tid = threadIdx.x;
    int my_valid = 0;
    for (int p = tid; p < S; p += kThreads) {
        const uint32_t kp = OrderKey(ex[p]);
        const uint64_t cp = (static_cast<uint64_t>(kp) << 32) | surv[p];
        int r = 0;
        for (int q = 0; q < S; ++q) r += ((static_cast<uint64_t>(OrderKey(ex[q])) << 32) | surv[q]) < cp;
        rank[p] = r;
        const bool valid = ex[p] < PosInf();
        my_valid += valid;
        if (valid && r < beam) lt.cand[r] = surv[p];
        if (valid && r == beam - 1) lt.key_b = kp;
    }
    if (my_valid) atomicAdd(&lt.n_slots, my_valid);
    __syncthreads();
    const int n_valid = lt.n_slots;
    if (n_valid > beam) {
        // Tie at the boundary: another survivor with the B-th smallest error's exact value.
        const uint32_t kb = lt.key_b;
        int tie = 0;
        for (int p = tid; p < S; p += kThreads) tie |= (rank[p] >= beam && OrderKey(ex[p]) == kb);
        if (__syncthreads_or(tie)) return -1;
    }
    return min(n_valid, beam);
}

template <int MAXM, int L>
__device__ int FastLayer(const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int curH,
                         const float* __restrict__ Grow, const float* __restrict__ Gdiag, const float* __restrict__ xc,
                         int beam, float* lo, LayerTable& lt, uint16_t* surv, float* ex, int* rank, int check,
                         unsigned int* err_flag) {
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L], H = dims.H;
    float alpha[kCpt], gamma[kCpt];
#pragma unroll
    for (int c = 0; c < kCpt; ++c) {
        const int k = tid + c * kThreads;
        alpha[c] = k < K ? __ldg(Gdiag + offL + k) : 0.0f;
        gamma[c] = k < K ? __ldg(xc + offL + k) : 0.0f;
    }
    uint32_t hmin = 0xffffffffu;
    for (int h = 0; h < curH; ++h) {
        const FlatArr<MAXM> flat = FlatOf<MAXM, L>(dims, cur, h);
        float l[kCpt], hi[kCpt];
        // Both codewords' bounds first, stores after: the slot state they read stays in registers.
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            l[c] = PosInf();
            hi[c] = PosInf();
            if (tid + c * kThreads < K)
                CheapBounds<MAXM, L>(cur, h, flat, Grow, H, offL + tid + c * kThreads, alpha[c], gamma[c], &l[c],
                                     &hi[c]);
        }
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K) {
                lo[h * K + k] = l[c];
                hmin = min(hmin, OrderKey(hi[c]));
            }
        }
        if (check) {  // self-check: the exact error must lie inside the bounds
            for (int c = 0; c < kCpt; ++c) {
                const int k = tid + c * kThreads;
                if (k >= K) continue;
                const float e = EvalExact<MAXM, L>(cur, h, flat, Grow, H, offL + k, alpha[c], gamma[c], nullptr,
                                                   nullptr, nullptr, nullptr);
                if (e < PosInf() && !(e >= l[c] && e <= hi[c])) atomicOr(err_flag, kErrFilterMiss);
            }
        }
    }
    const int S = SelectSurvivors(lo, curH * K, hmin, beam, lt, surv);
    if (S < 0) return -1;
    for (int p = tid; p < S; p += kThreads) {
        const int idx = surv[p];
        const int h = idx / K, k = idx - h * K;
        ex[p] = EvalExact<MAXM, L>(cur, h, FlatOf<MAXM, L>(dims, cur, h), Grow, H, offL + k, __ldg(Gdiag + offL + k),
                                   __ldg(xc + offL + k), nullptr, nullptr, nullptr, nullptr);
    }
    __syncthreads();
    const int newH = RankSurvivors(ex, surv, S, beam, lt, rank);
    if (newH < 0) return -1;
    if (newH == 0) {
        const int keep = KeepPrevious<MAXM, L>(cur, nxt, curH, beam);
        __syncthreads();
        return keep;
    }
    Materialize<MAXM, L>(dims, cur, nxt, lt, newH, Grow, Gdiag, xc);
    __syncthreads();
    return newH;
}

template <int MAXM>
__device__ int FastDispatch(int L, const Dims& dims, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int curH,
                            const float* Grow, const float* Gdiag, const float* xc, int beam, float* lo,
                            LayerTable& lt, uint16_t* surv, float* ex, int* rank, int check, unsigned int* err) {
#define STLQ_B200_FAST(LL)                                                                                   \
    case LL:                                                                                                 \
        if constexpr (LL < MAXM)                                                                             \
            return FastLayer<MAXM, LL>(dims, cur, nxt, curH, Grow, Gdiag, xc, beam, lo, lt, surv, ex, rank,    \
                                       check, err);                                                          \
        break;
    switch (L) {
        STLQ_B200_FAST(1) STLQ_B200_FAST(2) STLQ_B200_FAST(3) STLQ_B200_FAST(4) STLQ_B200_FAST(5)
        STLQ_B200_FAST(6) STLQ_B200_FAST(7) STLQ_B200_FAST(8) STLQ_B200_FAST(9) STLQ_B200_FAST(10)
        STLQ_B200_FAST(11) STLQ_B200_FAST(12) STLQ_B200_FAST(13) STLQ_B200_FAST(14) STLQ_B200_FAST(15)
        default: break;
    }
#undef STLQ_B200_FAST
    return -1;
}

template <int MAXM>
__global__ void __launch_bounds__(kThreads, MAXM <= 8 ? 5 : 1) BeamFastKernel(Dims dims, const float* __restrict__ Grow,
                                                           const float* __restrict__ Gdiag,
                                                           const float* __restrict__ xnorm2,
                                                           const float* __restrict__ xC, int64_t n, int beam,
                                                           uint8_t* __restrict__ Bout, int* redo_list, int* redo_count,
                                                           int check, unsigned int* err_flag,
                                                           unsigned long long* stats) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t sv = SlotView<MAXM>::Bytes(beam);
    size_t off = (2 * sv + 15) & ~size_t(15);
    LayerTable& lt = *reinterpret_cast<LayerTable*>(smem + off);
    off = (off + sizeof(LayerTable) + 15) & ~size_t(15);
    float* lo = reinterpret_cast<float*>(smem + off);
    float* ex = lo + beam * dims.maxK;
    int* rank = reinterpret_cast<int*>(ex + kSurvCap);
    uint16_t* surv = reinterpret_cast<uint16_t*>(rank + kSurvCap);
    const int tid = threadIdx.x;
    const int m = dims.m, K0 = dims.h_vec[0];
    unsigned long long n_surv = 0, n_layers = 0, n_vec = 0, n_redo = 0;  // thread 0's tallies
    for (int64_t vec = blockIdx.x; vec < n; vec += gridDim.x) {
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        // Layer 0: exact errors are cheap; they serve as their own bounds.
        uint32_t hmin = 0xffffffffu;
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = tid + c * kThreads;
            if (k < K0) {
                const float e1 = Layer0Error(Gdiag, xc, nx2, k);
                lo[k] = e1;
                hmin = min(hmin, OrderKey(e1));
            }
        }
        int curH = SelectSurvivors(lo, K0, hmin, beam, lt, surv);
        if (curH >= 0) {
            for (int p = tid; p < curH; p += kThreads) ex[p] = lo[surv[p]];
            __syncthreads();
            curH = RankSurvivors(ex, surv, curH, beam, lt, rank);
        }
        const SlotView<MAXM> s0 = SlotView<MAXM>::At(smem, beam);
        if (curH > 0 && tid < curH) InitSlot0<MAXM>(s0, tid, lt.cand[tid], Gdiag, xc, nx2);
        if (curH == 0) {
            DeadSlot0<MAXM>(s0);
            curH = 1;
        }
        __syncthreads();
        int ci = 0;
        for (int L = 1; L < m && curH > 0; ++L) {
            curH = FastDispatch<MAXM>(L, dims, SlotView<MAXM>::At(smem + ci * sv, beam),
                                      SlotView<MAXM>::At(smem + (ci ^ 1) * sv, beam), curH, Grow, Gdiag, xc, beam, lo,
                                      lt, surv, ex, rank, check, err_flag);
            ci ^= 1;
            n_surv += lt.n_surv;
            ++n_layers;
        }
        const SlotView<MAXM> cur = SlotView<MAXM>::At(smem + ci * sv, beam);
        // Slots are sorted by (error, scan index): slot 0 is the pick unless the minimum is tied.
        const bool redo = curH < 0 || (curH >= 2 && OrderKey(cur.E[0]) == OrderKey(cur.E[1]));
        ++n_vec;
        n_redo += redo;
        if (redo) {
            if (tid == 0) redo_list[atomicAdd(redo_count, 1)] = static_cast<int>(vec);
        } else if (tid < m) {
            Bout[vec * m + tid] = static_cast<uint8_t>(cur.codeh(0)[tid]);
        }
        __syncthreads();
    }
    if (stats && tid == 0) {  // survivors evaluated exactly, layers, vectors, vectors handed to replay
        atomicAdd(stats + 0, n_surv);
        atomicAdd(stats + 1, n_layers);
        atomicAdd(stats + 2, n_vec);
        atomicAdd(stats + 3, n_redo);
    }
}

template <int MAXM>
size_t FastSmemBytes(int beam, int maxK) {
    size_t b = (2 * SlotView<MAXM>::Bytes(beam) + 15) & ~size_t(15);
    b = (b + sizeof(LayerTable) + 15) & ~size_t(15);
    return b + sizeof(float) * beam * maxK + (sizeof(float) + sizeof(int) + sizeof(uint16_t)) * kSurvCap + 16;
}

template <int MAXM>
size_t ReplaySmemBytes(int beam, int maxK) {
    size_t b = (2 * SlotView<MAXM>::Bytes(beam) + 15) & ~size_t(15);
    b = (b + sizeof(LayerTable) + 15) & ~size_t(15);
    return b + sizeof(float) * beam * maxK + 16;
}

template <typename KernelT>
cudaError_t Prepare(KernelT kernel, size_t smem, int num_sms, int64_t n, int* grid) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             static_cast<int>(cudaSharedmemCarveoutMaxShared));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    *grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1))));
    return cudaSuccess;
}

template <int MAXM>
cudaError_t LaunchBeamT(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2, const float* xC,
                        int64_t n, int beam, uint8_t* Bout, int* redo, int check, unsigned int* err_flag,
                        unsigned long long* stats, int num_sms, cudaStream_t stream) {
    int grid = 0;
    const size_t fsm = FastSmemBytes<MAXM>(beam, dims.maxK);
    cudaError_t e = Prepare(BeamFastKernel<MAXM>, fsm, num_sms, n, &grid);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(redo, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
    BeamFastKernel<MAXM><<<grid, kThreads, fsm, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, redo + 1, redo,
                                                          check, err_flag, stats);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t rsm = ReplaySmemBytes<MAXM>(beam, dims.maxK);
    e = Prepare(BeamReplayKernel<MAXM>, rsm, num_sms, n, &grid);
    if (e != cudaSuccess) return e;
    BeamReplayKernel<MAXM><<<grid, kThreads, rsm, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, redo + 1,
                                                            redo);
    return cudaGetLastError();
}

template <int MAXM>
cudaError_t PrepareT(const Dims& dims, int beam) {
    const size_t fsm = FastSmemBytes<MAXM>(beam, dims.maxK);
    const size_t rsm = ReplaySmemBytes<MAXM>(beam, dims.maxK);
    cudaError_t e = cudaFuncSetAttribute(BeamFastKernel<MAXM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(fsm));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(BeamReplayKernel<MAXM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(rsm));
}

}  // namespace

cudaError_t PrepareBeamKernels(const Dims& dims, int beam) {
    return dims.m <= 8 ? PrepareT<8>(dims, beam) : PrepareT<16>(dims, beam);
}

// redo: n + 1 ints of scratch (a count, then vector ids handed from the fast to the replay kernel).
cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, uint8_t* Bout, int* redo, int check,
                             unsigned int* err_flag, int num_sms, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    // The encoder's flag word is followed by four 64-bit counters (BeamStats).
    unsigned long long* stats = err_flag ? reinterpret_cast<unsigned long long*>(err_flag + 4) : nullptr;
    if (dims.m <= 8)
        return LaunchBeamT<8>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, redo, check, err_flag, stats, num_sms,
                              stream);
    return LaunchBeamT<16>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, redo, check, err_flag, stats, num_sms,
                           stream);
}

}  // namespace stlq_b200
