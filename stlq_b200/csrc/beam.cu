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
// exact errors (its slots hold them in ascending (error, scan index) order).  When an exact tie
// sits at the boundary (or at the final minimum), or the survivor list would overflow, the vector
// is handed to BeamReplayKernel.
//
// BeamReplayKernel replays the reference's replacement scan itself (warp 0, slots one per lane), so
// ties resolve exactly as in the reference; it evaluates exactly every candidate that the cheap
// bounds cannot exclude from entering the scan (ReplayLayer).
//
// The layer index is a run-time argument of every routine (see beam_common.cuh).
//
// STRICT mode (the kStrict instantiations): xC comes from the tensor cores and differs from the
// exact GEMM's by at most dg = kappa ||c|| ||x|| per entry.  Every bound is widened by that term
// (layer 0: Layer0Bounds; later layers: BoundsTail), and every value the selection or the
// outputs depend on -- the survivors' exact errors, the winners' state, the replay's scans -- is
// computed from the exact xC entry, recomputed on demand in the exact GEMM's order (ExactCtx::Gamma,
// with the vector staged in shared memory).  The codes are therefore the exact mode's.
#include <cstdint>

#include "beam_common.cuh"
#include "launch.h"

namespace stlq_b200 {

using namespace beam;

namespace {

constexpr int kSurvCap = 512;  // exactly evaluated survivors per layer in the fast kernel
constexpr int kKeep = 64;      // survivors whose exact-evaluation results are kept for Materialize

// The exact xC entry of flat codeword `flat`: the row itself (EXACT and FAST modes take xC as exact)
// or, in STRICT mode, recomputed in the exact GEMM's order.
template <bool kStrict>
__device__ __forceinline__ float ExactGamma(const ExactCtx& ctx, const float* xc, int flat) {
    if constexpr (kStrict) return ctx.Gamma(flat);
    else return __ldg(xc + flat);
}

// STRICT mode: the exact xC entries of the codewords flat_of(p), p < S, into gex[p], entry p by
// thread p % kThreads (the thread that uses it next).  Staging the rows in shared memory for
// coalesced loads was measured slower: the larger carve-out costs the cheap pass's Gram gathers
// their L1 hits.
template <class FlatOf>
__device__ __forceinline__ void SurvivorGammas(const ExactCtx& ctx, int S, FlatOf flat_of, float* gex) {
    for (int p = threadIdx.x; p < S; p += kThreads) gex[p] = ctx.Gamma(flat_of(p));
}

// Per kept survivor: y[MAXM], v[MAXM], denom, a_last.
template <int MAXM>
__host__ __device__ constexpr int KeepStride() { return 2 * MAXM + 2; }

// Floats of each candidate array of the replay kernel: beam x maxKs, at least 64 (STRICT mode's
// layer 0 splits the first array into a list and its errors, chunks of at least 32).
__host__ __device__ inline int ReplayCandFloats(int beam, int maxKs) { return beam * maxKs > 64 ? beam * maxKs : 64; }
__host__ __device__ inline int Align4(int d) { return (d + 3) & ~3; }

struct LayerTable {
    int cand[kMaxBeam];   // candidate (scan index) held by each slot, slot order
    int candp[kMaxBeam];  // fast kernel: the winner's position in the survivor list
    int n_slots;          // slots filled
    int n_surv;
    uint32_t key_b;       // fast kernel: error keys ranked B-1 and B (boundary tie test)
    uint32_t key_n;
    uint32_t mins[kWarps * kMaxBeam];  // each warp's B smallest per-thread upper bounds, sorted
};

// Copies the winners' state into the next slot buffer (beam_search.cpp:337-383): parent prefix of
// R, then each winner's own R column (y, sqrt(denom)), coefficients a_t - v_t a_last, a_last, code.
// With `keep` (fast kernel) a winner whose survivor position is below kKeep takes y, v, denom,
// a_last and its error from the exact evaluation already made; otherwise they are recomputed (in
// STRICT mode from the exact xC entry: the fast kernel's gex[survivor position], else recomputed).
template <int MAXM, bool kStrict>
__device__ void Materialize(const Dims& dims, int L, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt,
                            const LayerTable& lt, int newH, const float* __restrict__ Grow,
                            const float* __restrict__ Gdiag, const float* __restrict__ xc, const ExactCtx& ctx,
                            const float* keep = nullptr, const float* ex = nullptr, const float* gex = nullptr) {
    constexpr int NL = MAXM - 1;
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L], ldg = dims.ldg, colL = offL - dims.c0;
    // R prefix of each winner's parent: rows r <= c < L, one (winner, column) pair per thread.
    for (int e = tid; e < newH * L; e += kThreads) {
        const int o = e / L, c = e - o * L;
        const float* src = cur.Rh(lt.cand[o] / K) + c * MAXM;
        float* dst = nxt.Rh(o) + c * MAXM;
        for (int r = 0; r <= c; ++r) dst[r] = src[r];
    }
    if (tid < newH) {
        const int o = tid;
        const int idx = lt.cand[o];
        const int h = idx / K, k = idx - h * K;
        float y[NL], v[NL], denom, a_last, e;
        const float ak = __ldg(Gdiag + offL + k);
        const int p = keep ? lt.candp[o] : kKeep;
        if (p < kKeep) {
            const float* st = keep + p * KeepStride<MAXM>();
#pragma unroll
            for (int t = 0; t < NL; ++t) {
                y[t] = st[t];
                v[t] = st[MAXM + t];
            }
            denom = st[2 * MAXM];
            a_last = st[2 * MAXM + 1];
            e = ex[p];
        } else {
            float gamma;
            if constexpr (kStrict) gamma = gex ? gex[lt.candp[o]] : ctx.Gamma(offL + k);
            else gamma = __ldg(xc + offL + k);
            e = EvalExactL<MAXM>(cur, h, L, RowsOf<MAXM>(cur, h, L), Grow, ldg, colL + k, ak, gamma, y, v, &denom,
                                 &a_last, dims.large_root != 0);
        }
#pragma unroll
        for (int t = 0; t < NL; ++t) {
            if (t >= L) break;
            nxt.rowh(o)[t] = cur.rowh(h)[t];
            nxt.ah(o)[t] = sub_rn(cur.ah(h)[t], mul_rn(v[t], a_last));
            nxt.Rh(o)[L * MAXM + t] = y[t];
            nxt.rinvh(o)[t] = cur.rinvh(h)[t];
        }
        const float rll = __fsqrt_rn(denom);
        nxt.rowh(o)[L] = (offL + k) * ldg;
        nxt.ah(o)[L] = a_last;
        nxt.Rh(o)[L * MAXM + L] = rll;
        nxt.rinvh(o)[L] = __frcp_rn(rll);
        nxt.E[o] = e;
        nxt.ill[o] = cur.ill[h] | !(denom >= kIllCond * ak);
    }
}

// No finite candidate in a layer (beam_search.cpp:385-400): the previous slots are kept.  The code
// of this layer is written as 0 (Grow row row0 = offL * ldg); the reference copies a stale buffer
// value there.
template <int MAXM>
__device__ int KeepPrevious(int L, int row0, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int curH,
                            int beam) {
    const int tid = threadIdx.x;
    const int keep = min(curH, beam);
    for (int e = tid; e < keep * MAXM * MAXM; e += kThreads) nxt.R[e] = cur.R[e];
    for (int e = tid; e < keep * MAXM; e += kThreads) {
        const int t = e % MAXM;
        nxt.row[e] = t < L ? cur.row[e] : row0;
        nxt.a[e] = t < L ? cur.a[e] : 0.0f;
        nxt.rinv[e] = cur.rinv[e];
    }
    for (int h = tid; h < keep; h += kThreads) {
        nxt.E[h] = cur.E[h];
        nxt.ill[h] = cur.ill[h];
    }
    return max(1, keep);
}

// Layer 0 state of slot o holding codeword k with exact xC entry gamma (beam_search.cpp:248-258).
template <int MAXM>
__device__ void InitSlot0(const SlotView<MAXM>& s, int o, int k, int ldg, const float* Gdiag, float gamma,
                          float nx2) {
    const float alpha = __ldg(Gdiag + k);
    const float a1 = div_rn(gamma, alpha);
    const float r00 = __fsqrt_rn(alpha);
    s.rowh(o)[0] = k * ldg;  // layer 0 starts at flat index 0
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
__device__ void DeadSlot0(const Dims& dims, const SlotView<MAXM>& s) {
    const int tid = threadIdx.x;
    if (tid < MAXM) {
        s.rowh(0)[tid] = tid < dims.m ? dims.off[tid] * dims.ldg : 0;
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
__device__ __forceinline__ float Layer0ErrorG(const float* Gdiag, float gamma, float nx2, int k) {
    const float alpha = __ldg(Gdiag + k);
    const float e1 = sub_rn(nx2, mul_rn(gamma, div_rn(gamma, alpha)));
    return (alpha != 0.0f && e1 < PosInf()) ? e1 : PosInf();
}
__device__ __forceinline__ float Layer0Error(const float* Gdiag, const float* xc, float nx2, int k) {
    return Layer0ErrorG(Gdiag, __ldg(xc + k), nx2, k);
}

// STRICT mode: bounds [lo, hi] on Layer0Error of codeword k from the tensor-core entry g (the exact
// one lies within dg of it): e1 = nx2 - g^2/alpha over |g| in [|g| - dg, |g| + dg], widened by
// 1e-6 (|nx2| + q_max), far more than the roundings of both this and the exact sequence.  A zero
// codeword (skipped by the reference) gets [+inf, +inf]; anything non-finite [-inf, +inf].
__device__ __forceinline__ void Layer0Bounds(const float* Gdiag, const float* xc, const ExactCtx& ctx, float nx2,
                                             int k, float& lo, float& hi) {
    const float alpha = __ldg(Gdiag + k);
    if (alpha == 0.0f) {
        lo = hi = PosInf();
        return;
    }
    const float ag = fabsf(__ldg(xc + k)), dg = ctx.Bound(k);
    const float gmax = ag + dg, gmin = fmaxf(ag - dg, 0.0f);
    const float qmax = gmax * gmax / alpha, qmin = gmin * gmin / alpha;
    const float slack = 1e-6f * (fabsf(nx2) + qmax);
    lo = (nx2 - qmax) - slack;
    hi = (nx2 - qmin) + slack;
    if (!(lo == lo) || !(hi == hi) || !(slack < PosInf())) {
        lo = -PosInf();
        hi = PosInf();
    }
}

// STRICT mode, a root too large to keep one bound per codeword: lower bounds recomputed where the
// selection reads them.
struct Layer0LoSource {
    const float* Gdiag;
    const float* xc;
    ExactCtx ctx;
    float nx2;
    static constexpr bool kVec = false;
    __device__ float operator()(int k) const {
        float lo, hi;
        Layer0Bounds(Gdiag, xc, ctx, nx2, k, lo, hi);
        return lo;
    }
    __device__ const float* v0() const { return nullptr; }
};

// Where the selection reads a candidate's error (or lower bound): a shared-memory array
// (16-byte aligned, read four at a time), or, for a layer-0 codebook too large to keep one float
// per codeword, recomputed from xC.
struct ArraySource {
    const float* v;
    static constexpr bool kVec = true;
    __device__ float operator()(int idx) const { return v[idx]; }
    __device__ const float* v0() const { return v; }
};
struct Layer0Source {
    const float* Gdiag;
    const float* xc;
    float nx2;
    static constexpr bool kVec = false;
    __device__ float operator()(int k) const { return Layer0Error(Gdiag, xc, nx2, k); }
    __device__ const float* v0() const { return nullptr; }  // no array: never read four at a time
};

// A thread's two smallest upper bounds as selection keys: the smallest in the low word.
__device__ __forceinline__ uint64_t BoundKeys(float h1, float h2) {
    return (static_cast<uint64_t>(OrderKey(h2)) << 32) | OrderKey(h1);
}

// ---------------------------------------------------------------------------------------------
// Cheap pass shared by both kernels.

// Self-check of the cheap bounds (STLQ_B200_CHECK_FILTER): the exact error of each candidate must
// lie inside them; a miss raises kErrFilterMiss.  Inlined: a call site inside the hot loop, even
// one never taken, costs the loop registers.
// In STRICT mode the exact error comes from the exact xC entry (flat index = Gram column + coff).
template <int MAXM, bool kStrict>
__device__ __forceinline__ void CheckBounds(const SlotView<MAXM> cur, int h, int L, const float* __restrict__ Grow, int ldg,
                                         const int (&col)[kCpt], const bool (&ok)[kCpt], const float (&alpha)[kCpt],
                                         const float (&gamma)[kCpt], const float (&l)[kCpt], const float (&hi)[kCpt],
                                         unsigned int* err_flag, bool recip, const ExactCtx& ctx, int coff) {
    const RowArr<MAXM> flat = RowsOf<MAXM>(cur, h, L);
    for (int c = 0; c < kCpt; ++c) {
        if (!ok[c]) continue;
        float g = gamma[c];
        if constexpr (kStrict) g = ctx.Gamma(col[c] + coff);
        const float e = EvalExactL<MAXM>(cur, h, L, flat, Grow, ldg, col[c], alpha[c], g, nullptr, nullptr,
                                         nullptr, nullptr, recip);
        if (e < PosInf() && !(e >= l[c] && e <= hi[c])) atomicOr(err_flag, kErrFilterMiss);
    }
}

// The cheap pass of layer L over every live slot: lower bounds into lo[h * K + k] (with kHi also
// the upper bounds into hi_out), and the thread's smallest upper bound as the return value.  One
// inlined copy serves every layer (L at run time): per-layer copies, fully unrolled, ran 11%
// slower at M = 8 because together they overflow the instruction cache; out of line, the call
// boundary's register saves cost more still.
template <int MAXM, bool kHi, bool kWide, bool kStrict>
__device__ __forceinline__ uint64_t CheapPass(const SlotView<MAXM> cur, int L, int curH, int K, int offL, int colL,
                                           const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                                           const float* __restrict__ xc, float* lo, float* hi_out, int check,
                                           unsigned int* err_flag, bool recip, const ExactCtx& ctx) {
    const int tid = threadIdx.x;
    float hmin = PosInf(), hmin2 = PosInf();  // never NaN: a bound is finite or +-inf
    // Codebooks above 256 codewords (the kWide kernels) are walked in chunks of kMaxK, kCpt
    // codewords per thread; the other kernels make one pass with kc = 0 known at compile time.
    for (int kc = 0; kc < (kWide ? K : 1); kc += kMaxK) {
        float alpha[kCpt], gamma[kCpt], dg[kCpt];
        int col[kCpt];
        bool ok[kCpt];
#pragma unroll
        for (int c = 0; c < kCpt; ++c) {
            const int k = kc + tid + c * kThreads;
            ok[c] = k < K;
            col[c] = colL + k;  // Gram column; Gdiag and xc are indexed by the flat index
            alpha[c] = ok[c] ? __ldg(Gdiag + offL + k) : 0.0f;
            gamma[c] = ok[c] ? __ldg(xc + offL + k) : 0.0f;
            dg[c] = (kStrict && ok[c]) ? ctx.Bound(offL + k) : 0.0f;
        }
        const float* gq[kCpt];
#pragma unroll
        for (int c = 0; c < kCpt; ++c) gq[c] = Grow + col[c];
        for (int h = 0; h < curH; ++h) {
            float l[kCpt], hi[kCpt];
            CheapBounds<MAXM, kStrict>(cur, h, L, gq, ok, alpha, gamma, dg, l, hi);
#pragma unroll
            for (int c = 0; c < kCpt; ++c) {
                if (ok[c]) {
                    lo[h * K + kc + tid + c * kThreads] = l[c];
                    if (kHi) hi_out[h * K + kc + tid + c * kThreads] = hi[c];
                    hmin2 = fminf(hmin2, fmaxf(hmin, hi[c]));
                    hmin = fminf(hmin, hi[c]);
                }
            }
            if (check)
                CheckBounds<MAXM, kStrict>(cur, h, L, Grow, 0, col, ok, alpha, gamma, l, hi, err_flag, recip, ctx,
                                           offL - colL);
        }
    }
    return BoundKeys(hmin, hmin2);
}

template <int MAXM, bool kHi, bool kWide, bool kStrict>
__device__ uint64_t CheapDispatch(int L, const SlotView<MAXM>& cur, int curH, int K, int offL, int colL,
                                  const float* Grow, const float* Gdiag, const float* xc, float* lo, float* hi_out,
                                  int check, unsigned int* err, bool recip, const ExactCtx& ctx) {
    return CheapPass<MAXM, kHi, kWide, kStrict>(cur, L, curH, K, offL, colL, Grow, Gdiag, xc, lo, hi_out, check, err,
                                                recip, ctx);
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
    // Scans errors 0..n of `src` in order: one ballot per 32 candidates, entering ones replayed in
    // order.
    template <class Src>
    __device__ void Scan(Src src, int n) {
        const int lane = threadIdx.x & 31;
        for (int base = 0; base < n; base += 32) {
            const float e = base + lane < n ? src(base + lane) : PosInf();
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
    // Scan over the candidates list[0..n) only (their indices, in scan order), every other
    // candidate's error being +inf: +inf never enters (it is not below any worst), so the
    // replacement history, slot order included, is Scan's over all candidates.
    __device__ void ScanList(const float* errs, const int* list, int n) {
        const int lane = threadIdx.x & 31;
        for (int base = 0; base < n; base += 32) {
            const int idx = base + lane < n ? list[base + lane] : -1;
            const float e = idx >= 0 ? errs[idx] : PosInf();
            unsigned mask = __ballot_sync(kFull, e < worst);
            while (mask) {
                const int l = __ffs(mask) - 1;
                mask &= mask - 1;
                const float el = __shfl_sync(kFull, e, l);
                const int il = __shfl_sync(kFull, idx, l);
                if (el < worst) {
                    if (lane == widx) {
                        es = el;
                        cs = il;
                    }
                    Refresh();
                }
            }
        }
    }
    // Pre-scan on the cheap bounds.  Scanning hi[] with the same rule makes `worst` the B-th
    // smallest upper bound of the prefix, an upper bound of the exact scan's worst at the same
    // position (each exact error is <= its hi).  A candidate whose lo is not below that bound at the
    // start of its 32-candidate batch can never enter the exact scan: its error is set to +inf in
    // lo[] and it needs no exact evaluation.  The others keep their lo and their indices are
    // appended to list[] (which may overwrite hi[] entries already consumed).  Returns their count.
    __device__ int PreScan(float* lo, float* hi, int n, int* list) {
        const int lane = threadIdx.x & 31;
        int count = 0;
        for (int base = 0; base < n; base += 32) {
            const bool in = base + lane < n;
            const float h = in ? hi[base + lane] : PosInf();
            const float l = in ? lo[base + lane] : PosInf();
            const bool need = in && l < worst;
            __syncwarp();  // every lane has read its batch entries before list[] overwrites them
            const unsigned nm = __ballot_sync(kFull, need);
            if (need) list[count + __popc(nm & ((1u << lane) - 1u))] = base + lane;
            else if (in) lo[base + lane] = PosInf();
            count += __popc(nm);
            unsigned mask = __ballot_sync(kFull, h < worst);
            while (mask) {
                const int b = __ffs(mask) - 1;
                mask &= mask - 1;
                const float hb = __shfl_sync(kFull, h, b);
                if (hb < worst) {
                    if (lane == widx) es = hb;
                    Refresh();
                }
            }
        }
        return count;
    }
    // PreScan over candidates [base0, base0 + n) whose bounds src(idx, lo, hi) computes: the indices
    // of the candidates that can enter are written to list[] (in scan order); returns their count.
    // Called chunk after chunk, the state carries over, so the chunks together are one pre-scan.
    template <class Src>
    __device__ int PreScanFn(Src src, int base0, int n, int* list) {
        const int lane = threadIdx.x & 31;
        int count = 0;
        for (int b = 0; b < n; b += 32) {
            const bool in = b + lane < n;
            float l = PosInf(), h = PosInf();
            if (in) src(base0 + b + lane, l, h);
            const bool need = in && l < worst;
            const unsigned nm = __ballot_sync(kFull, need);
            if (need) list[count + __popc(nm & ((1u << lane) - 1u))] = base0 + b + lane;
            count += __popc(nm);
            unsigned mask = __ballot_sync(kFull, h < worst);
            while (mask) {
                const int q = __ffs(mask) - 1;
                mask &= mask - 1;
                const float hq = __shfl_sync(kFull, h, q);
                if (hq < worst) {
                    if (lane == widx) es = hq;
                    Refresh();
                }
            }
        }
        return count;
    }
    // ScanList with the errors stored by list position (exl[p] is the error of candidate list[p]).
    __device__ void ScanListPos(const float* exl, const int* list, int n) {
        const int lane = threadIdx.x & 31;
        for (int base = 0; base < n; base += 32) {
            const bool in = base + lane < n;
            const int idx = in ? list[base + lane] : -1;
            const float e = in ? exl[base + lane] : PosInf();
            unsigned mask = __ballot_sync(kFull, e < worst);
            while (mask) {
                const int l = __ffs(mask) - 1;
                mask &= mask - 1;
                const float el = __shfl_sync(kFull, e, l);
                const int il = __shfl_sync(kFull, idx, l);
                if (el < worst) {
                    if (lane == widx) {
                        es = el;
                        cs = il;
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

// One layer of the replay: cheap bounds for every candidate, the pre-scan that finds the
// candidates able to enter, exact errors for those only (all others are +inf, which enters no
// slot), then the reference's replacement scan over the exact errors.  Without room for the upper
// bounds (his == nullptr: beam x codebook size too large for shared memory) every candidate is
// evaluated exactly; the scan's result is the same.
template <int MAXM, bool kWide, bool kStrict>
__device__ void ReplayLayer(const Dims& dims, int L, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int& curH,
                            const float* __restrict__ Grow, const float* __restrict__ Gdiag,
                            const float* __restrict__ xc, int beam, float* errs, float* his, LayerTable& lt,
                            const ExactCtx& ctx) {
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L], colL = offL - dims.c0;
    const int n_cand = curH * K;
    int* list = reinterpret_cast<int*>(his);
    if (his) {
        CheapDispatch<MAXM, true, kWide, kStrict>(L, cur, curH, K, offL, colL, Grow, Gdiag, xc, errs, his, 0, nullptr,
                                                  dims.large_root != 0, ctx);
        __syncthreads();
        if (tid < 32) {
            Replay rp;
            rp.Init(beam);
            const int need = rp.PreScan(errs, his, n_cand, list);
            if (tid == 0) lt.n_surv = need;
        }
        __syncthreads();
    }
    const int need = his ? lt.n_surv : n_cand;
    for (int p = tid; p < need; p += kThreads) {
        const int idx = his ? list[p] : p;
        const int h = idx / K, k = idx - h * K;
        errs[idx] = EvalExactL<MAXM>(cur, h, L, RowsOf<MAXM>(cur, h, L), Grow, dims.ldg, colL + k, __ldg(Gdiag + offL + k),
                                     ExactGamma<kStrict>(ctx, xc, offL + k), nullptr, nullptr, nullptr, nullptr,
                                     dims.large_root != 0);
    }
    __syncthreads();
    if (tid < 32) {
        Replay rp;
        rp.Init(beam);
        if (his) rp.ScanList(errs, list, need);  // the pre-scan's candidates, in scan order
        else rp.Scan(ArraySource{errs}, n_cand);
        rp.Publish(beam, lt);
    }
    __syncthreads();
    const int newH = lt.n_slots;
    if (newH == 0) {
        curH = KeepPrevious<MAXM>(L, offL * dims.ldg, cur, nxt, curH, beam);
    } else {
        Materialize<MAXM, kStrict>(dims, L, cur, nxt, lt, newH, Grow, Gdiag, xc, ctx);
        curH = newH;
    }
    __syncthreads();
}

// STRICT mode, layer 0 of the replay: the pre-scan over the layer-0 bounds (computed where they
// are read, so the root may be of any size), in chunks of `ch` candidates: each chunk's entering
// candidates are listed (list[0..ch)), evaluated exactly (exl[0..ch)) and scanned.  The two scans'
// states carry over from chunk to chunk, so the result is the scan over all K0 exact errors.
// Fills lt.cand / lt.n_slots like Replay::Publish.
__device__ void ReplayLayer0Strict(const float* __restrict__ Gdiag, const float* __restrict__ xc, float nx2, int K0,
                                   int beam, int* list, float* exl, int ch, LayerTable& lt, const ExactCtx& ctx) {
    const int tid = threadIdx.x;
    Replay pre, scan;  // used by warp 0 only
    if (tid < 32) {
        pre.Init(beam);
        scan.Init(beam);
    }
    auto bounds = [&](int k, float& lo, float& hi) { Layer0Bounds(Gdiag, xc, ctx, nx2, k, lo, hi); };
    for (int base = 0; base < K0; base += ch) {
        const int n = min(ch, K0 - base);
        if (tid < 32) {
            const int cnt = pre.PreScanFn(bounds, base, n, list);
            if (tid == 0) lt.n_surv = cnt;
        }
        __syncthreads();
        const int cnt = lt.n_surv;
        for (int p = tid; p < cnt; p += kThreads) exl[p] = Layer0ErrorG(Gdiag, ctx.Gamma(list[p]), nx2, list[p]);
        __syncthreads();
        if (tid < 32) scan.ScanListPos(exl, list, cnt);
        __syncthreads();
    }
    if (tid < 32) scan.Publish(beam, lt);
    __syncthreads();
}

// Encodes the vectors listed in vec_list[0 .. *count) (or 0 .. n when vec_list is null).  kWide
// (BigCodebooks): a codebook of layers 1..m-1 has more than kMaxK codewords, or layer 0's errors do
// not fit the candidate array; the other kernels, the common sizes, compile neither case in.
template <class T>
__device__ __forceinline__ T* Align16(void* p) {
    return reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
}

// STRICT mode: stages vector `vec` as float in xs (d floats) and returns its exact-entry context.
__device__ __forceinline__ ExactCtx StageVector(const ExactDotArgs& ea, const Dims& dims, int64_t vec,
                                                const float* xc, float nx2, float* xs, unsigned int* err) {
    const int d = dims.d;
    if (ea.x_dtype == 0) {
        const float* xv = static_cast<const float*>(ea.X) + vec * d;
        for (int i = threadIdx.x; i < d; i += kThreads) xs[i] = xv[i];
    } else {
        const uint8_t* xv = static_cast<const uint8_t*>(ea.X) + vec * d;
        for (int i = threadIdx.x; i < d; i += kThreads) xs[i] = static_cast<float>(xv[i]);
    }
    return ExactCtx{ea.C, ea.cn, xc, xs, d, StrictKx(ea.kappa, nx2), err};
}

template <int MAXM, bool kWide, bool kStrict>
__global__ void __launch_bounds__(kThreads) BeamReplayKernel(Dims dims, const float* __restrict__ Grow,
                                                             const float* __restrict__ Gdiag,
                                                             const float* __restrict__ xnorm2,
                                                             const float* __restrict__ xC, int64_t n, int beam,
                                                             void* __restrict__ Bout, const int* vec_list,
                                                             const int* count, bool prescan, ExactDotArgs ea,
                                                             unsigned int* err_flag) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t sv = SlotView<MAXM>::Bytes(beam);
    size_t off = (2 * sv + 15) & ~size_t(15);
    LayerTable& lt = *reinterpret_cast<LayerTable*>(smem + off);
    float* errs = reinterpret_cast<float*>(smem + ((off + sizeof(LayerTable) + 15) & ~size_t(15)));
    const int nc = ReplayCandFloats(beam, dims.maxKs);
    float* his = prescan ? errs + nc : nullptr;
    float* after = errs + (prescan ? 2 : 1) * nc;
    float* xs = Align16<float>(after);  // STRICT: the vector being encoded
    const int tid = threadIdx.x;
    const int m = dims.m, K0 = dims.h_vec[0];
    const int64_t total = vec_list ? static_cast<int64_t>(*count) : n;
    for (int64_t i = blockIdx.x; i < total; i += gridDim.x) {
        const int64_t vec = vec_list ? vec_list[i] : i;
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        ExactCtx ctx{};
        if constexpr (kStrict) {
            ctx = StageVector(ea, dims, vec, xc, nx2, xs, err_flag);
            ReplayLayer0Strict(Gdiag, xc, nx2, K0, beam, reinterpret_cast<int*>(errs), errs + (nc / 2 & ~31),
                               nc / 2 & ~31, lt, ctx);
        } else {
            // Layer 0 keeps its errors in errs[] when they fit (beam x maxKs floats), else recomputes them.
            const bool stored0 = !kWide || K0 <= beam * dims.maxKs;
            if (stored0)
                for (int k = tid; k < K0; k += kThreads) errs[k] = Layer0Error(Gdiag, xc, nx2, k);
            __syncthreads();
            if (tid < 32) {
                Replay rp;
                rp.Init(beam);
                if constexpr (kWide) {
                    if (stored0) rp.Scan(ArraySource{errs}, K0);
                    else rp.Scan(Layer0Source{Gdiag, xc, nx2}, K0);
                } else {
                    rp.Scan(ArraySource{errs}, K0);
                }
                rp.Publish(beam, lt);
            }
            __syncthreads();
        }
        int curH = lt.n_slots;
        const SlotView<MAXM> s0 = SlotView<MAXM>::At(smem, beam);
        if (tid < curH) InitSlot0<MAXM>(s0, tid, lt.cand[tid], dims.ldg, Gdiag, ExactGamma<kStrict>(ctx, xc, lt.cand[tid]), nx2);
        if (curH == 0) {
            DeadSlot0<MAXM>(dims, s0);
            curH = 1;
        }
        __syncthreads();
        int ci = 0;
        for (int L = 1; L < m; ++L) {
            ReplayLayer<MAXM, kWide, kStrict>(dims, L, SlotView<MAXM>::At(smem + ci * sv, beam),
                                              SlotView<MAXM>::At(smem + (ci ^ 1) * sv, beam), curH, Grow, Gdiag, xc,
                                              beam, errs, his, lt, ctx);
            ci ^= 1;
        }
        if (tid < 32) {  // first slot with the smallest error (beam_search.cpp:409-416)
            const SlotView<MAXM> cur = SlotView<MAXM>::At(smem + ci * sv, beam);
            const uint32_t key = tid < curH ? OrderKey(cur.E[tid]) : 0xffffffffu;
            const uint32_t kmin = __reduce_min_sync(kFull, key);
            const int best = __ffs(__ballot_sync(kFull, key == kmin)) - 1;
            if (tid < m) StoreCode(Bout, vec * m + tid, cur.rowh(best)[tid] / dims.ldg - dims.off[tid], dims.wide);
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
// layer.  Inputs: src(idx) (a lower bound of each candidate's exact error; the exact error itself
// in layer 0) and `hmin`, this thread's two smallest upper bounds as order keys (BoundKeys).  The
// 256 values belong to distinct candidates, so their B-th smallest, tau, bounds the B-th smallest
// exact error from above; every candidate with lo <= tau is a survivor (all others are provably
// larger than the B-th smallest exact error).  Two values per thread rather than one cut the
// survivors per layer from 44 to 27 at the benchmark shape.  Returns the survivor count, or -1
// when the list overflows.
template <class Src>
__device__ __noinline__ int SelectSurvivors(Src src, int n_cand, uint64_t hmin, int beam, LayerTable& lt,
                                            uint16_t* surv) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Each warp sorts its 32 minima; only a warp's B smallest can be among the B smallest of all
    // 128, so ranking those 4B values (binary search into the other sorted lists) finds tau.  Every
    // warp does it, so tau needs no second barrier.
    // Each thread gives its two smallest upper bounds (distinct candidates): the warp's 32 smallest
    // of its 64 are min(a[i], b[31 - i]) of the two sorted lists, a bitonic sequence, then sorted.
    const uint32_t sa = WarpSortAsc(static_cast<uint32_t>(hmin));
    const uint32_t sb = __shfl_sync(kFull, WarpSortAsc(static_cast<uint32_t>(hmin >> 32)), 31 - lane);
    uint32_t sorted = min(sa, sb);
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const uint32_t o = __shfl_xor_sync(kFull, sorted, j);
        sorted = (lane & j) ? max(sorted, o) : min(sorted, o);
    }
    if (lane < beam) lt.mins[warp * kMaxBeam + lane] = sorted;
    if (tid == 0) lt.n_surv = 0;
    __syncthreads();
    // Rank of value v (list w, position j) among all 4B values: j plus, in each other list, the
    // number of entries ordered before it (ties broken by list index).  The searches over the
    // other lists are independent: fixed-step binary searches, interleaved.
    uint32_t tb = 0xffffffffu;
    for (int i = lane; i < kWarps * beam; i += 32) {
        const int w = i / beam, j = i - w * beam;
        const uint32_t v = lt.mins[w * kMaxBeam + j];
        int pos[kWarps];
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) pos[w2] = 0;
#pragma unroll
        for (int step = kMaxBeam; step > 0; step >>= 1) {  // counts up to 2 * kMaxBeam - 1 >= beam
#pragma unroll
            for (int w2 = 0; w2 < kWarps; ++w2) {
                const int t = pos[w2] + step;  // entries [0, pos) are known to come before v
                if (t <= beam) {
                    const uint32_t u = lt.mins[w2 * kMaxBeam + t - 1];
                    if (u < v || (u == v && w2 < w)) pos[w2] = t;
                }
            }
        }
        int r = j;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) r += w2 == w ? 0 : pos[w2];
        if (r == beam - 1) tb = v;
    }
    tb = __reduce_min_sync(kFull, tb);
    const float tau = tb >= OrderKey(PosInf()) ? PosInf() : KeyToFloat(tb);  // < B finite bounds: keep all
    // One pass: each thread marks its survivors among up to 32 candidates per round (eight 128-bit
    // loads), the warp scans the counts and reserves its range of the list with one atomic, and
    // the marked candidates are written there.  The list's order does not matter: survivors are
    // ranked by (exact error, scan index), which is unique.
    const float4* lo4 = reinterpret_cast<const float4*>(src.v0());
    const int n4 = Src::kVec ? n_cand >> 2 : 0;
    const auto emit = [&](uint32_t mask, auto idx_of) {
        const int cnt = __popc(mask);
        int incl = cnt;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(kFull, incl, d);
            if (lane >= d) incl += o;
        }
        int base = 0;
        if (lane == 31 && incl > 0) base = atomicAdd(&lt.n_surv, incl);
        base = __shfl_sync(kFull, base, 31);
        int p = base + incl - cnt;
        if (p + cnt <= kSurvCap) {
            while (mask) {
                const int b = __ffs(mask) - 1;
                mask &= mask - 1;
                surv[p++] = static_cast<uint16_t>(idx_of(b));
            }
        }
    };
    // Rounds are warp-uniform: every lane takes part in each round's scan.
    for (int c0 = warp * 32; c0 < n4; c0 += 8 * kThreads) {
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = c0 + j * kThreads + lane;
            if (c < n4) {
                const float4 v = lo4[c];
                mask |= ((v.x <= tau) | ((v.y <= tau) << 1) | ((v.z <= tau) << 2) | ((v.w <= tau) << 3)) << (4 * j);
            }
        }
        emit(mask, [&](int b) { return 4 * (c0 + (b >> 2) * kThreads + lane) + (b & 3); });
    }
    for (int i0 = 4 * n4 + warp * 32; i0 < n_cand; i0 += 32 * kThreads) {
        uint32_t mask = 0;
        for (int j = 0; j < 32; ++j) {
            const int idx = i0 + j * kThreads + lane;
            if (idx < n_cand && src(idx) <= tau) mask |= 1u << j;
        }
        emit(mask, [&](int b) { return i0 + b * kThreads + lane; });
    }
    __syncthreads();
    const int S = lt.n_surv;
    return S > kSurvCap ? -1 : S;
}

// Survivor sort key: (error, scan index, survivor position); the scan index makes it unique.
__device__ __forceinline__ uint64_t SurvKey(float e, int idx, int p) {
    return (static_cast<uint64_t>(OrderKey(e)) << 32) | (static_cast<uint32_t>(idx) << 9) | static_cast<uint32_t>(p);
}

// Ranks the S survivors by (exact error, scan index) and fills lt.cand / lt.candp with the B
// smallest in that order.  Returns the slot count, or -1 when an exact tie sits at the selection
// boundary.  keys: kSurvCap 64-bit words of scratch.
__device__ __noinline__ int RankSurvivors(const float* ex, const uint16_t* surv, int S, int beam, LayerTable& lt,
                                          uint64_t* keys) {
    const int tid = threadIdx.x;
    constexpr uint64_t kInvalid = static_cast<uint64_t>(0xff800000u) << 32;  // OrderKey(+inf)
    for (int p = tid; p < S; p += kThreads) keys[p] = SurvKey(ex[p], surv[p], p);
    if (tid == 0) {
        lt.n_slots = 0;
        lt.key_b = 0u;
        lt.key_n = 1u;
    }
    __syncthreads();
    int my_valid = 0;
    for (int p = tid; p < S; p += kThreads) {
        const uint64_t kp = keys[p];
        int r = 0;
        for (int q = 0; q < S; ++q) r += keys[q] < kp;
        const bool valid = kp < kInvalid;
        my_valid += valid;
        if (valid && r < beam) {
            lt.cand[r] = static_cast<int>(static_cast<uint32_t>(kp) >> 9);
            lt.candp[r] = p;
        }
        if (r == beam - 1) lt.key_b = static_cast<uint32_t>(kp >> 32);
        if (r == beam) lt.key_n = static_cast<uint32_t>(kp >> 32);
    }
    if (my_valid) atomicAdd(&lt.n_slots, my_valid);
    __syncthreads();
    const int n_valid = lt.n_slots;
    // Tie at the boundary: the survivor ranked B has the B-th smallest error's exact value.
    if (n_valid > beam && lt.key_b == lt.key_n) return -1;
    return min(n_valid, beam);
}

// gex (STRICT): the survivors' exact xC entries by survivor position, for Materialize.
template <int MAXM, bool kWide, bool kStrict>
__device__ int FastLayer(const Dims& dims, int L, const SlotView<MAXM>& cur, const SlotView<MAXM>& nxt, int curH,
                         const float* __restrict__ Grow, const float* __restrict__ Gdiag, const float* __restrict__ xc,
                         int beam, float* lo, LayerTable& lt, uint16_t* surv, float* ex, uint64_t* keys, float* keep,
                         int check, unsigned int* err_flag, const ExactCtx& ctx, float* gex) {
    const int tid = threadIdx.x;
    const int K = dims.h_vec[L], offL = dims.off[L], colL = offL - dims.c0;
    const uint64_t hmin = CheapDispatch<MAXM, false, kWide, kStrict>(
        L, cur, curH, K, offL, colL, Grow, Gdiag, xc, lo, nullptr, check, err_flag, dims.large_root != 0, ctx);
    const int S = SelectSurvivors(ArraySource{lo}, curH * K, hmin, beam, lt, surv);
    if (S < 0) return -1;
    if constexpr (kStrict)
        SurvivorGammas(ctx, S, [&](int p) { return offL + surv[p] % K; }, gex);
    for (int p = tid; p < S; p += kThreads) {
        const int idx = surv[p];
        const int h = idx / K, k = idx - h * K;
        float* st = keep + p * KeepStride<MAXM>();
        const bool kp = p < kKeep;
        const float gamma = kStrict ? gex[p] : __ldg(xc + offL + k);
        ex[p] = EvalExactL<MAXM>(cur, h, L, RowsOf<MAXM>(cur, h, L), Grow, dims.ldg, colL + k, __ldg(Gdiag + offL + k),
                                 gamma, kp ? st : nullptr, kp ? st + MAXM : nullptr,
                                 kp ? st + 2 * MAXM : nullptr, kp ? st + 2 * MAXM + 1 : nullptr, dims.large_root != 0);
    }
    __syncthreads();
    const int newH = RankSurvivors(ex, surv, S, beam, lt, keys);
    if (newH < 0) return -1;
    if (newH == 0) {
        const int kept = KeepPrevious<MAXM>(L, offL * dims.ldg, cur, nxt, curH, beam);
        __syncthreads();
        return kept;
    }
    Materialize<MAXM, kStrict>(dims, L, cur, nxt, lt, newH, Grow, Gdiag, xc, ctx, keep, ex, kStrict ? gex : nullptr);
    __syncthreads();
    return newH;
}

template <int MAXM, bool kWide, bool kStrict>
__global__ void __launch_bounds__(kThreads, MAXM <= 8 ? 4 : 2) BeamFastKernel(Dims dims, const float* __restrict__ Grow,
                                                           const float* __restrict__ Gdiag,
                                                           const float* __restrict__ xnorm2,
                                                           const float* __restrict__ xC, int64_t n, int beam,
                                                           void* __restrict__ Bout, int* redo_list, int* redo_count,
                                                           int check, unsigned int* err_flag,
                                                           unsigned long long* stats, ExactDotArgs ea) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t sv = SlotView<MAXM>::Bytes(beam);
    size_t off = (2 * sv + 15) & ~size_t(15);
    LayerTable& lt = *reinterpret_cast<LayerTable*>(smem + off);
    off = (off + sizeof(LayerTable) + 15) & ~size_t(15);
    uint64_t* keys = reinterpret_cast<uint64_t*>(smem + off);
    float* lo = reinterpret_cast<float*>(keys + kSurvCap);
    float* ex = lo + beam * dims.maxKs;
    float* keep = ex + kSurvCap;
    uint16_t* surv = reinterpret_cast<uint16_t*>(keep + kKeep * KeepStride<MAXM>());
    // STRICT: the vector being encoded, then the survivors' exact xC entries.
    float* xs = Align16<float>(surv + kSurvCap);
    float* gex = xs + Align4(dims.d);
    const int tid = threadIdx.x;
    const int m = dims.m, K0 = dims.h_vec[0];
    unsigned long long n_surv = 0, n_layers = 0, n_vec = 0, n_redo = 0;  // thread 0's tallies
    for (int64_t vec = blockIdx.x; vec < n; vec += gridDim.x) {
        const float* xc = xC + vec * dims.H;
        const float nx2 = __ldg(xnorm2 + vec);
        // Layer 0 errors are kept in lo[] when they fit (beam x maxKs floats), else recomputed
        // where the selection reads them.
        const bool stored0 = !kWide || K0 <= beam * dims.maxKs;
        uint32_t hmin = 0xffffffffu, hmin2 = 0xffffffffu;  // the thread's two smallest bound keys
        ExactCtx ctx{};
        int curH;
        if constexpr (kStrict) {
            // Bounds from the tensor-core entries; the survivors' errors exactly.
            ctx = StageVector(ea, dims, vec, xc, nx2, xs, err_flag);
            if (check) __syncthreads();  // the self-check below reads the staged vector
            for (int k = tid; k < K0; k += kThreads) {
                float l, h;
                Layer0Bounds(Gdiag, xc, ctx, nx2, k, l, h);
                if (stored0) lo[k] = l;
                hmin2 = min(hmin2, max(hmin, OrderKey(h)));
                hmin = min(hmin, OrderKey(h));
                if (check) {
                    const float e = Layer0ErrorG(Gdiag, ctx.Gamma(k), nx2, k);
                    if (e < PosInf() && !(e >= l && e <= h)) atomicOr(err_flag, kErrFilterMiss);
                }
            }
            const uint64_t keys0 = (static_cast<uint64_t>(hmin2) << 32) | hmin;
            if constexpr (kWide)
                curH = stored0 ? SelectSurvivors(ArraySource{lo}, K0, keys0, beam, lt, surv)
                               : SelectSurvivors(Layer0LoSource{Gdiag, xc, ctx, nx2}, K0, keys0, beam, lt, surv);
            else
                curH = SelectSurvivors(ArraySource{lo}, K0, keys0, beam, lt, surv);
            if (curH >= 0) {
                SurvivorGammas(ctx, curH, [&](int p) { return static_cast<int>(surv[p]); }, gex);
                for (int p = tid; p < curH; p += kThreads) ex[p] = Layer0ErrorG(Gdiag, gex[p], nx2, surv[p]);
                __syncthreads();
                curH = RankSurvivors(ex, surv, curH, beam, lt, keys);
            }
        } else {
            // Exact errors are cheap here; they serve as their own bounds.
            for (int k = tid; k < K0; k += kThreads) {
                const float e1 = Layer0Error(Gdiag, xc, nx2, k);
                if (stored0) lo[k] = e1;
                hmin2 = min(hmin2, max(hmin, OrderKey(e1)));
                hmin = min(hmin, OrderKey(e1));
            }
            const uint64_t keys0 = (static_cast<uint64_t>(hmin2) << 32) | hmin;
            if constexpr (kWide)
                curH = stored0 ? SelectSurvivors(ArraySource{lo}, K0, keys0, beam, lt, surv)
                               : SelectSurvivors(Layer0Source{Gdiag, xc, nx2}, K0, keys0, beam, lt, surv);
            else
                curH = SelectSurvivors(ArraySource{lo}, K0, keys0, beam, lt, surv);
            if (curH >= 0) {
                for (int p = tid; p < curH; p += kThreads)
                    ex[p] = stored0 ? lo[surv[p]] : Layer0Error(Gdiag, xc, nx2, surv[p]);
                __syncthreads();
                curH = RankSurvivors(ex, surv, curH, beam, lt, keys);
            }
        }
        const SlotView<MAXM> s0 = SlotView<MAXM>::At(smem, beam);
        if (curH > 0 && tid < curH)
            InitSlot0<MAXM>(s0, tid, lt.cand[tid], dims.ldg, Gdiag,
                            kStrict ? gex[lt.candp[tid]] : __ldg(xc + lt.cand[tid]), nx2);
        if (curH == 0) {
            DeadSlot0<MAXM>(dims, s0);
            curH = 1;
        }
        __syncthreads();
        int ci = 0;
        for (int L = 1; L < m && curH > 0; ++L) {
            curH = FastLayer<MAXM, kWide, kStrict>(dims, L, SlotView<MAXM>::At(smem + ci * sv, beam),
                                                   SlotView<MAXM>::At(smem + (ci ^ 1) * sv, beam), curH, Grow, Gdiag,
                                                   xc, beam, lo, lt, surv, ex, keys, keep, check, err_flag, ctx,
                                                   gex);
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
            StoreCode(Bout, vec * m + tid, cur.rowh(0)[tid] / dims.ldg - dims.off[tid], dims.wide);
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

// STRICT mode's shared arrays: the staged vector (strict_d floats, 0 when not STRICT) and, in the
// fast kernel, the survivors' exact xC entries; with alignment slack.
size_t StrictBytes(int strict_d, bool fast) {
    return strict_d > 0 ? 16 + sizeof(float) * (Align4(strict_d) + (fast ? kSurvCap : 0)) : 0;
}

template <int MAXM>
size_t FastSmemBytes(int beam, int maxK, int strict_d = 0) {
    size_t b = (2 * SlotView<MAXM>::Bytes(beam) + 15) & ~size_t(15);
    b = (b + sizeof(LayerTable) + 15) & ~size_t(15);
    return b + sizeof(uint64_t) * kSurvCap + sizeof(float) * beam * maxK + (sizeof(float) + sizeof(uint16_t)) * kSurvCap +
           sizeof(float) * kKeep * KeepStride<MAXM>() + 16 + StrictBytes(strict_d, true);
}

// With the pre-scan: errors (lower bounds first) and upper bounds; without: errors only.
template <int MAXM>
size_t ReplaySmemBytes(int beam, int maxK, bool prescan, int strict_d = 0) {
    size_t b = (2 * SlotView<MAXM>::Bytes(beam) + 15) & ~size_t(15);
    b = (b + sizeof(LayerTable) + 15) & ~size_t(15);
    return b + (prescan ? 2 : 1) * sizeof(float) * ReplayCandFloats(beam, maxK) + 16 + StrictBytes(strict_d, false);
}

// The largest dynamic shared memory a block of the current device may opt into.
size_t MaxBlockSmem() {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return 0;
    return static_cast<size_t>(v);
}

// The replay runs its pre-scan whenever the upper bounds fit beside the errors.
template <int MAXM>
bool ReplayPrescan(int beam, int maxK, int strict_d = 0) {
    return ReplaySmemBytes<MAXM>(beam, maxK, true, strict_d) <= MaxBlockSmem();
}

// Sets the kernel's shared-memory size, finds how many CTAs fit on an SM, then asks for the
// smallest shared-memory carve-out that still holds them: the rest of the SM's unified 256 KB
// stays L1 cache for the gathers of Gram-matrix entries.  Grid: one CTA per resident slot.
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
    int dev = 0, sm_smem = 0, reserved = 0;
    if (per_sm > 0 && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) == cudaSuccess && sm_smem > 0) {
        const int64_t need = static_cast<int64_t>(per_sm) * (static_cast<int64_t>(smem) + reserved);
        const int pct = static_cast<int>(std::min<int64_t>(100, (100 * need + sm_smem - 1) / sm_smem));
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, pct);
        if (e != cudaSuccess) return e;
        int check = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&check, kernel, kThreads, smem);
        if (e != cudaSuccess) return e;
        if (check < per_sm) {  // the hint cost occupancy: keep the maximum carve-out
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     static_cast<int>(cudaSharedmemCarveoutMaxShared));
            if (e != cudaSuccess) return e;
        }
    }
    *grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(n, static_cast<int64_t>(num_sms) * std::max(per_sm, 1))));
    return cudaSuccess;
}

// strict_d: STRICT mode (ea.X non-null): the vector dimension, for the staged vector.
template <int MAXM, bool kWide, bool kStrict>
cudaError_t LaunchBeamT(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2, const float* xC,
                        int64_t n, int beam, void* Bout, int* redo, int check, unsigned int* err_flag,
                        unsigned long long* stats, int num_sms, cudaStream_t stream, const ExactDotArgs& ea) {
    const int sd = kStrict ? dims.d : 0;
    int grid = 0;
    const size_t fsm = FastSmemBytes<MAXM>(beam, dims.maxKs, sd);
    cudaError_t e = Prepare(BeamFastKernel<MAXM, kWide, kStrict>, fsm, num_sms, n, &grid);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(redo, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
    BeamFastKernel<MAXM, kWide, kStrict><<<grid, kThreads, fsm, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout,
                                                                          redo + 1, redo, check, err_flag, stats, ea);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const bool prescan = ReplayPrescan<MAXM>(beam, dims.maxKs, sd);
    const size_t rsm = ReplaySmemBytes<MAXM>(beam, dims.maxKs, prescan, sd);
    e = Prepare(BeamReplayKernel<MAXM, kWide, kStrict>, rsm, num_sms, n, &grid);
    if (e != cudaSuccess) return e;
    BeamReplayKernel<MAXM, kWide, kStrict><<<grid, kThreads, rsm, stream>>>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout,
                                                                            redo + 1, redo, prescan, ea, err_flag);
    return cudaGetLastError();
}

template <int MAXM, bool kWide>
cudaError_t PrepareT(const Dims& dims, int beam) {
    // The sizes a launch asks for.
    const size_t fsm = FastSmemBytes<MAXM>(beam, dims.maxKs);
    const bool prescan = ReplayPrescan<MAXM>(beam, dims.maxKs);
    const size_t rsm = ReplaySmemBytes<MAXM>(beam, dims.maxKs, prescan);
    cudaError_t e = cudaFuncSetAttribute(BeamFastKernel<MAXM, kWide, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(fsm));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(BeamReplayKernel<MAXM, kWide, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(rsm));
}

}  // namespace

size_t BeamFastSmemBytes(const Dims& dims, int beam, bool strict) {
    const int sd = strict ? dims.d : 0;
    return dims.m <= 8 ? FastSmemBytes<8>(beam, dims.maxKs, sd) : FastSmemBytes<16>(beam, dims.maxKs, sd);
}

// The kWide kernels: a codebook of layers 1..m-1 above kMaxK codewords (chunked cheap passes) or
// layer-0 errors that do not fit the beam x maxKs candidate array (recomputed from xC).
bool BigCodebooks(const Dims& dims, int beam) {
    return dims.maxKs > kMaxK || dims.h_vec[0] > beam * dims.maxKs;
}

cudaError_t PrepareBeamKernels(const Dims& dims, int beam) {
    const bool wide = BigCodebooks(dims, beam);
    if (dims.m <= 8) return wide ? PrepareT<8, true>(dims, beam) : PrepareT<8, false>(dims, beam);
    return wide ? PrepareT<16, true>(dims, beam) : PrepareT<16, false>(dims, beam);
}

// Querying a kernel's attributes makes the runtime load it (under lazy module loading too), so
// no later launch of any beam kernel variant does that first-use work.
cudaError_t LoadAllBeamKernels() {
    cudaFuncAttributes a{};
    const void* kernels[] = {reinterpret_cast<const void*>(BeamFastKernel<8, false, false>),
                             reinterpret_cast<const void*>(BeamFastKernel<8, true, false>),
                             reinterpret_cast<const void*>(BeamFastKernel<16, false, false>),
                             reinterpret_cast<const void*>(BeamFastKernel<16, true, false>),
                             reinterpret_cast<const void*>(BeamReplayKernel<8, false, false>),
                             reinterpret_cast<const void*>(BeamReplayKernel<8, true, false>),
                             reinterpret_cast<const void*>(BeamReplayKernel<16, false, false>),
                             reinterpret_cast<const void*>(BeamReplayKernel<16, true, false>)};
    for (const void* k : kernels) {
        const cudaError_t e = cudaFuncGetAttributes(&a, k);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// redo: n + 1 ints of scratch (a count, then vector ids handed from the fast to the replay kernel).
// ea (may be null): STRICT mode's exact-entry inputs; with ea->X non-null the kStrict kernels run.
cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, void* Bout, int* redo, int check,
                             unsigned int* err_flag, int num_sms, cudaStream_t stream, const ExactDotArgs* ea) {
    if (n <= 0) return cudaSuccess;
    // The encoder's flag word is followed by four 64-bit counters (BeamStats).
    unsigned long long* stats = err_flag ? reinterpret_cast<unsigned long long*>(err_flag + 4) : nullptr;
    const bool wide = BigCodebooks(dims, beam);  // separate kernels: the common sizes keep the simple paths
    const bool strict = ea && ea->X;
    const ExactDotArgs none{};
    const ExactDotArgs& a = strict ? *ea : none;
#define STLQ_B200_LAUNCH(MM, WW, SS) \
    LaunchBeamT<MM, WW, SS>(dims, Grow, Gdiag, xnorm2, xC, n, beam, Bout, redo, check, err_flag, stats, num_sms, stream, a)
    if (strict) {
        if (dims.m <= 8) return wide ? STLQ_B200_LAUNCH(8, true, true) : STLQ_B200_LAUNCH(8, false, true);
        return wide ? STLQ_B200_LAUNCH(16, true, true) : STLQ_B200_LAUNCH(16, false, true);
    }
    if (dims.m <= 8) return wide ? STLQ_B200_LAUNCH(8, true, false) : STLQ_B200_LAUNCH(8, false, false);
    return wide ? STLQ_B200_LAUNCH(16, true, false) : STLQ_B200_LAUNCH(16, false, false);
#undef STLQ_B200_LAUNCH
}

}  // namespace stlq_b200
