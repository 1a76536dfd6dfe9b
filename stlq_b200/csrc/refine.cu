// Least squares, cost, MSE and ICM/ILS refinement for sm_100a, fused per vector.
//
// Reference semantics:
//   SolveLeastSquaresAll / SolveLeastSquaresSample   src/quantizer/least_squares.cpp:86-129, 252-318, 406-560
//   SampleCost / ComputeCosts                         src/quantizer/cost_utils.cpp:112-158
//   MeanMseFromPrecomp (per-vector term, double)      src/linkage/linkage_tools.cpp:170-219
//   RunIcm<UseAbs>, DynamicIcmWithIlsImpl             src/quantizer/icm.cpp:89-344, 872-1003
//
// Every step of ICM and ILS is independent across vectors once the layer orders are known (the
// reference draws them on the host from one std::mt19937 and the same orders apply to every
// vector), so one warp carries its vectors through LS, cost, all ICM sweeps and all ILS rounds
// without returning to the host: the reference launches one kernel per layer per sweep and
// copies state through the host between them (icm_cuda_kernels.inc:2183-2261).
//
// Layout: 4 warps per CTA; a warp refines its vectors 32 at a time, lane i holding the codes,
// coefficients and cost of the i-th.  The ICM scores of a layer are computed by the whole warp
// for one vector at a time (coalesced reads of G's column segment, argmax by shuffles); the
// serial parts (LS solves, costs, trial changes, ILS perturbations, MSE terms) then run on every
// lane at once, each for its own vector, reading Gram entries from the global matrix.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kWarps = 4;
constexpr int kScoreT = 8;  // ICM codewords per lane held in registers (a chunk of 256 per warp)
constexpr int kRefineThreads = 32 * kWarps;
// Resident CTAs per SM the kernel is compiled for (64 registers a thread): the scoring's Gram
// gathers are latency-bound, and 32 warps per SM hide twice what 16 do, which outweighs the
// spills of the serial routines.
constexpr int kRefineBlocksPerSm = 8;

__device__ __forceinline__ float PosInfF() { return __int_as_float(0x7f800000); }

// The codes and coefficients of the vector the warp is scoring, staged by the lane that holds it.
struct WarpStage {
    int code[kMaxM];
    float a[kMaxM];
};

// One lane's scratch for an LS solve (local memory: the lanes' copies interleave, so a warp's
// accesses to one element coalesce).
struct LaneScratch {
    float A[kMaxM * kMaxM];
    float b[kMaxM];
    float x[kMaxM];
    float y[kMaxM];
};

// G(row, col) of two flat indices from the refinement's Gram array: G(r, c), r >= c0, at
// g[c * ldg + (r - c0)] (the layout is described with Dims).  Regular encoders have c0 = 0; in a
// large-root encoder a root row is read through symmetry, and two root codewords are only ever
// the root's own diagonal.
struct GramRef {
    const float* g;
    const float* diag;
    int ldg, c0;
    __device__ float operator()(int row, int col) const {
        if (row >= c0) return g[static_cast<size_t>(col) * ldg + (row - c0)];
        if (col >= c0) return g[static_cast<size_t>(row) * ldg + (col - c0)];
        return diag[row];
    }
};

__device__ __forceinline__ GramRef MakeGram(const Dims& dims, const float* g, const float* diag) {
    return GramRef{g, diag, dims.ldg, dims.c0};
}

// Gram entry G(flat_r, flat_c) of layers r and c for the codes `code`.
struct GramGlobal {
    GramRef g;
    const int* off;
    const int* code;
    __device__ float operator()(int r, int c) const { return g(off[r] + code[r], off[c] + code[c]); }
};
// Fixed-size Cholesky for m in {5, 10} (CholeskyUpperFixed, least_squares.cpp:44-66), row-major.
__device__ __noinline__ bool CholFixed(float* A, int m) {
    for (int k = 0; k < m; ++k) {
        float sum = A[k * m + k];
        for (int j = 0; j < k; ++j) {
            const float v = A[j * m + k];
            sum = sub_rn(sum, mul_rn(v, v));
        }
        if (sum <= kIcmEps) return false;
        const float diag = __fsqrt_rn(sum);
        A[k * m + k] = diag;
        for (int i = k + 1; i < m; ++i) {
            float s = A[k * m + i];
            for (int j = 0; j < k; ++j) s = sub_rn(s, mul_rn(A[j * m + k], A[j * m + i]));
            A[k * m + i] = div_rn(s, diag);
        }
    }
    return true;
}

// LAPACK spotrf('U') / spotrs for the other m (least_squares.cpp:278-316), in the arithmetic of
// the BLAS/LAPACK build the reference links (OpenBLAS 0.3.15 SkylakeX kernels, pinned element
// by element against that library):
//  * pivot: a_jj - sum of float products accumulated in double; sqrt; fails when <= 0;
//  * row update through SGEMV-T: rows in blocks of 4 reduced per 4-column group on 4 (+8) FMA
//    lanes as (l0+l1)+(l2+l3), leftover columns on 4 mul/add lanes, the last j%4 rows by
//    contracted FMAs; the row is then scaled by the float reciprocal of the pivot;
//  * spotrs: triangular blocks of 16/8/4/2/1 rows solved with the reciprocal diagonal and FMA
//    updates, blocks joined by FMA-chain updates.
__device__ float PotfBlockAvx(const float* a, const float* x, int nb) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int r = 0;
    if (nb & 4) {
        for (int l = 0; l < 4; ++l) lane[l] = __fmaf_rn(a[l], x[l], lane[l]);
        r = 4;
    }
    for (; r < nb; r += 8)
        for (int l = 0; l < 8; ++l) lane[l] = __fmaf_rn(a[r + l], x[r + l], lane[l]);
    float q[4];
    for (int l = 0; l < 4; ++l) q[l] = add_rn(lane[l], lane[l + 4]);
    return add_rn(add_rn(q[0], q[1]), add_rn(q[2], q[3]));
}

__device__ float PotfBlockSse(const float* a, const float* x, int nb) {
    float lane[4] = {0, 0, 0, 0};
    for (int r = 0; r < nb; r += 4)
        for (int l = 0; l < 4; ++l) lane[l] = add_rn(lane[l], mul_rn(a[r + l], x[r + l]));
    return add_rn(add_rn(lane[0], lane[1]), add_rn(lane[2], lane[3]));
}

__device__ float PotfLeftover(float y, const float* a, const float* x, int m1, int m3) {
    if (m3 == 0) return y;
    const float xt0 = -x[m1];
    if (m3 == 1) return __fmaf_rn(a[m1], xt0, y);
    const float p1 = mul_rn(a[m1 + 1], -x[m1 + 1]);
    float e = __fmaf_rn(a[m1], xt0, p1);
    if (m3 == 3) e = __fmaf_rn(a[m1 + 2], -x[m1 + 2], e);
    return add_rn(y, e);
}

// The LAPACK path keeps only the upper triangle, packed by columns: element (r, c), r <= c, at
// c (c + 1) / 2 + r (column c's first c + 1 rows contiguous).  Fewer words per lane than a full
// m x m column-major array, so the lanes' scratch stays in L1; the arithmetic is unchanged.
__device__ __forceinline__ int Pk(int r, int c) { return c * (c + 1) / 2 + r; }

__device__ __noinline__ bool CholLapack(float* A, int m) {  // packed upper triangle (Pk)
    for (int j = 0; j < m; ++j) {
        const float* xj = A + Pk(0, j);
        double acc = 0.0;
        for (int k = 0; k < j; ++k) acc = __dadd_rn(acc, static_cast<double>(mul_rn(xj[k], xj[k])));
        float ajj = sub_rn(A[Pk(j, j)], static_cast<float>(acc));
        if (ajj <= 0.0f) return false;
        ajj = __fsqrt_rn(ajj);
        A[Pk(j, j)] = ajj;
        const float r = div_rn(1.0f, ajj);
        const int ncol = m - j - 1, m3 = j & 3, m1 = j - m3, n1 = (ncol >> 2) * 4;
        for (int ci = 0; ci < ncol; ++ci) {
            const int c = j + 1 + ci;
            const float* ac = A + Pk(0, c);
            float y = A[Pk(j, c)];
            if (m1 > 0) {
                const float K = ci < n1 ? PotfBlockAvx(ac, xj, m1) : PotfBlockSse(ac, xj, m1);
                y = __fmaf_rn(K, -1.0f, y);
            }
            y = PotfLeftover(y, ac, xj, m1, m3);
            A[Pk(j, c)] = mul_rn(y, r);
        }
    }
    return true;
}

// c[r] -= sum_t U(t,r) c[t] (forward) or U(r,t) c[t] (backward) over t in [t0, t1), as one FMA
// chain from zero subtracted once (the GEMM update between STRSM blocks).
__device__ void TrsmUpdate(const float* A, int m, float* c, int r0, int nr, int t0, int t1, bool fwd) {
    for (int r = r0; r < r0 + nr; ++r) {
        float acc = 0.0f;
        for (int t = t0; t < t1; ++t) acc = __fmaf_rn(fwd ? A[Pk(t, r)] : A[Pk(r, t)], c[t], acc);
        c[r] = __fmaf_rn(acc, -1.0f, c[r]);
    }
}

__device__ void TrsmFwdBlock(const float* A, int m, float* c, int r0, int bs) {
    for (int i = r0; i < r0 + bs; ++i) {
        const float bb = mul_rn(c[i], div_rn(1.0f, A[Pk(i, i)]));
        c[i] = bb;
        for (int k = i + 1; k < r0 + bs; ++k) c[k] = __fmaf_rn(-bb, A[Pk(i, k)], c[k]);
    }
}

__device__ void TrsmBwdBlock(const float* A, int m, float* c, int r0, int bs) {
    for (int i = r0 + bs - 1; i >= r0; --i) {
        const float bb = mul_rn(c[i], div_rn(1.0f, A[Pk(i, i)]));
        c[i] = bb;
        for (int k = r0; k < i; ++k) c[k] = __fmaf_rn(-bb, A[Pk(k, i)], c[k]);
    }
}

__device__ __noinline__ void SolveLapack(const float* A, int m, float* c) {  // U^T y = b, U x = y, in place
    constexpr int UM = 16;
    int kk = 0;
    for (int b = 0; b < m / UM; ++b) {
        if (kk > 0) TrsmUpdate(A, m, c, kk, UM, 0, kk, true);
        TrsmFwdBlock(A, m, c, kk, UM);
        kk += UM;
    }
    for (int i = UM / 2; i > 0; i >>= 1) {
        if (!(m & i)) continue;
        if (kk > 0) TrsmUpdate(A, m, c, kk, i, 0, kk, true);
        TrsmFwdBlock(A, m, c, kk, i);
        kk += i;
    }
    kk = m;
    for (int i = 1; i < UM; i *= 2) {
        if (!(m & i)) continue;
        const int st = (m & ~(i - 1)) - i;
        if (m - kk > 0) TrsmUpdate(A, m, c, st, i, kk, m, false);
        TrsmBwdBlock(A, m, c, st, i);
        kk -= i;
    }
    for (int b = m / UM - 1; b >= 0; --b) {
        const int st = b * UM;
        if (m - kk > 0) TrsmUpdate(A, m, c, st, UM, kk, m, false);
        TrsmBwdBlock(A, m, c, st, UM);
        kk -= UM;
    }
}

// One vector's LS solve with the reference's retry policy (3 diagonal bumps 1e-6 x10^i).
// Out of line, like the other per-vector serial routines of this file: inlined at every call site
// (initial solve, each ICM change, each ILS round) they made the kernel large enough for
// instruction fetch to be its main stall.
template <class Gram, class Scratch>
__device__ __noinline__ bool SolveLs(const Dims& dims, const Gram& G, const float* xc, const int* code, Scratch& ws,
                        float* a_out) {
    const int m = dims.m;
    const bool fixed = (m == 5 || m == 10);
    float lambda = 0.0f;
    for (int attempt = 0; attempt < 4; ++attempt) {
        // Only the upper triangle is written and read (both Cholesky variants and both solves
        // index k <= j), so the strict lower triangle is never set: one solve touches fewer
        // words of the lane's scratch.
        for (int j = 0; j < m; ++j) {
            const int fj = dims.off[j] + code[j];
            ws.b[j] = xc[fj];
            for (int k = 0; k <= j; ++k) {
                const float g = G(k, j);
                if (fixed) ws.A[k * m + j] = g;
                else ws.A[Pk(k, j)] = g;
            }
            if (fixed) ws.A[j * m + j] = add_rn(ws.A[j * m + j], lambda);
            else ws.A[Pk(j, j)] = add_rn(ws.A[Pk(j, j)], lambda);
        }
        const bool ok = fixed ? CholFixed(ws.A, m) : CholLapack(ws.A, m);
        if (ok) {
            if (fixed) {
                for (int i = 0; i < m; ++i) {
                    float s = ws.b[i];
                    for (int k = 0; k < i; ++k) s = sub_rn(s, mul_rn(ws.A[k * m + i], ws.y[k]));
                    ws.y[i] = div_rn(s, ws.A[i * m + i]);
                }
                for (int i = m - 1; i >= 0; --i) {
                    float s = ws.y[i];
                    for (int k = i + 1; k < m; ++k) s = sub_rn(s, mul_rn(ws.A[i * m + k], ws.x[k]));
                    ws.x[i] = div_rn(s, ws.A[i * m + i]);
                }
                for (int i = 0; i < m; ++i) a_out[i] = ws.x[i];
            } else {
                SolveLapack(ws.A, m, ws.b);
                for (int i = 0; i < m; ++i) a_out[i] = ws.b[i];
            }
            return true;
        }
        lambda = (attempt == 0) ? kIcmEps : mul_rn(lambda, 10.0f);
    }
    return false;
}

// SampleCost (cost_utils.cpp:112-137).
template <class Gram>
__device__ __noinline__ float SampleCost(const Dims& dims, const Gram& G, const float* xc, const int* code, const float* a,
                            float xn2) {
    const int m = dims.m;
    float term1 = 0.0f, term2 = 0.0f;
    for (int l = 0; l < m; ++l) {
        const int fl = dims.off[l] + code[l];
        term1 = add_rn(term1, mul_rn(a[l], xc[fl]));
        for (int k = 0; k < m; ++k) term2 = add_rn(term2, mul_rn(mul_rn(a[l], a[k]), G(l, k)));
    }
    return add_rn(sub_rn(xn2, mul_rn(2.0f, term1)), term2);
}

// SampleCostLargeRoot (cost_utils.cpp:160-209): the same quantity in the large-root encoder's
// order — root term first, then root-small cross terms 2 a_0 a_j G(0, j), then small-small terms.
// xc[flat_0] holds the reference's SIMD-order dot of the root codeword with x (LaunchRootDot) and
// G(0, 0) the root codeword's norm0.
template <class Gram>
__device__ __noinline__ float SampleCostLargeRoot(const Dims& dims, const Gram& G, const float* xc, const int* code,
                                     const float* a, float xn2) {
    const int m = dims.m;
    float term1 = mul_rn(a[0], xc[dims.off[0] + code[0]]);
    for (int l = 1; l < m; ++l) term1 = add_rn(term1, mul_rn(a[l], xc[dims.off[l] + code[l]]));
    float term2 = mul_rn(mul_rn(a[0], a[0]), G(0, 0));
    for (int j = 1; j < m; ++j) {
        term2 = add_rn(term2, mul_rn(mul_rn(mul_rn(2.0f, a[0]), a[j]), G(0, j)));
        for (int k = 1; k < m; ++k) term2 = add_rn(term2, mul_rn(mul_rn(a[j], a[k]), G(j, k)));
    }
    return add_rn(sub_rn(xn2, mul_rn(2.0f, term1)), term2);
}

template <class Gram>
__device__ __forceinline__ float Cost(const Dims& dims, const Gram& G, const float* xc, const int* code,
                                      const float* a, float xn2) {
    return dims.large_root ? SampleCostLargeRoot(dims, G, xc, code, a, xn2) : SampleCost(dims, G, xc, code, a, xn2);
}

// Per-vector term of MeanMseFromPrecomp in double, clamped at 0.
template <class Gram>
__device__ double VectorSse(const Dims& dims, const Gram& G, const float* xc, const int* code, const float* a,
                            double nx) {
    const int m = dims.m;
    double t1 = 0.0, t2 = 0.0;
    for (int j = 0; j < m; ++j)
        t1 = __dadd_rn(t1, __dmul_rn(static_cast<double>(a[j]), static_cast<double>(xc[dims.off[j] + code[j]])));
    for (int j = 0; j < m; ++j)
        for (int k = 0; k < m; ++k)
            t2 = __dadd_rn(t2, __dmul_rn(__dmul_rn(static_cast<double>(a[j]), static_cast<double>(a[k])),
                                         static_cast<double>(G(j, k))));
    const double e = __dadd_rn(__dsub_rn(nx, __dmul_rn(2.0, t1)), t2);
    return e < 0.0 ? 0.0 : e;
}

struct SplitMix64 {  // icm.cpp:55-65
    uint64_t state;
    __device__ uint64_t Next() {
        uint64_t z = (state += 0x9e3779b97f4a7c15ULL);
        z = (z ^ (z >> 30U)) * 0xbf58476d1ce4e5b9ULL;
        z = (z ^ (z >> 27U)) * 0x94d049bb133111ebULL;
        return z ^ (z >> 31U);
    }
};

__device__ __forceinline__ uint32_t UniformBelow(SplitMix64& r, uint32_t bound) {  // icm.cpp:76-87
    return static_cast<uint32_t>(__umul64hi(r.Next(), static_cast<uint64_t>(bound)));
}

// The ICM choice for layer j of the staged vector, by the whole warp (icm.cpp:272-300): the
// codeword t with the largest score (xC(t) - sum_{l != j} a_l G(t, flat_l)) * invnorm(t),
// absolute with use_abs, the first strict maximum in t order; code[j] when no score beats -inf.
// Each lane holds kScoreT codewords t = t0 + lane + 32 i; the layers l run outermost (the same
// per-t subtraction order), so a lane's kScoreT gathers of one Gram row are issued together.
__device__ __forceinline__ int ScoreLayer(const Dims& dims, const GramRef& Gr, const float* invnorm, const float* xc,
                                          int j, const int* code, const float* a, bool use_abs) {
    const int lane = threadIdx.x & 31;
    const int m = dims.m, hj = dims.h_vec[j], startf = dims.off[j];
    float best_s = __int_as_float(0xff800000);  // -inf
    int best_t = 0x7fffffff;
    for (int t0 = 0; t0 < hj; t0 += 32 * kScoreT) {
        float v[kScoreT];
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = t0 + lane + 32 * i;
            v[i] = t < hj ? __ldcs(xc + startf + t) : 0.0f;  // streamed once: evict first
        }
        for (int l = 0; l < m; ++l) {
            if (l == j) continue;
            const float al = a[l];
            // G(startf + t, flat_l): codebook j >= 1, so the row is always stored (>= c0).
            const float* grow =
                Gr.g + static_cast<size_t>(dims.off[l] + code[l]) * Gr.ldg + (startf - Gr.c0) + t0 + lane;
            float g[kScoreT];
#pragma unroll
            for (int i = 0; i < kScoreT; ++i) g[i] = t0 + lane + 32 * i < hj ? __ldg(grow + 32 * i) : 0.0f;
#pragma unroll
            for (int i = 0; i < kScoreT; ++i) v[i] = sub_rn(v[i], mul_rn(al, g[i]));
        }
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = t0 + lane + 32 * i;
            if (t >= hj) continue;
            const float val = mul_rn(v[i], __ldg(invnorm + startf + t));
            const float s = use_abs ? fabsf(val) : val;
            if (s > best_s) {  // first strict maximum in t order (t increases with i and t0)
                best_s = s;
                best_t = t;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float s2 = __shfl_xor_sync(0xffffffffu, best_s, o);
        const int t2 = __shfl_xor_sync(0xffffffffu, best_t, o);
        if (s2 > best_s || (s2 == best_s && t2 < best_t)) {
            best_s = s2;
            best_t = t2;
        }
    }
    return (best_s > __int_as_float(0xff800000)) ? best_t : code[j];
}

// ---------------------------------------------------------------------------------------------
// STRICT mode: xC holds tensor-core entries, within kx ||c_t|| of the exact ones (kx = kappa ||x||).
// A lane writes the exact entry of a codeword into its vector's xC row before an LS solve or a
// cost reads it (FixEntry), and an ICM choice is made from bounds on the scores, with exact
// scores only where the bounds cannot decide (ScoreLayerStrict).

// The exact xC entry of flat codeword `flat` for vector row `xrow` (the exact GEMM's order).
__device__ __noinline__ float LaneExact(const ExactDotArgs& ex, int d, const void* xrow, int flat) {
    const float* c = ex.C + static_cast<size_t>(flat) * d;
    return ex.x_dtype ? ExactDot(c, static_cast<const uint8_t*>(xrow), d) : ExactDot(c, static_cast<const float*>(xrow), d);
}

__device__ __forceinline__ void FixEntry(const ExactDotArgs& ex, int d, const void* xrow, float* xcw, int flat, float kx,
                                         unsigned int* err) {
    const float g = LaneExact(ex, d, xrow, flat);
    CheckTcBound(g, xcw[flat], kx * __ldg(ex.cn + flat), err);
    xcw[flat] = g;
}

// FixEntry for the codes of layers l0..m-1, four chains at a time.
__device__ __noinline__ void FixCodes(const ExactDotArgs& ex, const Dims& dims, const void* xrow, float* xcw,
                                      const int* code, int l0, float kx, unsigned int* err) {
    const int m = dims.m, d = dims.d;
    for (int l = l0; l < m; l += 4) {
        int f[4];
        const float* rows[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int lr = min(l + r, m - 1);  // past the last layer: a repeat, not written
            f[r] = dims.off[lr] + code[lr];
            rows[r] = ex.C + static_cast<size_t>(f[r]) * d;
        }
        float g[4];
        if (ex.x_dtype) ExactDotRows<4>(rows, static_cast<const uint8_t*>(xrow), d, g);
        else ExactDotRows<4>(rows, static_cast<const float*>(xrow), d, g);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (l + r >= m) break;
            CheckTcBound(g[r], xcw[f[r]], kx * __ldg(ex.cn + f[r]), err);
            xcw[f[r]] = g[r];
        }
    }
}

// The ICM choice for layer j of the staged vector, like ScoreLayer, from the tensor-core row xc of
// that vector.  Each score s_t = |val_t| (or val_t) with val_t = (xc_t - sum_l a_l G(t, flat_l)) *
// invnorm_t in the reference's order moves by at most
//   r_t = (dg_t + 2 m u (|xc_t| + dg_t + ||c_t|| A)) invnorm_t (1 + 1e-4) + 3 u |val_t|,
// dg_t = kx ||c_t||, A >= sum_l |a_l| ||c_{flat_l}||, when the exact xc_t replaces the tensor-core
// one (the first term is the input's own error, the second the roundings of both chains, the last
// the final product's).  With LB = max_t (s_t - r_t), every codeword with s_t + r_t < LB scores
// below the exact maximum, so only the others (the contenders) can be chosen: one contender is the
// choice; with several, their exact scores decide (first maximum in t order, as the reference).
// xrow: the staged vector's row of X, for the exact entries.
__device__ __noinline__ int ScoreLayerStrict(const Dims& dims, const GramRef& Gr, const float* invnorm, const float* xc,
                                             int j, const int* code, const float* a, bool use_abs,
                                             const ExactDotArgs& ex, const void* xrow, float kx) {
    const int lane = threadIdx.x & 31;
    const int m = dims.m, hj = dims.h_vec[j], startf = dims.off[j];
    constexpr float u = 5.9604645e-8f;  // 2^-24
    float A = 0.0f;
    for (int l = 0; l < m; ++l)
        if (l != j) A = fmaf(fabsf(a[l]), __ldg(ex.cn + dims.off[l] + code[l]), A);
    A *= 1.001f;
    const float cm = 2.0f * m * u;
    // Score and radius of this lane's kScoreT codewords of chunk t0.
    auto score = [&](int t0, float (&s)[kScoreT], float (&r)[kScoreT]) {
        float v[kScoreT];
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = t0 + lane + 32 * i;
            v[i] = t < hj ? __ldcs(xc + startf + t) : 0.0f;
        }
        float xa[kScoreT];
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) xa[i] = fabsf(v[i]);
        for (int l = 0; l < m; ++l) {
            if (l == j) continue;
            const float al = a[l];
            const float* grow =
                Gr.g + static_cast<size_t>(dims.off[l] + code[l]) * Gr.ldg + (startf - Gr.c0) + t0 + lane;
            float g[kScoreT];
#pragma unroll
            for (int i = 0; i < kScoreT; ++i) g[i] = t0 + lane + 32 * i < hj ? __ldg(grow + 32 * i) : 0.0f;
#pragma unroll
            for (int i = 0; i < kScoreT; ++i) v[i] = sub_rn(v[i], mul_rn(al, g[i]));
        }
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = t0 + lane + 32 * i;
            if (t >= hj) {
                s[i] = -PosInfF();
                r[i] = 0.0f;
                continue;
            }
            const float inv = __ldg(invnorm + startf + t), cnt = __ldg(ex.cn + startf + t);
            const float val = mul_rn(v[i], inv);
            const float dg = kx * cnt;
            s[i] = use_abs ? fabsf(val) : val;
            r[i] = (dg + cm * (xa[i] + dg + cnt * A)) * inv * 1.0001f + 3.0f * u * fabsf(val);
        }
    };
    // The exact score of codeword t (its exact entry, then the same sequence as ScoreLayer).
    auto exact = [&](int t) {
        float v = LaneExact(ex, dims.d, xrow, startf + t);
        for (int l = 0; l < m; ++l) {
            if (l == j) continue;
            v = sub_rn(v, mul_rn(a[l], __ldg(Gr.g + static_cast<size_t>(dims.off[l] + code[l]) * Gr.ldg +
                                             (startf - Gr.c0) + t)));
        }
        const float val = mul_rn(v, __ldg(invnorm + startf + t));
        return use_abs ? fabsf(val) : val;
    };
    const int nchunk = (hj + 32 * kScoreT - 1) / (32 * kScoreT);
    float s[kScoreT], r[kScoreT];
    // LB over every chunk (the last chunk's scores stay in registers).
    float lb = -PosInfF();
    for (int c = 0; c < nchunk; ++c) {
        score(c * 32 * kScoreT, s, r);
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) lb = fmaxf(lb, s[i] - r[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lb = fmaxf(lb, __shfl_xor_sync(0xffffffffu, lb, o));
    // Contenders: t < hj with !(s + r < LB).  Count them and find the first.
    int count = 0, first = 0x7fffffff;
    for (int c = nchunk - 1; c >= 0; --c) {
        if (c != nchunk - 1) score(c * 32 * kScoreT, s, r);
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = c * 32 * kScoreT + lane + 32 * i;
            const bool cont = t < hj && !(s[i] + r[i] < lb);
            const unsigned bal = __ballot_sync(0xffffffffu, cont);
            count += __popc(bal);
            if (bal) first = min(first, c * 32 * kScoreT + (__ffs(bal) - 1) + 32 * i);
        }
    }
    if (count == 1 && lb > -PosInfF()) return first;
    // Exact scores of the contenders; first strict maximum in t order.
    float best_s = -PosInfF();
    int best_t = 0x7fffffff;
    for (int c = 0; c < nchunk; ++c) {
        score(c * 32 * kScoreT, s, r);
#pragma unroll
        for (int i = 0; i < kScoreT; ++i) {
            const int t = c * 32 * kScoreT + lane + 32 * i;
            if (t < hj && !(s[i] + r[i] < lb)) {
                const float se = exact(t);
                if (se > best_s) {
                    best_s = se;
                    best_t = t;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float s2 = __shfl_xor_sync(0xffffffffu, best_s, o);
        const int t2 = __shfl_xor_sync(0xffffffffu, best_t, o);
        if (s2 > best_s || (s2 == best_s && t2 < best_t)) {
            best_s = s2;
            best_t = t2;
        }
    }
    return (best_s > -PosInfF()) ? best_t : code[j];
}

// One lane's trial change of layer j to `best` for its own vector (icm.cpp:300-340): LS for the
// new codes and their cost; the change is kept only if the cost drops by more than kIcmEps,
// otherwise code and a are restored.  Returns whether it was kept.  STRICT (ex.X non-null): the
// new codeword's exact xC entry is written into the row first.
template <bool kStrict>
__device__ __noinline__ bool TryChange(const Dims& dims, const GramRef& Gr, const float* xc, float xn2, int j, int best,
                                       int* code, float* a, float* cost, LaneScratch& sc, const ExactDotArgs& ex,
                                       const void* xrow, float kx, unsigned int* err) {
    const int m = dims.m;
    const int old_code = code[j];
    if constexpr (kStrict) FixEntry(ex, dims.d, xrow, const_cast<float*>(xc), dims.off[j] + best, kx, err);
    float backup[kMaxM];
    for (int l = 0; l < m; ++l) backup[l] = a[l];
    code[j] = best;
    const GramGlobal G{Gr, dims.off, code};
    bool keep = SolveLs(dims, G, xc, code, sc, a);
    if (keep) {
        const float nc = Cost(dims, G, xc, code, a, xn2);
        keep = add_rn(nc, kIcmEps) < *cost;
        if (keep) *cost = nc;
    }
    if (!keep) {
        code[j] = old_code;
        for (int l = 0; l < m; ++l) a[l] = backup[l];
    }
    return keep;
}

template <typename T>
__device__ __forceinline__ const T* ShflPtr(const T* ptr, int src) {
    return reinterpret_cast<const T*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(ptr), src));
}

// RunIcm's sweeps (icm.cpp:116-344) for the vectors of a warp's group after its first step: lane
// i < ng holds the i-th vector's codes, coefficients and cost (in/out) and its xC row.  For each
// layer of the order, the warp scores the active vectors one at a time from the codes their lanes
// stage in `st`; then every lane tries its own vector's change at once.  A vector stops after a
// sweep without a kept change, as RunIcm does.
// kStrict: xc is the lane's tensor-core row (exact at its codes), xrow its vector's row of X and
// kx its bound factor (see ScoreLayerStrict, FixEntry).
template <bool kStrict>
__device__ __noinline__ void RunIcmGroup(const Dims& dims, const GramRef& Gr, const float* invnorm, const float* xc,
                                         float xn2, int ng, int icm_iters, const int* orders, bool use_abs,
                                         int* code, float* a, float* cost, WarpStage& st, LaneScratch& sc,
                                         const ExactDotArgs& ex, const void* xrow, float kx, unsigned int* err) {
    const int lane = threadIdx.x & 31;
    const int m = dims.m;
    bool active = lane < ng;
    for (int it = 0; it < icm_iters; ++it) {
        if (!__any_sync(0xffffffffu, active)) break;
        bool changed = false;
        for (int oi = 0; oi < m; ++oi) {
            const int j = orders[it * m + oi];
            if (j == 0 || dims.h_vec[j] <= 1) continue;
            int mine = 0;
            for (unsigned act = __ballot_sync(0xffffffffu, active); act; act &= act - 1) {
                const int gi = __ffs(act) - 1;
                __syncwarp();
                if (lane == gi)
                    for (int l = 0; l < m; ++l) {
                        st.code[l] = code[l];
                        st.a[l] = a[l];
                    }
                const float* xg = ShflPtr(xc, gi);
                __syncwarp();
                int best;
                if constexpr (kStrict)
                    best = ScoreLayerStrict(dims, Gr, invnorm, xg, j, st.code, st.a, use_abs, ex, ShflPtr(xrow, gi),
                                            __shfl_sync(0xffffffffu, kx, gi));
                else
                    best = ScoreLayer(dims, Gr, invnorm, xg, j, st.code, st.a, use_abs);
                if (lane == gi) mine = best;
            }
            if (active && mine != code[j])
                changed |= TryChange<kStrict>(dims, Gr, xc, xn2, j, mine, code, a, cost, sc, ex, xrow, kx, err);
        }
        active = active && changed;
    }
}

}  // namespace

// kStrict: STRICT mode (p.ex.X non-null, mode 1): the lane's xC row holds tensor-core entries and
// is made exact at every codeword an LS solve or a cost reads (FixEntry); ICM choices come from
// ScoreLayerStrict.  The codes, coefficients and costs equal the exact mode's.
template <bool kStrict>
__global__ void __launch_bounds__(kRefineThreads, kRefineBlocksPerSm) RefineKernel(RefineArgs p) {
    __shared__ WarpStage stage[kWarps];
    __shared__ double sse_w[kWarps][2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Dims& dims = p.dims;
    const int m = dims.m;
    const GramRef Gr = MakeGram(dims, p.Gcol, p.Gdiag);
    double sse_beam = 0.0, sse_final = 0.0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    // The warp's vectors are blockIdx.x * kWarps + warp + i * stride, taken 32 at a time (lane i
    // holds the i-th of a group), the order in which one vector at a time would take them.
    for (int64_t g0 = static_cast<int64_t>(blockIdx.x) * kWarps + warp; g0 < p.n; g0 += 32 * stride) {
        const int ng = static_cast<int>(min(int64_t{32}, (p.n - g0 + stride - 1) / stride));
        const bool own = lane < ng;
        const int64_t vec = own ? g0 + lane * stride : 0;
        const float* xc = p.xC + vec * dims.H;
        int code[kMaxM];
        float a[kMaxM];
        LaneScratch sc;
        float cost = 0.0f, xn2 = 0.0f;
        double tb = 0.0, tf = 0.0;
        const void* xrow = nullptr;  // STRICT: this lane's vector (row of X) and its bound factor
        float kx = 0.0f;
        if (own) {
            // RunIcm's first step (icm.cpp:109-114), or with mode 0 the whole LS stage.
            for (int l = 0; l < m; ++l) code[l] = LoadCode(p.B, vec * m + l, dims.wide);
            if constexpr (kStrict) {
                // The beam codes' exact entries (a large-root encoder's root entry is already the
                // reference's own dot product, written by LaunchRootDot).
                xrow = static_cast<const char*>(p.ex.X) + vec * dims.d * (p.ex.x_dtype ? 1 : 4);
                kx = StrictKx(p.ex.kappa, p.xnorm2[vec]);
                FixCodes(p.ex, dims, xrow, const_cast<float*>(xc), code, dims.large_root ? 1 : 0, kx, p.err_flag);
            }
            const GramGlobal G{Gr, dims.off, code};
            if (!SolveLs(dims, G, xc, code, sc, a))
                for (int l = 0; l < m; ++l) a[l] = 0.0f;
            if (p.mode == 0) {
                for (int l = 0; l < m; ++l) p.a[vec * m + l] = a[l];
            } else {
                xn2 = p.xnorm2[vec];
                cost = Cost(dims, G, xc, code, a, xn2);
                // Beam-stage error: MeanMseFromPrecomp's term, or for a large-root encoder the float
                // cost itself (the large pipeline averages ComputeCostsLargeRoot,
                // encode_base_streaming.cpp:301-311).
                if (p.partials)
                    tb = dims.large_root ? static_cast<double>(cost)
                                         : VectorSse(dims, G, xc, code, a, p.xnorm2_d[vec]);
            }
        }
        if (p.mode == 0) continue;
        WarpStage& st = stage[warp];
        if (p.icm_iters > 0)
            RunIcmGroup<kStrict>(dims, Gr, p.invnorm, xc, xn2, ng, p.icm_iters, p.orders, p.use_abs, code, a, &cost,
                                 st, sc, p.ex, xrow, kx, p.err_flag);
        const int ksel = min(p.perturb_k, m);
        for (int outer = 0; outer < p.n_ils; ++outer) {
            int cand[kMaxM];
            float acand[kMaxM];
            float ccost = 0.0f;
            if (own) {
                for (int l = 0; l < m; ++l) cand[l] = code[l];
                const uint64_t ig = p.sample_id_offset + static_cast<uint64_t>(vec);  // icm.cpp:953-972
                SplitMix64 r{static_cast<uint64_t>(p.seed) ^
                             (static_cast<uint64_t>(outer + 1) * 0x9e3779b97f4a7c15ULL) ^
                             ((ig + 1) * 0xbf58476d1ce4e5b9ULL)};
                for (int s = 0; s < ksel; ++s) {
                    const int layer = 1 + static_cast<int>(UniformBelow(r, static_cast<uint32_t>(m - 1)));
                    const int h = dims.h_vec[layer];
                    if (h <= 1) continue;
                    const int old_code = cand[layer];
                    const int raw = static_cast<int>(UniformBelow(r, static_cast<uint32_t>(h - 1)));
                    cand[layer] = raw >= old_code ? raw + 1 : raw;
                }
                if constexpr (kStrict)
                    for (int l = 1; l < m; ++l)
                        if (cand[l] != code[l])
                            FixEntry(p.ex, dims.d, xrow, const_cast<float*>(xc), dims.off[l] + cand[l], kx, p.err_flag);
                const GramGlobal G{Gr, dims.off, cand};
                if (!SolveLs(dims, G, xc, cand, sc, acand))
                    for (int l = 0; l < m; ++l) acand[l] = 0.0f;
                ccost = Cost(dims, G, xc, cand, acand, xn2);
            }
            if (p.icm_iters > 0)
                RunIcmGroup<kStrict>(dims, Gr, p.invnorm, xc, xn2, ng, p.icm_iters,
                                     p.orders + static_cast<size_t>(outer + 1) * p.icm_iters * m, p.use_abs, cand,
                                     acand, &ccost, st, sc, p.ex, xrow, kx, p.err_flag);
            if (own && add_rn(ccost, kIcmEps) < cost) {  // icm.cpp:979-990
                for (int l = 0; l < m; ++l) {
                    code[l] = cand[l];
                    a[l] = acand[l];
                }
                cost = ccost;
            }
        }
        if (own) {
            if (p.partials)
                tf = dims.large_root ? static_cast<double>(cost)
                                     : VectorSse(dims, GramGlobal{Gr, dims.off, code}, xc, code, a, p.xnorm2_d[vec]);
            for (int l = 0; l < m; ++l) {
                StoreCode(p.B, vec * m + l, code[l], dims.wide);
                if (p.a) p.a[vec * m + l] = a[l];
            }
            if (p.cost) p.cost[vec] = cost;
        }
        if (p.partials)  // added in the warp's vector order
            for (int gi = 0; gi < ng; ++gi) {
                const double b = __shfl_sync(0xffffffffu, tb, gi), f = __shfl_sync(0xffffffffu, tf, gi);
                if (lane == 0) {
                    sse_beam += b;
                    sse_final += f;
                }
            }
    }
    if (p.partials) {
        if (lane == 0) {
            sse_w[warp][0] = sse_beam;
            sse_w[warp][1] = sse_final;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double s0 = 0.0, s1 = 0.0;
            for (int w = 0; w < kWarps; ++w) {
                s0 += sse_w[w][0];
                s1 += sse_w[w][1];
            }
            p.partials[2 * blockIdx.x] = s0;
            p.partials[2 * blockIdx.x + 1] = s1;
        }
    }
}

// xC[vec][root] = Dot(C[root], x) in the reference's SIMD order: 4 lanes over the first 4*(d/4)
// elements (lane = index mod 4), the tail into lane 0, lanes summed in order; each product rounded,
// then added (no contraction).  4 threads per vector.
template <typename T>
__global__ void RootDotKernel(Dims dims, const float* __restrict__ C, const T* __restrict__ X,
                              const void* __restrict__ B, int64_t n, float* __restrict__ xC) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t vec = t >> 2;
    const int l = static_cast<int>(t & 3);
    const bool ok = vec < n;
    const int d = dims.d;
    int root = 0;
    float s = 0.0f;
    if (ok) {
        root = LoadCode(B, vec * dims.m, dims.wide);
        const float* c = C + static_cast<size_t>(root) * d;
        const T* x = X + vec * d;
        const int body = (d / 4) * 4;
        for (int k = l; k < body; k += 4) s = __fadd_rn(s, __fmul_rn(c[k], static_cast<float>(x[k])));
        if (l == 0)
            for (int k = body; k < d; ++k) s = __fadd_rn(s, __fmul_rn(c[k], static_cast<float>(x[k])));
    }
    const int base = (threadIdx.x & 31) & ~3;
    const float s1 = __shfl_sync(0xffffffffu, s, base + 1);
    const float s2 = __shfl_sync(0xffffffffu, s, base + 2);
    const float s3 = __shfl_sync(0xffffffffu, s, base + 3);
    if (ok && l == 0) xC[vec * dims.H + root] = __fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3);
}

// Sums the per-CTA partials in a fixed order and adds them into out[0..1].
__global__ void ReducePartialsKernel(const double* partials, int nblocks, double* out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        double s0 = 0.0, s1 = 0.0;
        for (int b = 0; b < nblocks; ++b) {
            s0 += partials[2 * b];
            s1 += partials[2 * b + 1];
        }
        out[0] += s0;
        out[1] += s1;
    }
}

// Per-vector MSE term alone (stlq_b200_sse): one thread per vector.
__global__ void SseKernel(Dims dims, const float* Gcol, const float* Gdiag, const float* xC, const double* xnorm2_d,
                          const void* B, const float* a, int64_t n, double* partials) {
    __shared__ double red[256];
    double s = 0.0;
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int code[kMaxM];
        for (int l = 0; l < dims.m; ++l) code[l] = LoadCode(B, v * dims.m + l, dims.wide);
        s += VectorSse(dims, GramGlobal{MakeGram(dims, Gcol, Gdiag), dims.off, code}, xC + v * dims.H, code, a + v * dims.m,
                       xnorm2_d[v]);
    }
    red[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < blockDim.x; ++i) t += red[i];
        partials[2 * blockIdx.x] = 0.0;
        partials[2 * blockIdx.x + 1] = t;
    }
}

cudaError_t LaunchRefine(const RefineArgs& args, int grid, cudaStream_t stream) {
    if (args.n <= 0) return cudaSuccess;
    if (args.ex.X && args.mode == 1) RefineKernel<true><<<grid, kRefineThreads, 0, stream>>>(args);
    else RefineKernel<false><<<grid, kRefineThreads, 0, stream>>>(args);
    return cudaGetLastError();
}

cudaError_t LaunchReducePartials(const double* partials, int nblocks, double* out, cudaStream_t stream) {
    ReducePartialsKernel<<<1, 32, 0, stream>>>(partials, nblocks, out);
    return cudaGetLastError();
}

cudaError_t LaunchSse(const Dims& dims, const float* Gcol, const float* Gdiag, const float* xC, const double* xnorm2_d,
                      const void* B, const float* a, int64_t n, double* partials, int grid, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    SseKernel<<<grid, 256, 0, stream>>>(dims, Gcol, Gdiag, xC, xnorm2_d, B, a, n, partials);
    return cudaGetLastError();
}

int RefineWarpsPerBlock() { return kWarps; }

int RefineBlocksPerSm() { return kRefineBlocksPerSm; }

// Large-root outputs from the internal m x n codes: cluster id (the root code) and the (m-1) small
// codes of each vector (BeamSearchPrefixLSLargeRoot's cluster_id / B_small, beam_search.h:26-32).
// Internal codes are uint16 when the root has more than 256 codewords.
__global__ void SplitRootCodesKernel(int m, const void* __restrict__ B, int wide, int64_t n,
                                     uint32_t* __restrict__ cluster, uint8_t* __restrict__ B_small) {
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        cluster[v] = static_cast<uint32_t>(LoadCode(B, v * m, wide));
        for (int l = 1; l < m; ++l) B_small[v * (m - 1) + l - 1] = static_cast<uint8_t>(LoadCode(B, v * m + l, wide));
    }
}

cudaError_t LaunchSplitRootCodes(int m, const void* B, int wide, int64_t n, uint32_t* cluster, uint8_t* B_small,
                                 cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 32));
    SplitRootCodesKernel<<<grid, 256, 0, stream>>>(m, B, wide, n, cluster, B_small);
    return cudaGetLastError();
}

cudaError_t LaunchRootDot(const Dims& dims, const float* C, const void* X, int x_dtype, const void* B, int64_t n,
                          float* xC, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int grid = static_cast<int>((n * 4 + 255) / 256);
    if (x_dtype == 0) RootDotKernel<float><<<grid, 256, 0, stream>>>(dims, C, static_cast<const float*>(X), B, n, xC);
    else RootDotKernel<uint8_t><<<grid, 256, 0, stream>>>(dims, C, static_cast<const uint8_t*>(X), B, n, xC);
    return cudaGetLastError();
}

}  // namespace stlq_b200
