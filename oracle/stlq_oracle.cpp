// CPU restatement of the reference's base-encoding hot path: TEST INFRASTRUCTURE ONLY.
// Loaded by tests/, __graft_entry__.smoke() and bench.py's baseline legs as the checker; the
// product path never links or calls it.  Compiled with -ffp-contract=off so that every `a*b+c`
// below rounds twice, like the reference's baseline-ISA (no FMA) build; the one place the
// reference's arithmetic does fuse (its BLAS kernel) calls std::fma explicitly.
// Function-by-function citations are in stlq_oracle.h.
#include "stlq_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <random>
#include <vector>

namespace {

inline float GAt(const float* G, int H, int row, int col) {
    return G[static_cast<size_t>(col) * H + row];
}

// OpenBLAS level-3 driver K split (driver/level3: min_l = GEMM_Q when >= 2*GEMM_Q remain,
// else half the remainder rounded up to the M unroll), measured here as GEMM_Q = 448.
int NextKBlock(int rem) {
    const int Q = 448, U = 16;
    if (rem >= 2 * Q) return Q;
    if (rem > Q) return ((rem / 2) + U - 1) & ~(U - 1);
    return rem;
}

}  // namespace

extern "C" void oracle_gemm_tn(int d, int rows, int n, const float* A, const float* X, float* out) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; ++j) {
        const float* x = X + static_cast<size_t>(j) * d;
        for (int r = 0; r < rows; ++r) {
            const float* c = A + static_cast<size_t>(r) * d;
            float acc = 0.0f;
            bool first = true;
            for (int k0 = 0; k0 < d;) {
                const int L = NextKBlock(d - k0);
                float part = 0.0f;
                for (int k = k0; k < k0 + L; ++k) part = std::fma(c[k], x[k], part);
                acc = first ? part : acc + part;
                first = false;
                k0 += L;
            }
            out[static_cast<size_t>(j) * rows + r] = acc;
        }
    }
}

extern "C" void oracle_xnorm2(int d, int n, const float* X, float* out) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; ++j) {
        const float* x = X + static_cast<size_t>(j) * d;
        float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int body = (d / 4) * 4;
        for (int i = 0; i < body; i += 4) {
            for (int l = 0; l < 4; ++l) {
                const float p = x[i + l] * x[i + l];
                lane[l] = lane[l] + p;
            }
        }
        for (int i = body; i < d; ++i) {
            const float p = x[i] * x[i];
            lane[0] = lane[0] + p;
        }
        float s = lane[0] + lane[1];
        s = s + lane[2];
        s = s + lane[3];
        out[j] = s;
    }
}

extern "C" void oracle_precomp(int d, int H, const float* C_all, float* G, float* invnorm) {
    oracle_gemm_tn(d, H, H, C_all, C_all, G);
    for (int h = 0; h < H; ++h) {
        const float* c = C_all + static_cast<size_t>(h) * d;
        float norm_sq = 0.0f;
        for (int r = 0; r < d; ++r) {
            const float p = c[r] * c[r];
            norm_sq = norm_sq + p;
        }
        invnorm[h] = norm_sq > 0.0f ? 1.0f / std::sqrt(norm_sq) : 0.0f;
    }
}

namespace {

// Per-thread beam state, one slot per beam entry: codes, coefficients, error and the upper
// Cholesky factor R (row-major, stride m) of the slot's prefix Gram matrix.
struct Beam {
    int m, B;
    std::vector<int> codes;    // [B][m]
    std::vector<float> a;      // [B][m]
    std::vector<float> err;    // [B]
    std::vector<float> R;      // [B][m][m]
    Beam(int m_, int B_) : m(m_), B(B_), codes(size_t(m_) * B_), a(size_t(m_) * B_), err(B_),
                           R(size_t(m_) * m_ * B_) {}
    float* Rp(int h) { return R.data() + static_cast<size_t>(h) * m * m; }
};

// First slot holding the maximum error (RecomputeWorst, beam_search.cpp:101-113).
int WorstSlot(const std::vector<float>& e, int B, float* worst) {
    int idx = 0;
    float we = e[0];
    for (int h = 1; h < B; ++h) {
        if (e[h] > we) {
            we = e[h];
            idx = h;
        }
    }
    *worst = we;
    return idx;
}

int CountFinite(const std::vector<float>& e, int B) {
    int c = 0;
    for (int h = 0; h < B; ++h) c += (e[h] < std::numeric_limits<float>::infinity());
    return c;
}

// Forward solve R^T y = b, then back solve R x = y, R upper with row stride `stride`
// (SolveCholUpperRawFixed, beam_search.cpp:127-162).
void SolveUpper(const float* R, int L, const float* b, float* x, float* y, int stride) {
    for (int i = 0; i < L; ++i) {
        float s = b[i];
        for (int k = 0; k < i; ++k) {
            const float p = R[k * stride + i] * y[k];
            s = s - p;
        }
        y[i] = s / R[i * stride + i];
    }
    for (int i = L - 1; i >= 0; --i) {
        float s = y[i];
        for (int k = i + 1; k < L; ++k) {
            const float p = R[i * stride + k] * x[k];
            s = s - p;
        }
        x[i] = s / R[i * stride + i];
    }
}

}  // namespace

extern "C" void oracle_beam_search(int m, const int* h_vec, int H, const float* G, int n,
                                   const float* xnorm2, const float* xC, int beam, uint16_t* Bout) {
    std::vector<int> off(m);
    for (int l = 0, o = 0; l < m; ++l) {
        off[l] = o;
        o += h_vec[l];
    }
    const int B = std::max(1, beam);
    const float inf = std::numeric_limits<float>::infinity();
#pragma omp parallel
    {
        Beam cur(m, B), nxt(m, B);
        std::vector<int> sel_h(B), sel_k(B);
        std::vector<float> sel_denom(B), sel_alast(B), sel_v(size_t(m) * B), sel_y(size_t(m) * B);
        std::vector<float> A(m), v(m), y(m);
#pragma omp for schedule(static)
        for (int i = 0; i < n; ++i) {
            const float* xc = xC + static_cast<size_t>(i) * H;
            const float nx2 = xnorm2[i];
            std::fill(cur.err.begin(), cur.err.end(), inf);
            std::fill(nxt.err.begin(), nxt.err.end(), inf);
            std::fill(nxt.R.begin(), nxt.R.end(), 0.0f);
            // Layer 0 (beam_search.cpp:238-263): e1 = ||x||^2 - gamma*a1, not clamped.
            float worst;
            int ws = WorstSlot(nxt.err, B, &worst);
            for (int k = 0; k < h_vec[0]; ++k) {
                const int flat = off[0] + k;
                const float alpha = GAt(G, H, flat, flat);
                if (alpha == 0.0f) continue;
                const float gamma = xc[flat];
                const float a1 = gamma / alpha;
                const float p = gamma * a1;
                const float e1 = nx2 - p;
                if (e1 >= worst) continue;
                nxt.err[ws] = e1;
                nxt.codes[size_t(ws) * m + 0] = k;
                nxt.a[size_t(ws) * m + 0] = a1;
                nxt.Rp(ws)[0] = std::sqrt(alpha);
                ws = WorstSlot(nxt.err, B, &worst);
            }
            int curH = CountFinite(nxt.err, B);
            std::swap(cur, nxt);
            for (int L = 1; L < m; ++L) {
                std::fill(nxt.err.begin(), nxt.err.end(), inf);
                ws = WorstSlot(nxt.err, B, &worst);
                std::fill(sel_h.begin(), sel_h.end(), -1);
                const int offL = off[L], K = h_vec[L];
                for (int h = 0; h < curH; ++h) {
                    const float* R = cur.Rp(h);
                    const float* a_old = cur.a.data() + size_t(h) * m;
                    const float E_old = cur.err[h];
                    for (int k = 0; k < K; ++k) {
                        const int flat = offL + k;
                        const float alpha = GAt(G, H, flat, flat);
                        const float gamma = xc[flat];
                        for (int t = 0; t < L; ++t) {
                            A[t] = GAt(G, H, off[t] + cur.codes[size_t(h) * m + t], flat);
                        }
                        SolveUpper(R, L, A.data(), v.data(), y.data(), m);
                        float delta = 0.0f, eta = 0.0f;
                        for (int t = 0; t < L; ++t) {
                            const float pd = A[t] * v[t];
                            delta = delta + pd;
                            const float pe = A[t] * a_old[t];
                            eta = eta + pe;
                        }
                        const float denom = alpha - delta;
                        if (denom == 0.0f) continue;
                        const float diff = gamma - eta;
                        const float a_last = diff / denom;
                        const float pr = diff * a_last;
                        float e = E_old - pr;
                        if (e < 0.0f) e = 0.0f;
                        if (e >= worst) continue;
                        nxt.err[ws] = e;
                        sel_h[ws] = h;
                        sel_k[ws] = k;
                        sel_denom[ws] = denom;
                        sel_alast[ws] = a_last;
                        for (int t = 0; t < L; ++t) {
                            sel_v[size_t(t) * B + ws] = v[t];
                            sel_y[size_t(t) * B + ws] = y[t];
                        }
                        ws = WorstSlot(nxt.err, B, &worst);
                    }
                }
                // Winner materialisation (beam_search.cpp:337-383).
                for (int o = 0; o < B; ++o) {
                    if (nxt.err[o] >= inf) continue;
                    const int src = sel_h[o];
                    for (int t = 0; t < L; ++t) nxt.codes[size_t(o) * m + t] = cur.codes[size_t(src) * m + t];
                    nxt.codes[size_t(o) * m + L] = sel_k[o];
                    const float al = sel_alast[o];
                    for (int t = 0; t < L; ++t) {
                        const float p = sel_v[size_t(t) * B + o] * al;
                        nxt.a[size_t(o) * m + t] = cur.a[size_t(src) * m + t] - p;
                    }
                    nxt.a[size_t(o) * m + L] = al;
                    float* Rn = nxt.Rp(o);
                    std::memcpy(Rn, cur.Rp(src), sizeof(float) * L * m);
                    for (int t = 0; t < L; ++t) Rn[t * m + L] = sel_y[size_t(t) * B + o];
                    Rn[L * m + L] = std::sqrt(sel_denom[o]);
                }
                int newH = CountFinite(nxt.err, B);
                if (newH == 0) {
                    // Fallback (beam_search.cpp:385-400).  The reference copies position L of
                    // each slot from a stale buffer; this restatement writes code 0 there.
                    newH = std::min(curH, B);
                    for (int h = 0; h < newH; ++h) {
                        nxt.err[h] = cur.err[h];
                        for (int t = 0; t <= L; ++t) {
                            nxt.codes[size_t(h) * m + t] = t < L ? cur.codes[size_t(h) * m + t] : 0;
                            nxt.a[size_t(h) * m + t] = t < L ? cur.a[size_t(h) * m + t] : 0.0f;
                        }
                        std::memcpy(nxt.Rp(h), cur.Rp(h), sizeof(float) * m * m);
                    }
                }
                curH = std::max(1, newH);
                std::swap(cur, nxt);
            }
            int best = 0;
            float be = cur.err[0];
            for (int h = 1; h < curH; ++h) {
                if (cur.err[h] < be) {
                    be = cur.err[h];
                    best = h;
                }
            }
            for (int l = 0; l < m; ++l) Bout[static_cast<size_t>(i) * m + l] = static_cast<uint16_t>(cur.codes[size_t(best) * m + l]);
        }
    }
}

namespace {

constexpr float kEps = 1e-6f;

// Fixed-size Cholesky for m in {5, 10} (CholeskyUpperFixed, least_squares.cpp:44-66): A is
// row-major [r*m+c], upper triangle filled; fails when a pivot is <= 1e-6.
bool CholFixed(float* A, int m) {
    for (int k = 0; k < m; ++k) {
        float sum = A[k * m + k];
        for (int j = 0; j < k; ++j) {
            const float v = A[j * m + k];
            const float p = v * v;
            sum = sum - p;
        }
        if (sum <= kEps) return false;
        const float diag = std::sqrt(sum);
        A[k * m + k] = diag;
        for (int i = k + 1; i < m; ++i) {
            float s = A[k * m + i];
            for (int j = 0; j < k; ++j) {
                const float p = A[j * m + k] * A[j * m + i];
                s = s - p;
            }
            A[k * m + i] = s / diag;
        }
    }
    return true;
}

// LAPACK spotrf('U') + spotrs for the other m (least_squares.cpp:278-316), in the arithmetic of
// the BLAS/LAPACK the reference links in this image (OpenBLAS 0.3.15, SkylakeX kernels), measured
// element by element against that library (oracle/Makefile links it into oracle/_ref):
//  * spotrf = xPOTF2 for m <= 32: pivot a_jj - dot(U[0:j,j], U[0:j,j]) with float products summed
//    in double; the row update is y - U[0:j,c].U[0:j,j] through the SGEMV-T kernel (rows in
//    blocks of 4: 4-column groups use 4 FMA lanes [+ 8-lane steps] reduced (l0+l1)+(l2+l3), the
//    remaining columns 4 mul/add lanes; the last j%4 rows added by contracted FMAs); then the row
//    is scaled by the float reciprocal of the pivot.  A pivot <= 0 fails (NaN does not).
//  * spotrs = two STRSM calls: triangular blocks of 16/8/4/2/1 rows, each solved by multiplying
//    with the reciprocal diagonal and FMA updates, blocks joined by FMA-chain GEMM updates.
float PotfBlockAvx(const float* a, const float* x, int nb) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int r = 0;
    if (nb & 4) {
        for (int l = 0; l < 4; ++l) lane[l] = std::fma(a[l], x[l], lane[l]);
        r = 4;
    }
    for (; r < nb; r += 8)
        for (int l = 0; l < 8; ++l) lane[l] = std::fma(a[r + l], x[r + l], lane[l]);
    float q[4];
    for (int l = 0; l < 4; ++l) q[l] = lane[l] + lane[l + 4];
    return (q[0] + q[1]) + (q[2] + q[3]);
}

float PotfBlockSse(const float* a, const float* x, int nb) {
    float lane[4] = {0, 0, 0, 0};
    for (int r = 0; r < nb; r += 4)
        for (int l = 0; l < 4; ++l) {
            const float p = a[r + l] * x[r + l];
            lane[l] = lane[l] + p;
        }
    return (lane[0] + lane[1]) + (lane[2] + lane[3]);
}

float PotfLeftover(float y, const float* a, const float* x, int m1, int m3) {
    if (m3 == 0) return y;
    const float xt0 = -x[m1];
    if (m3 == 1) return std::fma(a[m1], xt0, y);
    const float xt1 = -x[m1 + 1];
    const float p1 = a[m1 + 1] * xt1;
    float e = std::fma(a[m1], xt0, p1);
    if (m3 == 3) e = std::fma(a[m1 + 2], -x[m1 + 2], e);
    return y + e;
}

bool CholLapack(float* A, int m) {  // column-major A[r + c*m], upper triangle
    for (int j = 0; j < m; ++j) {
        const float* xj = A + static_cast<size_t>(j) * m;
        double acc = 0.0;
        for (int k = 0; k < j; ++k) {
            const float p = xj[k] * xj[k];
            acc += static_cast<double>(p);
        }
        float ajj = A[j + j * m] - static_cast<float>(acc);
        if (ajj <= 0.0f) return false;
        ajj = std::sqrt(ajj);
        A[j + j * m] = ajj;
        const float r = 1.0f / ajj;
        const int ncol = m - j - 1, m3 = j & 3, m1 = j - m3, n1 = (ncol >> 2) * 4;
        for (int ci = 0; ci < ncol; ++ci) {
            const int c = j + 1 + ci;
            const float* ac = A + static_cast<size_t>(c) * m;
            float y = A[j + c * m];
            if (m1 > 0) {
                const float K = ci < n1 ? PotfBlockAvx(ac, xj, m1) : PotfBlockSse(ac, xj, m1);
                y = std::fma(K, -1.0f, y);
            }
            y = PotfLeftover(y, ac, xj, m1, m3);
            A[j + c * m] = y * r;
        }
    }
    return true;
}

void TrsmRowsUpdate(const float* A, int m, float* c, int r0, int nr, int t0, int t1, bool upper_t) {
    // c[r] -= sum_{t in [t0,t1)} U(t,r) c[t] (forward, upper_t) or U(r,t) c[t] (backward), as an
    // FMA chain from zero, subtracted once.
    for (int r = r0; r < r0 + nr; ++r) {
        float acc = 0.0f;
        for (int t = t0; t < t1; ++t) acc = std::fma(upper_t ? A[t + r * m] : A[r + t * m], c[t], acc);
        c[r] = std::fma(acc, -1.0f, c[r]);
    }
}

void SolveLapack(const float* A, int m, float* c) {  // U^T y = b, then U x = y, in place
    const int UM = 16;
    int kk = 0;
    auto fwd = [&](int r0, int bs) {
        for (int i = r0; i < r0 + bs; ++i) {
            const float bb = c[i] * (1.0f / A[i + i * m]);
            c[i] = bb;
            for (int k = i + 1; k < r0 + bs; ++k) c[k] = std::fma(-bb, A[i + k * m], c[k]);
        }
    };
    auto bwd = [&](int r0, int bs) {
        for (int i = r0 + bs - 1; i >= r0; --i) {
            const float bb = c[i] * (1.0f / A[i + i * m]);
            c[i] = bb;
            for (int k = r0; k < i; ++k) c[k] = std::fma(-bb, A[k + i * m], c[k]);
        }
    };
    for (int b = 0; b < m / UM; ++b) {
        if (kk > 0) TrsmRowsUpdate(A, m, c, kk, UM, 0, kk, true);
        fwd(kk, UM);
        kk += UM;
    }
    for (int i = UM / 2; i > 0; i >>= 1) {
        if (!(m & i)) continue;
        if (kk > 0) TrsmRowsUpdate(A, m, c, kk, i, 0, kk, true);
        fwd(kk, i);
        kk += i;
    }
    kk = m;
    for (int i = 1; i < UM; i *= 2) {
        if (!(m & i)) continue;
        const int st = (m & ~(i - 1)) - i;
        if (m - kk > 0) TrsmRowsUpdate(A, m, c, st, i, kk, m, false);
        bwd(st, i);
        kk -= i;
    }
    for (int b = m / UM - 1; b >= 0; --b) {
        const int st = b * UM;
        if (m - kk > 0) TrsmRowsUpdate(A, m, c, st, UM, kk, m, false);
        bwd(st, UM);
        kk -= UM;
    }
}

// One vector's LS solve (SolveLeastSquaresSample, least_squares.cpp:252-318 and the fixed-m
// path :86-129) with the 3 diagonal-bump retries.  codes[l] is the layer-l code.
bool SolveLsSample(int m, const int* off, int H, const float* G, const float* xc, const uint16_t* codes,
                   float* a_out) {
    std::vector<float> A(size_t(m) * m), b(m), x(m), y(m);
    const bool fixed = (m == 5 || m == 10);
    auto fill = [&](float lambda) {
        std::fill(A.begin(), A.end(), 0.0f);
        for (int j = 0; j < m; ++j) {
            const int fj = off[j] + codes[j];
            b[j] = xc[fj];
            for (int k = 0; k <= j; ++k) {
                const int fk = off[k] + codes[k];
                // row k, col j: fixed path is row-major A[k*m+j]; LAPACK path column-major A[k+j*m]
                if (fixed) A[size_t(k) * m + j] = GAt(G, H, fk, fj);
                else A[size_t(k) + size_t(j) * m] = GAt(G, H, fk, fj);
            }
            if (fixed) A[size_t(j) * m + j] = A[size_t(j) * m + j] + lambda;
            else A[size_t(j) + size_t(j) * m] = A[size_t(j) + size_t(j) * m] + lambda;
        }
    };
    fill(0.0f);
    bool ok = fixed ? CholFixed(A.data(), m) : CholLapack(A.data(), m);
    float bump = kEps;
    for (int attempt = 0; attempt < 3 && !ok; ++attempt) {
        fill(bump);
        ok = fixed ? CholFixed(A.data(), m) : CholLapack(A.data(), m);
        bump *= 10.0f;
    }
    if (!ok) return false;
    if (fixed) {
        SolveUpper(A.data(), m, b.data(), x.data(), y.data(), m);
        std::copy(x.begin(), x.end(), a_out);
    } else {
        SolveLapack(A.data(), m, b.data());
        std::copy(b.begin(), b.end(), a_out);
    }
    return true;
}

// SampleCost (cost_utils.cpp:112-137): ||x||^2 - 2*term1 + term2 in float.
float SampleCost(int m, const int* off, int H, const float* G, const float* xc, const uint16_t* codes,
                 const float* a, float xn2) {
    float term1 = 0.0f, term2 = 0.0f;
    for (int l = 0; l < m; ++l) {
        const int fl = off[l] + codes[l];
        const float p1 = a[l] * xc[fl];
        term1 = term1 + p1;
        for (int k = 0; k < m; ++k) {
            const int fk = off[k] + codes[k];
            const float aa = a[l] * a[k];
            const float p2 = aa * GAt(G, H, fl, fk);
            term2 = term2 + p2;
        }
    }
    const float t = 2.0f * term1;
    const float r = xn2 - t;
    return r + term2;
}

std::vector<int> Offsets(int m, const int* h_vec) {
    std::vector<int> off(m);
    for (int l = 0, o = 0; l < m; ++l) {
        off[l] = o;
        o += h_vec[l];
    }
    return off;
}

}  // namespace

extern "C" int oracle_solve_ls_all(int m, const int* h_vec, int H, const float* G, int n, const float* xC,
                                   const uint16_t* B, float* a) {
    const std::vector<int> off = Offsets(m, h_vec);
    int fails = 0;
#pragma omp parallel for schedule(static) reduction(+ : fails)
    for (int i = 0; i < n; ++i) {
        float* ai = a + size_t(i) * m;
        if (!SolveLsSample(m, off.data(), H, G, xC + size_t(i) * H, B + size_t(i) * m, ai)) {
            std::fill(ai, ai + m, 0.0f);
            ++fails;
        }
    }
    return fails;
}

extern "C" void oracle_costs(int m, const int* h_vec, int H, const float* G, int n, const float* xC,
                             const uint16_t* B, const float* a, const float* xnorm2, float* cost) {
    const std::vector<int> off = Offsets(m, h_vec);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        cost[i] = SampleCost(m, off.data(), H, G, xC + size_t(i) * H, B + size_t(i) * m, a + size_t(i) * m,
                             xnorm2[i]);
    }
}

extern "C" double oracle_sse(int d, int m, const int* h_vec, int H, const float* G, int n, const float* X,
                             const float* xC, const uint16_t* B, const float* a) {
    const std::vector<int> off = Offsets(m, h_vec);
    double sum = 0.0;
#pragma omp parallel for schedule(static) reduction(+ : sum)
    for (int i = 0; i < n; ++i) {
        const float* x = X + size_t(i) * d;
        double nx = 0.0;
        for (int r = 0; r < d; ++r) nx += double(x[r]) * double(x[r]);
        const float* xc = xC + size_t(i) * H;
        const uint16_t* c = B + size_t(i) * m;
        const float* ai = a + size_t(i) * m;
        double t1 = 0.0, t2 = 0.0;
        for (int j = 0; j < m; ++j) t1 += double(ai[j]) * double(xc[off[j] + c[j]]);
        for (int j = 0; j < m; ++j)
            for (int k = 0; k < m; ++k)
                t2 += double(ai[j]) * double(ai[k]) * double(GAt(G, H, off[j] + c[j], off[k] + c[k]));
        double e = nx - 2.0 * t1 + t2;
        sum += e < 0.0 ? 0.0 : e;
    }
    return sum;
}

extern "C" void oracle_icm_orders(int m, int icm_iters, int ils_iters, uint32_t seed, int* orders) {
    std::mt19937 rng(static_cast<std::mt19937::result_type>(seed));
    std::vector<int> order(m);
    size_t w = 0;
    for (int call = 0; call <= ils_iters; ++call) {
        std::iota(order.begin(), order.end(), 0);
        for (int it = 0; it < icm_iters; ++it) {
            std::shuffle(order.begin(), order.end(), rng);
            for (int l = 0; l < m; ++l) orders[w++] = order[l];
        }
    }
}

namespace {

struct SplitMix64 {  // icm.cpp:55-65
    uint64_t state;
    uint64_t Next() {
        uint64_t z = (state += 0x9e3779b97f4a7c15ULL);
        z = (z ^ (z >> 30U)) * 0xbf58476d1ce4e5b9ULL;
        z = (z ^ (z >> 27U)) * 0x94d049bb133111ebULL;
        return z ^ (z >> 31U);
    }
};

uint32_t UniformBelow(SplitMix64* r, uint32_t bound) {  // icm.cpp:76-87
    const unsigned __int128 p = static_cast<unsigned __int128>(r->Next()) * bound;
    return static_cast<uint32_t>(p >> 64);
}

// One RunIcm call (icm.cpp:89-344) for one vector: LS + cost, then icm_iters sweeps in the
// given layer orders; layer 0 is never changed; a change is kept only if it lowers the cost
// by more than 1e-6.
void RunIcmVector(int m, const int* h_vec, const int* off, int H, const float* G, const float* invnorm,
                  const float* xc, float xn2, int icm_iters, const int* orders, int use_abs,
                  uint16_t* codes, float* a, float* cost) {
    if (!SolveLsSample(m, off, H, G, xc, codes, a)) std::fill(a, a + m, 0.0f);
    *cost = SampleCost(m, off, H, G, xc, codes, a, xn2);
    bool active = true;
    std::vector<float> tmp, backup(m);
    for (int it = 0; it < icm_iters; ++it) {
        bool changed = false;
        const int* order = orders + size_t(it) * m;
        for (int oi = 0; oi < m; ++oi) {
            const int j = order[oi];
            if (j == 0) continue;
            const int hj = h_vec[j], startf = off[j];
            if (hj <= 1) continue;
            if (!active) continue;
            const int old_code = codes[j];
            tmp.assign(xc + startf, xc + startf + hj);
            for (int l = 0; l < m; ++l) {
                if (l == j) continue;
                const float al = a[l];
                const int fl = off[l] + codes[l];
                for (int t = 0; t < hj; ++t) {
                    const float p = al * GAt(G, H, startf + t, fl);
                    tmp[t] = tmp[t] - p;
                }
            }
            int best = old_code;
            float best_score = -std::numeric_limits<float>::infinity();
            for (int t = 0; t < hj; ++t) {
                const float val = tmp[t] * invnorm[startf + t];
                const float score = use_abs ? std::fabs(val) : val;
                if (score > best_score) {
                    best_score = score;
                    best = t;
                }
            }
            if (best == old_code) continue;
            std::copy(a, a + m, backup.begin());
            codes[j] = static_cast<uint16_t>(best);
            if (!SolveLsSample(m, off, H, G, xc, codes, a)) {
                codes[j] = static_cast<uint16_t>(old_code);
                std::copy(backup.begin(), backup.end(), a);
                continue;
            }
            const float nc = SampleCost(m, off, H, G, xc, codes, a, xn2);
            if (nc + kEps < *cost) {
                *cost = nc;
                changed = true;
            } else {
                codes[j] = static_cast<uint16_t>(old_code);
                std::copy(backup.begin(), backup.end(), a);
            }
        }
        if (active && !changed) active = false;
    }
}

}  // namespace

extern "C" void oracle_icm(int m, const int* h_vec, int H, const float* G, const float* invnorm, int n,
                           const float* xC, const float* xnorm2, int icm_iters, int ils_iters, int perturb_k,
                           int use_abs, uint32_t seed, uint64_t sample_id_offset, uint16_t* B, float* a,
                           float* cost) {
    const std::vector<int> off = Offsets(m, h_vec);
    const int n_ils = (ils_iters <= 0 || perturb_k <= 0 || m <= 1) ? 0 : ils_iters;
    std::vector<int> orders(size_t(n_ils + 1) * std::max(icm_iters, 0) * m + 1);
    oracle_icm_orders(m, std::max(icm_iters, 0), n_ils, seed, orders.data());
    const int ksel = std::min(perturb_k, m);
    const size_t per_call = size_t(std::max(icm_iters, 0)) * m;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        const float* xc = xC + size_t(i) * H;
        uint16_t* ci = B + size_t(i) * m;
        float* ai = a + size_t(i) * m;
        RunIcmVector(m, h_vec, off.data(), H, G, invnorm, xc, xnorm2[i], icm_iters, orders.data(), use_abs, ci,
                     ai, &cost[i]);
        std::vector<uint16_t> cand(m);
        std::vector<float> acand(m);
        for (int outer = 0; outer < n_ils; ++outer) {
            std::copy(ci, ci + m, cand.begin());
            const uint64_t ig = sample_id_offset + static_cast<uint64_t>(i);
            SplitMix64 r{static_cast<uint64_t>(seed) ^ (static_cast<uint64_t>(outer + 1) * 0x9e3779b97f4a7c15ULL) ^
                         ((ig + 1) * 0xbf58476d1ce4e5b9ULL)};
            for (int s = 0; s < ksel; ++s) {  // icm.cpp:953-972
                const int layer = 1 + static_cast<int>(UniformBelow(&r, static_cast<uint32_t>(m - 1)));
                const int h = h_vec[layer];
                if (h <= 1) continue;
                const int old_code = cand[layer];
                const int raw = static_cast<int>(UniformBelow(&r, static_cast<uint32_t>(h - 1)));
                cand[layer] = static_cast<uint16_t>(raw >= old_code ? raw + 1 : raw);
            }
            float ccost;
            RunIcmVector(m, h_vec, off.data(), H, G, invnorm, xc, xnorm2[i], icm_iters,
                         orders.data() + per_call * (outer + 1), use_abs, cand.data(), acand.data(), &ccost);
            if (ccost + kEps < cost[i]) {  // icm.cpp:979-990
                std::copy(cand.begin(), cand.end(), ci);
                std::copy(acand.begin(), acand.end(), ai);
                cost[i] = ccost;
            }
        }
    }
}
