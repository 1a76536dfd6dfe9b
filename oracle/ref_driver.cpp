// Test infrastructure only (parity checker and CPU baseline); never part of the product path.
//
// A thin extern "C" driver around the REFERENCE's own hot-path functions, compiled from the
// reference sources where they lie (oracle/Makefile lists them).  Python tests and bench.py's
// reference arm load the resulting oracle/_ref/libstlq_ref.so through ctypes.
//
// Every entry point calls the reference's code; the only logic restated here is the glue that
// the reference keeps in translation units too heavy to compile on their own:
//   - ref_precomp_create restates BuildPrecomp (src/quantizer/encoder_precomp.inc:1-53)
//     and calls the reference's stlq::Gemm for G, exactly as BuildPrecomp does.
//   - ref_encode_base restates the stage order of EncodeBase
//     (src/quantizer/encoder_encode_base.inc:1-106), CPU branch.
//   - ref_large_root_encode restates the stage order of the large pipeline's basic encode
//     (src/quantizer/encode_base_streaming.cpp:1040-1300, CPU branch).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <omp.h>

#include "stlq/common/types.h"
#include "stlq/core/blas.h"
#include "stlq/core/threading.h"
#include "stlq/linkage/linkage_summary.h"
#include "stlq/quantizer/beam_search.h"
#include "stlq/quantizer/cost_utils.h"
#include "stlq/quantizer/icm.h"
#include "stlq/quantizer/least_squares.h"
#include "stlq/quantizer/precomp_large_root.h"

extern "C" char* openblas_get_corename(void);

namespace {

using stlq::ColMajorMatrix;
using stlq::FullCode;
using stlq::Precomp;

ColMajorMatrix<float> Wrap(const float* p, int rows, int cols) {
    ColMajorMatrix<float> m(rows, cols);
    std::memcpy(m.data.data(), p, sizeof(float) * static_cast<std::size_t>(rows) * cols);
    return m;
}

ColMajorMatrix<FullCode> WrapCodes(const std::uint8_t* p, int rows, int cols) {
    ColMajorMatrix<FullCode> m(rows, cols);
    std::memcpy(m.data.data(), p, static_cast<std::size_t>(rows) * cols);
    return m;
}

double Now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

extern "C" void openblas_set_num_threads(int);

extern "C" {

const char* ref_blas_core(void) { return openblas_get_corename(); }

void ref_set_threads(int n) {
    omp_set_num_threads(std::max(1, n));
    stlq::SetOmpDefaultThreads(std::max(1, n));
    stlq::BlasSetThreads(1);
}

int ref_max_threads(void) { return omp_get_max_threads(); }

// Restates BuildPrecomp (encoder_precomp.inc:1-53): C_all = concat of books, invnorm, offsets,
// flat_layer, and G = C_all^T C_all through the reference's stlq::Gemm.
void* ref_precomp_create(int d, int m, const int* h_vec, const float* C_all) {
    auto* p = new Precomp();
    int H = 0;
    for (int l = 0; l < m; ++l) H += h_vec[l];
    p->C_all = Wrap(C_all, d, H);
    p->G = ColMajorMatrix<float>(H, H);
    p->offsets.resize(m);
    p->flat_layer.resize(H);
    p->invnorm_flat.resize(H);
    p->h_vec.assign(h_vec, h_vec + m);
    p->H = H;
    p->m = m;
    p->d = d;
    int off = 0;
    for (int l = 0; l < m; ++l) {
        p->offsets[l] = off;
        for (int c = 0; c < h_vec[l]; ++c) {
            const float* col = p->C_all.Col(off + c);
            float norm_sq = 0.0f;
            for (int r = 0; r < d; ++r) norm_sq += col[r] * col[r];
            p->flat_layer[off + c] = l;
            p->invnorm_flat[off + c] = norm_sq > 0.0f ? 1.0f / std::sqrt(norm_sq) : 0.0f;
        }
        off += h_vec[l];
    }
    {
        stlq::ScopedBlasThreads blas_scope(stlq::OmpMaxThreads());
        stlq::Gemm(true, false, 1.0f, p->C_all, p->C_all, 0.0f, &p->G);
    }
    static std::uint64_t tag = 0;
    p->build_tag = ++tag;
    return p;
}

void ref_precomp_destroy(void* h) { delete static_cast<Precomp*>(h); }

int ref_precomp_H(void* h) { return static_cast<Precomp*>(h)->H; }

void ref_precomp_get(void* h, float* G_out, float* invnorm_out) {
    const auto* p = static_cast<Precomp*>(h);
    if (G_out) std::memcpy(G_out, p->G.data.data(), sizeof(float) * p->G.data.size());
    if (invnorm_out) std::memcpy(invnorm_out, p->invnorm_flat.data(), sizeof(float) * p->H);
}

// xC = C_all^T X with the reference's Gemm (encoder_encode_base.inc:33-37).
void ref_gemm_xc(void* h, const float* X, int n, float* xC_out) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> Xm = Wrap(X, p->d, n);
    ColMajorMatrix<float> xC(p->H, n);
    {
        stlq::ScopedBlasThreads blas_scope(stlq::OmpMaxThreads());
        stlq::Gemm(true, false, 1.0f, p->C_all, Xm, 0.0f, &xC);
    }
    std::memcpy(xC_out, xC.data.data(), sizeof(float) * xC.data.size());
}

// BeamSearchPrefixLS (beam_search.cpp:196-422).
void ref_beam_search(void* h, const float* X, int n, const float* xC, int beam, std::uint8_t* B_out) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> Xm = Wrap(X, p->d, n);
    ColMajorMatrix<float> xCm = Wrap(xC, p->H, n);
    ColMajorMatrix<FullCode> B;
    stlq::BeamSearchPrefixLS(Xm, *p, xCm, std::max(1, beam), &B);
    std::memcpy(B_out, B.data.data(), B.data.size());
}

// SolveLeastSquaresAll (least_squares.cpp:406+).
void ref_solve_ls(void* h, const float* xC, int n, const std::uint8_t* B, float* a_out) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> xCm = Wrap(xC, p->H, n);
    ColMajorMatrix<FullCode> Bm = WrapCodes(B, p->m, n);
    ColMajorMatrix<float> a;
    stlq::SolveLeastSquaresAll(*p, xCm, Bm, &a);
    std::memcpy(a_out, a.data.data(), sizeof(float) * a.data.size());
}

// ComputeXNorm2 (cost_utils.cpp:88-110).
void ref_xnorm2(const float* X, int d, int n, float* out) {
    ColMajorMatrix<float> Xm = Wrap(X, d, n);
    std::vector<float> v;
    stlq::ComputeXNorm2(Xm, &v);
    std::memcpy(out, v.data(), sizeof(float) * v.size());
}

// ComputeCosts (cost_utils.cpp:139-158).
void ref_costs(void* h, const float* xC, int n, const std::uint8_t* B, const float* a,
               const float* xnorm2, float* out) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> xCm = Wrap(xC, p->H, n);
    ColMajorMatrix<FullCode> Bm = WrapCodes(B, p->m, n);
    ColMajorMatrix<float> am = Wrap(a, p->m, n);
    std::vector<float> xn(xnorm2, xnorm2 + n), c;
    stlq::ComputeCosts(*p, xCm, Bm, am, xn, &c);
    std::memcpy(out, c.data(), sizeof(float) * c.size());
}

// MeanMseFromPrecomp (src/linkage/linkage_tools.cpp:170-219).
float ref_mean_mse(void* h, const float* X, int n, const float* xC, const std::uint8_t* B, const float* a) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> Xm = Wrap(X, p->d, n);
    ColMajorMatrix<float> xCm = Wrap(xC, p->H, n);
    ColMajorMatrix<FullCode> Bm = WrapCodes(B, p->m, n);
    ColMajorMatrix<float> am = Wrap(a, p->m, n);
    return stlq::MeanMseFromPrecomp(Xm, *p, xCm, Bm, am);
}

// DynamicIcmWithIls{Abs,NoAbs}NoNormal (icm.cpp:872-1003, 1132-1170).  B is in/out; a and cost
// are outputs (cost may be null).
void ref_icm(void* h, const float* X, int n, const float* xC, int icm_iters, int ils_iters, int perturb_k,
             int use_abs, std::uint32_t seed, std::uint64_t sample_id_offset, std::uint8_t* B_io,
             float* a_out, float* cost_out) {
    const auto* p = static_cast<Precomp*>(h);
    ColMajorMatrix<float> Xm = Wrap(X, p->d, n);
    ColMajorMatrix<float> xCm = Wrap(xC, p->H, n);
    ColMajorMatrix<FullCode> Bm = WrapCodes(B_io, p->m, n);
    ColMajorMatrix<float> a;
    std::vector<float> xn, cost;
    if (use_abs) {
        stlq::DynamicIcmWithIlsAbsNoNormal(Xm, *p, xCm, icm_iters, ils_iters, perturb_k, seed, &Bm, &a, &xn,
                                           &cost, false, sample_id_offset);
    } else {
        stlq::DynamicIcmWithIlsNoAbsNoNormal(Xm, *p, xCm, icm_iters, ils_iters, perturb_k, seed, &Bm, &a, &xn,
                                             &cost, false, sample_id_offset);
    }
    std::memcpy(B_io, Bm.data.data(), Bm.data.size());
    if (a_out) std::memcpy(a_out, a.data.data(), sizeof(float) * a.data.size());
    if (cost_out) std::memcpy(cost_out, cost.data(), sizeof(float) * cost.size());
}

// The CPU branch of EncodeBase (encoder_encode_base.inc:1-106), stage by stage.
// t_stages (optional, 5 doubles): seconds in GEMM, beam, LS + beam MSE, ICM, final MSE.
int ref_encode_base(void* h, const float* X, int n, int beam, int icm_iters, int ils_iters, int perturb_k,
                    int use_abs, std::uint32_t seed, std::uint8_t* B_out, float* a_out, float* cost_out,
                    float* beam_mse, float* final_mse, double* t_stages) {
    const auto* p = static_cast<Precomp*>(h);
    if (n <= 0 || p->d <= 0) return 1;
    double t0 = Now();
    ColMajorMatrix<float> Xm = Wrap(X, p->d, n);
    ColMajorMatrix<float> xC(p->H, n);
    {
        stlq::ScopedBlasThreads blas_scope(stlq::OmpMaxThreads());
        stlq::Gemm(true, false, 1.0f, p->C_all, Xm, 0.0f, &xC);
    }
    double t1 = Now();
    stlq::BaseEncoding base;
    stlq::BeamSearchPrefixLS(Xm, *p, xC, std::max(1, beam), &base.B);
    double t2 = Now();
    stlq::SolveLeastSquaresAll(*p, xC, base.B, &base.a);
    const float bm = stlq::MeanMseFromPrecomp(Xm, *p, xC, base.B, base.a);
    double t3 = Now();
    std::vector<float> xn, cost;
    if (use_abs) {
        stlq::DynamicIcmWithIlsAbsNoNormal(Xm, *p, xC, icm_iters, ils_iters, perturb_k, seed, &base.B, &base.a,
                                           &xn, &cost, false, 0);
    } else {
        stlq::DynamicIcmWithIlsNoAbsNoNormal(Xm, *p, xC, icm_iters, ils_iters, perturb_k, seed, &base.B,
                                             &base.a, &xn, &cost, false, 0);
    }
    double t4 = Now();
    const float fm = stlq::MeanMseFromPrecomp(Xm, *p, xC, base.B, base.a);
    double t5 = Now();
    std::memcpy(B_out, base.B.data.data(), base.B.data.size());
    if (a_out) std::memcpy(a_out, base.a.data.data(), sizeof(float) * base.a.data.size());
    if (cost_out && cost.size() == static_cast<std::size_t>(n)) {
        std::memcpy(cost_out, cost.data(), sizeof(float) * n);
    }
    if (beam_mse) *beam_mse = bm;
    if (final_mse) *final_mse = fm;
    if (t_stages) {
        t_stages[0] = t1 - t0;
        t_stages[1] = t2 - t1;
        t_stages[2] = t3 - t2;
        t_stages[3] = t4 - t3;
        t_stages[4] = t5 - t4;
    }
    return 0;
}

// ApplyRotationInPlace's product (src/pipeline/app_utils.cpp:203-227): X_rot = R X with the
// reference's GemmRaw (no transposes), R d x d and X d x n column-major.  (The identity test that
// skips it is left to the caller.)
// The reference's BLAS wrapper as the kernel providers call it (stlq::GemmRaw,
// src/core/blas.cpp:61-80): column-major sgemm with `threads` BLAS threads.  The thread count goes
// straight to OpenBLAS: BlasSetThreads caches the last value per copy of blas.cpp, and the tests
// load two libraries with their own copies over one OpenBLAS.
void ref_gemm(int trans_a, int trans_b, int m, int n, int k, float alpha, const float* A, int lda, const float* B,
              int ldb, float beta, float* C, int ldc, int threads) {
    openblas_set_num_threads(threads);
    stlq::GemmRaw(trans_a != 0, trans_b != 0, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc);
}

void ref_rotate(const float* R, int d, const float* X, int n, float* out) {
    stlq::ScopedBlasThreads blas_scope(stlq::OmpMaxThreads());
    stlq::GemmRaw(false, false, d, n, d, 1.0f, R, d, X, d, 0.0f, out, d);
}

// Large-root basic encode: BuildPrecompLargeRoot (codebook 0 is the root), ComputeXcSmall,
// BeamSearchPrefixLSLargeRoot, SolveLeastSquaresAllLargeRoot + ComputeCostsLargeRoot (the beam
// costs), DynamicIcmWithIls{Abs,NoAbs}NoNormalLargeRoot (final codes, coefficients and costs).
// C_all: d x H column-major, root codewords first.  Outputs: cluster (n), B_small ((m-1) x n),
// a (m x n), cost_beam and cost (n each; may be null).  Returns 0 on success.
int ref_large_root_encode(int d, int m, const int* h_vec, const float* C_all, const float* X, int n, int beam,
                          int icm_iters, int ils_iters, int perturb_k, int use_abs, std::uint32_t seed,
                          std::uint64_t sample_id_offset, std::uint32_t* cluster_out, std::uint8_t* B_small_out,
                          float* a_out, float* cost_beam_out, float* cost_out) {
    if (n <= 0 || d <= 0 || m <= 0) return 1;
    stlq::CodebookPack pack;
    pack.d = d;
    int off = 0;
    for (int l = 0; l < m; ++l) {
        pack.h_vec.push_back(h_vec[l]);
        pack.books.push_back(Wrap(C_all + static_cast<std::size_t>(off) * d, d, h_vec[l]));
        off += h_vec[l];
    }
    stlq::PrecompLargeRoot pre;
    stlq::PrecompLargeRootBuildOptions opts;
    std::string err;
    if (!stlq::BuildPrecompLargeRoot(pack, nullptr, opts, &pre, &err)) return 2;
    ColMajorMatrix<float> Xm = Wrap(X, d, n);
    ColMajorMatrix<float> xC_small;
    stlq::ComputeXcSmall(pre, Xm, nullptr, &xC_small);
    std::vector<std::uint32_t> cluster;
    ColMajorMatrix<stlq::Code> B_small;
    stlq::BeamSearchPrefixLSLargeRoot(Xm, pre, xC_small, std::max(1, beam), &cluster, &B_small, nullptr);
    ColMajorMatrix<float> a;
    stlq::SolveLeastSquaresAllLargeRoot(pre, Xm, xC_small, cluster, B_small, &a);
    std::vector<float> xn, cost_beam, cost;
    stlq::ComputeXNorm2(Xm, &xn);
    stlq::ComputeCostsLargeRoot(pre, Xm, xC_small, cluster, B_small, a, xn, &cost_beam);
    if (use_abs) {
        stlq::DynamicIcmWithIlsAbsNoNormalLargeRoot(Xm, pre, xC_small, icm_iters, ils_iters, perturb_k, seed, cluster,
                                                    &B_small, &a, &xn, &cost, false, sample_id_offset);
    } else {
        stlq::DynamicIcmWithIlsNoAbsNoNormalLargeRoot(Xm, pre, xC_small, icm_iters, ils_iters, perturb_k, seed,
                                                      cluster, &B_small, &a, &xn, &cost, false, sample_id_offset);
    }
    std::memcpy(cluster_out, cluster.data(), sizeof(std::uint32_t) * n);
    if (m > 1) std::memcpy(B_small_out, B_small.data.data(), B_small.data.size());
    if (a_out) std::memcpy(a_out, a.data.data(), sizeof(float) * a.data.size());
    if (cost_beam_out) std::memcpy(cost_beam_out, cost_beam.data(), sizeof(float) * n);
    if (cost_out && cost.size() == static_cast<std::size_t>(n)) std::memcpy(cost_out, cost.data(), sizeof(float) * n);
    return 0;
}

}  // extern "C"

// The reference's own base-store writer (src/io/base_store.cpp, BaseBasicWriter): Open, one append
// per block (x_kind 0: AppendBlock without raw vectors; 1: AppendBlockRawU8; 2: AppendBlockRawF32),
// Close.  Block b has block_n[b] vectors starting at global id block_start[b]; the arrays hold the
// blocks one after another (cluster ids, (m-1) x n codes, m x n coefficients, raw vectors).
#include "stlq/io/base_store.h"

extern "C" int ref_store_write(const char* dir, int d, int m, const int* h_vec, int shard_size, int bucket_size,
                               int bucket_flush_mb, int write_vector_bucket, int write_basic_to_bucket,
                               int raw_bytes_per_vec, int nblocks, const std::int64_t* block_n,
                               const std::uint64_t* block_start, const std::uint32_t* cluster,
                               const std::uint8_t* B_small, const float* a, const std::uint8_t* x_raw, int x_kind,
                               char* err, int errlen) {
    stlq::io::BaseBasicStoreConfig cfg;
    cfg.dir = dir;
    cfg.d = d;
    cfg.m = m;
    cfg.h_vec.assign(h_vec, h_vec + m);
    cfg.shard_size = shard_size;
    cfg.bucket_size = bucket_size;
    cfg.bucket_flush_mb = bucket_flush_mb;
    cfg.write_vector_bucket = write_vector_bucket != 0;
    cfg.write_basic_to_bucket = write_basic_to_bucket != 0;
    cfg.raw_bytes_per_vec = raw_bytes_per_vec;
    stlq::io::BaseBasicWriter w;
    std::string e;
    auto fail = [&] {
        std::strncpy(err, e.c_str(), static_cast<size_t>(errlen) - 1);
        err[errlen - 1] = 0;
        return 1;
    };
    if (!w.Open(cfg, &e)) return fail();
    const int mc = std::max(0, m - 1);
    const int raw = write_vector_bucket ? (raw_bytes_per_vec > 0 ? raw_bytes_per_vec : d) : 0;
    for (int b = 0; b < nblocks; ++b) {
        const int n = static_cast<int>(block_n[b]);
        std::vector<std::uint32_t> cid(cluster, cluster + n);
        ColMajorMatrix<stlq::Code> B(mc, n);
        std::memcpy(B.data.data(), B_small, static_cast<size_t>(mc) * n);
        ColMajorMatrix<float> A(m, n);
        std::memcpy(A.data.data(), a, sizeof(float) * static_cast<size_t>(m) * n);
        bool ok;
        if (x_kind == 1) {
            ok = w.AppendBlockRawU8(block_start[b], cid, B, A, x_raw, raw, &e);
        } else if (x_kind == 2) {
            ok = w.AppendBlockRawF32(block_start[b], cid, B, A, reinterpret_cast<const float*>(x_raw), raw / 4, &e);
        } else {
            ok = w.AppendBlock(block_start[b], cid, B, A, nullptr, &e);
        }
        if (!ok) return fail();
        cluster += n;
        B_small += static_cast<size_t>(mc) * n;
        a += static_cast<size_t>(m) * n;
        if (x_raw) x_raw += static_cast<size_t>(raw) * n;
    }
    if (!w.Close(&e)) return fail();
    return 0;
}

// The reference's vector-file readers (src/io/{bvecs,fvecs,fbin}_reader.cpp): Open, then
// ReadBlockInto(start, count) into dst (d x count column-major).  format 1 bvecs, 2 fvecs, 3 fbin.
// *nread = min(count, n - start) (0 past the end).
#include "stlq/io/bvecs_reader.h"
#include "stlq/io/fbin_reader.h"
#include "stlq/io/fvecs_reader.h"

extern "C" int ref_read_block(const char* path, int format, std::uint64_t start, std::uint32_t count, void* dst,
                              std::size_t dst_bytes, int* d_out, std::uint64_t* n_out, std::int64_t* nread,
                              char* err, int errlen) {
    std::string e;
    auto fail = [&] {
        std::strncpy(err, e.c_str(), static_cast<size_t>(errlen) - 1);
        err[errlen - 1] = 0;
        return 1;
    };
    auto run = [&](auto& r, auto* p) {
        if (!r.Open(path, &e)) return fail();
        *d_out = r.d();
        *n_out = r.n();
        *nread = (count == 0 || start >= r.n()) ? 0 : static_cast<std::int64_t>(std::min<std::uint64_t>(r.n() - start, count));
        if (!r.ReadBlockInto(start, count, p, dst_bytes, &e)) return fail();
        return 0;
    };
    if (format == 1) {
        stlq::io::BvecsReader r;
        return run(r, static_cast<std::uint8_t*>(dst));
    }
    if (format == 2) {
        stlq::io::FvecsReader r;
        return run(r, static_cast<float*>(dst));
    }
    stlq::io::FbinReader r;
    return run(r, static_cast<float*>(dst));
}
