/* CPU restatement of the reference's base-encoding hot path: TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may load
 * this library, and only as the checker or the timed CPU baseline -- never on the product path.
 *
 * Pinning: tests/test_oracle_pin.py checks every function below against the reference's own code
 * (oracle/_ref/libstlq_ref.so, compiled from the reference sources by oracle/Makefile) and
 * against the committed golden fixtures in tests/golden/ (bit-exact for codes, xC, G and norms).
 *
 * Layout follows the reference: column-major matrices (types.h:37-55), G(row, col) stored at
 * G[col * H + row] (GAt, linear_algebra.h:17-19).  Codes are widened to uint16 so K up to 65535
 * can be restated (the reference stores uint8, types.h:22-32).
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* xC = C_all^T X in the summation order of the reference's BLAS backend as measured in this image
 * (OpenBLAS 0.3.15, SkylakeX SGEMM kernel): per output one FMA chain over each K-block, K split
 * into blocks of 448 (remainder halved, rounded up to 16), blocks summed in order.  Call site:
 * encoder_encode_base.inc:33-37 -> src/core/blas.cpp:35-56. */
void oracle_gemm_tn(int d, int rows, int n, const float* A, const float* X, float* out);

/* ||x||^2 per column in the order GCC 13 -O3 gives `#pragma omp simd reduction(+:s)` on the
 * x86-64 baseline ISA (cost_utils.cpp:99-109, beam_search.cpp:218-223): 4 lanes over the first
 * 4*floor(d/4) elements, the tail added into lane 0, then ((l0+l1)+l2)+l3. */
void oracle_xnorm2(int d, int n, const float* X, float* out);

/* BuildPrecomp (encoder_precomp.inc:1-53): G = C_all^T C_all (same GEMM order) and invnorm. */
void oracle_precomp(int d, int H, const float* C_all, float* G, float* invnorm);

/* BeamSearchPrefixLS (beam_search.cpp:196-422) with its replace-worst beam, slot order included.
 * xnorm2 is the per-vector ||x||^2 (oracle_xnorm2).  Threads: OpenMP over vectors. */
void oracle_beam_search(int m, const int* h_vec, int H, const float* G, int n, const float* xnorm2,
                        const float* xC, int beam, uint16_t* B);

/* SolveLeastSquaresAll (least_squares.cpp:406-560).  Returns the number of failed solves
 * (coefficients zeroed, as the reference does). */
int oracle_solve_ls_all(int m, const int* h_vec, int H, const float* G, int n, const float* xC,
                        const uint16_t* B, float* a);

/* ComputeCosts / SampleCost (cost_utils.cpp:112-158). */
void oracle_costs(int m, const int* h_vec, int H, const float* G, int n, const float* xC,
                  const uint16_t* B, const float* a, const float* xnorm2, float* cost);

/* Sum over vectors of MeanMseFromPrecomp's clamped per-vector error in double
 * (src/linkage/linkage_tools.cpp:170-219); divide by n for the reference's mean. */
double oracle_sse(int d, int m, const int* h_vec, int H, const float* G, int n, const float* X,
                  const float* xC, const uint16_t* B, const float* a);

/* The ICM layer orders the reference draws: std::mt19937(seed) shared by every RunIcm call,
 * order reset to iota at each call and std::shuffle'd once per ICM iteration
 * (icm.cpp:119-122,239-243,890-895,974-975).  Writes (ils_iters+1)*icm_iters*m ints. */
void oracle_icm_orders(int m, int icm_iters, int ils_iters, uint32_t seed, int* orders);

/* DynamicIcmWithIls{Abs,NoAbs}NoNormal (icm.cpp:89-344 RunIcm, 872-1003 ILS).  B is in/out,
 * a and cost are outputs; xnorm2 as from oracle_xnorm2. */
void oracle_icm(int m, const int* h_vec, int H, const float* G, const float* invnorm, int n,
                const float* xC, const float* xnorm2, int icm_iters, int ils_iters, int perturb_k,
                int use_abs, uint32_t seed, uint64_t sample_id_offset, uint16_t* B, float* a, float* cost);

#ifdef __cplusplus
}
#endif
