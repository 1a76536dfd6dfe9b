/* stlq_b200: B200-native (sm_100a) base-encoding hot path of STLQ behind a C ABI.
 *
 * One encoder handle holds one frozen codebook set on one GPU.  All matrices use the reference's
 * column-major layout (include/stlq/common/types.h:37-55 in the reference): a d x n matrix is n
 * columns of d contiguous floats, i.e. vector j starts at X + j*d.  Codes are m x n uint8 (the
 * reference's FullCode, types.h:22-32): vector j's codes start at B + j*m.  Coefficients are
 * m x n floats in the same layout.
 *
 * Errors: every entry point returns 0 on success or a nonzero STLQ_B200_E* code; the message is
 * available from stlq_b200_last_error() on the calling thread.  Nothing throws across the ABI.
 * Thread safety: a handle may be used by one host thread at a time; distinct handles are
 * independent (one per GPU / per host thread, like the reference's thread_local CUDA sessions).
 */
#ifndef STLQ_B200_H_
#define STLQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct stlq_b200_encoder stlq_b200_encoder;

enum {
    STLQ_B200_OK = 0,
    STLQ_B200_EINVAL = 1,   /* bad argument (null pointer, size out of range, unsupported shape) */
    STLQ_B200_ECUDA = 2,    /* CUDA runtime error */
    STLQ_B200_ENOMEM = 3,   /* device allocation failed */
    STLQ_B200_EDEVICE = 4   /* a kernel reported an internal error (bounded wait expired, ...) */
};

/* How xC = C_all^T X is computed.
 *   STLQ_B200_GEMM_EXACT  FP32 FMA chains in the order of the reference's CPU BLAS backend
 *                         (OpenBLAS SkylakeX SGEMM: one chain per 448-deep K block, blocks summed);
 *                         xC and therefore the codes are bit-identical to the reference's.
 *   STLQ_B200_GEMM_STRICT tcgen05 tensor cores, 3xTF32 split, with error bounds carried through
 *                         the beam and the refinement: every xC entry a decision or an output
 *                         depends on is recomputed in the CPU BLAS's order, so the results are
 *                         bit-identical to EXACT's (a tensor-core entry outside its bound is
 *                         reported as an error, never used).
 *   STLQ_B200_GEMM_FAST   tcgen05 tensor cores, 1xTF32 (the reference's TF32 fast mode). */
enum {
    STLQ_B200_GEMM_EXACT = 0,
    STLQ_B200_GEMM_STRICT = 1,
    STLQ_B200_GEMM_FAST = 2
};

/* Input element types for X. */
enum { STLQ_B200_F32 = 0, STLQ_B200_U8 = 1 };

/* Limits of this build. */
#define STLQ_B200_MAX_M 16      /* codebooks (layers) */
#define STLQ_B200_MAX_K 256     /* codewords per codebook with uint8 codes */
#define STLQ_B200_MAX_K_WIDE 1024 /* codewords per codebook with uint16 codes (the _u16 entry points) */
#define STLQ_B200_MAX_BEAM 32   /* beam width */
#define STLQ_B200_MAX_ROOT 65536 /* root codewords of a large-root encoder */

/* Message for the last failed call on this host thread ("" if none). */
const char* stlq_b200_last_error(void);

/* Version string of the library ("stlq_b200 <semver> sm_100a"). */
const char* stlq_b200_version(void);

/* Create an encoder on CUDA device `device`.
 * Replaces BuildPrecomp (reference: src/quantizer/encoder_precomp.inc:1-53) plus the device
 * uploads of FullIcmCudaSession::EnsurePrecomp (src/quantizer/icm_cuda_kernels.inc:2100-2150).
 *   C_all   d x H column-major (H = sum of h_vec), the reference's Precomp::C_all.
 *   G       optional H x H column-major Gram matrix (the reference's Precomp::G); when NULL it is
 *           computed on the device as C_all^T C_all in the order selected by gemm_mode.
 *   invnorm optional H floats (Precomp::invnorm_flat); computed when NULL.
 * h_vec[l] in [1, 1024], m in [1, 16], d >= 1.  With every h_vec[l] <= 256 codes are uint8 (the
 * reference's FullCode) and the uint8 entry points apply; a codebook above 256 codewords makes them
 * uint16 (the _u16 entry points, which the reference has no counterpart for: its codes are uint8;
 * the results follow the reference's algorithm with wider codes), limited to beam x max(h_vec) <=
 * 16384. */
int stlq_b200_create(int device, int d, int m, const int* h_vec, const float* C_all, const float* G,
                     const float* invnorm, int gemm_mode, stlq_b200_encoder** out);

int stlq_b200_destroy(stlq_b200_encoder* enc);

/* Encode n vectors held in HOST memory: the whole EncodeBase stage
 * (src/quantizer/encoder_encode_base.inc:1-106): xC GEMM, BeamSearchPrefixLS, SolveLeastSquaresAll,
 * beam MSE, DynamicIcmWithIls{Abs,NoAbs}NoNormal, final MSE.  Host<->device copies are staged
 * through pinned buffers in slices and overlapped with compute.
 *   X            d x n, element type x_dtype (STLQ_B200_F32 or STLQ_B200_U8).
 *   B_out        m x n uint8 codes.          a_out    m x n LS coefficients (may be NULL).
 *   cost_out     n floats, ICM cost (SampleCost) per vector (may be NULL).
 *   sse_out      2 doubles (may be NULL): sum over vectors of the clamped squared error after
 *                the beam and after ICM/ILS (MeanMseFromPrecomp x n, linkage_tools.cpp:170-219).
 *   sample_id_offset  global id of vector 0 (ILS perturbation stream, icm.cpp:950-960). */
int stlq_b200_encode_base(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                          int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                          uint8_t* B_out, float* a_out, float* cost_out, double* sse_out);

/* stlq_b200_encode_base with uint16 codes (B_out m x n), for codebooks above 256 codewords. */
int stlq_b200_encode_base_u16(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                              int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                              uint16_t* B_out, float* a_out, float* cost_out, double* sse_out);

/* Same stage on DEVICE buffers (all pointers on the encoder's device), enqueued on `stream`
 * (a cudaStream_t; NULL = the legacy default stream).  Asynchronous: returns after enqueueing.
 * sse_out_dev: 2 doubles on the device (may be NULL). */
int stlq_b200_encode_base_device(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, int beam,
                                 int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                 uint64_t sample_id_offset, uint8_t* B_dev, float* a_dev, float* cost_dev,
                                 double* sse_out_dev, void* stream);
int stlq_b200_encode_base_device_u16(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, int beam,
                                     int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                     uint64_t sample_id_offset, uint16_t* B_dev, float* a_dev, float* cost_dev,
                                     double* sse_out_dev, void* stream);

/* ---- Stage-level entry points (device buffers, asynchronous on `stream`) ---- */

/* xC = C_all^T X  (H x n).  Replaces the Gemm call of EncodeBase (encoder_encode_base.inc:33-37)
 * and StreamKernelProvider::GemmDevice (include/stlq/core/kernel_provider.h:75-100). */
int stlq_b200_xc_gemm(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* xC_dev,
                      void* stream);

/* ||x||^2 per vector (ComputeXNorm2, src/quantizer/cost_utils.cpp:88-110), same float order. */
int stlq_b200_xnorm2(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* xnorm2_dev,
                     void* stream);

/* BeamSearchPrefixLS (src/quantizer/beam_search.cpp:196-422; declared in
 * include/stlq/quantizer/beam_search.h:18-22): m x n codes from xC and ||x||^2. */
int stlq_b200_beam_search(stlq_b200_encoder* enc, const float* xnorm2_dev, const float* xC_dev, int64_t n,
                          int beam, uint8_t* B_dev, void* stream);

/* SolveLeastSquaresAll (src/quantizer/least_squares.cpp:406-560): m x n coefficients. */
int stlq_b200_solve_ls(stlq_b200_encoder* enc, const float* xC_dev, const uint8_t* B_dev, int64_t n,
                       float* a_dev, void* stream);

/* DynamicIcmWithIls{Abs,NoAbs}NoNormalCudaDeviceXc (include/stlq/quantizer/icm_cuda.h:70-101;
 * CPU semantics icm.cpp:89-344, 872-1003).  B_dev is in/out; a_dev and cost_dev are outputs.
 * The ICM layer orders are drawn on the host with std::mt19937(seed) + std::shuffle, exactly
 * as the reference does. */
int stlq_b200_icm(stlq_b200_encoder* enc, const float* xC_dev, const float* xnorm2_dev, int64_t n, int icm_iters,
                  int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                  uint8_t* B_dev, float* a_dev, float* cost_dev, void* stream);

/* Sum over vectors of MeanMseFromPrecomp's clamped per-vector error, in double, added into
 * *sse_dev (src/linkage/linkage_tools.cpp:170-219). */
int stlq_b200_sse(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, const float* xC_dev,
                  const uint8_t* B_dev, const float* a_dev, int64_t n, double* sse_dev, void* stream);

/* Beam search like stlq_b200_beam_search, but the call allocates no device memory: no cudaMalloc,
 * cudaFree or allocating library routine.  It exists for callers that cannot allocate while they
 * encode, for example a service or framework whose caching allocator or memory pool owns all
 * free device memory (an allocation would fail, or fragment and stall that pool), or a
 * latency-critical path where an allocation's implicit device synchronisation is unacceptable.
 * It has no counterpart in the reference.
 *
 * The beam search hands vectors whose exact errors tie at a selection boundary between its two
 * kernels through a scratch list; here that list is a static device array sized for
 * STLQ_B200_NOALLOC_MAX_VECTORS vectors (4 MiB, held by every GPU that loads the library until
 * the process exits).  n above that limit is rejected with STLQ_B200_EINVAL; split such calls.
 * The encoder handle (which allocates its codebook tables) and the inputs and outputs are the
 * caller's, created beforehand.
 * The first call on each device sets up that device (it looks up the array's device address and
 * loads every beam kernel variant, for any encoder shape); make that first call before any stream
 * capture.  The address is kept for the process: do not reset the device (cudaDeviceReset) while
 * the library is loaded.  Arguments are checked as stlq_b200_beam_search checks them (the same
 * STLQ_B200_EINVAL results), plus the size limit.  All calls share the
 * one array: each clears it before use, and calls whose work overlaps on the GPU (concurrent
 * streams, several host threads) race and must not be issued. */
#define STLQ_B200_NOALLOC_MAX_VECTORS (1 << 20)
int stlq_b200_beam_search_noalloc(stlq_b200_encoder* enc, const float* xnorm2_dev, const float* xC_dev, int64_t n,
                                  int beam, uint8_t* B_dev, void* stream);

/* Input rotation X <- R X (ApplyRotationInPlace, src/pipeline/app_utils.cpp:203-227; the OPQ
 * rotation of the train result, applied to the base set before encoding,
 * stlq_non_large_pipeline_flow.cpp:58).  R: d x d column-major; NULL or the exact identity turns it
 * off (the reference skips the product then, IsIdentityRotation :186-201).  When set, the
 * whole-stage entry points (stlq_b200_encode_base*, the large-root ones included) rotate each
 * slice on the device with the reference's GEMM order before encoding; the stage entry points take
 * already rotated vectors, as the reference's stage functions do. */
int stlq_b200_set_rotation(stlq_b200_encoder* enc, const float* R);

/* out_dev (d x n floats) = R X_dev (or X_dev converted to float when no rotation is set), the
 * reference's ConvertU8ToF32AndRotate (include/stlq/core/kernel_provider.h:48-54). */
int stlq_b200_rotate(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* out_dev, void* stream);

/* ---- Large-root encoder (the large pipeline's basic encode) ----
 * Replaces BuildPrecompLargeRoot (src/quantizer/precomp_large_root.cpp:27-160),
 * BeamSearchPrefixLSLargeRoot (src/quantizer/beam_search.cpp:579-992, declared in
 * include/stlq/quantizer/beam_search.h:26-32), SolveLeastSquaresAllLargeRoot
 * (least_squares.cpp:567-745), ComputeCostsLargeRoot (cost_utils.cpp:160-235) and
 * DynamicIcmWithIls{Abs,NoAbs}NoNormalLargeRoot (icm.cpp:347-870, 1005-1210), as the large
 * pipeline runs them per block (src/quantizer/encode_base_streaming.cpp:1040-1300).
 * Codebook 0 of C_all is the root (cluster ids): h_vec[0] in [1, 65536], the other codebooks
 * in [1, 256] (uint8 codes, as the reference's B_small).  Like PrecompLargeRoot the handle holds
 * no root-root Gram block: only the G0S and G_small columns ((H - h0) x H floats) and the root
 * norms.  The large-root arithmetic differs from the regular encoder's in the root codewords'
 * norms and the root dot products (the reference's SIMD-order loops), the beam's triangular
 * solves (multiplied by 1/R_ii) and the cost's summation order; the codes equal the reference's
 * large-root codes.  With h_vec[0] <= 256 the uint8 stage entry points above also accept such a
 * handle (codes as m x n, root first). */
int stlq_b200_create_large_root(int device, int d, int m, const int* h_vec, const float* C_all, int gemm_mode,
                                stlq_b200_encoder** out);

/* Host buffers.  cluster_out: n root codes; B_small_out: (m-1) x n codes of layers 1..m-1;
 * a_out: m x n coefficients; cost_out: n final costs (may be NULL); cost_sums_out: 2 doubles
 * (may be NULL): the sums over vectors of the beam-stage and the final SampleCostLargeRoot, whose
 * means the large pipeline reports as beam and final MSE. */
int stlq_b200_encode_base_large_root(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam,
                                     int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                     uint64_t sample_id_offset, uint32_t* cluster_out, uint8_t* B_small_out,
                                     float* a_out, float* cost_out, double* cost_sums_out);

/* Device buffers, asynchronous on `stream` (cost_sums_dev: 2 doubles on the device or NULL). */
int stlq_b200_encode_base_large_root_device(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n,
                                            int beam, int icm_iters, int ils_iters, int perturb_k, int use_abs,
                                            uint32_t seed, uint64_t sample_id_offset, uint32_t* cluster_dev,
                                            uint8_t* B_small_dev, float* a_dev, float* cost_dev,
                                            double* cost_sums_dev, void* stream);

/* ---- Multi-GPU encode (one process, several GPUs of one node) ----
 * The reference encodes the base set on one device (RunStlq -> EncodeBase, src/stlq.cpp:48-55;
 * EncodeBase is declared in include/stlq/quantizer/encoder.h:66-74).  Base vectors are
 * independent, so a sharded encoder holds one encoder per device and splits the vectors into
 * contiguous shards (vector j of n on device floor-split: the first n % N shards one larger), one
 * host thread per device, each shard with its global sample ids (ILS is keyed by them,
 * icm.cpp:950-960): the codes, coefficients and costs equal one device's, bit for bit.  Only two
 * things cross GPUs: the codebook set (C_all, and G / invnorm when given), uploaded to devices[0]
 * and replicated by one NCCL broadcast, and the per-shard MSE sums, combined by one NCCL reduce
 * onto devices[0].  NCCL (libnccl.so.2) is loaded at run time by the first call; without it these
 * calls fail with STLQ_B200_ECUDA.  Collective waits are bounded (the communicators are aborted
 * and STLQ_B200_EDEVICE returned on expiry).  devices: n_devices distinct ordinals.  The other
 * arguments are stlq_b200_create's / stlq_b200_create_large_root's. */
typedef struct stlq_b200_sharded stlq_b200_sharded;
int stlq_b200_sharded_create(int n_devices, const int* devices, int d, int m, const int* h_vec, const float* C_all,
                             const float* G, const float* invnorm, int gemm_mode, stlq_b200_sharded** out);
int stlq_b200_sharded_create_large_root(int n_devices, const int* devices, int d, int m, const int* h_vec,
                                        const float* C_all, int gemm_mode, stlq_b200_sharded** out);
int stlq_b200_sharded_destroy(stlq_b200_sharded* sh);
/* The per-device encoder i (owned by the sharded handle), e.g. for stlq_b200_set_rotation. */
int stlq_b200_sharded_encoder(stlq_b200_sharded* sh, int i, stlq_b200_encoder** out);
/* stlq_b200_encode_base / _u16 / stlq_b200_encode_base_large_root over all devices at once (host
 * buffers, same arguments and outputs; sse_out / cost_sums_out: the NCCL-reduced sums). */
int stlq_b200_encode_sharded(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                             int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                             uint8_t* B_out, float* a_out, float* cost_out, double* sse_out);
int stlq_b200_encode_sharded_u16(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam,
                                 int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                 uint64_t sample_id_offset, uint16_t* B_out, float* a_out, float* cost_out,
                                 double* sse_out);
int stlq_b200_encode_sharded_large_root(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam,
                                        int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                        uint64_t sample_id_offset, uint32_t* cluster_out, uint8_t* B_small_out,
                                        float* a_out, float* cost_out, double* cost_sums_out);

/* ---- Base-store writer fed from device buffers ----
 * Writes the reference's basic base store (BaseBasicWriter, include/stlq/io/base_store.h:29-97;
 * src/io/base_store.cpp): meta.json, meta.bin, cluster_id.u32, codes_shard_NNNN.bin,
 * coeffs_shard_NNNN.bin and bucket_NNNN.bin, byte for byte as the reference writes them for the
 * same blocks (Open, then AppendBlock / AppendBlockRawU8 / AppendBlockRawF32 per block, Close).
 * The parameters are BaseBasicStoreConfig's; raw_bytes_per_vec 0 means d (uint8 vectors), d * 4 for
 * float vectors.  device >= 0: blocks may sit in device memory (outputs of the encode entry points);
 * an append enqueues their copy into a pinned staging slot on the store's own copy stream, after the
 * work already enqueued on `stream`, and returns; one writer thread writes blocks in append order
 * as their copies complete (an append waits only when three blocks are in flight).  device < 0:
 * host buffers only, no CUDA call.  max_block: the largest block (vectors) an append may pass.
 * One host thread per store.  Errors of the writer thread are returned by the next call. */
typedef struct stlq_b200_store stlq_b200_store;
int stlq_b200_store_open(const char* dir, int d, int m, const int* h_vec, int shard_size, int bucket_size,
                         int bucket_flush_mb, int write_vector_bucket, int write_basic_to_bucket, int raw_bytes_per_vec,
                         int device, int64_t max_block, stlq_b200_store** out);
/* One block of n vectors with global ids start_id..: cluster (n root codes), B_small ((m-1) x n
 * codes), a (m x n coefficients), x_raw (vector i at x_raw + i * ld_x_bytes; only read with
 * write_vector_bucket).  Host or device pointers (device stores).  Device stores: work enqueued on
 * `stream` after the append waits for the block's staging copy, so the caller may reuse or free
 * its buffers in that stream's order. */
int stlq_b200_store_append(stlq_b200_store* st, uint64_t start_id, int64_t n, const uint32_t* cluster,
                           const uint8_t* B_small, const float* a, const void* x_raw, int64_t ld_x_bytes,
                           void* stream);
/* Writes everything appended so far (BaseBasicWriter::Flush). */
int stlq_b200_store_flush(stlq_b200_store* st);
/* Flushes, closes the files and frees the store (BaseBasicWriter::Close); returns the first error. */
int stlq_b200_store_close(stlq_b200_store* st);

/* ---- Vector-file reader (input side of the large pipeline's block loop) ----
 * The reference's BvecsReader / FvecsReader / FbinReader (include/stlq/io/{bvecs,fvecs,fbin}_reader.h)
 * and its block prefetcher (AsyncBasicBlockPrefetcher, src/quantizer/encode_base_streaming.cpp:72-230).
 * format: STLQ_B200_FMT_AUTO takes it from the suffix (.bvecs/.siftbin, .fbin, .fvecs), as the
 * reference's dataset reader factory does.  A prefetch thread reads blocks of `block` vectors of
 * [begin, end) (end 0: the file's n) into `depth` (>= 2) pinned slots with io_threads parallel
 * reads.  device >= 0: next() copies a block to device memory on `stream` and strips the records'
 * dimension prefixes there; device < 0: host-only, no CUDA call.  Every record's prefix is checked
 * against d (a mismatch of a device block is returned by a later call).  Blocks are row-major
 * count x d (the reference's column-major d x count), uint8 for .bvecs, float32 otherwise. */
enum { STLQ_B200_FMT_AUTO = 0, STLQ_B200_FMT_BVECS = 1, STLQ_B200_FMT_FVECS = 2, STLQ_B200_FMT_FBIN = 3 };
typedef struct stlq_b200_reader stlq_b200_reader;
int stlq_b200_reader_open(const char* path, int format, uint64_t begin, uint64_t end, int64_t block, int depth,
                          int io_threads, int device, stlq_b200_reader** out);
/* d, n (vectors in the file) and the element type (STLQ_B200_U8 or STLQ_B200_F32). */
int stlq_b200_reader_info(const stlq_b200_reader* rd, int* d, uint64_t* n, int* x_dtype);
/* The next block, in file order: *start = its first vector, *count = its size (0 once the range is
 * done).  dst: device memory (device readers) or host memory of at least block * d * element bytes;
 * asynchronous on `stream` for device readers. */
int stlq_b200_reader_next(stlq_b200_reader* rd, void* dst, size_t dst_bytes, void* stream, uint64_t* start,
                          int64_t* count);
/* ReadBlockInto: vectors start..start+count-1 (clipped to n) into host memory, synchronously. */
int stlq_b200_reader_read(stlq_b200_reader* rd, uint64_t start, int64_t count, void* dst, size_t dst_bytes,
                          int64_t* nread);
int stlq_b200_reader_close(stlq_b200_reader* rd);

/* The large pipeline's block loop (src/quantizer/encode_base_streaming.cpp:640-1310, basic encode):
 * every block of the reader's range is copied to the device, encoded by the large-root encoder
 * `enc` (sample ids = global vector ids) and, when `st` is not NULL, appended to the store, the
 * next block's copy and the store's copies overlapping the encode.  The reader must be a device
 * reader on the encoder's device; the store a device store there with d and m of the encoder and
 * max_block >= the reader's block.  mse_sums_out (2 doubles, may be NULL): sum over blocks of
 * float(mean beam cost of the block) x block size, and the same for the final cost (the reference's
 * mse_sum_beam / mse_sum_final, 1303-1304).  vectors_out: vectors encoded.  Returns when every
 * block is encoded and handed to the store (the store's files are complete after its close). */
int stlq_b200_encode_file_large_root(stlq_b200_encoder* enc, stlq_b200_reader* rd, stlq_b200_store* st, int beam,
                                     int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                     double* mse_sums_out, int64_t* vectors_out);

/* ---- Kernel-provider primitives ----
 * The device operations behind StreamKernelProvider (include/stlq/core/kernel_provider.h:28-221,
 * the reference's GPU backend seam; its CUDA implementation is src/core/kernel_provider_cuda_stream*
 * over cuBLAS).  The C++ provider class stlq::b200::B200StreamKernels
 * (stlq_b200/adapter/stlq_b200_kernels.h) implements that interface on them.  All pointers are on
 * the handle's device; work is enqueued on `stream` (NULL: the legacy default stream). */
typedef struct stlq_b200_kernels stlq_b200_kernels;
int stlq_b200_kernels_create(int device, stlq_b200_kernels** out);
int stlq_b200_kernels_destroy(stlq_b200_kernels* k);

/* C = alpha op(A) op(B) + beta C, column-major, BLAS sgemm semantics (replaces stlq::GemmRaw /
 * cblas_sgemm, src/core/blas.cpp:61-80, and the providers' Gemm*).  The result is bit-identical to
 * the reference's single-thread OpenBLAS 0.3.15 sgemm: K split into blocks of 448 (a remainder in
 * (448, 896) halved and rounded up to 16), one FMA chain per block, C = fl(beta C) (0 when beta is 0)
 * and then C = fma(alpha, chain, C) per block in order.  k == 0 or alpha == 0 scales C by beta. */
int stlq_b200_sgemm(stlq_b200_kernels* k, int trans_a, int trans_b, int m, int n, int kdim, float alpha,
                    const float* A, int lda, const float* B, int ldb, float beta, float* C, int ldc, void* stream);

/* out (rows x cols, leading dimension rows) = float(in) for a uint8 tile with leading dimension
 * ld_in (ConvertU8ToF32, ConvertU8ToF32AndRotatePtr's first step). */
int stlq_b200_u8_to_f32(stlq_b200_kernels* k, const uint8_t* in, int ld_in, int rows, int64_t cols, float* out,
                        void* stream);

/* Per column of scores (rows x cols, leading dimension ld): idx = the first row holding the maximum,
 * val = that maximum (NaN never wins; no value above -inf gives row 0, -inf) (ArgmaxColsF32[Device]).
 * idx or val may be NULL. */
int stlq_b200_argmax_cols(stlq_b200_kernels* k, const float* scores, int ld, int rows, int64_t cols, int* idx,
                          float* val, void* stream);

/* Block until all work this encoder enqueued on `stream` has finished; returns
 * STLQ_B200_EDEVICE if a kernel flagged an internal error since the last check. */
int stlq_b200_sync(stlq_b200_encoder* enc, void* stream);

/* Beam-search counters accumulated since the last reset (diagnostics, no counterpart in the
 * reference): out[0] candidates evaluated exactly by the fast kernel, out[1] layers expanded,
 * out[2] vectors, out[3] vectors handed to the slot-replay kernel (exact ties).  Synchronises the
 * device; reset != 0 clears the counters. */
int stlq_b200_beam_stats(stlq_b200_encoder* enc, uint64_t out[4], int reset);

/* Shape queries. */
int stlq_b200_dims(const stlq_b200_encoder* enc, int* d, int* m, int* H);

#ifdef __cplusplus
}
#endif

#endif /* STLQ_B200_H_ */
