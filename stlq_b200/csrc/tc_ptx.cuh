// Thin wrappers over the sm_100a PTX used by the tensor-core GEMM: mbarriers, TMA tile loads,
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and their ordering fences.
#pragma once

#include <cstdint>

#include "types.h"

namespace stlq_b200 {
namespace tc {

__device__ __forceinline__ uint32_t SmemAddr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void MbarInit(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void FenceBarrierInit() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void MbarArriveExpectTx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(SmemAddr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool MbarTryWait(uint64_t* bar, uint32_t parity) {
    uint32_t ok = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(SmemAddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t GlobalTimerNs() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the barrier phase with a wall-clock limit.  Returns false (after raising *err) when the
// limit passes, so a kernel can release its resources and return instead of hanging.  With
// abort_on_err it also gives up as soon as another CTA has raised *err; waits for the kernel's own
// copies in flight pass false, so that the CTA never exits while a copy still writes its memory.
__device__ __forceinline__ bool MbarWait(uint64_t* bar, uint32_t parity, unsigned int* err, uint64_t limit_ns,
                                         bool abort_on_err = true) {
    if (MbarTryWait(bar, parity)) return true;
    const uint64_t t0 = GlobalTimerNs();
    while (!MbarTryWait(bar, parity)) {
        if ((abort_on_err && (*reinterpret_cast<volatile unsigned int*>(err) & kErrWaitTimeout)) ||
            GlobalTimerNs() - t0 > limit_ns) {
            atomicOr(err, static_cast<unsigned int>(kErrWaitTimeout));
            return false;
        }
    }
    return true;
}

// 2-D TMA tile load into shared memory, completing on `bar` (byte count set by expect_tx).
__device__ __forceinline__ void TmaLoad2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            SmemAddr(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(SmemAddr(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle:
// rows of 128 bytes, 8-row core groups 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t SmemDescSw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
    d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused with this swizzle)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;                  // descriptor version
    d |= static_cast<uint64_t>(2) << 61;                  // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor: kind::tf32, f32 accumulator, A and B K-major, M x N tile.
__host__ __device__ constexpr uint32_t InstrDescTf32(int M, int N) {
    return (1u << 4)                                  // D format: f32
           | (2u << 7)                                // A format: tf32
           | (2u << 10)                               // B format: tf32
           | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void UmmaTf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}

// Arrives on `bar` once every previously issued tcgen05.mma of this thread has completed.
__device__ __forceinline__ void UmmaCommit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(SmemAddr(bar))
                 : "memory");
}

__device__ __forceinline__ void TmemAlloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(SmemAddr(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void TmemDealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void FenceBeforeSync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void FenceAfterSync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane (32x32b shape, 32 repetitions).
__device__ __forceinline__ void TmemLoad32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace stlq_b200
