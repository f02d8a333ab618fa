// dq_common.cuh -- shared device helpers for the dyn-quant sm_100a kernels.
//
// Everything here is plain inline PTX or CUDA intrinsics; the kernels are
// compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dq {

// Group size of the INT4 format: one FP16 scale and zero-point per 128
// consecutive input columns of a row (src/quant_format.cuh:10).
constexpr int kGroup = 128;
// Rows per MMA row-block (the M of mma.m16n8k16).
constexpr int kRowBlock = 16;

// ---------------------------------------------------------------------------
// Global loads
// ---------------------------------------------------------------------------

// Streaming 16-byte load of read-only data that is used once (packed weights):
// bypasses L1 allocation.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

// ---------------------------------------------------------------------------
// Tensor-core MMA: D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
// Fragment ownership (lane = 4*g + t):
//   a0 = A[g][2t..2t+1]   a1 = A[g+8][2t..2t+1]   a2 = A[g][2t+8..+9]   a3 = A[g+8][2t+8..+9]
//   b0 = B[2t..2t+1][g]   b1 = B[2t+8..+9][g]
//   d0 = D[g][2t] d1 = D[g][2t+1] d2 = D[g+8][2t] d3 = D[g+8][2t+1]
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// INT4 -> FP16 dequantisation of one 32-bit word of the packed format.
//
// The packed format (src/quant_format.cuh:25-38) stores column 2j in the low
// nibble and column 2j+1 in the high nibble of byte j, so nibble n of a
// little-endian 32-bit word is column n of that word's 8 columns.
//
// (w & 0x000F000F) | 0x6400_6400 is the f16 pair (1024 + q0, 1024 + q4);
// (w & 0x00F000F0) | 0x6400_6400 is (1024 + 16 q1, 1024 + 16 q5).  Removing
// the bias is exact in f16: (1024+q) - 1024 = q and (1024+16q)/16 - 64 = q, both
// single-rounding operations whose exact result is a small integer.
// Output pairs: p04 = (q0,q4), p15 = (q1,q5), p26 = (q2,q6), p37 = (q3,q7).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

struct Deq4 {
    uint32_t p04, p15, p26, p37;
};

__device__ __forceinline__ Deq4 dequant_word(uint32_t w) {
    constexpr uint32_t kMagic = 0x64006400u;     // f16 pair (1024, 1024)
    constexpr uint32_t kSixteenth = 0x2C002C00u; // f16 pair (1/16, 1/16)
    constexpr uint32_t kMinus64 = 0xD400D400u;   // f16 pair (-64, -64)
    const uint32_t w2 = w >> 8;
    Deq4 r;
    r.p04 = hsub2_u32(lop3_and_or(w, 0x000F000Fu, kMagic), kMagic);
    r.p15 = hfma2_u32(lop3_and_or(w, 0x00F000F0u, kMagic), kSixteenth, kMinus64);
    r.p26 = hsub2_u32(lop3_and_or(w2, 0x000F000Fu, kMagic), kMagic);
    r.p37 = hfma2_u32(lop3_and_or(w2, 0x00F000F0u, kMagic), kSixteenth, kMinus64);
    return r;
}

__device__ __forceinline__ uint32_t pack_h2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

__device__ __forceinline__ float h2f_bits(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// ---------------------------------------------------------------------------
// Deterministic block reductions (fixed xor-butterfly + warp-order tree).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// All threads of the block get the same sum.  red must hold >= NW floats and
// is reused (a barrier guards it on entry and exit).
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = (lane < NW) ? red[lane] : 0.f;
    s = warp_sum(s);
    return s;
}

}  // namespace dq

// ---------------------------------------------------------------------------
// Bulk async copies (TMA, non-tensor form) and mbarriers
// ---------------------------------------------------------------------------
namespace dq {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after ~2^31 SM cycles (about a second) and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > (1ll << 31)) return false;
    }
    return true;
}

// Bulk prefetch of global memory into L2 (16-byte aligned address, size a
// multiple of 16); no completion to wait for.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Global -> shared bulk copy completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

}  // namespace dq

namespace dq {

// Biased INT4 -> FP16 dequantisation for the batch-1 kernel: one shift and
// four lop3 per packed word, keeping the f16 exponent bias (removed per group
// in FP32 by the caller):
//   lo0 = (1024 + q0, 1024 + q4)        lo1 = (1024 + q2, 1024 + q6)
//   hi0 = (1024 + 16 q1, 1024 + 16 q5)  hi1 = (1024 + 16 q3, 1024 + 16 q7)
// All values are exact in f16, so the MMA products with x are exact.
struct Biased4 {
    uint32_t lo0, lo1, hi0, hi1;
};

__device__ __forceinline__ Biased4 biased_word(uint32_t w) {
    constexpr uint32_t kMagic = 0x64006400u;
    const uint32_t w8 = w >> 8;
    Biased4 r;
    r.lo0 = lop3_and_or(w, 0x000F000Fu, kMagic);
    r.lo1 = lop3_and_or(w8, 0x000F000Fu, kMagic);
    r.hi0 = lop3_and_or(w, 0x00F000F0u, kMagic);
    r.hi1 = lop3_and_or(w8, 0x00F000F0u, kMagic);
    return r;
}

}  // namespace dq

namespace dq {

// Adds expected transaction bytes to the barrier's current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only), tracked by the
// thread's cp.async group.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Waits until at most N of this thread's cp.async groups are still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Makes the barrier's current phase also wait for this thread's prior
// cp.async copies (pending count +1 now, arrive when they complete).
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue / wait until the preceding kernel's results are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float ldcg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

}  // namespace dq

namespace dq {

// Mixed-precision FP32 arithmetic with an FP16 operand (sm_100 PTX): the f16
// value is widened exactly, then one FP32 operation rounds once.  Same results
// as __half2float followed by the FP32 operation, without the conversion.
__device__ __forceinline__ float add_f16_f32(uint16_t h, float c) {  // h + c
    float d;
    asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
    return d;
}
__device__ __forceinline__ float sub_f16_f32(uint16_t h, float c) {  // h - c
    float d;
    asm("sub.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
    return d;
}
__device__ __forceinline__ float fma_f16_f32(uint16_t a, uint16_t b, float c) {  // a * b + c
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}
__device__ __forceinline__ uint16_t lo16(uint32_t w) { return static_cast<uint16_t>(w & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t w) { return static_cast<uint16_t>(w >> 16); }

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(addr));
    return r;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(addr));
    return r;
}

// Named barriers (ids 1..15) among `threads` threads, a multiple of 32.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The gather's tagged words: one 32-bit access each, so value and tag are
// seen together (morally strong at system scope on both sides).
__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const unsigned int* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u32(unsigned int* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Four 8x8 b16 matrices from shared memory, transposed: lanes 8j .. 8j+7 give
// the 16-byte row addresses of matrix j; register j receives the fragment of
// that matrix's transpose in the mma A/B register layout.
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Four 8x8 b16 matrices from shared memory: lanes 8j .. 8j+7 give the 16-byte
// row addresses of matrix j; lane 4g + t receives in register j the 32-bit word
// t of row g of matrix j.
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Loads of data written by an earlier kernel of the stream (or by other CTAs
// of this one, after a fence): L2, not the incoherent L1.
__device__ __forceinline__ uint32_t ldcg_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldcg_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint16_t ldcg_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

}  // namespace dq
