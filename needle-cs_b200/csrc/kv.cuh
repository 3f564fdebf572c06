// Paged int8 KV cache layout and the PTX helpers the attention kernels use.
//
// A page holds 64 consecutive positions of one slot for every layer.  Inside
// a page, the block of (layer, head) is one contiguous 8704-byte record of
// two 4352-byte halves:
//     K half: [K int8 64x64][K scale f32 x64]
//     V half: [V scale f32 x64][V int8 64x64]
// so one 16-byte-aligned bulk copy brings either half of 64 positions of one
// head into shared memory.  This replaces the reference's flat per-slot
// arrays [layer][capacity][kvWidth] + scales (src/Needle/Engine.cs:184-187,
// 220-223) with the same per-(position, head) int8 + fp32-scale contents:
//  * K (row = position, col = dim) is an int8 64x64 matrix in m16n8k32
//    A-fragment order (frag_byte): a lane's four A registers of one (16-row
//    tile, 32-col k-step) are one 16-byte chunk and a warp reads 512
//    contiguous bytes; the K scale of position p sits at scale_slot(p), so
//    the lane that owns p's score reads its scale pair as one float2;
//  * V is stored dim-major, 64 positions of one dim in 64 bytes, its four
//    16-byte chunks rotated by (dim >> 1) & 3 so that eight lanes reading
//    chunk c of eight consecutive dims hit eight distinct bank groups; the V
//    scales are in position order.
// The query vector is stored with its dims in k_slot order: a lane's
// m16n8k32 B registers for both k-steps are one 16-byte chunk.
#pragma once

#include <stdint.h>

namespace ndl {

constexpr int kPagePositions = 64;
constexpr int kHeadDim = 64;
constexpr int kKvBlockBytes = 2 * (kPagePositions * kHeadDim + kPagePositions * 4);  // 8704
constexpr int kKvHalfBytes = kKvBlockBytes / 2;                                       // 4352
constexpr int kKScaleOffset = kPagePositions * kHeadDim;                              // 4096
constexpr int kVScaleOffset = kKvHalfBytes;                                           // 4352
constexpr int kVOffset = kVScaleOffset + kPagePositions * 4;                          // 4608

__host__ __device__ __forceinline__ int k_slot(int d) { return ((d & 15) >> 2) * 16 + (d >> 4) * 4 + (d & 3); }

// Byte of element (row, col) of a 64x64 int8 matrix in m16n8k32 A-fragment
// order: [16-row tile][32-col k-step][lane = 4*(row&7) + ((col>>2)&3)]
// [register = (row>>3&1) + 2*(col>>4&1)][col&3].
__host__ __device__ __forceinline__ int frag_byte(int row, int col) {
    return (row >> 4) * 1024 + (col >> 5) * 512 + ((row & 7) * 4 + ((col >> 2) & 3)) * 16 +
           (((row >> 3) & 1) + 2 * ((col >> 4) & 1)) * 4 + (col & 3);
}
// The QK step leaves position p's score with lane 4*(p&7) + (p>>4&3) (half
// p>>3&1); its K scale sits at that lane's float2.
__host__ __device__ __forceinline__ int scale_slot(int p) { return 2 * ((p & 7) * 4 + ((p >> 4) & 3)) + ((p >> 3) & 1); }
__host__ __device__ __forceinline__ int k_byte(int p, int d) { return frag_byte(p, d); }
__host__ __device__ __forceinline__ int k_scale_index(int p) { return scale_slot(p); }
__host__ __device__ __forceinline__ int v_scale_index(int p) { return p; }
__host__ __device__ __forceinline__ int v_byte(int p, int d) {
    return kVOffset + d * 64 + ((((p >> 4) ^ ((d >> 1) & 3)) << 4) | (p & 15));
}

__host__ __device__ __forceinline__ size_t kv_page_bytes(int layers, int heads) {
    return (size_t)layers * heads * kKvBlockBytes;
}
__host__ __device__ __forceinline__ size_t kv_block_offset(int layer, int head, int heads) {
    return ((size_t)layer * heads + head) * kKvBlockBytes;
}

// Device status word bits (written by kernels, read by the host).
constexpr int kStatusTimeout = 1;
constexpr int kStatusBadPage = 2;

#ifdef __CUDACC__
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Non-tensor bulk copy global -> shared, completion counted on `bar`.
// No multicast: every CTA fetches its own bytes.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Non-blocking test: has the phase with this parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// One test of the phase.  While it is incomplete the thread is suspended
// (not spinning) until the phase completes or about kWaitHintNs pass, so
// waiting warps leave the issue slots to the working ones.
constexpr uint32_t kWaitHintNs = 1000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after `limit` tests (each at most about
// kWaitHintNs) and reports false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
#endif

}  // namespace ndl
