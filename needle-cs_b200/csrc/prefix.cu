// Primed-prefix blobs (Engine.ExportPrimedPrefix / ImportPrimedPrefix,
// src/Needle/Engine.cs:398-464): a slot's first `len` KV positions moved
// between the paged cache and the reference's blob layout
//   [int32 len] then per layer:
//     keys   int8 [len][heads * 64]   (position-major, the cache rows)
//     values int8 [len][heads * 64]
//     key scales   fp32 [len][heads]
//     value scales fp32 [len][heads]
// The synthetic decoders keep no recurrent engine state, so the state
// section of the reference's blob is empty.  Block per (layer, position),
// thread per (head, dim); dim 0 also moves the two scales.
#include "common.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {

__global__ void __launch_bounds__(1024) prefix_move_kernel(bool to_blob, int layers, int heads, int len,
                                                           const int32_t *__restrict__ pages, uint8_t *pool,
                                                           long long page_bytes, int num_pages, uint8_t *blob,
                                                           int *status) {
    pdl_enter();
    const int layer = blockIdx.x / len, pos = blockIdx.x - layer * len;
    const int h = threadIdx.x >> 6, d = threadIdx.x & 63;
    if (h >= heads) return;
    const int page = pages[pos / kPagePositions], j = pos % kPagePositions;
    if (page < 0 || page >= num_pages) {
        if (d == 0 && status) atomicOr(status, kStatusBadPage);
        return;
    }
    uint8_t *blk = pool + (size_t)page * page_bytes + kv_block_offset(layer, h, heads);
    const size_t row = (size_t)heads * kHeadDim;
    uint8_t *base = blob + 4 + (size_t)layer * len * (2 * row + 8 * heads);
    uint8_t *kq = base + (size_t)pos * row + h * kHeadDim + d;
    uint8_t *vq = kq + (size_t)len * row;
    float *ks = reinterpret_cast<float *>(base + 2 * (size_t)len * row) + (size_t)pos * heads + h;
    float *vs = ks + (size_t)len * heads;
    float *kso = reinterpret_cast<float *>(blk + kKScaleOffset) + k_scale_index(j);
    float *vso = reinterpret_cast<float *>(blk + kVScaleOffset) + v_scale_index(j);
    if (to_blob) {
        *kq = blk[k_byte(j, d)];
        *vq = blk[v_byte(j, d)];
        if (d == 0) *ks = *kso, *vs = *vso;
    } else {
        blk[k_byte(j, d)] = *kq;
        blk[v_byte(j, d)] = *vq;
        if (d == 0) *kso = *ks, *vso = *vs;
    }
}

size_t prefix_blob_bytes(int layers, int heads, int len) {
    return 4 + (size_t)layers * len * (2 * (size_t)heads * kHeadDim + 8 * (size_t)heads);
}

int launch_prefix_move(bool to_blob, int layers, int heads, int len, const int32_t *pages, uint8_t *pool,
                       long long page_bytes, int num_pages, uint8_t *blob, int *status, cudaStream_t stream) {
    if (len == 0) return NDL_OK;
    if (heads < 1 || heads > 16) return set_error(NDL_ERR_UNSUPPORTED, "prefix move: %d heads (1..16)", heads);
    const long long blocks = (long long)layers * len;
    if (blocks > 0x7FFFFFFF) return set_error(NDL_ERR_INVALID_ARG, "prefix move: too many positions");
    launch_kernel(prefix_move_kernel, dim3((unsigned)blocks), dim3(heads * kHeadDim), 0, stream, to_blob, layers,
                  heads, len, pages, pool, page_bytes, num_pages, blob, status);
    return check_launch("prefix_move");
}

}  // namespace ndl
