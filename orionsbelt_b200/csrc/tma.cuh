// tma.cuh -- tensor-map (TMA) loads of one chunk of a [B][T][H][D] 16-bit
// tensor (D = 128) into shared memory in a layout the tcgen05 MMAs read.
//
// A chunk tile holds rows t0 .. t0+63 (tokens) x all D features of one
// (batch, head) (D = 128; the swizzled form also D = 256), in one of two
// layouts:
//
// Core-matrix (no swizzle), one box.  The map describes the tensor as five
// dimensions, innermost first: d%8 (contiguous), t (stride H*D), d/8 (stride
// 8 elements), h (stride D), b (stride T*H*D), with a box of {8, 64, 16, 1, 1}.
// TMA writes the box innermost-first, so element (t, d) lands at
//   (d/8)*1024 + (t/8)*128 + (t%8)*16 + (d%8)*2
// which reads as K-major (rows t, K = d: LBO 1024, SBO 128) or as MN-major
// (MN = d, K = t: LBO 128, SBO 1024).
//
// 128-byte swizzle, two boxes.  The map is the plain four-dimensional view
// {d, h, t, b} with a box of {64, 1, 64, 1}; box j (features 64j .. 64j+63)
// fills 8 KB at offset 8192*j, row t at t*128 with its 16-byte chunks
// permuted by chunk ^= (t % 8).
//
// Tokens past T read as zeros (TMA out-of-bounds fill).  No multicast.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {
namespace tma {

constexpr int ROWS = 64;  // tokens per box

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's cuTensorMapEncodeTiled, looked up once through the runtime
// (the library does not link libcuda directly).
inline EncodeTiled encoder() {
    static EncodeTiled fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

// Host: map of a [B][T][H][D] tensor of 16-bit elements.  Returns 0 or the
// failing CUresult (-1 when the driver entry point is unavailable).
inline int make_chunk_map(CUtensorMap *map, const void *base, bool bf16, uint64_t B, uint64_t T, uint64_t H,
                          uint64_t D, bool swizzle128, uint32_t rows = ROWS) {
    EncodeTiled enc = encoder();
    if (!enc) return -1;
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r;
    if (!swizzle128) {
        const cuuint64_t dims[5] = {8, T, D / 8, H, B};
        const cuuint64_t strides[4] = {H * D * 2, 16, D * 2, T * H * D * 2};
        const cuuint32_t box[5] = {8, ROWS, static_cast<cuuint32_t>(D / 8), 1, 1};
        const cuuint32_t es[5] = {1, 1, 1, 1, 1};
        r = enc(map, dt, 5, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[4] = {D, H, T, B};
        const cuuint64_t strides[3] = {D * 2, H * D * 2, T * H * D * 2};
        const cuuint32_t box[4] = {64, 1, rows, 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        r = enc(map, dt, 4, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    return static_cast<int>(r);
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Core-matrix layout: tokens t0 .. t0+63 of (b, h) into `dst` (16 KB,
// 128-byte aligned); completion counted on `bar` as transaction bytes.
__device__ __forceinline__ void load_chunk(void *dst, const CUtensorMap *map, int t0, int h, int b, uint64_t *bar) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const uint32_t m = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(d),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(t0), "r"(0), "r"(h), "r"(b), "r"(m)
        : "memory");
}

// 128-byte swizzle: features 64j .. 64j+63 (j < nbox = D/64) of the map's
// rows (64 by default) from token t0 into `dst` + box_bytes*j (1024-byte
// aligned; box_bytes = rows * 128).
__device__ __forceinline__ void load_chunk_sw128(void *dst, const CUtensorMap *map, int t0, int h, int b,
                                                 uint64_t *bar, int nbox = 2, uint32_t box_bytes = 8192) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const uint32_t m = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    for (int j = 0; j < nbox; ++j)
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
            "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(d + box_bytes * j),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(64 * j), "r"(h), "r"(t0), "r"(b), "r"(m)
            : "memory");
}

}  // namespace tma
}  // namespace gdn
