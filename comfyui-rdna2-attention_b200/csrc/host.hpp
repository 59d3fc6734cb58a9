// Host-side helpers shared by the C-ABI entry points: status codes with a thread-local message,
// CUDA error mapping, and TMA tensor-map encoding through the driver entry point (no -lcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "rdna2_b200.h"

namespace b2 {

// Records a message for b2_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps the pending CUDA launch error (if any) to B2_ERR_CUDA.
inline int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return B2_OK;
}

// cuTensorMapEncodeTiled from the driver, resolved once.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// 2D map over a row-major matrix [rows, cols] with `ld_bytes` between rows, boxes of
// box_cols x box_rows elements, 128-byte swizzle (box_cols * elem_bytes must be 128), zero fill.
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                uint64_t rows, uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// 4D map over [d3, d2, d1, d0] (d0 innermost, contiguous) with byte strides s1, s2, s3.
int make_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, const uint64_t dims[4],
                const uint64_t strides_bytes[3], const uint32_t box[4],
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Raises the dynamic shared-memory limit of a kernel once.
template <class K>
inline int set_smem(K kernel, int bytes) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaFuncSetAttribute(%d bytes): %s", bytes, cudaGetErrorString(e));
    return B2_OK;
}

// Per-translation-unit device status words, read and cleared by b2_device_status().
unsigned int read_status_gemm();
unsigned int read_status_attention();
unsigned int read_status_gemm_w4a8();

}  // namespace b2
