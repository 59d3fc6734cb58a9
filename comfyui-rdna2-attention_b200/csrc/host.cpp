// Library-wide C-ABI entry points (version, last error, device status) and the host helpers of host.hpp.
#include "host.hpp"

#include <mutex>
#include <string.h>

namespace b2 {

static thread_local char g_message[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_message, sizeof(g_message), fmt, ap);
    va_end(ap);
    return code;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                uint64_t rows, uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(B2_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (!aligned16(base) || (ld_bytes & 15)) return fail(B2_ERR_UNSUPPORTED, "TMA needs 16-byte aligned base and row pitch");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled(2d) failed with %d", (int)r);
    (void)elem_bytes;
    return B2_OK;
}

int make_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, const uint64_t dims[4],
                const uint64_t strides_bytes[3], const uint32_t box[4], CUtensorMapSwizzle swizzle) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(B2_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (!aligned16(base)) return fail(B2_ERR_UNSUPPORTED, "TMA needs a 16-byte aligned base");
    for (int i = 0; i < 3; ++i)
        if (strides_bytes[i] & 15) return fail(B2_ERR_UNSUPPORTED, "TMA needs strides that are multiples of 16 bytes");
    cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
    cuuint64_t s[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
    cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, dtype, 4, const_cast<void*>(base), d, s, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled(4d) failed with %d", (int)r);
    (void)elem_bytes;
    return B2_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

}  // namespace b2

extern "C" {

int b2_version(void) { return 100; }

const char* b2_last_error(void) { return b2::g_message; }

int b2_device_status(unsigned int* flags) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return b2::fail(B2_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    unsigned int f = b2::read_status_gemm() | b2::read_status_attention() | b2::read_status_gemm_w4a8();
    if (flags) *flags = f;
    if (f) return b2::fail(B2_ERR_DEVICE, "device status 0x%x: a bounded wait ran out", f);
    return B2_OK;
}

}  // extern "C"
