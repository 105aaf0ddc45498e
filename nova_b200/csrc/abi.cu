// Library identification, thread-local error reporting and tensor-map
// encoding shared by every entry point.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace nova {

static thread_local char g_last_error[512] = "";
static int g_launch_flags = 0;

int launch_flags() { return __atomic_load_n(&g_launch_flags, __ATOMIC_RELAXED); }

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();   // also consumes the error, so it is not reported twice
    if (e != cudaSuccess) return fail(NOVA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return NOVA_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

int make_tmap_u8_rows128(CUtensorMap* tm, const void* base, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(NOVA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
    if (reinterpret_cast<uintptr_t>(base) % 16) return fail(NOVA_ERR_ALIGN, "tensor map base not 16-byte aligned");
    cuuint64_t gdim[2] = {128, rows};
    cuuint64_t gstride[1] = {128};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NOVA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return NOVA_OK;
}

int make_tmap_f16_rows64(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                         uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(NOVA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
    if (reinterpret_cast<uintptr_t>(base) % 16 || row_stride % 8)
        return fail(NOVA_ERR_ALIGN, "tensor map base 16-byte aligned and row stride a multiple of 8");
    cuuint64_t gdim[2] = {cols, rows};
    cuuint64_t gstride[1] = {row_stride * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NOVA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return NOVA_OK;
}

}  // namespace nova

extern "C" const char* nova_version(void) { return "nova_b200 0.1 (sm_100a, abi 1)"; }

extern "C" const char* nova_last_error(void) { return nova::g_last_error; }

extern "C" int nova_abi_sizes(int64_t* out, int n) {
    const int64_t sizes[] = {int64_t(sizeof(nova_attn_int8_args)),    int64_t(sizeof(nova_nf4_args)),
                             int64_t(sizeof(nova_qk_args)),           int64_t(sizeof(nova_prefill_attn_args)),
                             int64_t(sizeof(nova_qk_prefill_args)),   int64_t(sizeof(nova_sample_args)),
                             int64_t(sizeof(nova_tp_allreduce_args))};
    const int count = int(sizeof(sizes) / sizeof(sizes[0]));
    for (int i = 0; i < n && i < count && out; ++i) out[i] = sizes[i];
    return count;
}

extern "C" int nova_set_launch_flags(int flags) {
    if (flags & ~3) return nova::fail(NOVA_ERR_INVALID, "unknown launch flags 0x%x", flags);
    __atomic_store_n(&nova::g_launch_flags, flags, __ATOMIC_RELAXED);
    return NOVA_OK;
}

extern "C" int nova_get_launch_flags(void) { return nova::launch_flags(); }
