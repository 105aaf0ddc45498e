// nova_attn_decode_int8_noalloc: the fused int8-KV decode attention for
// callers that cannot allocate device memory -- an allocator-free runtime, a
// host that hands out only its own arenas, or code running where a
// cudaMalloc would synchronise the device or fail (inside a custom memory
// pool, a signal-free serving loop).  The split partials, per-head arrival
// counters and error word live in one file-scope device array instead of a
// caller-supplied workspace; nothing here calls cudaMalloc, cudaFree or an
// allocating library.
//
// The array is shared by every call in the process on a given device and
// keeps its contents between calls: each call clears the counters and the
// error word (on the caller's stream, before the kernel) and the kernel
// rewrites every partial it reads.  Two calls that overlap in time -- on
// different streams, or from different host threads -- race on the array.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int64_t kScratchBytes = NOVA_ATTN_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Address of the scratch array on the current device, looked up once per
// device (with that device current).
int scratch_for_current_device(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return nova::fail(NOVA_ERR_CUDA, "cudaGetDevice failed");
    }
    if (dev < 0 || dev >= kMaxDevices) return nova::fail(NOVA_ERR_UNSUPPORTED, "device ordinal %d too large", dev);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (err != cudaSuccess || !p) {
            cudaGetLastError();
            return nova::fail(NOVA_ERR_CUDA, "cudaGetSymbolAddress(attention scratch) failed: %s",
                              cudaGetErrorString(err));
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return NOVA_OK;
}

}  // namespace

extern "C" int nova_attn_decode_int8_noalloc(const nova_attn_int8_args* a, void* stream) {
    if (!a) return nova::fail(NOVA_ERR_INVALID, "args must not be NULL");
    int64_t need = 0;
    if (int rc = nova_attn_workspace_bytes(a->batch, a->q_heads, a->kv_heads, a->n_splits, a->tail_k != nullptr, &need))
        return rc;
    if (need > kScratchBytes)
        return nova::fail(NOVA_ERR_UNSUPPORTED,
                          "nova_attn_decode_int8_noalloc: this shape needs %lld bytes of scratch, the built-in "
                          "array holds %lld (reduce batch, heads or n_splits, or use nova_attn_decode_int8)",
                          (long long)need, (long long)kScratchBytes);
    void* scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    // error word (first 256 bytes) and the per-(batch, kv head) arrival counters start at zero
    const int64_t bh = a->batch * a->kv_heads;
    const size_t head_bytes = size_t(256 + (bh * 4 + 255) / 256 * 256);
    const cudaError_t err = cudaMemsetAsync(scratch, 0, head_bytes, (cudaStream_t)stream);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return nova::fail(NOVA_ERR_CUDA, "clearing the attention scratch failed: %s", cudaGetErrorString(err));
    }
    nova_attn_int8_args b = *a;
    b.workspace = scratch;
    b.workspace_bytes = kScratchBytes;
    return nova_attn_decode_int8(&b, stream);
}

// The kernel's error word is the first word of the built-in array: copy it to
// the host and clear it (synchronous; current device).  Every call of
// nova_attn_decode_int8_noalloc clears it before its kernel, so this reports
// the latest call only.
extern "C" int nova_attn_noalloc_read_error(int* host_value) {
    if (!host_value) return nova::fail(NOVA_ERR_INVALID, "host_value must not be NULL");
    void* scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    if (cudaMemcpy(host_value, scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return nova::fail(NOVA_ERR_CUDA, "reading the attention scratch error word failed");
    }
    if (*host_value && cudaMemset(scratch, 0, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return nova::fail(NOVA_ERR_CUDA, "clearing the attention scratch error word failed");
    }
    return NOVA_OK;
}
