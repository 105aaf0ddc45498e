// int8 KV cache: token-axis quantize / dequantize and the decode-step append
// into the 64-slot fp16 ring + int8 groups.
//
// Numerics follow the reference quantizer exactly (src/nova/kvquant.py:118-176,
// src/nova/kvattn.py:716-743): fp32 min/max, step = max((max-min)/255, 1e-8)
// with an IEEE division, codes = clamp(rint((x-min)/step), 0, 255) with an
// IEEE division and round-half-even, min/step stored as fp16 (RN).
#include "common.cuh"

namespace nova {

// Per-column group statistics and codes for `cnt` tokens at `src` (stride
// `ld` elements between tokens); writes codes with stride `qld` bytes.
__device__ __forceinline__ void quant_column(const __half* src, int64_t ld, int cnt, uint8_t* q, int64_t qld,
                                             __half* mn_out, __half* st_out) {
    float mn = INFINITY, mx = -INFINITY;
    for (int t = 0; t < cnt; ++t) {
        float v = __half2float(src[t * ld]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    float step = fmaxf(__fdiv_rn(mx - mn, 255.0f), 1e-8f);
    for (int t = 0; t < cnt; ++t) {
        float v = __half2float(src[t * ld]);
        float c = rintf(__fdiv_rn(v - mn, step));
        c = fminf(fmaxf(c, 0.0f), 255.0f);
        q[t * qld] = static_cast<uint8_t>(c);
    }
    *mn_out = __float2half_rn(mn);
    *st_out = __float2half_rn(step);
}

__global__ void kv_quant_int8_kernel(const __half* __restrict__ x, int64_t xs, uint8_t* __restrict__ q, int64_t qs,
                                     __half* __restrict__ mins, __half* __restrict__ steps, int64_t ss, int n,
                                     int dim, int group) {
    const int g = blockIdx.x;
    const int64_t row = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    const int t0 = g * group;
    const int cnt = min(group, n - t0);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        quant_column(x + row * xs + int64_t(t0) * dim + d, dim, cnt, q + row * qs + int64_t(t0) * dim + d, dim,
                     mins + row * ss + int64_t(g) * dim + d, steps + row * ss + int64_t(g) * dim + d);
    }
}

__global__ void kv_dequant_int8_kernel(const uint8_t* __restrict__ q, int64_t qs, const __half* __restrict__ mins,
                                       const __half* __restrict__ steps, int64_t ss, __half* __restrict__ x,
                                       int64_t xs, int n, int dim, int group) {
    const int64_t row = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    const int64_t total = int64_t(n) * dim;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int t = int(i / dim), d = int(i % dim);
        const int64_t si = row * ss + int64_t(t / group) * dim + d;
        float v = __fadd_rn(__fmul_rn(float(q[row * qs + i]), __half2float(steps[si])), __half2float(mins[si]));
        x[row * xs + i] = __float2half_rn(v);
    }
}

__global__ void kv_append_int8_kernel(const __half* __restrict__ k_new, const __half* __restrict__ v_new,
                                      int64_t nbs, int64_t nhs, __half* __restrict__ tail_k,
                                      __half* __restrict__ tail_v, uint8_t* __restrict__ kq,
                                      uint8_t* __restrict__ vq, __half* __restrict__ kmn, __half* __restrict__ kst,
                                      __half* __restrict__ vmn, __half* __restrict__ vst,
                                      const int64_t* __restrict__ pos_p, int64_t* __restrict__ written,
                                      int64_t* __restrict__ qlen, int64_t* __restrict__ pg, int kv_heads,
                                      int64_t max_len, int dim, int group) {
    const int bh = blockIdx.x;
    const int b = bh / kv_heads, h = bh % kv_heads;
    pdl_trigger();
    pdl_wait();
    const int64_t pos = *pos_p;
    if (bh == 0 && threadIdx.x == 0) {
        const int64_t w = pos + 1;
        const int64_t ql = (w / group) * group;
        *written = w;
        *qlen = ql;
        *pg = ql / group;
    }
    if (pos < 0 || pos >= max_len) return;  // out of capacity: write nothing
    const int slot = int(pos % group);
    const int64_t g = pos / group;
    const int64_t ngroups = (max_len + group - 1) / group;
    __half* tk = tail_k + int64_t(bh) * group * dim;
    __half* tv = tail_v + int64_t(bh) * group * dim;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        tk[slot * dim + d] = k_new[b * nbs + h * nhs + d];
        tv[slot * dim + d] = v_new[b * nbs + h * nhs + d];
    }
    if (slot != group - 1) return;
    // The ring now holds exactly the `group` tokens of group g, slot == in-group
    // offset; each thread requantizes the columns it just wrote (no sync needed).
    const int64_t code_off = int64_t(bh) * max_len * dim + g * group * dim;
    const int64_t sc_off = (int64_t(bh) * ngroups + g) * dim;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        quant_column(tk + d, dim, group, kq + code_off + d, dim, kmn + sc_off + d, kst + sc_off + d);
        quant_column(tv + d, dim, group, vq + code_off + d, dim, vmn + sc_off + d, vst + sc_off + d);
    }
}

}  // namespace nova

using namespace nova;

static int check_common(int64_t rows, int64_t n, int64_t dim, int64_t group) {
    if (rows < 0 || n < 0) return fail(NOVA_ERR_INVALID, "rows/n must be >= 0");
    if (dim <= 0 || dim > 1024) return fail(NOVA_ERR_INVALID, "dim must be in [1, 1024], got %lld", (long long)dim);
    if (group <= 0 || group > 4096) return fail(NOVA_ERR_INVALID, "group must be in [1, 4096]");
    if (rows > 65535) return fail(NOVA_ERR_INVALID, "rows must be <= 65535");
    return NOVA_OK;
}

extern "C" int nova_kv_quant_int8(const void* x, int64_t x_row_stride, void* q, int64_t q_row_stride, void* mins,
                                  void* steps, int64_t s_row_stride, int64_t rows, int64_t n, int64_t dim,
                                  int64_t group, void* stream) {
    if (int rc = check_common(rows, n, dim, group)) return rc;
    if (!rows || !n) return NOVA_OK;
    const int64_t ng = (n + group - 1) / group;
    if (ng > 0x7fffffff) return fail(NOVA_ERR_INVALID, "too many groups");
    dim3 grid{unsigned(ng), unsigned(rows), 1u};
    const cudaError_t err = launch(kv_quant_int8_kernel, grid, dim3(128), 0, (cudaStream_t)stream, (const __half*)x,
                                   x_row_stride, (uint8_t*)q, q_row_stride, (__half*)mins, (__half*)steps,
                                   s_row_stride, int(n), int(dim), int(group));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_kv_quant_int8: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_kv_dequant_int8(const void* q, int64_t q_row_stride, const void* mins, const void* steps,
                                    int64_t s_row_stride, void* x, int64_t x_row_stride, int64_t rows, int64_t n,
                                    int64_t dim, int64_t group, void* stream) {
    if (int rc = check_common(rows, n, dim, group)) return rc;
    if (!rows || !n) return NOVA_OK;
    const int64_t total = n * dim;
    unsigned blocks = unsigned(std::min<int64_t>((total + 255) / 256, 4096));
    dim3 grid{blocks, unsigned(rows), 1u};
    const cudaError_t err =
        launch(kv_dequant_int8_kernel, grid, dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)q, q_row_stride,
               (const __half*)mins, (const __half*)steps, s_row_stride, (__half*)x, x_row_stride, int(n), int(dim),
               int(group));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_kv_dequant_int8: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_kv_append_int8(const void* k_new, const void* v_new, int64_t new_b_stride, int64_t new_h_stride,
                                   void* tail_k, void* tail_v, void* kq, void* vq, void* kmn, void* kst, void* vmn,
                                   void* vst, const int64_t* pos, int64_t* written, int64_t* qlen, int64_t* pg,
                                   int64_t batch, int64_t kv_heads, int64_t max_len, int64_t dim, int64_t group,
                                   void* stream) {
    if (batch <= 0 || kv_heads <= 0 || batch * kv_heads > 0x7fffffff)
        return fail(NOVA_ERR_INVALID, "batch/kv_heads out of range");
    if (dim <= 0 || dim > 1024) return fail(NOVA_ERR_INVALID, "dim must be in [1, 1024]");
    if (group <= 0 || group > 1024 || max_len <= 0) return fail(NOVA_ERR_INVALID, "group/max_len out of range");
    if (!pos || !written || !qlen || !pg) return fail(NOVA_ERR_INVALID, "device scalars must not be NULL");
    const cudaError_t err = launch(
        kv_append_int8_kernel, dim3(unsigned(batch * kv_heads)), dim3(128), 0, (cudaStream_t)stream,
        (const __half*)k_new, (const __half*)v_new, new_b_stride, new_h_stride, (__half*)tail_k, (__half*)tail_v,
        (uint8_t*)kq, (uint8_t*)vq, (__half*)kmn, (__half*)kst, (__half*)vmn, (__half*)vst, pos, written, qlen, pg,
        int(kv_heads), max_len, int(dim), int(group));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_kv_append_int8: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}
