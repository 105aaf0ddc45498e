// RMSNorm (optionally with the residual add in front) and the decoder's
// fused per-head q_norm / k_norm + RoPE + int8 KV append.
//
// Numerics follow the reference exactly where it is defined op by op on fp16
// tensors: RMSNorm in HF order (src/nova/norm.py:37-42, src/nova/kernels.py:
// 51-69): fp32 mean of squares, 1/sqrt(var + eps) with IEEE sqrt and divide,
// h = fp16(x * r), y = fp16(w * h); residual add = fp16(a + b); RoPE
// (src/nova/layers.py:24-36) = fp16(fp16(x*cos) + fp16(rotate_half(x)*sin))
// with the fp16 cos/sin table the HF rotary produces.
#include "common.cuh"
#include "qk_common.cuh"

namespace nova {
namespace norm {

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red may still be read from a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) s += red[w];
    return s;
}

constexpr int RN_THREADS = 256;

__global__ void __launch_bounds__(RN_THREADS) rmsnorm_kernel(const __half* __restrict__ x, int64_t xs,
                                                             const __half* __restrict__ rin, int64_t rins,
                                                             __half* __restrict__ rout, int64_t routs,
                                                             const __half* __restrict__ w, __half* __restrict__ y,
                                                             int64_t ys, int n, float eps) {
    __shared__ float red[RN_THREADS / 32];
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x;
    const __half* xr = x + row * xs;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += RN_THREADS) {
        float h = __half2float(xr[i]);
        if (rin) {
            h = __half2float(__float2half_rn(h + __half2float(rin[row * rins + i])));
            if (rout) rout[row * routs + i] = __float2half_rn(h);
        }
        ss += h * h;
    }
    const float total = block_sum<RN_THREADS>(ss, red);
    const float r = rsqrt_ieee(__fdiv_rn(total, float(n)) + eps);
    for (int i = threadIdx.x; i < n; i += RN_THREADS) {
        float h = __half2float(xr[i]);
        if (rin) h = __half2float(__float2half_rn(h + __half2float(rin[row * rins + i])));
        const float hn = __half2float(__float2half_rn(h * r));
        y[row * ys + i] = __float2half_rn(__half2float(w[i]) * hn);
    }
}

// resid = fp16(resid + fp16(x)) for an fp32 x: the residual add after the
// all-reduce of tensor-parallel partial sums, rounded like the single-GPU
// epilogue (fp16 projection output, then the fp16 add).
__global__ void residual_add_f32_kernel(const float* __restrict__ x, int64_t xs, __half* __restrict__ r, int64_t rs,
                                        int n) {
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float o = __half2float(__float2half_rn(x[row * xs + i]));
        r[row * rs + i] = __float2half_rn(__half2float(r[row * rs + i]) + o);
    }
}

// ---------------------------------------------------------------------------
// One CTA per (batch row, head) over q heads then kv heads; 128 threads = one
// per channel.  q heads: q_norm + RoPE -> q_out.  kv heads: k_norm + RoPE on
// K, both K and V into ring slot pos % 64; when that slot completes the group,
// the ring is requantized into the int8 cache (each thread its own column).

constexpr int D = qk::D;
constexpr int GT = qk::GT;

struct QKParams {
    const __half* qkv;
    int64_t qkv_stride;
    const __half* q_norm_w;
    const __half* k_norm_w;
    const __half* cos;
    const __half* sin;
    int64_t rope_len;
    __half* q_out;
    int64_t q_out_stride;
    __half* tail_k;
    __half* tail_v;
    uint8_t* kq;
    uint8_t* vq;
    __half* kmn;
    __half* kst;
    __half* vmn;
    __half* vst;
    const int64_t* pos;
    int64_t* written;
    int64_t* qlen;
    int64_t* pg;
    int q_heads, kv_heads;
    int64_t max_len;
    float eps;
};

__global__ void __launch_bounds__(D) qk_norm_rope_append_kernel(const __grid_constant__ QKParams p) {
    __shared__ float red[D / 32][1];
    __shared__ __half ybuf[1][D];
    const int m = blockIdx.y;
    const int head = blockIdx.x;
    const int d = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const int64_t pos = *p.pos;
    if (m == 0 && head == 0 && d == 0) {
        const int64_t w = pos + 1;
        const int64_t ql = (w / GT) * GT;
        *p.written = w;
        *p.qlen = ql;
        *p.pg = ql / GT;
    }
    const bool is_q = head < p.q_heads;
    const int kvh = head - p.q_heads;
    const __half* src = p.qkv + m * p.qkv_stride + int64_t(head) * D;
    const __half* nw = is_q ? p.q_norm_w : p.k_norm_w;

    // per-head RMSNorm + RoPE
    const __half xin[1] = {src[d]};
    const int64_t cp = pos < 0 ? 0 : (pos < p.rope_len ? pos : p.rope_len - 1);
    const float c = __half2float(p.cos[cp * D + d]), s = __half2float(p.sin[cp * D + d]);
    __half embv[1];
    qk::norm_rope<1>(xin, nw[d], c, s, p.eps, red, ybuf, embv);
    const __half emb = embv[0];

    if (is_q) {
        p.q_out[m * p.q_out_stride + int64_t(head) * D + d] = emb;
        return;
    }
    if (pos < 0 || pos >= p.max_len) return;
    const __half v = p.qkv[m * p.qkv_stride + int64_t(p.q_heads + p.kv_heads + kvh) * D + d];
    const int64_t bh = int64_t(m) * p.kv_heads + kvh;
    const int slot = int(pos % GT);
    __half* tk = p.tail_k + bh * GT * D;
    __half* tv = p.tail_v + bh * GT * D;
    tk[slot * D + d] = emb;
    tv[slot * D + d] = v;
    if (slot != GT - 1) return;
    const int64_t g = pos / GT;
    const int64_t ngroups = (p.max_len + GT - 1) / GT;
    const int64_t code_off = bh * p.max_len * D + g * GT * D + d;
    const int64_t sc_off = (bh * ngroups + g) * D + d;
    qk::quant_col(tk + d, p.kmn + sc_off, p.kst + sc_off, [&](int t, uint8_t c8) { p.kq[code_off + t * D] = c8; });
    qk::quant_col(tv + d, p.vmn + sc_off, p.vst + sc_off, [&](int t, uint8_t c8) { p.vq[code_off + t * D] = c8; });
}

}  // namespace norm
}  // namespace nova

using namespace nova;

extern "C" int nova_rmsnorm(const void* x, int64_t x_stride, const void* residual_in, int64_t rin_stride,
                            void* residual_out, int64_t rout_stride, const void* weight, void* y, int64_t y_stride,
                            int64_t rows, int64_t n, double eps, void* stream) {
    if (rows < 0 || n <= 0 || n > (1 << 24)) return fail(NOVA_ERR_INVALID, "bad rows/n");
    if (!x || !weight || !y) return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (residual_out && !residual_in) return fail(NOVA_ERR_INVALID, "residual_out needs residual_in");
    if (rows == 0) return NOVA_OK;
    if (rows > 0x7fffffff) return fail(NOVA_ERR_INVALID, "too many rows");
    const cudaError_t err =
        launch(norm::rmsnorm_kernel, dim3(unsigned(rows)), dim3(norm::RN_THREADS), 0, (cudaStream_t)stream,
               (const __half*)x, x_stride, (const __half*)residual_in, rin_stride, (__half*)residual_out, rout_stride,
               (const __half*)weight, (__half*)y, y_stride, int(n), float(eps));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_rmsnorm: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_qk_norm_rope_append(const nova_qk_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->head_dim != 128 || a->group != 64)
        return fail(NOVA_ERR_UNSUPPORTED, "head_dim must be 128 and group 64");
    if (a->batch <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 || a->batch > 65535 || a->q_heads + a->kv_heads > 65535)
        return fail(NOVA_ERR_INVALID, "bad batch/heads");
    if (a->rope_len <= 0 || a->max_len <= 0) return fail(NOVA_ERR_INVALID, "bad rope_len/max_len");
    if (!a->qkv || !a->q_norm_weight || !a->k_norm_weight || !a->cos || !a->sin || !a->q_out || !a->tail_k ||
        !a->tail_v || !a->kq || !a->vq || !a->kmn || !a->kst || !a->vmn || !a->vst || !a->pos || !a->written ||
        !a->qlen || !a->pg)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    norm::QKParams p;
    p.qkv = (const __half*)a->qkv;
    p.qkv_stride = a->qkv_stride;
    p.q_norm_w = (const __half*)a->q_norm_weight;
    p.k_norm_w = (const __half*)a->k_norm_weight;
    p.cos = (const __half*)a->cos;
    p.sin = (const __half*)a->sin;
    p.rope_len = a->rope_len;
    p.q_out = (__half*)a->q_out;
    p.q_out_stride = a->q_out_stride;
    p.tail_k = (__half*)a->tail_k;
    p.tail_v = (__half*)a->tail_v;
    p.kq = (uint8_t*)a->kq;
    p.vq = (uint8_t*)a->vq;
    p.kmn = (__half*)a->kmn;
    p.kst = (__half*)a->kst;
    p.vmn = (__half*)a->vmn;
    p.vst = (__half*)a->vst;
    p.pos = a->pos;
    p.written = a->written;
    p.qlen = a->qlen;
    p.pg = a->pg;
    p.q_heads = int(a->q_heads);
    p.kv_heads = int(a->kv_heads);
    p.max_len = a->max_len;
    p.eps = float(a->eps);
    dim3 grid{unsigned(a->q_heads + a->kv_heads), unsigned(a->batch), 1u};
    const cudaError_t err = launch(norm::qk_norm_rope_append_kernel, grid, dim3(128), 0, (cudaStream_t)stream, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_qk_norm_rope_append: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_residual_add_f32(const void* x, int64_t x_stride, void* residual, int64_t r_stride, int64_t rows,
                                     int64_t n, void* stream) {
    if (rows < 0 || n <= 0 || n > (1 << 24) || rows > 65535) return fail(NOVA_ERR_INVALID, "bad rows/n");
    if (!x || !residual) return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (rows == 0) return NOVA_OK;
    const unsigned blocks = unsigned(std::min<int64_t>((n + 255) / 256, 64));
    const cudaError_t err = launch(norm::residual_add_f32_kernel, dim3(blocks, unsigned(rows)), dim3(256), 0,
                                   (cudaStream_t)stream, (const float*)x, x_stride, (__half*)residual, r_stride, int(n));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_residual_add_f32: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}
