// Per-head q_norm / k_norm + RoPE and the requantization of a full fp16 ring
// group into the int8t64 cache, shared by the standalone q/k kernel (norm.cu)
// and the decode attention that runs them in its prologue (attn.cu), so both
// produce the same bits.  Thread d of a 128-thread CTA owns channel d.
//
// Numerics (src/nova/norm.py:37-42, src/nova/layers.py:24-36,
// src/nova/kvquant.py int8t64 group quantization): fp32 mean of squares,
// r = 1/sqrt(mean + eps) with IEEE sqrt and divide, h = fp16(x * r),
// y = fp16(w * h); RoPE = fp16(fp16(y*cos) + fp16(rotate_half(y)*sin)) with
// the fp16 cos/sin table; group codes = clamp(rint((v - mn) / step), 0, 255)
// with step = max((mx - mn) / 255, 1e-8) in fp32, mn and step stored as fp16.
// Products and sums use explicit round-to-nearest intrinsics so that no
// multiply-add is contracted differently in the two kernels.
#pragma once

#include "common.cuh"

namespace nova {
namespace qk {

constexpr int D = 128;
constexpr int GT = 64;

// Sum over the 128 channels of NH values per thread, in a fixed order: warp
// butterfly (xor 16, 8, 4, 2, 1), then the four warp sums in warp order.
// red: shared [4][NH].  Every thread gets the sums.
template <int NH>
__device__ __forceinline__ void sum128(float (&v)[NH], float (*red)[NH]) {
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v[h] = __fadd_rn(v[h], __shfl_xor_sync(0xffffffffu, v[h], off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();   // red (and the caller's ybuf) may still be read from a previous call
    if (lane == 0)
#pragma unroll
        for (int h = 0; h < NH; ++h) red[warp][h] = v[h];
    __syncthreads();
#pragma unroll
    for (int h = 0; h < NH; ++h) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < D / 32; ++w) s = __fadd_rn(s, red[w][h]);
        v[h] = s;
    }
}

// RMSNorm (weight nw of this channel) + RoPE (c, s of this channel) of NH
// heads; xin: this channel of each head.  ybuf: shared [NH][128].
template <int NH>
__device__ __forceinline__ void norm_rope(const __half (&xin)[NH], __half nw, float c, float s, float eps,
                                          float (*red)[NH], __half (*ybuf)[D], __half (&emb)[NH]) {
    const int d = threadIdx.x;
    float x[NH], ss[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
        x[h] = __half2float(xin[h]);
        ss[h] = __fmul_rn(x[h], x[h]);
    }
    sum128<NH>(ss, red);
    const float w = __half2float(nw);
    __half y[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
        const float r = rsqrt_ieee(__fadd_rn(__fdiv_rn(ss[h], float(D)), eps));
        const float hn = __half2float(__float2half_rn(__fmul_rn(x[h], r)));
        y[h] = __float2half_rn(__fmul_rn(w, hn));
        ybuf[h][d] = y[h];
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < NH; ++h) {
        // rotate_half(y)[d] = -y[d + 64] (d < 64) or y[d - 64]
        const float yr = d < D / 2 ? -__half2float(ybuf[h][d + D / 2]) : __half2float(ybuf[h][d - D / 2]);
        const float a = __half2float(__float2half_rn(__fmul_rn(__half2float(y[h]), c)));
        const float b = __half2float(__float2half_rn(__fmul_rn(yr, s)));
        emb[h] = __float2half_rn(__fadd_rn(a, b));
    }
}

// Channel d of a full ring group: src[t * 128], t = 0..63 (fp16).  Writes the
// fp16 min and step and hands every code to emit(t, code).
template <typename Emit>
__device__ __forceinline__ void quant_col(const __half* src, __half* mn_out, __half* st_out, Emit&& emit) {
    float mn = INFINITY, mx = -INFINITY;
    for (int t = 0; t < GT; ++t) {
        const float v = __half2float(src[t * D]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    const float step = fmaxf(__fdiv_rn(mx - mn, 255.0f), 1e-8f);
    for (int t = 0; t < GT; ++t) {
        const float v = __half2float(src[t * D]);
        float c = rintf(__fdiv_rn(v - mn, step));
        c = fminf(fmaxf(c, 0.0f), 255.0f);
        emit(t, static_cast<uint8_t>(c));
    }
    *mn_out = __float2half_rn(mn);
    *st_out = __float2half_rn(step);
}

}  // namespace qk
}  // namespace nova
