// Prefill kernels on the int8 cache (sm_100a): causal multi-token GQA
// attention of a chunk of queries over the int8 prefix read in place plus
// fp16 keys, and the per-head q/k norm + RoPE of a chunk of q|k|v rows.
//
// nova_attn_prefill_int8 -- grid (ceil(n/64) query blocks, q heads, batch), 4
// warps; warp w owns the 16 query tokens 64*blockIdx.x + 16w .. +15 of one q
// head.  Keys come in 64-token tiles staged in shared memory as fp16 (rows
// padded to 136 halves, so the fragment loads below are bank-conflict free):
// the int8 tiles [0, int8_len) dequantized on the way in exactly as the
// reference does it (fp32 code * fp32 step, + fp32 min, rounded to fp16;
// src/nova/kvquant.py:166-176), the fp16 tiles copied.  S = Q K^T and
// O += P V run on mma.sync m16n8k16 with fp32 accumulators; P is fed to the
// PV product as its fp16 high part plus its fp16 low part (two MMAs), so the
// weights keep ~22 bits; the online softmax is fp32 (exp2 domain).  Output
// fp16(O / l), written row = token, columns = head * 128 + d (the o_proj
// input layout).
//
// Reference semantics: KVInt8Cache.attend_prefill over the fp16 staging
// (src/nova/kvattn.py:791-815, causal mask, optional window) and the chunked
// int8 prefill the reference plans (reports/kv-int8-streaming-cache.md
// section 5.1): later chunks attend to the dequantized int8 prefix.
#include <algorithm>

#include "common.cuh"
#include "qk_common.cuh"

namespace nova {
namespace prefill {

constexpr int D = 128;
constexpr int GT = 64;
constexpr int NW = 4;
constexpr int THREADS = NW * 32;
constexpr int QB = 64;             // query tokens per CTA
constexpr int KT = 64;             // keys per tile
constexpr int LD = D + 8;          // padded row, halves
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
    const __half* q;               // [b][h][t][d] strides in elements
    int64_t q_b, q_h, q_t;
    const __half* k;               // fp16 keys of positions [int8_len, prefix + n)
    const __half* v;
    int64_t kv_b, kv_h, kv_t;
    const uint8_t* kq;             // int8 cache [b][h][max_len][d] (positions [0, int8_len))
    const uint8_t* vq;
    const __half* kmn;             // [b][h][groups][d]
    const __half* kst;
    const __half* vmn;
    const __half* vst;
    int64_t max_len, groups;
    __half* out;                   // [b][t][q_heads * d]
    int64_t o_b, o_t;
    int q_heads, kv_heads, n, prefix, int8_len, window;
    int kv_vec;                    // fp16 k / v rows 16-byte aligned: 8-channel vector loads
    float scale_log2;
};

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    __half2 v = __halves2half2(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Four 8x8 fp16 matrices from shared memory (lane l gives a row address of
// matrix l / 8); .trans hands each thread the transposed fragment.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__global__ void __launch_bounds__(THREADS) attn_prefill_kernel(const __grid_constant__ Params p) {
    __shared__ __align__(16) __half Ks[KT * LD];
    __shared__ __align__(16) __half Vs[KT * LD];
    const int qb = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int kvh = hq / (p.q_heads / p.kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int q0 = qb * QB + 16 * warp;                 // this warp's first query (chunk-relative)
    pdl_trigger();
    pdl_wait();

    // Q A-fragments: rows q0 + g (a0, a2) and q0 + g + 8 (a1, a3), k-step s covers dims 16s .. 16s+15
    uint32_t qa[8][4];
    {
        const __half* qp = p.q + b * p.q_b + int64_t(hq) * p.q_h;
        const int r0 = min(q0 + g, p.n - 1), r1 = min(q0 + g + 8, p.n - 1);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            qa[s][0] = *reinterpret_cast<const uint32_t*>(qp + int64_t(r0) * p.q_t + 16 * s + 2 * t);
            qa[s][1] = *reinterpret_cast<const uint32_t*>(qp + int64_t(r1) * p.q_t + 16 * s + 2 * t);
            qa[s][2] = *reinterpret_cast<const uint32_t*>(qp + int64_t(r0) * p.q_t + 16 * s + 8 + 2 * t);
            qa[s][3] = *reinterpret_cast<const uint32_t*>(qp + int64_t(r1) * p.q_t + 16 * s + 8 + 2 * t);
        }
    }
    float acc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int64_t pos_row[2] = {int64_t(p.prefix) + q0 + g, int64_t(p.prefix) + q0 + g + 8};

    // key positions this CTA needs: [lo, hi)
    const int64_t cta_last = int64_t(p.prefix) + min(qb * QB + QB, p.n) - 1;
    int64_t lo = 0;
    if (p.window > 0) lo = max(int64_t(0), int64_t(p.prefix) + qb * QB - p.window + 1);
    const int64_t hi = cta_last + 1;
    const int tile_lo = int(lo / KT), tile_hi = int((hi + KT - 1) / KT);
    const int64_t bh = int64_t(b) * p.kv_heads + kvh;

    for (int tile = tile_lo; tile < tile_hi; ++tile) {
        const int64_t p0 = int64_t(tile) * KT;
        __syncthreads();   // the previous tile's fragments have been read
        // ---- stage 64 keys: thread i owns channels 8c .. 8c+7 (c = i % 16) of rows i / 16 + 8j
        {
            const int c = threadIdx.x & 15, rb = threadIdx.x >> 4;
            if (p0 < p.int8_len) {   // int8 tile (int8_len is a multiple of 64)
                const int64_t gi = p0 / GT;
                const int64_t so = (bh * p.groups + gi) * D + 8 * c;
                float ks[8], km[8], vs[8], vm[8];
                {
                    const uint4 a = *reinterpret_cast<const uint4*>(p.kst + so);
                    const uint4 b = *reinterpret_cast<const uint4*>(p.kmn + so);
                    const uint4 e = *reinterpret_cast<const uint4*>(p.vst + so);
                    const uint4 f = *reinterpret_cast<const uint4*>(p.vmn + so);
                    const __half* ah = reinterpret_cast<const __half*>(&a);
                    const __half* bh2 = reinterpret_cast<const __half*>(&b);
                    const __half* eh = reinterpret_cast<const __half*>(&e);
                    const __half* fh = reinterpret_cast<const __half*>(&f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        ks[i] = __half2float(ah[i]);
                        km[i] = __half2float(bh2[i]);
                        vs[i] = __half2float(eh[i]);
                        vm[i] = __half2float(fh[i]);
                    }
                }
                const uint8_t* kc = p.kq + (bh * p.max_len + p0) * D + 8 * c;
                const uint8_t* vc = p.vq + (bh * p.max_len + p0) * D + 8 * c;
#pragma unroll 2
                for (int j = 0; j < KT / 8; ++j) {
                    const int r = rb + 8 * j;
                    const uint2 kb = *reinterpret_cast<const uint2*>(kc + r * D);
                    const uint2 vb = *reinterpret_cast<const uint2*>(vc + r * D);
                    uint4 ko, vo;
                    __half* kh = reinterpret_cast<__half*>(&ko);
                    __half* vh = reinterpret_cast<__half*>(&vo);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {   // the reference's dequant: fp32 code * step + min, to fp16
                        const uint32_t kw = i < 4 ? kb.x : kb.y, vw = i < 4 ? vb.x : vb.y;
                        const float kcode = float((kw >> (8 * (i & 3))) & 0xFFu);
                        const float vcode = float((vw >> (8 * (i & 3))) & 0xFFu);
                        kh[i] = __float2half_rn(__fadd_rn(__fmul_rn(kcode, ks[i]), km[i]));
                        vh[i] = __float2half_rn(__fadd_rn(__fmul_rn(vcode, vs[i]), vm[i]));
                    }
                    *reinterpret_cast<uint4*>(Ks + r * LD + 8 * c) = ko;
                    *reinterpret_cast<uint4*>(Vs + r * LD + 8 * c) = vo;
                }
            } else {
                const __half* kp = p.k + b * p.kv_b + int64_t(kvh) * p.kv_h;
                const __half* vp = p.v + b * p.kv_b + int64_t(kvh) * p.kv_h;
                const int64_t nk = int64_t(p.prefix) + p.n - p.int8_len;   // fp16 keys held
#pragma unroll 2
                for (int j = 0; j < KT / 8; ++j) {
                    const int r = rb + 8 * j;
                    const int64_t kr = p0 + r - p.int8_len;
                    const bool in = kr >= 0 && kr < nk;
                    uint4 ko = make_uint4(0u, 0u, 0u, 0u), vo = ko;
                    if (in && p.kv_vec) {
                        ko = *reinterpret_cast<const uint4*>(kp + kr * p.kv_t + 8 * c);
                        vo = *reinterpret_cast<const uint4*>(vp + kr * p.kv_t + 8 * c);
                    } else if (in) {
                        __half* kh = reinterpret_cast<__half*>(&ko);
                        __half* vh = reinterpret_cast<__half*>(&vo);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            kh[i] = kp[kr * p.kv_t + 8 * c + i];
                            vh[i] = vp[kr * p.kv_t + 8 * c + i];
                        }
                    }
                    *reinterpret_cast<uint4*>(Ks + r * LD + 8 * c) = ko;
                    *reinterpret_cast<uint4*>(Vs + r * LD + 8 * c) = vo;
                }
            }
        }
        __syncthreads();
        if (q0 >= p.n) continue;   // a ragged last block: warps past n only help staging
        // ---- S = Q K^T: 8 n-tiles of 8 keys
        // B fragments by ldmatrix: matrix i of lane l = keys 8j .. 8j+7, dims 16s + 8i (two k-steps per load)
        float sc[8][4];
        const uint32_t ks_base = smem_u32(Ks) + uint32_t(((lane & 7) * LD + 8 * (lane >> 3)) * 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
            for (int s = 0; s < 8; s += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(ks_base + uint32_t((8 * j * LD + 16 * s) * 2), b0, b1, b2, b3);
                mma_16816(sc[j], qa[s][0], qa[s][1], qa[s][2], qa[s][3], b0, b1);
                mma_16816(sc[j], qa[s + 1][0], qa[s + 1][1], qa[s + 1][2], qa[s + 1][3], b2, b3);
            }
        }
        // ---- mask, online softmax (rows g: sc[j][0..1], row g + 8: sc[j][2..3])
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const int64_t kp = p0 + 8 * j + 2 * t + (e & 1);
                bool ok = kp <= pos_row[rr] && kp < int64_t(p.prefix) + p.n;
                if (p.window > 0) ok = ok && pos_row[rr] - kp < p.window;
                sc[j][e] = ok ? sc[j][e] * p.scale_log2 : -INFINITY;
                mx[rr] = fmaxf(mx[rr], sc[j][e]);
            }
        float alpha[2];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
            const float m_new = fmaxf(m_run[rr], mx[rr]);
            alpha[rr] = m_new == -INFINITY ? 1.f : exp2f(m_run[rr] - m_new);
            m_run[rr] = m_new;
        }
        float rs[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const float x = m_run[rr] == -INFINITY ? 0.f : exp2f(sc[j][e] - m_run[rr]);
                sc[j][e] = x;
                rs[rr] += x;
            }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 1);
            rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 2);
            l_run[rr] = l_run[rr] * alpha[rr] + rs[rr];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            acc[j][0] *= alpha[0];
            acc[j][1] *= alpha[0];
            acc[j][2] *= alpha[1];
            acc[j][3] *= alpha[1];
        }
        // ---- O += P V: k-step s = keys 16s .. 16s+15, P as fp16 high + low parts
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t ah[4], al[4];
            const float* c0 = sc[2 * s];
            const float* c1 = sc[2 * s + 1];
            const float pv[8] = {c0[0], c0[1], c0[2], c0[3], c1[0], c1[1], c1[2], c1[3]};
            __half hv[8], lv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                hv[i] = __float2half_rn(pv[i]);
                lv[i] = __float2half_rn(pv[i] - __half2float(hv[i]));
            }
            // a0 = row g keys 2t,2t+1 (tile 2s), a1 = row g+8 (tile 2s), a2/a3 = tile 2s+1
            ah[0] = pack_h2(hv[0], hv[1]); ah[1] = pack_h2(hv[2], hv[3]);
            ah[2] = pack_h2(hv[4], hv[5]); ah[3] = pack_h2(hv[6], hv[7]);
            al[0] = pack_h2(lv[0], lv[1]); al[1] = pack_h2(lv[2], lv[3]);
            al[2] = pack_h2(lv[4], lv[5]); al[3] = pack_h2(lv[6], lv[7]);
            // matrix i of lane l = keys 16s + 8 (i & 1) .. +7, dims 8j + 8 (i >> 1): transposed, the B
            // fragments of n-tiles j and j + 1
            const uint32_t vs_base = smem_u32(Vs) +
                                     uint32_t(((16 * s + 8 * ((lane >> 3) & 1) + (lane & 7)) * LD + 8 * (lane >> 4)) * 2);
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(vs_base + uint32_t(16 * j), b0, b1, b2, b3);
                mma_16816(acc[j], ah[0], ah[1], ah[2], ah[3], b0, b1);
                mma_16816(acc[j], al[0], al[1], al[2], al[3], b0, b1);
                mma_16816(acc[j + 1], ah[0], ah[1], ah[2], ah[3], b2, b3);
                mma_16816(acc[j + 1], al[0], al[1], al[2], al[3], b2, b3);
            }
        }
    }
    if (q0 >= p.n) return;
    // ---- out = fp16(O / l); rows q0 + g and q0 + g + 8, dims 8j + 2t, +1
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int row = q0 + g + 8 * rr;
        if (row >= p.n) continue;
        const float l = l_run[rr];
        __half* op = p.out + b * p.o_b + int64_t(row) * p.o_t + int64_t(hq) * D;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float a = l > 0.f ? __fdiv_rn(acc[j][2 * rr], l) : 0.f;
            const float c = l > 0.f ? __fdiv_rn(acc[j][2 * rr + 1], l) : 0.f;
            *reinterpret_cast<__half2*>(op + 8 * j + 2 * t) = __floats2half2_rn(a, c);
        }
    }
}

// q|k|v rows of a chunk (fp16 [b][t][(q_heads + 2 kv_heads) * 128]) -> q after
// q_norm + RoPE [b][q_heads][t][128], k after k_norm (before RoPE, k_pre,
// optional) and after RoPE [b][kv_heads][t][128], v [b][kv_heads][t][128], for
// positions pos0 + t.  One CTA per (token, head-slot); the arithmetic of the
// decode step's q/k kernel (qk::norm_rope).
struct QkParams {
    const __half* qkv;
    int64_t qkv_b, qkv_t;
    const __half* q_norm_w;
    const __half* k_norm_w;
    const __half* cos;
    const __half* sin;
    int64_t rope_len;
    __half* q_out;
    __half* k_out;
    __half* k_pre;
    __half* v_out;
    int64_t qo_b, qo_h, ko_b, ko_h;     // token stride is 128 in every output
    int q_heads, kv_heads, n;
    int64_t pos0;
    float eps;
};

__global__ void __launch_bounds__(D) qk_prefill_kernel(const __grid_constant__ QkParams p) {
    __shared__ float red[D / 32][1];
    __shared__ __align__(16) __half ybuf[1][D];
    const int tok = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
    const int d = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const __half* row = p.qkv + b * p.qkv_b + int64_t(tok) * p.qkv_t;
    const int64_t pos = p.pos0 + tok;
    const int64_t cp = pos < 0 ? 0 : (pos < p.rope_len ? pos : p.rope_len - 1);
    const float c = __half2float(p.cos[cp * D + d]), s = __half2float(p.sin[cp * D + d]);
    if (head < p.q_heads) {
        __half x[1] = {row[int64_t(head) * D + d]}, e[1];
        qk::norm_rope<1>(x, p.q_norm_w[d], c, s, p.eps, red, ybuf, e);
        p.q_out[b * p.qo_b + int64_t(head) * p.qo_h + int64_t(tok) * D + d] = e[0];
    } else if (head < p.q_heads + p.kv_heads) {
        const int kh = head - p.q_heads;
        __half x[1] = {row[int64_t(p.q_heads + kh) * D + d]}, e[1];
        qk::norm_rope<1>(x, p.k_norm_w[d], c, s, p.eps, red, ybuf, e);
        const int64_t o = b * p.ko_b + int64_t(kh) * p.ko_h + int64_t(tok) * D + d;
        p.k_out[o] = e[0];
        if (p.k_pre) p.k_pre[o] = ybuf[0][d];   // the normed value before RoPE
    } else {
        const int vh = head - p.q_heads - p.kv_heads;
        p.v_out[b * p.ko_b + int64_t(vh) * p.ko_h + int64_t(tok) * D + d] = row[int64_t(p.q_heads + p.kv_heads + vh) * D + d];
    }
}

}  // namespace prefill
}  // namespace nova

using namespace nova;

extern "C" int nova_attn_prefill_int8(const nova_prefill_attn_args* a, void* stream) {
    using namespace nova::prefill;
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->head_dim != D) return fail(NOVA_ERR_UNSUPPORTED, "head_dim must be 128");
    if (a->batch <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 || a->q_heads % a->kv_heads || a->n <= 0)
        return fail(NOVA_ERR_INVALID, "bad batch / heads / n");
    if (a->batch > 65535 || a->q_heads > 65535 || (a->n + QB - 1) / QB > 0x7fffffff)
        return fail(NOVA_ERR_INVALID, "grid too large");
    if (a->prefix < 0 || a->int8_len < 0 || a->int8_len > a->prefix || a->int8_len % GT || a->window < 0)
        return fail(NOVA_ERR_INVALID, "need 0 <= int8_len <= prefix, int8_len a multiple of 64, window >= 0");
    if (!a->q || !a->out || (a->prefix + a->n > a->int8_len && (!a->k || !a->v)))
        return fail(NOVA_ERR_INVALID, "q / out / fp16 k, v must not be NULL");
    if (a->int8_len &&
        (!a->kq || !a->vq || !a->kmn || !a->kst || !a->vmn || !a->vst || a->int8_len > a->max_len ||
         a->groups != (a->max_len + GT - 1) / GT))
        return fail(NOVA_ERR_INVALID, "the int8 prefix needs the cache buffers, int8_len <= max_len and "
                                      "groups = ceil(max_len / 64)");
    auto mis = [](const void* ptr, int al) { return ptr && (reinterpret_cast<uintptr_t>(ptr) % al); };
    if (a->int8_len && (mis(a->kq, 8) || mis(a->vq, 8) || mis(a->kmn, 16) || mis(a->kst, 16) || mis(a->vmn, 16) ||
                        mis(a->vst, 16)))
        return fail(NOVA_ERR_ALIGN, "int8 codes 8-byte and scale vectors 16-byte aligned");
    if (mis(a->q, 4) || mis(a->out, 4) || (a->q_t_stride % 2) || (a->q_h_stride % 2) || (a->q_b_stride % 2) ||
        (a->o_t_stride % 2) || (a->o_b_stride % 2))
        return fail(NOVA_ERR_ALIGN, "q / out need 4-byte alignment and even strides");
    Params p;
    p.q = (const __half*)a->q;
    p.q_b = a->q_b_stride;
    p.q_h = a->q_h_stride;
    p.q_t = a->q_t_stride;
    p.k = (const __half*)a->k;
    p.v = (const __half*)a->v;
    p.kv_b = a->kv_b_stride;
    p.kv_h = a->kv_h_stride;
    p.kv_t = a->kv_t_stride;
    p.kq = (const uint8_t*)a->kq;
    p.vq = (const uint8_t*)a->vq;
    p.kmn = (const __half*)a->kmn;
    p.kst = (const __half*)a->kst;
    p.vmn = (const __half*)a->vmn;
    p.vst = (const __half*)a->vst;
    p.max_len = a->max_len;
    p.groups = a->groups;
    p.out = (__half*)a->out;
    p.o_b = a->o_b_stride;
    p.o_t = a->o_t_stride;
    p.q_heads = int(a->q_heads);
    p.kv_heads = int(a->kv_heads);
    p.n = int(a->n);
    p.prefix = int(a->prefix);
    p.int8_len = int(a->int8_len);
    p.window = int(std::min<int64_t>(a->window, 0x7fffffff));
    p.kv_vec = (!mis(a->k, 16) && !mis(a->v, 16) && a->kv_t_stride % 8 == 0 && a->kv_h_stride % 8 == 0 &&
                a->kv_b_stride % 8 == 0) ? 1 : 0;
    p.scale_log2 = float(1.0 / sqrt(double(D))) * LOG2E;
    const dim3 grid(unsigned((a->n + QB - 1) / QB), unsigned(a->q_heads), unsigned(a->batch));
    const cudaError_t err = launch(attn_prefill_kernel, grid, dim3(THREADS), 0, (cudaStream_t)stream, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_attn_prefill_int8: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_qk_prefill(const nova_qk_prefill_args* a, void* stream) {
    using namespace nova::prefill;
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->head_dim != D) return fail(NOVA_ERR_UNSUPPORTED, "head_dim must be 128");
    if (a->batch <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 || a->n <= 0 || a->batch > 65535 ||
        a->q_heads + 2 * a->kv_heads > 65535 || a->n > 0x7fffffff || a->rope_len <= 0)
        return fail(NOVA_ERR_INVALID, "bad batch / heads / n / rope_len");
    if (!a->qkv || !a->q_norm_weight || !a->k_norm_weight || !a->cos || !a->sin || !a->q_out || !a->k_out ||
        !a->v_out)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    QkParams p;
    p.qkv = (const __half*)a->qkv;
    p.qkv_b = a->qkv_b_stride;
    p.qkv_t = a->qkv_t_stride;
    p.q_norm_w = (const __half*)a->q_norm_weight;
    p.k_norm_w = (const __half*)a->k_norm_weight;
    p.cos = (const __half*)a->cos;
    p.sin = (const __half*)a->sin;
    p.rope_len = a->rope_len;
    p.q_out = (__half*)a->q_out;
    p.k_out = (__half*)a->k_out;
    p.k_pre = (__half*)a->k_pre;
    p.v_out = (__half*)a->v_out;
    p.qo_b = a->q_b_stride;
    p.qo_h = a->q_h_stride;
    p.ko_b = a->kv_b_stride;
    p.ko_h = a->kv_h_stride;
    p.q_heads = int(a->q_heads);
    p.kv_heads = int(a->kv_heads);
    p.n = int(a->n);
    p.pos0 = a->pos0;
    p.eps = float(a->eps);
    const dim3 grid(unsigned(a->n), unsigned(a->q_heads + 2 * a->kv_heads), unsigned(a->batch));
    const cudaError_t err = launch(qk_prefill_kernel, grid, dim3(D), 0, (cudaStream_t)stream, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_qk_prefill: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}
