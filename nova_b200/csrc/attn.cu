// Fused GQA decode attention over the streaming int8 KV cache (sm_100a).
//
// One CTA = (split, kv head, batch row).  Splits 0..n_splits-1 cover `chunk`
// tokens of the int8 prefix each; split n_splits (when the fp16 tail ring is
// given) covers the 64-slot ring.  Four warps per CTA; each warp owns one
// 18 KiB shared-memory stage and walks the 64-token scale groups of its split
// with stride 4:
//   * the elected lane issues one mbarrier-tracked TMA tile load for the K
//     codes and one for the V codes (64 rows x 128 B, 128-byte swizzle, so the
//     fragment reads below are bank-conflict free) plus four 256-byte bulk
//     copies for the group's fp16 min/step vectors;
//   * codes are turned into fp16 in registers (byte permute with the 0x64
//     exponent, subtract 1024, then one f16x2 FMA q*step+min -- the same value
//     the reference's fp32 multiply-add rounded to fp16 produces);
//   * S^T = K Q^T and O^T += V^T P^T run on mma.sync m16n8k16 (fp16 in, fp32
//     accumulate).  The 8 MMA columns carry the 4 query heads twice: for QK
//     both copies hold q (products are exact in fp32), for PV they hold the
//     fp16 high and low parts of each softmax weight, so P keeps ~22 bits;
//   * online softmax in fp32 (exp2 domain) with warp-shuffle max reductions.
// The four warps merge in shared memory, the CTA stores one partial
// (m, l, acc[128]) per query head, and the last CTA of each (batch, kv head)
// -- found with an arrival counter -- merges all partials, writes fp16 out and
// the fp32 log-sum-exp, and re-arms the counter.
//
// Reference semantics: src/nova/kvattn.py:110-253 (partial + combine kernels),
// :447-482 + :819-862 (fp16 tail ring and LSE merge), src/nova/decode.py:207-220
// (window mask).
#include <algorithm>

#include "common.cuh"
#include "qk_common.cuh"

namespace nova {
namespace attn {

constexpr int D = 128;
constexpr int GT = 64;
constexpr int NW = 4;
constexpr int THREADS = NW * 32;
constexpr int STAGE = 18432;      // K 8192 + V 8192 + 4 x 256 scales, rounded to 1 KiB
constexpr int SC_OFF = 16384;     // kst, kmn, vst, vmn (256 B each)
constexpr int TX_BYTES = 8192 + 8192 + 4 * 256;
constexpr int TX_HALF = 8192 + 2 * 256;   // the K half (codes + kst, kmn) or the V half of a group
constexpr int SMEM_BYTES = NW * STAGE + 1024;
constexpr int PART = 132;         // floats per (split, head): m, l, pad, pad, acc[128]
constexpr int MAX_GQ = 4;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct Params {
    const __half* q;
    int64_t q_b, q_h;
    const __half* kmn;
    const __half* kst;
    const __half* vmn;
    const __half* vst;
    const __half* tail_k;
    const __half* tail_v;
    __half* out;
    int64_t o_b, o_h;
    float* lse;
    int64_t lse_b;
    const uint8_t* kq;        // code rows (L2 prefetch only; the loads go through the tensor maps)
    const uint8_t* vq;
    const int64_t* qlen;
    const int64_t* pg;
    const int64_t* written;
    const int64_t* first;
    int* err;
    unsigned* counters;
    float* part;
    int kv_heads, gq, max_len, groups, chunk, n_splits, s_total, window;
    int prefetch_first;       // one-wave launches: each warp's first group is prefetched into L2 before the wait
    int defer_merge;          // FUSED: leave the split partials to the next kernel (no counters, no merge, no out)
    int win_rel;              // window > 0: split s covers [base + s*chunk, ...), base = the window's first group
    float scale_log2;
    // Fused q/k norm + RoPE + ring append (the FUSED kernel only; the
    // standalone kernel's job, src/nova/layers.py:24-36 + kvattn.py append):
    // q comes from the raw q|k|v row instead of `q`, the lengths from `pos`.
    const __half* qkv;        // fp16 [batch, (q_heads + 2 kv_heads) * 128]
    int64_t qkv_b;
    const __half* q_norm_w;
    const __half* k_norm_w;
    const __half* cos;
    const __half* sin;
    int64_t rope_len;
    const int64_t* pos;
    int64_t* written_out;
    int64_t* qlen_out;
    int64_t* pg_out;
    __half* ring_k;           // the tail ring and int8 cache above, writable
    __half* ring_v;
    uint8_t* kq_w;
    uint8_t* vq_w;
    __half* kmn_w;
    __half* kst_w;
    __half* vmn_w;
    __half* vst_w;
    float eps;
};

__device__ __forceinline__ float warp_max_g(float v) {  // across the 8 lanes sharing lane&3
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
    return v;
}
__device__ __forceinline__ float warp_sum_g(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    return v;
}

// fp16 high part (e == 0) or low part (e == 1) of a softmax weight.
__device__ __forceinline__ __half split_part(float p, int e) {
    __half hi = __float2half_rn(p);
    return e ? __float2half_rn(p - __half2float(hi)) : hi;
}

// P^T B-fragment for one 16-token tile: this lane (g, t) supplies column g =
// (head g>>1, part g&1) for tokens 2t, 2t+1 (b0) and 2t+8, 2t+9 (b1).  The
// weights live in lane (token&7)*4 + head as p_lo (token < 8) / p_hi (>= 8).
__device__ __forceinline__ void p_fragment(float p_lo, float p_hi, int g, int t, uint32_t& b0, uint32_t& b1) {
    const int h = g >> 1, e = g & 1;
    const int la = (2 * t) * 4 + h, lb = (2 * t + 1) * 4 + h;
    const float a0 = __shfl_sync(0xffffffffu, p_lo, la);
    const float a1 = __shfl_sync(0xffffffffu, p_lo, lb);
    const float a2 = __shfl_sync(0xffffffffu, p_hi, la);
    const float a3 = __shfl_sync(0xffffffffu, p_hi, lb);
    __half2 x0 = __halves2half2(split_part(a0, e), split_part(a1, e));
    __half2 x1 = __halves2half2(split_part(a2, e), split_part(a3, e));
    b0 = *reinterpret_cast<uint32_t*>(&x0);
    b1 = *reinterpret_cast<uint32_t*>(&x1);
}

// Online-softmax update for `n` scores (already in the log2 domain, -inf for
// masked tokens).  m_run is uniform over lanes with the same t (= head).
template <int N>
__device__ __forceinline__ void softmax_update(float (&x)[N], float& m_run, float& l_run, float (&acc)[8][4]) {
    float mloc = x[0];
#pragma unroll
    for (int i = 1; i < N; ++i) mloc = fmaxf(mloc, x[i]);
    mloc = warp_max_g(mloc);
    const float m_new = fmaxf(m_run, mloc);
    if (m_new == -INFINITY) {  // nothing valid yet for this head
#pragma unroll
        for (int i = 0; i < N; ++i) x[i] = 0.0f;
        return;
    }
    const float alpha = exp2f(m_run - m_new);  // m_run == -inf -> 0
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        x[i] = exp2f(x[i] - m_new);
        sum += x[i];
    }
    l_run = l_run * alpha + sum;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[j][c] *= alpha;
    m_run = m_new;
}

// Issue the loads of scale group `grp` of head row `bh` into `stage`: the K
// half (codes at 0, kst and kmn at SC_OFF) completes on bar_k, the V half
// (codes at 8192, vst and vmn at SC_OFF + 512) on bar_v, so that the next
// group's K can load while this group's V is still being read and vice versa.
__device__ __forceinline__ void issue_k(const Params& p, const CUtensorMap* tmK, uint8_t* stage, uint64_t* bar_k,
                                        int64_t bh, int grp) {
    mbar_arrive_expect_tx(bar_k, TX_HALF);
    tma_load_2d(stage, tmK, 0, int(bh * p.max_len + int64_t(grp) * GT), bar_k);
    const int64_t so = (bh * p.groups + grp) * D;
    bulk_g2s(stage + SC_OFF, p.kst + so, 256, bar_k);
    bulk_g2s(stage + SC_OFF + 256, p.kmn + so, 256, bar_k);
}
__device__ __forceinline__ void issue_v(const Params& p, const CUtensorMap* tmV, uint8_t* stage, uint64_t* bar_v,
                                        int64_t bh, int grp) {
    mbar_arrive_expect_tx(bar_v, TX_HALF);
    tma_load_2d(stage + 8192, tmV, 0, int(bh * p.max_len + int64_t(grp) * GT), bar_v);
    const int64_t so = (bh * p.groups + grp) * D;
    bulk_g2s(stage + SC_OFF + 512, p.vst + so, 256, bar_v);
    bulk_g2s(stage + SC_OFF + 768, p.vmn + so, 256, bar_v);
}

// L2 prefetch of scale group `grp` of head row `bh` (K and V code rows, the
// four scale vectors).  A hint, safe before the dependency wait: L2 is the
// point of coherence, so a later write to these lines is what a later load
// sees.  One lane.
__device__ __forceinline__ void prefetch_group_l2(const Params& p, int64_t bh, int grp) {
    const int64_t row = bh * p.max_len + int64_t(grp) * GT;
    const uint32_t bytes = uint32_t(min(GT, p.max_len - grp * GT)) * D;   // ragged last group
    const int64_t so = (bh * p.groups + grp) * D;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.kq + row * D), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.vq + row * D), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(p.kst + so) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(p.kmn + so) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(p.vst + so) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(p.vmn + so) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr) : "memory");
}

// One 64-token int8 group held in `stage`; tokens outside [lo, hi) are
// masked.  qk_part: scores from the K half and the online-softmax update
// (x = the group's probabilities); pv_part: O^T += V^T P^T from the V half.
__device__ __forceinline__ void qk_part(const uint8_t* stage, int gbase, int lo, int hi, const uint32_t (&qf)[16],
                                        float scale_log2, float (&acc)[8][4], float& m_run, float& l_run, int g,
                                        int t, float (&x)[8]) {
    const uint8_t* Ks = stage;
    const uint8_t* sc = stage + SC_OFF;
    // K scales for dims 32t..32t+31 (word w = dims 32t+2w, +1).
    uint32_t kst2[16], kmn2[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 a = lds128(sc + 64 * t + 16 * i);
        uint4 b = lds128(sc + 256 + 64 * t + 16 * i);
        kst2[4 * i] = a.x; kst2[4 * i + 1] = a.y; kst2[4 * i + 2] = a.z; kst2[4 * i + 3] = a.w;
        kmn2[4 * i] = b.x; kmn2[4 * i + 1] = b.y; kmn2[4 * i + 2] = b.z; kmn2[4 * i + 3] = b.w;
    }

    // ---- scores for the 4 tiles of 16 tokens
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r0 = 16 * i + g;
        const uint4 k0a = lds128(Ks + r0 * 128 + (((2 * t) ^ g) << 4));
        const uint4 k0b = lds128(Ks + r0 * 128 + (((2 * t + 1) ^ g) << 4));
        const uint4 k1a = lds128(Ks + (r0 + 8) * 128 + (((2 * t) ^ g) << 4));
        const uint4 k1b = lds128(Ks + (r0 + 8) * 128 + (((2 * t + 1) ^ g) << 4));
        const uint32_t w0[8] = {k0a.x, k0a.y, k0a.z, k0a.w, k0b.x, k0b.y, k0b.z, k0b.w};
        const uint32_t w1[8] = {k1a.x, k1a.y, k1a.z, k1a.w, k1b.x, k1b.y, k1b.z, k1b.w};
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t a0 = hfma2(u8x2_lo_to_f16x2(w0[s]), kst2[2 * s], kmn2[2 * s]);
            const uint32_t a2 = hfma2(u8x2_hi_to_f16x2(w0[s]), kst2[2 * s + 1], kmn2[2 * s + 1]);
            const uint32_t a1 = hfma2(u8x2_lo_to_f16x2(w1[s]), kst2[2 * s], kmn2[2 * s]);
            const uint32_t a3 = hfma2(u8x2_hi_to_f16x2(w1[s]), kst2[2 * s + 1], kmn2[2 * s + 1]);
            mma_16816(c, a0, a1, a2, a3, qf[2 * s], qf[2 * s + 1]);
        }
        const int p0 = gbase + r0, p1 = p0 + 8;
        x[2 * i] = (p0 >= lo && p0 < hi) ? c[0] * scale_log2 : -INFINITY;
        x[2 * i + 1] = (p1 >= lo && p1 < hi) ? c[2] * scale_log2 : -INFINITY;
    }
    softmax_update<8>(x, m_run, l_run, acc);
}

__device__ __forceinline__ void pv_part(const uint8_t* stage, const float (&x)[8], float (&acc)[8][4], int g, int t) {
    const uint8_t* Vs = stage + 8192;
    const uint8_t* sc = stage + SC_OFF;
    // V scales for dims 16g..16g+15, broadcast to both halves:
    // index j -> dim 16g+2j (row g of m-tile j), dim 16g+2j+1 (row g+8).
    uint32_t vsA[8], vsB[8], vmA[8], vmB[8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        uint4 a = lds128(sc + 512 + 32 * g + 16 * i);
        uint4 b = lds128(sc + 768 + 32 * g + 16 * i);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int j = 4 * i + k;
            vsA[j] = __byte_perm(aw[k], 0, 0x1010);
            vsB[j] = __byte_perm(aw[k], 0, 0x3232);
            vmA[j] = __byte_perm(bw[k], 0, 0x1010);
            vmB[j] = __byte_perm(bw[k], 0, 0x3232);
        }
    }

    // ---- O^T += V^T P^T, one 16-token tile at a time
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t b0, b1;
        p_fragment(x[2 * i], x[2 * i + 1], g, t, b0, b1);
        const int ta = 16 * i + 2 * t;
        const uint4 vA = lds128(Vs + ta * 128 + ((g ^ (ta & 7)) << 4));
        const uint4 vB = lds128(Vs + (ta + 1) * 128 + ((g ^ ((ta + 1) & 7)) << 4));
        const uint4 vC = lds128(Vs + (ta + 8) * 128 + ((g ^ (ta & 7)) << 4));
        const uint4 vD = lds128(Vs + (ta + 9) * 128 + ((g ^ ((ta + 1) & 7)) << 4));
        const uint32_t wa[4] = {vA.x, vA.y, vA.z, vA.w}, wb[4] = {vB.x, vB.y, vB.z, vB.w};
        const uint32_t wc[4] = {vC.x, vC.y, vC.z, vC.w}, wd[4] = {vD.x, vD.y, vD.z, vD.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            const uint32_t ab01 = __byte_perm(wa[wi], wb[wi], 0x5140);
            const uint32_t ab23 = __byte_perm(wa[wi], wb[wi], 0x7362);
            const uint32_t cd01 = __byte_perm(wc[wi], wd[wi], 0x5140);
            const uint32_t cd23 = __byte_perm(wc[wi], wd[wi], 0x7362);
            int j = 2 * wi;
            mma_16816(acc[j], hfma2(u8x2_lo_to_f16x2(ab01), vsA[j], vmA[j]),
                      hfma2(u8x2_hi_to_f16x2(ab01), vsB[j], vmB[j]), hfma2(u8x2_lo_to_f16x2(cd01), vsA[j], vmA[j]),
                      hfma2(u8x2_hi_to_f16x2(cd01), vsB[j], vmB[j]), b0, b1);
            j = 2 * wi + 1;
            mma_16816(acc[j], hfma2(u8x2_lo_to_f16x2(ab23), vsA[j], vmA[j]),
                      hfma2(u8x2_hi_to_f16x2(ab23), vsB[j], vmB[j]), hfma2(u8x2_lo_to_f16x2(cd23), vsA[j], vmA[j]),
                      hfma2(u8x2_hi_to_f16x2(cd23), vsB[j], vmB[j]), b0, b1);
        }
    }
}

__device__ __forceinline__ void process_group(const uint8_t* stage, int gbase, int lo, int hi,
                                              const uint32_t (&qf)[16], float scale_log2, float (&acc)[8][4],
                                              float& m_run, float& l_run, int g, int t) {
    float x[8];
    qk_part(stage, gbase, lo, hi, qf, scale_log2, acc, m_run, l_run, g, t, x);
    pv_part(stage, x, acc, g, t);
}

__device__ __forceinline__ int64_t pos_mod(int64_t a, int m) {
    int64_t r = a % m;
    return r < 0 ? r + m : r;
}

// The 16 ring slots [16w, 16w+16) of the fp16 tail, read straight from global.
__device__ __forceinline__ void process_tail_tile(const Params& p, int64_t bh, int w, int64_t u, int64_t tlo,
                                                  const uint32_t (&qf)[16], float (&acc)[8][4], float& m_run,
                                                  float& l_run, int g, int t) {
    const __half* tk = p.tail_k + bh * GT * D;
    const __half* tv = p.tail_v + bh * GT * D;
    auto slot_valid = [&](int i) -> bool {
        if (u < 0) return false;
        const int64_t pos = u - pos_mod(u - i, GT);
        return pos >= tlo && pos <= u;
    };
    const int r0 = 16 * w + g, r1 = r0 + 8;
    uint32_t k0[16], k1[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 a = *reinterpret_cast<const uint4*>(tk + r0 * D + 32 * t + 8 * i);
        const uint4 b = *reinterpret_cast<const uint4*>(tk + r1 * D + 32 * t + 8 * i);
        k0[4 * i] = a.x; k0[4 * i + 1] = a.y; k0[4 * i + 2] = a.z; k0[4 * i + 3] = a.w;
        k1[4 * i] = b.x; k1[4 * i + 1] = b.y; k1[4 * i + 2] = b.z; k1[4 * i + 3] = b.w;
    }
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; ++s) mma_16816(c, k0[2 * s], k1[2 * s], k0[2 * s + 1], k1[2 * s + 1], qf[2 * s], qf[2 * s + 1]);
    float x[2];
    x[0] = slot_valid(r0) ? c[0] * p.scale_log2 : -INFINITY;
    x[1] = slot_valid(r1) ? c[2] * p.scale_log2 : -INFINITY;
    softmax_update<2>(x, m_run, l_run, acc);

    uint32_t b0, b1;
    p_fragment(x[0], x[1], g, t, b0, b1);
    const int ta = 16 * w + 2 * t;
    const int tok[4] = {ta, ta + 1, ta + 8, ta + 9};
    uint32_t v[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool ok = slot_valid(tok[k]);
        const uint4 a = *reinterpret_cast<const uint4*>(tv + tok[k] * D + 16 * g);
        const uint4 b = *reinterpret_cast<const uint4*>(tv + tok[k] * D + 16 * g + 8);
        v[k][0] = ok ? a.x : 0u; v[k][1] = ok ? a.y : 0u; v[k][2] = ok ? a.z : 0u; v[k][3] = ok ? a.w : 0u;
        v[k][4] = ok ? b.x : 0u; v[k][5] = ok ? b.y : 0u; v[k][6] = ok ? b.z : 0u; v[k][7] = ok ? b.w : 0u;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        mma_16816(acc[j], __byte_perm(v[0][j], v[1][j], 0x5410), __byte_perm(v[0][j], v[1][j], 0x7632),
                  __byte_perm(v[2][j], v[3][j], 0x5410), __byte_perm(v[2][j], v[3][j], 0x7632), b0, b1);
    }
}

// FUSED: the q/k norm + RoPE + ring append of this step runs in the
// prologue.  Every CTA normalises and rotates its q heads; the ring CTA of
// each (batch row, KV head) also does K, writes the ring slot and, when the
// slot completes a group, requantizes the group into the int8 cache and
// attends it from its own shared memory (the prefix splits stop before it,
// so no CTA reads a group while it is written).
template <bool FUSED>
__global__ void __launch_bounds__(THREADS, 3)
    attn_decode_int8_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[2][NW];   // per warp: K half, V half of its stage
    __shared__ float sm_m[NW][MAX_GQ], sm_l[NW][MAX_GQ];
    __shared__ int sm_last;

    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int64_t bh = int64_t(b) * p.kv_heads + h;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool is_tail = split == p.n_splits;
    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
    }
    // Split size.  The host's chunk covers the whole capacity with the launched splits; the fused decode
    // step (absolute splits) uses the smallest multiple of one group per warp that covers the current
    // prefix instead, at most that chunk, so a cache filled far below its capacity still gives every
    // warp one group per split rather than several in a row.
    auto chunk_for = [&](int64_t pend_) -> int64_t {
        if (!FUSED || p.win_rel) return p.chunk;
        const int64_t step = int64_t(GT) * NW;
        int64_t c = (max(pend_, int64_t(1)) + p.n_splits - 1) / p.n_splits;
        c = (c + step - 1) / step * step;
        return c < p.chunk ? c : int64_t(p.chunk);
    };
    int64_t chunk = p.chunk;
    // The group this warp takes first when no prefix is masked (every group
    // of the chunk lies inside the cache allocation, so a copy is in bounds).
    int spec = 0;
    bool spec_on = false;
    auto set_spec = [&]() {
        spec = int(int64_t(split) * chunk / GT) + warp;
        spec_on = !p.win_rel && split < p.n_splits && spec < p.groups &&
                  int64_t(spec) * GT < int64_t(split) * chunk + chunk;
    };
    if (!FUSED) set_spec();
    __half nwq = __float2half_rn(0.f), nwk = __float2half_rn(0.f);
    uint8_t* stage = smem + warp * STAGE;
    uint64_t* bar_k = &bars[0][warp];
    uint64_t* bar_v = &bars[1][warp];
    // Speculative first load of this warp's group (in bounds whatever the lengths turn out to be).
    auto spec_issue = [&]() {
        if (lane == 0) {
            mbar_init(bar_k, 1);
            mbar_init(bar_v, 1);
            fence_mbar_init();
            if (spec_on) {
                issue_k(p, &tmK, stage, bar_k, bh, spec);
                issue_v(p, &tmV, stage, bar_v, bh, spec);
            }
        }
        __syncwarp();
    };
    int64_t pos_hint = -1;
    float cos_hint = 0.f, sin_hint = 0.f;
    if (FUSED) {
        // Before the dependency wait: the norm weights and the RoPE row of the
        // position the previous step left (a hint, checked after the wait), and
        // the first group of the int8 prefix -- the q|k|v projection launched
        // just before does not write the cache, and the group this step
        // completes is never read by a prefix split.
        nwq = p.q_norm_w[threadIdx.x];
        if (is_tail) nwk = p.k_norm_w[threadIdx.x];
        pos_hint = *reinterpret_cast<const volatile int64_t*>(p.pos);
        {   // the prefix this step will attend if the position is still pos_hint
            const int64_t ql = (pos_hint + 1) / GT * GT;
            const bool rq = pos_hint >= 0 && pos_hint < p.max_len && pos_hint % GT == GT - 1;
            chunk = chunk_for(min(rq ? ql - GT : ql, int64_t(p.max_len)));
            set_spec();
        }
        const int64_t cp = pos_hint < 0 ? 0 : (pos_hint < p.rope_len ? pos_hint : p.rope_len - 1);
        cos_hint = __half2float(p.cos[cp * D + threadIdx.x]);
        sin_hint = __half2float(p.sin[cp * D + threadIdx.x]);
        spec_issue();
    }
    if (threadIdx.x == 64 && p.first) prefetch_l2(p.first);
    if (!FUSED && p.prefetch_first && spec_on && lane == 0) prefetch_group_l2(p, bh, spec);
    pdl_trigger();
    pdl_wait();   // q, the cache and the lengths come from the previous kernels

    // FUSED: this CTA's raw q (and, for the ring CTA, k and v) channel, requested first
    __half xq[MAX_GQ], xk[1] = {__float2half_rn(0.f)}, xv = __float2half_rn(0.f);
    if (FUSED) {
        const __half* row = p.qkv + b * p.qkv_b;
        const int hq_all = p.kv_heads * p.gq;
#pragma unroll
        for (int hh = 0; hh < MAX_GQ; ++hh)
            xq[hh] = hh < p.gq ? row[int64_t(h * p.gq + hh) * D + threadIdx.x] : __float2half_rn(0.f);
        if (is_tail) {
            xk[0] = row[int64_t(hq_all + h) * D + threadIdx.x];
            xv = row[int64_t(hq_all + p.kv_heads + h) * D + threadIdx.x];
        }
    } else {
        spec_issue();
    }
    uint32_t phase_k = 0, phase_v = 0;   // completed waits on bar_k / bar_v
    bool pend_k = spec_on, pend_v = spec_on;   // a copy is in flight on bar_k / bar_v

    int64_t qlen, pgv, written, pos = 0;
    bool requant = false;   // FUSED: this step's token completes group pos / 64
    if (FUSED) {
        pos = *p.pos;
        written = pos + 1;
        qlen = (written / GT) * GT;
        pgv = qlen / GT;
        requant = pos >= 0 && pos < p.max_len && pos % GT == GT - 1;
    } else {
        qlen = *p.qlen;
        pgv = *p.pg;
        written = p.written ? *p.written : qlen;
    }
    const int64_t first = p.first ? *p.first : 0;
    const int64_t u = written - 1;
    int64_t lo = first > 0 ? first : 0;
    if (p.window > 0) lo = max(lo, u - p.window + 1);
    const int64_t pend = min(min(requant ? qlen - GT : qlen, pgv * GT), int64_t(p.max_len));
    chunk = chunk_for(pend);   // FUSED: from the real position (a different spec group is drained and reloaded)

    // Q^T B-fragments: column g carries head g>>1; dims 32t..32t+31.
    uint32_t qf[16];
    if (FUSED) {
        // scratch in the last KiB of stages 0-2, which no group copy writes
        // (TX_BYTES of each stage are used); no longer needed once qf is built
        auto qemb = reinterpret_cast<__half(*)[D]>(smem + TX_BYTES);                // [MAX_GQ][D]
        auto qbuf = reinterpret_cast<__half(*)[D]>(smem + STAGE + TX_BYTES);        // [MAX_GQ][D]
        auto qred = reinterpret_cast<float(*)[MAX_GQ]>(smem + 2 * STAGE + TX_BYTES);  // [NW][MAX_GQ]
        auto kred = reinterpret_cast<float(*)[1]>(smem + 2 * STAGE + TX_BYTES + 64);  // [NW][1]
        auto kbuf = reinterpret_cast<__half(*)[D]>(smem + 2 * STAGE + TX_BYTES + 128);  // [1][D]
        static_assert(TX_BYTES % 16 == 0 && STAGE - TX_BYTES >= MAX_GQ * D * 2 && 128 + D * 2 <= STAGE - TX_BYTES,
                      "prologue scratch must fit in the unused stage tails");
        const int d = threadIdx.x;
        float c = cos_hint, sn = sin_hint;
        if (pos != pos_hint) {   // the position moved since the hint: the RoPE row of the real one
            const int64_t cp = pos < 0 ? 0 : (pos < p.rope_len ? pos : p.rope_len - 1);
            c = __half2float(p.cos[cp * D + d]);
            sn = __half2float(p.sin[cp * D + d]);
        }
        __half eq[MAX_GQ];
        qk::norm_rope<MAX_GQ>(xq, nwq, c, sn, p.eps, qred, qbuf, eq);
#pragma unroll
        for (int hh = 0; hh < MAX_GQ; ++hh) qemb[hh][d] = eq[hh];
        if (is_tail) {   // uniform per CTA: norm_rope synchronises the CTA
            __half ek[1];
            qk::norm_rope<1>(xk, nwk, c, sn, p.eps, kred, kbuf, ek);
            if (b == 0 && h == 0 && d == 0) {   // the lengths, for later readers (nothing in this launch reads them)
                *p.written_out = written;
                *p.qlen_out = qlen;
                *p.pg_out = pgv;
            }
            if (pos >= 0 && pos < p.max_len) {
                const int slot = int(pos % GT);
                __half* tk = p.ring_k + bh * GT * D;
                __half* tv = p.ring_v + bh * GT * D;
                tk[slot * D + d] = ek[0];
                tv[slot * D + d] = xv;
                if (requant) {   // the group into the cache, and into stage 0 the way a TMA copy lays it out
                    const int64_t gidx = pos / GT;
                    const int64_t code_off = bh * p.max_len * D + gidx * GT * D + d;
                    const int64_t sc_off = (bh * p.groups + gidx) * D + d;
                    uint8_t* st = smem;
                    auto at = [d](int tt) { return tt * 128 + ((((d >> 4) ^ (tt & 7))) << 4) + (d & 15); };
                    qk::quant_col(tk + d, p.kmn_w + sc_off, p.kst_w + sc_off, [&](int tt, uint8_t c8) {
                        p.kq_w[code_off + int64_t(tt) * D] = c8;
                        st[at(tt)] = c8;
                    });
                    qk::quant_col(tv + d, p.vmn_w + sc_off, p.vst_w + sc_off, [&](int tt, uint8_t c8) {
                        p.vq_w[code_off + int64_t(tt) * D] = c8;
                        st[8192 + at(tt)] = c8;
                    });
                    __half* scs = reinterpret_cast<__half*>(smem + SC_OFF);   // kst, kmn, vst, vmn
                    scs[d] = p.kst_w[sc_off];
                    scs[D + d] = p.kmn_w[sc_off];
                    scs[2 * D + d] = p.vst_w[sc_off];
                    scs[3 * D + d] = p.vmn_w[sc_off];
                }
            }
        }
        __syncthreads();   // qemb, the ring slot and stage 0 are complete
        const int hq = g >> 1;
        if (hq < p.gq) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 v = *reinterpret_cast<const uint4*>(&qemb[hq][32 * t + 8 * i]);
                qf[4 * i] = v.x; qf[4 * i + 1] = v.y; qf[4 * i + 2] = v.z; qf[4 * i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) qf[i] = 0u;
        }
    } else {
        const int hq = g >> 1;
        if (hq < p.gq) {
            const __half* qp = p.q + b * p.q_b + int64_t(h * p.gq + hq) * p.q_h + 32 * t;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 v = *reinterpret_cast<const uint4*>(qp + 8 * i);
                qf[4 * i] = v.x; qf[4 * i + 1] = v.y; qf[4 * i + 2] = v.z; qf[4 * i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) qf[i] = 0u;
        }
    }

    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    if (split < p.n_splits) {
        // window-relative splits start at the window's first group (known only after the lengths are read)
        const int64_t s0 = (p.win_rel ? lo / GT * GT : int64_t(0)) + int64_t(split) * chunk;
        const int64_t t_begin = max(s0, lo);
        const int64_t t_end = min(s0 + chunk, pend);
        if (t_begin < t_end) {
            const int g_first = int(t_begin / GT), g_last = int((t_end - 1) / GT);
            int gi = g_first + warp;
            if (gi <= g_last) {
                if (!(pend_k && spec == gi)) {   // masked prefix: drain the speculative copy, load gi
                    if (pend_k) {
                        mbar_wait(bar_k, phase_k & 1u, p.err, 1);
                        ++phase_k;
                        mbar_wait(bar_v, phase_v & 1u, p.err, 1);
                        ++phase_v;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        fence_proxy_async();
                        issue_k(p, &tmK, stage, bar_k, bh, gi);
                        issue_v(p, &tmV, stage, bar_v, bh, gi);
                    }
                    pend_k = pend_v = true;
                }
                // K of the next group loads during this group's PV, its V during the next QK
                for (; gi <= g_last; gi += NW) {
                    if (!mbar_wait(bar_k, phase_k & 1u, p.err, 1)) break;
                    ++phase_k;
                    pend_k = false;
                    float x[8];
                    qk_part(stage, gi * GT, int(t_begin), int(t_end), qf, p.scale_log2, acc, m_run, l_run, g, t, x);
                    __syncwarp();
                    const bool more = gi + NW <= g_last;
                    if (more) {
                        if (lane == 0) {
                            fence_proxy_async();
                            issue_k(p, &tmK, stage, bar_k, bh, gi + NW);
                        }
                        pend_k = true;
                    }
                    if (!mbar_wait(bar_v, phase_v & 1u, p.err, 1)) break;
                    ++phase_v;
                    pend_v = false;
                    pv_part(stage, x, acc, g, t);
                    __syncwarp();
                    if (more) {
                        if (lane == 0) {
                            fence_proxy_async();
                            issue_v(p, &tmV, stage, bar_v, bh, gi + NW);
                        }
                        pend_v = true;
                    }
                    __syncwarp();
                }
            }
        }
        // a copy nobody used must land before exit
        if (pend_k) mbar_wait(bar_k, phase_k & 1u, p.err, 1);
        if (pend_v) mbar_wait(bar_v, phase_v & 1u, p.err, 1);
    } else {
        int64_t tlo = max(lo, qlen);
        process_tail_tile(p, bh, warp, u, tlo, qf, acc, m_run, l_run, g, t);
        if (FUSED && requant && warp == 0)   // the group this step completed, from stage 0
            process_group(smem, int(qlen - GT), int(max(lo, qlen - GT)), int(qlen), qf, p.scale_log2, acc, m_run,
                          l_run, g, t);
    }

    // ---- merge the 4 warps of this CTA
    const float l_warp = warp_sum_g(l_run);
    __syncthreads();  // every warp is done with its stage: reuse it as obuf
    float* obuf = reinterpret_cast<float*>(smem);  // [NW][MAX_GQ][D]
    if (t < p.gq) {
        if (g == 0) {
            sm_m[warp][t] = m_run;
            sm_l[warp][t] = l_warp;
        }
        float* ob = obuf + (warp * MAX_GQ + t) * D + 16 * g;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            ob[2 * j] = acc[j][0] + acc[j][1];
            ob[2 * j + 1] = acc[j][2] + acc[j][3];
        }
    }
    __syncthreads();
    const int hh = threadIdx.x >> 5, d0 = (threadIdx.x & 31) * 4;
    float* part_bh = p.part + bh * int64_t(p.s_total) * p.gq * PART;
    if (hh < p.gq) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][hh]);
        float L = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float mw = sm_m[w][hh];
                if (mw == -INFINITY) continue;
                const float wt = exp2f(mw - M);
                L += wt * sm_l[w][hh];
                const float4 a = *reinterpret_cast<const float4*>(obuf + (w * MAX_GQ + hh) * D + d0);
                o.x += wt * a.x; o.y += wt * a.y; o.z += wt * a.z; o.w += wt * a.w;
            }
        }
        float* dst = part_bh + (int64_t(split) * p.gq + hh) * PART;
        if (d0 == 0) {
            dst[0] = M;
            dst[1] = L;
        }
        if (M != -INFINITY) *reinterpret_cast<float4*>(dst + 4 + d0) = o;
    }
    if (FUSED && p.defer_merge) return;   // complete for the next kernel once this launch has finished
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(p.counters + bh, 1u);
        sm_last = (prev == unsigned(p.s_total - 1));
    }
    __syncthreads();
    if (!sm_last) return;
    __threadfence();

    // ---- last CTA of this (batch, kv head): merge all splits.  When the
    // partials of the head fit in the (now idle) stage memory, one bulk copy
    // brings them all in and warp hh merges its head from shared memory:
    // weights from the split maxima, then the accumulators in split order.
    // Otherwise the partials are read from global memory split by split.
    const int64_t part_bytes = int64_t(p.s_total) * p.gq * PART * 4;
    const bool staged = part_bytes <= NW * STAGE;
    const float* src_base = part_bh;
    if (staged) {
        __shared__ __align__(8) uint64_t bar_comb;
        if (threadIdx.x == 0) {
            mbar_init(&bar_comb, 1);
            fence_mbar_init();
            asm volatile("fence.proxy.async.global;" ::: "memory");   // the partials were written by other CTAs
            fence_proxy_async();   // and this CTA's merge buffer in the same shared memory was written generically
            mbar_arrive_expect_tx(&bar_comb, uint32_t(part_bytes));
            bulk_g2s(smem, part_bh, uint32_t(part_bytes), &bar_comb);
        }
        __syncthreads();
        mbar_wait(&bar_comb, 0u, p.err, 4);
        src_base = reinterpret_cast<const float*>(smem);
    } else {   // every (m, l) pair at once into shared memory (host checks s_total * gq <= 9216)
        float2* ml = reinterpret_cast<float2*>(smem);
        for (int i = threadIdx.x; i < p.s_total * p.gq; i += THREADS)
            ml[i] = __ldcg(reinterpret_cast<const float2*>(part_bh + int64_t(i) * PART));
        __syncthreads();
    }
    if (hh < p.gq) {
        float M = -INFINITY, L = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (staged) {
            float* sp = reinterpret_cast<float*>(smem);
            for (int s2 = lane; s2 < p.s_total; s2 += 32) M = fmaxf(M, sp[(s2 * p.gq + hh) * PART]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            if (M != -INFINITY) {
                for (int s2 = lane; s2 < p.s_total; s2 += 32) {
                    float* e = sp + (s2 * p.gq + hh) * PART;
                    e[2] = e[0] == -INFINITY ? 0.f : exp2f(e[0] - M);   // weight into the pad slot
                }
                __syncwarp();
                for (int s2 = 0; s2 < p.s_total; ++s2) {
                    const float* e = sp + (s2 * p.gq + hh) * PART;
                    const float wt = e[2];
                    if (wt == 0.f) continue;
                    L += wt * e[1];
                    const float4 a = *reinterpret_cast<const float4*>(e + 4 + d0);
                    o.x += wt * a.x; o.y += wt * a.y; o.z += wt * a.z; o.w += wt * a.w;
                }
            }
        } else {   // (m, l) pairs were fetched into shared memory above; accumulators 8 loads in flight
            const float2* ml = reinterpret_cast<const float2*>(smem);
            for (int s2 = lane; s2 < p.s_total; s2 += 32) M = fmaxf(M, ml[s2 * p.gq + hh].x);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            if (M != -INFINITY) {
                for (int s0 = 0; s0 < p.s_total; s0 += 8) {
                    float4 a[8];
                    float wt[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        wt[k] = 0.f;
                        if (s0 + k < p.s_total) {
                            const float2 v = ml[(s0 + k) * p.gq + hh];
                            if (v.x != -INFINITY) {
                                wt[k] = exp2f(v.x - M);
                                a[k] = __ldcg(reinterpret_cast<const float4*>(
                                    src_base + (int64_t(s0 + k) * p.gq + hh) * PART + 4 + d0));
                            }
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        if (wt[k] == 0.f) continue;
                        L += wt[k] * ml[(s0 + k) * p.gq + hh].y;
                        o.x += wt[k] * a[k].x; o.y += wt[k] * a[k].y; o.z += wt[k] * a[k].z; o.w += wt[k] * a[k].w;
                    }
                }
            }
        }
        const int qh = h * p.gq + hh;
        __half* op = p.out + b * p.o_b + int64_t(qh) * p.o_h + d0;
        if (L > 0.f) {  // acc / l then one rounding to fp16, like the reference combine
            *reinterpret_cast<__half2*>(op) = __floats2half2_rn(__fdiv_rn(o.x, L), __fdiv_rn(o.y, L));
            *reinterpret_cast<__half2*>(op + 2) = __floats2half2_rn(__fdiv_rn(o.z, L), __fdiv_rn(o.w, L));
        } else {
            *reinterpret_cast<__half2*>(op) = __floats2half2_rn(0.f, 0.f);
            *reinterpret_cast<__half2*>(op + 2) = __floats2half2_rn(0.f, 0.f);
        }
        if (p.lse && d0 == 0) p.lse[b * p.lse_b + qh] = (L > 0.f) ? (M + log2f(L)) * LN2 : -INFINITY;
    }
    if (threadIdx.x == 0) p.counters[bh] = 0u;
}

}  // namespace attn
}  // namespace nova

using namespace nova;

static int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

extern "C" int nova_attn_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t n_splits,
                                         int has_tail, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (batch <= 0 || kv_heads <= 0 || q_heads <= 0 || q_heads % kv_heads || n_splits < 0)
        return fail(NOVA_ERR_INVALID, "bad batch/heads/n_splits");
    const int64_t bh = batch * kv_heads;
    const int64_t s_total = n_splits + (has_tail ? 1 : 0);
    *bytes = 256 + align_up(bh * 4, 256) + bh * s_total * (q_heads / kv_heads) * attn::PART * 4;
    return NOVA_OK;
}

extern "C" int nova_attn_read_error(void* workspace, int64_t, int64_t, int* host_value) {
    if (!workspace || !host_value) return fail(NOVA_ERR_INVALID, "NULL argument");
    if (cudaMemcpy(host_value, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(NOVA_ERR_CUDA, "reading the attention error word failed");
    if (*host_value && cudaMemset(workspace, 0, sizeof(int)) != cudaSuccess)
        return fail(NOVA_ERR_CUDA, "clearing the attention error word failed");
    return NOVA_OK;
}

// Shared by nova_attn_decode_int8 (qk == nullptr) and
// nova_qk_append_attn_int8 (qk: the fused q/k norm + RoPE + append, checked
// by the caller against `a`).
static int attn_launch(const nova_attn_int8_args* a, const nova_qk_args* qk, void* stream) {
    using namespace nova::attn;
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->head_dim != D) return fail(NOVA_ERR_UNSUPPORTED, "head_dim must be 128, got %lld", (long long)a->head_dim);
    if (a->group != GT) return fail(NOVA_ERR_UNSUPPORTED, "group must be 64, got %lld", (long long)a->group);
    if (a->batch <= 0 || a->kv_heads <= 0 || a->q_heads <= 0 || a->q_heads % a->kv_heads)
        return fail(NOVA_ERR_INVALID, "bad batch/heads (%lld, %lld, %lld)", (long long)a->batch,
                    (long long)a->q_heads, (long long)a->kv_heads);
    const int64_t gq = a->q_heads / a->kv_heads;
    if (gq > MAX_GQ) return fail(NOVA_ERR_UNSUPPORTED, "q_heads/kv_heads must be <= 4, got %lld", (long long)gq);
    if (a->chunk <= 0 || a->chunk % GT) return fail(NOVA_ERR_INVALID, "chunk must be a positive multiple of 64");
    if (a->max_len <= 0 || a->groups != (a->max_len + GT - 1) / GT)
        return fail(NOVA_ERR_INVALID, "groups must equal ceil(max_len/64)");
    if (a->n_splits < 0 || (a->n_splits == 0 && !a->tail_k)) return fail(NOVA_ERR_INVALID, "n_splits must be >= 1");
    if (a->n_splits > 65535 || a->batch > 65535 || a->kv_heads > 65535)
        return fail(NOVA_ERR_INVALID, "grid too large");
    if ((a->n_splits + 1) * gq > NW * STAGE / 8)
        return fail(NOVA_ERR_UNSUPPORTED, "n_splits * q_heads/kv_heads must be at most %d", NW * STAGE / 8 - gq);
    if ((!qk && (!a->q || !a->qlen || !a->pg)) || !a->out || !a->workspace)
        return fail(NOVA_ERR_INVALID, "q/out/qlen/pg/workspace must not be NULL");
    if (a->n_splits && (!a->kq || !a->vq || !a->kmn || !a->kst || !a->vmn || !a->vst))
        return fail(NOVA_ERR_INVALID, "int8 buffers must not be NULL");
    if ((a->tail_k == nullptr) != (a->tail_v == nullptr)) return fail(NOVA_ERR_INVALID, "tail_k/tail_v: both or none");
    if (a->tail_k && !a->written) return fail(NOVA_ERR_INVALID, "the tail ring needs the `written` scalar");
    if (a->window < 0) return fail(NOVA_ERR_INVALID, "window must be >= 0");
    auto mis = [](const void* ptr, int al) { return ptr && (reinterpret_cast<uintptr_t>(ptr) % al); };
    if (mis(a->q, 16) || mis(a->out, 8) || mis(a->kq, 16) || mis(a->vq, 16) || mis(a->kmn, 16) ||
        mis(a->kst, 16) || mis(a->vmn, 16) || mis(a->vst, 16) || mis(a->tail_k, 16) || mis(a->tail_v, 16) ||
        mis(a->workspace, 256))
        return fail(NOVA_ERR_ALIGN, "q/kv/scale/tail pointers must be 16-byte aligned (out 8, workspace 256)");
    if ((a->q_h_stride % 8) || (a->q_b_stride % 8) || (a->o_h_stride % 4) || (a->o_b_stride % 4))
        return fail(NOVA_ERR_ALIGN, "q strides must be multiples of 8 elements, out strides of 4");
    const int64_t bh = a->batch * a->kv_heads;
    const int64_t s_total = a->n_splits + (a->tail_k ? 1 : 0);
    int64_t need = 0;
    nova_attn_workspace_bytes(a->batch, a->q_heads, a->kv_heads, a->n_splits, a->tail_k != nullptr, &need);
    if (a->workspace_bytes < need)
        return fail(NOVA_ERR_INVALID, "workspace too small: %lld < %lld bytes", (long long)a->workspace_bytes,
                    (long long)need);
    if (bh * a->max_len > 0x7fffffffLL) return fail(NOVA_ERR_INVALID, "batch*kv_heads*max_len must fit in int32");

    CUtensorMap tmK, tmV;
    const uint64_t rows = uint64_t(bh * a->max_len);
    if (a->n_splits) {
        if (int rc = make_tmap_u8_rows128(&tmK, a->kq, rows, GT)) return rc;
        if (int rc = make_tmap_u8_rows128(&tmV, a->vq, rows, GT)) return rc;
    } else {
        memset(&tmK, 0, sizeof(tmK));
        memset(&tmV, 0, sizeof(tmV));
    }

    Params p;
    p.q = (const __half*)a->q;
    p.q_b = a->q_b_stride;
    p.q_h = a->q_h_stride;
    p.kmn = (const __half*)a->kmn;
    p.kst = (const __half*)a->kst;
    p.vmn = (const __half*)a->vmn;
    p.vst = (const __half*)a->vst;
    p.tail_k = (const __half*)a->tail_k;
    p.tail_v = (const __half*)a->tail_v;
    p.out = (__half*)a->out;
    p.o_b = a->o_b_stride;
    p.o_h = a->o_h_stride;
    p.lse = (float*)a->lse;
    p.lse_b = a->lse_b_stride;
    p.qlen = a->qlen;
    p.pg = a->pg;
    p.written = a->written;
    p.first = a->first;
    uint8_t* ws = (uint8_t*)a->workspace;
    p.err = (int*)ws;
    p.counters = (unsigned*)(ws + 256);
    p.part = (float*)(ws + 256 + align_up(bh * 4, 256));
    p.kv_heads = int(a->kv_heads);
    p.gq = int(gq);
    p.max_len = int(a->max_len);
    p.groups = int(a->groups);
    p.chunk = int(a->chunk);
    p.n_splits = int(a->n_splits);
    p.s_total = int(s_total);
    p.defer_merge = (qk && a->defer_merge) ? 1 : 0;
    p.window = int(std::min<int64_t>(a->window, 0x7fffffff));
    p.scale_log2 = float(1.0 / sqrt(double(D))) * LOG2E;
    p.kq = (const uint8_t*)a->kq;
    p.vq = (const uint8_t*)a->vq;
    // every CTA resident at once (3 per SM): the first groups can be prefetched while the previous kernel ends
    p.prefetch_first = (a->n_splits > 0 && s_total * a->kv_heads * a->batch <= 3 * int64_t(sm_count())) ? 1 : 0;
    // a window that the splits can cover from its own first group: map the splits onto the window, so a
    // small window gets all the splits (the grid need not cover the whole capacity)
    p.win_rel = (a->window > 0 && a->n_splits > 0 && a->n_splits * a->chunk >= a->window + GT) ? 1 : 0;
    p.qkv = nullptr;
    p.qkv_b = 0;
    p.q_norm_w = p.k_norm_w = p.cos = p.sin = nullptr;
    p.rope_len = 0;
    p.pos = nullptr;
    p.written_out = p.qlen_out = p.pg_out = nullptr;
    p.ring_k = p.ring_v = nullptr;
    p.kq_w = p.vq_w = nullptr;
    p.kmn_w = p.kst_w = p.vmn_w = p.vst_w = nullptr;
    p.eps = 0.f;
    if (qk) {
        p.qkv = (const __half*)qk->qkv;
        p.qkv_b = qk->qkv_stride;
        p.q_norm_w = (const __half*)qk->q_norm_weight;
        p.k_norm_w = (const __half*)qk->k_norm_weight;
        p.cos = (const __half*)qk->cos;
        p.sin = (const __half*)qk->sin;
        p.rope_len = qk->rope_len;
        p.pos = qk->pos;
        p.written_out = qk->written;
        p.qlen_out = qk->qlen;
        p.pg_out = qk->pg;
        p.ring_k = (__half*)qk->tail_k;
        p.ring_v = (__half*)qk->tail_v;
        p.kq_w = (uint8_t*)qk->kq;
        p.vq_w = (uint8_t*)qk->vq;
        p.kmn_w = (__half*)qk->kmn;
        p.kst_w = (__half*)qk->kst;
        p.vmn_w = (__half*)qk->vmn;
        p.vst_w = (__half*)qk->vst;
        p.eps = float(qk->eps);
    }

    using Kern = void (*)(Params, CUtensorMap, CUtensorMap);
    Kern kern = qk ? attn_decode_int8_kernel<true> : attn_decode_int8_kernel<false>;
    static bool attr_set[2][kMaxDevices] = {};   // the attribute is per device
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(NOVA_ERR_CUDA, "no usable current device (%d)", dev);
    if (!attr_set[qk ? 1 : 0][dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
            cudaGetLastError();
            return fail(NOVA_ERR_CUDA, "cudaFuncSetAttribute(max dynamic smem) failed");
        }
        attr_set[qk ? 1 : 0][dev] = true;
    }
    dim3 grid(unsigned(s_total), unsigned(a->kv_heads), unsigned(a->batch));
    const cudaError_t err = launch(kern, grid, dim3(THREADS), size_t(SMEM_BYTES), (cudaStream_t)stream, p, tmK, tmV);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "%s: launch failed: %s", qk ? "nova_qk_append_attn_int8" : "nova_attn_decode_int8",
                    cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_attn_decode_int8(const nova_attn_int8_args* a, void* stream) {
    return attn_launch(a, nullptr, stream);
}

extern "C" int nova_qk_append_attn_int8(const nova_qk_args* qk, const nova_attn_int8_args* a, void* stream) {
    if (!qk || !a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (qk->head_dim != 128 || qk->group != 64) return fail(NOVA_ERR_UNSUPPORTED, "head_dim must be 128 and group 64");
    if (qk->batch != a->batch || qk->q_heads != a->q_heads || qk->kv_heads != a->kv_heads ||
        qk->max_len != a->max_len)
        return fail(NOVA_ERR_INVALID, "q/k args and attention args disagree on batch/heads/max_len");
    if (!a->tail_k || a->n_splits < 1)
        return fail(NOVA_ERR_INVALID, "the fused append needs the fp16 tail ring and at least one int8 split");
    if (qk->tail_k != a->tail_k || qk->tail_v != a->tail_v || qk->kq != a->kq || qk->vq != a->vq ||
        qk->kmn != a->kmn || qk->kst != a->kst || qk->vmn != a->vmn || qk->vst != a->vst)
        return fail(NOVA_ERR_INVALID, "q/k args and attention args must name the same ring and int8 cache");
    if (!qk->qkv || !qk->q_norm_weight || !qk->k_norm_weight || !qk->cos || !qk->sin || !qk->pos || !qk->written ||
        !qk->qlen || !qk->pg)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (qk->rope_len <= 0) return fail(NOVA_ERR_INVALID, "bad rope_len");
    if (qk->qkv_stride < (qk->q_heads + 2 * qk->kv_heads) * 128)
        return fail(NOVA_ERR_INVALID, "qkv_stride shorter than a q|k|v row");
    return attn_launch(a, qk, stream);
}
