// NF4 weight GEMV / skinny GEMM (M <= 8) for sm_100a, plus the NF4 quantizer,
// dequantizer and the packer into the B200-native weight layout.
//
// Reference weight format (src/nova/quant.py:39-69): packed uint8 [N, K/2],
// K-contiguous, byte j of a row = element 2j in the high nibble, 2j+1 in the
// low nibble; absmax [K/64, N] (fp32 in the reference, fp16 here); the
// codebook as the reference's 256-entry fp16x2 LUT (src/nova/kernels.py:
// 170-182: low half = code[b>>4], high half = code[b&15]).
//
//   y[m, n] = sum_blocks absmax[blk, n] * sum_{k in blk} x[m, k] * code16[idx(n, k)]
//
// Native layout ("units"): the matrix is cut into 32-row x 64-k units, stored
// row-group major, block minor, each as one contiguous 1088-byte record.
// Bytes [16L, 16L+16) hold, for MMA lane L = 4g + t, bytes [8t, 8t+8) of the
// 32-byte blocks (the k values 16t..16t+15) of rows g and g+8 of the group;
// bytes [512 + 16L, +16) the same for rows g+16 and g+24; bytes 1024..1087 the
// 32 fp16 absmax values ordered so lane group g finds rows g, g+8, g+16, g+24
// at [4g, 4g+4).  Every 16-byte lane read of a warp covers 512 contiguous
// bytes (one wavefront per quarter warp), and a warp's range of consecutive
// units is one contiguous stretch of memory that a single bulk copy fetches.
//
// Work split ("stream-K"): the units are dealt out in equal contiguous ranges
// to every warp of a persistent grid, so all SMs stream the same number of
// bytes whatever N and K are.  A warp that covers a whole row group finishes
// it; a partial group leaves its accumulator fragments in a workspace slot and
// the last of the group's warps to arrive (arrival counter) adds the slots in
// warp order -- deterministic -- and runs the epilogue.
//
// Decode: each byte becomes one f16x2 A-fragment register through one byte
// permute (forms a LUT address from the byte and the lane id) and one
// bank-conflict-free shared-memory load (the LUT is replicated per lane).  The
// products code16 * x16 are exact in fp32 and accumulated in fp32 by mma.sync
// m16n8k16 (x in the B operand, columns = the M <= 8 rows); each 64-element
// block gets a fresh accumulator scaled by its absmax, as in the reference
// kernel (src/nova/kernels.py:213-232).
#include "common.cuh"

namespace nova {
namespace nf4 {

constexpr int LUT_WORDS = 256 * 64;      // entry v at word v*64 + lane (256-byte rows)
constexpr int LUT_BYTES = LUT_WORDS * 4;
constexpr int MAX_M = 8;
constexpr int UNIT_ROWS = 32;
constexpr int UNIT_CODE_BYTES = 1024;
constexpr int UNIT_BYTES = 1088;

enum Epi { EPI_PLAIN = 0, EPI_RESIDUAL = 1, EPI_SILU_MUL = 2, EPI_ARGMAX = 3, EPI_F32 = 4, EPI_SLOTS = 5 };
constexpr int SLOTS_PER_CTA = 4;   // NF4_SLOTS: row groups one CTA's share of the k-blocks may touch

struct Params {
    const __half* x;          // fp16 [M, K] (the residual when norm_w != nullptr)
    int64_t x_stride;
    const __half* norm_w;     // fp16 [K] RMSNorm weight or nullptr
    float eps;
    const uint8_t* packed;    // reference layout [N, K/2] or native units
    const void* absmax;       // reference layout only
    const uint32_t* lut;
    const __half* bias;
    const __half* residual;
    int64_t res_stride;
    __half* out;
    int64_t out_stride;
    unsigned long long* argmax;
    int64_t* token_out;       // finalize (ARGMAX): next token per row
    int64_t* pos;             // finalize: device position, += 1
    const __half* embed;      // finalize: embedding table [vocab, embed_dim]
    __half* embed_out;        // finalize: next-step hidden [M, embed_dim]
    int64_t embed_out_stride;
    int embed_dim;
    float4* partial;          // [total_warps][2][32][2] float4
    unsigned* counters;       // [n_tiles]
    unsigned* done;           // finalize arrival counter
    int M, N, K, KB, n_tiles, total_warps;
    int64_t units;
    int res_rows = 0;         // CTA kernel: residual rows staged in shared memory per CTA (0: read in the epilogue)
    // deferred row-parallel reduction: x += the slots of the previous GEMV (its units, grid, k-blocks per row
    // group), stored to resid_out by CTA 0
    const float* add_slots = nullptr;
    int64_t add_units = 0;
    int add_G = 0, add_KB = 0;
    __half* resid_out = nullptr;
    // SiLU·mul split at CTA edges (M = 1): edge_out receives, per CTA, the fp32 sums of its first and
    // last row group when a neighbouring CTA shares them; edge_in (the next launch) completes those
    // outputs while staging x (producer units, grid, k-blocks per row group)
    float* edge_out = nullptr;
    const float* edge_in = nullptr;
    int64_t edge_units = 0;
    int edge_G = 0, edge_KB = 0;
    // o_proj over the decode attention's split partials (EPI_F32, M = 1): the rows are (KV head, output
    // row) pairs of one head's K-column block (the head-major unit stream), each CTA owns whole row groups
    // of one head and merges that head's partials ([heads][splits][K / 128][132] floats) into x
    const float* mrg_part = nullptr;
    int mrg_splits = 0, mrg_heads = 0;
    // x += fp16(sum of the add_nheads fp32 rows add_heads[h][K] in head order) before the norm prologue
    const float* add_heads = nullptr;
    int add_nheads = 0;
};

template <typename T>
__device__ __forceinline__ float absmax_at(const void* a, int64_t i) {
    return float(__ldg(reinterpret_cast<const T*>(a) + i));
}
template <>
__device__ __forceinline__ float absmax_at<__half>(const void* a, int64_t i) {
    return __half2float(__ldg(reinterpret_cast<const __half*>(a) + i));
}

__device__ __forceinline__ int64_t unit_begin(int64_t units, int w, int W) { return units * w / W; }
__device__ __forceinline__ int owner_of(int64_t u, int64_t units, int W) {
    return int(((u + 1) * W - 1) / units);
}

// Orderable key: larger fp16 value -> larger key; equal values -> smaller index wins
// (torch.argmax returns the first maximal index).
__device__ __forceinline__ unsigned long long argmax_key(__half v, int idx) {
    unsigned short b = __half_as_ushort(v);
    unsigned short o = (b & 0x8000) ? (unsigned short)(~b) : (unsigned short)(b | 0x8000);
    return (static_cast<unsigned long long>(o) << 32) | static_cast<unsigned long long>(0xffffffffu - unsigned(idx));
}

// fp16(silu(fp16(gate)) * fp16(up)) from the fp32 sums, silu rounded to fp16 as
// the reference's fp16 activation does (src/nova/layers.py:173-174).
__device__ __forceinline__ __half silu_mul_h(float gate_sum, float up_sum) {
    const float gate = __half2float(__float2half_rn(gate_sum));
    const float up = __half2float(__float2half_rn(up_sum));
    const float s = __half2float(__float2half_rn(__fdiv_rn(gate, 1.0f + expf(-gate))));
    return __float2half_rn(s * up);
}

// Epilogue of one 16-row tile: lane (g, t) holds rows 16*tile+g (c[0], c[1])
// and 16*tile+g+8 (c[2], c[3]) for batch rows m = m0 + 2t, m0 + 2t + 1.
// `rs`: the residual rows [rs_row0, rs_row0 + rs_rows) of every batch row,
// staged in shared memory ([m][rs_rows]); nullptr reads p.residual.
template <int EPI>
__device__ __forceinline__ void epilogue(const Params& p, int tile, const float (&c)[4], int g, int t, int m0 = 0,
                                         const __half* rs = nullptr, int rs_row0 = 0, int rs_rows = 0) {
    if (EPI == EPI_F32) {   // fp32 accumulators as they are (tensor-parallel partial sums)
        float* o = reinterpret_cast<float*>(p.out);
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int m = m0 + 2 * t + e;
                if (m < p.M) o[m * p.out_stride + tile * 16 + g + 8 * hrow] = c[2 * hrow + e];
            }
        return;
    }
    if (EPI == EPI_SILU_MUL) {
        // tile rows 0..7 are gate rows 8*tile+g, rows 8..15 the matching up rows
        const int n = tile * 8 + g;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int m = m0 + 2 * t + e;
            if (m >= p.M) continue;
            p.out[m * p.out_stride + n] = silu_mul_h(c[e], c[2 + e]);
        }
        return;
    }
    unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
        const int n = tile * 16 + g + 8 * hrow;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int m = m0 + 2 * t + e;
            if (m >= p.M) continue;
            float v = c[2 * hrow + e];
            __half h;
            if (EPI == EPI_RESIDUAL) {
                const __half r = rs ? rs[m * rs_rows + (n - rs_row0)] : __ldcg(p.residual + m * p.res_stride + n);
                h = __float2half_rn(__half2float(r) + __half2float(__float2half_rn(v)));
            } else {
                if (p.bias) v += __half2float(p.bias[n]);
                h = __float2half_rn(v);
            }
            p.out[m * p.out_stride + n] = h;
            if (EPI == EPI_ARGMAX) {
                const unsigned long long k = argmax_key(h, n);
                best[e] = k > best[e] ? k : best[e];
            }
        }
    }
    if (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            unsigned long long k = best[e];
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                k = o > k ? o : k;
            }
            const int m = m0 + 2 * t + e;
            if (g == 0 && m < p.M) atomicMax(p.argmax + m, k);
        }
    }
}

// Greedy-step finalize, run by the last warp of the lm_head launch: token =
// argmax index, re-arm the argmax slot, gather the token's embedding row as
// the next step's hidden state and advance the position
// (src/nova/decode.py:318-319 and the embed_tokens lookup of src/nova/model.py:131).
__device__ __forceinline__ void finalize_step(const Params& p, int lane) {
    for (int m = 0; m < p.M; ++m) {
        const unsigned long long key = __ldcg(p.argmax + m);
        const int64_t tok = int64_t(0xffffffffu - unsigned(key & 0xffffffffull));
        if (lane == 0) {
            p.token_out[m] = tok;
            p.argmax[m] = 0ull;
        }
        if (p.embed) {
            const uint4* src = reinterpret_cast<const uint4*>(p.embed + tok * p.embed_dim);
            uint4* dst = reinterpret_cast<uint4*>(p.embed_out + m * p.embed_out_stride);
            for (int i = lane; i < p.embed_dim / 8; i += 32) dst[i] = __ldg(src + i);
        }
    }
    if (lane == 0) {
        if (p.pos) *p.pos += 1;
        *p.done = 0u;
    }
}

// Per-lane replicated LUT: entry v for lane l at word v*64 + l (l < 32).
// Every thread's loads are issued before its first store: one L2 round trip.
template <int THREADS>
__device__ __forceinline__ void build_lut(uint32_t* lut_s, const uint32_t* lut) {
    constexpr int IT = (256 * 4 + THREADS - 1) / THREADS;
    uint32_t w[IT];
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int v = threadIdx.x + i * THREADS;
        w[i] = v < 256 * 4 ? __ldg(lut + (v >> 2)) : 0u;
    }
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int v = threadIdx.x + i * THREADS;
        if (v >= 256 * 4) break;
        uint4* dst = reinterpret_cast<uint4*>(lut_s + (v >> 2) * 64 + 8 * (v & 3));
        dst[0] = make_uint4(w[i], w[i], w[i], w[i]);
        dst[1] = make_uint4(w[i], w[i], w[i], w[i]);
    }
}

// Stage x in shared memory, optionally RMS-normalised in HF order (x read
// through L2 only: the previous kernel wrote it from other SMs).  When
// every thread holds at most one 8-element chunk per row (K <= 8 * THREADS),
// the chunk stays in registers between the sum of squares and the scaling,
// so x and the norm weight are read once.
// The RMSNorm weight slice stage_x's single-chunk path uses (thread i holds
// elements 8i..8i+7).  A weight, so it may be read before the dependency wait.
template <int THREADS>
__device__ __forceinline__ uint4 norm_w_chunk(const Params& p) {
    const int i = threadIdx.x;
    if (p.norm_w && p.K / 8 <= THREADS && i < p.K / 8) return *reinterpret_cast<const uint4*>(p.norm_w + 8 * i);
    return make_uint4(0u, 0u, 0u, 0u);
}

// Deferred row-parallel reduction for the 8 columns 8i .. 8i+7 of row 0: the
// previous GEMV's CTAs c in [cf, cl] each left fp32 sums of their k-blocks of
// this row group in slot (c, row group == their first ? 0 : 1); they are added
// in CTA order, rounded to fp16 (the projection's output) and added to the
// residual chunk xv as the reference's fp16 residual add does.  CTA 0 stores
// the result for the later kernels.
struct SlotPlan {
    const float4* src[4];   // contributors in CTA order (n of them)
    int n;
};

// The slot addresses of chunk i (static: computed before the dependency wait).
__device__ __forceinline__ SlotPlan slot_plan(const Params& p, int i) {
    SlotPlan sp;
    sp.n = 0;
    const int kv8 = p.K / 8;
    if (!p.add_slots || i >= kv8) return sp;
    const int rg = i >> 2, r0 = 8 * (i & 3);
    const int U = int(p.add_units), G = p.add_G, KB = p.add_KB;   // U * G < 2^31 (host-checked)
    const int u0 = rg * KB;
    const int cf = ((u0 + 1) * G - 1) / U;
    const int cl = ((u0 + KB) * G - 1) / U;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int cc = cf + q;
        const int first = ((U * cc) / G) / KB;
        sp.src[q] = reinterpret_cast<const float4*>(p.add_slots + (int64_t(cc) * SLOTS_PER_CTA + (rg - first)) * 32 + r0);
    }
    sp.n = cl - cf + 1;
    return sp;
}

__device__ __forceinline__ void add_residual_chunk(const Params& p, int i, const float (&sum)[8], uint4& xv);

// Deferred row-parallel reduction for the 8 columns 8i .. 8i+7 of row 0: the
// previous GEMV's CTAs each left fp32 sums of their k-blocks of this row group
// in a slot (SlotPlan); they are added in CTA order, rounded to fp16 (the
// projection's output) and added to the residual chunk xv as the reference's
// fp16 residual add does.  CTA 0 stores the result for the later kernels.

__device__ __forceinline__ void add_slots_chunk(const Params& p, const SlotPlan& sp, int i, uint4& xv) {
    float4 a[4][2];
#pragma unroll
    for (int q = 0; q < 4; ++q)
        if (q < sp.n) {
            a[q][0] = __ldcg(sp.src[q]);
            a[q][1] = __ldcg(sp.src[q] + 1);
        }
    float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (q >= sp.n) break;
        sum[0] += a[q][0].x; sum[1] += a[q][0].y; sum[2] += a[q][0].z; sum[3] += a[q][0].w;
        sum[4] += a[q][1].x; sum[5] += a[q][1].y; sum[6] += a[q][1].z; sum[7] += a[q][1].w;
    }
    add_residual_chunk(p, i, sum, xv);
}

// The projection's 8 fp32 sums rounded to fp16 and added to the residual chunk xv (fp16 add, the
// reference's residual arithmetic); CTA 0 stores the result for the later kernels.
__device__ __forceinline__ void add_residual_chunk(const Params& p, int i, const float (&sum)[8], uint4& xv) {
    __half2* h = reinterpret_cast<__half2*>(&xv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 r = __half22float2(h[e]);
        const float o0 = __half2float(__float2half_rn(sum[2 * e])), o1 = __half2float(__float2half_rn(sum[2 * e + 1]));
        h[e] = __floats2half2_rn(r.x + o0, r.y + o1);
    }
    if (blockIdx.x == 0 && p.resid_out) *reinterpret_cast<uint4*>(p.resid_out + 8 * i) = xv;
}

// The output chunk (8 columns) that thread j completes from the previous
// launch's CTA edges, and its two contributors (static: computed before the
// dependency wait).  Boundary j / 2 + 1 lies between producer CTAs bnd - 1 and
// bnd; when it falls inside a row group, that group's 16 outputs (two chunks,
// j & 1) are summed from the last-row-group slot of CTA bnd - 1 and the
// first-row-group slot of CTA bnd.
struct EdgePlan {
    const float4* a;   // contributors in CTA order: gate sums [0, 2), up sums [2, 4)
    const float4* b;
    int i;             // chunk index (outputs 8i .. 8i+7), -1: none
};

__device__ __forceinline__ EdgePlan edge_plan(const Params& p, int j) {
    EdgePlan e;
    e.a = e.b = nullptr;
    e.i = -1;
    if (!p.edge_in || j >= 2 * (p.edge_G - 1)) return e;
    const int bnd = j / 2 + 1, tl = j & 1;
    const int u = int(p.edge_units) * bnd / p.edge_G;   // units * G < 2^31 (host-checked)
    if (u % p.edge_KB == 0) return e;
    e.i = 2 * (u / p.edge_KB) + tl;
    e.a = reinterpret_cast<const float4*>(p.edge_in + ((bnd - 1) * 2 + 1) * 32 + 16 * tl);
    e.b = reinterpret_cast<const float4*>(p.edge_in + (bnd * 2) * 32 + 16 * tl);
    return e;
}

// `wpre`: norm_w_chunk() loaded earlier (nullptr: loaded here).
// ADD_HEADS: the add_heads prologue is compiled in (only the gate|up kernel takes it).
template <int THREADS, bool ADD_HEADS = false>
__device__ __forceinline__ void stage_x(const Params& p, __half* xs, const uint4* wpre = nullptr,
                                        const SlotPlan* sp = nullptr, const EdgePlan* ep = nullptr) {
    __shared__ float red[THREADS / 32][MAX_M];
    __shared__ float rstd[MAX_M];
    const int kv8 = p.K / 8;
    if (ADD_HEADS && p.add_heads && p.norm_w) {
        // M = 1 and one chunk per thread (host-checked): x += fp16(the heads' sums), then the norm; only one
        // row's registers live, so the 8 heads' loads are in flight together with x's
        const int i = threadIdx.x;
        float ss = 0.f;
        uint4 xv = make_uint4(0u, 0u, 0u, 0u), wv = make_uint4(0u, 0u, 0u, 0u);
        if (i < kv8) {
            wv = wpre ? *wpre : *reinterpret_cast<const uint4*>(p.norm_w + 8 * i);
            xv = __ldcg(reinterpret_cast<const uint4*>(p.x + 8 * i));
            float4 a[8][2];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (q < p.add_nheads) {
                    const float4* src = reinterpret_cast<const float4*>(p.add_heads + int64_t(q) * p.K + 8 * i);
                    a[q][0] = __ldcg(src);
                    a[q][1] = __ldcg(src + 1);
                }
            float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (q >= p.add_nheads) break;
                sum[0] += a[q][0].x; sum[1] += a[q][0].y; sum[2] += a[q][0].z; sum[3] += a[q][0].w;
                sum[4] += a[q][1].x; sum[5] += a[q][1].y; sum[6] += a[q][1].z; sum[7] += a[q][1].w;
            }
            add_residual_chunk(p, i, sum, xv);
            const __half2* h = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h[q]);
                ss += f.x * f.x + f.y * f.y;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][0] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = 0.f;
            for (int w = 0; w < THREADS / 32; ++w) v += red[w][0];
            rstd[0] = rsqrt_ieee(__fdiv_rn(v, float(p.K)) + p.eps);
        }
        __syncthreads();
        if (i < kv8) {
            const float r = rstd[0];
            const __half2* h = reinterpret_cast<const __half2*>(&xv);
            const __half2* wh = reinterpret_cast<const __half2*>(&wv);
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h[q]);
                const float2 wf = __half22float2(wh[q]);
                const float2 nf = __half22float2(__floats2half2_rn(f.x * r, f.y * r));
                oh[q] = __floats2half2_rn(wf.x * nf.x, wf.y * nf.y);
            }
            *reinterpret_cast<uint4*>(xs + 8 * i) = o;
        }
        return;
    }
    if (p.norm_w) {
        const bool one = kv8 <= THREADS;
        float ss[MAX_M];
        uint4 xv[MAX_M];
        uint4 wv = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int m = 0; m < MAX_M; ++m) {
            ss[m] = 0.f;
            xv[m] = make_uint4(0u, 0u, 0u, 0u);
        }
        auto add_sq = [&](const uint4& v, float& acc) {
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h[q]);
                acc += f.x * f.x + f.y * f.y;
            }
        };
        if (one) {
            const int i = threadIdx.x;
            if (i < kv8) {
                wv = wpre ? *wpre : *reinterpret_cast<const uint4*>(p.norm_w + 8 * i);
#pragma unroll
                for (int m = 0; m < MAX_M; ++m) {
                    if (m >= p.M) break;
                    xv[m] = __ldcg(reinterpret_cast<const uint4*>(p.x + m * p.x_stride + 8 * i));
                }
                if (sp && sp->n) add_slots_chunk(p, *sp, i, xv[0]);   // M == 1
#pragma unroll
                for (int m = 0; m < MAX_M; ++m) {
                    if (m >= p.M) break;
                    add_sq(xv[m], ss[m]);
                }
            }
        } else {
            for (int i = threadIdx.x; i < kv8; i += THREADS) {
#pragma unroll
                for (int m = 0; m < MAX_M; ++m) {
                    if (m >= p.M) break;
                    add_sq(__ldcg(reinterpret_cast<const uint4*>(p.x + m * p.x_stride + 8 * i)), ss[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAX_M; ++m) {
            float v = ss[m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][m] = v;
        }
        __syncthreads();
        if (threadIdx.x < MAX_M) {
            float v = 0.f;
            for (int w = 0; w < THREADS / 32; ++w) v += red[w][threadIdx.x];
            rstd[threadIdx.x] = rsqrt_ieee(__fdiv_rn(v, float(p.K)) + p.eps);
        }
        __syncthreads();
        auto scale = [&](const uint4& v, const uint4& w8, float r) {
            const __half2* h = reinterpret_cast<const __half2*>(&v);
            const __half2* wh = reinterpret_cast<const __half2*>(&w8);
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h[q]);
                const float2 wf = __half22float2(wh[q]);
                const float2 nf = __half22float2(__floats2half2_rn(f.x * r, f.y * r));
                oh[q] = __floats2half2_rn(wf.x * nf.x, wf.y * nf.y);
            }
            return o;
        };
        if (one) {
            const int i = threadIdx.x;
            if (i < kv8) {
#pragma unroll
                for (int m = 0; m < MAX_M; ++m) {
                    if (m >= p.M) break;
                    *reinterpret_cast<uint4*>(xs + m * p.K + 8 * i) = scale(xv[m], wv, rstd[m]);
                }
            }
        } else {
            for (int i = threadIdx.x; i < kv8; i += THREADS) {
                const uint4 w8 = *reinterpret_cast<const uint4*>(p.norm_w + 8 * i);
                for (int m = 0; m < p.M; ++m)
                    *reinterpret_cast<uint4*>(xs + m * p.K + 8 * i) =
                        scale(__ldcg(reinterpret_cast<const uint4*>(p.x + m * p.x_stride + 8 * i)), w8, rstd[m]);
            }
        }
    } else {
        // up to four 16-byte chunks per thread requested before any is stored: one L2 round trip
        constexpr int XU = 4;
        const int total = p.M * kv8;
        for (int base = threadIdx.x; base < total; base += XU * THREADS) {
            uint4 v[XU];
#pragma unroll
            for (int u = 0; u < XU; ++u) {
                const int i = base + u * THREADS;
                if (i < total) v[u] = __ldcg(reinterpret_cast<const uint4*>(p.x + (i / kv8) * p.x_stride) + i % kv8);
            }
#pragma unroll
            for (int u = 0; u < XU; ++u) {
                const int i = base + u * THREADS;
                if (i < total) *reinterpret_cast<uint4*>(xs + (i / kv8) * p.K + 8 * (i % kv8)) = v[u];
            }
        }
        if (ep && p.edge_in) {   // uniform: the chunks split at the producer's CTA edges replace what x held
            // (M = 1; the contributors' loads wait out the barrier, which orders these stores after x's)
            const bool fix = ep->i >= 0;
            float4 ea[4], eb[4];
            if (fix) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    ea[q] = __ldcg(ep->a + q);
                    eb[q] = __ldcg(ep->b + q);
                }
            }
            __syncthreads();
            if (fix) {
                // silu_mul_h's arithmetic, with the eight exponentials issued before the divisions
                const float ga[8] = {ea[0].x + eb[0].x, ea[0].y + eb[0].y, ea[0].z + eb[0].z, ea[0].w + eb[0].w,
                                     ea[1].x + eb[1].x, ea[1].y + eb[1].y, ea[1].z + eb[1].z, ea[1].w + eb[1].w};
                const float ua[8] = {ea[2].x + eb[2].x, ea[2].y + eb[2].y, ea[2].z + eb[2].z, ea[2].w + eb[2].w,
                                     ea[3].x + eb[3].x, ea[3].y + eb[3].y, ea[3].z + eb[3].z, ea[3].w + eb[3].w};
                float gt[8], den[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    gt[e] = __half2float(__float2half_rn(ga[e]));
                    den[e] = 1.0f + expf(-gt[e]);
                }
                uint4 o;
                __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float sl = __half2float(__float2half_rn(__fdiv_rn(gt[e], den[e])));
                    oh[e] = __float2half_rn(sl * __half2float(__float2half_rn(ua[e])));
                }
                *reinterpret_cast<uint4*>(xs + 8 * ep->i) = o;
            }
        }
    }
}

// Partial-tile protocol: store this warp's fragments, count arrivals, and let
// the last contributor add all fragments in warp order and run the epilogue.
template <int EPI, int NT>
__device__ __forceinline__ void flush_partial(const Params& p, int rg, const float (&acc)[NT][4], int w,
                                              int first_rg, int lane, int g, int t) {
    const int W = p.total_warps;
    const int slot = 2 * w + (rg == first_rg ? 0 : 1);
    float4* dst = p.partial + (int64_t(slot) * 32 + lane) * 2;
#pragma unroll
    for (int i = 0; i < NT; ++i) dst[i] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    fence_acq_rel_gpu();
    __syncwarp();
    const int64_t u0 = int64_t(rg) * p.KB;
    const int w_first = owner_of(u0, p.units, W);
    const int w_last = owner_of(u0 + p.KB - 1, p.units, W);
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(p.counters + rg, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != unsigned(w_last - w_first)) return;
    fence_acq_rel_gpu();
    float c[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.f;
    // Contributors are added in warp order; the loads of four of them are in
    // flight at once.  Every contributor after the first starts inside rg (its
    // slot 0); the first one used slot 1 if its range began in an earlier group.
    const int first_slot1 = unit_begin(p.units, w_first, W) < u0 ? 1 : 0;
    for (int w0 = w_first; w0 <= w_last; w0 += 4) {
        float4 v[4][NT];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int ww = w0 + q;
            if (ww > w_last) break;
            const int sl = 2 * ww + (ww == w_first ? first_slot1 : 0);
            const float4* src = p.partial + (int64_t(sl) * 32 + lane) * 2;
#pragma unroll
            for (int i = 0; i < NT; ++i) v[q][i] = __ldcg(src + i);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (w0 + q > w_last) break;
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                c[i][0] += v[q][i].x; c[i][1] += v[q][i].y; c[i][2] += v[q][i].z; c[i][3] += v[q][i].w;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < NT; ++i) epilogue<EPI>(p, rg * NT + i, c[i], g, t);
    if (lane == 0) p.counters[rg] = 0u;
}

template <int EPI>
__device__ __forceinline__ void finish_launch(const Params& p, int lane) {
    if (EPI != EPI_ARGMAX || !p.token_out) return;
    fence_acq_rel_gpu();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(p.done, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev == unsigned(p.total_warps - 1)) {
        fence_acq_rel_gpu();
        finalize_step(p, lane);
    }
}

// ---------------------------------------------------------------------------
// Native-layout kernel: one 16-warp CTA per SM.  Each warp owns a contiguous
// range of units, which is one contiguous stretch of the unit stream, and
// streams it through a private two-stage shared-memory ring: one bulk copy
// (cp.async.bulk, mbarrier-tracked) per stage of up to `stage_units` units.
// The first two stages are requested before the prologue (they are weights,
// independent of every previous kernel), so the LUT build and x staging
// overlap the first DRAM round trip.

constexpr int NAT_WARPS = 16;
constexpr int NAT_THREADS = NAT_WARPS * 32;
constexpr int EDGE_RED_BYTES = NAT_WARPS * 2 * 32 * 4;   // [warp][first / last row group][32 rows] fp32
constexpr int NAT_STAGES = 2;
constexpr int NAT_MIN_UNITS = 8;   // units per warp at least (few contributors per row group)

// SiLU·mul with CTA edges (M = 1): the 16 warps of a CTA own consecutive
// unit ranges, and each leaves its sums of a row group it shares with another
// warp in edge_red[warp][0 = its first row group, 1 = its last].  After the
// CTA's last barrier warp j adds the contributors of the CTA's j-th row group
// in warp order; a row group inside the CTA's units gets the SiLU·mul
// epilogue, the first and last one, when a neighbouring CTA has the rest of
// their k-blocks, go to edge_out[CTA][0 / 1] as fp32 sums that the next launch
// completes (EdgePlan).  Row groups one warp covered alone were finished in
// its loop.  No cross-CTA reduction, no fence, no counter.
struct EdgeRed {
    int rg;          // row group, -1: nothing to add
    int w0, n;       // contributors: CTA warps w0 .. w0 + n - 1
    unsigned slots;  // bit k: contributor w0 + k left it in its slot 1
    int dst;         // -1: the launch's own epilogue (SiLU·mul; fp32 sums per head for o_proj over the
                     // attention's partials); else edge_out slot index (CTA * 2 + 0 / 1)
};

// Static (int32, computed before the dependency wait; units * W < 2^31 host-checked).
__device__ __forceinline__ EdgeRed edge_red_plan(const Params& p, int warp) {
    EdgeRed e;
    e.rg = -1;
    e.w0 = e.n = 0;
    e.slots = 0u;
    e.dst = -1;
    const int U = int(p.units), W = p.total_warps, KB = p.KB, c = int(blockIdx.x);
    const int cu0 = U * (c * NAT_WARPS) / W, cu1 = U * ((c + 1) * NAT_WARPS) / W;
    const int r0 = cu0 / KB, r1 = (cu1 - 1) / KB;
    const int rg = r0 + warp;
    if (rg > r1) return e;
    const int base = rg * KB;
    const int s0 = max(cu0, base), s1 = min(cu1, base + KB);
    const int wf = ((s0 + 1) * W - 1) / U, wl = (s1 * W - 1) / U;   // owners of s0 and s1 - 1
    if (wf == wl && s0 == base && s1 == base + KB) return e;
    e.rg = rg;
    e.w0 = wf - c * NAT_WARPS;
    e.n = wl - wf + 1;
    for (int k = 0; k < e.n; ++k)
        if ((U * (wf + k) / W) / KB != rg) e.slots |= 1u << k;
    if (!(cu0 <= base && cu1 >= base + KB)) e.dst = c * 2 + (rg == r0 ? 0 : 1);
    return e;
}

__device__ __forceinline__ void edge_finish(const Params& p, const EdgeRed& e, const float* edge_red, int lane) {
    if (e.rg < 0) return;
    float v = 0.f;
    for (int k = 0; k < e.n; ++k) v += edge_red[((e.w0 + k) * 2 + ((e.slots >> k) & 1u)) * 32 + lane];
    if (e.dst < 0) {
        // lane l holds row 16 tile + g + 8 hr (l = 16 tl + 8 hr + g): gate rows hr = 0, up rows hr = 1
        const float up = __shfl_down_sync(0xffffffffu, v, 8);
        if ((lane & 8) == 0) p.out[(2 * e.rg + (lane >> 4)) * 8 + (lane & 7)] = silu_mul_h(v, up);
    } else {
        p.edge_out[e.dst * 32 + lane] = v;
    }
}

// o_proj over the attention's split partials (M = 1): the rows of the launch
// are (KV head h, output row) pairs over head h's K-column block, so row group
// h * R + r (R = row groups per head) is output row group r restricted to the
// columns of head h.  The CTAs of head h (G*h/heads .. G*(h+1)/heads - 1) own
// consecutive whole row groups of it, their warps consecutive unit ranges.
__device__ __forceinline__ void heads_cta_range(const Params& p, int c, int& cu0, int& cu1, int& head) {
    const int G = int(gridDim.x), nh = p.mrg_heads;
    const int h = ((c + 1) * nh - 1) / G;
    const int c0 = G * h / nh, n = G * (h + 1) / nh - c0;
    const int R = (p.N / UNIT_ROWS) / nh, j = c - c0;
    cu0 = (h * R + R * j / n) * p.KB;
    cu1 = (h * R + R * (j + 1) / n) * p.KB;
    head = h;
}

// The row group of the CTA's that warp `warp` adds after the CTA's last
// barrier (whole row groups: no CTA edges; the sum goes out as fp32).
__device__ __forceinline__ EdgeRed heads_red_plan(const Params& p, int warp) {
    EdgeRed e;
    e.rg = -1;
    e.w0 = e.n = 0;
    e.slots = 0u;
    e.dst = -1;
    int cu0, cu1, h;
    heads_cta_range(p, int(blockIdx.x), cu0, cu1, h);
    const int KB = p.KB, len = cu1 - cu0;
    const int rg = cu0 / KB + warp;
    if (rg > (cu1 - 1) / KB) return e;
    const int base = rg * KB;
    const int wf = ((base - cu0 + 1) * NAT_WARPS - 1) / len, wl = ((base + KB - cu0) * NAT_WARPS - 1) / len;
    if (wf == wl) return e;   // one warp had all of it: finished in its loop
    e.rg = rg;
    e.w0 = wf;
    e.n = wl - wf + 1;
    for (int k = 0; k < e.n; ++k)
        if ((cu0 + len * (wf + k) / NAT_WARPS) / KB != rg) e.slots |= 1u << k;
    return e;
}

__device__ __forceinline__ void heads_finish(const Params& p, const EdgeRed& e, const float* red, int lane) {
    if (e.rg < 0) return;
    float v = 0.f;
    for (int k = 0; k < e.n; ++k) v += red[((e.w0 + k) * 2 + ((e.slots >> k) & 1u)) * 32 + lane];
    reinterpret_cast<float*>(p.out)[int64_t(e.rg) * 32 + lane] = v;
}

// x of head `head` (K = 128 * q heads per KV head columns) merged from the
// decode attention's split partials, with the attention's own merge
// arithmetic: M = the largest split maximum, weights exp2(m_s - M) (0 for an
// empty split), L and the accumulator summed in split order, then one
// rounding of acc / L to fp16 (0 when L is 0).  `scratch` holds 3 * 160 + 4
// floats of shared memory.
constexpr int MRG_MAX_SPLITS = 40;
constexpr int MRG_PART = 132;   // floats per (split, q head): m, l, 2 pad, acc[128]
__device__ __forceinline__ void stage_merge(const Params& p, __half* xs, int head, float* scratch) {
    float* sm = scratch;                            // [S * gq] split maxima
    float* sl = scratch + MRG_MAX_SPLITS * 4;       // [S * gq] split sums
    float* sw = scratch + 2 * MRG_MAX_SPLITS * 4;   // [S * gq] weights
    float* sM = scratch + 3 * MRG_MAX_SPLITS * 4;   // [gq]
    const int gq = p.K / 128, S = p.mrg_splits, tid = threadIdx.x;
    const int qh = tid >> 7, d = tid & 127;
    const float* base = p.mrg_part + int64_t(head) * S * gq * MRG_PART;
    float a[MRG_MAX_SPLITS];   // this thread's channel, split by split (requested with m and l: one round trip)
#pragma unroll
    for (int s = 0; s < MRG_MAX_SPLITS; ++s)
        a[s] = (s < S && qh < gq) ? __ldcg(base + (s * gq + qh) * MRG_PART + 4 + d) : 0.f;
    if (tid < S * gq) {
        sm[tid] = __ldcg(base + tid * MRG_PART);
        sl[tid] = __ldcg(base + tid * MRG_PART + 1);
    }
    __syncthreads();
    if (tid < gq) {
        float M = -INFINITY;
        for (int s = 0; s < S; ++s) M = fmaxf(M, sm[s * gq + tid]);
        sM[tid] = M;
    }
    __syncthreads();
    if (tid < S * gq) {
        const float M = sM[tid % gq], m = sm[tid];
        sw[tid] = (M == -INFINITY || m == -INFINITY) ? 0.f : exp2f(m - M);
    }
    __syncthreads();
    if (qh < gq) {
        float L = 0.f, o = 0.f;
        if (sM[qh] != -INFINITY) {
#pragma unroll
            for (int s = 0; s < MRG_MAX_SPLITS; ++s) {
                if (s >= S) break;
                const float wt = sw[s * gq + qh];
                if (wt == 0.f) continue;
                L += wt * sl[s * gq + qh];
                o += wt * a[s];
            }
        }
        xs[tid] = L > 0.f ? __float2half_rn(__fdiv_rn(o, L)) : __float2half_rn(0.f);
    }
}

__device__ __forceinline__ void mma_unit_smem(const uint8_t* unit, const uint32_t (&xb)[8], uint32_t lut_base,
                                              uint32_t laneword, int lane, int g, float (&acc)[2][4]) {
    const uint4 c0 = lds128(unit + 16 * lane);          // rows g, g+8
    const uint4 c1 = lds128(unit + 512 + 16 * lane);    // rows g+16, g+24
    uint2 am;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(am.x), "=r"(am.y)
                 : "r"(smem_u32(unit + UNIT_CODE_BYTES + 8 * g)));
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    float blk[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int wi = s >> 1;
        const uint32_t sel0 = 0x5504u | (uint32_t((s & 1) * 2) << 4);
        const uint32_t sel1 = sel0 + 0x10u;
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
            const uint32_t r0w = w[4 * tile + wi], r1w = w[4 * tile + 2 + wi];
            const uint32_t a0 = lds32(lut_base + __byte_perm(r0w, laneword, sel0));
            const uint32_t a2 = lds32(lut_base + __byte_perm(r0w, laneword, sel1));
            const uint32_t a1 = lds32(lut_base + __byte_perm(r1w, laneword, sel0));
            const uint32_t a3 = lds32(lut_base + __byte_perm(r1w, laneword, sel1));
            mma_16816(blk[tile], a0, a1, a2, a3, xb[2 * s], xb[2 * s + 1]);
        }
    }
    const float2 a01 = __half22float2(*reinterpret_cast<const __half2*>(&am.x));
    const float2 a23 = __half22float2(*reinterpret_cast<const __half2*>(&am.y));
    acc[0][0] += a01.x * blk[0][0];
    acc[0][1] += a01.x * blk[0][1];
    acc[0][2] += a01.y * blk[0][2];
    acc[0][3] += a01.y * blk[0][3];
    acc[1][0] += a23.x * blk[1][0];
    acc[1][1] += a23.x * blk[1][1];
    acc[1][2] += a23.y * blk[1][2];
    acc[1][3] += a23.y * blk[1][3];
}

// XG: x is read through L1 from global memory instead of being staged (large
// M*K without the norm prologue, where the staged copy would crowd out the
// weight rings).  Warp w of the launch is warp w / gridDim.x of CTA
// w % gridDim.x, so small launches spread their warps over all SMs.
template <int EPI, bool XG>
__global__ void __launch_bounds__(NAT_THREADS, 1)
    nf4_gemv_native_kernel(const __grid_constant__ Params p, int stage_units, int* err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NAT_WARPS][NAT_STAGES];
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem_raw);
    __half* xs = reinterpret_cast<__half*>(smem_raw + LUT_BYTES);
    const int xs_bytes = XG ? 0 : (p.M * p.K * 2 + 127) / 128 * 128;
    const int stage_bytes = stage_units * UNIT_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem_raw + LUT_BYTES + xs_bytes + size_t(warp) * NAT_STAGES * stage_bytes;
    // EDGE (SiLU·mul with edge_out, M = 1, every warp active): the warps of a CTA take consecutive
    // ranges, so most shared row groups are added in shared memory (edge_finish); otherwise warp w
    // of the grid is warp w / G of CTA w % G
    const bool edge = EPI == EPI_SILU_MUL && p.edge_out != nullptr;
    // HEADS (EPI_F32 over the attention's partials, M = 1, every warp active): head-aligned CTAs, the
    // same consecutive warp ranges and shared-memory sums
    const bool heads = EPI == EPI_F32 && p.mrg_part != nullptr;
    float* edge_red = reinterpret_cast<float*>(smem_raw + LUT_BYTES + xs_bytes +
                                               size_t(NAT_WARPS) * NAT_STAGES * stage_bytes);
    const int w = (edge || heads) ? int(blockIdx.x) * NAT_WARPS + warp : warp * int(gridDim.x) + int(blockIdx.x);
    const int W = p.total_warps;
    const bool active = w < W;
    int h_cu0 = 0, h_cu1 = 0, h_head = 0;
    if (EPI == EPI_F32 && heads) heads_cta_range(p, int(blockIdx.x), h_cu0, h_cu1, h_head);
    const int64_t u_begin = !active ? 0
                            : heads ? h_cu0 + int64_t(h_cu1 - h_cu0) * warp / NAT_WARPS
                                    : unit_begin(p.units, w, W);
    const int64_t u_end = !active ? 0
                          : heads ? h_cu0 + int64_t(h_cu1 - h_cu0) * (warp + 1) / NAT_WARPS
                                  : unit_begin(p.units, w + 1, W);
    const int n_chunks = int((u_end - u_begin + stage_units - 1) / stage_units);

    auto issue = [&](int chunk) {   // lane 0 only
        const int64_t u0 = u_begin + int64_t(chunk) * stage_units;
        const int cnt = int(min(int64_t(stage_units), u_end - u0));
        uint64_t* bar = &bars[warp][chunk % NAT_STAGES];
        const uint32_t bytes = uint32_t(cnt) * UNIT_BYTES;
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(ring + (chunk % NAT_STAGES) * stage_bytes, p.packed + u0 * UNIT_BYTES, bytes, bar);
    };

    // Prologue, overlapping the previous kernel: weights only.
    if (lane == 0 && active) {
#pragma unroll
        for (int s = 0; s < NAT_STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
        for (int c = 0; c < NAT_STAGES && c < n_chunks; ++c) issue(c);
    }
    const uint4 wpre = norm_w_chunk<NAT_THREADS>(p);   // in flight with the LUT loads
    const SlotPlan sp = slot_plan(p, threadIdx.x);
    EdgeRed er;
    er.rg = -1;
    if (EPI == EPI_SILU_MUL && edge) er = edge_red_plan(p, warp);
    if (EPI == EPI_F32 && heads) er = heads_red_plan(p, warp);
    build_lut<NAT_THREADS>(lut_s, p.lut);
    pdl_trigger();
    pdl_wait();
    if (EPI == EPI_F32 && heads) {
        if (!XG) stage_merge(p, xs, h_head, edge_red);   // edge_red is free until the loop ends
    } else if (!XG) {
        stage_x<NAT_THREADS, EPI == EPI_SILU_MUL>(p, xs, &wpre, &sp);
    }
    __syncthreads();
    if (!active) return;

    const uint32_t lut_base = smem_u32(lut_s);
    const uint32_t laneword = uint32_t(lane) << 2;
    const int first_rg = int(u_begin / p.KB);
    const bool xlane = g < p.M;
    const __half* xrow = XG ? p.x + (xlane ? g : 0) * p.x_stride + 16 * t : xs + (xlane ? g : 0) * p.K + 16 * t;
    uint32_t xb[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    int cur_rg = first_rg;
    int seg_b0 = int(u_begin - int64_t(first_rg) * p.KB);
    int rg = first_rg, b = seg_b0;   // (row group, block) of the next unit, advanced incrementally
    // EDGE: this warp's sums of a row group it shares (rows 16 tile + g (+8), batch row 0)
    auto keep = [&](int r) {
        float* d = edge_red + (warp * 2 + (r == first_rg ? 0 : 1)) * 32;
        if (t == 0) {
            d[g] = acc[0][0];
            d[8 + g] = acc[0][2];
            d[16 + g] = acc[1][0];
            d[24 + g] = acc[1][2];
        }
    };
    bool ok = true;

    for (int c = 0; c < n_chunks; ++c) {
        const int stage = c % NAT_STAGES;
        if (!mbar_wait(&bars[warp][stage], uint32_t((c / NAT_STAGES) & 1), err, 2)) {
            // give the other copies in flight a bounded chance to land, then leave
            for (int c2 = c + 1; c2 < n_chunks && c2 < c + NAT_STAGES; ++c2)
                mbar_wait(&bars[warp][c2 % NAT_STAGES], uint32_t((c2 / NAT_STAGES) & 1), err, 2);
            ok = false;
            break;
        }
        const int64_t u0 = u_begin + int64_t(c) * stage_units;
        const int cnt = int(min(int64_t(stage_units), u_end - u0));
        const uint8_t* sbuf = ring + stage * stage_bytes;
        for (int j = 0; j < cnt; ++j) {
            if (rg != cur_rg) {   // the previous group ended inside this range at block KB-1
                if (seg_b0 == 0) {
                    epilogue<EPI>(p, 2 * cur_rg, acc[0], g, t);
                    epilogue<EPI>(p, 2 * cur_rg + 1, acc[1], g, t);
                } else if (edge || heads) {
                    keep(cur_rg);
                } else {
                    flush_partial<EPI, 2>(p, cur_rg, acc, w, first_rg, lane, g, t);
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
                cur_rg = rg;
                seg_b0 = 0;
            }
            if (xlane) {
                uint4 x0, x1;
                if (XG) {
                    x0 = __ldg(reinterpret_cast<const uint4*>(xrow + 64 * b));
                    x1 = __ldg(reinterpret_cast<const uint4*>(xrow + 64 * b + 8));
                } else {
                    x0 = lds128(xrow + 64 * b);
                    x1 = lds128(xrow + 64 * b + 8);
                }
                xb[0] = x0.x; xb[1] = x0.y; xb[2] = x0.z; xb[3] = x0.w;
                xb[4] = x1.x; xb[5] = x1.y; xb[6] = x1.z; xb[7] = x1.w;
            }
            mma_unit_smem(sbuf + j * UNIT_BYTES, xb, lut_base, laneword, lane, g, acc);
            if (++b == p.KB) {
                b = 0;
                ++rg;
            }
        }
        __syncwarp();
        if (lane == 0 && c + NAT_STAGES < n_chunks) {
            fence_proxy_async();
            issue(c + NAT_STAGES);
        }
    }
    if (ok && u_end > u_begin) {
        if (seg_b0 == 0 && b == 0) {   // the range ended exactly at the end of cur_rg
            epilogue<EPI>(p, 2 * cur_rg, acc[0], g, t);
            epilogue<EPI>(p, 2 * cur_rg + 1, acc[1], g, t);
        } else if (edge || heads) {
            keep(cur_rg);
        } else {
            flush_partial<EPI, 2>(p, cur_rg, acc, w, first_rg, lane, g, t);
        }
    }
    if (EPI == EPI_SILU_MUL && edge) {   // every warp of the CTA is active (host-checked) and gets here
        __syncthreads();
        edge_finish(p, er, edge_red, lane);
        return;
    }
    if (EPI == EPI_F32 && heads) {
        __syncthreads();
        heads_finish(p, er, edge_red, lane);
        return;
    }
    if (ok) finish_launch<EPI>(p, lane);
}

// ---------------------------------------------------------------------------
// Native-layout kernel, CTA-level split-K, for launches with fewer than two
// row groups per SM: CTA c owns the whole row groups
// [R*c/G, R*(c+1)/G).  Each row group is split over the 16 warps by blocks,
// every warp streams its slice through its private two-stage ring (one bulk
// copy per chunk of up to `stage_units` units), and the 16 partial fragments
// are added in shared memory in warp order by the group's reducer warp (group
// index mod 16), which runs the epilogue.  No cross-CTA reduction.
//
// The red buffer [16 warps][32 lanes][8 floats] is single-buffered:
// `full` completes when all 16 warps wrote segment j, `empty` when its reducer
// has read it, and no warp writes segment j + 1 before that.

template <int EPI, bool XG>
__global__ void __launch_bounds__(NAT_THREADS, 1)
    nf4_gemv_cta_kernel(const __grid_constant__ Params p, int stage_units, int* err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NAT_WARPS][NAT_STAGES];
    __shared__ __align__(8) uint64_t bar_full, bar_empty;
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem_raw);
    __half* xs = reinterpret_cast<__half*>(smem_raw + LUT_BYTES);
    const int xs_bytes = XG ? 0 : (p.M * p.K * 2 + 127) / 128 * 128;
    float4* red = reinterpret_cast<float4*>(smem_raw + LUT_BYTES + xs_bytes);   // [16][32][2]
    __half* res_s = reinterpret_cast<__half*>(smem_raw + LUT_BYTES + xs_bytes + NAT_WARPS * 32 * 32);
    const int res_bytes = (p.res_rows * p.M * 2 + 127) / 128 * 128;
    const int stage_bytes = stage_units * UNIT_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem_raw + LUT_BYTES + xs_bytes + NAT_WARPS * 32 * 32 + res_bytes +
                    size_t(warp) * NAT_STAGES * stage_bytes;
    const int c = blockIdx.x;
    const int G = gridDim.x;
    const int KB = p.KB;
    const int64_t n_rg = p.units / KB;
    // whole row groups; SLOTS: an equal share of all units (at most two row groups, N / 32 <= G)
    const int64_t u_begin = EPI == EPI_SLOTS ? p.units * c / G : n_rg * c / G * KB;
    const int64_t u_end = EPI == EPI_SLOTS ? p.units * (c + 1) / G : n_rg * (c + 1) / G * KB;
    const int rg_first = int(u_begin / KB);
    const int rg_last = u_end > u_begin ? int((u_end - 1) / KB) : rg_first - 1;

    // this warp's block slice [a, b) of segment rg
    auto slice = [&](int rg, int& a, int& b) {
        const int64_t base = int64_t(rg) * KB;
        const int s0 = int(max(u_begin, base) - base);
        const int s1 = int(min(u_end, base + KB) - base);
        const int len = s1 - s0;
        a = s0 + len * warp / NAT_WARPS;
        b = s0 + len * (warp + 1) / NAT_WARPS;
    };
    // issue cursor over this warp's chunks (segment by segment)
    int is_rg = rg_first, is_off = 0, is_b = 0;
    {
        int a, b;
        if (is_rg <= rg_last) {
            slice(is_rg, a, b);
            is_off = a;
            is_b = b;
        }
    }
    int issued = 0;
    auto issue_next = [&]() {   // lane 0 only; returns false when no chunk is left
        while (is_rg <= rg_last && is_off >= is_b) {
            ++is_rg;
            if (is_rg > rg_last) return false;
            int a, b;
            slice(is_rg, a, b);
            is_off = a;
            is_b = b;
        }
        if (is_rg > rg_last) return false;
        const int cnt = min(stage_units, is_b - is_off);
        const int st = issued % NAT_STAGES;
        uint64_t* bar = &bars[warp][st];
        const uint32_t bytes = uint32_t(cnt) * UNIT_BYTES;
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(ring + st * stage_bytes, p.packed + (int64_t(is_rg) * KB + is_off) * UNIT_BYTES, bytes, bar);
        is_off += cnt;
        ++issued;
        return true;
    };

    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < NAT_STAGES; ++st) mbar_init(&bars[warp][st], 1);
        if (warp == 0) {
            mbar_init(&bar_full, NAT_WARPS);
            mbar_init(&bar_empty, 1);
        }
        fence_mbar_init();
        for (int k = 0; k < NAT_STAGES; ++k)
            if (!issue_next()) break;
    }
    const uint4 wpre = norm_w_chunk<NAT_THREADS>(p);   // in flight with the LUT loads
    const SlotPlan sp = slot_plan(p, threadIdx.x);
    const EdgePlan ep = edge_plan(p, threadIdx.x);
    build_lut<NAT_THREADS>(lut_s, p.lut);
    pdl_trigger();
    pdl_wait();
    // The residual rows of this CTA's row groups, read with x so that the
    // epilogue does not wait on L2 (out may alias residual: these rows are
    // written only by this CTA, after this read).
    const int res_row0 = rg_first * UNIT_ROWS;
    const int res_n = (rg_last - rg_first + 1) * UNIT_ROWS;
    // Up to 4 values per thread are requested before x and stored after it,
    // so both reads share one L2 round trip.
    const bool res_staged = EPI == EPI_RESIDUAL && p.res_rows > 0 && res_n <= p.res_rows &&
                            p.M * res_n <= 4 * NAT_THREADS;
    __half rv[4];
    if (res_staged) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = threadIdx.x + u * NAT_THREADS;
            if (i < p.M * res_n) rv[u] = __ldcg(p.residual + (i / res_n) * p.res_stride + res_row0 + i % res_n);
        }
    }
    if (!XG) stage_x<NAT_THREADS>(p, xs, &wpre, &sp, &ep);
    if (res_staged) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = threadIdx.x + u * NAT_THREADS;
            if (i < p.M * res_n) res_s[(i / res_n) * p.res_rows + i % res_n] = rv[u];
        }
    }
    __syncthreads();

    const uint32_t lut_base = smem_u32(lut_s);
    const uint32_t laneword = uint32_t(lane) << 2;
    const bool xlane = g < p.M;
    const __half* xrow = XG ? p.x + (xlane ? g : 0) * p.x_stride + 16 * t : xs + (xlane ? g : 0) * p.K + 16 * t;
    uint32_t xb[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    int consumed = 0;
    bool ok = true;

    for (int rg = rg_first, j = 0; rg <= rg_last; ++rg, ++j) {
        int a, b;
        slice(rg, a, b);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int off = a; off < b && ok;) {
            const int cnt = min(stage_units, b - off);
            const int st = consumed % NAT_STAGES;
            if (!mbar_wait(&bars[warp][st], uint32_t((consumed / NAT_STAGES) & 1), err, 2)) {
                ok = false;
                break;
            }
            const uint8_t* sbuf = ring + st * stage_bytes;
            for (int jj = 0; jj < cnt; ++jj) {
                const int blk = off + jj;
                if (xlane) {
                    uint4 x0, x1;
                    if (XG) {
                        x0 = __ldg(reinterpret_cast<const uint4*>(xrow + 64 * blk));
                        x1 = __ldg(reinterpret_cast<const uint4*>(xrow + 64 * blk + 8));
                    } else {
                        x0 = lds128(xrow + 64 * blk);
                        x1 = lds128(xrow + 64 * blk + 8);
                    }
                    xb[0] = x0.x; xb[1] = x0.y; xb[2] = x0.z; xb[3] = x0.w;
                    xb[4] = x1.x; xb[5] = x1.y; xb[6] = x1.z; xb[7] = x1.w;
                }
                mma_unit_smem(sbuf + jj * UNIT_BYTES, xb, lut_base, laneword, lane, g, acc);
            }
            ++consumed;
            off += cnt;
            __syncwarp();
            if (lane == 0) {
                fence_proxy_async();
                issue_next();
            }
        }
        if (!ok) break;
        // ---- segment reduction in shared memory
        if (j > 0 && !mbar_wait(&bar_empty, uint32_t((j - 1) & 1), err, 3)) {
            ok = false;
            break;
        }
        red[(warp * 32 + lane) * 2] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
        red[(warp * 32 + lane) * 2 + 1] = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_full);
        if (warp == (j & (NAT_WARPS - 1))) {
            if (!mbar_wait(&bar_full, uint32_t(j & 1), err, 3)) {
                ok = false;
                break;
            }
            float r[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
            for (int ww = 0; ww < NAT_WARPS; ++ww) {
                const float4 v0 = red[(ww * 32 + lane) * 2], v1 = red[(ww * 32 + lane) * 2 + 1];
                r[0][0] += v0.x; r[0][1] += v0.y; r[0][2] += v0.z; r[0][3] += v0.w;
                r[1][0] += v1.x; r[1][1] += v1.y; r[1][2] += v1.z; r[1][3] += v1.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_empty);
            const int64_t base = int64_t(rg) * KB;
            if (EPI == EPI_SLOTS) {   // this CTA's sums of row group rg, rows 16 tile + g (+8), batch rows 2t, 2t+1
                float* slot = reinterpret_cast<float*>(p.out) + (int64_t(c) * SLOTS_PER_CTA + (rg - rg_first)) * p.M * 32;
#pragma unroll
                for (int tl = 0; tl < 2; ++tl)
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int m = 2 * t + e;
                            if (m < p.M) slot[m * 32 + 16 * tl + g + 8 * hr] = r[tl][2 * hr + e];
                        }
            } else if (u_begin <= base && u_end >= base + KB) {
                const __half* rs = res_staged ? res_s : nullptr;
                epilogue<EPI>(p, 2 * rg, r[0], g, t, 0, rs, res_row0, p.res_rows);
                epilogue<EPI>(p, 2 * rg + 1, r[1], g, t, 0, rs, res_row0, p.res_rows);
            } else {
                flush_partial<EPI, 2>(p, rg, r, c, rg_first, lane, g, t);
            }
        }
    }
    // every copy this warp issued has been consumed unless a wait gave up
    if (!ok && lane == 0)
        for (; consumed < issued; ++consumed)
            mbar_wait(&bars[warp][consumed % NAT_STAGES], uint32_t((consumed / NAT_STAGES) & 1), err, 2);
    __syncthreads();
    if (warp == 0 && ok) finish_launch<EPI>(p, lane);
}

// ---------------------------------------------------------------------------
// Reference-layout kernel (packed [N, K/2], absmax [K/64, N]) for callers that
// hand over the reference's tensors per call; 16-row x 64-k units.

constexpr int REF_WARPS = 16;
constexpr int REF_THREADS = REF_WARPS * 32;
constexpr int REF_BATCH = 8;

template <typename AbsT, int EPI>
__global__ void __launch_bounds__(REF_THREADS, 1) nf4_gemv_ref_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(16) uint32_t lut_s[];
    __half* xs = reinterpret_cast<__half*>(lut_s + LUT_WORDS);
    build_lut<REF_THREADS>(lut_s, p.lut);
    pdl_trigger();
    pdl_wait();
    stage_x<REF_THREADS>(p, xs);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int w = blockIdx.x * REF_WARPS + warp;
    if (w >= p.total_warps) return;
    const int W = p.total_warps;
    const int64_t u_begin = unit_begin(p.units, w, W), u_end = unit_begin(p.units, w + 1, W);
    const uint32_t lut_base = smem_u32(lut_s);
    const uint32_t laneword = uint32_t(lane) << 2;
    const int first_tile = int(u_begin / p.KB);
    const int64_t row_bytes = p.K / 2;
    const __half* xrow = xs + (g < p.M ? g : 0) * p.K + 16 * t;

    for (int64_t u = u_begin; u < u_end;) {
        const int tile = int(u / p.KB);
        const int b0 = int(u % p.KB);
        const int span = int(min(u_end - u, int64_t(p.KB - b0)));
        const int r0 = tile * 16;
        const uint8_t* wrow0 = p.packed + int64_t(r0 + g) * row_bytes + 8 * t;
        const uint8_t* wrow1 = wrow0 + 8 * row_bytes;
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};

        for (int i = 0; i < span; i += REF_BATCH) {
            const int nb = min(REF_BATCH, span - i);
            uint2 wa[REF_BATCH], wb[REF_BATCH];
            float am0[REF_BATCH], am1[REF_BATCH];
#pragma unroll
            for (int j = 0; j < REF_BATCH; ++j) {
                if (j < nb) {
                    const int b = b0 + i + j;
                    wa[j] = ldg_stream64(wrow0 + 32 * b);
                    wb[j] = ldg_stream64(wrow1 + 32 * b);
                    am0[j] = absmax_at<AbsT>(p.absmax, int64_t(b) * p.N + r0 + g);
                    am1[j] = absmax_at<AbsT>(p.absmax, int64_t(b) * p.N + r0 + g + 8);
                }
            }
#pragma unroll
            for (int j = 0; j < REF_BATCH; ++j) {
                if (j < nb) {
                    const int b = b0 + i + j;
                    const uint4 x0 = lds128(xrow + 64 * b), x1 = lds128(xrow + 64 * b + 8);
                    const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    const uint32_t ww[4] = {wa[j].x, wa[j].y, wb[j].x, wb[j].y};
                    float blk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t r0w = ww[s >> 1], r1w = ww[2 + (s >> 1)];
                        const uint32_t sel0 = 0x5504u | (uint32_t((s & 1) * 2) << 4);
                        const uint32_t a0 = lds32(lut_base + __byte_perm(r0w, laneword, sel0));
                        const uint32_t a2 = lds32(lut_base + __byte_perm(r0w, laneword, sel0 + 0x10u));
                        const uint32_t a1 = lds32(lut_base + __byte_perm(r1w, laneword, sel0));
                        const uint32_t a3 = lds32(lut_base + __byte_perm(r1w, laneword, sel0 + 0x10u));
                        mma_16816(blk, a0, a1, a2, a3, xb[2 * s], xb[2 * s + 1]);
                    }
                    acc[0][0] += am0[j] * blk[0];
                    acc[0][1] += am0[j] * blk[1];
                    acc[0][2] += am1[j] * blk[2];
                    acc[0][3] += am1[j] * blk[3];
                }
            }
        }
        if (span == p.KB)
            epilogue<EPI>(p, tile, acc[0], g, t);
        else
            flush_partial<EPI, 1>(p, tile, acc, w, first_tile, lane, g, t);
        u += span;
    }
    finish_launch<EPI>(p, lane);
}

// ---------------------------------------------------------------------------
// Batched NF4 GEMM on the tcgen05 tensor cores (M = 1..64 batch rows).
//
// Tile = 128 weight rows (four 32-row groups) x all batch rows; the MMA is
// M = 128 (weight rows) x N = M rounded up to 16 (batch rows) x K = 16, fp16
// operands, fp32 accumulators in tensor memory.  The work
// items are the (tile, 2 k-blocks) pairs, tile-major; CTA c of the one-wave
// grid takes the contiguous range [W*c/G, W*(c+1)/G) (stream-K), so every SM
// decodes the same number of weight units whatever N and K are.  Per item:
//   producer warp   bulk-copies the tile's units of the item's k-blocks into
//                   the weight ring;
//   x producer      TMA-loads the x tiles [N x 64] (128-byte swizzle; rows
//                   past M read as zero);
//   decode warps    warp d (group d / 4, row group d % 4; group g takes the
//                   items j with j % 3 == g) turns its unit's codes into the
//                   fp16 codebook values through a lane-replicated LUT and
//                   stores them as the A tile in tensor memory (lane = weight
//                   row, column = two consecutive k: tcgen05.st.32x32b);
//   MMA thread      per k-block, 4 x tcgen05.mma (K = 16 slices, A from
//                   tensor memory, x by shared-memory descriptor) into a
//                   fresh accumulator, one of four TMEM buffers;
//                   tcgen05.commit signals the buffer full and, after the
//                   item, frees its A and x stages;
//   epilogue warps  8 warps (lane quarter w % 4, batch-column half): per
//                   k-block read the buffer (tcgen05.ld), free it, and add
//                   absmax(row, k-block) x block sum into fp32 registers --
//                   the reference kernel's per-64-block scaling
//                   (src/nova/kernels.py:213-232), so the products are exact
//                   and nothing is rounded to fp16 before the output.  At the
//                   end of a tile segment they run the epilogue (whole tile)
//                   or store the partial; the last contributor of a split tile
//                   (arrival counter) adds all partials in CTA order --
//                   deterministic -- and runs it.
// Every wait is bounded; on a failed wait the roles stop, the MMA thread
// waits for its MMAs and the producers for their copies before TMEM is freed.

constexpr int TC_ROWS = 128;
constexpr int TC_GROUPS = 3;                       // decode warp groups (item j -> group j % 3)
constexpr int TC_DEC_WARPS = 4 * TC_GROUPS;
constexpr int TC_PROD_WARP = TC_DEC_WARPS;         // weight units
constexpr int TC_MMA_WARP = TC_DEC_WARPS + 1;
constexpr int TC_EPI_WARP0 = TC_DEC_WARPS + 2;     // 8 epilogue warps: lane quarter w % 4, column half
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_XPROD_WARP = TC_EPI_WARP0 + TC_EPI_WARPS;   // x tiles
constexpr int TC_WARPS = TC_XPROD_WARP + 1;
constexpr int TC_THREADS = TC_WARPS * 32;
constexpr int TC_AS = 4;                           // A stages (items) in tensor memory
constexpr int TC_XS = 6;                           // x stages (items): the TMA -> MMA -> release chain
constexpr int TC_WS_MAX = 24;                      // weight ring depth: as many stages as shared memory holds
constexpr int TC_KG = 2;                           // k-blocks per work item
static_assert(TC_KG == 1 || TC_KG == 2, "the epilogue's absmax pipeline holds up to 2 k-blocks per item");
constexpr int TC_W_BYTES = 4 * TC_KG * UNIT_BYTES;
constexpr int TC_NB = 4;                           // TMEM accumulator buffers (k-blocks in flight)
constexpr int TC_D_COLS = 64;
constexpr int TC_A_COL0 = TC_NB * TC_D_COLS;       // A stages after the accumulators
constexpr int TC_A_KB_COLS = 32;                   // one k-block of A: 64 fp16 per lane = 32 columns
constexpr int TC_TMEM_COLS = 512;
static_assert(TC_A_COL0 + TC_AS * TC_KG * TC_A_KB_COLS <= TC_TMEM_COLS, "tensor memory columns");
constexpr int TC_LUT_BYTES = 256 * 32 * 4;         // entry v, lane l at word 32 v + l
constexpr int TC_HALF = 32;                        // batch columns per epilogue warp
constexpr int TC_SLOT_FLOATS = 64 * TC_ROWS;       // partial tile [batch row / 4][weight row][4]
constexpr int TC_MAX_M = 64;
constexpr int TC_MAX_TILES = 4096;                 // N up to 524288 rows
constexpr int TC_MIN_ITEMS = 4;                    // work items per CTA at least (bounds the split fan-in)
constexpr int TC_CNT_PER_TILE = 8;                 // split arrivals per tile: lane quarter x column half

struct TcArgs {
    int n_mma;            // MMA N: M rounded up to 16
    int ws;               // weight ring stages (<= TC_WS_MAX)
    int G;                // CTAs
    int64_t W;            // work items = tiles * ceil(KB / TC_KG)
    float* part;          // [G][2][TC_SLOT_FLOATS]
    unsigned* tile_cnt;   // [tiles][8] arrivals of split tiles per lane quarter and column half
    int* err;
};

// The LUT replicated per lane with 128-byte entries (32 KB).
template <int THREADS>
__device__ __forceinline__ void build_lut32(uint32_t* lut_s, const uint32_t* lut) {
    for (int v = threadIdx.x; v < 256 * 4; v += THREADS) {
        const uint32_t w = __ldg(lut + (v >> 2));
        uint4* dst = reinterpret_cast<uint4*>(lut_s + (v >> 2) * 32 + 8 * (v & 3));
        dst[0] = make_uint4(w, w, w, w);
        dst[1] = make_uint4(w, w, w, w);
    }
}

// LUT lookups of the 4 code bytes of `w` (k 2i, 2i+1 from byte i) as one
// 16-byte chunk of fp16 codebook values; lane_b8 = lane << 3.
__device__ __forceinline__ uint4 decode_word(uint32_t lut_base, uint32_t w, uint32_t lane_b8) {
    // byte i -> (byte << 8) | (lane << 3), halved: (byte << 7) | (lane << 2)
    const uint32_t a0 = __byte_perm(w, lane_b8, 0x5504u) >> 1;
    const uint32_t a1 = __byte_perm(w, lane_b8, 0x5514u) >> 1;
    const uint32_t a2 = __byte_perm(w, lane_b8, 0x5524u) >> 1;
    const uint32_t a3 = __byte_perm(w, lane_b8, 0x5534u) >> 1;
    return make_uint4(lds32(lut_base + a0), lds32(lut_base + a1), lds32(lut_base + a2), lds32(lut_base + a3));
}

// Epilogue of one weight row n for the batch rows m0 .. m0 + 31 (v[i] is
// row m0 + i); every lane of the warp calls it (SiLU*up and argmax exchange
// values between lanes).
template <int EPI>
__device__ __forceinline__ void tc_epilogue_row(const Params& p, int n, int rho, const float (&v)[TC_HALF], int m0,
                                                int lane) {
    const bool valid = n < p.N;
    if constexpr (EPI == EPI_SILU_MUL) {   // rows 16i..16i+7 gate, 16i+8..16i+15 the matching up rows
        const bool gate_row = (rho & 15) < 8;
        const int n_out = (n >> 4) * 8 + (n & 7);
#pragma unroll
        for (int i = 0; i < TC_HALF; ++i) {
            const int m = m0 + i;
            if (m >= p.M) break;
            const float upv = __shfl_down_sync(0xffffffffu, v[i], 8);
            if (valid && gate_row) {
                const float gate = __half2float(__float2half_rn(v[i]));
                const float up = __half2float(__float2half_rn(upv));
                const float s = __half2float(__float2half_rn(__fdiv_rn(gate, 1.0f + expf(-gate))));
                p.out[m * p.out_stride + n_out] = __float2half_rn(s * up);
            }
        }
        return;
    } else if constexpr (EPI == EPI_F32) {
        float* o = reinterpret_cast<float*>(p.out);
#pragma unroll
        for (int i = 0; i < TC_HALF; ++i) {
            const int m = m0 + i;
            if (m >= p.M) break;
            if (valid) o[m * p.out_stride + n] = v[i];
        }
        return;
    } else {
#pragma unroll
        for (int i = 0; i < TC_HALF; ++i) {
            const int m = m0 + i;
            if (m >= p.M) break;
            __half h = __float2half_rn(v[i]);
            if (EPI == EPI_RESIDUAL && valid)
                h = __float2half_rn(__half2float(__ldcg(p.residual + m * p.res_stride + n)) + __half2float(h));
            if (valid) p.out[m * p.out_stride + n] = h;
            if (EPI == EPI_ARGMAX) {
                unsigned long long k = valid ? argmax_key(h, n) : 0ull;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                    k = o > k ? o : k;
                }
                if (lane == 0 && k) atomicMax(p.argmax + m, k);
            }
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1)
    nf4_gemm_tc_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap xmap, const TcArgs ta) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_w[TC_WS_MAX], empty_w[TC_WS_MAX], full_x[TC_XS], empty_x[TC_XS];
    __shared__ __align__(8) uint64_t full_a[TC_AS], empty_a[TC_AS], acc_full[TC_NB], acc_empty[TC_NB], drain;
    __shared__ uint32_t tmem_s;
    // 1024-byte aligned carve-up: x ring | LUT | weight ring
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t* x_ring = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
    const int xs_bytes = ta.n_mma * 128;
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(x_ring + TC_XS * TC_KG * xs_bytes);
    uint8_t* w_ring = reinterpret_cast<uint8_t*>(lut_s) + TC_LUT_BYTES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const int KB = p.KB;
    const int n_rg = p.N / UNIT_ROWS;
    const int64_t u0 = ta.W * c / ta.G, u1 = ta.W * (c + 1) / ta.G;
    const int n_items = int(u1 - u0);
    const int NKG = (KB + TC_KG - 1) / TC_KG;   // items per tile
    const int first_tile = int(u0 / NKG);
    const int WS = ta.ws;

    auto issue_w = [&](int j) {   // producer lane 0: the tile's units of item j (row group r: nk consecutive units)
        const int64_t u = u0 + j;
        const int T = int(u / NKG), kb0 = int(u % NKG) * TC_KG;
        const int nk = min(TC_KG, KB - kb0);
        const int rgs = min(4, n_rg - 4 * T);
        const int s = j % WS;
        mbar_arrive_expect_tx(&full_w[s], uint32_t(rgs * nk) * UNIT_BYTES);
        for (int r = 0; r < rgs; ++r)
            bulk_g2s(w_ring + s * TC_W_BYTES + r * TC_KG * UNIT_BYTES,
                     p.packed + (int64_t(4 * T + r) * KB + kb0) * UNIT_BYTES, uint32_t(nk) * UNIT_BYTES, &full_w[s]);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < WS; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&empty_w[s], 4);   // the item's decode warps
        }
        for (int s = 0; s < TC_XS; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&empty_x[s], 1);
        }
        for (int s = 0; s < TC_AS; ++s) {
            mbar_init(&full_a[s], 4);
            mbar_init(&empty_a[s], 1);
        }
        for (int b = 0; b < TC_NB; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TC_EPI_WARPS);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
    }
    if (warp == TC_MMA_WARP) {
        tmem_alloc(&tmem_s, TC_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    int issued_w = 0;
    if (warp == TC_PROD_WARP && lane == 0)   // weights: independent of every earlier kernel
        for (; issued_w < WS && issued_w < n_items; ++issued_w) issue_w(issued_w);
    build_lut32<TC_THREADS>(lut_s, p.lut);
    pdl_trigger();
    pdl_wait();
    __syncthreads();

    if (warp == TC_PROD_WARP) {
        if (lane == 0) {
            bool ok = true;
            for (int j = issued_w; j < n_items; ++j) {
                if (!mbar_wait(&empty_w[j % WS], uint32_t(((j / WS) + 1) & 1), ta.err, 20)) {
                    ok = false;
                    break;
                }
                issue_w(j);
                ++issued_w;
            }
            if (!ok)   // copies in flight land before the CTA ends
                for (int j = max(0, issued_w - WS); j < issued_w; ++j)
                    mbar_wait(&full_w[j % WS], uint32_t((j / WS) & 1), ta.err, 20);
        }
    } else if (warp == TC_XPROD_WARP) {
        if (lane == 0) {
            int issued_x = 0;
            bool ok = true;
            for (int j = 0; j < n_items; ++j) {
                if (j >= TC_XS && !mbar_wait(&empty_x[j % TC_XS], uint32_t(((j / TC_XS) + 1) & 1), ta.err, 21)) {
                    ok = false;
                    break;
                }
                const int s = j % TC_XS;
                const int kb0 = int((u0 + j) % NKG) * TC_KG, nk = min(TC_KG, KB - kb0);
                mbar_arrive_expect_tx(&full_x[s], uint32_t(nk * xs_bytes));
                for (int q = 0; q < nk; ++q)
                    tma_load_2d(x_ring + (s * TC_KG + q) * xs_bytes, &xmap, (kb0 + q) * 64, 0, &full_x[s]);
                ++issued_x;
            }
            if (!ok)
                for (int j = max(0, issued_x - TC_XS); j < issued_x; ++j)
                    mbar_wait(&full_x[j % TC_XS], uint32_t((j / TC_XS) & 1), ta.err, 21);
        }
    } else if (warp < TC_DEC_WARPS) {
        const int grp = warp >> 2, r = warp & 3;
        const uint32_t lut_base = smem_u32(lut_s);
        const uint32_t lane_b8 = uint32_t(lane) << 3;
        int T = int((u0 + grp) / NKG), kg = int((u0 + grp) % NKG);
        for (int j = grp; j < n_items; j += TC_GROUPS) {
            const int nk = min(TC_KG, KB - kg * TC_KG);
            if (!mbar_wait(&full_w[j % WS], uint32_t((j / WS) & 1), ta.err, 22)) break;
            if (j >= TC_AS && !mbar_wait(&empty_a[j % TC_AS], uint32_t(((j / TC_AS) + 1) & 1), ta.err, 23)) break;
            if (4 * T + r < n_rg) {
                for (int q = 0; q < nk; ++q) {
                    const uint8_t* unit = w_ring + (j % WS) * TC_W_BYTES + (r * TC_KG + q) * UNIT_BYTES;
                    const uint4 c0 = lds128(unit + 16 * lane), c1 = lds128(unit + 512 + 16 * lane);
                    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                    // lanes 32r .. 32r + 31 of the stage: column i = k 2i, 2i + 1
                    const uint32_t ta0 = tmem + (uint32_t(32 * r) << 16) +
                                         uint32_t(TC_A_COL0 + ((j % TC_AS) * TC_KG + q) * TC_A_KB_COLS);
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        uint32_t d[16];
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            const uint4 v = decode_word(lut_base, cw[4 * hh + ch], lane_b8);
                            d[4 * ch] = v.x; d[4 * ch + 1] = v.y; d[4 * ch + 2] = v.z; d[4 * ch + 3] = v.w;
                        }
                        tmem_st16(ta0 + uint32_t(16 * hh), d);
                    }
                }
                tmem_wait_st();
            }
            kg += TC_GROUPS;
            while (kg >= NKG) {
                kg -= NKG;
                ++T;
            }
            tc_fence_before();   // the A tile's tensor-memory stores before the MMA thread's wait
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty_w[j % WS]);
                mbar_arrive(&full_a[j % TC_AS]);
            }
        }
    } else if (warp == TC_MMA_WARP) {   // the whole warp waits, one lane issues (warp kept converged)
        const uint32_t idesc = tc_idesc_f16(TC_ROWS, ta.n_mma);
        const uint64_t bdesc0 = sw128_kmajor_desc(smem_u32(x_ring));   // start address field steps by 16-byte units
        int kbc = 0;   // k-blocks issued: accumulator buffer kbc % TC_NB
        int kg = int(u0 % NKG);
        bool ok = true;
        for (int j = 0; j < n_items && ok; ++j, kg = kg + 1 == NKG ? 0 : kg + 1) {
            const int nk = min(TC_KG, KB - kg * TC_KG);
            if (!mbar_wait(&full_a[j % TC_AS], uint32_t((j / TC_AS) & 1), ta.err, 25)) break;
            if (!mbar_wait(&full_x[j % TC_XS], uint32_t((j / TC_XS) & 1), ta.err, 26)) break;
            for (int q = 0; q < nk; ++q, ++kbc) {
                const int buf = kbc % TC_NB;
                if (kbc >= TC_NB && !mbar_wait(&acc_empty[buf], uint32_t(((kbc / TC_NB) + 1) & 1), ta.err, 24)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a0 = tmem + uint32_t(TC_A_COL0 + ((j % TC_AS) * TC_KG + q) * TC_A_KB_COLS);
                    const uint64_t b0 = bdesc0 + uint64_t((((j % TC_XS) * TC_KG + q) * xs_bytes) >> 4);
                    const uint32_t d0 = tmem + uint32_t(buf * TC_D_COLS);
#pragma unroll
                    for (int k = 0; k < 4; ++k)   // a fresh accumulator per k-block
                        tc_mma_f16_ta(d0, a0 + uint32_t(8 * k), b0 + uint64_t((32 * k) >> 4), idesc, k ? 1u : 0u);
                    tc_commit(&acc_full[buf]);
                }
                __syncwarp();
            }
            if (lane == 0) {   // frees the item's A and x stages once its MMAs have completed
                tc_commit(&empty_a[j % TC_AS]);
                tc_commit(&empty_x[j % TC_XS]);
            }
            __syncwarp();
        }
        if (lane == 0) tc_commit(&drain);   // every MMA of this CTA has completed before TMEM is freed
        __syncwarp();
        mbar_wait(&drain, 0u, ta.err, 27);
    } else {   // epilogue warps
        const int q4 = warp & 3;                          // TMEM lane quarter
        const int half = (warp - TC_EPI_WARP0) >> 2;      // batch columns [32 half, 32 half + 32)
        const int m0 = TC_HALF * half;
        const bool cols = m0 < ta.n_mma;
        const int rho = 32 * q4 + lane;                   // weight row within the tile
        float v[TC_HALF];
        int kbc = 0;
        bool ok = true;
        for (int j = 0; j < n_items && ok;) {
            const int64_t u = u0 + j;
            const int T = int(u / NKG), kg0 = int(u % NKG);
            const int len = min(n_items - j, NKG - kg0);
            const bool whole = kg0 == 0 && len == NKG;
            const bool row_ok = 4 * T + q4 < n_rg;
            // absmax of this lane's row, k-block kb, read from the unit stream in global memory (L2: the
            // producer has just fetched it) two items ahead of its use
            const __half* am_g = reinterpret_cast<const __half*>(
                p.packed + int64_t(4 * T + q4) * KB * UNIT_BYTES + UNIT_CODE_BYTES + 2 * lane);
            auto am_load = [&](int kb) -> unsigned short {
                return (cols && row_ok && kb < KB) ? __ldg(reinterpret_cast<const unsigned short*>(am_g) +
                                                           int64_t(kb) * (UNIT_BYTES / 2))
                                                   : (unsigned short)0;
            };
            unsigned short am_pipe[3][TC_KG];   // items jj, jj + 1, jj + 2
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int q = 0; q < TC_KG; ++q) am_pipe[a][q] = am_load((kg0 + a) * TC_KG + q);
#pragma unroll
            for (int i = 0; i < TC_HALF; ++i) v[i] = 0.f;
            for (int jj = j; jj < j + len && ok; ++jj) {
                const int kb0 = (kg0 + (jj - j)) * TC_KG, nk = min(TC_KG, KB - kb0);
#pragma unroll
                for (int q = 0; q < TC_KG; ++q) am_pipe[2][q] = am_load(kb0 + 2 * TC_KG + q);
                for (int q = 0; q < nk; ++q, ++kbc) {
                    const int buf = kbc % TC_NB;
                    if (!mbar_wait(&acc_full[buf], uint32_t((kbc / TC_NB) & 1), ta.err, 28)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (cols) {   // 16 columns at a time: v += absmax * block sum
                        const float am = __half2float(__ushort_as_half(q ? am_pipe[0][1] : am_pipe[0][0]));
                        const uint32_t ta0 = tmem + (uint32_t(32 * q4) << 16) + uint32_t(buf * TC_D_COLS + m0);
#pragma unroll
                        for (int h16 = 0; h16 < TC_HALF / 16; ++h16) {
                            if (m0 + 16 * h16 < ta.n_mma) {
                                uint32_t d[16];
                                tmem_ld16(ta0 + uint32_t(16 * h16), d);
                                tmem_wait_ld();
#pragma unroll
                                for (int i = 0; i < 16; ++i)
                                    v[16 * h16 + i] = fmaf(am, __uint_as_float(d[i]), v[16 * h16 + i]);
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                }
#pragma unroll
                for (int q = 0; q < TC_KG; ++q) {
                    am_pipe[0][q] = am_pipe[1][q];
                    am_pipe[1][q] = am_pipe[2][q];
                }
            }
            if (!ok) break;
            const int n = T * TC_ROWS + rho;
            bool run = cols;
            if (cols && !whole) {   // split tile: partial to this CTA's slot; per lane quarter and column
                                    // half, the last contributing warp adds the partials in CTA order
                float4* slot = reinterpret_cast<float4*>(ta.part + (int64_t(c) * 2 + (T == first_tile ? 0 : 1)) *
                                                                         TC_SLOT_FLOATS);   // [m / 4][row][4]
#pragma unroll
                for (int f = 0; f < TC_HALF / 4; ++f)
                    if (m0 + 4 * f < p.M)
                        __stcg(slot + (m0 / 4 + f) * TC_ROWS + rho, make_float4(v[4 * f], v[4 * f + 1], v[4 * f + 2],
                                                                                v[4 * f + 3]));
                __threadfence();
                __syncwarp();
                const int cf = owner_of(int64_t(T) * NKG, ta.W, ta.G);
                const int cl = owner_of(int64_t(T) * NKG + NKG - 1, ta.W, ta.G);
                unsigned* cnt = ta.tile_cnt + TC_CNT_PER_TILE * T + 4 * half + q4;
                unsigned last = 0;
                if (lane == 0) last = atomicAdd(cnt, 1u) == unsigned(cl - cf);
                run = __shfl_sync(0xffffffffu, last, 0) != 0;
                if (run) {
                    __threadfence();
#pragma unroll
                    for (int i = 0; i < TC_HALF; ++i) v[i] = 0.f;
                    for (int cc = cf; cc <= cl; ++cc) {
                        const int ft = int((ta.W * cc / ta.G) / NKG);
                        const float4* src = reinterpret_cast<const float4*>(
                            ta.part + (int64_t(cc) * 2 + (T == ft ? 0 : 1)) * TC_SLOT_FLOATS);
                        float4 t4[TC_HALF / 4];
#pragma unroll
                        for (int f = 0; f < TC_HALF / 4; ++f)
                            t4[f] = m0 + 4 * f < p.M ? __ldcg(src + (m0 / 4 + f) * TC_ROWS + rho)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int f = 0; f < TC_HALF / 4; ++f) {
                            v[4 * f] += t4[f].x;
                            v[4 * f + 1] += t4[f].y;
                            v[4 * f + 2] += t4[f].z;
                            v[4 * f + 3] += t4[f].w;
                        }
                    }
                    if (lane == 0) *cnt = 0u;   // re-armed for the next launch
                }
            }
            if (run) tc_epilogue_row<EPI>(p, n, rho, v, m0, lane);
            j += len;
        }
        if (EPI == EPI_ARGMAX && p.token_out) {   // the last epilogue warp to finish runs the step finalize
            __threadfence();
            __syncwarp();
            unsigned last = 0;
            if (lane == 0) last = atomicAdd(p.done, 1u) == unsigned(TC_EPI_WARPS * ta.G - 1);
            if (__shfl_sync(0xffffffffu, last, 0)) {
                __threadfence();
                finalize_step(p, lane);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TC_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, TC_TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Wide NF4 GEMM for M > 64 rows (prefill chunks): a dense contraction, so the
// tile is 128 weight rows x 128 token rows and every MMA is M 128 x N 128 x
// K 16 (full tcgen05 rate per flop).  Each k-block's A tile carries the
// weights as two fp16 terms, hi = fp16(code * absmax) and lo = fp16(code *
// absmax - hi) (the product of two fp16 values is exact in fp32, and so is the
// difference), both multiplied by x into the same TMEM accumulator: code *
// absmax * x to ~2^-22 per product, so K need not be cut at every 64-block
// boundary.  The tensor cores accumulate a group of TW_G k-blocks (64 MMAs)
// into one of two TMEM buffers; the epilogue warps add each group's sums into
// fp32 registers (round to nearest), which keeps the long-K error at the
// level of the reference kernel's per-block fp32 sums
// (src/nova/kernels.py:213-232).  Work items = (weight tile, 128-row token
// tile) pairs, dealt round-robin to a persistent grid; no split-K.
//   producer warp   bulk-copies each k-block's 4 units into the weight ring;
//   x producer      TMA-loads the [128 x 64] x tile of each k-block;
//   decode warps    2 groups (k-block parity) x 4 row groups: LUT -> code,
//                   x absmax in fp32, split into hi/lo, tcgen05.st.32x32b
//                   into the k-block's A stage (hi columns, then lo);
//   MMA thread      per k-block 4 K slices x (hi, lo) MMAs into the group's
//                   buffer; commits free the A / x stages and hand a finished
//                   group to the epilogue;
//   epilogue warps  8 warps (lane quarter x 64 token columns): per group
//                   tcgen05.ld + fp32 add into registers; after the item's
//                   last group the plain / residual / SiLU*up / fp32 epilogue.

constexpr int TW_MT = 128;                         // token rows per tile (MMA N)
constexpr int TW_G = 8;                            // k-blocks per TMEM accumulation group
constexpr int TW_DEC_WARPS = 8;                    // 2 groups x 4 row groups
constexpr int TW_PROD_WARP = TW_DEC_WARPS;
constexpr int TW_MMA_WARP = TW_DEC_WARPS + 1;
constexpr int TW_EPI_WARP0 = TW_DEC_WARPS + 2;     // 8 epilogue warps
constexpr int TW_EPI_WARPS = 8;
constexpr int TW_XPROD_WARP = TW_EPI_WARP0 + TW_EPI_WARPS;
constexpr int TW_WARPS = TW_XPROD_WARP + 1;
constexpr int TW_THREADS = TW_WARPS * 32;
constexpr int TW_COLS = TW_MT / 2;                 // token columns per epilogue warp
constexpr int TW_AS = 4;                           // A stages (k-blocks) in tensor memory
constexpr int TW_XS = 6;                           // x stages (k-blocks), 16 KB each
constexpr int TW_WS_MAX = 16;
constexpr int TW_W_BYTES = 4 * UNIT_BYTES;         // one k-block of a 128-row tile
constexpr int TW_X_BYTES = TW_MT * 128;
constexpr int TW_A_COL0 = 2 * TW_MT;               // accumulators [0, 256), A stages after them
constexpr int TW_A_COLS = 64;                      // hi 32 + lo 32 columns per k-block
static_assert(TW_A_COL0 + TW_AS * TW_A_COLS <= 512, "tensor memory columns");

struct TwArgs {
    int ws;               // weight ring stages
    int m_tiles;
    int64_t items;        // weight tiles * m_tiles
    int* err;
};

// fp16x2 codebook values (k, k+1) times absmax -> hi and lo fp16x2 words
__device__ __forceinline__ void split_hi_lo(uint32_t code2, float am, uint32_t& hi, uint32_t& lo) {
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&code2));
    const float p0 = c.x * am, p1 = c.y * am;   // exact: 11-bit x 11-bit significands
    const __half2 h = __floats2half2_rn(p0, p1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Epilogue of weight row n for token rows m0 .. m0 + 15 (v[i] = row m0 + i).
template <int EPI>
__device__ __forceinline__ void tw_epilogue16(const Params& p, int n, int rho, const float* v, int m0) {
    const bool valid = n < p.N;
    if constexpr (EPI == EPI_SILU_MUL) {   // rows 16i..16i+7 gate, 16i+8..16i+15 the matching up rows
        const bool gate_row = (rho & 15) < 8;
        const int n_out = (n >> 4) * 8 + (n & 7);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int m = m0 + i;
            const float upv = __shfl_down_sync(0xffffffffu, v[i], 8);
            if (m < p.M && valid && gate_row) {
                const float gate = __half2float(__float2half_rn(v[i]));
                const float up = __half2float(__float2half_rn(upv));
                const float s = __half2float(__float2half_rn(__fdiv_rn(gate, 1.0f + expf(-gate))));
                p.out[int64_t(m) * p.out_stride + n_out] = __float2half_rn(s * up);
            }
        }
    } else if constexpr (EPI == EPI_F32) {
        float* o = reinterpret_cast<float*>(p.out);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int m = m0 + i;
            if (m < p.M && valid) o[int64_t(m) * p.out_stride + n] = v[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int m = m0 + i;
            if (m >= p.M || !valid) continue;
            __half h = __float2half_rn(v[i]);
            if (EPI == EPI_RESIDUAL)
                h = __float2half_rn(__half2float(__ldcg(p.residual + int64_t(m) * p.res_stride + n)) +
                                    __half2float(h));
            p.out[int64_t(m) * p.out_stride + n] = h;
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(TW_THREADS, 1)
    nf4_gemm_wide_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap xmap, const TwArgs ta) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_w[TW_WS_MAX], empty_w[TW_WS_MAX], full_x[TW_XS], empty_x[TW_XS];
    __shared__ __align__(8) uint64_t full_a[TW_AS], empty_a[TW_AS], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_s;
    // 1024-byte aligned carve-up: x ring | LUT | weight ring
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t* x_ring = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(x_ring + TW_XS * TW_X_BYTES);
    uint8_t* w_ring = reinterpret_cast<uint8_t*>(lut_s) + TC_LUT_BYTES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = p.KB;
    const int NG = (KB + TW_G - 1) / TW_G;   // accumulation groups per item
    const int n_rg = p.N / UNIT_ROWS;
    const int WS = ta.ws;
    // this CTA's items: i = blockIdx.x + j * gridDim.x; item -> (weight tile, token tile)
    const int n_items = ta.items > blockIdx.x ? int((ta.items - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const int total_kb = n_items * KB;   // k-blocks of all this CTA's items, in order
    auto item_of = [&](int j, int& T, int& mt) {
        const int64_t i = int64_t(blockIdx.x) + int64_t(j) * gridDim.x;
        T = int(i / ta.m_tiles);
        mt = int(i % ta.m_tiles);
    };

    auto issue_w = [&](int g) {   // producer lane 0: the 4 units of global k-block g of this CTA
        int T, mt;
        item_of(g / KB, T, mt);
        const int kb = g % KB;
        const int rgs = min(4, n_rg - 4 * T);
        const int s = g % WS;
        mbar_arrive_expect_tx(&full_w[s], uint32_t(rgs) * UNIT_BYTES);
        for (int r = 0; r < rgs; ++r)
            bulk_g2s(w_ring + s * TW_W_BYTES + r * UNIT_BYTES, p.packed + (int64_t(4 * T + r) * KB + kb) * UNIT_BYTES,
                     UNIT_BYTES, &full_w[s]);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < WS; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&empty_w[s], 4);
        }
        for (int s = 0; s < TW_XS; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&empty_x[s], 1);
        }
        for (int s = 0; s < TW_AS; ++s) {
            mbar_init(&full_a[s], 4);
            mbar_init(&empty_a[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TW_EPI_WARPS);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
    }
    if (warp == TW_MMA_WARP) {
        tmem_alloc(&tmem_s, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    int issued_w = 0;
    if (warp == TW_PROD_WARP && lane == 0)   // weights: independent of every earlier kernel
        for (; issued_w < WS && issued_w < total_kb; ++issued_w) issue_w(issued_w);
    build_lut32<TW_THREADS>(lut_s, p.lut);
    pdl_trigger();
    pdl_wait();
    __syncthreads();

    if (warp == TW_PROD_WARP) {
        if (lane == 0) {
            bool ok = true;
            for (int g = issued_w; g < total_kb; ++g) {
                if (!mbar_wait(&empty_w[g % WS], uint32_t(((g / WS) + 1) & 1), ta.err, 30)) {
                    ok = false;
                    break;
                }
                issue_w(g);
                ++issued_w;
            }
            if (!ok)
                for (int g = max(0, issued_w - WS); g < issued_w; ++g)
                    mbar_wait(&full_w[g % WS], uint32_t((g / WS) & 1), ta.err, 30);
        }
    } else if (warp == TW_XPROD_WARP) {
        if (lane == 0) {
            int issued_x = 0;
            bool ok = true;
            for (int g = 0; g < total_kb; ++g) {
                if (g >= TW_XS && !mbar_wait(&empty_x[g % TW_XS], uint32_t(((g / TW_XS) + 1) & 1), ta.err, 31)) {
                    ok = false;
                    break;
                }
                int T, mt;
                item_of(g / KB, T, mt);
                const int s = g % TW_XS;
                mbar_arrive_expect_tx(&full_x[s], uint32_t(TW_X_BYTES));
                tma_load_2d(x_ring + s * TW_X_BYTES, &xmap, (g % KB) * 64, mt * TW_MT, &full_x[s]);
                ++issued_x;
            }
            if (!ok)
                for (int g = max(0, issued_x - TW_XS); g < issued_x; ++g)
                    mbar_wait(&full_x[g % TW_XS], uint32_t((g / TW_XS) & 1), ta.err, 31);
        }
    } else if (warp < TW_DEC_WARPS) {
        const int grp = warp >> 2, r = warp & 3;
        const uint32_t lut_base = smem_u32(lut_s);
        const uint32_t lane_b8 = uint32_t(lane) << 3;
        for (int g = grp; g < total_kb; g += 2) {
            int T, mt;
            item_of(g / KB, T, mt);
            if (!mbar_wait(&full_w[g % WS], uint32_t((g / WS) & 1), ta.err, 32)) break;
            if (g >= TW_AS && !mbar_wait(&empty_a[g % TW_AS], uint32_t(((g / TW_AS) + 1) & 1), ta.err, 33)) break;
            if (4 * T + r < n_rg) {
                const uint8_t* unit = w_ring + (g % WS) * TW_W_BYTES + r * UNIT_BYTES;
                const uint4 c0 = lds128(unit + 16 * lane), c1 = lds128(unit + 512 + 16 * lane);
                const float am = __half2float(*reinterpret_cast<const __half*>(unit + UNIT_CODE_BYTES + 2 * lane));
                const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const uint32_t ta0 =
                    tmem + (uint32_t(32 * r) << 16) + uint32_t(TW_A_COL0 + (g % TW_AS) * TW_A_COLS);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t dh[16], dl[16];
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) {
                        const uint4 v = decode_word(lut_base, cw[4 * hh + ch], lane_b8);
                        split_hi_lo(v.x, am, dh[4 * ch], dl[4 * ch]);
                        split_hi_lo(v.y, am, dh[4 * ch + 1], dl[4 * ch + 1]);
                        split_hi_lo(v.z, am, dh[4 * ch + 2], dl[4 * ch + 2]);
                        split_hi_lo(v.w, am, dh[4 * ch + 3], dl[4 * ch + 3]);
                    }
                    tmem_st16(ta0 + uint32_t(16 * hh), dh);
                    tmem_st16(ta0 + uint32_t(32 + 16 * hh), dl);
                }
                tmem_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty_w[g % WS]);
                mbar_arrive(&full_a[g % TW_AS]);
            }
        }
    } else if (warp == TW_MMA_WARP) {   // the whole warp waits, one lane issues
        const uint32_t idesc = tc_idesc_f16(TC_ROWS, TW_MT);
        const uint64_t bdesc0 = sw128_kmajor_desc(smem_u32(x_ring));
        int gc = 0;   // accumulation groups started: buffer gc % 2
        for (int g = 0; g < total_kb; ++g) {
            const int kb = g % KB;
            const bool first = kb % TW_G == 0, last = kb % TW_G == TW_G - 1 || kb == KB - 1;
            const int buf = gc & 1;
            if (first && gc >= 2 && !mbar_wait(&acc_empty[buf], uint32_t(((gc >> 1) + 1) & 1), ta.err, 34)) break;
            if (!mbar_wait(&full_a[g % TW_AS], uint32_t((g / TW_AS) & 1), ta.err, 35)) break;
            if (!mbar_wait(&full_x[g % TW_XS], uint32_t((g / TW_XS) & 1), ta.err, 36)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a0 = tmem + uint32_t(TW_A_COL0 + (g % TW_AS) * TW_A_COLS);
                const uint64_t b0 = bdesc0 + uint64_t(((g % TW_XS) * TW_X_BYTES) >> 4);
                const uint32_t d0 = tmem + uint32_t(buf * TW_MT);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint64_t bk = b0 + uint64_t((32 * k) >> 4);
                    tc_mma_f16_ta(d0, a0 + uint32_t(8 * k), bk, idesc, (first && k == 0) ? 0u : 1u);
                    tc_mma_f16_ta(d0, a0 + uint32_t(32 + 8 * k), bk, idesc, 1u);
                }
                tc_commit(&empty_a[g % TW_AS]);
                tc_commit(&empty_x[g % TW_XS]);
                if (last) tc_commit(&acc_full[buf]);
            }
            __syncwarp();
            if (last) ++gc;
        }
        if (lane == 0) tc_commit(&drain);   // every MMA of this CTA has completed before TMEM is freed
        __syncwarp();
        mbar_wait(&drain, 0u, ta.err, 37);
    } else if (warp < TW_EPI_WARP0 + TW_EPI_WARPS) {   // epilogue warps
        const int q4 = warp & 3;
        const int half = (warp - TW_EPI_WARP0) >> 2;
        const int rho = 32 * q4 + lane;
        float v[TW_COLS];
        int gc = 0;
        bool ok = true;
        for (int j = 0; j < n_items && ok; ++j) {
            int T, mt;
            item_of(j, T, mt);
            const int m0 = mt * TW_MT + half * TW_COLS;   // first token row of this warp's columns
            const int ncols = min(TW_COLS, p.M - m0);       // may be <= 0 for a ragged token tile
#pragma unroll
            for (int i = 0; i < TW_COLS; ++i) v[i] = 0.f;
            for (int grp = 0; grp < NG; ++grp, ++gc) {
                const int buf = gc & 1;
                if (!mbar_wait(&acc_full[buf], uint32_t((gc >> 1) & 1), ta.err, 38)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c16 = 0; c16 < TW_COLS / 16; ++c16) {
                    if (16 * c16 < ncols) {
                        uint32_t d[16];
                        tmem_ld16(tmem + (uint32_t(32 * q4) << 16) + uint32_t(buf * TW_MT + half * TW_COLS + 16 * c16),
                                  d);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[16 * c16 + i] += __uint_as_float(d[i]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
            }
            if (!ok) break;
            const int n = T * TC_ROWS + rho;
#pragma unroll
            for (int c16 = 0; c16 < TW_COLS / 16; ++c16)
                if (16 * c16 < ncols) tw_epilogue16<EPI>(p, n, rho, v + 16 * c16, m0 + 16 * c16);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TW_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------- quantizer / packer

__global__ void nf4_quantize_kernel(const __half* __restrict__ w, int64_t n_blocks, int kb, int N,
                                    const float* __restrict__ mid, uint8_t* __restrict__ packed, void* absmax,
                                    int absmax_fp32) {
    __shared__ float smid[15];
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x < 15) smid[threadIdx.x] = mid[threadIdx.x];
    __syncthreads();
    for (int64_t blk = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; blk < n_blocks;
         blk += int64_t(gridDim.x) * blockDim.x) {
        const int64_t n = blk / kb, b = blk % kb;
        const __half* src = w + blk * 64;
        float am = 0.f;
        for (int i = 0; i < 64; ++i) am = fmaxf(am, fabsf(__half2float(src[i])));
        const float safe = am > 0.f ? am : 1.0f;
        uint8_t* dst = packed + blk * 32;
        for (int i = 0; i < 64; i += 2) {
            uint32_t idx[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v = __fdiv_rn(__half2float(src[i + e]), safe);
                uint32_t c = 0;
#pragma unroll
                for (int j = 0; j < 15; ++j) c += (smid[j] < v) ? 1u : 0u;
                idx[e] = c;
            }
            dst[i / 2] = uint8_t((idx[0] << 4) | idx[1]);
        }
        if (absmax_fp32)
            reinterpret_cast<float*>(absmax)[b * N + n] = am;
        else
            reinterpret_cast<__half*>(absmax)[b * N + n] = __float2half_rn(am);
    }
}

template <typename AbsT>
__global__ void nf4_dequant_kernel(const uint8_t* __restrict__ packed, const void* absmax,
                                   const uint32_t* __restrict__ lut, __half* __restrict__ out, int64_t N, int K) {
    pdl_trigger();
    pdl_wait();
    const int64_t total = N * (K / 2);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t n = i / (K / 2);
        const int kk = int(i % (K / 2)) * 2;
        const uint32_t e = __ldg(lut + packed[i]);
        const float a = absmax_at<AbsT>(absmax, int64_t(kk / 64) * N + n);
        const float c0 = f16_bits_to_f32(uint16_t(e & 0xffff)), c1 = f16_bits_to_f32(uint16_t(e >> 16));
        *reinterpret_cast<__half2*>(out + n * K + kk) = __floats2half2_rn(c0 * a, c1 * a);
    }
}

// One thread per (unit, lane): the lane's 2 x 16 code bytes and, for t == 0,
// the four absmax values of its lane group.
// TC = true: the tcgen05 GEMM's variant of the unit layout -- lane (g, t) holds,
// for each of its rows, the code bytes 2t + 8p and 2t + 8p + 1 (p = 0..3; the
// k values 4t + 16p .. 4t + 16p + 3) instead of bytes 8t .. 8t + 7, so that the
// decoded fp16x2 values of a lane are exactly its share of a 16x256b tensor-
// memory store in natural k order.
template <typename AbsT, bool TC>
__global__ void nf4_pack_native_kernel(const uint8_t* __restrict__ packed, const void* absmax,
                                       uint8_t* __restrict__ out, int64_t n_units, int KB, int N) {
    pdl_trigger();
    pdl_wait();
    const int64_t row_bytes = int64_t(KB) * 32;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_units * 32;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t u = i >> 5;
        const int lane = int(i & 31), g = lane >> 2, t = lane & 3;
        const int64_t rg = u / KB;
        const int b = int(u % KB);
        uint8_t* rec = out + u * UNIT_BYTES;
        if constexpr (TC) {   // GEMM units: row `lane` owns bytes 16 lane (k 0..31) and 512 + 16 lane (k 32..63)
            const int64_t row = rg * UNIT_ROWS + lane;
            const uint2* src = reinterpret_cast<const uint2*>(packed + row * row_bytes + 32 * b);
            uint2* d0 = reinterpret_cast<uint2*>(rec + 16 * lane);
            uint2* d1 = reinterpret_cast<uint2*>(rec + 512 + 16 * lane);
            d0[0] = src[0];
            d0[1] = src[1];
            d1[0] = src[2];
            d1[1] = src[3];
            const float a = absmax_at<AbsT>(absmax, int64_t(b) * N + row);
            reinterpret_cast<__half*>(rec + UNIT_CODE_BYTES)[lane] = __float2half_rn(a);
        } else {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int64_t row = rg * UNIT_ROWS + g + 8 * r;
                const uint2 v = *reinterpret_cast<const uint2*>(packed + row * row_bytes + 32 * b + 8 * t);
                // rows g, g+8 -> first half, rows g+16, g+24 -> second half; 16 bytes per lane in each
                *reinterpret_cast<uint2*>(rec + (r >> 1) * 512 + 16 * lane + 8 * (r & 1)) = v;
                if (t == 0) {
                    const float a = absmax_at<AbsT>(absmax, int64_t(b) * N + row);
                    reinterpret_cast<__half*>(rec + UNIT_CODE_BYTES)[4 * g + r] = __float2half_rn(a);
                }
            }
        }
    }
}

}  // namespace nf4
}  // namespace nova

using namespace nova;
using namespace nova::nf4;

// Workspace layout: [partial slots of every warp of the persistent grid |
// per-row-tile arrival counters + the finalize counter].  The partial region
// has the same size for every N (it is sized for the largest grid either
// kernel uses), so one workspace sized for the largest N serves every GEMV
// on a stream: each launch leaves its counters at zero.
static int64_t max_warps() { return int64_t(sm_count()) * 16; }
static int64_t partial_bytes() { return max_warps() * 2 * 32 * 32; }

static int* gemv_error_word(void* ws) { return reinterpret_cast<int*>((uint8_t*)ws + partial_bytes() + 4); }

// Copy a device error word to the host and clear it when set (synchronous).
static int read_error_word(int* dev_word, int* host_value, const char* what) {
    if (!dev_word || !host_value) return fail(NOVA_ERR_INVALID, "NULL argument");
    if (cudaMemcpy(host_value, dev_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "reading the %s error word failed", what);
    }
    if (*host_value && cudaMemset(dev_word, 0, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "clearing the %s error word failed", what);
    }
    return NOVA_OK;
}

extern "C" int nova_nf4_gemv_read_error(void* workspace, int* host_value) {
    if (!workspace) return fail(NOVA_ERR_INVALID, "NULL workspace");
    return read_error_word(gemv_error_word(workspace), host_value, "GEMV");
}

extern "C" int nova_nf4_workspace_bytes(int64_t n, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (n <= 0 || n % 16) return fail(NOVA_ERR_INVALID, "N must be a positive multiple of 16");
    *bytes = partial_bytes() + 256 + ((n / 16) * 4 + 255) / 256 * 256;   // done + error word, counters
    return NOVA_OK;
}

extern "C" int nova_nf4_native_bytes(int64_t n, int64_t k, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (n <= 0 || n % UNIT_ROWS || k <= 0 || k % 64)
        return fail(NOVA_ERR_INVALID, "native layout needs N %% 32 == 0 and K %% 64 == 0");
    *bytes = (n / UNIT_ROWS) * (k / 64) * UNIT_BYTES;
    return NOVA_OK;
}

template <bool TC>
static int pack_units(const void* packed, const void* absmax, int absmax_fp32, void* out, int64_t n, int64_t k,
                      void* stream) {
    if (n <= 0 || n % UNIT_ROWS || k <= 0 || k % 64)
        return fail(NOVA_ERR_INVALID, "native layout needs N %% 32 == 0 and K %% 64 == 0");
    if (!packed || !absmax || !out) return fail(NOVA_ERR_INVALID, "NULL pointer");
    auto mis = [](const void* ptr, int al) { return reinterpret_cast<uintptr_t>(ptr) % al != 0; };
    if (mis(packed, 8) || mis(out, 16)) return fail(NOVA_ERR_ALIGN, "packed must be 8-byte, out 16-byte aligned");
    const int64_t n_units = (n / UNIT_ROWS) * (k / 64);
    const unsigned grid = unsigned(std::min<int64_t>((n_units * 32 + 255) / 256, 65535 * 8));
    if (absmax_fp32)
        nf4_pack_native_kernel<float, TC><<<grid, 256, 0, (cudaStream_t)stream>>>(
            (const uint8_t*)packed, absmax, (uint8_t*)out, n_units, int(k / 64), int(n));
    else
        nf4_pack_native_kernel<__half, TC><<<grid, 256, 0, (cudaStream_t)stream>>>(
            (const uint8_t*)packed, absmax, (uint8_t*)out, n_units, int(k / 64), int(n));
    return check_launch(TC ? "nova_nf4_pack_tc" : "nova_nf4_pack_native");
}

extern "C" int nova_nf4_pack_native(const void* packed, const void* absmax, int absmax_fp32, void* out, int64_t n,
                                    int64_t k, void* stream) {
    return pack_units<false>(packed, absmax, absmax_fp32, out, n, k, stream);
}

extern "C" int nova_nf4_pack_tc(const void* packed, const void* absmax, int absmax_fp32, void* out, int64_t n,
                                int64_t k, void* stream) {
    return pack_units<true>(packed, absmax, absmax_fp32, out, n, k, stream);
}

template <typename Kern>
static int prepare_smem(Kern kern, int64_t smem, int64_t (&set_to_per_device)[kMaxDevices]) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(NOVA_ERR_CUDA, "no usable current device (%d)", dev);
    int64_t* set_to = &set_to_per_device[dev];   // the attribute is per device
    if (smem <= *set_to) return NOVA_OK;
    int optin = 0;
    cudaFuncAttributes fa;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "querying shared-memory limits failed");
    }
    if (smem + int64_t(fa.sharedSizeBytes) > optin)
        return fail(NOVA_ERR_UNSUPPORTED, "M*K needs %lld B of shared memory, the device allows %d",
                    (long long)(smem + fa.sharedSizeBytes), optin);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "cudaFuncSetAttribute(dynamic smem %lld) failed", (long long)smem);
    }
    *set_to = smem;
    return NOVA_OK;
}

template <typename Kern>
static int resident_ctas(Kern kern, int threads, int64_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, size_t(smem)) != cudaSuccess || n < 1) {
        cudaGetLastError();
        return 1;
    }
    return n;
}

extern "C" int nova_nf4_gemv(const nova_nf4_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    const int64_t m = a->m, n = a->n, k = a->k;
    const bool native = a->layout == 1;
    if (a->layout != 0 && a->layout != 1) return fail(NOVA_ERR_INVALID, "layout must be 0 or 1");
    if (m < 1 || m > MAX_M) return fail(NOVA_ERR_UNSUPPORTED, "M must be in [1, %d], got %lld", MAX_M, (long long)m);
    if (n <= 0 || n % (native ? UNIT_ROWS : 16))
        return fail(NOVA_ERR_INVALID, "N must be a positive multiple of %d, got %lld", native ? UNIT_ROWS : 16,
                    (long long)n);
    if (k <= 0 || k % 64) return fail(NOVA_ERR_INVALID, "K must be a positive multiple of 64, got %lld", (long long)k);
    if (n > (1 << 30) || k > (1 << 20)) return fail(NOVA_ERR_INVALID, "N/K too large");
    const int64_t smem = int64_t(LUT_BYTES) + m * k * 2;   // LUT + staged x
    if (!a->x || !a->packed || (!native && !a->absmax) || !a->lut || !a->out || !a->workspace)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    const int epi = int(a->epilogue);
    if (epi < EPI_PLAIN || epi > EPI_SLOTS) return fail(NOVA_ERR_INVALID, "bad epilogue %d", epi);
    if ((epi == EPI_F32 || epi == EPI_SLOTS) && (reinterpret_cast<uintptr_t>(a->out) % 16))
        return fail(NOVA_ERR_ALIGN, "the fp32 and slot epilogues need a 16-byte aligned out");
    if (epi == EPI_SLOTS &&
        (!native || ((n / UNIT_ROWS) * (k / 64) / sm_count() + (k / 64) - 1) / (k / 64) + 1 > SLOTS_PER_CTA))
        return fail(NOVA_ERR_UNSUPPORTED, "the slot epilogue needs the native layout and at most %d row groups per "
                                          "SM's share of the k-blocks", SLOTS_PER_CTA);
    if (a->add_slots) {   // deferred reduction of a SLOTS launch with N = this K, K = add_k
        const int64_t akb = a->add_k / 64, units = (k / UNIT_ROWS) * akb, G = sm_count();
        if (m != 1 || !native || !a->norm_weight || k / 8 > NAT_THREADS || k % UNIT_ROWS || a->add_k <= 0 ||
            a->add_k % 64 || (units / G + akb - 1) / akb + 1 > SLOTS_PER_CTA || (akb - 1) * G / units + 2 > 4 ||
            (units + akb) * G >= (1ll << 31))
            return fail(NOVA_ERR_UNSUPPORTED, "add_slots needs M = 1, the native layout, a norm prologue, K <= %d "
                                              "and a SLOTS producer with at most 4 CTAs per row group",
                        8 * NAT_THREADS);
        if (reinterpret_cast<uintptr_t>(a->add_slots) % 16 || (a->resid_out && reinterpret_cast<uintptr_t>(a->resid_out) % 16))
            return fail(NOVA_ERR_ALIGN, "add_slots and resid_out must be 16-byte aligned");
        if (a->resid_out == a->x) return fail(NOVA_ERR_INVALID, "resid_out must not alias x");
    }
    const int64_t G_sm = sm_count();
    if (a->edge_out) {   // SiLU·mul leaving the row groups split between CTAs as fp32 sums
        const int64_t kb = k / 64, units = (n / UNIT_ROWS) * kb, per = (units + G_sm - 1) / G_sm;
        if (epi != EPI_SILU_MUL || !native || m != 1 || units < int64_t(NAT_MIN_UNITS) * NAT_WARPS * G_sm ||
            units / G_sm < 2 * kb || (per + kb - 1) / kb + 1 > NAT_WARPS ||
            (units + 1) * NAT_WARPS * G_sm >= (1ll << 31))
            return fail(NOVA_ERR_UNSUPPORTED, "edge_out needs SILU_MUL, the native layout, M = 1, at least %d units "
                                              "per SM and 2 to %d row groups per SM",
                        NAT_MIN_UNITS * NAT_WARPS, NAT_WARPS - 1);
        if (reinterpret_cast<uintptr_t>(a->edge_out) % 16) return fail(NOVA_ERR_ALIGN, "edge_out must be 16-byte aligned");
    }
    if (a->edge_in) {   // x completed from a SiLU·mul launch's edges (its N = 2 * this K, its K = edge_k)
        const int64_t kb = a->edge_k / 64, units = (2 * k / UNIT_ROWS) * kb;
        if (!native || m != 1 || a->norm_weight || a->add_slots || a->edge_k <= 0 || a->edge_k % 64 ||
            units < int64_t(NAT_MIN_UNITS) * NAT_WARPS * G_sm || units / G_sm < 2 * kb ||
            2 * (G_sm - 1) > NAT_THREADS || units * G_sm >= (1ll << 31))
            return fail(NOVA_ERR_UNSUPPORTED, "edge_in needs the native layout, M = 1, no norm prologue or add_slots, "
                                              "and an edge_out producer of N = 2K, K = edge_k");
        if (reinterpret_cast<uintptr_t>(a->edge_in) % 16) return fail(NOVA_ERR_ALIGN, "edge_in must be 16-byte aligned");
    }
    if (a->attn_part) {   // o_proj over the attention's split partials, head-aligned CTAs
        const int64_t nh = a->attn_heads, kb = k / 64;
        const int64_t R = nh > 0 ? n / UNIT_ROWS / nh : 0, nmax = nh > 0 ? (G_sm + nh - 1) / nh : 0;
        if (epi != EPI_F32 || !native || m != 1 || a->norm_weight || a->add_slots || a->add_heads || a->edge_out ||
            a->edge_in || k % 128 || k / 128 > 4 || a->attn_splits < 1 || a->attn_splits > MRG_MAX_SPLITS ||
            nh < 1 || nh > G_sm || n % (UNIT_ROWS * nh) || R < nmax || (R / (G_sm / nh)) + 1 > NAT_WARPS ||
            (R / nmax) * kb < NAT_WARPS)
            return fail(NOVA_ERR_UNSUPPORTED, "attn_part needs F32, the native layout, M = 1, no other prologue, "
                                              "K = 128 x (1..4) q heads, 1..%d splits, and N / attn_heads row groups "
                                              "per head for 1..15 row groups per SM", MRG_MAX_SPLITS);
        if (reinterpret_cast<uintptr_t>(a->attn_part) % 16) return fail(NOVA_ERR_ALIGN, "attn_part must be 16-byte aligned");
    }
    if (a->add_heads) {   // x += the per-head sums of an attn_part launch (its N / attn_heads = this K)
        if (m != 1 || !native || !a->norm_weight || a->add_slots || k / 8 > NAT_THREADS || a->add_nheads < 1 ||
            a->add_nheads > 8)
            return fail(NOVA_ERR_UNSUPPORTED, "add_heads needs M = 1, the native layout, a norm prologue, K <= %d, "
                                              "no add_slots and 1..8 heads", 8 * NAT_THREADS);
        if (reinterpret_cast<uintptr_t>(a->add_heads) % 16 || (a->resid_out && reinterpret_cast<uintptr_t>(a->resid_out) % 16))
            return fail(NOVA_ERR_ALIGN, "add_heads and resid_out must be 16-byte aligned");
        if (a->resid_out == a->x) return fail(NOVA_ERR_INVALID, "resid_out must not alias x");
    }
    if (epi == EPI_RESIDUAL && !a->residual) return fail(NOVA_ERR_INVALID, "residual epilogue needs residual");
    if (epi == EPI_ARGMAX && !a->argmax) return fail(NOVA_ERR_INVALID, "argmax epilogue needs argmax");
    if (epi != EPI_PLAIN && a->bias) return fail(NOVA_ERR_UNSUPPORTED, "bias only with the plain epilogue");
    if (a->token_out && epi != EPI_ARGMAX) return fail(NOVA_ERR_INVALID, "token_out needs the argmax epilogue");
    if (a->embed && (!a->token_out || !a->embed_out || a->embed_dim <= 0 || a->embed_dim % 8))
        return fail(NOVA_ERR_INVALID, "embedding gather needs token_out, embed_out and embed_dim % 8 == 0");
    auto mis = [](const void* ptr, int al) { return ptr && (reinterpret_cast<uintptr_t>(ptr) % al); };
    if (mis(a->x, 16) || (a->x_stride % 8) || mis(a->norm_weight, 16) || mis(a->packed, native ? 16 : 8) ||
        mis(a->absmax, 4) || mis(a->workspace, 256) || mis(a->argmax, 8) || mis(a->embed, 16) ||
        mis(a->embed_out, 16) || (a->embed_out_stride % 8))
        return fail(NOVA_ERR_ALIGN, "x/norm_weight/embed must be 16-byte aligned (row strides multiples of 8), "
                                    "packed 8 (native 16), workspace 256");
    int64_t need = 0;
    nova_nf4_workspace_bytes(n, &need);
    if (a->workspace_bytes < need)
        return fail(NOVA_ERR_INVALID, "workspace too small: %lld < %lld", (long long)a->workspace_bytes, (long long)need);

    Params p;
    p.x = (const __half*)a->x;
    p.x_stride = a->x_stride;
    p.norm_w = (const __half*)a->norm_weight;
    p.eps = float(a->eps);
    p.packed = (const uint8_t*)a->packed;
    p.absmax = a->absmax;
    p.lut = (const uint32_t*)a->lut;
    p.bias = (const __half*)a->bias;
    p.residual = (const __half*)a->residual;
    p.res_stride = a->res_stride;
    p.out = (__half*)a->out;
    p.out_stride = a->out_stride;
    p.argmax = (unsigned long long*)a->argmax;
    p.token_out = a->token_out;
    p.pos = a->pos;
    p.embed = (const __half*)a->embed;
    p.embed_out = (__half*)a->embed_out;
    p.embed_out_stride = a->embed_out_stride;
    p.embed_dim = int(a->embed_dim);
    p.M = int(m);
    p.N = int(n);
    p.K = int(k);
    p.KB = int(k / 64);
    p.n_tiles = int(n / 16);
    uint8_t* ws = (uint8_t*)a->workspace;
    p.partial = (float4*)ws;
    // [partial slots | finalize counter, error word (fixed offsets: every shape that shares the
    //  workspace finds them at the same place) | per-row-tile counters]
    p.done = (unsigned*)(ws + partial_bytes());
    p.counters = (unsigned*)(ws + partial_bytes() + 256);
    if (a->add_slots) {
        p.add_slots = (const float*)a->add_slots;
        p.add_KB = int(a->add_k / 64);
        p.add_units = int64_t(k / UNIT_ROWS) * p.add_KB;
        p.add_G = sm_count();
        p.resid_out = (__half*)a->resid_out;
    }
    p.edge_out = (float*)a->edge_out;
    if (a->attn_part) {
        p.mrg_part = (const float*)a->attn_part;
        p.mrg_splits = int(a->attn_splits);
        p.mrg_heads = int(a->attn_heads);
    }
    if (a->add_heads) {
        p.add_heads = (const float*)a->add_heads;
        p.add_nheads = int(a->add_nheads);
        p.resid_out = (__half*)a->resid_out;
    }
    if (a->edge_in) {
        p.edge_in = (const float*)a->edge_in;
        p.edge_KB = int(a->edge_k / 64);
        p.edge_units = int64_t(2 * k / UNIT_ROWS) * p.edge_KB;
        p.edge_G = int(G_sm);
    }

    using Kern = void (*)(Params);
    cudaError_t err;
    if (native) {
        using NKern = void (*)(Params, int, int*);
        static const NKern kernels[2][5] = {
            {nf4_gemv_native_kernel<0, false>, nf4_gemv_native_kernel<1, false>, nf4_gemv_native_kernel<2, false>,
             nf4_gemv_native_kernel<3, false>, nf4_gemv_native_kernel<4, false>},
            {nf4_gemv_native_kernel<0, true>, nf4_gemv_native_kernel<1, true>, nf4_gemv_native_kernel<2, true>,
             nf4_gemv_native_kernel<3, true>, nf4_gemv_native_kernel<4, true>}};
        static int64_t smem_set[2][5][kMaxDevices] = {};
        static int optin = 0;
        if (!optin) {
            int dev = 0;
            if (cudaGetDevice(&dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
                cudaGetLastError();
                optin = 0;
                return fail(NOVA_ERR_CUDA, "querying the shared-memory limit failed");
            }
        }
        // LUT + staged x, then the per-warp rings with as many units per stage
        // as fit (at most 4); x stays in global memory when staging it would
        // leave less than 2 units per stage and there is no norm prologue.
        const int64_t ring_unit = int64_t(NAT_WARPS) * NAT_STAGES * UNIT_BYTES;
        const int64_t slack = 1024;   // static shared memory
        const int64_t edge_bytes = (a->edge_out || a->attn_part) ? EDGE_RED_BYTES : 0;   // after the rings
        auto units_for = [&](int64_t xs_bytes) {
            return std::min<int64_t>(4, (optin - int64_t(LUT_BYTES) - xs_bytes - edge_bytes - slack) / ring_unit);
        };
        int64_t xs_bytes = (m * k * 2 + 127) / 128 * 128;
        int64_t stage_units = units_for(xs_bytes);
        int xg = 0;
        if (stage_units < 2 && !a->norm_weight) {
            xg = 1;
            xs_bytes = 0;
            stage_units = units_for(0);
        }
        if (stage_units < 1)
            return fail(NOVA_ERR_UNSUPPORTED, "M*K = %lld with the norm prologue leaves no shared memory for the "
                                              "weight ring", (long long)(m * k));
        p.units = int64_t(n / UNIT_ROWS) * p.KB;
        int* errp = gemv_error_word(ws);
        // Warp-level stream-K from two row groups per SM up (gate/up, the
        // lm_head: with several row groups per CTA the CTA-level schedule
        // would synchronise its 16 warps once per row group); CTA-level
        // split-K on whole row groups below that (no cross-CTA reduction).
        const bool warp_level = a->edge_out || a->attn_part || (epi != EPI_SLOTS && ((launch_flags() & 2) ||
                                                                      n / UNIT_ROWS >= 2 * int64_t(sm_count())));
        if (a->attn_part && xg) return fail(NOVA_ERR_UNSUPPORTED, "attn_part needs x staged in shared memory");
        if (a->edge_in && (warp_level || xg))
            return fail(NOVA_ERR_UNSUPPORTED, "edge_in needs the CTA-level schedule with x staged (SLOTS or fewer "
                                              "than two row groups per SM)");
        if (warp_level) {
            NKern kern = kernels[xg][epi];
            const int64_t nsmem = int64_t(LUT_BYTES) + xs_bytes + stage_units * ring_unit + edge_bytes;
            if (int rc = prepare_smem(kern, nsmem, smem_set[xg][epi])) return rc;
            const int64_t want = (p.units + NAT_MIN_UNITS - 1) / NAT_MIN_UNITS;
            // edge_out: every warp of every CTA active (checked above: want >= SMs x 16)
            p.total_warps = int(std::max<int64_t>(1, std::min<int64_t>(int64_t(sm_count()) * NAT_WARPS, want)));
            if (a->attn_part) p.total_warps = int(sm_count()) * NAT_WARPS;   // head-aligned CTAs, every warp busy
            const unsigned grid = unsigned(std::min<int64_t>(sm_count(), p.total_warps));
            err = launch(kern, dim3(grid), dim3(NAT_THREADS), size_t(nsmem), (cudaStream_t)stream, p, int(stage_units),
                         errp);
        } else {   // CTA-level split-K
            static const NKern cta_kernels[2][6] = {
                {nf4_gemv_cta_kernel<0, false>, nf4_gemv_cta_kernel<1, false>, nf4_gemv_cta_kernel<2, false>,
                 nf4_gemv_cta_kernel<3, false>, nf4_gemv_cta_kernel<4, false>, nf4_gemv_cta_kernel<5, false>},
                {nf4_gemv_cta_kernel<0, true>, nf4_gemv_cta_kernel<1, true>, nf4_gemv_cta_kernel<2, true>,
                 nf4_gemv_cta_kernel<3, true>, nf4_gemv_cta_kernel<4, true>, nf4_gemv_cta_kernel<5, true>}};
            static int64_t cta_smem_set[2][6][kMaxDevices] = {};
            const int64_t red_bytes = int64_t(NAT_WARPS) * 32 * 32;
            // SLOTS: one CTA per SM over an equal share of all units; otherwise whole row groups
            const int64_t grid = epi == EPI_SLOTS ? int64_t(sm_count()) : std::min<int64_t>(sm_count(), n / UNIT_ROWS);
            const int64_t rg_max = (n / UNIT_ROWS + grid - 1) / grid;   // row groups of the largest CTA share
            // residual rows staged per CTA when they fit in 4 values per thread
            p.res_rows = (epi == EPI_RESIDUAL && rg_max * UNIT_ROWS * m <= 4 * NAT_THREADS) ? int(rg_max * UNIT_ROWS) : 0;
            const int64_t res_bytes = (int64_t(p.res_rows) * m * 2 + 127) / 128 * 128;
            const int64_t cu = std::min<int64_t>(
                4, (optin - int64_t(LUT_BYTES) - xs_bytes - red_bytes - res_bytes - slack) / ring_unit);
            if (cu < 1)
                return fail(NOVA_ERR_UNSUPPORTED, "M*K = %lld leaves no shared memory for the weight ring",
                            (long long)(m * k));
            NKern kern = cta_kernels[xg][epi];
            const int64_t nsmem = int64_t(LUT_BYTES) + xs_bytes + red_bytes + res_bytes + cu * ring_unit;
            if (int rc = prepare_smem(kern, nsmem, cta_smem_set[xg][epi])) return rc;
            p.total_warps = int(grid);   // contributors and finalize arrivals are counted per CTA
            err = launch(kern, dim3(unsigned(grid)), dim3(NAT_THREADS), size_t(nsmem), (cudaStream_t)stream, p,
                         int(cu), errp);
        }
    } else {
        static const Kern kernels[2][5] = {
            {nf4_gemv_ref_kernel<__half, 0>, nf4_gemv_ref_kernel<__half, 1>, nf4_gemv_ref_kernel<__half, 2>,
             nf4_gemv_ref_kernel<__half, 3>, nf4_gemv_ref_kernel<__half, 4>},
            {nf4_gemv_ref_kernel<float, 0>, nf4_gemv_ref_kernel<float, 1>, nf4_gemv_ref_kernel<float, 2>,
             nf4_gemv_ref_kernel<float, 3>, nf4_gemv_ref_kernel<float, 4>}};
        static int64_t smem_set[2][5][kMaxDevices] = {};
        const int ai = a->absmax_fp32 ? 1 : 0;
        Kern kern = kernels[ai][epi];
        if (int rc = prepare_smem(kern, smem, smem_set[ai][epi])) return rc;
        p.units = int64_t(p.n_tiles) * p.KB;
        p.total_warps = int(std::min<int64_t>(int64_t(sm_count()) * REF_WARPS, p.units));
        const unsigned grid = unsigned((p.total_warps + REF_WARPS - 1) / REF_WARPS);
        err = launch(kern, dim3(grid), dim3(REF_THREADS), size_t(smem), (cudaStream_t)stream, p);
    }
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_nf4_gemv: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_nf4_quantize(const void* w, int64_t n, int64_t k, const void* midpoints, void* packed,
                                 void* absmax, int absmax_fp32, void* stream) {
    if (n <= 0 || k <= 0 || k % 64) return fail(NOVA_ERR_INVALID, "need N > 0 and K a positive multiple of 64");
    if (!w || !midpoints || !packed || !absmax) return fail(NOVA_ERR_INVALID, "NULL pointer");
    const int64_t n_blocks = n * (k / 64);
    const unsigned grid = unsigned(std::min<int64_t>((n_blocks + 255) / 256, 65535 * 4));
    nf4_quantize_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const __half*)w, n_blocks, int(k / 64), int(n),
                                                               (const float*)midpoints, (uint8_t*)packed, absmax,
                                                               absmax_fp32);
    return check_launch("nova_nf4_quantize");
}

extern "C" int nova_nf4_dequant(const void* packed, const void* absmax, int absmax_fp32, const void* lut, void* out,
                                int64_t n, int64_t k, void* stream) {
    if (n <= 0 || k <= 0 || k % 64) return fail(NOVA_ERR_INVALID, "need N > 0 and K a positive multiple of 64");
    if (!packed || !absmax || !lut || !out) return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (reinterpret_cast<uintptr_t>(out) % 4) return fail(NOVA_ERR_ALIGN, "out must be 4-byte aligned");
    const int64_t total = n * (k / 2);
    const unsigned grid = unsigned(std::min<int64_t>((total + 255) / 256, 65535 * 8));
    if (absmax_fp32)
        nf4_dequant_kernel<float><<<grid, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)packed, absmax,
                                                                          (const uint32_t*)lut, (__half*)out, n, int(k));
    else
        nf4_dequant_kernel<__half><<<grid, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)packed, absmax,
                                                                           (const uint32_t*)lut, (__half*)out, n, int(k));
    return check_launch("nova_nf4_dequant");
}

// ---------------------------------------------------------------- batched GEMM (host)

// Split count: no more CTAs than SMs (one wave), and about sqrt(3 * k-blocks): each split adds
// ~KB/S k-block steps of work per CTA but one more 128 KB partial for the last CTA to add.
static int64_t tc_grid(int64_t items) {
    return std::max<int64_t>(1, std::min<int64_t>(sm_count(), (items + TC_MIN_ITEMS - 1) / TC_MIN_ITEMS));
}

// tcgen05 GEMM workspace: [0] finalize arrivals, [4] error word, [256, 256 +
// 32 * TC_MAX_TILES) split arrivals per tile, lane quarter and column half,
// then 2 partial slots per CTA.  The offsets are the same for every shape, so launches of
// different shapes can share one workspace: each leaves its counters at zero,
// and no shape's partials reach another's counters.
static int64_t tc_workspace_layout(int64_t n, int64_t k, int64_t* part_off) {
    const int64_t tiles = (n + TC_ROWS - 1) / TC_ROWS;
    const int64_t w = tiles * ((k / 64 + TC_KG - 1) / TC_KG);
    const int64_t g = tc_grid(w);
    const int64_t off = (256 + int64_t(TC_MAX_TILES) * TC_CNT_PER_TILE * 4 + 1023) / 1024 * 1024;
    if (part_off) *part_off = off;
    return off + g * 2 * int64_t(TC_SLOT_FLOATS) * 4;
}

extern "C" int nova_nf4_gemm_workspace_bytes(int64_t n, int64_t k, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (n <= 0 || n % UNIT_ROWS || k <= 0 || k % 64) return fail(NOVA_ERR_INVALID, "N multiple of 32, K of 64");
    *bytes = tc_workspace_layout(n, k, nullptr);
    return NOVA_OK;
}

extern "C" int nova_nf4_gemm_read_error(void* workspace, int* host_value) {
    if (!workspace) return fail(NOVA_ERR_INVALID, "NULL workspace");
    return read_error_word(reinterpret_cast<int*>((uint8_t*)workspace + 4), host_value, "GEMM");
}

// tcgen05 path of nova_nf4_gemm (arguments already validated).
static int nf4_gemm_tc(const nova_nf4_args* a, int epi, cudaStream_t stream) {
    const int64_t m = a->m, n = a->n, k = a->k;
    Params p{};
    p.x = (const __half*)a->x;
    p.x_stride = a->x_stride;
    p.packed = (const uint8_t*)a->packed;
    p.lut = (const uint32_t*)a->lut;
    p.residual = (const __half*)a->residual;
    p.res_stride = a->res_stride;
    p.out = (__half*)a->out;
    p.out_stride = a->out_stride;
    p.argmax = (unsigned long long*)a->argmax;
    p.token_out = a->token_out;
    p.pos = a->pos;
    p.embed = (const __half*)a->embed;
    p.embed_out = (__half*)a->embed_out;
    p.embed_out_stride = a->embed_out_stride;
    p.embed_dim = int(a->embed_dim);
    p.M = int(m);
    p.N = int(n);
    p.K = int(k);
    p.KB = int(k / 64);
    const int64_t tiles = (n + TC_ROWS - 1) / TC_ROWS;
    int64_t part_off = 0;
    tc_workspace_layout(n, k, &part_off);
    uint8_t* ws = (uint8_t*)a->workspace;
    TcArgs ta;
    ta.n_mma = int((m + 15) / 16 * 16);
    ta.W = tiles * ((p.KB + TC_KG - 1) / TC_KG);
    ta.G = int(tc_grid(ta.W));
    ta.part = (float*)(ws + part_off);
    ta.tile_cnt = (unsigned*)(ws + 256);
    ta.err = (int*)(ws + 4);
    p.done = (unsigned*)ws;
    CUtensorMap xmap;
    if (int rc = make_tmap_f16_rows64(&xmap, a->x, uint64_t(m), uint64_t(k), uint64_t(a->x_stride), uint32_t(ta.n_mma)))
        return rc;
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "device queries failed");
    }
    const int64_t fixed = 1024 + int64_t(TC_XS) * TC_KG * ta.n_mma * 128 + TC_LUT_BYTES;
    ta.ws = int(std::min<int64_t>(TC_WS_MAX, (optin - 1024 - fixed) / TC_W_BYTES));   // 1 KB for static smem
    if (ta.ws < 2) return fail(NOVA_ERR_UNSUPPORTED, "shared memory");
    const int64_t nsmem = fixed + int64_t(ta.ws) * TC_W_BYTES;
    using TKern = void (*)(Params, CUtensorMap, TcArgs);
    static const TKern kernels[5] = {nf4_gemm_tc_kernel<0>, nf4_gemm_tc_kernel<1>, nf4_gemm_tc_kernel<2>,
                                     nf4_gemm_tc_kernel<3>, nf4_gemm_tc_kernel<4>};
    static int64_t smem_set[5][kMaxDevices] = {};
    if (int rc = prepare_smem(kernels[epi], nsmem, smem_set[epi])) return rc;
    const cudaError_t err = launch(kernels[epi], dim3(unsigned(ta.G)), dim3(TC_THREADS), size_t(nsmem), stream, p,
                                   xmap, ta);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_nf4_gemm: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

// Wide path of nova_nf4_gemm (M > 64; arguments already validated).
static int nf4_gemm_wide(const nova_nf4_args* a, int epi, cudaStream_t stream) {
    const int64_t m = a->m, n = a->n, k = a->k;
    Params p{};
    p.x = (const __half*)a->x;
    p.x_stride = a->x_stride;
    p.packed = (const uint8_t*)a->packed;
    p.lut = (const uint32_t*)a->lut;
    p.residual = (const __half*)a->residual;
    p.res_stride = a->res_stride;
    p.out = (__half*)a->out;
    p.out_stride = a->out_stride;
    p.M = int(m);
    p.N = int(n);
    p.K = int(k);
    p.KB = int(k / 64);
    TwArgs ta;
    ta.m_tiles = int((m + TW_MT - 1) / TW_MT);
    ta.items = ((n + TC_ROWS - 1) / TC_ROWS) * ta.m_tiles;
    ta.err = (int*)((uint8_t*)a->workspace + 4);
    CUtensorMap xmap;
    if (int rc = make_tmap_f16_rows64(&xmap, a->x, uint64_t(m), uint64_t(k), uint64_t(a->x_stride), uint32_t(TW_MT)))
        return rc;
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "device queries failed");
    }
    const int64_t fixed = 1024 + int64_t(TW_XS) * TW_X_BYTES + TC_LUT_BYTES;
    ta.ws = int(std::min<int64_t>(TW_WS_MAX, (optin - 1024 - fixed) / TW_W_BYTES));   // 1 KB for static smem
    if (ta.ws < 2) return fail(NOVA_ERR_UNSUPPORTED, "shared memory");
    const int64_t nsmem = fixed + int64_t(ta.ws) * TW_W_BYTES;
    using TKern = void (*)(Params, CUtensorMap, TwArgs);
    static const TKern kernels[5] = {nf4_gemm_wide_kernel<0>, nf4_gemm_wide_kernel<1>, nf4_gemm_wide_kernel<2>,
                                     nullptr, nf4_gemm_wide_kernel<4>};
    static int64_t smem_set[5][kMaxDevices] = {};
    if (!kernels[epi]) return fail(NOVA_ERR_UNSUPPORTED, "the argmax epilogue needs M <= 64");
    if (int rc = prepare_smem(kernels[epi], nsmem, smem_set[epi])) return rc;
    const unsigned grid = unsigned(std::min<int64_t>(sm_count(), ta.items));
    const cudaError_t err = launch(kernels[epi], dim3(grid), dim3(TW_THREADS), size_t(nsmem), stream, p, xmap, ta);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_nf4_gemm: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_nf4_gemm(const nova_nf4_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    const int64_t m = a->m, n = a->n, k = a->k;
    if (a->layout != 2) return fail(NOVA_ERR_UNSUPPORTED, "tcgen05 unit layout (2, nova_nf4_pack_tc) only");
    if (m < 1 || m > (1 << 20)) return fail(NOVA_ERR_UNSUPPORTED, "M must be in [1, 2^20], got %lld", (long long)m);
    if (n <= 0 || n % UNIT_ROWS || n > (1 << 30) || k <= 0 || k % 64 || k > (1 << 20))
        return fail(NOVA_ERR_INVALID, "N multiple of 32, K multiple of 64");
    if (a->norm_weight) return fail(NOVA_ERR_UNSUPPORTED, "no norm prologue in the batched GEMM (normalize x first)");
    if (a->bias) return fail(NOVA_ERR_UNSUPPORTED, "no bias in the batched GEMM");
    const int epi = int(a->epilogue);
    if (epi < EPI_PLAIN || epi > EPI_F32) return fail(NOVA_ERR_INVALID, "bad epilogue %d", epi);
    if (!a->x || !a->packed || !a->lut || !a->out || !a->workspace) return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (epi == EPI_RESIDUAL && !a->residual) return fail(NOVA_ERR_INVALID, "residual epilogue needs residual");
    if (epi == EPI_ARGMAX && !a->argmax) return fail(NOVA_ERR_INVALID, "argmax epilogue needs argmax");
    if (a->embed && (!a->token_out || !a->embed_out || a->embed_dim <= 0 || a->embed_dim % 8))
        return fail(NOVA_ERR_INVALID, "embedding gather needs token_out, embed_out and embed_dim % 8 == 0");
    auto mis = [](const void* ptr, int al) { return ptr && (reinterpret_cast<uintptr_t>(ptr) % al); };
    if (mis(a->x, 16) || (a->x_stride % 8) || mis(a->packed, 16) || mis(a->workspace, 256) || mis(a->argmax, 8) ||
        mis(a->embed, 16) || mis(a->embed_out, 16) || (a->embed_out_stride % 8) || (epi == EPI_F32 && mis(a->out, 4)))
        return fail(NOVA_ERR_ALIGN, "x / packed 16-byte aligned (x_stride % 8), workspace 256");
    int64_t need = 0;
    nova_nf4_gemm_workspace_bytes(n, k, &need);
    if (a->workspace_bytes < need) return fail(NOVA_ERR_INVALID, "workspace too small: %lld < %lld",
                                               (long long)a->workspace_bytes, (long long)need);
    if ((n + TC_ROWS - 1) / TC_ROWS > TC_MAX_TILES)
        return fail(NOVA_ERR_UNSUPPORTED, "N above %d rows", TC_MAX_TILES * TC_ROWS);
    if (m > TC_MAX_M) {
        if (epi == EPI_ARGMAX || a->token_out || a->embed)
            return fail(NOVA_ERR_UNSUPPORTED, "the argmax epilogue and the step finalize need M <= 64");
        return nf4_gemm_wide(a, epi, (cudaStream_t)stream);
    }
    return nf4_gemm_tc(a, epi, (cudaStream_t)stream);
}
