// NF4 weight GEMV / skinny GEMM (M <= 8) for sm_100a, plus the NF4 quantizer
// and dequantizer.
//
// Weight format (reference src/nova/quant.py:39-69): packed uint8 [N, K/2],
// K-contiguous, byte j of a row = element 2j in the high nibble, 2j+1 in the
// low nibble; absmax [K/64, N] (fp32 in the reference, fp16 in the native
// format); 16-entry NF4 codebook given as the reference's 256-entry fp16x2
// LUT (src/nova/kernels.py:170-182: low half = code[b>>4], high = code[b&15]).
//
// y[m, n] = sum_blocks absmax[blk, n] * sum_{k in blk} x[m, k] * code16[idx(n, k)]
//
// Work split ("stream-K"): the (16-row tile, 64-k block) units of the whole
// matrix are dealt out in equal contiguous ranges to every warp of a
// persistent grid (one 16-warp CTA per SM), so all SMs stream the same number
// of weight bytes whatever N and K are.  A warp that covers a whole row tile
// finishes it; partial tiles leave their MMA accumulator fragment in a
// workspace slot and the last of the tile's warps to arrive (arrival counter)
// adds the slots in warp order -- deterministic -- and runs the epilogue.
//
// Per unit and lane: two 8-byte streaming loads of packed weights; each byte
// becomes one f16x2 A-fragment register via one byte-permute (forms the LUT
// address from the byte and the lane id) and one bank-conflict-free
// shared-memory load (the LUT is replicated once per lane).  The products
// code16 * x16 are exact in fp32 and accumulated in fp32 by mma.sync
// m16n8k16 (x in the B operand, columns = the M <= 8 rows); each 64-element
// block gets a fresh accumulator that is scaled by its absmax, as in the
// reference kernel (src/nova/kernels.py:213-232).
#include "common.cuh"

namespace nova {
namespace nf4 {

constexpr int WARPS = 16;
constexpr int THREADS = WARPS * 32;
constexpr int LUT_WORDS = 256 * 64;      // entry v at word v*64 + lane (256-byte rows)
constexpr int SMEM_BYTES = LUT_WORDS * 4;
constexpr int BATCH = 8;                 // units whose loads are issued together
constexpr int MAX_M = 8;

enum Epi { EPI_PLAIN = 0, EPI_RESIDUAL = 1, EPI_SILU_MUL = 2, EPI_ARGMAX = 3 };

struct Params {
    const __half* x;          // fp16 [M, K] (the residual when norm_w != nullptr)
    int64_t x_stride;
    const __half* norm_w;     // fp16 [K] RMSNorm weight or nullptr
    float eps;
    const uint8_t* packed;
    const void* absmax;
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
    float4* partial;          // [total_warps][2][32] float4
    unsigned* counters;       // [n_tiles]
    unsigned* done;           // finalize arrival counter
    int M, N, K, KB, n_tiles, total_warps;
    int64_t units;
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

template <int EPI>
__device__ __forceinline__ void epilogue(const Params& p, int tile, const float (&c)[4], int g, int t) {
    if (EPI == EPI_SILU_MUL) {
        // tile rows 0..7 are gate rows 8*tile+g, rows 8..15 the matching up rows
        const int n = tile * 8 + g;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int m = 2 * t + e;
            if (m >= p.M) continue;
            const float gate = __half2float(__float2half_rn(c[e]));
            const float up = __half2float(__float2half_rn(c[2 + e]));
            const float s = __half2float(__float2half_rn(__fdiv_rn(gate, 1.0f + expf(-gate))));
            p.out[m * p.out_stride + n] = __float2half_rn(s * up);
        }
        return;
    }
    unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
        const int n = tile * 16 + g + 8 * hrow;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int m = 2 * t + e;
            if (m >= p.M) continue;
            float v = c[2 * hrow + e];
            __half h;
            if (EPI == EPI_RESIDUAL) {
                h = __float2half_rn(__half2float(p.residual[m * p.res_stride + n]) +
                                    __half2float(__float2half_rn(v)));
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
            const int m = 2 * t + e;
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

template <typename AbsT, int EPI>
__global__ void __launch_bounds__(THREADS, 1) nf4_gemv_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(16) uint32_t lut_s[];
    __half* xs = reinterpret_cast<__half*>(lut_s + LUT_WORDS);   // [M][K]
    __shared__ float red[WARPS][MAX_M];
    __shared__ float rstd[MAX_M];
    for (int i = threadIdx.x; i < 256 * 32; i += THREADS) lut_s[(i >> 5) * 64 + (i & 31)] = __ldg(p.lut + (i >> 5));

    // ---- stage x (optionally RMS-normalised, HF order) in shared memory
    const int kv8 = p.K / 8;
    if (p.norm_w) {
        float ss[MAX_M];
#pragma unroll
        for (int m = 0; m < MAX_M; ++m) ss[m] = 0.f;
        for (int i = threadIdx.x; i < kv8; i += THREADS) {
#pragma unroll
            for (int m = 0; m < MAX_M; ++m) {
                if (m >= p.M) break;
                const uint4 v = *reinterpret_cast<const uint4*>(p.x + m * p.x_stride + 8 * i);
                const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = __half22float2(h[q]);
                    ss[m] += f.x * f.x + f.y * f.y;
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
            for (int w = 0; w < WARPS; ++w) v += red[w][threadIdx.x];
            rstd[threadIdx.x] = rsqrt_ieee(__fdiv_rn(v, float(p.K)) + p.eps);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < kv8; i += THREADS) {
            const uint4 wv = *reinterpret_cast<const uint4*>(p.norm_w + 8 * i);
            const __half2* wh = reinterpret_cast<const __half2*>(&wv);
            for (int m = 0; m < p.M; ++m) {
                const uint4 v = *reinterpret_cast<const uint4*>(p.x + m * p.x_stride + 8 * i);
                const __half2* h = reinterpret_cast<const __half2*>(&v);
                uint4 o;
                __half2* oh = reinterpret_cast<__half2*>(&o);
                const float r = rstd[m];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = __half22float2(h[q]);
                    const float2 wf = __half22float2(wh[q]);
                    const __half2 n16 = __floats2half2_rn(f.x * r, f.y * r);
                    const float2 nf = __half22float2(n16);
                    oh[q] = __floats2half2_rn(wf.x * nf.x, wf.y * nf.y);
                }
                *reinterpret_cast<uint4*>(xs + m * p.K + 8 * i) = o;
            }
        }
    } else {
        for (int i = threadIdx.x; i < p.M * kv8; i += THREADS) {
            const int m = i / kv8, j = i % kv8;
            *reinterpret_cast<uint4*>(xs + m * p.K + 8 * j) =
                __ldg(reinterpret_cast<const uint4*>(p.x + m * p.x_stride) + j);
        }
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int w = blockIdx.x * WARPS + warp;
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
        float acc[4] = {0.f, 0.f, 0.f, 0.f};

        for (int i = 0; i < span; i += BATCH) {
            const int nb = min(BATCH, span - i);
            uint2 wa[BATCH], wb[BATCH];
            float am0[BATCH], am1[BATCH];
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                if (j < nb) {
                    const int b = b0 + i + j;
                    wa[j] = ldg_stream64(wrow0 + 32 * b);
                    wb[j] = ldg_stream64(wrow1 + 32 * b);
                    am0[j] = absmax_at<AbsT>(p.absmax, int64_t(b) * p.N + r0 + g);
                    am1[j] = absmax_at<AbsT>(p.absmax, int64_t(b) * p.N + r0 + g + 8);
                }
            }
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                if (j < nb) {
                    const int b = b0 + i + j;
                    // B fragments: x[m = g][64b + 16t .. +15] (zero columns for g >= M)
                    uint32_t xb[8];
                    {
                        const uint4 x0 = lds128(xrow + 64 * b), x1 = lds128(xrow + 64 * b + 8);
                        const bool on = g < p.M;
                        xb[0] = on ? x0.x : 0u; xb[1] = on ? x0.y : 0u; xb[2] = on ? x0.z : 0u; xb[3] = on ? x0.w : 0u;
                        xb[4] = on ? x1.x : 0u; xb[5] = on ? x1.y : 0u; xb[6] = on ? x1.z : 0u; xb[7] = on ? x1.w : 0u;
                    }
                    const uint32_t ww[4] = {wa[j].x, wa[j].y, wb[j].x, wb[j].y};
                    float blk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        // bytes 2s, 2s+1 of this lane's 8 bytes of each row
                        const uint32_t r0w = ww[s >> 1], r1w = ww[2 + (s >> 1)];
                        const int bl = (s & 1) * 2;
                        const uint32_t a0 = lds32(lut_base + __byte_perm(r0w, laneword, 0x5504 | (bl << 4)));
                        const uint32_t a2 = lds32(lut_base + __byte_perm(r0w, laneword, 0x5504 | ((bl + 1) << 4)));
                        const uint32_t a1 = lds32(lut_base + __byte_perm(r1w, laneword, 0x5504 | (bl << 4)));
                        const uint32_t a3 = lds32(lut_base + __byte_perm(r1w, laneword, 0x5504 | ((bl + 1) << 4)));
                        mma_16816(blk, a0, a1, a2, a3, xb[2 * s], xb[2 * s + 1]);
                    }
                    acc[0] += am0[j] * blk[0];
                    acc[1] += am0[j] * blk[1];
                    acc[2] += am1[j] * blk[2];
                    acc[3] += am1[j] * blk[3];
                }
            }
        }

        if (span == p.KB) {
            epilogue<EPI>(p, tile, acc, g, t);
        } else {
            const int slot = 2 * w + (tile == first_tile ? 0 : 1);
            p.partial[int64_t(slot) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __threadfence();
            __syncwarp();
            const int64_t tu0 = int64_t(tile) * p.KB;
            const int w_first = owner_of(tu0, p.units, W);
            const int w_last = owner_of(tu0 + p.KB - 1, p.units, W);
            unsigned prev = 0;
            if (lane == 0) prev = atomicAdd(p.counters + tile, 1u);
            prev = __shfl_sync(0xffffffffu, prev, 0);
            if (prev == unsigned(w_last - w_first)) {
                __threadfence();
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                for (int ww2 = w_first; ww2 <= w_last; ++ww2) {
                    const int ft = int(unit_begin(p.units, ww2, W) / p.KB);
                    const int sl = 2 * ww2 + (tile == ft ? 0 : 1);
                    const float4 v = __ldcg(p.partial + int64_t(sl) * 32 + lane);
                    c[0] += v.x; c[1] += v.y; c[2] += v.z; c[3] += v.w;
                }
                epilogue<EPI>(p, tile, c, g, t);
                if (lane == 0) p.counters[tile] = 0u;
            }
        }
        u += span;
    }

    if (EPI == EPI_ARGMAX && p.token_out) {
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(p.done, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == unsigned(W - 1)) {
            __threadfence();
            finalize_step(p, lane);
        }
    }
}

// ---------------------------------------------------------------- quantizer

// One block of 64 weights per warp-half... kept simple: one thread per block.
__global__ void nf4_quantize_kernel(const __half* __restrict__ w, int64_t n_blocks, int kb, int N,
                                    const float* __restrict__ mid, uint8_t* __restrict__ packed, void* absmax,
                                    int absmax_fp32) {
    __shared__ float smid[15];
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

}  // namespace nf4
}  // namespace nova

using namespace nova;
using namespace nova::nf4;

static int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

// Workspace layout: [partial slots of every warp of the persistent grid |
// per-row-tile arrival counters + the finalize counter].  The partial region
// has the same size for every N, so one workspace sized for the largest N can
// be shared by all GEMVs on a stream: each launch leaves its counters at zero.
static int64_t partial_bytes() { return int64_t(sm_count()) * WARPS * 2 * 32 * 16; }

extern "C" int nova_nf4_workspace_bytes(int64_t n, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (n <= 0 || n % 16) return fail(NOVA_ERR_INVALID, "N must be a positive multiple of 16");
    *bytes = partial_bytes() + ((n / 16) * 4 + 4 + 255) / 256 * 256;
    return NOVA_OK;
}

extern "C" int nova_nf4_gemv(const nova_nf4_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    const int64_t m = a->m, n = a->n, k = a->k;
    if (m < 1 || m > MAX_M) return fail(NOVA_ERR_UNSUPPORTED, "M must be in [1, %d], got %lld", MAX_M, (long long)m);
    if (n <= 0 || n % 16) return fail(NOVA_ERR_INVALID, "N must be a positive multiple of 16, got %lld", (long long)n);
    if (k <= 0 || k % 64) return fail(NOVA_ERR_INVALID, "K must be a positive multiple of 64, got %lld", (long long)k);
    if (n > (1 << 30) || k > (1 << 20)) return fail(NOVA_ERR_INVALID, "N/K too large");
    const int64_t smem = int64_t(SMEM_BYTES) + m * k * 2;   // LUT + staged x
    if (!a->x || !a->packed || !a->absmax || !a->lut || !a->out || !a->workspace)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    const int epi = int(a->epilogue);
    if (epi < EPI_PLAIN || epi > EPI_ARGMAX) return fail(NOVA_ERR_INVALID, "bad epilogue %d", epi);
    if (epi == EPI_RESIDUAL && !a->residual) return fail(NOVA_ERR_INVALID, "residual epilogue needs residual");
    if (epi == EPI_ARGMAX && !a->argmax) return fail(NOVA_ERR_INVALID, "argmax epilogue needs argmax");
    if (epi != EPI_PLAIN && a->bias) return fail(NOVA_ERR_UNSUPPORTED, "bias only with the plain epilogue");
    if (a->token_out && epi != EPI_ARGMAX) return fail(NOVA_ERR_INVALID, "token_out needs the argmax epilogue");
    if (a->embed && (!a->token_out || !a->embed_out || a->embed_dim <= 0 || a->embed_dim % 8))
        return fail(NOVA_ERR_INVALID, "embedding gather needs token_out, embed_out and embed_dim % 8 == 0");
    auto mis = [](const void* ptr, int al) { return ptr && (reinterpret_cast<uintptr_t>(ptr) % al); };
    if (mis(a->x, 16) || (a->x_stride % 8) || mis(a->norm_weight, 16) || mis(a->packed, 8) || mis(a->absmax, 4) ||
        mis(a->workspace, 256) || mis(a->argmax, 8) || mis(a->embed, 16) || mis(a->embed_out, 16) ||
        (a->embed_out_stride % 8))
        return fail(NOVA_ERR_ALIGN, "x/norm_weight/embed must be 16-byte aligned (row strides multiples of 8), packed "
                                    "8, workspace 256");
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
    p.units = int64_t(p.n_tiles) * p.KB;
    const int64_t max_warps = int64_t(sm_count()) * WARPS;
    p.total_warps = int(std::min<int64_t>(max_warps, p.units));
    uint8_t* ws = (uint8_t*)a->workspace;
    p.partial = (float4*)ws;
    p.counters = (unsigned*)(ws + partial_bytes());
    p.done = p.counters + p.n_tiles;
    const unsigned grid = unsigned((p.total_warps + WARPS - 1) / WARPS);

    using Kern = void (*)(Params);
    static const Kern kernels[2][4] = {
        {nf4_gemv_kernel<__half, 0>, nf4_gemv_kernel<__half, 1>, nf4_gemv_kernel<__half, 2>, nf4_gemv_kernel<__half, 3>},
        {nf4_gemv_kernel<float, 0>, nf4_gemv_kernel<float, 1>, nf4_gemv_kernel<float, 2>, nf4_gemv_kernel<float, 3>}};
    static int64_t smem_set[2][4] = {};
    const int ai = a->absmax_fp32 ? 1 : 0;
    Kern kern = kernels[ai][epi];
    if (smem > smem_set[ai][epi]) {
        int dev = 0, optin = 0;
        cudaFuncAttributes fa;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
            cudaGetLastError();
            return fail(NOVA_ERR_CUDA, "querying shared-memory limits failed");
        }
        if (smem + int64_t(fa.sharedSizeBytes) > optin)
            return fail(NOVA_ERR_UNSUPPORTED, "M*K = %lld needs %lld B of shared memory, the device allows %d",
                        (long long)(m * k), (long long)(smem + fa.sharedSizeBytes), optin);
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
            cudaGetLastError();
            return fail(NOVA_ERR_CUDA, "cudaFuncSetAttribute(dynamic smem %lld) failed", (long long)smem);
        }
        smem_set[ai][epi] = smem;
    }
    kern<<<grid, THREADS, size_t(smem), (cudaStream_t)stream>>>(p);
    return check_launch("nova_nf4_gemv");
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
