// Sampling of the next token from the logits buffer, outside the decode graph
// (src/chat.py:46-75, sample_next): temperature <= 0 -> greedy argmax;
// otherwise repetition penalty on the tokens already seen, the top-k logits,
// softmax(vals / temperature), the top-p cut, and one draw from what is left.
// The draw is made by inverse CDF from a uniform number the caller supplies
// (one per row, e.g. torch.rand with the caller's generator), so a given
// uniform always picks the same token; the reference draws with
// torch.multinomial from the same probabilities.
//
// One CTA per row.  Top-k: radix selection of the k-th largest order-preserving
// key of the penalized fp32 logits (4 passes over the row, 8 bits each), ties
// at the boundary taken by lowest index; the <= k candidates are gathered in
// index order, sorted (value descending, index ascending) in shared memory and
// turned into probabilities in fp32.
#include "common.cuh"

namespace nova {
namespace sample {

constexpr int ST = 1024;       // threads per row
constexpr int MAXK = 256;      // largest top_k

struct Params {
    const __half* logits;
    int64_t lstride;
    const uint8_t* seen;       // [rows, vocab] or nullptr
    int64_t sstride;
    const float* uniform;      // [rows], in [0, 1)
    int64_t* token_out;        // [rows]
    const __half* embed;       // [vocab, embed_dim] or nullptr
    __half* embed_out;         // [rows, embed_dim]
    int64_t eostride;
    int embed_dim;
    float* probs_out;          // [rows, k] or nullptr (the final probabilities, zeros past the top-p cut)
    int64_t* idx_out;          // [rows, k] or nullptr
    uint8_t* seen_mark;        // [rows, vocab] or nullptr: marks the chosen token
    int64_t mstride;
    int vocab, k;
    float temperature, top_p, rep;
};

__device__ __forceinline__ uint32_t okey(float f) {   // larger float -> larger key
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Exclusive prefix sum of one int per thread over the CTA; returns the total.
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int& excl) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;   // inclusive over warps
    }
    __syncthreads();
    excl = x - v + (warp ? warp_sums[warp - 1] : 0);
    const int total = warp_sums[ST / 32 - 1];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(ST, 1) sample_topk_kernel(const __grid_constant__ Params p) {
    __shared__ unsigned hist[256];
    __shared__ int warp_sums[ST / 32];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_rem;
    __shared__ unsigned long long cand[MAXK];   // (key << 32) | ~index: distinct, larger = earlier
    __shared__ float prob[MAXK];
    __shared__ int s_pick;
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    const int tid = threadIdx.x;
    const __half* lg = p.logits + int64_t(row) * p.lstride;
    const uint8_t* seen = p.seen ? p.seen + int64_t(row) * p.sstride : nullptr;
    const int V = p.vocab;
    const int per = (V + ST - 1) / ST;
    const int j0 = min(V, tid * per), j1 = min(V, j0 + per);   // this thread's contiguous index range

    int64_t token;
    if (p.temperature <= 0.f) {   // greedy: first index of the largest raw logit
        unsigned long long best = 0ull;
        for (int j = j0; j < j1; ++j) {
            const unsigned long long key =
                (uint64_t(okey(__half2float(lg[j]))) << 32) | uint64_t(0xffffffffu - uint32_t(j));
            best = key > best ? key : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
            best = y > best ? y : best;
        }
        if ((tid & 31) == 0) cand[tid >> 5] = best;
        __syncthreads();
        if (tid < 32) {
            best = tid < ST / 32 ? cand[tid] : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
                best = y > best ? y : best;
            }
            if (tid == 0) s_pick = int(0xffffffffu - uint32_t(best & 0xffffffffull));
        }
        __syncthreads();
        token = s_pick;
    } else {
        const float rep = p.rep;
        auto value = [&](int j) {
            float l = __half2float(lg[j]);
            if (seen && rep != 1.f && seen[j]) l = l < 0.f ? l * rep : __fdiv_rn(l, rep);
            return l;
        };
        const int K = min(p.k, V);
        // ---- radix selection of the K-th largest key
        if (tid == 0) {
            s_prefix = 0u;
            s_mask = 0u;
            s_rem = K;
        }
        for (int pass = 3; pass >= 0; --pass) {
            for (int b = tid; b < 256; b += ST) hist[b] = 0u;
            __syncthreads();
            const uint32_t pre = s_prefix, msk = s_mask;
            for (int j = j0; j < j1; ++j) {
                const uint32_t key = okey(value(j));
                if ((key & msk) == pre) atomicAdd(&hist[(key >> (8 * pass)) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int rem = s_rem, cum = 0, b = 255;
                for (; b > 0; --b) {
                    if (cum + int(hist[b]) >= rem) break;
                    cum += int(hist[b]);
                }
                s_prefix = pre | (uint32_t(b) << (8 * pass));
                s_mask = msk | (255u << (8 * pass));
                s_rem = rem - cum;   // elements equal to the K-th key still to take
            }
            __syncthreads();
        }
        const uint32_t kth = s_prefix;
        const int take_eq = s_rem;
        // ---- gather: every key above the K-th, the first take_eq equal ones by index
        int n_gt = 0, n_eq = 0;
        for (int j = j0; j < j1; ++j) {
            const uint32_t key = okey(value(j));
            n_gt += key > kth;
            n_eq += key == kth;
        }
        int off_gt, off_eq;
        const int tot_gt = block_scan(n_gt, warp_sums, off_gt);
        block_scan(n_eq, warp_sums, off_eq);
        for (int i = tid; i < MAXK; i += ST) cand[i] = 0ull;
        __syncthreads();
        int pos = off_gt, e = off_eq;
        for (int j = j0; j < j1; ++j) {
            const uint32_t key = okey(value(j));
            const unsigned long long c = (uint64_t(key) << 32) | uint64_t(0xffffffffu - uint32_t(j));
            if (key > kth) {
                cand[pos++] = c;
            } else if (key == kth) {
                if (e < take_eq) cand[tot_gt + e] = c;
                ++e;
            }
        }
        __syncthreads();
        // ---- bitonic sort of MAXK keys, descending
        for (int size = 2; size <= MAXK; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < MAXK; i += ST) {
                    const int jn = i ^ stride;
                    if (jn > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = cand[i], b = cand[jn];
                        if (desc ? a < b : a > b) {
                            cand[i] = b;
                            cand[jn] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        // ---- probabilities (warp 0), top-p, inverse CDF
        if (tid < 32) {
            const float T = p.temperature;
            const float x0 = __fdiv_rn(key_value(uint32_t(cand[0] >> 32)), T);
            float s = 0.f;
            for (int i = tid; i < K; i += 32) {
                const float ei = expf(__fdiv_rn(key_value(uint32_t(cand[i] >> 32)), T) - x0);
                prob[i] = ei;
                s += ei;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            __syncwarp();
            if (tid == 0) {
                float kept = 0.f, cum = 0.f;
                int n_keep = K;
                for (int i = 0; i < K; ++i) {
                    const float pi = __fdiv_rn(prob[i], s);
                    if (p.top_p < 1.f && cum > p.top_p) {   // (cumsum - p_i) > top_p: dropped
                        n_keep = i;
                        break;
                    }
                    cum += pi;
                    prob[i] = pi;
                    kept += pi;
                }
                for (int i = n_keep; i < K; ++i) prob[i] = 0.f;
                float acc = 0.f;
                int pick = n_keep - 1;
                const float u = p.uniform ? p.uniform[row] : 0.f;
                for (int i = 0; i < n_keep; ++i) {
                    prob[i] = __fdiv_rn(prob[i], kept);
                    acc += prob[i];
                    if (u < acc && pick == n_keep - 1) pick = i;
                }
                s_pick = pick;
            }
            __syncwarp();
        }
        __syncthreads();
        if (p.probs_out)
            for (int i = tid; i < K; i += ST) {
                p.probs_out[int64_t(row) * K + i] = prob[i];
                p.idx_out[int64_t(row) * K + i] = int64_t(0xffffffffu - uint32_t(cand[i] & 0xffffffffull));
            }
        token = int64_t(0xffffffffu - uint32_t(cand[s_pick] & 0xffffffffull));
    }
    if (tid == 0) {
        p.token_out[row] = token;
        if (p.seen_mark) p.seen_mark[int64_t(row) * p.mstride + token] = 1;
    }
    if (p.embed) {
        const uint4* src = reinterpret_cast<const uint4*>(p.embed + token * p.embed_dim);
        uint4* dst = reinterpret_cast<uint4*>(p.embed_out + int64_t(row) * p.eostride);
        for (int i = tid; i < p.embed_dim / 8; i += ST) dst[i] = __ldg(src + i);
    }
}

}  // namespace sample
}  // namespace nova

using namespace nova;

extern "C" int nova_sample_topk(const nova_sample_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->rows < 1 || a->rows > 65535 || a->vocab < 1 || a->vocab > (1 << 30))
        return fail(NOVA_ERR_INVALID, "rows in [1, 65535], vocab in [1, 2^30]");
    if (!(a->temperature <= 0.0) && (a->top_k < 1 || a->top_k > sample::MAXK))
        return fail(NOVA_ERR_UNSUPPORTED, "top_k must be in [1, %d]", sample::MAXK);
    if (!a->logits || !a->token_out) return fail(NOVA_ERR_INVALID, "NULL pointer");
    if (!(a->temperature <= 0.0) && !a->uniform) return fail(NOVA_ERR_INVALID, "sampling needs the uniform draws");
    if (!(a->top_p > 0.0) || a->top_p > 1.0) return fail(NOVA_ERR_INVALID, "top_p must be in (0, 1]");
    if (!(a->repetition_penalty > 0.0)) return fail(NOVA_ERR_INVALID, "repetition_penalty must be > 0");
    if ((a->probs_out == nullptr) != (a->idx_out == nullptr))
        return fail(NOVA_ERR_INVALID, "probs_out and idx_out go together");
    if (a->embed && (!a->embed_out || a->embed_dim <= 0 || a->embed_dim % 8 ||
                     reinterpret_cast<uintptr_t>(a->embed) % 16 || reinterpret_cast<uintptr_t>(a->embed_out) % 16 ||
                     a->embed_out_stride % 8))
        return fail(NOVA_ERR_ALIGN, "embedding gather needs 16-byte aligned rows and embed_dim % 8 == 0");
    sample::Params p;
    memset(&p, 0, sizeof(p));
    p.logits = (const __half*)a->logits;
    p.lstride = a->logits_stride;
    p.seen = (const uint8_t*)a->seen;
    p.sstride = a->seen_stride;
    p.uniform = (const float*)a->uniform;
    p.token_out = a->token_out;
    p.embed = (const __half*)a->embed;
    p.embed_out = (__half*)a->embed_out;
    p.eostride = a->embed_out_stride;
    p.embed_dim = int(a->embed_dim);
    p.probs_out = (float*)a->probs_out;
    p.idx_out = a->idx_out;
    p.seen_mark = (uint8_t*)a->seen_mark;
    p.mstride = a->seen_mark_stride;
    p.vocab = int(a->vocab);
    p.k = int(a->temperature <= 0.0 ? 1 : a->top_k);
    p.temperature = float(a->temperature);
    p.top_p = float(a->top_p);
    p.rep = float(a->repetition_penalty);
    const cudaError_t err = launch(sample::sample_topk_kernel, dim3(unsigned(a->rows)), dim3(sample::ST), 0,
                                   (cudaStream_t)stream, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_sample_topk: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}
