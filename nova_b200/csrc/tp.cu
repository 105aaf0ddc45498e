// Tensor-parallel all-reduce of the o_proj / down_proj partial sums, fused
// with the residual add, over NVLink peer memory (sm_100a).
//
// Every rank owns a receive buffer (nova_tp_recv_bytes) that all ranks map
// through CUDA IPC: [2 parities][world][count] 8-byte words, each holding one
// fp32 value in its low half and a 32-bit epoch stamp in its high half
// (the "LL" idea: a reader that sees the stamp sees the value of the same
// 8-byte store, so no fences or separate flags are needed).  One launch
// (grid = chunks of the [rows, n] partial):
//   1. CTA c stores its chunk of this rank's partial, stamped with the epoch,
//      into slot `rank` of every rank's buffer (parity = epoch & 1);
//   2. each thread polls, in its own buffer, the words of every rank for the
//      elements it owns until their stamps match (bounded by a time limit),
//      adding them in rank order -- the same order on every rank, so all
//      ranks compute identical bits;
//   3. residual = fp16(residual + fp16(sum)), rounded like the single-GPU
//      residual epilogue.
// The epoch lives in device memory and is advanced by the last CTA, so a
// captured graph replays correctly.  Two parities keep a fast rank's next
// all-reduce from overwriting words a slow rank is still reading: a rank can
// start epoch e+2 only after every peer has sent epoch e+1, which each peer
// does after finishing epoch e.  No TMA, no multicast: plain 16-byte stores to
// peer memory and volatile polling of local memory.
//
// Large partials (batched decode) take two phases instead, cutting what each
// rank sends from (world - 1) x count words to ~1.5 x count x (world - 1) /
// world: rank r owns slice r of the elements;
//   1. every rank stores slice d of its partial, stamped, into rank d's buffer;
//   2. rank r sums its slice from every rank in rank order (the same bits as
//      the one-shot path), applies the residual add, and stores the finished
//      fp16 pairs (2 values + stamp per 8-byte word) into every rank's buffer;
//   3. every rank copies the other slices' finished pairs into its residual.
// A thread stores all it sends before it waits, phase 2 waits only on phase-1
// stores and phase 3 only on phase-2 stores, and the grid is resident, so no
// wait is circular; every rank's epoch e+1 still needs words that each peer
// writes only after finishing epoch e, so the two parities stay sufficient.
#include "common.cuh"

namespace nova {
namespace tp {

constexpr int MAX_WORLD = 8;
constexpr int MAX_CHUNKS = 32;
constexpr int THREADS = 128;
constexpr int64_t TWO_PHASE_MIN = 16384;   // elements (rows * n) from which the two-phase exchange is used

struct Params {
    const float* part;             // [rows, n] this rank's partial sums (contiguous)
    __half* resid;                 // [rows, r_stride]
    int64_t r_stride;
    uint8_t* bufs[MAX_WORLD];      // every rank's receive buffer, mapped in this process
    int64_t* epoch;                // device epoch counter (local)
    unsigned* done;                // CTA arrival counter (local)
    int* err;                      // error word (local)
    int64_t count, chunk;          // rows * n, elements per CTA (multiple of 4)
    int64_t slice;                 // two-phase: elements per rank's slice (even)
    int rows, n, rank, world;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// LL words: low 32 bits = fp32 data, high 32 bits = epoch stamp.  A reader
// that sees the stamp sees the data of the same 8-byte store.
__device__ __forceinline__ uint64_t* words_of(uint8_t* buf, int parity, int src, int64_t count) {
    return reinterpret_cast<uint64_t*>(buf) + (int64_t(parity) * MAX_WORLD + src) * count;
}
__device__ __forceinline__ void st_ll(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_ll(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__global__ void __launch_bounds__(THREADS) allreduce_add_kernel(const __grid_constant__ Params p) {
    __shared__ int s_last;
    pdl_trigger();
    pdl_wait();   // the partial sums come from the previous kernel
    const int c = blockIdx.x;
    const int64_t e = *p.epoch + 1;
    const uint64_t stamp = uint64_t(uint32_t(e)) << 32;
    const int par = int(e & 1);
    const int64_t lo = int64_t(c) * p.chunk;
    const int64_t hi = min(p.count, lo + p.chunk);
    // 1. this rank's chunk, stamped, into slot `rank` of every rank's buffer
    for (int64_t i = lo + 2 * threadIdx.x; i < hi; i += 2 * THREADS) {
        const float2 v = *reinterpret_cast<const float2*>(p.part + i);
        const uint64_t a = stamp | __float_as_uint(v.x), b = stamp | __float_as_uint(v.y);
        for (int r = 0; r < p.world; ++r) st_ll(words_of(p.bufs[r], par, p.rank, p.count) + i, a, b);
    }
    // 2. every rank's words for the same elements, summed in rank order as they arrive
    const unsigned long long t0 = gtime();
    bool ok = true;
    for (int64_t i = lo + 2 * threadIdx.x; i < hi && ok; i += 2 * THREADS) {
        float acc0 = 0.f, acc1 = 0.f;
        for (int r = 0; r < p.world && ok; ++r) {
            const uint64_t* w = words_of(p.bufs[p.rank], par, r, p.count) + i;
            uint64_t a, b;
            ld_ll(w, a, b);
            while ((a >> 32) != (stamp >> 32) || (b >> 32) != (stamp >> 32)) {
                if (gtime() - t0 > p.timeout_ns) {
                    atomicExch(p.err, 1);
                    ok = false;
                    break;
                }
                ld_ll(w, a, b);
            }
            acc0 += __uint_as_float(uint32_t(a));
            acc1 += __uint_as_float(uint32_t(b));
        }
        if (!ok) break;
        const int64_t row = i / p.n, col = i % p.n;   // n even: the pair stays in one row
        __half2* rp = reinterpret_cast<__half2*>(p.resid + row * p.r_stride + col);
        const float2 r0 = __half22float2(*rp);
        *rp = __floats2half2_rn(r0.x + __half2float(__float2half_rn(acc0)), r0.y + __half2float(__float2half_rn(acc1)));
    }
    // the last CTA publishes the epoch for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(p.done, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) {
            *p.done = 0u;
            *p.epoch = e;
        }
    }
}

__global__ void __launch_bounds__(THREADS) allreduce_add_2phase_kernel(const __grid_constant__ Params p) {
    __shared__ int s_last;
    pdl_trigger();
    pdl_wait();
    const int64_t e = *p.epoch + 1;
    const uint32_t st32 = uint32_t(e);
    const uint64_t stamp = uint64_t(st32) << 32;
    const int par = int(e & 1);
    const int64_t npairs = p.count / 2;
    const int64_t tid = int64_t(blockIdx.x) * THREADS + threadIdx.x, nthr = int64_t(gridDim.x) * THREADS;
    const int64_t my_lo = int64_t(p.rank) * p.slice, my_hi = min(p.count, my_lo + p.slice);
    // 1. slice d of this rank's partial into slot `rank` of rank d's buffer
    for (int64_t q = tid; q < npairs; q += nthr) {
        const int64_t i = 2 * q;
        const int d = int(i / p.slice);
        const float2 v = *reinterpret_cast<const float2*>(p.part + i);
        st_ll(words_of(p.bufs[d], par, p.rank, p.count) + i, stamp | __float_as_uint(v.x), stamp | __float_as_uint(v.y));
    }
    const unsigned long long t0 = gtime();
    bool ok = true;
    // 2. this rank's slice: sum in rank order, residual add, finished pairs to every rank
    for (int64_t i = my_lo + 2 * tid; i < my_hi && ok; i += 2 * nthr) {
        float acc0 = 0.f, acc1 = 0.f;
        for (int r = 0; r < p.world && ok; ++r) {
            const uint64_t* w = words_of(p.bufs[p.rank], par, r, p.count) + i;
            uint64_t a, b;
            ld_ll(w, a, b);
            while (uint32_t(a >> 32) != st32 || uint32_t(b >> 32) != st32) {
                if (gtime() - t0 > p.timeout_ns) {
                    atomicExch(p.err, 1);
                    ok = false;
                    break;
                }
                ld_ll(w, a, b);
            }
            acc0 += __uint_as_float(uint32_t(a));
            acc1 += __uint_as_float(uint32_t(b));
        }
        if (!ok) break;
        const int64_t row = i / p.n, col = i % p.n;
        __half2* rp = reinterpret_cast<__half2*>(p.resid + row * p.r_stride + col);
        const float2 r0 = __half22float2(*rp);
        const __half2 h = __floats2half2_rn(r0.x + __half2float(__float2half_rn(acc0)),
                                            r0.y + __half2float(__float2half_rn(acc1)));
        *rp = h;
        const uint64_t word = stamp | uint64_t(*reinterpret_cast<const uint32_t*>(&h));
        for (int r = 0; r < p.world; ++r)
            if (r != p.rank)
                asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(words_of(p.bufs[r], par, p.rank, p.count) + i),
                             "l"(word)
                             : "memory");
    }
    // 3. the other ranks' finished pairs
    for (int64_t q = tid; q < npairs && ok; q += nthr) {
        const int64_t i = 2 * q;
        const int src = int(i / p.slice);
        if (src == p.rank) continue;
        const uint64_t* w = words_of(p.bufs[p.rank], par, src, p.count) + i;
        uint64_t a;
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(w) : "memory");
        while (uint32_t(a >> 32) != st32) {
            if (gtime() - t0 > p.timeout_ns) {
                atomicExch(p.err, 1);
                ok = false;
                break;
            }
            asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(w) : "memory");
        }
        if (!ok) break;
        const int64_t row = i / p.n, col = i % p.n;
        const uint32_t hv = uint32_t(a);
        *reinterpret_cast<__half2*>(p.resid + row * p.r_stride + col) = *reinterpret_cast<const __half2*>(&hv);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(p.done, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) {
            *p.done = 0u;
            *p.epoch = e;
        }
    }
}

}  // namespace tp
}  // namespace nova

using namespace nova;

extern "C" int nova_tp_recv_bytes(int64_t world, int64_t rows, int64_t n, int64_t* bytes) {
    if (!bytes) return fail(NOVA_ERR_INVALID, "bytes must not be NULL");
    if (world < 1 || world > tp::MAX_WORLD || rows < 1 || n < 2 || n % 2)
        return fail(NOVA_ERR_INVALID, "need 1 <= world <= 8, rows >= 1 and an even n");
    *bytes = 2 * int64_t(tp::MAX_WORLD) * rows * n * 8;
    return NOVA_OK;
}

extern "C" int nova_tp_allreduce_add(const nova_tp_allreduce_args* a, void* stream) {
    if (!a) return fail(NOVA_ERR_INVALID, "args must not be NULL");
    if (a->world < 1 || a->world > tp::MAX_WORLD || a->rank < 0 || a->rank >= a->world)
        return fail(NOVA_ERR_INVALID, "bad rank %lld of world %lld", (long long)a->rank, (long long)a->world);
    if (a->rows < 1 || a->n < 2 || a->n % 2 || a->rows * a->n > (int64_t(1) << 30))
        return fail(NOVA_ERR_INVALID, "n must be a positive even number");
    if (!a->partial || !a->residual || !a->epoch || !a->counter || !a->err)
        return fail(NOVA_ERR_INVALID, "NULL pointer");
    auto mis = [](const void* ptr, int al) { return reinterpret_cast<uintptr_t>(ptr) % al != 0; };
    if (mis(a->partial, 8) || mis(a->residual, 4) || (a->res_stride % 2) || mis(a->epoch, 8))
        return fail(NOVA_ERR_ALIGN, "partial 8-byte, residual 4-byte (even stride), epoch 8-byte aligned");
    tp::Params p;
    for (int r = 0; r < tp::MAX_WORLD; ++r) {
        p.bufs[r] = nullptr;
        if (r < a->world) {
            if (!a->recv[r] || mis(a->recv[r], 16)) return fail(NOVA_ERR_INVALID, "recv[%d] missing or unaligned", r);
            p.bufs[r] = (uint8_t*)a->recv[r];
        }
    }
    p.part = (const float*)a->partial;
    p.resid = (__half*)a->residual;
    p.r_stride = a->res_stride;
    p.epoch = a->epoch;
    p.done = (unsigned*)a->counter;
    p.err = a->err;
    p.count = a->rows * a->n;
    p.rows = int(a->rows);
    p.n = int(a->n);
    p.rank = int(a->rank);
    p.world = int(a->world);
    p.timeout_ns = a->timeout_ns > 0 ? (unsigned long long)a->timeout_ns : 2000000000ull;
    const int64_t chunks = std::min<int64_t>(tp::MAX_CHUNKS, (p.count + 255) / 256);
    p.chunk = ((p.count + chunks - 1) / chunks + 1) / 2 * 2;
    const int64_t grid = (p.count + p.chunk - 1) / p.chunk;
    p.slice = ((p.count + p.world - 1) / p.world + 1) / 2 * 2;
    // one shot below 16K elements (latency: one exchange), two phases above (bandwidth)
    const bool two_phase = p.world > 1 && p.count >= tp::TWO_PHASE_MIN;
    const cudaError_t err =
        two_phase ? launch(tp::allreduce_add_2phase_kernel, dim3(unsigned(tp::MAX_CHUNKS)), dim3(tp::THREADS), 0,
                           (cudaStream_t)stream, p)
                  : launch(tp::allreduce_add_kernel, dim3(unsigned(grid)), dim3(tp::THREADS), 0, (cudaStream_t)stream,
                           p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "nova_tp_allreduce_add: launch failed: %s", cudaGetErrorString(err));
    }
    return NOVA_OK;
}

extern "C" int nova_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) return fail(NOVA_ERR_INVALID, "NULL argument");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "cudaIpcGetMemHandle failed");
    }
    void* base = nullptr;
    // the handle names the whole allocation; find where ptr sits inside it
    using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn range = nullptr;
    if (!range) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess || !f) {
            cudaGetLastError();
            return fail(NOVA_ERR_CUDA, "cuMemGetAddressRange unavailable");
        }
        range = (RangeFn)f;
    }
    CUdeviceptr b = 0;
    size_t sz = 0;
    if (range(&b, &sz, (CUdeviceptr)ptr) != CUDA_SUCCESS) return fail(NOVA_ERR_CUDA, "cuMemGetAddressRange failed");
    base = (void*)b;
    memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)((const uint8_t*)ptr - (const uint8_t*)base);
    return NOVA_OK;
}

extern "C" int nova_ipc_open(const void* handle, int64_t offset, void** ptr, void** base) {
    if (!handle || !ptr || !base || offset < 0) return fail(NOVA_ERR_INVALID, "bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* b = nullptr;
    if (cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "cudaIpcOpenMemHandle failed");
    }
    *base = b;
    *ptr = (uint8_t*)b + offset;
    return NOVA_OK;
}

extern "C" int nova_ipc_close(void* base) {
    if (!base) return NOVA_OK;
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        cudaGetLastError();
        return fail(NOVA_ERR_CUDA, "cudaIpcCloseMemHandle failed");
    }
    return NOVA_OK;
}
