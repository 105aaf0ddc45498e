/*
 * nova_b200 -- C ABI of the B200 (sm_100a) kernels for Nova's quantized decode
 * hot path.  Plain pointers, int64 sizes/strides and a cudaStream_t passed as
 * `void*`; no torch types.  Every call is asynchronous on `stream`, allocates
 * nothing and never synchronizes, so all of them can be captured in a CUDA
 * graph.  Every call returns a status code (NOVA_OK == 0); on failure
 * nova_last_error() returns a message (thread-local).  Argument problems are
 * detected on the host before anything is launched.
 *
 * Reference citations are paths inside captain-wangrun-cn/Nova.
 */
#ifndef NOVA_B200_H
#define NOVA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NOVA_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define NOVA_API __attribute__((visibility("default")))
#else
#define NOVA_API
#endif

enum nova_status {
    NOVA_OK = 0,
    NOVA_ERR_INVALID = 1,     /* bad shape / size / range  -> Python ValueError   */
    NOVA_ERR_ALIGN = 2,       /* pointer or stride alignment -> ValueError         */
    NOVA_ERR_UNSUPPORTED = 3, /* valid but not built for (e.g. head_dim != 128)    */
    NOVA_ERR_CUDA = 4         /* launch / runtime failure   -> Python RuntimeError */
};

/* Library identification and the last error message of the calling thread. */
NOVA_API const char* nova_version(void);
/* sizeof of the argument structs, in this order: nova_attn_int8_args,
 * nova_nf4_args, nova_qk_args, nova_prefill_attn_args, nova_qk_prefill_args,
 * nova_sample_args, nova_tp_allreduce_args (n entries at most are written;
 * returns how many there are).  Lets a binding check its struct mirrors. */
NOVA_API int nova_abi_sizes(int64_t* out, int n);
NOVA_API const char* nova_last_error(void);

/* Process-wide launch flags.  Bit 0: launch every kernel with programmatic
 * stream serialization (programmatic dependent launch), so a kernel's
 * prologue -- weight prefetch, LUT build -- overlaps the previous kernel's
 * tail; every kernel waits (griddepcontrol.wait) before touching data a
 * previous kernel writes.  Bit 1: every native-layout NF4 GEMV splits K over
 * the warps of the whole grid (warp-level stream-K); by default only GEMVs
 * with at least two 32-row groups per SM do, smaller ones split each row
 * group over the warps of one CTA.  Default 0.  No counterpart in the
 * reference. */
NOVA_API int nova_set_launch_flags(int flags);
NOVA_API int nova_get_launch_flags(void);

/* ------------------------------------------------------------------ int8 KV */

/*
 * Token-axis int8 quantization ("int8t64"): for each of `rows` independent
 * [n, dim] fp16 matrices, per channel and per group of `group` consecutive
 * tokens: step = max((max-min)/255, 1e-8), q = clamp(rne((x-min)/step), 0, 255);
 * min/step stored as fp16 [ceil(n/group), dim].  A ragged last group uses only
 * its real tokens (the reference pads by repeating the last token, which does
 * not change min/max).  Strides are in elements between consecutive rows.
 * Replaces src/nova/kvquant.py:118-149 quantize_int8(x, group, "token") and the
 * prefill path KVInt8Cache.finish_prefill (src/nova/kvattn.py:745-783).
 */
NOVA_API int nova_kv_quant_int8(const void* x, int64_t x_row_stride, void* q, int64_t q_row_stride, void* mins,
                       void* steps, int64_t s_row_stride, int64_t rows, int64_t n, int64_t dim, int64_t group,
                       void* stream);

/*
 * Inverse of nova_kv_quant_int8: x = fp16(q * step + min).
 * Replaces src/nova/kvquant.py:152-176 dequantize_int8(..., axis="token").
 */
NOVA_API int nova_kv_dequant_int8(const void* q, int64_t q_row_stride, const void* mins, const void* steps,
                         int64_t s_row_stride, void* x, int64_t x_row_stride, int64_t rows, int64_t n, int64_t dim,
                         int64_t group, void* stream);

/*
 * Decode-step append into the streaming int8 cache of one layer.
 * k_new/v_new: fp16 [batch, kv_heads, dim] (strides in elements); the token
 * goes to ring slot pos % group of tail_k/tail_v (fp16 [batch, kv_heads,
 * group, dim]).  When that write completes a group (pos % group == group-1)
 * the ring is requantized into group pos / group of kq/vq (uint8 [batch,
 * kv_heads, max_len, dim]) and kmn/kst/vmn/vst (fp16 [batch, kv_heads,
 * ceil(max_len/group), dim]).  The device scalars become written = pos+1,
 * qlen = group*floor(written/group), pg = qlen/group.  `pos` is read on the
 * device, so one captured graph stays valid as the context grows.
 * Replaces KVInt8Cache.update decode branch (src/nova/kvattn.py:668-691),
 * _quantize_ring (:716-743) and _sync_scalars (:699-710).  The reference
 * requantizes the partially filled ring at every step into a group that is
 * not read until it is full; this call writes it once, when it is full, so
 * every byte that attention reads is identical.
 */
NOVA_API int nova_kv_append_int8(const void* k_new, const void* v_new, int64_t new_b_stride, int64_t new_h_stride,
                        void* tail_k, void* tail_v, void* kq, void* vq, void* kmn, void* kst, void* vmn, void* vst,
                        const int64_t* pos, int64_t* written, int64_t* qlen, int64_t* pg, int64_t batch,
                        int64_t kv_heads, int64_t max_len, int64_t dim, int64_t group, void* stream);

/* ------------------------------------------------------------ attention */

/*
 * Fused GQA decode attention over the streaming int8 cache: int8 prefix
 * [0, min(qlen, pg*group, max_len)) dequantized in registers, plus (when
 * tail_k != NULL) the fp16 ring tail (slot i holds position
 * u - ((u - i) mod group), u = written-1, valid when qlen <= p <= u), one
 * softmax over both, split-K over `chunk`-token splits with the combine done
 * by the last CTA of each (batch, kv head).  window > 0 keeps positions
 * p > u - window (prefix and tail); first (optional) drops p < first.  With a
 * window and n_splits * chunk >= window + 64 the splits are laid over the
 * window (split s starts s * chunk tokens after the window's first 64-token
 * group), so a grid of about (window + 64) / chunk splits suffices whatever
 * max_len is; otherwise split s covers [s * chunk, (s + 1) * chunk).
 * Lengths are device scalars so a captured graph stays valid; n_splits fixes
 * the grid (ceil(max_len/chunk) for a graph).  lse (optional) receives
 * log-sum-exp of the scaled scores (-inf and out = 0 when nothing is valid).
 * Requires head_dim == 128, group == 64, chunk % 64 == 0, q_heads/kv_heads <= 4.
 * Replaces int8_attn_decode (src/nova/kvattn.py:281-427: partial kernel
 * :110-203, combine :206-253), tail_attend (:447-482) and the merge in
 * KVInt8Cache.attend (:835-862).
 */
typedef struct nova_attn_int8_args {
    const void* q;          /* fp16 [batch, q_heads, 128]                      */
    int64_t q_b_stride, q_h_stride;
    const void* kq;         /* uint8 [batch, kv_heads, max_len, 128], contiguous */
    const void* vq;
    const void* kmn;        /* fp16 [batch, kv_heads, groups, 128], contiguous   */
    const void* kst;
    const void* vmn;
    const void* vst;
    const void* tail_k;     /* fp16 [batch, kv_heads, 64, 128] or NULL          */
    const void* tail_v;
    void* out;              /* fp16 [batch, q_heads, 128]                      */
    int64_t o_b_stride, o_h_stride;
    void* lse;              /* fp32 [batch, q_heads] or NULL                   */
    int64_t lse_b_stride;
    const int64_t* qlen;    /* device scalar: int8 prefix length (tokens)     */
    const int64_t* pg;      /* device scalar: valid scale groups              */
    const int64_t* written; /* device scalar or NULL (= qlen): tokens written */
    const int64_t* first;   /* device scalar or NULL (= 0)                    */
    void* workspace;        /* nova_attn_workspace_bytes() bytes, zeroed once  */
    int64_t workspace_bytes;
    int64_t batch, q_heads, kv_heads, max_len, groups, head_dim, group, chunk, n_splits, window;
    /* nova_qk_append_attn_int8 only (ignored elsewhere): non-zero leaves the
       split partials in the workspace for nova_nf4_gemv's attn_part (batch-1
       decode) and writes neither out nor lse.  Partials: floats from byte
       256 + align_up(batch * kv_heads * 4, 256), [batch * kv_heads][n_splits
       + 1][q_heads / kv_heads][132] = m, l, 2 unused, acc[128] (m = -inf:
       nothing valid in that split, acc not written).                        */
    int64_t defer_merge;
} nova_attn_int8_args;

/* Bytes of workspace nova_attn_decode_int8 needs (split partials, per-head
 * arrival counters and an error word).  Zero it once; the kernel leaves the
 * counters at zero when it finishes. */
NOVA_API int nova_attn_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t n_splits, int has_tail,
                              int64_t* bytes);

NOVA_API int nova_attn_decode_int8(const nova_attn_int8_args* args, void* stream);

/* Device error word inside an attention workspace (non-zero = a bounded wait
 * gave up); copies it to *host_value synchronously and clears it. */
NOVA_API int nova_attn_read_error(void* workspace, int64_t batch, int64_t kv_heads, int* host_value);

/* Size of the built-in scratch array of nova_attn_decode_int8_noalloc. */
#define NOVA_ATTN_NOALLOC_SCRATCH_BYTES (4 << 20)

/* nova_attn_decode_int8 for callers that cannot allocate device memory (an
 * allocator-free runtime, or a host whose device memory is all in its own
 * pools): args->workspace and args->workspace_bytes are ignored and the
 * split partials, arrival counters and error word live in a 4 MiB array
 * built into the library, one per device.  Nothing is allocated.  Shapes
 * whose nova_attn_workspace_bytes() exceeds NOVA_ATTN_NOALLOC_SCRATCH_BYTES
 * are rejected with NOVA_ERR_UNSUPPORTED.  The first call on a device looks
 * up the array's address (cudaGetSymbolAddress, with that device current):
 * make it before any stream capture.  Each call clears the counters and the
 * error word on `stream` before the kernel; the array is shared by all calls
 * on the device, so calls that overlap in time (other streams, other host
 * threads) race on it.  No counterpart in the reference, whose decode
 * attention allocates its scratch through torch (src/nova/kvattn.py:281-427). */
NOVA_API int nova_attn_decode_int8_noalloc(const nova_attn_int8_args* args, void* stream);

/* Error word of nova_attn_decode_int8_noalloc on the current device (non-zero
 * = a bounded wait in the latest call gave up and its output is not valid):
 * copied to *host_value synchronously and cleared.  Each call of
 * nova_attn_decode_int8_noalloc clears the word before its kernel, so this
 * reports the most recent call only. */
NOVA_API int nova_attn_noalloc_read_error(int* host_value);

/* ------------------------------------------------------------------ NF4 */

/* Epilogues of nova_nf4_gemv. */
enum nova_nf4_epilogue {
    NOVA_NF4_PLAIN = 0,    /* out = fp16(acc + bias)                                      */
    NOVA_NF4_RESIDUAL = 1, /* out = fp16(residual + fp16(acc))  (decoder residual add)     */
    NOVA_NF4_SILU_MUL = 2, /* rows interleaved per 16-row tile: 8 gate rows, then the 8
                              matching up rows; out[:, n] = fp16(silu(fp16 gate)) * fp16 up,
                              out has N/2 columns (LeanMLP act_fn(gate) * up)              */
    NOVA_NF4_ARGMAX = 3,   /* PLAIN, plus atomicMax of a packed (fp16 logit, -index) key
                              into argmax[m] (uint64, zero before the call): greedy token  */
    NOVA_NF4_F32 = 4,      /* out is fp32 [M, out_stride]: the accumulators unrounded, the
                              partial sum of one tensor-parallel rank before the all-reduce */
    NOVA_NF4_SLOTS = 5     /* native layout, M <= 8: the k-blocks of all row groups are
                              split evenly over one CTA per SM and each CTA writes its
                              fp32 sums of the (at most four) row groups it touches into
                              out = float [SMs][4][M][32], slot = row group - the CTA's
                              first (no residual add, no cross-CTA reduction): the next
                              GEMV adds them while it stages its input (add_slots)      */
};

/* Workspace bytes for nova_nf4_gemv with N output rows on the current device
 * (stream-K partial slots + per-row-tile counters).  Zero it once; a
 * workspace sized for the largest N can be shared by every GEMV launched on
 * one stream (each launch leaves its counters at zero). */
NOVA_API int nova_nf4_workspace_bytes(int64_t n, int64_t* bytes);

/*
 * y[M, N] = x[M, K] (fp16) * W^T with W in NF4: packed uint8 [N, K/2], absmax
 * [K/64, N] (fp32 if absmax_fp32 else fp16), lut = the 256-entry fp16x2
 * codebook table (low half code[b>>4], high half code[b&15]).  fp32
 * accumulation.  M <= 8, N % 16 == 0, K % 64 == 0, M*K*2 + 64 KiB <= 227 KiB.
 *   norm_weight != NULL: x is normalised first (RMSNorm, HF order, eps) --
 *       the input_layernorm / post_attention_layernorm / final norm folded in;
 *   residual/out/argmax per the epilogue; bias (fp16 [N]) only with PLAIN;
 *   token_out != NULL (ARGMAX only): the last warp writes the argmax index of
 *       each row to token_out[m], re-zeroes argmax[m], increments *pos (if
 *       given) and, with embed != NULL, copies embed[token] (fp16 rows of
 *       embed_dim) to embed_out -- the next step's hidden state.
 * Replaces fused_nf4_linear / _nf4_gemv_kernel (src/nova/kernels.py:187-289),
 * NF4Linear.forward (src/nova/quant.py:101-102), fused_rms_norm in front of
 * the projections (src/nova/kernels.py:97-115, src/nova/layers.py:199, :216,
 * src/nova/model.py:179), the 4-bit lm_head (src/nova/model.py:200-204) with
 * the greedy argmax / input_ids / pos update of GraphDecoder._body
 * (src/nova/decode.py:318-319) and the embedding lookup (src/nova/model.py:131),
 * and the residual adds / SiLU*up of src/nova/layers.py:174, :213, :218.
 */
typedef struct nova_nf4_args {
    const void* x;            /* fp16 [m, k]                                   */
    int64_t x_stride;
    const void* norm_weight;  /* fp16 [k] or NULL                              */
    double eps;
    const void* packed;       /* uint8 [n, k/2]                                */
    const void* absmax;       /* [k/64, n]                                      */
    int64_t absmax_fp32;
    const void* lut;          /* uint32 [256]                                  */
    const void* bias;         /* fp16 [n] or NULL                              */
    const void* residual;     /* fp16 [m, n] (RESIDUAL)                        */
    int64_t res_stride;
    void* out;                /* fp16 [m, n] ([m, n/2] for SILU_MUL)           */
    int64_t out_stride;
    void* argmax;             /* uint64 [m] (ARGMAX)                           */
    int64_t* token_out;       /* int64 [m] or NULL                             */
    int64_t* pos;             /* device scalar or NULL                         */
    const void* embed;        /* fp16 [vocab, embed_dim] or NULL               */
    void* embed_out;          /* fp16 [m, embed_dim]                           */
    int64_t embed_out_stride;
    int64_t embed_dim;
    void* workspace;          /* nova_nf4_workspace_bytes(n), zeroed once      */
    int64_t workspace_bytes;
    int64_t m, n, k;
    int64_t epilogue;         /* enum nova_nf4_epilogue                        */
    int64_t layout;           /* 0: reference packed/absmax; 1: native units   */
    /* Deferred row-parallel reduction (with a norm prologue, K <= 8 * 512):
       x = fp16(x + fp16(sum of the SLOTS written by the previous GEMV, whose
       N is this K and whose K is add_k)), summed in a fixed CTA order, is what
       this launch normalizes; CTA 0 also stores it to resid_out (fp16 [m, k],
       stride x_stride; must not alias x).  NULL add_slots: off.             */
    const void* add_slots;
    int64_t add_k;
    void* resid_out;
    /* SiLU·mul split at CTA edges (batch-1 decode, gate|up -> down_proj):
       with edge_out (fp32 [SMs * 2, 32], SILU_MUL, native layout, M = 1) the
       launch writes out only where one CTA holds all k-blocks of a row group
       and leaves, per CTA, the fp32 sums of its first and last row group that
       a neighbouring CTA shares in edge_out[CTA][0 / 1]; a following launch
       with edge_in (that buffer) and edge_k (the producer's K; its own K must
       be the producer's N / 2; no norm prologue; SLOTS or the CTA-level
       schedule) completes those outputs, summed in CTA order with the SiLU·mul
       arithmetic, while it stages x.  The producer's out is then incomplete on
       its own.  NULL: off.                                                   */
    void* edge_out;
    const void* edge_in;
    int64_t edge_k;
    /* o_proj over the decode attention's split partials (batch-1 decode): with
       attn_part (the partials nova_qk_append_attn_int8 left with defer_merge),
       attn_splits (its n_splits + 1) and attn_heads (its kv_heads), an
       NF4_F32 launch at M = 1 takes the head-major unit stream of o_proj (the
       [N, attn_heads * K] matrix with each head's K-column block as rows
       h * N / attn_heads ..: n = attn_heads * N rows, k = the 128 * q_heads /
       kv_heads columns of one head), merges each head's x from the partials
       with the attention's merge arithmetic, and writes fp32 out[h][N] per
       head (x is not read).  add_heads / add_nheads: a launch with a norm
       prologue first adds fp16(sum over h of add_heads[h][0..k)) to x (head
       order), as add_slots does; CTA 0 stores the result to resid_out.      */
    const void* attn_part;
    int64_t attn_splits, attn_heads;
    const void* add_heads;
    int64_t add_nheads;
} nova_nf4_args;

NOVA_API int nova_nf4_gemv(const nova_nf4_args* args, void* stream);

/* Error word inside a nova_nf4_gemv workspace (non-zero = a bounded wait of a
 * launch that used it gave up and that launch's output is not valid): copied
 * to *host_value synchronously and cleared. */
NOVA_API int nova_nf4_gemv_read_error(void* workspace, int* host_value);

/*
 * B200-native NF4 layout: the [N, K] matrix as 32-row x 64-k units, row-group
 * major, each one contiguous 1088-byte record (1024 code bytes in MMA-lane
 * order, then the 32 fp16 absmax values).  nova_nf4_native_bytes gives the
 * size; nova_nf4_pack_native converts the reference layout (packed [N, K/2],
 * absmax [K/64, N]) into it.  Needs N % 32 == 0.  With layout = 1,
 * nova_nf4_gemv takes the unit stream in `packed` and ignores `absmax`.
 * The reference has no counterpart (its GEMV reads the bitsandbytes layout).
 */
NOVA_API int nova_nf4_native_bytes(int64_t n, int64_t k, int64_t* bytes);
NOVA_API int nova_nf4_pack_native(const void* packed, const void* absmax, int absmax_fp32, void* out, int64_t n,
                                  int64_t k, void* stream);

/*
 * The tcgen05 GEMM's unit layout (nf4 args layout = 2): 32-row x 64-k,
 * 1088-byte units in the native layout's order, row-major inside: bytes
 * [16 r, 16 r + 16) = codes of k 0..31 of row r, [512 + 16 r, ...) = k 32..63,
 * then the 32 fp16 absmax in row order.  Same arguments as
 * nova_nf4_pack_native.
 */
NOVA_API int nova_nf4_pack_tc(const void* packed, const void* absmax, int absmax_fp32, void* out, int64_t n,
                              int64_t k, void* stream);

/*
 * Blockwise NF4 quantizer: w fp16 [N, K] -> packed uint8 [N, K/2], absmax
 * [K/64, N].  Level = number of the 15 fp32 `midpoints` below w/absmax (ties
 * to the lower level); an all-zero block uses absmax 1 for the division.
 * Stands in for bitsandbytes quantize_4bit used by the reference loader
 * (src/nova/loader.py:20-42, :86-119), which is not part of the reference tree.
 */
NOVA_API int nova_nf4_quantize(const void* w, int64_t n, int64_t k, const void* midpoints, void* packed, void* absmax,
                               int absmax_fp32, void* stream);

/*
 * NF4 -> fp16 weights [N, K] (code16 * absmax rounded to fp16), for the
 * prefill path.  Same result as the reference test's dequant with the fp16
 * codebook (tests/test_nf4_linear.py:46-57).
 */
NOVA_API int nova_nf4_dequant(const void* packed, const void* absmax, int absmax_fp32, const void* lut, void* out,
                              int64_t n, int64_t k, void* stream);

/* ------------------------------------------------------------ RMSNorm / RoPE */

/*
 * y = RMSNorm(h) * weight in HF order (fp32 mean of squares, 1/sqrt(var+eps),
 * h*r rounded to fp16, times the fp16 weight, rounded to fp16), one row of n
 * per block.  With residual_in: h = fp16(x + residual_in) and, if
 * residual_out != NULL, h is stored there too (fused residual add).
 * Replaces fused_rms_norm / _rms_norm_fwd (src/nova/kernels.py:51-69, :97-115),
 * LeanRMSNorm.forward (src/nova/norm.py:34-42) and the residual add of
 * LeanDecoderLayer.forward (src/nova/layers.py:213).
 */
NOVA_API int nova_rmsnorm(const void* x, int64_t x_stride, const void* residual_in, int64_t rin_stride,
                          void* residual_out, int64_t rout_stride, const void* weight, void* y, int64_t y_stride,
                          int64_t rows, int64_t n, double eps, void* stream);

/*
 * residual[r, i] = fp16(residual[r, i] + fp16(x[r, i])) for fp32 x (strides in
 * elements): the decoder residual add after the tensor-parallel all-reduce of
 * the o_proj / down_proj partial sums, rounded like the single-GPU residual
 * epilogue.  rows <= 65535.  Replaces the residual adds of
 * LeanDecoderLayer.forward (src/nova/layers.py:213, :218) on the sharded path.
 */
NOVA_API int nova_residual_add_f32(const void* x, int64_t x_stride, void* residual, int64_t r_stride, int64_t rows,
                                   int64_t n, void* stream);

/*
 * The decoder's per-head step after the fused q/k/v projection, one launch:
 * qkv row m = [q (q_heads*128) | k (kv_heads*128) | v (kv_heads*128)] fp16;
 * q heads -> q_norm, RoPE at position *pos -> q_out; k heads -> k_norm, RoPE;
 * K and V -> ring slot *pos % 64 and, when that completes a group, the group's
 * int8 requantization, exactly as nova_kv_append_int8; device scalars
 * written/qlen/pg updated.  cos/sin: fp16 [rope_len, 128] tables.
 * Replaces LeanAttention.forward's q_norm / k_norm / apply_rotary_pos_emb /
 * cache.update (src/nova/layers.py:108-133, :24-36; src/nova/kvattn.py:668-743).
 */
typedef struct nova_qk_args {
    const void* qkv;            /* fp16 [batch, (q_heads + 2*kv_heads)*128]      */
    int64_t qkv_stride;
    const void* q_norm_weight;  /* fp16 [128]                                    */
    const void* k_norm_weight;  /* fp16 [128]                                    */
    double eps;
    const void* cos;            /* fp16 [rope_len, 128]                          */
    const void* sin;
    int64_t rope_len;
    void* q_out;                /* fp16 [batch, q_heads*128]                     */
    int64_t q_out_stride;
    void* tail_k;               /* cache of this layer, as nova_kv_append_int8   */
    void* tail_v;
    void* kq;
    void* vq;
    void* kmn;
    void* kst;
    void* vmn;
    void* vst;
    const int64_t* pos;
    int64_t* written;
    int64_t* qlen;
    int64_t* pg;
    int64_t batch, q_heads, kv_heads, head_dim, max_len, group;
} nova_qk_args;

NOVA_API int nova_qk_norm_rope_append(const nova_qk_args* args, void* stream);

/*
 * nova_qk_norm_rope_append followed by nova_attn_decode_int8, in one launch
 * (the decode step's q/k norm + RoPE + ring append and the fused attention of
 * src/nova/decode.py:207-220 / src/nova/kvattn.py:447-482).  attn describes
 * the attention as for nova_attn_decode_int8 except that attn->q, qlen, pg
 * and written are not read: q is normalised and rotated from qk->qkv, and the
 * lengths follow from *qk->pos (written = pos + 1, qlen = written rounded down
 * to 64, pg = qlen / 64; stored to qk->written / qlen / pg for later readers).
 * Both structs must name the same ring and int8 cache, batch, heads and
 * max_len; attn needs the ring (tail_k/tail_v) and n_splits >= 1.  When the
 * new token completes a 64-token group, the group is requantized into the
 * cache and attended in its int8 form, as after the two separate calls.
 * qk->q_out is not written.  Without a window-relative layout, attn->chunk is
 * an upper bound here: the launch splits the prefix it attends into the
 * smallest multiple of 256 tokens that covers it with attn->n_splits splits
 * (at most chunk), so a cache filled far below max_len still gives each warp
 * one 64-token group per split.  With programmatic dependent launch on, the first
 * groups of the int8 prefix are requested before the kernel launched just
 * before this call has finished: that kernel must not write the int8 cache
 * (in the decode step it is the q|k|v projection).
 */
NOVA_API int nova_qk_append_attn_int8(const nova_qk_args* qk, const nova_attn_int8_args* attn, void* stream);

/*
 * Prefill attention on the int8 cache: the queries of a chunk of n tokens at
 * positions [prefix, prefix + n) (q fp16 [batch, q_heads, n, 128], RoPE
 * applied) attend causally to every earlier position and to themselves.
 * Positions [0, int8_len) are read from the int8 cache in place (dequantized
 * as fp16(code * step + min) with the reference's two fp32 roundings),
 * positions [int8_len, prefix + n) from fp16 k / v ([batch, kv_heads, rows,
 * 128], row r = position int8_len + r).  int8_len is 0 (all fp16: a staged
 * prefill) or a multiple of 64 up to prefix (the chunked prefill straight into
 * the int8 cache).  window > 0 keeps positions p > q - window.  fp32 softmax,
 * out = fp16(O / l) in [batch, n, q_heads * 128] layout (row = token).
 * Replaces the SDPA of KVInt8Cache.attend_prefill (src/nova/kvattn.py:791-815)
 * and of the prefill forward (src/nova/layers.py:140-161), and does the
 * reference's planned chunked int8 prefill (reports/kv-int8-streaming-cache.md
 * section 5.1).
 */
typedef struct nova_prefill_attn_args {
    const void* q;            /* fp16, element strides below                    */
    int64_t q_b_stride, q_h_stride, q_t_stride;
    const void* k;            /* fp16 keys / values of positions [int8_len, prefix + n) */
    const void* v;
    int64_t kv_b_stride, kv_h_stride, kv_t_stride;
    const void* kq;           /* int8 cache as for nova_attn_decode_int8, or NULL */
    const void* vq;
    const void* kmn;
    const void* kst;
    const void* vmn;
    const void* vst;
    int64_t max_len, groups;
    void* out;                /* fp16 [batch, n, q_heads * 128]                 */
    int64_t o_b_stride, o_t_stride;
    int64_t batch, q_heads, kv_heads, head_dim, n, prefix, int8_len, window;
} nova_prefill_attn_args;

NOVA_API int nova_attn_prefill_int8(const nova_prefill_attn_args* args, void* stream);

/*
 * The prefill's per-head step for a chunk of n q|k|v rows at positions
 * pos0 .. pos0 + n - 1: q heads -> q_norm + RoPE -> q_out [batch, q_heads, n,
 * 128]; k heads -> k_norm (-> k_pre, optional: the captured, un-rotated K of
 * the memory store) + RoPE -> k_out [batch, kv_heads, n, 128]; v -> v_out
 * (same layout).  The arithmetic of nova_qk_norm_rope_append.  Replaces
 * q_norm / k_norm / apply_rotary_pos_emb of LeanAttention.forward for a
 * prompt (src/nova/layers.py:108-124).
 */
typedef struct nova_qk_prefill_args {
    const void* qkv;            /* fp16 [batch, n, (q_heads + 2*kv_heads)*128]   */
    int64_t qkv_b_stride, qkv_t_stride;
    const void* q_norm_weight;
    const void* k_norm_weight;
    double eps;
    const void* cos;            /* fp16 [rope_len, 128]                          */
    const void* sin;
    int64_t rope_len;
    void* q_out;
    void* k_out;
    void* k_pre;                /* or NULL                                       */
    void* v_out;
    int64_t q_b_stride, q_h_stride, kv_b_stride, kv_h_stride;   /* token stride 128 */
    int64_t batch, q_heads, kv_heads, head_dim, n, pos0;
} nova_qk_prefill_args;

NOVA_API int nova_qk_prefill(const nova_qk_prefill_args* args, void* stream);

/*
 * Batched NF4 GEMM for M >= 1 rows (M <= 64: batched decode; above: prefill):
 * y = x @ dequant(W)^T computed as the reference kernel does
 * (src/nova/kernels.py:213-232): per 64-element block the fp32 sum of
 * code * x (fp16 codebook values, products exact), times the block's absmax,
 * accumulated in fp32; the epilogues of nova_nf4_gemv (PLAIN without bias,
 * RESIDUAL, SILU_MUL, ARGMAX with the step finalize, F32).  No norm prologue
 * (normalize x with nova_rmsnorm).  Weights in the tcgen05 unit layout
 * (layout = 2, from nova_nf4_pack_tc): codes decoded into tensor-memory A
 * tiles, x tiles by TMA, block sums in tensor memory, (tile, k-block) work
 * split evenly over one wave of CTAs with deterministic partial sums.  M > 64
 * (no ARGMAX epilogue, no step finalize): 128 x 256 tiles, each weight
 * k-block as fp16 hi + lo terms (code * absmax = hi + lo to ~2^-22) so that
 * all of K accumulates in tensor memory in fp32.  Other layouts:
 * NOVA_ERR_UNSUPPORTED.
 * x needs a 16-byte aligned base and a row stride that is a multiple of 8.
 * Workspace: nova_nf4_gemm_workspace_bytes(), zeroed once.
 * Replaces NF4Linear.forward / fused_nf4_linear for batched rows
 * (src/nova/quant.py:101-102, src/nova/kernels.py:243-289).
 */
NOVA_API int nova_nf4_gemm_workspace_bytes(int64_t n, int64_t k, int64_t* bytes);
NOVA_API int nova_nf4_gemm(const nova_nf4_args* args, void* stream);
/* Error word inside a nova_nf4_gemm workspace, as nova_nf4_gemv_read_error. */
NOVA_API int nova_nf4_gemm_read_error(void* workspace, int* host_value);

/*
 * Next-token sampling from the logits buffer, outside the decode graph
 * (sample_next, src/chat.py:46-75): temperature <= 0 -> the first index of the
 * largest logit; otherwise fp32 logits with the repetition penalty on seen
 * tokens (l < 0 ? l * rp : l / rp), the top_k largest (ties at the boundary by
 * lowest index), softmax(vals / temperature), tokens whose exclusive cumulative
 * probability exceeds top_p dropped, renormalized, and the token picked by
 * inverse CDF with uniform[row] in [0, 1) (the reference draws with
 * torch.multinomial from the same probabilities).  Optional: the final
 * probabilities and token ids in descending order (probs_out / idx_out,
 * [rows, top_k]), the chosen token's embedding row gathered into embed_out
 * (the next graph step's input), and seen_mark[row, token] = 1.
 * top_k in [1, 256].  One CTA per row; no allocation.
 */
typedef struct nova_sample_args {
    const void* logits;        /* fp16 [rows, vocab]                              */
    int64_t logits_stride;
    const void* seen;          /* uint8 [rows, vocab] or NULL                     */
    int64_t seen_stride;
    const void* uniform;       /* fp32 [rows] (unused when temperature <= 0)      */
    int64_t* token_out;        /* int64 [rows]                                    */
    const void* embed;         /* fp16 [vocab, embed_dim] or NULL                 */
    void* embed_out;           /* fp16 [rows, embed_dim]                          */
    int64_t embed_out_stride;
    int64_t embed_dim;
    void* probs_out;           /* fp32 [rows, top_k] or NULL                      */
    int64_t* idx_out;          /* int64 [rows, top_k] or NULL                     */
    void* seen_mark;           /* uint8 [rows, vocab] or NULL                     */
    int64_t seen_mark_stride;
    int64_t rows, vocab, top_k;
    double temperature, top_p, repetition_penalty;
} nova_sample_args;

NOVA_API int nova_sample_topk(const nova_sample_args* args, void* stream);

/* --------------------------------------------------- tensor parallelism */

/*
 * All-reduce of the tensor-parallel partial sums of o_proj / down_proj fused
 * with the decoder residual add, over NVLink peer memory:
 *     residual = fp16(residual + fp16(sum over ranks of partial))
 * with the rank sum taken in rank order, so every rank computes identical
 * bits.  Each rank allocates a receive buffer of nova_tp_recv_bytes() bytes
 * (zeroed), shares it with nova_ipc_handle / nova_ipc_open, and passes every
 * rank's buffer (its own included) in recv[0..world-1], in rank order.  The
 * call stores this rank's partial, stamped with a device epoch (advanced by
 * the call itself, so graph replays work), into every buffer and polls its
 * own buffer until every rank's stamped values have arrived; a wait that
 * exceeds timeout_ns (default 2 s) sets *err to 1 and leaves the rest of the
 * residual unchanged instead of hanging.  Every rank must make the same
 * sequence of calls.  n even; epoch (int64), counter (uint32) and err (int32)
 * are device words of this rank, zeroed once.  Replaces the residual adds of
 * src/nova/layers.py:213, :218 on the sharded path; the all-reduce itself has
 * no counterpart in the single-GPU reference.
 */
typedef struct nova_tp_allreduce_args {
    const void* partial;      /* fp32 [rows, n], contiguous, 8-byte aligned    */
    void* residual;           /* fp16 [rows, res_stride]                       */
    int64_t res_stride;
    void* recv[8];            /* receive buffer of every rank, in rank order   */
    int64_t* epoch;
    void* counter;
    int* err;
    int64_t rows, n, rank, world;
    int64_t timeout_ns;       /* 0 = 2 s                                       */
} nova_tp_allreduce_args;

NOVA_API int nova_tp_recv_bytes(int64_t world, int64_t rows, int64_t n, int64_t* bytes);
NOVA_API int nova_tp_allreduce_add(const nova_tp_allreduce_args* args, void* stream);

/* CUDA IPC of a device buffer: handle (64 bytes) + offset of ptr inside its
 * allocation; open maps a peer's buffer into this process (returns the
 * buffer pointer and the mapping base to pass to nova_ipc_close). */
NOVA_API int nova_ipc_handle(const void* ptr, void* handle, int64_t* offset);
NOVA_API int nova_ipc_open(const void* handle, int64_t offset, void** ptr, void** base);
NOVA_API int nova_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

#endif /* NOVA_B200_H */
