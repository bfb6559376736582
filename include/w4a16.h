/*
 * w4a16.h -- C ABI of the B200 (sm_100a) W4A16 GEMM.
 *
 *     y[M, N] = x[M, K] @ W^T,   W[n, k] = (q[n, k] - 8) * scales[k / G, n]
 *
 * x: fp16 [M, K] row-major.  q: 4-bit codes packed into int32 words in the
 * mma.m16n8k16 fragment order of the reference format (word index
 * (((n/16)*(K/64) + k/64)*32 + lane)*4 + (k%64)/16; nibble i of a lane's word
 * holds n = g + 8*((i&3)&1), k = 2t + 8*((i&3)>>1) + (i>>2), g = lane/4,
 * t = lane%4).  scales: fp16 [groups, N] with G = K / groups in {64, 128}.
 *
 * All pointers are CUDA device pointers; `stream` is a cudaStream_t (NULL =
 * legacy default stream).  Functions return W4A16_OK or an error status; the
 * human-readable reason of the last failure on the calling thread is available
 * from w4a16_last_error().  No function allocates device memory except the
 * set-up call w4a16_peer_alloc, so GEMM and exchange launches may be captured in
 * CUDA graphs.
 *
 * Workspace: the decode path (M <= 16) may split K across SMs and combine the
 * split partial sums through a caller-provided device workspace of
 * w4a16_workspace_bytes() bytes (256-byte aligned).  It is scratch: a call
 * writes every byte it later reads, so it needs no initialisation, and one
 * workspace serves any number of calls, of any shapes, issued in stream order.
 * Calls that may run concurrently need separate workspaces.
 *
 * Stream order: each GEMM reads nothing (weights, scales, activations, workspace)
 * before the kernel launched just before it on the stream has completed and its
 * writes are visible, whatever that kernel was.  Kernels are launched with
 * programmatic dependent launch, so the next launch's set-up overlaps the previous
 * one's tail.  A caller whose weights and scales are resident -- not written by the
 * kernel launched immediately before the GEMM -- may pass W4A16_FLAG_WEIGHTS_RESIDENT
 * to w4a16_gemm_ex: the decode kernel then starts streaming them before that
 * kernel has finished.  The environment variable W4A16_PDL=0 (read once per
 * process) launches every kernel in plain stream order and ignores the flag.
 *
 * This header replaces the reference's torch-typed entry point
 *     torch::Tensor w4a16_gemm_cuda(Tensor Wp, Tensor x, Tensor scales, int64_t variant)
 * (akshay919191/W4A16-GEMM src/vectorized/kernel.cu:218, bound as
 * w4a16_opt.w4a16_gemm in src/vectorized/extension.cpp:5-8) with plain
 * pointers and sizes.
 */
#ifndef W4A16_H_
#define W4A16_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W4A16_ABI_VERSION 4

/* Size of the scratch array built into the library for w4a16_gemm_noalloc
 * (6 MiB per device: the decode path's partials on a GPU of up to 192 SMs). */
#define W4A16_NOALLOC_SCRATCH_BYTES (6u << 20)

typedef enum w4a16_status {
    W4A16_OK = 0,
    W4A16_ERR_NULL_POINTER = 1,      /* a required pointer is NULL */
    W4A16_ERR_VARIANT = 2,           /* "variant must be -1 (auto), 0 (decode) or 1..4" (kernel.cu:224) */
    W4A16_ERR_M = 3,                 /* "M must be at least 1" (kernel.cu:227) */
    W4A16_ERR_DIM_RANGE = 4,         /* "dimensions must fit in int32" (kernel.cu:228) */
    W4A16_ERR_K_MULTIPLE = 5,        /* "K must be a multiple of 64" (kernel.cu:230) */
    W4A16_ERR_N_MULTIPLE = 6,        /* "N must be a multiple of 16" (kernel.cu:231) */
    W4A16_ERR_GROUPS = 7,            /* "K must be divisible by the number of groups" (kernel.cu:232) */
    W4A16_ERR_WP_SIZE = 8,           /* "Wp must hold N*K/8 words" (kernel.cu:233) */
    W4A16_ERR_ALIGNMENT = 9,         /* "Wp, x and scales must be 16-byte aligned" (kernel.cu:234-237) */
    W4A16_ERR_GROUP_SIZE = 10,       /* "unsupported group size G, supported: 64, 128" (kernel.cu:240) */
    W4A16_ERR_DECODE_SHAPE = 11,     /* "decode kernel needs M in [1, 16], ..." (kernel.cu:246-249) */
    W4A16_ERR_OUT_DTYPE = 12,        /* out_dtype is not a w4a16_out_dtype value */
    W4A16_ERR_DEVICE = 13,           /* current device is not an sm_100 GPU */
    W4A16_ERR_CUDA = 14,             /* a CUDA runtime / driver call failed */
    W4A16_ERR_DEVICE_TIMEOUT = 15,   /* a kernel's bounded wait ran out (see w4a16_device_status) */
    W4A16_ERR_WORKSPACE = 16,        /* workspace missing, too small or misaligned */
    W4A16_ERR_FLAGS = 17,            /* flags holds bits that are not w4a16_flags values */
    W4A16_ERR_TP_GROUP = 18          /* a w4a16_tp_group or an exchange's sizes are not usable */
} w4a16_status;

typedef enum w4a16_flags {
    /* Wp and scales are not written by the kernel launched immediately before this GEMM on
     * its stream (they were written earlier, copied, or made by this library's format entry
     * points): the decode kernel may start reading them before that kernel completes. */
    W4A16_FLAG_WEIGHTS_RESIDENT = 1,
    /* Decode path, M <= 8: multiply each 64-wide chunk's products by its group scale in fp32
     * after the tensor-core product, instead of multiplying every weight by its scale in
     * fp16 before it.  The products then use the unrounded (q - 8) * scale (more accurate
     * than the reference's fp16-rounded dequantised weights, and about 6 % faster on the
     * decode sweep), so results differ from the default in the last bits; they are not the
     * reference's bit-identical dequantised values.  Ignored for M > 8 and for prefill. */
    W4A16_FLAG_FP32_SCALE = 2
} w4a16_flags;

typedef enum w4a16_out_dtype {
    W4A16_OUT_F16 = 0,               /* y is fp16 [M, N] (the reference's output) */
    W4A16_OUT_F32 = 1                /* y is fp32 [M, N] (row-parallel partial sums) */
} w4a16_out_dtype;

typedef enum w4a16_w_dtype {
    W4A16_W_F32 = 0,                 /* unquantised weights are fp32 [N, K] */
    W4A16_W_F16 = 1                  /* unquantised weights are fp16 [N, K] */
} w4a16_w_dtype;

typedef struct w4a16_route {
    int32_t kernel;     /* 0 = decode (M <= 16 weight-streaming GEMV), 1 = prefill (tcgen05) */
    int32_t config;     /* prefill tile config 1..4 (token tile 32/64/128/256); 0 for decode */
    int32_t tile_m;     /* tokens per tile (decode: 8 or 16 padded rows) */
    int32_t tile_n;     /* output channels per tile (decode 256, prefill 128) */
    int32_t split_k;    /* decode: stream-K work units (256 columns x one 64-wide K chunk); prefill: 1 */
    int32_t grid;       /* CTAs launched */
    int32_t stages;     /* pipeline depth */
    int32_t smem_bytes; /* dynamic shared memory per CTA */
    uint64_t workspace_bytes; /* workspace the call needs (see w4a16_workspace_bytes) */
    int32_t launches;   /* kernels one call launches (decode: 2 when a column group is split
                           across CTAs -- the combine kernel runs behind the main one) */
    int32_t reserved;
} w4a16_route;

/* Version of this ABI (W4A16_ABI_VERSION). */
int32_t w4a16_abi_version(void);

/* Validate a GEMM call without launching anything.  Checks, in the order of
 * the reference (kernel.cu:224-249): variant range, M >= 1, int32 range,
 * K % 64, N % 16, K % groups, wp_words == N*K/8, 16-byte alignment of
 * Wp/x/scales, G = K/groups in {64, 128}, and the decode contract when
 * variant == 0.  Pointers may be NULL here (alignment is then not checked). */
w4a16_status w4a16_validate(const void* Wp, const void* x, const void* scales,
                            int64_t M, int64_t N, int64_t K, int64_t groups,
                            int64_t wp_words, int32_t variant);

/* Bytes of workspace w4a16_gemm needs for this call (0 if none). */
w4a16_status w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t groups, int32_t variant,
                                   uint64_t* bytes);

/* y = x @ W^T on `stream`.  variant: -1 auto, 0 decode kernel (reference decode
 * contract: M <= 16, N % 64 == 0, K % 512 == 0), 1..4 force a prefill tile
 * config.  out_dtype selects fp16 or fp32 y.  Replaces w4a16_gemm_cuda
 * (kernel.cu:218-267); unlike it, y and the workspace are caller-allocated.
 * Same as w4a16_gemm_ex with flags = 0. */
w4a16_status w4a16_gemm(const int32_t* Wp, const void* x, const void* scales, void* y,
                        int64_t M, int64_t N, int64_t K, int64_t groups, int64_t wp_words,
                        int32_t variant, int32_t out_dtype, void* workspace, uint64_t workspace_bytes,
                        void* stream);

/* w4a16_gemm with flags (w4a16_flags bits; 0 = plain stream order).  No counterpart in
 * the reference: its kernels are launched in plain stream order. */
w4a16_status w4a16_gemm_ex(const int32_t* Wp, const void* x, const void* scales, void* y,
                           int64_t M, int64_t N, int64_t K, int64_t groups, int64_t wp_words,
                           int32_t variant, int32_t out_dtype, uint32_t flags, void* workspace,
                           uint64_t workspace_bytes, void* stream);

/* Same GEMM as w4a16_gemm for callers that cannot allocate device memory
 * (fixed device-memory budgets, bindings without a device allocator).  No
 * counterpart in the reference, whose entry point allocates y itself.  The
 * scratch the decode path needs comes from an array of
 * W4A16_NOALLOC_SCRATCH_BYTES built into the library instead of a caller
 * workspace; y stays caller-allocated.  Nothing in it needs to start at zero.
 * Limits: a call whose scratch need exceeds the array fails with
 * W4A16_ERR_WORKSPACE; every call on a device uses the same array, so calls
 * that overlap in time (other streams, other host threads) race -- serialise
 * them.  Each call made outside stream capture looks up the array's device
 * address with the device current (a cheap call); a call under capture uses the
 * address found by the last call outside it, so make at least one call on each
 * device before any stream capture. */
w4a16_status w4a16_gemm_noalloc(const int32_t* Wp, const void* x, const void* scales, void* y,
                                int64_t M, int64_t N, int64_t K, int64_t groups, int64_t wp_words,
                                int32_t variant, int32_t out_dtype, void* stream);

/* The launch w4a16_gemm would make for this call (kernel choice, tiles, grid).
 * Mirrors the reference's routing (kernel.cu:242-249) and prefill config
 * selection (kernel.cu:140-214).  Queries the current device. */
w4a16_status w4a16_query_route(int64_t M, int64_t N, int64_t K, int64_t groups, int32_t variant,
                               w4a16_route* out);

/* out[N, K] (fp16) = the dequantised weights, bit-identical to the reference's
 * dequantize_w4 (tests/quant.py:77-80).  Debug / verification entry. */
w4a16_status w4a16_dequant(const int32_t* Wp, const void* scales, void* out,
                           int64_t N, int64_t K, int64_t groups, void* stream);

/* Load-time weight preparation on the GPU (the steps before the GEMM).  All
 * pointers are device pointers, 16-byte aligned; N % 16 == 0, K % 64 == 0.  Inputs are
 * expected finite.  Return after enqueueing on `stream`; each enqueues its kernel and
 * then an empty kernel, so a GEMM launched right after reads the finished weights. */

/* q: uint8 codes [N, K] (values 0..15; only the low 4 bits are read) -> Wp int32 [N*K/8]
 * in the kernel word order.  Replaces the reference's CPU/torch pack_int4
 * (tests/quant.py:34-48), bit for bit. */
w4a16_status w4a16_pack(const uint8_t* q, int32_t* Wp, int64_t N, int64_t K, void* stream);

/* W [N, K] (fp32 or fp16, w_dtype) -> q uint8 codes [N, K] and scales fp16 [K/G, N]:
 * scale = fp16(max(absmax of the row's G-group / 7, 1e-4)), q = clamp(round-half-even(W /
 * scale), -8, 7) + 8.  Replaces the reference's quantize_w4 (tests/quant.py:62-74), bit for
 * bit.  group_size G in {64, 128}. */
w4a16_status w4a16_quantize(const void* W, int32_t w_dtype, uint8_t* q, void* scales, int64_t N, int64_t K,
                            int64_t group_size, void* stream);

/* w4a16_quantize followed by w4a16_pack in one pass over W (no code array):
 * W -> Wp int32 [N*K/8] and scales fp16 [K/G, N].  No counterpart as one call in the
 * reference (it quantises, then packs). */
w4a16_status w4a16_quantize_pack(const void* W, int32_t w_dtype, int32_t* Wp, void* scales, int64_t N, int64_t K,
                                 int64_t group_size, void* stream);

/* ------------------------------------------------------------------------------
 * Tensor-parallel exchange over peer memory (one process per GPU, one node, GPUs that
 * can map each other's memory, e.g. over NVLink).  No counterpart in the reference,
 * which has no distributed code.  Each rank allocates one exchange buffer with
 * w4a16_peer_alloc, sends its handle to the other ranks (any host channel: e.g.
 * torch.distributed) and maps theirs with w4a16_peer_open.  The first
 * W4A16_TP_CTRL_BYTES of every buffer are the exchange's flags; the caller places its
 * data regions after them (offsets multiples of 16).  Every rank must issue the same
 * exchanges in the same order (on one stream each).  The kernels only load and store
 * peer memory directly (no multicast, no bulk copies from peer memory).  Every wait for
 * a peer is bounded: a peer that never arrives sets the device status (see
 * w4a16_device_status) and the kernel returns instead of hanging. */
#define W4A16_TP_MAX_RANKS 8
#define W4A16_TP_CTRL_BYTES 8192u
/* Largest per-rank contribution (bytes) that an exchange sends in one round (see
 * w4a16_tp_group.recv_off). */
#define W4A16_TP_PUSH_MAX_BYTES (1u << 20)

typedef struct w4a16_ipc_handle {
    unsigned char bytes[64];   /* a cudaIpcMemHandle_t */
} w4a16_ipc_handle;

typedef struct w4a16_tp_group {
    int32_t rank;                          /* this rank, 0 .. world-1 */
    int32_t world;                         /* ranks, 1 .. W4A16_TP_MAX_RANKS */
    void* buf[W4A16_TP_MAX_RANKS];         /* every rank's exchange buffer as mapped here (buf[rank]: own) */
    uint64_t buf_bytes;                    /* size of each buffer */
    /* Optional receive area in every buffer (recv_bytes 0: none).  An exchange whose per-rank
     * contribution c (allgather: M * N / world * 2 bytes, allreduce: M * N * 4 bytes) is at
     * most W4A16_TP_PUSH_MAX_BYTES and fits 2 * world slots of c bytes (rounded up to 256)
     * here runs in one round: every rank stores its contribution into its slot of every
     * peer's receive area and raises one flag, and each rank builds its y from the slots.
     * Other exchanges run in two rounds (a ready flag, then loads from the peers' source
     * regions).  Results are the same either way. */
    uint64_t recv_off;
    uint64_t recv_bytes;
} w4a16_tp_group;

/* Allocates a zero-filled exchange buffer of `bytes` on the current device and its IPC
 * handle (a set-up call: it allocates). */
w4a16_status w4a16_peer_alloc(uint64_t bytes, void** ptr, w4a16_ipc_handle* handle);
/* Maps another process's exchange buffer into this one (current device). */
w4a16_status w4a16_peer_open(const w4a16_ipc_handle* handle, void** ptr);
/* Unmaps a buffer mapped by w4a16_peer_open. */
w4a16_status w4a16_peer_close(void* ptr);
/* Frees a buffer allocated by w4a16_peer_alloc (after every peer has unmapped it). */
w4a16_status w4a16_peer_free(void* ptr);

/* Row-parallel reduction: every rank holds an fp32 partial sum [M, N] at byte offset
 * partial_off of its own buffer.  On return (in stream order) every rank's buffer holds
 * y = the sum of the ranks' partials, added in rank order, as fp16 [M, N] at y_off.  N %
 * (8 * world) == 0.  Replaces an NCCL all-reduce of the partials followed by a cast. */
w4a16_status w4a16_tp_allreduce(const w4a16_tp_group* group, uint64_t partial_off, uint64_t y_off, int64_t M,
                                int64_t N, void* stream);

/* Column-parallel gather: every rank holds its columns y_r fp16 [M, N / world] at byte
 * offset src_off of its own buffer.  On return every rank's buffer holds y fp16 [M, N]
 * at y_off, rank r's columns at [r * N / world, (r + 1) * N / world).  N % (8 * world)
 * == 0.  Replaces an NCCL all-gather and the copy into y's column order. */
w4a16_status w4a16_tp_allgather(const w4a16_tp_group* group, uint64_t src_off, uint64_t y_off, int64_t M,
                                int64_t N, void* stream);

/* Reads the current device's status word, set by a kernel whose bounded wait
 * ran out (0 = none).  Synchronises the device.  reset != 0 clears it. */
w4a16_status w4a16_device_status(int32_t* code, int32_t reset);

/* Diagnostic of the bounded-wait policy: launches two one-thread kernels that each wait for
 * an mbarrier phase nothing completes, with the busy-polling and the sleeping wait the GEMM
 * kernels use.  Each wait gives up after its limit (about 2 s), records its code in the
 * device status word (4, then 1) and returns; codes[0..1] receive the status word read after
 * each kernel, which is then cleared.  Synchronises the device; takes about 4 s. */
w4a16_status w4a16_check_wait_limits(int32_t* codes);

/* Short name of a status code. */
const char* w4a16_status_string(w4a16_status status);

/* Detailed message of the last failing call on this thread ("" if none). */
const char* w4a16_last_error(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* W4A16_H_ */
