/*
 * kvb_cuda.h -- C ABI of the B200 paged decode-attention library (libkvbcuda.so).
 *
 * This is the boundary a host binds to. Every entry point is extern "C", takes plain pointers,
 * sizes and plain structs, returns a status code, and never throws. The text of the last error
 * of the calling thread is available from kvb_last_error().
 *
 * Two levels:
 *   1. The reference-facing level (kvb_available ... kvb_flush_caches) implements, one for one,
 *      the functions of kv-cache-bench's C++ host API src/metal_attn.hpp (cited per function).
 *      kv_cache_bench_b200/csrc/metal_attn_cuda.cpp turns these into the C++ API itself (a
 *      drop-in for src/metal_attn.mm). Buffers are CUDA managed memory, which the host fills
 *      in place as it fills the reference's shared-storage MTLBuffers; lengths are checked on the
 *      host before any device work, and calls are synchronous unless pipelined mode is on.
 *   2. The stream level (kvb_paged_workspace_bytes, kvb_paged_decode_async) takes device
 *      pointers and a CUDA stream, reads nothing on the host, allocates nothing and never
 *      synchronizes. It is what a serving framework or a CUDA graph calls.
 *
 * Layouts (src/reference.hpp:38-58, src/metal_attn.hpp:53-69):
 *   q, out       float [B][H][D]
 *   k, v pools   [num_blocks][Hkv][page_size][D] of fp32, fp16 or int8
 *   block_table  int32 [B][max_blocks], -1 for unused entries
 *   seq_lens     int32 [B]
 *   k/v scales   float [num_blocks][Hkv] (int8 pools only), value = int8 * scale
 * Query head h reads KV head h / (H / Hkv). The softmax scale is 1/sqrt(D).
 */
#ifndef KVB_CUDA_H
#define KVB_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. KVB_ERR_INVALID corresponds to the reference's std::invalid_argument (raised
 * before any device work, outputs untouched), KVB_ERR_DEVICE to its std::runtime_error. */
enum {
    KVB_OK = 0,
    KVB_ERR_INVALID = 1,   /* bad argument; nothing was launched */
    KVB_ERR_DEVICE = 2,    /* CUDA error (launch, allocation, synchronization) */
    KVB_ERR_NO_DEVICE = 3, /* no CUDA device */
    KVB_ERR_STATE = 4      /* call out of order (e.g. end_pipelined without begin) */
};

/* Storage type of the K/V pools: src/metal_attn.hpp:37 (KvType). */
enum { KVB_F32 = 0, KVB_F16 = 1, KVB_I8 = 2 };

/* Kernel selection for kvb_paged_args.kernel. AUTO picks, in order, the first kernel that supports
 * the call:
 *   UMMA  tcgen05 tensor cores + TMA + tensor memory: fp16/int8, head dim 128, page size 8, 16, 32,
 *         64, 128 or 256, at most 8 query heads per KV-head group;
 *   MMA   mma.sync tensor cores + TMA: fp16/int8 with 128- or 256-byte rows, page size 8, 16, 32,
 *         64, 128 or 256, at most 8 query heads per group;
 *   SIMT  CUDA cores: every storage type, page size, head dim and group size. */
enum { KVB_KERNEL_AUTO = 0, KVB_KERNEL_SIMT = 1, KVB_KERNEL_MMA = 2, KVB_KERNEL_UMMA = 3 };

/* src/reference.hpp:17-23 (Shape). */
typedef struct kvb_shape {
    int batch;        /* B */
    int num_heads;    /* H, query heads */
    int num_kv_heads; /* Hkv; H % Hkv == 0 */
    int head_dim;     /* D, 64 or 128 */
} kvb_shape;

/* src/metal_attn.hpp:53-69 (PagedArgs), field for field, plus the pool size and a kernel choice.
 * num_blocks is the number of physical blocks in the K and V pools; block ids of live blocks are
 * checked against it (the reference does not check them at all). */
typedef struct kvb_paged_args {
    kvb_shape shape;
    int kv_type;          /* KVB_F32 / KVB_F16 / KVB_I8 */
    int page_size;        /* tokens per block, > 0 */
    int max_blocks;       /* row stride of block_table */
    int max_len;          /* longest sequence; sizes the split-K workspace. 0: all empty, out = 0 */
    int part_tokens;      /* split-K partition size; 0 = chosen by the library for B200 */
    const float* q;
    const void* k;
    const void* v;
    const int32_t* block_table;
    const int32_t* seq_lens;
    float* out;
    int share_kv;         /* 1: one CTA serves every query head of a KV head (GQA); 0: one per query head */
    const float* k_scale; /* required for KVB_I8 */
    const float* v_scale;
    int64_t num_blocks;   /* physical blocks in the pools (> 0 when any sequence is non-empty) */
    int kernel;           /* KVB_KERNEL_* */
    int flags;            /* KVB_FLAG_* (no counterpart in the reference); 0 for the default */
} kvb_paged_args;

/* kvb_paged_args.flags.
 * KVB_FLAG_TABLES_READY: seq_lens and block_table are not written by the kernel launched right
 *   before this call on the same stream (host copies, and kernels launched earlier, are fine). The
 *   tensor-core kernel then reads them while that kernel finishes (programmatic dependent launch)
 *   instead of after it; q, the pools, the scales and the workspace are still read after it. A
 *   decode loop whose tables come from host copies, or that launches steps back to back, sets it. */
#define KVB_FLAG_TABLES_READY 1
/* KVB_FLAG_INPUTS_READY (with KVB_FLAG_TABLES_READY): q, the K/V pools and the int8 scales are not
 *   written by the kernel launched right before this call on the same stream either. The tcgen05
 *   and CUDA-core kernels then read the pages while that kernel finishes: each warp (thread) waits
 *   for it only before its first access to the workspace or the output. Back-to-back decode steps,
 *   and steps whose inputs arrive by host copy, set it; a step right after the kernel that appends
 *   to the cache or computes q does not. */
#define KVB_FLAG_INPUTS_READY 2
/* KVB_FLAG_STEP_STREAM (with KVB_FLAG_INPUTS_READY): this call is one of a stream of independent
 *   decode steps launched back to back on one stream, and their throughput matters more than the
 *   latency of one step. With fewer (sequence, head group) pairs than a third of the SMs, the tcgen05
 *   kernel then splits the context into fewer, longer partitions, so that a step's grid covers about
 *   a third of the SMs and three consecutive steps stream at once, each overlapping the others'
 *   first and last microseconds (config 3 int8 on B200: 14.2 -> 10.3 us per step over 1000 steps).
 *   A step that runs alone takes longer, since its grid covers a third of the SMs. */
#define KVB_FLAG_STEP_STREAM 4

/* src/metal_attn.hpp:71-80 (NaiveArgs): contiguous cache [B][Hkv][max_len][D], fp32 or fp16. */
typedef struct kvb_naive_args {
    kvb_shape shape;
    int kv_type;
    int max_len;
    const float* q;
    const void* k;
    const void* v;
    const int32_t* seq_lens;
    float* out;
} kvb_naive_args;

/* ---- reference-facing level ----------------------------------------------------------------- */

/* src/metal_attn.hpp:13 metal_available(): 1 if a CUDA device is usable, else 0. */
int kvb_available(void);

/* src/metal_attn.hpp:14 device_name(): writes the device name (NUL-terminated, truncated to
 * `len`). */
int kvb_device_name(char* buf, size_t len);

/* src/metal_attn.hpp:18-33 Buffer(bytes) / ~Buffer(): host-visible, device-usable memory of at
 * least max(bytes, 16) bytes (CUDA managed memory; the same pointer serves data() and handle()). */
int kvb_buffer_alloc(size_t bytes, void** ptr);
int kvb_buffer_free(void* ptr);

/* src/metal_attn.hpp:86 run_paged() and :91 run_paged_steps(): `steps` decode steps, one after
 * another on the library's stream. Pointers may be managed, pinned-host-mapped or device memory;
 * seq_lens and block_table are read on the host (copied first when they are device memory) to
 * refuse a length below 0, above max_len or above max_blocks * page_size, and a live block id
 * outside [0, num_blocks), with KVB_ERR_INVALID before any device work. *gpu_ms receives the
 * device time of the steps (CUDA events), or 0 in pipelined mode. */
int kvb_run_paged(const kvb_paged_args* args, int steps, double* gpu_ms);

/* src/metal_attn.hpp:87 run_naive(): the three-pass baseline (scores, softmax, PV) on the
 * contiguous cache; fp32 and fp16 only. */
int kvb_run_naive(const kvb_naive_args* args, double* gpu_ms);

/* src/metal_attn.hpp:98-99 begin_pipelined() / end_pipelined(): between them, kvb_run_* and
 * kvb_flush_caches enqueue without waiting and run strictly in order; end waits and writes the
 * device milliseconds of every kvb_run_* call, in order, to ms[0 .. min(*count, cap)), setting
 * *count to the number of runs. */
int kvb_begin_pipelined(void);
int kvb_end_pipelined(double* ms, size_t cap, size_t* count);

/* Number of kvb_run_* calls queued since kvb_begin_pipelined (to size the array for
 * kvb_end_pipelined). */
int kvb_pipelined_runs(size_t* count);

/* src/metal_attn.hpp:102 run_read_bandwidth(): streams `bytes` of `src` once with 16-byte loads;
 * *gpu_ms receives the device time. */
int kvb_read_bandwidth(const void* src, size_t bytes, double* gpu_ms);

/* src/metal_attn.hpp:106 flush_gpu_caches(): overwrites a scratch buffer of max(256 MiB, 4 x L2)
 * so the next run starts with a cold L2. */
int kvb_flush_caches(void);

/* src/metal_attn.hpp:47-51 auto_part_tokens(): the reference's own split-K rule, kept for
 * callers that print it (largest power of two in [64, 512] giving >= 512 work groups). */
int kvb_auto_part_tokens(kvb_shape shape, int max_len);

/* Text of the calling thread's last error ("" if none). */
const char* kvb_last_error(void);

/* ---- stream level (no host reads, no allocation, no synchronization) ------------------------ */

/* The split-K partition size a call with these arguments uses (args->part_tokens, or the B200
 * rule when it is 0), or a negative status on a bad argument. Depends on shape, max_len, share_kv
 * and the current device's SM count only. */
int kvb_paged_part_tokens(const kvb_paged_args* args);

/* Device workspace a kvb_paged_decode_async call with these arguments needs. The workspace must
 * be zero-filled once before its first use (cudaMemset); every call leaves it ready for the next. */
int kvb_paged_workspace_bytes(const kvb_paged_args* args, size_t* bytes);

/* The split-K partition size for `args` given the sequence lengths on the host (host_lens[batch]),
 * to pass as args->part_tokens (same return convention as kvb_paged_part_tokens). It is the
 * automatic size, except on the tcgen05 kernel when that size gives more work units than CTAs but
 * fewer than five per CTA: then partitions shrink toward about five units per CTA (at least 1024
 * tokens), so that a ragged batch's last units end close together. No counterpart in the reference, whose partition follows
 * max_len alone (src/metal_attn.hpp:47-51). Reads nothing on the device. */
int kvb_paged_part_tokens_for(const kvb_paged_args* args, const int32_t* host_lens);

/* src/metal_attn.hpp:86 run_paged() as one stream-ordered launch: all pointers are device
 * pointers (q, seq_lens, block_table and out may also point at page-locked host memory, which the
 * kernels then read and write across the host link: the step's inputs need no staging copy), `stream`
 * is a cudaStream_t (NULL = legacy default stream). Nothing is read on the
 * host, so lengths cannot be refused up front: a length outside [0, min(max_len,
 * max_blocks * page_size)] or a live block id outside [0, num_blocks) makes the kernel write NaN
 * to that sequence's outputs and set a flag that kvb_paged_error_flag() reads; no access leaves
 * the buffers. Calls that share one workspace must not overlap on the device. */
int kvb_paged_decode_async(const kvb_paged_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* ---- page write path (the step before decode) --------------------------------------------- */

/* A contiguous cache written into the paged pool through the block table. Device pointers,
 * stream-ordered, nothing read on the host. */
typedef struct {
    kvb_shape shape;          /* batch, num_kv_heads, head_dim (a multiple of 8); num_heads unused */
    int kv_type;              /* pool type: KVB_F32 / KVB_F16 (scatter) or KVB_I8 (quantize) */
    int page_size, max_blocks, max_len;
    const void* contig;       /* [batch][num_kv_heads][max_len][head_dim]; fp32 for KVB_I8, else the pool type */
    const int* block_table;   /* [batch][max_blocks] */
    const int* seq_lens;      /* [batch] */
    void* pool;               /* [num_blocks][num_kv_heads][page_size][head_dim] */
    float* scales;            /* KVB_I8: [num_blocks][num_kv_heads] */
    long long num_blocks;
    unsigned int* error_word; /* optional device word: bit 1 bad length, bit 2 bad block id (pages skipped) */
} kvb_page_write_args;

/* src/reference.cpp:32-51 quantize_to_paged_i8 on the device: per (sequence, logical page, KV
 * head), scale = max|x| / 127 over the page's live tokens (fp32), q = clamp(nearbyint(x / scale),
 * -127, 127), 0 for a zero page; bit-identical to the reference for finite inputs. Slots past the
 * last token are not written. contig and pool 16-byte aligned. */
int kvb_quantize_paged_i8(const kvb_page_write_args* args, void* stream);

/* src/reference.hpp:60-68 scatter_to_paged on the device: the live tokens of an fp32 or fp16
 * contiguous cache copied into the pool of the same type. */
int kvb_scatter_paged(const kvb_page_write_args* args, void* stream);

/* Bytes of the library-owned workspace of kvb_paged_decode_static (16 MiB per device). */
#define KVB_STATIC_WORKSPACE_BYTES (16u << 20)

/* kvb_paged_decode_async without a caller workspace: the step's split-K partials, arrival counters
 * and error word live in a 16 MiB array of the library's own device memory, so the call allocates
 * nothing (no cudaMalloc, cudaFree or allocator of any library). No counterpart in the reference,
 * whose run_paged owns its buffers. For callers that cannot allocate device memory on their call
 * path: a plain C or FFI caller without a device allocator, or a latency-critical loop where an
 * allocation (which can synchronize the device) is not allowed.
 * Limits: a call whose workspace (kvb_paged_workspace_bytes: about batch x heads x partitions x
 * head_dim x 4 bytes) exceeds KVB_STATIC_WORKSPACE_BYTES is refused with KVB_ERR_INVALID and
 * launches nothing. Every call on a device uses the same array: calls that overlap on the device
 * (different streams without ordering, or several host threads) race on it, so serialize them.
 * The array starts zeroed at module load, which is what its error word and split-K counters need;
 * every completed call leaves the counters ready for the next. Bad lengths or block ids give NaN
 * outputs and set bits of the array's error word, as in kvb_paged_decode_async; read them with
 * kvb_paged_static_error_flag. A call that reported a TIMEOUT (4) or STATE (8) bit can leave the
 * counters stale, and the next call would then skip work: call kvb_paged_static_error_flag, which
 * also resets them, before decoding again.
 * The first call on each device looks up the array's address and sets kernel attributes: make it
 * outside any stream capture. Do not use the library across cudaDeviceReset. */
int kvb_paged_decode_static(const kvb_paged_args* args, void* stream);

/* kvb_paged_error_flag for the library-owned workspace of kvb_paged_decode_static on the current
 * device (synchronizes `stream`): reads and clears its error word, and after a TIMEOUT or STATE
 * bit resets its split-K and work counters. No counterpart in the reference. */
int kvb_paged_static_error_flag(void* stream, int* flag);

/* Reads and clears the error flag of a workspace (synchronizes `stream`). *flag = 0: no bad
 * length or block id since the last read. Bits: 1 bad length, 2 bad block id, 4 a bounded device
 * wait gave up, 8 a split-K arrival counter counted past its partition count (two launches sharing
 * the workspace at once, or an earlier launch that gave up); after 4 or 8 this call also resets
 * the counters, so the workspace can be used again. */
int kvb_paged_error_flag(void* workspace, void* stream, int* flag);

/* ---- sharded steps: the output gathered by the decode kernel itself ----------------------- */
/* No counterpart in the reference, which runs on one GPU. One process per GPU, ranks 0..n-1 on
 * GPUs with peer access (NVLink / NVSwitch). Each rank decodes its share of the step (some
 * sequences, or some KV heads of every sequence), and the kernel writes every finished output row
 * straight into every rank's global output buffer, in global order, over peer memory: there is no
 * separate all-gather and no reorder, and the transfers overlap the rest of the decode. A small
 * barrier kernel then tells each rank that every peer's rows have landed. */

#define KVB_MAX_PEERS 8

/* Device memory that other processes can map (CUDA IPC): cudaMalloc'd, zero-filled, with its
 * handle. Exchange the 64 handle bytes between ranks (any host channel), map peers' memory with
 * kvb_ipc_open. */
typedef struct { unsigned char bytes[64]; } kvb_ipc_handle;
int kvb_ipc_alloc(size_t bytes, void** ptr, kvb_ipc_handle* handle);
int kvb_ipc_free(void* ptr);
/* Maps another process's kvb_ipc_alloc memory on the current device (peer access enabled). */
int kvb_ipc_open(const kvb_ipc_handle* handle, void** ptr);
int kvb_ipc_close(void* ptr);

/* Where a sharded step's outputs go. Global output of every rank: [rows][out_heads][head_dim]
 * fp32. Local sequence b, local query head h (0 <= h < num_heads of this rank's args) is global row
 * out_rows[b] (or b when out_rows is NULL), global head out_head0 + h; each element is written to
 * peer_out[0..n_peers), peer_out[self] being this rank's own buffer. Rows outside [0, rows) are
 * refused on the device (error bit 2, nothing written). */
typedef struct kvb_peer_out {
    int n_peers;                        /* 1..KVB_MAX_PEERS */
    int self;                           /* index of this rank's own buffer in peer_out */
    int rows;                           /* global rows (sequences) of every peer buffer */
    int out_heads;                      /* query heads per global row */
    int out_head0;                      /* global head of this rank's head 0 */
    const int* out_rows;                /* device [batch] or NULL */
    float* peer_out[KVB_MAX_PEERS];     /* device pointers (this rank's own, or kvb_ipc_open'ed) */
} kvb_peer_out;

/* kvb_paged_decode_async with the outputs written through `peers` instead of args->out (which may
 * be NULL). Stream-ordered. The peers' buffers must not be read until kvb_peer_barrier_async has
 * passed on this step. */
int kvb_paged_decode_gather_async(const kvb_paged_args* args, const kvb_peer_out* peers, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* The step barrier after kvb_paged_decode_gather_async on every rank. signal[j] is rank j's signal
 * array (KVB_MAX_PEERS unsigned words, kvb_ipc memory: this rank's own and the others' mapped);
 * epoch is one word of this rank's device memory, zero at the start and never shared. One CTA: it
 * waits for the decode before it on `stream`, counts the epoch up, stores it into word `rank` of
 * every rank's signal array (system-scope release), then waits until every rank's word in its own
 * array reached it (acquire). A wait that runs past timeout_us (0: one second) gives up, sets bit 4
 * of the workspace's error word (kvb_paged_error_flag) and returns, so the context stays usable. */
typedef struct kvb_peer_barrier_args {
    int n_peers, rank;
    unsigned int timeout_us;
    unsigned int* epoch;
    unsigned int* signal[KVB_MAX_PEERS];
} kvb_peer_barrier_args;
int kvb_peer_barrier_async(const kvb_peer_barrier_args* args, void* workspace, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVB_CUDA_H */
