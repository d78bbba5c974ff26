// Host side of the C ABI declared in include/kvb_cuda.h: argument checks, managed buffers, the
// split-K workspace, tensor-map encoding, kernel choice, timing and pipelined mode.
//
// Mirrors the runtime of the reference's Metal host layer (src/metal_attn.mm): argument and length
// checks before any device work (:199-201, :107-117 check_lens), a grow-only workspace (:98-105),
// one queue (here one CUDA stream), device time per call (:119-130 finish), pipelined mode
// (:37-53, :278-293), the read-bandwidth probe (:249-264) and the cache flush (:266-276).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/kvb_cuda.h"
#include "kvb_internal.h"

namespace {

thread_local std::string t_err;

int fail(int code, const std::string& msg) {
    t_err = msg;
    return code;
}

#define KVB_CUDA(call)                                                                               \
    do {                                                                                             \
        const cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

size_t elem_size(int t) { return t == KVB_F32 ? 4 : t == KVB_F16 ? 2 : 1; }

// ---- per-device facts ------------------------------------------------------------------------

struct DeviceFacts {
    int num_sms = 0, l2_bytes = 0;
};

int device_facts(DeviceFacts* out) {
    static std::mutex mu;
    static std::vector<DeviceFacts> cache;
    int dev = 0;
    KVB_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1);
    DeviceFacts& f = cache[dev];
    if (!f.num_sms) {
        KVB_CUDA(cudaDeviceGetAttribute(&f.num_sms, cudaDevAttrMultiProcessorCount, dev));
        KVB_CUDA(cudaDeviceGetAttribute(&f.l2_bytes, cudaDevAttrL2CacheSize, dev));
    }
    *out = f;
    return KVB_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// ---- geometry of a paged call ------------------------------------------------------------------

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Geometry {
    int G, qg, gpk, nhg, part, max_parts;
    int kernel;  // KVB_KERNEL_SIMT / MMA / UMMA actually used
};

bool pool_rows_fit(const kvb_paged_args* a) {
    return (long long)a->num_blocks * a->shape.num_kv_heads * a->page_size < (1LL << 31);
}

// The kernel a call runs: the requested one, or for AUTO the first of UMMA, MMA, SIMT that supports
// the shape. Returns -1 when a specific tensor-core kernel was requested for a shape it cannot run.
int choose_kernel(const kvb_paged_args* a, int qg) {
    const int D = a->shape.head_dim;
    const bool tma_ok = a->max_len > 0 && pool_rows_fit(a) && aligned16(a->k) && aligned16(a->v);
    const bool umma = tma_ok && kvb_umma_supported(a->kv_type, D, a->page_size, qg, a->part_tokens);
    const bool mma = tma_ok && kvb_mma_supported(a->kv_type, D, a->page_size, qg);
    if (a->max_len == 0) return KVB_KERNEL_SIMT;  // nothing to read: the CUDA-core kernel writes the zeros
    switch (a->kernel) {
    case KVB_KERNEL_SIMT: return KVB_KERNEL_SIMT;
    case KVB_KERNEL_MMA: return mma ? KVB_KERNEL_MMA : -1;
    case KVB_KERNEL_UMMA: return umma ? KVB_KERNEL_UMMA : -1;
    default: return umma ? KVB_KERNEL_UMMA : mma ? KVB_KERNEL_MMA : KVB_KERNEL_SIMT;
    }
}

Geometry geometry(const kvb_paged_args* a, int num_sms) {
    Geometry g;
    const kvb_shape& s = a->shape;
    g.G = s.num_heads / s.num_kv_heads;
    g.qg = a->share_kv ? std::min(g.G, 8) : 1;
    g.gpk = (g.G + g.qg - 1) / g.qg;
    g.nhg = s.num_kv_heads * g.gpk;
    g.kernel = choose_kernel(a, g.qg);
    if (a->part_tokens > 0) {
        g.part = a->part_tokens;
    } else {
        // B200 rule: split each (sequence, head group) into as many partitions as keep all units in one
        // wave of the kernel's CTA slots (one CTA per SM for the tcgen05 kernel, two otherwise), and into
        // partitions of at most part_max tokens (bounded per-unit work balances ragged batches); rounded
        // up to whole chunks of the kernel. When the tcgen05 kernel would get more than 64 units per
        // SM even so, partitions grow to 8064 tokens (63 chunks): every unit boundary stalls one
        // softmax group for a few microseconds, and with that many units the balance does not suffer
        // (config 5: int8 0.71 -> 0.77, fp16 0.93 -> 0.95 of the copy bandwidth). The page table holds
        // such a partition only for pages of 32 tokens or more.
        const bool umma = g.kernel == KVB_KERNEL_UMMA;
        const long long chunk = umma ? 128 : KVB_CHUNK;
        long long part_max = umma && a->page_size >= 16 ? 4096 : 2048;  // tcgen05: its page table
        const long long S = std::max<long long>(1, (long long)s.batch * g.nhg);
        const long long slots = (umma ? 1LL : 2LL) * std::max(1, num_sms);
        // A step stream (KVB_FLAG_STEP_STREAM) on the tcgen05 kernel: about a third of the CTA slots
        // per step, so three steps stream at once (each CTA's fixed start and end overlap other
        // steps' streaming); partitions up to 8064 tokens where the page table holds them.
        const bool stream = umma && (a->flags & KVB_FLAG_STEP_STREAM) && 3 * S <= slots;
        if (umma && a->page_size >= 32 &&
            (stream || S * (((long long)a->max_len + part_max - 1) / part_max) > 64 * slots))
            part_max = 8064;
        long long n = S < slots ? std::max<long long>(1, slots / S) : 1;
        if (stream) n = std::max<long long>(1, (slots + 3 * S / 2) / (3 * S));  // slots / 3S, rounded
        n = std::max<long long>(n, ((long long)a->max_len + part_max - 1) / part_max);
        const long long per = ((long long)a->max_len + n - 1) / n;
        g.part = (int)std::max<long long>(chunk, (per + chunk - 1) / chunk * chunk);
    }
    g.max_parts = std::max(1, (int)(((long long)a->max_len + g.part - 1) / g.part));
    return g;
}

// Checks everything that can be checked without reading device data. Messages follow the
// reference's std::invalid_argument texts where it has one.
int check_static(const kvb_paged_args* a) {
    if (!a) return fail(KVB_ERR_INVALID, "null arguments");
    const kvb_shape& s = a->shape;
    if (a->part_tokens < 0 || a->max_len < 0 || a->page_size <= 0)
        return fail(KVB_ERR_INVALID, "part_tokens < 0, max_len < 0 or page_size <= 0");
    if (a->kv_type < KVB_F32 || a->kv_type > KVB_I8) return fail(KVB_ERR_INVALID, "unknown kv_type");
    if (a->kv_type == KVB_I8 && (!a->k_scale || !a->v_scale)) return fail(KVB_ERR_INVALID, "i8 cache without scales");
    if (s.batch < 0 || s.num_heads <= 0 || s.num_kv_heads <= 0) return fail(KVB_ERR_INVALID, "bad shape");
    if (s.head_dim != 64 && s.head_dim != 128) return fail(KVB_ERR_INVALID, "head_dim must be 64 or 128");
    if (s.num_heads % s.num_kv_heads != 0) return fail(KVB_ERR_INVALID, "H % Hkv != 0");
    if (a->max_blocks < 0) return fail(KVB_ERR_INVALID, "max_blocks < 0");
    if (a->kernel < KVB_KERNEL_AUTO || a->kernel > KVB_KERNEL_UMMA) return fail(KVB_ERR_INVALID, "unknown kernel");
    if (a->flags & ~(KVB_FLAG_TABLES_READY | KVB_FLAG_INPUTS_READY | KVB_FLAG_STEP_STREAM))
        return fail(KVB_ERR_INVALID, "unknown flags");
    if ((a->flags & KVB_FLAG_INPUTS_READY) && !(a->flags & KVB_FLAG_TABLES_READY))
        return fail(KVB_ERR_INVALID, "KVB_FLAG_INPUTS_READY needs KVB_FLAG_TABLES_READY");
    if ((a->flags & KVB_FLAG_STEP_STREAM) && !(a->flags & KVB_FLAG_INPUTS_READY))
        return fail(KVB_ERR_INVALID, "KVB_FLAG_STEP_STREAM needs KVB_FLAG_INPUTS_READY");
    if (s.batch > 0 && (!a->q || !a->out || !a->seq_lens)) return fail(KVB_ERR_INVALID, "null q, out or seq_lens");
    if (s.batch > 0 && a->max_len > 0) {
        if (!a->k || !a->v || !a->block_table) return fail(KVB_ERR_INVALID, "null k, v or block_table");
        if (a->num_blocks <= 0) return fail(KVB_ERR_INVALID, "num_blocks must be > 0 for a non-empty cache");
    }
    if ((s.batch > 0) && (!aligned16(a->q) || !aligned16(a->out)))
        return fail(KVB_ERR_INVALID, "q and out must be 16-byte aligned");
    if ((long long)s.batch * s.num_heads * s.head_dim > (1LL << 31))
        return fail(KVB_ERR_INVALID, "q/out larger than 2^31 elements");
    if (s.num_heads > 65536) return fail(KVB_ERR_INVALID, "more than 65536 query heads");
    return KVB_OK;
}

// Encodes the tile map of one pool: rows of D elements, num_blocks * Hkv * page rows, boxes of
// (128 bytes) x min(page, 64) rows, 128-byte swizzle.
// Launch ids for the split-K arrival counters: distinct per launch within the process, high bit set
// (never 0 or KVB_CTR_CLEAN, and as a float the bits of a negative denormal that no stored partial
// result holds).
unsigned next_launch_id() {
    static std::atomic<unsigned> n{0};
    return 0x80000000u | (n.fetch_add(1, std::memory_order_relaxed) & 0x7fffffffu);
}

int encode_pool_map(CUtensorMap* map, const void* pool, const kvb_paged_args* a, int box_rows_max) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return fail(KVB_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
    const size_t es = elem_size(a->kv_type);
    const cuuint64_t rows = (cuuint64_t)a->num_blocks * a->shape.num_kv_heads * a->page_size;
    const cuuint64_t dims[2] = {(cuuint64_t)a->shape.head_dim, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)a->shape.head_dim * es};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)std::min(a->page_size, box_rows_max)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, a->kv_type == KVB_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                           2, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ERR_DEVICE, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return KVB_OK;
}

// One decode step on `stream` with workspace `ws` (zeroed once, sized by kvb_paged_workspace_bytes);
// with `peers`, the outputs go to every rank's global buffer instead of a->out.
int launch_paged(const kvb_paged_args* a, void* ws, cudaStream_t stream, const kvb_peer_out* peers = nullptr) {
    DeviceFacts f;
    if (int rc = device_facts(&f)) return rc;
    const Geometry g = geometry(a, f.num_sms);
    const kvb_shape& s = a->shape;
    if (s.batch == 0) return KVB_OK;
    const WorkspaceLayout w = kvb_workspace_layout(s.batch, s.num_heads, g.nhg, g.max_parts, s.head_dim);
    char* wsb = static_cast<char*>(ws);

    DecodeParams p;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.block_table = a->block_table;
    p.seq_lens = a->seq_lens;
    p.k_scale = a->k_scale;
    p.v_scale = a->v_scale;
    p.out = a->out;
    p.part_o = reinterpret_cast<float*>(wsb + w.o_off);
    p.part_ml = reinterpret_cast<float2*>(wsb + w.ml_off);
    p.counters = reinterpret_cast<unsigned long long*>(wsb + w.counters_off);
    p.error_flag = reinterpret_cast<unsigned*>(wsb + w.flag_off);
    p.B = s.batch;
    p.H = s.num_heads;
    p.Hkv = s.num_kv_heads;
    p.G = g.G;
    p.qg = g.qg;
    p.gpk = g.gpk;
    p.nhg = g.nhg;
    p.page = a->page_size;
    p.max_blocks = a->max_blocks;
    p.max_len = a->max_len;
    p.part_tokens = g.part;
    p.max_parts = g.max_parts;
    // work units are numbered below 2^31 and divided by these launch constants on the device
    if ((long long)s.batch * g.nhg * g.max_parts >= (1LL << 31))
        return fail(KVB_ERR_INVALID, "more than 2^31 split-K work units (batch x head groups x partitions)");
    p.div_part = kvb_div_make((uint32_t)g.part);
    p.div_gpk = kvb_div_make((uint32_t)g.gpk);
    p.div_parts = kvb_div_make((uint32_t)g.max_parts);
    p.div_seq = kvb_div_make((uint32_t)(g.nhg * g.max_parts));
    p.num_blocks = a->num_blocks;
    p.q_scale = 1.4426950408889634f / std::sqrt(float(s.head_dim));
    p.launch = next_launch_id();
    p.tables_ready = (a->flags & KVB_FLAG_TABLES_READY) != 0;
    p.inputs_ready = (a->flags & KVB_FLAG_INPUTS_READY) != 0;
    p.n_peers = peers ? peers->n_peers : 0;
    p.peer_self = peers ? peers->self : 0;
    p.peer_rows = peers ? peers->rows : 0;
    p.out_heads = peers ? peers->out_heads : s.num_heads;
    p.out_head0 = peers ? peers->out_head0 : 0;
    p.out_rows = peers ? peers->out_rows : nullptr;
    for (int j = 0; j < KVB_MAX_PEERS; ++j) p.peer_out[j] = peers && j < peers->n_peers ? peers->peer_out[j] : nullptr;

    if (g.kernel < 0)
        return fail(KVB_ERR_INVALID, "the requested tensor-core kernel does not support this shape, page size or dtype");
    LaunchInfo li{f.num_sms, stream};
    cudaError_t e;
    if (g.kernel == KVB_KERNEL_UMMA || g.kernel == KVB_KERNEL_MMA) {
        const int box_rows = g.kernel == KVB_KERNEL_UMMA ? 128 : KVB_CHUNK;
        CUtensorMap tk, tv;
        if (int rc = encode_pool_map(&tk, a->k, a, box_rows)) return rc;
        if (int rc = encode_pool_map(&tv, a->v, a, box_rows)) return rc;
        e = g.kernel == KVB_KERNEL_UMMA ? kvb_launch_decode_umma(p, a->kv_type, s.head_dim, &tk, &tv, li)
                                         : kvb_launch_decode_mma(p, a->kv_type, s.head_dim, &tk, &tv, li);
    } else {
        e = kvb_launch_decode_simt(p, a->kv_type, s.head_dim, li);
    }
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("decode launch: ") + cudaGetErrorString(e));
    return KVB_OK;
}

// ---- reference-facing state ----------------------------------------------------------------------

struct State {
    std::mutex mu;
    bool ready = false;
    int dev = 0;
    cudaStream_t stream = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* scores = nullptr;
    size_t scores_bytes = 0;
    void* flush = nullptr;
    size_t flush_bytes = 0;
    float* sink = nullptr;
    uint32_t flush_value = 0;
    bool pipelined = false;
    bool pipeline_checks = false;  // a run in the current pipeline needs its error flag checked
    bool after_naive = false;      // the last kernel on the stream was the naive baseline (it writes an output)
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> timed;
};

// One state per device: the reference's API is single-device, and a caller that switches devices
// (cudaSetDevice) gets that device's own stream, workspace and pipeline.
constexpr int kMaxStateDevices = 64;

State& st() {
    static State s[kMaxStateDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = 0;
    }
    return s[dev >= 0 && dev < kMaxStateDevices ? dev : 0];
}

int ensure_ready(State& S) {
    if (S.ready) return KVB_OK;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(KVB_ERR_NO_DEVICE, "no CUDA device");
    }
    KVB_CUDA(cudaGetDevice(&S.dev));
    KVB_CUDA(cudaStreamCreateWithFlags(&S.stream, cudaStreamNonBlocking));
    KVB_CUDA(cudaMalloc(&S.sink, 256 * sizeof(float)));
    S.ready = true;
    return KVB_OK;
}

// Grows a device scratch buffer (contents not kept); zero-filled when `zero`.
int grow(State& S, void** buf, size_t* have, size_t need, bool zero) {
    need = std::max<size_t>(need, 256);
    if (*buf && *have >= need) return KVB_OK;
    if (*buf) {
        KVB_CUDA(cudaStreamSynchronize(S.stream));
        KVB_CUDA(cudaFree(*buf));
        *buf = nullptr;
        *have = 0;
    }
    KVB_CUDA(cudaMalloc(buf, need));
    *have = need;
    if (zero) KVB_CUDA(cudaMemsetAsync(*buf, 0, need, S.stream));
    return KVB_OK;
}

enum class Mem { host_only, host_and_device, device_only };

Mem classify(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return Mem::host_only;
    }
    switch (at.type) {
    case cudaMemoryTypeManaged: return Mem::host_and_device;
    case cudaMemoryTypeHost: return at.devicePointer ? Mem::host_and_device : Mem::host_only;
    case cudaMemoryTypeDevice: return Mem::device_only;
    default: return Mem::host_only;
    }
}

// Reads n ints of a buffer the host may or may not be able to address.
int read_ints(const int32_t* p, size_t n, std::vector<int32_t>* out) {
    out->resize(n);
    if (!n) return KVB_OK;
    if (classify(p) == Mem::device_only) {
        KVB_CUDA(cudaMemcpy(out->data(), p, n * sizeof(int32_t), cudaMemcpyDeviceToHost));
    } else {
        std::memcpy(out->data(), p, n * sizeof(int32_t));
    }
    return KVB_OK;
}

int require_device_accessible(const void* p, const char* what) {
    if (p && classify(p) == Mem::host_only)
        return fail(KVB_ERR_INVALID, std::string(what) + " is not device-accessible (use kvb_buffer_alloc)");
    return KVB_OK;
}

int prefetch(State& S, const void* p, size_t bytes) {
    if (!p || !bytes) return KVB_OK;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess || at.type != cudaMemoryTypeManaged) {
        cudaGetLastError();
        return KVB_OK;
    }
    KVB_CUDA(cudaMemPrefetchAsync(p, bytes, S.dev, S.stream));
    return KVB_OK;
}

int begin_timed(State& S, cudaEvent_t* e0, cudaEvent_t* e1) {
    KVB_CUDA(cudaEventCreate(e0));
    KVB_CUDA(cudaEventCreate(e1));
    KVB_CUDA(cudaEventRecord(*e0, S.stream));
    return KVB_OK;
}

// Reads and clears the error word of a workspace; after a TIMEOUT or STATE error also zeroes the
// arrival counters the last launch used (their count is workspace word 1), so the workspace is
// ready for the next call.
int read_clear_flag(void* ws, cudaStream_t s, unsigned* flag) {
    unsigned h[2] = {0, 0};
    KVB_CUDA(cudaMemcpyAsync(h, ws, sizeof h, cudaMemcpyDeviceToHost, s));
    KVB_CUDA(cudaStreamSynchronize(s));
    *flag = h[0];
    if (!h[0]) return KVB_OK;
    KVB_CUDA(cudaMemsetAsync(ws, 0, sizeof h[0], s));
    if (h[0] & (KVB_DEVERR_TIMEOUT | KVB_DEVERR_STATE)) {
        // a launch that gave up may have left the split-K counters and the work counters (words 2, 3)
        KVB_CUDA(cudaMemsetAsync(static_cast<char*>(ws) + 256, 0, sizeof(unsigned long long) * (size_t)h[1], s));
        KVB_CUDA(cudaMemsetAsync(static_cast<char*>(ws) + 8, 0, 2 * sizeof(unsigned), s));
    }
    KVB_CUDA(cudaStreamSynchronize(s));
    return KVB_OK;
}

int check_flag(State& S) {
    if (!S.ws) return KVB_OK;
    unsigned flag = 0;
    if (int rc = read_clear_flag(S.ws, S.stream, &flag)) return rc;
    if (!flag) return KVB_OK;
    return fail(KVB_ERR_DEVICE, "decode kernel reported error flags " + std::to_string(flag));
}

// Non-pipelined: waits and returns the device time. Pipelined: queues the pair and returns 0.
int end_timed(State& S, cudaEvent_t e0, cudaEvent_t e1, double* ms, bool check) {
    KVB_CUDA(cudaEventRecord(e1, S.stream));
    if (S.pipelined) {
        S.timed.emplace_back(e0, e1);
        S.pipeline_checks |= check;
        if (ms) *ms = 0;
        return KVB_OK;
    }
    const cudaError_t sync = cudaEventSynchronize(e1);
    float t = 0;
    if (sync == cudaSuccess) cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (sync != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("device failure: ") + cudaGetErrorString(sync));
    if (check)
        if (int rc = check_flag(S)) return rc;
    if (ms) *ms = t;
    return KVB_OK;
}

}  // namespace

// ==================================================================================================
extern "C" {

int kvb_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n > 0 ? 1 : 0;
}

int kvb_device_name(char* buf, size_t len) {
    if (!buf || !len) return fail(KVB_ERR_INVALID, "null buffer");
    buf[0] = 0;
    if (!kvb_available()) return fail(KVB_ERR_NO_DEVICE, "no CUDA device");
    int dev = 0;
    KVB_CUDA(cudaGetDevice(&dev));
    cudaDeviceProp prop;
    KVB_CUDA(cudaGetDeviceProperties(&prop, dev));
    std::strncpy(buf, prop.name, len - 1);
    buf[len - 1] = 0;
    return KVB_OK;
}

int kvb_buffer_alloc(size_t bytes, void** ptr) {
    if (!ptr) return fail(KVB_ERR_INVALID, "null ptr");
    *ptr = nullptr;
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    const cudaError_t e = cudaMallocManaged(ptr, std::max<size_t>(bytes, 16), cudaMemAttachGlobal);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        return fail(KVB_ERR_DEVICE, "managed allocation failed (" + std::to_string(bytes) + " bytes): " +
                                        cudaGetErrorString(e));
    }
    return KVB_OK;
}

int kvb_buffer_free(void* ptr) {
    if (!ptr) return KVB_OK;
    KVB_CUDA(cudaFree(ptr));
    return KVB_OK;
}

int kvb_auto_part_tokens(kvb_shape s, int max_len) {
    int part = 512;
    while (part > 64 && (long long)s.batch * s.num_kv_heads * ((max_len + part - 1) / part) < 512) part /= 2;
    return part;
}

int kvb_paged_part_tokens(const kvb_paged_args* a) {
    if (int rc = check_static(a)) return -rc;
    DeviceFacts f;
    if (int rc = device_facts(&f)) return -rc;
    return geometry(a, f.num_sms).part;
}

int kvb_paged_part_tokens_for(const kvb_paged_args* a, const int32_t* host_lens) {
    if (int rc = check_static(a)) return -rc;
    if (!host_lens && a->shape.batch > 0) return -fail(KVB_ERR_INVALID, "null host_lens");
    DeviceFacts f;
    if (int rc = device_facts(&f)) return -rc;
    const Geometry g = geometry(a, f.num_sms);
    if (a->part_tokens > 0 || g.kernel != KVB_KERNEL_UMMA) return g.part;
    // Units of the automatic partition; a launch with no more units than CTAs keeps it.
    const long long chunk = 128, slots = std::max(1, f.num_sms);
    long long units = 0, tokens = 0;
    for (int b = 0; b < a->shape.batch; ++b) {
        const long long len = std::min<long long>(std::max(0, host_lens[b]), a->max_len);
        units += (long long)g.nhg * std::max<long long>(1, (len + g.part - 1) / g.part);
        tokens += len * g.nhg;
    }
    // One wave keeps it, and so do five or more units per CTA.
    if (units <= slots || units >= 5 * slots) return g.part;
    // A few units per CTA, handed out dynamically: partitions small enough for about five units per
    // CTA, so that the last ones handed out end close together (a CTA with one 30-chunk unit too
    // many ends 20-40 us late), and not below 1024 tokens, since every unit costs its CTA about
    // 2 us of start and merge work. Config 4's first 8 sequences on one B200: 88.9 us per step with
    // the automatic 3712 tokens, 72.5 us with 1024; its first 16: 139.6 us with 3840, 140.3 with 2048.
    const long long want = (tokens + 5 * slots - 1) / (5 * slots);
    const long long part = std::max<long long>(1024, (want + chunk - 1) / chunk * chunk);
    return (int)std::min<long long>(part, g.part);
}

int kvb_paged_workspace_bytes(const kvb_paged_args* a, size_t* bytes) {
    if (!bytes) return fail(KVB_ERR_INVALID, "null bytes");
    if (int rc = check_static(a)) return rc;
    DeviceFacts f;
    if (int rc = device_facts(&f)) return rc;
    const Geometry g = geometry(a, f.num_sms);
    *bytes = kvb_workspace_layout(a->shape.batch, a->shape.num_heads, g.nhg, g.max_parts, a->shape.head_dim).total;
    return KVB_OK;
}

int kvb_paged_decode_async(const kvb_paged_args* a, void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = check_static(a)) return rc;
    size_t need = 0;
    if (int rc = kvb_paged_workspace_bytes(a, &need)) return rc;
    if (!workspace || workspace_bytes < need)
        return fail(KVB_ERR_INVALID, "workspace too small: need " + std::to_string(need) + " bytes");
    return launch_paged(a, workspace, static_cast<cudaStream_t>(stream));
}

int kvb_paged_decode_gather_async(const kvb_paged_args* a, const kvb_peer_out* peers, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (!a || !peers) return fail(KVB_ERR_INVALID, "null arguments");
    if (peers->n_peers < 1 || peers->n_peers > KVB_MAX_PEERS)
        return fail(KVB_ERR_INVALID, "n_peers must be in [1, KVB_MAX_PEERS]");
    if (peers->rows < 1 || peers->out_head0 < 0 || peers->out_heads < peers->out_head0 + a->shape.num_heads)
        return fail(KVB_ERR_INVALID, "peer rows must be > 0 and out_head0 + num_heads <= out_heads");
    if ((long long)peers->rows * peers->out_heads * a->shape.head_dim > (1LL << 40))
        return fail(KVB_ERR_INVALID, "peer output too large");
    if (peers->self < 0 || peers->self >= peers->n_peers) return fail(KVB_ERR_INVALID, "self must be in [0, n_peers)");
    for (int j = 0; j < peers->n_peers; ++j)
        if (!peers->peer_out[j] || !aligned16(peers->peer_out[j]))
            return fail(KVB_ERR_INVALID, "every peer output must be non-null and 16-byte aligned");
    kvb_paged_args local = *a;  // the local output is not written; the checks want one
    if (!local.out) local.out = peers->peer_out[0];
    if (int rc = check_static(&local)) return rc;
    size_t need = 0;
    if (int rc = kvb_paged_workspace_bytes(&local, &need)) return rc;
    if (!workspace || workspace_bytes < need)
        return fail(KVB_ERR_INVALID, "workspace too small: need " + std::to_string(need) + " bytes");
    return launch_paged(&local, workspace, static_cast<cudaStream_t>(stream), peers);
}

int kvb_peer_barrier_async(const kvb_peer_barrier_args* a, void* workspace, void* stream) {
    if (!a || !workspace) return fail(KVB_ERR_INVALID, "null arguments");
    if (a->n_peers < 1 || a->n_peers > KVB_MAX_PEERS || a->rank < 0 || a->rank >= a->n_peers)
        return fail(KVB_ERR_INVALID, "n_peers must be in [1, KVB_MAX_PEERS] and 0 <= rank < n_peers");
    if (!a->epoch) return fail(KVB_ERR_INVALID, "null epoch");
    for (int j = 0; j < a->n_peers; ++j)
        if (!a->signal[j]) return fail(KVB_ERR_INVALID, "null signal array");
    PeerBarrierParams p;
    p.n_peers = a->n_peers;
    p.rank = a->rank;
    p.timeout_ns = 1000ull * (a->timeout_us ? a->timeout_us : 1000000u);
    p.epoch = a->epoch;
    for (int j = 0; j < KVB_MAX_PEERS; ++j) p.signal[j] = j < a->n_peers ? a->signal[j] : nullptr;
    const WorkspaceLayout w = kvb_workspace_layout(0, 0, 0, 0, 0);
    p.error_flag = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + w.flag_off);
    const cudaError_t e = kvb_launch_peer_barrier(p, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("peer barrier launch: ") + cudaGetErrorString(e));
    return KVB_OK;
}

int kvb_ipc_alloc(size_t bytes, void** ptr, kvb_ipc_handle* handle) {
    if (!ptr || !handle || bytes == 0) return fail(KVB_ERR_INVALID, "null pointer or zero size");
    *ptr = nullptr;
    void* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) return fail(KVB_ERR_DEVICE, "cudaMalloc failed");
    cudaIpcMemHandle_t h;
    // zeroed before the handle leaves: a peer may store into the memory as soon as it has mapped it,
    // and a memset still in flight would wipe that store
    if (cudaMemset(d, 0, bytes) != cudaSuccess || cudaStreamSynchronize(0) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, d) != cudaSuccess) {
        cudaFree(d);
        return fail(KVB_ERR_DEVICE, "cudaIpcGetMemHandle failed");
    }
    static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
    std::memcpy(handle->bytes, &h, sizeof(h));
    *ptr = d;
    return KVB_OK;
}

int kvb_ipc_free(void* ptr) {
    if (ptr && cudaFree(ptr) != cudaSuccess) return fail(KVB_ERR_DEVICE, "cudaFree failed");
    return KVB_OK;
}

int kvb_ipc_open(const kvb_ipc_handle* handle, void** ptr) {
    if (!handle || !ptr) return fail(KVB_ERR_INVALID, "null arguments");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    return KVB_OK;
}

int kvb_ipc_close(void* ptr) {
    if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return fail(KVB_ERR_DEVICE, "cudaIpcCloseMemHandle failed");
    return KVB_OK;
}

// ---- page write path -------------------------------------------------------------------------------

int page_write(const kvb_page_write_args* a, bool quantize, void* stream) {
    if (!a) return fail(KVB_ERR_INVALID, "null arguments");
    const kvb_shape& s = a->shape;
    if (quantize ? a->kv_type != KVB_I8 : (a->kv_type != KVB_F32 && a->kv_type != KVB_F16))
        return fail(KVB_ERR_INVALID, quantize ? "quantize writes an int8 pool" : "scatter takes f32 or f16");
    if (s.batch < 0 || s.batch > 65535) return fail(KVB_ERR_INVALID, "batch must be in [0, 65535]");
    if (s.num_kv_heads < 1 || s.num_kv_heads > 65535) return fail(KVB_ERR_INVALID, "num_kv_heads must be in [1, 65535]");
    if (s.head_dim < 8 || s.head_dim % 8) return fail(KVB_ERR_INVALID, "head_dim must be a positive multiple of 8");
    if (a->page_size <= 0) return fail(KVB_ERR_INVALID, "page_size must be > 0");
    if (a->max_blocks < 0 || a->max_len < 0) return fail(KVB_ERR_INVALID, "max_blocks and max_len must be >= 0");
    if (a->num_blocks <= 0) return fail(KVB_ERR_INVALID, "num_blocks must be > 0");
    if (s.batch == 0 || a->max_blocks == 0) return KVB_OK;
    if (!a->contig || !a->block_table || !a->seq_lens || !a->pool || (quantize && !a->scales))
        return fail(KVB_ERR_INVALID, "null device pointer");
    if (!aligned16(a->contig) || !aligned16(a->pool)) return fail(KVB_ERR_INVALID, "contig and pool must be 16-byte aligned");
    PageWriteParams p;
    p.src = a->contig;
    p.dst = a->pool;
    p.scales = a->scales;
    p.block_table = a->block_table;
    p.seq_lens = a->seq_lens;
    p.error_flag = a->error_word;
    p.B = s.batch;
    p.Hkv = s.num_kv_heads;
    p.D = s.head_dim;
    p.page = a->page_size;
    p.max_blocks = a->max_blocks;
    p.max_len = a->max_len;
    p.elem = (int)elem_size(a->kv_type);
    p.src_elem = quantize ? (int)sizeof(float) : p.elem;
    p.num_blocks = a->num_blocks;
    DeviceFacts f;
    if (int rc = device_facts(&f)) return rc;
    p.num_sms = f.num_sms;
    const cudaError_t e = kvb_launch_page_write(p, quantize, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("page write launch: ") + cudaGetErrorString(e));
    return KVB_OK;
}

int kvb_quantize_paged_i8(const kvb_page_write_args* args, void* stream) { return page_write(args, true, stream); }

int kvb_scatter_paged(const kvb_page_write_args* args, void* stream) { return page_write(args, false, stream); }

// ---- library-owned workspace ---------------------------------------------------------------------

// The workspace of kvb_paged_decode_static: device memory of the library's own module (zero at module
// load), so the call path allocates nothing. One per device; calls on a device share it.
static __device__ __align__(256) unsigned char g_static_workspace[KVB_STATIC_WORKSPACE_BYTES];

// Device address of g_static_workspace on the current device, looked up once per device (with that
// device current) and cached. The host-side name g_static_workspace is a stand-in, never a device
// address: only the looked-up pointer is passed to kernels.
int static_workspace(void** out) {
    static KvbPerDevice<void*> addr;
    const cudaError_t e = addr.get(out, [](void** p) {
        const cudaError_t r = cudaGetSymbolAddress(p, g_static_workspace);
        return r == cudaSuccess && !*p ? cudaErrorInvalidSymbol : r;
    });
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("static workspace address: ") + cudaGetErrorString(e));
    return KVB_OK;
}

int kvb_paged_decode_static(const kvb_paged_args* a, void* stream) {
    if (int rc = check_static(a)) return rc;
    size_t need = 0;
    if (int rc = kvb_paged_workspace_bytes(a, &need)) return rc;
    if (need > KVB_STATIC_WORKSPACE_BYTES)
        return fail(KVB_ERR_INVALID, "this call needs a " + std::to_string(need) +
                                         "-byte workspace (batch x heads x partitions x head_dim floats and more); "
                                         "the static workspace holds " +
                                         std::to_string((size_t)KVB_STATIC_WORKSPACE_BYTES) +
                                         " bytes: use kvb_paged_decode_async with a workspace of that size");
    void* ws = nullptr;
    if (int rc = static_workspace(&ws)) return rc;
    return launch_paged(a, ws, static_cast<cudaStream_t>(stream));
}

int kvb_paged_static_error_flag(void* stream, int* flag) {
    if (!flag) return fail(KVB_ERR_INVALID, "null flag");
    void* ws = nullptr;
    if (int rc = static_workspace(&ws)) return rc;
    unsigned h = 0;
    if (int rc = read_clear_flag(ws, static_cast<cudaStream_t>(stream), &h)) return rc;
    *flag = (int)h;
    return KVB_OK;
}

int kvb_paged_error_flag(void* workspace, void* stream, int* flag) {
    if (!workspace || !flag) return fail(KVB_ERR_INVALID, "null workspace or flag");
    unsigned h = 0;
    if (int rc = read_clear_flag(workspace, static_cast<cudaStream_t>(stream), &h)) return rc;
    *flag = (int)h;
    return KVB_OK;
}

int kvb_run_paged(const kvb_paged_args* a, int steps, double* gpu_ms) {
    if (gpu_ms) *gpu_ms = 0;
    if (int rc = check_static(a)) return rc;
    if (steps < 0) return fail(KVB_ERR_INVALID, "steps < 0");
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    const kvb_shape& s = a->shape;
    const int B = s.batch;

    // Lengths and live block ids are checked on the host before anything is launched
    // (src/metal_attn.mm:107-117; the block ids are a check the reference does not make).
    std::vector<int32_t> lens, table;
    if (int rc = read_ints(a->seq_lens, (size_t)B, &lens)) return rc;
    const long long capacity = (long long)a->max_blocks * a->page_size;
    for (int b = 0; b < B; ++b) {
        const int len = lens[b];
        if (len < 0 || len > a->max_len || (long long)len > capacity)
            return fail(KVB_ERR_INVALID, "sequence " + std::to_string(b) + " has length " + std::to_string(len) +
                                             ", max_len " + std::to_string(a->max_len) + ", capacity " +
                                             std::to_string(capacity));
    }
    if (a->max_len > 0) {
        if (int rc = read_ints(a->block_table, (size_t)B * a->max_blocks, &table)) return rc;
        for (int b = 0; b < B; ++b) {
            const int live = (lens[b] + a->page_size - 1) / a->page_size;
            for (int i = 0; i < live; ++i) {
                const int32_t blk = table[(size_t)b * a->max_blocks + i];
                if (blk < 0 || blk >= a->num_blocks)
                    return fail(KVB_ERR_INVALID, "sequence " + std::to_string(b) + " block " + std::to_string(i) +
                                                     " has id " + std::to_string(blk) + ", pool of " +
                                                     std::to_string(a->num_blocks) + " blocks");
            }
        }
    }
    for (auto [p, what] : {std::pair<const void*, const char*>{a->q, "q"}, {a->out, "out"}, {a->k, "k"},
                           {a->v, "v"}, {a->block_table, "block_table"}, {a->seq_lens, "seq_lens"},
                           {a->k_scale, "k_scale"}, {a->v_scale, "v_scale"}})
        if (int rc = require_device_accessible(p, what)) return rc;

    size_t need = 0;
    if (int rc = kvb_paged_workspace_bytes(a, &need)) return rc;
    if (int rc = grow(S, &S.ws, &S.ws_bytes, need, true)) return rc;

    // Managed buffers are moved to the device before the timed region (the reference's GPU time
    // excludes encoding too).
    const size_t nq = (size_t)B * s.num_heads * s.head_dim * sizeof(float);
    const size_t pool = (size_t)a->num_blocks * s.num_kv_heads * a->page_size * s.head_dim * elem_size(a->kv_type);
    const size_t scales = (size_t)a->num_blocks * s.num_kv_heads * sizeof(float);
    const int live = a->max_len > 0;
    if (int rc = prefetch(S, a->q, nq)) return rc;
    if (int rc = prefetch(S, a->out, nq)) return rc;
    if (int rc = prefetch(S, a->seq_lens, (size_t)B * sizeof(int32_t))) return rc;
    if (live) {
        if (int rc = prefetch(S, a->block_table, (size_t)B * a->max_blocks * sizeof(int32_t))) return rc;
        if (int rc = prefetch(S, a->k, pool)) return rc;
        if (int rc = prefetch(S, a->v, pool)) return rc;
        if (a->kv_type == KVB_I8) {
            if (int rc = prefetch(S, a->k_scale, scales)) return rc;
            if (int rc = prefetch(S, a->v_scale, scales)) return rc;
        }
    }
    cudaEvent_t e0, e1;
    if (int rc = begin_timed(S, &e0, &e1)) return rc;
    // Kernels on the library's stream write no lengths, block tables, q, pools or scales (uploads
    // are host copies; decode steps, flushes and the bandwidth probe write only their own outputs),
    // so every step may read its inputs while the previous kernel finishes. After the naive baseline,
    // whose output buffer a caller could pass as q, the first step reads q after it.
    kvb_paged_args ready = *a;
    ready.flags |= KVB_FLAG_TABLES_READY | KVB_FLAG_INPUTS_READY;
    for (int i = 0; i < steps; ++i) {
        kvb_paged_args step = ready;
        if (i == 0 && S.after_naive) step.flags &= ~KVB_FLAG_INPUTS_READY;
        if (int rc = launch_paged(&step, S.ws, S.stream)) {
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            return rc;
        }
    }
    if (steps > 0) S.after_naive = false;
    return end_timed(S, e0, e1, gpu_ms, true);
}

int kvb_run_naive(const kvb_naive_args* a, double* gpu_ms) {
    if (gpu_ms) *gpu_ms = 0;
    if (!a) return fail(KVB_ERR_INVALID, "null arguments");
    const kvb_shape& s = a->shape;
    if (a->kv_type == KVB_I8) return fail(KVB_ERR_INVALID, "naive kernels take f32 or f16 caches");
    if (a->kv_type != KVB_F32 && a->kv_type != KVB_F16) return fail(KVB_ERR_INVALID, "unknown kv_type");
    if (a->max_len < 0) return fail(KVB_ERR_INVALID, "max_len < 0");
    if (s.batch < 0 || s.num_heads <= 0 || s.num_kv_heads <= 0) return fail(KVB_ERR_INVALID, "bad shape");
    if (s.head_dim != 64 && s.head_dim != 128) return fail(KVB_ERR_INVALID, "head_dim must be 64 or 128");
    if (s.num_heads % s.num_kv_heads != 0) return fail(KVB_ERR_INVALID, "H % Hkv != 0");
    if (s.batch > 0 && (!a->q || !a->out || !a->seq_lens || (a->max_len > 0 && (!a->k || !a->v))))
        return fail(KVB_ERR_INVALID, "null pointer argument");
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    std::vector<int32_t> lens;
    if (int rc = read_ints(a->seq_lens, (size_t)s.batch, &lens)) return rc;
    for (int b = 0; b < s.batch; ++b)
        if (lens[b] < 0 || lens[b] > a->max_len)
            return fail(KVB_ERR_INVALID, "sequence " + std::to_string(b) + " has length " + std::to_string(lens[b]) +
                                             ", max_len " + std::to_string(a->max_len) + ", capacity " +
                                             std::to_string(a->max_len));
    for (auto [p, what] : {std::pair<const void*, const char*>{a->q, "q"}, {a->out, "out"}, {a->k, "k"},
                           {a->v, "v"}, {a->seq_lens, "seq_lens"}})
        if (int rc = require_device_accessible(p, what)) return rc;
    const size_t nscores = (size_t)s.batch * s.num_heads * std::max(a->max_len, 1) * sizeof(float);
    if (int rc = grow(S, &S.scores, &S.scores_bytes, nscores, false)) return rc;
    const size_t nq = (size_t)s.batch * s.num_heads * s.head_dim * sizeof(float);
    const size_t nkv = (size_t)s.batch * s.num_kv_heads * a->max_len * s.head_dim * elem_size(a->kv_type);
    for (auto [p, n] : {std::pair<const void*, size_t>{a->q, nq}, {a->out, nq}, {a->k, nkv}, {a->v, nkv},
                        {a->seq_lens, (size_t)s.batch * sizeof(int32_t)}})
        if (int rc = prefetch(S, p, n)) return rc;
    cudaEvent_t e0, e1;
    if (int rc = begin_timed(S, &e0, &e1)) return rc;
    S.after_naive = true;
    const cudaError_t e = kvb_launch_naive(a->q, a->k, a->v, a->seq_lens, a->out, static_cast<float*>(S.scores),
                                           s.batch, s.num_heads, s.num_kv_heads, s.head_dim, a->max_len, a->kv_type,
                                           S.stream);
    if (e != cudaSuccess) {
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        return fail(KVB_ERR_DEVICE, std::string("naive launch: ") + cudaGetErrorString(e));
    }
    return end_timed(S, e0, e1, gpu_ms, false);
}

int kvb_begin_pipelined(void) {
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    for (auto& pr : S.timed) {
        cudaEventDestroy(pr.first);
        cudaEventDestroy(pr.second);
    }
    S.timed.clear();
    S.pipelined = true;
    S.pipeline_checks = false;
    return KVB_OK;
}

int kvb_pipelined_runs(size_t* count) {
    if (!count) return fail(KVB_ERR_INVALID, "null count");
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (!S.pipelined) return fail(KVB_ERR_STATE, "not in pipelined mode");
    *count = S.timed.size();
    return KVB_OK;
}

int kvb_end_pipelined(double* ms, size_t cap, size_t* count) {
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (!S.pipelined) return fail(KVB_ERR_STATE, "end_pipelined without begin_pipelined");
    S.pipelined = false;
    if (count) *count = S.timed.size();
    int rc = KVB_OK;
    for (size_t i = 0; i < S.timed.size(); ++i) {
        const cudaError_t sync = cudaEventSynchronize(S.timed[i].second);
        float t = 0;
        if (sync == cudaSuccess) cudaEventElapsedTime(&t, S.timed[i].first, S.timed[i].second);
        else if (rc == KVB_OK) rc = fail(KVB_ERR_DEVICE, std::string("device failure: ") + cudaGetErrorString(sync));
        if (ms && i < cap) ms[i] = t;
        cudaEventDestroy(S.timed[i].first);
        cudaEventDestroy(S.timed[i].second);
    }
    S.timed.clear();
    if (rc == KVB_OK && S.pipeline_checks) rc = check_flag(S);
    S.pipeline_checks = false;
    return rc;
}

int kvb_read_bandwidth(const void* src, size_t bytes, double* gpu_ms) {
    if (gpu_ms) *gpu_ms = 0;
    if (!src && bytes) return fail(KVB_ERR_INVALID, "null src");
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    if (int rc = require_device_accessible(src, "src")) return rc;
    if (int rc = prefetch(S, src, bytes)) return rc;
    DeviceFacts f;
    if (int rc = device_facts(&f)) return rc;
    cudaEvent_t e0, e1;
    if (int rc = begin_timed(S, &e0, &e1)) return rc;
    const cudaError_t e = kvb_launch_read_bw(src, bytes, S.sink, f.num_sms, S.stream);
    if (e != cudaSuccess) {
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        return fail(KVB_ERR_DEVICE, std::string("read_bw launch: ") + cudaGetErrorString(e));
    }
    return end_timed(S, e0, e1, gpu_ms, false);
}

int kvb_flush_caches(void) {
    State& S = st();
    std::lock_guard<std::mutex> lock(S.mu);
    if (int rc = ensure_ready(S)) return rc;
    DeviceFacts f;
    if (int rc = device_facts(&f)) return rc;
    const size_t want = std::max<size_t>(256u << 20, 4 * (size_t)f.l2_bytes);
    if (int rc = grow(S, &S.flush, &S.flush_bytes, want, false)) return rc;
    const cudaError_t e = kvb_launch_fill(S.flush, S.flush_bytes, ++S.flush_value, f.num_sms, S.stream);
    if (e != cudaSuccess) return fail(KVB_ERR_DEVICE, std::string("flush launch: ") + cudaGetErrorString(e));
    if (!S.pipelined) KVB_CUDA(cudaStreamSynchronize(S.stream));
    return KVB_OK;
}

const char* kvb_last_error(void) { return t_err.c_str(); }

}  // extern "C"
