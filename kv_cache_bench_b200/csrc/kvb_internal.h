// Types and constants shared by the host launchers (kvb_capi.cu) and the kernels. Not part of the
// public ABI (that is include/kvb_cuda.h).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include <cuda_runtime.h>

#include "kvb_cuda.h"

// A value set up once per device: kernel attributes (cudaFuncSetAttribute), occupancy and symbol
// addresses belong to a device's context, so a process that launches on several devices needs each
// of them once per device. get() runs `init(T*)` the first time it is called with a device current
// and returns the cached value afterwards; safe to call from several host threads (the fast path is
// one atomic load). Values do not survive cudaDeviceReset: the library must not be used across one.
template <typename T>
class KvbPerDevice {
public:
    template <typename F>
    cudaError_t get(T* out, F&& init) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        if (!ready_[dev].load(std::memory_order_acquire)) {
            std::lock_guard<std::mutex> lock(mu_);
            if (!ready_[dev].load(std::memory_order_relaxed)) {
                T v{};
                e = init(&v);
                if (e != cudaSuccess) return e;
                value_[dev] = v;
                ready_[dev].store(true, std::memory_order_release);
            }
        }
        *out = value_[dev];
        return cudaSuccess;
    }

private:
    static constexpr int kMaxDevices = 64;
    std::mutex mu_;
    std::atomic<bool> ready_[kMaxDevices] = {};
    T value_[kMaxDevices] = {};
};

// Bounded device waits give up after this much wall time (the kernel then reports
// KVB_DEVERR_TIMEOUT and returns instead of hanging the GPU).
#define KVB_WAIT_LIMIT_NS 2000000000ull

// Bits of the workspace error word.
#define KVB_DEVERR_LENGTH 1u    // a sequence length outside [0, min(max_len, max_blocks * page)]
#define KVB_DEVERR_BLOCK 2u     // a live block id outside [0, num_blocks)
#define KVB_DEVERR_TIMEOUT 4u   // a bounded wait gave up
#define KVB_DEVERR_STATE 8u     // a split-K arrival counter counted past its partition count
// Epoch of an arrival counter that a completed launch left behind (a NaN payload that neither a
// launch id nor a stored partial result takes).
#define KVB_CTR_CLEAN 0x7fffffffu
// Word 1 of the workspace holds the number of arrival counters the last launch used, so that the
// flag reader can zero them after a TIMEOUT or STATE error. Words 2 and 3 count the units the
// tcgen05 kernel handed out dynamically and the CTAs that found none left; a launch leaves both 0
// (the flag reader zeroes them after a TIMEOUT or STATE error too). Words 0-3 are the header.

// Sequences up to this batch size are enumerated through a prefix sum in shared memory.
#define KVB_PREFIX_MAX 256
// Heads merged per epilogue round (bounds the epilogue's shared memory).
#define KVB_EPI_HEADS 4
// Tokens per TMA stage of the tensor-core kernel.
#define KVB_CHUNK 64

// Division by an invariant divisor d in [1, 2^31) of numerators in [0, 2^31) with a multiply-high,
// an add and a shift (T. Granlund, P. Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> l; the sum stays below 2^32 because umulhi(n, m) < n < 2^31. The
// kernels divide unit indices by launch constants this way (kvb_div in kvb_device.cuh).
struct KvbDiv {
    uint32_t d, m, l;
};

inline KvbDiv kvb_div_make(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
    return KvbDiv{d, uint32_t(m), l};
}

// Everything a decode launch needs. Pointers are device pointers.
struct DecodeParams {
    const float* q;          // [B][H][D]
    const void* k;           // pools [num_blocks][Hkv][page][D]
    const void* v;
    const int* block_table;  // [B][max_blocks]
    const int* seq_lens;     // [B]
    const float* k_scale;    // [num_blocks][Hkv] (int8)
    const float* v_scale;
    float* out;              // [B][H][D]
    // workspace
    float* part_o;           // [B][H][max_parts][D], partition outputs (normalized)
    float2* part_ml;         // [B][H][max_parts], (max in log2 units, sum)
    unsigned long long* counters;  // [B][nhg]: (epoch << 32) | partitions finished
    unsigned* error_flag;    // KVB_DEVERR_* bits
    // shape
    int B, H, Hkv, G;
    int qg;    // query heads per head group (<= 8)
    int gpk;   // head groups per KV head
    int nhg;   // head groups per sequence = Hkv * gpk
    int page, max_blocks, max_len, part_tokens, max_parts;
    long long num_blocks;
    float q_scale;     // log2(e) / sqrt(D): scores come out in log2 units
    unsigned launch;   // launch id (high bit set): tells this launch's counter values from stale ones
    int tables_ready;  // KVB_FLAG_TABLES_READY: lengths and block table may be read before the PDL wait
    int inputs_ready;  // KVB_FLAG_INPUTS_READY (with tables_ready): q, pools and scales may be read before it too
    // the launch's invariant divisors: part_tokens, gpk, max_parts, nhg * max_parts
    KvbDiv div_part, div_gpk, div_parts, div_seq;
    // A sharded step gathered in the kernel (n_peers > 0): output element (b, h, d) goes to
    // peer_out[0..n_peers) at ((out_rows ? out_rows[b] : b) * out_heads + out_head0 + h) * D + d,
    // peer_out[peer_self] being this rank's own buffer, and out is not written. n_peers == 0:
    // out[b][h][d].
    int n_peers, peer_self, peer_rows, out_heads, out_head0;
    const int* out_rows;
    float* peer_out[KVB_MAX_PEERS];
};

// The step barrier of a sharded step gathered in the kernel (kvb_peer.cu).
struct PeerBarrierParams {
    int n_peers, rank;
    unsigned long long timeout_ns;
    unsigned* epoch;
    unsigned* signal[KVB_MAX_PEERS];
    unsigned* error_flag;
};
cudaError_t kvb_launch_peer_barrier(const PeerBarrierParams& p, cudaStream_t stream);

// The page write path (kvb_pages.cu): a contiguous cache into the paged pool.
struct PageWriteParams {
    const void* src;         // [B][Hkv][max_len][D]: fp32 (quantize) or the pool's type (scatter)
    void* dst;               // pool [num_blocks][Hkv][page][D]
    float* scales;           // quantize: [num_blocks][Hkv]
    const int* block_table;  // [B][max_blocks]
    const int* seq_lens;     // [B]
    unsigned* error_flag;    // optional: KVB_DEVERR_LENGTH / KVB_DEVERR_BLOCK bits
    int B, Hkv, D, page, max_blocks, max_len;
    int elem;      // bytes per pool element
    int src_elem;  // bytes per source element (4: fp32 for the quantizer)
    int num_sms;   // sizes the persistent grid
    long long num_blocks;
};
cudaError_t kvb_launch_page_write(const PageWriteParams& p, bool quantize, cudaStream_t stream);

// Workspace layout (offsets in bytes), shared by the size query and the launcher.
struct WorkspaceLayout {
    size_t flag_off, counters_off, ml_off, o_off, total;
};

constexpr inline size_t kvb_align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline WorkspaceLayout kvb_workspace_layout(int B, int H, int nhg, int max_parts, int D) {
    WorkspaceLayout w;
    w.flag_off = 0;
    w.counters_off = 256;
    w.ml_off = kvb_align_up(w.counters_off + sizeof(unsigned long long) * (size_t)B * nhg, 256);
    w.o_off = kvb_align_up(w.ml_off + sizeof(float) * 2 * (size_t)B * H * max_parts, 256);
    w.total = kvb_align_up(w.o_off + sizeof(float) * (size_t)B * H * max_parts * D, 256);
    return w;
}

// Kernel launchers (one per kernel family), implemented next to the kernels.
struct LaunchInfo {
    int num_sms;
    cudaStream_t stream;
};

// Launches `kernel` with programmatic stream serialization (the kernels call pdl_wait() before
// touching global memory, so they may start while the previous kernel in the stream finishes).
template <typename... KArgs, typename... Args>
cudaError_t kvb_launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                           Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// CUDA-core kernel: every storage type, page size, head dim and group size.
cudaError_t kvb_launch_decode_simt(const DecodeParams& p, int kv_type, int D, const LaunchInfo& li);

// mma.sync + TMA kernel: fp16/int8 with 128- or 256-byte rows, page a power of two in [8, 256],
// qg <= 8. `tmap_k`/`tmap_v` are CUtensorMap objects over the pools.
bool kvb_mma_supported(int kv_type, int D, int page, int qg);
cudaError_t kvb_launch_decode_mma(const DecodeParams& p, int kv_type, int D, const void* tmap_k,
                                  const void* tmap_v, const LaunchInfo& li);

// tcgen05 kernel: fp16/int8, head dim 128, page 8/16/32/64/128/256, qg <= 8, partitions of at most
// about 262 pages and 8064 tokens (part_tokens 0: automatic); tensor maps with boxes of (128 bytes) x
// min(page, 128) rows.
bool kvb_umma_supported(int kv_type, int D, int page, int qg, int part_tokens);
cudaError_t kvb_launch_decode_umma(const DecodeParams& p, int kv_type, int D, const void* tmap_k,
                                   const void* tmap_v, const LaunchInfo& li);

// Naive three-pass baseline on the contiguous cache.
cudaError_t kvb_launch_naive(const float* q, const void* k, const void* v, const int* seq_lens, float* out,
                             float* scores, int B, int H, int Hkv, int D, int max_len, int kv_type,
                             cudaStream_t stream);

// Streaming read probe and L2 flush.
cudaError_t kvb_launch_read_bw(const void* src, size_t bytes, float* sink, int num_sms, cudaStream_t stream);
cudaError_t kvb_launch_fill(void* dst, size_t bytes, uint32_t value, int num_sms, cudaStream_t stream);
