// Drop-in replacement for kv-cache-bench's src/metal_attn.mm on NVIDIA B200: defines every function
// declared in the reference's unchanged C++ header src/metal_attn.hpp on top of this project's C
// ABI (include/kvb_cuda.h, libkvbcuda.so). Compile it against that header (-I <reference>/src) and
// link libkvbcuda; workload.hpp, reference.cpp, bench/bench.cpp and the three test programs then run
// unchanged on the GPU.
//
// Error behaviour follows the reference: a bad argument or length throws std::invalid_argument
// before any device work (src/metal_attn.mm:199-201, :107-117), a device failure throws
// std::runtime_error (:128), an allocation failure throws std::runtime_error (:144).
#include <stdexcept>
#include <string>
#include <vector>

#include "kvb_cuda.h"
#include "metal_attn.hpp"

namespace kvb {
namespace {

[[noreturn]] void raise(int rc, const char* what) {
    const std::string msg = std::string(what) + ": " + kvb_last_error();
    if (rc == KVB_ERR_INVALID) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

int kv_code(KvType t) { return t == KvType::f32 ? KVB_F32 : t == KvType::f16 ? KVB_F16 : KVB_I8; }

const void* dev(const Buffer* b) { return b ? b->handle() : nullptr; }

kvb_shape to_c(const Shape& s) { return kvb_shape{s.batch, s.num_heads, s.num_kv_heads, s.head_dim}; }

}  // namespace

bool metal_available() { return kvb_available() == 1; }

std::string device_name() {
    char buf[256];
    return kvb_device_name(buf, sizeof buf) == KVB_OK ? std::string(buf) : std::string();
}

// Managed memory: the host writes through data() and the kernels read the same pointer.
Buffer::Buffer(size_t bytes) : bytes_(bytes) {
    void* p = nullptr;
    if (kvb_buffer_alloc(bytes, &p) != KVB_OK)
        throw std::runtime_error("CUDA managed allocation failed (" + std::to_string(bytes) + " bytes): " +
                                 kvb_last_error());
    impl_ = p;
    data_ = p;
}

Buffer::~Buffer() { kvb_buffer_free(impl_); }

double run_paged(const PagedArgs& a) { return run_paged_steps(a, 1); }

double run_paged_steps(const PagedArgs& a, int steps) {
    kvb_paged_args c{};
    c.shape = to_c(a.shape);
    c.kv_type = kv_code(a.type);
    c.page_size = a.page_size;
    c.max_blocks = a.max_blocks;
    c.max_len = a.max_len;
    c.part_tokens = a.part_tokens;
    c.q = static_cast<const float*>(dev(a.q));
    c.k = dev(a.k);
    c.v = dev(a.v);
    c.block_table = static_cast<const int32_t*>(dev(a.block_table));
    c.seq_lens = static_cast<const int32_t*>(dev(a.seq_lens));
    c.out = static_cast<float*>(const_cast<void*>(dev(a.out)));
    c.share_kv = a.share_kv ? 1 : 0;
    c.k_scale = static_cast<const float*>(dev(a.k_scale));
    c.v_scale = static_cast<const float*>(dev(a.v_scale));
    // The pool size the reference never passes: the K buffer holds num_blocks * Hkv * page * D elements.
    const size_t per_block = size_t(a.page_size > 0 ? a.page_size : 0) * size_t(a.shape.num_kv_heads > 0 ? a.shape.num_kv_heads : 0) *
                             size_t(a.shape.head_dim > 0 ? a.shape.head_dim : 0) * elem_size(a.type);
    c.num_blocks = (a.k && per_block) ? int64_t(a.k->size() / per_block) : 0;
    c.kernel = KVB_KERNEL_AUTO;
    double ms = 0;
    if (const int rc = kvb_run_paged(&c, steps, &ms)) raise(rc, "run_paged");
    return ms;
}

double run_naive(const NaiveArgs& a) {
    kvb_naive_args c{};
    c.shape = to_c(a.shape);
    c.kv_type = kv_code(a.type);
    c.max_len = a.max_len;
    c.q = static_cast<const float*>(dev(a.q));
    c.k = dev(a.k);
    c.v = dev(a.v);
    c.seq_lens = static_cast<const int32_t*>(dev(a.seq_lens));
    c.out = static_cast<float*>(const_cast<void*>(dev(a.out)));
    double ms = 0;
    if (const int rc = kvb_run_naive(&c, &ms)) raise(rc, "run_naive");
    return ms;
}

void begin_pipelined() {
    if (const int rc = kvb_begin_pipelined()) raise(rc, "begin_pipelined");
}

std::vector<double> end_pipelined() {
    size_t n = 0;
    if (const int rc = kvb_pipelined_runs(&n)) raise(rc, "end_pipelined");
    std::vector<double> ms(n);
    if (const int rc = kvb_end_pipelined(ms.data(), ms.size(), &n)) raise(rc, "end_pipelined");
    ms.resize(n);
    return ms;
}

double run_read_bandwidth(const Buffer& src) {
    double ms = 0;
    if (const int rc = kvb_read_bandwidth(src.handle(), src.size(), &ms)) raise(rc, "run_read_bandwidth");
    return ms;
}

void flush_gpu_caches() {
    if (const int rc = kvb_flush_caches()) raise(rc, "flush_gpu_caches");
}

}  // namespace kvb
