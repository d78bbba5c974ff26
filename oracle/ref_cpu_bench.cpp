// Times the reference's own CPU implementation of one decode step (the CPU baseline of bench.py):
// the reference's Workload generator (src/workload.hpp:26-94), PagedCache int8 quantizer
// (src/workload.hpp:96-151) and fp64 oracle attention_reference (src/reference.cpp:65-100), threaded
// over (sequence, head) rows with all hardware threads, as the reference's bench does
// (bench/bench.cpp:231-242). For int8 the timed path is PagedCache::reference: dequantize, then the
// fp64 attention (src/workload.hpp:130-137).
//
// Test infrastructure, built into oracle/_ref/kvb_ref_cpu by oracle/Makefile from the reference
// sources where they lie. Buffer gets a host-only definition (no GPU is involved).
//
// Usage: kvb_ref_cpu --heads=32 --kv-heads=8 --dim=128 --type=i8 --lens=32768[,...] --page=128
//                    [--seed=1] [--q-amp=1] [--steps=3] [--threads=N]
// Prints one JSON line: {"ms_per_step": .., "ms_min": .., "threads": .., "tokens": .., "min_bytes": ..}.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "workload.hpp"

namespace kvb {
Buffer::Buffer(size_t bytes) : bytes_(bytes) {
    data_ = std::calloc(std::max<size_t>(bytes, 16), 1);
    if (!data_) throw std::runtime_error("host allocation failed");
    impl_ = data_;
}
Buffer::~Buffer() { std::free(data_); }
}  // namespace kvb

using namespace kvb;

int main(int argc, char** argv) {
    Shape shape{1, 32, 8, 128};
    KvType type = KvType::f16;
    std::vector<int> lens{4096};
    int page = 16, steps = 3, threads = int(std::max(1u, std::thread::hardware_concurrency()));
    uint64_t seed = 1;
    float q_amp = 1.0f;
    for (int i = 1; i < argc; ++i) {
        const char* a = argv[i];
        auto val = [&](const char* key) -> const char* {
            const size_t n = std::strlen(key);
            return std::strncmp(a, key, n) == 0 && a[n] == '=' ? a + n + 1 : nullptr;
        };
        if (auto v = val("--heads")) shape.num_heads = std::atoi(v);
        else if (auto v = val("--kv-heads")) shape.num_kv_heads = std::atoi(v);
        else if (auto v = val("--dim")) shape.head_dim = std::atoi(v);
        else if (auto v = val("--page")) page = std::atoi(v);
        else if (auto v = val("--steps")) steps = std::atoi(v);
        else if (auto v = val("--threads")) threads = std::atoi(v);
        else if (auto v = val("--seed")) seed = std::strtoull(v, nullptr, 10);
        else if (auto v = val("--q-amp")) q_amp = std::strtof(v, nullptr);
        else if (auto v = val("--type")) type = !std::strcmp(v, "f32") ? KvType::f32 : !std::strcmp(v, "i8") ? KvType::i8 : KvType::f16;
        else if (auto v = val("--lens")) {
            lens.clear();
            for (const char* p = v; *p;) {
                lens.push_back(std::atoi(p));
                p = std::strchr(p, ',');
                if (!p) break;
                ++p;
            }
        } else {
            std::fprintf(stderr, "unknown argument %s\n", a);
            return 2;
        }
    }
    const Workload w(shape, type, lens, seed, q_amp);
    std::unique_ptr<PagedCache> cache;
    if (type == KvType::i8) cache = std::make_unique<PagedCache>(w, page, seed * 1000 + page);
    std::vector<float> out(w.out_floats());
    auto step = [&] {
        if (cache) cache->reference(w, out.data(), threads);
        else w.reference(out.data(), threads);
    };
    step();  // warm-up
    double total = 0, best = 1e300;
    for (int i = 0; i < steps; ++i) {
        const auto t0 = std::chrono::steady_clock::now();
        step();
        const std::chrono::duration<double, std::milli> dt = std::chrono::steady_clock::now() - t0;
        total += dt.count();
        best = std::min(best, dt.count());
    }
    long long tokens = 0;
    for (int l : lens) tokens += l;
    std::printf("{\"ms_per_step\": %.6f, \"ms_min\": %.6f, \"threads\": %d, \"tokens\": %lld, \"min_bytes\": %.0f, "
                "\"steps\": %d, \"checksum\": %.9g}\n",
                total / std::max(steps, 1), best, threads, tokens, w.min_bytes(), steps, double(out[0]));
    return 0;
}
