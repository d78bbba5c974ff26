// Writes golden input/output vectors for the paged decode path with the reference's own code:
// its Workload / PagedCache generators (src/workload.hpp), its block-table allocator and int8
// quantizer (src/reference.cpp:11-51) and its fp64 oracle (src/reference.cpp:65-100).
//
// Test infrastructure: built by oracle/Makefile (target `golden`) into oracle/_ref/make_golden,
// run by tests/golden/make_golden.sh, which commits golden.bin + golden.json beside this file.
// The cases mirror the reference's tests: tests/gpu_tests.cpp:74-157 (shapes, ragged lengths
// {L, L/3+1, L+5}, seeds, pages), tests/boundary_tests.cpp:80-209 (page/partition boundaries,
// empty sequences, contiguous layout) and tests/cpu_tests.cpp:40-63 (known answers).
//
// Buffer is given a host-only definition here (zeroed host memory): the generator runs on a
// machine without a GPU and only needs host-visible storage.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
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

namespace {

struct Writer {
    std::FILE* bin;
    std::string json = "{\"cases\": [\n";
    size_t offset = 0;
    bool first_case = true, first_field = true;

    void begin(const std::string& name) {
        json += first_case ? "" : ",\n";
        json += "{\"name\": \"" + name + "\"";
        first_case = false;
    }
    void field(const std::string& key, long long v) { json += ", \"" + key + "\": " + std::to_string(v); }
    void field_f(const std::string& key, double v) {
        char buf[64];
        std::snprintf(buf, sizeof buf, "%.17g", v);
        json += ", \"" + key + "\": " + buf;
    }
    void array(const std::string& key, const char* dtype, const void* p, size_t bytes) {
        while (offset % 64) {  // keep every array 64-byte aligned in the file
            std::fputc(0, bin);
            ++offset;
        }
        if (bytes && std::fwrite(p, 1, bytes, bin) != bytes) throw std::runtime_error("write failed");
        json += ", \"" + key + "\": {\"dtype\": \"" + dtype + "\", \"offset\": " + std::to_string(offset) +
                ", \"bytes\": " + std::to_string(bytes) + "}";
        offset += bytes;
    }
    void end() { json += "}"; }
};

const char* kv_dtype(KvType t) { return t == KvType::f32 ? "f32" : t == KvType::f16 ? "f16" : "i8"; }

// One paged case: the inputs the kernel reads and the reference outputs.
void paged_case(Writer& w, const std::string& name, const Workload& wl, int page, uint64_t layout_seed, int part,
                bool contiguous, bool with_fp32_data) {
    const PagedCache cache(wl, page, layout_seed, contiguous);
    const size_t n = wl.out_floats();
    std::vector<float> ref(n), ref_data;
    cache.reference(wl, ref.data(), 4);  // on the values the kernel computes with
    if (wl.type != KvType::f32) {        // on the unrounded fp32 data (f16: k32/v32, i8: the workload's own)
        ref_data.resize(n);
        if (wl.type == KvType::i8)
            wl.reference(ref_data.data(), 4);
    }
    w.begin(name);
    w.field("batch", wl.shape.batch);
    w.field("num_heads", wl.shape.num_heads);
    w.field("num_kv_heads", wl.shape.num_kv_heads);
    w.field("head_dim", wl.shape.head_dim);
    w.field("kv_type", int(wl.type));
    w.field("page_size", cache.layout.page_size);
    w.field("max_blocks", cache.layout.max_blocks);
    w.field("num_blocks", cache.layout.num_blocks);
    w.field("max_len", wl.max_len);
    w.field("part_tokens", part);
    w.field("auto_part_tokens", auto_part_tokens(wl.shape, wl.max_len));
    w.array("q", "f32", wl.q->data(), wl.q->size());
    w.array("seq_lens", "i32", wl.seq_lens->data(), wl.lens.size() * sizeof(int));
    w.array("block_table", "i32", cache.layout.block_table.data(), cache.layout.block_table.size() * sizeof(int32_t));
    w.array("k", kv_dtype(wl.type), cache.k->data(), cache.k->size());
    w.array("v", kv_dtype(wl.type), cache.v->data(), cache.v->size());
    if (wl.type == KvType::i8) {
        w.array("k_scale", "f32", cache.k_scale->data(), cache.k_scale->size());
        w.array("v_scale", "f32", cache.v_scale->data(), cache.v_scale->size());
    }
    w.array("ref", "f32", ref.data(), n * sizeof(float));
    if (with_fp32_data && wl.type == KvType::f16) {
        const float scale = 1.0f / std::sqrt(float(wl.shape.head_dim));
        attention_reference<float>(wl.shape, wl.lens, wl.max_len, wl.q->as<float>(), wl.k32.data(), wl.v32.data(),
                                   ref_data.data(), scale, 4);
        w.array("k32", "f32", wl.k32.data(), wl.k32.size() * sizeof(float));
        w.array("v32", "f32", wl.v32.data(), wl.v32.size() * sizeof(float));
        w.array("ref_fp32_data", "f32", ref_data.data(), n * sizeof(float));
    }
    if (wl.type == KvType::i8) {
        w.array("ref_fp32_data", "f32", ref_data.data(), n * sizeof(float));
        if (with_fp32_data) {
            w.array("k_contig_f32", "f32", wl.k->data(), wl.k->size());
            w.array("v_contig_f32", "f32", wl.v->data(), wl.v->size());
        }
    }
    w.end();
}

// Contiguous-cache case for the naive kernels: the Workload's own [B][Hkv][max_len][D] cache.
void naive_case(Writer& w, const std::string& name, const Workload& wl) {
    const size_t n = wl.out_floats();
    std::vector<float> ref(n);
    wl.reference(ref.data(), 4);
    w.begin(name);
    w.field("batch", wl.shape.batch);
    w.field("num_heads", wl.shape.num_heads);
    w.field("num_kv_heads", wl.shape.num_kv_heads);
    w.field("head_dim", wl.shape.head_dim);
    w.field("kv_type", int(wl.type));
    w.field("max_len", wl.max_len);
    w.array("q", "f32", wl.q->data(), wl.q->size());
    w.array("seq_lens", "i32", wl.seq_lens->data(), wl.lens.size() * sizeof(int));
    w.array("k", kv_dtype(wl.type), wl.k->data(), wl.k->size());
    w.array("v", kv_dtype(wl.type), wl.v->data(), wl.v->size());
    w.array("ref", "f32", ref.data(), n * sizeof(float));
    w.end();
}

// Known answers of tests/cpu_tests.cpp:40-63 on the reference, as paged cases (page = max_len,
// one block per sequence, identity table): q = 0 gives the mean of V; one dominant key selects
// its V row exactly.
void known_answer_cases(Writer& w) {
    const Shape s{2, 4, 2, 64};
    const std::vector<int> lens{37, 5};
    const int max_len = 37, D = s.head_dim;
    const float scale = 1.0f / std::sqrt(float(D));
    const size_t nkv = size_t(s.batch) * s.num_kv_heads * max_len * D, nq = size_t(s.batch) * s.num_heads * D;
    std::mt19937_64 rng(2);
    std::uniform_real_distribution<float> u(-1.0f, 1.0f);
    std::vector<float> k(nkv), v(nkv);
    for (auto& e : k) e = u(rng);
    for (auto& e : v) e = u(rng);
    const std::vector<int32_t> table{0, 1};
    for (int which = 0; which < 2; ++which) {
        std::vector<float> q(nq, 0.0f), kk = k, out(nq);
        if (which == 1) {
            std::fill(kk.begin(), kk.end(), 0.0f);
            for (size_t i = 0; i < nq; i += D) q[i] = 1000.0f;
            const int hot[] = {11, 4};
            for (int b = 0; b < s.batch; ++b)
                for (int kvh = 0; kvh < s.num_kv_heads; ++kvh) kk[contig_index(s, max_len, b, kvh, hot[b], 0)] = 1.0f;
        }
        attention_reference<float>(s, lens, max_len, q.data(), kk.data(), v.data(), out.data(), scale);
        w.begin(which == 0 ? "known_zero_query_mean_of_v" : "known_dominant_key");
        w.field("batch", s.batch);
        w.field("num_heads", s.num_heads);
        w.field("num_kv_heads", s.num_kv_heads);
        w.field("head_dim", s.head_dim);
        w.field("kv_type", 0);
        w.field("page_size", max_len);
        w.field("max_blocks", 1);
        w.field("num_blocks", 2);
        w.field("max_len", max_len);
        w.field("part_tokens", 0);
        w.field("auto_part_tokens", auto_part_tokens(s, max_len));
        w.array("q", "f32", q.data(), nq * sizeof(float));
        w.array("seq_lens", "i32", lens.data(), lens.size() * sizeof(int));
        w.array("block_table", "i32", table.data(), table.size() * sizeof(int32_t));
        w.array("k", "f32", kk.data(), nkv * sizeof(float));  // contiguous == paged with page = max_len
        w.array("v", "f32", v.data(), nkv * sizeof(float));
        w.array("ref", "f32", out.data(), nq * sizeof(float));
        w.field("exact", 1);
        w.end();
    }
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s OUT.bin OUT.json\n", argv[0]);
        return 2;
    }
    Writer w{std::fopen(argv[1], "wb")};
    if (!w.bin) {
        std::perror(argv[1]);
        return 1;
    }
    const KvType types[] = {KvType::f32, KvType::f16, KvType::i8};

    // tests/gpu_tests.cpp:74-157: two shapes, ragged {L, L/3+1, L+5}, seeds with their partition
    // size and q amplitude, fp16 keeps the fp32 data, int8 gets varied magnitudes.
    struct SeedCfg { uint64_t seed; int part; float q_amp; };
    const SeedCfg seeds[] = {{1, 64, 1.0f}, {2, 256, 8.0f}, {3, 512, 3.0f}};
    const Shape shapes[] = {{1, 8, 2, 128}, {1, 4, 4, 64}};
    struct GridCase { int L; int seed_idx; int page; };
    const GridCase grid[] = {{1, 0, 16}, {7, 1, 16}, {40, 2, 32}, {100, 1, 64}};
    // L = 100 only for int8 (the pools of the other types would make the fixture large).
    for (const Shape& shape : shapes)
        for (const GridCase& g : grid)
            for (KvType t : types) {
                if (g.L == 100 && t != KvType::i8) continue;
                if (g.L == 40 && (shape.group() == 1 || t == KvType::f32)) continue;  // L = 40: GQA, f16/i8
                const SeedCfg& sc = seeds[g.seed_idx];
                const bool i8 = t == KvType::i8;
                const Workload wl(shape, t, {g.L, g.L / 3 + 1, g.L + 5}, sc.seed, sc.q_amp, t == KvType::f16, i8);
                const std::string case_name = std::string("grid_H") + std::to_string(shape.num_heads) + "_Hkv" +
                                         std::to_string(shape.num_kv_heads) + "_D" + std::to_string(shape.head_dim) +
                                         "_L" + std::to_string(g.L) + "_" + kvb::name(t) + "_p" + std::to_string(g.page);
                paged_case(w, case_name, wl, g.page, sc.seed * 1000 + g.page, sc.part, false, g.L <= 7);
                if (!i8 && g.L <= 7) naive_case(w, "naive_" + case_name, wl);
            }

    // tests/boundary_tests.cpp:116-130: odd page sizes and partitions of fewer tokens than warps.
    for (const Shape& shape : shapes)
        for (KvType t : types)
            for (int page : {1, 3})
                for (int L : {2, 3, 5}) {  // the tests run each case at several partition sizes
                    const Workload wl(shape, t, {L, L + 1}, 1, 3.0f, false, t == KvType::i8);
                    paged_case(w,
                               "boundary_D" + std::to_string(shape.head_dim) + "_" + kvb::name(t) + "_p" +
                                   std::to_string(page) + "_L" + std::to_string(L),
                               wl, page, uint64_t(page) * 1000 + 1, 1, false, false);
                }
    // tests/boundary_tests.cpp:190-208: empty sequences first, last, alone, whole batch.
    const std::vector<std::vector<int>> batches = {{0, 1}, {1, 0}, {0, 16}, {17, 0}, {0, 65, 0}, {0}, {0, 0}};
    int bi = 0;
    for (const std::vector<int>& lens : batches) {
        for (KvType t : types) {
            const Workload wl(shapes[bi % 2], t, lens, 1, 3.0f, false, t == KvType::i8);
            paged_case(w, "empty_" + std::to_string(bi) + "_" + kvb::name(t), wl, 16, 5, 0, false, false);
        }
        ++bi;
    }
    // tests/boundary_tests.cpp:133-139: one block per sequence (page = max_len).
    for (KvType t : types)
        for (int L : {1, 17}) {
            const Workload wl(shapes[0], t, {L, L + 1}, 1, 3.0f, false, t == KvType::i8);
            paged_case(w, "contiguous_" + std::string(kvb::name(t)) + "_L" + std::to_string(L), wl, L + 1,
                       uint64_t(L + 1) * 1000 + 64, 64, true, false);
        }
    // The BASELINE head configuration (32 query heads, 8 KV heads, D = 128) at short lengths, with
    // each config's storage type and page size.
    {
        const Shape s{1, 32, 8, 128};
        const Workload w1(s, KvType::f32, {20}, 1, 1.0f);
        paged_case(w, "cfg1_like_f32_p16", w1, 16, 1016, 0, false, false);
        const Workload w2(s, KvType::f16, {40}, 1, 1.0f);
        paged_case(w, "cfg2_like_f16_p32", w2, 32, 1032, 512, false, false);
        const Workload w3(s, KvType::i8, {100}, 1, 1.0f);
        paged_case(w, "cfg3_like_i8_p128", w3, 128, 1128, 0, false, false);
        const Workload w5(Shape{1, 64, 8, 128}, KvType::f16, {20, 3}, 5, 1.0f);
        paged_case(w, "cfg5_like_f16_p16_G8", w5, 16, 5016, 0, false, false);
        const Workload w5i(Shape{1, 64, 8, 128}, KvType::i8, {40, 1}, 5, 1.0f);
        paged_case(w, "cfg5_like_i8_p32_G8", w5i, 32, 5032, 0, false, false);
    }
    known_answer_cases(w);

    w.json += "\n]}\n";
    std::fclose(w.bin);
    std::FILE* js = std::fopen(argv[2], "w");
    if (!js || std::fputs(w.json.c_str(), js) < 0) {
        std::perror(argv[2]);
        return 1;
    }
    std::fclose(js);
    std::printf("wrote %zu bytes of arrays\n", w.offset);
    return 0;
}
