// Device-side building blocks shared by the paged decode kernels: inline-PTX wrappers for sm_100a
// (mbarrier, TMA tile loads, ldmatrix, mma.sync), bounded waits that report instead of hanging,
// the split-K work-unit enumeration, and the per-unit epilogue with the fused cross-partition merge.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kvb_internal.h"

namespace kvb_dev {

// A score that is "minus infinity" but finite: exp2(NEG_BIG - m) is exactly 0 for any real m and
// max/min arithmetic on it never produces NaN (the same convention as the reference kernel,
// src/kernels.metal:18-20).
constexpr float NEG_BIG = -1e30f;

// ---- error reporting -------------------------------------------------------------------------

// Sets bits of the workspace error word (KVB_DEVERR_* in kvb_internal.h).
__device__ __forceinline__ void raise_error(unsigned* flag, unsigned bits) { atomicOr(flag, bits); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- shared memory / mbarrier ------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Raises the transaction count the current phase waits for, without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test: has the phase with parity `parity` of `bar` completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with parity `parity` of `bar` to complete, for at most KVB_WAIT_LIMIT_NS of
// wall time (or until `*abort` is set by another warp). Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > KVB_WAIT_LIMIT_NS) return false;
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier among `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also returns whether `pred` was non-zero in any participating thread.
__device__ __forceinline__ int named_barrier_or(uint32_t id, uint32_t nthreads, int pred) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred), "r"(id), "r"(nthreads)
        : "memory");
    return r;
}

// ---- TMA ----------------------------------------------------------------------------------------

// 2-D tiled bulk tensor load global -> shared, completing on `bar` (transaction bytes). The
// innermost coordinate x is always 0 or a multiple of 128 bytes in this code.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// L2 policy for streamed K/V pages: evict first, so block tables, scales and partials stay.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Programmatic dependent launch. The decode kernels are launched with programmatic stream
// serialization, so a launch can start (and run its shared-memory setup) while the kernel before it
// in the stream finishes. Every thread calls pdl_wait() before its first global memory access: it
// returns once the previous grid has completed and its writes are visible. pdl_trigger() lets the
// next launch in the stream start as SMs free up; that launch waits for this grid the same way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// ---- shared-memory loads and tensor-core helpers -----------------------------------------------

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void lds64(uint32_t addr, uint32_t& a, uint32_t& b) {
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
}

__device__ __forceinline__ void sts128_zero(uint32_t addr) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Splits (x0, x1) into fp16 pairs hi + lo with hi = fp16(x), lo = fp16(x - hi): the pair carries
// about 22 significant bits, enough for fp32-level dot products on exact fp16/int8 operands.
__device__ __forceinline__ void split_hi_lo(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2_as_u32(h);
    lo = h2_as_u32(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

// int8 -> fp16 pairs. An fp16 with bit pattern 0x64XX is 1024 + XX for XX < 1024, so a signed byte
// b becomes 0x64 | (b ^ 0x80) = 1152 + b and one subtraction of 1152 gives b exactly.
//
// Bytes (lo_byte, hi_byte) of `w_biased` (already XORed with 0x80808080) to half2(b_lo, b_hi):
__device__ __forceinline__ uint32_t i8pair_to_h2(uint32_t w_biased, uint32_t sel) {
    const uint32_t x = __byte_perm(w_biased, 0x64646464u, sel);
    return h2_as_u32(__hsub2(u32_as_h2(x), __half2half2(__ushort_as_half(0x6480))));
}
// Selectors for i8pair_to_h2: bytes (0,1) and (2,3) of the word, 0x64 from the second operand.
constexpr uint32_t SEL_B01 = 0x4140;
constexpr uint32_t SEL_B23 = 0x4342;

// Byte i of `wa` and byte i of `wb` (unbiased) to half2(a_i, b_i): the transposing conversion used
// for V, where the two values of a pair come from two different token rows.
__device__ __forceinline__ uint32_t i8cross_to_h2(uint32_t wa, uint32_t wb, uint32_t i) {
    const uint32_t x = __byte_perm(wa, wb, i | ((4u + i) << 8));
    const uint32_t y = (x & 0x00FF00FFu) ^ 0x64806480u;
    return h2_as_u32(__hsub2(u32_as_h2(y), __half2half2(__ushort_as_half(0x6480))));
}

// ---- work units ---------------------------------------------------------------------------------

// n / f.d for 0 <= n < 2^31 (see KvbDiv).
__device__ __forceinline__ int kvb_div(int n, const KvbDiv& f) { return int((__umulhi(unsigned(n), f.m) + unsigned(n)) >> f.l); }

// n / d and n % d for 0 <= n < 2^31 and 1 <= d whose quotient is below 2^20: a float estimate within
// one of n / d (the inputs, the reciprocal and the product are each rounded once, a relative error
// below 2^-21 of a quotient below 2^20) and one correction step.
__device__ __forceinline__ int div_small_quotient(int n, int d, int* rem) {
    int q = __float2int_rz(__int2float_rn(n) * __frcp_rn(__int2float_rn(d)));
    int r = n - q * d;
    if (r < 0) {
        --q;
        r += d;
    } else if (r >= d) {
        ++q;
        r -= d;
    }
    *rem = r;
    return q;
}

// Output stores. Without peers: out[b][h][d]. With peers (a sharded step gathered in the kernel):
// the element's global position, in this rank's own global buffer (peer_out[peer_self]) and, by
// the same thread, in every other rank's over peer memory; a global row outside [0, peer_rows) is
// refused (error bit KVB_DEVERR_BLOCK, nothing stored).
__device__ __forceinline__ bool peer_index(const DecodeParams& p, int b, int h, int D, size_t* i) {
    const int row = p.out_rows ? __ldg(p.out_rows + b) : b;
    if (row < 0 || row >= p.peer_rows) {
        raise_error(p.error_flag, KVB_DEVERR_BLOCK);
        return false;
    }
    *i = ((size_t)row * p.out_heads + p.out_head0 + h) * D;
    return true;
}

// The element at offset i of this rank's own global buffer, stored by this thread, copied to the
// other ranks' buffers.
template <typename T>
__device__ __forceinline__ void copy_to_peers(const DecodeParams& p, size_t i) {
    const T v = *reinterpret_cast<const T*>(p.peer_out[p.peer_self] + i);
#pragma unroll 1
    for (int j = 0; j < p.n_peers; ++j)
        if (j != p.peer_self) *reinterpret_cast<T*>(p.peer_out[j] + i) = v;
}

// PEERS false compiles the peer path out (an instance that never serves a gathered launch).
template <int D, bool PEERS = true>
__device__ __forceinline__ void store_out(const DecodeParams& p, int b, int h, int d, float v) {
    if (!PEERS || p.n_peers == 0) {
        p.out[((size_t)b * p.H + h) * D + d] = v;
        return;
    }
    size_t i;
    if (!peer_index(p, b, h, D, &i)) return;
    p.peer_out[p.peer_self][i + d] = v;
    copy_to_peers<float>(p, i + d);
}

template <int D, bool PEERS = true>
__device__ __forceinline__ void store_out4(const DecodeParams& p, int b, int h, int d4, float4 v) {
    if (!PEERS || p.n_peers == 0) {
        reinterpret_cast<float4*>(p.out + ((size_t)b * p.H + h) * D)[d4] = v;
        return;
    }
    size_t i;
    if (!peer_index(p, b, h, D, &i)) return;
    reinterpret_cast<float4*>(p.peer_out[p.peer_self] + i)[d4] = v;
    copy_to_peers<float4>(p, i + 4 * d4);
}

// One work unit is one split-K partition [t0, t1) of one sequence b for one group of query heads
// that share a KV head. Units are numbered sequence-major, then head group, then partition.
struct Unit {
    int b, hg, part;
    int kvh, h0, nh;  // KV head, first query head, heads in the group
    int len;          // sequence length (validated)
    int t0, t1;       // token range of the partition
    int nparts;       // partitions of this sequence (0 when empty or invalid)
    bool bad;         // the length is out of range: outputs get NaN
};

// Partitions of a sequence of length len, or 0 for an empty or invalid one; invalid lengths are
// reported in *bad. Every (sequence, head group) owns max(1, partitions) units.
__device__ __forceinline__ int seq_partitions(const DecodeParams& p, int len, bool* bad) {
    *bad = len < 0 || len > p.max_len || (long long)len > (long long)p.max_blocks * p.page;
    if (*bad || len == 0) return 0;
    return kvb_div(len - 1, p.div_part) + 1;
}

__device__ __forceinline__ Unit make_unit(const DecodeParams& p, int b, int hg, int part, int len) {
    Unit u;
    u.b = b;
    u.hg = hg;
    u.part = part;
    u.len = len;
    u.nparts = seq_partitions(p, len, &u.bad);
    u.kvh = kvb_div(hg, p.div_gpk);
    const int in_kvh = hg - u.kvh * p.gpk;  // head group within the KV head
    u.h0 = u.kvh * p.G + in_kvh * p.qg;
    u.nh = min(p.qg, p.G - in_kvh * p.qg);
    u.t0 = part * p.part_tokens;
    u.t1 = u.nparts ? min(len, u.t0 + p.part_tokens) : 0;
    return u;
}

// Iterates this CTA's units (static round robin over the grid). With B <= KVB_PREFIX_MAX the
// units are packed through a prefix sum over sequences kept in shared memory (`prefix`, B + 1
// ints, filled by build_unit_prefix); otherwise every (b, hg, part < max_parts) slot is visited and
// slots past a sequence's partitions are skipped.
// The unit with index idx (0 <= idx < unit_total): false for a dense-mode slot past its sequence's
// partitions, which is no unit at all. `prefix` and `lens` as in UnitCursor.
__device__ __forceinline__ bool unit_at(const DecodeParams& P, const int* prefix, const int* lens, long long idx,
                                        Unit& u) {
    int b, hg, part, len;
    if (prefix) {
        // largest b with prefix[b] <= idx
        int lo = 0, hi = P.B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= idx) lo = mid;
            else hi = mid - 1;
        }
        b = lo;
        len = lens ? lens[b] : __ldg(P.seq_lens + b);
        bool bad;
        const int per = max(1, seq_partitions(P, len, &bad));
        hg = div_small_quotient(int(idx - prefix[b]), per, &part);
    } else {
        // unit indices stay below 2^31 (the host refuses larger launches)
        b = kvb_div(int(idx), P.div_seq);
        const int rem = int(idx) - b * int(P.div_seq.d);
        hg = kvb_div(rem, P.div_parts);
        part = rem - hg * P.max_parts;
        len = __ldg(P.seq_lens + b);
        bool bad;
        if (part >= max(1, seq_partitions(P, len, &bad))) return false;
    }
    u = make_unit(P, b, hg, part, len);
    return true;
}

struct UnitCursor {
    const DecodeParams* p;
    const int* prefix;  // nullptr: dense enumeration
    long long next, total;
    const int* lens = nullptr;  // sequence lengths cached in shared memory (prefix mode), or nullptr

    __device__ __forceinline__ bool advance(Unit& u) {
        while (next < total) {
            const long long idx = next;
            next += gridDim.x;
            if (unit_at(*p, prefix, lens, idx, u)) return true;
        }
        return false;
    }
};

// Fills prefix[0..B] with the running count of units per sequence (nhg * max(1, partitions)), and
// lens_out[0..B) with the lengths when it is not null. Called by `nthreads` threads (a multiple of
// 32, at most 1024) that then synchronize on barrier `bar_id`; `scratch` holds nthreads ints of
// shared memory.
__device__ __forceinline__ void build_unit_prefix(const DecodeParams& p, int* prefix, int* scratch, int tid,
                                                  int nthreads, uint32_t bar_id, int* lens_out = nullptr) {
    // Each thread counts a contiguous slice, then warp 0 scans the slice totals.
    const int per = (p.B + nthreads - 1) / nthreads;
    const int s0 = min(p.B, tid * per), s1 = min(p.B, s0 + per);
    int sum = 0;
    for (int b = s0; b < s1; ++b) {
        bool bad;
        const int len = __ldg(p.seq_lens + b);
        if (lens_out) lens_out[b] = len;
        sum += p.nhg * max(1, seq_partitions(p, len, &bad));
        prefix[b + 1] = sum;  // slice-local inclusive sums for now
    }
    scratch[tid] = sum;
    named_barrier(bar_id, nthreads);
    if (tid < 32) {
        int carry = 0;
        for (int base = 0; base < nthreads; base += 32) {
            int v = scratch[base + tid];
            int incl = v;
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += n;
            }
            scratch[base + tid] = carry + incl - v;  // exclusive offset of this slice
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    named_barrier(bar_id, nthreads);
    const int off = scratch[tid];
    for (int b = s0; b < s1; ++b) prefix[b + 1] += off;
    if (tid == 0) prefix[0] = 0;
    named_barrier(bar_id, nthreads);
}

// build_unit_prefix for blocks with at least one thread per sequence (nthreads >= KVB_PREFIX_MAX, a
// multiple of 32): thread b counts sequence b, each warp scans its 32 counts with shuffles, and each
// thread adds the totals of the warps before its own. A few dozen instructions, against the slice
// loops and the unrolled multi-round scan of the general form. `scratch` holds nthreads / 32 ints;
// `len` is thread tid's read of seq_lens[tid] (tid < B), which the caller may have started early.
__device__ __forceinline__ void build_unit_prefix_wide(const DecodeParams& p, int* prefix, int* scratch, int tid,
                                                       int nthreads, uint32_t bar_id, int* lens_out, int len) {
    int v = 0;
    if (tid < p.B) {
        bool bad;
        lens_out[tid] = len;
        v = p.nhg * max(1, seq_partitions(p, len, &bad));
    }
    const int lane = tid & 31, w = tid >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) scratch[w] = incl;
    named_barrier(bar_id, nthreads);
    int off = 0;
#pragma unroll 1
    for (int i = 0; i < w; ++i) off += scratch[i];
    if (tid < p.B) prefix[tid + 1] = off + incl;
    if (tid == 0) prefix[0] = 0;
    named_barrier(bar_id, nthreads);
}

__device__ __forceinline__ long long unit_total(const DecodeParams& p, const int* prefix) {
    return prefix ? (long long)prefix[p.B] : (long long)p.B * p.nhg * p.max_parts;
}

// Workspace words 2 and 3: the units handed out beyond the first grid-wide round, and the CTAs that
// found none left (kernels that take units dynamically; the last such CTA zeroes both).
__device__ __forceinline__ unsigned* work_counters(const DecodeParams& p) { return p.error_flag + 2; }

// Records in workspace word 1 how many arrival counters this launch uses (see KVB_DEVERR_STATE).
__device__ __forceinline__ void note_counter_count(const DecodeParams& p) {
    if (blockIdx.x == 0 && threadIdx.x == 0) p.error_flag[1] = unsigned(p.B * p.nhg);
}

// ---- epilogue -----------------------------------------------------------------------------------

// Finishes one unit once its per-slot online-softmax states are in shared memory:
//   slot_o  [nslots][KVB_EPI_HEADS][D]  unnormalized accumulators (already scaled by `o_scale`
//                                       when read), slot_ml [nslots][KVB_EPI_HEADS] (m, l), m in
//                                       log2 units.
// Heads are processed in rounds of KVB_EPI_HEADS by the caller; this handles heads
// [g0, g0 + ng) of unit u. A single-partition sequence writes `out` directly; otherwise the
// partition is stored to the workspace and the last partition to arrive (atomic counter per
// (sequence, head group)) merges all of them into `out`.
//
// Threads: `nthreads` consecutive threads starting at tid 0 of the group, barrier `bar_id`.
template <int D>
__device__ __forceinline__ void merge_slots_and_store(const DecodeParams& p, const Unit& u, const float* slot_o,
                                                      const float2* slot_ml, int nslots, int g0, int ng,
                                                      float o_scale, int tid, int nthreads) {
    for (int idx = tid; idx < ng * D; idx += nthreads) {
        const int g = idx / D, d = idx % D;
        float M = NEG_BIG;
        for (int s = 0; s < nslots; ++s) M = fmaxf(M, slot_ml[s * KVB_EPI_HEADS + g].x);
        float L = 0.f, o = 0.f;
        for (int s = 0; s < nslots; ++s) {
            const float2 ml = slot_ml[s * KVB_EPI_HEADS + g];
            const float w = exp2f(ml.x - M);
            L += ml.y * w;
            o += slot_o[(s * KVB_EPI_HEADS + g) * D + d] * w;
        }
        o *= o_scale;
        const int h = u.h0 + g0 + g;
        if (u.nparts == 1) {
            store_out<D>(p, u.b, h, d, o / L);
        } else {
            const size_t slot = ((size_t)u.b * p.H + h) * p.max_parts + u.part;
            p.part_o[slot * D + d] = o / L;
            if (d == 0) p.part_ml[slot] = make_float2(M, L);
        }
    }
}

// After every round of merge_slots_and_store for a multi-partition unit: counts the partition
// in and, if it was the last one, merges all partitions of (b, head group) into `out`.
//
// The arrival counter of (b, head group) is a 64-bit word (epoch << 32 | arrivals), counted with
// one atomic add per partition. The last arrival leaves it at (KVB_CTR_CLEAN << 32), which the next
// launch counts from directly. Any other epoch that is not this launch's id is stale -- a zeroed
// workspace, or partial results of a call with another layout where this call keeps its counters --
// and an arrival that meets one claims the word for this launch (compare-and-swap to
// launch << 32) and counts itself again, so only the first use after a layout change pays for a
// compare-and-swap. An arrival past the partition count (two launches sharing one workspace at the
// same time, or an aborted launch) raises KVB_DEVERR_STATE; the flag reader then resets the counters.
//
// The merge (src/kernels.metal:124-147): out = sum_i L_i 2^(m_i - M) o_i / sum_i L_i 2^(m_i - M)
// over the stored normalized partials o_i with their (m_i, L_i). `nthreads` threads split the
// (head, 4-dim slice) pairs; when there are fewer pairs than threads, SPLIT consecutive lanes share a
// pair and take every SPLIT-th partition, so more loads are in flight at once. Each lane keeps an
// online (M, S, A) over batches of BATCH partitions and the lanes of a pair combine with shuffles.
//
// Threads: `nthreads` consecutive threads (a multiple of 32) starting at tid 0, barrier `bar_id`.
// Atomic add with release (this CTA's earlier stores, ordered before it by a barrier, are visible
// to whoever observes the add) and acquire (later loads see what the other adders released).
__device__ __forceinline__ unsigned long long atom_add_acq_rel(unsigned long long* ptr, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(ptr), "l"(v) : "memory");
    return old;
}

// Counts partition u in: one atomic add on its (b, head group) counter, returning the old word.
// Called by one thread after a barrier that orders the CTA's partial stores before it (release).
__device__ __forceinline__ unsigned long long arrive_partition(const DecodeParams& p, const Unit& u) {
    return atom_add_acq_rel(p.counters + (size_t)u.b * p.nhg + u.hg, 1ull);
}

// Whether the arrival that returned `old` was the last partition of u (then the counter is left
// clean for the next launch). A stale epoch is claimed here; see above.
__device__ __forceinline__ bool resolve_arrival(const DecodeParams& p, const Unit& u, unsigned long long old) {
    unsigned long long* ctr = p.counters + (size_t)u.b * p.nhg + u.hg;
    const unsigned epoch = unsigned(old >> 32);
    unsigned arrived;
    if (epoch == p.launch || epoch == KVB_CTR_CLEAN) {
        arrived = unsigned(old) + 1u;
    } else {
        __threadfence();
        unsigned long long seen = old + 1ull;
        for (;;) {
            const unsigned long long cur = atomicCAS(ctr, seen, (unsigned long long)p.launch << 32);
            const unsigned e = unsigned(cur >> 32);
            if (cur == seen || e == p.launch || e == KVB_CTR_CLEAN) break;
            seen = cur;
        }
        arrived = unsigned(atom_add_acq_rel(ctr, 1ull)) + 1u;
    }
    const bool last = arrived == unsigned(u.nparts);
    if (arrived > unsigned(u.nparts)) raise_error(p.error_flag, KVB_DEVERR_STATE);
    if (last) atomicExch(ctr, (unsigned long long)KVB_CTR_CLEAN << 32);
    return last;
}

template <int D, int BATCH = 8, int MAXSPLIT = 32, bool PEERS = true>
__device__ __forceinline__ void merge_partitions(const DecodeParams& p, const Unit& u, int tid, int nthreads);

// MAXSPLIT bounds the lanes that share a (head, 4-dim slice) pair: a caller whose heads always fill
// half of its threads passes 1, and the lane combine is compiled out.
template <int D, int BATCH = 8, int MAXSPLIT = 32, bool PEERS = true>
__device__ __forceinline__ void finish_partition(const DecodeParams& p, const Unit& u, int tid, int nthreads,
                                                 uint32_t bar_id, int* s_flag) {
    if (u.nparts <= 1) return;
    named_barrier(bar_id, nthreads);  // every thread's partial stores come before the arrival below
    if (tid == 0) *s_flag = resolve_arrival(p, u, arrive_partition(p, u));
    named_barrier(bar_id, nthreads);
    if (*s_flag) merge_partitions<D, BATCH, MAXSPLIT, PEERS>(p, u, tid, nthreads);
}

// The merge of all partitions of u into `out` (the CTA of the last partition, every other
// partition's stores visible through the acquiring arrival).
template <int D, int BATCH, int MAXSPLIT, bool PEERS>
__device__ __forceinline__ void merge_partitions(const DecodeParams& p, const Unit& u, int tid, int nthreads) {
    constexpr int D4 = D / 4;
    const int np = u.nparts, nh = u.nh;
    const int pairs = nh * D4;
    int split = 1;
    while (split < MAXSPLIT && split * 2 * pairs <= nthreads) split *= 2;
    const int s = tid % split;
    for (int base = 0; base < pairs * split; base += nthreads) {  // the same trip count in every lane
        const int idx = base + tid;
        const bool active = idx < pairs * split;
        const int pair = active ? idx / split : 0;
        const int g = pair / D4, d4 = pair % D4, h = u.h0 + g;
        const size_t row = ((size_t)u.b * p.H + h) * p.max_parts;
        const float4* po = reinterpret_cast<const float4*>(p.part_o + row * D) + d4;
        float M = NEG_BIG, S = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i0 = active ? s : np; i0 < np; i0 += BATCH * split) {
            float2 ml[BATCH];
            float4 ov[BATCH];
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                const int i = i0 + j * split;
                if (i < np) {
                    ml[j] = __ldcg(&p.part_ml[row + i]);
                    ov[j] = __ldcg(po + (size_t)i * D4);
                } else {
                    ml[j] = make_float2(NEG_BIG, 0.f);
                    ov[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float Mb = M;
#pragma unroll
            for (int j = 0; j < BATCH; ++j) Mb = fmaxf(Mb, ml[j].x);
            const float sc = exp2f(M - Mb);
            S *= sc;
            A.x *= sc, A.y *= sc, A.z *= sc, A.w *= sc;
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                const float w = ml[j].y * exp2f(ml[j].x - Mb);
                S += w;
                A.x = fmaf(w, ov[j].x, A.x);
                A.y = fmaf(w, ov[j].y, A.y);
                A.z = fmaf(w, ov[j].z, A.z);
                A.w = fmaf(w, ov[j].w, A.w);
            }
            M = Mb;
        }
        // combine the `split` lanes of this pair (consecutive lanes)
        for (int off = 1; off < split; off <<= 1) {
            const float M2 = __shfl_xor_sync(0xffffffffu, M, off);
            const float S2 = __shfl_xor_sync(0xffffffffu, S, off);
            const float ax = __shfl_xor_sync(0xffffffffu, A.x, off), ay = __shfl_xor_sync(0xffffffffu, A.y, off);
            const float az = __shfl_xor_sync(0xffffffffu, A.z, off), aw = __shfl_xor_sync(0xffffffffu, A.w, off);
            const float Mn = fmaxf(M, M2), c1 = exp2f(M - Mn), c2 = exp2f(M2 - Mn);
            S = S * c1 + S2 * c2;
            A = make_float4(A.x * c1 + ax * c2, A.y * c1 + ay * c2, A.z * c1 + az * c2, A.w * c1 + aw * c2);
            M = Mn;
        }
        if (active && s == 0) {
            const float inv = 1.f / S;
            store_out4<D, PEERS>(p, u.b, h, d4, make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv));
        }
    }
}

// Units with no tokens: an empty sequence attends to nothing and gives exactly 0; a sequence whose
// length was refused gives NaN and raises the error flag.
template <int D, bool PEERS = true>
__device__ __forceinline__ void store_tokenless_unit(const DecodeParams& p, const Unit& u, int tid, int nthreads) {
    if (u.bad && tid == 0) raise_error(p.error_flag, KVB_DEVERR_LENGTH);
    const float val = u.bad ? __int_as_float(0x7fc00000) : 0.0f;
    for (int idx = tid; idx < u.nh * D; idx += nthreads) store_out<D, PEERS>(p, u.b, u.h0 + idx / D, idx % D, val);
}

}  // namespace kvb_dev
