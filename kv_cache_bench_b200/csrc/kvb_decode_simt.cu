// Paged split-K decode on CUDA cores: the general kernel. It covers every storage type (fp32,
// fp16, int8 + per-(block, KV head) scales), every page size (1, 3, ..., page = max_len), head dim
// 64/128 and any number of query heads per KV head; the tensor-core kernel (kvb_decode_mma.cu)
// takes the common fp16/int8 shapes.
//
// Restates the computation of the reference's paged_decode + paged_reduce
// (src/kernels.metal:43-147): per (sequence, KV-head group, partition) an online softmax over the
// partition's tokens in fp32, then a weighted merge of the partitions. B200 layout of the work:
//   * persistent CTAs of 4 warps loop over work units (kvb_device.cuh UnitCursor);
//   * a half-warp owns one token at a time, each lane D/16 consecutive head-dim elements, so a K or
//     V row is read with 16 coalesced 8-32 byte loads (the warp reads two full rows per load);
//   * scores are reduced with 4 butterfly shuffles per head inside the half-warp;
//   * K/V rows of TPJ tokens are loaded before any of them is used, for memory-level parallelism;
//   * the 8 half-warp states of a unit merge in shared memory, and the partitions of a sequence
//     merge in the last CTA to finish one (kvb_device.cuh finish_partition), so there is no
//     second kernel.
#include <cuda_fp16.h>

#include "kvb_device.cuh"

namespace {

using namespace kvb_dev;

constexpr int SIMT_THREADS = 128;
constexpr int SIMT_SLOTS = SIMT_THREADS / 16;

template <int KVT, int EPL>
struct RawRow;  // EPL elements of one K/V row as loaded

template <int EPL>
struct RawRow<0, EPL> {  // fp32
    float4 v[EPL / 4];
    __device__ __forceinline__ void load(const void* base, size_t off) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) v[i] = __ldg(p + i);
    }
    __device__ __forceinline__ void to_float(float (&f)[EPL]) const {
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) {
            f[4 * i + 0] = v[i].x;
            f[4 * i + 1] = v[i].y;
            f[4 * i + 2] = v[i].z;
            f[4 * i + 3] = v[i].w;
        }
    }
};

template <int EPL>
struct RawRow<1, EPL> {  // fp16
    static constexpr int W = EPL / 2;  // 32-bit words
    uint32_t w[W];
    __device__ __forceinline__ void load(const void* base, size_t off) {
        const __half* p = static_cast<const __half*>(base) + off;
        if constexpr (W == 4) {
            const uint4 x = __ldg(reinterpret_cast<const uint4*>(p));
            w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w;
        } else {
            const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
            w[0] = x.x, w[1] = x.y;
        }
    }
    __device__ __forceinline__ void to_float(float (&f)[EPL]) const {
#pragma unroll
        for (int i = 0; i < W; ++i) {
            const float2 t = __half22float2(u32_as_h2(w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
};

template <int EPL>
struct RawRow<2, EPL> {  // int8
    static constexpr int W = EPL / 4;
    uint32_t w[W];
    __device__ __forceinline__ void load(const void* base, size_t off) {
        const int8_t* p = static_cast<const int8_t*>(base) + off;
        if constexpr (W == 2) {
            const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
            w[0] = x.x, w[1] = x.y;
        } else {
            w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
        }
    }
    __device__ __forceinline__ void to_float(float (&f)[EPL]) const {
#pragma unroll
        for (int i = 0; i < W; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) f[4 * i + j] = float(int8_t(w[i] >> (8 * j)));
    }
};

template <int KVT, int D, int QGM>
__global__ void __launch_bounds__(SIMT_THREADS) decode_simt_kernel(const DecodeParams p) {
    constexpr int EPL = D / 16;                   // head-dim elements per lane
    constexpr int TPJ = QGM <= 4 ? 4 : 2;         // tokens per half-warp per step
    constexpr int STEP = SIMT_SLOTS * TPJ;        // tokens per CTA per step

    __shared__ int s_prefix[KVB_PREFIX_MAX + 1];
    __shared__ __align__(16) float s_slot_o[SIMT_SLOTS * KVB_EPI_HEADS * D];
    __shared__ float2 s_slot_ml[SIMT_SLOTS * KVB_EPI_HEADS];
    __shared__ int s_flag;

    const int tid = threadIdx.x, lane = tid & 31, l16 = lane & 15;
    const int slot = tid >> 4;
    // With KVB_FLAG_TABLES_READY and KVB_FLAG_INPUTS_READY, the lengths, block table, q, pools and
    // scales are not written by the kernel before this one: they are read while it finishes, and
    // each thread waits for it only before its first write (outputs, partials, split-K counters).
    const bool defer = p.tables_ready && p.inputs_ready;
    if (!defer) pdl_wait();
    pdl_trigger();
    bool waited = !defer;
    auto wait_prev = [&]() {
        if (!waited) {
            pdl_wait();
            waited = true;
        }
    };
    const int* prefix = nullptr;
    if (p.B <= KVB_PREFIX_MAX) {
        build_unit_prefix(p, s_prefix, reinterpret_cast<int*>(s_slot_o), tid, SIMT_THREADS, 1);
        prefix = s_prefix;
    }
    if (!defer) note_counter_count(p);
    UnitCursor cur{&p, prefix, (long long)blockIdx.x, unit_total(p, prefix)};

    Unit u;
    while (cur.advance(u)) {
        if (u.nparts == 0) {
            wait_prev();
            store_tokenless_unit<D>(p, u, tid, SIMT_THREADS);
            continue;
        }
        float qv[QGM][EPL];
#pragma unroll
        for (int g = 0; g < QGM; ++g)
#pragma unroll
            for (int e = 0; e < EPL; ++e)
                qv[g][e] = g < u.nh ? p.q[((size_t)u.b * p.H + u.h0 + g) * D + l16 * EPL + e] * p.q_scale : 0.f;
        float m[QGM], l[QGM], acc[QGM][EPL];
#pragma unroll
        for (int g = 0; g < QGM; ++g) {
            m[g] = NEG_BIG;
            l[g] = 0.f;
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
        }
        const int* bt = p.block_table + (size_t)u.b * p.max_blocks;
        bool bad = false;

        // The loop bound is uniform over each warp (the shuffles below need all 32 lanes); the two
        // half-warps take the two halves of the warp's 2 * TPJ tokens.
        for (int wbase = u.t0 + (slot >> 1) * 2 * TPJ; wbase < u.t1; wbase += STEP) {
            const int base = wbase + (slot & 1) * TPJ;
            RawRow<KVT, EPL> kr[TPJ], vr[TPJ];
            float ksc[TPJ], vsc[TPJ];
            bool valid[TPJ];
#pragma unroll
            for (int j = 0; j < TPJ; ++j) {
                const int t = base + j;
                valid[j] = t < u.t1;
                ksc[j] = vsc[j] = 1.f;
                kr[j] = RawRow<KVT, EPL>{};  // rows not loaded stay finite (zero)
                vr[j] = RawRow<KVT, EPL>{};
                if (valid[j]) {
                    long long blk = __ldg(bt + t / p.page);
                    if (blk < 0 || blk >= p.num_blocks) {  // refused block id: read nothing
                        bad = true;
                        valid[j] = false;
                        continue;
                    }
                    const size_t slot_kv = (size_t)blk * p.Hkv + u.kvh;
                    const size_t off = ((slot_kv * p.page) + (size_t)(t % p.page)) * D + l16 * EPL;
                    kr[j].load(p.k, off);
                    vr[j].load(p.v, off);
                    if constexpr (KVT == 2) {
                        ksc[j] = __ldg(p.k_scale + slot_kv);
                        vsc[j] = __ldg(p.v_scale + slot_kv);
                    }
                }
            }
            float s[TPJ][QGM];
#pragma unroll
            for (int j = 0; j < TPJ; ++j) {
                float kf[EPL];
                kr[j].to_float(kf);
#pragma unroll
                for (int g = 0; g < QGM; ++g) {
                    float d = 0.f;
#pragma unroll
                    for (int e = 0; e < EPL; ++e) d = fmaf(qv[g][e], kf[e], d);
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    s[j][g] = (valid[j] && g < u.nh) ? d * ksc[j] : NEG_BIG;
                }
            }
#pragma unroll
            for (int g = 0; g < QGM; ++g) {
                float mx = m[g];
#pragma unroll
                for (int j = 0; j < TPJ; ++j) mx = fmaxf(mx, s[j][g]);
                const float corr = exp2f(m[g] - mx);
                m[g] = mx;
                l[g] *= corr;
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[g][e] *= corr;
            }
#pragma unroll
            for (int j = 0; j < TPJ; ++j) {
                if (!valid[j]) continue;
                float vf[EPL];
                vr[j].to_float(vf);
#pragma unroll
                for (int g = 0; g < QGM; ++g) {
                    const float pr = exp2f(s[j][g] - m[g]);
                    l[g] += pr;
                    const float pv = pr * vsc[j];
#pragma unroll
                    for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pv, vf[e], acc[g][e]);
                }
            }
        }
        wait_prev();  // the outputs, partials and counters come next
        if (bad) raise_error(p.error_flag, KVB_DEVERR_BLOCK);
        // Also the barrier after which the previous unit's epilogue buffers are free.
        const int unit_bad = __syncthreads_or(bad);

        // Merge the 8 half-warp states, KVB_EPI_HEADS heads per round (rounds unrolled so the
        // accumulator stays in registers).
#pragma unroll
        for (int round = 0; round < (QGM + KVB_EPI_HEADS - 1) / KVB_EPI_HEADS; ++round) {
            const int g0 = round * KVB_EPI_HEADS;
            if (g0 >= u.nh) break;
            if (g0 > 0) __syncthreads();
#pragma unroll
            for (int gg = 0; gg < KVB_EPI_HEADS; ++gg) {
                const int g = g0 + gg;
                if (g >= QGM) break;
#pragma unroll
                for (int e = 0; e < EPL; ++e)
                    s_slot_o[(slot * KVB_EPI_HEADS + gg) * D + l16 * EPL + e] = acc[g][e];
                if (l16 == 0) s_slot_ml[slot * KVB_EPI_HEADS + gg] = make_float2(m[g], l[g]);
            }
            __syncthreads();
            const float o_scale = unit_bad ? __int_as_float(0x7fc00000) : 1.0f;
            merge_slots_and_store<D>(p, u, s_slot_o, s_slot_ml, SIMT_SLOTS, g0, min(KVB_EPI_HEADS, u.nh - g0),
                                     o_scale, tid, SIMT_THREADS);
        }
        finish_partition<D>(p, u, tid, SIMT_THREADS, 1, &s_flag);
        __syncthreads();
    }
    if (defer) {
        wait_prev();
        note_counter_count(p);
    }
}

template <int KVT, int D, int QGM>
cudaError_t launch_one(const DecodeParams& p, const LaunchInfo& li) {
    static KvbPerDevice<int> per_device;  // occupancy, per device
    int blocks_per_sm = 0;
    const cudaError_t e = per_device.get(&blocks_per_sm, [](int* n) {
        const cudaError_t r =
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, decode_simt_kernel<KVT, D, QGM>, SIMT_THREADS, 0);
        if (*n < 1) *n = 1;
        return r;
    });
    if (e != cudaSuccess) return e;
    const long long upper = (long long)p.B * p.nhg * p.max_parts;
    const long long grid = std::min<long long>(upper, (long long)li.num_sms * blocks_per_sm);
    if (grid <= 0) return cudaSuccess;
    return kvb_launch_pdl(decode_simt_kernel<KVT, D, QGM>, (unsigned)grid, SIMT_THREADS, 0, li.stream, p);
}

template <int KVT, int D>
cudaError_t launch_qg(const DecodeParams& p, const LaunchInfo& li) {
    if (p.qg <= 1) return launch_one<KVT, D, 1>(p, li);
    if (p.qg <= 2) return launch_one<KVT, D, 2>(p, li);
    if (p.qg <= 4) return launch_one<KVT, D, 4>(p, li);
    return launch_one<KVT, D, 8>(p, li);
}

template <int KVT>
cudaError_t launch_d(const DecodeParams& p, int D, const LaunchInfo& li) {
    return D == 64 ? launch_qg<KVT, 64>(p, li) : launch_qg<KVT, 128>(p, li);
}

}  // namespace

cudaError_t kvb_launch_decode_simt(const DecodeParams& p, int kv_type, int D, const LaunchInfo& li) {
    switch (kv_type) {
    case 0: return launch_d<0>(p, D, li);
    case 1: return launch_d<1>(p, D, li);
    default: return launch_d<2>(p, D, li);
    }
}
