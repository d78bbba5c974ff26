// The page write path in front of decode: a contiguous cache [B][Hkv][max_len][D] written into the
// paged pool [num_blocks][Hkv][page][D] through the block table.
//
//   quantize (int8)   src/reference.cpp:32-51 (quantize_to_paged_i8): per (sequence, logical page,
//                     KV head) amax over the page's live tokens and all D, scale = amax / 127 (fp32),
//                     q = clamp(nearbyint(x / scale), -127, 127) with an IEEE fp32 division and
//                     round-half-to-even, 0 when the scale is 0; the scale goes to
//                     scales[block * Hkv + kvh].
//   scatter           src/reference.hpp:60-68 (scatter_to_paged): the live tokens copied unchanged.
//
// Slots past a sequence's last token are not written (as in the reference). A persistent grid walks
// the runs (sequence, page slot, KV head): a live page's rows are one contiguous run in both layouts,
// moved with 16-byte vectors, PW_UNROLL of them in flight per thread, by one warp (runs under 64 KB)
// or one CTA (larger runs, so that enough bytes are in flight). Dead slots cost a shared-memory
// length lookup. The quantizer keeps a run of up to 8 KB in registers; a larger one it reads twice
// (amax, then quantize), the second pass from L1/L2, so HBM sees each input byte once. Bad lengths or block ids skip the
// page and raise the same error bits as the decode kernels.
#include <cuda_fp16.h>

#include <algorithm>

#include "kvb_device.cuh"

namespace {

using namespace kvb_dev;

constexpr int PW_THREADS = 256;
constexpr int PW_WARPS = PW_THREADS / 32;
constexpr int PW_UNROLL = 8;          // 16-byte loads in flight per lane
constexpr int PW_LENS_MAX = 8192;     // sequence lengths cached in shared memory up to this batch
constexpr int PW_REG_F4 = 16;         // quantizer runs of up to 32 x 16 float4 (8 KB) stay in registers

struct Run {
    const void* src;  // first source byte of the run
    void* dst;        // first pool byte of the run
    long long blk;    // physical block
    int kvh;          // KV head
    int n;            // live tokens of the page
};

// The run of (sequence b, page slot i, KV head kvh), or n = 0 for a dead or refused slot (refusals
// raise their error bit).
__device__ __forceinline__ Run run_of(const PageWriteParams& p, int b, int i, int kvh, const int* s_len, int lane) {
    Run r{nullptr, nullptr, 0, 0, 0};
    const int len = s_len ? s_len[b] : __ldg(p.seq_lens + b);
    if (len < 0 || len > p.max_len || (long long)len > (long long)p.max_blocks * p.page) {
        if (i == 0 && kvh == 0 && lane == 0 && p.error_flag) raise_error(p.error_flag, KVB_DEVERR_LENGTH);
        return r;
    }
    const int t0 = i * p.page;
    if (t0 >= len) return r;
    const int blk = __ldg(p.block_table + (size_t)b * p.max_blocks + i);
    if (blk < 0 || (long long)blk >= p.num_blocks) {
        if (kvh == 0 && lane == 0 && p.error_flag) raise_error(p.error_flag, KVB_DEVERR_BLOCK);
        return r;
    }
    const size_t row = (size_t)p.D * p.src_elem;
    r.src = static_cast<const char*>(p.src) + (((size_t)b * p.Hkv + kvh) * p.max_len + t0) * row;
    r.dst = static_cast<char*>(p.dst) + ((size_t)blk * p.Hkv + kvh) * p.page * (size_t)p.D * p.elem;
    r.blk = blk;
    r.kvh = kvh;
    r.n = min(len - t0, p.page);
    return r;
}

// Four values quantized with `scale` (0 when the scale is 0), packed low byte first:
// clamp(rint(x / scale), -127, 127) with the IEEE division of the reference. |x / scale| <= 127, so
// t = x * fl(1 / scale) is within 2^-16 of the exact quotient and fl(x / scale) within 2^-17 of it.
// When t is at least 2^-14 away from every half-integer, no rounding boundary lies between t and
// fl(x / scale), and the integer nearest t is the reference's value. t + 1.5 * 2^23 rounds t to that
// integer (ties to even) and holds it in its low mantissa bits: two full-rate additions instead of a
// round and a conversion. The fast path flags (in `near`) any value close to a boundary; the caller
// then redoes its values with quantize4_exact, which takes the division (rare: one test per run, not
// a branch per value). `rcp` = 1 / scale, finite.
__device__ __forceinline__ uint32_t quantize4_fast(const float4 v, float rcp, int& near) {
    constexpr float kMagic = 12582912.f;  // 1.5 * 2^23
    const float x[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float t = __fmul_rn(x[e], rcp);
        const float y = __fadd_rn(t, kMagic);
        const int q = min(max(__float_as_int(y) - 0x4B400000, -127), 127);
        near |= fabsf(__fsub_rn(t, __fsub_rn(y, kMagic))) >= 0.5f - 6.103515625e-05f;
        packed |= uint32_t(q & 255) << (8 * e);
    }
    return packed;
}

__device__ __noinline__ uint32_t quantize4_exact(const float4 v, float scale) {
    const float x[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int q = min(max(__float2int_rn(__fdiv_rn(x[e], scale)), -127), 127);
        packed |= uint32_t(q & 255) << (8 * e);
    }
    return packed;
}

__device__ __forceinline__ float finite_rcp(float scale) {
    const float r = 1.0f / scale;
    return scale > 0.f && r < 3.0e38f ? r : 0.f;
}

// TPR threads (a warp or the whole CTA) per run.
template <bool QUANT, int TPR>
__global__ void __launch_bounds__(PW_THREADS) page_write_kernel(const PageWriteParams p) {
    constexpr int GROUPS = PW_THREADS / TPR;  // runs in flight per CTA
    __shared__ float s_max[2][PW_WARPS];
    extern __shared__ int s_len_raw[];
    const int* s_len = nullptr;
    if (p.B <= PW_LENS_MAX) {
        for (int b = threadIdx.x; b < p.B; b += PW_THREADS) s_len_raw[b] = __ldg(p.seq_lens + b);
        __syncthreads();
        s_len = s_len_raw;
    }
    const int lane = threadIdx.x & 31;
    const int gl = threadIdx.x % TPR;  // thread within the run's group
    // Task t = (b * max_blocks + i) * Hkv + kvh, one group per task, tasks t, t + stride, ...; the
    // position is advanced in mixed radix (no division per task).
    const long long t0 = (long long)blockIdx.x * GROUPS + threadIdx.x / TPR;
    const long long stride = (long long)gridDim.x * GROUPS;
    int parity = 0;  // alternates the CTA-wide reduction slots
    int kvh = int(t0 % p.Hkv), i = int(t0 / p.Hkv % p.max_blocks);
    long long b = t0 / p.Hkv / p.max_blocks;
    const int dk = int(stride % p.Hkv), di = int(stride / p.Hkv % p.max_blocks);
    const long long db = stride / p.Hkv / p.max_blocks;
    for (; b < p.B; kvh += dk, i += di, b += db) {
        if (kvh >= p.Hkv) kvh -= p.Hkv, ++i;
        if (i >= p.max_blocks) i -= p.max_blocks, ++b;
        if (b >= p.B) break;
        const Run r = run_of(p, int(b), i, kvh, s_len, gl);
        if (r.n == 0) continue;
        if constexpr (!QUANT) {
            const uint4* s16 = static_cast<const uint4*>(r.src);
            uint4* d16 = static_cast<uint4*>(r.dst);
            const int n16 = int((size_t)r.n * p.D * p.elem / 16);  // rows are a multiple of 16 bytes
            for (int j0 = 0; j0 < n16; j0 += TPR * PW_UNROLL) {
                uint4 v[PW_UNROLL];
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u) {
                    const int j = j0 + u * TPR + gl;
                    if (j < n16) v[u] = __ldcs(s16 + j);
                }
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u) {
                    const int j = j0 + u * TPR + gl;
                    if (j < n16) d16[j] = v[u];
                }
            }
        } else {
            const float4* s4 = static_cast<const float4*>(r.src);
            const int n4 = r.n * p.D / 4;  // D is a multiple of 4
            if constexpr (TPR == 32) {
                if (n4 <= 32 * PW_REG_F4) {
                    // the whole run in registers: one read of the source
                    float4 v[PW_REG_F4];
                    float amax = 0.f;
#pragma unroll
                    for (int u = 0; u < PW_REG_F4; ++u) {
                        const int j = u * 32 + lane;
                        v[u] = j < n4 ? __ldcs(s4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int u = 0; u < PW_REG_F4; ++u)
                        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
                    float m;
                    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(amax));
                    const float scale = m / 127.0f, rcp = finite_rcp(scale);
                    if (lane == 0) p.scales[(size_t)r.blk * p.Hkv + r.kvh] = scale;
                    uint32_t* d4 = static_cast<uint32_t*>(r.dst);
                    int near = scale > 0.f && rcp == 0.f;
#pragma unroll
                    for (int u = 0; u < PW_REG_F4; ++u) {
                        const int j = u * 32 + lane;
                        if (j < n4) d4[j] = scale > 0.f ? quantize4_fast(v[u], rcp, near) : 0u;
                    }
                    if (near) {
#pragma unroll
                        for (int u = 0; u < PW_REG_F4; ++u) {
                            const int j = u * 32 + lane;
                            if (j < n4) d4[j] = quantize4_exact(v[u], scale);
                        }
                    }
                    continue;
                }
            }
            float amax = 0.f;
            for (int j0 = 0; j0 < n4; j0 += TPR * PW_UNROLL) {
                float4 v[PW_UNROLL];
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u) {
                    const int j = j0 + u * TPR + gl;
                    v[u] = j < n4 ? __ldg(s4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u)
                    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
            }
            float m;
            asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(amax));
            if constexpr (TPR > 32) {
                // the CTA's warps agree (two slot sets: a fast warp's next run cannot overwrite this one)
                if (lane == 0) s_max[parity][threadIdx.x >> 5] = m;
                __syncthreads();
#pragma unroll
                for (int w = 0; w < PW_WARPS; ++w) m = fmaxf(m, s_max[parity][w]);
                parity ^= 1;
            }
            const float scale = m / 127.0f, rcp = finite_rcp(scale);
            if (gl == 0) p.scales[(size_t)r.blk * p.Hkv + r.kvh] = scale;
            uint32_t* d4 = static_cast<uint32_t*>(r.dst);
            for (int j0 = 0; j0 < n4; j0 += TPR * PW_UNROLL) {
                float4 v[PW_UNROLL];
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u) {
                    const int j = j0 + u * TPR + gl;
                    v[u] = j < n4 ? __ldcs(s4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                int near = scale > 0.f && rcp == 0.f;
#pragma unroll
                for (int u = 0; u < PW_UNROLL; ++u) {
                    const int j = j0 + u * TPR + gl;
                    if (j < n4) d4[j] = scale > 0.f ? quantize4_fast(v[u], rcp, near) : 0u;
                }
                if (near) {
#pragma unroll
                    for (int u = 0; u < PW_UNROLL; ++u) {
                        const int j = j0 + u * TPR + gl;
                        if (j < n4) d4[j] = quantize4_exact(v[u], scale);
                    }
                }
            }
        }
    }
}

}  // namespace

cudaError_t kvb_launch_page_write(const PageWriteParams& p, bool quantize, cudaStream_t stream) {
    if (p.B == 0 || p.max_blocks == 0 || p.Hkv == 0) return cudaSuccess;
    const long long runs = (long long)p.B * p.max_blocks * p.Hkv;
    const size_t run_bytes = (size_t)p.page * p.D * p.src_elem;
    const bool cta_runs = run_bytes >= (size_t(64) << 10);
    const int groups = cta_runs ? 1 : PW_WARPS;
    const long long ctas = (runs + groups - 1) / groups;
    // CTAs per SM that fit (the warp-per-run quantizer holds a run in registers: about 128 a thread)
    const int per_sm = cta_runs ? 8 : quantize ? 2 : 4;
    const unsigned grid = (unsigned)std::min<long long>(ctas, (long long)p.num_sms * per_sm);
    const size_t smem = p.B <= PW_LENS_MAX ? sizeof(int) * (size_t)p.B : 0;
    if (quantize) {
        if (cta_runs) page_write_kernel<true, PW_THREADS><<<grid, PW_THREADS, smem, stream>>>(p);
        else page_write_kernel<true, 32><<<grid, PW_THREADS, smem, stream>>>(p);
    } else {
        if (cta_runs) page_write_kernel<false, PW_THREADS><<<grid, PW_THREADS, smem, stream>>>(p);
        else page_write_kernel<false, 32><<<grid, PW_THREADS, smem, stream>>>(p);
    }
    return cudaGetLastError();
}
