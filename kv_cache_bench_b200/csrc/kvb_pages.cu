// The page write path in front of decode: a contiguous cache [B][Hkv][max_len][D] written into the
// paged pool [num_blocks][Hkv][page][D] through the block table.
//
//   quantize_pages_i8  src/reference.cpp:32-51 (quantize_to_paged_i8): per (sequence, logical page,
//                      KV head) amax over the page's live tokens and all D, scale = amax / 127 (fp32),
//                      q = clamp(nearbyint(x / scale), -127, 127) with an IEEE fp32 division and
//                      round-half-to-even, 0 when the scale is 0; the scale goes to
//                      scales[block * Hkv + kvh].
//   scatter_pages      src/reference.hpp:60-68 (scatter_to_paged): the live tokens copied unchanged.
//
// Slots past a sequence's last token are not written (as in the reference). One CTA per (page, KV
// head, sequence): the page's live rows are one contiguous run in both layouts, read and written
// with 16-byte vectors. The quantizer reads its run twice (amax, then quantize); the second pass
// hits L1/L2, so HBM sees each input byte once. Bad lengths or block ids skip the page and raise the
// same error bits as the decode kernels.
#include <cuda_fp16.h>

#include "kvb_device.cuh"

namespace {

using namespace kvb_dev;

constexpr int PG_THREADS = 256;

struct PageUnit {
    bool live;
    int t0, n;      // first token and live tokens of the page
    long long blk;  // physical block
};

__device__ __forceinline__ PageUnit page_unit(const PageWriteParams& p, int b, int i, unsigned* flag) {
    PageUnit u{false, 0, 0, 0};
    const int len = __ldg(p.seq_lens + b);
    if (len < 0 || len > p.max_len || (long long)len > (long long)p.max_blocks * p.page) {
        if (i == 0 && threadIdx.x == 0 && flag) raise_error(flag, KVB_DEVERR_LENGTH);
        return u;
    }
    u.t0 = i * p.page;
    if (u.t0 >= len) return u;
    u.n = min(len - u.t0, p.page);
    const int blk = __ldg(p.block_table + (size_t)b * p.max_blocks + i);
    if (blk < 0 || (long long)blk >= p.num_blocks) {
        if (threadIdx.x == 0 && flag) raise_error(flag, KVB_DEVERR_BLOCK);
        return u;
    }
    u.blk = blk;
    u.live = true;
    return u;
}

__global__ void __launch_bounds__(PG_THREADS) quantize_pages_kernel(const PageWriteParams p) {
    const int i = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const PageUnit u = page_unit(p, b, i, p.error_flag);
    if (!u.live) return;
    const float* src = static_cast<const float*>(p.src) + (((size_t)b * p.Hkv + kvh) * p.max_len + u.t0) * p.D;
    int8_t* dst = static_cast<int8_t*>(p.dst) + ((size_t)u.blk * p.Hkv + kvh) * p.page * p.D;
    const int n4 = u.n * p.D / 4;  // D is a multiple of 4
    const float4* s4 = reinterpret_cast<const float4*>(src);

    float amax = 0.f;
    for (int j = threadIdx.x; j < n4; j += PG_THREADS) {
        const float4 x = __ldg(s4 + j);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
    __shared__ float s_max[PG_THREADS / 32];
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(amax));
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = r;
    __syncthreads();
    amax = s_max[0];
#pragma unroll
    for (int w = 1; w < PG_THREADS / 32; ++w) amax = fmaxf(amax, s_max[w]);
    const float scale = amax / 127.0f;
    if (threadIdx.x == 0) p.scales[(size_t)u.blk * p.Hkv + kvh] = scale;

    uint32_t* d4 = reinterpret_cast<uint32_t*>(dst);
    for (int j = threadIdx.x; j < n4; j += PG_THREADS) {
        const float4 x = __ldg(s4 + j);
        uint32_t packed = 0;
        if (scale > 0.f) {
            const float v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float q = fminf(fmaxf(rintf(__fdiv_rn(v[e], scale)), -127.f), 127.f);
                packed |= (uint32_t)(uint8_t)(int8_t)q << (8 * e);
            }
        }
        d4[j] = packed;
    }
}

__global__ void __launch_bounds__(PG_THREADS) scatter_pages_kernel(const PageWriteParams p) {
    const int i = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const PageUnit u = page_unit(p, b, i, p.error_flag);
    if (!u.live) return;
    const size_t row = (size_t)p.D * p.elem;  // bytes per token row (a multiple of 16)
    const uint4* s16 = reinterpret_cast<const uint4*>(static_cast<const char*>(p.src) +
                                                      (((size_t)b * p.Hkv + kvh) * p.max_len + u.t0) * row);
    uint4* d16 = reinterpret_cast<uint4*>(static_cast<char*>(p.dst) + ((size_t)u.blk * p.Hkv + kvh) * p.page * row);
    const int n16 = int((size_t)u.n * row / 16);
    for (int j = threadIdx.x; j < n16; j += PG_THREADS) d16[j] = __ldg(s16 + j);
}

}  // namespace

cudaError_t kvb_launch_page_write(const PageWriteParams& p, bool quantize, cudaStream_t stream) {
    if (p.B == 0 || p.max_blocks == 0 || p.Hkv == 0) return cudaSuccess;
    const dim3 grid((unsigned)p.max_blocks, (unsigned)p.Hkv, (unsigned)p.B);
    if (quantize) quantize_pages_kernel<<<grid, PG_THREADS, 0, stream>>>(p);
    else scatter_pages_kernel<<<grid, PG_THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}
