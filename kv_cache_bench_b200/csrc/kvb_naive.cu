// The naive three-pass baseline on the contiguous cache [B][Hkv][max_len][D] (scores in global
// memory, then softmax, then PV), the streaming read-bandwidth probe, and the cache-flush fill.
//
// Restates src/kernels.metal:150-233 of the reference (naive_scores, naive_softmax, naive_pv,
// read_bw) as plain CUDA; they are its correctness baseline and roofline probe, not a fast path.
#include <cuda_fp16.h>
#include <stdint.h>

#include "kvb_internal.h"

namespace {

template <int KVT>
__device__ __forceinline__ float load_kv(const void* base, size_t i) {
    if constexpr (KVT == 0) return static_cast<const float*>(base)[i];
    else return __half2float(static_cast<const __half*>(base)[i]);
}

// One thread per (t, h, b): scores[b][h][t] = scale * q . k_t   (src/kernels.metal:152-166)
template <int KVT>
__global__ void naive_scores(const float* q, const void* k, const int* seq_lens, float* scores, int H, int Hkv,
                             int D, int max_len, float scale) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (t >= seq_lens[b] || t >= max_len) return;
    const int G = H / Hkv;
    const size_t kb = (((size_t)b * Hkv + h / G) * max_len + t) * D;
    const float* qh = q + ((size_t)b * H + h) * D;
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += qh[d] * load_kv<KVT>(k, kb + d);
    scores[((size_t)b * H + h) * max_len + t] = s * scale;
}

// One block of 256 threads per (h, b): max, exp and sum, normalize, in place
// (src/kernels.metal:168-203). An empty row is left untouched.
__global__ void naive_softmax(float* scores, const int* seq_lens, int H, int max_len) {
    __shared__ float red[256];
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, len = seq_lens[b];
    float* row = scores + ((size_t)b * H + h) * max_len;
    float mx = -1e30f;
    for (int t = tid; t < len; t += 256) mx = fmaxf(mx, row[t]);
    red[tid] = mx;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (tid < s) red[tid] = fmaxf(red[tid], red[tid + s]);
        __syncthreads();
    }
    mx = red[0];
    __syncthreads();
    float sum = 0.f;
    for (int t = tid; t < len; t += 256) {
        const float e = expf(row[t] - mx);
        row[t] = e;
        sum += e;
    }
    red[tid] = sum;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (tid < s) red[tid] += red[tid + s];
        __syncthreads();
    }
    const float inv = 1.f / red[0];
    for (int t = tid; t < len; t += 256) row[t] *= inv;
}

// One thread per (d, h, b): out[b][h][d] = sum_t p_t v_t[d]   (src/kernels.metal:205-218)
template <int KVT>
__global__ void naive_pv(const float* scores, const void* v, const int* seq_lens, float* out, int H, int Hkv, int D,
                         int max_len) {
    const int d = threadIdx.x, h = blockIdx.x, b = blockIdx.y, len = seq_lens[b], G = H / Hkv;
    const float* pr = scores + ((size_t)b * H + h) * max_len;
    const size_t vb = ((size_t)b * Hkv + h / G) * max_len * D + d;
    float o = 0.f;
    for (int t = 0; t < len; ++t) o += pr[t] * load_kv<KVT>(v, vb + (size_t)t * D);
    out[((size_t)b * H + h) * D + d] = o;
}

// Grid-stride streaming read with four independent 16-byte loads in flight per thread; the
// guarded store never happens but keeps the loads alive (src/kernels.metal:223-233).
__global__ void read_bw_kernel(const uint4* __restrict__ src, size_t n16, float* sink) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t acc = 0;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride), c = __ldcs(src + i + 2 * stride),
                    d = __ldcs(src + i + 3 * stride);
        acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n16; i += stride) {
        const uint4 a = __ldcs(src + i);
        acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    if (acc == 0x9e3779b9u) sink[threadIdx.x] = 1.f;
}

// Overwrites a buffer with 16-byte stores (evicts L2 before a cold-cache timing).
__global__ void fill_kernel(uint4* dst, size_t n16, uint32_t value) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const uint4 v = make_uint4(value, value, value, value);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) dst[i] = v;
}

}  // namespace

cudaError_t kvb_launch_naive(const float* q, const void* k, const void* v, const int* seq_lens, float* out,
                             float* scores, int B, int H, int Hkv, int D, int max_len, int kv_type,
                             cudaStream_t stream) {
    if (B == 0) return cudaSuccess;
    const float scale = 1.0f / sqrtf(float(D));
    const dim3 g1((unsigned)((max_len > 0 ? max_len : 1) + 255) / 256, H, B);
    if (kv_type == 0) naive_scores<0><<<g1, 256, 0, stream>>>(q, k, seq_lens, scores, H, Hkv, D, max_len, scale);
    else naive_scores<1><<<g1, 256, 0, stream>>>(q, k, seq_lens, scores, H, Hkv, D, max_len, scale);
    naive_softmax<<<dim3(H, B), 256, 0, stream>>>(scores, seq_lens, H, max_len);
    if (kv_type == 0) naive_pv<0><<<dim3(H, B), D, 0, stream>>>(scores, v, seq_lens, out, H, Hkv, D, max_len);
    else naive_pv<1><<<dim3(H, B), D, 0, stream>>>(scores, v, seq_lens, out, H, Hkv, D, max_len);
    return cudaGetLastError();
}

cudaError_t kvb_launch_read_bw(const void* src, size_t bytes, float* sink, int num_sms, cudaStream_t stream) {
    const size_t n16 = bytes / 16;
    read_bw_kernel<<<num_sms * 8, 256, 0, stream>>>(static_cast<const uint4*>(src), n16, sink);
    return cudaGetLastError();
}

cudaError_t kvb_launch_fill(void* dst, size_t bytes, uint32_t value, int num_sms, cudaStream_t stream) {
    fill_kernel<<<num_sms * 8, 256, 0, stream>>>(static_cast<uint4*>(dst), bytes / 16, value);
    return cudaGetLastError();
}
