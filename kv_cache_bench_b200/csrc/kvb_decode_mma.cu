// Paged split-K decode for fp16 and int8 caches on B200: TMA-staged pages and mma.sync tensor-core
// contractions (page size a power of two from 8 to 256, rows of 128 or 256 bytes, up to 8 query
// heads per KV-head group). It serves the shapes the tcgen05 kernel does not (head dim 64).
//
// Computes what the reference's paged_decode + paged_reduce compute (src/kernels.metal:43-147):
// per (sequence, KV-head group, partition) an fp32 online softmax over the partition's tokens,
// then a weighted merge of the partitions. How it maps onto the B200:
//
// Data movement. A CTA is one producer warp and four consumer warps. The producer walks the
// CTA's work units in order and, for every 64-token chunk, issues 2-D TMA tile loads of the K and
// V rows of each page in the chunk (one box per page, or per 64 rows of a larger page, per 128-byte
// column slice) into a ring of shared-memory stages with 128-byte swizzling, signalling an
// mbarrier by transaction bytes. Block ids and int8 scales for a window of pages are fetched by
// the whole producer warp ahead of use. K/V tiles carry an L2 evict-first policy: they are read
// once, while the block table, scales and split-K partials should stay in L2. The ring
// (96 KB) lets each CTA keep up to 96 KB of loads in flight; two CTAs share an SM.
//
// Math. Each consumer warp takes 16 tokens of each chunk. QK^T and PV run as
// mma.sync.m16n8k16 (fp16 x fp16 -> fp32) with the 16 rows of the A operand holding the group's
// query heads twice: row g holds fp16(x) and row g + 8 holds fp16(x - fp16(x)), so the product
// carries ~22 bits of x, the fp32-level accuracy the reference's 2e-5 tolerance needs. K and V are
// exact in fp16 (fp16 storage, or int8 values before the scale). For QK^T the B operand is K
// itself (tokens x head-dim, head-dim contiguous): ldmatrix for fp16, 8-byte loads plus a byte
// permute for int8. For PV the B operand is V (head-dim contiguous, contracted over tokens):
// ldmatrix.trans for fp16, and for int8 a byte permute that pairs the same column of two token
// rows. The head-dim order inside each fragment is permuted (consistently for q and K, and for V
// and the output) so every shared-memory access is a conflict-free vector load. The S accumulator
// of QK^T is already in the A-operand layout of PV, so probabilities never leave registers.
//
// Softmax. Scores are in log2 units (q is pre-scaled by log2(e)/sqrt(D)); per warp an online
// max/sum per head; the accumulator is rescaled only when a row max grows. int8 scales are applied
// to the scores (k) and folded into the probabilities (v). Tokens outside the partition are
// masked by select; fp16 rows past the partition end are zeroed in shared memory before PV so
// dead pool slots or stale rows cannot inject NaN through 0 * NaN (int8 values are always finite).
//
// Epilogue. The four warp states merge in shared memory; single-partition sequences write the
// output directly, otherwise the partition goes to the workspace and the last CTA to finish a
// (sequence, head group) merges all partitions (kvb_device.cuh).
#include <cuda.h>
#include <cuda_fp16.h>

#include "kvb_device.cuh"

namespace {

using namespace kvb_dev;

constexpr int NCW = 4;                      // consumer warps
constexpr int MMA_THREADS = (NCW + 1) * 32;  // + producer warp
constexpr int SUB_BYTES = KVB_CHUNK * 128;   // one 64-row x 128-byte swizzled tile
constexpr int WIN = 64;                      // pages of block-table metadata per window
constexpr float PV_PRESCALE_I8 = 1024.0f;    // keeps the low fp16 half of p * v_scale normal (int8)

struct StageMeta {
    float ks[KVB_CHUNK / 8];  // K scale per 8-token n-tile (int8)
    float vs[KVB_CHUNK / 8];
    int bad;                  // a block id of this chunk was refused
    int pad[3];
};

template <int KVT, int D>
struct MmaCfg {
    static constexpr int ELEM = KVT == 1 ? 2 : 1;
    static constexpr int NSUB = D * ELEM / 128;  // 128-byte column slices per row
    static constexpr int STAGE_BYTES = 2 * NSUB * SUB_BYTES;
    static constexpr int STAGES = NSUB == 2 ? 3 : 6;
    static constexpr size_t RING = size_t(STAGES) * STAGE_BYTES;
    // shared memory carve-up after the 1024-aligned ring
    static constexpr size_t META_OFF = RING;
    static constexpr size_t BAR_OFF = META_OFF + STAGES * sizeof(StageMeta);
    static constexpr size_t EPI_O_OFF = kvb_align_up(BAR_OFF + 2 * STAGES * sizeof(uint64_t), 16);
    static constexpr size_t EPI_ML_OFF = EPI_O_OFF + sizeof(float) * NCW * KVB_EPI_HEADS * D;
    static constexpr size_t WIN_OFF = EPI_ML_OFF + sizeof(float2) * NCW * KVB_EPI_HEADS;
    static constexpr size_t PREFIX_OFF = WIN_OFF + 3 * sizeof(int) * WIN;
    static constexpr size_t MISC_OFF = PREFIX_OFF + sizeof(int) * (KVB_PREFIX_MAX + 1);
    static constexpr size_t SMEM = MISC_OFF + 64 + 1024;  // + slack for the 1024-byte alignment
};

// Address of byte `byte` of 16-byte chunk `chunk` of row `row` of a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t swz(uint32_t tile, int row, int chunk, int byte) {
    return tile + row * 128 + (((chunk ^ (row & 7)) & 7) << 4) + byte;
}

// Head-dim index of the A/B fragment element (k slot) of mma step s for lane column c4 = lane & 3.
// kk: 0/1 = k slots 2c4, 2c4+1; 2/3 = k slots 2c4+8, 2c4+9.
template <int KVT>
__device__ __forceinline__ int qk_dim(int s, int c4, int kk) {
    if constexpr (KVT == 1) {  // fp16: natural order
        return 16 * s + 2 * c4 + (kk & 1) + (kk >> 1) * 8;
    } else {  // int8: each lane's 8-byte load covers k slots of two steps
        const int pr = s >> 1, e = s & 1;
        const int base = c4 < 2 ? 16 * pr + 8 * c4 : 64 + 16 * pr + 8 * (c4 - 2);
        return base + 4 * e + kk;
    }
}

template <int KVT, int D, int QGM>
__global__ void __launch_bounds__(MMA_THREADS, 2)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      const DecodeParams p) {
    using C = MmaCfg<KVT, D>;
    constexpr int NSUB = C::NSUB, STAGES = C::STAGES;
    constexpr int KSTEPS = D / 16;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    StageMeta* meta = reinterpret_cast<StageMeta*>(smem + C::META_OFF);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + STAGES;
    float* epi_o = reinterpret_cast<float*>(smem + C::EPI_O_OFF);
    float2* epi_ml = reinterpret_cast<float2*>(smem + C::EPI_ML_OFF);
    int* win_blk = reinterpret_cast<int*>(smem + C::WIN_OFF);
    float* win_ks = reinterpret_cast<float*>(win_blk + WIN);
    float* win_vs = win_ks + WIN;
    int* s_prefix = reinterpret_cast<int*>(smem + C::PREFIX_OFF);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF);
    int* s_flag = reinterpret_cast<int*>(smem + C::MISC_OFF + 16);
    const uint32_t ring = smem_u32(smem);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Zero the ring once so rows that are never loaded hold finite values, then set up barriers.
    for (int i = tid; i < int(C::RING / 16); i += MMA_THREADS) sts128_zero(ring + 16 * i);
    fence_proxy_async_smem();  // the zeros must be ordered before the TMA writes
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        *s_abort = 0;
        fence_mbarrier_init();
    }
    if (tid == 32 * NCW) {
        prefetch_tensormap(&tmk);
        prefetch_tensormap(&tmv);
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int* prefix = nullptr;
    if (p.B <= KVB_PREFIX_MAX) {
        build_unit_prefix(p, s_prefix, reinterpret_cast<int*>(epi_o), tid, MMA_THREADS, 1);
        prefix = s_prefix;
    }
    const long long total = unit_total(p, prefix);
    note_counter_count(p);

    if (warp == NCW) {
        // ------------------------------------------------------------------ producer warp
        const uint64_t policy = l2_evict_first_policy();
        UnitCursor cur{&p, prefix, (long long)blockIdx.x, total};
        Unit u;
        int stage = 0;
        uint32_t phase = 0;
        const int box_rows = p.page < KVB_CHUNK ? p.page : KVB_CHUNK;
        const int nbox = KVB_CHUNK / box_rows;
        const int lp = __ffs(p.page) - 1;  // pages are powers of two on this path
        while (cur.advance(u)) {
            if (u.nparts == 0) continue;
            const int* bt = p.block_table + (size_t)u.b * p.max_blocks;
            const int unit_last = (u.t1 - 1) >> lp;  // last page this unit reads
            int w0 = -1;  // first page of the metadata window
            const int c0 = u.t0 / KVB_CHUNK, c1 = (u.t1 + KVB_CHUNK - 1) / KVB_CHUNK;
            for (int c = c0; c < c1; ++c) {
                const int tok0 = c * KVB_CHUNK;
                const int i_first = tok0 >> lp;
                const int i_last = min((tok0 + KVB_CHUNK - 1) >> lp, unit_last);
                if (w0 < 0 || i_first < w0 || i_last >= w0 + WIN) {
                    // Block ids (and int8 scales) of the next WIN pages this unit reads, one page per
                    // lane and pass: every lane's loads are independent, so a window costs about two
                    // memory round trips.
                    __syncwarp();
                    w0 = i_first;
                    const int w_end = min(w0 + WIN, unit_last + 1);
                    int blk[WIN / 32];
#pragma unroll
                    for (int r = 0; r < WIN / 32; ++r) {
                        const int i = w0 + r * 32 + lane;
                        blk[r] = i < w_end ? __ldg(bt + i) : -1;
                    }
#pragma unroll
                    for (int r = 0; r < WIN / 32; ++r) {
                        const int i = w0 + r * 32 + lane;
                        float ks = 0.f, vs = 0.f;
                        if (i < w_end && (blk[r] < 0 || (long long)blk[r] >= p.num_blocks)) {
                            blk[r] = -2;  // refused
                        } else if (KVT == 2 && i < w_end) {
                            ks = __ldg(p.k_scale + (size_t)blk[r] * p.Hkv + u.kvh);
                            vs = __ldg(p.v_scale + (size_t)blk[r] * p.Hkv + u.kvh);
                        }
                        win_blk[r * 32 + lane] = blk[r];
                        win_ks[r * 32 + lane] = ks;
                        win_vs[r * 32 + lane] = vs;
                    }
                    __syncwarp();
                }
                // Lane t < 8 fills the metadata of 8-token group t, lane j < nbox owns box j; lane 0 arms
                // the barrier with the byte count, then every owning lane issues its own tile loads.
                if (lane == 0 && !*s_abort && !mbar_wait_bounded(&empty[stage], phase ^ 1u, s_abort)) {
                    *s_abort = 1;
                    raise_error(p.error_flag, KVB_DEVERR_TIMEOUT);
                }
                __syncwarp();
                StageMeta& m = meta[stage];
                if (lane < KVB_CHUNK / 8) {
                    const int i = (tok0 + 8 * lane) >> lp;
                    const bool live = i <= unit_last;
                    m.ks[lane] = live ? win_ks[i - w0] : 0.f;
                    m.vs[lane] = live ? win_vs[i - w0] : 0.f;
                }
                int blk = -1;
                bool mine = false, refused = false;
                if (lane < nbox) {
                    const int i = (tok0 + lane * box_rows) >> lp;
                    if (i <= unit_last) {
                        blk = win_blk[i - w0];
                        refused = blk < 0;
                        mine = !refused;
                    }
                }
                const unsigned owned = __ballot_sync(0xffffffffu, mine);
                const bool bad = __any_sync(0xffffffffu, refused);
                const uint32_t bytes = uint32_t(__popc(owned)) * 2u * NSUB * box_rows * 128u;
                const bool abort_now = *s_abort;
                if (lane == 0) {
                    m.bad = bad;
                    if (bad) raise_error(p.error_flag, KVB_DEVERR_BLOCK);
                }
                __syncwarp();  // the metadata writes of every lane happen before the arrive below
                if (lane == 0) {
                    if (abort_now || bytes == 0) mbar_arrive(&full[stage]);
                    else mbar_arrive_expect_tx(&full[stage], bytes);
                }
                __syncwarp();
                if (mine && !abort_now) {
                    const int tok = tok0 + lane * box_rows;
                    const int y = (blk * p.Hkv + u.kvh) * p.page + (tok & (p.page - 1));
                    uint8_t* stg = smem + stage * C::STAGE_BYTES;
#pragma unroll
                    for (int sb = 0; sb < NSUB; ++sb) {
                        const int x = sb * (128 / C::ELEM);
                        const uint32_t off = sb * SUB_BYTES + lane * box_rows * 128;
                        tma_load_2d(stg + off, &tmk, &full[stage], x, y, policy);
                        tma_load_2d(stg + NSUB * SUB_BYTES + off, &tmv, &full[stage], x, y, policy);
                    }
                }
                __syncwarp();
                if (++stage == STAGES) stage = 0, phase ^= 1u;
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumer warps
    const int g = lane >> 2, c4 = lane & 3;
    const int r_base = 16 * warp;  // this warp's 16 rows of every chunk
    UnitCursor cur{&p, prefix, (long long)blockIdx.x, total};
    Unit u;
    int stage = 0;
    uint32_t phase = 0;
    while (cur.advance(u)) {
        if (u.nparts == 0) {
            store_tokenless_unit<D>(p, u, tid, NCW * 32);
            continue;
        }
        // q fragments: row g = fp16(x), row g + 8 = fp16(x - fp16(x)) with x = q * q_scale * qpre,
        // qpre a power of two per head that puts max|x| in [2^13, 2^14): no fp16 overflow for any q,
        // and the low half stays a normal fp16 number for all but the tiniest elements.
        uint32_t qa[KSTEPS][4];
        float qpre_inv;
        {
            const float* qrow = p.q + ((size_t)u.b * p.H + u.h0 + g) * D;
            float x[KSTEPS][4];
            float amax = 0.f;
#pragma unroll
            for (int s = 0; s < KSTEPS; ++s)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    x[s][kk] = g < u.nh ? __ldg(qrow + qk_dim<KVT>(s, c4, kk)) * p.q_scale : 0.f;
                    amax = fmaxf(amax, fabsf(x[s][kk]));
                }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            int e = 0;
            frexpf(amax, &e);
            const float qpre = amax > 0.f && amax < 3.0e38f ? ldexpf(1.f, 14 - e) : 1.f;
            qpre_inv = 1.f / qpre;
#pragma unroll
            for (int s = 0; s < KSTEPS; ++s) {
                split_hi_lo(x[s][0] * qpre, x[s][1] * qpre, qa[s][0], qa[s][1]);
                split_hi_lo(x[s][2] * qpre, x[s][3] * qpre, qa[s][2], qa[s][3]);
            }
        }
        // int8: probabilities carry v_scale * pvs into the fp16 split; pvs is a power of two that
        // starts at PV_PRESCALE_I8 and only shrinks, when a chunk's V scales would push p * v_scale *
        // pvs past 2^14 (the accumulator is rescaled by the same exact factor).
        float pvs = KVT == 2 ? PV_PRESCALE_I8 : 1.f;
        float o[D / 8][4];
#pragma unroll
        for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        float m = NEG_BIG, l = 0.f;
        int bad = 0;

        const int c0 = u.t0 / KVB_CHUNK, c1 = (u.t1 + KVB_CHUNK - 1) / KVB_CHUNK;
        for (int c = c0; c < c1; ++c) {
            if (!mbar_wait_bounded(&full[stage], phase, s_abort)) {
                if (lane == 0) {
                    *s_abort = 1;
                    raise_error(p.error_flag, KVB_DEVERR_TIMEOUT);
                }
            }
            const uint32_t kt = ring + stage * C::STAGE_BYTES;  // K tiles, then V tiles
            const uint32_t vt = kt + NSUB * SUB_BYTES;
            const StageMeta& md = meta[stage];
            bad |= md.bad;
            const int tok_w = c * KVB_CHUNK + r_base;  // token of this warp's first row
            const bool any = tok_w < u.t1 && tok_w + 16 > u.t0;
            bool zeroed = false;
            if (any) {
                // ---- S = Q K^T for the warp's two 8-token n-tiles
                float sacc[2][4];
#pragma unroll
                for (int t2 = 0; t2 < 2; ++t2) {
                    sacc[t2][0] = sacc[t2][1] = sacc[t2][2] = sacc[t2][3] = 0.f;
                    const int r0 = r_base + 8 * t2;
#pragma unroll
                    for (int sp = 0; sp < KSTEPS / 2; ++sp) {
                        uint32_t b0a, b1a, b0b, b1b;
                        if constexpr (KVT == 1) {
                            const int mi = lane >> 3, row = r0 + (lane & 7);
                            const int byte = 2 * (32 * sp + 8 * mi);
                            ldsm_x4(swz(kt + (byte >> 7) * SUB_BYTES, row, (byte & 127) >> 4, 0), b0a, b1a, b0b, b1b);
                        } else {
                            const int row = r0 + g;
                            const int ch = c4 < 2 ? sp : sp + 4;
                            uint32_t w0, w1;
                            lds64(swz(kt, row, ch, 8 * (c4 & 1)), w0, w1);
                            w0 ^= 0x80808080u;
                            w1 ^= 0x80808080u;
                            b0a = i8pair_to_h2(w0, SEL_B01);
                            b1a = i8pair_to_h2(w0, SEL_B23);
                            b0b = i8pair_to_h2(w1, SEL_B01);
                            b1b = i8pair_to_h2(w1, SEL_B23);
                        }
                        mma_16816(sacc[t2], qa[2 * sp], b0a, b1a);
                        mma_16816(sacc[t2], qa[2 * sp + 1], b0b, b1b);
                    }
                }
                // ---- scores, online softmax
                float sc[2][2];
                float mx = m;
#pragma unroll
                for (int t2 = 0; t2 < 2; ++t2) {
                    const float ks = (KVT == 2 ? md.ks[2 * warp + t2] : 1.f) * qpre_inv;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int tok = tok_w + 8 * t2 + 2 * c4 + e;
                        const bool valid = tok >= u.t0 && tok < u.t1 && g < u.nh;
                        sc[t2][e] = valid ? (sacc[t2][e] + sacc[t2][e + 2]) * ks : NEG_BIG;
                        mx = fmaxf(mx, sc[t2][e]);
                    }
                }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                if (__any_sync(0xffffffffu, mx > m)) {
                    const float corr = exp2f(m - mx);
                    l *= corr;
#pragma unroll
                    for (int j = 0; j < D / 8; ++j) {
                        o[j][0] *= corr;
                        o[j][1] *= corr;
                        o[j][2] *= corr;
                        o[j][3] *= corr;
                    }
                    m = mx;
                }
                if constexpr (KVT == 2) {
                    const float vmax = fmaxf(md.vs[2 * warp], md.vs[2 * warp + 1]);
                    if (vmax * pvs > 16384.f) {  // warp-uniform: every lane reads the same scales
                        int e = 0;
                        frexpf(vmax, &e);
                        const float npvs = ldexpf(1.f, 14 - e);
                        const float r = npvs / pvs;
#pragma unroll
                        for (int j = 0; j < D / 8; ++j) {
                            o[j][0] *= r;
                            o[j][1] *= r;
                            o[j][2] *= r;
                            o[j][3] *= r;
                        }
                        pvs = npvs;
                    }
                }
                uint32_t pa[4];
#pragma unroll
                for (int t2 = 0; t2 < 2; ++t2) {
                    const float vs = KVT == 2 ? md.vs[2 * warp + t2] * pvs : 1.f;
                    float pv[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float pr = sc[t2][e] > 0.5f * NEG_BIG ? exp2f(sc[t2][e] - m) : 0.f;
                        l += pr;
                        pv[e] = pr * vs;
                    }
                    split_hi_lo(pv[0], pv[1], pa[2 * t2], pa[2 * t2 + 1]);
                }
                // ---- fp16 rows past the partition end (dead pool slots, or pages this unit did not
                // load, which hold stale data): zero them before they meet p = 0
                if (KVT == 1 && tok_w + 16 > u.t1) {
                    const int first = max(0, u.t1 - tok_w);
                    for (int idx = lane; idx < (16 - first) * 8 * NSUB; idx += 32) {
                        const int row = r_base + first + idx / (8 * NSUB);
                        const int rest = idx % (8 * NSUB);
                        sts128_zero(vt + (rest >> 3) * SUB_BYTES + row * 128 + (rest & 7) * 16);
                    }
                    zeroed = true;
                    __syncwarp();
                }
                // ---- O += P V
                if constexpr (KVT == 1) {
#pragma unroll
                    for (int jp = 0; jp < D / 16; ++jp) {
                        const int mi = lane >> 3;
                        const int row = r_base + (mi & 1) * 8 + (lane & 7);
                        const int byte = 2 * (16 * jp + 8 * (mi >> 1));
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_trans(swz(vt + (byte >> 7) * SUB_BYTES, row, (byte & 127) >> 4, 0), b0, b1, b2, b3);
                        mma_16816(o[2 * jp], pa, b0, b1);
                        mma_16816(o[2 * jp + 1], pa, b2, b3);
                    }
                } else {
#pragma unroll
                    for (int a = 0; a < D / 32; ++a) {
                        const int ch = 2 * a + (g >> 2), byte = 4 * (g & 3);
                        const int r = r_base + 2 * c4;
                        const uint32_t w0 = lds32(swz(vt, r, ch, byte));
                        const uint32_t w1 = lds32(swz(vt, r + 1, ch, byte));
                        const uint32_t w2 = lds32(swz(vt, r + 8, ch, byte));
                        const uint32_t w3 = lds32(swz(vt, r + 9, ch, byte));
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            mma_16816(o[4 * a + i], pa, i8cross_to_h2(w0, w1, i), i8cross_to_h2(w2, w3, i));
                    }
                }
            }
            if (zeroed) fence_proxy_async_smem();  // generic writes before the next TMA write
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == STAGES) stage = 0, phase ^= 1u;
        }

        // ---- epilogue: merge the four warps, then the partitions
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        // Also the barrier after which the previous unit's epilogue buffers are free.
        const int unit_bad = named_barrier_or(1, NCW * 32, bad);
        // Warps may end with different pvs: fold 1 / pvs into each warp's accumulator before the merge.
        const float o_scale = unit_bad ? __int_as_float(0x7fc00000) : 1.0f;
        const float o_unscale = 1.0f / pvs;
        for (int g0 = 0; g0 < u.nh; g0 += KVB_EPI_HEADS) {
            if (g0 > 0) named_barrier(1, NCW * 32);
            const int gg = g - g0;
            if (gg >= 0 && gg < KVB_EPI_HEADS) {
                float* dst = epi_o + (warp * KVB_EPI_HEADS + gg) * D;
#pragma unroll
                for (int j = 0; j < D / 8; ++j) {
                    int d0, d1;
                    if constexpr (KVT == 1) {
                        d0 = 8 * j + 2 * c4;
                        d1 = d0 + 1;
                    } else {
                        d0 = 32 * (j >> 2) + 8 * c4 + (j & 3);
                        d1 = d0 + 4;
                    }
                    dst[d0] = (o[j][0] + o[j][2]) * o_unscale;
                    dst[d1] = (o[j][1] + o[j][3]) * o_unscale;
                }
                if (c4 == 0) epi_ml[warp * KVB_EPI_HEADS + gg] = make_float2(m, l);
            }
            named_barrier(1, NCW * 32);
            merge_slots_and_store<D>(p, u, epi_o, epi_ml, NCW, g0, min(KVB_EPI_HEADS, u.nh - g0), o_scale, tid,
                                     NCW * 32);
        }
        finish_partition<D>(p, u, tid, NCW * 32, 1, s_flag);
        named_barrier(1, NCW * 32);
    }
}

template <int KVT, int D, int QGM>
cudaError_t launch_one(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, const LaunchInfo& li) {
    using C = MmaCfg<KVT, D>;
    static KvbPerDevice<int> per_device;  // the shared-memory attribute and occupancy, per device
    int blocks_per_sm = 0;
    const cudaError_t e = per_device.get(&blocks_per_sm, [](int* n) {
        cudaError_t r = cudaFuncSetAttribute(decode_mma_kernel<KVT, D, QGM>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::SMEM));
        if (r != cudaSuccess) return r;
        r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, decode_mma_kernel<KVT, D, QGM>, MMA_THREADS, C::SMEM);
        if (*n < 1) *n = 1;
        return r;
    });
    if (e != cudaSuccess) return e;
    const long long upper = (long long)p.B * p.nhg * p.max_parts;
    const long long grid = std::min<long long>(upper, (long long)li.num_sms * blocks_per_sm);
    if (grid <= 0) return cudaSuccess;
    return kvb_launch_pdl(decode_mma_kernel<KVT, D, QGM>, (unsigned)grid, MMA_THREADS, C::SMEM, li.stream, tk, tv, p);
}

template <int KVT, int D>
cudaError_t launch_qg(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, const LaunchInfo& li) {
    if (p.qg <= 1) return launch_one<KVT, D, 1>(p, tk, tv, li);
    if (p.qg <= 2) return launch_one<KVT, D, 2>(p, tk, tv, li);
    if (p.qg <= 4) return launch_one<KVT, D, 4>(p, tk, tv, li);
    return launch_one<KVT, D, 8>(p, tk, tv, li);
}

}  // namespace

bool kvb_mma_supported(int kv_type, int D, int page, int qg) {
    const int row_bytes = D * (kv_type == 1 ? 2 : 1);
    if (kv_type != 1 && kv_type != 2) return false;
    if (row_bytes != 128 && row_bytes != 256) return false;
    if (page < 8 || page > 256 || (page & (page - 1)) != 0) return false;  // 8, 16, ..., 256
    return qg >= 1 && qg <= 8;
}

cudaError_t kvb_launch_decode_mma(const DecodeParams& p, int kv_type, int D, const void* tmap_k, const void* tmap_v,
                                  const LaunchInfo& li) {
    const CUtensorMap& tk = *static_cast<const CUtensorMap*>(tmap_k);
    const CUtensorMap& tv = *static_cast<const CUtensorMap*>(tmap_v);
    if (kv_type == 1) return D == 64 ? launch_qg<1, 64>(p, tk, tv, li) : launch_qg<1, 128>(p, tk, tv, li);
    return launch_qg<2, 128>(p, tk, tv, li);
}
