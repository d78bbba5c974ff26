// Paged split-K decode on B200 with tcgen05 (UMMA) tensor cores, TMA and tensor memory.
//
// Computes what the reference's paged_decode + paged_reduce compute (src/kernels.metal:43-147):
// per (sequence, KV-head group, partition) an fp32-accurate online softmax over the partition's
// tokens, then a weighted merge of the partitions. Shapes: head dim 128, fp16 or int8 pools, page
// size 8, 16, 32, 64, 128 or 256, up to 8 query heads per KV-head group.
//
// One CTA per SM, warp-specialized (12 warps in three warpgroups; the control warpgroup hands
// registers to the two softmax warpgroups with setmaxnreg):
//   warps 0-7   two softmax groups of 4 warps (below).
//   warp 8      TMA producer: reads the unit's block ids (and int8 scales) once into a shared-memory
//               page table, then for each 128-token chunk issues 2-D tile loads of the K and V rows
//               of every page in the chunk (128-byte swizzle) into a ring of shared-memory stages.
//   warps 9, 10 MMA issuers (one thread each), for the even and the odd chunks of the running chunk
//               index:
//                 S^T[128 tokens x N] = K[128 x 128] . Qhat^T[128 x N]      (tensor memory)
//                 O^T[128 dims x N]   = V^T[128 x 128 tokens] . Phat^T       (tensor memory)
//               reading K (K-major) and V (MN-major, the transposed view of the same TMA tile)
//               straight from the stage. tcgen05.commit releases the stage and signals the softmax.
//   warps 0-7   two softmax groups of 4 warps (128 threads, one per tensor-memory lane), group g for
//               the chunks of parity g: thread t reads token t's scores, the four warps agree on the
//               chunk max per head, write Phat^T to shared memory, and after the PV product thread d
//               folds O^T row d into registers. The groups merge once per unit.
//
// Exactness. The operands are exact in the MMA's input type, so the contraction is exact up to the
// accumulator:
//   int8 (kind::i8, int32 accumulate): K and V are the stored int8 values. q (per head) and the
//     probabilities (per chunk) are integers below 2^30 written as four signed 8-bit limbs,
//     x = ((l0*256 + l1)*256 + l2)*256 + l3, so S and O come out as four exact int32 partial
//     products recombined in fp32. The int8 scales are applied outside the MMA: k_scale to the
//     scores, v_scale folded into the probability integers (relative to the unit's largest scale).
//   fp16 (kind::f16, fp32 accumulate): K and V are the stored halves; q and p are split as
//     fp16(x) + fp16(x - fp16(x)) (about 22 significant bits), q prescaled per head by a power of two.
// N = (limbs or halves) x (query heads, padded): int8 4 x {1,2,4,8} -> 8..32, fp16 2 x {4,8} -> 8, 16.
#include <cuda.h>
#include <cuda_fp16.h>

#include "kvb_device.cuh"

namespace {

using namespace kvb_dev;

constexpr int UM_CHUNK = 128;         // tokens per stage = MMA M for QK^T
constexpr int UM_WARPS = 12;          // 8 softmax, producer, MMA (even chunks), MMA (odd chunks), TMEM owner
constexpr int UM_THREADS = UM_WARPS * 32;
constexpr int UM_PRODUCER = 8, UM_MMA0 = 9, UM_MMA1 = 10, UM_TMEM_WARP = 11;  // warp 11 also prepares Qhat
// Registers per thread after the split (the launch gives every thread 168: 65536 / 384, rounded
// down to 8). The control warpgroup keeps 88, the softmax warpgroups get 208; the shares add up to at
// most the launch's total, or setmaxnreg.inc would wait forever.
constexpr int UM_REGS_LAUNCH = 168, UM_REGS_CTRL = 88, UM_REGS_SOFT = 208;
static_assert(2 * 128 * UM_REGS_SOFT + 128 * UM_REGS_CTRL <= UM_THREADS * UM_REGS_LAUNCH, "register split");
constexpr int UM_SOFT = 128;          // threads of one softmax group
constexpr int UM_D = 128;             // head dim
constexpr int TILE = UM_CHUNK * 128;  // bytes of one [128 rows][128 B] swizzled tile
constexpr int UM_PT = 264;            // page-table entries: pages of one partition, at most
constexpr int UM_UCH = 64;            // chunks of one partition, at most (partitions <= 8064 tokens; the
                                      // int8 O^T accumulator sums at most 64 chunks below 2^22 per limb)
constexpr int UM_GRED = 144;          // reduction floats per softmax group
constexpr int UM_TMEM_COLS = 256;     // tensor-memory columns of the CTA
constexpr int UM_XCOL = 128;          // first column of the groups' unit shares
constexpr int UM_QBATCH = 4;          // query heads the Qhat warp loads at once
constexpr int UM_RQ = 8;              // entries of the unit ring (producer -> MMA issuers, Qhat warp)

// ---- tcgen05 wrappers -----------------------------------------------------------------------------

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

template <int KIND>  // 1: kind::f16, 2: kind::i8
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (KIND == 1) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Warpgroup register split (all four warps of a warpgroup execute the same one).
template <int N>
__device__ __forceinline__ void reg_alloc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void reg_dealloc() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 8 consecutive 32-bit tensor-memory columns of this thread's lane.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor. Layout (swizzling mode): SWZ_128B, atoms of 8 rows of 128 B
// (1024 B); SWZ_32B, atoms of 8 rows of 32 B (256 B). lbo / sbo in bytes (leading: stride between the
// swizzle-width column groups of an MN-major operand; stride: between 8-row groups).
constexpr uint64_t SWZ_128B = 2, SWZ_32B = 6;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t layout = SWZ_128B) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= layout << 61;
    return d;
}

// Phat^T (the PV product's B operand) is MN-major with the 32-byte swizzle: token t's row holds its
// N probability values (int8 limbs or fp16 halves, in MMA column order) as 32 contiguous bytes at
// byte 32 t, the two 16-byte halves exchanged for tokens with bit 2 set (address bit 4 XOR bit 7).
// A thread writes its whole row with one or two vector stores. WORDS: 32-bit words written (1 .. 8).
template <int WORDS>
__device__ __forceinline__ void store_p_row(uint8_t* pbuf, int t, const uint32_t (&w)[WORDS]) {
    uint8_t* row = pbuf + 32 * t;
    const int x = ((t >> 2) & 1) * 16;
    if constexpr (WORDS == 8) {
        *reinterpret_cast<uint4*>(row + x) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(row + (16 ^ x)) = make_uint4(w[4], w[5], w[6], w[7]);
    } else if constexpr (WORDS == 4) {
        *reinterpret_cast<uint4*>(row + x) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if constexpr (WORDS == 2) {
        *reinterpret_cast<uint2*>(row + x) = make_uint2(w[0], w[1]);
    } else {
        *reinterpret_cast<uint32_t*>(row + x) = w[0];
    }
}

// Instruction descriptor: D format (1 = f32, 2 = s32), A and B format (kind::f16: 0 = f16; kind::i8:
// 0 = unsigned, 1 = signed 8-bit), A/B major (0 = K-major, 1 = MN-major), N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, uint32_t a_mn,
                                                  uint32_t b_mn, uint32_t N, uint32_t M) {
    return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) |
           ((M >> 4) << 24);
}

// Byte offset of (row, byte column) in a [rows][128 B] tile with the 128-byte swizzle (1024-aligned).
__device__ __forceinline__ uint32_t swz_off(int row, int col) {
    return row * 128 + ((((col >> 4) ^ row) & 7) << 4) + (col & 15);
}

// Exact float of an integer |x| < 2^22 with two full-rate instructions (1.5 * 2^23 has a unit ulp)
// instead of a conversion. The int32 limb products of one chunk stay below 2^22: 128 terms of at
// most 128 * 128 (QK^T: int8 K times signed q limbs) or 128 * 255 (PV: int8 V times probability
// bytes).
__device__ __forceinline__ float small_int_to_float(int x) {
    return __int_as_float(x + 0x4B400000) - 12582912.0f;
}

// Four int32 limb products (high first) recombined: ((r0 * 256 + r1) * 256 + r2) * 256 + r3.
__device__ __forceinline__ float limbs_to_float(uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    return ((small_int_to_float(int(r0)) * 256.f + small_int_to_float(int(r1))) * 256.f +
            small_int_to_float(int(r2))) * 256.f + small_int_to_float(int(r3));
}

// The same recombination for limb sums of any int32 value (the int8 O^T accumulator sums up to 64
// chunks: below 2^28 per limb), with conversions.
__device__ __forceinline__ float limbs_to_float_wide(uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    return ((__int2float_rn(int(r0)) * 256.f + __int2float_rn(int(r1))) * 256.f + __int2float_rn(int(r2))) * 256.f +
           __int2float_rn(int(r3));
}

__device__ __forceinline__ float max4(float4 v) { return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)); }

// Largest value among the 32 lanes of the warp (redux.sync on floats, sm_100a).
__device__ __forceinline__ float warp_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

template <int KVT>
struct UCfg {
    static constexpr int NSUB = KVT == 1 ? 2 : 1;             // 128-byte column slices of a row
    static constexpr int STAGE = 2 * NSUB * TILE;              // K tiles, then V tiles
    static constexpr int STAGES = KVT == 1 ? 3 : 6;
    static constexpr int NMAX = KVT == 1 ? 16 : 32;            // MMA N (rows of Qhat / Phat)
    static constexpr int QBUF = NMAX * 128 * NSUB;             // one Qhat^T buffer ([N][128 B] per slice)
    static constexpr int PBUF = NMAX * 128 * NSUB;             // one Phat^T buffer
    static constexpr size_t RING = size_t(STAGES) * STAGE;
    static constexpr size_t Q_OFF = RING;                      // 2 Qhat buffers (1024-aligned)
    static constexpr size_t P_OFF = Q_OFF + 2 * QBUF;          // 2 Phat buffers
    static constexpr size_t BAD_OFF = P_OFF + 2 * PBUF;        // [STAGES] a block id of the chunk was refused
    // int8: the largest V scale of a unit's pages, [2 units]
    static constexpr size_t VSMAX_OFF = BAD_OFF + STAGES * sizeof(int);
    static constexpr size_t BAR_OFF = kvb_align_up(VSMAX_OFF + (KVT == 2 ? 2 : 0) * sizeof(float), 64);
    // full per (stage, chunk parity); empty per stage; q_full, q_free, s_full, s_free, p_full,
    // pt_free x2; r_full, r_empty x UM_RQ (the O^T products complete on the stage's empty barrier)
    // unit ring: full and empty per entry
    static constexpr int NBARS = 3 * STAGES + 2 * 6 + 2 * UM_RQ;
    static constexpr size_t RED_OFF = kvb_align_up(BAR_OFF + NBARS * sizeof(uint64_t), 16);
    static constexpr size_t WIN_OFF = RED_OFF + 2 * UM_GRED * sizeof(float);
    // page table: block ids [UM_PT]; int8: scales [2 buffers][UM_PT] for K and for V
    static constexpr size_t PT_BYTES = sizeof(int) * UM_PT * (KVT == 2 ? 5 : 1);
    static constexpr size_t PREFIX_OFF = WIN_OFF + PT_BYTES;
    static constexpr size_t LENS_OFF = PREFIX_OFF + sizeof(int) * (KVB_PREFIX_MAX + 1);
    static constexpr size_t SCRATCH_OFF = kvb_align_up(LENS_OFF + sizeof(int) * KVB_PREFIX_MAX, 16);
    static constexpr size_t SCRATCH_FLOATS = 512;              // prefix scan
    static constexpr size_t MISC_OFF = kvb_align_up(SCRATCH_OFF + SCRATCH_FLOATS * sizeof(float), 64);
    // Two unit slots (a unit's slot is its index among the CTA's units with tokens, mod 2): the unit
    // and its per-head score factors (written by the Qhat warp); per group, the m, L and refusal flag
    // of the group's share of the unit; the count of groups done with the unit; per group, the split-K
    // arrival flag.
    static constexpr size_t SLOT_UNIT_OFF = MISC_OFF + 64;                    // [2] Unit (64 B each)
    static constexpr size_t SLOT_QS_OFF = SLOT_UNIT_OFF + 2 * 64;             // [2][8] float
    static constexpr size_t XML_OFF = SLOT_QS_OFF + 2 * 8 * sizeof(float);    // [2 slots][2 groups][24] float
    static constexpr size_t XCNT_OFF = XML_OFF + 2 * 2 * 24 * sizeof(float);  // [2] int count, [2] int flags
    static constexpr size_t RING_OFF = XCNT_OFF + 16;                         // [UM_RQ] decoded units (64 B)
    static constexpr size_t RESTART_OFF = RING_OFF + UM_RQ * 64;              // [2] int8 PV restarts O^T
    static constexpr size_t SMEM = RESTART_OFF + 2 * sizeof(int) + 1024;
};

static_assert(UCfg<1>::SMEM <= 227 * 1024 && UCfg<2>::SMEM <= 227 * 1024, "shared memory budget");
static_assert(UCfg<1>::BAR_OFF % 64 == 0 && UCfg<2>::BAR_OFF % 64 == 0, "mbarrier alignment");
static_assert(UCfg<1>::MISC_OFF % 64 == 0 && UCfg<2>::MISC_OFF % 64 == 0, "alignment");
static_assert(UCfg<1>::Q_OFF % 1024 == 0 && UCfg<1>::P_OFF % 1024 == 0 && UCfg<2>::P_OFF % 1024 == 0,
              "swizzled operands need 1024-byte alignment");
static_assert(UCfg<2>::SCRATCH_FLOATS >= UM_THREADS, "prefix scan scratch");
static_assert(UM_THREADS >= KVB_PREFIX_MAX, "one thread per sequence in the unit prefix");
static_assert(sizeof(Unit) <= 64, "unit slot");

// QGP: query heads per group, padded to 1, 2, 4 or 8. MULTI: the launch may have more units than CTAs
// (dynamic hand-out from the workspace's work counter, units packed by a prefix over the sequences'
// partition counts); without it every CTA takes at most its one unit, dense slot blockIdx.x
// (sequence, head group, partition < max_parts; a slot past its sequence's partitions is empty), and
// the code of the hand-out and the prefix (about 14 KB of a 90 KB kernel) is left out, which keeps
// more of the kernel in the SM's instruction cache.
template <int KVT, int QGP, bool MULTI>
__global__ void __launch_bounds__(UM_THREADS, 1)
    decode_umma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                       const __grid_constant__ DecodeParams p) {
    using C = UCfg<KVT>;
    constexpr int NSUB = C::NSUB, STAGES = C::STAGES;
    constexpr int qgp = QGP;
    constexpr int RPH = KVT == 1 ? 2 : 4;  // rows of Qhat/Phat per head (halves or limbs)
    constexpr int N = RPH * qgp < 8 ? 8 : RPH * qgp;  // MMA N
    // The PV product reads Phat^T MN-major, whose rows it takes in 16-byte units: an int8 row of 8
    // values is padded to 16 (zero bytes, never written; the extra O^T columns are never read).
    constexpr int NPV = (KVT == 2 && N < 16) ? 16 : N;
    // Probabilities are exp2(score - m) <= 2^kTau (lazy re-referencing). int8: p * v_scale / (largest
    // v_scale of the unit) * kPScale is an integer below 2^30; kPUnit = 1 / kPScale.
    constexpr float kTau = KVT == 1 ? 8.f : 2.f;
    constexpr float kPScale = 268435456.f;          // 2^28 = 2^(30 - kTau) for int8
    constexpr float kPUnit = 3.7252902984619141e-09f;  // 2^-28

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    int* stage_bad = reinterpret_cast<int*>(smem + C::BAD_OFF);
    float* unit_vsmax = reinterpret_cast<float*>(smem + C::VSMAX_OFF);  // int8: [2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    // Chunk k (running index over the CTA's units) lives in stage k % STAGES and is announced on
    // full[k % (2 * STAGES)]: a stage alternates between even and odd chunks, whose consumers (MMA
    // warp and softmax group of that parity) each wait on their own barrier in chunk order, so a
    // parity wait never matches a phase two uses old.
    uint64_t* full = bars;
    uint64_t* empty = bars + 2 * STAGES;
    uint64_t* q_full = bars + 3 * STAGES;  // [2] Qhat^T and the unit slot written (Qhat warp -> MMA, softmax)
    uint64_t* q_free = q_full + 2;         // [2] the unit's QK^T products and both groups' shares done
    uint64_t* s_full = q_full + 4;         // [2] S^T ready (MMA -> softmax), one per chunk parity
    uint64_t* s_free = q_full + 6;         // [2] S^T read (softmax -> MMA)
    uint64_t* p_full = q_full + 8;         // [2] Phat^T written, previous O^T folded (softmax -> MMA)
    // A chunk's O^T product completes on its stage's empty barrier, which the softmax group of the
    // chunk waits on as well (stage k % STAGES, phase k / STAGES: only that group's later chunks
    // move it on).
    uint64_t* pt_free = q_full + 10;       // [2] int8 scale buffer read (softmax -> producer)
    uint64_t* r_full = q_full + 12;        // [UM_RQ] unit ring entry written (producer -> consumers)
    uint64_t* r_empty = r_full + UM_RQ;    // [UM_RQ] unit ring entry read (MMA issuers, Qhat warp)
    auto ring_at = [&](int e) -> Unit& { return *reinterpret_cast<Unit*>(smem + C::RING_OFF + 64 * e); };
    volatile int* p_restart = reinterpret_cast<volatile int*>(smem + C::RESTART_OFF);
    float* red = reinterpret_cast<float*>(smem + C::RED_OFF);
    int* pt_blk = reinterpret_cast<int*>(smem + C::WIN_OFF);
    float* pt_ks = reinterpret_cast<float*>(pt_blk + UM_PT);  // int8 only: [2][UM_PT]
    float* pt_vs = pt_ks + 2 * UM_PT;                         // int8 only: [2][UM_PT]
    int* s_prefix = reinterpret_cast<int*>(smem + C::PREFIX_OFF);
    int* s_lens = reinterpret_cast<int*>(smem + C::LENS_OFF);
    float* scratch = reinterpret_cast<float*>(smem + C::SCRATCH_OFF);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF);
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF + 16);
    auto slot_unit = [&](int qb) { return reinterpret_cast<Unit*>(smem + C::SLOT_UNIT_OFF + 64 * qb); };
    float* s_qs = reinterpret_cast<float*>(smem + C::SLOT_QS_OFF);  // [slot][8] score factors
    float* s_xml = reinterpret_cast<float*>(smem + C::XML_OFF);     // [slot][group][24]: m, L, refused
    int* s_xcnt = reinterpret_cast<int*>(smem + C::XCNT_OFF);       // [slot] groups done, [group] flag

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lp = __ffs(p.page) - 1;  // pages are powers of two on this path
    // With tables_ready the lengths and the block table are not written by the kernel before this
    // one, so the unit enumeration and the producer's first block ids are read while that kernel
    // finishes, and their reads start here, ahead of the setup.
    const bool early = p.tables_ready != 0;
    // The unit enumeration starts with the sequence lengths (prefix mode: thread b reads length b)
    // and the block table: have them on the way while the CTA sets up (the table cooperatively
    // across CTAs, when it is small).
    int my_len = 0;
    if (MULTI && tid < p.B && tid < KVB_PREFIX_MAX) {
        if (early) my_len = __ldg(p.seq_lens + tid);
        else prefetch_l2(p.seq_lens + tid);
    }
    // The producer also guesses its first unit before the lengths arrive: unit blockIdx.x of the
    // dense numbering (max_parts partitions for every sequence), which is the first unit of a launch
    // without MULTI (when it exists), and otherwise whenever every sequence before it has max_parts
    // partitions (a single sequence of max_len tokens, for one). It reads the guessed unit's block
    // ids (up to 64 pages) at once, and uses them if the decoded first unit is the guessed one.
    int g_b = -1, g_hg = 0, g_part = 0, g_npg = 0;
    int g_ids[2] = {0, 0};
    if (early && warp == UM_PRODUCER && (long long)blockIdx.x < (long long)p.B * p.div_seq.d) {
        g_b = kvb_div(int(blockIdx.x), p.div_seq);
        const int rem = int(blockIdx.x) - g_b * int(p.div_seq.d);
        g_hg = kvb_div(rem, p.div_parts);
        g_part = rem - g_hg * p.max_parts;
        const int t0 = g_part * p.part_tokens;  // below max_len, as g_part < max_parts
        const int t1 = min(p.max_len, t0 + p.part_tokens);
        const int pg0 = t0 >> lp;
        const int npg = min(((t1 - 1) >> lp) - pg0 + 1, p.max_blocks - pg0);
        if (npg > 0 && npg <= 64) {
            g_npg = npg;
            const int* bt = p.block_table + (size_t)g_b * p.max_blocks + pg0;
            if (lane < npg) g_ids[0] = __ldg(bt + lane);
            if (lane + 32 < npg) g_ids[1] = __ldg(bt + lane + 32);
        }
    }
    {
        const size_t tb = (size_t)p.B * p.max_blocks * sizeof(int);
        const size_t off0 = ((size_t)blockIdx.x * UM_THREADS + tid) * 128, step = (size_t)gridDim.x * UM_THREADS * 128;
        auto table_to_l2 = [&](size_t off) { prefetch_l2(reinterpret_cast<const char*>(p.block_table) + off); };
        // the loops here and below are kept rolled in the single-unit instance (less code; the
        // many-unit instance keeps the compiler's choice, which measured faster there)
        if (tb <= (size_t(256) << 10)) {
            if constexpr (MULTI) {
                for (size_t off = off0; off < tb; off += step) table_to_l2(off);
            } else {
#pragma unroll 1
                for (size_t off = off0; off < tb; off += step) table_to_l2(off);
            }
        }
    }

    // Barriers and tensor memory. The ring is not cleared: rows a chunk does not load are either
    // masked (K: the token's score is not used) or multiplied by an exactly zero probability (int8
    // V) or cleared by the softmax before the PV product (fp16 V, where 0 * NaN would not be 0).
    if constexpr (MULTI) {
        for (int i = tid; i < int((2 * C::QBUF + 2 * C::PBUF) / 16); i += UM_THREADS)
            sts128_zero(sbase + uint32_t(C::Q_OFF) + 16 * i);
    } else {
#pragma unroll 1
        for (int i = tid; i < int((2 * C::QBUF + 2 * C::PBUF) / 16); i += UM_THREADS)
            sts128_zero(sbase + uint32_t(C::Q_OFF) + 16 * i);
    }
    fence_proxy_async_smem();
    if (warp == 0) {
        // one barrier per lane: full and empty (one arrival), then q_full, q_free, s_full, s_free,
        // p_full, pt_free (two each; arrival counts packed four bits apiece), then the unit
        // ring's r_full (one) and r_empty (three: the two MMA issuers and the Qhat warp)
        constexpr uint32_t kCounts = 1u | (1u + 2 * UM_SOFT / 32) << 4 | 1u << 8 | (UM_SOFT / 32) << 12 |
                                     (UM_SOFT / 32) << 16 | (2u * UM_SOFT / 32) << 20;
        for (int i = lane; i < C::NBARS; i += 32) {
            const int j = i - 3 * STAGES;
            uint32_t cnt = 1;
            if (j >= 0 && j < 12) cnt = (kCounts >> (4 * (j >> 1))) & 15u;
            else if (j >= 12 + UM_RQ) cnt = 3;
            mbar_init(&bars[i], cnt);
        }
        if (lane == 0) {
            *s_abort = 0;
            s_xcnt[0] = s_xcnt[1] = 0;
        }
        fence_mbarrier_init();
    }
    if (warp == UM_TMEM_WARP) {
        tc_alloc(s_tmem, UM_TMEM_COLS);
        tc_relinquish();
    }
    if (tid == 0) {
        prefetch_tensormap(&tmk);
        prefetch_tensormap(&tmv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    // tensor-memory columns: S^T buffers at 0 and 32, O^T buffers at 64 and 96 (one per chunk parity),
    // the groups' shares of a unit at UM_XCOL + 8 * (2 * slot + group)
    // With tables_ready alone, q, the pools, the scales and the workspace are read only after the
    // PDL wait. With inputs_ready as well, q, the pools and the scales are not written by the kernel before this
    // one either: every read of them may come before the PDL wait, and each role waits only before its
    // first access to the workspace or the output (wait_prev). The MMA warps touch neither.
    const bool defer = early && p.inputs_ready != 0;
    if (!early) {
        pdl_wait();
        pdl_trigger();
    }
    const int* prefix = nullptr;
    // Prefix mode packs the units of sequences with fewer partitions; a launch with at most one unit
    // per CTA has a CTA for every dense slot (b, head group, partition < max_parts) and needs none.
    if (MULTI && p.B <= KVB_PREFIX_MAX) {
        if (!early && tid < p.B) my_len = __ldg(p.seq_lens + tid);
        build_unit_prefix_wide(p, s_prefix, reinterpret_cast<int*>(scratch), tid, UM_THREADS, 1, s_lens, my_len);
        prefix = s_prefix;
    }
    const long long total = unit_total(p, prefix);
    auto unit_of = [&](long long i, Unit& uu) { return unit_at(p, prefix, prefix ? s_lens : nullptr, i, uu); };
    // The CTA's first unit is unit blockIdx.x (when that is a unit): decoded here once for every role.
    // Later units are decoded by the producer alone and reach the other roles through the unit ring.
    Unit u_first;
    const bool has_first = (long long)blockIdx.x < total && unit_of(blockIdx.x, u_first);
    // Block ids of a unit's pages into the page table (producer warp); refused ones (outside
    // [0, num_blocks)) become -2.
    auto table_entry = [&](int blk) { return blk < 0 || (long long)blk >= p.num_blocks ? -2 : blk; };
    auto read_block_ids = [&](const Unit& uu) {
        const int* bt = p.block_table + (size_t)uu.b * p.max_blocks;
        const int pg0 = uu.t0 >> lp, pg1 = (uu.t1 - 1) >> lp;
        const int npg = min(pg1 - pg0 + 1, UM_PT);  // the host keeps partitions within UM_PT pages
        __syncwarp();
        if constexpr (MULTI) {
            for (int i = lane; i < npg; i += 32) pt_blk[i] = table_entry(__ldg(bt + pg0 + i));
        } else {
#pragma unroll 1
            for (int i = lane; i < npg; i += 32) pt_blk[i] = table_entry(__ldg(bt + pg0 + i));
        }
        __syncwarp();
    };
    bool ids_early = false;  // producer: the first unit's block ids are already in the page table
    if (early) {
        if (warp == UM_PRODUCER && has_first && u_first.nparts > 0) {
            // the guess holds the unit's pages (its first page is the guess's, its last one no later)
            if (g_npg > 0 && u_first.b == g_b && u_first.hg == g_hg && u_first.part == g_part) {
                __syncwarp();
                if (lane < g_npg) pt_blk[lane] = table_entry(g_ids[0]);
                if (lane + 32 < g_npg) pt_blk[lane + 32] = table_entry(g_ids[1]);
                __syncwarp();
            } else {
                read_block_ids(u_first);
            }
            ids_early = true;
        }
        if (!defer) pdl_wait();
        pdl_trigger();
    }
    bool waited = !defer;  // this thread has passed the PDL wait
    auto wait_prev = [&]() {
        if (!waited) {
            pdl_wait();
            waited = true;
        }
    };
    if (!defer) note_counter_count(p);

    // A wait that ran out sets the abort flag (every role's loops end on it); the error bit is
    // raised once, at the kernel's end (one store here instead of an atomic at each of the waits).
    auto give_up = [&]() { *s_abort = 1; };

    if (warp >= 8) reg_dealloc<UM_REGS_CTRL>();  // the split happens in each role's own code
    if (warp == UM_PRODUCER) {
        // ------------------------------------------------------------------ TMA producer
        const uint64_t policy = l2_evict_first_policy();
        // Units: first unit blockIdx.x; with more units than CTAs, the rest one at a time from the
        // workspace's work counter, the next index requested while the current unit streams (so an
        // SM that runs slow takes fewer). Every unit is published to the MMA issuers and the Qhat
        // warp through the unit ring, in order; -1 ends it.
        unsigned* wc = work_counters(p);
        const bool dyn = MULTI && total > (long long)gridDim.x;
        unsigned nxt = 0;
        bool asked = false;
        // The producer's first workspace access: the counter count, then (with more units than CTAs)
        // the request for its second unit, made while its first one streams.
        auto ask_next = [&]() {
            if (asked) return;
            asked = true;
            if (!waited) {
                wait_prev();
                if (blockIdx.x == 0 && lane == 0) p.error_flag[1] = unsigned(p.B * p.nhg);
            }
            if (dyn && lane == 0) nxt = atomicAdd(&wc[0], 1u);
        };
        if (!defer) ask_next();
        int wpos = 0;
        auto publish = [&](const Unit* uu) {  // nullptr ends the ring
            const int e = wpos % UM_RQ;
            if (lane == 0 && wpos >= UM_RQ && !*s_abort &&
                !mbar_wait_bounded(&r_empty[e], ((wpos / UM_RQ) - 1) & 1, s_abort))
                give_up();
            __syncwarp();
            if (lane == 0) {
                if (uu) ring_at(e) = *uu;
                else ring_at(e).b = -1;
                mbar_arrive(&r_full[e]);
            }
            ++wpos;
        };
        long long idx = blockIdx.x;
        Unit u;
        int stage = 0;
        uint32_t phase = 0;
        const int box_rows = p.page < UM_CHUNK ? p.page : UM_CHUNK;
        const int nbox = UM_CHUNK / box_rows;
        const uint32_t box_bytes = 2u * NSUB * uint32_t(box_rows) * 128u;
        int unit_no = 0;
        int kp = 0;  // running chunk index
        for (;;) {
            bool real;
            if (unit_no == 0 && idx == (long long)blockIdx.x) {
                real = has_first;
                u = u_first;
            } else {
                real = idx < total && unit_of(idx, u);
            }
            // A unit is published once its first chunk's loads are on their way (a tokenless one at once).
            if (real && u.nparts == 0) publish(&u);
            if (real && u.nparts > 0) {
                const int pg0 = u.t0 >> lp, pg1 = (u.t1 - 1) >> lp;  // the unit's pages (pg1 - pg0 < UM_PT)
                const int npg = min(pg1 - pg0 + 1, UM_PT);
                const int sb = unit_no & 1;
                if (!(ids_early && unit_no == 0)) read_block_ids(u);
                // a unit starting at an odd running index gets one empty chunk in front (see the softmax)
                const int c0 = u.t0 / UM_CHUNK - (kp & 1), c1 = (u.t1 + UM_CHUNK - 1) / UM_CHUNK;
                for (int c = c0; c < c1; ++c) {
                    const int tok0 = c * UM_CHUNK;
                    // With more units than CTAs, the second unit is requested once the ring is full (after
                    // the wait for the previous grid). A CTA with a single unit waits only at its end, so
                    // its whole unit may stream while the previous grid runs.
                    if (kp == STAGES && dyn) ask_next();
                    if (lane == 0 && !*s_abort && !mbar_wait_bounded(&empty[stage], phase ^ 1u, s_abort)) give_up();
                    __syncwarp();
                    // lane j < nbox owns box j (one page, or 128 rows of a larger page)
                    int blk = -1;
                    bool mine = false, refused = false;
                    if (lane < nbox) {
                        const int i = (tok0 + lane * box_rows) >> lp;
                        if (i >= pg0 && i <= pg1) {
                            blk = pt_blk[i - pg0];
                            refused = blk < 0;
                            mine = !refused;
                        }
                    }
                    const unsigned owned = __ballot_sync(0xffffffffu, mine);
                    const bool bad = __any_sync(0xffffffffu, refused);
                    const uint32_t bytes = uint32_t(__popc(owned)) * box_bytes;
                    const bool abort_now = *s_abort;
                    // The unit's first int8 chunk also publishes the unit's scales, fetched after the tile
                    // loads are on their way: its stage completes on the bytes plus the arrival below.
                    const bool scales_due = KVT == 2 && c == c0;
                    uint64_t* fb = &full[kp % (2 * STAGES)];
                    if (lane == 0) {
                        stage_bad[stage] = bad;
                        if (bad) raise_error(p.error_flag, KVB_DEVERR_BLOCK);
                        if (scales_due) {
                            if (!abort_now && bytes) mbar_expect_tx(fb, bytes);
                        } else if (abort_now || bytes == 0) {
                            mbar_arrive(fb);
                        } else {
                            mbar_arrive_expect_tx(fb, bytes);
                        }
                    }
                    __syncwarp();
                    if (mine && !abort_now) {
                        const int tok = tok0 + lane * box_rows;
                        const int y = (blk * p.Hkv + u.kvh) * p.page + (tok & (p.page - 1));
                        uint8_t* st = smem + stage * C::STAGE;
#pragma unroll
                        for (int s = 0; s < NSUB; ++s) {
                            const int x = s * (KVT == 1 ? 64 : 128);
                            const uint32_t off = s * TILE + lane * box_rows * 128;
                            tma_load_2d(st + off, &tmk, fb, x, y, policy);
                            tma_load_2d(st + NSUB * TILE + off, &tmv, fb, x, y, policy);
                        }
                    }
                    if (c == c0) publish(&u);
                    if (scales_due) {
                        // the softmax warps are done with this scale buffer's previous unit
                        if (lane == 0 && unit_no >= 2 && !*s_abort &&
                            !mbar_wait_bounded(&pt_free[sb], ((unit_no - 2) >> 1) & 1, s_abort))
                            give_up();
                        __syncwarp();
                        // the unit's page scales, and the largest V scale among them (the probability
                        // scale of the int8 O^T accumulator, constant over the unit)
                        float* ks_b = pt_ks + sb * UM_PT;
                        float* vs_b = pt_vs + sb * UM_PT;
                        float vunit = 0.f;
                        auto scale_of = [&](int i) {
                            const int b2 = pt_blk[i];
                            const float vsi = b2 >= 0 ? __ldg(p.v_scale + (size_t)b2 * p.Hkv + u.kvh) : 0.f;
                            ks_b[i] = b2 >= 0 ? __ldg(p.k_scale + (size_t)b2 * p.Hkv + u.kvh) : 0.f;
                            vs_b[i] = vsi;
                            vunit = fmaxf(vunit, vsi);
                        };
                        if constexpr (MULTI) {
                            for (int i = lane; i < npg; i += 32) scale_of(i);
                        } else {
#pragma unroll 1
                            for (int i = lane; i < npg; i += 32) scale_of(i);
                        }
                        vunit = warp_max(vunit);
                        if (lane == 0) unit_vsmax[sb] = vunit;
                        __syncwarp();  // every lane's scale writes happen before the arrive
                        if (lane == 0) mbar_arrive(fb);
                    }
                    __syncwarp();
                    ++kp;
                    if (++stage == STAGES) stage = 0, phase ^= 1u;
                }
                ++unit_no;
            }
            // the next unit
            ask_next();
            if (!dyn) break;
            long long nidx = 0;
            if (lane == 0) {
                nidx = (long long)gridDim.x + nxt;
                if (nidx < total) {
                    nxt = atomicAdd(&wc[0], 1u);
                } else if (atomicAdd(&wc[1], 1u) == gridDim.x - 1) {
                    // every CTA has found the units exhausted: leave the counters zero for the next launch
                    atomicExch(&wc[0], 0u);
                    atomicExch(&wc[1], 0u);
                }
            }
            nidx = __shfl_sync(0xffffffffu, nidx, 0);
            if (nidx >= total) break;
            idx = nidx;
        }
        ask_next();
        publish(nullptr);
    } else if (warp == UM_MMA0 || warp == UM_MMA1) {
        // ------------------------------------------------------------------ MMA issuers
        // Warp 9 issues every S^T = K Qhat^T product, warp 10 every O^T = V^T Phat^T product, each
        // in running chunk order (chunk k's products go to the S^T and O^T buffers of parity k & 1,
        // whose softmax group takes chunk k). One thread per warp, and every wait is a blocking
        // mbarrier wait, so neither issuer takes issue slots from the softmax warps that share its
        // SM sub-partition, and neither kind of product waits behind the other: S^T_k goes out as
        // soon as its stage is loaded and S^T_{k-2} was read, and O^T_k as soon as Phat_k is
        // written (which also releases the stage to the producer). One thread issuing four or eight
        // products takes 0.2-0.3 us, so one issuer for both kinds put that on the other's path.
        // QK for int8: A = K (signed), B = q limbs (signed). PV: A = V (signed), B = probability
        // bytes (unsigned).
        const bool s_issuer = warp == UM_MMA0;
        if (lane == 0) {
            const uint32_t idesc =
                s_issuer ? (KVT == 1 ? instr_desc(1, 0, 0, 0, 0, N, 128) : instr_desc(2, 1, 1, 0, 0, N, 128))
                         : (KVT == 1 ? instr_desc(1, 0, 0, 1, 1, NPV, 128) : instr_desc(2, 1, 0, 1, 1, NPV, 128));
            constexpr int KQK = KVT == 1 ? 16 : 32;  // contraction elements per instruction
            auto wait_on = [&](uint64_t* bar, uint32_t parity) {
                if (!*s_abort && !mbar_wait_bounded(bar, parity, s_abort)) give_up();
                return !*s_abort;
            };
            int rpos = 0;  // next unit ring entry
            int unit_no = -1, k_end = 0;
            while (!*s_abort) {
                // the next unit from the ring (units without tokens are skipped; -1 ends it)
                const int e = rpos % UM_RQ;
                if (!wait_on(&r_full[e], uint32_t(rpos / UM_RQ) & 1)) break;
                const Unit v = ring_at(e);
                mbar_arrive(&r_empty[e]);
                ++rpos;
                if (v.b < 0) break;
                if (v.nparts == 0) continue;
                ++unit_no;
                const int qb = unit_no & 1;
                const int k_base = k_end;
                k_end = k_base + (v.t1 + UM_CHUNK - 1) / UM_CHUNK - v.t0 / UM_CHUNK + (k_base & 1);
                if (s_issuer) {
                    if (!wait_on(&q_full[qb], (unit_no >> 1) & 1)) break;  // the unit's Qhat is written
                    const uint32_t qaddr = sbase + uint32_t(C::Q_OFF) + qb * C::QBUF;
                    for (int k = k_base; k < k_end; ++k) {
                        // chunk k's stage loaded, and S^T_{k-2} (same buffer) read
                        const int par = k & 1;
                        const uint32_t use = uint32_t(k >> 1);
                        if (use > 0 && !wait_on(&s_free[par], (use - 1) & 1)) break;
                        if (!wait_on(&full[k % (2 * STAGES)], uint32_t(k / (2 * STAGES)) & 1)) break;
                        tc_fence_after();
                        const uint32_t kt = sbase + (k % STAGES) * C::STAGE;
#pragma unroll
                        for (int s = 0; s < UM_D / KQK; ++s) {
                            // 32 bytes of the contraction per instruction: slice s*32/128, offset s*32%128
                            const uint32_t off = (s * 32 / 128) * TILE + (s * 32) % 128;
                            const uint32_t qoff = (s * 32 / 128) * (C::NMAX * 128) + (s * 32) % 128;
                            tc_mma<KVT>(tmem + 32 * par, smem_desc(kt + off, 16, 1024),
                                        smem_desc(qaddr + qoff, 16, 1024), idesc, s > 0);
                        }
                        tc_commit(&s_full[par]);
                    }
                    if (*s_abort) break;
                    tc_commit(&q_free[qb]);  // this warp's last read of the unit's Qhat buffer
                } else {
                    for (int k = k_base; k < k_end; ++k) {
                        // chunk k's Phat written by its softmax group
                        const int par = k & 1;
                        if (!wait_on(&p_full[par], uint32_t(k >> 1) & 1)) break;
                        tc_fence_after();
                        const int st = k % STAGES;
                        const uint32_t vt = sbase + st * C::STAGE + NSUB * TILE;
                        const uint32_t pb = sbase + uint32_t(C::P_OFF) + par * C::PBUF;
                        // int8: O^T accumulates over the group's chunks until the softmax restarts it
                        const bool keep = KVT == 2 && p_restart[par] == 0;
#pragma unroll
                        for (int s = 0; s < UM_CHUNK / KQK; ++s) {
                            // V^T (MN-major): KQK token rows per instruction = KQK/8 atoms of 1024 B; the
                            // second 64-dim slice of fp16 rows is the next tile (LBO). Phat^T (MN-major,
                            // 32-byte swizzle): KQK token rows of 32 B, atoms of 8 rows 256 B apart.
                            const uint32_t voff = s * (KQK / 8) * 1024;
                            const uint32_t poff = s * KQK * 32;
                            tc_mma<KVT>(tmem + 64 + 32 * par, smem_desc(vt + voff, TILE, 1024),
                                        smem_desc(pb + poff, C::PBUF, 256, SWZ_32B), idesc, s > 0 || keep);
                        }
                        tc_commit(&empty[st]);  // O^T_k done: K and V of chunk k are no longer read
                    }
                    if (*s_abort) break;
                }
            }
        }
    } else if (warp == UM_TMEM_WARP) {
        // ------------------------------------------------------------------ Qhat preparation
        // Runs ahead of the softmax groups. For the n-th unit with tokens (slot n & 1) it waits until
        // the slot's previous unit is done (its QK^T products and both groups' shares), writes Qhat^T
        // (row (head g, part r) = fp16 half r of q, or int8 limb r) and the per-head factors that turn
        // the combined MMA result into a log2 score, publishes the unit and arrives on q_full. A unit
        // with nparts < 0 ends the groups' loop. Units without tokens get their outputs here.
        Unit u;
        int rpos = 0;  // next unit ring entry
        auto ring_next = [&](Unit& uu) {  // the next published unit into uu (every lane); false at the end
            const int e = rpos % UM_RQ;
            int ok = 0;
            if (lane == 0) {
                if (!*s_abort && !mbar_wait_bounded(&r_full[e], uint32_t(rpos / UM_RQ) & 1, s_abort)) give_up();
                ok = !*s_abort && ring_at(e).b >= 0;
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) uu = ring_at(e);
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_empty[e]);
            ++rpos;
            return ok != 0;
        };
        // The producer's first entry is unit blockIdx.x whenever that is a unit: it is taken without
        // waiting for the ring (which is on the first unit's critical path), and its entry is
        // consumed with the next one.
        bool first = has_first;
        if (first) u = u_first;
        bool first_entry = first;
        for (int n = 0;; ++n) {
            // the next unit with tokens; units without tokens get their outputs here
            bool more = false;
            for (;;) {
                if (first) {
                    first = false;
                } else {
                    if (first_entry) {
                        first_entry = false;
                        Unit skip;
                        ring_next(skip);
                    }
                    if (!ring_next(u)) break;
                }
                if (u.nparts > 0) {
                    more = true;
                    break;
                }
                wait_prev();
                store_tokenless_unit<UM_D, MULTI>(p, u, lane, 32);
            }
            const int qb = n & 1;
            if (n >= 2) {
                if (lane == 0 && !*s_abort && !mbar_wait_bounded(&q_free[qb], ((n - 2) >> 1) & 1, s_abort))
                    give_up();
                __syncwarp();
            }
            if (!more) {
                if (lane == 0) {
                    slot_unit(qb)->nparts = -1;
                    mbar_arrive(&q_full[qb]);
                }
                break;
            }
            uint8_t* qbuf = smem + C::Q_OFF + qb * C::QBUF;
            const int d0 = 4 * lane;  // this lane's four head-dim elements
            const float* qrow = p.q + ((size_t)u.b * p.H + u.h0) * UM_D + d0;
            constexpr int QB = QGP < UM_QBATCH ? QGP : UM_QBATCH;
#pragma unroll
            for (int g0 = 0; g0 < QGP; g0 += QB) {
                float4 xs[QB];
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const float* row = qrow + (g0 + j) * UM_D;
                    // q is 16-byte aligned (the host checks it)
                    xs[j] = g0 + j < u.nh ? __ldg(reinterpret_cast<const float4*>(row)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < QB; ++j) {
                    const int g = g0 + j;
                    const float x[4] = {xs[j].x * p.q_scale, xs[j].y * p.q_scale, xs[j].z * p.q_scale,
                                        xs[j].w * p.q_scale};
                    const float amax = warp_max(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
                    // amax = f * 2^e with f in [0.5, 1), from the exponent bits; heads with amax below
                    // 2^-90 have scores that round to 0 and are treated as zero, which keeps every
                    // power of two below in range
                    const int e = int((__float_as_uint(amax) >> 23) & 0xffu) - 126;
                    const bool live = amax >= 8.0779356e-28f && amax < 3.0e38f;  // 2^-90
                    if constexpr (KVT == 1) {
                        // x * 2^(14 - e) in [-2^14, 2^14): hi + lo halves
                        // x * 2^(14 - e) and its inverse factor 2^(e - 14)
                        const float pre = live ? __uint_as_float(uint32_t(127 + 14 - e) << 23) : 1.f;
                        if (lane == 0) s_qs[qb * 8 + g] = live ? __uint_as_float(uint32_t(127 - 14 + e) << 23) : 1.f;
                        uint32_t hi[2], lo[2];
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            const float a = x[2 * t] * pre, b = x[2 * t + 1] * pre;
                            const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
                            const __half la = __float2half_rn(a - __half2float(ha));
                            const __half lb = __float2half_rn(b - __half2float(hb));
                            hi[t] = uint32_t(__half_as_ushort(ha)) | uint32_t(__half_as_ushort(hb)) << 16;
                            lo[t] = uint32_t(__half_as_ushort(la)) | uint32_t(__half_as_ushort(lb)) << 16;
                        }
                        const int col = (d0 % 64) * 2, sb = d0 / 64;
                        *reinterpret_cast<uint2*>(qbuf + sb * (C::NMAX * 128) + swz_off(g, col)) = make_uint2(hi[0], hi[1]);
                        *reinterpret_cast<uint2*>(qbuf + sb * (C::NMAX * 128) + swz_off(QGP + g, col)) =
                            make_uint2(lo[0], lo[1]);
                    } else {
                        // integer x * 2^(30 - e) with |.| < 2^30, as four signed limbs
                        const float pre = live ? __uint_as_float(uint32_t(127 + 30 - e) << 23) : 1.f;
                        if (lane == 0) s_qs[qb * 8 + g] = live ? __uint_as_float(uint32_t(127 - 30 + e) << 23) : 1.f;
                        // Limbs of element i packed in w[i] (byte 3 = limb 0 .. byte 0 = limb 3): adding 128
                        // to each of the three lower signed digits turns them into plain bytes (no
                        // carries), so the digits are the bytes of x + 0x808080 with those three flipped
                        // back by 0x80; the top byte is the signed top digit (|x| < 2^30).
                        uint32_t w[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) w[i] = uint32_t(__float2int_rn(x[i] * pre) + 0x808080) ^ 0x808080u;
                        // 4 x 4 byte transpose: row r gets limb r of the four elements, element i in byte i
                        const uint32_t a01 = __byte_perm(w[0], w[1], 0x5140), b01 = __byte_perm(w[0], w[1], 0x7362);
                        const uint32_t a23 = __byte_perm(w[2], w[3], 0x5140), b23 = __byte_perm(w[2], w[3], 0x7362);
                        const uint32_t rows[4] = {__byte_perm(b01, b23, 0x7632), __byte_perm(b01, b23, 0x5410),
                                                  __byte_perm(a01, a23, 0x7632), __byte_perm(a01, a23, 0x5410)};
#pragma unroll
                        for (int r = 0; r < 4; ++r) *reinterpret_cast<uint32_t*>(qbuf + swz_off(g * 4 + r, d0)) = rows[r];
                    }
                }
            }
            if (lane == 0) *slot_unit(qb) = u;
            fence_proxy_async_smem();  // generic writes of Qhat^T before the MMA reads them
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_full[qb]);
        }
    } else if (warp < 8) {
        // ------------------------------------------------------------------ softmax / accumulation
        reg_alloc<UM_REGS_SOFT>();
        // Two warpgroups take alternate chunks: group gi handles the chunks whose running index k has
        // k & 1 == gi, with its own tensor-memory S/O buffers and Phat buffer, and its own running
        // (max, sum, O). The groups merge once per unit.
        const int gi = warp >> 2;
        const int gt = tid - gi * UM_SOFT;  // 0..127 within the group
        const int sw = gt >> 5;                  // warp within the group
        const uint32_t gbar = 2 + gi;            // named barrier of the group
        // this warp's tensor-memory lane quarter is fixed by warp % 4
        const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
        const int my_lane = (warp & 3) * 32 + lane;  // token in S^T, head dim in O^T
        // [32,112) chunk max x2 ([value][warp]: 8 heads, V scale); [112,144) sums
        float* gred = red + gi * UM_GRED;
        int stage = 0;
        int k = 0;  // running chunk index
        for (int unit_no = 0;; ++unit_no) {
            // ---- the unit and its score factors, from the slot the Qhat warp filled
            const int qb = unit_no & 1;
            if (!*s_abort && !mbar_wait_bounded(&q_full[qb], (unit_no >> 1) & 1, s_abort)) give_up();
            const Unit u = *slot_unit(qb);
            // one decision for the whole group (after an abort the slot may never have been written)
            if (named_barrier_or(gbar, UM_SOFT, *s_abort || u.nparts < 0)) break;
            float qscale[QGP];  // per head: the factor that turns the combined MMA result into a log2 score
#pragma unroll
            for (int g = 0; g < QGP; ++g) qscale[g] = s_qs[qb * 8 + g];

            // ---- chunks
            float m[QGP], lsum[QGP], o[QGP];  // running max (group-uniform), this thread's sum share, O row
#pragma unroll
            for (int g = 0; g < QGP; ++g) m[g] = NEG_BIG, lsum[g] = 0.f, o[g] = 0.f;
            float m_prev[QGP];   // max the group's previous chunk's probabilities were computed with
            float vscale_prev = 0.f;
            bool have_prev = false;
            int k_own = -1;  // running index of this group's previous chunk
            int bad = 0;
            const uint32_t obuf = tmem + lane_base + 64 + 32 * gi;
            const int pg0 = u.t0 >> lp, pg_hi = ((u.t1 - 1) >> lp) - pg0;
            const float* ks_b = pt_ks + qb * UM_PT;  // int8 scales of the unit's pages
            const float* vs_b = pt_vs + qb * UM_PT;

            // Folds O^T of this group's previous chunk (running index kp; its PV product completes the
            // buffer's (kp >> 1)-th use) into the registers: loaded here, or already in `ro`.
            uint32_t ro[32];
            auto load_o = [&]() {
                tc_ld8(obuf, *reinterpret_cast<uint32_t(*)[8]>(&ro[0]));
                if (N > 8) tc_ld8(obuf + 8, *reinterpret_cast<uint32_t(*)[8]>(&ro[8]));
                if (N > 16) {
                    tc_ld8(obuf + 16, *reinterpret_cast<uint32_t(*)[8]>(&ro[16]));
                    tc_ld8(obuf + 24, *reinterpret_cast<uint32_t(*)[8]>(&ro[24]));
                }
            };
            // int8: adds the O^T accumulator (its PV products done; probabilities scaled by
            // kPScale / vunit) to the registers.
            auto fold_acc = [&](float vunit) {
                tc_fence_after();
                load_o();
                tc_wait_ld();
                tc_fence_before();
#pragma unroll
                for (int g = 0; g < QGP; ++g)
                    o[g] += limbs_to_float_wide(ro[4 * g], ro[4 * g + 1], ro[4 * g + 2], ro[4 * g + 3]) *
                            (vunit * kPUnit);
            };
            auto fold_prev = [&](int kp, bool loaded) {
                if (!loaded) {
                    if (!*s_abort && !mbar_wait_bounded(&empty[kp % STAGES], uint32_t(kp / STAGES) & 1, s_abort))
                        give_up();
                    tc_fence_after();
                    load_o();
                    tc_wait_ld();
                    tc_fence_before();
                }
                const uint32_t* r = ro;
                bool moved = false;  // the max moved since the previous chunk (group-uniform)
#pragma unroll
                for (int g = 0; g < QGP; ++g) moved |= m_prev[g] != m[g];
#pragma unroll
                for (int g = 0; g < QGP; ++g) {
                    float v;
                    if constexpr (KVT == 1) {
                        v = __uint_as_float(r[g]) + __uint_as_float(r[QGP + g]);
                    } else {
                        v = limbs_to_float(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]) *
                            (vscale_prev * kPUnit);
                    }
                    // o and the previous chunk are both relative to m_prev; move them to the current max
                    o[g] += v;
                }
                if (moved) {
#pragma unroll
                    for (int g = 0; g < QGP; ++g) o[g] *= exp2f(m_prev[g] - m[g]);
                }
            };

            // Group g takes the unit's chunks at running indices of parity g. A unit that would start at
            // an odd index gets one empty chunk (no valid token: nothing loaded, probabilities 0) in
            // front, so its first chunk goes to group 0 whatever ran before it on this CTA: which
            // chunks each group sums, and so the rounding of the unit's result, depend on the unit
            // alone, not on how units were handed out.
            const int c0 = u.t0 / UM_CHUNK - (k & 1), c1 = (u.t1 + UM_CHUNK - 1) / UM_CHUNK;
            for (int c = c0; c < c1; ++c, ++k) {
                const int cur_stage = stage;
                if (++stage == STAGES) stage = 0;
                if (int(k & 1) != gi) continue;
                const uint32_t use = uint32_t(k >> 1);
                // The stage's full barrier makes the producer's flags, scales and the TMA bytes visible
                // here (the fp16 path writes zeros into dead V rows, which must land after the TMA bytes).
                bool ok = true;
                if (!*s_abort)
                    ok = mbar_wait_bounded(&full[k % (2 * STAGES)], uint32_t(k / (2 * STAGES)) & 1, s_abort);
                if (ok && !*s_abort) ok = mbar_wait_bounded(&s_full[gi], use & 1, s_abort);
                if (!ok) give_up();
                tc_fence_after();
                const int tok = c * UM_CHUNK + my_lane;
                const bool valid = tok >= u.t0 && tok < u.t1;
                uint32_t r[32];
                const uint32_t sa = tmem + lane_base + 32 * gi;
                tc_ld8(sa, *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
                if (N > 8) tc_ld8(sa + 8, *reinterpret_cast<uint32_t(*)[8]>(&r[8]));
                if (N > 16) {
                    tc_ld8(sa + 16, *reinterpret_cast<uint32_t(*)[8]>(&r[16]));
                    tc_ld8(sa + 24, *reinterpret_cast<uint32_t(*)[8]>(&r[24]));
                }
                // this token's page scales (int8), read while the tensor-memory loads are in flight
                // the previous chunk's O^T too, when its PV product is already done (one load wait);
                // not for int8 with 8 heads, whose S^T and O^T together would not fit the registers
                constexpr bool kEarlyO = KVT == 1;  // int8 folds O^T only when its max moves
                const bool early_o =
                    kEarlyO && have_prev && mbar_test(&empty[k_own % STAGES], uint32_t(k_own / STAGES) & 1);
                if (early_o) load_o();
                float ks = 1.f, vs = 0.f;
                if constexpr (KVT == 2) {
                    const int slot = min(max((tok >> lp) - pg0, 0), pg_hi);
                    ks = ks_b[slot];
                    vs = valid ? vs_b[slot] : 0.f;
                }
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[gi]);
                // scores (log2 units) of this token for each head
                float sc[QGP];
#pragma unroll
                for (int g = 0; g < QGP; ++g) {
                    float v;
                    if constexpr (KVT == 1) {
                        v = __uint_as_float(r[g]) + __uint_as_float(r[QGP + g]);
                    } else {
                        v = limbs_to_float(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
                    }
                    sc[g] = (valid && g < u.nh) ? v * qscale[g] * ks : NEG_BIG;
                }
                bad |= stage_bad[cur_stage];
                // Lazy re-referencing: probabilities are taken relative to the group's running max m and
                // may reach 2^kTau; only when a score passes m + kTau (one vote per chunk) does the group
                // agree on the chunk max (warp, then its four warps) and move m.
                int exceed = 0;
#pragma unroll
                for (int g = 0; g < QGP; ++g) exceed |= sc[g] > m[g] + kTau;
                if (named_barrier_or(gbar, UM_SOFT, exceed)) {
                    float* rb = gred + 32 + 40 * int(use & 1);  // two alternating reduction slots, [head][warp]
#pragma unroll
                    for (int g = 0; g < QGP; ++g) {
                        const float mc = warp_max(sc[g]);
                        if (lane == 0) rb[g * 4 + sw] = mc;
                    }
                    named_barrier(gbar, UM_SOFT);
#pragma unroll
                    for (int g = 0; g < QGP; ++g) {
                        const float mn = fmaxf(m[g], max4(reinterpret_cast<const float4*>(rb)[g]));
                        lsum[g] *= exp2f(m[g] - mn);
                        m[g] = mn;
                    }
                }
                float pr[QGP];
#pragma unroll
                for (int g = 0; g < QGP; ++g) {
                    pr[g] = sc[g] > 0.5f * NEG_BIG ? exp2f(sc[g] - m[g]) : 0.f;
                    lsum[g] += pr[g];
                }
                // int8: probabilities relative to the unit's largest V scale, constant over the unit
                const float vscale_cur = KVT == 2 ? unit_vsmax[qb] : 0.f;
                if constexpr (KVT == 1) {
                    // The group's Phat buffer was last read by the PV product of its previous chunk: fold
                    // that chunk's O first (this also waits for that product), then overwrite.
                    if (have_prev) fold_prev(k_own, early_o);
                } else {
                    // int8: O^T accumulates in tensor memory over the group's chunks (int32, exact). The
                    // group waits for its previous PV product (it read the Phat buffer about to be
                    // overwritten), and folds the accumulator into the registers only when the running
                    // max moved, since the accumulator is relative to the old max; this chunk's PV
                    // product then restarts it.
                    int restart = 1;
                    if (have_prev) {
                        if (!*s_abort && !mbar_wait_bounded(&empty[k_own % STAGES], uint32_t(k_own / STAGES) & 1, s_abort))
                            give_up();
                        bool moved = false;  // group-uniform
#pragma unroll
                        for (int g = 0; g < QGP; ++g) moved |= m_prev[g] != m[g];
                        if (moved) {
                            fold_acc(vscale_cur);
#pragma unroll
                            for (int g = 0; g < QGP; ++g) o[g] *= exp2f(m_prev[g] - m[g]);
                        } else {
                            restart = 0;
                        }
                    }
                    if (gt == 0) p_restart[gi] = restart;  // before this chunk's p_full arrival
                }
                uint8_t* pbuf = smem + C::P_OFF + gi * C::PBUF;
                if constexpr (KVT == 1) {
                    // this token's row of Phat^T: the hi halves of the heads, then the lo halves
                    uint16_t h[2 * QGP];
#pragma unroll
                    for (int g = 0; g < QGP; ++g) {
                        const __half hi = __float2half_rn(pr[g]);
                        const __half lo = __float2half_rn(pr[g] - __half2float(hi));
                        h[g] = __half_as_ushort(hi);
                        h[QGP + g] = __half_as_ushort(lo);
                    }
                    uint32_t w[QGP];
#pragma unroll
                    for (int j = 0; j < QGP; ++j) w[j] = uint32_t(h[2 * j]) | uint32_t(h[2 * j + 1]) << 16;
                    store_p_row<QGP>(pbuf, my_lane, w);
                    // fp16 V rows outside the partition may hold stale data or dead pool slots, or were
                    // never loaded: zero this token's V row so 0 * NaN cannot reach O.
                    if (!valid) {
                        uint8_t* vrow = smem + cur_stage * C::STAGE + NSUB * TILE;
#pragma unroll
                        for (int sb2 = 0; sb2 < NSUB; ++sb2)
#pragma unroll
                            for (int ch = 0; ch < 8; ++ch)
                                sts128_zero(smem_u32(vrow + sb2 * TILE + my_lane * 128 + ch * 16));
                    }
                } else {
                    // probability * v_scale / (largest v_scale of the unit) as an unsigned integer below
                    // 2^30 whose four bytes are the four limbs (byte 3 = limb 0); this token's row of
                    // Phat^T holds head g's limbs 0..3 at bytes 4g..4g+3, so each word is byte-reversed.
                    const float f = vscale_cur > 0.f ? vs / vscale_cur * kPScale : 0.f;
                    uint32_t w[QGP];
#pragma unroll
                    for (int g = 0; g < QGP; ++g) w[g] = __byte_perm(__float2uint_rn(pr[g] * f), 0u, 0x0123);
                    store_p_row<QGP>(pbuf, my_lane, w);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[gi]);
#pragma unroll
                for (int g = 0; g < QGP; ++g) m_prev[g] = m[g];
                vscale_prev = vscale_cur;
                have_prev = true;
                k_own = k;
            }
            if (KVT == 2) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&pt_free[qb]);  // the unit's scales are no longer read
            }
            if (have_prev) {
                if constexpr (KVT == 1) {
                    fold_prev(k_own, false);
                } else {
                    if (!*s_abort && !mbar_wait_bounded(&empty[k_own % STAGES], uint32_t(k_own / STAGES) & 1, s_abort))
                        give_up();
                    fold_acc(vscale_prev);
                }
            }
            // ---- unit end: the group's sums over its 128 tokens
            wait_prev();  // the workspace and the output come next
            float L[QGP];
#pragma unroll
            for (int g = 0; g < QGP; ++g) {
                float a = lsum[g];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                L[g] = a;
            }
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g < QGP; ++g) gred[112 + g * 4 + sw] = L[g];
            }
            const int grp_bad = named_barrier_or(gbar, UM_SOFT, bad);
#pragma unroll
            for (int g = 0; g < QGP; ++g) {
                const float4 l4 = reinterpret_cast<const float4*>(gred + 112)[g];
                L[g] = (l4.x + l4.y) + (l4.z + l4.w);
            }
            // Each group leaves its share of the unit (O rows in tensor memory; m, L and the refusal
            // flag in shared memory) and counts itself in. The second group to finish merges the two
            // and stores the unit's result; the first goes on to its next unit without waiting.
            {
                uint32_t w[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) w[j] = j < QGP ? __float_as_uint(o[j]) : 0u;
                tc_st8(tmem + lane_base + uint32_t(UM_XCOL + 8 * (2 * qb + gi)), w);
            }
            float* xml = s_xml + (2 * qb + gi) * 24;
            if (gt == 0) {
#pragma unroll
                for (int g = 0; g < QGP; ++g) xml[g] = m[g], xml[8 + g] = L[g];
                xml[16] = grp_bad ? 1.f : 0.f;
            }
            tc_wait_st();
            tc_fence_before();
            named_barrier(gbar, UM_SOFT);  // the group's share is written
            if (gt == 0) {
                __threadfence_block();
                s_xcnt[2 + gi] = atomicAdd(&s_xcnt[qb], 1);
                __threadfence_block();
            }
            named_barrier(gbar, UM_SOFT);
            if (s_xcnt[2 + gi] == 1) {
                tc_fence_after();
                uint32_t w[8];
                tc_ld8(tmem + lane_base + uint32_t(UM_XCOL + 8 * (2 * qb + (gi ^ 1))), w);
                const float* yml = s_xml + (2 * qb + (gi ^ 1)) * 24;
                const bool any_bad = grp_bad || yml[16] != 0.f;
                tc_wait_ld();
                // group 0's share first whichever group merges, so the result does not depend on timing
#pragma unroll
                for (int g = 0; g < QGP; ++g) {
                    const float oy = __uint_as_float(w[g]), my = yml[g], ly = yml[8 + g];
                    const float o0 = gi == 0 ? o[g] : oy, o1 = gi == 0 ? oy : o[g];
                    const float m0 = gi == 0 ? m[g] : my, m1 = gi == 0 ? my : m[g];
                    const float l0 = gi == 0 ? L[g] : ly, l1 = gi == 0 ? ly : L[g];
                    const float mm = fmaxf(m0, m1);
                    const float w0 = exp2f(m0 - mm), w1 = exp2f(m1 - mm);
                    o[g] = o0 * w0 + o1 * w1;
                    L[g] = l0 * w0 + l1 * w1;
                    m[g] = mm;
                }
                if (gt == 0) s_xcnt[qb] = 0;  // both groups counted: the slot's next unit counts from zero
                const float nanv = __int_as_float(0x7fc00000);
                const int d = my_lane;
                // a single-partition unit's heads are consecutive rows of the output: local
                // out[b][h0 + g], or (peers) this rank's global buffer at the unit's global row
                // (the peer path only in the many-unit instance, which every gathered launch uses)
                float* obase = nullptr;
                if (u.nparts == 1) {
                    size_t i = 0;
                    if (!MULTI || p.n_peers == 0) obase = p.out + ((size_t)u.b * p.H + u.h0) * UM_D;
                    else if (peer_index(p, u.b, u.h0, UM_D, &i)) obase = p.peer_out[p.peer_self] + i;
                }
#pragma unroll
                for (int g = 0; g < QGP; ++g) {
                    if (g >= u.nh) break;
                    const int h = u.h0 + g;
                    const float val = any_bad ? nanv : o[g] / L[g];
                    if (u.nparts == 1) {
                        if (obase) obase[g * UM_D + d] = val;
                    } else {
                        const size_t slot = ((size_t)u.b * p.H + h) * p.max_parts + u.part;
                        p.part_o[slot * UM_D + d] = val;
                        if (d == 0) p.part_ml[slot] = make_float2(m[g], any_bad ? nanv : L[g]);
                    }
                }
                if (MULTI && p.n_peers > 0 && obase) {
                    // the elements this thread stored, to the other ranks
                    const size_t i = obase - p.peer_out[p.peer_self];
#pragma unroll 1
                    for (int g = 0; g < u.nh; ++g) copy_to_peers<float>(p, i + g * UM_D + d);
                }
                // count the partition in; the last partition's CTA merges them all
                finish_partition<UM_D, 12, (QGP >= 2 ? 1 : 32), MULTI>(p, u, gt, UM_SOFT, gbar, &s_xcnt[2 + gi]);
            }
            // this warp is done with the unit's slot (its factors, both shares)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_free[qb]);
        }
    }

    // every role done: release tensor memory
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == UM_TMEM_WARP) tc_dealloc(tmem, UM_TMEM_COLS);
    if (tid == 0 && *s_abort) raise_error(p.error_flag, KVB_DEVERR_TIMEOUT);
}

template <int KVT, int QGP, bool MULTI>
cudaError_t launch_grid(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, const LaunchInfo& li,
                        long long grid) {
    using C = UCfg<KVT>;
    static KvbPerDevice<int> configured;  // the shared-memory attribute, set on each device
    int done = 0;
    cudaError_t e = configured.get(&done, [](int* v) {
        *v = 1;
        return cudaFuncSetAttribute(decode_umma_kernel<KVT, QGP, MULTI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(C::SMEM));
    });
    if (e != cudaSuccess) return e;
    return kvb_launch_pdl(decode_umma_kernel<KVT, QGP, MULTI>, (unsigned)grid, UM_THREADS, C::SMEM, li.stream, tk,
                          tv, p);
}

template <int KVT, int QGP>
cudaError_t launch_one(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, const LaunchInfo& li) {
    // at most one unit per CTA when even the dense unit count (every sequence of max_len tokens) fits
    const long long upper = (long long)p.B * p.nhg * p.max_parts;
    const long long grid = std::min<long long>(upper, (long long)li.num_sms);
    if (grid <= 0) return cudaSuccess;
    // the single-unit instance has no peer path: a gathered launch takes the many-unit one
    return upper > grid || p.n_peers > 0 ? launch_grid<KVT, QGP, true>(p, tk, tv, li, grid)
                                         : launch_grid<KVT, QGP, false>(p, tk, tv, li, grid);
}

template <int KVT>
cudaError_t launch_kvt(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, const LaunchInfo& li) {
    if (p.qg <= 1) return launch_one<KVT, 1>(p, tk, tv, li);
    if (p.qg <= 2) return launch_one<KVT, 2>(p, tk, tv, li);
    if (p.qg <= 4) return launch_one<KVT, 4>(p, tk, tv, li);
    return launch_one<KVT, 8>(p, tk, tv, li);
}

}  // namespace

bool kvb_umma_supported(int kv_type, int D, int page, int qg, int part_tokens) {
    if (kv_type != 1 && kv_type != 2) return false;
    if (D != 128) return false;
    if (!(page == 8 || page == 16 || page == 32 || page == 64 || page == 128 || page == 256)) return false;
    // a partition's pages and chunks must fit the page table and the int8 O^T accumulator's bound
    // (part_tokens 0: the automatic size, at most 8064 tokens for pages of 32 tokens or more, 4096
    // for 16-token pages, 2048 for 8-token pages)
    if (part_tokens > 0 && (part_tokens / page + 2 > UM_PT || part_tokens > (UM_UCH - 1) * UM_CHUNK)) return false;
    return qg >= 1 && qg <= 8;
}

cudaError_t kvb_launch_decode_umma(const DecodeParams& p, int kv_type, int D, const void* tmap_k, const void* tmap_v,
                                   const LaunchInfo& li) {
    (void)D;
    const CUtensorMap& tk = *static_cast<const CUtensorMap*>(tmap_k);
    const CUtensorMap& tv = *static_cast<const CUtensorMap*>(tmap_v);
    return kv_type == 1 ? launch_kvt<1>(p, tk, tv, li) : launch_kvt<2>(p, tk, tv, li);
}
