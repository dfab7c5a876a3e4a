// tc05.cuh -- thin inline-PTX layer over the sm_100a async units used here:
// tcgen05 (tensor-core MMA with TMEM accumulators), TMA copies (untiled
// cp.async.bulk and tiled cp.async.bulk.tensor; never multicast) and mbarriers.
//
// Operand images.  Every MMA operand lives in shared memory as a K-major
// "SW128" image: rows of 128 bytes grouped 8 per 1024-byte atom, the 16-byte
// chunks of row r XOR-swizzled by (r & 7).  An operand with more than 128
// bytes of K per row is split into K-blocks, each a separate [rows][128 B]
// image placed back to back.  Element (r, c) of a fp32 image lives in K-block
// c / 32 at byte (c % 32) * 4 of row r; of a bf16 image in K-block c / 64 at
// byte (c % 64) * 2.  Image bases are 1024-byte aligned.  The same byte
// layout is used for operand images stored in global memory, so they move
// with one bulk copy.
//
// Accumulators.  cta_group::1 MMAs with M = 128 put row m in TMEM lane m; with
// M = 64 row m sits in lane (m % 16) + 32 * (m / 16), i.e. lanes 0-15 of each
// warp's 32-lane sub-partition.  Column n of the tile is TMEM column base + n.
#pragma once

#include <cuda.h>  // CUtensorMap
#include <stdint.h>

namespace gdn {
namespace tc05 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (row, byte-in-row) in a SW128 image whose K-blocks
// hold `rows` rows each.
__device__ __forceinline__ uint32_t sw128_off(int row, int byte_in_kblock_row, int kblock, int rows) {
    return static_cast<uint32_t>(kblock * rows * 128 + row * 128 +
                                 ((((byte_in_kblock_row >> 4) ^ (row & 7)) << 4) | (byte_in_kblock_row & 15)));
}
__device__ __forceinline__ uint32_t sw128_f32(int row, int col, int rows) {
    return sw128_off(row, (col & 31) * 4, col >> 5, rows);
}
__device__ __forceinline__ uint32_t sw128_bf16(int row, int col, int rows) {
    return sw128_off(row, (col & 63) * 2, col >> 6, rows);
}

// MN-major 32-bit (tf32) operand image, layout SWIZZLE_128B_BASE32B: rows =
// K index, 128-byte rows of 32 consecutive M (or N) elements, 4-row atoms of
// 512 B in which the 32-byte chunks of row k are XOR-swizzled by (k & 3);
// MN blocks of 32 elements are `krows * 128` bytes apart.
__device__ __forceinline__ uint32_t mn32_f32(int k, int mn, int krows) {
    const int b = (mn & 31) * 4;
    return static_cast<uint32_t>((mn >> 5) * krows * 128 + k * 128 + ((((b >> 5) ^ (k & 3)) << 5) | (b & 31)));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: gives up once kWaitLimitNs of wall time (the %globaltimer
// clock) have passed since the first unsuccessful poll, or after
// kWaitMaxPolls polls, whichever comes first, and returns false; callers
// record GDN_ERR_DEVICE_TIMEOUT and unwind instead of hanging the GPU.  Every
// wait in this library is on an mbarrier of the waiting CTA, completed by
// that CTA's own copies or MMAs (never by another CTA or GPU), which take
// microseconds; 10 ms is far above any legitimate wait.
constexpr uint64_t kWaitLimitNs = 10ull * 1000 * 1000;
constexpr uint32_t kWaitMaxPolls = 1u << 26;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kWaitMaxPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
    return false;
}

// ------------------------------------------------------------ bulk copies --
__device__ __forceinline__ void bulk_g2s(uint32_t dst_smem, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem), "r"(bytes)
                 : "memory");
}
// Tiled 3-D TMA load of one box into shared memory (box layout and swizzle
// come from the tensor map); completes `bar`'s transaction count.  c0 is the
// innermost coordinate: c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(uint32_t dst_smem, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst_smem),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
// L2 prefetch of one tensor-map box (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned address.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Tiled bulk tensor store shared::cta -> global, completion through the bulk group.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src_smem, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src_smem), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until at most N bulk-copy groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Generic-proxy shared-memory writes -> visible to the async proxy (MMA, bulk copy).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------- TMEM --
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 consecutive columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
    uint32_t u[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]),
          "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
          "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(u[i]);
}
// 32 lanes x 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
    uint32_t u[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = __uint_as_float(u[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 registers per thread -> 32 lanes x 32 consecutive columns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&u)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
        "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15]), "r"(u[16]), "r"(u[17]),
        "r"(u[18]), "r"(u[19]), "r"(u[20]), "r"(u[21]), "r"(u[22]), "r"(u[23]), "r"(u[24]), "r"(u[25]), "r"(u[26]),
        "r"(u[27]), "r"(u[28]), "r"(u[29]), "r"(u[30]), "r"(u[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column) relative to an allocation base.
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) {
    return base + (lane << 16) + col;
}

// ---------------------------------------------------------------- the MMA --
// Shared-memory matrix descriptor of a K-major SW128 image (sm_100 format:
// start >> 4 at [0,14), LBO >> 4 at [16,30) (unused for swizzled K-major,
// set to 1), SBO >> 4 at [32,46) = 1024 B between 8-row groups, version 1 at
// [46,48), base offset 0, layout SWIZZLE_128B (2) at [61,64)).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Descriptor of an MN-major 16-bit (bf16) SW128 image: the same byte layout
// with rows = K index and the 128-byte row holding consecutive M (or N)
// elements; 8-row K groups 1024 B apart (SBO), MN blocks `lbo` bytes apart
// (LBO = K rows of the image x 128).
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t smem_addr, uint32_t lbo) {
    return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Descriptor of an MN-major 32-bit image (mn32_f32 layout): layout type
// SWIZZLE_128B_BASE32B (1), 4-row K groups 512 B apart (SBO), MN blocks
// `lbo` bytes apart.
__device__ __forceinline__ uint64_t mn32_desc(uint32_t smem_addr, uint32_t lbo) {
    return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) | (32ull << 32) | (1ull << 46) | (1ull << 61);
}

// Operand formats: kind::f16 takes kF16 or kBF16, kind::tf32 takes kTF32; the value is
// the instruction descriptor's format code.
enum Kind : uint32_t { kF16 = 0, kBF16 = 1, kTF32 = 2 };

// Instruction descriptor (kind::f16 / kind::tf32): fp32 accumulator, A and B
// of the same format, no negation, dense; a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc(Kind k, int M, int N, bool a_mn = false, bool b_mn = false) {
    return (1u << 4) | (static_cast<uint32_t>(k) << 7) | (static_cast<uint32_t>(k) << 10) |
           (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// kind::f16: fp16 or bf16 operands, as the instruction descriptor says
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
// kind::f16 with the A operand in TMEM (M = 128: row m in lane m, K packed two
// 16-bit elements per 32-bit column, 8 columns per instruction's K = 16).
__device__ __forceinline__ void mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
// Arrives once on `bar` when every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D[M x N] (+)= A[M x Kdim] . B[N x Kdim]^T, issued by one thread.
// A K-major operand image has rows = M (or N) with `x_rows` rows per K-block
// (K-block stride x_rows * 128 B); an MN-major image has rows = K with
// `x_rows` = its K rows (MN-block stride x_rows * 128 B) -- SW128 for bf16,
// the mn32_f32 layout for tf32.  One instruction takes 32 bytes of K: 16 bf16
// or 8 tf32 elements, i.e. 16 or 8 rows of an MN-major image.
template <Kind KIND, bool A_MN = false, bool B_MN = false>
__device__ __forceinline__ void mma_tile(uint32_t d_tmem, uint32_t a_smem, int a_rows, uint32_t b_smem, int b_rows,
                                         int kdim, int M, int N, bool accumulate) {
    const uint32_t id = idesc(KIND, M, N, A_MN, B_MN);
    constexpr int kElemBytes = KIND == kTF32 ? 4 : 2;
    constexpr int kStepK = 32 / kElemBytes;  // K elements per instruction
    const int steps = kdim / kStepK;
#pragma unroll 1
    for (int s = 0; s < steps; ++s) {
        uint64_t ad, bd;
        if (A_MN) {
            ad = KIND != kTF32 ? sw128_desc_mn(a_smem + s * kStepK * 128, a_rows * 128)
                               : mn32_desc(a_smem + s * kStepK * 128, a_rows * 128);
        } else {
            const int kb = (s * 32) >> 7, in = (s * 32) & 127;
            ad = sw128_desc(a_smem + kb * a_rows * 128 + in);
        }
        if (B_MN) {
            bd = KIND != kTF32 ? sw128_desc_mn(b_smem + s * kStepK * 128, b_rows * 128)
                               : mn32_desc(b_smem + s * kStepK * 128, b_rows * 128);
        } else {
            const int kb = (s * 32) >> 7, in = (s * 32) & 127;
            bd = sw128_desc(b_smem + kb * b_rows * 128 + in);
        }
        if (KIND != kTF32)
            mma_bf16(d_tmem, ad, bd, id, (accumulate || s > 0) ? 1u : 0u);
        else
            mma_tf32(d_tmem, ad, bd, id, (accumulate || s > 0) ? 1u : 0u);
    }
}

// mma_tile with every shape known at compile time: the two base descriptors
// are built once and each K step only adds a constant to the start-address
// field (no carry out of its 14 bits: shared addresses stay below 256 KB).
template <Kind KIND, bool A_MN, bool B_MN, int KDIM, int AROWS, int BROWS, int M, int N>
__device__ __forceinline__ void mma_ct(uint32_t d_tmem, uint32_t a_smem, uint32_t b_smem, bool accumulate) {
    constexpr uint32_t id = idesc(KIND, M, N, A_MN, B_MN);
    constexpr int kElemBytes = KIND == kTF32 ? 4 : 2;
    constexpr int kStepK = 32 / kElemBytes;
    constexpr int kSteps = KDIM / kStepK;
    static_assert(KDIM % kStepK == 0, "K must be a whole number of instructions");
    const uint64_t a0 = A_MN ? (KIND != kTF32 ? sw128_desc_mn(a_smem, AROWS * 128) : mn32_desc(a_smem, AROWS * 128))
                             : sw128_desc(a_smem);
    const uint64_t b0 = B_MN ? (KIND != kTF32 ? sw128_desc_mn(b_smem, BROWS * 128) : mn32_desc(b_smem, BROWS * 128))
                             : sw128_desc(b_smem);
#pragma unroll
    for (int s = 0; s < kSteps; ++s) {
        const uint32_t a_off = A_MN ? s * kStepK * 128 : ((s * 32) >> 7) * AROWS * 128 + ((s * 32) & 127);
        const uint32_t b_off = B_MN ? s * kStepK * 128 : ((s * 32) >> 7) * BROWS * 128 + ((s * 32) & 127);
        const uint64_t ad = a0 + (a_off >> 4);
        const uint64_t bd = b0 + (b_off >> 4);
        const uint32_t acc = (accumulate || s > 0) ? 1u : 0u;
        if (KIND != kTF32)
            mma_bf16(d_tmem, ad, bd, id, acc);
        else
            mma_tf32(d_tmem, ad, bd, id, acc);
    }
}

// D[128 x N] (+)= A[128 x KDIM] . B^T with A (16-bit) in TMEM from column
// a_tmem (KDIM / 2 columns) and B a K-major SW128 image of BROWS rows per
// K-block, or (B_MN) an MN-major image of KDIM rows.
template <Kind KIND, bool B_MN, int KDIM, int BROWS, int N>
__device__ __forceinline__ void mma_ct_ta(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_smem, bool accumulate) {
    static_assert(KIND != kTF32, "A in TMEM: 16-bit kinds only");
    constexpr uint32_t id = idesc(KIND, 128, N, false, B_MN);
    constexpr int kSteps = KDIM / 16;
    const uint64_t b0 = B_MN ? sw128_desc_mn(b_smem, BROWS * 128) : sw128_desc(b_smem);
#pragma unroll
    for (int s = 0; s < kSteps; ++s) {
        const uint32_t b_off = B_MN ? s * 16 * 128 : ((s * 32) >> 7) * BROWS * 128 + ((s * 32) & 127);
        mma_f16_ta(d_tmem, a_tmem + 8 * s, b0 + (b_off >> 4), id, (accumulate || s > 0) ? 1u : 0u);
    }
}

// Vector stores of 4 fp32 into shared memory / 16 bytes anywhere.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// fp32 -> tf32 with round-to-nearest (ties away); low 13 bits cleared.
__device__ __forceinline__ float to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

}  // namespace tc05
}  // namespace gdn
