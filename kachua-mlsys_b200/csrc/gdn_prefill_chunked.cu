// gdn_prefill_chunked.cu -- chunked-WY varlen GDN prefill on tcgen05 tensor cores.
//
// Replaces the reference's three Triton paths (Direct-v2 kernel.py:886-993,
// Split-WY :379-540, Flat-WY :576-863) with one design in two kernels.
//
// Algebra for one chunk of C = 64 tokens of one v-head (state S is [V][K]):
//   G_i   = prod_{m<=i} g_m (kept as log2 G),  Gam_ij = G_i / G_j = exp2(lG_i - lG_j), j <= i
//   N_ij  = beta_i Gam_ij (k_i . k_j)          for j < i     (strictly lower)
//   A     = I + N,   Ainv = (I - N)(I + N^2)(I + N^4)...(I + N^32)   (Neumann doubling)
//   W     = Ainv (beta G (.) K),   U = Ainv (beta (.) V)
//   Delta = U - W S0^T                          (rows delta_i of the update)
//   P_ij  = Gam_ij (q_i . k_j)                  for j <= i
//   O     = scale (G (.) (Q S0^T) + P Delta)
//   S1    = G_C S0 + Delta^T (tail (.) K),      tail_j = G_C / G_j = exp2(lG_C - lG_j)
// (the reference's derivation: kernel.py:265-278; gates :925-952; Gram and
// decay mask :957-976; Neumann inverse :333-376; WY terms :432-458; carry
// :497-540).  Every ratio is formed as exp2 of a non-positive log2 difference,
// never as a division by G (the beta/G form overflows, experiment_log.md:1027-1050).
//
// Affine form used by the kernels (K' = tail (.) K):
//   S1 = S0 M^T + D^T,   M = G_C I - K'^T W   [k][k'],   D = K'^T U   [k][v]
//   O  = scale (Qt S0^T + Ut),   Qt = G (.) Q - P W,     Ut = P U
// -- the same identities with Delta expanded, so the chunk-to-chunk chain is
// one matrix product and everything else is per-chunk, parallel work.
//
// Kernel 1, gdn_chunk_prepare (one CTA per chunk x q/k head, both v-heads):
//   [K;Q] K^T on bf16 tcgen05 (M=128, N=64, K=128); per v-head the gates,
//   N and P; Ainv by Neumann doubling on fp16 tcgen05 64x64x64 products (both
//   v-heads packed into one M=64 accumulator pair); [W | U] = Ainv [bGK | bV]
//   (M=64, N=256); then P [W | U] and K'^T [W | U] (M=128, N=256), whose
//   epilogues write Qt, Ut, M and D to the workspace.
// Kernel 2, gdn_chunk_carry (one CTA per sequence x v-head x 64 value rows):
//   four state warps keep the fp32 state in registers and run the chain
//   S <- S M^T + D^T with one M=128, N=64, K=128 fp16 MMA per chunk; four
//   output warps finish O = scale (Qt S^T + Ut) from a second MMA on the same
//   state image, overlapped with the next chunk.  Operands arrive by bulk
//   copies issued two chunks ahead.
// Precision: tensor-core operands are fp16 (round-to-nearest, 11-bit
// significand like tf32) with fp32 accumulation; the state and D stay fp32
// between chunks, and only the MMA's copy of the state is rounded.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled
#include <string.h>

#include "gdn_common.cuh"
#include "tc05.cuh"

namespace gdn {
using namespace tc05;

constexpr int kC = 64;
// Per (chunk record, v-head) the prepare kernel leaves 96 KiB of f16 operand
// images for the carry, at these offsets:
constexpr int kRecM = 0;          // M = G_C I - K'^T W   [128 k][128 k']  K-major SW128        32 KiB
constexpr int kRecKb = 32768;     // K' = tail (.) K      [64 j][128 k]    MN-major (2 kblocks) 16 KiB
constexpr int kRecU = 49152;      // U                    [64 j][128 v]    MN-major (2 blocks)  16 KiB
constexpr int kRecQt = 65536;     // Qt = G (.) Q - P W   [64 i][128 k]    K-major              16 KiB
constexpr int kRecUt = 81920;     // Ut = P U             [64 i][128 v]    SW128 rows (2 blocks) 16 KiB
constexpr int kHeadRecBytes = 98304;

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace: header, per-sequence record bases, the chunk table and the
// per-record, per-head operand arrays (every array 1024-byte aligned).
struct WsLayout {
    int64_t R;  // record capacity: ceil(T / 64) + N bounds sum_s ceil(len_s / 64)
    int64_t off_hdr, off_base, off_table, off_rec, total;
};

__host__ __device__ inline WsLayout ws_layout(int64_t T, int64_t N) {
    WsLayout L;
    L.R = (T + kC - 1) / kC + N;
    int64_t o = 0;
    L.off_hdr = o;
    o += 1024;
    L.off_base = o;
    o = align_up(o + 4 * (N + 1), 1024);
    L.off_table = o;
    o = align_up(o + 16 * L.R, 1024);
    L.off_rec = o;
    o += L.R * kHV * kHeadRecBytes;
    L.total = align_up(o, 1024);
    return L;
}

size_t chunked_workspace_bytes(int64_t total_tokens, int64_t num_seqs) {
    return static_cast<size_t>(ws_layout(total_tokens, num_seqs).total);
}

// ------------------------------------------------------------ chunk table --
// One block: per sequence, ceil(len / 64) records; exclusive scan -> base[s];
// table[rec] = (seq, first token, length <= 64).  Records past the capacity
// (only reachable with overlapping, invalid cu_seqlens) are dropped and
// reported.
__global__ void __launch_bounds__(1024) gdn_chunk_table_kernel(const PrefillParams p, uint8_t* ws, WsLayout L) {
    int* base = reinterpret_cast<int*>(ws + L.off_base);
    int4* table = reinterpret_cast<int4*>(ws + L.off_table);
    __shared__ int warp_tot[32];
    __shared__ long long carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int64_t s0 = 0; s0 < p.num_seqs; s0 += 1024) {
        const int64_t s = s0 + tid;
        int64_t t0 = 0, t1 = 0;
        if (s < p.num_seqs) seq_bounds(p, s, t0, t1);
        const int nch = static_cast<int>((t1 - t0 + kC - 1) / kC);
        int x = nch;  // inclusive warp scan
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int w = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            warp_tot[lane] = w;  // inclusive over warps
        }
        __syncthreads();
        const long long excl = carry_s + (warp > 0 ? warp_tot[warp - 1] : 0) + (x - nch);
        if (s < p.num_seqs) {
            base[s] = static_cast<int>(excl < L.R ? excl : L.R);
            for (int j = 0; j < nch; ++j) {
                const long long rec = excl + j;
                if (rec >= L.R) {
                    record_status(16 /* GDN_ERR_DEVICE_BAD_SEQLENS */);
                    break;
                }
                const int64_t ts = t0 + static_cast<int64_t>(j) * kC;
                const int64_t len = t1 - ts < kC ? t1 - ts : kC;
                table[rec] = make_int4(static_cast<int>(s), static_cast<int>(ts), static_cast<int>(len), 0);
            }
        }
        __syncthreads();
        if (tid == 0) carry_s += warp_tot[31];
        __syncthreads();
    }
    if (tid == 0) {
        const long long tot = carry_s;
        base[p.num_seqs] = static_cast<int>(tot < L.R ? tot : L.R);
        reinterpret_cast<int*>(ws + L.off_hdr)[0] = static_cast<int>(tot < L.R ? tot : L.R);
    }
}

// ---------------------------------------------------------------- prepare --
// One CTA (128 threads) per chunk record and v-head: everything the carry's
// chain does not need, finished per chunk in fp16 operand images (fp32
// accumulation) and bulk-stored to the workspace:
//   M   = G_C I - K'^T W    [k][k']   K-major        (A of the state MMA)
//   K'  = tail (.) K        [j][k]    MN-major       (A of the carry's D = K'^T U)
//   U                       [j][v]    MN-major, two 64-column blocks
//   Qt  = G (.) Q - P W     [i][k]    K-major        (A of the output MMA)
//   Ut  = P U               [i][v]    SW128 rows, two 64-column blocks
// K, Q and V arrive by tiled TMA loads straight into SW128 images (rows past
// the chunk hold the next tokens or zeros; every use masks them).  A^-1 comes
// from an fp32 forward substitution ((I + N) x = e_j, one column per thread);
// W | U = A^-1 [bGK | bV] and the products with P and K' run on tcgen05 with
// two M=64 results packed into TMEM lanes 0-15 / 16-31.
constexpr int kPrepThreads = 128;
constexpr int kPrKQ = 0;        // bf16 [K;Q] K-major, kblock b at b*16K (rows 0-63 K, 64-127 Q); K rows -> K' in place
constexpr int kPrN = 32768;     // fp32 N [64][64], 16-byte chunks swizzled by (row & 15)  -> Ut staging
constexpr int kPrPO = 49152;    // f16 P [64 i][64 j] K-major                              } -> Qt staging
constexpr int kPrX = 57344;     // f16 A^-1 [64 i][64 m] K-major                           }
constexpr int kPrRHS = 65536;   // f16 [bGK | bV] MN-major [64 j][256] (V by TMA) -> [W | U] -> M staging
constexpr int kPrSmall = 98304;
constexpr int kPrSmem = kPrSmall + 1024 + 1024;
constexpr int kPrTmemCols = 256;

struct PrepSmall {
    float LG[kC];    // inclusive prefix of log2 g (0 past the chunk)
    float beta[kC];  // 0 past the chunk
    float wtot[4];
    uint64_t bar_load;
    uint64_t bar_mma;
    uint32_t tmem_base;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// 2^x on the SFU (ex2.approx: a couple of ulp); callers pass x <= 0 where the result is used.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 8 bf16 (one 16-byte chunk) -> 8 floats
__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}

// 8 floats -> 8 fp16 (round-to-nearest) in one 16-byte chunk
__device__ __forceinline__ uint4 f16x8(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __half2 h2 = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
        w[e] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void h16x8_to_f32(uint4 u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        f[2 * e] = p.x;
        f[2 * e + 1] = p.y;
    }
}

__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_shared_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void st_f32(uint8_t* img, uint32_t off, float v) {
    *reinterpret_cast<float*>(img + off) = v;
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// Offset of element (row, col) in a 16-bit SW128 image with `rows` rows per
// 128-byte column block; the same formula serves K-major (row = M/N index)
// and MN-major (row = K index) images, and the TMA SWIZZLE_128B box layout.
__device__ __forceinline__ uint32_t h16(int row, int col, int rows) { return sw128_bf16(row, col, rows); }

// fp32 N image: row i is 256 bytes; its 16-byte chunk c sits at position c ^ (i & 15)
__device__ __forceinline__ uint32_t n_off(int i, int m) { return i * 256 + ((((m >> 2) ^ (i & 15))) << 4); }

__global__ void __launch_bounds__(kPrepThreads, 2)
    gdn_chunk_prepare_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L,
                             const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmV) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    PrepSmall& sml = *reinterpret_cast<PrepSmall*>(sm + kPrSmall);
    const uint32_t aKQ = smem_u32(sm + kPrKQ), aN = smem_u32(sm + kPrN), aPO = smem_u32(sm + kPrPO),
                   aX = smem_u32(sm + kPrX), aRHS = smem_u32(sm + kPrRHS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t rec = blockIdx.x;
    const int h = blockIdx.y, hq = h / kGva;
    const int nrec = reinterpret_cast<const int*>(ws + L.off_hdr)[0];
    if (rec >= nrec) return;
    const int4 te = reinterpret_cast<const int4*>(ws + L.off_table)[rec];
    const int t0 = te.y;  // first token (T < 2^31, checked on the host)
    const int n = te.z;   // tokens in this chunk (1..64)
    uint8_t* out_rec = ws + L.off_rec + (rec * kHV + h) * kHeadRecBytes;

    const uint32_t barL = smem_u32(&sml.bar_load), barM = smem_u32(&sml.bar_mma);
    if (tid == 0) {
        mbar_init(barL, 1);
        mbar_init(barM, 1);
        fence_mbar_init();
        mbar_expect_tx(barL, 6 * 8192);
        tma_load_3d(aKQ, &tmK, 0, hq, t0, barL);
        tma_load_3d(aKQ + 16384, &tmK, 64, hq, t0, barL);
        tma_load_3d(aKQ + 8192, &tmQ, 0, hq, t0, barL);
        tma_load_3d(aKQ + 24576, &tmQ, 64, hq, t0, barL);
        tma_load_3d(aRHS + 16384, &tmV, 0, h, t0, barL);
        tma_load_3d(aRHS + 24576, &tmV, 64, h, t0, barL);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&sml.tmem_base), kPrTmemCols);
        tmem_relinquish();
    }
    // gates and the inclusive prefix of log2 g (threads 0-63 = tokens; warp scans)
    float lgs = 0.f;
    if (tid < kC) {
        float lg = 0.f, bt = 0.f;
        if (tid < n) {
            const int64_t t = static_cast<int64_t>(t0) + tid;
            lg = gdn_log2_decay(p.A_log[h], p.dt_bias[h], bf16_bits_to_float(p.a[t * kHV + h]));
            bt = 1.0f / (1.0f + expf(-bf16_bits_to_float(p.b[t * kHV + h])));
        }
        lgs = lg;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, lgs, o);
            if (lane >= o) lgs += y;
        }
        if (lane == 31) sml.wtot[warp] = lgs;
        sml.beta[tid] = bt;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid >= 32 && tid < kC) lgs += sml.wtot[0];
    if (tid < kC) sml.LG[tid] = lgs;
    const uint32_t tm = sml.tmem_base;
    __syncthreads();
    bool ok = mbar_wait(barL, 0);

    // 1. Gram [K;Q] K^T (bf16, M=128, N=64, K=128) -> TMEM columns 0-63
    if (tid == 0 && ok) {
        tc_fence_after();
        mma_ct<kBF16, false, false, kD, 128, 128, 128, 64>(tm, aKQ, aKQ, false);
        mma_commit(barM);
    }
    // meanwhile: [bGK | bV] in fp16 over the RHS (the scale depends on the row
    // only, so 16-byte chunks convert in place of their swizzled position)
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
        const int u = it * kPrepThreads + tid;
        const int blk = u >> 9;  // 0, 1: K kblocks -> RHS columns 0-127; 2, 3: V blocks in place
        const int row = (u >> 3) & 63;
        const uint32_t in_row = row * 128 + (u & 7) * 16;
        const uint32_t src = blk < 2 ? aKQ + blk * 16384 + in_row : aRHS + blk * 8192 + in_row;
        const float sc = blk < 2 ? sml.beta[row] * fast_exp2(sml.LG[row]) : sml.beta[row];
        const bool act = row < n;
        float f[8];
        bf16x8_to_f32(ld_shared_u4(src), f);
#pragma unroll
        for (int q = 0; q < 8; ++q) f[q] = act ? sc * f[q] : 0.f;
        st_shared_u4(aRHS + blk * 8192 + in_row, f16x8(f));
    }
    ok = mbar_wait(barM, 0) && ok;
    tc_fence_after();
    {
        // 2. Gram epilogue (thread = accumulator row): rows 0-63 give N (fp32),
        //    rows 64-127 the output-side P = Gam (.) Q K^T, j <= i (f16 image)
        float g[64];
        {
            float t32[32];
            tmem_ld32(taddr(tm, 32 * warp, 0), t32);
#pragma unroll
            for (int j = 0; j < 32; ++j) g[j] = t32[j];
            tmem_ld32(taddr(tm, 32 * warp, 32), t32);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) g[32 + j] = t32[j];
        }
        if (warp < 2) {
            const int i = tid;
            const float LGi = sml.LG[i], bi = sml.beta[i];
            const bool act = i < n;
#pragma unroll
            for (int j0 = 0; j0 < kC; j0 += 4) {
                float nv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = j0 + e;
                    nv[e] = (j < i && act) ? bi * fast_exp2(LGi - sml.LG[j]) * g[j] : 0.f;
                }
                st_shared_v4(aN + n_off(i, j0), make_float4(nv[0], nv[1], nv[2], nv[3]));
            }
        } else {
            const int i = tid - 64;
            const float LGi = sml.LG[i];
#pragma unroll
            for (int j0 = 0; j0 < kC; j0 += 8) {
                float pv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int j = j0 + e;
                    pv[e] = (j <= i) ? fast_exp2(LGi - sml.LG[j]) * g[j] : 0.f;
                }
                st_shared_u4(aPO + h16(i, j0, 64), f16x8(pv));
            }
        }
    }
    tc_fence_before();
    if (__syncthreads_or(!ok)) goto abort;
    if (warp < 2) {
        // 3a. A^-1 = (I + N)^-1 by forward substitution, column j = tid, fp32
        //     (eight independent partial sums per row keep the FMA chains short)
        const int j = tid;
        float x[kC];
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            float a[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = 0.f;
            a[0] = (i == j) ? 1.f : 0.f;
#pragma unroll
            for (int m0 = 0; m0 < i; m0 += 4) {
                const float4 nv = ld_shared_v4(aN + n_off(i, m0));
                const int s = ((m0 >> 2) & 1) * 4;
                a[s + 0] = fmaf(-nv.x, x[m0], a[s + 0]);
                if (m0 + 1 < i) a[s + 1] = fmaf(-nv.y, x[m0 + 1], a[s + 1]);
                if (m0 + 2 < i) a[s + 2] = fmaf(-nv.z, x[m0 + 2], a[s + 2]);
                if (m0 + 3 < i) a[s + 3] = fmaf(-nv.w, x[m0 + 3], a[s + 3]);
            }
            x[i] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
        }
#pragma unroll
        for (int i = 0; i < kC; ++i) st_shared_u16(aX + h16(i, j, 64), __half_as_ushort(__float2half_rn(x[i])));
    } else {
        // 3b. K' = tail (.) K in place over the K rows of [K;Q] (rows >= n zero)
        const float LGc = sml.LG[kC - 1];
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
            const int u = it * 64 + (tid - 64);
            const int kb = u >> 9, row = (u >> 3) & 63;
            const uint32_t addr = aKQ + kb * 16384 + row * 128 + (u & 7) * 16;
            const float sc = fast_exp2(LGc - sml.LG[row]);
            const bool act = row < n;
            float f[8];
            bf16x8_to_f32(ld_shared_u4(addr), f);
#pragma unroll
            for (int q = 0; q < 8; ++q) f[q] = act ? sc * f[q] : 0.f;
            st_shared_u4(addr, f16x8(f));
        }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {  // 4. W | U = A^-1 [bGK | bV]: W -> lanes 0-15, U -> lanes 16-31 (columns 0-127)
        tc_fence_after();
        mma_ct<kF16, false, true, 64, 64, 64, 64, 128>(taddr(tm, 0, 0), aX, aRHS, false);
        mma_ct<kF16, false, true, 64, 64, 64, 64, 128>(taddr(tm, 16, 0), aX, aRHS + 16384, false);
        mma_commit(barM);
        bulk_s2g(out_rec + kRecKb, aKQ, 8192);  // K' (final): two 8 KiB kblocks
        bulk_s2g(out_rec + kRecKb + 8192, aKQ + 16384, 8192);
        bulk_commit();
    }
    ok = mbar_wait(barM, 1) && ok;
    tc_fence_after();
    {  // W | U rows -> fp16 MN-major B image over the RHS (W columns 0-127, U 128-255)
        const int i = 16 * warp + (lane & 15);
        const uint32_t dst = aRHS + (lane >= 16 ? 16384 : 0);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            float acc[32];
            tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
            tmem_wait_ld();
#pragma unroll
            for (int j0 = 0; j0 < 32; j0 += 8) st_shared_u4(dst + h16(i, 32 * c + j0, 64), f16x8(acc + j0));
        }
    }
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) goto abort;
    if (tid == 0) {  // 5. P W -> lanes 0-15, P U -> lanes 16-31 (columns 0-127); K'^T W (M=128) -> columns 128-255
        tc_fence_after();
        mma_ct<kF16, false, true, 64, 64, 64, 64, 128>(taddr(tm, 0, 0), aPO, aRHS, false);
        mma_ct<kF16, false, true, 64, 64, 64, 64, 128>(taddr(tm, 16, 0), aPO, aRHS + 16384, false);
        mma_ct<kF16, true, true, 64, 128, 64, 128, 128>(taddr(tm, 0, 128), aKQ, aRHS, false);
        mma_commit(barM);
        bulk_s2g(out_rec + kRecU, aRHS + 16384, 16384);  // U: two 64-column MN-major blocks
        bulk_commit();
    }
    ok = mbar_wait(barM, 0) && ok;
    if (tid == 0) bulk_wait_read_all();  // U and K' have left shared memory before it is reused
    tc_fence_after();
    if (__syncthreads_or(!ok)) goto abort;
    {
        // 6a. Qt = G (.) Q - P W (lanes 0-15) and Ut = P U (lanes 16-31), row i
        const int i = 16 * warp + (lane & 15);
        const bool act = i < n;
        const float Gi = fast_exp2(sml.LG[i]);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            float acc[32];
            tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
            tmem_wait_ld();
            if (lane < 16) {
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 8) {
                    const int col = 32 * c + j0;
                    float qf[8];
                    bf16x8_to_f32(ld_shared_u4(aKQ + h16(64 + i, col, 128)), qf);
#pragma unroll
                    for (int q = 0; q < 8; ++q) qf[q] = act ? Gi * qf[q] - acc[j0 + q] : 0.f;
                    st_shared_u4(aPO + h16(i, col, 64), f16x8(qf));  // Qt staging over P and A^-1
                }
            } else {
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 8) {
                    const int col = 32 * c + j0;
                    float uf[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) uf[q] = act ? acc[j0 + q] : 0.f;
                    st_shared_u4(aN + (col >> 6) * 8192 + h16(i, col & 63, 64), f16x8(uf));  // Ut staging over N
                }
            }
        }
        // 6b. M = G_C I - K'^T W, row k = tid (f16 K-major, staging over the RHS)
        const float Gc = fast_exp2(sml.LG[kC - 1]);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            float acc[32];
            tmem_ld32(taddr(tm, 32 * warp, 128 + 32 * c), acc);
            tmem_wait_ld();
#pragma unroll
            for (int j0 = 0; j0 < 32; j0 += 8) {
                float f[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) f[q] = (32 * c + j0 + q == tid ? Gc : 0.f) - acc[j0 + q];
                st_shared_u4(aRHS + h16(tid, 32 * c + j0, 128), f16x8(f));
            }
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        bulk_s2g(out_rec + kRecQt, aPO, 16384);
        bulk_s2g(out_rec + kRecUt, aN, 16384);
        bulk_s2g(out_rec + kRecM, aRHS, 32768);
        bulk_commit();
        bulk_wait_all();
    }
    goto done;
abort:
    if (tid == 0) {
        record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
        mbar_wait(barL, 0);  // the input loads may still be in flight (bounded)
        bulk_wait_all();
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, kPrTmemCols);
    }
}

// ------------------------------------------------------------------ carry --
// One CTA per sequence x v-head x 64 value rows; the chunk-to-chunk chain
//   S_{c+1}^T = K'_c^T U_c + M_c S_c^T
// is one 12-instruction accumulation per chunk (the K'^T U part issued a chunk
// early into the second accumulator).  Warp roles:
//   warp 8 (one thread)  issues every MMA and bulk copy;
//   warps 0-3 (state)    read the accumulator (thread k = state column k),
//                        write the next fp16 state image, and at the end the
//                        fp32 final state;
//   warps 4-7 (output)   O_c = scale (Qt_c S_c^T + Ut_c) from a second MMA on
//                        the same state image, overlapped with the next chunk.
// M is double-buffered, [K' | U] and Qt triple-buffered, each refilled once
// the MMA that read it is known complete, two chunks before use.
constexpr int kCarryBV = 64;
constexpr int kCarryThreads = 288;
constexpr int kCaM = 0;                          // f16 M K-major [128][128], 2 x 32 KiB
constexpr int kCaKU = 65536;                     // K' [64 j][128 k] (16 KiB) + U tile [64 j][64 v] (8 KiB), 3 x
constexpr int kCaKUBytes = 24576;
constexpr int kCaQt = kCaKU + 3 * kCaKUBytes;    // f16 Qt K-major [64][128], 3 x 16 KiB
constexpr int kCaSI = kCaQt + 3 * 16384;         // f16 S MN-major [128 k][64 v], 2 x 16 KiB
constexpr int kCaSmall = kCaSI + 2 * 16384;
constexpr int kCaSmem = kCaSmall + 256 + 1024;
constexpr int kCaTmemCols = 256;                 // accS x 2 (columns 0-127), accO x 2 (128-255)

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(kCarryThreads, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, const uint8_t* __restrict__ ws, const WsLayout L) {
    constexpr int BV = kCarryBV;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const uint32_t aM = smem_u32(sm + kCaM), aKU = smem_u32(sm + kCaKU), aQt = smem_u32(sm + kCaQt),
                   aSI = smem_u32(sm + kCaSI);
    const uint32_t bar0 = smem_u32(sm + kCaSmall);
    auto fullM = [&](int b) { return bar0 + 8 * b; };         // 2
    auto fullKU = [&](int b) { return bar0 + 16 + 8 * b; };   // 3
    auto fullQt = [&](int b) { return bar0 + 40 + 8 * b; };   // 3
    const uint32_t mmaS = bar0 + 64;
    auto mmaO = [&](int b) { return bar0 + 72 + 8 * b; };     // 2
    const uint32_t imgReady = bar0 + 88;
    auto oFree = [&](int b) { return bar0 + 96 + 8 * b; };    // 2
    const uint32_t drain = bar0 + 112;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kCaSmall + 128);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t unit = blockIdx.x >> 1;
    const int vt = blockIdx.x & 1;
    const int64_t s = unit / kHV;
    const int h = static_cast<int>(unit - s * kHV);
    const int v0 = vt * BV;

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    const int len = static_cast<int>(t1 - t0);
    const int nch = (len + kC - 1) / kC;
    const int rec0 = reinterpret_cast<const int*>(ws + L.off_base)[s];
    if (nch == 0 || rec0 + nch > L.R) {
        if (nch != 0 && tid == 0) record_status(16);
        if (tid < kD) {  // empty sequence: zero state rows (oracle prefill :53-55)
            float* ns_col = p.new_state + (unit * kD + v0) * kD + tid;
#pragma unroll 8
            for (int v = 0; v < BV; ++v) ns_col[v * kD] = 0.f;
        }
        return;
    }
    auto rec_ptr = [&](int c) { return ws + L.off_rec + (static_cast<int64_t>(rec0 + c) * kHV + h) * kHeadRecBytes; };
    auto accS = [&](uint32_t tm, int b) { return tm + 64 * b; };
    auto accO = [&](uint32_t tm, int b) { return tm + 128 + 64 * b; };

    const bool issuer = tid == 256;
    int topM = -1, topKU = -1, topQt = -1;  // issuer: highest chunk whose copy was issued
    auto issue_M = [&](int c) {
        const int b = c & 1;
        mbar_expect_tx(fullM(b), 32768);
        bulk_g2s(aM + b * 32768, rec_ptr(c) + kRecM, 32768, fullM(b));
        topM = c;
    };
    auto issue_KU = [&](int c) {
        const int b = c % 3;
        mbar_expect_tx(fullKU(b), kCaKUBytes);
        bulk_g2s(aKU + b * kCaKUBytes, rec_ptr(c) + kRecKb, 16384, fullKU(b));
        bulk_g2s(aKU + b * kCaKUBytes + 16384, rec_ptr(c) + kRecU + vt * 8192, 8192, fullKU(b));
        topKU = c;
    };
    auto issue_Qt = [&](int c) {
        const int b = c % 3;
        mbar_expect_tx(fullQt(b), 16384);
        bulk_g2s(aQt + b * 16384, rec_ptr(c) + kRecQt, 16384, fullQt(b));
        topQt = c;
    };
    if (issuer) {
        for (int b = 0; b < 2; ++b) mbar_init(fullM(b), 1);
        for (int b = 0; b < 3; ++b) mbar_init(fullKU(b), 1);
        for (int b = 0; b < 3; ++b) mbar_init(fullQt(b), 1);
        mbar_init(mmaS, 1);
        for (int b = 0; b < 2; ++b) mbar_init(mmaO(b), 1);
        mbar_init(imgReady, 4);
        for (int b = 0; b < 2; ++b) mbar_init(oFree(b), 4);
        mbar_init(drain, 1);
        fence_mbar_init();
        for (int c = 0; c < 2 && c < nch; ++c) issue_M(c);
        for (int c = 0; c < 3 && c < nch; ++c) issue_KU(c);
        for (int c = 0; c < 2 && c < nch; ++c) issue_Qt(c);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kCaTmemCols);
        tmem_relinquish();
    }
    if (warp < 4) {  // S_0 -> fp16 state image 0 (thread k = column k; coalesced over k)
        float sv[8];
#pragma unroll
        for (int v = 0; v < BV; v += 8) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
                sv[e] = p.state != nullptr ? p.state[(unit * kD + v0 + v + e) * kD + tid] : 0.f;
            st_shared_u4(aSI + h16(tid, v, kD), f16x8(sv));
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;

    if (issuer) {
        bool ok = mbar_wait(fullKU(0), 0);
        if (ok) {
            tc_fence_after();
            mma_ct<kF16, true, true, 64, 64, 64, 128, BV>(accS(tm, 0), aKU, aKU + 16384, false);  // K'^T U of chunk 0
        }
        for (int c = 0; c < nch && ok; ++c) {
            ok = (c == 0 || mbar_wait(imgReady, (c - 1) & 1)) && mbar_wait(fullM(c & 1), (c >> 1) & 1);
            if (!ok) break;
            tc_fence_after();
            mma_ct<kF16, false, true, kD, 128, kD, 128, BV>(accS(tm, c & 1), aM + (c & 1) * 32768,
                                                           aSI + (c & 1) * 16384, true);
            mma_commit(mmaS);
            if (c + 1 < nch) {  // next chunk's K'^T U into the other accumulator (its reader is done)
                const int b = (c + 1) % 3;
                ok = mbar_wait(fullKU(b), ((c + 1) / 3) & 1);
                if (!ok) break;
                mma_ct<kF16, true, true, 64, 64, 64, 128, BV>(accS(tm, (c + 1) & 1), aKU + b * kCaKUBytes,
                                                             aKU + b * kCaKUBytes + 16384, false);
            }
            ok = mbar_wait(fullQt(c % 3), (c / 3) & 1) && (c < 2 || mbar_wait(oFree(c & 1), ((c - 2) >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            mma_ct<kF16, false, true, kD, 64, kD, 64, BV>(accO(tm, c & 1), aQt + (c % 3) * 16384,
                                                         aSI + (c & 1) * 16384, false);
            mma_commit(mmaO(c & 1));
            // MMA_S(c) complete => so is everything issued before it: refill
            ok = mbar_wait(mmaS, c & 1);
            if (!ok) break;
            if (c + 2 < nch) {
                issue_M(c + 2);
                issue_Qt(c + 2);
            }
            if (c + 3 < nch) issue_KU(c + 3);
        }
        if (!ok) {
            record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
            // wait (bounded) for the copies in flight: per buffer, its latest chunk
            for (int c = topM > 1 ? topM - 1 : 0; c <= topM; ++c) mbar_wait(fullM(c & 1), (c >> 1) & 1);
            for (int c = topKU > 2 ? topKU - 2 : 0; c <= topKU; ++c) mbar_wait(fullKU(c % 3), (c / 3) & 1);
            for (int c = topQt > 2 ? topQt - 2 : 0; c <= topQt; ++c) mbar_wait(fullQt(c % 3), (c / 3) & 1);
            mma_commit(drain);
            mbar_wait(drain, 0);
        }
    } else if (warp < 4) {
        const int k = tid;
        for (int c = 0; c < nch; ++c) {
            const bool okc = __all_sync(0xffffffffu, mbar_wait(mmaS, c & 1));  // warp-uniform exit
            tc_fence_after();
            float a0[32], a1[32];
            tmem_ld32(taddr(accS(tm, c & 1), 32 * warp, 0), a0);
            tmem_ld32(taddr(accS(tm, c & 1), 32 * warp, 32), a1);
            tmem_wait_ld();
            if (!okc) {
                record_status(32);
                break;
            }
            if (c + 1 < nch) {
                const uint32_t img = aSI + ((c + 1) & 1) * 16384;
#pragma unroll
                for (int v = 0; v < 32; v += 8) {
                    st_shared_u4(img + h16(k, v, kD), f16x8(a0 + v));
                    st_shared_u4(img + h16(k, 32 + v, kD), f16x8(a1 + v));
                }
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(imgReady);
            } else {
                float* ns_col = p.new_state + (unit * kD + v0) * kD + k;
#pragma unroll
                for (int v = 0; v < 32; ++v) {
                    ns_col[v * kD] = a0[v];
                    ns_col[(32 + v) * kD] = a1[v];
                }
            }
        }
    } else if (warp < 8) {
        // output rows: token i = 16 (warp - 4) + lane of each chunk (lanes 0-15)
        const int ow = warp - 4;
        const int i = 16 * ow + (lane & 15);
        uint16_t* out = p.out;
        for (int c = 0; c < nch; ++c) {
            const int tok = kC * c + i;
            const bool act = lane < 16 && tok < len;
            uint4 ut[8];  // Ut row i, logical 16-byte chunks (stored swizzled by i & 7)
            const uint8_t* urow = rec_ptr(c) + kRecUt + vt * 8192 + i * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                ut[q] = act ? __ldg(reinterpret_cast<const uint4*>(urow + ((q ^ (i & 7)) << 4))) : make_uint4(0, 0, 0, 0);
            const bool okc = __all_sync(0xffffffffu, mbar_wait(mmaO(c & 1), (c >> 1) & 1));
            tc_fence_after();
            float o0[32], o1[32];
            tmem_ld32(taddr(accO(tm, c & 1), 32 * ow, 0), o0);
            tmem_ld32(taddr(accO(tm, c & 1), 32 * ow, 32), o1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(oFree(c & 1));
            if (!okc) {
                if (lane == 0) record_status(32);
                break;
            }
            if (act) {
                uint16_t* dst = out + ((t0 + tok) * kHV + h) * kD + v0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    float u[8];
                    h16x8_to_f32(ut[q], u);
                    const float* o = q < 4 ? o0 + 8 * q : o1 + 8 * (q - 4);
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(p.scale * (o[2 * e] + u[2 * e]),
                                                                        p.scale * (o[2 * e + 1] + u[2 * e + 1]));
                        w[e] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                    *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kCaTmemCols);
    }
}

// ---------------------------------------------------------------- dispatch --
template <typename K>
static cudaError_t set_smem(K kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Path selection: 0 = auto, 1 = token-recurrent, 2 = chunked tensor-core.
constexpr int kPathAuto = 0, kPathRecurrent = 1, kPathChunked = 2;
constexpr int64_t kRecurrentMaxAvgLen = 48;

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); looked up once per process.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// Tensor map of a bf16 [T, heads, 128] token tensor: 3-D (dim, head, token),
// box = 64 dims x 1 head x 64 tokens, SWIZZLE_128B -- one SW128 image of 64
// rows per load; tokens >= T read as zeros.
static cudaError_t token_tensor_map(CUtensorMap* m, const void* base, int heads, int64_t T) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads),
                                static_cast<cuuint64_t>(T)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(heads) * kD * 2};
    const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kC)};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_prefill_chunked(const PrefillParams& p, void* workspace, cudaStream_t stream) {
    const WsLayout L = ws_layout(p.total_tokens, p.num_seqs);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (L.R > 0x7fffffffLL || p.total_tokens > 0x7fffffffLL) return cudaErrorInvalidValue;
    CUtensorMap tmK, tmQ, tmV;
    memset(&tmK, 0, sizeof(tmK));
    memset(&tmQ, 0, sizeof(tmQ));
    memset(&tmV, 0, sizeof(tmV));
    cudaError_t e;
    if (p.total_tokens > 0) {  // with no tokens there are no records and no loads
        if ((e = token_tensor_map(&tmK, p.k, kHQK, p.total_tokens)) != cudaSuccess) return e;
        if ((e = token_tensor_map(&tmQ, p.q, kHQK, p.total_tokens)) != cudaSuccess) return e;
        if ((e = token_tensor_map(&tmV, p.v, kHV, p.total_tokens)) != cudaSuccess) return e;
    }
    gdn_chunk_table_kernel<<<1, 1024, 0, stream>>>(p, ws, L);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_prepare_kernel, kPrSmem)) != cudaSuccess) return e;
    gdn_chunk_prepare_kernel<<<dim3(static_cast<unsigned>(L.R), kHV), kPrepThreads, kPrSmem, stream>>>(
        p, ws, L, tmK, tmQ, tmV);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_carry_kernel, kCaSmem)) != cudaSuccess) return e;
    const int64_t grid = p.num_seqs * kHV * (kD / kCarryBV);
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_chunk_carry_kernel<<<static_cast<unsigned>(grid), kCarryThreads, kCaSmem, stream>>>(p, ws, L);
    return cudaGetLastError();
}

cudaError_t launch_prefill(const PrefillParams& p, int path, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
    const int64_t avg = p.total_tokens / (p.num_seqs > 0 ? p.num_seqs : 1);
    const bool recurrent = path == kPathRecurrent || (path == kPathAuto && avg <= kRecurrentMaxAvgLen);
    if (recurrent) return launch_prefill_recurrent(p, stream);
    if (workspace == nullptr || workspace_bytes < chunked_workspace_bytes(p.total_tokens, p.num_seqs))
        return cudaErrorInvalidValue;
    return launch_prefill_chunked(p, workspace, stream);
}

// ------------------------------------------------------------- self-test --
// D[M x N] = A[M x K] . B[N x K]^T through the same image writers,
// descriptors and TMEM read-back as the kernels above (one CTA).  flags:
// bit 0 A MN-major, bit 1 B MN-major, bit 2 accumulator at TMEM lane 16
// (the second M=64 tile of a lane-packed pair; M = 64 only).
template <Kind KIND>
__device__ __forceinline__ void selftest_issue(int flags, uint32_t d, uint32_t a, uint32_t b, int M, int N, int K) {
    const int ar = (flags & 1) ? K : M, br = (flags & 2) ? K : N;
    switch (flags & 3) {
        case 0: mma_tile<KIND, false, false>(d, a, ar, b, br, K, M, N, false); break;
        case 1: mma_tile<KIND, true, false>(d, a, ar, b, br, K, M, N, false); break;
        case 2: mma_tile<KIND, false, true>(d, a, ar, b, br, K, M, N, false); break;
        default: mma_tile<KIND, true, true>(d, a, ar, b, br, K, M, N, false); break;
    }
}

__global__ void __launch_bounds__(128, 1)
    gdn_mma_selftest_kernel(int kind, int flags, int M, int N, int K, const void* A, const void* B, float* D) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int eb = kind == kTF32 ? 4 : 2;
    const int kblocks = K * eb / 128;
    const bool a_mn = flags & 1, b_mn = flags & 2, lane16 = flags & 4;
    uint8_t* sA = sm;
    uint8_t* sB = sm + M * K * eb;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sB + N * K * eb);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    (void)kblocks;
    for (int idx = tid; idx < M * K; idx += 128) {
        const int r = idx / K, c = idx % K;  // A[r][c]: row m = r, k = c
        const int row = a_mn ? c : r, col = a_mn ? r : c, rows = a_mn ? K : M;
        if (kind != kTF32)
            *reinterpret_cast<uint16_t*>(sA + sw128_bf16(row, col, rows)) = static_cast<const uint16_t*>(A)[idx];
        else
            st_f32(sA, a_mn ? mn32_f32(row, col, rows) : sw128_f32(row, col, rows),
                   to_tf32(static_cast<const float*>(A)[idx]));
    }
    for (int idx = tid; idx < N * K; idx += 128) {
        const int r = idx / K, c = idx % K;  // B[r][c]: n = r, k = c
        const int row = b_mn ? c : r, col = b_mn ? r : c, rows = b_mn ? K : N;
        if (kind != kTF32)
            *reinterpret_cast<uint16_t*>(sB + sw128_bf16(row, col, rows)) = static_cast<const uint16_t*>(B)[idx];
        else
            st_f32(sB, b_mn ? mn32_f32(row, col, rows) : sw128_f32(row, col, rows),
                   to_tf32(static_cast<const float*>(B)[idx]));
    }
    int ncols = 32;
    while (ncols < N) ncols <<= 1;
    if (tid == 0) {
        mbar_init(smem_u32(bar), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tslot), ncols);
        tmem_relinquish();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    const uint32_t d = lane16 ? taddr(tm, 16, 0) : tm;
    if (tid == 0) {
        if (kind == kBF16)
            selftest_issue<kBF16>(flags, d, smem_u32(sA), smem_u32(sB), M, N, K);
        else if (kind == kF16)
            selftest_issue<kF16>(flags, d, smem_u32(sA), smem_u32(sB), M, N, K);
        else
            selftest_issue<kTF32>(flags, d, smem_u32(sA), smem_u32(sB), M, N, K);
        mma_commit(smem_u32(bar));
    }
    const bool ok = mbar_wait(smem_u32(bar), 0);
    tc_fence_after();
    // M=128: row = lane of the whole CTA; M=64: lanes 0-15 (or 16-31) of each warp
    int row;
    bool has_row;
    if (M == 128) {
        row = tid;
        has_row = true;
    } else {
        row = 16 * warp + (lane & 15);
        has_row = lane16 ? lane >= 16 : lane < 16;
    }
    for (int c = 0; c < N; c += 16) {
        float r16[16];
        tmem_ld16(taddr(tm, 32 * warp, c), r16);
        tmem_wait_ld();
        if (has_row && ok)
            for (int j = 0; j < 16; ++j) D[row * N + c + j] = r16[j];
    }
    if (!ok && tid == 0) record_status(32);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, ncols);
    }
}

cudaError_t launch_mma_selftest(int kind, int flags, int M, int N, int K, const void* A, const void* B, float* D,
                                cudaStream_t stream) {
    // the whole opt-in shared memory, so even a misread descriptor stride stays inside the CTA's window
    const int smem = 227 * 1024;
    cudaError_t e = set_smem(gdn_mma_selftest_kernel, smem);
    if (e != cudaSuccess) return e;
    gdn_mma_selftest_kernel<<<1, 128, smem, stream>>>(kind, flags, M, N, K, A, B, D);
    return cudaGetLastError();
}

}  // namespace gdn
