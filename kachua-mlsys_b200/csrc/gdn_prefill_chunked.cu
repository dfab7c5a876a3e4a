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
#include "gdn_common.cuh"
#include "tc05.cuh"

namespace gdn {
using namespace tc05;

constexpr int kC = 64;
constexpr int kMImg = kD * kD * 2;        // f16 M K-major [128 k][128 k']        32 KiB
constexpr int kDBytes = kD * kD * 4;       // fp32 D rows [128 k][128 v]            64 KiB
constexpr int kQtImg = kC * kD * 2;        // f16 Qt K-major [64 i][128 k]           16 KiB
constexpr int kUtBytes = kC * kD * 2;      // f16 Ut [2 halves][64 i][64 v]          16 KiB
constexpr int kRecordBytes = kHV * (kMImg + kDBytes + kQtImg + kUtBytes);

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace: header, per-sequence record bases, the chunk table and the
// per-record, per-head operand arrays (every array 1024-byte aligned).
struct WsLayout {
    int64_t R;  // record capacity: ceil(T / 64) + N bounds sum_s ceil(len_s / 64)
    int64_t off_hdr, off_base, off_table, off_m, off_d, off_qt, off_ut, total;
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
    L.off_m = o;
    o += L.R * kHV * kMImg;
    L.off_d = o;
    o += L.R * kHV * kDBytes;
    L.off_qt = o;
    o += L.R * kHV * kQtImg;
    L.off_ut = o;
    o += L.R * kHV * kUtBytes;
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
// One CTA (128 threads) per chunk record and q/k head.  Everything the carry
// kernel's state chain does not need is finished here, in fp16 operand images
// (round-to-nearest; fp32 accumulation), per v-head h:
//   M  = G_C I - (tail K)^T W          [k][k']  fp16 K-major  (the carry's A operand)
//   D  = (tail K)^T U                  [k][v]   fp32 rows
//   Qt = G (.) Q - P W                 [i][k]   fp16 K-major  (the output MMA's A operand)
//   Ut = P U                           [i][v]   fp16, two 64-column halves
// so that one chunk of the carry is S1 = S0 M^T + D and O = scale (Qt S0^T + Ut).
// The two v-heads of the q/k head share every M=64 accumulator (head 0 in TMEM
// lanes 0-15, head 1 in lanes 16-31 of each warp's sub-partition); in those
// epilogues thread (warp w, lane l) owns row 16w + (l & 15) of head l >> 4.
constexpr int kPrepKQ = 0;          // bf16 [K;Q] K-major, 2 kblocks x 128 rows                 32 KiB
constexpr int kPrepX = 0;           // f16 X_h K-major [64][64] (Neumann iterate -> A^-1), over KQ  2 x 8 KiB
constexpr int kPrepPA = 16384;      // f16 power P_h K-major [64][64]                              2 x 8 KiB
constexpr int kPrepPB = 32768;      // f16 power P_h MN-major                                      2 x 8 KiB
constexpr int kPrepPO = 49152;      // f16 output-side P_h K-major [64 i][64 j]                    2 x 8 KiB
constexpr int kPrepRHS = 65536;     // f16 [beta G K | beta V] MN-major [64 j][256] -> then [W | U]  32 KiB
constexpr int kPrepKB = 16384;      // f16 tail K MN-major [64 j][128 k] over PA/PB (after Neumann) 16 KiB
constexpr int kPrepSmall = 98304;
constexpr int kPrepSmem = kPrepSmall + 2048 + 1024;
constexpr int kPrepTmemCols = 256;

struct PrepSmall {
    float lg[2][kC];   // log2 g per token (0 for inactive rows)
    float LG[2][kC];   // inclusive prefix of lg
    float beta[2][kC];
    uint64_t bar_mma;
    uint32_t tmem_base;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void st_f32(uint8_t* img, uint32_t off, float v) {
    *reinterpret_cast<float*>(img + off) = v;
}

__device__ __forceinline__ float4 tf32x4(float a, float b, float c, float d) {
    return make_float4(to_tf32(a), to_tf32(b), to_tf32(c), to_tf32(d));
}

// 2^x on the SFU (ex2.approx: a couple of ulp); x <= 0 here, so no overflow.
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

__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_shared_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
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

// Offset of element (row, col) in a 16-bit SW128 image with `rows` rows per
// 128-byte column block; the same formula serves K-major (row = M/N index)
// and MN-major (row = K index) images.
__device__ __forceinline__ uint32_t h16(int row, int col, int rows) { return sw128_bf16(row, col, rows); }

__global__ void __launch_bounds__(128, 2)
    gdn_chunk_prepare_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sKQ = sm + kPrepKQ;
    PrepSmall& sml = *reinterpret_cast<PrepSmall*>(sm + kPrepSmall);
    const uint32_t aKQ = smem_u32(sKQ), aX = smem_u32(sm + kPrepX), aPA = smem_u32(sm + kPrepPA),
                   aPB = smem_u32(sm + kPrepPB), aPO = smem_u32(sm + kPrepPO), aRHS = smem_u32(sm + kPrepRHS),
                   aKB = smem_u32(sm + kPrepKB);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t rec = blockIdx.x;
    const int hq = blockIdx.y;
    const int nrec = reinterpret_cast<const int*>(ws + L.off_hdr)[0];
    if (rec >= nrec) return;
    const int4 te = reinterpret_cast<const int4*>(ws + L.off_table)[rec];
    const int64_t t0 = te.y;
    const int n = te.z;

    const uint32_t bar = smem_u32(&sml.bar_mma);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&sml.tmem_base), kPrepTmemCols);
        tmem_relinquish();
    }

    // 1. K and Q tiles -> [K;Q] bf16 image (rows >= n zero); gates of both v-heads
#pragma unroll 4
    for (int idx = tid; idx < 2 * kC * 16; idx += 128) {
        const int m = idx >> 10;  // 0: K, 1: Q
        const int row = (idx >> 4) & 63;
        const int ch = idx & 15;  // 16-byte chunk of the 256-byte row
        uint4 val = make_uint4(0, 0, 0, 0);
        if (row < n) val = *reinterpret_cast<const uint4*>((m ? p.q : p.k) + ((t0 + row) * kHQK + hq) * kD + ch * 8);
        const int r = 64 * m + row;
        *reinterpret_cast<uint4*>(sKQ + (ch >> 3) * (128 * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) = val;
    }
    {
        const int hl = tid >> 6, i = tid & 63, h = 2 * hq + hl;
        float lg = 0.f, bt = 0.f;
        if (i < n) {
            const int64_t t = t0 + i;
            lg = gdn_log2_decay(p.A_log[h], p.dt_bias[h], bf16_bits_to_float(p.a[t * kHV + h]));
            bt = 1.0f / (1.0f + expf(-bf16_bits_to_float(p.b[t * kHV + h])));
        }
        sml.lg[hl][i] = lg;
        sml.beta[hl][i] = bt;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sml.tmem_base;
    uint32_t phase = 0;
    bool ok = true, aborted = false;
    const int hl = lane >> 4;               // head of this thread in packed M=64 epilogues
    const int row = 16 * warp + (lane & 15);  // its row there

    // 2. Gram: rows 0-63 K K^T, rows 64-127 Q K^T (bf16, M=128, N=64, K=128)
    if (tid == 0) {
        mma_ct<kBF16, false, false, kD, 128, 128, 128, 64>(tm, aKQ, aKQ, false);
        mma_commit(bar);
    }
    {  // inclusive prefix of log2 g (64 sequential adds; deterministic)
        const int h2 = tid >> 6, i = tid & 63;
        float acc = 0.f;
        for (int m = 0; m <= i; ++m) acc += sml.lg[h2][m];
        sml.LG[h2][i] = acc;
    }
    __syncthreads();
    ok = mbar_wait(bar, phase);
    phase ^= 1;
    tc_fence_after();
    __syncthreads();  // every thread is past the Gram MMA before X overwrites [K;Q]
    {
        // 3. Gram epilogue (M=128 rows: thread = row).  Rows 0-63 build N, its
        //    two operand copies and X = I - N of both heads; rows 64-127 the
        //    output-side P = Gam (.) Q K^T (j <= i).
        float gram[64];
        {
            float t32[32];
            tmem_ld32(taddr(tm, 32 * warp, 0), t32);
#pragma unroll
            for (int j = 0; j < 32; ++j) gram[j] = t32[j];
            tmem_ld32(taddr(tm, 32 * warp, 32), t32);
#pragma unroll
            for (int j = 0; j < 32; ++j) gram[32 + j] = t32[j];
            tmem_wait_ld();
        }
        const int i = tid & 63;
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {
            const float LGi = sml.LG[h2][i];
            if (tid < 64) {
                const float bi = sml.beta[h2][i];
#pragma unroll
                for (int j0 = 0; j0 < 64; j0 += 8) {
                    float nv[8], xv[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int j = j0 + e;
                        nv[e] = (j < i) ? bi * fast_exp2(LGi - sml.LG[h2][j]) * gram[j] : 0.f;
                        xv[e] = (j == i ? 1.f : 0.f) - nv[e];
                    }
                    const uint4 nh = f16x8(nv);
                    st_shared_u4(aPA + h2 * 8192 + h16(i, j0, 64), nh);
                    st_shared_u4(aPB + h2 * 8192 + h16(i, j0, 64), nh);
                    st_shared_u4(aX + h2 * 8192 + h16(i, j0, 64), f16x8(xv));
                }
            } else {
#pragma unroll
                for (int j0 = 0; j0 < 64; j0 += 8) {
                    float pv[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int j = j0 + e;
                        pv[e] = (j <= i) ? fast_exp2(LGi - sml.LG[h2][j]) * gram[j] : 0.f;
                    }
                    st_shared_u4(aPO + h2 * 8192 + h16(i, j0, 64), f16x8(pv));
                }
            }
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // Neumann round 0: N_h^2 for both heads (lanes 16 h, columns 64-127)
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h)
            mma_ct<kF16, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 64), aPA + h * 8192, aPB + h * 8192,
                                                         false);
        mma_commit(bar);
    }
    // 4. Neumann doubling, both heads packed: epilogue e updates X (e >= 1) and P (e <= 4)
    for (int e = 0; e <= 5; ++e) {
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        if (e >= 1) {
            const uint32_t xa = aX + hl * 8192;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float xp[32];
                tmem_ld32(taddr(tm, 32 * warp, 32 * half), xp);
                tmem_wait_ld();
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 8) {
                    const uint32_t off = xa + h16(row, 32 * half + j0, 64);
                    float x[8];
                    h16x8_to_f32(ld_shared_u4(off), x);
#pragma unroll
                    for (int q = 0; q < 8; ++q) x[q] += xp[j0 + q];
                    st_shared_u4(off, f16x8(x));
                }
            }
        }
        if (e <= 4) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float pp[32];
                tmem_ld32(taddr(tm, 32 * warp, 64 + 32 * half), pp);
                tmem_wait_ld();
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 8) {
                    const uint4 t = f16x8(pp + j0);
                    st_shared_u4(aPA + hl * 8192 + h16(row, 32 * half + j0, 64), t);
                    st_shared_u4(aPB + hl * 8192 + h16(row, 32 * half + j0, 64), t);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            goto done;
        }
        if (tid == 0 && e <= 4) {
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                mma_ct<kF16, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 0), aX + h * 8192, aPB + h * 8192,
                                                             false);  // X P
                if (e <= 3)
                    mma_ct<kF16, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 64), aPA + h * 8192,
                                                                 aPB + h * 8192, false);  // P P
            }
            mma_commit(bar);
        }
    }
    // 5. per head: [beta G K | beta V] and tail K, then [W | U] = A^-1 [..], then
    //    P [W | U] and (tail K)^T [W | U]; results straight to the workspace
#pragma unroll 1
    for (int h2 = 0; h2 < 2; ++h2) {
        const int h = 2 * hq + h2;
        const int64_t rh = rec * kHV + h;
        {
            const int j = tid & 63, part = tid >> 6;
            const float LGj = sml.LG[h2][j], bj = sml.beta[h2][j];
            const float Gj = exp2f(LGj), tail = exp2f(sml.LG[h2][63] - LGj);
            const bool act = j < n;
            if (part == 0) {  // K row j: beta G K -> RHS columns 0-127, tail K -> K-bar
                const uint16_t* ksrc = p.k + ((t0 + j) * kHQK + hq) * kD;
                const float s = bj * Gj;
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8], a[8], b[8];
                    bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(ksrc + d0) : make_uint4(0, 0, 0, 0), f);
#pragma unroll
                    for (int q = 0; q < 8; ++q) a[q] = s * f[q], b[q] = tail * f[q];
                    st_shared_u4(aRHS + h16(j, d0, 64), f16x8(a));
                    st_shared_u4(aKB + h16(j, d0, 64), f16x8(b));
                }
            } else {  // V row j: beta V -> RHS columns 128-255
                const uint16_t* vsrc = p.v + ((t0 + j) * kHV + h) * kD;
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8], a[8];
                    bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(vsrc + d0) : make_uint4(0, 0, 0, 0), f);
#pragma unroll
                    for (int q = 0; q < 8; ++q) a[q] = bj * f[q];
                    st_shared_u4(aRHS + h16(j, 128 + d0, 64), f16x8(a));
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            mma_ct<kF16, false, true, 64, 64, 64, 64, 256>(tm, aX + h2 * 8192, aRHS, false);  // [W | U], lanes 0-15
            mma_commit(bar);
        }
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        // [W | U] rows (lanes 0-15: this head) -> fp16 MN-major B image over the RHS;
        // every lane takes part in the (warp-collective) TMEM loads
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
            float acc[32];
            tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
            tmem_wait_ld();
            if ((lane & 16) == 0) {
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 8) st_shared_u4(aRHS + h16(row, 32 * c + j0, 64), f16x8(acc + j0));
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            goto done;
        }
        if (tid == 0) {  // P [W | U] (M=64, lanes 0-15, columns 0-255)
            tc_fence_after();
            mma_ct<kF16, false, true, 64, 64, 64, 64, 256>(tm, aPO + h2 * 8192, aRHS, false);
            mma_commit(bar);
        }
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        {  // Qt = G (.) Q - P W and Ut = P U (rows i = row, lanes 0-15)
            const float Gi = exp2f(sml.LG[h2][row & 63]);
            const bool act = (row & 63) < n;
            const uint16_t* qsrc = p.q + ((t0 + (row & 63)) * kHQK + hq) * kD;
            uint8_t* gqt = ws + L.off_qt + rh * kQtImg;
            uint16_t* gut = reinterpret_cast<uint16_t*>(ws + L.off_ut + rh * kUtBytes);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                float acc[32];
                tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
                tmem_wait_ld();
                if ((lane & 16) == 0) {
                    if (c < 4) {
#pragma unroll
                        for (int j0 = 0; j0 < 32; j0 += 8) {
                            float f[8];
                            bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(qsrc + 32 * c + j0)
                                              : make_uint4(0, 0, 0, 0),
                                          f);
#pragma unroll
                            for (int q = 0; q < 8; ++q) f[q] = Gi * f[q] - acc[j0 + q];
                            *reinterpret_cast<uint4*>(gqt + h16(row, 32 * c + j0, 64)) = f16x8(f);
                        }
                    } else {  // Ut: [half][i][64] with half = value column / 64
                        const int v = 32 * (c - 4);
#pragma unroll
                        for (int j0 = 0; j0 < 32; j0 += 8)
                            *reinterpret_cast<uint4*>(gut + ((v + j0) >> 6) * (kC * 64) + row * 64 + ((v + j0) & 63)) =
                                f16x8(acc + j0);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {  // (tail K)^T [W | U] (M=128: rows = state column k)
            tc_fence_after();
            mma_ct<kF16, true, true, 64, 64, 64, 128, 256>(tm, aKB, aRHS, false);
            mma_commit(bar);
        }
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        {  // M = G_C I - (tail K)^T W (row k = tid, fp16 K-major) and D = (tail K)^T U (fp32 rows)
            const float Gc = exp2f(sml.LG[h2][63]);
            uint8_t* gm = ws + L.off_m + rh * kMImg;
            float* gd = reinterpret_cast<float*>(ws + L.off_d + rh * kDBytes) + tid * kD;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                float acc[32];
                tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
                tmem_wait_ld();
                if (c < 4) {
#pragma unroll
                    for (int j0 = 0; j0 < 32; j0 += 8) {
                        float f[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) f[q] = (32 * c + j0 + q == tid ? Gc : 0.f) - acc[j0 + q];
                        *reinterpret_cast<uint4*>(gm + h16(tid, 32 * c + j0, 128)) = f16x8(f);
                    }
                } else {
#pragma unroll
                    for (int j0 = 0; j0 < 32; j0 += 4)
                        *reinterpret_cast<float4*>(gd + 32 * (c - 4) + j0) =
                            make_float4(acc[j0], acc[j0 + 1], acc[j0 + 2], acc[j0 + 3]);
                }
            }
        }
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            goto done;
        }
    }
done:
    if (tid == 0 && aborted) record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(sml.tmem_base, kPrepTmemCols);
    }
}

// ------------------------------------------------------------------ carry --
// One CTA (256 threads) per sequence x v-head x 64 value rows.  The state
// chain needs one tensor-core MMA per chunk:
//   S_{c+1}^T = M_c S_c^T + D_c^T      (M fp16 K-major, S fp16 MN-major, fp32 accumulate)
// Warps 0-3 own the state (thread k = column k of the 64 rows, fp32 registers):
// they add D_c (prefetched one chunk ahead) to the accumulator and write the
// next fp16 state image.  Warps 4-7 finish the outputs off the critical path:
//   O_c = scale (Qt_c S_c^T + Ut_c)    (Qt fp16 K-major; the MMA reads the same state image)
// Thread 0 issues every MMA and bulk copy.  M is double-buffered and
// [Qt | Ut] triple-buffered, each refilled as soon as its readers are done,
// so the copies run a chunk or more ahead of use.
constexpr int kCarryBV = 64;
constexpr int kCarryThreads = 256;
constexpr int kCarMI = 0;                         // f16 M K-major [128 k][128 k'], 2 x 32 KiB
constexpr int kCarQU = 65536;                     // 3 x (Qt f16 K-major [64 i][128 k] 16 KiB + Ut [64 i][64 v] f16 8 KiB)
constexpr int kCarQUBytes = 24576;
constexpr int kCarSI = kCarQU + 3 * kCarQUBytes;  // f16 S MN-major [128 k][64 v], 2 x 16 KiB
constexpr int kCarSmall = kCarSI + 2 * 16384;
constexpr int kCarSmem = kCarSmall + 256 + 1024;
constexpr int kCarTmemCols = 256;                 // accS [0,64), accO x 2 [64,192)

// bar.red.or on named barrier `id` among `count` threads
__device__ __forceinline__ bool named_sync_or(int id, int count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(kCarryThreads, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, const uint8_t* __restrict__ ws, const WsLayout L) {
    constexpr int BV = kCarryBV;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const uint32_t aMI = smem_u32(sm + kCarMI), aQU = smem_u32(sm + kCarQU), aSI = smem_u32(sm + kCarSI);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kCarSmall);
    // fullM[2], fullQ[3], mmaS, mmaO[2], oFree[2], quFree[3]
    const uint32_t bar0 = smem_u32(bars);
    auto fullM = [&](int b) { return bar0 + 8 * b; };
    auto fullQ = [&](int b) { return bar0 + 16 + 8 * b; };
    const uint32_t mmaS = bar0 + 40;
    auto mmaO = [&](int b) { return bar0 + 48 + 8 * b; };
    auto oFree = [&](int b) { return bar0 + 64 + 8 * b; };
    auto quFree = [&](int b) { return bar0 + 80 + 8 * b; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kCarSmall + 128);

    constexpr int kTiles = kD / BV;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t unit = blockIdx.x / kTiles;
    const int vt = static_cast<int>(blockIdx.x - unit * kTiles);
    const int64_t s = unit / kHV;
    const int h = static_cast<int>(unit - s * kHV);
    const int v0 = vt * BV;

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    const int len = static_cast<int>(t1 - t0);
    const int nch = (len + kC - 1) / kC;
    const int rec0 = reinterpret_cast<const int*>(ws + L.off_base)[s];
    const bool state_warp = warp < 4;
    const int k = tid;  // state column owned by state threads
    if (nch == 0 || rec0 + nch > L.R) {
        if (nch != 0 && tid == 0) record_status(16);
        if (state_warp) {  // empty sequence: zero state rows (oracle prefill :53-55)
            float* ns_col = p.new_state + (unit * kD + v0) * kD + k;
#pragma unroll 8
            for (int v = 0; v < BV; ++v) ns_col[v * kD] = 0.f;
        }
        return;
    }
    auto rhead = [&](int c) { return (int64_t)(rec0 + c) * kHV + h; };

    float S[BV];
    float Dn[BV];  // D of the next chunk to apply
    auto load_D = [&](int c) {
        const float4* src = reinterpret_cast<const float4*>(
            reinterpret_cast<const float*>(ws + L.off_d + rhead(c) * kDBytes) + k * kD + v0);
#pragma unroll
        for (int v = 0; v < BV; v += 4) {
            const float4 x = src[v / 4];
            Dn[v] = x.x, Dn[v + 1] = x.y, Dn[v + 2] = x.z, Dn[v + 3] = x.w;
        }
    };
    auto write_state_image = [&](int b) {
#pragma unroll
        for (int v = 0; v < BV; v += 8) st_shared_u4(aSI + b * 16384 + h16(k, v, kD), f16x8(S + v));
    };
    if (state_warp) {
        if (p.state != nullptr) {
            const float* st = p.state + (unit * kD + v0) * kD + k;
#pragma unroll
            for (int v = 0; v < BV; ++v) S[v] = st[v * kD];
        } else {
#pragma unroll
            for (int v = 0; v < BV; ++v) S[v] = 0.f;
        }
        write_state_image(0);
        load_D(0);
    }
    auto issue_M = [&](int c) {
        mbar_expect_tx(fullM(c & 1), kMImg);
        bulk_g2s(aMI + (c & 1) * kMImg, ws + L.off_m + rhead(c) * kMImg, kMImg, fullM(c & 1));
    };
    auto issue_QU = [&](int c) {
        const int b = c % 3;
        mbar_expect_tx(fullQ(b), kQtImg + kCarQUBytes - kQtImg);
        bulk_g2s(aQU + b * kCarQUBytes, ws + L.off_qt + rhead(c) * kQtImg, kQtImg, fullQ(b));
        bulk_g2s(aQU + b * kCarQUBytes + kQtImg, ws + L.off_ut + rhead(c) * kUtBytes + vt * (kC * 64 * 2),
                 kC * 64 * 2, fullQ(b));
    };
    int m_issued = -1, m_waited = -1, q_issued = -1, q_waited = -1;  // thread 0's copy bookkeeping
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) mbar_init(fullM(b), 1);
        for (int b = 0; b < 3; ++b) mbar_init(fullQ(b), 1);
        mbar_init(mmaS, 1);
        for (int b = 0; b < 2; ++b) mbar_init(mmaO(b), 1);
        for (int b = 0; b < 2; ++b) mbar_init(oFree(b), 4);
        for (int b = 0; b < 3; ++b) mbar_init(quFree(b), 4);
        fence_mbar_init();
        for (int c = 0; c < 2 && c < nch; ++c) issue_M(c), m_issued = c;
        for (int c = 0; c < 2 && c < nch; ++c) issue_QU(c), q_issued = c;  // chunk 2 is issued at c = 0
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kCarTmemCols);
        tmem_relinquish();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    const uint32_t t_accS = tm;
    auto t_accO = [&](int b) { return tm + 64 + 64 * b; };
    bool ok = true, aborted = false;

    if (state_warp) {
        for (int c = 0; c < nch; ++c) {
            if (tid == 0) {
                ok = ok && mbar_wait(fullM(c & 1), (c >> 1) & 1);  // ok is false after a failed refill wait
                if (ok) m_waited = c;
                ok = ok && mbar_wait(fullQ(c % 3), (c / 3) & 1);
                if (ok) q_waited = c;
                ok = ok && (c < 2 || mbar_wait(oFree(c & 1), ((c - 2) >> 1) & 1));
                if (ok) {
                    tc_fence_after();
                    mma_ct<kF16, false, true, kD, 128, kD, 128, BV>(t_accS, aMI + (c & 1) * kMImg,
                                                                   aSI + (c & 1) * 16384, false);
                    mma_commit(mmaS);
                    mma_ct<kF16, false, true, kD, 64, kD, 64, BV>(t_accO(c & 1), aQU + (c % 3) * kCarQUBytes,
                                                                 aSI + (c & 1) * 16384, false);
                    mma_commit(mmaO(c & 1));
                }
            }
            if (named_sync_or(1, 128, !ok)) {
                aborted = true;
                break;
            }
            ok = mbar_wait(mmaS, c & 1);
            tc_fence_after();
            {
                float a[32];
#pragma unroll
                for (int c0 = 0; c0 < BV; c0 += 32) {
                    tmem_ld32(taddr(t_accS, 32 * warp, c0), a);
                    tmem_wait_ld();
#pragma unroll
                    for (int v = 0; v < 32; ++v) S[c0 + v] = a[v] + Dn[c0 + v];
                }
            }
            if (c + 1 < nch) {
                write_state_image((c + 1) & 1);
                load_D(c + 1);
            }
            fence_async_smem();
            tc_fence_before();
            if (named_sync_or(1, 128, !ok)) {
                aborted = true;
                break;
            }
            if (tid == 0) {  // refill: M of chunk c+2 (MMA_S(c) done), [Qt | Ut] of chunk c+2
                tc_fence_after();
                if (c + 2 < nch) {
                    issue_M(c + 2);
                    m_issued = c + 2;
                    if (c >= 1 && !mbar_wait(quFree((c + 2) % 3), ((c - 1) / 3) & 1)) {
                        ok = false;  // caught by the next chunk's barrier
                    } else {
                        issue_QU(c + 2);
                        q_issued = c + 2;
                    }
                }
            }
        }
        if (tid == 0) {
            if (aborted) {
                record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
                for (int cc = m_waited + 1; cc <= m_issued; ++cc) mbar_wait(fullM(cc & 1), (cc >> 1) & 1);
                for (int cc = q_waited + 1; cc <= q_issued; ++cc) mbar_wait(fullQ(cc % 3), (cc / 3) & 1);
            }
        }
        float* ns_col = p.new_state + (unit * kD + v0) * kD + k;
#pragma unroll
        for (int v = 0; v < BV; ++v) ns_col[v * kD] = S[v];
    } else {
        // output warps: token i = 16 (warp - 4) + lane (lanes 0-15) of each chunk
        const int ow = warp - 4;
        const int i = 16 * ow + (lane & 15);
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
        for (int c = 0; c < nch; ++c) {
            bool okc = mbar_wait(mmaO(c & 1), (c >> 1) & 1) && mbar_wait(fullQ(c % 3), (c / 3) & 1);
            tc_fence_after();
            const int tok = kC * c + i;
            const uint32_t ut = aQU + (c % 3) * kCarQUBytes + kQtImg + (i & 63) * 128;
#pragma unroll
            for (int c0 = 0; c0 < BV; c0 += 32) {
                float o[32];
                tmem_ld32(taddr(t_accO(c & 1), 32 * ow, c0), o);
                tmem_wait_ld();
                if (okc && lane < 16 && tok < len) {
                    __nv_bfloat16* dst = out + ((t0 + tok) * kHV + h) * kD + v0 + c0;
#pragma unroll
                    for (int v = 0; v < 32; v += 8) {
                        float u[8];
                        h16x8_to_f32(ld_shared_u4(ut + (c0 + v) * 2), u);
                        __nv_bfloat162 w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            w[e] = __floats2bfloat162_rn(p.scale * (o[v + 2 * e] + u[2 * e]),
                                                         p.scale * (o[v + 2 * e + 1] + u[2 * e + 1]));
                        *reinterpret_cast<uint4*>(dst + v) = *reinterpret_cast<uint4*>(w);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(oFree(c & 1));
                mbar_arrive(quFree(c % 3));
            }
            if (!okc) {
                if (lane == 0) record_status(32);
                break;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kCarTmemCols);
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

cudaError_t launch_prefill_chunked(const PrefillParams& p, void* workspace, cudaStream_t stream) {
    const WsLayout L = ws_layout(p.total_tokens, p.num_seqs);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e;
    gdn_chunk_table_kernel<<<1, 1024, 0, stream>>>(p, ws, L);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_prepare_kernel, kPrepSmem)) != cudaSuccess) return e;
    if (L.R > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_chunk_prepare_kernel<<<dim3(static_cast<unsigned>(L.R), kHQK), 128, kPrepSmem, stream>>>(p, ws, L);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_carry_kernel, kCarSmem)) != cudaSuccess) return e;
    const int64_t grid = p.num_seqs * kHV * (kD / kCarryBV);
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_chunk_carry_kernel<<<static_cast<unsigned>(grid), kCarryThreads, kCarSmem, stream>>>(p, ws, L);
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
