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
// Kernel 1, gdn_chunk_prepare (one CTA per chunk x q/k head, both v-heads):
//   [K;Q] K^T on bf16 tcgen05 (M=128, N=64, K=128); per v-head the gates,
//   N and P; Ainv by six rounds of 64x64x64 tf32 tcgen05 products; W|U as one
//   M=64, N=256, K=64 tf32 MMA.  Results leave as SW128 operand images
//   (the carry's shared-memory layout) through bulk stores.
// Kernel 2, gdn_chunk_carry (one CTA per sequence x v-head x BV value rows):
//   walks the chunks in order with the fp32 state rows in registers; per chunk
//   four MMAs -- W S0^T (tf32), Q S0^T (bf16), (tail K)^T Delta (tf32),
//   P Delta (bf16) -- with the next chunk's operands bulk-copied into the other
//   half of a double buffer meanwhile.
// Precision: every operand that feeds the state (W, S, Delta, tail K, Ainv,
// the Neumann powers) is rounded fp32 -> tf32 with round-to-nearest; operands
// that only feed the bf16 output (Q S0^T, P Delta) run in bf16.
#include "gdn_common.cuh"
#include "tc05.cuh"

namespace gdn {
using namespace tc05;

constexpr int kC = 64;
constexpr int kWImg = kC * kD * 4;        // fp32 [64][128]        32 KiB
constexpr int kKTImg = kD * kC * 4;       // fp32 [128][64]        32 KiB
constexpr int kPImg = kC * kC * 4;        // tf32 [64][64]         16 KiB
constexpr int kUBytes = kC * kD * 4;      // fp32 [64][128] plain  32 KiB
constexpr int kVecBytes = 512;            // G[64], G_C
constexpr int kRecordBytes = kHV * (kWImg + kKTImg + kPImg + kUBytes + kVecBytes);

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace: header, per-sequence record bases, the chunk table and the
// per-record operand arrays (every array 1024-byte aligned).
struct WsLayout {
    int64_t R;  // record capacity: ceil(T / 64) + N bounds sum_s ceil(len_s / 64)
    int64_t off_hdr, off_base, off_table, off_w, off_kt, off_p, off_u, off_vec, total;
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
    L.off_w = o;
    o += L.R * kHV * kWImg;
    L.off_kt = o;
    o += L.R * kHV * kKTImg;
    L.off_p = o;
    o += L.R * kHV * kPImg;
    L.off_u = o;
    o += L.R * kHV * kUBytes;
    L.off_vec = o;
    o += L.R * kHV * kVecBytes;
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
// One CTA (128 threads) per chunk record and q/k head; the two v-heads of the
// q/k head share every M=64 accumulator, head 0 in TMEM lanes 0-15 and head 1
// in lanes 16-31 of each warp's sub-partition, so in the packed epilogues
// thread (warp w, lane l) owns row 16w + (l & 15) of head l >> 4.  Every
// operand image is written as whole 16-byte vectors of one row; B operands
// are MN-major images, so no transposed copy is ever made.
// Shared memory, 99 KB so that two CTAs share an SM: the X images reuse the
// [K;Q] tile once the Gram MMA and the Q-image store have read it, and the
// right-hand sides reuse the P images once the Neumann rounds are done.
constexpr int kPrepKQ = 0;          // bf16 [K;Q] K-major, 2 kblocks x 128 rows            32 KiB
constexpr int kPrepX = 0;           // tf32 X_h (Neumann iterate -> A^-1) K-major, 2 heads  2 x 16 KiB (over KQ)
constexpr int kPrepPA = 32768;      // tf32 P_h (power of N) K-major                         2 x 16 KiB
constexpr int kPrepPB = 65536;      // tf32 P_h MN-major (B operand)                          2 x 16 KiB
constexpr int kPrepRHS = kPrepPA;   // tf32 [beta G K | beta V] MN-major, 64 x 256, over PA+PB  64 KiB
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

// 2^x on the SFU (ex2.approx: a couple of ulp); x <= 0 here, so no overflow.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float4 tf32x4(float a, float b, float c, float d) {
    return make_float4(to_tf32(a), to_tf32(b), to_tf32(c), to_tf32(d));
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

__global__ void __launch_bounds__(128, 2)
    gdn_chunk_prepare_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sKQ = sm + kPrepKQ;
    PrepSmall& sml = *reinterpret_cast<PrepSmall*>(sm + kPrepSmall);
    const uint32_t aKQ = smem_u32(sKQ), aX = smem_u32(sm + kPrepX), aPA = smem_u32(sm + kPrepPA),
                   aPB = smem_u32(sm + kPrepPB), aRHS = smem_u32(sm + kPrepRHS);

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

    // 2. Gram: rows 0-63 K K^T, rows 64-127 Q K^T (bf16, M=128, N=64, K=128)
    if (tid == 0) {
        mma_ct<kBF16, false, false, kD, 128, 128, 128, 64>(tm, aKQ, aKQ, false);
        mma_commit(bar);
    }
    {  // inclusive prefix of log2 g (64 sequential adds; deterministic)
        const int hl = tid >> 6, i = tid & 63;
        float acc = 0.f;
        for (int m = 0; m <= i; ++m) acc += sml.lg[hl][m];
        sml.LG[hl][i] = acc;
    }
    __syncthreads();
    ok = mbar_wait(bar, phase);
    phase ^= 1;
    tc_fence_after();
    __syncthreads();  // every thread is past the Gram MMA before X overwrites [K;Q]
    {
        // 3. Gram epilogue (M=128 rows: thread = row).  Rows 0-63 build N, P and
        //    X = I - N of both heads; rows 64-127 build the output-side P.
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
        if (tid < 64) {
#pragma unroll 1
            for (int hl = 0; hl < 2; ++hl) {
                const float LGi = sml.LG[hl][i], bi = sml.beta[hl][i];
                const uint32_t xa = aX + hl * 16384, pa = aPA + hl * 16384, pb = aPB + hl * 16384;
#pragma unroll
                for (int j0 = 0; j0 < 64; j0 += 4) {
                    float nv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = j0 + e;
                        nv[e] = (j < i) ? bi * fast_exp2(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
                    }
                    const float4 t = tf32x4(nv[0], nv[1], nv[2], nv[3]);
                    st_shared_v4(pa + sw128_f32(i, j0, 64), t);
                    st_shared_v4(pb + mn32_f32(i, j0, 64), t);
                    st_shared_v4(xa + sw128_f32(i, j0, 64),
                                 tf32x4((j0 == i) - nv[0], (j0 + 1 == i) - nv[1], (j0 + 2 == i) - nv[2],
                                        (j0 + 3 == i) - nv[3]));
                }
            }
        } else {
#pragma unroll 1
            for (int hl = 0; hl < 2; ++hl) {
                const float LGi = sml.LG[hl][i];
                uint8_t* gp = ws + L.off_p + (rec * kHV + 2 * hq + hl) * kPImg;
#pragma unroll
                for (int j0 = 0; j0 < 64; j0 += 4) {
                    float pv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = j0 + e;
                        pv[e] = (j <= i) ? fast_exp2(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
                    }
                    *reinterpret_cast<float4*>(gp + sw128_f32(i, j0, 64)) = tf32x4(pv[0], pv[1], pv[2], pv[3]);
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
            mma_ct<kTF32, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 64), aPA + h * 16384, aPB + h * 16384,
                                                          false);
        mma_commit(bar);
    }
    // 4. Neumann doubling, both heads packed: epilogue e updates X (e >= 1) and P (e <= 4)
    const int hl = lane >> 4;
    const int row = 16 * warp + (lane & 15);
    for (int e = 0; e <= 5; ++e) {
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        if (e >= 1) {
            const uint32_t xa = aX + hl * 16384;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float xp[32];
                tmem_ld32(taddr(tm, 32 * warp, 32 * half), xp);
                tmem_wait_ld();
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 4) {
                    const uint32_t off = xa + sw128_f32(row, 32 * half + j0, 64);
                    const float4 x = ld_shared_v4(off);
                    st_shared_v4(off, tf32x4(x.x + xp[j0], x.y + xp[j0 + 1], x.z + xp[j0 + 2], x.w + xp[j0 + 3]));
                }
            }
        }
        if (e <= 4) {
            const uint32_t pa = aPA + hl * 16384, pb = aPB + hl * 16384;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float pp[32];
                tmem_ld32(taddr(tm, 32 * warp, 64 + 32 * half), pp);
                tmem_wait_ld();
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 4) {
                    const float4 t = tf32x4(pp[j0], pp[j0 + 1], pp[j0 + 2], pp[j0 + 3]);
                    st_shared_v4(pa + sw128_f32(row, 32 * half + j0, 64), t);
                    st_shared_v4(pb + mn32_f32(row, 32 * half + j0, 64), t);
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
                mma_ct<kTF32, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 0), aX + h * 16384,
                                                              aPB + h * 16384, false);  // X P
                if (e <= 3)
                    mma_ct<kTF32, false, true, 64, 64, 64, 64, 64>(taddr(tm, 16 * h, 64), aPA + h * 16384,
                                                                  aPB + h * 16384, false);  // P P
            }
            mma_commit(bar);
        }
    }
    // 5. per head: [beta G K | beta V] (MN-major, over the dead P images), the
    //    K-bar image and gate vector to global, then [W | U] = A^-1 [..]
#pragma unroll 1
    for (int h2 = 0; h2 < 2; ++h2) {
        const int h = 2 * hq + h2;
        const int64_t rh = rec * kHV + h;
        {
            const int j = tid & 63, part = tid >> 6;
            const float LGj = sml.LG[h2][j], bj = sml.beta[h2][j];
            const float Gj = exp2f(LGj), tail = exp2f(sml.LG[h2][63] - LGj);
            uint8_t* gkb = ws + L.off_kt + rh * kKTImg;
            // part 0: columns 0-127 (beta G K) and K-bar columns 0-63; part 1: beta V and K-bar 64-127
            const bool act = j < n;
            const uint16_t* ksrc = p.k + ((t0 + j) * kHQK + hq) * kD;  // K row j (L2-resident)
            if (part == 0) {
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8];
                    bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(ksrc + d0) : make_uint4(0, 0, 0, 0), f);
                    const float s = bj * Gj;
                    st_shared_v4(aRHS + mn32_f32(j, d0, 64), tf32x4(s * f[0], s * f[1], s * f[2], s * f[3]));
                    st_shared_v4(aRHS + mn32_f32(j, d0 + 4, 64), tf32x4(s * f[4], s * f[5], s * f[6], s * f[7]));
                    if (d0 < 64) {
                        *reinterpret_cast<float4*>(gkb + mn32_f32(j, d0, 64)) =
                            tf32x4(tail * f[0], tail * f[1], tail * f[2], tail * f[3]);
                        *reinterpret_cast<float4*>(gkb + mn32_f32(j, d0 + 4, 64)) =
                            tf32x4(tail * f[4], tail * f[5], tail * f[6], tail * f[7]);
                    }
                }
                float* gvec = reinterpret_cast<float*>(ws + L.off_vec + rh * kVecBytes);
                gvec[j] = Gj;
                if (j == 0) gvec[64] = exp2f(sml.LG[h2][63]);
            } else {
                const uint16_t* vsrc = p.v + ((t0 + j) * kHV + h) * kD;
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8];
                    bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(vsrc + d0) : make_uint4(0, 0, 0, 0), f);
                    st_shared_v4(aRHS + mn32_f32(j, 128 + d0, 64), tf32x4(bj * f[0], bj * f[1], bj * f[2], bj * f[3]));
                    st_shared_v4(aRHS + mn32_f32(j, 132 + d0, 64), tf32x4(bj * f[4], bj * f[5], bj * f[6], bj * f[7]));
                    if (d0 >= 64) {
                        float g[8];
                        bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(ksrc + d0) : make_uint4(0, 0, 0, 0), g);
                        *reinterpret_cast<float4*>(gkb + mn32_f32(j, d0, 64)) =
                            tf32x4(tail * g[0], tail * g[1], tail * g[2], tail * g[3]);
                        *reinterpret_cast<float4*>(gkb + mn32_f32(j, d0 + 4, 64)) =
                            tf32x4(tail * g[4], tail * g[5], tail * g[6], tail * g[7]);
                    }
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            mma_ct<kTF32, false, true, 64, 64, 64, 64, 256>(taddr(tm, 16 * h2, 0), aX + h2 * 16384, aRHS, false);
            mma_commit(bar);
        }
        ok = mbar_wait(bar, phase);  // also frees the RHS image for the next head
        phase ^= 1;
        tc_fence_after();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            goto done;
        }
    }
    {   // 6. [W | U] rows of both heads (packed): W as the carry's tf32 A image, U plain
        const int h = 2 * hq + hl;
        const int64_t rh = rec * kHV + h;
        uint8_t* gw = ws + L.off_w + rh * kWImg;
        float* gu = reinterpret_cast<float*>(ws + L.off_u + rh * kUBytes) + row * kD;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
            float acc[32];
            tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
            tmem_wait_ld();
            if (c < 4) {
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 4)
                    *reinterpret_cast<float4*>(gw + sw128_f32(row, 32 * c + j0, 64)) =
                        tf32x4(acc[j0], acc[j0 + 1], acc[j0 + 2], acc[j0 + 3]);
            } else {
#pragma unroll
                for (int j0 = 0; j0 < 32; j0 += 4)
                    *reinterpret_cast<float4*>(gu + 32 * (c - 4) + j0) =
                        make_float4(acc[j0], acc[j0 + 1], acc[j0 + 2], acc[j0 + 3]);
            }
        }
    }
done:
    if (tid == 0) {
        bulk_wait_all();
        if (aborted) record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(sml.tmem_base, kPrepTmemCols);
    }
}

// ------------------------------------------------------------------ carry --
// One CTA (128 threads) per sequence x v-head x BV value rows.  Per chunk:
//   MMA1  [W ; G(.)Q] S0^T  (tf32, M=128): TMEM lanes 0-63 hold W S0^T,
//         lanes 64-127 G(.)Q S0^T (one row per token in both halves)
//   epi A warps 0-1: Delta = U - W S0^T -> Delta image (tf32, MN-major)
//   MMA2  (tail K)^T Delta (M=128, rows = state columns k) and [0 ; P] Delta
//         accumulated onto lanes 64-127, which then hold the chunk's output
//   epi B every thread: S1 = G_C S0 + (tail K)^T Delta for its column k;
//         warps 2-3 store O = scale (G(.)Q S0^T + P Delta)
// Operands arrive by bulk copy; each is reloaded for the next chunk as soon
// as the MMA reading it completes (W after MMA1; tail K, P, G after MMA2), and
// warps 2-3 build the next chunk's G(.)Q rows from the raw q input while MMA2
// runs, so one buffer per operand suffices.  All operands feeding the state
// are tf32 (round-to-nearest); the state itself stays fp32 in registers.
template <int BV>
struct CarrySmem {
    static constexpr int kA1 = 0;                 // tf32 [W ; G Q] K-major, 4 kblocks x 128 rows   64 KiB
    static constexpr int kA2 = kA1 + 65536;       // tf32 [0 ; P]   K-major, 2 kblocks x 128 rows   32 KiB
    static constexpr int kKB = kA2 + 32768;       // tf32 tail K MN-major [64 j][128 k]             32 KiB
    static constexpr int kVec = kKB + 32768;      // two gate vectors G[64], G_C (by chunk parity)
    static constexpr int kS32 = kVec + 1024;      // tf32 S MN-major [128 k][BV]
    static constexpr int kD32 = kS32 + BV * 512;  // tf32 Delta MN-major [64 j][BV]
    static constexpr int kSmall = kD32 + BV * 256;
    static constexpr int kTotal = kSmall + 128 + 1024;
    static constexpr int kTmemCols = 2 * BV < 32 ? 32 : 2 * BV;
};
constexpr uint32_t kCarryTxA = kWImg;
constexpr uint32_t kCarryTxB = kKTImg + kPImg + kVecBytes;

template <int BV>
__global__ void __launch_bounds__(128, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, const uint8_t* __restrict__ ws, const WsLayout L) {
    using SM = CarrySmem<BV>;
    static_assert(BV == 32 || BV == 64, "value-row tile (MN-major tf32 images need 32-wide rows)");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const uint32_t aA1 = smem_u32(sm + SM::kA1), aA2 = smem_u32(sm + SM::kA2), aKB = smem_u32(sm + SM::kKB),
                   aVec = smem_u32(sm + SM::kVec), aS32 = smem_u32(sm + SM::kS32), aD32 = smem_u32(sm + SM::kD32);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM::kSmall);  // fullA, fullB, mma1, mma2
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + SM::kSmall + 64);

    constexpr int kTiles = kD / BV;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int64_t unit = blockIdx.x / kTiles;
    const int vt = static_cast<int>(blockIdx.x - unit * kTiles);
    const int64_t s = unit / kHV;
    const int h = static_cast<int>(unit - s * kHV);
    const int hq = h / kGva;
    const int v0 = vt * BV;

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    const int len = static_cast<int>(t1 - t0);
    const int nch = (len + kC - 1) / kC;
    const int rec0 = reinterpret_cast<const int*>(ws + L.off_base)[s];
    float* ns_col = p.new_state + (unit * kD + v0) * kD + tid;  // column k = tid of rows v0..
    if (nch == 0 || rec0 + nch > L.R) {
        if (nch != 0) record_status(16);
#pragma unroll
        for (int v = 0; v < BV; ++v) ns_col[v * kD] = 0.f;  // empty sequence: zero state row
        return;
    }

    // state rows v0..v0+BV, column k = tid, in registers; MN-major image for the MMAs
    float S[BV];
    if (p.state != nullptr) {
        const float* st = p.state + (unit * kD + v0) * kD + tid;
#pragma unroll
        for (int v = 0; v < BV; ++v) S[v] = st[v * kD];
    } else {
#pragma unroll
        for (int v = 0; v < BV; ++v) S[v] = 0.f;
    }
    auto write_state_image = [&]() {
#pragma unroll
        for (int v = 0; v < BV; v += 4)
            st_shared_v4(aS32 + mn32_f32(tid, v, kD), tf32x4(S[v], S[v + 1], S[v + 2], S[v + 3]));
    };
    write_state_image();
    {  // the zero upper half of [0 ; P] (rows 0-63 of both K-blocks), written once
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int idx = tid * 8 + e;  // 1024 chunks of 16 B
            st_shared_v4(aA2 + (idx >> 9) * 16384 + (idx & 511) * 16, z);
        }
    }
    auto gvec = [&](int c) {
        return reinterpret_cast<const float*>(ws + L.off_vec + ((int64_t)(rec0 + c) * kHV + h) * kVecBytes);
    };
    // G (.) Q rows of chunk c into rows 64-127 of [W ; G Q] (warps 2-3: token i = tid - 64)
    auto build_gq = [&](int c) {
        const int i = tid - 64;
        const int tok = kC * c + i;
        const bool act = tok < len;
        const float gi = act ? gvec(c)[i] : 0.f;
        const uint16_t* qrow = p.q + ((t0 + tok) * kHQK + hq) * kD;
#pragma unroll 4
        for (int k0 = 0; k0 < kD; k0 += 8) {
            float f[8];
            bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(qrow + k0) : make_uint4(0, 0, 0, 0), f);
            st_shared_v4(aA1 + sw128_f32(64 + i, k0, 128), tf32x4(gi * f[0], gi * f[1], gi * f[2], gi * f[3]));
            st_shared_v4(aA1 + sw128_f32(64 + i, k0 + 4, 128), tf32x4(gi * f[4], gi * f[5], gi * f[6], gi * f[7]));
        }
    };
    if (warp >= 2) build_gq(0);

    const uint32_t fullA = smem_u32(&bars[0]), fullB = smem_u32(&bars[1]), mma1 = smem_u32(&bars[2]),
                   mma2 = smem_u32(&bars[3]);
    auto issue_A = [&](int c) {  // W of chunk c -> rows 0-63 of each K-block of [W ; G Q]
        const uint8_t* gw = ws + L.off_w + ((int64_t)(rec0 + c) * kHV + h) * kWImg;
        mbar_expect_tx(fullA, kCarryTxA);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) bulk_g2s(aA1 + kb * 16384, gw + kb * 8192, 8192, fullA);
    };
    auto issue_B = [&](int c) {  // tail K, P (rows 64-127 of [0 ; P]) and G of chunk c
        const int64_t rh = (int64_t)(rec0 + c) * kHV + h;
        const uint8_t* gp = ws + L.off_p + rh * kPImg;
        mbar_expect_tx(fullB, kCarryTxB);
        bulk_g2s(aKB, ws + L.off_kt + rh * kKTImg, kKTImg, fullB);
        bulk_g2s(aA2 + 8192, gp, 8192, fullB);
        bulk_g2s(aA2 + 16384 + 8192, gp + 8192, 8192, fullB);
        bulk_g2s(aVec + (c & 1) * 512, ws + L.off_vec + rh * kVecBytes, kVecBytes, fullB);
    };
    if (tid == 0) {
        mbar_init(fullA, 1);
        mbar_init(fullB, 1);
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        fence_mbar_init();
        issue_A(0);
        issue_B(0);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), SM::kTmemCols);
        tmem_relinquish();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    const uint32_t t_acc = tm, t_up = tm + BV;

    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    bool ok = true, aborted = false;
    int a_issued = 0, a_landed = -1, b_issued = 0, b_landed = -1;
    for (int c = 0; c < nch; ++c) {
        const int64_t rh = (int64_t)(rec0 + c) * kHV + h;
        // MMA1 as soon as W of this chunk has landed
        if (tid == 0) {
            ok = mbar_wait(fullA, c & 1);
            if (ok) {
                a_landed = c;
                tc_fence_after();
                mma_ct<kTF32, false, true, kD, 128, kD, 128, BV>(t_acc, aA1, aS32, false);
                mma_commit(mma1);
            }
        }
        float u[BV];
        if (warp < 2) {  // U row of token j = tid, while MMA1 runs
            const float4* up =
                reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ws + L.off_u + rh * kUBytes) +
                                                tid * kD + v0);
#pragma unroll
            for (int v = 0; v < BV; v += 4) {
                const float4 x = up[v / 4];
                u[v] = x.x, u[v + 1] = x.y, u[v + 2] = x.z, u[v + 3] = x.w;
            }
        }
        ok = __syncthreads_and(ok) && mbar_wait(mma1, c & 1);
        tc_fence_after();
        if (tid == 0 && c + 1 < nch) issue_A(c + 1);  // W's rows of [W ; G Q] are free again
        if (c + 1 < nch) a_issued = c + 1;
        if (warp < 2) {  // epi A: Delta row j = tid
            float wsr[BV];
#pragma unroll
            for (int c0 = 0; c0 < BV; c0 += 32) {
                float a[32];
                tmem_ld32(taddr(t_acc, 32 * warp, c0), a);
                tmem_wait_ld();
#pragma unroll
                for (int v = 0; v < 32; ++v) wsr[c0 + v] = a[v];
            }
#pragma unroll
            for (int v = 0; v < BV; v += 4)
                st_shared_v4(aD32 + mn32_f32(tid, v, kC),
                             tf32x4(u[v] - wsr[v], u[v + 1] - wsr[v + 1], u[v + 2] - wsr[v + 2], u[v + 3] - wsr[v + 3]));
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        if (tid == 0) {
            ok = mbar_wait(fullB, c & 1);
            if (ok) {
                b_landed = c;
                tc_fence_after();
                mma_ct<kTF32, true, true, kC, kC, kC, 128, BV>(t_up, aKB, aD32, false);     // (tail K)^T Delta
                mma_ct<kTF32, false, true, kC, 128, kC, 128, BV>(t_acc, aA2, aD32, true);   // += [0 ; P] Delta
                mma_commit(mma2);
            }
        }
        if (warp >= 2 && c + 1 < nch) build_gq(c + 1);  // rows 64-127 of [W ; G Q] are free since MMA1
        ok = __syncthreads_and(ok) && mbar_wait(fullB, c & 1) && mbar_wait(mma2, c & 1);
        tc_fence_after();
        const float gc = *reinterpret_cast<const float*>(sm + SM::kVec + (c & 1) * 512 + 64 * 4);
        if (tid == 0 && c + 1 < nch) issue_B(c + 1);  // tail K and P are free again; G goes to the other half
        if (c + 1 < nch) b_issued = c + 1;
        {  // epi B: state column k = tid; warps 2-3 also store the outputs of token tid - 64
#pragma unroll
            for (int c0 = 0; c0 < BV; c0 += 32) {
                float a[32];
                tmem_ld32(taddr(t_up, 32 * warp, c0), a);
                tmem_wait_ld();
#pragma unroll
                for (int v = 0; v < 32; ++v) S[c0 + v] = fmaf(gc, S[c0 + v], a[v]);
            }
            write_state_image();
            if (warp >= 2) {
                const int i = tid - 64;
                const int tok = kC * c + i;
#pragma unroll
                for (int c0 = 0; c0 < BV; c0 += 32) {
                    float o[32];
                    tmem_ld32(taddr(t_acc, 32 * warp, c0), o);
                    tmem_wait_ld();
                    if (tok < len) {
                        __nv_bfloat16* dst = out + ((t0 + tok) * kHV + h) * kD + v0 + c0;
#pragma unroll
                        for (int v = 0; v < 32; v += 8) {
                            __nv_bfloat162 w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                w[e] = __floats2bfloat162_rn(p.scale * o[v + 2 * e], p.scale * o[v + 2 * e + 1]);
                            *reinterpret_cast<uint4*>(dst + v) = *reinterpret_cast<uint4*>(w);
                        }
                    }
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
    }
    if (aborted && tid == 0) {
        record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
        // drain the operand loads still in flight before the CTA exits
        for (int cc = a_landed + 1; cc <= a_issued; ++cc) mbar_wait(fullA, cc & 1);
        for (int cc = b_landed + 1; cc <= b_issued; ++cc) mbar_wait(fullB, cc & 1);
    }
#pragma unroll
    for (int v = 0; v < BV; ++v) ns_col[v * kD] = S[v];
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, SM::kTmemCols);
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
    // value-row tile: 64 rows (two CTAs per head) once that still fills the SMs, else 32
    if (p.num_seqs * kHV * (kD / 64) >= kSmCount) {
        using SM = CarrySmem<64>;
        if ((e = set_smem(gdn_chunk_carry_kernel<64>, SM::kTotal)) != cudaSuccess) return e;
        const int64_t grid = p.num_seqs * kHV * (kD / 64);
        if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
        gdn_chunk_carry_kernel<64><<<static_cast<unsigned>(grid), 128, SM::kTotal, stream>>>(p, ws, L);
    } else {
        using SM = CarrySmem<32>;
        if ((e = set_smem(gdn_chunk_carry_kernel<32>, SM::kTotal)) != cudaSuccess) return e;
        const int64_t grid = p.num_seqs * kHV * (kD / 32);
        if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
        gdn_chunk_carry_kernel<32><<<static_cast<unsigned>(grid), 128, SM::kTotal, stream>>>(p, ws, L);
    }
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
