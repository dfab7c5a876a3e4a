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
constexpr int kQImg = kC * kD * 2;        // bf16 [64][128]        16 KiB
constexpr int kWImg = kC * kD * 4;        // fp32 [64][128]        32 KiB
constexpr int kKTImg = kD * kC * 4;       // fp32 [128][64]        32 KiB
constexpr int kPImg = kC * kC * 2;        // bf16 [64][64]          8 KiB
constexpr int kUBytes = kC * kD * 4;      // fp32 [64][128] plain  32 KiB
constexpr int kVecBytes = 512;            // G[64], G_C
constexpr int kRecordBytes = kHQK * kQImg + kHV * (kWImg + kKTImg + kPImg + kUBytes + kVecBytes);

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace: header, per-sequence record bases, the chunk table and the
// per-record operand arrays (every array 1024-byte aligned).
struct WsLayout {
    int64_t R;  // record capacity: ceil(T / 64) + N bounds sum_s ceil(len_s / 64)
    int64_t off_hdr, off_base, off_table, off_q, off_w, off_kt, off_p, off_u, off_vec, total;
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
    L.off_q = o;
    o += L.R * kHQK * kQImg;
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
constexpr int kPrepKQ = 0;          // bf16 [K;Q] K-major, 2 kblocks x 128 rows            32 KiB
constexpr int kPrepX = 32768;       // tf32 X_h (Neumann iterate -> A^-1) K-major, 2 heads  2 x 16 KiB
constexpr int kPrepPA = 65536;      // tf32 P_h (power of N) K-major                         2 x 16 KiB
constexpr int kPrepPB = 98304;      // tf32 P_h MN-major (B operand)                          2 x 16 KiB
constexpr int kPrepRHS = kPrepPA;   // tf32 [beta G K | beta V] MN-major, 64 x 256, over PA+PB  64 KiB
constexpr int kPrepSmall = 131072;
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

// 8 bf16 (one 16-byte chunk) -> 8 floats
__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}

__global__ void __launch_bounds__(128, 1)
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
        // the chunk's Q image leaves for the carry kernel (rows 64-127 of each K-block)
        uint8_t* gq = ws + L.off_q + (rec * kHQK + hq) * kQImg;
        bulk_s2g(gq, aKQ + 64 * 128, 64 * 128);
        bulk_s2g(gq + 64 * 128, aKQ + 128 * 128 + 64 * 128, 64 * 128);
        bulk_commit();
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
                        nv[e] = (j < i) ? bi * exp2f(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
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
                for (int c = 0; c < 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = 8 * c + 2 * e;
                        const float a0 = (j <= i) ? exp2f(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
                        const float a1 = (j + 1 <= i) ? exp2f(LGi - sml.LG[hl][j + 1]) * gram[j + 1] : 0.f;
                        const __nv_bfloat162 v2 = __floats2bfloat162_rn(a0, a1);
                        w[e] = *reinterpret_cast<const uint32_t*>(&v2);
                    }
                    *reinterpret_cast<uint4*>(gp + i * 128 + ((c ^ (i & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
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
            if (part == 0) {
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8];
                    bf16x8_to_f32(*reinterpret_cast<const uint4*>(sKQ + sw128_bf16(j, d0, 128)), f);
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
                const bool act = j < n;
                const uint16_t* vsrc = p.v + ((t0 + j) * kHV + h) * kD;
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 8) {
                    float f[8];
                    bf16x8_to_f32(act ? *reinterpret_cast<const uint4*>(vsrc + d0) : make_uint4(0, 0, 0, 0), f);
                    st_shared_v4(aRHS + mn32_f32(j, 128 + d0, 64), tf32x4(bj * f[0], bj * f[1], bj * f[2], bj * f[3]));
                    st_shared_v4(aRHS + mn32_f32(j, 132 + d0, 64), tf32x4(bj * f[4], bj * f[5], bj * f[6], bj * f[7]));
                    if (d0 >= 64) {
                        float g[8];
                        bf16x8_to_f32(*reinterpret_cast<const uint4*>(sKQ + sw128_bf16(j, d0, 128)), g);
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
//   MMA1  W S0^T (tf32, B = S MN-major)  and  Q S0^T (bf16)      -> rows = tokens
//   epi A Delta = U - W S0^T  -> Delta images (tf32 MN-major, bf16 K-major)
//   MMA2  (tail K)^T Delta (tf32, both operands MN-major)  and  P Delta (bf16)
//   epi B S1 = G_C S0 + (tail K)^T Delta (thread k owns state column k),
//         O = scale (G (.) Q S0^T + P Delta) for the chunk's tokens
// The next chunk's operand images are bulk-copied into the other slot meanwhile.
constexpr int kSlotQ = 0;
constexpr int kSlotW = kSlotQ + kQImg;
constexpr int kSlotKT = kSlotW + kWImg;
constexpr int kSlotP = kSlotKT + kKTImg;
constexpr int kSlotVec = kSlotP + kPImg;
constexpr int kSlotBytes = kSlotVec + 1024;
constexpr uint32_t kSlotTx = kQImg + kWImg + kKTImg + kPImg + kVecBytes;

template <int BV>
struct CarrySmem {
    static constexpr int kSlots = 0;                      // 2 operand slots
    static constexpr int kS32 = kSlots + 2 * kSlotBytes;  // tf32 S MN-major [128 k][BV]
    static constexpr int kS16 = kS32 + BV * 512;          // bf16 S K-major [BV v][128 k]
    static constexpr int kD32 = kS16 + BV * 256;          // tf32 Delta MN-major [64 j][BV]
    static constexpr int kD16 = kD32 + BV * 256;          // bf16 Delta K-major [BV v][64 j]
    static constexpr int kSmall = kD16 + BV * 128;
    static constexpr int kTotal = kSmall + 128 + 1024;
    static constexpr int kTmemCols = 4 * BV < 32 ? 32 : 4 * BV;
};

template <int BV>
__global__ void __launch_bounds__(128, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, const uint8_t* __restrict__ ws, const WsLayout L) {
    using SM = CarrySmem<BV>;
    static_assert(BV == 32 || BV == 64, "value-row tile (MN-major tf32 images need 32-wide rows)");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const uint32_t aS32 = smem_u32(sm + SM::kS32), aS16 = smem_u32(sm + SM::kS16), aD32 = smem_u32(sm + SM::kD32),
                   aD16 = smem_u32(sm + SM::kD16);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM::kSmall);  // full[2], mma1, mma2
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + SM::kSmall + 64);

    constexpr int kTiles = kD / BV;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t unit = blockIdx.x / kTiles;
    const int vt = static_cast<int>(blockIdx.x - unit * kTiles);
    const int64_t s = unit / kHV;
    const int h = static_cast<int>(unit - s * kHV);
    const int v0 = vt * BV;

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    const int nch = static_cast<int>((t1 - t0 + kC - 1) / kC);
    const int rec0 = reinterpret_cast<const int*>(ws + L.off_base)[s];
    float* ns_col = p.new_state + (unit * kD + v0) * kD + tid;  // column k = tid of rows v0..
    if (nch == 0 || rec0 + nch > L.R) {
        if (nch != 0) record_status(16);
#pragma unroll
        for (int v = 0; v < BV; ++v) ns_col[v * kD] = 0.f;  // empty sequence: zero state row
        return;
    }

    // state rows v0..v0+BV, column k = tid, in registers; images for the MMAs
    float S[BV];
    if (p.state != nullptr) {
        const float* st = p.state + (unit * kD + v0) * kD + tid;
#pragma unroll
        for (int v = 0; v < BV; ++v) S[v] = st[v * kD];
    } else {
#pragma unroll
        for (int v = 0; v < BV; ++v) S[v] = 0.f;
    }
    auto write_state_images = [&]() {
#pragma unroll
        for (int v = 0; v < BV; v += 4) {
            st_shared_v4(aS32 + mn32_f32(tid, v, kD), tf32x4(S[v], S[v + 1], S[v + 2], S[v + 3]));
        }
#pragma unroll
        for (int v = 0; v < BV; ++v)
            *reinterpret_cast<__nv_bfloat16*>(sm + SM::kS16 + sw128_bf16(v, tid, BV)) = __float2bfloat16_rn(S[v]);
    };
    write_state_images();

    const uint32_t full0 = smem_u32(&bars[0]), mma1 = smem_u32(&bars[2]), mma2 = smem_u32(&bars[3]);
    if (tid == 0) {
        mbar_init(full0, 1);
        mbar_init(full0 + 8, 1);
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), SM::kTmemCols);
        tmem_relinquish();
    }
    auto issue_loads = [&](int c) {
        const int64_t r = rec0 + c;
        const int64_t rh = r * kHV + h;
        const uint32_t slot = smem_u32(sm + SM::kSlots + (c & 1) * kSlotBytes);
        const uint32_t fb = full0 + 8 * (c & 1);
        mbar_expect_tx(fb, kSlotTx);
        bulk_g2s(slot + kSlotQ, ws + L.off_q + (r * kHQK + h / kGva) * kQImg, kQImg, fb);
        bulk_g2s(slot + kSlotW, ws + L.off_w + rh * kWImg, kWImg, fb);
        bulk_g2s(slot + kSlotKT, ws + L.off_kt + rh * kKTImg, kKTImg, fb);
        bulk_g2s(slot + kSlotP, ws + L.off_p + rh * kPImg, kPImg, fb);
        bulk_g2s(slot + kSlotVec, ws + L.off_vec + rh * kVecBytes, kVecBytes, fb);
    };
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    const uint32_t t_ws = tm, t_qs = tm + BV, t_up = tm + 2 * BV, t_pd = tm + 3 * BV;
    if (tid == 0) issue_loads(0);

    const int row = 16 * warp + lane;  // token row of M=64 tiles (lanes < 16)
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    bool ok = true, aborted = false;
    int last_issued = 0, last_landed = -1;  // chunk indices of the operand loads
    for (int c = 0; c < nch; ++c) {
        const int slot = c & 1;
        const uint8_t* sl = sm + SM::kSlots + slot * kSlotBytes;
        const uint32_t asl = smem_u32(sl);
        const int64_t r = rec0 + c;
        const int64_t rh = r * kHV + h;
        if (c + 1 < nch) {
            if (tid == 0) issue_loads(c + 1);
            last_issued = c + 1;
        }
        ok = mbar_wait(full0 + 8 * slot, (c >> 1) & 1);
        if (ok) last_landed = c;
        if (tid == 0 && ok) {
            tc_fence_after();
            mma_ct<kTF32, false, true, kD, 64, kD, 64, BV>(t_ws, asl + kSlotW, aS32, false);
            mma_ct<kBF16, false, false, kD, 64, BV, 64, BV>(t_qs, asl + kSlotQ, aS16, false);
            mma_commit(mma1);
        }
        const int tok = 64 * c + row;
        const bool act = lane < 16 && tok < t1 - t0;
        float u[BV];
        {
            const float4* up = reinterpret_cast<const float4*>(
                reinterpret_cast<const float*>(ws + L.off_u + rh * kUBytes) + (row & 63) * kD + v0);
#pragma unroll
            for (int v = 0; v < BV; v += 4) {
                const float4 x = up[v / 4];
                u[v] = x.x;
                u[v + 1] = x.y;
                u[v + 2] = x.z;
                u[v + 3] = x.w;
            }
        }
        const float* vec = reinterpret_cast<const float*>(sl + kSlotVec);
        const float gc = vec[64];
        const float gi = vec[row & 63];
        ok = ok && mbar_wait(mma1, c & 1);
        tc_fence_after();
        {  // Delta = U - W S0^T -> Delta images (B operands of the next two MMAs)
            float wsr[BV];
            if constexpr (BV == 32) {
                tmem_ld32(taddr(t_ws, 32 * warp, 0), wsr);
            } else {
                float a[32], b[32];
                tmem_ld32(taddr(t_ws, 32 * warp, 0), a);
                tmem_ld32(taddr(t_ws, 32 * warp, 32), b);
#pragma unroll
                for (int v = 0; v < 32; ++v) wsr[v] = a[v], wsr[32 + v] = b[v];
            }
            tmem_wait_ld();
            if (lane < 16) {
#pragma unroll
                for (int v = 0; v < BV; v += 4) {
                    const float d0 = u[v] - wsr[v], d1 = u[v + 1] - wsr[v + 1], d2 = u[v + 2] - wsr[v + 2],
                                d3 = u[v + 3] - wsr[v + 3];
                    st_shared_v4(aD32 + mn32_f32(row, v, 64), tf32x4(d0, d1, d2, d3));
                    *reinterpret_cast<__nv_bfloat16*>(sm + SM::kD16 + sw128_bf16(v, row, BV)) = __float2bfloat16_rn(d0);
                    *reinterpret_cast<__nv_bfloat16*>(sm + SM::kD16 + sw128_bf16(v + 1, row, BV)) =
                        __float2bfloat16_rn(d1);
                    *reinterpret_cast<__nv_bfloat16*>(sm + SM::kD16 + sw128_bf16(v + 2, row, BV)) =
                        __float2bfloat16_rn(d2);
                    *reinterpret_cast<__nv_bfloat16*>(sm + SM::kD16 + sw128_bf16(v + 3, row, BV)) =
                        __float2bfloat16_rn(d3);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        if (tid == 0) {
            tc_fence_after();
            mma_ct<kTF32, true, true, 64, 64, 64, 128, BV>(t_up, asl + kSlotKT, aD32, false);
            mma_ct<kBF16, false, false, 64, 64, BV, 64, BV>(t_pd, asl + kSlotP, aD16, false);
            mma_commit(mma2);
        }
        ok = mbar_wait(mma2, c & 1);
        tc_fence_after();
        {  // S1 = G_C S0 + (tail K)^T Delta ; O = scale (G (.) Q S0^T + P Delta)
            float up[BV], qs[BV], pd[BV];
            if constexpr (BV == 32) {
                tmem_ld32(taddr(t_up, 32 * warp, 0), up);
                tmem_ld32(taddr(t_qs, 32 * warp, 0), qs);
                tmem_ld32(taddr(t_pd, 32 * warp, 0), pd);
            } else {
                float a[32];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    tmem_ld32(taddr(t_up, 32 * warp, 32 * hh), a);
#pragma unroll
                    for (int v = 0; v < 32; ++v) up[32 * hh + v] = a[v];
                    tmem_ld32(taddr(t_qs, 32 * warp, 32 * hh), a);
#pragma unroll
                    for (int v = 0; v < 32; ++v) qs[32 * hh + v] = a[v];
                    tmem_ld32(taddr(t_pd, 32 * warp, 32 * hh), a);
#pragma unroll
                    for (int v = 0; v < 32; ++v) pd[32 * hh + v] = a[v];
                }
            }
            tmem_wait_ld();
#pragma unroll
            for (int v = 0; v < BV; ++v) S[v] = fmaf(gc, S[v], up[v]);
            write_state_images();
            if (act) {
                __nv_bfloat16* o = out + ((t0 + tok) * kHV + h) * kD + v0;
#pragma unroll
                for (int v = 0; v < BV; v += 8) {
                    __nv_bfloat162 w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        w[e] = __floats2bfloat162_rn(p.scale * fmaf(gi, qs[v + 2 * e], pd[v + 2 * e]),
                                                     p.scale * fmaf(gi, qs[v + 2 * e + 1], pd[v + 2 * e + 1]));
                    *reinterpret_cast<uint4*>(o + v) = *reinterpret_cast<uint4*>(w);
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
        // drain the operand loads still in flight (at most two) before the CTA exits
        for (int cc = last_landed + 1; cc <= last_issued; ++cc) mbar_wait(full0 + 8 * (cc & 1), (cc >> 1) & 1);
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
    using SM = CarrySmem<32>;
    if ((e = set_smem(gdn_chunk_carry_kernel<32>, SM::kTotal)) != cudaSuccess) return e;
    const int64_t grid = p.num_seqs * kHV * (kD / 32);
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_chunk_carry_kernel<32><<<static_cast<unsigned>(grid), 128, SM::kTotal, stream>>>(p, ws, L);
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
    const int eb = kind == kBF16 ? 2 : 4;
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
        if (kind == kBF16)
            *reinterpret_cast<uint16_t*>(sA + sw128_bf16(row, col, rows)) = static_cast<const uint16_t*>(A)[idx];
        else
            st_f32(sA, a_mn ? mn32_f32(row, col, rows) : sw128_f32(row, col, rows),
                   to_tf32(static_cast<const float*>(A)[idx]));
    }
    for (int idx = tid; idx < N * K; idx += 128) {
        const int r = idx / K, c = idx % K;  // B[r][c]: n = r, k = c
        const int row = b_mn ? c : r, col = b_mn ? r : c, rows = b_mn ? K : N;
        if (kind == kBF16)
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
