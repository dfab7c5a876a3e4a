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
// Shared memory of the prepare kernel (offsets from a 1024-aligned base).
constexpr int kPrepKQ = 0;                         // bf16 [K;Q] image, 2 kblocks x 128 rows     32 KiB
constexpr int kPrepX = kPrepKQ + 2 * 128 * 128;    // fp32 X (Neumann iterate, then Ainv) [64][64] 16 KiB
constexpr int kPrepP = kPrepX + 2 * 64 * 128;      // fp32 power P [64][64]                     16 KiB
constexpr int kPrepPT = kPrepP + 2 * 64 * 128;     // fp32 P^T                                  16 KiB
constexpr int kPrepRHS = kPrepPT + 2 * 64 * 128;   // fp32 [(beta G K)^T ; (beta V)^T] [256][64] 64 KiB
constexpr int kPrepPout = kPrepRHS + 2 * 256 * 128;  // bf16 P (output-side) [64][64]             8 KiB
constexpr int kPrepSmall = kPrepPout + 64 * 128;
constexpr int kPrepSmem = kPrepSmall + 2048 + 1024;  // + gates/bars, + alignment slack
constexpr int kPrepTmemCols = 256;

struct PrepSmall {
    float lg[2][kC];   // log2 g per token (0 for inactive rows)
    float LG[2][kC];   // inclusive prefix of lg
    float beta[2][kC];
    uint64_t bar_mma;
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void st_f32(uint8_t* img, uint32_t off, float v) {
    *reinterpret_cast<float*>(img + off) = v;
}

__global__ void __launch_bounds__(128, 1)
    gdn_chunk_prepare_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sKQ = sm + kPrepKQ;
    uint8_t* sX = sm + kPrepX;
    uint8_t* sP = sm + kPrepP;
    uint8_t* sPT = sm + kPrepPT;
    uint8_t* sRHS = sm + kPrepRHS;
    uint8_t* sPout = sm + kPrepPout;
    PrepSmall& sml = *reinterpret_cast<PrepSmall*>(sm + kPrepSmall);

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
        sml.abort_flag = 0;
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&sml.tmem_base), kPrepTmemCols);
        tmem_relinquish();
    }

    // 1. K and Q tiles -> [K;Q] bf16 image (rows >= n zero); gates of both v-heads
    for (int idx = tid; idx < 2 * kC * 16; idx += 128) {
        const int m = idx >> 10;  // 0: K, 1: Q
        const int row = (idx >> 4) & 63;
        const int ch = idx & 15;  // 16-byte chunk of the 256-byte row
        uint4 val = make_uint4(0, 0, 0, 0);
        if (row < n) {
            const uint16_t* src = (m ? p.q : p.k) + ((t0 + row) * kHQK + hq) * kD + ch * 8;
            val = *reinterpret_cast<const uint4*>(src);
        }
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
        mma_tile<kBF16>(tm, smem_u32(sKQ), 128, smem_u32(sKQ), 128, kD, 128, 64, false);
        mma_commit(bar);
    }
    {  // prefix sums of log2 g (64 sequential adds per thread; deterministic)
        const int hl = tid >> 6, i = tid & 63;
        float acc = 0.f;
        for (int m = 0; m <= i; ++m) acc += sml.lg[hl][m];
        sml.LG[hl][i] = acc;
    }
    ok = mbar_wait(bar, phase);
    phase ^= 1;
    tc_fence_after();
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
    tc_fence_before();
    if (__syncthreads_or(!ok)) {
                aborted = true;
                goto done;
            }

    // 3. the Q image of this chunk and q/k head (rows 64-127 of each K-block)
    if (tid == 0) {
        uint8_t* gq = ws + L.off_q + (rec * kHQK + hq) * kQImg;
        bulk_s2g(gq, smem_u32(sKQ + 64 * 128), 64 * 128);
        bulk_s2g(gq + 64 * 128, smem_u32(sKQ + 128 * 128 + 64 * 128), 64 * 128);
        bulk_commit();
    }

    for (int hl = 0; hl < 2; ++hl) {
        const int h = 2 * hq + hl;
        const int64_t rh = rec * kHV + h;
        if (tid == 0) bulk_wait_read_all();  // staging buffers of the previous head are free
        __syncthreads();
        // a. N (strictly lower) -> P, P^T, X = I - N (threads 0-63 own K K^T rows);
        //    output-side P_out (threads 64-127 own Q K^T rows)
        {
            const int i = tid & 63;
            const float LGi = sml.LG[hl][i];
            if (tid < 64) {
                const float bi = sml.beta[hl][i];
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    const float nij = (j < i) ? bi * exp2f(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
                    const float tn = to_tf32(nij);
                    st_f32(sP, sw128_f32(i, j, 64), tn);
                    st_f32(sPT, sw128_f32(j, i, 64), tn);
                    st_f32(sX, sw128_f32(i, j, 64), to_tf32((j == i ? 1.f : 0.f) - nij));
                }
            } else {
#pragma unroll
                for (int j = 0; j < 64; j += 2) {
                    const float p0 = (j <= i) ? exp2f(LGi - sml.LG[hl][j]) * gram[j] : 0.f;
                    const float p1 = (j + 1 <= i) ? exp2f(LGi - sml.LG[hl][j + 1]) * gram[j + 1] : 0.f;
                    __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
                    *reinterpret_cast<__nv_bfloat162*>(sPout + sw128_bf16(i, j, 64)) = v2;
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(ws + L.off_p + rh * kPImg, smem_u32(sPout), kPImg);
            bulk_commit();
            tc_fence_after();
            mma_tile<kTF32>(tm + 64, smem_u32(sP), 64, smem_u32(sPT), 64, 64, 64, 64, false);  // N^2
            mma_commit(bar);
        }
        // b. Neumann rounds: epilogue e updates X (e >= 1) and P (e <= 4)
        for (int e = 0; e <= 5; ++e) {
            ok = mbar_wait(bar, phase);
            phase ^= 1;
            tc_fence_after();
            const int i = 16 * warp + lane;  // M=64 row of this lane (lanes < 16)
            if (e >= 1) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float xp[32];
                    tmem_ld32(taddr(tm, 32 * warp, 32 * half), xp);
                    tmem_wait_ld();
                    if (lane < 16) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const uint32_t off = sw128_f32(i, 32 * half + j, 64);
                            const float x = *reinterpret_cast<const float*>(sX + off);
                            st_f32(sX, off, to_tf32(x + xp[j]));
                        }
                    }
                }
            }
            if (e <= 4) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float pp[32];
                    tmem_ld32(taddr(tm, 32 * warp, 64 + 32 * half), pp);
                    tmem_wait_ld();
                    if (lane < 16) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float v = to_tf32(pp[j]);
                            st_f32(sP, sw128_f32(i, 32 * half + j, 64), v);
                            st_f32(sPT, sw128_f32(32 * half + j, i, 64), v);
                        }
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
                mma_tile<kTF32>(tm, smem_u32(sX), 64, smem_u32(sPT), 64, 64, 64, 64, false);  // X P
                if (e <= 3) mma_tile<kTF32>(tm + 64, smem_u32(sP), 64, smem_u32(sPT), 64, 64, 64, 64, false);
                mma_commit(bar);
            }
        }
        // c. right-hand sides, K-bar^T image (into the free P/P^T space) and the gate vector
        {
            const int j = tid & 63, part = tid >> 6;
            const float LGj = sml.LG[hl][j];
            const float LGc = sml.LG[hl][63];
            const float bj = sml.beta[hl][j];
            const float Gj = exp2f(LGj);
            const float tail = exp2f(LGc - LGj);
            uint8_t* sKT = sP;  // [128 rows k][64 cols j] fp32, 32 KiB over sP + sPT
            if (part == 0) {
#pragma unroll 4
                for (int k = 0; k < kD; ++k) {
                    const float kv =
                        __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(sKQ + sw128_bf16(j, k, 128)));
                    st_f32(sRHS, sw128_f32(k, j, 256), to_tf32(bj * Gj * kv));
                    if (k < 64) st_f32(sKT, sw128_f32(k, j, 128), to_tf32(tail * kv));
                }
            } else {
                const bool act = j < n;
                const uint16_t* vsrc = p.v + ((t0 + j) * kHV + h) * kD;
#pragma unroll 4
                for (int d0 = 0; d0 < kD; d0 += 4) {
                    float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (act) v4 = bf16x4_to_float4(ld_u2(vsrc + d0));
                    st_f32(sRHS, sw128_f32(128 + d0 + 0, j, 256), to_tf32(bj * v4.x));
                    st_f32(sRHS, sw128_f32(128 + d0 + 1, j, 256), to_tf32(bj * v4.y));
                    st_f32(sRHS, sw128_f32(128 + d0 + 2, j, 256), to_tf32(bj * v4.z));
                    st_f32(sRHS, sw128_f32(128 + d0 + 3, j, 256), to_tf32(bj * v4.w));
                }
#pragma unroll 4
                for (int k = 64; k < kD; ++k) {
                    const float kv =
                        __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(sKQ + sw128_bf16(j, k, 128)));
                    st_f32(sKT, sw128_f32(k, j, 128), to_tf32(tail * kv));
                }
                float* gvec = reinterpret_cast<float*>(ws + L.off_vec + rh * kVecBytes);
                gvec[j] = Gj;
                if (j == 0) gvec[64] = exp2f(LGc);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(ws + L.off_kt + rh * kKTImg, smem_u32(sP), kKTImg);
            bulk_commit();
            tc_fence_after();
            mma_tile<kTF32>(tm, smem_u32(sX), 64, smem_u32(sRHS), 256, 64, 64, 256, false);  // [W | U]
            mma_commit(bar);
        }
        ok = mbar_wait(bar, phase);
        phase ^= 1;
        tc_fence_after();
        if (__syncthreads_or(!ok)) {
                aborted = true;
                goto done;
            }
        // d. W (tf32 image) and U (plain fp32) rows -> staging (the RHS space) -> global
        {
            const int i = 16 * warp + lane;
            uint8_t* sW = sRHS;
            float* sU = reinterpret_cast<float*>(sRHS + kWImg);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                float acc[32];
                tmem_ld32(taddr(tm, 32 * warp, 32 * c), acc);
                tmem_wait_ld();
                if (lane < 16) {
                    if (c < 4) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) st_f32(sW, sw128_f32(i, 32 * c + j, 64), to_tf32(acc[j]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(sU + i * kD + 32 * (c - 4) + j) =
                                make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                    }
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(ws + L.off_w + rh * kWImg, smem_u32(sRHS), kWImg);
            bulk_s2g(ws + L.off_u + rh * kUBytes, smem_u32(sRHS + kWImg), kUBytes);
            bulk_commit();
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
constexpr int kSlotQ = 0;
constexpr int kSlotW = kSlotQ + kQImg;
constexpr int kSlotKT = kSlotW + kWImg;
constexpr int kSlotP = kSlotKT + kKTImg;
constexpr int kSlotVec = kSlotP + kPImg;
constexpr int kSlotBytes = kSlotVec + 1024;
constexpr uint32_t kSlotTx = kQImg + kWImg + kKTImg + kPImg + kVecBytes;

template <int BV>
struct CarrySmem {
    static constexpr int kSlots = 0;                               // 2 operand slots
    static constexpr int kS32 = kSlots + 2 * kSlotBytes;           // fp32 S image [BV][128], 4 kblocks
    static constexpr int kS16 = kS32 + BV * 512;                   // bf16 S image [BV][128], 2 kblocks
    static constexpr int kD32 = kS16 + BV * 256;                   // fp32 Delta^T image [BV][64], 2 kblocks
    static constexpr int kD16 = kD32 + BV * 256;                   // bf16 Delta^T image [BV][64], 1 kblock
    static constexpr int kSmall = kD16 + BV * 128;
    static constexpr int kTotal = kSmall + 128 + 1024;
    static constexpr int kTmemCols = 4 * BV < 32 ? 32 : 4 * BV;
};

template <int BV>
__global__ void __launch_bounds__(128, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, const uint8_t* __restrict__ ws, const WsLayout L) {
    using SM = CarrySmem<BV>;
    static_assert(BV == 16 || BV == 32, "value-row tile");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sS32 = sm + SM::kS32;
    uint8_t* sS16 = sm + SM::kS16;
    uint8_t* sD32 = sm + SM::kD32;
    uint8_t* sD16 = sm + SM::kD16;
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
    const int* wbase = reinterpret_cast<const int*>(ws + L.off_base);
    const int rec0 = wbase[s];
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
#pragma unroll
    for (int v = 0; v < BV; ++v) {
        st_f32(sS32, sw128_f32(v, tid, BV), to_tf32(S[v]));
        *reinterpret_cast<__nv_bfloat16*>(sS16 + sw128_bf16(v, tid, BV)) = __float2bfloat16_rn(S[v]);
    }

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
        uint8_t* slot = sm + SM::kSlots + (c & 1) * kSlotBytes;
        const uint32_t fb = full0 + 8 * (c & 1);
        mbar_expect_tx(fb, kSlotTx);
        bulk_g2s(smem_u32(slot + kSlotQ), ws + L.off_q + (r * kHQK + h / kGva) * kQImg, kQImg, fb);
        bulk_g2s(smem_u32(slot + kSlotW), ws + L.off_w + rh * kWImg, kWImg, fb);
        bulk_g2s(smem_u32(slot + kSlotKT), ws + L.off_kt + rh * kKTImg, kKTImg, fb);
        bulk_g2s(smem_u32(slot + kSlotP), ws + L.off_p + rh * kPImg, kPImg, fb);
        bulk_g2s(smem_u32(slot + kSlotVec), ws + L.off_vec + rh * kVecBytes, kVecBytes, fb);
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
            mma_tile<kTF32>(t_ws, smem_u32(sl + kSlotW), 64, smem_u32(sS32), BV, kD, 64, BV, false);
            mma_tile<kBF16>(t_qs, smem_u32(sl + kSlotQ), 64, smem_u32(sS16), BV, kD, 64, BV, false);
            mma_commit(mma1);
        }
        const int tok = 64 * c + row;
        const bool act = lane < 16 && tok < t1 - t0;
        float u[BV];
        if (lane < 16) {
            const float4* up = reinterpret_cast<const float4*>(
                reinterpret_cast<const float*>(ws + L.off_u + rh * kUBytes) + row * kD + v0);
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
        {  // Delta = U - W S0^T  -> Delta^T images (B operand of the next two MMAs)
            float ws_row[BV];
            if constexpr (BV == 16) {
                tmem_ld16(taddr(t_ws, 32 * warp, 0), ws_row);
            } else {
                tmem_ld32(taddr(t_ws, 32 * warp, 0), ws_row);
            }
            tmem_wait_ld();
            if (lane < 16) {
#pragma unroll
                for (int v = 0; v < BV; ++v) {
                    const float d = u[v] - ws_row[v];
                    st_f32(sD32, sw128_f32(v, row, BV), to_tf32(d));
                    *reinterpret_cast<__nv_bfloat16*>(sD16 + sw128_bf16(v, row, BV)) = __float2bfloat16_rn(d);
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
            mma_tile<kTF32>(t_up, smem_u32(sl + kSlotKT), 128, smem_u32(sD32), BV, 64, 128, BV, false);
            mma_tile<kBF16>(t_pd, smem_u32(sl + kSlotP), 64, smem_u32(sD16), BV, 64, 64, BV, false);
            mma_commit(mma2);
        }
        ok = mbar_wait(mma2, c & 1);
        tc_fence_after();
        {  // S1 = G_C S0 + (tail K)^T Delta ; O = scale (G (.) Q S0^T + P Delta)
            float up[BV], qs[BV], pd[BV];
            if constexpr (BV == 16) {
                tmem_ld16(taddr(t_up, 32 * warp, 0), up);
                tmem_ld16(taddr(t_qs, 32 * warp, 0), qs);
                tmem_ld16(taddr(t_pd, 32 * warp, 0), pd);
            } else {
                tmem_ld32(taddr(t_up, 32 * warp, 0), up);
                tmem_ld32(taddr(t_qs, 32 * warp, 0), qs);
                tmem_ld32(taddr(t_pd, 32 * warp, 0), pd);
            }
            tmem_wait_ld();
#pragma unroll
            for (int v = 0; v < BV; ++v) {
                S[v] = fmaf(gc, S[v], up[v]);
                st_f32(sS32, sw128_f32(v, tid, BV), to_tf32(S[v]));
                *reinterpret_cast<__nv_bfloat16*>(sS16 + sw128_bf16(v, tid, BV)) = __float2bfloat16_rn(S[v]);
            }
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
    const bool wide = p.num_seqs * kHV * (kD / 32) >= kSmCount;
    if (wide) {
        using SM = CarrySmem<32>;
        if ((e = set_smem(gdn_chunk_carry_kernel<32>, SM::kTotal)) != cudaSuccess) return e;
        const int64_t grid = p.num_seqs * kHV * (kD / 32);
        gdn_chunk_carry_kernel<32><<<static_cast<unsigned>(grid), 128, SM::kTotal, stream>>>(p, ws, L);
    } else {
        using SM = CarrySmem<16>;
        if ((e = set_smem(gdn_chunk_carry_kernel<16>, SM::kTotal)) != cudaSuccess) return e;
        const int64_t grid = p.num_seqs * kHV * (kD / 16);
        gdn_chunk_carry_kernel<16><<<static_cast<unsigned>(grid), 128, SM::kTotal, stream>>>(p, ws, L);
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
