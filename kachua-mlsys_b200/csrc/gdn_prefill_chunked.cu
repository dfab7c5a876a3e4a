// gdn_prefill_chunked.cu -- chunked-WY varlen GDN prefill on tcgen05 tensor cores.
//
// Replaces the reference's three Triton paths (Direct-v2 kernel.py:886-993,
// Split-WY :379-540, Flat-WY :576-863) with one design: a per-chunk prepare
// kernel and a carry kernel.
//
// Algebra for one chunk of C = 64 tokens of one v-head (state S is [V][K]):
//   G_i   = prod_{m<=i} g_m (kept as log2 G),  Gam_ij = G_i / G_j = exp2(lG_i - lG_j), j <= i
//   N_ij  = beta_i Gam_ij (k_i . k_j)          for j < i     (strictly lower)
//   A     = I + N,   Ainv = A^-1 (the reference: Neumann doubling (I - N)(I + N^2)...(I + N^32))
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
// The inverse.  Ainv is the inverse of a unit lower-triangular 64 x 64
// matrix; instead of the reference's Neumann doubling (log2 C squarings and
// products, each a dependent tensor-core round trip) it is formed blocked
// 2 x 2: the two 32 x 32 diagonal blocks by fp32 forward substitution (one
// column per thread), the off-diagonal block X21 = -X22 (N21 X11) by two
// tcgen05 products -- three dependent steps instead of ten, and the diagonal
// blocks exact in fp32.
//
// Kernels (one prefill call = table + prepare + carry, chained by
// programmatic dependent launch):
//   gdn_chunk_table   one block: chunk records (sequence, first token,
//                     length) for every 64-token chunk of every sequence,
//                     per-sequence record bases, sequences ordered longest
//                     first; zeroes output rows no sequence covers.
//   gdn_chunk_prepare persistent, two 256-thread CTAs per SM, one item =
//                     (chunk record, v-head): TMA loads of K, Q, V into SW128
//                     images; Gram [K;Q] K^T (bf16); N, P and the decay
//                     ratios; Ainv as above; [W | U]^T, Qt^T, Ut^T and
//                     W^T K' (= (K'^T W)^T) as M = 128 fp16 tcgen05
//                     products; 96 KiB of fp16 operand images per item
//                     bulk-stored to the workspace.
//   gdn_chunk_carry   one 448-thread CTA per sequence x v-head (per segment
//                     of one in the segmented and context-parallel modes):
//                     the state lives in TMEM, transposed, and is the A
//                     operand of its own next product; per chunk one
//                     product S [M^T | Qt^T] (M = 128, N = 192, K = 128)
//                     giving the next state and the chunk's output at once
//                     (plus U^T K' issued a chunk early), operands by bulk
//                     copies two chunks ahead, bf16 output tiles by TMA.
// Any q/k and v head counts (v a multiple of q/k): items, records and carry
// chains are per v-head, and v-head h reads q/k head h / (hv / hqk).
// Precision: tensor-core operands are fp16 (round-to-nearest, 11-bit
// significand) or bf16 (the Gram of the bf16 inputs) with fp32
// accumulation; the carried state is fp32 in TMEM and rounded to fp16 only
// as the operand of the next product.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled
#include <string.h>

#include "gdn_common.cuh"
#include "tc05.cuh"

namespace gdn {
using namespace tc05;

constexpr int kC = 64;
// Per (chunk record, v-head) the prepare kernel leaves 96 KiB of f16 operand
// images for the carry, at these offsets:
constexpr int kRecM = 0;          // M = G_C I - K'^T W   [128 k][128 k']  MN-major SW128 (row k: M[k'][k]) 32 KiB
constexpr int kRecQt = 32768;     // Qt^T = (G (.) Q - P W)^T [128 k][64 i] MN-major SW128 16 KiB (with M: one B operand)
constexpr int kRecKb = 49152;     // K' = tail (.) K      [64 j][128 k]    MN-major (2 kblocks) 16 KiB
constexpr int kRecUT = 65536;     // U^T                  [128 v][64 j]    K-major SW128        16 KiB
constexpr int kRecUt = 81920;     // Ut^T = (P U)^T       [128 v][64 i]    SW128 rows           16 KiB
constexpr int kHeadRecBytes = 98304;

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace: header, per-sequence record bases, the chunk table and the
// per-record, per-head operand arrays (every array 1024-byte aligned).
// Segmented carry summaries (few-sequence problems only): per sequence, v-head
// and segment, T (f16 image, 32 KiB) and Z (f16 rows, 32 KiB), or a state
// (Sum0's, or a rank's end state: fp32 rows, 64 KiB) at the Z offset.
constexpr int kSegMaxP = 8;
constexpr int kSegSlotBytes = 98304;

// Segments per chain for N sequences: the most (up to 8) for which both
// passes of the segmented carry fit one wave of CTAs, N x 8 x max(P, 2P - 3)
// <= sms, and pass C (which streams every chunk's operands) keeps to two
// thirds of the SMs, N x 8 x P <= 2 sms / 3: more concurrent chains than that
// saturate HBM (about 70 GB/s each) and the split costs more than it saves.
// Two segments were measured to gain nothing; 1 = no segmented carry.
__host__ __device__ inline int seg_segments(int64_t N, int sms, int hv = kHV) {
    int best = 1;
    for (int P = 3; P <= kSegMaxP; ++P)
        if (N > 0 && N * hv * (P > 2 * P - 3 ? P : 2 * P - 3) <= sms && 3 * N * hv * P <= 2 * sms) best = P;
    return best;
}

struct WsLayout {
    int64_t R;  // record capacity: ceil(T / 64) + N bounds sum_s ceil(len_s / 64)
    int64_t off_hdr, off_base, off_order, off_table, off_rec;
    int64_t total;      // everything the single-pass carry needs
    int64_t seg_slots;  // summary slots per chain (segments on a 148-SM part; 1: none)
    int64_t off_seg;    // segment summaries (0 without slots)
    int64_t total_seg;  // total + the summaries
    int64_t cp_world;   // context parallel: ranks (seg_slots = segments per rank); 0 otherwise
    int64_t off_gather; // context parallel: the all-gathered rank summaries (cp_world x N x 8 slots)
    int64_t hv;         // v-heads (records per chunk; carry chains per sequence)
};

__host__ __device__ inline WsLayout ws_layout(int64_t T, int64_t N, int hv = kHV) {
    WsLayout L;
    L.hv = hv;
    L.R = (T + kC - 1) / kC + N;
    int64_t o = 0;
    L.off_hdr = o;
    o += 1024;
    L.off_base = o;
    o = align_up(o + 4 * (N + 1), 1024);
    L.off_order = o;  // sequences by chunk count, longest first
    o = align_up(o + 4 * N, 1024);
    L.off_table = o;
    o = align_up(o + 16 * L.R, 1024);
    L.off_rec = o;
    o += L.R * hv * kHeadRecBytes;
    L.total = align_up(o, 1024);
    L.cp_world = 0;
    L.off_gather = 0;
    L.seg_slots = seg_segments(N, kSmCount, hv);
    L.off_seg = L.seg_slots >= 2 ? L.total : 0;
    L.total_seg = L.total + (L.seg_slots >= 2 ? N * hv * L.seg_slots * static_cast<int64_t>(kSegSlotBytes) : 0);
    return L;
}

// Workspace for the fastest dispatch (with room for the segmented carry when
// it may apply) and the minimum every chunked launch needs.
size_t chunked_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int hv = kHV) {
    return static_cast<size_t>(ws_layout(total_tokens, num_seqs, hv).total_seg);
}
size_t chunked_workspace_min_bytes(int64_t total_tokens, int64_t num_seqs, int hv = kHV) {
    return static_cast<size_t>(ws_layout(total_tokens, num_seqs, hv).total);
}

// ------------------------------------------------------------ chunk table --
// One block: per sequence, ceil(len / 64) records; exclusive scan -> base[s];
// table[rec] = (seq, first token, length <= 64).  Records past the capacity
// (only reachable with overlapping, invalid cu_seqlens) are dropped and
// reported.
// Block 0 builds the table; every block also zeroes the output rows of
// tokens outside [cu_seqlens[0], cu_seqlens[N]) (the oracle's torch.zeros),
// which saves the chunked path a separate launch.
__global__ void __launch_bounds__(1024) gdn_chunk_table_kernel(const PrefillParams p, uint8_t* ws, WsLayout L) {
    if (blockIdx.x == 0) {
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
                if (excl + nch > L.R) record_status(16 /* GDN_ERR_DEVICE_BAD_SEQLENS */);  // records dropped
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
        __syncthreads();  // base[] is complete (global writes of this block, visible after the barrier)
        {
            // the records, one per thread: record r belongs to the last sequence s
            // with base[s] <= r (binary search; empty sequences share a base)
            const int nrec = base[p.num_seqs];
            const int N = static_cast<int>(p.num_seqs);
            for (int r = tid; r < nrec; r += 1024) {
                int lo = 0, hi = N - 1;  // base[lo] <= r < base[N]
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (base[mid] <= r) lo = mid; else hi = mid - 1;
                }
                int64_t t0, t1;
                seq_bounds(p, lo, t0, t1);
                const int64_t ts = t0 + static_cast<int64_t>(r - base[lo]) * kC;
                const int64_t len = t1 - ts < kC ? t1 - ts : kC;
                table[r] = make_int4(lo, static_cast<int>(ts), static_cast<int>(len), 0);
            }
        }
        if (p.num_seqs == 1) {
            if (tid == 0) reinterpret_cast<int*>(ws + L.off_order)[0] = 0;
        } else {
            // Sequences in order of decreasing chunk count (counting sort, counts
            // above 1023 share the first bin): the single-pass carry starts the
            // longest chains first, so that short ones fill in behind them.
            __shared__ int hist[1024];
            hist[tid] = 0;
            __syncthreads();
            const int N = static_cast<int>(p.num_seqs);
            auto bin_of = [&](int s2) {
                const int n = base[s2 + 1] - base[s2];
                return 1023 - (n < 1023 ? n : 1023);
            };
            for (int s2 = tid; s2 < N; s2 += 1024) atomicAdd(&hist[bin_of(s2)], 1);
            __syncthreads();
            const int hv = hist[tid];
            int x = hv;  // exclusive scan of the 1024 bins
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
                warp_tot[lane] = w;
            }
            __syncthreads();
            hist[tid] = (warp > 0 ? warp_tot[warp - 1] : 0) + x - hv;
            __syncthreads();
            int* order = reinterpret_cast<int*>(ws + L.off_order);
            for (int s2 = tid; s2 < N; s2 += 1024) order[atomicAdd(&hist[bin_of(s2)], 1)] = s2;
        }
    }
    zero_uncovered_rows(p);
}

// ---------------------------------------------------------------- prepare --
// Per chunk record and v-head (an item; persistent CTAs of 256 threads, two per
// SM, take items blockIdx.x, + gridDim.x, ...): everything the carry's chain
// does not need, finished per chunk in fp16 operand images (fp32
// accumulation) and bulk-stored to the workspace:
//   M    = G_C I - K'^T W     [k][k']  MN-major   (row k holds M[k'][k])     } B of the carry's one
//   Qt^T = (G (.) Q - P W)^T  [k][i]   MN-major                              } product S [M^T | Qt^T]
//   K'   = tail (.) K         [j][k]   MN-major   (B of the carry's U^T K')
//   U^T                       [v][j]   K-major    (A of the carry's U^T K')
//   Ut^T = (P U)^T            [v][i]   SW128 rows (added by the output epilogue)
// K, Q and V arrive by tiled TMA loads straight into SW128 images (rows past
// the chunk hold the next tokens or zeros; every use masks them).  A^-1 of
// the unit-lower-triangular A = I + N is blocked 2 x 2: the two 32 x 32
// diagonal inverses by fp32 forward substitution (a column per thread), the
// off-diagonal block X21 = -X22 (N21 X11) by two tcgen05 products.  The
// remaining products are computed transposed (M = 128 = k or v rows, all TMEM
// lanes busy): [W | U]^T = [bGK | bV]^T A^-T, Qt^T = Q^T diag(G) + W^T (-P)^T,
// Ut^T = -(U^T (-P)^T) and W^T K' (the transpose of K'^T W, so that lane k
// holds column k of M and M is written MN-major, beside Qt^T).
constexpr int kPrepThreads = 256;
constexpr int kPrKQ = 0;        // bf16 [K;Q] K-major, kblock b at b*16K (rows 0-63 K, 64-127 Q); K rows -> K' in place
constexpr int kPrN = 32768;     // fp32 diagonal blocks of N (8K) | f16 NL (8K); later TB | diag(G); then Qt^T staging
constexpr int kPrPO = 49152;    // f16 -P [64 i][64 j] K-major                     } later Ut^T staging
constexpr int kPrX = 57344;     // f16 A^-1 [64 i][64 m] K-major                  }
constexpr int kPrRHS = 65536;   // f16 [bGK | bV] MN-major [64 j][256] (V by TMA) -> W^T | U^T K-major [128][64] -> M staging
constexpr int kPrSmall = 98304;
constexpr int kPrSmem = kPrSmall + 2048 + 1024;
constexpr int kPrTmemCols = 256;

struct PrepSmall {
    float LG[kC];     // inclusive prefix of log2 g (0 past the chunk)
    float beta[kC];   // 0 past the chunk
    float sBG[kC];    // beta G (0 past the chunk)
    float sTail[kC];  // G_C / G (0 past the chunk)
    float wtot[4];
    uint64_t bar_load;
    uint64_t bar_mma;
    uint64_t bar_w;
    uint64_t bar_e;
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

// Plain (compiler-scheduled) shared-memory accesses addressed by the 32-bit
// shared address used for descriptors: the generic pointer keeps the shared
// address space visible, so loads batch and overlap instead of serialising
// like volatile asm would.
struct Smem {
    uint8_t* p;  // generic pointer to the byte at shared address a
    uint32_t a;
    __device__ __forceinline__ uint4 ld16(uint32_t addr) const { return *reinterpret_cast<const uint4*>(p + (addr - a)); }
    __device__ __forceinline__ float4 ldf4(uint32_t addr) const {
        return *reinterpret_cast<const float4*>(p + (addr - a));
    }
    __device__ __forceinline__ void st16(uint32_t addr, uint4 v) const { *reinterpret_cast<uint4*>(p + (addr - a)) = v; }
    __device__ __forceinline__ void stf4(uint32_t addr, float4 v) const {
        *reinterpret_cast<float4*>(p + (addr - a)) = v;
    }
    __device__ __forceinline__ void st2(uint32_t addr, uint16_t v) const {
        *reinterpret_cast<uint16_t*>(p + (addr - a)) = v;
    }
};

// 1024-byte aligned base of the dynamic shared memory, derived from the
// __shared__ array itself so the address space stays visible.
__device__ __forceinline__ uint8_t* smem_align1024(uint8_t* raw) {
    return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

// bar.sync on named barrier `id` among `count` threads (a multiple of 32)
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// named barrier that also returns the AND of `pred` over the `count` threads
__device__ __forceinline__ bool named_sync_and(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// fp32 diagonal 32 x 32 block d of N: row r is 128 bytes, its 16-byte chunk c
// at position c ^ (r & 7)
__device__ __forceinline__ uint32_t nd_off(int d, int r, int m) {
    return d * 4096 + r * 128 + ((((m >> 2) ^ (r & 7))) << 4) + (m & 3) * 4;
}

__global__ void __launch_bounds__(kPrepThreads, 2)
    gdn_chunk_prepare_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L,
                             const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmV) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_align1024(smem_raw);
    const Smem S{sm, smem_u32(sm)};
    PrepSmall& sml = *reinterpret_cast<PrepSmall*>(sm + kPrSmall);
    const uint32_t aKQ = smem_u32(sm + kPrKQ), aN = smem_u32(sm + kPrN), aPO = smem_u32(sm + kPrPO),
                   aX = smem_u32(sm + kPrX), aRHS = smem_u32(sm + kPrRHS);
    const uint32_t aNL = aN + 8192;  // f16 N21 image (later diag(G)); aN: fp32 diagonal blocks (later TB)

    // Thread roles in the accumulator epilogues: warp w reads TMEM lanes
    // 32 (w & 3).. (its sub-partition) and column half hc = w >> 2.
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = warp & 3, hc = warp >> 2;
    griddep_launch_dependents();  // the carry may start its prologue on freed SMs
    griddep_wait();               // the chunk table is complete
    const int nrec = reinterpret_cast<const int*>(ws + L.off_hdr)[0];
    const int hv = p.hv, gva = p.hv / p.hqk;
    const int64_t nitems = static_cast<int64_t>(nrec) * hv;
    if (static_cast<int64_t>(blockIdx.x) >= nitems) return;
    const int4* table = reinterpret_cast<const int4*>(ws + L.off_table);

    // barL: the item's input loads (one phase per item); barM: Gram, T, X22 T
    // commits (three per item); barW: [W | U]^T and final commits; barE: TB and
    // X21 written (two phases per item each)
    const uint32_t barL = smem_u32(&sml.bar_load), barM = smem_u32(&sml.bar_mma), barW = smem_u32(&sml.bar_w),
                   barE = smem_u32(&sml.bar_e);
    if (tid == 0) {
        mbar_init(barL, 1);
        mbar_init(barM, 1);
        mbar_init(barW, 1);
        mbar_init(barE, 2);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&sml.tmem_base), kPrTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sml.tmem_base;

    // Persistent CTAs (two per SM) walk the items (chunk record, v-head)
    // blockIdx.x, + gridDim.x, ...; items are record-major, so the 8 v-heads of
    // a chunk run side by side (their K and Q loads share L2 lines).  The next
    // item's table entry and gate inputs are read, and its K, Q and V prefetched
    // into L2, while the current one is processed.
    int4 te = table[blockIdx.x / hv];
    uint16_t ga = 0, gb = 0;  // raw bf16 gate inputs a, b of token tid of the item (tid < 64)
    if (tid < te.z) {
        const int64_t t = static_cast<int64_t>(te.y) + tid;
        ga = p.a[t * hv + blockIdx.x % hv];
        gb = p.b[t * hv + blockIdx.x % hv];
    }
    bool stop = false;
    int it = 0;
    for (int64_t item = blockIdx.x; item < nitems && !stop; item += gridDim.x, ++it) {
        const int64_t rec = item / hv;
        const int h = static_cast<int>(item % hv), hq = h / gva;
        const uint32_t pl = static_cast<uint32_t>(it) & 1u;  // parity of the item's barL and first barM phase
        const int t0 = te.y;  // first token (T < 2^31, checked on the host)
        const int n = te.z;   // tokens in this chunk (1..64)
        uint8_t* out_rec = ws + L.off_rec + (rec * hv + h) * kHeadRecBytes;
        const int64_t nitem = item + gridDim.x;
        const int4 te_next = nitem < nitems ? table[nitem / hv] : te;  // used after the Gram issue
        uint16_t ga_next = 0, gb_next = 0;
        if (tid == 0) {
            mbar_expect_tx(barL, 6 * 8192);
            tma_load_3d(aRHS + 16384, &tmV, 0, h, t0, barL);
            tma_load_3d(aRHS + 24576, &tmV, 64, h, t0, barL);
            bulk_wait_read<0>();  // the previous item's M has left [K;Q]
            tma_load_3d(aKQ, &tmK, 0, hq, t0, barL);
            tma_load_3d(aKQ + 16384, &tmK, 64, hq, t0, barL);
            tma_load_3d(aKQ + 8192, &tmQ, 0, hq, t0, barL);
            tma_load_3d(aKQ + 24576, &tmQ, 64, hq, t0, barL);
        }
        // zero the A^-1 image (its off-diagonal blocks stay zero until X21 is known)
        S.st16(aX + tid * 32, make_uint4(0, 0, 0, 0));
        S.st16(aX + tid * 32 + 16, make_uint4(0, 0, 0, 0));
        // gates and the inclusive prefix of log2 g (threads 0-63 = tokens; warp scans)
        float lgs = 0.f;
        if (tid < kC) {
            float lg = 0.f, bt = 0.f;
            if (tid < n) {
                lg = gdn_log2_decay(p.A_log[h], p.dt_bias[h], bf16_bits_to_float(ga));
                bt = 1.0f / (1.0f + expf(-bf16_bits_to_float(gb)));
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
        __syncthreads();
        if (tid < kC) {  // per-row scales (0 past the chunk)
            const bool act = tid < n;
            sml.sBG[tid] = act ? sml.beta[tid] * fast_exp2(lgs) : 0.f;
            sml.sTail[tid] = act ? fast_exp2(sml.LG[kC - 1] - lgs) : 0.f;
        }
        bool ok = mbar_wait(barL, pl);
        // 1. Gram [K;Q] K^T (bf16, M=128, N=64, K=128) -> TMEM columns 0-63
        if (tid == 0 && ok) {
            tc_fence_after();
            mma_ct<kBF16, false, false, kD, 128, 128, 128, 64>(tm, aKQ, aKQ, false);
            mma_commit(barM);
        }
        __syncthreads();  // the row scales are visible
        if (nitem < nitems && tid < kC) {  // the next item: gate inputs, and its K, Q and V into L2
            const int nh = static_cast<int>(nitem % hv);
            if (tid < te_next.z) {
                const int64_t t = static_cast<int64_t>(te_next.y) + tid;
                ga_next = p.a[t * hv + nh];
                gb_next = p.b[t * hv + nh];
            }
            if (tid == 32) {
                const int nt0 = te_next.y;
                if (nh % gva == 0) {
                    tma_prefetch_3d(&tmK, 0, nh / gva, nt0);
                    tma_prefetch_3d(&tmK, 64, nh / gva, nt0);
                    tma_prefetch_3d(&tmQ, 0, nh / gva, nt0);
                    tma_prefetch_3d(&tmQ, 64, nh / gva, nt0);
                }
                tma_prefetch_3d(&tmV, 0, nh, nt0);
                tma_prefetch_3d(&tmV, 64, nh, nt0);
            }
        }
        ok = mbar_wait(barM, pl) && ok;
        tc_fence_after();
        {
            // 2. Gram epilogue, 32 columns j = 32 hc + e per thread.  Rows 0-63 give
            //    N: its fp32 diagonal 32-blocks and the f16 image NL of its
            //    lower-left block (zero elsewhere); rows 64-127 the f16 image of
            //    -P, P = Gam (.) Q K^T for j <= i.
            float g[32];
            tmem_ld32(taddr(tm, 32 * q, 32 * hc), g);
            tmem_wait_ld();
            if (q < 2) {
                const int i = 32 * q + lane;
                const float LGi = sml.LG[i], bi = sml.beta[i];
                const bool act = i < n;
                float nv[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int j = 32 * hc + e;
                    nv[e] = (j < i && act) ? bi * fast_exp2(LGi - sml.LG[j]) * g[e] : 0.f;
                }
                if (hc == q) {  // the diagonal block d = q: fp32 rows for the substitution
#pragma unroll
                    for (int m0 = 0; m0 < 32; m0 += 4)
                        S.stf4(aN + nd_off(q, lane, m0), make_float4(nv[m0], nv[m0 + 1], nv[m0 + 2], nv[m0 + 3]));
                }
                const bool lower_left = q == 1 && hc == 0;
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = lower_left ? nv[e0 + e] : 0.f;
                    S.st16(aNL + h16(i, 32 * hc + e0, 64), f16x8(f));
                }
            } else {
                const int i = 32 * (q - 2) + lane;
                const float LGi = sml.LG[i];
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float pv[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int j = 32 * hc + e0 + e;
                        pv[e] = (j <= i) ? -fast_exp2(LGi - sml.LG[j]) * g[e0 + e] : 0.f;
                    }
                    S.st16(aPO + h16(i, 32 * hc + e0, 64), f16x8(pv));
                }
            }
        }
        tc_fence_before();
        if (__syncthreads_or(!ok)) goto abort;
        if (warp < 2) {
            // 3a. diagonal blocks of A^-1: (I + N_dd) x = e_j, d = warp, column
            //     j = lane, 32 rows in fp32 (four partial sums per row)
            const int d = warp, j = lane;
            float x[32];
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                float a0 = (r == j) ? 1.f : 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
                for (int m = 0; m < r; m += 4) {
                    const float4 nv = S.ldf4(aN + nd_off(d, r, m));
                    a0 = fmaf(-nv.x, x[m], a0);
                    if (m + 1 < r) a1 = fmaf(-nv.y, x[m + 1], a1);
                    if (m + 2 < r) a2 = fmaf(-nv.z, x[m + 2], a2);
                    if (m + 3 < r) a3 = fmaf(-nv.w, x[m + 3], a3);
                }
                x[r] = (a0 + a1) + (a2 + a3);
            }
#pragma unroll
            for (int r = 0; r < 32; ++r) S.st2(aX + h16(32 * d + r, 32 * d + j, 64), __half_as_ushort(__float2half_rn(x[r])));
        } else {
            // 3b. [bGK | bV] in fp16 over the RHS (the scale depends on the row only,
            //     so 16-byte chunks convert in place of their swizzled position),
            //     while warps 0-1 solve; K stays bf16 here (read by the Gram MMA)
#pragma unroll 2
            for (int it = 0; it < 11; ++it) {
                const int u = it * (kPrepThreads - 64) + (tid - 64);
                if (u < 2048) {
                    const int blk = u >> 9;  // 0, 1: K kblocks -> RHS columns 0-127; 2, 3: V blocks in place
                    const int row = (u >> 3) & 63;
                    const uint32_t in_row = row * 128 + (u & 7) * 16;
                    const uint32_t src = blk < 2 ? aKQ + blk * 16384 + in_row : aRHS + blk * 8192 + in_row;
                    uint4 res = make_uint4(0, 0, 0, 0);
                    if (row < n) {
                        const float sc = blk < 2 ? sml.sBG[row] : sml.beta[row];
                        float f[8];
                        bf16x8_to_f32(S.ld16(src), f);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] *= sc;
                        res = f16x8(f);
                    }
                    S.st16(aRHS + blk * 8192 + in_row, res);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {  // 4. T = N21 X11 (lower-left block of NL . diag(X11, X22)) -> columns 0-63, M=64
            tc_fence_after();
            mma_ct<kF16, false, true, 64, 64, 64, 64, 64>(tm, aNL, aX, false);
            mma_commit(barM);
        }
        if (warp == 2 || warp == 3) {
            // The completion of A^-1 runs on sub-partitions 2, 3 (rows 32-63)
            // while the other warps convert K and Q:
            //   TB = [0 0; T 0] as the f16 MN-major B image (over the fp32
            //   diagonal blocks; lanes 16-31 write its zero rows 0-31), then
            //   X21 = -(X22 T) into A^-1 -- each step handed to the MMA issuer
            //   through barE.
            bool okw = mbar_wait(barM, pl ^ 1u);
            tc_fence_after();
            float t32[32];
            tmem_ld32(taddr(tm, 32 * q, 0), t32);
            tmem_wait_ld();
            {
                const int i = lane < 16 ? 16 * q + lane : 16 * (q - 2) + (lane - 16);
                const bool tri = lane < 16;
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = tri ? t32[e0 + e] : 0.f;
                    S.st16(aN + h16(i, e0, 64), f16x8(f));
                    S.st16(aN + h16(i, 32 + e0, 64), make_uint4(0, 0, 0, 0));
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(barE);
            okw = mbar_wait(barM, pl) && okw;
            tc_fence_after();
            tmem_ld32(taddr(tm, 32 * q, 64), t32);
            tmem_wait_ld();
            if (lane < 16) {
                const int i = 16 * q + lane;
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = -t32[e0 + e];
                    S.st16(aX + h16(i, e0, 64), f16x8(f));
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(barE);
            ok = ok && okw;
        } else if (warp >= 4) {
            // 4b. in place over [K;Q] (bf16 -> f16, rows >= n zero): K' = tail (.) K
            //     in the K rows, plain Q in the Q rows (the A operand of Qt^T)
#pragma unroll 2
            for (int it = 0; it < 16; ++it) {
                const int u = it * 128 + (tid - 128);
                const int kb = u >> 10, qrow = (u >> 9) & 1, row = (u >> 3) & 63;
                const uint32_t addr = aKQ + kb * 16384 + qrow * 8192 + row * 128 + (u & 7) * 16;
                uint4 res = make_uint4(0, 0, 0, 0);
                if (row < n) {
                    const float sc = qrow ? 1.f : sml.sTail[row];
                    float f[8];
                    bf16x8_to_f32(S.ld16(addr), f);
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] *= sc;
                    res = f16x8(f);
                }
                S.st16(addr, res);
            }
            fence_async_smem();
        }
        if (tid == 0) {
            // 5. X22 T -> columns 64-127 (M=64), once TB is written
            ok = mbar_wait(barE, 0) && ok;
            tc_fence_after();
            mma_ct<kF16, false, true, 64, 64, 64, 64, 64>(tm + 64, aX, aN, false);
            mma_commit(barM);
            // 6. [W | U]^T = [bGK | bV]^T A^-T, once X21 is written: W^T -> columns 0-63,
            //    U^T -> 64-127 (M=128)
            ok = mbar_wait(barE, 1) && ok;
            tc_fence_after();
            mma_ct<kF16, true, false, 64, 64, 64, 128, 64>(tm, aRHS, aX, false);
            mma_ct<kF16, true, false, 64, 64, 64, 128, 64>(tm + 64, aRHS + 16384, aX, false);
            mma_commit(barW);
        }
        ok = mbar_wait(barW, 0) && ok;
        tc_fence_after();
        if (tid < 2 * kC) {  // diag(G) (rows >= n zero) over NL, dead since T = N21 X11
            const int i = tid >> 1, half = tid & 1;
            const float Gi = i < n ? fast_exp2(sml.LG[i]) : 0.f;
#pragma unroll
            for (int e0 = 0; e0 < 32; e0 += 8) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = (32 * half + e0 + e == i) ? Gi : 0.f;
                S.st16(aNL + h16(i, 32 * half + e0, 64), f16x8(f));
            }
        }
        {  // row 32 q + lane of W^T (hc = 0) or U^T (hc = 1) -> f16 K-major images [128][64] over the RHS
            float a0[32], a1[32];
            tmem_ld32(taddr(tm, 32 * q, 64 * hc), a0);
            tmem_ld32(taddr(tm, 32 * q, 64 * hc + 32), a1);
            tmem_wait_ld();
            const int r = 32 * q + lane;
            const uint32_t img = aRHS + hc * 16384;
#pragma unroll
            for (int e0 = 0; e0 < 32; e0 += 8) {
                S.st16(img + h16(r, e0, 128), f16x8(a0 + e0));
                S.st16(img + h16(r, 32 + e0, 128), f16x8(a1 + e0));
            }
        }
        fence_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) goto abort;
        if (tid == 0) {
            // 7. Qt^T = Q^T diag(G) + W^T (-P)^T -> columns 0-63; -(Ut^T) = U^T (-P)^T -> 64-127;
            //    W^T K' = (K'^T W)^T -> 128-255 (all M=128)
            tc_fence_after();
            mma_ct<kF16, true, false, 64, 128, 64, 128, 64>(tm, aKQ + 8192, aNL, false);
            mma_ct<kF16, false, false, 64, 128, 64, 128, 64>(tm, aRHS, aPO, true);
            mma_ct<kF16, false, false, 64, 128, 64, 128, 64>(tm + 64, aRHS + 16384, aPO, false);
            mma_ct<kF16, false, true, 64, 128, 128, 128, 128>(tm + 128, aRHS, aKQ, false);
            mma_commit(barW);
            bulk_s2g(out_rec + kRecUT, aRHS + 16384, 16384);  // U^T
            bulk_s2g(out_rec + kRecKb, aKQ, 8192);            // K': two 8 KiB kblocks
            bulk_s2g(out_rec + kRecKb + 8192, aKQ + 16384, 8192);
            bulk_commit();
        }
        ok = mbar_wait(barW, 1) && ok;
        tc_fence_after();
        {
            // 8. row r = 32 q + lane: Qt^T (hc = 0, staging over N) or Ut^T (hc = 1,
            //    over -P and A^-1) -- regions no bulk store is reading -- then,
            //    once U^T and K' have left shared memory, half hc of
            //    M = G_C I - K'^T W (over [K;Q])
            const int r = 32 * q + lane;
            {
                float a0[32], a1[32];
                tmem_ld32(taddr(tm, 32 * q, 64 * hc), a0);
                tmem_ld32(taddr(tm, 32 * q, 64 * hc + 32), a1);
                tmem_wait_ld();
                const float sg = hc ? -1.f : 1.f;
                const uint32_t img = hc ? aPO : aN;
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float f[8], f2[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = sg * a0[e0 + e], f2[e] = sg * a1[e0 + e];
                    S.st16(img + h16(r, e0, 128), f16x8(f));
                    S.st16(img + h16(r, 32 + e0, 128), f16x8(f2));
                }
            }
            fence_async_smem();
            if (__syncthreads_or(!ok)) goto abort;
            if (tid == 0) {
                bulk_s2g(out_rec + kRecQt, aN, 16384);
                bulk_s2g(out_rec + kRecUt, aPO, 16384);
                bulk_commit();
                bulk_wait_read<1>();  // U^T and K' (the older group) have left shared memory
            }
            const float Gc = fast_exp2(sml.LG[kC - 1]);
            float acc[2][32];
#pragma unroll
            for (int c = 0; c < 2; ++c) tmem_ld32(taddr(tm, 32 * q, 128 + 64 * hc + 32 * c), acc[c]);
            tmem_wait_ld();
            __syncthreads();  // [K;Q] is free
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int col0 = 64 * hc + 32 * c;  // image column k' of row r = k: M[k'][k]
#pragma unroll
                for (int e0 = 0; e0 < 32; e0 += 8) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = (col0 + e0 + e == r ? Gc : 0.f) - acc[c][e0 + e];
                    S.st16(aKQ + h16(r, col0 + e0, 128), f16x8(f));
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(out_rec + kRecM, aKQ, 32768);
            bulk_commit();
            // Qt and Ut have left N, -P and A^-1 (rewritten from the next item's
            // start on); M's read of [K;Q] overlaps the next item's start and is
            // awaited before its K and Q loads
            bulk_wait_read<1>();
        }
        goto done;
abort:
        if (tid == 0) {
            record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
            mbar_wait(barL, pl);  // the input loads may still be in flight (bounded)
            bulk_wait_all();
        }
        stop = true;
done:
        tc_fence_before();
        __syncthreads();  // shared memory and TMEM are free for the next item
        tc_fence_after();
        te = te_next;
        ga = ga_next;
        gb = gb_next;
    }
    if (tid == 0) bulk_wait_read<0>();  // the last M has left shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, kPrTmemCols);
    }
}

// ------------------------------------------------------------------ carry --
// One CTA per sequence x v-head (or per segment of one, below).  The state
// lives in TMEM in transposed form (lane = value row v, columns = k) and is
// its own MMA operand:
//   chain   S_{c+1}^T <- U_c^T K'_c + S_c M_c^T     [v][k], fp32 accumulator
//   output  O_c^T      = S_c Qt_c^T                  [v][i]
// as ONE product per chunk, S_c [M_c^T | Qt_c^T] (M = 128, N = 192, K = 128;
// B = [M | Qt^T] MN-major, three 16 KiB N blocks), into the 192 accumulator
// columns [S | O] of the chunk's parity: U^T K' is issued one chunk early
// into the S columns, the O columns were cleared by the output warps.  One
// N = 192 product holds the tensor pipe for 8 x ~96 cycles where an N = 128
// and an N = 64 product took 8 x (64 + 45).  S is read from TMEM as fp16 --
// the A operand -- so no shared-memory state image exists.  Warp roles:
//   warps 0-7   state epilogue: warp w owns lanes 32 (w & 3).. and k columns
//               64 (w >> 2)..: fp32 accumulator -> fp16 A operand of the next
//               chunk, and the fp32 final state;
//   warps 8-11  output epilogue: lane = v, 64 columns = tokens; reads and
//               clears the O columns, adds Ut, writes bf16 rows;
//   warp 12     one thread issues every MMA;
//   warp 13     one thread issues the bulk copies (refills follow the state
//               MMA's completion, off the MMA issuer's path).
// [M | Qt^T] is double-buffered, [K' | U^T] triple-buffered, each refilled
// when the MMA that read it is known complete, two chunks before use.
//
// Segmented carry (few, long sequences): the chunks of a sequence are split
// into P segments and the affine chunk maps composed, S_b = S_a T + Z over a
// segment [a, b), with T = M_a^T ... M_{b-1}^T and Z the chain from S_a = 0.
// Pass A (mode 1) runs, per segment s < P-1, the chain from the true initial
// state (s = 0, giving S at the start of segment 1), or from I without the
// U^T K' terms (T_s) and from 0 (Z_s); pass C (mode 2) rebuilds each
// segment's initial state, S_{s+1} = S_s T_s + Z_s, and runs the segment with
// outputs.  Mode 0 is the single pass over whole sequences.
//
// Context parallel (modes 4-6): rank r holds the r-th token range of every
// sequence, cut into nP = seg_slots segments of its own.
// Mode 4 is pass A over the rank's segments (rank 0's segment 0: Sum0),
// writing every summary a later segment composes (an empty segment writes
// T = I, Z = 0).  Mode 6 composes them into one summary per rank (rank 0:
// its end state E_0); the ranks all-gather those; mode 5 is pass C, rank
// r >= 1 starting from E_0 and composing ranks 1 .. r-1, then its own
// segments before the CTA's.
constexpr int kCarryThreads = 448;
// [M | Qt^T] MN-major [128 k][128 k' | 64 i] (three 16 KiB N blocks), 2 x 48 KiB
constexpr int kCaM = 0;
constexpr int kCaMQBytes = 49152;
constexpr int kCaKU = 2 * kCaMQBytes;           // K' [64 j][128 k] (MN-major) + U^T [128 v][64 j] (K-major), 3 x 32 KiB
constexpr int kCaSmall = kCaKU + 3 * 32768;     // (the composition steps' T and Z buffers span [0, kCaSmall))
constexpr int kCaOut = kCaSmall + 1024;         // bf16 output tile [64 i][128 v]: two SW128 images (v 0-63, 64-127)
constexpr int kCaSmem = kCaOut + 16384 + 1024;
// per chunk parity b: [accS | accO] at 192 b (the product's N = 192 columns), fp16 S x 2 at [384, 512)
constexpr int kCaTmemCols = 512;

enum CarryRole { kRoleMain = 0, kRoleSum0 = 1, kRoleSumT = 2, kRoleSumZ = 3 };

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h2 = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h2);
}

// fp32 [128 v][128 k] matrices of the segment summaries: row v is 512 bytes,
// its 16-byte chunk c (k = 4c .. 4c+3) stored at position c ^ (v & 31)
__device__ __forceinline__ uint32_t zrow_off(int v, int c) { return v * 512 + ((c ^ (v & 31)) << 4); }
// f16 [128 v][128 k] segment Z summaries: row v is 256 bytes, its 16-byte
// chunk c (k = 8c .. 8c+7) stored at position c ^ (v & 15)
__device__ __forceinline__ uint32_t zh_off(int v, int c) { return v * 256 + ((c ^ (v & 15)) << 4); }

__global__ void __launch_bounds__(kCarryThreads, 1)
    gdn_chunk_carry_kernel(const PrefillParams p, uint8_t* __restrict__ ws, const WsLayout L, const int mode,
                           const int P, const __grid_constant__ CUtensorMap tmO) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_align1024(smem_raw);
    const Smem Sm{sm, smem_u32(sm)};
    const uint32_t aM = smem_u32(sm + kCaM), aKU = smem_u32(sm + kCaKU);
    const uint32_t bar0 = smem_u32(sm + kCaSmall);
    auto fullM = [&](int b) { return bar0 + 8 * b; };         // 2 ([M | Qt^T])
    auto fullKU = [&](int b) { return bar0 + 16 + 8 * b; };   // 3
    // the chunk's product done (next state and output), alternating by chunk
    // parity so that a late waiter never sees the same barrier complete twice
    auto mmaS = [&](int c) { return (c & 1) ? bar0 + 120 : bar0 + 64; };
    const uint32_t imgReady = bar0 + 88;
    auto oFree = [&](int b) { return bar0 + 96 + 8 * b; };    // 2
    const uint32_t drain = bar0 + 112;
    // composition steps: three load barriers (bar0 + 136, + 144, + 160) and the MMA's
    auto proLoad = [&](int b) { return b == 2 ? bar0 + 160 : bar0 + 136 + 8 * b; };
    const uint32_t proMma = bar0 + 152;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kCaSmall + 128);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    griddep_launch_dependents();
    // this CTA's task
    int64_t unit;
    int seg = 0, role = kRoleMain, nP = 1;
    if (mode == 0) {  // longest sequences first
        unit = static_cast<int64_t>(reinterpret_cast<const int*>(ws + L.off_order)[blockIdx.x / p.hv]) * p.hv +
               blockIdx.x % p.hv;
    } else if (mode == 2) {
        nP = P;
        unit = blockIdx.x / P;
        seg = static_cast<int>(blockIdx.x % P);
    } else if (mode == 4) {  // context parallel pass A on rank P: summaries of its nP segments
        nP = static_cast<int>(L.seg_slots);
        const int per = P == 0 ? 2 * nP - 1 : 2 * nP;
        unit = blockIdx.x / per;
        const int r = static_cast<int>(blockIdx.x % per);
        role = P == 0 && r == 0 ? kRoleSum0 : r < nP ? kRoleSumT : kRoleSumZ;
        seg = r < nP ? r : r - nP + (P == 0 ? 1 : 0);
    } else if (mode == 5) {  // context parallel pass C on rank P
        nP = static_cast<int>(L.seg_slots);
        unit = blockIdx.x / nP;
        seg = static_cast<int>(blockIdx.x % nP);
    } else if (mode == 6) {  // context parallel rank summary (rank 0: the state at the end of its range)
        nP = static_cast<int>(L.seg_slots);
        if (P == 0) {
            unit = blockIdx.x;
            role = kRoleSum0;
        } else {
            unit = blockIdx.x / 2;
            role = (blockIdx.x & 1) ? kRoleSumZ : kRoleSumT;
        }
    } else {
        nP = P;
        const int per = 2 * P - 3;
        unit = blockIdx.x / per;
        const int r = static_cast<int>(blockIdx.x % per);
        if (r == 0) {
            role = kRoleSum0;
        } else if (r <= P - 2) {
            seg = r;
            role = kRoleSumT;
        } else {
            seg = r - (P - 2);
            role = kRoleSumZ;
        }
    }
    const int64_t s = unit / p.hv;
    const int h = static_cast<int>(unit - s * p.hv);

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    const int len_all = static_cast<int>(t1 - t0);
    const int nch_all = (len_all + kC - 1) / kC;
    const int rec0_all = reinterpret_cast<const int*>(ws + L.off_base)[s];
    float* ns_head = p.new_state + unit * kD * kD;
    const bool cp = mode >= 4;  // context parallel: every rank holds >= 1 chunk of every sequence
    if (nch_all == 0 || rec0_all + nch_all > L.R) {
        if (cp && tid == 0) record_status(16);
        if (role == kRoleMain && seg == 0) {
            if (nch_all != 0 && tid == 0) record_status(16);
            // empty sequence: zero state (oracle prefill :53-55)
            for (int i = tid; i < kD * kD / 4; i += kCarryThreads)
                reinterpret_cast<float4*>(ns_head)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    const bool ranksum = mode == 6;  // composes the rank's segment summaries; no chunks
    const int Lseg = (nch_all + nP - 1) / nP;
    const int cb = ranksum ? 0 : seg * Lseg < nch_all ? seg * Lseg : nch_all;
    const int ce = ranksum ? 0 : cb + Lseg < nch_all ? cb + Lseg : nch_all;
    // a summary nobody composes: one reaching the end of the sequence (context
    // parallel: the end of the last rank's range)
    if (!ranksum && role != kRoleMain && ce >= nch_all && (!cp || P + 1 == L.cp_world)) return;
    const bool last = !ranksum && ce == nch_all, outputs = role == kRoleMain;
    const bool dpart = !ranksum && role != kRoleSumT;
    const int nch = ce - cb, rec0 = rec0_all + cb;
    t0 += static_cast<int64_t>(kC) * cb;
    const int len = len_all - kC * cb < kC * nch ? len_all - kC * cb : kC * nch;
    auto rec_ptr = [&](int c) { return ws + L.off_rec + (static_cast<int64_t>(rec0 + c) * p.hv + h) * kHeadRecBytes; };
    // summaries (T at +0, Z at +32 KiB): per unit and segment; context
    // parallel: the rank's own segments, and one all-gathered slot per rank
    const int64_t units = p.num_seqs * p.hv;
    auto slot = [&](int sg) {
        return ws + L.off_seg + (cp ? sg * units + unit : unit * L.seg_slots + sg) * static_cast<int64_t>(kSegSlotBytes);
    };
    auto gslot = [&](int r) { return ws + L.off_gather + (r * units + unit) * static_cast<int64_t>(kSegSlotBytes); };
    auto sum_base_fn = [&]() { return ranksum || (cp && nP == 1) ? gslot(P) : slot(role == kRoleSum0 ? 0 : seg); };
    const int qw = warp & 3, hk = warp >> 2;  // state warps: sub-partition, k half
    const int vrow = 32 * qw + lane;
    // this CTA's summary from a state warp's registers: row vrow, k = 64 hk + 32 half + (0 .. 31)
    auto put_half = [&](int half, const float* x) {
        uint8_t* const sum_base = sum_base_fn();
        if (role == kRoleSumT) {  // T as the f16 MN-major image [128 j][128 k]
#pragma unroll
            for (int e = 0; e < 4; ++e)
                *reinterpret_cast<uint4*>(sum_base + h16(vrow, 64 * hk + 32 * half + 8 * e, kD)) = f16x8(x + 8 * e);
        } else if (role == kRoleSumZ) {  // Z as f16 rows
#pragma unroll
            for (int e = 0; e < 4; ++e)
                *reinterpret_cast<uint4*>(sum_base + 32768 + zh_off(vrow, 8 * hk + 4 * half + e)) = f16x8(x + 8 * e);
        } else {  // a state (Sum0; a rank's end state): fp32 rows
#pragma unroll
            for (int e = 0; e < 8; ++e)
                *reinterpret_cast<float4*>(sum_base + 32768 + zrow_off(vrow, 16 * hk + 8 * half + e)) =
                    make_float4(x[4 * e], x[4 * e + 1], x[4 * e + 2], x[4 * e + 3]);
        }
    };
    if (!ranksum && cb >= ce) {  // an empty segment of a short sequence
        if (role != kRoleMain && warp < 8) {  // context parallel, composed by later ranks: T = I, Z = 0
            float a0[32], a1[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                a0[e] = role == kRoleSumT && 64 * hk + e == vrow ? 1.f : 0.f;
                a1[e] = role == kRoleSumT && 64 * hk + 32 + e == vrow ? 1.f : 0.f;
            }
            put_half(0, a0);
            put_half(1, a1);
        }
        return;
    }

    const bool issuer = tid == 12 * 32, loader = tid == 13 * 32;
    int topM = -1, topKU = -1;  // loader: highest chunk whose copy was issued
    auto issue_M = [&](int c) {  // M and Qt^T are adjacent in the record: [M | Qt^T]
        const int b = c & 1;
        const uint32_t bytes = outputs ? kCaMQBytes : 32768;
        mbar_expect_tx(fullM(b), bytes);
        bulk_g2s(aM + b * kCaMQBytes, rec_ptr(c) + kRecM, bytes, fullM(b));
        topM = c;
    };
    auto issue_KU = [&](int c) {  // K' and U^T are adjacent in the record
        const int b = c % 3;
        mbar_expect_tx(fullKU(b), 32768);
        bulk_g2s(aKU + b * 32768, rec_ptr(c) + kRecKb, 32768, fullKU(b));
        topKU = c;
    };
    if (issuer) {
        for (int b = 0; b < 2; ++b) mbar_init(fullM(b), 1);
        for (int b = 0; b < 3; ++b) mbar_init(fullKU(b), 1);
        mbar_init(mmaS(0), 1);
        mbar_init(mmaS(1), 1);
        mbar_init(imgReady, 8);
        for (int b = 0; b < 2; ++b) mbar_init(oFree(b), 4);
        mbar_init(drain, 1);
        for (int b = 0; b < 3; ++b) mbar_init(proLoad(b), 1);
        mbar_init(proMma, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kCaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();  // the operand images / segment summaries of the preceding kernel are complete
    const uint32_t tm = *tmem_slot;
    auto accS = [&](int b) { return tm + 192 * b; };
    auto accO = [&](int b) { return tm + 192 * b + 128; };
    auto sA = [&](int b) { return tm + 384 + 64 * b; };
    if (outputs && warp >= 8 && warp < 12) {
        // the output columns start cleared: each chunk's product accumulates S Qt^T
        // onto them, and the output warps clear them again once read
        const uint32_t z[32] = {};
        for (int b = 0; b < 2; ++b)
            for (int half = 0; half < 2; ++half) tmem_st32(taddr(accO(b), 32 * (warp - 8), 32 * half), z);
        tmem_wait_st();
        tc_fence_before();
    }

    // The chain's start, and the summaries composed onto it before any chunk:
    // segmented pass C starts at segment 1 (Sum0's state) and composes
    // segments 1 .. seg-1; context parallel, rank P >= 1 starts at rank 0's
    // end state and composes ranks 1 .. P-1, then its own segments
    // 0 .. seg-1; a rank summary composes the rank's segments (rank 0: onto
    // Sum0's state).
    const bool cp_tail = cp && role == kRoleMain && P > 0;
    const uint8_t* init_rows = nullptr;  // a state as fp32 rows (else p.state, I or 0)
    if (cp_tail)
        init_rows = gslot(0) + 32768;
    else if ((role == kRoleMain && seg > 0) || (ranksum && role == kRoleSum0))
        init_rows = slot(0) + 32768;
    const int ncomp = cp_tail ? P - 1 + seg
                      : role == kRoleMain ? (seg > 0 ? seg - 1 : 0)
                      : ranksum ? (role == kRoleSum0 ? nP - 1 : nP)
                                : 0;
    const bool addZ = role != kRoleSumT;  // a T chain only multiplies
    auto comp_slot = [&](int i) {
        if (cp_tail) return i < P - 1 ? gslot(i + 1) : slot(i - (P - 1));
        return ranksum && role != kRoleSum0 ? slot(i) : slot(i + 1);
    };
    // initial state -> fp16 A operand 0 (state warps)
    if (warp < 8) {
        uint32_t w[32];
        if (init_rows != nullptr) {
            const uint8_t* x1 = init_rows;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float4 x = *reinterpret_cast<const float4*>(x1 + zrow_off(vrow, 16 * hk + e));
                w[2 * e] = pack_half2(x.x, x.y);
                w[2 * e + 1] = pack_half2(x.z, x.w);
            }
        } else if (role == kRoleSumT || role == kRoleSumZ) {  // I (T) or 0 (Z)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const int k = 64 * hk + 2 * e;
                const float one = role == kRoleSumT ? 1.f : 0.f;
                w[e] = pack_half2(k == vrow ? one : 0.f, k + 1 == vrow ? one : 0.f);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float4 x = p.state != nullptr
                                     ? reinterpret_cast<const float4*>(p.state + unit * kD * kD + vrow * kD + 64 * hk)[e]
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                w[2 * e] = pack_half2(x.x, x.y);
                w[2 * e + 1] = pack_half2(x.z, x.w);
            }
        }
        tmem_st32(taddr(sA(0), 32 * qw, 32 * hk), w);
        tmem_wait_st();
        tc_fence_before();
    }
    __syncthreads();
    // composition: S <- S T_i + Z_i for i < ncomp (in place in A operand 0).
    // T_i (f16 MN-major [128 j][128 k]) and Z_i (f16 rows) go to 32 KiB
    // buffers i % 3 over the chunk operand space (T at 0 / 32 / 64 KiB, Z at
    // 96 / 128 / 160 KiB), loaded two steps ahead.  A rank summary stores its
    // last step's fp32 result.
    bool ok = true;
    auto aT = [&](int b) { return aM + b * 32768; };
    auto aZ = [&](int b) { return aM + 98304 + b * 32768; };
    auto issue_TZ = [&](int i) {
        const int b = i % 3;
        const uint8_t* src = comp_slot(i);
        mbar_expect_tx(proLoad(b), addZ ? 65536 : 32768);
        bulk_g2s(aT(b), src, 32768, proLoad(b));
        if (addZ) bulk_g2s(aZ(b), src + 32768, 32768, proLoad(b));
    };
    if (loader)
        for (int i = 0; i < ncomp && i < 3; ++i) issue_TZ(i);
    for (int j = 0; j < ncomp; ++j) {
        const int b = j % 3;
        const uint32_t ldbar = proLoad(b), ldpar = (j / 3) & 1;
        if (issuer) {
            ok = mbar_wait(ldbar, ldpar) && ok;
            tc_fence_after();
            mma_ct_ta<kF16, true, kD, kD, kD>(accS(0), sA(0), aT(b), false);
            mma_commit(proMma);
        }
        if (warp < 8) {
            // Z_j arrived by TMA (observe its barrier) and S_j T_j is complete
            const bool okj =
                __all_sync(0xffffffffu, mbar_wait(ldbar, ldpar) && mbar_wait(proMma, j & 1));
            tc_fence_after();
            uint32_t w[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float a[32];
                tmem_ld32(taddr(accS(0), 32 * qw, 64 * hk + 32 * half), a);
                tmem_wait_ld();
                if (addZ) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float z[8];
                        h16x8_to_f32(Sm.ld16(aZ(b) + zh_off(vrow, 8 * hk + 4 * half + e)), z);
#pragma unroll
                        for (int i = 0; i < 8; ++i) a[8 * e + i] += z[i];
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    w[16 * half + 2 * e] = pack_half2(a[4 * e], a[4 * e + 1]);
                    w[16 * half + 2 * e + 1] = pack_half2(a[4 * e + 2], a[4 * e + 3]);
                }
                if (ranksum && j + 1 == ncomp && okj) put_half(half, a);
            }
            tmem_st32(taddr(sA(0), 32 * qw, 32 * hk), w);
            tmem_wait_st();
            tc_fence_before();
            ok = ok && okj;
        }
        __syncthreads();
        tc_fence_after();
        if (loader && j + 3 < ncomp) issue_TZ(j + 3);  // into the buffers step j just released
    }
    if (loader) {  // first copies of the segment's chunks
        for (int c = 0; c < 2 && c < nch; ++c) issue_M(c);
        if (dpart)
            for (int c = 0; c < 3 && c < nch; ++c) issue_KU(c);
        if (outputs)  // Ut^T is read by the output warps straight from global memory
            for (int c = 0; c < 2 && c < nch; ++c) bulk_prefetch_l2(rec_ptr(c) + kRecUt, 16384);
    }

    if (warp < 8) {
        if (lane == 0) mbar_arrive(imgReady);  // image 0 (phase 0)
        for (int c = 0; c < nch; ++c) {
            const bool okc = __all_sync(0xffffffffu, mbar_wait(mmaS(c), (c >> 1) & 1));  // warp-uniform exit
            tc_fence_after();
            float a0[32], a1[32];
            tmem_ld32(taddr(accS(c & 1), 32 * qw, 64 * hk), a0);
            tmem_ld32(taddr(accS(c & 1), 32 * qw, 64 * hk + 32), a1);
            tmem_wait_ld();
            if (!okc) {
                if (lane == 0) record_status(32);
                break;
            }
            if (c + 1 < nch) {
                uint32_t w[32];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    w[e] = pack_half2(a0[2 * e], a0[2 * e + 1]);
                    w[16 + e] = pack_half2(a1[2 * e], a1[2 * e + 1]);
                }
                tmem_st32(taddr(sA((c + 1) & 1), 32 * qw, 32 * hk), w);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(imgReady);
            } else if (role == kRoleMain) {
                if (last) {
                    float* ns_row = ns_head + vrow * kD + 64 * hk;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        reinterpret_cast<float4*>(ns_row)[e] =
                            make_float4(a0[4 * e], a0[4 * e + 1], a0[4 * e + 2], a0[4 * e + 3]);
                        reinterpret_cast<float4*>(ns_row + 32)[e] =
                            make_float4(a1[4 * e], a1[4 * e + 1], a1[4 * e + 2], a1[4 * e + 3]);
                    }
                }
            } else {
                put_half(0, a0);
                put_half(1, a1);
            }
        }
    } else if (warp < 12) {
        // output epilogue: lane v, columns = the chunk's 64 tokens.  A full
        // chunk is staged as the bf16 tile [64 i][128 v] (two SW128 images)
        // and written by two tiled TMA stores; the last, partial chunk of a
        // sequence is stored element by element (a tile would spill into the
        // next sequence's rows).
        const int q = warp - 8;
        const int v = 32 * q + lane;
        const bool lead = tid == 8 * 32;  // issues the tile stores
        const uint32_t aOut = smem_u32(sm + kCaOut);
        const uint32_t ov = aOut + (v >> 6) * 8192 + (v & 7) * 2;
        const int och = (v & 63) >> 3;
        uint4 ut[8];  // Ut^T row v of the chunk: logical 16-byte chunk e (tokens 8e..8e+7) stored at e ^ (v & 7)
        auto load_ut = [&](int c) {
            const uint8_t* urow = rec_ptr(c) + kRecUt + v * 128;
#pragma unroll
            for (int e = 0; e < 8; ++e) ut[e] = __ldg(reinterpret_cast<const uint4*>(urow + ((e ^ (v & 7)) << 4)));
        };
        if (outputs && nch > 0) load_ut(0);
        for (int c = 0; outputs && c < nch; ++c) {
            const int rows = len - kC * c < kC ? len - kC * c : kC;
            // one verdict for the four warps (they meet at named barriers below)
            const bool okc = named_sync_and(1, 128, mbar_wait(mmaS(c), (c >> 1) & 1));
            tc_fence_after();
            if (!okc) {
                if (lane == 0) record_status(32);
                break;
            }
            // scale (O + Ut) as bf16 pairs pk[j] = tokens (2j, 2j + 1), one TMEM half at a time
            uint32_t pk[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float o[32];
                tmem_ld32(taddr(accO(c & 1), 32 * q, 32 * half), o);
                tmem_wait_ld();
                if (half == 1) {  // read: clear the columns for chunk c + 2 and release them before the stores
                    const uint32_t z[32] = {};
                    tmem_st32(taddr(accO(c & 1), 32 * q, 0), z);
                    tmem_st32(taddr(accO(c & 1), 32 * q, 32), z);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(oFree(c & 1));
                }
#pragma unroll
                for (int i0 = 0; i0 < 32; i0 += 8) {
                    float u[8];
                    h16x8_to_f32(ut[(32 * half + i0) >> 3], u);
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(p.scale * (o[i0 + e] + u[e]),
                                                                        p.scale * (o[i0 + e + 1] + u[e + 1]));
                        pk[(32 * half + i0 + e) >> 1] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                }
            }
            if (c + 1 < nch) load_ut(c + 1);  // in flight during this chunk's stores
            if (rows == kC) {
                if (lead) bulk_wait_read<0>();  // the previous tile has left the staging buffer
                named_sync(1, 128);
#pragma unroll
                for (int i = 0; i < kC; ++i)
                    st_shared_u16(ov + i * 128 + ((och ^ (i & 7)) << 4),
                                  static_cast<uint16_t>((i & 1) ? pk[i >> 1] >> 16 : pk[i >> 1] & 0xffffu));
                fence_async_smem();
                named_sync(1, 128);
                if (lead) {
                    const int tok = static_cast<int>(t0) + kC * c;
                    tma_store_3d(&tmO, aOut, 0, h, tok);
                    tma_store_3d(&tmO, aOut + 8192, 64, h, tok);
                    bulk_commit();
                }
            } else {
                uint16_t* dst = p.out + ((t0 + static_cast<int64_t>(kC) * c) * p.hv + h) * kD + v;
#pragma unroll
                for (int i = 0; i < kC; ++i)
                    if (i < rows)
                        dst[static_cast<int64_t>(i) * (p.hv * kD)] =
                            static_cast<uint16_t>((i & 1) ? pk[i >> 1] >> 16 : pk[i >> 1] & 0xffffu);
            }
        }
        if (lead) bulk_wait_read<0>();  // the last tile has left shared memory (its writes complete with the grid)
    } else if (issuer) {
        if (dpart) {
            ok = mbar_wait(fullKU(0), 0) && ok;
            tc_fence_after();
            // U_0^T K'_0 -> accS 0 (A = U^T K-major [128 v][64 j], B = K' MN-major [64 j][128 k])
            mma_ct<kF16, false, true, 64, 128, 64, 128, 128>(accS(0), aKU + 16384, aKU, false);
        }
        for (int c = 0; c < nch && ok; ++c) {
            // the output columns of this parity were read and cleared for chunk c - 2
            ok = mbar_wait(imgReady, c & 1) && mbar_wait(fullM(c & 1), (c >> 1) & 1) &&
                 (!outputs || c < 2 || mbar_wait(oFree(c & 1), ((c - 2) >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            const uint32_t bMQ = aM + (c & 1) * kCaMQBytes;
            if (outputs)  // S_c [M_c^T | Qt_c^T] (N = 192): the next state onto U_c^T K'_c, O_c^T onto zeros
                mma_ct_ta<kF16, true, kD, 128, 192>(accS(c & 1), sA(c & 1), bMQ, true);
            else  // S_c M_c^T (onto U_c^T K'_c, or alone for a T chain)
                mma_ct_ta<kF16, true, kD, 128, 128>(accS(c & 1), sA(c & 1), bMQ, dpart);
            mma_commit(mmaS(c));
            if (dpart && c + 1 < nch) {  // next chunk's U^T K' into the other accumulator (its reader is done)
                const int b = (c + 1) % 3;
                ok = mbar_wait(fullKU(b), ((c + 1) / 3) & 1);
                if (!ok) break;
                mma_ct<kF16, false, true, 64, 128, 64, 128, 128>(accS((c + 1) & 1), aKU + b * 32768 + 16384,
                                                                aKU + b * 32768, false);
            }
        }
        if (!ok) {
            record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
            mma_commit(drain);  // wait (bounded) for the MMAs in flight
            mbar_wait(drain, 0);
        }
    } else if (loader) {
        // chunk c's product complete => so is everything issued before it (U^T K'
        // of c): refill those buffers two (three) chunks ahead
        for (int c = 0; c < nch && ok; ++c) {
            ok = mbar_wait(mmaS(c), (c >> 1) & 1);
            if (!ok) break;
            if (c + 2 < nch) {
                issue_M(c + 2);
                if (outputs) bulk_prefetch_l2(rec_ptr(c + 2) + kRecUt, 16384);
            }
            if (dpart && c + 3 < nch) issue_KU(c + 3);
        }
        if (!ok) {
            record_status(32 /* GDN_ERR_DEVICE_TIMEOUT */);
            // wait (bounded) for the copies in flight: per buffer, its latest chunk
            for (int c = topM > 1 ? topM - 1 : 0; c <= topM; ++c) mbar_wait(fullM(c & 1), (c >> 1) & 1);
            for (int c = topKU > 2 ? topKU - 2 : 0; c <= topKU; ++c) mbar_wait(fullKU(c % 3), (c / 3) & 1);
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

// Path selection: 0 = auto, 1 = token-recurrent, 2 = chunked tensor-core, 3 = chunked
// with the segmented carry forced (P = 4, or the workspace's slots if fewer; needs
// the summary space, N <= 4).
constexpr int kPathAuto = 0, kPathRecurrent = 1, kPathChunked = 2, kPathSegmented = 3;
// Mean sequence length up to which the token recurrence beats the chunked path
// (measured on B200 with 32 and 256 equal sequences: recurrent faster at 16
// tokens, chunked at 32).
constexpr int64_t kRecurrentMaxAvgLen = 24;


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

// The chunk table and the operand records (table + prepare kernels); leaves
// the output tensor map and the SM count for the carry.
static cudaError_t chunk_records(const PrefillParams& p, uint8_t* ws, const WsLayout& L, CUtensorMap* tmO,
                                 int* sms_out, cudaStream_t stream) {
    if (L.R * p.hv > 0x7fffffffLL || p.total_tokens > 0x7fffffffLL) return cudaErrorInvalidValue;
    CUtensorMap tmK, tmQ, tmV;
    memset(&tmK, 0, sizeof(tmK));
    memset(&tmQ, 0, sizeof(tmQ));
    memset(&tmV, 0, sizeof(tmV));
    memset(tmO, 0, sizeof(*tmO));
    cudaError_t e;
    if (p.total_tokens > 0) {  // with no tokens there are no records and no loads
        if ((e = token_tensor_map(&tmK, p.k, p.hqk, p.total_tokens)) != cudaSuccess) return e;
        if ((e = token_tensor_map(&tmQ, p.q, p.hqk, p.total_tokens)) != cudaSuccess) return e;
        if ((e = token_tensor_map(&tmV, p.v, p.hv, p.total_tokens)) != cudaSuccess) return e;
        if ((e = token_tensor_map(tmO, p.out, p.hv, p.total_tokens)) != cudaSuccess) return e;
    }
    gdn_chunk_table_kernel<<<device_sm_count(), 1024, 0, stream>>>(p, ws, L);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_prepare_kernel, kPrSmem)) != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    *sms_out = sms;
    // persistent prepare: two CTAs per SM (or one per item when there are fewer)
    const int64_t items = L.R * p.hv;
    if ((e = launch_dependent(gdn_chunk_prepare_kernel, static_cast<unsigned>(items < 2 * sms ? items : 2 * sms),
                              kPrepThreads, kPrSmem, stream, p, ws, L, tmK, tmQ, tmV)) != cudaSuccess)
        return e;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return set_smem(gdn_chunk_carry_kernel, kCaSmem);
}

cudaError_t launch_prefill_chunked(const PrefillParams& p, void* workspace, size_t workspace_bytes, int path,
                                   cudaStream_t stream) {
    const WsLayout L = ws_layout(p.total_tokens, p.num_seqs, p.hv);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    CUtensorMap tmO;
    int sms = 148;
    cudaError_t e;
    if ((e = chunk_records(p, ws, L, &tmO, &sms, stream)) != cudaSuccess) return e;
    const int64_t units = p.num_seqs * p.hv;
    if (units > 0x7fffffffLL / (2 * kSegMaxP)) return cudaErrorInvalidValue;
    // Segmented carry: when sequences average 16 chunks or more and both
    // passes fit one wave with P >= 2 segments per chain (or when asked for:
    // P = 4 where the workspace has the slots), split each sequence into P
    // segments (pass A, then pass C).
    int P = 1;
    if (L.off_seg > 0 && workspace_bytes >= static_cast<size_t>(L.total_seg)) {
        const int fit = seg_segments(p.num_seqs, sms, p.hv);
        if (path == kPathSegmented)
            P = L.seg_slots < 4 ? static_cast<int>(L.seg_slots) : 4;
        else if (p.total_tokens >= p.num_seqs * 16 * kC)
            P = fit < L.seg_slots ? fit : static_cast<int>(L.seg_slots);
    }
    if (P >= 2) {
        if ((e = launch_dependent(gdn_chunk_carry_kernel, static_cast<unsigned>(units * (2 * P - 3)), kCarryThreads,
                                  kCaSmem, stream, p, ws, L, 1, P, tmO)) != cudaSuccess)
            return e;
        return launch_dependent(gdn_chunk_carry_kernel, static_cast<unsigned>(units * P), kCarryThreads, kCaSmem,
                                stream, p, ws, L, 2, P, tmO);
    }
    return launch_dependent(gdn_chunk_carry_kernel, static_cast<unsigned>(units), kCarryThreads, kCaSmem, stream, p,
                            ws, L, 0, 1, tmO);
}

// Context parallelism: every sequence's tokens are split over `world` ranks in
// consecutive ranges (every range at least one token; the composition is
// exact for any split, whole chunks only keep the chunks full); rank r holds
// range r of every sequence, cut into up to 8 segments.  Phase 0 on every
// rank builds its records, its segments' summaries (pass A) and their
// composition, the rank's carry summary (rank 0: the state at the end of its
// range; rank r >= 1: the affine map (T_r, Z_r) of its range), written at
// rank r's block of the summary region.  The caller then all-gathers that
// region (world blocks of num_seqs x 8 x 96 KiB); phase 1 (pass C) runs every
// segment with outputs from the composition of what precedes it (new_state:
// the state after the rank's range).
//
// Segments per rank for the context-parallel carry: up to 8, with a rank's
// pass A (2 CTAs per segment and unit) in one wave.  A function of N only,
// so that every rank lays out the same slots.
static int cp_segments(int64_t N) {
    const int64_t units = N * kHV;
    int q = 8;
    while (q > 1 && 2 * units * q > kSmCount) --q;
    return q;
}

// Context-parallel workspace: the single-GPU records, then the all-gathered
// rank summaries (world x N x 8 slots, at an offset that depends on the local
// token count and N only), then the rank's own segment summaries.
WsLayout cp_layout(int64_t T, int64_t N, int world) {
    WsLayout L = ws_layout(T, N);
    L.cp_world = world;
    L.seg_slots = cp_segments(N);
    L.off_gather = L.total;
    L.off_seg = L.off_gather + static_cast<int64_t>(world) * N * kHV * kSegSlotBytes;
    L.total_seg = L.off_seg + L.seg_slots * N * kHV * kSegSlotBytes;
    return L;
}

cudaError_t launch_prefill_cp(const PrefillParams& p, void* workspace, size_t workspace_bytes, int rank, int world,
                              int phase, cudaStream_t stream) {
    const WsLayout L = cp_layout(p.total_tokens, p.num_seqs, world);
    if (workspace_bytes < static_cast<size_t>(L.total_seg)) return cudaErrorInvalidValue;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int64_t units = p.num_seqs * p.hv, q = L.seg_slots;
    if (units == 0 || units > 0x7fffffffLL / (2 * q)) return units == 0 ? cudaSuccess : cudaErrorInvalidValue;
    CUtensorMap tmO;
    cudaError_t e;
    if (phase == 0) {  // records; pass A: Sum0 (rank 0), T and Z of the rank's segments; the rank summary
        int sms = 148;
        if ((e = chunk_records(p, ws, L, &tmO, &sms, stream)) != cudaSuccess) return e;
        if ((e = launch_dependent(gdn_chunk_carry_kernel,
                                  static_cast<unsigned>(units * (rank == 0 ? 2 * q - 1 : 2 * q)), kCarryThreads,
                                  kCaSmem, stream, p, ws, L, 4, rank, tmO)) != cudaSuccess)
            return e;
        // with one segment pass A wrote the rank summary itself; the last rank's is never read
        if (q == 1 || rank + 1 == world) return cudaSuccess;
        return launch_dependent(gdn_chunk_carry_kernel, static_cast<unsigned>(rank == 0 ? units : 2 * units),
                                kCarryThreads, kCaSmem, stream, p, ws, L, 6, rank, tmO);
    }
    // pass C over the rank's segments, with outputs
    memset(&tmO, 0, sizeof(tmO));
    if (p.total_tokens > 0 && (e = token_tensor_map(&tmO, p.out, p.hv, p.total_tokens)) != cudaSuccess) return e;
    if ((e = set_smem(gdn_chunk_carry_kernel, kCaSmem)) != cudaSuccess) return e;
    gdn_chunk_carry_kernel<<<static_cast<unsigned>(units * q), kCarryThreads, kCaSmem, stream>>>(p, ws, L, 5, rank,
                                                                                                 tmO);
    return cudaGetLastError();
}

// True when `path` resolves to the token-recurrent kernel for this problem
// (which needs no workspace): asked for, or AUTO with a short mean length.
bool prefill_path_is_recurrent(int path, int64_t total_tokens, int64_t num_seqs) {
    const int64_t avg = total_tokens / (num_seqs > 0 ? num_seqs : 1);
    return path == kPathRecurrent || (path == kPathAuto && avg <= kRecurrentMaxAvgLen);
}

cudaError_t launch_prefill(const PrefillParams& p, int path, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
    if (prefill_path_is_recurrent(path, p.total_tokens, p.num_seqs)) {
        cudaError_t e = launch_prefill_zero_uncovered(p, stream);
        return e != cudaSuccess ? e : launch_prefill_recurrent(p, stream);
    }
    if (workspace == nullptr || workspace_bytes < chunked_workspace_min_bytes(p.total_tokens, p.num_seqs, p.hv))
        return cudaErrorInvalidValue;
    return launch_prefill_chunked(p, workspace, workspace_bytes, path, stream);
}

// ------------------------------------------------------------- self-test --
// D[M x N] = A[M x K] . B[N x K]^T through the same image writers,
// descriptors and TMEM read-back as the kernels above (one CTA).  flags:
// bit 0 A MN-major, bit 1 B MN-major, bit 2 accumulator at TMEM lane 16
// (the second M=64 tile of a lane-packed pair; M = 64 only), bit 3 A read
// from TMEM (16-bit kinds, M = 128, K-major).
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
    const bool a_mn = flags & 1, b_mn = flags & 2, lane16 = flags & 4, a_tmem = flags & 8;
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
    if (a_tmem) ncols = 512;  // D at column 0, A from column 256
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
    if (a_tmem) {
        // A (16-bit, M = 128) into TMEM: row m = lane m, k pairs packed low-first
        const uint16_t* arow = static_cast<const uint16_t*>(A) + tid * K;
        for (int c0 = 0; c0 < K / 2; c0 += 32) {
            uint32_t w[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
                w[i] = static_cast<uint32_t>(arow[2 * (c0 + i)]) | (static_cast<uint32_t>(arow[2 * (c0 + i) + 1]) << 16);
            tmem_st32(taddr(tm, 32 * warp, 256 + c0), w);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (flags & 16) {
        // diagnostic: nothing is issued and nothing signals `bar`, so the
        // bounded wait below expires and the kernel unwinds (status bit, TMEM freed)
    } else if (tid == 0 && a_tmem) {
        const uint32_t id = idesc(kind == kBF16 ? kBF16 : kF16, 128, N, false, b_mn);
        const uint32_t b = smem_u32(sB);
        for (int s = 0; s < K / 16; ++s) {
            const uint64_t bd = b_mn ? sw128_desc_mn(b + s * 16 * 128, K * 128)
                                     : sw128_desc(b + ((s * 32) >> 7) * N * 128 + ((s * 32) & 127));
            mma_f16_ta(d, tm + 256 + 8 * s, bd, id, s > 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(bar));
    } else if (tid == 0) {
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
