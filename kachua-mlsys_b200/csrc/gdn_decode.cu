// gdn_decode.cu -- single-token GDN decode, streaming the fp32 k-last state.
//
// Math per (sequence b, v-head h), state S = [V=128][K=128] (k-last), as the
// reference oracle (decode reference_torch_impl.py:52-69) and the reference
// CUDA kernel (kernel.cu:551-835, steps listed at kernel.cu:579-744):
//   g = exp(-exp(A_log) softplus(a + dt_bias)),  beta = sigmoid(b)
//   kS_v  = k . S[v,:]             qS_v = q . S[v,:]
//   delta = beta (v_v - g kS_v)
//   S'[v,:] = g S[v,:] + delta k
//   o_v   = scale (g qS_v + delta (q . k))   ( = scale q . S'[v,:] )
// q/k head = h / 2 (grouped values).
//
// The step is a pure HBM stream (0.5 FLOP/byte): 64 KiB of state read and
// written per head.  Layout of the work:
//   * 8 lanes own one state row; lane `sub` holds floats 4*sub + 32*j
//     (j = 0..3) -- every float4 load/store instruction of the 8 lanes covers
//     128 contiguous bytes, a warp covers 4 rows per pass;
//   * a CTA is WARPS warps x RPW rows per warp (fp32 state: 4 rows, 2 or 4
//     warps; the choice is measured, see pick_decode_shape); every load of a
//     thread's rows is issued before any arithmetic, so a thread keeps
//     16 * RPW bytes in flight;
//   * both dot products reduce with 3 xor-shuffles inside the 8-lane group;
//   * the new state is written once with streaming (evict-first) stores.
// Each thread reads all of its state elements before writing any of them and
// no other thread touches them, so state == new_state (in place) is safe.
#include <type_traits>
#include "gdn_common.cuh"

namespace gdn {

struct DecodeParams {
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    const float* state;
    const float* A_log;
    const uint16_t* a;
    const float* dt_bias;
    const uint16_t* b;
    uint16_t* out;
    float* new_state;
    int64_t batch;
    float scale;
    int hqk, hv;  // q/k and v heads (4 / 8 in the reference; hv a multiple of hqk)
};

// BF16S: the state (in and out) is stored as bf16 instead of fp32; the
// arithmetic is the same fp32, the new state rounded to bf16 once.
template <int RPW, bool BF16S, int WARPS = 4>
__global__ void __launch_bounds__(32 * WARPS) gdn_decode_kernel(const DecodeParams p) {
    static_assert(RPW % 4 == 0, "rows per warp must be a multiple of 4");
    constexpr int kPasses = RPW / 4;
    constexpr int kRowsPerCta = WARPS * RPW;
    constexpr int kTiles = kD / kRowsPerCta;

    // Launched as a programmatic dependent of the previous kernel in the
    // stream (back-to-back decode steps: this step's state is the previous
    // step's output): the CTAs become resident while that kernel drains and
    // wait here, before any global access, until it has completed.
    griddep_launch_dependents();
    griddep_wait();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int grp = lane >> 3;  // row within a pass
    const int sub = lane & 7;   // position within the row

    const int64_t cta = blockIdx.x;
    const int64_t bh = cta / kTiles;  // b * 8 + h
    const int tile = static_cast<int>(cta - bh * kTiles);
    const int64_t bi = bh / p.hv;
    const int h = static_cast<int>(bh - bi * p.hv);
    const int hq = h / (p.hv / p.hqk);
    const int row0 = tile * kRowsPerCta + warp * RPW + grp;

    const float* src = p.state + bh * (kD * kD) + 4 * sub;
    float* dst = p.new_state + bh * (kD * kD) + 4 * sub;
    const uint16_t* src16 = reinterpret_cast<const uint16_t*>(p.state) + bh * (kD * kD) + 4 * sub;
    uint16_t* dst16 = reinterpret_cast<uint16_t*>(p.new_state) + bh * (kD * kD) + 4 * sub;

    // 1. issue every state load first (kPasses x 4 x 16 B per thread; 8 B with a
    // bf16 state, kept as raw bf16 words until its row is processed)
    using Raw = typename std::conditional<BF16S, uint2, float4>::type;
    Raw raw[kPasses][4];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if constexpr (BF16S)
                raw[ps][j] = ld_stream_u2(src16 + (row0 + 4 * ps) * kD + 32 * j);
            else
                raw[ps][j] = ld_stream_f4(src + (row0 + 4 * ps) * kD + 32 * j);
        }
    }

    // 2. per-head vectors and gates (small, L2/L1 resident)
    const uint16_t* qp = p.q + (bi * p.hqk + hq) * kD + 4 * sub;
    const uint16_t* kp = p.k + (bi * p.hqk + hq) * kD + 4 * sub;
    float4 q4[4], k4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q4[j] = bf16x4_to_float4(ld_u2(qp + 32 * j));
        k4[j] = bf16x4_to_float4(ld_u2(kp + 32 * j));
    }
    float vrow[kPasses];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps)
        vrow[ps] = bf16_bits_to_float(p.v[bh * kD + row0 + 4 * ps]);
    float g, beta;
    gdn_gates_fast(p.A_log[h], p.dt_bias[h], bf16_bits_to_float(p.a[bh]), bf16_bits_to_float(p.b[bh]), g,
                   beta);

    float qk = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        qk += q4[j].x * k4[j].x + q4[j].y * k4[j].y + q4[j].z * k4[j].z + q4[j].w * k4[j].w;
    qk += __shfl_xor_sync(0xffffffffu, qk, 1);
    qk += __shfl_xor_sync(0xffffffffu, qk, 2);
    qk += __shfl_xor_sync(0xffffffffu, qk, 4);

    // 3. per row: two dot products, the rank-1 update, the output
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
        float4 s[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if constexpr (BF16S)
                s[j] = bf16x4_to_float4(raw[ps][j]);
            else
                s[j] = raw[ps][j];
        }
        float ks = 0.f, qs = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ks += s[j].x * k4[j].x + s[j].y * k4[j].y + s[j].z * k4[j].z + s[j].w * k4[j].w;
            qs += s[j].x * q4[j].x + s[j].y * q4[j].y + s[j].z * q4[j].z + s[j].w * q4[j].w;
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            ks += __shfl_xor_sync(0xffffffffu, ks, off);
            qs += __shfl_xor_sync(0xffffffffu, qs, off);
        }
        const float delta = beta * (vrow[ps] - g * ks);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float4 o;
            o.x = fmaf(g, s[j].x, delta * k4[j].x);
            o.y = fmaf(g, s[j].y, delta * k4[j].y);
            o.z = fmaf(g, s[j].z, delta * k4[j].z);
            o.w = fmaf(g, s[j].w, delta * k4[j].w);
            if (BF16S)
                st_stream_u2(dst16 + (row0 + 4 * ps) * kD + 32 * j, float4_to_bf16x4(o));
            else
                st_stream_f4(dst + (row0 + 4 * ps) * kD + 32 * j, o);
        }
        if (sub == 0) {
            const float o = p.scale * fmaf(g, qs, delta * qk);
            reinterpret_cast<__nv_bfloat16*>(p.out)[bh * kD + row0 + 4 * ps] = __float2bfloat16_rn(o);
        }
    }
}

// Multi-token decode (T tokens per sequence in one call: speculative decoding,
// the decode definition's seq_len axis).  The decode kernel's layout and load
// order -- 8 lanes per row, every state load of a thread issued before any
// other work -- with the T updates applied to the rows in registers, so the
// state is read and written once per call; per token and row the math is the
// single-token step's.  Tokens are staged in shared memory kTokBlk at a time
// (q and k of the head as bf16, the CTA's v rows, the gates and q.k per
// token), their loads in flight together with the state's.
// q/k/v/a/b/out are [B, T, heads, ...].
//
// Measured at B = 256, per call with the L2 flushed (T = 2 / 4 / 8: 53 / 63 /
// 86 us, against 72 / 88 / 129 for the token-recurrent prefill kernel it
// replaces; back to back over rotating state buffers 45 / 53 / 77 us): the
// state stream alone takes ~41 us and each token adds ~5 us of fp32 FMA and
// shuffle work per SM that this load -> compute -> store order does not
// overlap with HBM.  The per-token dot products reduce by a transposed 8-lane
// reduction (12 shuffles per token and thread at 16 rows per warp instead of
// 24: 55 / 66 / 90 us before).  A persistent variant that double- (and 3- and
// 4-) buffered 16-32 KiB state tiles in shared memory with bulk async copies
// was slower at every T (T = 2 / 8: 64-82 / 114-143 us) and was not kept;
// so were 1- and 2-warp CTAs and 8 rows per warp (no faster at T = 2-4,
// slower at T = 8).
constexpr int kTokBlk = 16;

// One level of the transposed reduction over the lanes `bit` apart: a lane
// whose `bit` is set keeps the upper half of its CNT values and sends the
// lower half to its partner (and the other way round), adding what it
// receives; the first CNT / 2 entries then hold the kept half's partial sums.
template <int CNT, int N>
__device__ __forceinline__ void transpose_reduce_step(float (&v)[N], int sub, int bit) {
    const bool upper = (sub & bit) != 0;
#pragma unroll
    for (int e = 0; e < CNT / 2; ++e) {
        const float keep = upper ? v[CNT / 2 + e] : v[e];
        const float send = upper ? v[e] : v[CNT / 2 + e];
        v[e] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
}

template <int RPW>
__global__ void __launch_bounds__(128) gdn_decode_tokens_kernel(const DecodeParams p, int T) {
    static_assert(RPW % 4 == 0, "rows per warp must be a multiple of 4");
    constexpr int kPasses = RPW / 4;
    constexpr int kRowsPerCta = 4 * RPW;
    constexpr int kTiles = kD / kRowsPerCta;

    griddep_launch_dependents();  // as in gdn_decode_kernel
    griddep_wait();
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int grp = lane >> 3;
    const int sub = lane & 7;

    const int64_t cta = blockIdx.x;
    const int64_t bh = cta / kTiles;  // b * hv + h
    const int tile = static_cast<int>(cta - bh * kTiles);
    const int64_t bi = bh / p.hv;
    const int h = static_cast<int>(bh - bi * p.hv);
    const int hq = h / (p.hv / p.hqk);
    const int rbase = tile * kRowsPerCta;
    const int lrow0 = warp * RPW + grp;  // CTA-local row of pass 0
    const int row0 = rbase + lrow0;

    const float* src = p.state + bh * (kD * kD) + 4 * sub;
    float* dst = p.new_state + bh * (kD * kD) + 4 * sub;
    float4 st[kPasses][4];
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
        for (int j = 0; j < 4; ++j) st[ps][j] = ld_stream_f4(src + (row0 + 4 * ps) * kD + 32 * j);

    __shared__ uint2 s_q[kTokBlk][kD / 4], s_k[kTokBlk][kD / 4];  // 4 bf16 per uint2
    __shared__ uint16_t s_v[kTokBlk][kRowsPerCta];
    __shared__ float s_g[kTokBlk], s_b[kTokBlk], s_qk[kTokBlk];
    const float A_log = p.A_log[h], dt_bias = p.dt_bias[h];
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);

    for (int tb = 0; tb < T; tb += kTokBlk) {
        const int nb = T - tb < kTokBlk ? T - tb : kTokBlk;
        if (tb > 0) __syncthreads();  // the previous block is consumed
        // one warp per token: its q and k (32 x 4 dims) and their dot product
        for (int e = tid; e < nb * (kD / 4); e += 128) {
            const int i = e / (kD / 4), c = e % (kD / 4);
            const int64_t base = ((bi * T + tb + i) * p.hqk + hq) * (kD / 4) + c;
            const uint2 qu = reinterpret_cast<const uint2*>(p.q)[base], ku = reinterpret_cast<const uint2*>(p.k)[base];
            s_q[i][c] = qu;
            s_k[i][c] = ku;
            const float4 qf = bf16x4_to_float4(qu), kf = bf16x4_to_float4(ku);
            float d = qf.x * kf.x + qf.y * kf.y + qf.z * kf.z + qf.w * kf.w;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            if (c == 0) s_qk[i] = d;
        }
        for (int e = tid; e < nb * kRowsPerCta; e += 128) {
            const int i = e / kRowsPerCta, r = e % kRowsPerCta;
            s_v[i][r] = p.v[((bi * T + tb + i) * p.hv + h) * kD + rbase + r];
        }
        if (tid < nb) {
            const int64_t t = bi * T + tb + tid;
            float g, beta;
            gdn_gates(A_log, dt_bias, bf16_bits_to_float(p.a[t * p.hv + h]), bf16_bits_to_float(p.b[t * p.hv + h]), g,
                      beta);
            s_g[tid] = g;
            s_b[tid] = beta;
        }
        __syncthreads();
        for (int i = 0; i < nb; ++i) {
            float4 q4[4], k4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q4[j] = bf16x4_to_float4(s_q[i][sub + 8 * j]);
                k4[j] = bf16x4_to_float4(s_k[i][sub + 8 * j]);
            }
            const float g = s_g[i], beta = s_b[i], qk = s_qk[i];
            const int64_t orow = ((bi * T + tb + i) * p.hv + h) * kD + row0;
            // the 2 x kPasses partial dot products of this lane (k.S and q.S of each
            // of its rows), then a transposed reduction over the 8 lanes of the row
            // group: each xor level hands half of the remaining values to the
            // partner lane, so 2P values take 2P - 1 shuffles instead of 3 x 2P;
            // afterwards lane sub holds the total of value sub / (8 / 2P)
            constexpr int kVals = 2 * kPasses;
            float vals[kVals];
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                float ks = 0.f, qs = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 s = st[ps][j];
                    ks += s.x * k4[j].x + s.y * k4[j].y + s.z * k4[j].z + s.w * k4[j].w;
                    qs += s.x * q4[j].x + s.y * q4[j].y + s.z * q4[j].z + s.w * q4[j].w;
                }
                vals[ps] = ks;
                vals[kPasses + ps] = qs;
            }
            if constexpr (kVals == 8) {
                transpose_reduce_step<8>(vals, sub, 4);
                transpose_reduce_step<4>(vals, sub, 2);
                transpose_reduce_step<2>(vals, sub, 1);
            } else if constexpr (kVals == 4) {
                transpose_reduce_step<4>(vals, sub, 4);
                transpose_reduce_step<2>(vals, sub, 2);
                vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], 1);
            } else {
                transpose_reduce_step<2>(vals, sub, 4);
                vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], 2);
                vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], 1);
            }
            constexpr int kSpan = 8 / kVals;  // lanes holding each total
            const int vidx = sub / kSpan;
            const bool holds_ks = vidx < kPasses;
            const int own = holds_ks ? vidx : vidx - kPasses;  // the pass of the held total
            const float dl =
                holds_ks ? beta * (bf16_bits_to_float(s_v[i][lrow0 + 4 * own]) - g * vals[0]) : 0.f;
            const int gbase = lane & ~7;
            // the output row of a q.S holder needs its pass's delta
            const float dq = __shfl_sync(0xffffffffu, dl, gbase + own * kSpan);
            if (!holds_ks && sub % kSpan == 0)
                out[orow + 4 * own] = __float2bfloat16_rn(p.scale * fmaf(g, vals[0], dq * qk));
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                const float delta = __shfl_sync(0xffffffffu, dl, gbase + ps * kSpan);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    st[ps][j].x = fmaf(g, st[ps][j].x, delta * k4[j].x);
                    st[ps][j].y = fmaf(g, st[ps][j].y, delta * k4[j].y);
                    st[ps][j].z = fmaf(g, st[ps][j].z, delta * k4[j].z);
                    st[ps][j].w = fmaf(g, st[ps][j].w, delta * k4[j].w);
                }
            }
        }
    }
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps)
#pragma unroll
        for (int j = 0; j < 4; ++j) st_stream_f4(dst + (row0 + 4 * ps) * kD + 32 * j, st[ps][j]);
}

// A decode kernel launch: as a programmatic dependent of the previous kernel
// in the stream (pdl), or normally.
template <typename... Params, typename... Args>
static cudaError_t launch_decode_kernel(bool pdl, void (*kernel)(Params...), unsigned grid, unsigned block,
                                        cudaStream_t stream, Args... args) {
    if (pdl) return launch_dependent(kernel, grid, block, 0, stream, args...);
    kernel<<<grid, block, 0, stream>>>(static_cast<Params>(args)...);
    return cudaGetLastError();
}

// Programmatic dependent launch from 65 heads up (B >= 9 at 8 v-heads).  Back
// to back inside a CUDA graph (per step, normal launch / dependent launch):
// B = 16 3.46 / 3.40 us, B = 64 8.88 / 8.52, B = 256 41.18 / 40.70; issued
// one by one from the host, B = 256 43.1 / 41.1.  At B = 8 the dependent
// launch was slower in the graph (2.48 / 3.08 us), at B = 1 level.  Per call
// after an idle GPU it makes no difference.
static bool decode_pdl(int64_t heads) { return heads > 64; }

// Rows per warp of the multi-token kernel: 16 (the fastest at every T
// measured) while that still gives >= 2 CTAs per SM, else 8, else 4.
cudaError_t launch_decode_tokens(const DecodeParams& p, int T, cudaStream_t stream) {
    if (p.batch == 0) return cudaSuccess;
    const int64_t heads = p.batch * p.hv;
    const int sms = device_sm_count();
    const int rpw = heads * (kD / 64) >= 2 * sms ? 16 : heads * (kD / 32) >= 2 * sms ? 8 : 4;
    const int64_t grid = heads * (kD / (4 * rpw));
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    const unsigned g = static_cast<unsigned>(grid);
    const bool pdl = decode_pdl(heads);
    if (rpw == 16) return launch_decode_kernel(pdl, gdn_decode_tokens_kernel<16>, g, 128, stream, p, T);
    if (rpw == 8) return launch_decode_kernel(pdl, gdn_decode_tokens_kernel<8>, g, 128, stream, p, T);
    return launch_decode_kernel(pdl, gdn_decode_tokens_kernel<4>, g, 128, stream, p, T);
}

// CTA shape: rows per warp x warps per CTA.
//
// fp32 state: 4 rows per warp at every batch (16 rows per CTA of 4 warps; 2
// warps from 9 to 128 heads).  Kernel times from one ncu pass with the caches
// flushed before every launch, the reference's CUDA decode kernel in the same
// capture (4 rows x 4 warps / 2 warps / the earlier 16 rows x 4 warps /
// reference, us): B = 8: 4.35 / 4.10 / - / 4.22; B = 16: 5.25 / 4.90 / - /
// 5.12; B = 32: 6.66 / 7.17 / 7.94 / 7.10; B = 64: 10.62 / 10.40 / 12.03 /
// 10.46; B = 256: 36.61 / 36.93 / 38.59 / 36.48; B = 4096: 618.7 / - / 622.1 /
// 620.1.  Many small CTAs start and finish out of step, which keeps more of
// the stream in flight at every moment than a few large ones; back to back
// (three rotating state buffers) B = 256 takes 42.98 us at 4 rows against
// 43.86 at 16.
// bf16 state: 4 rows up to 128 heads, then the largest tile up to 16 rows
// that still gives >= 2 CTAs per SM (back to back / L2 flushed per call, B =
// 256: 24.67 / 26.44 us at 16 rows against 26.72 / 28.64 at 32 and 30.83 /
// 35.02 at 4; B = 64: 8.36 / 12.28 at 16 against 8.77 / 14.24 at 32).
struct DecodeShape {
    int rpw, warps;
};
static DecodeShape pick_decode_shape(int64_t heads, bool bf16_state) {
    if (!bf16_state) return {4, heads > 8 && heads <= 128 ? 2 : 4};
    const int sms = device_sm_count();
    if (heads <= 128) return {4, 4};
    if (heads * (kD / 64) >= 2 * sms) return {16, 4};
    if (heads * (kD / 32) >= 2 * sms) return {8, 4};
    return {4, 4};
}

// bf16_state: p.state / p.new_state point to bf16 [B, 8, 128, 128] arrays.
// pdl: launch as a programmatic dependent of the previous kernel in the
// stream (decode_pdl decides by size): consecutive steps overlap one
// kernel's drain with the next one's launch, and every global access of the
// next still follows the previous kernel's completion.  The host-staged path
// launches normally: its kernels follow waits on events of other streams.
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream, bool bf16_state = false, bool pdl = true) {
    if (p.batch == 0) return cudaSuccess;
    const int64_t heads = p.batch * p.hv;
    const DecodeShape sh = pick_decode_shape(heads, bf16_state);
    const int64_t grid = heads * (kD / (sh.warps * sh.rpw));
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    const unsigned g = static_cast<unsigned>(grid);
    pdl = pdl && decode_pdl(heads);
    if (!bf16_state) {
        if (sh.warps == 2) return launch_decode_kernel(pdl, gdn_decode_kernel<4, false, 2>, g, 64, stream, p);
        return launch_decode_kernel(pdl, gdn_decode_kernel<4, false, 4>, g, 128, stream, p);
    }
    switch (sh.rpw) {
        case 16: return launch_decode_kernel(pdl, gdn_decode_kernel<16, true>, g, 128, stream, p);
        case 8: return launch_decode_kernel(pdl, gdn_decode_kernel<8, true>, g, 128, stream, p);
        default: return launch_decode_kernel(pdl, gdn_decode_kernel<4, true>, g, 128, stream, p);
    }
}

}  // namespace gdn
