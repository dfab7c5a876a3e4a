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
//   * a CTA is 4 warps x RPW rows per warp; every load of a thread's rows is
//     issued before any arithmetic, so a 128-thread CTA keeps 16*RPW*128 bytes
//     in flight;
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
template <int RPW, bool BF16S>
__global__ void __launch_bounds__(128) gdn_decode_kernel(const DecodeParams p) {
    static_assert(RPW % 4 == 0, "rows per warp must be a multiple of 4");
    constexpr int kPasses = RPW / 4;
    constexpr int kRowsPerCta = 4 * RPW;
    constexpr int kTiles = kD / kRowsPerCta;

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
    gdn_gates(p.A_log[h], p.dt_bias[h], bf16_bits_to_float(p.a[bh]), bf16_bits_to_float(p.b[bh]), g,
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

// Rows per warp: the largest tile that still yields >= 2 CTAs per SM.
static int pick_rows_per_warp(int64_t heads, bool bf16_state) {
    // a bf16 row is half as many bytes: 32 rows keep the fp32 kernel's 256 B of loads in flight per thread
    if (bf16_state && heads >= 2 * kSmCount) return 32;
    if (heads * (kD / 64) >= 2 * kSmCount) return 16;
    if (heads * (kD / 32) >= 2 * kSmCount) return 8;
    return 4;
}

template <bool BF16S>
static void launch_decode_rpw(int rpw, unsigned grid, const DecodeParams& p, cudaStream_t stream) {
    switch (rpw) {
        case 32:  // bf16 state only
            if constexpr (BF16S) gdn_decode_kernel<32, true><<<grid, 128, 0, stream>>>(p);
            break;
        case 16: gdn_decode_kernel<16, BF16S><<<grid, 128, 0, stream>>>(p); break;
        case 8: gdn_decode_kernel<8, BF16S><<<grid, 128, 0, stream>>>(p); break;
        default: gdn_decode_kernel<4, BF16S><<<grid, 128, 0, stream>>>(p); break;
    }
}

// bf16_state: p.state / p.new_state point to bf16 [B, 8, 128, 128] arrays.
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream, bool bf16_state = false) {
    if (p.batch == 0) return cudaSuccess;
    const int64_t heads = p.batch * p.hv;
    const int rpw = pick_rows_per_warp(heads, bf16_state);
    const int64_t grid = heads * (kD / (4 * rpw));
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (bf16_state)
        launch_decode_rpw<true>(rpw, static_cast<unsigned>(grid), p, stream);
    else
        launch_decode_rpw<false>(rpw, static_cast<unsigned>(grid), p, stream);
    return cudaGetLastError();
}

}  // namespace gdn
