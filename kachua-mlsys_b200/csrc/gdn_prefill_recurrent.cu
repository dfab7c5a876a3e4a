// gdn_prefill_recurrent.cu -- token-recurrent varlen GDN prefill (SIMT, fp32).
//
// Runs the delta rule token by token, exactly the recurrence of the prefill
// oracle (prefill reference_torch_impl.py:66-91), with the state rows held in
// registers.  Rows of S (the v index) never interact, so a CTA owns
// (sequence, v-head, 16 state rows) and walks the sequence; the lane layout is
// the decode kernel's (8 lanes per row, float4 x 4 per lane).  The next
// token's q/k/v/gate inputs are fetched one step ahead of use.
//
// Cost is O(T d^2) on CUDA cores with a T-long dependency chain, so the host
// dispatcher only sends it short sequences; long ones go to the chunked
// tensor-core path.  It also gives the GPU tests an fp32 cross-check of the
// chunked path.
#include "gdn_common.cuh"

namespace gdn {

struct PrefillParams {
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    const float* state;  // may be null
    const float* A_log;
    const uint16_t* a;
    const float* dt_bias;
    const uint16_t* b;
    const void* cu_seqlens;
    int cu_is_int64;
    int64_t total_tokens;
    int64_t num_seqs;
    float scale;
    uint16_t* out;
    float* new_state;
};

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int64_t i) {
    return p.cu_is_int64 ? reinterpret_cast<const int64_t*>(p.cu_seqlens)[i]
                         : static_cast<int64_t>(reinterpret_cast<const int32_t*>(p.cu_seqlens)[i]);
}

// Sequence bounds with device-side validation: a range that is not
// non-decreasing or leaves [0, T] is reported and treated as empty.
__device__ __forceinline__ bool seq_bounds(const PrefillParams& p, int64_t s, int64_t& t0,
                                           int64_t& t1) {
    t0 = load_cu(p, s);
    t1 = load_cu(p, s + 1);
    if (t0 < 0 || t1 < t0 || t1 > p.total_tokens) {
        record_status(16 /* GDN_ERR_DEVICE_BAD_SEQLENS */);
        t0 = t1 = 0;
        return false;
    }
    return true;
}

constexpr int kRecRowsPerCta = 16;  // 4 warps x 4 rows
constexpr int kRecTiles = kD / kRecRowsPerCta;

struct TokenIn {
    float4 q[4], k[4];
    float v, a, b;
};

__device__ __forceinline__ void load_token(const PrefillParams& p, int64_t t, int hq, int h, int row,
                                           int sub, TokenIn& x) {
    const uint16_t* qp = p.q + (t * kHQK + hq) * kD + 4 * sub;
    const uint16_t* kp = p.k + (t * kHQK + hq) * kD + 4 * sub;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x.q[j] = bf16x4_to_float4(ld_u2(qp + 32 * j));
        x.k[j] = bf16x4_to_float4(ld_u2(kp + 32 * j));
    }
    x.v = bf16_bits_to_float(p.v[(t * kHV + h) * kD + row]);
    x.a = bf16_bits_to_float(p.a[t * kHV + h]);
    x.b = bf16_bits_to_float(p.b[t * kHV + h]);
}

__global__ void __launch_bounds__(128) gdn_prefill_recurrent_kernel(const PrefillParams p) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int grp = lane >> 3;
    const int sub = lane & 7;
    const int64_t unit = blockIdx.x / kRecTiles;  // s * 8 + h
    const int tile = static_cast<int>(blockIdx.x - unit * kRecTiles);
    const int64_t s = unit / kHV;
    const int h = static_cast<int>(unit - s * kHV);
    const int hq = h / kGva;
    const int row = tile * kRecRowsPerCta + warp * 4 + grp;

    int64_t t0, t1;
    seq_bounds(p, s, t0, t1);
    float* dst = p.new_state + (unit * kD + row) * kD + 4 * sub;
    float4 st[4];
    if (t1 <= t0) {  // empty sequence: zero new_state row (prefill reference_torch_impl.py:53-55)
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) st_stream_f4(dst + 32 * j, z);
        return;
    }
    if (p.state != nullptr) {
        const float* src = p.state + (unit * kD + row) * kD + 4 * sub;
#pragma unroll
        for (int j = 0; j < 4; ++j) st[j] = ld_stream_f4(src + 32 * j);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) st[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float A_log = p.A_log[h];
    const float dt_bias = p.dt_bias[h];
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);

    TokenIn cur, nxt;
    load_token(p, t0, hq, h, row, sub, nxt);
    for (int64_t t = t0; t < t1; ++t) {
        cur = nxt;
        if (t + 1 < t1) load_token(p, t + 1, hq, h, row, sub, nxt);
        float g, beta;
        gdn_gates(A_log, dt_bias, cur.a, cur.b, g, beta);
        float ks = 0.f, qs = 0.f, qk = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ks += st[j].x * cur.k[j].x + st[j].y * cur.k[j].y + st[j].z * cur.k[j].z +
                  st[j].w * cur.k[j].w;
            qs += st[j].x * cur.q[j].x + st[j].y * cur.q[j].y + st[j].z * cur.q[j].z +
                  st[j].w * cur.q[j].w;
            qk += cur.q[j].x * cur.k[j].x + cur.q[j].y * cur.k[j].y + cur.q[j].z * cur.k[j].z +
                  cur.q[j].w * cur.k[j].w;
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            ks += __shfl_xor_sync(0xffffffffu, ks, off);
            qs += __shfl_xor_sync(0xffffffffu, qs, off);
            qk += __shfl_xor_sync(0xffffffffu, qk, off);
        }
        const float delta = beta * (cur.v - g * ks);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            st[j].x = fmaf(g, st[j].x, delta * cur.k[j].x);
            st[j].y = fmaf(g, st[j].y, delta * cur.k[j].y);
            st[j].z = fmaf(g, st[j].z, delta * cur.k[j].z);
            st[j].w = fmaf(g, st[j].w, delta * cur.k[j].w);
        }
        if (sub == 0) out[(t * kHV + h) * kD + row] = __float2bfloat16_rn(p.scale * fmaf(g, qs, delta * qk));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) st_stream_f4(dst + 32 * j, st[j]);
}

// Zeroes output rows of tokens outside [cu[0], cu[N]) (the reference
// allocates its output with torch.zeros, prefill reference_torch_impl.py:41-45).
// Zero the output rows of tokens outside [cu_seqlens[0], cu_seqlens[N]) over
// the whole grid (the oracle's torch.zeros output).
__device__ __forceinline__ void zero_uncovered_rows(const PrefillParams& p) {
    int64_t lo = load_cu(p, 0), hi = load_cu(p, p.num_seqs);
    lo = lo < 0 ? 0 : (lo > p.total_tokens ? p.total_tokens : lo);
    hi = hi < lo ? lo : (hi > p.total_tokens ? p.total_tokens : hi);
    const int64_t per_tok = kHV * kD / 8;  // uint4 per token
    const int64_t n_head = lo * per_tok, n_tail = (p.total_tokens - hi) * per_tok;
    uint4* o = reinterpret_cast<uint4*>(p.out);
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_head + n_tail;
         i += (int64_t)gridDim.x * blockDim.x) {
        o[i < n_head ? i : hi * per_tok + (i - n_head)] = z;
    }
}

__global__ void gdn_prefill_zero_uncovered_kernel(const PrefillParams p) { zero_uncovered_rows(p); }

cudaError_t launch_prefill_recurrent(const PrefillParams& p, cudaStream_t stream) {
    const int64_t grid = p.num_seqs * kHV * kRecTiles;
    if (grid == 0) return cudaSuccess;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_prefill_recurrent_kernel<<<(unsigned)grid, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_zero_uncovered(const PrefillParams& p, cudaStream_t stream) {
    gdn_prefill_zero_uncovered_kernel<<<kSmCount, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gdn
