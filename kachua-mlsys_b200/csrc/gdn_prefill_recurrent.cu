// gdn_prefill_recurrent.cu -- token-recurrent varlen GDN prefill (SIMT, fp32).
//
// Runs the delta rule token by token, exactly the recurrence of the prefill
// oracle (prefill reference_torch_impl.py:66-91), with the state rows held in
// registers.  Rows of S (the v index) never interact, so a CTA owns
// (sequence, v-head, 16 state rows) and walks the sequence; the lane layout is
// the decode kernel's (8 lanes per row, float4 x 4 per lane).  Token inputs
// (q, k, the CTA's v rows, the gates) are staged in shared memory 32 tokens
// at a time.
//
// Cost is O(T d^2) on CUDA cores with a T-long dependency chain, so the host
// dispatcher only sends it short sequences; long ones go to the chunked
// tensor-core path.  It is also the multi-token decode (T tokens per sequence,
// state read and written once) and gives the GPU tests an fp32 cross-check
// of the chunked path.
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
    int64_t uniform_len;  // > 0: every sequence has this many tokens and cu_seqlens is unused
    int hqk, hv;          // q/k and v heads; the chunked kernels take only 4 / 8
};

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int64_t i) {
    if (p.uniform_len > 0) return i * p.uniform_len;
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
constexpr int kRecBlk = 32;  // tokens staged in shared memory at a time

__global__ void __launch_bounds__(128) gdn_prefill_recurrent_kernel(const PrefillParams p) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int grp = lane >> 3;
    const int sub = lane & 7;
    const int64_t unit = blockIdx.x / kRecTiles;  // s * 8 + h
    const int tile = static_cast<int>(blockIdx.x - unit * kRecTiles);
    const int64_t s = unit / p.hv;
    const int h = static_cast<int>(unit - s * p.hv);
    const int hq = h / (p.hv / p.hqk);
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

    // Tokens in blocks of 32: the CTA stages the block's q and k (its qk head),
    // v (its 16 rows) and gates (one token per lane of warp 0) in shared memory
    // with loads that are all in flight at once, then walks the block from
    // there, so a token costs shared-memory latency, not an L2 round trip.
    __shared__ uint2 s_q[kRecBlk][kD / 4], s_k[kRecBlk][kD / 4];  // 4 bf16 per uint2
    __shared__ uint16_t s_v[kRecBlk][kRecRowsPerCta];
    __shared__ float s_g[kRecBlk], s_b[kRecBlk], s_qk[kRecBlk];
    const int tid = threadIdx.x;
    const int vrow0 = tile * kRecRowsPerCta;
    for (int64_t tb = t0; tb < t1; tb += kRecBlk) {
        const int nb = t1 - tb < kRecBlk ? static_cast<int>(t1 - tb) : kRecBlk;
        __syncthreads();  // the previous block is consumed
        // a warp stages one token's q and k per pass (32 x 4 dims) and reduces q.k
        for (int e = tid; e < nb * (kD / 4); e += 128) {
            const int i = e / (kD / 4), c = e % (kD / 4);
            const int64_t base = ((tb + i) * p.hqk + hq) * (kD / 4) + c;
            const uint2 qu = reinterpret_cast<const uint2*>(p.q)[base], ku = reinterpret_cast<const uint2*>(p.k)[base];
            s_q[i][c] = qu;
            s_k[i][c] = ku;
            const float4 qf = bf16x4_to_float4(qu), kf = bf16x4_to_float4(ku);
            float d = qf.x * kf.x + qf.y * kf.y + qf.z * kf.z + qf.w * kf.w;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            if (c == 0) s_qk[i] = d;
        }
        for (int e = tid; e < nb * kRecRowsPerCta; e += 128) {
            const int i = e / kRecRowsPerCta, r = e % kRecRowsPerCta;
            s_v[i][r] = p.v[((tb + i) * p.hv + h) * kD + vrow0 + r];
        }
        if (tid < nb) {
            const int64_t t = tb + tid;
            float g, beta;
            gdn_gates(A_log, dt_bias, bf16_bits_to_float(p.a[t * p.hv + h]), bf16_bits_to_float(p.b[t * p.hv + h]), g,
                      beta);
            s_g[tid] = g;
            s_b[tid] = beta;
        }
        __syncthreads();
        for (int i = 0; i < nb; ++i) {
            const int64_t t = tb + i;
            float4 q4[4], k4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q4[j] = bf16x4_to_float4(s_q[i][sub + 8 * j]);
                k4[j] = bf16x4_to_float4(s_k[i][sub + 8 * j]);
            }
            const float v = bf16_bits_to_float(s_v[i][warp * 4 + grp]);
            const float g = s_g[i], beta = s_b[i], qk = s_qk[i];
            float ks = 0.f, qs = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ks += st[j].x * k4[j].x + st[j].y * k4[j].y + st[j].z * k4[j].z + st[j].w * k4[j].w;
                qs += st[j].x * q4[j].x + st[j].y * q4[j].y + st[j].z * q4[j].z + st[j].w * q4[j].w;
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) {
                ks += __shfl_xor_sync(0xffffffffu, ks, off);
                qs += __shfl_xor_sync(0xffffffffu, qs, off);
            }
            const float delta = beta * (v - g * ks);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                st[j].x = fmaf(g, st[j].x, delta * k4[j].x);
                st[j].y = fmaf(g, st[j].y, delta * k4[j].y);
                st[j].z = fmaf(g, st[j].z, delta * k4[j].z);
                st[j].w = fmaf(g, st[j].w, delta * k4[j].w);
            }
            if (sub == 0) out[(t * p.hv + h) * kD + row] = __float2bfloat16_rn(p.scale * fmaf(g, qs, delta * qk));
        }
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
    const int64_t per_tok = static_cast<int64_t>(p.hv) * kD / 8;  // uint4 per token
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
    const int64_t grid = p.num_seqs * p.hv * kRecTiles;
    if (grid == 0) return cudaSuccess;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_prefill_recurrent_kernel<<<(unsigned)grid, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_zero_uncovered(const PrefillParams& p, cudaStream_t stream) {
    gdn_prefill_zero_uncovered_kernel<<<device_sm_count(), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gdn
