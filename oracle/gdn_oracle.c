/*
 * gdn_oracle.c -- CPU restatement of the reference's GDN recurrences.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in kachua-mlsys_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm may load it.  The product path
 * never calls it and has no CPU fallback.
 *
 * It restates, token by token and head by head, the two PyTorch reference
 * implementations of romitjain/kachua-mlsys:
 *
 *   decode : gdn_decode_qk4_v8_d128_k_last/solution/reference_torch_impl.py:12-72
 *   prefill: gdn_prefill_qk4_v8_d128_k_last/solution/reference_torch_impl.py:17-92
 *
 * Arithmetic is fp32 (as torch's .float() path), in the reference's order:
 *   x        = a + dt_bias                              (decode :35, prefill :34)
 *   g        = exp(-exp(A_log) * softplus(x))           (decode :36, prefill :35)
 *   beta     = sigmoid(b)                               (decode :37, prefill :36)
 *   old      = g * S                                    (decode :60, prefill :74)
 *   old_v    = k @ old                                  (decode :61, prefill :75)
 *   new_v    = beta * v + (1 - beta) * old_v            (decode :62, prefill :76)
 *   S        = old - k (x) old_v + k (x) new_v          (decode :63-65, prefill :77-87)
 *   o        = scale * q @ S                            (decode :67, prefill :89)
 * with q/k head = v head / 2 (repeat_interleave, decode :46-47, prefill :38-39).
 * The *_heads entry points take other head counts (num_v_heads a multiple of
 * num_qk_heads, q/k head = v head / (num_v_heads / num_qk_heads), the same
 * repeat_interleave grouping); the plain ones are the reference's 4 / 8.
 * softplus follows torch.nn.functional.softplus (beta 1, threshold 20).
 * The state is stored k-last: S[v][k] (the reference transposes to [K,V]
 * and back, decode :57/:68, prefill :58/:91; the math is the same).
 *
 * Output conventions follow the references exactly:
 *   decode  output is fp32 [B, HV, V]                   (decode :50)
 *   prefill output is bf16 [T, HV, V], rounded per token (prefill :89)
 *   prefill: state == NULL means a zero initial state   (prefill :57-64)
 *   prefill: an empty sequence leaves its new_state row zero (prefill :53-55)
 *
 * Parity is pinned by tests/test_oracle_golden.py against vectors produced
 * by importing the reference's own reference_torch_impl.py
 * (tests/golden/gen_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORC_HQK 4
#define ORC_HV 8
#define ORC_D 128

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even float -> bf16, as torch's .to(torch.bfloat16). */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    }
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float softplus_torch(float x) {
    /* torch.nn.functional.softplus(x, beta=1, threshold=20) */
    return x > 20.0f ? x : log1pf(expf(x));
}

static inline void gates(float A_log, float dt_bias, float a, float b, float* g, float* beta) {
    float x = a + dt_bias;
    *g = expf(-expf(A_log) * softplus_torch(x));
    *beta = 1.0f / (1.0f + expf(-b));
}

/*
 * One token of the delta rule on one head.  S is [V][K] (k-last), updated in
 * place.  qf/kf/vf are the fp32 q, k, v vectors; out receives scale * q @ S.
 */
static void head_step(float* S, const float* qf, const float* kf, const float* vf,
                      float g, float beta, float scale, float* out) {
    for (int vi = 0; vi < ORC_D; ++vi) {
        float* row = S + (size_t)vi * ORC_D;
        float old_v = 0.0f;
        for (int ki = 0; ki < ORC_D; ++ki) {
            row[ki] = g * row[ki];            /* old = g * S */
            old_v += kf[ki] * row[ki];        /* old_v = k @ old */
        }
        float new_v = beta * vf[vi] + (1.0f - beta) * old_v;
        float acc = 0.0f;
        for (int ki = 0; ki < ORC_D; ++ki) {
            float s = row[ki] - kf[ki] * old_v + kf[ki] * new_v;
            row[ki] = s;
            acc += qf[ki] * s;
        }
        out[vi] = scale * acc;
    }
}

static void load_bf16_vec(const uint16_t* src, float* dst) {
    for (int i = 0; i < ORC_D; ++i) dst[i] = bf16_to_f32(src[i]);
}

/*
 * Decode: q,k bf16 [B,1,4,128]; v bf16 [B,1,8,128]; state fp32 [B,8,128,128];
 * A_log, dt_bias fp32 [8]; a, b bf16 [B,1,8]; output fp32 [B,8,128];
 * new_state fp32 [B,8,128,128].  scale == 0 selects 1/sqrt(128) (None maps to 0).
 */
int oracle_gdn_decode_heads(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                            const float* state, const float* A_log, const uint16_t* a,
                            const float* dt_bias, const uint16_t* b, float scale,
                            int64_t batch, float* output, float* new_state, int num_threads,
                            int hqk, int hv) {
    if (hqk < 1 || hv < hqk || hv % hqk) return -1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)ORC_D); /* `scale is None or scale == 0.0` */
    const int64_t units = batch * hv;
#pragma omp parallel for schedule(dynamic, 4) num_threads(num_threads)
    for (int64_t u = 0; u < units; ++u) {
        const int64_t bi = u / hv;
        const int h = (int)(u % hv);
        const int hq = h / (hv / hqk);
        float qf[ORC_D], kf[ORC_D], vf[ORC_D];
        load_bf16_vec(q + (bi * hqk + hq) * ORC_D, qf);
        load_bf16_vec(k + (bi * hqk + hq) * ORC_D, kf);
        load_bf16_vec(v + (bi * hv + h) * ORC_D, vf);
        float g, beta;
        gates(A_log[h], dt_bias[h], bf16_to_f32(a[bi * hv + h]),
              bf16_to_f32(b[bi * hv + h]), &g, &beta);
        float* S = new_state + u * ORC_D * ORC_D;
        if (S != state + u * ORC_D * ORC_D) {
            memcpy(S, state + u * ORC_D * ORC_D, sizeof(float) * ORC_D * ORC_D);
        }
        head_step(S, qf, kf, vf, g, beta, scale, output + u * ORC_D);
    }
    return 0;
}

int oracle_gdn_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const float* state, const float* A_log, const uint16_t* a,
                      const float* dt_bias, const uint16_t* b, float scale,
                      int64_t batch, float* output, float* new_state, int num_threads) {
    return oracle_gdn_decode_heads(q, k, v, state, A_log, a, dt_bias, b, scale, batch, output, new_state,
                                   num_threads, ORC_HQK, ORC_HV);
}

/*
 * Prefill: q,k bf16 [T,4,128]; v bf16 [T,8,128]; state fp32 [N,8,128,128] or
 * NULL; a, b bf16 [T,8]; cu_seqlens int64 [N+1]; output bf16 [T,8,128];
 * new_state fp32 [N,8,128,128].  Tokens outside every sequence keep the
 * output zero (the reference allocates output with torch.zeros, prefill :41-45).
 */
int oracle_gdn_prefill_heads(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                             const float* state, const float* A_log, const uint16_t* a,
                             const float* dt_bias, const uint16_t* b,
                             const int64_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                             float scale, uint16_t* output, float* new_state, int num_threads,
                             int hqk, int hv) {
    if (hqk < 1 || hv < hqk || hv % hqk) return -1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)ORC_D); /* `scale is None or scale == 0.0` */
    memset(output, 0, sizeof(uint16_t) * (size_t)total_tokens * hv * ORC_D);
    const int64_t units = num_seqs * hv;
#pragma omp parallel for schedule(dynamic, 1) num_threads(num_threads)
    for (int64_t u = 0; u < units; ++u) {
        const int64_t s = u / hv;
        const int h = (int)(u % hv);
        const int hq = h / (hv / hqk);
        float* S = new_state + u * ORC_D * ORC_D;
        const int64_t t0 = cu_seqlens[s], t1 = cu_seqlens[s + 1];
        if (t1 <= t0) {
            memset(S, 0, sizeof(float) * ORC_D * ORC_D);
            continue;
        }
        if (state) {
            memcpy(S, state + u * ORC_D * ORC_D, sizeof(float) * ORC_D * ORC_D);
        } else {
            memset(S, 0, sizeof(float) * ORC_D * ORC_D);
        }
        float qf[ORC_D], kf[ORC_D], vf[ORC_D], of[ORC_D];
        for (int64_t t = t0; t < t1; ++t) {
            load_bf16_vec(q + (t * hqk + hq) * ORC_D, qf);
            load_bf16_vec(k + (t * hqk + hq) * ORC_D, kf);
            load_bf16_vec(v + (t * hv + h) * ORC_D, vf);
            float g, beta;
            gates(A_log[h], dt_bias[h], bf16_to_f32(a[t * hv + h]),
                  bf16_to_f32(b[t * hv + h]), &g, &beta);
            head_step(S, qf, kf, vf, g, beta, scale, of);
            uint16_t* o = output + (t * hv + h) * ORC_D;
            for (int i = 0; i < ORC_D; ++i) o[i] = f32_to_bf16(of[i]);
        }
    }
    return 0;
}

int oracle_gdn_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                       const float* state, const float* A_log, const uint16_t* a,
                       const float* dt_bias, const uint16_t* b,
                       const int64_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                       float scale, uint16_t* output, float* new_state, int num_threads) {
    return oracle_gdn_prefill_heads(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                                    scale, output, new_state, num_threads, ORC_HQK, ORC_HV);
}

int oracle_abi_version(void) { return 2; }
