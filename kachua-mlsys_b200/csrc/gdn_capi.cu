// gdn_capi.cu -- the extern "C" boundary (include/gdn_b200.h).
//
// The library is built as one translation unit: this file includes every
// kernel source, so the per-device status word needs no relocatable device
// code.  Every entry point validates pointers, sizes and alignment on the
// host and returns a gdn_status_t before anything is launched; the reference
// plugin did no checking at all (kernel.cu:982-1064).
#include "gdn_b200.h"

#include "gdn_common.cuh"
#include "gdn_decode.cu"
#include "gdn_prefill_recurrent.cu"
#include "gdn_prefill_chunked.cu"

#include <math.h>

namespace gdn {
static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The current device must be an sm_100 part (the cubin is sm_100a only).
static int check_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_NO_DEVICE;
    static int cached[64];  // 0 = unknown, 1 = ok, 2 = bad
    if (dev >= 0 && dev < 64 && cached[dev] != 0) return cached[dev] == 1 ? GDN_OK : GDN_ERR_NO_DEVICE;
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
        return GDN_ERR_NO_DEVICE;
    const bool ok = (major == 10 && minor == 0);
    if (dev >= 0 && dev < 64) cached[dev] = ok ? 1 : 2;
    return ok ? GDN_OK : GDN_ERR_NO_DEVICE;
}

static float resolve_scale(float s) { return s == 0.0f ? 1.0f / sqrtf((float)kD) : s; }
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_abi_version(void) { return 9; }

extern "C" const char* gdn_status_string(int status) {
    switch (status) {
        case GDN_OK: return "ok";
        case GDN_ERR_NULL_POINTER: return "a required pointer is NULL";
        case GDN_ERR_BAD_SIZE: return "negative or inconsistent sizes";
        case GDN_ERR_MISALIGNED: return "a pointer violates its alignment rule";
        case GDN_ERR_WORKSPACE: return "workspace missing or too small";
        case GDN_ERR_CUDA: return "a CUDA runtime call failed";
        case GDN_ERR_BAD_DTYPE: return "unsupported cu_seqlens dtype code";
        case GDN_ERR_NO_DEVICE: return "no usable sm_100 device is current";
        case GDN_ERR_DEVICE_BAD_SEQLENS: return "device: cu_seqlens not monotone or out of range";
        case GDN_ERR_DEVICE_TIMEOUT: return "device: a bounded wait expired";
        default: return "unknown status";
    }
}

static bool heads_ok(int hqk, int hv) { return hqk >= 1 && hv >= hqk && hv % hqk == 0 && hv <= 4096; }

static int decode_launch(const GdnDecodeArgs* a, void* stream, bool bf16_state, int hqk = kHQK, int hv = kHV) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (a->batch < 0) return GDN_ERR_BAD_SIZE;
    if (a->batch == 0) return GDN_OK;
    if (!a->q || !a->k || !a->v || !a->state || !a->A_log || !a->a || !a->dt_bias || !a->b ||
        !a->output || !a->new_state)
        return GDN_ERR_NULL_POINTER;
    const uintptr_t sa = bf16_state ? 8 : 16;  // state rows are read 4 elements at a time
    if (!aligned(a->q, 8) || !aligned(a->k, 8) || !aligned(a->state, sa) || !aligned(a->new_state, sa) ||
        !aligned(a->v, 2) || !aligned(a->a, 2) || !aligned(a->b, 2) || !aligned(a->output, 2) ||
        !aligned(a->A_log, 4) || !aligned(a->dt_bias, 4))
        return GDN_ERR_MISALIGNED;
    if (int rc = check_device()) return rc;
    DecodeParams p;
    p.q = static_cast<const uint16_t*>(a->q);
    p.k = static_cast<const uint16_t*>(a->k);
    p.v = static_cast<const uint16_t*>(a->v);
    p.state = a->state;
    p.A_log = a->A_log;
    p.a = static_cast<const uint16_t*>(a->a);
    p.dt_bias = a->dt_bias;
    p.b = static_cast<const uint16_t*>(a->b);
    p.out = static_cast<uint16_t*>(a->output);
    p.new_state = a->new_state;
    p.batch = a->batch;
    p.scale = resolve_scale(a->scale);
    p.hqk = hqk;
    p.hv = hv;
    if (p.batch * hv * (kD / 16) > 0x7fffffffLL) return GDN_ERR_BAD_SIZE;
    return launch_decode(p, static_cast<cudaStream_t>(stream), bf16_state) == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_decode_launch(const GdnDecodeArgs* a, void* stream) { return decode_launch(a, stream, false); }

// The state kept in bf16 (half the HBM stream of the fp32 state); args->state
// and args->new_state point to bf16 arrays.
extern "C" int gdn_decode_launch_bf16_state(const GdnDecodeArgs* a, void* stream) {
    return decode_launch(a, stream, true);
}

// T tokens per sequence (speculative or multi-token decode): the state rows
// stay in registers for all T updates, so the state is read and written once
// per call, as in a single-token step (gdn_decode_tokens_kernel).
static int decode_tokens(const GdnDecodeArgs* a, int64_t tokens, void* stream, int hqk, int hv) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (tokens < 1 || a->batch < 0) return GDN_ERR_BAD_SIZE;
    if (tokens == 1) return decode_launch(a, stream, false, hqk, hv);
    if (a->batch == 0) return GDN_OK;
    if (tokens > 0x7fffffffLL || a->batch > (int64_t(1) << 40) / tokens || a->batch * hv * (kD / 16) > 0x7fffffffLL)
        return GDN_ERR_BAD_SIZE;
    if (!a->q || !a->k || !a->v || !a->state || !a->A_log || !a->a || !a->dt_bias || !a->b || !a->output ||
        !a->new_state)
        return GDN_ERR_NULL_POINTER;
    if (!aligned(a->q, 8) || !aligned(a->k, 8) || !aligned(a->state, 16) || !aligned(a->new_state, 16) ||
        !aligned(a->v, 2) || !aligned(a->a, 2) || !aligned(a->b, 2) || !aligned(a->output, 2) ||
        !aligned(a->A_log, 4) || !aligned(a->dt_bias, 4))
        return GDN_ERR_MISALIGNED;
    if (int rc = check_device()) return rc;
    DecodeParams p;
    p.q = static_cast<const uint16_t*>(a->q);
    p.k = static_cast<const uint16_t*>(a->k);
    p.v = static_cast<const uint16_t*>(a->v);
    p.state = a->state;  // may equal new_state: every tile is read before it is written, by one CTA
    p.A_log = a->A_log;
    p.a = static_cast<const uint16_t*>(a->a);
    p.dt_bias = a->dt_bias;
    p.b = static_cast<const uint16_t*>(a->b);
    p.out = static_cast<uint16_t*>(a->output);
    p.new_state = a->new_state;
    p.batch = a->batch;
    p.scale = resolve_scale(a->scale);
    p.hqk = hqk;
    p.hv = hv;
    return launch_decode_tokens(p, static_cast<int>(tokens), static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? GDN_OK
               : GDN_ERR_CUDA;
}

extern "C" int gdn_decode_launch_tokens(const GdnDecodeArgs* a, int64_t tokens, void* stream) {
    return decode_tokens(a, tokens, stream, kHQK, kHV);
}

// Other head counts: every decode form (tokens >= 1, fp32 state; or one token
// with a bf16 state) with num_qk_heads / num_v_heads given.
extern "C" int gdn_decode_launch_heads(const GdnDecodeArgs* a, int32_t num_qk_heads, int32_t num_v_heads,
                                       int64_t tokens, int32_t bf16_state, void* stream) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (!heads_ok(num_qk_heads, num_v_heads) || tokens < 1 || (bf16_state && tokens != 1)) return GDN_ERR_BAD_SIZE;
    if (bf16_state) return decode_launch(a, stream, true, num_qk_heads, num_v_heads);
    return decode_tokens(a, tokens, stream, num_qk_heads, num_v_heads);
}

extern "C" size_t gdn_prefill_workspace_size(int64_t total_tokens, int64_t num_seqs) {
    if (total_tokens < 0 || num_seqs < 0) return 0;
    return chunked_workspace_bytes(total_tokens, num_seqs);
}

// Argument checks shared by the prefill entry points, then the kernel parameters.
static int prefill_setup(const GdnPrefillArgs* a, PrefillParams& p, int hqk, int hv) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (a->total_tokens < 0 || a->num_seqs < 0) return GDN_ERR_BAD_SIZE;
    if (a->cu_seqlens_dtype != GDN_SEQLENS_INT32 && a->cu_seqlens_dtype != GDN_SEQLENS_INT64)
        return GDN_ERR_BAD_DTYPE;
    if (a->path < GDN_PREFILL_PATH_AUTO || a->path > GDN_PREFILL_PATH_SEGMENTED) return GDN_ERR_BAD_SIZE;
    if (!a->cu_seqlens || !a->A_log || !a->dt_bias) return GDN_ERR_NULL_POINTER;
    if (a->total_tokens > 0 &&
        (!a->q || !a->k || !a->v || !a->a || !a->b || !a->output))
        return GDN_ERR_NULL_POINTER;
    if (a->num_seqs > 0 && !a->new_state) return GDN_ERR_NULL_POINTER;
    if (!aligned(a->q, 16) || !aligned(a->k, 16) || !aligned(a->v, 16) || !aligned(a->output, 16) ||
        !aligned(a->new_state, 16) || !aligned(a->state, 16) || !aligned(a->a, 2) || !aligned(a->b, 2) ||
        !aligned(a->cu_seqlens, a->cu_seqlens_dtype == GDN_SEQLENS_INT64 ? 8 : 4))
        return GDN_ERR_MISALIGNED;
    if (a->state != nullptr && a->num_seqs > 0 && a->state == a->new_state) return GDN_ERR_BAD_SIZE;
    if (int rc = check_device()) return rc;
    p.q = static_cast<const uint16_t*>(a->q);
    p.k = static_cast<const uint16_t*>(a->k);
    p.v = static_cast<const uint16_t*>(a->v);
    p.state = a->state;
    p.A_log = a->A_log;
    p.a = static_cast<const uint16_t*>(a->a);
    p.dt_bias = a->dt_bias;
    p.b = static_cast<const uint16_t*>(a->b);
    p.cu_seqlens = a->cu_seqlens;
    p.cu_is_int64 = a->cu_seqlens_dtype == GDN_SEQLENS_INT64;
    p.total_tokens = a->total_tokens;
    p.num_seqs = a->num_seqs;
    p.scale = resolve_scale(a->scale);
    p.out = static_cast<uint16_t*>(a->output);
    p.new_state = a->new_state;
    p.uniform_len = 0;
    p.hqk = hqk;
    p.hv = hv;
    return GDN_OK;
}

extern "C" int gdn_prefill_launch(const GdnPrefillArgs* a, void* workspace, size_t workspace_bytes,
                                  void* stream) {
    PrefillParams p;
    if (int rc = prefill_setup(a, p, kHQK, kHV)) return rc;
    // the token-recurrent path needs no workspace; the chunked paths need the records
    const size_t need = prefill_path_is_recurrent(a->path, a->total_tokens, a->num_seqs)
                            ? 0
                            : chunked_workspace_min_bytes(a->total_tokens, a->num_seqs);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)))
        return GDN_ERR_WORKSPACE;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->num_seqs == 0)  // every token is uncovered: zero output
        return a->total_tokens > 0 && launch_prefill_zero_uncovered(p, s) != cudaSuccess ? GDN_ERR_CUDA : GDN_OK;
    const cudaError_t e = launch_prefill(p, a->path, workspace, workspace_bytes, s);
    return e == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

// Context parallelism (one batch of sequences split by token range over
// `world` ranks; see launch_prefill_cp for the protocol).
extern "C" size_t gdn_prefill_cp_workspace_size(int64_t local_tokens, int64_t num_seqs, int32_t world) {
    if (local_tokens < 0 || num_seqs < 0 || world < 1 || world > 4096) return 0;
    return static_cast<size_t>(cp_layout(local_tokens, num_seqs, world).total_seg);
}

extern "C" size_t gdn_prefill_cp_summary_offset(int64_t local_tokens, int64_t num_seqs) {
    if (local_tokens < 0 || num_seqs < 0) return 0;
    return static_cast<size_t>(ws_layout(local_tokens, num_seqs).total);
}

extern "C" int gdn_prefill_cp_launch(const GdnPrefillArgs* a, void* workspace, size_t workspace_bytes, int32_t rank,
                                     int32_t world, int32_t phase, void* stream) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (world < 1 || world > 4096 || rank < 0 || rank >= world || (phase != 0 && phase != 1)) return GDN_ERR_BAD_SIZE;
    PrefillParams p;
    if (int rc = prefill_setup(a, p, kHQK, kHV)) return rc;
    if (a->num_seqs == 0) return GDN_OK;
    const size_t need = static_cast<size_t>(cp_layout(a->total_tokens, a->num_seqs, world).total_seg);
    if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)) return GDN_ERR_WORKSPACE;
    const cudaError_t e =
        launch_prefill_cp(p, workspace, workspace_bytes, rank, world, phase, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

// Other head counts: the same paths as gdn_prefill_launch (the chunked
// kernels take the head counts from the parameters); the token-recurrent
// path needs no workspace.
extern "C" size_t gdn_prefill_workspace_size_heads(int64_t total_tokens, int64_t num_seqs, int32_t num_v_heads) {
    if (total_tokens < 0 || num_seqs < 0 || num_v_heads < 1 || num_v_heads > 4096) return 0;
    return chunked_workspace_bytes(total_tokens, num_seqs, num_v_heads);
}

extern "C" int gdn_prefill_launch_heads(const GdnPrefillArgs* a, int32_t num_qk_heads, int32_t num_v_heads,
                                        void* workspace, size_t workspace_bytes, void* stream) {
    if (a == nullptr) return GDN_ERR_NULL_POINTER;
    if (!heads_ok(num_qk_heads, num_v_heads)) return GDN_ERR_BAD_SIZE;
    PrefillParams p;
    if (int rc = prefill_setup(a, p, num_qk_heads, num_v_heads)) return rc;
    if (a->num_seqs * num_v_heads * (kD / 16) > 0x7fffffffLL) return GDN_ERR_BAD_SIZE;
    const size_t need = prefill_path_is_recurrent(a->path, a->total_tokens, a->num_seqs)
                            ? 0
                            : chunked_workspace_min_bytes(a->total_tokens, a->num_seqs, num_v_heads);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)))
        return GDN_ERR_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->num_seqs == 0)  // every token is uncovered: zero output
        return a->total_tokens > 0 && launch_prefill_zero_uncovered(p, s) != cudaSuccess ? GDN_ERR_CUDA : GDN_OK;
    return launch_prefill(p, a->path, workspace, workspace_bytes, s) == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_read_device_status(int* out, int clear, void* stream) {
    if (out == nullptr) return GDN_ERR_NULL_POINTER;
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return GDN_ERR_CUDA;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return GDN_ERR_CUDA;
    *out = v;
    if (clear) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_status, &z, sizeof(int)) != cudaSuccess) return GDN_ERR_CUDA;
    }
    return GDN_OK;
}

extern "C" int gdn_mma_selftest(int kind, int flags, int M, int N, int K, const void* A, const void* B, float* D,
                                void* stream) {
    if (!A || !B || !D) return GDN_ERR_NULL_POINTER;
    if ((kind != GDN_MMA_KIND_BF16 && kind != GDN_MMA_KIND_TF32 && kind != GDN_MMA_KIND_F16) || (M != 64 && M != 128) ||
        N < 16 ||
        N > 256 || N % 16 != 0 || (K != 64 && K != 128) || (flags & ~31) != 0 || ((flags & 4) && M != 64) ||
        ((flags & 8) && (M != 128 || kind == GDN_MMA_KIND_TF32 || (flags & 1))))
        return GDN_ERR_BAD_SIZE;
    // an MN-major image fills whole 128-byte rows: its M (or N) extent must be too
    const int row_elems = kind == GDN_MMA_KIND_TF32 ? 32 : 64;
    if (((flags & 1) && M % row_elems != 0) || ((flags & 2) && N % row_elems != 0)) return GDN_ERR_BAD_SIZE;
    if (int rc = check_device()) return rc;
    const int k = kind == GDN_MMA_KIND_F16 ? (int)kF16 : kind == GDN_MMA_KIND_BF16 ? (int)kBF16 : (int)kTF32;
    return launch_mma_selftest(k, flags, M, N, K, A, B, D, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? GDN_OK
               : GDN_ERR_CUDA;
}

// Allocation-free prefill entry point (fixed scratch array in this library).
#include "gdn_prefill_noalloc.cu"

// Decode with the state in host memory, transfers pipelined with the kernel.
#include "gdn_decode_staged.cu"
