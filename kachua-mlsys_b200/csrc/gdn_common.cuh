// gdn_common.cuh -- shared constants and device helpers for the GDN kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHQK = 4;        // q/k heads
constexpr int kHV = 8;         // v heads
constexpr int kGva = kHV / kHQK;
constexpr int kD = 128;        // head dim (K and V)
// SM count of a B200.  Only layouts that must not depend on the device (the
// prefill workspace's segment slots, the context-parallel segment count that
// every rank must agree on) use this constant; launch shapes use
// device_sm_count().
constexpr int kSmCount = 148;

// Per-device status word (OR of GDN_ERR_DEVICE_* bits); one copy per device
// that loads the library.  The library is a single translation unit
// (gdn_capi.cu includes every kernel file), so this is its only definition.
__device__ int g_status = 0;

__device__ __forceinline__ void record_status(int bits) { atomicOr(&g_status, bits); }

// Multiprocessor count of the current device, queried once per device (falls
// back to kSmCount if the query fails).
static int device_sm_count() {
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kSmCount;
    if (cached[dev] == 0) {
        int n = 0;
        cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0
                          ? n
                          : kSmCount;
    }
    return cached[dev];
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// 4 packed bf16 (8 bytes) -> 4 floats
__device__ __forceinline__ float4 bf16x4_to_float4(uint2 u) {
    float4 r;
    r.x = __uint_as_float(u.x << 16);
    r.y = __uint_as_float(u.x & 0xffff0000u);
    r.z = __uint_as_float(u.y << 16);
    r.w = __uint_as_float(u.y & 0xffff0000u);
    return r;
}

// torch.nn.functional.softplus(x) with beta=1, threshold=20.
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// Decay g = exp(-exp(A_log) * softplus(a + dt_bias)) and beta = sigmoid(b),
// as decode reference_torch_impl.py:35-38 / prefill :34-36.
__device__ __forceinline__ void gdn_gates(float A_log, float dt_bias, float a, float b, float& g,
                                          float& beta) {
    const float x = a + dt_bias;
    g = expf(-expf(A_log) * softplus_f(x));
    beta = 1.0f / (1.0f + expf(-b));
}

// The same gates on the special-function unit (__expf, __logf, __fdividef):
// a shorter dependent chain between the gate inputs' arrival and the state
// update, which a single decode step at small batch waits on.  softplus is
// formed as max(x, 0) + log(1 + exp(-|x|)) (no cancellation), torch's
// threshold kept; g's relative error stays near 1e-6 (the intrinsics' few
// ulp, times exp(A_log) <= 16 for |softplus| errors ~1e-7), far inside the
// 1e-3 state tolerance.  The reference CUDA decode used the same intrinsics
// (kernel.cu:579-582, 655-657).
__device__ __forceinline__ void gdn_gates_fast(float A_log, float dt_bias, float a, float b, float& g, float& beta) {
    const float x = a + dt_bias;
    const float sp = x > 20.0f ? x : fmaxf(x, 0.0f) + __logf(1.0f + __expf(-fabsf(x)));
    g = __expf(-__expf(A_log) * sp);
    beta = __fdividef(1.0f, 1.0f + __expf(-b));
}

// log2 of the decay, for the chunked path: log2 g = -exp(A_log) * softplus(x) / ln 2.
__device__ __forceinline__ float gdn_log2_decay(float A_log, float dt_bias, float a) {
    return -expf(A_log) * softplus_f(a + dt_bias) * 1.4426950408889634f;
}

// Streaming 16-byte load that bypasses L1.  Coherent (no .nc), so it stays
// correct when the state is updated in place (state == new_state).
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
    float4 r;
    asm volatile("ld.global.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint2 ld_u2(const void* p) {
    return *reinterpret_cast<const uint2*>(p);
}

// 8-byte forms of the streaming state accesses (4 bf16 values)
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
    uint2 r;
    asm volatile("ld.global.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ void st_stream_u2(void* p, uint2 v) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
// 4 floats -> 4 packed bf16, round to nearest even
__device__ __forceinline__ uint2 float4_to_bf16x4(float4 f) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y), hi = __floats2bfloat162_rn(f.z, f.w);
    return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// --------------------------------------------- programmatic dependent launch --
// In a kernel launched with programmatic stream serialization: wait until the
// preceding kernel in the stream has completed and its memory is visible (a
// no-op in a kernel launched normally).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next kernel (if launched with programmatic serialization) begin
// launching once every CTA of this grid has executed this or exited.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch `kernel` so that it may begin (prologue up to griddep_wait) while the
// previous kernel in the stream finishes (programmatic dependent launch).
template <typename... Params, typename... Args>
static cudaError_t launch_dependent(void (*kernel)(Params...), unsigned grid, unsigned block, size_t smem,
                                    cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace gdn
