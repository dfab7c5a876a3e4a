// gdn_decode_staged.cu -- decode with the recurrent state kept in host memory.
//
// A server that offloads the per-sequence state (128 KiB per head group,
// 512 KiB per sequence) to host memory between steps pays two PCIe transfers
// of it per step; the kernel itself is ~40 us for 256 sequences.  This entry
// point hides the transfers behind one another: the batch is cut into
// slices, and slice i's host->device copy, slice i-1's decode kernel and
// slice i-2's device->host copy run at once on three streams owned by this
// library (created once per device, with that device current).  The caller's
// device buffers receive the inputs and hold the state during the step.
// Everything is enqueued from C (one call per step), so the host keeps ahead
// of the copies even with many slices.  Host buffers must be pinned
// (page-locked) for the copies to run asynchronously.
#include <mutex>

namespace gdn {

constexpr int kStagedMaxSlices = 64;
constexpr int kStagedMaxDevices = 64;

struct StagedCtx {
    bool ready;
    cudaStream_t s[3];  // host->device, compute, device->host
    cudaEvent_t start, end[3], in[kStagedMaxSlices], done[kStagedMaxSlices];
};
static StagedCtx g_staged[kStagedMaxDevices];
static std::mutex g_staged_mutex;  // held while a call enqueues: calls share the streams and events

static cudaError_t staged_ctx_init(StagedCtx& c) {
    cudaError_t e;
    for (int i = 0; i < 3; ++i)
        if ((e = cudaStreamCreateWithFlags(&c.s[i], cudaStreamNonBlocking)) != cudaSuccess) return e;
    if ((e = cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming)) != cudaSuccess) return e;
    for (int i = 0; i < 3; ++i)
        if ((e = cudaEventCreateWithFlags(&c.end[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    for (int i = 0; i < kStagedMaxSlices; ++i) {
        if ((e = cudaEventCreateWithFlags(&c.in[i], cudaEventDisableTiming)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&c.done[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    c.ready = true;
    return cudaSuccess;
}

}  // namespace gdn

extern "C" int gdn_decode_launch_host_staged(const GdnDecodeArgs* host, const GdnDecodeArgs* dev, int slices,
                                             void* stream) {
    using namespace gdn;
    if (host == nullptr || dev == nullptr) return GDN_ERR_NULL_POINTER;
    if (host->batch < 0 || dev->batch != host->batch || slices < 1 || slices > kStagedMaxSlices)
        return GDN_ERR_BAD_SIZE;
    const int64_t B = host->batch;
    if (B == 0) return GDN_OK;
    if (!host->q || !host->k || !host->v || !host->state || !host->A_log || !host->a || !host->dt_bias ||
        !host->b || !host->output || !host->new_state)
        return GDN_ERR_NULL_POINTER;
    if (!dev->q || !dev->k || !dev->v || !dev->A_log || !dev->a || !dev->dt_bias || !dev->b || !dev->output ||
        !dev->new_state)
        return GDN_ERR_NULL_POINTER;
    if (dev->state != nullptr && dev->state != dev->new_state) return GDN_ERR_BAD_SIZE;  // one in-place buffer
    if (!aligned(dev->q, 8) || !aligned(dev->k, 8) || !aligned(dev->new_state, 16) || !aligned(dev->v, 2) ||
        !aligned(dev->a, 2) || !aligned(dev->b, 2) || !aligned(dev->output, 2) || !aligned(dev->A_log, 4) ||
        !aligned(dev->dt_bias, 4))
        return GDN_ERR_MISALIGNED;
    if (int rc = check_device()) return rc;
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kStagedMaxDevices) return GDN_ERR_NO_DEVICE;
    if (slices > B) slices = static_cast<int>(B);

    std::lock_guard<std::mutex> lock(g_staged_mutex);
    StagedCtx& c = g_staged[d];
    if (!c.ready && staged_ctx_init(c) != cudaSuccess) return GDN_ERR_CUDA;
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    cudaStream_t up = c.s[0], comp = c.s[1], down = c.s[2];
    const size_t qk = static_cast<size_t>(kHQK) * kD * 2, vv = static_cast<size_t>(kHV) * kD * 2,
                 ab = static_cast<size_t>(kHV) * 2, st = static_cast<size_t>(kHV) * kD * kD * 4;
    bool ok = cudaEventRecord(c.start, caller) == cudaSuccess;
    for (int i = 0; i < 3 && ok; ++i) ok = cudaStreamWaitEvent(c.s[i], c.start, 0) == cudaSuccess;
    // the input members of `dev` are this call's destinations (declared const for the plain launch)
    auto up_copy = [&](const void* dst, const void* src, size_t bytes) {
        ok = ok && cudaMemcpyAsync(const_cast<void*>(dst), src, bytes, cudaMemcpyHostToDevice, up) == cudaSuccess;
    };
    auto down_copy = [&](void* dst, const void* src, size_t bytes) {
        ok = ok && cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, down) == cudaSuccess;
    };
    up_copy(dev->q, host->q, B * qk);
    up_copy(dev->k, host->k, B * qk);
    up_copy(dev->v, host->v, B * vv);
    up_copy(dev->a, host->a, B * ab);
    up_copy(dev->b, host->b, B * ab);
    up_copy(dev->A_log, host->A_log, kHV * 4);
    up_copy(dev->dt_bias, host->dt_bias, kHV * 4);
    const char* hs = static_cast<const char*>(static_cast<const void*>(host->state));
    char* hns = reinterpret_cast<char*>(host->new_state);
    char* ds = reinterpret_cast<char*>(dev->new_state);
    for (int i = 0; i < slices && ok; ++i) {
        const int64_t lo = B * i / slices, hi = B * (i + 1) / slices;
        up_copy(ds + lo * st, hs + lo * st, (hi - lo) * st);
        ok = ok && cudaEventRecord(c.in[i], up) == cudaSuccess && cudaStreamWaitEvent(comp, c.in[i], 0) == cudaSuccess;
        DecodeParams p;
        p.q = static_cast<const uint16_t*>(dev->q) + lo * kHQK * kD;
        p.k = static_cast<const uint16_t*>(dev->k) + lo * kHQK * kD;
        p.v = static_cast<const uint16_t*>(dev->v) + lo * kHV * kD;
        p.state = reinterpret_cast<const float*>(ds + lo * st);
        p.A_log = dev->A_log;
        p.a = static_cast<const uint16_t*>(dev->a) + lo * kHV;
        p.dt_bias = dev->dt_bias;
        p.b = static_cast<const uint16_t*>(dev->b) + lo * kHV;
        p.out = static_cast<uint16_t*>(dev->output) + lo * kHV * kD;
        p.new_state = reinterpret_cast<float*>(ds + lo * st);  // in place
        p.batch = hi - lo;
        p.scale = resolve_scale(host->scale);
        p.hqk = kHQK;
        p.hv = kHV;
        ok = ok && launch_decode(p, comp, false, /*pdl=*/false) == cudaSuccess;  // follows an event wait
        ok = ok && cudaEventRecord(c.done[i], comp) == cudaSuccess &&
             cudaStreamWaitEvent(down, c.done[i], 0) == cudaSuccess;
        down_copy(hns + lo * st, ds + lo * st, (hi - lo) * st);
    }
    down_copy(host->output, dev->output, B * vv);
    // the caller's stream resumes after all three streams (also on an error: nothing is left dangling)
    for (int i = 0; i < 3; ++i)
        if (cudaEventRecord(c.end[i], c.s[i]) != cudaSuccess || cudaStreamWaitEvent(caller, c.end[i], 0) != cudaSuccess)
            ok = false;
    return ok ? GDN_OK : GDN_ERR_CUDA;
}
