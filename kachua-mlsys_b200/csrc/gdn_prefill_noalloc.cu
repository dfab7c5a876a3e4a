// gdn_prefill_noalloc.cu -- prefill for callers that cannot allocate device memory.
//
// Some callers have no way to give this library a workspace: a plugin host or
// inference server that owns every byte of device memory and hands extensions
// no allocator, or a step that must not call cudaMalloc (it can synchronise
// the device, and is not allowed while a stream is being captured).  For them
// gdn_prefill_launch_noalloc runs the same prefill kernels with their scratch
// in a fixed array that lives in this library's device image: every GPU that
// loads the library holds GDN_NOALLOC_SCRATCH_BYTES for it until the process
// exits, and nothing here allocates.
//
// In host code the array's name is only a host-side stand-in; the device
// address is looked up once per device with cudaGetSymbolAddress (with that
// device current) and cached.  That lookup happens inside the first call on
// each device, so make that first call before any stream capture begins.
//
// All calls on a device share the one array and it keeps whatever the last
// call left in it.  The prefill kernels write every scratch word they later
// read within the same call (chunk table, record bases, operand images), so
// nothing has to start at zero.  Two calls whose kernels overlap on the GPU
// (different streams, or several host threads on one device) race on the
// array; serialise them.
#include <mutex>

namespace gdn {

constexpr size_t kNoAllocScratchBytes = GDN_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static void* g_noalloc_ptr[kNoAllocMaxDevices];
static std::mutex g_noalloc_mutex;

// Device address of this device's scratch array (looked up once per device).
static int noalloc_scratch(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return GDN_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return GDN_ERR_CUDA;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return GDN_OK;
}

}  // namespace gdn

extern "C" int gdn_prefill_launch_noalloc(const GdnPrefillArgs* args, void* stream) {
    if (args == nullptr) return GDN_ERR_NULL_POINTER;
    if (args->total_tokens < 0 || args->num_seqs < 0) return GDN_ERR_BAD_SIZE;
    // The token-recurrent path (asked for, or chosen by AUTO for short mean
    // lengths) needs no scratch; the chunked paths need at least their operand
    // records in the array.  The segmented carry also needs its summaries and
    // runs only when gdn_prefill_workspace_size(T, N) fits as a whole.
    if (!gdn::prefill_path_is_recurrent(args->path, args->total_tokens, args->num_seqs) &&
        gdn::chunked_workspace_min_bytes(args->total_tokens, args->num_seqs) > gdn::kNoAllocScratchBytes)
        return GDN_ERR_WORKSPACE;
    void* scratch = nullptr;
    if (int rc = gdn::noalloc_scratch(&scratch)) return rc;
    return gdn_prefill_launch(args, scratch, gdn::kNoAllocScratchBytes, stream);
}
