// umsx_route_static: the router without a handle and without any allocation.
//
// Some callers cannot allocate device memory at all: an operator running inside a
// host framework that plans every buffer up front and hands each op only its own
// tensors (a ggml-style backend op is the example), or a process with a fixed
// device-memory budget that is already spent.  They cannot create a umsx_moe
// handle, whose workspace is a cudaMalloc.  This entry point runs the same
// router kernel as umsx_route, but all of the kernel's scratch lives in the
// fixed array below, which every GPU that loads this library holds until exit.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "umsx_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = 512 * 1024;
constexpr int kStaticMaxTokens = 64, kStaticMaxExperts = 256, kStaticMaxTopK = 8, kStaticMaxHidden = 4096;
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name stands in for the array and is NOT a
// device address; the host obtains the device address once per device below.
static __device__ __align__(256) unsigned char g_route_scratch[kStaticScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};

umsx_status fail(umsx_status s, const std::string &msg) {
    umsx::record_error(msg.c_str());  // read back through umsx_last_error()
    return s;
}

// Carves the router's scratch out of `base` (nullptr: only measures).
size_t carve(unsigned char *base, int tokens, int experts, int top_k, int hidden, int32_t *counts_out,
             umsx::Dispatch &d, size_t *zero_bytes) {
    size_t used = 0;
    auto take = [&](size_t bytes) {
        unsigned char *p = base ? base + used : nullptr;
        used = (used + bytes + 255) / 256 * 256;
        return p;
    };
    const size_t T = tokens, E = experts, K = top_k, H = hidden;
    // the counters that must read zero when the kernel starts come first
    d.token_done = reinterpret_cast<uint32_t *>(take(T * 4));
    d.all_done = reinterpret_cast<uint32_t *>(take(4));
    *zero_bytes = used;
    d.logits = reinterpret_cast<float *>(take(T * E * 4));
    d.counts = counts_out ? counts_out : reinterpret_cast<int32_t *>(take(E * 4));
    d.offsets = reinterpret_cast<int32_t *>(take((E + 1) * 4));
    d.active = reinterpret_cast<int32_t *>(take(E * 4));
    d.n_active = reinterpret_cast<int32_t *>(take(4));
    d.slots = reinterpret_cast<int4 *>(take(E * sizeof(int4)));
    d.job_token = reinterpret_cast<int32_t *>(take(T * K * 4));
    d.job_rank = reinterpret_cast<int32_t *>(take(T * K * 4));
    d.xq_codes = reinterpret_cast<uint8_t *>(take(T * H));
    d.xq_scales = reinterpret_cast<float *>(take(T * (H / 32) * 4));
    d.tile_done = nullptr;
    return used;
}

// Device address of the scratch on the current device; looked up on the first call per device.
umsx_status scratch_address(unsigned char **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(UMSX_EDEVICE, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(UMSX_EUNSUPPORTED, "device index beyond the static scratch table");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p)
            return fail(UMSX_EDEVICE, std::string("cudaGetSymbolAddress(route scratch): ") + cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<unsigned char *>(g_scratch_addr[dev]);
    return UMSX_OK;
}

}  // namespace

extern "C" {

umsx_status umsx_route_static(const void *x, int x_dtype, int tokens, const float *router_w, const float *router_b,
                              int hidden, int experts, int top_k, int routing, float routed_scale, int32_t *ids,
                              float *weights, int32_t *counts, umsx_stream stream) {
    if (!x || !router_w || !ids || !weights) return fail(UMSX_EINVAL, "null argument");
    if (x_dtype != UMSX_DTYPE_F32 && x_dtype != UMSX_DTYPE_BF16) return fail(UMSX_EINVAL, "x_dtype must be F32 or BF16");
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail(UMSX_EINVAL, "x must be 16-byte aligned");
    if (routing < 0 || routing > 2) return fail(UMSX_EINVAL, "unknown routing mode");
    if (tokens < 1 || tokens > kStaticMaxTokens || experts < 1 || experts > kStaticMaxExperts || top_k < 1 ||
        top_k > kStaticMaxTopK || top_k > experts || hidden < 64 || hidden > kStaticMaxHidden || hidden % 64)
        return fail(UMSX_EINVAL, "umsx_route_static supports tokens <= 64, experts <= 256, top_k <= min(8, experts), "
                                 "hidden a multiple of 64 up to 4096 (its scratch is a fixed 512 KiB array)");
    umsx::Dispatch d{};
    size_t zero_bytes = 0;
    const size_t need = carve(nullptr, tokens, experts, top_k, hidden, counts, d, &zero_bytes);
    if (need > kStaticScratchBytes)
        return fail(UMSX_EINVAL, "request needs " + std::to_string(need) + " scratch bytes; the static array holds " +
                                     std::to_string(kStaticScratchBytes));
    unsigned char *base = nullptr;
    if (umsx_status st = scratch_address(&base)) return st;
    carve(base, tokens, experts, top_k, hidden, counts, d, &zero_bytes);
    d.ids = ids;
    d.weights = weights;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // every call shares the array: the completion counters must start at zero
    cudaError_t e = cudaMemsetAsync(base, 0, zero_bytes, s);
    if (e != cudaSuccess) return fail(UMSX_EDEVICE, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    umsx::RouterParams p{};
    p.x = x;
    p.x_dtype = x_dtype;
    p.tokens = tokens;
    p.hidden = hidden;
    p.experts = experts;
    p.top_k = top_k;
    p.routing = routing;
    p.routed_scale = routed_scale;
    p.w = router_w;
    p.b = router_b;
    p.e_lo = 0;
    p.e_local = experts;
    umsx::record_launches((uint64_t)umsx::launch_router(p, d, s));
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(UMSX_EDEVICE, std::string("router launch: ") + cudaGetErrorString(e));
    return UMSX_OK;
}

}  // extern "C"
