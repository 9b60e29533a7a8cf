// cs1_gdn_prefill_noalloc: the chunked Gated DeltaNet prefill of cs1_gdn_prefill with its
// workspace in a fixed device array owned by this library, for callers that cannot
// allocate device memory.
//
// Who needs it: hosts that may not call cudaMalloc (or any allocating routine) on the
// path where they run the prefill -- for example code that runs inside a stream-ordered
// region owned by another framework's allocator, a real-time path that forbids
// allocation after start-up, or a sandboxed plugin whose memory budget is fixed by its
// host -- and so cannot provide the caller-owned workspace that cs1_gdn_prefill takes.
//
// The scratch is a file-scope device array of kScratchBytes (64 MiB, plus alignment
// slack); every GPU that loads the library holds it until the process exits. In host
// code the array's name is only a host-side stand-in, so the device address comes from
// cudaGetSymbolAddress, once per device, with that device current, on the first call
// on that device (that first call should therefore come before any stream capture).
// The address is kept for the life of the process: a cudaDeviceReset of a device while
// this library is loaded leaves it stale, so a process that resets a device must not call
// this entry point on it again.
#include <mutex>

#include "gdn.cuh"

namespace {

constexpr size_t kScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

// 1024 extra bytes so the 1024-byte aligned workspace fits after rounding the start up.
static __device__ __align__(256) unsigned char g_gdn_scratch[kScratchBytes + 1024];

std::mutex g_setup_lock;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_lock);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gdn_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int cs1_gdn_prefill_noalloc(const void* q, const void* k,
                                                                             const void* v, const float* g,
                                                                             const void* beta, void* o, int T, int H,
                                                                             int HK, float scale, void* stream) {
    if (T < 0 || HK <= 0 || H <= 0 || H % HK != 0) return cudaErrorInvalidValue;
    if (T == 0) return cudaSuccess;
    const size_t need = s1::gdn::workspace_bytes_for((T + 63) / 64, H, false);
    if (need > kScratchBytes) return cudaErrorInvalidValue;  // beyond the fixed scratch: use cs1_gdn_prefill
    void* base = nullptr;
    const cudaError_t e = scratch_address(&base);
    if (e != cudaSuccess) return e;
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    void* ws = reinterpret_cast<void*>((a + 1023) & ~static_cast<uintptr_t>(1023));
    s1::SeqTable tab;
    const size_t len = static_cast<size_t>(T);
    s1::make_table(tab, &len, 1);
    // Every workspace byte the scan reads is written by the prep kernel of the same call,
    // so nothing needs clearing between calls.
    return s1::gdn::run_two_pass(q, k, v, g, beta, o, ws, kScratchBytes, tab, H, HK, scale, nullptr, 0, nullptr,
                        static_cast<cudaStream_t>(stream));
}
