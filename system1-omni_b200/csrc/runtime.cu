// Runtime part of the C ABI: the CUDA calls a caller needs so that it loads this
// one library and never links CUDA itself (device, memory, streams, graphs,
// copies), the error strings, the fault-status word of the bounded device waits,
// and the host helpers the kernels share (tensor maps, SM count).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "ops_internal.h"
#include "tc.cuh"

namespace s1 {
namespace host {

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            return static_cast<EncodeTiledFn>(nullptr);
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType type, int elem_bytes, uint64_t rows,
                uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}

int make_map_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t mid, uint64_t rows,
                     uint64_t mid_pitch, uint64_t row_pitch, uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[3] = {inner, mid, rows};
    const cuuint64_t strides[2] = {mid_pitch * 2, row_pitch * 2};
    const cuuint32_t box[3] = {box_inner, 1, box_rows};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                          elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}

}  // namespace host

bool pdl_enabled() {
#ifdef S1_TUNING
    // tuning builds only: S1_PDL=0 launches in plain stream order, for A/B timing
    static const bool on = [] {
        const char* e = getenv("S1_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
#else
    return true;
#endif
}

int sm_count() {
    static int sms = 0;
    if (!sms) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) ==
                                                      cudaSuccess && n > 0)
            sms = n;
        else
            sms = 148;
    }
    return sms;
}

namespace host {

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace host
}  // namespace s1

S1_FAULT_WORD(selftest)

namespace {
// One thread waits, through the same bounded wait as the kernels' pipelines, on an
// mbarrier that nothing arrives on; when the wait gives up it records FAULT_WAIT_OTHER in
// this file's fault word and returns. No copy or MMA is in flight, so giving up is safe.
__global__ void wait_selftest_kernel(long long limit) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = s1::tc::smem_u32(&bar);
    s1::tc::mbar_init(b, 1);
    s1::tc::mbar_fence_init();
    if (!s1::tc::mbar_wait_for(b, 0, limit)) atomicOr(&g_fault_word, s1::tc::FAULT_WAIT_OTHER);
}
}  // namespace

extern "C" uint32_t s1_fault_read_gemm(int clear);
extern "C" uint32_t s1_fault_read_gdn(int clear);
extern "C" uint32_t s1_fault_read_gdn_fused(int clear);
extern "C" uint32_t s1_fault_read_attention(int clear);
extern "C" uint32_t s1_fault_read_elementwise(int clear);
extern "C" uint32_t s1_fault_read_norm(int clear);

extern "C" {

uint32_t cs1_abi_version(void) { return CS1_ABI_VERSION; }

const char* cs1_error_string(int code) {
    if (code >= 1000 && code < 2000) return "tensor-core GEMM status";
    return cudaGetErrorString(static_cast<cudaError_t>(code));
}

int cs1_set_device(int device) { return cudaSetDevice(device); }
int cs1_get_device(int* device) { return cudaGetDevice(device); }
int cs1_malloc(void** ptr, size_t bytes) { return cudaMalloc(ptr, bytes); }
int cs1_free(void* ptr) { return cudaFree(ptr); }

int cs1_stream_create(void** stream) {
    return cudaStreamCreateWithFlags(reinterpret_cast<cudaStream_t*>(stream), cudaStreamNonBlocking);
}
int cs1_stream_destroy(void* stream) { return cudaStreamDestroy(static_cast<cudaStream_t>(stream)); }
int cs1_stream_sync(void* stream) { return cudaStreamSynchronize(static_cast<cudaStream_t>(stream)); }

int cs1_upload(void* dst, const void* src, size_t bytes, void* stream) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st);
    return e != cudaSuccess ? e : cudaStreamSynchronize(st);
}

int cs1_download(void* dst, const void* src, size_t bytes, void* stream) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
    return e != cudaSuccess ? e : cudaStreamSynchronize(st);
}

int cs1_copy_dd(void* dst, const void* src, size_t bytes, void* stream) {
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
    return e != cudaSuccess ? e : cudaGetLastError();
}

int cs1_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height, void* stream) {
    const cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault,
                                            static_cast<cudaStream_t>(stream));
    return e != cudaSuccess ? e : cudaGetLastError();
}

int cs1_graph_begin(void* stream) {
    const cudaError_t e = cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e;
}

int cs1_graph_end(void* stream, void** exec) {
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph);
    if (e == cudaSuccess) e = cudaGraphInstantiate(reinterpret_cast<cudaGraphExec_t*>(exec), graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e;
}

int cs1_graph_launch(void* exec, void* stream) {
    const cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e;
}

int cs1_graph_destroy(void* exec) { return cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)); }

// Bit mask of the bounded device waits that gave up since the last clear
// (1 producer, 2 MMA issuer, 4 epilogue, 8 other), OR-ed over the kernel files.
int cs1_wait_selftest(long long cycles, void* stream) {
    if (cycles < 1000 || cycles > 4000000000ll) return cudaErrorInvalidValue;
    wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(cycles);
    return cudaGetLastError();
}

uint32_t cs1_fault_status(int clear) {
    return s1_fault_read_gemm(clear) | s1_fault_read_gdn(clear) | s1_fault_read_gdn_fused(clear) |
           s1_fault_read_attention(clear) | s1_fault_read_elementwise(clear) | s1_fault_read_norm(clear) |
           s1_fault_read_selftest(clear);
}

// ---- vision entry points: required symbols of the loader; the vision path is
// not part of this library, so every call reports cudaErrorNotSupported ----
int cs1_vision_linear(void*, const void*, const void*, const void*, void*, int, int, int, void*) {
    return cudaErrorNotSupported;
}
int cs1_gemm_f32(void*, const float*, const float*, float*, int, int, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_norm(const void*, const void*, const void*, void*, int, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_position(void*, const void*, const int*, const float*, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_rope(const void*, const float*, const float*, void*, void*, int, void*) {
    return cudaErrorNotSupported;
}
int cs1_vision_attention(const void*, const void*, const void*, void*, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_bias(void*, const void*, size_t, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_gelu(void*, size_t, int, void*) { return cudaErrorNotSupported; }
int cs1_vision_add(void*, const void*, size_t, void*) { return cudaErrorNotSupported; }
int cs1_vision_to_float(const void*, float*, size_t, void*) { return cudaErrorNotSupported; }
int cs1_vision_lora_add(void*, const float*, size_t, float, void*) { return cudaErrorNotSupported; }

}  // extern "C"
