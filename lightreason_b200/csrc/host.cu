// Status reporting, device checks and host-memory mapping for the C ABI.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace lrb {

namespace {
thread_local char g_error[512] = "";
}

int set_error(int status, const char *fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_error, sizeof g_error, fmt, args);
    va_end(args);
    return status;
}

int cuda_error(cudaError_t err, const char *where) {
    return set_error(MOE_ECUDA, "%s: %s (%s)", where, cudaGetErrorName(err), cudaGetErrorString(err));
}

int check_launch(const char *where) {
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? MOE_OK : cuda_error(err, where);
}

cudaStream_t side_stream() {
    static std::mutex mu;
    static cudaStream_t streams[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!streams[device]) {
        // not a stream operation: allowed while a stream of this thread captures
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        if (cudaStreamCreateWithFlags(&streams[device], cudaStreamNonBlocking) != cudaSuccess) streams[device] = nullptr;
        cudaThreadExchangeStreamCaptureMode(&mode);
    }
    return streams[device];
}

int sm_count() {
    static int cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    if (!cached[device]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        cached[device] = n > 0 ? n : 148;
    }
    return cached[device];
}

int smem_optin() {
    static int cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 0;
    if (!cached[device]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess) return 0;
        cached[device] = v;
    }
    return cached[device];
}

int ensure_dynamic_smem(const void *kernel, int bytes, const char *name) {
    struct Entry {
        const void *kernel;
        int device;
        int bytes;
    };
    static std::mutex mu;
    static std::vector<Entry> done;
    int device = 0;
    LRB_CUDA(cudaGetDevice(&device));
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry &e : done)
        if (e.kernel == kernel && e.device == device && e.bytes >= bytes) return MOE_OK;
    const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err != cudaSuccess) return cuda_error(err, name);
    done.push_back({kernel, device, bytes});
    return MOE_OK;
}

int require_sm100() {
    int device = 0;
    LRB_CUDA(cudaGetDevice(&device));
    return moe_device_check(device);
}

}  // namespace lrb

extern "C" {

int moe_version(void) { return 100; }

const char *moe_last_error(void) { return lrb::g_error; }

int moe_device_check(int device) {
    int major = 0, minor = 0;
    LRB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    LRB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0)
        return lrb::set_error(MOE_EARCH, "device %d is sm_%d%d; this library is built for sm_100a", device,
                              major, minor);
    return MOE_OK;
}

int moe_host_register(void *ptr, size_t bytes, uint64_t *device_ptr) {
    LRB_REQUIRE(ptr != nullptr && bytes > 0 && device_ptr != nullptr, "moe_host_register: null or empty range");
    LRB_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
    void *dev = nullptr;
    cudaError_t err = cudaHostGetDevicePointer(&dev, ptr, 0);
    if (err != cudaSuccess) {
        cudaHostUnregister(ptr);
        return lrb::cuda_error(err, "cudaHostGetDevicePointer");
    }
    *device_ptr = reinterpret_cast<uint64_t>(dev);
    return MOE_OK;
}

int moe_host_unregister(void *ptr) {
    LRB_REQUIRE(ptr != nullptr, "moe_host_unregister: null pointer");
    LRB_CUDA(cudaHostUnregister(ptr));
    return MOE_OK;
}

}  // extern "C"
