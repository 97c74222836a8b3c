// Host-side plumbing shared by every entry point: per-thread error
// messages, device binding from a stream or pointer, SM count cache.
#include "common.cuh"

#include <mutex>

namespace fl {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

// The device of the last stream seen on this thread.  Repeated calls on one
// stream (the common case, and every call while that stream is being captured
// into a CUDA graph) make no device query.
static thread_local fl_stream_t t_last_stream = nullptr;
static thread_local int t_last_dev = -1;

// Device of a device (or managed) pointer.
static int pointer_device(const void* ptr, int* dev) {
    cudaPointerAttributes attr;
    FL_CUDA(cudaPointerGetAttributes(&attr, ptr));
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
        set_error("pointer %p is not device memory", ptr);
        return FL_ERR_INVALID_ARGUMENT;
    }
    *dev = attr.device;
    return FL_OK;
}

int bind_device(fl_stream_t stream, const void* ptr) {
    int dev = -1;
    if (stream != nullptr && stream == t_last_stream) {
        dev = t_last_dev;
    } else if (stream != nullptr) {
        // A stream being captured into a CUDA graph refuses cudaStreamGetDevice,
        // and the refusal invalidates the capture; cudaStreamIsCapturing is
        // allowed.  While capturing, the device is the one of the output
        // buffer (every entry point passes one).
        const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        FL_CUDA(cudaStreamIsCapturing(s, &cs));
        if (cs == cudaStreamCaptureStatusNone) {
            FL_CUDA(cudaStreamGetDevice(s, &dev));
        } else if (ptr != nullptr) {
            if (int st = pointer_device(ptr, &dev)) return st;
        } else {
            FL_CUDA(cudaGetDevice(&dev));
        }
        t_last_stream = stream;
        t_last_dev = dev;
    } else if (ptr != nullptr) {
        if (int st = pointer_device(ptr, &dev)) return st;
    } else {
        FL_CUDA(cudaGetDevice(&dev));
    }
    int cur = -1;
    FL_CUDA(cudaGetDevice(&cur));
    if (cur != dev) FL_CUDA(cudaSetDevice(dev));
    return FL_OK;
}

int sm_count() {
    static std::atomic<int> cache[64];  // per device; 0 = not yet known
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kNumSMs;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = kNumSMs;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return FL_ERR_CUDA;
    }
    return FL_OK;
}

// A kernel of this library, for querying the binary the loaded module holds.
__global__ void probe_kernel(int* p) {
    if (p) *p = 0;
}

}  // namespace fl

extern "C" int fl_binary_version(int device, int* version) {
    fl::clear_error();
    FL_REQUIRE(device >= 0 && version, "fl_binary_version: bad arguments");
    FL_CUDA(cudaSetDevice(device));
    cudaFuncAttributes attr;
    FL_CUDA(cudaFuncGetAttributes(&attr, fl::probe_kernel));
    *version = attr.binaryVersion;
    return FL_OK;
}

extern "C" const char* fl_last_error(void) { return fl::g_last_error.c_str(); }

extern "C" int fl_version(void) { return 100; }  // 0.1.0
