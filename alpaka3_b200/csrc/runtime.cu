// Runtime services of the C ABI: error reporting, device properties, stream-ordered memory, cached scratch,
// device-side error word. Replaces the CUDA queue/device plumbing of alpaka3's unifiedCudaHip backend
// (include/alpaka/api/unifiedCudaHip/Queue.hpp:43-185, Device.hpp:205-325) for the primitive path.
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "common.cuh"

namespace a3b
{
    // device-side error word (one instance per device); kernels receive its address as an argument
    __device__ unsigned g_deviceError = 0u;

    namespace
    {
        thread_local std::string tlsError;
        std::atomic<uint64_t> gTimeoutNs{1000000000ull};

        std::mutex gPropsMutex;
        DeviceProps gProps[kMaxDevices];

        struct Scratch
        {
            void* ptr = nullptr;
            size_t bytes = 0;
            unsigned epoch = 0; // last epoch handed out for this scratch (calls on one stream are ordered)
        };

        std::mutex gScratchMutex;
        std::map<std::tuple<int, cudaStream_t, int>, Scratch> gScratch;
    } // namespace

    void setError(char const* fmt, ...)
    {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        tlsError = buf;
    }

    int cudaFail(cudaError_t e, char const* what)
    {
        setError("%s failed: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
        return e == cudaErrorMemoryAllocation ? A3B_ERR_NOMEM : A3B_ERR_CUDA;
    }

    int currentDevice(DeviceProps const** props)
    {
        int dev = 0;
        A3B_CUDA(cudaGetDevice(&dev));
        if(dev < 0 || dev >= kMaxDevices)
        {
            setError("device ordinal %d out of range", dev);
            return A3B_ERR_UNSUPPORTED;
        }
        std::lock_guard<std::mutex> lock(gPropsMutex);
        DeviceProps& p = gProps[dev];
        if(p.ordinal < 0)
        {
            A3B_CUDA(cudaDeviceGetAttribute(&p.smCount, cudaDevAttrMultiProcessorCount, dev));
            A3B_CUDA(cudaDeviceGetAttribute(&p.ccMajor, cudaDevAttrComputeCapabilityMajor, dev));
            A3B_CUDA(cudaDeviceGetAttribute(&p.ccMinor, cudaDevAttrComputeCapabilityMinor, dev));
            int l2 = 0;
            A3B_CUDA(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
            p.l2Bytes = static_cast<size_t>(l2);
            if(p.ccMajor != 10 || p.ccMinor != 0)
            {
                setError("device %d has compute capability %d.%d; this library is built for sm_100a only", dev,
                         p.ccMajor, p.ccMinor);
                return A3B_ERR_UNSUPPORTED;
            }
            void* ew = nullptr;
            A3B_CUDA(cudaGetSymbolAddress(&ew, g_deviceError));
            p.errWord = static_cast<unsigned*>(ew);
            p.ordinal = dev;
        }
        *props = &p;
        return A3B_OK;
    }

    uint64_t waitTimeoutNs()
    {
        return gTimeoutNs.load(std::memory_order_relaxed);
    }

    int streamScratch(cudaStream_t stream, int slot, size_t bytes, void** ptr, unsigned* epoch)
    {
        int dev = 0;
        A3B_CUDA(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(gScratchMutex);
        Scratch& s = gScratch[std::make_tuple(dev, stream, slot)];
        if(s.bytes < bytes)
        {
            // grow geometrically; the old block is released in stream order after the work that used it
            size_t want = s.bytes * 2 > bytes ? s.bytes * 2 : bytes;
            want = (want + 4095u) & ~size_t{4095u};
            void* p = nullptr;
            A3B_CUDA(cudaMallocAsync(&p, want, stream));
            cudaError_t e = cudaMemsetAsync(p, 0, want, stream);
            if(e != cudaSuccess)
            {
                cudaFreeAsync(p, stream);
                return cudaFail(e, "cudaMemsetAsync(scratch)");
            }
            if(s.ptr)
                A3B_CUDA(cudaFreeAsync(s.ptr, stream));
            s.ptr = p;
            s.bytes = want;
        }
        *ptr = s.ptr;
        if(epoch)
        {
            s.epoch = (s.epoch + 1u) & kScratchEpochMask;
            if(s.epoch == 0u)
                s.epoch = 1u;
            *epoch = s.epoch;
        }
        return A3B_OK;
    }

} // namespace a3b

using namespace a3b;

extern "C"
{
    int a3b_version(void)
    {
        return A3B_VERSION;
    }

    char const* a3b_last_error(void)
    {
        return tlsError.c_str();
    }

    int a3b_engine_scratch(a3b_stream_t stream, size_t bytes, void** ptr)
    {
        A3B_REQUIRE(ptr, "ptr is null");
        return streamScratch(static_cast<cudaStream_t>(stream), kScratchEngine, bytes > 0 ? bytes : 1, ptr);
    }

    int a3b_device_count(int* count)
    {
        A3B_REQUIRE(count, "count is null");
        *count = 0;
        cudaError_t e = cudaGetDeviceCount(count);
        if(e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
        {
            cudaGetLastError();
            *count = 0;
            return A3B_OK;
        }
        A3B_CUDA(e);
        return A3B_OK;
    }

    int a3b_device_info_get(int ordinal, a3b_device_info* info)
    {
        A3B_REQUIRE(info, "info is null");
        cudaDeviceProp p{};
        A3B_CUDA(cudaGetDeviceProperties(&p, ordinal));
        std::memset(info, 0, sizeof(*info));
        info->ordinal = ordinal;
        info->sm_count = p.multiProcessorCount;
        info->cc_major = p.major;
        info->cc_minor = p.minor;
        info->global_mem_bytes = p.totalGlobalMem;
        info->l2_bytes = static_cast<uint64_t>(p.l2CacheSize);
        info->max_threads_per_block = p.maxThreadsPerBlock;
        info->warp_size = p.warpSize;
        std::strncpy(info->name, p.name, sizeof(info->name) - 1);
        return A3B_OK;
    }

    int a3b_malloc_async(void** ptr, size_t bytes, a3b_stream_t stream)
    {
        A3B_REQUIRE(ptr, "ptr is null");
        *ptr = nullptr;
        if(bytes == 0)
            return A3B_OK;
        A3B_CUDA(cudaMallocAsync(ptr, bytes, static_cast<cudaStream_t>(stream)));
        return A3B_OK;
    }

    int a3b_free_async(void* ptr, a3b_stream_t stream)
    {
        if(ptr)
            A3B_CUDA(cudaFreeAsync(ptr, static_cast<cudaStream_t>(stream)));
        return A3B_OK;
    }

    int a3b_memcpy_async(void* dst, void const* src, size_t bytes, a3b_stream_t stream)
    {
        if(bytes == 0)
            return A3B_OK;
        A3B_REQUIRE(dst && src, "null pointer in memcpy");
        A3B_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
        return A3B_OK;
    }

    int a3b_stream_synchronize(a3b_stream_t stream)
    {
        A3B_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
        return A3B_OK;
    }

    int a3b_get_device_error(a3b_stream_t stream, uint32_t* error_bits, int clear)
    {
        A3B_REQUIRE(error_bits, "error_bits is null");
        auto s = static_cast<cudaStream_t>(stream);
        unsigned v = 0;
        A3B_CUDA(cudaMemcpyFromSymbolAsync(&v, g_deviceError, sizeof(v), 0, cudaMemcpyDeviceToHost, s));
        A3B_CUDA(cudaStreamSynchronize(s));
        *error_bits = v;
        if(clear && v != 0u)
        {
            unsigned const zero = 0u;
            A3B_CUDA(cudaMemcpyToSymbolAsync(g_deviceError, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s));
            A3B_CUDA(cudaStreamSynchronize(s));
        }
        return A3B_OK;
    }

    int a3b_set_wait_timeout_ns(uint64_t ns)
    {
        A3B_REQUIRE(ns > 0, "timeout must be positive");
        gTimeoutNs.store(ns, std::memory_order_relaxed);
        return A3B_OK;
    }
}
