// Shared device/host helpers of the alpaka3_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>

#include "alpaka3_b200.h"
#include "alpaka3_b200_testing.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "alpaka3_b200 is built for sm_100a (B200) only"
#endif

namespace a3b
{
    // ------------------------------------------------------------------------------------------- host errors
    void setError(char const* fmt, ...);
    int cudaFail(cudaError_t e, char const* what);

#define A3B_CUDA(call)                                                                                                \
    do                                                                                                                \
    {                                                                                                                 \
        cudaError_t a3b_e_ = (call);                                                                                  \
        if(a3b_e_ != cudaSuccess)                                                                                     \
            return ::a3b::cudaFail(a3b_e_, #call);                                                                    \
    } while(0)

#define A3B_CHECK_LAUNCH(what)                                                                                        \
    do                                                                                                                \
    {                                                                                                                 \
        cudaError_t a3b_e_ = cudaGetLastError();                                                                      \
        if(a3b_e_ != cudaSuccess)                                                                                     \
            return ::a3b::cudaFail(a3b_e_, what);                                                                     \
    } while(0)

#define A3B_REQUIRE(cond, msg)                                                                                        \
    do                                                                                                                \
    {                                                                                                                 \
        if(!(cond))                                                                                                   \
        {                                                                                                             \
            ::a3b::setError("%s", msg);                                                                               \
            return A3B_ERR_INVALID;                                                                                   \
        }                                                                                                             \
    } while(0)

    // -------------------------------------------------------------------------------- per-device properties
    struct DeviceProps
    {
        int ordinal = -1;
        int smCount = 0;
        int ccMajor = 0;
        int ccMinor = 0;
        size_t l2Bytes = 0;
        unsigned* errWord = nullptr; // device address of this device's error word
    };

    // properties of the current device (cached); returns A3B_OK or an error status
    int currentDevice(DeviceProps const** props);

    // device ordinals the library serves (0 .. kMaxDevices-1)
    constexpr int kMaxDevices = 64;

    // Resident blocks per SM of `kernel` at `threads` threads and no dynamic shared memory, queried once per device
    // and kept in `cache` (kMaxDevices entries indexed by ordinal, 0 = not queried yet). Threads racing on the first
    // query store the same value.
    template<typename Kernel>
    int residentPerSm(DeviceProps const* props, std::atomic<int>* cache, Kernel kernel, int threads, int* out)
    {
        int r = cache[props->ordinal].load(std::memory_order_relaxed);
        if(r == 0)
        {
            int b = 0;
            A3B_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0));
            r = b > 0 ? b : 1;
            cache[props->ordinal].store(r, std::memory_order_relaxed);
        }
        *out = r;
        return A3B_OK;
    }

    // Bounded-wait limit (ns) passed to kernels that spin.
    uint64_t waitTimeoutNs();

    // Scratch cached per (device, stream, slot): at least `bytes`, zero-filled when first allocated or grown.
    // Work ordered on `stream` may use it; each slot belongs to one kernel family, which leaves it in the state its
    // next call expects.
    enum ScratchSlot
    {
        kScratchReduce = 0,
        kScratchScan = 1,
        kScratchEngine = 2, // kernels of the header-only engines (a3b_engine_scratch)
        kScratchSlots = 3
    };
    // With `epoch` non-null, also hands out the next call epoch of this scratch (30 bits, never 0): kernels that tag
    // their scratch words with the epoch need no clearing between calls on the stream.
    int streamScratch(cudaStream_t stream, int slot, size_t bytes, void** ptr, unsigned* epoch = nullptr);
    constexpr unsigned kScratchEpochMask = 0x3FFFFFFFu;


    inline int dtypeSize(int dtype)
    {
        switch(dtype)
        {
        case A3B_I32:
        case A3B_U32:
        case A3B_F32:
            return 4;
        case A3B_I64:
        case A3B_U64:
        case A3B_F64:
            return 8;
        default:
            return 0;
        }
    }

    inline bool aligned16(void const* p)
    {
        return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u;
    }

    // ------------------------------------------------------------------------------------------ peer groups
    // One slot buffer per rank, mapped into every other rank's address space (CUDA IPC over NVLink). Slot
    // [parity][r] holds rank r's 8-byte value and the epoch of the call that wrote it; the parity of the epoch
    // double-buffers consecutive calls (a rank can be at most one call ahead of another).
    constexpr int kMaxPeers = 8;
    constexpr size_t kPeerSlotBytes = 4096;

    struct PeerSlots
    {
        unsigned long long* slots[kMaxPeers]; // rank r's slot buffer, as addressed from this device
        int world;
        int rank;
        unsigned epoch;
    };

} // namespace a3b

struct a3b_peer_group;

namespace a3b
{
    // Slot pointers of a connected group for the current device; advances the group's call epoch.
    int peerSlots(a3b_peer_group* g, PeerSlots* out);

    // ------------------------------------------------------------------------------------------ device side
    constexpr unsigned kErrTimeout = 1u;

    __device__ __forceinline__ uint64_t globalTimerNs()
    {
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        return t;
    }

    __device__ __forceinline__ uint64_t ldRelaxedU64(uint64_t const* p)
    {
        uint64_t v;
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
        return v;
    }

    __device__ __forceinline__ void stRelaxedU64(uint64_t* p, uint64_t v)
    {
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
    }

    __device__ __forceinline__ unsigned long long ldAcquireU64(unsigned long long const* p)
    {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
        return v;
    }

    __device__ __forceinline__ void stReleaseU64(unsigned long long* p, unsigned long long v)
    {
        asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
    }

    __device__ __forceinline__ unsigned ldAcquireU32(unsigned const* p)
    {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        return v;
    }

    __device__ __forceinline__ void stReleaseU32(unsigned* p, unsigned v)
    {
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
    }

    __device__ __forceinline__ unsigned ldRelaxedU32(unsigned const* p)
    {
        unsigned v;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        return v;
    }

    __device__ __forceinline__ void stRelaxedU32(unsigned* p, unsigned v)
    {
        asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
    }

    // streaming 16-byte loads/stores (data touched once: evict-first in L1/L2)
    template<typename V>
    __device__ __forceinline__ V ldStream(V const* p)
    {
        return __ldcs(p);
    }

    template<typename V>
    __device__ __forceinline__ void stStream(V* p, V v)
    {
        __stcs(p, v);
    }

    // ------------------------------------------------------------------------------ TMA bulk copy + mbarrier
    __device__ __forceinline__ uint32_t smemAddr(void const* p)
    {
        return static_cast<uint32_t>(__cvta_generic_to_shared(p));
    }

    __device__ __forceinline__ void mbarInit(uint32_t bar, unsigned count)
    {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
    }

    // global -> shared bulk copy of `bytes`, completing on `bar` (16-byte aligned addresses and size)
    __device__ __forceinline__ void bulkLoad(uint32_t dst, void const* src, unsigned bytes, uint32_t bar)
    {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
             ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
             : "memory");
    }

    // shared -> global bulk copy of `bytes` (16-byte aligned addresses and size), one bulk group
    __device__ __forceinline__ void bulkStore(void* dst, uint32_t src, unsigned bytes)
    {
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
             : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }

    // wait until all but the newest `N` bulk groups have finished reading shared memory
    template<int N>
    __device__ __forceinline__ void bulkWaitRead()
    {
        asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
    }

    __device__ __forceinline__ void bulkWaitAll()
    {
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }

    __device__ __forceinline__ bool mbarTryWait(uint32_t bar, unsigned parity)
    {
        unsigned done;
        asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
        return done != 0u;
    }

    // Bounded wait for the phase with `parity` of `bar`. A copy that never completes (it cannot, short of a
    // fault) is reported in the error word; the wait is then repeated once, so that the block does not leave
    // while the copy may still write its shared memory.
    __device__ inline void mbarWait(uint32_t bar, unsigned parity, uint64_t timeoutNs, unsigned* errWord)
    {
        for(int attempt = 0; attempt < 2; ++attempt)
        {
        uint64_t const t0 = globalTimerNs();
        while(!mbarTryWait(bar, parity))
            if(globalTimerNs() - t0 > timeoutNs)
            break;
        if(mbarTryWait(bar, parity))
            return;
        if(attempt == 0 && (threadIdx.x & 31) == 0)
            atomicOr(errWord, kErrTimeout);
        }
    }

    // ---------------------------------------------------------------------------------------------- Philox
    // Philox4x32-10 (Salmon et al., SC'11): counter (i_lo, i_hi, 0, 0), key (seed_lo, seed_hi)
    __host__ __device__ __forceinline__ uint4 philox4x32_10(uint64_t seed, uint64_t i)
    {
        uint32_t c0 = static_cast<uint32_t>(i), c1 = static_cast<uint32_t>(i >> 32), c2 = 0u, c3 = 0u;
        uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
        for(int r = 0; r < 10; ++r)
        {
            uint64_t const p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
            uint64_t const p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
            uint32_t const n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ k0;
            uint32_t const n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ k1;
            c1 = static_cast<uint32_t>(p1);
            c3 = static_cast<uint32_t>(p0);
            c0 = n0;
            c2 = n2;
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        return make_uint4(c0, c1, c2, c3);
    }
} // namespace a3b
