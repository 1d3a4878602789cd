// Peer groups: the ranks of one node (one process per GPU) map each other's slot buffers through CUDA IPC, so that a
// kernel can store a value into every peer's memory over NVLink and read its own slots. Used by the fused
// reduce + all-reduce (a3b_transform_reduce_allranks). alpaka3 has no multi-device layer; this is new.
#include <cstring>

#include "common.cuh"

struct a3b_peer_group
{
    int device = -1;
    int world = 0;
    int rank = 0;
    void* local = nullptr;                      // this rank's slot buffer (cudaMalloc, zero-filled)
    void* mapped[a3b::kMaxPeers] = {};          // other ranks' slot buffers mapped into this process
    unsigned epoch = 0;                         // calls made so far (same sequence on every rank)
    bool connected = false;
};

namespace a3b
{
    int peerSlots(a3b_peer_group* g, PeerSlots* out)
    {
        A3B_REQUIRE(g && g->connected, "peer group not connected");
        int dev = -1;
        A3B_CUDA(cudaGetDevice(&dev));
        A3B_REQUIRE(dev == g->device, "peer group used on a different device than the one it was created on");
        std::memset(out, 0, sizeof(*out));
        for(int r = 0; r < g->world; ++r)
            out->slots[r] = static_cast<unsigned long long*>(r == g->rank ? g->local : g->mapped[r]);
        out->world = g->world;
        out->rank = g->rank;
        g->epoch = (g->epoch + 1u) & 0x7FFFFFFFu;
        if(g->epoch == 0u)
            g->epoch = 1u;
        out->epoch = g->epoch;
        return A3B_OK;
    }
} // namespace a3b

using namespace a3b;

extern "C"
{
    size_t a3b_ipc_handle_size(void)
    {
        return sizeof(cudaIpcMemHandle_t);
    }

    int a3b_peer_group_create(int world, int rank, a3b_peer_group** group, void* local_handle)
    {
        A3B_REQUIRE(group && local_handle, "null argument");
        A3B_REQUIRE(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "world/rank out of range");
        auto* g = new a3b_peer_group{};
        g->world = world;
        g->rank = rank;
        cudaError_t e = cudaGetDevice(&g->device);
        if(e == cudaSuccess)
            e = cudaMalloc(&g->local, kPeerSlotBytes);
        if(e == cudaSuccess)
            e = cudaMemset(g->local, 0, kPeerSlotBytes);
        cudaIpcMemHandle_t h{};
        if(e == cudaSuccess)
            e = cudaIpcGetMemHandle(&h, g->local);
        if(e != cudaSuccess)
        {
            if(g->local)
                cudaFree(g->local);
            delete g;
            return cudaFail(e, "a3b_peer_group_create");
        }
        std::memcpy(local_handle, &h, sizeof(h));
        *group = g;
        return A3B_OK;
    }

    int a3b_peer_group_connect(a3b_peer_group* g, void const* handles)
    {
        A3B_REQUIRE(g && handles, "null argument");
        A3B_REQUIRE(!g->connected, "peer group already connected");
        auto const* hs = static_cast<cudaIpcMemHandle_t const*>(handles);
        for(int r = 0; r < g->world; ++r)
        {
            if(r == g->rank)
                continue;
            cudaError_t const e = cudaIpcOpenMemHandle(&g->mapped[r], hs[r], cudaIpcMemLazyEnablePeerAccess);
            if(e != cudaSuccess)
            {
                for(int q = 0; q < r; ++q)
                    if(g->mapped[q])
                    {
                        cudaIpcCloseMemHandle(g->mapped[q]);
                        g->mapped[q] = nullptr;
                    }
                return cudaFail(e, "cudaIpcOpenMemHandle (peer slot buffer)");
            }
        }
        g->connected = true;
        return A3B_OK;
    }

    int a3b_peer_group_destroy(a3b_peer_group* g)
    {
        if(!g)
            return A3B_OK;
        int rc = A3B_OK;
        for(int r = 0; r < kMaxPeers; ++r)
            if(g->mapped[r] && cudaIpcCloseMemHandle(g->mapped[r]) != cudaSuccess)
                rc = A3B_ERR_CUDA;
        if(g->local && cudaFree(g->local) != cudaSuccess)
            rc = A3B_ERR_CUDA;
        delete g;
        if(rc)
            setError("a3b_peer_group_destroy: releasing a mapping or the slot buffer failed");
        return rc;
    }
}
