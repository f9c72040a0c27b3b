// peer.cu - exchange regions for the KV-head-sharded decode, and the
// device-side wait that completes it.
//
// Each rank of a group owns one region of device memory (cudaMalloc, so that
// it can be exported with an IPC handle) and maps every peer's region into its
// process. lc_rope_append_decode_peer stores each finished output row into
// all ranks' regions and, when its grid is done, raises this rank's signal
// word in every peer's region; lc_peer_wait polls the peers' words in this
// rank's region. Only plain loads and stores cross NVLink: no TMA and no
// multicast object touch peer memory.
#include <stdint.h>
#include <string.h>

#include <new>

#include "lc_common.cuh"
#include "lc_host.h"

namespace lc {
namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == LC_PEER_HANDLE_BYTES, "IPC handle size");

__device__ __forceinline__ int ld_acquire_sys(const int *a) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// One warp. Lane r < world (r != rank) polls rank r's signal word until it
// reaches this rank's wait count + 1, for at most kWaitLimitNs; lane 0 then
// advances the wait count. The launch counts only grow, so a peer that is
// already further ahead also satisfies the wait (it is at most one launch
// ahead: its next peer decode stores only after its own wait for this rank).
__global__ void peer_wait_kernel(const int *flags, int world, int rank, int *wait_count,
                                 int *status) {
    // Let the next decode start streaming its pages; it stores outputs only
    // after this grid has finished.
    griddep_launch_dependents();
    griddep_wait();  // this rank's own peer decode has finished
    const int lane = threadIdx.x;
    const int want = *wait_count + 1;
    if (lane < world && lane != rank) {
        if ((int)((unsigned)ld_acquire_sys(flags + lane) - (unsigned)want) < 0) {
            const uint64_t t0 = global_timer_ns();
            for (uint32_t it = 1;; ++it) {
                if ((int)((unsigned)ld_acquire_sys(flags + lane) - (unsigned)want) >= 0) break;
                if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
                    set_status(status, LC_DEV_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncwarp();
    if (lane == 0) *wait_count = want;
}

int make_group(int rank, int world, uint8_t *const *regions, const bool *opened, size_t bytes,
               lc_peer_group **out) {
    lc_peer_group *g = new (std::nothrow) lc_peer_group;
    if (!g) return LC_ERR_OUT_OF_MEMORY;
    memset(g, 0, sizeof(*g));
    g->rank = rank;
    g->world = world;
    g->bytes = bytes;
    for (int r = 0; r < world; ++r) {
        g->region[r] = regions[r];
        g->opened[r] = opened[r];
    }
    *out = g;
    return LC_OK;
}

// Bytes from `p` to the end of the device allocation that holds it
// (cuMemGetAddressRange, through the runtime's driver entry point); 0 when the
// driver knows no allocation there; SIZE_MAX when there is no driver to ask
// (then no kernel can run either, so no store can overrun). Every region of a
// group must have room for region_bytes: the decode writes the same offsets
// into every peer's region.
size_t room_after(const void *p) {
    using RangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
    static RangeFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            f = nullptr;
        }
        return reinterpret_cast<RangeFn>(f);
    }();
    if (!p) return 0;
    if (!fn) return SIZE_MAX;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)(uintptr_t)p) != CUDA_SUCCESS) return 0;
    const size_t off = (size_t)((uintptr_t)p - (uintptr_t)base);
    return off < size ? size - off : 0;
}

bool group_args_ok(int rank, int world, size_t bytes, lc_peer_group **out) {
    return out && world >= 1 && world <= LC_PEER_MAX_RANKS && rank >= 0 && rank < world &&
           bytes > LC_PEER_SIGNAL_BYTES;
}

}  // namespace
}  // namespace lc

using namespace lc;

extern "C" int lc_peer_region_alloc(size_t bytes, void **region, void *handle_out) {
    if (!region || !handle_out || bytes <= LC_PEER_SIGNAL_BYTES) return LC_ERR_INVALID_ARGUMENT;
    *region = nullptr;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return LC_ERR_CUDA;
    }
    memcpy(handle_out, &h, sizeof(h));
    *region = p;
    return LC_OK;
}

extern "C" int lc_peer_region_free(void *region) {
    if (!region) return LC_OK;
    return cudaFree(region) == cudaSuccess ? LC_OK : LC_ERR_CUDA;
}

extern "C" int lc_peer_group_open(int rank, int world, void *region, size_t region_bytes,
                                  const void *handles, lc_peer_group **out) {
    if (!group_args_ok(rank, world, region_bytes, out) || !region || !handles)
        return LC_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (room_after(region) < region_bytes) return LC_ERR_INVALID_ARGUMENT;
    uint8_t *regions[LC_PEER_MAX_RANKS] = {};
    bool opened[LC_PEER_MAX_RANKS] = {};
    int rc = LC_OK;
    for (int r = 0; r < world; ++r) {
        if (r == rank) {
            regions[r] = (uint8_t *)region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + (size_t)r * LC_PEER_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            rc = LC_ERR_CUDA;
            break;
        }
        regions[r] = (uint8_t *)p;
        opened[r] = true;
        if (room_after(p) < region_bytes) {  // a peer allocated a smaller region
            rc = LC_ERR_INVALID_ARGUMENT;
            break;
        }
    }
    if (rc == LC_OK) rc = make_group(rank, world, regions, opened, region_bytes, out);
    if (rc != LC_OK)
        for (int r = 0; r < world; ++r)
            if (opened[r]) cudaIpcCloseMemHandle(regions[r]);
    return rc;
}

extern "C" int lc_peer_group_local(int rank, int world, void *const *regions,
                                   size_t region_bytes, lc_peer_group **out) {
    if (!group_args_ok(rank, world, region_bytes, out) || !regions) return LC_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    uint8_t *rs[LC_PEER_MAX_RANKS] = {};
    bool opened[LC_PEER_MAX_RANKS] = {};
    for (int r = 0; r < world; ++r) {
        if (!regions[r] || room_after(regions[r]) < region_bytes) return LC_ERR_INVALID_ARGUMENT;
        rs[r] = (uint8_t *)regions[r];
    }
    return make_group(rank, world, rs, opened, region_bytes, out);
}

extern "C" void lc_peer_group_destroy(lc_peer_group *g) {
    if (!g) return;
    for (int r = 0; r < g->world; ++r)
        if (g->opened[r]) cudaIpcCloseMemHandle(g->region[r]);
    delete g;
}

extern "C" int lc_peer_wait(const lc_peer_group *g, int *dev_status, lc_stream_t stream) {
    if (!g) return LC_ERR_INVALID_ARGUMENT;
    uint8_t *mine = g->region[g->rank];
    const int *flags = (const int *)mine;
    int *wait_count = (int *)mine + kPeerWaitWord;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent_launch_mode() > 0 ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, peer_wait_kernel, flags, g->world, g->rank, wait_count,
                           dev_status) != cudaSuccess) {
        cudaGetLastError();
        return LC_ERR_CUDA;
    }
    return LC_OK;
}
