// runtime.cpp - status strings, tensor-map cache, per-device launch attributes.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../lc_host.h"

extern "C" const char *lc_status_string(int status) {
    switch (status) {
        case LC_OK: return "ok";
        case LC_ERR_INVALID_ARGUMENT: return "invalid argument";
        case LC_ERR_UNSUPPORTED_HEAD_DIM: return "unsupported head dimension (64 or 128)";
        case LC_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
        case LC_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
        case LC_ERR_MISALIGNED: return "pointer or stride not 16-byte aligned";
        case LC_ERR_CUDA: return "CUDA error";
        case LC_ERR_DEVICE_BOUNDS: return "device saw an out-of-range block or position";
        case LC_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case LC_ERR_OUT_OF_BLOCKS: return "KV cache out of memory blocks";
        case LC_ERR_OUT_OF_MEMORY: return "not enough GPU memory for the KV cache";
        case LC_ERR_NOT_SUPPORTED: return "not supported on this device";
        case LC_ERR_NO_FREE_SLOT: return "every sequence slot of the KV pool is in use";
        default: return "unknown status";
    }
}

extern "C" int lc_status_from_device_word(int word) {
    if (word & LC_DEV_TIMEOUT) return LC_ERR_DEVICE_TIMEOUT;
    if (word & (LC_DEV_BAD_BLOCK | LC_DEV_BAD_POS)) return LC_ERR_DEVICE_BOUNDS;
    return LC_OK;
}

extern "C" const char *lc_version(void) { return "lucciola-b200 0.1 sm_100a"; }

namespace lc {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

struct MapKey {
    const void *ptr;
    int64_t rows;
    int head_dim;
    int device;
    bool operator==(const MapKey &o) const {
        return ptr == o.ptr && rows == o.rows && head_dim == o.head_dim && device == o.device;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31) ^
               (size_t)k.head_dim * 131 ^ (size_t)k.device * 7919;
    }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

}  // namespace

int pool_tensor_map(const void *pool, int64_t rows, int head_dim, CUtensorMap *out) {
    if (!aligned16(pool)) return LC_ERR_MISALIGNED;
    if (rows <= 0 || rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LC_ERR_CUDA;
    MapKey key{pool, rows, head_dim, dev};
    {
        std::lock_guard<std::mutex> lk(g_map_mu);
        auto it = g_maps.find(key);
        if (it != g_maps.end()) {
            *out = it->second;
            return LC_OK;
        }
    }
    auto fn = encode_fn();
    if (!fn) return LC_ERR_NOT_SUPPORTED;
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
    cuuint32_t box[2] = {64, 16};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(pool), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return LC_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_map_mu);
    if (g_maps.size() > 256) g_maps.clear();
    g_maps[key] = map;
    *out = map;
    return LC_OK;
}

int ensure_smem_attr(const void *func, int bytes) {
    static std::mutex mu;
    static std::unordered_map<const void *, std::vector<int>> done;  // per device: bytes set
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LC_ERR_CUDA;
    std::lock_guard<std::mutex> lk(mu);
    auto &v = done[func];
    if ((int)v.size() <= dev) v.resize(dev + 1, 0);
    if (v[dev] >= bytes) return LC_OK;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return LC_ERR_CUDA;
    v[dev] = bytes;
    return LC_OK;
}

int sm_count() {
    static std::mutex mu;
    static std::vector<int> counts;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)counts.size() <= dev) counts.resize(dev + 1, 0);
    if (!counts[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        counts[dev] = n > 0 ? n : 148;
    }
    return counts[dev];
}

}  // namespace lc

namespace lc {

// Same map as pool_tensor_map, encoded on the caller's stack without touching
// the cache (no host allocation). Used by the allocation-free decode entry.
int pool_tensor_map_nocache(const void *pool, int64_t rows, int head_dim, CUtensorMap *out) {
    if (!aligned16(pool)) return LC_ERR_MISALIGNED;
    if (rows <= 0 || rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;
    auto fn = encode_fn();
    if (!fn) return LC_ERR_NOT_SUPPORTED;
    cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
    cuuint32_t box[2] = {64, 16};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(pool), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? LC_OK : LC_ERR_CUDA;
}

}  // namespace lc

namespace lc {
namespace {
std::atomic<int> g_dependent_launch{0};
}
int dependent_launch_mode() { return g_dependent_launch.load(std::memory_order_relaxed); }
}  // namespace lc

extern "C" int lc_set_dependent_launch(int mode) {
    if (mode < 0 || mode > 2) return -1;
    return lc::g_dependent_launch.exchange(mode);
}

namespace lc {

// 2-D bf16 tensor map [rows][inner] (row pitch `row_bytes`), box {box_inner,
// box_rows}, 128-byte swizzle, zero fill out of bounds. Not cached.
int tensor_map_2d_sw128(const void *base, int64_t inner, int64_t rows, int64_t row_bytes,
                        int box_inner, int box_rows, CUtensorMap *out) {
    return tensor_map_2d(base, inner, rows, row_bytes, box_inner, box_rows, 128, out);
}

// The same with a chosen swizzle span: 0 (none), 32, 64 or 128 bytes.
int tensor_map_2d(const void *base, int64_t inner, int64_t rows, int64_t row_bytes, int box_inner,
                  int box_rows, int swizzle_bytes, CUtensorMap *out) {
    const CUtensorMapSwizzle swz = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                         : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (!aligned16(base) || (row_bytes & 15)) return LC_ERR_MISALIGNED;
    if (inner <= 0 || rows <= 0 || rows >= (int64_t(1) << 31)) return LC_ERR_INVALID_ARGUMENT;
    auto fn = encode_fn();
    if (!fn) return LC_ERR_NOT_SUPPORTED;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? LC_OK : LC_ERR_CUDA;
}

}  // namespace lc
