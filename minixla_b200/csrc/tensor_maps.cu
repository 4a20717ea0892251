// Encoded TMA tensor maps, cached per process.
//
// cuTensorMapEncodeTiled is a pure function of its arguments (global address,
// data type, dimensions, strides, box, swizzle, L2 promotion): the same
// arguments give the same 128-byte descriptor.  Every launch encodes two to
// eleven of them, for operands that a caller usually passes again and again
// (the same weights, the same buffers of a serving loop), so the descriptors
// are kept in a small table keyed by every argument and copied out on a hit;
// a pointer freed and reused with another shape simply misses.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "internal.h"

namespace mxb {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

struct MapKey {
    uint64_t base;
    uint32_t dtype, rank, swizzle, l2;
    uint64_t dims[3];
    uint64_t strides[2];
    uint32_t box[3];
    uint32_t pad;
};

struct MapEntry {
    MapKey key;
    CUtensorMap map;
    uint64_t used;
    bool valid;
};

constexpr int kMapCacheEntries = 64;
std::mutex g_map_mu;
MapEntry g_maps[kMapCacheEntries];
uint64_t g_map_clock = 0;

bool cache_enabled() {
    static const bool on = [] {
        const char* v = getenv("MINIXLA_TMAP_CACHE");
        return !(v && v[0] == '0');
    }();
    return on;
}

}  // namespace

bool encode_tensor_map(CUtensorMap* map, int dtype, int rank, const void* base, const unsigned long long* dims,
                       const unsigned long long* strides, const unsigned* box, int swizzle, int l2_promotion) {
    if (rank < 1 || rank > 3) return false;
    MapKey k;
    memset(&k, 0, sizeof(k));
    k.base = reinterpret_cast<uint64_t>(base);
    k.dtype = static_cast<uint32_t>(dtype);
    k.rank = static_cast<uint32_t>(rank);
    k.swizzle = static_cast<uint32_t>(swizzle);
    k.l2 = static_cast<uint32_t>(l2_promotion);
    for (int i = 0; i < rank; ++i) {
        k.dims[i] = dims[i];
        k.box[i] = box[i];
        if (i + 1 < rank) k.strides[i] = strides[i];
    }
    const bool cached = cache_enabled();
    if (cached) {
        std::lock_guard<std::mutex> lock(g_map_mu);
        for (MapEntry& e : g_maps) {
            if (e.valid && memcmp(&e.key, &k, sizeof(k)) == 0) {
                *map = e.map;
                e.used = ++g_map_clock;
                return true;
            }
        }
    }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t d[3], st[2];
    cuuint32_t bx[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = k.dims[i];
        bx[i] = k.box[i];
        if (i + 1 < rank) st[i] = k.strides[i];
    }
    const CUresult r = enc(map, static_cast<CUtensorMapDataType>(dtype), static_cast<cuuint32_t>(rank),
                           const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           static_cast<CUtensorMapSwizzle>(swizzle), static_cast<CUtensorMapL2promotion>(l2_promotion),
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    if (cached) {
        std::lock_guard<std::mutex> lock(g_map_mu);
        MapEntry* victim = &g_maps[0];
        for (MapEntry& e : g_maps) {
            if (!e.valid) {
                victim = &e;
                break;
            }
            if (e.used < victim->used) victim = &e;
        }
        victim->key = k;
        victim->map = *map;
        victim->used = ++g_map_clock;
        victim->valid = true;
    }
    return true;
}

}  // namespace mxb
