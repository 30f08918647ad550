// neighbor.cuh -- coordinate hash table and K-offset neighbor map.
//
// Replaces the reference's device builders (burn_flex_gmm
// src/wgpu/neighbor_kernels.rs: the single-lane serial insert :197-276 and
// its query :278-335) with a fully parallel open-addressing table:
//   * key   = (batch << 48) | (x << 32) | (y << 16) | z, every component in
//             [0, 65534], so the all-ones word is free to mark empty slots;
//   * slot  = 16 bytes {u64 key, i32 row, i32 pad}: one vector load per probe;
//   * build = one thread per input row, linear probing, atomicCAS on the key,
//             then atomicMin on the row -> duplicates keep the LOWEST row, the
//             rule of every reference device builder (neighbor_kernels.rs:
//             37-39, 249-256);
//   * query = one thread per (row, offset) pair so that the [N, K] output is
//             written fully coalesced.
// Negative neighbor components give -1 (reference lib.rs:95-97); components
// above 65534 cannot be present in the table and also give -1.
#pragma once

#include "sc_common.cuh"

namespace sc {

constexpr uint64_t kEmptyKey = ~0ull;
constexpr int32_t kMaxCoord = 65534;
constexpr int kMaxKernelRows = 1024;

enum : int32_t { NB_STATUS_RANGE = 1, NB_STATUS_CAPACITY = 2 };

struct __align__(16) HashSlot {
    unsigned long long key;
    int32_t row;
    int32_t pad;
};

struct NbStatus {
    int32_t bits;
    int32_t max_probe;
    int32_t pad[2];
};

struct KernelOffsets {
    int32_t k;
    int8_t d[3 * kMaxKernelRows];
};

// splitmix64 finaliser (Steele, Lea, Flood: "Fast splittable pseudorandom
// number generators", OOPSLA 2014).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ bool coord_in_range(int4 c) {
    return (unsigned)c.x <= (unsigned)kMaxCoord && (unsigned)c.y <= (unsigned)kMaxCoord &&
           (unsigned)c.z <= (unsigned)kMaxCoord && (unsigned)c.w <= (unsigned)kMaxCoord;
}

__device__ __forceinline__ uint64_t pack_key(int b, int x, int y, int z) {
    return ((uint64_t)(uint32_t)b << 48) | ((uint64_t)(uint32_t)x << 32) |
           ((uint64_t)(uint32_t)y << 16) | (uint64_t)(uint32_t)z;
}

__global__ void __launch_bounds__(256) nb_build_kernel(const int4* __restrict__ coords, int64_t n,
                                                       HashSlot* __restrict__ table, uint64_t mask,
                                                       NbStatus* __restrict__ status) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    int4 c = __ldg(coords + r);
    if (!coord_in_range(c)) {
        atomicOr(&status->bits, NB_STATUS_RANGE);
        return;
    }
    const unsigned long long key = pack_key(c.x, c.y, c.z, c.w);
    uint64_t s = mix64(key) & mask;
    for (uint64_t probe = 1; probe <= mask + 1; ++probe) {
        unsigned long long cur = table[s].key;
        if (cur == kEmptyKey) cur = atomicCAS(&table[s].key, kEmptyKey, key);
        if (cur == kEmptyKey || cur == key) {
            // The table is memset to all-ones: an empty row reads as UINT32_MAX,
            // so an unsigned minimum keeps the lowest inserting row.
            atomicMin(reinterpret_cast<unsigned*>(&table[s].row), (unsigned)r);
            atomicMax(&status->max_probe, probe > 0x7fffffffull ? 0x7fffffff : (int32_t)probe);
            return;
        }
        s = (s + 1) & mask;
    }
    atomicOr(&status->bits, NB_STATUS_CAPACITY);
}

__global__ void __launch_bounds__(256) nb_query_kernel(const int4* __restrict__ q, int64_t n_q,
                                                       const HashSlot* __restrict__ table,
                                                       uint64_t mask, const KernelOffsets off,
                                                       int32_t* __restrict__ out) {
    const int K = off.k;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_q * K) return;
    int64_t row = idx / K;
    int k = (int)(idx - row * K);
    int4 c = __ldg(q + row);
    int nx = c.y + off.d[3 * k], ny = c.z + off.d[3 * k + 1], nz = c.w + off.d[3 * k + 2];
    int32_t found = -1;
    if (nx >= 0 && ny >= 0 && nz >= 0 && nx <= kMaxCoord && ny <= kMaxCoord && nz <= kMaxCoord &&
        (unsigned)c.x <= (unsigned)kMaxCoord) {
        const unsigned long long key = pack_key(c.x, nx, ny, nz);
        uint64_t s = mix64(key) & mask;
        for (uint64_t probe = 0; probe <= mask; ++probe) {
            ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(table) + s);
            if (v.x == key) {
                found = (int32_t)(uint32_t)(v.y & 0xffffffffull);
                break;
            }
            if (v.x == kEmptyKey) break;
            s = (s + 1) & mask;
        }
    }
    out[idx] = found;
}

// Table slots: the power of two >= 4 n_in (load factor <= 0.25: an absent key -- most taps
// of a sparse grid -- ends its linear probe after ~1.4 slots on average, against ~2.5 at
// 0.5), or, in a workspace too small for that, >= 2 n_in (load factor <= 0.5).
inline uint64_t nb_capacity_min(int64_t n_in) {
    uint64_t cap = 1024;
    while (cap < (uint64_t)n_in * 2) cap <<= 1;
    return cap;
}

inline uint64_t nb_capacity(int64_t n_in) { return nb_capacity_min(n_in) * 2; }

inline size_t nb_workspace_bytes(int64_t n_in) {
    return 256 + (size_t)nb_capacity(n_in) * sizeof(HashSlot);
}

// Capacity used with a workspace of ws_bytes (0 if it cannot hold the minimum table).
inline uint64_t nb_capacity_for(int64_t n_in, size_t ws_bytes) {
    if (ws_bytes >= nb_workspace_bytes(n_in)) return nb_capacity(n_in);
    const uint64_t lo = nb_capacity_min(n_in);
    return ws_bytes >= 256 + (size_t)lo * sizeof(HashSlot) ? lo : 0;
}

}  // namespace sc
