// rowops.cuh -- element-wise and subdivision kernels of libsparseconv.
#pragma once

#include "sc_common.cuh"

namespace sc {

// RNE rounding of the f32 bit pattern to bf16, kept in f32, with no NaN
// special case (reference: burn_flex_gmm src/wgpu.rs:57-67).
__global__ void bf16_round_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ y) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t b = __float_as_uint(x[i]);
    b = (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
    y[i] = __uint_as_float(b);
}

template <typename A, typename B>
__global__ void cast_kernel(const A* __restrict__ x, int64_t n, B* __restrict__ y) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    y[i] = from_f32<B>(to_f32<A>(x[i]));
}

// --- channel-to-space subdivision -------------------------------------------
// Child c = cx + 2*cy + 4*cz of parent p is kept when mask[p*8+c] != 0; kept
// children are numbered parent-major / child-minor, the order of the
// reference's argwhere + expand (burn_trellis sparse_decoder_wgpu_ops.rs:
// 927-1054) and of its host channel2spatial (:1999-2054).
__global__ void subdiv_count_kernel(const uint8_t* __restrict__ mask, int64_t n_parent,
                                    int32_t* __restrict__ counts) {
    int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p > n_parent) return;
    int c = 0;
    if (p < n_parent) {
        const uint2 m = *reinterpret_cast<const uint2*>(mask + p * 8);
        c = __popc(__vsetne4(m.x, 0u) & 0x01010101u) + __popc(__vsetne4(m.y, 0u) & 0x01010101u);
    }
    counts[p] = c;  // counts[n_parent] = 0 so the exclusive scan yields the total
}

__global__ void subdiv_write_kernel(const int4* __restrict__ parent_coords,
                                    const uint8_t* __restrict__ mask, int64_t n_parent,
                                    int64_t parent_channels, const int32_t* __restrict__ offsets,
                                    int32_t* __restrict__ child_row, int4* __restrict__ child_coords,
                                    int64_t* __restrict__ skip_offset) {
    int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n_parent) return;
    const int4 pc = __ldg(parent_coords + p);
    int32_t r = offsets[p];
    const int64_t cw = parent_channels / 8;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        if (mask[p * 8 + c]) {
            child_row[p * 8 + c] = r;
            if (child_coords)
                child_coords[r] = make_int4(pc.x, pc.y * 2 + (c & 1), pc.z * 2 + ((c >> 1) & 1),
                                            pc.w * 2 + ((c >> 2) & 1));
            if (skip_offset) skip_offset[r] = p * parent_channels + c * cw;
            ++r;
        } else {
            child_row[p * 8 + c] = -1;
        }
    }
}

// --- mask-sorted row order ----------------------------------------------------
// key[r] = sum_j valid(r, tap_rank[j]) << (K-1-j): taps ranked farthest-from-
// centre first, so rows with equal outer-tap patterns end up adjacent.
struct TapRank {
    int32_t k;
    int8_t rank_of_tap[32];  // bit position (K-1-rank) for each tap
};

__global__ void row_mask_key_kernel(const int32_t* __restrict__ nbr, int64_t n, const TapRank tr,
                                    uint32_t* __restrict__ keys, int32_t* __restrict__ vals) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    uint32_t key = 0;
    for (int k = 0; k < tr.k; ++k)
        if (__ldg(nbr + r * tr.k + k) >= 0) key |= 1u << (tr.k - 1 - tr.rank_of_tap[k]);
    keys[r] = key;
    vals[r] = (int32_t)r;
}

// dst[i, :] = src[idx[i], :] for rows of `row_units` 16-byte units (halo packing).
__global__ void gather_rows_kernel(const uint4* __restrict__ src, int64_t row_units,
                                   const int32_t* __restrict__ idx, int64_t n, int64_t n_src,
                                   uint4* __restrict__ dst) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * row_units) return;
    const int64_t r = i / row_units;
    const int64_t u = i - r * row_units;
    const int32_t s = __ldg(idx + r);
    if (s < 0 || s >= n_src) {
        raise_fault(FAULT_BAD_NEIGHBOR);
        dst[i] = make_uint4(0, 0, 0, 0);
        return;
    }
    dst[i] = __ldg(src + (int64_t)s * row_units + u);
}

// ordered[p, :] = nbr[order[p], :]
__global__ void permute_rows_kernel(const int32_t* __restrict__ nbr, const int32_t* __restrict__ order,
                                    int64_t n, int K, int32_t* __restrict__ ordered) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * K) return;
    const int64_t p = i / K;
    const int k = (int)(i - p * K);
    ordered[i] = __ldg(nbr + (int64_t)__ldg(order + p) * K + k);
}

}  // namespace sc
