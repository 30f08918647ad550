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

// 64-bit key: the row's group (8 bits from a [n, 8] 0/1 mask, bit c = column
// c) above its 32-bit valid-tap key, so a stable sort groups rows by group
// first and by tap mask within a group.
__global__ void row_group_key_kernel(const int32_t* __restrict__ nbr, int64_t n, const TapRank tr,
                                     const uint8_t* __restrict__ group_mask8, uint64_t* __restrict__ keys,
                                     int32_t* __restrict__ vals) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    uint32_t key = 0;
    for (int k = 0; k < tr.k; ++k)
        if (__ldg(nbr + r * tr.k + k) >= 0) key |= 1u << (tr.k - 1 - tr.rank_of_tap[k]);
    uint32_t g = 0;
    if (group_mask8)
        for (int c = 0; c < 8; ++c) g |= (__ldg(group_mask8 + r * 8 + c) ? 1u : 0u) << c;
    keys[r] = ((uint64_t)g << 32) | key;
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

// Subdivision head: logits[r, c] = bias[c] + sum_k x[r, k] * W[c, k] for the
// 8 children (the decoder's to_subdiv linear layer, fp32 accumulate),
// optionally centred on the row's mean, and mask[r, c] = logit > thr[c].
// One warp per row; each lane accumulates a strided slice of the channels.
struct SubdivThresholds {
    float t[8];
};
template <typename T>
__global__ void subdiv_head_kernel(const T* __restrict__ x, int64_t n, int c, const T* __restrict__ w,
                                   const float* __restrict__ bias, SubdivThresholds thr, int center,
                                   float* __restrict__ logits, uint8_t* __restrict__ mask) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const T* xr = x + r * c;
    for (int k = lane; k < c; k += 32) {
        const float v = to_f32(xr[k]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += v * to_f32(__ldg(w + (int64_t)j * c + k));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    float lg[8];
    float mean = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        lg[j] = acc[j] + (bias ? __ldg(bias + j) : 0.f);
        mean += lg[j];
    }
    mean *= 0.125f;
    if (lane < 8) {
        float v = lg[0];
#pragma unroll
        for (int j = 1; j < 8; ++j)
            if (lane == j) v = lg[j];
        if (center) v -= mean;
        if (logits) logits[r * 8 + lane] = v;
        mask[r * 8 + lane] = v > thr.t[lane] ? 1 : 0;
    }
}

// Sparse 3-D patchify, gather half: for each coordinate row (batch,
// tubelet, patch_row, patch_col) the patch of the dense input [B, Cin, T, H, W]
// flattened in (c, dt, py, px) order -> im2col[row, K].  Coordinates outside
// the grid raise the fault word and give a zero row.
struct PatchGeom {
    int64_t cin, frames, height, width, batches;
    int tub, ph, pw;
};
template <typename T>
__global__ void patch_gather_kernel(const T* __restrict__ input, const int4* __restrict__ coords, int64_t rows,
                                    PatchGeom g, T* __restrict__ out) {
    const int64_t K = g.cin * g.tub * g.ph * g.pw;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * K) return;
    const int64_t r = i / K;
    const int64_t k0 = i - r * K;
    int64_t kk = k0;
    const int px = (int)(kk % g.pw);
    kk /= g.pw;
    const int py = (int)(kk % g.ph);
    kk /= g.ph;
    const int dt = (int)(kk % g.tub);
    const int64_t c = kk / g.tub;
    const int4 q = __ldg(coords + r);
    const int64_t t = (int64_t)q.y * g.tub + dt, y = (int64_t)q.z * g.ph + py, x = (int64_t)q.w * g.pw + px;
    if (q.x < 0 || q.x >= g.batches || q.y < 0 || t >= g.frames || q.z < 0 || y >= g.height || q.w < 0 ||
        x >= g.width) {
        if (k0 == 0) raise_fault(FAULT_BAD_NEIGHBOR);
        out[i] = T(0.f);
        return;
    }
    out[i] = __ldg(input + ((((int64_t)q.x * g.cin + c) * g.frames + t) * g.height + y) * g.width + x);
}

__global__ void iota_kernel(int32_t* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = (int32_t)i;
}

}  // namespace sc
