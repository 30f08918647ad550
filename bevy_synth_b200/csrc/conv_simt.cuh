// conv_simt.cuh -- CUDA-core gather-GEMM for the sparse submanifold conv.
//
// The fp32 path (exact fp32 FFMA accumulation) and the fallback for shapes the
// tensor-core kernel does not take (groups > 1, odd channel counts, K > 32).
// Semantics follow the reference device kernels (burn_flex_gmm
// src/wgpu/sparse_conv_kernels.rs:4-46 and the fused OC4 variants :89-337):
// out[r, o] = bias[o] + sum_k sum_i in[nbr[r,k], g*Cin_g + i] * W[o, k, i],
// invalid neighbors contribute nothing.  Instead of one thread per output
// scalar re-reading its neighbor rows Cout times, a 64x64 output tile is
// accumulated in registers (4x4 per thread) from 16-channel slices of the
// gathered rows and the weights staged in shared memory; taps with no valid
// row in the tile are skipped.
#pragma once

#include "sc_common.cuh"

namespace sc {

struct EpiParams {
    const void* residual;
    const int64_t* res_off;
    int res_rep;
    void* out;
    const int32_t* row_map;
    int map_cols;
    const int32_t* row_order;  // nullable: tile position -> output row
};

template <typename T>
__device__ __forceinline__ float load_residual(const T* res, const int64_t* res_off, int rep,
                                               int64_t row, int col, int cout) {
    if (res_off) return to_f32<T>(res[res_off[row] + col / rep]);
    return to_f32<T>(res[row * (int64_t)cout + col]);
}

constexpr int SIMT_BM = 64, SIMT_BN = 64, SIMT_BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) conv_simt_kernel(
    const T* __restrict__ in, int64_t n_in, int cin, int cin_g, const int32_t* __restrict__ nbr,
    int64_t n_rows, int K, const T* __restrict__ w, const float* __restrict__ bias, int cout,
    int cout_g, int blocks_per_group, EpiParams epi) {
    __shared__ float As[SIMT_BK][SIMT_BM + 4];
    __shared__ float Bs[SIMT_BK][SIMT_BN + 4];
    __shared__ int32_t nb_s[SIMT_BM];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t row0 = (int64_t)blockIdx.x * SIMT_BM;
    const int group = blockIdx.y / blocks_per_group;
    const int col0 = (blockIdx.y % blocks_per_group) * SIMT_BN;  // within the group
    const int in_base = group * cin_g;
    const int out_base = group * cout_g;

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    for (int k = 0; k < K; ++k) {
        int valid = 0;
        if (tid < SIMT_BM) {
            int64_t r = row0 + tid;
            int32_t v = -1;
            if (r < n_rows && epi.row_order) {
                r = epi.row_order[r];
                if (r < 0 || r >= n_rows) {
                    raise_fault(FAULT_BAD_NEIGHBOR);
                    r = n_rows;
                }
            }
            if (r < n_rows) {
                v = __ldg(nbr + r * K + k);
                if (v < -1 || v >= n_in) {
                    raise_fault(FAULT_BAD_NEIGHBOR);
                    v = -1;
                }
            }
            nb_s[tid] = v;
            valid = v >= 0;
        }
        if (!__syncthreads_or(valid)) continue;
        for (int c0 = 0; c0 < cin_g; c0 += SIMT_BK) {
            // A: 64 rows x 16 channels, 4 per thread
            {
                int r = tid >> 2, c = (tid & 3) * 4;
                int32_t src = nb_s[r];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float v = 0.f;
                    if (src >= 0 && c0 + c + u < cin_g)
                        v = to_f32<T>(in[(int64_t)src * cin + in_base + c0 + c + u]);
                    As[c + u][r] = v;
                }
            }
            // B: 64 output channels x 16 input channels of tap k
            {
                int o = tid >> 2, c = (tid & 3) * 4;
                int oc = col0 + o;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float v = 0.f;
                    if (oc < cout_g && c0 + c + u < cin_g)
                        v = to_f32<T>(w[((int64_t)(out_base + oc) * K + k) * cin_g + c0 + c + u]);
                    Bs[c + u][o] = v;
                }
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < SIMT_BK; ++kk) {
                float a[4], b[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            __syncthreads();
        }
    }

    // epilogue: bias, residual, scatter
    const T* res = reinterpret_cast<const T*>(epi.residual);
    T* out = reinterpret_cast<T*>(epi.out);
    const int wb = epi.row_map ? cout / epi.map_cols : cout;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t r = row0 + ty * 4 + i;
        if (r >= n_rows) continue;
        if (epi.row_order) {
            r = epi.row_order[r];
            if (r < 0 || r >= n_rows) continue;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int oc = col0 + tx * 4 + j;
            if (oc >= cout_g) continue;
            int o = out_base + oc;
            float v = acc[i][j] + (bias ? bias[o] : 0.f);
            if (res) v += load_residual<T>(res, epi.res_off, epi.res_rep, r, o, cout);
            int64_t orow = r;
            int ocol = o;
            if (epi.row_map) {
                orow = epi.row_map[r * epi.map_cols + o / wb];
                ocol = o % wb;
                if (orow < 0) continue;
            }
            out[orow * wb + ocol] = from_f32<T>(v);
        }
    }
}

// fp32 gather-GEMM with 8x8 outputs per thread (the fp32 path's main kernel).
// A 64-row x 64-column output tile per 128-thread CTA: two groups of two warps
// split the reduction steps (16 input channels of one tap each) between them,
// each group computing all 64 x 64 outputs in its own registers (8 x 8 per
// thread) from its own double-buffered shared-memory stages (A transposed to
// [channel][row], B to [channel][column]); the next step's 16-byte global
// loads are in registers while the current step's FMAs run, and the next
// channel's fragments while the current channel's.  Group 1 hands its partial
// sums to group 0 through shared memory at the end.  The tile's neighbor rows
// are read once into shared memory and taps with no valid row are skipped.
// The split doubles the warps per SM of a small layer (a 21k-row layer has only
// ~340 tiles), which the FMA pipe needs to hide its operand latencies.
// Taken for fp32, groups == 1, Cin % 16 == 0, Cout % 64 == 0, K <= 32, with
// 16-byte aligned features and weights; other shapes use conv_simt_kernel.
constexpr int F32_BM = 64, F32_BN = 64, F32_BK = 16, F32_THREADS = 128, F32_MAX_K = 32;

__device__ __forceinline__ void f32_group_sync(int group) {  // named barrier 1 or 2, 64 threads
    if (group == 0)
        asm volatile("bar.sync 1, 64;" ::: "memory");
    else
        asm volatile("bar.sync 2, 64;" ::: "memory");
}

__global__ void __launch_bounds__(F32_THREADS) conv_f32_tiled_kernel(
    const float* __restrict__ in, int64_t n_in, int cin, const int32_t* __restrict__ nbr, int64_t n_rows, int K,
    const float* __restrict__ w, const float* __restrict__ bias, int cout, EpiParams epi) {
    // [group][buffer][A | B][channel][row | column]; group 1's half doubles as the partial-sum tile
    __shared__ __align__(16) float stage[2][2][2][F32_BK][F32_BM];
    __shared__ int32_t nb_s[F32_MAX_K][F32_BM];
    __shared__ int32_t taps_s[F32_MAX_K];
    __shared__ uint32_t tap_mask;

    const int tid = threadIdx.x;
    const int grp = tid >> 6, lt = tid & 63;
    // compute: rows ty*4+i and 32+ty*4+i, columns tx*4+j and 32+tx*4+j (i, j < 4): each
    // 16-byte shared-memory read of a warp is then one contiguous 128-byte span
    const int ty = lt >> 3, tx = lt & 7;
    const int64_t row0 = (int64_t)blockIdx.x * F32_BM;
    const int col0 = blockIdx.y * F32_BN;

    if (tid == 0) tap_mask = 0u;
    __syncthreads();
    if (grp == 0) {
        // this thread's tile row: its neighbor rows (checked) and valid-tap bits
        int64_t r = row0 + lt;
        if (r < n_rows && epi.row_order) {
            r = epi.row_order[r];
            if (r < 0 || r >= n_rows) {
                raise_fault(FAULT_BAD_NEIGHBOR);
                r = n_rows;
            }
        }
        uint32_t m = 0;
        for (int k = 0; k < K; ++k) {
            int32_t v = -1;
            if (r < n_rows) {
                v = __ldg(nbr + r * K + k);
                if (v < -1 || v >= n_in) {
                    raise_fault(FAULT_BAD_NEIGHBOR);
                    v = -1;
                }
            }
            nb_s[k][lt] = v;
            if (v >= 0) m |= 1u << k;
        }
        m = __reduce_or_sync(0xffffffffu, m);
        if ((lt & 31) == 0) atomicOr(&tap_mask, m);
    }
    __syncthreads();
    const uint32_t mask = tap_mask;
    if (tid == 0) {
        int t = 0;
        for (uint32_t m = mask; m; m &= m - 1) taps_s[t++] = __ffs(m) - 1;
    }
    __syncthreads();
    const int cpt = cin / F32_BK;              // steps per tap
    const int n_steps = __popc(mask) * cpt;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    // global -> registers for step st: A row `lt` (16 channels), B column `lt` (16 channels)
    float4 ra[4], rb[4];
    auto gload = [&](int st) {
        const int k = taps_s[st / cpt], c0 = (st % cpt) * F32_BK;
        const int32_t src = nb_s[k][lt];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            ra[q] = src >= 0 ? __ldg(reinterpret_cast<const float4*>(in + (int64_t)src * cin + c0) + q)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        const float* wp = w + ((int64_t)(col0 + lt) * K + k) * cin + c0;
#pragma unroll
        for (int q = 0; q < 4; ++q) rb[q] = __ldg(reinterpret_cast<const float4*>(wp) + q);
    };
    auto sstore = [&](int b) {
        float(*A)[F32_BM] = stage[grp][b][0];
        float(*B)[F32_BN] = stage[grp][b][1];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            A[4 * q + 0][lt] = ra[q].x;
            A[4 * q + 1][lt] = ra[q].y;
            A[4 * q + 2][lt] = ra[q].z;
            A[4 * q + 3][lt] = ra[q].w;
            B[4 * q + 0][lt] = rb[q].x;
            B[4 * q + 1][lt] = rb[q].y;
            B[4 * q + 2][lt] = rb[q].z;
            B[4 * q + 3][lt] = rb[q].w;
        }
    };

    int st = grp;  // this group's steps: grp, grp + 2, ...
    if (st < n_steps) {
        gload(st);
        sstore(0);
        f32_group_sync(grp);
        for (int b = 0;; b ^= 1) {
            const int nst = st + 2;
            if (nst < n_steps) gload(nst);
            float(*A)[F32_BM] = stage[grp][b][0];
            float(*B)[F32_BN] = stage[grp][b][1];
            // fragments of channel kk + 1 are read while channel kk's 64 FMAs run
            float4 fa0 = *reinterpret_cast<const float4*>(&A[0][ty * 4]);
            float4 fa1 = *reinterpret_cast<const float4*>(&A[0][32 + ty * 4]);
            float4 fb0 = *reinterpret_cast<const float4*>(&B[0][tx * 4]);
            float4 fb1 = *reinterpret_cast<const float4*>(&B[0][32 + tx * 4]);
#pragma unroll
            for (int kk = 0; kk < F32_BK; ++kk) {
                const float av[8] = {fa0.x, fa0.y, fa0.z, fa0.w, fa1.x, fa1.y, fa1.z, fa1.w};
                const float bv[8] = {fb0.x, fb0.y, fb0.z, fb0.w, fb1.x, fb1.y, fb1.z, fb1.w};
                if (kk + 1 < F32_BK) {
                    fa0 = *reinterpret_cast<const float4*>(&A[kk + 1][ty * 4]);
                    fa1 = *reinterpret_cast<const float4*>(&A[kk + 1][32 + ty * 4]);
                    fb0 = *reinterpret_cast<const float4*>(&B[kk + 1][tx * 4]);
                    fb1 = *reinterpret_cast<const float4*>(&B[kk + 1][32 + tx * 4]);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (nst >= n_steps) break;
            sstore(b ^ 1);
            f32_group_sync(grp);
            st = nst;
        }
    }

    // group 1's partial sums -> group 0 (through group 1's stage buffers: 64 x 64 floats)
    __syncthreads();
    float(*part)[F32_BN] = reinterpret_cast<float(*)[F32_BN]>(&stage[1][0][0][0][0]);
    if (grp == 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int rr = i < 4 ? ty * 4 + i : 32 + ty * 4 + (i - 4);
            *reinterpret_cast<float4*>(&part[rr][tx * 4]) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            *reinterpret_cast<float4*>(&part[rr][32 + tx * 4]) =
                make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
        }
    }
    __syncthreads();
    if (grp == 1) return;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int rr = i < 4 ? ty * 4 + i : 32 + ty * 4 + (i - 4);
        const float4 p0 = *reinterpret_cast<const float4*>(&part[rr][tx * 4]);
        const float4 p1 = *reinterpret_cast<const float4*>(&part[rr][32 + tx * 4]);
        acc[i][0] += p0.x;
        acc[i][1] += p0.y;
        acc[i][2] += p0.z;
        acc[i][3] += p0.w;
        acc[i][4] += p1.x;
        acc[i][5] += p1.y;
        acc[i][6] += p1.z;
        acc[i][7] += p1.w;
    }

    // epilogue: bias, residual, scatter (as conv_simt_kernel)
    const float* res = reinterpret_cast<const float*>(epi.residual);
    float* out = reinterpret_cast<float*>(epi.out);
    const int wb = epi.row_map ? cout / epi.map_cols : cout;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int64_t r = row0 + (i < 4 ? ty * 4 + i : 32 + ty * 4 + (i - 4));
        if (r >= n_rows) continue;
        if (epi.row_order) {
            r = epi.row_order[r];
            if (r < 0 || r >= n_rows) continue;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int o = col0 + (j < 4 ? tx * 4 + j : 32 + tx * 4 + (j - 4));
            float v = acc[i][j] + (bias ? bias[o] : 0.f);
            if (res) v += load_residual<float>(res, epi.res_off, epi.res_rep, r, o, cout);
            int64_t orow = r;
            int ocol = o;
            if (epi.row_map) {
                orow = epi.row_map[r * epi.map_cols + o / wb];
                ocol = o % wb;
                if (orow < 0) continue;
            }
            out[orow * wb + ocol] = v;
        }
    }
}

// Row-wise LayerNorm (+affine) and/or SiLU, one warp per entry.  Entry e is
// the `width` values at element offset row*ld with row = map[e] (or e when
// map is null; skipped when negative).  Two-pass statistics as the reference
// (burn_trellis sparse_decoder_wgpu_ops.rs:1642-1711): mean, then biased
// variance sum((x-mean)^2)/C, inv_std = 1/sqrt(var + eps).
// rpw = 0: one warp per entry, scalar loads (any dtype, width, alignment).  rpw in
// {1, 2, 4, 8, 16, 32} (bf16 only; width % 8 == 0, width <= 1024, ld % 8 == 0, x and y
// 16-byte aligned; rows_norm_act_rpw decides, and takes it for width <= 128): rpw entries per warp, a group of
// 32 / rpw lanes per entry, each lane holding up to four 16-byte chunks of 8 values in
// registers, so a row is read from memory once and narrow rows keep every lane busy.
template <typename T>
__global__ void __launch_bounds__(256) rows_norm_act_kernel(
    const T* __restrict__ x, T* __restrict__ y, int64_t n_entries, int width, int64_t ld,
    const int32_t* __restrict__ row_map, const float* __restrict__ gamma,
    const float* __restrict__ beta, float eps, int do_ln, int do_silu, int rpw) {
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (rpw > 0) {
        const int G = 32 / rpw;                 // lanes per entry
        const int sub = lane & (G - 1);
        const int64_t e = warp_id * rpw + lane / G;
        const bool live = e < n_entries;
        const int64_t row = live ? (row_map ? (int64_t)row_map[e] : e) : -1;
        const int w8 = width >> 3;
        uint4 u[4];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c8 = sub + G * j;
            if (row >= 0 && c8 < w8) {
                u[j] = __ldg(reinterpret_cast<const uint4*>(x + row * ld) + c8);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = __bfloat1622float2(h[q]);
                    s += f.x + f.y;
                }
            }
        }
        float mean = 0.f, rstd = 1.f;
        if (do_ln) {
            for (int o = G >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            mean = s / (float)width;
            float v = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (row >= 0 && sub + G * j < w8) {
                    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 f = __bfloat1622float2(h[q]);
                        v += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
                    }
                }
            }
            for (int o = G >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            rstd = 1.0f / sqrtf(v / (float)width + eps);
        }
        if (row < 0) return;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c8 = sub + G * j;
            if (c8 < w8) {
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
                uint4 o4;
                __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = __bfloat1622float2(h[q]);
                    float a0 = f.x, a1 = f.y;
                    const int c = 8 * c8 + 2 * q;
                    if (do_ln) {
                        a0 = (a0 - mean) * rstd;
                        a1 = (a1 - mean) * rstd;
                        if (gamma) { a0 *= gamma[c]; a1 *= gamma[c + 1]; }
                        if (beta) { a0 += beta[c]; a1 += beta[c + 1]; }
                    }
                    if (do_silu) { a0 = silu_f(a0); a1 = silu_f(a1); }
                    oh[q] = __floats2bfloat162_rn(a0, a1);
                }
                reinterpret_cast<uint4*>(y + row * ld)[c8] = o4;
            }
        }
        return;
    }
    const int64_t e = warp_id;
    if (e >= n_entries) return;
    int64_t row = row_map ? (int64_t)row_map[e] : e;
    if (row < 0) return;
    const T* xr = x + row * ld;
    T* yr = y + row * ld;
    float mean = 0.f, rstd = 1.f;
    if (do_ln) {
        float s = 0.f;
        for (int c = lane; c < width; c += 32) s += to_f32<T>(xr[c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        mean = s / (float)width;
        float v = 0.f;
        for (int c = lane; c < width; c += 32) {
            float d = to_f32<T>(xr[c]) - mean;
            v += d * d;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        rstd = 1.0f / sqrtf(v / (float)width + eps);
    }
    for (int c = lane; c < width; c += 32) {
        float a = to_f32<T>(xr[c]);
        if (do_ln) {
            a = (a - mean) * rstd;
            if (gamma) a *= gamma[c];
            if (beta) a += beta[c];
        }
        if (do_silu) a = silu_f(a);
        yr[c] = from_f32<T>(a);
    }
}

// Entries per warp of rows_norm_act_kernel's vector path for these arguments, or 0 for the
// scalar path: one lane group of the smallest power of two >= width / 8 lanes per entry.
// Taken for rows of at most 128 values (two or more rows per warp).  Measured on B200 against
// the scalar path: 1M x 64 326 -> 150 us, 420k x 96 168 -> 131 us; wider rows were slower
// (105k x 192 59 -> 78 us, 102k x 256 50 -> 82 us).
template <typename T>
inline int rows_norm_act_rpw(const void* x, const void* y, int64_t width, int64_t ld) {
    if (sizeof(T) != 2 || width % 8 != 0 || width > 128 || ld % 8 != 0 ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) != 0)
        return 0;
    int g = 1;
    while (g < 32 && g < width / 8) g <<= 1;
    return 32 / g;
}

}  // namespace sc
