// conv_tc.cuh -- sm_100a tensor-core (tcgen05) implicit gather-GEMM for the
// sparse submanifold convolution, with the bias / residual / LayerNorm / SiLU
// epilogue fused on the TMEM accumulator.
//
// Math (reference: burn_flex_gmm src/lib.rs:242-375 and the device kernels
// src/wgpu/sparse_conv_kernels.rs:4-46):
//     out[r, o] = bias[o] + sum_k sum_c in[nbr[r,k], c] * W[o, k, c]
// computed as a GEMM with M = output rows (tile of 128), N = output channels
// (tile of up to 512), and the reduction running over (tap k, 64-channel
// chunk) steps:
//   * A (128 x 64 bf16 per step) is GATHERED: each of the 128 rows of the
//     tile copies the 128-byte channel slice of its neighbor row nbr[r,k]
//     with 16-byte cp.async into a 128B-swizzled K-major smem tile (zero fill
//     for invalid neighbors or channels >= Cin);
//   * B (tile_n x 64 bf16 per step) is the weight slice W[n0:n0+tile_n, k,
//     c0:c0+64], loaded by TMA straight from the reference layout
//     [Cout, 27, Cin] through a 3-D tensor map (128B swizzle, OOB zero fill);
//   * tcgen05.mma (M=128, N<=256 per instruction, K=16) accumulates in fp32
//     TMEM; taps with no valid neighbor anywhere in the tile are skipped.
// Roles (192 threads): warps 0-3 gather A and then run the epilogue (thread i
// owns TMEM lane / tile row i), warp 4 issues the weight TMA, warp 5 issues
// the MMAs.  Stage hand-off uses mbarriers; every wait is bounded and raises
// the device fault word instead of hanging.
#pragma once

#include "sc_common.cuh"

namespace sc {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;                      // channels per reduction step
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KB
constexpr int TC_THREADS = 192;
constexpr int TC_MAX_K = 32;

struct TcParams {
    const __nv_bfloat16* in;
    int64_t n_in;
    int cin;
    const int32_t* nbr;
    int64_t n_rows;
    int K;
    const float* bias;
    int cout;
    int tile_n;   // output columns per CTA (multiple of 32, <= 512)
    int n_sub;    // MMAs per reduction step (1 or 2)
    int sub_n;    // N of each MMA (= TMA box rows), tile_n = n_sub * sub_n
    int stages;
    uint32_t tmem_cols;
    // epilogue
    const __nv_bfloat16* residual;
    const int64_t* res_off;
    int res_rep;
    int ln;
    int ln_width;
    float eps;
    const float* gamma;
    const float* beta;
    int silu;
    __nv_bfloat16* out;
    __nv_bfloat16* out2;
    const int32_t* row_map;
    int map_cols;
};

__device__ __forceinline__ void cp_async_wait_dyn(int n) {
    if (n <= 0)
        cp_async_wait<0>();
    else if (n == 1)
        cp_async_wait<1>();
    else
        cp_async_wait<2>();
}

// 32 consecutive bf16 of `src` (16-byte aligned) -> fp32
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
    const uint4* p = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 u = __ldg(p + q);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float2 f = __bfloat1622float2(h[e]);
            v[q * 8 + 2 * e] = f.x;
            v[q * 8 + 2 * e + 1] = f.y;
        }
    }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
    uint4* p = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
        p[q] = u;
    }
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzle atoms
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int S = p.stages;
    const int B_BYTES = p.tile_n * 128;
    uint8_t* a_smem = smem;
    uint8_t* b_smem = smem + S * TC_A_BYTES;
    int32_t* nbr_s = reinterpret_cast<int32_t*>(b_smem + S * B_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(nbr_s + TC_BM * p.K);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* accum_full = bars + 2 * S;
    uint32_t* misc = reinterpret_cast<uint32_t*>(accum_full + 1);  // [0]=tmem, [1]=tap mask, [2]=abort

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t tile_base = (int64_t)blockIdx.x * TC_BM;
    const int n0 = blockIdx.y * p.tile_n;
    const int K = p.K;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 128 + 1);  // 128 gathering threads + the TMA arrive
            mbar_init(&empty[s], 1);       // one tcgen05.commit
        }
        mbar_init(accum_full, 1);
        misc[1] = 0;
        misc[2] = 0;
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    if (warp == 5) {
        tmem_alloc(&misc[0], p.tmem_cols);
        tmem_relinquish();
    }
    if (warp == 4 && lane == 0) tma_prefetch_desc(&wmap);

    // neighbor tile -> smem (contiguous block of the [N, K] map), tap mask
    __syncthreads();
    {
        uint32_t mask = 0;
        const int64_t g0 = tile_base * K;
        const int64_t g_end = p.n_rows * K;
        for (int i = tid; i < TC_BM * K; i += TC_THREADS) {
            int32_t v = -1;
            if (g0 + i < g_end) {
                v = __ldg(p.nbr + g0 + i);
                if (v < -1 || v >= p.n_in) {
                    raise_fault(FAULT_BAD_NEIGHBOR);
                    v = -1;
                }
            }
            nbr_s[i] = v;
            if (v >= 0) mask |= 1u << (i % K);
        }
        if (mask) atomicOr(&misc[1], mask);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const uint32_t tmem_base = misc[0];
    const uint32_t tap_mask = misc[1];
    const int n_chunks = (p.cin + TC_BK - 1) / TC_BK;
    const int n_iters = __popc(tap_mask) * n_chunks;

    if (warp < 4) {
        // ------------------------------------------------ A gather producer
        const int t = tid;  // tile row
        const int LAG = S > 2 ? 2 : 1;
        int it = 0;
        bool ok = true;
        for (uint32_t m = tap_mask; m && ok; m &= m - 1) {
            const int k = __ffs(m) - 1;
            const int32_t src = nbr_s[t * K + k];
            const __nv_bfloat16* src_row = p.in + (int64_t)(src < 0 ? 0 : src) * p.cin;
            for (int ch = 0; ch < n_chunks; ++ch) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t dst = smem_u32(a_smem + s * TC_A_BYTES + t * 128);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = ch * TC_BK + j * 8;
                    const bool v = src >= 0 && c < p.cin;
                    cp_async_16(dst + ((j ^ (t & 7)) << 4), v ? (const void*)(src_row + c) : (const void*)p.in,
                                v ? 16u : 0u);
                }
                cp_async_commit();
                if (it >= LAG) {
                    cp_async_wait_dyn(LAG);
                    fence_proxy_async_smem();
                    mbar_arrive(&full[(it - LAG) % S]);
                }
                ++it;
            }
        }
        cp_async_wait<0>();
        fence_proxy_async_smem();
        if (ok) {
            for (int j = (it > LAG ? it - LAG : 0); j < it; ++j) mbar_arrive(&full[j % S]);
        } else {
            atomicOr(&misc[2], 1u);
        }
    } else if (warp == 4) {
        // ------------------------------------------------ weight TMA producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (uint32_t m = tap_mask; m && ok; m &= m - 1) {
                const int k = __ffs(m) - 1;
                for (int ch = 0; ch < n_chunks; ++ch) {
                    const int s = it % S;
                    const uint32_t ph = (uint32_t)(it / S) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], (uint32_t)B_BYTES);
                    const uint32_t dst = smem_u32(b_smem + s * B_BYTES);
                    for (int j = 0; j < p.n_sub; ++j)
                        tma_load_3d(dst + j * p.sub_n * 128, &wmap, &full[s], ch * TC_BK, k,
                                    n0 + j * p.sub_n);
                    ++it;
                }
            }
            if (!ok) atomicOr(&misc[2], 1u);
        }
    } else {
        // ------------------------------------------------ MMA issuer (warp 5)
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16_m128((uint32_t)p.sub_n);
            bool ok = true;
            for (int it = 0; it < n_iters; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(&full[s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(a_smem + s * TC_A_BYTES);
                const uint32_t b0 = smem_u32(b_smem + s * B_BYTES);
#pragma unroll
                for (int kk = 0; kk < TC_BK / 16; ++kk) {
                    const uint64_t ad = umma_desc_sw128(a0 + kk * 32);
                    for (int j = 0; j < p.n_sub; ++j) {
                        const uint64_t bd = umma_desc_sw128(b0 + j * p.sub_n * 128 + kk * 32);
                        umma_bf16(tmem_base + j * p.sub_n, ad, bd, idesc, (it > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&empty[s]);
            }
            if (ok && n_iters > 0)
                umma_commit(accum_full);
            else
                mbar_arrive(accum_full);
            if (!ok) atomicOr(&misc[2], 1u);
        }
    }

    // ---------------------------------------------------- epilogue (warps 0-3)
    if (warp < 4) {
        // tcgen05.ld/st are warp-collective (.sync.aligned): the decision to
        // read TMEM must be uniform across the warp.
        const bool waited = mbar_wait(accum_full, 0);
        const bool have_acc = __all_sync(0xffffffffu, waited) && n_iters > 0;
        tc_fence_after();
        const int t = tid;
        const int64_t row = tile_base + t;
        const bool row_ok = row < p.n_rows;
        const uint32_t lane_addr = tmem_base + ((uint32_t)(warp * 32) << 16);
        const int W = p.ln_width;
        const bool aborted = *reinterpret_cast<volatile uint32_t*>(&misc[2]) != 0;

        // output addressing
        int64_t orow = row;
        int ocol0 = n0;
        int64_t old = p.cout;
        if (p.row_map) {
            const int wb = p.cout / p.map_cols;
            orow = row_ok ? (int64_t)p.row_map[row * p.map_cols + n0 / wb] : -1;
            ocol0 = n0 % wb;
            old = wb;
        }
        const bool store = row_ok && orow >= 0 && !aborted;
        const bool multi_pass = p.ln != 0;

        for (int g0 = 0; g0 < p.tile_n; g0 += W) {
            float mean = 0.f, rstd = 1.f;
            // pass 1: y = acc + bias + residual (kept in TMEM for later passes)
            float sum = 0.f;
            for (int c = g0; c < g0 + W; c += 32) {
                float v[32];
                if (have_acc)
                    tmem_ld32(lane_addr + c, v);
                else
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = 0.f;
                if (p.bias) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] += __ldg(p.bias + n0 + c + e);
                }
                if (p.residual && row_ok) {
                    if (p.res_off) {
                        const int64_t base = p.res_off[row];
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            v[e] += __bfloat162float(p.residual[base + (n0 + c + e) / p.res_rep]);
                    } else {
                        float r[32];
                        load_bf16x32(p.residual + row * (int64_t)p.cout + n0 + c, r);
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] += r[e];
                    }
                }
                if (multi_pass) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) sum += v[e];
                    // without an accumulator, y (bias + residual) is recomputed below
                    if (have_acc) tmem_st32(lane_addr + c, v);
                } else {
                    if (store) {
                        __nv_bfloat16* o = p.out + orow * old + ocol0 + c;
                        if (p.out2) {
                            store_bf16x32(o, v);
                            float a[32];
#pragma unroll
                            for (int e = 0; e < 32; ++e) a[e] = p.silu ? silu_f(v[e]) : v[e];
                            store_bf16x32(p.out2 + orow * old + ocol0 + c, a);
                        } else {
                            if (p.silu) {
#pragma unroll
                                for (int e = 0; e < 32; ++e) v[e] = silu_f(v[e]);
                            }
                            store_bf16x32(o, v);
                        }
                    }
                }
            }
            if (!multi_pass) continue;
            mean = sum / (float)W;
            // helper to re-materialise y for column block c
            auto load_y = [&](int c, float (&v)[32]) {
                if (have_acc) {
                    tmem_ld32(lane_addr + c, v);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = p.bias ? __ldg(p.bias + n0 + c + e) : 0.f;
                    if (p.residual && row_ok) {
                        if (p.res_off) {
                            const int64_t base = p.res_off[row];
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                v[e] += __bfloat162float(p.residual[base + (n0 + c + e) / p.res_rep]);
                        } else {
                            float r[32];
                            load_bf16x32(p.residual + row * (int64_t)p.cout + n0 + c, r);
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] += r[e];
                        }
                    }
                }
            };
            // pass 2: biased variance about the mean (two-pass, as the reference)
            float var = 0.f;
            for (int c = g0; c < g0 + W; c += 32) {
                float v[32];
                load_y(c, v);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float d = v[e] - mean;
                    var += d * d;
                }
            }
            rstd = 1.0f / sqrtf(var / (float)W + p.eps);
            // pass 3: outputs
            for (int c = g0; c < g0 + W; c += 32) {
                float v[32];
                load_y(c, v);
                if (store && p.out2) store_bf16x32(p.out + orow * old + ocol0 + c, v);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    float a = (v[e] - mean) * rstd;
                    const int gc = c - g0 + e;
                    if (p.gamma) a *= __ldg(p.gamma + gc);
                    if (p.beta) a += __ldg(p.beta + gc);
                    v[e] = p.silu ? silu_f(a) : a;
                }
                if (store) store_bf16x32((p.out2 ? p.out2 : p.out) + orow * old + ocol0 + c, v);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

}  // namespace sc
