// linear_tc.cuh -- sm_100a tensor-core dense linear layer for the decoder's
// 1x1 projections (ConvNeXt MLP, patch projections):
//     out[r, o] = act(bias[o] + sum_c x[r, c] * W[o, c] (+ residual[r, o]))
// (reference: linear_forward, burn_trellis src/runtime_model/
// sparse_decoder_wgpu_ops.rs:1-60, bias first, then the GEMM accumulates;
// the ConvNeXt MLP :355-489: mlp_0 + SiLU, mlp_2 + the block input).
//
// The rows are contiguous, so both operands arrive by TMA tile loads (A: 128
// rows x 64 channels, B: N outputs x 64 channels, 128B swizzle) -- no
// neighbor map, no per-row gathers.  One persistent CTA per SM, static
// round-robin over (row tile, column tile) pairs; warp roles:
//   0    TMA producer (one lane): A and B of every 64-channel stage;
//   1    MMA issuer (whole warp runs the loop, one elected lane issues
//        tcgen05.mma M=128, N, K=16) and TMEM owner;
//   2-9  epilogue, two warps per TMEM sub-partition: thread = tile row
//        (TMEM lane), 64-column boxes: + bias, [+ residual], [SiLU] (the
//        conv epilogue's order), bf16 into a swizzled staging box, one TMA
//        tile store per box.
// TMEM: two accumulators of N <= 256 columns, so a tile's epilogue overlaps
// the next tile's MMAs.  Every wait is bounded (device wait limit); on expiry
// the fault word is raised and the roles drain.
#pragma once

#include "conv_tc.cuh"

namespace sc {

constexpr int LIN_EPI_WARPS = 8;                 // two per TMEM sub-partition
constexpr int LIN_THREADS = (2 + LIN_EPI_WARPS) * 32;
constexpr int LIN_EPI_BYTES = LIN_EPI_WARPS * 32 * 128;  // one 32-row x 64-column bf16 box per warp
constexpr int LIN_A_BYTES = 128 * 128;  // 128 rows x 64 bf16

struct LinParams {
    int64_t rows;
    int cin;
    int cout;
    int tile_n;       // output columns per tile (multiple of 32, <= 256)
    int grid_y;       // column tiles
    int64_t n_tiles;  // row tiles * grid_y
    int stages;
    const float* bias;
    const __nv_bfloat16* residual;  // [rows, cout] or null
    int silu;
    __nv_bfloat16* out;
};

// 2-D tiled TMA load: the box at (c0, c1) of the map -> dst, completing on bar.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* desc, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(desc), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

inline size_t lin_smem_bytes(int tile_n, int stages) {
    return 1024 + (size_t)stages * (LIN_A_BYTES + (size_t)tile_n * 128) + LIN_EPI_BYTES +
           (size_t)(2 * stages + 4) * 8 + 16;
}

__global__ void __launch_bounds__(LIN_THREADS, 1) linear_tc_kernel(const __grid_constant__ CUtensorMap amap,
                                                                   const __grid_constant__ CUtensorMap bmap,
                                                                   const __grid_constant__ CUtensorMap omap,
                                                                   const LinParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const int S = p.stages;
    const int B_BYTES = p.tile_n * 128;
    uint8_t* a_smem = smem;                                    // [S][128 rows][128 B]
    uint8_t* b_smem = a_smem + (size_t)S * LIN_A_BYTES;        // [S][tile_n rows][128 B]
    uint8_t* epi_s = b_smem + (size_t)S * B_BYTES;             // [8 warps][32 rows][128 B], 1024-aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(epi_s + LIN_EPI_BYTES);
    uint64_t* empty = full + S;
    uint64_t* tmem_full = empty + S;   // [2]
    uint64_t* tmem_empty = tmem_full + 2;  // [2]
    uint32_t* misc = reinterpret_cast<uint32_t*>(tmem_empty + 2);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t n_ctas = gridDim.x;
    const int n_kb = (p.cin + 63) / 64;
    auto tile_of = [&](int64_t lt) -> int64_t {
        const int64_t t = (int64_t)blockIdx.x + lt * n_ctas;
        return t < p.n_tiles ? t : -1;
    };

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);    // the producer's expect_tx arrive (+ the two TMA loads' bytes)
            mbar_init(&empty[s], 1);   // tcgen05.commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);   // tcgen05.commit after a tile's last MMA
            mbar_init(&tmem_empty[b], LIN_EPI_WARPS);  // every epilogue warp
        }
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(&misc[0], TC_TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&amap);
        tma_prefetch_desc(&bmap);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = misc[0];

    if (warp == 0) {
        // ====================================================== TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t lt = 0; ok; ++lt) {
                const int64_t t = tile_of(lt);
                if (t < 0) break;
                const int r0 = (int)((t / p.grid_y) * 128);
                const int n0 = (int)(t % p.grid_y) * p.tile_n;
                for (int kb = 0; kb < n_kb; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], (uint32_t)(LIN_A_BYTES + B_BYTES));
                    tma_load_2d(smem_u32(a_smem + (size_t)s * LIN_A_BYTES), &amap, &full[s], kb * 64, r0);
                    tma_load_2d(smem_u32(b_smem + (size_t)s * B_BYTES), &bmap, &full[s], kb * 64, n0);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ====================================================== MMA issuer
        const bool issuer = elect_one();
        const uint32_t idesc = umma_idesc_bf16_m128((uint32_t)p.tile_n);
        const uint64_t adesc0 = umma_desc_sw128(smem_u32(a_smem));
        const uint64_t bdesc0 = umma_desc_sw128(smem_u32(b_smem));
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int64_t lt = 0; ok; ++lt) {
            const int64_t t = tile_of(lt);
            if (t < 0) break;
            const int b = (int)(lt & 1);
            const uint32_t use = (uint32_t)(lt >> 1);
            if (!__all_sync(0xffffffffu, mbar_wait(&tmem_empty[b], (use & 1u) ^ 1u))) break;
            tc_fence_after();
            const uint32_t acc = tmem_base + (uint32_t)(b * p.tile_n);
            for (int kb = 0; kb < n_kb; ++kb) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (issuer) {
                    const uint64_t ad = adesc0 + (uint64_t)(((size_t)s * LIN_A_BYTES) >> 4);
                    const uint64_t bd = bdesc0 + (uint64_t)(((size_t)s * B_BYTES) >> 4);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(acc, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                                  (kb == 0 && kk == 0) ? 0u : 1u);
                    umma_commit(&empty[s]);
                }
                __syncwarp();
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (!ok) break;
            if (issuer) umma_commit(&tmem_full[b]);
            __syncwarp();
        }
    } else {
        // ====================================================== epilogue
        // Two warps per TMEM sub-partition: warp e (= warp - 2) reads lanes 32 (e % 4) .. + 31
        // and the 64-column boxes h, h + 2, ... (h = e / 4) of the tile.  A box goes out through
        // this warp's 128B-swizzled 4 KB staging and one TMA tile store (whole 128-byte lines;
        // rows past the end are not written); the next box waits until that store has read the
        // staging.  The accumulator is released once every warp has its last columns.
        const int e = warp - 2;
        const int q = warp & 3;  // TMEM sub-partition of this warp
        const int h = e >> 2;
        uint8_t* es = epi_s + (size_t)e * 32 * 128;
        for (int64_t lt = 0;; ++lt) {
            const int64_t t = tile_of(lt);
            if (t < 0) break;
            const int b = (int)(lt & 1);
            const uint32_t use = (uint32_t)(lt >> 1);
            if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[b], use & 1u))) break;
            tc_fence_after();
            const int64_t row0 = (t / p.grid_y) * 128 + q * 32;
            const int64_t row = row0 + lane;
            const int n0 = (int)(t % p.grid_y) * p.tile_n;
            const uint32_t lane_addr = tmem_base + (uint32_t)(b * p.tile_n) + ((uint32_t)(q * 32) << 16);
            const bool live = row < p.rows;
            const uint8_t* res = p.residual
                ? reinterpret_cast<const uint8_t*>(p.residual + (live ? row : 0) * (int64_t)p.cout + n0)
                : nullptr;
            const int n_box = p.tile_n / 64;
            for (int bx = h; bx < n_box; bx += 2) {
                // the box's residual (64 values of this row) is loaded up front, so its latency
                // overlaps the TMEM loads and the staging wait
                uint4 rbox[8];
                if (res && live) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) rbox[i] = __ldg(reinterpret_cast<const uint4*>(res + bx * 128) + i);
                }
                if (lane == 0) bulk_wait_read_all();  // the previous box's store has read the staging
                __syncwarp();
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int c = bx * 64 + half * 32;
                    float v[32];
                    tmem_ld32(lane_addr + c, v);
                    if (p.bias) add_param32(v, p.bias + n0 + c, false);
                    if (res && live) {
#pragma unroll
                        for (int qq = 0; qq < 4; ++qq) {
                            float r[8];
                            load_bf16x8(reinterpret_cast<const uint8_t*>(&rbox[4 * half + qq]), r);
#pragma unroll
                            for (int k = 0; k < 8; ++k) v[8 * qq + k] += r[k];
                        }
                    }
                    if (p.silu) {
#pragma unroll
                        for (int k = 0; k < 32; ++k) v[k] = silu_bf16out(v[k]);
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        cvt_store_bf16x8(es + lane * 128 + (((4 * half + u) ^ (lane & 7)) << 4), v + 8 * u);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&omap, smem_u32(es), n0 + bx * 64, (int)row0);
                    bulk_commit();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[b]);
        }
        if (lane == 0) bulk_wait_all();  // every output box written before the CTA leaves
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TC_TMEM_COLS);
    }
}

}  // namespace sc
