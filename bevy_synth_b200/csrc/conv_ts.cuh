// conv_ts.cuh -- sm_100a tensor-core SubM conv for 64 input channels with the
// A operand built in tensor memory from each tile's unique source rows.
//
// Math as conv_tc_kernel (reference burn_flex_gmm src/lib.rs:242-375):
//     out[r, o] = bias[o] + sum_k sum_c in[nbr[r,k], c] * W[o, k, c]
// With Cin = 64 a tap is one 64-channel reduction step, and the step's A tile
// (128 rows x 64 channels, 16 KB) is what the generic kernel gathers from L2
// for every tap: 2,279 row gathers for a 128-row tile of the config-5 grid.
// In Morton order those rows come from only ~269 distinct source rows (8.5x
// reuse).  This kernel gathers each tile's distinct rows ONCE into shared
// memory and builds every tap's A tile in tensor memory (tcgen05.st) from
// there; tcgen05.mma then reads A from TMEM and B (the weights) from shared
// memory, so the per-tap shared-memory traffic is the 16 KB read of the staged
// rows plus B.
//
// Per-tile source lists come from a prepass over the neighbor map
// (ts_tile_sources_kernel, once per map): the sorted distinct valid source rows
// of the tile, a 16-bit local index per (row, tap) into that list (0xFFFF =
// no neighbor), and the tile's tap mask.
//
// Warp roles (18 warps, one CTA per SM, persistent, static round-robin over
// (row tile, column tile) pairs -- Morton tiles carry near-uniform work):
//   0-3   epilogue: TMEM accumulator -> + bias -> [SiLU] -> bf16 rows (plain
//         16-byte stores: the TMA unit is left to the weight loads);
//   4-11  A builders, two groups of four (one warp per TMEM sub-partition in
//         each) taking alternate taps: thread = tile row; per tap it reads its
//         row's 128-byte source row from the staging buffer and stores it as
//         32 TMEM columns of an A slot (a store and its wait are a latency
//         chain, so two warps per sub-partition interleave);
//   12-15 staging: cp.async gather of the tile's distinct rows (XOR-swizzled
//         16-byte chunks) and of its local index block; double-buffered when
//         shared memory allows, else single (the A slots give the gather of
//         the next tile a lead of up to the A slots' taps);
//   16    B loader: one lane issues the weight tile TMA of every tap;
//   17    MMA: whole warp runs the loop, one elected lane issues
//         tcgen05.mma (A from TMEM, M=128, N=tile_n, K=16) and the commits.
// TMEM: double-buffered accumulators in columns [0, 2 tile_n) and the A slots
// (32 columns each) in the rest: 12 for 64 outputs, 8 for 128.
// Every wait is bounded (device wait limit); on expiry the fault word is
// raised and the roles drain.
#pragma once

#include "conv_tc.cuh"

namespace sc {

constexpr int TS_UMAX = 576;      // distinct source rows a tile may have (staging capacity bound)
constexpr int TS_NA_MAX = 12;     // A slots in TMEM (32 columns each) at most
constexpr int TS_THREADS = 18 * 32;
constexpr int TS_EPI0 = 0, TS_BLD0 = 4, TS_STG0 = 12, TS_BLOADER = 16, TS_MMA = 17;
constexpr uint16_t TS_NONE = 0xFFFF;
constexpr int TS_EPI_BYTES = 4 * 32 * 128;  // TMA epilogue staging: one 32-row x 64-column bf16 box per warp

// ---- prepass: per-tile distinct source rows -----------------------------------
// Layout of the tile-source plan (one buffer):
//   [0, 64)                       header: int32 n_tiles, K, max distinct rows, overflow tiles
//   u_count [n_tiles] int32, tap_mask [n_tiles] uint32 (each padded to 16 bytes)
//   u_rows  [n_tiles][TS_UMAX] int32 (sorted distinct source rows)
//   lidx    [n_tiles][128][K] uint16 (local index into u_rows, TS_NONE = none)
struct TsPlanView {
    int32_t* header;
    int32_t* u_count;
    uint32_t* tap_mask;
    int32_t* u_rows;
    uint16_t* lidx;
};

__host__ __device__ inline size_t ts_align16(size_t b) { return (b + 15) / 16 * 16; }

__host__ __device__ inline size_t ts_plan_bytes(int64_t n_tiles, int K) {
    return 64 + 2 * ts_align16((size_t)n_tiles * 4) + (size_t)n_tiles * TS_UMAX * 4 +
           ts_align16((size_t)n_tiles * 128 * K * 2);
}

__host__ __device__ inline TsPlanView ts_plan_view(void* base, int64_t n_tiles) {
    uint8_t* b = static_cast<uint8_t*>(base);
    TsPlanView v;
    v.header = reinterpret_cast<int32_t*>(b);
    size_t off = 64;
    v.u_count = reinterpret_cast<int32_t*>(b + off);
    off += ts_align16((size_t)n_tiles * 4);
    v.tap_mask = reinterpret_cast<uint32_t*>(b + off);
    off += ts_align16((size_t)n_tiles * 4);
    v.u_rows = reinterpret_cast<int32_t*>(b + off);
    off += (size_t)n_tiles * TS_UMAX * 4;
    v.lidx = reinterpret_cast<uint16_t*>(b + off);
    return v;
}

constexpr int TSP_THREADS = 256;
constexpr int TSP_HASH = 4096;   // open-addressing slots (>= 128 * 32 entries)
constexpr int TSP_SORT = 1024;   // sort width (>= TS_UMAX, power of two)

// One CTA per 128-row tile: distinct valid neighbor ids of the tile's rows
// (hash set in shared memory), sorted ascending, then each (row, tap)'s index
// into the sorted list.  Tiles with more than TS_UMAX distinct rows are
// counted in header[3]; their plan entries are not usable.
__global__ void __launch_bounds__(TSP_THREADS) ts_tile_sources_kernel(const int32_t* __restrict__ nbr, int64_t n_rows,
                                                                      int K, int64_t n_in, void* plan_base,
                                                                      int64_t n_tiles) {
    __shared__ int32_t keys[TSP_HASH];
    __shared__ int16_t pos[TSP_HASH];
    __shared__ int32_t uniq[TSP_SORT];
    __shared__ int32_t count;
    __shared__ uint32_t mask;
    const TsPlanView v = ts_plan_view(plan_base, n_tiles);
    const int64_t t = blockIdx.x;
    const int tid = threadIdx.x;
    for (int i = tid; i < TSP_HASH; i += TSP_THREADS) keys[i] = -1;
    for (int i = tid; i < TSP_SORT; i += TSP_THREADS) uniq[i] = 0x7fffffff;
    if (tid == 0) {
        count = 0;
        mask = 0;
    }
    __syncthreads();
    const int64_t r0 = t * 128;
    const int n_ent = 128 * K;
    for (int i = tid; i < n_ent; i += TSP_THREADS) {
        const int rr = i / K, k = i - rr * K;
        const int64_t row = r0 + rr;
        int32_t id = row < n_rows ? __ldg(nbr + row * K + k) : -1;
        if (id < -1 || id >= n_in) {
            raise_fault(FAULT_BAD_NEIGHBOR);
            id = -1;
        }
        if (id < 0) continue;
        atomicOr(&mask, 1u << k);
        uint32_t h = ((uint32_t)id * 2654435761u) & (TSP_HASH - 1);
        for (int probe = 0; probe < TSP_HASH; ++probe) {
            const int32_t prev = atomicCAS(&keys[h], -1, id);
            if (prev == -1) {
                const int p = atomicAdd(&count, 1);
                if (p < TSP_SORT) uniq[p] = id;
                break;
            }
            if (prev == id) break;
            h = (h + 1) & (TSP_HASH - 1);
        }
    }
    __syncthreads();
    const int cnt = count;
    if (cnt > TS_UMAX) {
        if (tid == 0) {
            v.u_count[t] = cnt;
            v.tap_mask[t] = mask;
            atomicAdd(&v.header[3], 1);
            atomicMax(&v.header[2], cnt);
        }
        return;
    }
    // bitonic sort of uniq[0, TSP_SORT) (padding INT_MAX sorts last)
    for (int size = 2; size <= TSP_SORT; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < TSP_SORT / 2; i += TSP_THREADS) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const int32_t a = uniq[lo], b = uniq[hi];
                if ((a > b) == up) {
                    uniq[lo] = b;
                    uniq[hi] = a;
                }
            }
            __syncthreads();
        }
    }
    // sorted position of every distinct id, back into the hash set
    for (int p = tid; p < cnt; p += TSP_THREADS) {
        const int32_t id = uniq[p];
        uint32_t h = ((uint32_t)id * 2654435761u) & (TSP_HASH - 1);
        for (int probe = 0; probe < TSP_HASH; ++probe) {
            if (keys[h] == id) {
                pos[h] = (int16_t)p;
                break;
            }
            h = (h + 1) & (TSP_HASH - 1);
        }
        v.u_rows[t * TS_UMAX + p] = id;
    }
    __syncthreads();
    uint16_t* lid = v.lidx + t * 128 * (int64_t)K;
    for (int i = tid; i < n_ent; i += TSP_THREADS) {
        const int rr = i / K, k = i - rr * K;
        const int64_t row = r0 + rr;
        int32_t id = row < n_rows ? __ldg(nbr + row * K + k) : -1;
        uint16_t out = TS_NONE;
        if (id >= 0 && id < n_in) {
            uint32_t h = ((uint32_t)id * 2654435761u) & (TSP_HASH - 1);
            for (int probe = 0; probe < TSP_HASH; ++probe) {
                if (keys[h] == id) {
                    out = (uint16_t)pos[h];
                    break;
                }
                h = (h + 1) & (TSP_HASH - 1);
            }
        }
        lid[i] = out;
    }
    if (tid == 0) {
        v.u_count[t] = cnt;
        v.tap_mask[t] = mask;
        atomicMax(&v.header[2], cnt);
    }
}

// ---- the conv kernel ---------------------------------------------------------
struct TsParams {
    const __nv_bfloat16* in;
    int64_t n_in;
    int64_t n_rows;
    int K;
    const int32_t* u_count;
    const uint32_t* tap_mask;
    const int32_t* u_rows;
    const uint16_t* lidx;
    const float* bias;
    int silu;
    __nv_bfloat16* out;
    int cout;
    int tile_n;      // output columns per tile (multiple of 32, <= 256)
    int n_buf;       // accumulator buffers (2 when tile_n <= 128)
    int n_stg;       // staging buffers (1 or 2)
    int grid_y;      // column tiles per row tile
    int64_t n_tiles; // row tiles * grid_y
    int u_cap;       // staging rows per buffer (multiple of 8, >= every tile's distinct rows)
    int b_stages;    // weight slots (a multiple of grp)
    int grp;         // taps per pipeline step (G): 4 for tile_n <= 64, else 2
    int n_a;         // A slots (a multiple of grp, <= TS_NA_MAX)
    int a_col0;      // first TMEM column of the A slots (n_buf * tile_n)
    int tma_epi;     // 1: outputs by TMA tile stores of 32 rows x 64 columns (omap), tile_n % 64 == 0
};

// Named barrier 1 over the four staging warps (128 threads).
__device__ __forceinline__ void stg_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The same barrier with an OR reduction: true if `fail` is set in any of the 128 threads,
// so the staging warps leave their loop together (no thread is left waiting at the barrier).
__device__ __forceinline__ bool stg_bar_any(bool fail) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)fail)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ uint32_t ts_mask_of(const TsParams& p, int64_t row_tile) {
    const uint32_t m = __ldg(p.tap_mask + row_tile);
    return m ? m : 1u;  // a tile with no valid tap still runs one (all-zero) step
}

__global__ void __launch_bounds__(TS_THREADS, 1) conv_ts_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                 const __grid_constant__ CUtensorMap omap,
                                                                 const TsParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const int K = p.K;
    const int S = p.b_stages;
    const int NS = p.n_stg;
    const int B_BYTES = p.tile_n * 128;
    uint8_t* stg = smem;                                                 // [NS][u_cap][128]
    uint8_t* b_smem = stg + NS * (size_t)p.u_cap * 128;                  // [S][tile_n][128] (1024-aligned)
    uint8_t* lid_s = b_smem + (size_t)S * B_BYTES;                       // [NS][128 * K] uint16
    const int LID_BYTES = 128 * K * 2;
    int32_t* ulist = reinterpret_cast<int32_t*>(lid_s + NS * LID_BYTES);   // [2][TS_UMAX] source-row lists
    // [4][32 rows][128 B] TMA epilogue staging (1024-aligned: the 128-byte swizzle of the output map)
    uint8_t* epi_s = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(ulist + 2 * TS_UMAX) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(p.tma_epi ? epi_s + TS_EPI_BYTES : (uint8_t*)(ulist + 2 * TS_UMAX));
    uint64_t* stg_full = bars;            // [2]
    uint64_t* stg_empty = bars + 2;       // [2]
    uint64_t* a_full = bars + 4;              // [TS_NA_MAX]
    uint64_t* a_empty = a_full + TS_NA_MAX;   // [TS_NA_MAX]
    uint64_t* b_full = a_empty + TS_NA_MAX;   // [S]
    uint64_t* b_empty = b_full + S;       // [S]
    uint64_t* tmem_full = b_empty + S;    // [2]
    uint64_t* tmem_empty = tmem_full + 2; // [2]
    uint32_t* misc = reinterpret_cast<uint32_t*>(tmem_empty + 2);  // [0] tmem base

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t n_ctas = gridDim.x;
    auto tile_of = [&](int64_t lt) -> int64_t {
        const int64_t t = (int64_t)blockIdx.x + lt * n_ctas;
        return t < p.n_tiles ? t : -1;
    };

    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&stg_full[b], 128);     // every staging thread's cp.async arrive
            mbar_init(&stg_empty[b], 8);      // the eight builder warps
            mbar_init(&tmem_full[b], 1);      // tcgen05.commit after the tile's last MMA
            mbar_init(&tmem_empty[b], 4);     // the four epilogue warps
        }
        for (int s = 0; s < TS_NA_MAX; ++s) {
            mbar_init(&a_full[s], 4);         // the four warps of the slot group's builder group
            mbar_init(&a_empty[s], 1);        // tcgen05.commit
        }
        for (int s = 0; s < S; ++s) {
            mbar_init(&b_full[s], 1);         // the loader's expect_tx arrive
            mbar_init(&b_empty[s], 1);        // tcgen05.commit
        }
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    if (warp == TS_MMA) {
        tmem_alloc(&misc[0], TC_TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == TS_BLOADER && lane == 0) tma_prefetch_desc(&wmap);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = misc[0];

    if (warp >= TS_STG0 && warp < TS_STG0 + 4) {
        // ====================================================== staging
        // 8 lanes per source row (one 16-byte chunk each), 16 rows per pass of the 128 threads.
        // The next tile's source-row list (TS_UMAX int32) is copied into shared memory a tile
        // ahead (cp.async group + a named barrier of the four staging warps), so the row
        // copies issue with no dependent global index loads on their path.
        const int sid = tid - TS_STG0 * 32;
        const int c = sid & 7;
        constexpr int UCHUNKS = TS_UMAX * 4 / 16;
        auto fetch_list = [&](int64_t tt, int ib) {
            if (tt < 0) return;
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.u_rows + (tt / p.grid_y) * TS_UMAX);
            const uint32_t dst = smem_u32(ulist + ib * TS_UMAX);
            for (int q = sid; q < UCHUNKS; q += 128) cp_async_16(dst + q * 16, src + q * 16, 16u);
        };
        int64_t t = tile_of(0);
        fetch_list(t, 0);
        cp_async_commit();
        int cnt_next = t >= 0 ? __ldg(p.u_count + t / p.grid_y) : 0;
        cp_async_wait<0>();
        stg_bar_sync();
        for (int64_t lt = 0; t >= 0; ++lt) {
            const int sb = (int)(lt % NS);
            const uint32_t use = (uint32_t)(lt / NS);
            const int ib = (int)(lt & 1);
            const int64_t rt = t / p.grid_y;
            int cnt = cnt_next;
            const int64_t t_next = tile_of(lt + 1);
            fetch_list(t_next, ib ^ 1);   // the next tile's list, behind this tile's copies
            cp_async_commit();
            if (t_next >= 0) cnt_next = __ldg(p.u_count + t_next / p.grid_y);
            const bool fail = !mbar_wait(&stg_empty[sb], (use & 1u) ^ 1u);
            if (!fail) {
                if (cnt > p.u_cap) {  // the host checks the plan's maximum; never taken for a valid plan
                    raise_fault(FAULT_BAD_NEIGHBOR);
                    cnt = p.u_cap;
                }
                const uint32_t base = smem_u32(stg + (size_t)sb * p.u_cap * 128);
                const int32_t* ul = ulist + ib * TS_UMAX;
                for (int u = sid >> 3; u < cnt; u += 16) {
                    const int32_t src = ul[u];
                    const bool ok = src >= 0 && src < p.n_in;
                    if (!ok) raise_fault(FAULT_BAD_NEIGHBOR);
                    const void* g = ok ? (const void*)(p.in + (int64_t)src * 64 + c * 8) : (const void*)p.in;
                    cp_async_16(base + u * 128 + ((c ^ (u & 7)) << 4), g, ok ? 16u : 0u);
                }
                const uint32_t lbase = smem_u32(lid_s + sb * LID_BYTES);
                const uint8_t* lsrc = reinterpret_cast<const uint8_t*>(p.lidx + rt * 128 * (int64_t)K);
                for (int q = sid; q < LID_BYTES / 16; q += 128) cp_async_16(lbase + q * 16, lsrc + q * 16, 16u);
                cp_async_arrive_noinc(&stg_full[sb]);
            }
            cp_async_wait<0>();             // the next tile's list (committed groups; this tile's copies
            if (stg_bar_any(fail)) break;   // are tracked by the stage barrier), seen by all four warps
            t = t_next;
        }
        cp_async_wait<0>();
    } else if (warp >= TS_BLD0 && warp < TS_BLD0 + 8) {
        // ====================================================== A builders
        // Taps run in steps of G (the tile's taps in mask order, G per step, the last step of a
        // tile possibly shorter); the two builder groups take alternate steps, each step into
        // the next of the n_a / G slot groups, with one empty wait and one full arrive.  A step's
        // TMEM stores are issued back to back and completed by one wait before the arrive, so
        // the shared-memory reads of a tap overlap the previous tap's store.
        const int q = warp & 3;                 // TMEM sub-partition (warp id % 4)
        const uint32_t grp = (uint32_t)((warp - TS_BLD0) >> 2);
        const int r = q * 32 + lane;            // tile row == TMEM lane
        const int G = p.grp;
        const uint32_t NAG = (uint32_t)(p.n_a / G);
        const uint32_t lane_cols = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)p.a_col0;
        uint32_t stp = 0;                       // steps of the sequence (both groups)
        uint32_t mask_next = tile_of(0) >= 0 ? ts_mask_of(p, tile_of(0) / p.grid_y) : 0u;
        for (int64_t lt = 0;; ++lt) {
            const int64_t t = tile_of(lt);
            if (t < 0) break;
            const int sb = (int)(lt % NS);
            const uint32_t use = (uint32_t)(lt / NS);
            const uint32_t mask = mask_next;   // the tile's tap mask, read a tile ahead
            if (tile_of(lt + 1) >= 0) mask_next = ts_mask_of(p, tile_of(lt + 1) / p.grid_y);
            if (!__all_sync(0xffffffffu, mbar_wait(&stg_full[sb], use & 1u))) break;
            const uint16_t* lid = reinterpret_cast<const uint16_t*>(lid_s + sb * LID_BYTES) + r * K;
            const uint8_t* sbase = stg + (size_t)sb * p.u_cap * 128;
            bool ok = true;
            for (uint32_t m = mask; m; ++stp) {
                if ((stp & 1u) != grp) {        // the other group's step: skip its taps
                    for (int i = 0; i < G && m; ++i) m &= m - 1;
                    continue;
                }
                const uint32_t ag = stp % NAG;
                if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[ag], ((stp / NAG) & 1u) ^ 1u))) {
                    ok = false;
                    break;
                }
                tc_fence_after();  // the MMAs that read these slots are complete before they are rewritten
#pragma unroll 1
                for (int i = 0; i < G && m; ++i, m &= m - 1) {
                    const int k = __ffs(m) - 1;
                    const uint32_t idx = lid[k];
                    float v[32];
                    if (idx < (uint32_t)p.u_cap) {
                        const uint8_t* row = sbase + idx * 128;
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) {
                            const uint4 w4 = *reinterpret_cast<const uint4*>(row + ((cc ^ (idx & 7)) << 4));
                            v[4 * cc] = __uint_as_float(w4.x);
                            v[4 * cc + 1] = __uint_as_float(w4.y);
                            v[4 * cc + 2] = __uint_as_float(w4.z);
                            v[4 * cc + 3] = __uint_as_float(w4.w);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = 0.f;
                    }
                    tmem_st32_async(lane_cols + (uint32_t)((ag * G + i) * 32), v);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[ag]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&stg_empty[sb]);  // this warp no longer reads the staged rows
            if (!ok) break;
        }
    } else if (warp == TS_BLOADER) {
        // ====================================================== B loader
        // One weight slot group (G slots, one transaction barrier) per step.
        if (lane == 0) {
            const int G = p.grp;
            const uint32_t NBG = (uint32_t)(S / G);
            uint32_t stp = 0;
            bool ok = true;
            uint32_t mask_next = tile_of(0) >= 0 ? ts_mask_of(p, tile_of(0) / p.grid_y) : 0u;
            for (int64_t lt = 0; ok; ++lt) {
                const int64_t t = tile_of(lt);
                if (t < 0) break;
                const int n0 = (int)(t % p.grid_y) * p.tile_n;
                const uint32_t mask = mask_next;
                if (tile_of(lt + 1) >= 0) mask_next = ts_mask_of(p, tile_of(lt + 1) / p.grid_y);
                for (uint32_t m = mask; m; ++stp) {
                    const uint32_t bg = stp % NBG;
                    if (!mbar_wait(&b_empty[bg], ((stp / NBG) & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    const int g = min(G, __popc(m));
                    mbar_arrive_expect_tx(&b_full[bg], (uint32_t)(g * B_BYTES));
                    for (int i = 0; i < g; ++i, m &= m - 1)
                        tma_load_3d(smem_u32(b_smem + (size_t)(bg * G + i) * B_BYTES), &wmap, &b_full[bg], 0,
                                    __ffs(m) - 1, n0);
                }
            }
        }
    } else if (warp == TS_MMA) {
        // ====================================================== MMA issuer
        const bool issuer = elect_one();
        const uint32_t idesc = umma_idesc_bf16_m128((uint32_t)p.tile_n);
        const uint64_t bdesc0 = umma_desc_sw128(smem_u32(b_smem));
        const int G = p.grp;
        const uint32_t NAG = (uint32_t)(p.n_a / G), NBG = (uint32_t)(S / G);
        uint32_t stp = 0;
        bool ok = true;
        uint32_t mask_next = tile_of(0) >= 0 ? ts_mask_of(p, tile_of(0) / p.grid_y) : 0u;
        for (int64_t lt = 0; ok; ++lt) {
            const int64_t t = tile_of(lt);
            if (t < 0) break;
            const int b = p.n_buf == 2 ? (int)(lt & 1) : 0;
            const uint32_t use = (uint32_t)(p.n_buf == 2 ? (lt >> 1) : lt);
            const uint32_t mask = mask_next;
            if (tile_of(lt + 1) >= 0) mask_next = ts_mask_of(p, tile_of(lt + 1) / p.grid_y);
            if (!__all_sync(0xffffffffu, mbar_wait(&tmem_empty[b], (use & 1u) ^ 1u))) break;
            tc_fence_after();
            const uint32_t acc = tmem_base + (uint32_t)(b * p.tile_n);
            bool first = true;
            for (uint32_t m = mask; m; ++stp) {
                const uint32_t ag = stp % NAG, bg = stp % NBG;
                if (!__all_sync(0xffffffffu, mbar_wait(&a_full[ag], (stp / NAG) & 1u)) ||
                    !__all_sync(0xffffffffu, mbar_wait(&b_full[bg], (stp / NBG) & 1u))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int g = min(G, __popc(m));
                if (issuer) {
                    for (int i = 0; i < g; ++i) {
                        const uint64_t bd = bdesc0 + (uint64_t)(((bg * G + i) * B_BYTES) >> 4);
                        const uint32_t at = tmem_base + (uint32_t)(p.a_col0 + (ag * G + i) * 32);
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; ++kk)
                            umma_bf16_ts(acc, at + (uint32_t)(kk * 8), bd + (uint64_t)(kk * 2), idesc,
                                         (first && i == 0 && kk == 0) ? 0u : 1u);
                    }
                    umma_commit(&a_empty[ag]);
                    umma_commit(&b_empty[bg]);
                }
                __syncwarp();
                first = false;
                for (int i = 0; i < g; ++i) m &= m - 1;
            }
            if (!ok) break;
            if (issuer) umma_commit(&tmem_full[b]);
            __syncwarp();
        }
    } else if (warp < 4) {
        // ====================================================== epilogue
        // Thread = tile row.  Plain mode: each 32-column TMEM load becomes four 16-byte global
        // stores of the row.  (Measured: routing the stores through a shared-memory transpose so
        // that every store instruction writes whole 64-byte row segments made the drain slower,
        // 2,989 -> 4,053 cycles a 64-column tile.)  TMA mode (tma_epi, the single-buffered wide
        // accumulator, whose drain the MMAs wait for): 64 columns at a time, the warp writes its
        // 32 rows into a 128B-swizzled 4 KB box and one lane stores the box with a tiled TMA
        // store; the next box waits until that store has read the staging.  The accumulator is
        // released once its last columns are in registers.
        uint8_t* es = epi_s + warp * 32 * 128;
        for (int64_t lt = 0;; ++lt) {
            const int64_t t = tile_of(lt);
            if (t < 0) break;
            const int b = p.n_buf == 2 ? (int)(lt & 1) : 0;
            const uint32_t use = (uint32_t)(p.n_buf == 2 ? (lt >> 1) : lt);
            if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[b], use & 1u))) break;
            tc_fence_after();
            const int64_t rt = t / p.grid_y;
            const int n0 = (int)(t % p.grid_y) * p.tile_n;
            const int64_t row = rt * 128 + tid;
            const uint32_t lane_addr = tmem_base + (uint32_t)(b * p.tile_n) + ((uint32_t)(warp * 32) << 16);
            if (p.tma_epi) {
                for (int c = 0; c < p.tile_n; c += 64) {
                    if (lane == 0) bulk_wait_read_all();  // the previous box's store has read the staging
                    __syncwarp();
#pragma unroll 1
                    for (int h = 0; h < 2; ++h) {  // 32 columns at a time: chunks 4h .. 4h + 3 of the box rows
                        float v[32];
                        tmem_ld32(lane_addr + c + 32 * h, v);
                        if (c + 32 * h + 32 >= p.tile_n) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&tmem_empty[b]);
                        }
                        if (p.bias) add_param32(v, p.bias + n0 + c + 32 * h, false);
                        if (p.silu) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] = silu_bf16out(v[e]);
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            cvt_store_bf16x8(es + lane * 128 + (((4 * h + u) ^ (lane & 7)) << 4), v + 8 * u);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&omap, smem_u32(es), n0 + c, (int)(rt * 128 + warp * 32));
                        bulk_commit();
                    }
                }
                continue;
            }
            uint8_t* dst = reinterpret_cast<uint8_t*>(p.out + (row < p.n_rows ? row : 0) * (int64_t)p.cout + n0);
            for (int c = 0; c < p.tile_n; c += 32) {
                float v[32];
                tmem_ld32(lane_addr + c, v);
                if (c + 32 >= p.tile_n) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[b]);
                }
                if (p.bias) add_param32(v, p.bias + n0 + c, false);
                if (p.silu) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = silu_bf16out(v[e]);
                }
                if (row < p.n_rows) {
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) cvt_store_bf16x8(dst + (c + 8 * qq) * 2, v + 8 * qq);
                }
            }
        }
        if (p.tma_epi && lane == 0) bulk_wait_all();  // every output box written before the CTA leaves
    }

    tc_fence_before();
    __syncthreads();
    if (warp == TS_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TC_TMEM_COLS);
    }
}

// Dynamic shared memory of a launch (1 KB alignment slack included).
inline size_t ts_smem_bytes(int u_cap, int tile_n, int K, int b_stages, int n_stg, bool tma_epi = false) {
    return 1024 + (size_t)n_stg * u_cap * 128 + (size_t)b_stages * tile_n * 128 + (size_t)n_stg * 128 * K * 2 +
           2 * TS_UMAX * 4 + (tma_epi ? 1024 + TS_EPI_BYTES : 0) + (size_t)(4 + 2 * TS_NA_MAX + 2 * b_stages + 4) * 8 + 16;
}

}  // namespace sc
