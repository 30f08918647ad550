// conv_tc.cuh -- sm_100a tensor-core (tcgen05) implicit gather-GEMM for the
// sparse submanifold convolution, with the bias / residual / LayerNorm / SiLU
// epilogue fused on the TMEM accumulator.
//
// Math (reference: burn_flex_gmm src/lib.rs:242-375 and the device kernels
// src/wgpu/sparse_conv_kernels.rs:4-46):
//     out[r, o] = bias[o] + sum_k sum_c in[nbr[r,k], c] * W[o, k, c]
// computed as a GEMM with M = output rows (tiles of 128), N = output channels
// (tiles of up to 512) and the reduction over (tap k, 64-channel chunk) steps:
//   * A (128 x 64 bf16 per step) is GATHERED from the neighbor rows nbr[r,k]
//     with 16-byte cp.async into a 128B-swizzled K-major smem tile; every copy
//     instruction moves whole 128-byte row slices (zero fill for invalid
//     neighbors and for channels >= Cin);
//   * B (tile_n x 64 bf16 per step) is W[n0:n0+tile_n, k, c0:c0+64], loaded by
//     TMA from the reference layout [Cout, 27, Cin] (3-D tensor map, 128B
//     swizzle, OOB zero fill);
//   * tcgen05.mma (M=128, N<=256 per instruction, K=16) accumulates in fp32
//     TMEM; taps that are invalid for every row of a tile are skipped.
//
// Warp-specialised CTA, one per SM.  The single-CTA kernel is launched with
// one CTA per tile; a running CTA claims the tiles of CTAs that have not
// started (cluster launch control), so tiles spread dynamically, largest
// first.  Roles:
//   warps 0-3          epilogue: thread i owns TMEM lane / tile row i; output
//                      and residual rows move through padded smem staging so
//                      that global accesses are whole coalesced rows;
//   warps 4..4+PW-1    A gather producers (PW = 4 or 8: one or two per SM
//                      sub-partition); each reads its rows' map block one tile
//                      ahead; the weight TMA of a stage is issued by one
//                      producer lane in rotation (warp 4 in the full instance),
//                      the launch-control requests by warp 4 lane 0;
//   warp 4+PW          MMA warp: the whole warp runs the loop, one elected
//                      lane issues tcgen05.mma and the commits.
// Optionally (SC_TC_GATHER4=1) A rows arrive by TMA tile::gather4 instead of
// cp.async; on B200 that measured slower for 128-byte rows.
// The accumulator is double-buffered in TMEM (2 x 256 columns) when
// tile_n <= 256, so the epilogue of one tile overlaps the MMAs of the next.
//
// PAIR (2-SM) variant (the default for multi-tap convs with Cin, Cout <= 64;
// SC_TC_PAIR=0|1 turns it off / on elsewhere; persistent grid with static
// round-robin tiles), launched as clusters of two CTAs: a tile is 256 rows,
// 128 per CTA; the leader issues tcgen05.mma.cta_group::2 with M = 256, each
// CTA's A from its own shared memory and B split by N across the pair, so a
// CTA loads and the tensor cores read only half of every weight tile.  Both
// halves of B arrive by TMA on the leader's full barrier; the peer's "A
// landed" is relayed by its otherwise idle MMA warp (one lane per stage slot);
// commits are multicast to both CTAs.  (Measured: a peer gathering by TMA
// gather4 instead, with no relay, was slower.)
// Every mbarrier wait is bounded: on expiry the device fault word is raised
// and the CTA drains and exits instead of hanging.
#pragma once

#include "sc_common.cuh"

namespace sc {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;                      // channels per reduction step
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KB
// Gather producer warps (a kernel template parameter, 4 or 8): one or two per SM
// sub-partition.  A producer warp's per-stage instruction stream (empty wait, row
// indices, address math, copies, arrive) is latency-bound, so the stage rate of a
// 3x3x3 conv scales with the warps that interleave on a sub-partition; 8 warps
// leave 128 registers a thread (13 warps, 4 on one sub-partition), which the 1x1
// (linear) convs, epilogue-bound, do not trade for.
constexpr int TC_PW_MAX = 8;
__host__ __device__ constexpr int tc_threads(int pw) { return (4 + pw + 1) * 32; }
constexpr int TC_MAX_K = 32;
constexpr int TC_STG_COLS = 128;               // epilogue staging width (columns)
constexpr int TC_SCHED = 4;                    // launch-control responses in flight (ring)
constexpr uint32_t TC_TMEM_COLS = 512;

struct TcParams {
    const __nv_bfloat16* in;
    int64_t n_in;
    int cin;
    const int32_t* nbr;
    int64_t n_rows;
    int K;
    const float* bias;
    int cout;
    int tile_n;   // output columns per tile (multiple of 32, <= 512)
    int n_sub;    // MMAs per reduction step (1 or 2)
    int sub_n;    // N of each MMA (= TMA box rows), tile_n = n_sub * sub_n
    int stages;
    int n_buf;    // TMEM accumulator buffers (2 when tile_n <= 256)
    int grid_y;   // column tiles per row tile
    int64_t n_tiles;
    int dynamic;  // 1: one CTA per tile, CTAs claim unlaunched tiles by cluster launch control
    int tma_epi;  // 1: staging is TMA-swizzled (64 columns); outputs by scatter4 (omap, o2map), dense residual by gather4 (rmap)
    int gather4;  // 1: A rows gathered by TMA (tile::gather4 on `amap`) instead of cp.async; 2: half of them
    int stg_cols; // epilogue staging width: a multiple of 32 dividing tile_n, <= TC_STG_COLS
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
    const int32_t* row_order;    // nullable: tile position -> output row (a permutation)
    const int32_t* nbr_ordered;  // nullable: nbr rows in tile order (nbr[row_order[p]])
    int test_stall;              // test only (single CTA): the MMA warp waits on a barrier nothing completes
};

// Output row processed at tile position `pos` (< n_rows), or -1 if invalid.
__device__ __forceinline__ int64_t ordered_row(const int32_t* order, int64_t pos, int64_t n_rows) {
    if (!order) return pos;
    const int32_t r = __ldg(order + pos);
    if (r < 0 || r >= n_rows) {
        raise_fault(FAULT_BAD_NEIGHBOR);
        return -1;
    }
    return r;
}

__device__ __forceinline__ void cvt_store_bf16x8(uint8_t* dst, const float* v) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(dst) = u;
}

__device__ __forceinline__ void load_bf16x8(const uint8_t* src, float* v) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
    }
}

// Epilogue staging of one warp: 32 rows of `units` 16-byte units, padded by
// one unit per row so that the owning thread's row writes and the warp's
// row-wide reads are both free of bank conflicts.
// A warp's staging buffer: 32 rows of `units` 16-byte chunks.  Padded rows
// (one spare chunk per row) for per-row bulk copies; or, with swz (units ==
// 8), dense 128-byte rows in the TMA 128B swizzle (chunk u of row r at
// r*128 + ((u ^ (r & 7)) * 16), base 1024-aligned) for gather4 / scatter4.
struct Staging {
    uint8_t* base;
    int units;
    int swz;
    __device__ __forceinline__ uint8_t* at(int r, int u) const {
        return swz ? base + r * 128 + ((u ^ (r & 7)) << 4) : base + (r * (units + 1) + u) * 16;
    }
};

// Lane's staged row -> global row orow (< 0: skipped), columns [col0,
// col0 + 8*units) of a row-major matrix with leading dimension ld, as one
// bulk copy (TMA engine, no load/store-unit traffic).  The staged row was
// written by this lane; callers wait for the copy's reads (stg_reuse) before
// writing the staging buffer again.
__device__ __forceinline__ void store_staged_rows(const Staging& st, int64_t orow, __nv_bfloat16* dst,
                                                  int64_t ld, int col0, int lane) {
    fence_proxy_async_smem();  // this lane's staging writes -> the bulk copy's reads
    if (orow >= 0) bulk_store(dst + orow * ld + col0, smem_u32(st.at(lane, 0)), (uint32_t)(st.units * 16));
    bulk_commit();
}

// The staging buffer may be written again: this lane's bulk stores have read it.
__device__ __forceinline__ void stg_reuse() {
    bulk_wait_read_all();
    __syncwarp();  // lanes whose copies read other lanes' staged rows have waited too
}

// Global row rrow (per lane = row; < 0 gives zeros) -> the lane's staged row,
// by bulk copy completing on the warp's barrier `bar` (phase `ph`, flipped).
__device__ __forceinline__ bool load_staged_rows(const Staging& st, int64_t rrow, const __nv_bfloat16* src,
                                                 int64_t ld, int col0, int lane, uint64_t* bar, uint32_t& ph) {
    const uint32_t bytes = (uint32_t)(st.units * 16);
    const uint32_t n_rows = (uint32_t)__popc(__ballot_sync(0xffffffffu, rrow >= 0));
    if (lane == 0) mbar_arrive_expect_tx(bar, n_rows * bytes);
    __syncwarp();
    if (rrow >= 0) {
        bulk_load(smem_u32(st.at(lane, 0)), src + rrow * ld + col0, bytes, bar);
    } else {
        for (int u = 0; u < st.units; ++u) *reinterpret_cast<uint4*>(st.at(lane, u)) = make_uint4(0, 0, 0, 0);
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, ph));
    ph ^= 1u;
    return ok;
}

// Swizzled staging -> global rows orow (per lane = row) by TMA scatter4:
// lanes 0-7 each write four rows.  A group of four with a row to skip is
// written by the warp with 16-byte stores instead.
__device__ __forceinline__ void store_staged_tma(const Staging& st, int64_t orow, const CUtensorMap* map,
                                                 __nv_bfloat16* dst, int64_t ld, int col0, int lane) {
    fence_proxy_async_smem();  // this lane's staging writes -> the scatter's reads
    __syncwarp();
    const int g = lane & 7;
    int y[4];
    bool full = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t o = __shfl_sync(0xffffffffu, orow, 4 * g + i);
        y[i] = (int)o;
        full = full && o >= 0;
    }
    // row 4g starts at base + 4g * 128 (the swizzle permutes chunks within rows, base is 1024-aligned)
    if (lane < 8 && full) tma_scatter4(map, smem_u32(st.base + 4 * g * 128), col0, y[0], y[1], y[2], y[3]);
    if (lane < 8) bulk_commit();
    const unsigned partial = __ballot_sync(0xffffffffu, lane < 8 && !full);
    for (unsigned m = partial; m; m &= m - 1) {
        const int gg = __ffs(m) - 1;  // rows 4gg..4gg+3: one 16-byte chunk per lane
        const int r = 4 * gg + (lane >> 3), u = lane & 7;
        const int64_t o = __shfl_sync(0xffffffffu, orow, r);
        if (o >= 0) *reinterpret_cast<uint4*>(dst + o * ld + col0 + u * 8) = *reinterpret_cast<const uint4*>(st.at(r, u));
    }
}

// Global rows rrow (per lane = row; < 0 gives zeros) -> swizzled staging by
// TMA gather4 (lanes 0-7, four rows each; rows < 0 read past the tensor's end,
// which fills zeros), completing on the warp's barrier.
__device__ __forceinline__ bool load_staged_tma(const Staging& st, int64_t rrow, const CUtensorMap* map, int col0,
                                                int64_t n_rows_src, int lane, uint64_t* bar, uint32_t& ph) {
    if (lane == 0) mbar_arrive_expect_tx(bar, 32u * 128u);
    __syncwarp();
    const int g = lane & 7;
    int y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t o = __shfl_sync(0xffffffffu, rrow, 4 * g + i);
        y[i] = (int)(o >= 0 ? o : n_rows_src);
    }
    if (lane < 8) tma_gather4(smem_u32(st.base + 4 * g * 128), map, bar, col0, y[0], y[1], y[2], y[3]);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, ph));
    ph ^= 1u;
    return ok;
}

__device__ __forceinline__ void add_param32(float (&v)[32], const float* p, bool mul) {
    const float4* q4 = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(q4 + q);
        if (mul) {
            v[4 * q] *= b.x;
            v[4 * q + 1] *= b.y;
            v[4 * q + 2] *= b.z;
            v[4 * q + 3] *= b.w;
        } else {
            v[4 * q] += b.x;
            v[4 * q + 1] += b.y;
            v[4 * q + 2] += b.z;
            v[4 * q + 3] += b.w;
        }
    }
}

// MODE: the producer features a launch compiles in.  TC_LEAN: a pre-ordered (or unordered)
// map, cp.async gathers only; TC_DRY: + dry stages for scatter convs (C2S conv1);
// TC_FULL: + TMA gather4 modes and row orders without a pre-ordered map.  The lean
// instances run the same stages with a shorter producer loop (gather-bound layers ~15%
// faster than the full instance).
constexpr int TC_LEAN = 0, TC_DRY = 1, TC_FULL = 2;

template <bool PAIR, int TC_PW, int MODE>
__global__ void __launch_bounds__(tc_threads(TC_PW), 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap omap, const __grid_constant__ CUtensorMap o2map,
                   const __grid_constant__ CUtensorMap rmap, const TcParams p) {
    static_assert(TC_PW == 4 || TC_PW == 8, "producer warps");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int S = p.stages;
    const int K = p.K;
    // PAIR: a CTA holds half of every MMA's B rows (the pair splits N)
    const int B_ROWS = PAIR ? p.sub_n / 2 : p.sub_n;        // per sub-MMA, in this CTA
    const int B_BYTES = p.n_sub * B_ROWS * 128;            // per stage, in this CTA
    const int stg_cols = p.stg_cols;
    const int stg_units = stg_cols / 8;
    uint8_t* a_smem = smem;
    uint8_t* b_smem = a_smem + S * TC_A_BYTES;
    uint8_t* stg_smem = b_smem + S * B_BYTES;                                    // 4 warps
    int32_t* nbr_s = reinterpret_cast<int32_t*>(stg_smem + 4 * 32 * (stg_units + 1) * 16);  // [TC_BM][K]
    uint4* sched_resp = reinterpret_cast<uint4*>(nbr_s + TC_BM * K);  // [TC_SCHED] launch-control responses
    uint64_t* bars = reinterpret_cast<uint64_t*>(sched_resp + TC_SCHED);
    uint64_t* full = bars;                 // [S] MMA may read the stage (leader / single CTA)
    uint64_t* afull = bars + S;            // [S] PAIR peer: this CTA's A copies have landed
    uint64_t* empty = bars + 2 * S;        // [S] the MMAs reading the stage are done
    uint64_t* tmem_full = bars + 3 * S;    // [2]
    uint64_t* tmem_empty = bars + 3 * S + 2;
    uint64_t* sched_full = bars + 3 * S + 4;               // [TC_SCHED] response landed
    uint64_t* sched_empty = sched_full + TC_SCHED;         // [TC_SCHED] every role has read it
    uint64_t* mask_bar = sched_empty + TC_SCHED;           // every producer warp posted its tap mask
    uint64_t* pair_bar = mask_bar + 1;                     // PAIR: the peer CTA's tap mask arrived (single CTA:
                                                           // never arrived; the test stall mode waits on it)
    uint64_t* res_bar = pair_bar + 1;                      // [4] per epilogue warp: staged residual rows landed
    // [S] bit 1: a tile's last step (bookkeeping); bits 8+: the stage's 16-channel MMA steps
    // when fewer than TC_BK / 16 (the last 64-channel chunk of a Cin % 64 != 0 conv), else 0
    uint32_t* stage_flags = reinterpret_cast<uint32_t*>(res_bar + 4);
    uint32_t* tile_steps = stage_flags + S;  // [8] reduction steps per tile, ring over tiles
    // (the producers run at most S <= 8 stages, so at most 8 one-step tiles, ahead of the MMA thread)
    uint32_t* misc = tile_steps + 8;      // [0] tmem base, [1] abort
    uint32_t* mask_s = misc + 4;          // [2][TC_PW] tap masks per producer warp, by tile parity
    uint32_t* pair_mask_s = mask_s + 2 * TC_PW;  // [2] PAIR: the peer CTA's tap mask, by tile parity

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int64_t unit = PAIR ? (int64_t)(blockIdx.x >> 1) : (int64_t)blockIdx.x;
    const int64_t n_units = PAIR ? (int64_t)(gridDim.x >> 1) : (int64_t)gridDim.x;
    constexpr int TILE_ROWS = PAIR ? 2 * TC_BM : TC_BM;
    const int64_t my_tiles = p.n_tiles > unit ? (p.n_tiles - 1 - unit) / n_units + 1 : 0;
    const bool dyn = !PAIR && p.dynamic != 0;
    // Tile sequence of this CTA.  Static: unit, unit + n_units, ...  Dynamic:
    // its own tile, then one tile per successful launch-control response.
    // Tile ids run backwards from the launch order so that the last row
    // tiles (the fullest tap masks when rows are mask-sorted) start first.
    const int64_t first_tile = dyn ? p.n_tiles - 1 - (int64_t)blockIdx.x : (my_tiles > 0 ? unit : -1);
    // next tile after local tile lt, or -1; `arrive` makes this caller's read
    // of response lt count towards the slot's release
    auto next_tile = [&](int64_t lt, bool arrive) -> int64_t {
        if (!dyn) return lt + 1 < my_tiles ? unit + (lt + 1) * n_units : -1;
        const int q = (int)(lt % TC_SCHED);
        if (!mbar_wait(&sched_full[q], (uint32_t)((lt / TC_SCHED) & 1))) return -2;
        const int64_t x = clc_cancelled_x(&sched_resp[q]);
        if (arrive) mbar_arrive(&sched_empty[q]);
        return x < 0 ? -1 : p.n_tiles - 1 - x;
    };
    const int n_chunks = (p.cin + TC_BK - 1) / TC_BK;
    constexpr int MMA_WARP = 4 + TC_PW;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            // gather lanes (async, .noinc) + the producer's expect_tx arrive (+ the peer's relay);
            // with TMA gathers only the expect_tx arrive of the stage's bytes (both CTAs' for a pair)
            mbar_init(&full[s], p.gather4 == 1   ? 1
                                : p.gather4 == 2 ? (TC_PW / 2) * 32 + 1
                                                 : TC_PW * 32 + 1 + (PAIR ? 1 : 0));
            mbar_init(&afull[s], TC_PW * 32 + 1);   // PAIR peer: gather lanes + the flags arrive
            mbar_init(&empty[s], 1);                // one tcgen05.commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);            // tcgen05.commit after a tile's last MMA
            mbar_init(&tmem_empty[b], PAIR ? 8 : 4);  // one arrive per epilogue warp (of both CTAs)
        }
        for (int q = 0; q < TC_SCHED; ++q) {
            mbar_init(&sched_full[q], 1);           // the requester's expect_tx arrive
            mbar_init(&sched_empty[q], TC_PW + 1 + 4);  // producer warps, MMA thread, epilogue warps
        }
        mbar_init(mask_bar, TC_PW);
        mbar_init(pair_bar, 1);
        for (int w = 0; w < 4; ++w) mbar_init(&res_bar[w], 1);  // lane 0's expect_tx arrive
        misc[1] = 0;
        misc[2] = 0xffffffffu;
        for (int q = 0; q < S; ++q) stage_flags[q] = 0u;  // PAIR peer: stages its producers issued, once they are done
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    if (warp == MMA_WARP) {
        if (PAIR) {
            tmem_alloc_pair(&misc[0], TC_TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(&misc[0], TC_TMEM_COLS);
            tmem_relinquish();
        }
    }
    if (warp == 4 && lane == 0) tma_prefetch_desc(&wmap);
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive / TMA
    tc_fence_after();
    const uint32_t tmem_base = misc[0];
    volatile uint32_t* abort_flag = &misc[1];

    if (warp >= 4 && warp < 4 + TC_PW) {
        // ====================================================== A producers
        const int pw = warp - 4;
        const int sub = lane >> 3;  // row within a group of 4
        const int j = lane & 7;     // 16-byte chunk of the 128-byte slice
        constexpr int ROWS = TC_BM / TC_PW;     // rows per producer warp
        constexpr int GROUPS = ROWS / 4;        // copy instructions per stage
        int32_t* my_nbr = nbr_s + pw * ROWS * K;
        const int own0 = (int)rank * TC_BM + pw * ROWS;  // my rows within the tile
        uint64_t* arrive_bar = (PAIR && !leader) ? afull : full;
        const uint32_t leader_full0 = PAIR ? mapa_shared(smem_u32(full), 0) : 0u;
        int s = 0;          // stage ring position and its phase bit
        uint32_t ph = 0;
        bool ok = true;
        int64_t tile = first_tile;
        int64_t requested = 0;  // launch-control requests issued (producer warp 0)
        int64_t issued = 0;     // stages this warp has issued
        // Stages of every kind, counted alike by all producer warps: stage i's B tile (and the
        // flags the MMA thread reads) is issued by warp i % TC_PW, so no one warp carries the
        // extra per-stage work and sets the pace of the stage ring.
        uint32_t stage_no = 0;
        // Contiguous map rows (no row order, or a pre-ordered map) on one CTA:
        // each producer warp reads only its own rows' map block, one tile
        // ahead, into registers (16-byte loads, all in flight at once), and
        // the two warps OR their tap masks through mask_bar.
        const bool fast_map = MODE != TC_FULL || p.row_order == nullptr || p.nbr_ordered != nullptr;
        // gather4 == 2 (single CTA): the upper half of the producer warps gather by TMA, the lower
        // half by cp.async, so both copy engines carry A rows
        const bool G4 = MODE == TC_FULL && (p.gather4 == 1 || (!PAIR && p.gather4 == 2 && pw >= TC_PW / 2));
        const int32_t* map_rows = p.nbr_ordered ? p.nbr_ordered : p.nbr;
        constexpr int QV = (ROWS * TC_MAX_K / 4 + 31) / 32;  // int4 per lane for ROWS rows of <= 32 taps
        const int my_vec = ROWS * K / 4;                       // int4 of my rows' block (K * 64 / 4)
        int4 qmap[QV];
        auto load_my_map = [&](int64_t t_next) {
            const int64_t r0 = (t_next / p.grid_y) * TILE_ROWS + own0;
            const int64_t left = p.n_rows - r0;
            const int n_my = left <= 0 ? 0 : (left < ROWS ? (int)left : ROWS);
            const int n_int = n_my * K;
            const int32_t* blk = map_rows + r0 * K;
#pragma unroll
            for (int u = 0; u < QV; ++u) {
                const int f4 = u * 32 + lane;
                if (4 * f4 + 3 < n_int) {
                    qmap[u] = ldg_nc_v4(reinterpret_cast<const int4*>(blk) + f4);
                } else {
                    qmap[u].x = 4 * f4 < n_int ? __ldg(blk + 4 * f4) : -1;
                    qmap[u].y = 4 * f4 + 1 < n_int ? __ldg(blk + 4 * f4 + 1) : -1;
                    qmap[u].z = 4 * f4 + 2 < n_int ? __ldg(blk + 4 * f4 + 2) : -1;
                    qmap[u].w = -1;
                }
            }
        };
        // Launch-control requests run one tile ahead: response j names the tile after local tile
        // j; request j + 1 goes out when tile j starts, so the response for the next tile is
        // there when the tile starts and its map rows can be loaded a whole tile ahead.
        int64_t consumed = 0;  // responses this warp has read
        auto request = [&](int64_t j) -> bool {  // producer warp 0, lane 0
            const int q = (int)(j % TC_SCHED);
            if (!mbar_wait(&sched_empty[q], (uint32_t)(((j / TC_SCHED) & 1) ^ 1))) return false;
            fence_proxy_async_smem();  // earlier generic reads of the slot before the async write
            mbar_arrive_expect_tx(&sched_full[q], 16u);
            clc_try_cancel(&sched_resp[q], &sched_full[q]);
            requested = j + 1;
            return true;
        };
        if (dyn && pw == 0 && tile >= 0) {
            bool got = true;
            if (lane == 0) got = request(0);
            ok = __shfl_sync(0xffffffffu, got, 0);
        }
        if (fast_map && tile >= 0) load_my_map(tile);
        for (int64_t lt = 0; tile >= 0 && ok; ++lt) {
            if (dyn && pw == 0) {
                bool got = true;
                if (lane == 0) got = request(lt + 1);
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    ok = false;
                    break;
                }
            }
            const int64_t tile_row0 = (tile / p.grid_y) * TILE_ROWS;
            const int n0 = (int)(tile % p.grid_y) * p.tile_n;
            // neighbor rows of the whole tile (the common tap mask), mine kept in smem
            uint32_t mask = 0;
            const int64_t n_valid = p.n_rows - tile_row0 < TILE_ROWS ? p.n_rows - tile_row0 : TILE_ROWS;
            const int n_ints = (int)n_valid * K;
            const uint64_t kdiv = (1ull << 32) / (uint64_t)K + 1ull;  // f / K == (f * kdiv) >> 32 here
            if (fast_map) {
                // my rows' map block (prefetched) -> my_nbr, checked; this warp's tap mask
#pragma unroll
                for (int u = 0; u < QV; ++u) {
                    const int f4 = u * 32 + lane;
                    if (f4 < my_vec) {
                        int32_t v[4] = {qmap[u].x, qmap[u].y, qmap[u].z, qmap[u].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (v[e] < -1 || v[e] >= p.n_in) {
                                raise_fault(FAULT_BAD_NEIGHBOR);
                                v[e] = -1;
                            }
                            if (v[e] >= 0) {
                                const int f = 4 * f4 + e;
                                mask |= 1u << (f - (int)(((uint64_t)f * kdiv) >> 32) * K);
                            }
                        }
                        reinterpret_cast<int4*>(my_nbr)[f4] = make_int4(v[0], v[1], v[2], v[3]);
                    }
                }
            } else if (p.row_order == nullptr || p.nbr_ordered != nullptr) {
                // the tile's map rows are contiguous: independent 16-byte loads,
                // issued 8 deep before any is consumed (one latency per batch)
                const int32_t* blk = (p.nbr_ordered ? p.nbr_ordered : p.nbr) + tile_row0 * K;
                const int n_full = n_ints / 4;               // whole int4 vectors
                const int n_vec = (n_ints + 3) / 4;
                for (int base = 0; base < n_vec; base += 8 * 32) {
                    int4 q[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int f4 = base + u * 32 + lane;
                        if (f4 < n_full) {
                            q[u] = __ldg(reinterpret_cast<const int4*>(blk) + f4);
                        } else {
                            q[u].x = 4 * f4 < n_ints ? __ldg(blk + 4 * f4) : -1;
                            q[u].y = 4 * f4 + 1 < n_ints ? __ldg(blk + 4 * f4 + 1) : -1;
                            q[u].z = 4 * f4 + 2 < n_ints ? __ldg(blk + 4 * f4 + 2) : -1;
                            q[u].w = -1;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int f4 = base + u * 32 + lane;
                        const int32_t vals[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int f = 4 * f4 + e;
                            if (f >= n_ints) break;
                            const int t = (int)(((uint64_t)f * kdiv) >> 32), k = f - t * K;
                            int32_t v = vals[e];
                            if (v < -1 || v >= p.n_in) {
                                raise_fault(FAULT_BAD_NEIGHBOR);
                                v = -1;
                            }
                            if (v >= 0) mask |= 1u << k;
                            if (t >= own0 && t < own0 + ROWS) my_nbr[(t - own0) * K + k] = v;
                        }
                    }
                }
                for (int f = lane; f < ROWS * K; f += 32) {  // my rows past the end of the grid
                    const int t = (int)(((uint64_t)f * kdiv) >> 32);
                    if (own0 + t >= n_valid) my_nbr[f] = -1;
                }
            } else {
                // row order without a pre-ordered map: gather the rows
                for (int i = lane; i < TILE_ROWS * K; i += 32) {
                    const int t = (int)(((uint64_t)i * kdiv) >> 32), k = i - t * K;
                    int32_t v = -1;
                    if (i < n_ints) {
                        const int64_t r = ordered_row(p.row_order, tile_row0 + t, p.n_rows);
                        if (r >= 0) {
                            v = __ldg(p.nbr + r * K + k);
                            if (v < -1 || v >= p.n_in) {
                                raise_fault(FAULT_BAD_NEIGHBOR);
                                v = -1;
                            }
                        }
                    }
                    if (v >= 0) mask |= 1u << k;
                    if (t >= own0 && t < own0 + ROWS) my_nbr[(t - own0) * K + k] = v;
                }
            }
            mask = __reduce_or_sync(0xffffffffu, mask);
            {
                // OR of both producer warps' masks (equal on the other paths, which read every row)
                bool got = true;
                if (lane == 0) {
                    mask_s[TC_PW * (lt & 1) + pw] = mask;
                    mbar_arrive(mask_bar);
                    got = mbar_wait(mask_bar, (uint32_t)(lt & 1));
                    if (got) {
                        mask = 0;
#pragma unroll
                        for (int w = 0; w < TC_PW; ++w) mask |= mask_s[TC_PW * (lt & 1) + w];
                    }
                    if (PAIR && fast_map && got) {
                        // the pair's tile spans both CTAs: swap CTA masks through the peer's smem
                        if (pw == 0) {
                            st_shared_cluster_u32(mapa_shared(smem_u32(pair_mask_s + (lt & 1)), rank ^ 1u), mask);
                            mbar_arrive_cluster(mapa_shared(smem_u32(pair_bar), rank ^ 1u));
                        }
                        got = mbar_wait_cluster(pair_bar, (uint32_t)(lt & 1));
                        if (got) mask |= pair_mask_s[lt & 1];
                    }
                }
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    ok = false;
                    break;
                }
                mask = __shfl_sync(0xffffffffu, mask, 0);
            }
            if (mask == 0) mask = 1;  // a tile with no valid tap still runs one (all-zero) step
            __syncwarp();
            // the next tile (response lt, requested a tile ago); start loading its map rows
            int64_t nt = 0;
            if (lane == 0) nt = next_tile(lt, true);
            nt = __shfl_sync(0xffffffffu, nt, 0);
            consumed = lt + 1;
            if (nt == -2) {
                ok = false;
                break;
            }
            if (fast_map && nt >= 0) load_my_map(nt);
            // A scatter conv (C2S conv1: column tile = child block) whose tile keeps no child of
            // this block writes nothing: run it as one "dry" stage (no copies; the MMAs read stale
            // shared memory into an accumulator whose rows are all discarded).
            bool dry = false;
            if (MODE != TC_LEAN && !PAIR && p.gather4 == 0 && p.row_map != nullptr && p.map_cols > 1) {
                const int wb = p.cout / p.map_cols;
                const int blk = n0 / wb;
                bool kept = false;
                for (int i = lane; i < TILE_ROWS; i += 32) {
                    const int64_t pos = tile_row0 + i;
                    if (pos < p.n_rows) {
                        const int64_t row = ordered_row(p.row_order, pos, p.n_rows);
                        if (row >= 0 && __ldg(p.row_map + row * p.map_cols + blk) >= 0) kept = true;
                    }
                }
                dry = !__any_sync(0xffffffffu, kept);
            }
            const int chunks = dry ? 1 : n_chunks;
            if (dry) mask = mask & (~mask + 1u);  // the lowest valid tap only
            const int n_steps = __popc(mask) * chunks;
            int step = 0;
            // Source rows of tap kk for this lane's copies.  They are read one tap ahead, so the
            // shared-memory loads overlap the current tap's stages instead of heading them.
            auto load_rows = [&](int kk, int32_t (&d)[GROUPS]) {
                if (G4) {
                    // lanes below ROWS/4: the four rows 4*lane .. 4*lane+3 of my rows (absent rows read as zeros)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int32_t v = lane < ROWS / 4 ? my_nbr[(4 * lane + e) * K + kk] : -1;
                        d[e] = v >= 0 ? v : (int32_t)p.n_in;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < GROUPS; ++i) d[i] = my_nbr[(i * 4 + sub) * K + kk];
                }
            };
            int32_t next_rows[GROUPS];
            load_rows(__ffs(mask) - 1, next_rows);
            for (uint32_t m = mask; m && ok; m &= m - 1) {
                const int k = __ffs(m) - 1;
                int32_t src[GROUPS];
#pragma unroll
                for (int i = 0; i < GROUPS; ++i) src[i] = next_rows[i];
                const uint32_t m_next = m & (m - 1);
                if (m_next) load_rows(__ffs(m_next) - 1, next_rows);
                for (int ch = 0; ch < chunks; ++ch, ++step) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u))) {
                        ok = false;
                        break;
                    }
                    // (the full instance keeps warp 0: with gather4 == 2 only the lower warps take this path)
                    const bool b_lane = lane == 0 && (MODE == TC_FULL ? pw == 0
                                                                      : (int)(stage_no & (uint32_t)(TC_PW - 1)) == pw);
                    ++stage_no;
                    if (dry) {
                        // every arrival the stage expects, no copies
                        if (b_lane) {
                            if (step == 0) tile_steps[lt & 7] = (uint32_t)n_steps;
                            stage_flags[s] = 2u;
                            mbar_arrive(&full[s]);
                        }
                        mbar_arrive(&full[s]);
                        if (++s == S) {
                            s = 0;
                            ph ^= 1u;
                        }
                        continue;
                    }
                    if (G4) {
                        // A by TMA row gathers; one expect_tx (leader / single CTA) covers every byte
                        // of the stage, the other copies only complete transactions
                        const uint32_t stage = smem_u32(a_smem + s * TC_A_BYTES);
                        const uint32_t bar = PAIR ? leader_full0 + (uint32_t)(s * 8) : smem_u32(&full[s]);
                        if (lane == 0 && pw == 0) {
                            if (step == 0) tile_steps[lt & 7] = (uint32_t)n_steps;
                            const int tail16 = ch == n_chunks - 1 ? ((p.cin % TC_BK) + 15) / 16 : 0;
                            stage_flags[s] = (step == n_steps - 1 ? 2u : 0u) | ((uint32_t)tail16 << 8);
                            if (!PAIR || leader)
                                mbar_arrive_expect_tx(&full[s], (uint32_t)((PAIR ? 2 : 1) * (TC_A_BYTES + B_BYTES)));
                            const uint32_t dst = smem_u32(b_smem + s * B_BYTES);
                            for (int q = 0; q < p.n_sub; ++q) {
                                if (PAIR)
                                    tma_load_3d_pair(dst + q * B_ROWS * 128, &wmap, bar, ch * TC_BK, k,
                                                     n0 + q * p.sub_n + (int)rank * B_ROWS);
                                else
                                    tma_load_3d(dst + q * B_ROWS * 128, &wmap, &full[s], ch * TC_BK, k,
                                                n0 + q * p.sub_n);
                            }
                        }
                        if (lane < ROWS / 4) {
                            const uint32_t dst = stage + (uint32_t)((pw * ROWS + 4 * lane) * 128);
                            if (PAIR)
                                tma_gather4_pair(dst, &amap, bar, ch * TC_BK, src[0], src[1], src[2], src[3]);
                            else
                                tma_gather4(dst, &amap, &full[s], ch * TC_BK, src[0], src[1], src[2], src[3]);
                        }
                        if (++s == S) {
                            s = 0;
                            ph ^= 1u;
                        }
                        continue;
                    }
                    if (b_lane) {
                        // published to the MMA thread by this stage's full-barrier arrive below
                        if (step == 0) tile_steps[lt & 7] = (uint32_t)n_steps;
                        const int tail16 = ch == n_chunks - 1 ? ((p.cin % TC_BK) + 15) / 16 : 0;
                        stage_flags[s] = (step == n_steps - 1 ? 2u : 0u) | ((uint32_t)tail16 << 8);
                        const uint32_t dst = smem_u32(b_smem + s * B_BYTES);
                        if (!PAIR) {
                            mbar_arrive_expect_tx(&full[s], (uint32_t)(B_BYTES + (p.gather4 == 2 ? TC_A_BYTES / 2 : 0)));
                            for (int q = 0; q < p.n_sub; ++q)
                                tma_load_3d(dst + q * B_ROWS * 128, &wmap, &full[s], ch * TC_BK, k,
                                            n0 + q * p.sub_n);
                        } else {
                            // both halves of B complete on the leader's full barrier
                            if (leader) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * B_BYTES));
                            const uint32_t bar = leader_full0 + (uint32_t)(s * 8);
                            for (int q = 0; q < p.n_sub; ++q)
                                tma_load_3d_pair(dst + q * B_ROWS * 128, &wmap, bar, ch * TC_BK, k,
                                                 n0 + q * p.sub_n + (int)rank * B_ROWS);
                            if (!leader) mbar_arrive(&afull[s]);  // publishes stage_flags to the relay
                        }
                    }
                    const int c = ch * TC_BK + j * 8;
                    const uint32_t stage = smem_u32(a_smem + s * TC_A_BYTES);
#pragma unroll
                    for (int i = 0; i < GROUPS; ++i) {
                        const int r = pw * ROWS + i * 4 + sub;
                        const bool v = src[i] >= 0 && c < p.cin;
                        const void* g = v ? (const void*)(p.in + (int64_t)src[i] * p.cin + c) : (const void*)p.in;
                        cp_async_16(stage + r * 128 + ((j ^ (r & 7)) << 4), g, v ? 16u : 0u);
                    }
                    cp_async_arrive_noinc(&arrive_bar[s]);
                    ++issued;
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) break;
            tile = nt;
        }
        if (PAIR && pw == 0 && lane == 0) *reinterpret_cast<volatile uint32_t*>(&misc[2]) = (uint32_t)issued;
        if (dyn && pw == 0 && lane == 0) {
            // requests whose responses this warp did not read: let them land before the CTA exits
            for (int64_t q = consumed; q < requested; ++q)
                if (!mbar_wait(&sched_full[q % TC_SCHED], (uint32_t)((q / TC_SCHED) & 1))) break;
        }
        cp_async_wait<0>();
        if (!ok) *abort_flag = 1u;
    } else if (warp == MMA_WARP) {
        if (PAIR && !leader) {
            // ================================================ relay (pair peer)
            // Forwards "this CTA's A stage has landed" to the leader's full
            // barrier.  Lane l serves stage slot l, so the cluster-scope
            // release arrives of different stages overlap; a lane stops at the
            // first stage index at or past the producers' final count.  (With
            // TMA gathers the peer's rows complete on the leader's barrier.)
            if (lane < S && !p.gather4) {
                const uint32_t lf = mapa_shared(smem_u32(full), 0) + (uint32_t)(lane * 8);
                volatile uint32_t* total = &misc[2];
                uint32_t ph = 0;
                for (uint32_t it = (uint32_t)lane;; it += (uint32_t)S) {
                    bool got = false;
                    const uint64_t t0 = globaltimer();
                    for (uint32_t spin = 0;; ++spin) {
                        if (mbar_try_wait(&afull[lane], ph)) {
                            got = true;
                            break;
                        }
                        if (it >= *total) break;
                        if ((spin & 255u) == 255u && globaltimer() - t0 > wait_limit_ns()) {
                            raise_fault(FAULT_WAIT_TIMEOUT);
                            *abort_flag = 1u;
                            break;
                        }
                    }
                    if (!got) break;
                    fence_proxy_async_smem();  // cp.async data -> the tensor core's reads
                    mbar_arrive_cluster(lf);
                    ph ^= 1u;
                }
            }
        } else {
            // ================================================ MMA issuer
            // The whole warp runs the loop (waits, descriptors and tile
            // bookkeeping stay warp-uniform) and one elected lane issues the
            // MMAs and their commits: issued from single-lane divergent code
            // the same MMAs kept the tensor pipe idle ~40% of the time.
            const bool issuer = elect_one();
            const int issuer_lane = __ffs(__ballot_sync(0xffffffffu, issuer)) - 1;
            const uint32_t idesc = PAIR ? umma_idesc_bf16_m256((uint32_t)p.sub_n) : umma_idesc_bf16_m128((uint32_t)p.sub_n);
            const uint64_t adesc0 = umma_desc_sw128(smem_u32(a_smem));
            const uint64_t bdesc0 = umma_desc_sw128(smem_u32(b_smem));
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int64_t tile = first_tile;
            for (int64_t lt = 0; tile >= 0 && ok; ++lt) {
                const int b = p.n_buf == 2 ? (int)(lt & 1) : 0;
                const uint32_t use = (uint32_t)(p.n_buf == 2 ? (lt >> 1) : lt);
                // Test mode: a wait that nothing completes, so that every role reaches its wait
                // limit, raises FAULT_WAIT_TIMEOUT and drains (no stage is consumed, no MMA issued).
                if (!PAIR && p.test_stall && !__all_sync(0xffffffffu, mbar_wait(pair_bar, 0u))) {
                    ok = false;
                    break;
                }
                if (!__all_sync(0xffffffffu, mbar_wait(&tmem_empty[b], (use & 1u) ^ 1u))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem_base + (uint32_t)(b * 256);
                uint32_t steps = 0;
                for (uint32_t step = 0;; ++step) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    fence_proxy_async_smem();  // cp.async (generic proxy) data -> tcgen05.mma reads
                    if (step == 0) steps = tile_steps[lt & 7];
                    const uint64_t ad = adesc0 + (uint64_t)((s * TC_A_BYTES) >> 4);
                    const uint64_t bd = bdesc0 + (uint64_t)((s * B_BYTES) >> 4);
                    // a 32-channel tail chunk (e.g. Cin = 96) runs 2 of the 4 MMAs: the rest of its
                    // A and B rows are zero fill
                    const uint32_t kn = stage_flags[s] >> 8;
                    const int k16 = kn ? (int)kn : TC_BK / 16;
                    if (issuer) {
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; ++kk) {
                            if (kk >= k16) break;
                            const uint32_t accum = (step == 0 && kk == 0) ? 0u : 1u;
                            // K step kk: +32 bytes inside the 128-byte swizzled rows
                            if (PAIR) {
                                umma_bf16_pair(acc, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, accum);
                                if (p.n_sub == 2)
                                    umma_bf16_pair(acc + p.sub_n, ad + (uint64_t)(kk * 2),
                                                   bd + (uint64_t)((B_ROWS * 128 + kk * 32) >> 4), idesc, accum);
                            } else {
                                umma_bf16(acc, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, accum);
                                if (p.n_sub == 2)
                                    umma_bf16(acc + p.sub_n, ad + (uint64_t)(kk * 2),
                                              bd + (uint64_t)((B_ROWS * 128 + kk * 32) >> 4), idesc, accum);
                            }
                        }
                        if (PAIR)
                            umma_commit_pair(&empty[s], 0x3);
                        else
                            umma_commit(&empty[s]);
                    }
                    __syncwarp();
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                    if (step + 1 >= steps) break;
                }
                if (!ok) break;
                if (issuer) {
                    if (PAIR)
                        umma_commit_pair(&tmem_full[b], 0x3);
                    else
                        umma_commit(&tmem_full[b]);
                }
                __syncwarp();
                int64_t nt = 0;
                if (issuer) nt = next_tile(lt, true);
                tile = __shfl_sync(0xffffffffu, nt, issuer_lane);
                if (tile == -2) ok = false;
            }
            if (!ok && issuer) *abort_flag = 1u;
        }
    } else {
        // ====================================================== epilogue
        Staging st;
        st.units = stg_units;
        st.swz = p.tma_epi;
        st.base = p.tma_epi ? stg_smem + warp * 32 * 128 : stg_smem + warp * 32 * (stg_units + 1) * 16;
        uint32_t res_ph = 0;  // phase of this warp's residual barrier
        const int t = tid;  // TMEM lane == tile row (of this CTA's half)
        const int W = p.ln_width;
        const bool multi = p.ln != 0 || p.out2 != nullptr;
        const bool dense_res = p.residual != nullptr && p.res_off == nullptr;
        const uint32_t leader_tmem_empty = PAIR ? mapa_shared(smem_u32(tmem_empty), 0) : 0u;
        int64_t tile = first_tile;
        for (int64_t lt = 0; tile >= 0; ++lt) {
            const int64_t tile_base = (tile / p.grid_y) * TILE_ROWS + (int64_t)rank * TC_BM;
            const int n0 = (int)(tile % p.grid_y) * p.tile_n;
            const int b = p.n_buf == 2 ? (int)(lt & 1) : 0;
            const uint32_t use = (uint32_t)(p.n_buf == 2 ? (lt >> 1) : lt);
            const bool waited = mbar_wait(&tmem_full[b], use & 1u);
            if (!__all_sync(0xffffffffu, waited)) {
                *abort_flag = 1u;
                break;
            }
            tc_fence_after();
            const uint32_t lane_addr = tmem_base + (uint32_t)(b * 256) + ((uint32_t)(warp * 32) << 16);
            const int64_t pos = tile_base + t;
            const int64_t row = pos < p.n_rows ? ordered_row(p.row_order, pos, p.n_rows) : -1;
            int64_t orow = row, old = p.cout;
            int ocol0 = n0;
            if (p.row_map) {
                const int wb = p.cout / p.map_cols;
                orow = row >= 0 ? (int64_t)p.row_map[row * p.map_cols + n0 / wb] : -1;
                ocol0 = n0 % wb;
                old = wb;
            }

            // y = acc + bias + residual for the 32 columns at tile column c
            // (staging group starting at g0 holds the dense residual)
            auto compute_y = [&](int c, int g0, float (&v)[32]) {
                tmem_ld32(lane_addr + c, v);
                if (p.bias) add_param32(v, p.bias + n0 + c, false);
                if (dense_res) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float r8[8];
                        load_bf16x8(st.at(lane, (c - g0) / 8 + q), r8);
#pragma unroll
                        for (int e = 0; e < 8; ++e) v[q * 8 + e] += r8[e];
                    }
                } else if (p.residual && row >= 0) {
                    const int64_t base = p.res_off[row];
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        v[e] += __bfloat162float(p.residual[base + (n0 + c + e) / p.res_rep]);
                }
            };
            auto stage_out = [&](int c, int g0, const float (&v)[32]) {
#pragma unroll
                for (int q = 0; q < 4; ++q) cvt_store_bf16x8(st.at(lane, (c - g0) / 8 + q), v + 8 * q);
            };

            if (!multi) {
                for (int g0 = 0; g0 < p.tile_n; g0 += stg_cols) {
                    stg_reuse();
                    if (dense_res &&
                        !(p.tma_epi ? load_staged_tma(st, row, &rmap, n0 + g0, p.n_rows, lane, &res_bar[warp], res_ph)
                                    : load_staged_rows(st, row, p.residual, p.cout, n0 + g0, lane, &res_bar[warp], res_ph)))
                        *abort_flag = 1u;
                    for (int c = g0; c < g0 + stg_cols;) {
                        if (c + 64 <= g0 + stg_cols && !p.res_off) {
                            // 64 columns per TMEM wait
                            float v[64];
                            tmem_ld64(lane_addr + c, v);
                            float (&lo)[32] = *reinterpret_cast<float(*)[32]>(v);
                            float (&hi)[32] = *reinterpret_cast<float(*)[32]>(v + 32);
                            if (p.bias) {
                                add_param32(lo, p.bias + n0 + c, false);
                                add_param32(hi, p.bias + n0 + c + 32, false);
                            }
                            if (dense_res) {
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    float r8[8];
                                    load_bf16x8(st.at(lane, (c - g0) / 8 + q), r8);
#pragma unroll
                                    for (int e = 0; e < 8; ++e) v[q * 8 + e] += r8[e];
                                }
                            }
                            if (p.silu) {
#pragma unroll
                                for (int e = 0; e < 64; ++e) v[e] = silu_bf16out(v[e]);
                            }
                            stage_out(c, g0, lo);
                            stage_out(c + 32, g0, hi);
                            c += 64;
                        } else {
                            float v[32];
                            compute_y(c, g0, v);
                            if (p.silu) {
#pragma unroll
                                for (int e = 0; e < 32; ++e) v[e] = silu_bf16out(v[e]);
                            }
                            stage_out(c, g0, v);
                            c += 32;
                        }
                    }
                    __syncwarp();
                    if (p.tma_epi)
                        store_staged_tma(st, orow, &omap, p.out, old, ocol0 + g0, lane);
                    else
                        store_staged_rows(st, orow, p.out, old, ocol0 + g0, lane);
                    __syncwarp();
                }
            } else {
                // pass 1: y -> TMEM (residual folded in) and per-group sums
                float sum[4] = {0.f, 0.f, 0.f, 0.f};  // <= 4 LayerNorm groups per tile
                for (int g0 = 0; g0 < p.tile_n; g0 += stg_cols) {
                    stg_reuse();
                    if (dense_res &&
                        !(p.tma_epi ? load_staged_tma(st, row, &rmap, n0 + g0, p.n_rows, lane, &res_bar[warp], res_ph)
                                    : load_staged_rows(st, row, p.residual, p.cout, n0 + g0, lane, &res_bar[warp], res_ph)))
                        *abort_flag = 1u;
                    for (int c = g0; c < g0 + stg_cols; c += 32) {
                        float v[32];
                        compute_y(c, g0, v);
                        float s = 0.f;
#pragma unroll
                        for (int e = 0; e < 32; ++e) s += v[e];
                        const int g = c / W;
                        sum[0] += g == 0 ? s : 0.f;
                        sum[1] += g == 1 ? s : 0.f;
                        sum[2] += g == 2 ? s : 0.f;
                        sum[3] += g == 3 ? s : 0.f;
                        tmem_st32(lane_addr + c, v);
                    }
                    __syncwarp();
                }
                float mean[4], rstd[4] = {1.f, 1.f, 1.f, 1.f};
#pragma unroll
                for (int g = 0; g < 4; ++g) mean[g] = sum[g] / (float)W;
                if (p.ln) {
                    // pass 2: biased variance about the mean (two-pass, as the reference)
                    float var[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int c = 0; c < p.tile_n; c += 64) {  // tile_n and W are multiples of 32
                        float v[64];
                        if (c + 64 <= p.tile_n) {
                            tmem_ld64(lane_addr + c, v);
                        } else {
                            float h[32];
                            tmem_ld32(lane_addr + c, h);
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] = h[e];
                        }
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            const int cc = c + 32 * half;
                            if (cc >= p.tile_n) break;
                            const int g = cc / W;
                            const float mu = g == 0 ? mean[0] : g == 1 ? mean[1] : g == 2 ? mean[2] : mean[3];
                            float s = 0.f;
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                const float d = v[32 * half + e] - mu;
                                s += d * d;
                            }
                            var[0] += g == 0 ? s : 0.f;
                            var[1] += g == 1 ? s : 0.f;
                            var[2] += g == 2 ? s : 0.f;
                            var[3] += g == 3 ? s : 0.f;
                        }
                    }
#pragma unroll
                    for (int g = 0; g < 4; ++g) rstd[g] = 1.0f / sqrtf(var[g] / (float)W + p.eps);
                }
                // pass 3: out = y when a second output is requested
                if (p.out2) {
                    for (int g0 = 0; g0 < p.tile_n; g0 += stg_cols) {
                        stg_reuse();
                        for (int c = g0; c < g0 + stg_cols; c += 32) {
                            float v[32];
                            tmem_ld32(lane_addr + c, v);
                            stage_out(c, g0, v);
                        }
                        __syncwarp();
                        if (p.tma_epi)
                            store_staged_tma(st, orow, &omap, p.out, old, ocol0 + g0, lane);
                        else
                            store_staged_rows(st, orow, p.out, old, ocol0 + g0, lane);
                        __syncwarp();
                    }
                }
                // pass 4: post(y) = [LayerNorm(gamma, beta)] -> [SiLU]
                __nv_bfloat16* dst = p.out2 ? p.out2 : p.out;
                for (int g0 = 0; g0 < p.tile_n; g0 += stg_cols) {
                    stg_reuse();
                    for (int c = g0; c < g0 + stg_cols; c += 32) {
                        float v[32];
                        tmem_ld32(lane_addr + c, v);
                        if (p.ln) {
                            const int g = c / W;
                            const int gc = c - g * W;
                            const float mu = g == 0 ? mean[0] : g == 1 ? mean[1] : g == 2 ? mean[2] : mean[3];
                            const float rs = g == 0 ? rstd[0] : g == 1 ? rstd[1] : g == 2 ? rstd[2] : rstd[3];
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] = (v[e] - mu) * rs;
                            if (p.gamma) add_param32(v, p.gamma + gc, true);
                            if (p.beta) add_param32(v, p.beta + gc, false);
                        }
                        if (p.silu) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] = silu_bf16out(v[e]);
                        }
                        stage_out(c, g0, v);
                    }
                    __syncwarp();
                    if (p.tma_epi)
                        store_staged_tma(st, orow, p.out2 ? &o2map : &omap, dst, old, ocol0 + g0, lane);
                    else
                        store_staged_rows(st, orow, dst, old, ocol0 + g0, lane);
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR && !leader)
                    mbar_arrive_cluster(leader_tmem_empty + (uint32_t)(b * 8));
                else
                    mbar_arrive(&tmem_empty[b]);
            }
            int64_t nt = 0;
            if (lane == 0) nt = next_tile(lt, true);
            tile = __shfl_sync(0xffffffffu, nt, 0);
            if (tile == -2) {
                *abort_flag = 1u;
                break;
            }
        }
        bulk_wait_all();  // every output row written before the CTA leaves
    }

    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // no CTA leaves while its pair may still touch its barriers
    if (warp == MMA_WARP) {
        tc_fence_after();
        if (PAIR)
            tmem_dealloc_pair(tmem_base, TC_TMEM_COLS);
        else
            tmem_dealloc(tmem_base, TC_TMEM_COLS);
    }
}

// Epilogue staging width: the largest multiple of 32 that divides tile_n
// and is at most `cap` (<= TC_STG_COLS), so staging groups tile the row exactly.
inline int tc_stg_cols(int tile_n, int cap = TC_STG_COLS) {
    for (int c = cap; c >= 32; c -= 32)
        if (tile_n % c == 0) return c;
    return 32;
}

// Dynamic shared-memory bytes of a launch (1 KB alignment slack included);
// with `pair`, a CTA holds half of the B rows.
inline size_t tc_smem_bytes(int stages, int tile_n, int K, bool pair, int stg_cols) {
    const size_t b_bytes = (size_t)(pair ? tile_n / 2 : tile_n) * 128;
    return 1024 + (size_t)stages * (TC_A_BYTES + b_bytes) + 4 * 32 * (stg_cols / 8 + 1) * 16 +
           (size_t)TC_BM * K * 4 + (3 * stages + 4) * 8 + stages * 4 + 32 + 16 + TC_SCHED * (16 + 16) + 8 + 8 * TC_PW_MAX + 8 + 8 + 4 * 8;
}

}  // namespace sc
