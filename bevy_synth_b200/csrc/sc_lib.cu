// sc_lib.cu -- the C ABI of libsparseconv (declared in include/sparseconv.h).
//
// One translation unit: the kernels live in the *.cuh headers included here.
// Host-side validation mirrors the reference's shape/dtype checks
// (burn_flex_gmm src/lib.rs:698-725 validate_config; src/wgpu/sparse_conv.rs:
// 369-473 validate_tensor_shapes) and reports them as SC_ERR_INVALID with a
// message, as the reference returns Err(String).
#include <cub/device/device_radix_sort.cuh>
#include <cmath>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <string>

#include "conv_simt.cuh"
#include "conv_tc.cuh"
#include "conv_ts.cuh"
#include "linear_tc.cuh"
#include "neighbor.cuh"
#include "rowops.cuh"
#include "sc_common.cuh"

namespace sc {

thread_local std::string g_last_error;

static int validate_config(const sc_conv_config* c) {
    if (!c) return fail(SC_ERR_INVALID, "sparse conv config is null");
    if (c->in_channels <= 0 || c->out_channels <= 0)
        return fail(SC_ERR_INVALID, "sparse conv channel dimensions must be non-zero");
    if (c->kernel_d <= 0 || c->kernel_h <= 0 || c->kernel_w <= 0)
        return fail(SC_ERR_INVALID, "sparse conv kernel dimensions must be non-zero");
    if (c->groups <= 0) return fail(SC_ERR_INVALID, "sparse conv groups must be non-zero");
    if (c->in_channels_per_group * c->groups != c->in_channels)
        return fail(SC_ERR_INVALID, "sparse conv in_channels/group mismatch");
    if (c->out_channels_per_group * c->groups != c->out_channels)
        return fail(SC_ERR_INVALID, "sparse conv out_channels/group mismatch");
    bool used[3] = {false, false, false};
    for (int i = 0; i < 3; ++i) {
        int a = c->axis_order[i];
        if (a < 0 || a > 2 || used[a])
            return fail(SC_ERR_INVALID, "sparse conv axis_order must be a permutation of [0,1,2]");
        used[a] = true;
    }
    return SC_OK;
}

static int64_t kernel_rows_of(const sc_conv_config* c) {
    return c->kernel_d * c->kernel_h * c->kernel_w;
}

// kernel_layout (reference src/lib.rs:727-752)
static void kernel_offsets_of(const sc_conv_config* c, int32_t* off) {
    const int32_t cd = (int32_t)(c->kernel_d / 2), ch = (int32_t)(c->kernel_h / 2),
                  cw = (int32_t)(c->kernel_w / 2);
    int64_t k = 0;
    for (int64_t kd = 0; kd < c->kernel_d; ++kd)
        for (int64_t kh = 0; kh < c->kernel_h; ++kh)
            for (int64_t kw = 0; kw < c->kernel_w; ++kw, ++k) {
                const int32_t d[3] = {c->axis_sign[0] * ((int32_t)kd - cd),
                                      c->axis_sign[1] * ((int32_t)kh - ch),
                                      c->axis_sign[2] * ((int32_t)kw - cw)};
                int32_t o[3] = {0, 0, 0};
                o[c->axis_order[0]] = d[0];
                o[c->axis_order[1]] = d[1];
                o[c->axis_order[2]] = d[2];
                off[3 * k] = o[0];
                off[3 * k + 1] = o[1];
                off[3 * k + 2] = o[2];
            }
}

static inline unsigned grid1d(int64_t n, int block) { return (unsigned)((n + block - 1) / block); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// --- TMA descriptor encoding through the driver entry point ------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

static bool force_simt() {
    const char* e = std::getenv("SC_FORCE_SIMT");
    return e && e[0] == '1';
}

struct TcPlan {
    int tile_n, n_sub, sub_n, stages, grid_y, n_buf, stg_cols;
    int pw;     // gather producer warps of the kernel instance (4 or 8)
    bool pair;  // 2-SM (cta_group::2) kernel on CTA pairs
    size_t smem;
};

// SC_TC_STATIC=1: the single-CTA kernel on a persistent grid with round-robin tiles instead of
// cluster launch control.
static bool use_static_schedule() {
    static const bool v = [] {
        const char* e = std::getenv("SC_TC_STATIC");
        return e && e[0] == '1';
    }();
    return v;
}

// SC_TC_GATHER4: 1 = A rows by TMA gather4, 2 = half by gather4 and half by cp.async, else cp.async.
static int gather4_mode() {
    static const int v = [] {
        const char* e = std::getenv("SC_TC_GATHER4");
        return e ? std::atoi(e) : 0;
    }();
    return v == 1 || v == 2 ? v : 0;
}

static bool use_tma_epilogue() {
    static const bool v = [] {
        const char* e = std::getenv("SC_TC_TMA_EPI");
        return !(e && e[0] == '0');
    }();
    return v;
}

// SC_TC_PAIR=1 takes the pair kernel wherever it applies, SC_TC_PAIR=0 nowhere; unset, it is taken for
// narrow multi-tap convs (Cin and Cout <= 64), the one shape class where it measured faster.
static int pair_mode() {
    const char* e = std::getenv("SC_TC_PAIR");
    return !e ? -1 : (e[0] == '1' ? 1 : 0);
}

static constexpr size_t kMaxDynSmem = 232448;  // 227 KB opt-in per block on sm_100

static int sm_count() {
    static int count[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (count[dev] == 0) {
        int c = 0;
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
        count[dev] = c;
    }
    return count[dev];
}

// Decides whether the tensor-core kernel takes this conv and with which tiling.
// n_rows < 0: row count unknown (no column split for small grids).
static bool plan_tc(const sc_conv_config* c, sc_dtype dt, const sc_epilogue& e, TcPlan* plan, int64_t n_rows) {
    if (dt != SC_DTYPE_BF16 || c->groups != 1 || force_simt()) return false;
    const int64_t K = kernel_rows_of(c), cin = c->in_channels, cout = c->out_channels;
    if (K > TC_MAX_K || cin % 8 != 0 || cin < 64 || cout % 32 != 0) return false;
    int tile_n;
    if (e.d_out_row_map) {
        if (e.out_row_map_cols <= 0 || cout % e.out_row_map_cols != 0) return false;
        tile_n = (int)(cout / e.out_row_map_cols);
        if (e.layer_norm && e.ln_width != 0 && e.ln_width != tile_n) return false;
    } else if (e.layer_norm || e.d_out2) {
        const int64_t W = (e.layer_norm && e.ln_width) ? e.ln_width : cout;
        tile_n = (int)(cout <= 512 ? cout : W);
        if (tile_n % W != 0 || cout % tile_n != 0) return false;
    } else {
        // Column tiles up to 512 wide for multi-tap convs: every column tile gathers the
        // tile's rows again, and the gather, not the tensor pipe, bounds these convs, so
        // one wide tile with a single-buffered accumulator beats two double-buffered ones
        // (measured: 384->384 808 -> 550 us, 512->512 1158 -> 1048 us on config 2's grid).
        // 1x1 convs keep 256 (they are epilogue-bound and need the epilogue overlap).
        // SC_TC_WIDE=0|1 pins the choice.
        const char* wide_env = std::getenv("SC_TC_WIDE");
        const bool wide = wide_env ? wide_env[0] == '1' : K > 1;
        const int64_t cap = wide ? 512 : 256;
        int64_t n_tiles = (cout + cap - 1) / cap;
        while (cout % n_tiles != 0 || (cout / n_tiles) % 32 != 0) ++n_tiles;
        tile_n = (int)(cout / n_tiles);
        // A grid with fewer (row, column) tiles than SMs leaves SMs idle: halve the column tile
        // while it stays a multiple of 32 (a launch of one tile per SM is as long as its slowest
        // tile, so narrower tiles on more SMs finish sooner).  SC_TC_SPLIT=0 turns it off.
        const char* split_env = std::getenv("SC_TC_SPLIT");
        if (n_rows > 0 && !(split_env && split_env[0] == '0')) {
            const int64_t row_tiles = (n_rows + 127) / 128;
            while (row_tiles * (cout / tile_n) < sm_count() && tile_n >= 128 && (tile_n / 2) % 32 == 0 &&
                   cout % (tile_n / 2) == 0)
                tile_n /= 2;
        }
    }
    if (tile_n > 512 || tile_n % 32 != 0) return false;
    const int64_t W = (e.layer_norm && e.ln_width) ? e.ln_width : tile_n;
    if (W % 32 != 0 || tile_n % W != 0 || tile_n / W > 4) return false;
    plan->tile_n = tile_n;
    plan->n_sub = tile_n > 256 ? 2 : 1;
    plan->sub_n = tile_n / plan->n_sub;
    if (plan->sub_n % 16 != 0) return false;
    plan->n_buf = tile_n <= 256 ? 2 : 1;
    plan->grid_y = (int)(cout / tile_n);
    const int pm = pair_mode();
    const bool narrow = K > 1 && cin <= 64 && cout <= 64 && !e.d_out_row_map && gather4_mode() == 0;
    plan->pair = (pm == 1 || (pm < 0 && narrow)) && plan->sub_n >= 32 && c->in_channels % 8 == 0;
    // 8 gather warps for multi-tap convs (their producer instruction stream sets the stage
    // rate), 4 for 1x1 convs and the pair kernel (SC_TC_PW=4|8 pins it on the single-CTA kernel)
    plan->pw = (K > 1 && (!plan->pair || (pm < 0 && narrow))) ? 8 : 4;
    if (const char* pw_env = std::getenv("SC_TC_PW"))
        if (std::atoi(pw_env) == 4 || std::atoi(pw_env) == 8) plan->pw = std::atoi(pw_env);
    // Deepest stage ring that fits; a narrower epilogue staging buffer is
    // taken when it buys a stage (SC_TC_STG=64|128 pins the width).
    auto deepest = [&](int stg) {
        int S = 8;
        while (S >= 2 && tc_smem_bytes(S, tile_n, (int)K, plan->pair, stg) > kMaxDynSmem) --S;
        return S;
    };
    int stg = tc_stg_cols(tile_n, 128);
    int S = deepest(stg);
    const char* stg_env = std::getenv("SC_TC_STG");
    if (stg_env && std::atoi(stg_env) == 64) {
        stg = tc_stg_cols(tile_n, 64);
        S = deepest(stg);
    } else if (!stg_env && K > 1) {
        // (1x1 convs keep 128-column staging: they are epilogue-bound, and half as many staging
        // rounds beat the TMA epilogue and the extra stage there: ConvNeXt stage 1.136 -> 1.075 ms)
        const int stg64 = tc_stg_cols(tile_n, 64);
        const int s64 = deepest(stg64);
        // ties take 64 columns, which the TMA (scatter4 / gather4) epilogue needs; a tile whose
        // width 64 does not divide (e.g. 96) keeps the wider staging: fewer staging rounds beat the
        // extra stage (config 3 level 2, C=96: 4.66 -> 4.48 ms)
        if (s64 >= S && stg64 == 64) {
            stg = stg64;
            S = s64;
        }
    }
    if (const char* env = std::getenv("SC_TC_STAGES")) {  // tuning override, clamped to what fits
        const int want = std::atoi(env);
        if (want >= 2 && want < S) S = want;
    }
    if (S < 2) return false;
    plan->stages = S;
    plan->stg_cols = stg;
    plan->smem = tc_smem_bytes(S, tile_n, (int)K, plan->pair, stg);
    return true;
}

static int launch_tc(const sc_conv_config* c, const void* in, int64_t n_in, const int32_t* nbr,
                     int64_t n_rows, const void* w, const float* bias, const sc_epilogue& e,
                     void* out, cudaStream_t st, const TcPlan& plan) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const int64_t K = kernel_rows_of(c), cin = c->in_channels, cout = c->out_channels;
    CUtensorMap wmap;
    cuuint64_t dims[3] = {(cuuint64_t)cin, (cuuint64_t)K, (cuuint64_t)cout};
    cuuint64_t strides[2] = {(cuuint64_t)cin * 2, (cuuint64_t)(K * cin * 2)};
    cuuint32_t box[3] = {(cuuint32_t)TC_BK, 1u, (cuuint32_t)(plan.pair ? plan.sub_n / 2 : plan.sub_n)};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    CUresult r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));

    // A rows by TMA gather (tile::gather4): the features as a 2-D map [n_in, cin], 64-column boxes
    CUtensorMap amap;
    memset(&amap, 0, sizeof amap);
    const int g4_mode = (cin % 8 == 0 && n_in > 0 && n_in < 0x7fffffff) ? gather4_mode() : 0;
    const bool g4 = g4_mode == 1 || (g4_mode == 2 && !plan.pair);
    if (g4) {
        cuuint64_t adims[2] = {(cuuint64_t)cin, (cuuint64_t)n_in};
        cuuint64_t astr[1] = {(cuuint64_t)cin * 2};
        cuuint32_t abox[2] = {(cuuint32_t)TC_BK, 1u};
        cuuint32_t aes[2] = {1u, 1u};
        CUresult ra = enc(&amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(in), adims, astr, abox, aes,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (ra != CUDA_SUCCESS)
            return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled (features) failed with code " + std::to_string((int)ra));
    }

    // Epilogue through TMA row gathers / scatters: 64-column staging, outputs that
    // are plain rows (no child-row scatter); maps are [rows, cols] bf16, 64-column boxes.
    CUtensorMap omap, o2map, rmap;
    memset(&omap, 0, sizeof omap);
    memset(&o2map, 0, sizeof o2map);
    memset(&rmap, 0, sizeof rmap);
    const bool tma_epi = use_tma_epilogue() && plan.stg_cols == 64 && e.d_out_row_map == nullptr &&
                         n_rows > 0 && n_rows < 0x7fffffff;
    if (tma_epi) {
        auto enc_rows = [&](CUtensorMap* m, const void* base) -> CUresult {
            cuuint64_t d[2] = {(cuuint64_t)cout, (cuuint64_t)n_rows};
            cuuint64_t sd[1] = {(cuuint64_t)cout * 2};
            cuuint32_t bx[2] = {64u, 1u};
            cuuint32_t es[2] = {1u, 1u};
            return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), d, sd, bx, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        };
        CUresult r1 = enc_rows(&omap, out);
        CUresult r2 = e.d_out2 ? enc_rows(&o2map, e.d_out2) : CUDA_SUCCESS;
        CUresult r3 = (e.d_residual && !e.d_residual_offset) ? enc_rows(&rmap, e.d_residual) : CUDA_SUCCESS;
        if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS || r3 != CUDA_SUCCESS)
            return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled (epilogue) failed");
    }

    TcParams p;
    memset(&p, 0, sizeof p);
    p.gather4 = g4 ? g4_mode : 0;
    p.tma_epi = tma_epi ? 1 : 0;
    p.in = static_cast<const __nv_bfloat16*>(in);
    p.n_in = n_in;
    p.cin = (int)cin;
    p.nbr = nbr;
    p.n_rows = n_rows;
    p.K = (int)K;
    p.bias = bias;
    p.cout = (int)cout;
    p.tile_n = plan.tile_n;
    p.n_sub = plan.n_sub;
    p.sub_n = plan.sub_n;
    p.stages = plan.stages;
    p.n_buf = plan.n_buf;
    p.grid_y = plan.grid_y;
    const int64_t tile_rows = plan.pair ? 2 * TC_BM : TC_BM;
    p.n_tiles = ((n_rows + tile_rows - 1) / tile_rows) * plan.grid_y;
    p.stg_cols = plan.stg_cols;
    if (p.stg_cols % 32 != 0 || plan.tile_n % p.stg_cols != 0)
        return fail(SC_ERR_UNSUPPORTED, "internal: staging width does not tile the output tile");
    p.residual = static_cast<const __nv_bfloat16*>(e.d_residual);
    p.res_off = e.d_residual_offset;
    p.res_rep = e.residual_repeat > 0 ? e.residual_repeat : 1;
    p.ln = e.layer_norm;
    p.ln_width = e.layer_norm ? (e.ln_width ? e.ln_width : plan.tile_n) : plan.tile_n;
    p.eps = e.ln_eps;
    p.gamma = e.d_ln_gamma;
    p.beta = e.d_ln_beta;
    p.silu = e.silu;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.out2 = static_cast<__nv_bfloat16*>(e.d_out2);
    p.row_map = e.d_out_row_map;
    p.map_cols = e.d_out_row_map ? e.out_row_map_cols : 1;
    p.row_order = e.d_row_order;
    p.nbr_ordered = e.d_row_order ? e.d_neighbor_rows_ordered : nullptr;
    {
        // SC_TC_TEST_STALL=1 (tests only, read on every call): the single-CTA kernel's MMA warp waits
        // on a barrier that nothing completes, to drive the bounded waits to their limit
        const char* st_env = std::getenv("SC_TC_TEST_STALL");
        p.test_stall = (st_env && st_env[0] == '1' && !plan.pair) ? 1 : 0;
    }

    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        const void* fns[] = {(const void*)conv_tc_kernel<false, 4, TC_LEAN>, (const void*)conv_tc_kernel<false, 4, TC_FULL>,
                             (const void*)conv_tc_kernel<false, 8, TC_LEAN>, (const void*)conv_tc_kernel<false, 8, TC_DRY>,
                             (const void*)conv_tc_kernel<true, 4, TC_FULL>, (const void*)conv_tc_kernel<true, 8, TC_LEAN>};
        for (const void* f : fns)
            if (attr_err == cudaSuccess)
                attr_err = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDynSmem);
    });
    SC_CUDA_TRY(attr_err);
    if (!plan.pair) {
        // Default: one CTA per tile; a running CTA claims tiles of CTAs that
        // have not started (cluster launch control), so tiles are balanced
        // dynamically.  SC_TC_STATIC=1: a persistent grid with round-robin tiles.
        p.dynamic = use_static_schedule() ? 0 : 1;
        const int64_t ctas = p.dynamic ? p.n_tiles : std::min<int64_t>(p.n_tiles, sm_count());
        if (ctas > 0x7fffffff) return fail(SC_ERR_UNSUPPORTED, "too many row tiles for one launch");
        // the leanest instance that has every producer feature this launch uses
        const bool full = p.gather4 != 0 || (p.row_order != nullptr && p.nbr_ordered == nullptr);
        const bool dry = p.row_map != nullptr && p.map_cols > 1;
        const dim3 g((unsigned)ctas);
        if (plan.pw == 8 && !full && !dry)
            conv_tc_kernel<false, 8, TC_LEAN><<<g, tc_threads(8), plan.smem, st>>>(wmap, amap, omap, o2map, rmap, p);
        else if (plan.pw == 8 && !full)
            conv_tc_kernel<false, 8, TC_DRY><<<g, tc_threads(8), plan.smem, st>>>(wmap, amap, omap, o2map, rmap, p);
        else if (!full && !dry)
            conv_tc_kernel<false, 4, TC_LEAN><<<g, tc_threads(4), plan.smem, st>>>(wmap, amap, omap, o2map, rmap, p);
        else
            conv_tc_kernel<false, 4, TC_FULL><<<g, tc_threads(4), plan.smem, st>>>(wmap, amap, omap, o2map, rmap, p);
    } else {
        cudaLaunchConfig_t lc;
        memset(&lc, 0, sizeof lc);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        // SC_TC_PW=8 (tuning): the 8-warp lean pair instance, when the launch needs no full-instance feature
        const bool pair8 = plan.pw == 8 && p.gather4 == 0 && !(p.row_order != nullptr && p.nbr_ordered == nullptr);
        const void* fn = pair8 ? (const void*)conv_tc_kernel<true, 8, TC_LEAN> : (const void*)conv_tc_kernel<true, 4, TC_FULL>;
        lc.blockDim = dim3(tc_threads(pair8 ? 8 : 4));
        lc.dynamicSmemBytes = plan.smem;
        lc.stream = st;
        lc.attrs = attr;
        lc.numAttrs = 1;
        lc.gridDim = dim3((unsigned)(2 * sm_count()));
        int max_clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&max_clusters, fn, &lc) != cudaSuccess || max_clusters <= 0)
            max_clusters = sm_count() / 2;
        const int64_t pairs = std::min<int64_t>(p.n_tiles, max_clusters);
        lc.gridDim = dim3((unsigned)(2 * pairs));
        if (pair8)
            SC_CUDA_TRY(cudaLaunchKernelEx(&lc, conv_tc_kernel<true, 8, TC_LEAN>, wmap, amap, omap, o2map, rmap, p));
        else
            SC_CUDA_TRY(cudaLaunchKernelEx(&lc, conv_tc_kernel<true, 4, TC_FULL>, wmap, amap, omap, o2map, rmap, p));
    }
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

// The tile-source (A-from-TMEM) kernel: bf16, 64 input channels, <= 128 outputs, a plain bias/SiLU
// epilogue, map rows in order, and a usable tile-source plan.  SC_TS=0 turns it off.
struct TsPlan {
    int tile_n, grid_y, u_cap, stages, n_buf, n_stg, grp, n_a, a_col0, tma_epi;
    size_t smem;
};

static bool plan_ts(const sc_conv_config* c, sc_dtype dt, const sc_epilogue& e, TsPlan* plan) {
    if (dt != SC_DTYPE_BF16 || c->groups != 1 || force_simt() || !e.d_tile_sources) return false;
    if (const char* env = std::getenv("SC_TS"))
        if (env[0] == '0') return false;
    const int64_t K = kernel_rows_of(c), cin = c->in_channels, cout = c->out_channels;
    if (cin != 64 || K > 32 || cout % 32 != 0) return false;
    if (e.layer_norm || e.d_residual || e.d_out2 || e.d_out_row_map || e.d_row_order) return false;
    if (e.tile_sources_max < 0 || e.tile_sources_max > TS_UMAX) return false;
    // One column tile of at most 128 outputs, accumulators double-buffered (the epilogue of one
    // tile overlaps the next tile's MMAs).  Wider outputs stay on the generic kernel: measured on
    // config 5's 64->256 layer (isolated, max clock), one 256-wide single-buffered accumulator
    // (6.26 ms with per-row stores, 5.82 ms with TMA box stores) and two 128-wide column tiles that
    // stage and build A twice (7.8 ms) all lost to it (4.74 ms): in map order a tile executes all
    // 27 taps, against 17.9 on the conv schedule.
    // SC_TS_WIDE=1 (one single-buffered accumulator up to 256 wide) and SC_TS_WIDE=2 (128-wide
    // column tiles, each staging and building A again) opt wider outputs in.
    const char* wide_env = std::getenv("SC_TS_WIDE");
    const int wide = wide_env ? wide_env[0] - '0' : 0;
    int tile_n = (int)cout;
    if (cout > 128) {
        if (wide == 1 && cout <= 256) tile_n = (int)cout;
        else if (wide == 2 && cout % 128 == 0) tile_n = 128;
        else return false;
    }
    plan->tile_n = tile_n;
    plan->grid_y = (int)(cout / tile_n);
    plan->n_buf = tile_n <= 128 ? 2 : 1;
    plan->u_cap = std::max(8, (e.tile_sources_max + 7) / 8 * 8);
    // taps per pipeline step: the per-step barrier work is paid once per G taps, which narrow
    // outputs (little tensor work per tap) need most
    plan->grp = tile_n <= 64 ? 4 : 2;
    if (const char* g_env = std::getenv("SC_TS_G")) {  // tuning: taps per step (1, 2 or 4)
        const int g = std::atoi(g_env);
        if (g == 1 || g == 2 || g == 4) plan->grp = g;
    }
    // A slots: the TMEM columns the two accumulators leave, whole slot groups of G
    plan->a_col0 = plan->n_buf * tile_n;
    plan->n_a = std::min(TS_NA_MAX, ((int)TC_TMEM_COLS - plan->a_col0) / 32) / plan->grp * plan->grp;
    if (plan->n_a < 2 * plan->grp) return false;
    // outputs by TMA box stores for the single-buffered accumulator, whose drain the MMAs wait
    // for (SC_TS_TMAEPI=0|1 pins it)
    const char* te_env = std::getenv("SC_TS_TMAEPI");
    plan->tma_epi = (te_env ? te_env[0] == '1' : plan->n_buf == 1) && tile_n % 64 == 0 ? 1 : 0;
    // double-buffered staging with >= 3 weight stages if it fits, else single-buffered staging
    // (tuning: SC_TS_NSTG=1 forces single-buffered staging, SC_TS_SMAX caps the weight stages, <= 16)
    const char* ns_env = std::getenv("SC_TS_NSTG");
    const char* smax_env = std::getenv("SC_TS_SMAX");
    const int s_max = smax_env ? std::max(2, std::min(16, std::atoi(smax_env))) : 12;
    for (int ns = (ns_env && ns_env[0] == '1') ? 1 : 2; ns >= 1; --ns) {
        int S = s_max;
        while (S >= 2 && ts_smem_bytes(plan->u_cap, tile_n, (int)K, S, ns, plan->tma_epi) > kMaxDynSmem) --S;
        S = S / plan->grp * plan->grp;  // whole slot groups
        if (S >= 2 * plan->grp) {
            plan->stages = S;
            plan->n_stg = ns;
            plan->smem = ts_smem_bytes(plan->u_cap, tile_n, (int)K, S, ns, plan->tma_epi);
            return true;
        }
    }
    return false;
}

static int launch_ts(const sc_conv_config* c, const void* in, int64_t n_in, int64_t n_rows, const void* w,
                     const float* bias, const sc_epilogue& e, void* out, cudaStream_t st, const TsPlan& plan) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const int64_t K = kernel_rows_of(c), cout = c->out_channels;
    CUtensorMap wmap;
    cuuint64_t dims[3] = {64u, (cuuint64_t)K, (cuuint64_t)cout};
    cuuint64_t strides[2] = {64u * 2u, (cuuint64_t)(K * 64 * 2)};
    cuuint32_t box[3] = {64u, 1u, (cuuint32_t)plan.tile_n};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    CUresult r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
    const int64_t row_tiles = (n_rows + 127) / 128;
    TsPlanView v = ts_plan_view(const_cast<void*>(e.d_tile_sources), row_tiles);
    TsParams p;
    memset(&p, 0, sizeof p);
    p.in = static_cast<const __nv_bfloat16*>(in);
    p.n_in = n_in;
    p.n_rows = n_rows;
    p.K = (int)K;
    p.u_count = v.u_count;
    p.tap_mask = v.tap_mask;
    p.u_rows = v.u_rows;
    p.lidx = v.lidx;
    p.bias = bias;
    p.silu = e.silu;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.cout = (int)cout;
    p.tile_n = plan.tile_n;
    p.grid_y = plan.grid_y;
    p.n_buf = plan.n_buf;
    p.n_stg = plan.n_stg;
    p.n_tiles = row_tiles * plan.grid_y;
    p.u_cap = plan.u_cap;
    p.b_stages = plan.stages;
    p.grp = plan.grp;
    p.n_a = plan.n_a;
    p.a_col0 = plan.a_col0;
    p.tma_epi = plan.tma_epi;
    CUtensorMap omap;
    memset(&omap, 0, sizeof omap);
    if (plan.tma_epi) {
        cuuint64_t od[2] = {(cuuint64_t)cout, (cuuint64_t)n_rows};
        cuuint64_t os[1] = {(cuuint64_t)cout * 2};
        cuuint32_t ob[2] = {64u, 32u};
        cuuint32_t oe[2] = {1u, 1u};
        CUresult ro = enc(&omap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, od, os, ob, oe, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (ro != CUDA_SUCCESS)
            return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed with code " + std::to_string((int)ro));
    }
    static std::once_flag ts_once;
    static cudaError_t ts_err = cudaSuccess;
    std::call_once(ts_once, [] {
        ts_err = cudaFuncSetAttribute((const void*)conv_ts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kMaxDynSmem);
    });
    SC_CUDA_TRY(ts_err);
    const int64_t ctas = std::min<int64_t>(p.n_tiles, sm_count());
    conv_ts_kernel<<<(unsigned)ctas, TS_THREADS, plan.smem, st>>>(wmap, omap, p);
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

template <typename T>
static int launch_simt(const sc_conv_config* c, const void* in, int64_t n_in, const int32_t* nbr,
                       int64_t n_rows, const void* w, const float* bias, const sc_epilogue& e,
                       void* out, cudaStream_t st) {
    const int64_t K = kernel_rows_of(c);
    const int cout_g = (int)c->out_channels_per_group;
    const int bpg = (cout_g + SIMT_BN - 1) / SIMT_BN;
    EpiParams ep;
    ep.residual = e.d_residual;
    ep.res_off = e.d_residual_offset;
    ep.res_rep = e.residual_repeat > 0 ? e.residual_repeat : 1;
    ep.out = out;
    ep.row_map = e.d_out_row_map;
    ep.map_cols = e.d_out_row_map ? e.out_row_map_cols : 1;
    ep.row_order = e.d_row_order;
    bool tiled = false;
    if constexpr (std::is_same<T, float>::value) {
        // the 8x8-per-thread fp32 kernel for the common shapes (see conv_f32_tiled_kernel)
        tiled = c->groups == 1 && c->in_channels % F32_BK == 0 && c->out_channels % F32_BN == 0 &&
                K <= F32_MAX_K && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(w) % 16 == 0;
        if (tiled) {
            dim3 g(grid1d(n_rows, F32_BM), (unsigned)(c->out_channels / F32_BN));
            conv_f32_tiled_kernel<<<g, F32_THREADS, 0, st>>>(static_cast<const float*>(in), n_in,
                                                             (int)c->in_channels, nbr, n_rows, (int)K,
                                                             static_cast<const float*>(w), bias,
                                                             (int)c->out_channels, ep);
        }
    }
    if (!tiled) {
        dim3 grid(grid1d(n_rows, SIMT_BM), (unsigned)(bpg * c->groups));
        conv_simt_kernel<T><<<grid, 256, 0, st>>>(
            static_cast<const T*>(in), n_in, (int)c->in_channels, (int)c->in_channels_per_group, nbr,
            n_rows, (int)K, static_cast<const T*>(w), bias, (int)c->out_channels, cout_g, bpg, ep);
    }
    SC_CUDA_TRY(cudaGetLastError());
    if (e.layer_norm || e.silu) {
        // post(y) as a second row pass over the stored y
        const int64_t cout = c->out_channels;
        int64_t width, ld, entries;
        const int32_t* map = nullptr;
        if (e.d_out_row_map) {
            width = cout / e.out_row_map_cols;
            ld = width;
            entries = n_rows * e.out_row_map_cols;
            map = e.d_out_row_map;
        } else {
            width = (e.layer_norm && e.ln_width) ? e.ln_width : cout;
            ld = width;
            entries = n_rows * (cout / width);
        }
        T* dst = static_cast<T*>(e.d_out2 ? e.d_out2 : out);
        const int rpw = rows_norm_act_rpw<T>(out, dst, width, ld);
        rows_norm_act_kernel<T><<<grid1d((entries + (rpw ? rpw : 1) - 1) / (rpw ? rpw : 1) * 32, 256), 256, 0, st>>>(
            static_cast<const T*>(out), dst, entries, (int)width, ld, map, e.d_ln_gamma, e.d_ln_beta,
            e.ln_eps, e.layer_norm, e.silu, rpw);
        SC_CUDA_TRY(cudaGetLastError());
    } else if (e.d_out2) {
        const size_t bytes = (size_t)(e.d_out_row_map ? 0 : n_rows * c->out_channels) * sizeof(T);
        if (e.d_out_row_map)
            return fail(SC_ERR_UNSUPPORTED, "out2 without LayerNorm/SiLU is not supported with a row map");
        SC_CUDA_TRY(cudaMemcpyAsync(e.d_out2, out, bytes, cudaMemcpyDeviceToDevice, st));
    }
    return SC_OK;
}

// ---- static scratch of the no-allocation neighbor map ------------------------
// Some callers cannot allocate device memory: they hold only the buffers they
// pass in (their device memory belongs to another runtime's pool, e.g. a
// burn/CubeCL backend that hands a custom op its input and output tensors and
// nothing else), or they must not call cudaMalloc on their execution path.
// sc_neighbor_map_noalloc serves them with this fixed table, which every GPU
// that loads the library holds until process exit.
constexpr int64_t kStaticTableSlots = int64_t(1) << 19;          // 8 MiB of 16-byte slots
constexpr int64_t kStaticMaxRows = kStaticTableSlots / 2;        // 262,144 input rows
constexpr size_t kStaticScratchBytes = 256 + (size_t)kStaticTableSlots * sizeof(HashSlot);
static __device__ __align__(256) uint8_t g_nb_static_scratch[kStaticScratchBytes];

// Device address of g_nb_static_scratch on the calling thread's current device
// (in host code the symbol itself is only a host-side stand-in).  Resolved on
// every call rather than cached: the lookup is cheap, and a cached address
// would dangle once the device's primary context is reset and the module
// reloaded.
static int static_scratch_address(void** out) {
    void* p = nullptr;
    SC_CUDA_TRY(cudaGetSymbolAddress(&p, g_nb_static_scratch));
    *out = p;
    return SC_OK;
}

}  // namespace sc

using namespace sc;

extern "C" {

int sc_version(void) { return 1; }

int sc_last_error(char* buf, size_t len) {
    const std::string& m = g_last_error;
    if (buf && len) {
        size_t n = std::min(len - 1, m.size());
        memcpy(buf, m.data(), n);
        buf[n] = 0;
    }
    return (int)m.size();
}

int sc_device_fault(uint32_t* h_fault) {
    if (!h_fault) return fail(SC_ERR_INVALID, "h_fault is null");
    SC_CUDA_TRY(cudaDeviceSynchronize());
    SC_CUDA_TRY(cudaMemcpyFromSymbol(h_fault, g_fault, sizeof(uint32_t)));
    const uint32_t zero = 0;
    SC_CUDA_TRY(cudaMemcpyToSymbol(g_fault, &zero, sizeof(uint32_t)));
    return SC_OK;
}

int sc_set_wait_limit_ns(uint64_t ns) {
    const uint64_t v = ns ? ns : kWaitLimitNs;
    SC_CUDA_TRY(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof v));
    return SC_OK;
}

int sc_kernel_rows(const sc_conv_config* cfg, int64_t* rows) {
    if (int rc = validate_config(cfg)) return rc;
    if (!rows) return fail(SC_ERR_INVALID, "rows is null");
    *rows = kernel_rows_of(cfg);
    return SC_OK;
}

int sc_kernel_offsets(const sc_conv_config* cfg, int32_t* off) {
    if (int rc = validate_config(cfg)) return rc;
    if (!off) return fail(SC_ERR_INVALID, "offsets is null");
    kernel_offsets_of(cfg, off);
    return SC_OK;
}

int sc_neighbor_workspace_bytes(int64_t n_in, size_t* bytes) {
    if (n_in < 0 || !bytes) return fail(SC_ERR_INVALID, "invalid neighbor workspace query");
    *bytes = nb_workspace_bytes(n_in);
    return SC_OK;
}

int sc_neighbor_map_query(const sc_conv_config* cfg, const int32_t* in_coords, int64_t n_in,
                          const int32_t* q_coords, int64_t n_q, void* ws, size_t ws_bytes,
                          int32_t* out, void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    const int64_t K = kernel_rows_of(cfg);
    if (K > kMaxKernelRows)
        return fail(SC_ERR_UNSUPPORTED, "neighbor map supports at most 1024 kernel offsets");
    if (cfg->kernel_d > 255 || cfg->kernel_h > 255 || cfg->kernel_w > 255)
        return fail(SC_ERR_UNSUPPORTED, "neighbor map supports kernel extents up to 255");
    if (n_in < 0 || n_q < 0) return fail(SC_ERR_INVALID, "negative row count");
    if (n_in > 0x7ffffffeLL) return fail(SC_ERR_INVALID, "sparse conv coord row count exceeds i32::MAX");
    const uint64_t cap = nb_capacity_for(n_in, ws_bytes);
    if (!ws || cap == 0)
        return fail(SC_ERR_CAPACITY, "neighbor workspace too small: need " +
                                         std::to_string(nb_workspace_bytes(n_in)) + " bytes");
    if ((n_in && !in_coords) || (n_q && (!q_coords || !out)))
        return fail(SC_ERR_INVALID, "null coordinate or output pointer");
    if (!aligned16(in_coords) || !aligned16(q_coords) || !aligned16(ws))
        return fail(SC_ERR_INVALID, "coordinates and workspace must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    NbStatus* status = static_cast<NbStatus*>(ws);
    HashSlot* table = reinterpret_cast<HashSlot*>(static_cast<uint8_t*>(ws) + 256);
    SC_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(NbStatus), st));
    SC_CUDA_TRY(cudaMemsetAsync(table, 0xff, cap * sizeof(HashSlot), st));
    if (n_in > 0) {
        nb_build_kernel<<<grid1d(n_in, 256), 256, 0, st>>>(reinterpret_cast<const int4*>(in_coords),
                                                            n_in, table, cap - 1, status);
        SC_CUDA_TRY(cudaGetLastError());
    }
    if (n_q > 0) {
        KernelOffsets off;
        off.k = (int32_t)K;
        int32_t tmp[3 * kMaxKernelRows];
        kernel_offsets_of(cfg, tmp);
        for (int64_t i = 0; i < 3 * K; ++i) off.d[i] = (int8_t)tmp[i];
        nb_query_kernel<<<grid1d(n_q * K, 256), 256, 0, st>>>(reinterpret_cast<const int4*>(q_coords),
                                                               n_q, table, cap - 1, off, out);
        SC_CUDA_TRY(cudaGetLastError());
    }
    return SC_OK;
}

int sc_neighbor_map(const sc_conv_config* cfg, const int32_t* coords, int64_t n, void* ws,
                    size_t ws_bytes, int32_t* out, void* stream) {
    return sc_neighbor_map_query(cfg, coords, n, coords, n, ws, ws_bytes, out, stream);
}

int sc_neighbor_map_noalloc(const sc_conv_config* cfg, const int32_t* coords, int64_t n, int32_t* out,
                            void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    if (n < 0) return fail(SC_ERR_INVALID, "negative row count");
    if (n > kStaticMaxRows)
        return fail(SC_ERR_CAPACITY, "sc_neighbor_map_noalloc: " + std::to_string(n) +
                                         " rows exceed the static table limit of " +
                                         std::to_string(kStaticMaxRows) + " rows");
    if (n == 0) return SC_OK;
    void* ws = nullptr;
    if (int rc = static_scratch_address(&ws)) return rc;
    // the allocating path's kernels on the static table; it clears the table
    // and the status word at the start of every call
    if (int rc = sc_neighbor_map_query(cfg, coords, n, coords, n, ws, kStaticScratchBytes, out, stream)) return rc;
    return sc_neighbor_status(ws, nullptr, stream);
}

int sc_neighbor_status(const void* ws, int32_t* h_max_probe, void* stream) {
    if (!ws) return fail(SC_ERR_INVALID, "workspace is null");
    NbStatus h;
    SC_CUDA_TRY(cudaMemcpyAsync(&h, ws, sizeof h, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
    SC_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    if (h_max_probe) *h_max_probe = h.max_probe;
    if (h.bits & NB_STATUS_RANGE)
        return fail(SC_ERR_RANGE, "sparse conv coordinate component outside [0, 65534]");
    if (h.bits & NB_STATUS_CAPACITY) return fail(SC_ERR_CAPACITY, "neighbor hash table insert failed");
    return SC_OK;
}

static size_t order_cub_bytes(int64_t n) {
    size_t b = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, b, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 32);
    return b;
}

static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

int sc_neighbor_schedule_scratch_bytes(int64_t n, size_t* bytes) {
    if (n < 0 || !bytes) return fail(SC_ERR_INVALID, "invalid row order scratch query");
    *bytes = 3 * align256((size_t)n * 4) + order_cub_bytes(n) + 256;
    return SC_OK;
}

int sc_neighbor_schedule(const sc_conv_config* cfg, const int32_t* nbr, int64_t n, void* scratch,
                         size_t scratch_bytes, int32_t* order, int32_t* nbr_ordered, void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    const int64_t K = kernel_rows_of(cfg);
    if (K > 32) return fail(SC_ERR_UNSUPPORTED, "row order supports at most 32 kernel offsets");
    if (n < 0) return fail(SC_ERR_INVALID, "negative row count");
    if (n == 0) return SC_OK;
    if (n > 0x7fffffffLL) return fail(SC_ERR_UNSUPPORTED, "too many rows");
    size_t need = 0;
    sc_neighbor_schedule_scratch_bytes(n, &need);
    if (!scratch || scratch_bytes < need)
        return fail(SC_ERR_CAPACITY, "row order scratch too small: need " + std::to_string(need) + " bytes");
    if (!nbr || !order) return fail(SC_ERR_INVALID, "null pointer");
    // rank taps by L1 distance from the centre, farthest first (ties by index)
    int32_t off[3 * 32];
    kernel_offsets_of(cfg, off);
    TapRank tr;
    tr.k = (int32_t)K;
    int idx[32];
    for (int i = 0; i < K; ++i) idx[i] = i;
    auto l1 = [&](int i) { return std::abs(off[3 * i]) + std::abs(off[3 * i + 1]) + std::abs(off[3 * i + 2]); };
    std::stable_sort(idx, idx + K, [&](int a, int b) { return l1(a) > l1(b); });
    for (int r = 0; r < K; ++r) tr.rank_of_tap[idx[r]] = (int8_t)r;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    uint32_t* keys_in = reinterpret_cast<uint32_t*>(base);
    uint32_t* keys_out = reinterpret_cast<uint32_t*>(base + align256((size_t)n * 4));
    int32_t* vals_in = reinterpret_cast<int32_t*>(base + 2 * align256((size_t)n * 4));
    void* tmp = base + 3 * align256((size_t)n * 4);
    size_t tmp_bytes = order_cub_bytes(n);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    row_mask_key_kernel<<<grid1d(n, 256), 256, 0, st>>>(nbr, n, tr, keys_in, vals_in);
    SC_CUDA_TRY(cudaGetLastError());
    SC_CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys_in, keys_out, vals_in, order, (int)n, 0,
                                                (int)K, st));
    if (nbr_ordered) {
        permute_rows_kernel<<<grid1d(n * K, 256), 256, 0, st>>>(nbr, order, n, (int)K, nbr_ordered);
        SC_CUDA_TRY(cudaGetLastError());
    }
    return SC_OK;
}

int sc_neighbor_tile_sources_bytes(int64_t n_rows, int64_t kernel_rows, size_t* bytes) {
    if (n_rows < 0 || kernel_rows <= 0 || kernel_rows > 32 || !bytes)
        return fail(SC_ERR_INVALID, "invalid tile-source plan size query");
    *bytes = ts_plan_bytes((n_rows + 127) / 128, (int)kernel_rows);
    return SC_OK;
}

int sc_neighbor_tile_sources(const sc_conv_config* cfg, const int32_t* nbr, int64_t n_rows, int64_t n_in,
                             void* plan, size_t plan_bytes, int32_t* h_max_sources, void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    const int64_t K = kernel_rows_of(cfg);
    if (K > 32) return fail(SC_ERR_UNSUPPORTED, "tile-source plan supports at most 32 kernel offsets");
    if (n_rows < 0 || n_in < n_rows) return fail(SC_ERR_INVALID, "invalid row counts for the tile-source plan");
    const int64_t n_tiles = (n_rows + 127) / 128;
    if (!plan || plan_bytes < ts_plan_bytes(n_tiles, (int)K))
        return fail(SC_ERR_CAPACITY, "tile-source plan buffer too small: need " +
                                         std::to_string(ts_plan_bytes(n_tiles, (int)K)) + " bytes");
    if (!aligned16(plan) || (n_rows && !nbr)) return fail(SC_ERR_INVALID, "null or unaligned pointer");
    if (n_tiles > 0x7fffffff) return fail(SC_ERR_UNSUPPORTED, "too many row tiles");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    SC_CUDA_TRY(cudaMemsetAsync(plan, 0, 64, st));
    if (n_tiles > 0) {
        ts_tile_sources_kernel<<<(unsigned)n_tiles, TSP_THREADS, 0, st>>>(nbr, n_rows, (int)K, n_in, plan, n_tiles);
        SC_CUDA_TRY(cudaGetLastError());
    }
    int32_t h[4] = {0, 0, 0, 0};
    SC_CUDA_TRY(cudaMemcpyAsync(h, plan, sizeof h, cudaMemcpyDeviceToHost, st));
    SC_CUDA_TRY(cudaStreamSynchronize(st));
    if (h_max_sources) *h_max_sources = h[2];
    if (h[3] > 0)
        return fail(SC_ERR_CAPACITY, std::to_string(h[3]) + " row tiles read more than " + std::to_string(TS_UMAX) +
                                         " distinct source rows (largest " + std::to_string(h[2]) + ")");
    return SC_OK;
}

static size_t order64_cub_bytes(int64_t n) {
    size_t b = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, b, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                    (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 40);
    return b;
}

int sc_neighbor_schedule_grouped_scratch_bytes(int64_t n, size_t* bytes) {
    if (n < 0 || !bytes) return fail(SC_ERR_INVALID, "invalid row order scratch query");
    *bytes = 2 * align256((size_t)n * 8) + align256((size_t)n * 4) + order64_cub_bytes(n) + 256;
    return SC_OK;
}

int sc_neighbor_schedule_grouped(const sc_conv_config* cfg, const int32_t* nbr, int64_t n,
                                 const uint8_t* group_mask8, void* scratch, size_t scratch_bytes, int32_t* order,
                                 int32_t* nbr_ordered, void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    const int64_t K = kernel_rows_of(cfg);
    if (K > 32) return fail(SC_ERR_UNSUPPORTED, "row order supports at most 32 kernel offsets");
    if (n < 0) return fail(SC_ERR_INVALID, "negative row count");
    if (n == 0) return SC_OK;
    if (n > 0x7fffffffLL) return fail(SC_ERR_UNSUPPORTED, "too many rows");
    size_t need = 0;
    sc_neighbor_schedule_grouped_scratch_bytes(n, &need);
    if (!scratch || scratch_bytes < need)
        return fail(SC_ERR_CAPACITY, "row order scratch too small: need " + std::to_string(need) + " bytes");
    if (!nbr || !order) return fail(SC_ERR_INVALID, "null pointer");
    int32_t off[3 * 32];
    kernel_offsets_of(cfg, off);
    TapRank tr;
    tr.k = (int32_t)K;
    int idx[32];
    for (int i = 0; i < K; ++i) idx[i] = i;
    auto l1 = [&](int i) { return std::abs(off[3 * i]) + std::abs(off[3 * i + 1]) + std::abs(off[3 * i + 2]); };
    std::stable_sort(idx, idx + K, [&](int a, int b) { return l1(a) > l1(b); });
    for (int r = 0; r < K; ++r) tr.rank_of_tap[idx[r]] = (int8_t)r;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    uint64_t* keys_in = reinterpret_cast<uint64_t*>(base);
    uint64_t* keys_out = reinterpret_cast<uint64_t*>(base + align256((size_t)n * 8));
    int32_t* vals_in = reinterpret_cast<int32_t*>(base + 2 * align256((size_t)n * 8));
    void* tmp = base + 2 * align256((size_t)n * 8) + align256((size_t)n * 4);
    size_t tmp_bytes = order64_cub_bytes(n);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    row_group_key_kernel<<<grid1d(n, 256), 256, 0, st>>>(nbr, n, tr, group_mask8, keys_in, vals_in);
    SC_CUDA_TRY(cudaGetLastError());
    SC_CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys_in, keys_out, vals_in, order, (int)n, 0,
                                                32 + (group_mask8 ? 8 : 0), st));
    if (nbr_ordered) {
        permute_rows_kernel<<<grid1d(n * K, 256), 256, 0, st>>>(nbr, order, n, (int)K, nbr_ordered);
        SC_CUDA_TRY(cudaGetLastError());
    }
    return SC_OK;
}

int sc_conv_uses_tensor_cores(const sc_conv_config* cfg, sc_dtype dtype, int32_t* flag) {
    if (int rc = validate_config(cfg)) return rc;
    if (!flag) return fail(SC_ERR_INVALID, "flag is null");
    sc_epilogue e;
    memset(&e, 0, sizeof e);
    TcPlan plan;
    *flag = plan_tc(cfg, dtype, e, &plan, -1) ? 1 : 0;
    return SC_OK;
}

int sc_subm_conv_forward(const sc_conv_config* cfg, sc_dtype dtype, const void* in, int64_t n_in,
                         const int32_t* nbr, int64_t n_rows, const void* w, const float* bias,
                         const sc_epilogue* epi, void* out, void* stream) {
    if (int rc = validate_config(cfg)) return rc;
    if (dtype != SC_DTYPE_F32 && dtype != SC_DTYPE_BF16)
        return fail(SC_ERR_INVALID, "sparse conv dtype must be F32 or BF16");
    if (n_rows < 0 || n_in < 0) return fail(SC_ERR_INVALID, "negative row count");
    if (n_rows > n_in)
        return fail(SC_ERR_INVALID, "sparse conv neighbor row count exceeds input rows: got " +
                                        std::to_string(n_rows) + " input rows " + std::to_string(n_in));
    sc_epilogue e;
    if (epi)
        e = *epi;
    else
        memset(&e, 0, sizeof e);
    if (n_rows == 0) return SC_OK;
    if (!in || !nbr || !w || !out) return fail(SC_ERR_INVALID, "null input, neighbor, weight or output pointer");
    const int64_t cout = cfg->out_channels;
    if (e.d_out_row_map && (e.out_row_map_cols <= 0 || cout % e.out_row_map_cols != 0))
        return fail(SC_ERR_INVALID, "out_row_map_cols must divide out_channels");
    if (e.layer_norm && e.ln_width < 0) return fail(SC_ERR_INVALID, "ln_width must be >= 0");
    if (e.layer_norm && e.ln_width > 0 && cout % e.ln_width != 0)
        return fail(SC_ERR_INVALID, "ln_width must divide out_channels");
    if (e.layer_norm && e.d_out_row_map && e.ln_width && e.ln_width != cout / e.out_row_map_cols)
        return fail(SC_ERR_INVALID, "with a row map, ln_width must equal the block width");
    if (e.d_residual_offset && e.residual_repeat < 1)
        return fail(SC_ERR_INVALID, "residual_repeat must be >= 1");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    TcPlan plan;
    // the tensor-core kernel reads the map, bias and LayerNorm parameters in 16-byte vectors
    const bool al = aligned16(in) && aligned16(w) && aligned16(out) && aligned16(e.d_out2) &&
                    aligned16(e.d_residual) && aligned16(nbr) && aligned16(e.d_neighbor_rows_ordered) &&
                    aligned16(bias) && aligned16(e.d_ln_gamma) && aligned16(e.d_ln_beta);
    TsPlan tsp;
    if (al && aligned16(e.d_tile_sources) && plan_ts(cfg, dtype, e, &tsp))
        return launch_ts(cfg, in, n_in, n_rows, w, bias, e, out, st, tsp);
    if (al && plan_tc(cfg, dtype, e, &plan, n_rows))
        return launch_tc(cfg, in, n_in, nbr, n_rows, w, bias, e, out, st, plan);
    if (dtype == SC_DTYPE_F32) return launch_simt<float>(cfg, in, n_in, nbr, n_rows, w, bias, e, out, st);
    return launch_simt<__nv_bfloat16>(cfg, in, n_in, nbr, n_rows, w, bias, e, out, st);
}

int sc_layer_norm_act(sc_dtype dtype, const void* x, int64_t rows, int64_t channels, const float* gamma,
                      const float* beta, float eps, int32_t ln, int32_t silu, void* y, void* stream) {
    if (rows < 0 || channels <= 0) return fail(SC_ERR_INVALID, "invalid layer norm shape");
    if (rows == 0) return SC_OK;
    if (!x || !y) return fail(SC_ERR_INVALID, "null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == SC_DTYPE_F32) {
        rows_norm_act_kernel<float><<<grid1d(rows * 32, 256), 256, 0, st>>>(
            static_cast<const float*>(x), static_cast<float*>(y), rows, (int)channels, channels, nullptr,
            gamma, beta, eps, ln, silu, 0);
    } else {
        const int rpw = rows_norm_act_rpw<__nv_bfloat16>(x, y, channels, channels);
        rows_norm_act_kernel<__nv_bfloat16><<<grid1d((rows + (rpw ? rpw : 1) - 1) / (rpw ? rpw : 1) * 32, 256), 256,
                                               0, st>>>(
            static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), rows, (int)channels,
            channels, nullptr, gamma, beta, eps, ln, silu, rpw);
    }
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_linear_forward(sc_dtype dtype, const void* x, int64_t rows, int64_t cin, const void* w, int64_t cout,
                      const float* bias, const void* residual, int32_t silu, void* out, void* stream) {
    if (rows < 0 || cin <= 0 || cout <= 0) return fail(SC_ERR_INVALID, "invalid linear shape");
    if (rows == 0) return SC_OK;
    if (!x || !w || !out) return fail(SC_ERR_INVALID, "null pointer");
    if (dtype != SC_DTYPE_BF16 || force_simt()) return fail(SC_ERR_UNSUPPORTED, "linear: bf16 tensor-core path only");
    if (const char* env = std::getenv("SC_LINEAR_TC"))
        if (env[0] == '0') return fail(SC_ERR_UNSUPPORTED, "linear: tensor-core path switched off");
    if (cin % 8 != 0 || cout % 64 != 0) return fail(SC_ERR_UNSUPPORTED, "linear: needs in % 8 == 0, out % 64 == 0");
    if (rows > 0x7fffff00LL) return fail(SC_ERR_UNSUPPORTED, "linear: too many rows");
    if (!aligned16(x) || !aligned16(w) || !aligned16(out) || !aligned16(bias) || !aligned16(residual))
        return fail(SC_ERR_UNSUPPORTED, "linear: pointers must be 16-byte aligned");
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    // column tile: all outputs up to 256, else the smallest split into equal multiples of 64 <= 256
    // (the epilogue stores 64-column boxes); halved while the grid has fewer tiles than SMs
    int64_t ny = (cout + 255) / 256;
    while (cout % ny != 0 || (cout / ny) % 64 != 0) ++ny;
    int tile_n = (int)(cout / ny);
    const int64_t row_tiles = (rows + 127) / 128;
    while (row_tiles * (cout / tile_n) < sm_count() && tile_n >= 128 && (tile_n / 2) % 64 == 0 &&
           cout % (tile_n / 2) == 0)
        tile_n /= 2;
    int S = 8;
    while (S > 2 && lin_smem_bytes(tile_n, S) > kMaxDynSmem) --S;
    CUtensorMap amap, bmap;
    cuuint64_t ad[2] = {(cuuint64_t)cin, (cuuint64_t)rows};
    cuuint64_t bd[2] = {(cuuint64_t)cin, (cuuint64_t)cout};
    cuuint64_t st[1] = {(cuuint64_t)cin * 2};
    cuuint32_t abox[2] = {64u, 128u};
    cuuint32_t bbox[2] = {64u, (cuuint32_t)tile_n};
    cuuint32_t es[2] = {1u, 1u};
    CUresult r1 = enc(&amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), ad, st, abox, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = enc(&bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), bd, st, bbox, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUtensorMap omap;
    cuuint64_t od[2] = {(cuuint64_t)cout, (cuuint64_t)rows};
    cuuint64_t ost[1] = {(cuuint64_t)cout * 2};
    cuuint32_t obox[2] = {64u, 32u};
    CUresult r3 = enc(&omap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, od, ost, obox, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS || r3 != CUDA_SUCCESS)
        return fail(SC_ERR_CUDA, "cuTensorMapEncodeTiled (linear) failed");
    LinParams p;
    memset(&p, 0, sizeof p);
    p.rows = rows;
    p.cin = (int)cin;
    p.cout = (int)cout;
    p.tile_n = tile_n;
    p.grid_y = (int)(cout / tile_n);
    p.n_tiles = row_tiles * p.grid_y;
    p.stages = S;
    p.bias = bias;
    p.residual = static_cast<const __nv_bfloat16*>(residual);
    p.silu = silu;
    p.out = static_cast<__nv_bfloat16*>(out);
    static std::once_flag lin_once;
    static cudaError_t lin_err = cudaSuccess;
    std::call_once(lin_once, [] {
        lin_err = cudaFuncSetAttribute((const void*)linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kMaxDynSmem);
    });
    SC_CUDA_TRY(lin_err);
    const int64_t ctas = std::min<int64_t>(p.n_tiles, sm_count());
    linear_tc_kernel<<<(unsigned)ctas, LIN_THREADS, lin_smem_bytes(tile_n, S), static_cast<cudaStream_t>(stream)>>>(
        amap, bmap, omap, p);
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_gather_rows(const void* src, int64_t n_src, int64_t row_bytes, const int32_t* idx, int64_t n, void* dst,
                   void* stream) {
    if (n < 0 || n_src < 0 || row_bytes <= 0) return fail(SC_ERR_INVALID, "invalid gather shape");
    if (row_bytes % 16 != 0) return fail(SC_ERR_UNSUPPORTED, "gather rows must be a multiple of 16 bytes");
    if (n == 0) return SC_OK;
    if (!src || !idx || !dst || !aligned16(src) || !aligned16(dst))
        return fail(SC_ERR_INVALID, "null or unaligned gather pointer");
    const int64_t units = row_bytes / 16;
    gather_rows_kernel<<<grid1d(n * units, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), units, idx, n, n_src, static_cast<uint4*>(dst));
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_bf16_round(const float* x, int64_t n, float* y, void* stream) {
    if (n < 0) return fail(SC_ERR_INVALID, "negative length");
    if (n == 0) return SC_OK;
    bf16_round_kernel<<<grid1d(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, y);
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_cast(sc_dtype from, sc_dtype to, const void* x, int64_t n, void* y, void* stream) {
    if (n < 0) return fail(SC_ERR_INVALID, "negative length");
    if (n == 0) return SC_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (from == SC_DTYPE_F32 && to == SC_DTYPE_BF16)
        cast_kernel<float, __nv_bfloat16><<<grid1d(n, 256), 256, 0, st>>>(
            static_cast<const float*>(x), n, static_cast<__nv_bfloat16*>(y));
    else if (from == SC_DTYPE_BF16 && to == SC_DTYPE_F32)
        cast_kernel<__nv_bfloat16, float><<<grid1d(n, 256), 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(x), n, static_cast<float*>(y));
    else
        return fail(SC_ERR_INVALID, "unsupported cast");
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

static size_t subdiv_cub_bytes(int64_t n) {
    size_t b = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr, (int)(n + 1));
    return b;
}

int sc_subdivide_scratch_bytes(int64_t n_parent, size_t* bytes) {
    if (n_parent < 0 || !bytes) return fail(SC_ERR_INVALID, "invalid subdivide scratch query");
    const size_t a = ((size_t)(n_parent + 1) * 4 + 255) / 256 * 256;
    *bytes = 2 * a + subdiv_cub_bytes(n_parent) + 256;
    return SC_OK;
}

static int validate_patchify(const sc_patchify3d_config* c) {
    if (!c) return fail(SC_ERR_INVALID, "null config");
    if (c->in_channels <= 0 || c->out_channels <= 0)
        return fail(SC_ERR_INVALID, "sparse patchify channel dimensions must be non-zero");
    if (c->frames <= 0 || c->height <= 0 || c->width <= 0)
        return fail(SC_ERR_INVALID, "sparse patchify input dimensions must be non-zero");
    if (c->tubelet_size <= 0 || c->patch_h <= 0 || c->patch_w <= 0)
        return fail(SC_ERR_INVALID, "sparse patchify patch dimensions must be non-zero");
    if (c->frames % c->tubelet_size != 0)
        return fail(SC_ERR_INVALID, "sparse patchify frames must be divisible by tubelet_size: " +
                                        std::to_string(c->frames) + " % " + std::to_string(c->tubelet_size) + " != 0");
    if (c->height % c->patch_h != 0)
        return fail(SC_ERR_INVALID, "sparse patchify height must be divisible by patch_h: " +
                                        std::to_string(c->height) + " % " + std::to_string(c->patch_h) + " != 0");
    if (c->width % c->patch_w != 0)
        return fail(SC_ERR_INVALID, "sparse patchify width must be divisible by patch_w: " +
                                        std::to_string(c->width) + " % " + std::to_string(c->patch_w) + " != 0");
    return SC_OK;
}

int sc_patchify3d_scratch_bytes(const sc_patchify3d_config* c, int64_t rows, sc_dtype dtype, size_t* bytes) {
    if (int rc = validate_patchify(c)) return rc;
    if (!bytes || rows < 0) return fail(SC_ERR_INVALID, "invalid arguments");
    const int64_t K = c->in_channels * c->tubelet_size * c->patch_h * c->patch_w;
    const size_t es = dtype == SC_DTYPE_BF16 ? 2 : 4;
    *bytes = align256((size_t)rows * 4) + align256((size_t)rows * (size_t)K * es);
    return SC_OK;
}

int sc_patchify3d_forward(const sc_patchify3d_config* c, sc_dtype dtype, const void* input, int64_t input_elems,
                          const int32_t* coords, int64_t rows, const void* weight, const float* bias, void* scratch,
                          size_t scratch_bytes, void* out, void* stream) {
    if (int rc = validate_patchify(c)) return rc;
    if (dtype != SC_DTYPE_F32 && dtype != SC_DTYPE_BF16) return fail(SC_ERR_INVALID, "sparse patchify: bad dtype");
    const int64_t per_batch = c->in_channels * c->frames * c->height * c->width;
    if (input_elems < 0 || input_elems % per_batch != 0)
        return fail(SC_ERR_INVALID, "sparse patchify input len mismatch: got " + std::to_string(input_elems) +
                                        " expected a multiple of " + std::to_string(per_batch));
    if (rows < 0) return fail(SC_ERR_INVALID, "invalid row count");
    if (rows == 0) return SC_OK;
    if (rows > 0x7fffffff) return fail(SC_ERR_UNSUPPORTED, "sparse patchify: too many rows");
    size_t need = 0;
    sc_patchify3d_scratch_bytes(c, rows, dtype, &need);
    if (!scratch || scratch_bytes < need)
        return fail(SC_ERR_CAPACITY, "sparse patchify scratch too small: need " + std::to_string(need) + " bytes");
    if (!input || !coords || !weight || !out) return fail(SC_ERR_INVALID, "null pointer");
    if (!aligned16(coords)) return fail(SC_ERR_INVALID, "coordinates must be 16-byte aligned");
    const int64_t K = c->in_channels * c->tubelet_size * c->patch_h * c->patch_w;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* ident = static_cast<int32_t*>(scratch);
    void* cols = static_cast<uint8_t*>(scratch) + align256((size_t)rows * 4);
    iota_kernel<<<grid1d(rows, 256), 256, 0, st>>>(ident, rows);
    SC_CUDA_TRY(cudaGetLastError());
    PatchGeom g;
    g.cin = c->in_channels;
    g.frames = c->frames;
    g.height = c->height;
    g.width = c->width;
    g.batches = input_elems / per_batch;
    g.tub = (int)c->tubelet_size;
    g.ph = (int)c->patch_h;
    g.pw = (int)c->patch_w;
    if (dtype == SC_DTYPE_F32)
        patch_gather_kernel<float><<<grid1d(rows * K, 256), 256, 0, st>>>(
            static_cast<const float*>(input), reinterpret_cast<const int4*>(coords), rows, g, static_cast<float*>(cols));
    else
        patch_gather_kernel<__nv_bfloat16><<<grid1d(rows * K, 256), 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(input), reinterpret_cast<const int4*>(coords), rows, g,
            static_cast<__nv_bfloat16*>(cols));
    SC_CUDA_TRY(cudaGetLastError());
    // projection: the dense tensor-core linear where it applies, else a 1x1x1 conv over the
    // identity rows, weight [Cout, 1, 1, 1, K] = [Cout, K]
    {
        const int rc = sc_linear_forward(dtype, cols, rows, K, weight, c->out_channels, bias, nullptr, 0, out, stream);
        if (rc != SC_ERR_UNSUPPORTED) return rc;
    }
    sc_conv_config cc;
    memset(&cc, 0, sizeof cc);
    cc.in_channels = K;
    cc.out_channels = c->out_channels;
    cc.kernel_d = cc.kernel_h = cc.kernel_w = 1;
    cc.in_channels_per_group = K;
    cc.out_channels_per_group = c->out_channels;
    cc.groups = 1;
    for (int j = 0; j < 3; ++j) {
        cc.axis_order[j] = j;
        cc.axis_sign[j] = 1;
    }
    sc_epilogue e;
    memset(&e, 0, sizeof e);
    e.residual_repeat = 1;
    return sc_subm_conv_forward(&cc, dtype, cols, rows, ident, rows, weight, bias, &e, out, stream);
}

int sc_subdiv_head(sc_dtype dtype, const void* feats, int64_t n, int64_t channels, const void* weight,
                   const float* bias, float threshold, const float* h_child_thresholds, int center,
                   float* logits, uint8_t* mask, void* stream) {
    if (n < 0 || channels <= 0) return fail(SC_ERR_INVALID, "subdivision head: invalid sizes");
    if (n == 0) return SC_OK;
    if (!feats || !weight || !mask) return fail(SC_ERR_INVALID, "subdivision head: null pointer");
    if (dtype != SC_DTYPE_F32 && dtype != SC_DTYPE_BF16) return fail(SC_ERR_INVALID, "subdivision head: bad dtype");
    SubdivThresholds thr;
    for (int c = 0; c < 8; ++c) {
        const float ch = h_child_thresholds ? h_child_thresholds[c] : NAN;
        thr.t[c] = std::isfinite(ch) ? ch : threshold;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t threads = n * 32;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (dtype == SC_DTYPE_F32)
        subdiv_head_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(feats), n, (int)channels,
                                                         static_cast<const float*>(weight), bias, thr, center,
                                                         logits, mask);
    else
        subdiv_head_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(feats), n, (int)channels, static_cast<const __nv_bfloat16*>(weight),
            bias, thr, center, logits, mask);
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_subdivide_async(const int32_t* parent_coords, const uint8_t* mask, int64_t n_parent,
                       int64_t parent_channels, void* scratch, int32_t* child_row, int32_t* child_coords,
                       int64_t* skip_offset, int32_t* d_children, void* stream) {
    if (n_parent < 0 || !d_children) return fail(SC_ERR_INVALID, "invalid subdivide arguments");
    if (n_parent * 8 > 0x7fffffffLL) return fail(SC_ERR_UNSUPPORTED, "too many parents for int32 child rows");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_parent == 0) {
        SC_CUDA_TRY(cudaMemsetAsync(d_children, 0, 4, st));
        return SC_OK;
    }
    if (!parent_coords || !mask || !scratch || !child_row)
        return fail(SC_ERR_INVALID, "null pointer");
    if (parent_channels % 8 != 0) return fail(SC_ERR_INVALID, "channel2spatial: in_channels is not divisible by 8");
    if ((reinterpret_cast<uintptr_t>(mask) & 7u) != 0 || !aligned16(parent_coords) || !aligned16(child_coords))
        return fail(SC_ERR_INVALID, "mask must be 8-byte and coordinates 16-byte aligned");
    const size_t a = ((size_t)(n_parent + 1) * 4 + 255) / 256 * 256;
    int32_t* counts = static_cast<int32_t*>(scratch);
    int32_t* offsets = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + a);
    void* tmp = static_cast<uint8_t*>(scratch) + 2 * a;
    size_t tmp_bytes = subdiv_cub_bytes(n_parent);
    subdiv_count_kernel<<<grid1d(n_parent + 1, 256), 256, 0, st>>>(mask, n_parent, counts);
    SC_CUDA_TRY(cudaGetLastError());
    SC_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, offsets, (int)(n_parent + 1), st));
    SC_CUDA_TRY(cudaMemcpyAsync(d_children, offsets + n_parent, 4, cudaMemcpyDeviceToDevice, st));
    subdiv_write_kernel<<<grid1d(n_parent, 256), 256, 0, st>>>(
        reinterpret_cast<const int4*>(parent_coords), mask, n_parent, parent_channels, offsets, child_row,
        reinterpret_cast<int4*>(child_coords), skip_offset);
    SC_CUDA_TRY(cudaGetLastError());
    return SC_OK;
}

int sc_subdivide(const int32_t* parent_coords, const uint8_t* mask, int64_t n_parent,
                 int64_t parent_channels, void* scratch, int32_t* child_row, int32_t* child_coords,
                 int64_t* skip_offset, int64_t* h_children, void* stream) {
    if (n_parent < 0 || !h_children) return fail(SC_ERR_INVALID, "invalid subdivide arguments");
    *h_children = 0;
    if (n_parent == 0) return SC_OK;
    if (!scratch) return fail(SC_ERR_INVALID, "null pointer");
    // the count goes to the scratch's spare tail (sc_subdivide_scratch_bytes leaves 256 bytes)
    size_t bytes = 0;
    sc_subdivide_scratch_bytes(n_parent, &bytes);
    int32_t* d_count = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + (bytes - 256 + 15) / 16 * 16);
    if (int rc = sc_subdivide_async(parent_coords, mask, n_parent, parent_channels, scratch, child_row,
                                    child_coords, skip_offset, d_count, stream))
        return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t total = 0;
    SC_CUDA_TRY(cudaMemcpyAsync(&total, d_count, 4, cudaMemcpyDeviceToHost, st));
    SC_CUDA_TRY(cudaStreamSynchronize(st));
    *h_children = total;
    return SC_OK;
}

}  // extern "C"
