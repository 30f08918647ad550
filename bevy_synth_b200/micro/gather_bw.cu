// Random-row gather bandwidth of this GPU, by copy method: 128-byte rows chosen by a
// hash from an L2-resident 64 MB table, gathered into shared-memory stages of 128 rows
// (the conv kernel's A-operand pattern) by cp.async (4 or 8 warps), TMA tile::gather4,
// or register-staged loads; one CTA per SM, a consumer warp releases the stages.
// Build and run: python -m bevy_synth_b200.perf gather
#include "../csrc/sc_common.cuh"
#include <cstdio>
#include <cuda.h>
#include <vector>
using namespace sc;
thread_local std::string sc::g_last_error;

constexpr int ROWS = 128;        // rows per stage
constexpr int STAGE = ROWS * 128;  // 16 KB
__device__ __forceinline__ int32_t hrow(uint32_t k) { k ^= k >> 16; k *= 0x7feb352du; k ^= k >> 15; k *= 0x846ca68bu; k ^= k >> 16; return (int32_t)(k & ((512u * 1024u) - 1u)); }
__global__ void __launch_bounds__(416, 1) gk(const __grid_constant__ CUtensorMap amap, const uint8_t* src, int64_t n_rows,
                                             const int32_t* idx, int64_t n_idx, int iters, int method, int nw, int S,
                                             float* sink) {
    extern __shared__ __align__(1024) uint8_t raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[16], empty[16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nprod = nw;  // producer warps: 0..nw-1 ; consumer warp: nw
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            int cnt = method == 0 ? nprod * 32 + 0 : 1;
            if (method == 2) cnt = nprod * 32;
            mbar_init(&full[s], method == 1 ? 1 : cnt);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * 7919;
    if (warp < nprod) {
        const int rows_per_w = ROWS / nprod;
        for (int it = 0; it < iters; ++it) {
            const int s = it % S;
            const uint32_t ph = (it / S) & 1;
            mbar_wait(&empty[s], ph ^ 1);
            const uint32_t st = smem_u32(sm + s * STAGE);
            if (method == 0) {  // cp.async, 4 rows x 128 B per instruction
                const int sub = lane >> 3, j = lane & 7;
                for (int g = 0; g < rows_per_w / 4; ++g) {
                    const int r = warp * rows_per_w + g * 4 + sub;
                    const int64_t row = hrow((uint32_t)(base + (int64_t)it * ROWS + r));
                    cp_async_16(st + r * 128 + ((j ^ (r & 7)) << 4), src + row * 128 + j * 16, 16u);
                }
                cp_async_arrive_noinc(&full[s]);
            } else if (method == 1) {  // TMA gather4, lanes issue one each
                if (warp == 0 && lane == 0) mbar_arrive_expect_tx(&full[s], STAGE);
                __syncwarp();
                const int groups = rows_per_w / 4;
                if (lane < groups) {
                    const int r = warp * rows_per_w + lane * 4;
                    int y[4];
                    for (int e = 0; e < 4; ++e) y[e] = hrow((uint32_t)(base + (int64_t)it * ROWS + r + e));
                    tma_gather4(st + r * 128, &amap, &full[s], 0, y[0], y[1], y[2], y[3]);
                }
            } else if (method == 2) {  // ldg.128 + sts.128, then arrive
                const int sub = lane >> 3, j = lane & 7;
                int4 v[8];
                const int G = rows_per_w / 4;
                for (int g0 = 0; g0 < G; g0 += 8) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) if (g0 + u < G) {
                        const int r = warp * rows_per_w + (g0 + u) * 4 + sub;
                        const int64_t row = hrow((uint32_t)(base + (int64_t)it * ROWS + r));
                        v[u] = *reinterpret_cast<const int4*>(src + row * 128 + j * 16);
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) if (g0 + u < G) {
                        const int r = warp * rows_per_w + (g0 + u) * 4 + sub;
                        *reinterpret_cast<int4*>(sm + s * STAGE + r * 128 + ((j ^ (r & 7)) << 4)) = v[u];
                    }
                }
                mbar_arrive(&full[s]);
            }
        }
    } else if (warp == nprod) {
        float acc = 0.f;
        for (int it = 0; it < iters; ++it) {
            const int s = it % S;
            mbar_wait(&full[s], (it / S) & 1);
            if (method == 0) fence_proxy_async_smem();
            acc += (float)sm[s * STAGE + lane * 4];
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (acc == 12345.f) sink[0] = acc;
    }
    cp_async_wait<0>();
}

typedef CUresult (*EncFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                         const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                         CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
int main() {
    const int64_t n_rows = 512 * 1024;  // 64 MB of 128-byte rows (L2-resident)
    uint8_t* src; cudaMalloc(&src, n_rows * 128); cudaMemset(src, 1, n_rows * 128);
    const int64_t n_idx = 1 << 22;
    std::vector<int32_t> h(n_idx);
    uint64_t x = 88172645463325252ull;
    for (auto& v : h) { x ^= x << 13; x ^= x >> 7; x ^= x << 17; v = (int32_t)(x % n_rows); }
    int32_t* idx; cudaMalloc(&idx, n_idx * 4); cudaMemcpy(idx, h.data(), n_idx * 4, cudaMemcpyHostToDevice);
    float* sink; cudaMalloc(&sink, 4);
    EncFn enc = nullptr; cudaDriverEntryPointQueryResult q;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&enc, cudaEnableDefault, &q);
    CUtensorMap amap;
    cuuint64_t dims[2] = {64, (cuuint64_t)n_rows}; cuuint64_t str[1] = {128};
    cuuint32_t box[2] = {64, 1}; cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, src, dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r) { printf("encode failed %d\n", (int)r); return 1; }
    int sms; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const int smem = 1024 + 12 * STAGE;
    cudaFuncSetAttribute(gk, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    struct C { int method, nw, S; const char* name; } cs[] = {
        {0, 4, 8, "cp.async 4 warps S=8"}, {0, 8, 8, "cp.async 8 warps S=8"}, {0, 4, 12, "cp.async 4 warps S=12"},
        {0, 4, 4, "cp.async 4 warps S=4"}, {1, 4, 8, "gather4 4 warps S=8"}, {1, 1, 8, "gather4 1 warp S=8"},
        {1, 4, 12, "gather4 4 warps S=12"}, {2, 4, 8, "ldg+sts 4 warps S=8"}, {2, 8, 8, "ldg+sts 8 warps S=8"}};
    for (auto& c : cs) {
        const int iters = 2000;
        gk<<<sms, (c.nw + 1) * 32, smem>>>(amap, src, n_rows, idx, n_idx, 100, c.method, c.nw, c.S, sink);
        cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
        cudaEventRecord(a);
        gk<<<sms, (c.nw + 1) * 32, smem>>>(amap, src, n_rows, idx, n_idx, iters, c.method, c.nw, c.S, sink);
        cudaEventRecord(b); cudaEventSynchronize(b);
        float ms; cudaEventElapsedTime(&ms, a, b);
        const double bytes = (double)sms * iters * STAGE;
        printf("%-26s %7.2f TB/s  %6.1f B/clk/SM@1.9GHz  err=%s\n", c.name, bytes / ms / 1e9, bytes / ms / 1e-3 / sms / 1.9e9,
               cudaGetErrorString(cudaGetLastError()));
    }
    uint32_t f = 0; cudaMemcpyFromSymbol(&f, g_fault, 4); printf("fault %u\n", f);
    return 0;
}
