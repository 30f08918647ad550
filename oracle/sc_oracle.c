/*
 * sc_oracle.c -- CPU restatement of the reference's sparse submanifold
 * convolution path.  TEST INFRASTRUCTURE ONLY: the parity checker and the
 * timed CPU baseline.  The product (libsparseconv.so) never links it.
 *
 * Each function cites the reference lines it follows (paths relative to the
 * mosure/bevy_synth repository root).
 */
#include "sc_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_err[512];

const char* oc_last_error(void) { return g_err; }

static int fail(const char* msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return -1;
}

/* crates/burn_flex_gmm/src/lib.rs:698-725 (validate_config) */
int oc_validate_config(const oc_conv_config* c) {
    if (c->in_channels == 0 || c->out_channels == 0)
        return fail("sparse conv channel dimensions must be non-zero");
    if (c->kernel_d == 0 || c->kernel_h == 0 || c->kernel_w == 0)
        return fail("sparse conv kernel dimensions must be non-zero");
    if (c->groups == 0) return fail("sparse conv groups must be non-zero");
    if (c->in_channels_per_group * c->groups != c->in_channels)
        return fail("sparse conv in_channels/group mismatch");
    if (c->out_channels_per_group * c->groups != c->out_channels)
        return fail("sparse conv out_channels/group mismatch");
    int used[3] = {0, 0, 0};
    for (int i = 0; i < 3; ++i) {
        int a = c->axis_order[i];
        if (a < 0 || a > 2 || used[a])
            return fail("sparse conv axis_order must be a permutation of [0,1,2]");
        used[a] = 1;
    }
    return 0;
}

/* lib.rs:59-67 (kernel_rows) */
int oc_kernel_rows(const oc_conv_config* c, int64_t* rows) {
    if (oc_validate_config(c)) return -1;
    *rows = c->kernel_d * c->kernel_h * c->kernel_w;
    return 0;
}

/* lib.rs:727-752 (kernel_layout): k = (kd*KH + kh)*KW + kw,
 * delta = axis_sign * (idx - K/2), offset[axis_order[j]] = delta[j]. */
int oc_kernel_offsets(const oc_conv_config* c, int32_t* off) {
    if (oc_validate_config(c)) return -1;
    int32_t cd = (int32_t)(c->kernel_d / 2), ch = (int32_t)(c->kernel_h / 2),
            cw = (int32_t)(c->kernel_w / 2);
    int64_t k = 0;
    for (int64_t kd = 0; kd < c->kernel_d; ++kd)
        for (int64_t kh = 0; kh < c->kernel_h; ++kh)
            for (int64_t kw = 0; kw < c->kernel_w; ++kw, ++k) {
                int32_t d[3] = {c->axis_sign[0] * ((int32_t)kd - cd),
                                c->axis_sign[1] * ((int32_t)kh - ch),
                                c->axis_sign[2] * ((int32_t)kw - cw)};
                int32_t o[3] = {0, 0, 0};
                o[c->axis_order[0]] = d[0];
                o[c->axis_order[1]] = d[1];
                o[c->axis_order[2]] = d[2];
                off[k * 3 + 0] = o[0];
                off[k * 3 + 1] = o[1];
                off[k * 3 + 2] = o[2];
            }
    return 0;
}

/* ---- coordinate -> row map: a plain open-addressing table over the full
 * 128-bit (batch,x,y,z) key.  Stands in for std::collections::HashMap. ---- */
typedef struct {
    uint32_t* keys; /* [cap*4] */
    int32_t* vals;  /* [cap]   -1 = empty */
    uint64_t mask;
} coord_table;

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static uint64_t coord_hash(const uint32_t* k) {
    uint64_t a = ((uint64_t)k[0] << 32) | k[1];
    uint64_t b = ((uint64_t)k[2] << 32) | k[3];
    return mix64(a ^ mix64(b + 0x9e3779b97f4a7c15ULL));
}

static int table_init(coord_table* t, int64_t n) {
    uint64_t cap = 16;
    while (cap < (uint64_t)n * 2) cap <<= 1;
    t->keys = (uint32_t*)malloc(cap * 4 * sizeof(uint32_t));
    t->vals = (int32_t*)malloc(cap * sizeof(int32_t));
    if (!t->keys || !t->vals) return fail("oracle: out of host memory");
    for (uint64_t i = 0; i < cap; ++i) t->vals[i] = -1;
    t->mask = cap - 1;
    return 0;
}

static void table_free(coord_table* t) {
    free(t->keys);
    free(t->vals);
}

static void table_insert(coord_table* t, const uint32_t* key, int32_t row, int dup_rule) {
    uint64_t s = coord_hash(key) & t->mask;
    for (;;) {
        if (t->vals[s] < 0) {
            memcpy(t->keys + s * 4, key, 16);
            t->vals[s] = row;
            return;
        }
        if (memcmp(t->keys + s * 4, key, 16) == 0) {
            /* HashMap::insert overwrites (last wins, lib.rs:83-86); device
             * builders keep the minimum row (neighbor_kernels.rs:249-256). */
            if (dup_rule == OC_DUP_LAST || row < t->vals[s]) t->vals[s] = row;
            return;
        }
        s = (s + 1) & t->mask;
    }
}

static int32_t table_find(const coord_table* t, const uint32_t* key) {
    uint64_t s = coord_hash(key) & t->mask;
    for (;;) {
        if (t->vals[s] < 0) return -1;
        if (memcmp(t->keys + s * 4, key, 16) == 0) return t->vals[s];
        s = (s + 1) & t->mask;
    }
}

/* lib.rs:69-109 (build_neighbor_rows), generalised to a separate query set
 * so that chunked / halo queries (sparse_decoder_tests.rs:238-292) can be
 * expressed.  Negative neighbor components are rejected (lib.rs:95-97); no
 * upper bound check exists in the reference. */
int oc_build_neighbor_rows_query(const oc_conv_config* cfg, const uint32_t* in_coords,
                                 int64_t n_in, const uint32_t* q, int64_t n_q, int dup_rule,
                                 int32_t* out) {
    if (oc_validate_config(cfg)) return -1;
    if (n_in > 2147483647LL) return fail("sparse conv coord row count exceeds i32::MAX");
    int64_t K;
    oc_kernel_rows(cfg, &K);
    int32_t* off = (int32_t*)malloc((size_t)K * 3 * sizeof(int32_t));
    oc_kernel_offsets(cfg, off);
    for (int64_t i = 0; i < n_q * K; ++i) out[i] = -1;
    if (n_in == 0 || n_q == 0) {
        free(off);
        return 0;
    }
    coord_table t;
    if (table_init(&t, n_in)) {
        free(off);
        return -1;
    }
    for (int64_t r = 0; r < n_in; ++r) table_insert(&t, in_coords + r * 4, (int32_t)r, dup_rule);
    for (int64_t r = 0; r < n_q; ++r) {
        const uint32_t* c = q + r * 4;
        int32_t ox = (int32_t)c[1], oy = (int32_t)c[2], oz = (int32_t)c[3];
        for (int64_t k = 0; k < K; ++k) {
            int32_t nx = ox + off[k * 3], ny = oy + off[k * 3 + 1], nz = oz + off[k * 3 + 2];
            if (nx < 0 || ny < 0 || nz < 0) continue;
            uint32_t key[4] = {c[0], (uint32_t)nx, (uint32_t)ny, (uint32_t)nz};
            out[r * K + k] = table_find(&t, key);
        }
    }
    table_free(&t);
    free(off);
    return 0;
}

int oc_build_neighbor_rows(const oc_conv_config* cfg, const uint32_t* coords, int64_t n,
                           int dup_rule, int32_t* out) {
    return oc_build_neighbor_rows_query(cfg, coords, n, coords, n, dup_rule, out);
}

/* lib.rs:377-426 (pack_flex_weight): [Cout,KD,KH,KW,Cin/g] ->
 * [g][K*Cin/g][Cout/g] with k_col = kernel_idx*Cin/g + in_local. */
int oc_pack_flex_weight(const oc_conv_config* c, const float* w, float* packed) {
    if (oc_validate_config(c)) return -1;
    int64_t K = c->kernel_d * c->kernel_h * c->kernel_w;
    int64_t cin = c->in_channels_per_group, n = c->out_channels_per_group;
    int64_t k_in = K * cin;
    for (int64_t g = 0; g < c->groups; ++g) {
        float* pg = packed + g * k_in * n;
        for (int64_t ol = 0; ol < n; ++ol) {
            int64_t o = g * n + ol;
            for (int64_t k = 0; k < K; ++k)
                for (int64_t il = 0; il < cin; ++il)
                    pg[(k * cin + il) * n + ol] = w[(o * K + k) * cin + il];
        }
    }
    return 0;
}

/* C[m,n] += A[m,k] @ B[k,n] for a row block; stands in for the single
 * matrixmultiply::sgemm call of lib.rs:347-366 (alpha = beta = 1), which is
 * a packed, register-blocked SGEMM.  Here: K blocked by 256, a 6-row x
 * 16-column AVX2/FMA register tile (12 accumulators), scalar edges.  The full
 * K extent is multiplied, zero-filled (invalid) taps included, exactly as
 * the reference's dense sgemm does. */
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
static void tile_6x16(int64_t kc, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc) {
    __m256 c00 = _mm256_setzero_ps(), c01 = _mm256_setzero_ps(), c10 = _mm256_setzero_ps(),
           c11 = _mm256_setzero_ps(), c20 = _mm256_setzero_ps(), c21 = _mm256_setzero_ps(),
           c30 = _mm256_setzero_ps(), c31 = _mm256_setzero_ps(), c40 = _mm256_setzero_ps(),
           c41 = _mm256_setzero_ps(), c50 = _mm256_setzero_ps(), c51 = _mm256_setzero_ps();
    for (int64_t k = 0; k < kc; ++k) {
        const __m256 b0 = _mm256_loadu_ps(B + k * ldb), b1 = _mm256_loadu_ps(B + k * ldb + 8);
        __m256 a;
        a = _mm256_broadcast_ss(A + 0 * lda + k); c00 = _mm256_fmadd_ps(a, b0, c00); c01 = _mm256_fmadd_ps(a, b1, c01);
        a = _mm256_broadcast_ss(A + 1 * lda + k); c10 = _mm256_fmadd_ps(a, b0, c10); c11 = _mm256_fmadd_ps(a, b1, c11);
        a = _mm256_broadcast_ss(A + 2 * lda + k); c20 = _mm256_fmadd_ps(a, b0, c20); c21 = _mm256_fmadd_ps(a, b1, c21);
        a = _mm256_broadcast_ss(A + 3 * lda + k); c30 = _mm256_fmadd_ps(a, b0, c30); c31 = _mm256_fmadd_ps(a, b1, c31);
        a = _mm256_broadcast_ss(A + 4 * lda + k); c40 = _mm256_fmadd_ps(a, b0, c40); c41 = _mm256_fmadd_ps(a, b1, c41);
        a = _mm256_broadcast_ss(A + 5 * lda + k); c50 = _mm256_fmadd_ps(a, b0, c50); c51 = _mm256_fmadd_ps(a, b1, c51);
    }
#define ACC(r, lo, hi)                                                                        \
    _mm256_storeu_ps(C + r * ldc, _mm256_add_ps(_mm256_loadu_ps(C + r * ldc), lo));           \
    _mm256_storeu_ps(C + r * ldc + 8, _mm256_add_ps(_mm256_loadu_ps(C + r * ldc + 8), hi));
    ACC(0, c00, c01) ACC(1, c10, c11) ACC(2, c20, c21) ACC(3, c30, c31) ACC(4, c40, c41) ACC(5, c50, c51)
#undef ACC
}
#endif

static void gemm_edge(int64_t m0, int64_t m1, int64_t n0, int64_t n1, int64_t k0, int64_t kc,
                      const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc) {
    for (int64_t m = m0; m < m1; ++m)
        for (int64_t j = n0; j < n1; ++j) {
            float acc = 0.0f;
            for (int64_t k = k0; k < k0 + kc; ++k) acc += A[m * lda + k] * B[k * ldb + j];
            C[m * ldc + j] += acc;
        }
}

static void gemm_accumulate(int64_t M, int64_t Kd, int64_t N, const float* A, int64_t lda,
                            const float* B, int64_t ldb, float* C, int64_t ldc) {
    const int64_t KC = 256;
    for (int64_t k0 = 0; k0 < Kd; k0 += KC) {
        const int64_t kc = Kd - k0 < KC ? Kd - k0 : KC;
#if defined(__AVX2__) && defined(__FMA__)
        const int64_t M6 = M - M % 6, N16 = N - N % 16;
        for (int64_t j = 0; j < N16; j += 16)
            for (int64_t m = 0; m < M6; m += 6)
                tile_6x16(kc, A + m * lda + k0, lda, B + k0 * ldb + j, ldb, C + m * ldc + j, ldc);
        gemm_edge(M6, M, 0, N, k0, kc, A, lda, B, ldb, C, ldc);
        gemm_edge(0, M6, N16, N, k0, kc, A, lda, B, ldb, C, ldc);
#else
        gemm_edge(0, M, 0, N, k0, kc, A, lda, B, ldb, C, ldc);
#endif
    }
}

/* lib.rs:242-375 (sparse_subm_conv_forward_flex_precomputed).
 * out = bias; per group: gather [m, K*Cin/g] (zeros for -1), then
 * out[:, group cols] += gathered @ packed_group.  The gather is done in row
 * blocks of 256 so that memory stays bounded on large inputs; the per-element
 * arithmetic is the reference's.  n_threads > 1 spreads row blocks over
 * OpenMP threads (the reference is single-threaded: matrixmultiply 0.3.10
 * is built without its `threading` feature, Cargo.lock:6677-6684). */
int oc_subm_conv_flex_precomputed(const oc_conv_config* c, const float* weight, const float* bias,
                                  const float* input, int64_t input_rows, const int32_t* nbr,
                                  int64_t rows, const float* packed_in, int n_threads,
                                  float* out) {
    if (oc_validate_config(c)) return -1;
    if (input_rows < rows) return fail("sparse conv input row mismatch");
    if (rows == 0) return 0;
    int64_t K = c->kernel_d * c->kernel_h * c->kernel_w;
    int64_t cin = c->in_channels_per_group, n = c->out_channels_per_group;
    int64_t k_in = K * cin, Cout = c->out_channels;
    for (int64_t i = 0; i < rows * K; ++i) {
        int32_t r = nbr[i];
        if (r == -1) continue;
        if (r < 0) return fail("sparse conv neighbor row index is negative");
        if (r >= input_rows) return fail("sparse conv neighbor row index out of bounds");
    }
    float* packed_own = NULL;
    const float* packed = packed_in;
    if (!packed) {
        packed_own = (float*)malloc((size_t)(c->groups * k_in * n) * sizeof(float));
        if (!packed_own) return fail("oracle: out of host memory");
        oc_pack_flex_weight(c, weight, packed_own);
        packed = packed_own;
    }
    for (int64_t r = 0; r < rows; ++r) memcpy(out + r * Cout, bias, (size_t)Cout * sizeof(float));

    const int64_t RB = 256;
    int64_t nblocks = (rows + RB - 1) / RB;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel num_threads(n_threads)
#endif
    {
        float* g = (float*)malloc((size_t)(RB * k_in) * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (int64_t b = 0; b < nblocks; ++b) {
            int64_t r0 = b * RB, m = rows - r0 < RB ? rows - r0 : RB;
            for (int64_t grp = 0; grp < c->groups; ++grp) {
                memset(g, 0, (size_t)(m * k_in) * sizeof(float));
                for (int64_t i = 0; i < m; ++i)
                    for (int64_t k = 0; k < K; ++k) {
                        int32_t src = nbr[(r0 + i) * K + k];
                        if (src == -1) continue;
                        memcpy(g + i * k_in + k * cin, input + (int64_t)src * c->in_channels + grp * cin,
                               (size_t)cin * sizeof(float));
                    }
                gemm_accumulate(m, k_in, n, g, k_in, packed + grp * k_in * n, n,
                                out + r0 * Cout + grp * n, Cout);
            }
        }
        free(g);
    }
    free(packed_own);
    return 0;
}

/* lib.rs:428-510 (sparse_subm_conv_forward_legacy): naive per-pair dot
 * products, bias first; independent of the GEMM above. */
int oc_subm_conv_legacy(const oc_conv_config* c, const float* w, const float* bias,
                        const uint32_t* coords, int64_t n, const float* input, float* out) {
    if (oc_validate_config(c)) return -1;
    if (n == 0) return 0;
    int64_t K = c->kernel_d * c->kernel_h * c->kernel_w;
    int64_t Cout = c->out_channels, cin = c->in_channels_per_group;
    int32_t* off = (int32_t*)malloc((size_t)K * 3 * sizeof(int32_t));
    oc_kernel_offsets(c, off);
    for (int64_t r = 0; r < n; ++r) memcpy(out + r * Cout, bias, (size_t)Cout * sizeof(float));
    coord_table t;
    if (table_init(&t, n)) {
        free(off);
        return -1;
    }
    for (int64_t r = 0; r < n; ++r) table_insert(&t, coords + r * 4, (int32_t)r, OC_DUP_LAST);
    for (int64_t r = 0; r < n; ++r) {
        const uint32_t* cc = coords + r * 4;
        for (int64_t k = 0; k < K; ++k) {
            int32_t s[3] = {(int32_t)cc[1] + off[k * 3], (int32_t)cc[2] + off[k * 3 + 1],
                            (int32_t)cc[3] + off[k * 3 + 2]};
            if (s[0] < 0 || s[1] < 0 || s[2] < 0) continue;
            uint32_t key[4] = {cc[0], (uint32_t)s[0], (uint32_t)s[1], (uint32_t)s[2]};
            int32_t src = table_find(&t, key);
            if (src < 0) continue;
            const float* in_row = input + (int64_t)src * c->in_channels;
            for (int64_t grp = 0; grp < c->groups; ++grp)
                for (int64_t ol = 0; ol < c->out_channels_per_group; ++ol) {
                    int64_t o = grp * c->out_channels_per_group + ol;
                    const float* wr = w + (o * K + k) * cin;
                    float acc = 0.0f;
                    for (int64_t il = 0; il < cin; ++il) acc += in_row[grp * cin + il] * wr[il];
                    out[r * Cout + o] += acc;
                }
        }
    }
    table_free(&t);
    free(off);
    return 0;
}

/* burn_trellis/src/runtime_model/sparse_decoder_wgpu_ops.rs:1642-1711
 * (layer_norm_inplace): sequential-sum mean, then biased variance
 * sum((x-mean)^2)/C, inv_std = 1/sqrt(var+eps), optional gamma then beta. */
int oc_layer_norm_inplace(float* data, int64_t rows, int64_t C, const float* gamma,
                          const float* beta, float eps) {
    if (rows == 0 || C == 0) return 0;
    for (int64_t r = 0; r < rows; ++r) {
        float* x = data + r * C;
        float s = 0.0f;
        for (int64_t i = 0; i < C; ++i) s += x[i];
        float mean = s / (float)C;
        float v = 0.0f;
        for (int64_t i = 0; i < C; ++i) {
            float d = x[i] - mean;
            v += d * d;
        }
        float var = v / (float)C;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int64_t i = 0; i < C; ++i) {
            float y = (x[i] - mean) * inv_std;
            if (gamma) y *= gamma[i];
            if (beta) y += beta[i];
            x[i] = y;
        }
    }
    return 0;
}

/* sparse_decoder_wgpu_ops.rs:1713-1720 (silu_inplace): x / (1 + exp(-x)). */
void oc_silu_inplace(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* burn_flex_gmm/src/wgpu.rs:57-67 (bf16_round_to_f32_kernel): RNE on the f32
 * bit pattern, (bits + 0x7fff + lsb) & 0xffff0000, no NaN special case. */
void oc_bf16_round_inplace(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        uint32_t b;
        memcpy(&b, x + i, 4);
        uint32_t lsb = (b >> 16) & 1u;
        b = (b + 0x7fffu + lsb) & 0xffff0000u;
        memcpy(x + i, &b, 4);
    }
}

/* sparse_decoder_wgpu_ops.rs:1722-1726 (quantize_f16_inplace):
 * half::f16::from_f32 (round to nearest even) then back to f32. */
void oc_f16_round_inplace(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = (float)(_Float16)x[i];
}

/* sparse_decoder_wgpu_ops.rs:1999-2054 (channel2spatial): parent-major,
 * child-minor; child c = cx + 2cy + 4cz takes channel block
 * [c*Cin/8, (c+1)*Cin/8); child coord = 2*xyz + (cx,cy,cz). */
int oc_channel2spatial(const uint32_t* coords, int64_t rows, const float* feats, int64_t cin,
                       const uint8_t* mask, uint32_t* oc, float* of, int64_t* out_rows) {
    *out_rows = 0;
    if (rows == 0) return 0;
    if (cin % 8 != 0) return fail("channel2spatial: in_channels is not divisible by 8");
    int64_t co = cin / 8, w = 0;
    for (int64_t r = 0; r < rows; ++r)
        for (int child = 0; child < 8; ++child) {
            if (!mask[r * 8 + child]) continue;
            const uint32_t* c = coords + r * 4;
            oc[w * 4 + 0] = c[0];
            oc[w * 4 + 1] = c[1] * 2u + (uint32_t)(child & 1);
            oc[w * 4 + 2] = c[2] * 2u + (uint32_t)((child >> 1) & 1);
            oc[w * 4 + 3] = c[3] * 2u + (uint32_t)((child >> 2) & 1);
            memcpy(of + w * co, feats + r * cin + child * co, (size_t)co * sizeof(float));
            ++w;
        }
    *out_rows = w;
    return 0;
}

/* sparse_decoder_wgpu_ops.rs:2056-2076 (repeat_interleave_channels). */
int oc_repeat_interleave_channels(const float* f, int64_t rows, int64_t cin, int64_t rep,
                                  float* out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t i = 0; i < cin; ++i)
            for (int64_t j = 0; j < rep; ++j) out[(r * cin + i) * rep + j] = f[r * cin + i];
    return 0;
}
