/*
 * sparseconv.h -- C ABI of the B200 (sm_100a) sparse submanifold convolution
 * library (libsparseconv.so).
 *
 * The entry points are what the reference's operator boundary would bind
 * (mosure/bevy_synth, crate burn_flex_gmm, paths relative to the crate):
 *
 *   sc_neighbor_map        <- wgpu::neighbor_rows_tensor_from_coords_tensor
 *                             (src/wgpu/neighbor.rs:977-1006)
 *   sc_subm_conv_forward   <- wgpu::sparse_subm_conv_forward_cubecl
 *                             (src/wgpu/sparse_conv.rs:293-308); the fused
 *                             epilogue replaces the separate
 *                             layer_norm_affine(_silu)_forward_wgpu passes
 *                             (src/wgpu/ops.rs:1464-1639)
 *   sc_layer_norm_act      <- wgpu::layer_norm_affine(_silu)_forward_wgpu
 *                             (src/wgpu/ops.rs:1464-1639)
 *   sc_bf16_round          <- wgpu::bf16_round_to_f32_wgpu (src/wgpu.rs:57-102)
 *   sc_kernel_rows / sc_kernel_offsets
 *                          <- kernel_rows / kernel_layout (src/lib.rs:59-67, 727-752)
 *   sc_subdivide_*         <- burn_trellis decoder C2S helpers
 *                             (runtime_model/sparse_decoder_wgpu_ops.rs:995-1054,
 *                              1999-2076)
 *
 * Conventions (mirroring the reference's Result<_, String> boundary):
 *  - Every function returns SC_OK (0) or a negative SC_ERR_* code; the message
 *    of the last failure on the calling host thread is returned by
 *    sc_last_error().
 *  - Pointers named d_* are device pointers; h_* are host pointers.  Streams
 *    are cudaStream_t passed as void*; nothing synchronises implicitly unless
 *    documented (sc_neighbor_status, sc_device_fault).
 *  - Inputs are never modified; outputs are caller-allocated.  Empty inputs
 *    (zero rows) are valid and launch nothing.
 *  - Coordinates are int32 [N,4] = (batch, x, y, z), row-major.
 *  - Weights use the reference layout [Cout, KD, KH, KW, Cin/groups].
 */
#ifndef SPARSECONV_H
#define SPARSECONV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_OK 0
#define SC_ERR_INVALID (-1)     /* bad argument / shape (reference: Err(String)) */
#define SC_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define SC_ERR_UNSUPPORTED (-3) /* valid request outside what this build implements */
#define SC_ERR_CAPACITY (-4)    /* hash table full / probe limit / workspace too small */
#define SC_ERR_RANGE (-5)       /* coordinate component outside [0, 65534] */
#define SC_ERR_DEVICE (-6)      /* a kernel reported a fault (bounded wait expired,
                                   neighbor index out of range) */

typedef enum sc_dtype { SC_DTYPE_F32 = 0, SC_DTYPE_BF16 = 1 } sc_dtype;

/* Mirror of SparseSubmConvConfig (src/lib.rs:5-17). */
typedef struct sc_conv_config {
    int64_t in_channels;
    int64_t out_channels;
    int64_t kernel_d, kernel_h, kernel_w;
    int64_t in_channels_per_group;
    int64_t out_channels_per_group;
    int64_t groups;
    int32_t axis_order[3];
    int32_t axis_sign[3];
} sc_conv_config;

/* Fused epilogue of sc_subm_conv_forward.  With y = conv(x) + bias
 * (+ residual), the call writes
 *     out  = y                      when out2 != NULL, else  out = post(y)
 *     out2 = post(y)                (optional)
 * where post(y) = [LayerNorm over groups of ln_width columns, optional
 * affine gamma/beta] then [SiLU], each step only if enabled.
 * Zero-initialise the struct for "bias only". */
typedef struct sc_epilogue {
    const void* d_residual;        /* nullable; same dtype as out.  Element (i, j) is
                                      d_residual[i*Cout + j], or, when d_residual_offset
                                      is set, d_residual[d_residual_offset[i] + j / residual_repeat] */
    const int64_t* d_residual_offset; /* nullable [n_rows] element offsets (C2S skip path) */
    int32_t residual_repeat;       /* >= 1; channel repeat of the offset form */
    int32_t layer_norm;            /* 0/1 */
    int32_t ln_width;              /* LayerNorm group width in columns; 0 = Cout */
    float ln_eps;
    const float* d_ln_gamma;       /* nullable [ln_width] */
    const float* d_ln_beta;        /* nullable [ln_width] */
    int32_t silu;                  /* 0/1 */
    void* d_out2;                  /* nullable second output, same dtype/shape as out */
    const int32_t* d_out_row_map;  /* nullable [n_rows * out_row_map_cols]: scatter the
                                      column block b (width Cout / out_row_map_cols) of row i
                                      to output row d_out_row_map[i*cols + b] (skip if < 0);
                                      the output then has row width Cout / cols */
    int32_t out_row_map_cols;
    const int32_t* d_row_order;    /* nullable [n_rows] permutation: the order in which output
                                      rows are grouped into tiles (sc_neighbor_schedule);
                                      changes scheduling only, never results */
    const int32_t* d_neighbor_rows_ordered; /* nullable [n_rows, K]: d_neighbor_rows permuted into
                                      tile order (row p = row d_row_order[p]), as written by
                                      sc_neighbor_schedule; lets tiles read their map rows
                                      contiguously */
    const void* d_tile_sources;    /* nullable: the map's tile-source plan (sc_neighbor_tile_sources);
                                      with it a bf16 conv of 64 input channels, at most 128
                                      outputs and a bias/SiLU epilogue gathers each 128-row
                                      tile's distinct source rows once and builds the taps'
                                      A operands in tensor memory.  Rows run in map order
                                      (d_row_order unset).  Changes scheduling only. */
    int32_t tile_sources_max;      /* the plan's largest per-tile source count (its h_max_sources) */
} sc_epilogue;

/* ---- library / errors -------------------------------------------------- */
int sc_version(void);
/* Copies the calling thread's last error message; returns its length. */
int sc_last_error(char* h_buf, size_t len);
/* Reads and clears the sticky device fault word of the current device
 * (synchronises the device).  0 = no fault. */
int sc_device_fault(uint32_t* h_fault);
/* Sets the time limit of every bounded wait in this library's kernels on the
 * current device (ns; 0 restores the default of 2 s).  A wait that reaches it
 * raises FAULT_WAIT_TIMEOUT (bit 0 of the fault word) and its kernel drains
 * and returns.  No counterpart in the reference (its kernels do not wait). */
int sc_set_wait_limit_ns(uint64_t ns);

/* ---- kernel layout ------------------------------------------------------- */
int sc_kernel_rows(const sc_conv_config* cfg, int64_t* h_rows);
int sc_kernel_offsets(const sc_conv_config* cfg, int32_t* h_offsets /* [K*3] */);

/* ---- neighbor map ---------------------------------------------------------
 * Builds a coordinate hash table from d_in_coords and answers, for every
 * query row and kernel offset, the row of d_in_coords holding coord+offset
 * (same batch), or -1.  Duplicate coordinates resolve to the LOWEST row, as
 * every device builder of the reference does (src/wgpu/neighbor_kernels.rs:
 * 37-39, 249-256).  Coordinate components must lie in [0, 65534]; a violation
 * is recorded in the workspace status (SC_ERR_RANGE from sc_neighbor_status).
 * sc_neighbor_workspace_bytes gives a table of >= 4 n_in slots (load factor
 * <= 0.25); a workspace of at least 256 + 16 * (the power of two >= 2 n_in)
 * bytes is accepted and runs at load factor <= 0.5. */
int sc_neighbor_workspace_bytes(int64_t n_in, size_t* h_bytes);
int sc_neighbor_map(const sc_conv_config* cfg, const int32_t* d_coords, int64_t n_rows,
                    void* d_workspace, size_t workspace_bytes, int32_t* d_neighbor_rows,
                    void* stream);
int sc_neighbor_map_query(const sc_conv_config* cfg, const int32_t* d_in_coords, int64_t n_in,
                          const int32_t* d_query_coords, int64_t n_query, void* d_workspace,
                          size_t workspace_bytes, int32_t* d_neighbor_rows, void* stream);
/* Synchronises `stream`, then returns SC_OK or the error recorded by the
 * last map built in this workspace (SC_ERR_RANGE / SC_ERR_CAPACITY).
 * h_max_probe (nullable) receives the longest insert probe sequence. */
int sc_neighbor_status(const void* d_workspace, int32_t* h_max_probe, void* stream);

/* Neighbor map without any allocation, for callers that cannot allocate
 * device memory: they hold only the buffers they pass in (for instance a
 * burn/CubeCL backend whose device memory belongs to its own pool and which
 * hands a custom op nothing but its input and output tensors), or they must
 * not call cudaMalloc on their execution path.  Same result as
 * sc_neighbor_map.  No counterpart in the reference.
 *  - The hash table lives in a fixed 8 MiB static device array that every GPU
 *    loading the library holds until exit; n_rows is limited to 262,144
 *    (SC_ERR_CAPACITY beyond, checked before any GPU work).
 *  - Every call looks up the array's device address on the calling thread's
 *    current device (cudaGetSymbolAddress; no allocation).
 *  - Every call shares the one array and clears it first: calls that overlap
 *    on the GPU (other streams, other host threads) race and must be
 *    serialised by the caller.
 *  - Synchronises `stream` to read the table status, as sc_neighbor_status
 *    does, and returns SC_ERR_RANGE / SC_ERR_CAPACITY like it. */
int sc_neighbor_map_noalloc(const sc_conv_config* cfg, const int32_t* d_coords, int64_t n_rows,
                            int32_t* d_neighbor_rows, void* stream);

/* Conv schedule of a neighbor map, computed once and reused by every conv on
 * the same map: a processing order of output rows that groups rows with equal
 * neighbor masks (valid-tap bit patterns) so that tensor-core tiles skip more
 * taps, and (optional, nullable) the map permuted into that order.  Rows are
 * sorted by a K-bit key whose most significant bits are the taps farthest
 * from the centre; the sort is stable, so Morton order is kept within a
 * group.  K <= 32. */
int sc_neighbor_schedule_scratch_bytes(int64_t n_rows, size_t* h_bytes);
int sc_neighbor_schedule(const sc_conv_config* cfg, const int32_t* d_neighbor_rows, int64_t n_rows,
                         void* d_scratch, size_t scratch_bytes, int32_t* d_row_order,
                         int32_t* d_neighbor_rows_ordered, void* stream);

/* The same schedule with a per-row group above the tap key: rows are sorted
 * by group first (8 bits from d_group_mask8 [n_rows, 8] 0/1, bit c = column
 * c; nullable), then by their tap mask.  For the decoder's channel-to-space
 * conv1 the group is the kept-children mask: a tile of parents that keeps no
 * child in some column block then skips that block (see sc_epilogue). */
int sc_neighbor_schedule_grouped_scratch_bytes(int64_t n_rows, size_t* h_bytes);
int sc_neighbor_schedule_grouped(const sc_conv_config* cfg, const int32_t* d_neighbor_rows, int64_t n_rows,
                                 const uint8_t* d_group_mask8, void* d_scratch, size_t scratch_bytes,
                                 int32_t* d_row_order, int32_t* d_neighbor_rows_ordered, void* stream);

/* Tile-source plan of a neighbor map, computed once and reused by every
 * conv on the map: for each tile of 128 consecutive map rows, the sorted
 * distinct valid source rows it reads, a 16-bit index into that list for
 * every (row, tap), and the tile's tap mask.  On a Morton-ordered surface grid
 * a tile reads ~8x fewer distinct rows than (row, tap) pairs.  K <= 32.
 * Synchronises `stream` to read h_max_sources (the largest per-tile count);
 * returns SC_ERR_CAPACITY if a tile reads more than 576 distinct rows (the
 * plan is then unusable and convs run without it).  No counterpart in the
 * reference (a scheduling aid of this library). */
int sc_neighbor_tile_sources_bytes(int64_t n_rows, int64_t kernel_rows, size_t* h_bytes);
int sc_neighbor_tile_sources(const sc_conv_config* cfg, const int32_t* d_neighbor_rows, int64_t n_rows,
                             int64_t n_in, void* d_plan, size_t plan_bytes, int32_t* h_max_sources,
                             void* stream);

/* ---- convolution ----------------------------------------------------------
 * out[n_rows, Cout] = bias + sum_k sum_c in[nbr[r,k], c] * W[o,k,c]  (+ epilogue)
 * d_input [n_in, Cin], d_neighbor_rows [n_rows, K] with n_rows <= n_in
 * (SC_ERR_INVALID otherwise, as the reference's "neighbor row count exceeds
 * input rows" check, src/wgpu/sparse_conv.rs:439-444; the map's entries may
 * address any input row < n_in, e.g. halo rows appended after the query
 * rows), d_weight [Cout, KD, KH, KW, Cin/groups] in `dtype`, d_bias [Cout]
 * fp32 (nullable = zero).  fp32 accumulates in fp32 FFMA.  bf16 runs on
 * tcgen05 tensor cores (fp32 accumulation in TMEM) when groups == 1, K <= 32,
 * Cin >= 64, Cin % 8 == 0, Cout % 32 == 0, the output column tile (Cout, or
 * Cout / out_row_map_cols with a row map) is at most 512 wide with any
 * LayerNorm width dividing it, and every pointer the kernel reads in 16-byte
 * vectors (input, weight, bias, map, residual, LayerNorm parameters, outputs)
 * is 16-byte aligned; otherwise on a CUDA-core kernel
 * (sc_conv_uses_tensor_cores reports the choice for an unfused conv).
 * Neighbor indices outside [-1, n_in) read as zero and raise the device fault
 * word. */
int sc_subm_conv_forward(const sc_conv_config* cfg, sc_dtype dtype, const void* d_input,
                         int64_t n_in, const int32_t* d_neighbor_rows, int64_t n_rows,
                         const void* d_weight, const float* d_bias, const sc_epilogue* epi,
                         void* d_out, void* stream);

/* Chooses the kernel family for a conv: 1 = tcgen05, 0 = CUDA cores. */
int sc_conv_uses_tensor_cores(const sc_conv_config* cfg, sc_dtype dtype, int32_t* h_flag);

/* ---- row ops ------------------------------------------------------------- */
/* y = [SiLU]( LN(x) * gamma + beta ) over rows of `channels` (gamma/beta
 * nullable); layer_norm = 0 skips the normalisation.  In-place allowed. */
int sc_layer_norm_act(sc_dtype dtype, const void* d_x, int64_t rows, int64_t channels,
                      const float* d_gamma, const float* d_beta, float eps, int32_t layer_norm,
                      int32_t silu, void* d_y, void* stream);
/* dst[i] = src[idx[i]] for n rows of row_bytes (a multiple of 16) each: packs
 * the boundary rows another rank needs (halo exchange).  Indices outside
 * [0, n_src) give zero rows and raise the device fault word.  Plays the role
 * of burn's Tensor::select by row index (crates/burn_trellis/src/runtime_model/
 * sparse_decoder_runtime_impl.rs:2249-2255). */
int sc_gather_rows(const void* d_src, int64_t n_src, int64_t row_bytes, const int32_t* d_idx, int64_t n,
                   void* d_dst, void* stream);
/* fp32 -> fp32 rounded to bf16 (RNE, no NaN special case). */
int sc_bf16_round(const float* d_x, int64_t n, float* d_y, void* stream);
/* fp32 <-> bf16 storage conversion (RNE). */
int sc_cast(sc_dtype from, sc_dtype to, const void* d_x, int64_t n, void* d_y, void* stream);

/* ---- channel-to-space subdivision (decoder upsample) ----------------------
 * From a parent mask [n_parent, 8] (uint8, child c = cx + 2cy + 4cz), computes
 * child_row[p*8 + c] (-1 where not kept) in parent-major / child-minor order,
 * the child count, child coordinates (batch, 2x+cx, 2y+cy, 2z+cz) and the
 * element offsets of the skip path (p*Cin + c*Cin/8).  d_scratch must hold
 * sc_subdivide_scratch_bytes(n_parent) bytes.  h_children receives the count
 * (this synchronises the stream, as the reference's argwhere count does). */
int sc_subdivide_scratch_bytes(int64_t n_parent, size_t* h_bytes);
int sc_subdivide(const int32_t* d_parent_coords, const uint8_t* d_mask, int64_t n_parent,
                 int64_t parent_channels, void* d_scratch, int32_t* d_child_row,
                 int32_t* d_child_coords /* [<= 8*n_parent, 4] */,
                 int64_t* d_skip_offset /* [<= 8*n_parent] */, int64_t* h_children,
                 void* stream);

/* The same without the host read: the child count is written to d_children
 * (one int32 on the device) and nothing synchronises.  A caller enqueues the
 * work that needs no child count (the parents' LayerNorm, map and schedule,
 * and conv1, whose outputs it sizes by the 8*n_parent bound) before it reads
 * the count, so the GPU does not wait for the host at this point. */
int sc_subdivide_async(const int32_t* d_parent_coords, const uint8_t* d_mask, int64_t n_parent,
                       int64_t parent_channels, void* d_scratch, int32_t* d_child_row,
                       int32_t* d_child_coords /* [8*n_parent, 4] */,
                       int64_t* d_skip_offset /* [8*n_parent] */, int32_t* d_children,
                       void* stream);

/* ---- dense linear layer ---------------------------------------------------
 * out[r, o] = act(bias[o] + sum_c x[r, c] * W[o, c] (+ residual[r, o])) for
 * bf16 x [rows, cin], W [cout, cin] (PyTorch linear layout), fp32 bias
 * (nullable), bf16 residual [rows, cout] (nullable), act = SiLU when silu != 0
 * (the order of sc_subm_conv_forward's epilogue).  Replaces burn_trellis linear_forward
 * (runtime_model/sparse_decoder_wgpu_ops.rs:1-60) and the ConvNeXt MLP's two
 * layers (:355-489).  Both operands arrive by TMA tiles (no neighbor map).
 * Needs cin % 8 == 0, cout % 32 == 0 and 16-byte aligned pointers; returns
 * SC_ERR_UNSUPPORTED otherwise (or with SC_FORCE_SIMT / SC_LINEAR_TC=0 set),
 * and the caller runs the layer as a 1x1x1 sc_subm_conv_forward over the
 * identity map. */
int sc_linear_forward(sc_dtype dtype, const void* d_x, int64_t rows, int64_t in_features, const void* d_weight,
                      int64_t out_features, const float* d_bias, const void* d_residual, int32_t silu,
                      void* d_out, void* stream);

/* ---- subdivision head (decoder upsample without a guide) -----------------
 * logits[n, 8] = feats[n, C] @ weight[8, C]^T + bias (the to_subdiv linear
 * layer; weight in feats' dtype, bias fp32, fp32 accumulate), optionally
 * centred on each row's mean, and mask[n, 8] = logits > threshold[c], where
 * threshold[c] = h_child_thresholds[c] when finite, else `threshold`
 * (h_child_thresholds may be NULL).  Replaces burn_trellis
 * sparse_decoder_runtime_impl.rs:852-890 (to_subdiv + centring) and the
 * threshold of subdivision_active_indices_wgpu_async,
 * sparse_decoder_wgpu_ops.rs:928-992 / :1813-1822.  d_logits may be NULL.
 * The mask feeds sc_subdivide. */
int sc_subdiv_head(sc_dtype dtype, const void* d_feats, int64_t n, int64_t channels, const void* d_weight,
                   const float* d_bias, float threshold, const float* h_child_thresholds, int center,
                   float* d_logits, uint8_t* d_mask, void* stream);

/* ---- sparse 3-D patchify (patch embedding at listed patches) --------------
 * out[r, :] = bias + W · patch(r) with patch(r) the input block
 * [c, t0 + dt, y0 + py, x0 + px] (t0 = tubelet * tubelet_size, y0 = patch_row *
 * patch_h, x0 = patch_col * patch_w) flattened in (c, dt, py, px) order, for
 * coords[r] = (batch, tubelet, patch_row, patch_col).  Input [B, Cin, T, H, W],
 * weight [Cout, Cin, tubelet, patch_h, patch_w] and output share `dtype`; bias
 * fp32.  Replaces burn_flex_gmm sparse_patchify3d_forward_flex (lib.rs:133-240,
 * validation :558-696).  The gather writes an im2col block into d_scratch
 * (sc_patchify3d_scratch_bytes) and the projection runs on the conv path (a
 * 1x1x1 conv over the identity rows).  Coordinates outside the grid raise the
 * device fault word and give bias-only rows. */
typedef struct sc_patchify3d_config {
    int64_t in_channels, out_channels, frames, height, width, tubelet_size, patch_h, patch_w;
} sc_patchify3d_config;
int sc_patchify3d_scratch_bytes(const sc_patchify3d_config* cfg, int64_t rows, sc_dtype dtype, size_t* h_bytes);
int sc_patchify3d_forward(const sc_patchify3d_config* cfg, sc_dtype dtype, const void* d_input,
                          int64_t input_elems, const int32_t* d_coords, int64_t rows, const void* d_weight,
                          const float* d_bias, void* d_scratch, size_t scratch_bytes, void* d_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARSECONV_H */
