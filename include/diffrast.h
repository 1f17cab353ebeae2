/*
 * diffrast.h — C ABI of the B200-native differentiable rasterization chain.
 *
 * This is the drop-in boundary under the Swift `DiffRast.*` operator surface of
 * mlx-swift-diffrast (the .swift files of Sources/MLXDiffRast).  Every forward op is paired
 * with an explicit VJP ("_bwd") entry point; the Swift wrapper (or any other
 * host language) owns autograd and calls these two halves.
 *
 * Conventions (identical to the reference):
 *   - Layouts are NHWC, fp32; indices are int32.
 *   - pos is clip space (x*w, y*w, z*w, w).
 *   - Pixel (h=0, w=0) is the top-left pixel; NDC +y is up.
 *   - rast channels are (u, v, z/w, tri_id+1) with u = w1, v = w2 (the
 *     barycentric weights of vertices 1 and 2; w0 = 1-u-v).
 *   - rast_db channels are (du/dx, du/dy, dv/dx, dv/dy) in pixel units.
 *
 * Memory: every tensor pointer is a DEVICE pointer on the context's device,
 * except `diff_idx`, which is a host array (it is a Swift [Int32] in the
 * reference).  Outputs are caller-allocated and fully overwritten; gradient
 * accumulators are zeroed by the callee.  All calls are asynchronous on the
 * context's stream and return a status; device-side index errors (a triangle
 * that names a vertex >= V, a rast tri_id > T) are skipped by the kernels and
 * reported by the next dr_ctx_sync().
 *
 * Threading: a context is not re-entrant; use one context per host thread /
 * stream.  Contexts on different devices are independent.
 */
#ifndef DIFFRAST_H
#define DIFFRAST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DR_API __attribute__((visibility("default")))
#else
#define DR_API
#endif

#define DR_ABI_VERSION 2
#define DR_MAX_MIP_LEVELS 32
#define DR_MAX_DIFF_ATTRS 1024

typedef enum dr_status {
  DR_OK = 0,
  DR_EINVAL = 1,     /* bad shape / argument (reference: `precondition` failure) */
  DR_ENOMEM = 2,     /* workspace allocation failed */
  DR_ECUDA = 3,      /* CUDA runtime error (launch or earlier asynchronous fault) */
  DR_EOVERFLOW = 4,  /* a fixed capacity was exceeded (no-drop guarantee) */
  DR_EDEVICE = 5     /* a kernel saw out-of-range indices in its inputs */
} dr_status;

/* Texture filter modes: DiffRast.FilterMode (Texture.swift:35-40). */
typedef enum dr_filter {
  DR_FILTER_NEAREST = 0,
  DR_FILTER_LINEAR = 1,
  DR_FILTER_LINEAR_MIPMAP_NEAREST = 2,
  DR_FILTER_LINEAR_MIPMAP_LINEAR = 3
} dr_filter;

/* Boundary modes: DiffRast.BoundaryMode raw values (Texture.swift:8-17). */
typedef enum dr_boundary {
  DR_BOUNDARY_WRAP = 0,
  DR_BOUNDARY_CLAMP = 1,
  DR_BOUNDARY_ZERO = 2,
  DR_BOUNDARY_CUBE = 3
} dr_boundary;

/* Flag bit OR'ed into the `boundary` argument of dr_texture_bwd (ignored by
 * dr_texture_fwd).  Extension, cube textures only: d_uv receives d(loss)/d(dir)
 * through the face projection u = (sc/ma + 1)/2, v = (tc/ma + 1)/2 — and, for
 * the mipmap filters, through the LOD — instead of the reference's zero
 * (Texture.swift:196-197). */
#define DR_TEXTURE_CUBE_DIR_GRAD 0x100

typedef struct dr_ctx dr_ctx;

/* ---- context ----------------------------------------------------------- */

DR_API int dr_abi_version(void);

/* Create a context on `device`.  It owns a grow-only device workspace
 * (setup records, tile bins, mip pyramids, hash tables) and uses the legacy
 * default stream until dr_ctx_set_stream() is called. */
DR_API dr_status dr_ctx_create(int device, dr_ctx** out);
DR_API void dr_ctx_destroy(dr_ctx* ctx);
/* `stream` is a cudaStream_t. */
DR_API dr_status dr_ctx_set_stream(dr_ctx* ctx, void* stream);
DR_API void* dr_ctx_get_stream(const dr_ctx* ctx);
/* Message describing the last non-OK status on this context. */
DR_API const char* dr_last_error(const dr_ctx* ctx);
/* Synchronize the context's stream and report DR_EDEVICE if any kernel since
 * the previous sync saw out-of-range indices (the flag is then cleared). */
DR_API dr_status dr_ctx_sync(dr_ctx* ctx);
/* Number of kernels this context has launched (for launch accounting). */
DR_API uint64_t dr_ctx_launch_count(const dr_ctx* ctx);
DR_API size_t dr_ctx_workspace_bytes(const dr_ctx* ctx);
/* Instrumentation (no counterpart in the reference, which has no tracing):
 * when enabled, every kernel launch is bracketed by CUDA events on the
 * context's stream.  Enabling (or disabling) clears the records.  The report
 * synchronizes the stream and writes one line per kernel name,
 * "<name> <launches> <total_ms>\n", into buf. */
DR_API dr_status dr_ctx_set_timing(dr_ctx* ctx, int enable);
DR_API dr_status dr_ctx_timing_report(dr_ctx* ctx, char* buf, size_t n);

/* Graph-safe binning (no counterpart in the reference, whose bins hold 128
 * entries and drop the rest).  By default every rasterize call sizes its
 * (tile, triangle) list exactly, which takes one small device-to-host read of
 * the list length — a synchronisation that a CUDA graph capture cannot hold.
 * With pairs > 0 the list buffer holds `pairs` entries (allocated here, so
 * call this before a capture) and rasterize reads nothing back: a tile whose
 * list would run past the buffer tests every triangle of its view instead —
 * the same result, slower — and is counted.  pairs = 0 restores exact sizing.
 * dr_ctx_raster_overflow synchronizes the stream and returns (and resets) the
 * number of tiles that took that path.  A captured graph holds the context's
 * workspace pointers: replay it with the shapes it was captured with, and do
 * not change the capacity (or grow a workspace with larger calls) while it
 * lives. */
DR_API dr_status dr_ctx_set_raster_list_capacity(dr_ctx* ctx, int64_t pairs);
DR_API dr_status dr_ctx_raster_overflow(dr_ctx* ctx, int64_t* tiles);

/* Tile order (no counterpart in the reference, whose kernels run one thread
 * per pixel in image order).  Every view of a multi-view batch shows about
 * the same triangles, so interpolate (which gathers attribute rows by vertex
 * and, in its VJP, adds into a gradient table of the same shape) sweeps the
 * whole table once per view; when the table and its gradient do not fit L2,
 * each view misses on them again.  dr_tile_order writes a processing order of
 * the batch's 32 x 8 pixel tiles (dr_tile_count(N, H, W) int32 entries, a
 * permutation of 0 .. count-1, tile = view * tiles per view + tile row *
 * tiles per row + tile column) grouped by the world region each tile shows:
 * a few coarse regions, the views in order inside each, tiles that show
 * nothing last.  The region comes from the triangle the layer `rast`
 * ([N, H, W, 4]) shows at the tile's centre, through vertex 0 of tri ([T, 3])
 * in `pos` ([V, 4], one fixed frame for all views: the shared vertices of the
 * per-view transform mode, or one view's clip-space positions; x/w and y/w
 * are used).  dr_ctx_set_tile_order makes the interpolate forward and VJP
 * entry points (the _mse ones included) process batches of exactly
 * N x H x W pixels tile by tile in `order` (a permutation from dr_tile_order,
 * which must stay valid and unchanged while it is set); order = NULL restores
 * image order.  Outputs are the same in either order; gradients summed with
 * atomics differ only in their summation order, as between any two runs. */
DR_API int64_t dr_tile_count(int N, int H, int W);
DR_API dr_status dr_tile_order(dr_ctx* ctx, const float* rast, int N, int H, int W,
                               const int32_t* tri, int T, const float* pos, int V,
                               int32_t* order);
DR_API dr_status dr_ctx_set_tile_order(dr_ctx* ctx, const int32_t* order, int N, int H,
                                       int W);

/* ---- rasterize (Rasterize.swift:44-144) -------------------------------- */

/* Forward.  Replaces DiffRast.rasterize (Rasterize.swift:44) and its kernels
 * diffrast_rasterize_precompute/_bin/_fwd/_fwd_db (Rasterize.swift:280-609).
 *   Instanced mode: ranges == NULL, pos is [N, V, 4].
 *   Range mode:     ranges is [N, 2] int32 (start, count), pos is [V, 4].
 *   peel_layer: NULL, or a previous rast [N, H, W, 4] to peel through.
 *   rast: [N, H, W, 4] out.  rast_db: [N, H, W, 4] out, or NULL (gradDB=false).
 * Unlike the reference (MAX_PER_TILE=128, overflow dropped) no triangle is ever
 * dropped, and depth ties resolve to the lowest triangle index.
 * Limits: T < 2^24 (tri_id + 1 is stored as a float), H, W <= 32768, and the
 * (16x16 tile, triangle) pairs of one call (summed over its views) below 2^32
 * (the tile lists are offset by a 32-bit prefix sum). */
DR_API dr_status dr_rasterize_fwd(dr_ctx* ctx, const float* pos, int V,
                           const int32_t* tri, int T, const int32_t* ranges,
                           int N, int H, int W, const float* peel_layer,
                           float* rast, float* rast_db);

/* VJP.  Replaces the rasterize VJP closures (Rasterize.swift:109-117,
 * 129-138) and diffrast_rasterize_bwd (Rasterize.swift:637-812).
 *   d_rast: [N, H, W, 4] (channel 3 ignored); d_rast_db: [N, H, W, 4] or NULL.
 *   d_pos: out, [N, V, 4] instanced or [V, 4] in range mode (summed over the
 *   batch, as MLX's broadcast-backward does). */
DR_API dr_status dr_rasterize_bwd(dr_ctx* ctx, const float* pos, int V,
                           const int32_t* tri, int T, const int32_t* ranges,
                           int N, int H, int W, const float* rast,
                           const float* d_rast, const float* d_rast_db,
                           float* d_pos);

/* Depth peeling of num_layers layers in one call: layer 0 is the front-most
 * surface, layer l peels layer l-1 exactly as chained rasterize(peelLayer:)
 * calls do (Rasterize.swift:36-42, 384-392), and the results are identical to
 * those calls.  Setup and tile binning run once for all layers.
 *   rast[l]: [N, H, W, 4] out; rast_db: NULL or an array whose entries are
 *   [N, H, W, 4] outputs or NULL.  The arrays are host arrays of device pointers. */
DR_API dr_status dr_rasterize_layers_fwd(dr_ctx* ctx, const float* pos, int V,
                                  const int32_t* tri, int T, const int32_t* ranges,
                                  int N, int H, int W, int num_layers,
                                  float* const* rast, float* const* rast_db);

/* VJP of dr_rasterize_layers_fwd: d_pos = sum over layers of the per-layer
 * rasterize VJP (a layer with d_rast[l] == NULL contributes nothing). */
DR_API dr_status dr_rasterize_layers_bwd(dr_ctx* ctx, const float* pos, int V,
                                  const int32_t* tri, int T, const int32_t* ranges,
                                  int N, int H, int W, int num_layers,
                                  const float* const* rast,
                                  const float* const* d_rast,
                                  const float* const* d_rast_db, float* d_pos);

/* Per-view vertex transform ("xf") mode — no counterpart in the reference,
 * which takes pre-transformed clip positions.  The clip position of vertex v
 * in view n is M_n · verts[v] with xform = M [N, 4, 4] row-major, evaluated as
 *   clip_r = ((M[r][0]·x + M[r][1]·y) + M[r][2]·z) + M[r][3]·w
 * (each product and sum rounded separately), i.e. instanced mode with
 * pos = einsum('nij,vj->nvi', M, verts) but without materialising [N, V, 4].
 * Layers as in dr_rasterize_layers_fwd.  The VJP writes d_verts [V, 4], the
 * gradient of the shared vertices summed over views (M_n^T applied). */
DR_API dr_status dr_rasterize_xf_fwd(dr_ctx* ctx, const float* verts, int V,
                              const float* xform, const int32_t* tri, int T,
                              int N, int H, int W, int num_layers,
                              float* const* rast, float* const* rast_db);
DR_API dr_status dr_rasterize_xf_bwd(dr_ctx* ctx, const float* verts, int V,
                              const float* xform, const int32_t* tri, int T,
                              int N, int H, int W, int num_layers,
                              const float* const* rast, const float* const* d_rast,
                              const float* const* d_rast_db, float* d_verts);
/* Two depth layers of the xf mode with interpolate fused into the pass (no
 * counterpart in the reference, where rasterize and interpolate are separate
 * operators): writes, per layer l of 2, rast[l] and rast_db[l] exactly as
 * dr_rasterize_xf_fwd(num_layers = 2) and out[l] [N, H, W, A] / out_da[l]
 * [N, H, W, 2A] exactly as dr_interpolate_fwd(attr, rast[l], ..., rast_db[l],
 * diff_idx = NULL, K = A), computed from each pixel's winner instead of by a
 * second pass that reads rast back.  attr [attr_batch, V, A] shares verts'
 * V, with A a multiple of 4 and attr / out / out_da 16-byte aligned.  With
 * target[l] (and loss[l], both or neither; target may be NULL for no loss at
 * all) the layer also writes scale * sum((out[l] - target[l])^2) to the
 * device scalar *loss[l], as dr_interpolate_fwd_mse.  Its VJP is
 * dr_rasterize_xf_interp_bwd when only out reaches the loss (directly or
 * through the fused loss); otherwise the separate ones,
 * dr_interpolate_bwd(_mse) per layer and then dr_rasterize_xf_bwd. */
DR_API dr_status dr_rasterize_xf_interp_fwd(dr_ctx* ctx, const float* verts, int V,
                                     const float* xform, const int32_t* tri, int T,
                                     int N, int H, int W, const float* attr,
                                     int attr_batch, int A, float* const* rast,
                                     float* const* rast_db, float* const* out,
                                     float* const* out_da, const float* const* target,
                                     float scale, float* const* loss);
/* VJP of dr_rasterize_xf_interp_fwd when out_da, rast and rast_db take no
 * cotangent (no counterpart in the reference): the interpolate VJP and the
 * rasterize VJP of both layers in one pass, with each pixel's rast cotangent
 * (d_u, d_v, 0) handed from the one to the other in registers.  The same
 * values as dr_interpolate_bwd(_mse) per layer (diff_idx = NULL, K = 0)
 * followed by dr_rasterize_xf_bwd, up to the order of the atomic sums.
 * Per layer l of 2, out's cotangent is d_out[l] [N, H, W, A], or the fused
 * loss's, 2 * scale * (out[l] - target[l]) * (*d_loss[l]) (out, target and
 * d_loss together; not with d_out), or none (the layer adds nothing); any of
 * the pointer arrays may be NULL.  Writes d_attr [attr_batch, V, A] and
 * d_verts [V, 4] (both zeroed first).  rast, cotangent rows, attr, d_attr,
 * verts, xform and d_verts 16-byte aligned; A a multiple of 4. */
DR_API dr_status dr_rasterize_xf_interp_bwd(dr_ctx* ctx, const float* verts, int V,
                                     const float* xform, const int32_t* tri, int T,
                                     int N, int H, int W, const float* attr,
                                     int attr_batch, int A, const float* const* rast,
                                     const float* const* d_out, const float* const* out,
                                     const float* const* target, float scale,
                                     const float* const* d_loss, float* d_attr,
                                     float* d_verts);

/* ---- interpolate (Interpolate.swift:43-132) ---------------------------- */

/* Forward.  Replaces DiffRast.interpolate and diffrast_interp_fwd/_fwd_da
 * (Interpolate.swift:137-228).
 *   attr: [attr_batch, V, A] with attr_batch == 1 (broadcast; also the
 *         reference's [V, A] range-mode form) or attr_batch == N.
 *   rast: [N, H, W, 4]; tri: [T, 3].
 *   K == 0: no pixel derivatives (diffAttrs == nil); rast_db/out_da ignored.
 *   K  > 0: rast_db [N, H, W, 4]; diff_idx = HOST array of K attribute
 *           indices (.indices), or NULL with K == A (.all);
 *           out_da: [N, H, W, 2K].
 *   out: [N, H, W, A]. */
DR_API dr_status dr_interpolate_fwd(dr_ctx* ctx, const float* attr, int attr_batch,
                             int V, int A, const float* rast, int N, int H,
                             int W, const int32_t* tri, int T,
                             const float* rast_db, const int32_t* diff_idx,
                             int K, float* out, float* out_da);

/* VJP.  Replaces diffrast_interp_grad_attr/_grad_attr_da/_grad_rast/
 * _grad_rast_db (Interpolate.swift:231-417, 502-541).
 *   d_attr: out, [attr_batch, V, A] (summed over the batch when attr_batch==1).
 *   d_rast: out, [N, H, W, 4] (channels 2, 3 are zero).
 *   d_rast_db: out, [N, H, W, 4] when K > 0, else ignored. */
DR_API dr_status dr_interpolate_bwd(dr_ctx* ctx, const float* attr, int attr_batch,
                             int V, int A, const float* rast, int N, int H,
                             int W, const int32_t* tri, int T,
                             const float* rast_db, const int32_t* diff_idx,
                             int K, const float* d_out, const float* d_out_da,
                             float* d_attr, float* d_rast, float* d_rast_db);

/* Interpolate followed by a mean-squared-error loss of `out` against `target`
 * ([N, H, W, A]) in the same pass: the loss the reference's examples compute
 * after the op (`mean((out - target)^2)`, ColorFitExample/main.swift:57-60,
 * PoseFitExample/main.swift:89-92), fused here; no counterpart in the
 * reference's operator surface.  The forward writes out / out_da as
 * dr_interpolate_fwd and writes scale * sum((out - target)^2) to the device
 * scalar *loss (scale = 1 / numel for a mean).  The
 * VJP takes out (the forward's output), target, scale and d_loss (a device
 * scalar, the loss's cotangent) in place of d_out and forms out's cotangent
 * 2 * scale * (out - target) * (*d_loss) where it reads it; d_out_da is
 * out_da's cotangent as in dr_interpolate_bwd. */
DR_API dr_status dr_interpolate_fwd_mse(dr_ctx* ctx, const float* attr, int attr_batch,
                                 int V, int A, const float* rast, int N, int H,
                                 int W, const int32_t* tri, int T,
                                 const float* rast_db, const int32_t* diff_idx,
                                 int K, float* out, float* out_da,
                                 const float* target, float scale, float* loss);
DR_API dr_status dr_interpolate_bwd_mse(dr_ctx* ctx, const float* attr, int attr_batch,
                                 int V, int A, const float* rast, int N, int H,
                                 int W, const int32_t* tri, int T,
                                 const float* rast_db, const int32_t* diff_idx,
                                 int K, const float* out, const float* target,
                                 float scale, const float* d_loss,
                                 const float* d_out_da, float* d_attr,
                                 float* d_rast, float* d_rast_db);

/* ---- texture (Texture.swift:62-1313) ----------------------------------- */

/* Host-only: the mip pyramid layout textureConstructMip (Texture.swift:144-161)
 * produces for a [Nt, Ht, Wt, C] texture.  Level 0 is the texture itself; the
 * pyramid buffer holds levels 1..num_levels-1 back to back, level k as
 * [Nt, level_h[k], level_w[k], C] starting at float offset level_offset[k]
 * (level_offset[0] = -1).  max_level < 0 means "no limit". */
DR_API dr_status dr_texture_mip_layout(int Nt, int Ht, int Wt, int C, int max_level,
                                int* num_levels, int64_t* level_offset,
                                int* level_h, int* level_w,
                                int64_t* pyramid_floats);

/* textureConstructMip (Texture.swift:144-161): 2x2 box-filter levels 1.. into
 * `pyramid` (size from dr_texture_mip_layout). */
DR_API dr_status dr_texture_construct_mip(dr_ctx* ctx, const float* tex, int Nt,
                                   int Ht, int Wt, int C, int max_level,
                                   float* pyramid);

/* Forward.  Replaces DiffRast.texture (Texture.swift:62-131) and kernels
 * diffrast_texture_fwd / _nearest_fwd / _cube_fwd / _trilinear_fwd.
 *   tex: [Nt, Ht, Wt, C] (Nt == 1 broadcasts) or, for DR_BOUNDARY_CUBE,
 *        [Nt, 6, Ht, Wt, C].  Cube takes DR_FILTER_LINEAR as the reference;
 *        the two mipmap filters on a cube are an extension (the reference
 *        rejects them): the pyramid is that of the Nt * 6 faces, the LOD
 *        comes from the derivatives of the face coordinates.
 *   pyramid: mip levels >= 1 from dr_texture_construct_mip (for a cube, of
 *        the [Nt * 6, Ht, Wt, C] faces), or NULL to build them internally
 *        (mipmap filters only).  max_level as in the layout.
 *   uv: [N, Hi, Wi, 2] ([N, Hi, Wi, 3] direction for cube).
 *   uv_da: [N, Hi, Wi, 4], required for the mipmap filters; for a cube the
 *        direction's derivatives [N, Hi, Wi, 6] = (dx/dX, dx/dY, dy/dX,
 *        dy/dY, dz/dX, dz/dY), interpolate's diff_attrs layout, 8-byte
 *        aligned.
 *   mip_level_bias / mip_level_bias_map ([N, Hi, Wi] or NULL): scale uv_da by
 *        2^bias * 2^map before the LOD, as Texture.swift:104-126.
 *   out: [N, Hi, Wi, C]. */
DR_API dr_status dr_texture_fwd(dr_ctx* ctx, int filter, int boundary,
                         const float* tex, int Nt, int Ht, int Wt, int C,
                         const float* pyramid, int max_level, const float* uv,
                         const float* uv_da, float mip_level_bias,
                         const float* mip_level_bias_map, int N, int Hi,
                         int Wi, float* out);

/* VJP.  Replaces the texture VJP closures and kernels _grad_tex, _grad_uv,
 * _nearest_grad_tex, _cube_grad_tex, _trilinear_grad_pyramid/_grad_uv/
 * _grad_uvda (Texture.swift:405-521, 574-605, 686-738, 865-1102), plus the
 * MLX autograd of the pyramid build (folded into level 0 here).
 *   d_tex: out, same shape as tex (pyramid gradients folded in).
 *   d_uv: out, shape of uv (zero for nearest; zero d_dir for cube, as
 *         Texture.swift:196-197, unless boundary has DR_TEXTURE_CUBE_DIR_GRAD).
 *   d_uv_da: out, shape of uv_da, for mipmap filters, or NULL.
 *   d_bias_map: out [N, Hi, Wi] gradient of the bias map, or NULL. */
DR_API dr_status dr_texture_bwd(dr_ctx* ctx, int filter, int boundary,
                         const float* tex, int Nt, int Ht, int Wt, int C,
                         const float* pyramid, int max_level, const float* uv,
                         const float* uv_da, float mip_level_bias,
                         const float* mip_level_bias_map, int N, int Hi,
                         int Wi, const float* d_out, float* d_tex,
                         float* d_uv, float* d_uv_da, float* d_bias_map);

/* ---- antialias (Antialias.swift:19-601) -------------------------------- */

/* antialiasConstructTopologyHash (Antialias.swift:19-66), on the GPU.
 *   tri: [T, 3]; topo: out [T, 3] (neighbour tri, -1 boundary, -2 non-manifold).
 * Bit-identical to the reference's sort-based construction. */
DR_API dr_status dr_antialias_construct_topology_hash(dr_ctx* ctx,
                                               const int32_t* tri, int T,
                                               int32_t* topo);

/* Allocation-free variant of dr_antialias_construct_topology_hash — no
 * counterpart in the reference.  For callers that cannot allocate device
 * memory (their host owns the GPU's memory through its own pool, or they must
 * avoid the device-wide synchronisation of cudaMalloc): it needs no context and
 * allocates nothing, using a fixed hash table compiled into the library (about
 * 10.8 MB on every GPU that loads it, held until the process exits).
 *   tri: [T, 3] device; topo: out [T, 3] device; stream: a cudaStream_t.
 *   T must be <= DR_STATIC_TOPO_MAX_TRIS, else DR_EINVAL (nothing launched).
 * The first call on a device looks up the table's device address (with that
 * device current), so make it before any stream capture.  Every call reuses the
 * same table and clears what it uses; calls that overlap on the GPU race. */
#define DR_STATIC_TOPO_MAX_TRIS 65536
DR_API dr_status dr_antialias_construct_topology_hash_static(const int32_t* tri,
                                                             int T, int32_t* topo,
                                                             void* stream);

/* Forward.  Replaces DiffRast.antialias (Antialias.swift:90-131) and
 * diffrast_antialias_fwd (Antialias.swift:333-358).
 *   color: [N, H, W, C]; rast: [N, H, W, 4]; pos: [N, V, 4] (instanced, as the
 *   reference requires); tri: [T, 3]; topo: [T, 3]; out: [N, H, W, C].
 *   aa_work: NULL, or dr_antialias_work_bytes(N, H, W) bytes (16-byte aligned)
 *   that receive each pixel's silhouette record for the VJP.  It has no
 *   counterpart in the reference, whose VJP re-runs the silhouette search;
 *   passing it to dr_antialias_bwd gives the same gradients faster. */
DR_API dr_status dr_antialias_fwd(dr_ctx* ctx, const float* color, int N, int H,
                           int W, int C, const float* rast, const float* pos,
                           int V, const int32_t* tri, int T,
                           const int32_t* topo, float* out, void* aa_work);

/* VJP.  Replaces diffrast_antialias_bwd_color / _bwd_pos
 * (Antialias.swift:388-524).  d_color: out [N, H, W, C]; d_pos: out [N, V, 4].
 *   aa_work: NULL (the silhouettes are searched again, as the reference does)
 *   or the buffer the forward filled for this same rast / pos / tri / topo. */
DR_API dr_status dr_antialias_bwd(dr_ctx* ctx, const float* color, int N, int H,
                           int W, int C, const float* rast, const float* pos,
                           int V, const int32_t* tri, int T,
                           const int32_t* topo, const float* d_out,
                           float* d_color, float* d_pos, const void* aa_work);

/* Size of the aa_work buffer for N views of H x W pixels: 17 bytes per pixel
 * (a float4 of per-direction betas, then one byte of selected edges), rounded
 * up to 16.  No counterpart in the reference. */
DR_API size_t dr_antialias_work_bytes(int N, int H, int W);

/* Antialias with per-view transformed vertices (see dr_rasterize_xf_fwd);
 * no counterpart in the reference.  d_verts: out [V, 4].  aa_work as above. */
DR_API dr_status dr_antialias_xf_fwd(dr_ctx* ctx, const float* color, int N, int H,
                              int W, int C, const float* rast, const float* verts,
                              int V, const float* xform, const int32_t* tri, int T,
                              const int32_t* topo, float* out, void* aa_work);
DR_API dr_status dr_antialias_xf_bwd(dr_ctx* ctx, const float* color, int N, int H,
                              int W, int C, const float* rast, const float* verts,
                              int V, const float* xform, const int32_t* tri, int T,
                              const int32_t* topo, const float* d_out,
                              float* d_color, float* d_verts, const void* aa_work);

/* Antialias followed by a mean-squared-error loss of `out` against `target`
 * ([N, H, W, C]) in the same passes, as dr_interpolate_fwd_mse: the forward
 * also writes scale * sum((out - target)^2) to the device scalar *loss; the
 * VJP takes out, target, scale and d_loss in place of
 * d_out.  No counterpart in the reference's operator surface (its examples
 * compute the loss after the op, ColorFitExample/main.swift:57-60). */
DR_API dr_status dr_antialias_fwd_mse(dr_ctx* ctx, const float* color, int N, int H,
                               int W, int C, const float* rast, const float* pos,
                               int V, const int32_t* tri, int T,
                               const int32_t* topo, float* out, void* aa_work,
                               const float* target, float scale, float* loss);
DR_API dr_status dr_antialias_bwd_mse(dr_ctx* ctx, const float* color, int N, int H,
                               int W, int C, const float* rast, const float* pos,
                               int V, const int32_t* tri, int T,
                               const int32_t* topo, const float* out,
                               const float* target, float scale,
                               const float* d_loss, float* d_color, float* d_pos,
                               const void* aa_work);
DR_API dr_status dr_antialias_xf_fwd_mse(dr_ctx* ctx, const float* color, int N, int H,
                                  int W, int C, const float* rast, const float* verts,
                                  int V, const float* xform, const int32_t* tri, int T,
                                  const int32_t* topo, float* out, void* aa_work,
                                  const float* target, float scale, float* loss);
DR_API dr_status dr_antialias_xf_bwd_mse(dr_ctx* ctx, const float* color, int N, int H,
                                  int W, int C, const float* rast, const float* verts,
                                  int V, const float* xform, const int32_t* tri, int T,
                                  const int32_t* topo, const float* out,
                                  const float* target, float scale,
                                  const float* d_loss, float* d_color, float* d_verts,
                                  const void* aa_work);

/* ---- loss helper (the MSE of the reference's examples) ------------------ */

/* loss += scale * sum((pred - target)^2) into the device scalar `loss`
 * (zeroed by the callee when zero_loss != 0) and, when d_pred is not NULL,
 * d_pred = 2 * scale * (pred - target).  n elements. */
DR_API dr_status dr_mse_fwd_bwd(dr_ctx* ctx, const float* pred, const float* target,
                         int64_t n, float scale, float* d_pred, float* loss,
                         int zero_loss);

/* VJP of the loss alone: d_pred = (2 * scale * (pred - target)) * d_loss[0],
 * with the cotangent d_loss read on the device (NULL means 1). */
DR_API dr_status dr_mse_bwd(dr_ctx* ctx, const float* pred, const float* target,
                     int64_t n, float scale, const float* d_loss, float* d_pred);


/* ---- optimizer step of the reference's examples ----------------------- */

/* One Adam step in place (MLXDiffRastExamples/Adam.swift:36-43), fused:
 *   g = grad (* mask when mask != NULL); m = beta1 m + (1 - beta1) g;
 *   v = beta2 v + (1 - beta2) g^2;
 *   param -= (lr * m / bias_c1) / (sqrt(v / bias_c2) + eps)
 * with bias_c1 = 1 - beta1^t and bias_c2 = 1 - beta2^t for step t >= 1,
 * formed by the caller in float.  n elements; m and v start at zero. */
DR_API dr_status dr_adam_step(dr_ctx* ctx, float* param, const float* grad,
                       const float* mask, float* m, float* v, int64_t n,
                       float lr, float beta1, float beta2, float eps,
                       float bias_c1, float bias_c2);

#ifdef __cplusplus
}
#endif

#endif /* DIFFRAST_H */
