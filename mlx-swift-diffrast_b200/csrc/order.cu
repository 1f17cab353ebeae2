// order.cu — an L2-friendly processing order for the per-pixel kernels of a
// multi-view batch (interpolate's forward and VJP), and the context setting
// that makes them use it.  No counterpart in the reference: its kernels run
// one thread per pixel in image order.
//
// Interpolate gathers three attribute rows per pixel from a table indexed by
// vertex, and its VJP adds into a gradient table of the same shape.  Every
// view of a batch shows about the same triangles, so in image order each view
// sweeps the whole of both tables; when they do not fit L2 together (cfg4:
// 84 + 84 MB against 126 MB) every view misses on them again.  Here the
// batch's 32 x 8 pixel tiles are ordered by the world region they show: a few
// coarse regions, every view's tiles of one region before the next region,
// the views in order inside a region (a stable partition of the tiles by
// region).  One region's slice of the tables then stays in L2 while all the
// views pass over it, with about one view's tiles in flight at a time: more
// views over the same rows at once would serialise the VJP's atomics on them,
// which is why the regions are few and the views not interleaved.
//
// A tile's region comes from the position of the triangle it shows (layer
// rast, at the tile's centre or the centres of its quadrants) in one fixed
// frame: vertex 0's (x/w, y/w), binned on a G x G grid over the bounding box
// of all tiles' points.  Tiles that show no triangle go last.  The order
// changes no per-pixel result; gradients summed with atomics change only in
// their summation order, as between any two runs.
#include "common.cuh"

using dr::grid_for;

namespace {

constexpr int kTW = dr::kOrderTileW, kTH = dr::kOrderTileH;  // one 256-thread block of the per-pixel kernels
constexpr int kMaxGrid = 4;              // regions per axis at most
constexpr int kBins = kMaxGrid * kMaxGrid + 1;  // + the tiles that show no triangle
constexpr int kBlock = 256;

struct TileGeo {
  int N, H, W, ntx, ntiles;  // ntiles: tiles per view
};

// Order-preserving uint32 image of a float (larger float, larger image).
__device__ __forceinline__ unsigned ord(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord(unsigned u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// The world point of tile `tile`: vertex 0 of the first triangle found at the
// tile's centre or its quadrants' centres, as (x/w, y/w); false when those
// pixels show no triangle (or its vertex is not usable).
__device__ bool tile_point(const float4* __restrict__ rast, const int32_t* __restrict__ tri, int T,
                           const float4* __restrict__ pos, int V, const TileGeo& g, int64_t tile, float& x,
                           float& y) {
  const int n = (int)(tile / g.ntiles);
  const int t = (int)(tile - (int64_t)n * g.ntiles);
  const int ty = t / g.ntx, tx = t - ty * g.ntx;
#pragma unroll 1
  for (int s = 0; s < 5; ++s) {
    const int ox = s == 0 ? kTW / 2 : ((s & 1) ? kTW / 4 : 3 * kTW / 4);
    const int oy = s == 0 ? kTH / 2 : (s < 3 ? kTH / 4 : 3 * kTH / 4);
    const int px = min(tx * kTW + ox, g.W - 1), py = min(ty * kTH + oy, g.H - 1);
    const float4 r = __ldg(rast + ((int64_t)n * g.H + py) * g.W + px);
    const int tr = (int)r.w - 1;
    if (tr < 0 || tr >= T) continue;
    const int v = __ldg(tri + 3 * (int64_t)tr);
    if (v < 0 || v >= V) continue;
    const float4 p = __ldg(pos + v);
    if (!(p.w > 0.0f)) continue;
    const float px_ = p.x / p.w, py_ = p.y / p.w;
    if (!isfinite(px_) || !isfinite(py_)) continue;
    x = px_;
    y = py_;
    return true;
  }
  return false;
}

// Bounding box of the tiles' points: box[0..3] = ~ord(xmin), ~ord(ymin),
// ord(xmax), ord(ymax), all combined with atomicMax (zero-initialised).
__global__ void __launch_bounds__(kBlock) k_tile_box(const float4* __restrict__ rast, const int32_t* __restrict__ tri,
                                                    int T, const float4* __restrict__ pos, int V, const TileGeo g,
                                                    int64_t n_tiles, unsigned* __restrict__ box) {
  const int64_t tile = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float x = 0.0f, y = 0.0f;
  const bool ok = tile < n_tiles && tile_point(rast, tri, T, pos, V, g, tile, x, y);
  unsigned b0 = ok ? ~ord(x) : 0u, b1 = ok ? ~ord(y) : 0u, b2 = ok ? ord(x) : 0u, b3 = ok ? ord(y) : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    b0 = max(b0, __shfl_xor_sync(0xffffffffu, b0, o));
    b1 = max(b1, __shfl_xor_sync(0xffffffffu, b1, o));
    b2 = max(b2, __shfl_xor_sync(0xffffffffu, b2, o));
    b3 = max(b3, __shfl_xor_sync(0xffffffffu, b3, o));
  }
  if ((threadIdx.x & 31) == 0 && b2 != 0u) {
    atomicMax(box + 0, b0);
    atomicMax(box + 1, b1);
    atomicMax(box + 2, b2);
    atomicMax(box + 3, b3);
  }
}

// The tile's bin: its region on the G x G grid over the box, or G * G when it
// shows no triangle.  -1 past the last tile.
__device__ __forceinline__ int tile_bin(const float4* __restrict__ rast, const int32_t* __restrict__ tri, int T,
                                        const float4* __restrict__ pos, int V, const TileGeo& g, int64_t tile,
                                        int64_t n_tiles, const unsigned* __restrict__ box, int G) {
  if (tile >= n_tiles) return -1;
  float x, y;
  if (box[2] == 0u || !tile_point(rast, tri, T, pos, V, g, tile, x, y)) return G * G;
  const float x0 = unord(~box[0]), y0 = unord(~box[1]), x1 = unord(box[2]), y1 = unord(box[3]);
  const float sx = x1 > x0 ? (float)G / (x1 - x0) : 0.0f, sy = y1 > y0 ? (float)G / (y1 - y0) : 0.0f;
  const int gx = min(G - 1, max(0, (int)((x - x0) * sx)));
  const int gy = min(G - 1, max(0, (int)((y - y0) * sy)));
  return gy * G + gx;
}

// Per block: how many of its tiles fall in each bin (bin-major:
// count[bin * nblocks + block]).
__global__ void __launch_bounds__(kBlock) k_tile_count(const float4* __restrict__ rast, const int32_t* __restrict__ tri,
                                                      int T, const float4* __restrict__ pos, int V, const TileGeo g,
                                                      int64_t n_tiles, const unsigned* __restrict__ box, int G,
                                                      uint32_t* __restrict__ count) {
  __shared__ unsigned s_hist[kBins];
  if (threadIdx.x < kBins) s_hist[threadIdx.x] = 0u;
  __syncthreads();
  const int64_t tile = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int bin = tile_bin(rast, tri, T, pos, V, g, tile, n_tiles, box, G);
  if (bin >= 0) atomicAdd(&s_hist[bin], 1u);
  __syncthreads();
  if (threadIdx.x < kBins) count[(int64_t)threadIdx.x * gridDim.x + blockIdx.x] = s_hist[threadIdx.x];
}

// Writes every tile at its bin's offset for this block plus its rank among
// the block's earlier tiles of the same bin: a stable partition by bin.
__global__ void __launch_bounds__(kBlock) k_tile_scatter(const float4* __restrict__ rast,
                                                        const int32_t* __restrict__ tri, int T,
                                                        const float4* __restrict__ pos, int V, const TileGeo g,
                                                        int64_t n_tiles, const unsigned* __restrict__ box, int G,
                                                        const uint32_t* __restrict__ offset,
                                                        int32_t* __restrict__ order) {
  constexpr int kWarps = kBlock / 32;
  __shared__ unsigned s_cnt[kWarps][kBins];
  for (int i = threadIdx.x; i < kWarps * kBins; i += blockDim.x) (&s_cnt[0][0])[i] = 0u;
  __syncthreads();
  const int64_t tile = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int bin = tile_bin(rast, tri, T, pos, V, g, tile, n_tiles, box, G);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned peers = __match_any_sync(0xffffffffu, bin);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (bin >= 0 && rank == 0) s_cnt[warp][bin] = __popc(peers);
  __syncthreads();
  if (bin < 0) return;
  unsigned before = 0;
  for (int w = 0; w < warp; ++w) before += s_cnt[w][bin];
  order[offset[(int64_t)bin * gridDim.x + blockIdx.x] + before + rank] = (int32_t)tile;
}

}  // namespace

using namespace dr;

extern "C" {

int64_t dr_tile_count(int N, int H, int W) {
  if (N <= 0 || H <= 0 || W <= 0) return 0;
  return (int64_t)N * ((H + kTH - 1) / kTH) * ((W + kTW - 1) / kTW);
}

dr_status dr_tile_order(dr_ctx* ctx, const float* rast, int N, int H, int W, const int32_t* tri, int T,
                        const float* pos, int V, int32_t* order) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, rast && tri && pos && order, "tile_order: rast, tri, pos and order are required");
  DR_REQUIRE(ctx, N > 0 && H > 0 && W > 0 && T > 0 && V > 0, "tile_order: bad sizes");
  DR_REQUIRE(ctx, (((uintptr_t)rast | (uintptr_t)pos) & 15u) == 0, "tile_order: rast and pos must be 16-byte aligned");
  const int64_t n_tiles = dr_tile_count(N, H, W);
  DR_REQUIRE(ctx, n_tiles <= INT32_MAX, "tile_order: %lld tiles exceed the int32 order", (long long)n_tiles);
  TileGeo g;
  g.N = N;
  g.H = H;
  g.W = W;
  g.ntx = (W + kTW - 1) / kTW;
  g.ntiles = g.ntx * ((H + kTH - 1) / kTH);
  // Regions per axis: about one region per four waves of tiles of a view
  // (a view's tiles of one region then fill the GPU by themselves).
  const int64_t waves = (int64_t)g.ntiles / ((int64_t)ctx->num_sms * 4);
  const int G = waves >= 16 ? 4 : (waves >= 4 ? 2 : 1);
  const unsigned nb = grid_for(n_tiles, kBlock);
  const size_t count_n = (size_t)kBins * nb;
  // Workspace: the box (4 words, padded to 16) and the counts / offsets.
  unsigned* box = (unsigned*)ws_get(ctx, WS_ORDER, sizeof(uint32_t) * (16 + 2 * count_n + 1));
  if (!box) return DR_ENOMEM;
  uint32_t* count = box + 16;
  uint32_t* offset = count + count_n;
  uint32_t* total = offset + count_n;
  DR_CUDA(ctx, cudaMemsetAsync(box, 0, 4 * sizeof(unsigned), ctx->stream), "tile_order memset");
  const float4* r4 = reinterpret_cast<const float4*>(rast);
  const float4* p4 = reinterpret_cast<const float4*>(pos);
  DR_TB(ctx);
  k_tile_box<<<nb, kBlock, 0, ctx->stream>>>(r4, tri, T, p4, V, g, n_tiles, box);
  DR_LAUNCHED(ctx, "tile_box");
  DR_TB(ctx);
  k_tile_count<<<nb, kBlock, 0, ctx->stream>>>(r4, tri, T, p4, V, g, n_tiles, box, G, count);
  DR_LAUNCHED(ctx, "tile_count");
  dr_status st = scan_u32(ctx, count, offset, (int64_t)count_n, total);
  if (st != DR_OK) return st;
  DR_TB(ctx);
  k_tile_scatter<<<nb, kBlock, 0, ctx->stream>>>(r4, tri, T, p4, V, g, n_tiles, box, G, offset, order);
  DR_LAUNCHED(ctx, "tile_scatter");
  return DR_OK;
}

dr_status dr_ctx_set_tile_order(dr_ctx* ctx, const int32_t* order, int N, int H, int W) {
  DR_ENTER(ctx);
  if (!order) {
    ctx->tile_order = nullptr;
    ctx->order_n = ctx->order_h = ctx->order_w = 0;
    return DR_OK;
  }
  DR_REQUIRE(ctx, N > 0 && H > 0 && W > 0, "set_tile_order: bad sizes");
  DR_REQUIRE(ctx, dr_tile_count(N, H, W) <= INT32_MAX, "set_tile_order: too many tiles");
  ctx->tile_order = order;
  ctx->order_n = N;
  ctx->order_h = H;
  ctx->order_w = W;
  return DR_OK;
}

}  // extern "C"
