// ctx.cu — context lifecycle, workspace, status plumbing, the exclusive scan
// used by tile binning, and the MSE loss helper.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace dr {

dr_status fail(dr_ctx* ctx, dr_status st, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return st;
}

void timing_begin(dr_ctx* ctx) {
  if (!ctx->timing) return;
  while (ctx->ev_pool.size() < ctx->ev_next + 2) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return; }
    ctx->ev_pool.push_back(e);
  }
  cudaEventRecord(ctx->ev_pool[ctx->ev_next], ctx->stream);
  ctx->pending_start = (long)ctx->ev_next;
  ctx->ev_next += 2;
}

dr_status after_launch(dr_ctx* ctx, const char* what) {
  ctx->launches++;
  if (ctx->timing && ctx->pending_start >= 0) {
    cudaEventRecord(ctx->ev_pool[ctx->pending_start + 1], ctx->stream);
    ctx->trecs.emplace_back(what, (size_t)ctx->pending_start);
    ctx->pending_start = -1;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(ctx, DR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return DR_OK;
}

dr_status enter(dr_ctx* ctx) {
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return fail(ctx, DR_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  return DR_OK;
}

void* ws_get(dr_ctx* ctx, int slot, size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (ctx->ws_bytes[slot] >= bytes) return ctx->ws[slot];
  // Grow geometrically; the old buffer may still be read by queued work.
  size_t nb = ctx->ws_bytes[slot] * 3 / 2;
  if (nb < bytes) nb = bytes;
  nb = (nb + 255) & ~(size_t)255;
  if (ctx->ws[slot]) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->ws[slot]);
    ctx->ws[slot] = nullptr;
    ctx->ws_bytes[slot] = 0;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, nb);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(ctx, DR_ENOMEM, "workspace slot %d: cudaMalloc(%zu) failed: %s", slot, nb,
         cudaGetErrorString(e));
    return nullptr;
  }
  ctx->ws[slot] = p;
  ctx->ws_bytes[slot] = nb;
  return p;
}

// ---------------------------------------------------------------------------
// Exclusive scan over uint32 (tile candidate counts).  Three phases: per-block
// scan + block totals, a single-block scan of the totals, add block bases.

constexpr int SCAN_BLOCK = 1024;
constexpr int SCAN_ITEMS = 4;  // per thread
constexpr int SCAN_TILE = SCAN_BLOCK * SCAN_ITEMS;

__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* total) {
  __shared__ uint32_t warp_sums[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    uint32_t s = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_sums[lane] = s;
  }
  __syncthreads();
  uint32_t base = wid > 0 ? warp_sums[wid - 1] : 0u;
  if (total) *total = warp_sums[(blockDim.x >> 5) - 1];
  return base + x - v;
}

__global__ void k_scan_blocks(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                              uint32_t* __restrict__ block_sums, int64_t n) {
  int64_t base = (int64_t)blockIdx.x * SCAN_TILE + (int64_t)threadIdx.x * SCAN_ITEMS;
  uint32_t v[SCAN_ITEMS];
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    v[i] = (base + i < n) ? in[base + i] : 0u;
    s += v[i];
  }
  uint32_t tot;
  uint32_t ex = block_excl_scan(s, &tot);
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    if (base + i < n) out[base + i] = ex;
    ex += v[i];
  }
  if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

// Single block: exclusive scan of nb block totals in place; total -> *total.
__global__ void k_scan_sums(uint32_t* __restrict__ sums, int nb, uint32_t* __restrict__ total) {
  __shared__ uint32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int b0 = 0; b0 < nb; b0 += SCAN_BLOCK) {
    int i = b0 + threadIdx.x;
    uint32_t v = i < nb ? sums[i] : 0u;
    uint32_t tot;
    uint32_t ex = block_excl_scan(v, &tot);
    uint32_t c = carry;
    if (i < nb) sums[i] = c + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry = c + tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void k_scan_add(uint32_t* __restrict__ out, const uint32_t* __restrict__ sums, int64_t n) {
  int64_t base = (int64_t)blockIdx.x * SCAN_TILE;
  uint32_t add = sums[blockIdx.x];
  for (int i = threadIdx.x; i < SCAN_TILE; i += SCAN_BLOCK)
    if (base + i < n) out[base + i] += add;
}

dr_status scan_u32(dr_ctx* ctx, const uint32_t* in, uint32_t* out, int64_t n, uint32_t* total_dev) {
  int nb = (int)((n + SCAN_TILE - 1) / SCAN_TILE);
  if (nb < 1) nb = 1;
  uint32_t* sums = (uint32_t*)ws_get(ctx, WS_SCAN_TMP, sizeof(uint32_t) * (size_t)nb);
  if (!sums) return DR_ENOMEM;
  DR_TB(ctx);
  k_scan_blocks<<<nb, SCAN_BLOCK, 0, ctx->stream>>>(in, out, sums, n);
  DR_LAUNCHED(ctx, "scan_blocks");
  DR_TB(ctx);
  k_scan_sums<<<1, SCAN_BLOCK, 0, ctx->stream>>>(sums, nb, total_dev);
  DR_LAUNCHED(ctx, "scan_sums");
  if (nb > 1) {
    DR_TB(ctx);
    k_scan_add<<<nb, SCAN_BLOCK, 0, ctx->stream>>>(out, sums, n);
    DR_LAUNCHED(ctx, "scan_add");
  }
  return DR_OK;
}

// ---------------------------------------------------------------------------
// MSE: loss += scale * sum((p - t)^2) (when loss is given) and
// d = (2 * scale * (p - t)) * g (when d is given; g = *d_loss, or 1).
template <bool LOSS, bool GRAD>
__global__ void k_mse(const float* __restrict__ p, const float* __restrict__ t, int64_t n,
                      float scale, const float* __restrict__ d_loss, float* __restrict__ d,
                      float* __restrict__ loss) {
  float acc = 0.0f;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t n4 = n / 4;
  const float s2 = 2.0f * scale;
  const float g = (GRAD && d_loss) ? __ldg(d_loss) : 1.0f;
  const bool vec = ((((uintptr_t)p) | ((uintptr_t)t) | ((uintptr_t)d)) & 15) == 0;
  int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t i = i0; i < n4; i += stride) {
      float4 a = ldg4(p + 4 * i), b = ldg4(t + 4 * i);
      float4 r;
      r.x = a.x - b.x; r.y = a.y - b.y; r.z = a.z - b.z; r.w = a.w - b.w;
      if (LOSS) acc += r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
      if (GRAD)
        reinterpret_cast<float4*>(d)[i] = make_float4((s2 * r.x) * g, (s2 * r.y) * g, (s2 * r.z) * g, (s2 * r.w) * g);
    }
    for (int64_t i = 4 * n4 + i0; i < n; i += stride) {
      float r = p[i] - t[i];
      if (LOSS) acc += r * r;
      if (GRAD) d[i] = (s2 * r) * g;
    }
  } else {
    for (int64_t i = i0; i < n; i += stride) {
      float r = p[i] - t[i];
      if (LOSS) acc += r * r;
      if (GRAD) d[i] = (s2 * r) * g;
    }
  }
  if constexpr (LOSS) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ float ws[32];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (threadIdx.x == 0) atomicAdd(loss, v * scale);
    }
  }
}

// loss = the kLossSlots partial sums of a fused loss (one warp, a shuffle
// reduction).
__global__ void k_loss_finish(const float* __restrict__ part, float* __restrict__ loss) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < kLossSlots; i += 32) s += part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x == 0) *loss = s;
}

PixOrder pix_order(const dr_ctx* ctx, int N, int H, int W, unsigned& grid) {
  PixOrder o;
  if (ctx->tile_order && ctx->order_n == N && ctx->order_h == H && ctx->order_w == W) {
    o.order = ctx->tile_order;
    o.H = H;
    o.W = W;
    o.ntx = (W + kOrderTileW - 1) / kOrderTileW;
    o.ntiles = o.ntx * ((H + kOrderTileH - 1) / kOrderTileH);
    o.n_tiles = (int64_t)N * o.ntiles;
    grid = (unsigned)o.n_tiles;
  } else {
    grid = grid_for((int64_t)N * H * W, 256);
  }
  return o;
}

dr_status loss_begin(dr_ctx* ctx, float** part) {
  float* p = (float*)ws_get(ctx, WS_LOSS, sizeof(float) * kLossSlots);
  if (!p) return DR_ENOMEM;
  DR_CUDA(ctx, cudaMemsetAsync(p, 0, sizeof(float) * kLossSlots, ctx->stream), "loss memset");
  *part = p;
  return DR_OK;
}

dr_status loss_end(dr_ctx* ctx, const float* part, float* loss) {
  DR_TB(ctx);
  k_loss_finish<<<1, 32, 0, ctx->stream>>>(part, loss);
  DR_LAUNCHED(ctx, "loss_finish");
  return DR_OK;
}

}  // namespace dr

using namespace dr;

extern "C" {

int dr_abi_version(void) { return DR_ABI_VERSION; }

dr_status dr_ctx_create(int device, dr_ctx** out) {
  if (!out) return DR_EINVAL;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return DR_ECUDA;
  }
  dr_ctx* c = new dr_ctx();
  c->device = device;
  if (cudaSetDevice(device) != cudaSuccess) { delete c; return DR_ECUDA; }
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (cudaMalloc(&c->d_err, sizeof(unsigned)) != cudaSuccess) { delete c; return DR_ENOMEM; }
  cudaMemset(c->d_err, 0, sizeof(unsigned));
  if (cudaMalloc(&c->d_overflow, sizeof(unsigned)) != cudaSuccess) {
    cudaFree(c->d_err);
    delete c;
    return DR_ENOMEM;
  }
  cudaMemset(c->d_overflow, 0, sizeof(unsigned));
  if (cudaMallocHost(&c->h_pinned, 64) != cudaSuccess) {
    cudaFree(c->d_err);
    cudaFree(c->d_overflow);
    delete c;
    return DR_ENOMEM;
  }
  cudaDeviceSynchronize();
  *out = c;
  return DR_OK;
}

void dr_ctx_destroy(dr_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (cudaEvent_t e : ctx->ev_pool) cudaEventDestroy(e);
  for (int i = 0; i < WS_NUM_SLOTS; ++i)
    if (ctx->ws[i]) cudaFree(ctx->ws[i]);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->d_overflow) cudaFree(ctx->d_overflow);
  if (ctx->h_pinned) cudaFreeHost(ctx->h_pinned);
  delete ctx;
}

dr_status dr_ctx_set_raster_list_capacity(dr_ctx* ctx, int64_t pairs) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, pairs >= 0 && pairs < (int64_t)UINT32_MAX, "raster list capacity %lld out of range",
             (long long)pairs);
  if (pairs > 0 && !ws_get(ctx, WS_TILE_LIST, sizeof(int32_t) * (size_t)(pairs + 1))) return DR_ENOMEM;
  ctx->list_cap = pairs;
  return DR_OK;
}

dr_status dr_ctx_raster_overflow(dr_ctx* ctx, int64_t* tiles) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, tiles != nullptr, "raster_overflow: tiles is required");
  cudaError_t e = cudaMemcpyAsync(ctx->h_pinned, ctx->d_overflow, sizeof(unsigned), cudaMemcpyDeviceToHost,
                                  ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_overflow, 0, sizeof(unsigned), ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return fail(ctx, DR_ECUDA, "raster_overflow: %s", cudaGetErrorString(e));
  *tiles = (int64_t)(unsigned)ctx->h_pinned[0];
  return DR_OK;
}

dr_status dr_ctx_set_stream(dr_ctx* ctx, void* stream) {
  if (!ctx) return DR_EINVAL;
  ctx->stream = (cudaStream_t)stream;
  return DR_OK;
}

void* dr_ctx_get_stream(const dr_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

const char* dr_last_error(const dr_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

dr_status dr_ctx_sync(dr_ctx* ctx) {
  DR_ENTER(ctx);
  cudaError_t e = cudaMemcpyAsync(ctx->h_pinned, ctx->d_err, sizeof(unsigned),
                                  cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return fail(ctx, DR_ECUDA, "sync: %s", cudaGetErrorString(e));
  unsigned bits = (unsigned)ctx->h_pinned[0];
  if (bits) {
    cudaMemsetAsync(ctx->d_err, 0, sizeof(unsigned), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    return fail(ctx, DR_EDEVICE, "device-side input error bits 0x%x (%s%s%s)", bits,
                (bits & DR_DEVERR_VERTEX) ? "vertex index out of range; " : "",
                (bits & DR_DEVERR_TRI_ID) ? "rast tri_id out of range; " : "",
                (bits & DR_DEVERR_CAPACITY) ? "capacity exceeded; " : "");
  }
  return DR_OK;
}

uint64_t dr_ctx_launch_count(const dr_ctx* ctx) { return ctx ? ctx->launches : 0; }

dr_status dr_ctx_set_timing(dr_ctx* ctx, int enable) {
  if (!ctx) return DR_EINVAL;
  ctx->timing = enable != 0;
  ctx->ev_next = 0;
  ctx->pending_start = -1;
  ctx->trecs.clear();
  return DR_OK;
}

dr_status dr_ctx_timing_report(dr_ctx* ctx, char* buf, size_t n) {
  DR_ENTER(ctx);
  if (!buf || n == 0) return fail(ctx, DR_EINVAL, "timing_report: no buffer");
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return fail(ctx, DR_ECUDA, "timing_report: %s", cudaGetErrorString(e));
  std::vector<std::pair<std::string, std::pair<long, double>>> agg;
  for (auto& r : ctx->trecs) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, ctx->ev_pool[r.second], ctx->ev_pool[r.second + 1]) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    size_t i = 0;
    while (i < agg.size() && agg[i].first != r.first) ++i;
    if (i == agg.size()) agg.push_back({r.first, {0, 0.0}});
    agg[i].second.first += 1;
    agg[i].second.second += ms;
  }
  size_t off = 0;
  buf[0] = 0;
  for (auto& a : agg) {
    int w = snprintf(buf + off, n - off, "%s %ld %.6f\n", a.first.c_str(), a.second.first, a.second.second);
    if (w < 0 || (size_t)w >= n - off) return fail(ctx, DR_EOVERFLOW, "timing_report: buffer too small");
    off += (size_t)w;
  }
  return DR_OK;
}

size_t dr_ctx_workspace_bytes(const dr_ctx* ctx) {
  if (!ctx) return 0;
  size_t s = 0;
  for (int i = 0; i < WS_NUM_SLOTS; ++i) s += ctx->ws_bytes[i];
  return s;
}

dr_status dr_mse_fwd_bwd(dr_ctx* ctx, const float* pred, const float* target, int64_t n,
                         float scale, float* d_pred, float* loss, int zero_loss) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, n >= 0 && pred && target && loss, "mse: null pointer or n < 0");
  if (zero_loss) DR_CUDA(ctx, cudaMemsetAsync(loss, 0, sizeof(float), ctx->stream), "mse memset");
  if (n == 0) return DR_OK;
  int blocks = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)ctx->num_sms * 8);
  DR_TB(ctx);
  if (d_pred)
    k_mse<true, true><<<blocks, 256, 0, ctx->stream>>>(pred, target, n, scale, nullptr, d_pred, loss);
  else
    k_mse<true, false><<<blocks, 256, 0, ctx->stream>>>(pred, target, n, scale, nullptr, nullptr, loss);
  DR_LAUNCHED(ctx, "mse");
  return DR_OK;
}

dr_status dr_mse_bwd(dr_ctx* ctx, const float* pred, const float* target, int64_t n, float scale,
                     const float* d_loss, float* d_pred) {
  DR_ENTER(ctx);
  DR_REQUIRE(ctx, n >= 0 && pred && target && d_pred, "mse_bwd: null pointer or n < 0");
  if (n == 0) return DR_OK;
  int blocks = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)ctx->num_sms * 8);
  DR_TB(ctx);
  k_mse<false, true><<<blocks, 256, 0, ctx->stream>>>(pred, target, n, scale, d_loss, d_pred, nullptr);
  DR_LAUNCHED(ctx, "mse_bwd");
  return DR_OK;
}

}  // extern "C"
