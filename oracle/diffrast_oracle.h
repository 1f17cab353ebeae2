/*
 * diffrast_oracle.h — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement (C++17, std::thread) of the arithmetic of mlx-swift-diffrast's
 * Metal kernels, used only as the parity checker by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg.  Nothing in the
 * shipped library links or calls it.
 *
 * Every entry point mirrors the corresponding dr_* call of include/diffrast.h
 * but takes HOST pointers and a thread count.  Semantics follow the reference
 * kernels line by line (file:line cited at each function in the .cpp), with
 * three documented definitions where the reference is order-dependent:
 *   - tile binning never drops a triangle (the reference caps at 128/tile);
 *   - depth ties resolve to the lowest triangle index (the reference's
 *     unbinned iteration order);
 *   - atomic accumulations are summed in float64 per thread and reduced in a
 *     fixed order (deterministic).
 * Triangles with non-finite screen coordinates or out-of-range vertex indices
 * are treated as invalid (area = 0), as the CUDA path does.
 */
#ifndef DIFFRAST_ORACLE_H
#define DIFFRAST_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int orc_rasterize_fwd(const float* pos, int V, const int32_t* tri, int T,
                      const int32_t* ranges, int N, int H, int W,
                      const float* peel_layer, float* rast, float* rast_db,
                      int nthreads);
int orc_rasterize_bwd(const float* pos, int V, const int32_t* tri, int T,
                      const int32_t* ranges, int N, int H, int W,
                      const float* rast, const float* d_rast,
                      const float* d_rast_db, float* d_pos, int nthreads);

int orc_interpolate_fwd(const float* attr, int attr_batch, int V, int A,
                        const float* rast, int N, int H, int W,
                        const int32_t* tri, int T, const float* rast_db,
                        const int32_t* diff_idx, int K, float* out,
                        float* out_da, int nthreads);
int orc_interpolate_bwd(const float* attr, int attr_batch, int V, int A,
                        const float* rast, int N, int H, int W,
                        const int32_t* tri, int T, const float* rast_db,
                        const int32_t* diff_idx, int K, const float* d_out,
                        const float* d_out_da, float* d_attr, float* d_rast,
                        float* d_rast_db, int nthreads);

int orc_texture_mip_layout(int Nt, int Ht, int Wt, int C, int max_level,
                           int* num_levels, int64_t* level_offset,
                           int* level_h, int* level_w, int64_t* total);
int orc_texture_construct_mip(const float* tex, int Nt, int Ht, int Wt, int C,
                              int max_level, float* pyramid, int nthreads);
int orc_texture_fwd(int filter, int boundary, const float* tex, int Nt,
                    int Ht, int Wt, int C, int max_level, const float* uv,
                    const float* uv_da, float bias, const float* bias_map,
                    int N, int Hi, int Wi, float* out, int nthreads);
int orc_texture_bwd(int filter, int boundary, const float* tex, int Nt,
                    int Ht, int Wt, int C, int max_level, const float* uv,
                    const float* uv_da, float bias, const float* bias_map,
                    int N, int Hi, int Wi, const float* d_out, float* d_tex,
                    float* d_uv, float* d_uv_da, float* d_bias_map,
                    int nthreads);

int orc_topology_hash(const int32_t* tri, int T, int32_t* topo);
int orc_antialias_fwd(const float* color, int N, int H, int W, int C,
                      const float* rast, const float* pos, int V,
                      const int32_t* tri, int T, const int32_t* topo,
                      float* out, int nthreads);
int orc_antialias_bwd(const float* color, int N, int H, int W, int C,
                      const float* rast, const float* pos, int V,
                      const int32_t* tri, int T, const int32_t* topo,
                      const float* d_out, float* d_color, float* d_pos,
                      int nthreads);

double orc_mse_fwd_bwd(const float* pred, const float* target, int64_t n,
                       float scale, float* d_pred, int nthreads);

#ifdef __cplusplus
}
#endif

#endif
