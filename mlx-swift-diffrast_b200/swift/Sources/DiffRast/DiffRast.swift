// DiffRast.swift — the `DiffRast.*` operator surface of mlx-swift-diffrast
// (Sources/MLXDiffRast/*.swift) over the C ABI of libdiffrast (include/diffrast.h).
//
// SOURCE ONLY: this wrapper has not been compiled or run (it was written on a
// machine without a Swift toolchain).  It is a mechanical 1:1 mapping onto the
// C entry points: each forward returns its outputs, each `...VJP` function is
// the explicit backward the reference obtained from MLX's CustomFunction.
// Tensors are `DeviceTensor`s (a CUDA device pointer + shape) instead of
// MLXArray; a caller that keeps MLX on the host side copies in and out.

import CDiffRast
import Foundation

public struct DeviceTensor {
    public let pointer: UnsafeMutableRawPointer
    public let shape: [Int]
    public init(pointer: UnsafeMutableRawPointer, shape: [Int]) {
        self.pointer = pointer
        self.shape = shape
    }
    public var count: Int { shape.reduce(1, *) }
    var f: UnsafeMutablePointer<Float> { pointer.assumingMemoryBound(to: Float.self) }
    var i: UnsafeMutablePointer<Int32> { pointer.assumingMemoryBound(to: Int32.self) }
}

/// Allocator the wrapper uses for outputs (e.g. cudaMalloc via the caller's runtime).
public protocol DeviceAllocator {
    func allocate(bytes: Int) -> UnsafeMutableRawPointer
}

public enum DiffRast {
    public enum BoundaryMode: Int32 { case wrap = 0, clamp = 1, zero = 2, cube = 3 }
    public enum FilterMode: Int32 { case nearest = 0, linear = 1, linearMipmapNearest = 2, linearMipmapLinear = 3 }
    public enum DiffAttrs: Equatable { case all; case indices([Int32]) }

    /// One context per device/thread, as the C ABI requires.
    public final class Context {
        let raw: OpaquePointer
        public init(device: Int32 = 0) {
            precondition(dr_abi_version() == DR_ABI_VERSION, "libdiffrast ABI \(dr_abi_version()) != header \(DR_ABI_VERSION)")
            var p: OpaquePointer? = nil
            let st = dr_ctx_create(device, &p)
            precondition(st == DR_OK, "dr_ctx_create failed (\(st))")
            raw = p!
        }
        deinit { dr_ctx_destroy(raw) }
        public func setStream(_ s: UnsafeMutableRawPointer?) { _ = dr_ctx_set_stream(raw, s) }
        /// Fixed tile-list capacity (0 = exact sizing with one readback per
        /// rasterize): with a capacity a whole step can be captured in a CUDA graph.
        public func setRasterListCapacity(_ pairs: Int64) {
            check(dr_ctx_set_raster_list_capacity(raw, pairs), "setRasterListCapacity")
        }
        /// Tiles that scanned every triangle since the last call (synchronizes).
        public func rasterOverflow() -> Int64 {
            var n: Int64 = 0
            check(dr_ctx_raster_overflow(raw, &n), "rasterOverflow")
            return n
        }
        /// Interpolate (forward and VJP) walks [N, H, W] batches tile by tile in
        /// `order` (from `DiffRast.tileOrder`); nil restores image order.  The
        /// buffer must stay valid and unchanged while it is set.
        public func setTileOrder(_ order: DeviceTensor?, n: Int = 0, h: Int = 0, w: Int = 0) {
            check(dr_ctx_set_tile_order(raw, order?.i, Int32(n), Int32(h), Int32(w)), "setTileOrder")
        }
        /// Synchronizes the stream; crashes (as the reference's preconditions)
        /// if a kernel met an out-of-range index since the last sync.
        public func sync() { check(dr_ctx_sync(raw), "sync") }
        public var launchCount: UInt64 { dr_ctx_launch_count(raw) }
        public var workspaceBytes: Int { Int(dr_ctx_workspace_bytes(raw)) }
        func check(_ st: dr_status, _ what: String) {
            // The reference crashes on misuse with `precondition`; keep that.
            precondition(st == DR_OK, "\(what): \(String(cString: dr_last_error(raw)))")
        }
    }

    // MARK: rasterize (Rasterize.swift:44-144)

    public static func rasterize(_ ctx: Context, _ alloc: DeviceAllocator, _ pos: DeviceTensor,
                                 tri: DeviceTensor, resolution: (height: Int, width: Int),
                                 gradDB: Bool = true, ranges: DeviceTensor? = nil,
                                 peelLayer: DeviceTensor? = nil) -> (rast: DeviceTensor, rastDB: DeviceTensor) {
        let (N, V) = ranges != nil ? (ranges!.shape[0], pos.shape[0]) : (pos.shape[0], pos.shape[1])
        let H = resolution.height, W = resolution.width
        let rast = DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4])
        let db = DeviceTensor(pointer: alloc.allocate(bytes: gradDB ? N * H * W * 16 : 16),
                              shape: gradDB ? [N, H, W, 4] : [N, H, W, 0])
        ctx.check(dr_rasterize_fwd(ctx.raw, pos.f, Int32(V), tri.i, Int32(tri.shape[0]), ranges?.i,
                                   Int32(N), Int32(H), Int32(W), peelLayer?.f, rast.f, gradDB ? db.f : nil),
                  "rasterize")
        return (rast, db)
    }

    public static func rasterizeVJP(_ ctx: Context, _ alloc: DeviceAllocator, _ pos: DeviceTensor,
                                    tri: DeviceTensor, ranges: DeviceTensor?, rast: DeviceTensor,
                                    dRast: DeviceTensor, dRastDB: DeviceTensor?) -> DeviceTensor {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let V = ranges != nil ? pos.shape[0] : pos.shape[1]
        let dPos = DeviceTensor(pointer: alloc.allocate(bytes: pos.count * 4), shape: pos.shape)
        ctx.check(dr_rasterize_bwd(ctx.raw, pos.f, Int32(V), tri.i, Int32(tri.shape[0]), ranges?.i, Int32(N),
                                   Int32(H), Int32(W), rast.f, dRast.f, dRastDB?.f, dPos.f), "rasterize VJP")
        return dPos
    }

    // MARK: interpolate (Interpolate.swift:43-132)

    static func resolve(_ d: DiffAttrs?, _ A: Int) -> ([Int32]?, Int) {
        guard let d = d else { return (nil, 0) }
        switch d {
        case .all: return (nil, A)
        case .indices(let idx):
            precondition(!idx.isEmpty, "interpolate: diffAttrs.indices must be non-empty")
            return (idx, idx.count)
        }
    }

    /// Processing order of rast's 32 x 8 tiles grouped by the world region each
    /// shows (positions `pos` [V, 4] in one frame shared by all views), for
    /// `Context.setTileOrder`: Int32 [dr_tile_count(N, H, W)].
    public static func tileOrder(_ ctx: Context, _ alloc: DeviceAllocator, rast: DeviceTensor, pos: DeviceTensor,
                                 tri: DeviceTensor) -> DeviceTensor {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let n = Int(dr_tile_count(Int32(N), Int32(H), Int32(W)))
        let order = DeviceTensor(pointer: alloc.allocate(bytes: max(16, n * 4)), shape: [n])
        ctx.check(dr_tile_order(ctx.raw, rast.f, Int32(N), Int32(H), Int32(W), tri.i, Int32(tri.shape[0]), pos.f,
                                Int32(pos.shape[0]), order.i), "tileOrder")
        return order
    }

    public static func interpolate(_ ctx: Context, _ alloc: DeviceAllocator, _ attr: DeviceTensor,
                                   rast: DeviceTensor, tri: DeviceTensor, rastDB: DeviceTensor? = nil,
                                   diffAttrs: DiffAttrs? = nil) -> (out: DeviceTensor, outDA: DeviceTensor) {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0]
        let V = attr.shape[attr.shape.count - 2], A = attr.shape[attr.shape.count - 1]
        let (idx, K) = resolve(diffAttrs, A)
        let out = DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * A * 4), shape: [N, H, W, A])
        let oda = DeviceTensor(pointer: alloc.allocate(bytes: max(16, N * H * W * 2 * K * 4)), shape: [N, H, W, 2 * K])
        let st: dr_status = (idx ?? []).withUnsafeBufferPointer { ib in
            dr_interpolate_fwd(ctx.raw, attr.f, Int32(Na), Int32(V), Int32(A), rast.f, Int32(N), Int32(H),
                               Int32(W), tri.i, Int32(tri.shape[0]), rastDB?.f, idx == nil ? nil : ib.baseAddress,
                               Int32(K), out.f, K > 0 ? oda.f : nil)
        }
        ctx.check(st, "interpolate")
        return (out, oda)
    }

    public static func interpolateVJP(_ ctx: Context, _ alloc: DeviceAllocator, _ attr: DeviceTensor,
                                      rast: DeviceTensor, tri: DeviceTensor, rastDB: DeviceTensor?,
                                      diffAttrs: DiffAttrs?, dOut: DeviceTensor, dOutDA: DeviceTensor?)
        -> (dAttr: DeviceTensor, dRast: DeviceTensor, dRastDB: DeviceTensor?) {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0]
        let V = attr.shape[attr.shape.count - 2], A = attr.shape[attr.shape.count - 1]
        let (idx, K) = resolve(diffAttrs, A)
        let dAttr = DeviceTensor(pointer: alloc.allocate(bytes: attr.count * 4), shape: attr.shape)
        let dRast = DeviceTensor(pointer: alloc.allocate(bytes: rast.count * 4), shape: rast.shape)
        let dDB = K > 0 ? DeviceTensor(pointer: alloc.allocate(bytes: rast.count * 4), shape: rast.shape) : nil
        let st: dr_status = (idx ?? []).withUnsafeBufferPointer { ib in
            dr_interpolate_bwd(ctx.raw, attr.f, Int32(Na), Int32(V), Int32(A), rast.f, Int32(N), Int32(H),
                               Int32(W), tri.i, Int32(tri.shape[0]), rastDB?.f, idx == nil ? nil : ib.baseAddress,
                               Int32(K), dOut.f, dOutDA?.f, dAttr.f, dRast.f, dDB?.f)
        }
        ctx.check(st, "interpolate VJP")
        return (dAttr, dRast, dDB)
    }

    // MARK: texture (Texture.swift:62-161)

    public static func texture(_ ctx: Context, _ alloc: DeviceAllocator, _ tex: DeviceTensor, uv: DeviceTensor,
                               uvDA: DeviceTensor? = nil, filterMode: FilterMode = .linear,
                               boundaryMode: BoundaryMode = .wrap, mipLevelBias: Float = 0,
                               mipLevelBiasMap: DeviceTensor? = nil) -> DeviceTensor {
        let cube = boundaryMode == .cube
        let Nt = tex.shape[0], Ht = tex.shape[cube ? 2 : 1], Wt = tex.shape[cube ? 3 : 2]
        let C = tex.shape[cube ? 4 : 3]
        let N = uv.shape[0], Hi = uv.shape[1], Wi = uv.shape[2]
        let out = DeviceTensor(pointer: alloc.allocate(bytes: N * Hi * Wi * C * 4), shape: [N, Hi, Wi, C])
        ctx.check(dr_texture_fwd(ctx.raw, filterMode.rawValue, boundaryMode.rawValue, tex.f, Int32(Nt), Int32(Ht),
                                 Int32(Wt), Int32(C), nil, -1, uv.f, uvDA?.f, mipLevelBias, mipLevelBiasMap?.f,
                                 Int32(N), Int32(Hi), Int32(Wi), out.f), "texture")
        return out
    }

    /// DiffRast.textureConstructMip (Texture.swift:144-161): level 0 is `tex`
    /// itself; levels 1... are views into one pyramid buffer built on the GPU.
    public static func textureConstructMip(_ ctx: Context, _ alloc: DeviceAllocator, _ tex: DeviceTensor,
                                           maxLevel: Int? = nil) -> [DeviceTensor] {
        let Nt = tex.shape[0], Ht = tex.shape[1], Wt = tex.shape[2], C = tex.shape[3]
        let ml = Int32(maxLevel ?? -1)
        var n: Int32 = 0, total: Int64 = 0
        var off = [Int64](repeating: 0, count: Int(DR_MAX_MIP_LEVELS))
        var hh = [Int32](repeating: 0, count: Int(DR_MAX_MIP_LEVELS))
        var ww = [Int32](repeating: 0, count: Int(DR_MAX_MIP_LEVELS))
        ctx.check(dr_texture_mip_layout(Int32(Nt), Int32(Ht), Int32(Wt), Int32(C), ml, &n, &off, &hh, &ww, &total),
                  "textureConstructMip")
        var levels = [tex]
        if n <= 1 { return levels }
        let pyr = alloc.allocate(bytes: Int(total) * 4)
        ctx.check(dr_texture_construct_mip(ctx.raw, tex.f, Int32(Nt), Int32(Ht), Int32(Wt), Int32(C), ml,
                                           pyr.assumingMemoryBound(to: Float.self)), "textureConstructMip")
        for k in 1..<Int(n) {
            levels.append(DeviceTensor(pointer: pyr + Int(off[k]) * 4, shape: [Nt, Int(hh[k]), Int(ww[k]), C]))
        }
        return levels
    }

    /// `cubeDirGrad` (extension, cube textures only): the direction receives the
    /// chain rule through the face projection instead of the reference's zero.
    public static func textureVJP(_ ctx: Context, _ alloc: DeviceAllocator, _ tex: DeviceTensor, uv: DeviceTensor,
                                  uvDA: DeviceTensor?, filterMode: FilterMode, boundaryMode: BoundaryMode,
                                  mipLevelBias: Float, mipLevelBiasMap: DeviceTensor?, dOut: DeviceTensor,
                                  cubeDirGrad: Bool = false)
        -> (dTex: DeviceTensor, dUV: DeviceTensor, dUVDA: DeviceTensor?) {
        let cube = boundaryMode == .cube
        let Nt = tex.shape[0], Ht = tex.shape[cube ? 2 : 1], Wt = tex.shape[cube ? 3 : 2]
        let C = tex.shape[cube ? 4 : 3]
        let N = uv.shape[0], Hi = uv.shape[1], Wi = uv.shape[2]
        let dTex = DeviceTensor(pointer: alloc.allocate(bytes: tex.count * 4), shape: tex.shape)
        let dUV = DeviceTensor(pointer: alloc.allocate(bytes: uv.count * 4), shape: uv.shape)
        let mip = filterMode == .linearMipmapLinear || filterMode == .linearMipmapNearest
        // uvDA is [N, Hi, Wi, 4]; a mip-mapped cube's direction derivatives are [N, Hi, Wi, 6].
        let nDA = cube ? 6 : 4
        let dDA = mip ? DeviceTensor(pointer: alloc.allocate(bytes: N * Hi * Wi * nDA * 4), shape: [N, Hi, Wi, nDA])
                      : nil
        let bnd = boundaryMode.rawValue | (cube && cubeDirGrad ? Int32(DR_TEXTURE_CUBE_DIR_GRAD) : 0)
        ctx.check(dr_texture_bwd(ctx.raw, filterMode.rawValue, bnd, tex.f, Int32(Nt), Int32(Ht),
                                 Int32(Wt), Int32(C), nil, -1, uv.f, uvDA?.f, mipLevelBias, mipLevelBiasMap?.f,
                                 Int32(N), Int32(Hi), Int32(Wi), dOut.f, dTex.f, dUV.f, dDA?.f, nil),
                  "texture VJP")
        return (dTex, dUV, dDA)
    }

    // MARK: antialias (Antialias.swift:19-131)

    public static func antialiasConstructTopologyHash(_ ctx: Context, _ alloc: DeviceAllocator,
                                                      _ tri: DeviceTensor) -> DeviceTensor {
        let topo = DeviceTensor(pointer: alloc.allocate(bytes: tri.count * 4), shape: tri.shape)
        ctx.check(dr_antialias_construct_topology_hash(ctx.raw, tri.i, Int32(tri.shape[0]), topo.i),
                  "antialiasConstructTopologyHash")
        return topo
    }

    /// Bytes of the optional per-pixel silhouette record (`antialiasWork`)
    /// for N views of H x W pixels.
    public static func antialiasWorkBytes(views: Int, height: Int, width: Int) -> Int {
        Int(dr_antialias_work_bytes(Int32(views), Int32(height), Int32(width)))
    }

    /// DiffRast.antialias (Antialias.swift:90-131).  With `work` (a buffer of
    /// `antialiasWorkBytes` bytes) the forward also records each pixel's
    /// silhouettes, which `antialiasVJP` then replays instead of searching
    /// again; in an MLX CustomFunction it is a hidden second output of Forward.
    public static func antialias(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor, rast: DeviceTensor,
                                 pos: DeviceTensor, tri: DeviceTensor, topologyHash: DeviceTensor? = nil,
                                 work: UnsafeMutableRawPointer? = nil) -> DeviceTensor {
        let topo = topologyHash ?? antialiasConstructTopologyHash(ctx, alloc, tri)
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let out = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        ctx.check(dr_antialias_fwd(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, pos.f,
                                   Int32(pos.shape[1]), tri.i, Int32(tri.shape[0]), topo.i, out.f, work),
                  "antialias")
        return out
    }

    public static func antialiasVJP(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor, rast: DeviceTensor,
                                    pos: DeviceTensor, tri: DeviceTensor, topologyHash: DeviceTensor,
                                    dOut: DeviceTensor,
                                    work: UnsafeRawPointer? = nil) -> (dColor: DeviceTensor, dPos: DeviceTensor) {
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let dColor = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        let dPos = DeviceTensor(pointer: alloc.allocate(bytes: pos.count * 4), shape: pos.shape)
        ctx.check(dr_antialias_bwd(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, pos.f,
                                   Int32(pos.shape[1]), tri.i, Int32(tri.shape[0]), topologyHash.i, dOut.f,
                                   dColor.f, dPos.f, work), "antialias VJP")
        return (dColor, dPos)
    }

    // MARK: extensions (no counterpart in the reference's surface)

    /// Depth peeling of `numLayers` layers in one call, identical to chained
    /// rasterize(peelLayer:) calls; setup and tile binning run once.
    public static func rasterizeLayers(_ ctx: Context, _ alloc: DeviceAllocator, _ pos: DeviceTensor,
                                       tri: DeviceTensor, resolution: (height: Int, width: Int), numLayers: Int,
                                       gradDB: Bool = true, ranges: DeviceTensor? = nil)
        -> [(rast: DeviceTensor, rastDB: DeviceTensor?)] {
        let (N, V) = ranges != nil ? (ranges!.shape[0], pos.shape[0]) : (pos.shape[0], pos.shape[1])
        let H = resolution.height, W = resolution.width
        let layers: [(rast: DeviceTensor, rastDB: DeviceTensor?)] = (0..<numLayers).map { _ in
            (DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]),
             gradDB ? DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]) : nil)
        }
        let r: [UnsafeMutablePointer<Float>?] = layers.map { $0.rast.f }
        let d: [UnsafeMutablePointer<Float>?] = layers.map { $0.rastDB?.f }
        let st: dr_status = r.withUnsafeBufferPointer { rb in
            d.withUnsafeBufferPointer { db in
                dr_rasterize_layers_fwd(ctx.raw, pos.f, Int32(V), tri.i, Int32(tri.shape[0]), ranges?.i, Int32(N),
                                        Int32(H), Int32(W), Int32(numLayers), rb.baseAddress,
                                        gradDB ? db.baseAddress : nil)
            }
        }
        ctx.check(st, "rasterizeLayers")
        return layers
    }

    /// VJP of rasterizeLayers: d_pos summed over the layers (a layer without
    /// a cotangent contributes nothing).
    public static func rasterizeLayersVJP(_ ctx: Context, _ alloc: DeviceAllocator, _ pos: DeviceTensor,
                                          tri: DeviceTensor, ranges: DeviceTensor?, rast: [DeviceTensor],
                                          dRast: [DeviceTensor?], dRastDB: [DeviceTensor?]) -> DeviceTensor {
        let N = rast[0].shape[0], H = rast[0].shape[1], W = rast[0].shape[2]
        let V = ranges != nil ? pos.shape[0] : pos.shape[1]
        let dPos = DeviceTensor(pointer: alloc.allocate(bytes: pos.count * 4), shape: pos.shape)
        let r: [UnsafePointer<Float>?] = rast.map { UnsafePointer($0.f) }
        let g: [UnsafePointer<Float>?] = dRast.map { $0.map { UnsafePointer($0.f) } }
        let gd: [UnsafePointer<Float>?] = dRastDB.map { $0.map { UnsafePointer($0.f) } }
        let st: dr_status = r.withUnsafeBufferPointer { rb in
            g.withUnsafeBufferPointer { gb in
                gd.withUnsafeBufferPointer { gdb in
                    dr_rasterize_layers_bwd(ctx.raw, pos.f, Int32(V), tri.i, Int32(tri.shape[0]), ranges?.i,
                                            Int32(N), Int32(H), Int32(W), Int32(rast.count), rb.baseAddress,
                                            gb.baseAddress, gdb.baseAddress, dPos.f)
                }
            }
        }
        ctx.check(st, "rasterizeLayers VJP")
        return dPos
    }

    /// Layers of the views M_n · verts (xform [N, 4, 4] row-major, verts
    /// [V, 4]) without materialising the [N, V, 4] clip positions.
    public static func rasterizeXF(_ ctx: Context, _ alloc: DeviceAllocator, verts: DeviceTensor,
                                   xform: DeviceTensor, tri: DeviceTensor, resolution: (height: Int, width: Int),
                                   numLayers: Int = 1, gradDB: Bool = true)
        -> [(rast: DeviceTensor, rastDB: DeviceTensor?)] {
        let N = xform.shape[0], V = verts.shape[0], H = resolution.height, W = resolution.width
        let layers: [(rast: DeviceTensor, rastDB: DeviceTensor?)] = (0..<numLayers).map { _ in
            (DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]),
             gradDB ? DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]) : nil)
        }
        let r: [UnsafeMutablePointer<Float>?] = layers.map { $0.rast.f }
        let d: [UnsafeMutablePointer<Float>?] = layers.map { $0.rastDB?.f }
        let st: dr_status = r.withUnsafeBufferPointer { rb in
            d.withUnsafeBufferPointer { db in
                dr_rasterize_xf_fwd(ctx.raw, verts.f, Int32(V), xform.f, tri.i, Int32(tri.shape[0]), Int32(N),
                                    Int32(H), Int32(W), Int32(numLayers), rb.baseAddress,
                                    gradDB ? db.baseAddress : nil)
            }
        }
        ctx.check(st, "rasterizeXF")
        return layers
    }

    /// Two layers of rasterizeXF with interpolate (.all) fused into the pass:
    /// per layer rast, rastDB, out [N, H, W, A], outDA [N, H, W, 2A] and, with a
    /// target, its MSE loss (a device scalar).  Its VJP is rasterizeInterpolateXFVJP when
    /// only out reaches the loss; otherwise interpolateVJP /
    /// interpolateMSEVJP per layer, then rasterizeXFVJP.
    public static func rasterizeInterpolateXF(_ ctx: Context, _ alloc: DeviceAllocator, verts: DeviceTensor,
                                              xform: DeviceTensor, tri: DeviceTensor,
                                              resolution: (height: Int, width: Int), attr: DeviceTensor,
                                              targets: [DeviceTensor?] = [nil, nil])
        -> [(rast: DeviceTensor, rastDB: DeviceTensor, out: DeviceTensor, outDA: DeviceTensor,
             loss: DeviceTensor?)] {
        let N = xform.shape[0], V = verts.shape[0], H = resolution.height, W = resolution.width
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0], A = attr.shape[attr.shape.count - 1]
        let layers = (0..<2).map { l in
            (rast: DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]),
             rastDB: DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 16), shape: [N, H, W, 4]),
             out: DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * A * 4), shape: [N, H, W, A]),
             outDA: DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * 2 * A * 4), shape: [N, H, W, 2 * A]),
             loss: targets[l] == nil ? nil : DeviceTensor(pointer: alloc.allocate(bytes: 16), shape: []))
        }
        let r: [UnsafeMutablePointer<Float>?] = layers.map { $0.rast.f }
        let d: [UnsafeMutablePointer<Float>?] = layers.map { $0.rastDB.f }
        let o: [UnsafeMutablePointer<Float>?] = layers.map { $0.out.f }
        let od: [UnsafeMutablePointer<Float>?] = layers.map { $0.outDA.f }
        let t: [UnsafePointer<Float>?] = targets.map { $0.map { UnsafePointer($0.f) } }
        let lo: [UnsafeMutablePointer<Float>?] = layers.map { $0.loss?.f }
        let anyTarget = targets.contains { $0 != nil }
        let st: dr_status = r.withUnsafeBufferPointer { rb in d.withUnsafeBufferPointer { db in
            o.withUnsafeBufferPointer { ob in od.withUnsafeBufferPointer { odb in
                t.withUnsafeBufferPointer { tb in lo.withUnsafeBufferPointer { lb in
                    dr_rasterize_xf_interp_fwd(ctx.raw, verts.f, Int32(V), xform.f, tri.i, Int32(tri.shape[0]),
                                               Int32(N), Int32(H), Int32(W), attr.f, Int32(Na), Int32(A),
                                               rb.baseAddress, db.baseAddress, ob.baseAddress, odb.baseAddress,
                                               anyTarget ? tb.baseAddress : nil, 1.0 / Float(N * H * W * A),
                                               anyTarget ? lb.baseAddress : nil)
                } }
            } }
        } }
        ctx.check(st, "rasterizeInterpolateXF")
        return layers
    }

    /// VJP of rasterizeInterpolateXF when only out reaches the loss: both
    /// layers' interpolate and rasterize VJPs in one pass.  Per layer, out's
    /// cotangent is dOut[l], or the fused loss's (targets[l] with the loss's
    /// cotangent dLoss[l], a device scalar), or none.  Returns (d_attr, d_verts).
    public static func rasterizeInterpolateXFVJP(_ ctx: Context, _ alloc: DeviceAllocator, verts: DeviceTensor,
                                                 xform: DeviceTensor, tri: DeviceTensor, attr: DeviceTensor,
                                                 rast: [DeviceTensor], out: [DeviceTensor],
                                                 dOut: [DeviceTensor?] = [nil, nil],
                                                 targets: [DeviceTensor?] = [nil, nil],
                                                 dLoss: [DeviceTensor?] = [nil, nil])
        -> (dAttr: DeviceTensor, dVerts: DeviceTensor) {
        let N = xform.shape[0], V = verts.shape[0], H = rast[0].shape[1], W = rast[0].shape[2]
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0], A = attr.shape[attr.shape.count - 1]
        let dAttr = DeviceTensor(pointer: alloc.allocate(bytes: attr.count * 4), shape: attr.shape)
        let dVerts = DeviceTensor(pointer: alloc.allocate(bytes: verts.count * 4), shape: verts.shape)
        let r: [UnsafePointer<Float>?] = rast.map { UnsafePointer($0.f) }
        let g: [UnsafePointer<Float>?] = dOut.map { $0.map { UnsafePointer($0.f) } }
        let mse = (0..<2).map { targets[$0] != nil && dLoss[$0] != nil }
        let o: [UnsafePointer<Float>?] = (0..<2).map { mse[$0] ? UnsafePointer(out[$0].f) : nil }
        let t: [UnsafePointer<Float>?] = (0..<2).map { mse[$0] ? UnsafePointer(targets[$0]!.f) : nil }
        let dl: [UnsafePointer<Float>?] = (0..<2).map { mse[$0] ? UnsafePointer(dLoss[$0]!.f) : nil }
        let st: dr_status = r.withUnsafeBufferPointer { rb in g.withUnsafeBufferPointer { gb in
            o.withUnsafeBufferPointer { ob in t.withUnsafeBufferPointer { tb in dl.withUnsafeBufferPointer { lb in
                dr_rasterize_xf_interp_bwd(ctx.raw, verts.f, Int32(V), xform.f, tri.i, Int32(tri.shape[0]),
                                           Int32(N), Int32(H), Int32(W), attr.f, Int32(Na), Int32(A),
                                           rb.baseAddress, gb.baseAddress, ob.baseAddress, tb.baseAddress,
                                           1.0 / Float(N * H * W * A), lb.baseAddress, dAttr.f, dVerts.f)
            } } }
        } }
        ctx.check(st, "rasterizeInterpolateXF VJP")
        return (dAttr, dVerts)
    }

    /// VJP of rasterizeXF: d_verts [V, 4], summed over views (M_n^T applied).
    public static func rasterizeXFVJP(_ ctx: Context, _ alloc: DeviceAllocator, verts: DeviceTensor,
                                      xform: DeviceTensor, tri: DeviceTensor, rast: [DeviceTensor],
                                      dRast: [DeviceTensor?], dRastDB: [DeviceTensor?]) -> DeviceTensor {
        let N = xform.shape[0], V = verts.shape[0], H = rast[0].shape[1], W = rast[0].shape[2]
        let dVerts = DeviceTensor(pointer: alloc.allocate(bytes: verts.count * 4), shape: verts.shape)
        let r: [UnsafePointer<Float>?] = rast.map { UnsafePointer($0.f) }
        let g: [UnsafePointer<Float>?] = dRast.map { $0.map { UnsafePointer($0.f) } }
        let gd: [UnsafePointer<Float>?] = dRastDB.map { $0.map { UnsafePointer($0.f) } }
        let st: dr_status = r.withUnsafeBufferPointer { rb in
            g.withUnsafeBufferPointer { gb in
                gd.withUnsafeBufferPointer { gdb in
                    dr_rasterize_xf_bwd(ctx.raw, verts.f, Int32(V), xform.f, tri.i, Int32(tri.shape[0]), Int32(N),
                                        Int32(H), Int32(W), Int32(rast.count), rb.baseAddress, gb.baseAddress,
                                        gdb.baseAddress, dVerts.f)
                }
            }
        }
        ctx.check(st, "rasterizeXF VJP")
        return dVerts
    }

    /// antialias over the views M_n · verts (see rasterizeXF).
    public static func antialiasXF(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor, rast: DeviceTensor,
                                   verts: DeviceTensor, xform: DeviceTensor, tri: DeviceTensor,
                                   topologyHash: DeviceTensor, work: UnsafeMutableRawPointer? = nil) -> DeviceTensor {
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let out = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        ctx.check(dr_antialias_xf_fwd(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, verts.f,
                                      Int32(verts.shape[0]), xform.f, tri.i, Int32(tri.shape[0]), topologyHash.i,
                                      out.f, work), "antialiasXF")
        return out
    }

    public static func antialiasXFVJP(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor,
                                      rast: DeviceTensor, verts: DeviceTensor, xform: DeviceTensor,
                                      tri: DeviceTensor, topologyHash: DeviceTensor, dOut: DeviceTensor,
                                      work: UnsafeRawPointer? = nil) -> (dColor: DeviceTensor, dVerts: DeviceTensor) {
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let dColor = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        let dVerts = DeviceTensor(pointer: alloc.allocate(bytes: verts.count * 4), shape: verts.shape)
        ctx.check(dr_antialias_xf_bwd(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, verts.f,
                                      Int32(verts.shape[0]), xform.f, tri.i, Int32(tri.shape[0]), topologyHash.i,
                                      dOut.f, dColor.f, dVerts.f, work), "antialiasXF VJP")
        return (dColor, dVerts)
    }

    /// The examples' loss `((pred - target)^2).mean()` into a device scalar
    /// (a [1] tensor); with `dPred` also its gradient for a cotangent of 1.
    public static func mseLoss(_ ctx: Context, _ alloc: DeviceAllocator, pred: DeviceTensor, target: DeviceTensor,
                               dPred: DeviceTensor? = nil) -> DeviceTensor {
        let loss = DeviceTensor(pointer: alloc.allocate(bytes: 4), shape: [1])
        ctx.check(dr_mse_fwd_bwd(ctx.raw, pred.f, target.f, Int64(pred.count), 1.0 / Float(pred.count), dPred?.f,
                                 loss.f, 1), "mseLoss")
        return loss
    }

    /// antialias followed by the examples' loss `((out - target)^2).mean()`,
    /// computed in the antialias kernels: returns the loss (a device scalar)
    /// and out.  `verts` / `xform` select the per-view transform form (as
    /// antialiasXF); otherwise `pos` is [N, V, 4].
    public static func antialiasMSE(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor,
                                    rast: DeviceTensor, pos: DeviceTensor, xform: DeviceTensor? = nil,
                                    tri: DeviceTensor, topologyHash: DeviceTensor, target: DeviceTensor,
                                    work: UnsafeMutableRawPointer? = nil) -> (loss: DeviceTensor, out: DeviceTensor) {
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let out = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        let loss = DeviceTensor(pointer: alloc.allocate(bytes: 4), shape: [1])
        let scale = 1.0 / Float(color.count)
        if let xf = xform {
            ctx.check(dr_antialias_xf_fwd_mse(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f,
                                              pos.f, Int32(pos.shape[0]), xf.f, tri.i, Int32(tri.shape[0]),
                                              topologyHash.i, out.f, work, target.f, scale, loss.f),
                      "antialiasMSE")
        } else {
            ctx.check(dr_antialias_fwd_mse(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, pos.f,
                                           Int32(pos.shape[1]), tri.i, Int32(tri.shape[0]), topologyHash.i, out.f,
                                           work, target.f, scale, loss.f), "antialiasMSE")
        }
        return (loss, out)
    }

    /// VJP of antialiasMSE for the loss's cotangent dLoss (a device scalar);
    /// `out` is the forward's output.
    public static func antialiasMSEVJP(_ ctx: Context, _ alloc: DeviceAllocator, color: DeviceTensor,
                                       rast: DeviceTensor, pos: DeviceTensor, xform: DeviceTensor? = nil,
                                       tri: DeviceTensor, topologyHash: DeviceTensor, out: DeviceTensor,
                                       target: DeviceTensor, dLoss: DeviceTensor,
                                       work: UnsafeRawPointer? = nil) -> (dColor: DeviceTensor, dPos: DeviceTensor) {
        let N = color.shape[0], H = color.shape[1], W = color.shape[2], C = color.shape[3]
        let dColor = DeviceTensor(pointer: alloc.allocate(bytes: color.count * 4), shape: color.shape)
        let dPos = DeviceTensor(pointer: alloc.allocate(bytes: pos.count * 4), shape: pos.shape)
        let scale = 1.0 / Float(color.count)
        if let xf = xform {
            ctx.check(dr_antialias_xf_bwd_mse(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f,
                                              pos.f, Int32(pos.shape[0]), xf.f, tri.i, Int32(tri.shape[0]),
                                              topologyHash.i, out.f, target.f, scale, dLoss.f, dColor.f, dPos.f,
                                              work), "antialiasMSE VJP")
        } else {
            ctx.check(dr_antialias_bwd_mse(ctx.raw, color.f, Int32(N), Int32(H), Int32(W), Int32(C), rast.f, pos.f,
                                           Int32(pos.shape[1]), tri.i, Int32(tri.shape[0]), topologyHash.i, out.f,
                                           target.f, scale, dLoss.f, dColor.f, dPos.f, work), "antialiasMSE VJP")
        }
        return (dColor, dPos)
    }

    /// interpolate followed by `((out - target)^2).mean()` in the same kernel:
    /// returns the loss (a device scalar), out and outDA.
    public static func interpolateMSE(_ ctx: Context, _ alloc: DeviceAllocator, _ attr: DeviceTensor,
                                      rast: DeviceTensor, tri: DeviceTensor, target: DeviceTensor,
                                      rastDB: DeviceTensor? = nil, diffAttrs: DiffAttrs? = nil)
        -> (loss: DeviceTensor, out: DeviceTensor, outDA: DeviceTensor) {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0]
        let V = attr.shape[attr.shape.count - 2], A = attr.shape[attr.shape.count - 1]
        let (idx, K) = resolve(diffAttrs, A)
        let out = DeviceTensor(pointer: alloc.allocate(bytes: N * H * W * A * 4), shape: [N, H, W, A])
        let oda = DeviceTensor(pointer: alloc.allocate(bytes: max(16, N * H * W * 2 * K * 4)), shape: [N, H, W, 2 * K])
        let loss = DeviceTensor(pointer: alloc.allocate(bytes: 4), shape: [1])
        let st: dr_status = (idx ?? []).withUnsafeBufferPointer { ib in
            dr_interpolate_fwd_mse(ctx.raw, attr.f, Int32(Na), Int32(V), Int32(A), rast.f, Int32(N), Int32(H),
                                   Int32(W), tri.i, Int32(tri.shape[0]), rastDB?.f,
                                   idx == nil ? nil : ib.baseAddress, Int32(K), out.f, K > 0 ? oda.f : nil,
                                   target.f, 1.0 / Float(out.count), loss.f)
        }
        ctx.check(st, "interpolateMSE")
        return (loss, out, oda)
    }

    /// VJP of interpolateMSE: dLoss is the loss's cotangent (a device scalar),
    /// dOutDA outDA's (nil when it does not reach a loss).
    public static func interpolateMSEVJP(_ ctx: Context, _ alloc: DeviceAllocator, _ attr: DeviceTensor,
                                         rast: DeviceTensor, tri: DeviceTensor, rastDB: DeviceTensor?,
                                         diffAttrs: DiffAttrs?, out: DeviceTensor, target: DeviceTensor,
                                         dLoss: DeviceTensor, dOutDA: DeviceTensor?)
        -> (dAttr: DeviceTensor, dRast: DeviceTensor, dRastDB: DeviceTensor?) {
        let N = rast.shape[0], H = rast.shape[1], W = rast.shape[2]
        let Na = attr.shape.count == 2 ? 1 : attr.shape[0]
        let V = attr.shape[attr.shape.count - 2], A = attr.shape[attr.shape.count - 1]
        let (idx, K0) = resolve(diffAttrs, A)
        let K = dOutDA == nil ? 0 : K0  // outDA off the loss path: no DA terms
        let dAttr = DeviceTensor(pointer: alloc.allocate(bytes: attr.count * 4), shape: attr.shape)
        let dRast = DeviceTensor(pointer: alloc.allocate(bytes: rast.count * 4), shape: rast.shape)
        let dDB = K > 0 ? DeviceTensor(pointer: alloc.allocate(bytes: rast.count * 4), shape: rast.shape) : nil
        let st: dr_status = (K > 0 ? (idx ?? []) : []).withUnsafeBufferPointer { ib in
            dr_interpolate_bwd_mse(ctx.raw, attr.f, Int32(Na), Int32(V), Int32(A), rast.f, Int32(N), Int32(H),
                                   Int32(W), tri.i, Int32(tri.shape[0]), rastDB?.f,
                                   (K > 0 && idx != nil) ? ib.baseAddress : nil, Int32(K), out.f, target.f,
                                   1.0 / Float(out.count), dLoss.f, dOutDA?.f, dAttr.f, dRast.f, dDB?.f)
        }
        ctx.check(st, "interpolateMSE VJP")
        return (dAttr, dRast, dDB)
    }

    /// VJP of mseLoss for the cotangent dLoss (a device scalar; nil means 1).
    public static func mseVJP(_ ctx: Context, _ alloc: DeviceAllocator, pred: DeviceTensor, target: DeviceTensor,
                              dLoss: DeviceTensor? = nil) -> DeviceTensor {
        let dPred = DeviceTensor(pointer: alloc.allocate(bytes: pred.count * 4), shape: pred.shape)
        ctx.check(dr_mse_bwd(ctx.raw, pred.f, target.f, Int64(pred.count), 1.0 / Float(pred.count), dLoss?.f,
                             dPred.f), "mse VJP")
        return dPred
    }

    /// One fused Adam step in place (MLXDiffRastExamples/Adam.swift:36-43):
    /// `step` counts from 1; m and v start at zero.
    public static func adamStep(_ ctx: Context, param: DeviceTensor, grad: DeviceTensor, m: DeviceTensor,
                                v: DeviceTensor, step: Int, lr: Float, beta1: Float = 0.9, beta2: Float = 0.999,
                                eps: Float = 1e-8, mask: DeviceTensor? = nil) {
        let c1 = 1 - pow(beta1, Float(step)), c2 = 1 - pow(beta2, Float(step))
        ctx.check(dr_adam_step(ctx.raw, param.f, grad.f, mask?.f, m.f, v.f, Int64(param.count), lr, beta1, beta2,
                               eps, c1, c2), "adamStep")
    }

    /// Allocation-free topology hash (fixed table in the library, at most
    /// DR_STATIC_TOPO_MAX_TRIS triangles): writes `topo` [T, 3].
    public static func antialiasConstructTopologyHashStatic(tri: DeviceTensor, topo: DeviceTensor,
                                                            stream: UnsafeMutableRawPointer?) {
        let st = dr_antialias_construct_topology_hash_static(tri.i, Int32(tri.shape[0]), topo.i, stream)
        precondition(st == DR_OK, "antialiasConstructTopologyHashStatic failed (\(st))")
    }
}
